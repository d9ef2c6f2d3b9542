// The QKV epilogue's addressing and RoPE factors, shared by the GEMV's epilogue, the tensor-core
// epilogue kernel and the tensor-core GEMM's fused epilogue, so that all of them compute the same
// values (model.rs:426-449: RoPE on q and k, k and v appended to the stream's K/V ring).
#pragma once

#include "device.cuh"

namespace stt {

// RoPE factors (cos, sin) of output pair (ra, ra + 1), ra even, at the stream's position; zeros for
// the v rows, which take no rotation.
__device__ __forceinline__ float2 qkv_rope(const Ctx& c, const StreamState& st, int ra) {
    const int within = ra % c.D, d = within % c.HD;
    return ra < 2 * c.D ? c.rope[(int64_t)st.offset * (c.HD >> 1) + (d >> 1)] : make_float2(0.0f, 0.0f);
}

// RoPE::apply_rotation (model.rs:114-116) of the pair (va, vb), no fma contraction: the new first
// (odd = false) or second (odd = true) element.
__device__ __forceinline__ float qkv_rotate(float va, float vb, float2 cs, bool odd) {
    return odd ? __fadd_rn(__fmul_rn(va, cs.y), __fmul_rn(vb, cs.x))
               : __fsub_rn(__fmul_rn(va, cs.x), __fmul_rn(vb, cs.y));
}

// Element offset in the K/V rings of output row r (a k or v row: r >= D) of stream sid, at the
// stream's write position.
__device__ __forceinline__ int64_t qkv_kv_offset(const Ctx& c, int layer, int sid, const StreamState& st, int r) {
    const int part = r / c.D, within = r - part * c.D;
    const int h = within / c.HD, d = within - h * c.HD;
    return (int64_t)sid * c.kv_stream_stride + (int64_t)layer * c.kv_layer_stride +
           (part == 2 ? c.kv_half_stride : 0) + ((int64_t)h * c.ML + st.write_pos) * c.HD + d;
}

}  // namespace stt
