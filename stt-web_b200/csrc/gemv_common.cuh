// Pieces shared by the GEMV kernels of the batched step (kernels.cu, gemv_mma.cu): the output
// rows of a unit, the epilogues a product's outputs go through, and the limits of their waits and
// of one CTA's shared memory.
#pragma once

#include "device.cuh"
#include "kernels.h"
#include "qkv.cuh"

namespace stt {

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

constexpr uint32_t kSSpin = 1u << 22;         // polls of a bounded wait before it gives up
constexpr size_t kSmemLimit = 226 * 1024;     // dynamic shared memory of one CTA (227 KB on sm_100, less the static part)

template <int EPI>
__device__ __forceinline__ void unit_rows(const GemvArgs& a, int u, int* ra, int* rb) {
    if (EPI == EPI_GATE) {
        *ra = u;
        *rb = u + a.half_n;
    } else {
        *ra = 2 * u;
        *rb = 2 * u + 1 < a.W.n ? 2 * u + 1 : -1;
    }
}

// The QKV epilogue of output pair (ra, rb = ra + 1) of batch row bm (stream sid, state st, RoPE
// factors cs): RoPE on q and k, the row's q, k, v to the step's buffer and k, v to the stream's K/V
// ring.
__device__ __forceinline__ void qkv_store(const Ctx& c, const GemvArgs& a, int bm, int sid, const StreamState& st,
                                          float2 cs, int ra, int rb, float va, float vb) {
    float* o = a.out + (int64_t)bm * a.ldo;
    const int part = ra / c.D;  // 0 q, 1 k, 2 v
    if (part < 2) {
        const float r = qkv_rotate(va, vb, cs, false), im = qkv_rotate(va, vb, cs, true);
        va = r;
        vb = im;
    }
    o[ra] = va;
    o[rb] = vb;
    if (part >= 1) {
        const int64_t off = qkv_kv_offset(c, a.layer, sid, st, ra);
        if (c.kv_f32) {
            float* kv = reinterpret_cast<float*>(c.kv) + off;
            kv[0] = va;
            kv[1] = vb;
        } else {
            __nv_bfloat162* kv = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(c.kv) + off);
            *kv = __floats2bfloat162_rn(va, vb);
        }
    }
}

template <int EPI>
__device__ __forceinline__ void epilogue(const Ctx& c, const GemvArgs& a, int bm, int ra, int rb, float va, float vb) {
    if (EPI == EPI_PLAIN || EPI == EPI_LOGITS) {
        float* o = a.out + (int64_t)bm * a.ldo;
        o[ra] = va;
        if (rb >= 0) o[rb] = vb;
    } else if (EPI == EPI_RESID) {
        float* o = a.out + (int64_t)bm * a.ldo;
        o[ra] = __fadd_rn(va, o[ra]);
        if (rb >= 0) o[rb] = __fadd_rn(vb, o[rb]);
    } else if (EPI == EPI_GATE) {
        // silu(gate) * value, silu(x) = x * (1 / (1 + exp(-x)))
        const float sg = __fmul_rn(va, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-va))));
        a.out[(int64_t)bm * a.ldo + ra] = __fmul_rn(sg, vb);
    } else {  // EPI_QKV
        const int sid = c.ids[bm];
        const StreamState st = c.state[sid];
        qkv_store(c, a, bm, sid, st, qkv_rope(c, st, ra), ra, rb, va, vb);
    }
}

}  // namespace stt
