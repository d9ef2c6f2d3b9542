// Device-side data structures and helpers of the STT-1B decode step (sm_100a).
//
// HBM layout
//   Q4_0 matrix [n, k]  ->  nibble plane  uint4[n][k/32]   (the 16 payload bytes of each block,
//                                                            byte j = lo: elem j, hi: elem j+16)
//                           scale plane   uint16[n][k/32]  (the f16 block scales)
//     The reference keeps the 18-byte blocks back to back (gguf.rs:418-451), so every block after
//     the first is misaligned; splitting the 2-byte scale off makes every payload a 16-byte
//     aligned uint4 load and keeps the byte count identical.
//   KV ring  [stream][layer][K|V][head][slot 0..sliding_window][head_dim], bf16 or f32.
//     A head's slots are contiguous, so one (stream, head) attention split reads one range.
//   Step state per stream (StreamState) and a per-call StepDesc live in device memory, so one
//   captured CUDA graph serves every call with the same batch size.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace stt {

constexpr int kMaxLayers = 64;
constexpr int kMaxCodebooks = 64;

struct Q4Dev {
    const uint4* nib;      // [n][k/32]
    const uint16_t* scale; // [n][k/32]
    int32_t n, k;
};

struct LayerDev {
    Q4Dev qkv, out, fin, fout;  // in_proj [3D,D], out_proj [D,D], linear_in [2F,D], linear_out [D,F]
    const float* norm1;
    const float* norm2;
};

// Stream-loop state (stream.rs:20-41) plus the KVCache counters (model.rs:139-153).
struct StreamState {
    int32_t offset;      // absolute position = RoPE offset
    int32_t len;         // valid ring entries before this step
    int32_t write_pos;   // ring slot of this step's K/V
    int32_t frame_count;
    uint32_t last_text;
    uint32_t prev0, prev1;  // delay_prev
    uint32_t pad;
};

// Per-call description; kernels read it so a captured graph can be replayed for any call.
struct StepDesc {
    const uint32_t* audio;   // [steps][n][NC]
    const uint32_t* text;    // [steps][n] or NULL (use StreamState::last_text)
    int32_t* tokens;         // [steps][n] emitted tokens (-1 = None) or raw argmax
    float* logits;           // [steps][n][V] copy of the logits, or NULL
    int32_t step;            // step index inside the call, advanced by the final kernel
    int32_t mode;            // 0: raw forward (model.rs:631), 1: feed_frame (stream.rs:70)
    int32_t error;           // first error code raised by a kernel (STT_E_*), 0 if none
    int32_t pad;
};

enum EmbType : int32_t { EMB_Q4 = 2, EMB_F32 = 0, EMB_F16 = 1, EMB_BF16 = 30 };

// Everything a step kernel needs, passed by value.
struct Ctx {
    // model
    const LayerDev* layers;  // device array [L]
    Q4Dev head;
    const float* out_norm;
    const float2* rope;      // [max_seq_len][HD/2] (cos, sin)
    const uint8_t* emb_audio;  // [NC][AV][row bytes]
    const uint8_t* emb_text;   // [TV][row bytes]
    int32_t emb_type;
    int32_t emb_row_bytes;
    int32_t L, D, H, HD, F, V, TV, AV, NC, ML, max_seq_len;
    float attn_scale;
    uint32_t pad_id;
    int32_t text_delay;
    // streams
    void* kv;
    int32_t kv_f32;
    int64_t kv_stream_stride;  // elements
    int64_t kv_layer_stride;   // elements (K and V of one layer)
    int64_t kv_half_stride;    // elements (V = K + this)
    StreamState* state;
    // batch
    const int32_t* ids;        // [n] stream id of each batch row
    int32_t n;
    StepDesc* desc;
    // scratch, indexed by batch row
    float* x;       // [n][D] residual stream
    float* qkv;     // [n][3D] (q, k rotated)
    float* attn;    // [n][D]
    float* hid;     // [n][F] silu(gate) * value
    float* logits;  // [n][V]
    float* part;    // [n][H][nsplit][HD + 4] attention partials (max, sum, pad, pad, o[HD])
    uint32_t* tickets;  // [n*H] attention split counters, then one finish counter
    float* amax_val;    // [n][amax_ctas]
    int32_t* amax_idx;  // [n][amax_ctas]
    int32_t nsplit, chunk;
    // tensor-core steps: the attention kernel also writes its output as the output projection's
    // f16 input tiles (tc_layout.cuh); NULL otherwise
    __half* x16;
    int32_t x16_nt, x16_rows_pad;
};

// ---------------------------------------------------------------------------- helpers

__device__ __forceinline__ float f16_to_f32_ieee(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// gguf.rs:45-73: IEEE except that subnormals come out at half their value (exponent one low).
__device__ __forceinline__ float f16_to_f32_gguf(uint16_t b) {
    const float f = __half2float(__ushort_as_half(b));
    return ((b & 0x7C00u) == 0 && (b & 0x3FFu) != 0) ? f * 0.5f : f;
}

__device__ __forceinline__ float bf16_to_f32_dev(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// (nibble - 8) as an exact float: 2^23 + nib has the nibble in its low mantissa bits.
__device__ __forceinline__ float nib_m8(uint32_t v) {
    return __uint_as_float(0x4B000000u | v) - 8388616.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ void raise_error(StepDesc* d, int32_t code) {
    if (d) atomicCAS(&d->error, 0, code);
}

// Programmatic dependent launch.  A kernel launched with launch_pdl may start while the previous
// kernel of the stream is still running: it must call pdl_wait() before it touches anything that
// kernel writes or reads (pdl_wait returns once that kernel has completed and its writes are
// visible; it returns at once for a kernel launched the ordinary way), and every one of its CTAs
// must call it before exiting, so that completion stays ordered along the stream.  pdl_trigger()
// lets the next kernel's CTAs be scheduled before this one finishes.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace stt
