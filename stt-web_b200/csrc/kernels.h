// Host-side launchers of the step kernels (kernels.cu).
#pragma once

#include <cuda.h>

#include "device.cuh"

namespace stt {

constexpr int kMaxGemvK = 8448;  // largest reduction length the GEMV stages in shared memory

// TMA descriptors of one Q4 weight for the tensor-core GEMV (gemv_mma_kernel): boxes of 8 rows of
// one quad of nibbles (128 bytes) and of 64 scales (128 bytes), both with the 128-byte swizzle.
struct GemvMaps {
    CUtensorMap nib, sc;
    bool ok = false;  // K a multiple of 256 and both descriptors built
};
cudaError_t gemv_make_maps(const Q4Dev& w, GemvMaps* out);

enum Epi : int { EPI_PLAIN = 0, EPI_QKV = 1, EPI_GATE = 2, EPI_RESID = 3, EPI_LOGITS = 4 };

// One Q4 matmul of the step: out = W . vec for each batch row, with the epilogue `epi`.
struct GemvArgs {
    Q4Dev W;
    const float* in;                 // [rows][K] f32 input (ignored when in_bf16 != NULL)
    const __nv_bfloat16* in_bf16;    // [rows][K] bf16 input or NULL
    const float* norm;               // RMSNorm alpha applied to the input, or NULL
    float* out;                      // destination (see Epi)
    int64_t ldo;                     // destination row stride in floats
    int32_t layer;                   // layer of the K/V ring (EPI_QKV)
    int32_t n_units;                 // pairs of output rows
    int32_t half_n;                  // EPI_GATE: value rows start here (= ffn width)
    int* err;                        // where a kernel records a timeout when there is no step descriptor
    const GemvMaps* maps;            // host copy of W's GEMV descriptors, or NULL (host side only)
    int32_t stall_test;              // test hook: the integer-MMA GEMV's first stage is never loaded, so
                                     // its waits run out and report STT_E_DEVICE_FLAG
};

// Per-call descriptor and batch ids, written on the device from launch parameters so that
// back-to-back asynchronous calls never race on a host staging buffer.
constexpr int kMaxBatch = 4096;
constexpr int kSmallBatch = 64;  // batches up to this size use a 300-byte parameter block
struct DescInit {
    StepDesc desc;
    int32_t n;
    int32_t ids[kMaxBatch];
};

cudaError_t configure_kernels();
cudaError_t launch_set_state(StreamState* dst, const StreamState& value, cudaStream_t st);
cudaError_t launch_set_desc(StepDesc* d_desc, int32_t* d_ids, const DescInit& p, cudaStream_t st);
// Raw Q4_0 blocks -> the nibble and scale planes; big_scale (may be NULL) is set to 1 when a scale's
// magnitude is above 4 (the tensor-core product's limit).
cudaError_t launch_repack_q4(const uint8_t* raw, int64_t nblocks, uint4* nib, uint16_t* scale, cudaStream_t st,
                             int* big_scale = nullptr);
cudaError_t launch_dequant_q4(const Q4Dev& w, float* out, cudaStream_t st);
// The batched Q4 GEMV of the step (and of the isolated f32 / bf16 matmul): one launch per pass of
// up to 8 batch rows (4 when K > 4096), each pass reading the weights once; passes of several rows
// take the integer-MMA kernel when a.maps holds W's descriptors, single rows the dp4a kernels.
cudaError_t launch_gemv(const Ctx& c, const GemvArgs& a, int epi, int rows, cudaStream_t st);
// The integer-MMA GEMV (gemv_mma.cu) for passes of up to mb in {2, 4, 8} rows: whether it takes a
// pass of mb rows of this product, and its launch (one launch per pass).
bool gemv_mma_ok(const GemvArgs& a, int mb);
cudaError_t launch_gemv_mma(const Ctx& c, const GemvArgs& a, int epi, int mb, int rows, cudaStream_t st);
cudaError_t configure_gemv_mma();
cudaError_t launch_embed(const Ctx& c, cudaStream_t st);
cudaError_t launch_attention(const Ctx& c, int layer, cudaStream_t st);
cudaError_t launch_finish(const Ctx& c, cudaStream_t st);
// Adds the K-slice partial sums part[slices][rows][a.W.n] of a tensor-core product in slice order
// and applies the epilogue `epi` as launch_gemv does.
cudaError_t launch_tc_epilogue(const Ctx& c, const GemvArgs& a, int epi, int rows, const float* part, int slices,
                               cudaStream_t st);

}  // namespace stt
