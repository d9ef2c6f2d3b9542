// Q4_0 x f16 matmul on the tcgen05 tensor cores (tc_gemm.cu).
#pragma once

#include <cuda.h>

#include <cstddef>
#include <cstdint>

#include "device.cuh"

namespace stt {

// K must be a multiple of 256 (the kernel moves K in quads of 8 Q4_0 blocks).
bool tc_gemm_supported(const Q4Dev& w);

// True when every f16 scale of the raw Q4_0 blocks (18 bytes each) has |s| <= 4, the range in
// which the kernel's f16 weight parts stay finite; other weights use the f32 GEMV.
bool tc_gemm_scales_ok(const uint8_t* q4_blocks, int64_t nblocks);

// TMA descriptors of a Q4 weight's nibble and scale planes (built once per weight on the host).
struct TcWeight {
    CUtensorMap nib, sc;
    int n, k;
};
cudaError_t tc_make_weight(const Q4Dev& w, TcWeight* out);

// Launch shape of one product: batch rows per tile, batch tiles, weight-row tiles of 128, K slices.
struct TcPlan {
    int nt, mtiles, tiles, slices;
};
TcPlan tc_gemm_plan(const Q4Dev& w, int M, int num_sms);

// Scratch of one product of M batch rows: the tiled f16 input (hi and lo parts) and the K-slice
// partial sums.
size_t tc_x16_bytes(int k, int M);
size_t tc_part_bytes(const Q4Dev& w, int M, int num_sms);

// out[m][n] (row stride ldo floats) = x[m][:] . dequant(w)[n][:] for m < M, x f16 [M][w.k] taken
// as exact; x16 and part are scratch of tc_x16_bytes / tc_part_bytes.  On a timeout a CTA sets
// *err to 1 (device int, expected 0) and leaves its partial sums unwritten.
cudaError_t launch_q4_tc_gemm(const TcWeight& tw, const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo,
                              __half* x16, float* part, int* err, int num_sms, cudaStream_t st);

struct Ctx;
struct GemvArgs;
// Smallest batch the step's layers run on the tensor cores (smaller batches use the GEMV).
constexpr int kTcMinBatch = 16;
// One layer product of a batched decode step on the tensor cores: the input rows (RMSNorm'd with
// a.norm when set) are split into f16 hi and lo parts in x16, the GEMM writes K-slice partial sums
// to part, and the epilogue kernel adds them in slice order and applies `epi` (EPI_QKV, EPI_RESID,
// EPI_GATE, EPI_LOGITS or EPI_PLAIN) exactly as the GEMV does.
cudaError_t launch_tc_layer(const Ctx& c, const GemvArgs& a, const TcWeight& tw, int epi, int rows, __half* x16,
                            float* part, int* err, int num_sms, cudaStream_t st);

}  // namespace stt
