// Q4_0 x f16 matmul on the tcgen05 tensor cores (tc_gemm.cu).
#pragma once

#include "device.cuh"

namespace stt {

// K must be a multiple of 64.
bool tc_gemm_supported(const Q4Dev& w);

// out[m][n] (row stride ldo floats) = x[m][:] . dequant(w)[n][:] for m < M; x holds f16 hi parts
// [M][w.k] followed by lo parts [M][w.k] (x = hi + lo); on a timeout a CTA sets *err to 1 (device
// int, expected 0).
cudaError_t launch_q4_tc_gemm(const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo, int* err, cudaStream_t st);

struct Ctx;
struct GemvArgs;
// Smallest batch the step's layers run on the tensor cores (smaller batches use the GEMV).
constexpr int kTcMinBatch = 16;
// One layer product of a batched decode step on the tensor cores: the input rows (RMSNorm'd with
// a.norm when set) are written to x16 as f16 hi and lo parts [2][rows][a.W.k], then the GEMM
// applies the epilogue
// `epi` (EPI_QKV, EPI_RESID, EPI_GATE, EPI_LOGITS or EPI_PLAIN) exactly as the GEMV does.
cudaError_t launch_tc_layer(const Ctx& c, const GemvArgs& a, int epi, int rows, __half* x16, int* err, cudaStream_t st);

}  // namespace stt
