// Q4_0 x f16 matmul on the tcgen05 tensor cores (tc_gemm.cu).
#pragma once

#include "device.cuh"

namespace stt {

// K must be a multiple of 64.
bool tc_gemm_supported(const Q4Dev& w);

// out[m][n] (row stride ldo floats) = x[m][:] . dequant(w)[n][:] for m < M, f16 x [M][w.k]; on a
// timeout a CTA sets *err to 1 (device int, expected 0).
cudaError_t launch_q4_tc_gemm(const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo, int* err, cudaStream_t st);

}  // namespace stt
