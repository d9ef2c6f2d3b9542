// Split-K Q4 matmul whose scratch is a fixed device array of this library (noalloc.cu).
#pragma once

#include "device.cuh"

namespace stt {

// Partial sums of every split: splits x rows x n floats must fit here.
constexpr size_t kNoAllocPartialBytes = size_t(4) << 20;
// One arrival counter per tile of kNoAllocTileRows output rows: n <= 4096 * 16 = 65536.
constexpr int kNoAllocTickets = 4096;
constexpr int kNoAllocTileRows = 16;
constexpr int kNoAllocMaxSplits = 64;

// Device address of the fixed scratch on the current device.
cudaError_t noalloc_scratch_address(void** out);

// out[rows][n] = in[rows][k] . W^T with the reduction over k cut into `splits` ranges of whole
// Q4_0 blocks; `scratch` is the address noalloc_scratch_address returned for this device.
cudaError_t launch_q4_matmul_splitk(const Q4Dev& w, const float* in, const __nv_bfloat16* in_bf16, int rows,
                                    float* out, int splits, void* scratch, cudaStream_t st);

}  // namespace stt
