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
// which the kernel's f16 weight parts stay finite; other weights use the GEMV.
bool tc_gemm_scales_ok(const uint8_t* q4_blocks, int64_t nblocks);

// TMA descriptors of a Q4 weight's nibble and scale planes (built once per weight on the host).
struct TcWeight {
    CUtensorMap nib, sc;
    CUtensorMap nib64, sc64;  // boxes of 64 rows, for the gate product (tc_make_gate_maps)
    int n, k;
    bool gate_ok;
};
cudaError_t tc_make_weight(const Q4Dev& w, TcWeight* out);
// The 64-row descriptors of linear_in ([2F][K]: gate rows, then value rows), for
// launch_tc_product_gate; leaves gate_ok false when 2F is not a multiple of 128.
cudaError_t tc_make_gate_maps(const Q4Dev& w, TcWeight* out);

// A TMA descriptor of `rank` dimensions (dims[0] contiguous; strides[i] = byte stride of dimension
// i + 1) with a box of box[i] elements per dimension; loads outside the array read zeros.
cudaError_t tma_encode(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank, const uint64_t* dims,
                       const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle);
// A 2-D TMA descriptor of a row-major [rows][inner] array of `type` (rows row_bytes apart) with a
// box of box_inner x box_rows elements; loads outside the array read zeros.
cudaError_t tma_encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner,
                          uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                          CUtensorMapSwizzle swizzle);

// Scratch of one product of M batch rows: the tiled f16 input (hi and lo parts) and the K-slice
// partial sums.
size_t tc_x16_bytes(int k, int M);
size_t tc_part_bytes(const Q4Dev& w, int M, int num_sms);

// out[m][n] (row stride ldo floats) = x[m][:] . dequant(w)[n][:] for m < M, x f16 [M][w.k] taken
// as exact; x16 and part are scratch of tc_x16_bytes / tc_part_bytes.  On a timeout a CTA sets
// *err to -5 (STT_E_DEVICE_FLAG) if it was 0 and leaves its partial sums unwritten.
cudaError_t launch_q4_tc_gemm(const TcWeight& tw, const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo,
                              __half* x16, float* part, int* err, int num_sms, cudaStream_t st);

// Smallest batch the step's layers run on the tensor cores (smaller batches use the GEMV).
constexpr int kTcMinBatch = 16;

// A batched decode step on the tensor cores keeps every product's input in x16 (tc_layout.cuh):
// launch_tc_prep writes it for the first product, and each product's epilogue writes the next
// one's (launch_tc_resid_norm, launch_tc_gate; the attention kernel for the output projection).
// Batch rows per tile and padded rows of a batch of `rows`.
void tc_batch_tiles(int rows, int* nt, int* rows_pad);
// x16 = rows of `in` [rows][K], RMSNorm'd with alpha when set.
cudaError_t launch_tc_prep(const float* in, const float* alpha, int K, int rows, __half* x16, cudaStream_t st);
// The GEMM: K-slice partial sums part[slices][rows][tw.n] of the weight times the x16 rows; the
// slice count is returned in *slices.  A timeout records -5 in *err (a step descriptor's error word).
// x_lo: the activations' lo parts take part (three products, about 22 significant bits); without
// them the activations count as their f16 hi parts (two products).
cudaError_t launch_tc_product(const TcWeight& tw, const __half* x16, int rows, float* part, int* err, int num_sms,
                              int* slices, cudaStream_t st, bool x_lo = true);
// linear_in ([2F][K], gate rows then value rows) with the gate fused into its epilogue: x16_out (the
// linear_out input, F columns) = silu(gate) * value, the values launch_tc_product followed by
// launch_tc_gate give.  x16_out must not be x16.
cudaError_t launch_tc_product_gate(const TcWeight& tw, const __half* x16, int rows, __half* x16_out, int* err,
                                   cudaStream_t st, bool x_lo = true);
// x[rows][D] += the slices (in order); x16 = RMSNorm(x) * alpha.
cudaError_t launch_tc_resid_norm(float* x, const float* part, int slices, int rows, int D, const float* alpha,
                                 __half* x16, cudaStream_t st);
// x16 = silu(gate) * value of the linear_in slices ([slices][rows][2F]: gate rows, then value rows).
cudaError_t launch_tc_gate(const float* part, int slices, int rows, int F, __half* x16, cudaStream_t st);

}  // namespace stt
