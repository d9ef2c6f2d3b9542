// Layout of the tensor-core GEMM's activation operand (x16), shared by every kernel that writes it.
//
// x16 = [part: hi, lo][batch-row tile of nt rows][64-wide chunk of K][nt x 64 f16 in the MMA's
// no-swizzle K-major core-matrix order].  Within a chunk, 8-element piece k8 of row r sits at byte
// ((r / 8) * 8 + k8) * 128 + (r % 8) * 16.  A piece holds, of Q4_0 block pi / 4 and payload word
// w = pi % 4, the elements 4w + {0, 2, 1, 3} and 16 + 4w + {0, 2, 1, 3}: the order in which the
// GEMM's dequantisation unpacks a payload word (the MMA sums over K, so both operands only need
// the same order).  The lo parts (x - hi rounded to f16) follow the hi parts of all padded rows.
#pragma once

#include "device.cuh"

namespace stt {

__host__ __device__ __forceinline__ uint32_t core_off(int row, int k8) {
    return ((row >> 3) * 8 + k8) * 128 + (row & 7) * 16;
}

// First element (within the row) of piece pi's two runs of four: k0 .. k0+3 and k0+16 .. k0+19.
__host__ __device__ __forceinline__ int piece_k0(int pi) { return (pi >> 2) * 32 + 4 * (pi & 3); }

// Writes piece pi of batch row m from the row's values a = x[k0 .. k0+3], b = x[k0+16 .. k0+19]:
// the f16 hi parts and, when lo, the lo parts.  rows_pad = batch tiles * nt.
__device__ __forceinline__ void x16_store_piece(__half* x16, int nt, int rows_pad, int K, int m, int pi, float4 a,
                                                float4 b, bool lo) {
    const float v[8] = {a.x, a.z, a.y, a.w, b.x, b.z, b.y, b.w};
    __align__(16) __half h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        h[e] = __float2half_rn(v[e]);
        l[e] = __float2half_rn(__fsub_rn(v[e], __half2float(h[e])));
    }
    const int mt = m / nt, r = m - mt * nt;
    const size_t off = ((size_t)mt * (K / 64) + (pi >> 3)) * (size_t)(nt * 64 * 2) + core_off(r, pi & 7);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(x16) + off) = *reinterpret_cast<const uint4*>(h);
    if (lo)
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(x16 + (int64_t)rows_pad * K) + off) =
            *reinterpret_cast<const uint4*>(l);
}

}  // namespace stt
