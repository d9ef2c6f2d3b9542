// Split-K Q4 matmul that allocates nothing: its partial sums and arrival counters live in a
// fixed array of this library's device image instead of memory the call would have to request.
//
// The same product as the q4_matmul of gguf.rs:517-578 (and of stt_q4_matmul_device), with the
// reduction over k cut into `splits` ranges of whole Q4_0 blocks.  CTA (tile, split) computes
// the partial dot products of 16 output rows over its block range, in the per-block order of
// shader_naive.wgsl:47-97 (low-nibble and high-nibble halves summed apart, then scaled), writes
// them to the scratch and takes a ticket on the tile's counter.  The CTA that arrives last adds
// the partials of every split in split order, so the result does not depend on which CTA ran
// first, writes the output rows and sets the counter back to zero.
#include "noalloc.h"

namespace stt {

namespace {

constexpr int kThreads = 256;                   // 8 warps, one pair of output rows each
constexpr size_t kTicketBytes = size_t(kNoAllocTickets) * 4;
constexpr int kRowsPerPass = 4;                 // batch rows accumulated together per pass

}  // namespace

// [counters: kNoAllocTickets u32][partials: kNoAllocPartialBytes], 4 MiB + 16 KiB per device.
// The counters must be zero when a call starts: the module's static initialisation zeroes them
// and every call leaves each counter it used at zero again.  The partials need no initial value;
// a call writes every partial it reads.  One array per device serves all calls on that device,
// so two calls whose kernels overlap in time (different streams, or different host threads
// without ordering between them) race on it and give wrong results.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kTicketBytes + kNoAllocPartialBytes];

namespace {

__device__ __forceinline__ float4 load_x4(const float* in, const __nv_bfloat16* in_bf16, int64_t i) {
    if (in_bf16) {
        const uint2 r = __ldg(reinterpret_cast<const uint2*>(in_bf16 + i));
        return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u), __uint_as_float(r.y << 16),
                           __uint_as_float(r.y & 0xFFFF0000u));
    }
    return __ldg(reinterpret_cast<const float4*>(in + i));
}

// Sum over one block of (nibble - 8) * x: low nibbles (elements 0-15) and high nibbles
// (elements 16-31) accumulated apart in element order, then added.
__device__ __forceinline__ float block_dot_x(const uint4 q, const float* in, const __nv_bfloat16* in_bf16, int64_t x0) {
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const float4 lo = load_x4(in, in_bf16, x0 + 4 * wi);
        const float4 hi = load_x4(in, in_bf16, x0 + 16 + 4 * wi);
        const uint32_t w = words[wi];
        s0 = __fmaf_rn(nib_m8(w & 0xFu), lo.x, s0);
        s1 = __fmaf_rn(nib_m8((w >> 4) & 0xFu), hi.x, s1);
        s0 = __fmaf_rn(nib_m8((w >> 8) & 0xFu), lo.y, s0);
        s1 = __fmaf_rn(nib_m8((w >> 12) & 0xFu), hi.y, s1);
        s0 = __fmaf_rn(nib_m8((w >> 16) & 0xFu), lo.z, s0);
        s1 = __fmaf_rn(nib_m8((w >> 20) & 0xFu), hi.z, s1);
        s0 = __fmaf_rn(nib_m8((w >> 24) & 0xFu), lo.w, s0);
        s1 = __fmaf_rn(nib_m8(w >> 28), hi.w, s1);
    }
    return s0 + s1;
}

// grid (tiles, splits).  Partial of split s, batch row m, output row r at part[(s*rows + m)*n + r].
__global__ void __launch_bounds__(kThreads) q4_splitk_kernel(Q4Dev w, const float* __restrict__ in,
                                                             const __nv_bfloat16* __restrict__ in_bf16, int rows,
                                                             float* __restrict__ out, uint32_t* __restrict__ tickets,
                                                             float* __restrict__ part) {
    __shared__ int last;
    const int tile = blockIdx.x, s = blockIdx.y, splits = gridDim.y;
    const int n = w.n, K = w.k, NB = K >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = (int)((int64_t)NB * s / splits), b1 = (int)((int64_t)NB * (s + 1) / splits);
    const int ra = tile * kNoAllocTileRows + 2 * warp;
    const int rb = ra + 1;
    if (ra < n) {
        const int rbl = rb < n ? rb : ra;  // a lone last row reads its own weights twice
        const uint4* na = w.nib + (int64_t)ra * NB;
        const uint4* nb = w.nib + (int64_t)rbl * NB;
        const uint16_t* sa = w.scale + (int64_t)ra * NB;
        const uint16_t* sb = w.scale + (int64_t)rbl * NB;
        for (int m0 = 0; m0 < rows; m0 += kRowsPerPass) {
            float acc[2][kRowsPerPass];
#pragma unroll
            for (int i = 0; i < kRowsPerPass; ++i) acc[0][i] = acc[1][i] = 0.0f;
            for (int b = b0 + lane; b < b1; b += 32) {
                const uint4 qa = __ldg(na + b), qb = __ldg(nb + b);
                const float da = f16_to_f32_ieee(__ldg(sa + b)), db = f16_to_f32_ieee(__ldg(sb + b));
#pragma unroll
                for (int i = 0; i < kRowsPerPass; ++i) {
                    if (m0 + i < rows) {
                        const int64_t x0 = (int64_t)(m0 + i) * K + (int64_t)b * 32;
                        acc[0][i] = __fmaf_rn(da, block_dot_x(qa, in, in_bf16, x0), acc[0][i]);
                        acc[1][i] = __fmaf_rn(db, block_dot_x(qb, in, in_bf16, x0), acc[1][i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < kRowsPerPass; ++i) {
                if (m0 + i < rows) {
                    const float va = warp_sum(acc[0][i]), vb = warp_sum(acc[1][i]);
                    if (lane == 0) {
                        float* p = part + ((int64_t)s * rows + m0 + i) * n;
                        p[ra] = va;
                        if (rb < n) p[rb] = vb;
                    }
                }
            }
        }
    }
    // publish the partials, then take a ticket; the last of the tile's splits reduces
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(tickets + tile, 1u) == (uint32_t)(splits - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < rows * kNoAllocTileRows; idx += kThreads) {
        const int m = idx / kNoAllocTileRows;
        const int r = tile * kNoAllocTileRows + idx % kNoAllocTileRows;
        if (r >= n) continue;
        float v = __ldcg(part + (int64_t)m * n + r);
        for (int t = 1; t < splits; ++t) v = __fadd_rn(v, __ldcg(part + ((int64_t)t * rows + m) * n + r));
        out[(int64_t)m * n + r] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) atomicExch(tickets + tile, 0u);
}

}  // namespace

cudaError_t noalloc_scratch_address(void** out) { return cudaGetSymbolAddress(out, g_noalloc_scratch); }

cudaError_t launch_q4_matmul_splitk(const Q4Dev& w, const float* in, const __nv_bfloat16* in_bf16, int rows,
                                    float* out, int splits, void* scratch, cudaStream_t st) {
    uint8_t* base = static_cast<uint8_t*>(scratch);
    const int tiles = (w.n + kNoAllocTileRows - 1) / kNoAllocTileRows;
    q4_splitk_kernel<<<dim3(tiles, splits), kThreads, 0, st>>>(w, in, in_bf16, rows, out,
                                                               reinterpret_cast<uint32_t*>(base),
                                                               reinterpret_cast<float*>(base + kTicketBytes));
    return cudaGetLastError();
}

}  // namespace stt
