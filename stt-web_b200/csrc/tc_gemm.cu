// Q4_0 x f16 matmul on the 5th-generation tensor cores (tcgen05, accumulator in TMEM).
//
// part[z][m][n] = sum over the K slice z of x[m][k] * w[n][k], for a batch of rows m (streams)
// and the Q4_0 weight rows n: the product of q4_matmul (gguf.rs:517-578) on the f16 tensor cores
// with f32 accumulation.  An epilogue kernel (kernels.cu) then adds the slices in slice order and
// applies the layer's epilogue, the same one the GEMV uses.
//
// Precision.  Each operand is split into two f16 parts, w = w_hi + w_lo and x = x_hi + x_lo, and
// three MMAs add w_hi.x_hi + w_hi.x_lo + w_lo.x_hi: about 22 significant bits per product, close
// to the f32 reference.  The dequantised weight q * s (q = nibble - 8 in [-8, 7], s the block's
// f16 scale) has at most 15 significant bits; it is formed in f16 as hi = rn(q * s') and
// lo = rn(q * s' - hi) (one fused multiply-add), where s' = s * 2^10 keeps lo clear of f16
// subnormals, so hi + lo = q * s' exactly.  The accumulator is scaled back by 2^-10 (exact).
// Weights with |s| > 4 would overflow f16 and are not sent here (tc_gemm_scales_ok).
//
// K order.  A 16-byte word of four Q4_0 payload bytes yields, with one mask per nibble position,
// the element pairs (4i, 4i+2), (4i+1, 4i+3), (16+4i, 16+4i+2), (16+4i+1, 16+4i+3) of its block;
// those four pairs form one 8-element row piece of the MMA operand.  The MMA sums over K, so the
// activations are stored in the same order (prep_f16_kernel) instead of shuffling the weights.
//
// Layout of the activations (x16): [part hi/lo][row tile of NT][64-wide chunk][NT x 64 f16 in the
// MMA's no-swizzle K-major core-matrix order: 8 rows x 16 bytes per 128-byte core matrix, core
// matrices along K 128 bytes apart, 8-row groups 1024 bytes apart], so one chunk of one part is a
// single contiguous bulk copy of NT * 128 bytes.
//
// Grid: (weight-row tiles of 128, batch-row tiles of NT, K slices).  A CTA of 256 threads:
//   - warp 7 bulk-copies (cp.async.bulk) its slice of the 128 weight rows into shared memory, one
//     copy of nibbles and one of scales per row, all on one mbarrier;
//   - thread 0 bulk-copies the activation chunks into a ring of B stages, two chunks ahead when
//     the ring has four stages;
//   - per 64-wide chunk, two threads per weight row dequantise one Q4_0 block each into the A
//     operand (hi and lo parts, two buffers), and thread 0 issues 4 x 3 MMAs of 128 x NT x 16
//     and commits them to an mbarrier;
//   - each warp reads 32 TMEM lanes (tcgen05.ld 32x32b) for half of the batch columns and stores
//     the partial sums.
// Every wait is bounded; on a timeout the CTA stops issuing, records an error, waits (bounded) for
// its MMAs and copies in flight, frees its TMEM and returns.
#include "tc_gemm.h"

#include <algorithm>

#include "kernels.h"

namespace stt {

namespace {

constexpr int kTM = 128;            // weight rows per CTA (MMA M, one TMEM lane each)
constexpr int kKC = 64;             // K elements per chunk (two Q4_0 blocks)
constexpr int kQuad = 256;          // K granule of a slice: 8 blocks, so scale copies stay 16-byte sized
constexpr int kMaxQuads = 4;        // quads per slice held in shared memory (1024 K)
constexpr int kThreads = 256;
constexpr int kNibStride = kMaxQuads * 8 * 16 + 16;  // bytes per weight row, padded against bank conflicts
constexpr int kScStride = kMaxQuads * 8 * 2 + 16;
constexpr uint32_t kSpin = 1u << 22;
constexpr float kWUnscale = 1.0f / 1024.0f;

__host__ __device__ constexpr int b_stages(int nt) { return nt >= 128 ? 2 : 4; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor: K-major, no swizzle; start address, leading byte offset (the
// next core matrix along K) and stride byte offset (the next 8-row group), in 16-byte units.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version of the 5th-generation tensor cores
    // base offset 0, leading-byte-offset mode 0, layout type 0 (no swizzle)
    return d;
}

// Instruction descriptor of kind::f16: f32 accumulator, f16 A and B, both K-major, M x N.
__host__ __device__ constexpr uint32_t instr_desc_f16(int M, int N) {
    return (1u << 4)                     // D format: f32
           | (0u << 7) | (0u << 10)      // A, B format: f16
           | (0u << 15) | (0u << 16)     // A, B K-major
           | ((uint32_t)(N >> 3) << 17)  // N / 8
           | ((uint32_t)(M >> 4) << 24); // M / 16
}

__device__ __forceinline__ void mbar_init(uint64_t* m) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(m)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* m, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(m)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* m, uint32_t parity) {
    for (uint32_t i = 0; i < kSpin; ++i)
        if (mbar_try(m, parity)) return true;
    return false;
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* m, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(m)), "r"(bytes) : "memory");
}
// Bulk copy global -> this CTA's shared memory, completing `bytes` on the mbarrier (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* m) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(m))
        : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* m) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(m))
                 : "memory");
}

// 16 consecutive f32 columns of this thread's TMEM lane, scaled back by 2^-10.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(__uint_as_float(r[i]), kWUnscale);  // exact: a power of two
}

template <int NT>
struct TcSmem {
    alignas(128) uint8_t a[2][2][kTM * kKC * 2];           // [buffer][hi, lo] weights, core-matrix layout
    alignas(128) uint8_t b[b_stages(NT)][2][NT * kKC * 2];  // [stage][hi, lo] activations, same layout
    alignas(128) uint8_t nib[kTM * kNibStride];             // the slice's Q4_0 nibbles, row after row
    alignas(128) uint8_t sc[kTM * kScStride];               // and its scales
    alignas(8) uint64_t raw_bar;
    alignas(8) uint64_t b_full[b_stages(NT)];
    alignas(8) uint64_t mma_done[4];                        // chunk c commits to mma_done[c % 4]
    uint32_t tmem;
};

// byte offset of 8-element piece k8 of row `row` of a [rows x 64] K-major chunk in core-matrix
// order: core matrix (row / 8, k8) at ((row / 8) * 8 + k8) * 128, row % 8 at 16-byte steps
__host__ __device__ __forceinline__ uint32_t core_off(int row, int k8) {
    return ((row >> 3) * 8 + k8) * 128 + (row & 7) * 16;
}

__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, 4);
    return h;
}
__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}

// Dequantises one Q4_0 block (16 payload bytes, scale bits sbits) into four 8-element pieces of
// hi parts and four of lo parts, in the K order described at the top of this file.
__device__ __forceinline__ void dequant_block(uint4 q, uint16_t sbits, uint4 (&hi)[4], uint4 (&lo)[4]) {
    // s * 2^10 is exact in f16 for every |s| <= 4
    const __half2 s2 = __half2half2(__hmul(__ushort_as_half(sbits), __ushort_as_half(0x6400)));
    const __half2 bias = u32_as_h2(0x64086408u);  // 1032 = 1024 + 8 in both halves
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const uint32_t w = words[wi];
        // 0x6400 | n is the f16 value 1024 + n; minus 1032 gives n - 8 exactly
        const uint32_t u[4] = {(w & 0x000F000Fu) | 0x64006400u, ((w >> 8) & 0x000F000Fu) | 0x64006400u,
                               ((w >> 4) & 0x000F000Fu) | 0x64006400u, ((w >> 12) & 0x000F000Fu) | 0x64006400u};
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 qv = __hsub2(u32_as_h2(u[j]), bias);
            const __half2 hv = __hmul2_rn(qv, s2);
            h[j] = h2_as_u32(hv);
            l[j] = h2_as_u32(__hfma2(qv, s2, __hneg2(hv)));  // the exact remainder q * s' - hi
        }
        hi[wi] = make_uint4(h[0], h[1], h[2], h[3]);
        lo[wi] = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// x16 holds the hi parts, then (x_lo != 0) the lo parts, in the tiled order above; without lo
// parts the input is taken as exact f16 and the hi.lo product is skipped.  Slice z covers the
// quads [z * nq / slices, (z + 1) * nq / slices) of K.  part: [slices][M][w.n].
template <int NT>
__global__ void __launch_bounds__(kThreads, 1) q4_tc_kernel(Q4Dev w, const __half* __restrict__ x16, int x_lo, int M,
                                                          int mtiles, int slices, float* __restrict__ part,
                                                          int* __restrict__ err) {
    extern __shared__ __align__(128) uint8_t tc_raw[];
    TcSmem<NT>& sm = *reinterpret_cast<TcSmem<NT>*>(tc_raw);
    constexpr int NBS = b_stages(NT);
    constexpr uint32_t kCols = NT < 32 ? 32 : NT;  // TMEM columns (a power of two >= 32)
    constexpr uint32_t kBBytes = NT * kKC * 2;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int n0 = blockIdx.x * kTM, mt = blockIdx.y, z = blockIdx.z;
    const int K = w.k, NB = K >> 5, nch = K / kKC, nq = K / kQuad;
    const int q0 = (int)((int64_t)z * nq / slices), q1 = (int)((int64_t)(z + 1) * nq / slices);
    const int c0 = q0 * 4, nchunks = (q1 - q0) * 4, sb = (q1 - q0) * 8;
    const int rows = min(kTM, w.n - n0);
    const int64_t part_elems = (int64_t)mtiles * NT * K;  // f16 elements per part of x16
    const __half* xb = x16 + ((int64_t)mt * nch + c0) * (NT * kKC);
    if (t == 0) {
        mbar_init(&sm.raw_bar);
        for (int i = 0; i < NBS; ++i) mbar_init(&sm.b_full[i]);
        for (int i = 0; i < 4; ++i) mbar_init(&sm.mma_done[i]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem)),
                     "r"(kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = sm.tmem;
    // the weight slice: one nibble copy and one scale copy per row (both multiples of 16 bytes)
    if (warp == 7) {
        if (lane == 0) mbar_expect_tx(&sm.raw_bar, (uint32_t)rows * sb * 18u);
        __syncwarp();
        for (int r = lane; r < rows; r += 32) {
            const int64_t blk = (int64_t)(n0 + r) * NB + q0 * 8;
            bulk_g2s(sm.nib + r * kNibStride, w.nib + blk, (uint32_t)sb * 16u, &sm.raw_bar);
            bulk_g2s(sm.sc + r * kScStride, w.scale + blk, (uint32_t)sb * 2u, &sm.raw_bar);
        }
    }
    // thread 0: activation chunk j -> stage j % NBS
    int issued = 0;
    auto issue_b = [&](int j) {
        uint64_t* fb = &sm.b_full[j % NBS];
        mbar_expect_tx(fb, (1u + (x_lo ? 1u : 0u)) * kBBytes);
        bulk_g2s(sm.b[j % NBS][0], xb + (int64_t)j * (NT * kKC), kBBytes, fb);
        if (x_lo) bulk_g2s(sm.b[j % NBS][1], xb + part_elems + (int64_t)j * (NT * kKC), kBBytes, fb);
        issued = j + 1;
    };
    if (t == 0)
        for (int j = 0; j < NBS - 2 && j < nchunks; ++j) issue_b(j);
    bool ok = mbar_wait(&sm.raw_bar, 0);
    const int row = t & (kTM - 1), bb = t >> 7;  // this thread's weight row and block of each chunk
    const uint32_t idesc = instr_desc_f16(kTM, NT);
    int committed = 0;  // chunks whose MMAs are committed (tracked by every thread)
    for (int c = 0; c < nchunks; ++c) {
        const int buf = c & 1;
        // the A buffer and the B stage refilled now were read by the MMAs of chunk c - 2
        if (c >= 2 && !mbar_wait(&sm.mma_done[(c - 2) & 3], ((c - 2) >> 2) & 1)) ok = false;
        if (t == 0 && ok && c + NBS - 2 < nchunks && c + NBS - 2 >= issued) issue_b(c + NBS - 2);
        uint8_t* Ah = sm.a[buf][0];
        uint8_t* Al = sm.a[buf][1];
        if (row < rows) {
            const int blk = c * 2 + bb;  // block within the slice
            const uint4 q = *reinterpret_cast<const uint4*>(sm.nib + row * kNibStride + blk * 16);
            const uint16_t sbits = *reinterpret_cast<const uint16_t*>(sm.sc + row * kScStride + blk * 2);
            uint4 hi[4], lo[4];
            dequant_block(q, sbits, hi, lo);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                *reinterpret_cast<uint4*>(Ah + core_off(row, 4 * bb + wi)) = hi[wi];
                *reinterpret_cast<uint4*>(Al + core_off(row, 4 * bb + wi)) = lo[wi];
            }
        } else {
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                *reinterpret_cast<uint4*>(Ah + core_off(row, 4 * bb + wi)) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(Al + core_off(row, 4 * bb + wi)) = make_uint4(0, 0, 0, 0);
            }
        }
        // generic-proxy writes of A -> visible to the tensor cores (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        if (t == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (mbar_wait(&sm.b_full[c % NBS], (c / NBS) & 1)) {
                const uint32_t ah = smem_u32(sm.a[buf][0]), al = smem_u32(sm.a[buf][1]);
                const uint32_t bh = smem_u32(sm.b[c % NBS][0]), bl = smem_u32(sm.b[c % NBS][1]);
#pragma unroll
                for (int k16 = 0; k16 < kKC / 16; ++k16) {
                    // K = 16 is two core matrices along K: LBO 128 bytes, 8-row groups 1024 bytes apart
                    const uint32_t o = k16 * 256;
                    mma_f16(tmem, smem_desc(ah + o, 128, 1024), smem_desc(bh + o, 128, 1024), idesc,
                            (c > 0 || k16 > 0) ? 1u : 0u);
                    if (x_lo) mma_f16(tmem, smem_desc(ah + o, 128, 1024), smem_desc(bl + o, 128, 1024), idesc, 1u);
                    mma_f16(tmem, smem_desc(al + o, 128, 1024), smem_desc(bh + o, 128, 1024), idesc, 1u);
                }
            } else {
                ok = false;  // seen by every thread at the next __syncthreads_and
            }
            mma_commit(&sm.mma_done[c & 3]);  // arrives once the MMAs issued so far are done
        }
        committed = c + 1;
    }
    // the last commit covers every MMA of the CTA
    if (committed > 0) {
        const int lc = committed - 1;
        if (!mbar_wait(&sm.mma_done[lc & 3], (lc >> 2) & 1)) ok = false;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const bool all_ok = __syncthreads_and(ok) && committed == nchunks;
    if (all_ok) {
        // tile row = TMEM lane: warp w reads lanes 32 (w % 4) .. +31, columns of its half
        const int trow = (warp & 3) * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        float* pz = part + (int64_t)z * M * w.n + n0 + trow;
#pragma unroll 1
        for (int j0 = (warp >> 2) * 16; j0 < NT; j0 += 32) {
            float v[16];
            tmem_ld16(lane_addr + j0, v);
            if (trow < rows)
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = mt * NT + j0 + j;
                    if (m < M) pz[(int64_t)m * w.n] = v[j];
                }
        }
    } else if (t == 0) {
        atomicExch(err, 1);
        // copies still in flight land before the CTA's shared memory goes away
        mbar_wait(&sm.raw_bar, 0);
        for (int j = committed; j < issued; ++j) mbar_wait(&sm.b_full[j % NBS], (j / NBS) & 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

int pick_nt(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

// Slices: at least enough to fit 4 quads each in shared memory, and up to one CTA per SM.
TcPlan make_plan(int n, int k, int M, int num_sms) {
    TcPlan p;
    p.nt = pick_nt(M);
    p.mtiles = (M + p.nt - 1) / p.nt;
    p.tiles = (n + kTM - 1) / kTM;
    const int nq = k / kQuad;
    const int need = (nq + kMaxQuads - 1) / kMaxQuads;
    const int fill = num_sms / std::max(1, p.tiles * p.mtiles);
    p.slices = std::max(need, std::min(nq, fill));
    return p;
}

template <int NT>
cudaError_t launch_nt(const Q4Dev& w, const __half* x16, int x_lo, int M, const TcPlan& p, float* part, int* err,
                      cudaStream_t st) {
    const size_t smem = sizeof(TcSmem<NT>);
    cudaError_t e = cudaFuncSetAttribute(q4_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(p.tiles, p.mtiles, p.slices);
    q4_tc_kernel<NT><<<grid, kThreads, smem, st>>>(w, x16, x_lo, M, p.mtiles, p.slices, part, err);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const Q4Dev& w, const __half* x16, int x_lo, int M, const TcPlan& p, float* part, int* err,
                        cudaStream_t st) {
    switch (p.nt) {
        case 16: return launch_nt<16>(w, x16, x_lo, M, p, part, err, st);
        case 32: return launch_nt<32>(w, x16, x_lo, M, p, part, err, st);
        case 64: return launch_nt<64>(w, x16, x_lo, M, p, part, err, st);
        default: return launch_nt<128>(w, x16, x_lo, M, p, part, err, st);
    }
}

// Position within a 32-element block of element e of an 8-element piece (see the K order above).
__device__ __forceinline__ int piece_elem(int e) { return ((e & 1) << 1) | ((e >> 1) & 1) | ((e >> 2) << 4); }

// f16 GEMM input of a batch, in the tiled K order of the kernel above.  One CTA per padded batch
// row (mtiles * nt of them); row m < M is row m of `in` (f32, bf16 when in_bf16, f16 when in_f16),
// with RMSNorm when alpha is not NULL (the same arithmetic as the GEMV's prologue: x / rms *
// alpha); rows >= M are zero.  Writes the hi parts and, when lo != 0, the lo parts (x = hi + lo).
__global__ void __launch_bounds__(256) prep_f16_kernel(const float* __restrict__ in, const __nv_bfloat16* __restrict__ in_bf16,
                                                       const __half* __restrict__ in_f16, const float* __restrict__ alpha,
                                                       int K, int M, int nt, int lo, __half* __restrict__ out) {
    __shared__ float red[32];
    const int m = blockIdx.x, mt = m / nt, r = m - mt * nt;
    const int nch = K / kKC;
    const int64_t lo_off = (int64_t)gridDim.x * K;  // the lo parts follow the hi parts of all rows
    uint8_t* const hi_base = reinterpret_cast<uint8_t*>(out + (int64_t)mt * nch * (nt * kKC));
    uint8_t* const lo_base = reinterpret_cast<uint8_t*>(out + lo_off + (int64_t)mt * nch * (nt * kKC));
    const int64_t base = (int64_t)m * K;
    float rms = 1.0f;
    if (alpha && m < M) {
        float ss = 0.0f;
        for (int j = threadIdx.x; j < K; j += blockDim.x) {
            const float v = in[base + j];
            ss = __fmaf_rn(v, v, ss);
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
            v = warp_sum(v);
            if (threadIdx.x == 0) red[0] = v;
        }
        __syncthreads();
        rms = sqrtf(__fadd_rn(__fdiv_rn(red[0], (float)K), 1e-8f));
    }
    // piece pi: 8 elements of block pi / 4, word pi % 4; chunk pi / 8, piece pi % 8 of the chunk
    for (int pi = threadIdx.x; pi < K / 8; pi += blockDim.x) {
        const int blk = pi >> 2, wi = pi & 3;
        const size_t off = (size_t)(pi >> 3) * (nt * kKC * 2) + core_off(r, pi & 7);
        __align__(16) __half h[8], l[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float v = 0.0f;
            if (m < M) {
                const int64_t k = base + blk * 32 + 4 * wi + piece_elem(e);
                v = in_f16 ? __half2float(in_f16[k]) : in_bf16 ? __bfloat162float(in_bf16[k]) : in[k];
                if (alpha) v = __fmul_rn(__fdiv_rn(v, rms), alpha[blk * 32 + 4 * wi + piece_elem(e)]);
            }
            h[e] = __float2half_rn(v);
            l[e] = __float2half_rn(__fsub_rn(v, __half2float(h[e])));
        }
        *reinterpret_cast<uint4*>(hi_base + off) = *reinterpret_cast<const uint4*>(h);
        if (lo) *reinterpret_cast<uint4*>(lo_base + off) = *reinterpret_cast<const uint4*>(l);
    }
}

cudaError_t launch_prep(const float* in, const __nv_bfloat16* in_bf16, const __half* in_f16, const float* alpha, int K,
                        int M, const TcPlan& p, int lo, __half* x16, cudaStream_t st) {
    prep_f16_kernel<<<p.mtiles * p.nt, 256, 0, st>>>(in, in_bf16, in_f16, alpha, K, M, p.nt, lo, x16);
    return cudaGetLastError();
}

}  // namespace

bool tc_gemm_supported(const Q4Dev& w) { return w.k % kQuad == 0 && w.k > 0 && w.n > 0; }

bool tc_gemm_scales_ok(const uint8_t* q4_blocks, int64_t nblocks) {
    // Q4_0 block: f16 scale, then 16 payload bytes; |s| <= 4 keeps every q * s * 2^10 finite in f16
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint16_t s = (uint16_t)(q4_blocks[b * 18] | (q4_blocks[b * 18 + 1] << 8));
        if ((s & 0x7FFFu) > 0x4400u) return false;  // 0x4400 = 4.0; larger magnitudes, inf and nan fail
    }
    return true;
}

TcPlan tc_gemm_plan(const Q4Dev& w, int M, int num_sms) { return make_plan(w.n, w.k, M, num_sms); }

size_t tc_x16_bytes(int k, int M) {
    const TcPlan p = make_plan(1, k, M, 1);
    return 2 * (size_t)p.mtiles * p.nt * k * sizeof(__half);
}

size_t tc_part_bytes(const Q4Dev& w, int M, int num_sms) {
    const TcPlan p = make_plan(w.n, w.k, M, num_sms);
    return (size_t)p.slices * M * w.n * sizeof(float);
}

cudaError_t launch_q4_tc_gemm(const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo, __half* x16,
                              float* part, int* err, int num_sms, cudaStream_t st) {
    const TcPlan p = make_plan(w.n, w.k, M, num_sms);
    cudaError_t e = launch_prep(nullptr, nullptr, x, nullptr, w.k, M, p, 0, x16, st);
    if (e != cudaSuccess) return e;
    e = launch_gemm(w, x16, 0, M, p, part, err, st);
    if (e != cudaSuccess) return e;
    GemvArgs a{};
    a.W = w;
    a.out = out;
    a.ldo = ldo;
    a.n_units = (w.n + 1) / 2;
    return launch_tc_epilogue(Ctx{}, a, EPI_PLAIN, M, part, p.slices, st);
}

cudaError_t launch_tc_layer(const Ctx& c, const GemvArgs& a, int epi, int rows, __half* x16, float* part, int* err,
                            int num_sms, cudaStream_t st) {
    const TcPlan p = make_plan(a.W.n, a.W.k, rows, num_sms);
    cudaError_t e = launch_prep(a.in, a.in_bf16, nullptr, a.norm, a.W.k, rows, p, 1, x16, st);
    if (e != cudaSuccess) return e;
    e = launch_gemm(a.W, x16, 1, rows, p, part, err, st);
    if (e != cudaSuccess) return e;
    return launch_tc_epilogue(c, a, epi, rows, part, p.slices, st);
}

}  // namespace stt
