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
// K order.  A 32-bit word (four Q4_0 payload bytes) yields, with one mask per nibble position,
// the element pairs (4i, 4i+2), (4i+1, 4i+3), (16+4i, 16+4i+2), (16+4i+1, 16+4i+3) of its block;
// those four pairs form one 8-element row piece of the MMA operand.  The MMA sums over K, so the
// activations are stored in the same order (prep_f16_kernel) instead of shuffling the weights.
//
// Layout of the activations (x16): [part hi/lo][row tile of NT][64-wide chunk][NT x 64 f16 in the
// MMA's no-swizzle K-major core-matrix order: 8 rows x 16 bytes per 128-byte core matrix, core
// matrices along K 128 bytes apart, 8-row groups 1024 bytes apart], so one chunk of one part is a
// single contiguous bulk copy of NT * 128 bytes.
//
// Grid: (weight-row tiles of 128, batch-row tiles of NT, K slices).  A CTA (one per SM: it takes
// the SM's whole tensor memory) runs a warp-specialised pipeline with mbarrier hand-offs and no
// CTA-wide barrier inside the K loop:
//   - warp 0 loads, per 256-wide quad of K, the 128 rows' Q4_0 nibbles (16 KB, 128-byte swizzle)
//     and scales (2 KB) with two 2-D TMA loads into a ring of raw stages;
//   - warp 14 copies, per 64-wide chunk, the activation tile (hi, lo) with bulk copies into a
//     ring of B stages;
//   - warps 2..13 dequantise in three groups of four that take the chunks in turn: one thread per
//     weight row and chunk (two Q4_0 blocks), writing the hi and lo parts straight into a ring of
//     A stages in tensor memory (tcgen05.st; weight row = TMEM lane), then signalling the stage
//     with one arrive per warp;
//   - warp 1 issues from one elected lane, per round of 1 to 3 chunks (TcCfg), 4 x 3 MMAs of
//     128 x NT x 16 per chunk with A read from tensor memory and B from shared memory into the TMEM
//     accumulator, and commits them to the barriers that free the A and B stages they read;
//   - after the last commit, warps 2..13 read the accumulator (tcgen05.ld 32x32b; each warp its
//     32 TMEM lanes and a third of the batch columns) and store the partial sums.
// The copy and MMA roles run as whole warps and issue from one elected lane (elect.sync).
// Measured on the 16896 x 2048 product at 64 batch rows, the dequantisation sets the pace (the MMA
// lane waits for the slowest dequantising warp) and its per-iteration overhead (waits, fences,
// TMEM stores, index arithmetic) is a large share of it, hence whole chunks per thread.
// Every wait is bounded and polls a shared abort word; a timeout sets it, every role stops
// issuing, the copies and MMAs in flight are waited for (bounded), the CTA records an error,
// frees its TMEM and returns without storing.
#include "tc_gemm.h"

#include <cudaTypedefs.h>

#include <algorithm>

#include "kernels.h"
#include "tc_layout.cuh"

namespace stt {

namespace {

constexpr int kTM = 128;        // weight rows per CTA (MMA M, one TMEM lane each)
constexpr int kKC = 64;         // K elements per chunk (two Q4_0 blocks)
constexpr int kQuad = 256;      // K elements per raw stage (8 blocks: 128 nibble bytes, 16 scale bytes per row)
constexpr uint32_t kAStageCols = 64; // per A stage: hi part in 32 columns (64 f16 per lane), then lo
constexpr uint32_t kTmemCols = 512;  // allocated TMEM columns (the whole SM's; one CTA per SM)
constexpr int kDqGroups = 3;    // groups of four dequantising warps, taking chunks in turn
constexpr int kDqWarps = 4 * kDqGroups;  // warps 2 .. 13; warp 14 copies the activations
constexpr int kBWarp = 2 + kDqWarps;
constexpr int kThreads = 32 * (kBWarp + 1);
constexpr uint32_t kRNib = kTM * 128;  // raw nibble bytes per stage
constexpr uint32_t kRSc = kTM * 16;    // raw scale bytes per stage
constexpr uint32_t kSpin = 1u << 22;
constexpr uint32_t kNap = 64;  // ns between polls of a wait off the critical path
constexpr float kWUnscale = 1.0f / 1024.0f;

// Pipeline shape by batch tile.  Up to 64 batch rows: the accumulator takes TMEM columns 0 .. 63,
// leaving room for 6 A stages from column 64; 6 B stages; MMAs issued per round of 3 chunks.
// 128 rows: 4-stage rings, accumulator in columns 0 .. 127, A stages from column 128, rounds of
// 2 chunks.  256 rows: a 32 KB B tile per part, so 2 B stages and 3 raw stages fit in shared
// memory; accumulator in columns 0 .. 255, A stages from 256; the 12 MMAs of one chunk already
// keep the tensor cores busy for about 1,700 cycles, so they go out per chunk.
template <int NT>
struct TcCfg {
    static constexpr bool kWide = NT >= 256;
    static constexpr bool kNarrow = NT <= 64;          // accumulator in columns 0 .. 63: room for 6 A stages
    static constexpr int kRS = kWide ? 3 : 4;          // raw stages
    static constexpr int kAS = kNarrow ? 6 : 4;        // A stages in tensor memory
    static constexpr int NBS = kWide ? 2 : kNarrow ? 6 : 4;  // B stages
    static constexpr uint32_t kACol = kWide ? 256 : kNarrow ? 64 : 128;
    static constexpr int kStep = kWide ? 1 : kNarrow ? 3 : 2;  // chunks per MMA round
};

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

__device__ __forceinline__ void mbar_init(uint64_t* m, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(m)), "r"(count) : "memory");
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
// Bounded wait for the phase of parity `parity`; gives up when the CTA's abort word is set or
// after kSpin polls (then sets it).  Waits off the critical path back off by `nap` ns between
// polls, so that they leave the barrier unit to the MMA-issuing warp.
__device__ __forceinline__ bool mbar_wait(uint64_t* m, uint32_t parity, volatile int* abort, uint32_t nap = 0) {
    for (uint32_t i = 0; i < kSpin; ++i) {
        if (mbar_try(m, parity)) return true;
        if ((i & 63u) == 63u && *abort) return false;
        if (nap) __nanosleep(nap);
    }
    *abort = 1;
    return false;
}
// Bounded wait that ignores the abort word (draining copies and MMAs before exit).
__device__ __forceinline__ void mbar_drain(uint64_t* m, uint32_t parity) {
    for (uint32_t i = 0; i < kSpin; ++i)
        if (mbar_try(m, parity)) return;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* m) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(m)) : "memory");
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
// 2-D TMA tile load (x = innermost coordinate in elements), completing on the mbarrier (no multicast).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* m) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(m))
        : "memory");
}

// D (+)= A * B, f16 operands, f32 accumulator in TMEM, with A read from tensor memory (row i of A
// in TMEM lane i, two f16 per 32-bit column) and B from shared memory through its descriptor.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// Named barrier of `count` threads; bar_any also returns whether any of them passed cond.
__device__ __forceinline__ void bar_sync_n(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ bool bar_any(int id, int count, bool cond) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)cond), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}
// silu(g) = g * (1 / (1 + exp(-g))), times the value: the GEMV's gate epilogue.
__device__ __forceinline__ float gated(float g, float v) {
    return __fmul_rn(__fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)))), v);
}

// True in exactly one lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xFFFFFFFF;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}
// Arrives on the mbarrier once every MMA issued so far by this thread has completed.
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

// 16 consecutive 32-bit columns of this thread's TMEM lane (warp-collective).
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

template <int NT>
struct TcSmem {
    using C = TcCfg<NT>;
    uint8_t rnib[C::kRS][kRNib];                          // raw nibbles [128 rows][128 B], 128-byte swizzle
    uint8_t rsc[C::kRS][kRSc];                            // raw scales [128 rows][8]
    uint8_t b[2 * C::NBS][NT * kKC * 2];                  // activation parts, same layout: with lo parts
                                                          // NBS stages of (hi, lo), without them 2 NBS
                                                          // stages of hi parts only
    uint64_t r_full[C::kRS], r_empty[C::kRS], a_full[C::kAS], a_empty[C::kAS];
    uint64_t b_full[2 * C::NBS], b_empty[2 * C::NBS], done;
    uint32_t tmem;
    int abort;
};
// the TMA's 128-byte swizzle repeats every 1024 bytes: the shared-memory block is aligned to that;
// at least 120 KB, so that one CTA holds an SM (and all of its tensor memory) at a time
template <int NT>
constexpr size_t smem_bytes() { return sizeof(TcSmem<NT>) + 1024 > 120 * 1024 ? sizeof(TcSmem<NT>) + 1024 : 120 * 1024; }

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

// Dequantises W payload words of one Q4_0 block (scale bits sbits): each word gives one 8-element
// piece (4 half2) of hi parts and one of lo parts, in the K order described at the top of this file.
template <int W>
__device__ __forceinline__ void dequant_words(const uint32_t (&words)[W], uint16_t sbits, uint32_t (&h)[4 * W],
                                              uint32_t (&l)[4 * W]) {
    // s * 2^10 is exact in f16 for every |s| <= 4
    const __half2 s2 = __half2half2(__hmul(__ushort_as_half(sbits), __ushort_as_half(0x6400)));
    const __half2 bias = u32_as_h2(0x64086408u);  // 1032 = 1024 + 8 in both halves
#pragma unroll
    for (int wi = 0; wi < W; ++wi) {
        const uint32_t w = words[wi];
        // 0x6400 | n is the f16 value 1024 + n; minus 1032 gives n - 8 exactly
        const uint32_t u[4] = {(w & 0x000F000Fu) | 0x64006400u, ((w >> 8) & 0x000F000Fu) | 0x64006400u,
                               ((w >> 4) & 0x000F000Fu) | 0x64006400u, ((w >> 12) & 0x000F000Fu) | 0x64006400u};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 qv = __hsub2(u32_as_h2(u[j]), bias);
            const __half2 hv = __hmul2_rn(qv, s2);
            h[4 * wi + j] = h2_as_u32(hv);
            l[4 * wi + j] = h2_as_u32(__hfma2(qv, s2, __hneg2(hv)));  // the exact remainder q * s' - hi
        }
    }
}

// x16 holds the hi parts, then (x_lo != 0) the lo parts, in the tiled order above; without lo
// parts the input is taken as exact f16 and the hi.lo product is skipped.  Slice z covers the
// quads [z * nq / slices, (z + 1) * nq / slices) of K.  part: [slices][M][n].
//
// GATE (linear_in, one slice): the maps' boxes are 64 rows high, and CTA x loads the gate rows
// 64x .. 64x+63 into tile rows 0..63 and their value rows gate_f + 64x .. into tile rows 64..127;
// instead of partial sums the epilogue writes silu(gate) * value of its 64 units straight into the
// next product's input x16_out (gate_f columns, hi and lo parts; rows_pad = mtiles * NT), the
// gate_kernel's arithmetic.
template <int NT, bool XLO, bool GATE>
__global__ void __launch_bounds__(kThreads, 1) q4_tc_kernel(const __grid_constant__ CUtensorMap tm_nib,
                                                          const __grid_constant__ CUtensorMap tm_sc, int n, int K,
                                                          const __half* __restrict__ x16, int M, int mtiles, int slices,
                                                          float* __restrict__ part, int* __restrict__ err,
                                                          __half* __restrict__ x16_out, int gate_f) {
    constexpr bool x_lo = XLO;
    extern __shared__ uint8_t tc_raw[];
    TcSmem<NT>& sm = *reinterpret_cast<TcSmem<NT>*>(tc_raw + ((1024u - (smem_u32(tc_raw) & 1023u)) & 1023u));
    using C = TcCfg<NT>;
    constexpr int kRS = C::kRS, kAS = C::kAS, kStep = C::kStep;
    // activation stages: without lo parts each stage holds one part, so there are twice as many
    // (more copies in flight ahead of the MMAs in the same shared memory)
    constexpr int NBS = XLO ? C::NBS : 2 * C::NBS;
    constexpr uint32_t kACol = C::kACol;
    constexpr uint32_t kBBytes = NT * kKC * 2;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int n0 = blockIdx.x * kTM, mt = blockIdx.y, z = blockIdx.z;
    const int nch = K / kKC, nq = K / kQuad;
    const int q0 = (int)((int64_t)z * nq / slices), q1 = (int)((int64_t)(z + 1) * nq / slices);
    const int nquads = q1 - q0, nchunks = 4 * nquads;
    volatile int* abort = &sm.abort;
    if (t == 0) {
        for (int i = 0; i < kRS; ++i) {
            mbar_init(&sm.r_full[i], 1);
            mbar_init(&sm.r_empty[i], 16);  // each of a quad's 4 chunks is released by the 4 warps of its group
        }
        for (int i = 0; i < kAS; ++i) {
            mbar_init(&sm.a_full[i], 4);  // one group of four warps fills a stage
            mbar_init(&sm.a_empty[i], 1);
        }
        for (int i = 0; i < NBS; ++i) {
            mbar_init(&sm.b_full[i], 1);
            mbar_init(&sm.b_empty[i], 1);
        }
        mbar_init(&sm.done, 1);
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = sm.tmem;

    // The copy and MMA roles run as whole warps (loop state warp-uniform, so the addresses and
    // descriptors stay in uniform registers) and issue from one elected lane.
    if (warp == 0) {
        // weight copies: raw quad qi -> stage qi % kRS
        int rq = 0;  // quads issued
        for (int qi = 0; qi < nquads; ++qi) {
            const int s = qi % kRS;
            if (qi >= kRS && !__all_sync(0xFFFFFFFFu, mbar_wait(&sm.r_empty[s], ((qi / kRS) - 1) & 1, abort, kNap)))
                break;
            if (elect_one()) {
                mbar_expect_tx(&sm.r_full[s], kRNib + kRSc);
                if (GATE) {
                    const int g0 = blockIdx.x * (kTM / 2);
                    tma_load_2d(sm.rnib[s], &tm_nib, (q0 + qi) * 128, g0, &sm.r_full[s]);
                    tma_load_2d(sm.rnib[s] + kRNib / 2, &tm_nib, (q0 + qi) * 128, gate_f + g0, &sm.r_full[s]);
                    tma_load_2d(sm.rsc[s], &tm_sc, (q0 + qi) * 8, g0, &sm.r_full[s]);
                    tma_load_2d(sm.rsc[s] + kRSc / 2, &tm_sc, (q0 + qi) * 8, gate_f + g0, &sm.r_full[s]);
                } else {
                    tma_load_2d(sm.rnib[s], &tm_nib, (q0 + qi) * 128, n0, &sm.r_full[s]);
                    tma_load_2d(sm.rsc[s], &tm_sc, (q0 + qi) * 8, n0, &sm.r_full[s]);
                }
            }
            __syncwarp();
            rq = qi + 1;
        }
        pdl_trigger();
        // the last copy of each stage has landed before the CTA can exit
        for (int qi = std::max(0, rq - kRS); qi < rq; ++qi) mbar_drain(&sm.r_full[qi % kRS], (qi / kRS) & 1);
    } else if (warp == kBWarp) {
        // activation copies: chunk c -> stage c % NBS.  The activations come from the previous
        // kernel of the stream (launched as a programmatic dependent, this kernel may start first)
        pdl_wait();
        const __half* xb = x16 + ((int64_t)mt * nch + 4 * q0) * (NT * kKC);
        const int64_t part_elems = (int64_t)mtiles * NT * K;  // f16 elements per part of x16
        int bc = 0;                                           // chunks issued
        for (int c = 0; c < nchunks; ++c) {
            const int sb = c % NBS;
            if (c >= NBS && !__all_sync(0xFFFFFFFFu, mbar_wait(&sm.b_empty[sb], ((c / NBS) - 1) & 1, abort, kNap)))
                break;
            if (elect_one()) {
                mbar_expect_tx(&sm.b_full[sb], (x_lo ? 2u : 1u) * kBBytes);
                uint8_t* const bh = x_lo ? sm.b[2 * sb] : sm.b[sb];
                bulk_g2s(bh, xb + (int64_t)c * (NT * kKC), kBBytes, &sm.b_full[sb]);
                if (x_lo) bulk_g2s(sm.b[2 * sb + 1], xb + part_elems + (int64_t)c * (NT * kKC), kBBytes, &sm.b_full[sb]);
            }
            __syncwarp();
            bc = c + 1;
        }
        pdl_trigger();
        for (int c = std::max(0, bc - NBS); c < bc; ++c) mbar_drain(&sm.b_full[c % NBS], (c / NBS) & 1);
    } else if (warp == 1) {
        // kStep chunks per round: one round trip waits for all of their A and B stages (lane
        // L polls the A (L even) or B (L odd) stage of chunk c + (L / 2) % kStep), then the
        // round's MMAs go out back to back, since the tensor cores idle whenever this warp does
        // anything else
        const uint32_t idesc = instr_desc_f16(kTM, NT);
        for (int c = 0; c < nchunks; c += kStep) {
            const int nh = min(kStep, nchunks - c);  // chunks of this round
            const int cc = c + (lane >> 1) % kStep;
            const bool need = cc < nchunks;
            uint64_t* const bar = (lane & 1) == 0 ? &sm.a_full[cc % kAS] : &sm.b_full[cc % NBS];
            const uint32_t par = (lane & 1) == 0 ? (uint32_t)(cc / kAS) & 1u : (uint32_t)(cc / NBS) & 1u;
            if (!__all_sync(0xFFFFFFFFu, !need || mbar_wait(bar, par, abort))) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (elect_one()) {
#pragma unroll
                for (int h = 0; h < kStep; ++h) {
                    if (h >= nh) break;
                    const int sa = (c + h) % kAS, sb = (c + h) % NBS;
                    const uint32_t ah = tmem + kACol + sa * kAStageCols, al = ah + 32;
                    const uint32_t bh = smem_u32(x_lo ? sm.b[2 * sb] : sm.b[sb]), bl = smem_u32(sm.b[2 * sb + 1]);
#pragma unroll
                    for (int k16 = 0; k16 < kKC / 16; ++k16) {
                        // A: 8 TMEM columns per K = 16; B: two core matrices along K (LBO 128
                        // bytes, 8-row groups 1024 bytes apart)
                        const uint32_t oa = k16 * 8, ob = k16 * 256;
                        mma_f16_ts(tmem, ah + oa, smem_desc(bh + ob, 128, 1024), idesc,
                                   (c + h > 0 || k16 > 0) ? 1u : 0u);
                        if (x_lo) mma_f16_ts(tmem, ah + oa, smem_desc(bl + ob, 128, 1024), idesc, 1u);
                        mma_f16_ts(tmem, al + oa, smem_desc(bh + ob, 128, 1024), idesc, 1u);
                    }
                }
#pragma unroll
                for (int h = 0; h < kStep; ++h) {
                    if (h >= nh) break;
                    mma_commit(&sm.a_empty[(c + h) % kAS]);
                    mma_commit(&sm.b_empty[(c + h) % NBS]);
                }
            }
            __syncwarp();
        }
        if (elect_one()) mma_commit(&sm.done);  // also on abort: arrives once the MMAs issued so far are done
        __syncwarp();
        pdl_trigger();
    } else if (warp >= 2) {
        // dequantisers: kDqGroups groups of four warps take the chunks in turn (group g the chunks
        // c = g mod kDqGroups);
        // a warp may only reach TMEM lanes 32 (warp % 4) .. +31, so thread -> weight row
        // 32 (warp % 4) + lane, and a thread dequantises the row's whole chunk (2 blocks, 8 words)
        const int grp = (warp - 2) >> 2;
        const int row = 32 * (warp & 3) + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        const uint32_t rsw = (uint32_t)(row & 7);  // the swizzle's XOR for this row
        for (int c = grp; c < nchunks; c += kDqGroups) {
            const int qi = c >> 2, cq = c & 3, s = qi % kRS, sa = c % kAS;
            // lanes 0-15 poll the raw quad, lanes 16-31 the A stage, in one loop
            const bool need = lane < 16 ? true : c >= kAS;
            uint64_t* const bar = lane < 16 ? &sm.r_full[s] : &sm.a_empty[sa];
            const uint32_t par = lane < 16 ? (uint32_t)(qi / kRS) & 1u : (uint32_t)((c / kAS) - 1) & 1u;
            if (!__all_sync(0xFFFFFFFFu, !need || mbar_wait(bar, par, abort, kNap))) break;  // the warp leaves together
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // blocks 2 cq and 2 cq + 1 of the quad; their two scales are adjacent
            const uint8_t* rn = sm.rnib[s] + row * 128;
            const uint4 q0 = *reinterpret_cast<const uint4*>(rn + (((uint32_t)(2 * cq) ^ rsw) << 4));
            const uint4 q1 = *reinterpret_cast<const uint4*>(rn + (((uint32_t)(2 * cq + 1) ^ rsw) << 4));
            const uint32_t sc2 = *reinterpret_cast<const uint32_t*>(sm.rsc[s] + row * 16 + cq * 4);
            // rows past the matrix were zero-filled by the TMA: scale 0 gives zero weights
            const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w}, w1[4] = {q1.x, q1.y, q1.z, q1.w};
            uint32_t h0[16], l0[16], h1[16], l1[16];
            dequant_words<4>(w0, (uint16_t)(sc2 & 0xFFFFu), h0, l0);
            dequant_words<4>(w1, (uint16_t)(sc2 >> 16), h1, l1);
            // the stage's hi part: block 0 in columns 0-15, block 1 in 16-31; its lo part the same + 32
            const uint32_t col = lane_base + kACol + sa * kAStageCols;
            tmem_st(col, h0);
            tmem_st(col + 16, h1);
            tmem_st(col + 32, l0);
            tmem_st(col + 48, l1);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&sm.a_full[sa]);
                mbar_arrive(&sm.r_empty[s]);  // this warp is done with the chunk's rows of the raw quad
            }
        }
        // accumulator -> partial sums (the done barrier completes after the last MMAs)
        pdl_trigger();
        pdl_wait();
        mbar_drain(&sm.done, 0);
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (GATE) {
            // gate rows are tile rows 0..63 (quarters 0 and 1), their value rows 64..127 (quarters 2
            // and 3).  Per 16 columns, the group's value warps hand their sums to its gate warps through
            // shared memory (the raw weight stages are idle now), the gate warps form silu(g) * v, and
            // the group's 128 threads write one 8-element piece of x16_out each.  The group agrees on
            // the abort word first, so that its warps meet the same barriers.
            const int quarter = warp & 3, grp = (warp - 2) >> 2;
            const int trow = quarter * 32 + lane, gt = trow;  // gt: thread of the group, 0..127
            const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
            float* S = reinterpret_cast<float*>(sm.rnib[0]) + grp * (16 * 64);  // [16 columns][64 units]
            const int rows_pad = mtiles * NT;
            if (!bar_any(1 + grp, 128, *abort != 0)) {
                for (int j0 = grp * 16; j0 < NT; j0 += 16 * kDqGroups) {
                    float v[16];
                    tmem_ld16(lane_addr + j0, v);
                    if (quarter >= 2)
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) S[jj * 64 + trow - 64] = v[jj];
                    bar_sync_n(1 + grp, 128);
                    if (quarter < 2)
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) S[jj * 64 + trow] = gated(v[jj], S[jj * 64 + trow]);
                    bar_sync_n(1 + grp, 128);
                    const int jj = gt >> 3, pw = gt & 7;  // column, and piece of the tile's 64 units
                    const int m = mt * NT + j0 + jj;
                    if (m < M) {
                        const float* sp = S + jj * 64 + (pw >> 2) * 32 + 4 * (pw & 3);
                        x16_store_piece(x16_out, NT, rows_pad, gate_f, m, 8 * blockIdx.x + pw,
                                        make_float4(sp[0], sp[1], sp[2], sp[3]),
                                        make_float4(sp[16], sp[17], sp[18], sp[19]), true);
                    }
                    bar_sync_n(1 + grp, 128);
                }
            }
        } else if (__shfl_sync(0xFFFFFFFFu, *abort, 0) == 0) {  // warp-uniform: tcgen05.ld is warp-collective
            const int quarter = warp & 3, grp = (warp - 2) >> 2;  // kDqGroups column groups of 16
            const int trow = quarter * 32 + lane;
            const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
            float* pz = part + (int64_t)z * M * n + n0 + trow;
            const bool row_ok = n0 + trow < n;
#pragma unroll 1
            for (int j0 = grp * 16; j0 < NT; j0 += 16 * kDqGroups) {
                float v[16];
                tmem_ld16(lane_addr + j0, v);
                if (row_ok)
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int m = mt * NT + j0 + jj;
                        if (m < M) pz[(int64_t)m * n] = v[jj];
                    }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (t == 0 && *abort) atomicCAS(err, 0, -5);  // STT_E_DEVICE_FLAG, unless an earlier error is recorded
    __syncwarp();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Launch shape of one product: batch rows per tile, batch tiles, weight-row tiles of 128, K slices.
struct TcPlan {
    int nt, mtiles, tiles, slices;
};

int pick_nt(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }

// K slices: up to one CTA per SM.
TcPlan make_plan(int n, int k, int M, int num_sms) {
    TcPlan p;
    p.nt = pick_nt(M);
    p.mtiles = (M + p.nt - 1) / p.nt;
    p.tiles = (n + kTM - 1) / kTM;
    const int nq = k / kQuad;
    p.slices = std::max(1, std::min(nq, num_sms / std::max(1, p.tiles * p.mtiles)));
    return p;
}

// Gate mode: the descriptors are tw's 64-row ones and x16_out receives silu(gate) * value.
struct TcGate {
    __half* x16_out;
    int f;
};

template <int NT, bool XLO, bool GATE>
cudaError_t launch_nt_x(const TcWeight& tw, const __half* x16, int M, const TcPlan& p, float* part, int* err,
                        const TcGate& gt, cudaStream_t st) {
    const size_t smem = smem_bytes<NT>();
    cudaError_t e =
        cudaFuncSetAttribute(q4_tc_kernel<NT, XLO, GATE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(p.tiles, p.mtiles, p.slices);
    return launch_pdl(q4_tc_kernel<NT, XLO, GATE>, grid, dim3(kThreads), smem, st, GATE ? tw.nib64 : tw.nib,
                      GATE ? tw.sc64 : tw.sc, tw.n, tw.k, x16, M, p.mtiles, p.slices, part, err, gt.x16_out, gt.f);
}

template <int NT>
cudaError_t launch_nt(const TcWeight& tw, const __half* x16, int x_lo, int M, const TcPlan& p, float* part, int* err,
                      const TcGate* gt, cudaStream_t st) {
    const TcGate none{nullptr, 0};
    if (gt) return x_lo ? launch_nt_x<NT, true, true>(tw, x16, M, p, part, err, *gt, st)
                        : launch_nt_x<NT, false, true>(tw, x16, M, p, part, err, *gt, st);
    return x_lo ? launch_nt_x<NT, true, false>(tw, x16, M, p, part, err, none, st)
                : launch_nt_x<NT, false, false>(tw, x16, M, p, part, err, none, st);
}

cudaError_t launch_gemm(const TcWeight& tw, const __half* x16, int x_lo, int M, const TcPlan& p, float* part, int* err,
                        cudaStream_t st, const TcGate* gt = nullptr) {
    switch (p.nt) {
        case 16: return launch_nt<16>(tw, x16, x_lo, M, p, part, err, gt, st);
        case 32: return launch_nt<32>(tw, x16, x_lo, M, p, part, err, gt, st);
        case 64: return launch_nt<64>(tw, x16, x_lo, M, p, part, err, gt, st);
        case 128: return launch_nt<128>(tw, x16, x_lo, M, p, part, err, gt, st);
        default: return launch_nt<256>(tw, x16, x_lo, M, p, part, err, gt, st);
    }
}

// Four consecutive input elements k .. k+3 of a row (f32 rows are 16-byte aligned: K % 256 == 0).
__device__ __forceinline__ float4 load4(const float* __restrict__ in, const __nv_bfloat16* __restrict__ in_bf16,
                                        const __half* __restrict__ in_f16, int64_t k) {
    if (in_f16)
        return make_float4(__half2float(in_f16[k]), __half2float(in_f16[k + 1]), __half2float(in_f16[k + 2]),
                           __half2float(in_f16[k + 3]));
    if (in_bf16)
        return make_float4(__bfloat162float(in_bf16[k]), __bfloat162float(in_bf16[k + 1]),
                           __bfloat162float(in_bf16[k + 2]), __bfloat162float(in_bf16[k + 3]));
    return *reinterpret_cast<const float4*>(in + k);
}

// Sum of squares of row[0 .. K) (K % 4 == 0), the same in every thread of the CTA: float4
// loads, per-thread sums in order x, y, z, w, then warp and CTA sums.
__device__ __forceinline__ float row_sumsq(const float* __restrict__ row, int K, float* red) {
    float ss = 0.0f;
    for (int j = threadIdx.x; j < K / 4; j += blockDim.x) {
        const float4 v = *reinterpret_cast<const float4*>(row + 4 * j);
        ss = __fmaf_rn(v.x, v.x, ss);
        ss = __fmaf_rn(v.y, v.y, ss);
        ss = __fmaf_rn(v.z, v.z, ss);
        ss = __fmaf_rn(v.w, v.w, ss);
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
    return red[0];
}

// RMSNorm of a row: x / rms * alpha, rms = sqrt(mean(x^2) + 1e-8) (burn::nn::RmsNorm behind
// RmsNormLayer::forward, model.rs:369-373; the GEMV's prologue computes the same).
__device__ __forceinline__ float4 rms_scale(float4 v, float rms, const float* __restrict__ alpha, int k) {
    const float4 g = *reinterpret_cast<const float4*>(alpha + k);
    return make_float4(__fmul_rn(__fdiv_rn(v.x, rms), g.x), __fmul_rn(__fdiv_rn(v.y, rms), g.y),
                       __fmul_rn(__fdiv_rn(v.z, rms), g.z), __fmul_rn(__fdiv_rn(v.w, rms), g.w));
}

// f16 GEMM input of a batch (x16, layout in tc_layout.cuh).  Grid: (padded batch rows, groups of
// 256 pieces); a thread writes one piece.  Row m < M is row m of `in` (f32, bf16 when in_bf16, f16
// when in_f16), RMSNorm'd when alpha is not NULL; rows >= M are zero.  Writes the hi parts and,
// when lo != 0, the lo parts.
__global__ void __launch_bounds__(256) prep_f16_kernel(const float* __restrict__ in, const __nv_bfloat16* __restrict__ in_bf16,
                                                       const __half* __restrict__ in_f16, const float* __restrict__ alpha,
                                                       int K, int M, int nt, int lo, __half* __restrict__ out) {
    __shared__ float red[32];
    const int m = blockIdx.x;
    const int64_t base = (int64_t)m * K;
    const float rms = alpha && m < M ? sqrtf(__fadd_rn(__fdiv_rn(row_sumsq(in + base, K, red), (float)K), 1e-8f)) : 1.0f;
    const int pi = blockIdx.y * blockDim.x + threadIdx.x;
    if (pi >= K / 8) return;
    const int k0 = piece_k0(pi);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (m < M) {
        a = load4(in, in_bf16, in_f16, base + k0);
        b = load4(in, in_bf16, in_f16, base + k0 + 16);
        if (alpha) {
            a = rms_scale(a, rms, alpha, k0);
            b = rms_scale(b, rms, alpha, k0 + 16);
        }
    }
    x16_store_piece(out, nt, gridDim.x, K, m, pi, a, b, lo != 0);
}

// Residual epilogue fused with the next product's input: one CTA per batch row m.
// x[m] += sum over slices of part[z][m] (slices added in order, then the residual, as the GEMV's
// residual epilogue does), then x16 row m = RMSNorm(x[m]) * alpha, hi and lo parts.
__global__ void __launch_bounds__(512) resid_norm_kernel(float* __restrict__ x, const float* __restrict__ part, int slices,
                                                         int rows, int D, const float* __restrict__ alpha,
                                                         __half* __restrict__ x16, int nt, int rows_pad) {
    extern __shared__ float4 vrow[];  // the updated row
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    float4* xr = reinterpret_cast<float4*>(x + (int64_t)m * D);
    const float* pm = part + (int64_t)m * D;
    const int64_t plane = (int64_t)rows * D;
    for (int j = threadIdx.x; j < D / 4; j += blockDim.x) {
        float4 sum = reinterpret_cast<const float4*>(pm)[j];
        // slices 1 .. in groups of 4 loads issued together, added in slice order
        for (int z0 = 1; z0 < slices; z0 += 4) {
            float4 p[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (z0 + u < slices) p[u] = reinterpret_cast<const float4*>(pm + (z0 + u) * plane)[j];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (z0 + u < slices)
                    sum = make_float4(__fadd_rn(sum.x, p[u].x), __fadd_rn(sum.y, p[u].y), __fadd_rn(sum.z, p[u].z),
                                      __fadd_rn(sum.w, p[u].w));
        }
        const float4 o = xr[j];
        const float4 v = make_float4(__fadd_rn(sum.x, o.x), __fadd_rn(sum.y, o.y), __fadd_rn(sum.z, o.z), __fadd_rn(sum.w, o.w));
        xr[j] = v;
        vrow[j] = v;
    }
    __syncthreads();
    const float rms = sqrtf(__fadd_rn(__fdiv_rn(row_sumsq(reinterpret_cast<const float*>(vrow), D, red), (float)D), 1e-8f));
    for (int pi = threadIdx.x; pi < D / 8; pi += blockDim.x) {
        const int k0 = piece_k0(pi);
        x16_store_piece(x16, nt, rows_pad, D, m, pi, rms_scale(vrow[k0 / 4], rms, alpha, k0),
                        rms_scale(vrow[k0 / 4 + 4], rms, alpha, k0 + 16), true);
    }
}

// Gate epilogue fused with the next product's input: part[z][m][0 .. 2F) holds the gate rows
// (0 .. F) and value rows (F .. 2F) of linear_in; x16 row m = silu(gate) * value, hi and lo parts.
// A thread writes one piece of one row.
__global__ void __launch_bounds__(256) gate_kernel(const float* __restrict__ part, int slices, int rows, int F,
                                                   __half* __restrict__ x16, int nt, int rows_pad) {
    pdl_trigger();
    pdl_wait();
    const int npieces = F / 8;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * npieces) return;
    const int m = idx / npieces, pi = idx - m * npieces;
    const int k0 = piece_k0(pi);
    const int64_t plane = (int64_t)rows * 2 * F;
    const float* pm = part + (int64_t)m * 2 * F;
    float4 r[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int k = k0 + 16 * hh;
        float4 g = *reinterpret_cast<const float4*>(pm + k), v = *reinterpret_cast<const float4*>(pm + F + k);
        for (int z = 1; z < slices; ++z) {
            const float4 gz = *reinterpret_cast<const float4*>(pm + z * plane + k);
            const float4 vz = *reinterpret_cast<const float4*>(pm + z * plane + F + k);
            g = make_float4(__fadd_rn(g.x, gz.x), __fadd_rn(g.y, gz.y), __fadd_rn(g.z, gz.z), __fadd_rn(g.w, gz.w));
            v = make_float4(__fadd_rn(v.x, vz.x), __fadd_rn(v.y, vz.y), __fadd_rn(v.z, vz.z), __fadd_rn(v.w, vz.w));
        }
        r[hh] = make_float4(gated(g.x, v.x), gated(g.y, v.y), gated(g.z, v.z), gated(g.w, v.w));
    }
    x16_store_piece(x16, nt, rows_pad, F, m, pi, r[0], r[1], true);
}

cudaError_t launch_prep(const float* in, const __nv_bfloat16* in_bf16, const __half* in_f16, const float* alpha, int K,
                        int M, const TcPlan& p, int lo, __half* x16, cudaStream_t st) {
    dim3 grid(p.mtiles * p.nt, (K / 8 + 255) / 256);
    prep_f16_kernel<<<grid, 256, 0, st>>>(in, in_bf16, in_f16, alpha, K, M, p.nt, lo, x16);
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

cudaError_t tma_encode(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank, const uint64_t* dims,
                       const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
    // The driver's encoder, looked up once; a function-local static is initialised exactly once
    // even when threads load models on several devices at the same time.
    struct EncodeFn {
        PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
        cudaError_t err = cudaSuccess;
    };
    static const EncodeFn lookup = [] {
        EncodeFn r;
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        r.err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (r.err == cudaSuccess && (q != cudaDriverEntryPointSuccess || !fn)) r.err = cudaErrorNotSupported;
        if (r.err == cudaSuccess) r.fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        return r;
    }();
    if (lookup.err != cudaSuccess) return lookup.err;
    if (rank < 1 || rank > 5) return cudaErrorInvalidValue;
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides[i];
    }
    if (lookup.fn(map, type, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    return cudaSuccess;
}

cudaError_t tma_encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner,
                          uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                          CUtensorMapSwizzle swizzle) {
    const uint64_t dims[2] = {inner, rows};
    const uint32_t box[2] = {box_inner, box_rows};
    return tma_encode(map, type, base, 2, dims, &row_bytes, box, swizzle);
}

cudaError_t tc_make_weight(const Q4Dev& w, TcWeight* out) {
    const uint64_t nb = (uint64_t)(w.k / 32);
    // nibble plane: [n rows][k/32 * 16 bytes]; a box is one quad (128 bytes) of 128 rows
    cudaError_t e = tma_encode_2d(&out->nib, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.nib, nb * 16, (uint64_t)w.n, nb * 16,
                                  128, (uint32_t)kTM, CU_TENSOR_MAP_SWIZZLE_128B);
    // scale plane: [n rows][k/32 scales]; a box is one quad (8 scales, 16 bytes) of 128 rows
    if (e == cudaSuccess)
        e = tma_encode_2d(&out->sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.scale, nb, (uint64_t)w.n, nb * 2, 8,
                          (uint32_t)kTM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (e != cudaSuccess) return e;
    out->n = w.n;
    out->k = w.k;
    out->gate_ok = false;
    return cudaSuccess;
}

cudaError_t tc_make_gate_maps(const Q4Dev& w, TcWeight* out) {
    out->gate_ok = false;
    if (w.n % 128 != 0) return cudaSuccess;  // gate and value halves of 64-row multiples
    const uint64_t nb = (uint64_t)(w.k / 32);
    cudaError_t e = tma_encode_2d(&out->nib64, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.nib, nb * 16, (uint64_t)w.n, nb * 16,
                                  128, (uint32_t)(kTM / 2), CU_TENSOR_MAP_SWIZZLE_128B);
    if (e == cudaSuccess)
        e = tma_encode_2d(&out->sc64, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.scale, nb, (uint64_t)w.n, nb * 2, 8,
                          (uint32_t)(kTM / 2), CU_TENSOR_MAP_SWIZZLE_NONE);
    out->gate_ok = e == cudaSuccess;
    return e;
}

size_t tc_x16_bytes(int k, int M) {
    const TcPlan p = make_plan(1, k, M, 1);
    return 2 * (size_t)p.mtiles * p.nt * k * sizeof(__half);
}

size_t tc_part_bytes(const Q4Dev& w, int M, int num_sms) {
    const TcPlan p = make_plan(w.n, w.k, M, num_sms);
    return (size_t)p.slices * M * w.n * sizeof(float);
}

cudaError_t launch_q4_tc_gemm(const TcWeight& tw, const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo,
                              __half* x16, float* part, int* err, int num_sms, cudaStream_t st) {
    const TcPlan p = make_plan(w.n, w.k, M, num_sms);
    cudaError_t e = launch_prep(nullptr, nullptr, x, nullptr, w.k, M, p, 0, x16, st);
    if (e != cudaSuccess) return e;
    e = launch_gemm(tw, x16, 0, M, p, part, err, st);
    if (e != cudaSuccess) return e;
    GemvArgs a{};
    a.W = w;
    a.out = out;
    a.ldo = ldo;
    a.n_units = (w.n + 1) / 2;
    return launch_tc_epilogue(Ctx{}, a, EPI_PLAIN, M, part, p.slices, st);
}

void tc_batch_tiles(int rows, int* nt, int* rows_pad) {
    const TcPlan p = make_plan(1, kQuad, rows, 1);
    *nt = p.nt;
    *rows_pad = p.mtiles * p.nt;
}

cudaError_t launch_tc_prep(const float* in, const float* alpha, int K, int rows, __half* x16, cudaStream_t st) {
    return launch_prep(in, nullptr, nullptr, alpha, K, rows, make_plan(1, K, rows, 1), 1, x16, st);
}

cudaError_t launch_tc_product(const TcWeight& tw, const __half* x16, int rows, float* part, int* err, int num_sms,
                              int* slices, cudaStream_t st, bool x_lo) {
    const TcPlan p = make_plan(tw.n, tw.k, rows, num_sms);
    *slices = p.slices;
    return launch_gemm(tw, x16, x_lo ? 1 : 0, rows, p, part, err, st);
}

cudaError_t launch_tc_product_gate(const TcWeight& tw, const __half* x16, int rows, __half* x16_out, int* err,
                                   cudaStream_t st, bool x_lo) {
    if (!tw.gate_ok) return cudaErrorInvalidValue;
    TcPlan p = make_plan(tw.n, tw.k, rows, 1);
    p.slices = 1;  // the epilogue needs each unit's whole sum
    const TcGate gt{x16_out, tw.n / 2};
    return launch_gemm(tw, x16, x_lo ? 1 : 0, rows, p, nullptr, err, st, &gt);
}

cudaError_t launch_tc_resid_norm(float* x, const float* part, int slices, int rows, int D, const float* alpha,
                                 __half* x16, cudaStream_t st) {
    int nt, rows_pad;
    tc_batch_tiles(rows, &nt, &rows_pad);
    return launch_pdl(resid_norm_kernel, dim3(rows), dim3(512), (size_t)D * sizeof(float), st, x, part, slices, rows, D,
                      alpha, x16, nt, rows_pad);
}

cudaError_t launch_tc_gate(const float* part, int slices, int rows, int F, __half* x16, cudaStream_t st) {
    int nt, rows_pad;
    tc_batch_tiles(rows, &nt, &rows_pad);
    const int total = rows * (F / 8);
    return launch_pdl(gate_kernel, dim3((total + 255) / 256), dim3(256), 0, st, part, slices, rows, F, x16, nt, rows_pad);
}

}  // namespace stt
