// Persistent single-stream decode step for sm_100a.
//
// One cooperative launch of one 512-thread CTA per SM runs `steps` whole frames of one stream:
//   per layer   QKV -> attention -> out_proj -> linear_in -> linear_out, a grid barrier after each
//   per frame   head GEMV + per-CTA argmax -> barrier -> every CTA reduces the argmax, applies the
//               stream rule, and builds the next frame's input from the audio-embedding sum
//               (computed in the head phase) plus the text row.
// A single stream reads 627 MB of Q4_0 weights per frame but each phase is a few MB, so the
// design is about keeping the dependent chain of 81 phases short while HBM keeps streaming:
//   - every CTA owns fixed row ranges of every matrix.  Right after a phase's GEMV, before the
//     grid barrier, one thread bulk-copies (cp.async.bulk + mbarrier) the CTA's rows of the
//     NEXT phase into shared memory, so after the barrier only the activation vector has to be
//     fetched; the same thread issues cp.async.bulk.prefetch.L2 for the phases beyond, keeping
//     a byte budget of look-ahead in flight so HBM never idles during barriers;
//   - the GEMV reads weights from shared memory at about 1.5 instructions per weight: the input
//     vector becomes 24-bit fixed point per 32-element block (three byte limbs, shared
//     exponent) and every nibble goes through dp4a, so each block's dot product is exact;
//   - the grid barrier is a release add + acquire poll on one counter;
//   - every wait is bounded: a timed-out barrier or copy raises STT_E_DEVICE_FLAG in the step
//     descriptor, sets an abort word that releases the other CTAs, waits (bounded) for its own
//     copies in flight, and returns.
#include <algorithm>
#include <cfloat>
#include <cstdlib>

#include "kernels.h"
#include "mega.h"

namespace stt {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kNBMax = 264;                // K / 32 for K <= 8448
constexpr int kMaxK = kNBMax * 32;
constexpr int kWBuf = 144 * 1024;          // staged weight rows of one phase per CTA
constexpr int kMaxL = 32;                  // layers held in the shared layer table
constexpr int kMaxOwnRows = 256;           // rows of x one CTA owns (out_proj / linear_out rows)
constexpr int kQMax = (kMaxK / 4 + kThreads - 1) / kThreads;  // input quads per thread
constexpr uint32_t kSpinLimit = 1u << 26;  // bounded waits (~ seconds)

struct MegaArgs {
    Ctx c;
    int32_t steps;
    int32_t nsplit;        // attention splits per head
    uint32_t* bar;         // [0] arrivals (monotonic), [1] abort, [2..2+H) head tickets
    const float* xa;       // [steps][D] audio-embedding sums of every frame (audio_sum_kernel)
    float* amax_v;         // [grid] per-CTA best logit
    int32_t* amax_i;       // [grid] and its index
    uint32_t pf_budget;    // L2 look-ahead per CTA in bytes
    int32_t pf_lines;      // 1: warp 0 prefetches 128-byte lines; 0: bulk prefetch (TMA queue)
    unsigned long long* trace;  // optional: %globaltimer at each barrier of one frame
    int32_t trace_frame;
    int32_t trace_cap;
};

struct Smem {
    alignas(128) uint8_t wbuf[kWBuf];  // this CTA's weight rows of the current phase
    uint4 limbs[6 * kNBMax];           // [vec][block]: L0,L1,L2 of groups 0-3, then of groups 4-7
    float xs[kNBMax];                  // 2^(e_b - 27): block scale of the fixed-point input
    float xf[kMaxK];                   // the input vector in f32 / attention scratch
    LayerDev layers[kMaxL];
    float xown[kMaxOwnRows];           // this CTA's rows of the residual stream x
    float2 rope[64];                   // (cos, sin) of this frame's position, HD / 2 pairs
    float red[2][kWarps];
    float wv[kWarps];
    int32_t wi[kWarps];
    alignas(8) unsigned long long mbar;
    uint32_t staged, waited;  // staged copies issued / waited for (thread 0's bookkeeping)
    int32_t flag;
};

// The kernel's dynamic shared memory.  Functions that are not inlined recover the Smem through
// this file-scope array instead of a reference parameter, so the compiler keeps emitting
// shared-memory (LDS/STS) accesses rather than generic ones.
extern __shared__ __align__(128) uint4 mega_smem[];
__device__ __forceinline__ Smem& smem_ref() { return *reinterpret_cast<Smem*>(mega_smem); }

// ------------------------------------------------------------------------------ primitives

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_line(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
// Called by all 32 lanes of warp 0: bulk prefetch by lane 0, or line prefetches spread over lanes.
__device__ __forceinline__ void prefetch_range(const void* p, uint32_t bytes, bool lines, int lane) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    if (lines) {
        for (uint32_t o = (uint32_t)lane * 128u; o < bytes; o += 32u * 128u) prefetch_line(b + o);
    } else if (lane == 0) {
        for (uint32_t o = 0; o < bytes; o += 65536u) prefetch_l2(b + o, min(65536u, bytes - o));
    }
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long* m, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(m)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* m, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(m)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* m, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(m)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, unsigned long long* m) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(m))
        : "memory");
}
__device__ __forceinline__ int dp4a_su(int a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(int a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// exact int -> float for |v| < 2^22
__device__ __forceinline__ float i2f(int v) { return __int_as_float(0x4B400000 + v) - 12582912.0f; }

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Trace points of one frame of CTA 0: (tag, SM clock cycles) pairs, bracketed by (0, %globaltimer)
// pairs at the frame's start and end so the host can convert cycles to time.  Tags: 1 frame start,
// 2 barrier entry, 3 barrier exit, 10*k + {0 prologue done, 1 staged copy landed, 2 compute done}
// for phase kinds k = 1 qkv, 2 attention, 3 out_proj, 4 linear_in, 5 linear_out, 6 head.
struct Tracer {
    int slot = 0;
    bool on = false;
    __device__ void mark(const MegaArgs& P, unsigned long long tag) {
        if (on && threadIdx.x == 0 && slot + 1 < P.trace_cap) {
            P.trace[slot] = tag;
            P.trace[slot + 1] = clock64();
            slot += 2;
        }
    }
    // (tag 0, %globaltimer) pair: lets the host convert the cycle counts to nanoseconds
    __device__ void wall(const MegaArgs& P) {
        if (on && threadIdx.x == 0 && slot + 1 < P.trace_cap) {
            P.trace[slot] = 0;
            P.trace[slot + 1] = globaltimer();
            slot += 2;
        }
    }
};

__device__ __forceinline__ int64_t split_lo(int64_t total, int part, int parts) { return total * part / parts; }

// Grid barrier.  Returns false when the kernel must stop (a timeout here or in another CTA).
__device__ bool grid_sync(const MegaArgs& P, uint32_t& epoch, Smem& sm, Tracer& tr) {
    __syncthreads();
    tr.mark(P, 2);
    ++epoch;
    if (threadIdx.x == 0) {
        const uint32_t target = epoch * gridDim.x;
        red_release_add(P.bar, 1u);  // release: this CTA's writes, ordered by the barrier above
        int ok = 1;
        uint32_t spins = 0;
        for (;;) {
            if ((int32_t)(ld_acquire(P.bar) - target) >= 0) break;
            if (*(volatile uint32_t*)(P.bar + 1)) {
                ok = 0;
                break;
            }
            if (++spins > kSpinLimit) {
                atomicExch(P.bar + 1, 1u);
                raise_error(P.c.desc, -5);
                ok = 0;
                break;
            }
            if (spins > 2048) __nanosleep(32);
        }
        sm.flag = ok;
    }
    __syncthreads();
    tr.mark(P, 3);
    return sm.flag != 0;
}

// ------------------------------------------------------------------------------ phase geometry

enum Kind : int { K_QKV = 0, K_ATT = 1, K_OUT = 2, K_IN = 3, K_DOWN = 4, K_HEAD = 5 };

// The rows of one phase this CTA reads: one or two contiguous row ranges of one matrix.
struct Rows {
    const Q4Dev* W;
    int32_t r0[2];
    int32_t n[2];
    int32_t nr;  // number of ranges
};

__device__ __forceinline__ Kind kind_of(int p, int L) { return p == 5 * L ? K_HEAD : (Kind)(p % 5); }

__device__ Rows rows_of(const Smem& sm, const Ctx& c, int p, int cta, int ncta) {
    Rows r{};
    const Kind k = kind_of(p, c.L);
    if (k == K_HEAD) {
        const int64_t U = (c.V + 1) / 2;
        const int64_t a = 2 * split_lo(U, cta, ncta), b = min((int64_t)c.V, 2 * split_lo(U, cta + 1, ncta));
        r.W = &c.head;
        r.r0[0] = (int)a;
        r.n[0] = (int)max((int64_t)0, b - a);
        r.nr = 1;
        return r;
    }
    const LayerDev& L = sm.layers[p / 5];
    switch (k) {
        case K_QKV:
        case K_OUT:
        case K_DOWN: {
            const Q4Dev* W = k == K_QKV ? &L.qkv : (k == K_OUT ? &L.out : &L.fout);
            const int64_t U = W->n / 2;
            r.W = W;
            r.r0[0] = (int)(2 * split_lo(U, cta, ncta));
            r.n[0] = (int)(2 * split_lo(U, cta + 1, ncta)) - r.r0[0];
            r.nr = 1;
            break;
        }
        case K_IN: {
            const int u0 = (int)split_lo(c.F, cta, ncta), u1 = (int)split_lo(c.F, cta + 1, ncta);
            r.W = &L.fin;
            r.r0[0] = u0;
            r.r0[1] = c.F + u0;
            r.n[0] = r.n[1] = u1 - u0;
            r.nr = 2;
            break;
        }
        default:
            r.nr = 0;
            break;
    }
    return r;
}

// Shared-memory layout of a staged phase: for each range, nibbles then scales (16-byte aligned),
// then the phase's norm weight (D floats) when it has one.
struct Staged {
    uint32_t nib[2];
    uint32_t sc[2];
    uint32_t alpha;  // offset of the norm weight, or ~0u
    uint32_t bytes;
};

// The norm weight applied to a phase's input: norm1 (QKV), norm2 (linear_in), out_norm (head).
__device__ __forceinline__ const float* phase_alpha(const Smem& sm, const Ctx& c, int p) {
    const Kind k = kind_of(p, c.L);
    if (k == K_HEAD) return c.out_norm;
    if (k == K_QKV) return sm.layers[p / 5].norm1;
    if (k == K_IN) return sm.layers[p / 5].norm2;
    return nullptr;
}

__device__ __forceinline__ Staged staged_layout(const Rows& r, bool alpha, int D) {
    Staged s{};
    uint32_t off = 0;
    const uint32_t NB = r.nr ? (uint32_t)(r.W->k >> 5) : 0;
    for (int i = 0; i < r.nr; ++i) {
        s.nib[i] = off;
        off += (uint32_t)r.n[i] * NB * 16;
        s.sc[i] = off;
        off += ((uint32_t)r.n[i] * NB * 2 + 15) & ~15u;
    }
    s.alpha = ~0u;
    if (alpha) {
        s.alpha = off;
        off += (uint32_t)D * 4;
    }
    s.bytes = off;
    return s;
}

// Slots [j0, j1) of the attention split handled by this CTA (empty when h >= H).
struct Split {
    int h, s, j0, j1;
};
__device__ __forceinline__ Split split_of(const MegaArgs& P, int cta, int len) {
    Split r;
    r.h = cta / P.nsplit;
    r.s = cta % P.nsplit;
    const int chunk = (len + P.nsplit - 1) / P.nsplit;
    r.j0 = r.s * chunk;
    r.j1 = r.h < P.c.H ? min(len, r.j0 + chunk) : r.j0;
    if (r.j1 < r.j0) r.j1 = r.j0;
    return r;
}

// wbuf offset of the staged K/V slots: after the out_proj rows, which are staged with them.
__device__ __forceinline__ uint32_t kv_offset(const Smem& sm, const Ctx& c, int layer, int cta, int ncta) {
    const Staged so = staged_layout(rows_of(sm, c, 5 * layer + K_OUT, cta, ncta), false, c.D);
    return (so.bytes + 127u) & ~127u;
}

// Bytes a phase reads from HBM for this CTA (weights, or the K/V slots of its attention split).
__device__ uint32_t phase_bytes(const Smem& sm, const MegaArgs& P, int p, int cta, int ncta, int len) {
    const Ctx& c = P.c;
    if (kind_of(p, c.L) == K_ATT) {
        const int h = cta / P.nsplit, s = cta % P.nsplit;
        if (h >= c.H) return 0;
        const int chunk = (len + P.nsplit - 1) / P.nsplit;
        const int j0 = s * chunk, j1 = min(len, j0 + chunk);
        return j1 > j0 ? (uint32_t)(j1 - j0) * c.HD * 2 * (c.kv_f32 ? 4 : 2) : 0u;
    }
    const Rows r = rows_of(sm, c, p, cta, ncta);
    uint32_t b = 0;
    for (int i = 0; i < r.nr; ++i) b += (uint32_t)r.n[i] * (uint32_t)(r.W->k >> 5) * 18u;
    return b;
}

// L2 prefetch of one phase's ranges (all lanes of warp 0).
__device__ void prefetch_phase(const Smem& sm, const MegaArgs& P, int p, int cta, int ncta, int len, int lane) {
    const Ctx& c = P.c;
    const bool lines = P.pf_lines != 0;
    if (kind_of(p, c.L) == K_ATT) {
        const int h = cta / P.nsplit, s = cta % P.nsplit;
        if (h >= c.H) return;
        const int chunk = (len + P.nsplit - 1) / P.nsplit;
        const int j0 = s * chunk, j1 = min(len, j0 + chunk);
        if (j1 <= j0) return;
        const int es = c.kv_f32 ? 4 : 2;
        const uint8_t* kb = static_cast<const uint8_t*>(c.kv) +
                            ((int64_t)c.ids[0] * c.kv_stream_stride + (int64_t)(p / 5) * c.kv_layer_stride +
                             (int64_t)h * c.ML * c.HD + (int64_t)j0 * c.HD) * es;
        const uint32_t bytes = (uint32_t)(j1 - j0) * c.HD * es;
        prefetch_range(kb, bytes, lines, lane);
        prefetch_range(kb + c.kv_half_stride * es, bytes, lines, lane);
        return;
    }
    const Rows r = rows_of(sm, c, p, cta, ncta);
    for (int i = 0; i < r.nr; ++i) {
        if (r.n[i] <= 0) continue;
        const int64_t NB = r.W->k >> 5;
        prefetch_range(r.W->nib + (int64_t)r.r0[i] * NB, (uint32_t)(r.n[i] * NB * 16), lines, lane);
        const uint32_t sbytes = (uint32_t)(r.n[i] * NB * 2) & ~15u;
        if (sbytes) prefetch_range(r.W->scale + (int64_t)r.r0[i] * NB, sbytes, lines, lane);
    }
}

// Bulk copy of one row range's nibbles and scales into wbuf (thread 0).
__device__ __forceinline__ void stage_rows(Smem& sm, const Q4Dev* W, int r0, int n, uint32_t nib_off, uint32_t sc_off) {
    if (n <= 0) return;
    const int64_t NB = W->k >> 5;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(W->nib + (int64_t)r0 * NB);
    const uint32_t nbytes = (uint32_t)(n * NB * 16);
    for (uint32_t o = 0; o < nbytes; o += 32768u)
        bulk_g2s(sm.wbuf + nib_off + o, src + o, min(32768u, nbytes - o), &sm.mbar);
    const uint32_t sbytes = (uint32_t)(n * NB * 2);
    const uint32_t sfull = sbytes & ~15u;
    if (sfull) bulk_g2s(sm.wbuf + sc_off, W->scale + (int64_t)r0 * NB, sfull, &sm.mbar);
    if (sbytes != sfull) {
        // scale bytes not a multiple of 16: the tail is copied by this thread; the consumers
        // read it after the barrier that publishes the bulk copies
        const uint16_t* tail = W->scale + (int64_t)r0 * NB + sfull / 2;
        uint16_t* dst = reinterpret_cast<uint16_t*>(sm.wbuf + sc_off + sfull);
        for (uint32_t t = 0; t < (sbytes - sfull) / 2; ++t) dst[t] = tail[t];
    }
}

__device__ __forceinline__ uint32_t rows_tx(const Rows& r) {
    uint32_t tx = 0;
    for (int i = 0; i < r.nr; ++i)
        if (r.n[i] > 0) {
            const uint32_t NB = (uint32_t)(r.W->k >> 5);
            tx += (uint32_t)r.n[i] * NB * 16u + (((uint32_t)r.n[i] * NB * 2u) & ~15u);
        }
    return tx;
}

// Thread 0: bulk-copies phase p's rows of this CTA (and its norm weight) into wbuf; completion on
// sm.mbar.  No proxy fence is needed before overwriting wbuf: it was only read by the generic
// proxy, and every reader passed the __syncthreads that precedes this call.
__device__ void stage_phase(Smem& sm, const Ctx& c, int p, int cta, int ncta) {
    const Rows r = rows_of(sm, c, p, cta, ncta);
    const float* alpha = phase_alpha(sm, c, p);
    const Staged s = staged_layout(r, alpha != nullptr, c.D);
    ++sm.staged;
    mbar_expect_tx(&sm.mbar, rows_tx(r) + (alpha ? (uint32_t)c.D * 4u : 0u));
    for (int i = 0; i < r.nr; ++i) stage_rows(sm, r.W, r.r0[i], r.n[i], s.nib[i], s.sc[i]);
    if (alpha) bulk_g2s(sm.wbuf + s.alpha, alpha, (uint32_t)c.D * 4u, &sm.mbar);
}

// Thread 0, after the QKV GEMV of layer l: stages the out_proj rows and this CTA's K/V slots of
// layer l (as of the previous frames: the slot written this frame is read from qkv instead).
__device__ void stage_out_kv(Smem& sm, const MegaArgs& P, int l, int cta, int ncta, int len) {
    const Ctx& c = P.c;
    const Rows r = rows_of(sm, c, 5 * l + K_OUT, cta, ncta);
    const Staged s = staged_layout(r, false, c.D);
    const Split sp = split_of(P, cta, len);
    const int es = c.kv_f32 ? 4 : 2;
    const uint32_t kvb = (uint32_t)(sp.j1 - sp.j0) * c.HD * es;
    const uint32_t koff = kv_offset(sm, c, l, cta, ncta);
    ++sm.staged;
    mbar_expect_tx(&sm.mbar, rows_tx(r) + 2u * kvb);
    stage_rows(sm, r.W, r.r0[0], r.n[0], s.nib[0], s.sc[0]);
    if (kvb) {
        const uint8_t* kb = static_cast<const uint8_t*>(c.kv) +
                            ((int64_t)c.ids[0] * c.kv_stream_stride + (int64_t)l * c.kv_layer_stride +
                             (int64_t)sp.h * c.ML * c.HD + (int64_t)sp.j0 * c.HD) * es;
        for (uint32_t o = 0; o < kvb; o += 32768u) {
            bulk_g2s(sm.wbuf + koff + o, kb + o, min(32768u, kvb - o), &sm.mbar);
            bulk_g2s(sm.wbuf + koff + kvb + o, kb + c.kv_half_stride * es + o, min(32768u, kvb - o), &sm.mbar);
        }
    }
}

// Waits (bounded) for the staged copy of the current phase; the parity flips per staging.
__device__ bool wait_stage(Smem& sm, const MegaArgs& P, uint32_t& parity) {
    if (threadIdx.x == 0) {
        int ok = 1;
        uint32_t spins = 0;
        while (!mbar_try_wait(&sm.mbar, parity)) {
            if (++spins > kSpinLimit || *(volatile uint32_t*)(P.bar + 1)) {
                if (!*(volatile uint32_t*)(P.bar + 1)) raise_error(P.c.desc, -5);
                atomicExch(P.bar + 1, 1u);
                ok = 0;
                break;
            }
        }
        if (ok) ++sm.waited;
        sm.flag = ok;
    }
    __syncthreads();
    const bool ok = sm.flag != 0;
    if (ok) parity ^= 1u;
    return ok;
}

// ------------------------------------------------------------------------------ input vectors

// dp4a limbs of one quad (elements 4q .. 4q+3) of block b = q / 8; called by all 32 lanes of a
// warp with 8 consecutive lanes holding the 8 quads of a block.
__device__ __forceinline__ void quad_limbs(Smem& sm, int q, int NB, float4 v) {
    const int b = q >> 3, g = q & 7;
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 4));
    // max < 2^e with e = biased exponent - 126; scale the block by 2^(23 - e)
    int e = m > 0.0f ? (int)((__float_as_uint(m) >> 23) & 0xFF) - 126 : 0;
    e = max(-96, min(e, 120));
    const float up = __uint_as_float((uint32_t)(127 + 23 - e) << 23);
    const float vals[4] = {v.x, v.y, v.z, v.w};
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int X = __float2int_rn(vals[i] * up);
        X = max(-(1 << 23), min(X, (1 << 23) - 1));
        w0 |= (uint32_t)(X & 0xFF) << (8 * i);
        w1 |= (uint32_t)((X >> 8) & 0xFF) << (8 * i);
        w2 |= (uint32_t)((X >> 16) & 0xFF) << (8 * i);
    }
    uint32_t* L = reinterpret_cast<uint32_t*>(sm.limbs);
    const int base = g < 4 ? 0 : 3;
    L[((base + 0) * NB + b) * 4 + (g & 3)] = w0;
    L[((base + 1) * NB + b) * 4 + (g & 3)] = w1;
    L[((base + 2) * NB + b) * 4 + (g & 3)] = w2;
    if (g == 0) sm.xs[b] = __uint_as_float((uint32_t)(127 + e - 27) << 23);
}

// Block sum in a fixed order with one __syncthreads; `rb` alternates the two scratch rows so
// back-to-back reductions need no second barrier.
__device__ __forceinline__ float block_sum(float v, Smem& sm, uint32_t& rb) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sm.red[rb][warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += sm.red[rb][w];
    rb ^= 1u;
    return s;
}

// The GEMV input of a phase: K floats from `src` (global, read through L2) or, when src is NULL,
// from xf; RMSNorm with `alpha` when NORM (burn::nn::RmsNorm: (x / sqrt(mean(x^2) + 1e-8)) *
// alpha); then the dp4a limbs.  QN = quads per thread; a thread's x and alpha loads are all in
// flight together.
template <int QN, bool NORM>
__device__ __noinline__ void prep_vector_t(Smem& /*sm_param*/, const float* src, int K, const float* alpha, uint32_t& rb) {
    Smem& sm = smem_ref();
    const int nq = K >> 2, NB = K >> 5;
    float4 v[QN], a[NORM ? QN : 1];
#pragma unroll
    for (int i = 0; i < QN; ++i) {
        const int q = threadIdx.x + i * kThreads;
        if (q < nq) {
            v[i] = src ? __ldcg(reinterpret_cast<const float4*>(src) + q) : reinterpret_cast<const float4*>(sm.xf)[q];
            if (NORM) a[i] = reinterpret_cast<const float4*>(alpha)[q];  // staged in shared memory
        }
    }
    if (NORM) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < QN; ++i) {
            const int q = threadIdx.x + i * kThreads;
            if (q < nq) {
                ss = __fmaf_rn(v[i].x, v[i].x, ss);
                ss = __fmaf_rn(v[i].y, v[i].y, ss);
                ss = __fmaf_rn(v[i].z, v[i].z, ss);
                ss = __fmaf_rn(v[i].w, v[i].w, ss);
            }
        }
        ss = block_sum(ss, sm, rb);
        // x * (1 / rms) instead of x / rms: within 1.5 ulp, below the 24-bit fixed-point step of
        // the limbs that follow
        const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-8f)));
#pragma unroll
        for (int i = 0; i < QN; ++i) {
            v[i].x = __fmul_rn(__fmul_rn(v[i].x, inv), a[NORM ? i : 0].x);
            v[i].y = __fmul_rn(__fmul_rn(v[i].y, inv), a[NORM ? i : 0].y);
            v[i].z = __fmul_rn(__fmul_rn(v[i].z, inv), a[NORM ? i : 0].z);
            v[i].w = __fmul_rn(__fmul_rn(v[i].w, inv), a[NORM ? i : 0].w);
        }
    }
#pragma unroll
    for (int i = 0; i < QN; ++i) {
        const int q = threadIdx.x + i * kThreads;
        if (q < nq) quad_limbs(sm, q, NB, v[i]);  // nq is a multiple of 32: whole warps
    }
    __syncthreads();
}

__device__ __forceinline__ void prep_vector(Smem& sm, const float* src, int K, const float* alpha, uint32_t& rb) {
    const int qn = (K / 4 + kThreads - 1) / kThreads;
    if (alpha) {
        if (qn <= 1) prep_vector_t<1, true>(sm, src, K, alpha, rb);
        else prep_vector_t<2, true>(sm, src, K, alpha, rb);  // D <= 4096
    } else {
        if (qn <= 1) prep_vector_t<1, false>(sm, src, K, alpha, rb);
        else if (qn <= 2) prep_vector_t<2, false>(sm, src, K, alpha, rb);
        else prep_vector_t<kQMax, false>(sm, src, K, alpha, rb);
    }
}

// ------------------------------------------------------------------------------ GEMV

// 16 * sum over one Q4_0 block of (nibble - 8) * X in fixed point (S0 + 256 S1 + 65536 S2)
__device__ __forceinline__ float block_dp4a(const uint4 q, const uint4* L) {
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    const uint32_t l0[4] = {L[0].x, L[0].y, L[0].z, L[0].w}, l1[4] = {L[1].x, L[1].y, L[1].z, L[1].w};
    const uint32_t l2[4] = {L[2].x, L[2].y, L[2].z, L[2].w}, h0[4] = {L[3].x, L[3].y, L[3].z, L[3].w};
    const uint32_t h1[4] = {L[4].x, L[4].y, L[4].z, L[4].w}, h2[4] = {L[5].x, L[5].y, L[5].z, L[5].w};
    int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        // 16 * (nibble - 8) as signed bytes: low nibbles shifted up, high nibbles in place
        const int lo = (int)(((words[w] << 4) & 0xF0F0F0F0u) ^ 0x80808080u);
        const int hi = (int)((words[w] & 0xF0F0F0F0u) ^ 0x80808080u);
        s0 = dp4a_su(lo, l0[w], s0);
        s1 = dp4a_su(lo, l1[w], s1);
        s2 = dp4a_ss(lo, l2[w], s2);
        s0 = dp4a_su(hi, h0[w], s0);
        s1 = dp4a_su(hi, h1[w], s1);
        s2 = dp4a_ss(hi, h2[w], s2);
    }
    return __fmaf_rn(i2f(s2), 65536.0f, __fmaf_rn(i2f(s1), 256.0f, i2f(s0)));
}

struct HeadBest {
    float v;
    int i;
};

// One GEMV phase over the rows staged in wbuf.  Units are row pairs (2u, 2u+1) or, for
// linear_in, (gate row u, value row u + F); a warp takes one unit, its lanes split the blocks.
template <int EPI>
__device__ __noinline__ void gemv_phase(const MegaArgs& P, Smem& /*sm_param*/, const Rows& r, int layer,
                                        const StreamState& st, HeadBest* best, int frame) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    if (r.nr == 0 || r.n[0] <= 0) return;
    const Staged s = staged_layout(r, false, c.D);
    const int NB = r.W->k >> 5;
    const int units = EPI == EPI_GATE ? r.n[0] : (r.n[0] + 1) / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint4* nibs = reinterpret_cast<const uint4*>(sm.wbuf);
    const uint16_t* scs = reinterpret_cast<const uint16_t*>(sm.wbuf);
    for (int u = warp; u < units; u += kWarps) {
        int ra, rb;  // global rows (rb < 0: unit has one row)
        uint32_t na, nb, sa, sb;  // wbuf offsets in uint4 / uint16 units
        if (EPI == EPI_GATE) {
            ra = r.r0[0] + u;
            rb = r.r0[1] + u;
            na = s.nib[0] / 16 + (uint32_t)u * NB;
            nb = s.nib[1] / 16 + (uint32_t)u * NB;
            sa = s.sc[0] / 2 + (uint32_t)u * NB;
            sb = s.sc[1] / 2 + (uint32_t)u * NB;
        } else {
            const int la = 2 * u;
            const bool two = 2 * u + 1 < r.n[0];
            const int lb = two ? la + 1 : la;
            ra = r.r0[0] + la;
            rb = two ? r.r0[0] + lb : -1;
            na = s.nib[0] / 16 + (uint32_t)la * NB;
            nb = s.nib[0] / 16 + (uint32_t)lb * NB;
            sa = s.sc[0] / 2 + (uint32_t)la * NB;
            sb = s.sc[0] / 2 + (uint32_t)lb * NB;
        }
        float acc_a = 0.0f, acc_b = 0.0f;
        for (int b = lane; b < NB; b += 32) {
            const uint4 qa = nibs[na + b], qb = nibs[nb + b];
            const float x = sm.xs[b];
            const float da = __fmul_rn(f16_to_f32_ieee(scs[sa + b]), x);
            const float db = __fmul_rn(f16_to_f32_ieee(scs[sb + b]), x);
            uint4 L[6];
#pragma unroll
            for (int v = 0; v < 6; ++v) L[v] = sm.limbs[v * NB + b];
            acc_a = __fmaf_rn(block_dp4a(qa, L), da, acc_a);
            acc_b = __fmaf_rn(block_dp4a(qb, L), db, acc_b);
        }
        float va = warp_sum(acc_a), vb = warp_sum(acc_b);
        if (lane != 0) continue;
        if (EPI == EPI_RESID) {  // rows of this CTA: the residual lives in xown
            const int o = ra - r.r0[0];
            const float xa_ = __fadd_rn(va, sm.xown[o]);
            sm.xown[o] = xa_;
            c.x[ra] = xa_;
            if (rb >= 0) {
                const float xb_ = __fadd_rn(vb, sm.xown[o + 1]);
                sm.xown[o + 1] = xb_;
                c.x[rb] = xb_;
            }
        } else if (EPI == EPI_GATE) {
            const float sg = __fmul_rn(va, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-va))));
            c.hid[ra] = __fmul_rn(sg, vb);
        } else if (EPI == EPI_LOGITS) {
            c.logits[ra] = va;
            if (c.desc->logits) c.desc->logits[(int64_t)frame * c.V + ra] = va;
            if (va > best->v || (va == best->v && ra < best->i)) {
                best->v = va;
                best->i = ra;
            }
            if (rb >= 0) {
                c.logits[rb] = vb;
                if (c.desc->logits) c.desc->logits[(int64_t)frame * c.V + rb] = vb;
                if (vb > best->v || (vb == best->v && rb < best->i)) {
                    best->v = vb;
                    best->i = rb;
                }
            }
        } else {  // EPI_QKV: RoPE on q and k pairs, K/V ring write (row pairs are always complete)
            const int D = c.D, HD = c.HD;
            const int part = ra / D;
            const int within = ra - part * D;
            const int h = within / HD, d = within - h * HD;
            if (part < 2) {
                const float2 cs = sm.rope[d >> 1];
                const float re = __fsub_rn(__fmul_rn(va, cs.x), __fmul_rn(vb, cs.y));
                const float im = __fadd_rn(__fmul_rn(va, cs.y), __fmul_rn(vb, cs.x));
                va = re;
                vb = im;
            }
            c.qkv[ra] = va;
            c.qkv[ra + 1] = vb;
            if (part >= 1) {
                const int64_t off = (int64_t)c.ids[0] * c.kv_stream_stride + (int64_t)layer * c.kv_layer_stride +
                                    (part == 2 ? c.kv_half_stride : 0) + ((int64_t)h * c.ML + st.write_pos) * HD + d;
                if (c.kv_f32) {
                    float* kv = reinterpret_cast<float*>(c.kv) + off;
                    kv[0] = va;
                    kv[1] = vb;
                } else {
                    *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(c.kv) + off) =
                        __floats2bfloat162_rn(va, vb);
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------ attention

constexpr int kKeysPerBatch = 4;  // keys a warp loads before computing

template <typename KT>
__device__ __forceinline__ void load_kv(const KT* kp, const KT* vp, int lane, float4& k, float4& v) {
    if (sizeof(KT) == 4) {
        k = __ldcg(reinterpret_cast<const float4*>(kp) + lane);
        v = __ldcg(reinterpret_cast<const float4*>(vp) + lane);
    } else {
        const uint2 kr = __ldcg(reinterpret_cast<const uint2*>(kp) + lane);
        const uint2 vr = __ldcg(reinterpret_cast<const uint2*>(vp) + lane);
        k = make_float4(__uint_as_float(kr.x << 16), __uint_as_float(kr.x & 0xFFFF0000u), __uint_as_float(kr.y << 16),
                        __uint_as_float(kr.y & 0xFFFF0000u));
        v = make_float4(__uint_as_float(vr.x << 16), __uint_as_float(vr.x & 0xFFFF0000u), __uint_as_float(vr.y << 16),
                        __uint_as_float(vr.y & 0xFFFF0000u));
    }
}

// Split-KV attention of head h over ring slots [j0, j1) of this CTA, from the staged K/V (the
// slot written this frame, write_pos, comes from qkv).  Writes the partial (max, sum exp,
// sum exp * v); the out_proj prologue of every CTA combines the partials of all splits.
template <typename KT>
__device__ __noinline__ void attention_phase(const MegaArgs& P, Smem& /*sm_param*/, int layer, const StreamState& st,
                                             int cta, int ncta) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int len = min(st.len + 1, c.ML);
    const Split sp = split_of(P, cta, len);
    if (sp.h >= c.H) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int HD = c.HD, h = sp.h;
    const float4 q = __ldcg(reinterpret_cast<const float4*>(c.qkv + h * HD) + lane);
    const float4 kcur = __ldcg(reinterpret_cast<const float4*>(c.qkv + c.D + h * HD) + lane);
    const float4 vcur = __ldcg(reinterpret_cast<const float4*>(c.qkv + 2 * c.D + h * HD) + lane);
    const uint32_t koff = kv_offset(sm, c, layer, cta, ncta);
    const uint32_t kvb = (uint32_t)(sp.j1 - sp.j0) * HD * sizeof(KT);
    const KT* ks = reinterpret_cast<const KT*>(sm.wbuf + koff);
    const KT* vs = reinterpret_cast<const KT*>(sm.wbuf + koff + kvb);
    float m = -FLT_MAX, l = 0.0f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = sp.j0 + warp; j < sp.j1; j += kWarps) {
        float4 k, v;
        if (j == st.write_pos) {
            // this frame's K/V (the ring copy stores them rounded to the ring type)
            if (sizeof(KT) == 4) {
                k = kcur;
                v = vcur;
            } else {
                k = make_float4(__bfloat162float(__float2bfloat16_rn(kcur.x)), __bfloat162float(__float2bfloat16_rn(kcur.y)),
                                __bfloat162float(__float2bfloat16_rn(kcur.z)), __bfloat162float(__float2bfloat16_rn(kcur.w)));
                v = make_float4(__bfloat162float(__float2bfloat16_rn(vcur.x)), __bfloat162float(__float2bfloat16_rn(vcur.y)),
                                __bfloat162float(__float2bfloat16_rn(vcur.z)), __bfloat162float(__float2bfloat16_rn(vcur.w)));
            }
        } else {
            const int r = j - sp.j0;
            if (sizeof(KT) == 4) {
                k = reinterpret_cast<const float4*>(ks + (int64_t)r * HD)[lane];
                v = reinterpret_cast<const float4*>(vs + (int64_t)r * HD)[lane];
            } else {
                const uint2 kr = reinterpret_cast<const uint2*>(ks + (int64_t)r * HD)[lane];
                const uint2 vr = reinterpret_cast<const uint2*>(vs + (int64_t)r * HD)[lane];
                k = make_float4(__uint_as_float(kr.x << 16), __uint_as_float(kr.x & 0xFFFF0000u),
                                __uint_as_float(kr.y << 16), __uint_as_float(kr.y & 0xFFFF0000u));
                v = make_float4(__uint_as_float(vr.x << 16), __uint_as_float(vr.x & 0xFFFF0000u),
                                __uint_as_float(vr.y << 16), __uint_as_float(vr.y & 0xFFFF0000u));
            }
        }
        float dot = __fmul_rn(q.x, k.x);
        dot = __fmaf_rn(q.y, k.y, dot);
        dot = __fmaf_rn(q.z, k.z, dot);
        dot = __fmaf_rn(q.w, k.w, dot);
        dot = warp_sum(dot);
        const float score = __fmul_rn(dot, c.attn_scale);
        const float mn = fmaxf(m, score);
        const float corr = expf(m - mn);
        const float p = expf(score - mn);
        l = __fmaf_rn(l, corr, p);
        o.x = __fmaf_rn(o.x, corr, __fmul_rn(p, v.x));
        o.y = __fmaf_rn(o.y, corr, __fmul_rn(p, v.y));
        o.z = __fmaf_rn(o.z, corr, __fmul_rn(p, v.z));
        o.w = __fmaf_rn(o.w, corr, __fmul_rn(p, v.w));
        m = mn;
    }
    // combine the warps in warp order through shared memory (xf as scratch)
    float* wm = sm.xf;
    float* wl = sm.xf + kWarps;
    float4* wo = reinterpret_cast<float4*>(sm.xf + 2 * kWarps);
    if (lane == 0) {
        wm[warp] = m;
        wl[warp] = l;
    }
    wo[warp * 32 + lane] = o;
    __syncthreads();
    if (warp == 0) {
        float M = -FLT_MAX;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w]);
        float L = 0.0f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < kWarps; ++w) {
            if (wl[w] == 0.0f) continue;
            const float f = expf(wm[w] - M);
            L = __fmaf_rn(wl[w], f, L);
            const float4 ow = wo[w * 32 + lane];
            O.x = __fmaf_rn(ow.x, f, O.x);
            O.y = __fmaf_rn(ow.y, f, O.y);
            O.z = __fmaf_rn(ow.z, f, O.z);
            O.w = __fmaf_rn(ow.w, f, O.w);
        }
        float* part = c.part + ((int64_t)h * P.nsplit + sp.s) * (HD + 4);
        if (lane == 0) {
            part[0] = M;
            part[1] = L;
        }
        reinterpret_cast<float4*>(part + 4)[lane] = O;
    }
}

// The out_proj input: every CTA combines, for each head, the partials of all its splits (in
// split order) into softmax(q.k^T * scale).v, then builds the limbs.
template <int NSMAX>
__device__ __noinline__ void prep_attn(Smem& /*sm_param*/, const MegaArgs& P) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int NS = P.nsplit, HD = c.HD, NB = c.D >> 5;
    const int nq = c.D >> 2, qh = HD >> 2;
    for (int q = threadIdx.x; q < nq; q += kThreads) {
        const int h = q / qh, d4 = q - h * qh;
        const float* pb = c.part + (int64_t)h * NS * (HD + 4);
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        float L = 0.0f;
        if (NS <= NSMAX) {
            float2 ml[NSMAX];
            float4 os[NSMAX];
#pragma unroll
            for (int t = 0; t < NSMAX; ++t)
                if (t < NS) {
                    ml[t] = __ldcg(reinterpret_cast<const float2*>(pb + t * (HD + 4)));
                    os[t] = __ldcg(reinterpret_cast<const float4*>(pb + t * (HD + 4) + 4) + d4);
                }
            float M = -FLT_MAX;
#pragma unroll
            for (int t = 0; t < NSMAX; ++t)
                if (t < NS && ml[t].y != 0.0f) M = fmaxf(M, ml[t].x);
#pragma unroll
            for (int t = 0; t < NSMAX; ++t)
                if (t < NS && ml[t].y != 0.0f) {
                    const float f = expf(ml[t].x - M);
                    L = __fmaf_rn(ml[t].y, f, L);
                    O.x = __fmaf_rn(os[t].x, f, O.x);
                    O.y = __fmaf_rn(os[t].y, f, O.y);
                    O.z = __fmaf_rn(os[t].z, f, O.z);
                    O.w = __fmaf_rn(os[t].w, f, O.w);
                }
        } else {
            float M = -FLT_MAX;
            for (int t = 0; t < NS; ++t) {
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(pb + t * (HD + 4)));
                if (ml.y != 0.0f) M = fmaxf(M, ml.x);
            }
            for (int t = 0; t < NS; ++t) {
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(pb + t * (HD + 4)));
                if (ml.y == 0.0f) continue;
                const float4 ot = __ldcg(reinterpret_cast<const float4*>(pb + t * (HD + 4) + 4) + d4);
                const float f = expf(ml.x - M);
                L = __fmaf_rn(ml.y, f, L);
                O.x = __fmaf_rn(ot.x, f, O.x);
                O.y = __fmaf_rn(ot.y, f, O.y);
                O.z = __fmaf_rn(ot.z, f, O.z);
                O.w = __fmaf_rn(ot.w, f, O.w);
            }
        }
        const float4 a = make_float4(__fdiv_rn(O.x, L), __fdiv_rn(O.y, L), __fdiv_rn(O.z, L), __fdiv_rn(O.w, L));
        quad_limbs(sm, q, NB, a);  // c.D / 4 is a multiple of 32: whole warps
    }
    __syncthreads();
}

// ------------------------------------------------------------------------------ embedding

__device__ __forceinline__ float emb_val(const Ctx& c, const uint8_t* table, uint32_t row, int j) {
    const uint8_t* r = table + (int64_t)row * c.emb_row_bytes;
    switch (c.emb_type) {
        case EMB_BF16: return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(r)[j] << 16);
        case EMB_F32: return reinterpret_cast<const float*>(r)[j];
        case EMB_F16: return f16_to_f32_ieee(reinterpret_cast<const uint16_t*>(r)[j]);
        default: {
            const uint8_t* blk = r + (j >> 5) * 18;
            const float d = f16_to_f32_gguf((uint16_t)(blk[0] | (blk[1] << 8)));
            const int w = j & 31;
            const uint32_t byte = blk[2 + (w & 15)];
            return __fmul_rn(nib_m8(w < 16 ? (byte & 0xFu) : (byte >> 4)), d);
        }
    }
}

// ------------------------------------------------------------------------------ kernel

struct Look {
    int next;  // next global phase to L2-prefetch
    int end;   // one past the last global phase of the launch
};

// Warp 0, after staging global phase `staged`: L2-prefetch later phases until pf_budget bytes
// are requested beyond it.  Every lane keeps the same Look state.
__device__ void look_ahead(const Smem& sm, const MegaArgs& P, Look& lk, int staged, int per_frame, int cta, int ncta,
                           int len) {
    const int lane = threadIdx.x & 31;
    if (lk.next <= staged) lk.next = staged + 1;
    uint32_t ahead = 0;
    for (int g = staged + 1; g < lk.next; ++g) ahead += phase_bytes(sm, P, g % per_frame, cta, ncta, len);
    while (lk.next < lk.end && ahead < P.pf_budget) {
        const int p = lk.next % per_frame;
        prefetch_phase(sm, P, p, cta, ncta, len, lane);
        ahead += phase_bytes(sm, P, p, cta, ncta, len);
        ++lk.next;
    }
}

__global__ void __launch_bounds__(kThreads, 1) mega_kernel(const __grid_constant__ MegaArgs P) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int cta = blockIdx.x, ncta = gridDim.x;
    const int per_frame = 5 * c.L + 1;
    uint32_t epoch = 0, parity = 0, rb = 0;
    Tracer tr;
    Look lk{0, per_frame * P.steps};
    // rows of x this CTA owns: the out_proj / linear_out row range
    const int own0 = (int)(2 * split_lo(c.D / 2, cta, ncta));
    const int own1 = (int)(2 * split_lo(c.D / 2, cta + 1, ncta));

    for (int i = threadIdx.x; i < c.L; i += kThreads) sm.layers[i] = c.layers[i];
    if (threadIdx.x == 0) {
        mbar_init(&sm.mbar, 1);
        sm.staged = sm.waited = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const int sid = c.ids[0];
    StreamState st = c.state[sid];
    StepDesc* desc = c.desc;
    if (threadIdx.x == 0) stage_phase(sm, c, 0, cta, ncta);
    if (threadIdx.x < 32) look_ahead(sm, P, lk, 0, per_frame, cta, ncta, min(st.len + 1, c.ML));

    for (int f = 0; f < P.steps; ++f) {
        if (tr.on) tr.wall(P);  // end of the traced frame
        tr.on = P.trace != nullptr && cta == 0 && f == P.trace_frame;
        tr.wall(P);
        tr.mark(P, 1);
        {
            const int len_now = min(st.len + 1, c.ML);
            uint32_t text = desc->text ? __ldcg(desc->text + f) : st.last_text;
            if (text >= (uint32_t)c.TV) {
                raise_error(desc, -1);
                text = 0;
            }
            // x = audio sum + text row (model.rs:640-646): built whole by every CTA; the CTA keeps
            // its own rows in xown and publishes them
            const float* xa = P.xa + (int64_t)f * c.D;
            for (int j = threadIdx.x; j < c.D; j += kThreads) {
                const float v = __fadd_rn(__ldcg(xa + j), emb_val(c, c.emb_text, text, j));
                sm.xf[j] = v;
                if (j >= own0 && j < own1) {
                    sm.xown[j - own0] = v;
                    c.x[j] = v;
                }
            }
            if (threadIdx.x < (c.HD >> 1)) sm.rope[threadIdx.x] = c.rope[(int64_t)st.offset * (c.HD >> 1) + threadIdx.x];
            __syncthreads();
            for (int l = 0; l < c.L; ++l) {
                const int p0 = 5 * l, gp0 = f * per_frame + p0;
                // ---- QKV: weights and norm1 were staged before the previous barrier
                if (!wait_stage(sm, P, parity)) goto drain;
                tr.mark(P, 11);
                {
                    const Rows r = rows_of(sm, c, p0 + K_QKV, cta, ncta);
                    const Staged sg = staged_layout(r, true, c.D);
                    prep_vector(sm, l == 0 ? nullptr : c.x, c.D, reinterpret_cast<const float*>(sm.wbuf + sg.alpha), rb);
                    tr.mark(P, 10);
                    gemv_phase<EPI_QKV>(P, sm, r, l, st, nullptr, f);
                }
                __syncthreads();
                tr.mark(P, 12);
                if (threadIdx.x == 0) stage_out_kv(sm, P, l, cta, ncta, len_now);
                tr.mark(P, 70);
                if (threadIdx.x < 32) look_ahead(sm, P, lk, gp0 + K_OUT, per_frame, cta, ncta, len_now);
                tr.mark(P, 71);
                if (!grid_sync(P, epoch, sm, tr)) goto drain;
                // ---- attention over the staged K/V slots (staged together with out_proj's rows)
                if (!wait_stage(sm, P, parity)) goto drain;
                tr.mark(P, 21);
                if (c.kv_f32) attention_phase<float>(P, sm, l, st, cta, ncta);
                else attention_phase<__nv_bfloat16>(P, sm, l, st, cta, ncta);
                __syncthreads();
                tr.mark(P, 22);
                if (!grid_sync(P, epoch, sm, tr)) goto drain;
                // ---- out_proj + residual (input: the combined attention partials)
                if (P.nsplit <= 10) prep_attn<10>(sm, P);
                else prep_attn<1>(sm, P);
                tr.mark(P, 30);
                gemv_phase<EPI_RESID>(P, sm, rows_of(sm, c, p0 + K_OUT, cta, ncta), l, st, nullptr, f);
                __syncthreads();
                tr.mark(P, 32);
                if (threadIdx.x == 0) stage_phase(sm, c, p0 + K_IN, cta, ncta);
                tr.mark(P, 70);
                if (threadIdx.x < 32) look_ahead(sm, P, lk, gp0 + K_IN, per_frame, cta, ncta, len_now);
                tr.mark(P, 71);
                if (!grid_sync(P, epoch, sm, tr)) goto drain;
                // ---- linear_in + silu gate
                if (!wait_stage(sm, P, parity)) goto drain;
                tr.mark(P, 41);
                {
                    const Rows r = rows_of(sm, c, p0 + K_IN, cta, ncta);
                    const Staged sg = staged_layout(r, true, c.D);
                    prep_vector(sm, c.x, c.D, reinterpret_cast<const float*>(sm.wbuf + sg.alpha), rb);
                    tr.mark(P, 40);
                    gemv_phase<EPI_GATE>(P, sm, r, l, st, nullptr, f);
                }
                __syncthreads();
                tr.mark(P, 42);
                if (threadIdx.x == 0) stage_phase(sm, c, p0 + K_DOWN, cta, ncta);
                tr.mark(P, 70);
                if (threadIdx.x < 32) look_ahead(sm, P, lk, gp0 + K_DOWN, per_frame, cta, ncta, len_now);
                tr.mark(P, 71);
                if (!grid_sync(P, epoch, sm, tr)) goto drain;
                // ---- linear_out + residual
                if (!wait_stage(sm, P, parity)) goto drain;
                tr.mark(P, 51);
                prep_vector(sm, c.hid, c.F, nullptr, rb);
                tr.mark(P, 50);
                gemv_phase<EPI_RESID>(P, sm, rows_of(sm, c, p0 + K_DOWN, cta, ncta), l, st, nullptr, f);
                __syncthreads();
                tr.mark(P, 52);
                {  // next: QKV of layer l+1, or the head
                    const int pn = l + 1 < c.L ? p0 + 5 : 5 * c.L;
                    if (threadIdx.x == 0) stage_phase(sm, c, pn, cta, ncta);
                    tr.mark(P, 70);
                    if (threadIdx.x < 32) look_ahead(sm, P, lk, f * per_frame + pn, per_frame, cta, ncta, len_now);
                    tr.mark(P, 71);
                }
                if (!grid_sync(P, epoch, sm, tr)) goto drain;
            }
            // ---- head + argmax partials
            if (!wait_stage(sm, P, parity)) goto drain;
            tr.mark(P, 61);
            HeadBest best{-FLT_MAX, 0x7FFFFFFF};
            {
                const Rows r = rows_of(sm, c, 5 * c.L, cta, ncta);
                const Staged sg = staged_layout(r, true, c.D);
                prep_vector(sm, c.x, c.D, reinterpret_cast<const float*>(sm.wbuf + sg.alpha), rb);
                tr.mark(P, 60);
                gemv_phase<EPI_LOGITS>(P, sm, r, 0, st, &best, f);
            }
            {
                const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
                if (lane == 0) {
                    sm.wv[warp] = best.v;
                    sm.wi[warp] = best.i;
                }
                __syncthreads();
                if (threadIdx.x == 0) {
                    float bv = -FLT_MAX;
                    int bi = 0x7FFFFFFF;
                    for (int w = 0; w < kWarps; ++w)
                        if (sm.wv[w] > bv || (sm.wv[w] == bv && sm.wi[w] < bi)) {
                            bv = sm.wv[w];
                            bi = sm.wi[w];
                        }
                    P.amax_v[cta] = bv;
                    P.amax_i[cta] = bi;
                    if (f + 1 < P.steps) stage_phase(sm, c, 0, cta, ncta);  // next frame: layer 0's QKV
                }
                if (f + 1 < P.steps && threadIdx.x < 32)
                    look_ahead(sm, P, lk, (f + 1) * per_frame, per_frame, cta, ncta, min(st.len + 2, c.ML));
            }
            tr.mark(P, 62);
            if (!grid_sync(P, epoch, sm, tr)) goto drain;
        }
        // every CTA reduces the partials identically
        {
            float bv = -FLT_MAX;
            int bi = 0x7FFFFFFF;
            for (int t = 0; t < ncta; ++t) {
                const float v = __ldcg(P.amax_v + t);
                const int i = __ldcg(P.amax_i + t);
                if (v > bv || (v == bv && i < bi)) {
                    bv = v;
                    bi = i;
                }
            }
            const uint32_t token = (uint32_t)(bi == 0x7FFFFFFF ? 0 : bi);
            st.write_pos = (st.write_pos + 1) % c.ML;
            st.offset += 1;
            st.len = min(st.len + 1, c.ML);
            int32_t out = (int32_t)token;
            if (desc->mode == 1) {
                st.frame_count += 1;
                if (st.frame_count >= c.text_delay) {
                    st.last_text = token;
                } else {
                    const uint32_t p0 = st.prev0, p1 = st.prev1;
                    st.prev0 = p1;
                    st.prev1 = token;
                    st.last_text = (token != c.pad_id && token != 0u && token == p0 && token != p1) ? c.pad_id : token;
                    out = -1;
                }
            }
            if (cta == 0 && threadIdx.x == 0) {
                desc->tokens[f] = out;
                c.state[sid] = st;
                if (f + 1 == P.steps) desc->step = P.steps;
            }
        }
    }
    return;
drain:
    // stopping early: a staged copy that was issued but not yet waited for (stages and waits
    // alternate, so one is pending exactly when the issue count exceeds the wait count) must land
    // before the CTA's shared memory goes away
    if (threadIdx.x == 0 && sm.staged != sm.waited) {
        uint32_t spins = 0;
        while (!mbar_try_wait(&sm.mbar, parity) && ++spins < kSpinLimit) {
        }
    }
    __syncthreads();
}

// Audio-embedding sums of every frame of the call: xa[f][j] = sum over codebooks (in order) of
// the audio rows of frame f (model.rs:640-644), computed before the persistent kernel starts.
__global__ void __launch_bounds__(256) audio_sum_kernel(Ctx c, float* __restrict__ xa) {
    const int f = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    __shared__ uint32_t toks[kMaxCodebooks];
    const uint32_t* audio = c.desc->audio + (int64_t)f * c.NC;
    if (threadIdx.x < c.NC) {
        uint32_t t = audio[threadIdx.x];
        if (t >= (uint32_t)c.AV) {
            raise_error(c.desc, -1);
            t = 0;
        }
        toks[threadIdx.x] = t;
    }
    __syncthreads();
    if (j >= c.D) return;
    const int64_t table = (int64_t)c.AV * c.emb_row_bytes;
    float acc = 0.0f;
    for (int cb = 0; cb < c.NC; ++cb) acc = __fadd_rn(acc, emb_val(c, c.emb_audio + cb * table, toks[cb], j));
    xa[(int64_t)f * c.D + j] = acc;
}

// Grid-barrier latency probe: `iters` back-to-back barriers of the persistent kernel (mode 0),
// or of a variant where the last arriver (atom.add.acq_rel) publishes a generation flag on a
// separate line that the others poll (mode 1).
__global__ void __launch_bounds__(kThreads, 1) barrier_probe_kernel(const __grid_constant__ MegaArgs P, int iters,
                                                                    int mode) {
    Smem& sm = smem_ref();
    uint32_t epoch = 0;
    Tracer tr;
    if (mode == 0) {
        for (int i = 0; i < iters; ++i)
            if (!grid_sync(P, epoch, sm, tr)) return;
        return;
    }
    uint32_t* flag = P.bar + 32;  // 128 bytes away from the counter
    for (int i = 0; i < iters; ++i) {
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t gen = (uint32_t)i + 1u;
            uint32_t old;
            asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(P.bar) : "memory");
            if (old == gen * gridDim.x - 1u) {
                asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(gen) : "memory");
            } else {
                uint32_t spins = 0;
                while ((int32_t)(ld_acquire(flag) - gen) < 0 && ++spins < kSpinLimit) {
                }
            }
        }
        __syncthreads();
    }
}

// Largest staged phase of one CTA in bytes (must fit kWBuf).
size_t max_stage_bytes(int D, int F, int V, int ncta) {
    auto rows_max = [&](int64_t units, int rows_per_unit) { return (units + ncta - 1) / ncta * rows_per_unit; };
    auto bytes = [](int64_t rows, int k) {
        return (size_t)rows * (k / 32) * 16 + (((size_t)rows * (k / 32) * 2 + 15) & ~(size_t)15);
    };
    size_t m = bytes(rows_max(3 * D / 2, 2), D);
    m = std::max(m, bytes(rows_max(D / 2, 2), D));
    m = std::max(m, 2 * bytes(rows_max(F, 1), D));
    m = std::max(m, bytes(rows_max(D / 2, 2), F));
    m = std::max(m, bytes(rows_max((V + 1) / 2, 2), D));
    return m;
}

}  // namespace

cudaError_t mega_barrier_probe(void* scratch, int iters, int mode, float* ms_out) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(barrier_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
    if (e != cudaSuccess) return e;
    MegaArgs P{};
    P.bar = static_cast<uint32_t*>(scratch);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    e = cudaMemset(P.bar, 0, 256);
    void* args[] = {(void*)&P, (void*)&iters, (void*)&mode};
    if (e == cudaSuccess) e = cudaEventRecord(a, 0);
    if (e == cudaSuccess)
        e = cudaLaunchCooperativeKernel((const void*)barrier_probe_kernel, dim3(sms), dim3(kThreads), args, sizeof(Smem), 0);
    if (e == cudaSuccess) e = cudaEventRecord(b, 0);
    if (e == cudaSuccess) e = cudaEventSynchronize(b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms_out, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return e;
}

bool mega_supported(int L, int D, int F, int HD, int V, int num_sms, int ML, int kv_f32) {
    const int H = D / HD;
    const int nsplit = num_sms / (H > 0 ? H : 1);
    if (nsplit < 1) return false;
    // out_proj rows (plus alignment) and the K/V slots of one split share the staging buffer
    const size_t kv = (size_t)((ML + nsplit - 1) / nsplit) * HD * (kv_f32 ? 4 : 2) * 2;
    const size_t out_rows = (size_t)2 * ((D / 2 + num_sms - 1) / num_sms);
    const size_t out_bytes = out_rows * (D / 32) * 16 + ((out_rows * (D / 32) * 2 + 15) & ~(size_t)15);
    if (((out_bytes + 127) & ~(size_t)127) + kv > (size_t)kWBuf) return false;
    if (max_stage_bytes(D, F, V, num_sms) + (size_t)D * 4 > (size_t)kWBuf) return false;
    // head tickets live in the 64-word barrier block (2 + H <= 64); the layer table holds kMaxL;
    // a CTA keeps its x rows (2 * ceil(D/2 / num_sms)) in xown
    return HD == 128 && D % 256 == 0 && D <= 4096 && F % 128 == 0 && F <= kMaxK && L > 0 && L <= kMaxL &&
           2 * ((D / 2 + num_sms - 1) / num_sms) <= kMaxOwnRows &&
           D / HD <= 60 && max_stage_bytes(D, F, V, num_sms) <= (size_t)kWBuf &&
           std::getenv("STT_DISABLE_MEGA") == nullptr;
}

size_t mega_scratch_bytes(int num_sms, int D, int F, int V, int H, int HD) {
    return 256 + (size_t)D * 4 + (size_t)num_sms * 8 + 64 * 4;  // bar | (unused) | amax_v | amax_i
}

cudaError_t configure_mega() {
    return cudaFuncSetAttribute(mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
}

cudaError_t launch_mega_steps(MegaState& ms, const Ctx& c, const LayerDev* h_layers, int steps, cudaStream_t st) {
    int dev = 0, sms = 0, occ = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, mega_kernel, kThreads, sizeof(Smem));
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorCooperativeLaunchTooLarge;
    uint8_t* s = static_cast<uint8_t*>(ms.scratch);
    MegaArgs P;
    P.c = c;
    P.steps = steps;
    P.nsplit = sms / c.H;  // the stream set sizes its partials buffer for num_sms rows
    P.bar = reinterpret_cast<uint32_t*>(s);
    P.xa = ms.xa_all;
    P.amax_v = reinterpret_cast<float*>(s + 256 + (size_t)c.D * 4);
    P.amax_i = reinterpret_cast<int32_t*>(s + 256 + (size_t)c.D * 4 + (size_t)sms * 4);
    P.pf_budget = 0;  // off by default: issuing the prefetches stalls warp 0 longer than it saves
    if (const char* pb = std::getenv("STT_MEGA_PF_KB")) P.pf_budget = (uint32_t)std::atoi(pb) * 1024u;
    P.pf_lines = 1;
    if (const char* pm = std::getenv("STT_MEGA_PF_BULK")) P.pf_lines = std::atoi(pm) ? 0 : 1;
    P.trace = nullptr;
    P.trace_frame = -1;
    P.trace_cap = 0;
    if (ms.trace && ms.trace_frame >= 0) {
        P.trace = ms.trace;
        P.trace_frame = ms.trace_frame;
        P.trace_cap = ms.trace_cap;
    }
    if (P.nsplit < 1) return cudaErrorInvalidConfiguration;
    e = cudaMemsetAsync(P.bar, 0, 256, st);
    if (e != cudaSuccess) return e;
    audio_sum_kernel<<<dim3((c.D + 255) / 256, steps), 256, 0, st>>>(c, ms.xa_all);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    void* args[] = {(void*)&P};
    return cudaLaunchCooperativeKernel((const void*)mega_kernel, dim3(sms), dim3(kThreads), args, sizeof(Smem), st);
}

}  // namespace stt
