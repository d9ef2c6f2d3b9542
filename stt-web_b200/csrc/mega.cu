// Persistent single-stream decode step for sm_100a.
//
// One cooperative launch of one 512-thread CTA per SM runs `steps` whole frames of one stream.
// A frame is 5 phases per layer (QKV, attention, out_proj, linear_in, linear_out), then the head
// and the argmax: 82 dependent steps that together read 627 MB of Q4_0 weights.  A phase is a
// few MB, so the kernel is built to keep that chain short while HBM keeps streaming:
//
//   - Warp 15 is a producer.  It walks the same phase sequence as the other 15 warps, one
//     "segment" at a time (a norm weight vector, a run of whole weight rows, or the K/V slots of
//     an attention split), and bulk-copies (cp.async.bulk) each segment into a 192 KB
//     shared-memory ring with a full mbarrier per segment.  It runs ahead of the consumers,
//     across phases and frames, as far as the ring allows; the consumers release a phase's
//     segments through empty mbarriers when the phase ends.
//   - Phases exchange activations through flagged buffers instead of grid barriers: every value
//     is one 64-bit word (value bits | epoch << 32), and a reader polls the words it needs until
//     each carries the epoch of the phase that wrote it.  A reader waits exactly for its own
//     inputs, and one L2 round trip both synchronises and fetches.  Epochs are unique per
//     (frame, phase) over a stream set's lifetime (a base word persists across launches), every
//     buffer is double-buffered by layer or frame parity, and each phase's inputs depend on every
//     CTA's outputs two phases back, so a reader never meets a value of a later epoch.
//   - One release/acquire counter per frame orders the K/V ring writes of a frame (made by the
//     QKV epilogues) before the producers' bulk copies of those slots in later frames.
//   - The GEMV turns the input vector into 24-bit fixed point per 32-element block (three byte
//     limbs, shared exponent) and puts every nibble through dp4a, so each block's dot product is
//     exact; only the per-block scale and the f32 accumulation round.
//   - Every wait is bounded.  A wait that gives up raises STT_E_DEVICE_FLAG in the step
//     descriptor and sets an abort word; every other wait sees that word and returns, all
//     consumer threads run on to the end of the layer with in-bounds garbage and stop together,
//     the producer waits (bounded) for its copies in flight, and the CTA exits.
#include <algorithm>
#include <cfloat>
#include <cstdlib>

#include "kernels.h"
#include "dp4a.cuh"
#include "mega.h"

namespace stt {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kCWarps = kWarps - 1;        // consumer warps; warp kCWarps is the producer
constexpr int kCThreads = kCWarps * 32;
constexpr int kNBMax = 264;                // K / 32 for K <= 8448
constexpr int kMaxK = kNBMax * 32;
constexpr uint32_t kRing = 192u * 1024u;   // weight / K-V ring
constexpr uint32_t kSegMax = 32u * 1024u;  // target bytes of one weight segment
constexpr int kNBar = 32;                  // segments in flight at most
constexpr int kMaxL = 32;
constexpr int kMaxOwnRows = 256;
constexpr uint32_t kEpochsPerFrame = 256;  // steps of a frame: 5 L + 2 <= 256
constexpr int kPartPairs = 132;            // attention partial: M, L, 2 unused, O[128]
// Bounded waits: a legitimate wait lasts at most about a frame (milliseconds); these limits give
// up after roughly a second.
constexpr uint32_t kSpinLimit = 1u << 21;    // mbarrier / counter polls
constexpr uint32_t kLLSpinLimit = 1u << 20;  // flagged-word polls (each with a short sleep)
constexpr uint32_t kSleepLimit = 1u << 20;   // mbarrier waits with a suspend-time hint

enum Kind : int { K_QKV = 0, K_ATT = 1, K_OUT = 2, K_IN = 3, K_DOWN = 4, K_HEAD = 5 };

// Row ranges of one CTA in one kind of phase; the same for every layer.
struct Range {
    int32_t r0;     // first row (linear_in: first gate row)
    int32_t n;      // rows (linear_in: units)
    int32_t units;  // pairs of rows, or (gate, value) units
    int32_t ups;    // units per weight segment
};

struct MegaArgs {
    Ctx c;
    int32_t steps;
    int32_t nsplit;        // attention splits per head
    uint32_t* bar;         // [0] frames finished (summed over CTAs), [1] abort
    uint32_t* base;        // epoch base, persists across launches
    const float* xa;       // [steps][D] audio-embedding sums (audio_sum_kernel)
    uint64_t* xb[2][2];    // [layer parity][0 after out_proj, 1 after linear_out]: D words
    uint64_t* qkvb[2];     // [layer parity]: 3D words (q, k rotated; v)
    uint64_t* partb[2];    // [layer parity]: H * nsplit * kPartPairs words
    uint64_t* attb[2];     // [layer parity]: D words (softmax(q.k^T * scale).v per head)
    uint64_t* hidb[2];     // [layer parity]: F words
    uint64_t* argb[2];     // [frame parity]: 2 words per CTA (best logit, its index)
    unsigned long long* trace;  // optional: (tag, SM clock) pairs of one frame of CTA 0
    int32_t trace_frame;
    int32_t trace_cap;
    unsigned long long* tctas;  // optional: [cta][slot] %globaltimer of every CTA's marks
    int32_t tslots;
    int32_t stall_test;    // test of the bounded waits: frame 0 waits for an epoch nobody writes
};

struct Smem {
    alignas(128) uint8_t ring[kRing];
    uint4 limbs[6 * kNBMax];  // [vec][block]: L0,L1,L2 of groups 0-3, then of groups 4-7; attention scratch
    float xs[kNBMax];         // 2^(e_b - 27): block scale of the fixed-point input
    LayerDev layers[kMaxL];
    float xown[kMaxOwnRows];  // this CTA's rows of the residual stream x
    float2 rope[64];          // (cos, sin) of this frame's position
    float2 hpart[kWarps / 2]; // residual phases: the second half-row sums of each row pair
    float red[2][kWarps];
    float wv[kWarps];         // head: best logit of each warp
    int32_t wi[kWarps];
    float av[kWarps];         // argmax: best of each warp over the per-CTA words
    int32_t ai[kWarps];
    Range rg[6];              // per kind of phase; rg[K_ATT] unused
    StreamState st;           // stream state at the start of the current frame
    uint32_t text;            // text token of the current frame
    uint32_t seg_off[kNBar];  // ring offset of an issued segment (producer writes, consumers read)
    uint32_t seg_end[kNBar];  // its end in ring bytes since launch (producer only)
    alignas(8) unsigned long long full[kNBar];
    alignas(8) unsigned long long empty[kNBar];
    int32_t stop[2];          // consumers: some thread saw an abort (by agreement parity)
    int32_t tslot, tron;      // trace cursor (consumer thread 0)
    int32_t tall;             // every CTA records this frame's marks
    long long wseg, wll;      // traced frame: thread 0's cycles in segment / flagged-word waits
};
static_assert(sizeof(Smem) <= 232448, "shared memory per CTA");

// The kernel's dynamic shared memory.  Functions that are not inlined recover the Smem through
// this file-scope array so the compiler keeps emitting shared-memory accesses.
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
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(unsigned long long* m, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(m)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* m, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(m)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* m) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(m)) : "memory");
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
// The same with a suspend-time hint: the thread sleeps until the phase completes or about
// `ns` nanoseconds pass, instead of spinning on the issue slots the working warps need.
__device__ __forceinline__ bool mbar_wait_sleep(unsigned long long* m, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(m)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, unsigned long long* m) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src),
        "r"(bytes), "r"(smem_addr(m))
        : "memory");
}
// flagged words: value bits in the low half, epoch in the high half
__device__ __forceinline__ void ll_store(uint64_t* p, float v, uint32_t ep) {
    const uint64_t w = ((uint64_t)ep << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void ll_load2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint32_t ll_ep(uint64_t w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float((uint32_t)w); }

// consumer-only CTA barrier (the producer warp never joins it)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory"); }

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool aborted(const MegaArgs& P) { return *(volatile const uint32_t*)(P.bar + 1) != 0u; }
__device__ __noinline__ void give_up(const MegaArgs& P) {
    raise_error(P.c.desc, -5);
    atomicExch(P.bar + 1, 1u);
}

// Trace of one frame of CTA 0: (tag, SM clock) pairs from consumer thread 0, bracketed by
// (0, %globaltimer) pairs so the host can convert cycles to time.  Tags: 1 frame start, then per
// kind of phase k (1 qkv, 2 attention, 3 out_proj, 4 linear_in, 5 linear_out, 6 head):
// 10k+1 inputs ready, 10k+2 this thread's compute done, 10k+3 phase end; 24 the partials of the
// other attention splits merged (split-0 CTAs); 7 argmax reduced.
// Every CTA also records %globaltimer at the mark's fixed slot: 0 frame start, 1 + 16 l + i for
// the i-th mark of layer l (11 12 13 21 22 24 23 31 32 33 41 42 43 51 52 53), 1 + 16 L + i for
// 61 62 63 7.
// The recording is a call, so that the phase code, which runs once per layer, stays compact in
// the instruction cache (measured 1.5% faster than the recording inlined at every mark).
__device__ __noinline__ void trace_record(const MegaArgs& P, unsigned long long tag, int slot) {
    Smem& sm = smem_ref();
    if (sm.tron && sm.tslot + 1 < P.trace_cap) {
        P.trace[sm.tslot] = tag;
        P.trace[sm.tslot + 1] = clock64();
        sm.tslot += 2;
    }
    if (sm.tall && slot < P.tslots) P.tctas[(int64_t)blockIdx.x * P.tslots + slot] = globaltimer();
}
__device__ __forceinline__ void trace_mark(const MegaArgs& P, unsigned long long tag, int slot) {
    Smem& sm = smem_ref();
    if (threadIdx.x == 0 && (sm.tron | sm.tall)) trace_record(P, tag, slot);
}
__device__ __forceinline__ int lslot(int l, int i) { return 1 + 16 * l + i; }

// Traced frame, CTA 0: thread 0's wait cycles of the phase that just ended, as (100 + kind,
// cycles + 1) for segment waits and (110 + kind, cycles + 1) for flagged-word waits (the +1
// keeps a zero duration from reading as the end of the trace).
__device__ __noinline__ void trace_waits_record(const MegaArgs& P, int kind) {
    Smem& sm = smem_ref();
    if (sm.tslot + 3 < P.trace_cap) {
        P.trace[sm.tslot] = 100 + kind;
        P.trace[sm.tslot + 1] = (unsigned long long)sm.wseg + 1;
        P.trace[sm.tslot + 2] = 110 + kind;
        P.trace[sm.tslot + 3] = (unsigned long long)sm.wll + 1;
        sm.tslot += 4;
    }
    sm.wseg = sm.wll = 0;
}
__device__ __forceinline__ void trace_waits(const MegaArgs& P, int kind) {
    if (threadIdx.x == 0 && smem_ref().tron) trace_waits_record(P, kind);
}
__device__ __forceinline__ void trace_wall(const MegaArgs& P) {
    Smem& sm = smem_ref();
    if (threadIdx.x == 0 && sm.tron && sm.tslot + 1 < P.trace_cap) {
        P.trace[sm.tslot] = 0;
        P.trace[sm.tslot + 1] = globaltimer();
        sm.tslot += 2;
    }
}

// ------------------------------------------------------------------------------ waits

// Consumer wait for segment i to land.  Returns false after an abort (seen or raised).
__device__ __forceinline__ bool wait_seg(Smem& sm, const MegaArgs& P, uint32_t i) {
    unsigned long long* m = &sm.full[i % kNBar];
    const uint32_t par = (i / kNBar) & 1u;
    if (mbar_try_wait(m, par)) return true;
    const bool tr = threadIdx.x == 0 && sm.tron;
    const long long t0 = tr ? clock64() : 0;
    uint32_t spins = 0;
    bool ok = true;
    while (!mbar_wait_sleep(m, par, 2000u)) {
        if ((++spins & 15u) == 0) {
            if (aborted(P)) {
                ok = false;
                break;
            }
            if (spins > kSleepLimit) {
                give_up(P);
                ok = false;
                break;
            }
        }
        __nanosleep(64);  // in case the hint returns early: keep waiting warps off the issue slots
    }
    if (tr) sm.wseg += clock64() - t0;
    return ok;
}

// Waits until the words of N 16-byte pieces (two words each, at addr(i)) all carry epoch ep.
// All loads of a round are in flight together, so a wait costs one L2 round trip once the data
// is there; between rounds the thread sleeps 32 .. 96 ns.  (Every address must be valid:
// loads skipped under a condition make the compiler keep far more registers live.)
template <int N, typename Addr>
__device__ __forceinline__ bool ll_wait_n(const MegaArgs& P, Addr addr, uint32_t ep, uint64_t (&w)[N][2]) {
    uint32_t spins = 0, nap = 32;
    const bool tr = threadIdx.x == 0 && smem_ref().tron;
    const long long t0 = tr ? clock64() : 0;
    for (;;) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            ll_load2(addr(i), w[i][0], w[i][1]);
        }
        bool ok = true;
#pragma unroll
        for (int i = 0; i < N; ++i) ok = ok && ll_ep(w[i][0]) == ep && ll_ep(w[i][1]) == ep;
        if (ok) {
            if (tr) smem_ref().wll += clock64() - t0;
            return true;
        }
        ++spins;
        if ((spins & 63u) == 0) {
            if (aborted(P)) return false;
            if (spins > kLLSpinLimit) {
                give_up(P);
                return false;
            }
        }
        __nanosleep(nap);
        nap = min(nap * 2u, 96u);
    }
}

// ------------------------------------------------------------------------------ phase geometry

__device__ __forceinline__ Kind kind_of(int p, int L) { return p == 5 * L ? K_HEAD : (Kind)(p % 5); }
__device__ __forceinline__ int64_t split_lo(int64_t total, int part, int parts) { return total * part / parts; }

__device__ __forceinline__ const Q4Dev* matrix_of(const Smem& sm, const Ctx& c, int p) {
    const Kind k = kind_of(p, c.L);
    if (k == K_HEAD) return &c.head;
    const LayerDev& L = sm.layers[p / 5];
    return k == K_QKV ? &L.qkv : k == K_OUT ? &L.out : k == K_IN ? &L.fin : &L.fout;
}
__device__ __forceinline__ const float* alpha_of(const Smem& sm, const Ctx& c, int p) {
    const Kind k = kind_of(p, c.L);
    if (k == K_HEAD) return c.out_norm;
    if (k == K_QKV) return sm.layers[p / 5].norm1;
    if (k == K_IN) return sm.layers[p / 5].norm2;
    return nullptr;
}

// Attention split of this CTA: head h = cta / nsplit, split s; ring slots [j0, j1).
struct Split {
    int h, s, j0, j1;
};
__device__ __forceinline__ Split split_of(int cta, int nsplit, int H, int len) {
    Split r;
    r.h = cta / nsplit;
    r.s = cta % nsplit;
    const int chunk = (len + nsplit - 1) / nsplit;
    r.j0 = min(len, r.s * chunk);
    r.j1 = r.h < H ? min(len, r.j0 + chunk) : r.j0;
    return r;
}

// Segments of phase p for this CTA: [norm weight] + weight runs, or one K/V segment.
__device__ __forceinline__ int weight_segs(const Range& r) { return r.units > 0 ? (r.units + r.ups - 1) / r.ups : 0; }
__device__ __forceinline__ int phase_segs(const Smem& sm, const MegaArgs& P, int p, int cta) {
    const Kind k = kind_of(p, P.c.L);
    if (k == K_ATT) return cta / P.nsplit < P.c.H ? 1 : 0;
    const int w = weight_segs(sm.rg[k]);
    return w == 0 ? 0 : w + (alpha_of(sm, P.c, p) ? 1 : 0);
}

// Weight segment k of a phase: units [ua, ua + nu), nr rows in the first run (pairs: both rows
// of every unit; linear_in: the gate rows, then as many value rows), scales after the nibbles.
struct WSeg {
    int ua, nu;
    int nr;
    uint32_t sc_base;
};
__device__ __forceinline__ WSeg wseg(const Range& r, bool gate, int k, int NB) {
    WSeg s;
    s.ua = k * r.ups;
    s.nu = min(r.ups, r.units - s.ua);
    s.nr = gate ? s.nu : min(2 * s.nu, r.n - 2 * s.ua);
    s.sc_base = (uint32_t)(gate ? 2 * s.nu : s.nr) * NB * 16u;
    return s;
}

// ------------------------------------------------------------------------------ producer

struct Prod {
    uint32_t issued;    // segments issued
    uint32_t released;  // segments known released
    uint32_t head;      // ring bytes allocated since launch (monotonic)
    uint32_t tail;      // end of the last released segment
};

// Lane 0 waits for the release of the oldest unreleased segment; every lane gets the answer.
__device__ __forceinline__ bool prod_wait_release(Smem& sm, const MegaArgs& P, Prod& q) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        const uint32_t j = q.released;
        unsigned long long* m = &sm.empty[j % kNBar];
        const uint32_t par = (j / kNBar) & 1u;
        uint32_t spins = 0;
        while (!mbar_wait_sleep(m, par, 2000u)) {
            if ((++spins & 15u) == 0) {
                if (aborted(P)) {
                    ok = 0;
                    break;
                }
                if (spins > kSleepLimit) {
                    give_up(P);
                    ok = 0;
                    break;
                }
            }
            __nanosleep(256);  // the producer is ahead anyway: leave the issue slots to the consumers
        }
    }
    ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
    if (ok) {
        q.tail = sm.seg_end[q.released % kNBar];
        ++q.released;
    }
    return ok != 0;
}

// Allocates `bytes` (a multiple of 128, at most kRing) in the ring, waiting for releases as
// needed; returns the offset, or ~0u after an abort.
__device__ __forceinline__ uint32_t prod_alloc(Smem& sm, const MegaArgs& P, Prod& q, uint32_t bytes) {
    uint32_t start = q.head;
    uint32_t off = start % kRing;
    if (off + bytes > kRing) {
        start += kRing - off;
        off = 0;
    }
    const uint32_t end = start + bytes;
    while (q.issued - q.released >= (uint32_t)kNBar || end - q.tail > kRing)
        if (!prod_wait_release(sm, P, q)) return ~0u;
    q.head = end;
    if ((threadIdx.x & 31) == 0) {
        sm.seg_off[q.issued % kNBar] = off;
        sm.seg_end[q.issued % kNBar] = end;
    }
    return off;
}

// One segment: up to 4 bulk copies (source, bytes, offset inside the segment).
struct Copies {
    const void* src[4];
    uint32_t bytes[4];
    uint32_t dst[4];
    int n;
    uint32_t total;
    __device__ void add(const void* s, uint32_t b, uint32_t d) {
        if (b == 0) return;
        src[n] = s;
        bytes[n] = b;
        dst[n] = d;
        ++n;
        total = max(total, d + b);
    }
};

__device__ __forceinline__ bool prod_issue(Smem& sm, const MegaArgs& P, Prod& q, const Copies& cp) {
    const uint32_t off = prod_alloc(sm, P, q, (max(cp.total, 16u) + 127u) & ~127u);
    if (off == ~0u) return false;
    if ((threadIdx.x & 31) == 0) {
        uint32_t tx = 0;
        for (int i = 0; i < cp.n; ++i) tx += cp.bytes[i];
        unsigned long long* m = &sm.full[q.issued % kNBar];
        mbar_expect_tx(m, tx);  // the producer's arrival; the phase completes when tx bytes land
        const uint32_t base = smem_addr(sm.ring) + off;
        for (int i = 0; i < cp.n; ++i) bulk_g2s(base + cp.dst[i], cp.src[i], cp.bytes[i], m);
    }
    __syncwarp();
    ++q.issued;
    return true;
}

// The producer warp: every segment of every phase of every frame, in consumption order.
// Returns the number of segments issued.
__device__ __noinline__ uint32_t producer(const MegaArgs& P, int cta) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int per_frame = 5 * c.L + 1;
    Prod q{0, 0, 0, 0};
    StreamState st = c.state[c.ids[0]];
    const int es = c.kv_f32 ? 4 : 2;
    const uint32_t slot_bytes = (uint32_t)c.HD * es;
    for (int f = 0; f < P.steps; ++f) {
        const int len = min(st.len + 1, c.ML);
        const int wp = st.write_pos;
        for (int p = 0; p < per_frame; ++p) {
            const Kind k = kind_of(p, c.L);
            if (k == K_ATT) {
                const Split sp = split_of(cta, P.nsplit, c.H, len);
                if (sp.h >= c.H) continue;
                if (p == K_ATT && f > 0) {
                    // the slots come from earlier frames: wait until every CTA has finished
                    // frame f - 1 (its K/V writes are released with that count)
                    int ok = 1;
                    if ((threadIdx.x & 31) == 0) {
                        const uint32_t target = (uint32_t)f * gridDim.x;
                        uint32_t spins = 0;
                        while ((int32_t)(ld_acquire(P.bar) - target) < 0) {
                            if ((++spins & 63u) == 0) {
                                if (aborted(P)) {
                                    ok = 0;
                                    break;
                                }
                                if (spins > kSpinLimit) {
                                    give_up(P);
                                    ok = 0;
                                    break;
                                }
                            }
                            __nanosleep(128);
                        }
                        // generic-proxy writes, now visible to this thread, before the bulk
                        // copies (async proxy) read them
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                    }
                    if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return q.issued;
                }
                const uint8_t* kb = static_cast<const uint8_t*>(c.kv) +
                                    ((int64_t)c.ids[0] * c.kv_stream_stride + (int64_t)(p / 5) * c.kv_layer_stride +
                                     (int64_t)sp.h * c.ML * c.HD) * es;
                const uint8_t* vb = kb + c.kv_half_stride * es;
                const uint32_t n = (uint32_t)(sp.j1 - sp.j0);
                Copies cp{};
                // slot wp is this frame's: it is read from the QKV output, never copied, so the
                // copies cannot race with its write
                const bool in = wp >= sp.j0 && wp < sp.j1;
                const int a1 = in ? wp : sp.j1;
                const int b0 = in ? wp + 1 : sp.j1;
                cp.add(kb + (int64_t)sp.j0 * slot_bytes, (uint32_t)(a1 - sp.j0) * slot_bytes, 0);
                cp.add(kb + (int64_t)b0 * slot_bytes, (uint32_t)(sp.j1 - b0) * slot_bytes,
                       (uint32_t)(b0 - sp.j0) * slot_bytes);
                cp.add(vb + (int64_t)sp.j0 * slot_bytes, (uint32_t)(a1 - sp.j0) * slot_bytes, n * slot_bytes);
                cp.add(vb + (int64_t)b0 * slot_bytes, (uint32_t)(sp.j1 - b0) * slot_bytes,
                       n * slot_bytes + (uint32_t)(b0 - sp.j0) * slot_bytes);
                cp.total = max(cp.total, 2 * n * slot_bytes);
                if (!prod_issue(sm, P, q, cp)) return q.issued;
                continue;
            }
            const Range r = sm.rg[k];
            const int nw = weight_segs(r);
            if (nw == 0) continue;
            if (const float* alpha = alpha_of(sm, c, p)) {
                Copies cp{};
                cp.add(alpha, (uint32_t)c.D * 4u, 0);
                if (!prod_issue(sm, P, q, cp)) return q.issued;
            }
            const Q4Dev* W = matrix_of(sm, c, p);
            const int NB = W->k >> 5;
            const bool gate = k == K_IN;
            for (int s = 0; s < nw; ++s) {
                const WSeg g = wseg(r, gate, s, NB);
                Copies cp{};
                const int ra = gate ? r.r0 + g.ua : r.r0 + 2 * g.ua;
                cp.add(W->nib + (int64_t)ra * NB, (uint32_t)g.nr * NB * 16u, 0);
                cp.add(W->scale + (int64_t)ra * NB, (uint32_t)g.nr * NB * 2u, g.sc_base);
                if (gate) {
                    const int rb = c.F + r.r0 + g.ua;
                    cp.add(W->nib + (int64_t)rb * NB, (uint32_t)g.nu * NB * 16u, (uint32_t)g.nu * NB * 16u);
                    cp.add(W->scale + (int64_t)rb * NB, (uint32_t)g.nu * NB * 2u, g.sc_base + (uint32_t)g.nu * NB * 2u);
                }
                if (!prod_issue(sm, P, q, cp)) return q.issued;
            }
        }
        st.len = min(st.len + 1, c.ML);
        st.write_pos = (st.write_pos + 1) % c.ML;
    }
    return q.issued;
}

// Every issued copy must land before the CTA's shared memory goes away: wait (bounded) for the
// full barriers of the last kNBar segments issued (older ones were consumed or waited already).
__device__ void producer_drain(Smem& sm, uint32_t issued) {
    if ((threadIdx.x & 31) != 0) return;
    const uint32_t first = issued > (uint32_t)kNBar ? issued - kNBar : 0u;
    for (uint32_t i = first; i < issued; ++i) {
        uint32_t spins = 0;
        while (!mbar_try_wait(&sm.full[i % kNBar], (i / kNBar) & 1u) && ++spins < kSpinLimit) {
        }
    }
}

// ------------------------------------------------------------------------------ input vectors

// dp4a limbs of one quad (elements 4q .. 4q+3) of block b = q / 8 into the CTA's input vector;
// called by all 32 lanes of a warp with 8 consecutive lanes holding the 8 quads of a block.
__device__ __forceinline__ void quad_limbs(Smem& sm, int q, int NB, float4 v) {
    quad_limbs_store(sm.limbs, sm.xs, q, NB, v, true);
}

// Sum over each group of W consecutive lanes.
template <int W>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Sum over the consumer threads in a fixed order; `rb` alternates the two scratch rows so
// back-to-back sums need one barrier each.
__device__ __forceinline__ float block_sum(float v, Smem& sm, uint32_t rb) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sm.red[rb][warp] = v;
    csync();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kCWarps; ++w) s += sm.red[rb][w];
    return s;
}

// Out of line: only the first layer's input uses it, and inlined it made every instantiation of
// prep_vector several KB larger.
__device__ __noinline__ float emb_val(const Ctx& c, const uint8_t* table, uint32_t row, int j) {
    const uint8_t* r = table + (int64_t)row * c.emb_row_bytes;
    switch (c.emb_type) {
        case EMB_BF16: return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(r)[j] << 16);
        case EMB_F32: return reinterpret_cast<const float*>(r)[j];
        case EMB_F16: return f16_to_f32_ieee(reinterpret_cast<const uint16_t*>(r)[j]);
        default: {  // Q4_0 row, gguf.rs:616-633
            const uint8_t* blk = r + (j >> 5) * 18;
            const float d = f16_to_f32_gguf((uint16_t)(blk[0] | (blk[1] << 8)));
            const int w = j & 31;
            const uint32_t byte = blk[2 + (w & 15)];
            return __fmul_rn(nib_m8(w < 16 ? (byte & 0xFu) : (byte >> 4)), d);
        }
    }
}

// The GEMV input of a phase, K floats, then RMSNorm with `alpha` (a ring segment) when alpha is
// not NULL (burn::nn::RmsNorm: (x / sqrt(mean(x^2) + 1e-8)) * alpha), then the limbs.
//   src == 0: the flagged buffer `ll` at epoch `ep`
//   src == 1: the frame input x0 = audio sum (xa) + text row (model.rs:640-646); the CTA also
//             keeps its own rows [own0, own1) in xown
// QN = quads per thread.  Ends with a consumer barrier.  Returns false after an abort.
template <int QN>
__device__ __noinline__ bool prep_vector(const MegaArgs& P, const uint64_t* ll, uint32_t ep, int K,
                                         const float* alpha, uint32_t rb, int src, const float* xa, uint32_t text,
                                         int own0, int own1) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int nq = K >> 2, NB = K >> 5;
    float4 v[QN];
    bool ok = true;
    if (src == 0) {
        // all of a thread's quads in one wait: their loads are in flight together, so a K = 8448
        // input costs one L2 round trip, not three (slots past the end re-read the last quad and
        // are dropped)
        const int t = threadIdx.x;
        uint64_t w[2 * QN][2];
        ok = ll_wait_n<2 * QN>(
            P,
            [=](int j) -> const uint64_t* {
                const int q = min(t + (j >> 1) * kCThreads, nq - 1);
                return ll + 4 * q + 2 * (j & 1);
            },
            ep, w);
#pragma unroll
        for (int i = 0; i < QN; ++i)
            v[i] = make_float4(ll_val(w[2 * i][0]), ll_val(w[2 * i][1]), ll_val(w[2 * i + 1][0]), ll_val(w[2 * i + 1][1]));
#pragma unroll
        for (int i = 0; i < QN; ++i)
            if (t + i * kCThreads >= nq) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
#pragma unroll
        for (int i = 0; i < QN; ++i) {
            const int q = threadIdx.x + i * kCThreads;
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (q < nq) {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(xa) + q);
                const int j = 4 * q;
                v[i] = make_float4(__fadd_rn(a.x, emb_val(c, c.emb_text, text, j)),
                                   __fadd_rn(a.y, emb_val(c, c.emb_text, text, j + 1)),
                                   __fadd_rn(a.z, emb_val(c, c.emb_text, text, j + 2)),
                                   __fadd_rn(a.w, emb_val(c, c.emb_text, text, j + 3)));
                const float vv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (j + u >= own0 && j + u < own1) sm.xown[j + u - own0] = vv[u];
            }
        }
    }
    if (alpha) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < QN; ++i) {
            ss = __fmaf_rn(v[i].x, v[i].x, ss);
            ss = __fmaf_rn(v[i].y, v[i].y, ss);
            ss = __fmaf_rn(v[i].z, v[i].z, ss);
            ss = __fmaf_rn(v[i].w, v[i].w, ss);
        }
        ss = block_sum(ss, sm, rb);
        // x * (1 / rms) instead of x / rms: within 1.5 ulp, below the 24-bit fixed-point step of
        // the limbs that follow
        const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-8f)));
#pragma unroll
        for (int i = 0; i < QN; ++i) {
            const int q = threadIdx.x + i * kCThreads;
            if (q < nq) {
                const float4 a = reinterpret_cast<const float4*>(alpha)[q];
                v[i].x = __fmul_rn(__fmul_rn(v[i].x, inv), a.x);
                v[i].y = __fmul_rn(__fmul_rn(v[i].y, inv), a.y);
                v[i].z = __fmul_rn(__fmul_rn(v[i].z, inv), a.z);
                v[i].w = __fmul_rn(__fmul_rn(v[i].w, inv), a.w);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < QN; ++i) {
        const int q = threadIdx.x + i * kCThreads;
        if (q < nq) quad_limbs(sm, q, NB, v[i]);  // nq is a multiple of 32: whole warps
    }
    csync();
    return ok;
}

__device__ __forceinline__ bool prep_any(const MegaArgs& P, const uint64_t* ll, uint32_t ep, int K, const float* alpha,
                                         uint32_t rb, int src, const float* xa, uint32_t text, int own0, int own1) {
    const int qn = (K / 4 + kCThreads - 1) / kCThreads;
    if (qn <= 2) return prep_vector<2>(P, ll, ep, K, alpha, rb, src, xa, text, own0, own1);
    if (qn <= 3) return prep_vector<3>(P, ll, ep, K, alpha, rb, src, xa, text, own0, own1);
    return prep_vector<5>(P, ll, ep, K, alpha, rb, src, xa, text, own0, own1);
}

// ------------------------------------------------------------------------------ GEMV

// One GEMV phase over this CTA's units (row pairs; linear_in: gate/value pairs), in segment
// order.  The residual phases (7 units) give each unit two warps; the others give each unit a
// group of 16 lanes (linear_in: 8), so a warp takes two (four) units per round.  A unit's lanes wait for its segment and split
// its blocks: every round ends in a shuffle reduction and an epilogue, so fewer rounds of longer
// block loops measured faster.  `seg0` is the global index of the phase's first weight segment.
// Returns false after an abort.
//   EPI_QKV    RoPE on the q and k pairs, flagged qkv words, K/V ring write (model.rs:426-449)
//   EPI_RESID  x rows += result (kept in xown), flagged x words               (model.rs:565, 570)
//   EPI_GATE   silu(gate) * value, flagged hidden words                       (model.rs:517-524)
//   EPI_LOGITS logits, this warp's best (value, lowest index) in wv / wi
template <int EPI>
__device__ __noinline__ bool gemv_phase(const MegaArgs& P, int p, uint32_t seg0, uint64_t* outb, uint32_t ep, int frame) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const Range r = sm.rg[kind_of(p, c.L)];
    const Q4Dev* W = matrix_of(sm, c, p);
    const int NB = W->k >> 5;
    const bool gate = EPI == EPI_GATE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint4* nibs = reinterpret_cast<const uint4*>(sm.ring);
    const uint16_t* scs = reinterpret_cast<const uint16_t*>(sm.ring);
    float best_v = -FLT_MAX;
    int best_i = 0x7FFFFFFF;
    bool ok = true;
    if (EPI == EPI_RESID && 2 * r.units <= kCWarps) {
        // few row pairs (the residual phases own D / 148 rows): two warps per pair, each over
        // alternate runs of 32 blocks, the halves added in shared memory
        const int u = warp >> 1, h = warp & 1;
        float va = 0.0f, vb = 0.0f;
        int ra = 0, rb = -1;
        if (u < r.units) {
            const int k = u / r.ups;
            ok = wait_seg(sm, P, seg0 + (uint32_t)k) && ok;
            const WSeg g = wseg(r, false, k, NB);
            const uint32_t base = sm.seg_off[(seg0 + (uint32_t)k) % kNBar];
            const int la = 2 * (u - g.ua);
            const bool two = la + 1 < g.nr;
            const int lb = two ? la + 1 : la;
            ra = r.r0 + 2 * u;
            rb = two ? ra + 1 : -1;
            const uint32_t na = (base + (uint32_t)la * NB * 16u) / 16u, nb = (base + (uint32_t)lb * NB * 16u) / 16u;
            const uint32_t sa = (base + g.sc_base + (uint32_t)la * NB * 2u) / 2u;
            const uint32_t sb = (base + g.sc_base + (uint32_t)lb * NB * 2u) / 2u;
            float acc_a = 0.0f, acc_b = 0.0f;
            for (int b = lane + 32 * h; b < NB; b += 64) {
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
            va = warp_sum(acc_a);
            vb = warp_sum(acc_b);
            if (h == 1 && lane == 0) sm.hpart[u] = make_float2(va, vb);
        }
        csync();
        if (u < r.units && h == 0 && lane == 0) {
            const float2 o = sm.hpart[u];
            const int oi = ra - r.r0;
            const float xa_ = __fadd_rn(__fadd_rn(va, o.x), sm.xown[oi]);
            sm.xown[oi] = xa_;
            ll_store(outb + ra, xa_, ep);
            if (rb >= 0) {
                const float xb_ = __fadd_rn(__fadd_rn(vb, o.y), sm.xown[oi + 1]);
                sm.xown[oi + 1] = xb_;
                ll_store(outb + rb, xb_, ep);
            }
        }
        return ok;
    }
    // The other phases (K = D, 21 or more units per CTA): a group of 16 lanes per unit (8 in
    // linear_in, 57 units), so a warp takes kPer units at a time; a missing unit of a group
    // repeats the first of the warp and is dropped.
    constexpr int kLanes = EPI == EPI_GATE ? 8 : EPI == EPI_RESID ? 32 : 16, kPer = 32 / kLanes;
    const int hsel = lane / kLanes, hl = lane % kLanes;
    for (int u0 = warp * kPer; u0 < r.units; u0 += kCWarps * kPer) {
        const bool mine = u0 + hsel < r.units;
        const int u = mine ? u0 + hsel : u0;
        const int k = u / r.ups;
        ok = wait_seg(sm, P, seg0 + (uint32_t)k) && ok;
        const WSeg g = wseg(r, gate, k, NB);
        const uint32_t base = sm.seg_off[(seg0 + (uint32_t)k) % kNBar];
        const int lu = u - g.ua;
        int ra, rb;
        uint32_t na, nb, sa, sb;  // ring offsets in uint4 / uint16 units
        if (gate) {
            ra = r.r0 + u;
            rb = c.F + r.r0 + u;
            na = (base + (uint32_t)lu * NB * 16u) / 16u;
            nb = (base + (uint32_t)(g.nu + lu) * NB * 16u) / 16u;
            sa = (base + g.sc_base + (uint32_t)lu * NB * 2u) / 2u;
            sb = (base + g.sc_base + (uint32_t)(g.nu + lu) * NB * 2u) / 2u;
        } else {
            const int la = 2 * lu;
            const bool two = la + 1 < g.nr;
            const int lb = two ? la + 1 : la;
            ra = r.r0 + 2 * u;
            rb = two ? ra + 1 : -1;
            na = (base + (uint32_t)la * NB * 16u) / 16u;
            nb = (base + (uint32_t)lb * NB * 16u) / 16u;
            sa = (base + g.sc_base + (uint32_t)la * NB * 2u) / 2u;
            sb = (base + g.sc_base + (uint32_t)lb * NB * 2u) / 2u;
        }
        float acc_a = 0.0f, acc_b = 0.0f;
        for (int b = hl; b < NB; b += kLanes) {
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
        float va = group_sum<kLanes>(acc_a), vb = group_sum<kLanes>(acc_b);
        if (hl != 0 || !mine) continue;
        if (EPI == EPI_RESID) {
            const int o = ra - r.r0;
            const float xa_ = __fadd_rn(va, sm.xown[o]);
            sm.xown[o] = xa_;
            ll_store(outb + ra, xa_, ep);
            if (rb >= 0) {
                const float xb_ = __fadd_rn(vb, sm.xown[o + 1]);
                sm.xown[o + 1] = xb_;
                ll_store(outb + rb, xb_, ep);
            }
        } else if (EPI == EPI_GATE) {
            // silu(x) = x * (1 / (1 + exp(-x)))
            const float sg = __fmul_rn(va, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-va))));
            ll_store(outb + ra, __fmul_rn(sg, vb), ep);
        } else if (EPI == EPI_LOGITS) {
            c.logits[ra] = va;
            if (c.desc->logits) c.desc->logits[(int64_t)frame * c.V + ra] = va;
            if (va > best_v || (va == best_v && ra < best_i)) {
                best_v = va;
                best_i = ra;
            }
            if (rb >= 0) {
                c.logits[rb] = vb;
                if (c.desc->logits) c.desc->logits[(int64_t)frame * c.V + rb] = vb;
                if (vb > best_v || (vb == best_v && rb < best_i)) {
                    best_v = vb;
                    best_i = rb;
                }
            }
        } else {  // EPI_QKV (row pairs are always complete: 3D is even)
            const int D = c.D, HD = c.HD;
            const int part = ra / D;
            const int within = ra - part * D;
            const int h = within / HD, d = within - h * HD;
            if (part < 2) {
                // RoPE::apply_rotation (model.rs:114-116) on the pair (2i, 2i+1)
                const float2 cs = sm.rope[d >> 1];
                const float re = __fsub_rn(__fmul_rn(va, cs.x), __fmul_rn(vb, cs.y));
                const float im = __fadd_rn(__fmul_rn(va, cs.y), __fmul_rn(vb, cs.x));
                va = re;
                vb = im;
            }
            ll_store(outb + ra, va, ep);
            ll_store(outb + ra + 1, vb, ep);
            if (part >= 1) {
                const int64_t off = (int64_t)c.ids[0] * c.kv_stream_stride + (int64_t)(p / 5) * c.kv_layer_stride +
                                    (part == 2 ? c.kv_half_stride : 0) + ((int64_t)h * c.ML + sm.st.write_pos) * HD + d;
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
    if (EPI == EPI_LOGITS) {
        // the best of the two 16-lane groups (lowest index on ties)
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best_v, 16);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, best_i, 16);
        if (ov > best_v || (ov == best_v && oi < best_i)) {
            best_v = ov;
            best_i = oi;
        }
        if (lane == 0) {
            sm.wv[warp] = best_v;
            sm.wi[warp] = best_i;
        }
    }
    return ok;
}

// ------------------------------------------------------------------------------ attention

// Split-KV attention of head h over ring slots [j0, j1) (model.rs:450-472), HD = 128.
//   - q, k and v of this frame (flagged qkv words) go to shared memory once;
//   - a warp takes 4 keys at a time, one per group of 8 lanes; a lane holds 16 dimensions
//     (interleaved so that the 16-byte loads of a group are contiguous) and keeps an
//     online-softmax state (max, sum of exp, sum of exp * v) for its group's keys; the key slots
//     come from the ring segment `seg`, the slot of this frame (write_pos) from q/k/v above;
//   - the 4 groups of a warp merge by shuffles, the 15 warps through shared memory with one
//     thread per dimension (warp order);
//   - split 0 of each head then merges the partials of the other splits (three groups of
//     threads over consecutive splits, then the groups in order) into
//     softmax(q.k^T * scale).v and publishes it; the other splits publish their partials.
// Returns false after an abort.
template <typename KT>
__device__ __noinline__ bool attention_phase(const MegaArgs& P, int layer, uint32_t seg, uint32_t ep, int cta) {
    constexpr int HD = 128;
    constexpr int EPL = 16 / (int)sizeof(KT);  // elements of one 16-byte load
    constexpr int CH = 16 / EPL;               // 16-byte loads per lane for 16 dimensions
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int len = min(sm.st.len + 1, c.ML);
    const int wpos = sm.st.write_pos;
    const Split sp = split_of(cta, P.nsplit, c.H, len);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int h = sp.h, par = layer & 1;
    float* qs = reinterpret_cast<float*>(sm.limbs);  // [3][128]: q, k, v of this frame
    float* wst = qs + 3 * HD;                        // [15][HD + 4]: m, l, unused, unused, o[HD]
    bool ok = wait_seg(sm, P, seg);
    if (t < 3 * HD / 2) {
        const int part = t / (HD / 2), i = (t % (HD / 2)) * 2;
        const uint64_t* a = P.qkvb[par] + part * c.D + h * HD + i;
        uint64_t w[1][2];
        ok = ll_wait_n<1>(P, [=](int) -> const uint64_t* { return a; }, ep - 1u, w) && ok;
        qs[part * HD + i] = ll_val(w[0][0]);
        qs[part * HD + i + 1] = ll_val(w[0][1]);
    }
    csync();
    trace_mark(P, 21, lslot(layer, 3));
    const int g = lane >> 3, sub = lane & 7;
    // lane dimension i (0..15) is dims(i) = (i / EPL) * 8 * EPL + sub * EPL + i % EPL
    float q[16], o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        q[i] = qs[(i / EPL) * 8 * EPL + sub * EPL + i % EPL];
        o[i] = 0.0f;
    }
    const uint32_t base = sm.seg_off[seg % kNBar];
    const int n = sp.j1 - sp.j0;
    const uint8_t* ks = sm.ring + base;
    const uint8_t* vs = ks + (uint32_t)n * HD * sizeof(KT);
    float m = -FLT_MAX, l = 0.0f;
    for (int jb = sp.j0 + warp * 4; jb < sp.j1; jb += 4 * kCWarps) {
        const int j = jb + g;
        const bool valid = j < sp.j1;
        const bool cur = j == wpos;
        const int rr = valid && !cur ? j - sp.j0 : 0;
        float kv[16];
        if (cur) {
            // this frame's key (the ring copy stores it rounded to the ring type)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float x = qs[HD + (i / EPL) * 8 * EPL + sub * EPL + i % EPL];
                kv[i] = sizeof(KT) == 4 ? x : __bfloat162float(__float2bfloat16_rn(x));
            }
        } else {
#pragma unroll
            for (int ch = 0; ch < CH; ++ch) {
                const uint4 r = *reinterpret_cast<const uint4*>(ks + ((size_t)rr * HD + ch * 8 * EPL + sub * EPL) * sizeof(KT));
                if (sizeof(KT) == 4) {
                    kv[ch * 4 + 0] = __uint_as_float(r.x);
                    kv[ch * 4 + 1] = __uint_as_float(r.y);
                    kv[ch * 4 + 2] = __uint_as_float(r.z);
                    kv[ch * 4 + 3] = __uint_as_float(r.w);
                } else {
                    const uint32_t wv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        kv[ch * 8 + 2 * e] = __uint_as_float(wv[e] << 16);
                        kv[ch * 8 + 2 * e + 1] = __uint_as_float(wv[e] & 0xFFFF0000u);
                    }
                }
            }
        }
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) dot = __fmaf_rn(q[i], kv[i], dot);
        dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 1);
        dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 2);
        dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 4);
        if (!valid) continue;
        // value row
        if (cur) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float x = qs[2 * HD + (i / EPL) * 8 * EPL + sub * EPL + i % EPL];
                kv[i] = sizeof(KT) == 4 ? x : __bfloat162float(__float2bfloat16_rn(x));
            }
        } else {
#pragma unroll
            for (int ch = 0; ch < CH; ++ch) {
                const uint4 r = *reinterpret_cast<const uint4*>(vs + ((size_t)rr * HD + ch * 8 * EPL + sub * EPL) * sizeof(KT));
                if (sizeof(KT) == 4) {
                    kv[ch * 4 + 0] = __uint_as_float(r.x);
                    kv[ch * 4 + 1] = __uint_as_float(r.y);
                    kv[ch * 4 + 2] = __uint_as_float(r.z);
                    kv[ch * 4 + 3] = __uint_as_float(r.w);
                } else {
                    const uint32_t wv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        kv[ch * 8 + 2 * e] = __uint_as_float(wv[e] << 16);
                        kv[ch * 8 + 2 * e + 1] = __uint_as_float(wv[e] & 0xFFFF0000u);
                    }
                }
            }
        }
        const float score = __fmul_rn(dot, c.attn_scale);
        const float mn = fmaxf(m, score);
        const float corr = expf(m - mn);
        const float pr = expf(score - mn);
        l = __fmaf_rn(l, corr, pr);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = __fmaf_rn(o[i], corr, __fmul_rn(pr, kv[i]));
        m = mn;
    }
    // merge the 4 key groups of the warp (lanes with the same sub); the lower group keeps its
    // terms first
#pragma unroll
    for (int x = 8; x <= 16; x <<= 1) {
        const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m, x), l2 = __shfl_xor_sync(0xFFFFFFFFu, l, x);
        float o2[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) o2[i] = __shfl_xor_sync(0xFFFFFFFFu, o[i], x);
        const bool low = (lane & x) == 0;
        const float ma = low ? m : m2, la = low ? l : l2, mb = low ? m2 : m, lb = low ? l2 : l;
        if (lb != 0.0f) {
            if (la == 0.0f) {
                m = mb;
                l = lb;
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = low ? o2[i] : o[i];
            } else {
                const float M = fmaxf(ma, mb);
                const float fa = expf(ma - M), fb = expf(mb - M);
                l = __fmaf_rn(la, fa, __fmul_rn(lb, fb));
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float oa = low ? o[i] : o2[i], ob = low ? o2[i] : o[i];
                    o[i] = __fmaf_rn(oa, fa, __fmul_rn(ob, fb));
                }
                m = M;
            }
        } else if (la != 0.0f) {
            m = ma;
            l = la;
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = low ? o[i] : o2[i];
        }
    }
    if (g == 0) {
        float* d = wst + warp * (HD + 4);
        if (sub == 0) {
            d[0] = m;
            d[1] = l;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) d[4 + (i / EPL) * 8 * EPL + sub * EPL + i % EPL] = o[i];
    }
    csync();
    // 128 threads: the warps' states merged per dimension (warp order)
    float M = -FLT_MAX, L = 0.0f, O = 0.0f;
    if (t < HD) {
        for (int w = 0; w < kCWarps; ++w)
            if (wst[w * (HD + 4) + 1] != 0.0f) M = fmaxf(M, wst[w * (HD + 4)]);
        for (int w = 0; w < kCWarps; ++w) {
            const float lw = wst[w * (HD + 4) + 1];
            if (lw == 0.0f) continue;
            const float f = expf(wst[w * (HD + 4)] - M);
            L = __fmaf_rn(lw, f, L);
            O = __fmaf_rn(wst[w * (HD + 4) + 4 + t], f, O);
        }
    }
    trace_mark(P, 22, lslot(layer, 4));
    uint64_t* pb = P.partb[par] + (int64_t)h * P.nsplit * kPartPairs;
    if (sp.s != 0) {
        if (t < HD) {
            uint64_t* d = pb + (int64_t)sp.s * kPartPairs;
            if (t == 0) {
                ll_store(d, M, ep);
                ll_store(d + 1, L, ep);
            }
            ll_store(d + 4 + t, O, ep);
        }
        return ok;
    }
    // split 0: threads 0-127, 128-255 and 256-383 (one dimension each) merge three consecutive
    // ranges of the other splits, three splits a poll round; group 0 starts from this split's
    // own state
    const int grp = t / HD, dim = t % HD;
    const int others = P.nsplit - 1;
    const int per = (others + 2) / 3;
    const int s_lo = 1 + min(others, grp * per), s_hi = 1 + min(others, (grp + 1) * per);
    float gm = grp == 0 ? M : -FLT_MAX, gl = grp == 0 ? L : 0.0f, go = grp == 0 ? O : 0.0f;
    if (grp < 3) {
        for (int s0 = s_lo; s0 < s_hi; s0 += 3) {
            uint64_t w[6][2];
            ok = ll_wait_n<6>(
                     P,
                     [=](int i) -> const uint64_t* {
                         const int s = min(s0 + (i >> 1), s_hi - 1);
                         const uint64_t* d = pb + (int64_t)s * kPartPairs;
                         return (i & 1) ? d + 4 + (dim & ~1) : d;
                     },
                     ep, w) &&
                 ok;
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                if (s0 + i >= s_hi) break;
                const float ms = ll_val(w[2 * i][0]), ls = ll_val(w[2 * i][1]);
                const float os = ll_val(w[2 * i + 1][dim & 1]);
                if (ls == 0.0f) continue;
                if (gl == 0.0f) {
                    gm = ms;
                    gl = ls;
                    go = os;
                    continue;
                }
                const float Mx = fmaxf(gm, ms);
                const float fa = expf(gm - Mx), fb = expf(ms - Mx);
                gl = __fmaf_rn(gl, fa, __fmul_rn(ls, fb));
                go = __fmaf_rn(go, fa, __fmul_rn(os, fb));
                gm = Mx;
            }
        }
    }
    float* gst = wst;  // the warps' states are no longer needed: [grp][3] = m, l, o per dimension
    csync();
    if (grp >= 1 && grp < 3) {
        gst[(grp - 1) * 3 * HD + dim] = gm;
        gst[(grp - 1) * 3 * HD + HD + dim] = gl;
        gst[(grp - 1) * 3 * HD + 2 * HD + dim] = go;
    }
    csync();
    trace_mark(P, 24, lslot(layer, 5));
    if (t < HD) {
        for (int k = 0; k < 2; ++k) {
            const float ms = gst[k * 3 * HD + t], ls = gst[k * 3 * HD + HD + t], os = gst[k * 3 * HD + 2 * HD + t];
            if (ls == 0.0f) continue;
            if (gl == 0.0f) {
                gm = ms;
                gl = ls;
                go = os;
                continue;
            }
            const float Mx = fmaxf(gm, ms);
            const float fa = expf(gm - Mx), fb = expf(ms - Mx);
            gl = __fmaf_rn(gl, fa, __fmul_rn(ls, fb));
            go = __fmaf_rn(go, fa, __fmul_rn(os, fb));
            gm = Mx;
        }
        ll_store(P.attb[par] + h * HD + t, __fdiv_rn(go, gl), ep);
    }
    return ok;
}

// ------------------------------------------------------------------------------ consumers

__device__ __forceinline__ void release_phase(Smem& sm, uint32_t first, int n) {
    if (threadIdx.x == 0)
        for (int i = 0; i < n; ++i) mbar_arrive(&sm.empty[(first + (uint32_t)i) % kNBar]);
}

// Makes an abort seen by any consumer thread CTA-uniform; returns false when the CTA must stop.
// Agreement k uses slot k & 1, so a thread that is already writing agreement k + 1 can never
// change what a slower thread reads for agreement k.
__device__ __forceinline__ bool agree(Smem& sm, const MegaArgs& P, bool ok, uint32_t& k) {
    const uint32_t s = k & 1u;
    ++k;
    if (!ok || (threadIdx.x == 0 && aborted(P))) sm.stop[s] = 1;
    csync();
    return sm.stop[s] == 0;
}

// A frame's last step: every CTA reduces the per-CTA (best logit, index) words identically
// (lowest index on ties), applies the stream rule (stream.rs:90-107, 231-266) and advances the
// state.  Returns false after an abort.
__device__ __noinline__ bool argmax_phase(const MegaArgs& P, int f, uint32_t ep) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t* ab = P.argb[f & 1];
    bool ok = true;
    float bv = -FLT_MAX;
    int bi = 0x7FFFFFFF;
    if ((int)threadIdx.x < (int)gridDim.x) {
        const uint64_t* a = ab + 2 * threadIdx.x;
        uint64_t w[1][2];
        ok = ll_wait_n<1>(P, [=](int) -> const uint64_t* { return a; }, ep, w);
        bv = ll_val(w[0][0]);
        bi = (int)(uint32_t)w[0][1];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        sm.av[warp] = bv;
        sm.ai[warp] = bi;
    }
    csync();
    bv = -FLT_MAX;
    bi = 0x7FFFFFFF;
    for (int w = 0; w < kCWarps; ++w)
        if (sm.av[w] > bv || (sm.av[w] == bv && sm.ai[w] < bi)) {
            bv = sm.av[w];
            bi = sm.ai[w];
        }
    const uint32_t token = (uint32_t)(bi < 0 || bi >= c.V ? 0 : bi);
    StreamState st = sm.st;
    st.write_pos = (st.write_pos + 1) % c.ML;
    st.offset += 1;
    st.len = min(st.len + 1, c.ML);
    int32_t out = (int32_t)token;
    if (c.desc->mode == 1) {
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
    csync();  // every thread has read sm.st and sm.av
    if (threadIdx.x == 0) {
        sm.st = st;
        if (blockIdx.x == 0) {
            c.desc->tokens[f] = out;
            c.state[c.ids[0]] = st;
            if (f + 1 == P.steps) c.desc->step = P.steps;
        }
    }
    return ok;
}

__device__ __noinline__ void consumers(const MegaArgs& P, int cta) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int ph = 5 * c.L;  // the head's step
    const uint32_t ebase = *P.base;
    const int own0 = sm.rg[K_OUT].r0, own1 = sm.rg[K_OUT].r0 + sm.rg[K_OUT].n;
    uint32_t seg = 0;  // global index of the next segment to consume
    uint32_t rb = 0;
    uint32_t agreements = 0;
    for (int f = 0; f < P.steps; ++f) {
        if (threadIdx.x == 0) {
            if (sm.tron) trace_wall(P);  // end of the traced frame
            sm.tron = P.trace != nullptr && cta == 0 && f == P.trace_frame;
            sm.tall = P.tctas != nullptr && f == P.trace_frame;
        }
        trace_wall(P);
        trace_mark(P, 1, 0);
        const uint32_t E = ebase + (uint32_t)f * kEpochsPerFrame + 1u;  // epoch of step 0
        if (threadIdx.x == 0) {
            uint32_t text = c.desc->text ? __ldcg(c.desc->text + f) : sm.st.last_text;
            if (text >= (uint32_t)c.TV) {
                raise_error(c.desc, -1);
                text = 0;
            }
            sm.text = text;
        }
        if (threadIdx.x < (c.HD >> 1))
            sm.rope[threadIdx.x] = c.rope[(int64_t)sm.st.offset * (c.HD >> 1) + threadIdx.x];
        csync();
        bool ok = true;
        for (int l = 0; l < c.L && ok; ++l) {
            const int p0 = 5 * l, par = l & 1;
            // ---- QKV
            {
                const int n = phase_segs(sm, P, p0, cta);
                if (n > 0) {
                    ok = wait_seg(sm, P, seg) && ok;
                    const float* alpha = reinterpret_cast<const float*>(sm.ring + sm.seg_off[seg % kNBar]);
                    if (l == 0)
                        ok = prep_any(P, nullptr, 0, c.D, alpha, rb, 1, P.xa + (int64_t)f * c.D, sm.text, own0, own1) && ok;
                    else
                        ok = prep_any(P, P.xb[par ^ 1][1], E + (uint32_t)(p0 - 1), c.D, alpha, rb, 0, nullptr, 0, 0, 0) && ok;
                    rb ^= 1u;
                    trace_mark(P, 11, lslot(l, 0));
                    ok = gemv_phase<EPI_QKV>(P, p0, seg + 1, P.qkvb[par], E + (uint32_t)p0, f) && ok;
                    trace_mark(P, 12, lslot(l, 1));
                } else if (l == 0) {
                    // no QKV rows here, but the residual still needs x0's own rows
                    ok = prep_any(P, nullptr, 0, c.D, nullptr, rb, 1, P.xa + (int64_t)f * c.D, sm.text, own0, own1) && ok;
                }
                csync();
                trace_mark(P, 13, lslot(l, 2));
                trace_waits(P, 1);
                release_phase(sm, seg, n);
                seg += (uint32_t)n;
            }
            // ---- attention
            {
                const int n = phase_segs(sm, P, p0 + K_ATT, cta);
                if (n > 0) {
                    if (c.kv_f32)
                        ok = attention_phase<float>(P, l, seg, E + (uint32_t)(p0 + K_ATT), cta) && ok;
                    else
                        ok = attention_phase<__nv_bfloat16>(P, l, seg, E + (uint32_t)(p0 + K_ATT), cta) && ok;
                }
                csync();
                trace_mark(P, 23, lslot(l, 6));
                trace_waits(P, 2);
                release_phase(sm, seg, n);
                seg += (uint32_t)n;
            }
            // ---- out_proj + residual
            {
                const int n = phase_segs(sm, P, p0 + K_OUT, cta);
                if (n > 0) {
                    // stall_test: in frame 0 of a launch, layer 0's out_proj input is awaited at an
                    // epoch that no phase publishes, so the bounded wait runs out and the launch ends
                    // through the same abort path as a real timeout
                    const uint32_t ep_att = E + (uint32_t)(p0 + K_ATT);
                    const uint32_t ep_wait = (P.stall_test && f == 0 && l == 0) ? (ep_att ^ 0x80000000u) : ep_att;
                    ok = prep_any(P, P.attb[par], ep_wait, c.D, nullptr, rb, 0, nullptr, 0, 0, 0) && ok;
                    trace_mark(P, 31, lslot(l, 7));
                    ok = gemv_phase<EPI_RESID>(P, p0 + K_OUT, seg, P.xb[par][0], E + (uint32_t)(p0 + K_OUT), f) && ok;
                    trace_mark(P, 32, lslot(l, 8));
                }
                csync();
                trace_mark(P, 33, lslot(l, 9));
                trace_waits(P, 3);
                release_phase(sm, seg, n);
                seg += (uint32_t)n;
            }
            // ---- linear_in + silu gate
            {
                const int n = phase_segs(sm, P, p0 + K_IN, cta);
                if (n > 0) {
                    ok = wait_seg(sm, P, seg) && ok;
                    const float* alpha = reinterpret_cast<const float*>(sm.ring + sm.seg_off[seg % kNBar]);
                    ok = prep_any(P, P.xb[par][0], E + (uint32_t)(p0 + K_OUT), c.D, alpha, rb, 0, nullptr, 0, 0, 0) && ok;
                    rb ^= 1u;
                    trace_mark(P, 41, lslot(l, 10));
                    ok = gemv_phase<EPI_GATE>(P, p0 + K_IN, seg + 1, P.hidb[par], E + (uint32_t)(p0 + K_IN), f) && ok;
                    trace_mark(P, 42, lslot(l, 11));
                }
                csync();
                trace_mark(P, 43, lslot(l, 12));
                trace_waits(P, 4);
                release_phase(sm, seg, n);
                seg += (uint32_t)n;
            }
            // ---- linear_out + residual
            {
                const int n = phase_segs(sm, P, p0 + K_DOWN, cta);
                if (n > 0) {
                    ok = prep_any(P, P.hidb[par], E + (uint32_t)(p0 + K_IN), c.F, nullptr, rb, 0, nullptr, 0, 0, 0) && ok;
                    trace_mark(P, 51, lslot(l, 13));
                    ok = gemv_phase<EPI_RESID>(P, p0 + K_DOWN, seg, P.xb[par][1], E + (uint32_t)(p0 + K_DOWN), f) && ok;
                    trace_mark(P, 52, lslot(l, 14));
                }
                ok = agree(sm, P, ok, agreements);  // includes the phase-end barrier
                trace_mark(P, 53, lslot(l, 15));
                trace_waits(P, 5);
                release_phase(sm, seg, n);
                seg += (uint32_t)n;
            }
        }
        if (!ok) break;
        // ---- head + this CTA's argmax partial
        {
            const int n = phase_segs(sm, P, ph, cta);
            if (threadIdx.x < kCWarps) {
                sm.wv[threadIdx.x] = -FLT_MAX;
                sm.wi[threadIdx.x] = 0x7FFFFFFF;
            }
            csync();
            if (n > 0) {
                ok = wait_seg(sm, P, seg) && ok;
                const float* alpha = reinterpret_cast<const float*>(sm.ring + sm.seg_off[seg % kNBar]);
                ok = prep_any(P, P.xb[(c.L - 1) & 1][1], E + (uint32_t)(ph - 1), c.D, alpha, rb, 0, nullptr, 0, 0, 0) && ok;
                rb ^= 1u;
                trace_mark(P, 61, lslot(c.L, 0));
                ok = gemv_phase<EPI_LOGITS>(P, ph, seg + 1, nullptr, 0, f) && ok;
                trace_mark(P, 62, lslot(c.L, 1));
            }
            csync();
            if (threadIdx.x == 0) {
                float bv = -FLT_MAX;
                int bi = 0x7FFFFFFF;
                for (int w = 0; w < kCWarps; ++w)
                    if (sm.wv[w] > bv || (sm.wv[w] == bv && sm.wi[w] < bi)) {
                        bv = sm.wv[w];
                        bi = sm.wi[w];
                    }
                uint64_t* d = P.argb[f & 1] + 2 * cta;
                ll_store(d, bv, E + (uint32_t)ph);
                ll_store(d + 1, __int_as_float(bi), E + (uint32_t)ph);
            }
            trace_mark(P, 63, lslot(c.L, 2));
                trace_waits(P, 6);
            release_phase(sm, seg, n);
            seg += (uint32_t)n;
        }
        ok = argmax_phase(P, f, E + (uint32_t)ph) && ok;
        trace_mark(P, 7, lslot(c.L, 3));
        // this CTA's K/V writes of the frame are done: publish them to the producers
        ok = agree(sm, P, ok, agreements);
        if (threadIdx.x == 0) red_release_add(P.bar, 1u);
        if (!ok) break;
    }
    if (threadIdx.x == 0) {
        if (sm.tron) trace_wall(P);
        // epochs of the next launch start after every epoch this one could have used
        if (cta == 0) *P.base = ebase + (uint32_t)P.steps * kEpochsPerFrame;
    }
}

__global__ void __launch_bounds__(kThreads, 1) mega_kernel(const __grid_constant__ MegaArgs P) {
    Smem& sm = smem_ref();
    const Ctx& c = P.c;
    const int cta = blockIdx.x, ncta = gridDim.x;
    for (int i = threadIdx.x; i < c.L; i += kThreads) sm.layers[i] = c.layers[i];
    if (threadIdx.x == 0) {
        for (int i = 0; i < kNBar; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sm.st = c.state[c.ids[0]];
        sm.stop[0] = sm.stop[1] = 0;
        sm.tslot = 0;
        sm.tron = 0;
        sm.wseg = sm.wll = 0;
        sm.tall = 0;
        // row ranges of this CTA (the same for every layer)
        auto pairs = [&](int rows, uint32_t row_bytes) {
            Range r;
            const int64_t U = (rows + 1) / 2;
            r.r0 = (int)(2 * split_lo(U, cta, ncta));
            r.n = max(0, (int)min((int64_t)rows, 2 * split_lo(U, cta + 1, ncta)) - r.r0);
            r.units = (r.n + 1) / 2;
            r.ups = max(1, (int)(kSegMax / (2u * row_bytes)));
            return r;
        };
        const uint32_t rowD = (uint32_t)(c.D / 32) * 18u, rowF = (uint32_t)(c.F / 32) * 18u;
        sm.rg[K_QKV] = pairs(3 * c.D, rowD);
        sm.rg[K_ATT] = Range{0, 0, 0, 1};
        sm.rg[K_OUT] = pairs(c.D, rowD);
        sm.rg[K_DOWN] = pairs(c.D, rowF);
        sm.rg[K_HEAD] = pairs(c.V, rowD);
        Range g;
        g.r0 = (int)split_lo(c.F, cta, ncta);
        g.n = (int)split_lo(c.F, cta + 1, ncta) - g.r0;
        g.units = g.n;
        g.ups = max(1, (int)(kSegMax / (2u * rowD)));
        sm.rg[K_IN] = g;
    }
    __syncthreads();
    if ((int)threadIdx.x >= kCThreads) {
        const uint32_t issued = producer(P, cta);
        producer_drain(sm, issued);
    } else {
        consumers(P, cta);
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

// Grid-barrier latency probe: `iters` back-to-back grid barriers (mode 0: release add on one
// counter + acquire poll; mode 1: the last arriver publishes a generation flag on another line).
__global__ void __launch_bounds__(kThreads, 1) barrier_probe_kernel(uint32_t* bar, int iters, int mode) {
    __shared__ int go;
    uint32_t* flag = bar + 32;  // 128 bytes away from the counter
    for (int i = 0; i < iters; ++i) {
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t gen = (uint32_t)i + 1u;
            int ok = 1;
            uint32_t spins = 0;
            if (mode == 0) {
                red_release_add(bar, 1u);
                while ((int32_t)(ld_acquire(bar) - gen * gridDim.x) < 0)
                    if (++spins > kSpinLimit || *(volatile uint32_t*)(bar + 1)) {
                        ok = 0;
                        break;
                    }
            } else {
                uint32_t old;
                asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(bar) : "memory");
                if (old == gen * gridDim.x - 1u) {
                    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(gen) : "memory");
                } else {
                    while ((int32_t)(ld_acquire(flag) - gen) < 0)
                        if (++spins > kSpinLimit || *(volatile uint32_t*)(bar + 1)) {
                            ok = 0;
                            break;
                        }
                }
            }
            if (!ok) atomicExch(bar + 1, 1u);
            go = ok;
        }
        __syncthreads();
        if (!go) return;
    }
}

// Scratch layout of the persistent kernel inside the stream set's scratch.
struct ScratchLayout {
    size_t bar, base, xb, qkvb, partb, attb, hidb, argb, total;
};
ScratchLayout scratch_layout(int num_sms, int D, int F, int H) {
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    const int ns = num_sms / (H > 0 ? H : 1);
    ScratchLayout s;
    size_t o = 0;
    s.bar = o;
    o += 256;
    s.base = o;
    o += 256;
    s.xb = o;
    o += up((size_t)4 * D * 8);
    s.qkvb = o;
    o += up((size_t)2 * 3 * D * 8);
    s.partb = o;
    o += up((size_t)2 * H * ns * kPartPairs * 8);
    s.attb = o;
    o += up((size_t)2 * D * 8);
    s.hidb = o;
    o += up((size_t)2 * F * 8);
    s.argb = o;
    o += up((size_t)2 * num_sms * 2 * 8);
    s.total = o;
    return s;
}

}  // namespace

cudaError_t mega_barrier_probe(void* scratch, int iters, int mode, float* ms_out) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    uint32_t* bar = static_cast<uint32_t*>(scratch);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    e = cudaMemset(bar, 0, 256);
    void* args[] = {(void*)&bar, (void*)&iters, (void*)&mode};
    if (e == cudaSuccess) e = cudaEventRecord(a, 0);
    if (e == cudaSuccess)
        e = cudaLaunchCooperativeKernel((const void*)barrier_probe_kernel, dim3(sms), dim3(kThreads), args, 0, 0);
    if (e == cudaSuccess) e = cudaEventRecord(b, 0);
    if (e == cudaSuccess) e = cudaEventSynchronize(b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms_out, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return e;
}

bool mega_supported(int L, int D, int F, int HD, int V, int num_sms, int ML, int kv_f32) {
    if (std::getenv("STT_DISABLE_MEGA") != nullptr) return false;
    if (HD != 128 || D % 256 != 0 || D > 4096 || F % 256 != 0 || F > kMaxK || L < 1 || L > kMaxL) return false;
    const int H = D / HD;
    if (H < 1 || H > num_sms || num_sms > kCThreads) return false;
    if ((uint32_t)(5 * L + 2) > kEpochsPerFrame) return false;
    const int nsplit = num_sms / H;
    // a CTA keeps its x rows in xown
    if (2 * ((D / 2 + num_sms - 1) / num_sms) > kMaxOwnRows) return false;
    // every phase of one CTA must fit the ring at once (segments are released per phase), with
    // room for the alignment of each segment and one wrap of the ring
    auto phase_fits = [&](int units, uint32_t unit_bytes, uint32_t alpha_bytes) {
        const uint32_t ups = std::max<uint32_t>(1u, kSegMax / unit_bytes);
        const uint32_t segs = (uint32_t)(units + ups - 1) / ups;
        const uint64_t bytes = (uint64_t)units * unit_bytes + alpha_bytes + (segs + 1) * 128u + (uint64_t)ups * unit_bytes;
        return bytes <= kRing && segs + 1 <= (uint32_t)kNBar / 2;
    };
    const uint32_t rowD = (uint32_t)(D / 32) * 18u, rowF = (uint32_t)(F / 32) * 18u;
    auto per = [&](int64_t units) { return (int)((units + num_sms - 1) / num_sms); };
    if (!phase_fits(per(3 * D / 2), 2 * rowD, (uint32_t)D * 4)) return false;
    if (!phase_fits(per(D / 2), 2 * rowD, 0)) return false;
    if (!phase_fits(per(F), 2 * rowD, (uint32_t)D * 4)) return false;
    if (!phase_fits(per(D / 2), 2 * rowF, 0)) return false;
    if (!phase_fits(per((V + 1) / 2), 2 * rowD, (uint32_t)D * 4)) return false;
    const uint64_t kv = (uint64_t)((ML + nsplit - 1) / nsplit) * HD * (kv_f32 ? 4 : 2) * 2 + 256;
    return kv <= kRing;
}

size_t mega_scratch_bytes(int num_sms, int D, int F, int V, int H, int HD) {
    return scratch_layout(num_sms, D, F, H).total;
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
    const ScratchLayout sl = scratch_layout(sms, c.D, c.F, c.H);
    uint8_t* s = static_cast<uint8_t*>(ms.scratch);
    MegaArgs P;
    P.c = c;
    P.steps = steps;
    P.nsplit = sms / c.H;
    if (P.nsplit < 1) return cudaErrorInvalidConfiguration;
    P.bar = reinterpret_cast<uint32_t*>(s + sl.bar);
    P.base = reinterpret_cast<uint32_t*>(s + sl.base);
    P.xa = ms.xa_all;
    uint64_t* xb = reinterpret_cast<uint64_t*>(s + sl.xb);
    for (int i = 0; i < 2; ++i) {
        P.xb[i][0] = xb + (size_t)(2 * i) * c.D;
        P.xb[i][1] = xb + (size_t)(2 * i + 1) * c.D;
        P.qkvb[i] = reinterpret_cast<uint64_t*>(s + sl.qkvb) + (size_t)i * 3 * c.D;
        P.partb[i] = reinterpret_cast<uint64_t*>(s + sl.partb) + (size_t)i * c.H * P.nsplit * kPartPairs;
        P.attb[i] = reinterpret_cast<uint64_t*>(s + sl.attb) + (size_t)i * c.D;
        P.hidb[i] = reinterpret_cast<uint64_t*>(s + sl.hidb) + (size_t)i * c.F;
        P.argb[i] = reinterpret_cast<uint64_t*>(s + sl.argb) + (size_t)i * sms * 2;
    }
    P.trace = nullptr;
    P.trace_frame = -1;
    P.trace_cap = 0;
    P.tctas = nullptr;
    P.tslots = 0;
    P.stall_test = ms.stall_next;
    ms.stall_next = 0;
    if (ms.trace && ms.trace_frame >= 0) {
        P.trace = ms.trace;
        P.trace_frame = ms.trace_frame;
        P.trace_cap = ms.trace_cap;
        P.tctas = ms.trace_ctas;
        P.tslots = ms.trace_slots;
    }
    e = cudaMemsetAsync(P.bar, 0, 256, st);
    if (e != cudaSuccess) return e;
    audio_sum_kernel<<<dim3((c.D + 255) / 256, steps), 256, 0, st>>>(c, ms.xa_all);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    void* args[] = {(void*)&P};
    return cudaLaunchCooperativeKernel((const void*)mega_kernel, dim3(sms), dim3(kThreads), args, sizeof(Smem), st);
}

}  // namespace stt
