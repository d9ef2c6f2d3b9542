// Persistent single-stream decode step for sm_100a.
//
// One cooperative launch of one 512-thread CTA per SM runs `steps` whole frames of one stream:
//   per layer   QKV -> attention -> out_proj -> linear_in -> linear_out, a grid barrier after each
//   per frame   head GEMV + per-CTA argmax -> barrier -> every CTA reduces the argmax, applies the
//               stream rule, and builds the next frame's input from the audio sum precomputed in
//               the head phase plus the text row.
// The weight bytes (627 MB per frame) dwarf everything else, so the kernel is organised around
// keeping HBM streaming:
//   - each CTA owns fixed row ranges of every matrix and issues cp.async.bulk.prefetch.L2 for the
//     ranges of the coming phases (and the KV slots its attention split will read), keeping a byte
//     budget in flight ahead of its consumption, so the HBM queue never drains during barriers;
//   - the GEMV consumes those bytes at about 1.5 instructions per weight: the input vector is
//     turned into 24-bit fixed point per 32-element block (three byte limbs, shared exponent) and
//     every nibble goes through dp4a, which keeps the dot product of a block exact in integers;
//   - every spin (grid barrier) is bounded: on timeout the kernel raises STT_E_DEVICE_FLAG in the
//     step descriptor, sets an abort word that releases the other CTAs, and returns.
#include <cfloat>
#include <cstdlib>

#include "kernels.h"
#include "mega.h"

namespace stt {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kNBMax = 264;             // K / 32 for K <= 8448
constexpr int kMaxK = kNBMax * 32;
constexpr uint32_t kSpinLimit = 1u << 26;  // ~ seconds with the nanosleep back-off

struct MegaArgs {
    Ctx c;
    int32_t steps;
    int32_t nsplit;        // attention splits per head
    uint32_t* bar;         // [0] arrivals (monotonic), [1] abort, [2..2+H) head tickets
    float* xa;             // [D] audio-embedding sum of the next frame
    float* amax_v;         // [grid] per-CTA best logit
    int32_t* amax_i;       // [grid] and its index
    uint32_t pf_budget;    // L2 lookahead per CTA in bytes
    unsigned long long* trace;  // optional: globaltimer at every barrier entry/exit of one frame
    int32_t trace_frame;
    int32_t trace_cap;
};

struct Smem {
    uint4 limbs[6 * kNBMax];   // [vec][block]: L0,L1,L2 of element groups 0-3, then of groups 4-7
    float xs[kNBMax];          // 2^(e_b - 27): block scale of the fixed-point input (incl. 1/16)
    float xf[kMaxK];           // the input vector in f32
    float red[kWarps];
    float wv[kWarps];
    int32_t wi[kWarps];
    int32_t flag;
};

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
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

// Grid barrier: arrival counter with release/acquire and a bounded spin.  Returns false when the
// kernel must stop (timeout here or elsewhere).
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

struct Tracer {
    int slot = 0;
    bool on = false;
    __device__ void mark(const MegaArgs& P) {
        if (on && threadIdx.x == 0 && slot < P.trace_cap) P.trace[slot++] = globaltimer();
    }
};

__device__ bool grid_sync(const MegaArgs& P, uint32_t& epoch, Smem& sm, Tracer& tr) {
    __threadfence();
    __syncthreads();
    tr.mark(P);
    ++epoch;
    if (threadIdx.x == 0) {
        const uint32_t target = epoch * gridDim.x;
        atomicAdd(P.bar, 1u);
        int ok = 1;
        uint32_t spins = 0;
        for (;;) {
            if ((int32_t)(ld_acquire(P.bar) - target) >= 0) break;
            if (*(volatile uint32_t*)(P.bar + 1)) { ok = 0; break; }
            if (++spins > kSpinLimit) {
                atomicExch(P.bar + 1, 1u);
                raise_error(P.c.desc, -5);
                ok = 0;
                break;
            }
            if (spins > 32) __nanosleep(64);
        }
        __threadfence();
        sm.flag = ok;
    }
    __syncthreads();
    tr.mark(P);
    return sm.flag != 0;
}

__device__ __forceinline__ int64_t split_lo(int64_t total, int part, int parts) { return total * part / parts; }

// ------------------------------------------------------------------------------ phase geometry

enum Phase : int { PH_QKV = 0, PH_ATT = 1, PH_OUT = 2, PH_IN = 3, PH_DOWN = 4 };

struct Range {
    const void* p;
    uint32_t bytes;
};

// Byte ranges a CTA reads in global phase `gp` (frame-relative index gp % per_frame): at most 4.
__device__ int phase_ranges(const MegaArgs& P, int gp, int cta, int ncta, int len_next, Range* out) {
    const Ctx& c = P.c;
    const int per_frame = 5 * c.L + 1;
    const int p = gp % per_frame;
    int n = 0;
    auto q4 = [&](const Q4Dev& W, int64_t r0, int64_t r1) {
        if (r1 <= r0) return;
        const int64_t nb = W.k / 32;
        out[n++] = Range{W.nib + r0 * nb, (uint32_t)((r1 - r0) * nb * 16)};
        out[n++] = Range{W.scale + r0 * nb, (uint32_t)((r1 - r0) * nb * 2)};
    };
    if (p == 5 * c.L) {  // head
        const int64_t U = (c.V + 1) / 2;
        const int64_t r1 = 2 * split_lo(U, cta + 1, ncta);
        q4(c.head, 2 * split_lo(U, cta, ncta), r1 < c.V ? r1 : (int64_t)c.V);
        return n;
    }
    const int l = p / 5, k = p % 5;
    const LayerDev& L = c.layers[l];
    switch (k) {
        case PH_QKV: {
            const int64_t U = 3 * c.D / 2;
            q4(L.qkv, 2 * split_lo(U, cta, ncta), 2 * split_lo(U, cta + 1, ncta));
            break;
        }
        case PH_OUT: {
            const int64_t U = c.D / 2;
            q4(L.out, 2 * split_lo(U, cta, ncta), 2 * split_lo(U, cta + 1, ncta));
            break;
        }
        case PH_IN: {
            const int64_t u0 = split_lo(c.F, cta, ncta), u1 = split_lo(c.F, cta + 1, ncta);
            q4(L.fin, u0, u1);
            q4(L.fin, c.F + u0, c.F + u1);
            break;
        }
        case PH_DOWN: {
            const int64_t U = c.D / 2;
            q4(L.fout, 2 * split_lo(U, cta, ncta), 2 * split_lo(U, cta + 1, ncta));
            break;
        }
        default: {  // attention: K and V slots of this CTA's split (bf16 rings only)
            const int h = cta / P.nsplit, s = cta % P.nsplit;
            if (h >= c.H || c.kv_f32) break;
            const int chunk = (len_next + P.nsplit - 1) / P.nsplit;
            const int j0 = s * chunk, j1 = min(len_next, j0 + chunk);
            if (j1 <= j0) break;
            const int sid = c.ids[0];
            const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(c.kv) + (int64_t)sid * c.kv_stream_stride +
                                      (int64_t)l * c.kv_layer_stride + (int64_t)h * c.ML * c.HD;
            out[n++] = Range{kb + (int64_t)j0 * c.HD, (uint32_t)((j1 - j0) * c.HD * 2)};
            out[n++] = Range{kb + c.kv_half_stride + (int64_t)j0 * c.HD, (uint32_t)((j1 - j0) * c.HD * 2)};
            break;
        }
    }
    return n;
}

// Issues L2 prefetches for whole phases after `cur` until `budget` bytes are ahead.
struct Prefetcher {
    int next;          // next global phase to prefetch
    int limit;         // one past the last global phase of the launch
    __device__ void run(const MegaArgs& P, int cur, int cta, int ncta, int len_next_of_frame) {
        if (threadIdx.x != 0) return;
        uint32_t ahead = 0;
        Range r[4];
        // bytes already requested beyond the current phase
        for (int g = cur + 1; g < next; ++g) {
            const int n = phase_ranges(P, g, cta, ncta, len_next_of_frame, r);
            for (int i = 0; i < n; ++i) ahead += r[i].bytes;
        }
        while (next < limit && ahead < P.pf_budget) {
            const int n = phase_ranges(P, next, cta, ncta, len_next_of_frame, r);
            for (int i = 0; i < n; ++i) {
                const uint8_t* p = static_cast<const uint8_t*>(r[i].p);
                for (uint32_t o = 0; o < r[i].bytes; o += 65536u)
                    prefetch_l2(p + o, min(65536u, r[i].bytes - o));
                ahead += r[i].bytes;
            }
            ++next;
        }
    }
};

// ------------------------------------------------------------------------------ input vectors

// Builds the dp4a limbs of xf[0..K) (already in shared memory) for every 32-element block.
__device__ void build_limbs(Smem& sm, int K) {
    const int NB = K >> 5;
    for (int q = threadIdx.x; q < (K >> 2); q += kThreads) {  // quad q: elements 4q .. 4q+3
        const int b = q >> 3, g = q & 7;
        const float4 v = reinterpret_cast<const float4*>(sm.xf)[q];
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
}

__device__ float block_reduce_sum(float v, Smem& sm) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sm.red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int w = 0; w < kWarps; ++w) s += sm.red[w];
    __syncthreads();
    return s;
}

// xf = RMSNorm(src) with alpha (or a plain copy when alpha == NULL); src is read through L2.
__device__ void load_vector(Smem& sm, const float* src, int K, const float* alpha) {
    float ss = 0.0f;
    for (int j = threadIdx.x; j < K; j += kThreads) {
        const float v = __ldcg(src + j);
        sm.xf[j] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    if (alpha) {
        ss = block_reduce_sum(ss, sm);
        const float rms = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-8f));
        for (int j = threadIdx.x; j < K; j += kThreads) sm.xf[j] = __fmul_rn(__fdiv_rn(sm.xf[j], rms), alpha[j]);
    }
    __syncthreads();
    build_limbs(sm, K);
    __syncthreads();
}

// ------------------------------------------------------------------------------ GEMV

// sum over one Q4_0 block of (nibble - 8) * x, as 16 * sum in fixed point (S0 + 256 S1 + 65536 S2)
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

template <int EPI>
__device__ __forceinline__ void unit_rows_m(const Ctx& c, int u, int* ra, int* rb, int N) {
    if (EPI == EPI_GATE) {
        *ra = u;
        *rb = u + c.F;
    } else {
        *ra = 2 * u;
        *rb = 2 * u + 1 < N ? 2 * u + 1 : -1;
    }
}

struct HeadBest {
    float v;
    int i;
};

template <int EPI>
__device__ void gemv_phase(const MegaArgs& P, Smem& sm, const Q4Dev& W, int layer, const StreamState& st,
                           int cta, int ncta, HeadBest* best, int frame) {
    const Ctx& c = P.c;
    const int NB = W.k >> 5;
    const int64_t U = EPI == EPI_GATE ? c.F : (W.n + 1) / 2;
    const int64_t u0 = split_lo(U, cta, ncta), u1 = split_lo(U, cta + 1, ncta);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t u = u0 + warp; u < u1; u += kWarps) {
        int ra, rb;
        unit_rows_m<EPI>(c, (int)u, &ra, &rb, W.n);
        const int rb_ = rb >= 0 ? rb : ra;
        const uint4* na = W.nib + (int64_t)ra * NB;
        const uint4* nb = W.nib + (int64_t)rb_ * NB;
        const uint16_t* sa = W.scale + (int64_t)ra * NB;
        const uint16_t* sb = W.scale + (int64_t)rb_ * NB;
        float acc_a = 0.0f, acc_b = 0.0f;
        for (int b0 = lane; b0 < NB; b0 += 64) {
            const int b1 = b0 + 32;
            const bool has1 = b1 < NB;
            const uint4 qa0 = __ldg(na + b0), qb0 = __ldg(nb + b0);
            const uint4 qa1 = has1 ? __ldg(na + b1) : make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
            const uint4 qb1 = has1 ? __ldg(nb + b1) : make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
            const float da0 = f16_to_f32_ieee(__ldg(sa + b0)), db0 = f16_to_f32_ieee(__ldg(sb + b0));
            const float da1 = has1 ? f16_to_f32_ieee(__ldg(sa + b1)) : 0.0f;
            const float db1 = has1 ? f16_to_f32_ieee(__ldg(sb + b1)) : 0.0f;
            uint4 L[6];
#pragma unroll
            for (int v = 0; v < 6; ++v) L[v] = sm.limbs[v * NB + b0];
            const float x0 = sm.xs[b0];
            acc_a = __fmaf_rn(block_dp4a(qa0, L), __fmul_rn(da0, x0), acc_a);
            acc_b = __fmaf_rn(block_dp4a(qb0, L), __fmul_rn(db0, x0), acc_b);
            if (has1) {
#pragma unroll
                for (int v = 0; v < 6; ++v) L[v] = sm.limbs[v * NB + b1];
                const float x1 = sm.xs[b1];
                acc_a = __fmaf_rn(block_dp4a(qa1, L), __fmul_rn(da1, x1), acc_a);
                acc_b = __fmaf_rn(block_dp4a(qb1, L), __fmul_rn(db1, x1), acc_b);
            }
        }
        float va = warp_sum(acc_a), vb = warp_sum(acc_b);
        if (lane != 0) continue;
        if (EPI == EPI_RESID) {
            c.x[ra] = __fadd_rn(va, __ldcg(c.x + ra));
            if (rb >= 0) c.x[rb] = __fadd_rn(vb, __ldcg(c.x + rb));
        } else if (EPI == EPI_GATE) {
            const float sg = __fmul_rn(va, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-va))));
            c.hid[ra] = __fmul_rn(sg, vb);
        } else if (EPI == EPI_LOGITS) {
            c.logits[ra] = va;
            if (c.desc->logits) c.desc->logits[(int64_t)frame * c.V + ra] = va;
            if (va > best->v || (va == best->v && ra < best->i)) { best->v = va; best->i = ra; }
            if (rb >= 0) {
                c.logits[rb] = vb;
                if (c.desc->logits) c.desc->logits[(int64_t)frame * c.V + rb] = vb;
                if (vb > best->v || (vb == best->v && rb < best->i)) { best->v = vb; best->i = rb; }
            }
        } else {  // EPI_QKV: RoPE on q and k pairs, K/V ring write
            const int D = c.D, HD = c.HD;
            const int part = ra / D;
            const int within = ra - part * D;
            const int h = within / HD, d = within - h * HD;
            if (part < 2) {
                const float2 cs = c.rope[(int64_t)st.offset * (HD >> 1) + (d >> 1)];
                const float r = __fsub_rn(__fmul_rn(va, cs.x), __fmul_rn(vb, cs.y));
                const float im = __fadd_rn(__fmul_rn(va, cs.y), __fmul_rn(vb, cs.x));
                va = r;
                vb = im;
            }
            c.qkv[ra] = va;
            c.qkv[rb] = vb;
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

template <typename KT>
__device__ void attention_phase(const MegaArgs& P, Smem& sm, int layer, const StreamState& st, int cta) {
    const Ctx& c = P.c;
    const int NS = P.nsplit;
    const int h = cta / NS, s = cta % NS;
    if (h >= c.H) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int len = min(st.len + 1, c.ML);
    const int chunk = (len + NS - 1) / NS;
    const int j0 = s * chunk, j1 = min(len, j0 + chunk);
    const int HD = c.HD;
    const float4 q = __ldcg(reinterpret_cast<const float4*>(c.qkv + h * HD) + lane);
    const KT* kbase = reinterpret_cast<const KT*>(c.kv) + (int64_t)c.ids[0] * c.kv_stream_stride +
                      (int64_t)layer * c.kv_layer_stride + (int64_t)h * c.ML * HD;
    const KT* vbase = kbase + c.kv_half_stride;
    float m = -FLT_MAX, l = 0.0f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = j0 + warp; j < j1; j += kWarps) {
        float4 k, v;
        if (sizeof(KT) == 4) {
            k = __ldcg(reinterpret_cast<const float4*>(kbase + (int64_t)j * HD) + lane);
            v = __ldcg(reinterpret_cast<const float4*>(vbase + (int64_t)j * HD) + lane);
        } else {
            const uint2 kr = __ldcg(reinterpret_cast<const uint2*>(kbase + (int64_t)j * HD) + lane);
            const uint2 vr = __ldcg(reinterpret_cast<const uint2*>(vbase + (int64_t)j * HD) + lane);
            k = make_float4(__uint_as_float(kr.x << 16), __uint_as_float(kr.x & 0xFFFF0000u),
                            __uint_as_float(kr.y << 16), __uint_as_float(kr.y & 0xFFFF0000u));
            v = make_float4(__uint_as_float(vr.x << 16), __uint_as_float(vr.x & 0xFFFF0000u),
                            __uint_as_float(vr.y << 16), __uint_as_float(vr.y & 0xFFFF0000u));
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
    // combine the warps in warp order through shared memory (reuses xf as scratch)
    float* wm = sm.xf;              // [kWarps]
    float* wl = sm.xf + kWarps;     // [kWarps]
    float4* wo = reinterpret_cast<float4*>(sm.xf + 2 * kWarps);  // [kWarps][32]
    if (lane == 0) {
        wm[warp] = m;
        wl[warp] = l;
    }
    wo[warp * 32 + lane] = o;
    __syncthreads();
    float* part = c.part + ((int64_t)h * NS + s) * (HD + 4);
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
        if (lane == 0) {
            part[0] = M;
            part[1] = L;
        }
        reinterpret_cast<float4*>(part + 4)[lane] = O;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sm.flag = atomicAdd(P.bar + 2 + h, 1u) == (uint32_t)NS - 1u;
    __syncthreads();
    if (!sm.flag) return;
    __threadfence();
    if (warp == 0) {
        const float* pb = c.part + (int64_t)h * NS * (HD + 4);
        float M = -FLT_MAX;
        for (int t = 0; t < NS; ++t) M = fmaxf(M, __ldcg(pb + t * (HD + 4)));
        float L = 0.0f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int t = 0; t < NS; ++t) {
            const float lt = __ldcg(pb + t * (HD + 4) + 1);
            if (lt == 0.0f) continue;
            const float f = expf(__ldcg(pb + t * (HD + 4)) - M);
            L = __fmaf_rn(lt, f, L);
            const float4 ot = __ldcg(reinterpret_cast<const float4*>(pb + t * (HD + 4) + 4) + lane);
            O.x = __fmaf_rn(ot.x, f, O.x);
            O.y = __fmaf_rn(ot.y, f, O.y);
            O.z = __fmaf_rn(ot.z, f, O.z);
            O.w = __fmaf_rn(ot.w, f, O.w);
        }
        reinterpret_cast<float4*>(c.attn + h * HD)[lane] =
            make_float4(__fdiv_rn(O.x, L), __fdiv_rn(O.y, L), __fdiv_rn(O.z, L), __fdiv_rn(O.w, L));
        if (lane == 0) P.bar[2 + h] = 0u;
    }
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

// xa[j] for this CTA's slice of j: sum of the 32 audio rows of `frame` in codebook order.
__device__ void audio_sum_slice(const MegaArgs& P, int frame, int cta, int ncta) {
    const Ctx& c = P.c;
    const uint32_t* audio = c.desc->audio + (int64_t)frame * c.NC;
    const int j0 = (int)split_lo(c.D, cta, ncta), j1 = (int)split_lo(c.D, cta + 1, ncta);
    const int64_t table = (int64_t)c.AV * c.emb_row_bytes;
    for (int j = j0 + (int)threadIdx.x; j < j1; j += kThreads) {
        float acc = 0.0f;
        for (int cb = 0; cb < c.NC; ++cb) {
            uint32_t t = __ldcg(audio + cb);
            if (t >= (uint32_t)c.AV) {
                raise_error(c.desc, -1);
                t = 0;
            }
            acc = __fadd_rn(acc, emb_val(c, c.emb_audio + cb * table, t, j));
        }
        P.xa[j] = acc;
    }
}

// ------------------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kThreads, 1) mega_kernel(const __grid_constant__ MegaArgs P) {
    extern __shared__ uint4 smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const Ctx& c = P.c;
    const int cta = blockIdx.x, ncta = gridDim.x;
    uint32_t epoch = 0;
    const int sid = c.ids[0];
    StreamState st = c.state[sid];
    StepDesc* desc = c.desc;
    const int per_frame = 5 * c.L + 1;
    Prefetcher pf{0, per_frame * P.steps};
    Tracer tr;

    // prologue: audio sum of frame 0
    audio_sum_slice(P, 0, cta, ncta);
    if (!grid_sync(P, epoch, sm, tr)) return;

    for (int f = 0; f < P.steps; ++f) {
        tr.on = P.trace != nullptr && cta == 0 && f == P.trace_frame;
        tr.mark(P);
        const int len_now = min(st.len + 1, c.ML);
        // text token of this frame
        uint32_t text = desc->text ? __ldcg(desc->text + f) : st.last_text;
        if (text >= (uint32_t)c.TV) {
            raise_error(desc, -1);
            text = 0;
        }
        // x = audio sum + text row (model.rs:640-646); every CTA builds it, CTA slices are stored
        for (int j = threadIdx.x; j < c.D; j += kThreads) {
            const float v = __fadd_rn(__ldcg(P.xa + j), emb_val(c, c.emb_text, text, j));
            sm.xf[j] = v;
        }
        __syncthreads();
        {
            const int j0 = (int)split_lo(c.D, cta, ncta), j1 = (int)split_lo(c.D, cta + 1, ncta);
            for (int j = j0 + (int)threadIdx.x; j < j1; j += kThreads) c.x[j] = sm.xf[j];
        }
        for (int l = 0; l < c.L; ++l) {
            const LayerDev& Lw = c.layers[l];
            const int gp = f * per_frame + 5 * l;
            // ---- QKV
            pf.run(P, gp + PH_QKV, cta, ncta, len_now);
            if (l == 0) {
                // norm1 of the frame input already staged in xf
                float ss = 0.0f;
                for (int j = threadIdx.x; j < c.D; j += kThreads) ss = __fmaf_rn(sm.xf[j], sm.xf[j], ss);
                ss = block_reduce_sum(ss, sm);
                const float rms = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)c.D), 1e-8f));
                for (int j = threadIdx.x; j < c.D; j += kThreads)
                    sm.xf[j] = __fmul_rn(__fdiv_rn(sm.xf[j], rms), Lw.norm1[j]);
                __syncthreads();
                build_limbs(sm, c.D);
                __syncthreads();
            } else {
                load_vector(sm, c.x, c.D, Lw.norm1);
            }
            gemv_phase<EPI_QKV>(P, sm, Lw.qkv, l, st, cta, ncta, nullptr, f);
            if (!grid_sync(P, epoch, sm, tr)) return;
            // ---- attention
            pf.run(P, gp + PH_ATT, cta, ncta, len_now);
            if (c.kv_f32) attention_phase<float>(P, sm, l, st, cta);
            else attention_phase<__nv_bfloat16>(P, sm, l, st, cta);
            if (!grid_sync(P, epoch, sm, tr)) return;
            // ---- out_proj + residual
            pf.run(P, gp + PH_OUT, cta, ncta, len_now);
            load_vector(sm, c.attn, c.D, nullptr);
            gemv_phase<EPI_RESID>(P, sm, Lw.out, l, st, cta, ncta, nullptr, f);
            if (!grid_sync(P, epoch, sm, tr)) return;
            // ---- linear_in + silu gate
            pf.run(P, gp + PH_IN, cta, ncta, len_now);
            load_vector(sm, c.x, c.D, Lw.norm2);
            gemv_phase<EPI_GATE>(P, sm, Lw.fin, l, st, cta, ncta, nullptr, f);
            if (!grid_sync(P, epoch, sm, tr)) return;
            // ---- linear_out + residual
            pf.run(P, gp + PH_DOWN, cta, ncta, len_now);
            load_vector(sm, c.hid, c.F, nullptr);
            gemv_phase<EPI_RESID>(P, sm, Lw.fout, l, st, cta, ncta, nullptr, f);
            if (!grid_sync(P, epoch, sm, tr)) return;
        }
        // ---- head + argmax partials; audio sum of the next frame
        pf.run(P, f * per_frame + 5 * c.L, cta, ncta, min(st.len + 2, c.ML));
        load_vector(sm, c.x, c.D, c.out_norm);
        HeadBest best{-FLT_MAX, 0x7FFFFFFF};
        gemv_phase<EPI_LOGITS>(P, sm, c.head, 0, st, cta, ncta, &best, f);
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
            }
        }
        if (f + 1 < P.steps) audio_sum_slice(P, f + 1, cta, ncta);
        if (!grid_sync(P, epoch, sm, tr)) return;
        // every CTA reduces the partials identically
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

// Grid-barrier latency probe: `iters` back-to-back barriers of the persistent kernel.
__global__ void __launch_bounds__(kThreads, 1) barrier_probe_kernel(const __grid_constant__ MegaArgs P, int iters) {
    extern __shared__ uint4 smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    uint32_t epoch = 0;
    Tracer tr;
    for (int i = 0; i < iters; ++i)
        if (!grid_sync(P, epoch, sm, tr)) return;
}

}  // namespace

cudaError_t mega_barrier_probe(void* scratch, int iters, float* ms_out) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(barrier_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
    if (e != cudaSuccess) return e;
    MegaArgs P{};
    P.bar = static_cast<uint32_t*>(scratch);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    e = cudaMemset(P.bar, 0, 256);
    void* args[] = {(void*)&P, (void*)&iters};
    if (e == cudaSuccess) e = cudaEventRecord(a, 0);
    if (e == cudaSuccess) e = cudaLaunchCooperativeKernel((const void*)barrier_probe_kernel, dim3(sms), dim3(kThreads), args, sizeof(Smem), 0);
    if (e == cudaSuccess) e = cudaEventRecord(b, 0);
    if (e == cudaSuccess) e = cudaEventSynchronize(b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms_out, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return e;
}

bool mega_supported(int L, int D, int F, int HD) {
    // head tickets live in the 64-word barrier block: 2 + H <= 64
    return HD == 128 && D % 256 == 0 && D <= kMaxK && F % 128 == 0 && F <= kMaxK && L > 0 && D / HD <= 60 &&
           std::getenv("STT_DISABLE_MEGA") == nullptr;
}

size_t mega_scratch_bytes(int num_sms, int D, int F, int V, int H, int HD) {
    return 256 + (size_t)D * 4 + (size_t)num_sms * 8 + 64 * 4;
}

cudaError_t configure_mega() {
    return cudaFuncSetAttribute(mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
}

cudaError_t launch_mega_steps(MegaState& ms, const Ctx& c, const LayerDev* h_layers, int steps, cudaStream_t st) {
    int dev = 0, sms = 0, occ = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, mega_kernel, kThreads, sizeof(Smem));
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorCooperativeLaunchTooLarge;
    uint8_t* s = static_cast<uint8_t*>(ms.scratch);
    MegaArgs P;
    P.c = c;
    P.steps = steps;
    P.nsplit = sms / c.H;  // the stream set sizes its partials buffer for num_sms rows
    P.bar = reinterpret_cast<uint32_t*>(s);
    P.xa = reinterpret_cast<float*>(s + 256);
    P.amax_v = reinterpret_cast<float*>(s + 256 + (size_t)c.D * 4);
    P.amax_i = reinterpret_cast<int32_t*>(s + 256 + (size_t)c.D * 4 + (size_t)sms * 4);
    P.pf_budget = 256u * 1024u;
    if (const char* pb = std::getenv("STT_MEGA_PF_KB")) P.pf_budget = (uint32_t)std::atoi(pb) * 1024u;
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
    void* args[] = {(void*)&P};
    return cudaLaunchCooperativeKernel((const void*)mega_kernel, dim3(sms), dim3(kThreads), args, sizeof(Smem), st);
}

}  // namespace stt
