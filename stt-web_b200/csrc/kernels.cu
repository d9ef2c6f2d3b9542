// Step kernels of the STT-1B decode step for sm_100a.
//
// One decode step for a batch of n streams is
//   embed -> 16 x [qkv, attention, out_proj, linear_in, linear_out] -> head -> finish
// where each Q4 matmul is a dequant-fused GEMV (gemv_mma_kernel for passes of several batch rows,
// gemv_kernel or gemv_stream_kernel for one) with its neighbours fused in:
//   qkv        RMSNorm(norm1) prologue; RoPE + K/V ring write epilogue   (model.rs:426-449)
//   attention  split-KV softmax(q.k^T * scale).v, last split combines     (model.rs:450-472)
//   out_proj   residual-add epilogue                                       (model.rs:565)
//   linear_in  RMSNorm(norm2) prologue; silu(gate) * value epilogue        (model.rs:517-524)
//   linear_out residual-add epilogue                                       (model.rs:570)
//   head       RMSNorm(out_norm) prologue                                  (model.rs:662-663)
//   finish     argmax (lowest index on ties) and the stream-loop state update (stream.rs:90-107,
//              231-266)
#include <algorithm>
#include <cfloat>
#include <map>
#include <mutex>

#include "device.cuh"
#include "dp4a.cuh"
#include "gemv_common.cuh"
#include "kernels.h"
#include "tc_gemm.h"
#include "tc_layout.cuh"

namespace stt {


// ------------------------------------------------------------------------------------ Q4 layout

// Splits raw Q4_0 blocks (18 bytes: f16 scale, 16 nibble bytes) into the two device planes.  When
// big_scale is set, a block whose scale has magnitude above 4 (or is inf / nan) sets it to 1: such
// weights overflow the f16 parts of the tensor-core product (tc_gemm.cu).
__global__ void repack_q4_kernel(const uint8_t* __restrict__ raw, int64_t nblocks, uint4* __restrict__ nib,
                                 uint16_t* __restrict__ scale, int* __restrict__ big_scale) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const uint8_t* p = raw + b * 18;
    const uint16_t sb = (uint16_t)(p[0] | (p[1] << 8));
    scale[b] = sb;
    if (big_scale && (sb & 0x7FFFu) > 0x4400u) *big_scale = 1;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        w[i] = (uint32_t)p[2 + 4 * i] | ((uint32_t)p[3 + 4 * i] << 8) | ((uint32_t)p[4 + 4 * i] << 16) |
               ((uint32_t)p[5 + 4 * i] << 24);
    nib[b] = make_uint4(w[0], w[1], w[2], w[3]);
}

// out[r*k + j] = (nibble - 8) * scale, the value the reference shader uses (shader_naive.wgsl:64-81).
__global__ void dequant_q4_kernel(Q4Dev w, float* __restrict__ out) {
    const int64_t nb = w.k / 32;
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= (int64_t)w.n * nb) return;
    const uint4 q = w.nib[b];
    const float d = f16_to_f32_ieee(w.scale[b]);
    float* o = out + b * 32;
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t byte = (words[wi] >> (8 * i)) & 0xFFu;
            o[4 * wi + i] = __fmul_rn(nib_m8(byte & 0xFu), d);
            o[16 + 4 * wi + i] = __fmul_rn(nib_m8(byte >> 4), d);
        }
}

// ------------------------------------------------------------------------------------ embed

__device__ __forceinline__ float emb_value(const Ctx& c, const uint8_t* table, uint32_t row, int j) {
    const uint8_t* r = table + (int64_t)row * c.emb_row_bytes;
    switch (c.emb_type) {
        case EMB_BF16: return bf16_to_f32_dev(reinterpret_cast<const uint16_t*>(r)[j]);
        case EMB_F32: return reinterpret_cast<const float*>(r)[j];
        case EMB_F16: return f16_to_f32_ieee(reinterpret_cast<const uint16_t*>(r)[j]);
        default: {  // Q4_0 row, gguf.rs:616-633
            const uint8_t* blk = r + (j >> 5) * 18;
            const float d = f16_to_f32_gguf((uint16_t)(blk[0] | (blk[1] << 8)));
            const int w = j & 31;
            const uint32_t byte = blk[2 + (w & 15)];
            const uint32_t nib = w < 16 ? (byte & 0xFu) : (byte >> 4);
            return __fmul_rn(nib_m8(nib), d);
        }
    }
}

// x = sum of the 32 audio rows (codebook order) then the text row (model.rs:640-646), f32.
// grid (ceil(D/256), n): each CTA sums a 256-element slice of one batch row.
__global__ void __launch_bounds__(256) embed_kernel(Ctx c) {
    const int i = blockIdx.y;
    const int sid = c.ids[i];
    StepDesc* desc = c.desc;
    const int step = desc->step;
    const uint32_t* audio = desc->audio + ((int64_t)step * c.n + i) * c.NC;
    uint32_t text = desc->text ? desc->text[(int64_t)step * c.n + i] : c.state[sid].last_text;
    if (text >= (uint32_t)c.TV) {
        raise_error(desc, -1);
        text = 0;
    }
    __shared__ uint32_t toks[kMaxCodebooks];
    if (threadIdx.x < c.NC) {
        uint32_t t = audio[threadIdx.x];
        if (t >= (uint32_t)c.AV) {
            raise_error(desc, -1);
            t = 0;
        }
        toks[threadIdx.x] = t;
    }
    __syncthreads();
    const int64_t table_bytes = (int64_t)c.AV * c.emb_row_bytes;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= c.D) return;
    float acc = 0.0f;
    for (int cb = 0; cb < c.NC; ++cb) acc = __fadd_rn(acc, emb_value(c, c.emb_audio + cb * table_bytes, toks[cb], j));
    acc = __fadd_rn(acc, emb_value(c, c.emb_text, text, j));
    c.x[(int64_t)i * c.D + j] = acc;
}

// ------------------------------------------------------------------------------------ GEMV

// Deterministic block reduction (fixed order) of one value per thread; all threads get the sum.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int w = 0; w < nw; ++w) s += red[w];
    return s;
}

// The GEMV input: batch rows [row0, row0 + mb) of `in` (f32, or bf16 when in_bf16 is set),
// RMSNorm'd with alpha when alpha != NULL (burn::nn::RmsNorm: (x / sqrt(mean(x^2) + 1e-8)) * alpha),
// as dp4a limbs L[m] ([6][NB] uint4) and block exponents xs[m] ([NB]).  Every thread of the CTA
// takes part; ends with a CTA barrier.
__device__ void load_limbs(const float* __restrict__ in, const __nv_bfloat16* __restrict__ in_bf16, int K, int row0,
                           int mb, const float* __restrict__ alpha, uint4* L, float* xs, float* red) {
    const int NB = K >> 5, nq = K >> 2;
    const int nq_pad = (nq + 31) & ~31;  // whole warps join the shuffles of quad_limbs_store
    for (int m = 0; m < mb; ++m) {
        const int64_t base = (int64_t)(row0 + m) * K;
        float rms = 1.0f;
        if (alpha) {
            float ss = 0.0f;
            for (int j = threadIdx.x; j < K; j += blockDim.x) {
                const float v = in[base + j];
                ss = __fmaf_rn(v, v, ss);
            }
            ss = block_sum(ss, red);
            rms = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-8f));
        }
        for (int q = threadIdx.x; q < nq_pad; q += blockDim.x) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            const bool valid = q < nq;
            if (valid) {
                if (in_bf16) {
                    const uint2 r = *reinterpret_cast<const uint2*>(in_bf16 + base + 4 * q);
                    v = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                                    __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
                } else {
                    v = *reinterpret_cast<const float4*>(in + base + 4 * q);
                }
                if (alpha) {
                    const float4 al = reinterpret_cast<const float4*>(alpha)[q];
                    v.x = __fmul_rn(__fdiv_rn(v.x, rms), al.x);
                    v.y = __fmul_rn(__fdiv_rn(v.y, rms), al.y);
                    v.z = __fmul_rn(__fdiv_rn(v.z, rms), al.z);
                    v.w = __fmul_rn(__fdiv_rn(v.w, rms), al.w);
                }
            }
            quad_limbs_store(L + (size_t)m * 6 * NB, xs + (size_t)m * NB, q, NB, v, valid);
        }
    }
    __syncthreads();
}

// The register GEMV, for the passes that neither the integer-MMA GEMV (passes of several rows, K a
// multiple of 256) nor the streamed GEMV takes: K not a multiple of 256, or one row over more than
// 40 units per SM.  For each unit (a row pair; EPI_GATE: a gate row and its value row) and each
// batch row m < mb,
// sum over blocks of scale * dot(block, x[m]) with the exact dp4a block dot of dp4a.cuh, then the
// epilogue.  A unit is reduced by a team of `team` consecutive threads (8 .. 256, a power of two;
// past 32 the team spans warps), each taking blocks tl, tl + team, ... (at most kBPL of them), so
// that all of a unit's weight bytes are in flight at once and one launch keeps about 128 K lanes
// busy.  The CTA first issues its first unit's weight loads, then converts the input rows to limbs
// in shared memory while they are in flight; launched as a programmatic dependent, those weight
// loads also overlap the end of the previous kernel.  Deterministic: the team sums its lanes, then
// its warps, in a fixed order.
constexpr int kBPL = 4;           // blocks per team lane and row, at most
constexpr int kGemvThreads = 256;

template <int MB, int EPI>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(Ctx c, GemvArgs a, int row0, int mb, int team) {
    extern __shared__ uint4 gemv_smem[];
    const int K = a.W.k, NB = K >> 5;
    uint4* L = gemv_smem;                                           // [MB][6][NB]
    float* xs = reinterpret_cast<float*>(gemv_smem + (size_t)MB * 6 * NB);  // [MB][NB]
    __shared__ float red[32];
    __shared__ float tpart[2][kGemvThreads / 32][2 * MB];          // cross-warp team partials
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int teams = kGemvThreads / team, my_team = tid / team, tl = tid % team;
    const int64_t nteams = (int64_t)gridDim.x * teams;

    uint4 qa[kBPL], qb[kBPL];
    uint32_t sa[kBPL], sb[kBPL];
    auto load_unit = [&](int64_t u, int* ra, int* rb) {
        unit_rows<EPI>(a, (int)u, ra, rb);
        const uint4* na = a.W.nib + (int64_t)*ra * NB;
        const uint4* nb_ = a.W.nib + (int64_t)(*rb >= 0 ? *rb : *ra) * NB;
        const uint16_t* s_a = a.W.scale + (int64_t)*ra * NB;
        const uint16_t* s_b = a.W.scale + (int64_t)(*rb >= 0 ? *rb : *ra) * NB;
#pragma unroll
        for (int i = 0; i < kBPL; ++i) {
            const int b = tl + i * team;
            if (b < NB) {
                qa[i] = __ldg(na + b);
                qb[i] = __ldg(nb_ + b);
                sa[i] = __ldg(s_a + b);
                sb[i] = __ldg(s_b + b);
            }
        }
    };

    int64_t u = (int64_t)blockIdx.x * teams + my_team;
    int ra = 0, rb = -1;
    pdl_trigger();
    if (u < a.n_units) load_unit(u, &ra, &rb);  // weights first: they do not depend on the input
    // launched as a programmatic dependent: the input (and, for EPI_RESID, the output) belong to the
    // previous kernel of the stream until this wait returns
    pdl_wait();
    load_limbs(a.in, a.in_bf16, K, row0, mb, a.norm, L, xs, red);
    int parity = 0;
    for (; u < a.n_units; u += nteams) {
        float acc[MB][2];
#pragma unroll
        for (int m = 0; m < MB; ++m) acc[m][0] = acc[m][1] = 0.0f;
#pragma unroll
        for (int i = 0; i < kBPL; ++i) {
            const int b = tl + i * team;
            if (b < NB) {
                const float fa = f16_to_f32_ieee((uint16_t)sa[i]), fb = f16_to_f32_ieee((uint16_t)sb[i]);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    if (m < mb) {
                        const uint4* Lm = L + (size_t)m * 6 * NB;
                        uint4 Lb[6];
#pragma unroll
                        for (int v = 0; v < 6; ++v) Lb[v] = Lm[v * NB + b];
                        const float x = xs[m * NB + b];
                        acc[m][0] = __fmaf_rn(block_dp4a(qa[i], Lb), __fmul_rn(fa, x), acc[m][0]);
                        acc[m][1] = __fmaf_rn(block_dp4a(qb[i], Lb), __fmul_rn(fb, x), acc[m][1]);
                    }
                }
            }
        }
        const int cra = ra, crb = rb;
        const int64_t next = u + nteams;
        if (next < a.n_units) load_unit(next, &ra, &rb);  // the next unit's bytes fly during the reduction
        // team reduction: lanes of the team inside a warp, then (teams past 32 lanes) its warps
        const int span = team < 32 ? team : 32;
#pragma unroll
        for (int m = 0; m < MB; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                for (int o = span >> 1; o > 0; o >>= 1) acc[m][h] += __shfl_xor_sync(0xFFFFFFFFu, acc[m][h], o);
        if (team > 32) {
            if (lane == 0)
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    tpart[parity][warp][2 * m] = acc[m][0];
                    tpart[parity][warp][2 * m + 1] = acc[m][1];
                }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + my_team), "r"(team) : "memory");
            if (tl == 0) {
                const int w0 = warp, nw = team >> 5;
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    float s0 = tpart[parity][w0][2 * m], s1 = tpart[parity][w0][2 * m + 1];
                    for (int w = 1; w < nw; ++w) {
                        s0 += tpart[parity][w0 + w][2 * m];
                        s1 += tpart[parity][w0 + w][2 * m + 1];
                    }
                    acc[m][0] = s0;
                    acc[m][1] = s1;
                }
            }
            parity ^= 1;
        }
        if (tl == 0)
#pragma unroll
            for (int m = 0; m < MB; ++m)
                if (m < mb) epilogue<EPI>(c, a, row0 + m, cra, crb, acc[m][0], acc[m][1]);
    }
}

// The streamed GEMV: the same products as gemv_kernel, for K a multiple of 256, with the weights
// moved by bulk copies instead of register loads.  A CTA owns a contiguous range of units; its
// producer warp copies them, a few units per stage, into a ring of shared-memory stages
// (cp.async.bulk, one full mbarrier per stage), so the CTA's whole share of the matrix can be in
// flight at once without holding registers, and the consumer warps take the units of each stage
// as it lands: a warp per unit, the lanes splitting its blocks, the dp4a block dot on the limbs,
// a shuffle reduction and the epilogue.  Stage layout: the units' nibble rows (pairs: rows 2u and
// 2u + 1 of each unit; EPI_GATE: the gate rows, then the value rows), then their scale rows.  Every
// wait is bounded; a wait that gives up records STT_E_DEVICE_FLAG in the step descriptor (or in
// a.err) and the CTA stops, waiting (bounded) for its copies in flight before it exits.
// consumer warps of the streamed GEMV: 16, or 8 for 8 batch rows (register budget)
template <int MB>
constexpr int stream_cwarps() { return MB >= 8 ? 8 : 16; }
constexpr int kSStages = 6;
constexpr uint32_t kSStageBytes = 24 * 1024;

__device__ __forceinline__ bool gemv_mbar_wait(uint64_t* m, uint32_t parity, volatile int* stop) {
    for (uint32_t i = 0; i < kSSpin; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_addr(m)), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 255u) == 255u && *stop) return false;
    }
    return false;
}

template <int MB, int EPI>
__global__ void __launch_bounds__(32 * (stream_cwarps<MB>() + 1)) gemv_stream_kernel(Ctx c, GemvArgs a, int row0,
                                                                                      int mb, int ups, int stages,
                                                                                      int* err) {
    constexpr int kSCWarps = stream_cwarps<MB>();
    extern __shared__ __align__(128) uint8_t gs_smem[];
    const int K = a.W.k, NB = K >> 5;
    uint8_t* ring = gs_smem;                                                   // [stages][kSStageBytes]
    uint4* L = reinterpret_cast<uint4*>(gs_smem + (size_t)stages * kSStageBytes);  // [MB][6][NB]
    float* xs = reinterpret_cast<float*>(L + (size_t)MB * 6 * NB);            // [MB][NB]
    __shared__ __align__(8) uint64_t full[kSStages], empty[kSStages];  // the first `stages` are used
    __shared__ float red[32];
    __shared__ int stop;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t u0 = (int64_t)a.n_units * blockIdx.x / gridDim.x;
    const int64_t u1 = (int64_t)a.n_units * (blockIdx.x + 1) / gridDim.x;
    const int nchunks = (int)((u1 - u0 + ups - 1) / ups);
    if (tid == 0) {
        for (int i = 0; i < stages; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[i])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&empty[i])), "r"(ups) : "memory");
        }
        stop = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();
    const bool gate = EPI == EPI_GATE;
    const uint32_t row_nib = (uint32_t)NB * 16u, row_sc = (uint32_t)NB * 2u;
    if (warp == kSCWarps) {
        // producer: the weights are constant, so their copies start before the previous kernel ends
        int issued = 0;
        for (int k = 0; k < nchunks; ++k) {
            const int s = k % stages;
            if (k >= stages) {
                bool ok = true;
                if (lane == 0) ok = gemv_mbar_wait(&empty[s], ((k / stages) - 1) & 1, &stop);
                if (!__shfl_sync(0xFFFFFFFFu, (int)ok, 0)) break;
            }
            if (lane == 0) {
                const int64_t ua = u0 + (int64_t)k * ups;
                const int nu = (int)((int64_t)ups < u1 - ua ? (int64_t)ups : u1 - ua);
                const uint32_t dst = smem_addr(ring + (size_t)s * kSStageBytes);
                const uint32_t nr = gate ? (uint32_t)nu : (uint32_t)((int64_t)(2 * nu) < (int64_t)a.W.n - 2 * ua ? (int64_t)(2 * nu) : (int64_t)a.W.n - 2 * ua);
                const uint32_t bytes = gate ? 2u * nr * (row_nib + row_sc) : nr * (row_nib + row_sc);
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&full[s])),
                             "r"(bytes)
                             : "memory");
                const int64_t r0 = gate ? ua : 2 * ua;
                const uint8_t* nib = reinterpret_cast<const uint8_t*>(a.W.nib);
                const uint8_t* sc = reinterpret_cast<const uint8_t*>(a.W.scale);
                const uint32_t nib_bytes = gate ? 2u * nr * row_nib : nr * row_nib;
                auto copy = [&](uint32_t d, const void* src, uint32_t b) {
                    asm volatile(
                        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                            d),
                        "l"(src), "r"(b), "r"(smem_addr(&full[s]))
                        : "memory");
                };
                copy(dst, nib + r0 * row_nib, nr * row_nib);
                if (gate) copy(dst + nr * row_nib, nib + (r0 + a.half_n) * row_nib, nr * row_nib);
                copy(dst + nib_bytes, sc + r0 * row_sc, nr * row_sc);
                if (gate) copy(dst + nib_bytes + nr * row_sc, sc + (r0 + a.half_n) * row_sc, nr * row_sc);
            }
            __syncwarp();
            issued = k + 1;
        }
        // every copy must land before the CTA's shared memory goes away
        if (lane == 0)
            for (int k = max(0, issued - stages); k < issued; ++k) {
                const int s = k % stages;
                for (uint32_t i = 0; i < kSSpin; ++i) {
                    uint32_t ok;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                        "selp.u32 %0, 1, 0, p;\n\t}"
                        : "=r"(ok)
                        : "r"(smem_addr(&full[s])), "r"((uint32_t)(k / stages) & 1u)
                        : "memory");
                    if (ok) break;
                }
            }
        pdl_wait();
        return;
    }
    // consumers: the input rows become limbs (the producer's copies are already in flight)
    pdl_wait();
    {
        const int nq = K >> 2;
        for (int m = 0; m < mb; ++m) {
            const int64_t base = (int64_t)(row0 + m) * K;
            float rms = 1.0f;
            if (a.norm) {
                float ss = 0.0f;
                for (int j = tid; j < K; j += 32 * kSCWarps) {
                    const float v = a.in[base + j];
                    ss = __fmaf_rn(v, v, ss);
                }
                ss = warp_sum(ss);
                asm volatile("bar.sync 1, %0;" ::"n"(32 * kSCWarps) : "memory");
                if (lane == 0) red[warp] = ss;
                asm volatile("bar.sync 1, %0;" ::"n"(32 * kSCWarps) : "memory");
                float t = 0.0f;
                for (int w = 0; w < kSCWarps; ++w) t += red[w];
                rms = sqrtf(__fadd_rn(__fdiv_rn(t, (float)K), 1e-8f));
            }
            for (int q = tid; q < nq; q += 32 * kSCWarps) {  // nq is a multiple of 64: whole warps
                float4 v;
                if (a.in_bf16) {
                    const uint2 r = *reinterpret_cast<const uint2*>(a.in_bf16 + base + 4 * q);
                    v = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                                    __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
                } else {
                    v = *reinterpret_cast<const float4*>(a.in + base + 4 * q);
                }
                if (a.norm) {
                    const float4 al = reinterpret_cast<const float4*>(a.norm)[q];
                    v.x = __fmul_rn(__fdiv_rn(v.x, rms), al.x);
                    v.y = __fmul_rn(__fdiv_rn(v.y, rms), al.y);
                    v.z = __fmul_rn(__fdiv_rn(v.z, rms), al.z);
                    v.w = __fmul_rn(__fdiv_rn(v.w, rms), al.w);
                }
                quad_limbs_store(L + (size_t)m * 6 * NB, xs + (size_t)m * NB, q, NB, v, true);
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kSCWarps) : "memory");
    }
    // each warp takes the CTA's units j = warp, warp + kSCWarps, ... as their stages land; a stage is
    // free again once all of its units are done (every unit arrives once)
    const int64_t cta_units = u1 - u0;
    for (int64_t j = warp; j < cta_units; j += kSCWarps) {
        const int k = (int)(j / ups), s = k % stages;
        bool ok = true;
        if (lane == 0) ok = gemv_mbar_wait(&full[s], (k / stages) & 1, &stop);
        if (!__shfl_sync(0xFFFFFFFFu, (int)ok, 0)) {
            if (lane == 0) {
                stop = 1;
                if (c.desc) raise_error(c.desc, -5);  // STT_E_DEVICE_FLAG
                if (err) atomicCAS(err, 0, -5);
            }
            break;
        }
        const int64_t ua = u0 + (int64_t)k * ups;
        const int nu = (int)((int64_t)ups < u1 - ua ? (int64_t)ups : u1 - ua);
        const int jl = (int)(j - (int64_t)k * ups);  // the unit's place in its stage
        const uint8_t* st = ring + (size_t)s * kSStageBytes;
        const uint32_t nr = gate ? (uint32_t)nu : (uint32_t)((int64_t)(2 * nu) < (int64_t)a.W.n - 2 * ua ? (int64_t)(2 * nu) : (int64_t)a.W.n - 2 * ua);
        const uint4* nibs = reinterpret_cast<const uint4*>(st);
        const uint16_t* scs = reinterpret_cast<const uint16_t*>(st + (gate ? 2u * nr * row_nib : nr * row_nib));
        int ra, rb;
        unit_rows<EPI>(a, (int)(ua + jl), &ra, &rb);
        const int la = gate ? jl : 2 * jl;
        const int lb = gate ? (int)nr + jl : (rb >= 0 ? 2 * jl + 1 : 2 * jl);
        float acc[MB][2];
#pragma unroll
        for (int m = 0; m < MB; ++m) acc[m][0] = acc[m][1] = 0.0f;
        for (int b = lane; b < NB; b += 32) {
            const uint4 qa = nibs[(size_t)la * NB + b], qb = nibs[(size_t)lb * NB + b];
            const float fa = f16_to_f32_ieee(scs[(size_t)la * NB + b]), fb = f16_to_f32_ieee(scs[(size_t)lb * NB + b]);
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                if (m < mb) {
                    const uint4* Lm = L + (size_t)m * 6 * NB;
                    uint4 Lb[6];
#pragma unroll
                    for (int v = 0; v < 6; ++v) Lb[v] = Lm[v * NB + b];
                    const float x = xs[m * NB + b];
                    acc[m][0] = __fmaf_rn(block_dp4a(qa, Lb), __fmul_rn(fa, x), acc[m][0]);
                    acc[m][1] = __fmaf_rn(block_dp4a(qb, Lb), __fmul_rn(fb, x), acc[m][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&empty[s])) : "memory");
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            acc[m][0] = warp_sum(acc[m][0]);
            acc[m][1] = warp_sum(acc[m][1]);
        }
        if (lane == 0)
#pragma unroll
            for (int m = 0; m < MB; ++m)
                if (m < mb) epilogue<EPI>(c, a, row0 + m, ra, rb, acc[m][0], acc[m][1]);
    }
}

// Epilogue of a tensor-core product: the K-slice partial sums part[z][m][W.n] of each output pair
// are added in slice order (z = 0, 1, ...) and handed to the same epilogue as the GEMV's.  Grid
// (groups of kEpiUnits * 256 units, batch rows); a thread takes units u0 + 256 j, j < kEpiUnits, and
// issues all of their loads before it uses any (4 units from 128 batch rows up; below, one, which
// keeps more CTAs in flight).  The step's stream ids and states are written by kernels launched the
// ordinary way before any tensor-core product of the step, and the RoPE table is constant, so the
// QKV epilogue reads them before it waits for the product.
template <int EPI, int kEpiUnits>
__global__ void __launch_bounds__(256) tc_epilogue_kernel(Ctx c, GemvArgs a, const float* __restrict__ part, int rows,
                                                         int slices) {
    pdl_trigger();
    const int m = blockIdx.y;
    const int u0 = blockIdx.x * (256 * kEpiUnits) + threadIdx.x;
    int sid = 0;
    StreamState st{};
    float2 cs[kEpiUnits];
    if (EPI == EPI_QKV) {
        sid = c.ids[m];
        st = c.state[sid];
#pragma unroll
        for (int j = 0; j < kEpiUnits; ++j) {
            const int u = u0 + 256 * j;
            cs[j] = u < a.n_units ? qkv_rope(c, st, 2 * u) : make_float2(0.0f, 0.0f);
        }
    }
    pdl_wait();
    const int64_t plane = (int64_t)rows * a.W.n;
    const float* pm = part + (int64_t)m * a.W.n;
    int ra[kEpiUnits], rb[kEpiUnits];
    float va[kEpiUnits], vb[kEpiUnits];
#pragma unroll
    for (int j = 0; j < kEpiUnits; ++j) {
        const int u = u0 + 256 * j;
        ra[j] = 0, rb[j] = -1, va[j] = vb[j] = 0.0f;
        if (u < a.n_units) {
            unit_rows<EPI>(a, u, &ra[j], &rb[j]);
            va[j] = pm[ra[j]];
            if (rb[j] >= 0) vb[j] = pm[rb[j]];
        }
    }
    for (int z = 1; z < slices; ++z) {
        const float* p = pm + z * plane;
        float wa[kEpiUnits], wb[kEpiUnits];
#pragma unroll
        for (int j = 0; j < kEpiUnits; ++j) {
            wa[j] = wb[j] = 0.0f;
            if (u0 + 256 * j < a.n_units) {
                wa[j] = p[ra[j]];
                if (rb[j] >= 0) wb[j] = p[rb[j]];
            }
        }
#pragma unroll
        for (int j = 0; j < kEpiUnits; ++j) {
            va[j] = __fadd_rn(va[j], wa[j]);
            if (rb[j] >= 0) vb[j] = __fadd_rn(vb[j], wb[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < kEpiUnits; ++j) {
        if (u0 + 256 * j >= a.n_units) continue;
        if (EPI == EPI_QKV) qkv_store(c, a, m, sid, st, cs[j], ra[j], rb[j], va[j], vb[j]);
        else epilogue<EPI>(c, a, m, ra[j], rb[j], va[j], vb[j]);
    }
}

// ------------------------------------------------------------------------------------ attention

// One (split, head, batch row): keys [split*chunk, min(len, (split+1)*chunk)) of the ring
// (model.rs:450-472; ring order does not matter to the softmax).  HD = 128.  A warp takes 4 keys at
// a time, one per group of 8 lanes; a lane holds 16 dimensions of q, k, v and its group's
// online-softmax state (max, sum of exp, sum of exp * v), and two key groups' loads are issued
// before either is used.  The groups of a warp merge by shuffles, then the 4 warps in warp order.
// Partial = (max score, sum exp, sum exp * v).  The CTA finishing last for a (row, head)
// combines the partials in split order and writes attn[row][head]; with a single split the CTA
// writes it directly.
// K/V staging of the batched attention: chunks of CH keys, two stages of K and V.  Measured (bf16 K/V):
// 48-key chunks are best for 64 streams at positions 0..750, 32-key chunks for 512 streams at
// positions 0..250 (smaller stages let more CTAs share an SM).
template <typename KT, int CH>
constexpr size_t attn_smem_bytes() { return (size_t)2 * 2 * CH * 128 * sizeof(KT); }

// mbarrier and bulk-copy helpers of the attention kernel's K/V staging
__device__ __forceinline__ void attn_mbar_init(uint64_t* m) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(m)) : "memory");
}
__device__ __forceinline__ bool attn_mbar_wait(uint64_t* m, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_addr(m)), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}
// Bulk copies of `bytes` (a multiple of 16) of K and of V into this CTA's shared memory, both
// completing on the mbarrier (no multicast).
__device__ __forceinline__ void attn_stage_kv(void* kd, const void* ks, void* vd, const void* vs, uint32_t bytes,
                                              uint64_t* m) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(m)), "r"(2 * bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(kd)),
                 "l"(ks), "r"(bytes), "r"(smem_addr(m))
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(vd)),
                 "l"(vs), "r"(bytes), "r"(smem_addr(m))
                 : "memory");
}

template <typename KT>
__device__ __forceinline__ void load_row16(const KT* row, int sub, float (&x)[16]) {
    constexpr int EPL = 16 / (int)sizeof(KT);  // elements of one 16-byte load
    constexpr int CH = 16 / EPL;               // loads for 16 dimensions
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
        const uint4 r = *reinterpret_cast<const uint4*>(row + ch * 8 * EPL + sub * EPL);
        if (sizeof(KT) == 4) {
            x[ch * 4 + 0] = __uint_as_float(r.x);
            x[ch * 4 + 1] = __uint_as_float(r.y);
            x[ch * 4 + 2] = __uint_as_float(r.z);
            x[ch * 4 + 3] = __uint_as_float(r.w);
        } else {
            const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                x[ch * 8 + 2 * e] = __uint_as_float(w[e] << 16);
                x[ch * 8 + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
            }
        }
    }
}

// Warp-collective: lane holds dims 4 lane .. +3 of head h of batch row i; writes attn and, on a
// tensor-core step, the output projection's f16 input pieces (a piece of block h*4 + lane/8 takes
// word w = lane % 8 (< 4) from this lane and w + 16 from lane + 4).
__device__ __forceinline__ void write_head_output(const Ctx& c, int i, int h, int lane, float4 r) {
    reinterpret_cast<float4*>(c.attn + (int64_t)i * c.D + h * 128)[lane] = r;
    if (c.x16) {
        const float4 b = make_float4(__shfl_down_sync(0xFFFFFFFFu, r.x, 4), __shfl_down_sync(0xFFFFFFFFu, r.y, 4),
                                     __shfl_down_sync(0xFFFFFFFFu, r.z, 4), __shfl_down_sync(0xFFFFFFFFu, r.w, 4));
        if ((lane & 7) < 4)
            x16_store_piece(c.x16, c.x16_nt, c.x16_rows_pad, c.D, i, (h * 4 + (lane >> 3)) * 4 + (lane & 7), r, b, true);
    }
}

template <typename KT, int kAttnChunk>
__global__ void __launch_bounds__(128) attn_kernel(Ctx c, int layer) {
    pdl_trigger();
    pdl_wait();
    constexpr int HD = 128;
    constexpr int EPL = 16 / (int)sizeof(KT);
    const int s = blockIdx.x, h = blockIdx.y, i = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 3, sub = lane & 7;
    const int sid = c.ids[i];
    const StreamState st = c.state[sid];
    const int len = min(st.len + 1, c.ML);
    const int j0 = s * c.chunk, j1 = min(len, j0 + c.chunk);
    // lane dimension e (0..15) is dim(e) = (e / EPL) * 8 * EPL + sub * EPL + e % EPL
    float q[16], o[16];
    {
        const float* qh = c.qkv + (int64_t)i * 3 * c.D + h * HD;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            q[e] = qh[(e / EPL) * 8 * EPL + sub * EPL + e % EPL];
            o[e] = 0.0f;
        }
    }
    const KT* kbase = reinterpret_cast<const KT*>(c.kv) + (int64_t)sid * c.kv_stream_stride +
                      (int64_t)layer * c.kv_layer_stride + (int64_t)h * c.ML * HD;
    const KT* vbase = kbase + c.kv_half_stride;
    // K/V of the split stream through shared memory in chunks of kAttnChunk keys, two in flight
    extern __shared__ __align__(128) uint8_t attn_stage[];  // [2 stages][K, V][kAttnChunk][HD] KT
    __shared__ uint64_t full[2];
    KT* const stage = reinterpret_cast<KT*>(attn_stage);
    constexpr int kStageElems = kAttnChunk * HD;
    const int nkeys = max(0, j1 - j0), nchunks = (nkeys + kAttnChunk - 1) / kAttnChunk;
    int issued = 0;  // chunks whose copies thread 0 has issued
    if (threadIdx.x == 0) {
        attn_mbar_init(&full[0]);
        attn_mbar_init(&full[1]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int ci = 0; ci < 2 && ci < nchunks; ++ci) {
            const int ka = j0 + ci * kAttnChunk, kn = min(kAttnChunk, j1 - ka);
            attn_stage_kv(stage + (2 * ci) * kStageElems, kbase + (int64_t)ka * HD, stage + (2 * ci + 1) * kStageElems,
                          vbase + (int64_t)ka * HD, (uint32_t)(kn * HD * sizeof(KT)), &full[ci]);
            issued = ci + 1;
        }
    }
    __syncthreads();
    float m = -FLT_MAX, l = 0.0f;
    bool staged_ok = true;
    for (int ci = 0; ci < nchunks; ++ci) {
        const int cs = ci & 1, kn = min(kAttnChunk, nkeys - ci * kAttnChunk);
        if (!__syncthreads_and(attn_mbar_wait(&full[cs], (uint32_t)(ci >> 1) & 1u))) {
            staged_ok = false;
            break;
        }
        const KT* ks = stage + (2 * cs) * kStageElems;
        const KT* vs = stage + (2 * cs + 1) * kStageElems;
        // key groups of 16 per CTA step (4 per warp), two steps per iteration
        for (int jb = warp * 4; jb < kn; jb += 32) {
        float k0[16], v0[16], k1[16], v1[16];
        const int ja = jb + g, jc = jb + 16 + g;
        const bool va = ja < kn, vc = jc < kn;
        load_row16(ks + (va ? ja : 0) * HD, sub, k0);
        load_row16(vs + (va ? ja : 0) * HD, sub, v0);
        load_row16(ks + (vc ? jc : 0) * HD, sub, k1);
        load_row16(vs + (vc ? jc : 0) * HD, sub, v1);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float* kv = u == 0 ? k0 : k1;
            const float* vv = u == 0 ? v0 : v1;
            float dot = 0.0f;
#pragma unroll
            for (int e = 0; e < 16; ++e) dot = __fmaf_rn(q[e], kv[e], dot);
            dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 1);
            dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 2);
            dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 4);
            if (!(u == 0 ? va : vc)) continue;
            const float score = __fmul_rn(dot, c.attn_scale);
            const float mn = fmaxf(m, score);
            const float corr = expf(m - mn);
            const float p = expf(score - mn);
            l = __fmaf_rn(l, corr, p);
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __fmaf_rn(o[e], corr, __fmul_rn(p, vv[e]));
            m = mn;
        }
        }
        __syncthreads();  // every warp is done with stage cs
        if (threadIdx.x == 0 && ci + 2 < nchunks) {
            const int ka = j0 + (ci + 2) * kAttnChunk, kn2 = min(kAttnChunk, j1 - ka);
            attn_stage_kv(stage + (2 * cs) * kStageElems, kbase + (int64_t)ka * HD, stage + (2 * cs + 1) * kStageElems,
                          vbase + (int64_t)ka * HD, (uint32_t)(kn2 * HD * sizeof(KT)), &full[cs]);
            issued = ci + 3;
        }
    }
    if (!staged_ok) {
        // a copy did not land in time: record it, let the copies in flight land, produce nothing
        if (threadIdx.x == 0) {
            raise_error(c.desc, -5);
            for (int ci = max(0, issued - 2); ci < issued; ++ci) attn_mbar_wait(&full[ci & 1], (uint32_t)(ci >> 1) & 1u);
        }
        __syncthreads();
        return;
    }
    // the 4 key groups of the warp: groups g and g ^ 1, then g and g ^ 2
#pragma unroll
    for (int d = 8; d <= 16; d <<= 1) {
        const float mo = __shfl_xor_sync(0xFFFFFFFFu, m, d), lo = __shfl_xor_sync(0xFFFFFFFFu, l, d);
        const float mn = fmaxf(m, mo);
        const float fa = l == 0.0f ? 0.0f : expf(m - mn), fb = lo == 0.0f ? 0.0f : expf(mo - mn);
        // the lower group's terms first, so that both halves of a pair compute the same sums
        const bool lower = (lane & d) == 0;
        const float fl = lower ? fa : fb, fu = lower ? fb : fa;
        const float ll = lower ? l : lo, lu = lower ? lo : l;
        l = __fmaf_rn(lu, fu, __fmul_rn(ll, fl));
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const float oo = __shfl_xor_sync(0xFFFFFFFFu, o[e], d);
            const float ol = lower ? o[e] : oo, ou = lower ? oo : o[e];
            o[e] = __fmaf_rn(ou, fu, __fmul_rn(ol, fl));
        }
        m = mn;
    }
    // warp state -> shared memory in dimension order (group 0's lanes)
    __shared__ float sm_m[4], sm_l[4];
    __shared__ float4 sm_o[4][32];
    {
        float* od = reinterpret_cast<float*>(sm_o[warp]);
        if (g == 0) {
#pragma unroll
            for (int e = 0; e < 16; ++e) od[(e / EPL) * 8 * EPL + sub * EPL + e % EPL] = o[e];
        }
        if (lane == 0) {
            sm_m[warp] = l == 0.0f ? -FLT_MAX : m;
            sm_l[warp] = l;
        }
    }
    __syncthreads();
    // combine the 4 warps in warp order
    const int NS = c.nsplit;
    float* part = c.part + (((int64_t)i * c.H + h) * NS + s) * (HD + 4);
    if (NS == 1) {
        // one split: the warps' merge is the head's output
        if (warp == 0) {
            float M = -FLT_MAX;
            for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w]);
            float L = 0.0f;
            float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int w = 0; w < 4; ++w) {
                if (sm_l[w] == 0.0f) continue;
                const float f = expf(sm_m[w] - M);
                L = __fmaf_rn(sm_l[w], f, L);
                const float4 ow = sm_o[w][lane];
                O.x = __fmaf_rn(ow.x, f, O.x);
                O.y = __fmaf_rn(ow.y, f, O.y);
                O.z = __fmaf_rn(ow.z, f, O.z);
                O.w = __fmaf_rn(ow.w, f, O.w);
            }
            write_head_output(c, i, h, lane,
                              make_float4(__fdiv_rn(O.x, L), __fdiv_rn(O.y, L), __fdiv_rn(O.z, L), __fdiv_rn(O.w, L)));
        }
        return;
    }
    if (warp == 0) {
        float M = -FLT_MAX;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w]);
        float L = 0.0f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < 4; ++w) {
            if (sm_l[w] == 0.0f) continue;
            const float f = expf(sm_m[w] - M);
            L = __fmaf_rn(sm_l[w], f, L);
            const float4 ow = sm_o[w][lane];
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
    // last CTA of this (row, head) combines the splits
    __shared__ uint32_t last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(&c.tickets[i * c.H + h], 1u);
        last = (prev == (uint32_t)NS - 1u);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (warp == 0) {
        const float* pb = c.part + ((int64_t)i * c.H + h) * NS * (HD + 4);
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
        write_head_output(c, i, h, lane,
                          make_float4(__fdiv_rn(O.x, L), __fdiv_rn(O.y, L), __fdiv_rn(O.z, L), __fdiv_rn(O.w, L)));
        if (lane == 0) c.tickets[i * c.H + h] = 0u;
    }
}

// ------------------------------------------------------------------------------------ finish

// Greedy argmax of the logits (lowest index among equal maxima), then the end-of-step state
// update: KVCache ring counters (model.rs:204-207) and, in feed_frame mode, the delay gating
// and limit-cycle breaker of resolve_pending_as_token (stream.rs:231-266).
__global__ void __launch_bounds__(1024) finish_kernel(Ctx c) {
    const int i = blockIdx.x;
    const float* lg = c.logits + (int64_t)i * c.V;
    float best = -FLT_MAX;
    int bi = 0x7FFFFFFF;
    for (int j = threadIdx.x; j < c.V; j += blockDim.x) {
        const float v = lg[j];
        if (v > best || (v == best && j < bi)) {
            best = v;
            bi = j;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    __shared__ float wv[32];
    __shared__ int wi[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        wv[warp] = best;
        wi[warp] = bi;
    }
    StepDesc* desc = c.desc;
    const int step = desc->step;
    __syncthreads();
    if (desc->logits) {
        float* dst = desc->logits + ((int64_t)step * c.n + i) * c.V;
        for (int j = threadIdx.x; j < c.V; j += blockDim.x) dst[j] = lg[j];
    }
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (wv[w] > best || (wv[w] == best && wi[w] < bi)) {
                best = wv[w];
                bi = wi[w];
            }
        const uint32_t token = (uint32_t)(bi == 0x7FFFFFFF ? 0 : bi);
        const int sid = c.ids[i];
        StreamState st = c.state[sid];
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
        c.state[sid] = st;
        desc->tokens[(int64_t)step * c.n + i] = out;
        __threadfence();
        const uint32_t done = atomicAdd(&c.tickets[c.n * c.H], 1u);
        if (done == (uint32_t)c.n - 1u) {
            desc->step = step + 1;
            c.tickets[c.n * c.H] = 0u;
        }
    }
}

// ------------------------------------------------------------------------------------ launchers

template <int N>
struct DescParams {
    StepDesc desc;
    int32_t n;
    int32_t ids[N];
};

template <int N>
__global__ void set_desc_kernel(StepDesc* d_desc, int32_t* d_ids, const __grid_constant__ DescParams<N> p) {
    if (threadIdx.x == 0) *d_desc = p.desc;
    for (int i = threadIdx.x; i < p.n; i += blockDim.x) d_ids[i] = p.ids[i];
}

__global__ void set_state_kernel(StreamState* dst, StreamState v) { *dst = v; }

cudaError_t launch_set_state(StreamState* dst, const StreamState& value, cudaStream_t st) {
    set_state_kernel<<<1, 1, 0, st>>>(dst, value);
    return cudaGetLastError();
}

cudaError_t launch_set_desc(StepDesc* d_desc, int32_t* d_ids, const DescInit& p, cudaStream_t st) {
    if (p.n <= kSmallBatch) {
        DescParams<kSmallBatch> q;
        q.desc = p.desc;
        q.n = p.n;
        for (int i = 0; i < p.n; ++i) q.ids[i] = p.ids[i];
        set_desc_kernel<kSmallBatch><<<1, 64, 0, st>>>(d_desc, d_ids, q);
    } else {
        set_desc_kernel<kMaxBatch><<<1, 256, 0, st>>>(d_desc, d_ids, *reinterpret_cast<const DescParams<kMaxBatch>*>(&p));
    }
    return cudaGetLastError();
}

// Dynamic shared memory of a GEMV launch: the limbs (96 bytes) and exponent (4 bytes) of every
// block of every batch row of the pass.
constexpr size_t gemv_smem_bytes(int mb, int k) { return (size_t)mb * (k / 32) * (6 * 16 + 4); }
constexpr int kGemvMaxRowsLongK = 4;   // rows per pass when K > 4096 (the limbs of 8 rows would not fit)

template <int MB, int EPI>
static cudaError_t configure_gemv_t() {
    const int k = MB > kGemvMaxRowsLongK ? 4096 : kMaxGemvK;
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<MB, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)gemv_smem_bytes(MB, k));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_stream_kernel<MB, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmemLimit);
    return e;
}

template <int EPI>
static cudaError_t configure_gemv_e() {
    cudaError_t e = configure_gemv_t<1, EPI>();
    if (e == cudaSuccess) e = configure_gemv_t<2, EPI>();
    if (e == cudaSuccess) e = configure_gemv_t<4, EPI>();
    if (e == cudaSuccess) e = configure_gemv_t<8, EPI>();
    return e;
}

// Raises the dynamic shared memory limit of every GEMV instantiation (call once per device).
cudaError_t configure_kernels() {
    cudaError_t e = configure_gemv_e<EPI_PLAIN>();
    if (e == cudaSuccess) e = configure_gemv_e<EPI_QKV>();
    if (e == cudaSuccess) e = configure_gemv_e<EPI_GATE>();
    if (e == cudaSuccess) e = configure_gemv_e<EPI_RESID>();
    if (e == cudaSuccess) e = configure_gemv_e<EPI_LOGITS>();
    if (e == cudaSuccess) e = configure_gemv_mma();
    return e;
}

// Team size of a GEMV launch: at most kBPL blocks per lane and row, then doubled (up to 256 lanes,
// and not past one lane per block) until the launch has about 96 K lanes, so that a matrix with
// few units still spreads its bytes over the whole GPU.
int gemv_team(int64_t units, int NB) {
    int team = 8;
    while (team * kBPL < NB) team *= 2;
    while (team < 256 && team < NB && units * team < 96 * 1024) team *= 2;
    return team;
}

// CTAs of one GEMV launch: one per team-sized group of units, but no more than fit on the GPU at
// once, so that a CTA converts its input rows once and its teams then loop over units (each
// team's next unit in flight while it reduces the current one).
template <int MB, int EPI>
static int gemv_grid(int64_t units, int teams, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, int> resident;  // (device, smem) -> CTAs per GPU
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    int fit = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = resident.find({dev, smem});
        if (it != resident.end()) {
            fit = it->second;
        } else {
            int sms = 0, occ = 0;
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_kernel<MB, EPI>, kGemvThreads, smem) ==
                    cudaSuccess)
                fit = sms * std::max(occ, 1);
            (void)cudaGetLastError();
            resident[{dev, smem}] = fit;
        }
    }
    const int64_t want = (units + teams - 1) / teams;
    return (int)(fit > 0 ? std::min<int64_t>(want, fit) : want);
}

// Shared memory of the streamed GEMV: `stages` weight stages, then the limbs and exponents of MB
// rows; stages as many as fit (at most kSStages, at least 2).
static int gemv_stream_stages(int mb, int k) {
    const size_t limbs = gemv_smem_bytes(mb, k) + 1024;
    const int fit = (int)((kSmemLimit - std::min(kSmemLimit, limbs)) / kSStageBytes);
    return std::min(kSStages, fit);
}
// Which GEMV a launch takes.  The streamed kernel needs K a multiple of 256; it is the faster one
// except for one batch row over a large matrix (more than 40 units per SM: the 16896-row linear_in),
// where the register kernel's two resident CTAs per SM keep more loads in flight than one CTA's
// chain of stages (measured on B200: 6.5 against 7.7 us for 16896 x 2048, device time).
static bool gemv_streamed(const GemvArgs& a, int mb) {
    const int64_t row_bytes = (int64_t)(a.W.k / 32) * 18;
    if (a.W.k % 256 != 0 || 2 * row_bytes > kSStageBytes || gemv_stream_stages(mb, a.W.k) < 2) return false;
    return !(mb == 1 && a.n_units > 40 * 148);
}

template <int MB, int EPI>
static cudaError_t launch_gemv_stream(const Ctx& c, const GemvArgs& a, int rows, int* err, cudaStream_t st) {
    static std::mutex mu;
    static std::map<int, int> sms_of;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        std::lock_guard<std::mutex> lk(mu);
        auto it = sms_of.find(dev);
        if (it == sms_of.end()) {
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
            sms_of[dev] = sms;
        } else {
            sms = it->second;
        }
    }
    const int ups = (int)(kSStageBytes / (2u * (uint32_t)(a.W.k / 32) * 18u));
    const int grid = (int)std::min<int64_t>(sms, a.n_units);
    // no more stages than a CTA's share needs: a smaller CTA leaves room on the SM for the next kernel
    // of the stream (launched as a programmatic dependent) while this one finishes
    const int64_t per_cta = (a.n_units + grid - 1) / grid;
    const int stages = (int)std::max<int64_t>(
        2, std::min<int64_t>((int64_t)gemv_stream_stages(MB, a.W.k), (per_cta + ups - 1) / ups));
    const size_t smem = (size_t)stages * kSStageBytes + gemv_smem_bytes(MB, a.W.k);
    for (int r0 = 0; r0 < rows; r0 += MB) {
        const int mb = rows - r0 < MB ? rows - r0 : MB;
        const cudaError_t e = launch_pdl(gemv_stream_kernel<MB, EPI>, dim3(grid), dim3(32 * (stream_cwarps<MB>() + 1)),
                                         smem, st, c, a, r0, mb, ups, stages, err);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <int MB, int EPI>
static cudaError_t launch_gemv_t(const Ctx& c, const GemvArgs& a, int rows, cudaStream_t st) {
    if (gemv_mma_ok(a, MB)) return launch_gemv_mma(c, a, EPI, MB, rows, st);
    if (gemv_streamed(a, MB)) return launch_gemv_stream<MB, EPI>(c, a, rows, a.err, st);
    const int team = gemv_team(a.n_units, a.W.k / 32);
    const int teams = kGemvThreads / team;
    const size_t smem = gemv_smem_bytes(MB, a.W.k);
    const int grid = gemv_grid<MB, EPI>(a.n_units, teams, smem);
    for (int r0 = 0; r0 < rows; r0 += MB) {
        const int mb = rows - r0 < MB ? rows - r0 : MB;
        const cudaError_t e = launch_pdl(gemv_kernel<MB, EPI>, dim3(grid), dim3(kGemvThreads), smem, st, c, a, r0, mb,
                                         team);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <int EPI>
static cudaError_t launch_gemv_e(const Ctx& c, const GemvArgs& a, int rows, cudaStream_t st) {
    if (rows <= 1) return launch_gemv_t<1, EPI>(c, a, rows, st);
    if (rows == 2) return launch_gemv_t<2, EPI>(c, a, rows, st);
    if (rows <= 4 || a.W.k > 4096) return launch_gemv_t<4, EPI>(c, a, rows, st);
    return launch_gemv_t<8, EPI>(c, a, rows, st);
}

cudaError_t launch_gemv(const Ctx& c, const GemvArgs& a, int epi, int rows, cudaStream_t st) {
    if (rows <= 0 || a.n_units <= 0) return cudaSuccess;
    switch (epi) {
        case EPI_PLAIN: return launch_gemv_e<EPI_PLAIN>(c, a, rows, st);
        case EPI_QKV: return launch_gemv_e<EPI_QKV>(c, a, rows, st);
        case EPI_GATE: return launch_gemv_e<EPI_GATE>(c, a, rows, st);
        case EPI_RESID: return launch_gemv_e<EPI_RESID>(c, a, rows, st);
        default: return launch_gemv_e<EPI_LOGITS>(c, a, rows, st);
    }
}

cudaError_t launch_repack_q4(const uint8_t* raw, int64_t nblocks, uint4* nib, uint16_t* scale, cudaStream_t st,
                             int* big_scale) {
    if (nblocks <= 0) return cudaSuccess;
    const int64_t grid = (nblocks + 255) / 256;
    repack_q4_kernel<<<(unsigned)grid, 256, 0, st>>>(raw, nblocks, nib, scale, big_scale);
    return cudaGetLastError();
}

cudaError_t launch_dequant_q4(const Q4Dev& w, float* out, cudaStream_t st) {
    const int64_t nblocks = (int64_t)w.n * (w.k / 32);
    dequant_q4_kernel<<<(unsigned)((nblocks + 255) / 256), 256, 0, st>>>(w, out);
    return cudaGetLastError();
}

cudaError_t launch_embed(const Ctx& c, cudaStream_t st) {
    embed_kernel<<<dim3((c.D + 255) / 256, c.n), 256, 0, st>>>(c);
    return cudaGetLastError();
}

template <typename KT, int CH>
cudaError_t launch_attention_ch(const Ctx& c, int layer, dim3 grid, cudaStream_t st) {
    const size_t smem = attn_smem_bytes<KT, CH>();
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<KT, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_kernel<KT, CH>, grid, dim3(128), smem, st, c, layer);
}

cudaError_t launch_attention(const Ctx& c, int layer, cudaStream_t st) {
    dim3 grid(c.nsplit, c.H, c.n);
    const bool many = c.n >= 256;
    if (c.kv_f32)
        return many ? launch_attention_ch<float, 32>(c, layer, grid, st) : launch_attention_ch<float, 48>(c, layer, grid, st);
    return many ? launch_attention_ch<__nv_bfloat16, 32>(c, layer, grid, st)
                : launch_attention_ch<__nv_bfloat16, 48>(c, layer, grid, st);
}

cudaError_t launch_finish(const Ctx& c, cudaStream_t st) {
    finish_kernel<<<c.n, 1024, 0, st>>>(c);
    return cudaGetLastError();
}

template <int U>
static cudaError_t launch_tc_epilogue_u(const Ctx& c, const GemvArgs& a, int epi, int rows, const float* part,
                                        int slices, cudaStream_t st) {
    const dim3 grid((a.n_units + 256 * U - 1) / (256 * U), rows);
    switch (epi) {
        case EPI_QKV: return launch_pdl(tc_epilogue_kernel<EPI_QKV, U>, grid, dim3(256), 0, st, c, a, part, rows, slices);
        case EPI_GATE: return launch_pdl(tc_epilogue_kernel<EPI_GATE, U>, grid, dim3(256), 0, st, c, a, part, rows, slices);
        case EPI_RESID:
            return launch_pdl(tc_epilogue_kernel<EPI_RESID, U>, grid, dim3(256), 0, st, c, a, part, rows, slices);
        case EPI_LOGITS:
            return launch_pdl(tc_epilogue_kernel<EPI_LOGITS, U>, grid, dim3(256), 0, st, c, a, part, rows, slices);
        default: return launch_pdl(tc_epilogue_kernel<EPI_PLAIN, U>, grid, dim3(256), 0, st, c, a, part, rows, slices);
    }
}

cudaError_t launch_tc_epilogue(const Ctx& c, const GemvArgs& a, int epi, int rows, const float* part, int slices,
                               cudaStream_t st) {
    if (rows <= 0 || a.n_units <= 0) return cudaSuccess;
    return rows >= 128 ? launch_tc_epilogue_u<4>(c, a, epi, rows, part, slices, st)
                       : launch_tc_epilogue_u<1>(c, a, epi, rows, part, slices, st);
}

}  // namespace stt
