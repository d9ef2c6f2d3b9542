// The integer-MMA GEMV of the batched step: passes of 2 to 8 batch rows with K a multiple of 256
// (kernels.cu's launch_gemv chooses it; the dp4a kernels there take single rows).
#include <algorithm>
#include <map>
#include <mutex>

#include "device.cuh"
#include "gemv_common.cuh"
#include "kernels.h"
#include "tc_gemm.h"

namespace stt {

// ------------------------------------------------------------------------------------ MMA GEMV
//
// The batched Q4 GEMV on the integer tensor cores (1 to 8 batch rows per pass, K a multiple of 256):
// the same products as gemv_kernel, with each Q4_0 block's dot product computed exactly as an
// integer by mma.sync m16n8k32 (s8 x s8 -> s32), sixteen weight rows at a time.
//
// Operands.  A weight word holds 8 nibbles; 16 * (nibble - 8) is a signed byte.  A 32-element
// block is exactly one MMA k-extent, and the block's own element order is the fragment order: lane
// (g, t) of the warp holds, for weight rows g and g + 8, the low nibbles of word t (elements 4t ..
// 4t+3, k = 4t .. 4t+3) and its high nibbles (elements 16+4t .. 16+4t+3, k = 16+4t ..), which is
// word t of the block as loaded.  The input block becomes 23-bit fixed point with a per-block
// exponent e (max |x| < 2^e, X = rn(x * 2^(22 - e))), cut into three balanced signed digits
// X = D0 + 256 D1 + 65536 D2 (|D2| <= 64); each (digit, batch row) is one column of the MMA's B.
// So S = sum 16 (q - 8) D is exact (|S| <= 2^19), the block's value is
// d * 2^(e - 26) * (S0 + 256 S1 + 65536 S2), and only the f32 accumulation over digits and blocks
// rounds (as in the reference's f32 shader, crates/stt-wasm/src/wgsl/shader_naive.wgsl:51-95).
// The accumulator starts at the bit pattern of 2^23 + 2^22, so the int32 result read as an f32 is
// 12582912 + S exactly: one subtraction converts it.
//
// Columns of B: MB = 1: n = v; MB = 2: n = 3m + v; MB = 4: n = 2m + v (v < 2) in the first MMA and
// n = 2m (v = 2) in the second; MB = 8: MMA j = digit v, column n = m.  Lane (g, t) reads the
// accumulator columns 2t and 2t + 1, which then belong to at most two batch rows ("slots").
//
// Pipeline.  One CTA per SM: warp 16 TMA-loads, per 16-row tile and per stage of up to 8 quads
// (2048 elements of K), the tile's nibbles (two 3-D boxes of 8 quads x 8 rows: rows 0..7 and 8..15
// of the tile; for the gate product the 8 gate rows and their 8 value rows) and scales (two boxes of
// 64 scales x 8 rows), 128-byte swizzled so that the 8 lanes reading one word of 8 rows hit 8
// different banks, into a ring of stages: four loads per 18 KB stage.  The 16
// consumer warps first turn the input rows into digits (while the first loads fly), then work in
// `groups` groups of G = 16 / groups warps: a group takes the CTA's tiles i = group, group +
// groups, ..., its warps splitting each stage's blocks; at the end of a tile each lane adds its
// columns into its slots, the group's warps exchange them through shared memory (one named barrier
// per tile, double-buffered) and the group's threads add them in a fixed order and apply the
// epilogue.  Every wait is bounded; a wait that gives up records STT_E_DEVICE_FLAG and makes every
// later wait of the CTA return at once, while all warps still reach the same barriers.
namespace mg {
constexpr int kCWarps = 16;                         // consumer warps
constexpr int kThreads = 32 * (kCWarps + 1);        // and the producer warp
constexpr int kQuads = 8;                           // quads (8 blocks, 256 elements) per stage
constexpr uint32_t kNibBytes = kQuads * 2048;       // [row half][quad][8 rows][128 B]
constexpr uint32_t kStageBytes = kNibBytes + 2048;  // then the scales, [16 rows][128 B]
constexpr int kMaxStages = 10;
constexpr int kMaxGroups = 8;
constexpr uint32_t kMagic = 0x4B400000u;            // 12582912.0f
}  // namespace mg

template <int MB>
__host__ __device__ constexpr int mg_mmas() { return MB == 8 ? 3 : MB == 4 ? 2 : 1; }

// Column n of MMA j: 4 * (batch row) + digit, or -1 when unused.
template <int MB>
__host__ __device__ constexpr int mg_col(int j, int n) {
    return MB == 1   ? (j == 0 && n < 3 ? n : -1)
           : MB == 2 ? (n < 6 ? 4 * (n / 3) + n % 3 : -1)
           : MB == 4 ? (j == 0 ? 4 * (n / 2) + n % 2 : (n % 2 == 0 ? 4 * (n / 2) + 2 : -1))
                     : 4 * n + j;
}
// The batch row of slot 0 of lane group t (columns 2t, 2t + 1).
template <int MB>
__host__ __device__ constexpr int mg_mbase(int t) {
    return MB == 1 ? 0 : MB == 2 ? (2 * t) / 3 : MB == 4 ? t : 2 * t;
}
// Where batch row m's sums sit: lane groups t[i] and slots s[i], i < returned count.
template <int MB>
__host__ __device__ inline int mg_places(int m, int* t, int* s) {
    if (MB == 1 || (MB == 2 && m == 0)) {
        t[0] = 0, s[0] = 0, t[1] = 1, s[1] = 0;
        return 2;
    }
    if (MB == 2) {
        t[0] = 1, s[0] = 1, t[1] = 2, s[1] = 0;
        return 2;
    }
    if (MB == 4) {
        t[0] = m, s[0] = 0;
        return 1;
    }
    t[0] = m >> 1, s[0] = m & 1;
    return 1;
}

// Byte offsets inside a stage: word t of block lb (of the stage) of tile row g (box 0: rows 0..7,
// box 1: rows 8..15), and that row's scale of block lb; both follow the TMA's 128-byte swizzle
// (16-byte chunk c of 128-byte line r stored at chunk c ^ (r & 7)).
__host__ __device__ inline uint32_t mg_nib_off(int lb, int g, int t, int box) {
    return (uint32_t)(box * (mg::kQuads * 1024) + (lb >> 3) * 1024 + g * 128 + ((((lb & 7) ^ g) & 7) << 4) + 4 * t);
}
__host__ __device__ inline uint32_t mg_sc_off(int lb, int g, int box) {
    return mg::kNibBytes + (uint32_t)(box * 1024 + g * 128 + ((((lb >> 3) ^ g) & 7) << 4) + 2 * (lb & 7));
}
// Digit words: DW[block][half * 3 + digit][m][t] (half 0: elements 4t..4t+3, 1: 16+4t..16+4t+3),
// each block's record padded by 4 words so that the 4 blocks a warp converts at once start in
// different banks.
__host__ __device__ inline int mg_digit_word(int MB, int b, int half, int v, int m, int t) {
    return b * (24 * MB + 4) + ((half * 3 + v) * MB + m) * 4 + t;
}

// Shared memory of one CTA (offsets from the 1024-byte aligned base).
struct MgLayout {
    uint32_t dw, xv, ex, red, total;
};
__host__ __device__ inline MgLayout mg_layout(int MB, int NB, int stages) {
    const int nm = MB == 8 ? 3 : MB == 4 ? 2 : 1;
    MgLayout l;
    uint32_t off = (uint32_t)stages * mg::kStageBytes;
    l.dw = off;
    off += (uint32_t)NB * (24u * MB + 4u) * 4u;  // digits
    l.xv = off;
    off += (uint32_t)NB * nm * 8u * 4u;    // per (block, MMA, column): 2^(e - 26 + 8 v), or 0
    l.ex = off;
    off += (uint32_t)MB * NB * 4u;         // per (batch row, block): 2^(e - 26)
    l.red = off;
    off += 2u * mg::kCWarps * 128u * 4u;  // tile sums: [buffer][warp][row half][slot][lane]
    l.total = off + 1024u;                 // alignment slack
    return l;
}

__device__ __forceinline__ void mg_mma(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int (&d)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"((int)mg::kMagic));
}

__device__ __forceinline__ void mg_tma(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void mg_tma3(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// Bounded wait; returns at once (false) once the CTA's stop word is set.
__device__ __forceinline__ bool mg_wait(uint64_t* m, uint32_t parity, volatile int* stop) {
    for (uint32_t i = 0; i < kSSpin; ++i) {
        if ((i & 63u) == 0 && *stop) return false;
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

// Digits of one half block (16 elements: half h of block b of batch row m) and, from half 0,
// ex[m][b] = 2^(e - 26).  The two halves of a block are neighbouring lanes (h = lane & 1), which
// share the block's maximum by a shuffle, so every lane of the warp calls this (`valid` false: no
// stores; both halves of a block are valid or neither is).  With |X| <= 2^22, Y = X + 0x808080
// lies in [0, 2^24) and its three bytes are the balanced digits plus 128, so the digits are Y's
// bytes with the top bit flipped.
__device__ __forceinline__ void mg_half_digits(uint32_t* DW, float* ex, int MB, int NB, int m, int b, int h,
                                               const float (&x)[16], bool valid) {
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(x[i]));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
    if (!valid) return;
    // mx < 2^e; e >= -96 keeps 2^(e - 26) normal, and e <= 128 for every finite mx
    const int e = max(-96, mx > 0.0f ? (int)((__float_as_uint(mx) >> 23) & 0xFF) - 126 : 0);
    const float up = __uint_as_float((uint32_t)(127 + 22 - e) << 23);
    uint32_t* rec = DW + mg_digit_word(MB, b, h, 0, m, 0);
#pragma unroll
    for (int t = 0; t < 4; ++t) {  // elements 4t .. 4t+3 of the half
        const uint32_t y0 = (uint32_t)(__float2int_rn(__fmul_rn(x[4 * t + 0], up)) + 0x808080);
        const uint32_t y1 = (uint32_t)(__float2int_rn(__fmul_rn(x[4 * t + 1], up)) + 0x808080);
        const uint32_t y2 = (uint32_t)(__float2int_rn(__fmul_rn(x[4 * t + 2], up)) + 0x808080);
        const uint32_t y3 = (uint32_t)(__float2int_rn(__fmul_rn(x[4 * t + 3], up)) + 0x808080);
        const uint32_t t01 = __byte_perm(y0, y1, 0x5140), t23 = __byte_perm(y2, y3, 0x5140);  // bytes 0, 1
        const uint32_t u01 = __byte_perm(y0, y1, 0x0062), u23 = __byte_perm(y2, y3, 0x0062);  // byte 2
        rec[(0 * MB) * 4 + t] = __byte_perm(t01, t23, 0x5410) ^ 0x80808080u;
        rec[(1 * MB) * 4 + t] = __byte_perm(t01, t23, 0x7632) ^ 0x80808080u;
        rec[(2 * MB) * 4 + t] = __byte_perm(u01, u23, 0x5410) ^ 0x80808080u;
    }
    if (h == 0) ex[m * NB + b] = __uint_as_float((uint32_t)(127 + e - 26) << 23);
}

template <int MB, int EPI>
__global__ void __launch_bounds__(mg::kThreads, 1)
    gemv_mma_kernel(const __grid_constant__ CUtensorMap tm_nib, const __grid_constant__ CUtensorMap tm_sc, Ctx c,
                    GemvArgs a, int row0, int mb, int stages, int groups, int* err) {
    constexpr int NM = mg_mmas<MB>();
    extern __shared__ uint8_t mg_raw[];
    uint8_t* smem = mg_raw + ((1024u - (smem_addr(mg_raw) & 1023u)) & 1023u);
    const int K = a.W.k, NB = K >> 5, NQ = NB >> 3;
    const int nst = (NQ + mg::kQuads - 1) / mg::kQuads;
    const MgLayout lay = mg_layout(MB, NB, stages);
    uint32_t* DW = reinterpret_cast<uint32_t*>(smem + lay.dw);
    float* XV = reinterpret_cast<float*>(smem + lay.xv);
    float* EX = reinterpret_cast<float*>(smem + lay.ex);
    float* RED = reinterpret_cast<float*>(smem + lay.red);
    __shared__ __align__(8) uint64_t full[mg::kMaxStages], empty[mg::kMaxStages];
    __shared__ float nred[MB * mg::kCWarps];
    __shared__ int stop;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr bool gate = EPI == EPI_GATE;
    const int64_t tiles = gate ? ((int64_t)a.half_n + 7) / 8 : ((int64_t)a.W.n + 15) / 16;
    const int G = mg::kCWarps / groups;
    if (tid == 0) {
        for (int i = 0; i < stages; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[i])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&empty[i])), "r"(G) : "memory");
        }
        stop = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();
    if (warp == mg::kCWarps) {
        // producer: the weights are constant, so their loads start before the previous kernel ends
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int64_t tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
                const int yA = gate ? (int)(8 * tile) : (int)(16 * tile);
                const int yB = gate ? yA + a.half_n : yA + 8;
                for (int sj = 0; sj < nst; ++sj) {
                    const int k = issued, s = k % stages;
                    if (k >= stages && !mg_wait(&empty[s], (uint32_t)((k / stages) - 1) & 1u, &stop)) {
                        ok = false;
                        break;
                    }
                    if (k == 0 && a.stall_test && blockIdx.x == 0) {  // test hook: stage 0 never lands
                        issued = 1;
                        continue;
                    }
                    uint8_t* st = smem + (size_t)s * mg::kStageBytes;
                    // whole boxes, quads past the end read as zeros
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&full[s])),
                                 "r"(mg::kStageBytes)
                                 : "memory");
                    mg_tma3(st, &tm_nib, 0, yA, sj * mg::kQuads, &full[s]);
                    mg_tma3(st + mg::kNibBytes / 2, &tm_nib, 0, yB, sj * mg::kQuads, &full[s]);
                    mg_tma(st + mg::kNibBytes, &tm_sc, sj * 64, yA, &full[s]);
                    mg_tma(st + mg::kNibBytes + 1024, &tm_sc, sj * 64, yB, &full[s]);
                    issued = k + 1;
                }
            }
            if (!ok) {
                stop = 1;
                if (c.desc) raise_error(c.desc, -5);  // STT_E_DEVICE_FLAG
                if (err) atomicCAS(err, 0, -5);
            }
            // every load must land before the CTA's shared memory goes away (the stage the test hook
            // skipped has none)
            for (int k = max(0, issued - stages); k < issued; ++k) {
                if (k == 0 && a.stall_test && blockIdx.x == 0) continue;
                const int s = k % stages;
                for (uint32_t i = 0; i < kSSpin; ++i) {
                    uint32_t done;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                        "selp.u32 %0, 1, 0, p;\n\t}"
                        : "=r"(done)
                        : "r"(smem_addr(&full[s])), "r"((uint32_t)(k / stages) & 1u)
                        : "memory");
                    if (done) break;
                }
            }
        }
        __syncwarp();
        pdl_wait();
        return;
    }

    // consumers: the input rows become digits while the first loads fly.  A thread converts half a
    // block (16 elements of one row) at a time while the loads of its next half block fly; the two
    // halves of a block are neighbouring threads, and the CTAs start at different blocks so that
    // they do not all read the same lines at once.
    pdl_wait();
    {
        constexpr int kT = 32 * mg::kCWarps;
        const int total = mb * NB, total2 = 2 * total;  // blocks, half blocks
        const float inv_nb = 1.0f / (float)NB;
        // row of block item i: (i + 1/2) / NB is at least 1/(2 NB) from an integer, far more than
        // the rounding of the product
        auto row_of = [&](int i) { return __float2int_rz(__fmul_rn((float)i + 0.5f, inv_nb)); };
        const int rot = (int)((blockIdx.x * 37u) % (uint32_t)total);
        // half block j: half j & 1 of block item (j / 2 + rot) mod total
        auto half_item = [&](int j, int& m, int& b, int& h) {
            int i = (j >> 1) + rot;
            if (i >= total) i -= total;
            m = row_of(i);
            b = i - m * NB;
            h = j & 1;
        };
        auto load = [&](int m, int b, int h, float (&x)[16]) {
            const int64_t off = (int64_t)(row0 + m) * K + 32 * b + 16 * h;
            if (a.in_bf16) {
                const uint4* p = reinterpret_cast<const uint4*>(a.in_bf16 + off);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint4 r = p[c];
                    x[8 * c + 0] = __uint_as_float(r.x << 16), x[8 * c + 1] = __uint_as_float(r.x & 0xFFFF0000u);
                    x[8 * c + 2] = __uint_as_float(r.y << 16), x[8 * c + 3] = __uint_as_float(r.y & 0xFFFF0000u);
                    x[8 * c + 4] = __uint_as_float(r.z << 16), x[8 * c + 5] = __uint_as_float(r.z & 0xFFFF0000u);
                    x[8 * c + 6] = __uint_as_float(r.w << 16), x[8 * c + 7] = __uint_as_float(r.w & 0xFFFF0000u);
                }
            } else {
                const float4* p = reinterpret_cast<const float4*>(a.in + off);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 v = p[c];
                    x[4 * c + 0] = v.x, x[4 * c + 1] = v.y, x[4 * c + 2] = v.z, x[4 * c + 3] = v.w;
                }
            }
        };
        float rms[MB];
#pragma unroll
        for (int m = 0; m < MB; ++m) rms[m] = 1.0f;
        if (a.norm) {
            // RMSNorm denominators of the rows (burn::nn::RmsNorm: sqrt(mean(x^2) + 1e-8))
            float ss[MB];
#pragma unroll
            for (int m = 0; m < MB; ++m) ss[m] = 0.0f;
            for (int j = tid; j < total2; j += kT) {
                float x[16];
                int m, b, h;
                half_item(j, m, b, h);
                load(m, b, h, x);
                float q2 = 0.0f;
#pragma unroll
                for (int c = 0; c < 16; ++c) q2 = __fmaf_rn(x[c], x[c], q2);
#pragma unroll
                for (int mm = 0; mm < MB; ++mm)
                    if (mm == m) ss[mm] += q2;
            }
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                const float w = warp_sum(ss[m]);
                if (lane == 0 && m < mb) nred[m * mg::kCWarps + warp] = w;
            }
            asm volatile("bar.sync 15, %0;" ::"n"(32 * mg::kCWarps) : "memory");
#pragma unroll
            for (int m = 0; m < MB; ++m)
                if (m < mb) {
                    float tot = 0.0f;
                    for (int w = 0; w < mg::kCWarps; ++w) tot += nred[m * mg::kCWarps + w];
                    rms[m] = sqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), 1e-8f));
                }
        }
        // every thread runs the same rounds: the halves of a block share a shuffle
        const int rounds = (total2 + kT - 1) / kT;
        float xn[16];
        int mn = 0, bn = 0, hn = 0;
#pragma unroll
        for (int c = 0; c < 16; ++c) xn[c] = 0.0f;
        if (tid < total2) {
            half_item(tid, mn, bn, hn);
            load(mn, bn, hn, xn);
        }
        for (int r = 0; r < rounds; ++r) {
            const int j = tid + r * kT;
            const bool valid = j < total2;
            float x[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) x[c] = xn[c];
            const int m = mn, b = bn, h = hn;
            if (j + kT < total2) {  // the next half block's loads fly while this one is converted
                half_item(j + kT, mn, bn, hn);
                load(mn, bn, hn, xn);
            }
            if (valid && a.norm) {
                float rr = 1.0f;
#pragma unroll
                for (int mm = 0; mm < MB; ++mm)
                    if (mm == m) rr = rms[mm];
                const float4* al = reinterpret_cast<const float4*>(a.norm + 32 * b + 16 * h);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 w = al[c];
                    x[4 * c + 0] = __fmul_rn(__fdiv_rn(x[4 * c + 0], rr), w.x);
                    x[4 * c + 1] = __fmul_rn(__fdiv_rn(x[4 * c + 1], rr), w.y);
                    x[4 * c + 2] = __fmul_rn(__fdiv_rn(x[4 * c + 2], rr), w.z);
                    x[4 * c + 3] = __fmul_rn(__fdiv_rn(x[4 * c + 3], rr), w.w);
                }
            }
            mg_half_digits(DW, EX, MB, NB, m, b, h, x, valid);
        }
        asm volatile("bar.sync 15, %0;" ::"n"(32 * mg::kCWarps) : "memory");
        // column factors: 2^(e - 26 + 8 v) for the columns in use, 0 for the others (and for batch
        // rows past mb, whose digits were never written)
        for (int i = tid; i < NB * NM * 8; i += 32 * mg::kCWarps) {
            const int b = i / (NM * 8), j = (i / 8) % NM, n = i & 7;
            const int col = mg_col<MB>(j, n);
            float f = 0.0f;
            if (col >= 0 && (col >> 2) < mb) {
                const int v = col & 3;
                f = EX[(col >> 2) * NB + b] * (v == 0 ? 1.0f : v == 1 ? 256.0f : 65536.0f);
            }
            XV[i] = f;
        }
        asm volatile("bar.sync 15, %0;" ::"n"(32 * mg::kCWarps) : "memory");
    }

    const int gi = warp / G, wg = warp % G;
    const int g = lane >> 2, t = lane & 3;
    int boff[NM], slot[NM][2];
#pragma unroll
    for (int j = 0; j < NM; ++j) {
        const int col = mg_col<MB>(j, g);
        boff[j] = col < 0 ? -1 : mg_digit_word(MB, 0, 0, col & 3, col >> 2, t);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int c2 = mg_col<MB>(j, 2 * t + h);
            slot[j][h] = c2 < 0 ? -1 : (c2 >> 2) - mg_mbase<MB>(t);
        }
    }
    int buf = 0;
    for (int64_t i = gi;; i += groups) {
        const int64_t tile = blockIdx.x + i * (int64_t)gridDim.x;
        if (tile >= tiles) break;
        float acc[NM][4], acc2[NM][4];
#pragma unroll
        for (int j = 0; j < NM; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[j][i] = acc2[j][i] = 0.0f;
        for (int sj = 0; sj < nst; ++sj) {
            const int64_t k = i * nst + sj;
            const int s = (int)(k % stages);
            bool ok = true;
            if (lane == 0) ok = mg_wait(&full[s], (uint32_t)((k / stages) & 1), &stop);
            if (!__shfl_sync(0xFFFFFFFFu, (int)ok, 0) && lane == 0) {
                stop = 1;
                if (c.desc) raise_error(c.desc, -5);  // STT_E_DEVICE_FLAG
                if (err) atomicCAS(err, 0, -5);
            }
            const uint8_t* st = smem + (size_t)s * mg::kStageBytes;
            const int nb = 8 * min(mg::kQuads, NQ - sj * mg::kQuads);
            // one block of the stage into acc; two blocks per step, into separate sums, so that
            // their loads and MMAs overlap
            auto block = [&](int lb, float (&ac)[NM][4]) {
                const uint32_t wA = *reinterpret_cast<const uint32_t*>(st + mg_nib_off(lb, g, t, 0));
                const uint32_t wB = *reinterpret_cast<const uint32_t*>(st + mg_nib_off(lb, g, t, 1));
                const float dA = f16_to_f32_ieee(*reinterpret_cast<const uint16_t*>(st + mg_sc_off(lb, g, 0)));
                const float dB = f16_to_f32_ieee(*reinterpret_cast<const uint16_t*>(st + mg_sc_off(lb, g, 1)));
                uint32_t af[4];
                af[0] = ((wA << 4) & 0xF0F0F0F0u) ^ 0x80808080u;  // rows g, g+8: low nibbles, k = 4t..4t+3
                af[1] = ((wB << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
                af[2] = (wA & 0xF0F0F0F0u) ^ 0x80808080u;          // high nibbles, k = 16+4t..16+4t+3
                af[3] = (wB & 0xF0F0F0F0u) ^ 0x80808080u;
                const int b = sj * (8 * mg::kQuads) + lb;
                const uint32_t* dwb = DW + (size_t)b * (24 * MB + 4);
                const float* xvb = XV + (size_t)b * NM * 8 + 2 * t;
#pragma unroll
                for (int j = 0; j < NM; ++j) {
                    const uint32_t b0 = boff[j] >= 0 ? dwb[boff[j]] : 0u;
                    const uint32_t b1 = boff[j] >= 0 ? dwb[boff[j] + 12 * MB] : 0u;
                    int d[4];
                    mg_mma(af, b0, b1, d);
                    const float2 xv = *reinterpret_cast<const float2*>(xvb + j * 8);
                    ac[j][0] = __fmaf_rn(__fsub_rn(__int_as_float(d[0]), 12582912.0f), __fmul_rn(dA, xv.x), ac[j][0]);
                    ac[j][2] = __fmaf_rn(__fsub_rn(__int_as_float(d[2]), 12582912.0f), __fmul_rn(dB, xv.x), ac[j][2]);
                    if (mg_col<MB>(j, 1) >= 0 || mg_col<MB>(j, 3) >= 0) {  // odd columns in use
                        ac[j][1] = __fmaf_rn(__fsub_rn(__int_as_float(d[1]), 12582912.0f), __fmul_rn(dA, xv.y), ac[j][1]);
                        ac[j][3] = __fmaf_rn(__fsub_rn(__int_as_float(d[3]), 12582912.0f), __fmul_rn(dB, xv.y), ac[j][3]);
                    }
                }
            };
            int lb = wg;
            for (; lb + G < nb; lb += 2 * G) {
                block(lb, acc);
                block(lb + G, acc2);
            }
            if (lb < nb) block(lb, acc);
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&empty[s])) : "memory");
        }
        // this lane's columns into its slots, then the group's warps through shared memory
        float rs[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // [row half][slot]
#pragma unroll
        for (int j = 0; j < NM; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (slot[j][h] == 0) {
                    rs[0][0] += acc[j][h] + acc2[j][h];
                    rs[1][0] += acc[j][2 + h] + acc2[j][2 + h];
                } else if (slot[j][h] == 1) {
                    rs[0][1] += acc[j][h] + acc2[j][h];
                    rs[1][1] += acc[j][2 + h] + acc2[j][2 + h];
                }
            }
        float* R = RED + ((size_t)buf * mg::kCWarps + warp) * 128;
        R[lane] = rs[0][0];
        R[32 + lane] = rs[0][1];
        R[64 + lane] = rs[1][0];
        R[96 + lane] = rs[1][1];
        asm volatile("bar.sync %0, %1;" ::"r"(1 + gi), "r"(32 * G) : "memory");
        for (int it = wg * 32 + lane; it < 8 * mb; it += 32 * G) {
            const int m = it >> 3, p = it & 7;
            const int64_t u = 8 * tile + p;
            if (u >= a.n_units) continue;
            int pt[2], ps[2];
            const int np = mg_places<MB>(m, pt, ps);
            float vals[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = gate ? p + 8 * h : 2 * p + h;  // the unit's two rows in the tile
                float sum = 0.0f;
                for (int w = gi * G; w < gi * G + G; ++w) {
                    const float* Rw = RED + ((size_t)buf * mg::kCWarps + w) * 128 + (r >> 3) * 64 + 4 * (r & 7);
                    for (int x = 0; x < np; ++x) sum += Rw[ps[x] * 32 + pt[x]];
                }
                vals[h] = sum;
            }
            int ra, rb;
            unit_rows<EPI>(a, (int)u, &ra, &rb);
            epilogue<EPI>(c, a, row0 + m, ra, rb, vals[0], vals[1]);
        }
        buf ^= 1;
    }
}

// SMs of the current device (cached per device).
static int device_sms() {
    static std::mutex mu;
    static std::map<int, int> sms_of;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess) return sms;
    std::lock_guard<std::mutex> lk(mu);
    auto it = sms_of.find(dev);
    if (it != sms_of.end()) return it->second;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    sms_of[dev] = sms;
    return sms;
}

cudaError_t gemv_make_maps(const Q4Dev& w, GemvMaps* out) {
    out->ok = false;
    if (w.k % 256 != 0) return cudaSuccess;
    const uint64_t nb = (uint64_t)(w.k / 32);
    // nibbles as [quad][row][128 bytes]: one box is 8 quads (a stage) of 8 rows
    const uint64_t dims[3] = {128, (uint64_t)w.n, nb / 8};
    const uint64_t strides[2] = {nb * 16, 128};
    const uint32_t box[3] = {128, 8, (uint32_t)mg::kQuads};
    cudaError_t e = tma_encode(&out->nib, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.nib, 3, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (e == cudaSuccess)
        e = tma_encode_2d(&out->sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.scale, nb, (uint64_t)w.n, nb * 2, 64, 8,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    out->ok = e == cudaSuccess;
    return e;
}

// Stages of the MMA GEMV that fit beside its digits, column factors and tile sums.
static int mg_stages_fit(int mb, int nb) {
    const MgLayout l = mg_layout(mb, nb, 0);
    if (l.total >= kSmemLimit) return 0;
    return std::min<int>(mg::kMaxStages, (int)((kSmemLimit - l.total) / mg::kStageBytes));
}
// Which batches take the MMA GEMV: passes of 2 to 8 rows.  A single row fills 3 of an MMA's 8
// columns, and the dp4a kernels need fewer instructions per weight row for it.
bool gemv_mma_ok(const GemvArgs& a, int mb) {
    return mb >= 2 && a.maps && a.maps->ok && a.W.k % 256 == 0 && mg_stages_fit(mb, a.W.k / 32) >= 2;
}

// One CTA per SM (or per tile, when there are fewer tiles), groups of warps so that the CTA's tiles
// run side by side, each group with a stage in flight, and no more stages than the CTA's share of
// the matrix needs (the rest of the SM's shared memory is left to the next kernel of the stream,
// which starts early as a programmatic dependent).
template <int MB, int EPI>
static cudaError_t launch_gemv_mma_t(const Ctx& c, const GemvArgs& a, int rows, cudaStream_t st) {
    const int NB = a.W.k / 32, NQ = NB / 8, nst = (NQ + mg::kQuads - 1) / mg::kQuads;
    const int64_t tiles = EPI == EPI_GATE ? ((int64_t)a.half_n + 7) / 8 : ((int64_t)a.W.n + 15) / 16;
    const int grid = (int)std::min<int64_t>(tiles, device_sms());
    const int fit = mg_stages_fit(MB, NB);
    const int64_t per_cta = (tiles + grid - 1) / grid;
    int groups = 1;
    while (groups * 2 <= mg::kMaxGroups && groups * 2 <= per_cta && groups * 2 * nst <= fit) groups *= 2;
    const int stages = (int)std::max<int64_t>(2, std::min<int64_t>(fit, per_cta * nst));
    const size_t smem = mg_layout(MB, NB, stages).total;
    for (int r0 = 0; r0 < rows; r0 += MB) {
        const int mb = rows - r0 < MB ? rows - r0 : MB;
        const cudaError_t e = launch_pdl(gemv_mma_kernel<MB, EPI>, dim3(grid), dim3(mg::kThreads), smem, st,
                                         a.maps->nib, a.maps->sc, c, a, r0, mb, stages, groups, a.err);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <int MB>
static cudaError_t launch_gemv_mma_m(const Ctx& c, const GemvArgs& a, int epi, int rows, cudaStream_t st) {
    switch (epi) {
        case EPI_PLAIN: return launch_gemv_mma_t<MB, EPI_PLAIN>(c, a, rows, st);
        case EPI_QKV: return launch_gemv_mma_t<MB, EPI_QKV>(c, a, rows, st);
        case EPI_GATE: return launch_gemv_mma_t<MB, EPI_GATE>(c, a, rows, st);
        case EPI_RESID: return launch_gemv_mma_t<MB, EPI_RESID>(c, a, rows, st);
        default: return launch_gemv_mma_t<MB, EPI_LOGITS>(c, a, rows, st);
    }
}

cudaError_t launch_gemv_mma(const Ctx& c, const GemvArgs& a, int epi, int mb, int rows, cudaStream_t st) {
    switch (mb) {
        case 2: return launch_gemv_mma_m<2>(c, a, epi, rows, st);
        case 4: return launch_gemv_mma_m<4>(c, a, epi, rows, st);
        case 8: return launch_gemv_mma_m<8>(c, a, epi, rows, st);
        default: return cudaErrorInvalidValue;
    }
}

template <int MB, int EPI>
static cudaError_t configure_mma_t() {
    return cudaFuncSetAttribute(gemv_mma_kernel<MB, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);
}
template <int MB>
static cudaError_t configure_mma_m() {
    cudaError_t e = configure_mma_t<MB, EPI_PLAIN>();
    if (e == cudaSuccess) e = configure_mma_t<MB, EPI_QKV>();
    if (e == cudaSuccess) e = configure_mma_t<MB, EPI_GATE>();
    if (e == cudaSuccess) e = configure_mma_t<MB, EPI_RESID>();
    if (e == cudaSuccess) e = configure_mma_t<MB, EPI_LOGITS>();
    return e;
}

cudaError_t configure_gemv_mma() {
    cudaError_t e = configure_mma_m<2>();
    if (e == cudaSuccess) e = configure_mma_m<4>();
    if (e == cudaSuccess) e = configure_mma_m<8>();
    return e;
}

}  // namespace stt
