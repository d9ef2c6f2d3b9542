// Exact fixed-point dot products of Q4_0 blocks with dp4a (shared by the persistent single-stream
// kernel and the batched GEMV).
//
// An input vector is cut into its 32-element Q4_0 blocks.  Each block gets a shared exponent e
// (max |x| < 2^e) and its elements become 24-bit integers X = round(x * 2^(23 - e)), stored as
// three byte limbs: X = L0 + 256 L1 + 65536 L2 (L0, L1 unsigned, L2 signed).  A weight word holds
// 8 nibbles: its 4 low nibbles are elements 4w .. 4w+3 of the block and its 4 high nibbles elements
// 16+4w .. 16+4w+3, so the limbs are grouped the same way:
//   L[v][w] for v = 0, 1, 2: limb v of elements 4w .. 4w+3;  v = 3, 4, 5: of elements 16+4w .. +3.
// 16 * (nibble - 8) is a signed byte, so one dp4a per (limb, half-word) sums four products exactly;
// the three limb sums combine into 16 * sum((nibble - 8) * X) and the block scale and 2^(e - 27)
// bring it back.  Every block's dot product is therefore exact up to the input's 24-bit rounding,
// and only the per-block scale multiply and the f32 accumulation over blocks round, as in the
// reference's f32 shader (crates/stt-wasm/src/wgsl/shader_naive.wgsl:51-95).
#pragma once

#include "device.cuh"

namespace stt {

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

// 16 * sum over one Q4_0 block of (nibble - 8) * X in fixed point (S0 + 256 S1 + 65536 S2); L holds
// the block's six limb words in the order above.
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

// Limbs of one quad (elements 4q .. 4q+3, q = 8b + g of block b) into L ([6][NB] uint4, word g & 3
// of the low-half or high-half group) and, from the block's first quad, xs[b] = 2^(e - 27).  Called
// by all 32 lanes of a warp with 8 consecutive lanes holding the 8 quads of a block; a lane whose
// `store` is false (past the end of the vector) still joins the shuffles with zeros.
__device__ __forceinline__ void quad_limbs_store(uint4* L, float* xs, int q, int NB, float4 v, bool store) {
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
    uint32_t X[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) X[i] = (uint32_t)max(-(1 << 23), min(__float2int_rn(vals[i] * up), (1 << 23) - 1));
    // limb v of the four elements = byte v of each X (two's complement: byte 2 is the signed top)
    const uint32_t t01 = __byte_perm(X[0], X[1], 0x5140), t23 = __byte_perm(X[2], X[3], 0x5140);
    const uint32_t u01 = __byte_perm(X[0], X[1], 0x0062), u23 = __byte_perm(X[2], X[3], 0x0062);
    const uint32_t w0 = __byte_perm(t01, t23, 0x5410), w1 = __byte_perm(t01, t23, 0x7632);
    const uint32_t w2 = __byte_perm(u01, u23, 0x5410);
    if (!store) return;
    uint32_t* W = reinterpret_cast<uint32_t*>(L);
    const int base = g < 4 ? 0 : 3;
    W[((base + 0) * NB + b) * 4 + (g & 3)] = w0;
    W[((base + 1) * NB + b) * 4 + (g & 3)] = w1;
    W[((base + 2) * NB + b) * 4 + (g & 3)] = w2;
    if (g == 0) xs[b] = __uint_as_float((uint32_t)(127 + e - 27) << 23);
}

}  // namespace stt
