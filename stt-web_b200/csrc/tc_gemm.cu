// Q4_0 x f16 matmul on the 5th-generation tensor cores (tcgen05, accumulator in TMEM).
//
// out[m][n] = sum_k x[m][k] * w[n][k] for a batch of rows m (streams) and the Q4_0 weight rows n:
// the product of q4_matmul (gguf.rs:517-578) on the f16 tensor cores with f32 accumulation.  Each
// operand is split into two f16 parts, w = w_hi + w_lo and x = x_hi + x_lo, and three MMAs add
// w_hi.x_hi + w_hi.x_lo + w_lo.x_hi: about 22 significant bits per product, close to the f32
// reference.  The dequantised weight (nibble - 8) * scale is exact in f32; it is scaled by 2^10
// (exact) before the split so that w_lo stays clear of f16 subnormals, and the accumulator is
// scaled back in the epilogue.
//
// One CTA computes 128 weight rows (the MMA's M, one TMEM lane each) for NT batch rows (the MMA's
// N, one TMEM column each).  K advances in chunks of 64 (two Q4_0 blocks):
//   - 128 threads dequantise one weight row each into shared memory (hi and lo parts), in the
//     no-swizzle K-major "core matrix" layout of the MMA (8 rows x 16 bytes per 128-byte core
//     matrix), and copy the chunk of the batch rows (hi and lo parts) the same way;
//   - one thread issues 4 x 3 MMAs of 128 x NT x 16 and commits them to an mbarrier;
//   - two buffers alternate, so the threads prepare chunk c+1 while the MMAs of chunk c run.
// After the last chunk every warp reads its 32 TMEM lanes (tcgen05.ld 32x32b) and stores them.
// Every wait is bounded; on a timeout the CTA records an error, waits (bounded) for its MMAs,
// frees its TMEM and returns.
#include "tc_gemm.h"

#include "kernels.h"

namespace stt {

namespace {

constexpr int kTM = 128;          // weight rows per CTA (MMA M)
constexpr int kKC = 64;           // K elements per chunk
constexpr int kThreads = 128;     // one thread per weight row; warp w owns TMEM lanes 32w..32w+31
constexpr uint32_t kSpin = 1u << 22;
constexpr float kWScale = 1024.0f;          // weights enter the MMA scaled by 2^10
constexpr float kWUnscale = 1.0f / 1024.0f;

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

// 16 consecutive f32 columns of this thread's TMEM lane.
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
    alignas(128) uint8_t a[2][2][kTM * kKC * 2];  // [buffer][hi, lo] dequantised weights, core-matrix layout
    alignas(128) uint8_t b[2][2][NT * kKC * 2];   // [buffer][hi, lo] batch rows
    alignas(8) uint64_t mbar[2];
    uint32_t tmem;
    int32_t ok;
    float gv[64][17];  // EPI_GATE: the value rows' results, handed to the gate rows
    int2 pos[NT];      // EPI_QKV: (RoPE position, ring slot) of each batch row of the tile
};

// byte offset of element (row, k) of a [rows x 64] K-major chunk in the core-matrix layout:
// core matrix (row / 8, k / 8) at ((row / 8) * 8 + k / 8) * 128, row % 8 at 16-byte steps
__device__ __forceinline__ uint32_t core_off(int row, int k8) { return ((row >> 3) * 8 + k8) * 128 + (row & 7) * 16; }

// Weight row of tile row t: consecutive rows, or for the gate epilogue 64 gate rows followed by
// their 64 value rows (rows u and u + half_n of linear_in).
template <int EPI>
__device__ __forceinline__ int tile_row(int tile, int t, int half_n) {
    if (EPI == EPI_GATE) return t < 64 ? tile * 64 + t : half_n + tile * 64 + (t - 64);
    return tile * kTM + t;
}

// x holds the hi parts [M][K], then (x_lo != 0) the lo parts [M][K]; without lo parts the input
// is taken as exact f16 and the hi.lo product is skipped.
template <int NT, int EPI>
__global__ void __launch_bounds__(kThreads) q4_tc_kernel(Q4Dev w, const __half* __restrict__ x, int x_lo, int M,
                                                       float* __restrict__ out, int64_t ldo, int* __restrict__ err, Ctx c,
                                                       GemvArgs ga) {
    extern __shared__ __align__(128) uint8_t tc_raw[];
    TcSmem<NT>& sm = *reinterpret_cast<TcSmem<NT>*>(tc_raw);
    constexpr uint32_t kCols = NT < 32 ? 32 : NT;  // TMEM columns (a power of two >= 32)
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int m0 = blockIdx.y * NT;
    const int K = w.k, NB = K >> 5, nchunks = K / kKC;
    if (t == 0) {
        mbar_init(&sm.mbar[0]);
        mbar_init(&sm.mbar[1]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sm.ok = 1;
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
    const uint32_t idesc = instr_desc_f16(kTM, NT);
    const int row = tile_row<EPI>(blockIdx.x, t, ga.half_n);  // this thread's weight row
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
        const int buf = c & 1;
        if (c >= 2 && !mbar_wait(&sm.mbar[buf], ((c >> 1) - 1) & 1)) ok = false;  // MMAs of chunk c-2 are done
        // weights: two Q4_0 blocks of this row -> 64 values, each split into f16 hi and lo parts
        uint8_t* Ah = sm.a[buf][0];
        uint8_t* Al = sm.a[buf][1];
        if (row < w.n) {
            const int b0 = c * 2;
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
                const uint4 q = __ldg(w.nib + (int64_t)row * NB + b0 + bb);
                const float d = __fmul_rn(f16_to_f32_ieee(__ldg(w.scale + (int64_t)row * NB + b0 + bb)), kWScale);
                const uint32_t words[4] = {q.x, q.y, q.z, q.w};
                // element e of the block: e < 16 low nibble of byte e, e >= 16 high nibble of byte e-16
                __half hv[32], lv[32];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t byte = (words[wi] >> (8 * i)) & 0xFFu;
                        const float wl = __fmul_rn(nib_m8(byte & 0xFu), d), wh = __fmul_rn(nib_m8(byte >> 4), d);
                        const __half hl = __float2half_rn(wl), hh = __float2half_rn(wh);
                        hv[4 * wi + i] = hl;
                        lv[4 * wi + i] = __float2half_rn(__fsub_rn(wl, __half2float(hl)));
                        hv[16 + 4 * wi + i] = hh;
                        lv[16 + 4 * wi + i] = __float2half_rn(__fsub_rn(wh, __half2float(hh)));
                    }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    *reinterpret_cast<uint4*>(Ah + core_off(t, 4 * bb + j)) = *reinterpret_cast<const uint4*>(&hv[8 * j]);
                    *reinterpret_cast<uint4*>(Al + core_off(t, 4 * bb + j)) = *reinterpret_cast<const uint4*>(&lv[8 * j]);
                }
            }
        } else {
#pragma unroll
            for (int k8 = 0; k8 < 8; ++k8) {
                *reinterpret_cast<uint4*>(Ah + core_off(t, k8)) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(Al + core_off(t, k8)) = make_uint4(0, 0, 0, 0);
            }
        }
        // batch rows, hi and lo: NT x 64 f16 each = NT * 8 pieces of 16 bytes; piece p -> (k8 = p / NT,
        // r = p % NT)
        for (int part = 0; part < 1 + x_lo; ++part) {
            uint8_t* B = sm.b[buf][part];
            const __half* xp = x + (int64_t)part * M * K;
            for (int p = t; p < NT * 8; p += kThreads) {
                const int k8 = p / NT, r = p % NT;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (m0 + r < M) v = __ldg(reinterpret_cast<const uint4*>(xp + (int64_t)(m0 + r) * K + c * kKC + k8 * 8));
                *reinterpret_cast<uint4*>(B + core_off(r, k8)) = v;
            }
        }
        // generic-proxy writes of the tiles -> visible to the tensor cores (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        if (t == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ah = smem_u32(sm.a[buf][0]), al = smem_u32(sm.a[buf][1]);
            const uint32_t bh = smem_u32(sm.b[buf][0]), bl = smem_u32(sm.b[buf][1]);
#pragma unroll
            for (int k16 = 0; k16 < kKC / 16; ++k16) {
                // K = 16 is two core matrices along K: LBO 128 bytes, 8-row groups 1024 bytes apart
                const uint32_t o = k16 * 256;
                mma_f16(tmem, smem_desc(ah + o, 128, 1024), smem_desc(bh + o, 128, 1024), idesc, (c > 0 || k16 > 0) ? 1u : 0u);
                if (x_lo) mma_f16(tmem, smem_desc(ah + o, 128, 1024), smem_desc(bl + o, 128, 1024), idesc, 1u);
                mma_f16(tmem, smem_desc(al + o, 128, 1024), smem_desc(bh + o, 128, 1024), idesc, 1u);
            }
            mma_commit(&sm.mbar[buf]);
        }
    }
    // the last commit covers every MMA of the CTA
    const int last = nchunks - 1;
    if (!mbar_wait(&sm.mbar[last & 1], (last >> 1) & 1)) ok = false;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) sm.ok = 0;
    __syncthreads();
    if (EPI == EPI_QKV) {
        for (int j = t; j < NT; j += kThreads) {
            int2 v = make_int2(0, 0);
            if (m0 + j < M) {
                const StreamState st = c.state[c.ids[m0 + j]];
                v = make_int2(st.offset, st.write_pos);
            }
            sm.pos[j] = v;
        }
        __syncthreads();
    }
    if (sm.ok) {
        // tile row t = TMEM lane t = this thread (warp w reads lanes 32w .. 32w+31)
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
        for (int j0 = 0; j0 < NT; j0 += 16) {
            float v[16];
            tmem_ld16(lane_addr + j0, v);
            if (EPI == EPI_GATE) {
                // value rows hand their results to the gate rows
                if (t >= 64)
#pragma unroll
                    for (int j = 0; j < 16; ++j) sm.gv[t - 64][j] = v[j];
                __syncthreads();
                if (t < 64 && row < w.n)
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int m = m0 + j0 + j;
                        if (m >= M) break;
                        const float g = v[j];
                        // silu(x) = x * (1 / (1 + exp(-x)))
                        const float sg = __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
                        out[(int64_t)m * ldo + row] = __fmul_rn(sg, sm.gv[t][j]);
                    }
                __syncthreads();
            } else if (EPI == EPI_QKV) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float other = __shfl_xor_sync(0xFFFFFFFFu, v[j], 1);  // the pair's odd row
                    const int m = m0 + j0 + j;
                    if ((t & 1) || m >= M || row >= w.n) continue;
                    float va = v[j], vb = other;
                    const int D = c.D, HD = c.HD;
                    const int part = row / D, within = row - part * D;
                    const int h = within / HD, d = within - h * HD;
                    const int2 ps = sm.pos[j0 + j];
                    if (part < 2) {
                        // RoPE::apply_rotation (model.rs:114-116) on the pair (2i, 2i+1)
                        const float2 cs = c.rope[(int64_t)ps.x * (HD >> 1) + (d >> 1)];
                        const float re = __fsub_rn(__fmul_rn(va, cs.x), __fmul_rn(vb, cs.y));
                        const float im = __fadd_rn(__fmul_rn(va, cs.y), __fmul_rn(vb, cs.x));
                        va = re;
                        vb = im;
                    }
                    out[(int64_t)m * ldo + row] = va;
                    out[(int64_t)m * ldo + row + 1] = vb;
                    if (part >= 1) {
                        const int64_t off = (int64_t)c.ids[m] * c.kv_stream_stride + (int64_t)ga.layer * c.kv_layer_stride +
                                            (part == 2 ? c.kv_half_stride : 0) + ((int64_t)h * c.ML + ps.y) * HD + d;
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
            } else if (row < w.n) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = m0 + j0 + j;
                    if (m >= M) break;
                    float* o = out + (int64_t)m * ldo + row;
                    *o = EPI == EPI_RESID ? __fadd_rn(v[j], *o) : v[j];
                }
            }
        }
    } else if (t == 0) {
        atomicCAS(err, 0, 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

template <int NT, int EPI>
cudaError_t launch_nt(const Q4Dev& w, const __half* x, int x_lo, int M, float* out, int64_t ldo, int* err, const Ctx& c,
                      const GemvArgs& ga, cudaStream_t st) {
    const size_t smem = sizeof(TcSmem<NT>);
    cudaError_t e = cudaFuncSetAttribute(q4_tc_kernel<NT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int tiles = EPI == EPI_GATE ? ga.half_n / 64 : (w.n + kTM - 1) / kTM;
    dim3 grid(tiles, (M + NT - 1) / NT);
    q4_tc_kernel<NT, EPI><<<grid, kThreads, smem, st>>>(w, x, x_lo, M, out, ldo, err, c, ga);
    return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_epi(const Q4Dev& w, const __half* x, int x_lo, int M, float* out, int64_t ldo, int* err, const Ctx& c,
                       const GemvArgs& ga, cudaStream_t st) {
    if (M <= 16) return launch_nt<16, EPI>(w, x, x_lo, M, out, ldo, err, c, ga, st);
    if (M <= 32) return launch_nt<32, EPI>(w, x, x_lo, M, out, ldo, err, c, ga, st);
    if (M <= 64) return launch_nt<64, EPI>(w, x, x_lo, M, out, ldo, err, c, ga, st);
    if (M <= 128) return launch_nt<128, EPI>(w, x, x_lo, M, out, ldo, err, c, ga, st);
    return launch_nt<256, EPI>(w, x, x_lo, M, out, ldo, err, c, ga, st);
}

// f16 GEMM input of a batch: row m of `in` (f32, or bf16 when in_bf16), with RMSNorm when alpha is
// not NULL (the same arithmetic as the GEMV's prologue: x / rms * alpha), split into f16 hi and lo
// parts: out[m][k] = hi, out[rows + m][k] = lo.
__global__ void __launch_bounds__(256) prep_f16_kernel(const float* __restrict__ in, const __nv_bfloat16* __restrict__ in_bf16,
                                                       const float* __restrict__ alpha, int K, __half* __restrict__ out) {
    __shared__ float red[32];
    const int64_t base = (int64_t)blockIdx.x * K;
    float rms = 1.0f;
    if (alpha) {
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
    const int64_t lo_off = (int64_t)gridDim.x * K;  // the lo parts follow the hi parts of all rows
    for (int j = threadIdx.x; j < K; j += blockDim.x) {
        float v = in_bf16 ? __bfloat162float(in_bf16[base + j]) : in[base + j];
        if (alpha) v = __fmul_rn(__fdiv_rn(v, rms), alpha[j]);
        const __half h = __float2half_rn(v);
        out[base + j] = h;
        out[lo_off + base + j] = __float2half_rn(__fsub_rn(v, __half2float(h)));
    }
}

}  // namespace

bool tc_gemm_supported(const Q4Dev& w) { return w.k % kKC == 0 && w.k >= kKC; }

cudaError_t launch_q4_tc_gemm(const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo, int* err, cudaStream_t st) {
    return launch_epi<EPI_PLAIN>(w, x, 0, M, out, ldo, err, Ctx{}, GemvArgs{}, st);
}

cudaError_t launch_tc_layer(const Ctx& c, const GemvArgs& a, int epi, int rows, __half* x16, int* err, cudaStream_t st) {
    prep_f16_kernel<<<rows, 256, 0, st>>>(a.in, a.in_bf16, a.norm, a.W.k, x16);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    switch (epi) {
        case EPI_QKV: return launch_epi<EPI_QKV>(a.W, x16, 1, rows, a.out, a.ldo, err, c, a, st);
        case EPI_GATE: return launch_epi<EPI_GATE>(a.W, x16, 1, rows, a.out, a.ldo, err, c, a, st);
        case EPI_RESID: return launch_epi<EPI_RESID>(a.W, x16, 1, rows, a.out, a.ldo, err, c, a, st);
        case EPI_LOGITS: return launch_epi<EPI_LOGITS>(a.W, x16, 1, rows, a.out, a.ldo, err, c, a, st);
        default: return launch_epi<EPI_PLAIN>(a.W, x16, 1, rows, a.out, a.ldo, err, c, a, st);
    }
}

}  // namespace stt
