// Q4_0 x f16 matmul on the 5th-generation tensor cores (tcgen05, accumulator in TMEM).
//
// out[m][n] = sum_k x[m][k] * w[n][k] for a batch of rows m (streams) and the Q4_0 weight rows n:
// the product of q4_matmul (gguf.rs:517-578) with f16 operands.  The weights are dequantised to
// f16 ((nibble - 8) * scale, rounded to nearest) and multiplied with f16 inputs, accumulating in
// f32.  This is the batched-stream form of the layer product; its rounding (f16 operands) is the
// tolerance the multi-stream path is held to, not the exact per-block arithmetic of the
// single-stream kernel.
//
// One CTA computes 128 weight rows (the MMA's M, one TMEM lane each) for NT batch rows (the MMA's
// N, one TMEM column each).  K advances in chunks of 64 (two Q4_0 blocks):
//   - 128 threads dequantise one weight row each into shared memory, in the no-swizzle K-major
//     "core matrix" layout of the MMA (8 rows x 16 bytes per 128-byte core matrix), and copy the
//     chunk of the batch rows the same way;
//   - one thread issues four 128 x NT x 16 MMAs and commits them to an mbarrier;
//   - two buffers alternate, so the threads prepare chunk c+1 while the MMAs of chunk c run.
// After the last chunk every warp reads its 32 TMEM lanes (tcgen05.ld 32x32b) and stores them.
// Every wait is bounded; on a timeout the CTA records an error, waits (bounded) for its MMAs,
// frees its TMEM and returns.
#include "tc_gemm.h"

namespace stt {

namespace {

constexpr int kTM = 128;          // weight rows per CTA (MMA M)
constexpr int kKC = 64;           // K elements per chunk
constexpr int kThreads = 128;     // one thread per weight row; warp w owns TMEM lanes 32w..32w+31
constexpr uint32_t kSpin = 1u << 22;

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
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int NT>
struct TcSmem {
    alignas(128) uint8_t a[2][kTM * kKC * 2];  // dequantised weights, core-matrix layout
    alignas(128) uint8_t b[2][NT * kKC * 2];   // batch rows
    alignas(8) uint64_t mbar[2];
    uint32_t tmem;
    int32_t ok;
};

// byte offset of element (row, k) of a [rows x 64] K-major chunk in the core-matrix layout:
// core matrix (row / 8, k / 8) at ((row / 8) * 8 + k / 8) * 128, row % 8 at 16-byte steps
__device__ __forceinline__ uint32_t core_off(int row, int k8) { return ((row >> 3) * 8 + k8) * 128 + (row & 7) * 16; }

template <int NT>
__global__ void __launch_bounds__(kThreads) q4_tc_kernel(Q4Dev w, const __half* __restrict__ x, int M, float* __restrict__ out,
                                                       int64_t ldo, int* __restrict__ err) {
    extern __shared__ __align__(128) uint8_t tc_raw[];
    TcSmem<NT>& sm = *reinterpret_cast<TcSmem<NT>*>(tc_raw);
    constexpr uint32_t kCols = NT < 32 ? 32 : NT;  // TMEM columns (a power of two >= 32)
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int n0 = blockIdx.x * kTM, m0 = blockIdx.y * NT;
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
    const int row = n0 + t;  // this thread's weight row
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
        const int buf = c & 1;
        if (c >= 2 && !mbar_wait(&sm.mbar[buf], ((c >> 1) - 1) & 1)) ok = false;  // MMAs of chunk c-2 are done
        // weights: two Q4_0 blocks of this row -> 64 f16 values
        uint8_t* A = sm.a[buf];
        if (row < w.n) {
            const int b0 = c * 2;
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
                const uint4 q = __ldg(w.nib + (int64_t)row * NB + b0 + bb);
                const float d = f16_to_f32_ieee(__ldg(w.scale + (int64_t)row * NB + b0 + bb));
                const uint32_t words[4] = {q.x, q.y, q.z, q.w};
                __half lo[16], hi[16];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t byte = (words[wi] >> (8 * i)) & 0xFFu;
                        lo[4 * wi + i] = __float2half_rn(__fmul_rn(nib_m8(byte & 0xFu), d));
                        hi[4 * wi + i] = __float2half_rn(__fmul_rn(nib_m8(byte >> 4), d));
                    }
                // elements 0-15 (low nibbles) and 16-31 (high nibbles) of block bb: k8 = 4 bb + 0..3
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    *reinterpret_cast<uint4*>(A + core_off(t, 4 * bb + j)) = *reinterpret_cast<const uint4*>(&lo[8 * j]);
                    *reinterpret_cast<uint4*>(A + core_off(t, 4 * bb + 2 + j)) = *reinterpret_cast<const uint4*>(&hi[8 * j]);
                }
            }
        } else {
#pragma unroll
            for (int k8 = 0; k8 < 8; ++k8) *reinterpret_cast<uint4*>(A + core_off(t, k8)) = make_uint4(0, 0, 0, 0);
        }
        // batch rows: NT x 64 f16 = NT * 8 pieces of 16 bytes; piece p -> (k8 = p / NT, r = p % NT)
        uint8_t* B = sm.b[buf];
        for (int p = t; p < NT * 8; p += kThreads) {
            const int k8 = p / NT, r = p % NT;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (m0 + r < M) v = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)(m0 + r) * K + c * kKC + k8 * 8));
            *reinterpret_cast<uint4*>(B + core_off(r, k8)) = v;
        }
        // generic-proxy writes of the tiles -> visible to the tensor cores (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        if (t == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_addr = smem_u32(sm.a[buf]), b_addr = smem_u32(sm.b[buf]);
#pragma unroll
            for (int k16 = 0; k16 < kKC / 16; ++k16) {
                // K = 16 is two core matrices along K: LBO 128 bytes, 8-row groups 1024 bytes apart
                const uint64_t ad = smem_desc(a_addr + k16 * 256, 128, 1024);
                const uint64_t bd = smem_desc(b_addr + k16 * 256, 128, 1024);
                mma_f16(tmem, ad, bd, idesc, (c > 0 || k16 > 0) ? 1u : 0u);
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
    if (sm.ok) {
        const int orow = n0 + warp * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
        for (int j0 = 0; j0 < NT; j0 += 16) {
            float v[16];
            tmem_ld16(lane_addr + j0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int m = m0 + j0 + j;
                if (m < M && orow < w.n) out[(int64_t)m * ldo + orow] = v[j];
            }
        }
    } else if (t == 0) {
        atomicCAS(err, 0, 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

template <int NT>
cudaError_t launch_nt(const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo, int* err, cudaStream_t st) {
    const size_t smem = sizeof(TcSmem<NT>);
    cudaError_t e = cudaFuncSetAttribute(q4_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((w.n + kTM - 1) / kTM, (M + NT - 1) / NT);
    q4_tc_kernel<NT><<<grid, kThreads, smem, st>>>(w, x, M, out, ldo, err);
    return cudaGetLastError();
}

}  // namespace

bool tc_gemm_supported(const Q4Dev& w) { return w.k % kKC == 0 && w.k >= kKC; }

cudaError_t launch_q4_tc_gemm(const Q4Dev& w, const __half* x, int M, float* out, int64_t ldo, int* err, cudaStream_t st) {
    if (M <= 16) return launch_nt<16>(w, x, M, out, ldo, err, st);
    if (M <= 32) return launch_nt<32>(w, x, M, out, ldo, err, st);
    if (M <= 64) return launch_nt<64>(w, x, M, out, ldo, err, st);
    if (M <= 128) return launch_nt<128>(w, x, M, out, ldo, err, st);
    return launch_nt<256>(w, x, M, out, ldo, err, st);
}

}  // namespace stt
