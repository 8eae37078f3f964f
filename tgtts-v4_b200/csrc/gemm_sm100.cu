// The prefill's projection GEMM, C[m][n] = A[m][k] B[n][k]^T with f32 accumulation
// (kernels/gpu/gemm.mlir:14-29; a linear layer: A the activations, B the weights as a checkpoint
// lays them out, both K-major).
//
// bf16: a tcgen05 kernel. Each block computes a 128 x BN tile of C. One thread streams A and B
// tiles of 64 columns of K into a ring of shared-memory stages with TMA (128-byte swizzle, no
// multicast), one thread issues tcgen05.mma into a TMEM accumulator (M = 128, N = BN, K = 16 per
// instruction) and releases each stage with tcgen05.commit, and all four warps read the
// accumulator back with tcgen05.ld for the epilogue. Every wait on an mbarrier is bounded: past
// its limit the kernel sets the context's error word and runs to its end.
//
// f32: a SIMT kernel, each sum sequential in k.
#include "tc_common.cuh"

namespace tg {

// ---- f32 SIMT ---------------------------------------------------------------------------------

__global__ void __launch_bounds__(256)
    gemm_f32_kernel(int M, int N, int K, const float *__restrict__ A, const float *__restrict__ B,
                    float *__restrict__ C) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int r = i / 16, kk = i % 16;
            As[kk][r] = (m0 + r < M && k0 + kk < K) ? A[(size_t)(m0 + r) * K + k0 + kk] : 0.0f;
            Bs[kk][r] = (n0 + r < N && k0 + kk < K) ? B[(size_t)(n0 + r) * K + k0 + kk] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                a[i] = As[kk][ty * 4 + i];
                b[i] = Bs[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tx * 4 + j;
            if (n < N) C[(size_t)m * N + n] = acc[i][j];
        }
    }
}

// ---- tcgen05 bf16 ------------------------------------------------------------------------------

constexpr int TC_BM = 128, TC_BK = 64, TC_STAGES = 4, TC_THREADS = 128;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;  // 16 KiB per stage


template <int BN>
struct TcLayout {
    static constexpr int B_BYTES = BN * TC_BK * 2;
    static constexpr int STAGE = TC_A_BYTES + B_BYTES;
    static constexpr int BARRIERS = TC_STAGES * STAGE;  // offset of the mbarriers
    static constexpr int SMEM = BARRIERS + 256 + 1024;  // + barriers + alignment slack
};

// Epilogues: C in f32, or (BN = 256, B's rows in gate_up_row's order) SiLU(gate) up in bf16, the
// tile's columns 0..127 the gate and 128..255 the up of the same 128 outputs.
enum { TC_EPI_F32 = 0, TC_EPI_SILU = 1 };

template <int BN, int EPI = TC_EPI_F32>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   void *__restrict__ Cout, int M, int N, int K, uint32_t *err) {
    using L = TcLayout<BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_u32(smem);
    const uint32_t bars = base + L::BARRIERS;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (TC_STAGES + s); };
    const uint32_t done = bars + 8u * (2 * TC_STAGES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::BARRIERS + 8 * (2 * TC_STAGES + 1));
    __shared__ int gave_up;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * BN;
    const int nk = K / TC_BK;

    if (threadIdx.x == 0) {
        gave_up = 0;
        for (int s = 0; s < TC_STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // Producer: stage kb of A and B into slot kb % STAGES once the MMAs have released it.
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % TC_STAGES;
            mbar_wait(empty(s), ((kb / TC_STAGES) & 1) ^ 1, err, &gave_up);
            mbar_arrive_expect_tx(full(s), L::STAGE);
            tma_load_2d(base + s * L::STAGE, &map_a, kb * TC_BK, m0, full(s));
            tma_load_2d(base + s * L::STAGE + TC_A_BYTES, &map_b, kb * TC_BK, n0, full(s));
            issued = kb + 1;
        }
        // Every copy this thread started has landed before the block can end.
        for (int kb = issued > TC_STAGES ? issued - TC_STAGES : 0; kb < issued; kb++)
            mbar_wait(full(kb % TC_STAGES), (kb / TC_STAGES) & 1, err, &gave_up);
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: four K = 16 steps per stage, accumulating after the first.
        constexpr uint32_t idesc = bf16_idesc(TC_BM, BN);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % TC_STAGES;
            mbar_wait(full(s), (kb / TC_STAGES) & 1, err, &gave_up);
            tc_fence_after();
            const uint32_t a_addr = base + s * L::STAGE;
            const uint32_t b_addr = a_addr + TC_A_BYTES;
#pragma unroll
            for (int k = 0; k < TC_BK / 16; k++) {
                tc_mma(tmem, sw128_desc(a_addr + k * 32), sw128_desc(b_addr + k * 32), idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
            }
            tc_commit(empty(s));
        }
        tc_commit(done);
    }
    __syncwarp();

    // Epilogue: row m0 + 32 warp + lane, BN columns from TMEM, 16 at a time.
    mbar_wait(done, 0, err, &gave_up);
    tc_fence_after();
    const int row = m0 + warp * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    if constexpr (EPI == TC_EPI_SILU) {
        static_assert(BN == 256, "the SiLU epilogue pairs columns c and c + 128 of a 256-wide tile");
        bf16 *out = static_cast<bf16 *>(Cout);
        const int inner = N / 2;
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 16) {
            float g[16], u[16];
            tmem_ld16(lane_base + c0, g);
            tmem_ld16(lane_base + 128 + c0, u);
            if (row < M) {
                uint32_t packed[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const __nv_bfloat162 v = __floats2bfloat162_rn(silu_mul(g[2 * i], u[2 * i]), silu_mul(g[2 * i + 1], u[2 * i + 1]));
                    packed[i] = *reinterpret_cast<const uint32_t *>(&v);
                }
                uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)row * inner + n0 / 2 + c0);
                dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
            }
        }
    } else {
        float *C = static_cast<float *>(Cout);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            tmem_ld16(lane_base + c0, v);
            if (row < M && n0 + c0 < N) {
                float4 *dst = reinterpret_cast<float4 *>(C + (size_t)row * N + n0 + c0);
#pragma unroll
                for (int i = 0; i < 4; i++) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN)
                     : "memory");
    }
}

// ---- host -------------------------------------------------------------------------------------

template <int BN, int EPI = TC_EPI_F32>
static cudaError_t launch_tc(const void *a, const void *b, void *c, int M, int N, int K, uint32_t *err,
                             cudaStream_t s) {
    CUtensorMap ma, mb;
    if (!make_map_bf16(&ma, a, (uint64_t)M, (uint64_t)K, TC_BM) || !make_map_bf16(&mb, b, (uint64_t)N, (uint64_t)K, BN))
        return cudaErrorInvalidValue;
    auto kern = gemm_tc_kernel<BN, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TcLayout<BN>::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid(N / BN, (M + TC_BM - 1) / TC_BM);
    kern<<<grid, TC_THREADS, TcLayout<BN>::SMEM, s>>>(ma, mb, c, M, N, K, err);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const tg_params &p, const void *a, const void *b, float *c, uint32_t *err,
                        cudaStream_t s) {
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    if (M <= 0 || N <= 0 || K <= 0) return cudaErrorInvalidValue;
    if (p.dtype != TG_BF16) {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        gemm_f32_kernel<<<grid, 256, 0, s>>>(M, N, K, (const float *)a, (const float *)b, c);
        return cudaGetLastError();
    }
    if (K % TC_BK != 0) return cudaErrorInvalidValue;
    if (N % 256 == 0) return launch_tc<256>(a, b, c, M, N, K, err, s);
    if (N % 128 == 0) return launch_tc<128>(a, b, c, M, N, K, err, s);
    if (N % 64 == 0) return launch_tc<64>(a, b, c, M, N, K, err, s);
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemm_silu(const tg_params &p, const void *a, const void *b, void *out, uint32_t *err,
                             cudaStream_t s) {
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    if (p.dtype != TG_BF16 || M <= 0 || N % 256 || K % TC_BK) return cudaErrorInvalidValue;
    return launch_tc<256, TC_EPI_SILU>(a, b, out, M, N, K, err, s);
}

}  // namespace tg
