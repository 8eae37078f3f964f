// The prefill's causal attention (attention_rows.comp:46-126) on tcgen05, for bf16 and a head
// dimension of 64: flash attention with both products on the tensor cores and their accumulators
// in TMEM.
//
// Block (t, h) takes query rows [128 t, 128 t + 128) of the launch (one run's rows: runs start on
// multiples of 128) for query head h, and walks its slot's cache from position 0 to the tile's last
// position in tiles of 128 keys. Six warps:
//   warp 0   TMA: the Q tile once, then K and V tiles into two stages (128-byte swizzle, no
//            multicast);
//   warp 1   TMEM (two S buffers of 128 columns and O's 64) and the MMAs: S_j = Q K_j^T
//            (M = 128, N = 128, K = 64) into S[j % 2], one tile ahead of the softmax, and
//            PV_j = P_j V_j (M = 128, N = 64, K = 128; V read MN-major) into O;
//   warps 2-5 a thread to a query row: S_j from TMEM, the causal mask, the online softmax
//            (base 2, the scale folded in), P_j as bf16 into shared memory as PV's A operand,
//            and PV_{j-1} from TMEM folded into the row's f32 output in registers.
// Every wait on an mbarrier is bounded (the context's error word, then the block runs out).
#include "tc_common.cuh"

namespace tg {

namespace {

constexpr int FA_THREADS = 192;
constexpr uint32_t FA_TILE = 128 * 64 * 2;                    // a 128-row x 64-column bf16 box
constexpr uint32_t FA_Q = 0, FA_K = FA_TILE, FA_V = 3 * FA_TILE, FA_P = 5 * FA_TILE;  // P: 2 boxes
constexpr uint32_t FA_SMEM = 120 * 1024 + 1024;               // one block to an SM (TMEM: 512 columns)

// 2^x by the hardware's approximate base-2 exponential (PTX ex2.approx.ftz.f32: relative error
// about 2^-22, far below the bf16 rounding the probabilities take next); 2^-inf = 0.
TG_DEVICE float fa_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

TG_DEVICE uint32_t fa_sw128(int n, int c) {
    return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4));
}

// A K-major operand with 128-byte rows in the 128-byte swizzle (sw128_desc), or the same bytes read
// MN-major: V's tile [keys][64] is B = V^T with N = 64 along a row and K = keys down the rows, in
// atoms of 8 keys x 128 bytes, 1024 bytes apart along K.
TG_DEVICE uint64_t fa_desc_mn(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3fff) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

}  // namespace

__global__ void __launch_bounds__(FA_THREADS, 1)
    attention_rows_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, tg_params p, const uint32_t *__restrict__ at,
                             bf16 *__restrict__ out, uint32_t *err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_u32(smem);
    __shared__ __align__(8) uint64_t bq, bkv_full[2], bkv_empty[2], bs_full[2], bs_empty[2], bp_full, bo_full, bo_empty;
    __shared__ uint32_t tmem_slot, t_last, t_slot, t_slot_max;
    __shared__ int gave_up;
    __shared__ int pos_s[128];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int tile = gridDim.x - 1 - blockIdx.x;  // the latest rows, the longest walks, first
    const int head = blockIdx.y, heads = p.heads, kvh = p.kv_heads, kv = head / (heads / kvh);
    const int r0 = tile * 128;
    auto B = [](uint64_t &b) { return smem_u32(&b); };

    if (tid == 0) {
        gave_up = 0;
        t_last = 0;
        t_slot = 0xffffffffu;
        t_slot_max = 0;
        mbar_init(B(bq), 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(B(bkv_full[i]), 1);
            mbar_init(B(bkv_empty[i]), 1);
            mbar_init(B(bs_full[i]), 1);
            mbar_init(B(bs_empty[i]), 128);
        }
        mbar_init(B(bp_full), 128);
        mbar_init(B(bo_full), 1);
        mbar_init(B(bo_empty), 128);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(512u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    __syncthreads();  // the barriers and t_* are initialised
    if (tid < 128) {
        const int row = r0 + tid;
        uint32_t pos, slot;
        pos_s[tid] = -1;
        if (row < (int)p.rows && placed(at, p.rows, row, p.capacity, p.slots, pos, slot)) {
            pos_s[tid] = (int)pos;
            atomicMax(&t_last, pos);
            atomicMin(&t_slot, slot);
            atomicMax(&t_slot_max, slot);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    // A tile must hold one run's rows (one slot); one that does not is refused, not computed.
    const bool mixed = t_slot != 0xffffffffu && t_slot != t_slot_max;
    if (mixed && tid == 0) atomicExch(err, ERR_BAD_INDEX);
    const int n = (t_slot == 0xffffffffu || mixed) ? 0 : (int)(t_last / 128 + 1);  // key tiles

    if (warp == 0) {
        if (lane == 0 && n > 0) {
            mbar_arrive_expect_tx(B(bq), FA_TILE);
            tma_load_2d(base + FA_Q, &qmap, head * 64, r0, B(bq));
            const int row0 = (int)((t_slot * (uint32_t)kvh + kv) * p.capacity);
            for (int j = 0; j < n; j++) {
                const int b = j & 1;
                mbar_wait(B(bkv_empty[b]), ((j >> 1) & 1) ^ 1, err, &gave_up);
                mbar_arrive_expect_tx(B(bkv_full[b]), 2 * FA_TILE);
                tma_load_2d(base + FA_K + b * FA_TILE, &kmap, 0, row0 + j * 128, B(bkv_full[b]));
                tma_load_2d(base + FA_V + b * FA_TILE, &vmap, 0, row0 + j * 128, B(bkv_full[b]));
            }
            // Every copy this thread started has landed before the block can end.
            for (int j = n > 2 ? n - 2 : 0; j < n; j++) mbar_wait(B(bkv_full[j & 1]), (j >> 1) & 1, err, &gave_up);
        }
    } else if (warp == 1) {
        if (lane == 0 && n > 0) {
            constexpr uint32_t idesc_s = bf16_idesc(128, 128);
            constexpr uint32_t idesc_o = bf16_idesc(128, 64) | (1u << 16);  // B (V) MN-major
            mbar_wait(B(bq), 0, err, &gave_up);
            auto issue_s = [&](int j) {
                const int b = j & 1;
                mbar_wait(B(bkv_full[b]), (j >> 1) & 1, err, &gave_up);
                mbar_wait(B(bs_empty[b]), ((j >> 1) & 1) ^ 1, err, &gave_up);
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 4; k++)
                    tc_mma(tmem + (uint32_t)(b * 128), sw128_desc(base + FA_Q + k * 32),
                           sw128_desc(base + FA_K + b * FA_TILE + k * 32), idesc_s, k > 0 ? 1u : 0u);
                tc_commit(B(bs_full[b]));
            };
            issue_s(0);
            for (int j = 0; j < n; j++) {
                if (j + 1 < n) issue_s(j + 1);
                mbar_wait(B(bp_full), j & 1, err, &gave_up);
                if (j > 0) mbar_wait(B(bo_empty), (j - 1) & 1, err, &gave_up);
                tc_fence_after();
                const uint32_t v = base + FA_V + (j & 1) * FA_TILE;
#pragma unroll
                for (int kk = 0; kk < 8; kk++)
                    tc_mma(tmem + 256u, sw128_desc(base + FA_P + (kk / 4) * FA_TILE + (kk % 4) * 32),
                           fa_desc_mn(v + kk * 2048), idesc_o, kk > 0 ? 1u : 0u);
                tc_commit(B(bo_full));
                tc_commit(B(bkv_empty[j & 1]));
            }
        }
    } else if (n > 0) {
        // Softmax: thread = query row m of the tile.
        const int q = warp & 3, m = q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const int pos = pos_s[m];
        const float scale2 = 1.4426950408889634f / sqrtf((float)p.head_dim);  // log2(e) / sqrt(hd)
        float o[64];
#pragma unroll
        for (int d = 0; d < 64; d++) o[d] = 0.0f;
        float mrow = -INFINITY, l = 0.0f, a_pend = 0.0f;
        auto fold_pv = [&](int j) {  // o = o a_pend + PV_j, PV_j from TMEM
            mbar_wait(B(bo_full), j & 1, err, &gave_up);
            tc_fence_after();
            uint32_t v[4][16];
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld16_nowait(tmem + lane_off + 256u + c * 16, v[c]);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 64; d++) o[d] = __fmaf_rn(o[d], a_pend, __uint_as_float(v[d / 16][d % 16]));
        };
        for (int j = 0; j < n; j++) {
            const int b = j & 1;
            mbar_wait(B(bs_full[b]), (j >> 1) & 1, err, &gave_up);
            tc_fence_after();
            uint32_t sv[8][16];
#pragma unroll
            for (int c = 0; c < 8; c++) tmem_ld16_nowait(tmem + lane_off + (uint32_t)(b * 128 + c * 16), sv[c]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(B(bs_empty[b]));
            // Scores in base 2, masked past the row's position; a spare row takes none.
            const int k0 = j * 128;
            // Eight running maxima and sums (column c to c % 8), joined in a fixed order, so the
            // chains are short.
            float mx8[8];
#pragma unroll
            for (int e = 0; e < 8; e++) mx8[e] = -INFINITY;
#pragma unroll
            for (int c = 0; c < 128; c++) {
                const bool ok = k0 + c <= pos;
                const float s = ok ? __uint_as_float(sv[c / 16][c % 16]) * scale2 : -INFINITY;
                sv[c / 16][c % 16] = __float_as_uint(s);
                mx8[c % 8] = fmaxf(mx8[c % 8], s);
            }
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            const float m_new = fmaxf(mrow, mx);
            const bool live = m_new != -INFINITY;  // false only for a spare row
            const float a = live ? fa_exp2(mrow - m_new) : 1.0f;
            float sum8[8];
#pragma unroll
            for (int e = 0; e < 8; e++) sum8[e] = 0.0f;
            uint32_t pk[64];
#pragma unroll
            for (int c = 0; c < 128; c += 2) {
                const float p0 = live ? fa_exp2(__uint_as_float(sv[c / 16][c % 16]) - m_new) : 0.0f;
                const float p1 = live ? fa_exp2(__uint_as_float(sv[(c + 1) / 16][(c + 1) % 16]) - m_new) : 0.0f;
                sum8[c % 8] += p0;
                sum8[(c + 1) % 8] += p1;
                const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
                pk[c / 2] = *reinterpret_cast<const uint32_t *>(&pp);
            }
            const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
            l = __fmaf_rn(l, a, sum);
            mrow = m_new;
            if (j > 0) {
                fold_pv(j - 1);  // PV_{j-1} is done: P's buffer is free and O holds PV_{j-1}
                tc_fence_before();
                mbar_arrive(B(bo_empty));
            }
            // P_j, row m: keys 0..63 in the first box, 64..127 in the second, swizzled.
#pragma unroll
            for (int ch = 0; ch < 16; ch++) {
                uint8_t *dst = smem + FA_P + (ch / 8) * FA_TILE + fa_sw128(m, ch % 8);
                *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(B(bp_full));
            a_pend = a;
        }
        fold_pv(n - 1);
        if (pos >= 0) {
            const float inv = 1.0f / l;
            uint4 *dst = reinterpret_cast<uint4 *>(out + ((size_t)(r0 + m) * heads + head) * 64);
#pragma unroll
            for (int c = 0; c < 8; c++) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const __nv_bfloat162 pp =
                        __floats2bfloat162_rn(o[8 * c + 2 * e] * inv, o[8 * c + 2 * e + 1] * inv);
                    w[e] = *reinterpret_cast<const uint32_t *>(&pp);
                }
                dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
}

bool attention_tc_supported(const tg_params &p) {
    return p.dtype == TG_BF16 && p.head_dim == 64 && p.rows % 128 == 0 && p.rows > 0;
}

cudaError_t launch_attention_rows_tc(const tg_params &p, const uint32_t *at, const void *q, const void *kc,
                                     const void *vc, void *out, uint32_t *err, cudaStream_t s) {
    if (!attention_tc_supported(p)) return cudaErrorInvalidValue;
    CUtensorMap qm, km, vm;
    const uint64_t cache_rows = (uint64_t)p.slots * p.kv_heads * p.capacity;
    if (!make_map_bf16(&qm, q, p.rows, (uint64_t)p.heads * 64, 128) || !make_map_bf16(&km, kc, cache_rows, 64, 128) ||
        !make_map_bf16(&vm, vc, cache_rows, 64, 128))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(attention_rows_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FA_SMEM);
    if (e != cudaSuccess) return e;
    attention_rows_tc_kernel<<<dim3(p.rows / 128, p.heads), FA_THREADS, FA_SMEM, s>>>(qm, km, vm, p, at, (bf16 *)out, err);
    return cudaGetLastError();
}

}  // namespace tg
