// The prefill's causal attention (attention_rows.comp:46-126) on tcgen05, for bf16 and a head
// dimension of 64: flash attention with both products on the tensor cores and their accumulators
// in TMEM.
//
// Block (t, g) takes query rows [128 t, 128 t + 128) of the launch (one run's rows: runs start on
// multiples of 128) for query heads 2g and 2g + 1 (one KV head's), and walks its slot's cache from
// position 0 to the tile's last position in tiles of 128 keys, shared by the two heads. Ten warps:
//   warp 0     TMA: the two Q tiles once, then K and V tiles into FA_STAGES stages (128-byte
//              swizzle, no multicast);
//   warp 1     TMEM (per head: S, 128 columns; P, 64; O, 64: all 512) and the MMAs:
//              S_j = Q K_j^T (M = 128, N = 128, K = 64; Q and K in shared memory) and
//              O += P_j V_j (M = 128, N = 64, K = 128; P in TMEM, V in shared memory read
//              MN-major). Once a head's P_j is in, its S_{j+1} is issued ahead of its PV_j, so
//              that the head's next softmax starts after the four MMAs of S (an M = 128, K = 16
//              MMA of N up to 128 takes ~95 clocks here, measured), with PV_j under it; PV_j
//              waits for no later tile's copies;
//   warps 2-5  head 2g, warps 6-9 head 2g + 1: a thread to a query row: S_j from TMEM (the mask,
//              the base-2 exponentials with the scale folded in, the tile's maximum alongside)
//              and P_j as bf16 into TMEM, once PV_{j-1} has read P_{j-1}, against a reference
//              maximum that moves only when a tile's passes it by more than 2^FA_RESCALE - O in
//              TMEM then rescaled in place (as in FlashAttention-4) and the tile's pass run again
//              from S_j; O / l at the end.
// With P in shared memory PV read 192 bytes a tensor clock (P and V) against the SM's 128, and
// the softmax's P stores met those reads there.
// The two heads' softmax warps run while the other head's MMAs do. Every wait on an mbarrier is
// bounded (the context's error word, then the block runs out).
#include "tc_common.cuh"

namespace tg {

namespace {

constexpr int FA_THREADS = 320;
constexpr uint32_t FA_TILE = 128 * 64 * 2;  // a 128-row x 64-column bf16 box
constexpr int FA_STAGES = 4;                  // K and V tiles in flight
// Shared memory: Q of the two heads, K and V stages.
constexpr uint32_t FA_Q = 0, FA_K = 2 * FA_TILE, FA_V = FA_K + FA_STAGES * FA_TILE;
constexpr uint32_t FA_SMEM = FA_V + FA_STAGES * FA_TILE + 1024;
// How far (base 2) a tile's maximum may pass a row's reference before O and l are rescaled.
constexpr float FA_RESCALE = 8.0f;

// 2^x by the hardware's approximate base-2 exponential (PTX ex2.approx.ftz.f32: relative error
// about 2^-22, far below the bf16 rounding the probabilities take next); 2^-inf = 0.
TG_DEVICE float fa_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Two-wide f32 arithmetic (sm_100's fma/add .f32x2: each lane the scalar IEEE operation, so the
// same bits as two scalar instructions, in one issue) and the three-input maximum.
TG_DEVICE float2 fa_fma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<const uint64_t *>(&a)), "l"(*reinterpret_cast<const uint64_t *>(&b)),
          "l"(*reinterpret_cast<const uint64_t *>(&c)));
    return *reinterpret_cast<const float2 *>(&d);
}
TG_DEVICE float2 fa_add2(float2 a, float2 b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<const uint64_t *>(&a)), "l"(*reinterpret_cast<const uint64_t *>(&b)));
    return *reinterpret_cast<const float2 *>(&d);
}
TG_DEVICE float fa_max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// The same bytes as a K-major SW128 tile read MN-major: V's tile [keys][64] is B = V^T with N = 64
// along a row and K = keys down the rows, in atoms of 8 keys x 128 bytes, 1024 bytes apart along K.
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
    __shared__ __align__(8) uint64_t bq, bkv_full[FA_STAGES], bkv_empty[FA_STAGES];
    __shared__ __align__(8) uint64_t bs_full[2], bp_full[2], bo_full[2];  // by head
    __shared__ __align__(8) uint64_t bv_clear;  // V_{n-1}'s rows past the tile's last position are zero
    __shared__ uint32_t tmem_slot, t_last, t_slot, t_slot_max;
    __shared__ int gave_up;
    __shared__ int pos_s[128];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int tile = gridDim.x - 1 - blockIdx.x;  // the latest rows, the longest walks, first
    const int head0 = 2 * blockIdx.y, heads = p.heads, kvh = p.kv_heads, kv = head0 / (heads / kvh);
    const int r0 = tile * 128;
    auto B = [](uint64_t &b) { return smem_u32(&b); };

    if (tid == 0) {
        gave_up = 0;
        t_last = 0;
        t_slot = 0xffffffffu;
        t_slot_max = 0;
        mbar_init(B(bq), 1);
        for (int i = 0; i < FA_STAGES; i++) {
            mbar_init(B(bkv_full[i]), 1);
            mbar_init(B(bkv_empty[i]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(B(bs_full[i]), 1);
            mbar_init(B(bp_full[i]), 128);  // P_j in TMEM, S_j read and O rescaled
            mbar_init(B(bo_full[i]), 1);
        }
        mbar_init(B(bv_clear), 1);
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
    // Keys past the tile's last position are read as zero (attention_rows.comp:77-83): their
    // probabilities are 0, but a value there that is not finite (another request's, left in the
    // slot, or the next cache range's) would still make 0 x v NaN in PV. When the last key tile
    // reaches past it, warp 0 clears those rows of V_{n-1} before PV_{n-1} is issued.
    const bool clear_v = n > 0 && t_last % 128 != 127;
    // TMEM columns: head h's S at 256 h, P (bf16 pairs) at 256 h + 128, O at 256 h + 192.
    auto s_col = [](int h) { return (uint32_t)(256 * h); };
    auto p_col = [](int h) { return (uint32_t)(256 * h + 128); };
    auto o_col = [](int h) { return (uint32_t)(256 * h + 192); };

    if (warp == 0) {
        if (lane == 0 && n > 0) {
            mbar_arrive_expect_tx(B(bq), 2 * FA_TILE);
            tma_load_2d(base + FA_Q, &qmap, head0 * 64, r0, B(bq));
            tma_load_2d(base + FA_Q + FA_TILE, &qmap, (head0 + 1) * 64, r0, B(bq));
            const int row0 = (int)((t_slot * (uint32_t)kvh + kv) * p.capacity);
            for (int j = 0; j < n; j++) {
                const int b = j % FA_STAGES;
                mbar_wait(B(bkv_empty[b]), ((j / FA_STAGES) & 1) ^ 1, err, &gave_up);
                mbar_arrive_expect_tx(B(bkv_full[b]), 2 * FA_TILE);
                tma_load_2d(base + FA_K + b * FA_TILE, &kmap, 0, row0 + j * 128, B(bkv_full[b]));
                tma_load_2d(base + FA_V + b * FA_TILE, &vmap, 0, row0 + j * 128, B(bkv_full[b]));
            }
            // Every copy this thread started has landed before the block can end.
            for (int j = n > FA_STAGES ? n - FA_STAGES : 0; j < n; j++)
                mbar_wait(B(bkv_full[j % FA_STAGES]), (j / FA_STAGES) & 1, err, &gave_up);
        }
        if (clear_v) {
            __syncwarp();
            mbar_wait(B(bkv_full[(n - 1) % FA_STAGES]), ((n - 1) / FA_STAGES) & 1, err, &gave_up);
            uint8_t *vt = smem + FA_V + ((n - 1) % FA_STAGES) * FA_TILE;
            const int keep = (int)(t_last % 128) + 1;
            for (int i = lane; i < (128 - keep) * 8; i += 32) {
                const int r = keep + i / 8;  // a row of the swizzled tile is 128 whole bytes
                *reinterpret_cast<uint4 *>(vt + (r >> 3) * 1024 + (r & 7) * 128 + (i % 8) * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // for the tensor cores' reads
            __syncwarp();
            if (lane == 0) mbar_arrive(B(bv_clear));
        }
    } else if (warp == 1) {
        if (lane == 0 && n > 0) {
            constexpr uint32_t idesc_s = bf16_idesc(128, 128);
            constexpr uint32_t idesc_o = bf16_idesc(128, 64) | (1u << 16);  // B (V) MN-major
            // S_j of head h (Q and K_j in shared memory), issued once the head's S_{j-1} is read
            // and K_j has landed.
            auto issue_s = [&](int j, int h) {
                const uint32_t kt = base + FA_K + (j % FA_STAGES) * FA_TILE;
#pragma unroll
                for (int k = 0; k < 4; k++)
                    tc_mma(tmem + s_col(h), sw128_desc(base + FA_Q + h * FA_TILE + k * 32), sw128_desc(kt + k * 32),
                           idesc_s, k > 0 ? 1u : 0u);
                tc_commit(B(bs_full[h]));
            };
            mbar_wait(B(bq), 0, err, &gave_up);
            mbar_wait(B(bkv_full[0]), 0, err, &gave_up);
            tc_fence_after();
            issue_s(0, 0);
            issue_s(0, 1);
            for (int j = 0; j < n; j++) {
                const int b = j % FA_STAGES;
                const uint32_t v = base + FA_V + b * FA_TILE;
                if (clear_v && j == n - 1) mbar_wait(B(bv_clear), 0, err, &gave_up);
                for (int h = 0; h < 2; h++) {
                    // P_j in TMEM, S_j read, and O rescaled to the row's reference.
                    mbar_wait(B(bp_full[h]), j & 1, err, &gave_up);
                    if (j + 1 < n && h == 0)
                        mbar_wait(B(bkv_full[(j + 1) % FA_STAGES]), ((j + 1) / FA_STAGES) & 1, err, &gave_up);
                    tc_fence_after();
                    if (j + 1 < n) issue_s(j + 1, h);
#pragma unroll
                    for (int kk = 0; kk < 8; kk++)
                        tc_mma_ts(tmem + o_col(h), tmem + p_col(h) + 8 * kk, fa_desc_mn(v + kk * 2048), idesc_o,
                                  (j > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(B(bo_full[h]));
                    if (h == 1) tc_commit(B(bkv_empty[b]));  // K_j and V_j are read by every MMA issued so far
                }
            }
        }
    } else if (n > 0) {
        // Softmax: head h = head0 + (warps 6-9), thread = query row m of the tile.
        const int h = warp >= 6 ? 1 : 0;
        const int q = warp & 3, m = q * 32 + lane;
        const uint32_t lanes = tmem + ((uint32_t)(q * 32) << 16);
        const int pos = pos_s[m];
        const float scale2 = 1.4426950408889634f / sqrtf((float)p.head_dim);  // log2(e) / sqrt(hd)
        // P_j = 2^(S_j scale2 - mref) against the row's reference maximum mref (base 2, scaled), and
        // the running sum l against the same; O accumulates P_j V_j in TMEM over the tiles. mref
        // moves up to a tile's maximum only when that passes it by more than FA_RESCALE (so P stays
        // below 2^FA_RESCALE), and then O (in TMEM, once PV_{j-1} is in it) and l are rescaled to
        // it; the output is O / l after the last tile.
        float mref = -INFINITY, l = 0.0f;
        // Half c2 (64 keys) of S_j as the raw scores, masked past the row's position (-inf) only in
        // a half that reaches past it: the scale to base 2 is folded into the exponential's FMA, so
        // that a score costs a max, an FMA, an exponential and an add.
        auto load_half = [&](int j, int c2, float (&sv)[64]) {
            uint32_t r[4][16];
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld16_nowait(lanes + s_col(h) + (uint32_t)(c2 * 64 + c * 16), r[c]);
            tmem_wait_ld();
            const int k0 = j * 128 + c2 * 64;
            if (k0 + 63 <= pos) {
#pragma unroll
                for (int c = 0; c < 64; c++) sv[c] = __uint_as_float(r[c / 16][c % 16]);
            } else {
#pragma unroll
                for (int c = 0; c < 64; c++) sv[c] = k0 + c <= pos ? __uint_as_float(r[c / 16][c % 16]) : -INFINITY;
            }
        };
        for (int j = 0; j < n; j++) {
            mbar_wait(B(bs_full[h]), j & 1, err, &gave_up);
            tc_fence_after();
            // P_j against mref, the tile's maximum taken in the same pass and checked after it:
            // where it passes mref by more than FA_RESCALE (always on the first tile, where mref
            // is -inf and P_0 comes out 0) the reference moves, O is rescaled (PV_{j-1} is in it),
            // and the warp's pass runs again from S_j, still in TMEM - the same P and l as taking
            // the maximum first, without a pass over S_j on the critical path of later tiles.
            // One pass: P_j of the warp's rows against mref into TMEM, their sum; the tile's raw
            // maximum into mx. P_j replaces P_{j-1} once PV_{j-1} has read it (and is in O): the
            // first pass waits for that just before its first store, after half 0's exponentials.
            auto p_pass = [&](float &mx, bool first) {
                float2 sum4[4];  // the running sums of columns c % 8 = 2 e and 2 e + 1
#pragma unroll
                for (int e = 0; e < 4; e++) sum4[e] = make_float2(0.0f, 0.0f);
                float mxs[2] = {-INFINITY, -INFINITY};
                // A spare row (mref -inf, every score masked to -inf) takes -inf for -mref, so that
                // its exponentials are 2^-inf = 0 with no select in the loop.
                const float nm = mref != -INFINITY ? -mref : -INFINITY;
                const float2 scale22 = make_float2(scale2, scale2), neg_m = make_float2(nm, nm);
#pragma unroll
                for (int c2 = 0; c2 < 2; c2++) {
                    float sv[64];
                    load_half(j, c2, sv);
                    uint32_t pk[2][16];
#pragma unroll
                    for (int c = 0; c < 64; c += 2) {
                        mxs[(c / 2) % 2] = fa_max3(mxs[(c / 2) % 2], sv[c], sv[c + 1]);
                        const float2 x = fa_fma2(make_float2(sv[c], sv[c + 1]), scale22, neg_m);
                        const float p0 = fa_exp2(x.x), p1 = fa_exp2(x.y);
                        sum4[(c % 8) / 2] = fa_add2(sum4[(c % 8) / 2], make_float2(p0, p1));
                        const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
                        pk[c / 32][(c / 2) % 16] = *reinterpret_cast<const uint32_t *>(&pp);
                    }
                    if (c2 == 0 && first && j > 0) {
                        mbar_wait(B(bo_full[h]), (j - 1) & 1, err, &gave_up);
                        tc_fence_after();
                    }
                    // Keys 64 c2 .. 64 c2 + 63 of row m: P's columns 32 c2 .. 32 c2 + 31, bf16 pairs.
                    tmem_st16(lanes + p_col(h) + 32 * c2, pk[0]);
                    tmem_st16(lanes + p_col(h) + 32 * c2 + 16, pk[1]);
                }
                mx = fmaxf(mxs[0], mxs[1]);
                return ((sum4[0].x + sum4[0].y) + (sum4[1].x + sum4[1].y)) +
                       ((sum4[2].x + sum4[2].y) + (sum4[3].x + sum4[3].y));
            };
            float a = 1.0f, mx;
            float sum = p_pass(mx, true);
            const float m_tile = mx * scale2;  // the scale is positive: max, then scale
            const bool move = m_tile != -INFINITY && (mref == -INFINITY || m_tile > mref + FA_RESCALE);
            if (__any_sync(0xffffffffu, move)) {
                // A row of the warp moves: rescale O where the reference moved (a row that keeps
                // its reference times 1), then the warp's P_j again.
                a = move && mref != -INFINITY ? fa_exp2(mref - m_tile) : 1.0f;
                if (move) mref = m_tile;
                tmem_wait_st();
                if (__any_sync(0xffffffffu, a != 1.0f)) {
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        uint32_t v[16];
                        tmem_ld16_nowait(lanes + o_col(h) + c * 16, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; e++) v[e] = __float_as_uint(__uint_as_float(v[e]) * a);
                        tmem_st16(lanes + o_col(h) + c * 16, v);
                    }
                    tmem_wait_st();
                }
                sum = p_pass(mx, false);
            }
            tmem_wait_st();
            tc_fence_before();
            l = __fmaf_rn(l, a, sum);
            mbar_arrive(B(bp_full[h]));
        }
        // The output: O / l, once PV_{n-1} is in O.
        mbar_wait(B(bo_full[h]), (n - 1) & 1, err, &gave_up);
        tc_fence_after();
        uint32_t v[4][16];
#pragma unroll
        for (int c = 0; c < 4; c++) tmem_ld16_nowait(lanes + o_col(h) + c * 16, v[c]);
        tmem_wait_ld();
        if (pos >= 0) {
            const float inv = 1.0f / l;
            uint4 *dst = reinterpret_cast<uint4 *>(out + ((size_t)(r0 + m) * heads + head0 + h) * 64);
#pragma unroll
            for (int c = 0; c < 8; c++) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int d = 8 * c + 2 * e;
                    const __nv_bfloat162 pp = __floats2bfloat162_rn(__uint_as_float(v[d / 16][d % 16]) * inv,
                                                                    __uint_as_float(v[d / 16][d % 16 + 1]) * inv);
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
    return p.dtype == TG_BF16 && p.head_dim == 64 && p.rows % 128 == 0 && p.rows > 0 && p.kv_heads > 0 &&
           p.heads % p.kv_heads == 0 && (p.heads / p.kv_heads) % 2 == 0;
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
    attention_rows_tc_kernel<<<dim3(p.rows / 128, p.heads / 2), FA_THREADS, FA_SMEM, s>>>(qm, km, vm, p, at, (bf16 *)out, err);
    return cudaGetLastError();
}

}  // namespace tg
