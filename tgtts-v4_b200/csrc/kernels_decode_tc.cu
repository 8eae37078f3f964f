// The decode projections of a batched decoder on tcgen05 (the GEMVs gemv_qkv_rope.comp,
// gemv_gate_up.comp and gemv_residual.comp at larger batch): out = W x for the batch's rows, W a
// checkpoint's [out rows][k] bf16 matrix, x the rows' f32 activations.
//
// Each 128 rows of W (a tile; for gate/up a gate tile and its up tile) is one thread-block
// cluster of S blocks, block r taking columns [r Kc, (r + 1) Kc) of K (split-K):
//   1. its slice of W goes to shared memory by TMA (128-byte swizzle, no multicast) at once,
//      before the block waits on the kernel before (the weights do not depend on it);
//   2. where the projection norms its input (RMSNorm before q/k/v and gate/up), each block sums
//      the squares of its slice of every row and the cluster joins the S partial sums, in rank
//      order, through distributed shared memory;
//   3. each row's f32 activations over the slice (normed and scaled by the gain where asked) are
//      split into bf16 hi = bf16(v) and lo = bf16(v - hi) and written, swizzled, as two rows of the
//      MMA's B operand (2b and 2b + 1 for batch row b), so that W (hi + lo) carries 16 bits of each
//      value into the f32 accumulator;
//   4. one thread issues tcgen05.mma (M = 128, N = 2 rows, K = 16) into TMEM, in groups of rows
//      when B would not fit beside W;
//   5. the blocks stage their accumulators in shared memory, and after a cluster barrier block r
//      reduces its share of the tile's rows over the S partials, in rank order (hi and lo apart,
//      then their sum), and runs the epilogue: RoPE and the cache append for q/k/v, SiLU(gate) up,
//      or the scaled residual add.
// Every order of summation is fixed by the shape and the split alone, not by the batch, so a row's
// result is the same bits in every bucket of a decoder (crates/graph/src/decode.rs:8-11).
#include <cooperative_groups.h>

#include <algorithm>

#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace tg {

namespace {

constexpr int DTC_THREADS = 256;
constexpr int DTC_MAX_KB = 8;                    // k-blocks of 64 a block's slice may hold
constexpr uint32_t DTC_A_TILE = 128 * 64 * 2;    // one TMA box: 128 rows x 64 bf16
constexpr uint32_t DTC_SMEM_CAP = 200 * 1024;    // dynamic shared memory a block plans with
constexpr uint32_t DTC_SMEM_MIN = 120 * 1024;    // one block to an SM, so TMEM never runs short
constexpr int DTC_MAX_ROWS = 128;                // batch rows
constexpr int DTC_MAX_S = 8;                     // blocks in a cluster (the portable maximum)

struct DtcArgs {
    tg_params p;          // rows: the bucket's rows
    const float *x;       // [rows][K] f32
    const float *g;       // the RMSNorm gain over K, or null for an input taken as it is
    int K, Kc, S;         // input width, one block's slice of it, blocks in a cluster
    int G, Npg, groups;   // batch rows per MMA group, the MMA's N per group, groups
    uint32_t tmem_cols;   // a power of two >= 32
    int cc;               // accumulator columns staged per reduction pass (a multiple of 16)
    uint32_t a_bytes;     // W's slice: k-blocks x tiles x 16 KiB
    const float *res;     // residual: out[b][n] = res[b][n] + s y
    float *out;           // residual [rows][n]; gate/up [rows][inner]
    const float *cosv, *sinv;
    const uint32_t *at;
    float *q;
    void *kc, *vc;
    uint32_t *err;
};

TG_DEVICE uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// hi = bf16(v), lo = bf16(v - hi) for 8 values, packed as two 16-byte rows.
TG_DEVICE void split8(const float (&v)[8], uint4 &hi, uint4 &lo) {
    float h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        h[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
        l[i] = __fsub_rn(v[i], h[i]);
    }
    hi = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]), pack_bf16x2(h[6], h[7]));
    lo = make_uint4(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]), pack_bf16x2(l[4], l[5]), pack_bf16x2(l[6], l[7]));
}

// Byte offset of 16-byte chunk `c` (of 8) of row n in a K-major tile of 64 columns with 128-byte
// rows in the 128-byte swizzle (the layout TMA writes): 8-row groups of 1024 bytes, chunk index
// XOR the row within its group.
TG_DEVICE uint32_t sw128_offset(int n, int c) {
    return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4));
}

template <int EPI>
struct DtcTraits;
template <>
struct DtcTraits<0> {  // q/k/v with RoPE: a tile, units are RoPE pairs
    static constexpr int NT = 1, UNITS = 64;
};
template <>
struct DtcTraits<1> {  // gate/up: a gate tile and its up tile, units are output columns
    static constexpr int NT = 2, UNITS = 128;
};
template <>
struct DtcTraits<2> {  // residual: a tile, units are rows
    static constexpr int NT = 1, UNITS = 128;
};

}  // namespace

enum { DTC_QKV = 0, DTC_GATE_UP = 1, DTC_RESIDUAL = 2 };

template <int EPI>
__global__ void __launch_bounds__(DTC_THREADS, 1)
    dtc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ DtcArgs a) {
    constexpr int NT = DtcTraits<EPI>::NT, UNITS = DtcTraits<EPI>::UNITS;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_u32(smem);
    const uint32_t b_base = base + a.a_bytes;
    __shared__ __align__(8) uint64_t bar_a[DTC_MAX_KB];
    __shared__ __align__(8) uint64_t bar_mma;
    __shared__ uint32_t tmem_slot;
    __shared__ int gave_up;
    __shared__ float sq[DTC_MAX_ROWS];     // this block's partial sums of squares, by row
    __shared__ float scale[DTC_MAX_ROWS];  // the rows' RMSNorm scales
    __shared__ __align__(16) float gs[DTC_MAX_KB * 64];
    __shared__ uint32_t at_s[2 * DTC_MAX_ROWS];  // the placement words (written before the step)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int r = (int)cluster.block_rank(), S = a.S;
    const int tile = blockIdx.y;
    const int Kc = a.Kc, k0 = r * Kc, nkb = Kc / 64;
    const int R = (int)a.p.rows;
    const int Ntot = a.groups * a.Npg;  // accumulator columns of one tile

    if (tid == 0) {
        gave_up = 0;
        for (int kb = 0; kb < nkb; kb++) mbar_init(smem_u32(&bar_a[kb]), 1);
        mbar_init(smem_u32(&bar_mma), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    // 1. W's slice, all of it, before the wait on the kernel before.
    if (tid == 0) {
        for (int kb = 0; kb < nkb; kb++) {
            mbar_arrive_expect_tx(smem_u32(&bar_a[kb]), NT * DTC_A_TILE);
            for (int t = 0; t < NT; t++)
                tma_load_2d(base + (kb * NT + t) * DTC_A_TILE, &wmap, k0 + kb * 64, (tile * NT + t) * 128,
                            smem_u32(&bar_a[kb]));
        }
    }
    const bool norm = a.g != nullptr;
    if (norm)
        for (int i = tid; i < Kc / 4; i += DTC_THREADS)
            reinterpret_cast<float4 *>(gs)[i] = reinterpret_cast<const float4 *>(a.g + k0)[i];
    if constexpr (EPI == DTC_QKV)
        for (int i = tid; i < (a.p.slots > 1 ? 2 : 1) * R; i += DTC_THREADS) at_s[i] = a.at[i];
    pdl_launch_dependents();
    pdl_wait();
    __syncthreads();  // the gain and the placement are in shared memory for every warp

    // 2-4. B for each group of rows (four items' loads in flight per thread), then its MMAs. Where
    // the projection norms its input, B holds x g (the gain applied, the RMSNorm scale not yet):
    // the scale is a factor of each row's result, applied in the epilogue, so B needs nothing
    // from the other blocks. The same pass sums each row's squares over this slice: an item's
    // eight in order, then the xor butterfly over the `chunks` consecutive lanes holding the row.
    const uint32_t idesc = bf16_idesc(128, a.Npg);
    const uint32_t b_kb_bytes = (uint32_t)a.Npg * 128;  // one k-block of B
    const int chunks = Kc / 8;
    for (int gi = 0; gi < a.groups; gi++) {
        const int b0 = gi * a.G, nb = min(a.G, R - b0);
        if (gi > 0) mbar_wait(smem_u32(&bar_mma), (gi - 1) & 1, a.err, &gave_up);  // B is free again
        const int items = (a.Npg / 2) * chunks;
        for (int i0 = 0; i0 < items; i0 += 4 * DTC_THREADS) {
            float4 u[4][2];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int item = i0 + j * DTC_THREADS + tid, bl = item / chunks, ch = item % chunks;
                if (item < items && bl < nb) {
                    const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)(b0 + bl) * a.K + k0 + ch * 8);
                    u[j][0] = __ldcg(xr);
                    u[j][1] = __ldcg(xr + 1);
                } else {
                    u[j][0] = u[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int item = i0 + j * DTC_THREADS + tid, bl = item / chunks, ch = item % chunks;
                float v[8] = {u[j][0].x, u[j][0].y, u[j][0].z, u[j][0].w, u[j][1].x, u[j][1].y, u[j][1].z, u[j][1].w};
                if (norm) {
                    float q2 = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; i++) q2 = __fmaf_rn(v[i], v[i], q2);
                    for (int o = chunks / 2; o > 0; o >>= 1) q2 += __shfl_xor_sync(0xffffffffu, q2, o);
                    if (item < items && bl < nb && ch == 0) sq[b0 + bl] = q2;
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = __fmul_rn(v[i], gs[ch * 8 + i]);
                }
                if (item >= items) continue;
                uint4 hi, lo;
                split8(v, hi, lo);
                uint8_t *tile_b = smem + a.a_bytes + (size_t)(ch / 8) * b_kb_bytes;
                *reinterpret_cast<uint4 *>(tile_b + sw128_offset(2 * bl, ch % 8)) = hi;
                *reinterpret_cast<uint4 *>(tile_b + sw128_offset(2 * bl + 1, ch % 8)) = lo;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (warp == 1 && lane == 0) {
            tc_fence_after();
            for (int kb = 0; kb < nkb; kb++) {
                if (gi == 0) mbar_wait(smem_u32(&bar_a[kb]), 0, a.err, &gave_up);
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const uint64_t bd = sw128_desc(b_base + kb * b_kb_bytes + k * 32);
#pragma unroll
                    for (int t = 0; t < NT; t++)
                        tc_mma(tmem + (uint32_t)(t * Ntot + gi * a.Npg),
                               sw128_desc(base + (kb * NT + t) * DTC_A_TILE + k * 32), bd, idesc,
                               (kb > 0 || k > 0) ? 1u : 0u);
                }
            }
            tc_commit(smem_u32(&bar_mma));
        }
        __syncwarp();
    }
    mbar_wait(smem_u32(&bar_mma), (a.groups - 1) & 1, a.err, &gave_up);
    tc_fence_after();

    // 5. Passes of `cc` accumulator columns. Block r owns units [r per, (r + 1) per) of the tile
    // (rows for the residual, gate/up columns, RoPE pairs for q/k/v): every block adds each hi/lo
    // pair of the accumulator rows it holds and pushes the sums into the owner's receive buffer,
    // [from block][owned row][batch row], with stores into distributed shared memory; after a
    // cluster barrier each block sums its rows over the S partials in rank order from its own
    // shared memory and runs the epilogue, whose global inputs it loaded before the barrier. The
    // receive buffer reuses W's and B's space, so a barrier first makes sure every block's MMAs are
    // done with them. The RMSNorm scales join the S blocks' sums of squares in rank order.
    const int per = UNITS / S;                   // units a block owns
    const int own = NT * 128 / S;                // accumulator rows a block owns
    const int stride = a.cc / 2 + 4;             // floats per received row (padded against conflicts)
    float *recv = reinterpret_cast<float *>(smem);
    const int q = warp & 3, half_w = warp >> 2;  // TMEM lane quarter, and which half of the columns
    const int m = q * 32 + lane;                 // the accumulator row this thread holds
    int o_blk[NT], o_row[NT];                    // where row m of tile t goes: owner block, row there
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if constexpr (EPI == DTC_QKV) {
            const int hd = a.p.head_dim, hf = hd / 2;
            const int pair = (m / hd) * hf + (m % hf);
            o_blk[t] = pair / per;
            o_row[t] = (pair % per) * 2 + ((m % hd) >= hf ? 1 : 0);
        } else {
            o_blk[t] = m / per;
            o_row[t] = t * per + m % per;
        }
    }
    const uint32_t lanes = tmem + ((uint32_t)(q * 32) << 16);
    constexpr int PF = 8;  // epilogue items a thread takes per pass (the plan keeps it so)
    for (int c0 = 0; c0 < Ntot; c0 += a.cc) {
        const int cw = min(a.cc, Ntot - c0);
        const int nbr = cw / 2;  // batch rows of this pass
        cluster.sync();  // every block's MMAs (first pass) or reduction (later passes) is done
        if (norm && c0 == 0) {
            for (int b = tid; b < R; b += DTC_THREADS) {
                float part[DTC_MAX_S];
#pragma unroll
                for (int s = 0; s < DTC_MAX_S; s++) part[s] = s < S ? cluster.map_shared_rank(sq, s)[b] : 0.0f;
                float t = 0.0f;
#pragma unroll
                for (int s = 0; s < DTC_MAX_S; s++)
                    if (s < S) t = __fadd_rn(t, part[s]);
                scale[b] = 1.0f / sqrtf(__fdiv_rn(t, (float)a.K) + a.p.eps);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            float *dst = cluster.map_shared_rank(recv, o_blk[t]) + ((size_t)r * own + o_row[t]) * stride;
            for (int cc = half_w * 16; cc < cw; cc += 4 * 32) {
                // Up to four loads of 16 columns in flight, one wait.
                uint32_t v[4][16];
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (cc + 32 * i < cw) tmem_ld16_nowait(lanes + (uint32_t)(t * Ntot + c0 + cc + 32 * i), v[i]);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (cc + 32 * i >= cw) break;
                    float w[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) w[e] = __fadd_rn(__uint_as_float(v[i][2 * e]), __uint_as_float(v[i][2 * e + 1]));
                    float4 *d4 = reinterpret_cast<float4 *>(dst + (cc + 32 * i) / 2);
                    d4[0] = make_float4(w[0], w[1], w[2], w[3]);
                    d4[1] = make_float4(w[4], w[5], w[6], w[7]);
                }
            }
        }
        // This thread's epilogue items of the pass: their global inputs, before the barrier.
        const int items = per * nbr;
        float pre_a[PF], pre_b[PF];
#pragma unroll
        for (int k = 0; k < PF; k++) {
            pre_a[k] = pre_b[k] = 0.0f;
            const int idx = tid + k * DTC_THREADS;
            if (idx >= items) continue;
            const int ul = idx % per, c = c0 + 2 * (idx / per);
            const int gi = c / a.Npg, bl = (c % a.Npg) / 2, b = gi * a.G + bl;
            if (bl >= a.G || b >= R) continue;
            const int unit = r * per + ul;
            if constexpr (EPI == DTC_RESIDUAL) {
                pre_a[k] = __ldcg(a.res + (size_t)b * a.p.n + tile * 128 + unit);
            } else if constexpr (EPI == DTC_QKV) {
                const int hf = a.p.head_dim / 2, i = unit % hf;
                const uint32_t pos = at_s[b];
                if (a.p.rope && pos < a.p.capacity) {
                    pre_a[k] = __ldg(a.cosv + (size_t)pos * hf + i);
                    pre_b[k] = __ldg(a.sinv + (size_t)pos * hf + i);
                }
            }
        }
        cluster.sync();  // every push has landed (and the scales are in)
        auto reduce = [&](int row, int j) {
            float part[DTC_MAX_S];
#pragma unroll
            for (int s = 0; s < DTC_MAX_S; s++) part[s] = s < S ? recv[((size_t)s * own + row) * stride + j] : 0.0f;
            float y = 0.0f;
#pragma unroll
            for (int s = 0; s < DTC_MAX_S; s++)
                if (s < S) y = __fadd_rn(y, part[s]);
            return y;
        };
#pragma unroll
        for (int k = 0; k < PF; k++) {
            const int idx = tid + k * DTC_THREADS;
            if (idx >= items) break;
            const int ul = idx % per, j = idx / per, c = c0 + 2 * j;
            const int gi = c / a.Npg, bl = (c % a.Npg) / 2, b = gi * a.G + bl;
            if (bl >= a.G || b >= R) continue;
            const int unit = r * per + ul;
            if constexpr (EPI == DTC_RESIDUAL) {
                a.out[(size_t)b * a.p.n + tile * 128 + unit] = __fmaf_rn(a.p.residual_scale, reduce(ul, j), pre_a[k]);
            } else if constexpr (EPI == DTC_GATE_UP) {
                const float sc = scale[b];
                const float yg = __fmul_rn(reduce(ul, j), sc), yu = __fmul_rn(reduce(per + ul, j), sc);
                a.out[(size_t)b * a.p.inner + tile * 128 + unit] = silu_mul(yg, yu);
            } else {
                const int hd = a.p.head_dim, hf = hd / 2;
                const float sc = scale[b];
                float ra = __fmul_rn(reduce(2 * ul, j), sc), rc = __fmul_rn(reduce(2 * ul + 1, j), sc);
                const int head = tile * (128 / hd) + unit / hf, i = unit % hf;
                const uint32_t pos = at_s[b], slot = a.p.slots > 1 ? at_s[R + b] : 0u;
                if (pos >= a.p.capacity || slot >= a.p.slots) continue;  // a spare row stores nothing
                const int heads = a.p.heads, kvh = a.p.kv_heads;
                bf16 *kc = static_cast<bf16 *>(a.kc);
                bf16 *vc = static_cast<bf16 *>(a.vc);
                if (head >= heads + kvh) {
                    const size_t to = (((size_t)slot * kvh + (head - heads - kvh)) * a.p.capacity + pos) * hd + i;
                    vc[to] = from_f32<bf16>(ra);
                    vc[to + hf] = from_f32<bf16>(rc);
                    continue;
                }
                if (a.p.rope) {
                    // x cos + rotate_half(x) sin, as qkv_store (gemv_qkv_rope.comp:85-90).
                    const float co = pre_a[k], si = pre_b[k];
                    const float na = __fmaf_rn(ra, co, -__fmul_rn(rc, si));
                    const float nc = __fmaf_rn(rc, co, __fmul_rn(ra, si));
                    ra = na;
                    rc = nc;
                }
                if (head < heads) {
                    const size_t to = ((size_t)b * heads + head) * hd + i;
                    a.q[to] = ra;
                    a.q[to + hf] = rc;
                } else {
                    const size_t to = (((size_t)slot * kvh + (head - heads)) * a.p.capacity + pos) * hd + i;
                    kc[to] = from_f32<bf16>(ra);
                    kc[to + hf] = from_f32<bf16>(rc);
                }
            }
        }
    }
    cluster.sync();  // no block leaves while a peer may still push into it
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
}

// ---- host -------------------------------------------------------------------------------------

namespace {

struct DtcPlan {
    int S, Kc, G, Npg, groups, cc;
    uint32_t tmem_cols, a_bytes, smem;
};

// The split and the groups for a projection of K columns into NT tiles per cluster for `rows`
// batch rows; false when its slice of W would not fit (the decoder then keeps the GEMVs).
bool plan(int K, int NT, int S, int rows, bool norm, DtcPlan &pl) {
    if (rows < 1 || rows > DTC_MAX_ROWS || S > DTC_MAX_S || K % (128 * S)) return false;
    // A normed row's slice is 16 or 32 items of 8 columns: a half or a whole warp (the squares'
    // butterfly).
    if (norm && K / S > 256) return false;
    pl.S = S;
    pl.Kc = K / S;
    const int nkb = pl.Kc / 64;
    if (nkb < 1 || nkb > DTC_MAX_KB) return false;
    pl.a_bytes = (uint32_t)(nkb * NT) * DTC_A_TILE;
    if (pl.a_bytes + 16 * pl.Kc * 2 > DTC_SMEM_CAP) return false;
    // Rows per group: the largest power of two whose B fits beside W.
    int G = 128;
    while (G > 8 && pl.a_bytes + (uint32_t)(2 * G) * pl.Kc * 2 > DTC_SMEM_CAP) G /= 2;
    pl.G = G;
    const int gr = rows < G ? rows : G;
    pl.Npg = ((2 * gr + 15) / 16) * 16;
    pl.groups = (rows + G - 1) / G;
    const int ntot = pl.groups * pl.Npg;
    if (NT * ntot > 512) return false;
    uint32_t cols = 32;
    while (cols < (uint32_t)(NT * ntot)) cols *= 2;
    pl.tmem_cols = cols;
    const uint32_t b_bytes = (uint32_t)pl.Npg * pl.Kc * 2;
    uint32_t smem = pl.a_bytes + b_bytes;
    // Receive buffer: NT x 128 rows x (cc / 2 + 4) f32, as wide as the cap allows, up to every
    // column, and narrow enough that a thread takes at most 8 epilogue items a pass.
    const int per = (NT == 1 && !norm ? 128 : NT == 2 ? 128 : 64) / S;
    int cc = ntot;
    while (cc > 16 && ((uint32_t)(NT * 128 * (cc / 2 + 4) * 4) > DTC_SMEM_CAP || per * (cc / 2) > 8 * DTC_THREADS))
        cc -= 16;
    if ((uint32_t)(NT * 128 * (cc / 2 + 4) * 4) > DTC_SMEM_CAP || per * (cc / 2) > 8 * DTC_THREADS) return false;
    pl.cc = cc;
    smem = std::max<uint32_t>(smem, (uint32_t)(NT * 128 * (cc / 2 + 4) * 4));
    smem = std::max<uint32_t>(smem, DTC_SMEM_MIN);
    pl.smem = smem + 1024;  // alignment slack
    return true;
}

int split_for(int K, int NT) {
    // Eight blocks a cluster (the portable maximum); gate/up's two tiles a block take four while
    // a block's slice stays within the norm's 256 columns (hidden 1024), else eight (hidden 2048).
    return NT == 2 && K / 4 <= 256 ? 4 : 8;
}

template <int EPI>
cudaError_t launch_dtc(DtcArgs a, const void *w, int tiles, const DtcPlan &pl, cudaStream_t s) {
    constexpr int NT = DtcTraits<EPI>::NT;
    CUtensorMap map;
    if (!make_map_bf16(&map, w, (uint64_t)tiles * NT * 128, (uint64_t)a.K, 128)) return cudaErrorInvalidValue;
    a.S = pl.S;
    a.Kc = pl.Kc;
    a.G = pl.G;
    a.Npg = pl.Npg;
    a.groups = pl.groups;
    a.tmem_cols = pl.tmem_cols;
    a.cc = pl.cc;
    a.a_bytes = pl.a_bytes;
    auto kern = dtc_kernel<EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.S, tiles, 1);
    cfg.blockDim = dim3(DTC_THREADS);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = pl.S;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, map, a);
}

DtcArgs base_args(const tg_params &p, const float *x, const float *g, int K, uint32_t *err) {
    DtcArgs a{};
    a.p = p;
    a.x = x;
    a.g = g;
    a.K = K;
    a.err = err;
    return a;
}

}  // namespace

bool dtc_supported(const tg_params &p) {
    if (p.dtype != TG_BF16 || p.rows < 1 || p.rows > DTC_MAX_ROWS) return false;
    if (p.head_dim != 64 && p.head_dim != 128) return false;
    const int width = (int)((p.heads + 2 * p.kv_heads) * p.head_dim);
    if (width % 128 || p.hidden % 128 || p.inner % 128 || (p.heads * p.head_dim) % 128) return false;
    DtcPlan pl;
    return plan((int)p.hidden, 1, split_for((int)p.hidden, 1), (int)p.rows, true, pl) &&
           plan((int)p.hidden, 2, split_for((int)p.hidden, 2), (int)p.rows, true, pl) &&
           plan((int)(p.heads * p.head_dim), 1, split_for((int)(p.heads * p.head_dim), 1), (int)p.rows, false, pl);
}

bool dtc_residual_supported(const tg_params &p, int K) {
    DtcPlan pl;
    return p.dtype == TG_BF16 && plan(K, 1, split_for(K, 1), (int)p.rows, false, pl);
}

cudaError_t launch_dtc_qkv_rope(const tg_params &p, const float *x, const float *g, const void *w, const float *cosv,
                                const float *sinv, const uint32_t *at, float *q, void *kc, void *vc, uint32_t *err,
                                cudaStream_t s) {
    const int K = (int)p.hidden;
    DtcPlan pl;
    if (!plan(K, 1, split_for(K, 1), (int)p.rows, true, pl)) return cudaErrorInvalidValue;
    DtcArgs a = base_args(p, x, g, K, err);
    a.cosv = cosv;
    a.sinv = sinv;
    a.at = at;
    a.q = q;
    a.kc = kc;
    a.vc = vc;
    const int tiles = (int)((p.heads + 2 * p.kv_heads) * p.head_dim) / 128;
    return launch_dtc<DTC_QKV>(a, w, tiles, pl, s);
}

cudaError_t launch_dtc_gate_up(const tg_params &p, const float *x, const float *g, const void *w, float *out,
                               uint32_t *err, cudaStream_t s) {
    const int K = (int)p.hidden;
    DtcPlan pl;
    if (!plan(K, 2, split_for(K, 2), (int)p.rows, true, pl)) return cudaErrorInvalidValue;
    DtcArgs a = base_args(p, x, g, K, err);
    a.out = out;
    return launch_dtc<DTC_GATE_UP>(a, w, (int)p.inner / 128, pl, s);
}

cudaError_t launch_dtc_residual(const tg_params &p, const float *x, const void *w, const float *res, float *out,
                                uint32_t *err, cudaStream_t s) {
    const int K = (int)p.k;
    DtcPlan pl;
    if ((int)p.n % 128 || !plan(K, 1, split_for(K, 1), (int)p.rows, false, pl)) return cudaErrorInvalidValue;
    DtcArgs a = base_args(p, x, nullptr, K, err);
    a.res = res;
    a.out = out;
    return launch_dtc<DTC_RESIDUAL>(a, w, (int)p.n / 128, pl, s);
}

}  // namespace tg
