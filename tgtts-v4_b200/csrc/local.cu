// VoxCPM2's local stacks (crates/graph/src/local/mod.rs, dit.rs, encoder.rs): the sampler's DiT and
// the local encoder, bidirectional MiniCPM-4 stacks over the few tokens of one patch per sequence,
// f16 weights and activations with f32 sums.
//
// The projections (local_qkv_rope.comp, local_partial.comp and local_gate_up.comp over mma.glsl) run
// on tcgen05: a block takes 128 rows of W (M = 128) against a chunk of up to 256 tokens (N), the
// MMAs accumulating in TMEM. W is stored tiled (local_tiled_offset): each 128 rows x 64 columns is
// one contiguous 16 KiB block already in the 128-byte swizzle the MMA reads, and a tile's blocks
// follow each other, so that a block's share of W streams from HBM in a few large bulk copies
// (local::tiled lays W out for one stream a subgroup for the same reason, local/mod.rs:737-755).
// The tokens are staged by the block's own threads. Both go through a ring of shared-memory stages. The q/k/v, output and down projections cut their
// columns into parts (local::Tuning's o_parts and down_parts) and write each part's f32 sums; the
// kernel after joins the parts in their order: the attention (which also applies RoPE and rounds
// q, k and v to f16, as local_qkv_rope.comp's epilogue does) or the residual add with its norm.
// The gate/up projection takes whole rows (gate and up rows alternate in W) and stores
// SiLU(gate) up in f16. Each token is its own column of the MMAs, so what it comes to does not
// depend on the tokens beside it (local/mod.rs:9-11).
#include <cuda_fp16.h>

#include <algorithm>

#include "tc_common.cuh"

namespace tg {

namespace {

using half = __half;

TG_DEVICE float hround(float v) { return __half2float(__float2half_rn(v)); }

// The element (m, col) of a k-block-major [k / 64][M][64] matrix: how the tokens the projections
// read (the normed tokens, the attention's output, the SiLU output) are stored.
TG_DEVICE size_t blocked(int m, int col, int M) { return ((size_t)(col >> 6) * M + m) * 64 + (col & 63); }

// Sum of v over a block of NW warps in a fixed order (each warp's xor butterfly, then the warps
// in order); every thread gets it. `red` holds NW floats.
template <int NW>
TG_DEVICE float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; w++) t += red[w];
    __syncthreads();
    return t;
}

// ---- norms -------------------------------------------------------------------------------------

constexpr int LN_THREADS = 128;
constexpr int LN_PAIRS = 8;  // pairs of values a thread holds: rows of up to 2048
constexpr int LA_PARTS = 8;  // parts whose loads a thread issues at once

// local_norm.comp: out = f16(x scale g), scale = 1 / sqrt(mean square of x + eps). Block m takes
// token m; x is [m][hidden], out k-block-major.
__global__ void __launch_bounds__(LN_THREADS)
    local_norm_kernel(tg_params p, const half2 *__restrict__ x, const half2 *__restrict__ g, half2 *__restrict__ out) {
    __shared__ float red[LN_THREADS / 32];
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x, pairs = (int)p.hidden / 2;
    float2 v[LN_PAIRS];
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < LN_PAIRS; j++) {
        const int i = threadIdx.x + j * LN_THREADS;
        v[j] = i < pairs ? __half22float2(x[(size_t)m * pairs + i]) : make_float2(0.f, 0.f);
        sq = __fmaf_rn(v[j].x, v[j].x, sq);
        sq = __fmaf_rn(v[j].y, v[j].y, sq);
    }
    const float total = block_sum<LN_THREADS / 32>(sq, red);
    const float scale = 1.0f / sqrtf(total / (float)p.hidden + p.eps);
#pragma unroll
    for (int j = 0; j < LN_PAIRS; j++) {
        const int i = threadIdx.x + j * LN_THREADS;
        if (i >= pairs) continue;
        const float2 gg = __half22float2(g[i]);
        out[blocked(m, 2 * i, (int)p.m) / 2] = __floats2half2_rn(v[j].x * scale * gg.x, v[j].y * scale * gg.y);
    }
}

// local_add_norm.comp: sum = f16(residual + the parts' sums, joined in their order), normed =
// f16(sum scale g) with scale from the rounded sum. Block m takes token m; the residual and sum
// are [m][n], normed k-block-major.
__global__ void __launch_bounds__(LN_THREADS)
    local_add_norm_kernel(tg_params p, const float2 *__restrict__ part, const half2 *__restrict__ res,
                          const half2 *__restrict__ g, half2 *__restrict__ sum, half2 *__restrict__ normed) {
    __shared__ float red[LN_THREADS / 32];
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x, pairs = (int)p.n / 2, parts = (int)p.parts;
    const size_t part_stride = (size_t)p.m * pairs;
    float2 v[LN_PAIRS];
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < LN_PAIRS; j++) {
        const int i = threadIdx.x + j * LN_THREADS;
        v[j] = make_float2(0.f, 0.f);
        if (i < pairs) {
            float2 acc = make_float2(0.f, 0.f);
            for (int q0 = 0; q0 < parts; q0 += LA_PARTS) {
                float2 c[LA_PARTS];
#pragma unroll
                for (int q = 0; q < LA_PARTS; q++)
                    if (q0 + q < parts) c[q] = __ldcg(part + (q0 + q) * part_stride + (size_t)m * pairs + i);
#pragma unroll
                for (int q = 0; q < LA_PARTS; q++)
                    if (q0 + q < parts) acc.x += c[q].x, acc.y += c[q].y;
            }
            const float2 r = __half22float2(res[(size_t)m * pairs + i]);
            const half2 s = __floats2half2_rn(r.x + acc.x, r.y + acc.y);
            sum[(size_t)m * pairs + i] = s;
            v[j] = __half22float2(s);
        }
        sq = __fmaf_rn(v[j].x, v[j].x, sq);
        sq = __fmaf_rn(v[j].y, v[j].y, sq);
    }
    const float total = block_sum<LN_THREADS / 32>(sq, red);
    const float scale = 1.0f / sqrtf(total / (float)p.n + p.eps);
#pragma unroll
    for (int j = 0; j < LN_PAIRS; j++) {
        const int i = threadIdx.x + j * LN_THREADS;
        if (i >= pairs) continue;
        const float2 gg = __half22float2(g[i]);
        normed[blocked(m, 2 * i, (int)p.m) / 2] = __floats2half2_rn(v[j].x * scale * gg.x, v[j].y * scale * gg.y);
    }
}

// ---- attention ---------------------------------------------------------------------------------

constexpr int LA_THREADS = 256;
constexpr int LA_MAX_T = 32;

// local_qkv_rope.comp's epilogue and local_attention.comp for query head blockIdx.y of sequence
// blockIdx.x: the q/k/v projection's parts joined in order for the sequence's tokens (q of this
// head; k and v of its key-value head), q and k rotated (x cos + rotate_half(x) sin), all rounded
// to f16; then each token's scores against every key of the sequence, scaled by 1 / sqrt(hd), the
// softmax, and the weighted sum of the values, rounded to f16, stored k-block-major.
__global__ void __launch_bounds__(LA_THREADS)
    local_attention_kernel(tg_params p, const float *__restrict__ part, const float *__restrict__ cosv,
                           const float *__restrict__ sinv, half *__restrict__ out) {
    extern __shared__ __align__(16) float la_smem[];
    pdl_launch_dependents();
    pdl_wait();
    const int T = (int)p.capacity, hd = (int)p.head_dim, half_d = hd / 2, heads = (int)p.heads, kvh = (int)p.kv_heads;
    const int seq = blockIdx.x, h = blockIdx.y, kv = h / (heads / kvh), parts = (int)p.parts;
    const int width = (heads + 2 * kvh) * hd, m0 = seq * T;
    const size_t part_stride = (size_t)p.m * width;
    // q and k rows padded by 4 floats, so that the score loop's rows fall on different banks.
    const int hp = hd + 4;
    float *qs = la_smem, *ks = qs + T * hp, *vs = ks + T * hp, *sc = vs + T * hd;  // sc: [T][T + 1]
    const int cols[3] = {h * hd, (heads + kv) * hd, (heads + kvh + kv) * hd};
    float *dsts[3] = {qs, ks, vs};
    const int strides[3] = {hp, hp, hd};
    // Four columns a thread, every part's loads issued before the first sum.
    const int quads = half_d / 4;
    for (int i = threadIdx.x; i < 3 * T * quads; i += LA_THREADS) {
        const int which = i / (T * quads), t = (i / quads) % T, c = 4 * (i % quads);
        const float *src = part + (size_t)(m0 + t) * width + cols[which] + c;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
        for (int q0 = 0; q0 < parts; q0 += LA_PARTS) {
            float4 va[LA_PARTS], vb[LA_PARTS];
#pragma unroll
            for (int q = 0; q < LA_PARTS; q++) {
                if (q0 + q < parts) {
                    va[q] = __ldcg(reinterpret_cast<const float4 *>(src + (q0 + q) * part_stride));
                    vb[q] = __ldcg(reinterpret_cast<const float4 *>(src + (q0 + q) * part_stride + half_d));
                }
            }
#pragma unroll
            for (int q = 0; q < LA_PARTS; q++) {
                if (q0 + q < parts) {
                    a.x += va[q].x, a.y += va[q].y, a.z += va[q].z, a.w += va[q].w;
                    b.x += vb[q].x, b.y += vb[q].y, b.z += vb[q].z, b.w += vb[q].w;
                }
            }
        }
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float x0 = av[e], x1 = bv[e];
            if (which < 2) {
                const float cs = cosv[t * half_d + c + e], sn = sinv[t * half_d + c + e];
                const float ra = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
                const float rb = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x0, sn));
                x0 = ra;
                x1 = rb;
            }
            dsts[which][t * strides[which] + c + e] = hround(x0);
            dsts[which][t * strides[which] + c + e + half_d] = hround(x1);
        }
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf((float)hd);
    for (int i = threadIdx.x; i < T * T; i += LA_THREADS) {
        const int qi = i / T, j = i % T;
        const float4 *qq = reinterpret_cast<const float4 *>(qs + qi * hp), *kk = reinterpret_cast<const float4 *>(ks + j * hp);
        // Four running sums (dimension d to d % 4), joined (0 + 1) + (2 + 3).
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int d4 = 0; d4 < hd / 4; d4++) {
            const float4 a = qq[d4], b = kk[d4];
            acc.x = __fmaf_rn(a.x, b.x, acc.x);
            acc.y = __fmaf_rn(a.y, b.y, acc.y);
            acc.z = __fmaf_rn(a.z, b.z, acc.z);
            acc.w = __fmaf_rn(a.w, b.w, acc.w);
        }
        sc[qi * (T + 1) + j] = ((acc.x + acc.y) + (acc.z + acc.w)) * scale;
    }
    __syncthreads();
    if (threadIdx.x < T) {
        float *row = sc + threadIdx.x * (T + 1);
        float top = -INFINITY;
        for (int j = 0; j < T; j++) top = fmaxf(top, row[j]);
        float total = 0.0f;
        for (int j = 0; j < T; j++) {
            row[j] = expf(row[j] - top);
            total += row[j];
        }
        row[T] = total;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * hd; i += LA_THREADS) {
        const int qi = i / hd, d = i % hd;
        const float *row = sc + qi * (T + 1);
        float acc = 0.0f;
        for (int j = 0; j < T; j++) acc = __fmaf_rn(row[j], vs[j * hd + d], acc);
        out[blocked(m0 + qi, h * hd + d, (int)p.m)] = __float2half_rn(__fdiv_rn(acc, row[T]));
    }
}

// ---- the projections on tcgen05 ------------------------------------------------------------------

constexpr int LP_THREADS = 192;  // warp 0 streams, warp 1 issues the MMAs, warps 2-5 drain TMEM
constexpr int LP_BK = 64;
constexpr uint32_t LP_A_BYTES = 128 * LP_BK * 2;  // one k-block of W: 128 rows x 64 f16
constexpr uint32_t LP_SMEM_BUDGET = 192 * 1024;
constexpr int LP_MAX_STAGES = 8;
constexpr int LP_MAX_NT = 256;

enum { LP_PARTIAL = 0, LP_GATE_UP = 1 };

struct LocalProjArgs {
    const uint8_t *w;  // tiled: [N / 128][K / 64] blocks of 16 KiB
    int M, N, K, Kc, kblocks, NT, nkb, kb_stage, stages;
    uint32_t w_stage, stage_bytes, tmem_cols;
    float *partial;  // LP_PARTIAL: [parts][M][N]
    half *out;       // LP_GATE_UP: [M][N / 2]
    uint32_t *err;
};

// Block (tile, part, chunk): rows [128 tile, +128) of W over columns [Kc part, +Kc) against tokens
// [NT chunk, +NT). A stage is kb_stage k-blocks, two copies: W's as one bulk copy (the tile's
// k-blocks are consecutive in the tiled layout) and the tokens' as one 3-D TMA box (the tokens
// are stored k-block-major): an SM's copy engine takes about as long for a copy of 4 KiB as for
// one of tens of KiB, so that few large copies stream fastest.
template <int EPI>
__global__ void __launch_bounds__(LP_THREADS, 1)
    local_proj_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ LocalProjArgs a) {
    extern __shared__ __align__(1024) uint8_t lp_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(lp_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_u32(smem);
    __shared__ __align__(8) uint64_t full[LP_MAX_STAGES], empty[LP_MAX_STAGES], done;
    __shared__ uint32_t tmem_slot;
    __shared__ int gave_up;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, part = blockIdx.y, chunk = blockIdx.z;
    const int k0 = part * a.Kc, m0 = chunk * a.NT;
    const int S = a.stages, KB = a.kb_stage, nst = a.nkb / a.kb_stage;

    if (threadIdx.x == 0) {
        gave_up = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        mbar_init(smem_u32(&done), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
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
    // Only once every block of this launch holds its TMEM may the next launch's blocks start (and
    // allocate theirs): a block never waits for TMEM that a later launch holds.
    pdl_launch_dependents();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // W does not depend on the kernel before: its first stages are requested before the
            // wait on it, the tokens after.
            const uint8_t *wt = a.w + ((size_t)tile * a.kblocks + k0 / LP_BK) * LP_A_BYTES;
            const int pre = nst < S ? nst : S;
            for (int st = 0; st < pre; st++) {
                mbar_arrive_expect_tx(smem_u32(&full[st]), a.stage_bytes);
                bulk_load(base + st * a.stage_bytes, wt + (size_t)st * a.w_stage, a.w_stage, smem_u32(&full[st]));
            }
            pdl_wait();
            for (int st = 0; st < pre; st++)
                tma_load_3d(base + st * a.stage_bytes + a.w_stage, &xmap, 0, m0, k0 / LP_BK + st * KB, smem_u32(&full[st]));
            for (int st = pre; st < nst; st++) {
                const int s = st % S;
                mbar_wait(smem_u32(&empty[s]), ((st / S) - 1) & 1, a.err, &gave_up);
                mbar_arrive_expect_tx(smem_u32(&full[s]), a.stage_bytes);
                bulk_load(base + s * a.stage_bytes, wt + (size_t)st * a.w_stage, a.w_stage, smem_u32(&full[s]));
                tma_load_3d(base + s * a.stage_bytes + a.w_stage, &xmap, 0, m0, k0 / LP_BK + st * KB, smem_u32(&full[s]));
            }
            // Every copy this thread started has landed before the block can end.
            for (int st = nst > S ? nst - S : 0; st < nst; st++)
                mbar_wait(smem_u32(&full[st % S]), (st / S) & 1, a.err, &gave_up);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = f16_idesc(128, a.NT);
            for (int st = 0; st < nst; st++) {
                const int s = st % S;
                mbar_wait(smem_u32(&full[s]), (st / S) & 1, a.err, &gave_up);
                tc_fence_after();
                const uint32_t w_addr = base + s * a.stage_bytes, x_addr = w_addr + a.w_stage;
                for (int kb = 0; kb < KB; kb++)
#pragma unroll
                    for (int k = 0; k < LP_BK / 16; k++)
                        tc_mma(tmem, sw128_desc(w_addr + kb * LP_A_BYTES + k * 32),
                               sw128_desc(x_addr + kb * a.NT * 128 + k * 32), idesc, (st > 0 || kb > 0 || k > 0) ? 1u : 0u);
                tc_commit(smem_u32(&empty[s]));
            }
            tc_commit(smem_u32(&done));
        }
    } else {
        pdl_wait();
        mbar_wait(smem_u32(&done), 0, a.err, &gave_up);
        tc_fence_after();
        const int q = warp & 3, r = q * 32 + lane;
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
        const int m_end = min(a.M, m0 + a.NT), row0 = tile * 128;
#pragma unroll 1
        for (int c0 = 0; c0 < a.NT; c0 += 16) {
            uint32_t v[16];
            tmem_ld16_nowait(taddr + c0, v);
            tmem_wait_ld();
            if constexpr (EPI == LP_PARTIAL) {
                float *dst = a.partial + ((size_t)part * a.M) * a.N + row0 + r;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    const int m = m0 + c0 + e;
                    if (m < m_end) dst[(size_t)m * a.N] = __uint_as_float(v[e]);
                }
            } else {
                // Rows 2j and 2j + 1 of W are gate j and up j: lanes 2i and 2i + 1 trade their
                // tokens' sums, the even lane storing tokens c0 .. c0 + 7, the odd c0 + 8 .. + 15.
                const bool odd = lane & 1;
                const int j = (row0 + r) >> 1;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    const float mine = __uint_as_float(v[e]);
                    const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
                    const bool store = odd ? e >= 8 : e < 8;
                    const int m = m0 + c0 + e;
                    if (store && m < m_end) {
                        const float gate = odd ? other : mine, up = odd ? mine : other;
                        a.out[blocked(m, j, a.M)] = __float2half_rn(silu_mul(gate, up));
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
}

struct LocalPlan {
    int NT, chunks, nkb, kb_stage, stages;
    uint32_t w_stage, stage_bytes, smem, tmem_cols;
};

// The cut of a projection over M tokens and K columns in `parts`: token chunks of at most 256 (a
// multiple of 16 each); stages of as many k-blocks as let two stages (or all) fit, so that W comes
// in few large copies; TMEM columns; and shared memory enough that the blocks an SM can hold never
// ask for more than its 512 TMEM columns.
bool local_plan(int M, int K, int parts, LocalPlan &pl) {
    if (M <= 0 || parts <= 0 || K % parts) return false;
    const int Kc = K / parts;
    if (Kc % LP_BK) return false;
    pl.chunks = (M + LP_MAX_NT - 1) / LP_MAX_NT;
    pl.NT = ((M + pl.chunks - 1) / pl.chunks + 15) / 16 * 16;
    pl.nkb = Kc / LP_BK;
    const uint32_t per_kb = LP_A_BYTES + (uint32_t)pl.NT * LP_BK * 2;
    pl.kb_stage = 0;
    for (int kb : {8, 4, 2, 1}) {
        if (pl.nkb % kb) continue;
        const int nst = pl.nkb / kb;
        const int fit = (int)(LP_SMEM_BUDGET / (kb * per_kb));
        if (fit >= std::min(nst, 2)) {
            pl.kb_stage = kb;
            pl.stages = std::min({nst, fit, LP_MAX_STAGES});
            break;
        }
    }
    if (pl.kb_stage == 0) return false;
    pl.w_stage = (uint32_t)pl.kb_stage * LP_A_BYTES;
    pl.stage_bytes = (uint32_t)pl.kb_stage * per_kb;
    pl.tmem_cols = 32;
    while ((int)pl.tmem_cols < pl.NT) pl.tmem_cols *= 2;
    const uint32_t sm_bytes = 232448;  // shared memory of an SM
    const uint32_t min_smem = sm_bytes / (512 / pl.tmem_cols + 1) + 1024;
    pl.smem = std::max(pl.stages * pl.stage_bytes + 1024, min_smem);
    return true;
}

template <int EPI>
cudaError_t launch_proj(const void *x, const void *w, int M, int N, int K, int parts, float *partial, half *out,
                        uint32_t *err, cudaStream_t s) {
    LocalPlan pl;
    if (N % 128 || !local_plan(M, K, parts, pl) || reinterpret_cast<uintptr_t>(w) % 16) return cudaErrorInvalidValue;
    CUtensorMap xm;
    if (!make_map_f16_blocked(&xm, x, (uint64_t)M, (uint64_t)K, (uint32_t)pl.NT, (uint32_t)pl.kb_stage))
        return cudaErrorInvalidValue;
    LocalProjArgs a{static_cast<const uint8_t *>(w), M, N, K, K / parts, K / LP_BK, pl.NT, pl.nkb, pl.kb_stage,
                    pl.stages, pl.w_stage, pl.stage_bytes, pl.tmem_cols, partial, out, err};
    auto kern = local_proj_kernel<EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(N / 128, parts, pl.chunks), dim3(LP_THREADS), pl.smem, s, xm, a);
}

// ---- embedding, sampling ---------------------------------------------------------------------------

constexpr int LE_THREADS = 128;
constexpr int LE_MAX_FRAMES = 8;
constexpr int LE_BATCH = 4;

// local_embed.comp: for row blockIdx.y, tokens first .. first + frames - 1 of each of its `seqs`
// sequences = f16(W f16(frames) + bias) (frame f the patch's column f), and `copied` tokens at `at`
// copied from `tokens` ([copied][n] for every row when shared, else [rows][copied][n]), zero in all
// but the first sequence when guided.
__global__ void __launch_bounds__(LE_THREADS)
    local_embed_kernel(tg_params p, const float *__restrict__ src, const half *__restrict__ w,
                       const half *__restrict__ bias, const half *__restrict__ tokens, half *__restrict__ h) {
    extern __shared__ __align__(16) float le_frames[];  // [frames][feat]
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.y, feat = (int)p.feat, frames = (int)p.frames, N = (int)p.n, T = (int)p.capacity;
    for (int i = threadIdx.x; i < frames * feat; i += LE_THREADS) {
        const int f = i / feat, c = i % feat;
        le_frames[i] = hround(src[((size_t)row * feat + c) * frames + f]);
    }
    __syncthreads();
    const int n = blockIdx.x * LE_THREADS + threadIdx.x;
    if (n >= N) return;
    const bool guided = p.flags & 1, shared = p.flags & 2;
    const uint4 *wr = reinterpret_cast<const uint4 *>(w + (size_t)n * feat);
    const float b = __half2float(bias[n]);
    float acc[LE_MAX_FRAMES];
#pragma unroll
    for (int f = 0; f < LE_MAX_FRAMES; f++) acc[f] = 0.0f;
    // The row's weights 8 at a time, a batch of loads issued before the products.
    for (int c0 = 0; c0 < feat; c0 += 8 * LE_BATCH) {
        uint4 wv[LE_BATCH];
#pragma unroll
        for (int j = 0; j < LE_BATCH; j++)
            if (c0 + 8 * j < feat) wv[j] = __ldg(wr + c0 / 8 + j);
#pragma unroll
        for (int j = 0; j < LE_BATCH; j++) {
            if (c0 + 8 * j >= feat) continue;
            const half2 *h2 = reinterpret_cast<const half2 *>(&wv[j]);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 wf = __half22float2(h2[e]);
                const int c = c0 + 8 * j + 2 * e;
#pragma unroll
                for (int f = 0; f < LE_MAX_FRAMES; f++) {
                    if (f >= frames) break;
                    acc[f] = __fmaf_rn(wf.x, le_frames[f * feat + c], acc[f]);
                    acc[f] = __fmaf_rn(wf.y, le_frames[f * feat + c + 1], acc[f]);
                }
            }
        }
    }
    for (int f = 0; f < frames && f < LE_MAX_FRAMES; f++) {
        const half v = __float2half_rn(b + acc[f]);
        for (int q = 0; q < (int)p.seqs; q++) h[((size_t)(row * p.seqs + q) * T + p.first + f) * N + n] = v;
    }
    const size_t copied = shared ? 0 : (size_t)row * p.copied;
    for (int q = 0; q < (int)p.seqs; q++)
        for (int t = 0; t < (int)p.copied; t++)
            h[((size_t)(row * p.seqs + q) * T + p.at + t) * N + n] =
                guided && q > 0 ? __float2half_rn(0.0f) : tokens[(copied + t) * N + n];
}

// cfm_noise.comp: x = temperature noise, each row's temperature sampling[2 row].
__global__ void __launch_bounds__(256)
    cfm_noise_kernel(tg_params p, const float *__restrict__ noise, const float *__restrict__ sampling, float *__restrict__ x) {
    pdl_launch_dependents();
    pdl_wait();
    const int len = (int)(p.feat * p.frames);
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i < (int)p.rows * len) x[i] = sampling[2 * (i / len)] * noise[i];
}

constexpr int DE_THREADS = 256;
constexpr int DE_MAX_TOKENS = 16;  // 2 sequences x frames
constexpr int DE_BATCH = 4;        // 16-byte loads of a row a lane issues at once

// dit_euler.comp for row blockIdx.x: out_proj's velocities from tokens first .. first + frames - 1
// of the row's two sequences (conditional, unconditional; h k-block-major), CFG-Zero* guidance (the unconditional
// velocity scaled to best match the conditional, the difference scaled by the row's guidance), and
// x -= dt guided. Each velocity is a warp's xor-butterfly sum of its lanes' sums over k.
__global__ void __launch_bounds__(DE_THREADS)
    dit_euler_kernel(tg_params p, const half *__restrict__ h, const half *__restrict__ w,
                     const half *__restrict__ bias, const float *__restrict__ sampling, float *__restrict__ x) {
    extern __shared__ __align__(16) float de_smem[];
    __shared__ float red[DE_THREADS / 32];
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x, K = (int)p.k, T = (int)p.capacity, frames = (int)p.frames, feat = (int)p.feat;
    const int len = feat * frames, ntok = 2 * frames;
    float *hs = de_smem;             // [2 frames][K]
    float *vel = hs + ntok * K;      // [2][feat][frames]
    // The tokens' rows, 8 values a 16-byte load, a batch of loads issued before the stores.
    const int vecs = ntok * K / 8;
    for (int i0 = threadIdx.x; i0 < vecs; i0 += DE_THREADS * DE_BATCH) {
        uint4 v[DE_BATCH];
#pragma unroll
        for (int j = 0; j < DE_BATCH; j++) {
            const int i = i0 + j * DE_THREADS;
            if (i >= vecs) continue;
            const int m = i / (K / 8), k = 8 * (i % (K / 8)), q = m / frames, f = m % frames;
            v[j] = __ldg(reinterpret_cast<const uint4 *>(h) + blocked((2 * row + q) * T + (int)p.first + f, k, (int)p.m) / 8);
        }
#pragma unroll
        for (int j = 0; j < DE_BATCH; j++) {
            const int i = i0 + j * DE_THREADS;
            if (i >= vecs) continue;
            const half2 *h2 = reinterpret_cast<const half2 *>(&v[j]);
            float4 *dst = reinterpret_cast<float4 *>(hs + (size_t)i * 8);
            const float2 a = __half22float2(h2[0]), b = __half22float2(h2[1]), c = __half22float2(h2[2]),
                         d = __half22float2(h2[3]);
            dst[0] = make_float4(a.x, a.y, b.x, b.y);
            dst[1] = make_float4(c.x, c.y, d.x, d.y);
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Warp w takes channels w, w + 8, ...: each lane 8 columns of the channel's row at a time (all
    // of its 16-byte loads issued first), summed over the lane's columns in order, then the warp's
    // xor butterfly.
    for (int c = warp; c < feat; c += DE_THREADS / 32) {
        float acc[DE_MAX_TOKENS];
#pragma unroll
        for (int m = 0; m < DE_MAX_TOKENS; m++) acc[m] = 0.0f;
        const uint4 *wr = reinterpret_cast<const uint4 *>(w + (size_t)c * K);
        for (int k0 = 8 * lane; k0 < K; k0 += 8 * 32 * DE_BATCH) {
            uint4 wv[DE_BATCH];
#pragma unroll
            for (int j = 0; j < DE_BATCH; j++)
                if (k0 + 256 * j < K) wv[j] = __ldg(wr + (k0 + 256 * j) / 8);
#pragma unroll
            for (int j = 0; j < DE_BATCH; j++) {
                const int k = k0 + 256 * j;
                if (k >= K) continue;
                const half2 *h2 = reinterpret_cast<const half2 *>(&wv[j]);
                float wf[8];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f2 = __half22float2(h2[e]);
                    wf[2 * e] = f2.x;
                    wf[2 * e + 1] = f2.y;
                }
#pragma unroll
                for (int m = 0; m < DE_MAX_TOKENS; m++) {
                    if (m >= ntok) break;
                    const float4 x0 = *reinterpret_cast<const float4 *>(hs + m * K + k);
                    const float4 x1 = *reinterpret_cast<const float4 *>(hs + m * K + k + 4);
                    float t = acc[m];
                    t = __fmaf_rn(wf[0], x0.x, t);
                    t = __fmaf_rn(wf[1], x0.y, t);
                    t = __fmaf_rn(wf[2], x0.z, t);
                    t = __fmaf_rn(wf[3], x0.w, t);
                    t = __fmaf_rn(wf[4], x1.x, t);
                    t = __fmaf_rn(wf[5], x1.y, t);
                    t = __fmaf_rn(wf[6], x1.z, t);
                    t = __fmaf_rn(wf[7], x1.w, t);
                    acc[m] = t;
                }
            }
        }
        const float b = __half2float(bias[c]);
#pragma unroll
        for (int m = 0; m < DE_MAX_TOKENS; m++) {
            if (m >= ntok) break;
            const float s = warp_sum(acc[m]);
            if (lane == 0) vel[(m / frames) * len + c * frames + m % frames] = s + b;
        }
    }
    __syncthreads();
    float dd = 0.0f, nn = 0.0f;
    for (int i = threadIdx.x; i < len; i += DE_THREADS) {
        dd = __fmaf_rn(vel[i], vel[len + i], dd);
        nn = __fmaf_rn(vel[len + i], vel[len + i], nn);
    }
    dd = block_sum<DE_THREADS / 32>(dd, red);
    nn = block_sum<DE_THREADS / 32>(nn, red);
    const float alpha = __fdiv_rn(dd, nn + 1e-8f), cfg = sampling[2 * row + 1];
    for (int i = threadIdx.x; i < len; i += DE_THREADS) {
        const float scaled = __fmul_rn(vel[len + i], alpha);
        const float guided = __fadd_rn(scaled, __fmul_rn(cfg, __fsub_rn(vel[i], scaled)));
        x[(size_t)row * len + i] = __fsub_rn(x[(size_t)row * len + i], __fmul_rn(guided, p.dt));
    }
}

// local_rows.comp: out row r = x row r capacity (the first token of each sequence; x k-block-major).
__global__ void __launch_bounds__(128)
    local_rows_kernel(tg_params p, const uint4 *__restrict__ x, uint4 *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x, vecs = (int)p.n / 8;
    for (int v = threadIdx.x; v < vecs; v += 128)
        out[(size_t)r * vecs + v] = x[blocked(r * (int)p.capacity, 8 * v, (int)p.m) / 8];
}

// Rows [row0 + i step] of a tiled weight of K columns from src [rows][K] (row-major f16): 8 values
// a thread.
__global__ void __launch_bounds__(256)
    local_tile_rows_kernel(const uint4 *__restrict__ src, uint8_t *__restrict__ dst, int rows, int K, int row0,
                           int step) {
    const size_t n = (size_t)rows * (K / 8);
    for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (size_t)gridDim.x * 256) {
        const int r = (int)(i / (K / 8)), col = (int)(i % (K / 8)) * 8;
        *reinterpret_cast<uint4 *>(dst + local_tiled_offset(row0 + r * step, col, K)) = src[i];
    }
}

}  // namespace

cudaError_t launch_local_tile_rows(const void *src, int rows, int K, void *dst, int row0, int step, cudaStream_t s) {
    if (K % 64 || rows <= 0) return cudaErrorInvalidValue;
    const size_t n = (size_t)rows * (K / 8);
    const int blocks = (int)std::min<size_t>((n + 255) / 256, 4096);
    local_tile_rows_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint4 *>(src), static_cast<uint8_t *>(dst), rows,
                                                  K, row0, step);
    return cudaGetLastError();
}

bool local_proj_supported(int M, int N, int K, int parts) {
    LocalPlan pl;
    return N % 128 == 0 && K % 64 == 0 && local_plan(M, K, parts, pl);
}

cudaError_t launch_local_norm(const tg_params &p, const void *x, const void *g, void *out, cudaStream_t s) {
    if (p.hidden % 2 || p.hidden > 2 * LN_THREADS * LN_PAIRS) return cudaErrorInvalidValue;
    return launch_pdl(local_norm_kernel, dim3(p.m), dim3(LN_THREADS), 0, s, p, (const half2 *)x, (const half2 *)g,
                      (half2 *)out);
}

cudaError_t launch_local_add_norm(const tg_params &p, const float *part, const void *res, const void *g, void *sum,
                                  void *normed, cudaStream_t s) {
    if (p.n % 2 || p.n > 2 * LN_THREADS * LN_PAIRS) return cudaErrorInvalidValue;
    return launch_pdl(local_add_norm_kernel, dim3(p.m), dim3(LN_THREADS), 0, s, p, (const float2 *)part,
                      (const half2 *)res, (const half2 *)g, (half2 *)sum, (half2 *)normed);
}

size_t local_attention_smem(const tg_params &p) {
    return sizeof(float) * (2 * (size_t)p.capacity * (p.head_dim + 4) + (size_t)p.capacity * p.head_dim +
                            (size_t)p.capacity * (p.capacity + 1));
}

cudaError_t launch_local_attention(const tg_params &p, const float *part, const float *cosv, const float *sinv,
                                   void *out, cudaStream_t s) {
    if (p.capacity == 0 || p.capacity > LA_MAX_T || p.m % p.capacity || p.head_dim % 2 || p.kv_heads == 0 ||
        p.heads % p.kv_heads)
        return cudaErrorInvalidValue;
    const size_t smem = local_attention_smem(p);
    cudaError_t e = with_smem(local_attention_kernel, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(local_attention_kernel, dim3(p.m / p.capacity, p.heads), dim3(LA_THREADS), smem, s, p, part,
                      cosv, sinv, (half *)out);
}

cudaError_t launch_local_partial(const tg_params &p, const void *x, const void *w, float *part, uint32_t *err,
                                 cudaStream_t s) {
    return launch_proj<LP_PARTIAL>(x, w, (int)p.m, (int)p.n, (int)p.k, (int)p.parts, part, nullptr, err, s);
}

cudaError_t launch_local_gate_up(const tg_params &p, const void *x, const void *w, void *out, uint32_t *err,
                                 cudaStream_t s) {
    return launch_proj<LP_GATE_UP>(x, w, (int)p.m, (int)p.n, (int)p.k, 1, nullptr, (half *)out, err, s);
}

cudaError_t launch_local_embed(const tg_params &p, const float *src, const void *w, const void *bias,
                               const void *tokens, void *h, cudaStream_t s) {
    const size_t smem = sizeof(float) * p.frames * p.feat;
    cudaError_t e = with_smem(local_embed_kernel, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(local_embed_kernel, dim3((p.n + LE_THREADS - 1) / LE_THREADS, p.rows), dim3(LE_THREADS), smem,
                      s, p, src, (const half *)w, (const half *)bias, (const half *)tokens, (half *)h);
}

cudaError_t launch_cfm_noise(const tg_params &p, const float *noise, const float *sampling, float *x, cudaStream_t s) {
    const uint32_t n = p.rows * p.feat * p.frames;
    return launch_pdl(cfm_noise_kernel, dim3((n + 255) / 256), dim3(256), 0, s, p, noise, sampling, x);
}

size_t dit_euler_smem(const tg_params &p) {
    return sizeof(float) * (2 * (size_t)p.frames * p.k + 2 * (size_t)p.feat * p.frames);
}

cudaError_t launch_dit_euler(const tg_params &p, const void *h, const void *w, const void *bias,
                             const float *sampling, float *x, cudaStream_t s) {
    if (2 * p.frames > DE_MAX_TOKENS) return cudaErrorInvalidValue;
    const size_t smem = dit_euler_smem(p);
    cudaError_t e = with_smem(dit_euler_kernel, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(dit_euler_kernel, dim3(p.rows), dim3(DE_THREADS), smem, s, p, (const half *)h,
                      (const half *)w, (const half *)bias, sampling, x);
}

cudaError_t launch_local_rows(const tg_params &p, const void *x, void *out, cudaStream_t s) {
    if (p.n % 8) return cudaErrorInvalidValue;
    return launch_pdl(local_rows_kernel, dim3(p.rows), dim3(128), 0, s, p, (const uint4 *)x, (uint4 *)out);
}

}  // namespace tg
