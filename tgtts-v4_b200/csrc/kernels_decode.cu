// The decode step's kernels: weight-streaming GEMVs with the RMSNorm, RoPE + KV append, SiLU-mul
// and scaled residual add fused in, split-K GQA attention over the KV cache and its combine, and
// the final norm. They replace kernels/glsl/{rmsnorm,gemv_qkv_rope,attention_split,
// attention_combine,gemv_residual,gemv_gate_up}.comp.
//
// Batch invariance (crates/graph/src/decode.rs:8-11): for every (batch row, output) the sum is
// taken in one order that depends only on the weights' row length - lane l of the warp that owns
// the output takes the 16-byte vectors l, l + 32, ... in order, each element by one fused
// multiply-add, then the xor butterfly joins the lanes - never on how many rows run beside it or
// how the rows are cut over blocks. Norms are summed by tg::warp_rms_scale in every kernel.
#include <cooperative_groups.h>

#include <algorithm>

#include "tg_common.cuh"
#include "tg_internal.h"

namespace tg {

constexpr int GEMV_WARPS = 8;
// The blocks of a decode-attention cluster (the portable maximum).
constexpr int ATTN_CLUSTER = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;

// The vectors of the batch a GEMV block multiplies are staged in shared memory in f32 (the
// decode step keeps every activation in f32; only weights and the KV cache are in the storage
// type). For 8-wide bf16 weight vectors, element e of vector j of row b sits at
// xs[b][e / 4][4 j + e % 4], so that a warp's float4 reads of one half are consecutive.
template <typename T>
struct Stage {
    static constexpr int V = Vec<T>::N;
    static TG_DEVICE int index(int k, int b, int i) {  // element i of row b
        if constexpr (V == 4) return b * k + i;
        const int j = i / 8, e = i % 8;
        return b * k + (e / 4) * (k / 2) + 4 * j + (e % 4);
    }
    // The V floats of vector j of row b.
    static TG_DEVICE void load(const float *xs, int k, int b, int j, float (&x)[V]) {
        const float4 a = reinterpret_cast<const float4 *>(xs + (size_t)b * k)[j];
        x[0] = a.x;
        x[1] = a.y;
        x[2] = a.z;
        x[3] = a.w;
        if constexpr (V == 8) {
            const float4 c = reinterpret_cast<const float4 *>(xs + (size_t)b * k + k / 2)[j];
            x[4] = c.x;
            x[5] = c.y;
            x[6] = c.z;
            x[7] = c.w;
        }
    }
};

// Writes rows b0 .. b0 + NB - 1 of x ([rows][k] f32) into xs, each normed by RMSNorm with gain
// gs (already in shared memory) when `norm` (kernels/glsl/norm.glsl:47-53: x times its scale
// times the gain), rows past `rows` as zero. All threads load x at once; then warp b takes row b's
// scale from shared memory in tg::warp_rms_scale's order, and the rows are scaled in place.
template <typename T, int NB>
__device__ void stage_rows(const float *__restrict__ x, const float *gs, bool norm, int rows, int b0, int k,
                           float eps, float *xs, float *raw, float *scales) {
    const int quads = k / 4;
    for (int i = threadIdx.x; i < NB * quads; i += blockDim.x) {
        const int b = i / quads, c = i % quads;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b0 + b < rows) v = reinterpret_cast<const float4 *>(x + (size_t)(b0 + b) * k)[c];
        // Four consecutive elements 4c .. 4c + 3 stay together in either layout; `raw` is plain.
        if (norm)
            reinterpret_cast<float4 *>(raw)[i] = v;
        else
            *reinterpret_cast<float4 *>(xs + Stage<T>::index(k, b, 4 * c)) = v;
    }
    __syncthreads();
    if (!norm) return;
    const int warp = threadIdx.x >> 5;
    for (int b = warp; b < NB; b += GEMV_WARPS) {
        const float sc = (b0 + b < rows) ? warp_rms_scale(raw + (size_t)b * k, k, eps) : 0.0f;
        if ((threadIdx.x & 31) == 0) scales[b] = sc;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NB * quads; i += blockDim.x) {
        const int b = i / quads, c = i % quads;
        const float4 v = reinterpret_cast<const float4 *>(raw)[i];
        const float4 gg = reinterpret_cast<const float4 *>(gs)[c];
        const float s = scales[b];
        *reinterpret_cast<float4 *>(xs + Stage<T>::index(k, b, 4 * c)) =
            make_float4(v.x * s * gg.x, v.y * s * gg.y, v.z * s * gg.z, v.w * s * gg.w);
    }
    __syncthreads();
}

// acc[b][r] = W[r] . xs[b] for the warp's R rows, held in shared memory: lane l takes the
// 16-byte vectors l, l + 32, ... of each row in order, each element by one fused multiply-add
// (the lanes are joined by the caller). The order depends only on k.
template <typename T, int NB, int R>
TG_DEVICE void dot_smem(const T *const (&w)[R], int k, const float *xs, float (&acc)[NB][R]) {
    using VT = Vec<T>;
    using Raw = typename VT::Raw;
    constexpr int V = VT::N;
    const int lane = threadIdx.x & 31;
    const int nvec = k / V;
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int r = 0; r < R; r++) acc[b][r] = 0.0f;
#pragma unroll 4
    for (int j = lane; j < nvec; j += 32) {
        float wf[R][V];
#pragma unroll
        for (int r = 0; r < R; r++) VT::unpack(reinterpret_cast<const Raw *>(w[r])[j], wf[r]);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float xf[V];
            Stage<T>::load(xs, k, b, j, xf);
#pragma unroll
            for (int r = 0; r < R; r++)
#pragma unroll
                for (int e = 0; e < V; e++) acc[b][r] = __fmaf_rn(wf[r][e], xf[e], acc[b][r]);
        }
    }
}

template <int NB>
__device__ __forceinline__ float pick(const float (&v)[NB], int i) {
    float out = 0.0f;
#pragma unroll
    for (int b = 0; b < NB; b++)
        if (b == i) out = v[b];
    return out;
}

// What a GEMV computes for each unit of its output rows, and which weight rows a unit takes:
// gemv_qkv_rope.comp (a RoPE pair of rows of one head), gemv_gate_up.comp (gate row i and up row
// i), gemv_residual.comp (one row).
enum Epilogue { EPI_QKV_ROPE = 0, EPI_GATE_UP = 1, EPI_RESIDUAL = 2 };

struct GemvArgs {
    tg_params p;
    const float *x;  // [rows][k] f32
    const float *g;  // the RMSNorm gain, or null for an input taken as it is
    const void *w;   // [weight rows][k], storage type
    int k, units, per_block;
    const float *res;  // EPI_RESIDUAL: out = res + s W x
    float *out;        // EPI_RESIDUAL [rows][n], EPI_GATE_UP [rows][inner]
    const float *cosv, *sinv;
    const uint32_t *at;
    float *q;
    void *kc, *vc;
    uint32_t *err;
};

template <int EPI>
TG_DEVICE int unit_row(const tg_params &p, int u, int r) {
    if constexpr (EPI == EPI_QKV_ROPE) {
        const int half = p.head_dim / 2;
        return (u / half) * p.head_dim + u % half + r * half;
    } else if constexpr (EPI == EPI_GATE_UP) {
        return (int)gate_up_row((uint32_t)u, (uint32_t)r);
    } else {
        return u;
    }
}

// The epilogue of unit u for batch row b, given its R sums.
template <typename T, int EPI>
TG_DEVICE void gemv_epilogue(const GemvArgs &a, int u, int b, float y0, float y1) {
    const tg_params &p = a.p;
    if constexpr (EPI == EPI_RESIDUAL) {
        const size_t at = (size_t)b * p.n + u;
        a.out[at] = __fmaf_rn(p.residual_scale, y0, __ldcg(a.res + at));
    } else if constexpr (EPI == EPI_GATE_UP) {
        a.out[(size_t)b * p.inner + u] = silu_mul(y0, y1);
    } else {
        qkv_store<T>(p, a.at, a.cosv, a.sinv, a.q, a.kc, a.vc, u, b, y0, y1);
    }
}

// The decode GEMVs. Block i takes units [i per_block, (i + 1) per_block) of the output and streams
// their weight rows into shared memory with 1-D bulk copies (TMA, one per row) before anything
// else - before it waits on the kernel before it - so that a kernel's weights stream from HBM
// while the kernels ahead of it finish. Then it stages the batch's vectors (normed when a gain is
// given) NB rows at a time, and each warp takes units warp, warp + 8, ... against them.
// The block's units land in GEMV_STAGES groups, each on its own mbarrier, so that the warps start
// on the first group while the rest are still in flight.
constexpr int GEMV_STAGES = 1;

template <typename T, int NB, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_stream_kernel(const __grid_constant__ GemvArgs a) {
    constexpr int R = EPI == EPI_RESIDUAL ? 1 : 2;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float scales[NB];
    __shared__ __align__(8) uint64_t bar[GEMV_STAGES];
    const int k = a.k;
    const int u0 = blockIdx.x * a.per_block;
    const int nu = max(0, min(a.per_block, a.units - u0));
    const uint32_t row_bytes = (uint32_t)(k * sizeof(T));
    T *ws = reinterpret_cast<T *>(smem);
    float *xs = reinterpret_cast<float *>(smem + (size_t)a.per_block * R * row_bytes);  // [NB][k]
    float *raw = xs + (size_t)NB * k;                                                     // [NB][k]
    float *gs = raw + (size_t)NB * k;                                                     // [k]
    const bool norm = a.g != nullptr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Stage s holds units [s * per_stage, (s + 1) * per_stage) of the block's.
    const int per_stage = (nu + GEMV_STAGES - 1) / GEMV_STAGES;
    if (threadIdx.x == 0) {
        for (int st = 0; st < GEMV_STAGES; st++) mbar_init(smem_u32(&bar[st]), 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == 0) {
        if (lane < GEMV_STAGES) {
            const int lo = min(nu, lane * per_stage), hi = min(nu, (lane + 1) * per_stage);
            mbar_arrive_expect_tx(smem_u32(&bar[lane]), (uint32_t)(hi - lo) * R * row_bytes);
        }
        __syncwarp();
        // Rows that follow each other in W go in one bulk copy: a copy costs the SM's copy engine
        // about the same time whatever its size up to tens of KiB, so that row-sized copies cap a
        // block's stream well below its share of HBM. Lane r copies the block's r-th rows (unit
        // j's at ws row r nu + j), a run of consecutive rows at a time, split at stage edges.
        if (lane < R) {
            const int r = lane;
            const T *w = static_cast<const T *>(a.w);
            for (int j0 = 0; j0 < nu;) {
                const int stage = j0 / max(per_stage, 1);
                const int end = min(nu, (stage + 1) * max(per_stage, 1));
                const int row0 = unit_row<EPI>(a.p, u0 + j0, r);
                int j1 = j0 + 1;
                while (j1 < end && unit_row<EPI>(a.p, u0 + j1, r) == row0 + (j1 - j0)) j1++;
                bulk_load(smem_u32(ws + ((size_t)r * nu + j0) * k), w + (size_t)row0 * k, (uint32_t)(j1 - j0) * row_bytes,
                          smem_u32(&bar[stage]));
                j0 = j1;
            }
        }
    }
    if (norm)  // the gain is a constant: read before waiting on the kernel before
        for (int i = threadIdx.x; i < k / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(gs)[i] = reinterpret_cast<const float4 *>(a.g)[i];
    pdl_launch_dependents();
    pdl_wait();
    const int rows = a.p.rows;
    for (int b0 = 0; b0 < rows; b0 += NB) {
        stage_rows<T, NB>(a.x, gs, norm, rows, b0, k, a.p.eps, xs, raw, scales);
        for (int j = warp; j < nu; j += GEMV_WARPS) {
            // The first pass over the batch waits for each unit's stage (at once when it has landed).
            if (b0 == 0) mbar_wait_bounded(smem_u32(&bar[j / per_stage]), 0, a.err);
            const T *w[R];
#pragma unroll
            for (int r = 0; r < R; r++) w[r] = ws + ((size_t)r * nu + j) * k;
            float acc[NB][R];
            dot_smem<T, NB, R>(w, k, xs, acc);
            float y[NB][R];
#pragma unroll
            for (int b = 0; b < NB; b++)
#pragma unroll
                for (int r = 0; r < R; r++) y[b][r] = warp_sum(acc[b][r]);
            if (lane < NB && b0 + lane < rows) {
                float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
                for (int b = 0; b < NB; b++)
                    if (b == lane) {
                        y0 = y[b][0];
                        y1 = y[b][R - 1];
                    }
                gemv_epilogue<T, EPI>(a, u0 + j, b0 + lane, y0, y1);
            }
        }
        __syncthreads();
    }
    // Every stage has landed before the block ends (a block whose warps reached no unit of a stage).
    for (int st = 0; st < GEMV_STAGES; st++) mbar_wait_bounded(smem_u32(&bar[st]), 0, a.err);
}

// rmsnorm.comp: out = RMSNorm(x) g per row, a warp to a row, in f32.
__global__ void __launch_bounds__(128)
    rmsnorm_kernel(tg_params p, const float *__restrict__ x, const float *__restrict__ g,
                   float *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= (int)p.rows) return;
    const int k = p.hidden;
    const float *xr = x + (size_t)row * k;
    const float s = warp_rms_scale(xr, k, p.eps);
    float4 *o = reinterpret_cast<float4 *>(out + (size_t)row * k);
    for (int c = lane; c < k / 4; c += 32) {
        const float4 v = reinterpret_cast<const float4 *>(xr)[c];
        const float4 gg = reinterpret_cast<const float4 *>(g)[c];
        o[c] = make_float4(v.x * s * gg.x, v.y * s * gg.y, v.z * s * gg.z, v.w * s * gg.w);
    }
}

// One (chunk, kv head, row) of decode attention (attention_split.comp:52-112): the GROUP query
// heads kv head `kv` serves against ATTN_CHUNK positions from `start` of the row's slot, masked
// past `pos`: each head's chunk softmax, unnormalised, with its maximum and sum, into the
// partials. The keys and values before `pos` were written by earlier steps, so they are loaded
// before waiting on the kernel before (qkv_rope), the position's own and q after. Threads hold
// several independent sums (four heads each) so that the chains overlap; each sum is still taken
// in order over the head dimension or the positions.
//
// The partials go to o_out[h * o_stride + d] and ml_out[h * ml_stride + {0, 1}] for query head h
// of the group.
//
// `tid` and `nthreads` are the calling threads' index and count (a block, or the consumer warps
// of one), and Sync::sync() their barrier. Loads of q and the cache bypass L1 (a persistent kernel
// reads what other blocks wrote earlier in the same launch).
struct BlockSync {
    static TG_DEVICE void sync() { __syncthreads(); }
};

//
// With ONE_PASS (no kernel before it to wait on) q and every key and value are loaded in one batch.
template <typename T, typename Sync = BlockSync, bool ONE_PASS = false>
__device__ void attention_chunk(const tg_params &p, const float *__restrict__ q, const T *__restrict__ kc,
                                const T *__restrict__ vc, int b, int kv, int c, uint32_t pos, uint32_t slot,
                                float *__restrict__ o_out, size_t o_stride, float *__restrict__ ml_out,
                                size_t ml_stride, float *smem, int tid, int nthreads) {
    constexpr int C = ATTN_CHUNK;
    using VT = Vec<T>;
    using Raw = typename VT::Raw;
    constexpr int V = VT::N;
    const int hd = p.head_dim, heads = p.heads, kvh = p.kv_heads, group = heads / kvh;
    const int start = c * C;
    const int row4 = hd / 4 + 1;                  // a key row in float4s, padded
    float *qs = smem;                             // [group][hd]
    float4 *ks4 = reinterpret_cast<float4 *>(qs + group * hd);  // [C][hd/4 + 1]
    float *vs = reinterpret_cast<float *>(ks4 + C * row4);      // [C][hd]
    float *ps = vs + C * hd;                      // [group][C]
    const int first_head = kv * group;
    const size_t base = (((size_t)slot * kvh + kv) * p.capacity + start) * hd;
    const Raw *ksrc = reinterpret_cast<const Raw *>(kc + base);
    const Raw *vsrc = reinterpret_cast<const Raw *>(vc + base);
    const int per_row = hd / V;
    if (ONE_PASS) {
        const float4 *src = reinterpret_cast<const float4 *>(q + ((size_t)b * heads + first_head) * hd);
        for (int i = tid; i < group * hd / 4; i += nthreads) reinterpret_cast<float4 *>(qs)[i] = __ldcg(src + i);
    }
    for (int pass = ONE_PASS ? 1 : 0; pass < 2; pass++) {
        if (pass == 1 && !ONE_PASS) pdl_wait();  // a no-op after the first wait of the block
        for (int i = tid; i < C * per_row; i += nthreads) {
            const int pp = i / per_row, j = i % per_row;
            const int at_pos = start + pp;
            if (!ONE_PASS && (pass == 0) != (at_pos < (int)pos)) continue;
            float kf[V], vf[V];
            if (at_pos <= (int)pos) {
                VT::unpack(__ldcg(ksrc + i), kf);
                VT::unpack(__ldcg(vsrc + i), vf);
            } else {
#pragma unroll
                for (int e = 0; e < V; e++) kf[e] = vf[e] = 0.0f;
            }
            float *krow = reinterpret_cast<float *>(ks4 + pp * row4);
#pragma unroll
            for (int e = 0; e < V; e++) {
                krow[j * V + e] = kf[e];
                vs[pp * hd + j * V + e] = vf[e];
            }
        }
    }
    if (!ONE_PASS) {
        const float4 *src = reinterpret_cast<const float4 *>(q + ((size_t)b * heads + first_head) * hd);
        for (int i = tid; i < group * hd / 4; i += nthreads) reinterpret_cast<float4 *>(qs)[i] = __ldcg(src + i);
    }
    Sync::sync();
    const float scale = 1.0f / sqrtf((float)hd);
    // Scores: thread t takes position t % C for heads t / C, t / C + nh, ... (nh = threads / C).
    {
        const int nh = nthreads / C, pp = tid % C;
        for (int h0 = tid / C; h0 < group; h0 += 4 * nh) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const int hs[4] = {h0, h0 + nh, h0 + 2 * nh, h0 + 3 * nh};
            for (int d4 = 0; d4 < hd / 4; d4++) {
                const float4 kk = ks4[pp * row4 + d4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (hs[u] >= group) continue;
                    const float4 qq = reinterpret_cast<const float4 *>(qs + hs[u] * hd)[d4];
                    acc[u] = __fmaf_rn(qq.x, kk.x, acc[u]);
                    acc[u] = __fmaf_rn(qq.y, kk.y, acc[u]);
                    acc[u] = __fmaf_rn(qq.z, kk.z, acc[u]);
                    acc[u] = __fmaf_rn(qq.w, kk.w, acc[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (hs[u] < group) ps[hs[u] * C + pp] = (start + pp <= (int)pos) ? acc[u] * scale : -INFINITY;
        }
    }
    Sync::sync();
    const int warp = tid >> 5, lane = tid & 31;
    for (int h = warp; h < group; h += nthreads / 32) {
        float m = -INFINITY;
#pragma unroll
        for (int t = 0; t < C / 32; t++) m = fmaxf(m, ps[h * C + t * 32 + lane]);
        m = warp_max(m);
        float l = 0.0f;
#pragma unroll
        for (int t = 0; t < C / 32; t++) {
            const float e = expf(ps[h * C + t * 32 + lane] - m);
            ps[h * C + t * 32 + lane] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml_out[h * ml_stride] = m;
            ml_out[h * ml_stride + 1] = l;
        }
    }
    Sync::sync();
    // Outputs: thread t takes dimension t % hd for heads t / hd, t / hd + nh, ...
    {
        const int nh = nthreads / hd, d = tid % hd;
        for (int h0 = tid / hd; h0 < group; h0 += 4 * nh) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const int hs[4] = {h0, h0 + nh, h0 + 2 * nh, h0 + 3 * nh};
            for (int pp = 0; pp < C; pp++) {
                const float v = vs[pp * hd + d];
#pragma unroll
                for (int u = 0; u < 4; u++)
                    if (hs[u] < group) acc[u] = __fmaf_rn(ps[hs[u] * C + pp], v, acc[u]);
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (hs[u] < group) o_out[hs[u] * o_stride + d] = acc[u];
        }
    }
}

// acc + sum_c o[c * stride] * w[c] over c = 0 .. n - 1, folded in chunk order (one fused
// multiply-add each), with a batch of chunks' loads issued before the first is used: the loads
// come from L2 and would otherwise wait one after another.
TG_DEVICE float join_chunks(const float *o, size_t stride, const float *w, int n, float acc = 0.0f) {
    constexpr int BATCH = 16;
    for (int c0 = 0; c0 < n; c0 += BATCH) {
        float v[BATCH];
#pragma unroll
        for (int c = 0; c < BATCH; c++) v[c] = c0 + c < n ? __ldcg(o + (size_t)(c0 + c) * stride) : 0.0f;
#pragma unroll
        for (int c = 0; c < BATCH; c++)
            if (c0 + c < n) acc = __fmaf_rn(v[c], w[c0 + c], acc);
    }
    return acc;
}

// attention_combine.comp:29-58 for `n_heads` heads from `first_head` of row b: joins chunks
// 0 .. n - 1 in order - their largest maximum, the rescaled sums, and the division - into out (f32).
TG_DEVICE void attention_join(const tg_params &p, const float *__restrict__ po, const float *__restrict__ pml,
                              int b, int first_head, int n_heads, int n, float *__restrict__ out) {
    constexpr int MAXC = 64;  // chunks joined per pass of the weights below
    const int hd = p.head_dim, chunks = attn_chunks(p.capacity);
    for (int i = threadIdx.x; i < n_heads * hd; i += blockDim.x) {
        const int h = first_head + i / hd, d = i % hd;
        const float *ml = pml + ((size_t)b * p.heads + h) * chunks * 2;
        const float *o = po + ((size_t)b * p.heads + h) * chunks * hd;
        float m = -INFINITY;
        for (int c = 0; c < n; c++) m = fmaxf(m, __ldcg(ml + 2 * c));
        float total = 0.0f;
        for (int c = 0; c < n; c++) total = __fmaf_rn(__ldcg(ml + 2 * c + 1), expf(__ldcg(ml + 2 * c) - m), total);
        float acc = 0.0f;
        for (int c0 = 0; c0 < n; c0 += MAXC) {
            float w[MAXC];
            const int nc = min(MAXC, n - c0);
            for (int c = 0; c < nc; c++) w[c] = expf(__ldcg(ml + 2 * (c0 + c)) - m);
            acc = join_chunks(o + (size_t)c0 * hd + d, hd, w, nc, acc);
        }
        out[((size_t)b * p.heads + h) * hd + d] = __fdiv_rn(acc, total);
    }
}

static size_t attention_smem(const tg_params &p) {
    const size_t group = p.heads / p.kv_heads, hd = p.head_dim, C = ATTN_CHUNK;
    return sizeof(float) * (group * hd + C * (hd + 4) + C * hd + group * C);
}

// attention_split.comp as a kernel of its own: block (c, h, b). A chunk that starts past the row's
// position writes nothing, nor does a spare row.
template <typename T>
__global__ void __launch_bounds__(128)
    attention_split_kernel(tg_params p, const float *__restrict__ q, const T *__restrict__ kc,
                           const T *__restrict__ vc, const uint32_t *__restrict__ at,
                           float *__restrict__ po, float *__restrict__ pml) {
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_launch_dependents();
    uint32_t pos, slot;
    const int c = blockIdx.x, kv = blockIdx.y, b = blockIdx.z;
    if (!placed(at, p.rows, b, p.capacity, p.slots, pos, slot) || c * (int)ATTN_CHUNK > (int)pos) {
        pdl_wait();
        return;
    }
    const int group = p.heads / p.kv_heads, chunks = attn_chunks(p.capacity);
    const size_t head0 = (size_t)b * p.heads + kv * group;
    attention_chunk<T>(p, q, kc, vc, b, kv, c, pos, slot, po + (head0 * chunks + c) * p.head_dim,
                       (size_t)chunks * p.head_dim, pml + (head0 * chunks + c) * 2, (size_t)chunks * 2,
                       reinterpret_cast<float *>(smem), threadIdx.x, blockDim.x);
}

// attention_combine.comp as a kernel of its own: block (h, b). The chunks' maxima and sums are
// staged in shared memory in one parallel load, then folded in chunk order as attention_join does.
__global__ void __launch_bounds__(128)
    attention_combine_kernel(tg_params p, const uint32_t *__restrict__ at,
                             const float *__restrict__ po, const float *__restrict__ pml,
                             float *__restrict__ out, uint32_t width) {
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, b = blockIdx.y, hd = p.head_dim;
    uint32_t pos, slot;
    if (!placed(at, p.rows, b, p.capacity, p.slots, pos, slot)) return;
    // Partials of `width` positions each, laid out as ATTN_CHUNK's (attn_chunks(capacity) a head).
    const int chunks = attn_chunks(p.capacity), n = pos / width + 1;
    float *ml = reinterpret_cast<float *>(smem);  // [n][2]
    float *w = ml + 2 * chunks;                    // [n]
    __shared__ float m_s, total_s;
    const float *src = pml + ((size_t)b * p.heads + h) * chunks * 2;
    for (int i = threadIdx.x; i < 2 * n; i += blockDim.x) ml[i] = __ldcg(src + i);
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = -INFINITY;
        for (int c = 0; c < n; c++) m = fmaxf(m, ml[2 * c]);
        float total = 0.0f;
        for (int c = 0; c < n; c++) total = __fmaf_rn(ml[2 * c + 1], expf(ml[2 * c] - m), total);
        m_s = m;
        total_s = total;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < n; c += blockDim.x) w[c] = expf(ml[2 * c] - m_s);
    __syncthreads();
    const float *o = po + ((size_t)b * p.heads + h) * chunks * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x)
        out[((size_t)b * p.heads + h) * hd + d] = __fdiv_rn(join_chunks(o + d, hd, w, n), total_s);
}

// Split and combine in one kernel, as a thread-block cluster: the ATTN_CLUSTER blocks of cluster
// (b, kv) take chunks r, r + ATTN_CLUSTER, ... of row b's positions (block r), keep each chunk's
// partials in their own shared memory, and after a cluster barrier block h < GROUP joins query
// head h's chunks in chunk order, reading the other blocks' partials over distributed shared
// memory. The same sums in the same order as attention_split + attention_combine, so the same bits.
template <typename T>
__global__ void __launch_bounds__(128)
    attention_decode_kernel(tg_params p, const float *__restrict__ q, const T *__restrict__ kc,
                            const T *__restrict__ vc, const uint32_t *__restrict__ at, float *__restrict__ out) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_launch_dependents();
    const int r = (int)cluster.block_rank(), kv = blockIdx.y, b = blockIdx.z;
    const int hd = p.head_dim, heads = p.heads, group = heads / p.kv_heads;
    const int chunks = attn_chunks(p.capacity), mine = (chunks + ATTN_CLUSTER - 1) / ATTN_CLUSTER;
    // This block's partials: [mine][group][hd] outputs, then [mine][group][2] maxima and sums, then
    // (16-byte aligned) the chunk's working space.
    float *my_o = reinterpret_cast<float *>(smem);
    float *my_ml = my_o + (size_t)mine * group * hd;
    float *work = my_o + ((size_t)mine * group * (hd + 2) + 3) / 4 * 4;
    uint32_t pos = 0, slot = 0;
    const bool live = placed(at, p.rows, b, p.capacity, p.slots, pos, slot);
    const int n = live ? (int)(pos / ATTN_CHUNK) + 1 : 0;
    bool waited = false;
    for (int i = 0; i < mine; i++) {
        const int c = r + i * ATTN_CLUSTER;
        if (c >= n) break;
        if (i > 0) __syncthreads();
        attention_chunk<T>(p, q, kc, vc, b, kv, c, pos, slot, my_o + (size_t)i * group * hd, (size_t)hd,
                           my_ml + (size_t)i * group * 2, 2, work, threadIdx.x, blockDim.x);
        waited = true;
    }
    if (!waited) pdl_wait();
    cluster.sync();
    // Join: block r takes query heads r, r + ATTN_CLUSTER, ... It first gathers the head's chunk
    // partials from their blocks into its own shared memory (all loads at once), then takes
    // attention_combine's sums in chunk order.
    float *go = work;                        // [n][hd]
    float *gml = work + (size_t)chunks * hd;  // [n][2]
    for (int h = r; live && h < group; h += ATTN_CLUSTER) {
        for (int i = threadIdx.x; i < n * (hd + 2); i += blockDim.x) {
            const int c = i / (hd + 2), e = i % (hd + 2);
            const int owner = c % ATTN_CLUSTER, at_i = c / ATTN_CLUSTER;
            if (e < hd)
                go[(size_t)c * hd + e] = cluster.map_shared_rank(my_o, owner)[((size_t)at_i * group + h) * hd + e];
            else
                gml[(size_t)c * 2 + (e - hd)] = cluster.map_shared_rank(my_ml, owner)[((size_t)at_i * group + h) * 2 + (e - hd)];
        }
        __syncthreads();
        float m = -INFINITY;
        for (int c = 0; c < n; c++) m = fmaxf(m, gml[2 * c]);
        float total = 0.0f;
        for (int c = 0; c < n; c++) total = __fmaf_rn(gml[2 * c + 1], expf(gml[2 * c] - m), total);
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            float acc = 0.0f;
            for (int c = 0; c < n; c++) acc = __fmaf_rn(go[(size_t)c * hd + d], expf(gml[2 * c] - m), acc);
            out[((size_t)b * heads + kv * group + h) * hd + d] = __fdiv_rn(acc, total);
        }
        __syncthreads();
    }
    cluster.sync();  // no block leaves while another may still read its partials
}

// ---- the persistent decode step ----------------------------------------------------------------
//
// One cooperative launch runs the whole step - every layer's q/k/v projection with RoPE and the
// KV append, attention, the output projection, gate/up, down, and the final norm - with one block
// per SM. Each block's producer warp streams the block's share of every weight matrix, in the
// order the phases use them, through a ring of PS_SLOTS shared-memory slots with 1-D bulk copies
// (TMA, no multicast), so that HBM keeps streaming the next phases' weights while the consumer
// warps wait at the grid barriers between phases. The consumers take the same sums in the same
// order as the per-kernel step (dot_smem, warp_rms_scale, attention_chunk, attention_combine's
// join), so a row's results are the same bits on either path. Every wait is bounded in time: a
// block that gives up sets the context's error word and a global abort word that ends the others'
// waits, drains its copies in flight and returns.

constexpr int PS_CONSUMERS = 8;                 // consumer warps
constexpr int PS_CTHREADS = PS_CONSUMERS * 32;  // consumer threads
constexpr int PS_THREADS = PS_CTHREADS + 32;    // and one producer warp
constexpr int PS_SLOTS = 6;
constexpr uint32_t PS_SLOT_BYTES = 28 * 1024;
constexpr int PS_ROWS = 2;                      // the most rows a persistent step takes
constexpr uint64_t PS_WAIT_NS = 2000000000ull;  // 2 s

struct ConsumerSync {
    static TG_DEVICE void sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
};

enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3 };

struct PersistArgs {
    tg_params p;
    int layers;
    const unsigned char *weights;
    const uint64_t *offs;  // [layers][6] byte offsets of qkv, o, gate_up, down, input norm, post norm
    uint64_t final_norm;   // byte offset of the final gain
    const float *cosv, *sinv;
    const uint32_t *at;
    const float *x_in;
    float *h, *mid, *mlp, *q, *out, *po, *pml;
    unsigned char *kcache, *vcache;
    uint64_t cache_layer;
    uint32_t *sync;  // [0] grid-barrier arrivals, [1] abort; zero at launch
    uint32_t *err;
    int units[4], per[4], seg[4], nseg[4], k[4];
    int segs_per_layer;
    uint32_t xs_floats, raw_floats;  // shared-memory layout after the slots
};

TG_DEVICE uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits on an mbarrier phase, giving up at the time limit or when another block aborted.
TG_DEVICE bool mbar_wait_abortable(uint32_t bar, uint32_t parity, const PersistArgs &a) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*(volatile uint32_t *)(a.sync + 1)) return false;
            if (globaltimer() - t0 > PS_WAIT_NS) {
                atomicExch(a.err, ERR_WAIT_TIMEOUT);
                atomicExch(a.sync + 1, 1u);
                return false;
            }
        }
    }
}

// The grid barrier of the consumer warps: every block adds its arrival (release), then waits
// until all have (acquire). Returns false when the step was aborted.
TG_DEVICE bool grid_barrier(const PersistArgs &a, uint32_t &count, int *ok_s) {
    ConsumerSync::sync();
    count += gridDim.x;
    if (threadIdx.x == 0) {
        int ok = 1;
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.sync) : "memory");
        const uint64_t t0 = globaltimer();
        for (uint32_t i = 0;; i++) {
            if (ld_acquire(a.sync) >= count) break;
            if ((i & 15) == 0) {
                if (*(volatile uint32_t *)(a.sync + 1)) {
                    ok = 0;
                    break;
                }
                if (globaltimer() - t0 > PS_WAIT_NS) {
                    atomicExch(a.err, ERR_WAIT_TIMEOUT);
                    atomicExch(a.sync + 1, 1u);
                    ok = 0;
                    break;
                }
            }
        }
        *ok_s = ok;
    }
    ConsumerSync::sync();
    return *ok_s != 0;
}

TG_DEVICE int phase_rows(int ph) { return (ph == PH_QKV || ph == PH_GU) ? 2 : 1; }

template <typename T>
TG_DEVICE const T *phase_weights(const PersistArgs &a, int l, int ph) {
    return reinterpret_cast<const T *>(a.weights + a.offs[l * 6 + ph]);
}

TG_DEVICE int weight_row(const tg_params &p, int ph, int u, int r) {
    switch (ph) {
        case PH_QKV: return unit_row<EPI_QKV_ROPE>(p, u, r);
        case PH_GU: return unit_row<EPI_GATE_UP>(p, u, r);
        default: return u;
    }
}

// Segment g of the step: its layer, phase and index within the phase.
TG_DEVICE void segment_of(const PersistArgs &a, int g, int &l, int &ph, int &s) {
    l = g / a.segs_per_layer;
    int r = g % a.segs_per_layer;
    for (ph = 0; ph < 4; ph++) {
        if (r < a.nseg[ph]) break;
        r -= a.nseg[ph];
    }
    s = r;
}

// The units [ub, ue) of segment s of phase ph for this block.
TG_DEVICE void segment_units(const PersistArgs &a, int ph, int s, int &ub, int &ue) {
    const int b0 = blockIdx.x * a.per[ph];
    const int b1 = min(b0 + a.per[ph], a.units[ph]);
    ub = min(b0 + s * a.seg[ph], b1);
    ue = min(ub + a.seg[ph], b1);
}

// rows of x ([rows][k] f32, other blocks' writes) into xs in Stage layout, normed with gain g when
// given: the consumer-warp version of stage_rows.
template <typename T>
TG_DEVICE void persist_stage(const float *x, const float *g, int rows, int k, float eps, float *xs, float *raw,
                             float *scales, int ctid) {
    const int quads = k / 4;
    for (int i = ctid; i < PS_ROWS * quads; i += PS_CTHREADS) {
        const int b = i / quads, c = i % quads;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b < rows) v = __ldcg(reinterpret_cast<const float4 *>(x + (size_t)b * k) + c);
        if (g)
            reinterpret_cast<float4 *>(raw)[i] = v;
        else
            *reinterpret_cast<float4 *>(xs + Stage<T>::index(k, b, 4 * c)) = v;
    }
    ConsumerSync::sync();
    if (!g) return;
    const int warp = ctid >> 5;
    if (warp < PS_ROWS) {
        const float sc = warp < rows ? warp_rms_scale(raw + (size_t)warp * k, k, eps) : 0.0f;
        if ((ctid & 31) == 0) scales[warp] = sc;
    }
    ConsumerSync::sync();
    for (int i = ctid; i < PS_ROWS * quads; i += PS_CTHREADS) {
        const int b = i / quads, c = i % quads;
        const float4 v = reinterpret_cast<const float4 *>(raw)[i];
        const float4 gg = reinterpret_cast<const float4 *>(g)[c];
        const float sc = scales[b];
        *reinterpret_cast<float4 *>(xs + Stage<T>::index(k, b, 4 * c)) =
            make_float4(v.x * sc * gg.x, v.y * sc * gg.y, v.z * sc * gg.z, v.w * sc * gg.w);
    }
    ConsumerSync::sync();
}

template <typename T, int EPI>
TG_DEVICE void persist_gemv_segment(const PersistArgs &a, const GemvArgs &ga, const T *slot, int ub, int ue,
                                    int k, const float *xs, int rows, int ctid) {
    constexpr int R = EPI == EPI_RESIDUAL ? 1 : 2;
    const int warp = ctid >> 5, lane = ctid & 31;
    for (int j = warp; j < ue - ub; j += PS_CONSUMERS) {
        const T *w[R];
#pragma unroll
        for (int r = 0; r < R; r++) w[r] = slot + (size_t)(j * R + r) * k;
        float acc[PS_ROWS][R];
        dot_smem<T, PS_ROWS, R>(w, k, xs, acc);
        float y[PS_ROWS][R];
#pragma unroll
        for (int b = 0; b < PS_ROWS; b++)
#pragma unroll
            for (int r = 0; r < R; r++) y[b][r] = warp_sum(acc[b][r]);
        if (lane < rows) {
            float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
            for (int b = 0; b < PS_ROWS; b++)
                if (b == lane) {
                    y0 = y[b][0];
                    y1 = y[b][R - 1];
                }
            gemv_epilogue<T, EPI>(ga, ub + j, lane, y0, y1);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(PS_THREADS, 1) decode_step_kernel(const __grid_constant__ PersistArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[PS_SLOTS], empty[PS_SLOTS];
    __shared__ float scales[PS_ROWS];
    __shared__ int ok_s;
    const tg_params &p = a.p;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows = p.rows;
    T *slots = reinterpret_cast<T *>(smem);
    float *scratch = reinterpret_cast<float *>(smem + (size_t)PS_SLOTS * PS_SLOT_BYTES);
    float *xs = scratch;                      // [PS_ROWS][kmax], Stage layout
    float *raw = scratch + a.xs_floats;       // [PS_ROWS][hidden]
    float *comb = raw + a.raw_floats;         // the join's maxima, sums and weights
    float *work = scratch;                    // attention's working space (aliases the above)
    auto slot_ptr = [&](int g) { return slots + (size_t)(g % PS_SLOTS) * (PS_SLOT_BYTES / sizeof(T)); };
    if (threadIdx.x == 0) {
        for (int i = 0; i < PS_SLOTS; i++) {
            mbar_init(smem_u32(&full[i]), 1);
            mbar_init(smem_u32(&empty[i]), 1);
        }
        mbar_fence_init();
    }
    __syncthreads();
    const int total = a.layers * a.segs_per_layer;

    if (warp == PS_CONSUMERS) {
        // Producer: every segment in order, each into the next slot once its last use is released.
        int issued = 0;
        for (int g = 0; g < total; g++) {
            const int slot = g % PS_SLOTS;
            if (g >= PS_SLOTS && !mbar_wait_abortable(smem_u32(&empty[slot]), ((g / PS_SLOTS) - 1) & 1, a)) break;
            int l, ph, sg, ub, ue;
            segment_of(a, g, l, ph, sg);
            segment_units(a, ph, sg, ub, ue);
            const int R = phase_rows(ph);
            const uint32_t row_bytes = (uint32_t)(a.k[ph] * sizeof(T));
            const int n = (ue - ub) * R;
            if (lane == 0) mbar_arrive_expect_tx(smem_u32(&full[slot]), (uint32_t)n * row_bytes);
            __syncwarp();
            const T *w = phase_weights<T>(a, l, ph);
            T *dst = slot_ptr(g);
            for (int j = lane; j < n; j += 32) {
                const int row = weight_row(p, ph, ub + j / R, j % R);
                bulk_load(smem_u32(dst + (size_t)j * a.k[ph]), w + (size_t)row * a.k[ph], row_bytes,
                          smem_u32(&full[slot]));
            }
            issued = g + 1;
        }
        // Every copy issued has landed before the block ends.
        for (int g = max(0, issued - PS_SLOTS); g < issued; g++)
            mbar_wait_bounded(smem_u32(&full[g % PS_SLOTS]), (g / PS_SLOTS) & 1, a.err, 100000000ull);
        return;
    }

    // Consumers.
    const int ctid = threadIdx.x;
    uint32_t count = 0;
    bool ok = true;
    int g = 0;
    const int hd = p.head_dim, heads = p.heads, kvh = p.kv_heads, group = heads / kvh;
    const int chunks = attn_chunks(p.capacity), H = p.hidden;
    uint32_t pos[PS_ROWS], slotw[PS_ROWS];
    int nchunks[PS_ROWS];
    bool live[PS_ROWS];
    for (int b = 0; b < PS_ROWS; b++) {
        live[b] = b < rows && placed(a.at, rows, b, p.capacity, p.slots, pos[b], slotw[b]);
        nchunks[b] = live[b] ? (int)(pos[b] / ATTN_CHUNK) + 1 : 0;
    }
    auto take = [&](int gg) -> bool {
        return mbar_wait_abortable(smem_u32(&full[gg % PS_SLOTS]), (gg / PS_SLOTS) & 1, a);
    };
    auto give = [&](int gg) {
        ConsumerSync::sync();
        if (ctid == 0) mbar_arrive(smem_u32(&empty[gg % PS_SLOTS]));
    };
    for (int l = 0; l < a.layers && ok; l++) {
        const float *x = l == 0 ? a.x_in : a.h;
        const float *g_in = reinterpret_cast<const float *>(a.weights + a.offs[l * 6 + 4]);
        const float *g_post = reinterpret_cast<const float *>(a.weights + a.offs[l * 6 + 5]);
        T *kc = reinterpret_cast<T *>(a.kcache + (size_t)l * a.cache_layer);
        T *vc = reinterpret_cast<T *>(a.vcache + (size_t)l * a.cache_layer);
        // q, k, v with RoPE and the KV append.
        if (l > 0 && !(ok = grid_barrier(a, count, &ok_s))) break;
        persist_stage<T>(x, g_in, rows, H, p.eps, xs, raw, scales, ctid);
        {
            GemvArgs ga{};
            ga.p = p;
            ga.cosv = a.cosv;
            ga.sinv = a.sinv;
            ga.at = a.at;
            ga.q = a.q;
            ga.kc = kc;
            ga.vc = vc;
            for (int sg = 0; sg < a.nseg[PH_QKV] && ok; sg++, g++) {
                int ub, ue;
                segment_units(a, PH_QKV, sg, ub, ue);
                if (!(ok = take(g))) break;
                persist_gemv_segment<T, EPI_QKV_ROPE>(a, ga, slot_ptr(g), ub, ue, a.k[PH_QKV], xs, rows, ctid);
                give(g);
            }
        }
        if (!ok || !(ok = grid_barrier(a, count, &ok_s))) break;
        // Attention: items (row, kv head, chunk) dealt over the blocks.
        {
            int item = 0;
            for (int b = 0; b < rows; b++)
                for (int kv = 0; kv < kvh; kv++)
                    for (int c = 0; c < nchunks[b]; c++, item++) {
                        if (item % (int)gridDim.x != (int)blockIdx.x) continue;
                        const size_t head0 = (size_t)b * heads + kv * group;
                        attention_chunk<T, ConsumerSync, true>(p, a.q, kc, vc, b, kv, c, pos[b], slotw[b],
                                                         a.po + (head0 * chunks + c) * hd, (size_t)chunks * hd,
                                                         a.pml + (head0 * chunks + c) * 2, (size_t)chunks * 2,
                                                         work, ctid, PS_CTHREADS);
                        ConsumerSync::sync();
                    }
        }
        if (!(ok = grid_barrier(a, count, &ok_s))) break;
        // The join of every head's chunks (attention_combine's order), into xs as o_proj's input.
        {
            const int K = heads * hd;
            float *cml = comb;                                   // [PS_ROWS][heads][chunks][2]
            float *wts = cml + (size_t)PS_ROWS * heads * chunks * 2;  // [PS_ROWS][heads][chunks]
            float *tot = wts + (size_t)PS_ROWS * heads * chunks;      // [PS_ROWS][heads]
            for (int i = ctid; i < rows * heads * chunks * 2; i += PS_CTHREADS) {
                const int b = i / (heads * chunks * 2);
                const int c = (i / 2) % chunks;
                if (c < nchunks[b]) cml[i] = __ldcg(a.pml + i);
            }
            ConsumerSync::sync();
            for (int bh = ctid; bh < rows * heads; bh += PS_CTHREADS) {
                const int b = bh / heads, n = nchunks[b];
                const float *ml = cml + (size_t)bh * chunks * 2;
                float m = -INFINITY;
                for (int c = 0; c < n; c++) m = fmaxf(m, ml[2 * c]);
                float total = 0.0f;
                for (int c = 0; c < n; c++) total = __fmaf_rn(ml[2 * c + 1], expf(ml[2 * c] - m), total);
                for (int c = 0; c < n; c++) wts[(size_t)bh * chunks + c] = expf(ml[2 * c] - m);
                tot[bh] = total;
            }
            ConsumerSync::sync();
            // Thread t takes outputs t, t + 256, t + 512, t + 768 of each pass; the first NC chunks
            // of all four are loaded in one batch (static indices, so the loads stay independent
            // in registers), then each output is folded in chunk order (later chunks, if any, by
            // join_chunks, continuing the same fold).
            constexpr int U = 4, NC = 16;
            const int outs = PS_ROWS * K;
            for (int i0 = 0; i0 < outs; i0 += PS_CTHREADS * U) {
                float v[U][NC];
                int n_u[U], bh_u[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int i = i0 + u * PS_CTHREADS + ctid;
                    const int b = i / K, hdd = i % K, h = hdd / hd, d = hdd % hd;
                    const int n = (i < outs && b < rows && live[b]) ? nchunks[b] : 0;
                    n_u[u] = n;
                    bh_u[u] = b * heads + h;
                    const float *o = a.po + (size_t)(b * heads + h) * chunks * hd + d;
#pragma unroll
                    for (int c = 0; c < NC; c++) v[u][c] = c < n ? __ldcg(o + (size_t)c * hd) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int i = i0 + u * PS_CTHREADS + ctid;
                    if (i >= outs) continue;
                    const int b = i / K, hdd = i % K, d = hdd % hd, n = n_u[u], bh = bh_u[u];
                    float val = 0.0f;
                    if (n > 0) {
                        const float *w = wts + (size_t)bh * chunks;
                        float acc = 0.0f;
#pragma unroll
                        for (int c = 0; c < NC; c++)
                            if (c < n) acc = __fmaf_rn(v[u][c], w[c], acc);
                        if (n > NC)
                            acc = join_chunks(a.po + (size_t)bh * chunks * hd + d + (size_t)NC * hd, hd, w + NC, n - NC, acc);
                        val = __fdiv_rn(acc, tot[bh]);
                    }
                    xs[Stage<T>::index(K, b, hdd)] = val;
                }
            }
            ConsumerSync::sync();
            GemvArgs ga{};
            ga.p = p;
            ga.p.n = H;
            ga.res = x;
            ga.out = a.mid;
            for (int sg = 0; sg < a.nseg[PH_O] && ok; sg++, g++) {
                int ub, ue;
                segment_units(a, PH_O, sg, ub, ue);
                if (!(ok = take(g))) break;
                persist_gemv_segment<T, EPI_RESIDUAL>(a, ga, slot_ptr(g), ub, ue, a.k[PH_O], xs, rows, ctid);
                give(g);
            }
        }
        if (!ok || !(ok = grid_barrier(a, count, &ok_s))) break;
        // gate/up with the post-attention norm, SiLU-mul.
        persist_stage<T>(a.mid, g_post, rows, H, p.eps, xs, raw, scales, ctid);
        {
            GemvArgs ga{};
            ga.p = p;
            ga.out = a.mlp;
            for (int sg = 0; sg < a.nseg[PH_GU] && ok; sg++, g++) {
                int ub, ue;
                segment_units(a, PH_GU, sg, ub, ue);
                if (!(ok = take(g))) break;
                persist_gemv_segment<T, EPI_GATE_UP>(a, ga, slot_ptr(g), ub, ue, a.k[PH_GU], xs, rows, ctid);
                give(g);
            }
        }
        if (!ok || !(ok = grid_barrier(a, count, &ok_s))) break;
        // down with the residual.
        persist_stage<T>(a.mlp, nullptr, rows, p.inner, p.eps, xs, raw, scales, ctid);
        {
            GemvArgs ga{};
            ga.p = p;
            ga.p.n = H;
            ga.res = a.mid;
            ga.out = a.h;
            for (int sg = 0; sg < a.nseg[PH_DOWN] && ok; sg++, g++) {
                int ub, ue;
                segment_units(a, PH_DOWN, sg, ub, ue);
                if (!(ok = take(g))) break;
                persist_gemv_segment<T, EPI_RESIDUAL>(a, ga, slot_ptr(g), ub, ue, a.k[PH_DOWN], xs, rows, ctid);
                give(g);
            }
        }
    }
    if (ok && (ok = grid_barrier(a, count, &ok_s)) && blockIdx.x == 0) {
        // The final norm (rmsnorm.comp), in f32.
        const float *gf = reinterpret_cast<const float *>(a.weights + a.final_norm);
        for (int i = ctid; i < rows * (H / 4); i += PS_CTHREADS)
            reinterpret_cast<float4 *>(raw)[i] = __ldcg(reinterpret_cast<const float4 *>(a.h) + i);
        ConsumerSync::sync();
        const int w8 = ctid >> 5;
        if (w8 < rows) {
            const float sc = warp_rms_scale(raw + (size_t)w8 * H, H, p.eps);
            for (int c = lane; c < H / 4; c += 32) {
                const float4 v = reinterpret_cast<const float4 *>(raw + (size_t)w8 * H)[c];
                const float4 gg = reinterpret_cast<const float4 *>(gf)[c];
                reinterpret_cast<float4 *>(a.out + (size_t)w8 * H)[c] =
                    make_float4(v.x * sc * gg.x, v.y * sc * gg.y, v.z * sc * gg.z, v.w * sc * gg.w);
            }
        }
    }
    // An aborted step releases the slots it still holds, so that the producer is not left waiting.
    if (!ok && ctid == 0)
        for (int i = 0; i < PS_SLOTS; i++) mbar_arrive(smem_u32(&empty[i]));
}

// stream_read.comp: reads the buffer once, 16 bytes per load, and writes one word per block of
// their xor, so that no read can be left out: the HBM floor the GEMVs are measured against.
__global__ void __launch_bounds__(256) stream_read_kernel(const uint4 *__restrict__ data,
                                                          uint64_t n, uint32_t *__restrict__ out) {
    uint4 acc = make_uint4(0, 0, 0, 0);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) v[u] = (i + u * stride < n) ? ld_stream(data + i + u * stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            acc.x ^= v[u].x;
            acc.y ^= v[u].y;
            acc.z ^= v[u].z;
            acc.w ^= v[u].w;
        }
    }
    uint32_t w = acc.x ^ acc.y ^ acc.z ^ acc.w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w ^= __shfl_xor_sync(0xffffffffu, w, o);
    __shared__ uint32_t words[8];
    if ((threadIdx.x & 31) == 0) words[threadIdx.x >> 5] = w;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t x = 0;
        for (int i = 0; i < 8; i++) x ^= words[i];
        out[blockIdx.x] = x;
    }
}

// ---- launchers -------------------------------------------------------------------------------

#define TG_DISPATCH_NB(NB_VAR, ...)                           \
    switch (NB_VAR) {                                         \
        case 1: { constexpr int NB = 1; __VA_ARGS__; } break;  \
        case 2: { constexpr int NB = 2; __VA_ARGS__; } break;  \
        case 4: { constexpr int NB = 4; __VA_ARGS__; } break;  \
        default: { constexpr int NB = 8; __VA_ARGS__; } break; \
    }

// The SMs of the current device (the decode kernels size their grids to one wave).
static int device_sms() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// The shared memory a decode GEMV block may take, weights and staged vectors together.
constexpr size_t GEMV_SMEM_LIMIT = 200 * 1024;
#ifndef TG_GEMV_SMEM_SHARE
#define TG_GEMV_SMEM_SHARE (96 * 1024)
#endif
constexpr size_t GEMV_SMEM_SHARE = TG_GEMV_SMEM_SHARE;

// Launches gemv_stream_kernel over `units` units of R rows of k columns: one block per SM, each
// taking an equal share, or more blocks when a share's weights would not fit in shared memory.
template <typename T, int EPI>
static cudaError_t launch_gemv(GemvArgs a, cudaStream_t s) {
    constexpr int R = EPI == EPI_RESIDUAL ? 1 : 2;
    const uint32_t rows = a.p.rows;
    int nb = 8;
    while (nb > 1 && (uint32_t)nb / 2 >= rows) nb /= 2;
    const size_t row_bytes = (size_t)a.k * sizeof(T);
    // xs, and for a normed input its raw copy and the gain: fewer batch rows staged at once when a
    // wide input (a 6144-column down projection) would not fit beside a unit's weights. A row's sums
    // do not depend on how many rows are staged with it.
    auto staged = [&](int n) { return (size_t)n * a.k * 4 * (a.g ? 2 : 1) + (a.g ? (size_t)a.k * 4 : 0); };
    while (nb > 1 && staged(nb) + R * row_bytes > GEMV_SMEM_LIMIT) nb /= 2;
    const size_t xs_bytes = staged(nb);
    if (xs_bytes + R * row_bytes > GEMV_SMEM_LIMIT) return cudaErrorInvalidValue;
    int blocks = std::min(a.units, device_sms());
    a.per_block = (a.units + blocks - 1) / blocks;
    // Slices small enough that two blocks fit an SM: the next kernel's blocks can then start (and
    // stream their weights) beside this kernel's last ones.
    while (a.per_block > 1 && (size_t)a.per_block * R * row_bytes + xs_bytes > GEMV_SMEM_SHARE) {
        a.per_block = (a.per_block + 1) / 2;
    }
    blocks = (a.units + a.per_block - 1) / a.per_block;
    const size_t smem = (size_t)a.per_block * R * row_bytes + xs_bytes;
    cudaError_t e = cudaSuccess;
    TG_DISPATCH_NB(nb, {
        auto kern = gemv_stream_kernel<T, NB, EPI>;
        if ((e = with_smem(kern, smem)) != cudaSuccess) return e;
        e = launch_pdl(kern, dim3(blocks), dim3(GEMV_THREADS), smem, s, a);
    });
    return e;
}

template <int EPI>
static cudaError_t launch_gemv_t(const GemvArgs &a, cudaStream_t s) {
    return a.p.dtype == TG_BF16 ? launch_gemv<bf16, EPI>(a, s) : launch_gemv<float, EPI>(a, s);
}

cudaError_t launch_gemv_qkv_rope(const tg_params &p, const float *x, const float *g, const void *w,
                                 const float *cs, const float *sn, const uint32_t *at, void *q, void *kc, void *vc,
                                 uint32_t *err, cudaStream_t s) {
    GemvArgs a{};
    a.p = p;
    a.x = x;
    a.g = g;
    a.w = w;
    a.k = (int)p.hidden;
    a.units = (int)((p.heads + 2 * p.kv_heads) * p.head_dim / 2);
    a.cosv = cs;
    a.sinv = sn;
    a.at = at;
    a.q = static_cast<float *>(q);
    a.kc = kc;
    a.vc = vc;
    a.err = err;
    return launch_gemv_t<EPI_QKV_ROPE>(a, s);
}

cudaError_t launch_gemv_residual(const tg_params &p, const void *x, const void *w, const float *res, float *out,
                                 uint32_t *err, cudaStream_t s) {
    GemvArgs a{};
    a.p = p;
    a.x = static_cast<const float *>(x);
    a.w = w;
    a.k = (int)p.k;
    a.units = (int)p.n;
    a.res = res;
    a.out = out;
    a.err = err;
    return launch_gemv_t<EPI_RESIDUAL>(a, s);
}

cudaError_t launch_gemv_gate_up(const tg_params &p, const float *x, const float *g, const void *w, void *out,
                                uint32_t *err, cudaStream_t s) {
    GemvArgs a{};
    a.p = p;
    a.x = x;
    a.g = g;
    a.w = w;
    a.k = (int)p.hidden;
    a.units = (int)p.inner;
    a.out = static_cast<float *>(out);
    a.err = err;
    return launch_gemv_t<EPI_GATE_UP>(a, s);
}

cudaError_t launch_rmsnorm(const tg_params &p, const float *x, const float *g, float *out,
                           cudaStream_t s) {
    return launch_pdl(rmsnorm_kernel, dim3((p.rows + 3) / 4), dim3(128), 0, s, p, x, g, out);
}

template <typename T>
static cudaError_t split_t(const tg_params &p, const void *q, const void *kc, const void *vc,
                           const uint32_t *at, float *po, float *pml, cudaStream_t s) {
    const size_t smem = attention_smem(p);
    auto kern = attention_split_kernel<T>;
    cudaError_t e = with_smem(kern, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(attn_chunks(p.capacity), p.kv_heads, p.rows);
    return launch_pdl(kern, grid, dim3(128), smem, s, p, (const float *)q, (const T *)kc, (const T *)vc, at, po, pml);
}

cudaError_t launch_attention_split(const tg_params &p, const void *q, const void *kc,
                                   const void *vc, const uint32_t *at, float *po, float *pml,
                                   cudaStream_t s) {
    return p.dtype == TG_BF16 ? split_t<bf16>(p, q, kc, vc, at, po, pml, s)
                              : split_t<float>(p, q, kc, vc, at, po, pml, s);
}

cudaError_t launch_attention_combine_chunk(const tg_params &p, uint32_t chunk, const uint32_t *at, const float *po,
                                           const float *pml, void *out, cudaStream_t s) {
    dim3 grid(p.heads, p.rows);
    const int threads = p.head_dim < 128 ? p.head_dim : 128;
    const size_t smem = (size_t)3 * (attn_chunks(p.capacity)) * sizeof(float);
    return launch_pdl(attention_combine_kernel, grid, dim3(threads), smem, s, p, at, po, pml, (float *)out, chunk);
}

cudaError_t launch_attention_combine(const tg_params &p, const uint32_t *at, const float *po,
                                     const float *pml, void *out, cudaStream_t s) {
    return launch_attention_combine_chunk(p, ATTN_CHUNK, at, po, pml, out, s);
}

static size_t cluster_attention_smem(const tg_params &p) {
    const size_t group = p.heads / p.kv_heads, hd = p.head_dim;
    const size_t chunks = attn_chunks(p.capacity), mine = (chunks + ATTN_CLUSTER - 1) / ATTN_CLUSTER;
    const size_t gather = chunks * (hd + 2) * sizeof(float);  // the join's copy of one head's partials
    return sizeof(float) * ((mine * group * (hd + 2) + 3) / 4 * 4) + std::max(attention_smem(p), gather);
}

template <typename T>
static cudaError_t decode_attention_t(const tg_params &p, const void *q, const void *kc, const void *vc,
                                      const uint32_t *at, void *out, cudaStream_t s) {
    const size_t smem = cluster_attention_smem(p);
    auto kern = attention_decode_kernel<T>;
    cudaError_t e = with_smem(kern, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ATTN_CLUSTER, p.kv_heads, p.rows);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = ATTN_CLUSTER;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, p, (const float *)q, (const T *)kc, (const T *)vc, at, (float *)out);
}

cudaError_t launch_attention_decode(const tg_params &p, const void *q, const void *kc, const void *vc,
                                    const uint32_t *at, void *out, cudaStream_t s) {
    return p.dtype == TG_BF16 ? decode_attention_t<bf16>(p, q, kc, vc, at, out, s)
                              : decode_attention_t<float>(p, q, kc, vc, at, out, s);
}

// The persistent step over a decoder's buffers: partitions each phase's units over the SMs and
// its weight rows into slot-sized segments. Returns cudaErrorNotSupported for shapes or batches it
// does not take (more than PS_ROWS rows, a unit's rows larger than a slot).
cudaError_t launch_decode_step(const DecodeStep &d, int sm_count, cudaStream_t s) {
    const tg_params &p = d.p;
    if (p.rows == 0 || p.rows > (uint32_t)PS_ROWS) return cudaErrorNotSupported;
    const size_t es = p.dtype == TG_BF16 ? 2 : 4;
    PersistArgs a{};
    a.p = p;
    a.layers = d.layers;
    a.weights = d.weights;
    a.offs = d.offs;
    a.final_norm = d.final_norm;
    a.cosv = d.cosv;
    a.sinv = d.sinv;
    a.at = d.at;
    a.x_in = d.x_in;
    a.h = d.h;
    a.mid = d.mid;
    a.mlp = d.mlp;
    a.q = d.q;
    a.out = d.out;
    a.po = d.po;
    a.pml = d.pml;
    a.kcache = d.kcache;
    a.vcache = d.vcache;
    a.cache_layer = d.cache_layer;
    a.sync = d.sync;
    a.err = d.err;
    const int units[4] = {(int)((p.heads + 2 * p.kv_heads) * p.head_dim / 2), (int)p.hidden, (int)p.inner,
                          (int)p.hidden};
    const int ks[4] = {(int)p.hidden, (int)(p.heads * p.head_dim), (int)p.hidden, (int)p.inner};
    const int G = sm_count;
    a.segs_per_layer = 0;
    for (int ph = 0; ph < 4; ph++) {
        const int R = (ph == PH_QKV || ph == PH_GU) ? 2 : 1;
        const size_t unit_bytes = (size_t)R * ks[ph] * es;
        if (unit_bytes > PS_SLOT_BYTES) return cudaErrorNotSupported;
        a.units[ph] = units[ph];
        a.k[ph] = ks[ph];
        a.per[ph] = (units[ph] + G - 1) / G;
        a.seg[ph] = (int)(PS_SLOT_BYTES / unit_bytes);
        a.nseg[ph] = (a.per[ph] + a.seg[ph] - 1) / a.seg[ph];
        a.segs_per_layer += a.nseg[ph];
    }
    const uint32_t kmax = std::max({p.hidden, p.inner, p.heads * p.head_dim});
    a.xs_floats = PS_ROWS * kmax;
    a.raw_floats = PS_ROWS * p.hidden;
    const uint32_t chunks = attn_chunks(p.capacity);
    const size_t comb_floats = (size_t)PS_ROWS * p.heads * chunks * 3 + PS_ROWS * p.heads;
    const size_t scratch = std::max((size_t)(a.xs_floats + a.raw_floats) * 4 + comb_floats * 4, attention_smem(p));
    const size_t smem = (size_t)PS_SLOTS * PS_SLOT_BYTES + scratch;
    if (smem > 227 * 1024) return cudaErrorNotSupported;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(PS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (p.dtype == TG_BF16) {
        auto kern = decode_step_kernel<bf16>;
        if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess) return e;
        int per_sm = 0;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, PS_THREADS, smem)) != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorNotSupported;
        if ((e = cudaMemsetAsync(d.sync, 0, 8, s)) != cudaSuccess) return e;
        return cudaLaunchKernelEx(&cfg, kern, a);
    }
    auto kern = decode_step_kernel<float>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess) return e;
    int per_sm = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, PS_THREADS, smem)) != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    if ((e = cudaMemsetAsync(d.sync, 0, 8, s)) != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_stream_read(const tg_params &p, const uint32_t *data, uint32_t *out,
                               cudaStream_t s, int sm_count) {
    const uint64_t n = (uint64_t)p.k / 4;  // p.k words, 4 to a uint4
    int blocks = sm_count * 8;
    stream_read_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const uint4 *>(data), n, out);
    return cudaGetLastError();
}

}  // namespace tg
