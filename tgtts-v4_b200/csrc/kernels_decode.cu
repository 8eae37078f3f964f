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

#include <algorithm>
#include <type_traits>

#include "mma_common.cuh"
#include "tg_common.cuh"
#include "tg_internal.h"

namespace tg {

constexpr int GEMV_WARPS = 8;
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
// of one), and Sync::sync() their barrier. `wait()` is what the calling threads wait on before
// reading what the step wrote (q and the position's own key and value): the kernel before, or in
// the persistent step the phase counter of q/k/v. Loads of q and the cache bypass L1 (a persistent
// kernel reads what other blocks wrote earlier in the same launch).
struct BlockSync {
    static TG_DEVICE void sync() { __syncthreads(); }
};
struct PdlWait {
    TG_DEVICE void operator()() const { pdl_wait(); }
};

// A chunk's scores (attention_split.comp:73-86): thread t takes position t % C for the HPT heads
// t / C, t / C + nh, ... (nh = threads / C, HPT = group / nh rounded up); each score is one chain
// of fused multiply-adds in order over the head dimension, scaled, or -inf past the position. The
// heads' chains run side by side and the head dimension is unrolled, so that shared-memory loads
// run ahead of the arithmetic.
template <int HPT, int C>
TG_DEVICE void chunk_scores(const float *qs, const float4 *ks4, int row4, float *ps, int hd, int group, int start,
                            int pos, float scale, int tid, int nthreads) {
    const int nh = nthreads / C, pp = tid % C, h0 = tid / C;
    const float4 *qr[HPT];
#pragma unroll
    for (int u = 0; u < HPT; u++) qr[u] = reinterpret_cast<const float4 *>(qs + min(h0 + u * nh, group - 1) * hd);
    const float4 *kr = ks4 + pp * row4;
    float acc[HPT];
#pragma unroll
    for (int u = 0; u < HPT; u++) acc[u] = 0.0f;
#pragma unroll 8
    for (int d4 = 0; d4 < hd / 4; d4++) {
        const float4 kk = kr[d4];
#pragma unroll
        for (int u = 0; u < HPT; u++) {
            const float4 qq = qr[u][d4];
            acc[u] = __fmaf_rn(qq.x, kk.x, acc[u]);
            acc[u] = __fmaf_rn(qq.y, kk.y, acc[u]);
            acc[u] = __fmaf_rn(qq.z, kk.z, acc[u]);
            acc[u] = __fmaf_rn(qq.w, kk.w, acc[u]);
        }
    }
#pragma unroll
    for (int u = 0; u < HPT; u++) {
        const int h = h0 + u * nh;
        if (h < group) ps[h * C + pp] = (start + pp <= pos) ? acc[u] * scale : -INFINITY;
    }
}

// A chunk's unnormalised outputs (attention_split.comp:95-108): thread t takes dimension t % hd for
// the HPT heads t / hd, t / hd + nh, ...; each output one chain in order over the positions.
template <int HPT, int C>
TG_DEVICE void chunk_outputs(const float *vs, const float *ps, int hd, int group, float *o_out, size_t o_stride,
                             int tid, int nthreads) {
    const int nh = nthreads / hd, d = tid % hd, h0 = tid / hd;
    const float *pr[HPT];
#pragma unroll
    for (int u = 0; u < HPT; u++) pr[u] = ps + min(h0 + u * nh, group - 1) * C;
    float acc[HPT];
#pragma unroll
    for (int u = 0; u < HPT; u++) acc[u] = 0.0f;
#pragma unroll 16
    for (int pp = 0; pp < C; pp++) {
        const float v = vs[pp * hd + d];
#pragma unroll
        for (int u = 0; u < HPT; u++) acc[u] = __fmaf_rn(pr[u][pp], v, acc[u]);
    }
#pragma unroll
    for (int u = 0; u < HPT; u++) {
        const int h = h0 + u * nh;
        if (h < group) o_out[h * o_stride + d] = acc[u];
    }
}

// The chunk's softmax (attention_split.comp:84-94) over scaled scores ps [group][C] (masked
// positions -inf): m = the largest, e = exp(s - m) in place, l = sum e, a warp to a head; m and l
// stored.
template <typename Sync>
TG_DEVICE void chunk_softmax(float *ps, int group, float *__restrict__ ml_out, size_t ml_stride, int tid,
                             int nthreads) {
    constexpr int C = ATTN_CHUNK;
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
}

// attention_chunk for bf16 caches and a head dimension of 64, on the tensor cores: the chunk's keys
// and values stay bf16 in shared memory (rows padded for ldmatrix), the group's query heads are
// the rows of mma.sync.m16n8k16 (rows past the group zero): S = q K^T with q split into bf16 hi +
// lo (two MMAs a step, so the scores carry 16 bits of each query value), then chunk_softmax, then
// O = e V with e split the same way and V^T fragments by ldmatrix.trans. Warp w takes the 16-column
// tile pairs w, w + warps, ... of S and of O, so an element's MMAs and their order are the same
// for any thread count.
template <typename Sync, typename Wait>
__device__ void attention_chunk_mma(const tg_params &p, const float *__restrict__ q, const bf16 *__restrict__ kc,
                                    const bf16 *__restrict__ vc, int b, int kv, int c, uint32_t pos, uint32_t slot,
                                    float *__restrict__ o_out, size_t o_stride, float *__restrict__ ml_out,
                                    size_t ml_stride, float *smem, int tid, int nthreads, const Wait &wait) {
    constexpr int C = ATTN_CHUNK, HD = 64, ROW = HD + fa::PAD;
    static_assert(C == 64, "four 16-position k-steps and four tile pairs a chunk");
    const int heads = p.heads, kvh = p.kv_heads, group = heads / kvh;
    const int start = c * C, first_head = kv * group;
    bf16 *ks = reinterpret_cast<bf16 *>(smem);  // [C][ROW]
    bf16 *vs = ks + C * ROW;                    // [C][ROW]
    float *qs = reinterpret_cast<float *>(vs + C * ROW);  // [group][HD]
    float *ps = qs + group * HD;                          // [group][C]
    const size_t base = (((size_t)slot * kvh + kv) * p.capacity + start) * HD;
    const uint4 *ksrc = reinterpret_cast<const uint4 *>(kc + base);
    const uint4 *vsrc = reinterpret_cast<const uint4 *>(vc + base);
    // Keys and values, 8 bf16 at a time: the positions before the row's before the wait, the row's
    // own (which the kernel before appends) after it; past it zero.
    for (int pass = 0; pass < 2; pass++) {
        if (pass == 1) wait();  // a no-op after the first wait of the block
        for (int i = tid; i < C * (HD / 8); i += nthreads) {
            const int pp = i / (HD / 8), j = i % (HD / 8);
            const int at_pos = start + pp;
            if ((pass == 0) != (at_pos < (int)pos)) continue;
            uint4 kk = make_uint4(0u, 0u, 0u, 0u), vv = kk;
            if (at_pos <= (int)pos) {
                kk = __ldcg(ksrc + i);
                vv = __ldcg(vsrc + i);
            }
            *reinterpret_cast<uint4 *>(ks + pp * ROW + j * 8) = kk;
            *reinterpret_cast<uint4 *>(vs + pp * ROW + j * 8) = vv;
        }
    }
    {
        const float4 *src = reinterpret_cast<const float4 *>(q + ((size_t)b * heads + first_head) * HD);
        for (int i = tid; i < group * HD / 4; i += nthreads) reinterpret_cast<float4 *>(qs)[i] = __ldcg(src + i);
    }
    Sync::sync();
    const int warp = tid >> 5, lane = tid & 31, warps = nthreads >> 5, g = lane >> 2, t4 = lane & 3;
    const int mi = lane >> 3, rr = lane & 7;
    const float scale = 1.0f / sqrtf((float)HD);
    // Row r's columns k0 + 2 t4 and + 1 of a [group][ld] f32 matrix, as hi and lo bf16 pairs.
    auto frag = [&](const float *m, int ld, int r, int k0, uint32_t &hi, uint32_t &lo) {
        hi = lo = 0u;
        if (r < group) {
            const float2 x = *reinterpret_cast<const float2 *>(m + r * ld + k0 + 2 * t4);
            fa::split_pack(x.x, x.y, hi, lo);
        }
    };
    // S = q K^T: tile pair t covers positions 16 t .. 16 t + 15.
    for (int t = warp; t < C / 16; t += warps) {
        float sc[2][4] = {};
#pragma unroll
        for (int s = 0; s < HD / 16; s++) {
            uint32_t qh[4], ql[4], kb[4];
            frag(qs, HD, g, 16 * s, qh[0], ql[0]);
            frag(qs, HD, g + 8, 16 * s, qh[1], ql[1]);
            frag(qs, HD, g, 16 * s + 8, qh[2], ql[2]);
            frag(qs, HD, g + 8, 16 * s + 8, qh[3], ql[3]);
            fa::ldmatrix_x4(kb, ks + (16 * t + (mi >> 1) * 8 + rr) * ROW + 16 * s + (mi & 1) * 8);
            fa::mma_bf16(sc[0], qh, kb[0], kb[1]);
            fa::mma_bf16(sc[0], ql, kb[0], kb[1]);
            fa::mma_bf16(sc[1], qh, kb[2], kb[3]);
            fa::mma_bf16(sc[1], ql, kb[2], kb[3]);
        }
#pragma unroll
        for (int jj = 0; jj < 2; jj++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int h = g + 8 * (e >> 1), col = 16 * t + 8 * jj + 2 * t4 + (e & 1);
                if (h < group) ps[h * C + col] = start + col <= (int)pos ? sc[jj][e] * scale : -INFINITY;
            }
    }
    Sync::sync();
    chunk_softmax<Sync>(ps, group, ml_out, ml_stride, tid, nthreads);
    Sync::sync();
    // O = e V: tile pair t covers dimensions 16 t .. 16 t + 15.
    for (int t = warp; t < HD / 16; t += warps) {
        float o[2][4] = {};
#pragma unroll
        for (int s = 0; s < C / 16; s++) {
            uint32_t ph[4], pl[4], vb[4];
            frag(ps, C, g, 16 * s, ph[0], pl[0]);
            frag(ps, C, g + 8, 16 * s, ph[1], pl[1]);
            frag(ps, C, g, 16 * s + 8, ph[2], pl[2]);
            frag(ps, C, g + 8, 16 * s + 8, ph[3], pl[3]);
            fa::ldmatrix_x4_trans(vb, vs + (16 * s + (mi & 1) * 8 + rr) * ROW + 16 * t + (mi >> 1) * 8);
            fa::mma_bf16(o[0], ph, vb[0], vb[1]);
            fa::mma_bf16(o[0], pl, vb[0], vb[1]);
            fa::mma_bf16(o[1], ph, vb[2], vb[3]);
            fa::mma_bf16(o[1], pl, vb[2], vb[3]);
        }
#pragma unroll
        for (int jj = 0; jj < 2; jj++)
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int h = g + 8 * i;
                if (h < group)
                    *reinterpret_cast<float2 *>(o_out + h * o_stride + 16 * t + 8 * jj + 2 * t4) =
                        make_float2(o[jj][2 * i], o[jj][2 * i + 1]);
            }
    }
}

template <typename T, typename Sync = BlockSync, typename Wait = PdlWait>
__device__ void attention_chunk(const tg_params &p, const float *__restrict__ q, const T *__restrict__ kc,
                                const T *__restrict__ vc, int b, int kv, int c, uint32_t pos, uint32_t slot,
                                float *__restrict__ o_out, size_t o_stride, float *__restrict__ ml_out,
                                size_t ml_stride, float *smem, int tid, int nthreads, const Wait &wait = Wait()) {
    if constexpr (std::is_same<T, bf16>::value) {
        if (p.head_dim == 64) {
            attention_chunk_mma<Sync>(p, q, kc, vc, b, kv, c, pos, slot, o_out, o_stride, ml_out, ml_stride, smem, tid,
                                      nthreads, wait);
            return;
        }
    }
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
    for (int pass = 0; pass < 2; pass++) {
        if (pass == 1) wait();  // a no-op after the first wait of the block
        for (int i = tid; i < C * per_row; i += nthreads) {
            const int pp = i / per_row, j = i % per_row;
            const int at_pos = start + pp;
            if ((pass == 0) != (at_pos < (int)pos)) continue;
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
    {
        const float4 *src = reinterpret_cast<const float4 *>(q + ((size_t)b * heads + first_head) * hd);
        for (int i = tid; i < group * hd / 4; i += nthreads) reinterpret_cast<float4 *>(qs)[i] = __ldcg(src + i);
    }
    Sync::sync();
    const float scale = 1.0f / sqrtf((float)hd);
    switch ((group + nthreads / C - 1) / (nthreads / C)) {
        case 1: chunk_scores<1, C>(qs, ks4, row4, ps, hd, group, start, (int)pos, scale, tid, nthreads); break;
        case 2: chunk_scores<2, C>(qs, ks4, row4, ps, hd, group, start, (int)pos, scale, tid, nthreads); break;
        case 4: chunk_scores<4, C>(qs, ks4, row4, ps, hd, group, start, (int)pos, scale, tid, nthreads); break;
        default: chunk_scores<8, C>(qs, ks4, row4, ps, hd, group, start, (int)pos, scale, tid, nthreads); break;
    }
    Sync::sync();
    chunk_softmax<Sync>(ps, group, ml_out, ml_stride, tid, nthreads);
    Sync::sync();
    switch ((group + nthreads / hd - 1) / (nthreads / hd)) {
        case 1: chunk_outputs<1, C>(vs, ps, hd, group, o_out, o_stride, tid, nthreads); break;
        case 2: chunk_outputs<2, C>(vs, ps, hd, group, o_out, o_stride, tid, nthreads); break;
        case 4: chunk_outputs<4, C>(vs, ps, hd, group, o_out, o_stride, tid, nthreads); break;
        default: chunk_outputs<8, C>(vs, ps, hd, group, o_out, o_stride, tid, nthreads); break;
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

static size_t attention_smem(const tg_params &p) {
    const size_t group = p.heads / p.kv_heads, hd = p.head_dim, C = ATTN_CHUNK;
    if (p.dtype == TG_BF16 && hd == 64)  // attention_chunk_mma: bf16 keys and values, f32 q and scores
        return 2 * C * (64 + fa::PAD) * sizeof(bf16) + sizeof(float) * (group * hd + group * C);
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
// staged in shared memory in one parallel load, then folded in chunk order. The output in f32, or
// rounded to bf16 (OT) for a tcgen05 GEMM's operand.
template <typename OT>
__global__ void __launch_bounds__(128)
    attention_combine_kernel(tg_params p, const uint32_t *__restrict__ at,
                             const float *__restrict__ po, const float *__restrict__ pml,
                             OT *__restrict__ out, uint32_t width) {
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
        out[((size_t)b * p.heads + h) * hd + d] = from_f32<OT>(__fdiv_rn(join_chunks(o + d, hd, w, n), total_s));
}

// ---- the persistent decode step ----------------------------------------------------------------
//
// One cooperative launch runs the whole step, one block per SM, as a dataflow over per-phase
// arrival counters instead of grid-wide barriers. A layer is five phases: q/k/v (+ RMSNorm, RoPE,
// KV append), attention over 64-position chunks, the join of the chunks with the output
// projection (+ residual), gate/up (+ RMSNorm, SiLU-mul), and down (+ residual). Each block takes
// a fixed share of every phase - a run of the projection's output units, and attention chunks dealt
// from the last block down, to the blocks that q/k/v leaves idle - and bumps the phase's counter
// once its share is written. A block with work in a phase first waits until every block has
// bumped the counter of the phase before; a block without work bumps at once. Every counter is used
// once per step (the launch zeroes them), so no barrier is reused and no block waits for one that
// has nothing to give it.
//
// The producer warp streams the block's share of every weight matrix, in the order the phases use
// them, into a byte ring in shared memory with 1-D bulk copies (TMA, no multicast): one copy per run
// of consecutive weight rows, one to four runs of up to ~112 KB a projection - few large copies,
// which is what lets each SM's copy engine take its share of HBM. It runs ahead of the consumers by
// up to the ring, so the next phases' weights land while the consumer warps wait on a handoff.
//
// The consumers take the same sums in the same order as the six-kernels-a-layer step (dot_smem,
// warp_rms_scale, attention_chunk, attention_combine's join, the epilogues), so a row comes out the
// same bits on either path. Every wait is bounded in time: a block that gives up sets the context's
// error word and an abort word that ends the other blocks' waits, waits (bounded) for its copies in
// flight, and returns.

constexpr int PS_CONSUMERS = 8;                 // consumer warps
constexpr int PS_CTHREADS = PS_CONSUMERS * 32;  // consumer threads
constexpr int PS_THREADS = PS_CTHREADS + 32;    // and one producer warp
constexpr int PS_ROWS = 2;                      // the most rows a persistent step takes
constexpr int PS_NBAR = 16;                     // weight segments a block has in flight at most
constexpr int PS_NCOUNT = 4;                    // a phase's arrivals, spread over this many words
constexpr int PS_PHASES = 5;
constexpr uint64_t PS_WAIT_NS = 2000000000ull;  // 2 s

enum { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4 };

struct ConsumerSync {
    static TG_DEVICE void sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
};

struct PersistArgs {
    tg_params p;
    int layers;
    const unsigned char *weights;
    const uint64_t *offs;  // [layers][6] byte offsets of qkv, o, gate_up, down, input norm, post norm
    uint64_t final_norm;   // byte offset of the final gain
    const float *cosv, *sinv;
    const uint32_t *at;
    const float *x_in;
    float *h, *mid, *mlp, *q, *att, *out, *po, *pml;
    unsigned char *kcache, *vcache;
    uint64_t cache_layer;
    // [layers][PS_PHASES][PS_NCOUNT] arrivals, then the abort word; zero at launch.
    uint32_t *flags;
    uint32_t *err;
    uint32_t ring;    // bytes of the weight ring at the start of dynamic shared memory
    int prefetch;     // at the end, prefetch the block's first-layer weights into L2 for the next step
};

TG_DEVICE uint32_t *abort_word(const PersistArgs &a) { return a.flags + (size_t)a.layers * PS_PHASES * PS_NCOUNT; }

// The units, row length and rows per unit of weight phase wi (0 q/k/v, 1 o, 2 gate/up, 3 down).
struct WPhase {
    int units, k, R;
};
TG_DEVICE WPhase wphase(const tg_params &p, int wi) {
    switch (wi) {
        case 0: return {(int)((p.heads + 2 * p.kv_heads) * p.head_dim / 2), (int)p.hidden, 2};
        case 1: return {(int)p.hidden, (int)(p.heads * p.head_dim), 1};
        case 2: return {(int)p.inner, (int)p.hidden, 2};
        default: return {(int)p.hidden, (int)p.inner, 1};
    }
}
TG_DEVICE int wrow(const tg_params &p, int wi, int u, int r) {
    if (wi == 0) return unit_row<EPI_QKV_ROPE>(p, u, r);
    if (wi == 2) return unit_row<EPI_GATE_UP>(p, u, r);
    return u;
}
// This block's units [ub, ue) of weight phase wi, dealt in runs of ceil(units / blocks) from block
// 0 up. q/k/v leaves as many blocks at the top of the grid as the step can have attention items (at
// most half of them), so that the blocks that take attention have no q/k/v to finish first.
__host__ __device__ inline int phase_blocks(const tg_params &p, int wi, int grid) {
    if (wi != 0) return grid;
    const int most = (int)(p.rows * p.kv_heads * attn_chunks(p.capacity));
    return grid - min(most, grid / 2);
}
TG_DEVICE void share(const tg_params &p, int wi, int units, int &ub, int &ue) {
    const int blocks = phase_blocks(p, wi, gridDim.x);
    const int per = (units + blocks - 1) / blocks;
    ub = min(units, (int)blockIdx.x * per);
    ue = min(units, ub + per);
}
// Places a segment of `bytes` at the next linear ring position from `lin` that is a multiple of
// its row length: returns its linear start and moves lin past it. Producer and consumers place
// alike. A segment may wrap around the ring's end; the ring is a multiple of every row length, so
// no row is split by the wrap.
TG_DEVICE uint32_t ring_place(uint32_t &lin, uint32_t bytes, uint32_t row_bytes) {
    lin = (lin + row_bytes - 1) / row_bytes * row_bytes;
    const uint32_t start = lin;
    lin += bytes;
    return start;
}

// A weight segment in the ring: row i (unit j's row r is row r nu + j) starts at linear position
// start + i row_bytes, taken modulo the ring.
struct SegRef {
    const unsigned char *ring;
    uint32_t start, size, row_bytes;
    template <typename T>
    TG_DEVICE const T *row(int i) const {
        return reinterpret_cast<const T *>(ring + (start + (uint32_t)i * row_bytes) % size);
    }
};

// The consumers' arrival at phase ph of layer l: every store of the phase issued (the barrier),
// then one thread publishes them and bumps one of the phase's counters in one release (the
// barrier orders the other threads' stores before it, as a grid barrier's fence does).
TG_DEVICE void arrive(const PersistArgs &a, int l, int ph, int ctid) {
    ConsumerSync::sync();
    if (ctid == 0) {
        uint32_t *c = a.flags + ((size_t)l * PS_PHASES + ph) * PS_NCOUNT + blockIdx.x % PS_NCOUNT;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(c) : "memory");
    }
}

// Waits until every block has arrived at phase ph of layer l (lanes 0 .. PS_NCOUNT - 1 of the first
// consumer warp each watch one counter), then lets all consumer threads on. False when a wait gave
// up or another block aborted.
TG_DEVICE bool wait_phase(const PersistArgs &a, int l, int ph, int ctid, int *ok_s) {
    if (ctid < 32) {
        bool ok = true;
        if (ctid < PS_NCOUNT) {
            const uint32_t target = (gridDim.x - ctid + PS_NCOUNT - 1) / PS_NCOUNT;
            ok = flag_wait_bounded(a.flags + ((size_t)l * PS_PHASES + ph) * PS_NCOUNT + ctid, target, a.err,
                                   PS_WAIT_NS, abort_word(a));
        }
        ok = __all_sync(0xffffffffu, ok);
        if (ctid == 0) *ok_s = ok;
    }
    ConsumerSync::sync();
    return *ok_s != 0;
}

// Waits on an mbarrier phase, giving up at the time limit or when another block aborted.
TG_DEVICE bool mbar_wait_abortable(uint32_t bar, uint32_t parity, const PersistArgs &a) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*(volatile uint32_t *)abort_word(a)) return false;
            if (globaltimer() - t0 > PS_WAIT_NS) {
                atomicExch(a.err, ERR_WAIT_TIMEOUT);
                atomicExch(abort_word(a), 1u);
                return false;
            }
        }
    }
}

// Rows of x ([rows][k] f32, other blocks' writes) into xs in Stage layout, normed when `norm` with
// the gain staged in gs (stage_rows' arithmetic: the row's scale by warp_rms_scale's sums, then
// x s g). Every thread loads its share of x at once (at most PS_STAGE float4s) while warp b takes
// row b's scale straight from L2, so the staging costs one trip to L2.
constexpr int PS_STAGE = 8;
template <typename T, int NB>
TG_DEVICE void flow_stage(const float *x, const float *gs, bool norm, int rows, int k, float eps, float *xs,
                          float *scales, int ctid) {
    const int quads = k / 4, n = NB * quads;
    float4 v[PS_STAGE];
#pragma unroll
    for (int u = 0; u < PS_STAGE; u++) {
        const int i = ctid + u * PS_CTHREADS, b = i / quads, c = i % quads;
        v[u] = (i < n && b < rows) ? __ldcg(reinterpret_cast<const float4 *>(x + (size_t)b * k) + c)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (norm) {
        const int warp = ctid >> 5;
        if (warp < NB) {
            const float sc = warp < rows ? warp_rms_scale_cg(x + (size_t)warp * k, k, eps) : 0.0f;
            if ((ctid & 31) == 0) scales[warp] = sc;
        }
        ConsumerSync::sync();
    }
#pragma unroll
    for (int u = 0; u < PS_STAGE; u++) {
        const int i = ctid + u * PS_CTHREADS, b = i / quads, c = i % quads;
        if (i >= n) continue;
        float4 o = v[u];
        if (norm) {
            const float4 gg = reinterpret_cast<const float4 *>(gs)[c];
            const float sc = scales[b];
            o = make_float4(o.x * sc * gg.x, o.y * sc * gg.y, o.z * sc * gg.z, o.w * sc * gg.w);
        }
        *reinterpret_cast<float4 *>(xs + Stage<T>::index(k, b, 4 * c)) = o;
    }
    ConsumerSync::sync();
}

// A gain ([k] f32, a weight: constant) into shared memory, before the wait it is needed after.
TG_DEVICE void stage_gain(const float *g, int k, float *gs, int ctid) {
    for (int i = ctid; i < k / 4; i += PS_CTHREADS)
        reinterpret_cast<float4 *>(gs)[i] = __ldg(reinterpret_cast<const float4 *>(g) + i);
}

// attention_combine (attention_combine.comp:29-58) as the output projection's staging: every
// head of every row joined from the attention phase's chunk partials straight into xs (Stage
// layout, as flow_stage would stage att [rows][heads hd]). Thread t takes four dimensions of one
// head, loads the head's chunk maxima and sums and its four columns of every chunk's partial output
// in one batch (the first 16 chunks; longer caches continue chunk by chunk), and folds them in
// chunk order as attention_combine_kernel does, so the staged values are its bits. Each block joins
// for itself: one round trip through L2 after the attention phase, instead of a join by one block,
// a store and a second round trip. A spare row stages zeros.
template <typename T, int NB>
TG_DEVICE void flow_stage_join(const PersistArgs &a, int rows, const int (&nch)[PS_ROWS], float *xs, int ctid) {
    constexpr int B = 16;
    const tg_params &p = a.p;
    const int hd = p.head_dim, heads = p.heads, q4 = hd / 4, k = heads * hd;
    const int chunks = attn_chunks(p.capacity);
    for (int i = ctid; i < NB * heads * q4; i += PS_CTHREADS) {
        const int b = i / (heads * q4), h = (i / q4) % heads, d4 = i % q4;
        const int n = b < rows ? nch[b] : 0;
        const float2 *ml = reinterpret_cast<const float2 *>(a.pml) + ((size_t)b * heads + h) * chunks;
        const float4 *o = reinterpret_cast<const float4 *>(a.po) + ((size_t)b * heads + h) * chunks * q4 + d4;
        float2 mv[B];
        float4 ov[B];
#pragma unroll
        for (int c = 0; c < B; c++) {
            mv[c] = c < n ? __ldcg(ml + c) : make_float2(-INFINITY, 0.f);
            ov[c] = c < n ? __ldcg(o + (size_t)c * q4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float m = -INFINITY;
#pragma unroll
        for (int c = 0; c < B; c++)
            if (c < n) m = fmaxf(m, mv[c].x);
        for (int c = B; c < n; c++) m = fmaxf(m, __ldcg(ml + c).x);
        float total = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int c = 0; c < B; c++) {
            if (c >= n) continue;
            const float w = expf(mv[c].x - m);
            total = __fmaf_rn(mv[c].y, w, total);
            acc.x = __fmaf_rn(ov[c].x, w, acc.x);
            acc.y = __fmaf_rn(ov[c].y, w, acc.y);
            acc.z = __fmaf_rn(ov[c].z, w, acc.z);
            acc.w = __fmaf_rn(ov[c].w, w, acc.w);
        }
        for (int c = B; c < n; c++) {
            const float2 v = __ldcg(ml + c);
            const float4 oc = __ldcg(o + (size_t)c * q4);
            const float w = expf(v.x - m);
            total = __fmaf_rn(v.y, w, total);
            acc.x = __fmaf_rn(oc.x, w, acc.x);
            acc.y = __fmaf_rn(oc.y, w, acc.y);
            acc.z = __fmaf_rn(oc.z, w, acc.z);
            acc.w = __fmaf_rn(oc.w, w, acc.w);
        }
        const float4 v = n > 0 ? make_float4(__fdiv_rn(acc.x, total), __fdiv_rn(acc.y, total),
                                             __fdiv_rn(acc.z, total), __fdiv_rn(acc.w, total))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(xs + Stage<T>::index(k, b, 4 * (h * q4 + d4))) = v;
    }
    ConsumerSync::sync();
}

// One weight segment's dot products and epilogues. Warp w takes units w, w + 8, ..., U of them at
// once (their rows' sums interleaved, each in dot_smem's order), and lane u NB + b runs the epilogue
// of the pass's unit u for row b; a residual is loaded before the sums that it waits behind.
template <typename T, int NB, int EPI, int U>
TG_DEVICE void flow_dots(const GemvArgs &ga, const SegRef &seg, int ub, int nu, int k, const float *xs, int rows,
                         int ctid) {
    constexpr int R = EPI == EPI_RESIDUAL ? 1 : 2;
    static_assert(U * NB <= 32, "one lane per (unit, row)");
    const int warp = ctid >> 5, lane = ctid & 31;
    for (int j0 = warp; j0 < nu; j0 += PS_CONSUMERS * U) {
        const int eu = lane / NB, eb = lane % NB, ej = j0 + PS_CONSUMERS * eu;
        const bool mine = eu < U && eb < rows && ej < nu;
        float res = 0.0f;
        if constexpr (EPI == EPI_RESIDUAL)
            if (mine) res = __ldcg(ga.res + (size_t)eb * ga.p.n + ub + ej);
        const T *w[R * U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = min(j0 + PS_CONSUMERS * u, nu - 1);  // past the share: a row whose sums go unused
#pragma unroll
            for (int r = 0; r < R; r++) w[u * R + r] = seg.row<T>(r * nu + j);
        }
        float acc[NB][R * U];
        dot_smem<T, NB, R * U>(w, k, xs, acc);
        float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
            for (int u = 0; u < U; u++) {
                const float s0 = warp_sum(acc[b][u * R]);
                const float s1 = R == 2 ? warp_sum(acc[b][u * R + R - 1]) : s0;
                if (u == eu && b == eb) {
                    y0 = s0;
                    y1 = s1;
                }
            }
        if (mine) {
            if constexpr (EPI == EPI_RESIDUAL) {
                const size_t at = (size_t)eb * ga.p.n + ub + ej;
                ga.out[at] = __fmaf_rn(ga.p.residual_scale, y0, res);
            } else {
                gemv_epilogue<T, EPI>(ga, ub + ej, eb, y0, y1);
            }
        }
    }
}

template <typename T, int NB>
__global__ void __launch_bounds__(PS_THREADS, 1) decode_step_kernel(const __grid_constant__ PersistArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[PS_NBAR];
    // The consumers' release mark: bit 63 an abort, bits 32..62 the segments released, bits 0..31
    // the linear ring end of the last one.
    __shared__ volatile unsigned long long released;
    __shared__ int ok_t;
    __shared__ float scales[PS_ROWS];
    __shared__ int ok_s;
    const tg_params &p = a.p;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows = p.rows;
    const int H = p.hidden;
    const size_t es = sizeof(T);
    unsigned char *ring = smem;
    float *gs = reinterpret_cast<float *>(smem + a.ring);  // [hidden]: the RMSNorm gain in use
    float *xs = gs + H;                                     // [NB][k], Stage layout
    float *work = xs + (size_t)NB * H;                      // attention's working space (past q/k/v's xs)
    if (threadIdx.x == 0) {
        for (int i = 0; i < PS_NBAR; i++) mbar_init(smem_u32(&full[i]), 1);
        released = 0ull;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == PS_CONSUMERS) {
        // Producer: the block's segment of every weight phase of every layer, in the consumers' order.
        uint32_t lin = 0;
        int g = 0;
        bool ok = true;
        for (int l = 0; l < a.layers && ok; l++) {
            for (int wi = 0; wi < 4 && ok; wi++) {
                const WPhase ph = wphase(p, wi);
                int ub, ue;
                share(p, wi, ph.units, ub, ue);
                if (ub >= ue) continue;
                const int nu = ue - ub;
                const uint32_t row_bytes = (uint32_t)(ph.k * es);
                const uint32_t bytes = (uint32_t)nu * ph.R * row_bytes;
                const uint32_t start = ring_place(lin, bytes, row_bytes);
                const uint32_t end = start + bytes;
                // The ring bytes it takes were last used by segments that start before end - ring
                // (all of them released once every segment before it is, or once the released ones
                // reach end - ring), and its barrier by segment g - PS_NBAR.
                if (lane == 0) {
                    const uint64_t t0 = globaltimer();
                    for (uint32_t i = 0;; i++) {
                        const unsigned long long rel = released;
                        if (rel >> 63) {
                            ok = false;
                            break;
                        }
                        const int count = (int)(rel >> 32);
                        if ((count >= g || (uint32_t)rel + a.ring >= end) && count >= g + 1 - PS_NBAR) break;
                        if ((i & 63) == 0) {
                            if (*(volatile uint32_t *)abort_word(a)) {
                                ok = false;
                                break;
                            }
                            if (globaltimer() - t0 > PS_WAIT_NS) {
                                atomicExch(a.err, ERR_WAIT_TIMEOUT);
                                atomicExch(abort_word(a), 1u);
                                ok = false;
                                break;
                            }
                        }
                    }
                    if (ok) {
                        const uint32_t bar = smem_u32(&full[g % PS_NBAR]);
                        mbar_arrive_expect_tx(bar, bytes);
                        const unsigned char *w = a.weights + a.offs[l * 6 + wi];
                        // Rows that follow each other in W go in one copy (unit j's row r at
                        // segment row r nu + j), split in two where it wraps around the ring.
                        for (int r = 0; r < ph.R; r++)
                            for (int j0 = 0; j0 < nu;) {
                                const int row0 = wrow(p, wi, ub + j0, r);
                                int j1 = j0 + 1;
                                while (j1 < nu && wrow(p, wi, ub + j1, r) == row0 + (j1 - j0)) j1++;
                                const uint32_t at = (start + (uint32_t)(r * nu + j0) * row_bytes) % a.ring;
                                const uint32_t n = (uint32_t)(j1 - j0) * row_bytes;
                                const uint32_t first = min(n, a.ring - at);
                                const unsigned char *src = w + (size_t)row0 * row_bytes;
                                bulk_load(smem_u32(ring + at), src, first, bar);
                                if (first < n) bulk_load(smem_u32(ring), src + first, n - first, bar);
                                j0 = j1;
                            }
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (ok) g++;
            }
        }
        // The first layer's weights into L2 for the next step, while this step's last layers finish.
        if (ok && lane == 0 && a.prefetch) {
            for (int wi = 0; wi < 4; wi++) {
                const WPhase ph = wphase(p, wi);
                int ub, ue;
                share(p, wi, ph.units, ub, ue);
                const char *w = reinterpret_cast<const char *>(a.weights + a.offs[wi]);
                for (int r = 0; r < ph.R && ub < ue; r++)
                    for (int j0 = 0; j0 < ue - ub;) {
                        const int row0 = wrow(p, wi, ub + j0, r);
                        int j1 = j0 + 1;
                        while (j1 < ue - ub && wrow(p, wi, ub + j1, r) == row0 + (j1 - j0)) j1++;
                        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(w + (size_t)row0 * ph.k * es),
                                     "r"((uint32_t)((j1 - j0) * ph.k * es))
                                     : "memory");
                        j0 = j1;
                    }
            }
        }
        // Every copy issued has landed before the block ends.
        if (lane == 0)
            for (int s = max(0, g - PS_NBAR); s < g; s++)
                mbar_wait_bounded(smem_u32(&full[s % PS_NBAR]), (s / PS_NBAR) & 1, a.err, 100000000ull);
        return;
    }

    // Consumers.
    const int ctid = threadIdx.x;
    const int G = gridDim.x;
    const int hd = p.head_dim, heads = p.heads, kvh = p.kv_heads, group = heads / kvh;
    const int chunks = attn_chunks(p.capacity);
    uint32_t pos[PS_ROWS], slotw[PS_ROWS];
    int nch[PS_ROWS];
    bool live[PS_ROWS];
    int items = 0;
#pragma unroll
    for (int b = 0; b < PS_ROWS; b++) {
        live[b] = b < rows && placed(a.at, rows, b, p.capacity, p.slots, pos[b], slotw[b]);
        nch[b] = live[b] ? (int)(pos[b] / ATTN_CHUNK) + 1 : 0;
        items += kvh * nch[b];
    }
    uint32_t lin = 0;
    int g = 0;
    bool ok = true;
    // Takes the block's next segment of weight phase wi: waits for it to land, returns its start.
    // One thread waits (bounded); once it has seen the copies land, the phase stays complete until
    // the segment is released, so every thread's own check of it passes at once.
    auto take = [&](int wi, int nu) -> SegRef {
        const WPhase ph = wphase(p, wi);
        const uint32_t row_bytes = (uint32_t)(ph.k * es);
        const uint32_t bytes = (uint32_t)nu * ph.R * row_bytes;
        const uint32_t start = ring_place(lin, bytes, row_bytes);
        const uint32_t bar = smem_u32(&full[g % PS_NBAR]), parity = (g / PS_NBAR) & 1;
        if (ctid == 0) ok_t = ok && mbar_wait_abortable(bar, parity, a);
        ConsumerSync::sync();
        if (!ok_t) ok = false;
        if (ok) mbar_wait_bounded(bar, parity, a.err, 1000000ull);
        return SegRef{ring, start, a.ring, row_bytes};
    };
    auto give = [&]() {
        ConsumerSync::sync();
        if (ctid == 0 && ok) released = ((unsigned long long)(g + 1) << 32) | lin;
        g++;
    };
    const float *x = a.x_in;
    for (int l = 0; l < a.layers; l++) {
        const float *g_in = reinterpret_cast<const float *>(a.weights + a.offs[l * 6 + 4]);
        const float *g_post = reinterpret_cast<const float *>(a.weights + a.offs[l * 6 + 5]);
        T *kc = reinterpret_cast<T *>(a.kcache + (size_t)l * a.cache_layer);
        T *vc = reinterpret_cast<T *>(a.vcache + (size_t)l * a.cache_layer);
        int ub, ue;
        // q, k, v with RoPE and the KV append.
        share(p, 0, wphase(p, 0).units, ub, ue);
        if (ub < ue) {
            stage_gain(g_in, H, gs, ctid);
            if (l > 0 && !wait_phase(a, l - 1, PH_DOWN, ctid, &ok_s)) ok = false;
            flow_stage<T, NB>(x, gs, true, rows, H, p.eps, xs, scales, ctid);
            const SegRef seg = take(0, ue - ub);
            GemvArgs ga{};
            ga.p = p;
            ga.cosv = a.cosv;
            ga.sinv = a.sinv;
            ga.at = a.at;
            ga.q = a.q;
            ga.kc = kc;
            ga.vc = vc;
            if (ok) flow_dots<T, NB, EPI_QKV_ROPE, 1>(ga, seg, ub, ue - ub, H, xs, rows, ctid);
            give();
        }
        if (!ok) break;
        arrive(a, l, PH_QKV, ctid);
        // Attention: items (row, kv head, chunk) dealt from the last block down. The keys and
        // values before each row's position are staged before the wait on q/k/v.
        {
            bool waited = false;
            auto wait_qkv = [&]() {
                if (!waited && !wait_phase(a, l, PH_QKV, ctid, &ok_s)) ok = false;
                waited = true;
            };
            for (int it = G - 1 - (int)blockIdx.x, first = it; it < items; it += G) {
                // Item `it`: rows in order, then kv heads, then chunks.
                int b = 0, rest = it;
                while (b < PS_ROWS - 1 && rest >= kvh * nch[b]) {
                    rest -= kvh * nch[b];
                    b++;
                }
                const int kv = rest / nch[b], c = rest % nch[b];
                const uint32_t pb = pos[b], sb = slotw[b];
                if (it != first) ConsumerSync::sync();  // the previous item's reads of `work` are done
                const size_t head0 = (size_t)b * heads + kv * group;
                attention_chunk<T, ConsumerSync>(p, a.q, kc, vc, b, kv, c, pb, sb, a.po + (head0 * chunks + c) * hd,
                                                 (size_t)chunks * hd, a.pml + (head0 * chunks + c) * 2,
                                                 (size_t)chunks * 2, work, ctid, PS_CTHREADS, wait_qkv);
            }
        }
        if (!ok) break;
        arrive(a, l, PH_ATT, ctid);
        // The join of every head's chunks (each block its own), then the output projection with the
        // residual.
        share(p, 1, wphase(p, 1).units, ub, ue);
        if (ub < ue) {
            if (!wait_phase(a, l, PH_ATT, ctid, &ok_s)) ok = false;
            flow_stage_join<T, NB>(a, rows, nch, xs, ctid);
            const SegRef seg = take(1, ue - ub);
            GemvArgs ga{};
            ga.p = p;
            ga.p.n = H;
            ga.res = x;
            ga.out = a.mid;
            if (ok) flow_dots<T, NB, EPI_RESIDUAL, 1>(ga, seg, ub, ue - ub, heads * hd, xs, rows, ctid);
            give();
        }
        if (!ok) break;
        arrive(a, l, PH_O, ctid);
        // gate/up with the post-attention norm, SiLU-mul.
        share(p, 2, wphase(p, 2).units, ub, ue);
        if (ub < ue) {
            stage_gain(g_post, H, gs, ctid);
            if (!wait_phase(a, l, PH_O, ctid, &ok_s)) ok = false;
            flow_stage<T, NB>(a.mid, gs, true, rows, H, p.eps, xs, scales, ctid);
            const SegRef seg = take(2, ue - ub);
            GemvArgs ga{};
            ga.p = p;
            ga.out = a.mlp;
            if (ok) flow_dots<T, NB, EPI_GATE_UP, 4>(ga, seg, ub, ue - ub, H, xs, rows, ctid);
            give();
        }
        if (!ok) break;
        arrive(a, l, PH_GU, ctid);
        // down with the residual.
        share(p, 3, wphase(p, 3).units, ub, ue);
        if (ub < ue) {
            if (!wait_phase(a, l, PH_GU, ctid, &ok_s)) ok = false;
            flow_stage<T, NB>(a.mlp, nullptr, false, rows, p.inner, p.eps, xs, scales, ctid);
            const SegRef seg = take(3, ue - ub);
            GemvArgs ga{};
            ga.p = p;
            ga.p.n = H;
            ga.res = a.mid;
            ga.out = a.h;
            if (ok) flow_dots<T, NB, EPI_RESIDUAL, 1>(ga, seg, ub, ue - ub, p.inner, xs, rows, ctid);
            give();
        }
        if (!ok) break;
        arrive(a, l, PH_DOWN, ctid);
        x = a.h;
    }
    if (ok && blockIdx.x == 0 && wait_phase(a, a.layers - 1, PH_DOWN, ctid, &ok_s)) {
        // The final norm (rmsnorm.comp), in f32.
        const float *gf = reinterpret_cast<const float *>(a.weights + a.final_norm);
        float *raw = xs;  // [rows][hidden]
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
    // An aborted step tells the producer to stop issuing copies (it then waits for those in flight).
    if (!ok && ctid == 0) {
        atomicExch(abort_word(a), 1u);
        released = released | (1ull << 63);
    }
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
                                           const float *pml, void *out, cudaStream_t s, bool out_bf16) {
    dim3 grid(p.heads, p.rows);
    const int threads = p.head_dim < 128 ? p.head_dim : 128;
    const size_t smem = (size_t)3 * (attn_chunks(p.capacity)) * sizeof(float);
    if (out_bf16)
        return launch_pdl(attention_combine_kernel<bf16>, grid, dim3(threads), smem, s, p, at, po, pml, (bf16 *)out, chunk);
    return launch_pdl(attention_combine_kernel<float>, grid, dim3(threads), smem, s, p, at, po, pml, (float *)out, chunk);
}

cudaError_t launch_attention_combine(const tg_params &p, const uint32_t *at, const float *po,
                                     const float *pml, void *out, cudaStream_t s) {
    return launch_attention_combine_chunk(p, ATTN_CHUNK, at, po, pml, out, s);
}

// The persistent step over a decoder's buffers: one block per SM, the ring as large as shared
// memory allows beside the block's staging space. Returns cudaErrorNotSupported for batches or
// shapes it does not take (more than PS_ROWS rows; a block's share of a projection larger than
// the ring).
size_t decode_step_flag_bytes(int layers) {
    return ((size_t)layers * PS_PHASES * PS_NCOUNT + 1) * sizeof(uint32_t);
}

template <typename T, int NB>
static cudaError_t launch_step_t(const PersistArgs &a, int sms, size_t smem, size_t flag_bytes, cudaStream_t s) {
    auto kern = decode_step_kernel<T, NB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, PS_THREADS, smem)) != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    if ((e = cudaMemsetAsync(a.flags, 0, flag_bytes, s)) != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(PS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_decode_step(const DecodeStep &d, int sm_count, cudaStream_t s) {
    const tg_params &p = d.p;
    if (p.rows == 0 || p.rows > (uint32_t)PS_ROWS) return cudaErrorNotSupported;
    const int NB = p.rows == 1 ? 1 : 2;
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
    a.att = d.att;
    a.out = d.out;
    a.po = d.po;
    a.pml = d.pml;
    a.kcache = d.kcache;
    a.vcache = d.vcache;
    a.cache_layer = d.cache_layer;
    a.flags = d.sync;
    a.err = d.err;
    a.prefetch = 1;
    // The largest share of a projection one block streams at once.
    const uint64_t units[4] = {(uint64_t)(p.heads + 2 * p.kv_heads) * p.head_dim / 2, p.hidden, p.inner, p.hidden};
    const uint64_t ks[4] = {p.hidden, (uint64_t)p.heads * p.head_dim, p.hidden, p.inner};
    const uint64_t rs[4] = {2, 1, 2, 1};
    uint64_t seg = 0;
    for (int i = 0; i < 4; i++) {
        const uint64_t blocks = (uint64_t)phase_blocks(p, i, sm_count);
        seg = std::max(seg, (units[i] + blocks - 1) / blocks * rs[i] * ks[i] * es);
    }
    // The gain [hidden], then xs [NB][kmax] with attention's working space past q/k/v's part of it.
    const uint64_t kmax = std::max({(uint64_t)p.hidden, (uint64_t)p.inner, (uint64_t)p.heads * p.head_dim});
    if ((uint64_t)NB * kmax > (uint64_t)4 * PS_STAGE * PS_CTHREADS) return cudaErrorNotSupported;
    const uint64_t scratch =
        4 * (uint64_t)p.hidden + std::max<uint64_t>(4 * NB * kmax, 4 * (uint64_t)NB * p.hidden + attention_smem(p));
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    const int64_t room = (int64_t)optin - 1024 - (int64_t)scratch;  // 1 KiB for the static barriers
    if (room < (int64_t)seg) return cudaErrorNotSupported;
    const int64_t row_max = (int64_t)(kmax * es);
    a.ring = (uint32_t)(room / row_max * row_max);  // a multiple of every phase's row length
    if (a.ring < seg) return cudaErrorNotSupported;
    const size_t smem = a.ring + scratch;
    const size_t flag_bytes = decode_step_flag_bytes(d.layers);
    if (p.dtype == TG_BF16)
        return NB == 1 ? launch_step_t<bf16, 1>(a, sm_count, smem, flag_bytes, s)
                       : launch_step_t<bf16, 2>(a, sm_count, smem, flag_bytes, s);
    return NB == 1 ? launch_step_t<float, 1>(a, sm_count, smem, flag_bytes, s)
                   : launch_step_t<float, 2>(a, sm_count, smem, flag_bytes, s);
}

cudaError_t launch_stream_read(const tg_params &p, const uint32_t *data, uint32_t *out,
                               cudaStream_t s, int sm_count) {
    const uint64_t n = (uint64_t)p.k / 4;  // p.k words, 4 to a uint4
    int blocks = sm_count * 8;
    stream_read_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const uint4 *>(data), n, out);
    return cudaGetLastError();
}

}  // namespace tg
