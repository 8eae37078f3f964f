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
#include "tg_common.cuh"
#include "tg_internal.h"

namespace tg {

constexpr int GEMV_WARPS = 4;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;

// Programmatic dependent launch: a kernel lets the next one start as soon as all of its blocks
// are running (launch_dependents), and waits for the one before it to finish and its writes to
// land (wait) only where it first reads what that one wrote. The GEMVs load their weights -
// constants - before the wait, so the weight stream runs across kernel boundaries. Every block
// waits before it ends, so a kernel never finishes ahead of the one before it. Both are no-ops
// in a launch without the programmatic attribute.
TG_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
TG_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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

// Writes rows b0 .. b0 + NB - 1 of x ([rows][k] f32) into xs, each normed by RMSNorm with gain g
// when g is given (kernels/glsl/norm.glsl:47-53: x times its scale times the gain), rows past
// `rows` as zero.
template <typename T, int NB>
__device__ void stage_rows(const float *__restrict__ x, const float *__restrict__ g, int rows,
                           int b0, int k, float eps, float *xs) {
    __shared__ float scales[NB];
    const int warp = threadIdx.x >> 5;
    if (g) {
        for (int b = warp; b < NB; b += GEMV_WARPS) {
            float sc = 0.0f;
            if (b0 + b < rows) sc = warp_rms_scale(x + (size_t)(b0 + b) * k, k, eps);
            if ((threadIdx.x & 31) == 0) scales[b] = sc;
        }
        __syncthreads();
    }
    const int quads = k / 4;
    for (int i = threadIdx.x; i < NB * quads; i += blockDim.x) {
        const int b = i / quads, c = i % quads;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b0 + b < rows) v = reinterpret_cast<const float4 *>(x + (size_t)(b0 + b) * k)[c];
        if (g) {
            const float4 gg = reinterpret_cast<const float4 *>(g)[c];
            const float s = scales[b];
            v = make_float4(v.x * s * gg.x, v.y * s * gg.y, v.z * s * gg.z, v.w * s * gg.w);
        }
        // Four consecutive elements 4c .. 4c + 3 stay together in either layout.
        *reinterpret_cast<float4 *>(xs + Stage<T>::index(k, b, 4 * c)) = v;
    }
    __syncthreads();
}

// The first AHEAD vectors of each of a warp's rows, loaded before the kernel waits on the one
// before it.
template <typename T, int R, int AHEAD>
struct Prefetch {
    typename Vec<T>::Raw v[AHEAD][R];
};

template <typename T, int R, int AHEAD>
TG_DEVICE void prefetch_rows(const T *__restrict__ w, const int (&rows)[R], int k, Prefetch<T, R, AHEAD> &pf) {
    using Raw = typename Vec<T>::Raw;
    const int lane = threadIdx.x & 31, nvec = k / Vec<T>::N;
#pragma unroll
    for (int t = 0; t < AHEAD; t++) {
        const int j = t * 32 + lane;
#pragma unroll
        for (int r = 0; r < R; r++)
            pf.v[t][r] = j < nvec ? ld_stream(reinterpret_cast<const Raw *>(w + (size_t)rows[r] * k) + j) : Raw{};
    }
}

// acc[b][r] = W[rows[r]] . xs[b] for the warp: lane l takes the 16-byte vectors l, l + 32, ... of
// each row in order, each element by one fused multiply-add (the lanes are joined by the caller).
// The first AHEAD steps come from `pf`; the rest are loaded AHEAD steps at a time.
template <typename T, int NB, int R, int AHEAD>
TG_DEVICE void dot_rows(const T *__restrict__ w, const int (&rows)[R], int k, const float *xs,
                        const Prefetch<T, R, AHEAD> &pf, float (&acc)[NB][R]) {
    using VT = Vec<T>;
    using Raw = typename VT::Raw;
    constexpr int V = VT::N;
    const int lane = threadIdx.x & 31;
    const int nvec = k / V;
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int r = 0; r < R; r++) acc[b][r] = 0.0f;
    for (int j0 = 0; j0 < nvec; j0 += 32 * AHEAD) {
        Raw wv[AHEAD][R];
        if (j0 == 0) {
#pragma unroll
            for (int t = 0; t < AHEAD; t++)
#pragma unroll
                for (int r = 0; r < R; r++) wv[t][r] = pf.v[t][r];
        } else {
#pragma unroll
            for (int t = 0; t < AHEAD; t++) {
                const int j = j0 + t * 32 + lane;
#pragma unroll
                for (int r = 0; r < R; r++)
                    wv[t][r] = j < nvec ? ld_stream(reinterpret_cast<const Raw *>(w + (size_t)rows[r] * k) + j) : Raw{};
            }
        }
#pragma unroll
        for (int t = 0; t < AHEAD; t++) {
            const int j = j0 + t * 32 + lane;
            if (j >= nvec) break;
            float wf[R][V];
#pragma unroll
            for (int r = 0; r < R; r++) VT::unpack(wv[t][r], wf[r]);
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
}

template <int NB>
__device__ __forceinline__ float pick(const float (&v)[NB], int i) {
    float out = 0.0f;
#pragma unroll
    for (int b = 0; b < NB; b++)
        if (b == i) out = v[b];
    return out;
}

constexpr int AHEAD_PAIRS = 4;  // vectors per row loaded ahead by the two-row GEMVs
constexpr int AHEAD_ROW = 8;    // and by the one-row GEMV

// gemv_qkv_rope.comp:51-107: q, k, v = W RMSNorm(x); q and k rotated at the row's position; k, v
// into the row's slot there. A warp takes the pair of rows (i, i + hd/2) of one head, the pair
// RoPE turns together. q is kept in f32. Grid: [pairs / GEMV_WARPS, ceil(rows / NB)].
template <typename T, int NB>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_qkv_rope_kernel(tg_params p, const float *__restrict__ x, const float *__restrict__ g,
                         const T *__restrict__ w, const float *__restrict__ cosv,
                         const float *__restrict__ sinv, const uint32_t *__restrict__ at,
                         float *__restrict__ q, T *__restrict__ kc, T *__restrict__ vc) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *xs = reinterpret_cast<float *>(smem);
    pdl_launch_dependents();
    const int k = p.hidden, hd = p.head_dim, half = hd / 2;
    const int heads = p.heads, kvh = p.kv_heads;
    const int b0 = blockIdx.y * NB;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = blockIdx.x * GEMV_WARPS + warp;
    const bool active = pair < (heads + 2 * kvh) * half;
    const int head = pair / half, i = pair % half;
    const int rows[2] = {active ? head * hd + i : 0, active ? head * hd + i + half : 0};
    Prefetch<T, 2, AHEAD_PAIRS> pf;
    prefetch_rows<T, 2, AHEAD_PAIRS>(w, rows, k, pf);
    pdl_wait();
    stage_rows<T, NB>(x, g, p.rows, b0, k, p.eps, xs);
    if (!active) return;
    float acc[NB][2];
    dot_rows<T, NB, 2, AHEAD_PAIRS>(w, rows, k, xs, pf, acc);
    float a[NB], c[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
        a[b] = warp_sum(acc[b][0]);
        c[b] = warp_sum(acc[b][1]);
    }
    if (lane >= NB || b0 + lane >= (int)p.rows) return;
    const int b = b0 + lane;
    uint32_t pos, slot;
    if (!placed(at, p.rows, b, p.capacity, p.slots, pos, slot)) return;
    float ra = pick<NB>(a, lane), rc = pick<NB>(c, lane);
    if (head >= heads + kvh) {
        const size_t to = (((size_t)slot * kvh + (head - heads - kvh)) * p.capacity + pos) * hd + i;
        vc[to] = from_f32<T>(ra);
        vc[to + half] = from_f32<T>(rc);
        return;
    }
    if (p.rope) {
        // As upstream: x cos + rotate_half(x) sin (gemv_qkv_rope.comp:85-90).
        const float co = cosv[(size_t)pos * half + i], si = sinv[(size_t)pos * half + i];
        const float na = __fmaf_rn(ra, co, -__fmul_rn(rc, si));
        const float nc = __fmaf_rn(rc, co, __fmul_rn(ra, si));
        ra = na;
        rc = nc;
    }
    if (head < heads) {
        const size_t to = ((size_t)b * heads + head) * hd + i;
        q[to] = ra;
        q[to + half] = rc;
    } else {
        const size_t to = (((size_t)slot * kvh + (head - heads)) * p.capacity + pos) * hd + i;
        kc[to] = from_f32<T>(ra);
        kc[to + half] = from_f32<T>(rc);
    }
}

// gemv_residual.comp:28-45: out = residual + s W x, a warp to an output row; x in f32.
template <typename T, int NB>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_residual_kernel(tg_params p, const float *__restrict__ x, const T *__restrict__ w,
                         const float *__restrict__ res, float *__restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *xs = reinterpret_cast<float *>(smem);
    pdl_launch_dependents();
    const int k = p.k, n = p.n;
    const int b0 = blockIdx.y * NB;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * GEMV_WARPS + warp;
    const bool active = row < n;
    const int rows[1] = {active ? row : 0};
    Prefetch<T, 1, AHEAD_ROW> pf;
    prefetch_rows<T, 1, AHEAD_ROW>(w, rows, k, pf);
    pdl_wait();
    stage_rows<T, NB>(x, nullptr, p.rows, b0, k, 0.0f, xs);
    if (!active) return;
    float acc[NB][1];
    dot_rows<T, NB, 1, AHEAD_ROW>(w, rows, k, xs, pf, acc);
    float y[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) y[b] = warp_sum(acc[b][0]);
    if (lane >= NB || b0 + lane >= (int)p.rows) return;
    const size_t at = (size_t)(b0 + lane) * n + row;
    out[at] = __fmaf_rn(p.residual_scale, pick<NB>(y, lane), res[at]);
}

// gemv_gate_up.comp:31-52: RMSNorm(x) with the post-attention gain, then gate row i and up row i
// (rows i and inner + i of W) by one warp, out = SiLU(gate) up, in f32.
template <typename T, int NB>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_gate_up_kernel(tg_params p, const float *__restrict__ x, const float *__restrict__ g,
                        const T *__restrict__ w, float *__restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *xs = reinterpret_cast<float *>(smem);
    pdl_launch_dependents();
    const int k = p.hidden, inner = p.inner;
    const int b0 = blockIdx.y * NB;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * GEMV_WARPS + warp;
    const bool active = i < inner;
    const int rows[2] = {active ? i : 0, active ? inner + i : 0};
    Prefetch<T, 2, AHEAD_PAIRS> pf;
    prefetch_rows<T, 2, AHEAD_PAIRS>(w, rows, k, pf);
    pdl_wait();
    stage_rows<T, NB>(x, g, p.rows, b0, k, p.eps, xs);
    if (!active) return;
    float acc[NB][2];
    dot_rows<T, NB, 2, AHEAD_PAIRS>(w, rows, k, xs, pf, acc);
    float gate[NB], up[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
        gate[b] = warp_sum(acc[b][0]);
        up[b] = warp_sum(acc[b][1]);
    }
    if (lane >= NB || b0 + lane >= (int)p.rows) return;
    out[(size_t)(b0 + lane) * inner + i] = silu_mul(pick<NB>(gate, lane), pick<NB>(up, lane));
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

// attention_split.comp:52-112: block (c, h, b) scores the GROUP query heads that kv head h serves
// against ATTN_CHUNK positions from c ATTN_CHUNK of row b's slot, masked past the row's position,
// and writes each head's chunk softmax unnormalised with its maximum and sum. A chunk that starts
// past the position writes nothing, nor does a spare row. The keys and values before the row's
// position were written by earlier steps, so they are loaded before waiting on qkv_rope; the
// position's own, and q, after.
template <typename T>
__global__ void __launch_bounds__(128)
    attention_split_kernel(tg_params p, const float *__restrict__ q, const T *__restrict__ kc,
                           const T *__restrict__ vc, const uint32_t *__restrict__ at,
                           float *__restrict__ po, float *__restrict__ pml) {
    constexpr int C = ATTN_CHUNK;
    using VT = Vec<T>;
    using Raw = typename VT::Raw;
    constexpr int V = VT::N;
    extern __shared__ __align__(16) unsigned char smem[];
    pdl_launch_dependents();
    const int hd = p.head_dim, heads = p.heads, kvh = p.kv_heads, group = heads / kvh;
    const int c = blockIdx.x, kv = blockIdx.y, b = blockIdx.z;
    const int start = c * C;
    uint32_t pos, slot;
    if (!placed(at, p.rows, b, p.capacity, p.slots, pos, slot) || start > (int)pos) {
        pdl_wait();
        return;
    }
    float *qs = reinterpret_cast<float *>(smem);   // [group][hd]
    float *ks = qs + group * hd;                   // [C][hd + 1]
    float *vs = ks + C * (hd + 1);                 // [C][hd]
    float *ps = vs + C * hd;                       // [group][C]
    const int tid = threadIdx.x;
    const int first_head = kv * group;
    const size_t base = (((size_t)slot * kvh + kv) * p.capacity + start) * hd;
    const Raw *ksrc = reinterpret_cast<const Raw *>(kc + base);
    const Raw *vsrc = reinterpret_cast<const Raw *>(vc + base);
    const int per_row = hd / V;
    // pass 0: positions before the row's (earlier steps wrote them); pass 1: the row's own.
    for (int pass = 0; pass < 2; pass++) {
        if (pass == 1) pdl_wait();
        for (int i = tid; i < C * per_row; i += blockDim.x) {
            const int pp = i / per_row, j = i % per_row;
            const int at_pos = start + pp;
            if ((pass == 0) != (at_pos < (int)pos)) continue;
            float kf[V], vf[V];
            if (at_pos <= (int)pos) {
                VT::unpack(ksrc[i], kf);
                VT::unpack(vsrc[i], vf);
            } else {
#pragma unroll
                for (int e = 0; e < V; e++) kf[e] = vf[e] = 0.0f;
            }
#pragma unroll
            for (int e = 0; e < V; e++) {
                ks[pp * (hd + 1) + j * V + e] = kf[e];
                vs[pp * hd + j * V + e] = vf[e];
            }
        }
    }
    {
        const float4 *src = reinterpret_cast<const float4 *>(q + ((size_t)b * heads + first_head) * hd);
        for (int i = tid; i < group * hd / 4; i += blockDim.x) reinterpret_cast<float4 *>(qs)[i] = src[i];
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf((float)hd);
    for (int i = tid; i < group * C; i += blockDim.x) {
        const int h = i / C, pp = i % C;
        float s = 0.0f;
        for (int d = 0; d < hd; d++) s = __fmaf_rn(qs[h * hd + d], ks[pp * (hd + 1) + d], s);
        ps[i] = (start + pp <= (int)pos) ? s * scale : -INFINITY;
    }
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31;
    const int chunks = p.capacity / C;
    for (int h = warp; h < group; h += blockDim.x / 32) {
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
            float *ml = pml + (((size_t)b * heads + first_head + h) * chunks + c) * 2;
            ml[0] = m;
            ml[1] = l;
        }
    }
    __syncthreads();
    for (int i = tid; i < group * hd; i += blockDim.x) {
        const int h = i / hd, d = i % hd;
        float acc = 0.0f;
        for (int pp = 0; pp < C; pp++) acc = __fmaf_rn(ps[h * C + pp], vs[pp * hd + d], acc);
        po[(((size_t)b * heads + first_head + h) * chunks + c) * hd + d] = acc;
    }
}

// attention_combine.comp:29-58: joins chunks 0 .. pos / ATTN_CHUNK of each (row, head) in order:
// their largest maximum, the rescaled sums, and the division; out in f32.
__global__ void __launch_bounds__(128)
    attention_combine_kernel(tg_params p, const uint32_t *__restrict__ at,
                             const float *__restrict__ po, const float *__restrict__ pml,
                             float *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, b = blockIdx.y, hd = p.head_dim;
    uint32_t pos, slot;
    if (!placed(at, p.rows, b, p.capacity, p.slots, pos, slot)) return;
    const int chunks = p.capacity / ATTN_CHUNK;
    const int n = pos / ATTN_CHUNK + 1;
    const float *ml = pml + ((size_t)b * p.heads + h) * chunks * 2;
    const float *o = po + ((size_t)b * p.heads + h) * chunks * hd;
    float m = -INFINITY;
    for (int c = 0; c < n; c++) m = fmaxf(m, ml[2 * c]);
    float total = 0.0f;
    for (int c = 0; c < n; c++) total = __fmaf_rn(ml[2 * c + 1], expf(ml[2 * c] - m), total);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.0f;
        for (int c = 0; c < n; c++) acc = __fmaf_rn(o[(size_t)c * hd + d], expf(ml[2 * c] - m), acc);
        out[((size_t)b * p.heads + h) * hd + d] = __fdiv_rn(acc, total);
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

// The rows of a batch a GEMV block takes: up to 8, fewer when their vectors of k would not fit in
// `limit` bytes of shared memory. What a block takes never changes what is summed.
static int rows_per_block(uint32_t rows, uint32_t k, size_t elem = 4, size_t limit = 160 * 1024) {
    int nb = 8;
    while (nb > 1 && ((uint32_t)nb / 2 >= rows || nb * k * elem > limit)) nb /= 2;
    return nb;
}

template <typename F>
static cudaError_t with_smem(F kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// Launches `kern` with the programmatic-stream-serialization attribute, so that in a stream (or a
// graph captured from one) it may start while the kernel before it finishes (see pdl_wait).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

#define TG_DISPATCH_NB(NB_VAR, ...)                           \
    switch (NB_VAR) {                                         \
        case 1: { constexpr int NB = 1; __VA_ARGS__; } break;  \
        case 2: { constexpr int NB = 2; __VA_ARGS__; } break;  \
        case 4: { constexpr int NB = 4; __VA_ARGS__; } break;  \
        default: { constexpr int NB = 8; __VA_ARGS__; } break; \
    }

template <typename T>
static cudaError_t qkv_rope_t(const tg_params &p, const float *x, const float *g, const void *w,
                              const float *cs, const float *sn, const uint32_t *at, void *q,
                              void *kc, void *vc, cudaStream_t s) {
    const int nb = rows_per_block(p.rows, p.hidden);
    const uint32_t pairs = (p.heads + 2 * p.kv_heads) * p.head_dim / 2;
    dim3 grid((pairs + GEMV_WARPS - 1) / GEMV_WARPS, (p.rows + nb - 1) / nb);
    cudaError_t e = cudaSuccess;
    TG_DISPATCH_NB(nb, {
        const size_t smem = (size_t)NB * p.hidden * 4;
        auto kern = gemv_qkv_rope_kernel<T, NB>;
        if ((e = with_smem(kern, smem)) != cudaSuccess) return e;
        e = launch_pdl(kern, grid, dim3(GEMV_THREADS), smem, s, p, x, g, (const T *)w, cs, sn, at, (float *)q,
                       (T *)kc, (T *)vc);
    });
    return e;
}

cudaError_t launch_gemv_qkv_rope(const tg_params &p, const float *x, const float *g,
                                 const void *w, const float *cs, const float *sn,
                                 const uint32_t *at, void *q, void *kc, void *vc, cudaStream_t s) {
    return p.dtype == TG_BF16 ? qkv_rope_t<bf16>(p, x, g, w, cs, sn, at, q, kc, vc, s)
                              : qkv_rope_t<float>(p, x, g, w, cs, sn, at, q, kc, vc, s);
}

template <typename T>
static cudaError_t residual_t(const tg_params &p, const void *x, const void *w, const float *res,
                              float *out, cudaStream_t s) {
    const int nb = rows_per_block(p.rows, p.k);
    dim3 grid((p.n + GEMV_WARPS - 1) / GEMV_WARPS, (p.rows + nb - 1) / nb);
    cudaError_t e = cudaSuccess;
    TG_DISPATCH_NB(nb, {
        const size_t smem = (size_t)NB * p.k * 4;
        auto kern = gemv_residual_kernel<T, NB>;
        if ((e = with_smem(kern, smem)) != cudaSuccess) return e;
        e = launch_pdl(kern, grid, dim3(GEMV_THREADS), smem, s, p, (const float *)x, (const T *)w, res, out);
    });
    return e;
}

cudaError_t launch_gemv_residual(const tg_params &p, const void *x, const void *w,
                                 const float *res, float *out, cudaStream_t s) {
    return p.dtype == TG_BF16 ? residual_t<bf16>(p, x, w, res, out, s)
                              : residual_t<float>(p, x, w, res, out, s);
}

template <typename T>
static cudaError_t gate_up_t(const tg_params &p, const float *x, const float *g, const void *w,
                             void *out, cudaStream_t s) {
    const int nb = rows_per_block(p.rows, p.hidden);
    dim3 grid((p.inner + GEMV_WARPS - 1) / GEMV_WARPS, (p.rows + nb - 1) / nb);
    cudaError_t e = cudaSuccess;
    TG_DISPATCH_NB(nb, {
        const size_t smem = (size_t)NB * p.hidden * 4;
        auto kern = gemv_gate_up_kernel<T, NB>;
        if ((e = with_smem(kern, smem)) != cudaSuccess) return e;
        e = launch_pdl(kern, grid, dim3(GEMV_THREADS), smem, s, p, x, g, (const T *)w, (float *)out);
    });
    return e;
}

cudaError_t launch_gemv_gate_up(const tg_params &p, const float *x, const float *g,
                                const void *w, void *out, cudaStream_t s) {
    return p.dtype == TG_BF16 ? gate_up_t<bf16>(p, x, g, w, out, s)
                              : gate_up_t<float>(p, x, g, w, out, s);
}

cudaError_t launch_rmsnorm(const tg_params &p, const float *x, const float *g, float *out,
                           cudaStream_t s) {
    return launch_pdl(rmsnorm_kernel, dim3((p.rows + 3) / 4), dim3(128), 0, s, p, x, g, out);
}

static size_t split_smem(const tg_params &p) {
    const size_t group = p.heads / p.kv_heads, hd = p.head_dim, C = ATTN_CHUNK;
    return sizeof(float) * (group * hd + C * (hd + 1) + C * hd + group * C);
}

template <typename T>
static cudaError_t split_t(const tg_params &p, const void *q, const void *kc, const void *vc,
                           const uint32_t *at, float *po, float *pml, cudaStream_t s) {
    const size_t smem = split_smem(p);
    auto kern = attention_split_kernel<T>;
    cudaError_t e = with_smem(kern, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(p.capacity / ATTN_CHUNK, p.kv_heads, p.rows);
    return launch_pdl(kern, grid, dim3(128), smem, s, p, (const float *)q, (const T *)kc, (const T *)vc, at, po, pml);
}

cudaError_t launch_attention_split(const tg_params &p, const void *q, const void *kc,
                                   const void *vc, const uint32_t *at, float *po, float *pml,
                                   cudaStream_t s) {
    return p.dtype == TG_BF16 ? split_t<bf16>(p, q, kc, vc, at, po, pml, s)
                              : split_t<float>(p, q, kc, vc, at, po, pml, s);
}

cudaError_t launch_attention_combine(const tg_params &p, const uint32_t *at, const float *po,
                                     const float *pml, void *out, cudaStream_t s) {
    dim3 grid(p.heads, p.rows);
    const int threads = p.head_dim < 128 ? p.head_dim : 128;
    return launch_pdl(attention_combine_kernel, grid, dim3(threads), 0, s, p, at, po, pml, (float *)out);
}

cudaError_t launch_stream_read(const tg_params &p, const uint32_t *data, uint32_t *out,
                               cudaStream_t s, int sm_count) {
    const uint64_t n = (uint64_t)p.k / 4;  // p.k words, 4 to a uint4
    int blocks = sm_count * 8;
    stream_read_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const uint4 *>(data), n, out);
    return cudaGetLastError();
}

}  // namespace tg
