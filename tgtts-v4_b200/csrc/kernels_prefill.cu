// The prefill's row kernels, around its projection GEMMs: the first input norm, RoPE with the KV
// append, causal GQA attention over the slot's cache, the residual add with the next norm, and
// SiLU-mul. They replace kernels/glsl/{norm_rows,rope_rows,attention_rows,add_norm_rows,
// silu_mul_rows}.comp. Rows carry placement words like the decode step's (a position, then a
// slot): a row placed past the cache is padding, which writes no cache and attends to nothing.
#include "tg_common.cuh"
#include "tg_internal.h"

namespace tg {

// norm_rows.comp: out = RMSNorm(x) g, rounded to T; a warp to a row.
template <typename T>
__global__ void __launch_bounds__(128)
    norm_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ x,
                     const float *__restrict__ g, T *__restrict__ out) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= (int)p.rows) return;
    const int k = p.hidden;
    const float *xr = x + (size_t)row * k;
    const float s = warp_rms_scale(xr, k, p.eps);
    for (int c = lane; c < k / 4; c += 32) {
        const float4 v = reinterpret_cast<const float4 *>(xr)[c];
        const float4 gg = reinterpret_cast<const float4 *>(g)[c];
        T *o = out + (size_t)row * k + 4 * c;
        o[0] = from_f32<T>(v.x * s * gg.x);
        o[1] = from_f32<T>(v.y * s * gg.y);
        o[2] = from_f32<T>(v.z * s * gg.z);
        o[3] = from_f32<T>(v.w * s * gg.w);
    }
}

// add_norm_rows.comp:21-45: sum = residual + s c in f32, normed = RMSNorm(sum) g (from the f32
// sum), rounded to T, or kept in f32 for the final norm; a warp to a row.
template <typename T, bool NORMED_F32>
__global__ void __launch_bounds__(128)
    add_norm_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ c,
                         const float *__restrict__ res, const float *__restrict__ g,
                         float *__restrict__ sum, void *__restrict__ normed) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= (int)p.rows) return;
    const int k = p.hidden;
    const size_t base = (size_t)row * k;
    const float sc = p.residual_scale;
    for (int q = lane; q < k / 4; q += 32) {
        const float4 cv = reinterpret_cast<const float4 *>(c + base)[q];
        const float4 rv = reinterpret_cast<const float4 *>(res + base)[q];
        reinterpret_cast<float4 *>(sum + base)[q] =
            make_float4(__fmaf_rn(sc, cv.x, rv.x), __fmaf_rn(sc, cv.y, rv.y),
                        __fmaf_rn(sc, cv.z, rv.z), __fmaf_rn(sc, cv.w, rv.w));
    }
    __syncwarp();
    const float s = warp_rms_scale(sum + base, k, p.eps);
    for (int q = lane; q < k / 4; q += 32) {
        const float4 v = reinterpret_cast<const float4 *>(sum + base)[q];
        const float4 gg = reinterpret_cast<const float4 *>(g)[q];
        const float o[4] = {v.x * s * gg.x, v.y * s * gg.y, v.z * s * gg.z, v.w * s * gg.w};
        if (NORMED_F32) {
            reinterpret_cast<float4 *>(static_cast<float *>(normed) + base)[q] =
                make_float4(o[0], o[1], o[2], o[3]);
        } else {
            T *n = static_cast<T *>(normed) + base + 4 * q;
#pragma unroll
            for (int e = 0; e < 4; e++) n[e] = from_f32<T>(o[e]);
        }
    }
}

// rope_rows.comp:33-70: from the f32 q/k/v projection of each row, q and k rotated at the row's
// position, q stored, k and v written into the row's slot there. A thread to a pair (i, i + hd/2)
// of a head.
template <typename T>
__global__ void __launch_bounds__(256)
    rope_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ c,
                     const float *__restrict__ cosv, const float *__restrict__ sinv,
                     T *__restrict__ q, T *__restrict__ kc, T *__restrict__ vc) {
    const int row = blockIdx.x;
    uint32_t pos, slot;
    if (!placed(at, p.rows, row, p.capacity, p.slots, pos, slot)) return;
    const int hd = p.head_dim, half = hd / 2, heads = p.heads, kvh = p.kv_heads;
    const int width = (heads + 2 * kvh) * hd;
    for (int pair = threadIdx.x; pair < width / 2; pair += blockDim.x) {
        const int head = pair / half, i = pair % half;
        const float *src = c + (size_t)row * width + head * hd + i;
        float a = src[0], b = src[half];
        if (head >= heads + kvh) {
            const size_t to = (((size_t)slot * kvh + (head - heads - kvh)) * p.capacity + pos) * hd + i;
            vc[to] = from_f32<T>(a);
            vc[to + half] = from_f32<T>(b);
            continue;
        }
        if (p.rope) {
            const float co = cosv[(size_t)pos * half + i], si = sinv[(size_t)pos * half + i];
            const float na = __fmaf_rn(a, co, -__fmul_rn(b, si));
            const float nb = __fmaf_rn(b, co, __fmul_rn(a, si));
            a = na;
            b = nb;
        }
        if (head < heads) {
            const size_t to = ((size_t)row * heads + head) * hd + i;
            q[to] = from_f32<T>(a);
            q[to + half] = from_f32<T>(b);
        } else {
            const size_t to = (((size_t)slot * kvh + (head - heads)) * p.capacity + pos) * hd + i;
            kc[to] = from_f32<T>(a);
            kc[to + half] = from_f32<T>(b);
        }
    }
}

// silu_mul_rows.comp:16-27: out = SiLU(gate) up from the f32 gate/up projection, gate first.
template <typename T>
__global__ void __launch_bounds__(256)
    silu_mul_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ c,
                         T *__restrict__ out) {
    const int inner = p.inner;
    const size_t total = (size_t)p.rows * inner;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t row = idx / inner, i = idx % inner;
        const float *cr = c + row * 2 * inner;
        out[idx] = from_f32<T>(silu_mul(cr[i], cr[inner + i]));
    }
}

// attention_rows.comp:46-126: causal attention, flash-style. Block (t, h) takes the PREFILL_TILE
// rows from t PREFILL_TILE for query head h, and walks the slot's cache from position 0 to the
// last of their positions in tiles of 32 keys, each query keeping a running maximum, sum and
// output. Four threads take a query, each the float4s j * 4 + lane4 of it; the scores are summed
// over the four by a butterfly. Keys past a query's position are masked; keys past the tile's last
// are read as zero.
template <typename T, int HD>
__global__ void __launch_bounds__(256)
    attention_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const T *__restrict__ q,
                          const T *__restrict__ kc, const T *__restrict__ vc, T *__restrict__ out) {
    constexpr int KEYS = 32, Q4 = HD / 16;  // float4s of q per thread
    __shared__ float4 ks[KEYS * HD / 4];
    __shared__ float4 vs[KEYS * HD / 4];
    __shared__ uint32_t tile_last, tile_slot;
    const int tid = threadIdx.x, query = tid >> 2, lane4 = tid & 3;
    const int row = blockIdx.x * PREFILL_TILE + query;
    const int head = blockIdx.y, heads = p.heads, kvh = p.kv_heads, kv = head / (heads / kvh);
    uint32_t pos = 0, slot = 0;
    const bool live = row < (int)p.rows && placed(at, p.rows, row, p.capacity, p.slots, pos, slot);
    if (tid == 0) {
        tile_last = 0;
        tile_slot = 0xffffffffu;
    }
    __syncthreads();
    if (live) {
        atomicMax(&tile_last, pos);
        atomicMin(&tile_slot, slot);
    }
    __syncthreads();
    if (tile_slot == 0xffffffffu) return;  // every row of the tile is padding
    const uint32_t last = tile_last, tslot = tile_slot;
    float4 qv[Q4], o[Q4];
#pragma unroll
    for (int j = 0; j < Q4; j++) {
        o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        qv[j] = o[j];
        if (live) {
            const T *src = q + ((size_t)row * heads + head) * HD + (j * 4 + lane4) * 4;
            qv[j] = make_float4(to_f32<T>(src[0]), to_f32<T>(src[1]), to_f32<T>(src[2]), to_f32<T>(src[3]));
        }
    }
    const float scale = 1.0f / sqrtf((float)HD);
    float m = -INFINITY, l = 0.0f;
    const size_t cache = ((size_t)tslot * kvh + kv) * p.capacity;
    for (uint32_t from = 0; from <= last; from += KEYS) {
        __syncthreads();
        for (int i = tid; i < KEYS * HD / 4; i += blockDim.x) {
            const int pp = i / (HD / 4), j = i % (HD / 4);
            float4 kf = make_float4(0.f, 0.f, 0.f, 0.f), vf = kf;
            if (from + pp <= last) {
                const T *ksrc = kc + (cache + from + pp) * HD + j * 4;
                const T *vsrc = vc + (cache + from + pp) * HD + j * 4;
                kf = make_float4(to_f32<T>(ksrc[0]), to_f32<T>(ksrc[1]), to_f32<T>(ksrc[2]), to_f32<T>(ksrc[3]));
                vf = make_float4(to_f32<T>(vsrc[0]), to_f32<T>(vsrc[1]), to_f32<T>(vsrc[2]), to_f32<T>(vsrc[3]));
            }
            ks[i] = kf;
            vs[i] = vf;
        }
        __syncthreads();
        float scores[KEYS];
        float top = -INFINITY;
#pragma unroll
        for (int pp = 0; pp < KEYS; pp++) {
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < Q4; j++) {
                const float4 kk = ks[pp * (HD / 4) + j * 4 + lane4];
                part = __fmaf_rn(qv[j].x, kk.x, part);
                part = __fmaf_rn(qv[j].y, kk.y, part);
                part = __fmaf_rn(qv[j].z, kk.z, part);
                part = __fmaf_rn(qv[j].w, kk.w, part);
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            scores[pp] = (live && from + pp <= pos) ? part * scale : -INFINITY;
            top = fmaxf(top, scores[pp]);
        }
        const float next = fmaxf(m, top);
        // A live query sees position 0 in the first tile, so `next` is finite from there on.
        const float rescale = (next == -INFINITY) ? 1.0f : expf(m - next);
        l *= rescale;
#pragma unroll
        for (int j = 0; j < Q4; j++) {
            o[j].x *= rescale;
            o[j].y *= rescale;
            o[j].z *= rescale;
            o[j].w *= rescale;
        }
#pragma unroll
        for (int pp = 0; pp < KEYS; pp++) {
            const float e = (scores[pp] == -INFINITY) ? 0.0f : expf(scores[pp] - next);
            l += e;
#pragma unroll
            for (int j = 0; j < Q4; j++) {
                const float4 vv = vs[pp * (HD / 4) + j * 4 + lane4];
                o[j].x = __fmaf_rn(e, vv.x, o[j].x);
                o[j].y = __fmaf_rn(e, vv.y, o[j].y);
                o[j].z = __fmaf_rn(e, vv.z, o[j].z);
                o[j].w = __fmaf_rn(e, vv.w, o[j].w);
            }
        }
        m = next;
    }
    if (!live) return;
#pragma unroll
    for (int j = 0; j < Q4; j++) {
        T *dst = out + ((size_t)row * heads + head) * HD + (j * 4 + lane4) * 4;
        dst[0] = from_f32<T>(__fdiv_rn(o[j].x, l));
        dst[1] = from_f32<T>(__fdiv_rn(o[j].y, l));
        dst[2] = from_f32<T>(__fdiv_rn(o[j].z, l));
        dst[3] = from_f32<T>(__fdiv_rn(o[j].w, l));
    }
}

// ---- launchers -------------------------------------------------------------------------------

cudaError_t launch_norm_rows(const tg_params &p, const uint32_t *at, const float *x,
                             const float *g, void *out, cudaStream_t s) {
    const dim3 grid((p.rows + 3) / 4);
    if (p.dtype == TG_BF16)
        norm_rows_kernel<bf16><<<grid, 128, 0, s>>>(p, at, x, g, (bf16 *)out);
    else
        norm_rows_kernel<float><<<grid, 128, 0, s>>>(p, at, x, g, (float *)out);
    return cudaGetLastError();
}

cudaError_t launch_add_norm_rows(const tg_params &p, const uint32_t *at, const float *c,
                                 const float *res, const float *g, float *sum, void *normed,
                                 cudaStream_t s) {
    const dim3 grid((p.rows + 3) / 4);
    if (p.normed_f32)
        add_norm_rows_kernel<float, true><<<grid, 128, 0, s>>>(p, at, c, res, g, sum, normed);
    else if (p.dtype == TG_BF16)
        add_norm_rows_kernel<bf16, false><<<grid, 128, 0, s>>>(p, at, c, res, g, sum, normed);
    else
        add_norm_rows_kernel<float, false><<<grid, 128, 0, s>>>(p, at, c, res, g, sum, normed);
    return cudaGetLastError();
}

cudaError_t launch_rope_rows(const tg_params &p, const uint32_t *at, const float *c,
                             const float *cs, const float *sn, void *q, void *kc, void *vc,
                             cudaStream_t s) {
    if (p.dtype == TG_BF16)
        rope_rows_kernel<bf16><<<p.rows, 256, 0, s>>>(p, at, c, cs, sn, (bf16 *)q, (bf16 *)kc, (bf16 *)vc);
    else
        rope_rows_kernel<float><<<p.rows, 256, 0, s>>>(p, at, c, cs, sn, (float *)q, (float *)kc, (float *)vc);
    return cudaGetLastError();
}

cudaError_t launch_silu_mul_rows(const tg_params &p, const uint32_t *at, const float *c,
                                 void *out, cudaStream_t s) {
    const size_t total = (size_t)p.rows * p.inner;
    const int blocks = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    if (p.dtype == TG_BF16)
        silu_mul_rows_kernel<bf16><<<blocks, 256, 0, s>>>(p, at, c, (bf16 *)out);
    else
        silu_mul_rows_kernel<float><<<blocks, 256, 0, s>>>(p, at, c, (float *)out);
    return cudaGetLastError();
}

cudaError_t launch_attention_rows(const tg_params &p, const uint32_t *at, const void *q,
                                  const void *kc, const void *vc, void *out, cudaStream_t s) {
    const dim3 grid((p.rows + PREFILL_TILE - 1) / PREFILL_TILE, p.heads);
    const int threads = PREFILL_TILE * 4;
    if (p.head_dim == 64) {
        if (p.dtype == TG_BF16)
            attention_rows_kernel<bf16, 64><<<grid, threads, 0, s>>>(p, at, (const bf16 *)q, (const bf16 *)kc, (const bf16 *)vc, (bf16 *)out);
        else
            attention_rows_kernel<float, 64><<<grid, threads, 0, s>>>(p, at, (const float *)q, (const float *)kc, (const float *)vc, (float *)out);
    } else if (p.head_dim == 128) {
        if (p.dtype == TG_BF16)
            attention_rows_kernel<bf16, 128><<<grid, threads, 0, s>>>(p, at, (const bf16 *)q, (const bf16 *)kc, (const bf16 *)vc, (bf16 *)out);
        else
            attention_rows_kernel<float, 128><<<grid, threads, 0, s>>>(p, at, (const float *)q, (const float *)kc, (const float *)vc, (float *)out);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace tg
