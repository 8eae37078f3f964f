// The prefill's row kernels, around its projection GEMMs: the first input norm, RoPE with the KV
// append, causal GQA attention over the slot's cache, the residual add with the next norm, and
// SiLU-mul. They replace kernels/glsl/{norm_rows,rope_rows,attention_rows,add_norm_rows,
// silu_mul_rows}.comp. Rows carry placement words like the decode step's (a position, then a
// slot): a row placed past the cache is padding, which writes no cache and attends to nothing.
#include "tg_common.cuh"
#include "tg_internal.h"
#include "mma_common.cuh"

namespace tg {

// Four consecutive values rounded to T in one store (o is 4 T-aligned within a 16-byte aligned
// row): 16 bytes of f32, or 8 of bf16 where four 2-byte stores left a warp's 256 bytes in partial
// sectors.
template <typename T>
TG_DEVICE void store4(T *o, float a, float b, float c, float d);
template <>
TG_DEVICE void store4<float>(float *o, float a, float b, float c, float d) {
    *reinterpret_cast<float4 *>(o) = make_float4(a, b, c, d);
}
template <>
TG_DEVICE void store4<bf16>(bf16 *o, float a, float b, float c, float d) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    *reinterpret_cast<uint2 *>(o) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
}

// norm_rows.comp: out = RMSNorm(x) g, rounded to T; a warp to a row. A row of up to 1024 values is
// read once into registers (lane l holding its 16-byte vectors l, l + 32, ...) and its sum of squares
// taken from them in warp_rms_scale's order, so the same bits as warp_rms_scale over memory.
template <typename T>
__global__ void __launch_bounds__(128)
    norm_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ x,
                     const float *__restrict__ g, T *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= (int)p.rows) return;
    const int k = p.hidden;
    const float *xr = x + (size_t)row * k;
    if (k <= 1024) {
        constexpr int NV = 1024 / 128;  // vectors a lane at most
        float4 v[NV];
        const int nv = k / 128;
#pragma unroll
        for (int i = 0; i < NV; i++)
            if (i < nv) v[i] = reinterpret_cast<const float4 *>(xr)[lane + 32 * i];
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            if (i >= nv) continue;
            ss = __fmaf_rn(v[i].x, v[i].x, ss);
            ss = __fmaf_rn(v[i].y, v[i].y, ss);
            ss = __fmaf_rn(v[i].z, v[i].z, ss);
            ss = __fmaf_rn(v[i].w, v[i].w, ss);
        }
        ss = warp_sum(ss);
        const float s = 1.0f / sqrtf(__fdiv_rn(ss, (float)k) + p.eps);
#pragma unroll
        for (int i = 0; i < NV; i++) {
            if (i >= nv) continue;
            const int c = lane + 32 * i;
            const float4 gg = reinterpret_cast<const float4 *>(g)[c];
            store4<T>(out + (size_t)row * k + 4 * c, v[i].x * s * gg.x, v[i].y * s * gg.y, v[i].z * s * gg.z,
                      v[i].w * s * gg.w);
        }
        return;
    }
    const float s = warp_rms_scale(xr, k, p.eps);
    for (int c = lane; c < k / 4; c += 32) {
        const float4 v = reinterpret_cast<const float4 *>(xr)[c];
        const float4 gg = reinterpret_cast<const float4 *>(g)[c];
        store4<T>(out + (size_t)row * k + 4 * c, v.x * s * gg.x, v.y * s * gg.y, v.z * s * gg.z, v.w * s * gg.w);
    }
}

// add_norm_rows.comp:21-45: sum = residual + s c in f32, normed = RMSNorm(sum) g (from the f32
// sum), rounded to T, or kept in f32 for the final norm. With p.parts > 1, c is a GEMM's partial
// sums over parts of K, [parts][rows][hidden], added in part order first. A warp to a row (the
// prefill's many rows).
template <typename T, bool NORMED_F32>
__global__ void __launch_bounds__(128)
    add_norm_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ c,
                         const float *__restrict__ res, const float *__restrict__ g,
                         float *__restrict__ sum, void *__restrict__ normed) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= (int)p.rows) return;
    const int k = p.hidden;
    const size_t base = (size_t)row * k, part = (size_t)p.rows * k;
    const int parts = p.parts > 1 ? (int)p.parts : 1;
    const float sc = p.residual_scale;
    for (int q = lane; q < k / 4; q += 32) {
        float4 cv = reinterpret_cast<const float4 *>(c + base)[q];
        for (int j = 1; j < parts; j++) {
            const float4 v = reinterpret_cast<const float4 *>(c + j * part + base)[q];
            cv = make_float4(cv.x + v.x, cv.y + v.y, cv.z + v.z, cv.w + v.w);
        }
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
            store4<T>(static_cast<T *>(normed) + base + 4 * q, o[0], o[1], o[2], o[3]);
        }
    }
}

// add_norm_rows for few rows (a batched decode step's): a block to a row and a thread to 4
// columns, so that all of a row's loads are in flight at once; the sum of squares is each thread's
// 4 in column order, then each warp's (butterfly), then the warps' in order.
template <typename T, bool NORMED_F32>
__global__ void __launch_bounds__(1024)
    add_norm_rows_block_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ c,
                         const float *__restrict__ res, const float *__restrict__ g,
                         float *__restrict__ sum, void *__restrict__ normed) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float warp_ss[32];
    const int row = blockIdx.x, t = threadIdx.x;
    const int k = p.hidden;
    const size_t base = (size_t)row * k, part = (size_t)p.rows * k;
    const int parts = p.parts > 1 ? (int)p.parts : 1;
    float4 v[ADD_NORM_MAX_PARTS];
#pragma unroll
    for (int j = 0; j < ADD_NORM_MAX_PARTS; j++)
        if (j < parts) v[j] = reinterpret_cast<const float4 *>(c + j * part + base)[t];
    const float4 rv = reinterpret_cast<const float4 *>(res + base)[t];
    const float4 gg = reinterpret_cast<const float4 *>(g)[t];
    float4 cv = v[0];
#pragma unroll
    for (int j = 1; j < ADD_NORM_MAX_PARTS; j++)
        if (j < parts) cv = make_float4(cv.x + v[j].x, cv.y + v[j].y, cv.z + v[j].z, cv.w + v[j].w);
    const float sc = p.residual_scale;
    const float4 sv = make_float4(__fmaf_rn(sc, cv.x, rv.x), __fmaf_rn(sc, cv.y, rv.y), __fmaf_rn(sc, cv.z, rv.z),
                                  __fmaf_rn(sc, cv.w, rv.w));
    reinterpret_cast<float4 *>(sum + base)[t] = sv;
    float ss = __fmul_rn(sv.x, sv.x);
    ss = __fmaf_rn(sv.y, sv.y, ss);
    ss = __fmaf_rn(sv.z, sv.z, ss);
    ss = __fmaf_rn(sv.w, sv.w, ss);
    ss = warp_sum(ss);
    if ((t & 31) == 0) warp_ss[t >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += warp_ss[w];
    const float s = 1.0f / sqrtf(__fdiv_rn(tot, (float)k) + p.eps);
    const float o[4] = {sv.x * s * gg.x, sv.y * s * gg.y, sv.z * s * gg.z, sv.w * s * gg.w};
    if (NORMED_F32) {
        reinterpret_cast<float4 *>(static_cast<float *>(normed) + base)[t] = make_float4(o[0], o[1], o[2], o[3]);
    } else {
        store4<T>(static_cast<T *>(normed) + base + 4 * t, o[0], o[1], o[2], o[3]);
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

// silu_mul_rows.comp:16-27: out = SiLU(gate) up from the f32 gate/up projection, whose columns
// follow gate_up's rows (gate_up_row). A block to a row, four columns a thread.
template <typename T>
__global__ void __launch_bounds__(256)
    silu_mul_rows_kernel(tg_params p, const uint32_t *__restrict__ at, const float *__restrict__ c,
                         T *__restrict__ out) {
    const int inner = p.inner, row = blockIdx.x;
    const float *cr = c + (size_t)row * 2 * inner;
    for (int i = 4 * threadIdx.x; i < inner; i += 4 * blockDim.x) {
        const float4 g = *reinterpret_cast<const float4 *>(cr + gate_up_row(i, 0));
        const float4 u = *reinterpret_cast<const float4 *>(cr + gate_up_row(i, 1));
        T *o = out + (size_t)row * inner + i;
        o[0] = from_f32<T>(silu_mul(g.x, u.x));
        o[1] = from_f32<T>(silu_mul(g.y, u.y));
        o[2] = from_f32<T>(silu_mul(g.z, u.z));
        o[3] = from_f32<T>(silu_mul(g.w, u.w));
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

// attention_rows.comp on tensor cores, for bf16: flash attention with mma.sync m16n8k16 (bf16 in,
// f32 accumulate). Block (t, h) takes the PREFILL_TILE rows from t PREFILL_TILE for query head h,
// a warp to 16 rows; the keys and values of the rows' slot stream through shared memory in tiles
// of 64 positions (cp.async, two buffers), up to the last of the rows' positions. Per tile: S =
// Q K^T by 32 MMAs a warp, scaled and masked past each row's position, an online softmax in
// registers, then O += P V by 32 MMAs, P taken from S's accumulators as bf16 A fragments. Keys
// past the tile's last position are read as zero.

template <int HD>
__global__ void __launch_bounds__(128)
    attention_rows_mma_kernel(tg_params p, const uint32_t *__restrict__ at, const bf16 *__restrict__ q,
                              const bf16 *__restrict__ kc, const bf16 *__restrict__ vc, bf16 *__restrict__ out) {
    using namespace fa;
    constexpr int ROW = HD + PAD;  // shared row stride in bf16
    constexpr int KS = HD / 16;    // k-steps over the head dimension
    constexpr int NT = HD / 8;     // n-tiles of the output
    extern __shared__ __align__(128) unsigned char fa_smem[];
    bf16 *qs = reinterpret_cast<bf16 *>(fa_smem);  // [PREFILL_TILE][ROW]
    bf16 *ks[2] = {qs + PREFILL_TILE * ROW, qs + PREFILL_TILE * ROW + KT * ROW};  // [KT][ROW] each
    bf16 *vs[2] = {qs + PREFILL_TILE * ROW + 2 * KT * ROW, qs + PREFILL_TILE * ROW + 3 * KT * ROW};
    __shared__ uint32_t tile_last, tile_slot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int r0 = blockIdx.x * PREFILL_TILE;
    const int head = blockIdx.y, heads = p.heads, kvh = p.kv_heads, kv = head / (heads / kvh);
    if (tid == 0) {
        tile_last = 0;
        tile_slot = 0xffffffffu;
    }
    __syncthreads();
    if (tid < PREFILL_TILE && r0 + tid < (int)p.rows) {
        uint32_t pos, slot;
        if (placed(at, p.rows, r0 + tid, p.capacity, p.slots, pos, slot)) {
            atomicMax(&tile_last, pos);
            atomicMin(&tile_slot, slot);
        }
    }
    __syncthreads();
    if (tile_slot == 0xffffffffu) return;  // every row of the tile is padding
    const uint32_t last = tile_last;
    const size_t cache = ((size_t)tile_slot * kvh + kv) * p.capacity;
    // This thread's two rows (g and g + 8 of its warp's 16) and their positions (-1: padding).
    int qpos[2];
    for (int i = 0; i < 2; i++) {
        const int row = r0 + warp * 16 + g + 8 * i;
        uint32_t pos, slot;
        qpos[i] = (row < (int)p.rows && placed(at, p.rows, row, p.capacity, p.slots, pos, slot)) ? (int)pos : -1;
    }
    // Q tile into shared memory (rows past the run read as zero), then A fragments.
    for (int i = tid; i < PREFILL_TILE * HD / 8; i += blockDim.x) {
        const int r = i / (HD / 8), c = i % (HD / 8);
        const bool ok = r0 + r < (int)p.rows;
        cp_async16(qs + r * ROW + c * 8, q + ((size_t)(ok ? r0 + r : r0) * heads + head) * HD + c * 8, ok);
    }
    auto load_kv = [&](int kt, int buf) {
        for (int i = tid; i < KT * HD / 8; i += blockDim.x) {
            const int r = i / (HD / 8), c = i % (HD / 8);
            const uint32_t key = kt * KT + r;
            const bool ok = key <= last;
            const size_t off = (cache + (ok ? key : 0)) * HD + c * 8;
            cp_async16(ks[buf] + r * ROW + c * 8, kc + off, ok);
            cp_async16(vs[buf] + r * ROW + c * 8, vc + off, ok);
        }
    };
    load_kv(0, 0);
    cp_async_commit();
    const int ntiles = (int)(last / KT) + 1;
    uint32_t qa[KS][4];
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    const float scale = 1.0f / sqrtf((float)HD);
    for (int kt = 0; kt < ntiles; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < ntiles) load_kv(kt + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (kt == 0) {
#pragma unroll
            for (int s = 0; s < KS; s++) {
                const int mi = lane >> 3, rr = lane & 7;
                ldmatrix_x4(qa[s], qs + (warp * 16 + (mi & 1) * 8 + rr) * ROW + s * 16 + (mi >> 1) * 8);
            }
        }
        // S = Q K^T: 8 n-tiles of 8 keys.
        float sc[KT / 8][4];
#pragma unroll
        for (int j = 0; j < KT / 8; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
        for (int s = 0; s < KS; s++) {
#pragma unroll
            for (int j = 0; j < KT / 8; j += 2) {
                // Two n-tiles (keys 8j .. 8j + 15) by one ldmatrix.x4: matrices (keys 8j.., hd 16s),
                // (keys 8j.., hd 16s + 8), (keys 8j + 8.., hd 16s), (keys 8j + 8.., hd 16s + 8).
                uint32_t b[4];
                const int mi = lane >> 3, rr = lane & 7;
                ldmatrix_x4(b, ks[buf] + (8 * j + (mi >> 1) * 8 + rr) * ROW + s * 16 + (mi & 1) * 8);
                mma_bf16(sc[j], qa[s], b[0], b[1]);
                mma_bf16(sc[j + 1], qa[s], b[2], b[3]);
            }
        }
        // Scale, mask past each row's position, online softmax.
        float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < KT / 8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int key = kt * KT + 8 * j + 2 * t4 + (e & 1);
                const int i = e >> 1;
                const float v = key <= qpos[i] ? sc[j][e] * scale : -INFINITY;
                sc[j][e] = v;
                tmax[i] = fmaxf(tmax[i], v);
            }
        float corr[2];
#pragma unroll
        for (int i = 0; i < 2; i++) {
            tmax[i] = fmaxf(tmax[i], __shfl_xor_sync(0xffffffffu, tmax[i], 1));
            tmax[i] = fmaxf(tmax[i], __shfl_xor_sync(0xffffffffu, tmax[i], 2));
            const float next = fmaxf(m[i], tmax[i]);
            corr[i] = next == -INFINITY ? 1.0f : expf(m[i] - next);
            m[i] = next;
            l[i] *= corr[i];
        }
#pragma unroll
        for (int j = 0; j < NT; j++) {
            o[j][0] *= corr[0];
            o[j][1] *= corr[0];
            o[j][2] *= corr[1];
            o[j][3] *= corr[1];
        }
        float tsum[2] = {0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < KT / 8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = e >> 1;
                const float pe = sc[j][e] == -INFINITY ? 0.0f : expf(sc[j][e] - m[i]);
                sc[j][e] = pe;
                tsum[i] += pe;
            }
#pragma unroll
        for (int i = 0; i < 2; i++) {
            tsum[i] += __shfl_xor_sync(0xffffffffu, tsum[i], 1);
            tsum[i] += __shfl_xor_sync(0xffffffffu, tsum[i], 2);
            l[i] += tsum[i];
        }
        // O += P V: P's accumulators as A fragments (k-step s = keys 16s .. 16s + 15).
#pragma unroll
        for (int s = 0; s < KT / 16; s++) {
            uint32_t pa[4];
            pa[0] = pack_bf16(sc[2 * s][0], sc[2 * s][1]);
            pa[1] = pack_bf16(sc[2 * s][2], sc[2 * s][3]);
            pa[2] = pack_bf16(sc[2 * s + 1][0], sc[2 * s + 1][1]);
            pa[3] = pack_bf16(sc[2 * s + 1][2], sc[2 * s + 1][3]);
#pragma unroll
            for (int j = 0; j < NT; j += 2) {
                // V^T fragments by ldmatrix.trans: matrices (keys 16s.., hd 8j), (keys 16s + 8.., hd 8j),
                // (keys 16s.., hd 8j + 8), (keys 16s + 8.., hd 8j + 8).
                uint32_t b[4];
                const int mi = lane >> 3, rr = lane & 7;
                ldmatrix_x4_trans(b, vs[buf] + (16 * s + (mi & 1) * 8 + rr) * ROW + 8 * j + (mi >> 1) * 8);
                mma_bf16(o[j], pa, b[0], b[1]);
                mma_bf16(o[j + 1], pa, b[2], b[3]);
            }
        }
        __syncthreads();
    }
    // Normalise and store the live rows, bf16.
#pragma unroll
    for (int i = 0; i < 2; i++) {
        if (qpos[i] < 0) continue;
        const int row = r0 + warp * 16 + g + 8 * i;
        const float inv = 1.0f / l[i];
        bf16 *dst = out + ((size_t)row * heads + head) * HD;
#pragma unroll
        for (int j = 0; j < NT; j++) {
            const __nv_bfloat162 v = __floats2bfloat162_rn(o[j][2 * i] * inv, o[j][2 * i + 1] * inv);
            *reinterpret_cast<__nv_bfloat162 *>(dst + 8 * j + 2 * t4) = v;
        }
    }
}

// ---- launchers -------------------------------------------------------------------------------

cudaError_t launch_norm_rows(const tg_params &p, const uint32_t *at, const float *x,
                             const float *g, void *out, cudaStream_t s) {
    const dim3 grid((p.rows + 3) / 4);
    if (p.dtype == TG_BF16 && !p.normed_f32)
        return launch_pdl(norm_rows_kernel<bf16>, grid, dim3(128), 0, s, p, at, x, g, (bf16 *)out);
    return launch_pdl(norm_rows_kernel<float>, grid, dim3(128), 0, s, p, at, x, g, (float *)out);
}

cudaError_t launch_add_norm_rows(const tg_params &p, const uint32_t *at, const float *c,
                                 const float *res, const float *g, float *sum, void *normed,
                                 cudaStream_t s) {
    if (p.hidden % 128 || p.hidden > 4 * 1024 || p.parts > (uint32_t)ADD_NORM_MAX_PARTS) return cudaErrorInvalidValue;
    if (p.flags & 2) {  // few rows: a block to a row
        const dim3 grid(p.rows), block(p.hidden / 4);
        if (p.normed_f32)
            return launch_pdl(add_norm_rows_block_kernel<float, true>, grid, block, 0, s, p, at, c, res, g, sum, normed);
        if (p.dtype == TG_BF16)
            return launch_pdl(add_norm_rows_block_kernel<bf16, false>, grid, block, 0, s, p, at, c, res, g, sum, normed);
        return launch_pdl(add_norm_rows_block_kernel<float, false>, grid, block, 0, s, p, at, c, res, g, sum, normed);
    }
    const dim3 grid((p.rows + 3) / 4);
    if (p.normed_f32)
        return launch_pdl(add_norm_rows_kernel<float, true>, grid, dim3(128), 0, s, p, at, c, res, g, sum, normed);
    if (p.dtype == TG_BF16)
        return launch_pdl(add_norm_rows_kernel<bf16, false>, grid, dim3(128), 0, s, p, at, c, res, g, sum, normed);
    return launch_pdl(add_norm_rows_kernel<float, false>, grid, dim3(128), 0, s, p, at, c, res, g, sum, normed);
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
    if (p.inner % 4) return cudaErrorInvalidValue;
    if (p.dtype == TG_BF16)
        silu_mul_rows_kernel<bf16><<<p.rows, 256, 0, s>>>(p, at, c, (bf16 *)out);
    else
        silu_mul_rows_kernel<float><<<p.rows, 256, 0, s>>>(p, at, c, (float *)out);
    return cudaGetLastError();
}

cudaError_t launch_attention_rows(const tg_params &p, const uint32_t *at, const void *q,
                                  const void *kc, const void *vc, void *out, cudaStream_t s) {
    const dim3 grid((p.rows + PREFILL_TILE - 1) / PREFILL_TILE, p.heads);
    const int threads = PREFILL_TILE * 4;
    if (p.dtype == TG_BF16) {
        // Tensor cores for bf16.
        auto run = [&](auto kern, int hd) {
            const size_t smem = (size_t)(PREFILL_TILE + 4 * fa::KT) * (hd + fa::PAD) * sizeof(bf16);
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            kern<<<grid, 128, smem, s>>>(p, at, (const bf16 *)q, (const bf16 *)kc, (const bf16 *)vc, (bf16 *)out);
            return cudaGetLastError();
        };
        if (p.head_dim == 64) return run(attention_rows_mma_kernel<64>, 64);
        if (p.head_dim == 128) return run(attention_rows_mma_kernel<128>, 128);
        return cudaErrorInvalidValue;
    }
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
