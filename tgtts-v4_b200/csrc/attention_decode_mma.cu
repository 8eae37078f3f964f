// The batched decoder's attention_split (attention_split.comp:52-112) on the tensor cores, for bf16
// caches and a head dimension of 64: a warp takes one chunk of ATTN_CHUNK positions of one row's
// KV head, its query heads (a GQA group of up to 16) the rows of mma.sync.m16n8k16:
//   S = q K^T over the chunk (8 n-tiles of 8 positions x 4 k-steps of 16 dimensions), q split
//       into bf16 hi + lo (two MMAs a step) so the scores carry 16 bits of each query value;
//   the chunk's softmax, unnormalised: m = the largest scaled score (positions past the row's
//       masked), e = exp(s - m), l = sum e — each row's values in its quad of lanes;
//   O = e V, e split into bf16 hi + lo the same way, V^T fragments by ldmatrix.trans.
// It writes partials in attention_split_kernel's layout and meaning (natural exponent, scale
// 1/sqrt(hd)), not the same bits, each over DECODE_WIDE_CHUNK positions rather than ATTN_CHUNK (a
// warp walks its sub-chunks of ATTN_CHUNK with an online softmax), which attention_combine joins
// told that width. A block holds four
// warps (four consecutive chunks of one row and KV head); each warp streams its chunk's keys and
// values into its own shared memory with cp.async: the positions before the row's (written by
// earlier steps) before the wait on the kernel before, the row's own position after it.
#include <type_traits>

#include "mma_common.cuh"
#include "tg_internal.h"

namespace tg {

namespace {

constexpr int AM_WARPS = 4;
constexpr int AM_ROW = 64 + fa::PAD;  // bf16 per shared row
constexpr int AM_WARP_SMEM = 2 * (int)ATTN_CHUNK * AM_ROW * 2;  // K and V of one chunk

using fa::split_pack;

}  // namespace

// The joins of a JOIN launch (see attention_split_mma_kernel): the block's warps' partials (m, l and
// the unnormalised o fragments of mma.sync's accumulator layout, zero and -inf for a warp past the
// row), then, in the last block of the row's KV head to arrive, the block partials.
TG_DEVICE void join_block(const tg_params &p, int b, int kv, uint32_t pos, const float (&m)[2], const float (&l)[2],
                          const float (&o)[8][4], float *__restrict__ po, float *__restrict__ pml,
                          bf16 *__restrict__ out, uint32_t *__restrict__ counts) {
    extern __shared__ __align__(128) unsigned char am_smem[];
    constexpr int HD = 64, G = 16;  // G: the accumulator's rows (query heads)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const int heads = p.heads, group = heads / p.kv_heads;
    const int stride = (int)attn_chunks(p.capacity), nb = (int)pos / (AM_WARPS * (int)ATTN_CHUNK) + 1;
    float *red = reinterpret_cast<float *>(am_smem);  // [AM_WARPS][G][HD] o, then [AM_WARPS][G][2] m, l
    float *red_ml = red + AM_WARPS * G * HD;
    __shared__ int last;
    __syncthreads();  // every warp is done with its keys and values
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int h = g + 8 * i;
        if (h >= group) continue;
        float *dst = red + (warp * G + h) * HD;
#pragma unroll
        for (int j = 0; j < 8; j++) *reinterpret_cast<float2 *>(dst + 8 * j + 2 * t4) = make_float2(o[j][2 * i], o[j][2 * i + 1]);
        if (t4 == 0) *reinterpret_cast<float2 *>(red_ml + (warp * G + h) * 2) = make_float2(m[i], l[i]);
    }
    __syncthreads();
    const size_t head0 = (size_t)b * heads + (size_t)kv * group;
    for (int i = threadIdx.x; i < group * HD; i += blockDim.x) {
        const int h = i / HD, d = i % HD;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < AM_WARPS; w++) mx = fmaxf(mx, red_ml[(w * G + h) * 2]);
        float sum = 0.0f, acc = 0.0f;
#pragma unroll
        for (int w = 0; w < AM_WARPS; w++) {
            const float mw = red_ml[(w * G + h) * 2];
            if (mw == -INFINITY) continue;
            const float e = expf(mw - mx);
            sum = __fmaf_rn(red_ml[(w * G + h) * 2 + 1], e, sum);
            acc = __fmaf_rn(red[(w * G + h) * HD + d], e, acc);
        }
        const size_t head = head0 + h;
        if (nb == 1) {
            out[head * HD + d] = __float2bfloat16_rn(__fdiv_rn(acc, sum));
        } else {
            po[(head * stride + blockIdx.x) * HD + d] = acc;
            if (d == 0) *reinterpret_cast<float2 *>(pml + (head * stride + blockIdx.x) * 2) = make_float2(mx, sum);
        }
    }
    if (nb == 1) return;
    // The last block of the row's KV head to arrive joins the block partials.
    __threadfence();
    __syncthreads();
    uint32_t *count = counts + (size_t)b * p.kv_heads + kv;
    if (threadIdx.x == 0) last = atomicAdd(count, 1u) == (uint32_t)(nb - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // A thread to four dimensions of a head: every block partial's loads in flight at once.
    constexpr int NB = 16;
    for (int i = threadIdx.x; i < group * (HD / 4); i += blockDim.x) {
        const int h = i / (HD / 4), d4 = i % (HD / 4);
        const size_t head = head0 + h;
        const float2 *ml = reinterpret_cast<const float2 *>(pml) + head * stride;
        const float4 *ob = reinterpret_cast<const float4 *>(po + head * stride * HD) + d4;
        float2 mv[NB];
        float4 ov[NB];
#pragma unroll
        for (int k = 0; k < NB; k++) {
            mv[k] = k < nb ? __ldcg(ml + k) : make_float2(-INFINITY, 0.0f);
            ov[k] = k < nb ? __ldcg(ob + (size_t)k * (HD / 4)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < NB; k++) mx = fmaxf(mx, mv[k].x);
        for (int k = NB; k < nb; k++) mx = fmaxf(mx, __ldcg(ml + k).x);
        float sum = 0.0f;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        auto add = [&](const float2 v, const float4 o4) {
            const float e = expf(v.x - mx);
            sum = __fmaf_rn(v.y, e, sum);
            acc = make_float4(__fmaf_rn(o4.x, e, acc.x), __fmaf_rn(o4.y, e, acc.y), __fmaf_rn(o4.z, e, acc.z),
                              __fmaf_rn(o4.w, e, acc.w));
        };
#pragma unroll
        for (int k = 0; k < NB; k++)
            if (k < nb) add(mv[k], ov[k]);
        for (int k = NB; k < nb; k++) add(__ldcg(ml + k), __ldcg(ob + (size_t)k * (HD / 4)));
        __nv_bfloat162 *dst = reinterpret_cast<__nv_bfloat162 *>(out + head * HD + 4 * d4);
        dst[0] = __floats2bfloat162_rn(__fdiv_rn(acc.x, sum), __fdiv_rn(acc.y, sum));
        dst[1] = __floats2bfloat162_rn(__fdiv_rn(acc.z, sum), __fdiv_rn(acc.w, sum));
    }
    if (threadIdx.x == 0) *count = 0u;
}

// SUB sub-chunks of ATTN_CHUNK positions a warp (a partial covers ATTN_CHUNK SUB positions): the
// warp walks them in order with an online softmax (the running maximum, the sum and the output
// rescaled as the maximum grows), so the partial is the same as one chunk's would be. QT is q's
// type: f32 (split into hi + lo) or bf16 (already a bf16 value: the hi part alone, one MMA a step).
//
// JOIN: the kernel also does attention_combine's work. A block joins its warps' partials in shared
// memory (the maxima, then the sums and outputs rescaled to them, in warp order) into one partial of
// AM_WARPS chunks, stored at partial index blockIdx.x; the last block of a row's KV head to finish
// (an arrival counter, zero between launches: the last block resets it) joins the row's block
// partials in block order and stores the heads' outputs in bf16. Which block arrives last does not
// change a bit, and a row of one block stores its output at once.
template <int SUB, typename QT, bool JOIN = false>
__global__ void __launch_bounds__(AM_WARPS * 32)
    attention_split_mma_kernel(tg_params p, const QT *__restrict__ q, const bf16 *__restrict__ kc,
                               const bf16 *__restrict__ vc, const uint32_t *__restrict__ at, float *__restrict__ po,
                               float *__restrict__ pml, bf16 *__restrict__ out, uint32_t *__restrict__ counts) {
    using namespace fa;
    extern __shared__ __align__(128) unsigned char am_smem[];
    constexpr int C = ATTN_CHUNK, HD = 64, W = C * SUB;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const int c = blockIdx.x * AM_WARPS + warp, kv = blockIdx.y, b = blockIdx.z;
    const int heads = p.heads, kvh = p.kv_heads, group = heads / kvh;
    const int chunks = ((int)p.capacity + W - 1) / W, stride = (int)attn_chunks(p.capacity);
    bf16 *ks = reinterpret_cast<bf16 *>(am_smem + (size_t)warp * AM_WARP_SMEM);
    bf16 *vs = ks + C * AM_ROW;
    pdl_launch_dependents();
    uint32_t pos = 0, slot = 0;
    const bool row_ok = placed(at, p.rows, b, p.capacity, p.slots, pos, slot);
    const bool live = row_ok && c < chunks && c * W <= (int)pos;
    const size_t slot_base = ((size_t)slot * kvh + kv) * p.capacity * HD;
    // Sub-chunk i's keys and values into shared memory: positions before the row's as they are,
    // past it zero; the row's own position only when `own_too` (after the wait).
    auto load = [&](int i, bool own_too) {
        const int start = c * W + i * C, own = (int)pos - start;
        for (int e = lane; e < C * 8; e += 32) {
            const int r = e / 8, ch = e % 8;
            if (r == own && !own_too) continue;
            const bool ok = r <= own && start + r < (int)p.capacity;
            const size_t src = slot_base + (size_t)(ok ? start + r : 0) * HD + ch * 8;
            cp_async16(ks + r * AM_ROW + ch * 8, kc + src, ok);
            cp_async16(vs + r * AM_ROW + ch * 8, vc + src, ok);
        }
        cp_async_commit();
    };
    if (live) load(0, false);  // the first sub-chunk's earlier positions, before the wait
    pdl_wait();
    if (!JOIN && !live) return;
    // A block whose first chunk is live joins (every warp, live or not, to its barriers).
    if (JOIN && !(row_ok && (int)blockIdx.x * AM_WARPS * W <= (int)pos)) return;
    const float scale = 1.0f / sqrtf((float)HD);
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    if (live) {
        {
            const int own = (int)pos - c * W;
            if (own < C && lane < 8) {  // the row's own position, if in the first sub-chunk
                const size_t src = slot_base + (size_t)pos * HD + lane * 8;
                cp_async16(ks + own * AM_ROW + lane * 8, kc + src, true);
                cp_async16(vs + own * AM_ROW + lane * 8, vc + src, true);
            }
            cp_async_commit();
        }
        // q of the group's heads (rows g < group; rows g + 8 and past the group are zero), hi and lo.
        constexpr bool QBF = std::is_same<QT, bf16>::value;
        uint32_t qh[4][4], ql[4][4];
        const QT *qg = q + ((size_t)b * heads + kv * group) * HD;
#pragma unroll
        for (int s = 0; s < 4; s++) {
#pragma unroll
            for (int r = 0; r < 4; r++) qh[s][r] = ql[s][r] = 0u;
            const int row0 = g, row1 = g + 8;
            if constexpr (QBF) {
                auto pair = [&](int row, int col) { return __ldcg(reinterpret_cast<const unsigned int *>(qg + row * HD + col)); };
                if (row0 < group) {
                    qh[s][0] = pair(row0, 16 * s + 2 * t4);
                    qh[s][2] = pair(row0, 16 * s + 8 + 2 * t4);
                }
                if (row1 < group) {
                    qh[s][1] = pair(row1, 16 * s + 2 * t4);
                    qh[s][3] = pair(row1, 16 * s + 8 + 2 * t4);
                }
                continue;
            }
            if (row0 < group) {
                const float2 x0 = __ldcg(reinterpret_cast<const float2 *>(qg + row0 * HD + 16 * s + 2 * t4));
                const float2 x2 = __ldcg(reinterpret_cast<const float2 *>(qg + row0 * HD + 16 * s + 8 + 2 * t4));
                split_pack(x0.x, x0.y, qh[s][0], ql[s][0]);
                split_pack(x2.x, x2.y, qh[s][2], ql[s][2]);
            }
            if (row1 < group) {
                const float2 x1 = __ldcg(reinterpret_cast<const float2 *>(qg + row1 * HD + 16 * s + 2 * t4));
                const float2 x3 = __ldcg(reinterpret_cast<const float2 *>(qg + row1 * HD + 16 * s + 8 + 2 * t4));
                split_pack(x1.x, x1.y, qh[s][1], ql[s][1]);
                split_pack(x3.x, x3.y, qh[s][3], ql[s][3]);
            }
        }
        for (int i = 0; i < SUB; i++) {
            const int start = c * W + i * C;
            if (start > (int)pos) break;
            if (i > 0) {
                __syncwarp();  // every lane is done with the last sub-chunk's shared memory
                load(i, true);
            }
            cp_async_wait<0>();
            __syncwarp();
            // S = q K^T: 8 n-tiles of 8 positions.
            float sc[8][4];
#pragma unroll
            for (int j = 0; j < 8; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
            for (int s = 0; s < 4; s++) {
#pragma unroll
                for (int j = 0; j < 8; j += 2) {
                    uint32_t kb[4];
                    const int mi = lane >> 3, rr = lane & 7;
                    ldmatrix_x4(kb, ks + (8 * j + (mi >> 1) * 8 + rr) * AM_ROW + s * 16 + (mi & 1) * 8);
                    mma_bf16(sc[j], qh[s], kb[0], kb[1]);
                    if (!QBF) mma_bf16(sc[j], ql[s], kb[0], kb[1]);
                    mma_bf16(sc[j + 1], qh[s], kb[2], kb[3]);
                    if (!QBF) mma_bf16(sc[j + 1], ql[s], kb[2], kb[3]);
                }
            }
            // The sub-chunk's maxima joined with the running ones; the running sums and outputs
            // rescaled to the new maxima (the first sub-chunk's scale is 0 against an empty run).
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < 8; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int at_pos = start + 8 * j + 2 * t4 + (e & 1);
                    const float v = at_pos <= (int)pos ? sc[j][e] * scale : -INFINITY;
                    sc[j][e] = v;
                    mx[e >> 1] = fmaxf(mx[e >> 1], v);
                }
            float alpha[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
                const float next = fmaxf(m[r], mx[r]);
                alpha[r] = m[r] == -INFINITY ? 0.0f : expf(m[r] - next);
                m[r] = next;
            }
            float ls[2] = {0.0f, 0.0f};
#pragma unroll
            for (int j = 0; j < 8; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float v = sc[j][e] == -INFINITY ? 0.0f : expf(sc[j][e] - m[e >> 1]);
                    sc[j][e] = v;
                    ls[e >> 1] += v;
                }
#pragma unroll
            for (int r = 0; r < 2; r++) {
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
                l[r] = __fmaf_rn(l[r], alpha[r], ls[r]);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                o[j][0] *= alpha[0];
                o[j][1] *= alpha[0];
                o[j][2] *= alpha[1];
                o[j][3] *= alpha[1];
            }
            // O += e V: e's accumulators as A fragments (hi and lo), V^T fragments by ldmatrix.trans.
#pragma unroll
            for (int s = 0; s < 4; s++) {
                uint32_t ph[4], pl[4];
                split_pack(sc[2 * s][0], sc[2 * s][1], ph[0], pl[0]);
                split_pack(sc[2 * s][2], sc[2 * s][3], ph[1], pl[1]);
                split_pack(sc[2 * s + 1][0], sc[2 * s + 1][1], ph[2], pl[2]);
                split_pack(sc[2 * s + 1][2], sc[2 * s + 1][3], ph[3], pl[3]);
#pragma unroll
                for (int j = 0; j < 8; j += 2) {
                    uint32_t vb[4];
                    const int mi = lane >> 3, rr = lane & 7;
                    ldmatrix_x4_trans(vb, vs + (16 * s + (mi & 1) * 8 + rr) * AM_ROW + 8 * j + (mi >> 1) * 8);
                    mma_bf16(o[j], ph, vb[0], vb[1]);
                    mma_bf16(o[j], pl, vb[0], vb[1]);
                    mma_bf16(o[j + 1], ph, vb[2], vb[3]);
                    mma_bf16(o[j + 1], pl, vb[2], vb[3]);
                }
            }
        }
    }  // live
    if constexpr (JOIN) {
        join_block(p, b, kv, pos, m, l, o, po, pml, out, counts);
    } else {
        // The partials of the group's heads (rows < group), at partial index c of `stride`.
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int h = g + 8 * i;
            if (h >= group) continue;
            const size_t head = (size_t)b * heads + kv * group + h;
            float *dst = po + (head * stride + c) * HD;
#pragma unroll
            for (int j = 0; j < 8; j++)
                *reinterpret_cast<float2 *>(dst + 8 * j + 2 * t4) = make_float2(o[j][2 * i], o[j][2 * i + 1]);
            if (t4 == 0) *reinterpret_cast<float2 *>(pml + (head * stride + c) * 2) = make_float2(m[i], l[i]);
        }
    }
}

bool attention_split_mma_supported(const tg_params &p) {
    return p.dtype == TG_BF16 && p.head_dim == 64 && p.kv_heads > 0 && p.heads % p.kv_heads == 0 &&
           p.heads / p.kv_heads <= 16 && p.capacity % CAPACITY_STEP == 0;
}

template <typename QT, bool JOIN = false>
static cudaError_t split_mma_t(const tg_params &p, const void *q, const void *kc, const void *vc, const uint32_t *at,
                               float *po, float *pml, cudaStream_t s, void *out = nullptr, uint32_t *counts = nullptr) {
    constexpr int SUB = DECODE_WIDE_CHUNK / ATTN_CHUNK;
    static_assert(!JOIN || SUB == 1, "the join counts blocks of AM_WARPS chunks of ATTN_CHUNK positions");
    auto kern = attention_split_mma_kernel<SUB, QT, JOIN>;
    const size_t smem = (size_t)AM_WARPS * AM_WARP_SMEM;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int chunks = (int)((p.capacity + DECODE_WIDE_CHUNK - 1) / DECODE_WIDE_CHUNK);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((chunks + AM_WARPS - 1) / AM_WARPS, p.kv_heads, p.rows);
    cfg.blockDim = dim3(AM_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, (const QT *)q, (const bf16 *)kc, (const bf16 *)vc, at, po, pml,
                              (bf16 *)out, counts);
}

cudaError_t launch_attention_split_mma(const tg_params &p, const void *q, const void *kc, const void *vc,
                                       const uint32_t *at, float *po, float *pml, cudaStream_t s, bool q_bf16) {
    if (!attention_split_mma_supported(p)) return cudaErrorInvalidValue;
    return q_bf16 ? split_mma_t<bf16>(p, q, kc, vc, at, po, pml, s) : split_mma_t<float>(p, q, kc, vc, at, po, pml, s);
}

cudaError_t launch_attention_split_join(const tg_params &p, const void *q, const void *kc, const void *vc,
                                        const uint32_t *at, float *po, float *pml, void *out, uint32_t *counts,
                                        cudaStream_t s) {
    if (!attention_split_mma_supported(p)) return cudaErrorInvalidValue;
    return split_mma_t<bf16, true>(p, q, kc, vc, at, po, pml, s, out, counts);
}

}  // namespace tg
