// The LM side's linear layers (kernels/glsl/gemv_linear.comp:1-62): out[b][offset + i] =
// act(W [x0; x1] + bias)[i] for each of up to 64 batch rows, W [n][k + k1] in the storage type, x0
// [rows][k] and x1 [rows][k1] f32 (the two inputs side by side, as fusion_concat_proj's input is
// concatenated upstream), act none, SiLU, or the scalar quantizer's tanh rounded to a multiple of
// 1 / levels.
//
// A warp takes one row of W: each lane sums 16-byte vectors lane, lane + 32, ... of the row in
// order (x0's then x1's columns), one fused multiply-add a value, then the xor butterfly joins the
// lanes — the order of every sum is fixed by k and k1 alone, so a batch row's output does not
// depend on the batch beside it. The batch's inputs are staged in shared memory, 8 rows at a time.
#include "tg_common.cuh"
#include "tg_internal.h"

namespace tg {

namespace {

constexpr int LIN_WARPS = 8;
constexpr int LIN_NB = 8;  // batch rows a pass

template <typename T>
__global__ void __launch_bounds__(LIN_WARPS * 32)
    gemv_linear_kernel(tg_params p, const float *__restrict__ x0, const float *__restrict__ x1, const T *__restrict__ w,
                       const float *__restrict__ bias, float *__restrict__ out) {
    extern __shared__ __align__(16) float xs[];  // [LIN_NB][k + k1]
    const int K0 = (int)p.k, K1 = (int)p.k1, K = K0 + K1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * LIN_WARPS + warp;
    using V = Vec<T>;
    constexpr int E = V::N;  // values a 16-byte load
    pdl_launch_dependents();
    pdl_wait();
    for (int b0 = 0; b0 < (int)p.rows; b0 += LIN_NB) {
        const int nb = min(LIN_NB, (int)p.rows - b0);
        for (int i = threadIdx.x; i < nb * K / 4; i += blockDim.x) {
            const int b = i / (K / 4), c = (i % (K / 4)) * 4;
            const float *src = c < K0 ? x0 + (size_t)(b0 + b) * K0 + c : x1 + (size_t)(b0 + b) * K1 + (c - K0);
            *reinterpret_cast<float4 *>(xs + (size_t)b * K + c) = *reinterpret_cast<const float4 *>(src);
        }
        __syncthreads();
        if (row < (int)p.n) {
            float acc[LIN_NB];
#pragma unroll
            for (int b = 0; b < LIN_NB; b++) acc[b] = 0.0f;
            const typename V::Raw *wr = reinterpret_cast<const typename V::Raw *>(w + (size_t)row * K);
            for (int v = lane; v < K / E; v += 32) {
                float wf[E];
                V::unpack(ld_stream(wr + v), wf);
#pragma unroll
                for (int b = 0; b < LIN_NB; b++) {
                    if (b >= nb) break;
                    const float *xb = xs + (size_t)b * K + v * E;
#pragma unroll
                    for (int e = 0; e < E; e++) acc[b] = __fmaf_rn(wf[e], xb[e], acc[b]);
                }
            }
#pragma unroll
            for (int b = 0; b < LIN_NB; b++) acc[b] = warp_sum(acc[b]);
            if (lane < nb) {
                float y = 0.0f;
#pragma unroll
                for (int b = 0; b < LIN_NB; b++)
                    if (b == lane) y = acc[b];
                float v = y + bias[row];
                if (p.act == 1) {
                    v = __fdiv_rn(v, 1.0f + expf(-v));  // SiLU, gemv_linear.comp:50-51
                } else if (p.act == 2) {
                    // tanh from exp (gemv_linear.comp:52-56), then rounded to a multiple of 1/levels,
                    // halves to even.
                    const float t = 1.0f - __fdiv_rn(2.0f, expf(2.0f * fabsf(v)) + 1.0f);
                    v = __fdiv_rn(rintf(copysignf(t, v) * p.levels), p.levels);
                }
                out[(size_t)(b0 + lane) * p.stride + p.offset + row] = v;
            }
        }
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_gemv_linear(const tg_params &p, const float *x0, const float *x1, const void *w, const float *bias,
                               float *out, cudaStream_t s) {
    const int K = (int)(p.k + p.k1);
    const size_t smem = (size_t)LIN_NB * K * sizeof(float);
    const dim3 grid((p.n + LIN_WARPS - 1) / LIN_WARPS);
    auto go = [&](auto kern, const auto *wt) {
        cudaError_t e = cudaSuccess;
        if (smem > 32 * 1024 && (e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)))
            return e;
        kern<<<grid, LIN_WARPS * 32, smem, s>>>(p, x0, x1, wt, bias, out);
        return cudaGetLastError();
    };
    if (p.rows == 0) return cudaSuccess;
    if (p.dtype == TG_BF16) return go(gemv_linear_kernel<bf16>, static_cast<const bf16 *>(w));
    return go(gemv_linear_kernel<float>, static_cast<const float *>(w));
}

}  // namespace tg
