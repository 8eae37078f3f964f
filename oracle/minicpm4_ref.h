/*
 * TEST INFRASTRUCTURE ONLY. This is the CPU oracle that the parity tests, `__graft_entry__.smoke()`
 * and the `cpu_baseline` / `--impl reference` legs of `bench.py` check the CUDA path against. It
 * is never linked into, loaded by or called from the product library (`libtgcuda.so`).
 *
 * A plain-C, fp32 restatement of one MiniCPM-4 stack as tgtts-v4's `graph` crate runs it:
 *
 *   decode step  crates/graph/src/decode.rs:618-735 (per layer: qkv_rope, attention_split,
 *                attention_combine, o_proj + residual, gate_up, down_proj + residual; then the
 *                final norm)
 *   prefill      crates/graph/src/prefill.rs:318-411 (the same per row, causal over the slot)
 *   kernels      kernels/glsl/norm.glsl:10-53 (RMSNorm), gemv_qkv_rope.comp:51-107 (row pairs,
 *                RoPE sign convention, cache layout), attention_split.comp:52-112 +
 *                attention_combine.comp:29-58 (scale 1/sqrt(hd), GQA head -> kv head / group),
 *                gemv_residual.comp:28-45, gemv_gate_up.comp:31-52 (SiLU = g / (1 + e^-g)),
 *                add_norm_rows.comp:21-45, attention_rows.comp:46-126
 *   RoPE tables  crates/graph/src/decode.rs:143-168
 *
 * The stated oracle of the reference is "burn's CPU model in f32" (not in the reference tree);
 * this computes every value in f32 with f32 accumulation. One addition the reference does not
 * have: `residual_scale`, applied as x + s * branch (s = 1 reproduces the reference).
 *
 * Every sum is taken in a fixed order that does not depend on the thread count, so results are
 * bit-identical for any `threads`.
 *
 * Pinned against the reference's own known answers (tests/test_oracle.py): the rms_layernorm
 * golden of crates/testkit/tests/fixtures/testkit.safetensors, the RoPE table answers of
 * decode.rs:1232-1242, zero weights giving zero (tests/prefill.rs:303-319) and the sequential-K
 * GEMM definition (kernels/gpu/cpu_oracle.py:276-286). Parity of whole stacks against the
 * reference is unpinned: tgtts-v4 keeps no backbone goldens in its tree (they need the external
 * VoxCPM2 checkpoint) and cannot run here (Rust, Vulkan); an independent numpy restatement
 * (ref_numpy.py) cross-checks this one instead.
 */
#ifndef TGTTS_ORACLE_MINICPM4_REF_H
#define TGTTS_ORACLE_MINICPM4_REF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int32_t hidden, inner, heads, kv_heads, head_dim, layers, capacity, slots;
    float eps, residual_scale;
    int32_t rope; /* 0: q and k are not rotated (VoxCPM2's residual LM) */
    const float *cos, *sin; /* [capacity][head_dim / 2] each */
} tgo_shape;

/* One layer's weights (row-major, f32) and its cache. qkv = rows[q_proj; k_proj; v_proj]
 * ([(heads + 2 kv_heads) head_dim][hidden]), gate_up = rows[gate_proj; up_proj]
 * ([2 inner][hidden]), as crates/graph/src/decode.rs:764-775 joins them. */
typedef struct {
    const float *input_norm, *qkv, *o, *post_norm, *gate_up, *down;
    float *k_cache, *v_cache; /* [slots][kv_heads][capacity][head_dim] */
} tgo_layer;

/* cos/sin[t][i] = cos/sin(t * (1 / factor_i) * theta^(-2i / head_dim)), in f32 in that order
 * (crates/graph/src/decode.rs:146-168). factors may be NULL (all 1). */
void tgo_rope_tables(int32_t head_dim, int32_t capacity, float theta, const double *factors,
                     float *cos_out, float *sin_out);

/* out = x * (1 / sqrt(mean(x^2) + eps)) * g (kernels/glsl/norm.glsl:12-53). */
void tgo_rmsnorm(const float *x, const float *g, int32_t k, float eps, float *out);

/* One decode step over `rows` rows, row b at position[b] of slot[b]; a row whose position is at
 * or past the capacity (u32 max) is spare: it writes no cache and its output is zero
 * (crates/graph/src/decode.rs:198-227, kernels/glsl/batch.glsl:9-14). x, out: [rows][hidden].
 * Returns 0, or -1 on a shape error. */
int32_t tgo_decode_step(const tgo_shape *s, const tgo_layer *layers, const float *final_norm,
                        int32_t rows, const uint32_t *position, const uint32_t *slot,
                        const float *x, float *out, int32_t threads);

/* A run of `len` positions from `start` in `slot`, causal over the slot's cache
 * (crates/graph/src/prefill.rs:473-503). x, out: [len][hidden]. Returns 0, or -1. */
int32_t tgo_prefill(const tgo_shape *s, const tgo_layer *layers, const float *final_norm,
                    uint32_t start, uint32_t len, uint32_t slot, const float *x, float *out,
                    int32_t threads);

/* C[m][n] = sum_k A[m][k] B[n][k], in f32, each sum sequential in k
 * (kernels/gpu/gemm.mlir:14-29, kernels/gpu/cpu_oracle.py:276-286). */
void tgo_gemm_abt(const float *a, const float *b, float *c, int32_t m, int32_t n, int32_t k,
                  int32_t threads);

/* The LM side's linear layer (kernels/glsl/gemv_linear.comp:41-60): for each of `rows` rows,
 * out[b][offset + i] = act(W[i] . [x0[b]; x1[b]] + bias[i]) over W [n][k0 + k1], each dot in f32
 * and sequential over the columns; act 0 none, 1 SiLU v / (1 + e^-v), 2 the scalar quantizer:
 * t = 1 - 2 / (e^(2|v|) + 1), round-half-even(sign(v) t levels) / levels. */
void tgo_gemv_linear(const float *x0, const float *x1, const float *w, const float *bias, float *out,
                     int32_t rows, int32_t n, int32_t k0, int32_t k1, int32_t offset, int32_t stride,
                     int32_t act, float levels);

#ifdef __cplusplus
}
#endif
#endif
