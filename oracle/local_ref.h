/* TEST INFRASTRUCTURE ONLY: a CPU restatement of VoxCPM2's local stacks as tgtts-v4 runs them
 * (crates/graph/src/local/{mod,dit,encoder}.rs and kernels/glsl/local_*.comp, cfm_noise.comp,
 * dit_euler.comp), which the parity tests check the CUDA path against. Never linked into the
 * product.
 *
 * Every tensor the reference keeps in f16 is rounded to f16 (RNE) at the same point here and held
 * as the f32 value of that f16; products are summed exactly enough (f64) that only the reference's
 * roundings remain.
 *
 * Parity against the reference itself is unpinned for the stacks' values: the reference's local
 * goldens (crates/graph/tests/local.rs) need the VoxCPM2 checkpoint, which is not here. What is
 * pinned: the sampler's schedule and Euler steps against the reference's rules (dit.rs:39-81,
 * "two steps, the first of which stays where it starts: one run of the DiT", local.rs:372-374),
 * and the whole restatement against an independent numpy one (oracle/ref_numpy.py). */
#ifndef TG_LOCAL_REF_H
#define TG_LOCAL_REF_H

#include <stdint.h>

typedef struct {
    int32_t hidden, inner, heads, kv_heads, head_dim, layers;
    int32_t tokens; /* a sequence's tokens (the stack's capacity) */
    float eps;
    const float *cos, *sin; /* [tokens][head_dim / 2] */
} tgo_local_shape;

/* One layer's weights as f32 values of f16: qkv [(heads + 2 kv) hd][hidden] (q, k, v rows),
 * o [hidden][heads hd], gate and up [inner][hidden] each, down [hidden][inner], gains [hidden]. */
typedef struct {
    const float *input_norm, *qkv, *o, *post_norm, *gate, *up, *down;
} tgo_local_layer;

/* Threads the matrix products and the attention use (1 by default). */
void tgo_local_set_threads(int32_t threads);

/* f16 rounding (RNE) of each value in place. */
void tgo_round_f16(float *x, int64_t n);

/* Stack::layers (local/mod.rs:573-680) over `seqs` sequences of `tokens` tokens: x
 * [seqs tokens][hidden] -> out, the tokens after the final norm. */
void tgo_local_stack(const tgo_local_shape *s, const tgo_local_layer *layers, const float *final_norm,
                     int32_t seqs, const float *x, float *out);

/* dit.rs:39-81: schedule (timesteps + 1 times) and the Euler steps (time, length); returns the
 * count of steps written. */
void tgo_schedule(int32_t timesteps, float *out);
int32_t tgo_euler_steps(int32_t timesteps, float *t, float *dt);

/* dit.rs:372-422: each step's time token (f64 values, before the f16 rounding), from the time and
 * delta-time MLPs' weights (f32 values of f16: w1 [hidden][hidden], b1, w2, b2). */
void tgo_time_tokens(int32_t hidden, const float *tw1, const float *tb1, const float *tw2, const float *tb2,
                     const float *dw1, const float *db1, const float *dw2, const float *db2, int32_t steps,
                     const float *times, double *out);

/* The sampler (dit.rs:112-271): `rows` rows; mu [rows][2][hidden] (f16 values), cond and noise
 * [rows][feat][patch], sampling [rows][2] (temperature, guidance), time tokens [steps][hidden]
 * (f16 values), dts [steps] -> patch [rows][feat][patch]. in_w and cond_w [hidden][feat],
 * out_w [feat][hidden], biases f16 values. */
void tgo_sampler(const tgo_local_shape *s, const tgo_local_layer *layers, const float *final_norm,
                 const float *in_w, const float *in_b, const float *cond_w, const float *cond_b,
                 const float *out_w, const float *out_b, const float *times, const float *dts, int32_t steps,
                 int32_t rows, int32_t feat, int32_t patch, const float *mu, const float *cond,
                 const float *noise, const float *sampling, float *patch_out);

/* The local encoder (encoder.rs:41-124): patches [rows][feat][patch] -> out [rows][hidden]
 * (f16 values); special [hidden] and in_b f16 values, in_w [hidden][feat]. */
void tgo_encoder(const tgo_local_shape *s, const tgo_local_layer *layers, const float *final_norm,
                 const float *in_w, const float *in_b, const float *special, int32_t rows, int32_t feat,
                 int32_t patch, const float *patches, float *out);

#endif
