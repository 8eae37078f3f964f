/*
 * TEST INFRASTRUCTURE ONLY: the CPU restatement of VoxCPM2's local stacks (the sampler's DiT and
 * the local encoder) that the parity tests check the CUDA path against. local_ref.h says what it
 * follows; each function cites the reference lines it restates.
 */
#include "local_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static int32_t g_threads = 1;

void tgo_local_set_threads(int32_t threads) { g_threads = threads < 1 ? 1 : (threads > 256 ? 256 : threads); }

typedef void (*range_fn)(void *ctx, int64_t lo, int64_t hi);
typedef struct {
    range_fn fn;
    void *ctx;
    int64_t lo, hi;
} piece;

static void *run_piece(void *p) {
    piece *q = (piece *)p;
    q->fn(q->ctx, q->lo, q->hi);
    return NULL;
}

/* fn over [0, n) in contiguous pieces, one thread each; what is computed for an index does not
 * depend on the thread that takes it. */
static void parallel_for(int64_t n, range_fn fn, void *ctx) {
    int32_t threads = g_threads;
    if (threads < 1 || threads > 256) threads = 1;
    if (n < 2 * threads || threads == 1) {
        fn(ctx, 0, n);
        return;
    }
    pthread_t tid[256];
    piece pieces[256];
    int32_t started = 0;
    for (int32_t t = 0; t < threads; t++) {
        pieces[t] = (piece){fn, ctx, n * t / threads, n * (t + 1) / threads};
    }
    for (int32_t t = 1; t < threads; t++) {
        if (pthread_create(&tid[t], NULL, run_piece, &pieces[t]) != 0) break;
        started = t;
    }
    run_piece(&pieces[0]);
    for (int32_t t = 1; t <= started; t++) pthread_join(tid[t], NULL);
    for (int32_t t = started + 1; t < threads; t++) run_piece(&pieces[t]);
}

static float f16r(float v) { return (float)(_Float16)v; }

void tgo_round_f16(float *x, int64_t n) {
    for (int64_t i = 0; i < n; i++) x[i] = f16r(x[i]);
}

/* sum_k w[k] x[k] summed in f64 and rounded once to f32: the products of f16 values are exact in
 * f32, so this is the exact sum to f32 precision whatever order the GPU's tiles take. */
static float dotd(const float *w, const float *x, int32_t k) {
    double a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    int32_t i = 0;
    for (; i + 4 <= k; i += 4) {
        a0 += (double)(w[i] * x[i]);
        a1 += (double)(w[i + 1] * x[i + 1]);
        a2 += (double)(w[i + 2] * x[i + 2]);
        a3 += (double)(w[i + 3] * x[i + 3]);
    }
    for (; i < k; i++) a0 += (double)(w[i] * x[i]);
    return (float)((a0 + a1) + (a2 + a3));
}

/* y[m][n] = W[n] . x[m] for m < M, n < N (f32 of the exact sums). */
typedef struct {
    const float *w, *x;
    float *y;
    int32_t n, k;
} mm_job;

static void mm_range(void *c, int64_t lo, int64_t hi) {
    mm_job *j = (mm_job *)c;
    for (int64_t i = lo; i < hi; i++) {
        int64_t m = i / j->n, n = i % j->n;
        j->y[i] = dotd(j->w + n * (int64_t)j->k, j->x + m * (int64_t)j->k, j->k);
    }
}

static void matmul(const float *w, const float *x, float *y, int32_t M, int32_t N, int32_t K) {
    mm_job j = {w, x, y, N, K};
    parallel_for((int64_t)M * N, mm_range, &j);
}

/* local_norm.comp:19-46 / local_add_norm.comp:49-74: f16(v scale g), scale = 1 / sqrt(mean
 * square + eps) of the row as it is (f16 values). */
static void norm_row(const float *x, const float *g, int32_t n, float eps, float *out) {
    double sq = 0;
    for (int32_t i = 0; i < n; i++) sq += (double)(x[i] * x[i]);
    const float scale = 1.0f / sqrtf((float)sq / (float)n + eps);
    for (int32_t i = 0; i < n; i++) out[i] = f16r(x[i] * scale * g[i]);
}

/* local_qkv_rope.comp:70-90: q and k rotated (x cos + rotate_half(x) sin) and every value rounded
 * to f16; qkv [M][(heads + 2 kv) hd] holds the projection's f32 sums. */
static void rope_round(const tgo_local_shape *s, float *qkv, int32_t M) {
    const int32_t hd = s->head_dim, half = hd / 2, width = (s->heads + 2 * s->kv_heads) * hd;
    for (int32_t m = 0; m < M; m++) {
        const int32_t t = m % s->tokens;
        for (int32_t head = 0; head < s->heads + 2 * s->kv_heads; head++) {
            float *v = qkv + (int64_t)m * width + head * hd;
            for (int32_t i = 0; i < half; i++) {
                float a = v[i], b = v[i + half];
                if (head < s->heads + s->kv_heads) {
                    const float c = s->cos[t * half + i], sn = s->sin[t * half + i];
                    const float ra = a * c - b * sn, rb = b * c + a * sn;
                    a = ra;
                    b = rb;
                }
                v[i] = f16r(a);
                v[i + half] = f16r(b);
            }
        }
    }
}

/* local_attention.comp:27-70: each token's query head against every key of its sequence. */
typedef struct {
    const tgo_local_shape *s;
    const float *qkv;
    float *out;
} attn_job;

static void attn_range(void *c, int64_t lo, int64_t hi) {
    attn_job *j = (attn_job *)c;
    const tgo_local_shape *s = j->s;
    const int32_t hd = s->head_dim, T = s->tokens, heads = s->heads, kvh = s->kv_heads;
    const int32_t width = (heads + 2 * kvh) * hd;
    const float scale = 1.0f / sqrtf((float)hd);
    float sc[256];
    for (int64_t it = lo; it < hi; it++) {
        const int64_t m = it / heads;
        const int32_t h = (int32_t)(it % heads), kv = h / (heads / kvh);
        const int64_t first = m / T * T;
        const float *q = j->qkv + m * width + h * hd;
        float top = -INFINITY;
        for (int32_t k = 0; k < T; k++) {
            const float *key = j->qkv + (first + k) * width + (heads + kv) * hd;
            sc[k] = dotd(q, key, hd) * scale;
            top = fmaxf(top, sc[k]);
        }
        float total = 0.0f;
        for (int32_t k = 0; k < T; k++) {
            sc[k] = expf(sc[k] - top);
            total += sc[k];
        }
        for (int32_t d = 0; d < hd; d++) {
            float acc = 0.0f;
            for (int32_t k = 0; k < T; k++) acc += sc[k] * j->qkv[(first + k) * width + (heads + kvh + kv) * hd + d];
            j->out[m * (int64_t)heads * hd + h * hd + d] = f16r(acc / total);
        }
    }
}

void tgo_local_stack(const tgo_local_shape *s, const tgo_local_layer *layers, const float *final_norm,
                     int32_t seqs, const float *x, float *out) {
    const int32_t H = s->hidden, I = s->inner, hd = s->head_dim, A = s->heads * hd;
    const int32_t width = (s->heads + 2 * s->kv_heads) * hd, M = seqs * s->tokens;
    float *cur = malloc(sizeof(float) * (size_t)M * H), *mid = malloc(sizeof(float) * (size_t)M * H);
    float *normed = malloc(sizeof(float) * (size_t)M * H), *qkv = malloc(sizeof(float) * (size_t)M * width);
    float *att = malloc(sizeof(float) * (size_t)M * A), *y = malloc(sizeof(float) * (size_t)M * (I > H ? I : H));
    float *g = malloc(sizeof(float) * (size_t)M * I), *u = malloc(sizeof(float) * (size_t)M * I);
    memcpy(cur, x, sizeof(float) * (size_t)M * H);
    /* mod.rs:613-619: the first layer's input norm. */
    for (int32_t m = 0; m < M; m++) norm_row(cur + (int64_t)m * H, layers[0].input_norm, H, s->eps, normed + (int64_t)m * H);
    for (int32_t l = 0; l < s->layers; l++) {
        const tgo_local_layer *L = &layers[l];
        matmul(L->qkv, normed, qkv, M, width, H);
        rope_round(s, qkv, M);
        attn_job aj = {s, qkv, att};
        parallel_for((int64_t)M * s->heads, attn_range, &aj);
        /* o_proj and o_proj_add (local_add_norm.comp:35-47): sum = f16(residual + W att). */
        matmul(L->o, att, y, M, H, A);
        for (int64_t i = 0; i < (int64_t)M * H; i++) mid[i] = f16r(cur[i] + y[i]);
        for (int32_t m = 0; m < M; m++) norm_row(mid + (int64_t)m * H, L->post_norm, H, s->eps, normed + (int64_t)m * H);
        /* local_gate_up.comp:40-55: f16(SiLU(gate) up). */
        matmul(L->gate, normed, g, M, I, H);
        matmul(L->up, normed, u, M, I, H);
        for (int64_t i = 0; i < (int64_t)M * I; i++) g[i] = f16r(g[i] / (1.0f + expf(-g[i])) * u[i]);
        matmul(L->down, g, y, M, H, I);
        for (int64_t i = 0; i < (int64_t)M * H; i++) cur[i] = f16r(mid[i] + y[i]);
        const float *gain = l + 1 < s->layers ? layers[l + 1].input_norm : final_norm;
        for (int32_t m = 0; m < M; m++) norm_row(cur + (int64_t)m * H, gain, H, s->eps, normed + (int64_t)m * H);
    }
    memcpy(out, normed, sizeof(float) * (size_t)M * H);
    free(cur), free(mid), free(normed), free(qkv), free(att), free(y), free(g), free(u);
}

/* dit.rs:41-54, in f32 as there. */
void tgo_schedule(int32_t timesteps, float *out) {
    const int32_t steps = timesteps + 1;
    const float step = (0.0f - 1.0f) / (float)timesteps;
    const float half_pi = (float)1.57079632679489661923;
    for (int32_t i = 0; i < steps; i++) {
        const float t = i < steps / 2 ? 1.0f + step * (float)i : 0.0f - step * (float)(steps - i - 1);
        out[i] = t + (cosf(half_pi * t) - 1.0f + t);
    }
}

/* dit.rs:59-76. */
int32_t tgo_euler_steps(int32_t timesteps, float *t_out, float *dt_out) {
    const int32_t ts = timesteps < 1 ? 1 : timesteps, len = ts + 1;
    float *span = malloc(sizeof(float) * (size_t)len);
    tgo_schedule(ts, span);
    int32_t zero_init = (int32_t)((double)len * 0.04);
    if (zero_init < 1) zero_init = 1;
    float t = span[0], dt = span[0] - span[1];
    int32_t n = 0;
    for (int32_t step = 1; step < len; step++) {
        if (step > zero_init) {
            t_out[n] = t;
            dt_out[n] = dt;
            n++;
        }
        t -= dt;
        if (step < len - 1) dt = t - span[step + 1];
    }
    free(span);
    return n;
}

/* dit.rs:387-421: SinusoidalPosEmb at scale 1000 in f32, then linear_2(SiLU(linear_1(x))) in f64. */
static void sinusoid(float t, int32_t hidden, double *out) {
    const int32_t half = hidden / 2;
    const float rate = (float)(-(log(10000.0) / (double)(half - 1)));
    const float ts = t * 1000.0f;
    for (int32_t i = 0; i < half; i++) {
        const float a = ts * expf((float)i * rate);
        out[i] = (double)sinf(a);
        out[half + i] = (double)cosf(a);
    }
}

static void mlp(int32_t hidden, const float *w1, const float *b1, const float *w2, const float *b2, const double *x,
                double *out) {
    double *inner = malloc(sizeof(double) * (size_t)hidden);
    for (int32_t n = 0; n < hidden; n++) {
        double acc = 0;
        for (int32_t k = 0; k < hidden; k++) acc += (double)w1[(int64_t)n * hidden + k] * x[k];
        const double v = (double)b1[n] + acc;
        inner[n] = v / (1.0 + exp(-v));
    }
    for (int32_t n = 0; n < hidden; n++) {
        double acc = 0;
        for (int32_t k = 0; k < hidden; k++) acc += (double)w2[(int64_t)n * hidden + k] * inner[k];
        out[n] = (double)b2[n] + acc;
    }
    free(inner);
}

void tgo_time_tokens(int32_t hidden, const float *tw1, const float *tb1, const float *tw2, const float *tb2,
                     const float *dw1, const float *db1, const float *dw2, const float *db2, int32_t steps,
                     const float *times, double *out) {
    double *e = malloc(sizeof(double) * (size_t)hidden), *delta = malloc(sizeof(double) * (size_t)hidden);
    double *tok = malloc(sizeof(double) * (size_t)hidden);
    sinusoid(0.0f, hidden, e);
    mlp(hidden, dw1, db1, dw2, db2, e, delta);
    for (int32_t s = 0; s < steps; s++) {
        sinusoid(times[s], hidden, e);
        mlp(hidden, tw1, tb1, tw2, tb2, e, tok);
        for (int32_t n = 0; n < hidden; n++) out[(int64_t)s * hidden + n] = tok[n] + delta[n];
    }
    free(e), free(delta), free(tok);
}

/* local_embed.comp:42-68 for one row: `patch` frames of `src` [feat][patch] projected (W [n][feat]
 * + bias) into tokens first .. first + patch - 1 of the row's sequence `tokens_out`. */
static void embed_frames(const float *w, const float *b, const float *src, int32_t feat, int32_t patch,
                         int32_t hidden, float *tokens_out, int32_t first) {
    float *frames = malloc(sizeof(float) * (size_t)feat * patch);
    for (int32_t f = 0; f < patch; f++)
        for (int32_t c = 0; c < feat; c++) frames[f * feat + c] = f16r(src[c * patch + f]);
    for (int32_t f = 0; f < patch; f++)
        for (int32_t n = 0; n < hidden; n++)
            tokens_out[(int64_t)(first + f) * hidden + n] = f16r(b[n] + dotd(w + (int64_t)n * feat, frames + f * feat, feat));
    free(frames);
}

void tgo_sampler(const tgo_local_shape *s, const tgo_local_layer *layers, const float *final_norm,
                 const float *in_w, const float *in_b, const float *cond_w, const float *cond_b,
                 const float *out_w, const float *out_b, const float *times, const float *dts, int32_t steps,
                 int32_t rows, int32_t feat, int32_t patch, const float *mu, const float *cond,
                 const float *noise, const float *sampling, float *patch_out) {
    const int32_t H = s->hidden, T = s->tokens, len = feat * patch;
    const int32_t time_at = 2, cond_at = 3, x_at = cond_at + patch;
    const int64_t seq = (int64_t)T * H;
    float *h = calloc((size_t)rows * 2 * seq, sizeof(float)), *o = malloc(sizeof(float) * (size_t)rows * 2 * seq);
    float *v = malloc(sizeof(float) * (size_t)2 * len);
    /* cfm_noise.comp: x = temperature noise. */
    for (int32_t r = 0; r < rows; r++)
        for (int32_t i = 0; i < len; i++) patch_out[(int64_t)r * len + i] = sampling[2 * r] * noise[(int64_t)r * len + i];
    /* cond_proj (dit.rs:239-244): the patch before's frames in both sequences, mu in the first. */
    for (int32_t r = 0; r < rows; r++) {
        for (int32_t q = 0; q < 2; q++) {
            float *sq = h + ((int64_t)r * 2 + q) * seq;
            embed_frames(cond_w, cond_b, cond + (int64_t)r * len, feat, patch, H, sq, cond_at);
            for (int32_t t = 0; t < 2; t++)
                for (int32_t n = 0; n < H; n++) sq[(int64_t)t * H + n] = q == 0 ? mu[((int64_t)r * 2 + t) * H + n] : 0.0f;
        }
    }
    for (int32_t st = 0; st < steps; st++) {
        /* in_proj (dit.rs:246-252): the time token and the noisy patch in both sequences. */
        for (int32_t r = 0; r < rows; r++) {
            for (int32_t q = 0; q < 2; q++) {
                float *sq = h + ((int64_t)r * 2 + q) * seq;
                embed_frames(in_w, in_b, patch_out + (int64_t)r * len, feat, patch, H, sq, x_at);
                memcpy(sq + (int64_t)time_at * H, times + (int64_t)st * H, sizeof(float) * (size_t)H);
            }
        }
        tgo_local_stack(s, layers, final_norm, 2 * rows, h, o);
        /* dit_euler.comp: out_proj's velocities, CFG-Zero* guidance, x -= dt v. */
        for (int32_t r = 0; r < rows; r++) {
            for (int32_t q = 0; q < 2; q++)
                for (int32_t c = 0; c < feat; c++)
                    for (int32_t f = 0; f < patch; f++) {
                        const float *tok = o + ((int64_t)r * 2 + q) * seq + (int64_t)(x_at + f) * H;
                        v[q * len + c * patch + f] = dotd(out_w + (int64_t)c * H, tok, H) + out_b[c];
                    }
            double dd = 0, nn = 0;
            for (int32_t i = 0; i < len; i++) {
                dd += (double)(v[i] * v[len + i]);
                nn += (double)(v[len + i] * v[len + i]);
            }
            const float alpha = (float)dd / ((float)nn + 1e-8f), cfg = sampling[2 * r + 1];
            for (int32_t i = 0; i < len; i++) {
                const float scaled = v[len + i] * alpha;
                const float guided = scaled + cfg * (v[i] - scaled);
                patch_out[(int64_t)r * len + i] -= guided * dts[st];
            }
        }
    }
    free(h), free(o), free(v);
}

void tgo_encoder(const tgo_local_shape *s, const tgo_local_layer *layers, const float *final_norm,
                 const float *in_w, const float *in_b, const float *special, int32_t rows, int32_t feat,
                 int32_t patch, const float *patches, float *out) {
    const int32_t H = s->hidden, T = s->tokens, len = feat * patch;
    const int64_t seq = (int64_t)T * H;
    float *h = calloc((size_t)rows * seq, sizeof(float)), *o = malloc(sizeof(float) * (size_t)rows * seq);
    for (int32_t r = 0; r < rows; r++) {
        memcpy(h + r * seq, special, sizeof(float) * (size_t)H);
        embed_frames(in_w, in_b, patches + (int64_t)r * len, feat, patch, H, h + r * seq, 1);
    }
    tgo_local_stack(s, layers, final_norm, rows, h, o);
    /* local_rows.comp: the special token's output, the first of each sequence. */
    for (int32_t r = 0; r < rows; r++) memcpy(out + (int64_t)r * H, o + r * seq, sizeof(float) * (size_t)H);
    free(h), free(o);
}
