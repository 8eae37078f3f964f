/*
 * TEST INFRASTRUCTURE ONLY: the CPU oracle the parity tests and the CPU baseline use. See
 * minicpm4_ref.h for what it restates and where in tgtts-v4 each part comes from.
 */
#include "minicpm4_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define LANES 8

/* fn(ctx, lo, hi) over [0, n) cut into `threads` contiguous pieces, one pthread each. Which
 * thread takes an index never changes what is computed for it. */
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

static void parallel_for(int64_t n, int32_t threads, range_fn fn, void *ctx) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (n < 2 * threads || threads == 1) {
        fn(ctx, 0, n);
        return;
    }
    pthread_t tid[256];
    piece pieces[256];
    int32_t started = 0;
    for (int32_t t = 0; t < threads; t++) {
        pieces[t].fn = fn;
        pieces[t].ctx = ctx;
        pieces[t].lo = n * t / threads;
        pieces[t].hi = n * (t + 1) / threads;
    }
    for (int32_t t = 1; t < threads; t++) {
        if (pthread_create(&tid[t], NULL, run_piece, &pieces[t]) != 0) break;
        started = t;
    }
    run_piece(&pieces[0]);
    for (int32_t t = 1; t <= started; t++) pthread_join(tid[t], NULL);
    /* Pieces whose thread could not be started run here. */
    for (int32_t t = started + 1; t < threads; t++) run_piece(&pieces[t]);
}

/* sum_k w[k] x[k] in f32: eight running sums, lane j taking k = j mod 8, then joined
 * ((0+4)+(2+6))+((1+5)+(3+7)). A fixed order, so every caller gets the same bits. */
static float dot(const float *w, const float *x, int32_t k) {
    float acc[LANES] = {0};
    int32_t i = 0;
    for (; i + LANES <= k; i += LANES) {
        for (int j = 0; j < LANES; j++) acc[j] += w[i + j] * x[i + j];
    }
    for (; i < k; i++) acc[i % LANES] += w[i] * x[i];
    float a = (acc[0] + acc[4]) + (acc[2] + acc[6]);
    float b = (acc[1] + acc[5]) + (acc[3] + acc[7]);
    return a + b;
}

void tgo_rope_tables(int32_t head_dim, int32_t capacity, float theta, const double *factors,
                     float *cos_out, float *sin_out) {
    int32_t half = head_dim / 2;
    for (int32_t i = 0; i < half; i++) {
        /* decode.rs:149-158: inv = 1 / theta^(2i / dim) and rate = 1 / factor, both f32. */
        float inv = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
        float rate = 1.0f / (float)(factors ? factors[i] : 1.0);
        for (int32_t t = 0; t < capacity; t++) {
            float f = (float)t * rate * inv;
            cos_out[(size_t)t * half + i] = cosf(f);
            sin_out[(size_t)t * half + i] = sinf(f);
        }
    }
}

static float rms_scale(const float *x, int32_t k, float eps) {
    float sq = dot(x, x, k);
    return 1.0f / sqrtf(sq / (float)k + eps);
}

void tgo_rmsnorm(const float *x, const float *g, int32_t k, float eps, float *out) {
    float scale = rms_scale(x, k, eps);
    for (int32_t i = 0; i < k; i++) out[i] = x[i] * scale * g[i];
}

typedef struct {
    const float *a, *b;
    float *c;
    int64_t n, k;
} gemm_job;

static void gemm_range(void *p, int64_t lo, int64_t hi) {
    gemm_job *j = (gemm_job *)p;
    for (int64_t mn = lo; mn < hi; mn++) {
        int64_t i = mn / j->n, jj = mn % j->n;
        float acc = 0.0f;
        for (int64_t kk = 0; kk < j->k; kk++) acc += j->a[i * j->k + kk] * j->b[jj * j->k + kk];
        j->c[mn] = acc;
    }
}

void tgo_gemm_abt(const float *a, const float *b, float *c, int32_t m, int32_t n, int32_t k,
                  int32_t threads) {
    gemm_job j = {a, b, c, n, k};
    parallel_for((int64_t)m * n, threads, gemm_range, &j);
}

static int32_t shape_ok(const tgo_shape *s) {
    return s->hidden > 0 && s->inner > 0 && s->heads > 0 && s->kv_heads > 0 &&
           s->heads % s->kv_heads == 0 && s->head_dim > 0 && s->head_dim % 2 == 0 &&
           s->layers > 0 && s->capacity > 0 && s->slots > 0;
}

/* Where each of `rows` rows runs: its position and slot, or -1 for a spare row. */
typedef struct {
    int64_t pos, slot;
} place;

/* out[b][r] = base[b][r] + scale * (W[r] . v[b]) (or the bare product when base is NULL), for
 * the rows of `n` outputs of each of the batch's vectors: a GEMV over the batch. */
typedef struct {
    const float *w, *v, *base;
    float *out;
    float scale;
    int64_t n, k;
} gemv_job;

static void gemv_range(void *p, int64_t lo, int64_t hi) {
    gemv_job *j = (gemv_job *)p;
    for (int64_t bi = lo; bi < hi; bi++) {
        int64_t b = bi / j->n, r = bi % j->n;
        float d = dot(j->w + r * j->k, j->v + b * j->k, (int32_t)j->k);
        j->out[bi] = j->base ? j->base[bi] + j->scale * d : d;
    }
}

static void gemv(int32_t rows, const float *w, int64_t n, int64_t k, const float *v,
                 const float *base, float scale, float *out, int32_t threads) {
    gemv_job j = {w, v, base, out, scale, n, k};
    parallel_for(rows * n, threads, gemv_range, &j);
}

typedef struct {
    const tgo_shape *s;
    const tgo_layer *w;
    const place *at;
    const float *qkv;
    float *att;
} attention_job;

/* Attention of each (row, q head) over positions 0..pos: softmax of q.k / sqrt(hd), then the
 * weighted sum of v (attention_split.comp:84-111, attention_combine.comp:38-57). */
static void attention_range(void *p, int64_t lo, int64_t hi) {
    attention_job *j = (attention_job *)p;
    const tgo_shape *s = j->s;
    const int32_t hd = s->head_dim, heads = s->heads, kvh = s->kv_heads;
    const int32_t group = heads / kvh, width = (heads + 2 * kvh) * hd;
    const int64_t cap = s->capacity;
    const float scale = 1.0f / sqrtf((float)hd);
    float *p_t = malloc(sizeof(float) * (size_t)cap);
    for (int64_t bh = lo; bh < hi; bh++) {
        int64_t b = bh / heads, h = bh % heads;
        float *o = j->att + bh * hd;
        for (int32_t d = 0; d < hd; d++) o[d] = 0.0f;
        if (j->at[b].pos < 0) continue;
        int64_t pos = j->at[b].pos, kv = h / group;
        const float *q = j->qkv + b * width + h * hd;
        const float *kc = j->w->k_cache + (size_t)((j->at[b].slot * kvh + kv) * cap) * hd;
        const float *vc = j->w->v_cache + (size_t)((j->at[b].slot * kvh + kv) * cap) * hd;
        float m = -INFINITY;
        for (int64_t t = 0; t <= pos; t++) {
            p_t[t] = dot(q, kc + t * hd, hd) * scale;
            if (p_t[t] > m) m = p_t[t];
        }
        float l = 0.0f;
        for (int64_t t = 0; t <= pos; t++) {
            p_t[t] = expf(p_t[t] - m);
            l += p_t[t];
        }
        for (int64_t t = 0; t <= pos; t++) {
            for (int32_t d = 0; d < hd; d++) o[d] += p_t[t] * vc[t * hd + d];
        }
        for (int32_t d = 0; d < hd; d++) o[d] /= l;
    }
    free(p_t);
}

/*
 * One layer over `n` rows whose places are `at`, from the residual stream x (updated in place,
 * [n][hidden]). Per row (crates/graph/src/decode.rs:667-712):
 *   xn = RMSNorm(x) g_in; [q;k;v] = W_qkv xn; q, k rotated by RoPE at the row's position;
 *   k, v written into the cache at (slot, position); attention of each q head over the cache
 *   positions 0..position of its kv head; mid = x + s W_o att; mn = RMSNorm(mid) g_post;
 *   mlp = SiLU(W_gate mn) (W_up mn); x = mid + s W_down mlp.
 * Every row's k and v are written before any row attends, which is how a prefill runs a layer
 * over its rows (prefill.rs:366-377) and makes no difference to a decode step, whose rows are in
 * distinct slots. So a prefill of n positions gives the same bits as n decode steps.
 */
static void layer_rows(const tgo_shape *s, const tgo_layer *w, int32_t n, const place *at,
                       float *x, int32_t threads) {
    const int32_t H = s->hidden, I = s->inner, hd = s->head_dim, half = hd / 2;
    const int32_t heads = s->heads, kvh = s->kv_heads;
    const int32_t width = (heads + 2 * kvh) * hd;
    const int64_t cap = s->capacity;
    float *xn = malloc(sizeof(float) * (size_t)n * H);
    float *qkv = malloc(sizeof(float) * (size_t)n * width);
    float *att = malloc(sizeof(float) * (size_t)n * heads * hd);
    float *gu = malloc(sizeof(float) * (size_t)n * 2 * I);
    float *mlp = malloc(sizeof(float) * (size_t)n * I);

    for (int32_t b = 0; b < n; b++)
        tgo_rmsnorm(x + (size_t)b * H, w->input_norm, H, s->eps, xn + (size_t)b * H);
    gemv(n, w->qkv, width, H, xn, NULL, 0.0f, qkv, threads);
    /* RoPE on row pairs (i, i + hd/2) of each q and k head (gemv_qkv_rope.comp:82-104), and the
     * cache writes at ((slot * kv + h) * cap + pos) * hd + i. */
    for (int32_t b = 0; b < n; b++) {
        if (at[b].pos < 0) continue;
        int64_t pos = at[b].pos, slot = at[b].slot;
        float *r = qkv + (size_t)b * width;
        for (int32_t h = 0; s->rope && h < heads + kvh; h++) {
            for (int32_t i = 0; i < half; i++) {
                float a = r[h * hd + i], c = r[h * hd + i + half];
                float co = s->cos[pos * half + i], si = s->sin[pos * half + i];
                r[h * hd + i] = a * co - c * si;
                r[h * hd + i + half] = c * co + a * si;
            }
        }
        for (int32_t h = 0; h < kvh; h++) {
            size_t to = (size_t)(((slot * kvh + h) * cap + pos) * hd);
            memcpy(w->k_cache + to, r + (heads + h) * hd, sizeof(float) * hd);
            memcpy(w->v_cache + to, r + (heads + kvh + h) * hd, sizeof(float) * hd);
        }
    }
    attention_job aj = {s, w, at, qkv, att};
    parallel_for((int64_t)n * heads, threads, attention_range, &aj);
    /* mid = x + s W_o att (gemv_residual.comp:38-44, plus the residual scale). */
    gemv(n, w->o, H, (int64_t)heads * hd, att, x, s->residual_scale, x, threads);
    for (int32_t b = 0; b < n; b++)
        tgo_rmsnorm(x + (size_t)b * H, w->post_norm, H, s->eps, xn + (size_t)b * H);
    gemv(n, w->gate_up, 2 * (int64_t)I, H, xn, NULL, 0.0f, gu, threads);
    for (int64_t bi = 0; bi < (int64_t)n * I; bi++) {
        int64_t b = bi / I, i = bi % I;
        float g = gu[b * 2 * I + i], u = gu[b * 2 * I + I + i];
        mlp[bi] = g / (1.0f + expf(-g)) * u;
    }
    gemv(n, w->down, H, I, mlp, x, s->residual_scale, x, threads);
    free(xn);
    free(qkv);
    free(att);
    free(gu);
    free(mlp);
}

static void final_norm(const tgo_shape *s, const float *g, int32_t n, const place *at,
                       const float *x, float *out) {
    for (int32_t b = 0; b < n; b++) {
        float *o = out + (size_t)b * s->hidden;
        if (at[b].pos < 0) {
            memset(o, 0, sizeof(float) * s->hidden);
            continue;
        }
        tgo_rmsnorm(x + (size_t)b * s->hidden, g, s->hidden, s->eps, o);
    }
}

int32_t tgo_decode_step(const tgo_shape *s, const tgo_layer *layers, const float *final_norm_g,
                        int32_t rows, const uint32_t *position, const uint32_t *slot,
                        const float *x, float *out, int32_t threads) {
    if (!shape_ok(s) || rows <= 0) return -1;
    place *at = malloc(sizeof(place) * rows);
    for (int32_t b = 0; b < rows; b++) {
        uint32_t sl = s->slots > 1 ? slot[b] : 0;
        if (position[b] >= (uint32_t)s->capacity || sl >= (uint32_t)s->slots) {
            at[b].pos = -1;
            at[b].slot = -1;
        } else {
            at[b].pos = position[b];
            at[b].slot = sl;
        }
    }
    float *h = malloc(sizeof(float) * (size_t)rows * s->hidden);
    memcpy(h, x, sizeof(float) * (size_t)rows * s->hidden);
    for (int32_t l = 0; l < s->layers; l++) layer_rows(s, &layers[l], rows, at, h, threads);
    final_norm(s, final_norm_g, rows, at, h, out);
    free(h);
    free(at);
    return 0;
}

int32_t tgo_prefill(const tgo_shape *s, const tgo_layer *layers, const float *final_norm_g,
                    uint32_t start, uint32_t len, uint32_t slot, const float *x, float *out,
                    int32_t threads) {
    if (!shape_ok(s) || len == 0 || (uint64_t)start + len > (uint64_t)s->capacity ||
        slot >= (uint32_t)s->slots)
        return -1;
    place *at = malloc(sizeof(place) * len);
    for (uint32_t r = 0; r < len; r++) {
        at[r].pos = start + r;
        at[r].slot = slot;
    }
    float *h = malloc(sizeof(float) * (size_t)len * s->hidden);
    memcpy(h, x, sizeof(float) * (size_t)len * s->hidden);
    for (int32_t l = 0; l < s->layers; l++) layer_rows(s, &layers[l], (int32_t)len, at, h, threads);
    final_norm(s, final_norm_g, (int32_t)len, at, h, out);
    free(h);
    free(at);
    return 0;
}

void tgo_gemv_linear(const float *x0, const float *x1, const float *w, const float *bias, float *out,
                     int32_t rows, int32_t n, int32_t k0, int32_t k1, int32_t offset, int32_t stride,
                     int32_t act, float levels) {
    const int64_t k = (int64_t)k0 + k1;
    for (int32_t b = 0; b < rows; b++) {
        for (int32_t i = 0; i < n; i++) {
            const float *wr = w + (int64_t)i * k;
            float acc = 0.0f;
            for (int64_t c = 0; c < k0; c++) acc = fmaf(wr[c], x0[(int64_t)b * k0 + c], acc);
            for (int64_t c = 0; c < k1; c++) acc = fmaf(wr[k0 + c], x1[(int64_t)b * k1 + c], acc);
            float v = acc + bias[i];
            if (act == 1) {
                v = v / (1.0f + expf(-v));
            } else if (act == 2) {
                const float t = 1.0f - 2.0f / (expf(2.0f * fabsf(v)) + 1.0f);
                v = rintf(copysignf(t, v) * levels) / levels;
            }
            out[(int64_t)b * stride + offset + i] = v;
        }
    }
}
