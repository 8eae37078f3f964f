// The MiniCPM-4 stack over the runtime: its shape and byte model (crates/graph/src/decode.rs:66-168),
// placements (decode.rs:171-235), the decode step recorded once per batch (decode.rs:457-736,
// :778-913) and the prefill programs over the decoder's weights and cache (prefill.rs:181-504).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>

#include "model.h"
#include "tg_common.cuh"

using namespace tg;

// ---- shape ----------------------------------------------------------------------------------------

extern "C" uint64_t tg_shape_weight_bytes(const tg_shape *s, uint32_t bytes_per_weight) {
    if (!s) return 0;
    const uint64_t h = s->hidden, i = s->inner, d = s->head_dim;
    const uint64_t qkv = (uint64_t)(s->heads + 2 * s->kv_heads) * d * h;
    const uint64_t layer = qkv + (uint64_t)s->heads * d * h + 2 * i * h + i * h + 2 * h;
    return (uint64_t)bytes_per_weight * ((uint64_t)s->layers * layer + h);
}

extern "C" uint64_t tg_shape_cache_bytes(const tg_shape *s, uint32_t position, uint32_t bytes_per_value) {
    if (!s) return 0;
    // decode.rs:137-141: positions 0 .. position in whole CHUNKs of 32, as the reference's kernels
    // read them, at most the capacity.
    const uint64_t chunked = ((uint64_t)position + CAPACITY_STEP) / CAPACITY_STEP * CAPACITY_STEP;
    const uint64_t read = std::min<uint64_t>(chunked, s->capacity);
    return (uint64_t)s->layers * 2 * s->kv_heads * read * s->head_dim * bytes_per_value;
}

static void rope_tables(const tg_shape &s, const double *factors, float *cs, float *sn) {
    const uint32_t half = s.head_dim / 2;
    for (uint32_t i = 0; i < half; i++) {
        // 1 / theta^(2i / dim) and 1 / factor in f32, then t * rate * inv (decode.rs:146-168).
        const float inv = 1.0f / powf(s.rope_theta, (float)(2 * i) / (float)s.head_dim);
        const float rate = 1.0f / (float)(factors ? factors[i] : 1.0);
        for (uint32_t t = 0; t < s.capacity; t++) {
            const float f = (float)t * rate * inv;
            cs[(size_t)t * half + i] = cosf(f);
            sn[(size_t)t * half + i] = sinf(f);
        }
    }
}

extern "C" int tg_shape_rope_tables(const tg_shape *s, float *cs, float *sn) {
    if (!s || !cs || !sn) return fail(TG_EINVAL, "tg_shape_rope_tables: null argument");
    rope_tables(*s, s->rope_factors, cs, sn);
    return TG_OK;
}

extern "C" int tg_batch_placement(uint32_t n_rows, uint32_t slots, const tg_row *rows, uint32_t capacity,
                                  uint32_t *words, uint32_t *n_words) {
    if ((n_rows && (!rows || !words)) || slots == 0) return fail(TG_EINVAL, "tg_batch_placement: null argument");
    const uint32_t nw = slots > 1 ? 2 * n_rows : n_rows;
    for (uint32_t i = 0; i < nw; i++) words[i] = TG_SPARE;
    std::vector<bool> taken(slots, false);
    for (uint32_t b = 0; b < n_rows; b++) {
        const tg_row r = rows[b];
        if (r.position == TG_SPARE) continue;
        if (r.position >= capacity || r.slot >= slots || taken[r.slot])
            return fail(TG_ESHAPE, "row %u at position %u of %u in slot %u of %u, taken: %s", b, r.position, capacity,
                        r.slot, slots, r.slot < slots && taken[r.slot] ? "true" : "false");
        taken[r.slot] = true;
        words[b] = r.position;
        if (slots > 1) words[n_rows + b] = r.slot;
    }
    if (n_words) *n_words = nw;
    return TG_OK;
}

// ---- decoder --------------------------------------------------------------------------------------

static int check_shape(const tg_shape &s, tg_dtype dtype) {
    const uint32_t vec = dtype == TG_BF16 ? 256 : 128;
    if (dtype != TG_F32 && dtype != TG_BF16) return fail(TG_ESHAPE, "dtype %d", (int)dtype);
    if (s.layers == 0 || s.hidden == 0 || s.inner == 0 || s.heads == 0 || s.kv_heads == 0)
        return fail(TG_ESHAPE, "an empty shape");
    if (s.hidden % vec || s.inner % vec || (s.heads * s.head_dim) % vec)
        return fail(TG_ESHAPE, "%u hidden, %u inner and %u attention columns in steps of %u", s.hidden, s.inner,
                    s.heads * s.head_dim, vec);
    if (s.heads % s.kv_heads || s.heads / s.kv_heads > MAX_GROUP || (s.head_dim != 64 && s.head_dim != 128))
        return fail(TG_ESHAPE, "%u heads over %u of %u", s.heads, s.kv_heads, s.head_dim);
    if (s.inner % GU_BLOCK) return fail(TG_ESHAPE, "inner %u is not a multiple of %u", s.inner, GU_BLOCK);
    if (s.capacity == 0 || s.capacity % CAPACITY_STEP)
        return fail(TG_ESHAPE, "a cache of %u positions (a multiple of %u)", s.capacity, CAPACITY_STEP);
    if (!(s.eps >= 0.0f) || !std::isfinite(s.residual_scale)) return fail(TG_ESHAPE, "eps %g, residual scale %g", s.eps, s.residual_scale);
    return TG_OK;
}

static void push(std::vector<Launch> &v, uint32_t kernel, const tg_params &p, const char *label,
                 std::initializer_list<std::pair<void *, uint64_t>> b) {
    Launch l;
    l.kernel = kernel;
    l.p = p;
    l.label = label;
    for (auto &x : b) {
        l.ptr.push_back(x.first);
        l.bytes.push_back(x.second);
    }
    v.push_back(std::move(l));
}

// The GEMM family's step for R rows (bf16, R >= DTC_MIN_ROWS): the prefill's chain of kernels
// (prefill.rs:318-411) over rows that are each a run of one position in its own slot, with the
// decode attention in place of attention_rows: per layer the q/k/v GEMM with RoPE and the cache
// append in its epilogue, attention_split (mma.sync) and attention_combine, the o GEMM, the
// residual add with the post-attention norm, the gate/up GEMM with SiLU-mul in its epilogue, the
// down GEMM, and the residual add with the next layer's input norm (the last layer's with the final
// norm, in f32). Activations between them are bf16 where a GEMM reads them, the residual stream f32.
// Every GEMM's B is a weight, so its first tiles stream while the kernel before it finishes.
// The parts of K a batched decode step's o and down GEMMs are cut into (n outputs of k): the most,
// a power of two, that keeps the 64-column tiles within one wave of B200's 148 SMs. The shape
// alone fixes it, so a row's sums do not depend on the bucket.
static uint32_t decode_gemm_parts(uint64_t n, uint64_t k) {
    uint32_t parts = 1;
    while ((n / 64) * parts * 2 <= 148 && (k / 64) % (parts * 2) == 0) parts *= 2;
    return parts;
}

static std::vector<Launch> decode_gemm_launches(tg_decoder &d, uint32_t R) {
    const tg_params base = d.params(R);
    const tg_shape &s = d.shape;
    const uint64_t T = d.esize, F = 4, H = s.hidden, I = s.inner, hd = s.head_dim, heads = s.heads;
    const uint64_t W = d.width(), A = d.attn(), chunks = attn_chunks(s.capacity);
    const uint64_t words = (d.slots > 1 ? 2 : 1) * (uint64_t)R * 4;
    const uint64_t table = (uint64_t)s.capacity * (hd / 2) * F;
    std::vector<Launch> v;
    const uint32_t o_parts = decode_gemm_parts(H, A), down_parts = decode_gemm_parts(H, I);
    auto gemm = [&](uint32_t kernel, const char *label, void *a, void *b, void *c, uint64_t c_bytes, uint64_t n,
                    uint64_t k, uint32_t parts = 1) {
        tg_params g = base;
        g.m = R;
        g.n = (uint32_t)n;
        g.k = (uint32_t)k;
        g.parts = parts;
        g.flags = 1 | 2;  // b a weight; narrow tiles
        push(v, kernel, g, label, {{a, R * k * T}, {b, n * k * T}, {c, c_bytes}});
    };
    push(v, TG_KERNEL_NORM_ROWS, base, "input_norm",
         {{d.words.ptr(), words}, {d.x_in.ptr(), R * H * F}, {d.w(d.layer[0].in_norm), H * F}, {d.g_normed.ptr(), R * H * T}});
    for (uint32_t l = 0; l < s.layers; l++) {
        const LayerOffsets &o = d.layer[l];
        char *in = l == 0 ? d.x_in.ptr() : d.h.ptr();
        {
            tg_params g = base;
            g.m = R;
            g.n = (uint32_t)W;
            g.k = (uint32_t)H;
            g.flags = 2;  // narrow tiles: one head a tile
            push(v, TG_KERNEL_GEMM_QKV_ROPE, g, "qkv_proj",
                 {{d.g_normed.ptr(), R * H * T}, {d.w(o.qkv), W * H * T}, {d.words.ptr(), words}, {d.cos.ptr(), table},
                  {d.sin.ptr(), table}, {d.g_q.ptr(), R * A * T}, {d.kc(l), d.cache_layer}, {d.vc(l), d.cache_layer}});
        }
        // attention_split and attention_combine in one launch.
        push(v, KERNEL_ATTN_SPLIT_JOIN, base, "attention",
             {{d.g_q.ptr(), R * A * F}, {d.kc(l), d.cache_layer}, {d.vc(l), d.cache_layer}, {d.words.ptr(), words},
              {d.po.ptr(), R * heads * chunks * hd * F}, {d.pml.ptr(), R * heads * chunks * 2 * F},
              {d.g_att.ptr(), R * A * 2}, {d.g_counts.ptr(), R * s.kv_heads * 4}});
        // o and down in parts of K, each part's sums added by the add_norm after it.
        gemm(TG_KERNEL_GEMM, "o_proj", d.g_att.ptr(), d.w(o.o), d.g_proj.ptr(), o_parts * R * H * F, H, A, o_parts);
        tg_params on = base;
        on.parts = o_parts;
        on.flags = 2;  // few rows: a block to a row
        push(v, TG_KERNEL_ADD_NORM_ROWS, on, "add_norm",
             {{d.words.ptr(), words}, {d.g_proj.ptr(), o_parts * R * H * F}, {in, R * H * F}, {d.w(o.post_norm), H * F},
              {d.mid.ptr(), R * H * F}, {d.g_normed.ptr(), R * H * T}});
        gemm(TG_KERNEL_GEMM_SILU, "gate_up", d.g_normed.ptr(), d.w(o.gate_up), d.g_mlp.ptr(), R * I * T, 2 * I, H);
        gemm(TG_KERNEL_GEMM, "down_proj", d.g_mlp.ptr(), d.w(o.down), d.g_proj.ptr(), down_parts * R * H * F, H, I,
             down_parts);
        const bool last = l + 1 == s.layers;
        tg_params an = base;
        an.normed_f32 = last ? 1 : 0;
        an.parts = down_parts;
        an.flags = 2;
        push(v, TG_KERNEL_ADD_NORM_ROWS, an, last ? "final_norm" : "add_norm",
             {{d.words.ptr(), words}, {d.g_proj.ptr(), down_parts * R * H * F}, {d.mid.ptr(), R * H * F},
              {d.w(last ? d.final_norm : d.layer[l + 1].in_norm), H * F}, {d.h.ptr(), R * H * F},
              {last ? d.out.ptr() : d.g_normed.ptr(), R * H * (last ? F : T)}});
    }
    return v;
}

// Whether a decoder's shape and rows take the GEMM family (the prefill GEMMs' tiles and epilogues,
// the batched attention).
static bool gemm_family_supported(const tg_decoder &d) {
    const tg_shape &s = d.shape;
    return d.dtype == TG_BF16 && d.rows >= DTC_MIN_ROWS && d.width() % 256 == 0 && (2 * (uint64_t)s.inner) % 256 == 0 &&
           s.hidden % 64 == 0 && s.inner % 64 == 0 && d.attn() % 64 == 0 && 256 % s.head_dim == 0 &&
           attention_split_mma_supported(d.params(d.rows));
}

// decode_batch_graph (decode.rs:457-736): per layer qkv_rope, attention_split, attention_combine,
// o_proj (+ residual), gate_up (+ norm, SiLU), down_proj (+ residual); then the final norm.
static std::vector<Launch> decode_launches(tg_decoder &d, uint32_t R) {
    const tg_params base = d.params(R);
    std::vector<Launch> v;
    if (d.persistent) {
        Launch l;
        l.kernel = KERNEL_DECODE_STEP;
        l.p = base;
        l.label = "decode_step";
        DecodeStep &st = l.step;
        st.p = base;
        st.layers = (int)d.shape.layers;
        st.weights = reinterpret_cast<const unsigned char *>(d.weights.ptr());
        st.offs = reinterpret_cast<const uint64_t *>(d.offs.ptr());
        st.final_norm = d.final_norm;
        st.cosv = reinterpret_cast<const float *>(d.cos.ptr());
        st.sinv = reinterpret_cast<const float *>(d.sin.ptr());
        st.at = reinterpret_cast<const uint32_t *>(d.words.ptr());
        st.x_in = reinterpret_cast<const float *>(d.x_in.ptr());
        st.h = reinterpret_cast<float *>(d.h.ptr());
        st.mid = reinterpret_cast<float *>(d.mid.ptr());
        st.mlp = reinterpret_cast<float *>(d.mlp.ptr());
        st.q = reinterpret_cast<float *>(d.q.ptr());
        st.att = reinterpret_cast<float *>(d.att.ptr());
        st.out = reinterpret_cast<float *>(d.out.ptr());
        st.po = reinterpret_cast<float *>(d.po.ptr());
        st.pml = reinterpret_cast<float *>(d.pml.ptr());
        st.kcache = reinterpret_cast<unsigned char *>(d.kcache.ptr());
        st.vcache = reinterpret_cast<unsigned char *>(d.vcache.ptr());
        st.cache_layer = d.cache_layer;
        st.sync = reinterpret_cast<uint32_t *>(d.psync.ptr());
        st.err = d.ctx->err_dev;
        v.push_back(l);
        return v;
    }
    const uint64_t T = d.esize, F = 4;
    const tg_shape &s = d.shape;
    const uint64_t H = s.hidden, I = s.inner, hd = s.head_dim, heads = s.heads;
    const uint64_t chunks = attn_chunks(s.capacity);
    const uint64_t words = (d.slots > 1 ? 2 : 1) * (uint64_t)R * 4;
    const uint64_t table = (uint64_t)s.capacity * (hd / 2) * F;
    if (d.tensor && d.gemm) return decode_gemm_launches(d, R);
    for (uint32_t l = 0; l < s.layers; l++) {
        const LayerOffsets &o = d.layer[l];
        char *in = l == 0 ? d.x_in.ptr() : d.h.ptr();
        push(v, d.tensor ? KERNEL_DTC_QKV_ROPE : (uint32_t)TG_KERNEL_GEMV_QKV_ROPE, base, "qkv_rope",
             {{in, R * H * F}, {d.w(o.in_norm), H * F}, {d.w(o.qkv), d.width() * H * T}, {d.cos.ptr(), table},
              {d.sin.ptr(), table}, {d.words.ptr(), words}, {d.q.ptr(), R * d.attn() * F},
              {d.kc(l), d.cache_layer}, {d.vc(l), d.cache_layer}});
        const bool wide = d.tensor && attention_split_mma_supported(base);
        push(v, wide ? KERNEL_ATTN_SPLIT_MMA : (uint32_t)TG_KERNEL_ATTENTION_SPLIT, base, "attention_split",
             {{d.q.ptr(), R * d.attn() * F}, {d.kc(l), d.cache_layer}, {d.vc(l), d.cache_layer},
              {d.words.ptr(), words}, {d.po.ptr(), R * heads * chunks * hd * F},
              {d.pml.ptr(), R * heads * chunks * 2 * F}});
        push(v, wide ? KERNEL_ATTN_COMBINE_WIDE : (uint32_t)TG_KERNEL_ATTENTION_COMBINE, base, "attention_combine",
             {{d.words.ptr(), words}, {d.po.ptr(), R * heads * chunks * hd * F},
              {d.pml.ptr(), R * heads * chunks * 2 * F}, {d.att.ptr(), R * d.attn() * F}});
        tg_params po = base;
        po.n = (uint32_t)H;
        po.k = (uint32_t)d.attn();
        push(v, d.tensor ? KERNEL_DTC_RESIDUAL : (uint32_t)TG_KERNEL_GEMV_RESIDUAL, po, "o_proj",
             {{d.att.ptr(), R * d.attn() * F}, {d.w(o.o), H * d.attn() * T}, {in, R * H * F}, {d.mid.ptr(), R * H * F}});
        push(v, d.tensor ? KERNEL_DTC_GATE_UP : (uint32_t)TG_KERNEL_GEMV_GATE_UP, base, "gate_up",
             {{d.mid.ptr(), R * H * F}, {d.w(o.post_norm), H * F}, {d.w(o.gate_up), 2 * I * H * T},
              {d.mlp.ptr(), R * I * F}});
        tg_params pd = base;
        pd.n = (uint32_t)H;
        pd.k = (uint32_t)I;
        const bool tc_down = d.tensor && dtc_residual_supported(d.params(d.rows), (int)I);
        push(v, tc_down ? KERNEL_DTC_RESIDUAL : (uint32_t)TG_KERNEL_GEMV_RESIDUAL, pd, "down_proj",
             {{d.mlp.ptr(), R * I * F}, {d.w(o.down), H * I * T}, {d.mid.ptr(), R * H * F}, {d.h.ptr(), R * H * F}});
    }
    push(v, TG_KERNEL_RMSNORM, base, "final_norm",
         {{d.h.ptr(), R * H * F}, {d.w(d.final_norm), H * F}, {d.out.ptr(), R * H * F}});
    return v;
}

namespace tg {

std::vector<uint32_t> program_rows(uint32_t rows) {
    std::vector<uint32_t> out;
    for (uint32_t r = 1; r < rows; r *= 2) out.push_back(r);
    out.push_back(rows);
    return out;
}

size_t bucket_for(const tg_decoder &d, uint32_t n) {
    for (size_t i = 0; i < d.buckets.size(); i++)
        if (d.buckets[i].rows >= n) return i;
    return d.buckets.size() - 1;
}

int decoder_place(tg_decoder &d, size_t b, uint32_t n, const tg_row *rows) {
    const uint32_t R = d.buckets[b].rows;
    std::vector<tg_row> all(R, tg_row{TG_SPARE, 0});
    std::copy(rows, rows + n, all.begin());
    uint32_t nw = 0;
    size_t i = 0;
    TG_TRY(d.word_ring.acquire(i));
    TG_TRY(tg_batch_placement(R, d.slots, all.data(), d.shape.capacity, static_cast<uint32_t *>(d.word_ring.host(i)),
                              &nw));
    TG_TRY(d.word_ring.upload(i, d.words.ptr(), (uint64_t)nw * 4, d.ctx->stream));
    d.active = b;
    d.n_active = n;
    return TG_OK;
}

}  // namespace tg

static int record_step(tg_decoder &d, bool persistent);

extern "C" int tg_decoder_create(tg_ctx *ctx, const tg_shape *s, uint32_t rows, uint32_t slots, tg_dtype dtype,
                                 int timed, tg_decoder **out) {
    if (!ctx || !s || !out) return fail(TG_EINVAL, "tg_decoder_create: null argument");
    *out = nullptr;
    TG_TRY(check_shape(*s, dtype));
    if (rows == 0 || rows > slots) return fail(TG_ESHAPE, "%u rows in %u slots", rows, slots);
    TG_CUDA(cudaSetDevice(ctx->device));
    std::unique_ptr<tg_decoder> d(new tg_decoder());
    d->ctx = ctx;
    d->shape = *s;
    if (s->rope_factors) d->factors.assign(s->rope_factors, s->rope_factors + s->head_dim / 2);
    d->shape.rope_factors = nullptr;
    d->rows = rows;
    d->slots = slots;
    d->dtype = dtype;
    d->timed = timed != 0;
    d->esize = dtype == TG_BF16 ? 2 : 4;
    const uint64_t T = d->esize, F = 4, H = s->hidden, I = s->inner;
    uint64_t off = 0;
    for (uint32_t l = 0; l < s->layers; l++) {
        LayerOffsets o;
        o.qkv = off;
        off = align256(off + d->width() * H * T);
        o.o = off;
        off = align256(off + H * d->attn() * T);
        o.gate_up = off;
        off = align256(off + 2 * I * H * T);
        o.down = off;
        off = align256(off + H * I * T);
        o.in_norm = off;
        off = align256(off + H * F);
        o.post_norm = off;
        off = align256(off + H * F);
        d->layer.push_back(o);
    }
    d->final_norm = off;
    off = align256(off + H * F);
    TG_TRY(d->weights.alloc(ctx, off));
    const uint64_t table = (uint64_t)s->capacity * (s->head_dim / 2) * F;
    TG_TRY(d->cos.alloc(ctx, table));
    TG_TRY(d->sin.alloc(ctx, table));
    {
        std::vector<float> cs(table / 4), sn(table / 4);
        rope_tables(d->shape, d->factors.empty() ? nullptr : d->factors.data(), cs.data(), sn.data());
        TG_TRY(tg_mem_write(d->cos.m, 0, cs.data(), table));
        TG_TRY(tg_mem_write(d->sin.m, 0, sn.data(), table));
    }
    d->cache_layer = align256((uint64_t)slots * s->kv_heads * s->capacity * s->head_dim * T);
    TG_TRY(d->kcache.alloc(ctx, d->cache_layer * s->layers));
    TG_TRY(d->vcache.alloc(ctx, d->cache_layer * s->layers));
    const uint64_t R = rows, chunks = attn_chunks(s->capacity);
    TG_TRY(d->x_in.alloc(ctx, R * H * F));
    TG_TRY(d->h.alloc(ctx, R * H * F));
    TG_TRY(d->mid.alloc(ctx, R * H * F));
    TG_TRY(d->out.alloc(ctx, R * H * F));
    TG_TRY(d->q.alloc(ctx, R * d->attn() * F));
    TG_TRY(d->att.alloc(ctx, R * d->attn() * F));
    TG_TRY(d->mlp.alloc(ctx, R * I * F));
    TG_TRY(d->words.alloc(ctx, 2 * R * 4));
    TG_TRY(d->po.alloc(ctx, R * s->heads * chunks * s->head_dim * F));
    TG_TRY(d->pml.alloc(ctx, R * s->heads * chunks * 2 * F));
    TG_TRY(d->psync.alloc(ctx, decode_step_flag_bytes((int)s->layers)));
    {
        std::vector<uint64_t> offs;
        for (const LayerOffsets &o : d->layer) {
            for (uint64_t v : {o.qkv, o.o, o.gate_up, o.down, o.in_norm, o.post_norm}) offs.push_back(v);
        }
        TG_TRY(d->offs.alloc(ctx, offs.size() * 8));
        TG_TRY(tg_mem_write(d->offs.m, 0, offs.data(), offs.size() * 8));
    }
    TG_TRY(d->stage_x.alloc(ctx, R * H * F, TG_RES_UPLOAD));
    TG_TRY(d->word_ring.init(ctx, 8, 2 * R * 4));
    TG_TRY(d->stage_out.alloc(ctx, R * H * F, TG_RES_READBACK));
    TG_CUDA(cudaEventCreateWithFlags(&d->out_done, cudaEventDisableTiming));
    TG_TRY(tg_mem_fill(d->words.m, 0, TG_SPARE, 2 * R * 4));
    // A decoder of DTC_MIN_ROWS rows or more runs its projections on tcgen05 in every bucket (so that
    // a row's bits do not depend on the bucket); smaller ones run the GEMVs.
    // Both tcgen05 forms are recorded on request; by default the GEMMs, where they take the shape
    // (on B200 a step at 16 / 64 / 128 rows: 1.16 / 1.44 / 1.77 ms against 1.25 / 1.99 / 3.29 ms as
    // split-K clusters).
    const bool gemm_ok = gemm_family_supported(*d);
    const bool dtc_ok = dtype == TG_BF16 && rows >= DTC_MIN_ROWS && dtc_supported(d->params(rows));
    d->gemm = gemm_ok;
    d->tensor = dtype == TG_BF16 && rows >= DTC_MIN_ROWS && (gemm_ok || dtc_ok);
    if (gemm_ok) {
        TG_TRY(d->g_normed.alloc(ctx, R * H * 2));
        TG_TRY(d->g_q.alloc(ctx, R * d->attn() * F));  // bf16 values, sized as the checks size f32 q
        TG_TRY(d->g_att.alloc(ctx, R * d->attn() * F));
        const uint64_t parts = std::max(decode_gemm_parts(H, d->attn()), decode_gemm_parts(H, I));
        TG_TRY(d->g_proj.alloc(ctx, parts * R * H * F));
        TG_TRY(d->g_mlp.alloc(ctx, R * I * 2));
        TG_TRY(d->g_counts.alloc(ctx, R * s->kv_heads * 4));
    }
    // A bf16 decoder of one or two rows records its step as the one persistent launch (on B200
    // 0.61-0.63 ms a step at config 2 against 0.67-0.70 ms for six kernels a layer, the same bits);
    // anything else as six kernels a layer. tg_decoder_retune selects either.
    TG_TRY(record_step(*d, dtype == TG_BF16 && rows <= 2 && !d->tensor));
    *out = d.release();
    return TG_OK;
}

// Records every bucket's step as one persistent launch or as six kernels a layer. A persistent
// recording the device or shape does not take falls back to the kernels (the same results bit for
// bit).
static int record_buckets(tg_decoder &d) {
    for (Bucket &b : d.buckets) {
        program_release(b.prog);
        b.prog = Program();
        b.launches = decode_launches(d, b.rows);
        TG_TRY(program_build(d.ctx, b.launches, d.timed, b.prog));
    }
    return TG_OK;
}

static int record_step(tg_decoder &d, bool persistent) {
    TG_TRY(d.wait_pending());
    if (d.buckets.empty())
        for (uint32_t r : program_rows(d.rows)) {
            d.buckets.emplace_back();
            d.buckets.back().rows = r;
        }
    d.persistent = persistent;
    int st = record_buckets(d);
    if (st != TG_OK && persistent) {
        d.persistent = false;
        st = record_buckets(d);
    }
    return st;
}

extern "C" int tg_decoder_retune(tg_decoder *d, int persistent, int timed) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    TG_CUDA(cudaSetDevice(d->ctx->device));
    d->timed = timed != 0;
    TG_TRY(record_step(*d, persistent != 0));
    if (persistent && !d->persistent) return fail(TG_ESHAPE, "this decoder's batch or shape has no persistent step");
    return TG_OK;
}

extern "C" int tg_decoder_persistent(const tg_decoder *d) { return d && d->persistent ? 1 : 0; }

extern "C" int tg_decoder_tensor(const tg_decoder *d) { return d && d->tensor ? (d->gemm ? 1 : 2) : 0; }

extern "C" int tg_decoder_set_tensor(tg_decoder *d, int tensor) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    if (tensor < 0 || tensor > 2) return fail(TG_EINVAL, "tg_decoder_set_tensor: %d", tensor);
    if (tensor == 1 && !(d->g_normed.m || (d->dtype == TG_BF16 && dtc_supported(d->params(d->rows)))))
        return fail(TG_ESHAPE, "no tcgen05 projections for this decoder's dtype or shape");
    if (tensor == 2 && !(d->dtype == TG_BF16 && dtc_supported(d->params(d->rows))))
        return fail(TG_ESHAPE, "no split-K tcgen05 projections for this decoder's dtype or shape");
    TG_CUDA(cudaSetDevice(d->ctx->device));
    d->tensor = tensor != 0;
    d->gemm = tensor == 1 && d->g_normed.m != nullptr;
    return record_step(*d, d->persistent && !d->tensor);
}

extern "C" int tg_decoder_destroy(tg_decoder *d) {
    if (!d) return TG_OK;
    cudaSetDevice(d->ctx->device);
    d->wait_pending();
    delete d;
    return TG_OK;
}

__global__ void to_bf16_kernel(const float *__restrict__ src, bf16 *__restrict__ dst, uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

// Writes `count` values from the host into the weight arena at `off`, in the decoder's storage
// type (`as_f32` forces f32, for gains): f32 to bf16 rounds to nearest even on the GPU
// (__float2bfloat16_rn); bf16 to f32 widens exactly.
static int write_values(tg_decoder *d, uint64_t off, const void *src, uint64_t count, tg_dtype src_dtype, bool as_f32) {
    const bool dst_bf16 = !as_f32 && d->dtype == TG_BF16;
    const uint64_t dst_bytes = count * (dst_bf16 ? 2 : 4);
    if (off + dst_bytes > tg_mem_size(d->weights.m)) return fail(TG_ESHAPE, "a weight past its arena");
    if (src_dtype == TG_BF16 && dst_bf16) return tg_mem_write(d->weights.m, off, src, dst_bytes);
    std::vector<float> f32;
    const float *vals = static_cast<const float *>(src);
    if (src_dtype == TG_BF16) {
        f32.resize(count);
        const uint16_t *b = static_cast<const uint16_t *>(src);
        for (uint64_t i = 0; i < count; i++) {
            const uint32_t bits = (uint32_t)b[i] << 16;
            memcpy(&f32[i], &bits, 4);
        }
        vals = f32.data();
    }
    if (!dst_bf16) return tg_mem_write(d->weights.m, off, vals, dst_bytes);
    Owned tmp;
    TG_TRY(tmp.alloc(d->ctx, count * 4));
    TG_TRY(tg_mem_write(tmp.m, 0, vals, count * 4));
    to_bf16_kernel<<<d->ctx->sm_count * 4, 256, 0, d->ctx->stream>>>(
        reinterpret_cast<const float *>(tmp.ptr()), reinterpret_cast<bf16 *>(d->w(off)), count);
    TG_CUDA(cudaGetLastError());
    return tg_ctx_synchronize(d->ctx, 0);
}

extern "C" int tg_decoder_load(tg_decoder *d, const char *name, const void *src, uint64_t count, tg_dtype src_dtype) {
    if (!d || !name || !src) return fail(TG_EINVAL, "tg_decoder_load: null argument");
    if (src_dtype != TG_F32 && src_dtype != TG_BF16) return fail(TG_EINVAL, "source dtype %d", (int)src_dtype);
    TG_CUDA(cudaSetDevice(d->ctx->device));
    const tg_shape &s = d->shape;
    const uint64_t H = s.hidden, I = s.inner, hd = s.head_dim, T = d->esize;
    auto want = [&](uint64_t n) -> int {
        if (count != n) return fail(TG_ESHAPE, "%s: %llu values, not %llu", name, (unsigned long long)count, (unsigned long long)n);
        return TG_OK;
    };
    if (!strcmp(name, "norm.weight")) {
        TG_TRY(want(H));
        return write_values(d, d->final_norm, src, count, src_dtype, true);
    }
    unsigned l = 0;
    char rest[128] = {0};
    if (sscanf(name, "layers.%u.%127s", &l, rest) != 2 || l >= s.layers)
        return fail(TG_EINVAL, "no weight %s in a stack of %u layers", name, s.layers);
    const LayerOffsets &o = d->layer[l];
    const std::string r = rest;
    // load_stack's joins: qkv = rows[q; k; v], gate_up = rows[gate; up] (decode.rs:764-775).
    if (r == "self_attn.q_proj.weight") {
        TG_TRY(want(s.heads * hd * H));
        return write_values(d, o.qkv, src, count, src_dtype, false);
    }
    if (r == "self_attn.k_proj.weight") {
        TG_TRY(want(s.kv_heads * hd * H));
        return write_values(d, o.qkv + s.heads * hd * H * T, src, count, src_dtype, false);
    }
    if (r == "self_attn.v_proj.weight") {
        TG_TRY(want(s.kv_heads * hd * H));
        return write_values(d, o.qkv + (s.heads + s.kv_heads) * hd * H * T, src, count, src_dtype, false);
    }
    if (r == "self_attn.o_proj.weight") {
        TG_TRY(want(H * s.heads * hd));
        return write_values(d, o.o, src, count, src_dtype, false);
    }
    if (r == "mlp.gate_proj.weight" || r == "mlp.up_proj.weight") {
        TG_TRY(want(I * H));
        // Interleaved in blocks of GU_BLOCK rows (gate_up_row).
        const uint32_t up = r == "mlp.up_proj.weight" ? 1 : 0;
        const uint64_t src_es = src_dtype == TG_BF16 ? 2 : 4;
        for (uint32_t i = 0; i < I; i += GU_BLOCK) {
            const uint64_t rows = std::min<uint64_t>(GU_BLOCK, I - i);
            TG_TRY(write_values(d, o.gate_up + (uint64_t)gate_up_row(i, up) * H * T,
                                static_cast<const char *>(src) + (uint64_t)i * H * src_es, rows * H, src_dtype, false));
        }
        return TG_OK;
    }
    if (r == "mlp.down_proj.weight") {
        TG_TRY(want(H * I));
        return write_values(d, o.down, src, count, src_dtype, false);
    }
    if (r == "input_layernorm.weight") {
        TG_TRY(want(H));
        return write_values(d, o.in_norm, src, count, src_dtype, true);
    }
    if (r == "post_attention_layernorm.weight") {
        TG_TRY(want(H));
        return write_values(d, o.post_norm, src, count, src_dtype, true);
    }
    return fail(TG_EINVAL, "no weight %s", name);
}

extern "C" int tg_decoder_set_rows_n(tg_decoder *d, uint32_t n, const tg_row *rows, const float *x) {
    if (!d || !rows || !x) return fail(TG_EINVAL, "tg_decoder_set_rows: null argument");
    if (n == 0 || n > d->rows) return fail(TG_ESHAPE, "%u rows in a decoder of %u", n, d->rows);
    TG_CUDA(cudaSetDevice(d->ctx->device));
    TG_TRY(d->wait_pending());
    const uint64_t bytes = (uint64_t)n * d->shape.hidden * 4;
    memcpy(d->stage_x.host(), x, bytes);
    TG_TRY(decoder_place(*d, bucket_for(*d, n), n, rows));
    TG_CUDA(cudaMemcpyAsync(d->x_in.ptr(), d->stage_x.ptr(), bytes, cudaMemcpyDefault, d->ctx->stream));
    return TG_OK;
}

extern "C" int tg_decoder_set_rows(tg_decoder *d, const tg_row *rows, const float *x) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    return tg_decoder_set_rows_n(d, d->rows, rows, x);
}

extern "C" int tg_decoder_start(tg_decoder *d) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    TG_CUDA(cudaSetDevice(d->ctx->device));
    std::lock_guard<std::mutex> lock(d->ctx->mu);
    return program_start(d->prog());
}

extern "C" int tg_decoder_wait(tg_decoder *d, uint64_t timeout_ns) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    return program_wait(d->prog(), timeout_ns);
}

extern "C" int tg_decoder_output(tg_decoder *d, float *out) {
    if (!d || !out) return fail(TG_EINVAL, "tg_decoder_output: null argument");
    TG_CUDA(cudaSetDevice(d->ctx->device));
    TG_TRY(d->wait_pending());
    const uint64_t bytes = (uint64_t)(d->n_active ? d->n_active : d->rows) * d->shape.hidden * 4;
    TG_CUDA(cudaMemcpyAsync(d->stage_out.ptr(), d->out.ptr(), bytes, cudaMemcpyDefault, d->ctx->stream));
    TG_CUDA(cudaStreamSynchronize(d->ctx->stream));
    memcpy(out, d->stage_out.host(), bytes);
    return TG_OK;
}

extern "C" int tg_decoder_step_rows_n(tg_decoder *d, uint32_t n, const tg_row *rows, const float *x, float *out) {
    if (!out) return fail(TG_EINVAL, "tg_decoder_step_rows: null output");
    TG_TRY(tg_decoder_set_rows_n(d, n, rows, x));
    TG_TRY(tg_decoder_start(d));
    // The output's copy goes behind the step on the stream, so that one wait covers both.
    const uint64_t bytes = (uint64_t)n * d->shape.hidden * 4;
    TG_CUDA(cudaMemcpyAsync(d->stage_out.ptr(), d->out.ptr(), bytes, cudaMemcpyDefault, d->ctx->stream));
    TG_CUDA(cudaEventRecord(d->out_done, d->ctx->stream));
    TG_TRY(wait_event(d->out_done, 60ull * 1000000000ull));
    TG_TRY(tg_decoder_wait(d, 0));  // done by now: clears the pending run and reads the error word
    memcpy(out, d->stage_out.host(), bytes);
    return TG_OK;
}

extern "C" int tg_decoder_step_rows(tg_decoder *d, const tg_row *rows, const float *x, float *out) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    return tg_decoder_step_rows_n(d, d->rows, rows, x, out);
}

extern "C" int tg_decoder_step_device(tg_decoder *d, const uint32_t *words, const float *x_dev, float *out_dev) {
    if (!d || !words || !x_dev || !out_dev) return fail(TG_EINVAL, "tg_decoder_step_device: null argument");
    TG_CUDA(cudaSetDevice(d->ctx->device));
    const uint32_t nw = d->slots > 1 ? 2 * d->rows : d->rows;
    const uint64_t bytes = (uint64_t)d->rows * d->shape.hidden * 4;
    std::lock_guard<std::mutex> lock(d->ctx->mu);
    // Queued behind the step before without waiting for it: the placement goes through the word
    // ring, x and out are stream-ordered device copies.
    size_t i = 0;
    TG_TRY(d->word_ring.acquire(i));
    memcpy(d->word_ring.host(i), words, (uint64_t)nw * 4);
    d->active = d->buckets.size() - 1;
    d->n_active = d->rows;
    TG_TRY(d->word_ring.upload(i, d->words.ptr(), (uint64_t)nw * 4, d->ctx->stream));
    TG_CUDA(cudaMemcpyAsync(d->x_in.ptr(), x_dev, bytes, cudaMemcpyDeviceToDevice, d->ctx->stream));
    TG_TRY(program_launch(d->prog()));
    TG_CUDA(cudaMemcpyAsync(out_dev, d->out.ptr(), bytes, cudaMemcpyDeviceToDevice, d->ctx->stream));
    return TG_OK;
}

extern "C" int tg_decoder_elapsed_ns(tg_decoder *d, double *ns) {
    if (!d || !ns) return fail(TG_EINVAL, "null argument");
    TG_TRY(d->wait_pending());
    *ns = program_elapsed_ns(d->prog());
    return TG_OK;
}

extern "C" int tg_decoder_timings(tg_decoder *d, double *ns, size_t n, size_t *n_dispatches) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    if (n_dispatches) *n_dispatches = d->cur().launches.size();
    if (!ns) return TG_OK;
    TG_TRY(d->wait_pending());
    return program_timings(d->prog(), ns, n);
}

extern "C" int tg_decoder_dispatch_label(tg_decoder *d, size_t i, char *label, size_t label_bytes) {
    if (!d || !label) return fail(TG_EINVAL, "null argument");
    const std::vector<Launch> &l = d->cur().launches;
    if (i >= l.size()) return fail(TG_EINVAL, "dispatch %zu of %zu", i, l.size());
    snprintf(label, label_bytes, "%s", l[i].label.c_str());
    return TG_OK;
}

extern "C" int tg_decoder_read_cache(tg_decoder *d, uint32_t layer, uint32_t slot, uint32_t kind, uint32_t first,
                                     uint32_t count, float *out) {
    if (!d || !out) return fail(TG_EINVAL, "null argument");
    const tg_shape &s = d->shape;
    if (layer >= s.layers || slot >= d->slots || kind > 1 || first > s.capacity || count > s.capacity - first)
        return fail(TG_ESHAPE, "cache layer %u slot %u kind %u positions %u+%u", layer, slot, kind, first, count);
    TG_CUDA(cudaSetDevice(d->ctx->device));
    TG_TRY(d->wait_pending());
    const uint64_t hd = s.head_dim, T = d->esize;
    std::vector<uint8_t> raw((uint64_t)count * hd * T);
    tg_mem *m = kind == 0 ? d->kcache.m : d->vcache.m;
    for (uint32_t kv = 0; kv < s.kv_heads; kv++) {
        const uint64_t off = layer * d->cache_layer + ((((uint64_t)slot * s.kv_heads + kv) * s.capacity + first) * hd) * T;
        TG_TRY(tg_mem_read(m, off, raw.data(), raw.size()));
        float *o = out + (uint64_t)kv * count * hd;
        for (uint64_t i = 0; i < (uint64_t)count * hd; i++) {
            if (T == 4) {
                memcpy(&o[i], &raw[i * 4], 4);
            } else {
                uint16_t b;
                memcpy(&b, &raw[i * 2], 2);
                const uint32_t bits = (uint32_t)b << 16;
                memcpy(&o[i], &bits, 4);
            }
        }
    }
    return TG_OK;
}

extern "C" int tg_decoder_copy_slot(tg_decoder *d, uint32_t from, uint32_t to, uint32_t count) {
    if (!d) return fail(TG_EINVAL, "null decoder");
    const tg_shape &s = d->shape;
    if (from >= d->slots || to >= d->slots || count > s.capacity)
        return fail(TG_ESHAPE, "copy of %u positions from slot %u to %u of %u", count, from, to, d->slots);
    if (from == to || count == 0) return TG_OK;
    TG_CUDA(cudaSetDevice(d->ctx->device));
    TG_TRY(d->wait_pending());
    const uint64_t hd = s.head_dim, T = d->esize;
    std::vector<tg_region> regions;
    for (uint32_t l = 0; l < s.layers; l++)
        for (uint32_t kv = 0; kv < s.kv_heads; kv++) {
            const uint64_t a = l * d->cache_layer + (((uint64_t)from * s.kv_heads + kv) * s.capacity) * hd * T;
            const uint64_t b = l * d->cache_layer + (((uint64_t)to * s.kv_heads + kv) * s.capacity) * hd * T;
            regions.push_back({a, b, (uint64_t)count * hd * T});
        }
    TG_TRY(tg_copy_regions(d->ctx, d->kcache.m, d->kcache.m, regions.data(), regions.size()));
    return tg_copy_regions(d->ctx, d->vcache.m, d->vcache.m, regions.data(), regions.size());
}

extern "C" uint64_t tg_decoder_prefix_bytes(const tg_decoder *d, uint32_t count) {
    if (!d) return 0;
    return (uint64_t)d->shape.layers * 2 * d->shape.kv_heads * count * d->shape.head_dim * d->esize;
}

// Positions [0, count) of `slot`, every layer and KV head, to (out) or from (in) `m` at `offset`.
static int copy_prefix(tg_decoder *d, uint32_t slot, uint32_t count, tg_mem *m, uint64_t offset, bool out) {
    if (!d || !m) return fail(TG_EINVAL, "null argument");
    const tg_shape &s = d->shape;
    if (slot >= d->slots || count > s.capacity)
        return fail(TG_ESHAPE, "%u positions of slot %u of %u", count, slot, d->slots);
    const uint64_t bytes = tg_decoder_prefix_bytes(d, count);
    if (offset + bytes > tg_mem_size(m)) return fail(TG_ESHAPE, "a prefix of %llu bytes past its buffer", (unsigned long long)bytes);
    if (count == 0) return TG_OK;
    TG_CUDA(cudaSetDevice(d->ctx->device));
    const uint64_t hd = s.head_dim, T = d->esize, run = (uint64_t)count * hd * T;
    uint64_t at = offset;
    for (uint32_t l = 0; l < s.layers; l++)
        for (int kind = 0; kind < 2; kind++)
            for (uint32_t kv = 0; kv < s.kv_heads; kv++) {
                char *cache = (kind == 0 ? d->kcache.ptr() : d->vcache.ptr()) + l * d->cache_layer +
                              (((uint64_t)slot * s.kv_heads + kv) * s.capacity) * hd * T;
                char *buf = static_cast<char *>(m->ptr) + at;
                TG_CUDA(cudaMemcpyAsync(out ? buf : cache, out ? cache : buf, run, cudaMemcpyDeviceToDevice,
                                        d->ctx->stream));
                at += run;
            }
    return TG_OK;
}

extern "C" int tg_decoder_copy_out(tg_decoder *d, uint32_t slot, uint32_t count, tg_mem *m, uint64_t offset) {
    return copy_prefix(d, slot, count, m, offset, true);
}

extern "C" int tg_decoder_copy_in(tg_decoder *d, uint32_t slot, uint32_t count, tg_mem *m, uint64_t offset) {
    return copy_prefix(d, slot, count, m, offset, false);
}

extern "C" uint64_t tg_decoder_weight_bytes(const tg_decoder *d) {
    return d ? tg_shape_weight_bytes(&d->shape, (uint32_t)d->esize) : 0;
}

extern "C" void *tg_ctx_stream(tg_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

// ---- prefill ----------------------------------------------------------------------------------------

// prefill_graph / append_prefill (prefill.rs:181-413): the first input norm, then per layer the
// q/k/v GEMM, rope_rows, attention_rows, the o GEMM, add_norm_rows, the gate/up GEMM,
// silu_mul_rows, the down GEMM and add_norm_rows with the next gain (the final norm's after the
// last layer).
static std::vector<Launch> prefill_launches(tg_prefill &p, uint32_t rows) {
    tg_decoder &d = *p.d;
    const tg_shape &s = d.shape;
    tg_params base = d.params();
    base.rows = rows;
    const uint64_t T = d.esize, F = 4, R = rows, H = s.hidden, I = s.inner, hd = s.head_dim;
    const uint64_t W = d.width(), A = d.attn();
    const uint64_t words = (d.slots > 1 ? 2 : 1) * R * 4;
    const uint64_t table = (uint64_t)s.capacity * (hd / 2) * F;
    std::vector<Launch> v;
    push(v, TG_KERNEL_NORM_ROWS, base, "input_norm",
         {{p.words.ptr(), words}, {p.x_in.ptr(), R * H * F}, {d.w(d.layer[0].in_norm), H * F}, {p.normed.ptr(), R * H * T}});
    auto gemm = [&](const char *label, void *a, void *b, void *c, uint64_t n, uint64_t k) {
        tg_params g = base;
        g.m = rows;
        g.n = (uint32_t)n;
        g.k = (uint32_t)k;
        g.flags = 1;  // b is a weight: its first tiles stream while the kernel before finishes
        push(v, TG_KERNEL_GEMM, g, label, {{a, R * k * T}, {b, n * k * T}, {c, R * n * F}});
    };
    // bf16: the residual added in the GEMM's epilogue (sum = residual + s a b^T), then norm_rows
    // over the sum - add_norm_rows' sums and norm, without the GEMM's f32 rows going through memory.
    const bool fused_res = d.dtype == TG_BF16;
    auto gemm_res = [&](const char *label, void *a, void *b, void *sum, void *res, uint64_t n, uint64_t k) {
        tg_params g = base;
        g.m = rows;
        g.n = (uint32_t)n;
        g.k = (uint32_t)k;
        g.flags = 1;
        push(v, KERNEL_GEMM_RESIDUAL, g, label, {{a, R * k * T}, {b, n * k * T}, {sum, R * n * F}, {res, R * n * F}});
    };
    auto norm = [&](const char *label, void *x, uint64_t gain, void *out, bool f32_out) {
        tg_params nr = base;
        nr.normed_f32 = f32_out ? 1 : 0;
        push(v, TG_KERNEL_NORM_ROWS, nr, label,
             {{p.words.ptr(), words}, {x, R * H * F}, {d.w(gain), H * F}, {out, R * H * (f32_out ? F : T)}});
    };
    for (uint32_t l = 0; l < s.layers; l++) {
        const LayerOffsets &o = d.layer[l];
        char *in = l == 0 ? p.x_in.ptr() : p.h.ptr();
        if (d.dtype == TG_BF16 && W % 256 == 0) {
            // RoPE and the cache append in the GEMM's epilogue: the f32 q/k/v rows never reach memory.
            tg_params g = base;
            g.m = rows;
            g.n = (uint32_t)W;
            g.k = (uint32_t)H;
            push(v, TG_KERNEL_GEMM_QKV_ROPE, g, "qkv_proj",
                 {{p.normed.ptr(), R * H * T}, {d.w(o.qkv), W * H * T}, {p.words.ptr(), words}, {d.cos.ptr(), table},
                  {d.sin.ptr(), table}, {p.q.ptr(), R * A * T}, {d.kc(l), d.cache_layer}, {d.vc(l), d.cache_layer}});
        } else {
            gemm("qkv_proj", p.normed.ptr(), d.w(o.qkv), p.qkv.ptr(), W, H);
            push(v, TG_KERNEL_ROPE_ROWS, base, "rope_rows",
                 {{p.words.ptr(), words}, {p.qkv.ptr(), R * W * F}, {d.cos.ptr(), table}, {d.sin.ptr(), table},
                  {p.q.ptr(), R * A * T}, {d.kc(l), d.cache_layer}, {d.vc(l), d.cache_layer}});
        }
        push(v, attention_tc_supported(base) ? TG_KERNEL_ATTENTION_ROWS_TC : TG_KERNEL_ATTENTION_ROWS, base, "attention_rows",
             {{p.words.ptr(), words}, {p.q.ptr(), R * A * T}, {d.kc(l), d.cache_layer}, {d.vc(l), d.cache_layer},
              {p.att.ptr(), R * A * T}});
        if (fused_res) {
            gemm_res("o_proj", p.att.ptr(), d.w(o.o), p.mid.ptr(), in, H, A);
            norm("norm_rows", p.mid.ptr(), o.post_norm, p.normed.ptr(), false);
        } else {
            gemm("o_proj", p.att.ptr(), d.w(o.o), p.proj.ptr(), H, A);
            push(v, TG_KERNEL_ADD_NORM_ROWS, base, "add_norm_rows",
                 {{p.words.ptr(), words}, {p.proj.ptr(), R * H * F}, {in, R * H * F}, {d.w(o.post_norm), H * F},
                  {p.mid.ptr(), R * H * F}, {p.normed.ptr(), R * H * T}});
        }
        if (d.dtype == TG_BF16) {
            // SiLU-mul in the GEMM's epilogue: the f32 gate/up rows never reach memory.
            tg_params g = base;
            g.m = rows;
            g.n = (uint32_t)(2 * I);
            g.k = (uint32_t)H;
            push(v, TG_KERNEL_GEMM_SILU, g, "gate_up_proj",
                 {{p.normed.ptr(), R * H * T}, {d.w(o.gate_up), 2 * I * H * T}, {p.mlp.ptr(), R * I * T}});
        } else {
            gemm("gate_up_proj", p.normed.ptr(), d.w(o.gate_up), p.gu.ptr(), 2 * I, H);
            push(v, TG_KERNEL_SILU_MUL_ROWS, base, "silu_mul_rows",
                 {{p.words.ptr(), words}, {p.gu.ptr(), R * 2 * I * F}, {p.mlp.ptr(), R * I * T}});
        }
        const bool last = l + 1 == s.layers;
        if (fused_res) {
            gemm_res("down_proj", p.mlp.ptr(), d.w(o.down), p.h.ptr(), p.mid.ptr(), H, I);
            norm("norm_rows", p.h.ptr(), last ? d.final_norm : d.layer[l + 1].in_norm, last ? p.out.ptr() : p.normed.ptr(),
                 last);
            continue;
        }
        gemm("down_proj", p.mlp.ptr(), d.w(o.down), p.proj.ptr(), H, I);
        tg_params an = base;
        an.normed_f32 = last ? 1 : 0;
        push(v, TG_KERNEL_ADD_NORM_ROWS, an, "add_norm_rows",
             {{p.words.ptr(), words}, {p.proj.ptr(), R * H * F}, {p.mid.ptr(), R * H * F},
              {d.w(last ? d.final_norm : d.layer[l + 1].in_norm), H * F}, {p.h.ptr(), R * H * F},
              {last ? p.out.ptr() : p.normed.ptr(), R * H * (last ? F : T)}});
    }
    return v;
}

extern "C" int tg_prefill_create(tg_decoder *d, uint32_t max_rows, int timed, tg_prefill **out) {
    if (!d || !out) return fail(TG_EINVAL, "tg_prefill_create: null argument");
    *out = nullptr;
    if (max_rows == 0 || max_rows > (1u << 20)) return fail(TG_ESHAPE, "programs of up to %u rows", max_rows);
    TG_CUDA(cudaSetDevice(d->ctx->device));
    std::unique_ptr<tg_prefill> p(new tg_prefill());
    p->d = d;
    p->timed = timed != 0;
    p->max_rows = (max_rows + 127) / 128 * 128;
    const tg_shape &s = d->shape;
    const uint64_t R = p->max_rows, T = d->esize, F = 4, H = s.hidden, I = s.inner;
    tg_ctx *ctx = d->ctx;
    TG_TRY(p->words.alloc(ctx, 2 * R * 4));
    TG_TRY(p->x_in.alloc(ctx, R * H * F));
    TG_TRY(p->h.alloc(ctx, R * H * F));
    TG_TRY(p->mid.alloc(ctx, R * H * F));
    TG_TRY(p->normed.alloc(ctx, R * H * T));
    if (d->dtype != TG_BF16 || d->width() % 256)  // else RoPE runs in the q/k/v GEMM's epilogue
        TG_TRY(p->qkv.alloc(ctx, R * d->width() * F));
    TG_TRY(p->q.alloc(ctx, R * d->attn() * T));
    TG_TRY(p->att.alloc(ctx, R * d->attn() * T));
    TG_TRY(p->proj.alloc(ctx, R * H * F));
    if (d->dtype != TG_BF16) TG_TRY(p->gu.alloc(ctx, R * 2 * I * F));  // bf16 fuses SiLU into the GEMM
    TG_TRY(p->mlp.alloc(ctx, R * I * T));
    TG_TRY(p->out.alloc(ctx, R * H * F));
    TG_TRY(p->stage_x.alloc(ctx, R * H * F, TG_RES_UPLOAD));
    TG_TRY(p->stage_words.alloc(ctx, 2 * R * 4, TG_RES_UPLOAD));
    TG_TRY(p->stage_out.alloc(ctx, R * H * F, TG_RES_READBACK));
    *out = p.release();
    return TG_OK;
}

extern "C" int tg_prefill_destroy(tg_prefill *p) {
    if (!p) return TG_OK;
    cudaSetDevice(p->d->ctx->device);
    for (auto &kv : p->programs)
        if (kv.second.pending) program_wait(kv.second, 0);
    delete p;
    return TG_OK;
}

static int program_for(tg_prefill *p, uint32_t rows, Program **out) {
    auto it = p->programs.find(rows);
    if (it == p->programs.end()) {
        Program prog;
        const int st = program_build(p->d->ctx, prefill_launches(*p, rows), p->timed, prog);
        if (st) {
            program_release(prog);
            return st;
        }
        it = p->programs.emplace(rows, prog).first;
    }
    *out = &it->second;
    return TG_OK;
}

// Lays `runs` out as rows of one launch: each run's rows start on a multiple of RUN_ALIGN
// (padding rows between are spare). Fills the words (positions, then slots, at the bucket's
// stride) and returns the rows used and each run's first row.
static int layout_runs(tg_prefill *p, const tg_run *runs, uint32_t n_runs, uint32_t &used,
                       std::vector<uint32_t> &first) {
    const tg_shape &s = p->d->shape;
    std::vector<bool> slot_taken(p->d->slots, false);
    uint32_t row = 0;
    first.clear();
    for (uint32_t i = 0; i < n_runs; i++) {
        const tg_run &r = runs[i];
        if (r.len == 0 || (uint64_t)r.start + r.len > s.capacity || r.slot >= p->d->slots || slot_taken[r.slot])
            return fail(TG_ESHAPE, "run %u: %u positions from %u in slot %u of %u in a cache of %u", i, r.len, r.start,
                        r.slot, p->d->slots, s.capacity);
        slot_taken[r.slot] = true;
        row = (row + RUN_ALIGN - 1) / RUN_ALIGN * RUN_ALIGN;
        first.push_back(row);
        row += r.len;
        if (row > p->max_rows) return fail(TG_ESHAPE, "runs of %u rows in a prefill of at most %u", row, p->max_rows);
    }
    used = row;
    return TG_OK;
}

int tg::prefill_rows(tg_prefill *p, const tg_run *runs, uint32_t n_runs, const float *x, bool x_on_device,
                     float *out, bool out_on_device) {
    tg_decoder *d = p->d;
    tg_ctx *ctx = d->ctx;
    const uint64_t H = d->shape.hidden, F = 4;
    uint32_t used = 0;
    std::vector<uint32_t> first;
    TG_TRY(layout_runs(p, runs, n_runs, used, first));
    const uint32_t rows = (used + 127) / 128 * 128;
    Program *prog = nullptr;
    TG_TRY(program_for(p, rows, &prog));
    // The staging buffers are free once this prefill's last launch has run; the decoder's steps
    // need no wait (the stream orders them with this launch).
    for (auto &kv : p->programs)
        if (kv.second.pending) TG_TRY(program_wait(kv.second, 0));
    uint32_t *w = reinterpret_cast<uint32_t *>(p->stage_words.host());
    for (uint32_t i = 0; i < 2 * rows; i++) w[i] = TG_SPARE;
    for (uint32_t i = 0; i < n_runs; i++)
        for (uint32_t j = 0; j < runs[i].len; j++) {
            w[first[i] + j] = runs[i].start + j;
            w[rows + first[i] + j] = runs[i].slot;
        }
    std::lock_guard<std::mutex> lock(ctx->mu);
    TG_CUDA(cudaMemcpyAsync(p->words.ptr(), p->stage_words.ptr(), (uint64_t)2 * rows * 4, cudaMemcpyDefault, ctx->stream));
    uint64_t src_row = 0;
    for (uint32_t i = 0; i < n_runs; i++) {
        const uint64_t bytes = (uint64_t)runs[i].len * H * F;
        char *dst = p->x_in.ptr() + (uint64_t)first[i] * H * F;
        if (x_on_device) {
            TG_CUDA(cudaMemcpyAsync(dst, x + src_row * H, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
        } else {
            memcpy(p->stage_x.host() + (uint64_t)first[i] * H * F, x + src_row * H, bytes);
            TG_CUDA(cudaMemcpyAsync(dst, p->stage_x.ptr() + (uint64_t)first[i] * H * F, bytes, cudaMemcpyDefault, ctx->stream));
        }
        src_row += runs[i].len;
    }
    TG_TRY(program_start(*prog));
    p->last = prog;
    src_row = 0;
    for (uint32_t i = 0; i < n_runs; i++) {
        const uint64_t bytes = (uint64_t)runs[i].len * H * F;
        const char *src = p->out.ptr() + (uint64_t)first[i] * H * F;
        if (out_on_device) {
            TG_CUDA(cudaMemcpyAsync(out + src_row * H, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
        } else {
            TG_CUDA(cudaMemcpyAsync(p->stage_out.ptr() + (uint64_t)first[i] * H * F, src, bytes, cudaMemcpyDefault, ctx->stream));
        }
        src_row += runs[i].len;
    }
    if (out_on_device) return TG_OK;
    TG_TRY(program_wait(*prog, 600ull * 1000000000ull));
    TG_CUDA(cudaStreamSynchronize(ctx->stream));
    src_row = 0;
    for (uint32_t i = 0; i < n_runs; i++) {
        memcpy(out + src_row * H, p->stage_out.host() + (uint64_t)first[i] * H * F, (uint64_t)runs[i].len * H * F);
        src_row += runs[i].len;
    }
    return TG_OK;
}

extern "C" int tg_prefill_run(tg_prefill *p, uint32_t start, uint32_t slot, const float *x, uint32_t len, float *out) {
    if (!p || !x || !out) return fail(TG_EINVAL, "tg_prefill_run: null argument");
    const tg_shape &s = p->d->shape;
    if (len == 0 || (uint64_t)start + len > s.capacity || slot >= p->d->slots)
        return fail(TG_ESHAPE, "%u positions from %u in slot %u of a cache of %u", len, start, slot, s.capacity);
    TG_CUDA(cudaSetDevice(p->d->ctx->device));
    // A run of more than max_rows positions runs in pieces (prefill.rs:487-502).
    for (uint32_t done = 0; done < len;) {
        const uint32_t n = std::min(len - done, p->max_rows);
        const tg_run r = {start + done, n, slot};
        TG_TRY(prefill_rows(p, &r, 1, x + (uint64_t)done * s.hidden, false, out + (uint64_t)done * s.hidden, false));
        done += n;
    }
    return TG_OK;
}

extern "C" int tg_prefill_run_batch(tg_prefill *p, const tg_run *runs, uint32_t n_runs, const float *x, float *out) {
    if (!p || !runs || !n_runs || !x || !out) return fail(TG_EINVAL, "tg_prefill_run_batch: null argument");
    TG_CUDA(cudaSetDevice(p->d->ctx->device));
    return prefill_rows(p, runs, n_runs, x, false, out, false);
}

extern "C" int tg_prefill_run_batch_device(tg_prefill *p, const tg_run *runs, uint32_t n_runs, const float *x_dev,
                                           float *out_dev) {
    if (!p || !runs || !n_runs || !x_dev || !out_dev) return fail(TG_EINVAL, "tg_prefill_run_batch_device: null argument");
    TG_CUDA(cudaSetDevice(p->d->ctx->device));
    return prefill_rows(p, runs, n_runs, x_dev, true, out_dev, true);
}

extern "C" int tg_prefill_elapsed_ns(tg_prefill *p, double *ns) {
    if (!p || !ns || !p->last) return fail(TG_EINVAL, "no prefill has run");
    if (p->last->pending) TG_TRY(program_wait(*p->last, 0));
    *ns = program_elapsed_ns(*p->last);
    return TG_OK;
}

extern "C" int tg_prefill_timings(tg_prefill *p, double *ns, size_t n, size_t *n_dispatches) {
    if (!p || !p->last) return fail(TG_EINVAL, "no prefill has run");
    if (n_dispatches) *n_dispatches = p->last->labels.size();
    if (!ns) return TG_OK;
    if (p->last->pending) TG_TRY(program_wait(*p->last, 0));
    return program_timings(*p->last, ns, n);
}

extern "C" int tg_prefill_dispatch_label(tg_prefill *p, size_t i, char *label, size_t label_bytes) {
    if (!p || !label || !p->last) return fail(TG_EINVAL, "no prefill has run");
    if (i >= p->last->labels.size()) return fail(TG_EINVAL, "dispatch %zu of %zu", i, p->last->labels.size());
    snprintf(label, label_bytes, "%s", p->last->labels[i].c_str());
    return TG_OK;
}

extern "C" uint32_t tg_prefill_max_rows(const tg_prefill *p) { return p ? p->max_rows : 0; }
