// VoxCPM2's local stacks over the runtime (crates/graph/src/local): a stack's weights, tables and
// activations (Stack, local/mod.rs:315-570), the patch sampler (dit.rs) and the local encoder
// (encoder.rs), each recorded once as one program of the local kernels (local.cu).
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "model.h"
#include "tg_common.cuh"

using namespace tg;

namespace tg {

// A stack's f16 weights, one allocation: per layer q/k/v [(heads + 2 kv) hd][hidden], o [hidden]
// [heads hd], gate/up [2 inner][hidden] (gate row i at 2i, up row i at 2i + 1), down [hidden]
// [inner], the two gains; then the final gain.
struct LocalLayer {
    uint64_t qkv, o, gate_up, down, in_norm, post_norm;
};

struct LocalStack {
    tg_ctx *ctx = nullptr;
    tg_shape shape{};  // capacity: a sequence's tokens
    std::vector<double> factors;
    uint32_t seqs = 0, M = 0;
    tg_local_tuning tuning{};
    Owned weights, cos, sin;
    std::vector<LocalLayer> layer;
    uint64_t final_norm = 0, weight_bytes = 0;
    // Activations: the stack's input x (written by the embedding), the residual stream, the
    // post-attention sum, the normed tokens, the attention's output, the SiLU output, and the
    // projections' partial sums.
    Owned x, cur, mid, normed, att, mlp, part;
    uint64_t part_bytes = 0;

    uint32_t width() const { return (shape.heads + 2 * shape.kv_heads) * shape.head_dim; }
    uint32_t attn() const { return shape.heads * shape.head_dim; }
    char *w(uint64_t off) const { return weights.ptr() + off; }
    uint64_t tokens_bytes(uint32_t n) const { return (uint64_t)M * n * 2; }

    tg_params params() const {
        tg_params p{};
        p.dtype = TG_F16;
        p.hidden = shape.hidden;
        p.inner = shape.inner;
        p.heads = shape.heads;
        p.kv_heads = shape.kv_heads;
        p.head_dim = shape.head_dim;
        p.capacity = shape.capacity;
        p.rows = seqs;
        p.slots = 1;
        p.eps = shape.eps;
        p.residual_scale = 1.0f;
        p.rope = shape.rope;
        p.m = M;
        return p;
    }
};

// The largest part count at most `want` (at least 1) that cuts k into multiples of 64 columns.
static uint32_t fit_parts(uint32_t k, uint32_t want) {
    for (uint32_t p = std::max(1u, want); p > 1; p--)
        if (k % (64 * p) == 0) return p;
    return 1;
}

static int local_init(LocalStack &st, tg_ctx *ctx, const tg_shape &s, uint32_t seqs, const tg_local_tuning *tuning) {
    const uint32_t H = s.hidden, I = s.inner, hd = s.head_dim;
    // local/mod.rs:366-385 (hidden a multiple of 256, head_dim of 32, heads of kv_heads), and
    // what the tcgen05 projections tile (outputs in 128s, columns in 64s).
    if (!ctx) return fail(TG_EINVAL, "null context");
    if (s.layers == 0 || s.kv_heads == 0 || s.heads % s.kv_heads || hd % 32 || hd > 256 || H % 256 || H > 2048 ||
        I == 0 || I % 64 || (s.heads * hd) % 64 || ((s.heads + 2 * s.kv_heads) * hd) % 128)
        return fail(TG_ESHAPE, "local stack: %u heads over %u of %u, %u wide, %u inner", s.heads, s.kv_heads, hd, H, I);
    if (s.capacity == 0 || s.capacity > 32) return fail(TG_ESHAPE, "local stack: sequences of %u tokens", s.capacity);
    if (!(s.eps >= 0.0f)) return fail(TG_ESHAPE, "eps %g", s.eps);
    st.ctx = ctx;
    st.shape = s;
    if (s.rope_factors) st.factors.assign(s.rope_factors, s.rope_factors + hd / 2);
    st.shape.rope_factors = nullptr;
    st.seqs = seqs;
    st.M = seqs * s.capacity;
    const tg_local_tuning want = tuning ? *tuning : tg_local_tuning{0, 0, 0};
    st.tuning.qkv_parts = fit_parts(H, want.qkv_parts ? want.qkv_parts : 4);
    st.tuning.o_parts = fit_parts(st.attn(), want.o_parts ? want.o_parts : 8);
    st.tuning.down_parts = fit_parts(I, want.down_parts ? want.down_parts : 8);
    for (uint32_t parts : {st.tuning.qkv_parts, st.tuning.o_parts, st.tuning.down_parts})
        if (!local_proj_supported((int)st.M, 128, 64 * (int)parts, (int)parts))
            return fail(TG_ESHAPE, "local stack: %u tokens in one launch", st.M);
    // Weights.
    uint64_t off = 0;
    auto take = [&](uint64_t values) {
        const uint64_t at = off;
        off = align256(off + values * 2);
        return at;
    };
    for (uint32_t l = 0; l < s.layers; l++) {
        LocalLayer L;
        L.qkv = take((uint64_t)st.width() * H);
        L.o = take((uint64_t)H * st.attn());
        L.gate_up = take(2ull * I * H);
        L.down = take((uint64_t)H * I);
        L.in_norm = take(H);
        L.post_norm = take(H);
        st.layer.push_back(L);
    }
    st.final_norm = take(H);
    st.weight_bytes = 2ull * ((uint64_t)s.layers * ((uint64_t)st.width() * H + (uint64_t)H * st.attn() + 3ull * I * H + 2ull * H) + H);
    TG_TRY(st.weights.alloc(ctx, off));
    // Rotation tables over the sequence's places (Shape::rope_tables, decode.rs:143-168).
    const uint64_t table = (uint64_t)s.capacity * (hd / 2);
    std::vector<float> cs(table), sn(table);
    tg_shape ts = st.shape;
    ts.rope_factors = st.factors.empty() ? nullptr : st.factors.data();
    TG_TRY(tg_shape_rope_tables(&ts, cs.data(), sn.data()));
    TG_TRY(st.cos.alloc(ctx, table * 4));
    TG_TRY(st.sin.alloc(ctx, table * 4));
    TG_TRY(tg_mem_write(st.cos.m, 0, cs.data(), table * 4));
    TG_TRY(tg_mem_write(st.sin.m, 0, sn.data(), table * 4));
    // Activations.
    for (Owned *o : {&st.x, &st.cur, &st.mid, &st.normed}) TG_TRY(o->alloc(ctx, st.tokens_bytes(H)));
    TG_TRY(st.att.alloc(ctx, st.tokens_bytes(st.attn())));
    TG_TRY(st.mlp.alloc(ctx, st.tokens_bytes(I)));
    st.part_bytes = 4ull * st.M *
                    std::max({(uint64_t)st.tuning.qkv_parts * st.width(), (uint64_t)st.tuning.o_parts * H,
                              (uint64_t)st.tuning.down_parts * H});
    TG_TRY(st.part.alloc(ctx, st.part_bytes));
    return TG_OK;
}

// Host values of `count` elements of src_dtype as f16 bits (RNE).
static int to_f16(const void *src, uint64_t count, tg_dtype src_dtype, std::vector<uint16_t> &out) {
    out.resize(count);
    if (src_dtype == TG_F16) {
        memcpy(out.data(), src, count * 2);
        return TG_OK;
    }
    for (uint64_t i = 0; i < count; i++) {
        float v;
        if (src_dtype == TG_F32) {
            v = static_cast<const float *>(src)[i];
        } else if (src_dtype == TG_BF16) {
            const uint32_t bits = (uint32_t)static_cast<const uint16_t *>(src)[i] << 16;
            memcpy(&v, &bits, 4);
        } else {
            return fail(TG_EINVAL, "source dtype %d", (int)src_dtype);
        }
        const __half h = __float2half_rn(v);
        memcpy(&out[i], &h, 2);
    }
    return TG_OK;
}

static double f16_value(uint16_t bits) {
    __half_raw raw;
    raw.x = bits;
    return (double)__half2float(__half(raw));
}

static bool parse_layer(const std::string &name, uint32_t &l, std::string &rest) {
    unsigned li = 0;
    int used = 0;
    if (sscanf(name.c_str(), "layers.%u.%n", &li, &used) != 1 || used == 0) return false;
    l = li;
    rest = name.substr((size_t)used);
    return true;
}

// Stack::load (local/mod.rs:486-530): one tensor by its name below the stack's prefix ("layers.{l}
// ..." or "norm.weight"), rounded to f16; the projections tiled (local_tiled_offset), q/k/v joined
// along their rows, gate and up rows alternating.
static int local_load(LocalStack &st, const std::string &name, const void *src, uint64_t count, tg_dtype src_dtype) {
    const tg_shape &s = st.shape;
    const uint64_t H = s.hidden, I = s.inner, hd = s.head_dim;
    std::vector<uint16_t> v;
    auto check_count = [&](uint64_t want) {
        return count == want ? TG_OK
                             : fail(TG_ESHAPE, "%s: %llu values, not %llu", name.c_str(), (unsigned long long)count,
                                    (unsigned long long)want);
    };
    // A gain: as it is.
    auto gain = [&](uint64_t off) -> int {
        TG_TRY(check_count(H));
        TG_TRY(to_f16(src, count, src_dtype, v));
        return tg_mem_write(st.weights.m, off, v.data(), count * 2);
    };
    // `rows` rows of K columns into the tiled weight at `off`, as its rows row0, row0 + step, ...
    auto rows_of = [&](uint64_t off, uint64_t rows, uint64_t K, uint32_t row0, uint32_t step) -> int {
        TG_TRY(check_count(rows * K));
        TG_TRY(to_f16(src, count, src_dtype, v));
        Owned tmp;
        TG_TRY(tmp.alloc(st.ctx, count * 2));
        TG_TRY(tg_mem_write(tmp.m, 0, v.data(), count * 2));
        TG_CUDA(launch_local_tile_rows(tmp.ptr(), (int)rows, (int)K, st.w(off), (int)row0, (int)step, st.ctx->stream));
        return tg_ctx_synchronize(st.ctx, 0);
    };
    if (name == "norm.weight") return gain(st.final_norm);
    uint32_t l;
    std::string rest;
    if (!parse_layer(name, l, rest) || l >= s.layers) return fail(TG_EINVAL, "local stack: no weight %s", name.c_str());
    const LocalLayer &L = st.layer[l];
    const uint32_t q_rows = (uint32_t)(s.heads * hd), kv_rows = (uint32_t)(s.kv_heads * hd);
    if (rest == "self_attn.q_proj.weight") return rows_of(L.qkv, q_rows, H, 0, 1);
    if (rest == "self_attn.k_proj.weight") return rows_of(L.qkv, kv_rows, H, q_rows, 1);
    if (rest == "self_attn.v_proj.weight") return rows_of(L.qkv, kv_rows, H, q_rows + kv_rows, 1);
    if (rest == "self_attn.o_proj.weight") return rows_of(L.o, H, q_rows, 0, 1);
    if (rest == "mlp.gate_proj.weight") return rows_of(L.gate_up, I, H, 0, 2);
    if (rest == "mlp.up_proj.weight") return rows_of(L.gate_up, I, H, 1, 2);
    if (rest == "mlp.down_proj.weight") return rows_of(L.down, H, I, 0, 1);
    if (rest == "input_layernorm.weight") return gain(L.in_norm);
    if (rest == "post_attention_layernorm.weight") return gain(L.post_norm);
    return fail(TG_EINVAL, "local stack: no weight %s", name.c_str());
}

static void push(std::vector<Launch> &v, uint32_t kernel, const tg_params &p, const std::string &label,
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

// Stack::layers (local/mod.rs:573-680) over st.x: the first input norm, then per layer q/k/v,
// attention, the output projection and its residual add with the post-attention norm, gate/up with
// SiLU, the down projection and its residual add with the next layer's input norm (or the final
// norm). The output after the final norm is st.normed.
static void local_layers(LocalStack &st, std::vector<Launch> &v, const std::string &name) {
    const tg_shape &s = st.shape;
    const uint64_t H = s.hidden, I = s.inner;
    const tg_params base = st.params();
    const uint64_t tokH = st.tokens_bytes((uint32_t)H);
    auto label = [&](uint32_t l, const char *what) { return name + ".layers." + std::to_string(l) + "." + what; };
    push(v, TG_KERNEL_LOCAL_NORM, base, label(0, "input_norm"),
         {{st.x.ptr(), tokH}, {st.w(st.layer[0].in_norm), H * 2}, {st.normed.ptr(), tokH}});
    for (uint32_t l = 0; l < s.layers; l++) {
        const LocalLayer &L = st.layer[l];
        char *res = l == 0 ? st.x.ptr() : st.cur.ptr();
        tg_params q = base;
        q.n = st.width();
        q.k = (uint32_t)H;
        q.parts = st.tuning.qkv_parts;
        push(v, TG_KERNEL_LOCAL_PARTIAL, q, label(l, "qkv_rope"),
             {{st.normed.ptr(), tokH}, {st.w(L.qkv), (uint64_t)q.n * H * 2}, {st.part.ptr(), st.part_bytes}});
        const uint64_t table = (uint64_t)s.capacity * (s.head_dim / 2) * 4;
        push(v, TG_KERNEL_LOCAL_ATTENTION, q, label(l, "attention"),
             {{st.part.ptr(), st.part_bytes}, {st.cos.ptr(), table}, {st.sin.ptr(), table},
              {st.att.ptr(), st.tokens_bytes(st.attn())}});
        tg_params o = base;
        o.n = (uint32_t)H;
        o.k = st.attn();
        o.parts = st.tuning.o_parts;
        push(v, TG_KERNEL_LOCAL_PARTIAL, o, label(l, "o_proj"),
             {{st.att.ptr(), st.tokens_bytes(st.attn())}, {st.w(L.o), H * o.k * 2}, {st.part.ptr(), st.part_bytes}});
        push(v, TG_KERNEL_LOCAL_ADD_NORM, o, label(l, "o_proj_add"),
             {{st.part.ptr(), st.part_bytes}, {res, tokH}, {st.w(L.post_norm), H * 2}, {st.mid.ptr(), tokH},
              {st.normed.ptr(), tokH}});
        tg_params g = base;
        g.n = 2 * (uint32_t)I;
        g.k = (uint32_t)H;
        push(v, TG_KERNEL_LOCAL_GATE_UP, g, label(l, "gate_up"),
             {{st.normed.ptr(), tokH}, {st.w(L.gate_up), 2 * I * H * 2}, {st.mlp.ptr(), st.tokens_bytes((uint32_t)I)}});
        tg_params d = base;
        d.n = (uint32_t)H;
        d.k = (uint32_t)I;
        d.parts = st.tuning.down_parts;
        push(v, TG_KERNEL_LOCAL_PARTIAL, d, label(l, "down_proj"),
             {{st.mlp.ptr(), st.tokens_bytes((uint32_t)I)}, {st.w(L.down), H * I * 2}, {st.part.ptr(), st.part_bytes}});
        const uint64_t gain = l + 1 < s.layers ? st.layer[l + 1].in_norm : st.final_norm;
        push(v, TG_KERNEL_LOCAL_ADD_NORM, d, label(l, "down_proj_add"),
             {{st.part.ptr(), st.part_bytes}, {st.mid.ptr(), tokH}, {st.w(gain), H * 2}, {st.cur.ptr(), tokH},
              {st.normed.ptr(), tokH}});
    }
}

// A linear layer's f16 weight and bias.
struct Linear {
    Owned w, b;
    uint32_t n = 0, k = 0;
    int init(tg_ctx *ctx, uint32_t n_, uint32_t k_) {
        n = n_;
        k = k_;
        TG_TRY(w.alloc(ctx, align256((uint64_t)n * k * 2)));
        return b.alloc(ctx, align256((uint64_t)n * 2));
    }
    // "weight" or "bias".
    int load(const std::string &part, const std::string &name, const void *src, uint64_t count, tg_dtype dt) {
        const bool weight = part == "weight";
        if (!weight && part != "bias") return fail(TG_EINVAL, "no weight %s", name.c_str());
        const uint64_t want = weight ? (uint64_t)n * k : n;
        if (count != want) return fail(TG_ESHAPE, "%s: %llu values, not %llu", name.c_str(), (unsigned long long)count, (unsigned long long)want);
        std::vector<uint16_t> v;
        TG_TRY(to_f16(src, count, dt, v));
        return tg_mem_write(weight ? w.m : b.m, 0, v.data(), count * 2);
    }
};

static int wait_program(Program &p, uint64_t timeout_ns) { return program_wait(p, timeout_ns); }

}  // namespace tg

// ---- the sampler (local/dit.rs) ------------------------------------------------------------------

struct tg_sampler {
    tg_ctx *ctx = nullptr;
    LocalStack dit;
    uint32_t rows = 0, feat = 0, patch = 0, T = 0;
    std::vector<float> t, dt;  // the steps the DiT runs at
    Linear in_proj, cond_proj, out_proj;
    Owned mu, cond, noise, sampling, patch_buf, times;
    // The time and delta-time MLPs as the GPU would hold them (f16 values), for the host's tokens.
    std::vector<double> mlp[8];  // time l1 w, b, l2 w, b; delta l1 w, b, l2 w, b
    bool times_dirty = true;
    Owned stage_in, stage_out;  // pinned: mu, cond, noise, sampling; the patch
    Program prog;
    std::vector<Launch> launches;
    bool timed = false;
    uint64_t mu_bytes() const { return (uint64_t)rows * 2 * dit.shape.hidden * 2; }
    uint64_t patch_bytes() const { return (uint64_t)rows * feat * patch * 4; }
    ~tg_sampler() { program_release(prog); }
};

extern "C" int tg_cfm_schedule(uint32_t timesteps, float *out) {
    // dit.rs:41-54, in f32.
    if (!out || timesteps == 0) return fail(TG_EINVAL, "tg_cfm_schedule: null output or 0 steps");
    const uint32_t steps = timesteps + 1;
    const float step = (0.0f - 1.0f) / (float)timesteps;
    const float half_pi = (float)1.57079632679489661923;
    for (uint32_t i = 0; i < steps; i++) {
        const float t = i < steps / 2 ? 1.0f + step * (float)i : 0.0f - step * (float)(steps - i - 1);
        out[i] = t + (cosf(half_pi * t) - 1.0f + t);
    }
    return TG_OK;
}

extern "C" int tg_cfm_euler_steps(uint32_t timesteps, float *t_out, float *dt_out, size_t n, size_t *count) {
    // dit.rs:59-76: the first 4% of the steps (at least one) stay where they are.
    const uint32_t ts = std::max(1u, timesteps), len = ts + 1;
    std::vector<float> span(len);
    TG_TRY(tg_cfm_schedule(ts, span.data()));
    const uint32_t zero_init = std::max<uint32_t>(1, (uint32_t)((double)len * 0.04));
    float t = span[0], dt = span[0] - span[1];
    size_t k = 0;
    for (uint32_t step = 1; step < len; step++) {
        if (step > zero_init) {
            if (k < n && t_out) t_out[k] = t;
            if (k < n && dt_out) dt_out[k] = dt;
            k++;
        }
        t -= dt;
        if (step < len - 1) dt = t - span[step + 1];
    }
    if (count) *count = k;
    return TG_OK;
}

// dit.rs:386-422: SinusoidalPosEmb at scale 1000 in f32, then linear_2(SiLU(linear_1(x))) in f64.
static void sinusoid(float t, uint32_t hidden, std::vector<double> &out) {
    const uint32_t half = hidden / 2;
    out.assign(hidden, 0.0);
    const float rate = (float)(-(std::log(10000.0) / (double)(half - 1)));
    const float ts = t * 1000.0f;
    for (uint32_t i = 0; i < half; i++) {
        const float a = ts * expf((float)i * rate);
        out[i] = (double)sinf(a);
        out[half + i] = (double)cosf(a);
    }
}

static void time_mlp(const std::vector<double> *w, uint32_t H, const std::vector<double> &x, std::vector<double> &out) {
    std::vector<double> inner(H);
    for (uint32_t n = 0; n < H; n++) {
        double acc = 0;
        for (uint32_t k = 0; k < H; k++) acc += w[0][(uint64_t)n * H + k] * x[k];
        const double v = w[1][n] + acc;
        inner[n] = v / (1.0 + std::exp(-v));
    }
    out.assign(H, 0.0);
    for (uint32_t n = 0; n < H; n++) {
        double acc = 0;
        for (uint32_t k = 0; k < H; k++) acc += w[2][(uint64_t)n * H + k] * inner[k];
        out[n] = w[3][n] + acc;
    }
}

static int sampler_times(tg_sampler *s) {
    const uint32_t H = s->dit.shape.hidden;
    std::vector<double> e, delta, tok;
    sinusoid(0.0f, H, e);
    time_mlp(s->mlp + 4, H, e, delta);
    std::vector<uint16_t> bits((size_t)s->t.size() * H);
    for (size_t st = 0; st < s->t.size(); st++) {
        sinusoid(s->t[st], H, e);
        time_mlp(s->mlp, H, e, tok);
        for (uint32_t n = 0; n < H; n++) {
            const __half h = __double2half(tok[n] + delta[n]);
            memcpy(&bits[st * H + n], &h, 2);
        }
    }
    if (!bits.empty()) TG_TRY(tg_mem_write(s->times.m, 0, bits.data(), bits.size() * 2));
    s->times_dirty = false;
    return TG_OK;
}

// sampler_graph (dit.rs:112-271): the noise, the condition tokens once, then per step the time
// token and the noisy patch, the stack, and the Euler step.
static std::vector<Launch> sampler_launches(tg_sampler &s) {
    std::vector<Launch> v;
    LocalStack &st = s.dit;
    const uint32_t H = st.shape.hidden, T = s.T;
    const uint32_t time_at = 2, cond_at = 3, x_at = cond_at + s.patch;
    tg_params p = st.params();
    p.rows = s.rows;
    p.feat = s.feat;
    p.frames = s.patch;
    p.n = H;
    p.seqs = 2;
    const uint64_t pb = s.patch_bytes(), sb = (uint64_t)s.rows * 8;
    const uint64_t xb = st.tokens_bytes(H);
    push(v, TG_KERNEL_CFM_NOISE, p, "noise", {{s.noise.ptr(), pb}, {s.sampling.ptr(), sb}, {s.patch_buf.ptr(), pb}});
    tg_params c = p;
    c.first = cond_at;
    c.at = 0;
    c.copied = 2;
    c.flags = 1;
    push(v, TG_KERNEL_LOCAL_EMBED, c, "cond_proj",
         {{s.cond.ptr(), pb}, {s.cond_proj.w.ptr(), (uint64_t)H * s.feat * 2}, {s.cond_proj.b.ptr(), H * 2ull},
          {s.mu.ptr(), s.mu_bytes()}, {st.x.ptr(), xb}});
    for (size_t k = 0; k < s.t.size(); k++) {
        const std::string step = "step." + std::to_string(k);
        tg_params e = p;
        e.first = x_at;
        e.at = time_at;
        e.copied = 1;
        e.flags = 2;
        push(v, TG_KERNEL_LOCAL_EMBED, e, step + ".in_proj",
             {{s.patch_buf.ptr(), pb}, {s.in_proj.w.ptr(), (uint64_t)H * s.feat * 2}, {s.in_proj.b.ptr(), H * 2ull},
              {s.times.ptr() + k * H * 2, H * 2ull}, {st.x.ptr(), xb}});
        local_layers(st, v, step + ".dit");
        tg_params u = p;
        u.k = H;
        u.capacity = T;
        u.first = x_at;
        u.dt = s.dt[k];
        push(v, TG_KERNEL_DIT_EULER, u, step + ".euler",
             {{st.normed.ptr(), xb}, {s.out_proj.w.ptr(), (uint64_t)s.feat * H * 2}, {s.out_proj.b.ptr(), s.feat * 2ull},
              {s.sampling.ptr(), sb}, {s.patch_buf.ptr(), pb}});
    }
    return v;
}

extern "C" int tg_sampler_create(tg_ctx *ctx, const tg_shape *stack, uint32_t feat_dim, uint32_t patch_size,
                                 uint32_t timesteps, uint32_t rows, const tg_local_tuning *tuning, int timed,
                                 tg_sampler **out) {
    if (!ctx || !stack || !out) return fail(TG_EINVAL, "tg_sampler_create: null argument");
    *out = nullptr;
    if (rows == 0) return fail(TG_ESHAPE, "no rows");
    // dit.rs:196-212: channels a multiple of 8 (and of the euler kernel's clusters).
    if (feat_dim == 0 || feat_dim % 8 || patch_size == 0 || 2 * patch_size > 16 || timesteps == 0)
        return fail(TG_ESHAPE, "patches of %u frames of %u channels, %u steps", patch_size, feat_dim, timesteps);
    TG_CUDA(cudaSetDevice(ctx->device));
    std::unique_ptr<tg_sampler> s(new tg_sampler());
    s->ctx = ctx;
    s->rows = rows;
    s->feat = feat_dim;
    s->patch = patch_size;
    s->T = 3 + 2 * patch_size;
    s->timed = timed != 0;
    tg_shape sh = *stack;
    sh.capacity = s->T;
    TG_TRY(local_init(s->dit, ctx, sh, 2 * rows, tuning));
    size_t n = 0;
    TG_TRY(tg_cfm_euler_steps(timesteps, nullptr, nullptr, 0, &n));
    s->t.resize(n);
    s->dt.resize(n);
    TG_TRY(tg_cfm_euler_steps(timesteps, s->t.data(), s->dt.data(), n, &n));
    const uint32_t H = sh.hidden;
    TG_TRY(s->in_proj.init(ctx, H, feat_dim));
    TG_TRY(s->cond_proj.init(ctx, H, feat_dim));
    TG_TRY(s->out_proj.init(ctx, feat_dim, H));
    TG_TRY(s->mu.alloc(ctx, s->mu_bytes()));
    for (Owned *o : {&s->cond, &s->noise, &s->patch_buf}) TG_TRY(o->alloc(ctx, s->patch_bytes()));
    TG_TRY(s->sampling.alloc(ctx, (uint64_t)rows * 8));
    TG_TRY(s->times.alloc(ctx, std::max<uint64_t>(16, (uint64_t)n * H * 2)));
    const uint64_t HH = (uint64_t)H * H;
    const uint64_t sizes[8] = {HH, H, HH, H, HH, H, HH, H};
    for (int i = 0; i < 8; i++) s->mlp[i].assign(sizes[i], 0.0);
    TG_TRY(s->stage_in.alloc(ctx, s->mu_bytes() + 2 * s->patch_bytes() + (uint64_t)rows * 8, TG_RES_UPLOAD));
    TG_TRY(s->stage_out.alloc(ctx, s->patch_bytes(), TG_RES_READBACK));
    s->launches = sampler_launches(*s);
    TG_TRY(program_build(ctx, s->launches, s->timed, s->prog));
    *out = s.release();
    return TG_OK;
}

extern "C" int tg_sampler_destroy(tg_sampler *s) {
    if (!s) return TG_OK;
    cudaSetDevice(s->ctx->device);
    if (s->prog.pending) wait_program(s->prog, 0);
    delete s;
    return TG_OK;
}

extern "C" int tg_sampler_load(tg_sampler *s, const char *name_c, const void *src, uint64_t count, tg_dtype src_dtype) {
    if (!s || !name_c || !src) return fail(TG_EINVAL, "tg_sampler_load: null argument");
    TG_CUDA(cudaSetDevice(s->ctx->device));
    const std::string name = name_c, pre = "feat_decoder.estimator.";
    if (name.compare(0, pre.size(), pre) != 0) return fail(TG_EINVAL, "sampler: no weight %s", name_c);
    const std::string rest = name.substr(pre.size());
    if (rest.compare(0, 8, "decoder.") == 0) return local_load(s->dit, rest.substr(8), src, count, src_dtype);
    for (auto &lin : {std::make_pair("in_proj.", &s->in_proj), std::make_pair("cond_proj.", &s->cond_proj),
                      std::make_pair("out_proj.", &s->out_proj)}) {
        const std::string p = lin.first;
        if (rest.compare(0, p.size(), p) == 0) return lin.second->load(rest.substr(p.size()), name, src, count, src_dtype);
    }
    // The timestep MLPs, kept on the host as the GPU would hold them (f16 values).
    const char *mlps[2] = {"time_mlp.", "delta_time_mlp."};
    for (int m = 0; m < 2; m++) {
        const std::string p = mlps[m];
        if (rest.compare(0, p.size(), p) != 0) continue;
        const std::string part = rest.substr(p.size());
        const char *parts[4] = {"linear_1.weight", "linear_1.bias", "linear_2.weight", "linear_2.bias"};
        for (int i = 0; i < 4; i++) {
            if (part != parts[i]) continue;
            std::vector<double> &dst = s->mlp[4 * m + i];
            if (count != dst.size())
                return fail(TG_ESHAPE, "%s: %llu values, not %zu", name_c, (unsigned long long)count, dst.size());
            std::vector<uint16_t> bits;
            TG_TRY(to_f16(src, count, src_dtype, bits));
            for (uint64_t j = 0; j < count; j++) dst[j] = f16_value(bits[j]);
            s->times_dirty = true;
            return TG_OK;
        }
    }
    return fail(TG_EINVAL, "sampler: no weight %s", name_c);
}

static int sampler_run(tg_sampler *s, const void *mu, const float *cond, const float *noise, const float *sampling,
                       float *patch_dev, bool device) {
    TG_CUDA(cudaSetDevice(s->ctx->device));
    std::lock_guard<std::mutex> lock(s->ctx->mu);
    if (s->prog.pending) TG_TRY(wait_program(s->prog, 0));
    if (s->times_dirty) TG_TRY(sampler_times(s));
    const uint64_t mb = s->mu_bytes(), pb = s->patch_bytes(), sb = (uint64_t)s->rows * 8;
    cudaStream_t st = s->ctx->stream;
    if (device) {
        TG_CUDA(cudaMemcpyAsync(s->mu.ptr(), mu, mb, cudaMemcpyDeviceToDevice, st));
        TG_CUDA(cudaMemcpyAsync(s->cond.ptr(), cond, pb, cudaMemcpyDeviceToDevice, st));
        TG_CUDA(cudaMemcpyAsync(s->noise.ptr(), noise, pb, cudaMemcpyDeviceToDevice, st));
        TG_CUDA(cudaMemcpyAsync(s->sampling.ptr(), sampling, sb, cudaMemcpyDeviceToDevice, st));
    } else {
        char *h = s->stage_in.host();
        memcpy(h, mu, mb);
        memcpy(h + mb, cond, pb);
        memcpy(h + mb + pb, noise, pb);
        memcpy(h + mb + 2 * pb, sampling, sb);
        char *d = s->stage_in.ptr();
        TG_CUDA(cudaMemcpyAsync(s->mu.ptr(), d, mb, cudaMemcpyDefault, st));
        TG_CUDA(cudaMemcpyAsync(s->cond.ptr(), d + mb, pb, cudaMemcpyDefault, st));
        TG_CUDA(cudaMemcpyAsync(s->noise.ptr(), d + mb + pb, pb, cudaMemcpyDefault, st));
        TG_CUDA(cudaMemcpyAsync(s->sampling.ptr(), d + mb + 2 * pb, sb, cudaMemcpyDefault, st));
    }
    TG_TRY(program_launch(s->prog));
    TG_CUDA(cudaMemcpyAsync(device ? (void *)patch_dev : (void *)s->stage_out.ptr(), s->patch_buf.ptr(), pb,
                            device ? cudaMemcpyDeviceToDevice : cudaMemcpyDefault, st));
    return TG_OK;
}

extern "C" int tg_sampler_sample(tg_sampler *s, const uint16_t *mu, const float *cond, const float *noise,
                                 const float *sampling, float *patch) {
    if (!s || !mu || !cond || !noise || !sampling || !patch) return fail(TG_EINVAL, "tg_sampler_sample: null argument");
    TG_TRY(sampler_run(s, mu, cond, noise, sampling, nullptr, false));
    TG_TRY(wait_program(s->prog, 60ull * 1000000000ull));
    TG_CUDA(cudaStreamSynchronize(s->ctx->stream));
    memcpy(patch, s->stage_out.host(), s->patch_bytes());
    // generator.rs:418-421: a patch that is not finite ends its request (the stop head might
    // never say to stop after it).
    const uint64_t per_row = (uint64_t)s->feat * s->patch;
    for (uint32_t r = 0; r < s->rows; r++)
        for (uint64_t i = 0; i < per_row; i++)
            if (!std::isfinite(patch[r * per_row + i]))
                return fail(TG_ENOTFINITE, "the patch of row %u came out NaN or infinite", r);
    return TG_OK;
}

extern "C" int tg_sampler_sample_device(tg_sampler *s, const void *mu, const float *cond, const float *noise,
                                        const float *sampling, float *patch) {
    if (!s || !mu || !cond || !noise || !sampling || !patch) return fail(TG_EINVAL, "tg_sampler_sample_device: null argument");
    return sampler_run(s, mu, cond, noise, sampling, patch, true);
}

extern "C" int tg_sampler_wait(tg_sampler *s, uint64_t timeout_ns) {
    if (!s) return fail(TG_EINVAL, "null sampler");
    return wait_program(s->prog, timeout_ns);
}

extern "C" int tg_sampler_steps(const tg_sampler *s, float *t, float *dt, size_t n, size_t *count) {
    if (!s) return fail(TG_EINVAL, "null sampler");
    for (size_t i = 0; i < s->t.size() && i < n; i++) {
        if (t) t[i] = s->t[i];
        if (dt) dt[i] = s->dt[i];
    }
    if (count) *count = s->t.size();
    return TG_OK;
}

extern "C" int tg_sampler_elapsed_ns(tg_sampler *s, double *ns) {
    if (!s || !ns) return fail(TG_EINVAL, "null argument");
    TG_TRY(wait_program(s->prog, 0));
    *ns = program_elapsed_ns(s->prog);
    return TG_OK;
}

extern "C" int tg_sampler_timings(tg_sampler *s, double *ns, size_t n, size_t *n_dispatches) {
    if (!s) return fail(TG_EINVAL, "null sampler");
    if (n_dispatches) *n_dispatches = s->launches.size();
    if (!ns) return TG_OK;
    TG_TRY(wait_program(s->prog, 0));
    return program_timings(s->prog, ns, n);
}

extern "C" int tg_sampler_dispatch_label(tg_sampler *s, size_t i, char *label, size_t label_bytes) {
    if (!s || !label) return fail(TG_EINVAL, "null argument");
    if (i >= s->launches.size()) return fail(TG_EINVAL, "dispatch %zu of %zu", i, s->launches.size());
    snprintf(label, label_bytes, "%s", s->launches[i].label.c_str());
    return TG_OK;
}

extern "C" uint64_t tg_sampler_weight_bytes(const tg_sampler *s) {
    return s ? s->dit.weight_bytes + 2ull * ((uint64_t)s->feat * s->dit.shape.hidden + s->feat) : 0;
}

// ---- the local encoder (local/encoder.rs) --------------------------------------------------------

struct tg_encoder {
    tg_ctx *ctx = nullptr;
    LocalStack enc;
    uint32_t rows = 0, feat = 0, patch = 0, T = 0;
    Linear in_proj;
    Owned special, patches, out, stage_in, stage_out;
    Program prog;
    std::vector<Launch> launches;
    bool timed = false;
    uint64_t patch_bytes() const { return (uint64_t)rows * feat * patch * 4; }
    uint64_t out_bytes() const { return (uint64_t)rows * enc.shape.hidden * 2; }
    ~tg_encoder() { program_release(prog); }
};

// encoder_graph (encoder.rs:41-124): the learned token and the frames projected, the stack, and
// each sequence's first token.
static std::vector<Launch> encoder_launches(tg_encoder &e) {
    std::vector<Launch> v;
    LocalStack &st = e.enc;
    const uint32_t H = st.shape.hidden;
    tg_params p = st.params();
    p.rows = e.rows;
    p.feat = e.feat;
    p.frames = e.patch;
    p.n = H;
    p.seqs = 1;
    p.first = 1;
    p.at = 0;
    p.copied = 1;
    p.flags = 2;
    const uint64_t xb = st.tokens_bytes(H);
    push(v, TG_KERNEL_LOCAL_EMBED, p, "in_proj",
         {{e.patches.ptr(), e.patch_bytes()}, {e.in_proj.w.ptr(), (uint64_t)H * e.feat * 2}, {e.in_proj.b.ptr(), H * 2ull},
          {e.special.ptr(), H * 2ull}, {st.x.ptr(), xb}});
    local_layers(st, v, "encoder");
    tg_params r = p;
    push(v, TG_KERNEL_LOCAL_ROWS, r, "first", {{st.normed.ptr(), xb}, {e.out.ptr(), e.out_bytes()}});
    return v;
}

extern "C" int tg_encoder_create(tg_ctx *ctx, const tg_shape *stack, uint32_t feat_dim, uint32_t patch_size,
                                 uint32_t rows, const tg_local_tuning *tuning, int timed, tg_encoder **out) {
    if (!ctx || !stack || !out) return fail(TG_EINVAL, "tg_encoder_create: null argument");
    *out = nullptr;
    if (rows == 0) return fail(TG_ESHAPE, "no rows");
    if (feat_dim == 0 || feat_dim % 8 || patch_size == 0 || patch_size > 8)
        return fail(TG_ESHAPE, "patches of %u frames of %u channels", patch_size, feat_dim);
    TG_CUDA(cudaSetDevice(ctx->device));
    std::unique_ptr<tg_encoder> e(new tg_encoder());
    e->ctx = ctx;
    e->rows = rows;
    e->feat = feat_dim;
    e->patch = patch_size;
    e->T = 1 + patch_size;
    e->timed = timed != 0;
    tg_shape sh = *stack;
    sh.capacity = e->T;
    TG_TRY(local_init(e->enc, ctx, sh, rows, tuning));
    const uint32_t H = sh.hidden;
    TG_TRY(e->in_proj.init(ctx, H, feat_dim));
    TG_TRY(e->special.alloc(ctx, align256((uint64_t)H * 2)));
    TG_TRY(e->patches.alloc(ctx, e->patch_bytes()));
    TG_TRY(e->out.alloc(ctx, e->out_bytes()));
    TG_TRY(e->stage_in.alloc(ctx, e->patch_bytes(), TG_RES_UPLOAD));
    TG_TRY(e->stage_out.alloc(ctx, e->out_bytes(), TG_RES_READBACK));
    e->launches = encoder_launches(*e);
    TG_TRY(program_build(ctx, e->launches, e->timed, e->prog));
    *out = e.release();
    return TG_OK;
}

extern "C" int tg_encoder_destroy(tg_encoder *e) {
    if (!e) return TG_OK;
    cudaSetDevice(e->ctx->device);
    if (e->prog.pending) wait_program(e->prog, 0);
    delete e;
    return TG_OK;
}

extern "C" int tg_encoder_load(tg_encoder *e, const char *name_c, const void *src, uint64_t count, tg_dtype src_dtype) {
    if (!e || !name_c || !src) return fail(TG_EINVAL, "tg_encoder_load: null argument");
    TG_CUDA(cudaSetDevice(e->ctx->device));
    const std::string name = name_c, pre = "feat_encoder.";
    if (name.compare(0, pre.size(), pre) != 0) return fail(TG_EINVAL, "encoder: no weight %s", name_c);
    const std::string rest = name.substr(pre.size());
    if (rest.compare(0, 8, "encoder.") == 0) return local_load(e->enc, rest.substr(8), src, count, src_dtype);
    if (rest.compare(0, 8, "in_proj.") == 0) return e->in_proj.load(rest.substr(8), name, src, count, src_dtype);
    if (rest == "special_token") {
        const uint64_t H = e->enc.shape.hidden;
        if (count != H) return fail(TG_ESHAPE, "%s: %llu values, not %llu", name_c, (unsigned long long)count, (unsigned long long)H);
        std::vector<uint16_t> v;
        TG_TRY(to_f16(src, count, src_dtype, v));
        return tg_mem_write(e->special.m, 0, v.data(), count * 2);
    }
    return fail(TG_EINVAL, "encoder: no weight %s", name_c);
}

static int encoder_run(tg_encoder *e, const float *patches, void *out_dev, bool device) {
    TG_CUDA(cudaSetDevice(e->ctx->device));
    std::lock_guard<std::mutex> lock(e->ctx->mu);
    if (e->prog.pending) TG_TRY(wait_program(e->prog, 0));
    cudaStream_t st = e->ctx->stream;
    if (device) {
        TG_CUDA(cudaMemcpyAsync(e->patches.ptr(), patches, e->patch_bytes(), cudaMemcpyDeviceToDevice, st));
    } else {
        memcpy(e->stage_in.host(), patches, e->patch_bytes());
        TG_CUDA(cudaMemcpyAsync(e->patches.ptr(), e->stage_in.ptr(), e->patch_bytes(), cudaMemcpyDefault, st));
    }
    TG_TRY(program_launch(e->prog));
    TG_CUDA(cudaMemcpyAsync(device ? out_dev : (void *)e->stage_out.ptr(), e->out.ptr(), e->out_bytes(),
                            device ? cudaMemcpyDeviceToDevice : cudaMemcpyDefault, st));
    return TG_OK;
}

extern "C" int tg_encoder_encode(tg_encoder *e, const float *patches, uint16_t *out) {
    if (!e || !patches || !out) return fail(TG_EINVAL, "tg_encoder_encode: null argument");
    TG_TRY(encoder_run(e, patches, nullptr, false));
    TG_TRY(wait_program(e->prog, 60ull * 1000000000ull));
    TG_CUDA(cudaStreamSynchronize(e->ctx->stream));
    memcpy(out, e->stage_out.host(), e->out_bytes());
    return TG_OK;
}

extern "C" int tg_encoder_encode_device(tg_encoder *e, const float *patches, void *out) {
    if (!e || !patches || !out) return fail(TG_EINVAL, "tg_encoder_encode_device: null argument");
    return encoder_run(e, patches, out, true);
}

extern "C" int tg_encoder_wait(tg_encoder *e, uint64_t timeout_ns) {
    if (!e) return fail(TG_EINVAL, "null encoder");
    return wait_program(e->prog, timeout_ns);
}

extern "C" int tg_encoder_elapsed_ns(tg_encoder *e, double *ns) {
    if (!e || !ns) return fail(TG_EINVAL, "null argument");
    TG_TRY(wait_program(e->prog, 0));
    *ns = program_elapsed_ns(e->prog);
    return TG_OK;
}

extern "C" int tg_encoder_timings(tg_encoder *e, double *ns, size_t n, size_t *n_dispatches) {
    if (!e) return fail(TG_EINVAL, "null encoder");
    if (n_dispatches) *n_dispatches = e->launches.size();
    if (!ns) return TG_OK;
    TG_TRY(wait_program(e->prog, 0));
    return program_timings(e->prog, ns, n);
}

extern "C" int tg_encoder_dispatch_label(tg_encoder *e, size_t i, char *label, size_t label_bytes) {
    if (!e || !label) return fail(TG_EINVAL, "null argument");
    if (i >= e->launches.size()) return fail(TG_EINVAL, "dispatch %zu of %zu", i, e->launches.size());
    snprintf(label, label_bytes, "%s", e->launches[i].label.c_str());
    return TG_OK;
}

extern "C" uint64_t tg_encoder_weight_bytes(const tg_encoder *e) {
    return e ? e->enc.weight_bytes + 2ull * ((uint64_t)e->enc.shape.hidden * e->feat + 2ull * e->enc.shape.hidden) : 0;
}
