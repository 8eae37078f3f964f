// The stack's handles behind the C ABI (tg_decoder, tg_prefill) and what the decoder, the prefill
// and the continuous-batching server share of them.
#pragma once

#include <map>
#include <string>
#include <vector>

#include "tg_internal.h"

namespace tg {

// A device (or pinned host) allocation freed with its owner.
struct Owned {
    tg_mem *m = nullptr;
    Owned() = default;
    Owned(const Owned &) = delete;
    Owned &operator=(const Owned &) = delete;
    ~Owned() { tg_mem_free(m); }
    int alloc(tg_ctx *ctx, uint64_t bytes, tg_residence r = TG_RES_DEVICE) { return tg_mem_alloc(ctx, bytes, r, &m); }
    char *ptr() const { return static_cast<char *>(m->ptr); }
    char *host() const { return static_cast<char *>(m->host); }
};

inline uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

struct LayerOffsets {
    uint64_t qkv, o, gate_up, down, in_norm, post_norm;
};

// One recorded decode step for `rows` rows: the decoder records one for each of program_rows(its
// rows) (the generator's row buckets, crates/graph/src/generator.rs:113-123), all over the same
// buffers, so that a step of n rows runs the smallest that holds them.
struct Bucket {
    uint32_t rows = 0;
    Program prog;
    std::vector<Launch> launches;
};

// Each power of two below `rows`, then `rows` (generator.rs:115-123).
std::vector<uint32_t> program_rows(uint32_t rows);

// Pinned host buffers for small uploads issued back to back: each is reused only after the copy
// out of it has run (an event per buffer), so that the host never waits on the step before.
struct StageRing {
    std::vector<tg_mem *> bufs;
    std::vector<cudaEvent_t> done;
    size_t next = 0;
    StageRing() = default;
    StageRing(const StageRing &) = delete;
    StageRing &operator=(const StageRing &) = delete;
    ~StageRing() {
        for (tg_mem *m : bufs) tg_mem_free(m);
        for (cudaEvent_t e : done) cudaEventDestroy(e);
    }
    int init(tg_ctx *ctx, size_t entries, uint64_t bytes) {
        for (size_t i = 0; i < entries; i++) {
            tg_mem *m = nullptr;
            const int st = tg_mem_alloc(ctx, bytes, TG_RES_UPLOAD, &m);
            if (st) return st;
            bufs.push_back(m);
            cudaEvent_t e;
            TG_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            done.push_back(e);
        }
        return TG_OK;
    }
    // The next buffer, once its last copy has run.
    int acquire(size_t &i) {
        i = next;
        next = (next + 1) % bufs.size();
        TG_CUDA(cudaEventSynchronize(done[i]));
        return TG_OK;
    }
    void *host(size_t i) const { return bufs[i]->host; }
    void *ptr(size_t i) const { return bufs[i]->ptr; }
    // Copies `bytes` of buffer i to `dst` on `s` and marks the buffer busy until the copy has run.
    int upload(size_t i, void *dst, uint64_t bytes, cudaStream_t s) {
        TG_CUDA(cudaMemcpyAsync(dst, bufs[i]->ptr, bytes, cudaMemcpyDefault, s));
        TG_CUDA(cudaEventRecord(done[i], s));
        return TG_OK;
    }
};

#define TG_TRY(x)                 \
    do {                          \
        const int st_ = (x);      \
        if (st_) return st_;      \
    } while (0)

}  // namespace tg

struct tg_decoder {
    tg_ctx *ctx = nullptr;
    tg_shape shape{};
    std::vector<double> factors;
    uint32_t rows = 0, slots = 0;
    tg_dtype dtype = TG_F32;
    bool timed = false;
    uint64_t esize = 4;
    // Weights: every layer's projections (storage type) and gains (f32), then the final gain.
    tg::Owned weights;
    std::vector<tg::LayerOffsets> layer;
    uint64_t final_norm = 0;
    tg::Owned cos, sin, kcache, vcache;  // caches: [layers][slots][kv][capacity][hd]
    uint64_t cache_layer = 0;            // bytes of one layer's cache
    // Activations of the step, [rows][...].
    tg::Owned x_in, h, mid, out, q, att, mlp, words;
    tg::Owned po, pml, psync, offs;  // the persistent step's attention partials, barrier words, weight offsets
    bool persistent = false;         // the step is one persistent launch (rows <= 2), else six kernels a layer
    bool tensor = false;             // the projections run on tcgen05 (rows >= DTC_MIN_ROWS, bf16)
    // With `tensor`: the projections as the prefill's tcgen05 GEMMs (a weight tile a block over the
    // whole of K, bf16 activations), else as split-K clusters over f32 activations split into hi/lo.
    bool gemm = false;
    tg::Owned g_normed, g_q, g_att, g_proj, g_mlp;  // the GEMM family's activations
    tg::Owned g_counts;  // its attention's arrival counters, [rows][kv_heads], zero between launches
    tg::Owned stage_x, stage_out;  // pinned host staging
    cudaEvent_t out_done = nullptr;  // recorded after a step's output copy (tg_decoder_step_rows_n)
    tg::StageRing word_ring;                    // placements of device-resident steps
    std::vector<tg::Bucket> buckets;            // ascending rows; the last holds `rows`
    size_t active = 0;                          // the bucket the next start runs
    uint32_t n_active = 0;                      // the rows given to the last set_rows

    // Releases the recorded programs and the event, also when creation fails part way (the
    // caller has waited for any run in flight and made the decoder's device current).
    ~tg_decoder() {
        for (tg::Bucket &b : buckets) tg::program_release(b.prog);
        if (out_done) cudaEventDestroy(out_done);
    }

    uint64_t width() const { return (uint64_t)(shape.heads + 2 * shape.kv_heads) * shape.head_dim; }
    uint64_t attn() const { return (uint64_t)shape.heads * shape.head_dim; }
    tg_params params(uint32_t R) const {
        tg_params p{};
        p.dtype = dtype;
        p.hidden = shape.hidden;
        p.inner = shape.inner;
        p.heads = shape.heads;
        p.kv_heads = shape.kv_heads;
        p.head_dim = shape.head_dim;
        p.capacity = shape.capacity;
        p.rows = R;
        p.slots = slots;
        p.eps = shape.eps;
        p.residual_scale = shape.residual_scale;
        p.rope = shape.rope;
        return p;
    }
    tg_params params() const { return params(rows); }
    char *w(uint64_t off) const { return weights.ptr() + off; }
    char *kc(uint32_t l) const { return kcache.ptr() + l * cache_layer; }
    char *vc(uint32_t l) const { return vcache.ptr() + l * cache_layer; }
    tg::Bucket &cur() { return buckets[active]; }
    tg::Program &prog() { return buckets[active].prog; }
    // Waits for whichever bucket is still running.
    int wait_pending() {
        for (tg::Bucket &b : buckets)
            if (b.prog.pending) TG_TRY(tg::program_wait(b.prog, 0));
        return TG_OK;
    }
};

struct tg_prefill {
    tg_decoder *d = nullptr;
    uint32_t max_rows = 0;  // a multiple of 128
    bool timed = false;
    tg::Owned words, x_in, h, mid, normed, qkv, q, att, proj, gu, mlp, out;
    tg::Owned stage_x, stage_words, stage_out;
    std::map<uint32_t, tg::Program> programs;  // by rows, a multiple of 128
    tg::Program *last = nullptr;

    ~tg_prefill() {
        for (auto &kv : programs) tg::program_release(kv.second);
    }
};

namespace tg {

// The smallest bucket of `d` that holds `n` rows (n <= d->rows).
size_t bucket_for(const tg_decoder &d, uint32_t n);
// Makes bucket `b` the active one and writes the placement of its rows (`rows`, n of them, then
// spare rows) to the device, on the context's stream, through the word ring (no wait on an
// earlier step).
int decoder_place(tg_decoder &d, size_t b, uint32_t n, const tg_row *rows);
// Prefill of `runs` in one launch (x and out on the host or the device; out on the device leaves
// the program running on the context's stream).
int prefill_rows(tg_prefill *p, const tg_run *runs, uint32_t n_runs, const float *x, bool x_on_device, float *out,
                 bool out_on_device);

}  // namespace tg
