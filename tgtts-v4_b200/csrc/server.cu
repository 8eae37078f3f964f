// Continuous batching over one decoder and its prefill: requests hold the decoder's slots, each
// step packs the requests under way into rows and runs the smallest row bucket that holds them,
// and requests are admitted between steps by a prefill into their slots. This is the generator's
// pattern (crates/graph/src/generator.rs:99-123 slots and programs, :189-262 start, :295-352
// step) on the backbone alone: a request's next input is its last output, fed back on the GPU
// (the backbone's caller, which turns an output into the next input, is outside this library).
#include <algorithm>
#include <cstring>
#include <memory>
#include <vector>

#include "model.h"
#include "tg_common.cuh"

using namespace tg;

namespace {

// x_in[b] = next[slot of row b] for the n rows of a bucket of R rows (words as the decoder's).
__global__ void __launch_bounds__(256)
    gather_rows_kernel(const uint32_t *__restrict__ words, uint32_t R, uint32_t slots, const float4 *__restrict__ next,
                       float4 *__restrict__ x_in, uint32_t h4) {
    const uint32_t b = blockIdx.x;
    const uint32_t slot = slots > 1 ? words[R + b] : 0u;
    if (words[b] == TG_SPARE || slot >= slots) return;
    for (uint32_t i = threadIdx.x; i < h4; i += blockDim.x) x_in[(size_t)b * h4 + i] = next[(size_t)slot * h4 + i];
}

// next[slot of row b] = out[b].
__global__ void __launch_bounds__(256)
    scatter_rows_kernel(const uint32_t *__restrict__ words, uint32_t R, uint32_t slots, const float4 *__restrict__ out,
                        float4 *__restrict__ next, uint32_t h4) {
    const uint32_t b = blockIdx.x;
    const uint32_t slot = slots > 1 ? words[R + b] : 0u;
    if (words[b] == TG_SPARE || slot >= slots) return;
    for (uint32_t i = threadIdx.x; i < h4; i += blockDim.x) next[(size_t)slot * h4 + i] = out[(size_t)b * h4 + i];
}

struct Request {
    bool held = false;
    uint32_t position = 0;  // where its next step decodes
    uint32_t left = 0;      // steps still to run
};

}  // namespace

struct tg_server {
    tg_decoder *d = nullptr;
    tg_prefill *p = nullptr;
    std::vector<Request> req;  // by slot
    Owned next;                // [slots][hidden] f32: each slot's next input
    Owned pre_out;             // [prefill max rows][hidden] f32: a prefill's outputs
    Owned stage_x, stage_out;  // pinned [rows][hidden]
    uint64_t steps = 0, tokens = 0;
};

extern "C" int tg_server_create(tg_decoder *d, tg_prefill *p, tg_server **out) {
    if (!d || !p || !out) return fail(TG_EINVAL, "tg_server_create: null argument");
    *out = nullptr;
    if (p->d != d) return fail(TG_EINVAL, "the prefill is not over this decoder");
    if (d->rows != d->slots) return fail(TG_ESHAPE, "a server needs a row for each slot (%u rows, %u slots)", d->rows, d->slots);
    TG_CUDA(cudaSetDevice(d->ctx->device));
    std::unique_ptr<tg_server> s(new tg_server());
    s->d = d;
    s->p = p;
    s->req.resize(d->slots);
    const uint64_t H = d->shape.hidden, F = 4;
    TG_TRY(s->next.alloc(d->ctx, (uint64_t)d->slots * H * F));
    TG_TRY(s->pre_out.alloc(d->ctx, (uint64_t)p->max_rows * H * F));
    TG_TRY(s->stage_x.alloc(d->ctx, (uint64_t)d->rows * H * F, TG_RES_UPLOAD));
    TG_TRY(s->stage_out.alloc(d->ctx, (uint64_t)d->rows * H * F, TG_RES_READBACK));
    *out = s.release();
    return TG_OK;
}

extern "C" int tg_server_destroy(tg_server *s) {
    if (!s) return TG_OK;
    cudaSetDevice(s->d->ctx->device);
    s->d->wait_pending();
    delete s;
    return TG_OK;
}

extern "C" int tg_server_start(tg_server *s, const tg_request *reqs, uint32_t n, const float *x) {
    if (!s || (n && (!reqs || !x))) return fail(TG_EINVAL, "tg_server_start: null argument");
    tg_decoder *d = s->d;
    const tg_shape &sh = d->shape;
    const uint64_t H = sh.hidden, F = 4;
    std::vector<bool> seen(d->slots, false);
    for (uint32_t i = 0; i < n; i++) {
        const tg_request &r = reqs[i];
        if (r.slot >= d->slots || seen[r.slot] || r.start >= r.len || r.steps == 0 ||
            (uint64_t)r.len + r.steps > sh.capacity)
            return fail(TG_ESHAPE, "request %u: slot %u of %u, positions %u..%u and %u steps in a cache of %u", i,
                        r.slot, d->slots, r.start, r.len, r.steps, sh.capacity);
        seen[r.slot] = true;
    }
    TG_CUDA(cudaSetDevice(d->ctx->device));
    // Runs go into launches of at most max_rows rows (each run's rows start on a tile boundary); a
    // run longer than that is cut into pieces that run one after another (prefill.rs:487-502).
    struct Piece {
        tg_run run;
        uint64_t src_row;  // first row of x
        bool last;         // the request's last piece
    };
    std::vector<Piece> pieces;
    uint64_t src = 0;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t first = reqs[i].start;
        for (uint32_t done = first; done < reqs[i].len;) {
            const uint32_t len = std::min(reqs[i].len - done, s->p->max_rows);
            pieces.push_back({{done, len, reqs[i].slot}, src + (done - first), done + len == reqs[i].len});
            done += len;
        }
        src += reqs[i].len - first;
    }
    // Pieces of one slot run in order; each launch takes pieces of distinct slots while they fit.
    size_t at = 0;
    std::vector<bool> launched(pieces.size(), false);
    while (at < pieces.size()) {
        std::vector<size_t> take;
        std::vector<bool> slot_in(d->slots, false);
        uint32_t rows = 0;
        for (size_t i = at; i < pieces.size(); i++) {
            if (launched[i]) continue;
            const Piece &pc = pieces[i];
            if (slot_in[pc.run.slot]) break;  // a later piece of a slot in this launch waits
            const uint32_t start = (rows + RUN_ALIGN - 1) / RUN_ALIGN * RUN_ALIGN;
            if (start + pc.run.len > s->p->max_rows) break;
            slot_in[pc.run.slot] = true;
            rows = start + pc.run.len;
            take.push_back(i);
        }
        std::vector<tg_run> runs;
        std::vector<float> xs;
        for (size_t i : take) {
            runs.push_back(pieces[i].run);
            xs.insert(xs.end(), x + pieces[i].src_row * H, x + (pieces[i].src_row + pieces[i].run.len) * H);
        }
        TG_TRY(prefill_rows(s->p, runs.data(), (uint32_t)runs.size(), xs.data(), false,
                            reinterpret_cast<float *>(s->pre_out.ptr()), true));
        // The prompt's last output is the request's first input.
        uint64_t row = 0;
        for (size_t i : take) {
            const Piece &pc = pieces[i];
            row += pc.run.len;
            if (pc.last)
                TG_CUDA(cudaMemcpyAsync(s->next.ptr() + (uint64_t)pc.run.slot * H * F, s->pre_out.ptr() + (row - 1) * H * F,
                                        H * F, cudaMemcpyDeviceToDevice, d->ctx->stream));
            launched[i] = true;
        }
        while (at < pieces.size() && launched[at]) at++;
    }
    for (uint32_t i = 0; i < n; i++) s->req[reqs[i].slot] = {true, reqs[i].len, reqs[i].steps};
    return TG_OK;
}

extern "C" int tg_server_under_way(const tg_server *s, uint32_t *slots, uint32_t *n) {
    if (!s || !n) return fail(TG_EINVAL, "tg_server_under_way: null argument");
    uint32_t k = 0;
    for (uint32_t slot = 0; slot < s->req.size(); slot++)
        if (s->req[slot].held && s->req[slot].left > 0) {
            if (slots) slots[k] = slot;
            k++;
        }
    *n = k;
    return TG_OK;
}

extern "C" int tg_server_step(tg_server *s, const float *x, uint32_t *n_rows, uint32_t *slots, float *out) {
    if (!s || !n_rows) return fail(TG_EINVAL, "tg_server_step: null argument");
    tg_decoder *d = s->d;
    std::vector<uint32_t> under;
    for (uint32_t slot = 0; slot < s->req.size(); slot++)
        if (s->req[slot].held && s->req[slot].left > 0) under.push_back(slot);
    const uint32_t n = (uint32_t)under.size();
    *n_rows = n;
    if (n == 0) return TG_OK;
    TG_CUDA(cudaSetDevice(d->ctx->device));
    const uint64_t H = d->shape.hidden, F = 4;
    std::vector<tg_row> rows(n);
    for (uint32_t b = 0; b < n; b++) rows[b] = {s->req[under[b]].position, under[b]};
    std::lock_guard<std::mutex> lock(d->ctx->mu);
    if (x) {
        TG_TRY(d->wait_pending());  // the staging buffer is free once the step before has run
        memcpy(s->stage_x.host(), x, n * H * F);
    }
    const size_t b = bucket_for(*d, n);
    const uint32_t R = d->buckets[b].rows;
    TG_TRY(decoder_place(*d, b, n, rows.data()));
    cudaStream_t st = d->ctx->stream;
    const uint32_t h4 = (uint32_t)(H / 4);
    if (x) {
        TG_CUDA(cudaMemcpyAsync(d->x_in.ptr(), s->stage_x.ptr(), n * H * F, cudaMemcpyDefault, st));
    } else {
        gather_rows_kernel<<<n, 256, 0, st>>>(reinterpret_cast<const uint32_t *>(d->words.ptr()), R, d->slots,
                                              reinterpret_cast<const float4 *>(s->next.ptr()),
                                              reinterpret_cast<float4 *>(d->x_in.ptr()), h4);
        TG_CUDA(cudaGetLastError());
    }
    TG_TRY(program_launch(d->prog()));
    scatter_rows_kernel<<<n, 256, 0, st>>>(reinterpret_cast<const uint32_t *>(d->words.ptr()), R, d->slots,
                                           reinterpret_cast<const float4 *>(d->out.ptr()),
                                           reinterpret_cast<float4 *>(s->next.ptr()), h4);
    TG_CUDA(cudaGetLastError());
    for (uint32_t i = 0; i < n; i++) {
        Request &r = s->req[under[i]];
        r.position++;
        r.left--;
        if (slots) slots[i] = under[i];
    }
    s->steps++;
    s->tokens += n;
    if (out) {
        TG_CUDA(cudaMemcpyAsync(s->stage_out.ptr(), d->out.ptr(), n * H * F, cudaMemcpyDefault, st));
        TG_TRY(program_wait(d->prog(), 60ull * 1000000000ull));
        TG_CUDA(cudaStreamSynchronize(st));
        memcpy(out, s->stage_out.host(), n * H * F);
    }
    return TG_OK;
}

extern "C" int tg_server_request(const tg_server *s, uint32_t slot, uint32_t *held, uint32_t *position,
                                 uint32_t *left) {
    if (!s) return fail(TG_EINVAL, "null server");
    if (slot >= s->req.size()) return fail(TG_ESHAPE, "slot %u of %zu", slot, s->req.size());
    const Request &r = s->req[slot];
    if (held) *held = r.held ? 1 : 0;
    if (position) *position = r.position;
    if (left) *left = r.left;
    return TG_OK;
}

extern "C" int tg_server_finish(tg_server *s, uint32_t slot) {
    if (!s) return fail(TG_EINVAL, "null server");
    if (slot >= s->req.size() || !s->req[slot].held) return fail(TG_EINVAL, "no request in slot %u", slot);
    s->req[slot] = Request();
    return TG_OK;
}

extern "C" int tg_server_last_output(tg_server *s, uint32_t slot, float *out) {
    if (!s || !out) return fail(TG_EINVAL, "tg_server_last_output: null argument");
    if (slot >= s->req.size() || !s->req[slot].held) return fail(TG_EINVAL, "no request in slot %u", slot);
    tg_decoder *d = s->d;
    TG_CUDA(cudaSetDevice(d->ctx->device));
    TG_TRY(d->wait_pending());
    const uint64_t bytes = (uint64_t)d->shape.hidden * 4;
    TG_CUDA(cudaMemcpyAsync(s->stage_out.ptr(), s->next.ptr() + slot * bytes, bytes, cudaMemcpyDefault, d->ctx->stream));
    TG_CUDA(cudaStreamSynchronize(d->ctx->stream));
    memcpy(out, s->stage_out.host(), bytes);
    return TG_OK;
}

extern "C" int tg_server_sync(tg_server *s, uint64_t timeout_ns) {
    if (!s) return fail(TG_EINVAL, "null server");
    TG_CUDA(cudaSetDevice(s->d->ctx->device));
    for (Bucket &b : s->d->buckets)
        if (b.prog.pending) TG_TRY(program_wait(b.prog, timeout_ns));
    TG_CUDA(cudaStreamSynchronize(s->d->ctx->stream));
    return take_kernel_error(s->d->ctx);
}
