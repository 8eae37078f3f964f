// The runtime behind the C ABI: contexts, buffers by residence, the kernel table with its
// dispatch checks, and programs - chains of dispatches captured once into a CUDA graph and
// launched as often as needed - with waits that give up at a deadline instead of hanging.
// It stands where crates/vulkan stands under crates/graph (context.rs, memory.rs, recording.rs).
#include <time.h>

#include <chrono>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <thread>

#include "tg_common.cuh"
#include "tg_internal.h"

namespace tg {

static thread_local std::string g_error;

int fail(int status, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    const int status = e == cudaErrorMemoryAllocation ? TG_ENOMEM : TG_ECUDA;
    return fail(status, "%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void clear_error() { g_error.clear(); }

int wait_event(cudaEvent_t ev, uint64_t timeout_ns) {
    const auto t0 = std::chrono::steady_clock::now();
    // Spin through a step's whole time (a batch-1 decode step takes ~0.7 ms: a sleep, which the
    // OS rounds up to tens of microseconds, would land after the step ends), then poll with short
    // sleeps (crates/vulkan/src/context.rs:119-136 spins, then blocks up to its limit).
    for (uint64_t i = 0;; i++) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return TG_OK;
        if (e != cudaErrorNotReady) return cuda_fail(e, "cudaEventQuery");
        const uint64_t waited = (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                    std::chrono::steady_clock::now() - t0)
                                    .count();
        if (timeout_ns && waited > timeout_ns)
            return fail(TG_ETIMEOUT, "the GPU did not finish within %.3f ms", timeout_ns / 1e6);
        if (waited > 2000000) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int take_kernel_error(tg_ctx *ctx) {
    const uint32_t word = __atomic_exchange_n(ctx->err_host, 0u, __ATOMIC_SEQ_CST);
    if (word == ERR_NONE) return TG_OK;
    return fail(TG_EKERNEL, "a kernel reported error word %u (%s)", word,
                word == ERR_WAIT_TIMEOUT ? "a bounded wait gave up" : "a placement out of range");
}

// ---- the kernel table's checks -----------------------------------------------------------------

static uint64_t esize(uint32_t dtype) { return dtype == TG_F32 ? 4 : 2; }

static bool is_local(uint32_t k) { return k >= TG_KERNEL_LOCAL_NORM && k <= TG_KERNEL_DIT_EULER; }

struct Need {
    const char *name;
    uint64_t bytes;
};

// What each binding of a dispatch must hold, in order (the kernels index by their params and do
// not check bounds, as Kernels::check requires, crates/graph/src/kernels.rs:232-263).
static int needs(const Launch &l, std::vector<Need> &out) {
    const tg_params &p = l.p;
    const uint64_t T = esize(p.dtype), F = 4;
    const uint64_t rows = p.rows, H = p.hidden, I = p.inner, hd = p.head_dim;
    const uint64_t heads = p.heads, kvh = p.kv_heads, cap = p.capacity, slots = p.slots;
    const uint64_t width = (heads + 2 * kvh) * hd, attn = heads * hd;
    const uint64_t words = (slots > 1 ? 2 : 1) * rows * 4;
    const uint64_t cache = slots * kvh * cap * hd * T;
    const uint64_t chunks = attn_chunks((uint32_t)cap);
    const uint64_t table = cap * (hd / 2) * F;
    switch (l.kernel) {
        case TG_KERNEL_RMSNORM:
            out = {{"x", rows * H * F}, {"gain", H * F}, {"out", rows * H * F}};
            break;
        case TG_KERNEL_GEMV_QKV_ROPE:
            out = {{"x", rows * H * F}, {"gain", H * F}, {"W", width * H * T}, {"cos", table},
                   {"sin", table}, {"at", words}, {"q", rows * attn * F}, {"k_cache", cache},
                   {"v_cache", cache}};
            break;
        case TG_KERNEL_ATTENTION_SPLIT:
            out = {{"q", rows * attn * F}, {"k_cache", cache}, {"v_cache", cache}, {"at", words},
                   {"partial_o", rows * heads * chunks * hd * F},
                   {"partial_ml", rows * heads * chunks * 2 * F}};
            break;
        case TG_KERNEL_ATTENTION_COMBINE:
            out = {{"at", words}, {"partial_o", rows * heads * chunks * hd * F},
                   {"partial_ml", rows * heads * chunks * 2 * F}, {"out", rows * attn * F}};
            break;
        case TG_KERNEL_GEMV_RESIDUAL:
            out = {{"x", rows * p.k * F}, {"W", (uint64_t)p.n * p.k * T}, {"residual", rows * p.n * F},
                   {"out", rows * p.n * F}};
            break;
        case TG_KERNEL_GEMV_GATE_UP:
            out = {{"x", rows * H * F}, {"gain", H * F}, {"W", 2 * I * H * T}, {"out", rows * I * F}};
            break;
        case TG_KERNEL_STREAM_READ:
            out = {{"data", (uint64_t)p.k * 4}, {"out", (uint64_t)p.n * 4}};
            break;
        case TG_KERNEL_NORM_ROWS:
            out = {{"at", words}, {"x", rows * H * F}, {"gain", H * F}, {"out", rows * H * (p.normed_f32 ? F : T)}};
            break;
        case TG_KERNEL_ADD_NORM_ROWS:
            out = {{"at", words}, {"c", (p.parts > 1 ? p.parts : 1) * rows * H * F}, {"residual", rows * H * F}, {"gain", H * F},
                   {"sum", rows * H * F}, {"normed", rows * H * (p.normed_f32 ? F : T)}};
            break;
        case TG_KERNEL_ROPE_ROWS:
            out = {{"at", words}, {"c", rows * width * F}, {"cos", table}, {"sin", table},
                   {"q", rows * attn * T}, {"k_cache", cache}, {"v_cache", cache}};
            break;
        case TG_KERNEL_ATTENTION_ROWS:
        case TG_KERNEL_ATTENTION_ROWS_TC:
            out = {{"at", words}, {"q", rows * attn * T}, {"k_cache", cache}, {"v_cache", cache},
                   {"out", rows * attn * T}};
            break;
        case TG_KERNEL_SILU_MUL_ROWS:
            out = {{"at", words}, {"c", rows * 2 * I * F}, {"out", rows * I * T}};
            break;
        case TG_KERNEL_GEMM:
            out = {{"a", (uint64_t)p.m * p.k * T}, {"b", (uint64_t)p.n * p.k * T},
                   {"c", (uint64_t)(p.parts > 1 ? p.parts : 1) * p.m * p.n * F}};
            break;
        case TG_KERNEL_GEMM_SILU:
            out = {{"a", (uint64_t)p.m * p.k * T}, {"b", (uint64_t)p.n * p.k * T},
                   {"out", (uint64_t)p.m * (p.n / 2) * T}};
            break;
        case TG_KERNEL_GEMM_QKV_ROPE:
            out = {{"a", (uint64_t)p.m * p.k * T}, {"b", (uint64_t)p.n * p.k * T}, {"at", words}, {"cos", table},
                   {"sin", table}, {"q", rows * attn * T}, {"k_cache", cache}, {"v_cache", cache}};
            break;
        case TG_KERNEL_GEMV_LINEAR:
            out = {{"x0", rows * p.k * F}, {"x1", std::max<uint64_t>(rows * p.k1 * F, 16)},
                   {"W", (uint64_t)p.n * (p.k + p.k1) * T}, {"bias", (uint64_t)p.n * F},
                   {"out", rows * p.stride * F}};
            break;
        // The local stacks: f16 (2 bytes) throughout but for the partial sums, tables and patches.
        case TG_KERNEL_LOCAL_NORM:
            out = {{"x", (uint64_t)p.m * H * 2}, {"gain", H * 2}, {"out", (uint64_t)p.m * H * 2}};
            break;
        case TG_KERNEL_LOCAL_PARTIAL:
            out = {{"x", (uint64_t)p.m * p.k * 2}, {"W", (uint64_t)p.n * p.k * 2},
                   {"partial", (uint64_t)p.parts * p.m * p.n * F}};
            break;
        case TG_KERNEL_LOCAL_GATE_UP:
            out = {{"x", (uint64_t)p.m * p.k * 2}, {"W", (uint64_t)p.n * p.k * 2}, {"out", (uint64_t)p.m * (p.n / 2) * 2}};
            break;
        case TG_KERNEL_LOCAL_ATTENTION:
            out = {{"partial", (uint64_t)p.parts * p.m * width * F}, {"cos", table}, {"sin", table},
                   {"out", (uint64_t)p.m * attn * 2}};
            break;
        case TG_KERNEL_LOCAL_ADD_NORM:
            out = {{"partial", (uint64_t)p.parts * p.m * p.n * F}, {"residual", (uint64_t)p.m * p.n * 2},
                   {"gain", (uint64_t)p.n * 2}, {"sum", (uint64_t)p.m * p.n * 2}, {"normed", (uint64_t)p.m * p.n * 2}};
            break;
        case TG_KERNEL_LOCAL_ROWS:
            out = {{"x", rows * cap * p.n * 2}, {"out", rows * p.n * 2}};
            break;
        case TG_KERNEL_LOCAL_EMBED:
            out = {{"src", rows * p.feat * p.frames * F}, {"W", (uint64_t)p.n * p.feat * 2}, {"bias", (uint64_t)p.n * 2},
                   {"tokens", std::max<uint64_t>((p.flags & 2 ? 1 : rows) * p.copied * p.n * 2, 16)},
                   {"h", rows * p.seqs * cap * p.n * 2}};
            break;
        case TG_KERNEL_CFM_NOISE:
            out = {{"noise", rows * p.feat * p.frames * F}, {"sampling", rows * 2 * F}, {"x", rows * p.feat * p.frames * F}};
            break;
        case TG_KERNEL_DIT_EULER:
            out = {{"h", rows * 2 * cap * p.k * 2}, {"W", (uint64_t)p.feat * p.k * 2}, {"bias", (uint64_t)p.feat * 2},
                   {"sampling", rows * 2 * F}, {"x", rows * p.feat * p.frames * F}};
            break;
        default:
            return fail(TG_EINVAL, "no kernel %u", l.kernel);
    }
    return TG_OK;
}

static const char *kernel_name(uint32_t k) {
    static const char *names[TG_KERNEL_COUNT] = {
        "rmsnorm", "gemv_qkv_rope", "attention_split", "attention_combine", "gemv_residual",
        "gemv_gate_up", "stream_read", "norm_rows", "add_norm_rows", "rope_rows", "attention_rows",
        "silu_mul_rows", "gemm", "(unused)", "gemm_silu", "attention_rows_tc", "gemm_qkv_rope", "gemv_linear",
        "local_norm", "local_partial", "local_gate_up", "local_attention", "local_add_norm", "local_rows",
        "local_embed", "cfm_noise", "dit_euler"};
    return k < TG_KERNEL_COUNT ? names[k] : "?";
}

// The local stacks' kernels' shape rules (local/mod.rs:366-385, dit.rs:196-212, encoder.rs:70-72).
static int check_local_shape(const Launch &l) {
    const tg_params &p = l.p;
    const char *name = kernel_name(l.kernel);
    if (p.dtype != TG_F16) return fail(TG_ESHAPE, "%s: dtype %u (the local stacks are f16)", name, p.dtype);
    bool ok = true;
    switch (l.kernel) {
        case TG_KERNEL_LOCAL_NORM:
            ok = p.m > 0 && p.hidden > 0 && p.hidden % 2 == 0 && p.hidden <= 2048;
            break;
        case TG_KERNEL_LOCAL_PARTIAL:
            ok = p.parts > 0 && p.k % p.parts == 0 && local_proj_supported((int)p.m, (int)p.n, (int)p.k, (int)p.parts);
            break;
        case TG_KERNEL_LOCAL_GATE_UP:
            ok = local_proj_supported((int)p.m, (int)p.n, (int)p.k, 1);
            break;
        case TG_KERNEL_LOCAL_ATTENTION:
            ok = p.parts > 0 && p.capacity > 0 && p.capacity <= 32 && p.m > 0 && p.m % p.capacity == 0 &&
                 p.kv_heads > 0 && p.heads % p.kv_heads == 0 && p.head_dim > 0 && p.head_dim % 8 == 0 &&
                 p.head_dim <= 256;
            break;
        case TG_KERNEL_LOCAL_ADD_NORM:
            ok = p.parts > 0 && p.m > 0 && p.n > 0 && p.n % 2 == 0 && p.n <= 2048;
            break;
        case TG_KERNEL_LOCAL_ROWS:
            ok = p.rows > 0 && p.capacity > 0 && p.n > 0 && p.n % 8 == 0;
            break;
        case TG_KERNEL_LOCAL_EMBED:
            ok = p.rows > 0 && p.seqs > 0 && p.n > 0 && p.feat > 0 && p.feat % 8 == 0 && p.frames > 0 && p.frames <= 8 &&
                 p.first + p.frames <= p.capacity &&
                 p.at + p.copied <= p.capacity && (uint64_t)p.feat * p.frames * 4 <= 200 * 1024;
            break;
        case TG_KERNEL_CFM_NOISE:
            ok = p.rows > 0 && p.feat > 0 && p.frames > 0;
            break;
        case TG_KERNEL_DIT_EULER:
            ok = p.rows > 0 && p.k > 0 && p.k % 8 == 0 && p.feat > 0 && p.frames > 0 && 2 * p.frames <= 16 &&
                 p.first + p.frames <= p.capacity && 4 * (2ull * p.frames * p.k + 2ull * p.feat * p.frames) <= 200 * 1024;
            break;
    }
    if (!ok)
        return fail(TG_ESHAPE, "%s: shape not taken (m %u, n %u, k %u, parts %u, capacity %u, heads %u/%u of %u, rows %u)",
                    name, p.m, p.n, p.k, p.parts, p.capacity, p.heads, p.kv_heads, p.head_dim, p.rows);
    return TG_OK;
}

// Shapes the kernels cannot cover exactly are refused (decode.rs:468-491, prefill.rs:233-262).
static int check_shape(const Launch &l) {
    const tg_params &p = l.p;
    if (is_local(l.kernel)) return check_local_shape(l);
    if (p.dtype != TG_F32 && p.dtype != TG_BF16) return fail(TG_ESHAPE, "dtype %u", p.dtype);
    const uint32_t vec = p.dtype == TG_BF16 ? 256 : 128;  // a warp's 16-byte step over K
    auto heads_ok = [&] {
        return p.kv_heads > 0 && p.heads % p.kv_heads == 0 && p.heads / p.kv_heads <= MAX_GROUP &&
               (p.head_dim == 64 || p.head_dim == 128) && p.capacity > 0 && p.capacity % CAPACITY_STEP == 0;
    };
    switch (l.kernel) {
        case TG_KERNEL_RMSNORM:
        case TG_KERNEL_NORM_ROWS:
            if (p.hidden == 0 || p.hidden % 128) return fail(TG_ESHAPE, "%s: hidden %u is not a multiple of 128", kernel_name(l.kernel), p.hidden);
            break;
        case TG_KERNEL_ADD_NORM_ROWS:
            if (p.hidden == 0 || p.hidden % 128 || p.hidden > 4096 || p.parts > (uint32_t)ADD_NORM_MAX_PARTS)
                return fail(TG_ESHAPE, "add_norm_rows: hidden %u (a multiple of 128, at most 4096), %u parts (at most %u)",
                            p.hidden, p.parts, ADD_NORM_MAX_PARTS);
            break;
        case TG_KERNEL_GEMV_QKV_ROPE:
            if (p.hidden % vec || !heads_ok()) return fail(TG_ESHAPE, "gemv_qkv_rope: hidden %u (multiple of %u), %u heads over %u of %u, capacity %u", p.hidden, vec, p.heads, p.kv_heads, p.head_dim, p.capacity);
            if (p.hidden % 128) return fail(TG_ESHAPE, "gemv_qkv_rope: hidden %u", p.hidden);
            break;
        case TG_KERNEL_GEMV_GATE_UP:
            if (p.hidden == 0 || p.hidden % vec || p.inner == 0) return fail(TG_ESHAPE, "gemv_gate_up: hidden %u is not a multiple of %u", p.hidden, vec);
            break;
        case TG_KERNEL_GEMV_RESIDUAL:
            if (p.k == 0 || p.k % vec || p.n == 0) return fail(TG_ESHAPE, "gemv_residual: %u columns are not a multiple of %u", p.k, vec);
            break;
        case TG_KERNEL_ATTENTION_SPLIT:
        case TG_KERNEL_ATTENTION_COMBINE:
        case TG_KERNEL_ROPE_ROWS:
        case TG_KERNEL_ATTENTION_ROWS:
            if (!heads_ok()) return fail(TG_ESHAPE, "%s: %u heads over %u of %u, capacity %u (multiple of %u)", kernel_name(l.kernel), p.heads, p.kv_heads, p.head_dim, p.capacity, CAPACITY_STEP);
            break;
        case TG_KERNEL_SILU_MUL_ROWS:
            if (p.inner == 0) return fail(TG_ESHAPE, "silu_mul_rows: inner 0");
            break;
        case TG_KERNEL_GEMV_LINEAR: {
            const uint32_t vec = p.dtype == TG_BF16 ? 8 : 4;  // a 16-byte load of each input's columns
            if (p.n == 0 || p.k == 0 || p.k % vec || p.k1 % vec || p.act > 2 || p.offset + p.n > p.stride ||
                (p.act == 2 && !(p.levels > 0.0f)) || p.rows > 64)
                return fail(TG_ESHAPE, "gemv_linear: %u outputs of %u + %u (multiples of %u) at %u of rows %u long, "
                            "act %u, levels %g, %u rows (at most 64)", p.n, p.k, p.k1, vec, p.offset, p.stride, p.act,
                            p.levels, p.rows);
            break;
        }
        case TG_KERNEL_GEMM_QKV_ROPE:
            if (p.dtype != TG_BF16 || !heads_ok() || p.m == 0 || p.m != p.rows || p.k % 64 || p.n % 256 ||
                p.n != (p.heads + 2 * p.kv_heads) * p.head_dim)
                return fail(TG_ESHAPE, "gemm_qkv_rope %ux%ux%u: bf16, rows = m, n = (heads + 2 kv) hd a multiple of 256",
                            p.m, p.n, p.k);
            break;
        case TG_KERNEL_ATTENTION_ROWS_TC:
            if (!heads_ok() || !attention_tc_supported(p))
                return fail(TG_ESHAPE, "attention_rows_tc: bf16, head_dim 64 and rows a multiple of 128 (%u rows, hd %u)",
                            p.rows, p.head_dim);
            break;
        case TG_KERNEL_STREAM_READ:
            if (p.k % 4 || p.n < 1) return fail(TG_ESHAPE, "stream_read: %u words", p.k);
            break;
        case TG_KERNEL_GEMM_SILU:
            if (p.dtype != TG_BF16 || p.m == 0 || p.k % 64 || p.n == 0 || p.n % 256)
                return fail(TG_ESHAPE, "gemm_silu %ux%ux%u: bf16 with n a multiple of 256 and k of 64", p.m, p.n, p.k);
            break;
        case TG_KERNEL_GEMM:
            if (p.m == 0 || p.n == 0 || p.k == 0) return fail(TG_ESHAPE, "gemm %ux%ux%u", p.m, p.n, p.k);
            if (p.dtype == TG_BF16 && (p.k % 64 || p.n % 64))
                return fail(TG_ESHAPE, "gemm %ux%ux%u: bf16 needs n and k multiples of 64", p.m, p.n, p.k);
            if (p.parts > 1 && (p.dtype != TG_BF16 || p.k % (64 * p.parts)))
                return fail(TG_ESHAPE, "gemm %ux%ux%u in %u parts: bf16 with k a multiple of 64 parts", p.m, p.n, p.k, p.parts);
            break;
        default:
            return fail(TG_EINVAL, "no kernel %u", l.kernel);
    }
    if (l.kernel != TG_KERNEL_STREAM_READ && l.kernel != TG_KERNEL_GEMM && l.kernel != TG_KERNEL_GEMM_SILU &&
        l.kernel != TG_KERNEL_GEMV_RESIDUAL && p.rows == 0)
        return fail(TG_ESHAPE, "%s: 0 rows", kernel_name(l.kernel));
    if (p.rows > 0 && p.slots == 0) return fail(TG_ESHAPE, "%s: 0 slots", kernel_name(l.kernel));
    return TG_OK;
}

// The table kernel whose bindings and shape rules a library-recorded launch shares.
static uint32_t table_kernel(uint32_t k) {
    switch (k) {
        case KERNEL_DTC_QKV_ROPE: return TG_KERNEL_GEMV_QKV_ROPE;
        case KERNEL_DTC_GATE_UP: return TG_KERNEL_GEMV_GATE_UP;
        case KERNEL_DTC_RESIDUAL: return TG_KERNEL_GEMV_RESIDUAL;
        case KERNEL_ATTN_SPLIT_MMA:
        case KERNEL_ATTN_SPLIT_MMA_BQ:
        case KERNEL_ATTN_SPLIT_JOIN: return TG_KERNEL_ATTENTION_SPLIT;
        case KERNEL_GEMM_RESIDUAL: return TG_KERNEL_GEMM;
        case KERNEL_ATTN_COMBINE_WIDE:
        case KERNEL_ATTN_COMBINE_WIDE_BF: return TG_KERNEL_ATTENTION_COMBINE;
        default: return k;
    }
}

int check_launch(const Launch &l0) {
    if (l0.kernel == KERNEL_DECODE_STEP) return TG_OK;  // recorded by the decoder over its own buffers
    Launch l = l0;
    l.kernel = table_kernel(l0.kernel);
    const bool wide = l0.kernel == KERNEL_ATTN_SPLIT_MMA || l0.kernel == KERNEL_ATTN_COMBINE_WIDE ||
                      l0.kernel == KERNEL_ATTN_SPLIT_MMA_BQ || l0.kernel == KERNEL_ATTN_COMBINE_WIDE_BF ||
                      l0.kernel == KERNEL_ATTN_SPLIT_JOIN;
    if (wide ? !attention_split_mma_supported(l.p) : (l.kernel != l0.kernel && l0.kernel != KERNEL_GEMM_RESIDUAL && !dtc_supported(l.p)))
        return fail(TG_ESHAPE, "%s: no tcgen05 plan for %u rows of this shape", l0.label.c_str(), l.p.rows);
    int st = check_shape(l);
    if (st) return st;
    std::vector<Need> need;
    if ((st = needs(l, need))) return st;
    if (l0.kernel == KERNEL_GEMM_RESIDUAL) need.push_back({"residual", (uint64_t)l.p.m * l.p.n * 4});
    if (l0.kernel == KERNEL_ATTN_SPLIT_JOIN) {
        need.push_back({"out", (uint64_t)l.p.rows * l.p.heads * l.p.head_dim * 2});
        need.push_back({"counts", (uint64_t)l.p.rows * l.p.kv_heads * 4});
    }
    if (l.ptr.size() != need.size() || l.bytes.size() != need.size())
        return fail(TG_EINVAL, "%s: %zu bindings, takes %zu", kernel_name(l.kernel), l.ptr.size(), need.size());
    for (size_t i = 0; i < need.size(); i++) {
        if (!l.ptr[i]) return fail(TG_EINVAL, "%s: binding %zu (%s) is null", kernel_name(l.kernel), i, need[i].name);
        if (reinterpret_cast<uintptr_t>(l.ptr[i]) % 16)
            return fail(TG_EINVAL, "%s: binding %zu (%s) is not 16-byte aligned", kernel_name(l.kernel), i, need[i].name);
        if (l.bytes[i] < need[i].bytes)
            return fail(TG_ESHAPE, "%s: binding %zu (%s) holds %llu bytes, the dispatch reaches %llu",
                        kernel_name(l.kernel), i, need[i].name, (unsigned long long)l.bytes[i],
                        (unsigned long long)need[i].bytes);
    }
    return TG_OK;
}

int enqueue_launch(const Launch &l, uint32_t *err, cudaStream_t s, int sm_count) {
    const tg_params &p = l.p;
    void *const *b = l.ptr.data();
    auto F = [&](int i) { return static_cast<float *>(b[i]); };
    auto U = [&](int i) { return static_cast<uint32_t *>(b[i]); };
    cudaError_t e = cudaSuccess;
    switch (l.kernel) {
        case TG_KERNEL_RMSNORM: e = launch_rmsnorm(p, F(0), F(1), F(2), s); break;
        case TG_KERNEL_GEMV_QKV_ROPE: e = launch_gemv_qkv_rope(p, F(0), F(1), b[2], F(3), F(4), U(5), b[6], b[7], b[8], err, s); break;
        case TG_KERNEL_ATTENTION_SPLIT: e = launch_attention_split(p, b[0], b[1], b[2], U(3), F(4), F(5), s); break;
        case TG_KERNEL_ATTENTION_COMBINE: e = launch_attention_combine(p, U(0), F(1), F(2), b[3], s); break;
        case TG_KERNEL_GEMV_RESIDUAL: e = launch_gemv_residual(p, b[0], b[1], F(2), F(3), err, s); break;
        case TG_KERNEL_GEMV_GATE_UP: e = launch_gemv_gate_up(p, F(0), F(1), b[2], b[3], err, s); break;
        case TG_KERNEL_STREAM_READ: e = launch_stream_read(p, U(0), U(1), s, sm_count); break;
        case TG_KERNEL_NORM_ROWS: e = launch_norm_rows(p, U(0), F(1), F(2), b[3], s); break;
        case TG_KERNEL_ADD_NORM_ROWS: e = launch_add_norm_rows(p, U(0), F(1), F(2), F(3), F(4), b[5], s); break;
        case TG_KERNEL_ROPE_ROWS: e = launch_rope_rows(p, U(0), F(1), F(2), F(3), b[4], b[5], b[6], s); break;
        case TG_KERNEL_ATTENTION_ROWS: e = launch_attention_rows(p, U(0), b[1], b[2], b[3], b[4], s); break;
        case TG_KERNEL_SILU_MUL_ROWS: e = launch_silu_mul_rows(p, U(0), F(1), b[2], s); break;
        case TG_KERNEL_GEMM: e = launch_gemm(p, b[0], b[1], F(2), err, s); break;
        case TG_KERNEL_GEMM_SILU: e = launch_gemm_silu(p, b[0], b[1], b[2], err, s); break;
        case KERNEL_DECODE_STEP: e = launch_decode_step(l.step, sm_count, s); break;
        case KERNEL_DTC_QKV_ROPE: e = launch_dtc_qkv_rope(p, F(0), F(1), b[2], F(3), F(4), U(5), F(6), b[7], b[8], err, s); break;
        case KERNEL_DTC_GATE_UP: e = launch_dtc_gate_up(p, F(0), F(1), b[2], F(3), err, s); break;
        case KERNEL_DTC_RESIDUAL: e = launch_dtc_residual(p, F(0), b[1], F(2), F(3), err, s); break;
        case KERNEL_ATTN_SPLIT_MMA: e = launch_attention_split_mma(p, b[0], b[1], b[2], U(3), F(4), F(5), s); break;
        case KERNEL_ATTN_SPLIT_MMA_BQ: e = launch_attention_split_mma(p, b[0], b[1], b[2], U(3), F(4), F(5), s, true); break;
        case KERNEL_GEMM_RESIDUAL: e = launch_gemm_residual(p, b[0], b[1], F(3), F(2), err, s); break;
        case KERNEL_ATTN_SPLIT_JOIN:
            e = launch_attention_split_join(p, b[0], b[1], b[2], U(3), F(4), F(5), b[6], U(7), s);
            break;
        case KERNEL_ATTN_COMBINE_WIDE_BF:
            e = launch_attention_combine_chunk(p, DECODE_WIDE_CHUNK, U(0), F(1), F(2), b[3], s, true);
            break;
        case KERNEL_ATTN_COMBINE_WIDE:
            e = launch_attention_combine_chunk(p, DECODE_WIDE_CHUNK, U(0), F(1), F(2), b[3], s);
            break;
        case TG_KERNEL_ATTENTION_ROWS_TC: e = launch_attention_rows_tc(p, U(0), b[1], b[2], b[3], b[4], err, s); break;
        case TG_KERNEL_GEMV_LINEAR: e = launch_gemv_linear(p, F(0), F(1), b[2], F(3), F(4), s); break;
        case TG_KERNEL_GEMM_QKV_ROPE:
            e = launch_gemm_qkv_rope(p, b[0], b[1], U(2), F(3), F(4), b[5], b[6], b[7], err, s);
            break;
        case TG_KERNEL_LOCAL_NORM: e = launch_local_norm(p, b[0], b[1], b[2], s); break;
        case TG_KERNEL_LOCAL_PARTIAL: e = launch_local_partial(p, b[0], b[1], F(2), err, s); break;
        case TG_KERNEL_LOCAL_GATE_UP: e = launch_local_gate_up(p, b[0], b[1], b[2], err, s); break;
        case TG_KERNEL_LOCAL_ATTENTION: e = launch_local_attention(p, F(0), F(1), F(2), b[3], s); break;
        case TG_KERNEL_LOCAL_ADD_NORM: e = launch_local_add_norm(p, F(0), b[1], b[2], b[3], b[4], s); break;
        case TG_KERNEL_LOCAL_ROWS: e = launch_local_rows(p, b[0], b[1], s); break;
        case TG_KERNEL_LOCAL_EMBED: e = launch_local_embed(p, F(0), b[1], b[2], b[3], b[4], s); break;
        case TG_KERNEL_CFM_NOISE: e = launch_cfm_noise(p, F(0), F(1), F(2), s); break;
        case TG_KERNEL_DIT_EULER: e = launch_dit_euler(p, b[0], b[1], b[2], F(3), F(4), s); break;
        default: return fail(TG_EINVAL, "no kernel %u", l.kernel);
    }
    if (e != cudaSuccess)
        return fail(e == cudaErrorNotSupported ? TG_ESHAPE : TG_ECUDA, "launching %s (%s): %s",
                    l.kernel == KERNEL_DECODE_STEP ? "decode_step" : kernel_name(table_kernel(l.kernel)), l.label.c_str(),
                    cudaGetErrorString(e));
    return TG_OK;
}

// ---- programs ------------------------------------------------------------------------------------

void program_release(Program &p) {
    if (p.exec) cudaGraphExecDestroy(p.exec);
    if (p.graph) cudaGraphDestroy(p.graph);
    for (cudaEvent_t e : p.events) cudaEventDestroy(e);
    p.exec = nullptr;
    p.graph = nullptr;
    p.events.clear();
}

int program_build(tg_ctx *ctx, const std::vector<Launch> &launches, bool timed, Program &out) {
    for (const Launch &l : launches) {
        const int st = check_launch(l);
        if (st) return st;
    }
    out.ctx = ctx;
    out.timed = timed;
    out.labels.clear();
    for (const Launch &l : launches) out.labels.push_back(l.label.empty() ? kernel_name(table_kernel(l.kernel)) : l.label);
    const size_t nev = timed ? launches.size() + 1 : 2;
    for (size_t i = 0; i < nev; i++) {
        cudaEvent_t e;
        TG_CUDA(cudaEventCreate(&e));
        out.events.push_back(e);
    }
    cudaStream_t cap;
    TG_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) {
        cudaStreamDestroy(cap);
        return cuda_fail(e, "cudaStreamBeginCapture");
    }
    int st = TG_OK;
    // External event nodes, so that the host can query and time them after each launch.
    auto record = [&](cudaEvent_t ev) {
        const cudaError_t r = cudaEventRecordWithFlags(ev, cap, cudaEventRecordExternal);
        if (r != cudaSuccess && st == TG_OK) st = cuda_fail(r, "cudaEventRecordWithFlags");
    };
    record(out.events[0]);
    for (size_t i = 0; i < launches.size() && st == TG_OK; i++) {
        st = enqueue_launch(launches[i], ctx->err_dev, cap, ctx->sm_count);
        if (timed) record(out.events[i + 1]);
    }
    if (!timed) record(out.events[1]);
    cudaGraph_t graph = nullptr;
    e = cudaStreamEndCapture(cap, &graph);
    cudaStreamDestroy(cap);
    if (st != TG_OK) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    out.graph = graph;
    TG_CUDA(cudaGraphInstantiate(&out.exec, graph, 0));
    return TG_OK;
}

int program_start(Program &p) {
    if (p.pending) {
        // A run a wait gave up on is waited for before the next (recording.rs:631-642).
        const int st = program_wait(p, 0);
        if (st) return st;
    }
    TG_CUDA(cudaGraphLaunch(p.exec, p.ctx->stream));
    p.pending = true;
    return TG_OK;
}

int program_launch(Program &p) {
    TG_CUDA(cudaGraphLaunch(p.exec, p.ctx->stream));
    p.pending = true;
    return TG_OK;
}

int program_wait(Program &p, uint64_t timeout_ns) {
    if (!p.pending) return TG_OK;
    const int st = wait_event(p.events.back(), timeout_ns);
    if (st == TG_ETIMEOUT) return st;
    p.pending = false;
    if (st) return st;
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "a program's kernels");
    return take_kernel_error(p.ctx);
}

double program_elapsed_ns(Program &p) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, p.events.front(), p.events.back()) != cudaSuccess) return -1.0;
    return ms * 1e6;
}

int program_timings(Program &p, double *ns, size_t n) {
    if (!p.timed) return fail(TG_EINVAL, "the program was not recorded timed");
    for (size_t i = 0; i + 1 < p.events.size() && i < n; i++) {
        float ms = 0.0f;
        TG_CUDA(cudaEventElapsedTime(&ms, p.events[i], p.events[i + 1]));
        ns[i] = ms * 1e6;
    }
    return TG_OK;
}

}  // namespace tg

using namespace tg;

// ---- C ABI: errors, context, memory ---------------------------------------------------------------

extern "C" const char *tg_last_error(void) { return g_error.c_str(); }
extern "C" uint32_t tg_abi_version(void) { return TGCUDA_ABI_VERSION; }

extern "C" int tg_ctx_create(int device, tg_ctx **out) {
    if (!out) return fail(TG_EINVAL, "tg_ctx_create: out is null");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return fail(TG_ENODEVICE, "no CUDA device: %s", e == cudaSuccess ? "none found" : cudaGetErrorString(e));
    if (device < 0 || device >= count) return fail(TG_ENODEVICE, "device %d of %d", device, count);
    cudaDeviceProp prop;
    TG_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(TG_ENODEVICE, "device %d (%s) is sm_%d%d; these kernels are built for sm_100a", device, prop.name, prop.major, prop.minor);
    TG_CUDA(cudaSetDevice(device));
    tg_ctx *ctx = new tg_ctx();
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->cc_major = prop.major;
    ctx->cc_minor = prop.minor;
    snprintf(ctx->name, sizeof ctx->name, "%s", prop.name);
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void **>(&ctx->err_host), 64, cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&ctx->err_dev), ctx->err_host, 0);
    if (e != cudaSuccess) {
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        if (ctx->err_host) cudaFreeHost(ctx->err_host);
        delete ctx;
        return cuda_fail(e, "tg_ctx_create");
    }
    *ctx->err_host = 0;
    *out = ctx;
    return TG_OK;
}

extern "C" int tg_ctx_destroy(tg_ctx *ctx) {
    if (!ctx) return TG_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
    cudaFreeHost(ctx->err_host);
    delete ctx;
    return TG_OK;
}

extern "C" int tg_ctx_synchronize(tg_ctx *ctx, uint64_t timeout_ns) {
    if (!ctx) return fail(TG_EINVAL, "null context");
    cudaEvent_t ev;
    TG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    cudaEventRecord(ev, ctx->stream);
    const int st = wait_event(ev, timeout_ns);
    cudaEventDestroy(ev);
    if (st) return st;
    return take_kernel_error(ctx);
}

extern "C" int tg_ctx_info(tg_ctx *ctx, char *name, size_t name_bytes, int *sm_count) {
    if (!ctx) return fail(TG_EINVAL, "null context");
    if (name && name_bytes) snprintf(name, name_bytes, "%s", ctx->name);
    if (sm_count) *sm_count = ctx->sm_count;
    return TG_OK;
}

extern "C" int tg_mem_alloc(tg_ctx *ctx, uint64_t bytes, tg_residence residence, tg_mem **out) {
    if (!ctx || !out) return fail(TG_EINVAL, "tg_mem_alloc: null argument");
    *out = nullptr;
    if (bytes == 0) return fail(TG_EINVAL, "tg_mem_alloc: 0 bytes");
    TG_CUDA(cudaSetDevice(ctx->device));
    tg_mem *m = new tg_mem();
    m->ctx = ctx;
    m->bytes = bytes;
    m->residence = residence;
    cudaError_t e;
    if (residence == TG_RES_DEVICE) {
        e = cudaMalloc(&m->ptr, bytes);
        // Zeroed on the context's stream, which every later copy and launch of the context uses:
        // the stream does not wait for the legacy default stream, so a cudaMemset there could
        // land after a write that follows it.
        if (e == cudaSuccess) e = cudaMemsetAsync(m->ptr, 0, bytes, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    } else if (residence == TG_RES_UPLOAD || residence == TG_RES_READBACK) {
        e = cudaHostAlloc(&m->host, bytes, cudaHostAllocMapped);
        if (e == cudaSuccess) e = cudaHostGetDevicePointer(&m->ptr, m->host, 0);
        if (e == cudaSuccess) memset(m->host, 0, bytes);
    } else {
        delete m;
        return fail(TG_EINVAL, "residence %d", (int)residence);
    }
    if (e != cudaSuccess) {
        // What the failing step left allocated goes back before the error is reported.
        if (residence == TG_RES_DEVICE && m->ptr) cudaFree(m->ptr);
        if (residence != TG_RES_DEVICE && m->host) cudaFreeHost(m->host);
        delete m;
        return cuda_fail(e, "tg_mem_alloc");
    }
    *out = m;
    return TG_OK;
}

extern "C" int tg_mem_free(tg_mem *m) {
    if (!m) return TG_OK;
    cudaSetDevice(m->ctx->device);
    if (m->residence == TG_RES_DEVICE)
        cudaFree(m->ptr);
    else
        cudaFreeHost(m->host);
    delete m;
    return TG_OK;
}

extern "C" uint64_t tg_mem_size(const tg_mem *m) { return m ? m->bytes : 0; }
extern "C" void *tg_mem_device_ptr(const tg_mem *m) { return m ? m->ptr : nullptr; }

static int mem_range(const tg_mem *m, uint64_t offset, uint64_t bytes, const char *what) {
    if (!m) return fail(TG_EINVAL, "%s: null buffer", what);
    if (offset > m->bytes || bytes > m->bytes - offset)
        return fail(TG_ESHAPE, "%s: %llu bytes at %llu of a buffer of %llu", what, (unsigned long long)bytes,
                    (unsigned long long)offset, (unsigned long long)m->bytes);
    return TG_OK;
}

extern "C" int tg_mem_write(tg_mem *m, uint64_t offset, const void *src, uint64_t bytes) {
    int st = mem_range(m, offset, bytes, "tg_mem_write");
    if (st) return st;
    if (!bytes) return TG_OK;
    if (!src) return fail(TG_EINVAL, "tg_mem_write: null source");
    if (m->residence != TG_RES_DEVICE) {
        memcpy(static_cast<char *>(m->host) + offset, src, bytes);
        return TG_OK;
    }
    TG_CUDA(cudaSetDevice(m->ctx->device));
    TG_CUDA(cudaMemcpyAsync(static_cast<char *>(m->ptr) + offset, src, bytes, cudaMemcpyHostToDevice, m->ctx->stream));
    TG_CUDA(cudaStreamSynchronize(m->ctx->stream));
    return TG_OK;
}

extern "C" int tg_mem_read(tg_mem *m, uint64_t offset, void *dst, uint64_t bytes) {
    int st = mem_range(m, offset, bytes, "tg_mem_read");
    if (st) return st;
    if (!bytes) return TG_OK;
    if (!dst) return fail(TG_EINVAL, "tg_mem_read: null destination");
    TG_CUDA(cudaSetDevice(m->ctx->device));
    if (m->residence != TG_RES_DEVICE) {
        TG_CUDA(cudaStreamSynchronize(m->ctx->stream));
        memcpy(dst, static_cast<const char *>(m->host) + offset, bytes);
        return TG_OK;
    }
    TG_CUDA(cudaMemcpyAsync(dst, static_cast<const char *>(m->ptr) + offset, bytes, cudaMemcpyDeviceToHost, m->ctx->stream));
    TG_CUDA(cudaStreamSynchronize(m->ctx->stream));
    return TG_OK;
}

extern "C" int tg_mem_fill(tg_mem *m, uint64_t offset, uint32_t word, uint64_t bytes) {
    int st = mem_range(m, offset, bytes, "tg_mem_fill");
    if (st) return st;
    if (bytes % 4 || offset % 4) return fail(TG_EINVAL, "tg_mem_fill: %llu bytes at %llu are not whole words", (unsigned long long)bytes, (unsigned long long)offset);
    std::vector<uint32_t> words(bytes / 4, word);
    return tg_mem_write(m, offset, words.data(), bytes);
}

extern "C" int tg_copy_regions(tg_ctx *ctx, tg_mem *src, tg_mem *dst, const tg_region *regions, size_t n) {
    if (!ctx || !src || !dst || (n && !regions)) return fail(TG_EINVAL, "tg_copy_regions: null argument");
    for (size_t i = 0; i < n; i++) {
        int st = mem_range(src, regions[i].src_offset, regions[i].bytes, "tg_copy_regions (source)");
        if (!st) st = mem_range(dst, regions[i].dst_offset, regions[i].bytes, "tg_copy_regions (destination)");
        if (st) return st;
    }
    TG_CUDA(cudaSetDevice(ctx->device));
    for (size_t i = 0; i < n; i++) {
        // One copy per region, in order.
        TG_CUDA(cudaMemcpyAsync(static_cast<char *>(dst->ptr) + regions[i].dst_offset,
                                static_cast<const char *>(src->ptr) + regions[i].src_offset, regions[i].bytes,
                                cudaMemcpyDefault, ctx->stream));
    }
    return tg_ctx_synchronize(ctx, 0);
}

// ---- C ABI: dispatches and programs ---------------------------------------------------------------

static int resolve(const tg_dispatch &d, Launch &l) {
    if (!d.params) return fail(TG_EINVAL, "dispatch of kernel %u without params", d.kernel);
    if (d.n_bindings && !d.bindings) return fail(TG_EINVAL, "dispatch of kernel %u: null bindings", d.kernel);
    l.kernel = d.kernel;
    l.p = *d.params;
    l.label = d.label ? d.label : "";
    for (uint32_t i = 0; i < d.n_bindings; i++) {
        const tg_binding &b = d.bindings[i];
        if (!b.mem) return fail(TG_EINVAL, "%s: binding %u has no buffer", kernel_name(d.kernel), i);
        int st = mem_range(b.mem, b.offset, b.bytes, "binding");
        if (st) return st;
        l.ptr.push_back(static_cast<char *>(b.mem->ptr) + b.offset);
        l.bytes.push_back(b.bytes);
    }
    return TG_OK;
}

struct tg_program {
    Program prog;
};

extern "C" int tg_dispatch_once(tg_ctx *ctx, const tg_dispatch *d, double *ns) {
    if (!ctx || !d) return fail(TG_EINVAL, "tg_dispatch_once: null argument");
    Launch l;
    int st = resolve(*d, l);
    if (!st) st = check_launch(l);
    if (st) return st;
    TG_CUDA(cudaSetDevice(ctx->device));
    std::lock_guard<std::mutex> lock(ctx->mu);
    cudaEvent_t e0, e1;
    TG_CUDA(cudaEventCreate(&e0));
    TG_CUDA(cudaEventCreate(&e1));
    cudaEventRecord(e0, ctx->stream);
    st = enqueue_launch(l, ctx->err_dev, ctx->stream, ctx->sm_count);
    cudaEventRecord(e1, ctx->stream);
    if (!st) st = wait_event(e1, 0);
    if (!st) {
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) st = cuda_fail(e, l.label.empty() ? kernel_name(l.kernel) : l.label.c_str());
    }
    if (!st) st = take_kernel_error(ctx);
    if (!st && ns) {
        float ms = 0;
        cudaEventElapsedTime(&ms, e0, e1);
        *ns = ms * 1e6;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return st;
}

extern "C" int tg_program_create(tg_ctx *ctx, const tg_dispatch *ds, size_t n, int timed, tg_program **out) {
    if (!ctx || !out || (n && !ds)) return fail(TG_EINVAL, "tg_program_create: null argument");
    *out = nullptr;
    std::vector<Launch> launches(n);
    for (size_t i = 0; i < n; i++) {
        const int st = resolve(ds[i], launches[i]);
        if (st) return st;
    }
    TG_CUDA(cudaSetDevice(ctx->device));
    tg_program *p = new tg_program();
    const int st = program_build(ctx, launches, timed != 0, p->prog);
    if (st) {
        program_release(p->prog);
        delete p;
        return st;
    }
    *out = p;
    return TG_OK;
}

extern "C" int tg_program_destroy(tg_program *p) {
    if (!p) return TG_OK;
    cudaSetDevice(p->prog.ctx->device);
    if (p->prog.pending) program_wait(p->prog, 0);
    program_release(p->prog);
    delete p;
    return TG_OK;
}

extern "C" int tg_program_start(tg_program *p) {
    if (!p) return fail(TG_EINVAL, "null program");
    TG_CUDA(cudaSetDevice(p->prog.ctx->device));
    std::lock_guard<std::mutex> lock(p->prog.ctx->mu);
    return program_start(p->prog);
}

extern "C" int tg_program_wait(tg_program *p, uint64_t timeout_ns) {
    if (!p) return fail(TG_EINVAL, "null program");
    return program_wait(p->prog, timeout_ns);
}

extern "C" int tg_program_elapsed_ns(tg_program *p, double *ns) {
    if (!p || !ns) return fail(TG_EINVAL, "null argument");
    *ns = program_elapsed_ns(p->prog);
    return *ns < 0 ? fail(TG_ECUDA, "no completed run to time") : TG_OK;
}

extern "C" int tg_program_timings(tg_program *p, double *ns, size_t n) {
    if (!p || !ns) return fail(TG_EINVAL, "null argument");
    return program_timings(p->prog, ns, n);
}
