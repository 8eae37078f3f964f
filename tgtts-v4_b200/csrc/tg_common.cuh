// Device-side building blocks shared by every kernel: the storage types, 16-byte vector loads,
// and the fixed reduction orders that make a row's result independent of the batch it runs in
// (tgtts-v4's invariant, crates/graph/src/decode.rs:8-11, kernels/glsl/gemv.glsl:1-5).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tgcuda.h"

#define TG_DEVICE __device__ __forceinline__

namespace tg {

using bf16 = __nv_bfloat16;

// Error words a kernel may set in the context's error buffer (read by the host after a wait).
enum : uint32_t {
    ERR_NONE = 0,
    ERR_WAIT_TIMEOUT = 1,  // a bounded spin on an mbarrier gave up
    ERR_BAD_INDEX = 2,     // a placement word pointed outside its buffer and was skipped
};

// One 16-byte load of storage type T: 4 f32 or 8 bf16, widened to f32.
template <typename T>
struct Vec;
template <>
struct Vec<float> {
    static constexpr int N = 4;
    using Raw = float4;
    static TG_DEVICE void unpack(const Raw &r, float (&f)[N]) {
        f[0] = r.x;
        f[1] = r.y;
        f[2] = r.z;
        f[3] = r.w;
    }
};
template <>
struct Vec<bf16> {
    static constexpr int N = 8;
    using Raw = uint4;
    static TG_DEVICE void unpack(const Raw &r, float (&f)[N]) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
};

template <typename T>
TG_DEVICE float to_f32(T v);
template <>
TG_DEVICE float to_f32<float>(float v) { return v; }
template <>
TG_DEVICE float to_f32<bf16>(bf16 v) { return __bfloat162float(v); }

// Rounds to the storage type, to nearest even (the only rounding points are where a tensor is
// stored, kernels/glsl/common.glsl:1-7).
template <typename T>
TG_DEVICE T from_f32(float v);
template <>
TG_DEVICE float from_f32<float>(float v) { return v; }
template <>
TG_DEVICE bf16 from_f32<bf16>(float v) { return __float2bfloat16_rn(v); }

// A read-only 16-byte load through the non-coherent path.
template <typename R>
TG_DEVICE R ldg16(const R *p) { return __ldg(p); }

// Streaming variant for weights that are read once per step.
TG_DEVICE uint4 ld_stream(const uint4 *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
TG_DEVICE float4 ld_stream(const float4 *p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

// Warp sum by the xor butterfly 16, 8, 4, 2, 1: every lane ends with the same bits, and the order
// depends on nothing but the lane values.
TG_DEVICE float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
TG_DEVICE float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The canonical RMSNorm scale of one f32 row of k values (k a multiple of 128), taken by one warp:
// lane l sums the squares of float4 chunks l, l + 32, ... in order (one fused multiply-add per
// value), then the butterfly joins the lanes. Every kernel that norms a row calls this, so a row's
// scale is the same bits wherever and beside whatever it is computed. 1 / sqrt(mean + eps) as
// kernels/glsl/norm.glsl:29 (IEEE division and square root).
TG_DEVICE float warp_rms_scale(const float *row, int k, float eps) {
    const int lane = threadIdx.x & 31;
    const float4 *v = reinterpret_cast<const float4 *>(row);
    float s = 0.0f;
    for (int c = lane; c < k / 4; c += 32) {
        float4 q = v[c];
        s = __fmaf_rn(q.x, q.x, s);
        s = __fmaf_rn(q.y, q.y, s);
        s = __fmaf_rn(q.z, q.z, s);
        s = __fmaf_rn(q.w, q.w, s);
    }
    s = warp_sum(s);
    return 1.0f / sqrtf(__fdiv_rn(s, (float)k) + eps);
}

// warp_rms_scale of a row in global memory that other blocks of the same launch wrote: the same
// sums in the same order, its loads through L2 (ld.global.cg), eight chunks a lane in flight at once.
TG_DEVICE float warp_rms_scale_cg(const float *row, int k, float eps) {
    const int lane = threadIdx.x & 31;
    const float4 *v = reinterpret_cast<const float4 *>(row);
    const int n = k / 4;
    float s = 0.0f;
    for (int c0 = lane; c0 < n; c0 += 32 * 8) {
        float4 q[8];
#pragma unroll
        for (int u = 0; u < 8; u++) q[u] = c0 + 32 * u < n ? __ldcg(v + c0 + 32 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; u++) {
            if (c0 + 32 * u >= n) continue;
            s = __fmaf_rn(q[u].x, q[u].x, s);
            s = __fmaf_rn(q[u].y, q[u].y, s);
            s = __fmaf_rn(q[u].z, q[u].z, s);
            s = __fmaf_rn(q[u].w, q[u].w, s);
        }
    }
    s = warp_sum(s);
    return 1.0f / sqrtf(__fdiv_rn(s, (float)k) + eps);
}

TG_DEVICE float silu_mul(float g, float u) { return __fdiv_rn(g, 1.0f + expf(-g)) * u; }

// Placement words (crates/graph/src/decode.rs:198-227, kernels/glsl/batch.glsl:9-14): positions
// of `rows` rows, then their slots when slots > 1. A row placed past the capacity or the slots is
// spare: it writes no cache and attends to nothing.
TG_DEVICE bool placed(const uint32_t *at, int rows, int b, uint32_t capacity, uint32_t slots,
                      uint32_t &pos, uint32_t &slot) {
    pos = at[b];
    slot = slots > 1 ? at[rows + b] : 0u;
    return pos < capacity && slot < slots;
}

// The q/k/v epilogue of decode unit u (a RoPE pair of rows (i, i + hd/2) of head u / (hd/2)) for
// batch row b, given the pair's two sums (gemv_qkv_rope.comp:51-107): q heads are rotated and
// stored f32 at q[b][head][hd], k heads rotated and v heads as they are into the row's slot of the
// caches at its position. A spare row stores nothing.
template <typename T>
TG_DEVICE void qkv_store(const tg_params &p, const uint32_t *at, const float *cosv, const float *sinv, float *q,
                         void *kcache, void *vcache, int u, int b, float ra, float rc) {
    const int hd = p.head_dim, half = hd / 2, heads = p.heads, kvh = p.kv_heads;
    const int head = u / half, i = u % half;
    uint32_t pos, slot;
    if (!placed(at, p.rows, b, p.capacity, p.slots, pos, slot)) return;
    T *kc = static_cast<T *>(kcache);
    T *vc = static_cast<T *>(vcache);
    if (head >= heads + kvh) {
        const size_t to = (((size_t)slot * kvh + (head - heads - kvh)) * p.capacity + pos) * hd + i;
        vc[to] = from_f32<T>(ra);
        vc[to + half] = from_f32<T>(rc);
        return;
    }
    if (p.rope) {
        // As upstream: x cos + rotate_half(x) sin (gemv_qkv_rope.comp:85-90).
        const float co = cosv[(size_t)pos * half + i], si = sinv[(size_t)pos * half + i];
        const float na = __fmaf_rn(ra, co, -__fmul_rn(rc, si));
        const float nc = __fmaf_rn(rc, co, __fmul_rn(ra, si));
        ra = na;
        rc = nc;
    }
    if (head < heads) {
        const size_t to = ((size_t)b * heads + head) * hd + i;
        q[to] = ra;
        q[to + half] = rc;
    } else {
        const size_t to = (((size_t)slot * kvh + (head - heads)) * p.capacity + pos) * hd + i;
        kc[to] = from_f32<T>(ra);
        kc[to + half] = from_f32<T>(rc);
    }
}

// ---- mbarriers, bulk copies, programmatic dependent launch (sm_90+) ------------------------------

TG_DEVICE uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

TG_DEVICE uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

TG_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

TG_DEVICE void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

TG_DEVICE void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

TG_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

TG_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of parity `parity` of `bar` to complete, for at most `limit_ns`. Past that it
// records ERR_WAIT_TIMEOUT in `err` and returns false, so that the kernel always ends.
TG_DEVICE bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint32_t *err, uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > limit_ns) {
            if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

// An acquiring load of a word other blocks (of this grid or another) update.
TG_DEVICE uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until the word at `flag` is at least `target`, for at most `limit_ns`; gives up early when
// `abort` (if given) is nonzero. Past the limit it records ERR_WAIT_TIMEOUT in `err`, sets `abort`
// so that the grid's other waits end too, and returns false. Called by one thread.
TG_DEVICE bool flag_wait_bounded(const uint32_t *flag, uint32_t target, uint32_t *err, uint64_t limit_ns,
                                 uint32_t *abort = nullptr) {
    if (ld_acquire_gpu(flag) >= target) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; i++) {
        if (ld_acquire_gpu(flag) >= target) return true;
        if ((i & 7) == 0) {
            if (abort && *(volatile uint32_t *)abort) return false;
            if (globaltimer() - t0 > limit_ns) {
                if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
                if (abort) atomicExch(abort, 1u);
                return false;
            }
        }
    }
}

// A 1-D bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global to
// this block's shared memory, completing on mbarrier `bar` (no multicast).
TG_DEVICE void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// Programmatic dependent launch: a kernel lets the next one start as soon as all of its blocks
// are running (launch_dependents), and waits for the one before it to finish and its writes to
// land (wait) only where it first reads what that one wrote. Every block waits before it ends,
// so that a kernel never finishes ahead of the one before it. Both are no-ops in a launch
// without the programmatic attribute.
TG_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
TG_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- host ---------------------------------------------------------------------------------------

// Launches `kern` with the programmatic-stream-serialization attribute, so that in a stream (or a
// graph captured from one) it may start while the kernel before it finishes (see pdl_wait).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <typename F>
inline cudaError_t with_smem(F kernel, size_t bytes) {
    // Past 48 KiB of shared memory a block needs the opt-in, static arrays included: opt in well
    // before.
    if (bytes <= 32 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}


}  // namespace tg
