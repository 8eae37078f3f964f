// Failure detection exercised without a fault. Every wait in this library's kernels - on an
// mbarrier a copy or another warp completes, or on a word in global memory another block bumps -
// is bounded by %globaltimer: past its limit the kernel records ERR_WAIT_TIMEOUT in the context's
// error word and returns, and the host's next wait reports TG_EKERNEL instead of hanging. This
// kernel runs both kinds of wait on something that never comes - an mbarrier no thread arrives on,
// a word no code writes - so that a test can watch them give up and then use the context again.
// Nothing is in flight when they give up: no copy was issued on the mbarrier.
#include "tg_common.cuh"
#include "tg_internal.h"

namespace {

__device__ uint32_t g_never_written;  // no code stores to it: it stays 0

__global__ void __launch_bounds__(32) bounded_wait_selftest_kernel(uint32_t *err, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    if (blockIdx.x == 0) {
        tg::mbar_init(tg::smem_u32(&bar), 1);  // one arrival expected, none made
        tg::mbar_fence_init();
        tg::mbar_wait_bounded(tg::smem_u32(&bar), 0, err, limit_ns);
    } else {
        tg::flag_wait_bounded(&g_never_written, 1u, err, limit_ns);
    }
}

}  // namespace

extern "C" int tg_ctx_selftest_wait(tg_ctx *ctx, uint64_t limit_ns) {
    using namespace tg;
    if (!ctx) return fail(TG_EINVAL, "null context");
    if (limit_ns < 1000 || limit_ns > 2000000000ull)
        return fail(TG_EINVAL, "tg_ctx_selftest_wait: a limit of %llu ns (1 us to 2 s)", (unsigned long long)limit_ns);
    TG_CUDA(cudaSetDevice(ctx->device));
    {
        std::lock_guard<std::mutex> lock(ctx->mu);
        bounded_wait_selftest_kernel<<<2, 32, 0, ctx->stream>>>(ctx->err_dev, limit_ns);
        TG_CUDA(cudaGetLastError());
    }
    return tg_ctx_synchronize(ctx, 0);
}
