// Decode attention for callers that must not allocate device memory.
//
// Some embedders of this library run under an allocator they own: a serving engine that hands
// out every byte of HBM from its own pool and budgets it up front, or code that records its work
// into a CUDA graph, where a cudaMalloc in the middle would break the capture. Such a caller can
// pass in its inputs and outputs but cannot let a kernel allocate its own temporaries. Decode
// attention (attention_split, then attention_combine) needs temporaries - each chunk's partial
// output, maximum and sum - so this entry point keeps them in a fixed array compiled into the
// library instead.
//
// The array is a file-scope `static __device__` buffer of TG_NOALLOC_SCRATCH_BYTES. Every device
// that loads the library holds one copy until the process exits. Host code cannot hand the
// array's name to a kernel - on the host it is only a stand-in, not a device address - so the
// first call on each device looks the address up with cudaGetSymbolAddress (with that device
// current) and remembers it. That first call may load the library's module on the device, so make
// it before any stream capture. Every call on a device shares the one array and it keeps the last
// call's contents: calls that overlap on the GPU (on different streams without ordering between
// them) race on it. Nothing in it needs to start at zero: each call writes every partial it reads.
// The array used is the current device's, so the stream passed must belong to the current device;
// a stream of another device is refused.
#include <mutex>

#include "tg_common.cuh"
#include "tg_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_attention_scratch[TG_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_setup;
void *g_scratch_addr[MAX_DEVICES] = {nullptr};

uint64_t round256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

}  // namespace

extern "C" int tg_attention_decode_noalloc(const tg_params *p, const float *q, const void *k_cache,
                                           const void *v_cache, const uint32_t *at, float *out, void *stream) {
    using namespace tg;
    if (!p || !q || !k_cache || !v_cache || !at || !out)
        return fail(TG_EINVAL, "tg_attention_decode_noalloc: null argument");
    const void *ptrs[] = {q, k_cache, v_cache, at, out};
    for (const void *ptr : ptrs)
        if (reinterpret_cast<uintptr_t>(ptr) % 16)
            return fail(TG_EINVAL, "tg_attention_decode_noalloc: a pointer is not 16-byte aligned");
    if (p->dtype != TG_F32 && p->dtype != TG_BF16) return fail(TG_ESHAPE, "dtype %u", p->dtype);
    if (p->rows == 0 || p->slots == 0 || p->heads == 0 || p->kv_heads == 0 || p->heads % p->kv_heads || p->heads / p->kv_heads > MAX_GROUP ||
        (p->head_dim != 64 && p->head_dim != 128) || p->capacity == 0 || p->capacity % CAPACITY_STEP)
        return fail(TG_ESHAPE, "tg_attention_decode_noalloc: %u rows, %u heads over %u of %u, a cache of %u",
                    p->rows, p->heads, p->kv_heads, p->head_dim, p->capacity);
    const uint64_t partials = (uint64_t)p->rows * p->heads * attn_chunks(p->capacity);
    const uint64_t o_bytes = round256(partials * p->head_dim * 4);
    const uint64_t need = o_bytes + partials * 2 * 4;
    if (need > TG_NOALLOC_SCRATCH_BYTES)
        return fail(TG_ESHAPE,
                    "tg_attention_decode_noalloc: %u rows x %u heads x %u chunks need %llu bytes of scratch; "
                    "the fixed array holds %u",
                    p->rows, p->heads, attn_chunks(p->capacity), (unsigned long long)need,
                    (unsigned)TG_NOALLOC_SCRATCH_BYTES);
    int dev = 0;
    TG_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= MAX_DEVICES) return fail(TG_ENODEVICE, "device %d", dev);
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup);
        if (!g_scratch_addr[dev]) {
            void *addr = nullptr;
            TG_CUDA(cudaGetSymbolAddress(&addr, g_attention_scratch));
            g_scratch_addr[dev] = addr;
        }
        base = g_scratch_addr[dev];
    }
    float *po = static_cast<float *>(base);
    float *pml = reinterpret_cast<float *>(static_cast<char *>(base) + o_bytes);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (s) {
        int stream_dev = dev;
        TG_CUDA(cudaStreamGetDevice(s, &stream_dev));
        if (stream_dev != dev)
            return fail(TG_EINVAL, "tg_attention_decode_noalloc: the stream belongs to device %d, the current device is %d",
                        stream_dev, dev);
    }
    cudaError_t e = launch_attention_split(*p, q, k_cache, v_cache, at, po, pml, s);
    if (e == cudaSuccess) e = launch_attention_combine(*p, at, po, pml, out, s);
    if (e != cudaSuccess) return cuda_fail(e, "tg_attention_decode_noalloc");
    return TG_OK;
}
