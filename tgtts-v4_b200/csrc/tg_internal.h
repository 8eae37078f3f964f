// Host-side internals shared by the runtime, the kernel table and the model: the handle types
// behind the C ABI, per-thread error messages, and the launch interface every kernel implements.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "tgcuda.h"

struct tg_ctx {
    int device = 0;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    char name[256] = {0};
    cudaStream_t stream = nullptr;
    // One error word the kernels may set (tg::ERR_*), in mapped pinned memory so the host reads
    // it after a wait without a copy.
    uint32_t *err_host = nullptr;
    uint32_t *err_dev = nullptr;
    std::mutex mu;  // submission is behind a mutex (crates/vulkan/src/recording.rs:622-628)
};

struct tg_mem {
    tg_ctx *ctx = nullptr;
    void *ptr = nullptr;  // device pointer, or the mapped device address of pinned memory
    void *host = nullptr; // pinned host address for UPLOAD / READBACK
    uint64_t bytes = 0;
    tg_residence residence = TG_RES_DEVICE;
};

namespace tg {

// Records `msg` as the calling thread's last error and returns `status`.
int fail(int status, const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);
void clear_error();

#define TG_CUDA(call)                                             \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return ::tg::cuda_fail(e_, #call); \
    } while (0)

// The persistent decode step: everything it reads and writes (a decoder's buffers).
struct DecodeStep {
    tg_params p;
    int layers;
    const unsigned char *weights;
    const uint64_t *offs;  // device [layers][6]: qkv, o, gate_up, down, input norm, post norm
    uint64_t final_norm;
    const float *cosv, *sinv;
    const uint32_t *at;
    const float *x_in;
    float *h, *mid, *mlp, *q, *att, *out, *po, *pml;
    unsigned char *kcache, *vcache;
    uint64_t cache_layer;
    uint32_t *sync;  // decode_step_flag_bytes(layers): the step's counters, zeroed by the launch
    uint32_t *err;
};
// Kernel ids past the table's, for launches the library records itself.
constexpr uint32_t KERNEL_DECODE_STEP = 1000;  // the persistent decode step (DecodeStep)
// The batched decoder's projections on tcgen05, with the bindings of GEMV_QKV_ROPE, GEMV_GATE_UP
// and GEMV_RESIDUAL.
constexpr uint32_t KERNEL_DTC_QKV_ROPE = 1001;
constexpr uint32_t KERNEL_DTC_GATE_UP = 1002;
constexpr uint32_t KERNEL_DTC_RESIDUAL = 1003;

// The batched decoder's attention_split on mma.sync (bf16, head_dim 64), ATTENTION_SPLIT's bindings,
// each partial over DECODE_WIDE_CHUNK positions; and attention_combine over such partials.
constexpr uint32_t KERNEL_ATTN_SPLIT_MMA = 1004;
constexpr uint32_t KERNEL_ATTN_COMBINE_WIDE = 1005;
// The same two for the GEMM-family decoder: q in bf16 (as the q/k/v GEMM's epilogue stores it; its
// binding still sized as f32 q), the joined output in bf16 (the o GEMM's A operand; sized as f32).
constexpr uint32_t KERNEL_ATTN_SPLIT_MMA_BQ = 1006;
constexpr uint32_t KERNEL_ATTN_COMBINE_WIDE_BF = 1007;
// The two of the GEMM-family decoder in one launch (the split's bindings, then out bf16 [rows][heads
// hd] and counts u32 [rows][kv_heads], zero before the first launch and after each).
constexpr uint32_t KERNEL_ATTN_SPLIT_JOIN = 1008;
// The prefill's o and down projections with the residual add in the GEMM's epilogue: GEMM's
// bindings (a, b, c: the sum) and then the residual f32 [m][n] (scaled by params.residual_scale).
constexpr uint32_t KERNEL_GEMM_RESIDUAL = 1009;
cudaError_t launch_gemm_residual(const tg_params &p, const void *a, const void *b, const float *res, float *out,
                                 uint32_t *err, cudaStream_t s);
// 64: wider partials (a warp walking sub-chunks) measured slower on B200 at 16-128 rows: 2.15 ms
// a step at 64 rows with 256 against 2.00 ms with 64.
constexpr uint32_t DECODE_WIDE_CHUNK = 64;
cudaError_t launch_attention_combine_chunk(const tg_params &p, uint32_t chunk, const uint32_t *at, const float *po,
                                           const float *pml, void *out, cudaStream_t s, bool out_bf16 = false);
bool attention_split_mma_supported(const tg_params &p);
cudaError_t launch_attention_split_mma(const tg_params &p, const void *q, const void *kc, const void *vc,
                                       const uint32_t *at, float *po, float *pml, cudaStream_t s, bool q_bf16 = false);
cudaError_t launch_attention_split_join(const tg_params &p, const void *q, const void *kc, const void *vc,
                                        const uint32_t *at, float *po, float *pml, void *out, uint32_t *counts,
                                        cudaStream_t s);
// Decoders of at least this many rows run their projections on tcgen05 (every bucket of them).
constexpr uint32_t DTC_MIN_ROWS = 16;

// One dispatch resolved to device pointers, as the kernel table launches it.
struct Launch {
    uint32_t kernel = 0;
    tg_params p{};
    std::vector<void *> ptr;
    std::vector<uint64_t> bytes;
    std::string label;
    DecodeStep step{};  // KERNEL_DECODE_STEP only
};

// The kernel table: checks a dispatch's params against its bindings' sizes (what each binding
// must hold for the grid the params give), then launches it on `stream`.
int check_launch(const Launch &l);
int enqueue_launch(const Launch &l, uint32_t *err_dev, cudaStream_t stream, int sm_count);

// A captured chain of launches (a CUDA graph) with optional events between them.
struct Program {
    tg_ctx *ctx = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    std::vector<cudaEvent_t> events;  // [n + 1] when timed, else [2]
    std::vector<std::string> labels;
    bool timed = false;
    bool pending = false;
};

// Captures `launches` (plus any host-to-device copies `pre` issues first) into a graph on the
// context's stream. `pre` may be empty.
int program_build(tg_ctx *ctx, const std::vector<Launch> &launches, bool timed, Program &out);
int program_start(Program &p);
// Launches the program behind whatever the stream holds, without waiting for an earlier run of it
// (stream order keeps the runs apart); a later wait waits for the last.
int program_launch(Program &p);
int program_wait(Program &p, uint64_t timeout_ns);
void program_release(Program &p);
double program_elapsed_ns(Program &p);
int program_timings(Program &p, double *ns, size_t n);

// Polls `ev` until it completes or `timeout_ns` passes (0: no limit).
int wait_event(cudaEvent_t ev, uint64_t timeout_ns);
// Reads and clears the context's kernel error word; TG_EKERNEL when it was set.
int take_kernel_error(tg_ctx *ctx);

// Kernel launchers, one per family (kernels_decode.cu, kernels_prefill.cu, gemm_sm100.cu).
cudaError_t launch_rmsnorm(const tg_params &p, const float *x, const float *g, float *out,
                           cudaStream_t s);
cudaError_t launch_gemv_qkv_rope(const tg_params &p, const float *x, const float *g,
                                 const void *w, const float *cos, const float *sin,
                                 const uint32_t *at, void *q, void *kc, void *vc, uint32_t *err,
                                 cudaStream_t s);
cudaError_t launch_attention_split(const tg_params &p, const void *q, const void *kc,
                                   const void *vc, const uint32_t *at, float *po, float *pml,
                                   cudaStream_t s);
cudaError_t launch_attention_combine(const tg_params &p, const uint32_t *at, const float *po,
                                     const float *pml, void *out, cudaStream_t s);
cudaError_t launch_gemv_residual(const tg_params &p, const void *x, const void *w,
                                 const float *res, float *out, uint32_t *err, cudaStream_t s);
cudaError_t launch_gemv_gate_up(const tg_params &p, const float *x, const float *g,
                                const void *w, void *out, uint32_t *err, cudaStream_t s);
// Split and combine in one kernel: a thread-block cluster per (row, kv head).
cudaError_t launch_stream_read(const tg_params &p, const uint32_t *data, uint32_t *out,
                               cudaStream_t s, int sm_count);
cudaError_t launch_norm_rows(const tg_params &p, const uint32_t *at, const float *x,
                             const float *g, void *out, cudaStream_t s);
// The most parts of K an add_norm_rows dispatch adds (tg_params.parts).
constexpr int ADD_NORM_MAX_PARTS = 16;
cudaError_t launch_add_norm_rows(const tg_params &p, const uint32_t *at, const float *c,
                                 const float *res, const float *g, float *sum, void *normed,
                                 cudaStream_t s);
cudaError_t launch_rope_rows(const tg_params &p, const uint32_t *at, const float *c,
                             const float *cos, const float *sin, void *q, void *kc, void *vc,
                             cudaStream_t s);
cudaError_t launch_attention_rows(const tg_params &p, const uint32_t *at, const void *q,
                                  const void *kc, const void *vc, void *out, cudaStream_t s);
cudaError_t launch_silu_mul_rows(const tg_params &p, const uint32_t *at, const float *c,
                                 void *out, cudaStream_t s);
// C[m][n] = A[m][k] B[n][k]^T in f32. bf16 operands run on tcgen05 (TMA-fed, TMEM accumulator);
// f32 operands on a SIMT kernel. Returns cudaErrorInvalidValue for shapes it does not tile.
cudaError_t launch_gemm(const tg_params &p, const void *a, const void *b, float *c,
                        uint32_t *err, cudaStream_t s);
// The batched decode projections (kernels_decode_tc.cu): true when the q/k/v, gate/up and output
// projections of a step of p.rows rows of this shape have a plan; the down projection runs on
// tcgen05 when dtc_residual_supported(p, inner) too, else as the GEMV (a 6144-column slice of W
// does not fit a cluster's shared memory).
bool dtc_supported(const tg_params &p);
bool dtc_residual_supported(const tg_params &p, int K);
cudaError_t launch_dtc_qkv_rope(const tg_params &p, const float *x, const float *g, const void *w, const float *cosv,
                                const float *sinv, const uint32_t *at, float *q, void *kc, void *vc, uint32_t *err,
                                cudaStream_t s);
cudaError_t launch_dtc_gate_up(const tg_params &p, const float *x, const float *g, const void *w, float *out,
                               uint32_t *err, cudaStream_t s);
cudaError_t launch_dtc_residual(const tg_params &p, const float *x, const void *w, const float *res, float *out,
                                uint32_t *err, cudaStream_t s);
// One cooperative launch for the whole step (batches of up to 2 rows); cudaErrorNotSupported when
// the shape or batch is not one it takes.
cudaError_t launch_decode_step(const DecodeStep &d, int sm_count, cudaStream_t s);
// The bytes of the persistent step's arrival counters for a stack of `layers` layers.
size_t decode_step_flag_bytes(int layers);
// The decode constants: positions per attention chunk.
constexpr uint32_t ATTN_CHUNK = 64;
// The most query heads one KV head may serve: decode attention gives a thread at most 8 of a
// group's heads (attention_chunk's chunk_scores / chunk_outputs).
constexpr uint32_t MAX_GROUP = 8;
// A cache's capacity is a multiple of this, as the reference's (decode.rs:28 CHUNK, :480); the
// last attention chunk of a cache may then be half full.
constexpr uint32_t CAPACITY_STEP = 32;
// The attention chunks of a cache of `capacity` positions, the last perhaps partial.
__host__ __device__ inline uint32_t attn_chunks(uint32_t capacity) { return (capacity + ATTN_CHUNK - 1) / ATTN_CHUNK; }
// The rows of a prefill attention tile (the CUDA-core and mma.sync kernels).
constexpr uint32_t PREFILL_TILE = 64;
// Each run of a prefill launch starts on a multiple of this many rows (the tcgen05 attention's tile).
constexpr uint32_t RUN_ALIGN = 128;
bool attention_tc_supported(const tg_params &p);
cudaError_t launch_attention_rows_tc(const tg_params &p, const uint32_t *at, const void *q, const void *kc,
                                     const void *vc, void *out, uint32_t *err, cudaStream_t s);
// gate_up's rows are gate and up interleaved in blocks of GU_BLOCK: gate rows i .. i + 127 then up
// rows i .. i + 127, for i = 0, 128, ... (so that a 256-wide GEMM tile holds matching gate and up
// columns, and its epilogue can take SiLU(gate) up).
constexpr uint32_t GU_BLOCK = 128;
__host__ __device__ inline uint32_t gate_up_row(uint32_t i, uint32_t up) {
    return (i / GU_BLOCK) * (2 * GU_BLOCK) + up * GU_BLOCK + i % GU_BLOCK;
}
// gemv_linear.comp: out[b][offset + i] = act(W [x0; x1] + bias)[i] (kernels_linear.cu).
cudaError_t launch_gemv_linear(const tg_params &p, const float *x0, const float *x1, const void *w, const float *bias,
                               float *out, cudaStream_t s);
// The q/k/v projection with rope_rows in its epilogue (bf16, n = (heads + 2 kv) hd, a multiple of 256).
cudaError_t launch_gemm_qkv_rope(const tg_params &p, const void *a, const void *b, const uint32_t *at,
                                 const float *cosv, const float *sinv, void *q, void *kc, void *vc, uint32_t *err,
                                 cudaStream_t s);
// out[m][n / 2] = SiLU(gate) up of C = A B^T, B's rows in gate_up_row's order (bf16, n % 256 == 0).
cudaError_t launch_gemm_silu(const tg_params &p, const void *a, const void *b, void *out, uint32_t *err,
                             cudaStream_t s);

// The local stacks (local.cu): f16 kernels over m tokens in sequences of p.capacity.
bool local_proj_supported(int M, int N, int K, int parts);
// A local projection's weight W [N][K] (f16) is stored tiled: the 128 x 64 block of rows
// [128 t, +128) and columns [64 b, +64) is 16 KiB at ((t K / 64 + b) 16 KiB), its row r's 16-byte
// chunk c (columns 64 b + 8 c ..) at (r / 8) 1024 + (r % 8) 128 + ((c ^ (r % 8)) 16): the 128-byte
// swizzle of a K-major tcgen05 operand. The byte offset of element (row, col):
__host__ __device__ inline uint64_t local_tiled_offset(uint32_t row, uint32_t col, uint32_t K) {
    const uint32_t t = row / 128, r = row % 128, b = col / 64, c = (col % 64) / 8;
    return ((uint64_t)t * (K / 64) + b) * 16384 + (r / 8) * 1024 + (r % 8) * 128 + ((c ^ (r % 8)) << 4) + (col % 8) * 2;
}
// Writes rows [row0 + i step] (i < rows) of a tiled weight of K columns from src [rows][K] f16.
cudaError_t launch_local_tile_rows(const void *src, int rows, int K, void *dst, int row0, int step, cudaStream_t s);
cudaError_t launch_local_norm(const tg_params &p, const void *x, const void *g, void *out, cudaStream_t s);
cudaError_t launch_local_partial(const tg_params &p, const void *x, const void *w, float *part, uint32_t *err,
                                 cudaStream_t s);
cudaError_t launch_local_gate_up(const tg_params &p, const void *x, const void *w, void *out, uint32_t *err,
                                 cudaStream_t s);
cudaError_t launch_local_attention(const tg_params &p, const float *part, const float *cosv, const float *sinv,
                                   void *out, cudaStream_t s);
cudaError_t launch_local_add_norm(const tg_params &p, const float *part, const void *res, const void *g, void *sum,
                                  void *normed, cudaStream_t s);
cudaError_t launch_local_rows(const tg_params &p, const void *x, void *out, cudaStream_t s);
cudaError_t launch_local_embed(const tg_params &p, const float *src, const void *w, const void *bias,
                               const void *tokens, void *h, cudaStream_t s);
cudaError_t launch_cfm_noise(const tg_params &p, const float *noise, const float *sampling, float *x, cudaStream_t s);
cudaError_t launch_dit_euler(const tg_params &p, const void *h, const void *w, const void *bias,
                             const float *sampling, float *x, cudaStream_t s);

}  // namespace tg
