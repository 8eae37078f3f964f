/*
 * tgcuda: the B200 (sm_100a) runtime and kernels for the MiniCPM-4 stack that tgtts-v4's `graph`
 * crate drives, behind a plain C ABI. It replaces the `vulkan` crate (crates/vulkan/src/lib.rs:50-60)
 * as the layer under `graph::step::Step`, and the GLSL/MLIR kernels of kernels/glsl and
 * kernels/gpu, for the decode step (crates/graph/src/decode.rs) and the prefill
 * (crates/graph/src/prefill.rs).
 *
 * Every function returns a tg_status; on failure, tg_last_error() holds a message for the calling
 * thread. Shape and size violations are refused before anything is launched. Nothing here
 * falls back to the CPU: without a usable CUDA device, tg_ctx_create fails.
 *
 * Element types: the residual stream, norms' gains, RoPE tables, partial attention sums and every
 * host-facing hidden state are f32, and so is every activation of the decode step (q, attention
 * output, SiLU output). The storage type of a stack (tg_dtype) is that of its weights and KV
 * cache, and of the prefill's GEMM operands (normed inputs, q, attention output, SiLU output):
 * f32 or bf16, always with f32 accumulation.
 */
#ifndef TGCUDA_H
#define TGCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TGCUDA_ABI_VERSION 1u

/* graph::Error / vulkan::Error (crates/graph/src/lib.rs:41-59, crates/vulkan/src/error.rs:3-40),
 * as status codes. */
typedef enum {
    TG_OK = 0,
    TG_EINVAL = 1,     /* a null handle or pointer, an unknown name or kernel */
    TG_ESHAPE = 2,     /* graph::Error::Shape: shapes or placements the kernels cannot run */
    TG_ECUDA = 3,      /* vulkan::Error::Vk: a CUDA call failed */
    TG_ENOMEM = 4,     /* vulkan::Error::NoMemoryType: an allocation failed */
    TG_ETIMEOUT = 5,   /* a wait ran past its deadline (crates/vulkan/src/context.rs:119-136) */
    TG_ENOTFINITE = 6, /* graph::Error::NotFinite: a sampled patch came out NaN or infinite */
    TG_EKERNEL = 7,    /* a kernel reported an error word (a bounded wait that gave up) */
    TG_ENODEVICE = 8   /* vulkan::Error::NoDevice */
} tg_status;

/* vulkan::Residence (crates/vulkan/src/memory.rs): where a buffer lives. */
typedef enum {
    TG_RES_DEVICE = 0,   /* HBM, for the GPU alone; the host reaches it by copies */
    TG_RES_UPLOAD = 1,   /* pinned host memory the host writes and the GPU reads */
    TG_RES_READBACK = 2  /* pinned host memory the GPU writes and the host reads */
} tg_residence;

/* TG_F16 is the local stacks' storage type (and a source type for loads). */
typedef enum { TG_F32 = 0, TG_BF16 = 1, TG_F16 = 2 } tg_dtype;

typedef struct tg_ctx tg_ctx;
typedef struct tg_mem tg_mem;
typedef struct tg_program tg_program;
typedef struct tg_decoder tg_decoder;
typedef struct tg_prefill tg_prefill;

/* The message of the calling thread's last failure, or "" (never NULL). */
const char *tg_last_error(void);
uint32_t tg_abi_version(void);

/* ---- Context (crates/vulkan/src/context.rs:198-240) ------------------------------------- */

/* A context on CUDA device `device`, with its own stream. Fails with TG_ENODEVICE when there is
 * no such device or it is not an sm_100 part. */
int tg_ctx_create(int device, tg_ctx **out);
int tg_ctx_destroy(tg_ctx *ctx);
/* Waits for all work on the context's stream, polling until `timeout_ns` (0: no limit). */
int tg_ctx_synchronize(tg_ctx *ctx, uint64_t timeout_ns);
/* The device's name and SM count. */
int tg_ctx_info(tg_ctx *ctx, char *name, size_t name_bytes, int *sm_count);
/* The context's CUDA stream (a cudaStream_t), on which every program of the context runs: callers
 * time them with events recorded on it. */
void *tg_ctx_stream(tg_ctx *ctx);
/* Checks the kernels' failure detection (Submission::wait's bound, crates/vulkan/src/context.rs:
 * 119-136, carried into the device): runs a kernel whose two waits - on an mbarrier no thread
 * arrives on, and on a global word nothing writes - can never be met, each bounded by
 * `limit_ns` (1 us to 2 s) as every wait in the library's kernels is. Both give up, the kernel
 * returns, and this call returns what the context's next wait reports: TG_EKERNEL ("a bounded
 * wait gave up"). The context stays usable afterwards. */
int tg_ctx_selftest_wait(tg_ctx *ctx, uint64_t limit_ns);

/* ---- Memory (Context::memory_in / buffer_in, crates/vulkan/src/context.rs:487-495) -------- */

int tg_mem_alloc(tg_ctx *ctx, uint64_t bytes, tg_residence residence, tg_mem **out);
int tg_mem_free(tg_mem *mem);
uint64_t tg_mem_size(const tg_mem *mem);
/* The buffer's address for the GPU (a device pointer, or the mapped address of pinned memory). */
void *tg_mem_device_ptr(const tg_mem *mem);
/* Buffer::write_at / read_at (crates/vulkan/src/memory.rs:518-548): synchronous. */
int tg_mem_write(tg_mem *mem, uint64_t offset, const void *src, uint64_t bytes);
int tg_mem_read(tg_mem *mem, uint64_t offset, void *dst, uint64_t bytes);
int tg_mem_fill(tg_mem *mem, uint64_t offset, uint32_t word, uint64_t bytes);

/* Recording::copy_in / copy_out (crates/vulkan/src/recording.rs:522-532): copies of byte ranges
 * between two buffers on the GPU, in order, on the context's stream; waits for them. */
typedef struct {
    uint64_t src_offset, dst_offset, bytes;
} tg_region;
int tg_copy_regions(tg_ctx *ctx, tg_mem *src, tg_mem *dst, const tg_region *regions, size_t n);

/* ---- Kernel table (crates/graph/src/kernels.rs:104-161, crates/graph/src/prefill.rs:32-131) --
 * Each kernel takes its bindings in the order listed and a params struct. A dispatch whose
 * bindings are too small for what its params say it reaches is refused (Kernels::check,
 * crates/graph/src/kernels.rs:232-263). "T" is the params' dtype. */
typedef enum {
    /* x f32 [rows][hidden], gain f32 [hidden] -> out f32 [rows][hidden]           rmsnorm.comp */
    TG_KERNEL_RMSNORM = 0,
    /* x f32 [rows][hidden], gain f32, W T [(heads+2kv)hd][hidden], cos f32, sin f32,
     * at u32 [2 rows] -> q f32 [rows][heads][hd], k cache T, v cache T          gemv_qkv_rope.comp */
    TG_KERNEL_GEMV_QKV_ROPE = 1,
    /* q f32, k cache T, v cache T, at u32 -> partial_o f32 [rows][heads][chunks][hd],
     * partial_ml f32 [rows][heads][chunks][2]                                  attention_split.comp */
    TG_KERNEL_ATTENTION_SPLIT = 2,
    /* at u32, partial_o f32, partial_ml f32 -> out f32 [rows][heads hd]      attention_combine.comp */
    TG_KERNEL_ATTENTION_COMBINE = 3,
    /* x f32 [rows][k], W T [n][k], residual f32 [rows][n] -> out f32 [rows][n] gemv_residual.comp */
    TG_KERNEL_GEMV_RESIDUAL = 4,
    /* x f32 [rows][hidden], gain f32, W T [2 inner][hidden] (gate and up rows interleaved as for
     * TG_KERNEL_GEMM_SILU) -> out f32 [rows][inner]                             gemv_gate_up.comp */
    TG_KERNEL_GEMV_GATE_UP = 5,
    /* data u32 -> out u32 (one word per block)                                  stream_read.comp */
    TG_KERNEL_STREAM_READ = 6,
    /* at u32 [2 rows], x f32, gain f32 -> out T (f32 when params.normed_f32)     norm_rows.comp */
    TG_KERNEL_NORM_ROWS = 7,
    /* at u32, c f32 [parts][rows][hidden], residual f32, gain f32 -> sum f32, normed (T, or f32
     * when params.normed_f32); c's parts (params.parts, 0 or 1: one; at most 16) are a GEMM's
     * partial sums, added in part order; hidden at most 4096. params.flags bit 1: few rows (a
     * block to a row rather than a warp; the same sums in another order)    add_norm_rows.comp */
    TG_KERNEL_ADD_NORM_ROWS = 8,
    /* at u32, c f32 [rows][(heads+2kv)hd], cos f32, sin f32 -> q T, k cache T, v cache T
     *                                                                             rope_rows.comp */
    TG_KERNEL_ROPE_ROWS = 9,
    /* at u32, q T [rows][heads][hd], k cache T, v cache T -> out T           attention_rows.comp */
    TG_KERNEL_ATTENTION_ROWS = 10,
    /* at u32, c f32 [rows][2 inner] (columns in gate_up's interleaved order) -> out T [rows][inner]
     *                                                                           silu_mul_rows.comp */
    TG_KERNEL_SILU_MUL_ROWS = 11,
    /* a T [m][k], b T [n][k] -> c f32 [m][n] = a b^T        gemm.mlir (tcgen05 for bf16, SIMT f32)
     * params.flags bit 0: b is constant for the program (a weight), so that its first tiles may be
     * loaded while the kernel before is still running (programmatic dependent launch); bit 1:
     * narrow tiles (64 columns; GEMM_QKV_ROPE: one head), for launches of few rows.
     * params.parts > 1 (bf16): K in that many equal parts (k a multiple of 64 parts), c f32
     * [parts][m][n] the partial sum over each, for ADD_NORM_ROWS to add in part order */
    TG_KERNEL_GEMM = 12,
    /* 13: not used (an earlier fused split + combine, measured slower than the two dispatches) */
    /* a bf16 [m][k], b bf16 [2 inner][k] with gate and up rows interleaved in blocks of 128
     * (gate rows i..i+127, then up rows i..i+127, i = 0, 128, ...) -> out bf16 [m][inner] =
     * SiLU(gate) up of a b^T, in the tcgen05 GEMM's epilogue     gemm.mlir + silu_mul_rows.comp */
    TG_KERNEL_GEMM_SILU = 14,
    /* ATTENTION_ROWS on tcgen05, for bf16 and head_dim 64: the same bindings and results within
     * rounding; rows a multiple of 128, each 128-row tile one run's rows (one slot; a tile that
     * mixes slots is refused at run time with the kernel error word). attention_rows.comp */
    TG_KERNEL_ATTENTION_ROWS_TC = 15,
    /* a bf16 [m][hidden] normed rows, b bf16 [(heads + 2 kv) hd][hidden] (the q/k/v projection),
     * at u32 (rows = m), cos, sin -> q T [m][heads hd], k/v appended to the caches: the GEMM with
     * ROPE_ROWS in its epilogue (the f32 projection never stored); bf16, (heads + 2 kv) hd a
     * multiple of 256.                                                gemm.mlir + rope_rows.comp */
    TG_KERNEL_GEMM_QKV_ROPE = 16,
    /* x0 f32 [rows][k], x1 f32 [rows][k1] (any 16 bytes when k1 = 0), W T [n][k + k1], bias f32 [n]
     * -> out f32 [rows][stride]: out[b][offset + i] = act(W [x0; x1] + bias)[i] (the LM side's
     * linear layers: enc_to_lm_proj, the scalar quantizer's in/out, fusion_concat_proj,
     * stop_proj/stop_head). The reference stores f16 bias and output; here both are f32.
     *                                                                       gemv_linear.comp */
    TG_KERNEL_GEMV_LINEAR = 17,
    /* ---- VoxCPM2's local stacks (crates/graph/src/local/mod.rs:29-109), dtype TG_F16: f16
     * weights and activations, f32 sums. `m` tokens in sequences of `capacity` tokens. The tokens
     * a projection reads are stored k-block-major, [k / 64][m][64] ("kb"); the residual stream
     * row-major [m][hidden].
     * x f16 [m][hidden], gain f16 [hidden] -> out f16 kb                         local_norm.comp */
    TG_KERNEL_LOCAL_NORM = 18,
    /* x f16 kb [k / 64][m][64], W f16 [n][k] tiled -> partial f32 [parts][m][n]: part j the sums over columns
     * [j k / parts, (j + 1) k / parts) (tcgen05; n a multiple of 128, k / parts of 64). W tiled: each
     * 128 rows x 64 columns one contiguous 16 KiB block, block (t, b) at (t k / 64 + b) 16 KiB, row
     * r's 16-byte chunk c of it at (r / 8) 1024 + (r % 8) 128 + (c ^ (r % 8)) 16 (the 128-byte
     * swizzle; local::tiled's purpose, local/mod.rs:737-755). The q/k/v, output and down
     * projections.                        local_partial.comp, local_qkv_rope.comp's products */
    TG_KERNEL_LOCAL_PARTIAL = 19,
    /* x f16 kb, W f16 [n][k] tiled as LOCAL_PARTIAL's, gate and up rows alternating (row 2i
     * gate_proj row i, row 2i + 1 up_proj row i) -> out f16 kb [n / 128][m][64] = SiLU(gate) up (tcgen05)
     *                                                                          local_gate_up.comp */
    TG_KERNEL_LOCAL_GATE_UP = 20,
    /* partial f32 [parts][m][(heads + 2 kv) hd] (the q/k/v projection's), cos f32, sin f32
     * [capacity][hd / 2] -> out f16 kb [heads hd / 64][m][64]: the parts joined in order, q and k rotated, all
     * rounded to f16, each token attending to every token of its sequence
     *                                     local_qkv_rope.comp:57-91 + local_attention.comp */
    TG_KERNEL_LOCAL_ATTENTION = 21,
    /* partial f32 [parts][m][n], residual f16 [m][n], gain f16 [n] -> sum f16 [m][n], normed f16 kb
     *                                                                       local_add_norm.comp */
    TG_KERNEL_LOCAL_ADD_NORM = 22,
    /* x f16 kb (m = rows capacity tokens) -> out f16 [rows][n], each sequence's first token
     *                                                                            local_rows.comp */
    TG_KERNEL_LOCAL_ROWS = 23,
    /* src f32 [rows][feat][frames], W f16 [n][feat], bias f16 [n], tokens f16 ([copied][n] when
     * flags & 2, else [rows][copied][n]) -> h f16 [rows][seqs][capacity][n]: tokens first ..
     * first + frames - 1 projected from the frames, `copied` tokens at `at` copied (zero past the
     * first sequence when flags & 1); the others left                           local_embed.comp */
    TG_KERNEL_LOCAL_EMBED = 24,
    /* noise f32 [rows][feat frames], sampling f32 [rows][2] -> x f32 = temperature noise
     *                                                                            cfm_noise.comp */
    TG_KERNEL_CFM_NOISE = 25,
    /* h f16 kb (m = rows 2 capacity tokens), W f16 [feat][k], bias f16 [feat], sampling f32 [rows][2],
     * x f32 [rows][feat][frames] (read and written): x -= dt times the guided velocity of tokens
     * first .. first + frames - 1                                                dit_euler.comp */
    TG_KERNEL_DIT_EULER = 26,
    TG_KERNEL_COUNT = 27
} tg_kernel_id;

/* The stack's shape, as one struct all kernels' params share (decode.rs:66-83 `Shape`, plus the
 * residual scale BASELINE's configs use; 1.0 reproduces tgtts-v4). `rows` is the rows a
 * dispatch covers and `slots` the cache's slots. */
typedef struct {
    uint32_t dtype; /* tg_dtype */
    uint32_t hidden, inner, heads, kv_heads, head_dim, capacity;
    uint32_t rows, slots;
    float eps, residual_scale;
    uint32_t rope;       /* 0: q and k are not rotated */
    uint32_t normed_f32; /* ADD_NORM_ROWS: normed is f32 (the final norm) rather than T */
    uint32_t m, n, k;    /* GEMM, GEMV_RESIDUAL (n outputs of k), STREAM_READ (k words) */
    /* GEMV_LINEAR: n outputs of k + k1 inputs (x0's k then x1's k1), written at out[b][offset + i]
     * of rows `stride` long, through activation `act` (0 none, 1 SiLU, 2 the scalar quantizer's
     * tanh rounded to a multiple of 1 / levels). */
    uint32_t k1, offset, stride, act;
    float levels;
    /* The local stacks' kernels: the column parts of a projection's partial sums; LOCAL_EMBED's
     * sequences a row, first projected token, first copied token, tokens copied and flags (1: the
     * copies are zero past the first sequence, 2: one set of copied tokens for every row); a
     * patch's frames and channels; DIT_EULER's step length. */
    uint32_t parts, seqs, first, at, copied, flags, frames, feat;
    float dt;
} tg_params;

typedef struct {
    tg_mem *mem;
    uint64_t offset, bytes;
} tg_binding;

/* vulkan::Dispatch (crates/vulkan/src/recording.rs:33-87); the grid is derived from the params. */
typedef struct {
    uint32_t kernel; /* tg_kernel_id */
    const tg_params *params;
    const tg_binding *bindings;
    uint32_t n_bindings;
    const char *label; /* for timings; may be NULL */
} tg_dispatch;

/* Context::dispatch (crates/vulkan/src/context.rs:520): runs one dispatch, waits, and gives its
 * GPU time in ns (may be NULL). */
int tg_dispatch_once(tg_ctx *ctx, const tg_dispatch *d, double *ns);

/* ---- Programs (Context::record / Recording, crates/vulkan/src/recording.rs:161-260, :599-760).
 * A program is a chain of dispatches, checked once and captured into one CUDA graph, run as
 * often as needed. `timed` adds an event between dispatches for per-dispatch times. */
int tg_program_create(tg_ctx *ctx, const tg_dispatch *dispatches, size_t n, int timed,
                      tg_program **out);
int tg_program_destroy(tg_program *p);
/* Recording::start_program: launches the graph and returns without waiting. */
int tg_program_start(tg_program *p);
/* Submission::wait: polls until the run ends or `timeout_ns` passes (TG_ETIMEOUT; the run stays
 * pending and is waited for again before the next start). 0: no limit. */
int tg_program_wait(tg_program *p, uint64_t timeout_ns);
/* The last run's GPU time, and with `timed`, each dispatch's (n = dispatch count). */
int tg_program_elapsed_ns(tg_program *p, double *ns);
int tg_program_timings(tg_program *p, double *ns, size_t n);

/* ---- The stack: shape, placement, decoder, prefill (crates/graph/src/decode.rs,
 * crates/graph/src/prefill.rs) --------------------------------------------------------------- */

/* decode.rs:66-83 `Shape`, plus `residual_scale`. capacity: a multiple of 32 (decode.rs:28 CHUNK).
 * rope_factors: head_dim/2 LongRoPE divisors, or NULL for all 1 (plain RoPE). */
typedef struct {
    uint32_t hidden, inner, heads, kv_heads, head_dim, layers, capacity;
    float eps, rope_theta, residual_scale;
    uint32_t rope;
    const double *rope_factors;
} tg_shape;

/* Shape::weight_bytes / cache_bytes (decode.rs:127-141) at `bytes_per_weight` (2 for f16/bf16).
 * cache_bytes counts positions 0 .. position in whole chunks of 32, at most the capacity, as the
 * reference does; the kernels here read position + 1 of them. */
uint64_t tg_shape_weight_bytes(const tg_shape *s, uint32_t bytes_per_weight);
uint64_t tg_shape_cache_bytes(const tg_shape *s, uint32_t position, uint32_t bytes_per_value);
/* Shape::rope_tables (decode.rs:143-168): [capacity][head_dim/2] each, computed in f32. */
int tg_shape_rope_tables(const tg_shape *s, float *cos_out, float *sin_out);

/* decode.rs:230-235 `Row`: a position of a cache slot, or spare (position = TG_SPARE). */
#define TG_SPARE 0xffffffffu
typedef struct {
    uint32_t position, slot;
} tg_row;

/* Batch::placement (decode.rs:198-227): the words for `n_rows` rows of a batch of `slots` slots
 * (positions, then slots when slots > 1; spare rows TG_SPARE). Refuses two rows in one slot and
 * places past the capacity or slots (TG_ESHAPE). `words` holds 2 n_rows. */
int tg_batch_placement(uint32_t n_rows, uint32_t slots, const tg_row *rows, uint32_t capacity,
                       uint32_t *words, uint32_t *n_words);

/* Decoder::with_batch (decode.rs:790-806): the decode step of `s` for a batch of `rows` rows
 * in a cache of `slots` slots, recorded once, with zero weights until loaded. The step is recorded
 * for each of the generator's row buckets (each power of two below `rows`, then `rows`,
 * crates/graph/src/generator.rs:115-123) over the same buffers. */
int tg_decoder_create(tg_ctx *ctx, const tg_shape *s, uint32_t rows, uint32_t slots,
                      tg_dtype dtype, int timed, tg_decoder **out);
int tg_decoder_destroy(tg_decoder *d);
/* Decoder::load (decode.rs:808-820, load_stack :740-776): one weight by its upstream name
 * ("layers.{l}.self_attn.{q,k,v,o}_proj.weight", "layers.{l}.mlp.{gate,up,down}_proj.weight",
 * "layers.{l}.{input,post_attention}_layernorm.weight", "norm.weight"), from host f32
 * (src_dtype TG_F32) or bf16 bits (TG_BF16), converted to the decoder's dtype (RNE). q/k/v and
 * gate/up are joined along their rows as load_stack joins them. */
int tg_decoder_load(tg_decoder *d, const char *name, const void *src, uint64_t count,
                    tg_dtype src_dtype);
/* Decoder::step_rows (decode.rs:849-853): x [rows][hidden] f32 in, out [rows][hidden] f32 out;
 * a spare row's output is meaningless. */
int tg_decoder_step_rows(tg_decoder *d, const tg_row *rows, const float *x, float *out);
/* Decoder::set_rows / start / output (decode.rs:857-872), for callers that overlap host work. */
int tg_decoder_set_rows(tg_decoder *d, const tg_row *rows, const float *x);
/* A step of the first n (1 <= n <= rows) rows, run by the smallest row bucket that holds them (the
 * bucket's other rows spare), as the generator runs the rows under way (generator.rs:306-330).
 * x and out hold n rows. A row's result is the same bits whatever n and bucket it runs in. */
int tg_decoder_set_rows_n(tg_decoder *d, uint32_t n, const tg_row *rows, const float *x);
int tg_decoder_step_rows_n(tg_decoder *d, uint32_t n, const tg_row *rows, const float *x,
                           float *out);
int tg_decoder_start(tg_decoder *d);
int tg_decoder_wait(tg_decoder *d, uint64_t timeout_ns);
int tg_decoder_output(tg_decoder *d, float *out);
/* Device-resident step for callers whose inputs are already on the GPU: placement words (as
 * tg_batch_placement gives) from the host, x and out device pointers of [rows][hidden] f32. */
int tg_decoder_step_device(tg_decoder *d, const uint32_t *words, const float *x_dev,
                           float *out_dev);
/* Decoder::timings: the last step's GPU time, and per dispatch when created timed. */
int tg_decoder_elapsed_ns(tg_decoder *d, double *ns);
int tg_decoder_timings(tg_decoder *d, double *ns, size_t n, size_t *n_dispatches);
/* The recorded dispatches' count and labels (decode.rs:935-951: 6 per layer and the final norm;
 * one, "decode_step", when the step is the persistent launch). */
int tg_decoder_dispatch_label(tg_decoder *d, size_t i, char *label, size_t label_bytes);
/* Copies positions [first, first+count) of a slot's keys (kind 0) or values (1) of a layer to the
 * host as f32 [kv_heads][count][head_dim]. */
int tg_decoder_read_cache(tg_decoder *d, uint32_t layer, uint32_t slot, uint32_t kind,
                          uint32_t first, uint32_t count, float *out);
/* Recording::copy_out / copy_in of KV ranges (crates/graph/src/step.rs:295-339,
 * crates/graph/src/prompt.rs:587-633): moves positions [0, count) of slot `from` to slot `to`
 * in every layer, on the GPU. */
int tg_decoder_copy_slot(tg_decoder *d, uint32_t from, uint32_t to, uint32_t count);
/* Recording::copy_out / copy_in of a prefix's keys and values (crates/graph/src/prompt.rs:587-633,
 * the prompt cache's kept prefix): positions [0, count) of `slot` in every layer, to or from
 * `m` at `offset`, laid out [layers][k, v][kv_heads][count][head_dim] in the decoder's storage
 * type; tg_decoder_prefix_bytes gives the size. Ordered on the context's stream with the steps
 * and prefills around it. */
uint64_t tg_decoder_prefix_bytes(const tg_decoder *d, uint32_t count);
int tg_decoder_copy_out(tg_decoder *d, uint32_t slot, uint32_t count, tg_mem *m, uint64_t offset);
int tg_decoder_copy_in(tg_decoder *d, uint32_t slot, uint32_t count, tg_mem *m, uint64_t offset);
/* Decoder::retuned (decode.rs:874-890): records the step again over the same weights and cache, as
 * one persistent launch (persistent != 0; batches of up to 2 rows) or as six kernels a layer, timed
 * per dispatch when `timed`. Both give the same results bit for bit. A new bf16 decoder of one or
 * two rows starts recorded as the persistent launch, any other as kernels. TG_ESHAPE when the
 * persistent step does not take the decoder (it is then left recorded as kernels). */
int tg_decoder_retune(tg_decoder *d, int persistent, int timed);
/* 1 when the decoder's step is the persistent launch. */
int tg_decoder_persistent(const tg_decoder *d);
/* How the decoder's projections run (bf16 decoders of 16 rows or more run on tcgen05 in every row
 * bucket): 1 as the prefill's tcgen05 GEMMs over bf16 activations (the step the prefill chain of
 * prefill.rs:318-411 over one-position runs, with the decode attention; the default where the
 * shape takes it), 2 as tcgen05 split-K clusters over f32 activations split into bf16 hi and lo,
 * 0 as GEMVs on the CUDA cores. */
int tg_decoder_tensor(const tg_decoder *d);
/* Records the step again with its projections as `tensor` names (1: tcgen05 GEMMs, falling back to
 * split-K clusters where the GEMMs do not take the shape; 2: split-K clusters; 0: GEMVs), over the
 * same weights and cache. The families give results within their roundings of each other, not the
 * same bits: a decoder that checks a request against its run beside others uses the family those
 * ran in. TG_ESHAPE when the family asked for does not take the decoder's dtype or shape. */
int tg_decoder_set_tensor(tg_decoder *d, int tensor);
/* The weight bytes one step reads at this dtype (Shape::weight_bytes at its element size). */
uint64_t tg_decoder_weight_bytes(const tg_decoder *d);

/* Prefill::new (prefill.rs:431-461): programs over the decoder's weights, tables and cache for up
 * to `max_rows` rows at once. */
int tg_prefill_create(tg_decoder *d, uint32_t max_rows, int timed, tg_prefill **out);
int tg_prefill_destroy(tg_prefill *p);
/* Prefill::run (prefill.rs:473-503): x [len][hidden] f32 of positions start..start+len-1 into
 * `slot`, out [len][hidden] f32 after the final norm. Longer runs than max_rows go in pieces. */
int tg_prefill_run(tg_prefill *p, uint32_t start, uint32_t slot, const float *x, uint32_t len,
                   float *out);
/* Several runs at once, each in its own slot, rows packed in order (each run's rows start on a
 * multiple of 128 inside the launch): the batched prefill of BASELINE config 4. */
typedef struct {
    uint32_t start, len, slot;
} tg_run;
int tg_prefill_run_batch(tg_prefill *p, const tg_run *runs, uint32_t n_runs, const float *x,
                         float *out);
/* Device-resident variant: x_dev/out_dev are device pointers [sum len][hidden] f32. */
int tg_prefill_run_batch_device(tg_prefill *p, const tg_run *runs, uint32_t n_runs,
                                const float *x_dev, float *out_dev);
int tg_prefill_elapsed_ns(tg_prefill *p, double *ns);
int tg_prefill_timings(tg_prefill *p, double *ns, size_t n, size_t *n_dispatches);
int tg_prefill_dispatch_label(tg_prefill *p, size_t i, char *label, size_t label_bytes);
uint32_t tg_prefill_max_rows(const tg_prefill *p);

/* ---- Continuous batching (crates/graph/src/generator.rs:99-352) ---------------------------------
 * Requests hold the decoder's slots; each step packs the requests under way into rows (in slot
 * order) and runs the smallest row bucket that holds them; requests are admitted between steps by
 * a prefill into their slots. On the backbone alone a request's next input is its last output
 * (the prompt's last, then each step's), fed back on the GPU. The decoder needs a row per slot. */
typedef struct tg_server tg_server;
typedef struct {
    uint32_t slot;  /* the slot it holds (a request there before is ended) */
    uint32_t len;   /* prompt positions, prefilled at start..len-1 */
    uint32_t steps; /* decode steps after it, at positions len..len+steps-1 */
    uint32_t start; /* positions already in the slot (a kept prefix copied in); 0 for none */
} tg_request;
int tg_server_create(tg_decoder *d, tg_prefill *p, tg_server **out);
int tg_server_destroy(tg_server *s);
/* Generator::start (generator.rs:189-262): runs the requests' prompts, x [sum (len - start)]
 * [hidden] f32 in request order (each request's rows from its `start`), into their slots (as few
 * prefill launches as max_rows allows). Refuses a slot twice, no positions to run or no steps,
 * and len + steps past the capacity (TG_ESHAPE). */
int tg_server_start(tg_server *s, const tg_request *reqs, uint32_t n, const float *x);
/* Generator::step (generator.rs:295-352): one decode step of every request under way. x: NULL to
 * feed each request's last output back (on the GPU), else [n][hidden] f32 inputs in slot order.
 * Writes the number of rows run, their slots (if `slots`), and their outputs [n][hidden] (if
 * `out`: the step is then waited for; else it is only enqueued and later steps queue behind it). A
 * request whose steps have all run stays held, no longer under way, until finished. */
int tg_server_step(tg_server *s, const float *x, uint32_t *n_rows, uint32_t *slots, float *out);
/* The slots under way (ascending; `slots` may be NULL to count them). */
int tg_server_under_way(const tg_server *s, uint32_t *slots, uint32_t *n);
int tg_server_request(const tg_server *s, uint32_t slot, uint32_t *held, uint32_t *position,
                      uint32_t *left);
/* Generator::finish: frees the slot. */
int tg_server_finish(tg_server *s, uint32_t slot);
/* The slot's last output (its next input), [hidden] f32. */
int tg_server_last_output(tg_server *s, uint32_t slot, float *out);
/* Waits for every step enqueued (TG_ETIMEOUT after timeout_ns; 0: no limit). */
int tg_server_sync(tg_server *s, uint64_t timeout_ns);

/* ---- The local stacks: VoxCPM2's patch sampler and local encoder (crates/graph/src/local) ------
 * Each is a bidirectional MiniCPM-4 stack over the few tokens of one patch per sequence (f16
 * weights and activations, f32 sums), recorded once as one program (a CUDA graph) and run whole.
 * A row's results are the same bits whatever rows run beside it. */
typedef struct tg_sampler tg_sampler;
typedef struct tg_encoder tg_encoder;

/* local::Tuning's cuts that decide the order of the sums (local/mod.rs:187-214): the column parts
 * of the q/k/v, output and down projections' sums, each part a multiple of 64 columns (0: the
 * default, 4, 8 and 8, or the most the width allows). */
typedef struct {
    uint32_t qkv_parts, o_parts, down_parts;
} tg_local_tuning;

/* sampler_graph / Sampler::new (local/dit.rs:112-281): the DiT's stack `stack` (its capacity is
 * set here: 2 + 1 + 2 patch_size tokens a sequence; `rope_factors` as the base LM's), patches of
 * `patch_size` frames of `feat_dim` channels, `timesteps` Euler steps, `rows` rows (two
 * sequences each). Every weight zero until loaded. Refuses shapes the kernels do not take
 * (TG_ESHAPE), as the reference's checks (local/mod.rs:366-385, dit.rs:196-212). */
int tg_sampler_create(tg_ctx *ctx, const tg_shape *stack, uint32_t feat_dim, uint32_t patch_size,
                      uint32_t timesteps, uint32_t rows, const tg_local_tuning *tuning, int timed,
                      tg_sampler **out);
int tg_sampler_destroy(tg_sampler *s);
/* load_sampler (local/dit.rs:325-370): one tensor by its upstream name, from f32, bf16 or f16
 * values, rounded to f16: "feat_decoder.estimator.decoder.layers.{l}.self_attn.{q,k,v,o}_proj.weight",
 * "...layers.{l}.mlp.{gate,up,down}_proj.weight", "...layers.{l}.{input,post_attention}_layernorm.weight",
 * "feat_decoder.estimator.decoder.norm.weight", "feat_decoder.estimator.{in,cond,out}_proj.{weight,bias}",
 * "feat_decoder.estimator.{time,delta_time}_mlp.linear_{1,2}.{weight,bias}". The steps' time tokens
 * are computed from the two MLPs on the host in f64 (dit.rs:386-422) before the next sample. */
int tg_sampler_load(tg_sampler *s, const char *name, const void *src, uint64_t count, tg_dtype src_dtype);
/* Sampler::sample (local/dit.rs:298-313): mu f16 bits [rows][2][hidden], cond and noise f32
 * [rows][feat_dim][patch_size], sampling f32 [rows][2] (temperature, guidance scale) -> patch f32
 * [rows][feat_dim][patch_size]. TG_ENOTFINITE, with every patch written, when a row's patch came
 * out NaN or infinite (the check crates/graph/src/generator.rs:418-421 makes on each sampled
 * patch, Error::NotFinite); the device form leaves that check to its caller. */
int tg_sampler_sample(tg_sampler *s, const uint16_t *mu, const float *cond, const float *noise,
                      const float *sampling, float *patch);
/* The same from device pointers, enqueued on the context's stream without waiting. */
int tg_sampler_sample_device(tg_sampler *s, const void *mu, const float *cond, const float *noise,
                             const float *sampling, float *patch);
int tg_sampler_wait(tg_sampler *s, uint64_t timeout_ns);
/* The time and step length of each step the DiT runs at (euler_steps). */
int tg_sampler_steps(const tg_sampler *s, float *t, float *dt, size_t n, size_t *count);
int tg_sampler_elapsed_ns(tg_sampler *s, double *ns);
int tg_sampler_timings(tg_sampler *s, double *ns, size_t n, size_t *n_dispatches);
int tg_sampler_dispatch_label(tg_sampler *s, size_t i, char *label, size_t label_bytes);
/* Bytes of weights one run of the DiT reads (f16). */
uint64_t tg_sampler_weight_bytes(const tg_sampler *s);

/* dit.rs:39-81 as functions: the timesteps + 1 times the sampler steps through, and the steps
 * (time, length) the DiT runs at (count written to *count; n the room in t and dt). */
int tg_cfm_schedule(uint32_t timesteps, float *out);
int tg_cfm_euler_steps(uint32_t timesteps, float *t, float *dt, size_t n, size_t *count);

/* encoder_graph / Encoder (local/encoder.rs:41-124, :160-215): sequences of 1 + patch_size tokens,
 * `rows` rows. Names: "feat_encoder.encoder.layers.{l}...", "feat_encoder.encoder.norm.weight",
 * "feat_encoder.special_token", "feat_encoder.in_proj.{weight,bias}". */
int tg_encoder_create(tg_ctx *ctx, const tg_shape *stack, uint32_t feat_dim, uint32_t patch_size,
                      uint32_t rows, const tg_local_tuning *tuning, int timed, tg_encoder **out);
int tg_encoder_destroy(tg_encoder *e);
int tg_encoder_load(tg_encoder *e, const char *name, const void *src, uint64_t count, tg_dtype src_dtype);
/* Encoder::encode: patches f32 [rows][feat_dim][patch_size] -> out f16 bits [rows][hidden]. */
int tg_encoder_encode(tg_encoder *e, const float *patches, uint16_t *out);
int tg_encoder_encode_device(tg_encoder *e, const float *patches, void *out);
int tg_encoder_wait(tg_encoder *e, uint64_t timeout_ns);
int tg_encoder_elapsed_ns(tg_encoder *e, double *ns);
int tg_encoder_timings(tg_encoder *e, double *ns, size_t n, size_t *n_dispatches);
int tg_encoder_dispatch_label(tg_encoder *e, size_t i, char *label, size_t label_bytes);
uint64_t tg_encoder_weight_bytes(const tg_encoder *e);

/* ---- Decode attention without allocation -------------------------------------------------------
 * No counterpart in tgtts-v4. For callers that cannot allocate device memory themselves or let a
 * library do it (an engine that owns every byte of HBM through its own pool, or code recording a
 * CUDA graph, where an allocation would break the capture): attention_split + attention_combine of
 * the decode step (TG_KERNEL_ATTENTION_SPLIT / _COMBINE, same params and results) with their
 * partial sums kept in a fixed array inside the library, TG_NOALLOC_SCRATCH_BYTES per device,
 * instead of a buffer the caller passes. It allocates nothing. The caller passes q (f32
 * [rows][heads][hd]), the caches (storage type), the placement words and out (f32
 * [rows][heads hd]), all device pointers, and a cudaStream_t of the current device (NULL: the
 * legacy stream; a stream of another device is refused with TG_EINVAL); the work is enqueued
 * there and not waited for. Refuses (TG_ESHAPE) a shape with no heads or whose partials,
 * rows x heads x ceil(capacity/64) x (head_dim + 2) f32, do not fit. The first call on a device looks the
 * array up for that device (and may load the library's module there): make it before any stream
 * capture. All calls on a device share the array, so calls that overlap on the GPU race. */
#define TG_NOALLOC_SCRATCH_BYTES (4u << 20)
int tg_attention_decode_noalloc(const tg_params *p, const float *q, const void *k_cache,
                                const void *v_cache, const uint32_t *at, float *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif
