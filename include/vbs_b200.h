/* vbs_b200.h -- C ABI of libvbs_b200.so, the B200 (sm_100a) CUDA backend for
 * Verum's per-token decode step.
 *
 * Two layers:
 *
 * 1. The drop-in boundary. `g_vbs_cuda_backend` and `vbs_cuda_last_error`
 *    are the two symbols the reference engine binds for its CUDA backend
 *    (declared at include/vbs_backend.h:101 and
 *    include/vbs_backend_select.h:40 of the reference; referenced from
 *    src/vbs_backend_select.c:20,35 and src/vbs_profiler.c:152-170). A
 *    maintainer removes src/vbs_backend_cuda.c from the reference build and
 *    links this library instead; nothing above the ops table changes.
 *    The types below are layout-identical restatements of the reference's
 *    vbs_device_t / vbs_buffer_t / vbs_arg_t / vbs_prim_pipeline_t /
 *    vbs_backend_ops_t (include/vbs_backend.h:13-99) and of the enums they
 *    use (include/vbs_gguf.h:13-48, include/vbs_graph.h:12-24). When the
 *    reference headers are included first, their definitions are used and
 *    these are skipped.
 *
 * 2. Extension entry points (vbs_cu_*), plain pointers and sizes. They
 *    serve what the ops table cannot express: the fused decode program
 *    (the reference's JIT forward_token / verum_forward,
 *    src/vbs_specializer.c:231-359, replayed as one CUDA graph), batched
 *    matvec and attention, tensor parallelism, and seeded weight synthesis
 *    for benchmarks. Each cites the reference interface it replaces.
 *
 * Errors: every call returns 0 / a non-NULL handle on success. The first
 * error is latched (sticky) and reported by vbs_cuda_last_error(); the ops
 * table's void and dropped-bool paths surface it at the next copy_to_host,
 * which then returns false (the bridge ignores dispatch results,
 * src/vbs_specializer_bridge.c:83-90 of the reference).
 */
#ifndef VBS_B200_H
#define VBS_B200_H

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Symbols of libvbs_b200.so (built with hidden default visibility). */
#if defined(__GNUC__)
#define VBS_API __attribute__((visibility("default")))
#else
#define VBS_API
#endif

#ifndef VBS_BACKEND_H
/* ---- restated reference types (layout must not change) ---- */
typedef enum {
    VBS_GGML_TYPE_F32 = 0, VBS_GGML_TYPE_F16 = 1, VBS_GGML_TYPE_Q4_0 = 2, VBS_GGML_TYPE_Q4_1 = 3,
    VBS_GGML_TYPE_Q5_0 = 6, VBS_GGML_TYPE_Q5_1 = 7, VBS_GGML_TYPE_Q8_0 = 8, VBS_GGML_TYPE_Q8_1 = 9,
    VBS_GGML_TYPE_Q2_K = 10, VBS_GGML_TYPE_Q3_K = 11, VBS_GGML_TYPE_Q4_K = 12, VBS_GGML_TYPE_Q5_K = 13,
    VBS_GGML_TYPE_Q6_K = 14, VBS_GGML_TYPE_Q8_K = 15, VBS_GGML_TYPE_BF16 = 30, VBS_GGML_TYPE_LNS8 = 40
} vbs_ggml_type_t;

typedef enum {
    VBS_OP_EMBEDDING, VBS_OP_LINEAR, VBS_OP_NORMALIZE, VBS_OP_ATTENTION, VBS_OP_ROTARY,
    VBS_OP_ACTIVATION, VBS_OP_ELEMENTWISE, VBS_OP_STATE_SPACE, VBS_OP_CONVOLUTION,
    VBS_OP_CACHE, VBS_OP_PROJECTION
} vbs_op_kind_t;

typedef enum {
    VBS_BACKEND_METAL, VBS_BACKEND_CUDA, VBS_BACKEND_HIP, VBS_BACKEND_CPU, VBS_BACKEND_VULKAN
} vbs_backend_type_t;

typedef struct vbs_device {
    char name[128];
    vbs_backend_type_t type;
    uint64_t max_working_set_bytes;
    uint64_t max_buffer_bytes;
    void *internal_handle;
} vbs_device_t;

typedef struct vbs_buffer {
    void *internal_handle;      /* device address */
    void *host_ptr;             /* staging mirror (see alloc_buffer) */
    size_t size;
    vbs_device_t *device;
} vbs_buffer_t;

typedef enum { VBS_ARG_BUFFER = 0, VBS_ARG_SCALAR = 1 } vbs_arg_tag_t;

typedef struct {
    vbs_arg_tag_t tag;
    const void *value;          /* BUFFER: device address; SCALAR: pointer to the value */
    size_t size;
} vbs_arg_t;

typedef struct {
    void *native;
    vbs_op_kind_t kind;
} vbs_prim_pipeline_t;

typedef struct vbs_backend_ops {
    bool (*init)(void);
    size_t (*get_device_count)(void);
    vbs_device_t *(*get_device)(size_t index);
    vbs_buffer_t *(*alloc_buffer)(vbs_device_t *dev, size_t bytes, bool shared);
    void (*free_buffer)(vbs_buffer_t *buf);
    bool (*copy_to_device)(vbs_buffer_t *dst, const void *src, size_t bytes);
    bool (*copy_to_host)(void *dst, const vbs_buffer_t *src, size_t bytes);
    void *(*compile_linear_pipeline)(vbs_device_t *dev, vbs_ggml_type_t type, char *err_buf, size_t err_cap);
    void *(*compile_embed_pipeline)(vbs_device_t *dev, vbs_ggml_type_t type, char *err_buf, size_t err_cap);
    void *(*compile_primitive_pipeline)(vbs_device_t *dev, vbs_op_kind_t kind, char *err_buf, size_t err_cap);
    bool (*dispatch_linear_tile)(vbs_device_t *dev, void *pipeline, vbs_buffer_t *weight_private,
                                 vbs_buffer_t *weight_stage, size_t copied_bytes, vbs_buffer_t *input,
                                 vbs_buffer_t *output, uint32_t cols, uint32_t rows, uint32_t col_offset,
                                 uint32_t row_offset, bool accumulate);
    bool (*dispatch_primitive)(vbs_device_t *dev, void *pipeline, const vbs_arg_t *args, size_t n_args,
                               size_t grid_x, size_t block_x);
    void (*synchronize_device)(vbs_device_t *dev);
    bool (*launch_persistent_kernel)(vbs_device_t *dev, void *pipeline, vbs_buffer_t *control_buffer);
} vbs_backend_ops_t;
#endif /* VBS_BACKEND_H */

#ifndef VBS_ENGINE_H
/* ---- restated engine control block (include/vbs_engine.h:22-40 of the
 * reference; layout must not change): the device-resident state of a
 * generation run, read and written by launch_persistent_kernel. ---- */
typedef enum {
    VBS_PGAE_IDLE = 0, VBS_PGAE_PREFILL = 1, VBS_PGAE_GENERATE = 2, VBS_PGAE_EXIT = 3
} vbs_pgae_state_t;
#define VBS_PGAE_EOS_NONE ((uint32_t)0xFFFFFFFFu)
typedef struct {
    volatile uint32_t state;
    volatile uint32_t current_token;
    volatile uint32_t position;
    volatile uint32_t max_tokens;
    volatile uint32_t vocab_size;
    volatile uint32_t eos_token_id;
    uint64_t generated_tokens_dev;
    uint64_t logits_dev;
} vbs_gpu_control_t;
#endif /* VBS_ENGINE_H */

/* ================================================================== */
/* 1. Drop-in boundary                                                 */
/* ================================================================== */

/* Replaces the table defined at src/vbs_backend_cuda.c:313-327 (declared
 * include/vbs_backend.h:101). Semantics per entry:
 *  init            idempotent; false when no usable sm_100 device exists.
 *  get_device      name, type=CUDA, max_working_set_bytes = device memory,
 *                  max_buffer_bytes = free memory at init.
 *  alloc_buffer    device allocation; host_ptr is pinned host memory for
 *                  shared=true, a pageable mirror for device buffers up to
 *                  64 MiB (the reference self-test stages through it,
 *                  src/vbs_backend_test.c:863), NULL above.
 *  copy_*          synchronous; copy_to_host returns false once an error
 *                  has been latched.
 *  compile_linear_pipeline  F32, F16, Q4_0, Q4_1, Q8_0, Q4_K, Q6_K and the
 *                  reference's LNS8; refuses every other type with a message.
 *  compile_embed_pipeline   the same types without LNS8 (no embedding
 *                  kernel in the reference either).
 *  compile_primitive_pipeline  EMBEDDING, NORMALIZE, ROTARY, CACHE,
 *                  ATTENTION, ACTIVATION, ELEMENTWISE.
 *  dispatch_linear_tile  both calling conventions: resident weights
 *                  (weight_stage == NULL, src/vbs_specializer_bridge.c:89)
 *                  and staged tiles read from weight_stage->host_ptr with
 *                  col/row offsets and accumulation
 *                  (src/vbs_slice_executor.c:84-96).
 *  dispatch_primitive  canonical bridge argument order
 *                  (include/vbs_specializer_bridge.h:44-53); grid/block
 *                  hints are ignored, the backend picks its own launch.
 *  launch_persistent_kernel  (include/vbs_backend.h:94-98, NULL in every
 *                  reference backend) device-driven greedy generation:
 *                  `pipeline` is a vbs_cu_decoder_t of a model on `dev`,
 *                  `control_buffer` a device buffer holding a
 *                  vbs_gpu_control_t; runs vbs_cu_decoder_run_control. */
extern VBS_API const vbs_backend_ops_t g_vbs_cuda_backend;

/* Last error message, "ok" when none (include/vbs_backend_select.h:40). */
VBS_API const char *vbs_cuda_last_error(void);

/* ================================================================== */
/* 2. Extension entry points                                           */
/* ================================================================== */

/* Sticky error state: 0 when no error has been latched. */
VBS_API int vbs_cu_status(void);
VBS_API void vbs_cu_clear_error(void);

/* Build/feature string, e.g. "vbs_b200 sm_100a tma-bulk mma-s8 pdl". */
VBS_API const char *vbs_cu_version(void);

/* Number of kernels this library has launched since load (all entry
 * points, captured graph launches counted per contained kernel). */
VBS_API uint64_t vbs_cu_kernel_launches(void);

/* Bit-exact block dequantization of n_elems elements (a whole number of
 * blocks) on the device. Replaces nothing in the reference engine; it is
 * the device twin of vbs_dequant_block (src/vbs_dequant.c:339-356) used to
 * prove the kernels' decode tables. `stream` is a cudaStream_t (NULL: the
 * legacy default stream). */
VBS_API int vbs_cu_dequant(int type, const void *w, float *out, uint64_t n_elems, void *stream);

/* Quantized matvec y[b][r] (+)= sum_c dequant(W)[r][c] * x[b][c], for
 * b < batch (x: batch x cols floats, y: batch x rows floats, device
 * pointers). The device twin of dispatch_linear_tile with offsets 0
 * (src/vbs_specializer_bridge.c:83-90), extended with the batch dimension
 * the engine lacks (batched decode, B = 8 / 16). flags: bit 0 accumulate
 * into y, bit 1 force the portable (non-TMA) kernel. */
#define VBS_CU_MV_ACCUMULATE 1u
#define VBS_CU_MV_PORTABLE   2u
VBS_API int vbs_cu_matvec(int type, const void *w, const float *x, float *y, uint32_t rows, uint32_t cols,
                  uint32_t batch, uint32_t flags, void *stream);

/* The FFN's first half as one kernel: h[r] = silu(g_r) * u_r with
 * g = W_gate xn, u = W_up xn and xn = RMSNorm(x) * norm_w (norm_w NULL: xn
 * = x). Replaces the bridge sequence vram(gate), vram(up), silu
 * (src/vbs_specializer.c:316-325 of the reference). Q4_K, Q6_K and Q8_0
 * weights take the fused TMA kernel; other types run norm, two matvecs
 * and the SiLU as separate kernels. */
VBS_API int vbs_cu_ffn_gate_up(int type, const void *w_gate, const void *w_up, const float *x, const float *norm_w,
                               float eps, float *h, uint32_t rows, uint32_t cols, void *stream);

/* GQA decode attention over the engine's fp16 cache layout
 * [layer][max_ctx][n_kv_heads*head_dim] (src/vbs_engine.c:113-148),
 * split-KV flash decoding. Same arguments as the ATTENTION primitive
 * (include/vbs_specializer_bridge.h:50-51) plus a batch: sequence b reads
 * q + b*nqh*hd, caches + b*kv_batch_stride elements, writes out +
 * b*nqh*hd. seq_len positions 0..seq_len-1 are attended. */
VBS_API int vbs_cu_attention(const float *q, const uint16_t *kc, const uint16_t *vc, float *out,
                     uint32_t seq_len, uint32_t layer, uint32_t max_ctx, uint32_t n_q_heads,
                     uint32_t n_kv_heads, uint32_t head_dim, float scale, uint32_t batch,
                     uint64_t kv_batch_stride, void *stream);

/* vbs_cu_attention without any device allocation. No reference counterpart:
 * an addition of this library for callers that cannot allocate device memory
 * on the call path, e.g. code running under a fixed device-memory budget, or
 * code where a cudaMalloc (which can fail, and can synchronize the device) is
 * not acceptable in the middle of a decode loop. vbs_cu_attention grows a
 * workspace on demand; this entry point uses a fixed scratch of 2 MiB per
 * device in the library's static device memory instead.
 *  - Limit: the split partials must fit the scratch. The number of splits is
 *    lowered until they do; at one split the result goes straight to `out`
 *    and no scratch is used, so every valid call runs. Calls that need fewer
 *    splits than vbs_cu_attention picks (large batch x n_kv_heads at long
 *    contexts) are slower, not different beyond float rounding.
 *  - Setup: the first call on a device initialises the backend for that
 *    device if needed and looks up the scratch address (cudaGetSymbolAddress
 *    with that device current); make that first call before any stream
 *    capture. Later calls allocate nothing.
 *  - State: the scratch's merge counters are zero when the library loads and
 *    every call leaves them at zero again; nothing else needs an initial
 *    value.
 *  - Concurrency: all calls on a device share the one scratch. Calls that
 *    can overlap in time (different streams, or different host threads)
 *    race on it and must be serialized by the caller.
 * Arguments, layout and results as vbs_cu_attention. */
VBS_API int vbs_cu_attention_static(const float *q, const uint16_t *kc, const uint16_t *vc, float *out,
                                    uint32_t seq_len, uint32_t layer, uint32_t max_ctx, uint32_t n_q_heads,
                                    uint32_t n_kv_heads, uint32_t head_dim, float scale, uint32_t batch,
                                    uint64_t kv_batch_stride, void *stream);

/* Seeded synthetic weights: the [rows x cols] tile at (row0, col0) of a
 * tensor with full_cols columns, element (r, c) drawn from the Irwin-Hall
 * (n = 4) normal approximation of stream `seed` at index r*full_cols + c,
 * times `scale`, then quantized to `type` (F32, F16, Q8_0, Q4_K, Q6_K).
 * Bit-identical to oracle/vbs_oracle.c:orc_synth_tensor. No reference
 * counterpart (the reference has no K-quant quantizer). */
VBS_API int vbs_cu_synth(int type, void *dst, uint64_t rows, uint64_t cols, uint64_t row0, uint64_t col0,
                 uint64_t full_cols, uint64_t seed, float scale, void *stream);

/* Copies byte ranges of a file into device memory: range i, the bytes
 * [offsets[i], offsets[i] + sizes[i]) of the file at `path`, lands at the
 * device pointer dst[i] (on the current device). Replaces the reference
 * loader's host mirror plus one synchronous copy_to_device per tensor
 * (src/vbs_fabric.c:81-94, src/vbs_backend_cuda.c:148). n_threads reader
 * threads (0: 4, at most 32) pread chunks of chunk_bytes (0: 16 MiB;
 * clamped to 1 MiB..1 GiB) into two pinned staging buffers each and copy
 * them with cudaMemcpyAsync on their own streams, so reads and copies
 * overlap. Returns 0 once every byte has landed (all its streams
 * synchronized); -1, with the error latched, for a range outside the file,
 * a missing destination, a short read or a CUDA error. Device work the
 * caller queued before the call (e.g. clearing dst) must be complete. */
VBS_API int vbs_cu_upload_file(const char *path, size_t n, const uint64_t *offsets, const uint64_t *sizes,
                               void *const *dst, uint32_t n_threads, uint64_t chunk_bytes);

/* ---- decode program (the JIT forward pass, src/vbs_specializer.c:231-372) ---- */

/* A llama-style model resident on the device. Per-layer fields are host
 * arrays of n_layers device pointers / types. Under tensor parallelism a
 * rank's descriptor holds its shard: n_heads / n_kv_heads / ffn / vocab
 * are the rank-local counts, dim is the full model width. */
typedef struct {
    uint32_t n_layers, dim, n_heads, n_kv_heads, head_dim, ffn, vocab;
    float eps, theta;
    int embd_type, out_type;
    const void *embd;               /* [vocab_full x dim] packed */
    const void *out;                /* [vocab x dim] packed (rank-local rows) */
    const float *out_norm;
    const float *const *attn_norm, *const *ffn_norm;
    const void *const *wq, *const *wk, *const *wv, *const *wo;
    const void *const *wgate, *const *wup, *const *wdown;
    const int *tq, *tk, *tv, *to, *tgate, *tup, *tdown;
    uint32_t vocab_full;            /* 0: same as vocab */
    uint32_t vocab_offset;          /* first output row this rank owns */
} vbs_cu_model_t;

#define VBS_CU_DEC_STRICT   1u   /* vbs_cpu arithmetic (src/vbs_cpu.c:572-639), fp32 KV */
#define VBS_CU_DEC_NO_GRAPH 2u   /* launch kernel by kernel instead of one CUDA graph */
#define VBS_CU_DEC_NO_PDL   4u   /* no programmatic dependent launch between kernels */
#define VBS_CU_DEC_NO_PERSIST 8u /* per-op kernels instead of the persistent one-launch step */
#define VBS_CU_DEC_TP_NCCL 16u   /* tensor parallelism: per-layer sums with ncclAllReduce instead of peer memory */
#define VBS_CU_DEC_WORDS 32u     /* one GPU: run the step kernel's tensor-parallel instance (exchange words in place of
                                    the grid barriers after o_proj and down) over a local area. Same results; slower
                                    on one GPU (every thread polls its words), there to test that instance. */
#define VBS_CU_DEC_STREAM 64u    /* slice streaming (the reference's slice executor, src/vbs_slice_executor.c:8-107,
                                    for models above device memory): the per-layer matrices wq..wdown of the model
                                    description are PINNED HOST pointers (cudaHostAlloc / cudaHostRegister), every
                                    layer with the first layer's types; embedding, output matrix and norm weights stay
                                    on the device. Two device slots of one layer each; every step copies each layer
                                    in (one cudaMemcpyAsync per matrix, its own stream) while the previous layer's
                                    kernels run. Per-op kernels, one GPU, no strict mode; same results as the same
                                    model resident with VBS_CU_DEC_NO_PERSIST. */

typedef struct vbs_cu_decoder vbs_cu_decoder_t;

/* Allocates the activations, the KV cache (fp16 [layer][kv head][max_ctx]
 * [head_dim]; fp32 [layer][max_ctx][kv_dim] under STRICT) and the control
 * block on the current device. Synchronizes the device first, so weights
 * still being written by work on other streams are complete before the
 * decoder's own stream reads them. Every later vbs_cu_decoder_* call makes
 * the decoder's device current for its duration and leaves the caller's
 * current device as it found it.
 * Steps run as one persistent kernel launch when the model fits that
 * kernel's plan and its repacked weight copy fits in device memory with
 * 1 GiB to spare. The plan wants one weight type per op (Q4_K, Q6_K or
 * Q8_0), head_dim 64 or 128, 1 to 8 query heads per KV head and a width of
 * at most 16384 (4096 under tensor parallelism). Otherwise steps run as
 * per-op kernels. vbs_cu_decoder_kernels_per_step() returns 1 for the
 * persistent kernel. */
VBS_API vbs_cu_decoder_t *vbs_cu_decoder_create(const vbs_cu_model_t *m, uint32_t max_ctx, uint32_t flags,
                                        char *err, size_t err_cap);
VBS_API void vbs_cu_decoder_destroy(vbs_cu_decoder_t *d);

/* Mirrors verum_forward (src/vbs_specializer.c:351-359): one decode step per
 * token at consecutive positions, then the logits of the last step are
 * copied to logits_out (host, vocab floats; NULL skips the readback). */
VBS_API int vbs_cu_decoder_forward(vbs_cu_decoder_t *d, const uint32_t *tokens, size_t n_tokens, float *logits_out);
/* Prompt tokens as context: their KV rows are computed and stored at
 * positions position()..position()+n-1, up to 512 tokens sharing one pass
 * over the weights (the tcgen05 GEMM; a last chunk of up to 8 tokens through
 * the batched matvec; causal split-KV attention), no logits. The
 * next vbs_cu_decoder_forward / generate continues at position()+n; feed
 * the prompt's last token through it to get its logits. The reference feeds
 * prompts one token at a time through forward_token (src/main.c:901-904);
 * the stored rows agree with that to the kernels' rounding. One GPU, not in
 * strict mode. 0, or -1 with the error latched. */
VBS_API int vbs_cu_decoder_prefill(vbs_cu_decoder_t *d, const uint32_t *tokens, size_t n_tokens);

/* Mirrors verum_reset_cache (src/vbs_specializer.c:370): position 0. */
VBS_API void vbs_cu_decoder_reset(vbs_cu_decoder_t *d);

/* Greedy decode with the argmax on the device (first maximum wins, as
 * src/vbs_cpu_main.c:78-80): feeds the prompt, then n_new tokens chosen
 * by argmax, each fed back without a host round trip. out_tokens receives
 * n_new ids. The engine-owned loop this replaces is
 * src/vbs_engine.c:240-327. */
VBS_API int vbs_cu_decoder_generate(vbs_cu_decoder_t *d, const uint32_t *prompt, size_t n_prompt, uint32_t n_new,
                            uint32_t *out_tokens);

/* Device-driven greedy generation, the engine's autonomy loop
 * (src/vbs_engine.c:240-327) with every decision on the device. `control`
 * is the device address of a vbs_gpu_control_t with state PREFILL or
 * GENERATE, current_token the next token to feed (the prompt's last, as the
 * reference's Phase 1 sets it), max_tokens >= 1, vocab_size the decoder's
 * vocabulary, eos_token_id (VBS_PGAE_EOS_NONE: none) and
 * generated_tokens_dev (max_tokens uint32 on the device); the decoder holds
 * the rest of the prompt as context. Each step feeds current_token at the
 * decoder's position; a one-thread kernel after it takes the step's argmax
 * (first maximum wins), stops on EOS (not stored) or when max_tokens tokens
 * are stored, else appends the token to generated_tokens_dev, sets
 * current_token and position (= tokens generated), exactly as the
 * reference's loop does; once stopped, state is EXIT and the steps still
 * queued do nothing. The host only enqueues steps and looks at the stop word
 * every 16 steps. logits_dev (when not 0) receives the last step's logits
 * (vocab_size floats). 0 on success; -1 with the error latched for a bad
 * control block or when max_tokens steps would exceed the KV capacity.
 * Tensor-parallel decoders are not supported (the engine binds one
 * device). */
VBS_API int vbs_cu_decoder_run_control(vbs_cu_decoder_t *d, void *control);

/* Bounded-wait test control (no reference counterpart). Every wait of the
 * persistent step kernel (mbarriers, grid barriers, exchange words,
 * attention counters) gives up after wait_ns of global time (1 ms .. 2 s;
 * 2 s by default), records DERR_TIMEOUT_* in the device error word and
 * unwinds every CTA; the next synchronising call reports it. drop_op (a step
 * op index: 5 * layer + {0 QKV, 1 ATTN, 2 O, 3 GU, 4 DOWN}, then 5 * layers
 * for the output; ~0u: none) makes CTA 0 withhold its arrival at that op's
 * grid barrier, so the other CTAs' waits run out as they would for a stalled
 * peer. The decoder launches its step directly afterwards (no graph). 0, or
 * -1 for a decoder without the persistent step kernel. */
VBS_API int vbs_cu_decoder_set_wait_test(vbs_cu_decoder_t *d, uint64_t wait_ns, uint32_t drop_op);

/* Enqueue n decode steps on the decoder's stream that feed each step's
 * argmax back as the next token (no host work between steps); returns
 * without synchronising. For timing loops. */
VBS_API int vbs_cu_decoder_enqueue_steps(vbs_cu_decoder_t *d, uint32_t n_steps);
VBS_API int vbs_cu_decoder_set_position(vbs_cu_decoder_t *d, uint32_t pos, uint32_t token);
VBS_API uint32_t vbs_cu_decoder_position(vbs_cu_decoder_t *d);
VBS_API void *vbs_cu_decoder_stream(vbs_cu_decoder_t *d);

/* ---- batched decode: B sequences in lockstep (no reference counterpart) ----
 * The reference's engine decodes one sequence (src/vbs_engine.c:240-327);
 * every step streams every weight for one token. This decoder steps B
 * sequences together, all at the same position, one token each per step,
 * with the per-op kernels: each weight is read once per step for B tokens
 * (the batched tensor-core matvec up to 8 sequences, the tcgen05 GEMM
 * above). Each sequence has its own fp16 KV cache, head-major
 * [layer][kv head][max_ctx][head_dim]; its logits equal a one-sequence
 * decoder fed the same tokens, to the kernels' rounding. One GPU; the
 * model description as for vbs_cu_decoder_create (vocab_full = vocab). */
typedef struct vbs_cu_batch_decoder vbs_cu_batch_decoder_t;
/* batch 1..64 sequences; allocates B KV caches of max_ctx positions and
 * copies [wq; wk; wv] and [wgate; wup] of every layer into one matrix each
 * (when their types agree), so later changes to those weights are not
 * seen. */
VBS_API vbs_cu_batch_decoder_t *vbs_cu_batch_decoder_create(const vbs_cu_model_t *m, uint32_t max_ctx, uint32_t batch,
                                                            char *err, size_t err_cap);
VBS_API void vbs_cu_batch_decoder_destroy(vbs_cu_batch_decoder_t *d);
/* One step at position(): tokens (host, B ids; NULL feeds the previous
 * step's argmax of every sequence), then logits_out (host, B x vocab floats)
 * and next_tokens (host, B ids: each sequence's argmax, first maximum wins)
 * when not NULL. Synchronizes. 0, or -1 with the error latched. */
VBS_API int vbs_cu_batch_decoder_step(vbs_cu_batch_decoder_t *d, const uint32_t *tokens, float *logits_out,
                                      uint32_t *next_tokens);
/* n_steps greedy steps enqueued on the decoder's stream, each feeding the
 * previous argmaxes; returns without synchronizing. For timing loops. */
VBS_API int vbs_cu_batch_decoder_enqueue_steps(vbs_cu_batch_decoder_t *d, uint32_t n_steps);
/* Moves every sequence to position pos (the cache rows before it stay as
 * they are) and, when tokens is not NULL, sets the next tokens (host, B). */
VBS_API int vbs_cu_batch_decoder_set_position(vbs_cu_batch_decoder_t *d, uint32_t pos, const uint32_t *tokens);
VBS_API uint32_t vbs_cu_batch_decoder_position(vbs_cu_batch_decoder_t *d);
VBS_API void vbs_cu_batch_decoder_reset(vbs_cu_batch_decoder_t *d);
VBS_API void *vbs_cu_batch_decoder_stream(vbs_cu_batch_decoder_t *d);
VBS_API const float *vbs_cu_decoder_logits_device(vbs_cu_decoder_t *d);
/* Kernels one decode step launches. */
VBS_API uint32_t vbs_cu_decoder_kernels_per_step(vbs_cu_decoder_t *d);
/* How the decoder sums the per-layer tensor-parallel partials: 0 one GPU,
 * 1 ncclAllReduce, 2 peer memory (the o_proj/down epilogue stores into every
 * rank's receive slots over NVLink; the next kernel waits for the ranks'
 * flags and sums the slots in rank order). */
VBS_API uint32_t vbs_cu_decoder_tp_mode(vbs_cu_decoder_t *d);

/* ---- tensor parallelism (no reference counterpart: the engine binds one
 * device, src/vbs_engine.c:142-169) ---- */

/* 128-byte NCCL unique id for rank 0 to broadcast. */
VBS_API int vbs_cu_tp_unique_id(void *out128);
/* Join the TP group; the decoder created afterwards on this process
 * all-reduces after o_proj and down_proj and gathers the logits. */
VBS_API int vbs_cu_tp_init(int rank, int world, const void *id128);
VBS_API int vbs_cu_tp_finalize(void);

#ifdef __cplusplus
}
#endif
#endif /* VBS_B200_H */
