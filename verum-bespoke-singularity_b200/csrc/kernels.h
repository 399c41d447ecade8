// kernels.h -- host-side launch interface between the backend and the
// kernel translation units. Device pointers only; every launcher returns a
// cudaError_t and never synchronises.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace vbs {

// ---- fp16 KV cache layouts ---------------------------------------------------
// Position-major (the reference's, src/vbs_host_math.h:150-159):
//   [layer][position][kv head][head_dim]
// Head-major (the decoder's own cache): [layer][kv head][position][head_dim],
// so one KV head's positions are contiguous and a split of the attention
// streams one run of bytes.
__host__ __device__ inline uint64_t kv_index(bool head_major, uint32_t layer, uint32_t pos, uint32_t local,
                                            uint32_t max_ctx, uint32_t kv_dim, uint32_t head_dim) {
    const uint64_t lbase = (uint64_t)layer * max_ctx * kv_dim;
    if (!head_major) return lbase + (uint64_t)pos * kv_dim + local;
    return lbase + ((uint64_t)(local / head_dim) * max_ctx + pos) * head_dim + local % head_dim;
}

// ---- matvec ----------------------------------------------------------------

enum MvEpi : int {
    MV_EPI_STORE = 0,   // y[r] = v, or y[r] += v when accumulate
    MV_EPI_SILU = 1,    // dual: y[r] = silu(gate_r) * up_r
    MV_EPI_QKV = 2,     // rows [q | k | v]: RoPE on q/k, k/v stored as fp16 into the KV cache
};

// Tensor-parallel exchange region of this rank (device memory), set up by
// vbs_cu_tp_init. Rank r's receive region holds two alternating slot sets
// of world x dim_max floats (set k % 2 for the k-th exchange) and one flag
// per sender. A writer stores its partial rows into slot set [k % 2][its
// rank] of every peer's region, fences at system scope, and the last of its
// CTAs publishes k + 1 into flag [its rank] of every peer. A reader waits
// until every flag of its own region reached its own counter, then sums the
// slots in rank order.
constexpr int TP_MAX_WORLD = 8;
constexpr uint32_t TP_DIM_MAX = 16384;
constexpr uint32_t TP_VOCAB_MAX = 262144;
struct TpComm {
    float *slots[TP_MAX_WORLD];      // region of rank q (own region at [rank])
    float *logits[TP_MAX_WORLD];     // rank q's full-logits area (the step kernel's argmax leaves the gathered logits there)
    uint32_t *flags[TP_MAX_WORLD];   // flag words of rank q's region, [world]
    // The step kernel's exchanges carry their own flag: one 64-bit word per
    // value, (exchange index + 1) << 32 | float bits, stored and loaded
    // whole, so a reader checks each word itself (no fence, no flag store).
    uint64_t *ll[TP_MAX_WORLD];        // rank q's word slots: 2 sets x world x TP_DIM_MAX
    uint64_t *ll_logits[TP_MAX_WORLD]; // rank q's gathered logits words, TP_VOCAB_MAX
    uint32_t *seq;                   // this rank: exchanges completed
    uint32_t *ticket;                // this rank: CTAs finished in the current writer kernel
    uint32_t world, rank;
};

struct MvParams {
    const uint8_t *w[3];        // row segments of matrix A (concatenated row space)
    uint32_t seg_end[3];        // cumulative row ends of the segments
    const uint8_t *wb;          // dual: matrix B (row r pairs with A's row r)
    uint64_t rb;                // packed bytes per row
    uint32_t rows, cols;
    const float *x;             // input (cols floats)
    const float *norm_w;        // optional RMSNorm weight applied to x first (NULL: none)
    float eps;
    const float *x_add;         // optional: x := x + x_add (before the norm), CTA 0 writes x back
    float *x_write;             // where CTA 0 stores the summed x (may alias x)
    float *y;                   // STORE / SILU output
    uint32_t accumulate;
    uint32_t nstage;
    uint32_t *err;
    // QKV epilogue
    float *q_out;
    uint16_t *kc, *vc;          // full caches; layer offset folded in from layer/max_ctx
    const uint32_t *ctrl;       // ctrl[0] = current position
    uint32_t layer, max_ctx, kv_dim, head_dim;
    uint32_t kv_head_major;     // cache layout, see KV_HEAD_MAJOR
    float theta;
    // tensor parallelism over peer memory (NULL: none)
    const TpComm *tp;
    uint32_t tp_write;          // epilogue: rows go to every peer's slot set, then the flags
    uint32_t tp_read;           // prologue: x_add := the rank-ordered sum of the own slot set
};

// ---- batched matvec (mvb.cu): Y[b] = W X[b] for b < batch <= 8 ----
struct MvbParams {
    const uint8_t *w;
    uint64_t rb;                // packed bytes per row
    uint32_t rows, cols, batch;
    const float *x;             // [batch][x_stride]
    uint64_t x_stride;
    float *y;                   // [batch][y_stride]
    uint64_t y_stride;
    float *y_plane;             // set by the launcher: per-chunk partial planes when rows span several chunks
    uint32_t accumulate;
    uint32_t *err;
};
bool mvb_supported(int type, uint32_t rows, uint32_t cols, uint32_t batch, const void *w, const void *x);
// Device workspace the launch needs (0: none).
size_t mvb_workspace_bytes(int type, uint32_t rows, uint32_t cols, uint32_t batch);
cudaError_t mvb_configure();
cudaError_t mvb_launch(int type, const MvbParams &p, float *work, int n_sm, cudaStream_t st);

// ---- quantized GEMM on tcgen05 (gemm.cu): Y[t][r] (+)= W[r] . X[t] ----
struct QgemmParams {
    const uint8_t *w;           // [rows] packed GGUF rows
    uint64_t rb;                // packed bytes per row
    uint32_t rows, cols, tokens;
    const __half *x16;          // set by the launcher: X in fp16, tokens padded to whole tiles
    float *planes;              // set by the launcher: split-K partial planes [split][tokens][rows]
    float *y;                   // [tokens][y_stride]
    uint64_t y_stride;
    uint32_t accumulate;
    uint32_t *err;
};
bool qgemm_supported(int type, uint32_t rows, uint32_t cols, uint32_t tokens);
// Device workspace: the fp16 copy of X, then the split-K planes.
size_t qgemm_workspace_bytes(uint32_t rows, uint32_t cols, uint32_t tokens, int n_sm);
cudaError_t qgemm_configure();
cudaError_t qgemm_launch(int type, QgemmParams p, const float *x, uint64_t x_stride, void *work, int n_sm,
                         cudaStream_t st);
// The same in two parts, for callers that feed one input to several
// matrices: the activations converted once (fp16, in the operand's tile
// layout, qgemm_x16_bytes), then any number of GEMMs on them (planes: the
// split-K workspace, qgemm_planes_bytes; may be NULL when that is 0).
size_t qgemm_x16_bytes(uint32_t tokens, uint32_t cols);
size_t qgemm_planes_bytes(uint32_t rows, uint32_t cols, uint32_t tokens, int n_sm);
cudaError_t qgemm_to_half(const float *x, uint64_t x_stride, __half *x16, uint32_t tokens, uint32_t cols, int n_sm,
                          cudaStream_t st);
cudaError_t qgemm_launch_x16(int type, QgemmParams p, const __half *x16, void *planes, int n_sm, cudaStream_t st);

// True when the TMA/mma kernel can serve this shape/alignment.
bool mv_fast_supported(int type, uint32_t rows, uint32_t cols, const void *const *w, int nw,
                       const void *x, int dual);
cudaError_t mv_fast_launch(int type, int dual, int epi, const MvParams &p, int n_sm, cudaStream_t st,
                           bool pdl, int grid_override);
// Raise the dynamic shared-memory limit of every fast-kernel instance on the
// current device (done once per device at initialisation, never during
// stream capture).
cudaError_t mv_configure();

// Portable exact-dequant fp32 kernel (any type, any alignment, batched).
cudaError_t mv_generic_launch(int type, const uint8_t *w, const float *x, float *y, uint32_t rows,
                              uint32_t cols, uint32_t batch, uint64_t x_stride, uint64_t y_stride,
                              int accumulate, int n_sm, cudaStream_t st);

cudaError_t dequant_launch(int type, const uint8_t *w, float *out, uint64_t n_elems, cudaStream_t st);

// ---- primitives (host_math semantics, src/vbs_host_math.h) -----------------

// Token from token_dev when non-NULL; a token >= rows flags DERR_BAD_ARG
// and writes zeros.
cudaError_t embed_launch(int type, const uint8_t *w, const uint32_t *token_dev, uint32_t token, uint32_t rows,
                         float *out, uint32_t dim, uint32_t *err, cudaStream_t st, bool pdl);
// n rows: out[b] = the embedding row of tokens_dev[b] (prompt chunks)
cudaError_t embed_rows_launch(int type, const uint8_t *w, const uint32_t *tokens_dev, uint32_t n, uint32_t rows,
                              float *out, uint32_t dim, uint32_t *err, cudaStream_t st);
cudaError_t rmsnorm_launch(const float *in, const float *w, float *out, uint32_t n, float eps, cudaStream_t st);
// rope/cache store take the position from ctrl[0] when ctrl != NULL.
cudaError_t rope_launch(float *x, uint32_t pos, const uint32_t *ctrl, uint32_t head_dim, uint32_t n_heads, float theta,
                        cudaStream_t st);
cudaError_t silu_mul_launch(const float *g, const float *u, float *out, uint32_t n, cudaStream_t st);
cudaError_t add_launch(const float *a, const float *b, float *out, uint32_t n, cudaStream_t st);
cudaError_t cache_store_launch(const float *k, const float *v, uint16_t *kc, uint16_t *vc, uint32_t pos,
                               const uint32_t *ctrl, uint32_t layer, uint32_t max_ctx, uint32_t kv_dim,
                               uint32_t head_dim, bool head_major, cudaStream_t st);
// prompt chunks (prefill.cu): `rows` rows at positions p0.., cache layout
// 0 engine order, 1 head-major, 2 head-major swizzled (kv_index_swz)
cudaError_t pf_rmsnorm_rows_launch(const float *in, const float *w, float *out, uint32_t rows, uint32_t n, float eps,
                                   cudaStream_t st);
cudaError_t pf_rope_store_launch(float *q, const float *k, const float *v, uint16_t *kc, uint16_t *vc, uint32_t rows,
                                 uint32_t p0, uint32_t layer, uint32_t max_ctx, uint32_t nqh, uint32_t nkh, uint32_t hd,
                                 float theta, int layout, cudaStream_t st);
// B sequences in lockstep (batch.cu): row b at position *pos_dev (read on
// the device, so a captured step replays at every position), its K/V into
// the head-major cache starting seq_stride * b elements in. Input rows qs
// (queries) and ks (keys, values) floats apart; RoPE'd queries to q_out.
cudaError_t rope_store_seqs_launch(const float *q_in, float *q_out, uint32_t qs, const float *k, const float *v,
                                   uint32_t ks, uint16_t *kc, uint16_t *vc, uint32_t seqs, uint64_t seq_stride,
                                   const uint32_t *pos_dev, uint32_t layer, uint32_t max_ctx, uint32_t nqh, uint32_t nkh,
                                   uint32_t hd, float theta, cudaStream_t st);

// Split-KV GQA decode attention. seq_len from `seq_dev` (+1) when non-NULL,
// else `seq_len`. `work` holds the split partials and merge counters:
// attn_workspace_bytes() bytes, counters zero on first use (self-resetting).
// attn_configure() raises the shared-memory limit of the tensor-core kernels
// on the current device (once per device, outside stream capture).
struct AttnParams {
    const float *q;
    const uint16_t *kc, *vc;
    float *out;
    uint32_t seq_len;
    const uint32_t *seq_dev;
    uint32_t layer, max_ctx, nqh, nkh, hd;
    float scale;
    uint32_t batch;
    uint64_t kv_batch_stride;   // elements between sequences' caches
    uint32_t head_major;        // cache layout (kv_index)
    uint32_t swz;               // head-major rows with the step kernel's chunk swizzle (kv_index_swz); hd 64/128
    uint32_t seq_step;          // sequence b attends seq_len + b * seq_step positions (causal prompt chunks)
    void *work;
    uint32_t *err;
};
size_t attn_workspace_bytes(uint32_t nqh, uint32_t nkh, uint32_t hd, uint32_t batch, uint32_t max_splits);
uint32_t attn_num_splits(uint32_t seq_len_hint, uint32_t nkh, uint32_t batch, int n_sm);
cudaError_t attn_launch(const AttnParams &p, uint32_t n_splits, cudaStream_t st, bool pdl);
cudaError_t attn_configure();
// Causal attention of a prompt chunk (seq_step 1, head-major cache, hd 64 or
// 128, one sequence): query token b attends positions < seq_len + b. One CTA
// per (kv head, 8 tokens), no position splits and no workspace.
bool attn_prefill_supported(const AttnParams &p);
cudaError_t attn_prefill_launch(const AttnParams &p, cudaStream_t st);
// The fixed per-device scratch of vbs_cu_attention_static: its size, and its
// address on the current device.
size_t attn_static_bytes();
cudaError_t attn_static_address(void **ptr);

// argmax over n floats (first maximum wins); writes out_token and, when
// ctrl != NULL, advances ctrl[0] (position) by one, stores the token in
// ctrl[1] and in hist[new position] when hist != NULL and it fits.
// `work` (argmax_workspace_bytes(), zeroed once, self-resetting) lets the
// scan run on several CTAs; NULL runs one CTA.
cudaError_t argmax_launch(const float *v, uint32_t n, uint32_t *out_token, uint32_t *ctrl, uint32_t *hist,
                          uint32_t hist_cap, void *work, cudaStream_t st, bool pdl);
size_t argmax_workspace_bytes();

// ---- persistent decode step (step.cu) -----------------------------------------
// One cooperative launch per token runs every op of the step; see step.cu.

// Per-layer weights of the step kernel, repacked by step_repack into stage
// units: unit (tile, chunk) = 16 slot rows x rs bytes, one contiguous run, so
// the kernel moves a whole stage with one bulk copy.
struct StepLayer {
    const uint8_t *qkv, *o, *gu, *down;
    const float *attn_norm, *ffn_norm;
};

struct StepMvGeom {
    uint32_t ck;       // columns per stage chunk
    uint32_t rs;       // row slot stride in the stage (bytes)
    uint32_t nch;      // chunks per row
    uint32_t ntiles;   // 16-row tiles
};

enum : int { STEP_QKV = 0, STEP_O = 1, STEP_GU = 2, STEP_DOWN = 3, STEP_OUT = 4 };

struct StepParams {
    uint32_t n_layers, dim, nqh, nkh, hd, ffn, vocab, max_ctx;
    float eps, theta, scale;
    int t_embd, t_qkv, t_o, t_gu, t_down, t_out;
    const uint8_t *embd;        // embedding table, GGUF layout
    const uint8_t *out;         // output matrix, repacked (step_repack)
    const float *out_norm;
    const StepLayer *layers;    // device array [n_layers]
    uint16_t *kc, *vc;          // fp16 KV cache, head-major, 16-byte chunks swizzled by position (kv_index_swz)
    float *acc;                 // per layer [q|k|v | o_proj | h | down partials per column chunk]
    uint64_t acc_layer;         // floats per layer in `acc`
    float *logits;              // [vocab]
    float *att;                 // [nqh * hd]
    void *attn_work;            // split partials
    uint32_t attn_splits;       // at most this many splits per KV head (nkh * attn_splits <= grid)
    uint32_t *sync;             // zeroed before each step: grid barrier, abort word, tickets, argmax slots
    uint32_t *ctrl, *hist;
    uint32_t hist_cap;
    uint32_t *err;
    StepMvGeom geo[5];          // by STEP_* op
    uint32_t ring_bytes, stage_max, x_off, xq_off, xf_off, ring_off;   // shared-memory plan (byte ring)
    // tensor parallelism (tp NULL: one GPU). This rank's shard: nqh, nkh,
    // ffn and vocab above are per rank; o_proj/down partials and the logits
    // are exchanged over peer memory (TpComm), 2 exchanges per layer and 1
    // for the logits per step.
    const TpComm *tp;
    uint32_t tp_world, tp_rank, vocab_full;
    // Bounded waits: every wait of the step gives up after wait_ns of global
    // time (2 s by default) and records DERR_TIMEOUT_*. A test can shorten
    // it and name an op (drop_op, else ~0u) before whose grid barrier CTA 0
    // does not arrive, so the other CTAs' waits run out.
    uint64_t wait_ns;
    uint32_t drop_op;
    // Timeline of one step, written only by builds with VBS_STEP_TRACE
    // (a profiling build): per CTA and op, SK_TR_SLOTS %globaltimer stamps.
    unsigned long long *trace;
};
// Slots: 0 op start, 1 prologue done, 2 op done, 3/4 producer first / last
// issue, 5..15 phases inside the op (bench.py --profile timeline names them).
constexpr int SK_TR_SLOTS = 16;

// Element (pos, i) of one layer's KV block in the step kernel's cache:
// [kv head][position][head_dim] with the 16-byte chunk index of each row
// XOR-ed with (position & 7), so 8 consecutive rows read at one logical
// chunk fall in 8 different bank groups.
__host__ __device__ inline uint64_t kv_index_swz(uint32_t layer, uint32_t pos, uint32_t local, uint32_t max_ctx,
                                                uint32_t n_kv, uint32_t head_dim) {
    const uint32_t h = local / head_dim, d = local % head_dim;
    const uint32_t c = (d >> 3) ^ (pos & 7u);
    return (((uint64_t)layer * n_kv + h) * max_ctx + pos) * head_dim + (c << 3) + (d & 7u);
}

// Fills the geometry/shared-memory plan of `p` for a grid of n_sm CTAs;
// false (with a reason) when the model shape is outside what the step
// kernel serves.
bool step_plan(StepParams &p, int n_sm, char *why, size_t cap);
size_t step_attn_work_bytes(const StepParams &p);
// Repacked size of op `op`'s matrix, and the repack from GGUF rows: QKV takes
// w0/w1/w2 = q/k/v, GU w0/w1 = gate/up, the others w0.
size_t step_packed_bytes(const StepParams &p, int op);
cudaError_t step_repack(const StepParams &p, int op, const uint8_t *w0, const uint8_t *w1, const uint8_t *w2,
                        uint8_t *dst, cudaStream_t st);
size_t step_sync_words(int n_sm);
cudaError_t step_configure();
cudaError_t step_launch(const StepParams &p, int n_sm, cudaStream_t st);

// ---- strict-parity kernels (vbs_cpu arithmetic) -----------------------------
cudaError_t strict_quantize_q8_launch(const float *x, uint32_t cols, int8_t *xq, float *qd, cudaStream_t st);
cudaError_t strict_matvec_q8_0_launch(const uint8_t *w, uint32_t rows, uint32_t cols, const int8_t *xq,
                                      const float *qd, float *y, int accumulate, cudaStream_t st);
cudaError_t strict_matvec_f32_launch(const float *w, uint32_t rows, uint32_t cols, const float *x, float *y,
                                     int accumulate, cudaStream_t st);
cudaError_t strict_rmsnorm_launch(const float *in, const float *w, float *out, uint32_t n, float eps,
                                  cudaStream_t st);
cudaError_t strict_rope_launch(float *x, uint32_t n_heads, uint32_t head_dim, const uint32_t *ctrl,
                               float theta, cudaStream_t st);
cudaError_t strict_attention_launch(const float *q, const float *k, const float *v, float *kcache, float *vcache,
                                    float *out, const uint32_t *ctrl, uint32_t layer, uint32_t context,
                                    uint32_t nqh, uint32_t nkh, uint32_t hd, float *scores, uint32_t *err,
                                    cudaStream_t st);
cudaError_t strict_silu_launch(const float *g, const float *u, float *h, uint32_t n, cudaStream_t st);
cudaError_t strict_add_launch(float *x, const float *t, uint32_t n, cudaStream_t st);

// ---- synthetic weights -------------------------------------------------------
cudaError_t synth_launch(int type, uint8_t *dst, uint64_t rows, uint64_t cols, uint64_t row0, uint64_t col0,
                         uint64_t full_cols, uint64_t seed, float scale, cudaStream_t st);

// Launch bookkeeping (counts kernels for vbs_cu_kernel_launches).
void note_launches(uint64_t n);

}  // namespace vbs
