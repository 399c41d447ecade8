/* vbs_oracle.h -- CPU restatement of Verum's per-token decode arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA
 * backend: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it. The product (libvbs_b200.so) never links or
 * calls it, and has no CPU fallback.
 *
 * Every function restates a reference function (path:line inside the
 * Verum-Bespoke-Singularity tree) in plain C11. It is compiled with
 * -std=c11 -ffp-contract=off, the same no-FMA float semantics the
 * reference build gets from `-std=c11 -O3` on x86-64.
 *
 * Parity is pinned two ways (tests/test_oracle_*.py):
 *   - the reference's own known-answer dequant blocks (src/main.c:433-519)
 *     and its test-local references (src/vbs_backend_test.c:82-429);
 *   - the reference itself, compiled from its unmodified sources into
 *     oracle/_ref/ by oracle/Makefile, on seeded inputs, with the results
 *     committed as fixtures under tests/golden/.
 *
 * The weight synthesizer and the Q4_K/Q6_K/Q8_0 quantizers have no
 * counterpart in the reference (it ships no K-quant quantizer,
 * src/vbs_backend_test.c:280-323 only packs unit scales); they are this
 * project's own deterministic definitions, shared bit-for-bit with the
 * device synthesizer so both sides can build identical weights.
 */
#ifndef VBS_ORACLE_H
#define VBS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids used here (include/vbs_gguf.h:13-48 of the reference). */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q8_0 = 8,
    ORC_Q4_K = 12, ORC_Q6_K = 14, ORC_LNS8 = 40
};

/* Block geometry: elements and bytes per block; 0 for unknown types. */
int orc_block_elems(int type);
int orc_block_bytes(int type);
uint64_t orc_row_bytes(int type, uint64_t cols);

/* Half precision. */
float orc_f16_to_f32(uint16_t h);           /* src/vbs_dequant.c:21-44 */
uint16_t orc_f32_to_f16(float f);           /* src/vbs_dequant.c:46-74 (KV store) */
uint16_t orc_f32_to_f16_rne(float f);       /* src/vbs_cpu.c:71-91 (Q8 act. scales) */

/* Dequantize n_blocks consecutive blocks of `type` (exact, bit-for-bit the
 * reference's vbs_dequant_block, src/vbs_dequant.c:339-356). F32/F16 take
 * n_blocks as an element count. Returns elements written, 0 if unsupported. */
size_t orc_dequant(int type, const void *src, size_t n_blocks, float *out);

/* ---- host_math semantics (src/vbs_host_math.h) ---- */
void orc_rms_norm(const float *in, const float *w, float *out, uint32_t n, float eps);
void orc_rope(float *x, uint32_t pos, uint32_t head_dim, uint32_t n_heads, float theta);
void orc_silu_mul(const float *g, const float *u, float *out, uint32_t n);
void orc_add(const float *a, const float *b, float *out, uint32_t n);
int  orc_embed_row(const uint8_t *w, int type, uint32_t token, float *out, uint32_t dim);
void orc_cache_store(const float *k, const float *v, uint16_t *kc, uint16_t *vc,
                     uint32_t pos, uint32_t layer, uint32_t max_ctx, uint32_t kv_dim);
void orc_attention(const float *q, const uint16_t *kc, const uint16_t *vc, float *out,
                   uint32_t seq_len, uint32_t layer, uint32_t max_ctx, uint32_t n_q_heads,
                   uint32_t n_kv_heads, uint32_t head_dim, float scale);
int  orc_linear_tile(const uint8_t *w, int type, const float *x, float *y, uint32_t cols,
                     uint32_t rows, uint32_t col_off, uint32_t row_off, int accumulate);

/* ---- vbs_cpu semantics (src/vbs_cpu.c, src/hotkernels/vbs_hot_ref_impl.h) ---- */
void orc_cpu_quantize_q8(const float *x, size_t cols, int8_t *xq, float *qd, float *qsum);
void orc_cpu_matvec_q8_0(const uint8_t *w, size_t rows, size_t cols, const int8_t *xq,
                         const float *qd, float *y);
void orc_cpu_matvec_f32(const float *w, size_t rows, size_t cols, const float *x, float *y);
void orc_cpu_rms_norm(const float *in, const float *w, float *out, size_t n, float eps);
void orc_cpu_rope(float *x, size_t n_heads, size_t head_dim, size_t pos, float theta);

/* A llama-style model held in host memory (packed tensors, row-major). */
typedef struct {
    uint32_t n_layers, dim, n_heads, n_kv_heads, head_dim, ffn, vocab;
    float eps, theta;
    int embd_type, out_type;
    const uint8_t *embd, *out;
    const float *out_norm;
    const float *const *attn_norm, *const *ffn_norm;   /* [n_layers] */
    const uint8_t *const *wq, *const *wk, *const *wv, *const *wo;
    const uint8_t *const *wgate, *const *wup, *const *wdown;
    const int *tq, *tk, *tv, *to, *tgate, *tup, *tdown;  /* per-layer types */
} orc_model_t;

typedef struct orc_state orc_state_t;

/* mode 0: vbs_cpu semantics (Q8 activations, int dots, row-order float sums,
 *         fp32 KV, two-pass softmax; src/vbs_cpu.c:572-639). Q8_0 and F32
 *         weights only, like the reference CPU path's native types.
 * mode 1: engine / host_math semantics (exact dequant, double accumulation,
 *         fp16 KV cache, online softmax; the op order the JIT emits,
 *         src/vbs_specializer.c:270-349). */
orc_state_t *orc_state_create(const orc_model_t *m, uint32_t context, int mode);
void orc_state_destroy(orc_state_t *s);
/* One decode step at the current position; writes vocab logits when
 * logits != NULL. Returns 0 on success. */
int orc_step(orc_state_t *s, uint32_t token, float *logits);
uint32_t orc_argmax(const float *v, size_t n);   /* first max wins, src/vbs_cpu_main.c:78-80 */

/* ---- seeded synthetic weights and quantizers (this project's own) ---- */
float orc_synth_scale(float std);
/* out[i] = synthetic N(0, std) value of element (row0+r)*full_cols + col0 + c. */
void orc_synth_f32(uint64_t seed, uint64_t rows, uint64_t cols, uint64_t row0,
                   uint64_t col0, uint64_t full_cols, float scale, float *out);
void orc_quantize_q8_0(const float *x, size_t n_blocks, uint8_t *out);
void orc_quantize_q4_k(const float *x, size_t n_blocks, uint8_t *out);
void orc_quantize_q6_k(const float *x, size_t n_blocks, uint8_t *out);
/* Synthesize and quantize a [rows x cols] tile of a seeded tensor. */
int orc_synth_tensor(int type, uint64_t seed, uint64_t rows, uint64_t cols, uint64_t row0,
                     uint64_t col0, uint64_t full_cols, float scale, uint8_t *out);

#ifdef __cplusplus
}
#endif
#endif
