/* ref_shim.c -- exports the reference's own CPU arithmetic for the tests.
 *
 * TEST INFRASTRUCTURE ONLY. Compiled by oracle/Makefile against the
 * UNMODIFIED reference sources (REF=<reference tree>/src and include),
 * into oracle/_ref/libvbsref.so. vbs_host_math.h is a header of static
 * inline functions, so this file gives each one an exported name; the
 * bodies that run are the reference's.
 */
#include "vbs_host_math.h"
#include "vbs_hotpath.h"
#include "vbs_cpu.h"

int ref_dequant_block(int type, const void *blk, float *out) {
    return vbs_dequant_block((vbs_ggml_type_t)type, blk, out);
}
float ref_f16_to_f32(uint16_t h) { return vbs_f16_to_f32(h); }
uint16_t ref_f32_to_f16(float f) { return vbs_f32_to_f16(f); }

void ref_rms_norm(const float *in, const float *w, float *out, uint32_t n, float eps) {
    vbs_host_rms_norm(in, w, out, n, eps);
}
void ref_rope(float *x, uint32_t pos, uint32_t hd, uint32_t nh, float theta) {
    vbs_host_rope(x, pos, hd, nh, theta);
}
void ref_silu_mul(const float *g, const float *u, float *o, uint32_t n) { vbs_host_silu_mul(g, u, o, n); }
void ref_add(const float *a, const float *b, float *o, uint32_t n) { vbs_host_add(a, b, o, n); }
int ref_embed_row(const uint8_t *w, int type, uint32_t token, float *out, uint32_t dim) {
    return vbs_host_embed_row(w, (vbs_ggml_type_t)type, token, out, dim) ? 0 : -1;
}
void ref_cache_store(const float *k, const float *v, uint16_t *kc, uint16_t *vc, uint32_t pos,
                     uint32_t layer, uint32_t max_ctx, uint32_t kv_dim) {
    vbs_host_cache_store(k, v, kc, vc, pos, layer, max_ctx, kv_dim);
}
void ref_attention(const float *q, const uint16_t *kc, const uint16_t *vc, float *out,
                   uint32_t seq_len, uint32_t layer, uint32_t max_ctx, uint32_t nqh,
                   uint32_t nkh, uint32_t hd, float scale) {
    vbs_host_attention(q, kc, vc, out, seq_len, layer, max_ctx, nqh, nkh, hd, scale);
}
int ref_linear_tile(const uint8_t *w, int type, const float *x, float *y, uint32_t cols,
                    uint32_t rows, uint32_t col_off, uint32_t row_off, int accumulate) {
    return vbs_host_linear_tile(w, (vbs_ggml_type_t)type, x, y, cols, rows, col_off, row_off,
                                accumulate != 0) ? 0 : -1;
}
void ref_hot_matvec_q8_0(const uint8_t *w, size_t rows, size_t cols, const int8_t *xq,
                         const float *qd, float *y) {
    vbs_hot_builtin()->matvec_q8_0(w, rows, cols, xq, qd, y);
}
void ref_hot_matvec_f32(const float *w, size_t rows, size_t cols, const float *x, float *y) {
    vbs_hot_builtin()->matvec_f32(w, rows, cols, x, y);
}
