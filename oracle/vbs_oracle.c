/* vbs_oracle.c -- CPU restatement of Verum's decode-step arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see vbs_oracle.h). Citations are paths inside
 * the Verum-Bespoke-Singularity source tree. Build: oracle/Makefile
 * (gcc -std=c11 -O2 -ffp-contract=off, no FMA, like the reference build).
 */
#include "vbs_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* geometry (include/vbs_gguf.h:53-58, src/vbs_gguf.c block table)      */
/* ------------------------------------------------------------------ */

int orc_block_elems(int type) {
    switch (type) {
        case ORC_F32: case ORC_F16: return 1;
        case ORC_Q4_0: case ORC_Q4_1: case ORC_Q8_0: case ORC_LNS8: return 32;
        case ORC_Q4_K: case ORC_Q6_K: return 256;
        default: return 0;
    }
}

int orc_block_bytes(int type) {
    switch (type) {
        case ORC_F32: return 4;
        case ORC_F16: return 2;
        case ORC_Q4_0: return 18;
        case ORC_Q4_1: return 20;
        case ORC_Q8_0: return 34;
        case ORC_Q4_K: return 144;
        case ORC_Q6_K: return 210;
        case ORC_LNS8: return 36;
        default: return 0;
    }
}

uint64_t orc_row_bytes(int type, uint64_t cols) {
    int e = orc_block_elems(type);
    if (!e || cols % (uint64_t)e) return 0;
    return cols / (uint64_t)e * (uint64_t)orc_block_bytes(type);
}

static uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
static float bits_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* ------------------------------------------------------------------ */
/* half precision                                                       */
/* ------------------------------------------------------------------ */

/* Exact binary16 -> binary32 (src/vbs_dequant.c:21-44): subnormals are
 * renormalised, inf/nan keep their payload shifted into place. */
float orc_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 1023u;
    if (e == 31u) return bits_f32(s | 0x7F800000u | (m << 13));
    if (e != 0u) return bits_f32(s | ((e + 112u) << 23) | (m << 13));
    if (m == 0u) return bits_f32(s);
    int k = 0;                      /* shift until the implicit bit appears */
    while (!(m & 0x400u)) { m <<= 1; k++; }
    return bits_f32(s | ((uint32_t)(113 - k) << 23) | ((m & 1023u) << 13));
}

/* binary32 -> binary16 as src/vbs_dequant.c:46-74 rounds it (used by the
 * fp16 KV store, src/vbs_host_math.h:150-159): nearest-even for normal
 * results, half-up for subnormal results, NaN -> quiet 0x7C01 pattern. */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x = f32_bits(f);
    uint16_t s = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t be = (x >> 23) & 255u, m = x & 0x7FFFFFu;
    if (be == 255u) return (uint16_t)(s | 0x7C00u | (m ? 1u : 0u));
    int e = (int)be - 112;          /* rebias 127 -> 15 */
    if (e >= 31) return (uint16_t)(s | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return s;
        uint32_t full = m | 0x800000u;
        uint32_t sh = (uint32_t)(14 - e);
        uint32_t q = (full + (1u << (sh - 1))) >> sh;
        return (uint16_t)(s | (q >= 0x400u ? 0x400u : q));
    }
    uint32_t r = m + 0xFFFu + ((m >> 13) & 1u);
    if (r & 0x800000u) { r = 0; e++; }
    if (e >= 31) return (uint16_t)(s | 0x7C00u);
    return (uint16_t)(s | ((uint32_t)e << 10) | (r >> 13));
}

/* binary32 -> binary16, nearest-even everywhere (src/vbs_cpu.c:71-91, the
 * converter quantize_q8 uses for its block scales). */
uint16_t orc_f32_to_f16_rne(float f) {
    uint32_t x = f32_bits(f);
    uint16_t s = (uint16_t)((x >> 16) & 0x8000u);
    int e = (int)((x >> 23) & 255u) - 127;
    uint32_t m = x & 0x7FFFFFu;
    if (e > 15) return (uint16_t)(s | 0x7C00u);
    if (e >= -14) {
        uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13);
        uint32_t rem = m & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(s | h);
    }
    if (e < -25) return s;
    m |= 0x800000u;
    int sh = -e - 1;
    uint32_t h = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(s | h);
}

/* ------------------------------------------------------------------ */
/* block dequantization (src/vbs_dequant.c:123-333), same float order   */
/* ------------------------------------------------------------------ */

static void dq_q8_0(const uint8_t *b, float *y) {             /* :174-179 */
    float d = orc_f16_to_f32(rd16(b));
    for (int i = 0; i < 32; i++) y[i] = d * (float)(int8_t)b[2 + i];
}

static void dq_q4_0(const uint8_t *b, float *y) {             /* :123-132 */
    float d = orc_f16_to_f32(rd16(b));
    for (int i = 0; i < 16; i++) {
        y[i] = ((float)(b[2 + i] & 15) - 8.0f) * d;
        y[i + 16] = ((float)(b[2 + i] >> 4) - 8.0f) * d;
    }
}

static void dq_q4_1(const uint8_t *b, float *y) {             /* :134-144 */
    float d = orc_f16_to_f32(rd16(b)), mn = orc_f16_to_f32(rd16(b + 2));
    for (int i = 0; i < 16; i++) {
        y[i] = d * (float)(b[4 + i] & 15) + mn;
        y[i + 16] = d * (float)(b[4 + i] >> 4) + mn;
    }
}

/* 6-bit scale/min pair j of a Q4_K super-block (src/vbs_dequant.c:225-233). */
static void k4_scale_min(const uint8_t *s, int j, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void dq_q4_k(const uint8_t *b, float *y) {             /* :258-277 */
    float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
    const uint8_t *sc6 = b + 4, *qs = b + 16;
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        k4_scale_min(sc6, j, &sc, &mn);
        float a = d * (float)sc, c = dmin * (float)mn;
        const uint8_t *q = qs + (j >> 1) * 32;
        for (int i = 0; i < 32; i++) {
            int nib = (j & 1) ? (q[i] >> 4) : (q[i] & 15);
            y[j * 32 + i] = a * (float)nib - c;
        }
    }
}

static void dq_q6_k(const uint8_t *b, float *y) {             /* :316-333 */
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = orc_f16_to_f32(rd16(b + 208));
    for (int e = 0; e < 256; e++) {
        int half = e >> 7, quarter = (e >> 5) & 3, l = e & 31;
        int lo = (ql[half * 64 + (quarter & 1) * 32 + l] >> ((quarter >> 1) * 4)) & 15;
        int hi = (qh[half * 32 + l] >> (quarter * 2)) & 3;
        y[e] = d * (float)sc[e >> 4] * (float)((lo | (hi << 4)) - 32);
    }
}

/* LNS8 (36 B: 32 u8 log2 values, f32 scale at byte 32): value = 2^q *
 * scale, src/vbs_host_math.h:111-121 (exp2f of an integer 0..255 is the
 * exact power of two, +inf from 128 on). */
static void dq_lns8(const uint8_t *b, float *y) {
    float s;
    memcpy(&s, b + 32, 4);
    for (int i = 0; i < 32; i++) y[i] = ldexpf(1.0f, b[i]) * s;
}

size_t orc_dequant(int type, const void *src, size_t n_blocks, float *out) {
    const uint8_t *p = (const uint8_t *)src;
    int be = orc_block_elems(type), bb = orc_block_bytes(type);
    if (!be) return 0;
    for (size_t i = 0; i < n_blocks; i++) {
        const uint8_t *b = p + i * (size_t)bb;
        float *y = out + i * (size_t)be;
        switch (type) {
            case ORC_F32: memcpy(y, b, 4); break;
            case ORC_F16: y[0] = orc_f16_to_f32(rd16(b)); break;
            case ORC_Q4_0: dq_q4_0(b, y); break;
            case ORC_Q4_1: dq_q4_1(b, y); break;
            case ORC_Q8_0: dq_q8_0(b, y); break;
            case ORC_Q4_K: dq_q4_k(b, y); break;
            case ORC_Q6_K: dq_q6_k(b, y); break;
            case ORC_LNS8: dq_lns8(b, y); break;
            default: return 0;
        }
    }
    return n_blocks * (size_t)be;
}

/* ------------------------------------------------------------------ */
/* host_math semantics (src/vbs_host_math.h)                            */
/* ------------------------------------------------------------------ */

void orc_rms_norm(const float *in, const float *w, float *out, uint32_t n, float eps) {
    double ss = 0.0;                                           /* :28-36 */
    for (uint32_t i = 0; i < n; i++) ss += (double)in[i] * in[i];
    float scale = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (uint32_t i = 0; i < n; i++) out[i] = in[i] * scale * w[i];
}

void orc_rope(float *x, uint32_t pos, uint32_t head_dim, uint32_t n_heads, float theta) {
    for (uint32_t h = 0; h < n_heads; h++) {                   /* :38-51 */
        float *xh = x + (size_t)h * head_dim;
        for (uint32_t i = 0; i + 1 < head_dim; i += 2) {
            float ang = (float)pos * powf(theta, -(float)i / (float)head_dim);
            float c = cosf(ang), s = sinf(ang);
            float a = xh[i], b = xh[i + 1];
            xh[i] = a * c - b * s;
            xh[i + 1] = a * s + b * c;
        }
    }
}

void orc_silu_mul(const float *g, const float *u, float *out, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) out[i] = g[i] / (1.0f + expf(-g[i])) * u[i]; /* :53-57 */
}

void orc_add(const float *a, const float *b, float *out, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) out[i] = a[i] + b[i];      /* :59-62 */
}

int orc_embed_row(const uint8_t *w, int type, uint32_t token, float *out, uint32_t dim) {
    uint64_t rb = orc_row_bytes(type, dim);                     /* :136-142 */
    if (!rb) return -1;
    orc_dequant(type, w + (uint64_t)token * rb, dim / (uint32_t)orc_block_elems(type), out);
    return 0;
}

void orc_cache_store(const float *k, const float *v, uint16_t *kc, uint16_t *vc,
                     uint32_t pos, uint32_t layer, uint32_t max_ctx, uint32_t kv_dim) {
    uint64_t base = ((uint64_t)layer * max_ctx + pos) * kv_dim; /* :150-159 */
    for (uint32_t i = 0; i < kv_dim; i++) {
        kc[base + i] = orc_f32_to_f16(k[i]);
        vc[base + i] = orc_f32_to_f16(v[i]);
    }
}

/* Online-softmax GQA decode attention (src/vbs_host_math.h:170-209). */
void orc_attention(const float *q, const uint16_t *kc, const uint16_t *vc, float *out,
                   uint32_t seq_len, uint32_t layer, uint32_t max_ctx, uint32_t nqh,
                   uint32_t nkh, uint32_t hd, float scale) {
    if (!nkh || !nqh || !hd) return;
    uint32_t group = nqh / nkh ? nqh / nkh : 1;
    uint64_t lbase = (uint64_t)layer * max_ctx * nkh * hd;
    for (uint32_t h = 0; h < nqh; h++) {
        uint32_t kvh = h / group;
        const float *qh = q + (size_t)h * hd;
        float *acc = out + (size_t)h * hd;
        float mx = -3.4028235e38f, l = 0.0f;
        memset(acc, 0, hd * sizeof(float));
        for (uint32_t t = 0; t < seq_len; t++) {
            uint64_t row = lbase + ((uint64_t)t * nkh + kvh) * hd;
            double dot = 0.0;
            for (uint32_t d = 0; d < hd; d++) dot += (double)qh[d] * (double)orc_f16_to_f32(kc[row + d]);
            float sc = (float)dot * scale;
            float mnew = sc > mx ? sc : mx;
            float r = expf(mx - mnew), e = expf(sc - mnew);
            l = l * r + e;
            mx = mnew;
            for (uint32_t d = 0; d < hd; d++) acc[d] = acc[d] * r + e * orc_f16_to_f32(vc[row + d]);
        }
        float inv = 1.0f / l;
        for (uint32_t d = 0; d < hd; d++) acc[d] *= inv;
    }
}

/* Exact dequant + double-accumulated matvec tile (src/vbs_host_math.h:223-267). */
int orc_linear_tile(const uint8_t *w, int type, const float *x, float *y, uint32_t cols,
                    uint32_t rows, uint32_t col_off, uint32_t row_off, int accumulate) {
    int be = orc_block_elems(type);
    uint64_t rb = orc_row_bytes(type, cols);
    if (!be || !rb) return -1;
    float vals[256];
    for (uint32_t r = 0; r < rows; r++) {
        const uint8_t *row = w + (uint64_t)r * rb;
        double sum = 0.0;
        if (be == 1) {
            for (uint32_t c = 0; c < cols; c++) {
                float wv;
                orc_dequant(type, row + (size_t)c * (size_t)orc_block_bytes(type), 1, &wv);
                sum += (double)wv * x[col_off + c];
            }
        } else {
            for (uint32_t b = 0; b < cols / (uint32_t)be; b++) {
                orc_dequant(type, row + (size_t)b * (size_t)orc_block_bytes(type), 1, vals);
                for (int i = 0; i < be; i++) sum += (double)vals[i] * x[col_off + b * (uint32_t)be + (uint32_t)i];
            }
        }
        float *dst = y + row_off + r;
        *dst = accumulate ? *dst + (float)sum : (float)sum;
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* vbs_cpu semantics                                                    */
/* ------------------------------------------------------------------ */

/* Per-32 Q8 activation quantization (src/vbs_cpu.c:166-182). */
void orc_cpu_quantize_q8(const float *x, size_t cols, int8_t *xq, float *qd, float *qsum) {
    for (size_t b = 0; b < cols / 32; b++) {
        const float *xb = x + b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) if (fabsf(xb[i]) > amax) amax = fabsf(xb[i]);
        float d = amax / 127.0f, inv = d ? 1.0f / d : 0.0f;
        int sum = 0;
        for (int i = 0; i < 32; i++) {
            int q = (int)roundf(xb[i] * inv);
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            xq[b * 32 + (size_t)i] = (int8_t)q;
            sum += q;
        }
        qd[b] = orc_f16_to_f32(orc_f32_to_f16_rne(d));
        if (qsum) qsum[b] = orc_f16_to_f32(orc_f32_to_f16_rne((float)sum * d));
    }
}

/* Q8_0 x Q8 integer block dots, float sums in block order
 * (src/hotkernels/vbs_hot_ref_impl.h:49-64). */
void orc_cpu_matvec_q8_0(const uint8_t *w, size_t rows, size_t cols, const int8_t *xq,
                         const float *qd, float *y) {
    size_t nb = cols / 32;
    for (size_t r = 0; r < rows; r++) {
        const uint8_t *row = w + r * nb * 34;
        float sum = 0.0f;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * 34;
            int dot = 0;
            for (int i = 0; i < 32; i++) dot += (int)(int8_t)blk[2 + i] * (int)xq[b * 32 + (size_t)i];
            sum += orc_f16_to_f32(rd16(blk)) * qd[b] * (float)dot;
        }
        y[r] = sum;
    }
}

/* Sequential float dot per row (src/hotkernels/vbs_hot_ref_impl.h:110-118). */
void orc_cpu_matvec_f32(const float *w, size_t rows, size_t cols, const float *x, float *y) {
    for (size_t r = 0; r < rows; r++) {
        float sum = 0.0f;
        for (size_t i = 0; i < cols; i++) sum += w[r * cols + i] * x[i];
        y[r] = sum;
    }
}

void orc_cpu_rms_norm(const float *in, const float *w, float *out, size_t n, float eps) {
    double sum = 0.0;                                          /* src/vbs_cpu.c:251-262 */
    for (size_t i = 0; i < n; i++) sum += (double)in[i] * in[i];
    float scale = 1.0f / sqrtf((float)(sum / (double)n) + eps);
    for (size_t i = 0; i < n; i++) out[i] = in[i] * scale * w[i];
}

void orc_cpu_rope(float *x, size_t n_heads, size_t head_dim, size_t pos, float theta) {
    for (size_t h = 0; h < n_heads; h++) {                     /* src/vbs_cpu.c:264-275 */
        for (size_t i = 0; i < head_dim; i += 2) {
            float ang = (float)pos * powf(theta, -(float)i / (float)head_dim);
            float c = cosf(ang), s = sinf(ang);
            size_t j = h * head_dim + i;
            float a = x[j], b = x[j + 1];
            x[j] = a * c - b * s;
            x[j + 1] = a * s + b * c;
        }
    }
}

uint32_t orc_argmax(const float *v, size_t n) {
    uint32_t best = 0;
    for (size_t k = 1; k < n; k++) if (v[k] > v[best]) best = (uint32_t)k;
    return best;
}

/* ------------------------------------------------------------------ */
/* full decode step                                                     */
/* ------------------------------------------------------------------ */

struct orc_state {
    orc_model_t m;
    int mode;
    uint32_t context, pos, kv_dim;
    float *x, *norm, *q, *k, *v, *att, *tmp, *gate, *up, *hidden, *scores;
    float *kf, *vf;             /* mode 0: fp32 KV [layer][context][kv_dim] */
    uint16_t *kh, *vh;          /* mode 1: fp16 KV, same layout */
    int8_t *xq;
    float *qd, *qsum;
};

orc_state_t *orc_state_create(const orc_model_t *m, uint32_t context, int mode) {
    orc_state_t *s = (orc_state_t *)calloc(1, sizeof(*s));
    if (!s) return NULL;
    s->m = *m;
    s->mode = mode;
    s->context = context;
    s->kv_dim = m->n_kv_heads * m->head_dim;
    size_t big = m->dim > m->ffn ? m->dim : m->ffn;
    size_t cache_n = (size_t)m->n_layers * context * s->kv_dim;
    s->x = calloc(m->dim, 4); s->norm = calloc(m->dim, 4); s->q = calloc(m->dim, 4);
    s->k = calloc(s->kv_dim, 4); s->v = calloc(s->kv_dim, 4); s->att = calloc(m->dim, 4);
    s->tmp = calloc(m->dim, 4); s->gate = calloc(m->ffn, 4); s->up = calloc(m->ffn, 4);
    s->hidden = calloc(m->ffn, 4); s->scores = calloc(context, 4);
    s->xq = calloc(big, 1); s->qd = calloc(big / 32 + 1, 4); s->qsum = calloc(big / 32 + 1, 4);
    if (mode == 0) { s->kf = calloc(cache_n, 4); s->vf = calloc(cache_n, 4); }
    else { s->kh = calloc(cache_n, 2); s->vh = calloc(cache_n, 2); }
    if (!s->x || !s->norm || !s->q || !s->k || !s->v || !s->att || !s->tmp || !s->gate ||
        !s->up || !s->hidden || !s->scores || !s->xq || !s->qd || !s->qsum ||
        (mode == 0 ? (!s->kf || !s->vf) : (!s->kh || !s->vh))) {
        orc_state_destroy(s);
        return NULL;
    }
    return s;
}

void orc_state_destroy(orc_state_t *s) {
    if (!s) return;
    free(s->x); free(s->norm); free(s->q); free(s->k); free(s->v); free(s->att); free(s->tmp);
    free(s->gate); free(s->up); free(s->hidden); free(s->scores); free(s->kf); free(s->vf);
    free(s->kh); free(s->vh); free(s->xq); free(s->qd); free(s->qsum);
    free(s);
}

/* y = W x with the state's semantics: vbs_cpu's matrix() for mode 0
 * (src/vbs_cpu.c:184-219), vbs_host_linear_tile for mode 1. */
static int state_matrix(orc_state_t *s, const uint8_t *w, int type, uint32_t rows,
                        uint32_t cols, const float *x, float *y) {
    if (s->mode == 1) return orc_linear_tile(w, type, x, y, cols, rows, 0, 0, 0);
    for (uint32_t i = 0; i < cols; i++) {
        if (!isfinite(x[i])) {
            for (uint32_t r = 0; r < rows; r++) y[r] = NAN;
            return 0;
        }
    }
    if (type == ORC_F32) {
        orc_cpu_matvec_f32((const float *)(const void *)w, rows, cols, x, y);
        return 0;
    }
    if (type == ORC_Q8_0) {
        orc_cpu_quantize_q8(x, cols, s->xq, s->qd, s->qsum);
        orc_cpu_matvec_q8_0(w, rows, cols, s->xq, s->qd, y);
        return 0;
    }
    return -1;
}

int orc_step(orc_state_t *s, uint32_t token, float *logits) {
    const orc_model_t *m = &s->m;
    if (token >= m->vocab || s->pos >= s->context) return -1;
    uint32_t pos = s->pos, dim = m->dim, hd = m->head_dim, kvd = s->kv_dim;
    if (orc_embed_row(m->embd, m->embd_type, token, s->x, dim)) return -1;
    for (uint32_t L = 0; L < m->n_layers; L++) {
        if (s->mode == 0) orc_cpu_rms_norm(s->x, m->attn_norm[L], s->norm, dim, m->eps);
        else orc_rms_norm(s->x, m->attn_norm[L], s->norm, dim, m->eps);
        if (state_matrix(s, m->wq[L], m->tq[L], dim, dim, s->norm, s->q)) return -1;
        if (state_matrix(s, m->wk[L], m->tk[L], kvd, dim, s->norm, s->k)) return -1;
        if (state_matrix(s, m->wv[L], m->tv[L], kvd, dim, s->norm, s->v)) return -1;
        float att_scale = 1.0f / sqrtf((float)hd);
        if (s->mode == 0) {
            /* src/vbs_cpu.c:583-611: fp32 cache, per-head two-pass softmax. */
            orc_cpu_rope(s->q, m->n_heads, hd, pos, m->theta);
            orc_cpu_rope(s->k, m->n_kv_heads, hd, pos, m->theta);
            size_t here = ((size_t)L * s->context + pos) * kvd;
            memcpy(s->kf + here, s->k, kvd * 4);
            memcpy(s->vf + here, s->v, kvd * 4);
            uint32_t groups = m->n_heads / m->n_kv_heads;
            for (uint32_t h = 0; h < m->n_heads; h++) {
                uint32_t kh = h / groups;
                const float *qh = s->q + (size_t)h * hd;
                float mx = -INFINITY;
                for (uint32_t t = 0; t <= pos; t++) {
                    const float *kt = s->kf + ((size_t)L * s->context + t) * kvd + (size_t)kh * hd;
                    float dot = 0.0f;
                    for (uint32_t i = 0; i < hd; i++) dot += qh[i] * kt[i];
                    s->scores[t] = dot * att_scale;
                    if (s->scores[t] > mx) mx = s->scores[t];
                }
                float den = 0.0f;
                for (uint32_t t = 0; t <= pos; t++) { s->scores[t] = expf(s->scores[t] - mx); den += s->scores[t]; }
                if (!isfinite(den) || den <= 0.0f) return -1;
                float *o = s->att + (size_t)h * hd;
                memset(o, 0, hd * 4);
                for (uint32_t t = 0; t <= pos; t++) {
                    const float *vt = s->vf + ((size_t)L * s->context + t) * kvd + (size_t)kh * hd;
                    float p = s->scores[t] / den;
                    for (uint32_t i = 0; i < hd; i++) o[i] += p * vt[i];
                }
            }
        } else {
            /* JIT op order (src/vbs_specializer.c:285-300) on host_math ops. */
            orc_rope(s->q, pos, hd, m->n_heads, m->theta);
            orc_rope(s->k, pos, hd, m->n_kv_heads, m->theta);
            orc_cache_store(s->k, s->v, s->kh, s->vh, pos, L, s->context, kvd);
            orc_attention(s->q, s->kh, s->vh, s->att, pos + 1, L, s->context, m->n_heads,
                          m->n_kv_heads, hd, att_scale);
        }
        if (state_matrix(s, m->wo[L], m->to[L], dim, dim, s->att, s->tmp)) return -1;
        for (uint32_t i = 0; i < dim; i++) s->x[i] += s->tmp[i];
        if (s->mode == 0) orc_cpu_rms_norm(s->x, m->ffn_norm[L], s->norm, dim, m->eps);
        else orc_rms_norm(s->x, m->ffn_norm[L], s->norm, dim, m->eps);
        if (state_matrix(s, m->wgate[L], m->tgate[L], m->ffn, dim, s->norm, s->gate)) return -1;
        if (state_matrix(s, m->wup[L], m->tup[L], m->ffn, dim, s->norm, s->up)) return -1;
        if (s->mode == 0) {
            for (uint32_t i = 0; i < m->ffn; i++)
                s->hidden[i] = (s->gate[i] / (1.0f + expf(-s->gate[i]))) * s->up[i];
        } else {
            orc_silu_mul(s->gate, s->up, s->hidden, m->ffn);
        }
        if (state_matrix(s, m->wdown[L], m->tdown[L], dim, m->ffn, s->hidden, s->tmp)) return -1;
        for (uint32_t i = 0; i < dim; i++) s->x[i] += s->tmp[i];
    }
    if (logits) {
        if (s->mode == 0) orc_cpu_rms_norm(s->x, m->out_norm, s->norm, dim, m->eps);
        else orc_rms_norm(s->x, m->out_norm, s->norm, dim, m->eps);
        if (state_matrix(s, m->out, m->out_type, m->vocab, dim, s->norm, logits)) return -1;
    }
    s->pos++;
    return 0;
}

/* ------------------------------------------------------------------ */
/* seeded synthetic weights and quantizers                              */
/* ------------------------------------------------------------------ */

/* splitmix64 output function (Steele, Lea & Flood, OOPSLA 2014). */
static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* A normal deviate approximated by the centred sum of four 16-bit uniforms
 * (Irwin-Hall, n = 4): integer exact, so host and device agree bit for bit.
 * The float scale maps the sum's standard deviation to `std`. */
float orc_synth_scale(float std) {
    return (float)((double)std / sqrt((65536.0 * 65536.0 - 1.0) / 3.0));
}

static float synth_value(uint64_t seed, uint64_t idx, float scale) {
    uint64_t h = mix64(seed + 0x9E3779B97F4A7C15ULL * (idx + 1));
    int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) +
                (int32_t)((h >> 32) & 0xFFFF) + (int32_t)(h >> 48);
    return (float)(s - 131070) * scale;
}

void orc_synth_f32(uint64_t seed, uint64_t rows, uint64_t cols, uint64_t row0,
                   uint64_t col0, uint64_t full_cols, float scale, float *out) {
    for (uint64_t r = 0; r < rows; r++)
        for (uint64_t c = 0; c < cols; c++)
            out[r * cols + c] = synth_value(seed, (row0 + r) * full_cols + col0 + c, scale);
}

static void wr16(uint8_t *p, uint16_t v) { memcpy(p, &v, 2); }
static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q8_0: d = amax/127 (fp16), q = round(x / d). */
void orc_quantize_q8_0(const float *x, size_t n_blocks, uint8_t *out) {
    for (size_t b = 0; b < n_blocks; b++) {
        const float *xb = x + b * 32;
        uint8_t *o = out + b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(xb[i]));
        uint16_t dh = orc_f32_to_f16_rne(amax / 127.0f);
        float d = orc_f16_to_f32(dh);
        wr16(o, dh);
        for (int i = 0; i < 32; i++)
            o[2 + i] = (uint8_t)(int8_t)(d > 0.0f ? clampi((int)roundf(xb[i] / d), -127, 127) : 0);
    }
}

/* Q4_K: per 32-element sub-block an affine range [min(0, lo), hi] split in
 * 15 steps; 6-bit sub-block scales/mins relative to fp16 d/dmin; nibble
 * q = round((x + dmin*m) / (d*sc)). Layout per src/vbs_dequant.c:258-277. */
void orc_quantize_q4_k(const float *x, size_t n_blocks, uint8_t *out) {
    for (size_t b = 0; b < n_blocks; b++) {
        const float *xb = x + b * 256;
        uint8_t *o = out + b * 144;
        float scl[8], mins[8], smax = 0.0f, mmax = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = xb[j * 32];
            for (int i = 0; i < 32; i++) { lo = fminf(lo, xb[j * 32 + i]); hi = fmaxf(hi, xb[j * 32 + i]); }
            scl[j] = (hi - lo) / 15.0f;
            mins[j] = -lo;
            smax = fmaxf(smax, scl[j]);
            mmax = fmaxf(mmax, mins[j]);
        }
        uint16_t dh = orc_f32_to_f16_rne(smax / 63.0f), mh = orc_f32_to_f16_rne(mmax / 63.0f);
        float d = orc_f16_to_f32(dh), dmin = orc_f16_to_f32(mh);
        int sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = d > 0.0f ? clampi((int)roundf(scl[j] / d), 0, 63) : 0;
            mn[j] = dmin > 0.0f ? clampi((int)roundf(mins[j] / dmin), 0, 63) : 0;
        }
        memset(o, 0, 144);
        wr16(o, dh);
        wr16(o + 2, mh);
        uint8_t *s6 = o + 4, *qs = o + 16;
        for (int j = 0; j < 4; j++) {
            s6[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            s6[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
            s6[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
        }
        for (int j = 0; j < 8; j++) {
            float step = d * (float)sc[j], off = dmin * (float)mn[j];
            for (int i = 0; i < 32; i++) {
                int q = step > 0.0f ? clampi((int)roundf((xb[j * 32 + i] + off) / step), 0, 15) : 0;
                uint8_t *p = qs + (j >> 1) * 32 + i;
                *p = (uint8_t)(*p | ((j & 1) ? (q << 4) : q));
            }
        }
    }
}

/* Q6_K: per 16-element group scale amax/31 stored as int8 relative to
 * fp16 d; q = round(x / (d*sc)) in [-32, 31], stored biased by 32.
 * Layout per src/vbs_dequant.c:316-333. */
void orc_quantize_q6_k(const float *x, size_t n_blocks, uint8_t *out) {
    for (size_t b = 0; b < n_blocks; b++) {
        const float *xb = x + b * 256;
        uint8_t *o = out + b * 210;
        float gs[16], smax = 0.0f;
        for (int g = 0; g < 16; g++) {
            float amax = 0.0f;
            for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(xb[g * 16 + i]));
            gs[g] = amax / 31.0f;
            smax = fmaxf(smax, gs[g]);
        }
        uint16_t dh = orc_f32_to_f16_rne(smax / 127.0f);
        float d = orc_f16_to_f32(dh);
        memset(o, 0, 210);
        uint8_t *ql = o, *qh = o + 128;
        for (int g = 0; g < 16; g++) {
            int sc = d > 0.0f ? clampi((int)roundf(gs[g] / d), 0, 127) : 0;
            o[192 + g] = (uint8_t)(int8_t)sc;
            float step = d * (float)sc;
            for (int i = 0; i < 16; i++) {
                int e = g * 16 + i;
                int q = step > 0.0f ? clampi((int)roundf(xb[e] / step), -32, 31) : 0;
                int u = q + 32;
                int half = e >> 7, quarter = (e >> 5) & 3, l = e & 31;
                ql[half * 64 + (quarter & 1) * 32 + l] |= (uint8_t)((u & 15) << ((quarter >> 1) * 4));
                qh[half * 32 + l] |= (uint8_t)((u >> 4) << (quarter * 2));
            }
        }
        wr16(o + 208, dh);
    }
}

int orc_synth_tensor(int type, uint64_t seed, uint64_t rows, uint64_t cols, uint64_t row0,
                     uint64_t col0, uint64_t full_cols, float scale, uint8_t *out) {
    uint64_t rb = orc_row_bytes(type, cols);
    if (!rb) return -1;
    float *tmp = (float *)malloc((size_t)cols * sizeof(float));
    if (!tmp) return -1;
    for (uint64_t r = 0; r < rows; r++) {
        orc_synth_f32(seed, 1, cols, row0 + r, col0, full_cols, scale, tmp);
        uint8_t *o = out + r * rb;
        size_t nb = (size_t)(cols / (uint64_t)orc_block_elems(type));
        switch (type) {
            case ORC_F32: memcpy(o, tmp, (size_t)cols * 4); break;
            case ORC_F16: for (uint64_t c = 0; c < cols; c++) wr16(o + c * 2, orc_f32_to_f16_rne(tmp[c])); break;
            case ORC_Q8_0: orc_quantize_q8_0(tmp, nb, o); break;
            case ORC_Q4_K: orc_quantize_q4_k(tmp, nb, o); break;
            case ORC_Q6_K: orc_quantize_q6_k(tmp, nb, o); break;
            default: free(tmp); return -1;
        }
    }
    free(tmp);
    return 0;
}
