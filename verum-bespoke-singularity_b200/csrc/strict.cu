// strict.cu -- strict-parity decode kernels: the arithmetic of the
// reference's scalar CPU inference (src/vbs_cpu.c:572-639), reproduced so
// that greedy token ids match it exactly on small models. Built with
// -fmad=false and explicit round-to-nearest intrinsics (no FMA
// contraction, IEEE division and square root), integer-exact Q8 block dots,
// sequential float sums in the reference's order, an fp32 KV cache and the
// two-pass softmax. Transcendentals (expf, powf, sinf, cosf) are CUDA's own
// (<= 2 ulp from glibc's).
//
// Parallelism is spent only where the reference's result does not depend
// on order: integer dots, maxima, and independent rows/heads/elements.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vbs {

// quantize_q8 (src/vbs_cpu.c:166-182): one thread per 32-element block.
__global__ void strict_quantize_q8_kernel(const float *x, uint32_t cols, int8_t *xq, float *qd) {
    const uint32_t nb = cols / 32;
    for (uint32_t b = blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += gridDim.x * blockDim.x) {
        const float *xb = x + (size_t)b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i)
            if (fabsf(xb[i]) > amax) amax = fabsf(xb[i]);
        const float d = __fdiv_rn(amax, 127.0f);
        const float inv = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        for (int i = 0; i < 32; ++i) {
            int q = (int)roundf(__fmul_rn(xb[i], inv));
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            xq[(size_t)b * 32 + i] = (int8_t)q;
        }
        qd[b] = f16_exact(f32_to_f16_rne(d));
    }
}

cudaError_t strict_quantize_q8_launch(const float *x, uint32_t cols, int8_t *xq, float *qd, cudaStream_t st) {
    note_launches(1);
    strict_quantize_q8_kernel<<<std::max(1u, (cols / 32 + 127) / 128), 128, 0, st>>>(x, cols, xq, qd);
    return cudaGetLastError();
}

// vbs_hot_ref_matvec_q8_0 (src/hotkernels/vbs_hot_ref_impl.h:49-64): one warp
// per row; lanes form the exact int32 block dots and the per-block products
// (d_w * qd[b]) * dot, lane 0 sums them in block order.
constexpr int SQ_MAXB = 16;   // blocks per lane (cols <= 16384)
__global__ void strict_matvec_q8_0_kernel(const uint8_t *w, uint32_t rows, uint32_t cols, const int8_t *xq,
                                          const float *qd, float *y, int accumulate) {
    const int lane = threadIdx.x & 31;
    const uint32_t nb = cols / 32;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const uint8_t *row = w + (size_t)r * nb * 34;
        float term[SQ_MAXB];
#pragma unroll
        for (int k = 0; k < SQ_MAXB; ++k) {
            const uint32_t b = (uint32_t)k * 32 + lane;
            term[k] = 0.0f;
            if (b < nb) {
                const uint8_t *blk = row + (size_t)b * 34;
                int dot = 0;
                for (int i = 0; i < 32; ++i) dot += (int)(int8_t)blk[2 + i] * (int)xq[(size_t)b * 32 + i];
                term[k] = __fmul_rn(__fmul_rn(f16_exact(ld_u16(blk)), qd[b]), (float)dot);
            }
        }
        float sum = 0.0f;
        for (uint32_t b = 0; b < nb; ++b) {
            float t = 0.0f;
#pragma unroll
            for (int k = 0; k < SQ_MAXB; ++k)
                if ((b >> 5) == (uint32_t)k) t = term[k];
            t = __shfl_sync(0xffffffffu, t, b & 31);
            sum = __fadd_rn(sum, t);
        }
        if (lane == 0) y[r] = accumulate ? __fadd_rn(y[r], sum) : sum;
    }
}

cudaError_t strict_matvec_q8_0_launch(const uint8_t *w, uint32_t rows, uint32_t cols, const int8_t *xq, const float *qd,
                                      float *y, int accumulate, cudaStream_t st) {
    if (cols % 32 || cols / 32 > 32u * SQ_MAXB) return cudaErrorInvalidValue;
    note_launches(1);
    strict_matvec_q8_0_kernel<<<std::max(1u, (rows + 7) / 8), 256, 0, st>>>(w, rows, cols, xq, qd, y, accumulate);
    return cudaGetLastError();
}

// vbs_hot_ref_matvec_f32 (src/hotkernels/vbs_hot_ref_impl.h:110-118): one
// thread per row, sequential mul-then-add.
__global__ void strict_matvec_f32_kernel(const float *w, uint32_t rows, uint32_t cols, const float *x, float *y,
                                         int accumulate) {
    for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
        const float *wr = w + (size_t)r * cols;
        float sum = 0.0f;
        for (uint32_t i = 0; i < cols; ++i) sum = __fadd_rn(sum, __fmul_rn(wr[i], x[i]));
        y[r] = accumulate ? __fadd_rn(y[r], sum) : sum;
    }
}

cudaError_t strict_matvec_f32_launch(const float *w, uint32_t rows, uint32_t cols, const float *x, float *y,
                                     int accumulate, cudaStream_t st) {
    note_launches(1);
    strict_matvec_f32_kernel<<<std::max(1u, (rows + 63) / 64), 64, 0, st>>>(w, rows, cols, x, y, accumulate);
    return cudaGetLastError();
}

// rms_norm (src/vbs_cpu.c:251-262): sequential double sum of squares.
__global__ void strict_rmsnorm_kernel(const float *in, const float *w, float *out, uint32_t n, float eps) {
    __shared__ float scale;
    if (threadIdx.x == 0) {
        double sum = 0.0;
        for (uint32_t i = 0; i < n; ++i) sum = __dadd_rn(sum, __dmul_rn((double)in[i], (double)in[i]));
        const float mean = __double2float_rn(__ddiv_rn(sum, (double)n));
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(in[i], scale), w[i]);
}

cudaError_t strict_rmsnorm_launch(const float *in, const float *w, float *out, uint32_t n, float eps, cudaStream_t st) {
    note_launches(1);
    strict_rmsnorm_kernel<<<1, 256, 0, st>>>(in, w, out, n, eps);
    return cudaGetLastError();
}

// rope (src/vbs_cpu.c:264-275), position from ctrl[0].
__global__ void strict_rope_kernel(float *x, uint32_t nh, uint32_t hd, const uint32_t *ctrl, float theta) {
    const uint32_t pos = ctrl[0], half = hd / 2;
    for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < nh * half; k += gridDim.x * blockDim.x) {
        const uint32_t h = k / half, i = (k % half) * 2;
        const float ang = __fmul_rn((float)pos, powf(theta, __fdiv_rn(-(float)i, (float)hd)));
        const float c = cosf(ang), s = sinf(ang);
        float *p = x + (size_t)h * hd + i;
        const float a = p[0], b = p[1];
        p[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        p[1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
}

cudaError_t strict_rope_launch(float *x, uint32_t nh, uint32_t hd, const uint32_t *ctrl, float theta, cudaStream_t st) {
    note_launches(1);
    strict_rope_kernel<<<std::max(1u, (nh * hd / 2 + 127) / 128), 128, 0, st>>>(x, nh, hd, ctrl, theta);
    return cudaGetLastError();
}

// Attention with the fp32 cache (src/vbs_cpu.c:585-611): one block per
// query head. The block first writes its KV head's k/v at `pos` into the
// cache (blocks of the same group write identical values), then scores
// (sequential dot per position), max, exp, a sequential denominator, and
// the sequential weighted V sum per output element.
__global__ void strict_attention_kernel(const float *q, const float *k, const float *v, float *kcache, float *vcache,
                                        float *out, const uint32_t *ctrl, uint32_t layer, uint32_t context, uint32_t nqh,
                                        uint32_t nkh, uint32_t hd, float *scores_all, uint32_t *err) {
    const uint32_t h = blockIdx.x, pos = ctrl[0], kvd = nkh * hd;
    if (pos >= context) {
        if (h == 0 && threadIdx.x == 0) dev_flag_error(err, DERR_BAD_ARG);
        return;
    }
    const uint32_t groups = nqh / nkh, kh = h / groups;
    float *scores = scores_all + (size_t)h * context;
    const size_t here = ((size_t)layer * context + pos) * kvd + (size_t)kh * hd;
    for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
        kcache[here + i] = k[(size_t)kh * hd + i];
        vcache[here + i] = v[(size_t)kh * hd + i];
    }
    __syncthreads();
    const float att_scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
    const float *qh = q + (size_t)h * hd;
    for (uint32_t t = threadIdx.x; t <= pos; t += blockDim.x) {
        const float *kt = kcache + ((size_t)layer * context + t) * kvd + (size_t)kh * hd;
        float s = 0.0f;
        for (uint32_t i = 0; i < hd; ++i) s = __fadd_rn(s, __fmul_rn(qh[i], kt[i]));
        scores[t] = __fmul_rn(s, att_scale);
    }
    __syncthreads();
    __shared__ float red[256];
    float mx = -INFINITY;
    for (uint32_t t = threadIdx.x; t <= pos; t += blockDim.x) mx = fmaxf(mx, scores[t]);
    red[threadIdx.x] = mx;
    __syncthreads();
    __shared__ float denom_s, max_s;
    if (threadIdx.x == 0) {
        float m = -INFINITY;
        for (uint32_t i = 0; i < blockDim.x; ++i) m = fmaxf(m, red[i]);
        max_s = m;
    }
    __syncthreads();
    for (uint32_t t = threadIdx.x; t <= pos; t += blockDim.x) scores[t] = expf(__fsub_rn(scores[t], max_s));
    __syncthreads();
    if (threadIdx.x == 0) {
        float den = 0.0f;
        for (uint32_t t = 0; t <= pos; ++t) den = __fadd_rn(den, scores[t]);
        if (!isfinite(den) || den <= 0.0f) dev_flag_error(err, DERR_BAD_ARG);
        denom_s = den;
    }
    __syncthreads();
    const float den = denom_s;
    for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
        float o = 0.0f;
        for (uint32_t t = 0; t <= pos; ++t) {
            const float pt = __fdiv_rn(scores[t], den);
            o = __fadd_rn(o, __fmul_rn(pt, vcache[((size_t)layer * context + t) * kvd + (size_t)kh * hd + i]));
        }
        out[(size_t)h * hd + i] = o;
    }
}

cudaError_t strict_attention_launch(const float *q, const float *k, const float *v, float *kcache, float *vcache,
                                    float *out, const uint32_t *ctrl, uint32_t layer, uint32_t context, uint32_t nqh,
                                    uint32_t nkh, uint32_t hd, float *scores, uint32_t *err, cudaStream_t st) {
    note_launches(1);
    strict_attention_kernel<<<nqh, 256, 0, st>>>(q, k, v, kcache, vcache, out, ctrl, layer, context, nqh, nkh, hd,
                                                 scores, err);
    return cudaGetLastError();
}

// SiLU*up and residual add in the reference's form (src/vbs_cpu.c:626, :613).
__global__ void strict_silu_kernel(const float *g, const float *u, float *h, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        h[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i]))), u[i]);
}
__global__ void strict_add_kernel(float *x, const float *t, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], t[i]);
}

cudaError_t strict_silu_launch(const float *g, const float *u, float *h, uint32_t n, cudaStream_t st) {
    note_launches(1);
    strict_silu_kernel<<<std::max(1u, (n + 255) / 256), 256, 0, st>>>(g, u, h, n);
    return cudaGetLastError();
}
cudaError_t strict_add_launch(float *x, const float *t, uint32_t n, cudaStream_t st) {
    note_launches(1);
    strict_add_kernel<<<std::max(1u, (n + 255) / 256), 256, 0, st>>>(x, t, n);
    return cudaGetLastError();
}

}  // namespace vbs
