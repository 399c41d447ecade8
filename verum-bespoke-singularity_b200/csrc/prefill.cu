// prefill.cu -- the per-chunk kernels of the batched prompt pass.
//
// The reference feeds a prompt one token at a time through forward_token
// (src/main.c:901-904), so every prompt token streams all weights once.
// The decoder's prefill instead takes the prompt in chunks of up to 512
// tokens: the matrices run through the tcgen05 GEMM (one weight pass per
// chunk), attention is the query-tiled causal kernel, and the kernels here
// do the row-wise rest: RMSNorm of each chunk row, and RoPE plus the fp16
// KV store at the rows' positions. The batch decoder (batch.cu) uses the
// same two for its B sequences at one position.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vbs {

// RMSNorm of `rows` rows of n floats, one CTA per row, with the arithmetic
// of rmsnorm_kernel (src/vbs_host_math.h:28-36: sum of squares in double).
// 256 threads per row for prompt chunks; 1024 when there are few rows (a
// decode batch), so the few CTAs still cover a row in a short loop.
__global__ void __launch_bounds__(1024) pf_rmsnorm_rows_kernel(const float *__restrict__ in, const float *__restrict__ w,
                                                               float *__restrict__ out, uint32_t n, float eps) {
    __shared__ double part[32];
    const float *x = in + (size_t)blockIdx.x * n;
    float *y = out + (size_t)blockIdx.x * n;
    double ss = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += (double)x[i] * (double)x[i];
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
    for (uint32_t k = 0; k < blockDim.x / 32; ++k) tot += part[k];
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(tot / (double)n), eps)));
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
}

cudaError_t pf_rmsnorm_rows_launch(const float *in, const float *w, float *out, uint32_t rows, uint32_t n, float eps,
                                   cudaStream_t st) {
    if (!rows || !n) return cudaSuccess;
    note_launches(1);
    pf_rmsnorm_rows_kernel<<<rows, rows < 64 ? 1024 : 256, 0, st>>>(in, w, out, n, eps);
    return cudaGetLastError();
}

// Row b sits at position p0 + b * pos_step (a prompt chunk: step 1; B
// sequences decoded in lockstep: step 0, each with its own cache seq_stride
// elements after the previous one): RoPE on its query heads in place and
// on its key heads (adjacent pairs, src/vbs_host_math.h:38-51, the rounding
// of rope_kernel), then its key and value rows go into the cache as fp16
// with the engine's rounding (src/vbs_host_math.h:150-159) in `layout`:
// 0 engine order, 1 head-major, 2 head-major with the step kernel's chunk
// swizzle. One CTA per row.
// q_in rows are qs floats apart, k and v rows ks apart (separate buffers,
// or the q|k|v rows of one fused projection); the RoPE'd queries go to q_out
// rows of nqh * hd (which may be q_in itself).
__global__ void __launch_bounds__(256) pf_rope_store_kernel(const float *q_in, float *q_out, uint32_t qs, const float *k,
                                                            const float *v, uint32_t ks, uint16_t *kc, uint16_t *vc,
                                                            uint32_t p0, uint32_t layer, uint32_t max_ctx, uint32_t nqh,
                                                            uint32_t nkh, uint32_t hd, float theta, int layout,
                                                            uint32_t pos_step, uint64_t seq_stride, const uint32_t *pos_dev) {
    const uint32_t b = blockIdx.x, pos = (pos_dev ? *pos_dev : p0) + b * pos_step, half = hd / 2;
    kc += b * seq_stride;
    vc += b * seq_stride;
    const float *qi = q_in + (size_t)b * qs;
    float *qb = q_out + (size_t)b * nqh * hd;
    const float *kb = k + (size_t)b * ks, *vb = v + (size_t)b * ks;
    auto rope = [&](float a, float c2, uint32_t i, float &o0, float &o1) {
        const float ang = __fmul_rn((float)pos, powf(theta, __fdiv_rn(-(float)i, (float)hd)));
        const float c = cosf(ang), s = sinf(ang);
        o0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(c2, s));
        o1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(c2, c));
    };
    for (uint32_t t = threadIdx.x + blockIdx.y * blockDim.x; t < (nqh + nkh) * half; t += blockDim.x * gridDim.y) {
        const bool isq = t < nqh * half;
        const uint32_t u = isq ? t : t - nqh * half, h = u / half, i = 2 * (u % half);
        if (isq) {
            const float *src = qi + (size_t)h * hd + i;
            float o0, o1;
            rope(src[0], src[1], i, o0, o1);
            qb[(size_t)h * hd + i] = o0;
            qb[(size_t)h * hd + i + 1] = o1;
            continue;
        }
        if (pos >= max_ctx) continue;   // the host checks capacity; never write past the cache
        const uint32_t local = h * hd + i;
        float k0, k1;
        rope(kb[local], kb[local + 1], i, k0, k1);
        // dims i, i+1 (i even) are adjacent in every layout: same 16-byte chunk
        const uint64_t at = layout == 2 ? kv_index_swz(layer, pos, local, max_ctx, nkh, hd)
                                        : kv_index(layout == 1, layer, pos, local, max_ctx, nkh * hd, hd);
        kc[at] = f32_to_f16_kv(k0);
        kc[at + 1] = f32_to_f16_kv(k1);
        vc[at] = f32_to_f16_kv(vb[local]);
        vc[at + 1] = f32_to_f16_kv(vb[local + 1]);
    }
}

cudaError_t pf_rope_store_launch(float *q, const float *k, const float *v, uint16_t *kc, uint16_t *vc, uint32_t rows,
                                 uint32_t p0, uint32_t layer, uint32_t max_ctx, uint32_t nqh, uint32_t nkh, uint32_t hd,
                                 float theta, int layout, cudaStream_t st) {
    if (!rows) return cudaSuccess;
    if (!hd || hd % 2 || p0 + rows > max_ctx || layout < 0 || layout > 2 || (layout == 2 && hd != 64 && hd != 128))
        return cudaErrorInvalidValue;
    note_launches(1);
    pf_rope_store_kernel<<<rows, 256, 0, st>>>(q, q, nqh * hd, k, v, nkh * hd, kc, vc, p0, layer, max_ctx, nqh, nkh, hd,
                                               theta, layout, 1u, 0, nullptr);
    return cudaGetLastError();
}

cudaError_t rope_store_seqs_launch(const float *q_in, float *q_out, uint32_t qs, const float *k, const float *v,
                                   uint32_t ks, uint16_t *kc, uint16_t *vc, uint32_t seqs, uint64_t seq_stride,
                                   const uint32_t *pos_dev, uint32_t layer, uint32_t max_ctx, uint32_t nqh, uint32_t nkh,
                                   uint32_t hd, float theta, cudaStream_t st) {
    if (!seqs) return cudaSuccess;
    if (!hd || hd % 2 || !pos_dev) return cudaErrorInvalidValue;
    note_launches(1);
    // few rows: each row's items over 8 CTAs
    pf_rope_store_kernel<<<dim3(seqs, seqs < 64 ? 8 : 1), 256, 0, st>>>(q_in, q_out, qs, k, v, ks, kc, vc, 0u, layer, max_ctx,
                                                                         nqh, nkh, hd, theta, 1, 0u, seq_stride, pos_dev);
    return cudaGetLastError();
}

}  // namespace vbs
