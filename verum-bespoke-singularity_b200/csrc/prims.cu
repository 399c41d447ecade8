// prims.cu -- the decode step's non-matvec ops, with the op contracts of
// the reference's host math (src/vbs_host_math.h): embedding row (:136-142),
// RMSNorm (:28-36), RoPE (:38-51), SiLU*up (:53-57), add (:59-62), fp16 KV
// store (:150-159) and GQA decode attention (:170-209); plus the greedy
// argmax the engine does on the host (src/main.c:909-932).
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vbs {

// ---------------------------------------------------------------------------
// embedding: out[e] = dequant(row token)[e], exact
// ---------------------------------------------------------------------------
__global__ void embed_kernel(int type, const uint8_t *__restrict__ w, const uint32_t *token_dev, uint32_t token,
                             uint32_t rows, float *__restrict__ out, uint32_t dim, uint32_t *err) {
    pdl_wait();
    const uint32_t tok = token_dev ? *token_dev : token;
    if (tok >= rows) {
        if (blockIdx.x == 0 && threadIdx.x == 0) dev_flag_error(err, DERR_BAD_ARG);
        for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < dim; e += gridDim.x * blockDim.x) out[e] = 0.0f;
        pdl_launch_dependents();
        return;
    }
    const int E = block_elems(type), BB = block_bytes(type);
    const uint8_t *row = w + (uint64_t)tok * row_bytes(type, dim);
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < dim; e += gridDim.x * blockDim.x)
        out[e] = dq_elem(type, row + (uint64_t)(e / E) * BB, (int)(e % E));
    pdl_launch_dependents();
}

cudaError_t embed_launch(int type, const uint8_t *w, const uint32_t *token_dev, uint32_t token, uint32_t rows,
                         float *out, uint32_t dim, uint32_t *err, cudaStream_t st, bool pdl) {
    if (!block_elems(type) || dim % block_elems(type)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(1u, std::min(64u, (dim + 255) / 256)));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    note_launches(1);
    return cudaLaunchKernelEx(&cfg, embed_kernel, type, w, token_dev, token, rows, out, dim, err);
}

// n embedding rows at once (prompt chunks): block (x, b) covers part of the
// row of tokens_dev[b]; out is [n][dim].
__global__ void embed_rows_kernel(int type, const uint8_t *__restrict__ w, const uint32_t *__restrict__ tokens_dev,
                                  uint32_t rows, float *__restrict__ out, uint32_t dim, uint32_t *err) {
    const uint32_t tok = tokens_dev[blockIdx.y];
    float *o = out + (uint64_t)blockIdx.y * dim;
    if (tok >= rows) {
        if (blockIdx.x == 0 && threadIdx.x == 0) dev_flag_error(err, DERR_BAD_ARG);
        for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < dim; e += gridDim.x * blockDim.x) o[e] = 0.0f;
        return;
    }
    const int E = block_elems(type), BB = block_bytes(type);
    const uint8_t *row = w + (uint64_t)tok * row_bytes(type, dim);
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < dim; e += gridDim.x * blockDim.x)
        o[e] = dq_elem(type, row + (uint64_t)(e / E) * BB, (int)(e % E));
}

cudaError_t embed_rows_launch(int type, const uint8_t *w, const uint32_t *tokens_dev, uint32_t n, uint32_t rows,
                              float *out, uint32_t dim, uint32_t *err, cudaStream_t st) {
    if (!block_elems(type) || dim % block_elems(type) || !n) return cudaErrorInvalidValue;
    note_launches(1);
    embed_rows_kernel<<<dim3(std::max(1u, std::min(16u, (dim + 255) / 256)), n), 256, 0, st>>>(type, w, tokens_dev, rows,
                                                                                                out, dim, err);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// RMSNorm with double accumulation (src/vbs_host_math.h:28-36)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float *__restrict__ in, const float *__restrict__ w,
                                                       float *__restrict__ out, uint32_t n, float eps) {
    __shared__ double part[32];
    double ss = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += (double)in[i] * (double)in[i];
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) part[0] = v;
    }
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(part[0] / (double)n), eps)));
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(in[i], scale), w[i]);
}

cudaError_t rmsnorm_launch(const float *in, const float *w, float *out, uint32_t n, float eps, cudaStream_t st) {
    note_launches(1);
    rmsnorm_kernel<<<1, 1024, 0, st>>>(in, w, out, n, eps);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// RoPE on adjacent pairs (src/vbs_host_math.h:38-51)
// ---------------------------------------------------------------------------
__global__ void rope_kernel(float *x, uint32_t pos_arg, const uint32_t *ctrl, uint32_t hd, uint32_t nh, float theta) {
    const uint32_t pos = ctrl ? ctrl[0] : pos_arg;
    const uint32_t half = hd / 2, total = half * nh;
    for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < total; k += gridDim.x * blockDim.x) {
        const uint32_t h = k / half, i = (k % half) * 2;
        const float ang = __fmul_rn((float)pos, powf(theta, __fdiv_rn(-(float)i, (float)hd)));
        const float c = cosf(ang), s = sinf(ang);
        float *p = x + (size_t)h * hd + i;
        const float a = p[0], b = p[1];
        p[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        p[1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
}

cudaError_t rope_launch(float *x, uint32_t pos, const uint32_t *ctrl, uint32_t hd, uint32_t nh, float theta,
                        cudaStream_t st) {
    const uint32_t total = hd / 2 * nh;
    if (!total) return cudaSuccess;
    note_launches(1);
    rope_kernel<<<std::max(1u, std::min(1024u, (total + 255) / 256)), 256, 0, st>>>(x, pos, ctrl, hd, nh, theta);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// elementwise
// ---------------------------------------------------------------------------
__global__ void silu_mul_kernel(const float *g, const float *u, float *o, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        o[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i]))), u[i]);
}
__global__ void add_kernel(const float *a, const float *b, float *o, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        o[i] = __fadd_rn(a[i], b[i]);
}
__global__ void cache_store_kernel(const float *k, const float *v, uint16_t *kc, uint16_t *vc, uint32_t pos_arg,
                                   const uint32_t *ctrl, uint32_t layer, uint32_t max_ctx, uint32_t kv_dim,
                                   uint32_t head_dim, bool head_major) {
    const uint32_t pos = ctrl ? ctrl[0] : pos_arg;
    if (pos >= max_ctx) return;   // past the KV capacity (attention reports it)
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < kv_dim; i += gridDim.x * blockDim.x) {
        const uint64_t at = kv_index(head_major, layer, pos, i, max_ctx, kv_dim, head_dim);
        kc[at] = f32_to_f16_kv(k[i]);
        vc[at] = f32_to_f16_kv(v[i]);
    }
}

static unsigned ew_blocks(uint32_t n) { return std::max(1u, std::min(2048u, (n + 255) / 256)); }

cudaError_t silu_mul_launch(const float *g, const float *u, float *out, uint32_t n, cudaStream_t st) {
    if (!n) return cudaSuccess;
    note_launches(1);
    silu_mul_kernel<<<ew_blocks(n), 256, 0, st>>>(g, u, out, n);
    return cudaGetLastError();
}
cudaError_t add_launch(const float *a, const float *b, float *out, uint32_t n, cudaStream_t st) {
    if (!n) return cudaSuccess;
    note_launches(1);
    add_kernel<<<ew_blocks(n), 256, 0, st>>>(a, b, out, n);
    return cudaGetLastError();
}
cudaError_t cache_store_launch(const float *k, const float *v, uint16_t *kc, uint16_t *vc, uint32_t pos,
                               const uint32_t *ctrl, uint32_t layer, uint32_t max_ctx, uint32_t kv_dim,
                               uint32_t head_dim, bool head_major, cudaStream_t st) {
    if (!ctrl && pos >= max_ctx) return cudaErrorInvalidValue;
    if (!head_dim || kv_dim % head_dim) return cudaErrorInvalidValue;
    note_launches(1);
    cache_store_kernel<<<ew_blocks(kv_dim), 256, 0, st>>>(k, v, kc, vc, pos, ctrl, layer, max_ctx, kv_dim, head_dim,
                                                          head_major);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// greedy argmax (first maximum wins, src/vbs_cpu_main.c:78-80)
// ---------------------------------------------------------------------------
// Each CTA scans a contiguous slice; the last CTA to finish (atomic ticket)
// merges the CTA results in slice order and resets the ticket.
constexpr uint32_t AM_THREADS = 512, AM_MAX_CTAS = 64;

__device__ __forceinline__ void am_pick(float &best, uint32_t &bi, float ov, uint32_t oi) {
    if (oi != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
}

__device__ __forceinline__ void am_block_reduce(float &best, uint32_t &bi) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    for (int o = 16; o; o >>= 1) am_pick(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        const bool have = threadIdx.x < (blockDim.x >> 5);
        best = have ? sv[threadIdx.x] : -INFINITY;
        bi = have ? si[threadIdx.x] : 0xFFFFFFFFu;
        for (int o = 16; o; o >>= 1) am_pick(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    }
}

__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(const float *__restrict__ v, uint32_t n, uint32_t per,
                                                            uint32_t *out_token, uint32_t *ctrl, uint32_t *hist,
                                                            uint32_t hist_cap, uint32_t *work) {
    pdl_wait();
    const uint32_t lo = blockIdx.x * per, hi = min(n, lo + per);
    float best = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) am_pick(best, bi, v[i], i);
    am_block_reduce(best, bi);
    if (gridDim.x > 1) {
        // work: [0] ticket, [2 + 2c] value bits, [3 + 2c] index of CTA c
        __shared__ uint32_t last;
        if (threadIdx.x == 0) {
            work[2 + 2 * blockIdx.x] = __float_as_uint(best);
            work[3 + 2 * blockIdx.x] = bi;
            __threadfence();
            last = atomicAdd(&work[0], 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (!last) { pdl_launch_dependents(); return; }
        __threadfence();
        best = -INFINITY;
        bi = 0xFFFFFFFFu;
        if (threadIdx.x < gridDim.x) {
            best = __uint_as_float(__ldcg(&work[2 + 2 * threadIdx.x]));
            bi = __ldcg(&work[3 + 2 * threadIdx.x]);
        }
        am_block_reduce(best, bi);   // element indices: ties resolve to the first maximum
        if (threadIdx.x == 0) work[0] = 0u;
    }
    if (threadIdx.x == 0) {
        if (bi == 0xFFFFFFFFu) bi = 0;
        if (out_token) *out_token = bi;
        if (ctrl) {
            const uint32_t np = ctrl[0] + 1u;
            ctrl[1] = bi;
            ctrl[0] = np;
            if (hist && np < hist_cap) hist[np] = bi;
        }
    }
    pdl_launch_dependents();
}

size_t argmax_workspace_bytes() { return (2 + 2 * AM_MAX_CTAS) * sizeof(uint32_t); }

cudaError_t argmax_launch(const float *v, uint32_t n, uint32_t *out_token, uint32_t *ctrl, uint32_t *hist,
                          uint32_t hist_cap, void *work, cudaStream_t st, bool pdl) {
    if (!n) return cudaErrorInvalidValue;
    // slices of >= 4096 entries; one CTA without a workspace
    uint32_t ctas = work ? std::min(AM_MAX_CTAS, (n + 4095) / 4096) : 1u;
    const uint32_t per = (n + ctas - 1) / ctas;
    ctas = (n + per - 1) / per;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(AM_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    note_launches(1);
    return cudaLaunchKernelEx(&cfg, argmax_kernel, v, n, per, out_token, ctrl, hist, hist_cap,
                              static_cast<uint32_t *>(work));
}

}  // namespace vbs
