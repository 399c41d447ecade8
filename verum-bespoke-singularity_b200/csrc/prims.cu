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
__global__ void cache_store_kernel(const float *k, const float *v, uint16_t *kc, uint16_t *vc, uint64_t base_arg,
                                   const uint32_t *ctrl, uint32_t layer, uint32_t max_ctx, uint32_t kv_dim) {
    if (ctrl && ctrl[0] >= max_ctx) return;   // past the KV capacity (attention reports it)
    const uint64_t base = ctrl ? ((uint64_t)layer * max_ctx + ctrl[0]) * kv_dim : base_arg;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < kv_dim; i += gridDim.x * blockDim.x) {
        kc[base + i] = f32_to_f16_kv(k[i]);
        vc[base + i] = f32_to_f16_kv(v[i]);
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
                               const uint32_t *ctrl, uint32_t layer, uint32_t max_ctx, uint32_t kv_dim, cudaStream_t st) {
    if (!kv_dim) return cudaSuccess;
    note_launches(1);
    cache_store_kernel<<<ew_blocks(kv_dim), 256, 0, st>>>(k, v, kc, vc, ((uint64_t)layer * max_ctx + pos) * kv_dim, ctrl,
                                                          layer, max_ctx, kv_dim);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// split-KV GQA decode attention (flash decoding)
//
// CTA = (kv head, split, sequence). The CTA streams its slice of the fp16
// K and V rows once and serves all G = nqh/nkh query heads of the group.
// Lanes are grouped LP = HD/DPL per position; each lane holds DPL dims of
// q (pre-scaled by scale*log2 e), K and V, and an online-softmax state per
// head. Partial (m, l, o) are merged across lane groups, warps and, through
// `work`, across splits: the last CTA of a (sequence, kv head) to finish
// (atomic ticket) merges the splits in split order and resets the ticket.
// ---------------------------------------------------------------------------
constexpr int AT_NW = 4;   // warps per CTA
constexpr size_t ATTN_TICKET_BYTES = 64 * 1024;        // one ticket per (sequence, kv head)
constexpr uint32_t ATTN_MAX_SLOTS = ATTN_TICKET_BYTES / 4;

template <int HD, int DPL, int GMAX>
__global__ void __launch_bounds__(AT_NW * 32) attn_kernel(const AttnParams p, uint32_t n_splits) {
    constexpr int LP = HD / DPL, PPW = 32 / LP;
    constexpr int NV = DPL / 8;                    // uint4 (8 halves) per lane per row
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = lane / LP, sub = lane % LP;
    const uint32_t kvh = blockIdx.x, split = blockIdx.y, bq = blockIdx.z;
    const uint32_t G = p.nqh / p.nkh;

    pdl_wait();
    uint32_t seq = p.seq_dev ? (*p.seq_dev + 1u) : p.seq_len;
    if (seq > p.max_ctx) {   // never read past the cache; report instead
        if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) dev_flag_error(p.err, DERR_BAD_ARG);
        seq = p.max_ctx;
    }
    const uint32_t per = (seq + n_splits - 1) / n_splits;
    const uint32_t t0 = split * per, t1 = min(seq, t0 + per);

    const float qscale = p.scale * 1.4426950408889634f;
    float qv[GMAX][DPL], o[GMAX][DPL], m[GMAX], l[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
        const float *qh = p.q + ((size_t)bq * p.nqh + kvh * G + (g < (int)G ? g : 0)) * HD + sub * DPL;
#pragma unroll
        for (int d = 0; d < DPL; ++d) {
            qv[g][d] = (g < (int)G) ? qh[d] * qscale : 0.f;
            o[g][d] = 0.f;
        }
    }
    const uint64_t lstride = (uint64_t)p.nkh * HD;   // elements per position
    const uint16_t *kb = p.kc + (uint64_t)bq * p.kv_batch_stride + (uint64_t)p.layer * p.max_ctx * lstride + kvh * HD + sub * DPL;
    const uint16_t *vb = p.vc + (uint64_t)bq * p.kv_batch_stride + (uint64_t)p.layer * p.max_ctx * lstride + kvh * HD + sub * DPL;

    // K/V rows of the next position batch are loaded before the current
    // batch is used (two batches in flight per warp)
    auto load_rows = [&](uint32_t tb, uint4 *kr, uint4 *vr) {
        const uint32_t t = tb + grp;
        const bool valid = t < t1;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            kr[i] = valid ? __ldg(reinterpret_cast<const uint4 *>(kb + (uint64_t)t * lstride) + i) : make_uint4(0, 0, 0, 0);
            vr[i] = valid ? __ldg(reinterpret_cast<const uint4 *>(vb + (uint64_t)t * lstride) + i) : make_uint4(0, 0, 0, 0);
        }
    };
    uint4 kr[NV], vr[NV], kn[NV], vn[NV];
    uint32_t tb = t0 + warp * PPW;
    if (tb < t1) load_rows(tb, kr, vr);
    for (; tb < t1; tb += AT_NW * PPW) {
        const uint32_t tnext = tb + AT_NW * PPW;
        if (tnext < t1) load_rows(tnext, kn, vn);
        const bool valid = tb + grp < t1;
        float kf[DPL], vf[DPL];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const uint32_t kw[4] = {kr[i].x, kr[i].y, kr[i].z, kr[i].w};
            const uint32_t vw[4] = {vr[i].x, vr[i].y, vr[i].z, vr[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&kw[j]));
                float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&vw[j]));
                kf[i * 8 + 2 * j] = a.x; kf[i * 8 + 2 * j + 1] = a.y;
                vf[i * 8 + 2 * j] = b.x; vf[i * 8 + 2 * j + 1] = b.y;
            }
        }
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            if (g >= (int)G) break;
            float s = 0.f;
#pragma unroll
            for (int d = 0; d < DPL; ++d) s = fmaf(qv[g][d], kf[d], s);
#pragma unroll
            for (int off = LP / 2; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            if (valid) {
                const float mn = fmaxf(m[g], s);
                const float r = exp2f(m[g] - mn), e = exp2f(s - mn);
                l[g] = fmaf(l[g], r, e);
#pragma unroll
                for (int d = 0; d < DPL; ++d) o[g][d] = fmaf(o[g][d], r, e * vf[d]);
                m[g] = mn;
            }
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) { kr[i] = kn[i]; vr[i] = vn[i]; }
    }

    // merge lane groups (same `sub`, different `grp`) within the warp
#pragma unroll
    for (int off = LP; off < 32; off <<= 1) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            if (g >= (int)G) break;
            const float m2 = __shfl_xor_sync(0xffffffffu, m[g], off);
            const float l2 = __shfl_xor_sync(0xffffffffu, l[g], off);
            const float mn = fmaxf(m[g], m2);
            const float a = (m[g] == -INFINITY) ? 0.f : exp2f(m[g] - mn);
            const float b = (m2 == -INFINITY) ? 0.f : exp2f(m2 - mn);
            l[g] = l[g] * a + l2 * b;
#pragma unroll
            for (int d = 0; d < DPL; ++d) {
                const float o2 = __shfl_xor_sync(0xffffffffu, o[g][d], off);
                o[g][d] = o[g][d] * a + o2 * b;
            }
            m[g] = mn;
        }
    }
    // merge warps through shared memory: [warp][g][2 + HD]
    __shared__ float sh[AT_NW][GMAX][2 + HD];
    if (grp == 0) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            if (g >= (int)G) break;
            if (sub == 0) { sh[warp][g][0] = m[g]; sh[warp][g][1] = l[g]; }
#pragma unroll
            for (int d = 0; d < DPL; ++d) sh[warp][g][2 + sub * DPL + d] = o[g][d];
        }
    }
    __syncthreads();
    // thread layout for the final stages: one thread per (g, d)
    // workspace: merge tickets first (fixed place, left at zero by every
    // launch), then the split partials
    uint32_t *counters = reinterpret_cast<uint32_t *>(p.work);
    float *work = reinterpret_cast<float *>(static_cast<char *>(p.work) + ATTN_TICKET_BYTES);
    const uint32_t slot = bq * p.nkh + kvh;
    const size_t part_stride = (size_t)GMAX * (2 + HD);
    float *mypart = work + ((size_t)slot * n_splits + split) * part_stride;
    for (uint32_t k = threadIdx.x; k < G * HD; k += blockDim.x) {
        const uint32_t g = k / HD, d = k % HD;
        float M = -INFINITY;
        for (int w = 0; w < AT_NW; ++w) M = fmaxf(M, sh[w][g][0]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < AT_NW; ++w) {
            const float a = (sh[w][g][0] == -INFINITY) ? 0.f : exp2f(sh[w][g][0] - M);
            L += sh[w][g][1] * a;
            O += sh[w][g][2 + d] * a;
        }
        if (n_splits == 1) {
            p.out[((size_t)bq * p.nqh + kvh * G + g) * HD + d] = O / L;
        } else {
            if (d == 0) { mypart[g * (2 + HD)] = M; mypart[g * (2 + HD) + 1] = L; }
            mypart[g * (2 + HD) + 2 + d] = O;
        }
    }
    if (n_splits == 1) { pdl_launch_dependents(); return; }
    __threadfence();
    __syncthreads();
    __shared__ uint32_t ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(&counters[slot], 1u);
    __syncthreads();
    if (ticket != n_splits - 1) { pdl_launch_dependents(); return; }
    __threadfence();
    const float *parts = work + (size_t)slot * n_splits * part_stride;
    // split weights a[g][s] = exp2(m_s - M_g) in shared memory (reusing sh)
    float *wsm = &sh[0][0][0];                      // AT_NW*GMAX*(2+HD) floats >= GMAX*(n_splits+2)
    __shared__ float Mg[GMAX], Lg[GMAX];
    if (threadIdx.x < G) {
        const uint32_t g = threadIdx.x;
        float M = -INFINITY;
        for (uint32_t s2 = 0; s2 < n_splits; ++s2) M = fmaxf(M, __ldcg(parts + s2 * part_stride + g * (2 + HD)));
        float L = 0.f;
        for (uint32_t s2 = 0; s2 < n_splits; ++s2) {
            const float *ps = parts + s2 * part_stride + g * (2 + HD);
            const float ms = __ldcg(ps);
            const float a = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
            wsm[g * n_splits + s2] = a;
            L += __ldcg(ps + 1) * a;
        }
        Mg[g] = M;
        Lg[g] = L;
    }
    __syncthreads();
    for (uint32_t k = threadIdx.x; k < G * HD; k += blockDim.x) {
        const uint32_t g = k / HD, d = k % HD;
        float O = 0.f;
        for (uint32_t s2 = 0; s2 < n_splits; ++s2)
            O = fmaf(__ldcg(parts + s2 * part_stride + g * (2 + HD) + 2 + d), wsm[g * n_splits + s2], O);
        p.out[((size_t)bq * p.nqh + kvh * G + g) * HD + d] = O / Lg[g];
    }
    if (threadIdx.x == 0) counters[slot] = 0u;
    pdl_launch_dependents();
}

size_t attn_workspace_bytes(uint32_t nqh, uint32_t nkh, uint32_t hd, uint32_t batch, uint32_t max_splits) {
    (void)nqh;
    const size_t gmax = 8;
    return ATTN_TICKET_BYTES + ((size_t)batch * nkh * max_splits * gmax * (2 + hd)) * sizeof(float);
}

uint32_t attn_num_splits(uint32_t seq_len_hint, uint32_t nkh, uint32_t batch, int n_sm) {
    const uint32_t target = (uint32_t)n_sm * 2u;
    uint32_t s = (target + nkh * batch - 1) / (nkh * batch);
    s = std::min(s, std::max(1u, (seq_len_hint + 63) / 64));
    // the merge keeps GMAX x n_splits weights in the CTA's shared scratch
    return std::max(1u, std::min(s, 128u));
}

template <int HD, int DPL, int GMAX>
static cudaError_t attn_go(const AttnParams &p, uint32_t n_splits, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nkh, n_splits, p.batch);
    cfg.blockDim = dim3(AT_NW * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    note_launches(1);
    return cudaLaunchKernelEx(&cfg, attn_kernel<HD, DPL, GMAX>, p, n_splits);
}

cudaError_t attn_launch(const AttnParams &p, uint32_t n_splits, cudaStream_t st, bool pdl) {
    if (!p.nkh || !p.nqh || p.nqh % p.nkh || p.nqh / p.nkh > 8 || !p.batch) return cudaErrorInvalidValue;
    if ((uint64_t)p.batch * p.nkh > ATTN_MAX_SLOTS) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(p.kc) | reinterpret_cast<uintptr_t>(p.vc)) & 15) return cudaErrorInvalidValue;
    const uint32_t G = p.nqh / p.nkh;
    switch (p.hd) {
        case 32: return G <= 4 ? attn_go<32, 8, 4>(p, n_splits, st, pdl) : attn_go<32, 8, 8>(p, n_splits, st, pdl);
        case 64: return G <= 4 ? attn_go<64, 16, 4>(p, n_splits, st, pdl) : attn_go<64, 8, 8>(p, n_splits, st, pdl);
        case 128: return G <= 4 ? attn_go<128, 16, 4>(p, n_splits, st, pdl) : attn_go<128, 8, 8>(p, n_splits, st, pdl);
        case 256: return G <= 4 ? attn_go<256, 16, 4>(p, n_splits, st, pdl) : attn_go<256, 16, 8>(p, n_splits, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// greedy argmax (first maximum wins, src/vbs_cpu_main.c:78-80)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ v, uint32_t n, uint32_t *out_token,
                                                      uint32_t *ctrl, uint32_t *hist, uint32_t hist_cap) {
    pdl_wait();
    float best = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = v[i];
        if (x > best || bi == 0xFFFFFFFFu) { best = x; bi = i; }
    }
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        const bool have = threadIdx.x < (blockDim.x >> 5);
        best = have ? sv[threadIdx.x] : -INFINITY;
        bi = have ? si[threadIdx.x] : 0xFFFFFFFFu;
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
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
    }
    pdl_launch_dependents();
}

cudaError_t argmax_launch(const float *v, uint32_t n, uint32_t *out_token, uint32_t *ctrl, uint32_t *hist,
                          uint32_t hist_cap, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    note_launches(1);
    return cudaLaunchKernelEx(&cfg, argmax_kernel, v, n, out_token, ctrl, hist, hist_cap);
}

}  // namespace vbs
