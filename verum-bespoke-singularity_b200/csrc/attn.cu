// attn.cu -- split-KV GQA decode attention over the fp16 KV cache.
//
// Op contract: the reference's vbs_host_attention (src/vbs_host_math.h:170-209):
// for each query head h of KV group g = h / (nqh/nkh),
//   out_h = sum_t softmax_t(scale * q_h . K[t]) V[t],  t < seq_len,
// K/V read from the fp16 cache of `layer` and widened to fp32.
//
// Work split (flash decoding): CTA = (kv head, split, sequence). A CTA streams
// its slice of positions of one KV head once and serves all G = nqh/nkh query
// heads of the group from it. Per-CTA results (m, l, o) -- running max in
// log2 units, softmax denominator, unnormalised output -- go to a workspace;
// the last CTA of a (sequence, kv head) to finish (atomic ticket) merges the
// splits in split order and resets its ticket, so no second launch is needed.
//
// Tensor-core kernel (head_dim 32/64/128, G <= 8), B200 design:
//  * K/V tiles of 16 positions per warp are staged into shared memory with
//    16-byte cp.async copies, several stages in flight per CTA. Rows are
//    padded by 16 bytes so ldmatrix reads are bank-conflict free.
//  * Scores and the weighted V sum are mma.sync m16n8k16 (f16 in, fp32
//    accumulate). fp32 accuracy with f16 operands: the 16 A rows carry each
//    query head twice, rows g = fp16(x) and g+8 = fp16(x - fp16(x)), so every
//    product is exact to ~2^-22 relative and the two halves are summed in
//    fp32 (K and V are fp16 already and need no split). The score fragment
//    of the first MMA is, register for register, the A fragment of the second.
//  * Online softmax per warp with a lazy rescale: the running maximum moves
//    (and the accumulators are rescaled) only when a block's maximum exceeds
//    it by more than 8 (log2 units), so exp2 weights stay <= 256.
//
// head_dim 256 (or more than 8 query heads per KV head) runs on the SIMT
// kernel: lanes grouped per position, online softmax per position.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vbs {

constexpr size_t ATTN_TICKET_BYTES = 64 * 1024;   // one ticket per (sequence, kv head)
constexpr uint32_t ATTN_MAX_SLOTS = ATTN_TICKET_BYTES / 4;
constexpr int ATTN_GS = 8;                         // query-head slots per KV head
constexpr uint32_t ATTN_MAX_SPLITS = 128;
constexpr float ATTN_LAZY = 8.0f;                  // rescale threshold (log2 units)

// Per-head state rows, [m, l, pad, pad, o[HD]]: o 16-byte aligned.
template <int HD> struct AttnRow { static constexpr int RS = 4 + HD; };

struct KvSlice {
    const uint16_t *k, *v;   // position 0 of (sequence, layer, kv head)
    uint64_t ps;             // elements between consecutive positions
};

__device__ __forceinline__ KvSlice attn_slice(const AttnParams &p, uint32_t bq, uint32_t kvh) {
    const uint64_t kv_dim = (uint64_t)p.nkh * p.hd;
    uint64_t off = (uint64_t)bq * p.kv_batch_stride + (uint64_t)p.layer * p.max_ctx * kv_dim;
    off += p.head_major ? (uint64_t)kvh * p.max_ctx * p.hd : (uint64_t)kvh * p.hd;
    return KvSlice{p.kc + off, p.vc + off, p.head_major ? (uint64_t)p.hd : kv_dim};
}

__device__ __forceinline__ uint32_t attn_seq(const AttnParams &p, uint32_t bq) {
    uint32_t seq = (p.seq_dev ? (*p.seq_dev + 1u) : p.seq_len) + bq * p.seq_step;
    if (seq > p.max_ctx) {   // never read past the cache; report instead
        if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) dev_flag_error(p.err, DERR_BAD_ARG);
        seq = p.max_ctx;
    }
    return seq;
}

// ---------------------------------------------------------------------------
// Merge of the CTA's warp states and of the splits.
// sh: [nw][ATTN_GS][RS] warp states (m, l, o) for heads g < G; reused as
// scratch for the split weights afterwards (needs ATTN_GS*(ATTN_MAX_SPLITS+2)
// floats).
// ---------------------------------------------------------------------------
template <int HD>
__device__ void attn_tail(const AttnParams &p, uint32_t n_splits, float *sh, int nw, uint32_t G, uint32_t kvh,
                          uint32_t split, uint32_t bq) {
    constexpr int RS = AttnRow<HD>::RS;
    uint32_t *counters = reinterpret_cast<uint32_t *>(p.work);
    float *work = reinterpret_cast<float *>(static_cast<char *>(p.work) + ATTN_TICKET_BYTES);
    const uint32_t slot = bq * p.nkh + kvh;
    constexpr size_t part_stride = (size_t)ATTN_GS * RS;
    float *mypart = work + ((size_t)slot * n_splits + split) * part_stride;
    float *outp = p.out + ((size_t)bq * p.nqh + kvh * G) * HD;
    for (uint32_t k = threadIdx.x; k < G * HD; k += blockDim.x) {
        const uint32_t g = k / HD, d = k % HD;
        float M = -INFINITY;
        for (int w = 0; w < nw; ++w) M = fmaxf(M, sh[(w * ATTN_GS + g) * RS]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < nw; ++w) {
            const float *r = sh + (w * ATTN_GS + g) * RS;
            const float a = (r[0] == -INFINITY) ? 0.f : exp2f(r[0] - M);
            L += r[1] * a;
            O += r[4 + d] * a;
        }
        if (n_splits == 1) {
            outp[g * HD + d] = O / L;
        } else {
            if (d == 0) { mypart[g * RS] = M; mypart[g * RS + 1] = L; }
            mypart[g * RS + 4 + d] = O;
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
    // split weights w[g][s] = exp2(m_s - M_g), one warp per head; every
    // load of a phase is issued before any is used (one L2 round trip each)
    float *wsm = sh;                                  // [ATTN_GS][n_splits]
    float *Lg = sh + ATTN_GS * ATTN_MAX_SPLITS;       // [ATTN_GS]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    static_assert(ATTN_MAX_SPLITS <= 128, "four splits per lane");
    for (uint32_t g = warp; g < G; g += nwarps) {
        float ms[4], ls[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t s2 = lane + 32 * k;
            const float *ps = parts + s2 * part_stride + g * RS;
            ms[k] = s2 < n_splits ? __ldcg(ps) : -INFINITY;
            ls[k] = s2 < n_splits ? __ldcg(ps + 1) : 0.f;
        }
        const float M = warp_max(fmaxf(fmaxf(ms[0], ms[1]), fmaxf(ms[2], ms[3])));
        float L = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t s2 = lane + 32 * k;
            const float a = (ms[k] == -INFINITY) ? 0.f : exp2f(ms[k] - M);
            if (s2 < n_splits) wsm[g * n_splits + s2] = a;
            L += ls[k] * a;
        }
        L = warp_sum(L);
        if (lane == 0) Lg[g] = L;
    }
    __syncthreads();
    // outputs, 4 consecutive dims per thread, 16 splits' loads in flight
    constexpr uint32_t MB = 16;
    for (uint32_t k = threadIdx.x; k < G * HD / 4; k += blockDim.x) {
        const uint32_t g = k / (HD / 4), d = (k % (HD / 4)) * 4;
        const float *src = parts + g * RS + 4 + d;
        const float *wg = wsm + g * n_splits;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t s0 = 0; s0 < n_splits; s0 += MB) {
            float4 v[MB];
#pragma unroll
            for (uint32_t u = 0; u < MB; ++u)
                v[u] = s0 + u < n_splits ? __ldcg(reinterpret_cast<const float4 *>(src + (s0 + u) * part_stride))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (uint32_t u = 0; u < MB; ++u) {
                const float a = s0 + u < n_splits ? wg[s0 + u] : 0.f;
                acc.x = fmaf(v[u].x, a, acc.x); acc.y = fmaf(v[u].y, a, acc.y);
                acc.z = fmaf(v[u].z, a, acc.z); acc.w = fmaf(v[u].w, a, acc.w);
            }
        }
        const float il = 1.0f / Lg[g];
        *reinterpret_cast<float4 *>(outp + g * HD + d) = make_float4(acc.x * il, acc.y * il, acc.z * il, acc.w * il);
    }
    if (threadIdx.x == 0) counters[slot] = 0u;
    pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// tensor-core kernel
// ---------------------------------------------------------------------------
template <int HD> struct AttnMma {
    static constexpr int NW = 4;                       // warps per CTA
    static constexpr int SP = 16 * NW;                 // positions per stage (16 per warp)
    static constexpr int RSB = HD * 2 + 16;            // staged row bytes (padded)
    static constexpr int STAGE = 2 * SP * RSB;         // K rows, then V rows
    static constexpr int NST = HD >= 128 ? 3 : (HD >= 64 ? 5 : 8);
    static constexpr int SMEM = NST * STAGE;
    static constexpr int CPR = HD * 2 / 16;            // 16-byte copies per row
    static_assert(SMEM >= NW * ATTN_GS * AttnRow<HD>::RS * 4, "state scratch");
    static_assert(SMEM >= ATTN_GS * (ATTN_MAX_SPLITS + 1) * 4, "merge scratch");
};

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// hi = fp16(a), lo = fp16(a - hi): a ~= hi + lo to ~2^-22 relative
__device__ __forceinline__ void split_h2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = pack_h2(a - f.x, b - f.y);
}

template <int HD>
__global__ void __launch_bounds__(AttnMma<HD>::NW * 32) attn_mma_kernel(const AttnParams p, uint32_t n_splits) {
    using C = AttnMma<HD>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t kvh = blockIdx.x, split = blockIdx.y, bq = blockIdx.z;
    const uint32_t G = p.nqh / p.nkh;
    const KvSlice kv = attn_slice(p, bq, kvh);

    pdl_wait();
    const uint32_t seq = attn_seq(p, bq);
    uint32_t per = (seq + n_splits - 1) / n_splits;
    per = (per + 15) & ~15u;
    const uint32_t t0 = min(seq, split * per), t1 = min(seq, t0 + per);
    const uint32_t nch = (t1 - t0 + C::SP - 1) / C::SP;
    const uint32_t sbase = smem_u32(smem);

    auto issue = [&](uint32_t c) {
        const uint32_t slot = sbase + (c % C::NST) * C::STAGE;
        const uint32_t pb = t0 + c * C::SP;
#pragma unroll 4
        for (int i = threadIdx.x; i < 2 * C::SP * C::CPR; i += C::NW * 32) {
            const int isv = i / (C::SP * C::CPR), r = (i / C::CPR) % C::SP, ch = i % C::CPR;
            const uint32_t t = pb + r;
            const bool ok = t < t1;
            const uint32_t tr = ok ? t : t0;
            const uint32_t cs = p.swz ? (ch ^ (tr & 7u)) : (uint32_t)ch;   // the row's 16-byte chunk in memory
            const uint16_t *src = (isv ? kv.v : kv.k) + (uint64_t)tr * kv.ps + cs * 8;
            cp_async16(slot + (isv * C::SP + r) * C::RSB + ch * 16, src, ok ? 16u : 0u);
        }
    };

    // q: A fragments, rows g = fp16(q), g+8 = fp16 remainder, pre-scaled by scale*log2(e)
    const int g = lane >> 2, qd = 2 * (lane & 3);
    const float qscale = p.scale * 1.4426950408889634f;
    uint32_t qa[HD / 16][4];
    {
        const bool has = (uint32_t)g < G;
        const float *qh = p.q + ((size_t)bq * p.nqh + kvh * G + (has ? g : 0)) * HD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float2 v = has ? *reinterpret_cast<const float2 *>(qh + 16 * kk + 8 * h + qd) : make_float2(0.f, 0.f);
                split_h2(v.x * qscale, v.y * qscale, qa[kk][2 * h], qa[kk][2 * h + 1]);
            }
        }
    }

#pragma unroll
    for (int c = 0; c < C::NST - 1; ++c) {
        if ((uint32_t)c < nch) issue(c);
        cp_async_commit();
    }

    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float mrun = -INFINITY, lrun = 0.f;

    for (uint32_t c = 0; c < nch; ++c) {
        if (c + C::NST - 1 < nch) issue(c + C::NST - 1);
        cp_async_commit();
        cp_async_wait<C::NST - 1>();
        __syncthreads();
        const uint32_t tb = t0 + c * C::SP + 16 * warp;
        if (tb < t1) {
            const uint32_t kst = sbase + (c % C::NST) * C::STAGE + 16 * warp * C::RSB;
            const uint32_t vst = kst + C::SP * C::RSB;
            float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk += 2) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kst + (8 * j + (lane & 7)) * C::RSB + (16 * kk + 8 * (lane >> 3)) * 2, b0, b1, b2, b3);
                    mma_f16_acc(s[j], qa[kk], b0, b1);
                    mma_f16_acc(s[j], qa[kk + 1], b2, b3);
                }
            }
            // scores of positions tb + {qd, qd+1, 8+qd, 9+qd} for head g
            float sc[4] = {s[0][0] + s[0][2], s[0][1] + s[0][3], s[1][0] + s[1][2], s[1][1] + s[1][3]};
            const uint32_t pq = tb + qd;
            if (pq >= t1) sc[0] = -INFINITY;
            if (pq + 1 >= t1) sc[1] = -INFINITY;
            if (pq + 8 >= t1) sc[2] = -INFINITY;
            if (pq + 9 >= t1) sc[3] = -INFINITY;
            float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            if (mx > mrun + ATTN_LAZY) {
                const float r = exp2f(mrun - mx);   // 0 on the first block
                lrun *= r;
#pragma unroll
                for (int n = 0; n < HD / 8; ++n) { o[n][0] *= r; o[n][1] *= r; o[n][2] *= r; o[n][3] *= r; }
                mrun = mx;
            }
            float pe[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) pe[e] = exp2f(sc[e] - mrun);
            lrun += (pe[0] + pe[1]) + (pe[2] + pe[3]);
            uint32_t pa[4];
            split_h2(pe[0], pe[1], pa[0], pa[1]);
            split_h2(pe[2], pe[3], pa[2], pa[3]);
#pragma unroll
            for (int n = 0; n < HD / 8; n += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(vst + ((lane & 7) + 8 * ((lane >> 3) & 1)) * C::RSB + (8 * n + 8 * (lane >> 4)) * 2, b0, b1,
                              b2, b3);
                mma_f16_acc(o[n], pa, b0, b1);
                mma_f16_acc(o[n + 1], pa, b2, b3);
            }
        }
        __syncthreads();
    }

    // warp states -> shared memory (the stage buffers are free: every copy
    // was waited for and the loop ended on a barrier)
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
    float *sh = reinterpret_cast<float *>(smem);
    constexpr int RS = AttnRow<HD>::RS;
    if ((uint32_t)g < G) {
        float *row = sh + (warp * ATTN_GS + g) * RS;
        if ((lane & 3) == 0) { row[0] = mrun; row[1] = lrun; }
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
            row[4 + 8 * n + qd] = o[n][0] + o[n][2];
            row[5 + 8 * n + qd] = o[n][1] + o[n][3];
        }
    }
    __syncthreads();
    attn_tail<HD>(p, n_splits, sh, C::NW, G, kvh, split, bq);
}

// ---------------------------------------------------------------------------
// SIMT kernel (any head_dim multiple of 8 up to 256 via the instances below)
// Lanes are grouped LP = HD/DPL per position; each lane holds DPL dims of
// q (pre-scaled by scale*log2 e), K and V, and an online-softmax state per
// head.
// ---------------------------------------------------------------------------
constexpr int AT_NW = 4;   // warps per CTA

template <int HD, int DPL, int GMAX>
__global__ void __launch_bounds__(AT_NW * 32) attn_simt_kernel(const AttnParams p, uint32_t n_splits) {
    constexpr int LP = HD / DPL, PPW = 32 / LP;
    constexpr int NV = DPL / 8;                    // uint4 (8 halves) per lane per row
    constexpr int RS = AttnRow<HD>::RS;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = lane / LP, sub = lane % LP;
    const uint32_t kvh = blockIdx.x, split = blockIdx.y, bq = blockIdx.z;
    const uint32_t G = p.nqh / p.nkh;
    const KvSlice kv = attn_slice(p, bq, kvh);

    pdl_wait();
    const uint32_t seq = attn_seq(p, bq);
    const uint32_t per = (seq + n_splits - 1) / n_splits;
    const uint32_t t0 = min(seq, split * per), t1 = min(seq, t0 + per);

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
    const uint16_t *kb = kv.k + sub * DPL, *vb = kv.v + sub * DPL;

    // K/V rows of the next position batch are loaded before the current
    // batch is used (two batches in flight per warp)
    auto load_rows = [&](uint32_t tb, uint4 *kr, uint4 *vr) {
        const uint32_t t = tb + grp;
        const bool valid = t < t1;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            kr[i] = valid ? __ldg(reinterpret_cast<const uint4 *>(kb + (uint64_t)t * kv.ps) + i) : make_uint4(0, 0, 0, 0);
            vr[i] = valid ? __ldg(reinterpret_cast<const uint4 *>(vb + (uint64_t)t * kv.ps) + i) : make_uint4(0, 0, 0, 0);
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
    __shared__ float sh[AT_NW * ATTN_GS * RS];
    static_assert(AT_NW * ATTN_GS * RS >= ATTN_GS * (ATTN_MAX_SPLITS + 1), "merge scratch");
    if (grp == 0) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            if (g >= (int)G) break;
            float *row = sh + (warp * ATTN_GS + g) * RS;
            if (sub == 0) { row[0] = m[g]; row[1] = l[g]; }
#pragma unroll
            for (int d = 0; d < DPL; ++d) row[4 + sub * DPL + d] = o[g][d];
        }
    }
    __syncthreads();
    attn_tail<HD>(p, n_splits, sh, AT_NW, G, kvh, split, bq);
}

// ---------------------------------------------------------------------------
// Fixed scratch of the no-allocation entry point (vbs_cu_attention_static):
// one per device, in the module's static device memory. Zero at module load;
// every launch leaves its merge tickets at zero again, and the split partials
// need no initial value.
// ---------------------------------------------------------------------------
constexpr size_t ATTN_STATIC_BYTES = 2u << 20;
static __device__ __align__(256) unsigned char g_attn_static[ATTN_STATIC_BYTES];

size_t attn_static_bytes() { return ATTN_STATIC_BYTES; }

// Device address of the fixed scratch on the current device.
cudaError_t attn_static_address(void **ptr) { return cudaGetSymbolAddress(ptr, g_attn_static); }

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t attn_workspace_bytes(uint32_t nqh, uint32_t nkh, uint32_t hd, uint32_t batch, uint32_t max_splits) {
    (void)nqh;
    return ATTN_TICKET_BYTES + (size_t)batch * nkh * max_splits * ATTN_GS * (4 + hd) * sizeof(float);
}

uint32_t attn_num_splits(uint32_t seq_len_hint, uint32_t nkh, uint32_t batch, int n_sm) {
    // two CTAs per SM; at least 64 positions per split
    const uint32_t target = (uint32_t)n_sm * 2u;
    uint32_t s = (target + nkh * batch - 1) / (nkh * batch);
    s = std::min(s, std::max(1u, (seq_len_hint + 63) / 64));
    return std::max(1u, std::min(s, ATTN_MAX_SPLITS));
}

static cudaLaunchConfig_t attn_cfg(dim3 grid, int threads, size_t smem, cudaStream_t st, bool pdl,
                                   cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

template <int HD>
static cudaError_t attn_mma_go(const AttnParams &p, uint32_t n_splits, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg =
        attn_cfg(dim3(p.nkh, n_splits, p.batch), AttnMma<HD>::NW * 32, AttnMma<HD>::SMEM, st, pdl, attr);
    note_launches(1);
    return cudaLaunchKernelEx(&cfg, attn_mma_kernel<HD>, p, n_splits);
}

template <int HD, int DPL, int GMAX>
static cudaError_t attn_simt_go(const AttnParams &p, uint32_t n_splits, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = attn_cfg(dim3(p.nkh, n_splits, p.batch), AT_NW * 32, 0, st, pdl, attr);
    note_launches(1);
    return cudaLaunchKernelEx(&cfg, attn_simt_kernel<HD, DPL, GMAX>, p, n_splits);
}

// ---------------------------------------------------------------------------
// Causal prompt-chunk attention (prefill): CTA = (kv head, 8 consecutive
// query tokens). Query token b of the chunk attends positions
// 0 .. seq_len + b - 1 (seq_step 1). Every KV tile of 64 positions is
// staged once per CTA and serves all 8 tokens of all G query heads of the
// group: warp w computes query head kvh * G + w for the 8 tokens.
//  * A rows: token r (0..7) as fp16(q), row r + 8 as the fp16 remainder, so
//    the products are exact to ~2^-22 relative as in attn_mma_kernel; P is
//    split the same way for p.V, and the two halves are summed in fp32.
//  * No split of the positions, so no merge: the CTA writes the outputs.
// The decode kernel, used for chunks before, is one CTA per token and
// re-reads the whole context for each of a chunk's tokens.
// ---------------------------------------------------------------------------
constexpr uint32_t APF_TOK = 8, APF_SP = 64, APF_NST = 3;
template <int HD> struct AttnPf {
    static constexpr uint32_t RSB = HD * 2 + 16;       // padded row: conflict-free ldmatrix
    static constexpr uint32_t STAGE = 2 * APF_SP * RSB;  // K rows then V rows
    static constexpr uint32_t SMEM = APF_NST * STAGE;
    static constexpr int CPR = HD * 2 / 16;
};

template <int HD>
__global__ void __launch_bounds__(ATTN_GS * 32, 1) attn_prefill_kernel(const AttnParams p) {
    using C = AttnPf<HD>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t kvh = blockIdx.x, b0 = blockIdx.y * APF_TOK;
    const uint32_t G = p.nqh / p.nkh, nthr = blockDim.x;
    const KvSlice kv = attn_slice(p, 0, kvh);
    const uint32_t blast = min(b0 + APF_TOK, p.batch) - 1;   // the CTA's last real token
    uint32_t t1 = p.seq_len + blast;                          // positions any of its tokens sees
    if (t1 > p.max_ctx) {
        if (threadIdx.x == 0) dev_flag_error(p.err, DERR_BAD_ARG);
        return;
    }
    const uint32_t nch = (t1 + APF_SP - 1) / APF_SP;
    const uint32_t sbase = smem_u32(smem);

    auto issue = [&](uint32_t c) {
        const uint32_t slot = sbase + (c % APF_NST) * C::STAGE;
        const uint32_t pb = c * APF_SP;
        for (uint32_t i = threadIdx.x; i < 2 * APF_SP * C::CPR; i += nthr) {
            const uint32_t isv = i / (APF_SP * C::CPR), r = (i / C::CPR) % APF_SP, ch = i % C::CPR;
            const uint32_t t = pb + r;
            const bool ok = t < t1;
            const uint32_t tr = ok ? t : 0u;
            const uint32_t cs = p.swz ? (ch ^ (tr & 7u)) : ch;
            const uint16_t *src = (isv ? kv.v : kv.k) + (uint64_t)tr * kv.ps + cs * 8;
            cp_async16(slot + (isv * APF_SP + r) * C::RSB + ch * 16, src, ok ? 16u : 0u);
        }
    };

    // q of token b0 + g, head kvh * G + warp: rows g = fp16(q), g + 8 = remainder
    const int g = lane >> 2, qd = 2 * (lane & 3);
    const uint32_t tok = b0 + g;
    const bool tok_ok = tok < p.batch;
    const uint32_t lim = p.seq_len + (tok_ok ? tok : blast);   // this row's positions: t < lim
    const float qscale = p.scale * 1.4426950408889634f;
    uint32_t qa[HD / 16][4];
    {
        const float *qh = p.q + (size_t)(tok_ok ? tok : blast) * p.nqh * HD + (size_t)(kvh * G + warp) * HD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float2 v = tok_ok ? *reinterpret_cast<const float2 *>(qh + 16 * kk + 8 * h + qd) : make_float2(0.f, 0.f);
                split_h2(v.x * qscale, v.y * qscale, qa[kk][2 * h], qa[kk][2 * h + 1]);
            }
        }
    }
#pragma unroll
    for (uint32_t c = 0; c < APF_NST - 1; ++c) {
        if (c < nch) issue(c);
        cp_async_commit();
    }
    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float mrun = -INFINITY, lrun = 0.f;

    for (uint32_t c = 0; c < nch; ++c) {
        if (c + APF_NST - 1 < nch) issue(c + APF_NST - 1);
        cp_async_commit();
        cp_async_wait<APF_NST - 1>();
        __syncthreads();
        const uint32_t kst = sbase + (c % APF_NST) * C::STAGE, vst = kst + APF_SP * C::RSB;
        const uint32_t tb = c * APF_SP;
        // scores: 8 blocks of 8 positions; rows g (hi) and g + 8 (lo) summed
        float sc[APF_SP / 8][2];
#pragma unroll
        for (int j = 0; j < (int)APF_SP / 8; ++j) {
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk += 2) {
                uint32_t b0r, b1r, b2r, b3r;
                ldsm_x4(kst + (8 * j + (lane & 7)) * C::RSB + (16 * kk + 8 * (lane >> 3)) * 2, b0r, b1r, b2r, b3r);
                mma_f16_acc(s4, qa[kk], b0r, b1r);
                mma_f16_acc(s4, qa[kk + 1], b2r, b3r);
            }
            const uint32_t pq = tb + 8 * j + qd;
            sc[j][0] = pq < lim ? s4[0] + s4[2] : -INFINITY;
            sc[j][1] = pq + 1 < lim ? s4[1] + s4[3] : -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < (int)APF_SP / 8; ++j) mx = fmaxf(mx, fmaxf(sc[j][0], sc[j][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (mx > mrun + ATTN_LAZY) {   // the first tile always holds position 0 of every row
            const float r = exp2f(mrun - mx);
            lrun *= r;
#pragma unroll
            for (int n = 0; n < HD / 8; ++n) { o[n][0] *= r; o[n][1] *= r; o[n][2] *= r; o[n][3] *= r; }
            mrun = mx;
        }
#pragma unroll
        for (int kc = 0; kc < (int)APF_SP / 16; ++kc) {
            const float p0 = exp2f(sc[2 * kc][0] - mrun), p1 = exp2f(sc[2 * kc][1] - mrun);
            const float p2 = exp2f(sc[2 * kc + 1][0] - mrun), p3 = exp2f(sc[2 * kc + 1][1] - mrun);
            lrun += (p0 + p1) + (p2 + p3);
            uint32_t pa[4];
            split_h2(p0, p1, pa[0], pa[1]);
            split_h2(p2, p3, pa[2], pa[3]);
#pragma unroll
            for (int n = 0; n < HD / 8; n += 2) {
                uint32_t b0r, b1r, b2r, b3r;
                ldsm_x4_trans(vst + (16 * kc + (lane & 7) + 8 * ((lane >> 3) & 1)) * C::RSB + (8 * n + 8 * (lane >> 4)) * 2,
                              b0r, b1r, b2r, b3r);
                mma_f16_acc(o[n], pa, b0r, b1r);
                mma_f16_acc(o[n + 1], pa, b2r, b3r);
            }
        }
        __syncthreads();
    }
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
    if (tok_ok) {
        const float il = 1.0f / lrun;
        float *dst = p.out + (size_t)tok * p.nqh * HD + (size_t)(kvh * G + warp) * HD;
#pragma unroll
        for (int n = 0; n < HD / 8; ++n)
            *reinterpret_cast<float2 *>(dst + 8 * n + qd) = make_float2((o[n][0] + o[n][2]) * il, (o[n][1] + o[n][3]) * il);
    }
}

bool attn_prefill_supported(const AttnParams &p) {
    return (p.hd == 64 || p.hd == 128) && p.head_major && p.nkh && p.nqh % p.nkh == 0 && p.nqh / p.nkh >= 1 &&
           p.nqh / p.nkh <= (uint32_t)ATTN_GS && p.seq_step == 1 && p.batch && !p.seq_dev && p.kv_batch_stride == 0;
}

cudaError_t attn_prefill_launch(const AttnParams &p, cudaStream_t st) {
    if (!attn_prefill_supported(p)) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(p.kc) | reinterpret_cast<uintptr_t>(p.vc) | reinterpret_cast<uintptr_t>(p.q) |
         reinterpret_cast<uintptr_t>(p.out)) & 15)
        return cudaErrorInvalidValue;
    note_launches(1);
    const dim3 grid(p.nkh, (p.batch + APF_TOK - 1) / APF_TOK);
    const uint32_t threads = 32 * (p.nqh / p.nkh);
    if (p.hd == 128) attn_prefill_kernel<128><<<grid, threads, AttnPf<128>::SMEM, st>>>(p);
    else attn_prefill_kernel<64><<<grid, threads, AttnPf<64>::SMEM, st>>>(p);
    return cudaGetLastError();
}

cudaError_t attn_configure() {
    cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnMma<32>::SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnMma<64>::SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnMma<128>::SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnPf<64>::SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnPf<128>::SMEM);
    return e;
}

cudaError_t attn_launch(const AttnParams &p, uint32_t n_splits, cudaStream_t st, bool pdl) {
    if (!p.nkh || !p.nqh || p.nqh % p.nkh || p.nqh / p.nkh > (uint32_t)ATTN_GS || !p.batch) return cudaErrorInvalidValue;
    if ((uint64_t)p.batch * p.nkh > ATTN_MAX_SLOTS || !n_splits || n_splits > ATTN_MAX_SPLITS) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(p.kc) | reinterpret_cast<uintptr_t>(p.vc) |
         reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.out)) & 15)
        return cudaErrorInvalidValue;
    if (p.kv_batch_stride % 8) return cudaErrorInvalidValue;   // keeps every sequence's rows 16-byte aligned
    if (p.swz && (!p.head_major || (p.hd != 64 && p.hd != 128))) return cudaErrorInvalidValue;   // 8+ chunks per row
    const uint32_t G = p.nqh / p.nkh;
    switch (p.hd) {
        case 32: return attn_mma_go<32>(p, n_splits, st, pdl);
        case 64: return attn_mma_go<64>(p, n_splits, st, pdl);
        case 128: return attn_mma_go<128>(p, n_splits, st, pdl);
        case 256: return G <= 4 ? attn_simt_go<256, 16, 4>(p, n_splits, st, pdl) : attn_simt_go<256, 16, 8>(p, n_splits, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace vbs
