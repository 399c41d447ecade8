// mv.cu -- quantized matrix-vector kernels (the decode step's hot path).
//
// Op contract: y[r] = sum_c dequant(W)[r][c] * x[c], the reference's
// vbs_host_linear_tile (src/vbs_host_math.h:223-267) with W packed row-major
// in GGUF blocks (Q8_0 34 B / 32, Q4_K 144 B / 256, Q6_K 210 B / 256).
//
// Fast kernel (mv_fast_kernel), B200 design:
//  * One CTA per SM slice of rows. A producer warp streams the CTA's rows in
//    stages of 16 rows x 1024 columns from HBM into shared memory with 1-D
//    bulk copies (cp.async.bulk, the TMA engine; no tensor map, no
//    multicast), completing on mbarriers; the 16-byte-unaligned head and
//    tail of a row segment (Q6_K and Q8_0 rows are only 2-byte aligned)
//    are copied by the producer lanes with plain loads.
//  * x is quantized once per CTA into shared memory as two int8 levels per
//    32-element block: x ~= d2 * (254*q1 + q2), |error| <= amax/64516/2
//    (1.6e-5 of the block maximum). Weights stay in their packed form; the
//    int8 tensor-core MMA (m16n8k32, u8 x s8 -> s32) forms the exact
//    integer block dots, one MMA per 16 rows x 32 columns, so the per-weight
//    instruction cost is a mask and a fraction of an MMA. Block scales are
//    applied to the integer dots in fp32.
//  * Epilogues fuse what follows the matvec in the decode step: residual
//    add (accumulate), SiLU(gate)*up for the paired gate/up matrices, and
//    RoPE + fp16 KV-cache store for the fused Q/K/V projection.
//  * Programmatic dependent launch: the producer starts streaming weights
//    before griddepcontrol.wait; only the x prologue waits for the previous
//    kernel.
//
// Portable kernel (mv_generic_kernel): one warp per row, exact element
// dequantization (same float operation order as src/vbs_dequant.c), fp32
// FMA accumulation. Serves every type/shape/alignment the fast kernel does
// not, and batches.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vbs {

constexpr int MV_NCW = 8;                       // consumer warps
constexpr int MV_THREADS = (MV_NCW + 1) * 32;   // + one producer warp
constexpr uint32_t MV_CK = 1024;                // columns per stage (8 units of 128)
constexpr uint32_t MV_MAXST = 16;               // barrier slots
constexpr uint32_t MV_HDR = 2560;               // barriers, misc, reduction scratch
constexpr uint32_t MV_STAGE_BUDGET = 80 * 1024; // bytes of stages per CTA

template <int TYPE> struct MvT;
// Row slot stride: > chunk bytes + 2 x 15 alignment bytes, 16-byte multiple,
// stride/4 == 28 mod 32 so 8 rows x 4 lanes hit 32 distinct banks, and an
// odd number of 16-byte units for conflict-free ldmatrix.
template <> struct MvT<T_Q4_K> { static constexpr int E = 256, BB = 144, RS = 624; };
template <> struct MvT<T_Q6_K> { static constexpr int E = 256, BB = 210, RS = 880; };
template <> struct MvT<T_Q8_0> { static constexpr int E = 32, BB = 34, RS = 1136; };

__device__ __forceinline__ const uint8_t *seg_row_ptr(const MvParams &p, uint32_t row) {
    if (row < p.seg_end[0]) return p.w[0] + (uint64_t)row * p.rb;
    if (row < p.seg_end[1]) return p.w[1] + (uint64_t)(row - p.seg_end[0]) * p.rb;
    return p.w[2] + (uint64_t)(row - p.seg_end[1]) * p.rb;
}

__device__ __forceinline__ void sts_u8(uint32_t addr, uint8_t v) {
    asm volatile("st.shared.u8 [%0], %1;" ::"r"(addr), "r"((uint32_t)v) : "memory");
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ int lds_s8(uint32_t addr) {
    int16_t v;
    asm volatile("ld.shared.s8 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// ---------------------------------------------------------------------------
// x prologue: optional residual add and RMSNorm, then two-level int8
// quantization into the MMA B-fragment layout.
//   xq[J*64 + s*8 .. +8]: slot s<4: q1 bytes k=4s..4s+3 and k=16+4s..+3;
//                         slot 4+s: the same for q2.
//   xf[J] = {d2, d2 * sum(254 q1 + q2), sum_k<16, sum_k>=16} (floats/ints)
// ---------------------------------------------------------------------------
__device__ void mv_prologue(const MvParams &p, uint8_t *xq, float4 *xf, float *misc, int ctid) {
    const uint32_t nsub = p.cols / 32;
    float scale = 1.0f;
    if (p.norm_w) {
        float ss = 0.0f;
        for (uint32_t i = ctid; i < p.cols; i += MV_NCW * 32) {
            float v = p.x[i];
            if (p.x_add) v += p.x_add[i];
            ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        if ((ctid & 31) == 0) misc[8 + (ctid >> 5)] = ss;
        named_bar_sync(1, MV_NCW * 32);
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < MV_NCW; ++w) tot += misc[8 + w];
        scale = 1.0f / sqrtf(tot / (float)p.cols + p.eps);
    }
    const bool write_x = p.x_add && p.x_write && blockIdx.x == 0;
    for (uint32_t J = ctid; J < nsub; J += MV_NCW * 32) {
        float v[32];
        const float4 *x4 = reinterpret_cast<const float4 *>(p.x + (size_t)J * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 t = x4[i];
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
        if (p.x_add) {
            const float4 *a4 = reinterpret_cast<const float4 *>(p.x_add + (size_t)J * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float4 t = a4[i];
                v[4 * i] += t.x; v[4 * i + 1] += t.y; v[4 * i + 2] += t.z; v[4 * i + 3] += t.w;
            }
            if (write_x) {
                float4 *o4 = reinterpret_cast<float4 *>(p.x_write + (size_t)J * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
        }
        if (p.norm_w) {
            const float4 *w4 = reinterpret_cast<const float4 *>(p.norm_w + (size_t)J * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float4 t = w4[i];
                v[4 * i] = v[4 * i] * scale * t.x; v[4 * i + 1] = v[4 * i + 1] * scale * t.y;
                v[4 * i + 2] = v[4 * i + 2] * scale * t.z; v[4 * i + 3] = v[4 * i + 3] * scale * t.w;
            }
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        const float d2 = amax / (127.0f * 254.0f);
        const float d1 = d2 * 254.0f;
        const float r1 = d1 > 0.0f ? 1.0f / d1 : 0.0f, r2 = d2 > 0.0f ? 1.0f / d2 : 0.0f;
        uint32_t q1w[8], q2w[8];
        int s_lo = 0, s_hi = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) { q1w[i] = 0; q2w[i] = 0; }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            int a = __float2int_rn(v[i] * r1);
            a = max(-127, min(127, a));
            float res = fmaf(-(float)a, d1, v[i]);
            int b = __float2int_rn(res * r2);
            b = max(-127, min(127, b));
            q1w[i >> 2] |= (uint32_t)(a & 0xFF) << (8 * (i & 3));
            q2w[i >> 2] |= (uint32_t)(b & 0xFF) << (8 * (i & 3));
            if (i < 16) s_lo += 254 * a + b; else s_hi += 254 * a + b;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(xq + (size_t)J * 64);
        // slots s=0..3: {q1 word s, q1 word 4+s}; slots 4..7 the same for q2
        dst[0] = make_uint4(q1w[0], q1w[4], q1w[1], q1w[5]);
        dst[1] = make_uint4(q1w[2], q1w[6], q1w[3], q1w[7]);
        dst[2] = make_uint4(q2w[0], q2w[4], q2w[1], q2w[5]);
        dst[3] = make_uint4(q2w[2], q2w[6], q2w[3], q2w[7]);
        xf[J] = make_float4(d2, d2 * (float)(s_lo + s_hi), __int_as_float(s_lo), __int_as_float(s_hi));
    }
}

// Q4_K 6-bit scale/min of sub-block j from the header words s0,s1,s2
// (scales bytes 0-3, 4-7, 8-11), per src/vbs_dequant.c:225-233.
__device__ __forceinline__ void k4_sm(uint32_t s0, uint32_t s1, uint32_t s2, int j, float &sc, float &mn) {
    uint32_t a, b;
    if (j < 4) {
        a = (s0 >> (8 * j)) & 63u;
        b = (s1 >> (8 * j)) & 63u;
    } else {
        const int k = 8 * (j - 4);
        a = ((s2 >> k) & 15u) | (((s0 >> (k + 6)) & 3u) << 4);
        b = ((s2 >> (k + 4)) & 15u) | (((s1 >> (k + 6)) & 3u) << 4);
    }
    sc = (float)a;
    mn = (float)b;
}

// ---------------------------------------------------------------------------
// per-unit compute: one warp, 16 rows (matrix slot base `ms`), 128 columns
// starting at chunk-local element `eo` and x sub-block J0.
// acc[0], acc[1]: rows g, g+8 (lanes with (lane&3)==0 hold them; Q6_K
// splits each over lanes t=0,1).
// ---------------------------------------------------------------------------
template <int TYPE>
__device__ __forceinline__ void mv_unit(uint32_t ms, uint32_t pad0, uint32_t pad1, uint32_t eo, uint32_t J0,
                                        uint32_t xq, uint32_t xf, int lane, uint32_t nvalid_cols, float acc[2]) {
    constexpr int RS = MvT<TYPE>::RS;
    const int g = lane >> 2, t = lane & 3;
    if constexpr (TYPE == T_Q4_K) {
        const uint32_t sbl = eo >> 8, hh = (eo >> 7) & 1u;
        const uint4 h0 = lds_u128(ms + g * RS + sbl * 144);
        const uint4 h1 = lds_u128(ms + (g + 8) * RS + sbl * 144);
        const uint32_t lrow = (lane & 7) + ((lane >> 3) & 1) * 8, lcol = (lane >> 4) * 16;
        float f0 = 0.f, f1 = 0.f, m0 = 0.f, m1 = 0.f;
#pragma unroll
        for (int gg = 0; gg < 2; ++gg) {
            const uint32_t G = 2 * hh + gg;
            uint32_t a[4];
            ldsm_x4(ms + lrow * RS + sbl * 144 + 16 + 32 * G + lcol, a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t av[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) av[i] = half ? (a[i] & 0xF0F0F0F0u) : (a[i] & 0x0F0F0F0Fu);
                const uint32_t J = J0 + 2 * gg + half;
                uint2 bq = make_uint2(0u, 0u);
                if (lane < 8) bq = lds_u64(xq + J * 64 + lane * 8);
                int c[4];
                mma_u8s8(av, bq.x, bq.y, c);
                const uint2 xv = lds_u64(xf + J * 16);
                const float xd = __uint_as_float(xv.x) * (half ? 0.0625f : 1.0f), xs = __uint_as_float(xv.y);
                float sc0, mn0, sc1, mn1;
                k4_sm(h0.y, h0.z, h0.w, (int)(2 * G + half), sc0, mn0);
                k4_sm(h1.y, h1.z, h1.w, (int)(2 * G + half), sc1, mn1);
                f0 = fmaf((float)(c[0] * 254 + c[1]) * xd, sc0, f0);
                f1 = fmaf((float)(c[2] * 254 + c[3]) * xd, sc1, f1);
                m0 = fmaf(mn0, xs, m0);
                m1 = fmaf(mn1, xs, m1);
            }
        }
        acc[0] += f16f(h0.x & 0xFFFFu) * f0 - f16f(h0.x >> 16) * m0;
        acc[1] += f16f(h1.x & 0xFFFFu) * f1 - f16f(h1.x >> 16) * m1;
    } else if constexpr (TYPE == T_Q6_K) {
        const uint32_t sbl = eo >> 8, h = (eo >> 7) & 1u;
        const uint32_t b0 = ms + g * RS + pad0 + sbl * 210, b1 = ms + (g + 8) * RS + pad1 + sbl * 210;
        const float d0 = f16f(lds_u16(b0 + 208)), d1 = f16f(lds_u16(b1 + 208));
        float f0 = 0.f, f1 = 0.f;
        uint32_t qh[2][2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            qh[0][kk] = lds_u32_any(b0 + 128 + h * 32 + kk * 16 + 4 * t);
            qh[1][kk] = lds_u32_any(b1 + 128 + h * 32 + kk * 16 + 4 * t);
        }
#pragma unroll
        for (int qp = 0; qp < 2; ++qp) {          // ql run (q & 1)
            uint32_t ql[2][2];
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                ql[0][kk] = lds_u32_any(b0 + h * 64 + qp * 32 + kk * 16 + 4 * t);
                ql[1][kk] = lds_u32_any(b1 + h * 64 + qp * 32 + kk * 16 + 4 * t);
            }
#pragma unroll
            for (int qs = 0; qs < 2; ++qs) {      // nibble half (q >> 1)
                const int q = qs * 2 + qp;
                uint32_t av[4];
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk)
                        av[r + 2 * kk] = ((ql[r][kk] >> (4 * qs)) & 0x0F0F0F0Fu) |
                                         (((qh[r][kk] >> (2 * q)) & 0x03030303u) << 4);
                const uint32_t J = J0 + q;
                uint2 bq = make_uint2(0u, 0u);
                if (lane < 16) {
                    bq = lds_u64(xq + J * 64 + (lane & 7) * 8);
                    if (lane < 8) bq.y = 0u; else bq.x = 0u;
                }
                int c[4];
                mma_u8s8(av, bq.x, bq.y, c);
                const uint4 xv = lds_u128(xf + J * 16);
                const float xd = __uint_as_float(xv.x);
                const int sq = (t & 1) ? (int)xv.w : (int)xv.z;
                const uint32_t gi = h * 8 + q * 2 + (t & 1);
                const float sc0 = (float)lds_s8(b0 + 192 + gi), sc1 = (float)lds_s8(b1 + 192 + gi);
                f0 = fmaf((float)(c[0] * 254 + c[1] - 32 * sq) * xd, sc0, f0);
                f1 = fmaf((float)(c[2] * 254 + c[3] - 32 * sq) * xd, sc1, f1);
            }
        }
        acc[0] += d0 * f0;
        acc[1] += d1 * f1;
    } else {  // Q8_0: four 34-byte blocks
        const uint32_t blk0 = eo >> 5;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
            if ((uint32_t)kb * 32 >= nvalid_cols) break;
            const uint32_t b0 = ms + g * RS + pad0 + (blk0 + kb) * 34, b1 = ms + (g + 8) * RS + pad1 + (blk0 + kb) * 34;
            uint32_t av[4];
            av[0] = lds_u32_any(b0 + 2 + 4 * t);
            av[1] = lds_u32_any(b1 + 2 + 4 * t);
            av[2] = lds_u32_any(b0 + 18 + 4 * t);
            av[3] = lds_u32_any(b1 + 18 + 4 * t);
            const uint32_t J = J0 + kb;
            uint2 bq = make_uint2(0u, 0u);
            if (lane < 8) bq = lds_u64(xq + J * 64 + lane * 8);
            int c[4];
            mma_s8s8(av, bq.x, bq.y, c);
            const float xd = __uint_as_float(lds_u32(xf + J * 16));
            acc[0] = fmaf((float)(c[0] * 254 + c[1]), f16f(lds_u16(b0)) * xd, acc[0]);
            acc[1] = fmaf((float)(c[2] * 254 + c[3]), f16f(lds_u16(b1)) * xd, acc[1]);
        }
    }
}

// ---------------------------------------------------------------------------
// epilogue for one row (run by consumer warp 0, lane i = row in tile)
// ---------------------------------------------------------------------------
template <int EPI>
__device__ __forceinline__ void mv_epilogue(const MvParams &p, uint32_t row, bool valid, float va, float vb) {
    if constexpr (EPI == MV_EPI_STORE) {
        if (valid) p.y[row] = p.accumulate ? p.y[row] + va : va;
    } else if constexpr (EPI == MV_EPI_SILU) {
        if (valid) p.y[row] = va / (1.0f + expf(-va)) * vb;
    } else {  // QKV: q/k rows get RoPE on (2i, 2i+1) pairs; k/v go to the fp16 cache
        const float other = __shfl_xor_sync(0x0000FFFFu, va, 1);
        if (!valid) return;
        const uint32_t pos = p.ctrl[0];
        if (pos >= p.max_ctx) {   // position past the KV capacity: report, never write out of bounds
            dev_flag_error(p.err, DERR_BAD_ARG);
            return;
        }
        const uint64_t kvbase = ((uint64_t)p.layer * p.max_ctx + pos) * p.kv_dim;
        if (row >= p.seg_end[1]) {
            p.vc[kvbase + (row - p.seg_end[1])] = f32_to_f16_kv(va);
            return;
        }
        const bool is_q = row < p.seg_end[0];
        const uint32_t local = is_q ? row : row - p.seg_end[0];
        const uint32_t i = local % p.head_dim, ie = i & ~1u;
        const float ang = (float)pos * powf(p.theta, -(float)ie / (float)p.head_dim);
        float s, c;
        sincosf(ang, &s, &c);
        const float a = (i & 1u) ? other : va, b = (i & 1u) ? va : other;
        const float outv = (i & 1u) ? (a * s + b * c) : (a * c - b * s);
        if (is_q) p.q_out[local] = outv;
        else p.kc[kvbase + local] = f32_to_f16_kv(outv);
    }
}

template <int TYPE, int DUAL, int EPI>
__global__ void __launch_bounds__(MV_THREADS, 1) mv_fast_kernel(const MvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int E = MvT<TYPE>::E, BB = MvT<TYPE>::BB, RS = MvT<TYPE>::RS;
    constexpr int SLOTS = DUAL ? 32 : 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nsub = p.cols / 32, nstage = p.nstage;

    const uint32_t sbase = smem_u32(smem);
    float *misc = reinterpret_cast<float *>(smem + 256);          // 64 floats
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 256 + 60 * 4);
    float *red = reinterpret_cast<float *>(smem + 512);           // [2][8][32]
    uint8_t *xq = smem + MV_HDR;
    float4 *xf = reinterpret_cast<float4 *>(xq + (size_t)nsub * 64);
    const uint32_t xq_a = sbase + MV_HDR, xf_a = xq_a + nsub * 64;
    const uint32_t stage0 = (MV_HDR + nsub * 80 + 1023u) & ~1023u;
    const uint32_t stage_bytes = SLOTS * RS;
    auto full_bar = [&](uint32_t s) { return sbase + 8u * s; };
    auto empty_bar = [&](uint32_t s) { return sbase + 8u * (MV_MAXST + s); };
    auto stage_addr = [&](uint32_t s) { return sbase + stage0 + s * stage_bytes; };

    // rows of this CTA: an even-aligned balanced slice
    const uint32_t G = gridDim.x, b = blockIdx.x, hr = p.rows / 2;
    const uint32_t r0 = (uint32_t)(((uint64_t)b * hr) / G) * 2;
    const uint32_t r1 = (b + 1 == G) ? p.rows : (uint32_t)(((uint64_t)(b + 1) * hr) / G) * 2;
    const uint32_t nch = (p.cols + MV_CK - 1) / MV_CK;
    const uint32_t ntiles = (r1 - r0 + 15) / 16;
    const uint32_t nst = ntiles * nch;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < nstage; ++i) {
            mbar_init(full_bar(i), 1);
            mbar_init(empty_bar(i), MV_NCW);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == MV_NCW) {
        // ------------------------------ producer ------------------------------
        uint32_t issued = 0;
        for (uint32_t s = 0; s < nst; ++s) {
            const uint32_t slot = s % nstage;
            if (s >= nstage) {
                if (!mbar_wait_bounded(empty_bar(slot), ((s / nstage) - 1) & 1, kWaitNs)) {
                    if (lane == 0) { *abort_flag = 1; dev_flag_error(p.err, DERR_TIMEOUT_EMPTY); }
                    break;
                }
            }
            if (*abort_flag) break;
            const uint32_t tile = s / nch, ch = s % nch;
            const uint32_t c0 = ch * MV_CK, c1 = min(p.cols, c0 + MV_CK);
            const uint64_t boff = (uint64_t)(c0 / E) * BB, blen = (uint64_t)((c1 - c0) / E) * BB;
            const int mat = lane >> 4, ri = lane & 15;
            const uint32_t row = r0 + tile * 16 + ri;
            const bool valid = row < r1 && (DUAL || mat == 0);
            uint32_t tx = 0, dst_al = 0;
            uintptr_t lo = 0;
            if (valid) {
                const uint8_t *rp = mat ? (p.wb + (uint64_t)row * p.rb) : seg_row_ptr(p, row);
                const uintptr_t a = reinterpret_cast<uintptr_t>(rp + boff);
                lo = (a + 15) & ~(uintptr_t)15;
                const uintptr_t hi = (a + blen) & ~(uintptr_t)15;
                const uint32_t dst = stage_addr(slot) + (uint32_t)lane * RS + (uint32_t)(a & 15);
                if (hi > lo) {
                    tx = (uint32_t)(hi - lo);
                    dst_al = dst + (uint32_t)(lo - a);
                    for (uintptr_t q = a; q < lo; ++q) sts_u8(dst + (uint32_t)(q - a), __ldg(reinterpret_cast<const uint8_t *>(q)));
                    for (uintptr_t q = hi; q < a + blen; ++q) sts_u8(dst + (uint32_t)(q - a), __ldg(reinterpret_cast<const uint8_t *>(q)));
                } else {
                    for (uintptr_t q = a; q < a + blen; ++q) sts_u8(dst + (uint32_t)(q - a), __ldg(reinterpret_cast<const uint8_t *>(q)));
                }
            }
            __syncwarp();
            const uint32_t total = __reduce_add_sync(0xffffffffu, tx);
            if (lane == 0) mbar_arrive_expect_tx(full_bar(slot), total);
            __syncwarp();
            if (tx) bulk_g2s(dst_al, reinterpret_cast<const void *>(lo), tx, full_bar(slot));
            ++issued;
            if (issued == min(nst, nstage) && lane == 0) pdl_launch_dependents();
        }
        if (nst == 0 && lane == 0) pdl_launch_dependents();
        if (*abort_flag) {
            // drain copies that may still be in flight before the CTA exits
            const uint32_t first = issued > nstage ? issued - nstage : 0;
            for (uint32_t s = first; s < issued; ++s)
                mbar_wait_bounded(full_bar(s % nstage), (s / nstage) & 1, kWaitNs);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    const int ctid = threadIdx.x;
    pdl_wait();
    mv_prologue(p, xq, xf, misc, ctid);
    named_bar_sync(1, MV_NCW * 32);

    float accA[2] = {0.f, 0.f}, accB[2] = {0.f, 0.f};
    const int g = lane >> 2;
    for (uint32_t s = 0; s < nst; ++s) {
        const uint32_t slot = s % nstage;
        bool ok = !*abort_flag;
        if (ok && !mbar_wait_bounded(full_bar(slot), (s / nstage) & 1, kWaitNs)) {
            ok = false;
            if (lane == 0) { *abort_flag = 1; dev_flag_error(p.err, DERR_TIMEOUT_FULL); }
        }
        const uint32_t tile = s / nch, ch = s % nch;
        const uint32_t c0 = ch * MV_CK, c1 = min(p.cols, c0 + MV_CK);
        const uint32_t eo = (uint32_t)warp * 128;
        if (ok && c0 + eo < c1) {
            const uint32_t ms = stage_addr(slot);
            uint32_t pad0 = 0, pad1 = 0, padb0 = 0, padb1 = 0;
            if constexpr (TYPE != T_Q4_K) {
                const uint64_t boff = (uint64_t)(c0 / E) * BB;
                const uint32_t ra = min(r0 + tile * 16 + g, r1 - 1), rb_ = min(r0 + tile * 16 + g + 8, r1 - 1);
                pad0 = (uint32_t)(reinterpret_cast<uintptr_t>(seg_row_ptr(p, ra) + boff) & 15);
                pad1 = (uint32_t)(reinterpret_cast<uintptr_t>(seg_row_ptr(p, rb_) + boff) & 15);
                if constexpr (DUAL) {
                    padb0 = (uint32_t)(reinterpret_cast<uintptr_t>(p.wb + (uint64_t)ra * p.rb + boff) & 15);
                    padb1 = (uint32_t)(reinterpret_cast<uintptr_t>(p.wb + (uint64_t)rb_ * p.rb + boff) & 15);
                }
            }
            const uint32_t J0 = (c0 + eo) >> 5;
            mv_unit<TYPE>(ms, pad0, pad1, eo, J0, xq_a, xf_a, lane, c1 - c0 - eo, accA);
            if constexpr (DUAL) mv_unit<TYPE>(ms + 16 * RS, padb0, padb1, eo, J0, xq_a, xf_a, lane, c1 - c0 - eo, accB);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(slot));
        if (ch + 1 == nch) {
            // tile complete: reduce the 8 warps' partial row sums
            if constexpr (TYPE == T_Q6_K) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    accA[i] += __shfl_xor_sync(0xffffffffu, accA[i], 1);
                    if constexpr (DUAL) accB[i] += __shfl_xor_sync(0xffffffffu, accB[i], 1);
                }
            }
            float *rbuf = red + (tile & 1) * (MV_NCW * 32);
            if ((lane & 3) == 0) {
                rbuf[warp * 32 + g] = accA[0];
                rbuf[warp * 32 + g + 8] = accA[1];
                if constexpr (DUAL) {
                    rbuf[warp * 32 + 16 + g] = accB[0];
                    rbuf[warp * 32 + 24 + g] = accB[1];
                }
            }
            accA[0] = accA[1] = accB[0] = accB[1] = 0.f;
            named_bar_sync(1, MV_NCW * 32);
            if (warp == 0 && lane < 16) {
                float va = 0.f, vb = 0.f;
#pragma unroll
                for (int w = 0; w < MV_NCW; ++w) {
                    va += rbuf[w * 32 + lane];
                    if constexpr (DUAL) vb += rbuf[w * 32 + 16 + lane];
                }
                const uint32_t row = r0 + tile * 16 + lane;
                if (!*abort_flag) mv_epilogue<EPI>(p, row, row < r1, va, vb);
                else if constexpr (EPI == MV_EPI_QKV) (void)__shfl_xor_sync(0x0000FFFFu, va, 1);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// host side of the fast kernel
// ---------------------------------------------------------------------------

template <int TYPE> static uint32_t mv_smem_bytes(uint32_t cols, int dual, uint32_t nstage) {
    const uint32_t stage0 = (MV_HDR + (cols / 32) * 80 + 1023u) & ~1023u;
    return stage0 + nstage * (dual ? 32u : 16u) * (uint32_t)MvT<TYPE>::RS;
}
template <int TYPE> static uint32_t mv_nstage(int dual) {
    uint32_t sb = (dual ? 32u : 16u) * (uint32_t)MvT<TYPE>::RS;
    return std::max(2u, std::min(MV_MAXST, MV_STAGE_BUDGET / sb));
}

bool mv_fast_supported(int type, uint32_t rows, uint32_t cols, const void *const *w, int nw, const void *x,
                       int dual) {
    if (type != T_Q4_K && type != T_Q6_K && type != T_Q8_0) return false;
    if (rows == 0 || cols == 0 || cols % 32 || (block_elems(type) == 256 && cols % 256)) return false;
    if (reinterpret_cast<uintptr_t>(x) & 15) return false;
    for (int i = 0; i < nw; ++i) {
        if (!w[i]) return false;
        // ldmatrix needs 16-byte aligned rows in shared memory: Q4_K rows
        // must start 16-byte aligned in global memory too.
        if (type == T_Q4_K && (reinterpret_cast<uintptr_t>(w[i]) & 15)) return false;
    }
    uint32_t smem = 0;
    switch (type) {
        case T_Q4_K: smem = mv_smem_bytes<T_Q4_K>(cols, dual, mv_nstage<T_Q4_K>(dual)); break;
        case T_Q6_K: smem = mv_smem_bytes<T_Q6_K>(cols, dual, mv_nstage<T_Q6_K>(dual)); break;
        default: smem = mv_smem_bytes<T_Q8_0>(cols, dual, mv_nstage<T_Q8_0>(dual)); break;
    }
    return smem <= 227u * 1024u;
}

template <int TYPE, int DUAL, int EPI>
static cudaError_t mv_fast_go(const MvParams &p0, int n_sm, cudaStream_t st, bool pdl, int grid_override) {
    MvParams p = p0;
    p.nstage = mv_nstage<TYPE>(DUAL);
    const uint32_t smem = mv_smem_bytes<TYPE>(p.cols, DUAL, p.nstage);
    auto kern = mv_fast_kernel<TYPE, DUAL, EPI>;
    uint32_t grid = grid_override > 0 ? (uint32_t)grid_override
                                      : std::max(1u, std::min((uint32_t)n_sm, (p.rows + 1) / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    note_launches(1);
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int TYPE, int DUAL, int EPI> static cudaError_t mv_set_attr() {
    return cudaFuncSetAttribute(mv_fast_kernel<TYPE, DUAL, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t mv_configure() {
    const cudaError_t es[] = {
        mv_set_attr<T_Q4_K, 0, MV_EPI_STORE>(), mv_set_attr<T_Q4_K, 0, MV_EPI_QKV>(), mv_set_attr<T_Q4_K, 1, MV_EPI_SILU>(),
        mv_set_attr<T_Q6_K, 0, MV_EPI_STORE>(), mv_set_attr<T_Q6_K, 0, MV_EPI_QKV>(), mv_set_attr<T_Q6_K, 1, MV_EPI_SILU>(),
        mv_set_attr<T_Q8_0, 0, MV_EPI_STORE>(), mv_set_attr<T_Q8_0, 0, MV_EPI_QKV>(), mv_set_attr<T_Q8_0, 1, MV_EPI_SILU>()};
    for (cudaError_t e : es)
        if (e != cudaSuccess) return e;
    return cudaSuccess;
}

template <int TYPE>
static cudaError_t mv_fast_dispatch_t(int dual, int epi, const MvParams &p, int n_sm, cudaStream_t st, bool pdl,
                                      int go) {
    if (dual) return mv_fast_go<TYPE, 1, MV_EPI_SILU>(p, n_sm, st, pdl, go);
    if (epi == MV_EPI_QKV) return mv_fast_go<TYPE, 0, MV_EPI_QKV>(p, n_sm, st, pdl, go);
    return mv_fast_go<TYPE, 0, MV_EPI_STORE>(p, n_sm, st, pdl, go);
}

cudaError_t mv_fast_launch(int type, int dual, int epi, const MvParams &p, int n_sm, cudaStream_t st, bool pdl,
                           int grid_override) {
    switch (type) {
        case T_Q4_K: return mv_fast_dispatch_t<T_Q4_K>(dual, epi, p, n_sm, st, pdl, grid_override);
        case T_Q6_K: return mv_fast_dispatch_t<T_Q6_K>(dual, epi, p, n_sm, st, pdl, grid_override);
        case T_Q8_0: return mv_fast_dispatch_t<T_Q8_0>(dual, epi, p, n_sm, st, pdl, grid_override);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// portable kernel: warp per row, exact element dequant, fp32 FMA
// ---------------------------------------------------------------------------
template <int TYPE>
__global__ void __launch_bounds__(256) mv_generic_kernel(const uint8_t *__restrict__ w, const float *__restrict__ x,
                                                         float *__restrict__ y, uint32_t rows, uint32_t cols,
                                                         uint32_t batch, uint64_t xs, uint64_t ys, int accumulate) {
    constexpr int GB = 8;   // batch columns per pass
    const int lane = threadIdx.x & 31;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    const int E = block_elems(TYPE), BB = block_bytes(TYPE);
    const uint64_t rbytes = row_bytes(TYPE, cols);
    for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const uint8_t *row = w + (uint64_t)r * rbytes;
        for (uint32_t b0 = 0; b0 < batch; b0 += GB) {
            float acc[GB];
#pragma unroll
            for (int i = 0; i < GB; ++i) acc[i] = 0.f;
            for (uint32_t e = lane; e < cols; e += 32) {
                float wv;
                if constexpr (TYPE == T_F32) wv = reinterpret_cast<const float *>(row)[e];
                else wv = dq_elem(TYPE, row + (uint64_t)(e / E) * BB, (int)(e % E));
#pragma unroll
                for (int i = 0; i < GB; ++i)
                    if (b0 + i < batch) acc[i] = fmaf(wv, x[(uint64_t)(b0 + i) * xs + e], acc[i]);
            }
#pragma unroll
            for (int i = 0; i < GB; ++i) {
                float v = warp_sum(acc[i]);
                if (lane == 0 && b0 + i < batch) {
                    float *dst = y + (uint64_t)(b0 + i) * ys + r;
                    *dst = accumulate ? *dst + v : v;
                }
            }
        }
    }
}

cudaError_t mv_generic_launch(int type, const uint8_t *w, const float *x, float *y, uint32_t rows, uint32_t cols,
                              uint32_t batch, uint64_t x_stride, uint64_t y_stride, int accumulate, int n_sm,
                              cudaStream_t st) {
    uint32_t blocks = std::max(1u, std::min((uint32_t)n_sm * 8u, (rows + 7) / 8));
    note_launches(1);
#define VBS_GEN(T) mv_generic_kernel<T><<<blocks, 256, 0, st>>>(w, x, y, rows, cols, batch, x_stride, y_stride, accumulate)
    switch (type) {
        case T_F32: VBS_GEN(T_F32); break;
        case T_F16: VBS_GEN(T_F16); break;
        case T_Q4_0: VBS_GEN(T_Q4_0); break;
        case T_Q4_1: VBS_GEN(T_Q4_1); break;
        case T_Q8_0: VBS_GEN(T_Q8_0); break;
        case T_Q4_K: VBS_GEN(T_Q4_K); break;
        case T_Q6_K: VBS_GEN(T_Q6_K); break;
        default: return cudaErrorInvalidValue;
    }
#undef VBS_GEN
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// bit-exact dequantization (device twin of vbs_dequant_block)
// ---------------------------------------------------------------------------
__global__ void dequant_kernel(int type, const uint8_t *__restrict__ w, float *__restrict__ out, uint64_t n) {
    const int E = block_elems(type), BB = block_bytes(type);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = dq_elem(type, w + (i / E) * BB, (int)(i % E));
}

cudaError_t dequant_launch(int type, const uint8_t *w, float *out, uint64_t n, cudaStream_t st) {
    if (!block_elems(type)) return cudaErrorInvalidValue;
    uint64_t blocks = std::min<uint64_t>((n + 255) / 256, 65535ull * 8);
    if (!blocks) return cudaSuccess;
    note_launches(1);
    dequant_kernel<<<(unsigned)blocks, 256, 0, st>>>(type, w, out, n);
    return cudaGetLastError();
}

}  // namespace vbs
