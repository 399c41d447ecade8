// mv_core.cuh -- the quantized dot-product core shared by the per-op matvec
// kernel (mv.cu) and the persistent decode-step kernel (step.cu): GGUF block
// geometry, shared-memory helpers and mv_unit, which turns one staged
// 16-row x 256-column unit of packed weights and the two-level int8 x into
// fp32 partial dot products on the int8 tensor cores.
#pragma once

#include "common.cuh"

namespace vbs {

// Bytes per 32-element block of the quantized x in shared memory, padded
// from 64 so the eight lanes carrying one MMA's B operand read distinct
// banks (slot layout: q1/q2 halves of slot i at 16i / 16i+8; plain layout:
// q1 words then q2 words). xf follows xq at nsub * XQ_MAX_STRIDE.
constexpr uint32_t XQ_SLOT_STRIDE = 72, XQ_PLAIN_STRIDE = 80, XQ_MAX_STRIDE = 80;
template <bool PLAIN> __host__ __device__ constexpr uint32_t xq_stride() { return PLAIN ? XQ_PLAIN_STRIDE : XQ_SLOT_STRIDE; }

// Q6_K super-block as repacked for the step kernel (224 bytes, 16-byte
// aligned): ql[128] | qh half 0 [32] | scales[16] | d | pad | qh half 1 [32],
// so the qh loads have the same lane offset pattern as the ql loads.
constexpr uint32_t Q6P_BYTES = 224, Q6P_SC = 160, Q6P_D = 176;
__host__ __device__ constexpr uint32_t q6p_qh(uint32_t h) { return 128u + 64u * h; }

template <int TYPE> struct MvT;
template <> struct MvT<T_Q4_K> { static constexpr int E = 256, BB = 144; };
template <> struct MvT<T_Q6_K> { static constexpr int E = 256, BB = 210; };
template <> struct MvT<T_Q8_0> { static constexpr int E = 32, BB = 34; };

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

// 16 bytes from a shared address that is only 2-byte aligned.
__device__ __forceinline__ uint4 lds128_any(uint32_t a) {
    const uint32_t off = a & 3u;
    if (off == 0) {
        if ((a & 15u) == 0) return lds_u128(a);
        return make_uint4(lds_u32(a), lds_u32(a + 4), lds_u32(a + 8), lds_u32(a + 12));
    }
    const uint32_t b = a - off, sh = off * 8;
    const uint32_t w0 = lds_u32(b), w1 = lds_u32(b + 4), w2 = lds_u32(b + 8), w3 = lds_u32(b + 12), w4 = lds_u32(b + 16);
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

// byte k of w as an exact float (magic-number conversion: 2^23 + byte).
__device__ __forceinline__ float byte_f(uint32_t w, uint32_t k) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | k)) - 8388608.0f;
}

// D += A(16x32, u8) * B(32x8, s8), int32 accumulate in place.
__device__ __forceinline__ void mma_u8s8_acc(const uint32_t a[4], uint32_t b0, uint32_t b1, int c[4]) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8_acc(const uint32_t a[4], uint32_t b0, uint32_t b1, int c[4]) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// per-unit compute. One warp, 16 rows (row slots r0s..r0s+15 of the stage
// at `ms`), one 256-element unit of the chunk starting at chunk-local
// element `eo` (global element e0, x block J0 = e0/32).
//
// Block-diagonal MMA: lane (g, t) = (lane/4, lane%4). Thread column t owns
// the k-slots 4t..4t+3 and 16+4t..19+4t of every m16n8k32 and fills them
// with weights of ITS OWN scale group; the B operand is nonzero only in the
// column pair (2t, 2t+1) = (q1, q2) of that group's x values. One MMA thus
// forms 4 groups' partial dots at once and every lane ends up holding the
// integer dots of one group for rows g and g+8 (C accumulates across the
// MMAs of a group), so the float scale epilogue runs once per (row, group)
// with no idle lanes. acc[0], acc[1] collect rows g, g+8.
// ---------------------------------------------------------------------------
// PACKED: rows come from the step kernel's repack (Q6_K in the 224-byte
// aligned layout above, no alignment pads); else GGUF rows as staged.
template <int TYPE, bool PACKED = false>
__device__ __forceinline__ void mv_unit(uint32_t ms, uint32_t RS, uint32_t pad0, uint32_t pad1, uint32_t eo,
                                        uint32_t J0, uint32_t xq, uint32_t xf, int lane, uint32_t nvalid,
                                        float acc[2]) {
    // every shared load of the unit is issued first (the loads are ordered
    // asm; the MMAs are free to be scheduled around them)
    const int g = lane >> 2, t = lane & 3;
    const bool bact = t == (g >> 1);       // this lane carries B column g (group g/2)
    const uint32_t lev = g & 1;           // ... for x level q1 (0) or q2 (1)
    const uint32_t rowA = ms + g * RS, rowB = rowA + 8 * RS;
    if constexpr (TYPE == T_Q4_K) {
        const uint32_t sa = rowA + (eo >> 8) * 144, sb = rowB + (eo >> 8) * 144;
        const uint4 hA = lds_u128(sa), hB = lds_u128(sb);
        const uint4 a0 = lds_u128(sa + 16 + 32 * t), a1 = lds_u128(sa + 32 + 32 * t);
        const uint4 b0 = lds_u128(sb + 16 + 32 * t), b1 = lds_u128(sb + 32 + 32 * t);
        const uint32_t bq = xq + (J0 + 2 * (g >> 1)) * XQ_SLOT_STRIDE + lev * 8;   // slot layout, lo sub-block
        uint2 blo[4], bhi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            blo[i] = bact ? lds_u64(bq + i * 16) : make_uint2(0u, 0u);
            bhi[i] = bact ? lds_u64(bq + XQ_SLOT_STRIDE + i * 16) : make_uint2(0u, 0u);
        }
        const uint4 fl = lds_u128(xf + (J0 + 2 * t) * 16), fh = lds_u128(xf + (J0 + 2 * t + 1) * 16);
        const uint32_t WA[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t WB[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        int clo[4] = {0, 0, 0, 0}, chi[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t alo[4] = {WA[i] & 0x0F0F0F0Fu, WB[i] & 0x0F0F0F0Fu, WA[4 + i] & 0x0F0F0F0Fu, WB[4 + i] & 0x0F0F0F0Fu};
            const uint32_t ahi[4] = {WA[i] & 0xF0F0F0F0u, WB[i] & 0xF0F0F0F0u, WA[4 + i] & 0xF0F0F0F0u, WB[4 + i] & 0xF0F0F0F0u};
            mma_u8s8_acc(alo, blo[i].x, blo[i].y, clo);
            mma_u8s8_acc(ahi, bhi[i].x, bhi[i].y, chi);
        }
        // this lane's sub-blocks: 2t (low nibbles) and 2t+1 (high nibbles, x16)
        const uint32_t k0 = (2 * t) & 3, k1 = k0 + 1;
        float r[2];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const uint4 h = rr ? hB : hA;
            // packed 6-bit scales/mins of sub-blocks 0-3 and 4-7 (src/vbs_dequant.c:225-233)
            const uint32_t sc = (t < 2) ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
            const uint32_t mn = (t < 2) ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
            const int *c = rr ? clo + 2 : clo;
            const int *ch = rr ? chi + 2 : chi;
            const float tl = (float)(c[0] * 254 + c[1]), th = (float)(ch[0] * 254 + ch[1]);
            const float f = tl * __uint_as_float(fl.x) * byte_f(sc, k0) + th * (__uint_as_float(fh.x) * 0.0625f) * byte_f(sc, k1);
            const float m = byte_f(mn, k0) * __uint_as_float(fl.y) + byte_f(mn, k1) * __uint_as_float(fh.y);
            r[rr] = f16f(h.x & 0xFFFFu) * f - f16f(h.x >> 16) * m;
        }
        acc[0] += r[0];
        acc[1] += r[1];
    } else if constexpr (TYPE == T_Q6_K) {
        // thread column t <-> (half h, l-half lh); its groups are (h, q, lh), q = 0..3
        const uint32_t h = t >> 1, lh = t & 1;
        constexpr uint32_t QB = PACKED ? Q6P_BYTES : 210u, SC = PACKED ? Q6P_SC : 192u, DO = PACKED ? Q6P_D : 208u;
        const uint32_t sa = rowA + pad0 + (eo >> 8) * QB, sb = rowB + pad1 + (eo >> 8) * QB;
        uint4 qlA0, qlA1, qlB0, qlB1, qhA, qhB;
        if constexpr (PACKED) {   // 16-byte aligned blocks
            qlA0 = lds_u128(sa + h * 64 + 16 * lh); qlA1 = lds_u128(sa + h * 64 + 32 + 16 * lh);
            qlB0 = lds_u128(sb + h * 64 + 16 * lh); qlB1 = lds_u128(sb + h * 64 + 32 + 16 * lh);
            qhA = lds_u128(sa + q6p_qh(h) + 16 * lh); qhB = lds_u128(sb + q6p_qh(h) + 16 * lh);
        } else {
            qlA0 = lds128_any(sa + h * 64 + 16 * lh); qlA1 = lds128_any(sa + h * 64 + 32 + 16 * lh);
            qlB0 = lds128_any(sb + h * 64 + 16 * lh); qlB1 = lds128_any(sb + h * 64 + 32 + 16 * lh);
            qhA = lds128_any(sa + 128 + h * 32 + 16 * lh); qhB = lds128_any(sb + 128 + h * 32 + 16 * lh);
        }
        // B: the lane carrying column g serves thread column tb = g/2 = (hb, lhb)
        const uint32_t tb = g >> 1, hb = tb >> 1, lhb = tb & 1;
        uint2 bw[4][2];
        uint4 fx[4];
        int scA[4], scB[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t bq = xq + (J0 + hb * 4 + q) * XQ_PLAIN_STRIDE + lev * 32 + lhb * 16;   // plain layout
            bw[q][0] = bact ? lds_u64(bq) : make_uint2(0u, 0u);
            bw[q][1] = bact ? lds_u64(bq + 8) : make_uint2(0u, 0u);
            fx[q] = lds_u128(xf + (J0 + h * 4 + q) * 16);
            const uint32_t gi = h * 8 + q * 2 + lh;
            scA[q] = lds_s8(sa + SC + gi);
            scB[q] = lds_s8(sb + SC + gi);
        }
        const uint32_t dA = lds_u16(sa + DO), dB = lds_u16(sb + DO);
        const uint32_t LA[2][4] = {{qlA0.x, qlA0.y, qlA0.z, qlA0.w}, {qlA1.x, qlA1.y, qlA1.z, qlA1.w}};
        const uint32_t LB[2][4] = {{qlB0.x, qlB0.y, qlB0.z, qlB0.w}, {qlB1.x, qlB1.y, qlB1.z, qlB1.w}};
        const uint32_t HA[4] = {qhA.x, qhA.y, qhA.z, qhA.w}, HB[4] = {qhB.x, qhB.y, qhB.z, qhB.w};
        float fA = 0.f, fB = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int c[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                uint32_t a[4];
                const int s = 4 * (q >> 1), hs = 2 * q;
                a[0] = ((LA[q & 1][2 * i] >> s) & 0x0F0F0F0Fu) | (((HA[2 * i] >> hs) & 0x03030303u) << 4);
                a[1] = ((LB[q & 1][2 * i] >> s) & 0x0F0F0F0Fu) | (((HB[2 * i] >> hs) & 0x03030303u) << 4);
                a[2] = ((LA[q & 1][2 * i + 1] >> s) & 0x0F0F0F0Fu) | (((HA[2 * i + 1] >> hs) & 0x03030303u) << 4);
                a[3] = ((LB[q & 1][2 * i + 1] >> s) & 0x0F0F0F0Fu) | (((HB[2 * i + 1] >> hs) & 0x03030303u) << 4);
                mma_u8s8_acc(a, bw[q][i].x, bw[q][i].y, c);
            }
            // this lane's group (h, q, lh): x block J0 + 4h + q, k-half lh
            const int sq = lh ? (int)fx[q].w : (int)fx[q].z;
            const float xd = __uint_as_float(fx[q].x);
            fA = fmaf((float)(c[0] * 254 + c[1] - 32 * sq) * xd, (float)scA[q], fA);
            fB = fmaf((float)(c[2] * 254 + c[3] - 32 * sq) * xd, (float)scB[q], fB);
        }
        acc[0] += f16f(dA) * fA;
        acc[1] += f16f(dB) * fB;
    } else {  // Q8_0: eight 34-byte blocks; thread column t owns blocks t and t+4
        const uint32_t blk0 = eo >> 5;
        uint4 ra[2][2], rb[2][2];
        uint2 bw[2][4];
        float xd[2];
        uint32_t hA[2], hB[2];
        bool mine[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t bi = (uint32_t)t + 4 * k;          // this lane's block
            const uint32_t bb = (uint32_t)(g >> 1) + 4 * k;   // block whose B column this lane carries
            mine[k] = bi * 32 < nvalid;
            const bool bvalid = bb * 32 < nvalid;
            const uint32_t sa = rowA + pad0 + (blk0 + bi) * 34, sb = rowB + pad1 + (blk0 + bi) * 34;
            const uint4 z = make_uint4(0, 0, 0, 0);
            ra[k][0] = mine[k] ? lds128_any(sa + 2) : z; ra[k][1] = mine[k] ? lds128_any(sa + 18) : z;
            rb[k][0] = mine[k] ? lds128_any(sb + 2) : z; rb[k][1] = mine[k] ? lds128_any(sb + 18) : z;
            hA[k] = mine[k] ? lds_u16(sa) : 0u;
            hB[k] = mine[k] ? lds_u16(sb) : 0u;
            xd[k] = mine[k] ? __uint_as_float(lds_u32(xf + (J0 + bi) * 16)) : 0.f;
            const uint32_t bq = xq + (J0 + bb) * XQ_SLOT_STRIDE + lev * 8;
#pragma unroll
            for (int i = 0; i < 4; ++i) bw[k][i] = (bact && bvalid) ? lds_u64(bq + i * 16) : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t WA[8] = {ra[k][0].x, ra[k][0].y, ra[k][0].z, ra[k][0].w, ra[k][1].x, ra[k][1].y, ra[k][1].z, ra[k][1].w};
            const uint32_t WB[8] = {rb[k][0].x, rb[k][0].y, rb[k][0].z, rb[k][0].w, rb[k][1].x, rb[k][1].y, rb[k][1].z, rb[k][1].w};
            int c[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t a[4] = {WA[i], WB[i], WA[4 + i], WB[4 + i]};
                mma_s8s8_acc(a, bw[k][i].x, bw[k][i].y, c);
            }
            if (mine[k]) {
                acc[0] = fmaf((float)(c[0] * 254 + c[1]), f16f(hA[k]) * xd[k], acc[0]);
                acc[1] = fmaf((float)(c[2] * 254 + c[3]), f16f(hB[k]) * xd[k], acc[1]);
            }
        }
    }
}

// Two-level int8 quantization of the 32-element block J: x ~= d2*(254*q1 + q2).
// The four lanes of `qmask` hold 8 consecutive values each (quarter u).
// Layouts per block (xq_stride bytes):
//   slot layout (Q4_K, Q8_0): slot s<4 = {q1 word s, q1 word 4+s} at 16s,
//     the same for q2 at 16s + 8 (word w = elements 4w..4w+3);
//   plain layout (Q6_K): q1 words 0..7 then q2 words 0..7.
//   xf[J] = {d2, d2 * sum(254 q1 + q2), sum over k<16, sum over k>=16}.
template <bool PLAIN>
__device__ __forceinline__ void quant_block8(const float v[8], uint32_t u, uint32_t qmask, uint32_t J, uint8_t *xq,
                                             float4 *xf) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 2));
    const float d2 = amax * (1.0f / (127.0f * 254.0f));
    const float d1 = d2 * 254.0f;
    float r1 = 0.0f, r2 = 0.0f;
    if (d2 > 0.0f) {   // approximate reciprocals: only the rounding of x changes, the scales d1, d2 are exact
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r2) : "f"(d2));
    }
    // Round to nearest even by adding 1.5 * 2^23: the float's low mantissa
    // bits are then the integer (two's complement in the low byte), and
    // t - 1.5 * 2^23 is that integer as an exact float. |q| <= 127 by the
    // choice of d1, d2; the clamps guard the approximate reciprocals.
    constexpr float kMagic = 12582912.0f;
    constexpr int kMagicBits = 0x4B400000;
    uint32_t t1[8], t2[8];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fminf(fmaxf(v[i] * r1, -127.0f), 127.0f) + kMagic;
        const float res = fmaf(-(a - kMagic), d1, v[i]);
        const float b = fminf(fmaxf(res * r2, -127.0f), 127.0f) + kMagic;
        t1[i] = __float_as_uint(a);
        t2[i] = __float_as_uint(b);
        sum += 254 * (__float_as_int(a) - kMagicBits) + (__float_as_int(b) - kMagicBits);
    }
    uint32_t q1w[2], q2w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {   // low bytes of four words -> one word
        q1w[k] = __byte_perm(__byte_perm(t1[4 * k], t1[4 * k + 1], 0x0040u), __byte_perm(t1[4 * k + 2], t1[4 * k + 3], 0x0040u), 0x5410u);
        q2w[k] = __byte_perm(__byte_perm(t2[4 * k], t2[4 * k + 1], 0x0040u), __byte_perm(t2[4 * k + 2], t2[4 * k + 3], 0x0040u), 0x5410u);
    }
    // this thread holds words 2u and 2u+1 of the block
    uint8_t *blk = xq + (size_t)J * xq_stride<PLAIN>();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint32_t w = 2 * u + k;
        if constexpr (PLAIN) {
            *reinterpret_cast<uint32_t *>(blk + 4 * w) = q1w[k];
            *reinterpret_cast<uint32_t *>(blk + 32 + 4 * w) = q2w[k];
        } else {
            const uint32_t off = (w & 3) * 16 + (w >> 2) * 4;
            *reinterpret_cast<uint32_t *>(blk + off) = q1w[k];
            *reinterpret_cast<uint32_t *>(blk + 8 + off) = q2w[k];
        }
    }
    const int other = __shfl_xor_sync(qmask, sum, 1);   // pairs (0,1) = k<16, (2,3) = k>=16
    const int half = sum + other;
    const int half_hi = __shfl_xor_sync(qmask, half, 2);
    if (u == 0) xf[J] = make_float4(d2, d2 * (float)(half + half_hi), __int_as_float(half), __int_as_float(half_hi));
}

// quant_block8 for two blocks J[0], J[1] of the same quad at once, their
// dependent chains (block maxima, shuffles, roundings) interleaved. Block 1
// is skipped (computed, not stored) when !has1; the quad's four lanes agree
// on has1, so the shuffles stay uniform.
template <bool PLAIN>
__device__ __forceinline__ void quant_block8x2(const float v[2][8], uint32_t u, uint32_t qmask, const uint32_t J[2],
                                               bool has1, uint8_t *xq, float4 *xf) {
    float amax[2] = {0.0f, 0.0f};
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int i = 0; i < 8; ++i) amax[b] = fmaxf(amax[b], fabsf(v[b][i]));
#pragma unroll
    for (int b = 0; b < 2; ++b) amax[b] = fmaxf(amax[b], __shfl_xor_sync(qmask, amax[b], 1));
#pragma unroll
    for (int b = 0; b < 2; ++b) amax[b] = fmaxf(amax[b], __shfl_xor_sync(qmask, amax[b], 2));
    constexpr float kMagic = 12582912.0f;
    constexpr int kMagicBits = 0x4B400000;
    float d2[2];
    int sum[2] = {0, 0};
    uint32_t q1w[2][2], q2w[2][2];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        d2[b] = amax[b] * (1.0f / (127.0f * 254.0f));
        const float d1 = d2[b] * 254.0f;
        float r1 = 0.0f, r2 = 0.0f;
        if (d2[b] > 0.0f) {   // approximate reciprocals, as quant_block8
            asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
            asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r2) : "f"(d2[b]));
        }
        uint32_t t1[8], t2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a = fminf(fmaxf(v[b][i] * r1, -127.0f), 127.0f) + kMagic;
            const float res = fmaf(-(a - kMagic), d1, v[b][i]);
            const float c = fminf(fmaxf(res * r2, -127.0f), 127.0f) + kMagic;
            t1[i] = __float_as_uint(a);
            t2[i] = __float_as_uint(c);
            sum[b] += 254 * (__float_as_int(a) - kMagicBits) + (__float_as_int(c) - kMagicBits);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            q1w[b][k] = __byte_perm(__byte_perm(t1[4 * k], t1[4 * k + 1], 0x0040u), __byte_perm(t1[4 * k + 2], t1[4 * k + 3], 0x0040u), 0x5410u);
            q2w[b][k] = __byte_perm(__byte_perm(t2[4 * k], t2[4 * k + 1], 0x0040u), __byte_perm(t2[4 * k + 2], t2[4 * k + 3], 0x0040u), 0x5410u);
        }
    }
    int half[2], half_hi[2];
#pragma unroll
    for (int b = 0; b < 2; ++b) half[b] = sum[b] + __shfl_xor_sync(qmask, sum[b], 1);
#pragma unroll
    for (int b = 0; b < 2; ++b) half_hi[b] = __shfl_xor_sync(qmask, half[b], 2);
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        if (b == 1 && !has1) break;
        uint8_t *blk = xq + (size_t)J[b] * xq_stride<PLAIN>();
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t w = 2 * u + k;
            if constexpr (PLAIN) {
                *reinterpret_cast<uint32_t *>(blk + 4 * w) = q1w[b][k];
                *reinterpret_cast<uint32_t *>(blk + 32 + 4 * w) = q2w[b][k];
            } else {
                const uint32_t off = (w & 3) * 16 + (w >> 2) * 4;
                *reinterpret_cast<uint32_t *>(blk + off) = q1w[b][k];
                *reinterpret_cast<uint32_t *>(blk + 8 + off) = q2w[b][k];
            }
        }
        if (u == 0)
            xf[J[b]] = make_float4(d2[b], d2[b] * (float)(half[b] + half_hi[b]), __int_as_float(half[b]), __int_as_float(half_hi[b]));
    }
}

}  // namespace vbs
