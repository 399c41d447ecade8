// mvb.cu -- batched quantized matvec: Y[b][r] = sum_c dequant(W)[r][c] * X[b][c]
// for b < B <= 8 (the BASELINE sweep's batched decode, x [B x cols]).
//
// The reference's op contract is vbs_host_linear_tile (src/vbs_host_math.h:
// 223-267) applied to each row of X. At B = 8 a weight element feeds 8
// products, so the work is a real (skinny) GEMM and runs on the tensor cores:
//  * Grid: (row blocks) x (column chunks of at most 4096). Each CTA streams
//    its rows' chunk in stages of 16 rows through a shared-memory ring (1-D
//    bulk TMA copies, one per row, issued by a producer warp; the copy
//    scheme of mv.cu).
//  * X: the CTA's chunk of every sequence as fp16 in shared memory (absent
//    sequences are zero), and for Q4_K the per-group sums of those fp16
//    values (the min term).
//  * mma.sync m16n8k16 f16 x f16 -> fp32, one MMA column per sequence. The A
//    operand holds the raw quants, exact in fp16: Q4_K 1024 + nibble (the
//    bits 0x6400 | n, formed by one mask; the bias goes out with the group's
//    x sum, which the min term needs anyway), Q6_K q - 32. The k-slots of an
//    MMA are permuted so that each lane's four weights are four consecutive
//    bytes and its x values one contiguous load (the dot product does not
//    care about the order of its terms); x is stored with each group of 4 in
//    the order (0, 2, 1, 3), so a mask of the weight word yields the pairs
//    directly. One MMA pair covers one Q4_K sub-block (32) and one MMA one
//    Q6_K scale group (16), so the group's dot gets its scale in fp32:
//    Q4_K y += d*sc * dot - (dmin*m + 1024*d*sc) * sum(x), Q6_K y += d*sc * dot.
//  * x in fp16 rounds each element by at most 2^-11 relative: the result is
//    within ~2.5e-4 of the exact dot (the batch-1 kernel's two-level int8
//    x is tighter; 1e-3 is the bar).
//  * Rows wider than one chunk: each chunk's sums go to a plane, and a small
//    kernel adds the planes in chunk order (deterministic).
#include "common.cuh"
#include "kernels.h"
#include "mv_core.cuh"

#include <algorithm>

namespace vbs {

constexpr int MB_NCW = 16;                       // consumer warps: one 256-column super-block each at 4096 columns
constexpr int MB_THREADS = (MB_NCW + 1) * 32;    // + one producer warp
constexpr uint32_t MB_B = 8;                     // sequences per MMA (the n dimension)
constexpr uint32_t MB_CK = 4096;                 // max columns per chunk
constexpr uint32_t MB_MAXST = 16;
constexpr uint32_t MB_SMEM = 227u * 1024u;
// shared memory: barriers [0, 256) | abort 256 | red [MB_NCW warps][16 rows][8 seqs] fp32 at 1024 |
// x fp16 [8][ck] | group sums [8][ck/16] fp32 | ring
constexpr uint32_t MB_NU = 4;                      // tiles whose row sums share one pair of consumer barriers
constexpr uint32_t MB_RED = 1024, MB_X = MB_RED + MB_NU * MB_NCW * 16 * MB_B * 4;

struct MbGeom {
    uint32_t ck, rs, nstage, stage0, nch, xs_off;
    uint32_t xstride;   // bytes per sequence's fp16 x row
};

template <int TYPE> __host__ __device__ constexpr uint32_t mb_group() { return TYPE == T_Q6_K ? 16u : 32u; }
// x row padding: the 8 lanes sharing a column offset read 8 sequences' rows;
// a row pad of 16 words (Q4_K: 16-byte loads by quarter warps) or 8 words
// (Q6_K: 8-byte loads by half warps) puts them in distinct banks
template <int TYPE> __host__ __device__ constexpr uint32_t mb_xpad() { return TYPE == T_Q6_K ? 32u : 64u; }

template <int TYPE> static MbGeom mb_geom(uint32_t cols) {
    MbGeom g = {};
    g.nch = (cols + MB_CK - 1) / MB_CK;
    g.ck = (cols + g.nch - 1) / g.nch;
    g.ck = (g.ck + 255) / 256 * 256;
    g.xstride = g.ck * 2 + mb_xpad<TYPE>();
    g.xs_off = MB_X + MB_B * g.xstride;
    g.stage0 = (g.xs_off + MB_B * (g.ck / mb_group<TYPE>()) * 4 + 1023u) & ~1023u;
    // stage row stride: Q4_K rows are read as 8-byte words by half warps
    // (rows g = 0..3, lanes t): a stride of 32 mod 128 bytes puts the four
    // rows in distinct banks. Q6_K (4-byte words, whole warps): an odd
    // number of 16-byte units does.
    uint32_t rs = ((g.ck / 256) * (uint32_t)MvT<TYPE>::BB + 32 + 15) & ~15u;
    if (TYPE == T_Q4_K) {
        while (rs % 128 != 32) rs += 16;
    } else if (((rs / 16) & 1u) == 0) {
        rs += 16;
    }
    g.rs = rs;
    const uint32_t avail = MB_SMEM > g.stage0 ? MB_SMEM - g.stage0 : 0;
    g.nstage = std::min(MB_MAXST, avail / (16 * rs));
    return g;
}

// weights w0..w3 in the bytes of one word -> f16x2 pairs (w0, w2) and (w1, w3)
// of the nibbles at bit `sh` (0 low, 4 high), as 1024 + n (exact)
__device__ __forceinline__ void mb_nib_pairs(uint32_t w, int sh, uint32_t &p02, uint32_t &p13) {
    p02 = ((w >> sh) & 0x000F000Fu) | 0x64006400u;
    p13 = ((w >> (sh + 8)) & 0x000F000Fu) | 0x64006400u;
}
// 6-bit values v0..v3 in the bytes of one word -> f16x2 (v0-32, v2-32), (v1-32, v3-32)
__device__ __forceinline__ void mb_q6_pairs(uint32_t v, uint32_t &p02, uint32_t &p13) {
    const __half2 k1056 = __floats2half2_rn(1056.f, 1056.f);
    const uint32_t a = (v & 0x00FF00FFu) | 0x64006400u, b = ((v >> 8) & 0x00FF00FFu) | 0x64006400u;
    const __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), k1056);
    const __half2 hb = __hsub2(*reinterpret_cast<const __half2 *>(&b), k1056);
    p02 = *reinterpret_cast<const uint32_t *>(&ha);
    p13 = *reinterpret_cast<const uint32_t *>(&hb);
}

// This lane's B fragments of one 256-column super-block (8 sequences), held
// in registers for every tile of the launch: a warp always works on the
// same super-block of the chunk, so x is read from shared memory once.
template <int TYPE> struct MbX;
template <> struct MbX<T_Q4_K> { uint4 xv[8]; const float2 *xg; };   // per sub-block: x words; its group sums in shared memory
template <> struct MbX<T_Q6_K> { uint2 xv[16]; };                 // per (half, 16-column part, quarter)

template <int TYPE>
__device__ __forceinline__ void mb_xfrag(uint32_t e, uint32_t xh, uint32_t xstride, const float *xs, int lane, MbX<TYPE> &f) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t xrow = xh + (uint32_t)g * xstride;   // this lane's B column is sequence g
    if constexpr (TYPE == T_Q4_K) {
#pragma unroll
        for (int s = 0; s < 8; ++s) f.xv[s] = lds_u128(xrow + (e + 32 * s + 8 * t) * 2);
        f.xg = reinterpret_cast<const float2 *>(xs + (e >> 5) * MB_B + 2 * t);   // [group][sequence]: + s * MB_B / 2
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int l = 0; l < 2; ++l)
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    f.xv[(h * 2 + l) * 4 + q] = lds_u64(xrow + (e + 128 * h + 32 * q + 4 * t + 16 * l) * 2);
    }
}

// One warp, 16 rows (stage rows g, g+8 at rowA/rowB, pads pa/pb), one
// 256-column super-block at chunk column e, x fragments in registers.
// acc: rows g, g+8 x sequences 2t, 2t+1.
template <int TYPE>
__device__ __forceinline__ void mb_unit(uint32_t rowA, uint32_t rowB, uint32_t pa, uint32_t pb, uint32_t e,
                                        const MbX<TYPE> &xf, int lane, float acc[4]) {
    const int t = lane & 3;
    if constexpr (TYPE == T_Q4_K) {
        const uint32_t sa = rowA + (e >> 8) * 144, sb = rowB + (e >> 8) * 144;
        const uint4 hA = lds_u128(sa), hB = lds_u128(sb);
        float dsc[2][8], dmm[2][8];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const uint4 h = rr ? hB : hA;
            const float d = f16f(h.x & 0xFFFFu), dmin = f16f(h.x >> 16);
            // 6-bit scales/mins of sub-blocks 0-3 and 4-7 (src/vbs_dequant.c:225-233)
            const uint32_t sc0 = h.y & 0x3F3F3F3Fu, mn0 = h.z & 0x3F3F3F3Fu;
            const uint32_t sc1 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t mn1 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                dsc[rr][s] = d * byte_f(s < 4 ? sc0 : sc1, s & 3);
                dmm[rr][s] = dmin * byte_f(s < 4 ? mn0 : mn1, s & 3) + 1024.0f * dsc[rr][s];   // min term + the 1024 bias
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {   // sub-block pair (2j low nibbles, 2j+1 high)
            const uint2 wA = lds_u64(sa + 16 + 32 * j + 8 * t), wB = lds_u64(sb + 16 + 32 * j + 8 * t);
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {
                const int s = 2 * j + hi;
                const uint4 xv = xf.xv[s];
                float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {   // weights 8t+4hf .. +3
                    uint32_t a[4];
                    mb_nib_pairs(hf ? wA.y : wA.x, 4 * hi, a[0], a[2]);
                    mb_nib_pairs(hf ? wB.y : wB.x, 4 * hi, a[1], a[3]);
                    mma_f16_acc(c, a, hf ? xv.z : xv.x, hf ? xv.w : xv.y);
                }
                const float2 xg = xf.xg[s * (MB_B / 2)];   // the sub-block's x sums, sequences 2t, 2t+1
                const float x0 = xg.x, x1 = xg.y;
                acc[0] += dsc[0][s] * c[0] - dmm[0][s] * x0;
                acc[1] += dsc[0][s] * c[1] - dmm[0][s] * x1;
                acc[2] += dsc[1][s] * c[2] - dmm[1][s] * x0;
                acc[3] += dsc[1][s] * c[3] - dmm[1][s] * x1;
            }
        }
    } else {   // Q6_K: {ql[128], qh[64], i8 sc[16], f16 d}; rows 2-byte aligned (pads)
        const uint32_t sa = rowA + pa + (e >> 8) * 210, sb = rowB + pb + (e >> 8) * 210;
        const float dA = f16f(lds_u16(sa + 208)), dB = f16f(lds_u16(sb + 208));
#pragma unroll
        for (int h = 0; h < 2; ++h) {   // 128-element halves
#pragma unroll
            for (int l0 = 0; l0 < 32; l0 += 16) {
                const uint32_t o = 4 * t + l0;
                const uint32_t qlA0 = lds_u32_any(sa + 64 * h + o), qlA1 = lds_u32_any(sa + 64 * h + 32 + o);
                const uint32_t qlB0 = lds_u32_any(sb + 64 * h + o), qlB1 = lds_u32_any(sb + 64 * h + 32 + o);
                const uint32_t qhA = lds_u32_any(sa + 128 + 32 * h + o), qhB = lds_u32_any(sb + 128 + 32 * h + o);
#pragma unroll
                for (int q = 0; q < 4; ++q) {   // quarters: elements q*32 + l
                    const uint32_t lA = (q & 1) ? qlA1 : qlA0, lB = (q & 1) ? qlB1 : qlB0, sh = (q >> 1) * 4;
                    const uint32_t vA = ((lA >> sh) & 0x0F0F0F0Fu) | (((qhA >> (2 * q)) & 0x03030303u) << 4);
                    const uint32_t vB = ((lB >> sh) & 0x0F0F0F0Fu) | (((qhB >> (2 * q)) & 0x03030303u) << 4);
                    uint32_t a[4];
                    mb_q6_pairs(vA, a[0], a[2]);
                    mb_q6_pairs(vB, a[1], a[3]);
                    const uint2 xv = xf.xv[(h * 2 + (l0 >> 4)) * 4 + q];
                    float c[4] = {0.f, 0.f, 0.f, 0.f};
                    mma_f16_acc(c, a, xv.x, xv.y);
                    const uint32_t is = 8 * h + 2 * q + (l0 >> 4);
                    const float sA = dA * (float)lds_s8(sa + 192 + is), sB = dB * (float)lds_s8(sb + 192 + is);
                    acc[0] += sA * c[0];
                    acc[1] += sA * c[1];
                    acc[2] += sB * c[2];
                    acc[3] += sB * c[3];
                }
            }
        }
    }
}

template <int TYPE>
__global__ void __launch_bounds__(MB_THREADS, 1) mvb_kernel(const MvbParams p, const MbGeom geo) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr uint32_t E = 256, BB = MvT<TYPE>::BB;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t sbase = smem_u32(smem), RS = geo.rs, nstage = geo.nstage;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 256);
    float *red = reinterpret_cast<float *>(smem + MB_RED);
    const uint32_t xh = sbase + MB_X;
    float *xs = reinterpret_cast<float *>(smem + geo.xs_off);
    auto full_bar = [&](uint32_t s) { return sbase + 8u * s; };
    auto empty_bar = [&](uint32_t s) { return sbase + 8u * (MB_MAXST + s); };
    auto stage_addr = [&](uint32_t s) { return sbase + geo.stage0 + s * 16u * RS; };

    // rows of this CTA (whole 16-row tiles), column chunk blockIdx.y
    const uint32_t ntile_all = (p.rows + 15) / 16;
    const uint32_t t0 = (uint32_t)(((uint64_t)blockIdx.x * ntile_all) / gridDim.x);
    const uint32_t t1 = (uint32_t)(((uint64_t)(blockIdx.x + 1) * ntile_all) / gridDim.x);
    const uint32_t c0 = blockIdx.y * geo.ck, c1 = min(p.cols, c0 + geo.ck), ncol = c1 - c0;
    const uint64_t boff = (uint64_t)(c0 / E) * BB, blen = (uint64_t)(ncol / E) * BB;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < nstage; ++i) {
            mbar_init(full_bar(i), 1);
            mbar_init(empty_bar(i), MB_NCW);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == MB_NCW) {
        // ------------------------------ producer ------------------------------
        // one bulk copy per row (16-byte aligned middle), head/tail bytes by
        // the lanes; rows keep their global address modulo 16 in the slot
        uint32_t slot = 0, round = 0, issued = 0;
        const uint32_t ri = (uint32_t)lane & 15u;
        for (uint32_t tile = t0; tile < t1; ++tile) {
            if (issued >= nstage && !mbar_wait_bounded(empty_bar(slot), (round - 1) & 1, kWaitNs)) {
                if (lane == 0) { *abort_flag = 1; dev_flag_error(p.err, DERR_TIMEOUT_EMPTY); }
                break;
            }
            if (*abort_flag) break;
            const uint32_t row = tile * 16 + ri;
            uint32_t tx = 0, dst_al = 0;
            uintptr_t lo = 0;
            if (lane < 16 && row < p.rows) {
                const uint8_t *rp = p.w + (uint64_t)row * p.rb + boff;
                const uintptr_t a = reinterpret_cast<uintptr_t>(rp);
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
            if (++slot == nstage) { slot = 0; ++round; }
        }
        if (*abort_flag) {
            const uint32_t first = issued > nstage ? issued - nstage : 0;
            for (uint32_t s = first; s < issued; ++s) mbar_wait_bounded(full_bar(s % nstage), (s / nstage) & 1, kWaitNs);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    // x chunk as fp16 [8][ck] (sequences >= batch and columns >= ncol zero),
    // then the per-group sums of those fp16 values
    // stored with each group of 4 in the order (0, 2, 1, 3): the MMA k-slot order
    for (uint32_t i = threadIdx.x; i < MB_B * geo.ck / 4; i += MB_NCW * 32) {
        const uint32_t b = i / (geo.ck / 4), c = 4 * (i % (geo.ck / 4));
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b < p.batch && c < ncol) v = *reinterpret_cast<const float4 *>(p.x + (uint64_t)b * p.x_stride + c0 + c);
        const __half2 h02 = __floats2half2_rn(v.x, v.z), h13 = __floats2half2_rn(v.y, v.w);
        asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(xh + b * geo.xstride + c * 2),
                     "r"(*reinterpret_cast<const uint32_t *>(&h02)), "r"(*reinterpret_cast<const uint32_t *>(&h13)) : "memory");
    }
    named_bar_sync(1, MB_NCW * 32);
    if constexpr (TYPE == T_Q4_K) {
        const uint32_t ng = geo.ck / 32;
        for (uint32_t i = threadIdx.x; i < MB_B * ng; i += MB_NCW * 32) {
            const uint32_t gg = i / MB_B, b = i % MB_B;   // stored [group][sequence]
            float s = 0.f;
            for (int k = 0; k < 32; k += 2) {
                const uint32_t w = lds_u32(xh + b * geo.xstride + (gg * 32 + k) * 2);
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
                s += f.x + f.y;
            }
            xs[i] = s;
        }
        named_bar_sync(1, MB_NCW * 32);
    }

    const int g = lane >> 2, t = lane & 3;
    // chunks are at most MB_CK = MB_NCW * 256 columns: one super-block per warp
    const uint32_t e = (uint32_t)warp * 256u;
    const bool has_e = e < ncol;
    MbX<TYPE> xf;
    if (has_e) mb_xfrag<TYPE>(e, xh, geo.xstride, xs, lane, xf);
    uint32_t slot = 0, round = 0;
    for (uint32_t tile = t0; tile < t1; ++tile) {
        bool ok = !*abort_flag;
        if (ok && !mbar_wait_bounded(full_bar(slot), round & 1, kWaitNs)) {
            ok = false;
            if (lane == 0) { *abort_flag = 1; dev_flag_error(p.err, DERR_TIMEOUT_FULL); }
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
            const uint32_t rowA = stage_addr(slot) + (uint32_t)g * RS, rowB = rowA + 8 * RS;
            uint32_t pa = 0, pb = 0;
            if constexpr (TYPE == T_Q6_K) {   // rows keep their global address modulo 16
                const uint32_t ra = min(tile * 16 + g, p.rows - 1), rb = min(tile * 16 + g + 8, p.rows - 1);
                pa = (uint32_t)(reinterpret_cast<uintptr_t>(p.w + (uint64_t)ra * p.rb + boff) & 15);
                pb = (uint32_t)(reinterpret_cast<uintptr_t>(p.w + (uint64_t)rb * p.rb + boff) & 15);
            }
            if (has_e) mb_unit<TYPE>(rowA, rowB, pa, pb, e, xf, lane, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(slot));
        if (++slot == nstage) { slot = 0; ++round; }
        // rows g, g+8 x sequences 2t, 2t+1 -> the warps' sum, in warp order,
        // for MB_NU tiles at a time behind one pair of consumer barriers
        const uint32_t k = (tile - t0) % MB_NU;
        float *rw = red + (k * MB_NCW + warp) * 16 * MB_B;
        rw[g * MB_B + 2 * t] = acc[0];
        rw[g * MB_B + 2 * t + 1] = acc[1];
        rw[(g + 8) * MB_B + 2 * t] = acc[2];
        rw[(g + 8) * MB_B + 2 * t + 1] = acc[3];
        if (k == MB_NU - 1 || tile + 1 == t1) {
            named_bar_sync(1, MB_NCW * 32);
            static_assert(MB_NU * 16 * MB_B <= MB_NCW * 32, "one thread per buffered (tile, row, sequence)");
            const uint32_t j = threadIdx.x / (16 * MB_B), rr = (threadIdx.x / MB_B) % 16, b = threadIdx.x % MB_B;
            const uint32_t tj = tile - k + j, row = tj * 16 + rr;
            if (j <= k && !*abort_flag) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < MB_NCW; ++w) v += red[((j * MB_NCW + w) * 16 + rr) * MB_B + b];
                if (b < p.batch && row < p.rows) {
                    float *dst = p.y_plane ? p.y_plane + ((uint64_t)blockIdx.y * p.batch + b) * p.rows + row
                                           : p.y + (uint64_t)b * p.y_stride + row;
                    *dst = (p.accumulate && !p.y_plane) ? *dst + v : v;
                }
            }
            named_bar_sync(1, MB_NCW * 32);
        }
    }
}

// y[b][r] (+)= sum over chunks c of plane[c][b][r], in chunk order
__global__ void mvb_reduce_kernel(const float *planes, uint32_t nch, uint32_t batch, uint32_t rows, float *y,
                                  uint64_t y_stride, int accumulate) {
    const uint64_t n = (uint64_t)batch * rows;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        float v = 0.f;
        for (uint32_t c = 0; c < nch; ++c) v += planes[(uint64_t)c * n + i];
        const uint32_t b = (uint32_t)(i / rows), r = (uint32_t)(i % rows);
        float *dst = y + (uint64_t)b * y_stride + r;
        *dst = accumulate ? *dst + v : v;
    }
}

bool mvb_supported(int type, uint32_t rows, uint32_t cols, uint32_t batch, const void *w, const void *x) {
    if (type != T_Q4_K && type != T_Q6_K) return false;
    if (!rows || batch < 1 || batch > MB_B || cols % 256) return false;
    if (reinterpret_cast<uintptr_t>(x) & 15) return false;   // float4 loads of x
    // Q4_K rows (144-byte blocks) must start 16-byte aligned for the 16-byte header loads
    if (type == T_Q4_K && (reinterpret_cast<uintptr_t>(w) & 15)) return false;
    const MbGeom g = type == T_Q4_K ? mb_geom<T_Q4_K>(cols) : mb_geom<T_Q6_K>(cols);
    return g.nstage >= 2;
}

size_t mvb_workspace_bytes(int type, uint32_t rows, uint32_t cols, uint32_t batch) {
    const MbGeom g = type == T_Q4_K ? mb_geom<T_Q4_K>(cols) : mb_geom<T_Q6_K>(cols);
    return g.nch > 1 ? (size_t)g.nch * batch * rows * 4 : 0;
}

template <int TYPE>
static cudaError_t mvb_go(MvbParams p, float *work, int n_sm, cudaStream_t st) {
    const MbGeom geo = mb_geom<TYPE>(p.cols);
    const uint32_t smem = geo.stage0 + geo.nstage * 16 * geo.rs;
    const uint32_t ntile = (p.rows + 15) / 16;
    const uint32_t gx = std::max(1u, std::min(ntile, ((uint32_t)n_sm + geo.nch - 1) / geo.nch));
    float *y = p.y;
    p.y_plane = geo.nch > 1 ? work : nullptr;
    note_launches(geo.nch > 1 ? 2 : 1);
    mvb_kernel<TYPE><<<dim3(gx, geo.nch), MB_THREADS, smem, st>>>(p, geo);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || geo.nch == 1) return e;
    const uint64_t n = (uint64_t)p.batch * p.rows;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 4);
    mvb_reduce_kernel<<<blocks, 256, 0, st>>>(work, geo.nch, p.batch, p.rows, y, p.y_stride, p.accumulate);
    return cudaGetLastError();
}

cudaError_t mvb_configure() {
    cudaError_t e = cudaFuncSetAttribute(mvb_kernel<T_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, MB_SMEM);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(mvb_kernel<T_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, MB_SMEM);
    return e;
}

cudaError_t mvb_launch(int type, const MvbParams &p, float *work, int n_sm, cudaStream_t st) {
    if (type == T_Q4_K) return mvb_go<T_Q4_K>(p, work, n_sm, st);
    if (type == T_Q6_K) return mvb_go<T_Q6_K>(p, work, n_sm, st);
    return cudaErrorInvalidValue;
}

}  // namespace vbs
