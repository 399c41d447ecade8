// gemm.cu -- quantized-weight GEMM on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory), for prompt prefill and
// batched decode above the batched matvec's 8 sequences.
//
//   Y[t][r] (+)= sum_c dequant(W)[r][c] * X[t][c]     t < T tokens, r < N rows
//
// The reference has no batched path at all: the engine feeds a prompt one
// token at a time through forward_token (src/main.c:901-904), every token
// streaming every weight. Here one CTA owns a tile of 128 weight rows x 512
// tokens (two activation tiles of 256), so each weight is decoded once for
// 512 tokens:
//  * producer warps (512 threads) walk K in steps of 64: threads 4r..4r+3
//    dequantize row r's 64 weights, 16 each (the GGUF block decode of
//    src/vbs_dequant.c, rounded to fp16; the raw bytes are fetched two to
//    four stages ahead into registers) into the UMMA canonical K-major
//    layout in shared memory: 8-row x 16-byte core matrices 128 bytes apart
//    along M/N (SBO), k-chunks of 8 elements one operand-height x 16 bytes
//    apart (LBO);
//  * a loader warp moves each stage's activations with one bulk copy: they
//    were converted to fp16 once per call, already in that layout;
//  * one thread issues tcgen05.mma.kind::f16 (M = 128, N = 256, K = 16, four
//    per stage and activation tile) into two 128 x 256 fp32 accumulators in
//    tensor memory (all 512 columns) and releases each stage with
//    tcgen05.commit on its mbarrier;
//  * after the last stage the producer warps read the accumulator back with
//    tcgen05.ld (warp w: lanes 32 (w % 4).. = rows, columns 128 (w / 4).. =
//    tokens) and store Y (split-K: a plane per split, summed in order).
// Every wait is bounded; a timeout records DERR_TIMEOUT_* and the CTA
// skips the rest of its tile (tensor memory is always released).
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vbs {

constexpr int QG_M = 128;            // weight rows per tile (UMMA M)
constexpr int QG_N = 256;            // tokens per MMA (UMMA N) and per activation tile
constexpr int QG_NT = 2;             // activation tiles per CTA: each weight decoded once for 512 tokens
constexpr int QG_TT = QG_N * QG_NT;  // tokens per CTA
constexpr int QG_KT = 64;            // k per stage
constexpr int QG_NS = 2;             // stages (80 KB each)
constexpr int QG_PT = 512;           // producer / epilogue threads: 4 per weight row, 2 per token
constexpr uint32_t QG_PARTS = QG_PT / QG_M;   // threads per weight row, 16 of its 64 stage weights each
constexpr int QG_THREADS = QG_PT + 64;   // + the MMA warp + the activation loader warp
constexpr uint32_t QG_A_BYTES = QG_M * QG_KT * 2, QG_B_BYTES = QG_N * QG_KT * 2;
constexpr uint32_t QG_STAGE = QG_A_BYTES + QG_NT * QG_B_BYTES;
constexpr uint32_t QG_HDR = 1024;    // barriers + tensor-memory address
constexpr uint32_t QG_SMEM = QG_HDR + QG_NS * QG_STAGE;

// UMMA shared-memory descriptor, K-major, no swizzle (the canonical layout
// ((8, m), (8 elements, 2)) : ((16 B, SBO), (2 B, LBO)); addresses and
// offsets in 16-byte units; version 1 for sm_100).
__device__ __forceinline__ uint64_t qg_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: D fp32, A and B fp16, both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t QG_IDESC = (1u << 4) | ((uint32_t)(QG_N >> 3) << 17) | ((uint32_t)(QG_M >> 4) << 24);

__device__ __forceinline__ void qg_mma(uint32_t tmem, uint64_t da, uint64_t db, bool acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(tmem), "l"(da), "l"(db), "r"(QG_IDESC), "r"(acc ? 1u : 0u) : "memory");
}
__device__ __forceinline__ void qg_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void qg_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void qg_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void qg_fence_proxy() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 8 consecutive weights e0..e0+7 of one row as fp16x2 words, decoded as
// src/vbs_dequant.c does (dq_elem) and rounded to fp16.
template <int TYPE>
__device__ __forceinline__ uint4 qg_dq8(const uint8_t *row, uint32_t e0) {
    constexpr int E = TYPE == T_Q8_0 ? 32 : 256, BB = TYPE == T_Q4_K ? 144 : (TYPE == T_Q6_K ? 210 : 34);
    const uint8_t *blk = row + (uint64_t)(e0 / E) * BB;
    const uint32_t o = e0 % E;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = dq_elem(TYPE, blk, (int)(o + k));
    uint4 r;
    r.x = __half_as_ushort(__float2half_rn(v[0])) | ((uint32_t)__half_as_ushort(__float2half_rn(v[1])) << 16);
    r.y = __half_as_ushort(__float2half_rn(v[2])) | ((uint32_t)__half_as_ushort(__float2half_rn(v[3])) << 16);
    r.z = __half_as_ushort(__float2half_rn(v[4])) | ((uint32_t)__half_as_ushort(__float2half_rn(v[5])) << 16);
    r.w = __half_as_ushort(__float2half_rn(v[6])) | ((uint32_t)__half_as_ushort(__float2half_rn(v[7])) << 16);
    return r;
}

// a, b rounded to fp16 (round to nearest even), a in the low half: one
// paired conversion.
__device__ __forceinline__ uint32_t qg_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// Byte k of w as an exact float: 2^23 + byte by a byte permute, minus 2^23
// (no integer-to-float conversion).
__device__ __forceinline__ float qg_byte_f(uint32_t w, uint32_t k) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | k)) - 8388608.0f;
}

__device__ __forceinline__ uint32_t lo_word(const uint32_t (&w)[4], int i) { return w[i]; }

// The producers fetch a stage's raw weight bytes QgDepth stages before they
// decode them (QgRaw in registers), so the loads' latency overlaps the
// decode and the shared-memory stores of the stages in between.
// A thread's share of a stage is part pi (0..3) of its row's 64 weights:
// half h = pi / 2 (Q4_K: the low or high nibbles; Q6_K: the first or second
// 32 values), and within it the 16 weights of k-chunks 2 (pi % 2), +1.
template <int TYPE> struct QgRaw { uint32_t k0; };
template <> struct QgRaw<T_Q4_K> { uint4 hdr, q; uint32_t k0; };
template <> struct QgRaw<T_Q6_K> { uint32_t ql[4], qh[4], sc, d, k0; };
template <int TYPE> struct QgDepth { static constexpr int D = TYPE == T_Q4_K ? 4 : 2; };   // within 120 registers

// 16 bytes at a 2-byte aligned address, as 4 words: 5 aligned words and a
// funnel shift (the bytes past the range lie inside the same Q6_K block).
__device__ __forceinline__ void qg_ld16_a2(const uint8_t *ptr, uint32_t out[4]) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(reinterpret_cast<uintptr_t>(ptr) & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(ptr) & 3u) * 8u;
    uint32_t v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = __ldg(w + i);
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = __funnelshift_r(v[i], v[i + 1], sh);
}

template <int TYPE>
__device__ __forceinline__ void qg_fetch(const uint8_t *row, uint32_t k0, uint32_t pi, QgRaw<TYPE> &r) {
    r.k0 = k0;
    const uint32_t half = pi >> 1, part = pi & 1u;
    if constexpr (TYPE == T_Q4_K) {
        const uint8_t *b = row + (uint64_t)(k0 >> 8) * 144;
        const uint32_t j0 = (k0 & 255u) >> 5;
        r.hdr = __ldg(reinterpret_cast<const uint4 *>(b));
        r.q = __ldg(reinterpret_cast<const uint4 *>(b + 16 + (j0 >> 1) * 32 + 16 * part));
    } else if constexpr (TYPE == T_Q6_K) {
        const uint8_t *b = row + (uint64_t)(k0 >> 8) * 210;
        const uint32_t c = (k0 & 255u) >> 6, h = c >> 1;
        qg_ld16_a2(b + 64 * h + 32 * half + 16 * part, r.ql);   // quarter q = 2 (c % 2) + half: ql bytes 32 (q % 2) ..
        qg_ld16_a2(b + 128 + 32 * h + 16 * part, r.qh);
        r.sc = __ldg(reinterpret_cast<const unsigned short *>(b + 192 + 4 * c + 2 * half));
        r.d = __ldg(reinterpret_cast<const unsigned short *>(b + 208));
    }
}

// The 32 weights `half` of the stage from its raw bytes, decoded with the
// reference's operation order (src/vbs_dequant.c: Q4_K (d*sc)*q - dmin*m,
// Q6_K (d*sc)*(q-32), no FMA) and rounded to fp16. Q4_K: the stage is
// sub-blocks j0 and j0 + 1 of a super-block, the low and the high nibbles of
// the same 32 bytes. Q6_K: stage chunk c of a super-block is half h = c / 2,
// quarters 2 (c % 2) and 2 (c % 2) + 1; low bits from ql, high bits from qh,
// one scale byte per 16 weights.
template <int TYPE>
__device__ __forceinline__ void qg_decode(const uint8_t *row, const QgRaw<TYPE> &r, uint32_t pi, uint4 out[2]) {
    const uint32_t half = pi >> 1, part = pi & 1u;
    if constexpr (TYPE == T_Q4_K) {
        const uint32_t j = ((r.k0 & 255u) >> 5) + half;
        const uint8_t *s = reinterpret_cast<const uint8_t *>(&r.hdr) + 4;
        int sc, mn;
        if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
        else { sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
        const float d = f16_exact(r.hdr.x & 0xFFFFu), dmin = f16_exact(r.hdr.x >> 16);
        const float a = __fmul_rn(d, (float)sc), c = __fmul_rn(dmin, (float)mn);
        const uint32_t q[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
        const uint32_t sh = half ? 4u : 0u;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const uint32_t w0 = (q[2 * cc] >> sh) & 0x0F0F0F0Fu, w1 = (q[2 * cc + 1] >> sh) & 0x0F0F0F0Fu;
            float v[8];
#pragma unroll
            // a = d*sc has at most 17 significant bits and q at most 4, so
            // a*q is exact in fp32 and the FMA rounds once, as the
            // reference's fmul then fsub does
            for (int k = 0; k < 4; ++k) {
                v[k] = __fmaf_rn(a, qg_byte_f(w0, k), -c);
                v[4 + k] = __fmaf_rn(a, qg_byte_f(w1, k), -c);
            }
            out[cc] = make_uint4(qg_h2(v[0], v[1]), qg_h2(v[2], v[3]), qg_h2(v[4], v[5]), qg_h2(v[6], v[7]));
        }
    } else if constexpr (TYPE == T_Q6_K) {
        const uint32_t c = (r.k0 & 255u) >> 6, q = 2u * (c & 1u) + half;
        const float d = f16_exact(r.d);
        const float ds = __fmul_rn(d, (float)(int)(int8_t)((r.sc >> (8 * part)) & 255u));   // one scale per 16 weights
#pragma unroll
        for (int c4 = 0; c4 < 2; ++c4) {   // elements 16 part + 8 c4 .. + 7 of this half
            // four 6-bit values per word: low nibbles from ql, two high bits from qh
            const uint32_t lsh = (q >> 1) * 4, hsh = q * 2;
            const uint32_t e0 = ((lo_word(r.ql, 2 * c4) >> lsh) & 0x0F0F0F0Fu) | (((lo_word(r.qh, 2 * c4) >> hsh) & 0x03030303u) << 4);
            const uint32_t e1 = ((lo_word(r.ql, 2 * c4 + 1) >> lsh) & 0x0F0F0F0Fu) |
                                (((lo_word(r.qh, 2 * c4 + 1) >> hsh) & 0x03030303u) << 4);
            float v[8];
#pragma unroll
            for (int t = 0; t < 4; ++t) {   // q - 32 exactly: (2^23 + q) - (2^23 + 32)
                v[t] = __fmul_rn(ds, __uint_as_float(__byte_perm(e0, 0x4B000000u, 0x7440u | t)) - 8388640.0f);
                v[4 + t] = __fmul_rn(ds, __uint_as_float(__byte_perm(e1, 0x4B000000u, 0x7440u | t)) - 8388640.0f);
            }
            out[c4] = make_uint4(qg_h2(v[0], v[1]), qg_h2(v[2], v[3]), qg_h2(v[4], v[5]), qg_h2(v[6], v[7]));
        }
    } else {
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) out[cc] = qg_dq8<TYPE>(row, r.k0 + 32 * half + 16 * part + 8 * cc);
    }
}

__device__ __forceinline__ bool qg_wait(uint32_t bar, uint32_t parity) { return mbar_wait_bounded(bar, parity, kWaitNs); }

template <int TYPE>
__global__ void __launch_bounds__(QG_THREADS, 1) qgemm_kernel(QgemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t base = smem_u32(smem);
    const uint32_t full0 = base, empty0 = base + 8 * QG_NS, accb = base + 16 * QG_NS, bfull0 = accb + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 512);
    volatile int *bad = reinterpret_cast<volatile int *>(smem + 520);
    const uint32_t st0 = base + QG_HDR;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r0 = blockIdx.x * QG_M, t0 = blockIdx.y * QG_TT;
    // split-K: this CTA's stages [kb, kb + nk) of the row's K / 64
    const uint32_t nk_all = p.cols / QG_KT, per = (nk_all + gridDim.z - 1) / gridDim.z;
    const uint32_t kb = min(nk_all, blockIdx.z * per), nk = min(nk_all, kb + per) - kb;

    if (threadIdx.x == 0) {
        // full: one arrival per producer warp (A); bfull: the B copy's bytes
        for (int s = 0; s < QG_NS; ++s) {
            mbar_init(full0 + 8 * s, QG_PT / 32);
            mbar_init(empty0 + 8 * s, 1);
            mbar_init(bfull0 + 8 * s, 1);
        }
        mbar_init(accb, 1);
        *bad = 0;
        mbar_fence_init();
    }
    if (warp == QG_PT / 32) {   // tensor memory: QG_TT columns of 32-bit accumulators (all 512)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"((uint32_t)QG_TT) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    qg_fence_before();
    __syncthreads();
    qg_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < QG_PT / 32) {
        // ---- producers: part wh of weight row wr ----
        const uint32_t i = threadIdx.x, wr = i / QG_PARTS, wh = i % QG_PARTS;
        const uint32_t row = r0 + wr;
        const uint8_t *wrow = p.w + (uint64_t)min(row, p.rows - 1) * p.rb;
        // canonical offsets: core matrix r/8 at SBO = 128 B, row r%8 at 16 B
        const uint32_t aoff = (wr >> 3) * 128u + (wr & 7u) * 16u;
        auto fetch = [&](uint32_t kt, QgRaw<TYPE> &rw) {
            if (kt < nk && row < p.rows) qg_fetch<TYPE>(wrow, (kb + kt) * QG_KT, wh, rw);
        };
        // one stage: once the slot is free, this stage's weights are decoded
        // from rw, and rw is refilled with the raw bytes of stage kt + D
        auto stage = [&](uint32_t kt, QgRaw<TYPE> &rw) -> bool {
            const uint32_t s0 = kt % QG_NS;   // warp-uniform decision: the warp arrives as one below
            const bool freed = kt < QG_NS || qg_wait(empty0 + 8 * s0, ((kt / QG_NS) - 1) & 1u);
            if (!__all_sync(0xffffffffu, freed && !*bad)) return false;
            const uint32_t sa = st0 + s0 * QG_STAGE;
            uint4 wv[2];
            if (row < p.rows) {
                qg_decode<TYPE>(wrow, rw, wh, wv);
            } else {
                wv[0] = wv[1] = make_uint4(0, 0, 0, 0);
            }
            // A: k-chunks 2 wh, 2 wh + 1 of row wr (part wh = half * 2 + part:
            // chunk 4 half + 2 part), LBO = 128 rows x 16 B
#pragma unroll
            for (int c = 0; c < 2; ++c)
                asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(sa + (2 * wh + c) * (QG_M * 16u) + aoff),
                             "r"(wv[c].x), "r"(wv[c].y), "r"(wv[c].z), "r"(wv[c].w) : "memory");
            fetch(kt + QgDepth<TYPE>::D, rw);
            qg_fence_proxy();     // the tensor core (async proxy) reads what the generic stores wrote
            __syncwarp();         // every lane's stores and fence before the warp's one arrival
            if (lane == 0) mbar_arrive(full0 + 8 * (kt % QG_NS));
            return true;
        };
        constexpr int D = QgDepth<TYPE>::D;
        QgRaw<TYPE> raw[D];
#pragma unroll
        for (int d = 0; d < D; ++d) fetch(d, raw[d]);
        for (uint32_t kt = 0; kt < nk && !*bad; kt += D) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                if (kt + d < nk && !stage(kt + d, raw[d])) { *bad = 1; break; }
            }
        }
        // ---------------- epilogue: accumulator rows -> Y ------------------
        const bool ok = !*bad && qg_wait(accb, 0);
        qg_fence_after();
        constexpr uint32_t CW = QG_TT / (QG_PT / 128);   // columns per warp of a lane quadrant
        const uint32_t rr = r0 + 32u * (warp & 3) + lane;
#pragma unroll 1
        for (uint32_t c0 = (warp >> 2) * CW; c0 < (warp >> 2) * CW + CW; c0 += 16) {
            uint32_t v[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                : "r"(tmem + ((32u * (warp & 3)) << 16) + c0));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (!ok || rr >= p.rows) continue;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t t = t0 + c0 + j;
                if (t >= p.tokens) break;
                const float val = nk ? __uint_as_float(v[j]) : 0.0f;
                if (gridDim.z > 1) {   // split-K: this split's plane, summed in split order by qg_reduce_kernel
                    p.planes[((uint64_t)blockIdx.z * p.tokens + t) * p.rows + rr] = val;
                } else {
                    float *dst = p.y + (uint64_t)t * p.y_stride + rr;
                    *dst = p.accumulate ? *dst + val : val;
                }
            }
        }
        if (!ok && lane == 0) dev_flag_error(p.err, DERR_TIMEOUT_FULL);
    } else if (warp == QG_PT / 32 + 1) {
        // -------- activation loader: the B operand of every stage, one bulk
        // copy (no multicast) per stage, as soon as its slot is free --------
        if (lane == 0) {
            // this token tile's activations, already in the B layout: a stage
            // is QG_B_BYTES contiguous bytes
            const uint64_t tile_bytes = (uint64_t)(p.cols / 8) * QG_N * 16u;
            const uint8_t *xtile = reinterpret_cast<const uint8_t *>(p.x16) + (uint64_t)blockIdx.y * QG_NT * tile_bytes;
            uint32_t issued = 0;
            for (uint32_t kt = 0; kt < nk; ++kt) {
                const uint32_t s = kt % QG_NS;
                if ((kt >= QG_NS && !qg_wait(empty0 + 8 * s, ((kt / QG_NS) - 1) & 1u)) || *bad) { *bad = 1; break; }
                mbar_arrive_expect_tx(bfull0 + 8 * s, QG_NT * QG_B_BYTES);
#pragma unroll
                for (int n = 0; n < QG_NT; ++n)   // activation tile n of this CTA's tokens
                    bulk_g2s(st0 + s * QG_STAGE + QG_A_BYTES + n * QG_B_BYTES,
                             xtile + n * tile_bytes + (uint64_t)(kb + kt) * QG_B_BYTES, QG_B_BYTES, bfull0 + 8 * s);
                issued = kt + 1;
            }
            if (*bad) {
                // copies may still be landing in slots nobody will read: wait
                // (bounded) for the newest one of every slot (older ones were
                // consumed before their slot was reused) before the CTA exits
                for (uint32_t kt = issued > (uint32_t)QG_NS ? issued - QG_NS : 0; kt < issued; ++kt)
                    qg_wait(bfull0 + 8 * (kt % QG_NS), (kt / QG_NS) & 1u);
            }
        }
    } else if (lane == 0) {
        // ---------------- MMA issue (one thread) ----------------------------
        for (uint32_t kt = 0; kt < nk; ++kt) {
            const uint32_t s = kt % QG_NS;
            if (!qg_wait(full0 + 8 * s, (kt / QG_NS) & 1u) || !qg_wait(bfull0 + 8 * s, (kt / QG_NS) & 1u)) { *bad = 1; break; }
            qg_fence_after();
            const uint32_t sa = st0 + s * QG_STAGE, sb = sa + QG_A_BYTES;
#pragma unroll
            for (int ks = 0; ks < QG_KT / 16; ++ks) {   // K = 16 = two k-chunks per MMA
                const uint64_t da = qg_desc(sa + ks * (2 * QG_M * 16u), QG_M * 16u, 128u);
#pragma unroll
                for (int n = 0; n < QG_NT; ++n) {   // accumulator n: tensor-memory columns 256 n ..
                    const uint64_t db = qg_desc(sb + n * QG_B_BYTES + ks * (2 * QG_N * 16u), QG_N * 16u, 128u);
                    qg_mma(tmem + n * QG_N, da, db, kt > 0 || ks > 0);
                }
            }
            qg_commit(empty0 + 8 * s);   // the stage is free once these MMAs have read it
        }
        qg_commit(accb);                 // the accumulator is complete (no stage: nothing to wait for)
    }
    qg_fence_before();
    __syncthreads();
    if (warp == QG_PT / 32) {
        // every MMA this CTA issued has completed (the final commit) before
        // its tensor memory goes back; bounded like every other wait
        if (lane == 0) qg_wait(accb, 0);
        __syncwarp();
        qg_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)QG_TT) : "memory");
    }
}

// Split-K: Y[t][r] (+)= sum over splits z in order of planes[z][t][r].
__global__ void qg_reduce_kernel(const float *__restrict__ planes, uint32_t nz, uint32_t tokens, uint32_t rows,
                                 float *__restrict__ y, uint64_t ys, uint32_t accumulate) {
    const uint64_t n = (uint64_t)tokens * rows;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        float v = planes[i];
        for (uint32_t z = 1; z < nz; ++z) v += planes[(uint64_t)z * n + i];
        const uint32_t t = (uint32_t)(i / rows), r = (uint32_t)(i % rows);
        float *dst = y + (uint64_t)t * ys + r;
        *dst = accumulate ? *dst + v : v;
    }
}

// fp32 rows [rows x cols] -> fp16 [rows_pad x cols], rows past `rows` zero
// The activations as fp16 in the B operand's shared-memory layout, so one
// bulk copy moves a stage: [token tile][k-chunk of 8][QG_N tokens][8],
// tokens past `rows` zero. Each thread converts 8 consecutive values.
__global__ void qg_to_half_kernel(const float *__restrict__ x, uint64_t xs, __half *__restrict__ out, uint32_t rows,
                                  uint32_t rows_pad, uint32_t cols) {
    const uint32_t nch = cols / 8;
    const uint64_t n = (uint64_t)rows_pad * nch;   // 16-byte pieces
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t tt = (uint32_t)(i % QG_N), g = (uint32_t)((i / QG_N) % nch), y = (uint32_t)(i / ((uint64_t)QG_N * nch));
        const uint32_t r = y * QG_N + tt;
        uint4 h = make_uint4(0, 0, 0, 0);
        if (r < rows) {   // scalar loads: x may be only 4-byte aligned
            const float *src = x + (uint64_t)r * xs + 8 * g;
            h = make_uint4(qg_h2(src[0], src[1]), qg_h2(src[2], src[3]), qg_h2(src[4], src[5]), qg_h2(src[6], src[7]));
        }
        reinterpret_cast<uint4 *>(out)[i] = h;
    }
}

bool qgemm_supported(int type, uint32_t rows, uint32_t cols, uint32_t tokens) {
    if (type != T_Q4_K && type != T_Q6_K && type != T_Q8_0) return false;
    return rows && tokens && cols % QG_KT == 0 && cols % (uint32_t)block_elems(type) == 0;
}

// K splits for a grid of `tiles` output tiles: enough CTAs to cover the
// SMs, at least 8 stages of 64 per split.
static uint32_t qg_splits(uint32_t rows, uint32_t cols, uint32_t tokens, int n_sm) {
    const uint32_t tiles = ((rows + QG_M - 1) / QG_M) * ((tokens + QG_TT - 1) / QG_TT);
    uint32_t z = std::max(1u, (uint32_t)n_sm / std::max(1u, tiles));
    return std::max(1u, std::min(z, cols / QG_KT / 8u));
}

size_t qgemm_x16_bytes(uint32_t tokens, uint32_t cols);
size_t qgemm_planes_bytes(uint32_t rows, uint32_t cols, uint32_t tokens, int n_sm);
size_t qgemm_workspace_bytes(uint32_t rows, uint32_t cols, uint32_t tokens, int n_sm) {
    return qgemm_x16_bytes(tokens, cols) + qgemm_planes_bytes(rows, cols, tokens, n_sm);
}

cudaError_t qgemm_configure() {
    cudaError_t e = cudaFuncSetAttribute(qgemm_kernel<T_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, QG_SMEM);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(qgemm_kernel<T_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, QG_SMEM);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(qgemm_kernel<T_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, QG_SMEM);
    return e;
}

size_t qgemm_x16_bytes(uint32_t tokens, uint32_t cols) {
    return ((size_t)((tokens + QG_TT - 1) / QG_TT) * QG_TT * cols * sizeof(__half) + 255) & ~(size_t)255;
}
size_t qgemm_planes_bytes(uint32_t rows, uint32_t cols, uint32_t tokens, int n_sm) {
    const uint32_t z = qg_splits(rows, cols, tokens, n_sm);
    return z > 1 ? (size_t)z * tokens * rows * sizeof(float) : 0;
}

cudaError_t qgemm_to_half(const float *x, uint64_t x_stride, __half *x16, uint32_t tokens, uint32_t cols, int n_sm,
                          cudaStream_t st) {
    if (!tokens || cols % QG_KT || !x16) return cudaErrorInvalidValue;
    const uint32_t tpad = (tokens + QG_TT - 1) / QG_TT * QG_TT;
    const uint64_t n = (uint64_t)tpad * cols;
    note_launches(1);
    qg_to_half_kernel<<<(unsigned)std::min<uint64_t>((n / 8 + 255) / 256, (uint64_t)n_sm * 16), 256, 0, st>>>(
        x, x_stride, x16, tokens, tpad, cols);
    return cudaGetLastError();
}

cudaError_t qgemm_launch_x16(int type, QgemmParams p, const __half *x16, void *planes, int n_sm, cudaStream_t st) {
    if (!qgemm_supported(type, p.rows, p.cols, p.tokens) || !x16) return cudaErrorInvalidValue;
    const uint32_t tpad = (p.tokens + QG_TT - 1) / QG_TT * QG_TT;
    const uint32_t z = qg_splits(p.rows, p.cols, p.tokens, n_sm);
    if (z > 1 && !planes) return cudaErrorInvalidValue;
    note_launches(z > 1 ? 2 : 1);
    p.x16 = x16;
    p.planes = static_cast<float *>(planes);
    const dim3 grid((p.rows + QG_M - 1) / QG_M, tpad / QG_TT, z);
    switch (type) {
        case T_Q4_K: qgemm_kernel<T_Q4_K><<<grid, QG_THREADS, QG_SMEM, st>>>(p); break;
        case T_Q6_K: qgemm_kernel<T_Q6_K><<<grid, QG_THREADS, QG_SMEM, st>>>(p); break;
        default: qgemm_kernel<T_Q8_0><<<grid, QG_THREADS, QG_SMEM, st>>>(p); break;
    }
    if (z > 1) {
        const uint64_t m = (uint64_t)p.tokens * p.rows;
        qg_reduce_kernel<<<(unsigned)std::min<uint64_t>((m + 255) / 256, (uint64_t)n_sm * 8), 256, 0, st>>>(
            p.planes, z, p.tokens, p.rows, p.y, p.y_stride, p.accumulate);
    }
    return cudaGetLastError();
}

cudaError_t qgemm_launch(int type, QgemmParams p, const float *x, uint64_t x_stride, void *work, int n_sm,
                         cudaStream_t st) {
    if (!qgemm_supported(type, p.rows, p.cols, p.tokens) || !work) return cudaErrorInvalidValue;
    __half *x16 = static_cast<__half *>(work);
    const cudaError_t e = qgemm_to_half(x, x_stride, x16, p.tokens, p.cols, n_sm, st);
    if (e != cudaSuccess) return e;
    return qgemm_launch_x16(type, p, x16, static_cast<uint8_t *>(work) + qgemm_x16_bytes(p.tokens, p.cols), n_sm, st);
}

}  // namespace vbs
