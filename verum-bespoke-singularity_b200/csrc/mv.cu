// mv.cu -- quantized matrix-vector kernels (the decode step's hot path).
//
// Op contract: y[r] = sum_c dequant(W)[r][c] * x[c], the reference's
// vbs_host_linear_tile (src/vbs_host_math.h:223-267) with W packed row-major
// in GGUF blocks (Q8_0 34 B / 32, Q4_K 144 B / 256, Q6_K 210 B / 256).
//
// Fast kernel (mv_fast_kernel), B200 design:
//  * One CTA per SM, a balanced slice of rows each. A producer warp streams
//    stages of 16 rows (32 for the paired gate/up matrices) x a column chunk
//    from HBM into a ring of shared-memory stages with 1-D bulk TMA copies
//    (cp.async.bulk), one copy per row: whole rows when they fit, so each
//    copy is kilobytes long (short scattered segments were measured to
//    stream several times slower). Rows land in padded slots (an odd number
//    of 16-byte units apart) so the consumers' shared loads are
//    conflict-free; Q6_K/Q8_0 rows are only 2-byte aligned in GGUF, their
//    unaligned head and tail bytes are copied by the producer lanes.
//    Full/empty mbarriers, every wait bounded.
//  * x is quantized once per CTA into shared memory as two int8 levels per
//    32-element block: x ~= d2 * (254*q1 + q2), |error| <= amax/64516/2
//    (1.6e-5 of the block maximum). Weights stay in their packed form; the
//    int8 tensor-core MMA (m16n8k32, u8 x s8 -> s32) forms exact integer
//    block dots with a block-diagonal B operand (see mv_unit), and the block
//    scales are applied to the integer dots in fp32.
//  * Epilogues fuse what follows the matvec in the decode step: residual
//    add (accumulate), SiLU(gate)*up for the paired gate/up matrices, and
//    RoPE + fp16 KV-cache store for the fused Q/K/V projection.
//  * Programmatic dependent launch: weight copies start before
//    griddepcontrol.wait; only the x prologue waits for the previous kernel.
//
// Portable kernel (mv_generic_kernel): one warp per row, exact element
// dequantization (same float operation order as src/vbs_dequant.c), fp32
// FMA accumulation. Serves every type/shape/alignment the fast kernel does
// not, and batches.
#include "common.cuh"
#include "kernels.h"
#include "mv_core.cuh"

#include <algorithm>

namespace vbs {

constexpr int MV_NCW = 8;                       // consumer warps
constexpr int MV_THREADS = (MV_NCW + 1) * 32;   // + one producer warp
constexpr uint32_t MV_MAXST = 16;               // barrier slots
constexpr uint32_t MV_HDR = 2560;               // barriers, misc, reduction scratch
constexpr uint32_t MV_SMEM = 227u * 1024u;      // shared memory per CTA (one CTA per SM)

// A stage holds 16 rows (dual: 16 rows of each matrix) x a chunk of CK
// columns, each row one contiguous bulk copy into a padded slot. CK is the
// whole row when 16 rows of it fit, else the largest multiple of 256 columns
// (>= 1024) that keeps NSTAGE >= 3: HBM serves long contiguous row runs
// several times faster than the short scattered segments a 16 x 256 column
// unit would read.
struct MvGeom {
    uint32_t ck;       // columns per chunk (multiple of 256, or all columns)
    uint32_t rs;       // row slot stride in bytes
    uint32_t nstage;   // stages in the ring
    uint32_t stage0;   // byte offset of the first stage
};

__device__ __forceinline__ const uint8_t *seg_row_ptr(const MvParams &p, uint32_t row) {
    if (row < p.seg_end[0]) return p.w[0] + (uint64_t)row * p.rb;
    if (row < p.seg_end[1]) return p.w[1] + (uint64_t)(row - p.seg_end[0]) * p.rb;
    return p.w[2] + (uint64_t)(row - p.seg_end[1]) * p.rb;
}

// ---------------------------------------------------------------------------
// x prologue: optional residual add and RMSNorm, then two-level int8
// quantization: x ~= d2 * (254*q1 + q2) per 32-element block. Four threads
// share a block (8 elements each).
// Layouts per block J (64 bytes):
//   slot layout (Q4_K, Q8_0): 8 slots of 8 bytes; slot s<4 = {q1 word s,
//     q1 word 4+s}, slot 4+s the same for q2 (word w = elements 4w..4w+3);
//   plain layout (Q6_K): q1 words 0..7 then q2 words 0..7.
//   xf[J] = {d2, d2 * sum(254 q1 + q2), sum over k<16, sum over k>=16}.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *a) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}

// Tensor parallelism, reader side: wait (bounded) until every rank published
// the exchange this rank's counter names, then x_add is the rank-ordered sum
// of that exchange's slots. The slots were written over NVLink into this
// GPU's memory: read through L2 (ld.cg), never from a stale L1 line.
struct TpRead {
    const float *slots = nullptr;   // slot set of the exchange, sender 0
    uint32_t world = 0;
};
__device__ __forceinline__ bool tp_read_begin(const MvParams &p, int ctid, TpRead &t, float *misc) {
    const TpComm &c = *p.tp;
    const uint32_t k = *reinterpret_cast<const volatile uint32_t *>(c.seq);
    t.world = c.world;
    t.slots = c.slots[c.rank] + (size_t)((k - 1u) & 1u) * c.world * TP_DIM_MAX;
    volatile int *ok_s = reinterpret_cast<volatile int *>(misc + 40);   // free word of the misc scratch
    if (ctid == 0) {
        bool ok = true;
        const uint64_t t0 = global_ns();
        for (uint32_t q = 0; q < c.world && ok; ++q)
            while ((int)(ld_acquire_sys(c.flags[c.rank] + q) - k) < 0)
                if (global_ns() - t0 > kWaitNs) { ok = false; dev_flag_error(p.err, DERR_TIMEOUT_PEER); break; }
        *ok_s = ok;
    }
    named_bar_sync(1, MV_NCW * 32);
    return *ok_s != 0;
}
__device__ __forceinline__ float4 tp_add4(const TpRead &t, size_t i) {
    float4 a = __ldcg(reinterpret_cast<const float4 *>(t.slots + i));
    for (uint32_t q = 1; q < t.world; ++q) {
        const float4 b = __ldcg(reinterpret_cast<const float4 *>(t.slots + (size_t)q * TP_DIM_MAX + i));
        a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    return a;
}

template <bool PLAIN>
__device__ void mv_prologue(const MvParams &p, uint8_t *xq, float4 *xf, float *misc, int ctid) {
    const uint32_t nsub = p.cols / 32;
    float scale = 1.0f;
    TpRead tpr;
    const bool tp = p.tp_read != 0;
    if (tp && !tp_read_begin(p, ctid, tpr, misc)) return;   // error latched; the step's results are not used
    const bool has_add = tp || p.x_add;
    auto add4 = [&](size_t i) { return tp ? tp_add4(tpr, i) : *reinterpret_cast<const float4 *>(p.x_add + i); };
    if (p.norm_w) {
        float ss = 0.0f;
        for (uint32_t i = ctid * 4; i < p.cols; i += MV_NCW * 32 * 4) {
            float4 v = *reinterpret_cast<const float4 *>(p.x + i);
            if (has_add) {
                const float4 a = add4(i);
                v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
            }
            ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if ((ctid & 31) == 0) misc[8 + (ctid >> 5)] = ss;
        named_bar_sync(1, MV_NCW * 32);
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < MV_NCW; ++w) tot += misc[8 + w];
        scale = 1.0f / sqrtf(tot / (float)p.cols + p.eps);
    }
    const bool write_x = has_add && p.x_write && blockIdx.x == 0;
    const uint32_t u = ctid & 3;                                   // quarter of the block
    const uint32_t qmask = 0xFu << ((ctid & 31) & ~3u);            // the four lanes of this block
    for (uint32_t J = ctid >> 2; J < nsub; J += MV_NCW * 32 / 4) {
        const size_t e = (size_t)J * 32 + 8 * u;
        float v[8];
        float4 t0 = *reinterpret_cast<const float4 *>(p.x + e), t1 = *reinterpret_cast<const float4 *>(p.x + e + 4);
        v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w; v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
        if (has_add) {
            t0 = add4(e);
            t1 = add4(e + 4);
            v[0] += t0.x; v[1] += t0.y; v[2] += t0.z; v[3] += t0.w; v[4] += t1.x; v[5] += t1.y; v[6] += t1.z; v[7] += t1.w;
            if (write_x) {
                *reinterpret_cast<float4 *>(p.x_write + e) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4 *>(p.x_write + e + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
        }
        if (p.norm_w) {
            t0 = *reinterpret_cast<const float4 *>(p.norm_w + e);
            t1 = *reinterpret_cast<const float4 *>(p.norm_w + e + 4);
            const float w8[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = v[i] * scale * w8[i];
        }
        quant_block8<PLAIN>(v, u, qmask, J, xq, xf);
    }
}

// ---------------------------------------------------------------------------
// epilogue for one row (consumer warp 0; lane = row within the tile)
// ---------------------------------------------------------------------------
template <int EPI>
__device__ __forceinline__ void mv_epilogue(const MvParams &p, uint32_t row, bool valid, float va, float vb,
                                            uint32_t tp_k) {
    if constexpr (EPI == MV_EPI_STORE) {
        if (valid && p.tp_write) {   // this rank's partial row into slot [k % 2][rank] of every region
            const TpComm &c = *p.tp;
            const size_t off = ((size_t)(tp_k & 1u) * c.world + c.rank) * TP_DIM_MAX + row;
            for (uint32_t q = 0; q < c.world; ++q) c.slots[q][off] = va;
        } else if (valid) {
            p.y[row] = p.accumulate ? p.y[row] + va : va;
        }
    } else if constexpr (EPI == MV_EPI_SILU) {
        if (valid) p.y[row] = va / (1.0f + expf(-va)) * vb;
    } else {  // QKV: q/k rows get RoPE on (2i, 2i+1) pairs; k/v go to the fp16 cache
        const float other = __shfl_xor_sync(0xffffffffu, va, 1);
        if (!valid) return;
        const uint32_t pos = p.ctrl[0];
        if (pos >= p.max_ctx) {   // position past the KV capacity: report, never write out of bounds
            dev_flag_error(p.err, DERR_BAD_ARG);
            return;
        }
        const bool hm = p.kv_head_major != 0;
        if (row >= p.seg_end[1]) {
            p.vc[kv_index(hm, p.layer, pos, row - p.seg_end[1], p.max_ctx, p.kv_dim, p.head_dim)] = f32_to_f16_kv(va);
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
        else p.kc[kv_index(hm, p.layer, pos, local, p.max_ctx, p.kv_dim, p.head_dim)] = f32_to_f16_kv(outv);
    }
}

// Tiles of 16 rows. Non-dual: the 8 warps split the super-block columns of
// the chunk (warp w: columns w, w+8, ...). Dual (gate/up): warps 0-3 take
// W_gate, warps 4-7 the same rows of W_up, columns w%4, w%4+4, ...
template <int TYPE, int DUAL, int EPI>
__global__ void __launch_bounds__(MV_THREADS, 1) mv_fast_kernel(const MvParams p, const MvGeom geo) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int E = MvT<TYPE>::E, BB = MvT<TYPE>::BB;
    constexpr uint32_t SLOTS = DUAL ? 32u : 16u;
    constexpr uint32_t CW = DUAL ? 4u : 8u;             // warps sharing a matrix's columns
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nsub = p.cols / 32, nstage = geo.nstage, RS = geo.rs, CK = geo.ck;

    const uint32_t sbase = smem_u32(smem);
    float *misc = reinterpret_cast<float *>(smem + 256);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 256 + 60 * 4);
    float *red = reinterpret_cast<float *>(smem + 512);   // [2][8 warps][16 rows]
    uint8_t *xq = smem + MV_HDR;
    float4 *xf = reinterpret_cast<float4 *>(xq + (size_t)nsub * XQ_MAX_STRIDE);
    const uint32_t xq_a = sbase + MV_HDR, xf_a = xq_a + nsub * XQ_MAX_STRIDE;
    const uint32_t stage_bytes = SLOTS * RS;
    auto full_bar = [&](uint32_t s) { return sbase + 8u * s; };
    auto empty_bar = [&](uint32_t s) { return sbase + 8u * (MV_MAXST + s); };
    auto stage_addr = [&](uint32_t s) { return sbase + geo.stage0 + s * stage_bytes; };

    // rows of this CTA: an even-aligned balanced slice
    const uint32_t G = gridDim.x, b = blockIdx.x, hr = p.rows / 2;
    const uint32_t r0 = (uint32_t)(((uint64_t)b * hr) / G) * 2;
    const uint32_t r1 = (b + 1 == G) ? p.rows : (uint32_t)(((uint64_t)(b + 1) * hr) / G) * 2;
    const uint32_t nch = (p.cols + CK - 1) / CK;
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
        uint32_t slot = 0, round = 0, tile = 0, ch = 0, issued = 0;
        const bool mat = DUAL && lane >= 16;
        const uint32_t ri = (uint32_t)lane & 15u;
        const bool active = DUAL || lane < 16;
        for (uint32_t s = 0; s < nst; ++s) {
            if (s >= nstage && !mbar_wait_bounded(empty_bar(slot), (round - 1) & 1, kWaitNs)) {
                if (lane == 0) { *abort_flag = 1; dev_flag_error(p.err, DERR_TIMEOUT_EMPTY); }
                break;
            }
            if (*abort_flag) break;
            const uint32_t c0 = ch * CK, c1 = min(p.cols, c0 + CK);
            const uint64_t boff = (uint64_t)(c0 / E) * BB, blen = (uint64_t)((c1 - c0) / E) * BB;
            const uint32_t row = r0 + tile * 16 + ri;
            uint32_t tx = 0, dst_al = 0;
            uintptr_t lo = 0;
            if (active && row < r1) {
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
            if (++slot == nstage) { slot = 0; ++round; }
            if (++ch == nch) { ch = 0; ++tile; }
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
    pdl_wait();
    const uint32_t tp_k = (EPI == MV_EPI_STORE && p.tp_write) ? *reinterpret_cast<const volatile uint32_t *>(p.tp->seq) : 0u;
    mv_prologue<TYPE == T_Q6_K>(p, xq, xf, misc, threadIdx.x);
    named_bar_sync(1, MV_NCW * 32);

    float acc[2] = {0.f, 0.f};
    const int g = lane >> 2;
    const uint32_t msel = DUAL ? (uint32_t)warp >> 2 : 0u;       // matrix of this warp (dual)
    const uint32_t cw = DUAL ? (uint32_t)warp & 3u : (uint32_t)warp;
    uint32_t slot = 0, round = 0, tile = 0, ch = 0;
    for (uint32_t s = 0; s < nst; ++s) {
        bool ok = !*abort_flag;
        if (ok && !mbar_wait_bounded(full_bar(slot), round & 1, kWaitNs)) {
            ok = false;
            if (lane == 0) { *abort_flag = 1; dev_flag_error(p.err, DERR_TIMEOUT_FULL); }
        }
        const uint32_t c0 = ch * CK, c1 = min(p.cols, c0 + CK);
        if (ok) {
            const uint32_t ms = stage_addr(slot) + msel * 16u * RS;
            uint32_t pad0 = 0, pad1 = 0;
            if constexpr (TYPE != T_Q4_K) {
                // rows keep their global address modulo 16 in the slot
                const uint64_t boff = (uint64_t)(c0 / E) * BB;
                const uint32_t rbase = r0 + tile * 16;
                const uint32_t ra = min(rbase + g, r1 - 1), rb_ = min(rbase + g + 8, r1 - 1);
                const uint8_t *pa = msel ? p.wb + (uint64_t)ra * p.rb : seg_row_ptr(p, ra);
                const uint8_t *pb = msel ? p.wb + (uint64_t)rb_ * p.rb : seg_row_ptr(p, rb_);
                pad0 = (uint32_t)(reinterpret_cast<uintptr_t>(pa + boff) & 15);
                pad1 = (uint32_t)(reinterpret_cast<uintptr_t>(pb + boff) & 15);
            }
            for (uint32_t eo = cw * 256u; c0 + eo < c1; eo += CW * 256u)
                mv_unit<TYPE>(ms, RS, pad0, pad1, eo, (c0 + eo) >> 5, xq_a, xf_a, lane, c1 - c0 - eo, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(slot));
        if (++slot == nstage) { slot = 0; ++round; }
        if (++ch < nch) continue;
        ch = 0;
        // tile complete: per-warp row sums (over the 4 thread columns), then
        // over the warps of each matrix
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], 1);
            acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], 2);
        }
        float *rbuf = red + (tile & 1) * (MV_NCW * 16);
        if ((lane & 3) == 0) {
            rbuf[warp * 16 + g] = acc[0];
            rbuf[warp * 16 + g + 8] = acc[1];
        }
        acc[0] = acc[1] = 0.f;
        named_bar_sync(1, MV_NCW * 32);
        if (warp == 0) {
            const uint32_t li = (uint32_t)lane & 15u;
            float va = 0.f, vb = 0.f;
            if constexpr (DUAL) {
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    va += rbuf[w * 16 + li];
                    vb += rbuf[(4 + w) * 16 + li];
                }
            } else {
#pragma unroll
                for (int w = 0; w < 8; ++w) va += rbuf[w * 16 + li];
            }
            const uint32_t row = r0 + tile * 16 + li;
            // all 32 lanes take part (RoPE pairs use a warp shuffle); lanes 16-31 write nothing
            if (!*abort_flag) mv_epilogue<EPI>(p, row, lane < 16 && row < r1, va, vb, tp_k);
            else if constexpr (EPI == MV_EPI_QKV) (void)__shfl_xor_sync(0xffffffffu, va, 1);
        }
        ++tile;
    }
    if constexpr (EPI == MV_EPI_STORE) {
        if (p.tp_write) {
            // Tensor parallelism, writer side: once every CTA's rows are out
            // (system-scope fence, then a ticket), the last CTA publishes
            // exchange k + 1 into this rank's flag in every region and
            // advances the counter. The next writer kernel starts after this
            // one completes, so the ticket is back at zero by then.
            named_bar_sync(1, MV_NCW * 32);
            if (threadIdx.x == 0) {
                const TpComm &c = *p.tp;
                __threadfence_system();
                if (atomicAdd(c.ticket, 1u) == gridDim.x - 1) {
                    *c.ticket = 0u;
                    __threadfence_system();
                    for (uint32_t q = 0; q < c.world; ++q)
                        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(c.flags[q] + c.rank), "r"(tp_k + 1u) : "memory");
                    *reinterpret_cast<volatile uint32_t *>(c.seq) = tp_k + 1u;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// host side of the fast kernel
// ---------------------------------------------------------------------------

// Stage geometry for a shape: whole rows when 3+ stages of 16 (dual 32)
// full rows fit next to the x buffer, else 256-column multiples.
template <int TYPE> static MvGeom mv_geom(uint32_t cols, int dual) {
    MvGeom g = {};
    g.stage0 = (MV_HDR + (cols / 32) * (XQ_MAX_STRIDE + 16) + 1023u) & ~1023u;
    const uint32_t slots = dual ? 32u : 16u;
    const uint32_t avail = MV_SMEM > g.stage0 ? MV_SMEM - g.stage0 : 0;
    auto rs_for = [](uint32_t ck) {
        uint32_t rs = ((ck / MvT<TYPE>::E) * MvT<TYPE>::BB + 32 + 15) & ~15u;
        if (((rs / 16) & 1u) == 0) rs += 16;   // odd number of 16-byte units: conflict-free rows
        return rs;
    };
    uint32_t ck = (cols + 255) / 256 * 256;
    while (ck > 256 && avail / (slots * rs_for(ck)) < 3) ck = (ck / 2 + 255) / 256 * 256;
    g.ck = ck;
    g.rs = rs_for(ck);
    g.nstage = std::max(1u, std::min(MV_MAXST, avail / (slots * g.rs)));
    return g;
}
template <int TYPE> static uint32_t mv_smem_bytes(uint32_t cols, int dual) {
    const MvGeom g = mv_geom<TYPE>(cols, dual);
    return g.stage0 + g.nstage * (dual ? 32u : 16u) * g.rs;
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
    MvGeom g = {};
    switch (type) {
        case T_Q4_K: g = mv_geom<T_Q4_K>(cols, dual); break;
        case T_Q6_K: g = mv_geom<T_Q6_K>(cols, dual); break;
        default: g = mv_geom<T_Q8_0>(cols, dual); break;
    }
    return g.nstage >= 2 && g.stage0 + g.nstage * (dual ? 32u : 16u) * g.rs <= MV_SMEM;
}

template <int TYPE, int DUAL, int EPI>
static cudaError_t mv_fast_go(const MvParams &p0, int n_sm, cudaStream_t st, bool pdl, int grid_override) {
    const MvParams &p = p0;
    const MvGeom geo = mv_geom<TYPE>(p.cols, DUAL);
    const uint32_t smem = mv_smem_bytes<TYPE>(p.cols, DUAL);
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
    return cudaLaunchKernelEx(&cfg, kern, p, geo);
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
        case T_LNS8: VBS_GEN(T_LNS8); break;
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
