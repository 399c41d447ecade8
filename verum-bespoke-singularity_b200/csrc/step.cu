// step.cu -- the whole decode step as one persistent kernel.
//
// The op chain of a token (the reference's forward_token,
// src/vbs_specializer.c:270-349) is, per layer,
//   QKV   RMSNorm(attn_norm) + Q/K/V matvec
//   ATTN  RoPE + fp16 KV store + split-KV GQA attention
//   O     o_proj matvec
//   GU    residual add + RMSNorm(ffn_norm) + gate/up matvecs + SiLU(gate)*up
//   DOWN  down matvec
// then the residual add + RMSNorm(output_norm) + output matvec, and the
// greedy argmax. Launched as one kernel per op, every op pays a launch, a
// prologue and a pipeline fill and drain; on the small per-layer matrices
// that is as long as streaming their weights. Here one cooperative launch of
// one CTA per SM runs every op:
//
//  * A producer warp per CTA walks the same op list as the consumers and
//    streams the CTA's share of every op's weights (and of the KV cache
//    rows older than the current position) into a shared-memory ring with
//    1-D bulk TMA copies. Weights do not depend on activations, so it runs
//    ahead across op boundaries: while the consumers wait at a grid barrier
//    the next op's weights are already landing. The ring's empty/full
//    mbarriers are the only thing that paces it.
//  * Eight consumer warps run the ops. Between ops a grid barrier (one
//    counter in global memory, acquire/release, bounded spin) orders the
//    activations. Matvec units are (16-row tile x column chunk), split into
//    equal contiguous ranges per CTA. Each unit's row sums are stored
//    (plain stores, one writer per element) into its chunk's plane of
//    partial sums; the reader adds the planes in chunk order, so the sums
//    are deterministic and nothing needs clearing between steps. Only the
//    down projection is split into column chunk planes. Every other matvec
//    keeps whole rows: wider than one stage (the 70B shape's 8192 columns),
//    a tile's row chunks are consecutive stages of one CTA and its row sums
//    accumulate across them.
//  * What follows a matvec in the reference (residual add, RMSNorm, SiLU,
//    RoPE) is applied by the NEXT op as it reads the complete sums: every
//    CTA keeps its own copy of the residual stream x in shared memory and
//    updates it identically, so no extra pass or barrier is needed.
//  * Attention units are (KV head, split). The split that holds the current
//    position applies RoPE to the new key, stores the new K/V row (fp16, the
//    engine's rounding) into the cache and patches it into its staged copy.
//    q.K and p.V run on mma.sync m16n8k16 with f16 hi/lo operand splits
//    (fp32-accurate). Each split publishes its partial state on its head's
//    counter; once all have, the head's splits merge a share each.
//  * The argmax runs on slices per CTA; the last CTA advances the position
//    and token in the device control block.
//
// Every wait is bounded (p.wait_ns of %globaltimer, 2 s by default). A
// timeout sets an abort word that every other wait polls, records the error
// and unwinds the kernel.
#include "common.cuh"
#include "kernels.h"
#include "mv_core.cuh"

#include <algorithm>
#include <cstdio>

namespace vbs {

constexpr int SK_NCW = 8;                          // consumer warps (warpgroups 0 and 1)
constexpr int SK_CT = SK_NCW * 32;                 // consumer threads
constexpr int SK_THREADS = SK_CT + 128;            // + the producer warpgroup (one warp issues)
// Register split: launched at 168 per thread (384 x 168 = 64512), the
// producer warpgroup gives back to 40 and the consumers take 232:
// 256 x 232 + 128 x 40 = 64512, exactly the launch total.
constexpr uint32_t SK_REG_LAUNCH = 168, SK_REG_CONSUMER = 232, SK_REG_PRODUCER = 40;
static_assert(SK_CT * SK_REG_CONSUMER + 128 * SK_REG_PRODUCER <= SK_THREADS * SK_REG_LAUNCH, "register split");
constexpr uint32_t SK_NB = 8;                      // stages in flight at most (full/empty barrier pairs)
constexpr uint32_t SK_NU = 8;                      // matvec units per row-sum batch
constexpr uint32_t SK_PRM = 2048;                  // the launch's StepParams, copied once per launch
constexpr uint32_t SK_RED = 3072;                  // row-sum batches: [2][SK_NU][8 warps][16 rows] floats
constexpr uint32_t SK_HDR = SK_RED + 2 * SK_NU * 8 * 16 * 4;   // barriers, flags, row-sum batches
constexpr uint32_t SK_SMEM = 227u * 1024u;
constexpr uint32_t SK_AP = 64;                     // attention positions per stage
constexpr uint32_t SK_MAX_SPLITS = 128;
constexpr int SK_GS = 8;                           // query-head slots per KV head
constexpr float SK_LAZY = 8.0f;                    // softmax rescale threshold (log2 units)
// sync words: [0] grid barrier, [1] abort, [2] argmax ticket,
// [16 + h] KV head h's attention splits published in this step (all layers),
// [SK_SLOTS + 2c] argmax slots
constexpr uint32_t SK_TICKET0 = 16, SK_MAX_KV = 112, SK_SLOTS = SK_TICKET0 + SK_MAX_KV;

enum : int { K_QKV = 0, K_ATTN = 1, K_O = 2, K_GU = 3, K_DOWN = 4, K_OUT = 5, K_ARGMAX = 6 };

__host__ __device__ inline int sk_kind(uint32_t i, uint32_t L, uint32_t &layer) {
    if (i < 5 * L) { layer = i / 5; return (int)(i % 5); }
    layer = L - 1;
    return i == 5 * L ? K_OUT : K_ARGMAX;
}

// ---------------------------------------------------------------------------
// op descriptors
// ---------------------------------------------------------------------------
struct SkMv {
    int type;
    int gu;                 // gate/up: slot rows 0-7 gate, 8-15 up (tiles of 8 rows); writes h
    int chunk_major;        // units ordered chunk by chunk (a CTA spans one or two column chunks)
    const uint8_t *packed;  // stage units, (tile, chunk) at (tile * nch + chunk) * 16 * rs
    uint32_t rows, cols;
    float *out;             // chunk c's sums at out + c * rows (one writer per element)
    StepMvGeom g;
    int tpw;                // tensor parallelism: 0 local, 1 o/down partial planes to every rank, 2 logits shard to every rank
    int norm;               // the input was RMSNorm-ed without its scale: multiply the row sums by sk_norm_scale
    uint32_t tp_k;          // exchange index (its slot set is tp_k % 2)
};

// Tile and chunk of this op's unit u.
__device__ __forceinline__ void sk_unit(const SkMv &d, uint32_t u, uint32_t &tile, uint32_t &ch) {
    if (d.chunk_major) { ch = u / d.g.ntiles; tile = u % d.g.ntiles; }
    else { tile = u / d.g.nch; ch = u % d.g.nch; }
}

__device__ __forceinline__ float *sk_acc(const StepParams &p, uint32_t l) { return p.acc + (uint64_t)l * p.acc_layer; }
__device__ __forceinline__ uint32_t sk_qkv_rows(const StepParams &p) { return (p.nqh + 2 * p.nkh) * p.hd; }
// Per-layer activations: [q|k|v sums] [o_proj] [h = SiLU(gate)*up] [down,
// one plane of dim partial sums per column chunk]
__device__ __forceinline__ float *sk_acc_o(const StepParams &p, uint32_t l) { return sk_acc(p, l) + sk_qkv_rows(p); }
__device__ __forceinline__ float *sk_acc_h(const StepParams &p, uint32_t l) { return sk_acc_o(p, l) + p.dim; }
__device__ __forceinline__ float *sk_acc_down(const StepParams &p, uint32_t l) { return sk_acc_h(p, l) + p.ffn; }
__device__ __forceinline__ float *sk_logits(const StepParams &p) { return p.logits; }

__device__ __forceinline__ SkMv sk_mv_desc(const StepParams &p, int kind, uint32_t l) {
    SkMv d = {};
    const uint32_t qd = p.nqh * p.hd, kvd = p.nkh * p.hd;
    const StepLayer &L = p.layers[kind == K_OUT ? 0 : l];
    switch (kind) {
        case K_QKV:
            d.type = p.t_qkv; d.packed = L.qkv; d.norm = 1;
            d.rows = qd + 2 * kvd; d.cols = p.dim; d.out = sk_acc(p, l); d.g = p.geo[STEP_QKV];
            break;
        case K_O:
            d.type = p.t_o; d.packed = L.o;
            d.rows = p.dim; d.cols = qd; d.out = sk_acc_o(p, l); d.g = p.geo[STEP_O];
            break;
        case K_GU:
            d.type = p.t_gu; d.gu = 1; d.packed = L.gu; d.norm = 1;
            d.rows = p.ffn; d.cols = p.dim; d.out = sk_acc_h(p, l); d.g = p.geo[STEP_GU];
            break;
        case K_DOWN:
            d.type = p.t_down; d.packed = L.down; d.chunk_major = 1;
            d.rows = p.dim; d.cols = p.ffn; d.out = sk_acc_down(p, l); d.g = p.geo[STEP_DOWN];
            break;
        default:   // K_OUT
            d.type = p.t_out; d.packed = p.out; d.norm = 1;
            d.rows = p.vocab; d.cols = p.dim; d.out = sk_logits(p); d.g = p.geo[STEP_OUT];
            break;
    }
    return d;
}

// Output row held by stage slot r (0..15) of tile `tile`. Gate/up tiles hold
// 8 rows of each matrix: slot r < 8 is gate row tile*8 + r, slot r >= 8 the
// up row tile*8 + r - 8.
__host__ __device__ __forceinline__ uint32_t sk_slot_row(bool gu, uint32_t tile, uint32_t r) {
    return gu ? tile * 8 + (r & 7u) : tile * 16 + r;
}

// This CTA's contiguous share [u0, u1) of U units.
// (U * gridDim.x < 2^32: U is at most a few hundred thousand units.)
__device__ __forceinline__ void sk_range(uint32_t U, uint32_t &u0, uint32_t &u1) {
    u0 = blockIdx.x * U / gridDim.x;
    u1 = (blockIdx.x + 1) * U / gridDim.x;
}

// Stages per row unit. A matrix wider than one stage's column chunk is
// either split into chunk planes (the down projection: chunk-major units,
// the reader adds the planes) or, every other op, streamed as row chunks:
// a tile's chunks are consecutive stages whose row sums accumulate, and the
// sums are written once, whole (what SiLU, RoPE and the argmax need).
__device__ __forceinline__ uint32_t sk_row_stages(const SkMv &d) { return d.chunk_major ? 1u : d.g.nch; }

// This CTA's units of op d, whole tiles when a tile spans several stages
// (only in the WIDE kernel instances: elsewhere every such op has whole
// rows in one stage). The producer and the consumers walk the same range.
template <bool WIDE>
__device__ __forceinline__ void sk_mv_range(const SkMv &d, uint32_t &u0, uint32_t &u1) {
    const uint32_t rs = WIDE ? sk_row_stages(d) : 1u;
    sk_range(d.g.ntiles * d.g.nch / rs, u0, u1);
    u0 *= rs;
    u1 *= rs;
}

struct SkAttn {
    uint32_t S, h, split, t0, t1, nst;
    bool has;
};

// Attention unit of this CTA: KV head h, split `split` of S over [0, seq).
__device__ __forceinline__ SkAttn sk_attn_unit(const StepParams &p, uint32_t seq) {
    SkAttn a;
    a.S = max(1u, min(p.attn_splits, (seq + SK_AP - 1) / SK_AP));
    const uint32_t c = blockIdx.x;
    a.has = c < p.nkh * a.S;
    a.h = a.has ? c / a.S : 0;
    a.split = a.has ? c % a.S : 0;
    uint32_t per = (seq + a.S - 1) / a.S;
    per = (per + SK_AP - 1) / SK_AP * SK_AP;
    a.t0 = min(seq, a.split * per);
    a.t1 = min(seq, a.t0 + per);
    a.nst = a.has ? (a.t1 - a.t0 + SK_AP - 1) / SK_AP : 0;
    return a;
}

// Timeline stamps of a profiling build (VBS_STEP_TRACE): slot k of op i of
// this CTA. Nothing in the product build.
#ifdef VBS_STEP_TRACE
__device__ __forceinline__ void sk_stamp(const StepParams &p, uint32_t i, int k) {
    if (p.trace)
        p.trace[((size_t)blockIdx.x * (5 * p.n_layers + 2) + i) * SK_TR_SLOTS + k] = global_ns();
}
// The same, taken only once v has arrived (v feeds an instruction issued
// before the clock is read): the latency of the load that produced v.
__device__ __forceinline__ void sk_stamp_after(const StepParams &p, uint32_t i, int k, float v) {
    uint64_t t;
    asm volatile("{\n .reg .pred q;\n setp.nan.f32 q, %1, %1;\n mov.u64 %0, %%globaltimer;\n @q mov.u64 %0, 0;\n}"
                 : "=l"(t) : "f"(v) : "memory");
    if (p.trace) p.trace[((size_t)blockIdx.x * (5 * p.n_layers + 2) + i) * SK_TR_SLOTS + k] = t;
}
#define SK_STAMP(p, i, k) sk_stamp(p, i, k)
// One dependent L2 load of src by this thread, timed into slots k, k + 1.
#define SK_PROBE(p, i, k, src) do { SK_STAMP(p, i, k); sk_stamp_after(p, i, (k) + 1, __ldcg(src)); } while (0)
#else
#define SK_STAMP(p, i, k) ((void)0)
#define SK_PROBE(p, i, k, src) ((void)0)
#endif

// ---------------------------------------------------------------------------
// waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// mbarrier phase wait, bounded (p.wait_ns), giving up early when the grid aborts.
__device__ __forceinline__ bool sk_wait(uint32_t bar, uint32_t parity, const StepParams &p) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && (*reinterpret_cast<const volatile uint32_t *>(p.sync + 1) || global_ns() - t0 > p.wait_ns))
            return false;
    }
}

// Generic-proxy writes to a ring slot (byte copies, zero fill, the patched
// row) must be ordered before the TMA (async proxy) writes that later reuse
// the slot.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void sk_abort(const StepParams &p, uint32_t code) {
    atomicExch(&p.sync[1], 1u);
    dev_flag_error(p.err, code);
}

// Grid barrier among the consumer warps of all CTAs: arrive, then wait for
// `target` arrivals. Returns false, the same value in every consumer thread
// of the CTA, when this CTA or the grid aborted: thread 0 decides after the
// first CTA barrier and the second one publishes its decision. The arrival is
// one release add (it publishes the CTA's writes, which the CTA barrier
// ordered before it) and the poll an acquire load, with no separate fences:
// measured 1.6 -> 1.3 us per barrier and a third of the release skew.
__device__ __forceinline__ bool sk_grid_sync(const StepParams &p, uint32_t target, volatile int *flag,
                                             volatile int *cta_abort, uint32_t op) {
    named_bar_sync(1, SK_CT);
    if (threadIdx.x == 0) {
        // p.drop_op: a bounded-wait test withholds CTA 0's arrival here
        if (op != p.drop_op || blockIdx.x != 0)
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&p.sync[0]) : "memory");
        bool ok = *cta_abort == 0;
        uint64_t t0 = 0;
        for (uint32_t it = 1; ok && ld_acquire_gpu(&p.sync[0]) < target; ++it) {
            if ((it & 63u) == 0) {
                if (it == 64) t0 = global_ns();
                if (*reinterpret_cast<const volatile uint32_t *>(&p.sync[1])) { ok = false; break; }
                if (it > 64 && global_ns() - t0 > p.wait_ns) { sk_abort(p, DERR_TIMEOUT_PEER); ok = false; break; }
            }
        }
        *flag = ok ? 1 : 0;
    }
    named_bar_sync(1, SK_CT);
    return *flag != 0;
}

// ---------------------------------------------------------------------------
// tensor parallelism over peer memory (TpComm): per step, exchange 2l is
// layer l's o_proj partials, 2l + 1 its down partials, 2L the logits. Every
// value travels as one 64-bit word, (k + 1) << 32 | float bits, which the
// writers store into every rank's region in their row flush (st.relaxed.sys:
// single-copy atomic). A reader loads its own region's words until each
// carries k + 1, so it needs no fence, flag or grid barrier on either side:
// a word with k + 1 is the value. Exchange k uses slot set k % 2; a writer
// reaches exchange k + 2 only after reading k + 1 from every rank, and every
// rank wrote k + 1 behind a grid barrier that followed its reads of k.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sk_tp_index(const StepParams &p, uint32_t base, int kind, uint32_t l) {
    return base + (kind == K_OUT ? 2u * p.n_layers : 2u * l + (kind == K_DOWN ? 1u : 0u));
}

__device__ __forceinline__ void st_word_sys(uint64_t *a, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}

__device__ __forceinline__ void ld_words_sys(const uint64_t *a, uint64_t &x, uint64_t &y) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(a));
}

// A word load that has not seen k + 1 yet: true (give up) once the grid
// aborted or the wait passed its limit, recording a peer timeout.
__device__ __noinline__ bool sk_word_give_up(const StepParams &p, uint64_t t0, volatile int *cta_abort) {
    if (*reinterpret_cast<const volatile uint32_t *>(&p.sync[1])) { *cta_abort = 1; return true; }
    if (global_ns() - t0 <= p.wait_ns) return false;
    *cta_abort = 1;
    sk_abort(p, DERR_TIMEOUT_PEER);
    return true;
}

// v[c][0..7] = the 8 values at a + c * stride (words, 16-byte aligned) for
// planes c < n, once every word carries `want`; all planes' loads are in
// flight together. Garbage (and the abort set) when the wait gives up.
template <int NP>
__device__ __forceinline__ void sk_ld8_words(const StepParams &p, const uint64_t *a, uint64_t stride, uint32_t n,
                                             uint32_t want, float (&v)[NP][8], volatile int *cta_abort) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        bool ok = true;
#pragma unroll
        for (int c = 0; c < NP; ++c) {
            if ((uint32_t)c >= n) continue;
            uint64_t w[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) ld_words_sys(a + c * stride + 2 * k, w[2 * k], w[2 * k + 1]);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                ok &= (uint32_t)(w[k] >> 32) == want;
                v[c][k] = __uint_as_float((uint32_t)w[k]);
            }
        }
        if (ok) break;
        if (it == 0) t0 = global_ns();
        else if ((it & 15u) == 0 && sk_word_give_up(p, t0, cta_abort)) break;
    }
}

// ---------------------------------------------------------------------------
// shared-memory map
// ---------------------------------------------------------------------------
struct SkSmem {
    uint32_t base;                 // shared address of the dynamic buffer
    uint8_t *ptr;
    uint32_t ring, ring_bytes;     // the stage ring: shared address and size
    __device__ uint32_t full(uint32_t i) const { return base + 8u * (i % SK_NB); }            // of stage i
    __device__ uint32_t empty(uint32_t i) const { return base + 8u * (SK_NB + i % SK_NB); }
    __device__ volatile int *abort_flag() const { return reinterpret_cast<volatile int *>(ptr + 256); }
    __device__ volatile int *sync_flag() const { return reinterpret_cast<volatile int *>(ptr + 260); }
    __device__ uint32_t *scratch_u() const { return reinterpret_cast<uint32_t *>(ptr + 512); }   // 64 words
    __device__ float *misc() const { return reinterpret_cast<float *>(ptr + 1024); }            // 256 floats
    __device__ float *red() const { return reinterpret_cast<float *>(ptr + SK_RED); }          // [2][SK_NU][8][16]
};
static_assert(16 * SK_NB <= 256 && SK_HDR % 1024 == 0 && sizeof(StepParams) <= SK_RED - SK_PRM, "shared-memory header");

// Position in the stage sequence, walked identically by the producer and the
// consumers. Stages take their own size from a ring of bytes (a stage never
// straddles the end: it starts over at 0), so small stages (attention,
// Q4_K) keep more bytes in flight than the largest stage would allow in
// fixed slots. Stage i uses barrier pair i % SK_NB; the phase parity of its
// use is (i / SK_NB) & 1.
struct SkRing {
    uint32_t idx = 0, off = 0;
    __device__ __forceinline__ uint32_t place(uint32_t bytes, uint32_t ring_bytes) {
        if (off + bytes > ring_bytes) off = 0;
        return off;
    }
    __device__ __forceinline__ uint32_t parity() const { return (idx / SK_NB) & 1u; }
    __device__ __forceinline__ void advance(uint32_t bytes) { off += bytes; ++idx; }
};

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------
// Before stage r.idx of `bytes` may be issued, every older stage that held
// any of its bytes, and the stage SK_NB back that used its barrier pair, must
// be released by the consumers. Lane j of the producer warp tracks the
// in-flight stage with index = j (mod SK_NB): its byte range and whether it
// is still held. Stages are released in order, so the producer waits on the
// oldest one until the new range is free.
struct SkInflight {
    uint32_t s = 0, e = 0, tail = 0;   // lane's stage [s, e); oldest stage not seen released
    bool held = false;
};

__device__ __forceinline__ bool sk_reserve(const StepParams &p, const SkSmem &S, SkRing &r, SkInflight &f,
                                           uint32_t bytes, int lane) {
    const uint32_t o = r.place(bytes, S.ring_bytes);
    for (;;) {
        const bool clash = f.held && f.s < o + bytes && o < f.e;
        if (!__any_sync(0xffffffffu, clash) && r.idx - f.tail < SK_NB) return true;
        if (!sk_wait(S.empty(f.tail), (f.tail / SK_NB) & 1u, p)) {
            if (lane == 0) sk_abort(p, DERR_TIMEOUT_EMPTY);
            return false;
        }
        if ((uint32_t)lane == f.tail % SK_NB) f.held = false;
        ++f.tail;
    }
}

__device__ __forceinline__ void sk_issued(SkRing &r, SkInflight &f, uint32_t bytes, int lane) {
    if ((uint32_t)lane == r.idx % SK_NB) { f.s = r.off; f.e = r.off + bytes; f.held = true; }
    __syncwarp();
    r.advance(bytes);
}

template <bool WIDE>
__device__ __forceinline__ void sk_producer(const StepParams &p, const SkSmem &S, uint32_t seq) {
    const int lane = threadIdx.x & 31;
    const uint32_t nops = 5 * p.n_layers + 2;
    SkRing r;
    SkInflight f;
    bool ok = true;
    // weights and KV rows are read once per step: first out of L2, so the
    // activations, the norm weights and the kernel's code stay in it
    const uint64_t once = l2_policy_evict_first();
    for (uint32_t i = 0; i < nops && ok; ++i) {
        uint32_t l;
        const int kind = sk_kind(i, p.n_layers, l);
        if (kind == K_ARGMAX) continue;
        if (lane == 0) SK_STAMP(p, i, 3);
        if (kind == K_ATTN) {
            const SkAttn a = sk_attn_unit(p, seq);
            const uint64_t hb = (((uint64_t)l * p.nkh + a.h) * p.max_ctx) * p.hd;
            const uint32_t rowb = p.hd * 2, sb = 2 * SK_AP * rowb;   // K rows, then V rows at SK_AP * rowb
            for (uint32_t s = 0; s < a.nst; ++s) {
                if (!sk_reserve(p, S, r, f, sb, lane)) { ok = false; break; }
                const uint32_t t = a.t0 + s * SK_AP, len = min(SK_AP, a.t1 - t), bytes = len * rowb;
                if (lane == 0) {
                    const uint32_t dst = S.ring + r.off;
                    mbar_arrive_expect_tx(S.full(r.idx), 2 * bytes);
                    bulk_g2s_hint(dst, p.kc + hb + (uint64_t)t * p.hd, bytes, S.full(r.idx), once);
                    bulk_g2s_hint(dst + SK_AP * rowb, p.vc + hb + (uint64_t)t * p.hd, bytes, S.full(r.idx), once);
                }
                sk_issued(r, f, sb, lane);
            }
            if (lane == 0) SK_STAMP(p, i, 4);
            continue;
        }
        if (kind == K_QKV || kind == K_GU || kind == K_OUT) {   // the norm weight, for every CTA
            const float *nw = kind == K_QKV ? p.layers[l].attn_norm : (kind == K_GU ? p.layers[l].ffn_norm : p.out_norm);
            const uint32_t nb = p.dim * 4;
            if (!sk_reserve(p, S, r, f, nb, lane)) { ok = false; break; }
            if (lane == 0) {
                mbar_arrive_expect_tx(S.full(r.idx), nb);
                bulk_g2s(S.ring + r.off, nw, nb, S.full(r.idx));
            }
            sk_issued(r, f, nb, lane);
        }
        const SkMv d = sk_mv_desc(p, kind, l);
        const uint32_t bytes = 16u * d.g.rs;
        uint32_t u0, u1;
        sk_mv_range<WIDE>(d, u0, u1);
        for (uint32_t u = u0; u < u1; ++u) {
            if (!sk_reserve(p, S, r, f, bytes, lane)) { ok = false; break; }
            uint32_t tile, ch;
            sk_unit(d, u, tile, ch);
            if (lane == 0) {
                mbar_arrive_expect_tx(S.full(r.idx), bytes);
                bulk_g2s_hint(S.ring + r.off, d.packed + (uint64_t)(tile * d.g.nch + ch) * bytes, bytes, S.full(r.idx), once);
            }
            sk_issued(r, f, bytes, lane);
        }
        if (lane == 0) SK_STAMP(p, i, 4);
    }
    if (!ok) {
        // wait (bounded) for copies still in flight before the CTA may exit
        for (uint32_t s = f.tail; s < r.idx; ++s) mbar_wait_bounded(S.full(s), (s / SK_NB) & 1u, p.wait_ns);
    }
}

// ---------------------------------------------------------------------------
// consumer prologues: the quantized input vector of a matvec op. Thread
// (quad q = tid/4, quarter u = tid%4) owns elements 8u..8u+7 of the 32-value
// blocks q, q+64, q+128, ...: the layout quant_block8 consumes, so values stay
// in registers from the load to the quantizer. All loads of a prologue are
// issued before the first is used: while the weight stream saturates the
// memory system every dependent round trip costs microseconds.
// ---------------------------------------------------------------------------
constexpr int SK_PB = 2;        // blocks per thread and pass in the norm prologue (one pass to dim 4096)

__device__ __forceinline__ void ld8_cg(const float *src, float v[8]) {
    const float4 a = __ldcg(reinterpret_cast<const float4 *>(src)), b = __ldcg(reinterpret_cast<const float4 *>(src + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void ld8_g(const float *src, float v[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(src)), b = __ldg(reinterpret_cast<const float4 *>(src + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// The prologues run once per op: their code is cold in the instruction
// cache every time, so it is kept to one out-of-line copy per routine
// instead of being inlined at every call site and unrolled iteration.
__device__ __noinline__ void sk_quant(int type, float v0, float v1, float v2, float v3, float v4, float v5, float v6,
                                      float v7, uint32_t u, uint32_t qmask, uint32_t J, uint8_t *xq, float4 *xf) {
    const float v[8] = {v0, v1, v2, v3, v4, v5, v6, v7};
    if (type == T_Q6_K) quant_block8<true>(v, u, qmask, J, xq, xf);
    else quant_block8<false>(v, u, qmask, J, xq, xf);
}
__device__ __forceinline__ void sk_quant(int type, const float v[8], uint32_t u, uint32_t qmask, uint32_t J, uint8_t *xq,
                                         float4 *xf) {
    sk_quant(type, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], u, qmask, J, xq, xf);
}
// Two blocks J0, J1 of this quad at once (quant_block8x2); J1 only when has1.
__device__ __noinline__ void sk_quant2(int type, float a0, float a1, float a2, float a3, float a4, float a5, float a6,
                                       float a7, float b0, float b1, float b2, float b3, float b4, float b5, float b6,
                                       float b7, uint32_t u, uint32_t qmask, uint32_t J0, uint32_t J1, bool has1,
                                       uint8_t *xq, float4 *xf) {
    const float v[2][8] = {{a0, a1, a2, a3, a4, a5, a6, a7}, {b0, b1, b2, b3, b4, b5, b6, b7}};
    const uint32_t J[2] = {J0, J1};
    if (type == T_Q6_K) quant_block8x2<true>(v, u, qmask, J, has1, xq, xf);
    else quant_block8x2<false>(v, u, qmask, J, has1, xq, xf);
}
__device__ __forceinline__ void sk_quant2(int type, const float v[2][8], uint32_t u, uint32_t qmask, uint32_t J0,
                                          uint32_t J1, bool has1, uint8_t *xq, float4 *xf) {
    sk_quant2(type, v[0][0], v[0][1], v[0][2], v[0][3], v[0][4], v[0][5], v[0][6], v[0][7], v[1][0], v[1][1], v[1][2],
              v[1][3], v[1][4], v[1][5], v[1][6], v[1][7], u, qmask, J0, J1, has1, xq, xf);
}

// Elements e..e+7 of the embedding row of `token` (src/vbs_host_math.h:136-142).
__device__ __noinline__ void sk_embed8(const StepParams &p, uint32_t token, uint32_t e, float *out) {
    const uint32_t E = (uint32_t)block_elems(p.t_embd), BB = (uint32_t)block_bytes(p.t_embd);
    const uint8_t *row = p.embd + (uint64_t)token * row_bytes(p.t_embd, p.dim);
#pragma unroll 1
    for (int k = 0; k < 8; ++k) out[k] = dq_elem(p.t_embd, row + ((e + k) / E) * BB, (int)((e + k) % E));
}

// Residual update x += add (or x = the embedding row when add is NULL,
// src/vbs_host_math.h:136-142), RMSNorm (src/vbs_host_math.h:28-36) with
// the norm weight, and, when `quant`, the quantized vector. The norm weight
// arrives as a ring stage of dim floats (the producer issues it ahead of the
// op's weight stages), so it is never a load on this path. RMSNorm's scalar
// 1/rms(x) does not wait here: x * w is quantized as it is (the block
// quantization is scale-free) and the matvec multiplies its row sums by the
// scale (sk_norm_scale), once every warp's sum of squares is in misc[0..7].
constexpr int SK_MAXPL = 4;      // partial planes summed by the norm prologue

// WORDS (instances with tensor parallelism): when `want` is not 0 the planes
// are exchange words carrying it. WIDE: widths above 4096, in passes of
// SK_PB blocks per thread, the quantizer reading each pass's x back from
// shared memory; without it one pass with x in registers.
constexpr uint32_t SK_PSTEP = SK_PB * (SK_CT / 4);   // blocks per prologue pass
template <bool WORDS, bool WIDE>
__device__ __forceinline__ void sk_prologue_norm(const StepParams &p, const SkSmem &S, SkRing &r, float *x,
                                                 const void *add, uint32_t nadd, uint32_t want, uint32_t token,
                                                 bool quant, int type, uint8_t *xq, float4 *xf, uint32_t op) {
    const uint32_t ctid = threadIdx.x, q = ctid >> 2, u = ctid & 3u, nsub = p.dim / 32;
    const uint32_t qmask = 0xFu << ((ctid & 31u) & ~3u);
    constexpr uint32_t PSTEP = SK_PSTEP;
    const uint32_t npass = WIDE ? (nsub + PSTEP - 1) / PSTEP : 1u;
    if (ctid == 0) SK_STAMP(p, op, 8);
    float xv[SK_PB][8];
    float ss = 0.f;
#pragma unroll 1
    for (uint32_t pass = 0; pass < npass; ++pass) {
    const uint32_t qp = q + pass * PSTEP;
    // add = nadd planes of dim partial sums, summed in plane order
#pragma unroll
    for (int r = 0; r < SK_PB; ++r) {
        const uint32_t J = qp + r * (SK_CT / 4);
        if (J < nsub) {
            const uint32_t e = J * 32 + 8 * u;
            if (add) {
                // planes in order, SK_MAXPL loads in flight at a time
                for (uint32_t c0 = 0; c0 < nadd; c0 += SK_MAXPL) {
                    float pv[SK_MAXPL][8];
                    if (WORDS && want) {
                        sk_ld8_words<SK_MAXPL>(p, static_cast<const uint64_t *>(add) + (uint64_t)c0 * p.dim + e, p.dim,
                                               nadd - c0, want, pv, S.abort_flag());
                    } else {
#pragma unroll
                        for (int c = 0; c < SK_MAXPL; ++c)
                            if (c0 + c < nadd) ld8_cg(static_cast<const float *>(add) + (uint64_t)(c0 + c) * p.dim + e, pv[c]);
                    }
#pragma unroll
                    for (int k = 0; k < 8; ++k) xv[r][k] = c0 ? xv[r][k] + pv[0][k] : pv[0][k];
#pragma unroll
                    for (int c = 1; c < SK_MAXPL; ++c)
                        if (c0 + c < nadd)
#pragma unroll
                            for (int k = 0; k < 8; ++k) xv[r][k] += pv[c][k];
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < SK_PB; ++r) {
        const uint32_t J = qp + r * (SK_CT / 4);
        if (J >= nsub) continue;
        const uint32_t e = J * 32 + 8 * u;
        float4 *xs = reinterpret_cast<float4 *>(x + e);
        if (add) {
            const float4 o0 = xs[0], o1 = xs[1];
            xv[r][0] += o0.x; xv[r][1] += o0.y; xv[r][2] += o0.z; xv[r][3] += o0.w;
            xv[r][4] += o1.x; xv[r][5] += o1.y; xv[r][6] += o1.z; xv[r][7] += o1.w;
        } else {
            float ev[8];
            sk_embed8(p, token, e, ev);
#pragma unroll
            for (int k = 0; k < 8; ++k) xv[r][k] = ev[k];
        }
        xs[0] = make_float4(xv[r][0], xv[r][1], xv[r][2], xv[r][3]);
        xs[1] = make_float4(xv[r][4], xv[r][5], xv[r][6], xv[r][7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss = fmaf(xv[r][k], xv[r][k], ss);
    }
    }
    ss = warp_sum(ss);
    if (ctid == 0) SK_STAMP(p, op, 5);
    float *misc = S.misc();
    if ((ctid & 31u) == 0) misc[ctid >> 5] = ss;
    // the norm weight stage (long landed by now); released after use
    const int lane = (int)(ctid & 31u);
    volatile int *cta_abort = S.abort_flag();
    const uint32_t nb = p.dim * 4, ws = S.ring + r.place(nb, S.ring_bytes);
    const bool got = __all_sync(0xffffffffu, !*cta_abort && sk_wait(S.full(r.idx), r.parity(), p));
    if (!got && lane == 0 && !*cta_abort) { *cta_abort = 1; sk_abort(p, DERR_TIMEOUT_FULL); }
    if (ctid == 0) SK_STAMP(p, op, 6);
    static_assert(SK_PB == 2, "the prologue quantizes its two blocks together");
#pragma unroll 1
    for (uint32_t pass = 0; quant && got && pass < npass; ++pass) {
        const uint32_t qp = q + pass * PSTEP;
        if (qp >= nsub) break;
        float v[SK_PB][8];
#pragma unroll
        for (int r2 = 0; r2 < SK_PB; ++r2) {
            const uint32_t J = qp + r2 * (SK_CT / 4);
            const uint32_t e = (J < nsub ? J : qp) * 32 + 8 * u;
            if (WIDE) {   // this thread's x of this pass, as it stored it above
                const float4 o0 = reinterpret_cast<const float4 *>(x + e)[0], o1 = reinterpret_cast<const float4 *>(x + e)[1];
                xv[r2][0] = o0.x; xv[r2][1] = o0.y; xv[r2][2] = o0.z; xv[r2][3] = o0.w;
                xv[r2][4] = o1.x; xv[r2][5] = o1.y; xv[r2][6] = o1.z; xv[r2][7] = o1.w;
            }
            const uint4 w0 = lds_u128(ws + e * 4), w1 = lds_u128(ws + e * 4 + 16);
            const float wv[8] = {__uint_as_float(w0.x), __uint_as_float(w0.y), __uint_as_float(w0.z), __uint_as_float(w0.w),
                                 __uint_as_float(w1.x), __uint_as_float(w1.y), __uint_as_float(w1.z), __uint_as_float(w1.w)};
#pragma unroll
            for (int k = 0; k < 8; ++k) v[r2][k] = xv[r2][k] * wv[k];
        }
        sk_quant2(type, v, u, qmask, qp, qp + SK_CT / 4, qp + SK_CT / 4 < nsub, xq, xf);
    }
    if (ctid == 0) SK_STAMP(p, op, 7);
    if (ctid == 0 && add) SK_PROBE(p, op, 9, static_cast<const float *>(add) + 8 * nadd);
    __syncwarp();
    if (lane == 0) mbar_arrive(S.empty(r.idx));
    r.advance(nb);
}

// Quantizes the n values at src (fp32, global memory, written earlier in
// the step): NB blocks per thread per batch, every load of a batch issued
// before any is used.
template <int NB>
__device__ __noinline__ void sk_prologue_vec(uint32_t n, int type, const float *src, uint8_t *xq, float4 *xf) {
    static_assert(NB == 2, "blocks are quantized in pairs");
    const uint32_t ctid = threadIdx.x, q = ctid >> 2, u = ctid & 3u, nsub = n / 32;
    const uint32_t qmask = 0xFu << ((ctid & 31u) & ~3u);
    for (uint32_t J0 = q; J0 < nsub; J0 += NB * (SK_CT / 4)) {
        float v[NB][8];
        const uint32_t J1 = J0 + SK_CT / 4;
        ld8_cg(src + J0 * 32 + 8 * u, v[0]);
        if (J1 < nsub) ld8_cg(src + J1 * 32 + 8 * u, v[1]);
        else
#pragma unroll
            for (int k = 0; k < 8; ++k) v[1][k] = 0.0f;
        sk_quant2(type, v, u, qmask, J0, J1, J1 < nsub, xq, xf);
    }
}

// ---------------------------------------------------------------------------
// matvec consumer: this CTA's units of one op. The 8 warps split each
// stage's 256-column super-blocks; the unit's row sums go out with plain
// stores into its column chunk's plane, or for gate/up rows as
// SiLU(gate)*up.
// ---------------------------------------------------------------------------
// RMSNorm's scale 1/sqrt(mean(x^2) + eps) (src/vbs_host_math.h:28-36) from
// the warps' sums of squares the norm prologue left in misc[0..7], summed in
// warp order.
__device__ __forceinline__ float sk_norm_scale(const StepParams &p, const SkSmem &S) {
    const float *misc = S.misc();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < SK_NCW; ++w) tot += misc[w];
    return 1.0f / sqrtf(tot / (float)p.dim + p.eps);
}

template <int TYPE, bool TPX, bool WIDE>
__device__ __forceinline__ void sk_mv_consume(const StepParams &p, const SkMv &d, const SkSmem &S, SkRing &r,
                                              uint32_t xq_a, uint32_t xf_a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const float nscale = d.norm ? sk_norm_scale(p, S) : 1.0f;
    const uint32_t RS = d.g.rs, CK = d.g.ck, SB = 16u * RS;
    volatile int *cta_abort = S.abort_flag();
    float *red = S.red();
    const uint32_t RC = WIDE ? sk_row_stages(d) : 1u;
    uint32_t u0, u1;
    sk_mv_range<WIDE>(d, u0, u1);
    float acc[2] = {0.f, 0.f};   // WIDE: carried over a tile's row chunks
    uint32_t k = 0, ub = u0;     // WIDE: row units finished; first unit of the current batch
    for (uint32_t u = u0; u < u1; ++u) {
        uint32_t tile, ch;
        sk_unit(d, u, tile, ch);
        // one decision per warp: the MMAs and shuffles below need all 32 lanes
        const uint32_t ms = S.ring + r.place(SB, S.ring_bytes);
        const bool got = __all_sync(0xffffffffu, !*cta_abort && sk_wait(S.full(r.idx), r.parity(), p));
        if (!got && lane == 0 && !*cta_abort) { *cta_abort = 1; sk_abort(p, DERR_TIMEOUT_FULL); }
        if constexpr (!WIDE) acc[0] = acc[1] = 0.f;
        if (got) {
            const uint32_t c0 = ch * CK, c1 = min(d.cols, c0 + CK);
            // packed rows start 16-byte aligned in the stage: no alignment pads
            // chunks are at most 16 super-blocks (the plan caps them at 4096
            // columns): at most two per warp, as straight-line code so their
            // independent load/MMA chains interleave
            const uint32_t e0 = (uint32_t)warp * 256u, e1 = e0 + SK_NCW * 256u;
            if (c0 + e0 < c1) mv_unit<TYPE, true>(ms, RS, 0u, 0u, e0, (c0 + e0) >> 5, xq_a, xf_a, lane, c1 - c0 - e0, acc);
            if (c0 + e1 < c1) mv_unit<TYPE, true>(ms, RS, 0u, 0u, e1, (c0 + e1) >> 5, xq_a, xf_a, lane, c1 - c0 - e1, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(S.empty(r.idx));
        r.advance(SB);
        if (WIDE && ch + 1 < RC) continue;   // the tile's next row chunk adds to the same sums
        // the unit's row sums: over the thread columns here, then over the
        // warps for a batch of SK_NU units at once: each warp leaves its 16
        // partials in the batch buffer, and after one consumer barrier the
        // threads sum the batch's rows in warp order and write them. Batches
        // alternate between two buffers, so the next batch's partials never
        // meet a buffer still being read (its writers passed that barrier).
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], 1);
            acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], 2);
        }
        const uint32_t kk = WIDE ? k : u - u0, slot = kk % SK_NU;
        if (WIDE && slot == 0) ub = u + 1 - RC;
        float *batch = red + ((kk / SK_NU) & 1u) * (SK_NU * SK_NCW * 16);
        if ((lane & 3) == 0) {
            batch[(slot * SK_NCW + warp) * 16 + g] = acc[0];
            batch[(slot * SK_NCW + warp) * 16 + g + 8] = acc[1];
        }
        if constexpr (WIDE) {
            ++k;
            acc[0] = acc[1] = 0.f;
        }
        if (slot == SK_NU - 1 || u + 1 == u1) {
            named_bar_sync(1, SK_CT);
            const uint32_t n = slot + 1, j = threadIdx.x >> 4, rr = threadIdx.x & 15u;
            if (j < n && !*cta_abort) {
                uint32_t tile, ch;
                // WIDE: chunk 0 of a row-chunked tile, whose sums are whole
                sk_unit(d, WIDE ? ub + j * RC : u - slot + j, tile, ch);
                const float *b = batch + j * SK_NCW * 16;
                float va = 0.f;
#pragma unroll
                for (int w = 0; w < SK_NCW; ++w) va += b[w * 16 + rr];
                va *= nscale;
                const uint32_t row = sk_slot_row(d.gu != 0, tile, rr);
                if (d.gu) {   // h = SiLU(gate) * up (src/vbs_host_math.h:53-57): slot rr < 8 gate, rr + 8 up
                    if (rr < 8 && row < d.rows) {
                        float vu = 0.f;
#pragma unroll
                        for (int w = 0; w < SK_NCW; ++w) vu += b[w * 16 + rr + 8];
                        vu *= nscale;
                        d.out[row] = va / (1.0f + expf(-va)) * vu;
                    }
                } else if (TPX && row < d.rows && d.tpw) {   // this rank's partial into every rank's region
                    const TpComm &c = *p.tp;
                    const uint64_t word = (uint64_t)(d.tp_k + 1u) << 32 | __float_as_uint(va);
                    if (d.tpw == 1) {
                        const size_t off = (size_t)(d.tp_k & 1u) * c.world * TP_DIM_MAX +
                                           ((size_t)c.rank * d.g.nch + ch) * d.rows + row;
                        for (uint32_t q = 0; q < c.world; ++q) st_word_sys(c.ll[q] + off, word);
                    } else {
                        const size_t off = (size_t)c.rank * d.rows + row;
                        for (uint32_t q = 0; q < c.world; ++q) st_word_sys(c.ll_logits[q] + off, word);
                    }
                } else if (row < d.rows) {
                    d.out[(uint64_t)ch * d.rows + row] = va;
                }
            }
        }
    }
}

// Types the kernel instance carries code for: a compile-time list (a
// specialized instance) or all three (TQ4 = TQ6 = TQ8 = true).
template <bool HAS_Q4, bool HAS_Q6, bool HAS_Q8, bool TPX, bool WIDE>
__device__ __forceinline__ void sk_mv_dispatch(const StepParams &p, const SkMv &d, const SkSmem &S, SkRing &r,
                                               uint32_t xq_a, uint32_t xf_a) {
    if constexpr (HAS_Q4) if (d.type == T_Q4_K) { sk_mv_consume<T_Q4_K, TPX, WIDE>(p, d, S, r, xq_a, xf_a); return; }
    if constexpr (HAS_Q6) if (d.type == T_Q6_K) { sk_mv_consume<T_Q6_K, TPX, WIDE>(p, d, S, r, xq_a, xf_a); return; }
    if constexpr (HAS_Q8) if (d.type == T_Q8_0) { sk_mv_consume<T_Q8_0, TPX, WIDE>(p, d, S, r, xq_a, xf_a); return; }
}

// ---------------------------------------------------------------------------
// attention consumer
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sk_pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void sk_split_h2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = sk_pack_h2(a - f.x, b - f.y);
}

// RoPE of the pair (d, d+1), d even, at position pos (src/vbs_host_math.h:38-51,
// the same expression as the per-op kernels' Q/K/V epilogue).
__device__ __forceinline__ float2 sk_rope(float a, float b, uint32_t d, uint32_t pos, uint32_t hd, float theta) {
    const float ang = (float)pos * powf(theta, -(float)d / (float)hd);
    float s, c;
    sincosf(ang, &s, &c);
    return make_float2(a * c - b * s, a * s + b * c);
}

// Merges the S partial states [m, l, pad, pad, o[HD]] of a KV head's query
// heads in split order, for the outputs [e_lo, e_hi) of the G * HD (e_lo,
// e_hi even): every thread two outputs, all loads of a batch of splits in
// flight at once (a single round trip for S <= SK_MB), batches combined with
// the usual rescale.
constexpr uint32_t SK_MB = 20;
template <int HD>
__device__ __noinline__ void sk_attn_merge(const StepParams &p, const SkAttn &a, uint32_t G, const float *parts, float *outp,
                                           uint32_t e_lo, uint32_t e_hi) {
    constexpr uint32_t RS = 4 + HD;
    constexpr size_t part_stride = (size_t)SK_GS * RS;
    for (uint32_t e = e_lo + 2 * threadIdx.x; e < e_hi; e += 2 * SK_CT) {
        const uint32_t gg = e / HD, d = e % HD;
        const float *src = parts + gg * RS;
        float M = -INFINITY, L = 0.f, O0 = 0.f, O1 = 0.f;
        for (uint32_t s0 = 0; s0 < a.S; s0 += SK_MB) {
            float ms[SK_MB], ls[SK_MB];
            float2 os[SK_MB];
#pragma unroll
            for (uint32_t u = 0; u < SK_MB; ++u) {
                const bool in = s0 + u < a.S;
                const float *ps = src + (size_t)(s0 + u) * part_stride;
                ms[u] = in ? __ldcg(ps) : -INFINITY;
                ls[u] = in ? __ldcg(ps + 1) : 0.f;
                os[u] = in ? __ldcg(reinterpret_cast<const float2 *>(ps + 4 + d)) : make_float2(0.f, 0.f);
            }
            float Mb = M;
#pragma unroll
            for (uint32_t u = 0; u < SK_MB; ++u) Mb = fmaxf(Mb, ms[u]);
            if (Mb == -INFINITY) continue;
            const float rs = (M == -INFINITY) ? 0.f : exp2f(M - Mb);
            L *= rs;
            O0 *= rs;
            O1 *= rs;
#pragma unroll
            for (uint32_t u = 0; u < SK_MB; ++u) {
                const float wt = (ms[u] == -INFINITY) ? 0.f : exp2f(ms[u] - Mb);
                L = fmaf(ls[u], wt, L);
                O0 = fmaf(os[u].x, wt, O0);
                O1 = fmaf(os[u].y, wt, O1);
            }
            M = Mb;
        }
        const float il = 1.0f / L;
        *reinterpret_cast<float2 *>(outp + e) = make_float2(O0 * il, O1 * il);
    }
}

template <int HD>
__device__ __forceinline__ void sk_attn(const StepParams &p, uint32_t l, uint32_t pos, uint32_t seq, const SkSmem &S, SkRing &r,
                        float *sh, uint32_t op) {
    constexpr int RS = 4 + HD;                 // state row [m, l, pad, pad, o[HD]]
    constexpr uint32_t ROWB = HD * 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp >> 2, wl = warp & 3;  // warp groups take alternate stages
    volatile int *cta_abort = S.abort_flag();
    const SkAttn a = sk_attn_unit(p, seq);
    if (!a.has) return;
    const uint32_t G = p.nqh / p.nkh;
    const float *accq = sk_acc(p, l);
    const uint32_t qdim = p.nqh * HD, kvdim = p.nkh * HD;

    // q as the A operand: a 16 x HD f16 matrix in shared memory, row g =
    // fp16(q_g), row g+8 = fp16(q_g - fp16(q_g)) (zero for g >= G); RoPE'd
    // and pre-scaled by scale*log2(e). Read back with ldmatrix per k-step.
    // The split that holds the current position also forms the new cache
    // row here: RoPE'd key and value, fp16 with the engine's rounding, into
    // the cache and into kvn (plain order) for the stage patch below. One
    // loop, so RoPE's code exists once.
    constexpr uint32_t ASTR = HD * 2 + 16;     // padded row: conflict-free ldmatrix
    const uint32_t a_base = smem_u32(sh + SK_NCW * G * RS);
    const uint32_t kvn = a_base + 16 * ASTR;   // new K row [HD] f16, then the V row
    const int g = lane >> 2, qd = 2 * (lane & 3);
    const uint64_t hb = (((uint64_t)l * p.nkh + a.h) * p.max_ctx) * HD;
    const bool has_pos = pos >= a.t0 && pos < a.t1;
    {
        const float qscale = p.scale * 1.4426950408889634f;
        constexpr uint32_t NQ = SK_GS * (HD / 2);
        const uint32_t n_items = NQ + (has_pos ? HD / 2 : 0u);
        for (uint32_t k = threadIdx.x; k < n_items; k += SK_CT) {
            const bool isq = k < NQ;
            const uint32_t gg = isq ? k / (HD / 2) : 0u, dd = 2 * ((isq ? k : k - NQ) % (HD / 2));
            const float *src = isq ? accq + (a.h * G + gg) * HD + dd : accq + qdim + a.h * HD + dd;
            float2 v = make_float2(0.f, 0.f);
            if (!isq || gg < G) {
                const float2 raw = __ldcg(reinterpret_cast<const float2 *>(src));
                v = sk_rope(raw.x, raw.y, dd, pos, HD, p.theta);
            }
            if (isq) {
                uint32_t hi, lo;
                sk_split_h2(v.x * qscale, v.y * qscale, hi, lo);
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(a_base + gg * ASTR + dd * 2), "r"(hi) : "memory");
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(a_base + (gg + 8) * ASTR + dd * 2), "r"(lo) : "memory");
            } else {
                const float2 vr = __ldcg(reinterpret_cast<const float2 *>(src + kvdim));
                const uint32_t kh = (uint32_t)f32_to_f16_kv(v.x) | ((uint32_t)f32_to_f16_kv(v.y) << 16);
                const uint32_t vh = (uint32_t)f32_to_f16_kv(vr.x) | ((uint32_t)f32_to_f16_kv(vr.y) << 16);
                // swizzled place of dims dd, dd+1 (inside one 16-byte chunk)
                const uint32_t off = (((dd >> 3) ^ (pos & 7u)) << 3) + (dd & 7u);
                *reinterpret_cast<uint32_t *>(p.kc + hb + (uint64_t)pos * HD + off) = kh;
                *reinterpret_cast<uint32_t *>(p.vc + hb + (uint64_t)pos * HD + off) = vh;
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(kvn + dd * 2), "r"(kh) : "memory");
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(kvn + HD * 2 + dd * 2), "r"(vh) : "memory");
            }
        }
        named_bar_sync(1, SK_CT);
    }
    if (threadIdx.x == 0) SK_STAMP(p, op, 1);
    const uint32_t a_lane = a_base + (lane & 15) * ASTR + (lane >> 4) * 16;

    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float mrun = -INFINITY, lrun = 0.f;

    for (uint32_t s = 0; s < a.nst; ++s) {
        // one decision per warp: the MMAs and shuffles below need all 32 lanes
        const uint32_t stg = S.ring + r.place(2 * SK_AP * ROWB, S.ring_bytes);
        const bool got = __all_sync(0xffffffffu, !*cta_abort && sk_wait(S.full(r.idx), r.parity(), p));
        if (!got && lane == 0 && !*cta_abort) { *cta_abort = 1; sk_abort(p, DERR_TIMEOUT_FULL); }
        if (threadIdx.x == 0 && s == 0) SK_STAMP(p, op, 8);
        if (threadIdx.x == 0 && s + 1 == a.nst) SK_STAMP(p, op, 9);
        const uint32_t ts = a.t0 + s * SK_AP, tb = ts + 16 * wl;
        if (got && (int)(s & 1) == grp && tb < a.t1) {
            const uint32_t kst = stg + 16 * wl * ROWB;
            const uint32_t vst = stg + SK_AP * ROWB + 16 * wl * ROWB;
            // rows past the end of the unit: zero V (p = 0 must not meet stale bits)
            if (tb + 16 > a.t1) {
                const uint32_t nv = a.t1 - tb;
                for (uint32_t i = lane; i < (16 - nv) * (ROWB / 16); i += 32) {
                    const uint32_t rr = nv + i / (ROWB / 16), cc = i % (ROWB / 16);
                    asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(vst + rr * ROWB + cc * 16), "r"(0u) : "memory");
                }
            }
            // the current position: the new row (formed above) into this stage,
            // 16-byte chunks swizzled by the position as in the cache
            if (pos >= tb && pos < tb + 16 && pos < a.t1) {
                constexpr uint32_t NC = HD / 8;   // 16-byte chunks per row
                if ((uint32_t)lane < 2 * NC) {
                    const uint32_t isv = (uint32_t)lane >= NC, c = (uint32_t)lane % NC, rr = pos - tb;
                    const uint4 val = lds_u128(kvn + isv * HD * 2 + c * 16);
                    const uint32_t dst = (isv ? vst : kst) + rr * ROWB + ((c ^ (pos & 7u)) << 4);
                    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(val.x), "r"(val.y), "r"(val.z),
                                 "r"(val.w) : "memory");
                }
            }
            __syncwarp();
            float sc2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk += 2) {
                uint32_t qa0[4], qa1[4];
                ldsm_x4(a_lane + kk * 32, qa0[0], qa0[1], qa0[2], qa0[3]);
                ldsm_x4(a_lane + kk * 32 + 32, qa1[0], qa1[1], qa1[2], qa1[3]);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const uint32_t rr = 8 * j + (lane & 7), c = 2 * kk + (lane >> 3);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kst + rr * ROWB + ((c ^ (rr & 7u)) << 4), b0, b1, b2, b3);
                    mma_f16_acc(sc2[j], qa0, b0, b1);
                    mma_f16_acc(sc2[j], qa1, b2, b3);
                }
            }
            float sc[4] = {sc2[0][0] + sc2[0][2], sc2[0][1] + sc2[0][3], sc2[1][0] + sc2[1][2], sc2[1][1] + sc2[1][3]};
            const uint32_t pq = tb + qd;
            if (pq >= a.t1) sc[0] = -INFINITY;
            if (pq + 1 >= a.t1) sc[1] = -INFINITY;
            if (pq + 8 >= a.t1) sc[2] = -INFINITY;
            if (pq + 9 >= a.t1) sc[3] = -INFINITY;
            float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            if (mx > mrun + SK_LAZY) {
                const float rs = exp2f(mrun - mx);
                lrun *= rs;
#pragma unroll
                for (int n = 0; n < HD / 8; ++n) { o[n][0] *= rs; o[n][1] *= rs; o[n][2] *= rs; o[n][3] *= rs; }
                mrun = mx;
            }
            float pe[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) pe[e] = exp2f(sc[e] - mrun);
            lrun += (pe[0] + pe[1]) + (pe[2] + pe[3]);
            uint32_t pa[4];
            sk_split_h2(pe[0], pe[1], pa[0], pa[1]);
            sk_split_h2(pe[2], pe[3], pa[2], pa[3]);
#pragma unroll
            for (int n = 0; n < HD / 8; n += 2) {
                const uint32_t rr = (lane & 7) + 8 * ((lane >> 3) & 1), c = n + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(vst + rr * ROWB + ((c ^ (rr & 7u)) << 4), b0, b1, b2, b3);
                mma_f16_acc(o[n], pa, b0, b1);
                mma_f16_acc(o[n + 1], pa, b2, b3);
            }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(S.empty(r.idx));
        r.advance(2 * SK_AP * ROWB);
    }

    // warp states -> shared memory, merge over the 8 warps
    if (threadIdx.x == 0) SK_STAMP(p, op, 5);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
    lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
    if ((uint32_t)g < G) {
        float *row = sh + (warp * G + g) * RS;
        if ((lane & 3) == 0) { row[0] = mrun; row[1] = lrun; }
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
            row[4 + 8 * n + qd] = o[n][0] + o[n][2];
            row[5 + 8 * n + qd] = o[n][1] + o[n][3];
        }
    }
    named_bar_sync(1, SK_CT);
    // per query head: the maximum over the warps, each warp's weight, the sum
    float *wts = S.misc();   // [SK_NCW][SK_GS] weights, [SK_GS] maxima, [SK_GS] sums
    if (threadIdx.x < G) {
        const uint32_t gg = threadIdx.x;
        float M = -INFINITY, L = 0.f;
        for (int w = 0; w < SK_NCW; ++w) M = fmaxf(M, sh[(w * G + gg) * RS]);
        for (int w = 0; w < SK_NCW; ++w) {
            const float m = sh[(w * G + gg) * RS];
            const float wt = (m == -INFINITY) ? 0.f : exp2f(m - M);
            wts[w * SK_GS + gg] = wt;
            L += sh[(w * G + gg) * RS + 1] * wt;
        }
        wts[SK_NCW * SK_GS + gg] = M;
        wts[SK_NCW * SK_GS + SK_GS + gg] = L;
    }
    named_bar_sync(1, SK_CT);
    float *work = reinterpret_cast<float *>(p.attn_work);
    constexpr size_t part_stride = (size_t)SK_GS * RS;
    float *mypart = work + ((size_t)a.h * SK_MAX_SPLITS + a.split) * part_stride;
    float *outp = p.att + (size_t)a.h * G * HD;
    for (uint32_t k = threadIdx.x; k < G * HD; k += SK_CT) {
        const uint32_t gg = k / HD, d = k % HD;
        float O = 0.f;
#pragma unroll
        for (int w = 0; w < SK_NCW; ++w) O += sh[(w * G + gg) * RS + 4 + d] * wts[w * SK_GS + gg];
        const float L = wts[SK_NCW * SK_GS + SK_GS + gg];
        if (a.S == 1) {
            outp[gg * HD + d] = O / L;
        } else {
            if (d == 0) { mypart[gg * RS] = wts[SK_NCW * SK_GS + gg]; mypart[gg * RS + 1] = L; }
            mypart[gg * RS + 4 + d] = O;
        }
    }
    if (a.S == 1) return;
    // Publish this split's state with one release add on the head's counter
    // (the CTA barrier orders every thread's stores before it; the counter
    // counts splits over the step's layers, so layer l waits for S * (l + 1)),
    // wait until every split of the head published, then merge this split's
    // share of the head's outputs: the S CTAs of a head merge in parallel.
    named_bar_sync(1, SK_CT);
    if (threadIdx.x == 0) SK_STAMP(p, op, 6);
    volatile int *flag = S.sync_flag();
    if (threadIdx.x == 0) {
        uint32_t *cnt = &p.sync[SK_TICKET0 + a.h];
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
        const uint32_t want = a.S * (l + 1u);
        bool ok = !*cta_abort;
        uint64_t t0 = 0;
        for (uint32_t it = 1; ok && ld_acquire_gpu(cnt) < want; ++it) {
            if ((it & 63u) == 0) {
                if (it == 64) t0 = global_ns();
                if (*reinterpret_cast<const volatile uint32_t *>(&p.sync[1])) { ok = false; break; }
                if (it > 64 && global_ns() - t0 > p.wait_ns) { sk_abort(p, DERR_TIMEOUT_PEER); ok = false; break; }
            }
        }
        if (!ok) *cta_abort = 1;
        *flag = ok ? 1 : 0;
    }
    named_bar_sync(1, SK_CT);
    if (threadIdx.x == 0) SK_STAMP(p, op, 7);
    if (!*flag) return;
    const uint32_t per = ((G * HD + a.S - 1) / a.S + 1) & ~1u;
    const uint32_t e_lo = min(G * HD, a.split * per), e_hi = min(G * HD, e_lo + per);
    sk_attn_merge<HD>(p, a, G, work + (size_t)a.h * SK_MAX_SPLITS * part_stride, outp, e_lo, e_hi);
    if (threadIdx.x == 0) SK_PROBE(p, op, 10, work + (size_t)a.h * SK_MAX_SPLITS * part_stride + 4);
}

// ---------------------------------------------------------------------------
// argmax over the logits (first maximum wins, src/vbs_cpu_main.c:78-80)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void sk_pick(float &best, uint32_t &bi, float ov, uint32_t oi) {
    if (oi != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
}

__device__ __forceinline__ void sk_block_argmax(const SkSmem &S, float &best, uint32_t &bi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int o = 16; o; o >>= 1) sk_pick(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    float *mv = S.misc() + 64;
    uint32_t *mi = S.scratch_u();
    if (lane == 0) { mv[warp] = best; mi[warp] = bi; }
    named_bar_sync(1, SK_CT);
    best = lane < SK_NCW ? mv[lane] : -INFINITY;
    bi = lane < SK_NCW ? mi[lane] : 0xFFFFFFFFu;
    for (int o = 16; o; o >>= 1) sk_pick(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    named_bar_sync(1, SK_CT);
}

__device__ __noinline__ void sk_argmax(const StepParams &p, const SkSmem &S, uint32_t pos, uint32_t tp_base) {
    // under TP every rank gathers the full logits (exchange words) and picks
    // the same token; the values also go to the plain logits area for readback
    const uint32_t n = p.tp ? p.vocab_full : p.vocab, per = (n + gridDim.x - 1) / gridDim.x;
    const uint32_t lo = min(n, blockIdx.x * per), hi = min(n, lo + per);
    float best = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    if (p.tp) {
        const TpComm &c = *p.tp;
        const uint32_t want = tp_base + 2u * p.n_layers + 1u;
        const uint64_t *lw = c.ll_logits[c.rank];
        volatile int *cta_abort = S.abort_flag();
        for (uint32_t i = lo + threadIdx.x; i < hi; i += SK_CT) {
            uint64_t w = 0, t0 = 0;
            for (uint32_t it = 0;; ++it) {
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(lw + i));
                if ((uint32_t)(w >> 32) == want) break;
                if (it == 0) t0 = global_ns();
                else if ((it & 15u) == 0 && sk_word_give_up(p, t0, cta_abort)) break;
            }
            const float v = __uint_as_float((uint32_t)w);
            c.logits[c.rank][i] = v;
            sk_pick(best, bi, v, i);
        }
    } else {
        const float *lg = sk_logits(p);
        for (uint32_t i = lo + threadIdx.x; i < hi; i += SK_CT) sk_pick(best, bi, __ldcg(lg + i), i);
    }
    sk_block_argmax(S, best, bi);
    if (*S.abort_flag()) return;   // a word never came: no token, the error is recorded
    volatile int *flag = S.sync_flag();
    if (threadIdx.x == 0) {
        p.sync[SK_SLOTS + 2 * blockIdx.x] = __float_as_uint(best);
        p.sync[SK_SLOTS + 2 * blockIdx.x + 1] = bi;
        __threadfence();
        *flag = atomicAdd(&p.sync[2], 1u) == gridDim.x - 1;
    }
    named_bar_sync(1, SK_CT);
    if (!*flag) return;
    __threadfence();
    best = -INFINITY;
    bi = 0xFFFFFFFFu;
    for (uint32_t c = threadIdx.x; c < gridDim.x; c += SK_CT)
        sk_pick(best, bi, __uint_as_float(__ldcg(&p.sync[SK_SLOTS + 2 * c])), __ldcg(&p.sync[SK_SLOTS + 2 * c + 1]));
    sk_block_argmax(S, best, bi);
    if (threadIdx.x == 0) {
        if (bi == 0xFFFFFFFFu) bi = 0;
        const uint32_t np = pos + 1u;
        p.ctrl[1] = bi;
        p.ctrl[0] = np;
        if (p.tp) *reinterpret_cast<volatile uint32_t *>(p.tp->seq) = tp_base + 2u * p.n_layers + 1u;
        if (p.hist && np < p.hist_cap) p.hist[np] = bi;
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// Instances: step_kernel<0, true, true, true, *> serves every planned shape
// with runtime type and head_dim dispatch; specialized instances carry only
// the code their model uses (a kernel that runs every op of a step is large,
// and its instruction fetch is otherwise a bottleneck). TPX instances add
// the tensor-parallel exchanges; the one-GPU instances carry none of it.
// WIDE instances add row chunks across stages and the multi-pass norm
// prologue for models wider than 4096; the others carry none of that (one
// kernel with both paths ran the 8B shape 3% slower).
template <int HD, bool HAS_Q4, bool HAS_Q6, bool HAS_Q8, bool TPX, bool WIDE>
__global__ void __launch_bounds__(SK_THREADS, 1) step_kernel(const __grid_constant__ StepParams p_in) {
    static_assert(65536 / SK_THREADS / 8 * 8 >= SK_REG_LAUNCH, "launch register count");
    extern __shared__ __align__(1024) uint8_t smem[];
    // Every op reads the parameters right after a grid barrier, when the
    // constant cache has long lost them (an L2 round trip per dependent
    // read): they are read from shared memory instead, copied once here.
    {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&p_in);
        uint32_t *dst = reinterpret_cast<uint32_t *>(smem + SK_PRM);
        for (uint32_t k = threadIdx.x; k < sizeof(StepParams) / 4; k += blockDim.x) dst[k] = src[k];
    }
    const StepParams &p = *reinterpret_cast<const StepParams *>(smem + SK_PRM);
    static_assert(sizeof(StepParams) % 4 == 0, "parameter copy by words");
    SkSmem S;
    S.ptr = smem;
    S.base = smem_u32(smem);
    S.ring = S.base + p_in.ring_off;
    S.ring_bytes = p_in.ring_bytes;
    const int warp = threadIdx.x >> 5;
    // read once: the last CTA rewrites the control block at the end of the step
    const uint32_t pos = *reinterpret_cast<const volatile uint32_t *>(p_in.ctrl);
    const uint32_t token = *reinterpret_cast<const volatile uint32_t *>(p_in.ctrl + 1);
    // ctrl[2]: device-driven generation stopped (vbs_cu_decoder_run_control):
    // this step does nothing, the same decision in every CTA
    if (*reinterpret_cast<const volatile uint32_t *>(p_in.ctrl + 2)) return;
    if (pos >= p_in.max_ctx || token >= (p_in.tp ? p_in.vocab_full : p_in.vocab)) {   // the same decision in every CTA: nothing runs, nothing waits
        if (blockIdx.x == 0 && threadIdx.x == 0) dev_flag_error(p_in.err, DERR_BAD_ARG);
        return;
    }
    const uint32_t seq = pos + 1;
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < SK_NB; ++i) {
            mbar_init(S.full(i), 1);
            mbar_init(S.empty(i), SK_NCW);
        }
        *S.abort_flag() = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (warp >= SK_NCW) {   // producer warpgroup
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(SK_REG_PRODUCER));
        if (warp == SK_NCW) sk_producer<WIDE>(p, S, seq);
        return;
    }
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(SK_REG_CONSUMER));

    // ------------------------------ consumers ------------------------------
    float *x = reinterpret_cast<float *>(smem + p.x_off);
    uint8_t *xq = smem + p.xq_off;
    float4 *xf = reinterpret_cast<float4 *>(smem + p.xf_off);
    const uint32_t xq_a = S.base + p.xq_off, xf_a = S.base + p.xf_off;
    float *sh = reinterpret_cast<float *>(xq);   // attention states alias the x buffers
    SkRing r;
    const uint32_t nops = 5 * p.n_layers + 2;
    // tensor parallelism: exchanges completed before this step
    const uint32_t tp_base = (TPX && p.tp) ? *reinterpret_cast<const volatile uint32_t *>(p.tp->seq) : 0u;
    uint32_t nsync = 0;   // grid barriers taken (TPX instances skip some)
    for (uint32_t i = 0; i < nops; ++i) {
        if (i > 0) {
            uint32_t lp;
            const int pk = sk_kind(i - 1, p.n_layers, lp);
            if (TPX && p.tp && (pk == K_O || pk == K_DOWN)) {
                // the next op only reads exchange words, which it checks one
                // by one; an abort is taken at the next grid barrier
                named_bar_sync(1, SK_CT);
            } else if (!sk_grid_sync(p, (TPX ? ++nsync : i) * gridDim.x, S.sync_flag(), S.abort_flag(), i)) {
                break;
            }
        }
        uint32_t l;
        const int kind = sk_kind(i, p.n_layers, l);
        if (threadIdx.x == 0) SK_STAMP(p, i, 0);
        if (threadIdx.x == 0) SK_STAMP(p, i, 11);   // back to back: the cost of a stamp itself
        if (kind == K_ATTN) {
            if constexpr (HD != 0) sk_attn<HD>(p, l, pos, seq, S, r, sh, i);
            else if (p.hd == 128) sk_attn<128>(p, l, pos, seq, S, r, sh, i);
            else sk_attn<64>(p, l, pos, seq, S, r, sh, i);
            if (threadIdx.x == 0) SK_STAMP(p, i, 2);
            continue;
        }
        if (kind == K_ARGMAX) {
            sk_argmax(p, S, pos, tp_base);
            if (threadIdx.x == 0) SK_STAMP(p, i, 2);
            continue;
        }
        SkMv d = sk_mv_desc(p, kind, l);
#ifdef VBS_STEP_TRACE
        if (threadIdx.x == 0) {   // when a parameter-block value, then the layer's pointer, is in hand
            sk_stamp_after(p, i, 12, __uint_as_float(d.g.ntiles | 1u));
            sk_stamp_after(p, i, 13, __uint_as_float((uint32_t)reinterpret_cast<uintptr_t>(d.packed) | 1u));
        }
#endif
        if (TPX && p.tp && (kind == K_O || kind == K_DOWN || kind == K_OUT)) {
            d.tpw = kind == K_OUT ? 2 : 1;
            d.tp_k = sk_tp_index(p, tp_base, kind, l);
        }
        uint32_t u0, u1;
        sk_mv_range<WIDE>(d, u0, u1);
        const bool work = u1 > u0;
        uint32_t xq_u = xq_a, xf_u = xf_a;   // shared addresses of x block 0 for mv_unit
        if (kind == K_QKV || kind == K_GU || kind == K_OUT) {
            // every CTA keeps x current, whether or not it has units of this op
            const float *add = kind == K_QKV ? (l ? sk_acc_down(p, l - 1) : nullptr)
                                             : (kind == K_GU ? sk_acc_o(p, l) : sk_acc_down(p, p.n_layers - 1));
            uint32_t nadd = kind == K_GU ? 1u : p.geo[STEP_DOWN].nch, want = 0;
            const void *planes = add;
            if (TPX && p.tp && add) {   // the exchanged partials: every rank's planes, in rank order
                const int src = kind == K_GU ? K_O : K_DOWN;
                const uint32_t k = sk_tp_index(p, tp_base, src, kind == K_QKV ? l - 1 : (kind == K_GU ? l : p.n_layers - 1));
                planes = p.tp->ll[p.tp->rank] + (size_t)(k & 1u) * p.tp->world * TP_DIM_MAX;
                nadd *= p.tp->world;
                want = k + 1u;
            }
            sk_prologue_norm<TPX, WIDE>(p, S, r, x, planes, nadd, want, token, work, d.type, xq, xf, i);
        } else if (kind == K_O) {
            if (threadIdx.x == 0) SK_STAMP(p, i, 8);
            if (work) sk_prologue_vec<2>(d.cols, d.type, p.att, xq, xf);
            if (threadIdx.x == 0) SK_PROBE(p, i, 9, p.att + 64);
        } else if (work) {   // K_DOWN: only the column chunks of this CTA's units
            const uint32_t c_lo = u0 / d.g.ntiles, c_hi = (u1 - 1) / d.g.ntiles;
            const uint32_t col0 = c_lo * d.g.ck, col1 = min(d.cols, (c_hi + 1) * d.g.ck);
            const float *hp = sk_acc_h(p, l) + col0;
            if (threadIdx.x == 0) SK_STAMP(p, i, 8);
            sk_prologue_vec<2>(col1 - col0, d.type, hp, xq, xf);
            if (threadIdx.x == 0) SK_PROBE(p, i, 9, hp + 64);
            xq_u = xq_a - (col0 / 32) * (d.type == T_Q6_K ? XQ_PLAIN_STRIDE : XQ_SLOT_STRIDE);   // mv_unit indexes x blocks from column 0
            xf_u = xf_a - (col0 / 32) * 16;
        }
        if (threadIdx.x == 0) SK_STAMP(p, i, 1);
        if (!work) { if (threadIdx.x == 0) SK_STAMP(p, i, 2); continue; }
        named_bar_sync(1, SK_CT);
        sk_mv_dispatch<HAS_Q4, HAS_Q6, HAS_Q8, TPX, WIDE>(p, d, S, r, xq_u, xf_u);
        if (threadIdx.x == 0) SK_STAMP(p, i, 2);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Packed bytes of a row chunk (Q6_K blocks padded to Q6P_BYTES).
static uint32_t sk_chunk_bytes(int type, uint32_t ck) {
    return type == T_Q6_K ? ck / 256 * Q6P_BYTES : (uint32_t)row_bytes(type, ck);
}
// Row slot stride: Q6_K rows 32 or 96 (mod 128) bytes apart, the others an
// odd number of 16-byte units: the lane patterns of mv_unit's loads then
// fall in distinct banks.
static uint32_t sk_rs(int type, uint32_t ck) {
    uint32_t rs = (sk_chunk_bytes(type, ck) + 15) & ~15u;
    if (type == T_Q6_K) {
        while (rs % 128 != 32 && rs % 128 != 96) rs += 16;
    } else if (((rs / 16) & 1u) == 0) {
        rs += 16;
    }
    return rs;
}

size_t step_sync_words(int n_sm) { return SK_SLOTS + 2 * (size_t)n_sm + 16; }

size_t step_attn_work_bytes(const StepParams &p) {
    return (size_t)p.nkh * SK_MAX_SPLITS * SK_GS * (4 + p.hd) * sizeof(float);
}

bool step_plan(StepParams &p, int n_sm, char *why, size_t cap) {
    auto no = [&](const char *m) {
        if (why && cap) snprintf(why, cap, "%s", m);
        return false;
    };
    const uint32_t qd = p.nqh * p.hd, kvd = p.nkh * p.hd;
    if (p.hd != 64 && p.hd != 128) return no("head_dim must be 64 or 128");
    if (!p.nkh || p.nqh % p.nkh || p.nqh / p.nkh > (uint32_t)SK_GS) return no("query heads per KV head must be 1..8");
    if (p.nkh > SK_MAX_KV || p.nkh > (uint32_t)n_sm) return no("too many KV heads");
    const int ts[5] = {p.t_qkv, p.t_o, p.t_gu, p.t_down, p.t_out};
    const uint32_t cols[5] = {p.dim, qd, p.dim, p.ffn, p.dim};
    const uint32_t rows[5] = {qd + 2 * kvd, p.dim, p.ffn, p.dim, p.vocab};
    for (int k = 0; k < 5; ++k) {
        if (ts[k] != T_Q4_K && ts[k] != T_Q6_K && ts[k] != T_Q8_0) return no("matvec weights must be Q4_K, Q6_K or Q8_0");
        if (cols[k] % (uint32_t)block_elems(ts[k]) || cols[k] % 32) return no("matrix width not a whole number of blocks");
    }
    if (!block_elems(p.t_embd) || p.dim % (uint32_t)block_elems(p.t_embd)) return no("embedding type");
    if (p.dim % 32 || qd % 32 || p.ffn % 32) return no("widths must be multiples of 32");
    if (p.dim > 16384) return no("model width above 16384");
    if (p.tp && p.dim > SK_PSTEP * 32) return no("tensor parallelism: model width above 4096");
    // shared memory: header | x | quantized x (or attention states) | ring.
    // The down projection quantizes only its CTA's (at most two) column
    // chunks; the chunk size is fixed first from a provisional ring.
    const uint32_t G = p.nqh / p.nkh;
    const uint32_t attn_sh = (uint32_t)(SK_NCW * G * (4 + p.hd) * 4 + 16 * (p.hd * 2 + 16) + 4 * p.hd);
    const uint32_t merge_sh = (uint32_t)(SK_GS * (SK_MAX_SPLITS + 1) * 4);
    auto plan_smem = [&](uint32_t down_ck) {
        const uint32_t nb = std::max(std::max(p.dim, qd), std::min(p.ffn, 2 * down_ck)) / 32;
        p.x_off = SK_HDR;
        p.xq_off = (p.x_off + p.dim * 4 + 1023) & ~1023u;
        p.xf_off = p.xq_off + nb * XQ_MAX_STRIDE;
        const uint32_t region = std::max(nb * (XQ_MAX_STRIDE + 16), std::max(attn_sh, merge_sh));
        p.ring_off = (p.xq_off + region + 1023) & ~1023u;
    };
    plan_smem(4096);
    if (p.ring_off >= SK_SMEM) return no("model width too large for shared memory");
    const uint32_t ring = SK_SMEM - p.ring_off;
    const uint32_t slot_max = (ring / 3) & ~127u;
    uint32_t slot = 2 * SK_AP * p.hd * 2;   // attention stage
    for (int k = 0; k < 5; ++k) {
        const uint32_t SL = 16u, E = (uint32_t)block_elems(ts[k]);
        uint32_t ck = cols[k];
        // whole rows when 16 fit a slot, else 4096- or 2048-column chunks
        // (16 or 8 super-blocks: the 8 consumer warps share them evenly),
        // else halve in 256-column steps
        if (SL * sk_rs(ts[k], ck) > slot_max)
            for (uint32_t c : {4096u, 2048u})
                if (ck > c && SL * sk_rs(ts[k], c) <= slot_max) { ck = c; break; }
        while (ck > 256 && SL * sk_rs(ts[k], ck) > slot_max) ck = std::max(256u, (ck / 2 + 255) / 256 * 256);
        if (ck % E) return no("chunk not a whole number of blocks");
        StepMvGeom &gg = p.geo[k];
        gg.ck = ck;
        gg.rs = sk_rs(ts[k], ck);
        gg.nch = (cols[k] + ck - 1) / ck;
        gg.ntiles = (rows[k] + (k == STEP_GU ? 7 : 15)) / (k == STEP_GU ? 8 : 16);   // gate/up: 8 rows of each
        slot = std::max(slot, SL * gg.rs);
        // row chunks across stages (sk_row_stages); the tensor-parallel
        // exchange addresses one plane per rank, so it takes whole rows only
        if (k != STEP_DOWN && gg.nch != 1 && p.tp) return no("rows of this width do not fit one stage");
        if (gg.ck > 4096) return no("stage chunks above 4096 columns");
    }
    {   // down: chunk-major units, every CTA within at most two chunks
        const StepMvGeom &gd = p.geo[STEP_DOWN];
        const uint64_t U = (uint64_t)gd.ntiles * gd.nch;
        if (gd.nch > (uint32_t)(p.tp ? SK_MAXPL : 4 * SK_MAXPL)) return no("too many column chunks in the down projection");
        if (p.tp && (uint64_t)gd.nch * p.dim > TP_DIM_MAX) return no("down partial planes exceed the exchange slots");
        if ((U + n_sm - 1) / n_sm > gd.ntiles) return no("down projection units per CTA exceed a chunk");
        plan_smem(gd.ck);
        if (SK_SMEM - p.ring_off < ring) return no("shared-memory plan");
    }
    slot = std::max(slot, p.dim * 4);   // the norm weight stage
    p.stage_max = slot;
    p.ring_bytes = ring & ~127u;
    if (p.ring_bytes < 2 * slot) return no("shared-memory ring too small");
    p.attn_splits = std::max(1u, std::min(SK_MAX_SPLITS, (uint32_t)n_sm / p.nkh));
    p.acc_layer = (uint64_t)(qd + 2 * kvd) + p.dim + p.ffn + (uint64_t)p.geo[STEP_DOWN].nch * p.dim;
    return true;
}

// One CTA per stage unit: slot row r of unit (tile, chunk) <- the chunk's
// bytes of row sk_slot_row(tile, r), zero-padded to rs; rows past the
// matrix are zeros.
__global__ void step_repack_kernel(int type, const uint8_t *w0, const uint8_t *w1, const uint8_t *w2, uint32_t seg0,
                                   uint32_t seg1, int gu, uint32_t rows, uint32_t cols, StepMvGeom g, uint8_t *dst) {
    const uint32_t unit = blockIdx.x, tile = unit / g.nch, ch = unit % g.nch;
    const uint32_t E = (uint32_t)block_elems(type), BB = (uint32_t)block_bytes(type);
    const uint64_t rb = row_bytes(type, cols);
    const uint32_t c0 = ch * g.ck, c1 = min(cols, c0 + g.ck);
    const uint64_t boff = (uint64_t)(c0 / E) * BB;
    const bool q6 = type == T_Q6_K;
    const uint32_t pb = q6 ? Q6P_BYTES : BB;                 // packed bytes per block
    const uint32_t blen = (c1 - c0) / E * pb;
    uint8_t *out = dst + (uint64_t)unit * 16 * g.rs;
    for (uint32_t i = threadIdx.x; i < 16 * g.rs; i += blockDim.x) {
        const uint32_t r = i / g.rs, b = i % g.rs;
        const uint32_t row = sk_slot_row(gu != 0, tile, r);
        uint8_t v = 0;
        if (row < rows && b < blen) {
            const uint8_t *src;
            if (gu) src = (r >= 8 ? w1 : w0) + (uint64_t)row * rb;
            else if (row < seg0) src = w0 + (uint64_t)row * rb;
            else if (row < seg1) src = w1 + (uint64_t)(row - seg0) * rb;
            else src = w2 + (uint64_t)(row - seg1) * rb;
            src += boff;
            if (q6) {   // GGUF Q6_K block (ql 0, qh 128, scales 192, d 208) -> the packed layout
                const uint32_t blk = b / Q6P_BYTES, o = b % Q6P_BYTES;
                const uint8_t *sb = src + (uint64_t)blk * 210;
                if (o < 128) v = sb[o];
                else if (o < 160) v = sb[128 + (o - 128)];
                else if (o < 176) v = sb[192 + (o - 160)];
                else if (o < 178) v = sb[208 + (o - 176)];
                else if (o >= 192) v = sb[160 + (o - 192)];
            } else {
                v = src[b];
            }
        }
        out[i] = v;
    }
}

static void sk_op_shape(const StepParams &p, int op, int &type, uint32_t &rows, uint32_t &cols) {
    const uint32_t qd = p.nqh * p.hd, kvd = p.nkh * p.hd;
    switch (op) {
        case STEP_QKV: type = p.t_qkv; rows = qd + 2 * kvd; cols = p.dim; break;
        case STEP_O: type = p.t_o; rows = p.dim; cols = qd; break;
        case STEP_GU: type = p.t_gu; rows = p.ffn; cols = p.dim; break;
        case STEP_DOWN: type = p.t_down; rows = p.dim; cols = p.ffn; break;
        default: type = p.t_out; rows = p.vocab; cols = p.dim; break;
    }
}

size_t step_packed_bytes(const StepParams &p, int op) {
    const StepMvGeom &g = p.geo[op];
    return (size_t)g.ntiles * g.nch * 16 * g.rs;
}

cudaError_t step_repack(const StepParams &p, int op, const uint8_t *w0, const uint8_t *w1, const uint8_t *w2,
                        uint8_t *dst, cudaStream_t st) {
    int type;
    uint32_t rows, cols;
    sk_op_shape(p, op, type, rows, cols);
    const uint32_t qd = p.nqh * p.hd, kvd = p.nkh * p.hd;
    const uint32_t seg0 = op == STEP_QKV ? qd : rows, seg1 = op == STEP_QKV ? qd + kvd : rows;
    const StepMvGeom &g = p.geo[op];
    note_launches(1);
    step_repack_kernel<<<g.ntiles * g.nch, 256, 0, st>>>(type, w0, w1, w2, seg0, seg1, op == STEP_GU, rows, cols, g, dst);
    return cudaGetLastError();
}

// The Llama-3-8B mix: Q4_K attention and gate/up, Q6_K down and output, head_dim 128.
static bool sk_is_8b_mix(const StepParams &p) {
    return p.hd == 128 && p.t_qkv == T_Q4_K && p.t_o == T_Q4_K && p.t_gu == T_Q4_K && p.t_down == T_Q6_K &&
           p.t_out == T_Q6_K;
}
static bool sk_is_q4k_only(const StepParams &p) {
    return p.hd == 128 && p.t_qkv == T_Q4_K && p.t_o == T_Q4_K && p.t_gu == T_Q4_K && p.t_down == T_Q4_K &&
           p.t_out == T_Q4_K;
}
// Models whose norm prologue takes more than one pass, or with rows (other
// than the down projection's) spread over several stages: the WIDE instances.
static bool sk_is_wide(const StepParams &p) {
    if (p.dim > SK_PSTEP * 32) return true;
    for (int k = 0; k < 5; ++k)
        if (k != STEP_DOWN && p.geo[k].nch > 1) return true;
    return false;
}

template <int HD, bool A, bool B, bool C, bool T, bool W> static cudaError_t sk_attr() {
    return cudaFuncSetAttribute(step_kernel<HD, A, B, C, T, W>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM);
}

cudaError_t step_configure() {
    const cudaError_t es[] = {sk_attr<0, true, true, true, false, false>(), sk_attr<128, true, true, false, false, false>(),
                              sk_attr<128, true, false, false, false, false>(), sk_attr<0, true, true, true, true, false>(),
                              sk_attr<128, true, true, false, true, false>(), sk_attr<0, true, true, true, false, true>(),
                              sk_attr<128, true, false, false, false, true>()};
    for (cudaError_t e : es)
        if (e != cudaSuccess) return e;
    return cudaSuccess;
}

cudaError_t step_launch(const StepParams &p, int n_sm, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_sm);
    cfg.blockDim = dim3(SK_THREADS);
    cfg.dynamicSmemBytes = SK_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs co-resident: the grid barrier relies on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launches(1);
    // tensor-parallel instances carry the exchange code; the one-GPU ones do
    // not. Models wider than 4096 have instances of their own (row chunks,
    // prologue passes), so the others carry none of that code.
    if (p.tp) {
        if (sk_is_8b_mix(p)) return cudaLaunchKernelEx(&cfg, step_kernel<128, true, true, false, true, false>, p);
        return cudaLaunchKernelEx(&cfg, step_kernel<0, true, true, true, true, false>, p);
    }
    if (sk_is_wide(p)) {
        if (sk_is_q4k_only(p)) return cudaLaunchKernelEx(&cfg, step_kernel<128, true, false, false, false, true>, p);
        return cudaLaunchKernelEx(&cfg, step_kernel<0, true, true, true, false, true>, p);
    }
    if (sk_is_8b_mix(p)) return cudaLaunchKernelEx(&cfg, step_kernel<128, true, true, false, false, false>, p);
    if (sk_is_q4k_only(p)) return cudaLaunchKernelEx(&cfg, step_kernel<128, true, false, false, false, false>, p);
    return cudaLaunchKernelEx(&cfg, step_kernel<0, true, true, true, false, false>, p);
}

}  // namespace vbs
