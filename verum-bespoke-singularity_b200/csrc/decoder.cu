// decoder.cu -- the per-token decode step as one device program.
//
// The reference JIT emits forward_token() as ~16 host calls per layer
// through the bridge (src/vbs_specializer.c:270-349) and reads all logits
// back after every call (:351-359). Here the same step, in the same op
// order, is a short chain of fused kernels recorded once into a CUDA graph
// and replayed per token; the position and the token live in a device
// control block (ctrl[0] = position, ctrl[1] = token), so consecutive steps
// need no host work: the argmax at the end of a step writes the next token
// and advances the position.
//
// Fast step, per layer (5 kernels, programmatic dependent launch between
// them so each kernel's weight stream starts while the previous one ends):
//   1. RMSNorm(attn_norm) + Q/K/V matvec + RoPE + fp16 KV store
//   2. split-KV GQA attention
//   3. o_proj matvec + residual add
//   4. RMSNorm(ffn_norm) + gate/up matvec + SiLU*up
//   5. down matvec + residual add
// then RMSNorm(output_norm) + output matvec, and the argmax.
//
// Strict step (VBS_CU_DEC_STRICT): the vbs_cpu arithmetic
// (src/vbs_cpu.c:572-639) op by op, fp32 KV cache, for token-exact parity.
//
// Tensor parallelism: o_proj and down produce partial sums that are
// all-reduced (NCCL) and added into the residual by the next kernel's
// prologue; the output rows are sharded and all-gathered before the argmax.
#include "vbs_b200.h"
#include "backend.h"
#include "common.cuh"
#include "kernels.h"
#include "tp.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace vbs;

namespace {

struct Layer {
    const float *attn_norm, *ffn_norm;
    const uint8_t *wq, *wk, *wv, *wo, *wgate, *wup, *wdown;
    int tq, tk, tv, to, tgate, tup, tdown;
};

}  // namespace

constexpr uint32_t kDecoderMagic = 0x56424443u;   // "VBDC": a live vbs_cu_decoder

struct vbs_cu_decoder {
    uint32_t magic = kDecoderMagic;
    vbs_cu_model_t m;
    std::vector<Layer> L;
    uint32_t flags = 0, max_ctx = 0, kv_dim = 0, q_dim = 0, vocab_full = 0;
    bool strict = false, use_graph = true, use_pdl = true;
    int tp_world = 1;
    bool tp_p2p = false;   // per-layer sums over peer memory (else NCCL all-reduce)
    DevState *dev = nullptr;
    cudaStream_t st = nullptr;
    // activations
    float *x = nullptr, *x2 = nullptr, *q = nullptr, *att = nullptr, *hid = nullptr, *logits = nullptr,
          *logits_full = nullptr, *partial = nullptr;
    float *norm = nullptr, *k = nullptr, *v = nullptr, *gate = nullptr, *up = nullptr, *tmp = nullptr, *scores = nullptr;
    int8_t *xq = nullptr;
    float *qd = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;
    float *kcf = nullptr, *vcf = nullptr;
    uint32_t *ctrl = nullptr, *hist = nullptr, *tok_dev = nullptr;
    size_t tok_cap = 0;
    uint32_t *pinned = nullptr;      // [0..1] ctrl readback
    float *logits_pinned = nullptr;
    void *attn_work = nullptr;
    void *argmax_work = nullptr;
    // persistent step kernel (one cooperative launch per token)
    bool persist = false;
    StepParams sp = {};
    StepLayer *step_layers = nullptr;
    uint8_t *step_packed = nullptr;   // weights repacked into stage units
    float *step_acc = nullptr;        // accumulation buffers, then the sync words
    size_t step_acc_bytes = 0;
    void *step_attn = nullptr;
    void *words_mem = nullptr;        // one GPU, VBS_CU_DEC_WORDS: the local exchange-word area
    TpComm *words_comm = nullptr;
    uint32_t n_splits = 1;
    // prompt chunks (vbs_cu_decoder_prefill), allocated on first use
    float *pf_x = nullptr, *pf_xn = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_att = nullptr,
          *pf_g = nullptr, *pf_u = nullptr, *pf_h = nullptr;
    void *pf_attn_work = nullptr;
    __half *pf_x16 = nullptr;   // a prompt chunk's normed rows as GEMM activations (fp16, tile layout)
    uint32_t pf_splits = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint32_t kernels_per_step = 0;
    uint64_t host_pos = 0;           // host shadow of ctrl[0] (steps enqueued since the last reset)
    // slice streaming (VBS_CU_DEC_STREAM): the layers' matrices stay in
    // pinned host memory (L[l] holds host pointers); each layer is copied
    // into one of two device slots on its own stream, layer g + 1's copy
    // overlapping layer g's kernels
    bool stream = false;
    cudaStream_t cst = nullptr;              // copy stream
    uint8_t *slot[2] = {nullptr, nullptr};
    cudaEvent_t copied[2] = {nullptr, nullptr}, done[2] = {nullptr, nullptr};
    size_t off[7] = {}, slot_bytes = 0;      // per matrix (q k v o gate up down): offset in a slot
    uint64_t layers_queued = 0;              // layers whose copy has been enqueued
    uint64_t layers_run = 0;                 // layers whose kernels have been enqueued
    unsigned long long *trace = nullptr;   // step timeline of a VBS_STEP_TRACE profiling build
};

namespace {

// Makes the decoder's device current for one entry point and puts the
// caller's current device back on every return path (a host thread may
// drive several devices, e.g. tensor-parallel ranks).
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int ordinal) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != ordinal) cudaSetDevice(ordinal);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

bool dmalloc(void **p, size_t bytes, const char *what) {
    return cuda_ok(cudaMalloc(p, bytes ? bytes : 16), what);
}

bool plan_persistent(vbs_cu_decoder *d);

// Launch one matvec y (+)= W x through the fastest kernel that supports it.
bool step_matvec(vbs_cu_decoder *d, int type, const uint8_t *w, const float *x, float *y, uint32_t rows, uint32_t cols,
                 bool accumulate, const float *norm_w, const float *x_add, float *x_write, bool tp_write = false,
                 bool tp_read = false) {
    const void *wv[1] = {w};
    if (mv_fast_supported(type, rows, cols, wv, 1, x, 0)) {
        MvParams p = {};
        p.w[0] = p.w[1] = p.w[2] = w;
        p.seg_end[0] = p.seg_end[1] = p.seg_end[2] = rows;
        p.rb = row_bytes(type, cols);
        p.rows = rows;
        p.cols = cols;
        p.x = x;
        p.norm_w = norm_w;
        p.eps = d->m.eps;
        p.x_add = x_add;
        p.x_write = x_write;
        p.y = y;
        p.accumulate = accumulate ? 1u : 0u;
        p.err = d->dev->err;
        p.tp = (tp_write || tp_read) ? tp_comm() : nullptr;
        p.tp_write = tp_write;
        p.tp_read = tp_read;
        return cuda_ok(mv_fast_launch(type, 0, MV_EPI_STORE, p, d->dev->n_sm, d->st, d->use_pdl, 0), "decode matvec");
    }
    if (tp_write || tp_read) {
        latch_error("decode matvec: peer-memory exchange needs the fast kernel");
        return false;
    }
    // portable path: explicit norm into d->norm when requested
    const float *xin = x;
    if (x_add) {
        if (!cuda_ok(add_launch(x, x_add, x_write, cols, d->st), "decode residual")) return false;
        xin = x_write;
    }
    if (norm_w) {
        if (!cuda_ok(rmsnorm_launch(xin, norm_w, d->norm, cols, d->m.eps, d->st), "decode norm")) return false;
        xin = d->norm;
    }
    return cuda_ok(mv_generic_launch(type, w, xin, y, rows, cols, 1, cols, rows, accumulate ? 1 : 0, d->dev->n_sm, d->st),
                   "decode matvec");
}

// Bytes of layer matrix k (q k v o gate up down) of a streamed model.
size_t stream_matrix_bytes(const vbs_cu_decoder *d, const Layer &y, int k) {
    const vbs_cu_model_t &m = d->m;
    const uint32_t qd = d->q_dim, kvd = d->kv_dim;
    switch (k) {
        case 0: return row_bytes(y.tq, m.dim) * qd;
        case 1: return row_bytes(y.tk, m.dim) * kvd;
        case 2: return row_bytes(y.tv, m.dim) * kvd;
        case 3: return row_bytes(y.to, qd) * m.dim;
        case 4: return row_bytes(y.tgate, m.dim) * m.ffn;
        case 5: return row_bytes(y.tup, m.dim) * m.ffn;
        default: return row_bytes(y.tdown, m.ffn) * m.dim;
    }
}

// Enqueues the copy of the next layer (in step order, wrapping to layer 0)
// into its slot on the copy stream, after the kernels that last read that
// slot: one cudaMemcpyAsync per matrix, then the slot's `copied` event.
bool stream_queue_copy(vbs_cu_decoder *d) {
    const uint64_t g = d->layers_queued;
    const int sl = (int)(g & 1u);
    const Layer &y = d->L[g % d->m.n_layers];
    if (g >= 2 && !cuda_ok(cudaStreamWaitEvent(d->cst, d->done[sl], 0), "stream: slot free")) return false;
    const uint8_t *src[7] = {y.wq, y.wk, y.wv, y.wo, y.wgate, y.wup, y.wdown};
    for (int k = 0; k < 7; ++k)
        if (!cuda_ok(cudaMemcpyAsync(d->slot[sl] + d->off[k], src[k], stream_matrix_bytes(d, y, k), cudaMemcpyHostToDevice,
                                     d->cst), "stream: layer copy"))
            return false;
    if (!cuda_ok(cudaEventRecord(d->copied[sl], d->cst), "stream: copied")) return false;
    d->layers_queued = g + 1;
    return true;
}

// The device view of layer l for the next layer of kernels: waits (on the
// compute stream) for its copy and queues the copy of the layer after it.
bool stream_layer(vbs_cu_decoder *d, uint32_t l, Layer &out) {
    const uint64_t g = d->layers_run;
    const int sl = (int)(g & 1u);
    if (d->layers_queued <= g && !stream_queue_copy(d)) return false;
    if (!cuda_ok(cudaStreamWaitEvent(d->st, d->copied[sl], 0), "stream: wait copy")) return false;
    out = d->L[l];
    uint8_t *b = d->slot[sl];
    out.wq = b + d->off[0]; out.wk = b + d->off[1]; out.wv = b + d->off[2]; out.wo = b + d->off[3];
    out.wgate = b + d->off[4]; out.wup = b + d->off[5]; out.wdown = b + d->off[6];
    return true;
}

// After layer l's kernels: the slot is free once they finish; the next
// layer's copy goes out now, overlapping them.
bool stream_layer_done(vbs_cu_decoder *d) {
    const int sl = (int)(d->layers_run & 1u);
    if (!cuda_ok(cudaEventRecord(d->done[sl], d->st), "stream: done")) return false;
    d->layers_run++;
    return d->layers_queued > d->layers_run || stream_queue_copy(d);
}

bool enqueue_persistent_step(vbs_cu_decoder *d) {
    // every activation is written once per step; only the barrier and ticket words start at zero
    const size_t sync_bytes = step_sync_words(d->dev->n_sm) * 4;
    if (!cuda_ok(cudaMemsetAsync(d->sp.sync, 0, sync_bytes, d->st), "step sync words")) return false;
    return cuda_ok(step_launch(d->sp, d->dev->n_sm, d->st), "decode step kernel");
}

bool enqueue_fast_step(vbs_cu_decoder *d) {
    if (d->persist) return enqueue_persistent_step(d);
    const vbs_cu_model_t &m = d->m;
    const uint32_t dim = m.dim, hd = m.head_dim, nq = m.n_heads * hd, nk = d->kv_dim;
    cudaStream_t st = d->st;
    const bool tp = d->tp_world > 1;
    // residual ping-pong (TP): xr is the residual read by this kernel's
    // prologue, xw where the summed residual is written
    float *xr = d->x, *xw = d->x2;

    if (!cuda_ok(embed_launch(m.embd_type, static_cast<const uint8_t *>(m.embd), d->ctrl + 1, 0, d->vocab_full, d->x, dim, d->dev->err, st, d->use_pdl),
                 "decode embed"))
        return false;
    const float *pending = nullptr;   // TP over NCCL: partial sum to add into the residual
    bool pending_tp = false;          // TP over peer memory: the exchange to add into the residual
    for (uint32_t l = 0; l < m.n_layers; ++l) {
        Layer streamed;
        if (d->stream && !stream_layer(d, l, streamed)) return false;
        const Layer &ly = d->stream ? streamed : d->L[l];
        // ---- 1. norm + QKV + RoPE + KV store ----
        const void *wv[3] = {ly.wq, ly.wk, ly.wv};
        const bool fused = ly.tq == ly.tk && ly.tq == ly.tv && mv_fast_supported(ly.tq, nq + 2 * nk, dim, wv, 3, xr, 0);
        if (fused) {
            MvParams p = {};
            p.w[0] = ly.wq; p.w[1] = ly.wk; p.w[2] = ly.wv;
            p.seg_end[0] = nq; p.seg_end[1] = nq + nk; p.seg_end[2] = nq + 2 * nk;
            p.rb = row_bytes(ly.tq, dim);
            p.rows = nq + 2 * nk;
            p.cols = dim;
            p.x = xr;
            p.norm_w = ly.attn_norm;
            p.eps = m.eps;
            p.x_add = pending;
            p.x_write = (pending || pending_tp) ? xw : nullptr;
            p.tp = pending_tp ? tp_comm() : nullptr;
            p.tp_read = pending_tp;
            p.err = d->dev->err;
            p.q_out = d->q;
            p.kc = d->kc; p.vc = d->vc;
            p.ctrl = d->ctrl;
            p.layer = l; p.max_ctx = d->max_ctx; p.kv_dim = nk; p.head_dim = hd;
            p.kv_head_major = 1;
            p.theta = m.theta;
            if (!cuda_ok(mv_fast_launch(ly.tq, 0, MV_EPI_QKV, p, d->dev->n_sm, st, d->use_pdl, 0), "decode qkv")) return false;
        } else {
            if (!step_matvec(d, ly.tq, ly.wq, xr, d->q, nq, dim, false, ly.attn_norm, pending,
                             (pending || pending_tp) ? xw : nullptr, false, pending_tp))
                return false;
            const float *xin = (pending || pending_tp) ? xw : xr;
            if (!step_matvec(d, ly.tk, ly.wk, xin, d->k, nk, dim, false, ly.attn_norm, nullptr, nullptr)) return false;
            if (!step_matvec(d, ly.tv, ly.wv, xin, d->v, nk, dim, false, ly.attn_norm, nullptr, nullptr)) return false;
            if (!cuda_ok(rope_launch(d->q, 0, d->ctrl, hd, m.n_heads, m.theta, st), "decode rope")) return false;
            if (!cuda_ok(rope_launch(d->k, 0, d->ctrl, hd, m.n_kv_heads, m.theta, st), "decode rope")) return false;
            if (!cuda_ok(cache_store_launch(d->k, d->v, d->kc, d->vc, 0, d->ctrl, l, d->max_ctx, nk, hd, true, st), "decode kv store"))
                return false;
        }
        if (pending || pending_tp) { std::swap(xr, xw); pending = nullptr; pending_tp = false; }
        // ---- 2. attention ----
        AttnParams ap = {};
        ap.q = d->q; ap.kc = d->kc; ap.vc = d->vc; ap.out = d->att;
        ap.seq_dev = d->ctrl;
        ap.layer = l; ap.max_ctx = d->max_ctx;
        ap.nqh = m.n_heads; ap.nkh = m.n_kv_heads; ap.hd = hd;
        ap.scale = 1.0f / sqrtf((float)hd);
        ap.batch = 1;
        ap.head_major = 1;
        ap.work = d->attn_work;
        ap.err = d->dev->err;
        if (!cuda_ok(attn_launch(ap, d->n_splits, st, d->use_pdl), "decode attention")) return false;
        // ---- 3. o_proj (+ residual, or partial under TP) ----
        if (tp && d->tp_p2p) {
            if (!step_matvec(d, ly.to, ly.wo, d->att, d->partial, dim, nq, false, nullptr, nullptr, nullptr, true)) return false;
            pending_tp = true;
        } else if (tp) {
            if (!step_matvec(d, ly.to, ly.wo, d->att, d->partial, dim, nq, false, nullptr, nullptr, nullptr)) return false;
            if (!tp_allreduce_sum(d->partial, dim, st)) return false;
            pending = d->partial;
        } else {
            if (!step_matvec(d, ly.to, ly.wo, d->att, xr, dim, nq, true, nullptr, nullptr, nullptr)) return false;
        }
        // ---- 4. norm + gate/up + SiLU ----
        const void *wg[2] = {ly.wgate, ly.wup};
        const bool dual = ly.tgate == ly.tup && mv_fast_supported(ly.tgate, m.ffn, dim, wg, 2, xr, 1);
        if (dual) {
            MvParams p = {};
            p.w[0] = p.w[1] = p.w[2] = ly.wgate;
            p.seg_end[0] = p.seg_end[1] = p.seg_end[2] = m.ffn;
            p.wb = ly.wup;
            p.rb = row_bytes(ly.tgate, dim);
            p.rows = m.ffn;
            p.cols = dim;
            p.x = xr;
            p.norm_w = ly.ffn_norm;
            p.eps = m.eps;
            p.x_add = pending;
            p.x_write = (pending || pending_tp) ? xw : nullptr;
            p.tp = pending_tp ? tp_comm() : nullptr;
            p.tp_read = pending_tp;
            p.y = d->hid;
            p.err = d->dev->err;
            if (!cuda_ok(mv_fast_launch(ly.tgate, 1, MV_EPI_SILU, p, d->dev->n_sm, st, d->use_pdl, 0), "decode gate/up")) return false;
        } else {
            if (!step_matvec(d, ly.tgate, ly.wgate, xr, d->gate, m.ffn, dim, false, ly.ffn_norm, pending,
                             (pending || pending_tp) ? xw : nullptr, false, pending_tp))
                return false;
            const float *xin = (pending || pending_tp) ? xw : xr;
            if (!step_matvec(d, ly.tup, ly.wup, xin, d->up, m.ffn, dim, false, ly.ffn_norm, nullptr, nullptr)) return false;
            if (!cuda_ok(silu_mul_launch(d->gate, d->up, d->hid, m.ffn, st), "decode silu")) return false;
        }
        if (pending || pending_tp) { std::swap(xr, xw); pending = nullptr; pending_tp = false; }
        // ---- 5. down (+ residual, or partial under TP) ----
        if (tp && d->tp_p2p) {
            if (!step_matvec(d, ly.tdown, ly.wdown, d->hid, d->partial, dim, m.ffn, false, nullptr, nullptr, nullptr, true))
                return false;
            pending_tp = true;
        } else if (tp) {
            if (!step_matvec(d, ly.tdown, ly.wdown, d->hid, d->partial, dim, m.ffn, false, nullptr, nullptr, nullptr)) return false;
            if (!tp_allreduce_sum(d->partial, dim, st)) return false;
            pending = d->partial;
        } else {
            if (!step_matvec(d, ly.tdown, ly.wdown, d->hid, xr, dim, m.ffn, true, nullptr, nullptr, nullptr)) return false;
        }
        if (d->stream && !stream_layer_done(d)) return false;
    }
    // ---- final norm + output ----
    if (!step_matvec(d, m.out_type, static_cast<const uint8_t *>(m.out), xr, d->logits, m.vocab, dim, false, m.out_norm,
                     pending, (pending || pending_tp) ? xw : nullptr, false, pending_tp))
        return false;
    if (pending || pending_tp) std::swap(xr, xw);
    const float *lg = d->logits;
    if (tp) {
        if (!tp_allgather(d->logits, d->logits_full, m.vocab, st)) return false;
        lg = d->logits_full;
    }
    // the embedding of the next step writes d->x: the residual must end in d->x
    (void)xr;
    return cuda_ok(argmax_launch(lg, d->vocab_full, nullptr, d->ctrl, d->hist, (uint32_t)d->max_ctx + 1, d->argmax_work, st,
                                 d->use_pdl),
                   "decode argmax");
}

bool enqueue_strict_step(vbs_cu_decoder *d) {
    const vbs_cu_model_t &m = d->m;
    const uint32_t dim = m.dim, hd = m.head_dim, nq = m.n_heads * hd, nk = d->kv_dim;
    cudaStream_t st = d->st;
    auto mat = [&](int type, const uint8_t *w, const float *x, float *y, uint32_t rows, uint32_t cols, bool quantized) -> bool {
        if (type == T_F32) return cuda_ok(strict_matvec_f32_launch(reinterpret_cast<const float *>(w), rows, cols, x, y, 0, st), "strict matvec");
        if (type != T_Q8_0) { latch_error("strict mode supports Q8_0 and F32 weights only (type %d)", type); return false; }
        if (!quantized && !cuda_ok(strict_quantize_q8_launch(x, cols, d->xq, d->qd, st), "strict quantize")) return false;
        return cuda_ok(strict_matvec_q8_0_launch(w, rows, cols, d->xq, d->qd, y, 0, st), "strict matvec");
    };
    if (!cuda_ok(embed_launch(m.embd_type, static_cast<const uint8_t *>(m.embd), d->ctrl + 1, 0, d->vocab_full, d->x, dim, d->dev->err, st, false), "strict embed"))
        return false;
    for (uint32_t l = 0; l < m.n_layers; ++l) {
        const Layer &ly = d->L[l];
        if (!cuda_ok(strict_rmsnorm_launch(d->x, ly.attn_norm, d->norm, dim, m.eps, st), "strict norm")) return false;
        if (!mat(ly.tq, ly.wq, d->norm, d->q, nq, dim, false)) return false;
        const bool shared_q8 = ly.tq == T_Q8_0;
        if (!mat(ly.tk, ly.wk, d->norm, d->k, nk, dim, shared_q8 && ly.tk == T_Q8_0)) return false;
        if (!mat(ly.tv, ly.wv, d->norm, d->v, nk, dim, shared_q8 && ly.tk == T_Q8_0 && ly.tv == T_Q8_0)) return false;
        if (!cuda_ok(strict_rope_launch(d->q, m.n_heads, hd, d->ctrl, m.theta, st), "strict rope")) return false;
        if (!cuda_ok(strict_rope_launch(d->k, m.n_kv_heads, hd, d->ctrl, m.theta, st), "strict rope")) return false;
        if (!cuda_ok(strict_attention_launch(d->q, d->k, d->v, d->kcf, d->vcf, d->att, d->ctrl, l, d->max_ctx, m.n_heads,
                                             m.n_kv_heads, hd, d->scores, d->dev->err, st),
                     "strict attention"))
            return false;
        if (!mat(ly.to, ly.wo, d->att, d->tmp, dim, nq, false)) return false;
        if (!cuda_ok(strict_add_launch(d->x, d->tmp, dim, st), "strict add")) return false;
        if (!cuda_ok(strict_rmsnorm_launch(d->x, ly.ffn_norm, d->norm, dim, m.eps, st), "strict norm")) return false;
        if (!mat(ly.tgate, ly.wgate, d->norm, d->gate, m.ffn, dim, false)) return false;
        if (!mat(ly.tup, ly.wup, d->norm, d->up, m.ffn, dim, ly.tgate == T_Q8_0 && ly.tup == T_Q8_0)) return false;
        if (!cuda_ok(strict_silu_launch(d->gate, d->up, d->hid, m.ffn, st), "strict silu")) return false;
        if (!mat(ly.tdown, ly.wdown, d->hid, d->tmp, dim, m.ffn, false)) return false;
        if (!cuda_ok(strict_add_launch(d->x, d->tmp, dim, st), "strict add")) return false;
    }
    if (!cuda_ok(strict_rmsnorm_launch(d->x, m.out_norm, d->norm, dim, m.eps, st), "strict norm")) return false;
    if (!mat(m.out_type, static_cast<const uint8_t *>(m.out), d->norm, d->logits, m.vocab, dim, false)) return false;
    return cuda_ok(argmax_launch(d->logits, m.vocab, nullptr, d->ctrl, d->hist, (uint32_t)d->max_ctx + 1, d->argmax_work, st,
                                 false), "strict argmax");
}

bool enqueue_step_raw(vbs_cu_decoder *d) { return d->strict ? enqueue_strict_step(d) : enqueue_fast_step(d); }

// One step: graph replay when available, else direct launches.
bool enqueue_step(vbs_cu_decoder *d) {
    if (d->host_pos >= d->max_ctx) {
        latch_error("decode step at position %llu exceeds the KV capacity %u", (unsigned long long)d->host_pos, d->max_ctx);
        return false;
    }
    d->host_pos++;
    if (d->exec) {
        note_launches(d->kernels_per_step);
        return cuda_ok(cudaGraphLaunch(d->exec, d->st), "decode graph launch");
    }
    return enqueue_step_raw(d);
}

bool build_graph(vbs_cu_decoder *d) {
    const uint64_t before = vbs_cu_kernel_launches();
    if (!cuda_ok(cudaStreamBeginCapture(d->st, cudaStreamCaptureModeThreadLocal), "graph capture")) return false;
    const bool ok = enqueue_step_raw(d);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(d->st, &g);
    if (!ok || !cuda_ok(e, "graph capture")) {
        if (g) cudaGraphDestroy(g);
        return false;
    }
    d->kernels_per_step = (uint32_t)(vbs_cu_kernel_launches() - before);
    d->graph = g;
    return cuda_ok(cudaGraphInstantiate(&d->exec, g, 0), "graph instantiate");
}

bool sync_and_check(vbs_cu_decoder *d) {
    if (!cuda_ok(cudaStreamSynchronize(d->st), "decode synchronise")) return false;
    return check_device_error(d->dev, d->st);
}

bool put_tokens(vbs_cu_decoder *d, const uint32_t *tokens, size_t n) {
    if (n > d->tok_cap) {
        if (d->tok_dev) cudaFree(d->tok_dev);
        d->tok_dev = nullptr;
        d->tok_cap = 0;
        if (!dmalloc(reinterpret_cast<void **>(&d->tok_dev), n * 4, "token buffer")) return false;
        d->tok_cap = n;
    }
    return cuda_ok(cudaMemcpyAsync(d->tok_dev, tokens, n * 4, cudaMemcpyHostToDevice, d->st), "token upload");
}

// Chooses the persistent step kernel when the model fits its plan (uniform
// per-op weight types, head_dim 64/128, one GPU); otherwise the per-op
// kernels stay in use. Returns false only on an allocation failure.
bool plan_persistent(vbs_cu_decoder *d) {
    const vbs_cu_model_t &m = d->m;
    const Layer &y0 = d->L[0];
    auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    for (const Layer &y : d->L)
        if (y.tq != y0.tq || y.tk != y0.tq || y.tv != y0.tq || y.to != y0.to || y.tgate != y0.tgate ||
            y.tup != y0.tgate || y.tdown != y0.tdown || !a16(y.attn_norm) || !a16(y.ffn_norm))
            return true;   // norm weights are bulk-copied: 16-byte aligned
    if (!a16(m.out_norm)) return true;
    StepParams &p = d->sp;
    p = StepParams{};
    p.n_layers = m.n_layers; p.dim = m.dim; p.nqh = m.n_heads; p.nkh = m.n_kv_heads; p.hd = m.head_dim;
    p.ffn = m.ffn; p.vocab = m.vocab; p.max_ctx = d->max_ctx;
    p.eps = m.eps; p.theta = m.theta; p.scale = 1.0f / sqrtf((float)m.head_dim);
    p.wait_ns = kWaitNs;
    p.drop_op = ~0u;
    p.t_embd = m.embd_type; p.t_qkv = y0.tq; p.t_o = y0.to; p.t_gu = y0.tgate; p.t_down = y0.tdown; p.t_out = m.out_type;
    p.embd = static_cast<const uint8_t *>(m.embd);
    p.out_norm = m.out_norm;
    if (d->tp_world > 1) {   // the step's exchanges go over peer memory; the logits gather into the region
        if (!d->tp_p2p || !tp_own_logits() || d->vocab_full > TP_VOCAB_MAX || m.dim > TP_DIM_MAX) return true;
        p.tp = tp_comm();
        p.tp_world = (uint32_t)d->tp_world;
        p.tp_rank = (uint32_t)tp_rank();
        p.vocab_full = d->vocab_full;
    } else if ((d->flags & VBS_CU_DEC_WORDS) && m.dim <= TP_DIM_MAX && m.vocab <= TP_VOCAB_MAX) {
        // one GPU on request: the tensor-parallel instance (exchange words,
        // no grid barrier after o_proj and down) over a local area
        if (!tp_local_area(d->logits, &d->words_mem, &d->words_comm)) return false;
        p.tp = d->words_comm;
        p.tp_world = 1;
        p.tp_rank = 0;
        p.vocab_full = m.vocab;
    }
    char why[160];
    if (!step_plan(p, d->dev->n_sm, why, sizeof why)) {
        if (d->tp_world > 1 || !p.tp) return true;
        p.tp = nullptr;   // the plain one-GPU instance
        if (!step_plan(p, d->dev->n_sm, why, sizeof why)) return true;
    }
    // repacked weights: per layer QKV | O | GU | DOWN, then the output matrix
    const size_t bq = step_packed_bytes(p, STEP_QKV), bo = step_packed_bytes(p, STEP_O),
                 bg = step_packed_bytes(p, STEP_GU), bd = step_packed_bytes(p, STEP_DOWN),
                 bout = step_packed_bytes(p, STEP_OUT);
    const size_t per_layer = bq + bo + bg + bd;
    {   // the repacked copy sits beside the GGUF weights (the per-op and
        // prefill kernels read those): without room for both plus 1 GiB of
        // headroom the per-op path stays in use
        size_t free_b = 0, total_b = 0;
        if (!cuda_ok(cudaMemGetInfo(&free_b, &total_b), "memory info")) return false;
        if (per_layer * m.n_layers + bout + (1ull << 30) > free_b) return true;
    }
    if (!dmalloc((void **)&d->step_packed, per_layer * m.n_layers + bout, "repacked weights")) return false;
    std::vector<StepLayer> hl(m.n_layers);
    for (uint32_t l = 0; l < m.n_layers; ++l) {
        const Layer &y = d->L[l];
        uint8_t *base = d->step_packed + per_layer * l;
        hl[l] = StepLayer{base, base + bq, base + bq + bo, base + bq + bo + bg, y.attn_norm, y.ffn_norm};
        if (!cuda_ok(step_repack(p, STEP_QKV, y.wq, y.wk, y.wv, base, d->st), "repack") ||
            !cuda_ok(step_repack(p, STEP_O, y.wo, nullptr, nullptr, base + bq, d->st), "repack") ||
            !cuda_ok(step_repack(p, STEP_GU, y.wgate, y.wup, nullptr, base + bq + bo, d->st), "repack") ||
            !cuda_ok(step_repack(p, STEP_DOWN, y.wdown, nullptr, nullptr, base + bq + bo + bg, d->st), "repack"))
            return false;
    }
    uint8_t *pout = d->step_packed + per_layer * m.n_layers;
    if (!cuda_ok(step_repack(p, STEP_OUT, static_cast<const uint8_t *>(m.out), nullptr, nullptr, pout, d->st), "repack"))
        return false;
    p.out = pout;
    const size_t acc_floats = (size_t)p.n_layers * p.acc_layer;
    const size_t sync_words = step_sync_words(d->dev->n_sm);
    d->step_acc_bytes = acc_floats * 4 + sync_words * 4;
    const size_t aw = step_attn_work_bytes(p);
    if (!dmalloc((void **)&d->step_layers, hl.size() * sizeof(StepLayer), "step layers") ||
        !dmalloc((void **)&d->step_acc, d->step_acc_bytes, "step buffers") || !dmalloc(&d->step_attn, aw, "step attention"))
        return false;
    if (!cuda_ok(cudaMemcpy(d->step_layers, hl.data(), hl.size() * sizeof(StepLayer), cudaMemcpyHostToDevice), "step layers") ||
        !cuda_ok(cudaMemset(d->step_attn, 0, aw), "step attention") ||
        !cuda_ok(cudaMemset(d->step_acc, 0, d->step_acc_bytes), "step buffers"))
        return false;
    p.layers = d->step_layers;
    p.kc = d->kc; p.vc = d->vc;
    p.acc = d->step_acc;
    p.logits = d->logits;
    p.att = d->att;
    p.attn_work = d->step_attn;
    p.sync = reinterpret_cast<uint32_t *>(d->step_acc + acc_floats);
    p.ctrl = d->ctrl; p.hist = d->hist; p.hist_cap = d->max_ctx + 1;
    p.err = d->dev->err;
#ifdef VBS_STEP_TRACE
    if (!dmalloc((void **)&d->trace, (size_t)d->dev->n_sm * (5 * p.n_layers + 2) * SK_TR_SLOTS * 8, "step trace") ||
        !cuda_ok(cudaMemset(d->trace, 0, (size_t)d->dev->n_sm * (5 * p.n_layers + 2) * SK_TR_SLOTS * 8), "step trace"))
        return false;
    p.trace = d->trace;
#endif
    d->persist = true;
    return true;
}

// ---------------------------------------------------------------------------
// prompt chunks: up to PF_CHUNK tokens share one pass over the weights
// ---------------------------------------------------------------------------
// Chunks of up to 512 tokens (one GEMM tile of tokens): the matrices go
// through the tcgen05 GEMM (above 8 tokens) or the batched matvec (the
// last, short chunk).
constexpr uint32_t PF_CHUNK = 512;

bool prefill_buffers(vbs_cu_decoder *d) {
    if (d->pf_x) return true;
    const vbs_cu_model_t &m = d->m;
    const size_t B = PF_CHUNK;
    // the most splits any chunk takes (fewer for larger batches), and the
    // largest split workspace over the chunk sizes a prompt can end with
    d->pf_splits = attn_num_splits(d->max_ctx, m.n_kv_heads, 1, d->dev->n_sm);
    size_t aw = 0;
    for (uint32_t b = 1; b <= PF_CHUNK; ++b)
        aw = std::max(aw, attn_workspace_bytes(m.n_heads, m.n_kv_heads, m.head_dim, b,
                                               std::min(d->pf_splits, attn_num_splits(d->max_ctx, m.n_kv_heads, b, d->dev->n_sm))));
    return dmalloc((void **)&d->pf_x, B * m.dim * 4, "prefill rows") && dmalloc((void **)&d->pf_xn, B * m.dim * 4, "prefill rows") &&
           dmalloc((void **)&d->pf_q, B * d->q_dim * 4, "prefill rows") && dmalloc((void **)&d->pf_att, B * d->q_dim * 4, "prefill rows") &&
           dmalloc((void **)&d->pf_k, B * d->kv_dim * 4, "prefill rows") && dmalloc((void **)&d->pf_v, B * d->kv_dim * 4, "prefill rows") &&
           dmalloc((void **)&d->pf_g, B * m.ffn * 4, "prefill rows") && dmalloc((void **)&d->pf_u, B * m.ffn * 4, "prefill rows") &&
           dmalloc((void **)&d->pf_h, B * m.ffn * 4, "prefill rows") && dmalloc(&d->pf_attn_work, aw, "prefill attention") &&
           dmalloc((void **)&d->pf_x16, qgemm_x16_bytes(PF_CHUNK, m.dim), "prefill fp16 rows") &&
           cuda_ok(cudaMemset(d->pf_attn_work, 0, aw), "prefill attention");
}

// One chunk of B tokens (token ids at tok, positions p0..p0+B-1) through
// every layer: the KV rows land in the cache, the hidden rows are dropped.
bool prefill_chunk(vbs_cu_decoder *d, const uint32_t *tok, uint32_t B, uint32_t p0) {
    const vbs_cu_model_t &m = d->m;
    cudaStream_t st = d->st;
    const uint32_t dim = m.dim, nq = d->q_dim, nk = d->kv_dim, ffn = m.ffn, hd = m.head_dim;
    const int layout = d->persist ? 2 : 1;   // the cache layout of the decoder's steps
    DevState *dev = d->dev;
    if (!cuda_ok(embed_rows_launch(m.embd_type, static_cast<const uint8_t *>(m.embd), tok, B, d->vocab_full, d->pf_x, dim,
                                   dev->err, st),
                 "prefill embed"))
        return false;
    for (uint32_t l = 0; l < m.n_layers; ++l) {
        Layer streamed;
        if (d->stream && !stream_layer(d, l, streamed)) return false;
        const Layer &y = d->stream ? streamed : d->L[l];
        // one input, several matrices: through the GEMM, its activations are
        // converted once (q, k, v here; gate, up below)
        const bool qkv16 = gemm_x16_ok(y.tq, y.wq, nq, dim, B) && gemm_x16_ok(y.tk, y.wk, nk, dim, B) &&
                           gemm_x16_ok(y.tv, y.wv, nk, dim, B);
        const bool gu16 = gemm_x16_ok(y.tgate, y.wgate, ffn, dim, B) && gemm_x16_ok(y.tup, y.wup, ffn, dim, B);
        if (!cuda_ok(pf_rmsnorm_rows_launch(d->pf_x, y.attn_norm, d->pf_xn, B, dim, m.eps, st), "prefill norm"))
            return false;
        if (qkv16 ? (!cuda_ok(qgemm_to_half(d->pf_xn, dim, d->pf_x16, B, dim, dev->n_sm, st), "prefill fp16 rows") ||
                     gemm_x16(dev, y.tq, y.wq, d->pf_x16, d->pf_q, nq, dim, B, 0, st) ||
                     gemm_x16(dev, y.tk, y.wk, d->pf_x16, d->pf_k, nk, dim, B, 0, st) ||
                     gemm_x16(dev, y.tv, y.wv, d->pf_x16, d->pf_v, nk, dim, B, 0, st))
                  : (matvec_any(dev, y.tq, y.wq, d->pf_xn, d->pf_q, nq, dim, B, 0, st) ||
                     matvec_any(dev, y.tk, y.wk, d->pf_xn, d->pf_k, nk, dim, B, 0, st) ||
                     matvec_any(dev, y.tv, y.wv, d->pf_xn, d->pf_v, nk, dim, B, 0, st)))
            return false;
        if (!cuda_ok(pf_rope_store_launch(d->pf_q, d->pf_k, d->pf_v, d->kc, d->vc, B, p0, l, d->max_ctx, m.n_heads,
                                          m.n_kv_heads, hd, m.theta, layout, st),
                     "prefill rope/kv store"))
            return false;
        // row b attends positions 0..p0+b: seq_len p0 + 1, one more per row
        AttnParams ap = {};
        ap.q = d->pf_q; ap.kc = d->kc; ap.vc = d->vc; ap.out = d->pf_att;
        ap.seq_len = p0 + 1; ap.seq_step = 1;
        ap.layer = l; ap.max_ctx = d->max_ctx;
        ap.nqh = m.n_heads; ap.nkh = m.n_kv_heads; ap.hd = hd;
        ap.scale = 1.0f / sqrtf((float)hd);
        ap.batch = B; ap.kv_batch_stride = 0;
        ap.head_major = 1; ap.swz = layout == 2 ? 1u : 0u;
        ap.work = d->pf_attn_work;
        ap.err = dev->err;
        const uint32_t ns = std::min(d->pf_splits, attn_num_splits(p0 + B, m.n_kv_heads, B, dev->n_sm));
        if (!cuda_ok(attn_prefill_supported(ap) ? attn_prefill_launch(ap, st) : attn_launch(ap, ns, st, false),
                     "prefill attention") ||
            matvec_any(dev, y.to, y.wo, d->pf_att, d->pf_x, dim, nq, B, VBS_CU_MV_ACCUMULATE, st) ||
            !cuda_ok(pf_rmsnorm_rows_launch(d->pf_x, y.ffn_norm, d->pf_xn, B, dim, m.eps, st), "prefill norm") ||
            (gu16 ? (!cuda_ok(qgemm_to_half(d->pf_xn, dim, d->pf_x16, B, dim, dev->n_sm, st), "prefill fp16 rows") ||
                     gemm_x16(dev, y.tgate, y.wgate, d->pf_x16, d->pf_g, ffn, dim, B, 0, st) ||
                     gemm_x16(dev, y.tup, y.wup, d->pf_x16, d->pf_u, ffn, dim, B, 0, st))
                  : (matvec_any(dev, y.tgate, y.wgate, d->pf_xn, d->pf_g, ffn, dim, B, 0, st) ||
                     matvec_any(dev, y.tup, y.wup, d->pf_xn, d->pf_u, ffn, dim, B, 0, st))) ||
            !cuda_ok(silu_mul_launch(d->pf_g, d->pf_u, d->pf_h, B * ffn, st), "prefill silu") ||
            matvec_any(dev, y.tdown, y.wdown, d->pf_h, d->pf_x, dim, ffn, B, VBS_CU_MV_ACCUMULATE, st))
            return false;
        if (d->stream && !stream_layer_done(d)) return false;
    }
    return true;
}

// One step's stop decision of device-driven generation (the engine's loop,
// src/vbs_engine.c:295-316), one thread, after the step: ctrl[1] holds the
// step's argmax (first maximum), which the next step feeds. ctrl[2] is the
// decoder's stop word: once set, later steps (the step kernel) and decisions
// do nothing.
__global__ void control_step_kernel(uint32_t *ctrl, vbs_gpu_control_t *gc) {
    if (ctrl[2]) return;
    const uint32_t t = ctrl[1];
    if (gc->eos_token_id != VBS_PGAE_EOS_NONE && t == gc->eos_token_id) {
        gc->state = VBS_PGAE_EXIT;
        ctrl[2] = 1u;
        return;
    }
    const uint32_t n = gc->position;
    reinterpret_cast<uint32_t *>(gc->generated_tokens_dev)[n] = t;
    gc->position = n + 1u;
    gc->current_token = t;
    if (n + 1u >= gc->max_tokens) {
        gc->state = VBS_PGAE_EXIT;
        ctrl[2] = 1u;
    }
}

// The first token to feed comes from the control block; the stop word starts clear.
__global__ void control_start_kernel(uint32_t *ctrl, vbs_gpu_control_t *gc) {
    ctrl[1] = gc->current_token;
    ctrl[2] = 0u;
    gc->state = VBS_PGAE_GENERATE;
    gc->position = 0u;
}

}  // namespace

extern "C" {

vbs_cu_decoder_t *vbs_cu_decoder_create(const vbs_cu_model_t *m, uint32_t max_ctx, uint32_t flags, char *err, size_t cap) {
    auto fail = [&](const char *msg, vbs_cu_decoder *d) -> vbs_cu_decoder_t * {
        if (err && cap) snprintf(err, cap, "%s%s%s", msg, has_error() ? ": " : "", has_error() ? vbs_cuda_last_error() : "");
        if (d) vbs_cu_decoder_destroy(d);
        return nullptr;
    };
    DevState *dev = backend_current();
    if (!dev) return fail("no usable sm_100 device", nullptr);
    if (!m || !m->n_layers || !m->dim || !m->n_heads || !m->n_kv_heads || !m->head_dim || m->n_heads % m->n_kv_heads ||
        !m->ffn || !m->vocab || !max_ctx || m->head_dim % 2 || !m->embd || !m->out || !m->out_norm)
        return fail("invalid model description", nullptr);
    // The decoder runs on its own non-blocking stream, which does not order
    // itself after work on other streams: weights written by kernels or
    // copies still in flight elsewhere (uploads, on-device synthesis) must be
    // complete before its first step reads them.
    if (!cuda_ok(cudaDeviceSynchronize(), "decoder create: pending work")) return fail("device error", nullptr);
    vbs_cu_decoder *d = new vbs_cu_decoder();
    d->m = *m;
    d->flags = flags;
    d->strict = (flags & VBS_CU_DEC_STRICT) != 0;
    d->stream = (flags & VBS_CU_DEC_STREAM) != 0;
    // streamed layers: direct launches around the copy events (no graph, no
    // programmatic overlap across the event waits)
    d->use_graph = !(flags & VBS_CU_DEC_NO_GRAPH) && !d->stream;
    d->use_pdl = !(flags & VBS_CU_DEC_NO_PDL) && !d->strict && !d->stream;
    d->max_ctx = max_ctx;
    d->dev = dev;
    d->kv_dim = m->n_kv_heads * m->head_dim;
    d->q_dim = m->n_heads * m->head_dim;
    d->vocab_full = m->vocab_full ? m->vocab_full : m->vocab;
    d->tp_world = tp_world();
    if (d->tp_world > 1 && d->strict) return fail("strict mode runs on one GPU", d);
    if (d->stream && (d->strict || d->tp_world > 1)) return fail("slice streaming runs the fast per-op step on one GPU", d);
    d->tp_p2p = d->tp_world > 1 && tp_comm() && !(flags & VBS_CU_DEC_TP_NCCL) && m->dim <= TP_DIM_MAX;
    if (d->tp_world == 1 && d->vocab_full != m->vocab) return fail("vocab_full differs from vocab without TP", d);
    if (d->tp_world > 1 && (d->vocab_full != (uint32_t)d->tp_world * m->vocab ||
                            m->vocab_offset != (uint32_t)tp_rank() * m->vocab))   // the logits gather in rank order
        return fail("tensor parallelism: the output rows must split evenly, rank r owning rows r * vocab onward", d);
    d->L.resize(m->n_layers);
    for (uint32_t l = 0; l < m->n_layers; ++l) {
        Layer &y = d->L[l];
        y.attn_norm = m->attn_norm[l]; y.ffn_norm = m->ffn_norm[l];
        y.wq = static_cast<const uint8_t *>(m->wq[l]); y.wk = static_cast<const uint8_t *>(m->wk[l]);
        y.wv = static_cast<const uint8_t *>(m->wv[l]); y.wo = static_cast<const uint8_t *>(m->wo[l]);
        y.wgate = static_cast<const uint8_t *>(m->wgate[l]); y.wup = static_cast<const uint8_t *>(m->wup[l]);
        y.wdown = static_cast<const uint8_t *>(m->wdown[l]);
        y.tq = m->tq[l]; y.tk = m->tk[l]; y.tv = m->tv[l]; y.to = m->to[l];
        y.tgate = m->tgate[l]; y.tup = m->tup[l]; y.tdown = m->tdown[l];
    }
    // the peer-memory exchange lives in the fast kernel's epilogue/prologue:
    // every writer (o_proj, down) and reader (q or fused QKV, gate or fused
    // gate/up, output) must be a fast-kernel launch
    for (const Layer &y : d->L) {
        if (!d->tp_p2p) break;
        const void *wo[1] = {y.wo}, *wd[1] = {y.wdown}, *wq[1] = {y.wq}, *wg[1] = {y.wgate};
        d->tp_p2p = mv_fast_supported(y.to, m->dim, d->q_dim, wo, 1, nullptr, 0) &&
                    mv_fast_supported(y.tdown, m->dim, m->ffn, wd, 1, nullptr, 0) &&
                    mv_fast_supported(y.tq, d->q_dim, m->dim, wq, 1, nullptr, 0) &&
                    mv_fast_supported(y.tgate, m->ffn, m->dim, wg, 1, nullptr, 0);
    }
    {
        const void *wout[1] = {m->out};
        if (d->tp_p2p) d->tp_p2p = mv_fast_supported(m->out_type, m->vocab, m->dim, wout, 1, nullptr, 0);
    }
    if (!cuda_ok(cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking), "decoder stream")) return fail("stream", d);
    if (d->stream) {
        // matrices of one layer, each 256-byte aligned with 256 zero bytes
        // after it (the fast kernels may read past a row end); every layer
        // must have the first layer's types
        const Layer &y0 = d->L[0];
        for (const Layer &y : d->L)
            if (y.tq != y0.tq || y.tk != y0.tk || y.tv != y0.tv || y.to != y0.to || y.tgate != y0.tgate ||
                y.tup != y0.tup || y.tdown != y0.tdown)
                return fail("slice streaming: every layer must have the same weight types", d);
        size_t o = 0;
        for (int k = 0; k < 7; ++k) {
            d->off[k] = o;
            o += (stream_matrix_bytes(d, y0, k) + 256 + 255) & ~(size_t)255;
        }
        d->slot_bytes = o;
        bool sok = cuda_ok(cudaStreamCreateWithFlags(&d->cst, cudaStreamNonBlocking), "copy stream");
        for (int i = 0; sok && i < 2; ++i)
            sok = dmalloc((void **)&d->slot[i], d->slot_bytes, "layer slot") &&
                  cuda_ok(cudaMemset(d->slot[i], 0, d->slot_bytes), "layer slot") &&
                  cuda_ok(cudaEventCreateWithFlags(&d->copied[i], cudaEventDisableTiming), "event") &&
                  cuda_ok(cudaEventCreateWithFlags(&d->done[i], cudaEventDisableTiming), "event");
        if (!sok) return fail("slice streaming buffers", d);
    }
    const size_t big = std::max<size_t>(std::max<size_t>(m->dim, m->ffn), d->q_dim);
    bool ok = dmalloc((void **)&d->x, m->dim * 4, "x") && dmalloc((void **)&d->x2, m->dim * 4, "x2") &&
              dmalloc((void **)&d->q, d->q_dim * 4, "q") && dmalloc((void **)&d->att, d->q_dim * 4, "att") &&
              dmalloc((void **)&d->hid, m->ffn * 4, "hidden") && dmalloc((void **)&d->logits, m->vocab * 4, "logits") &&
              dmalloc((void **)&d->norm, big * 4, "norm") && dmalloc((void **)&d->k, d->kv_dim * 4, "k") &&
              dmalloc((void **)&d->v, d->kv_dim * 4, "v") && dmalloc((void **)&d->gate, m->ffn * 4, "gate") &&
              dmalloc((void **)&d->up, m->ffn * 4, "up") && dmalloc((void **)&d->tmp, big * 4, "tmp") &&
              dmalloc((void **)&d->ctrl, 64, "ctrl") && dmalloc((void **)&d->hist, ((size_t)max_ctx + 2) * 4, "history") &&
              dmalloc((void **)&d->partial, m->dim * 4, "partial");
    if (ok && d->tp_world > 1) ok = dmalloc((void **)&d->logits_full, (size_t)d->vocab_full * 4, "logits_full");
    const size_t cache_elems = (size_t)m->n_layers * max_ctx * d->kv_dim;
    if (ok && d->strict) {
        ok = dmalloc((void **)&d->kcf, cache_elems * 4, "kv cache") && dmalloc((void **)&d->vcf, cache_elems * 4, "kv cache") &&
             dmalloc((void **)&d->scores, (size_t)m->n_heads * max_ctx * 4, "scores") &&
             dmalloc((void **)&d->xq, big, "xq") && dmalloc((void **)&d->qd, (big / 32 + 1) * 4, "qd");
    } else if (ok) {
        ok = dmalloc((void **)&d->kc, cache_elems * 2, "kv cache") && dmalloc((void **)&d->vc, cache_elems * 2, "kv cache");
        if (ok && !(flags & VBS_CU_DEC_NO_PERSIST) && !d->stream && (d->tp_world == 1 || d->tp_p2p)) ok = plan_persistent(d);
        if (ok) {
            d->n_splits = attn_num_splits(max_ctx, m->n_kv_heads, 1, dev->n_sm);
            const size_t wb = attn_workspace_bytes(m->n_heads, m->n_kv_heads, m->head_dim, 1, d->n_splits);
            ok = dmalloc(&d->attn_work, wb, "attention workspace") && cuda_ok(cudaMemset(d->attn_work, 0, wb), "workspace");
        }
    }
    if (ok) ok = dmalloc(&d->argmax_work, argmax_workspace_bytes(), "argmax workspace") &&
                 cuda_ok(cudaMemset(d->argmax_work, 0, argmax_workspace_bytes()), "workspace");
    if (ok) ok = cuda_ok(cudaMallocHost((void **)&d->pinned, 64), "pinned") &&
                 cuda_ok(cudaMallocHost((void **)&d->logits_pinned, (size_t)d->vocab_full * 4), "pinned logits");
    if (!ok) return fail("device allocation failed", d);
    if (d->kc) {
        cudaMemsetAsync(d->kc, 0, cache_elems * 2, d->st);
        cudaMemsetAsync(d->vc, 0, cache_elems * 2, d->st);
    }
    cudaMemsetAsync(d->ctrl, 0, 64, d->st);
    cudaMemsetAsync(d->x, 0, m->dim * 4, d->st);
    if (d->use_graph && !build_graph(d)) {
        if (!d->persist) return fail("decode graph build failed", d);
        // a cooperative launch that cannot be captured: launch the step directly
        cudaGetLastError();
        vbs_cu_clear_error();
        d->use_graph = false;
    }
    if (!d->use_graph) d->kernels_per_step = d->persist ? 1 : 0;
    if (!sync_and_check(d)) return fail("decoder initialisation failed", d);
    return d;
}

void vbs_cu_decoder_destroy(vbs_cu_decoder_t *d) {
    if (!d) return;
    d->magic = 0;
    DeviceGuard guard(d->dev ? d->dev->ordinal : 0);
    if (d->st) cudaStreamSynchronize(d->st);
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->graph) cudaGraphDestroy(d->graph);
    void *bufs[] = {d->x, d->x2, d->q, d->att, d->hid, d->logits, d->logits_full, d->partial, d->norm, d->k, d->v,
                    d->gate, d->up, d->tmp, d->scores, d->xq, d->qd, d->kc, d->vc, d->kcf, d->vcf, d->ctrl, d->hist,
                    d->tok_dev, d->attn_work, d->argmax_work, d->step_layers, d->step_acc, d->step_attn, d->step_packed,
                    d->words_mem, d->words_comm, d->pf_x, d->pf_xn, d->pf_q, d->pf_k, d->pf_v, d->pf_att,
                    d->pf_g, d->pf_u, d->pf_h, d->pf_attn_work, d->pf_x16, d->trace};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (d->cst) cudaStreamSynchronize(d->cst);
    for (int i = 0; i < 2; ++i) {
        if (d->slot[i]) cudaFree(d->slot[i]);
        if (d->copied[i]) cudaEventDestroy(d->copied[i]);
        if (d->done[i]) cudaEventDestroy(d->done[i]);
    }
    if (d->cst) cudaStreamDestroy(d->cst);
    if (d->pinned) cudaFreeHost(d->pinned);
    if (d->logits_pinned) cudaFreeHost(d->logits_pinned);
    if (d->st) cudaStreamDestroy(d->st);
    delete d;
}

int vbs_cu_decoder_forward(vbs_cu_decoder_t *d, const uint32_t *tokens, size_t n, float *logits_out) {
    if (!d || (!tokens && n)) { latch_error("decoder_forward: invalid arguments"); return -1; }
    DeviceGuard guard(d->dev->ordinal);
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] >= d->vocab_full) { latch_error("decoder_forward: token %u >= vocab %u", tokens[i], d->vocab_full); return -1; }
    if (d->host_pos + n > d->max_ctx) { latch_error("decoder_forward: %zu tokens exceed the KV capacity", n); return -1; }
    if (n) {
        if (!put_tokens(d, tokens, n)) return -1;
        for (size_t i = 0; i < n; ++i) {
            if (!cuda_ok(cudaMemcpyAsync(d->ctrl + 1, d->tok_dev + i, 4, cudaMemcpyDeviceToDevice, d->st), "token feed")) return -1;
            if (!enqueue_step(d)) return -1;
        }
    }
    if (logits_out) {
        const float *src = d->tp_world > 1 ? (d->persist ? tp_own_logits() : d->logits_full) : d->logits;
        if (!cuda_ok(cudaMemcpyAsync(d->logits_pinned, src, (size_t)d->vocab_full * 4, cudaMemcpyDeviceToHost, d->st), "logits readback"))
            return -1;
    }
    if (!sync_and_check(d)) return -1;
    if (logits_out) memcpy(logits_out, d->logits_pinned, (size_t)d->vocab_full * 4);
    return 0;
}

int vbs_cu_decoder_prefill(vbs_cu_decoder_t *d, const uint32_t *tokens, size_t n) {
    if (!d || (!tokens && n)) { latch_error("decoder_prefill: invalid arguments"); return -1; }
    if (d->strict) { latch_error("decoder_prefill: strict mode feeds prompts token by token (vbs_cpu arithmetic)"); return -1; }
    if (d->tp_world > 1) { latch_error("decoder_prefill: tensor parallelism feeds prompts token by token"); return -1; }
    DeviceGuard guard(d->dev->ordinal);
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] >= d->vocab_full) { latch_error("decoder_prefill: token %u >= vocab %u", tokens[i], d->vocab_full); return -1; }
    if (d->host_pos + n > d->max_ctx) { latch_error("decoder_prefill: %zu tokens exceed the KV capacity", n); return -1; }
    if (!n) return 0;
    if (!prefill_buffers(d) || !put_tokens(d, tokens, n)) return -1;
    for (size_t c0 = 0; c0 < n; c0 += PF_CHUNK)
        if (!prefill_chunk(d, d->tok_dev + c0, (uint32_t)std::min<size_t>(PF_CHUNK, n - c0), (uint32_t)(d->host_pos + c0)))
            return -1;
    d->host_pos += n;
    d->pinned[0] = (uint32_t)d->host_pos;   // the next step's position; its token comes with that step
    if (!cuda_ok(cudaMemcpyAsync(d->ctrl, d->pinned, 4, cudaMemcpyHostToDevice, d->st), "prefill position")) return -1;
    return sync_and_check(d) ? 0 : -1;
}

void vbs_cu_decoder_reset(vbs_cu_decoder_t *d) {
    if (!d) return;
    DeviceGuard guard(d->dev->ordinal);
    cudaMemsetAsync(d->ctrl, 0, 4, d->st);
    cudaStreamSynchronize(d->st);
    d->host_pos = 0;
}

int vbs_cu_decoder_set_position(vbs_cu_decoder_t *d, uint32_t pos, uint32_t token) {
    if (!d || pos >= d->max_ctx) { latch_error("decoder_set_position: position out of range"); return -1; }
    DeviceGuard guard(d->dev->ordinal);
    d->pinned[0] = pos;
    d->pinned[1] = token;
    if (!cuda_ok(cudaMemcpyAsync(d->ctrl, d->pinned, 8, cudaMemcpyHostToDevice, d->st), "set position")) return -1;
    d->host_pos = pos;
    return cuda_ok(cudaStreamSynchronize(d->st), "set position") ? 0 : -1;
}

uint32_t vbs_cu_decoder_position(vbs_cu_decoder_t *d) {
    if (!d) return 0;
    DeviceGuard guard(d->dev->ordinal);
    if (!cuda_ok(cudaMemcpyAsync(d->pinned, d->ctrl, 8, cudaMemcpyDeviceToHost, d->st), "position")) return 0;
    cudaStreamSynchronize(d->st);
    return d->pinned[0];
}

int vbs_cu_decoder_generate(vbs_cu_decoder_t *d, const uint32_t *prompt, size_t n_prompt, uint32_t n_new, uint32_t *out) {
    if (!d || !prompt || !n_prompt || (n_new && !out)) { latch_error("decoder_generate: invalid arguments"); return -1; }
    DeviceGuard guard(d->dev->ordinal);
    for (size_t i = 0; i < n_prompt; ++i)
        if (prompt[i] >= d->vocab_full) { latch_error("decoder_generate: token %u >= vocab", prompt[i]); return -1; }
    if (d->host_pos + n_prompt + (n_new ? n_new - 1 : 0) > d->max_ctx) {
        latch_error("decoder_generate: exceeds context capacity");
        return -1;
    }
    const uint32_t start = (uint32_t)d->host_pos;
    if (vbs_cu_decoder_forward(d, prompt, n_prompt, nullptr)) return -1;
    for (uint32_t i = 1; i < n_new; ++i)
        if (!enqueue_step(d)) return -1;
    if (n_new) {
        if (!cuda_ok(cudaMemcpyAsync(out, d->hist + start + n_prompt, (size_t)n_new * 4, cudaMemcpyDeviceToHost, d->st), "tokens"))
            return -1;
    }
    return sync_and_check(d) ? 0 : -1;
}

int vbs_cu_decoder_run_control(vbs_cu_decoder_t *d, void *control) {
    if (!d || d->magic != kDecoderMagic || !control) { latch_error("decoder_run_control: invalid decoder or control block"); return -1; }
    if (d->tp_world > 1) { latch_error("decoder_run_control: tensor-parallel decoders are driven per rank"); return -1; }
    DeviceGuard guard(d->dev->ordinal);
    vbs_gpu_control_t gc;
    if (!cuda_ok(cudaMemcpyAsync(&gc, control, sizeof gc, cudaMemcpyDeviceToHost, d->st), "control block") ||
        !cuda_ok(cudaStreamSynchronize(d->st), "control block"))
        return -1;
    if ((gc.state != VBS_PGAE_PREFILL && gc.state != VBS_PGAE_GENERATE) || !gc.max_tokens || !gc.generated_tokens_dev ||
        gc.vocab_size != d->vocab_full || gc.current_token >= d->vocab_full) {
        latch_error("decoder_run_control: control block state %u, max_tokens %u, vocab %u (decoder %u), token %u, "
                    "tokens buffer %s", gc.state, gc.max_tokens, gc.vocab_size, d->vocab_full, gc.current_token,
                    gc.generated_tokens_dev ? "set" : "missing");
        return -1;
    }
    if (d->host_pos + gc.max_tokens > d->max_ctx) {
        latch_error("decoder_run_control: %u steps from position %llu exceed the KV capacity %u", gc.max_tokens,
                    (unsigned long long)d->host_pos, d->max_ctx);
        return -1;
    }
    auto *gcd = static_cast<vbs_gpu_control_t *>(control);
    note_launches(1);
    control_start_kernel<<<1, 1, 0, d->st>>>(d->ctrl, gcd);
    if (!cuda_ok(cudaGetLastError(), "control start")) return -1;
    // the persistent step kernel returns at once when the stop word is set,
    // so steps go out 16 at a time; the per-op and strict steps do not look
    // at it and go out one at a time
    const uint32_t chunk = d->persist ? 16u : 1u;
    uint32_t done = 0;
    while (done < gc.max_tokens) {
        const uint32_t n = std::min(chunk, gc.max_tokens - done);
        for (uint32_t i = 0; i < n; ++i) {
            if (!enqueue_step(d)) return -1;
            note_launches(1);
            control_step_kernel<<<1, 1, 0, d->st>>>(d->ctrl, gcd);
            if (!cuda_ok(cudaGetLastError(), "control step")) return -1;
        }
        done += n;
        if (!cuda_ok(cudaMemcpyAsync(d->pinned + 2, d->ctrl + 2, 4, cudaMemcpyDeviceToHost, d->st), "stop word") ||
            !sync_and_check(d))
            return -1;
        if (d->pinned[2]) break;
    }
    // the decoder's position: steps that ran (the stopped ones did nothing)
    if (!cuda_ok(cudaMemcpyAsync(d->pinned, d->ctrl, 4, cudaMemcpyDeviceToHost, d->st), "position")) return -1;
    // the next steps of the decoder run normally
    if (!cuda_ok(cudaMemsetAsync(d->ctrl + 2, 0, 4, d->st), "stop word")) return -1;
    if (!sync_and_check(d)) return -1;
    d->host_pos = d->pinned[0];
    if (gc.logits_dev) {
        const float *src = vbs_cu_decoder_logits_device(d);
        if (!cuda_ok(cudaMemcpyAsync(reinterpret_cast<void *>(gc.logits_dev), src, (size_t)d->vocab_full * 4,
                                     cudaMemcpyDeviceToDevice, d->st), "logits copy") ||
            !sync_and_check(d))
            return -1;
    }
    return 0;
}

int vbs_cu_decoder_set_wait_test(vbs_cu_decoder_t *d, uint64_t wait_ns, uint32_t drop_op) {
    if (!d || d->magic != kDecoderMagic) { latch_error("decoder_set_wait_test: invalid decoder"); return -1; }
    if (!d->persist) { latch_error("decoder_set_wait_test: the decoder does not run the persistent step kernel"); return -1; }
    if (wait_ns < 1000000ull || wait_ns > kWaitNs) { latch_error("decoder_set_wait_test: wait limit outside 1 ms .. 2 s"); return -1; }
    DeviceGuard guard(d->dev->ordinal);
    if (!cuda_ok(cudaStreamSynchronize(d->st), "decoder_set_wait_test")) return -1;
    d->sp.wait_ns = wait_ns;
    d->sp.drop_op = drop_op;
    // the step graph holds the old parameters: launch directly from now on
    if (d->exec) { cudaGraphExecDestroy(d->exec); d->exec = nullptr; }
    if (d->graph) { cudaGraphDestroy(d->graph); d->graph = nullptr; }
    d->use_graph = false;
    return 0;
}

int vbs_cu_decoder_enqueue_steps(vbs_cu_decoder_t *d, uint32_t n) {
    if (!d) return -1;
    DeviceGuard guard(d->dev->ordinal);
    if (d->host_pos + n > d->max_ctx) { latch_error("enqueue_steps: exceeds the KV capacity"); return -1; }
    for (uint32_t i = 0; i < n; ++i)
        if (!enqueue_step(d)) return -1;
    return 0;
}

void *vbs_cu_decoder_stream(vbs_cu_decoder_t *d) { return d ? d->st : nullptr; }
const float *vbs_cu_decoder_logits_device(vbs_cu_decoder_t *d) {
    return d ? (d->tp_world > 1 ? (d->persist ? tp_own_logits() : d->logits_full) : d->logits) : nullptr;
}
uint32_t vbs_cu_decoder_kernels_per_step(vbs_cu_decoder_t *d) { return d ? d->kernels_per_step : 0; }
#ifdef VBS_STEP_TRACE
// Profiling builds only: the device address of the last step's timeline,
// [CTA][op][SK_TR_SLOTS] %globaltimer stamps.
VBS_API void *vbs_cu_decoder_trace(vbs_cu_decoder_t *d, uint32_t *n_ctas, uint32_t *n_ops, uint32_t *n_slots) {
    if (!d || !d->trace) return nullptr;
    if (n_ctas) *n_ctas = (uint32_t)d->dev->n_sm;
    if (n_ops) *n_ops = 5 * d->m.n_layers + 2;
    if (n_slots) *n_slots = SK_TR_SLOTS;
    return d->trace;
}
#endif
uint32_t vbs_cu_decoder_tp_mode(vbs_cu_decoder_t *d) { return !d || d->tp_world == 1 ? 0u : (d->tp_p2p ? 2u : 1u); }

}  // extern "C"
