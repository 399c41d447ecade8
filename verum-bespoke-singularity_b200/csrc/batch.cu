// batch.cu -- B sequences decoded in lockstep (batched decode).
//
// The reference's engine has one sequence and no batch dimension: every
// decode step streams every weight for one token (src/vbs_specializer.c:
// 231-359). Serving B sequences together reads each weight once for B
// tokens, which is where the batched matvec (B <= 8, csrc/mvb.cu) and the
// tcgen05 GEMM (B > 8, csrc/gemm.cu) earn their keep. Each step here takes
// one token per sequence, all at the same position, through the per-op
// kernels:
//   embedding rows -> per layer: row RMSNorm, Q/K/V for B rows, RoPE and
//   the KV store into each sequence's own head-major cache, split-KV
//   attention over B sequences (one cache stride apart), o_proj + residual,
//   RMSNorm, gate/up, SiLU*up, down + residual -> output norm, logits
//   [B][vocab], per-sequence argmax (first maximum) fed back as the next
//   tokens.
// The op order and the arithmetic of every op are those of the one-sequence
// per-op decoder, so each sequence's logits match a one-sequence decoder
// fed the same tokens to the kernels' rounding. The position lives on the
// device (RoPE, the KV store and attention read it; the step's last kernel
// advances it), so after one direct step, which sizes every workspace, a
// step is captured once as a CUDA graph and replayed.
#include "backend.h"
#include "common.cuh"
#include "kernels.h"
#include "vbs_b200.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

using namespace vbs;

namespace {

constexpr uint32_t kBatchMagic = 0x56424254u;   // "VBBT": a live batch decoder
constexpr uint32_t kBatchMax = 64;              // sequences per decoder

struct BLayer {
    const float *attn_norm, *ffn_norm;
    const uint8_t *wq, *wk, *wv, *wo, *wgate, *wup, *wdown;
    int tq, tk, tv, to, tgate, tup, tdown;
    // the decoder's own copies of [wq; wk; wv] and [wgate; wup] as one
    // matrix each (NULL when the types differ): one launch per group
    uint8_t *wqkv, *wgu;
};

// h[b][i] = SiLU(gu[b][i]) * gu[b][ffn + i] (src/vbs_host_math.h:53-57, the
// expression of silu_mul_kernel), rows of the fused gate|up projection.
__global__ void bd_silu_rows_kernel(const float *__restrict__ gu, float *__restrict__ h, uint32_t rows, uint32_t ffn) {
    const uint64_t n = (uint64_t)rows * ffn;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = t / ffn, i = t % ffn;
        const float g = gu[b * 2 * ffn + i], u = gu[b * 2 * ffn + ffn + i];
        h[t] = g / (1.0f + expf(-g)) * u;
    }
}

// Makes `ordinal` current for the scope and restores the caller's device.
struct BatchDeviceGuard {
    int prev = -1;
    explicit BatchDeviceGuard(int ordinal) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != ordinal) cudaSetDevice(ordinal);
    }
    ~BatchDeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

template <typename T> bool balloc(T **p, size_t bytes, const char *what) {
    return cuda_ok(cudaMalloc(reinterpret_cast<void **>(p), bytes ? bytes : 16), what);
}

}  // namespace

struct vbs_cu_batch_decoder {
    uint32_t magic = kBatchMagic;
    vbs_cu_model_t m;
    std::vector<BLayer> L;
    DevState *dev = nullptr;
    // The device's state with workspaces of this decoder's own: its graph
    // holds their addresses, which the device-wide ones (regrown by other
    // callers) would not keep.
    DevState own;
    cudaStream_t st = nullptr;
    uint32_t B = 0, max_ctx = 0, q_dim = 0, kv_dim = 0, splits = 1, pos = 0;
    uint64_t seq_stride = 0;   // cache elements per sequence: [layer][kv head][max_ctx][head_dim]
    float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *g = nullptr,
          *u = nullptr, *h = nullptr, *logits = nullptr;
    float *qkv = nullptr;      // [B][q_dim + 2 kv_dim]: the fused projection's rows (g holds [B][2 ffn])
    uint16_t *kc = nullptr, *vc = nullptr;
    uint32_t *tok = nullptr;   // [B] the tokens the next step feeds (device)
    uint32_t *pos_dev = nullptr;   // the position of the next step (device)
    void *attn_work = nullptr, *argmax_work = nullptr;
    bool warm = false;         // a direct step ran: every workspace has its final size
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {

bool bd_valid(const vbs_cu_batch_decoder *d) { return d && d->magic == kBatchMagic; }

__global__ void bd_advance_kernel(uint32_t *pos_dev) { ++*pos_dev; }

// The kernels of one lockstep step at position *pos_dev: feeds d->tok,
// leaves the logits in d->logits and the argmax of every sequence in
// d->tok, advances *pos_dev.
bool bd_record(vbs_cu_batch_decoder *d) {
    const vbs_cu_model_t &m = d->m;
    cudaStream_t st = d->st;
    DevState *dev = &d->own;
    const uint32_t B = d->B, dim = m.dim, nq = d->q_dim, nk = d->kv_dim, ffn = m.ffn, hd = m.head_dim;
    if (!cuda_ok(embed_rows_launch(m.embd_type, static_cast<const uint8_t *>(m.embd), d->tok, B, m.vocab, d->x, dim,
                                   dev->err, st),
                 "batch embed"))
        return false;
    for (uint32_t l = 0; l < m.n_layers; ++l) {
        const BLayer &y = d->L[l];
        const uint32_t nqkv = nq + 2 * nk;
        if (!cuda_ok(pf_rmsnorm_rows_launch(d->x, y.attn_norm, d->xn, B, dim, m.eps, st), "batch norm"))
            return false;
        if (y.wqkv ? (matvec_any(dev, y.tq, y.wqkv, d->xn, d->qkv, nqkv, dim, B, 0, st) ||
                      !cuda_ok(rope_store_seqs_launch(d->qkv, d->q, nqkv, d->qkv + nq, d->qkv + nq + nk, nqkv, d->kc,
                                                      d->vc, B, d->seq_stride, d->pos_dev, l, d->max_ctx, m.n_heads,
                                                      m.n_kv_heads, hd, m.theta, st),
                               "batch rope/kv store"))
                   : (matvec_any(dev, y.tq, y.wq, d->xn, d->q, nq, dim, B, 0, st) ||
                      matvec_any(dev, y.tk, y.wk, d->xn, d->k, nk, dim, B, 0, st) ||
                      matvec_any(dev, y.tv, y.wv, d->xn, d->v, nk, dim, B, 0, st) ||
                      !cuda_ok(rope_store_seqs_launch(d->q, d->q, nq, d->k, d->v, nk, d->kc, d->vc, B, d->seq_stride,
                                                      d->pos_dev, l, d->max_ctx, m.n_heads, m.n_kv_heads, hd, m.theta,
                                                      st),
                               "batch rope/kv store")))
            return false;
        AttnParams ap = {};
        ap.q = d->q; ap.kc = d->kc; ap.vc = d->vc; ap.out = d->att;
        ap.seq_dev = d->pos_dev; ap.seq_step = 0;   // positions <= *pos_dev
        ap.layer = l; ap.max_ctx = d->max_ctx;
        ap.nqh = m.n_heads; ap.nkh = m.n_kv_heads; ap.hd = hd;
        ap.scale = 1.0f / sqrtf((float)hd);
        ap.batch = B; ap.kv_batch_stride = d->seq_stride;
        ap.head_major = 1; ap.swz = 0;
        ap.work = d->attn_work;
        ap.err = dev->err;
        if (!cuda_ok(attn_launch(ap, d->splits, st, false), "batch attention") ||
            matvec_any(dev, y.to, y.wo, d->att, d->x, dim, nq, B, VBS_CU_MV_ACCUMULATE, st) ||
            !cuda_ok(pf_rmsnorm_rows_launch(d->x, y.ffn_norm, d->xn, B, dim, m.eps, st), "batch norm"))
            return false;
        if (y.wgu) {
            if (matvec_any(dev, y.tgate, y.wgu, d->xn, d->g, 2 * ffn, dim, B, 0, st)) return false;
            note_launches(1);
            bd_silu_rows_kernel<<<std::min<uint32_t>((B * ffn + 255) / 256, (uint32_t)dev->n_sm * 8), 256, 0, st>>>(
                d->g, d->h, B, ffn);
            if (!cuda_ok(cudaGetLastError(), "batch silu")) return false;
        } else if (matvec_any(dev, y.tgate, y.wgate, d->xn, d->g, ffn, dim, B, 0, st) ||
                   matvec_any(dev, y.tup, y.wup, d->xn, d->u, ffn, dim, B, 0, st) ||
                   !cuda_ok(silu_mul_launch(d->g, d->u, d->h, B * ffn, st), "batch silu")) {
            return false;
        }
        if (matvec_any(dev, y.tdown, y.wdown, d->h, d->x, dim, ffn, B, VBS_CU_MV_ACCUMULATE, st)) return false;
    }
    if (!cuda_ok(pf_rmsnorm_rows_launch(d->x, m.out_norm, d->xn, B, dim, m.eps, st), "batch output norm") ||
        matvec_any(dev, m.out_type, static_cast<const uint8_t *>(m.out), d->xn, d->logits, m.vocab, dim, B, 0, st))
        return false;
    for (uint32_t b = 0; b < B; ++b)   // first maximum wins (src/vbs_cpu_main.c:78-80)
        if (!cuda_ok(argmax_launch(d->logits + (size_t)b * m.vocab, m.vocab, d->tok + b, nullptr, nullptr, 0, d->argmax_work,
                                   st, false),
                     "batch argmax"))
            return false;
    note_launches(1);
    bd_advance_kernel<<<1, 1, 0, st>>>(d->pos_dev);
    return cuda_ok(cudaGetLastError(), "batch position");
}

// One step: the first directly (it sizes the workspaces), then a graph of
// one step, captured once and replayed.
bool bd_step(vbs_cu_batch_decoder *d) {
    if (d->pos >= d->max_ctx) {
        latch_error("batch decoder: position %u reaches the KV capacity %u", d->pos, d->max_ctx);
        return false;
    }
    if (!d->warm) {
        if (!bd_record(d)) return false;
        d->warm = true;
    } else {
        if (!d->exec) {
            if (!cuda_ok(cudaStreamBeginCapture(d->st, cudaStreamCaptureModeThreadLocal), "batch capture")) return false;
            const bool ok = bd_record(d);
            cudaGraph_t g = nullptr;
            const cudaError_t e = cudaStreamEndCapture(d->st, &g);
            if (!ok || !cuda_ok(e, "batch capture")) {
                if (g) cudaGraphDestroy(g);
                return false;
            }
            d->graph = g;
            if (!cuda_ok(cudaGraphInstantiate(&d->exec, d->graph, 0), "batch graph")) return false;
        }
        if (!cuda_ok(cudaGraphLaunch(d->exec, d->st), "batch graph launch")) return false;
    }
    ++d->pos;
    return true;
}

bool bd_sync(vbs_cu_batch_decoder *d) {
    return cuda_ok(cudaStreamSynchronize(d->st), "batch decoder") && check_device_error(d->dev, d->st);
}

}  // namespace

extern "C" {

VBS_API void vbs_cu_batch_decoder_destroy(vbs_cu_batch_decoder_t *d) {
    if (!bd_valid(d)) return;
    d->magic = 0;
    BatchDeviceGuard guard(d->dev ? d->dev->ordinal : 0);
    if (d->st) cudaStreamSynchronize(d->st);
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->graph) cudaGraphDestroy(d->graph);
    for (BLayer &y : d->L) {
        if (y.wqkv) cudaFree(y.wqkv);
        if (y.wgu) cudaFree(y.wgu);
    }
    void *bufs[] = {d->x, d->xn, d->q, d->k, d->v, d->att, d->g, d->u, d->h, d->logits, d->qkv, d->kc, d->vc, d->tok,
                    d->pos_dev, d->attn_work, d->argmax_work, d->own.mvb_work, d->own.qg_work};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (d->st) cudaStreamDestroy(d->st);
    delete d;
}

VBS_API vbs_cu_batch_decoder_t *vbs_cu_batch_decoder_create(const vbs_cu_model_t *m, uint32_t max_ctx, uint32_t batch,
                                                            char *err, size_t err_cap) {
    auto fail = [&](const char *why, vbs_cu_batch_decoder *d) -> vbs_cu_batch_decoder_t * {
        if (err && err_cap) snprintf(err, err_cap, "%s", why);
        latch_error("batch decoder: %s", why);
        if (d) vbs_cu_batch_decoder_destroy(d);
        return nullptr;
    };
    if (!m || !m->n_layers || !m->dim || !m->n_heads || !m->n_kv_heads || m->n_heads % m->n_kv_heads || !m->head_dim ||
        m->head_dim % 8 || !m->ffn || !m->vocab || !m->embd || !m->out || !m->out_norm || !max_ctx)
        return fail("invalid model description", nullptr);
    if (!batch || batch > kBatchMax) return fail("batch must be 1..64 sequences", nullptr);
    if (m->vocab_full && m->vocab_full != m->vocab) return fail("one GPU: vocab_full must equal vocab", nullptr);
    DevState *dev = backend_current();
    if (!dev) return fail("no usable sm_100 device is current", nullptr);
    BatchDeviceGuard guard(dev->ordinal);
    // weights written by work still in flight on other streams must be
    // complete before this decoder's own stream reads them
    if (!cuda_ok(cudaDeviceSynchronize(), "batch decoder create: pending work")) return fail("device error", nullptr);
    vbs_cu_batch_decoder *d = new vbs_cu_batch_decoder();
    d->m = *m;
    d->dev = dev;
    d->own = *dev;
    d->own.attn_work = nullptr;
    d->own.attn_work_bytes = 0;
    d->own.mvb_work = nullptr;
    d->own.mvb_work_bytes = 0;
    d->own.qg_work = nullptr;
    d->own.qg_work_bytes = 0;
    d->B = batch;
    d->max_ctx = max_ctx;
    d->q_dim = m->n_heads * m->head_dim;
    d->kv_dim = m->n_kv_heads * m->head_dim;
    d->seq_stride = (uint64_t)m->n_layers * max_ctx * d->kv_dim;
    d->L.resize(m->n_layers);
    for (uint32_t l = 0; l < m->n_layers; ++l) {
        BLayer &y = d->L[l];
        y.attn_norm = m->attn_norm[l];
        y.ffn_norm = m->ffn_norm[l];
        y.wq = static_cast<const uint8_t *>(m->wq[l]);
        y.wk = static_cast<const uint8_t *>(m->wk[l]);
        y.wv = static_cast<const uint8_t *>(m->wv[l]);
        y.wo = static_cast<const uint8_t *>(m->wo[l]);
        y.wgate = static_cast<const uint8_t *>(m->wgate[l]);
        y.wup = static_cast<const uint8_t *>(m->wup[l]);
        y.wdown = static_cast<const uint8_t *>(m->wdown[l]);
        y.tq = m->tq[l]; y.tk = m->tk[l]; y.tv = m->tv[l]; y.to = m->to[l];
        y.tgate = m->tgate[l]; y.tup = m->tup[l]; y.tdown = m->tdown[l];
        y.wqkv = y.wgu = nullptr;
    }
    // [wq; wk; wv] and [wgate; wup] copied once into one matrix each (same
    // type, same width: the rows simply follow one another), 256 bytes of
    // zero tail as the matvec kernels may read past a row end
    for (uint32_t l = 0; l < m->n_layers; ++l) {
        BLayer &y = d->L[l];
        if (y.tq == y.tk && y.tq == y.tv) {
            const size_t rb = row_bytes(y.tq, m->dim), nq = (size_t)d->q_dim * rb, nk = (size_t)d->kv_dim * rb;
            if (!balloc(&y.wqkv, nq + 2 * nk + 256, "batch fused q/k/v") ||
                !cuda_ok(cudaMemset(y.wqkv + nq + 2 * nk, 0, 256), "batch fused q/k/v") ||
                !cuda_ok(cudaMemcpy(y.wqkv, y.wq, nq, cudaMemcpyDeviceToDevice), "batch fused q/k/v") ||
                !cuda_ok(cudaMemcpy(y.wqkv + nq, y.wk, nk, cudaMemcpyDeviceToDevice), "batch fused q/k/v") ||
                !cuda_ok(cudaMemcpy(y.wqkv + nq + nk, y.wv, nk, cudaMemcpyDeviceToDevice), "batch fused q/k/v"))
                return fail("device allocation failed", d);
        }
        if (y.tgate == y.tup) {
            const size_t half = (size_t)m->ffn * row_bytes(y.tgate, m->dim);
            if (!balloc(&y.wgu, 2 * half + 256, "batch fused gate/up") ||
                !cuda_ok(cudaMemset(y.wgu + 2 * half, 0, 256), "batch fused gate/up") ||
                !cuda_ok(cudaMemcpy(y.wgu, y.wgate, half, cudaMemcpyDeviceToDevice), "batch fused gate/up") ||
                !cuda_ok(cudaMemcpy(y.wgu + half, y.wup, half, cudaMemcpyDeviceToDevice), "batch fused gate/up"))
                return fail("device allocation failed", d);
        }
    }
    const size_t B = batch, kv_bytes = B * d->seq_stride * sizeof(uint16_t);
    d->splits = attn_num_splits(max_ctx, m->n_kv_heads, batch, dev->n_sm);
    const size_t aw = attn_workspace_bytes(m->n_heads, m->n_kv_heads, m->head_dim, batch, d->splits);
    if (!cuda_ok(cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking), "batch decoder stream") ||
        !balloc(&d->x, B * m->dim * 4, "batch rows") || !balloc(&d->xn, B * m->dim * 4, "batch rows") ||
        !balloc(&d->q, B * d->q_dim * 4, "batch rows") || !balloc(&d->k, B * d->kv_dim * 4, "batch rows") ||
        !balloc(&d->v, B * d->kv_dim * 4, "batch rows") || !balloc(&d->att, B * d->q_dim * 4, "batch rows") ||
        !balloc(&d->g, B * 2 * m->ffn * 4, "batch rows") || !balloc(&d->u, B * m->ffn * 4, "batch rows") ||
        !balloc(&d->qkv, B * (d->q_dim + 2 * d->kv_dim) * 4, "batch rows") ||
        !balloc(&d->h, B * m->ffn * 4, "batch rows") || !balloc(&d->logits, B * m->vocab * 4, "batch logits") ||
        !balloc(&d->kc, kv_bytes, "batch KV cache") || !balloc(&d->vc, kv_bytes, "batch KV cache") ||
        !balloc(&d->tok, B * 4, "batch tokens") || !balloc(&d->pos_dev, 4, "batch position") ||
        !balloc(&d->attn_work, aw, "batch attention") ||
        !balloc(&d->argmax_work, argmax_workspace_bytes(), "batch argmax") ||
        !cuda_ok(cudaMemsetAsync(d->attn_work, 0, aw, d->st), "batch attention") ||
        !cuda_ok(cudaMemsetAsync(d->argmax_work, 0, argmax_workspace_bytes(), d->st), "batch argmax") ||
        !cuda_ok(cudaMemsetAsync(d->kc, 0, kv_bytes, d->st), "batch KV cache") ||
        !cuda_ok(cudaMemsetAsync(d->vc, 0, kv_bytes, d->st), "batch KV cache") ||
        !cuda_ok(cudaMemsetAsync(d->tok, 0, B * 4, d->st), "batch tokens") ||
        !cuda_ok(cudaMemsetAsync(d->pos_dev, 0, 4, d->st), "batch position") || !bd_sync(d))
        return fail("device allocation failed", d);
    return d;
}

VBS_API int vbs_cu_batch_decoder_step(vbs_cu_batch_decoder_t *d, const uint32_t *tokens, float *logits_out,
                                      uint32_t *next_tokens) {
    if (!bd_valid(d)) { latch_error("batch decoder step: invalid decoder"); return -1; }
    BatchDeviceGuard guard(d->dev->ordinal);
    if (tokens) {
        for (uint32_t b = 0; b < d->B; ++b)
            if (tokens[b] >= d->m.vocab) { latch_error("batch decoder step: token %u >= vocab", tokens[b]); return -1; }
        if (!cuda_ok(cudaMemcpyAsync(d->tok, tokens, (size_t)d->B * 4, cudaMemcpyHostToDevice, d->st), "batch tokens"))
            return -1;
    }
    if (!bd_step(d)) return -1;
    if (logits_out && !cuda_ok(cudaMemcpyAsync(logits_out, d->logits, (size_t)d->B * d->m.vocab * 4,
                                               cudaMemcpyDeviceToHost, d->st), "batch logits"))
        return -1;
    if (next_tokens &&
        !cuda_ok(cudaMemcpyAsync(next_tokens, d->tok, (size_t)d->B * 4, cudaMemcpyDeviceToHost, d->st), "batch tokens"))
        return -1;
    return bd_sync(d) ? 0 : -1;
}

VBS_API int vbs_cu_batch_decoder_enqueue_steps(vbs_cu_batch_decoder_t *d, uint32_t n_steps) {
    if (!bd_valid(d)) { latch_error("batch decoder: invalid decoder"); return -1; }
    BatchDeviceGuard guard(d->dev->ordinal);
    for (uint32_t i = 0; i < n_steps; ++i)
        if (!bd_step(d)) return -1;
    return 0;
}

VBS_API int vbs_cu_batch_decoder_set_position(vbs_cu_batch_decoder_t *d, uint32_t pos, const uint32_t *tokens) {
    if (!bd_valid(d) || pos >= d->max_ctx) { latch_error("batch decoder: invalid decoder or position"); return -1; }
    BatchDeviceGuard guard(d->dev->ordinal);
    if (tokens) {
        for (uint32_t b = 0; b < d->B; ++b)
            if (tokens[b] >= d->m.vocab) { latch_error("batch decoder: token %u >= vocab", tokens[b]); return -1; }
        if (!cuda_ok(cudaMemcpyAsync(d->tok, tokens, (size_t)d->B * 4, cudaMemcpyHostToDevice, d->st), "batch tokens") ||
            !bd_sync(d))
            return -1;
    }
    if (!cuda_ok(cudaMemcpyAsync(d->pos_dev, &pos, 4, cudaMemcpyHostToDevice, d->st), "batch position") || !bd_sync(d))
        return -1;
    d->pos = pos;
    return 0;
}

VBS_API uint32_t vbs_cu_batch_decoder_position(vbs_cu_batch_decoder_t *d) { return bd_valid(d) ? d->pos : 0u; }
VBS_API void vbs_cu_batch_decoder_reset(vbs_cu_batch_decoder_t *d) {
    if (!bd_valid(d)) return;
    BatchDeviceGuard guard(d->dev->ordinal);
    if (cuda_ok(cudaMemsetAsync(d->pos_dev, 0, 4, d->st), "batch position") && bd_sync(d)) d->pos = 0;
}
VBS_API void *vbs_cu_batch_decoder_stream(vbs_cu_batch_decoder_t *d) { return bd_valid(d) ? d->st : nullptr; }

}  // extern "C"
