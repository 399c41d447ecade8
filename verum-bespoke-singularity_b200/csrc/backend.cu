// backend.cu -- g_vbs_cuda_backend, the ops table the reference engine
// binds for CUDA (include/vbs_backend.h:64-101 of the reference), and the
// vbs_cu_* extension entry points (include/vbs_b200.h).
//
// Replaces src/vbs_backend_cuda.c. Differences in behaviour, all on
// purpose:
//  * devices report max_working_set_bytes / max_buffer_bytes (the reference
//    left them 0, which zeroes the profiler's VRAM and the engine's KV
//    budget, src/vbs_profiler.c:160-161, src/vbs_engine.c:127-138);
//  * every linear tile row is computed (the reference launched rows/32
//    warps, src/vbs_backend_cuda.c:255-256) and both calling conventions are
//    honoured (staged tile with offsets and accumulation as well as the
//    bridge's resident weights);
//  * Q4_K has a kernel; attention is correct for any head_dim in
//    {32, 64, 128, 256};
//  * the first failure is latched: dispatch errors the bridge drops
//    (src/vbs_specializer_bridge.c:83-90) make the next copy_to_host fail
//    and print the message.
#include "vbs_b200.h"
#include "backend.h"
#include "common.cuh"
#include "kernels.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

namespace vbs {

// ---------------------------------------------------------------------------
// error latch
// ---------------------------------------------------------------------------
static std::mutex g_err_mu;
static char g_err_msg[512] = "ok";
static std::atomic<int> g_err_set{0};
static std::atomic<uint64_t> g_launches{0};

void note_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void latch_error(const char *fmt, ...) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (g_err_set.load()) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err_msg, sizeof(g_err_msg), fmt, ap);
    va_end(ap);
    g_err_set.store(1);
}
bool has_error() { return g_err_set.load() != 0; }

bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    latch_error("%s: %s", what, cudaGetErrorString(e));
    return false;
}

// ---------------------------------------------------------------------------
// devices
// ---------------------------------------------------------------------------
static std::mutex g_init_mu;
static bool g_probed = false, g_ready = false;
static vbs_device_t g_devices[8];
static DevState g_state[8];
static int g_ndev = 0;
static char g_init_msg[256] = "not probed yet";

static bool do_init() {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (g_probed) return g_ready;
    g_probed = true;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count <= 0) {
        snprintf(g_init_msg, sizeof(g_init_msg), "no CUDA device (%s)", e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
        return false;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    for (int i = 0; i < count && g_ndev < 8; ++i) {
        cudaDeviceProp pr;
        if (cudaGetDeviceProperties(&pr, i) != cudaSuccess) continue;
        if (pr.major != 10 || pr.minor != 0) continue;   // code is built for sm_100a only
        if (cudaSetDevice(i) != cudaSuccess) continue;
        size_t fr = 0, tot = 0;
        cudaMemGetInfo(&fr, &tot);
        DevState &s = g_state[g_ndev];
        s.ordinal = i;
        s.n_sm = pr.multiProcessorCount;
        if (cudaMalloc(&s.err, 256) != cudaSuccess) continue;
        cudaMemset(s.err, 0, 256);
        if (mv_configure() != cudaSuccess || mvb_configure() != cudaSuccess || attn_configure() != cudaSuccess ||
            step_configure() != cudaSuccess || qgemm_configure() != cudaSuccess) { cudaFree(s.err); s.err = nullptr; continue; }
        vbs_device_t &d = g_devices[g_ndev];
        memset(&d, 0, sizeof(d));
        snprintf(d.name, sizeof(d.name), "%s", pr.name);
        d.type = VBS_BACKEND_CUDA;
        d.max_working_set_bytes = tot;
        d.max_buffer_bytes = fr;
        d.internal_handle = &s;
        ++g_ndev;
    }
    cudaSetDevice(prev);
    g_ready = g_ndev > 0;
    snprintf(g_init_msg, sizeof(g_init_msg), "%s", g_ready ? "ok" : "no sm_100 (B200) device initialised");
    return g_ready;
}

int backend_device_count() { return g_ndev; }
DevState *backend_device(size_t i) { return i < (size_t)g_ndev ? &g_state[i] : nullptr; }

DevState *backend_current() {
    if (!do_init()) return nullptr;
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return nullptr;
    for (int i = 0; i < g_ndev; ++i)
        if (g_state[i].ordinal == cur) return &g_state[i];
    return nullptr;
}

static DevState *dev_of(vbs_device_t *dev) {
    if (!dev || !dev->internal_handle) return nullptr;
    DevState *s = static_cast<DevState *>(dev->internal_handle);
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != s->ordinal) cudaSetDevice(s->ordinal);
    return s;
}

bool check_device_error(DevState *d, cudaStream_t st) {
    if (!d) return false;
    uint32_t v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, d->err, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (!cuda_ok(e, "device synchronisation")) return false;
    if (v) {
        cudaMemsetAsync(d->err, 0, 4, st);
        latch_error("device kernel reported error 0x%x (%s)", v,
                    (v & (DERR_TIMEOUT_FULL | DERR_TIMEOUT_EMPTY | DERR_TIMEOUT_PEER)) ? "bounded wait expired"
                                                                                        : "invalid data");
        return false;
    }
    return true;
}

void *attn_workspace(DevState *d, size_t bytes) {
    if (d->attn_work_bytes >= bytes) return d->attn_work;
    if (d->attn_work) {
        cudaDeviceSynchronize();
        cudaFree(d->attn_work);
        d->attn_work = nullptr;
        d->attn_work_bytes = 0;
    }
    if (!cuda_ok(cudaMalloc(&d->attn_work, bytes), "attention workspace")) return nullptr;
    if (!cuda_ok(cudaMemset(d->attn_work, 0, bytes), "attention workspace")) return nullptr;
    d->attn_work_bytes = bytes;
    return d->attn_work;
}

void *qg_workspace(DevState *d, size_t bytes) {
    if (d->qg_work_bytes >= bytes) return d->qg_work;
    if (d->qg_work) {
        cudaDeviceSynchronize();
        cudaFree(d->qg_work);
        d->qg_work = nullptr;
        d->qg_work_bytes = 0;
    }
    if (!cuda_ok(cudaMalloc(&d->qg_work, bytes), "GEMM workspace")) return nullptr;
    d->qg_work_bytes = bytes;
    return d->qg_work;
}

bool gemm_x16_ok(int type, const void *w, uint32_t rows, uint32_t cols, uint32_t batch) {
    return batch > 8 && qgemm_supported(type, rows, cols, batch) && !(reinterpret_cast<uintptr_t>(w) & 15);
}

int gemm_x16(DevState *d, int type, const void *w, const __half *x16, float *y, uint32_t rows, uint32_t cols,
             uint32_t batch, uint32_t flags, cudaStream_t st) {
    QgemmParams p = {};
    p.w = static_cast<const uint8_t *>(w);
    p.rb = row_bytes(type, cols);
    p.rows = rows;
    p.cols = cols;
    p.tokens = batch;
    p.y = y;
    p.y_stride = rows;
    p.accumulate = (flags & VBS_CU_MV_ACCUMULATE) ? 1u : 0u;
    p.err = d->err;
    void *planes = nullptr;
    const size_t pb = qgemm_planes_bytes(rows, cols, batch, d->n_sm);
    if (pb && !(planes = qg_workspace(d, pb))) return -1;
    return cuda_ok(qgemm_launch_x16(type, p, x16, planes, d->n_sm, st), "GEMM launch") ? 0 : -1;
}

void *mvb_workspace(DevState *d, size_t bytes) {
    if (d->mvb_work_bytes >= bytes) return d->mvb_work;
    if (d->mvb_work) {
        cudaDeviceSynchronize();
        cudaFree(d->mvb_work);
        d->mvb_work = nullptr;
        d->mvb_work_bytes = 0;
    }
    if (!cuda_ok(cudaMalloc(&d->mvb_work, bytes), "batched matvec workspace")) return nullptr;
    d->mvb_work_bytes = bytes;
    return d->mvb_work;
}

// ---------------------------------------------------------------------------
// pipelines
// ---------------------------------------------------------------------------
struct Pipe {
    uint32_t magic;
    int kind;   // vbs_op_kind_t
    int type;   // weight type for LINEAR / EMBEDDING
};
constexpr uint32_t kPipeMagic = 0x56425342u;   // "VBSB"

static bool type_supported(int t) {
    return t == T_F32 || t == T_F16 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K;
}
// Weight types of linear tiles: the above plus LNS8, which the reference's
// bridge dispatches as a linear type (src/vbs_specializer_bridge.c:116-118)
// but has no embedding for (its self-test expects that refusal,
// src/vbs_backend_test.c:959-960).
static bool linear_type_supported(int t) { return type_supported(t) || t == T_LNS8; }

int matvec_any(DevState *d, int type, const uint8_t *w, const float *x, float *y, uint32_t rows, uint32_t cols,
               uint32_t batch, uint32_t flags, cudaStream_t st) {
    if (!linear_type_supported(type) || !w || !x || !y || !rows || !cols || !batch || cols % (uint32_t)block_elems(type)) {
        latch_error("matvec: invalid arguments (type %d, %ux%u, batch %u)", type, rows, cols, batch);
        return -1;
    }
    const void *wv[1] = {w};
    if (batch == 1 && !(flags & VBS_CU_MV_PORTABLE) && mv_fast_supported(type, rows, cols, wv, 1, x, 0)) {
        MvParams p = {};
        p.w[0] = p.w[1] = p.w[2] = w;
        p.seg_end[0] = p.seg_end[1] = p.seg_end[2] = rows;
        p.rb = row_bytes(type, cols);
        p.rows = rows;
        p.cols = cols;
        p.x = x;
        p.y = y;
        p.accumulate = (flags & VBS_CU_MV_ACCUMULATE) ? 1u : 0u;
        p.err = d->err;
        return cuda_ok(mv_fast_launch(type, 0, MV_EPI_STORE, p, d->n_sm, st, false, 0), "matvec launch") ? 0 : -1;
    }
    if (batch > 8 && !(flags & VBS_CU_MV_PORTABLE) && qgemm_supported(type, rows, cols, batch) &&
        !(reinterpret_cast<uintptr_t>(w) & 15)) {
        // many sequences (prompt chunks, large decode batches): the tcgen05 GEMM
        QgemmParams p = {};
        p.w = w;
        p.rb = row_bytes(type, cols);
        p.rows = rows;
        p.cols = cols;
        p.tokens = batch;
        p.y = y;
        p.y_stride = rows;
        p.accumulate = (flags & VBS_CU_MV_ACCUMULATE) ? 1u : 0u;
        p.err = d->err;
        void *work = qg_workspace(d, qgemm_workspace_bytes(rows, cols, batch, d->n_sm));
        if (!work) return -1;
        return cuda_ok(qgemm_launch(type, p, x, cols, work, d->n_sm, st), "GEMM launch") ? 0 : -1;
    }
    if (batch > 1 && !(flags & VBS_CU_MV_PORTABLE) && mvb_supported(type, rows, cols, batch, w, x)) {
        // batched decode on the tensor cores (mvb.cu)
        MvbParams p = {};
        p.w = w;
        p.rb = row_bytes(type, cols);
        p.rows = rows;
        p.cols = cols;
        p.batch = batch;
        p.x = x;
        p.x_stride = cols;
        p.y = y;
        p.y_stride = rows;
        p.accumulate = (flags & VBS_CU_MV_ACCUMULATE) ? 1u : 0u;
        p.err = d->err;
        float *work = nullptr;
        if (const size_t wb = mvb_workspace_bytes(type, rows, cols, batch)) {
            work = static_cast<float *>(mvb_workspace(d, wb));
            if (!work) return -1;
        }
        return cuda_ok(mvb_launch(type, p, work, d->n_sm, st), "batched matvec launch") ? 0 : -1;
    }
    return cuda_ok(mv_generic_launch(type, w, x, y, rows, cols, batch, cols, rows, (flags & VBS_CU_MV_ACCUMULATE) ? 1 : 0,
                                     d->n_sm, st),
                   "matvec launch")
               ? 0
               : -1;
}

}  // namespace vbs

using namespace vbs;

// ===========================================================================
// ops table
// ===========================================================================
extern "C" {

const char *vbs_cuda_last_error(void) {
    if (has_error()) return g_err_msg;
    return g_probed ? g_init_msg : "not probed yet";
}

static bool ops_init(void) { return do_init(); }
static size_t ops_get_device_count(void) { return (size_t)g_ndev; }
static vbs_device_t *ops_get_device(size_t i) { return i < (size_t)g_ndev ? &g_devices[i] : nullptr; }

static vbs_buffer_t *ops_alloc_buffer(vbs_device_t *dev, size_t bytes, bool shared) {
    DevState *d = dev_of(dev);
    if (!d) { latch_error("alloc_buffer: invalid device"); return nullptr; }
    const size_t padded = ((bytes ? bytes : 1) + 255) & ~(size_t)255;
    void *dp = nullptr;
    if (!cuda_ok(cudaMalloc(&dp, padded), "alloc_buffer")) return nullptr;
    vbs_buffer_t *b = static_cast<vbs_buffer_t *>(calloc(1, sizeof(vbs_buffer_t)));
    if (!b) { cudaFree(dp); return nullptr; }
    b->internal_handle = dp;
    b->size = bytes;
    b->device = dev;
    if (shared) {
        if (cudaMallocHost(&b->host_ptr, padded) != cudaSuccess) b->host_ptr = nullptr;
    } else if (bytes <= (64u << 20)) {
        b->host_ptr = calloc(1, padded);
    }
    if (shared && !b->host_ptr) {
        latch_error("alloc_buffer: pinned host staging of %zu bytes failed", bytes);
        cudaFree(dp);
        free(b);
        return nullptr;
    }
    return b;
}

static void ops_free_buffer(vbs_buffer_t *b) {
    if (!b) return;
    dev_of(b->device);
    cudaFree(b->internal_handle);
    if (b->host_ptr) {
        cudaPointerAttributes at;
        if (cudaPointerGetAttributes(&at, b->host_ptr) == cudaSuccess && at.type == cudaMemoryTypeHost)
            cudaFreeHost(b->host_ptr);
        else {
            cudaGetLastError();
            free(b->host_ptr);
        }
    }
    free(b);
}

static bool ops_copy_to_device(vbs_buffer_t *dst, const void *src, size_t bytes) {
    if (!dst || !dst->internal_handle || (!src && bytes)) { latch_error("copy_to_device: invalid arguments"); return false; }
    if (dst->size && bytes > dst->size) { latch_error("copy_to_device: %zu bytes into a %zu-byte buffer", bytes, dst->size); return false; }
    dev_of(dst->device);
    return cuda_ok(cudaMemcpy(dst->internal_handle, src, bytes, cudaMemcpyHostToDevice), "copy_to_device");
}

static bool ops_copy_to_host(void *dst, const vbs_buffer_t *src, size_t bytes) {
    if (!src || !src->internal_handle || (!dst && bytes)) { latch_error("copy_to_host: invalid arguments"); return false; }
    DevState *d = dev_of(src->device);
    if (d) check_device_error(d, 0);
    if (has_error()) {
        fprintf(stderr, "[VBS] CUDA backend error: %s\n", g_err_msg);
        return false;
    }
    return cuda_ok(cudaMemcpy(dst, src->internal_handle, bytes, cudaMemcpyDeviceToHost), "copy_to_host");
}

static void *ops_compile_linear_pipeline(vbs_device_t *dev, vbs_ggml_type_t type, char *err, size_t cap) {
    (void)dev;
    if (!linear_type_supported((int)type)) {
        if (err && cap) snprintf(err, cap, "CUDA linear pipeline refusal: no sm_100a kernel for weight type %d", (int)type);
        return nullptr;
    }
    Pipe *p = static_cast<Pipe *>(malloc(sizeof(Pipe)));
    if (!p) return nullptr;
    p->magic = kPipeMagic;
    p->kind = VBS_OP_LINEAR;
    p->type = (int)type;
    return p;
}

static vbs_prim_pipeline_t *make_prim(int kind, int type) {
    Pipe *n = static_cast<Pipe *>(malloc(sizeof(Pipe)));
    vbs_prim_pipeline_t *pp = static_cast<vbs_prim_pipeline_t *>(malloc(sizeof(vbs_prim_pipeline_t)));
    if (!n || !pp) { free(n); free(pp); return nullptr; }
    n->magic = kPipeMagic;
    n->kind = kind;
    n->type = type;
    pp->native = n;
    pp->kind = (vbs_op_kind_t)kind;
    return pp;
}

static void *ops_compile_embed_pipeline(vbs_device_t *dev, vbs_ggml_type_t type, char *err, size_t cap) {
    (void)dev;
    if (!type_supported((int)type)) {
        if (err && cap) snprintf(err, cap, "CUDA embedding pipeline refusal: no kernel for type %d", (int)type);
        return nullptr;
    }
    return make_prim(VBS_OP_EMBEDDING, (int)type);
}

static void *ops_compile_primitive_pipeline(vbs_device_t *dev, vbs_op_kind_t kind, char *err, size_t cap) {
    (void)dev;
    switch (kind) {
        case VBS_OP_EMBEDDING:
        case VBS_OP_NORMALIZE:
        case VBS_OP_ROTARY:
        case VBS_OP_CACHE:
        case VBS_OP_ATTENTION:
        case VBS_OP_ACTIVATION:
        case VBS_OP_ELEMENTWISE:
            return make_prim((int)kind, T_F32);
        default:
            if (err && cap) snprintf(err, cap, "CUDA has no primitive kernel for op kind %d", (int)kind);
            return nullptr;
    }
}

static bool ops_dispatch_linear_tile(vbs_device_t *dev, void *pipeline, vbs_buffer_t *wp, vbs_buffer_t *ws,
                                     size_t copied, vbs_buffer_t *in, vbs_buffer_t *out, uint32_t cols, uint32_t rows,
                                     uint32_t col_off, uint32_t row_off, bool accumulate) {
    DevState *d = dev_of(dev);
    const Pipe *p = static_cast<const Pipe *>(pipeline);
    if (!d || !p || p->magic != kPipeMagic || p->kind != VBS_OP_LINEAR || !in || !out || !in->internal_handle ||
        !out->internal_handle) {
        latch_error("dispatch_linear_tile: invalid pipeline or buffers");
        return false;
    }
    if (!rows || !cols) return true;
    const uint64_t need = row_bytes(p->type, cols) * rows;
    if (!need || cols % (uint32_t)block_elems(p->type)) {
        latch_error("dispatch_linear_tile: %u columns are not whole %d-element blocks", cols, block_elems(p->type));
        return false;
    }
    const uint8_t *w;
    if (ws) {
        // staged tile (slice executor): the packed tile sits in the stage
        // buffer's host mirror; move it to device memory first
        vbs_buffer_t *dstb = (wp && wp->internal_handle) ? wp : ws;
        const size_t bytes = copied ? copied : (size_t)need;
        if (!ws->host_ptr || bytes < need || (dstb->size && bytes > dstb->size)) {
            latch_error("dispatch_linear_tile: staged tile of %zu bytes does not fit (need %llu)", bytes,
                        (unsigned long long)need);
            return false;
        }
        if (!cuda_ok(cudaMemcpyAsync(dstb->internal_handle, ws->host_ptr, bytes, cudaMemcpyHostToDevice, 0), "stage copy"))
            return false;
        w = static_cast<const uint8_t *>(dstb->internal_handle);
    } else {
        if (!wp || !wp->internal_handle) { latch_error("dispatch_linear_tile: no weights"); return false; }
        w = static_cast<const uint8_t *>(wp->internal_handle);
    }
    const float *x = static_cast<const float *>(in->internal_handle) + col_off;
    float *y = static_cast<float *>(out->internal_handle) + row_off;
    return matvec_any(d, p->type, w, x, y, rows, cols, 1, accumulate ? VBS_CU_MV_ACCUMULATE : 0u, 0) == 0;
}

// Scalar / buffer argument readers for the canonical bridge order.
static bool arg_ptr(const vbs_arg_t *a, void **out) {
    if (a->tag != VBS_ARG_BUFFER || !a->value) return false;
    *out = const_cast<void *>(a->value);
    return true;
}
static bool arg_u32(const vbs_arg_t *a, uint32_t *out) {
    if (a->tag != VBS_ARG_SCALAR || !a->value || a->size != 4) return false;
    memcpy(out, a->value, 4);
    return true;
}
static bool arg_f32(const vbs_arg_t *a, float *out) {
    if (a->tag != VBS_ARG_SCALAR || !a->value || a->size != 4) return false;
    memcpy(out, a->value, 4);
    return true;
}

static bool ops_dispatch_primitive(vbs_device_t *dev, void *pipeline, const vbs_arg_t *args, size_t n, size_t grid_x,
                                   size_t block_x) {
    (void)grid_x;
    (void)block_x;
    DevState *d = dev_of(dev);
    const vbs_prim_pipeline_t *pp = static_cast<const vbs_prim_pipeline_t *>(pipeline);
    const Pipe *np = pp ? static_cast<const Pipe *>(pp->native) : nullptr;
    if (!d || !np || np->magic != kPipeMagic || !args) {
        latch_error("dispatch_primitive: invalid pipeline");
        return false;
    }
    bool ok = false;
    cudaError_t e = cudaSuccess;
    switch ((int)pp->kind) {
        case VBS_OP_EMBEDDING: {   // B w, S token, B out, S dim
            void *w, *o;
            uint32_t tok, dim;
            ok = n == 4 && arg_ptr(&args[0], &w) && arg_u32(&args[1], &tok) && arg_ptr(&args[2], &o) && arg_u32(&args[3], &dim);
            if (ok) e = embed_launch(np->type, static_cast<const uint8_t *>(w), nullptr, tok, 0xFFFFFFFFu, static_cast<float *>(o), dim, d->err, 0, false);
            break;
        }
        case VBS_OP_NORMALIZE: {   // B in, B w, B out, S dim, S eps
            void *in, *w, *o;
            uint32_t dim;
            float eps;
            ok = n == 5 && arg_ptr(&args[0], &in) && arg_ptr(&args[1], &w) && arg_ptr(&args[2], &o) && arg_u32(&args[3], &dim) &&
                 arg_f32(&args[4], &eps);
            if (ok) e = rmsnorm_launch(static_cast<const float *>(in), static_cast<const float *>(w), static_cast<float *>(o), dim, eps, 0);
            break;
        }
        case VBS_OP_ROTARY: {   // B x, S pos, S head_dim, S n_heads, S theta
            void *x;
            uint32_t pos, hd, nh;
            float th;
            ok = n == 5 && arg_ptr(&args[0], &x) && arg_u32(&args[1], &pos) && arg_u32(&args[2], &hd) && arg_u32(&args[3], &nh) &&
                 arg_f32(&args[4], &th);
            if (ok) e = rope_launch(static_cast<float *>(x), pos, nullptr, hd, nh, th, 0);
            break;
        }
        case VBS_OP_CACHE: {   // B k, B v, B kc, B vc, S pos, S layer, S max_ctx, S kv_dim
            void *k, *v, *kc, *vc;
            uint32_t pos, layer, mc, kvd;
            ok = n == 8 && arg_ptr(&args[0], &k) && arg_ptr(&args[1], &v) && arg_ptr(&args[2], &kc) && arg_ptr(&args[3], &vc) &&
                 arg_u32(&args[4], &pos) && arg_u32(&args[5], &layer) && arg_u32(&args[6], &mc) && arg_u32(&args[7], &kvd);
            ok = ok && pos < mc;
            if (ok)
                e = cache_store_launch(static_cast<const float *>(k), static_cast<const float *>(v), static_cast<uint16_t *>(kc),
                                       static_cast<uint16_t *>(vc), pos, nullptr, layer, mc, kvd, kvd, false, 0);
            break;
        }
        case VBS_OP_ATTENTION: {   // B q, B kc, B vc, B out, S seq_len, S layer, S max_ctx, S nqh, S nkh, S hd, S scale
            void *q, *kc, *vc, *o;
            AttnParams ap = {};
            ok = n == 11 && arg_ptr(&args[0], &q) && arg_ptr(&args[1], &kc) && arg_ptr(&args[2], &vc) && arg_ptr(&args[3], &o) &&
                 arg_u32(&args[4], &ap.seq_len) && arg_u32(&args[5], &ap.layer) && arg_u32(&args[6], &ap.max_ctx) &&
                 arg_u32(&args[7], &ap.nqh) && arg_u32(&args[8], &ap.nkh) && arg_u32(&args[9], &ap.hd) && arg_f32(&args[10], &ap.scale);
            ok = ok && ap.seq_len >= 1 && ap.seq_len <= ap.max_ctx;
            if (ok) {
                ap.q = static_cast<const float *>(q);
                ap.kc = static_cast<const uint16_t *>(kc);
                ap.vc = static_cast<const uint16_t *>(vc);
                ap.out = static_cast<float *>(o);
                ap.batch = 1;
                ap.err = d->err;
                const uint32_t ns = attn_num_splits(ap.seq_len, ap.nkh, 1, d->n_sm);
                ap.work = attn_workspace(d, attn_workspace_bytes(ap.nqh, ap.nkh, ap.hd, 1, ns));
                ok = ap.work != nullptr;
                if (ok) e = attn_launch(ap, ns, 0, false);
            }
            break;
        }
        case VBS_OP_ACTIVATION:
        case VBS_OP_ELEMENTWISE: {   // B a, B b, B out, S n
            void *a, *b, *o;
            uint32_t len;
            ok = n == 4 && arg_ptr(&args[0], &a) && arg_ptr(&args[1], &b) && arg_ptr(&args[2], &o) && arg_u32(&args[3], &len);
            if (ok)
                e = (pp->kind == VBS_OP_ACTIVATION)
                        ? silu_mul_launch(static_cast<const float *>(a), static_cast<const float *>(b), static_cast<float *>(o), len, 0)
                        : add_launch(static_cast<const float *>(a), static_cast<const float *>(b), static_cast<float *>(o), len, 0);
            break;
        }
        default:
            break;
    }
    if (!ok) {
        latch_error("dispatch_primitive: bad arguments for op kind %d (%zu args)", (int)pp->kind, n);
        return false;
    }
    return cuda_ok(e, "dispatch_primitive launch");
}

static void ops_synchronize(vbs_device_t *dev) {
    DevState *d = dev_of(dev);
    if (!d) return;
    cuda_ok(cudaDeviceSynchronize(), "synchronize_device");
    check_device_error(d, 0);
}

// The reference's Phase 2 hook (include/vbs_backend.h:94-98): `pipeline` is
// a vbs_cu_decoder_t of a model on `dev`, `control_buffer` holds the
// engine's vbs_gpu_control_t (include/vbs_engine.h:31-40). Generation runs on
// the device, steered by that block (vbs_cu_decoder_run_control).
static bool ops_launch_persistent_kernel(vbs_device_t *dev, void *pipeline, vbs_buffer_t *control) {
    DevState *d = dev_of(dev);
    if (!d || !pipeline || !control || !control->internal_handle || control->size < sizeof(vbs_gpu_control_t)) {
        latch_error("launch_persistent_kernel: needs a device, a decoder and a control buffer of %zu bytes",
                    sizeof(vbs_gpu_control_t));
        return false;
    }
    return vbs_cu_decoder_run_control(static_cast<vbs_cu_decoder_t *>(pipeline), control->internal_handle) == 0;
}

const vbs_backend_ops_t g_vbs_cuda_backend = {
    ops_init,
    ops_get_device_count,
    ops_get_device,
    ops_alloc_buffer,
    ops_free_buffer,
    ops_copy_to_device,
    ops_copy_to_host,
    ops_compile_linear_pipeline,
    ops_compile_embed_pipeline,
    ops_compile_primitive_pipeline,
    ops_dispatch_linear_tile,
    ops_dispatch_primitive,
    ops_synchronize,
    ops_launch_persistent_kernel,
};

// ===========================================================================
// extension entry points
// ===========================================================================

int vbs_cu_status(void) { return has_error() ? 1 : 0; }

void vbs_cu_clear_error(void) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_err_set.store(0);
    snprintf(g_err_msg, sizeof(g_err_msg), "ok");
    cudaGetLastError();
}

const char *vbs_cu_version(void) { return "vbs_b200 0.2 sm_100a cp.async mma.m16n8k32.s8 griddepcontrol cuda-graph nccl"; }

uint64_t vbs_cu_kernel_launches(void) { return g_launches.load(); }

int vbs_cu_dequant(int type, const void *w, float *out, uint64_t n, void *stream) {
    DevState *d = backend_current();
    if (!d) { latch_error("vbs_cu_dequant: no usable device"); return -1; }
    if (!linear_type_supported(type) || !w || !out || n % (uint64_t)block_elems(type)) {
        latch_error("vbs_cu_dequant: invalid arguments");
        return -1;
    }
    return cuda_ok(dequant_launch(type, static_cast<const uint8_t *>(w), out, n, static_cast<cudaStream_t>(stream)), "dequant") ? 0 : -1;
}

int vbs_cu_matvec(int type, const void *w, const float *x, float *y, uint32_t rows, uint32_t cols, uint32_t batch,
                  uint32_t flags, void *stream) {
    DevState *d = backend_current();
    if (!d) { latch_error("vbs_cu_matvec: no usable device"); return -1; }
    return matvec_any(d, type, static_cast<const uint8_t *>(w), x, y, rows, cols, batch, flags, static_cast<cudaStream_t>(stream));
}

int vbs_cu_ffn_gate_up(int type, const void *w_gate, const void *w_up, const float *x, const float *norm_w, float eps,
                       float *h, uint32_t rows, uint32_t cols, void *stream) {
    DevState *d = backend_current();
    if (!d) { latch_error("vbs_cu_ffn_gate_up: no usable device"); return -1; }
    if (!type_supported(type) || !w_gate || !w_up || !x || !h || !rows || !cols || cols % (uint32_t)block_elems(type)) {
        latch_error("vbs_cu_ffn_gate_up: invalid arguments");
        return -1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const void *wv[2] = {w_gate, w_up};
    if (mv_fast_supported(type, rows, cols, wv, 2, x, 1)) {
        MvParams p = {};
        p.w[0] = p.w[1] = p.w[2] = static_cast<const uint8_t *>(w_gate);
        p.seg_end[0] = p.seg_end[1] = p.seg_end[2] = rows;
        p.wb = static_cast<const uint8_t *>(w_up);
        p.rb = row_bytes(type, cols);
        p.rows = rows;
        p.cols = cols;
        p.x = x;
        p.norm_w = norm_w;
        p.eps = eps;
        p.y = h;
        p.err = d->err;
        return cuda_ok(mv_fast_launch(type, 1, MV_EPI_SILU, p, d->n_sm, st, false, 0), "ffn_gate_up launch") ? 0 : -1;
    }
    // portable sequence: norm, two matvecs, SiLU (scratch from the workspace)
    float *tmp = static_cast<float *>(attn_workspace(d, ((size_t)cols + 2 * (size_t)rows) * sizeof(float) + 256));
    if (!tmp) return -1;
    const float *xin = x;
    if (norm_w) {
        if (!cuda_ok(rmsnorm_launch(x, norm_w, tmp, cols, eps, st), "ffn norm")) return -1;
        xin = tmp;
    }
    float *g = tmp + cols, *u = g + rows;
    if (matvec_any(d, type, static_cast<const uint8_t *>(w_gate), xin, g, rows, cols, 1, 0, st)) return -1;
    if (matvec_any(d, type, static_cast<const uint8_t *>(w_up), xin, u, rows, cols, 1, 0, st)) return -1;
    return cuda_ok(silu_mul_launch(g, u, h, rows, st), "ffn silu") ? 0 : -1;
}

int vbs_cu_attention(const float *q, const uint16_t *kc, const uint16_t *vc, float *out, uint32_t seq_len, uint32_t layer,
                     uint32_t max_ctx, uint32_t nqh, uint32_t nkh, uint32_t hd, float scale, uint32_t batch,
                     uint64_t kv_batch_stride, void *stream) {
    // arguments first: a zero head count must not reach the split arithmetic
    if (!q || !kc || !vc || !out || !seq_len || seq_len > max_ctx || !batch || !nkh || !nqh || nqh % nkh) {
        latch_error("vbs_cu_attention: invalid arguments");
        return -1;
    }
    DevState *d = backend_current();
    if (!d) { latch_error("vbs_cu_attention: no usable device"); return -1; }
    AttnParams ap = {};
    ap.q = q; ap.kc = kc; ap.vc = vc; ap.out = out;
    ap.seq_len = seq_len; ap.layer = layer; ap.max_ctx = max_ctx;
    ap.nqh = nqh; ap.nkh = nkh; ap.hd = hd; ap.scale = scale;
    ap.batch = batch; ap.kv_batch_stride = kv_batch_stride; ap.err = d->err;
    const uint32_t ns = attn_num_splits(seq_len, nkh, batch, d->n_sm);
    ap.work = attn_workspace(d, attn_workspace_bytes(nqh, nkh, hd, batch, ns));
    if (!ap.work) return -1;
    return cuda_ok(attn_launch(ap, ns, static_cast<cudaStream_t>(stream), false), "attention") ? 0 : -1;
}


int vbs_cu_attention_static(const float *q, const uint16_t *kc, const uint16_t *vc, float *out, uint32_t seq_len,
                            uint32_t layer, uint32_t max_ctx, uint32_t nqh, uint32_t nkh, uint32_t hd, float scale,
                            uint32_t batch, uint64_t kv_batch_stride, void *stream) {
    // arguments first: a zero head count must not reach the split arithmetic
    if (!q || !kc || !vc || !out || !seq_len || seq_len > max_ctx || !batch || !nkh || !nqh || nqh % nkh) {
        latch_error("vbs_cu_attention_static: invalid arguments");
        return -1;
    }
    DevState *d = backend_current();
    if (!d) { latch_error("vbs_cu_attention_static: no usable device"); return -1; }
    if (!d->attn_static) {   // first call on this device: look the scratch up (its device is current here)
        void *ptr = nullptr;
        if (!cuda_ok(attn_static_address(&ptr), "vbs_cu_attention_static: scratch address")) return -1;
        d->attn_static = ptr;
    }
    // as many splits as the fixed scratch holds, never more than the allocating
    // entry point uses. One split writes its result straight to `out` and
    // touches neither the merge tickets nor the partials, so it always fits.
    uint32_t ns = attn_num_splits(seq_len, nkh, batch, d->n_sm);
    while (ns > 1 && attn_workspace_bytes(nqh, nkh, hd, batch, ns) > attn_static_bytes()) --ns;
    AttnParams ap = {};
    ap.q = q; ap.kc = kc; ap.vc = vc; ap.out = out;
    ap.seq_len = seq_len; ap.layer = layer; ap.max_ctx = max_ctx;
    ap.nqh = nqh; ap.nkh = nkh; ap.hd = hd; ap.scale = scale;
    ap.batch = batch; ap.kv_batch_stride = kv_batch_stride; ap.err = d->err;
    ap.work = d->attn_static;
    return cuda_ok(attn_launch(ap, ns, static_cast<cudaStream_t>(stream), false), "attention (static scratch)") ? 0 : -1;
}

int vbs_cu_synth(int type, void *dst, uint64_t rows, uint64_t cols, uint64_t row0, uint64_t col0, uint64_t full_cols,
                 uint64_t seed, float scale, void *stream) {
    DevState *d = backend_current();
    if (!d) { latch_error("vbs_cu_synth: no usable device"); return -1; }
    if (!dst) { latch_error("vbs_cu_synth: null destination"); return -1; }
    return cuda_ok(synth_launch(type, static_cast<uint8_t *>(dst), rows, cols, row0, col0, full_cols, seed, scale,
                                static_cast<cudaStream_t>(stream)),
                   "synth")
               ? 0
               : -1;
}

}  // extern "C"
