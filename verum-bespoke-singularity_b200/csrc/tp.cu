// tp.cu -- tensor parallelism over NVLink / NVSwitch.
//
// One process per GPU. Rank 0 creates an NCCL unique id
// (vbs_cu_tp_unique_id), the host side broadcasts it (the tests and
// bench.py use torch.distributed's store), every rank joins with
// vbs_cu_tp_init. The decode program then sums the o_proj and down_proj
// partials (dim floats, 16 KB for the 8B shape) across the ranks twice per
// layer and all-gathers the sharded logits. The reference has no multi-GPU
// path (its engine binds one device, src/vbs_engine.c:142-169).
//
// The per-layer sums do not go through NCCL: the writing matvec stores its
// rows straight into every peer's receive region over NVLink (CUDA IPC
// mappings of each rank's region, exchanged here with one NCCL all-gather
// of the handles). The per-op kernels then publish a flag, which the next
// kernel's prologue waits for before it sums the slots; the persistent step
// kernel stores each value with its exchange index in one 64-bit word,
// which the reader checks word by word (TpComm, kernels.h). NCCL's
// all-reduce stays available as the reference collective
// (VBS_CU_DEC_TP_NCCL).
#include "vbs_b200.h"
#include "backend.h"
#include "kernels.h"
#include "tp.h"

#include <nccl.h>
#include <cstring>
#include <vector>

namespace vbs {

static ncclComm_t g_comm = nullptr;
static int g_world = 1, g_rank = 0;

// the peer-memory exchange
static void *g_region = nullptr;              // this rank's receive region
static void *g_peer_base[TP_MAX_WORLD] = {};  // IPC mappings of the peers' regions
static TpComm *g_comm_dev = nullptr;          // device copy of the TpComm
constexpr size_t TP_SLOT_BYTES_PER_RANK = 2ull * TP_DIM_MAX * 4;   // two slot sets of one sender

// region: [slot sets 2 x world x TP_DIM_MAX][logits TP_VOCAB_MAX][flags | seq | ticket]
//         [word slot sets 2 x world x TP_DIM_MAX][logits words TP_VOCAB_MAX]
static size_t logits_offset(int world) { return TP_SLOT_BYTES_PER_RANK * world; }
static size_t flags_offset(int world) { return logits_offset(world) + (size_t)TP_VOCAB_MAX * 4; }
static size_t ll_offset(int world) { return flags_offset(world) + 1024; }
static size_t ll_logits_offset(int world) { return ll_offset(world) + 2 * TP_SLOT_BYTES_PER_RANK * world; }
static size_t region_bytes(int world) { return ll_logits_offset(world) + (size_t)TP_VOCAB_MAX * 8; }

const TpComm *tp_comm() { return g_comm_dev; }
float *tp_own_logits() {
    return g_comm_dev ? reinterpret_cast<float *>(static_cast<uint8_t *>(g_region) + logits_offset(g_world)) : nullptr;
}

static void p2p_teardown() {
    for (int q = 0; q < TP_MAX_WORLD; ++q)
        if (g_peer_base[q]) { cudaIpcCloseMemHandle(g_peer_base[q]); g_peer_base[q] = nullptr; }
    if (g_comm_dev) { cudaFree(g_comm_dev); g_comm_dev = nullptr; }
    if (g_region) { cudaFree(g_region); g_region = nullptr; }
}

// Every rank: allocate and clear the region, all-gather the IPC handles,
// map the peers' regions. Returns false (with the error latched) when the
// mapping is impossible; the decoders then use NCCL for the sums.
static bool p2p_setup(int rank, int world) {
    const size_t bytes = region_bytes(world);
    if (!cuda_ok(cudaMalloc(&g_region, bytes), "tp region") || !cuda_ok(cudaMemset(g_region, 0, bytes), "tp region"))
        return false;
    cudaIpcMemHandle_t mine;
    if (!cuda_ok(cudaIpcGetMemHandle(&mine, g_region), "tp ipc handle")) return false;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    uint8_t *dh = nullptr;
    if (!cuda_ok(cudaMalloc(&dh, 64 * (world + 1)), "tp handles")) return false;
    std::vector<uint8_t> all(64 * world);
    bool ok = cuda_ok(cudaMemcpy(dh + 64 * world, &mine, 64, cudaMemcpyHostToDevice), "tp handles");
    if (ok) {
        const ncclResult_t r = ncclAllGather(dh + 64 * world, dh, 64, ncclUint8, g_comm, 0);
        if (r != ncclSuccess) { latch_error("ncclAllGather (handles): %s", ncclGetErrorString(r)); ok = false; }
    }
    ok = ok && cuda_ok(cudaStreamSynchronize(0), "tp handles") &&
         cuda_ok(cudaMemcpy(all.data(), dh, 64 * world, cudaMemcpyDeviceToHost), "tp handles");
    cudaFree(dh);
    if (!ok) return false;
    TpComm c = {};
    c.world = (uint32_t)world;
    c.rank = (uint32_t)rank;
    for (int q = 0; q < world; ++q) {
        uint8_t *base = nullptr;
        if (q == rank) {
            base = static_cast<uint8_t *>(g_region);
        } else {
            cudaIpcMemHandle_t h;
            memcpy(&h, all.data() + 64 * q, 64);
            void *pp = nullptr;
            if (!cuda_ok(cudaIpcOpenMemHandle(&pp, h, cudaIpcMemLazyEnablePeerAccess), "tp ipc open")) return false;
            g_peer_base[q] = pp;
            base = static_cast<uint8_t *>(pp);
        }
        c.slots[q] = reinterpret_cast<float *>(base);
        c.logits[q] = reinterpret_cast<float *>(base + logits_offset(world));
        c.flags[q] = reinterpret_cast<uint32_t *>(base + flags_offset(world));
        c.ll[q] = reinterpret_cast<uint64_t *>(base + ll_offset(world));
        c.ll_logits[q] = reinterpret_cast<uint64_t *>(base + ll_logits_offset(world));
    }
    uint8_t *own = static_cast<uint8_t *>(g_region) + flags_offset(world);
    c.seq = reinterpret_cast<uint32_t *>(own + 512);
    c.ticket = reinterpret_cast<uint32_t *>(own + 768);
    return cuda_ok(cudaMalloc(&g_comm_dev, sizeof(TpComm)), "tp comm") &&
           cuda_ok(cudaMemcpy(g_comm_dev, &c, sizeof(TpComm), cudaMemcpyHostToDevice), "tp comm");
}

bool tp_local_area(float *logits, void **mem, TpComm **comm) {
    *mem = nullptr;
    *comm = nullptr;
    const size_t words = 2ull * TP_DIM_MAX * 8, lw = (size_t)TP_VOCAB_MAX * 8;
    uint8_t *base = nullptr;
    if (!cuda_ok(cudaMalloc((void **)&base, words + lw + 128), "word area")) return false;
    *mem = base;
    if (!cuda_ok(cudaMemset(base, 0, words + lw + 128), "word area")) return false;
    TpComm c = {};
    c.world = 1;
    c.rank = 0;
    c.ll[0] = reinterpret_cast<uint64_t *>(base);
    c.ll_logits[0] = reinterpret_cast<uint64_t *>(base + words);
    c.logits[0] = logits;
    c.seq = reinterpret_cast<uint32_t *>(base + words + lw);
    return cuda_ok(cudaMalloc((void **)comm, sizeof(TpComm)), "word area") &&
           cuda_ok(cudaMemcpy(*comm, &c, sizeof(TpComm), cudaMemcpyHostToDevice), "word area");
}

int tp_world() { return g_comm ? g_world : 1; }
int tp_rank() { return g_comm ? g_rank : 0; }

bool tp_allreduce_sum(float *buf, size_t n, cudaStream_t st) {
    if (!g_comm) return true;
    ncclResult_t r = ncclAllReduce(buf, buf, n, ncclFloat32, ncclSum, g_comm, st);
    if (r != ncclSuccess) { latch_error("ncclAllReduce: %s", ncclGetErrorString(r)); return false; }
    return true;
}

bool tp_allgather(const float *local, float *full, size_t n_local, cudaStream_t st) {
    if (!g_comm) return cuda_ok(cudaMemcpyAsync(full, local, n_local * 4, cudaMemcpyDeviceToDevice, st), "allgather");
    ncclResult_t r = ncclAllGather(local, full, n_local, ncclFloat32, g_comm, st);
    if (r != ncclSuccess) { latch_error("ncclAllGather: %s", ncclGetErrorString(r)); return false; }
    return true;
}

}  // namespace vbs

using namespace vbs;

extern "C" {

int vbs_cu_tp_unique_id(void *out128) {
    if (!out128) return -1;
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) { latch_error("ncclGetUniqueId: %s", ncclGetErrorString(r)); return -1; }
    static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
    memcpy(out128, &id, 128);
    return 0;
}

int vbs_cu_tp_init(int rank, int world, const void *id128) {
    if (g_comm) { latch_error("vbs_cu_tp_init: already initialised"); return -1; }
    if (!id128 || world < 1 || rank < 0 || rank >= world) { latch_error("vbs_cu_tp_init: invalid arguments"); return -1; }
    if (!backend_current()) { latch_error("vbs_cu_tp_init: no usable device"); return -1; }
    if (world == 1) return 0;
    ncclUniqueId id;
    memcpy(&id, id128, 128);
    ncclResult_t r = ncclCommInitRank(&g_comm, world, id, rank);
    if (r != ncclSuccess) { g_comm = nullptr; latch_error("ncclCommInitRank: %s", ncclGetErrorString(r)); return -1; }
    g_world = world;
    g_rank = rank;
    if (world > TP_MAX_WORLD || !p2p_setup(rank, world)) {
        // no peer-memory exchange: the decoders sum with NCCL instead
        p2p_teardown();
        cudaGetLastError();
        vbs_cu_clear_error();
    }
    return 0;
}

int vbs_cu_tp_finalize(void) {
    if (!g_comm) return 0;
    cudaDeviceSynchronize();
    p2p_teardown();
    ncclResult_t r = ncclCommDestroy(g_comm);
    g_comm = nullptr;
    g_world = 1;
    g_rank = 0;
    if (r != ncclSuccess) { latch_error("ncclCommDestroy: %s", ncclGetErrorString(r)); return -1; }
    return 0;
}

}  // extern "C"
