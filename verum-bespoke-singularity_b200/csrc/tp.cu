// tp.cu -- tensor parallelism over NVLink / NVSwitch with NCCL.
//
// One process per GPU. Rank 0 creates an NCCL unique id
// (vbs_cu_tp_unique_id), the host side broadcasts it (the tests and
// bench.py use torch.distributed's store), every rank joins with
// vbs_cu_tp_init. The decode program then all-reduces the o_proj and
// down_proj partial sums (dim floats, 16 KB for the 8B shape) and
// all-gathers the sharded logits. The reference has no multi-GPU path (its
// engine binds one device, src/vbs_engine.c:142-169).
#include "vbs_b200.h"
#include "backend.h"
#include "tp.h"

#include <nccl.h>
#include <cstring>

namespace vbs {

static ncclComm_t g_comm = nullptr;
static int g_world = 1, g_rank = 0;

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
    return 0;
}

int vbs_cu_tp_finalize(void) {
    if (!g_comm) return 0;
    ncclResult_t r = ncclCommDestroy(g_comm);
    g_comm = nullptr;
    g_world = 1;
    g_rank = 0;
    if (r != ncclSuccess) { latch_error("ncclCommDestroy: %s", ncclGetErrorString(r)); return -1; }
    return 0;
}

}  // extern "C"
