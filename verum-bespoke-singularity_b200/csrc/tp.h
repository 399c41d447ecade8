// tp.h -- tensor-parallel collectives used by the decode program.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace vbs {

int tp_world();   // 1 when no TP group has been joined
int tp_rank();
// In-place sum of n floats across the group, enqueued on `st`.
bool tp_allreduce_sum(float *buf, size_t n, cudaStream_t st);
// full[r * n_local .. +n_local) = rank r's `local`.
bool tp_allgather(const float *local, float *full, size_t n_local, cudaStream_t st);
// The peer-memory exchange region (device pointer), or NULL when the group
// has none (one rank, or peers not mappable).
const struct TpComm *tp_comm();
// This rank's full-logits area in its exchange region (the step kernel
// gathers the vocab shards there), or NULL.
float *tp_own_logits();

}  // namespace vbs
