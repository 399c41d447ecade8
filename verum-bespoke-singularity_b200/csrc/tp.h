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
// A one-GPU exchange area for the step kernel's word instances: word slots,
// logits words and the exchange counter in this device's memory; the
// argmax leaves the plain logits in `logits`. The caller frees *mem and
// *comm with cudaFree (also after a false return).
bool tp_local_area(float *logits, void **mem, struct TpComm **comm);

}  // namespace vbs
