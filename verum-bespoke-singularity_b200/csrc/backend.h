// backend.h -- state shared between the ops-table implementation
// (backend.cu) and the decode program (decoder.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace vbs {

struct DevState {
    int ordinal = -1;
    int n_sm = 0;
    uint32_t *err = nullptr;        // device error word (see common.cuh)
    void *attn_work = nullptr;      // shared split-KV workspace for the ops table / vbs_cu_attention
    size_t attn_work_bytes = 0;
    void *attn_static = nullptr;    // address of the fixed scratch of vbs_cu_attention_static
    void *mvb_work = nullptr;       // chunk planes of the batched matvec
    size_t mvb_work_bytes = 0;
    void *qg_work = nullptr;        // fp16 copy of X for the tcgen05 GEMM
    size_t qg_work_bytes = 0;
};

// Devices usable by this library (sm_100). Index = position in the ops
// table's device list; ordinal = CUDA device ordinal.
int backend_device_count();
DevState *backend_device(size_t index);
// DevState of the calling thread's current CUDA device (initialising the
// backend if needed); NULL when that device is not usable.
DevState *backend_current();

// Sticky error: the first message wins until vbs_cu_clear_error().
void latch_error(const char *fmt, ...);
bool has_error();
// Latch and return false when e != cudaSuccess.
bool cuda_ok(cudaError_t e, const char *what);
// Read (and clear) the device error word of `d`; latch when nonzero.
bool check_device_error(DevState *d, cudaStream_t st);

// Grow the device's shared attention workspace to `bytes` (zeroed).
void *attn_workspace(DevState *d, size_t bytes);
// Grow the device's batched-matvec plane workspace to `bytes`.
void *mvb_workspace(DevState *d, size_t bytes);
// Grow the device's GEMM activation workspace to `bytes`.
void *qg_workspace(DevState *d, size_t bytes);
// Prompt chunks: one matrix on activations already converted by
// qgemm_to_half (one input, several matrices). gemm_x16_ok: the GEMM takes it.
bool gemm_x16_ok(int type, const void *w, uint32_t rows, uint32_t cols, uint32_t batch);
int gemm_x16(DevState *d, int type, const void *w, const __half *x16, float *y, uint32_t rows, uint32_t cols,
             uint32_t batch, uint32_t flags, cudaStream_t st);
// y[b] (+)= W x[b] for b < batch on `st`, through the kernel the shape and
// type allow (fast, batched tensor-core, the tcgen05 GEMM above 8
// sequences, or portable); flags VBS_CU_MV_*.
// 0, or -1 with the error latched.
int matvec_any(DevState *d, int type, const uint8_t *w, const float *x, float *y, uint32_t rows, uint32_t cols,
               uint32_t batch, uint32_t flags, cudaStream_t st);

}  // namespace vbs
