/* abi_layout.c -- prints the layout of the ops-table types.
 *
 * TEST INFRASTRUCTURE ONLY. Built twice by oracle/Makefile: once against
 * the reference's include/vbs_backend.h (oracle/_ref/abi-layout-ref) and
 * once against this library's include/vbs_b200.h (oracle/abi-layout), so a
 * test can compare every offset and size of the two definitions. The
 * engine calls through these structs (include/vbs_backend.h:24-99) and
 * hands launch_persistent_kernel its control block (include/vbs_engine.h:
 * 31-40), so they must agree field for field.
 */
#ifdef LAYOUT_OF_REFERENCE
#include "vbs_backend.h"
#include "vbs_engine.h"
#else
#include "vbs_b200.h"
#endif
#include <stddef.h>
#include <stdio.h>

#define TYPE(T) printf("sizeof %s %zu align %zu\n", #T, sizeof(T), _Alignof(T))
#define FIELD(T, f) printf("%s.%s %zu %zu\n", #T, #f, offsetof(T, f), sizeof(((T *)0)->f))

int main(void) {
    TYPE(vbs_device_t);
    FIELD(vbs_device_t, name); FIELD(vbs_device_t, type); FIELD(vbs_device_t, max_working_set_bytes);
    FIELD(vbs_device_t, max_buffer_bytes); FIELD(vbs_device_t, internal_handle);
    TYPE(vbs_buffer_t);
    FIELD(vbs_buffer_t, internal_handle); FIELD(vbs_buffer_t, host_ptr); FIELD(vbs_buffer_t, size);
    FIELD(vbs_buffer_t, device);
    TYPE(vbs_arg_t);
    FIELD(vbs_arg_t, tag); FIELD(vbs_arg_t, value); FIELD(vbs_arg_t, size);
    TYPE(vbs_prim_pipeline_t);
    FIELD(vbs_prim_pipeline_t, native); FIELD(vbs_prim_pipeline_t, kind);
    TYPE(vbs_backend_ops_t);
    FIELD(vbs_backend_ops_t, init); FIELD(vbs_backend_ops_t, get_device_count); FIELD(vbs_backend_ops_t, get_device);
    FIELD(vbs_backend_ops_t, alloc_buffer); FIELD(vbs_backend_ops_t, free_buffer);
    FIELD(vbs_backend_ops_t, copy_to_device); FIELD(vbs_backend_ops_t, copy_to_host);
    FIELD(vbs_backend_ops_t, compile_linear_pipeline); FIELD(vbs_backend_ops_t, compile_embed_pipeline);
    FIELD(vbs_backend_ops_t, compile_primitive_pipeline); FIELD(vbs_backend_ops_t, dispatch_linear_tile);
    FIELD(vbs_backend_ops_t, dispatch_primitive); FIELD(vbs_backend_ops_t, synchronize_device);
    FIELD(vbs_backend_ops_t, launch_persistent_kernel);
    TYPE(vbs_gpu_control_t);
    FIELD(vbs_gpu_control_t, state); FIELD(vbs_gpu_control_t, current_token); FIELD(vbs_gpu_control_t, position);
    FIELD(vbs_gpu_control_t, max_tokens); FIELD(vbs_gpu_control_t, vocab_size); FIELD(vbs_gpu_control_t, eos_token_id);
    FIELD(vbs_gpu_control_t, generated_tokens_dev); FIELD(vbs_gpu_control_t, logits_dev);
    printf("VBS_PGAE_GENERATE %d VBS_PGAE_EXIT %d VBS_PGAE_EOS_NONE %u\n", (int)VBS_PGAE_GENERATE, (int)VBS_PGAE_EXIT,
           (unsigned)VBS_PGAE_EOS_NONE);
    /* enum values the engine passes across the boundary */
    printf("VBS_GGML_TYPE_Q4_K %d VBS_GGML_TYPE_Q6_K %d VBS_GGML_TYPE_Q8_0 %d VBS_GGML_TYPE_F32 %d\n",
           (int)VBS_GGML_TYPE_Q4_K, (int)VBS_GGML_TYPE_Q6_K, (int)VBS_GGML_TYPE_Q8_0, (int)VBS_GGML_TYPE_F32);
    printf("VBS_OP_ATTENTION %d VBS_OP_CACHE %d VBS_OP_PROJECTION %d VBS_BACKEND_CUDA %d VBS_ARG_SCALAR %d\n",
           (int)VBS_OP_ATTENTION, (int)VBS_OP_CACHE, (int)VBS_OP_PROJECTION, (int)VBS_BACKEND_CUDA,
           (int)VBS_ARG_SCALAR);
    return 0;
}
