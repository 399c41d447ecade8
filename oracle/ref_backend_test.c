/* ref_backend_test.c -- runs the reference's own backend self-test body
 * against this library's ops table.
 *
 * TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file against the
 * UNMODIFIED reference sources (-I <reference>/src) into
 * oracle/_ref/cuda-backend-test, linked with libvbs_b200.so in place of the
 * reference's src/vbs_backend_cuda.c. The reference runs its full suite,
 * test_one_backend (src/vbs_backend_test.c:456-963), only for the CPU,
 * Vulkan and HIP tables and gives CUDA a smoke check
 * (src/vbs_backend_test.c:1135-1147); including the file here reaches that
 * static function and runs every one of its checks on g_vbs_cuda_backend.
 * Exit status: 0 all checks passed, 1 some failed, 2 no usable device.
 */
#include "vbs_backend_test.c"

int main(void) {
    if (!g_vbs_cuda_backend.init()) {
        printf("CUDA backend unavailable: %s\n", vbs_cuda_last_error());
        return 2;
    }
    test_one_backend("CUDA", &g_vbs_cuda_backend);
    printf("cuda backend suite: %d checks, %d failures\n", g_checks, g_fails);
    return g_fails ? 1 : 0;
}
