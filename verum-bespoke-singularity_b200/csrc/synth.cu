// synth.cu -- seeded synthetic weights, quantized on the device.
//
// Benchmark models (Llama-3-8B / 70B shapes, 4.8-39 GB packed) are
// generated in place instead of uploaded. Every value is a pure function of
// (seed, element index): the centred sum of four 16-bit uniforms from a
// splitmix64 hash (Irwin-Hall n = 4 approximation of a normal), times a
// float scale; the block quantizers use only IEEE basic operations and
// roundf. Built with -fmad=false and _rn intrinsics, the bytes are identical
// to oracle/vbs_oracle.c:orc_synth_tensor on the host. The quantizers are
// this project's own (the reference ships none for K-quants); the block
// layouts are GGUF's (src/vbs_dequant.c:174-179, :258-277, :316-333).
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vbs {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth_val(uint64_t seed, uint64_t idx, float scale) {
    const uint64_t h = mix64(seed + 0x9E3779B97F4A7C15ull * (idx + 1));
    const int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
                      (int32_t)(h >> 48);
    return __fmul_rn((float)(s - 131070), scale);
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ __forceinline__ void st16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

// One thread per block of the [rows x cols] tile.
__global__ void synth_kernel(int type, uint8_t *dst, uint64_t rows, uint64_t cols, uint64_t row0, uint64_t col0,
                             uint64_t full_cols, uint64_t seed, float scale) {
    const int E = block_elems(type), BB = block_bytes(type);
    const uint64_t nb_row = cols / (uint64_t)E, total = rows * nb_row;
    for (uint64_t bi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; bi < total;
         bi += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = bi / nb_row, cb = bi % nb_row;
        const uint64_t base = (row0 + r) * full_cols + col0 + cb * (uint64_t)E;
        uint8_t *o = dst + r * nb_row * (uint64_t)BB + cb * (uint64_t)BB;
        if (type == T_F32) {
            const float v = synth_val(seed, base, scale);
            const uint32_t u = __float_as_uint(v);
            o[0] = (uint8_t)u; o[1] = (uint8_t)(u >> 8); o[2] = (uint8_t)(u >> 16); o[3] = (uint8_t)(u >> 24);
        } else if (type == T_F16) {
            st16(o, f32_to_f16_rne(synth_val(seed, base, scale)));
        } else if (type == T_Q8_0) {
            float v[32], amax = 0.0f;
            for (int i = 0; i < 32; ++i) { v[i] = synth_val(seed, base + i, scale); amax = fmaxf(amax, fabsf(v[i])); }
            const uint16_t dh = f32_to_f16_rne(__fdiv_rn(amax, 127.0f));
            const float d = f16_exact(dh);
            st16(o, dh);
            for (int i = 0; i < 32; ++i)
                o[2 + i] = (uint8_t)(int8_t)(d > 0.0f ? clampi((int)roundf(__fdiv_rn(v[i], d)), -127, 127) : 0);
        } else if (type == T_Q4_K) {
            float scl[8], mins[8], smax = 0.0f, mmax = 0.0f;
            for (int j = 0; j < 8; ++j) {
                float lo = 0.0f, hi = synth_val(seed, base + j * 32, scale);
                for (int i = 0; i < 32; ++i) {
                    const float x = synth_val(seed, base + j * 32 + i, scale);
                    lo = fminf(lo, x);
                    hi = fmaxf(hi, x);
                }
                scl[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
                mins[j] = -lo;
                smax = fmaxf(smax, scl[j]);
                mmax = fmaxf(mmax, mins[j]);
            }
            const uint16_t dh = f32_to_f16_rne(__fdiv_rn(smax, 63.0f)), mh = f32_to_f16_rne(__fdiv_rn(mmax, 63.0f));
            const float d = f16_exact(dh), dmin = f16_exact(mh);
            int sc[8], mn[8];
            for (int j = 0; j < 8; ++j) {
                sc[j] = d > 0.0f ? clampi((int)roundf(__fdiv_rn(scl[j], d)), 0, 63) : 0;
                mn[j] = dmin > 0.0f ? clampi((int)roundf(__fdiv_rn(mins[j], dmin)), 0, 63) : 0;
            }
            st16(o, dh);
            st16(o + 2, mh);
            for (int j = 0; j < 4; ++j) {
                o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
                o[8 + j] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
                o[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
            }
            for (int G = 0; G < 4; ++G) {
                const int ja = 2 * G, jb = 2 * G + 1;
                const float sa = __fmul_rn(d, (float)sc[ja]), oa = __fmul_rn(dmin, (float)mn[ja]);
                const float sb = __fmul_rn(d, (float)sc[jb]), ob = __fmul_rn(dmin, (float)mn[jb]);
                for (int i = 0; i < 32; ++i) {
                    const float xa = synth_val(seed, base + ja * 32 + i, scale);
                    const float xb = synth_val(seed, base + jb * 32 + i, scale);
                    const int qa = sa > 0.0f ? clampi((int)roundf(__fdiv_rn(__fadd_rn(xa, oa), sa)), 0, 15) : 0;
                    const int qb = sb > 0.0f ? clampi((int)roundf(__fdiv_rn(__fadd_rn(xb, ob), sb)), 0, 15) : 0;
                    o[16 + G * 32 + i] = (uint8_t)(qa | (qb << 4));
                }
            }
        } else if (type == T_Q6_K) {
            float gs[16], smax = 0.0f;
            for (int g = 0; g < 16; ++g) {
                float amax = 0.0f;
                for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(synth_val(seed, base + g * 16 + i, scale)));
                gs[g] = __fdiv_rn(amax, 31.0f);
                smax = fmaxf(smax, gs[g]);
            }
            const uint16_t dh = f32_to_f16_rne(__fdiv_rn(smax, 127.0f));
            const float d = f16_exact(dh);
            for (int i = 0; i < 192; ++i) o[i] = 0;
            for (int g = 0; g < 16; ++g) {
                const int sc = d > 0.0f ? clampi((int)roundf(__fdiv_rn(gs[g], d)), 0, 127) : 0;
                o[192 + g] = (uint8_t)(int8_t)sc;
                const float step = __fmul_rn(d, (float)sc);
                for (int i = 0; i < 16; ++i) {
                    const int e = g * 16 + i;
                    const float x = synth_val(seed, base + e, scale);
                    const int q = step > 0.0f ? clampi((int)roundf(__fdiv_rn(x, step)), -32, 31) : 0;
                    const int u = q + 32;
                    const int half = e >> 7, quarter = (e >> 5) & 3, l = e & 31;
                    o[half * 64 + (quarter & 1) * 32 + l] |= (uint8_t)((u & 15) << ((quarter >> 1) * 4));
                    o[128 + half * 32 + l] |= (uint8_t)((u >> 4) << (quarter * 2));
                }
            }
            st16(o + 208, dh);
        }
    }
}

cudaError_t synth_launch(int type, uint8_t *dst, uint64_t rows, uint64_t cols, uint64_t row0, uint64_t col0,
                         uint64_t full_cols, uint64_t seed, float scale, cudaStream_t st) {
    if (type != T_F32 && type != T_F16 && type != T_Q8_0 && type != T_Q4_K && type != T_Q6_K) return cudaErrorInvalidValue;
    if (cols % (uint64_t)block_elems(type)) return cudaErrorInvalidValue;
    const uint64_t total = rows * (cols / (uint64_t)block_elems(type));
    if (!total) return cudaSuccess;
    const uint64_t blocks = std::min<uint64_t>((total + 127) / 128, 148ull * 64);
    note_launches(1);
    synth_kernel<<<(unsigned)blocks, 128, 0, st>>>(type, dst, rows, cols, row0, col0, full_cols, seed, scale);
    return cudaGetLastError();
}

}  // namespace vbs
