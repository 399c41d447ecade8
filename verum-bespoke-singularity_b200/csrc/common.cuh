// common.cuh -- shared device/host helpers for the sm_100a decode backend.
//
// Block formats follow the GGUF layouts the reference decodes in
// src/vbs_dequant.c (Q8_0 :174-179, Q4_K :258-277, Q6_K :316-333); the
// fp16 converters restate src/vbs_dequant.c:21-74 and src/vbs_cpu.c:71-91
// bit for bit, because the KV store and the strict-parity path must
// produce the reference's exact halves.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace vbs {

// GGML type ids (include/vbs_gguf.h:13-48).
// LNS8 (40) is the reference's own log-scaled 8-bit type (src/vbs_gguf.c:35).
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_LNS8 = 40 };

__host__ __device__ inline int block_elems(int t) {
    switch (t) {
        case T_F32: case T_F16: return 1;
        case T_Q4_0: case T_Q4_1: case T_Q8_0: case T_LNS8: return 32;
        case T_Q4_K: case T_Q6_K: return 256;
        default: return 0;
    }
}
__host__ __device__ inline int block_bytes(int t) {
    switch (t) {
        case T_F32: return 4;
        case T_F16: return 2;
        case T_Q4_0: return 18;
        case T_Q4_1: return 20;
        case T_Q8_0: return 34;
        case T_Q4_K: return 144;
        case T_Q6_K: return 210;
        case T_LNS8: return 36;
        default: return 0;
    }
}
__host__ __device__ inline uint64_t row_bytes(int t, uint64_t cols) {
    int e = block_elems(t);
    return e ? cols / (uint64_t)e * (uint64_t)block_bytes(t) : 0;
}

// ---------------------------------------------------------------------------
// error reporting
// ---------------------------------------------------------------------------

// Device-side error word (one per device, allocated by the backend and
// passed to every kernel that can fail): kernels that give up a bounded
// wait or meet an invalid argument OR a code in and return; the host reads
// it at the next synchronisation point.
enum : uint32_t { DERR_TIMEOUT_FULL = 1u, DERR_TIMEOUT_EMPTY = 2u, DERR_TIMEOUT_PEER = 4u, DERR_BAD_ARG = 8u };

__device__ inline void dev_flag_error(uint32_t *err, uint32_t code) {
    if (err) atomicOr(err, code);
}

// ---------------------------------------------------------------------------
// fp16 helpers (exact restatements)
// ---------------------------------------------------------------------------

// binary16 -> binary32, exact, NaN payload kept (src/vbs_dequant.c:21-44).
__device__ __forceinline__ float f16_exact(uint32_t h) {
    uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t bits;
    if (e == 31u) bits = s | 0x7F800000u | (m << 13);
    else if (e) bits = s | ((e + 112u) << 23) | (m << 13);
    else if (!m) bits = s;
    else {
        int k = __clz(m) - 21;                      // shifts until bit 10 is set
        bits = s | ((uint32_t)(113 - k) << 23) | (((m << k) & 1023u) << 13);
    }
    return __uint_as_float(bits);
}

// binary16 -> binary32 for finite data in hot loops (hardware convert).
__device__ __forceinline__ float f16f(uint32_t h) {
    return __half2float(__ushort_as_half((unsigned short)h));
}

// binary32 -> binary16 with the KV-store rounding of src/vbs_dequant.c:46-74.
__device__ __forceinline__ uint16_t f32_to_f16_kv(float f) {
    uint32_t x = __float_as_uint(f);
    uint32_t s = (x >> 16) & 0x8000u, be = (x >> 23) & 255u, m = x & 0x7FFFFFu;
    if (be == 255u) return (uint16_t)(s | 0x7C00u | (m ? 1u : 0u));
    int e = (int)be - 112;
    if (e >= 31) return (uint16_t)(s | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)s;
        uint32_t full = m | 0x800000u, sh = (uint32_t)(14 - e);
        uint32_t q = (full + (1u << (sh - 1))) >> sh;
        return (uint16_t)(s | (q >= 0x400u ? 0x400u : q));
    }
    uint32_t r = m + 0xFFFu + ((m >> 13) & 1u);
    if (r & 0x800000u) { r = 0; e++; }
    if (e >= 31) return (uint16_t)(s | 0x7C00u);
    return (uint16_t)(s | ((uint32_t)e << 10) | (r >> 13));
}

// binary32 -> binary16, nearest-even everywhere (src/vbs_cpu.c:71-91).
__device__ __forceinline__ uint16_t f32_to_f16_rne(float f) {
    uint32_t x = __float_as_uint(f);
    uint32_t s = (x >> 16) & 0x8000u;
    int e = (int)((x >> 23) & 255u) - 127;
    uint32_t m = x & 0x7FFFFFu;
    if (e > 15) return (uint16_t)(s | 0x7C00u);
    if (e >= -14) {
        uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13), rem = m & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(s | h);
    }
    if (e < -25) return (uint16_t)s;
    m |= 0x800000u;
    int sh = -e - 1;
    uint32_t h = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(s | h);
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// ---------------------------------------------------------------------------
// exact element dequantization (same float operation order as the
// reference; callers compile with FMA contraction disabled or rely on the
// explicit _rn intrinsics used here)
// ---------------------------------------------------------------------------

// Value of element e (0 <= e < block_elems) of one block.
__device__ __forceinline__ float dq_elem(int type, const uint8_t *b, int e) {
    switch (type) {
        case T_F32: { uint32_t v = ld_u16(b) | (ld_u16(b + 2) << 16); return __uint_as_float(v); }
        case T_F16: return f16_exact(ld_u16(b));
        case T_Q8_0: return __fmul_rn(f16_exact(ld_u16(b)), (float)(int8_t)b[2 + e]);
        case T_Q4_0: {
            int n = (e < 16) ? (b[2 + e] & 15) : (b[2 + e - 16] >> 4);
            return __fmul_rn(__fsub_rn((float)n, 8.0f), f16_exact(ld_u16(b)));
        }
        case T_Q4_1: {
            int n = (e < 16) ? (b[4 + e] & 15) : (b[4 + e - 16] >> 4);
            return __fadd_rn(__fmul_rn(f16_exact(ld_u16(b)), (float)n), f16_exact(ld_u16(b + 2)));
        }
        case T_Q4_K: {
            const uint8_t *s = b + 4;
            int j = e >> 5, sc, mn;
            if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
            else { sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
            uint8_t q = b[16 + (j >> 1) * 32 + (e & 31)];
            int nib = (j & 1) ? (q >> 4) : (q & 15);
            float a = __fmul_rn(f16_exact(ld_u16(b)), (float)sc);
            float c = __fmul_rn(f16_exact(ld_u16(b + 2)), (float)mn);
            return __fsub_rn(__fmul_rn(a, (float)nib), c);
        }
        case T_Q6_K: {
            int h = e >> 7, q = (e >> 5) & 3, l = e & 31;
            int lo = (b[h * 64 + (q & 1) * 32 + l] >> ((q >> 1) * 4)) & 15;
            int hi = (b[128 + h * 32 + l] >> (q * 2)) & 3;
            float ds = __fmul_rn(f16_exact(ld_u16(b + 208)), (float)(int8_t)b[192 + (e >> 4)]);
            return __fmul_rn(ds, (float)((lo | (hi << 4)) - 32));
        }
        case T_LNS8: {   // value = 2^q * scale (src/vbs_host_math.h:111-121); 2^q built exactly, +inf from q = 128
            const uint32_t q = b[e];
            const float p2 = q < 128u ? __uint_as_float((q + 127u) << 23) : __uint_as_float(0x7F800000u);
            return __fmul_rn(p2, __uint_as_float(ld_u16(b + 32) | (ld_u16(b + 34) << 16)));
        }
        default: return 0.0f;
    }
}

// ---------------------------------------------------------------------------
// PTX wrappers: shared-memory addresses, mbarriers, bulk copies, PDL, mma
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

// Wait for phase `parity` of a barrier, giving up after `limit_ns` of
// global time. Returns false on timeout (the caller records the error and
// skips its work; it never spins forever).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > limit_ns) return false;
    }
    return true;
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map, no multicast).
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// The same with an L2 cache policy (createpolicy), e.g. evict_first for a
// stream that is read once, so it does not displace what is read again.
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Programmatic dependent launch: wait for the upstream grid's memory, and
// allow the downstream grid to start its prologue. Both are no-ops when the
// launch carries no programmatic dependency.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3) : "r"(addr));
}

// C += A(16x16 f16) * B(16x8 f16), fp32 accumulators.
__device__ __forceinline__ void mma_f16_acc(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16-byte global -> shared copy; src_bytes < 16 fills the rest with zeros
// (0: nothing is read, the destination is zeroed).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes = 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// D = A(16x32, unsigned bytes) * B(32x8, signed bytes), int32, no accumulate-in.
__device__ __forceinline__ void mma_u8s8(const uint32_t a[4], uint32_t b0, uint32_t b1, int c[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_s8s8(const uint32_t a[4], uint32_t b0, uint32_t b1, int c[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// 4 bytes from a shared address that is only 2-byte aligned.
__device__ __forceinline__ uint32_t lds_u32_any(uint32_t addr) {
    uint32_t base = addr & ~3u, lo, hi;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(lo) : "r"(base));
    if ((addr & 3u) == 0) return lo;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(hi) : "r"(base + 4));
    return __funnelshift_r(lo, hi, (addr & 3u) * 8);
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds_u128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds_u64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Bounded-wait budget for all device spins (2 s of global time).
constexpr uint64_t kWaitNs = 2000000000ull;

}  // namespace vbs
