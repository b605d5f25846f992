// pkv_common.cuh -- shared device helpers for the PrismKV sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/prismkv_b200.h"

#define PKV_MAX_BITS 8          // per component
#define PKV_MAX_TOTAL_BITS 16   // per code
#define PKV_NUM_SMS_B200 148

namespace pkv {

// Device error word: set when a bounded wait expires; read by pkv_device_error.
__device__ int32_t g_device_error = 0;   // single definition: the library is one translation unit

// 4: a split-sequence exchange waited past its bound for the other ranks' outputs
// 5: a kernel found its dynamic shared window at another address than its layout assumes
enum : int32_t { kErrWaitFull = 1, kErrWaitEmpty = 2, kErrWaitDrain = 3, kErrPeerWait = 4, kErrSmemLayout = 5 };

__device__ __forceinline__ void flag_error(int32_t code) { atomicCAS(&g_device_error, 0, code); }

// ---------------------------------------------------------------------------
// element loads
// ---------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<PKV_F32> {
    using T = float;
    static __device__ __forceinline__ float load(const T* p) { return __ldg(p); }
    static __device__ __forceinline__ void store(T* p, float v) { *p = v; }
};
template <> struct Elem<PKV_BF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float load(const T* p) { return __bfloat162float(__ldg(p)); }
    static __device__ __forceinline__ void store(T* p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct Elem<PKV_F16> {
    using T = __half;
    static __device__ __forceinline__ float load(const T* p) { return __half2float(__ldg(p)); }
    static __device__ __forceinline__ void store(T* p, float v) { *p = __float2half_rn(v); }
};

template <int CB> struct Code;
template <> struct Code<1> {
    using T = uint8_t;
    static __device__ __forceinline__ uint32_t load(const T* p) { return __ldg(p); }
    static __device__ __forceinline__ void store(T* p, uint32_t v) { *p = (T)v; }
};
template <> struct Code<2> {
    using T = uint16_t;
    static __device__ __forceinline__ uint32_t load(const T* p) { return __ldg(p); }
    static __device__ __forceinline__ void store(T* p, uint32_t v) { *p = (T)v; }
};
template <> struct Code<8> {
    using T = int64_t;
    static __device__ __forceinline__ uint32_t load(const T* p) { return (uint32_t)__ldg(p); }
    static __device__ __forceinline__ void store(T* p, uint32_t v) { *p = (T)v; }
};

// Count of ascending thresholds t[0..n-1] with v >= t[i]  (branch-free
// binary search; n = 2^bits - 1, so the search runs `bits` steps).  NaN
// compares false everywhere and yields 0.
__device__ __forceinline__ int count_ge(const float* t, int bits, float v) {
    int lo = 0;  // answer in [lo, lo + 2^k)
    #pragma unroll 1
    for (int k = bits - 1; k >= 0; --k) {
        int probe = lo + (1 << k);         // candidate count; threshold index probe-1
        lo = (v >= t[probe - 1]) ? probe : lo;
    }
    return lo;
}

// The same count, branch-free, when the true count lies within 2 of `guess`:
// every threshold below the window counts and none above it does, so the count
// is the window's base plus its four comparisons.  NaN yields 0 (all compares
// false, and a NaN guess is 0).
__device__ __forceinline__ int count_ge_window(const float* t, int n, float v, int guess) {
    const int base = min(max(guess - 2, 0), n);
    int c = base;
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int b = base + i;
        const float tb = t[min(b, n - 1)];
        c += (b < n && v >= tb) ? 1 : 0;
    }
    return c;
}

// Binary-search count with a fixed, unrolled step count (bits <= 8), predicated
// rather than branched, so independent searches interleave.
__device__ __forceinline__ int count_ge_unrolled(const float* t, int bits, float v) {
    int lo = 0;
    #pragma unroll
    for (int k = 7; k >= 0; --k) {
        if (k < bits) {
            const int probe = lo + (1 << k);
            lo = (v >= t[probe - 1]) ? probe : lo;
        }
    }
    return lo;
}

// The same count from a first guess: `guess` is any integer (a linear
// interpolation of the thresholds is exact up to one step for uniform bins);
// the loops move it to the unique g with t[g-1] <= v < t[g].  NaN yields 0.
__device__ __forceinline__ int count_ge_from(const float* t, int n, float v, int guess) {
    int g = min(max(guess, 0), n);
    if (g > 0 && !(v >= t[g - 1])) {
        do { --g; } while (g > 0 && !(v >= t[g - 1]));
    } else {
        while (g < n && v >= t[g]) ++g;
    }
    return g;
}

// ---------------------------------------------------------------------------
// mbarrier / bulk-copy PTX (sm_90+), with bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    // suspends the thread in hardware until the phase completes or ~20 us pass
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(20000u) : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete.  Gives up after `limit`
// suspended polls (about 20 us each, so ~2.6 s by default), sets the device
// error word and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t err,
                                          uint32_t limit = (1u << 17)) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    flag_error(err);
    return false;
}

// The same wait without a suspend-time hint: try_wait returns after a short
// hardware-defined interval, so the phase is seen sooner (tensor-core commits
// arrive in bursts); the bound is counted in polls (~2^22, a few seconds).
__device__ __forceinline__ bool mbar_try_wait_spin(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int32_t err,
                                               uint32_t limit = (1u << 22)) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait_spin(bar, parity)) return true;
    flag_error(err);
    return false;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// dst, src 16-byte aligned; bytes a multiple of 16.
// Pull one 128-byte line into L2 ahead of its use (no register result, no wait).
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" :: "l"(ptr));
}

// Ask `bytes` (a multiple of 16, 16-byte aligned) of global memory into L2; nothing waits on it.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// paired fp32 arithmetic on sm_100 with both values in one 64-bit register: the operands keep
// that form from load to store, so no instruction splits or rebuilds the register pair
// ---------------------------------------------------------------------------
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 f2_pack(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ float2 f2_unpack(f32x2 v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}

__device__ __forceinline__ f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ f32x2 f2_add(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ f32x2 f2_mul(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// 16 bytes of shared memory as two pairs; 8 bytes as one pair.
__device__ __forceinline__ void lds_f2x2(uint32_t addr, f32x2& a, f32x2& b) {
    asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

__device__ __forceinline__ f32x2 lds_f2(uint32_t addr) {
    f32x2 v;
    asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace pkv
