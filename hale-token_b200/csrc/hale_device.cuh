// hale_device.cuh -- device helpers shared by the kernels.
//
// Exactness rules used throughout (they make the GPU results bit-identical
// to the Rust reference's CPU arithmetic):
//   * f32 products and sums use __fmul_rn / __fadd_rn, which the compiler
//     never contracts into FMAs (Rust never emits FMA contraction);
//   * float division and sqrt are the IEEE-rounded forms (nvcc's default
//     -prec-div=true -prec-sqrt=true; the build never passes fast-math);
//   * exp is hale_expf below, a restatement of glibc's expf;
//   * f32 -> i8 / i32 casts saturate and send NaN to 0, like Rust `as`.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#ifndef HALE_HD
#define HALE_HD __host__ __device__ __forceinline__
#endif

namespace hale {

// ---------------------------------------------------------------------------
// exp: glibc's expf, restated.
//
// glibc (since 2.28) computes expf with the method published by Szabolcs
// Nagy in ARM's optimized-routines: x*N/ln2 = k + r with N = 32, the table
// value 2^(k/N) and a cubic polynomial in r, all in double precision. On
// x86-64 glibc selects a build compiled with FMA, where the compiler fuses
// the multiply-adds; the fused steps below follow that build. The result is
// bit-identical to this machine's glibc expf for every one of the 2^32 float
// inputs (tests/test_capi_cpu.py checks the whole range against the oracle's
// libm), which is what makes softmax and SiLU match the reference exactly.
// ---------------------------------------------------------------------------
// 2^(i/32) as correctly rounded double bits, i = 0..31.
#define HALE_EXP2_TAB                                                                         \
    {0x3ff0000000000000ull, 0x3ff059b0d3158574ull, 0x3ff0b5586cf9890full,                    \
     0x3ff11301d0125b51ull, 0x3ff172b83c7d517bull, 0x3ff1d4873168b9aaull,                    \
     0x3ff2387a6e756238ull, 0x3ff29e9df51fdee1ull, 0x3ff306fe0a31b715ull,                    \
     0x3ff371a7373aa9cbull, 0x3ff3dea64c123422ull, 0x3ff44e086061892dull,                    \
     0x3ff4bfdad5362a27ull, 0x3ff5342b569d4f82ull, 0x3ff5ab07dd485429ull,                    \
     0x3ff6247eb03a5585ull, 0x3ff6a09e667f3bcdull, 0x3ff71f75e8ec5f74ull,                    \
     0x3ff7a11473eb0187ull, 0x3ff82589994cce13ull, 0x3ff8ace5422aa0dbull,                    \
     0x3ff93737b0cdc5e5ull, 0x3ff9c49182a3f090ull, 0x3ffa5503b23e255dull,                    \
     0x3ffae89f995ad3adull, 0x3ffb7f76f2fb5e47ull, 0x3ffc199bdd85529cull,                    \
     0x3ffcb720dcef9069ull, 0x3ffd5818dcfba487ull, 0x3ffdfc97337b9b5full,                    \
     0x3ffea4afa2a490daull, 0x3fff50765b6e4540ull}

__device__ const uint64_t kExp2TabDev[32] = HALE_EXP2_TAB;
static const uint64_t kExp2TabHost[32] = HALE_EXP2_TAB;

HALE_HD uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
    return u;
#endif
}
HALE_HD float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}
HALE_HD uint64_t d2u(double d) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u;
    __builtin_memcpy(&u, &d, 8);
    return u;
#endif
}
HALE_HD double u2d(uint64_t u) {
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)u);
#else
    double d;
    __builtin_memcpy(&d, &u, 8);
    return d;
#endif
}
HALE_HD double dfma(double a, double b, double c) {
#ifdef __CUDA_ARCH__
    return __fma_rn(a, b, c);
#else
    return __builtin_fma(a, b, c);
#endif
}
HALE_HD double dmul(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dmul_rn(a, b);
#else
    return a * b;
#endif
}

// exp with the 2^(i/32) table read from `tab` (device code may pass a copy
// in shared memory); hale_expf below uses the built-in table.
HALE_HD float hale_expf_tab(float x, const uint64_t* tab) {
    // Polynomial and scaling constants of the published method (N = 32).
    const double kInvLn2N = 0x1.71547652b82fep+0 * 32;
    const double kShift = 0x1.8p+52;
    const double kC0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
    const double kC1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
    const double kC2 = 0x1.62e42ff0c52d6p-1 / 32;
    uint32_t ux = f2u(x);
    uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                         // |x| >= 88 or NaN
        if (ux == 0xff800000u) return 0.0f;         // -inf
        if (abstop >= 0x7f8u) return x + x;         // inf / NaN
        if (x > 0x1.62e42ep6f) return u2f(0x7f800000u);   // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;              // underflow
    }
    double xd = (double)x;
    double kd = dfma(kInvLn2N, xd, kShift);
    uint64_t ki = d2u(kd);
    kd -= kShift;
    double r = dfma(kInvLn2N, xd, -kd);
    uint64_t t = tab[ki & 31];
    // 2^(k/32) = 2^(i/32) * 2^(k div 32): add k div 32 to the exponent field.
    t += (ki >> 5) << 52;
    double s = u2d(t);
    double z = dfma(kC0, r, kC1);
    double r2 = dmul(r, r);
    double y = dfma(kC2, r, 1.0);
    y = dfma(z, r2, y);
    y = dmul(y, s);
#ifdef __CUDA_ARCH__
    return __double2float_rn(y);
#else
    return (float)y;
#endif
}

HALE_HD float hale_expf(float x) {
#ifdef __CUDA_ARCH__
    return hale_expf_tab(x, kExp2TabDev);
#else
    return hale_expf_tab(x, kExp2TabHost);
#endif
}

#ifdef __CUDACC__
// ---------------------------------------------------------------------------
// f32 arithmetic in the reference's order (no contraction)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// ops::silu (src/ops/activation.rs:5-7): v / (1 + exp(-v)).
__device__ __forceinline__ float silu(float v) { return fdiv(v, fadd(1.0f, hale_expf(-v))); }

// Rust `f as i8`.
__device__ __forceinline__ int sat_i8(float f) {
    if (f != f) return 0;
    if (f >= 127.0f) return 127;
    if (f <= -128.0f) return -128;
    return (int)f;
}

// f32::total_cmp order key (larger key = larger float in IEEE total order).
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// ---------------------------------------------------------------------------
// device error word (per context): kernels OR bits in, the host reads it
// ---------------------------------------------------------------------------
enum : uint32_t { kErrTimeout = 1u, kErrBounds = 2u };

__device__ __forceinline__ void raise_error(uint32_t* err, uint32_t bit) {
    if (err) atomicOr(err, bit);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA engine, plain per-CTA loads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Global -> shared bulk copy completing on `bar`. dst, src 16-byte aligned;
// bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that may suspend the thread in hardware until the phase completes
// or `ns` nanoseconds pass, so waiting warps stop taking issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after ~`budget` clock cycles (well above any real
// copy latency), raising kErrTimeout. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err,
                                          long long budget = 4000000000LL) {
    if (mbar_try_wait(bar, parity)) return true;
    long long start = clock64();
    while (!mbar_try_wait_sleep(bar, parity, 1000000u)) {
        if (clock64() - start > budget) {
            raise_error(err, kErrTimeout);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------------------
// warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max_abs(float v) {
    // fold(0.0, |m, v| m.max(v.abs())): max is order-independent, NaN ignored
    float m = fmaxf(0.0f, fabsf(v));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
#endif  // __CUDACC__

}  // namespace hale
