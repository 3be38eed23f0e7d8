// oxide_common.cuh -- device helpers shared by every oxide kernel (sm_100a).
//
// Arithmetic that must match the reference's Rust f32 semantics goes through
// the explicitly rounded intrinsics below (__fmul_rn, __fadd_rn, __fsub_rn,
// __fdiv_rn, __fsqrt_rn).  nvcc never contracts those into an FMA and never
// replaces the IEEE divide by a reciprocal-multiply, so each step rounds
// exactly as the corresponding Rust expression does.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "oxide_ops.h"

namespace oxide {

typedef uint16_t bf16_t;  // raw bf16 bits (high half of an f32)

// ---------------------------------------------------------------------------
// IEEE-rounded scalar arithmetic (no contraction)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }

// ---------------------------------------------------------------------------
// bf16 <-> f32
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f32(bf16_t h) { return __uint_as_float((uint32_t)h << 16); }

// Round two floats to bf16 (nearest-even) and pack: lo in bits 0..15.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ bf16_t f32_to_bf16(float f) {
    __nv_bfloat16 v = __float2bfloat16_rn(f);
    return *reinterpret_cast<bf16_t*>(&v);
}
// Round-trip through bf16: the value a bf16 tensor store would hold.
__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// ---------------------------------------------------------------------------
// 128-bit global memory access
// ---------------------------------------------------------------------------
// Streaming read of data touched once: read-only path, no L1 allocation, L2
// prefetch of the surrounding 256 B sector group.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
// Read of small operands reused by many threads (weights, tables, masks).
__device__ __forceinline__ uint4 ld_keep(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}
// Streaming write (evict-first in L2).
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// ---------------------------------------------------------------------------
// Per-thread asynchronous 16-byte copies global -> shared (cp.async, L1
// bypass).  A thread that later reads only the vectors it copied itself needs
// no barrier: cp.async.wait_group makes its own completed copies visible to it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds16(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
    return v;
}

// A 16-byte vector viewed as V floats (V = 4 for f32, 8 for bf16).
template <typename T>
struct Vec;

template <>
struct Vec<float> {
    static constexpr int N = 4;
    __device__ __forceinline__ static void unpack(uint4 v, float* f) {
        f[0] = __uint_as_float(v.x);
        f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z);
        f[3] = __uint_as_float(v.w);
    }
    __device__ __forceinline__ static uint4 pack(const float* f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                          __float_as_uint(f[3]));
    }
    // Value a store of this dtype would hold (identity for f32).
    __device__ __forceinline__ static float rnd(float f) { return f; }
    __device__ __forceinline__ static float load1(const float* p) { return __ldg(p); }
    __device__ __forceinline__ static void store1(float* p, float f) { *p = f; }
};

template <>
struct Vec<bf16_t> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void unpack(uint4 v, float* f) {
        f[0] = bf16_lo(v.x);
        f[1] = bf16_hi(v.x);
        f[2] = bf16_lo(v.y);
        f[3] = bf16_hi(v.y);
        f[4] = bf16_lo(v.z);
        f[5] = bf16_hi(v.z);
        f[6] = bf16_lo(v.w);
        f[7] = bf16_hi(v.w);
    }
    __device__ __forceinline__ static uint4 pack(const float* f) {
        return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                          pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
    }
    __device__ __forceinline__ static float rnd(float f) { return round_bf16(f); }
    __device__ __forceinline__ static float load1(const bf16_t* p) {
        return bf16_to_f32(__ldg(reinterpret_cast<const unsigned short*>(p)));
    }
    __device__ __forceinline__ static void store1(bf16_t* p, float f) { *p = f32_to_bf16(f); }
};

// ---------------------------------------------------------------------------
// Division by a divisor shared by a whole row (RMSNorm's rms, softmax's sum),
// rounded exactly like the IEEE quotient a / b.  Markstein's method: with
// y = RN(1/b) (the correctly rounded reciprocal), q0 = RN(a*y) lies within a
// few ulps of a/b; each correction q' = RN(q + RN(a - q*b) * y) (two FMAs)
// shrinks the error, and once q is within one ulp of a/b the correction
// returns RN(a/b) (P. Markstein, IBM J. Res. Dev. 34(1), 1990; the same
// residual step as in the IA-64 division sequences).  Two corrections are
// applied.  The residuals must stay normal numbers, so the fast path holds for
// a positive divisor b in [2^-60, 2^60] (checked once per row; otherwise every
// element takes the IEEE divide) and for numerators with |a| in
// [lo, hi] = [2^-100 max(1, b), 2^100 min(1, b)], which keeps |a|, the
// quotient and the residuals normal.  fast2() raises `redo` for a pair with a
// numerator outside (zero, tiny, huge, inf, NaN); callers redo that vector
// with the IEEE divide -- the callers' quotients are bounded (|x / rms| <=
// sqrt(cols), e / sum <= 1), so in practice only underflowing exponentials
// and exact zeros get there.  Two quotients at a time on Blackwell's paired
// f32 pipe (__fmul2_rn / __ffma2_rn: IEEE round-to-nearest per lane), so a
// quotient costs 2.5 FMA-pipe instructions plus a compare.
// oxide_selftest_rowdiv checks operator() against __fdiv_rn, all subnormal
// numerators included.
// ---------------------------------------------------------------------------
struct RowDiv {
    float b, y, lo, hi;
    bool ieee;  // divisor outside the fast path's range: IEEE divide
    __device__ __forceinline__ explicit RowDiv(float bb) : b(bb) {
        y = __frcp_rn(bb);
        ieee = !(bb >= 0x1p-60f && bb <= 0x1p60f);
        lo = 0x1p-100f * fmaxf(1.0f, bb);
        hi = 0x1p100f * fminf(1.0f, bb);
    }
    __device__ __forceinline__ float2 fast2(float2 a, bool& redo) const {
        const float2 y2 = make_float2(y, y), nb = make_float2(-b, -b);
        const float2 q0 = __fmul2_rn(a, y2);
        float2 q = __ffma2_rn(__ffma2_rn(q0, nb, a), y2, q0);
        q = __ffma2_rn(__ffma2_rn(q, nb, a), y2, q);
        const float ax = fabsf(a.x), ay = fabsf(a.y);
        redo |= !((fminf(ax, ay) >= lo) & (fmaxf(ax, ay) <= hi));
        return q;
    }
    __device__ __forceinline__ float operator()(float a) const {
        if (ieee) return __fdiv_rn(a, b);
        bool redo = false;
        const float q = fast2(make_float2(a, a), redo).x;
        return redo ? __fdiv_rn(a, b) : q;
    }
};

// Paired f32 arithmetic (IEEE round-to-nearest per lane, no contraction).
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// ---------------------------------------------------------------------------
// Unsigned 32-bit division by a run-time constant (multiply-high + shift).
// For divisor d >= 1: s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1,
// q = (umulhi(n, m) + n) >> s, exact for every n < 2^32.
// ---------------------------------------------------------------------------
struct FastDiv {
    uint32_t d, m, s;
    __host__ __device__ FastDiv() : d(1), m(0), s(0) {}
    __host__ explicit FastDiv(uint32_t div) : d(div) {
        s = 0;
        while ((1ull << s) < div) ++s;
        m = (uint32_t)((((1ull << s) - div) << 32) / div + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        uint64_t t = (uint64_t)__umulhi(n, m) + n;
        return (uint32_t)(t >> s);
    }
    __device__ __forceinline__ uint32_t mod(uint32_t n) const { return n - div(n) * d; }
};

// ---------------------------------------------------------------------------
// e^x rounded to f32, for parity with a correctly rounded host expf (glibc's,
// which the reference's f32::exp calls).
//
// exp_rn_f32 evaluates e^x in f32 float-float arithmetic and checks, with
// Ziv's rounding test (A. Ziv, ACM TOMS 17(3), 1991), that the f32 nearest
// to the approximation is the f32 nearest to e^x; on the rare inputs where
// that cannot be decided (about 1 in 10^4) it calls exp_rn_f32_dp, the same
// reduction in double, after an exception list of the 17 inputs the double
// evaluation cannot resolve.  The result is the correctly rounded e^x for
// every float.  Every step of both is an IEEE f32 or f64 operation
// written out explicitly (no contraction), so the host compilation of these
// functions returns the device's bits (tests/test_exp_rn.py runs it over
// every float).
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ double exp_dfma(double a, double b, double c) {
#ifdef __CUDA_ARCH__
    return __fma_rn(a, b, c);
#else
    return __builtin_fma(a, b, c);
#endif
}
__host__ __device__ __forceinline__ double exp_bits_double(uint64_t b) {
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)b);
#else
    double d;
    __builtin_memcpy(&d, &b, 8);
    return d;
#endif
}
__host__ __device__ __forceinline__ uint64_t exp_double_bits(double d) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t b;
    __builtin_memcpy(&b, &d, 8);
    return b;
#endif
}
// f32 operations with one rounding each, the same on host and device.
__host__ __device__ __forceinline__ float exp_ffma(float a, float b, float c) {
#ifdef __CUDA_ARCH__
    return __fmaf_rn(a, b, c);
#else
    return __builtin_fmaf(a, b, c);
#endif
}
__host__ __device__ __forceinline__ float exp_fadd(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fadd_rn(a, b);
#else
    volatile float s = a + b;  // volatile: never contracted with a product
    return s;
#endif
}
__host__ __device__ __forceinline__ float exp_fsub(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fsub_rn(a, b);
#else
    volatile float s = a - b;
    return s;
#endif
}
__host__ __device__ __forceinline__ float exp_fmul(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    volatile float s = a * b;
    return s;
#endif
}
__host__ __device__ __forceinline__ int exp_f2i(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_int(f);
#else
    int i;
    __builtin_memcpy(&i, &f, 4);
    return i;
#endif
}
__host__ __device__ __forceinline__ float exp_i2f(int i) {
#ifdef __CUDA_ARCH__
    return __int_as_float(i);
#else
    float f;
    __builtin_memcpy(&f, &i, 4);
    return f;
#endif
}

// 2^(j/N) for j in [0, N): the nearest doubles.
template <int N>
__host__ __device__ __forceinline__ double exp_table(int j) {
    if (N == 1) return 1.0;
    if (N == 4) {
        const double a = (j & 1) ? 0x1.306fe0a31b715p+0 : 1.0;                  // 2^(1/4) : 1
        const double b = (j & 1) ? 0x1.ae89f995ad3adp+0 : 0x1.6a09e667f3bcdp+0;  // 2^(3/4) : 2^(1/2)
        return (j & 2) ? b : a;
    }
    // N == 8
    const double a = (j & 1) ? 0x1.172b83c7d517bp+0 : 1.0;
    const double b = (j & 1) ? 0x1.4bfdad5362a27p+0 : 0x1.306fe0a31b715p+0;
    const double c = (j & 1) ? 0x1.8ace5422aa0dbp+0 : 0x1.6a09e667f3bcdp+0;
    const double d = (j & 1) ? 0x1.d5818dcfba487p+0 : 0x1.ae89f995ad3adp+0;
    const double lo = (j & 2) ? b : a, hi = (j & 2) ? d : c;
    return (j & 4) ? hi : lo;
}

// The double path: the table-driven reduction of P. T. P. Tang (ACM TOMS
// 15(2), 1989) with an N-entry table, in double with fused multiply-adds:
// x = (kN + j) ln2 / N + r with k N + j = round(x N / ln2), |r| <= ln2 / (2N);
// e^x = 2^k * 2^(j/N) * e^r, e^r from its Taylor series to the degree D that
// keeps the truncation below 2^-43 (N = 1: D = 10; N = 4: D = 7; N = 8:
// D = 6), Horner in double; 2^(j/N) is the nearest double (picked by
// selects, no memory access) and 2^k goes into its exponent field; the
// product is rounded once to f32.  The result is RN(e^x) except where e^x
// lies within ~2^-43 (relative) of a rounding boundary between two floats
// (17 of the 2^32 inputs, listed in exp_rn_f32_hard).  |x| is clamped to 110 first, beyond the f32
// overflow (88.73) and underflow (-103.98) points; NaN propagates.
template <int N = 4>
__host__ __device__ __forceinline__ float exp_rn_f32_dp(float x) {
    static_assert(N == 1 || N == 4 || N == 8, "table sizes 1, 4, 8");
    // N / ln 2 and ln 2 / N: the nearest doubles (N a power of two, so only
    // the exponent differs from 1 / ln 2 and ln 2)
    const double kInv = 0x1.71547652b82fep+0 * N;
    const double kLn2 = 0x1.62e42fefa39efp-1 / N;
    const double kLn2Lo = 0x1.abc9e3b39803fp-56 / N;  // ln 2 / N - kLn2 (used for N = 1)
    const double kShift = 0x1.8p52;                    // 1.5 * 2^52: rounds to an integer in the low bits
    double xd = (double)x;
    xd = xd < -110.0 ? -110.0 : xd;  // comparisons are false for NaN: it passes through
    xd = xd > 110.0 ? 110.0 : xd;
    const double t = exp_dfma(xd, kInv, kShift);
    const double kd = t - kShift;  // round(x N / ln 2)
    const int kj = (int)(uint32_t)exp_double_bits(t);
    // r = x - kd ln2 / N: one fused step is exact to |kd| * 2^-53 ln2 / N
    // <= 2^-46 for N >= 4; N = 1 (|kd| <= 159) adds the low part of ln 2.
    double r = exp_dfma(-kd, kLn2, xd);
    if (N == 1) r = exp_dfma(-kd, kLn2Lo, r);
    double p;
    if (N == 1) {  // 1/n!, n = 10 .. 2: the nearest doubles
        p = 0x1.27e4fb7789f5cp-22;
        p = exp_dfma(p, r, 0x1.71de3a556c734p-19);
        p = exp_dfma(p, r, 0x1.a01a01a01a01ap-16);
        p = exp_dfma(p, r, 0x1.a01a01a01a01ap-13);
        p = exp_dfma(p, r, 0x1.6c16c16c16c17p-10);
        p = exp_dfma(p, r, 0x1.1111111111111p-7);
        p = exp_dfma(p, r, 0x1.5555555555555p-5);
        p = exp_dfma(p, r, 0x1.5555555555555p-3);
        p = exp_dfma(p, r, 0.5);
    } else if (N == 4) {  // n = 7 .. 2
        p = 0x1.a01a01a01a01ap-13;
        p = exp_dfma(p, r, 0x1.6c16c16c16c17p-10);
        p = exp_dfma(p, r, 0x1.1111111111111p-7);
        p = exp_dfma(p, r, 0x1.5555555555555p-5);
        p = exp_dfma(p, r, 0x1.5555555555555p-3);
        p = exp_dfma(p, r, 0.5);
    } else {  // n = 6 .. 2
        p = 0x1.6c16c16c16c17p-10;
        p = exp_dfma(p, r, 0x1.1111111111111p-7);
        p = exp_dfma(p, r, 0x1.5555555555555p-5);
        p = exp_dfma(p, r, 0x1.5555555555555p-3);
        p = exp_dfma(p, r, 0.5);
    }
    p = exp_dfma(p, r, 1.0);
    p = exp_dfma(p, r, 1.0);  // e^r
    // 2^(j/N) * 2^k: k = floor(kj / N) added to the table entry's exponent
    // (|k| <= 159 after the clamp; for a NaN input kj is arbitrary and the
    // product stays NaN)
    const int k = kj >> (N == 1 ? 0 : N == 4 ? 2 : 3);
    const uint64_t sbits = exp_double_bits(exp_table<N>(kj & (N - 1))) + ((uint64_t)(int64_t)k << 52);
    return (float)(p * exp_bits_double(sbits));
}

// 2^(j/64) = hi + lo for j in [0, 64): hi the nearest float, lo the float
// nearest to the remainder (|lo| <= 2^-24, relative error of the pair
// <= 2^-47).
#define OXIDE_EXP2_64_TABLE                                                                                 \
    {0x1p+0f, 0.0f}, {0x1.02c9a4p+0f, -0x1.887fap-28f}, {0x1.059b0ep+0f, -0x1.9d4f52p-25f},                  \
        {0x1.087452p+0f, -0x1.e2990ep-26f}, {0x1.0b5586p+0f, 0x1.9f3122p-25f},                             \
        {0x1.0e3ec4p+0f, -0x1.a585ccp-25f}, {0x1.11301ep+0f, -0x1.fdb496p-25f},                            \
        {0x1.1429aap+0f, 0x1.d525bcp-25f}, {0x1.172b84p+0f, -0x1.c15742p-27f},                             \
        {0x1.1a35bep+0f, 0x1.6df96ep-25f}, {0x1.1d4874p+0f, -0x1.d2e8cap-25f},                             \
        {0x1.2063b8p+0f, 0x1.0c519ap-25f}, {0x1.2387a6p+0f, 0x1.ceac48p-25f},                              \
        {0x1.26b456p+0f, 0x1.789f38p-26f}, {0x1.29e9e0p+0f, -0x1.5c0424p-25f},                             \
        {0x1.2d285ap+0f, 0x1.b900c2p-26f}, {0x1.306fe0p+0f, 0x1.4636e2p-25f},                              \
        {0x1.33c08cp+0f, -0x1.b37d2p-25f}, {0x1.371a74p+0f, -0x1.18aac6p-25f},                             \
        {0x1.3a7db4p+0f, -0x1.634c02p-25f}, {0x1.3dea64p+0f, 0x1.824684p-25f},                             \
        {0x1.4160a2p+0f, 0x1.f72e2ap-28f}, {0x1.44e086p+0f, 0x1.8624b4p-30f},                              \
        {0x1.486a2cp+0f, -0x1.47d866p-25f}, {0x1.4bfdaep+0f, -0x1.593abcp-25f},                            \
        {0x1.4f9b28p+0f, -0x1.2c5a6cp-25f}, {0x1.5342b6p+0f, -0x1.2c561p-25f},                             \
        {0x1.56f474p+0f, -0x1.295b04p-25f}, {0x1.5ab07ep+0f, -0x1.5bd5ecp-27f},                            \
        {0x1.5e76f2p+0f, -0x1.4a5bd6p-25f}, {0x1.6247ecp+0f, -0x1.f8b55p-25f},                             \
        {0x1.662388p+0f, 0x1.2a9112p-27f}, {0x1.6a09e6p+0f, 0x1.9fcef4p-26f},                              \
        {0x1.6dfb24p+0f, -0x1.cd72e8p-27f}, {0x1.71f75ep+0f, 0x1.1d8beep-25f},                             \
        {0x1.75feb6p+0f, -0x1.37b306p-25f}, {0x1.7a1148p+0f, -0x1.829fdp-25f},                             \
        {0x1.7e2f34p+0f, -0x1.261634p-25f}, {0x1.82589ap+0f, -0x1.accc7cp-26f},                            \
        {0x1.868d9ap+0f, -0x1.2edb44p-26f}, {0x1.8ace54p+0f, 0x1.15506ep-27f},                             \
        {0x1.8f1aeap+0f, -0x1.baa232p-26f}, {0x1.93737cp+0f, -0x1.e64744p-25f},                            \
        {0x1.97d82ap+0f, -0x1.0d8d84p-31f}, {0x1.9c4918p+0f, 0x1.51f848p-27f},                             \
        {0x1.a0c668p+0f, -0x1.2886a6p-26f}, {0x1.a5503cp+0f, -0x1.b83b54p-25f},                            \
        {0x1.a9e6b6p+0f, -0x1.50c048p-25f}, {0x1.ae89fap+0f, -0x1.a94b14p-26f},                            \
        {0x1.b33a2cp+0f, -0x1.ec3a82p-26f}, {0x1.b7f770p+0f, -0x1.a09438p-25f},                            \
        {0x1.bcc1eap+0f, -0x1.f687c6p-25f}, {0x1.c199bep+0f, -0x1.3d56b2p-27f},                            \
        {0x1.c67f12p+0f, 0x1.cafa2ap-25f}, {0x1.cb720ep+0f, -0x1.8837ccp-27f},                             \
        {0x1.d072d4p+0f, 0x1.40f13p-25f}, {0x1.d5818ep+0f, -0x1.822dbcp-27f},                              \
        {0x1.da9e60p+0f, 0x1.ed9942p-27f}, {0x1.dfc974p+0f, -0x1.908c94p-25f},                             \
        {0x1.e502eep+0f, 0x1.e2cffep-26f}, {0x1.ea4afap+0f, 0x1.52486cp-27f},                              \
        {0x1.efa1bep+0f, 0x1.cc2b44p-25f}, {0x1.f50766p+0f, -0x1.246ebp-26f}, {0x1.fa7c18p+0f, 0x1.9e90d8p-28f}
#ifdef __CUDA_ARCH__
static __device__ const float2 kExp2Tab64[64] = {OXIDE_EXP2_64_TABLE};
#else
static const float2 kExp2Tab64[64] = {OXIDE_EXP2_64_TABLE};
#endif
__host__ __device__ __forceinline__ float2 exp2_64(int j) {
#ifdef __CUDA_ARCH__
    return __ldg(&kExp2Tab64[j]);  // 512 bytes: stays in L1 beside the streaming loads
#else
    return kExp2Tab64[j];
#endif
}

// f32x2 operations (Blackwell's paired f32 pipe: each lane one IEEE
// round-to-nearest operation), the same on host and device.  No paired
// product below feeds a paired add: the compiler may fuse such a pair into
// one rounding.
__host__ __device__ __forceinline__ float2 exp_ffma2(float2 a, float2 b, float2 c) {
#ifdef __CUDA_ARCH__
    return __ffma2_rn(a, b, c);
#else
    return make_float2(exp_ffma(a.x, b.x, c.x), exp_ffma(a.y, b.y, c.y));
#endif
}
__host__ __device__ __forceinline__ float2 exp_fadd2(float2 a, float2 b) {
#ifdef __CUDA_ARCH__
    return __fadd2_rn(a, b);
#else
    return make_float2(exp_fadd(a.x, b.x), exp_fadd(a.y, b.y));
#endif
}
__host__ __device__ __forceinline__ float2 exp_fmul2(float2 a, float2 b) {
#ifdef __CUDA_ARCH__
    return __fmul2_rn(a, b);
#else
    return make_float2(exp_fmul(a.x, b.x), exp_fmul(a.y, b.y));
#endif
}
__host__ __device__ __forceinline__ float2 exp_c2(float c) { return make_float2(c, c); }

// The f32 path, two inputs at a time.  Reduction (Tang's, N = 64):
// K = round(x 64 / ln2) from one fused multiply-add against 1.5 * 2^23;
// x = K Lh + rh with Lh = RN(ln2 / 64) (20 significant bits) -- rh is exact:
// x - K Lh is a multiple of min(ulp(x), 2^-27) below 2^-7 in magnitude, so it
// fits in 24 bits and the fused step does not round -- and r = rh + rl,
// rl = -K Ll with Ll = RN(ln2 / 64 - Lh) (~2^-35): within 2^-53 of
// x - K ln2 / 64 for |K| <= 8192.  e^r = 1 + rh + E with
// E = rl + s^2 (1/2 + s/6 + s^2/24), s = RN(rh + rl) (truncation < 2^-44 for
// |r| <= ln2 / 128), held as the unevaluated pair ah + al (Fast2Sum of 1 and
// rh, plus E).  With 2^(j/64) = Th + Tl from the table, e^x 2^-k =
// Th ah + yl + d, yl = RN(Th al + RN(Tl ah)); the largest |d| over every
// float x of the fast range is 2^-37.1 (measured against the
// 64-bit-significand expl), and EPS = 2^-36.  Ziv's test (A. Ziv, ACM TOMS
// 17(3), 1991): the nearest floats to Th ah + (yl + EPS) and to
// Th ah + (yl - EPS) -- each one fused multiply-add, the product exact --
// agree, so (rounding being monotonic) so does every value in between, e^x 2^-k
// among them; yl +- EPS is rounded first (|yl| < 2^-14.9: by at most 2^-39),
// which leaves a margin of 1.9.  The scaling by 2^k goes into the exponent
// field, exact for K in [-8000, 8063] (results in [2^-126, 2^126): x in
// about [-86.6, 87.3]).  Where the test fails or K is outside, ok = false.
constexpr float EXP_FF_EPS = 0x1p-36f;
// The shared steps: zh and zl (Th ah + (yl +- EPS), before the scaling by
// 2^k) and the bit patterns of t, whose low bits hold K.
__host__ __device__ __forceinline__ void exp_ff_core(float2 x, float2& zh, float2& zl, uint32_t& b0, uint32_t& b1) {
    const float2 t = exp_ffma2(x, exp_c2(0x1.715476p+6f), exp_c2(0x1.8p23f));  // 1.5 * 2^23 + K
    const float2 kf = exp_fadd2(t, exp_c2(-0x1.8p23f));
    // K = bits(t) - 0x4B400000; that constant's low 15 bits are zero, so
    // K mod 64 = bits(t) mod 64 and (K >> 6) << 23 = (bits(t) >> 6) << 23
    // modulo 2^32, and the range test is one unsigned comparison.
    b0 = (uint32_t)exp_f2i(t.x);
    b1 = (uint32_t)exp_f2i(t.y);
    const float2 rh = exp_ffma2(kf, exp_c2(-0x1.62e43p-7f), x);
    const float2 rl = exp_fmul2(kf, exp_c2(0x1.05c61p-35f));  // -K Ll (Ll < 0)
    const float2 s = exp_ffma2(kf, exp_c2(0x1.05c61p-35f), rh);
    const float2 q = exp_ffma2(exp_ffma2(s, exp_c2(0x1.555556p-5f), exp_c2(0x1.555556p-3f)), s, exp_c2(0.5f));
    const float2 e = exp_ffma2(exp_fmul2(s, s), q, rl);
    const float2 ah = exp_fadd2(exp_c2(1.0f), rh);
    const float2 al = exp_fadd2(exp_fadd2(rh, exp_ffma2(ah, exp_c2(-1.0f), exp_c2(1.0f))), e);  // rh - (ah - 1) exactly
    const float2 t0 = exp2_64((int)(b0 & 63u)), t1 = exp2_64((int)(b1 & 63u));
    const float2 th = make_float2(t0.x, t1.x), tl = make_float2(t0.y, t1.y);
    const float2 yl = exp_ffma2(th, al, exp_fmul2(tl, ah));
    zh = exp_ffma2(th, ah, exp_fadd2(yl, exp_c2(EXP_FF_EPS)));
    zl = exp_ffma2(th, ah, exp_fadd2(yl, exp_c2(-EXP_FF_EPS)));
}
__host__ __device__ __forceinline__ float exp_ff_scale(float z, uint32_t b) {
    return exp_i2f((int)((uint32_t)exp_f2i(z) + ((b >> 6) << 23)));
}
__host__ __device__ __forceinline__ float2 exp_rn_f32x2_ff(float2 x, bool& ok0, bool& ok1) {
    float2 zh, zl;
    uint32_t b0, b1;
    exp_ff_core(x, zh, zl, b0, b1);
    ok0 = (b0 - (0x4B400000u - 8000u) < 16064u) & (zh.x == zl.x);  // K in [-8000, 8063]
    ok1 = (b1 - (0x4B400000u - 8000u) < 16064u) & (zh.y == zl.y);
    return make_float2(exp_ff_scale(zh.x, b0), exp_ff_scale(zh.y, b1));
}
// The same value for inputs the caller has checked to lie in
// [-EXP_FF_XMAX, EXP_FF_XMAX] (K within [-7988, 7988], so the scaling by 2^k
// stays exact and the result normal): instead of two flags, the bits of
// zh - zl of both lanes are OR-ed into `diff`.  zh - zl is exact, so `diff`
// stays zero exactly when both rounding tests pass (a NaN or an infinity
// leaves nonzero bits).
constexpr float EXP_FF_XMAX = 86.5f;
__host__ __device__ __forceinline__ float2 exp_rn_f32x2_ffr(float2 x, uint32_t& diff) {
    float2 zh, zl;
    uint32_t b0, b1;
    exp_ff_core(x, zh, zl, b0, b1);
    const float2 dz = exp_fadd2(zh, make_float2(-zl.x, -zl.y));
    diff |= (uint32_t)exp_f2i(dz.x) | (uint32_t)exp_f2i(dz.y);
    return make_float2(exp_ff_scale(zh.x, b0), exp_ff_scale(zh.y, b1));
}
// One input through the same steps (the first lane of the pair).
__host__ __device__ __forceinline__ float exp_rn_f32_ff(float x, bool& ok) {
    bool ok1;
    const float2 y = exp_rn_f32x2_ff(make_float2(x, x), ok, ok1);
    return y.x;
}

// The inputs on which the double path misrounds: the 17 floats whose e^x
// lies within 2^-44 (relative) of a rounding boundary, found by comparing it
// with the 64-bit-significand expl over every float (tests/test_exp_rn.py
// repeats that comparison), with their correctly rounded results -- the
// exception list of a correctly rounded libm.
__host__ __device__ __forceinline__ float exp_rn_f32_hard(float x) {
    const uint32_t b = (uint32_t)exp_f2i(x);
    if (b == 0x3da59a3fu) return exp_i2f((int)0x3f8ac7b7u);
    if (b == 0x3e777fecu) return exp_i2f((int)0x3fa2ff20u);
    if (b == 0x3f76527bu) return exp_i2f((int)0x4027841cu);
    if (b == 0x4016bd40u) return exp_i2f((int)0x4128a92bu);
    if (b == 0x4119f639u) return exp_i2f((int)0x466bf9d8u);
    if (b == 0x4140c8dfu) return exp_i2f((int)0x4826edd8u);
    if (b == 0x4288942bu) return exp_i2f((int)0x70b7a4c5u);
    if (b == 0xbd98bce5u) return exp_i2f((int)0x3f6d9a33u);
    if (b == 0xbda7375du) return exp_i2f((int)0x3f6bedb4u);
    if (b == 0xbdaeda7au) return exp_i2f((int)0x3f6b0ce5u);
    if (b == 0xbdb393ebu) return exp_i2f((int)0x3f6a823fu);
    if (b == 0xbee0e6cdu) return exp_i2f((int)0x3f24fec8u);
    if (b == 0xbfd04462u) return exp_i2f((int)0x3e49379bu);
    if (b == 0xc0382e72u) return exp_i2f((int)0x3d666d27u);
    if (b == 0xc159fa1eu) return exp_i2f((int)0x35a29e78u);
    if (b == 0xc16912cdu) return exp_i2f((int)0x34fd331bu);
    if (b == 0xc2abb454u) return exp_i2f((int)0x018d2f96u);
    return exp_rn_f32_dp<4>(x);
}
// The fallback is a real call on the device, so that the double path runs
// only in the warps where some lane needs it (an inlined conditional would
// be evaluated for every element).
#ifdef __CUDA_ARCH__
__device__ __noinline__ float exp_rn_f32_fallback(float x) { return exp_rn_f32_hard(x); }
#else
inline float exp_rn_f32_fallback(float x) { return exp_rn_f32_hard(x); }
#endif
__host__ __device__ __forceinline__ float exp_rn_f32(float x) {
    bool ok;
    float y = exp_rn_f32_ff(x, ok);
    if (!ok) y = exp_rn_f32_fallback(x);
    return y;
}

// ---------------------------------------------------------------------------
// Special-function unit approximations (relative error ~2^-22; subnormal
// results kept).  Used only where the result is rounded to bf16 afterwards or
// the tolerance is stated beside the caller.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float t) {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(t));
    return y;
}
__device__ __forceinline__ float lg2_approx(float t) {
    float y;
    asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(t));
    return y;
}

// ---------------------------------------------------------------------------
// Warp / block reductions (fixed shuffle trees: deterministic)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fadd(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

// Reduce within groups of `group_threads` consecutive threads (a multiple of
// 32) of a block.  Every thread of a group receives the group's result.
// `red` must hold blockDim.x / 32 elements.  Contains __syncthreads().
template <typename T, typename Op>
__device__ __forceinline__ T group_reduce(T v, T* red, int group_threads, Op op) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (group_threads == 32) return v;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    const int wpg = group_threads >> 5;
    const int first = (warp / wpg) * wpg;
    T r = red[first];
    for (int i = 1; i < wpg; ++i) r = op(r, red[first + i]);
    __syncthreads();  // red may be reused right after
    return r;
}

struct OpAddF {
    __device__ __forceinline__ float operator()(float a, float b) const { return fadd(a, b); }
};
struct OpMaxF {
    __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); }
};
struct OpMaxU64 {
    __device__ __forceinline__ uint64_t operator()(uint64_t a, uint64_t b) const {
        return a > b ? a : b;
    }
};

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel is launched with programmatic
// stream serialization (launch_k below), so its CTAs may be scheduled while
// the kernel before it on the stream is still finishing.  pdl_begin() is the
// first statement of every kernel: it lets the next kernel launch early
// (griddepcontrol.launch_dependents -- that kernel's own pdl_begin() then
// waits) and waits until the previous kernel has completed with its memory
// visible (griddepcontrol.wait) before this kernel touches global memory.  A
// kernel launched without the attribute returns from the wait at once.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_begin() {
    pdl_trigger();
    pdl_wait();
}

bool pdl_enabled();  // false when OXIDE_NO_PDL=1 is set (read once)

// Append the programmatic-serialization attribute to attr[0..n) (room for one
// more) when it is enabled; returns the new count.
inline int add_pdl_attr(cudaLaunchAttribute* attr, int n) {
    if (!pdl_enabled()) return n;
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    return n + 1;
}

// cudaLaunchKernelEx with programmatic stream serialization; launch_kx adds
// the extra attributes given (e.g. a cluster shape).
template <typename... P, typename... A>
cudaError_t launch_kx(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      const cudaLaunchAttribute* extra, int n_extra, A&&... args) {
    cudaLaunchAttribute attr[4];
    int n = 0;
    for (int i = 0; i < n_extra && n < 3; ++i) attr[n++] = extra[i];
    if (pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}
template <typename... P, typename... A>
cudaError_t launch_k(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
    return launch_kx(kernel, grid, block, smem, st, (const cudaLaunchAttribute*)nullptr, 0,
                     static_cast<A&&>(args)...);
}

// ---------------------------------------------------------------------------
// Host-side helpers (defined in oxide_runtime.cu)
// ---------------------------------------------------------------------------
int sm_count();                      // SMs of the current device (cached)
// Resident CTAs of `kernel` across the whole current device (occupancy x SMs),
// cached per (device, kernel, block size, dynamic smem).
int resident_blocks(const void* kernel, int threads, size_t smem);
// Opt `kernel` in to `smem` bytes of dynamic shared memory on the current
// device (needed above 48 KiB); cached.  False if the device refuses.
bool ensure_dyn_smem(const void* kernel, size_t smem);
int set_error(int code, const char* fmt, ...);  // records message, returns code
int check_launch(const char* op);    // cudaGetLastError -> status
int injected_failure(const char* op);  // host-side fault injection hook
bool aligned16(const void* p);
void* driver_fn(const char* symbol);  // driver API entry point, nullptr if absent
unsigned long long current_context_id();  // cuCtxGetId of the current context, 0 if none

}  // namespace oxide

// Common argument checks: every entry point returns a status instead of
// aborting.  OXIDE_INJECT runs first so fault-injection tests never launch.
#define OXIDE_INJECT(op)                                      \
    do {                                                      \
        int _inj = ::oxide::injected_failure(op);             \
        if (_inj) return _inj;                                \
    } while (0)
#define OXIDE_REQUIRE(cond, op, msg)                                                     \
    do {                                                                                 \
        if (!(cond)) return ::oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: %s", op, msg); \
    } while (0)
