// Host build of the f32 SiLU arithmetic of the library's kernels:
// silu(x) = x * RN(1 / RN(1 + exp_rn_f32(-x))), each step one IEEE f32
// operation, with oxide::exp_rn_f32 from csrc/oxide_common.cuh.  The GPU
// tests compare the device kernels' bits with this over a sample of every
// f32 bit pattern (the device computes the same operations, so any
// difference would mean the compiler changed an operation's rounding).
#include <omp.h>
#include <stdint.h>

#include "oxide_common.cuh"

static float silu_host(float x) {
    const float e = oxide::exp_rn_f32(-x);
    const float d = oxide::exp_fadd(1.0f, e);
    volatile float r = 1.0f / d;
    return oxide::exp_fmul(x, r);
}

extern "C" void silu_bits_host(uint32_t first, uint32_t stride, uint64_t n, float* out) {
#pragma omp parallel for schedule(static, 1 << 16)
    for (long long i = 0; i < (long long)n; ++i) {
        const uint32_t b = first + (uint32_t)i * stride;
        float x;
        __builtin_memcpy(&x, &b, 4);
        out[i] = silu_host(x);
    }
}
