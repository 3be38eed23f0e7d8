// Host check of oxide::exp_rn_f32 (csrc/oxide_common.cuh) against the host C
// library's expf over every f32 bit pattern (or a stride of them).  The
// function is plain IEEE double arithmetic (fused multiply-adds, one multiply,
// one conversion), so its host compilation returns the device's bits.
//
//   exp_rn_check [stride]   prints: total mismatches max_ulp nan_ok
#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "oxide_common.cuh"

static long long ord(float f) {
    int32_t i;
    memcpy(&i, &f, 4);
    return i < 0 ? -(long long)(i & 0x7fffffff) : (long long)i;
}

int main(int argc, char** argv) {
    const uint64_t stride = argc > 1 ? strtoull(argv[1], 0, 10) : 1;
    long long mism = 0, maxu = 0, total = 0, nan_bad = 0;
#pragma omp parallel for schedule(static, 1 << 16) reduction(+ : mism, total, nan_bad) reduction(max : maxu)
    for (long long b = 0; b < (1ll << 32); b += (long long)stride) {
        uint32_t u = (uint32_t)b;
        float x;
        memcpy(&x, &u, 4);
        const float got = oxide::exp_rn_f32(x), ref = expf(x);
        ++total;
        if (x != x) {
            nan_bad += got == got;
            continue;
        }
        if (memcmp(&got, &ref, 4) != 0) {
            ++mism;
            const long long d = llabs(ord(got) - ord(ref));
            if (d > maxu) maxu = d;
        }
    }
    printf("%lld %lld %lld %lld\n", total, mism, maxu, nan_bad);
    return 0;
}
