// Host check of oxide::exp_rn_f32 (csrc/oxide_common.cuh) over every f32 bit
// pattern (or a stride of them): against the host C library's expf (the
// function the reference's f32::exp calls) and against the correctly rounded
// value RN(expl(x)) (64-bit significand).  The function is IEEE f32 and f64
// arithmetic written out operation by operation, so its host compilation
// returns the device's bits.
//
//   exp_rn_check [stride]
//   prints: total mismatches_vs_expf max_ulp_vs_expf nan_bad
//           mismatches_vs_rn fast_path_misses_in_normal_range
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
    long long mism = 0, maxu = 0, total = 0, nan_bad = 0, mism_rn = 0, slow = 0;
#pragma omp parallel for schedule(static, 1 << 16) reduction(+ : mism, total, nan_bad, mism_rn, slow) \
    reduction(max : maxu)
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
        const float rn = (float)expl((long double)x);
        mism_rn += memcmp(&got, &rn, 4) != 0;
        bool ok;
        (void)oxide::exp_rn_f32_ff(x, ok);
        slow += (x > -86.0f && x < 87.0f && !ok);
    }
    printf("%lld %lld %lld %lld %lld %lld\n", total, mism, maxu, nan_bad, mism_rn, slow);
    return 0;
}
