// k_sample.cu -- token sampling: softmax_with_temperature and the top-k / top-p
// selection of the reference's sample_next_token, on the GPU.
//
// Reference: src/pipeline.rs:181-205 takes the last row of logits, computes
// probs = softmax_with_temperature(row, T) (src/tokenizer.rs:166-180:
// s = x / T, m = fold(-inf, f32::max), sum = sum exp(s - m), p = exp(s - m) / sum)
// and then, when top_p < 1, sample_top_p (:182-211), else sample_top_k
// (:213-232).  Both sort the probabilities in descending order (a stable sort:
// equal probabilities keep ascending index order), keep a prefix (the first k,
// or the shortest prefix whose running sum reaches top_p), draw
// r = u * total with u = fastrand::f32() and total the prefix's sum, and
// return the first index of the prefix whose running sum reaches r.  Here the
// uniform draw is an input (one per row), so the caller keeps the reference's
// generator; everything after it runs on the device.
//
// Design: one CTA per row of up to 32768 logits, or a thread-block cluster of
// 2-8 CTAs (up to 262144), each CTA holding a contiguous segment of the row of
// up to 32768 elements in shared memory (128 KB, natural order; thread t owns
// the float4 groups t, t + 512, ...).  Rows are split over more CTAs than
// their length needs when the grid would otherwise leave SMs idle (few rows:
// one decode step's logits), down to 4096 logits per CTA.  No full sort:
//   1. softmax_with_temperature with three passes over shared memory and two
//      block reductions (max, then sum); x / T and e / sum are IEEE quotients;
//   2. a threshold v whose candidates (every probability >= v) hold the kept
//      prefix and number at most 2048, by bisection on the probability bits
//      (non-negative floats order like their bit patterns): for a pivot x the
//      count / sum of the probabilities >= x is one block reduction, and the
//      search stops at the first pivot that is both far enough down and
//      selective enough (usually after ~10 halvings);
//   3. the candidates are gathered into the first CTA as 64-bit keys
//      (probability bits << 32 | ~index: descending key order is descending
//      probability, then ascending index -- the stable sort's order), sorted
//      by a bitonic network, and one thread runs the reference's sequential
//      f32 loops over them, so the token equals the reference's for the same
//      probabilities, bit for bit.
// When the kept prefix is longer than 2048 (top-p over a flat row, top-k >
// 2048), step 3 is replaced by the bisection carried to the crossing element
// itself, with f64 running sums (sums of per-thread f32 sums in a fixed
// order): the token then equals the reference's unless r lies within the
// reference's own sequential-sum drift of a boundary.  Equal probabilities
// cut by the prefix are ordered by index with a bisection on the index.
//
// A row whose probabilities are not all numbers (a NaN logit, a scaled logit
// of +-inf, or all -inf) yields OXIDE_SAMPLE_INVALID: the reference's sort
// panics on NaN there.  vocab == 1 yields 0, as the reference does.  All loops
// are bounded (bisections halve an interval, the sort has fixed stages), and
// every branch before a barrier depends only on reduced values, which are
// bit-identical in every thread and CTA of the cluster.
#include <cooperative_groups.h>

#include "oxide_common.cuh"

namespace cg = cooperative_groups;

namespace oxide {

constexpr int SMP_THREADS = 512;
constexpr int SMP_WARPS = SMP_THREADS / 32;
constexpr uint32_t SMP_SPAN = 32768;                      // logits per CTA
constexpr int SMP_GATHER = 2048;                          // candidates walked exactly
// candidates sorted after narrowing: top-k stops at 256 keys; top-p at 512,
// since its mass criterion leaves a narrow window of pivots above a nucleus
// of a few hundred keys (measured at C3, top-p 0.9 at T = 0.7: 41.8 us with
// 256, 36.1 us with 512; top-k 50: 26.0 us with 256, 26.6 us with 512)
constexpr uint32_t SMP_SORT_CAP_K = 256;
constexpr uint32_t SMP_SORT_CAP_P = 512;
constexpr int SMP_NARROW_STEPS = 12;                      // bisection steps spent narrowing
constexpr uint32_t SMP_FALLBACK = 0xFFFFFFFEu;            // the walk needs more than was gathered
// row segment, gathered keys, the walk's running sums
constexpr size_t SMP_SMEM = (size_t)SMP_SPAN * 4 + (size_t)SMP_GATHER * 8 + (size_t)SMP_GATHER * 4;  // 155,648 B

struct SmpArgs {
    const void* logits;
    uint64_t rows;
    uint32_t vocab;
    float temperature;
    uint64_t top_k;
    float top_p;
    const float* uniforms;
    uint32_t* tokens;  // null: probabilities only
    float* probs;      // null: not stored
    uint32_t span;     // logits per CTA of a row's cluster: a multiple of 4, <= SMP_SPAN
};

enum { RSUM = 0, RMAX = 1, RMIN = 2 };

template <int OP>
__device__ __forceinline__ double rop(double a, double b) {
    if (OP == RSUM) return a + b;
    if (OP == RMAX) return a > b ? a : b;
    return a < b ? a : b;
}
template <int OP>
__device__ __forceinline__ double rident() {
    return OP == RSUM ? 0.0 : (OP == RMAX ? -INFINITY : INFINITY);
}

// Block (and cluster) reduction of two doubles with ops OA / OB.  The warp
// partials are double-buffered by `phase`, so one barrier per call suffices:
// a slot is rewritten two calls later, after every reader has passed the
// barrier of the call in between.
template <int CL>
struct Reducer {
    double2* red;   // [2][SMP_WARPS] warp partials
    double2* cred;  // [2] CTA partials (cluster only)
    uint32_t phase;

    template <int OA, int OB>
    __device__ __forceinline__ double2 run(double a, double b) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            a = rop<OA>(a, __shfl_xor_sync(0xffffffffu, a, o));
            b = rop<OB>(b, __shfl_xor_sync(0xffffffffu, b, o));
        }
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        double2* slot = red + phase * SMP_WARPS;
        if (lane == 0) slot[warp] = make_double2(a, b);
        __syncthreads();
        double2 r;
        if (CL == 1) {
            r = slot[0];
#pragma unroll
            for (int w = 1; w < SMP_WARPS; ++w) {
                const double2 v = slot[w];
                r.x = rop<OA>(r.x, v.x);
                r.y = rop<OB>(r.y, v.y);
            }
        } else {
            if (warp == 0) {
                double2 v = lane < SMP_WARPS ? slot[lane] : make_double2(rident<OA>(), rident<OB>());
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    v.x = rop<OA>(v.x, __shfl_xor_sync(0xffffffffu, v.x, o));
                    v.y = rop<OB>(v.y, __shfl_xor_sync(0xffffffffu, v.y, o));
                }
                if (lane == 0) cred[phase] = v;
            }
            cg::cluster_group cluster = cg::this_cluster();
            cluster.sync();
            r = *cluster.map_shared_rank(cred + phase, 0);
#pragma unroll
            for (int q = 1; q < CL; ++q) {
                const double2 v = *cluster.map_shared_rank(cred + phase, q);
                r.x = rop<OA>(r.x, v.x);
                r.y = rop<OB>(r.y, v.y);
            }
        }
        phase ^= 1u;
        return r;
    }
};

// The element at which the running measure, in (probability desc, index asc)
// order, first reaches t.
struct Cross {
    float v;          // its probability
    uint32_t idx;     // its index (when asked for)
    double cum_sum;   // sum of the probabilities up to and including it
    double j;         // its rank among the elements equal to v (1-based)
    double ties;      // number of probabilities == v
};

// A threshold whose candidates hold the kept prefix (see coarse()).
struct Coarse {
    float v;
    bool ok;
    double count, c_gt, s_gt, ties;
};

// One CTA's segment of a row of probabilities in shared memory; slots past
// the row hold -1, which no pivot >= 0 counts.
template <int CL>
struct Row {
    const float4* sp;  // this CTA's segment, natural order
    uint32_t ng;       // its float4 groups (span / 4)
    uint32_t base;     // row index of sp[0]
    uint32_t vocab;
    Reducer<CL>* rd;

    // (sum, count) of the probabilities >= x; f32 per thread in a fixed order
    // (monotone in the set), f64 across threads.
    __device__ double2 measure(float x) {
        float s = 0.0f;
        uint32_t c = 0;
#pragma unroll 4
        for (uint32_t q = threadIdx.x; q < ng; q += SMP_THREADS) {
            const float4 v = sp[q];
            if (v.x >= x) { s = fadd(s, v.x); ++c; }
            if (v.y >= x) { s = fadd(s, v.y); ++c; }
            if (v.z >= x) { s = fadd(s, v.z); ++c; }
            if (v.w >= x) { s = fadd(s, v.w); ++c; }
        }
        return rd->template run<RSUM, RSUM>((double)s, (double)c);
    }

    // The j-th (1-based) index holding exactly v, in ascending index order.
    __device__ uint32_t tie_index(float v, double ties, double j) {
        if (ties == 1.0) {
            double mi = 4294967296.0;
            for (uint32_t q = threadIdx.x; q < ng; q += SMP_THREADS) {
                const float4 w = sp[q];
                const double i0 = (double)(base + 4 * q);
                if (w.x == v) mi = fmin(mi, i0);
                if (w.y == v) mi = fmin(mi, i0 + 1.0);
                if (w.z == v) mi = fmin(mi, i0 + 2.0);
                if (w.w == v) mi = fmin(mi, i0 + 3.0);
            }
            return (uint32_t)rd->template run<RMIN, RMIN>(mi, 0.0).x;
        }
        // smallest I with count(p == v, index <= I) >= j
        uint32_t lo = 0, hi = vocab - 1;
        while (lo < hi) {
            const uint32_t mid = lo + (hi - lo) / 2;
            uint32_t c = 0;
            for (uint32_t q = threadIdx.x; q < ng; q += SMP_THREADS) {
                const float4 w = sp[q];
                const uint32_t i0 = base + 4 * q;
                c += (w.x == v && i0 <= mid) + (w.y == v && i0 + 1 <= mid) + (w.z == v && i0 + 2 <= mid) +
                     (w.w == v && i0 + 3 <= mid);
            }
            const double n = rd->template run<RSUM, RSUM>((double)c, 0.0).x;
            if (n >= j) hi = mid;
            else lo = mid + 1;
        }
        return lo;
    }

    // A value v with M(v) >= t and at most `cap` probabilities >= v, by
    // bisection that stops at the first such pivot (the crossing value itself
    // is not needed: the candidates >= v are sorted afterwards).  On entry
    // M(lo) >= t > M(hi) = 0.  When the crossing value alone has more than
    // `cap` elements >= it (a long run of equal probabilities), ok is false and
    // v is that value, with the count and sum of the elements above it.
    template <bool SUM>
    __device__ Coarse coarse(double t, uint32_t lo, uint32_t hi, double c_lo, uint32_t cap) {
        Coarse g{__uint_as_float(lo), true, c_lo, 0.0, 0.0, 0.0};
        if (c_lo <= (double)cap) return g;
        double c_hi = 0.0, s_hi = 0.0;
        while (hi - lo > 1) {
            const uint32_t mid = lo + (hi - lo) / 2;
            const double2 m = measure(__uint_as_float(mid));
            if ((SUM ? m.x : m.y) >= t) {
                lo = mid;
                c_lo = m.y;
                if (m.y <= (double)cap) {
                    g.v = __uint_as_float(mid);
                    g.count = m.y;
                    return g;
                }
            } else {
                hi = mid;
                c_hi = m.y;
                s_hi = m.x;
            }
        }
        g.ok = false;
        g.v = __uint_as_float(lo);
        g.count = c_lo;
        g.c_gt = c_hi;
        g.s_gt = s_hi;
        g.ties = c_lo - c_hi;
        return g;
    }

    // The crossing element itself: bisection over probability bits in
    // [lo, hi) with M(lo) >= t > M(hi) on entry, c_lo the count of
    // measure(lo) and (s_hi, c_hi) = measure(hi).  SUM: t is a probability
    // mass, else a count.  j_cap (> 0) bounds the rank among ties of cap_v (a
    // kept prefix that ends inside a run of equal probabilities).
    template <bool SUM>
    __device__ Cross bisect(double t, uint32_t lo, uint32_t hi, double c_lo, double s_hi, double c_hi,
                            float cap_v, double j_cap, bool want_idx) {
        while (hi - lo > 1) {
            const uint32_t mid = lo + (hi - lo) / 2;
            const double2 m = measure(__uint_as_float(mid));
            if ((SUM ? m.x : m.y) >= t) {
                lo = mid;
                c_lo = m.y;
            } else {
                hi = mid;
                s_hi = m.x;
                c_hi = m.y;
            }
        }
        const float v = __uint_as_float(lo);
        const double ties = c_lo - c_hi;
        const double vd = (double)v;
        double j;
        if (SUM) {
            if (vd > 0.0) {
                j = ceil((t - s_hi) / vd);
                if (j < 1.0) j = 1.0;
                if (j > ties) j = ties;
                while (j > 1.0 && s_hi + (j - 1.0) * vd >= t) j -= 1.0;
                while (j < ties && s_hi + j * vd < t) j += 1.0;
            } else {
                j = ties;
            }
        } else {
            j = t - c_hi;
            if (j < 1.0) j = 1.0;
            if (j > ties) j = ties;
        }
        if (v == cap_v && j > j_cap) j = j_cap;
        Cross x;
        x.v = v;
        x.j = j;
        x.ties = ties;
        x.cum_sum = s_hi + j * vd;
        x.idx = want_idx ? tie_index(v, ties, j) : 0u;
        return x;
    }
};

// One compare-exchange step (k, j) across shared memory.
__device__ __forceinline__ void bitonic_step_smem(unsigned long long* buf, uint32_t n, uint32_t k, uint32_t j) {
    for (uint32_t i = threadIdx.x; i < n; i += SMP_THREADS) {
        const uint32_t ixj = i ^ j;
        if (ixj > i) {
            const unsigned long long x = buf[i], y = buf[ixj];
            const bool desc = (i & k) == 0;
            if (desc ? x < y : x > y) {
                buf[i] = y;
                buf[ixj] = x;
            }
        }
    }
    __syncthreads();
}
// The steps j = j0, j0 / 2, .. 1 of stage k for n >= 32: element i lives in
// lane i % 32 of its warp, so partners i ^ j (j < 32) are exchanged by shuffle
// and each element is read and written once.
__device__ __forceinline__ void bitonic_steps_warp(unsigned long long* buf, uint32_t n, uint32_t k, uint32_t j0) {
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t base = threadIdx.x & ~31u; base < n; base += SMP_THREADS) {
        const uint32_t i = base + lane;
        unsigned long long x = buf[i];
        const bool desc = (i & k) == 0;
        for (uint32_t j = j0; j > 0; j >>= 1) {
            const unsigned long long y = __shfl_xor_sync(0xffffffffu, x, j);
            // the lower index of a pair keeps the larger key in a descending
            // block, the smaller in an ascending one; the upper the other
            const bool take_max = desc == ((lane & j) == 0);
            x = take_max ? (x > y ? x : y) : (x < y ? x : y);
        }
        buf[i] = x;
    }
    __syncthreads();
}
// Sorts buf[0, n) in descending order, n a power of two.
__device__ __forceinline__ void bitonic_desc(unsigned long long* buf, uint32_t n) {
    if (n < 32) {
        for (uint32_t k = 2; k <= n; k <<= 1)
            for (uint32_t j = k >> 1; j > 0; j >>= 1) bitonic_step_smem(buf, n, k, j);
        return;
    }
    for (uint32_t k = 2; k <= n; k <<= 1) {
        uint32_t j = k >> 1;
        for (; j >= 32; j >>= 1) bitonic_step_smem(buf, n, k, j);
        bitonic_steps_warp(buf, n, k, j);
    }
}

// Narrows the gathered keys buf[0, n) (probability bits << 32 | ~index, a
// prefix of the sorted order) to the keys of probability >= v for a higher
// v the walk allows: for top-p (sum) those probabilities still sum to at
// least t -- t carries the same margin over top_p as the first search, so
// the reference's running sum reaches top_p inside them -- and for top-k at
// least t of them remain, t = the walk's prefix length.  A bisection on the
// probability bits between the smallest and the largest key, one block
// reduction per step (f64 sums, fixed order), at most SMP_NARROW_STEPS
// steps, stopping at the first pivot that keeps at most `cap` keys;
// the keys kept are moved to the front (their order does not matter: they
// are sorted next).  The set stays a prefix of the sorted order, so the walk
// over it takes the same steps.  Returns the new count (n if no pivot
// qualified).  CTA-wide: every thread of the CTA calls it.
// Block reductions of the narrowing: 32-bit counts and probability bits by
// the warp reduction instructions, the f64 mass (top-p only) by shuffles;
// warp partials in shared memory, double-buffered by phase so one barrier
// per call suffices; warps combined in a fixed order (deterministic).
struct NarrowRed {
    uint32_t* wu;  // [2][SMP_WARPS][2]
    double* wd;    // [2][SMP_WARPS]
    uint32_t phase;
    __device__ __forceinline__ uint2 run(uint32_t a, uint32_t b, double m, bool want_m, bool minmax, double& msum) {
        if (minmax) {
            a = __reduce_max_sync(0xffffffffu, a);
            b = __reduce_min_sync(0xffffffffu, b);
        } else {
            a = __reduce_add_sync(0xffffffffu, a);
        }
        if (want_m) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
        }
        const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
        uint32_t* su = wu + phase * SMP_WARPS * 2;
        double* sd = wd + phase * SMP_WARPS;
        if (lane == 0) {
            su[2 * warp] = a;
            su[2 * warp + 1] = b;
            if (want_m) sd[warp] = m;
        }
        __syncthreads();
        uint2 r = make_uint2(su[0], su[1]);
        msum = want_m ? sd[0] : 0.0;
#pragma unroll
        for (int w = 1; w < SMP_WARPS; ++w) {
            const uint32_t x = su[2 * w], y = su[2 * w + 1];
            r.x = minmax ? (x > r.x ? x : r.x) : r.x + x;
            r.y = minmax ? (y < r.y ? y : r.y) : r.y;
            if (want_m) msum += sd[w];
        }
        phase ^= 1u;
        return r;
    }
};

// Narrows the gathered keys buf[0, n) (probability bits << 32 | ~index, a
// prefix of the sorted order) to the keys of probability >= v for a higher
// v the walk allows: for top-p (sum) those probabilities still sum to at
// least t -- t carries the same margin over top_p as the first search, so
// the reference's running sum reaches top_p inside them -- and for top-k at
// least t of them remain, t = the walk's prefix length.  A bisection on the
// probability bits (non-negative floats order like their bit patterns)
// between the smallest and the largest key, one block reduction per step
// (f64 sums, fixed order), at most SMP_NARROW_STEPS steps, stopping at the
// first pivot that keeps at most `cap` keys; the keys kept are moved
// to the front (their order does not matter: they are sorted next).  The set
// stays a prefix of the sorted order, so the walk over it takes the same
// steps.  Returns the new count (n if no pivot qualified).  CTA-wide: every
// thread of the CTA calls it.
__device__ uint32_t narrow_candidates(unsigned long long* buf, uint32_t n, double t, bool sum, uint32_t cap,
                                      NarrowRed& rd, uint32_t* cnt) {
    constexpr int K = SMP_GATHER / SMP_THREADS;
    unsigned long long key[K];
    uint32_t pb[K];  // probability bits; keys past n get none
    uint32_t hi_b = 0u, lo_b = 0xFFFFFFFFu;
#pragma unroll
    for (int c = 0; c < K; ++c) {
        const uint32_t i = threadIdx.x + c * SMP_THREADS;
        key[c] = i < n ? buf[i] : 0ull;
        pb[c] = (uint32_t)(key[c] >> 32);
        if (i < n) {
            hi_b = pb[c] > hi_b ? pb[c] : hi_b;
            lo_b = pb[c] < lo_b ? pb[c] : lo_b;
        }
    }
    double unused;
    const uint2 bb = rd.run(hi_b, lo_b, 0.0, false, true, unused);
    uint32_t lo = bb.y, hi = bb.x + 1u;
    uint32_t best = lo, best_c = n;
    for (int step = 0; step < SMP_NARROW_STEPS && hi - lo > 1; ++step) {
        const uint32_t mid = lo + (hi - lo) / 2;
        uint32_t cn = 0;
        double sm = 0.0;
#pragma unroll
        for (int c = 0; c < K; ++c)
            if (threadIdx.x + c * SMP_THREADS < n && pb[c] >= mid) {
                ++cn;
                if (sum) sm += (double)__uint_as_float(pb[c]);
            }
        double msum;
        const uint32_t ct = rd.run(cn, 0u, sm, sum, false, msum).x;
        if (sum ? msum >= t : (double)ct >= t) {
            lo = mid;
            best = mid;
            best_c = ct;
            if (ct <= cap) break;
        } else {
            hi = mid;
        }
    }
    if (best_c >= n) return n;  // uniform: every thread saw the same reductions
    // every thread holds its keys in registers; move the kept ones forward
    if (threadIdx.x == 0) *cnt = 0;
    __syncthreads();
#pragma unroll
    for (int c = 0; c < K; ++c)
        if (threadIdx.x + c * SMP_THREADS < n && pb[c] >= best) buf[atomicAdd(cnt, 1u)] = key[c];
    __syncthreads();
    return *cnt;
}

// sample_top_k / sample_top_p on the sorted keys (src/tokenizer.rs:182-232),
// CTA-wide.  The reference's loops repeat one sequential f32 running sum:
// sample_top_p's cumsum up to the first value >= top_p, the running total
// over the kept prefix (the same additions from 0 in the same order, so the
// total is the last of those values) and the running sum compared with
// r = u * total.  Thread 0 computes that sum once and stores every prefix
// value; r's position -- the first prefix value >= r -- is then found by all
// threads at once.  The result (a token, or SMP_FALLBACK when top-p needs
// more than the n keys of a partial row) is written to *res.
__device__ void walk_sorted_cta(const unsigned long long* buf, float* pfx, uint32_t n, bool whole_row, bool topp,
                                uint64_t top_k, float top_p, float u, uint32_t* res, uint32_t* keep_s, float* r_s) {
    auto pr = [&](uint32_t i) { return __uint_as_float((uint32_t)(buf[i] >> 32)); };
    auto ix = [&](uint32_t i) { return ~(uint32_t)buf[i]; };
    const uint32_t lim = topp ? n : (uint32_t)(top_k < n ? top_k : n);
    if (threadIdx.x == 0) {
        // the running sum in blocks of 32 additions without a branch; top-p
        // stops after the block in which it reaches top_p
        float acc = 0.0f;
        uint32_t i0 = 0;
        while (i0 < lim) {
            if (lim - i0 >= 32) {
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    acc = fadd(acc, pr(i0 + e));
                    pfx[i0 + e] = acc;
                }
                i0 += 32;
            } else {
                for (; i0 < lim; ++i0) {
                    acc = fadd(acc, pr(i0));
                    pfx[i0] = acc;
                }
            }
            if (topp && acc >= top_p) break;
        }
        *keep_s = topp ? (whole_row ? n : 0u) : lim;  // top-p: unless a running sum reaches top_p
        *res = i0;                                     // prefix values computed
    }
    __syncthreads();
    const uint32_t done = *res;
    __syncthreads();
    // top-p keeps up to the first running sum >= top_p (pfx never decreases,
    // so exactly one index, if any, is the first to reach it)
    if (topp)
        for (uint32_t i = threadIdx.x; i < done; i += SMP_THREADS)
            if (pfx[i] >= top_p && (i == 0 || pfx[i - 1] < top_p)) *keep_s = i + 1;
    __syncthreads();
    const uint32_t keep = *keep_s;
    if (threadIdx.x == 0) {
        if (keep == 0) {
            *res = SMP_FALLBACK;
        } else {
            *r_s = fmul(u, pfx[keep - 1]);
            *res = ix(keep - 1);  // the reference's answer when no running sum reaches r
        }
    }
    __syncthreads();
    if (keep == 0) return;
    const float r = *r_s;
    for (uint32_t i = threadIdx.x; i < keep; i += SMP_THREADS)
        if (pfx[i] >= r && (i == 0 || pfx[i - 1] < r)) *res = ix(i);
    __syncthreads();
}

__device__ __forceinline__ float load_logit(const float* x, uint64_t i) { return __ldg(x + i); }
__device__ __forceinline__ float load_logit(const bf16_t* x, uint64_t i) { return bf16_to_f32(__ldg(x + i)); }

// Logits 4q .. 4q + 3 of the segment into v (0 past seg): one vector load when
// the segment start is aligned to 4 elements (vx) and the group is whole.
__device__ __forceinline__ void load_group(const float* x, uint32_t q, uint32_t seg, bool vx, float (&v)[4]) {
    if (vx && 4 * q + 3 < seg) {
        const float4 f = __ldg(reinterpret_cast<const float4*>(x) + q);
        v[0] = f.x;
        v[1] = f.y;
        v[2] = f.z;
        v[3] = f.w;
        return;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = 4 * q + c < seg ? load_logit(x, 4 * q + c) : 0.0f;
}
__device__ __forceinline__ void load_group(const bf16_t* x, uint32_t q, uint32_t seg, bool vx, float (&v)[4]) {
    if (vx && 4 * q + 3 < seg) {
        const uint2 h = __ldg(reinterpret_cast<const uint2*>(x) + q);
        v[0] = bf16_lo(h.x);
        v[1] = bf16_hi(h.x);
        v[2] = bf16_lo(h.y);
        v[3] = bf16_hi(h.y);
        return;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = 4 * q + c < seg ? load_logit(x, 4 * q + c) : 0.0f;
}
constexpr int SMP_QB = 8;  // logit groups in flight per thread in the first pass

// v[c] / d for a whole group of 4: RowDiv's paired fast path on two pairs,
// the IEEE divide where it does not apply -- the same quotients as d(v[c]).
__device__ __forceinline__ void div4(const RowDiv& d, float (&v)[4]) {
    if (!d.ieee) {
        bool redo = false;
        const float2 q0 = d.fast2(make_float2(v[0], v[1]), redo);
        const float2 q1 = d.fast2(make_float2(v[2], v[3]), redo);
        if (!redo) {
            v[0] = q0.x;
            v[1] = q0.y;
            v[2] = q1.x;
            v[3] = q1.y;
            return;
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = __fdiv_rn(v[c], d.b);
}

template <typename T, int CL>
__global__ void __launch_bounds__(SMP_THREADS, 1) sample_kernel(SmpArgs a) {
    pdl_begin();
    extern __shared__ __align__(16) unsigned char smem[];
    float* sp = reinterpret_cast<float*>(smem);                                           // [SMP_SPAN]
    unsigned long long* gbuf = reinterpret_cast<unsigned long long*>(smem + SMP_SPAN * 4);  // [SMP_GATHER]
    float* pfx = reinterpret_cast<float*>(smem + SMP_SPAN * 4 + SMP_GATHER * 8);          // [SMP_GATHER]
    float4* sp4 = reinterpret_cast<float4*>(sp);
    __shared__ double2 red[2 * SMP_WARPS];
    __shared__ double2 cred[2];
    __shared__ uint32_t nred_u[2 * SMP_WARPS * 2];
    __shared__ double nred_d[2 * SMP_WARPS];
    __shared__ uint32_t gcount, gresult, wkeep, ncount, ccnt;
    __shared__ uint32_t wsum[SMP_WARPS];
    __shared__ float wr;
    Reducer<CL> rd{red, cred, 0u};
    const uint32_t crank = CL == 1 ? 0u : (uint32_t)cg::this_cluster().block_rank();
    unsigned long long* gbuf0 = gbuf;
    uint32_t* gresult0 = &gresult;
    if (CL > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        gbuf0 = cluster.map_shared_rank(gbuf, 0);
        gresult0 = cluster.map_shared_rank(&gresult, 0);
    }
    auto group_sync = [&]() {
        if (CL > 1) cg::this_cluster().sync();
        else __syncthreads();
    };
    Row<CL> row;
    row.sp = sp4;
    row.ng = a.span / 4;
    row.base = crank * a.span;
    row.vocab = a.vocab;
    row.rd = &rd;
    const uint32_t seg = a.vocab > row.base ? min(a.vocab - row.base, a.span) : 0u;  // valid slots
    const RowDiv div_t(a.temperature);
    const uint64_t groups = gridDim.x / CL;
    for (uint64_t r = blockIdx.x / CL; r < a.rows; r += groups) {
        const T* x = static_cast<const T*>(a.logits) + r * a.vocab + row.base;
        // s = x / T (the IEEE quotient: RowDiv for the row-constant divisor);
        // row max (NaN skipped, as f32::max does) and a NaN flag
        float mx = -INFINITY;
        bool nan = false;
        const bool vx = (reinterpret_cast<uintptr_t>(x) & (4 * sizeof(T) - 1)) == 0;
        for (uint32_t q0 = threadIdx.x; q0 < row.ng; q0 += SMP_THREADS * SMP_QB) {
            float v[SMP_QB][4];
#pragma unroll
            for (int k = 0; k < SMP_QB; ++k) load_group(x, q0 + k * SMP_THREADS, seg, vx, v[k]);
#pragma unroll
            for (int k = 0; k < SMP_QB; ++k) {
                const uint32_t q = q0 + k * SMP_THREADS;
                if (q >= row.ng) break;
                if (4 * q + 3 < seg) {
                    div4(div_t, v[k]);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        nan |= v[k][c] != v[k][c];
                        mx = fmaxf(mx, v[k][c]);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (4 * q + c < seg) {
                            v[k][c] = div_t(v[k][c]);
                            nan |= v[k][c] != v[k][c];
                            mx = fmaxf(mx, v[k][c]);
                        } else {
                            v[k][c] = -INFINITY;
                        }
                    }
                }
                sp4[q] = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
            }
        }
        const double2 mr = rd.template run<RMAX, RMAX>((double)mx, nan ? 1.0 : 0.0);
        const float m = (float)mr.x;
        const bool invalid = mr.y != 0.0 || isinf(m);  // exp(inf - inf) / exp(-inf + inf) is NaN
        float ls = 0.0f;
#pragma unroll 4
        for (uint32_t q = threadIdx.x; q < row.ng; q += SMP_THREADS) {
            float4 w = sp4[q];
            float* v = reinterpret_cast<float*>(&w);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (4 * q + c < seg) {
                    v[c] = expf(fsub(v[c], m));
                    ls = fadd(ls, v[c]);
                }
            }
            sp4[q] = w;
        }
        const float S = (float)rd.template run<RSUM, RSUM>((double)ls, 0.0).x;
        const RowDiv div_s(S);
        float* prow = a.probs ? a.probs + r * a.vocab + row.base : nullptr;
        const bool vp = (reinterpret_cast<uintptr_t>(prow) & 15) == 0;
#pragma unroll 4
        for (uint32_t q = threadIdx.x; q < row.ng; q += SMP_THREADS) {
            float4 w = sp4[q];
            float v[4] = {w.x, w.y, w.z, w.w};
            if (4 * q + 3 < seg) {
                div4(div_s, v);
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) v[c] = 4 * q + c < seg ? div_s(v[c]) : -1.0f;
            }
            w = make_float4(v[0], v[1], v[2], v[3]);
            if (prow) {
                if (vp && 4 * q + 3 < seg) {
                    reinterpret_cast<float4*>(prow)[q] = w;
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        if (4 * q + c < seg) prow[4 * q + c] = v[c];
                }
            }
            sp4[q] = w;
        }
        __syncthreads();  // the probabilities are in place for every thread
        if (!a.tokens) continue;
        // Every probability is <= 1, so M(bits(1) + 1) = 0.  A threshold t <= 0
        // is reached by the first element, as is the smallest positive double:
        // t is raised to that.
        constexpr uint32_t top = 0x3F800001u;
        // every probability is RN(e / S) with e <= 1 (the row max gives
        // e = 1), so none exceeds RN(1 / S): the threshold search starts
        // there instead of at 1
        const uint32_t ptop = __float_as_uint(div_s(1.0f)) + 1u;
        constexpr double tiny = 4.9406564584124654e-324;
        const bool topp = a.top_p < 1.0f;
        const uint64_t k_top = a.top_k < a.vocab ? a.top_k : a.vocab;
        uint32_t tok = 0;
        bool done = true;
        if (a.vocab == 1) {
            tok = 0;
        } else if (invalid) {
            tok = OXIDE_SAMPLE_INVALID;
        } else if (!topp && k_top == 0) {
            tok = 0;  // the reference's empty prefix returns 0
        } else {
            // the set to walk exactly: the probabilities > gv and those == gv
            // at indices <= gidx, at most SMP_GATHER of them
            uint32_t gidx = 0xFFFFFFFFu;
            bool short_prefix;
            double tq = 0.0;
            Coarse g;
            if (topp) {
                // a sequential f32 running sum of n terms is within
                // gam = n 2^-24 / (1 - n 2^-24) of the exact one, so the reference
                // reaches top_p no later than the exact sum reaches top_p (1 + 2 gam)
                const double nu = (double)a.vocab * 5.9604644775390625e-8;
                const double gam = nu / (1.0 - nu);
                tq = fmax((double)a.top_p, tiny) * (1.0 + 2.0 * gam);
                const double2 all = row.measure(0.0f);
                if (tq >= all.x) {  // the whole row
                    g = Coarse{0.0f, true, all.y, 0.0, 0.0, 0.0};
                    short_prefix = all.y <= (double)SMP_GATHER;
                } else {
                    g = row.template coarse<true>(tq, 0u, ptop, all.y, SMP_GATHER);
                    short_prefix = g.ok;
                }
            } else {
                g = row.template coarse<false>((double)k_top, 0u, ptop, (double)a.vocab, SMP_GATHER);
                short_prefix = g.ok;
            }
            const float gv = g.v;
            if (!g.ok) {
                // the prefix ends inside a run of equal probabilities gv longer
                // than SMP_GATHER: keep the elements above gv and the first m
                // of the run in index order (the stable sort's order)
                double mm = topp ? (gv > 0.0f ? ceil((tq - g.s_gt) / (double)gv) + 1.0 : g.ties)
                                 : (double)k_top - g.c_gt;
                mm = fmin(fmax(mm, 1.0), g.ties);
                if (g.c_gt + mm <= (double)SMP_GATHER) {
                    gidx = row.tie_index(gv, g.ties, mm);
                    short_prefix = true;
                }
            }
            done = false;
            if (short_prefix) {
                // gather without atomics: each thread counts its candidates, a
                // block scan gives its offset in the CTA's run, the CTAs of the
                // cluster exchange their counts, and every thread then stores
                // its candidates at its place in the first CTA's buffer
                auto take = [&](float v, uint32_t i) { return v > gv || (v == gv && i <= gidx); };
                uint32_t mine = 0;
                for (uint32_t q = threadIdx.x; q < row.ng; q += SMP_THREADS) {
                    const float4 w = sp4[q];
                    const uint32_t i0 = row.base + 4 * q;
                    mine += (uint32_t)take(w.x, i0) + (uint32_t)take(w.y, i0 + 1) + (uint32_t)take(w.z, i0 + 2) +
                            (uint32_t)take(w.w, i0 + 3);
                }
                const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
                uint32_t incl = mine;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= (uint32_t)o) incl += y;
                }
                if (lane == 31) wsum[warp] = incl;
                __syncthreads();
                uint32_t off = incl - mine, ctot = 0;
#pragma unroll
                for (int w2 = 0; w2 < SMP_WARPS; ++w2) {
                    const uint32_t c = wsum[w2];
                    off += (uint32_t)w2 < warp ? c : 0u;
                    ctot += c;
                }
                uint32_t base = 0, total = ctot;
                if constexpr (CL > 1) {
                    if (threadIdx.x == 0) ccnt = ctot;
                    cg::cluster_group cluster = cg::this_cluster();
                    cluster.sync();
                    total = 0;
#pragma unroll
                    for (int q2 = 0; q2 < CL; ++q2) {
                        const uint32_t c = *cluster.map_shared_rank(&ccnt, q2);
                        base += (uint32_t)q2 < crank ? c : 0u;
                        total += c;
                    }
                }
                uint32_t pos = base + off;
                for (uint32_t q = threadIdx.x; q < row.ng && mine != 0; q += SMP_THREADS) {
                    const float4 w = sp4[q];
                    const float v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t i = row.base + 4 * q + c;
                        if (take(v[c], i)) {
                            if (pos < (uint32_t)SMP_GATHER)
                                gbuf0[pos] = ((unsigned long long)__float_as_uint(v[c]) << 32) |
                                             (unsigned long long)(~i);
                            ++pos;
                            --mine;
                        }
                    }
                }
                if (threadIdx.x == 0) gcount = total;
                group_sync();
                if (crank == 0) {
                    uint32_t n = gcount < (uint32_t)SMP_GATHER ? gcount : (uint32_t)SMP_GATHER;
                    bool whole = n == a.vocab;
                    const uint32_t cap = topp ? SMP_SORT_CAP_P : SMP_SORT_CAP_K;
                    if (n > cap) {
                        NarrowRed lr{nred_u, nred_d, 0u};
                        const uint32_t n2 = narrow_candidates(
                            gbuf, n, topp ? tq : (double)(k_top < n ? k_top : (uint64_t)n), topp, cap, lr, &ncount);
                        whole = whole && n2 == n;
                        n = n2;
                    }
                    uint32_t np2 = 1;
                    while (np2 < n) np2 <<= 1;
                    for (uint32_t i = n + threadIdx.x; i < np2; i += SMP_THREADS) gbuf[i] = 0ull;
                    __syncthreads();
                    bitonic_desc(gbuf, np2);
                    walk_sorted_cta(gbuf, pfx, n, whole, topp, a.top_k, a.top_p, a.uniforms[r], &gresult, &wkeep,
                                    &wr);
                }
                group_sync();
                tok = *gresult0;
                done = tok != SMP_FALLBACK;
            }
        }
        if (!done) {
            // Long prefixes: the f64 running sums of the bisection stand in for
            // the sequential walk.  The kept prefix ends at (kv, kj-th tie);
            // kv < 0: the whole row.
            float kv = -1.0f;
            double kj = 0.0, kties = 0.0, total = 0.0;
            if (topp) {  // sample_top_p: shortest prefix whose sum reaches top_p
                const double t = fmax((double)a.top_p, tiny);
                const double2 all = row.measure(0.0f);
                total = all.x;
                if (all.x >= t) {
                    const Cross c = row.template bisect<true>(t, 0u, top, all.y, 0.0, 0.0, -1.0f, 0.0, false);
                    kv = c.v;
                    kj = c.j;
                    kties = c.ties;
                    total = c.cum_sum;
                }
            } else {  // sample_top_k: the first min(k, vocab) elements
                const Cross c = row.template bisect<false>((double)k_top, 0u, top, (double)a.vocab, 0.0, 0.0,
                                                           -1.0f, 0.0, false);
                kv = c.v;
                kj = c.j;
                kties = c.ties;
                total = c.cum_sum;
            }
            // r = u * total in f32, as the reference computes it; the walk
            // never passes the prefix's last element
            double t = (double)fmul(a.uniforms[r], (float)total);
            t = fmax(fmin(t, total), tiny);
            const uint32_t lo = kv >= 0.0f ? __float_as_uint(kv) : 0u;
            const double2 at = row.measure(__uint_as_float(lo));
            if (at.x >= t || kv < 0.0f)
                tok = row.template bisect<true>(fmin(t, at.x), lo, top, at.y, 0.0, 0.0, kv, kj, true).idx;
            else  // rounding left r above the prefix's measure: its last element
                tok = row.tie_index(kv, kties, kj);
        }
        if (crank == 0 && threadIdx.x == 0) a.tokens[r] = tok;
        __syncthreads();  // the segment is rewritten by the next row
    }
    if (CL > 1) cg::this_cluster().sync();  // peers' slots stay valid until read
}

template <typename T>
static int sample_entry(const char* name, const T* logits, uint64_t rows, uint64_t vocab, float temperature,
                        uint64_t top_k, float top_p, const float* uniforms, uint32_t* tokens, float* probs,
                        cudaStream_t st) {
    OXIDE_INJECT(name);
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(tokens || probs, name, "null pointer");
    OXIDE_REQUIRE(!tokens || uniforms, name, "uniforms must be given when tokens are sampled");
    if (vocab == 0) {  // empty rows: the reference's empty prefix returns 0
        const cudaError_t e = tokens ? cudaMemsetAsync(tokens, 0, rows * sizeof(uint32_t), st) : cudaSuccess;
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(OXIDE_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
        }
        return OXIDE_OK;
    }
    OXIDE_REQUIRE(logits, name, "null pointer");
    OXIDE_REQUIRE(vocab <= 8ull * SMP_SPAN, name, "vocab must be <= 262144");
    OXIDE_REQUIRE(rows <= UINT64_MAX / vocab, name, "logits size overflows");
    // the fewest CTAs per row whose segments hold it; then, while the grid
    // (one CTA per SM: the segment takes 128 KB of shared memory) would leave
    // SMs idle, split rows over twice as many, down to 4096 logits per CTA
    int cl = 1;
    while ((uint64_t)cl * SMP_SPAN < vocab) cl *= 2;
    while (cl < 8 && rows * (uint64_t)(2 * cl) <= (uint64_t)sm_count() && vocab / (uint64_t)(2 * cl) >= 4096)
        cl *= 2;
    const uint64_t per_cta = (vocab + cl - 1) / cl;
    const uint32_t span = (uint32_t)((per_cta + 3) / 4 * 4);
    const uint64_t cap = ((uint64_t)1 << 30) / (uint64_t)cl;
    const uint64_t groups = rows < cap ? rows : cap;
    SmpArgs a{logits, rows, (uint32_t)vocab, temperature, top_k, top_p, uniforms, tokens, probs, span};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(groups * cl), 1, 1);
    cfg.blockDim = dim3(SMP_THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMP_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = add_pdl_attr(attr, 1);
    const void* kern;
    switch (cl) {
        case 1: kern = reinterpret_cast<const void*>(sample_kernel<T, 1>); break;
        case 2: kern = reinterpret_cast<const void*>(sample_kernel<T, 2>); break;
        case 4: kern = reinterpret_cast<const void*>(sample_kernel<T, 4>); break;
        default: kern = reinterpret_cast<const void*>(sample_kernel<T, 8>); break;
    }
    if (!ensure_dyn_smem(kern, SMP_SMEM))
        return set_error(OXIDE_ERR_LAUNCH, "%s: cannot reserve %zu bytes of shared memory", name, SMP_SMEM);
    cudaError_t e;
    switch (cl) {
        case 1: e = cudaLaunchKernelEx(&cfg, sample_kernel<T, 1>, a); break;
        case 2: e = cudaLaunchKernelEx(&cfg, sample_kernel<T, 2>, a); break;
        case 4: e = cudaLaunchKernelEx(&cfg, sample_kernel<T, 4>, a); break;
        default: e = cudaLaunchKernelEx(&cfg, sample_kernel<T, 8>, a); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(OXIDE_ERR_LAUNCH, "%s: launch failed: %s", name, cudaGetErrorString(e));
    }
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_sample_f32(const float* logits, uint64_t rows, uint64_t vocab, float temperature, uint64_t top_k,
                     float top_p, const float* uniforms, uint32_t* tokens, float* probs, oxide_stream_t stream) {
    return oxide::sample_entry<float>("oxide_sample_f32", logits, rows, vocab, temperature, top_k, top_p, uniforms,
                                      tokens, probs, stream);
}
int oxide_sample_bf16(const oxide_bf16* logits, uint64_t rows, uint64_t vocab, float temperature, uint64_t top_k,
                      float top_p, const float* uniforms, uint32_t* tokens, float* probs, oxide_stream_t stream) {
    return oxide::sample_entry<bf16_t>("oxide_sample_bf16", reinterpret_cast<const bf16_t*>(logits), rows, vocab,
                                       temperature, top_k, top_p, uniforms, tokens, probs, stream);
}
int oxide_softmax_with_temperature_f32(const float* logits, float* probs, uint64_t rows, uint64_t vocab,
                                       float temperature, oxide_stream_t stream) {
    return oxide::sample_entry<float>("oxide_softmax_with_temperature_f32", logits, rows, vocab, temperature, 0,
                                      1.0f, nullptr, nullptr, probs, stream);
}
int oxide_softmax_with_temperature_bf16(const oxide_bf16* logits, float* probs, uint64_t rows, uint64_t vocab,
                                        float temperature, oxide_stream_t stream) {
    return oxide::sample_entry<bf16_t>("oxide_softmax_with_temperature_bf16",
                                       reinterpret_cast<const bf16_t*>(logits), rows, vocab, temperature, 0, 1.0f,
                                       nullptr, nullptr, probs, stream);
}

}  // extern "C"
