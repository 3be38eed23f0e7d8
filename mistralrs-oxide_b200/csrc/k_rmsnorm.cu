// k_rmsnorm.cu -- RMSNorm and fused residual-add + RMSNorm.
//
// Reference: src/ops/norm.rs:33-47 (per row: ss = sum x*x; rms =
// sqrt(ss / cols + eps); y = (x / rms) * w) and the residual add that
// precedes post_attention_layernorm (src/layers/transformer.rs:64-67;
// fusion intent src/kernels/normalization.rs:41-77).
//
// Design: each row is owned by a group of `tpr` threads (a warp for short
// rows, a power-of-two group with several rows per 256-thread CTA, or one CTA
// of up to 1024 threads for long rows).  The group reads the whole row with
// 16-byte streaming loads issued back to back and keeps it PACKED in
// registers (bf16 stays 2 bytes per element), four 16-byte vectors per thread
// (32 bf16 or 16 f32 elements), so the row crosses HBM once in and once out
// and many rows are in flight per SM.  The sum of
// squares is reduced with a fixed shuffle/shared-memory tree; for f32 x / rms
// uses the row-shared RowDiv (the correctly rounded quotient, as the
// reference's IEEE divide), for bf16 a multiply by the rounded reciprocal (see
// bf16_recip_ok), followed by a separate multiply by w.  Rows beyond the
// register path, or with unaligned/odd lengths, take a two-pass kernel that
// re-reads the row (the second read is served by L2).
#include "oxide_common.cuh"

namespace oxide {

struct NormArgs {
    uint64_t rows;
    uint32_t cols;
    int tpr;  // threads per row (multiple of 32; a power of 2 when < 256)
    float eps;
};

// bf16 outputs compute x / rms as x * RN(1 / rms): the product is within 1.5
// f32 ulp of the correctly rounded quotient, far inside half a bf16 ulp, so
// the bf16 result differs from the reference's by at most one ulp -- the same
// bar as the rounding of the f32 sum of squares -- and the per-element divide
// (RowDiv's residual corrections and range checks) becomes one multiply.  A
// row whose rms is outside [2^-126, 2^126] (1 / rms would leave the normal
// range) keeps the division.  f32 outputs always divide.
__device__ __forceinline__ bool bf16_recip_ok(float rms) {
    return rms >= 0x1p-126f && rms <= 0x1p126f;
}

// Vectors per thread: 4 (32 bf16 or 16 f32 elements).  Measured on B200 at
// 4096 columns: f32 rows run 10-20% faster with 16 elements per thread and
// twice the threads per row than with 32, and bf16 rows fastest with 32.
template <typename T, bool ADD>
constexpr int norm_vpt() {
    return 4;
}

// Sum of squares of one unpacked vector into two lane accumulators, each term
// added with a fused multiply-add (one rounding per term; the reference's
// `ss += v * v` rounds the product first -- on sm_100a a paired multiply
// feeding a paired add comes out fused anyway, so the fused form is explicit).
// The lanes are combined after the thread's last vector.
template <int V>
__device__ __forceinline__ void sumsq_add(float2& acc, const float (&v)[V]) {
#pragma unroll
    for (int e = 0; e < V; e += 2) {
        const float2 p = f2(v[e], v[e + 1]);
        acc = __ffma2_rn(p, p, acc);
    }
}

// y = (v / rms) * w for a thread's VPT packed vectors j = t + k * tpr < jhi.
// RowDiv's paired fast path per vector; a vector holding a numerator outside
// its range (or a row whose rms is outside it) is redone with the IEEE divide.
template <typename T, int VPT>
__device__ __forceinline__ void norm_store_rms(T* yrow, const T* w, const uint4 (&raw)[VPT],
                                               uint32_t t, uint32_t tpr, uint32_t jhi, float rms) {
    constexpr int V = Vec<T>::N;
    if (V == 8 && bf16_recip_ok(rms)) {
        // bf16 output: (x * RN(1 / rms)) * w -- see bf16_recip_ok
        const float inv = __frcp_rn(rms);
        const float2 inv2 = f2(inv, inv);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * tpr;
            if (j < jhi) {
                float v[V], wv[V], o[V];
                Vec<T>::unpack(raw[k], v);
                Vec<T>::unpack(ld_keep(w + (uint64_t)j * V), wv);
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 oo = fmul2(fmul2(f2(v[e], v[e + 1]), inv2), f2(wv[e], wv[e + 1]));
                    o[e] = oo.x;
                    o[e + 1] = oo.y;
                }
                st_stream(yrow + (uint64_t)j * V, Vec<T>::pack(o));
            }
        }
        return;
    }
    const RowDiv div(rms);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = t + k * tpr;
        if (j < jhi) {
            float v[V], wv[V], q[V], o[V];
            Vec<T>::unpack(raw[k], v);
            Vec<T>::unpack(ld_keep(w + (uint64_t)j * V), wv);
            bool redo = div.ieee;
#pragma unroll
            for (int e = 0; e < V; e += 2) {
                const float2 qq = div.fast2(f2(v[e], v[e + 1]), redo);
                q[e] = qq.x;
                q[e + 1] = qq.y;
            }
            if (redo) {
#pragma unroll
                for (int e = 0; e < V; ++e) q[e] = __fdiv_rn(v[e], rms);
            }
#pragma unroll
            for (int e = 0; e < V; e += 2) {
                const float2 oo = fmul2(f2(q[e], q[e + 1]), f2(wv[e], wv[e + 1]));
                o[e] = oo.x;
                o[e + 1] = oo.y;
            }
            st_stream(yrow + (uint64_t)j * V, Vec<T>::pack(o));
        }
    }
}

// BIG: one row per CTA of up to 1024 threads; otherwise 256-thread CTAs with a
// register budget of 6 CTAs per SM (40 registers) for RMSNorm and 4 (64) for
// add + RMSNorm, which holds both inputs.  Measured on the C5 rows: RMSNorm bf16
// 341.8 / 327.0 / 314.6 us at 4 / 5 / 6 CTAs per SM (the few registers spilled
// at 6 cost less than the rows gained in flight); add + RMSNorm 621 / 660 / 745.
template <typename T, int VPT, bool ADD, bool BIG>
__global__ void __launch_bounds__(BIG ? 1024 : 256, BIG ? 1 : (ADD ? 4 : 6))
    rmsnorm_vec_kernel(const T* x, const T* r, const T* w, T* h, T* y, NormArgs p) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    __shared__ float red[32];
    const int rpc = blockDim.x / p.tpr;
    const int sub = threadIdx.x / p.tpr, t = threadIdx.x % p.tpr;
    const uint32_t nvec = p.cols / V;
    for (uint64_t row0 = (uint64_t)blockIdx.x * rpc; row0 < p.rows;
         row0 += (uint64_t)gridDim.x * rpc) {
        const uint64_t row = row0 + sub;
        const bool active = row < p.rows;
        const uint64_t off = row * p.cols;
        uint4 raw[VPT], rawr[ADD ? VPT : 1];
        // Issue every load of the row before using any of them.
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                raw[k] = ld_stream(x + off + (uint64_t)j * V);
                if (ADD) rawr[k] = ld_stream(r + off + (uint64_t)j * V);
            }
        }
        // pass 1: h = x + r (stored, kept packed in raw) and the sum of squares
        float2 acc = f2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                float v[V];
                Vec<T>::unpack(raw[k], v);
                if (ADD) {
                    float rv[V];
                    Vec<T>::unpack(rawr[ADD ? k : 0], rv);
#pragma unroll
                    for (int e = 0; e < V; e += 2) {
                        const float2 s = fadd2(f2(v[e], v[e + 1]), f2(rv[e], rv[e + 1]));
                        v[e] = Vec<T>::rnd(s.x);
                        v[e + 1] = Vec<T>::rnd(s.y);
                    }
                    raw[k] = Vec<T>::pack(v);  // exact: v already holds T values
                    st_stream(h + off + (uint64_t)j * V, raw[k]);
                }
                sumsq_add(acc, v);
            }
        }
        const float ss = group_reduce(fadd(acc.x, acc.y), red, p.tpr, OpAddF());
        // pass 2: y = (h / rms) * w
        norm_store_rms<T, VPT>(y + off, w, raw, t, p.tpr, active ? nvec : 0,
                               fsqrt(fadd(fdiv(ss, (float)p.cols), p.eps)));
    }
}

// Two-pass fallback: any cols, any alignment.  One CTA per row.  Pass 2
// re-reads x (or the stored h) with coherent loads, so in-place use is safe.
template <typename T, bool ADD>
__global__ void __launch_bounds__(256)
    rmsnorm_scalar_kernel(const T* x, const T* r, const T* w, T* h, T* y, NormArgs p) {
    pdl_begin();
    __shared__ float red[32];
    for (uint64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint64_t off = row * p.cols;
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < p.cols; i += blockDim.x) {
            float v = Vec<T>::load1(x + off + i);
            if (ADD) {
                v = Vec<T>::rnd(fadd(v, Vec<T>::load1(r + off + i)));
                Vec<T>::store1(h + off + i, v);
            }
            ss = __fmaf_rn(v, v, ss);  // one rounding per term, as sumsq_add
        }
        ss = group_reduce(ss, red, (int)blockDim.x, OpAddF());
        const float rms = fsqrt(fadd(fdiv(ss, (float)p.cols), p.eps));
        const RowDiv div(rms);
        const bool recip = sizeof(T) == 2 && bf16_recip_ok(rms);
        const float inv = __frcp_rn(rms);
        const T* src = ADD ? h : x;
        for (uint32_t i = threadIdx.x; i < p.cols; i += blockDim.x) {
            const T* q = src + off + i;
            float v;
            if (sizeof(T) == 4) v = *reinterpret_cast<const volatile float*>(q);
            else v = bf16_to_f32(*reinterpret_cast<const volatile uint16_t*>(q));
            Vec<T>::store1(y + off + i, fmul(recip ? fmul(v, inv) : div(v), Vec<T>::load1(w + i)));
        }
    }
}

template <typename T, int VPT, bool ADD, bool BIG>
static void launch_norm_vec(const T* x, const T* r, const T* w, T* h, T* y, NormArgs p,
                            cudaStream_t st) {
    const int rpc = p.tpr >= 256 ? 1 : 256 / p.tpr;
    const int threads = p.tpr * rpc;
    const uint64_t want = (p.rows + rpc - 1) / rpc;
    const uint64_t cap = (uint64_t)1 << 30;
    launch_k(rmsnorm_vec_kernel<T, VPT, ADD, BIG>, (unsigned)(want < cap ? want : cap), threads, 0, st, x, r, w, h, y, p);
}

template <typename T, bool ADD>
static int norm_dispatch(const char* name, const T* x, const T* r, const T* w, T* h, T* y,
                         uint64_t rows, uint64_t cols, float eps, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    constexpr int VT = norm_vpt<T, ADD>();
    NormArgs p{rows, (uint32_t)cols, 32, eps};
    const bool vec = cols % V == 0 && aligned16(x) && aligned16(w) && aligned16(y) &&
                     (!ADD || (aligned16(r) && aligned16(h)));
    const uint64_t nvec = cols / V;
    if (vec && nvec <= 32ull * VT) {  // short rows: a warp per row, 8 rows per CTA
        int vpt = 1;
        while ((uint64_t)vpt * 32 < nvec) vpt *= 2;
        if (vpt == VT) launch_norm_vec<T, VT, ADD, false>(x, r, w, h, y, p, st);
        else if (vpt == 1) launch_norm_vec<T, 1, ADD, false>(x, r, w, h, y, p, st);
        else if (vpt == 2) launch_norm_vec<T, 2, ADD, false>(x, r, w, h, y, p, st);
        else launch_norm_vec<T, (VT >= 4 ? 4 : VT), ADD, false>(x, r, w, h, y, p, st);
    } else if (vec && nvec <= 256ull * VT) {  // 64..256 threads per row
        uint64_t tpr = 64;
        while (tpr * VT < nvec) tpr *= 2;
        p.tpr = (int)tpr;
        launch_norm_vec<T, VT, ADD, false>(x, r, w, h, y, p, st);
    } else if (vec && nvec <= 1024ull * VT) {  // one CTA of up to 1024 threads per row
        p.tpr = (int)(((nvec + VT - 1) / VT + 31) / 32 * 32);
        launch_norm_vec<T, VT, ADD, true>(x, r, w, h, y, p, st);
    } else {
        const uint64_t cap = (uint64_t)1 << 30;
        launch_k(rmsnorm_scalar_kernel<T, ADD>, (unsigned)(rows < cap ? rows : cap), 256, 0, st, x, r, w, h, y, p);
    }
    return check_launch(name);
}

template <typename T>
static int rms_entry(const char* name, const T* x, const T* w, T* y, uint64_t rows,
                     uint64_t cols, float eps, cudaStream_t st) {
    OXIDE_INJECT(name);
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && w && y, name, "null pointer");
    OXIDE_REQUIRE(cols >= 1 && cols < (1ull << 31), name, "cols must be in [1, 2^31)");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    return norm_dispatch<T, false>(name, x, nullptr, w, nullptr, y, rows, cols, eps, st);
}

template <typename T>
static int add_rms_entry(const char* name, const T* x, const T* r, const T* w, T* h, T* y,
                         uint64_t rows, uint64_t cols, float eps, cudaStream_t st) {
    OXIDE_INJECT(name);
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && r && w && h && y, name, "null pointer");
    OXIDE_REQUIRE(h != y, name, "h and y must not alias");
    OXIDE_REQUIRE(cols >= 1 && cols < (1ull << 31), name, "cols must be in [1, 2^31)");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    return norm_dispatch<T, true>(name, x, r, w, h, y, rows, cols, eps, st);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_rms_norm_f32(const float* x, const float* w, float* out, uint64_t rows, uint64_t cols,
                       float eps, oxide_stream_t stream) {
    return oxide::rms_entry<float>("oxide_rms_norm_f32", x, w, out, rows, cols, eps, stream);
}
int oxide_rms_norm_bf16(const oxide_bf16* x, const oxide_bf16* w, oxide_bf16* out,
                        uint64_t rows, uint64_t cols, float eps, oxide_stream_t stream) {
    return oxide::rms_entry<bf16_t>("oxide_rms_norm_bf16", x, w, out, rows, cols, eps, stream);
}
int oxide_add_rms_norm_f32(const float* x, const float* r, const float* w, float* h, float* y,
                           uint64_t rows, uint64_t cols, float eps, oxide_stream_t stream) {
    return oxide::add_rms_entry<float>("oxide_add_rms_norm_f32", x, r, w, h, y, rows, cols, eps,
                                       stream);
}
int oxide_add_rms_norm_bf16(const oxide_bf16* x, const oxide_bf16* r, const oxide_bf16* w,
                            oxide_bf16* h, oxide_bf16* y, uint64_t rows, uint64_t cols,
                            float eps, oxide_stream_t stream) {
    return oxide::add_rms_entry<bf16_t>("oxide_add_rms_norm_bf16", x, r, w, h, y, rows, cols,
                                        eps, stream);
}

}  // extern "C"
