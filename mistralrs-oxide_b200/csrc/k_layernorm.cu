// k_layernorm.cu -- LayerNorm over the last dimension.
//
// Reference: src/ops/norm.rs:92-113 (per row: sum -> mean = sum / cols; sum of
// (x - mean)^2 -> var = sum_sq / cols; std = sqrt(var + eps); out =
// ((x - mean) / std) * w + b) and KernelManager::launch_layer_norm
// (src/cuda_backend/kernels.rs:334-356).
//
// The fused add variant (oxide_add_layer_norm_*) normalises x + r, as the
// reference's layer_norm_fused_add_f32 (src/kernels/normalization.rs:123-167)
// intends, with the sum rounded to the I/O type first (exact for f32), so the
// fused op equals add followed by layer_norm; the sum is not stored.
//
// Design: the row layout of the RMSNorm kernels -- a group of `tpr` threads
// per row (a warp for short rows, 64..256 threads with several rows per
// 256-thread CTA, or one CTA of up to 1024 threads), the whole row read once
// with 16-byte streaming loads and kept packed in registers (four vectors per
// thread) -- with two fixed-tree reductions (the sum, then the sum of squared
// deviations from the mean; two-pass like the reference, not the one-pass
// E[x^2] - E[x]^2), then the output from registers.  Rounding: x - mean,
// (x - mean)^2 accumulated with a fused multiply-add, the IEEE divide by std
// (RowDiv; f32) or a multiply by RN(1 / std) (bf16 outputs), then
// normalized * w + b as one fused multiply-add.  Rows beyond the register
// path or with unaligned/odd lengths take a three-pass kernel that re-reads
// the row (served by L2).
#include "oxide_common.cuh"

namespace oxide {

struct LnArgs {
    uint64_t rows;
    uint32_t cols;
    int tpr;  // threads per row
    float eps;
};

constexpr int LN_VPT = 4;  // 16-byte vectors per thread

// y = ((x - mean) / sd) * w + b for a thread's VPT packed vectors.
template <typename T, int VPT>
__device__ __forceinline__ void ln_store(T* yrow, const T* w, const T* b, const uint4 (&raw)[VPT],
                                         uint32_t t, uint32_t tpr, uint32_t jhi, float mean, float sd) {
    constexpr int V = Vec<T>::N;
    const RowDiv div(sd);
    const bool recip = V == 8 && sd >= 0x1p-126f && sd <= 0x1p126f;  // bf16 output (see k_rmsnorm.cu)
    const float inv = __frcp_rn(sd);
    const float2 nm = f2(-mean, -mean);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = t + k * tpr;
        if (j < jhi) {
            float v[V], wv[V], bv[V], q[V], o[V];
            Vec<T>::unpack(raw[k], v);
            Vec<T>::unpack(ld_keep(w + (uint64_t)j * V), wv);
            Vec<T>::unpack(ld_keep(b + (uint64_t)j * V), bv);
#pragma unroll
            for (int e = 0; e < V; e += 2) {
                const float2 d = fadd2(f2(v[e], v[e + 1]), nm);
                v[e] = d.x;
                v[e + 1] = d.y;
            }
            if (recip) {
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 qq = fmul2(f2(v[e], v[e + 1]), f2(inv, inv));
                    q[e] = qq.x;
                    q[e + 1] = qq.y;
                }
            } else {
                bool redo = div.ieee;
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 qq = div.fast2(f2(v[e], v[e + 1]), redo);
                    q[e] = qq.x;
                    q[e + 1] = qq.y;
                }
                if (redo) {
#pragma unroll
                    for (int e = 0; e < V; ++e) q[e] = __fdiv_rn(v[e], sd);
                }
            }
#pragma unroll
            for (int e = 0; e < V; e += 2) {
                const float2 oo = __ffma2_rn(f2(q[e], q[e + 1]), f2(wv[e], wv[e + 1]), f2(bv[e], bv[e + 1]));
                o[e] = oo.x;
                o[e + 1] = oo.y;
            }
            st_stream(yrow + (uint64_t)j * V, Vec<T>::pack(o));
        }
    }
}

// 5 CTAs of 256 threads per SM (51 registers): measured 446 us on the C5 rows
// (bf16) against 457 at 4 and 464 at 6; 15.7 us against 16.4 / 21.3 at C1 (f32).
// The add variant holds both inputs in flight: 4 CTAs per SM, 568 us for the
// bf16 C5 rows against 602 at 3.
template <typename T, int VPT, bool BIG, bool ADD>
__global__ void __launch_bounds__(BIG ? 1024 : 256, BIG ? 1 : (ADD ? 4 : 5))
    layernorm_vec_kernel(const T* x, const T* r, const T* w, const T* b, T* y, LnArgs p) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    __shared__ float red[32];
    const int rpc = blockDim.x / p.tpr;
    const int sub = threadIdx.x / p.tpr, t = threadIdx.x % p.tpr;
    const uint32_t nvec = p.cols / V;
    for (uint64_t row0 = (uint64_t)blockIdx.x * rpc; row0 < p.rows; row0 += (uint64_t)gridDim.x * rpc) {
        const uint64_t row = row0 + sub;
        const bool active = row < p.rows;
        const uint64_t off = row * p.cols;
        uint4 raw[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) raw[k] = ld_stream(x + off + (uint64_t)j * V);
        }
        if (ADD) {  // the row is x + r, rounded to T as the add's output would be
            uint4 rr[VPT];
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const uint32_t j = t + k * p.tpr;
                if (active && j < nvec) rr[k] = ld_stream(r + off + (uint64_t)j * V);
            }
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const uint32_t j = t + k * p.tpr;
                if (active && j < nvec) {
                    float u[V], v[V];
                    Vec<T>::unpack(raw[k], u);
                    Vec<T>::unpack(rr[k], v);
#pragma unroll
                    for (int e = 0; e < V; ++e) u[e] = fadd(u[e], v[e]);
                    raw[k] = Vec<T>::pack(u);
                }
            }
        }
        // pass 1: the mean
        float2 acc = f2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                float v[V];
                Vec<T>::unpack(raw[k], v);
#pragma unroll
                for (int e = 0; e < V; e += 2) acc = fadd2(acc, f2(v[e], v[e + 1]));
            }
        }
        const float mean = fdiv(group_reduce(fadd(acc.x, acc.y), red, p.tpr, OpAddF()), (float)p.cols);
        // pass 2: the variance of the deviations
        const float2 nm = f2(-mean, -mean);
        acc = f2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                float v[V];
                Vec<T>::unpack(raw[k], v);
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 d = fadd2(f2(v[e], v[e + 1]), nm);
                    acc = __ffma2_rn(d, d, acc);
                }
            }
        }
        const float var = fdiv(group_reduce(fadd(acc.x, acc.y), red, p.tpr, OpAddF()), (float)p.cols);
        ln_store<T, VPT>(y + off, w, b, raw, t, p.tpr, active ? nvec : 0, mean, fsqrt(fadd(var, p.eps)));
    }
}

// Three-pass fallback: any cols, any alignment; one CTA per row.  The output
// pass re-reads x with coherent loads, so in-place use is safe.
template <typename T, bool ADD>
__global__ void __launch_bounds__(256) layernorm_scalar_kernel(const T* x, const T* r, const T* w, const T* b,
                                                               T* y, LnArgs p) {
    pdl_begin();
    __shared__ float red[32];
    // element i of the row: x, or x + r rounded to T
    auto val = [&](uint64_t i) {
        const float v = Vec<T>::load1(x + i);
        return ADD ? Vec<T>::rnd(fadd(v, Vec<T>::load1(r + i))) : v;
    };
    for (uint64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint64_t off = row * p.cols;
        float s = 0.0f;
        for (uint32_t i = threadIdx.x; i < p.cols; i += blockDim.x) s = fadd(s, val(off + i));
        const float mean = fdiv(group_reduce(s, red, (int)blockDim.x, OpAddF()), (float)p.cols);
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < p.cols; i += blockDim.x) {
            const float d = fsub(val(off + i), mean);
            ss = __fmaf_rn(d, d, ss);
        }
        const float var = fdiv(group_reduce(ss, red, (int)blockDim.x, OpAddF()), (float)p.cols);
        const float sd = fsqrt(fadd(var, p.eps));
        const RowDiv div(sd);
        const bool recip = sizeof(T) == 2 && sd >= 0x1p-126f && sd <= 0x1p126f;
        const float inv = __frcp_rn(sd);
        __syncthreads();  // every thread has read its inputs before any write (in place)
        for (uint32_t i = threadIdx.x; i < p.cols; i += blockDim.x) {
            auto vload = [](const T* q) {
                return sizeof(T) == 4 ? *reinterpret_cast<const volatile float*>(q)
                                      : bf16_to_f32(*reinterpret_cast<const volatile uint16_t*>(q));
            };
            float v = vload(x + off + i);
            if (ADD) v = Vec<T>::rnd(fadd(v, vload(r + off + i)));
            const float d = fsub(v, mean);
            const float nrm = recip ? fmul(d, inv) : div(d);
            Vec<T>::store1(y + off + i, __fmaf_rn(nrm, Vec<T>::load1(w + i), Vec<T>::load1(b + i)));
        }
    }
}

template <typename T, int VPT, bool BIG>
static void launch_ln_vec(const T* x, const T* r, const T* w, const T* b, T* y, LnArgs p, cudaStream_t st) {
    const int rpc = p.tpr >= 256 ? 1 : 256 / p.tpr;
    const uint64_t want = (p.rows + rpc - 1) / rpc, cap = (uint64_t)1 << 30;
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    if (r) launch_k(layernorm_vec_kernel<T, VPT, BIG, true>, grid, p.tpr * rpc, 0, st, x, r, w, b, y, p);
    else launch_k(layernorm_vec_kernel<T, VPT, BIG, false>, grid, p.tpr * rpc, 0, st, x, r, w, b, y, p);
}

// add: layer_norm(x + r); otherwise layer_norm(x) (r unused).
template <typename T>
static int ln_entry(const char* name, const T* x, bool add, const T* r, const T* w, const T* b, T* y,
                    uint64_t rows, uint64_t cols, float eps, cudaStream_t st) {
    constexpr int V = Vec<T>::N, VT = LN_VPT;
    OXIDE_INJECT(name);
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && w && b && y && (!add || r), name, "null pointer");
    if (!add) r = nullptr;
    OXIDE_REQUIRE(cols >= 1 && cols < (1ull << 31), name, "cols must be in [1, 2^31)");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    LnArgs p{rows, (uint32_t)cols, 32, eps};
    const bool vec = cols % V == 0 && aligned16(x) && aligned16(w) && aligned16(b) && aligned16(y) &&
                     (!r || aligned16(r));
    const uint64_t nvec = cols / V;
    if (vec && nvec <= 32ull * VT) {  // a warp per row
        if (nvec <= 32) launch_ln_vec<T, 1, false>(x, r, w, b, y, p, st);
        else if (nvec <= 64) launch_ln_vec<T, 2, false>(x, r, w, b, y, p, st);
        else launch_ln_vec<T, VT, false>(x, r, w, b, y, p, st);
    } else if (vec && nvec <= 256ull * VT) {  // 64..256 threads per row
        uint64_t tpr = 64;
        while (tpr * VT < nvec) tpr *= 2;
        p.tpr = (int)tpr;
        launch_ln_vec<T, VT, false>(x, r, w, b, y, p, st);
    } else if (vec && nvec <= 1024ull * VT) {  // one CTA of up to 1024 threads per row
        p.tpr = (int)(((nvec + VT - 1) / VT + 31) / 32 * 32);
        launch_ln_vec<T, VT, true>(x, r, w, b, y, p, st);
    } else {
        const uint64_t cap = (uint64_t)1 << 30;
        const unsigned grid = (unsigned)(rows < cap ? rows : cap);
        if (r) launch_k(layernorm_scalar_kernel<T, true>, grid, 256, 0, st, x, r, w, b, y, p);
        else launch_k(layernorm_scalar_kernel<T, false>, grid, 256, 0, st, x, r, w, b, y, p);
    }
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_layer_norm_f32(const float* x, const float* w, const float* b, float* out, uint64_t rows,
                         uint64_t cols, float eps, oxide_stream_t stream) {
    return oxide::ln_entry<float>("oxide_layer_norm_f32", x, false, nullptr, w, b, out, rows, cols, eps, stream);
}
int oxide_layer_norm_bf16(const oxide_bf16* x, const oxide_bf16* w, const oxide_bf16* b,
                          oxide_bf16* out, uint64_t rows, uint64_t cols, float eps,
                          oxide_stream_t stream) {
    return oxide::ln_entry<bf16_t>("oxide_layer_norm_bf16", x, false, nullptr, w, b, out, rows, cols, eps, stream);
}
int oxide_add_layer_norm_f32(const float* x, const float* r, const float* w, const float* b, float* out,
                             uint64_t rows, uint64_t cols, float eps, oxide_stream_t stream) {
    return oxide::ln_entry<float>("oxide_add_layer_norm_f32", x, true, r, w, b, out, rows, cols, eps, stream);
}
int oxide_add_layer_norm_bf16(const oxide_bf16* x, const oxide_bf16* r, const oxide_bf16* w,
                              const oxide_bf16* b, oxide_bf16* out, uint64_t rows, uint64_t cols, float eps,
                              oxide_stream_t stream) {
    return oxide::ln_entry<bf16_t>("oxide_add_layer_norm_bf16", x, true, r, w, b, out, rows, cols, eps,
                                   stream);
}

}  // extern "C"
