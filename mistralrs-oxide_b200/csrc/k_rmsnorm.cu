// k_rmsnorm.cu -- RMSNorm and fused residual-add + RMSNorm.
//
// Reference: src/ops/norm.rs:33-47 (per row: ss = sum x*x; rms =
// sqrt(ss / cols + eps); y = (x / rms) * w) and the residual add that
// precedes post_attention_layernorm (src/layers/transformer.rs:64-67;
// fusion intent src/kernels/normalization.rs:41-77).
//
// Design: each row is owned by a group of `tpr` threads (a warp for short
// rows, up to 1024 threads for long ones) that loads the whole row into
// registers with 16-byte streaming reads issued back to back, so the row
// crosses HBM exactly once in and once out.  Each thread holds 16 row
// elements (32 for rows beyond 16K elements), which keeps every instance
// inside its register budget without spills.  The sum of squares is reduced
// with a fixed shuffle/shared-memory tree; the normalisation keeps the
// reference's IEEE divide and separate multiply.  Rows beyond the register
// path, or with unaligned/odd lengths, take a two-pass kernel that re-reads
// the row (the second read is served by L2).
#include "oxide_rowstream.cuh"

namespace oxide {

struct NormArgs {
    uint64_t rows;
    uint32_t cols;
    int tpr;  // threads per row (multiple of 32; a power of 2 when < 256)
    float eps;
};

// Row elements held per thread: EPT = VPT * V.  Plain RMSNorm with EPT <= 16
// fits a 64-register budget (blocks up to 1024 threads); the fused add (two
// inputs in flight) and EPT = 32 use blocks of at most 512 threads so up to
// 128 registers are available.
template <typename T, int VPT, bool ADD>
constexpr int norm_block_cap() {
    return (VPT * Vec<T>::N <= 16 && !ADD) ? 1024 : 512;
}

template <typename T, int VPT, bool ADD>
__global__ void __launch_bounds__(norm_block_cap<T, VPT, ADD>())
    rmsnorm_vec_kernel(const T* x, const T* r, const T* w, T* h, T* y, NormArgs p) {
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
        float v[VPT][V];
        uint4 raw[VPT], rawr[VPT];
        // Issue every load of the row before using any of them.
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                raw[k] = ld_stream(x + off + (uint64_t)j * V);
                if (ADD) rawr[k] = ld_stream(r + off + (uint64_t)j * V);
            }
        }
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                Vec<T>::unpack(raw[k], v[k]);
                if (ADD) {
                    float rv[V];
                    Vec<T>::unpack(rawr[k], rv);
#pragma unroll
                    for (int e = 0; e < V; ++e) v[k][e] = Vec<T>::rnd(fadd(v[k][e], rv[e]));
                    st_stream(h + off + (uint64_t)j * V, Vec<T>::pack(v[k]));
                }
#pragma unroll
                for (int e = 0; e < V; ++e) ss = fadd(ss, fmul(v[k][e], v[k][e]));
            }
        }
        ss = group_reduce(ss, red, p.tpr, OpAddF());
        const float rms = fsqrt(fadd(fdiv(ss, (float)p.cols), p.eps));
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                float wv[V], o[V];
                Vec<T>::unpack(ld_keep(w + (uint64_t)j * V), wv);
#pragma unroll
                for (int e = 0; e < V; ++e) o[e] = fmul(fdiv(v[k][e], rms), wv[e]);
                st_stream(y + off + (uint64_t)j * V, Vec<T>::pack(o));
            }
        }
    }
}

// Two-pass fallback: any cols, any alignment.  One CTA per row.  Pass 2
// re-reads x (or the stored h) with coherent loads, so in-place use is safe.
template <typename T, bool ADD>
__global__ void __launch_bounds__(256)
    rmsnorm_scalar_kernel(const T* x, const T* r, const T* w, T* h, T* y, NormArgs p) {
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
            ss = fadd(ss, fmul(v, v));
        }
        ss = group_reduce(ss, red, (int)blockDim.x, OpAddF());
        const float rms = fsqrt(fadd(fdiv(ss, (float)p.cols), p.eps));
        const T* src = ADD ? h : x;
        for (uint32_t i = threadIdx.x; i < p.cols; i += blockDim.x) {
            const T* q = src + off + i;
            float v;
            if (sizeof(T) == 4) v = *reinterpret_cast<const volatile float*>(q);
            else v = bf16_to_f32(*reinterpret_cast<const volatile uint16_t*>(q));
            Vec<T>::store1(y + off + i, fmul(fdiv(v, rms), Vec<T>::load1(w + i)));
        }
    }
}

template <typename T, int VPT, bool ADD>
static void launch_norm_vec(const T* x, const T* r, const T* w, T* h, T* y, NormArgs p,
                            cudaStream_t st) {
    const int rpc = p.tpr >= 256 ? 1 : 256 / p.tpr;
    const int threads = p.tpr * rpc;
    const uint64_t want = (p.rows + rpc - 1) / rpc;
    const uint64_t cap = (uint64_t)1 << 30;
    rmsnorm_vec_kernel<T, VPT, ADD>
        <<<(unsigned)(want < cap ? want : cap), threads, 0, st>>>(x, r, w, h, y, p);
}

// Kernel shape for a row of nvec 16-byte vectors: returns VPT (0 = fallback)
// and the threads per row.
template <typename T, bool ADD>
static int norm_shape(uint64_t nvec, uint64_t* tpr_out) {
    constexpr int VPT16 = 16 / Vec<T>::N;  // vectors per thread for 16 elements
    constexpr uint64_t MAX16 = ADD ? 512 : 1024;  // block cap of the EPT-16 instance
    int vpt = 0;
    uint64_t tpr = 32;
    if (nvec <= 32ull * VPT16) {  // short rows: a warp per row, 8 rows per CTA
        vpt = 1;
        while ((uint64_t)vpt * 32 < nvec) vpt *= 2;
    } else if (nvec <= MAX16 * VPT16) {
        vpt = VPT16;
        tpr = (nvec + vpt - 1) / vpt;
    } else if (nvec <= 512ull * 2 * VPT16) {
        vpt = 2 * VPT16;
        tpr = (nvec + vpt - 1) / vpt;
    }
    if (tpr < 256) {  // sub-CTA groups must tile a 256-thread CTA: a power of 2
        uint64_t t2 = 32;
        while (t2 < tpr) t2 *= 2;
        tpr = t2;
    } else {
        tpr = (tpr + 31) / 32 * 32;
    }
    *tpr_out = tpr;
    return vpt;
}

template <typename T, bool ADD>
static int norm_dispatch(const char* name, const T* x, const T* r, const T* w, T* h, T* y,
                         uint64_t rows, uint64_t cols, float eps, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    // Rows of 2-32 KiB stream through the shared-memory bulk-copy ring.
    if (rms_stream_launch<T>(x, ADD ? r : nullptr, w, h, y, rows, (uint32_t)cols, eps, st))
        return check_launch(name);
    NormArgs p{rows, (uint32_t)cols, 32, eps};
    const bool vec = cols % V == 0 && aligned16(x) && aligned16(w) && aligned16(y) &&
                     (!ADD || (aligned16(r) && aligned16(h)));
    uint64_t tpr = 32;
    const int vpt = vec ? norm_shape<T, ADD>(cols / V, &tpr) : 0;
    p.tpr = (int)tpr;
    bool launched = true;
    if (vpt == 1) launch_norm_vec<T, 1, ADD>(x, r, w, h, y, p, st);
    else if (vpt == 2) launch_norm_vec<T, 2, ADD>(x, r, w, h, y, p, st);
    else if (vpt == 4) launch_norm_vec<T, 4, ADD>(x, r, w, h, y, p, st);
    else if constexpr (V == 4) {
        if (vpt == 8) launch_norm_vec<T, 8, ADD>(x, r, w, h, y, p, st);
        else launched = false;
    } else {
        launched = false;
    }
    if (!launched) {
        const uint64_t cap = (uint64_t)1 << 30;
        rmsnorm_scalar_kernel<T, ADD>
            <<<(unsigned)(rows < cap ? rows : cap), 256, 0, st>>>(x, r, w, h, y, p);
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
