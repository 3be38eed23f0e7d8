// k_reduce.cu -- row and whole-tensor sum / max / sum of squares.
//
// API additions: the reference has these only inline (sum of squares
// src/ops/norm.rs:36-40, max src/ops/activation.rs:99-103, running sum
// src/ops/activation.rs:105-110).  Row results are f32 like those loops; the
// whole-tensor result is f64, because a sequential f32 sum over ~10^8-10^9
// terms stalls once the running sum's ulp exceeds the terms.
//
// Whole-tensor design (deterministic for a given n): stage 1 deals the whole
// 16-byte vectors of x to at most RED_BLOCKS CTAs in grid-stride order; each
// thread keeps per-lane f32 partials, the CTA combines them in f64 with a
// fixed tree and writes one f64 partial to the workspace.  Stage 2,
// one CTA, combines the partials in a fixed order.  No atomics, no
// initialised state: the workspace is only ever written before it is read.
#include "oxide_common.cuh"

#include <atomic>
#include <mutex>

namespace oxide {

constexpr int RED_BLOCKS = 1024;
constexpr int RED_THREADS = 256;

template <int OP>
__device__ __forceinline__ float red_step(float acc, float v) {
    if (OP == OXIDE_RED_SUM) return fadd(acc, v);
    if (OP == OXIDE_RED_MAX) return fmaxf(acc, v);
    return fadd(acc, fmul(v, v));
}
template <int OP>
__device__ __forceinline__ double red_comb(double a, double b) {
    return OP == OXIDE_RED_MAX ? fmax(a, b) : a + b;
}
template <int OP>
__device__ __forceinline__ float red_init() {
    return OP == OXIDE_RED_MAX ? -INFINITY : 0.0f;
}

template <int OP>
struct OpComb {
    __device__ __forceinline__ double operator()(double a, double b) const { return red_comb<OP>(a, b); }
};
template <int OP>
struct OpCombF {
    __device__ __forceinline__ float operator()(float a, float b) const {
        return OP == OXIDE_RED_MAX ? fmaxf(a, b) : fadd(a, b);
    }
};

// ---- row reductions -----------------------------------------------------------
template <typename T, int OP, bool VEC>
__global__ void __launch_bounds__(256)
    reduce_rows_kernel(const T* x, uint64_t rows, uint32_t cols, float* out, int tpr) {
    pdl_begin();
    constexpr int V = VEC ? Vec<T>::N : 1;
    __shared__ float red[8];
    const int rpc = blockDim.x / tpr;
    const int sub = threadIdx.x / tpr, t = threadIdx.x % tpr;
    const uint32_t n = cols / V;
    for (uint64_t row0 = (uint64_t)blockIdx.x * rpc; row0 < rows; row0 += (uint64_t)gridDim.x * rpc) {
        const uint64_t row = row0 + sub;
        float acc = red_init<OP>();
        if (row < rows) {
            const T* xr = x + row * cols;
            if (VEC) {
                // RU loads in flight per thread, accumulated in index order
                constexpr int RU = 4;
                for (uint32_t u0 = t; u0 < n; u0 += (uint32_t)tpr * RU) {
                    uint4 raw[RU];
#pragma unroll
                    for (int k = 0; k < RU; ++k) {
                        const uint32_t u = u0 + k * tpr;
                        if (u < n) raw[k] = ld_stream(xr + (uint64_t)u * Vec<T>::N);
                    }
#pragma unroll
                    for (int k = 0; k < RU; ++k) {
                        if (u0 + k * tpr < n) {
                            float f[Vec<T>::N];
                            Vec<T>::unpack(raw[k], f);
#pragma unroll
                            for (int e = 0; e < Vec<T>::N; ++e) acc = red_step<OP>(acc, f[e]);
                        }
                    }
                }
            } else {
                for (uint32_t u = t; u < n; u += tpr) acc = red_step<OP>(acc, Vec<T>::load1(xr + u));
            }
        }
        acc = group_reduce(acc, red, tpr, OpCombF<OP>());
        if (row < rows && t == 0) out[row] = acc;
    }
}

// ---- whole-tensor, stage 1 ------------------------------------------------------
// The grid sweeps the tensor together (vector u to thread u mod the grid's
// threads), so all CTAs stream neighbouring addresses at any moment; the
// scalar path below, for unaligned bases, keeps contiguous slices.
template <typename T, int OP>
__global__ void __launch_bounds__(RED_THREADS)
    reduce_stage1_kernel(const T* x, uint64_t n, uint64_t nvec, double* partial) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    __shared__ double red[RED_THREADS / 32];
    const uint64_t stride = (uint64_t)gridDim.x * RED_THREADS;
    float lane[V];
#pragma unroll
    for (int e = 0; e < V; ++e) lane[e] = red_init<OP>();
    // 8 loads in flight per thread (4: 186.8 us for the bf16 [131072 x 4096] sum
    // of squares, 8: 151.5 us); the per-lane accumulation order is the same
    constexpr int UNROLL = 8;
    for (uint64_t u0 = (uint64_t)blockIdx.x * RED_THREADS + threadIdx.x; u0 < nvec; u0 += stride * UNROLL) {
        uint4 raw[UNROLL];
#pragma unroll
        for (int k = 0; k < UNROLL; ++k) {
            const uint64_t u = u0 + (uint64_t)k * stride;
            if (u < nvec) raw[k] = ld_stream(x + u * V);
        }
#pragma unroll
        for (int k = 0; k < UNROLL; ++k) {
            const uint64_t u = u0 + (uint64_t)k * stride;
            if (u < nvec) {
                float f[V];
                Vec<T>::unpack(raw[k], f);
#pragma unroll
                for (int e = 0; e < V; ++e) lane[e] = red_step<OP>(lane[e], f[e]);
            }
        }
    }
    double acc = OP == OXIDE_RED_MAX ? -INFINITY : 0.0;
#pragma unroll
    for (int e = 0; e < V; ++e) acc = red_comb<OP>(acc, (double)lane[e]);
    // Elements after the last whole vector belong to the last block.
    if (blockIdx.x == gridDim.x - 1) {
        for (uint64_t i = nvec * V + threadIdx.x; i < n; i += RED_THREADS) {
            const double v = (double)Vec<T>::load1(x + i);
            acc = red_comb<OP>(acc, OP == OXIDE_RED_SUMSQ ? v * v : v);
        }
    }
    acc = group_reduce(acc, red, RED_THREADS, OpComb<OP>());
    if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

// ---- whole-tensor, stage 2 (one CTA) ----------------------------------------------
template <int OP>
__global__ void __launch_bounds__(RED_THREADS)
    reduce_stage2_kernel(const double* partial, int nblocks, double* out) {
    pdl_begin();
    __shared__ double red[RED_THREADS / 32];
    double acc = OP == OXIDE_RED_MAX ? -INFINITY : 0.0;
    for (int i = threadIdx.x; i < nblocks; i += RED_THREADS) acc = red_comb<OP>(acc, partial[i]);
    acc = group_reduce(acc, red, RED_THREADS, OpComb<OP>());
    if (threadIdx.x == 0) *out = acc;
}

// Scalar whole-tensor stage 1 for unaligned bases.
template <typename T, int OP>
__global__ void __launch_bounds__(RED_THREADS)
    reduce_stage1_scalar_kernel(const T* x, uint64_t n, uint64_t per_block, double* partial) {
    pdl_begin();
    __shared__ double red[RED_THREADS / 32];
    const uint64_t lo = (uint64_t)blockIdx.x * per_block;
    const uint64_t hi = lo + per_block < n ? lo + per_block : n;
    float acc32 = red_init<OP>();
    for (uint64_t i = lo + threadIdx.x; i < hi; i += RED_THREADS)
        acc32 = red_step<OP>(acc32, Vec<T>::load1(x + i));
    double acc = group_reduce((double)acc32, red, RED_THREADS, OpComb<OP>());
    if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

static uint64_t stage1_blocks(uint64_t units) {
    // At least 16 units per thread before a slice is split further.
    const uint64_t min_units = (uint64_t)RED_THREADS * 16;
    uint64_t b = (units + min_units - 1) / min_units;
    if (b < 1) b = 1;
    if (b > RED_BLOCKS) b = RED_BLOCKS;
    return b;
}

template <typename T, int OP>
static void launch_reduce(const T* x, uint64_t n, double* out, double* partial, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    if (aligned16(x)) {
        const uint64_t nvec = n / V;
        const uint64_t blocks = stage1_blocks(nvec);
        launch_k(reduce_stage1_kernel<T, OP>, (unsigned)blocks, RED_THREADS, 0, st, x, n, nvec, partial);
        launch_k(reduce_stage2_kernel<OP>, 1, RED_THREADS, 0, st, partial, (int)blocks, out);
    } else {
        const uint64_t blocks = stage1_blocks(n);
        const uint64_t per = (n + blocks - 1) / blocks;
        launch_k(reduce_stage1_scalar_kernel<T, OP>, (unsigned)blocks, RED_THREADS, 0, st, x, n, per, partial);
        launch_k(reduce_stage2_kernel<OP>, 1, RED_THREADS, 0, st, partial, (int)blocks, out);
    }
}

template <typename T>
static int reduce_entry(const char* name, int op, const T* x, uint64_t n, double* out,
                        void* ws, uint64_t ws_bytes, cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(op >= OXIDE_RED_SUM && op <= OXIDE_RED_SUMSQ, name, "unknown reduction");
    OXIDE_REQUIRE(out, name, "null output pointer");
    OXIDE_REQUIRE(n == 0 || x, name, "null input pointer");
    if (!ws || ws_bytes < oxide_reduce_workspace_bytes(n) || (reinterpret_cast<uintptr_t>(ws) & 7))
        return set_error(OXIDE_ERR_WORKSPACE, "%s: workspace must be 8-byte aligned and >= %llu bytes",
                         name, (unsigned long long)oxide_reduce_workspace_bytes(n));
    double* partial = static_cast<double*>(ws);
    if (n == 0) {
        // Empty input: the identity of the operation, written by a kernel so
        // the result is stream-ordered like every other result.
        if (op == OXIDE_RED_MAX)
            launch_k(reduce_stage2_kernel<OXIDE_RED_MAX>, 1, RED_THREADS, 0, st, partial, 0, out);
        else
            launch_k(reduce_stage2_kernel<OXIDE_RED_SUM>, 1, RED_THREADS, 0, st, partial, 0, out);
        return check_launch(name);
    }
    switch (op) {
        case OXIDE_RED_SUM: launch_reduce<T, OXIDE_RED_SUM>(x, n, out, partial, st); break;
        case OXIDE_RED_MAX: launch_reduce<T, OXIDE_RED_MAX>(x, n, out, partial, st); break;
        default: launch_reduce<T, OXIDE_RED_SUMSQ>(x, n, out, partial, st); break;
    }
    return check_launch(name);
}

// ---- whole-tensor reduction with library-owned scratch ----------------------------
// oxide_reduce_static_* run the same two kernels as oxide_reduce_*, with the
// stage-1 partials in this fixed array instead of a caller workspace.  Stage 1
// writes every slot that stage 2 of the same call reads, so the array needs no
// clearing and what an earlier call left in it is never read.
static_assert(RED_BLOCKS <= OXIDE_REDUCE_STATIC_SLOTS, "stage 1 may use every scratch slot");
static __device__ __align__(256) double g_static_partials[OXIDE_REDUCE_STATIC_SLOTS];

constexpr int kMaxDevices = 64;
struct StaticAddr {
    unsigned long long ctx = 0;  // cuCtxGetId of the context the address belongs to
    double* addr = nullptr;
};
static StaticAddr g_static_addr[kMaxDevices];
static std::mutex g_static_mu;

// Device address of g_static_partials on the calling thread's current device.
// It is looked up (cudaGetSymbolAddress, which may load this module's device
// code) on the first call in each CUDA context and kept for that context; a
// new context on the device -- after cudaDeviceReset, say -- has a new id and
// gets a fresh lookup, so an address from a destroyed context is never used.
static int static_partials(const char* name, double** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return set_error(OXIDE_ERR_CUDA, "%s: cudaGetDevice: %s", name, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(OXIDE_ERR_UNSUPPORTED, "%s: device ordinal %d >= %d", name, dev, kMaxDevices);
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_static_mu);
    StaticAddr& slot = g_static_addr[dev];
    if (!slot.addr || ctx == 0 || slot.ctx != ctx) {
        void* addr = nullptr;
        e = cudaGetSymbolAddress(&addr, g_static_partials);
        if (e != cudaSuccess || !addr)
            return set_error(OXIDE_ERR_CUDA, "%s: cudaGetSymbolAddress of the scratch array: %s",
                             name, cudaGetErrorString(e));
        slot.addr = static_cast<double*>(addr);
        // The id is read after the lookup: the lookup creates the primary
        // context when the thread had none yet.
        slot.ctx = current_context_id();
    }
    *out = slot.addr;
    return OXIDE_OK;
}

template <typename T>
static int reduce_static_entry(const char* name, int op, const T* x, uint64_t n, double* out,
                               cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(op >= OXIDE_RED_SUM && op <= OXIDE_RED_SUMSQ, name, "unknown reduction");
    OXIDE_REQUIRE(out, name, "null output pointer");
    OXIDE_REQUIRE(n == 0 || x, name, "null input pointer");
    if (n > OXIDE_REDUCE_STATIC_MAX_N)
        return set_error(OXIDE_ERR_INVALID_ARG,
                         "%s: n = %llu exceeds the %llu elements its fixed scratch of %d partials "
                         "covers; use the workspace form for larger inputs",
                         name, (unsigned long long)n, (unsigned long long)OXIDE_REDUCE_STATIC_MAX_N,
                         OXIDE_REDUCE_STATIC_SLOTS);
    double* partial = nullptr;
    const int rc = static_partials(name, &partial);
    if (rc != OXIDE_OK) return rc;
    return reduce_entry<T>(name, op, x, n, out, partial,
                           (uint64_t)OXIDE_REDUCE_STATIC_SLOTS * sizeof(double), st);
}

template <typename T>
static int reduce_rows_entry(const char* name, int op, const T* x, uint64_t rows, uint64_t cols,
                             float* out, cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(op >= OXIDE_RED_SUM && op <= OXIDE_RED_SUMSQ, name, "unknown reduction");
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && out, name, "null pointer");
    OXIDE_REQUIRE(cols >= 1 && cols < (1ull << 32), name, "cols must be in [1, 2^32)");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    constexpr int V = Vec<T>::N;
    const bool vec = cols % V == 0 && aligned16(x);
    const uint64_t units = vec ? cols / V : cols;
    int tpr = 32;
    while (tpr < 256 && (uint64_t)tpr * 8 < units) tpr *= 2;
    const int rpc = 256 / tpr;
    const uint64_t want = (rows + rpc - 1) / rpc, cap = (uint64_t)1 << 30;
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    const uint32_t c32 = (uint32_t)cols;
#define OXIDE_ROWS_LAUNCH(OPV)                                                              \
    (vec ? launch_k(reduce_rows_kernel<T, OPV, true>, grid, 256, 0, st, x, rows, c32, out, tpr) \
         : launch_k(reduce_rows_kernel<T, OPV, false>, grid, 256, 0, st, x, rows, c32, out, tpr))
    switch (op) {
        case OXIDE_RED_SUM: OXIDE_ROWS_LAUNCH(OXIDE_RED_SUM); break;
        case OXIDE_RED_MAX: OXIDE_ROWS_LAUNCH(OXIDE_RED_MAX); break;
        default: OXIDE_ROWS_LAUNCH(OXIDE_RED_SUMSQ); break;
    }
#undef OXIDE_ROWS_LAUNCH
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

uint64_t oxide_reduce_workspace_bytes(uint64_t n) {
    (void)n;
    return (uint64_t)oxide::RED_BLOCKS * sizeof(double);
}

int oxide_reduce_f32(int op, const float* x, uint64_t n, double* out, void* workspace,
                     uint64_t workspace_bytes, oxide_stream_t stream) {
    return oxide::reduce_entry<float>("oxide_reduce_f32", op, x, n, out, workspace,
                                      workspace_bytes, stream);
}
int oxide_reduce_bf16(int op, const oxide_bf16* x, uint64_t n, double* out, void* workspace,
                      uint64_t workspace_bytes, oxide_stream_t stream) {
    return oxide::reduce_entry<bf16_t>("oxide_reduce_bf16", op, x, n, out, workspace,
                                       workspace_bytes, stream);
}
int oxide_reduce_static_f32(int op, const float* x, uint64_t n, double* out,
                            oxide_stream_t stream) {
    return oxide::reduce_static_entry<float>("oxide_reduce_static_f32", op, x, n, out, stream);
}
int oxide_reduce_static_bf16(int op, const oxide_bf16* x, uint64_t n, double* out,
                             oxide_stream_t stream) {
    return oxide::reduce_static_entry<bf16_t>("oxide_reduce_static_bf16", op, x, n, out, stream);
}
int oxide_reduce_rows_f32(int op, const float* x, uint64_t rows, uint64_t cols, float* out,
                          oxide_stream_t stream) {
    return oxide::reduce_rows_entry<float>("oxide_reduce_rows_f32", op, x, rows, cols, out, stream);
}
int oxide_reduce_rows_bf16(int op, const oxide_bf16* x, uint64_t rows, uint64_t cols,
                           float* out, oxide_stream_t stream) {
    return oxide::reduce_rows_entry<bf16_t>("oxide_reduce_rows_bf16", op, x, rows, cols, out,
                                            stream);
}

}  // extern "C"
