// k_rowstream.cu -- row kernels fed by a bulk-copy pipeline through shared
// memory: RMSNorm / add+RMSNorm (src/ops/norm.rs:33-47,
// src/layers/transformer.rs:64-67) and scale+mask+softmax
// (src/ops/attention.rs:41,60,63-79; src/ops/activation.rs:95-120) for rows of
// 1-32 KiB.
//
// Why: a row op has a serial chain per row (load, block reduction, divide,
// store).  Holding the row in registers ties the bytes in flight to the
// register file and to one row per thread group, which leaves HBM idle for
// short rows.  Here each persistent CTA owns rows blockIdx.x + i*gridDim.x
// and keeps `nst` of them in flight in a ring of shared-memory stages filled
// by cp.async.bulk (the TMA's 1-D copy engine, no multicast), each stage
// completing on its own mbarrier.  Thread 0 refills a stage as soon as every
// thread has moved that row into registers, so the copy of row i + nst
// overlaps the reductions, divides and stores of rows i .. i + nst - 1.
//
// Masked keys (lens / causal) are neither copied nor read: only the valid
// prefix of a row (rounded up to 16 bytes) is fetched.  Every mbarrier wait is
// bounded; a timeout sets a bit in the device error word read by
// oxide_device_errors() and the CTA drains its copies (bounded) and exits.
#include <stdio.h>

#include "oxide_bulk.cuh"
#include "oxide_rowstream.cuh"

namespace oxide {

__device__ unsigned g_stream_err;

constexpr int RS_THREADS = 256;
constexpr int RS_MAX_STAGES = 8;
constexpr uint32_t RS_SMEM_TARGET = 64 * 1024;  // ring bytes per CTA (3 CTAs per SM)

// After a failed wait: wait (bounded) for every stage issued but not yet
// consumed, so no bulk copy still targets this CTA's shared memory.
__device__ __forceinline__ void rs_drain(uint64_t* bars, uint64_t from, uint64_t issued, int nst) {
    if (threadIdx.x != 0) return;
    for (uint64_t i = from; i < issued; ++i)
        mbar_wait(&bars[i % nst], (uint32_t)((i / nst) & 1), &g_stream_err);
}

// ---------------------------------------------------------------- RMSNorm
template <typename T, int VPT, bool ADD>
__global__ void __launch_bounds__(RS_THREADS)
    rms_stream_kernel(const T* x, const T* r, const T* w, T* h, T* y, uint64_t rows,
                      uint32_t cols, float eps, int nst) {
    constexpr int V = Vec<T>::N;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t bars[RS_MAX_STAGES];
    __shared__ float red[RS_THREADS / 32];
    const uint32_t row_bytes = cols * (uint32_t)sizeof(T);
    const uint32_t stage_bytes = row_bytes * (ADD ? 2 : 1);
    const uint32_t nvec = cols / V;
    const uint64_t first = blockIdx.x, step = gridDim.x;
    const uint64_t nmine = first < rows ? (rows - first + step - 1) / step : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](uint64_t i) {  // thread 0: row i of this CTA into stage i % nst
        const int s = (int)(i % nst);
        const uint64_t row = first + i * step;
        unsigned char* dst = ring + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&bars[s], stage_bytes);
        bulk_g2s(dst, x + row * cols, row_bytes, &bars[s]);
        if (ADD) bulk_g2s(dst + row_bytes, r + row * cols, row_bytes, &bars[s]);
    };
    uint64_t issued = nmine < (uint64_t)nst ? nmine : (uint64_t)nst;
    if (threadIdx.x == 0)
        for (uint64_t i = 0; i < issued; ++i) issue(i);

    for (uint64_t i = 0; i < nmine; ++i) {
        const int s = (int)(i % nst);
        const bool ok = mbar_wait(&bars[s], (uint32_t)((i / nst) & 1), &g_stream_err);
        if (!__syncthreads_and(ok)) {
            rs_drain(bars, i + 1, issued, nst);
            return;
        }
        const uint64_t off = (first + i * step) * cols;
        const unsigned char* src = ring + (size_t)s * stage_bytes;
        float v[VPT][V];
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = threadIdx.x + k * RS_THREADS;
            if (j < nvec) {
                Vec<T>::unpack(lds128(src + (size_t)j * 16), v[k]);
                if (ADD) {
                    float rv[V];
                    Vec<T>::unpack(lds128(src + row_bytes + (size_t)j * 16), rv);
#pragma unroll
                    for (int e = 0; e < V; ++e) v[k][e] = Vec<T>::rnd(fadd(v[k][e], rv[e]));
                    st_stream(h + off + (uint64_t)j * V, Vec<T>::pack(v[k]));
                }
#pragma unroll
                for (int e = 0; e < V; ++e) ss = fadd(ss, fmul(v[k][e], v[k][e]));
            }
        }
        ss = group_reduce(ss, red, RS_THREADS, OpAddF());  // every thread is done with stage s
        if (threadIdx.x == 0 && issued < nmine) {
            fence_proxy_async_smem();
            issue(issued);
            ++issued;
        }
        const float rms = fsqrt(fadd(fdiv(ss, (float)cols), eps));
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = threadIdx.x + k * RS_THREADS;
            if (j < nvec) {
                float wv[V], o[V];
                Vec<T>::unpack(ld_keep(w + (uint64_t)j * V), wv);
#pragma unroll
                for (int e = 0; e < V; ++e) o[e] = fmul(fdiv(v[k][e], rms), wv[e]);
                st_stream(y + off + (uint64_t)j * V, Vec<T>::pack(o));
            }
        }
    }
}

// ---------------------------------------------------------------- softmax
// G = 256 / tpr rows per stage; `tpr` threads own one row; VPT vectors each.
// 16 elements per thread fit 3 CTAs per SM (the 64 KiB ring allows 3);
// 32 elements per thread (rows of 4-8K keys) run 2.
template <typename T, int VPT>
constexpr int smax_stream_min_blocks() {
    return VPT * Vec<T>::N <= 16 ? 3 : 2;
}

template <typename T, int VPT>
__global__ void __launch_bounds__(RS_THREADS, smax_stream_min_blocks<T, VPT>())
    smax_stream_kernel(const T* x, T* out, SmaxArgs p, int nst) {
    constexpr int V = Vec<T>::N;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t bars[RS_MAX_STAGES];
    __shared__ float red[RS_THREADS / 32];
    const int G = RS_THREADS / p.tpr;
    const uint32_t row_bytes = p.cols * (uint32_t)sizeof(T);
    const uint32_t stage_bytes = row_bytes * G;
    const uint32_t nvec = p.cols / V;
    const uint64_t ngroups = (p.rows + G - 1) / G;
    const uint64_t first = blockIdx.x, step = gridDim.x;
    const uint64_t nmine = first < ngroups ? (ngroups - first + step - 1) / step : 0;
    const int sub = threadIdx.x / p.tpr, t = threadIdx.x % p.tpr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](uint64_t i) {  // thread 0: the valid prefixes of group i's rows
        const int s = (int)(i % nst);
        const uint64_t row0 = (first + i * step) * G;
        unsigned char* dst = ring + (size_t)s * stage_bytes;
        uint32_t total = 0;
        uint32_t bytes[RS_THREADS / 32];
        for (int rr = 0; rr < G; ++rr) {
            const uint64_t row = row0 + rr;
            uint32_t b = 0;
            if (row < p.rows) b = (valid_len(p, row) * (uint32_t)sizeof(T) + 15u) & ~15u;
            bytes[rr] = b;
            total += b;
        }
        mbar_arrive_expect_tx(&bars[s], total);
        for (int rr = 0; rr < G; ++rr)
            if (bytes[rr]) bulk_g2s(dst + (size_t)rr * row_bytes, x + (row0 + rr) * p.cols, bytes[rr], &bars[s]);
    };
    uint64_t issued = nmine < (uint64_t)nst ? nmine : (uint64_t)nst;
    if (threadIdx.x == 0)
        for (uint64_t i = 0; i < issued; ++i) issue(i);

    for (uint64_t i = 0; i < nmine; ++i) {
        const int s = (int)(i % nst);
        const bool ok = mbar_wait(&bars[s], (uint32_t)((i / nst) & 1), &g_stream_err);
        if (!__syncthreads_and(ok)) {
            rs_drain(bars, i + 1, issued, nst);
            return;
        }
        const uint64_t row = (first + i * step) * G + sub;
        const bool active = row < p.rows;
        const uint32_t len = active ? valid_len(p, row) : 0;
        const unsigned char* src = ring + (size_t)s * stage_bytes + (size_t)sub * row_bytes;
        float sv[VPT][V];
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec && j * V < len) {
                Vec<T>::unpack(lds128(src + (size_t)j * 16), sv[k]);
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    const uint32_t c = j * V + e;
                    sv[k][e] = c < len ? score(p, sv[k][e], c) : -INFINITY;
                    m = fmaxf(m, sv[k][e]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < V; ++e) sv[k][e] = -INFINITY;
            }
        }
        m = group_reduce(m, red, p.tpr, OpMaxF());
        if (p.tpr == 32) __syncthreads();  // warp groups reduce without a block barrier
        // every thread is done with stage s
        if (threadIdx.x == 0 && issued < nmine) {
            fence_proxy_async_smem();
            issue(issued);
            ++issued;
        }
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
#pragma unroll
            for (int e = 0; e < V; ++e) {
                sv[k][e] = expf(fsub(sv[k][e], m));
                sum = fadd(sum, sv[k][e]);
            }
        }
        sum = group_reduce(sum, red, p.tpr, OpAddF());
        T* orow = out + row * p.cols;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = t + k * p.tpr;
            if (active && j < nvec) {
                float o[V];
#pragma unroll
                for (int e = 0; e < V; ++e) o[e] = (j * V + e < len) ? fdiv(sv[k][e], sum) : 0.0f;
                st_stream(orow + (uint64_t)j * V, Vec<T>::pack(o));
            }
        }
    }
}

// ---------------------------------------------------------------- launchers
template <typename K>
static bool prepare(K kernel, uint32_t smem) {
    // The per-device opt-in for more than 48 KiB of dynamic shared memory.
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return true;
}

static int ring_stages(uint32_t stage_bytes) {
    int nst = (int)(RS_SMEM_TARGET / stage_bytes);
    return nst < 2 ? 2 : (nst > RS_MAX_STAGES ? RS_MAX_STAGES : nst);
}

template <typename T, int VPT, bool ADD>
static bool rms_go(const T* x, const T* r, const T* w, T* h, T* y, uint64_t rows, uint32_t cols,
                   float eps, cudaStream_t st) {
    const uint32_t stage = cols * (uint32_t)sizeof(T) * (ADD ? 2 : 1);
    const int nst = ring_stages(stage);
    const uint32_t smem = stage * nst;
    auto kern = rms_stream_kernel<T, VPT, ADD>;
    if (!prepare(kern, smem)) return false;
    const int cap = resident_blocks(reinterpret_cast<const void*>(kern), RS_THREADS, smem);
    if (cap <= 0) return false;
    const unsigned grid = (unsigned)(rows < (uint64_t)cap ? rows : (uint64_t)cap);
    kern<<<grid, RS_THREADS, smem, st>>>(x, r, w, h, y, rows, cols, eps, nst);
    return true;
}

template <typename T>
bool rms_stream_launch(const T* x, const T* r, const T* w, T* h, T* y, uint64_t rows,
                       uint32_t cols, float eps, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    const bool add = r != nullptr;
    const uint64_t row_bytes = (uint64_t)cols * sizeof(T);
    if (cols % V || row_bytes < 2048 || row_bytes * (add ? 2 : 1) > 32768) return false;
    if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (add && (!aligned16(r) || !aligned16(h))))
        return false;
    const uint32_t nvec = cols / V;
    const int vpt = (int)((nvec + RS_THREADS - 1) / RS_THREADS);
    if (add) {
        if (vpt <= 1) return rms_go<T, 1, true>(x, r, w, h, y, rows, cols, eps, st);
        if (vpt <= 2) return rms_go<T, 2, true>(x, r, w, h, y, rows, cols, eps, st);
        if (vpt <= 4) return rms_go<T, 4, true>(x, r, w, h, y, rows, cols, eps, st);
        return false;
    }
    if (vpt <= 1) return rms_go<T, 1, false>(x, r, w, h, y, rows, cols, eps, st);
    if (vpt <= 2) return rms_go<T, 2, false>(x, r, w, h, y, rows, cols, eps, st);
    if (vpt <= 4) return rms_go<T, 4, false>(x, r, w, h, y, rows, cols, eps, st);
    if constexpr (V == 4) {
        if (vpt <= 8) return rms_go<T, 8, false>(x, r, w, h, y, rows, cols, eps, st);
    }
    return false;
}

template <typename T, int VPT>
static bool smax_go(const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    const uint32_t stage = p.cols * (uint32_t)sizeof(T) * (RS_THREADS / p.tpr);
    const int nst = ring_stages(stage);
    const uint32_t smem = stage * nst;
    auto kern = smax_stream_kernel<T, VPT>;
    if (!prepare(kern, smem)) return false;
    const int cap = resident_blocks(reinterpret_cast<const void*>(kern), RS_THREADS, smem);
    if (cap <= 0) return false;
    const uint64_t groups = (p.rows + RS_THREADS / p.tpr - 1) / (RS_THREADS / p.tpr);
    const unsigned grid = (unsigned)(groups < (uint64_t)cap ? groups : (uint64_t)cap);
    kern<<<grid, RS_THREADS, smem, st>>>(x, out, p, nst);
    return true;
}

template <typename T>
bool smax_stream_launch(const T* x, T* out, const SmaxArgs& args, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    const uint64_t row_bytes = (uint64_t)args.cols * sizeof(T);
    if (args.cols % V || row_bytes < 1024 || row_bytes > 32768) return false;
    if (!aligned16(x) || !aligned16(out)) return false;
    SmaxArgs p = args;
    p.cl = 1;
    const uint64_t nvec = args.cols / V;
    constexpr int VPT16 = 16 / V;  // 16 row elements per thread
    uint64_t tpr = 32;
    while (tpr < 256 && tpr * VPT16 < nvec) tpr *= 2;
    p.tpr = (int)tpr;
    if (tpr * VPT16 >= nvec) return smax_go<T, VPT16>(x, out, p, st);
    if (256ull * 2 * VPT16 >= nvec) return smax_go<T, 2 * VPT16>(x, out, p, st);
    return false;
}

template bool rms_stream_launch<float>(const float*, const float*, const float*, float*, float*,
                                       uint64_t, uint32_t, float, cudaStream_t);
template bool rms_stream_launch<bf16_t>(const bf16_t*, const bf16_t*, const bf16_t*, bf16_t*,
                                        bf16_t*, uint64_t, uint32_t, float, cudaStream_t);
template bool smax_stream_launch<float>(const float*, float*, const SmaxArgs&, cudaStream_t);
template bool smax_stream_launch<bf16_t>(const bf16_t*, bf16_t*, const SmaxArgs&, cudaStream_t);

}  // namespace oxide

extern "C" int oxide_device_errors(unsigned* flags, int clear) {
    if (!flags) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "oxide_device_errors: null pointer");
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(flags, oxide::g_stream_err, sizeof(unsigned));
    if (e == cudaSuccess && clear) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(oxide::g_stream_err, &zero, sizeof(unsigned));
    }
    if (e != cudaSuccess)
        return oxide::set_error(OXIDE_ERR_CUDA, "oxide_device_errors: %s", cudaGetErrorString(e));
    return OXIDE_OK;
}
