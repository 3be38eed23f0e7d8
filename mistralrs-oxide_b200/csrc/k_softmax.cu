// k_softmax.cu -- softmax(x, dim) and scale + mask + softmax over rows.
//
// Reference: src/ops/activation.rs:95-120 (max, exp(x - max) with a running
// sum, divide) and the scale/mask/softmax block of scaled_dot_product_attention
// (src/ops/attention.rs:41,60,63-79: s = dot * scale; s += mask[j % len];
// softmax over the key axis).
//
// Design (rows of a contiguous [rows, cols] tensor):
//   * rows that tile a 256-thread CTA (a warp or a power-of-two group per
//     row, 256 / group rows per CTA) read straight from HBM, many CTAs per SM
//     in flight, the row kept in registers; longer rows are streamed three
//     times (max, sum, store) by one CTA or a thread-block cluster of up to 8
//     CTAs per row, the second and third reads served by L2, the cluster
//     exchanging slice maxima and sums through distributed shared memory;
//   * each thread holds its part of the row PACKED (bf16 stays 2 bytes per
//     element), 32 elements for bf16 and 16 for f32; the kernels are
//     instruction-bound, so fully valid 16-byte vectors take a path without
//     per-element bounds checks and the additive mask is a template
//     parameter; max and sum use fixed reduction trees (deterministic); the
//     divide by the row sum is RowDiv (the correctly rounded quotient);
//   * keys at or beyond a row's valid length (lens / causal) are written as 0
//     and never read;
//   * bf16 rows of whole vectors up to 2048 keys without an additive mask (the
//     attention-probability shape) take a warp-per-row kernel whose f32
//     intermediate is accurate to ~1e-5 relative, far inside the one-bf16-ulp
//     output tolerance (see smax_bf16_warp_kernel).
// softmax over an inner (non-last) dim, odd lengths and unaligned pointers take
// scalar multi-pass kernels.
#include <cooperative_groups.h>

#include <type_traits>

#include "oxide_softmax.cuh"

namespace cg = cooperative_groups;

namespace oxide {

// ---- scores and exp arguments ---------------------------------------------------
// s = x * scale, plus mask[c] as fma(x, scale, mask[c]) (one rounding); the exp
// argument is d = s - m, formed without a mask as fma(x, scale, -m) (one
// rounding).  The reference rounds x * scale before adding; on sm_100a a paired
// multiply feeding a paired add comes out fused anyway, so the fused forms are
// written explicitly and the scalar and paired lanes of every kernel agree.
template <bool MASK>
__device__ __forceinline__ float score_t(const SmaxArgs& p, float x, uint32_t c) {
    return MASK ? __fmaf_rn(x, p.scale, __ldg(p.mask + p.mask_div.mod(c))) : fmul(x, p.scale);
}
template <bool MASK>
__device__ __forceinline__ float2 score2(const SmaxArgs& p, float x0, float x1, uint32_t c) {
    const float2 sc = f2(p.scale, p.scale);
    if (MASK)
        return __ffma2_rn(f2(x0, x1), sc,
                          f2(__ldg(p.mask + p.mask_div.mod(c)), __ldg(p.mask + p.mask_div.mod(c + 1))));
    return fmul2(f2(x0, x1), sc);
}
template <bool MASK>
__device__ __forceinline__ float diff_t(const SmaxArgs& p, float x, uint32_t c, float m) {
    return MASK ? fsub(score_t<MASK>(p, x, c), m) : __fmaf_rn(x, p.scale, -m);
}
template <bool MASK>
__device__ __forceinline__ float2 diff2(const SmaxArgs& p, float x0, float x1, uint32_t c, float2 nm) {
    return MASK ? fadd2(score2<MASK>(p, x0, x1, c), nm) : __ffma2_rn(f2(x0, x1), f2(p.scale, p.scale), nm);
}

// ---- per-thread row chunk: VPT packed vectors j = j0 + k * jstep ------------
// Max of the valid scores of the chunk (vectors j < jhi, keys c < len).
template <typename T, int VPT, bool MASK>
__device__ __forceinline__ float chunk_max(const uint4 (&raw)[VPT], const SmaxArgs& p, uint32_t j0,
                                           uint32_t jstep, uint32_t jhi, uint32_t len) {
    constexpr int V = Vec<T>::N;
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = j0 + k * jstep;
        if (j < jhi && j * V < len) {
            float f[V];
            Vec<T>::unpack(raw[k], f);
            if (j * V + V <= len) {
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 s = score2<MASK>(p, f[e], f[e + 1], j * V + e);
                    m = fmaxf(m, fmaxf(s.x, s.y));
                }
            } else {
#pragma unroll
                for (int e = 0; e < V; ++e)
                    if (j * V + e < len) m = fmaxf(m, score_t<MASK>(p, f[e], j * V + e));
            }
        }
    }
    return m;
}

// ev = exp(score - m) for valid keys (0 for masked keys of a partial vector);
// returns the thread's sum (two lane accumulators, combined at the end).
template <typename T, int VPT, bool MASK>
__device__ __forceinline__ float chunk_exp(const uint4 (&raw)[VPT], float (&ev)[VPT][Vec<T>::N],
                                           const SmaxArgs& p, uint32_t j0, uint32_t jstep,
                                           uint32_t jhi, uint32_t len, float m) {
    constexpr int V = Vec<T>::N;
    const float2 nm = f2(-m, -m);
    float2 acc = f2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = j0 + k * jstep;
        if (j < jhi && j * V < len) {
            float f[V];
            Vec<T>::unpack(raw[k], f);
            if (j * V + V <= len) {  // every key valid: no per-key checks
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 d = diff2<MASK>(p, f[e], f[e + 1], j * V + e, nm);
                    ev[k][e] = expf(d.x);
                    ev[k][e + 1] = expf(d.y);
                    acc = fadd2(acc, f2(ev[k][e], ev[k][e + 1]));
                }
            } else {  // the one vector of the row that straddles len
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 d = diff2<MASK>(p, f[e], f[e + 1], j * V + e, nm);
                    ev[k][e] = j * V + e < len ? expf(d.x) : 0.0f;
                    ev[k][e + 1] = j * V + e + 1 < len ? expf(d.y) : 0.0f;
                    acc = fadd2(acc, f2(ev[k][e], ev[k][e + 1]));
                }
            }
        }
    }
    return fadd(acc.x, acc.y);
}

// Write p = ev / sum (0 beyond len) for every vector j < jhi of the chunk.
// RowDiv's paired fast path per vector; a vector holding a numerator outside
// its range (or a row whose sum is outside it) is redone with the IEEE divide.
template <typename T, int VPT>
__device__ __forceinline__ void chunk_store_div(T* orow, const float (&ev)[VPT][Vec<T>::N],
                                                uint32_t j0, uint32_t jstep, uint32_t jhi,
                                                uint32_t len, float sum) {
    constexpr int V = Vec<T>::N;
    const RowDiv div(sum);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = j0 + k * jstep;
        if (j < jhi) {
            float o[V];
            if (j * V + V <= len) {  // every key valid: RowDiv's paired fast path
                bool redo = div.ieee;
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 q = div.fast2(f2(ev[k][e], ev[k][e + 1]), redo);
                    o[e] = q.x;
                    o[e + 1] = q.y;
                }
                if (redo) {
#pragma unroll
                    for (int e = 0; e < V; ++e) o[e] = __fdiv_rn(ev[k][e], sum);
                }
            } else if (j * V < len) {  // the straddling vector: IEEE divide, 0 past len
#pragma unroll
                for (int e = 0; e < V; ++e) o[e] = j * V + e < len ? __fdiv_rn(ev[k][e], sum) : 0.0f;
            } else {
#pragma unroll
                for (int e = 0; e < V; ++e) o[e] = 0.0f;
            }
            st_stream(orow + (uint64_t)j * V, Vec<T>::pack(o));
        }
    }
}

// Vectors per thread: 32 row elements for bf16 (2 bytes each in flight), 16
// for f32, so the kept exp values fit the register budgets below.
constexpr int SMAX_VPT = 4;

// ---- rows that tile a CTA, read straight from HBM --------------------------------
// A 256-thread CTA holds 256 / tpr rows of tpr threads each; each thread keeps
// VPT packed vectors of its row in registers between the max, exp and store.
template <typename T, int VPT, bool MASK>
__global__ void __launch_bounds__(256, 3) smax_rows_kernel(const T* x, T* out, SmaxArgs p) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    __shared__ float red[32];
    const uint32_t nvec = p.cols / V;
    const int rpc = blockDim.x / p.tpr, sub = threadIdx.x / p.tpr, t = threadIdx.x % p.tpr;
    for (uint64_t row0 = (uint64_t)blockIdx.x * rpc; row0 < p.rows; row0 += (uint64_t)gridDim.x * rpc) {
        const uint64_t row = row0 + sub;
        const bool active = row < p.rows;
        const uint32_t len = active ? valid_len(p, row) : 0;
        const uint32_t jhi = active ? nvec : 0;
        const T* xr = x + row * p.cols;
        const uint32_t j0 = t;
        uint4 raw[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = j0 + k * p.tpr;
            if (j < jhi && j * V < len) raw[k] = ld_stream(xr + (uint64_t)j * V);
        }
        const float m = group_reduce(chunk_max<T, VPT, MASK>(raw, p, j0, p.tpr, jhi, len), red, p.tpr,
                                     OpMaxF());
        float ev[VPT][V];
        const float sum = group_reduce(chunk_exp<T, VPT, MASK>(raw, ev, p, j0, p.tpr, jhi, len, m), red,
                                       p.tpr, OpAddF());
        chunk_store_div<T, VPT>(out + row * p.cols, ev, j0, p.tpr, jhi, len, sum);
    }
}

// ---- long rows: two streaming passes, the second served by L2 ---------------------
// A row is split over a cluster of p.cl CTAs (p.cl = 1: one CTA per row).
// Pass 1 streams the CTA's slice from HBM once, keeping per thread the
// running max m and the sum s of exp(score - m) (s rescaled by exp(m_old - m)
// when the max grows); the CTA and then the cluster (through distributed
// shared memory, in rank order) combine the (m, s) pairs into the row's max M
// and sum S.  Pass 2 re-reads the slice -- from L2, where pass 1 left it -- and
// writes p = exp(score - M) * RN(1 / S) (IEEE score; exp_sfu below); S
// carries the extra roundings of the rescaling and p those of the reciprocal
// and of exp_sfu, a few 1e-6 in all, inside the f32 tolerance.  Nothing is held across
// passes, so each thread keeps U vectors in flight with few registers and a
// decode-sized batch of long rows runs in one wave.  In place (out == x) is
// safe: a CTA writes only its own slice, after its own last read of it.
// e^d for d = score - max <= 0 on the special-function unit: ex2 of
// RN(d log2 e).  Relative error at most 2^-24 |d log2 e| ln 2 from the
// argument's rounding plus ~2^-22 from ex2.approx -- under 6e-6 down to
// the subnormal range (d log2 e >= -126), inside the f32 softmax tolerance
// of 1e-5; subnormal results are kept (non-flushing ex2).  d is computed
// first, as the reference does, so large scores lose nothing to it.
// Measured on the C3 decode rows: 17.3 -> 15.9 us against expf.
__device__ __forceinline__ float exp_sfu(float d) { return ex2_approx(fmul(d, 1.4426950408889634f)); }

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Merge (m, s) into the running pair (M, S): both sums are taken relative to
// their own max.
__device__ __forceinline__ void online_merge(float& M, float& S, float m, float s) {
    if (m > M) {
        S = fadd(fmul(S, expf(fsub(M, m))), s);
        M = m;
    } else if (m == M || m != m) {
        S = fadd(S, s);
    } else {
        S = fadd(S, fmul(s, expf(fsub(m, M))));
    }
}

template <typename T, bool MASK, int NT, int U>
__global__ void __launch_bounds__(NT, 2048 / NT / 2)
    smax_stream_kernel(const T* x, T* out, SmaxArgs p) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    __shared__ float red[32];
    __shared__ float slot[2];
    const uint32_t cl = (uint32_t)p.cl;
    const uint32_t rank = cl > 1 ? cg::this_cluster().block_rank() : 0u;
    const uint32_t nvec = p.cols / V;
    const uint32_t per = (nvec + cl - 1) / cl;
    const uint32_t lo = min(nvec, rank * per), hi = min(nvec, lo + per);
    for (uint64_t row = blockIdx.x / cl; row < p.rows; row += gridDim.x / cl) {
        const uint32_t len = valid_len(p, row);
        const uint32_t vv = min(hi, (len + V - 1) / V);  // slice vectors [lo, vv) hold valid keys
        const T* xr = x + row * p.cols;
        // pass 1: running max and rescaled sum of exp
        float m = -INFINITY, ssum = 0.0f;
        for (uint32_t j0 = lo + threadIdx.x; j0 < vv; j0 += NT * U) {
            uint4 r[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = j0 + u * NT;
                if (j < vv) r[u] = ld_stream(xr + (uint64_t)j * V);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = j0 + u * NT;
                if (j < vv) {
                    float f[V];
                    Vec<T>::unpack(r[u], f);
                    const bool full = j * V + V <= len;
                    float sc[V];
                    float vm = -INFINITY;
#pragma unroll
                    for (int e = 0; e < V; e += 2) {
                        const float2 s2 = score2<MASK>(p, f[e], f[e + 1], j * V + e);
                        sc[e] = full || j * V + e < len ? s2.x : -INFINITY;
                        sc[e + 1] = full || j * V + e + 1 < len ? s2.y : -INFINITY;
                        vm = fmaxf(vm, fmaxf(sc[e], sc[e + 1]));
                    }
                    if (vm > m) {
                        ssum = fmul(ssum, expf(fsub(m, vm)));
                        m = vm;
                    }
                    // while every score so far is -inf, exp(score - 0) adds 0
                    // (and NaN for a NaN key) instead of exp(-inf + inf)
                    const float mr = m == -INFINITY ? 0.0f : m;
                    const float2 nm = f2(-mr, -mr);
                    float2 acc = f2(0.0f, 0.0f);
#pragma unroll
                    for (int e = 0; e < V; e += 2) {
                        const float2 d = diff2<MASK>(p, f[e], f[e + 1], j * V + e, nm);
                        const float e0 = full || j * V + e < len ? exp_sfu(d.x) : 0.0f;
                        const float e1 = full || j * V + e + 1 < len ? exp_sfu(d.y) : 0.0f;
                        acc = fadd2(acc, f2(e0, e1));
                    }
                    ssum = fadd(ssum, fadd(acc.x, acc.y));
                }
            }
        }
        // combine (m, s) over the CTA: max, then the sums rescaled to it
        const float mb = group_reduce(m, red, NT, OpMaxF());
        const float sb = group_reduce(m == mb ? ssum : fmul(ssum, expf(fsub(m, mb))), red, NT, OpAddF());
        float M = mb, S = sb;
        if (cl > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            if (threadIdx.x == 0) {
                slot[0] = mb;
                slot[1] = sb;
            }
            cluster.sync();
            M = -INFINITY;
            S = 0.0f;
            for (uint32_t q = 0; q < cl; ++q)
                online_merge(M, S, *cluster.map_shared_rank(&slot[0], q), *cluster.map_shared_rank(&slot[1], q));
            cluster_arrive();  // this CTA is done reading its peers' slots
        }
        // pass 2: p = exp(s - M) * RN(1 / S) for valid keys, 0 beyond the valid
        // length.  S >= 1 (the max key contributes exp(0)), so the reciprocal
        // is normal and the product is within 1.5 ulp of exp(s - M) / S -- the
        // sum itself carries more rounding than that; measured 7% faster than
        // the per-element division on the decode shape.
        const float inv = __frcp_rn(S);
        const float2 inv2 = f2(inv, inv);
        const float2 nm = f2(-M, -M);
        T* orow = out + row * p.cols;
        for (uint32_t j0 = lo + threadIdx.x; j0 < hi; j0 += NT * U) {
            uint4 r[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = j0 + u * NT;
                if (j < vv) r[u] = ld_stream(xr + (uint64_t)j * V);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t j = j0 + u * NT;
                if (j < hi) {
                    float o[V];
                    if (j < vv) {
                        float f[V];
                        Vec<T>::unpack(r[u], f);
                        const bool full = j * V + V <= len;
#pragma unroll
                        for (int e = 0; e < V; e += 2) {
                            const float2 d = diff2<MASK>(p, f[e], f[e + 1], j * V + e, nm);
                            const float2 q = fmul2(f2(exp_sfu(d.x), exp_sfu(d.y)), inv2);
                            o[e] = full || j * V + e < len ? q.x : 0.0f;
                            o[e + 1] = full || j * V + e + 1 < len ? q.y : 0.0f;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < V; ++e) o[e] = 0.0f;
                    }
                    st_stream(orow + (uint64_t)j * V, Vec<T>::pack(o));
                }
            }
        }
        if (cl > 1) cluster_wait();  // peers are done with this CTA's slots
    }
}

// 512 threads, 2 CTAs per SM (64 registers); vectors in flight per thread:
// 4, or 2 with the additive mask (whose loads need registers of their own).
constexpr int STREAM_THREADS = 512;
template <bool MASK>
constexpr int stream_unroll() { return MASK ? 2 : 4; }

// ---- fallbacks -----------------------------------------------------------------
// Multi-pass row kernel: any cols, any alignment.  One CTA per row; reads the
// unmasked part of the row three times (max, sum, write).
template <typename T>
__global__ void __launch_bounds__(256) smax_rows_scalar_kernel(const T* x, T* out, SmaxArgs p) {
    pdl_begin();
    __shared__ float red[8];
    for (uint64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint32_t len = valid_len(p, row);
        const T* xr = x + row * p.cols;
        T* orow = out + row * p.cols;
        float m = -INFINITY;
        for (uint32_t j = threadIdx.x; j < len; j += blockDim.x)
            m = fmaxf(m, score(p, Vec<T>::load1(xr + j), j));
        m = group_reduce(m, red, (int)blockDim.x, OpMaxF());
        float sum = 0.0f;
        for (uint32_t j = threadIdx.x; j < len; j += blockDim.x)
            sum = fadd(sum, expf(score_diff(p, Vec<T>::load1(xr + j), j, m)));
        sum = group_reduce(sum, red, (int)blockDim.x, OpAddF());
        __syncthreads();  // every thread has read its inputs before any write (in place)
        const RowDiv div(sum);
        for (uint32_t j = threadIdx.x; j < p.cols; j += blockDim.x) {
            float o = 0.0f;
            if (j < len) o = div(expf(score_diff(p, Vec<T>::load1(xr + j), j, m)));
            Vec<T>::store1(orow + j, o);
        }
    }
}

// softmax over a non-last dim: x viewed as [outer, dim, inner]; one thread
// per (outer, inner) column, consecutive threads on consecutive inner indices
// (coalesced).  out must not alias x.
template <typename T>
__global__ void __launch_bounds__(256)
    smax_inner_kernel(const T* x, T* out, uint64_t outer, uint64_t dim, uint64_t inner) {
    pdl_begin();
    const uint64_t total = outer * inner;
    for (uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
         c += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t base = (c / inner) * dim * inner + (c % inner);
        float m = -INFINITY;
        for (uint64_t d = 0; d < dim; ++d) m = fmaxf(m, Vec<T>::load1(x + base + d * inner));
        float sum = 0.0f;
        for (uint64_t d = 0; d < dim; ++d)
            sum = fadd(sum, expf(fsub(Vec<T>::load1(x + base + d * inner), m)));
        const RowDiv div(sum);
        for (uint64_t d = 0; d < dim; ++d)
            Vec<T>::store1(out + base + d * inner,
                           div(expf(fsub(Vec<T>::load1(x + base + d * inner), m))));
    }
}

// ---- launchers -------------------------------------------------------------------
static cudaError_t launch_cluster(const void* kern, void** args, SmaxArgs& p, cudaStream_t st) {
    const uint64_t cap = (uint64_t)1 << 30;
    const uint64_t clusters = p.rows < cap / p.cl ? p.rows : cap / p.cl;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(clusters * p.cl), 1, 1);
    cfg.blockDim = dim3(p.tpr, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = add_pdl_attr(attr, 1);
    return cudaLaunchKernelExC(&cfg, kern, args);
}

template <typename T, int VPT, bool MASK>
static cudaError_t launch_tiled(const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    // One tile of 256 / tpr rows per 256-thread CTA; the hardware keeps the
    // next CTAs' loads in flight while resident ones compute.
    const int rpc = 256 / p.tpr;
    const uint64_t tiles = (p.rows + rpc - 1) / rpc, cap = (uint64_t)1 << 30;
    launch_k(smax_rows_kernel<T, VPT, MASK>, (unsigned)(tiles < cap ? tiles : cap), 256, 0, st, x, out, p);
    return cudaSuccess;
}

// Long rows: clusters of up to 8 CTAs per row while all CTAs still fit one
// wave and each keeps at least two vectors per thread.
template <typename T, bool MASK>
static cudaError_t launch_stream(const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    auto kern = smax_stream_kernel<T, MASK, STREAM_THREADS, stream_unroll<MASK>()>;
    const uint64_t slots =
        (uint64_t)resident_blocks(reinterpret_cast<const void*>(kern), STREAM_THREADS, 0);
    const uint64_t nvec = p.cols / V;
    int cl = 1;
    while (cl < 8 && p.rows * (uint64_t)(2 * cl) <= slots && nvec / (2 * cl) >= 2ull * STREAM_THREADS)
        cl *= 2;
    p.cl = cl;
    p.tpr = STREAM_THREADS;
    if (cl > 1) {
        void* args[] = {(void*)&x, (void*)&out, (void*)&p};
        return launch_cluster(reinterpret_cast<const void*>(kern), args, p, st);
    }
    const uint64_t cap = (uint64_t)1 << 30;
    launch_k(kern, (unsigned)(p.rows < cap ? p.rows : cap), STREAM_THREADS, 0, st, x, out, p);
    return cudaSuccess;
}

// vpt > 0: tiled rows of vpt vectors per thread; vpt == 0: streamed long rows.
template <typename T, bool MASK>
static cudaError_t launch_vec(const T* x, T* out, SmaxArgs p, int vpt, cudaStream_t st) {
    if (vpt == 0) return launch_stream<T, MASK>(x, out, p, st);
    if (vpt == 1) return launch_tiled<T, 1, MASK>(x, out, p, st);
    if (vpt == 2) return launch_tiled<T, 2, MASK>(x, out, p, st);
    return launch_tiled<T, SMAX_VPT, MASK>(x, out, p, st);
}

// ---- bf16 rows of up to 32 * 8 * VPT keys, no additive mask ---------------------
// One warp per row, lane l owning the 8-key vectors l, l + 32, ...; rows are
// taken in a grid-stride loop by a persistent grid.  Only vectors holding a
// valid key are read.  The output is bf16, so the f32 intermediate only has to
// be accurate far below half a bf16 ulp (2^-9 relative) for every output to
// be within one bf16 ulp of the reference; that allows:
//   * the row max taken on the packed bf16 keys (max.bf16x2): for scale > 0,
//     x -> RN(x * scale) is non-decreasing, so RN(max(x) * scale) is the max
//     of the scaled scores; NaN keys are skipped like f32::max skips them;
//   * exp(s - m) as ex2(x * (scale * log2 e) - m * log2 e): one paired FMA and
//     one ex2.approx (relative error ~2^-22, subnormal results kept) per key,
//     error ~|s - m| * 2^-24 relative, at most ~1e-5 for |s - m| <= 100;
//   * p = e / sum as ex2(x * (scale * log2 e) - m * log2 e - log2(sum)): the
//     exponent is recomputed in the store pass instead of keeping e, so a lane
//     holds only its packed keys (64 registers, 4 CTAs of 256 threads per SM:
//     measured 10% faster than keeping e at 2 CTAs per SM); lg2.approx adds
//     ~2^-22 absolute to the exponent, ~1.7e-7 relative to p.
__device__ __forceinline__ uint32_t bf16x2_max(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// Keys k >= keep (0 < keep < 8) of a vector of 8 bf16 set to `fill`.
__device__ __forceinline__ uint4 bf16_tail(uint4 v, uint32_t keep, uint32_t fill) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (2u * i >= keep) w[i] = fill | (fill << 16);
        else if (2u * i + 1 >= keep) w[i] = (w[i] & 0xffffu) | (fill << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr float kLog2e = 1.4426950408889634f;

template <int VPT>
__global__ void __launch_bounds__(256, 4)
    smax_bf16_warp_kernel(const bf16_t* __restrict__ x, bf16_t* __restrict__ out, SmaxArgs p) {
    pdl_begin();
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t warp0 = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    const uint32_t nvec = p.cols >> 3;
    const float c1 = fmul(p.scale, kLog2e);
    for (uint64_t row = warp0; row < p.rows; row += nwarps) {
        const uint32_t len = valid_len(p, row);
        const uint32_t nv = (len + 7u) >> 3;  // vectors holding a valid key
        const uint32_t tail = len & 7u;       // valid keys of vector nv - 1 (0: all 8)
        const uint4* xr = reinterpret_cast<const uint4*>(x + row * p.cols);
        uint4* orow = reinterpret_cast<uint4*>(out + row * p.cols);
        uint4 raw[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nv) raw[k] = ld_stream(xr + v);
        }
        uint32_t mx = 0xff80ff80u;  // (-inf, -inf)
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nv) {
                if (tail && v == nv - 1) raw[k] = bf16_tail(raw[k], tail, 0xff80u);
                mx = bf16x2_max(mx, bf16x2_max(bf16x2_max(raw[k].x, raw[k].y),
                                               bf16x2_max(raw[k].z, raw[k].w)));
            }
        }
        const float m = warp_max(fmaxf(bf16_lo(mx), bf16_hi(mx)));
        const float c2 = fmul(-fmul(m, p.scale), kLog2e);
        float2 acc = f2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nv) {
                const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 t = __ffma2_rn(f2(bf16_lo(w[i]), bf16_hi(w[i])), f2(c1, c1), f2(c2, c2));
                    acc = fadd2(acc, f2(ex2_approx(t.x), ex2_approx(t.y)));
                }
            }
        }
        const float c3 = fsub(c2, lg2_approx(warp_sum(fadd(acc.x, acc.y))));
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nvec) {
                uint4 o = make_uint4(0u, 0u, 0u, 0u);
                if (v < nv) {
                    const uint32_t r[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 t = __ffma2_rn(f2(bf16_lo(r[i]), bf16_hi(r[i])), f2(c1, c1), f2(c3, c3));
                        w[i] = pack_bf16x2(ex2_approx(t.x), ex2_approx(t.y));
                    }
                    o = make_uint4(w[0], w[1], w[2], w[3]);
                    if (tail && v == nv - 1) o = bf16_tail(o, tail, 0u);
                }
                st_stream(orow + v, o);
            }
        }
    }
}

template <int VPT>
static cudaError_t launch_bf16_warp(const bf16_t* x, bf16_t* out, const SmaxArgs& p, cudaStream_t st) {
    const auto kern = smax_bf16_warp_kernel<VPT>;
    const uint64_t want = (p.rows + 7) / 8;
    // two CTAs per resident slot: measured ~2% faster than one
    const uint64_t cap = 2ull * resident_blocks(reinterpret_cast<const void*>(kern), 256, 0);
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    launch_k(kern, grid, 256, 0, st, x, out, p);
    return cudaSuccess;
}

// The bf16 warp kernel serves rows of whole vectors up to 2048 keys when the
// scores are x * scale with 0 < scale < inf and no additive mask.
template <typename T>
static bool try_bf16_warp(const T* x, T* out, const SmaxArgs& p, cudaStream_t st, cudaError_t& e) {
    if constexpr (!std::is_same<T, bf16_t>::value) {
        return false;
    } else {
        if (p.mask || !(p.scale > 0.0f && p.scale <= 3.4028235e38f)) return false;
        if (p.cols % 8 != 0 || p.cols > 2048 || !aligned16(x) || !aligned16(out)) return false;
        const uint32_t nvec = p.cols / 8;
        if (nvec <= 32) e = launch_bf16_warp<1>(x, out, p, st);
        else if (nvec <= 64) e = launch_bf16_warp<2>(x, out, p, st);
        else if (nvec <= 128) e = launch_bf16_warp<4>(x, out, p, st);
        else e = launch_bf16_warp<8>(x, out, p, st);
        return true;
    }
}

template <typename T>
static int rows_dispatch(const char* name, const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    // 32-bit multiply-shift divisions for the per-row lens / causal lookups.
    p.narrow = p.rows < 0xffffffffull;
    p.len_div = FastDiv((uint32_t)(p.rows_per_len < 0xffffffffull ? p.rows_per_len : 0xffffffffull));
    p.causal_div = FastDiv((uint32_t)(p.causal_q ? p.causal_q : 1));
    {
        cudaError_t e = cudaSuccess;
        if (try_bf16_warp(x, out, p, st, e)) {
            if (e != cudaSuccess) {
                cudaGetLastError();
                return set_error(OXIDE_ERR_LAUNCH, "%s: launch failed: %s", name, cudaGetErrorString(e));
            }
            return check_launch(name);
        }
    }
    constexpr int VT = SMAX_VPT;
    const uint64_t cap = (uint64_t)1 << 30;
    const uint64_t nvec = p.cols / V;
    const bool vec = p.cols % V == 0 && aligned16(x) && aligned16(out);
    int vpt = 0;
    p.cl = 1;
    if (vec && nvec <= 32ull * VT) {  // a warp per row, 8 rows per tile
        p.tpr = 32;
        vpt = 1;
        while ((uint64_t)vpt * 32 < nvec) vpt *= 2;
    } else if (vec && nvec <= 256ull * VT) {  // 64..256 threads per row
        uint64_t tpr = 64;
        while (tpr * VT < nvec) tpr *= 2;
        p.tpr = (int)tpr;
        vpt = VT;
    }
    cudaError_t e = cudaSuccess;
    if (!vec) {
        launch_k(smax_rows_scalar_kernel<T>, (unsigned)(p.rows < cap ? p.rows : cap), 256, 0, st, x, out, p);
    } else if (p.mask) {
        e = launch_vec<T, true>(x, out, p, vpt, st);
    } else {
        e = launch_vec<T, false>(x, out, p, vpt, st);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(OXIDE_ERR_LAUNCH, "%s: launch failed: %s", name, cudaGetErrorString(e));
    }
    return check_launch(name);
}

template <typename T>
static int scale_mask_entry(const char* name, const T* x, T* out, uint64_t rows, uint64_t cols,
                            float scale, const float* mask, uint64_t mask_len,
                            const int32_t* lens, uint64_t rows_per_len, uint64_t causal_q,
                            cudaStream_t st) {
    OXIDE_INJECT(name);
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && out, name, "null pointer");
    OXIDE_REQUIRE(cols >= 1 && cols < (1ull << 31), name, "cols must be in [1, 2^31)");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    OXIDE_REQUIRE(!mask || (mask_len >= 1 && mask_len < (1ull << 32)), name,
                  "mask_len must be in [1, 2^32)");
    OXIDE_REQUIRE(!lens || rows_per_len >= 1, name, "rows_per_len must be >= 1 with lens");
    OXIDE_REQUIRE(causal_q <= cols, name, "causal_q_len must be <= cols");
    SmaxArgs p{};
    p.rows = rows;
    p.cols = (uint32_t)cols;
    p.scale = scale;
    p.mask = mask;
    p.mask_len = mask ? (uint32_t)mask_len : 1u;
    p.mask_div = FastDiv(p.mask_len);
    p.lens = lens;
    p.rows_per_len = lens ? rows_per_len : 1;
    p.causal_q = causal_q;
    return rows_dispatch<T>(name, x, out, p, st);
}

template <typename T>
static int softmax_entry(const char* name, const T* x, T* out, uint64_t outer, uint64_t dim,
                         uint64_t inner, cudaStream_t st) {
    OXIDE_INJECT(name);
    if (outer == 0 || inner == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && out, name, "null pointer");
    OXIDE_REQUIRE(dim >= 1 && dim < (1ull << 31), name, "dim must be in [1, 2^31)");
    OXIDE_REQUIRE(outer <= UINT64_MAX / dim / inner, name, "outer * dim * inner overflows");
    if (inner == 1) {
        SmaxArgs p{};
        p.rows = outer;
        p.cols = (uint32_t)dim;
        p.scale = 1.0f;  // x * 1.0f is exact: plain softmax
        p.mask_len = 1;
        p.mask_div = FastDiv(1);
        p.rows_per_len = 1;
        return rows_dispatch<T>(name, x, out, p, st);
    }
    OXIDE_REQUIRE(x != out, name, "out must not alias x when inner > 1");
    const uint64_t total = outer * inner;
    const uint64_t blocks = (total + 255) / 256;
    const uint64_t cap = (uint64_t)sm_count() * 8;
    launch_k(smax_inner_kernel<T>, (unsigned)(blocks < cap ? blocks : cap), 256, 0, st, x, out, outer, dim,
                                                                                  inner);
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_softmax_f32(const float* x, float* out, uint64_t outer, uint64_t dim, uint64_t inner,
                      oxide_stream_t stream) {
    return oxide::softmax_entry<float>("oxide_softmax_f32", x, out, outer, dim, inner, stream);
}
int oxide_softmax_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t outer, uint64_t dim,
                       uint64_t inner, oxide_stream_t stream) {
    return oxide::softmax_entry<bf16_t>("oxide_softmax_bf16", x, out, outer, dim, inner, stream);
}
int oxide_scale_mask_softmax_f32(const float* x, float* out, uint64_t rows, uint64_t cols,
                                 float scale, const float* mask, uint64_t mask_len,
                                 const int32_t* lens, uint64_t rows_per_len,
                                 uint64_t causal_q_len, oxide_stream_t stream) {
    return oxide::scale_mask_entry<float>("oxide_scale_mask_softmax_f32", x, out, rows, cols,
                                          scale, mask, mask_len, lens, rows_per_len,
                                          causal_q_len, stream);
}
int oxide_scale_mask_softmax_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t rows,
                                  uint64_t cols, float scale, const float* mask,
                                  uint64_t mask_len, const int32_t* lens,
                                  uint64_t rows_per_len, uint64_t causal_q_len,
                                  oxide_stream_t stream) {
    return oxide::scale_mask_entry<bf16_t>("oxide_scale_mask_softmax_bf16", x, out, rows, cols,
                                           scale, mask, mask_len, lens, rows_per_len,
                                           causal_q_len, stream);
}

}  // extern "C"
