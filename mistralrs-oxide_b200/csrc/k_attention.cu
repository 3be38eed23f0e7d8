// k_attention.cu -- one-token (decode) attention over a KV cache (flash-decoding).
//
// Reference: the inline attention of scaled_dot_product_attention
// (src/ops/attention.rs:41-87) for q_len = 1: s_j = (q . k_j) * scale,
// softmax over the keys, out = sum_j p_j v_j; grouped-query heads read their
// kv head directly (q head h uses kv head h / (q_heads / kv_heads), the head
// map of repeat_kv, attention.rs:161-201) instead of materialising repeat_kv;
// keys j >= lens[b] (the sequence's KV length) are masked.
//
// Design (split-K, two launches):
//   1. grid (splits, kv_heads, batch): one CTA streams the keys
//      [split * split_len, ...) of one (batch, kv head) into shared memory with
//      16-byte cp.async copies (rows padded by 16 bytes against bank
//      conflicts), computes the scores of all `rep` query heads of the group
//      (each K row is read from HBM once for the group), keeps a running max /
//      sum per head (online softmax) and accumulates the unnormalised output;
//      it writes (m, l, o[d]) per head to the workspace.  bf16 caches: four
//      warps stream interleaved 16-key tiles independently and run both tile
//      products on the tensor cores (decode_attn_warp_kernel); f32 caches: a
//      two-stage block ring on the CUDA cores, thread d owning output dim d
//      (decode_attn_split_kernel);
//   2. one CTA per (batch, q head) merges the splits in order:
//      M = max m_s, L = sum l_s e^(m_s - M), out = sum o_s e^(m_s - M) / L.
// Arithmetic is f32 accumulation (bf16 operands multiplied exactly), dot
// products and P.V with fused multiply-adds; the result differs from the
// reference's sequential f32 sums by rounding only.  head_dim 128 with rep in
// {1, 2, 4, 8} takes this path; other shapes take a one-CTA-per-(batch, head)
// kernel.  A sequence of length 0 yields zeros.
#include <type_traits>

#include "oxide_common.cuh"

namespace oxide {

struct DecArgs {
    uint64_t batch, max_seq;
    uint32_t q_heads, kv_heads, rep, head_dim;
    uint32_t split_len, splits;
    float scale;
    const int32_t* lens;
};

constexpr int DA_D = 128;        // head_dim of the split-K path
constexpr int DA_THREADS = 128;  // one thread per output dim

__device__ __forceinline__ uint64_t seq_len_of(const DecArgs& p, uint64_t b) {
    if (!p.lens) return p.max_seq;
    const int32_t l = p.lens[b];
    return l < 0 ? 0 : ((uint64_t)l < p.max_seq ? (uint64_t)l : p.max_seq);
}

template <typename T>
struct DaTile {
    static constexpr int RB = DA_D * (int)sizeof(T);  // bytes per cached row
    static constexpr int RS = RB + 16;                // shared-memory row stride
    static constexpr int TK = sizeof(T) == 2 ? 64 : 32;  // keys per tile
    static constexpr int CPR = RB / 16;               // 16-byte chunks per row
    static constexpr int TPK = DA_THREADS / TK;       // threads per key in the score pass
    static constexpr int DPT = DA_D / TPK;            // dims per thread in the score pass
};

template <typename T, int NR>
constexpr size_t decode_smem_bytes() {
    return (size_t)4 * DaTile<T>::TK * DaTile<T>::RS + (size_t)NR * DA_D * 4 + (size_t)NR * DaTile<T>::TK * 4 +
           (size_t)4 * NR * 4;
}

template <typename T, int NR>
__global__ void __launch_bounds__(DA_THREADS)
    decode_attn_split_kernel(const T* q, const T* kc, const T* vc, float* part_ml, float* part_o, DecArgs p) {
    using TL = DaTile<T>;
    constexpr int TK = TL::TK, RS = TL::RS, RB = TL::RB, CPR = TL::CPR, TPK = TL::TPK, DPT = TL::DPT;
    constexpr int V = 16 / (int)sizeof(T);
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char* kbuf = smem;
    unsigned char* vbuf = smem + 2 * TK * RS;
    float* qs = reinterpret_cast<float*>(smem + 4 * TK * RS);  // [NR][D]
    float* S = qs + NR * DA_D;                                 // [NR][TK]
    float* m_run = S + NR * TK;                                // [NR]
    float* l_run = m_run + NR;
    float* corr = l_run + NR;

    const uint32_t split = blockIdx.x, kvh = blockIdx.y;
    const uint64_t b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t len = seq_len_of(p, b);
    const uint64_t s0 = (uint64_t)split * p.split_len;
    const uint64_t s1 = s0 + p.split_len < len ? s0 + p.split_len : len;
    const uint32_t qh0 = kvh * NR;

    for (int i = tid; i < NR * DA_D; i += DA_THREADS)
        qs[i] = Vec<T>::load1(q + (b * p.q_heads + qh0 + i / DA_D) * DA_D + (i % DA_D));
    if (tid < NR) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.0f;
    }
    float o[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) o[r] = 0.0f;

    const uint64_t row0 = (b * p.kv_heads + kvh) * p.max_seq;
    const char* kbase = reinterpret_cast<const char*>(kc + row0 * DA_D);
    const char* vbase = reinterpret_cast<const char*>(vc + row0 * DA_D);
    const uint32_t nkeys = s1 > s0 ? (uint32_t)(s1 - s0) : 0u;
    const uint32_t ntiles = (nkeys + TK - 1) / TK;
    auto issue = [&](uint32_t t) {
        const uint32_t stage = t & 1u;
        const uint64_t key0 = s0 + (uint64_t)t * TK;
        const uint32_t nk = nkeys - t * TK < (uint32_t)TK ? nkeys - t * TK : (uint32_t)TK;
        for (uint32_t c = tid; c < nk * CPR; c += DA_THREADS) {
            const uint32_t row = c / CPR, col = c % CPR;
            const uint64_t src = (key0 + row) * RB + col * 16;
            cp_async16(kbuf + stage * TK * RS + row * RS + col * 16, kbase + src);
            cp_async16(vbuf + stage * TK * RS + row * RS + col * 16, vbase + src);
        }
        cp_async_commit();
    };
    if (ntiles > 0) issue(0);
    __syncthreads();  // qs, m_run, l_run visible
    for (uint32_t t = 0; t < ntiles; ++t) {
        if (t + 1 < ntiles) issue(t + 1);
        else cp_async_commit();  // empty group: the wait below counts uniformly
        cp_async_wait<1>();
        __syncthreads();  // tile t is in shared memory for every thread
        const uint32_t stage = t & 1u;
        const uint32_t nk = nkeys - t * TK < (uint32_t)TK ? nkeys - t * TK : (uint32_t)TK;
        // scores: TPK threads per key, DPT dims each
        {
            const int jj = tid / TPK, part = tid % TPK;
            float acc[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
            if ((uint32_t)jj < nk) {
                const unsigned char* krow = kbuf + stage * TK * RS + jj * RS + part * DPT * (int)sizeof(T);
#pragma unroll
                for (int c = 0; c < DPT / V; ++c) {
                    float kf[V];
                    Vec<T>::unpack(lds16(krow + c * 16), kf);
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        const float4* qv = reinterpret_cast<const float4*>(qs + r * DA_D + part * DPT + c * V);
#pragma unroll
                        for (int e4 = 0; e4 < V / 4; ++e4) {
                            const float4 qq = qv[e4];
                            acc[r] = __fmaf_rn(qq.x, kf[4 * e4], acc[r]);
                            acc[r] = __fmaf_rn(qq.y, kf[4 * e4 + 1], acc[r]);
                            acc[r] = __fmaf_rn(qq.z, kf[4 * e4 + 2], acc[r]);
                            acc[r] = __fmaf_rn(qq.w, kf[4 * e4 + 3], acc[r]);
                        }
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < NR; ++r) {
#pragma unroll
                for (int o2 = 1; o2 < TPK; o2 <<= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o2));
                if (part == 0) S[r * TK + jj] = (uint32_t)jj < nk ? fmul(acc[r], p.scale) : -INFINITY;
            }
        }
        __syncthreads();
        // online softmax per head: warp w handles heads w, w + 4, ...
        for (int r = warp; r < NR; r += DA_THREADS / 32) {
            float* sr = S + r * TK;
            float tmax = -INFINITY;
            for (int j = lane; j < TK; j += 32) tmax = fmaxf(tmax, sr[j]);
            tmax = warp_max(tmax);
            const float m_old = m_run[r];
            const float m_new = fmaxf(m_old, tmax);
            float psum = 0.0f;
            for (int j = lane; j < TK; j += 32) {
                const float pj = m_new == -INFINITY ? 0.0f : expf(fsub(sr[j], m_new));
                sr[j] = pj;
                psum = fadd(psum, pj);
            }
            psum = warp_sum(psum);
            if (lane == 0) {
                const float c = m_old == -INFINITY ? 0.0f : expf(fsub(m_old, m_new));
                corr[r] = c;
                l_run[r] = __fmaf_rn(l_run[r], c, psum);
                m_run[r] = m_new;
            }
        }
        __syncthreads();
        // P.V: thread d accumulates o[r] += p[r][j] * v[j][d]
        {
            const int d = tid;
#pragma unroll
            for (int r = 0; r < NR; ++r) o[r] = fmul(o[r], corr[r]);
            const unsigned char* vcol = vbuf + stage * TK * RS + d * (int)sizeof(T);
            auto vat = [&](uint32_t j) {
                if (sizeof(T) == 4) return *reinterpret_cast<const float*>(vcol + j * RS);
                return bf16_to_f32(*reinterpret_cast<const bf16_t*>(vcol + j * RS));
            };
            uint32_t j = 0;
            for (; j + 4 <= nk; j += 4) {  // probabilities 4 at a time (one 16-byte load per head)
                const float v0 = vat(j), v1 = vat(j + 1), v2 = vat(j + 2), v3 = vat(j + 3);
#pragma unroll
                for (int r = 0; r < NR; ++r) {
                    const float4 pp = *reinterpret_cast<const float4*>(S + r * TK + j);
                    o[r] = __fmaf_rn(pp.x, v0, o[r]);
                    o[r] = __fmaf_rn(pp.y, v1, o[r]);
                    o[r] = __fmaf_rn(pp.z, v2, o[r]);
                    o[r] = __fmaf_rn(pp.w, v3, o[r]);
                }
            }
            for (; j < nk; ++j) {  // rows past nk hold stale data: never read
                const float v = vat(j);
#pragma unroll
                for (int r = 0; r < NR; ++r) o[r] = __fmaf_rn(S[r * TK + j], v, o[r]);
            }
        }
        __syncthreads();  // every thread is done with this stage before it is refilled
    }
    cp_async_wait<0>();
    // partial results of this split
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const uint64_t slot = ((b * p.q_heads + qh0 + r) * p.splits + split);
        part_o[slot * DA_D + tid] = o[r];
        if (tid == 0) {
            part_ml[slot * 2] = m_run[r];
            part_ml[slot * 2 + 1] = l_run[r];
        }
    }
}

// ---- bf16 caches: per-warp key streams on the tensor cores -------------------
// Each warp of a 4-warp CTA streams every 4th 16-key tile of the split through
// its own 3-stage cp.async ring and keeps its own online-softmax state, so the
// key loop has no block barrier; the four warp states are merged once at the
// end.  The tile products run transposed on warp-level mma.sync m16n8k16
// (bf16 operands, f32 accumulate) so that the rep <= 8 query heads of the
// group are the n = 8 side:
//   S^T[16 keys x 8 heads]  = K[16 x 128] . Q^T       (A = K rows, ldmatrix)
//   O^T[128 dims x 8 heads] += V^T[128 x 16] . P^T    (A = V rows, ldmatrix.trans)
// The score fragment (key g / g + 8, heads 2t4, 2t4 + 1) becomes the P^T
// operand fragment (keys 2t4.., head g) by one movmatrix.trans per 8x8 block,
// without a round trip through shared memory.  Q . K: bf16 x bf16 products
// are exact in the f32 accumulator.  P enters as the sum of two bf16 halves
// (p_hi = RN_bf16(p), p_lo = RN_bf16(p - p_hi): 16 significant bits), so P V
// keeps f32-level accuracy.  Scores are kept in the base-2 domain,
// t = (q . k) * (scale * log2 e), and p = ex2.approx(t - m): relative error
// ~2^-22 per probability, far below the bf16 output rounding (2^-9).
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// d += a * b for one 16x8x16 tile (A row-major 16x16, B column-major 16x8).
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Transpose an 8x8 b16 matrix held as one fragment register per lane
// (lane g * 4 + t holds row g, columns 2t and 2t + 1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

constexpr int DW_WARPS = 4;                                     // warps per CTA
constexpr int DW_TK = 16;                                       // keys per warp tile
constexpr int DW_STAGES = 3;                                    // cp.async ring depth per warp
constexpr int DW_RS = DA_D * 2 + 16;                            // 272-byte rows: conflict-free ldmatrix
constexpr int DW_STAGE = 2 * DW_TK * DW_RS;                     // K and V tile of one stage
constexpr size_t DW_SMEM = (size_t)DW_WARPS * DW_STAGES * DW_STAGE;  // 104,448 B: 2 CTAs per SM
constexpr float DW_LOG2E = 1.4426950408889634f;
constexpr float DW_LN2 = 0.6931471805599453f;

template <int NR>
__global__ void __launch_bounds__(DW_WARPS * 32, 2)
    decode_attn_warp_kernel(const bf16_t* q, const bf16_t* kc, const bf16_t* vc, float* part_ml, float* part_o,
                            DecArgs p) {
    static_assert(DW_WARPS * 32 == DA_D, "the merge maps one thread to one output dim");
    extern __shared__ __align__(16) unsigned char smem[];
    const uint32_t split = blockIdx.x, kvh = blockIdx.y;
    const uint64_t b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;  // fragment row group / thread in group
    const uint64_t len = seq_len_of(p, b);
    const uint64_t s0 = (uint64_t)split * p.split_len;
    const uint64_t s1 = s0 + p.split_len < len ? s0 + p.split_len : len;
    const uint32_t nkeys = s1 > s0 ? (uint32_t)(s1 - s0) : 0u;
    const uint32_t ntiles = (nkeys + DW_TK - 1) / DW_TK;
    const uint32_t qh0 = kvh * NR;

    // Q^T as the B operand: b0 = Q[head g][16 ks + 2 t4, +1], b1 = Q[head g][16 ks + 8 + 2 t4, +1]
    uint32_t qb0[8], qb1[8];
    {
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(q + (b * p.q_heads + qh0 + (g < NR ? g : 0)) * DA_D);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            qb0[ks] = g < NR ? qrow[ks * 8 + t4] : 0u;
            qb1[ks] = g < NR ? qrow[ks * 8 + 4 + t4] : 0u;
        }
    }
    // O^T m-tile mt: o[mt][0] (dim 16 mt + g, head 2 t4), [1] (same dim, head 2 t4 + 1),
    // [2] / [3] the same heads at dim 16 mt + g + 8
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[mt][e] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY;  // running max of heads 2 t4, 2 t4 + 1 (base 2)
    float l0 = 0.0f, l1 = 0.0f;            // this lane's share of the running sums
    const float c1 = fmul(p.scale, DW_LOG2E);

    unsigned char* wbuf = smem + (size_t)warp * DW_STAGES * DW_STAGE;
    const uint64_t row0 = (b * p.kv_heads + kvh) * p.max_seq + s0;
    const char* kbase = reinterpret_cast<const char*>(kc + row0 * DA_D);
    const char* vbase = reinterpret_cast<const char*>(vc + row0 * DA_D);
    // copy slots of this lane: rows 2 i + (lane >> 4), 16-byte column lane & 15
    const uint32_t crow = lane >> 4, ccol = (lane & 15) * 16;
    const uint32_t my_tiles = ntiles > (uint32_t)warp ? (ntiles - warp + DW_WARPS - 1) / DW_WARPS : 0u;
    auto issue = [&](uint32_t it) {
        unsigned char* kd = wbuf + (it % DW_STAGES) * DW_STAGE;
        unsigned char* vd = kd + DW_TK * DW_RS;
        const uint32_t key0 = (warp + it * DW_WARPS) * DW_TK;
        const uint32_t nk = nkeys - key0 < (uint32_t)DW_TK ? nkeys - key0 : (uint32_t)DW_TK;
#pragma unroll
        for (int i = 0; i < DW_TK / 2; ++i) {
            const uint32_t row = 2 * i + crow;
            // rows past the last key repeat the last key: finite data that p = 0 multiplies
            const uint32_t src = row < nk ? row : nk - 1;
            const uint64_t off = (uint64_t)(key0 + src) * (DA_D * 2) + ccol;
            cp_async16(kd + row * DW_RS + ccol, kbase + off);
            cp_async16(vd + row * DW_RS + ccol, vbase + off);
        }
    };
#pragma unroll
    for (int s = 0; s < DW_STAGES - 1; ++s) {
        if ((uint32_t)s < my_tiles) issue(s);
        cp_async_commit();
    }
    const uint32_t wbuf_s = (uint32_t)__cvta_generic_to_shared(wbuf);
    // ldmatrix row addresses: K as A (keys x dims), V as A^T (dims x keys)
    const uint32_t k_lane = ((lane & 7) + ((lane >> 3) & 1) * 8) * DW_RS + (lane >> 4) * 16;
    const uint32_t v_lane = DW_TK * DW_RS + ((lane & 7) + (lane >> 4) * 8) * DW_RS + ((lane >> 3) & 1) * 16;
    for (uint32_t it = 0; it < my_tiles; ++it) {
        if (it + DW_STAGES - 1 < my_tiles) issue(it + DW_STAGES - 1);
        cp_async_commit();
        cp_async_wait<DW_STAGES - 1>();
        __syncwarp();  // every lane's copies of this tile are visible to the warp
        const uint32_t base = wbuf_s + (it % DW_STAGES) * DW_STAGE;
        const uint32_t key0 = (warp + it * DW_WARPS) * DW_TK;
        const uint32_t nk = nkeys - key0 < (uint32_t)DW_TK ? nkeys - key0 : (uint32_t)DW_TK;
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(base + k_lane + ks * 32, a0, a1, a2, a3);
            mma_bf16(s, a0, a1, a2, a3, qb0[ks], qb1[ks]);
        }
        // s: (key g, head 2t4), (key g, head 2t4+1), (key g+8, head 2t4), (key g+8, head 2t4+1)
        const float t0 = (uint32_t)g < nk ? fmul(s[0], c1) : -INFINITY;
        const float t1 = (uint32_t)g < nk ? fmul(s[1], c1) : -INFINITY;
        const float t2 = (uint32_t)g + 8 < nk ? fmul(s[2], c1) : -INFINITY;
        const float t3 = (uint32_t)g + 8 < nk ? fmul(s[3], c1) : -INFINITY;
        float x0 = fmaxf(t0, t2), x1 = fmaxf(t1, t3);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, off));
            x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, off));
        }
        const float mn0 = fmaxf(m0, x0), mn1 = fmaxf(m1, x1);
        const float cr0 = m0 == -INFINITY ? 0.0f : ex2_approx(fsub(m0, mn0));
        const float cr1 = m1 == -INFINITY ? 0.0f : ex2_approx(fsub(m1, mn1));
        m0 = mn0;
        m1 = mn1;
        const float p0 = mn0 == -INFINITY ? 0.0f : ex2_approx(fsub(t0, mn0));
        const float p2 = mn0 == -INFINITY ? 0.0f : ex2_approx(fsub(t2, mn0));
        const float p1 = mn1 == -INFINITY ? 0.0f : ex2_approx(fsub(t1, mn1));
        const float p3 = mn1 == -INFINITY ? 0.0f : ex2_approx(fsub(t3, mn1));
        l0 = __fmaf_rn(l0, cr0, fadd(p0, p2));
        l1 = __fmaf_rn(l1, cr1, fadd(p1, p3));
        if (__any_sync(0xffffffffu, cr0 != 1.0f || cr1 != 1.0f)) {
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                o[mt][0] = fmul(o[mt][0], cr0);
                o[mt][1] = fmul(o[mt][1], cr1);
                o[mt][2] = fmul(o[mt][2], cr0);
                o[mt][3] = fmul(o[mt][3], cr1);
            }
        }
        // P^T operand: the 8x8 blocks P[keys 0-7 | 8-15][heads] transposed
        const float h0 = round_bf16(p0), h1 = round_bf16(p1), h2 = round_bf16(p2), h3 = round_bf16(p3);
        const uint32_t bh0 = movmatrix_trans(pack_bf16x2(h0, h1));
        const uint32_t bh1 = movmatrix_trans(pack_bf16x2(h2, h3));
        const uint32_t bl0 = movmatrix_trans(pack_bf16x2(fsub(p0, h0), fsub(p1, h1)));
        const uint32_t bl1 = movmatrix_trans(pack_bf16x2(fsub(p2, h2), fsub(p3, h3)));
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4_trans(base + v_lane + mt * 32, a0, a1, a2, a3);
            mma_bf16(o[mt], a0, a1, a2, a3, bh0, bh1);
            mma_bf16(o[mt], a0, a1, a2, a3, bl0, bl1);
        }
        __syncwarp();  // the whole warp is done with this stage before it is refilled
    }
    cp_async_wait<0>();
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l0 = fadd(l0, __shfl_xor_sync(0xffffffffu, l0, off));
        l1 = fadd(l1, __shfl_xor_sync(0xffffffffu, l1, off));
    }
    // merge the four warp states: [W][8] max, [W][8] sum, [W][NR][D] output
    __syncthreads();  // every warp is done with its ring: the buffers are reused
    float* wm = reinterpret_cast<float*>(smem);
    float* wl = wm + DW_WARPS * 8;
    float* wo = wl + DW_WARPS * 8;
    if (g == 0) {
        wm[warp * 8 + 2 * t4] = m0;
        wm[warp * 8 + 2 * t4 + 1] = m1;
        wl[warp * 8 + 2 * t4] = l0;
        wl[warp * 8 + 2 * t4 + 1] = l1;
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        const int d0 = mt * 16 + g;
        if (2 * t4 < NR) {
            wo[(warp * NR + 2 * t4) * DA_D + d0] = o[mt][0];
            wo[(warp * NR + 2 * t4) * DA_D + d0 + 8] = o[mt][2];
        }
        if (2 * t4 + 1 < NR) {
            wo[(warp * NR + 2 * t4 + 1) * DA_D + d0] = o[mt][1];
            wo[(warp * NR + 2 * t4 + 1) * DA_D + d0 + 8] = o[mt][3];
        }
    }
    __syncthreads();
    const int d = tid;
#pragma unroll
    for (int h = 0; h < NR; ++h) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < DW_WARPS; ++w) M = fmaxf(M, wm[w * 8 + h]);
        float L = 0.0f, acc = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < DW_WARPS; ++w) {
                const float mw = wm[w * 8 + h];
                if (mw == -INFINITY) continue;
                const float sc = ex2_approx(fsub(mw, M));
                L = __fmaf_rn(wl[w * 8 + h], sc, L);
                acc = __fmaf_rn(wo[(w * NR + h) * DA_D + d], sc, acc);
            }
        }
        const uint64_t slot = (b * p.q_heads + qh0 + h) * p.splits + split;
        part_o[slot * DA_D + d] = acc;
        if (d == 0) {
            part_ml[slot * 2] = M == -INFINITY ? M : fmul(M, DW_LN2);  // natural-log domain for the merge
            part_ml[slot * 2 + 1] = L;
        }
    }
}

// Merge the splits of one (batch, q head); thread d writes out[d].
template <typename T>
__global__ void __launch_bounds__(DA_THREADS)
    decode_attn_combine_kernel(const float* part_ml, const float* part_o, T* out, DecArgs p) {
    const uint64_t bh = blockIdx.x;
    const int d = threadIdx.x;
    const uint64_t base = bh * p.splits;
    float M = -INFINITY;
    for (uint32_t s = 0; s < p.splits; ++s) M = fmaxf(M, part_ml[(base + s) * 2]);
    float res = 0.0f;
    if (M != -INFINITY) {
        float L = 0.0f, acc = 0.0f;
        for (uint32_t s = 0; s < p.splits; ++s) {
            const float ms = part_ml[(base + s) * 2];
            if (ms == -INFINITY) continue;
            const float w = expf(fsub(ms, M));
            L = __fmaf_rn(part_ml[(base + s) * 2 + 1], w, L);
            acc = __fmaf_rn(part_o[(base + s) * DA_D + d], w, acc);
        }
        res = fdiv(acc, L);
    }
    Vec<T>::store1(out + bh * DA_D + d, res);
}

// General shapes: one CTA per (batch, q head), three passes over the keys
// (scores into the workspace, max / sum, P.V); head_dim any, rep any.
template <typename T>
__global__ void __launch_bounds__(256)
    decode_attn_generic_kernel(const T* q, const T* kc, const T* vc, T* out, float* scores, DecArgs p) {
    __shared__ float red[32];
    const uint64_t bh = blockIdx.x, b = bh / p.q_heads;
    const uint32_t qh = (uint32_t)(bh % p.q_heads), kvh = qh / p.rep;
    const uint64_t len = seq_len_of(p, b);
    const T* qr = q + bh * p.head_dim;
    const T* kr = kc + (b * p.kv_heads + kvh) * p.max_seq * p.head_dim;
    const T* vr = vc + (b * p.kv_heads + kvh) * p.max_seq * p.head_dim;
    float* sc = scores + bh * p.max_seq;
    float m = -INFINITY;
    for (uint64_t j = threadIdx.x; j < len; j += blockDim.x) {
        float dot = 0.0f;
        for (uint32_t i = 0; i < p.head_dim; ++i)
            dot = __fmaf_rn(Vec<T>::load1(qr + i), Vec<T>::load1(kr + j * p.head_dim + i), dot);
        sc[j] = fmul(dot, p.scale);
        m = fmaxf(m, sc[j]);
    }
    m = group_reduce(m, red, (int)blockDim.x, OpMaxF());
    float s = 0.0f;
    for (uint64_t j = threadIdx.x; j < len; j += blockDim.x) {
        const float e = expf(fsub(sc[j], m));
        sc[j] = e;
        s = fadd(s, e);
    }
    s = group_reduce(s, red, (int)blockDim.x, OpAddF());
    __syncthreads();  // all probabilities written
    for (uint32_t i = threadIdx.x; i < p.head_dim; i += blockDim.x) {
        float acc = 0.0f;
        for (uint64_t j = 0; j < len; ++j) acc = __fmaf_rn(sc[j], Vec<T>::load1(vr + j * p.head_dim + i), acc);
        Vec<T>::store1(out + bh * p.head_dim + i, len == 0 ? 0.0f : fdiv(acc, s));
    }
}

// Workspace: split-K partials (2 + head_dim floats per (batch, q head, split))
// or the generic kernel's score rows.
static uint32_t max_splits(uint64_t max_seq, uint64_t tk) {
    const uint64_t s = (max_seq + tk - 1) / tk;
    return (uint32_t)(s < 1 ? 1 : (s > 1024 ? 1024 : s));
}

template <typename T, int NR>
static cudaError_t launch_split(const T* q, const T* kc, const T* vc, T* out, float* ws, DecArgs p,
                                cudaStream_t st) {
    float* part_ml = ws;
    float* part_o = ws + (size_t)2 * p.batch * p.q_heads * p.splits;
    const dim3 grid(p.splits, p.kv_heads, (unsigned)p.batch);
    if constexpr (std::is_same<T, bf16_t>::value) {  // tensor-core tile products
        auto kern = decode_attn_warp_kernel<NR>;
        if (!ensure_dyn_smem(reinterpret_cast<const void*>(kern), DW_SMEM)) return cudaErrorInvalidConfiguration;
        kern<<<grid, DW_WARPS * 32, DW_SMEM, st>>>(q, kc, vc, part_ml, part_o, p);
    } else {
        auto kern = decode_attn_split_kernel<T, NR>;
        const size_t smem = decode_smem_bytes<T, NR>();
        if (!ensure_dyn_smem(reinterpret_cast<const void*>(kern), smem)) return cudaErrorInvalidConfiguration;
        kern<<<grid, DA_THREADS, smem, st>>>(q, kc, vc, part_ml, part_o, p);
    }
    decode_attn_combine_kernel<T><<<(unsigned)(p.batch * p.q_heads), DA_THREADS, 0, st>>>(part_ml, part_o, out, p);
    return cudaSuccess;
}

template <typename T>
static int decode_entry(const char* name, const T* q, const T* kc, const T* vc, const int32_t* lens, T* out,
                        uint64_t batch, uint64_t q_heads, uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim,
                        float scale, void* ws, uint64_t ws_bytes, cudaStream_t st) {
    OXIDE_INJECT(name);
    if (batch == 0 || q_heads == 0) return OXIDE_OK;
    OXIDE_REQUIRE(q && kc && vc && out, name, "null pointer");
    OXIDE_REQUIRE(kv_heads >= 1 && q_heads % kv_heads == 0, name, "q_heads must be a multiple of kv_heads");
    OXIDE_REQUIRE(q_heads < (1u << 20) && head_dim >= 1 && head_dim < (1u << 16), name,
                  "q_heads must be < 2^20 and head_dim in [1, 65536)");
    OXIDE_REQUIRE(batch < (1u << 16) && max_seq >= 1 && max_seq < (1ull << 31), name,
                  "batch must be < 65536 and max_seq in [1, 2^31)");
    const uint64_t need = oxide_decode_attention_workspace_bytes(batch, q_heads, max_seq, head_dim);
    if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 15))
        return set_error(OXIDE_ERR_WORKSPACE, "%s: workspace must be 16-byte aligned and >= %llu bytes", name,
                         (unsigned long long)need);
    DecArgs p{};
    p.batch = batch;
    p.max_seq = max_seq;
    p.q_heads = (uint32_t)q_heads;
    p.kv_heads = (uint32_t)kv_heads;
    p.rep = (uint32_t)(q_heads / kv_heads);
    p.head_dim = (uint32_t)head_dim;
    p.scale = scale;
    p.lens = lens;
    const int rep = (int)p.rep;
    const bool fast = head_dim == DA_D && (rep == 1 || rep == 2 || rep == 4 || rep == 8) && aligned16(q) &&
                      aligned16(kc) && aligned16(vc) && kv_heads < 65536;
    cudaError_t e = cudaSuccess;
    if (fast) {
        // splits: enough CTAs for ~4 waves, whole tiles per split
        const uint64_t tk = DaTile<T>::TK;
        const uint64_t groups = batch * kv_heads;
        const uint64_t target = 4ull * 3 * sm_count();
        uint64_t splits = (target + groups - 1) / groups;
        const uint64_t cap = max_splits(max_seq, tk);
        if (splits > cap) splits = cap;
        if (splits < 1) splits = 1;
        uint64_t split_len = (max_seq + splits - 1) / splits;
        split_len = (split_len + tk - 1) / tk * tk;
        p.split_len = (uint32_t)split_len;
        p.splits = (uint32_t)((max_seq + split_len - 1) / split_len);
        float* w = static_cast<float*>(ws);
        switch (rep) {
            case 1: e = launch_split<T, 1>(q, kc, vc, out, w, p, st); break;
            case 2: e = launch_split<T, 2>(q, kc, vc, out, w, p, st); break;
            case 4: e = launch_split<T, 4>(q, kc, vc, out, w, p, st); break;
            default: e = launch_split<T, 8>(q, kc, vc, out, w, p, st); break;
        }
    } else {
        decode_attn_generic_kernel<T><<<(unsigned)(batch * q_heads), 256, 0, st>>>(q, kc, vc, out,
                                                                                  static_cast<float*>(ws), p);
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

uint64_t oxide_decode_attention_workspace_bytes(uint64_t batch, uint64_t q_heads, uint64_t max_seq,
                                                uint64_t head_dim) {
    // split-K partials at the finest split (tiles of 32 keys), or one score row per head
    const uint64_t splits = oxide::max_splits(max_seq, 32);
    const uint64_t split_k = batch * q_heads * splits * (2 + (uint64_t)oxide::DA_D) * sizeof(float);
    const uint64_t generic = batch * q_heads * max_seq * sizeof(float);
    (void)head_dim;
    return split_k > generic ? split_k : generic;
}
int oxide_decode_attention_f32(const float* q, const float* k_cache, const float* v_cache, const int32_t* lens,
                               float* out, uint64_t batch, uint64_t q_heads, uint64_t kv_heads, uint64_t max_seq,
                               uint64_t head_dim, float scale, void* workspace, uint64_t workspace_bytes,
                               oxide_stream_t stream) {
    return oxide::decode_entry<float>("oxide_decode_attention_f32", q, k_cache, v_cache, lens, out, batch, q_heads,
                                      kv_heads, max_seq, head_dim, scale, workspace, workspace_bytes, stream);
}
int oxide_decode_attention_bf16(const oxide_bf16* q, const oxide_bf16* k_cache, const oxide_bf16* v_cache,
                                const int32_t* lens, oxide_bf16* out, uint64_t batch, uint64_t q_heads,
                                uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim, float scale,
                                void* workspace, uint64_t workspace_bytes, oxide_stream_t stream) {
    return oxide::decode_entry<bf16_t>("oxide_decode_attention_bf16", q, k_cache, v_cache, lens, out, batch,
                                       q_heads, kv_heads, max_seq, head_dim, scale, workspace, workspace_bytes,
                                       stream);
}

}  // extern "C"
