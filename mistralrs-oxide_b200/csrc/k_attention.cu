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
//   1. grid (splits, kv_heads, batch): a 128-thread CTA streams the keys
//      [split * split_len, ...) of one (batch, kv head) through a two-stage
//      cp.async ring of 16-byte copies into shared memory (K and V tiles of 64
//      bf16 / 32 f32 rows, rows padded by 16 bytes against bank conflicts),
//      computes the scores of all `rep` query heads of the group (each K row
//      is read from HBM once for the group), keeps a running max / sum per
//      head (online softmax) and accumulates the unnormalised output in
//      registers (thread d owns output dim d); it writes (m, l, o[d]) per head
//      to the workspace;
//   2. one CTA per (batch, q head) merges the splits in order:
//      M = max m_s, L = sum l_s e^(m_s - M), out = sum o_s e^(m_s - M) / L.
// bf16 caches run the tile products on the tensor cores (decode_attn_mma_kernel);
// f32 caches on the CUDA cores.  Arithmetic is f32 accumulation (bf16 operands
// widened or multiplied exactly), dot products and P.V with fused
// multiply-adds; the result differs from the reference's sequential f32 sums
// by rounding only.  head_dim 128 with rep in {1, 2, 4, 8} takes this path;
// other shapes take a one-CTA-per-(batch, head) kernel.  A sequence of length 0
// yields zeros.
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

// ---- bf16 caches: the two tile products on the tensor cores --------------------
// Same split-K structure and cp.async ring as decode_attn_split_kernel, with
// S = Q K^T and O += P V as warp-level mma.sync m16n8k16 (bf16 operands, f32
// accumulate).  The rep query heads of the group are rows 0..rep-1 of a
// 16-row A operand (the rest zero); a memory-bound op, so the padding costs
// nothing -- the tensor cores replace the per-element shared-memory loads
// and FMAs that made the CUDA-core loop instruction-bound (tcgen05's smallest
// tile, 64 rows, would be 94 % padding for 4 heads).  Q . K: bf16 x bf16
// products are exact in the f32 accumulator.  P enters as the sum of two bf16
// halves (p_hi = RN_bf16(p), p_lo = RN_bf16(p - p_hi): 16 significant bits)
// multiplied by the bf16 V rows, so P V keeps f32-level accuracy.
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
// d += a * b for one 16x8x16 tile; rows 8..15 of A are zero here (a1 = a3 = 0).
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

template <int NR>
__global__ void __launch_bounds__(DA_THREADS)
    decode_attn_mma_kernel(const bf16_t* q, const bf16_t* kc, const bf16_t* vc, float* part_ml, float* part_o,
                           DecArgs p) {
    using TL = DaTile<bf16_t>;
    constexpr int TK = TL::TK, RS = TL::RS, RB = TL::RB, CPR = TL::CPR;  // 64 keys, 272-byte rows
    constexpr int SS = TK + 4;                                         // S row stride (floats)
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char* kbuf = smem;
    unsigned char* vbuf = smem + 2 * TK * RS;
    float* S = reinterpret_cast<float*>(smem + 4 * TK * RS);  // [NR][SS]
    float* m_run = S + NR * SS;
    float* l_run = m_run + NR;
    float* corr = l_run + NR;

    const uint32_t split = blockIdx.x, kvh = blockIdx.y;
    const uint64_t b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;  // mma fragment row group / thread in group
    const uint64_t len = seq_len_of(p, b);
    const uint64_t s0 = (uint64_t)split * p.split_len;
    const uint64_t s1 = s0 + p.split_len < len ? s0 + p.split_len : len;
    const uint32_t qh0 = kvh * NR;

    // Q fragments (rows g < NR), 8 k-steps of 16 dims: a0 = Q[g][16ks + 2t4 ..], a2 = Q[g][16ks + 8 + 2t4 ..]
    uint32_t qa0[8], qa2[8];
    {
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(q + (b * p.q_heads + qh0 + (g < NR ? g : 0)) * DA_D);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            qa0[ks] = g < NR ? qrow[ks * 8 + t4] : 0u;
            qa2[ks] = g < NR ? qrow[ks * 8 + 4 + t4] : 0u;
        }
    }
    if (tid < NR) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.0f;
    }
    float o[4][4];  // 4 n-tiles of 8 dims (dims warp*32 + nt*8 ..), fragment rows g / g + 8
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[nt][e] = 0.0f;

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
    __syncthreads();
    const uint32_t kbuf_s = (uint32_t)__cvta_generic_to_shared(kbuf);
    const uint32_t vbuf_s = (uint32_t)__cvta_generic_to_shared(vbuf);
    for (uint32_t t = 0; t < ntiles; ++t) {
        if (t + 1 < ntiles) issue(t + 1);
        else cp_async_commit();
        cp_async_wait<1>();
        const uint32_t stage = t & 1u;
        const uint32_t nk = nkeys - t * TK < (uint32_t)TK ? nkeys - t * TK : (uint32_t)TK;
        if (nk < (uint32_t)TK) {
            // rows past the last key hold stale bytes; P V multiplies them by p = 0, so
            // they must be finite: zero them
            for (uint32_t c = nk * CPR + tid; c < (uint32_t)TK * CPR; c += DA_THREADS) {
                const uint32_t row = c / CPR, col = c % CPR;
                *reinterpret_cast<uint4*>(vbuf + stage * TK * RS + row * RS + col * 16) = make_uint4(0, 0, 0, 0);
            }
        }
        __syncthreads();
        // S = Q K^T: warp w computes keys 16w .. 16w + 15 (two n-tiles)
        {
            float s0f[4] = {0.f, 0.f, 0.f, 0.f}, s1f[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t key = warp * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
            const uint32_t base = kbuf_s + stage * TK * RS + key * RS + ((lane >> 3) & 1) * 16;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                uint32_t b00, b01, b10, b11;
                ldsm_x4(base + ks * 32, b00, b01, b10, b11);
                mma_bf16(s0f, qa0[ks], qa2[ks], b00, b01);
                mma_bf16(s1f, qa0[ks], qa2[ks], b10, b11);
            }
            if (g < NR) {
                const uint32_t j0 = warp * 16 + 2 * t4;
                S[g * SS + j0] = j0 < nk ? fmul(s0f[0], p.scale) : -INFINITY;
                S[g * SS + j0 + 1] = j0 + 1 < nk ? fmul(s0f[1], p.scale) : -INFINITY;
                S[g * SS + j0 + 8] = j0 + 8 < nk ? fmul(s1f[0], p.scale) : -INFINITY;
                S[g * SS + j0 + 9] = j0 + 9 < nk ? fmul(s1f[1], p.scale) : -INFINITY;
            }
        }
        __syncthreads();
        for (int r = warp; r < NR; r += DA_THREADS / 32) {
            float* sr = S + r * SS;
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
        // O += P V: warp w owns dims 32w .. 32w + 31 (four n-tiles)
        {
            const float cg = g < NR ? corr[g] : 0.0f;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                o[nt][0] = fmul(o[nt][0], cg);
                o[nt][1] = fmul(o[nt][1], cg);
            }
            const uint32_t vkey = (lane & 7) + ((lane >> 3) & 1) * 8;   // key within the 16-key step
            const uint32_t vdim = warp * 32 + ((lane >> 4) & 1) * 8;     // first dim of the n-tile pair
#pragma unroll
            for (int ks = 0; ks < TK / 16; ++ks) {
                uint32_t ph0 = 0, ph2 = 0, pl0 = 0, pl2 = 0;
                if (g < NR) {
                    const float* pr = S + g * SS + ks * 16 + 2 * t4;
                    const float p0 = pr[0], p1 = pr[1], p8 = pr[8], p9 = pr[9];
                    const float h0 = round_bf16(p0), h1 = round_bf16(p1), h8 = round_bf16(p8), h9 = round_bf16(p9);
                    ph0 = pack_bf16x2(h0, h1);
                    ph2 = pack_bf16x2(h8, h9);
                    pl0 = pack_bf16x2(fsub(p0, h0), fsub(p1, h1));
                    pl2 = pack_bf16x2(fsub(p8, h8), fsub(p9, h9));
                }
#pragma unroll
                for (int np = 0; np < 2; ++np) {  // n-tile pairs (16 dims each)
                    uint32_t b00, b01, b10, b11;
                    ldsm_x4_trans(vbuf_s + stage * TK * RS + (ks * 16 + vkey) * RS + (vdim + np * 16) * 2, b00, b01,
                                  b10, b11);
                    mma_bf16(o[2 * np], ph0, ph2, b00, b01);
                    mma_bf16(o[2 * np], pl0, pl2, b00, b01);
                    mma_bf16(o[2 * np + 1], ph0, ph2, b10, b11);
                    mma_bf16(o[2 * np + 1], pl0, pl2, b10, b11);
                }
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    if (g < NR) {
        const uint64_t slot = (b * p.q_heads + qh0 + g) * p.splits + split;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const uint32_t d = warp * 32 + nt * 8 + 2 * t4;
            part_o[slot * DA_D + d] = o[nt][0];
            part_o[slot * DA_D + d + 1] = o[nt][1];
        }
        if (warp == 0 && t4 == 0) {
            part_ml[slot * 2] = m_run[g];
            part_ml[slot * 2 + 1] = l_run[g];
        }
    }
}

template <int NR>
constexpr size_t decode_mma_smem_bytes() {
    return (size_t)4 * DaTile<bf16_t>::TK * DaTile<bf16_t>::RS + (size_t)NR * (DaTile<bf16_t>::TK + 4) * 4 +
           (size_t)3 * NR * 4;
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
        auto kern = decode_attn_mma_kernel<NR>;
        const size_t smem = decode_mma_smem_bytes<NR>();
        if (!ensure_dyn_smem(reinterpret_cast<const void*>(kern), smem)) return cudaErrorInvalidConfiguration;
        kern<<<grid, DA_THREADS, smem, st>>>(q, kc, vc, part_ml, part_o, p);
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
