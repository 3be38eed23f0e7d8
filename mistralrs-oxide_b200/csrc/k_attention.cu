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
//      products on the tensor cores (decode_attn_warp_kernel); f32 caches:
//      the same warp streams with 8-key tiles on the CUDA cores
//      (decode_attn_warp_f32_kernel);
//   2. one CTA per (batch, q head) merges the splits:
//      M = max m_s, L = sum l_s e^(m_s - M), out = sum o_s e^(m_s - M) / L.
// Arithmetic is f32 accumulation (bf16 operands multiplied exactly), dot
// products and P.V with fused multiply-adds; the result differs from the
// reference's sequential f32 sums by rounding only.  head_dim 128 with rep in
// {1, 2, 4, 8} takes this path; other shapes take a one-CTA-per-(batch, head)
// kernel.  A sequence of length 0 yields zeros.
#include <atomic>
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

// Split lengths are whole multiples of one CTA's key granule: 4 warps x 16
// keys (bf16) or 4 warps x 8 keys (f32).
template <typename T>
constexpr uint64_t split_granule() { return sizeof(T) == 2 ? 64 : 32; }

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
    pdl_begin();
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
        // two accumulators (even / odd 16-dim steps) halve the dependent mma chain
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int ks = 0; ks < 8; ks += 2) {
            uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
            ldsm_x4(base + k_lane + ks * 32, a0, a1, a2, a3);
            ldsm_x4(base + k_lane + ks * 32 + 32, c0, c1, c2, c3);
            mma_bf16(s, a0, a1, a2, a3, qb0[ks], qb1[ks]);
            mma_bf16(s2, c0, c1, c2, c3, qb0[ks + 1], qb1[ks + 1]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) s[e] = fadd(s[e], s2[e]);
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

// ---- f32 caches: per-warp key streams on the CUDA cores ---------------------
// The split-K and warp-stream structure of the bf16 kernel, with 8-key tiles of
// f32 rows (512 B, padded to 528 B: conflict-free 16-byte reads) through a
// private 2-stage cp.async ring per warp (3 CTAs per SM).  Scores: lane l holds key l & 7 and
// dims 32 (l >> 3) .. + 31, reading the group's query heads from shared memory
// (a broadcast within each 8-lane phase), and the four dim quarters are summed
// by shuffles.  P V: lane l owns dims 4 l .. 4 l + 3 of every head's output,
// each key's probabilities broadcast from its lane by shuffle.  f32 throughout,
// expf for the exponentials, FMAs for the dot products and P V.
constexpr int DF_TK = 8;                                         // keys per warp tile
constexpr int DF_STAGES = 2;
constexpr int DF_RS = DA_D * 4 + 16;                             // 528-byte rows
constexpr int DF_RSF = DF_RS / 4;                                // the same in floats
constexpr int DF_STAGE = 2 * DF_TK * DF_RS;                      // 8448 B: K and V tile
constexpr size_t DF_RING = (size_t)DW_WARPS * DF_STAGES * DF_STAGE;  // 67,584 B
template <int NR>
constexpr size_t df_smem() {
    return DF_RING + (size_t)NR * DA_D * 4;  // + the group's query heads
}

template <int NR>
__global__ void __launch_bounds__(DW_WARPS * 32, 3)
    decode_attn_warp_f32_kernel(const float* q, const float* kc, const float* vc, float* part_ml, float* part_o,
                                DecArgs p) {
    pdl_begin();
    extern __shared__ __align__(16) unsigned char smem[];
    float* qs = reinterpret_cast<float*>(smem + DF_RING);  // [NR][D]
    const uint32_t split = blockIdx.x, kvh = blockIdx.y;
    const uint64_t b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kk = lane & 7, qq = lane >> 3;  // score pass: key in tile, dim quarter
    const uint64_t len = seq_len_of(p, b);
    const uint64_t s0 = (uint64_t)split * p.split_len;
    const uint64_t s1 = s0 + p.split_len < len ? s0 + p.split_len : len;
    const uint32_t nkeys = s1 > s0 ? (uint32_t)(s1 - s0) : 0u;
    const uint32_t ntiles = (nkeys + DF_TK - 1) / DF_TK;
    const uint32_t qh0 = kvh * NR;
    {
        const float4* qsrc = reinterpret_cast<const float4*>(q + (b * p.q_heads + qh0) * DA_D);
        for (int i = tid; i < NR * DA_D / 4; i += DW_WARPS * 32) reinterpret_cast<float4*>(qs)[i] = qsrc[i];
    }
    float acc[NR][4];
    float m[NR], l[NR];
#pragma unroll
    for (int h = 0; h < NR; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[h][c] = 0.0f;
    }
    unsigned char* wbuf = smem + (size_t)warp * DF_STAGES * DF_STAGE;
    const uint64_t row0 = (b * p.kv_heads + kvh) * p.max_seq + s0;
    const char* kbase = reinterpret_cast<const char*>(kc + row0 * DA_D);
    const char* vbase = reinterpret_cast<const char*>(vc + row0 * DA_D);
    const uint32_t my_tiles = ntiles > (uint32_t)warp ? (ntiles - warp + DW_WARPS - 1) / DW_WARPS : 0u;
    auto issue = [&](uint32_t it) {
        unsigned char* kd = wbuf + (it % DF_STAGES) * DF_STAGE;
        unsigned char* vd = kd + DF_TK * DF_RS;
        const uint32_t key0 = (warp + it * DW_WARPS) * DF_TK;
        const uint32_t nk = nkeys - key0 < (uint32_t)DF_TK ? nkeys - key0 : (uint32_t)DF_TK;
#pragma unroll
        for (int row = 0; row < DF_TK; ++row) {  // lane copies 16-byte column `lane` of each row
            // rows past the last key repeat the last key: finite data that p = 0 multiplies
            const uint32_t src = (uint32_t)row < nk ? (uint32_t)row : nk - 1;
            const uint64_t off = (uint64_t)(key0 + src) * (DA_D * 4) + lane * 16;
            cp_async16(kd + row * DF_RS + lane * 16, kbase + off);
            cp_async16(vd + row * DF_RS + lane * 16, vbase + off);
        }
    };
#pragma unroll
    for (int st = 0; st < DF_STAGES - 1; ++st) {
        if ((uint32_t)st < my_tiles) issue(st);
        cp_async_commit();
    }
    __syncthreads();  // the query heads are in shared memory
    for (uint32_t it = 0; it < my_tiles; ++it) {
        if (it + DF_STAGES - 1 < my_tiles) issue(it + DF_STAGES - 1);
        cp_async_commit();
        cp_async_wait<DF_STAGES - 1>();
        __syncwarp();  // every lane's copies of this tile are visible to the warp
        const float* kt = reinterpret_cast<const float*>(wbuf + (it % DF_STAGES) * DF_STAGE);
        const float* vt = kt + DF_TK * DF_RSF;
        const uint32_t key0 = (warp + it * DW_WARPS) * DF_TK;
        const uint32_t nk = nkeys - key0 < (uint32_t)DF_TK ? nkeys - key0 : (uint32_t)DF_TK;
        float dot[NR];
#pragma unroll
        for (int h = 0; h < NR; ++h) dot[h] = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float4 kv = *reinterpret_cast<const float4*>(kt + kk * DF_RSF + qq * 32 + c * 4);
#pragma unroll
            for (int h = 0; h < NR; ++h) {
                const float4 qv = *reinterpret_cast<const float4*>(qs + h * DA_D + qq * 32 + c * 4);
                dot[h] = __fmaf_rn(kv.x, qv.x, dot[h]);
                dot[h] = __fmaf_rn(kv.y, qv.y, dot[h]);
                dot[h] = __fmaf_rn(kv.z, qv.z, dot[h]);
                dot[h] = __fmaf_rn(kv.w, qv.w, dot[h]);
            }
        }
        bool rescale = false;
        float pr[NR], corr[NR];
#pragma unroll
        for (int h = 0; h < NR; ++h) {
            dot[h] = fadd(dot[h], __shfl_xor_sync(0xffffffffu, dot[h], 8));
            dot[h] = fadd(dot[h], __shfl_xor_sync(0xffffffffu, dot[h], 16));
            const float sc = (uint32_t)kk < nk ? fmul(dot[h], p.scale) : -INFINITY;
            float x = sc;
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
            const float mn = fmaxf(m[h], x);
            corr[h] = m[h] == -INFINITY ? 0.0f : expf(fsub(m[h], mn));
            rescale |= corr[h] != 1.0f;
            m[h] = mn;
            pr[h] = mn == -INFINITY ? 0.0f : expf(fsub(sc, mn));
            float ps = pr[h];
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) ps = fadd(ps, __shfl_xor_sync(0xffffffffu, ps, off));
            l[h] = __fmaf_rn(l[h], corr[h], ps);
        }
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
            for (int h = 0; h < NR; ++h)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[h][c] = fmul(acc[h][c], corr[h]);
        }
#pragma unroll
        for (int j = 0; j < DF_TK; ++j) {
            const float4 vv = *reinterpret_cast<const float4*>(vt + j * DF_RSF + lane * 4);
#pragma unroll
            for (int h = 0; h < NR; ++h) {
                const float pj = __shfl_sync(0xffffffffu, pr[h], j);  // lane j holds key j
                acc[h][0] = __fmaf_rn(pj, vv.x, acc[h][0]);
                acc[h][1] = __fmaf_rn(pj, vv.y, acc[h][1]);
                acc[h][2] = __fmaf_rn(pj, vv.z, acc[h][2]);
                acc[h][3] = __fmaf_rn(pj, vv.w, acc[h][3]);
            }
        }
        __syncwarp();  // the whole warp is done with this stage before it is refilled
    }
    cp_async_wait<0>();
    // merge the four warp states: [W][8] max, [W][8] sum, [W][NR][D] output
    __syncthreads();  // every warp is done with its ring: the buffers are reused
    float* wm = reinterpret_cast<float*>(smem);
    float* wl = wm + DW_WARPS * 8;
    float* wo = wl + DW_WARPS * 8;
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < NR; ++h) {
            wm[warp * 8 + h] = m[h];
            wl[warp * 8 + h] = l[h];
        }
    }
#pragma unroll
    for (int h = 0; h < NR; ++h)
        *reinterpret_cast<float4*>(wo + (warp * NR + h) * DA_D + lane * 4) =
            make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    __syncthreads();
    const int d = tid;
#pragma unroll
    for (int h = 0; h < NR; ++h) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < DW_WARPS; ++w) M = fmaxf(M, wm[w * 8 + h]);
        float L = 0.0f, o = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < DW_WARPS; ++w) {
                const float mw = wm[w * 8 + h];
                if (mw == -INFINITY) continue;
                const float sc = expf(fsub(mw, M));
                L = __fmaf_rn(wl[w * 8 + h], sc, L);
                o = __fmaf_rn(wo[(w * NR + h) * DA_D + d], sc, o);
            }
        }
        const uint64_t slot = (b * p.q_heads + qh0 + h) * p.splits + split;
        part_o[slot * DA_D + d] = o;
        if (d == 0) {
            part_ml[slot * 2] = M;
            part_ml[slot * 2 + 1] = L;
        }
    }
}

// Merge the splits of one (batch, q head); thread d writes out[d].  The
// splits' weights e^(m_s - M) and the sum L are found cooperatively (block
// reductions), the weights kept in shared memory, so the loop over the
// splits' outputs is a run of independent loads.
constexpr int DA_MAX_SPLITS = 1024;
template <typename T>
__global__ void __launch_bounds__(DA_THREADS)
    decode_attn_combine_kernel(const float* part_ml, const float* part_o, T* out, DecArgs p) {
    pdl_begin();
    __shared__ float wts[DA_MAX_SPLITS];
    __shared__ float red[32];
    const uint64_t bh = blockIdx.x;
    const int d = threadIdx.x;
    const uint64_t base = bh * p.splits;
    float M = -INFINITY;
    for (uint32_t s = d; s < p.splits; s += DA_THREADS) M = fmaxf(M, part_ml[(base + s) * 2]);
    M = group_reduce(M, red, DA_THREADS, OpMaxF());
    float lp = 0.0f;
    for (uint32_t s = d; s < p.splits; s += DA_THREADS) {
        const float ms = part_ml[(base + s) * 2];
        const float w = (M == -INFINITY || ms == -INFINITY) ? 0.0f : expf(fsub(ms, M));
        wts[s] = w;
        lp = __fmaf_rn(part_ml[(base + s) * 2 + 1], w, lp);
    }
    const float L = group_reduce(lp, red, DA_THREADS, OpAddF());  // its barrier also publishes wts
    float acc = 0.0f;
    const float* po = part_o + base * DA_D + d;
#pragma unroll 8
    for (uint32_t s = 0; s < p.splits; ++s) acc = __fmaf_rn(po[(uint64_t)s * DA_D], wts[s], acc);
    Vec<T>::store1(out + bh * DA_D + d, M == -INFINITY ? 0.0f : fdiv(acc, L));
}

// General shapes: one CTA per (batch, q head), three passes over the keys
// (scores into the workspace, max / sum, P.V); head_dim any, rep any.
template <typename T>
__global__ void __launch_bounds__(256)
    decode_attn_generic_kernel(const T* q, const T* kc, const T* vc, T* out, float* scores, DecArgs p) {
    pdl_begin();
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
        launch_k(kern, grid, DW_WARPS * 32, DW_SMEM, st, q, kc, vc, part_ml, part_o, p);
    } else {  // f32: CUDA-core tile products
        auto kern = decode_attn_warp_f32_kernel<NR>;
        const size_t smem = df_smem<NR>();
        if (!ensure_dyn_smem(reinterpret_cast<const void*>(kern), smem)) return cudaErrorInvalidConfiguration;
        launch_k(kern, grid, DW_WARPS * 32, smem, st, q, kc, vc, part_ml, part_o, p);
    }
    launch_k(decode_attn_combine_kernel<T>, (unsigned)(p.batch * p.q_heads), DA_THREADS, 0, st, part_ml, part_o, out, p);
    return cudaSuccess;
}

// The tcgen05 / TMA kernel of k_attention_tc.cu (bf16, head_dim 128); *used
// is false when the shapes or the device do not allow it.
cudaError_t decode_attention_tc_bf16(const bf16_t* q, const bf16_t* kc, const bf16_t* vc, const int32_t* lens,
                                     bf16_t* out, uint64_t batch, uint64_t q_heads, uint64_t kv_heads,
                                     uint64_t max_seq, float scale, void* ws, uint64_t ws_bytes, cudaStream_t st,
                                     bool withhold, bool* used);
int device_status(int reset, uint32_t* flags);
// 0: the tcgen05 kernel where it applies, else the split-K kernel; 1: always
// the split-K (mma.sync) kernel; 2: the tcgen05 kernel with its loads
// withheld (oxide_debug_decode_attention_path).
static std::atomic<int> g_decode_path{0};

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
    bool done = false;  // the tcgen05 kernel ran
    if constexpr (std::is_same<T, bf16_t>::value) {
        const int path = g_decode_path.load(std::memory_order_relaxed);
        if (fast && path != 1)
            e = decode_attention_tc_bf16(q, kc, vc, lens, out, batch, q_heads, kv_heads, max_seq, scale, ws, ws_bytes,
                                         st, path == 2, &done);
    }
    if (done) {
        // nothing more to launch
    } else if (fast) {
        // splits: enough CTAs for ~4 waves, whole tiles per split
        const uint64_t tk = split_granule<T>();
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
        launch_k(decode_attn_generic_kernel<T>, (unsigned)(batch * q_heads), 256, 0, st, q, kc, vc, out,
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

void oxide_debug_decode_attention_path(int path) {
    oxide::g_decode_path.store(path == 1 || path == 2 ? path : 0);
}

int oxide_device_status(int reset, uint32_t* flags) {
    OXIDE_INJECT("oxide_device_status");
    OXIDE_REQUIRE(flags, "oxide_device_status", "null flags pointer");
    return oxide::device_status(reset, flags);
}

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
