// k_attention_tc.cu -- one-token (decode) attention over bf16 KV caches on the
// 5th-generation tensor cores: TMA tile loads into an mbarrier ring, tcgen05
// matrix products into tensor memory, warp-specialised.
//
// Reference: the inline attention of scaled_dot_product_attention
// (src/ops/attention.rs:41-87) for q_len = 1 -- s_j = (q . k_j) * scale,
// softmax over the keys j < lens[b], out = sum_j p_j v_j -- with query head h
// reading kv head h / rep (repeat_kv's map, attention.rs:161-201, not
// materialised).  Numerics match the split-K kernel of k_attention.cu: exact
// bf16 products accumulated in f32, base-2 online softmax with ex2.approx, P
// entering the P.V product as two bf16 halves (16 significant bits), the
// split partials merged in f32.
//
// Work division: the (batch, kv head) pairs' 128-key tiles are laid end to
// end (pair order batch-major; a batch with L valid keys has ceil(L / 128)
// tiles per kv head) and CTA c of G (one per SM) takes tiles
// [c T / G, (c + 1) T / G): every CTA streams the same number of tiles
// (+-1) whatever the lengths.  A CTA writes one partial (max, sum, o[128]) per
// pair it touches, in the slot of its first tile's offset within the pair;
// the combine kernel recomputes the same division to find each pair's
// occupied slots.
//
// CTA of 6 warps:
//   warp 0   (one lane) TMA producer: K and V tiles [128 keys x 64 dims] x 2
//            halves, 128-byte swizzled, into a 3-stage ring; the group's
//            query heads (16 rows: the rep heads, the rest unused) per pair;
//   warp 1   TMEM owner and (one lane) MMA issuer:
//              S^T[128 keys x 16]  = K . Q^T    (A = K, K-major; B = Q, K-major)
//              O^T[128 dims x 16]  = V^T . P^T  (A = V read MN-major; B = P^T)
//            S is issued one tile ahead of the softmax, S and O double-buffered
//            in TMEM (64 columns);
//   warps 2-5 softmax and epilogue, thread i = key i of the S tile and dim i
//            of the O tile (its TMEM lane): per-tile maximum over the 128 keys
//            (shuffles + one named barrier), p = 2^(t - m), P^T written to
//            shared memory as bf16 hi / lo halves in columns [0, rep) and
//            [rep, 2 rep) of the 16, the output accumulated in registers with
//            the online-softmax rescale.
// Every wait is bounded (oxide_tc.cuh): a wait that runs out raises the CTA's
// abort flag, all roles stop issuing, in-flight copies and products are
// waited for, TMEM is freed and the error word in the workspace is set, which
// makes the combine kernel write NaN.
#include "oxide_tc.cuh"

namespace oxide {

constexpr int TC_D = 128;    // head_dim
constexpr int TC_TK = 128;   // keys per tile
constexpr int TC_STAGES = 3;
constexpr int TC_N = 16;     // MMA N: 2 x rep columns used (rep <= 8)
constexpr int TC_THREADS = 192;
constexpr int TC_MAX_BATCH = 1024;
constexpr int TC_MAX_TILES = 1024;  // tiles per sequence: max_seq <= 131,072
constexpr uint32_t TC_TMEM_COLS = 64;                  // S[2] x 16, O[2] x 16
constexpr uint32_t TC_HALF = TC_TK * 128;              // 16 KB: 128 rows x 128 B
constexpr uint32_t TC_STAGE_BYTES = 4 * TC_HALF;       // K lo, K hi, V lo, V hi
constexpr uint32_t TC_QHALF = TC_N * 128;              // 2 KB: 16 rows x 128 B
constexpr uint32_t TC_Q_BYTES = 2 * TC_QHALF;
constexpr uint32_t TC_P_BYTES = TC_N * TC_TK * 2;      // 4 KB: P^T, bf16
// shared memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t TC_OFF_STAGE = 0;
constexpr uint32_t TC_OFF_Q = TC_OFF_STAGE + TC_STAGES * TC_STAGE_BYTES;  // 196,608
constexpr uint32_t TC_OFF_P = TC_OFF_Q + 2 * TC_Q_BYTES;                  // 204,800
constexpr uint32_t TC_OFF_PRE = TC_OFF_P + 2 * TC_P_BYTES;                // 212,992
constexpr uint32_t TC_OFF_BAR = TC_OFF_PRE + (TC_MAX_BATCH + 8) * 4;      // 217,120
constexpr int TC_NBAR = 24;
constexpr uint32_t TC_OFF_MISC = TC_OFF_BAR + TC_NBAR * 8;                // 217,312
constexpr uint32_t TC_MISC_BYTES = 16 + 64 * 4 + 32 * 4 + 32;
constexpr size_t TC_SMEM = TC_OFF_MISC + TC_MISC_BYTES + 1024;            // + alignment slack
static_assert(TC_SMEM <= 227 * 1024, "shared memory of one CTA");
// barrier indices
enum : int {
    B_FULL = 0,                    // [3] stage loaded (TMA transaction bytes)
    B_EMPTY = B_FULL + TC_STAGES,  // [3] stage consumed (MMA commit)
    B_QFULL = B_EMPTY + TC_STAGES, // [2]
    B_QEMPTY = B_QFULL + 2,        // [2]
    B_SFULL = B_QEMPTY + 2,        // [2] scores in TMEM (MMA commit)
    B_SEMPTY = B_SFULL + 2,        // [2] scores read (4 softmax warps)
    B_PFULL = B_SEMPTY + 2,        // [2] P^T in shared memory (1 softmax thread)
    B_PEMPTY = B_PFULL + 2,        // [2] P^T read (MMA commit)
    B_OFULL = B_PEMPTY + 2,        // [2] tile output in TMEM (MMA commit)
    B_OEMPTY = B_OFULL + 2,        // [2] tile output read (4 softmax warps)
    B_DONE = B_OEMPTY + 2,         // every product issued has completed
    B_COUNT = B_DONE + 1
};
static_assert(B_COUNT <= TC_NBAR, "barrier slots");

struct TcArgs {
    uint64_t batch, max_seq;
    uint32_t q_heads, kv_heads, stride;  // stride: split slots per (batch, q head)
    float c1;                            // scale * log2(e)
    const int32_t* lens;
    float* part_ml;
    float* part_o;
    uint32_t* err;
    uint32_t* pre_out;  // [batch + 1]: tiles per kv head before each batch, written by CTA 0 for the combine
    uint32_t withhold;  // failure-detection tests: the producer issues no loads, so every wait runs out
};

// Sticky device-side failure flags of this library on each device (bit 0:
// a bounded wait in the tcgen05 decode-attention kernel ran out), read and
// cleared by oxide_device_status.
__device__ unsigned int g_device_status;

__device__ __forceinline__ uint32_t tc_len(const TcArgs& p, uint64_t b) {
    if (!p.lens) return (uint32_t)p.max_seq;
    const int32_t l = p.lens[b];
    return l <= 0 ? 0u : ((uint64_t)l < p.max_seq ? (uint32_t)l : (uint32_t)p.max_seq);
}

// Walks the flattened tile space in order: pair (b, kvh), tile lt of tb.
struct TileWalk {
    const uint32_t* pre;  // pre[b] = tiles per kv head of batches < b; pre[B] = total
    uint32_t nb, hkv;
    uint32_t b, kvh, lt, tb;
    __device__ void seek(uint32_t t) {
        // the batch holding global tile t: pre[b] * hkv <= t < pre[b + 1] * hkv
        uint32_t lo = 0, hi = nb;
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (pre[mid] * hkv <= t) lo = mid;
            else hi = mid;
        }
        b = lo;
        while (b + 1 < nb && pre[b + 1] * hkv <= t) ++b;  // skip batches without tiles
        tb = pre[b + 1] - pre[b];
        const uint32_t r = t - pre[b] * hkv;
        kvh = tb ? r / tb : 0;
        lt = tb ? r % tb : 0;
    }
    __device__ void next() {
        if (++lt < tb) return;
        lt = 0;
        if (++kvh < hkv) return;
        kvh = 0;
        do {
            ++b;
            tb = b < nb ? pre[b + 1] - pre[b] : 0;
        } while (b < nb && tb == 0);
    }
};

// The CTA (of G) whose tile range holds global tile t: the largest c with
// floor(c T / G) <= t.
__device__ __forceinline__ uint32_t tc_owner(uint32_t t, uint32_t T, uint32_t G) {
    return (uint32_t)((((uint64_t)t + 1) * G - 1) / T);
}

template <int NR>
__global__ void __launch_bounds__(TC_THREADS, 1)
    decode_attn_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                          const __grid_constant__ CUtensorMap tmq, TcArgs p) {
    // Set-up that touches no global memory (barriers, TMEM, the tensor maps'
    // descriptors) overlaps the previous kernel; the wait comes before the
    // first global access.
    pdl_trigger();
    static_assert(NR == 1 || NR == 2 || NR == 4 || NR == 8, "rep in {1, 2, 4, 8}");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* pre = reinterpret_cast<uint32_t*>(smem + TC_OFF_PRE);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TC_OFF_MISC);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + TC_OFF_MISC + 4);
    volatile int* consumed = reinterpret_cast<volatile int*>(smem + TC_OFF_MISC + 8);   // stages the MMA warp waited for
    volatile int* qconsumed = reinterpret_cast<volatile int*>(smem + TC_OFF_MISC + 12); // query loads it waited for
    float* red = reinterpret_cast<float*>(smem + TC_OFF_MISC + 16);    // [2][4][8] tile maxima
    float* lsum = red + 64;                                            // [4][8] row sums
    auto bar = [&](int i) { return sbase + TC_OFF_BAR + 8u * (uint32_t)i; };
    const uint32_t nb = (uint32_t)p.batch, hkv = p.kv_heads;

    if (tid == 0) {
        *abort = 0;
        *consumed = 0;
        *qconsumed = 0;
        for (int i = 0; i < TC_STAGES; ++i) {
            mbar_init(bar(B_FULL + i), 1);
            mbar_init(bar(B_EMPTY + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(B_QFULL + i), 1);
            mbar_init(bar(B_QEMPTY + i), 1);
            mbar_init(bar(B_SFULL + i), 1);
            mbar_init(bar(B_SEMPTY + i), 4);
            mbar_init(bar(B_PFULL + i), 1);
            mbar_init(bar(B_PEMPTY + i), 1);
            mbar_init(bar(B_OFULL + i), 1);
            mbar_init(bar(B_OEMPTY + i), 4);
        }
        mbar_init(bar(B_DONE), 1);
        mbar_init_fence();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&tmk);
        tma_prefetch_map(&tmv);
        tma_prefetch_map(&tmq);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TC_TMEM_COLS);
        tmem_relinquish();
    }
    pdl_wait();  // the previous kernel's writes (lengths, caches, queries) are visible
    if (warp == 2) {  // tiles per kv head of each batch, and their prefix sums
        uint32_t carry = 0;
        for (uint32_t b0 = 0; b0 < nb; b0 += 32) {
            const uint32_t b = b0 + lane;
            uint32_t v = b < nb ? (tc_len(p, b) + TC_TK - 1) / TC_TK : 0u;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {  // inclusive scan over the warp
                const uint32_t u = __shfl_up_sync(0xffffffffu, v, off);
                if (lane >= off) v += u;
            }
            const uint32_t incl = carry + v;
            if (b < nb) pre[b + 1] = incl;
            carry = __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) pre[0] = 0;
        if (blockIdx.x == 0) {
            __syncwarp();
            for (uint32_t i = lane; i <= nb; i += 32) p.pre_out[i] = pre[i];
        }
    }
    if (tid == 0 && blockIdx.x == 0) *p.err = 0u;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t T = pre[nb] * hkv, G = gridDim.x;
    const uint32_t t0 = (uint32_t)((uint64_t)blockIdx.x * T / G);
    const uint32_t t1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * T / G);
    TileWalk w{pre, nb, hkv, 0, 0, 0, 0};

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        uint32_t n = 0, q = 0;
        if (lane == 0 && t0 < t1 && !p.withhold) {
            w.seek(t0);
            for (uint32_t t = t0; t < t1 && !*abort; ++t, w.next()) {
                if (t == t0 || w.lt == 0) {  // first tile of a pair in this CTA: its query heads
                    const uint32_t qs = q & 1u;
                    if (!tc_wait(bar(B_QEMPTY + qs), ((q >> 1) & 1u) ^ 1u, abort)) break;
                    mbar_arrive_expect_tx(bar(B_QFULL + qs), TC_Q_BYTES);
                    const int row = (int)(w.b * p.q_heads + w.kvh * NR);
                    const uint32_t qd = sbase + TC_OFF_Q + qs * TC_Q_BYTES;
                    tma_load_2d(qd, &tmq, bar(B_QFULL + qs), 0, row);
                    tma_load_2d(qd + TC_QHALF, &tmq, bar(B_QFULL + qs), 64, row);
                    ++q;
                }
                const uint32_t s = n % TC_STAGES;
                if (!tc_wait(bar(B_EMPTY + s), ((n / TC_STAGES) & 1u) ^ 1u, abort)) break;
                mbar_arrive_expect_tx(bar(B_FULL + s), TC_STAGE_BYTES);
                const int y = (int)(((uint64_t)w.b * hkv + w.kvh) * p.max_seq + (uint64_t)w.lt * TC_TK);
                const uint32_t sd = sbase + TC_OFF_STAGE + s * TC_STAGE_BYTES;
                tma_load_2d(sd, &tmk, bar(B_FULL + s), 0, y);
                tma_load_2d(sd + TC_HALF, &tmk, bar(B_FULL + s), 64, y);
                tma_load_2d(sd + 2 * TC_HALF, &tmv, bar(B_FULL + s), 0, y);
                tma_load_2d(sd + 3 * TC_HALF, &tmv, bar(B_FULL + s), 64, y);
                ++n;
            }
        }
        // Drain (after an abort): copies issued but never waited for by the
        // MMA warp land before the CTA exits.
        if (lane == 0 && *abort) {
            for (uint32_t i = (uint32_t)*consumed; i < n; ++i)
                tc_wait_drain(bar(B_FULL + i % TC_STAGES), (i / TC_STAGES) & 1u);
            for (uint32_t i = (uint32_t)*qconsumed; i < q; ++i) tc_wait_drain(bar(B_QFULL + (i & 1u)), (i >> 1) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && t0 < t1) {
            constexpr uint32_t IDESC_S = umma_idesc_bf16(128, TC_N, false, false);
            constexpr uint32_t IDESC_O = umma_idesc_bf16(128, TC_N, true, false);
            TileWalk ws = w;  // the S (first) product runs one tile ahead of the O product
            ws.seek(t0);
            uint32_t q = 0;
            // S product of tile n into S buffer n & 1
            auto issue_s = [&](uint32_t n, uint32_t t) -> bool {
                if (t == t0 || ws.lt == 0) {
                    if (!tc_wait(bar(B_QFULL + (q & 1u)), (q >> 1) & 1u, abort)) return false;
                    *qconsumed = (int)q + 1;
                }
                const uint32_t s = n % TC_STAGES, sb = n & 1u;
                if (!tc_wait(bar(B_FULL + s), (n / TC_STAGES) & 1u, abort)) return false;
                *consumed = (int)n + 1;
                if (!tc_wait(bar(B_SEMPTY + sb), ((n >> 1) & 1u) ^ 1u, abort)) return false;
                tc_fence_after();
                const uint32_t kaddr = sbase + TC_OFF_STAGE + s * TC_STAGE_BYTES;
                const uint32_t qaddr = sbase + TC_OFF_Q + (q & 1u) * TC_Q_BYTES;
#pragma unroll
                for (int kk = 0; kk < TC_D / 16; ++kk) {
                    const uint32_t koff = (uint32_t)(kk >> 2) * TC_HALF + (uint32_t)(kk & 3) * 32;
                    const uint32_t qoff = (uint32_t)(kk >> 2) * TC_QHALF + (uint32_t)(kk & 3) * 32;
                    umma_bf16(tmem + sb * TC_N, umma_desc(kaddr + koff, 16, 1024, UMMA_SWIZZLE_128B),
                              umma_desc(qaddr + qoff, 16, 1024, UMMA_SWIZZLE_128B), IDESC_S, kk > 0);
                }
                umma_commit(bar(B_SFULL + sb));
                const bool last = (t + 1 == t1) || (ws.lt + 1 == ws.tb);
                if (last) {  // this pair's last product that reads its query heads
                    umma_commit(bar(B_QEMPTY + (q & 1u)));
                    ++q;
                }
                return true;
            };
            bool ok = issue_s(0, t0);
            ws.next();
            for (uint32_t n = 0, t = t0; ok && t < t1; ++n, ++t) {
                if (t + 1 < t1) {
                    ok = issue_s(n + 1, t + 1);
                    ws.next();
                    if (!ok) break;
                }
                // O product of tile n: needs its P^T and a free O buffer
                const uint32_t s = n % TC_STAGES, sb = n & 1u;
                if (!tc_wait(bar(B_PFULL + sb), (n >> 1) & 1u, abort)) break;
                if (!tc_wait(bar(B_OEMPTY + sb), ((n >> 1) & 1u) ^ 1u, abort)) break;
                tc_fence_after();
                const uint32_t vaddr = sbase + TC_OFF_STAGE + s * TC_STAGE_BYTES + 2 * TC_HALF;
                const uint32_t paddr = sbase + TC_OFF_P + sb * TC_P_BYTES;
#pragma unroll
                for (int kk = 0; kk < TC_TK / 16; ++kk) {
                    umma_bf16(tmem + 2 * TC_N + sb * TC_N,
                              umma_desc(vaddr + (uint32_t)kk * 2048, TC_HALF, 1024, UMMA_SWIZZLE_128B),
                              umma_desc(paddr + (uint32_t)kk * 256, 128, 2048, UMMA_SWIZZLE_NONE), IDESC_O, kk > 0);
                }
                umma_commit(bar(B_OFULL + sb));
                umma_commit(bar(B_EMPTY + s));
                umma_commit(bar(B_PEMPTY + sb));
            }
        }
        if (lane == 0) {  // every product issued above has completed before TMEM is freed
            umma_commit(bar(B_DONE));
            if (!tc_wait_drain(bar(B_DONE), 0)) *abort = 1;
        }
        __syncwarp();
    } else {
        // ---------------- softmax and epilogue (warps 2-5) ----------------
        const uint32_t q4 = (uint32_t)(warp & 3);  // this warp's TMEM lane quarter
        const uint32_t L = q4 * 32 + (uint32_t)lane;  // key of the S tile, dim of the O tile
        const uint32_t lane_tmem = tmem + ((q4 * 32u) << 16);
        const float LN2 = 0.6931471805599453f;
        // per tile parity (0 / 1): kept in registers, picked by selects
        float m[NR], l[NR], acc[NR], corr0[NR], corr1[NR], mf0[NR], mf1[NR], lf0[NR], lf1[NR];
#pragma unroll
        for (int h = 0; h < NR; ++h) {
            m[h] = -INFINITY;
            l[h] = 0.0f;
            acc[h] = 0.0f;
            mf0[h] = mf1[h] = -INFINITY;
            lf0[h] = lf1[h] = 0.0f;
            corr0[h] = corr1[h] = 0.0f;
        }
        bool fail = false;
        // The O tile of the previous iteration is read after this tile's
        // softmax (its product runs meanwhile); its pair if it was the last.
        struct Pend {
            bool on, last;
            uint32_t n, b, kvh, tb;
        } pend{false, false, 0, 0, 0, 0};
        auto epilogue = [&](const Pend& e) {
            const uint32_t sb = e.n & 1u;
            const bool ok = warp_wait(bar(B_OFULL + sb), (e.n >> 1) & 1u, abort);
            fail |= !ok;
            if (ok) {
                tc_fence_after();
                uint32_t o[16];
                tmem_ld16(lane_tmem + 2 * TC_N + sb * TC_N, o);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_OEMPTY + sb));
#pragma unroll
                for (int h = 0; h < NR; ++h)
                    acc[h] = __fmaf_rn(acc[h], sb ? corr1[h] : corr0[h],
                                       fadd(__uint_as_float(o[h]), __uint_as_float(o[NR + h])));
            }
            if (!e.last) return;
            // the pair is complete: row sums over the 128 threads, then the partial
#pragma unroll
            for (int h = 0; h < NR; ++h) {
                float x = sb ? lf1[h] : lf0[h];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) x = fadd(x, __shfl_xor_sync(0xffffffffu, x, off));
                if (lane == 0) lsum[q4 * 8 + h] = x;
            }
            nbar_sync128();
            if (!fail) {
                // slot: the offset, within the pair, of this CTA's first tile of it
                const uint32_t tfirst = pre[e.b] * hkv + e.kvh * e.tb;
                const uint32_t split = t0 > tfirst ? t0 - tfirst : 0u;
#pragma unroll
                for (int h = 0; h < NR; ++h) {
                    const uint64_t slot = ((uint64_t)e.b * p.q_heads + e.kvh * NR + h) * p.stride + split;
                    p.part_o[slot * TC_D + L] = acc[h];
                    if (L == 0) {
                        const float ls = fadd(fadd(lsum[h], lsum[8 + h]), fadd(lsum[16 + h], lsum[24 + h]));
                        const float mfh = sb ? mf1[h] : mf0[h];
                        p.part_ml[slot * 2] = mfh == -INFINITY ? -INFINITY : fmul(mfh, LN2);
                        p.part_ml[slot * 2 + 1] = ls;
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < NR; ++h) acc[h] = 0.0f;
            nbar_sync128();  // lsum is read before it is written again
        };

        uint32_t n = 0;
        if (t0 < t1) w.seek(t0);
        for (uint32_t t = t0; t < t1; ++t, ++n, w.next()) {
            const uint32_t sb = n & 1u, s = n % TC_STAGES;
            const bool first = (t == t0) || (w.lt == 0);
            const bool last = (t + 1 == t1) || (w.lt + 1 == w.tb);
            const uint32_t len = tc_len(p, w.b), key0 = w.lt * TC_TK;
            const uint32_t valid = len - key0 < (uint32_t)TC_TK ? len - key0 : (uint32_t)TC_TK;
            if (first) {
#pragma unroll
                for (int h = 0; h < NR; ++h) {
                    m[h] = -INFINITY;
                    l[h] = 0.0f;
                }
            }
            // scores of this tile (key L), in the base-2 domain
            float tt[NR];
            bool ok = warp_wait(bar(B_SFULL + sb), (n >> 1) & 1u, abort);
            fail |= !ok;
            if (ok) {
                tc_fence_after();
                uint32_t v[16];
                tmem_ld16(lane_tmem + sb * TC_N, v);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_SEMPTY + sb));
#pragma unroll
                for (int h = 0; h < NR; ++h) tt[h] = L < valid ? fmul(__uint_as_float(v[h]), p.c1) : -INFINITY;
            } else {
#pragma unroll
                for (int h = 0; h < NR; ++h) tt[h] = -INFINITY;
            }
#pragma unroll
            for (int h = 0; h < NR; ++h) {
                float x = tt[h];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
                if (lane == 0) red[(sb * 4 + q4) * 8 + h] = x;
            }
            // this P^T buffer is free once the product of tile n - 2 has read it
            ok = warp_wait(bar(B_PEMPTY + sb), ((n >> 1) & 1u) ^ 1u, abort);
            fail |= !ok;
            nbar_sync128();  // the four warps' tile maxima are in red[sb]
            unsigned char* pt = smem + TC_OFF_P + sb * TC_P_BYTES;
#pragma unroll
            for (int h = 0; h < NR; ++h) {
                const float* r = red + sb * 32 + h;
                const float mt = fmaxf(fmaxf(r[0], r[8]), fmaxf(r[16], r[24]));
                const float mn = fmaxf(m[h], mt);
                const float cr = m[h] == -INFINITY ? 0.0f : ex2_approx(fsub(m[h], mn));
                if (sb) corr1[h] = cr;
                else corr0[h] = cr;
                m[h] = mn;
                const float pr = mn == -INFINITY ? 0.0f : ex2_approx(fsub(tt[h], mn));
                l[h] = __fmaf_rn(l[h], cr, pr);
                const float hi = round_bf16(pr);
                // P^T[col][key L], K-major without swizzle: 8 x 16-byte core rows
                const uint32_t kof = (L >> 3) * 128 + (L & 7) * 2;
                const int chi = h, clo = NR + h;
                *reinterpret_cast<bf16_t*>(pt + (chi >> 3) * 2048 + kof + (chi & 7) * 16) = f32_to_bf16(hi);
                *reinterpret_cast<bf16_t*>(pt + (clo >> 3) * 2048 + kof + (clo & 7) * 16) = f32_to_bf16(fsub(pr, hi));
            }
            if (last) {
#pragma unroll
                for (int h = 0; h < NR; ++h) {
                    if (sb) {
                        mf1[h] = m[h];
                        lf1[h] = l[h];
                    } else {
                        mf0[h] = m[h];
                        lf0[h] = l[h];
                    }
                }
            }
            if (valid < (uint32_t)TC_TK && L >= valid) {
                // keys past the sequence: zero their V rows (a 128-byte row of
                // each swizzled half), so 0 * whatever the cache holds there
                // cannot turn into NaN in the product
                uint4* v0 = reinterpret_cast<uint4*>(smem + TC_OFF_STAGE + s * TC_STAGE_BYTES + 2 * TC_HALF + L * 128);
                uint4* v1 = reinterpret_cast<uint4*>(smem + TC_OFF_STAGE + s * TC_STAGE_BYTES + 3 * TC_HALF + L * 128);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v0[i] = make_uint4(0u, 0u, 0u, 0u);
                    v1[i] = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_async_smem();  // P^T (and zeroed V rows) visible to the tensor core
            if (nbar_or128(fail)) {
                fail = true;
                break;
            }
            if (tid == 64) mbar_arrive(bar(B_PFULL + sb));  // after the barrier: every thread has written P^T
            if (pend.on) epilogue(pend);
            pend = Pend{true, last, n, w.b, w.kvh, w.tb};
        }
        if (pend.on) {  // uniform: the loop ran to its end (or stopped at a uniform decision)
            if (!nbar_or128(fail)) epilogue(pend);
            else fail = true;
        }
        if (fail) *abort = 1;
    }
    // ---------------- teardown ----------------
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TC_TMEM_COLS);
    if (tid == 0 && *abort) {
        atomicOr(p.err, 1u);
        atomicOr(&g_device_status, OXIDE_DEVICE_WAIT_TIMEOUT);
    }
}

// Merge the split partials of one (batch, q head): the same tile division as
// the main kernel (from the tile prefix it wrote) gives the CTAs that took part
// of the pair -- enumerated in parallel, one thread per candidate -- and the
// slot of each (its first tile's offset within the pair).  out = sum_s o_s
// e^(m_s - M) / sum_s l_s e^(m_s - M), merged online over chunks of slots
// whose loads are all issued first; a pair without keys gives zeros; NaN
// everywhere if the main kernel reported an abort.  Two dependent memory
// round trips in all (the prefix, then the partials).
constexpr int TC_MAX_PARTS = 1024;  // CTAs sharing one pair: at most the grid size
constexpr uint32_t TC_NOSLOT = 0xFFFFFFFFu;
template <int NR>
__global__ void __launch_bounds__(128)
    decode_attn_tc_combine_kernel(bf16_t* out, TcArgs p, uint32_t G) {
    pdl_begin();
    __shared__ uint32_t slot[TC_MAX_PARTS];
    const uint64_t bh = blockIdx.x, b = bh / p.q_heads;
    const uint32_t h = (uint32_t)(bh % p.q_heads), kvh = h / NR;
    const int d = threadIdx.x;
    const uint32_t before = p.pre_out[b], tb = p.pre_out[b + 1] - before;
    const uint32_t T = p.pre_out[p.batch] * p.kv_heads;
    const uint32_t failed = *p.err;
    uint32_t nspan = 0;
    if (tb) {
        const uint32_t tfirst = before * p.kv_heads + kvh * tb, tlast = tfirst + tb - 1;
        const uint32_t c0 = tc_owner(tfirst, T, G);
        nspan = min(tc_owner(tlast, T, G) - c0 + 1, (uint32_t)TC_MAX_PARTS);
        for (uint32_t i = (uint32_t)d; i < nspan; i += 128) {
            const uint32_t c = c0 + i;
            const uint32_t f0 = (uint32_t)((uint64_t)c * T / G), f1 = (uint32_t)((uint64_t)(c + 1) * T / G);
            slot[i] = f0 < f1 ? (f0 > tfirst ? f0 : tfirst) - tfirst : TC_NOSLOT;
        }
    }
    __syncthreads();
    const uint64_t base = bh * p.stride;
    float M = -INFINITY, L = 0.0f, acc = 0.0f;
    constexpr int CH = 8;
    for (uint32_t i0 = 0; i0 < nspan; i0 += CH) {
        float ms[CH], ls[CH], os[CH];
#pragma unroll
        for (int k = 0; k < CH; ++k) {
            const uint32_t sk = i0 + k < nspan ? slot[i0 + k] : TC_NOSLOT;
            ms[k] = -INFINITY;
            ls[k] = 0.0f;
            os[k] = 0.0f;
            if (sk != TC_NOSLOT) {
                const uint64_t sl = base + sk;
                ms[k] = p.part_ml[sl * 2];
                ls[k] = p.part_ml[sl * 2 + 1];
                os[k] = p.part_o[sl * TC_D + d];
            }
        }
#pragma unroll
        for (int k = 0; k < CH; ++k) {
            if (ms[k] == -INFINITY) continue;  // no slot, or a CTA part without valid keys
            if (ms[k] > M) {
                const float w = M == -INFINITY ? 0.0f : expf(fsub(M, ms[k]));
                L = __fmaf_rn(L, w, ls[k]);
                acc = __fmaf_rn(acc, w, os[k]);
                M = ms[k];
            } else {
                const float w = expf(fsub(ms[k], M));
                L = __fmaf_rn(ls[k], w, L);
                acc = __fmaf_rn(os[k], w, acc);
            }
        }
    }
    float r = M == -INFINITY ? 0.0f : fdiv(acc, L);
    if (failed) r = __uint_as_float(0x7fc00000u);
    Vec<bf16_t>::store1(out + bh * TC_D + d, r);
}

typedef CUresult (*TensorMapEncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                           const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                           CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                           CUtensorMapFloatOOBfill);

// A [rows, 128] bf16 matrix as a TMA map with boxes of [box_rows, 64]
// (128 bytes, 128-byte swizzle); false if the driver refuses it.
static bool tc_map(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows) {
    static TensorMapEncodeTiledFn enc =
        reinterpret_cast<TensorMapEncodeTiledFn>(driver_fn("cuTensorMapEncodeTiled"));
    if (!enc) return false;
    const cuuint64_t dims[2] = {TC_D, rows};
    const cuuint64_t strides[1] = {TC_D * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool tc_enabled() {
    static const bool on = [] {
        const char* v = getenv("OXIDE_NO_TCGEN05");
        if (v && v[0] == '1') return false;
        int dev = 0, major = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        return major == 10;
    }();
    return on;
}

template <int NR>
static cudaError_t tc_launch(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq, bf16_t* out,
                             const TcArgs& a, uint32_t G, cudaStream_t st) {
    auto kern = decode_attn_tc_kernel<NR>;
    if (!ensure_dyn_smem(reinterpret_cast<const void*>(kern), TC_SMEM)) return cudaErrorInvalidConfiguration;
    cudaError_t e = launch_k(kern, G, TC_THREADS, TC_SMEM, st, mk, mv, mq, a);
    if (e != cudaSuccess) return e;
    return launch_k(decode_attn_tc_combine_kernel<NR>, (unsigned)(a.batch * a.q_heads), 128, 0, st, out, a, G);
}

// Decode attention on the tcgen05 path when the shapes allow it; *used says
// whether it ran (otherwise the caller takes the split-K mma.sync kernel).
cudaError_t decode_attention_tc_bf16(const bf16_t* q, const bf16_t* kc, const bf16_t* vc, const int32_t* lens,
                                     bf16_t* out, uint64_t batch, uint64_t q_heads, uint64_t kv_heads,
                                     uint64_t max_seq, float scale, void* ws, uint64_t ws_bytes, cudaStream_t st,
                                     bool withhold, bool* used) {
    *used = false;
    const uint64_t rep = q_heads / kv_heads;
    if (!tc_enabled() || batch > (uint64_t)TC_MAX_BATCH || max_seq < 256 ||
        batch * kv_heads * max_seq >= (1ull << 31) || batch * q_heads >= (1ull << 31) ||
        !(rep == 1 || rep == 2 || rep == 4 || rep == 8))
        return cudaSuccess;
    const uint32_t G = (uint32_t)sm_count();
    if (G > (uint32_t)TC_MAX_PARTS) return cudaSuccess;
    const uint64_t tiles_max = (max_seq + TC_TK - 1) / TC_TK;
    if (tiles_max > (uint64_t)TC_MAX_TILES) return cudaSuccess;
    const uint32_t stride = (uint32_t)tiles_max;  // a partial slot per tile offset of a sequence
    const uint64_t need = (uint64_t)batch * q_heads * stride * (2 + TC_D) * sizeof(float) + 16 + (batch + 1) * 4;
    if (ws_bytes < need) return cudaSuccess;
    CUtensorMap mk, mv, mq;
    if (!tc_map(&mk, kc, batch * kv_heads * max_seq, TC_TK) || !tc_map(&mv, vc, batch * kv_heads * max_seq, TC_TK) ||
        !tc_map(&mq, q, batch * q_heads, TC_N))
        return cudaSuccess;
    TcArgs a{};
    a.batch = batch;
    a.max_seq = max_seq;
    a.q_heads = (uint32_t)q_heads;
    a.kv_heads = (uint32_t)kv_heads;
    a.stride = stride;
    a.c1 = scale * 1.4426950408889634f;
    a.lens = lens;
    a.part_ml = static_cast<float*>(ws);
    a.part_o = a.part_ml + (size_t)2 * batch * q_heads * stride;
    a.err = reinterpret_cast<uint32_t*>(a.part_o + (size_t)batch * q_heads * stride * TC_D);
    a.pre_out = a.err + 4;
    a.withhold = withhold ? 1u : 0u;
    *used = true;
    switch (rep) {
        case 1: return tc_launch<1>(mk, mv, mq, out, a, G, st);
        case 2: return tc_launch<2>(mk, mv, mq, out, a, G, st);
        case 4: return tc_launch<4>(mk, mv, mq, out, a, G, st);
        default: return tc_launch<8>(mk, mv, mq, out, a, G, st);
    }
}

int device_status(int reset, uint32_t* flags) {
    unsigned int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v));
    if (e == cudaSuccess && reset) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
    }
    if (e != cudaSuccess)
        return set_error(OXIDE_ERR_CUDA, "oxide_device_status: %s", cudaGetErrorString(e));
    *flags = v;
    return OXIDE_OK;
}

}  // namespace oxide
