// k_rope.cu -- rotate-half rotary position embedding of q and k in one launch.
//
// Reference: src/ops/attention.rs:139-155 (o[d] = x1*c - x2*s,
// o[d+half] = x1*s + x2*c with cos/sin tables [pos, half]); token-major
// layout of apply_rope_f32 (src/kernels/attention.rs:91-118); the two calls of
// MultiHeadAttention::forward (src/layers/attention.rs:88-94) become one
// launch.  Tables follow precompute_rope_cache (src/models/mistral.rs:91-115).
//
// Design: one CTA per group of ROPE_TOK tokens.  Its threads cover (head,
// 16-byte chunk of the first half) items of q and then k, each for every
// token of the group (all their loads issued first); an item reads the
// matching chunk of the second half, the token's cos/sin chunk (shared by all
// heads of the token, so it is served by L1 after the first head), and writes
// both halves.
// Arithmetic is f32 with each product and sum rounded separately, as in the
// reference; bf16 results are rounded once at the store.  A position beyond
// the table yields NaN for that token instead of an out-of-bounds read.
#include <math.h>

#include "oxide_common.cuh"

namespace oxide {

struct RopeArgs {
    uint64_t tokens;
    uint64_t table_rows;
    uint32_t q_heads, k_heads, head_dim;
    int layout;      // 0 token-major [T,H,D], 1 head-major [H,T,D]
    FastDiv cph_div;  // division by the 16-byte chunks per half head
};

__device__ __forceinline__ uint64_t rope_base(const RopeArgs& p, uint64_t t, uint32_t h,
                                              uint32_t heads) {
    return p.layout == 0 ? (t * heads + h) * p.head_dim : ((uint64_t)h * p.tokens + t) * p.head_dim;
}

__device__ __forceinline__ void rot(float x1, float x2, float c, float s, float& o1, float& o2) {
    o1 = fsub(fmul(x1, c), fmul(x2, s));
    o2 = fadd(fmul(x1, s), fmul(x2, c));
}
// Tokens per CTA pass: a thread issues the loads of its item for all of them
// before it rotates any, so more bytes are in flight per thread.
constexpr int ROPE_TOK = 2;

template <typename T>
__global__ void __launch_bounds__(512)
    rope_vec_kernel(const T* q, T* qo, const T* k, T* ko, const float* cos_t, const float* sin_t,
                    const int32_t* pos, RopeArgs p) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    const uint32_t half = p.head_dim / 2;
    const uint32_t cph = half / V;  // chunks per head
    const uint32_t items = (p.q_heads + (k ? p.k_heads : 0)) * cph;
    for (uint64_t t0 = (uint64_t)blockIdx.x * ROPE_TOK; t0 < p.tokens; t0 += (uint64_t)gridDim.x * ROPE_TOK) {
        for (uint32_t it = threadIdx.x; it < items; it += blockDim.x) {
            const uint32_t hh = p.cph_div.div(it), c = it - hh * cph;
            const bool isq = hh < p.q_heads;
            const uint32_t h = isq ? hh : hh - p.q_heads;
            const uint32_t heads = isq ? p.q_heads : p.k_heads;
            const T* src = isq ? q : k;
            T* dst = isq ? qo : ko;
            uint4 r1[ROPE_TOK], r2[ROPE_TOK];
            int64_t pr[ROPE_TOK];
#pragma unroll
            for (int u = 0; u < ROPE_TOK; ++u) {
                const uint64_t t = t0 + u;
                if (t < p.tokens) {
                    const uint64_t base = rope_base(p, t, h, heads) + c * V;
                    r1[u] = ld_stream(src + base);
                    r2[u] = ld_stream(src + base + half);
                    pr[u] = pos ? (int64_t)pos[t] : (int64_t)t;
                }
            }
#pragma unroll
            for (int u = 0; u < ROPE_TOK; ++u) {
                const uint64_t t = t0 + u;
                if (t >= p.tokens) break;
                const uint64_t base = rope_base(p, t, h, heads) + c * V;
                float x1[V], x2[V], cs[V], sn[V], o1[V], o2[V];
                Vec<T>::unpack(r1[u], x1);
                Vec<T>::unpack(r2[u], x2);
                if (pr[u] >= 0 && (uint64_t)pr[u] < p.table_rows) {
                    const float* cp = cos_t + (uint64_t)pr[u] * half + c * V;
                    const float* sp = sin_t + (uint64_t)pr[u] * half + c * V;
#pragma unroll
                    for (int e = 0; e < V; e += 4) {
                        uint4 cv = ld_keep(cp + e), sv = ld_keep(sp + e);
                        Vec<float>::unpack(cv, cs + e);
                        Vec<float>::unpack(sv, sn + e);
                    }
                    // Scalar on purpose: a paired multiply feeding a paired add was
                    // measured to come out fused (one rounding) on sm_100a, which
                    // would break the bit-exact match with the reference's
                    // separately rounded x1*c - x2*s.
#pragma unroll
                    for (int e = 0; e < V; ++e) rot(x1[e], x2[e], cs[e], sn[e], o1[e], o2[e]);
                } else {
#pragma unroll
                    for (int e = 0; e < V; ++e) o1[e] = o2[e] = __int_as_float(0x7fc00000);
                }
                st_stream(dst + base, Vec<T>::pack(o1));
                st_stream(dst + base + half, Vec<T>::pack(o2));
            }
        }
    }
}

// Any alignment / head_dim: one thread per (token, head, d < half).
template <typename T>
__global__ void __launch_bounds__(256)
    rope_scalar_kernel(const T* q, T* qo, const T* k, T* ko, const float* cos_t,
                       const float* sin_t, const int32_t* pos, RopeArgs p) {
    pdl_begin();
    const uint32_t half = p.head_dim / 2;
    const uint64_t heads = p.q_heads + (k ? p.k_heads : 0);
    const uint64_t total = p.tokens * heads * half;
    for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t d = (uint32_t)(g % half);
        const uint64_t th = g / half;
        const uint64_t t = th / heads;
        const uint32_t hh = (uint32_t)(th % heads);
        const bool isq = hh < p.q_heads;
        const uint32_t h = isq ? hh : hh - p.q_heads;
        const uint64_t base = rope_base(p, t, h, isq ? p.q_heads : p.k_heads);
        const T* src = isq ? q : k;
        T* dst = isq ? qo : ko;
        const int64_t pr = pos ? (int64_t)pos[t] : (int64_t)t;
        float o1 = __int_as_float(0x7fc00000), o2 = o1;
        const float x1 = Vec<T>::load1(src + base + d), x2 = Vec<T>::load1(src + base + d + half);
        if (pr >= 0 && (uint64_t)pr < p.table_rows) {
            rot(x1, x2, __ldg(cos_t + (uint64_t)pr * half + d), __ldg(sin_t + (uint64_t)pr * half + d),
                o1, o2);
        }
        Vec<T>::store1(dst + base + d, o1);
        Vec<T>::store1(dst + base + d + half, o2);
    }
}

template <typename T>
static int rope_entry(const char* name, const T* q, T* qo, uint64_t qh, const T* k, T* ko,
                      uint64_t kh, const float* cos_t, const float* sin_t, uint64_t table_rows,
                      const int32_t* pos, uint64_t tokens, uint64_t head_dim, int layout,
                      cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    OXIDE_INJECT(name);
    if (tokens == 0) return OXIDE_OK;
    OXIDE_REQUIRE(q && qo && cos_t && sin_t, name, "null pointer");
    OXIDE_REQUIRE(!k || ko, name, "k_out is null while k is given");
    OXIDE_REQUIRE(layout == 0 || layout == 1, name, "layout must be 0 or 1");
    OXIDE_REQUIRE(head_dim >= 2 && head_dim % 2 == 0 && head_dim < (1u << 16), name,
                  "head_dim must be even and in [2, 65536)");
    OXIDE_REQUIRE(qh >= 1 && qh < (1u << 20) && (!k || (kh >= 1 && kh < (1u << 20))), name,
                  "head counts must be in [1, 2^20)");
    OXIDE_REQUIRE(pos || table_rows >= tokens, name, "table_rows < tokens without positions");
    OXIDE_REQUIRE(tokens <= UINT64_MAX / ((qh + kh) * head_dim), name, "tensor size overflows");
    RopeArgs p{tokens, table_rows, (uint32_t)qh, (uint32_t)(k ? kh : 0), (uint32_t)head_dim,
               layout, FastDiv()};
    const uint64_t half = head_dim / 2;
    const bool vec = half % V == 0 && half % 4 == 0 && aligned16(q) && aligned16(qo) &&
                     aligned16(cos_t) && aligned16(sin_t) && (!k || (aligned16(k) && aligned16(ko))) &&
                     (qh + (k ? kh : 0)) * (half / V) < (1ull << 31);  // items per token fit 32 bits
    p.cph_div = FastDiv((uint32_t)(half / V > 0 ? half / V : 1));
    const uint64_t cap = (uint64_t)1 << 30;
    if (vec) {
        const uint64_t items = (qh + (k ? kh : 0)) * (half / V);
        uint64_t threads = (items + 31) / 32 * 32;
        if (threads > 512) threads = 256;
        const uint64_t groups = (tokens + ROPE_TOK - 1) / ROPE_TOK;
        launch_k(rope_vec_kernel<T>, (unsigned)(groups < cap ? groups : cap), (unsigned)threads, 0, st, 
            q, qo, k, ko, cos_t, sin_t, pos, p);
    } else {
        const uint64_t total = tokens * (qh + (k ? kh : 0)) * half;
        const uint64_t blocks = (total + 255) / 256;
        const uint64_t bcap = (uint64_t)sm_count() * 8;
        launch_k(rope_scalar_kernel<T>, (unsigned)(blocks < bcap ? blocks : bcap), 256, 0, st, 
            q, qo, k, ko, cos_t, sin_t, pos, p);
    }
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_rope_f32(const float* q, float* q_out, uint64_t q_heads, const float* k, float* k_out,
                   uint64_t k_heads, const float* cos_t, const float* sin_t, uint64_t table_rows,
                   const int32_t* positions, uint64_t tokens, uint64_t head_dim, int layout,
                   oxide_stream_t stream) {
    return oxide::rope_entry<float>("oxide_rope_f32", q, q_out, q_heads, k, k_out, k_heads, cos_t,
                                    sin_t, table_rows, positions, tokens, head_dim, layout,
                                    stream);
}
int oxide_rope_bf16(const oxide_bf16* q, oxide_bf16* q_out, uint64_t q_heads,
                    const oxide_bf16* k, oxide_bf16* k_out, uint64_t k_heads,
                    const float* cos_t, const float* sin_t, uint64_t table_rows,
                    const int32_t* positions, uint64_t tokens, uint64_t head_dim, int layout,
                    oxide_stream_t stream) {
    return oxide::rope_entry<bf16_t>("oxide_rope_bf16", q, q_out, q_heads, k, k_out, k_heads,
                                     cos_t, sin_t, table_rows, positions, tokens, head_dim,
                                     layout, stream);
}

// Model set-up on the host: glibc powf/cosf/sinf, the functions Rust's
// f32::powf/cos/sin call, so the tables equal precompute_rope_cache's.
int oxide_rope_table_host_f32(float theta, uint64_t head_dim, uint64_t max_pos, float* cos_host,
                              float* sin_host) {
    OXIDE_INJECT("oxide_rope_table_host_f32");
    if (max_pos == 0) return OXIDE_OK;
    OXIDE_REQUIRE(cos_host && sin_host, "oxide_rope_table_host_f32", "null pointer");
    OXIDE_REQUIRE(head_dim >= 2 && head_dim % 2 == 0, "oxide_rope_table_host_f32",
                  "head_dim must be even and >= 2");
    const uint64_t half = head_dim / 2;
    for (uint64_t pos = 0; pos < max_pos; ++pos) {
        for (uint64_t i = 0; i < half; ++i) {
            volatile float expo = (-2.0f * (float)i) / (float)head_dim;
            float freq = powf(theta, expo);
            volatile float angle = (float)pos * freq;
            cos_host[pos * half + i] = cosf(angle);
            sin_host[pos * half + i] = sinf(angle);
        }
    }
    return OXIDE_OK;
}

}  // extern "C"
