// k_kvcache.cu -- KV-cache append and grouped-query head repetition.
//
// Reference: repeat_kv (src/ops/attention.rs:161-201; kernel intent
// repeat_kv_f32, src/kernels/attention.rs:235-266): x [batch, kv_heads, seq,
// head_dim] -> out [batch, kv_heads * n_rep, seq, head_dim] with
// out[b, h * n_rep + r] = x[b, h].  KVCache::update (src/cache/kv_cache.rs:55-85;
// kernel intent kv_cache_update_f32, src/kernels/attention.rs:121-158): the new
// keys and values [batch, kv_heads, new_len, head_dim] are written at positions
// [cur_len, cur_len + new_len) of per-layer caches [batch, kv_heads, max_seq,
// head_dim], rejecting an append past max_seq ("KV cache overflow").
//
// Both are pure copies (bit-exact): a grid-stride loop over 16-byte vectors of
// the source, each read once; repeat_kv writes every source vector to its
// n_rep destinations, the append copies k and v in one launch.  Unaligned
// pointers or rows that are not whole vectors take element-wise kernels.
#include "oxide_common.cuh"

namespace oxide {

constexpr int KV_THREADS = 256;

// 16-byte vectors (bytes are copied as uint4 regardless of T), KV_UNROLL
// loads in flight per thread before their stores.  Index divisions use
// precomputed 32-bit multiply-shift division while every vector index fits 32
// bits (narrow), 64-bit division otherwise.
constexpr int KV_UNROLL = 4;
__global__ void __launch_bounds__(KV_THREADS)
    repeat_kv_vec_kernel(const uint4* x, uint4* out, uint64_t heads_total, uint32_t vec_per_head,
                         uint32_t kv_heads, uint32_t n_rep, FastDiv vdiv, FastDiv hdiv, bool narrow) {
    pdl_begin();
    const uint64_t n = heads_total * vec_per_head;
    const uint64_t stride = (uint64_t)gridDim.x * KV_THREADS;
    for (uint64_t i0 = (uint64_t)blockIdx.x * KV_THREADS + threadIdx.x; i0 < n; i0 += stride * KV_UNROLL) {
        uint4 v[KV_UNROLL];
#pragma unroll
        for (int u = 0; u < KV_UNROLL; ++u) {
            const uint64_t i = i0 + u * stride;
            if (i < n) v[u] = ld_stream(x + i);
        }
#pragma unroll
        for (int u = 0; u < KV_UNROLL; ++u) {
            const uint64_t i = i0 + u * stride;
            if (i >= n) break;
            uint64_t bh, b;
            if (narrow) {
                bh = vdiv.div((uint32_t)i);
                b = hdiv.div((uint32_t)bh);
            } else {
                bh = i / vec_per_head;
                b = bh / kv_heads;
            }
            const uint64_t off = i - bh * vec_per_head, h = bh - b * kv_heads;
            uint4* dst = out + ((b * kv_heads + h) * n_rep) * vec_per_head + off;
            for (uint32_t r = 0; r < n_rep; ++r) st_stream(dst + (uint64_t)r * vec_per_head, v[u]);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(KV_THREADS)
    repeat_kv_scalar_kernel(const T* x, T* out, uint64_t heads_total, uint64_t per_head, uint64_t kv_heads,
                            uint32_t n_rep) {
    pdl_begin();
    const uint64_t n = heads_total * per_head;
    for (uint64_t i = (uint64_t)blockIdx.x * KV_THREADS + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * KV_THREADS) {
        const uint64_t bh = i / per_head, off = i - bh * per_head;
        const uint64_t b = bh / kv_heads, h = bh - b * kv_heads;
        const T v = x[i];
        T* dst = out + ((b * kv_heads + h) * n_rep) * per_head + off;
        for (uint32_t r = 0; r < n_rep; ++r) dst[(uint64_t)r * per_head] = v;
    }
}

// k and v rows of `new_len` tokens -> cache positions [cur, cur + new_len).
// Work item i < 2 * heads_total * new_vec: the first half copies k, the second v.
__global__ void __launch_bounds__(KV_THREADS)
    kv_append_vec_kernel(uint4* kc, uint4* vc, const uint4* k, const uint4* v, uint64_t heads_total,
                         uint64_t new_vec, uint64_t max_vec, uint64_t cur_vec, FastDiv ndiv, bool narrow) {
    pdl_begin();
    const uint64_t half = heads_total * new_vec;
    for (uint64_t i = (uint64_t)blockIdx.x * KV_THREADS + threadIdx.x; i < 2 * half;
         i += (uint64_t)gridDim.x * KV_THREADS) {
        const bool is_v = i >= half;
        const uint64_t j = is_v ? i - half : i;
        const uint64_t bh = narrow ? ndiv.div((uint32_t)j) : j / new_vec, off = j - bh * new_vec;
        const uint4 val = ld_stream((is_v ? v : k) + j);
        st_stream((is_v ? vc : kc) + bh * max_vec + cur_vec + off, val);
    }
}

template <typename T>
__global__ void __launch_bounds__(KV_THREADS)
    kv_append_scalar_kernel(T* kc, T* vc, const T* k, const T* v, uint64_t heads_total, uint64_t new_elems,
                            uint64_t max_elems, uint64_t cur_elems) {
    pdl_begin();
    const uint64_t half = heads_total * new_elems;
    for (uint64_t i = (uint64_t)blockIdx.x * KV_THREADS + threadIdx.x; i < 2 * half;
         i += (uint64_t)gridDim.x * KV_THREADS) {
        const bool is_v = i >= half;
        const uint64_t j = is_v ? i - half : i;
        const uint64_t bh = j / new_elems, off = j - bh * new_elems;
        (is_v ? vc : kc)[bh * max_elems + cur_elems + off] = (is_v ? v : k)[j];
    }
}

static unsigned copy_grid(const void* kern, uint64_t items) {
    const uint64_t cap = (uint64_t)resident_blocks(kern, KV_THREADS, 0);
    uint64_t need = (items + KV_THREADS - 1) / KV_THREADS;
    if (need < 1) need = 1;
    return (unsigned)(need < cap ? need : cap);
}

template <typename T>
static int repeat_kv_entry(const char* name, const T* x, T* out, uint64_t batch, uint64_t kv_heads,
                           uint64_t seq, uint64_t head_dim, uint64_t n_rep, cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(n_rep >= 1 && n_rep < (1ull << 16), name, "n_rep must be in [1, 65536)");
    if (batch == 0 || kv_heads == 0 || seq == 0 || head_dim == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && out, name, "null pointer");
    OXIDE_REQUIRE(kv_heads < (1ull << 32), name, "kv_heads must be < 2^32");
    OXIDE_REQUIRE(seq <= UINT64_MAX / head_dim && batch <= UINT64_MAX / kv_heads / n_rep / (seq * head_dim),
                  name, "tensor size overflows");
    OXIDE_REQUIRE(x != out, name, "out must not alias x");
    const uint64_t per_head = seq * head_dim, heads_total = batch * kv_heads;
    constexpr uint64_t V = 16 / sizeof(T);
    if (aligned16(x) && aligned16(out) && per_head % V == 0 && per_head / V < (1ull << 32)) {
        const uint64_t vph = per_head / V, items = heads_total * vph;
        const bool narrow = items < (1ull << 32);
        launch_k(repeat_kv_vec_kernel, copy_grid(reinterpret_cast<const void*>(repeat_kv_vec_kernel), items), KV_THREADS, 0, st, reinterpret_cast<const uint4*>(x), reinterpret_cast<uint4*>(out),
                                                    heads_total, (uint32_t)vph, (uint32_t)kv_heads,
                                                    (uint32_t)n_rep, FastDiv((uint32_t)vph),
                                                    FastDiv((uint32_t)kv_heads), narrow);
    } else {
        auto kern = repeat_kv_scalar_kernel<T>;
        launch_k(kern, copy_grid(reinterpret_cast<const void*>(kern), heads_total * per_head), KV_THREADS, 0, st, 
            x, out, heads_total, per_head, kv_heads, (uint32_t)n_rep);
    }
    return check_launch(name);
}

template <typename T>
static int kv_append_entry(const char* name, T* kc, T* vc, const T* k, const T* v, uint64_t batch,
                           uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim, uint64_t cur_len,
                           uint64_t new_len, cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(cur_len <= max_seq && new_len <= max_seq - cur_len, name,
                  "KV cache overflow: cur_len + new_len > max_seq");
    if (batch == 0 || kv_heads == 0 || new_len == 0 || head_dim == 0) return OXIDE_OK;
    OXIDE_REQUIRE(kc && vc && k && v, name, "null pointer");
    OXIDE_REQUIRE(max_seq <= UINT64_MAX / head_dim && batch <= UINT64_MAX / kv_heads / (max_seq * head_dim),
                  name, "cache size overflows");
    const uint64_t heads_total = batch * kv_heads;
    constexpr uint64_t V = 16 / sizeof(T);
    if (aligned16(kc) && aligned16(vc) && aligned16(k) && aligned16(v) && head_dim % V == 0) {
        const uint64_t hv = head_dim / V, new_vec = new_len * hv;
        const bool narrow = heads_total * new_vec < (1ull << 32);
        launch_k(kv_append_vec_kernel, copy_grid(reinterpret_cast<const void*>(kv_append_vec_kernel),
                                         2 * heads_total * new_vec), KV_THREADS, 0, st, reinterpret_cast<uint4*>(kc), reinterpret_cast<uint4*>(vc),
                                                    reinterpret_cast<const uint4*>(k), reinterpret_cast<const uint4*>(v),
                                                    heads_total, new_vec, max_seq * hv, cur_len * hv,
                                                    FastDiv((uint32_t)(narrow ? new_vec : 1)), narrow);
    } else {
        auto kern = kv_append_scalar_kernel<T>;
        launch_k(kern, copy_grid(reinterpret_cast<const void*>(kern), 2 * heads_total * new_len * head_dim), KV_THREADS, 0, st, kc, vc, k, v, heads_total, new_len * head_dim, max_seq * head_dim, cur_len * head_dim);
    }
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_repeat_kv_f32(const float* x, float* out, uint64_t batch, uint64_t kv_heads, uint64_t seq_len,
                        uint64_t head_dim, uint64_t n_rep, oxide_stream_t stream) {
    return oxide::repeat_kv_entry<float>("oxide_repeat_kv_f32", x, out, batch, kv_heads, seq_len, head_dim,
                                         n_rep, stream);
}
int oxide_repeat_kv_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t batch, uint64_t kv_heads,
                         uint64_t seq_len, uint64_t head_dim, uint64_t n_rep, oxide_stream_t stream) {
    return oxide::repeat_kv_entry<bf16_t>("oxide_repeat_kv_bf16", x, out, batch, kv_heads, seq_len, head_dim,
                                          n_rep, stream);
}
int oxide_kv_cache_append_f32(float* k_cache, float* v_cache, const float* k, const float* v, uint64_t batch,
                              uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim, uint64_t cur_len,
                              uint64_t new_len, oxide_stream_t stream) {
    return oxide::kv_append_entry<float>("oxide_kv_cache_append_f32", k_cache, v_cache, k, v, batch, kv_heads,
                                         max_seq, head_dim, cur_len, new_len, stream);
}
int oxide_kv_cache_append_bf16(oxide_bf16* k_cache, oxide_bf16* v_cache, const oxide_bf16* k,
                               const oxide_bf16* v, uint64_t batch, uint64_t kv_heads, uint64_t max_seq,
                               uint64_t head_dim, uint64_t cur_len, uint64_t new_len, oxide_stream_t stream) {
    return oxide::kv_append_entry<bf16_t>("oxide_kv_cache_append_bf16", k_cache, v_cache, k, v, batch, kv_heads,
                                          max_seq, head_dim, cur_len, new_len, stream);
}

}  // extern "C"
