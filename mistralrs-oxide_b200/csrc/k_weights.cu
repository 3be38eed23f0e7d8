// k_weights.cu -- decoding of safetensors element bytes into device tensors.
//
// Reference: SafetensorsLoader::load_tensor_from_view
// (src/loading/safetensors.rs:48-82) turns each tensor's little-endian bytes
// into an f32 tensor: F32 as f32::from_le_bytes, F16 through half::f16 ->
// f32 (exact), and BF16 -- by mistake -- also through half::f16, which
// misreads every bf16 value.  Here BF16 is decoded as what it is, the high
// half of an f32 (exact); F16 follows the half crate's conversion bit for bit,
// including NaN payloads (quiet bit set, payload kept).  The bf16 entry point
// stores the decoded values rounded to nearest-even bf16 (exact for BF16).
//
// An HBM-bound elementwise pass: 16-byte loads of the source (8 halves or 4
// floats) when the pointers and the element count allow it, element loads
// otherwise (safetensors data offsets need not be 16-byte aligned).
#include <type_traits>

#include "oxide_common.cuh"

namespace oxide {

constexpr int WD_THREADS = 256;

// binary16 bits -> f32, exactly as the half crate converts them
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    if (exp == 0) {
        if (man == 0) return __uint_as_float(sign);
        return __uint_as_float(sign | __float_as_uint((float)man * 0x1p-24f));  // subnormal, exact
    }
    if (exp == 31) return __uint_as_float(man == 0 ? (sign | 0x7F800000u) : (sign | 0x7FC00000u | (man << 13)));
    return __uint_as_float(sign | ((exp + 112u) << 23) | (man << 13));
}

template <int SRC>
__device__ __forceinline__ float decode_one(const unsigned char* src, uint64_t i) {
    if (SRC == OXIDE_WDT_F32) return reinterpret_cast<const float*>(src)[i];
    const uint32_t h = reinterpret_cast<const uint16_t*>(src)[i];
    return SRC == OXIDE_WDT_F16 ? f16_bits_to_f32(h) : __uint_as_float(h << 16);
}

template <typename O>
__device__ __forceinline__ void store_one(O* out, uint64_t i, float v);
template <>
__device__ __forceinline__ void store_one<float>(float* out, uint64_t i, float v) {
    out[i] = v;
}
template <>
__device__ __forceinline__ void store_one<bf16_t>(bf16_t* out, uint64_t i, float v) {
    out[i] = f32_to_bf16(v);
}

// 16-byte groups: 4 source elements (F32) or 8 (F16 / BF16) per group
template <int SRC, typename O>
__global__ void __launch_bounds__(WD_THREADS)
    decode_vec_kernel(const unsigned char* src, O* out, uint64_t groups) {
    constexpr int E = SRC == OXIDE_WDT_F32 ? 4 : 8;
    for (uint64_t g = (uint64_t)blockIdx.x * WD_THREADS + threadIdx.x; g < groups;
         g += (uint64_t)gridDim.x * WD_THREADS) {
        const uint4 w = ld_stream(src + g * 16);
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
        float v[E];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (SRC == OXIDE_WDT_F32) {
                v[k] = __uint_as_float(wv[k]);
            } else {
                const uint32_t lo = wv[k] & 0xFFFFu, hi = wv[k] >> 16;
                v[2 * k] = SRC == OXIDE_WDT_F16 ? f16_bits_to_f32(lo) : __uint_as_float(lo << 16);
                v[2 * k + 1] = SRC == OXIDE_WDT_F16 ? f16_bits_to_f32(hi) : __uint_as_float(hi << 16);
            }
        }
        if constexpr (std::is_same<O, float>::value) {
#pragma unroll
            for (int k = 0; k < E; k += 4)
                st_stream(out + g * E + k, make_uint4(__float_as_uint(v[k]), __float_as_uint(v[k + 1]),
                                                      __float_as_uint(v[k + 2]), __float_as_uint(v[k + 3])));
        } else {
            if (E == 8) {
                st_stream(out + g * E, make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                  pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7])));
            } else {
                uint2* o = reinterpret_cast<uint2*>(out + g * E);
                *o = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
            }
        }
    }
}

template <int SRC, typename O>
__global__ void __launch_bounds__(WD_THREADS)
    decode_scalar_kernel(const unsigned char* src, O* out, uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * WD_THREADS + threadIdx.x; i < n; i += (uint64_t)gridDim.x * WD_THREADS)
        store_one<O>(out, i, decode_one<SRC>(src, i));
}

template <int SRC, typename O>
static void launch_decode(const unsigned char* src, O* out, uint64_t n, cudaStream_t st) {
    constexpr uint64_t E = SRC == OXIDE_WDT_F32 ? 4 : 8;
    constexpr uint64_t OB = sizeof(O) * E;  // output bytes per group
    const bool vec = aligned16(src) && (reinterpret_cast<uintptr_t>(out) % (OB < 16 ? OB : 16)) == 0 && n % E == 0;
    const uint64_t items = vec ? n / E : n;
    const void* k = vec ? reinterpret_cast<const void*>(decode_vec_kernel<SRC, O>)
                        : reinterpret_cast<const void*>(decode_scalar_kernel<SRC, O>);
    const uint64_t cap = (uint64_t)resident_blocks(k, WD_THREADS, 0);
    uint64_t grid = (items + WD_THREADS - 1) / WD_THREADS;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    if (vec) decode_vec_kernel<SRC, O><<<(unsigned)grid, WD_THREADS, 0, st>>>(src, out, items);
    else decode_scalar_kernel<SRC, O><<<(unsigned)grid, WD_THREADS, 0, st>>>(src, out, n);
}

template <typename O>
static int decode_entry(const char* name, const void* src, uint64_t n, int dtype, O* out, cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(dtype == OXIDE_WDT_F32 || dtype == OXIDE_WDT_F16 || dtype == OXIDE_WDT_BF16, name,
                  "src_dtype must be OXIDE_WDT_F32, OXIDE_WDT_F16 or OXIDE_WDT_BF16");
    if (n == 0) return OXIDE_OK;
    OXIDE_REQUIRE(src && out, name, "null pointer");
    const uint64_t es = dtype == OXIDE_WDT_F32 ? 4 : 2;
    OXIDE_REQUIRE(n <= UINT64_MAX / 4, name, "element count overflows");
    OXIDE_REQUIRE(reinterpret_cast<uintptr_t>(src) % es == 0, name, "src must be aligned to its element size");
    const unsigned char* s = static_cast<const unsigned char*>(src);
    if (dtype == OXIDE_WDT_F32) launch_decode<OXIDE_WDT_F32, O>(s, out, n, st);
    else if (dtype == OXIDE_WDT_F16) launch_decode<OXIDE_WDT_F16, O>(s, out, n, st);
    else launch_decode<OXIDE_WDT_BF16, O>(s, out, n, st);
    return check_launch(name);
}

}  // namespace oxide

extern "C" {

int oxide_decode_weights_f32(const void* src, uint64_t n, int src_dtype, float* out, oxide_stream_t stream) {
    return oxide::decode_entry<float>("oxide_decode_weights_f32", src, n, src_dtype, out, stream);
}
int oxide_decode_weights_bf16(const void* src, uint64_t n, int src_dtype, oxide_bf16* out, oxide_stream_t stream) {
    return oxide::decode_entry<oxide::bf16_t>("oxide_decode_weights_bf16", src, n, src_dtype,
                                              reinterpret_cast<oxide::bf16_t*>(out), stream);
}

}  // extern "C"
