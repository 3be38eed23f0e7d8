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
// An HBM-bound elementwise pass: vector loads and stores when the pointers and
// the element count allow it, element loads otherwise (safetensors data
// offsets need not be 16-byte aligned).
#include <cuda_fp16.h>

#include <type_traits>

#include "oxide_common.cuh"

namespace oxide {

constexpr int WD_THREADS = 256;

// binary16 bits -> f32, exactly as the half crate converts them: the
// hardware conversion (exact for every number and infinity, subnormals
// included), with NaNs rebuilt as the crate builds them (quiet bit set,
// payload kept) rather than left to the hardware's NaN output.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    const float v = __half2float(__ushort_as_half((unsigned short)h));
    const uint32_t nan = ((h & 0x8000u) << 16) | 0x7FC00000u | ((h & 0x3FFu) << 13);
    return (h & 0x7FFFu) > 0x7C00u ? __uint_as_float(nan) : v;
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

// Items of E elements, sized so that every warp-wide store is contiguous (a
// lane's 16 output bytes next to its neighbours'): 2-byte sources decoded to
// f32 move 4 elements per item (8-byte load, 16-byte store), 2-byte sources to
// bf16 8 (16 + 16 bytes), f32 sources 4 (16 bytes in, 16 or 8 out).  Each
// thread has WD_UNROLL item loads in flight before it converts and stores.
constexpr int WD_UNROLL = 4;

template <int SRC, typename O>
struct DecodeItem {
    static constexpr bool HALF = SRC != OXIDE_WDT_F32;
    static constexpr int E = HALF && sizeof(O) == 2 ? 8 : 4;  // elements per item
    static constexpr int SB = E * (HALF ? 2 : 4);                // source bytes per item
};

template <int SRC>
__device__ __forceinline__ float decode_bits(uint32_t h) {
    return SRC == OXIDE_WDT_F16 ? f16_bits_to_f32(h) : __uint_as_float(h << 16);
}

template <int SRC, typename O>
__device__ __forceinline__ void decode_item(const uint4 w, O* out, uint64_t g) {
    constexpr int E = DecodeItem<SRC, O>::E;
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    float v[E];
    if (SRC == OXIDE_WDT_F32) {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __uint_as_float(wv[k]);
    } else {
#pragma unroll
        for (int k = 0; k < E / 2; ++k) {
            v[2 * k] = decode_bits<SRC>(wv[k] & 0xFFFFu);
            v[2 * k + 1] = decode_bits<SRC>(wv[k] >> 16);
        }
    }
    if constexpr (std::is_same<O, float>::value) {
        st_stream(out + g * 4, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                                          __float_as_uint(v[3])));
    } else if constexpr (E == 8) {
        st_stream(out + g * 8, make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                          pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7])));
    } else {
        *reinterpret_cast<uint2*>(out + g * 4) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
    }
}

template <int SRC, typename O>
__global__ void __launch_bounds__(WD_THREADS)
    decode_vec_kernel(const unsigned char* src, O* out, uint64_t items) {
    pdl_begin();
    constexpr int SB = DecodeItem<SRC, O>::SB;
    constexpr uint64_t STEP = (uint64_t)WD_THREADS * WD_UNROLL;
    for (uint64_t g0 = (uint64_t)blockIdx.x * STEP + threadIdx.x; g0 < items; g0 += (uint64_t)gridDim.x * STEP) {
        uint4 w[WD_UNROLL];
#pragma unroll
        for (int u = 0; u < WD_UNROLL; ++u) {
            const uint64_t g = g0 + (uint64_t)u * WD_THREADS;
            if (g < items) {
                if constexpr (SB == 16) {
                    w[u] = ld_stream(src + g * 16);
                } else {
                    const uint2 h = __ldcs(reinterpret_cast<const uint2*>(src + g * 8));
                    w[u] = make_uint4(h.x, h.y, 0u, 0u);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < WD_UNROLL; ++u) {
            const uint64_t g = g0 + (uint64_t)u * WD_THREADS;
            if (g < items) decode_item<SRC, O>(w[u], out, g);
        }
    }
}

template <int SRC, typename O>
__global__ void __launch_bounds__(WD_THREADS)
    decode_scalar_kernel(const unsigned char* src, O* out, uint64_t n) {
    pdl_begin();
    for (uint64_t i = (uint64_t)blockIdx.x * WD_THREADS + threadIdx.x; i < n; i += (uint64_t)gridDim.x * WD_THREADS)
        store_one<O>(out, i, decode_one<SRC>(src, i));
}

template <int SRC, typename O>
static void launch_decode(const unsigned char* src, O* out, uint64_t n, cudaStream_t st) {
    constexpr uint64_t E = DecodeItem<SRC, O>::E, SB = DecodeItem<SRC, O>::SB;
    constexpr uint64_t OB = sizeof(O) * E;  // output bytes per item
    const bool vec = reinterpret_cast<uintptr_t>(src) % SB == 0 && reinterpret_cast<uintptr_t>(out) % OB == 0 &&
                     n % E == 0;
    const uint64_t items = vec ? n / E : n;
    const void* k = vec ? reinterpret_cast<const void*>(decode_vec_kernel<SRC, O>)
                        : reinterpret_cast<const void*>(decode_scalar_kernel<SRC, O>);
    const uint64_t cap = (uint64_t)resident_blocks(k, WD_THREADS, 0);
    const uint64_t per = vec ? (uint64_t)WD_THREADS * WD_UNROLL : WD_THREADS;
    uint64_t grid = (items + per - 1) / per;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    if (vec) launch_k(decode_vec_kernel<SRC, O>, (unsigned)grid, WD_THREADS, 0, st, src, out, items);
    else launch_k(decode_scalar_kernel<SRC, O>, (unsigned)grid, WD_THREADS, 0, st, src, out, n);
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
