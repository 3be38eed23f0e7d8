// k_elementwise.cu -- elementwise and broadcast ops (HBM-bound streaming).
//
// Reference semantics (src/ops/matmul.rs:136-158, elementwise_op_cpu):
//     out[i] = a[i % na] op b[i % nb]
// plus scale (build.rs:240-276), silu (src/ops/activation.rs:21-37) and the
// MLP pair silu-then-mul (src/layers/attention.rs:144-145) fused in one pass.
//
// Design: a persistent grid (resident CTAs x SMs) streams 16-byte vectors;
// each thread keeps UNROLL independent vectors per operand in flight, reads
// with ld.global.nc.L1::no_allocate and writes with st.global.cs (evict-first),
// so the only traffic is one read of each input and one write of the output.
// A broadcast operand (e.g. a [cols] row vector) is addressed by a fast
// modulo on the vector index and stays resident in L1/L2.
#include <type_traits>

#include "oxide_common.cuh"

namespace oxide {

constexpr int EW_THREADS = 256;
// 16-byte vectors in flight per thread and operand, and the register bound
// (min CTAs per SM): f32 keeps 8 vectors under a 2-CTA bound (128 registers);
// bf16, with twice the arithmetic per byte, 4 vectors under a 4-CTA bound.
// Measured on silu * up: f32 C2 235.7 -> 212.6 us with 8 vectors; bf16 C5
// (packed) 1957 us with 4 vectors under the 4-CTA bound, against 2104 under a
// 3-CTA bound, 2038 with 6 under 3 and 2287 with 8 under 2.
template <typename T>
constexpr int ew_unroll() {
    return sizeof(T) == 4 ? 8 : 4;
}
template <typename T>
constexpr int ew_min_blocks() {
    return sizeof(T) == 4 ? 2 : 4;
}
// ---- per-element functors (f32 math, IEEE rounding per reference step) ----
// operator() is one element; pair() is two elements on Blackwell's paired
// f32 pipe (__fmul2_rn / __fadd2_rn: the same IEEE round-to-nearest per lane,
// half the instructions).
template <int OP>
struct FBin {
    __device__ __forceinline__ float operator()(float x, float y) const {
        if (OP == OXIDE_ADD) return fadd(x, y);
        if (OP == OXIDE_SUB) return fsub(x, y);
        if (OP == OXIDE_MUL) return fmul(x, y);
        return fdiv(x, y);
    }
    __device__ __forceinline__ float2 pair(float2 x, float2 y) const {
        if (OP == OXIDE_ADD) return fadd2(x, y);
        if (OP == OXIDE_SUB) return fadd2(x, f2(-y.x, -y.y));  // x - y == x + (-y) exactly
        if (OP == OXIDE_MUL) return fmul2(x, y);
        return f2(fdiv(x.x, y.x), fdiv(x.y, y.y));
    }
};

// silu(x) = x * (1 / (1 + exp(-x))), src/ops/activation.rs:30-33.  The
// reciprocal is __frcp_rn: the correctly rounded 1/d, i.e. the reference's
// IEEE 1.0 / d.  ACCURATE (the f32 kernels): exp is exp_rn_f32, the correctly
// rounded e^x the reference's glibc expf returns on all but 4e-5 of the
// floats, so every later step rounds as the reference's does and the result
// is its bits except there; otherwise (bf16 results, rounded to 8 bits after
// the f32 math) CUDA's expf, within 2 ulp and a third of the instructions.
template <bool ACCURATE>
__device__ __forceinline__ float silu_exp(float nx) {
    return ACCURATE ? exp_rn_f32(nx) : expf(nx);
}
template <bool ACCURATE = true>
__device__ __forceinline__ float silu_f(float x) {
    float e = silu_exp<ACCURATE>(-x);
    float r = __frcp_rn(fadd(1.0f, e));
    return fmul(x, r);
}
// The f32 path in two parts: silu_fast2 decides most inputs, two at a time,
// with the f32 exponential (ok = false where its rounding test cannot),
// silu_exact takes the rest through the double exponential.  Results are
// silu_f<true>'s bits.
__device__ __forceinline__ float2 silu_fast2(float2 x, bool& ok0, bool& ok1) {
    const float2 e = exp_rn_f32x2_ff(f2(-x.x, -x.y), ok0, ok1);
    const float2 d = fadd2(f2(1.0f, 1.0f), e);
    return fmul2(x, f2(__frcp_rn(d.x), __frcp_rn(d.y)));
}
// The same without the flags: inputs in [-EXP_FF_XMAX, EXP_FF_XMAX] (checked
// by the caller), undecided inputs leave nonzero bits in `diff`.
__device__ __forceinline__ float2 silu_fast2r(float2 x, uint32_t& diff) {
    const float2 e = exp_rn_f32x2_ffr(f2(-x.x, -x.y), diff);
    const float2 d = fadd2(f2(1.0f, 1.0f), e);
    return fmul2(x, f2(__frcp_rn(d.x), __frcp_rn(d.y)));
}
__device__ __forceinline__ float silu_exact(float x) {
    return fmul(x, __frcp_rn(fadd(1.0f, exp_rn_f32_fallback(-x))));
}
template <bool ACCURATE = true>
__device__ __forceinline__ float2 silu_f2(float2 x) {
    const float2 d = fadd2(f2(1.0f, 1.0f), f2(silu_exp<ACCURATE>(-x.x), silu_exp<ACCURATE>(-x.y)));
    return fmul2(x, f2(__frcp_rn(d.x), __frcp_rn(d.y)));
}

// bf16x2 product rounded once to bf16 (subnormals kept).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

template <typename T>
struct FSiluMul {  // mul(silu(g), u); silu(g) rounded to T as the pair stores it
    // bf16 words are processed packed: silu of the two gate halves rounded to
    // bf16 by one paired conversion, then the product with the two up halves
    // rounded once by mul.rn.bf16x2.  The f32 product of two bf16 values is
    // exact, so this is the f32 multiply rounded to bf16, except where the
    // f32 product is subnormal and its own rounding would come first (a
    // double rounding the single one avoids): within 1 bf16 ulp there.
    static constexpr bool PACKED = sizeof(T) == 2;
    static constexpr bool ACC = sizeof(T) == 4;
    static constexpr bool FIXUP = ACC;
    __device__ __forceinline__ float operator()(float g, float u) const {
        return fmul(Vec<T>::rnd(silu_f<ACC>(g)), u);
    }
    __device__ __forceinline__ float2 fast2(float2 g, float2 u, bool& ok0, bool& ok1) const {
        return fmul2(silu_fast2(g, ok0, ok1), u);
    }
    __device__ __forceinline__ float2 fast2r(float2 g, float2 u, uint32_t& diff) const {
        return fmul2(silu_fast2r(g, diff), u);
    }
    __device__ __forceinline__ float exact(float g, float u) const { return fmul(silu_exact(g), u); }
    __device__ __forceinline__ float2 pair(float2 g, float2 u) const {
        const float2 s = silu_f2<ACC>(g);
        return fmul2(f2(Vec<T>::rnd(s.x), Vec<T>::rnd(s.y)), u);
    }
    __device__ __forceinline__ uint32_t packed(uint32_t g, uint32_t u) const {
        const float2 s = silu_f2<false>(f2(__uint_as_float(g << 16), __uint_as_float(g & 0xFFFF0000u)));
        return mul_bf16x2(pack_bf16x2(s.x, s.y), u);
    }
};

// Functors with a packed bf16 form declare PACKED = true; functors with a
// fast form that may leave elements undecided declare FIXUP = true (fast2()
// for two elements with their ok flags, exact() for the undecided ones).
template <typename F, typename = void>
struct HasPacked {
    static constexpr bool value = false;
};
template <typename F>
struct HasPacked<F, std::void_t<decltype(F::PACKED)>> {
    static constexpr bool value = F::PACKED;
};
template <typename F, typename = void>
struct HasFixup {
    static constexpr bool value = false;
};
template <typename F>
struct HasFixup<F, std::void_t<decltype(F::FIXUP)>> {
    static constexpr bool value = F::FIXUP;
};

template <typename T>
struct FSilu {
    static constexpr bool ACC = sizeof(T) == 4;
    static constexpr bool FIXUP = ACC;
    __device__ __forceinline__ float operator()(float x, float) const { return silu_f<ACC>(x); }
    __device__ __forceinline__ float2 pair(float2 x, float2) const { return silu_f2<ACC>(x); }
    __device__ __forceinline__ float2 fast2(float2 x, float2, bool& ok0, bool& ok1) const {
        return silu_fast2(x, ok0, ok1);
    }
    __device__ __forceinline__ float2 fast2r(float2 x, float2, uint32_t& diff) const {
        return silu_fast2r(x, diff);
    }
    __device__ __forceinline__ float exact(float x, float) const { return silu_exact(x); }
};

struct FScale {
    float s;
    __device__ __forceinline__ float operator()(float x, float) const { return fmul(x, s); }
    __device__ __forceinline__ float2 pair(float2 x, float2) const { return fmul2(x, f2(s, s)); }
};

// Unary ops of src/ops/activation.rs and src/ops/math.rs, each step rounded as
// the reference's f32 expression (scalar __f*_rn: never fused).  a: the pow
// exponent, the clamp minimum or gelu's sqrt(2 / pi) (computed on the host as
// the reference's (2.0 / PI).sqrt() in f32); b: the clamp maximum.
template <int OP>
struct FUnary {
    float a, b;
    __device__ __forceinline__ float operator()(float x, float) const {
        switch (OP) {
            case OXIDE_RELU: return fmaxf(x, 0.0f);  // f32::max(x, 0.0): NaN -> 0
            case OXIDE_GELU: {  // 0.5 * x * (1 + tanh(k * (x + 0.044715 * (x * x) * x)))
                const float half_x = fmul(0.5f, x);
                const float p = fmul(fmul(x, x), x);
                const float u = fadd(x, fmul(0.044715f, p));
                return fmul(half_x, fadd(1.0f, tanhf(fmul(a, u))));
            }
            case OXIDE_GELU_QUICK:  // x * (1 / (1 + exp(-1.702 * x)))
                return fmul(x, __frcp_rn(fadd(1.0f, expf(fmul(-1.702f, x)))));
            case OXIDE_SIGMOID: return __frcp_rn(fadd(1.0f, expf(-x)));
            case OXIDE_TANH: return tanhf(x);
            case OXIDE_EXP: return expf(x);
            case OXIDE_LOG: return logf(x);
            case OXIDE_SQRT: return fsqrt(x);
            case OXIDE_POW: return powf(x, a);
            case OXIDE_CLAMP: {  // f32::clamp: below min -> min, above max -> max, NaN stays
                float r = x;
                if (r < a) r = a;
                if (r > b) r = b;
                return r;
            }
            case OXIDE_NEG: return -x;
            default: return fabsf(x);
        }
    }
    __device__ __forceinline__ float2 pair(float2 x, float2 y) const {
        return f2((*this)(x.x, y.x), (*this)(x.y, y.y));
    }
};

// ---- vectorised kernel ------------------------------------------------------
// NIN = 1 (b unused) or 2.  AMOD/BMOD: operand indexed modulo its length
// (in vectors).  Requires 16-byte aligned pointers and, for modulo operands,
// lengths that are multiples of the vector width.
// bf16: 64 registers (4 CTAs of 256 threads per SM), measured 10% faster than
// the unbounded allocation (70 registers, 3 CTAs) for silu * up.
template <typename T, typename F, int NIN, bool AMOD, bool BMOD>
__global__ void __launch_bounds__(EW_THREADS, (ew_min_blocks<T>()))
    ew_vec_kernel(const T* a, const T* b, T* out, uint64_t nvec, uint64_t nav, uint64_t nbv,
                  FastDiv adiv, FastDiv bdiv, bool wide, uint64_t tail_lo, uint64_t n, F f) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    constexpr int EW_UNROLL = ew_unroll<T>();
    const uint64_t stride = (uint64_t)gridDim.x * EW_THREADS;
    for (uint64_t base = (uint64_t)blockIdx.x * EW_THREADS + threadIdx.x; base < nvec;
         base += stride * EW_UNROLL) {
        uint4 va[EW_UNROLL], vb[EW_UNROLL];
#pragma unroll
        for (int k = 0; k < EW_UNROLL; ++k) {
            const uint64_t i = base + k * stride;
            if (i < nvec) {
                uint64_t ia = i, ib = i;
                if (AMOD) ia = wide ? i % nav : adiv.mod((uint32_t)i);
                if (BMOD) ib = wide ? i % nbv : bdiv.mod((uint32_t)i);
                va[k] = AMOD ? ld_keep(a + ia * V) : ld_stream(a + ia * V);
                if (NIN == 2) vb[k] = BMOD ? ld_keep(b + ib * V) : ld_stream(b + ib * V);
            }
        }
#pragma unroll
        for (int k = 0; k < EW_UNROLL; ++k) {
            const uint64_t i = base + k * stride;
            if constexpr (HasPacked<F>::value && NIN == 2) {
                if (i < nvec)
                    st_stream(out + i * V, make_uint4(f.packed(va[k].x, vb[k].x), f.packed(va[k].y, vb[k].y),
                                                      f.packed(va[k].z, vb[k].z), f.packed(va[k].w, vb[k].w)));
            } else if (i < nvec) {
                float x[V], y[V], o[V];
                Vec<T>::unpack(va[k], x);
                if (NIN == 2) Vec<T>::unpack(vb[k], y);
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 r = f.pair(f2(x[e], x[e + 1]),
                                            NIN == 2 ? f2(y[e], y[e + 1]) : f2(0.0f, 0.0f));
                    o[e] = r.x;
                    o[e + 1] = r.y;
                }
                st_stream(out + i * V, Vec<T>::pack(o));
            }
        }
    }
    // Scalar tail of a full-length (non-modulo) op: elements [tail_lo, n).
    if (blockIdx.x == 0) {
        for (uint64_t i = tail_lo + threadIdx.x; i < n; i += EW_THREADS) {
            float x = Vec<T>::load1(a + i);
            float y = NIN == 2 ? Vec<T>::load1(b + i) : 0.0f;
            Vec<T>::store1(out + i, f(x, y));
        }
    }
}

// ---- staged kernel for functors with undecided elements (the f32 SiLU) --------
// The correctly rounded f32 SiLU needs more arithmetic per byte than the
// other ops, so more warps per SM to hide it, while the stream still needs
// as many bytes in flight.  Here the bytes in flight live in shared memory:
// each thread copies its own vectors (cp.async, 16 bytes each) into a
// per-thread ring of STG_STAGES groups of STG_UNROLL vectors per operand,
// and computes group j while groups j+1.. are in flight; registers hold only
// the arithmetic.  No thread reads another's slots, so there is no block
// barrier.  Every element goes through the fast form and is stored; the
// undecided ones (about 1 in 10^4) are then recomputed one by one from the
// staged copy (the output may be an input) and stored again.
// Measured on silu * up f32 [8192 x 14336]: 2 stages of 2 vectors under a
// 6-CTA bound 237 us; 2 x 2 under 5 CTAs 239, 4 x 1 under 6 CTAs 241, 3 x 2
// under 4 CTAs 250, 3 x 1 under 6 CTAs 256.  (The same arithmetic from
// registers, 4 vectors per thread under a 4-CTA bound: 237 us; CUDA's expf,
// not correctly rounded, 208 us.)  The kernel is issue-bound: 53 instructions
// per element, 75 % issue-active, ALU pipe 56 %, FMA pipe 50 %.
constexpr int STG_STAGES = 2;
constexpr int STG_UNROLL = 2;
constexpr int STG_MIN_BLOCKS = 6;

template <typename F, int NIN>
__global__ void __launch_bounds__(EW_THREADS, STG_MIN_BLOCKS)
    ew_staged_f32_kernel(const float* a, const float* b, float* out, uint64_t nvec, uint64_t n, F f) {
    pdl_begin();
    constexpr int V = 4, S = STG_STAGES, U = STG_UNROLL;
    __shared__ __align__(16) float4 sa[S][U][EW_THREADS];
    __shared__ __align__(16) float4 sb[NIN == 2 ? S : 1][U][EW_THREADS];
    const int tid = threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * EW_THREADS;
    const uint64_t first = (uint64_t)blockIdx.x * EW_THREADS + tid;
    // group j: vectors first + (j U + k) stride, k < U
    auto issue = [&](uint64_t j, int stage) {
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint64_t i = first + (j * U + k) * stride;
            if (i < nvec) {
                cp_async16(&sa[stage][k][tid], a + i * V);
                if (NIN == 2) cp_async16(&sb[stage][k][tid], b + i * V);
            }
        }
        cp_async_commit();  // one group per call, empty or not, so the wait counts stay uniform
    };
#pragma unroll
    for (int st = 0; st < S - 1; ++st) issue((uint64_t)st, st);
    for (uint64_t j = 0; first + j * U * stride < nvec; ++j) {
        const int stage = (int)(j % S);
        issue(j + S - 1, (int)((j + S - 1) % S));
        cp_async_wait<S - 1>();  // this thread's group j has landed
        // The fast path decides all U V elements unless an input lies outside
        // [-EXP_FF_XMAX, EXP_FF_XMAX] (one comparison of the largest |x|) or
        // a rounding test fails (nonzero diff); then, rarely, the vectors are
        // redone element by element and stored again.
        uint32_t diff = 0;
        float xmax = 0.0f;
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint64_t i = first + (j * U + k) * stride;
            const float4 x = sa[stage][k][tid];
            const float4 y = NIN == 2 ? sb[stage][k][tid] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            xmax = fmaxf(xmax, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
            const float2 r0 = f.fast2r(f2(x.x, x.y), f2(y.x, y.y), diff);
            const float2 r1 = f.fast2r(f2(x.z, x.w), f2(y.z, y.w), diff);
            if (i < nvec)
                st_stream(out + i * V, make_uint4(__float_as_uint(r0.x), __float_as_uint(r0.y), __float_as_uint(r1.x),
                                                  __float_as_uint(r1.y)));
        }
        if (diff != 0 || !(xmax <= EXP_FF_XMAX)) {
#pragma unroll 1
            for (int k = 0; k < U; ++k) {
                const uint64_t i = first + (j * U + k) * stride;
                const float4 x = sa[stage][k][tid];
                const float4 y = NIN == 2 ? sb[stage][k][tid] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                bool o0, o1, o2, o3;
                float2 r0 = f.fast2(f2(x.x, x.y), f2(y.x, y.y), o0, o1);
                float2 r1 = f.fast2(f2(x.z, x.w), f2(y.z, y.w), o2, o3);
                if (!o0) r0.x = f.exact(x.x, y.x);
                if (!o1) r0.y = f.exact(x.y, y.y);
                if (!o2) r1.x = f.exact(x.z, y.z);
                if (!o3) r1.y = f.exact(x.w, y.w);
                if (i < nvec)
                    st_stream(out + i * V, make_uint4(__float_as_uint(r0.x), __float_as_uint(r0.y),
                                                      __float_as_uint(r1.x), __float_as_uint(r1.y)));
            }
        }
    }
    cp_async_wait<0>();  // nothing in flight into shared memory at exit
    // Scalar tail: elements [nvec V, n).
    if (blockIdx.x == 0) {
        for (uint64_t i = nvec * V + tid; i < n; i += EW_THREADS) {
            const float x = a[i];
            const float y = NIN == 2 ? b[i] : 0.0f;
            out[i] = f(x, y);
        }
    }
}

// ---- scalar kernel (any alignment, any lengths) ------------------------------
template <typename T, typename F, int NIN>
__global__ void __launch_bounds__(EW_THREADS)
    ew_scalar_kernel(const T* a, uint64_t na, const T* b, uint64_t nb, T* out, uint64_t n, F f) {
    pdl_begin();
    const uint64_t stride = (uint64_t)gridDim.x * EW_THREADS;
    for (uint64_t i = (uint64_t)blockIdx.x * EW_THREADS + threadIdx.x; i < n; i += stride) {
        float x = Vec<T>::load1(a + (na == n ? i : i % na));
        float y = NIN == 2 ? Vec<T>::load1(b + (nb == n ? i : i % nb)) : 0.0f;
        Vec<T>::store1(out + i, f(x, y));
    }
}

template <typename K>
static int resident_grid(K kernel, uint64_t work_items) {
    const int cap = resident_blocks(reinterpret_cast<const void*>(kernel), EW_THREADS, 0);
    uint64_t need = (work_items + EW_THREADS - 1) / EW_THREADS;
    if (need < 1) need = 1;
    return (int)(need < (uint64_t)cap ? need : (uint64_t)cap);
}

// Launch a vectorised kernel instance chosen by the modulo flags.
template <typename T, typename F, int NIN, bool AMOD, bool BMOD>
static void launch_vec(const T* a, uint64_t na, const T* b, uint64_t nb, T* out, uint64_t n,
                       F f, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    const uint64_t nvec = n / V;
    const uint64_t nav = na / V, nbv = nb / V;
    const bool wide = nvec >= 0xffffffffull;
    FastDiv adiv(AMOD && !wide ? (uint32_t)nav : 1u);
    FastDiv bdiv(BMOD && !wide ? (uint32_t)nbv : 1u);
    auto kern = ew_vec_kernel<T, F, NIN, AMOD, BMOD>;
    constexpr uint64_t U = ew_unroll<T>();
    uint64_t items = (nvec + U - 1) / U;
    int grid = resident_grid(kern, items > 0 ? items : 1);
    launch_k(kern, grid, EW_THREADS, 0, st, a, b, out, nvec, nav, nbv, adiv, bdiv, wide, nvec * V, n,
                                      f);
}

// Dispatch: vector path when every pointer is 16-byte aligned and every
// length that is indexed modulo is a multiple of the vector width; scalar
// path otherwise (still on the GPU).
template <typename T, typename F, int NIN>
static int ew_dispatch(const char* name, const T* a, uint64_t na, const T* b, uint64_t nb,
                       T* out, uint64_t n, F f, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    const bool amod = na != n, bmod = NIN == 2 && nb != n;
    bool vec = aligned16(a) && aligned16(out) && (NIN == 1 || aligned16(b));
    if (amod || bmod) vec = vec && n % V == 0 && na % V == 0 && (NIN == 1 || nb % V == 0);
    if constexpr (HasFixup<F>::value && sizeof(T) == 4) {
        if (vec && !amod && !bmod) {
            auto kern = ew_staged_f32_kernel<F, NIN>;
            const uint64_t nvec = n / 4;
            int grid = resident_grid(kern, (nvec + STG_UNROLL - 1) / STG_UNROLL);
            launch_k(kern, grid, EW_THREADS, 0, st, reinterpret_cast<const float*>(a),
                     reinterpret_cast<const float*>(b), reinterpret_cast<float*>(out), nvec, n, f);
            return check_launch(name);
        }
    }
    if (vec) {
        if (!amod && !bmod) launch_vec<T, F, NIN, false, false>(a, na, b, nb, out, n, f, st);
        else if (!amod && bmod) launch_vec<T, F, NIN, false, true>(a, na, b, nb, out, n, f, st);
        else if (amod && !bmod) launch_vec<T, F, NIN, true, false>(a, na, b, nb, out, n, f, st);
        else launch_vec<T, F, NIN, true, true>(a, na, b, nb, out, n, f, st);
    } else {
        auto kern = ew_scalar_kernel<T, F, NIN>;
        int grid = resident_grid(kern, n);
        launch_k(kern, grid, EW_THREADS, 0, st, a, na, b, nb, out, n, f);
    }
    return check_launch(name);
}

template <typename T>
static int binary_entry(const char* name, int op, const T* a, uint64_t na, const T* b,
                        uint64_t nb, T* out, uint64_t n, cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(op >= OXIDE_ADD && op <= OXIDE_DIV, name, "unknown binary operator");
    if (n == 0) return OXIDE_OK;
    OXIDE_REQUIRE(a && b && out, name, "null pointer");
    OXIDE_REQUIRE(na >= 1 && nb >= 1 && na <= n && nb <= n, name,
                  "operand lengths must be in [1, n]");
    // The reference's broadcast_shape (matmul.rs:160-177) only admits operands
    // whose length divides the output; out[i] reads a[i % na], b[i % nb].
    OXIDE_REQUIRE(n % na == 0 && n % nb == 0, name,
                  "operand lengths must divide the output length");
    switch (op) {
        case OXIDE_ADD: return ew_dispatch<T, FBin<OXIDE_ADD>, 2>(name, a, na, b, nb, out, n, {}, st);
        case OXIDE_SUB: return ew_dispatch<T, FBin<OXIDE_SUB>, 2>(name, a, na, b, nb, out, n, {}, st);
        case OXIDE_MUL: return ew_dispatch<T, FBin<OXIDE_MUL>, 2>(name, a, na, b, nb, out, n, {}, st);
        default: return ew_dispatch<T, FBin<OXIDE_DIV>, 2>(name, a, na, b, nb, out, n, {}, st);
    }
}

template <typename T>
static int rowbcast_entry(const char* name, const T* x, const T* s, T* out, uint64_t rows,
                          uint64_t cols, cudaStream_t st) {
    OXIDE_INJECT(name);
    if (rows == 0 || cols == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && s && out, name, "null pointer");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    const uint64_t n = rows * cols;
    return ew_dispatch<T, FBin<OXIDE_MUL>, 2>(name, x, n, s, cols, out, n, {}, st);
}

// ---- (a + b) * s[col]: residual add then row-broadcast multiply in one pass ----
// The sum is rounded to T before the product (the add's output, exact for
// f32's own rounding), so the result equals oxide_add_* then
// oxide_mul_rowbcast_* bit for bit.  Three operands, so not the two-input
// template: the same persistent grid and vectors in flight per thread.
template <typename T>
__global__ void __launch_bounds__(EW_THREADS, ew_min_blocks<T>())
    add_mul_vec_kernel(const T* a, const T* b, const T* s, T* out, uint64_t nvec, uint64_t nsv, FastDiv sdiv,
                       bool wide) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    constexpr int U = 4;  // vectors in flight per operand
    const uint64_t stride = (uint64_t)gridDim.x * EW_THREADS;
    for (uint64_t base = (uint64_t)blockIdx.x * EW_THREADS + threadIdx.x; base < nvec; base += stride * U) {
        uint4 va[U], vb[U], vs[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint64_t i = base + k * stride;
            if (i < nvec) {
                const uint64_t is = wide ? i % nsv : sdiv.mod((uint32_t)i);
                va[k] = ld_stream(a + i * V);
                vb[k] = ld_stream(b + i * V);
                vs[k] = ld_keep(s + is * V);
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint64_t i = base + k * stride;
            if (i < nvec) {
                float x[V], y[V], z[V];
                Vec<T>::unpack(va[k], x);
                Vec<T>::unpack(vb[k], y);
                Vec<T>::unpack(vs[k], z);
#pragma unroll
                for (int e = 0; e < V; ++e) x[e] = fmul(Vec<T>::rnd(fadd(x[e], y[e])), z[e]);
                st_stream(out + i * V, Vec<T>::pack(x));
            }
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(EW_THREADS)
    add_mul_scalar_kernel(const T* a, const T* b, const T* s, T* out, uint64_t n, uint64_t cols) {
    pdl_begin();
    const uint64_t stride = (uint64_t)gridDim.x * EW_THREADS;
    for (uint64_t i = (uint64_t)blockIdx.x * EW_THREADS + threadIdx.x; i < n; i += stride) {
        const float h = Vec<T>::rnd(fadd(Vec<T>::load1(a + i), Vec<T>::load1(b + i)));
        Vec<T>::store1(out + i, fmul(h, Vec<T>::load1(s + i % cols)));
    }
}

template <typename T>
static int add_mul_entry(const char* name, const T* a, const T* b, const T* s, T* out, uint64_t rows,
                         uint64_t cols, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    OXIDE_INJECT(name);
    if (rows == 0 || cols == 0) return OXIDE_OK;
    OXIDE_REQUIRE(a && b && s && out, name, "null pointer");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    const uint64_t n = rows * cols;
    if (cols % V == 0 && aligned16(a) && aligned16(b) && aligned16(s) && aligned16(out)) {
        const uint64_t nvec = n / V, nsv = cols / V;
        const bool wide = nvec >= 0xffffffffull;
        auto kern = add_mul_vec_kernel<T>;
        const int grid = resident_grid(kern, (nvec + 3) / 4);
        launch_k(kern, grid, EW_THREADS, 0, st, a, b, s, out, nvec, nsv, FastDiv(wide ? 1u : (uint32_t)nsv), wide);
    } else {
        auto kern = add_mul_scalar_kernel<T>;
        launch_k(kern, resident_grid(kern, n), EW_THREADS, 0, st, a, b, s, out, n, cols);
    }
    return check_launch(name);
}

template <typename T, typename F, int NIN>
static int full_entry(const char* name, const T* a, const T* b, T* out, uint64_t n, F f,
                      cudaStream_t st) {
    OXIDE_INJECT(name);
    if (n == 0) return OXIDE_OK;
    OXIDE_REQUIRE(a && out && (NIN == 1 || b), name, "null pointer");
    return ew_dispatch<T, F, NIN>(name, a, n, NIN == 2 ? b : a, n, out, n, f, st);
}

// Elementwise op over whole tensors (no broadcast): only the aligned-vector and
// the scalar kernel are instantiated.
template <typename T, typename F>
static int unary_dispatch(const char* name, const T* x, T* out, uint64_t n, F f, cudaStream_t st) {
    if (aligned16(x) && aligned16(out)) {
        launch_vec<T, F, 1, false, false>(x, n, x, n, out, n, f, st);
    } else {
        auto kern = ew_scalar_kernel<T, F, 1>;
        launch_k(kern, resident_grid(kern, n), EW_THREADS, 0, st, x, n, x, n, out, n, f);
    }
    return check_launch(name);
}

template <typename T>
static int unary_entry(const char* name, int op, const T* x, T* out, uint64_t n, float a, float b,
                       cudaStream_t st) {
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(op >= OXIDE_RELU && op <= OXIDE_ABS, name, "unknown unary operator");
    // f32::clamp asserts min <= max (neither NaN)
    OXIDE_REQUIRE(op != OXIDE_CLAMP || a <= b, name, "clamp requires min <= max");
    if (n == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && out, name, "null pointer");
    if (op == OXIDE_GELU) a = sqrtf(2.0f / 3.14159265358979323846f);  // (2.0 / PI).sqrt() in f32
    switch (op) {
#define OXIDE_UNARY_CASE(OPV) \
    case OPV: return unary_dispatch<T, FUnary<OPV>>(name, x, out, n, FUnary<OPV>{a, b}, st);
        OXIDE_UNARY_CASE(OXIDE_RELU)
        OXIDE_UNARY_CASE(OXIDE_GELU)
        OXIDE_UNARY_CASE(OXIDE_GELU_QUICK)
        OXIDE_UNARY_CASE(OXIDE_SIGMOID)
        OXIDE_UNARY_CASE(OXIDE_TANH)
        OXIDE_UNARY_CASE(OXIDE_EXP)
        OXIDE_UNARY_CASE(OXIDE_LOG)
        OXIDE_UNARY_CASE(OXIDE_SQRT)
        OXIDE_UNARY_CASE(OXIDE_POW)
        OXIDE_UNARY_CASE(OXIDE_CLAMP)
        OXIDE_UNARY_CASE(OXIDE_NEG)
        OXIDE_UNARY_CASE(OXIDE_ABS)
#undef OXIDE_UNARY_CASE
    }
    return set_error(OXIDE_ERR_INVALID_ARG, "%s: unknown unary operator", name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_unary_f32(int op, const float* x, float* out, uint64_t n, float a, float b,
                    oxide_stream_t stream) {
    return oxide::unary_entry<float>("oxide_unary_f32", op, x, out, n, a, b, stream);
}
int oxide_unary_bf16(int op, const oxide_bf16* x, oxide_bf16* out, uint64_t n, float a, float b,
                     oxide_stream_t stream) {
    return oxide::unary_entry<bf16_t>("oxide_unary_bf16", op, x, out, n, a, b, stream);
}
int oxide_relu_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::unary_entry<float>("oxide_relu_f32", OXIDE_RELU, x, out, n, 0.0f, 0.0f, stream);
}
int oxide_gelu_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::unary_entry<float>("oxide_gelu_f32", OXIDE_GELU, x, out, n, 0.0f, 0.0f, stream);
}
int oxide_sigmoid_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::unary_entry<float>("oxide_sigmoid_f32", OXIDE_SIGMOID, x, out, n, 0.0f, 0.0f,
                                     stream);
}
int oxide_tanh_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::unary_entry<float>("oxide_tanh_f32", OXIDE_TANH, x, out, n, 0.0f, 0.0f, stream);
}

int oxide_binary_f32(int op, const float* a, uint64_t na, const float* b, uint64_t nb,
                     float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::binary_entry<float>("oxide_binary_f32", op, a, na, b, nb, out, n, stream);
}
int oxide_binary_bf16(int op, const oxide_bf16* a, uint64_t na, const oxide_bf16* b,
                      uint64_t nb, oxide_bf16* out, uint64_t n, oxide_stream_t stream) {
    return oxide::binary_entry<bf16_t>("oxide_binary_bf16", op, a, na, b, nb, out, n, stream);
}
int oxide_add_f32(const float* a, const float* b, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::full_entry<float, oxide::FBin<OXIDE_ADD>, 2>("oxide_add_f32", a, b, out, n, {},
                                                                stream);
}
int oxide_add_bf16(const oxide_bf16* a, const oxide_bf16* b, oxide_bf16* out, uint64_t n,
                   oxide_stream_t stream) {
    return oxide::full_entry<bf16_t, oxide::FBin<OXIDE_ADD>, 2>("oxide_add_bf16", a, b, out, n,
                                                                 {}, stream);
}
int oxide_sub_f32(const float* a, const float* b, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::full_entry<float, oxide::FBin<OXIDE_SUB>, 2>("oxide_sub_f32", a, b, out, n, {},
                                                                stream);
}
int oxide_div_f32(const float* a, const float* b, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::full_entry<float, oxide::FBin<OXIDE_DIV>, 2>("oxide_div_f32", a, b, out, n, {},
                                                                stream);
}
int oxide_mul_rowbcast_f32(const float* x, const float* s, float* out, uint64_t rows,
                           uint64_t cols, oxide_stream_t stream) {
    return oxide::rowbcast_entry<float>("oxide_mul_rowbcast_f32", x, s, out, rows, cols, stream);
}
int oxide_mul_rowbcast_bf16(const oxide_bf16* x, const oxide_bf16* s, oxide_bf16* out,
                            uint64_t rows, uint64_t cols, oxide_stream_t stream) {
    return oxide::rowbcast_entry<bf16_t>("oxide_mul_rowbcast_bf16", x, s, out, rows, cols,
                                         stream);
}
int oxide_add_mul_rowbcast_f32(const float* a, const float* b, const float* s, float* out, uint64_t rows,
                               uint64_t cols, oxide_stream_t stream) {
    return oxide::add_mul_entry<float>("oxide_add_mul_rowbcast_f32", a, b, s, out, rows, cols, stream);
}
int oxide_add_mul_rowbcast_bf16(const oxide_bf16* a, const oxide_bf16* b, const oxide_bf16* s, oxide_bf16* out,
                                uint64_t rows, uint64_t cols, oxide_stream_t stream) {
    return oxide::add_mul_entry<bf16_t>("oxide_add_mul_rowbcast_bf16", a, b, s, out, rows, cols, stream);
}
int oxide_scale_f32(const float* x, float* out, float scale, uint64_t n, oxide_stream_t stream) {
    return oxide::full_entry<float, oxide::FScale, 1>("oxide_scale_f32", x, nullptr, out, n,
                                                      oxide::FScale{scale}, stream);
}
int oxide_scale_bf16(const oxide_bf16* x, oxide_bf16* out, float scale, uint64_t n,
                     oxide_stream_t stream) {
    return oxide::full_entry<bf16_t, oxide::FScale, 1>("oxide_scale_bf16", x, nullptr, out, n,
                                                       oxide::FScale{scale}, stream);
}
int oxide_silu_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream) {
    return oxide::full_entry<float, oxide::FSilu<float>, 1>("oxide_silu_f32", x, nullptr, out, n, {},
                                                     stream);
}
int oxide_silu_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t n, oxide_stream_t stream) {
    return oxide::full_entry<bf16_t, oxide::FSilu<bf16_t>, 1>("oxide_silu_bf16", x, nullptr, out, n, {},
                                                      stream);
}
int oxide_silu_mul_f32(const float* gate, const float* up, float* out, uint64_t n,
                       oxide_stream_t stream) {
    return oxide::full_entry<float, oxide::FSiluMul<float>, 2>("oxide_silu_mul_f32", gate, up,
                                                               out, n, {}, stream);
}
int oxide_silu_mul_bf16(const oxide_bf16* gate, const oxide_bf16* up, oxide_bf16* out,
                        uint64_t n, oxide_stream_t stream) {
    return oxide::full_entry<bf16_t, oxide::FSiluMul<bf16_t>, 2>("oxide_silu_mul_bf16", gate, up,
                                                                 out, n, {}, stream);
}

}  // extern "C"
