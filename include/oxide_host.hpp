// oxide_host.hpp -- C++ host layer over the C ABI (oxide_ops.h), mirroring the
// Rust interface of mistralrs-oxide that the tensor-op path sits behind:
//
//   oxide::OxideError / OxideResult      src/error.rs:3-47
//   oxide::Shape, DType, Tensor          src/core/dtype.rs:9,70-181, src/core/tensor.rs:29
//   oxide::ops::{add, sub, mul, div,     src/ops/matmul.rs:74-177
//                relu, silu, gelu, gelu_quick, softmax, sigmoid, tanh
//                                        src/ops/activation.rs
//                exp, log, sqrt, pow, clamp, neg, abs
//                                        src/ops/math.rs
//                rms_norm, layer_norm,   src/ops/norm.rs:4-117
//                apply_rotary_emb}       src/ops/attention.rs:96-159
//   oxide::precompute_rope_cache         src/models/mistral.rs:91-115
//   oxide::CudaBackend                   src/cuda_backend/mod.rs:43-140
//   oxide::KernelManager::launch_*       src/cuda_backend/kernels.rs:75-376
//
// plus the path's additions (silu_mul, add_rms_norm, scale_mask_softmax, rope
// of q and k in one launch, argmax, sum / max / sum of squares, bf16 tensors).
//
// Semantics follow the Rust originals: every op borrows its inputs and returns
// a newly allocated output tensor (Tensor::zeros) or an OxideError; shape
// errors are InvalidArgument with the reference's message.  Tensors live in
// device memory (the reference's CPU storage is replaced by the device); the
// ops enqueue one kernel on the calling thread's current stream (default: the
// legacy default stream, like cudarc's) and do not synchronise, except where a
// result is returned to the host (to_vec, the scalar reductions).
//
// Header-only; link liboxide_b200.so and the CUDA runtime.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <algorithm>
#include <cstring>
#include <memory>
#include <optional>
#include <sstream>
#include <string>
#include <utility>
#include <variant>
#include <cmath>
#include <vector>

#include "oxide_ops.h"

namespace oxide {

// ---- errors (src/error.rs:3-47) -----------------------------------------------------
struct OxideError {
    enum class Kind {
        ShapeMismatch,
        DtypeMismatch,
        DeviceMismatch,
        CudaError,
        DeviceError,
        UnsupportedOperation,
        InvalidArgument,
        OutOfMemory,
        KernelLaunchError,
    };
    Kind kind;
    std::string message;

    std::string to_string() const {
        switch (kind) {
            case Kind::ShapeMismatch: return "Shape mismatch: " + message;
            case Kind::DtypeMismatch: return "Dtype mismatch: " + message;
            case Kind::DeviceMismatch: return "Device mismatch: " + message;
            case Kind::CudaError: return "CUDA error: " + message;
            case Kind::DeviceError: return "Device error: " + message;
            case Kind::UnsupportedOperation: return "Unsupported operation: " + message;
            case Kind::InvalidArgument: return "Invalid argument: " + message;
            case Kind::OutOfMemory: return "Out of memory: " + message;
            case Kind::KernelLaunchError: return "Kernel launch error: " + message;
        }
        return message;
    }
    static OxideError invalid(std::string m) { return {Kind::InvalidArgument, std::move(m)}; }
    static OxideError cuda(std::string m) { return {Kind::CudaError, std::move(m)}; }
};

// Result<T>: a value or an OxideError (Rust's OxideResult<T>).
template <typename T>
class Result {
  public:
    Result(T v) : v_(std::move(v)) {}                 // NOLINT: implicit like Ok(v)
    Result(OxideError e) : v_(std::move(e)) {}        // NOLINT: implicit like Err(e)
    bool is_ok() const { return v_.index() == 0; }
    bool is_err() const { return !is_ok(); }
    T& value() & { return std::get<0>(v_); }
    T&& value() && { return std::get<0>(std::move(v_)); }
    const T& value() const& { return std::get<0>(v_); }
    const OxideError& error() const { return std::get<1>(v_); }

  private:
    std::variant<T, OxideError> v_;
};

struct Unit {};
using Status = Result<Unit>;
template <typename T>
using OxideResult = Result<T>;

// A non-zero oxide_status as an OxideError of the matching class.
inline OxideError error_from_status(int status) {
    const char* last = oxide_last_error();
    std::string msg = last && *last ? last : oxide_status_string(status);
    switch (status) {
        case OXIDE_ERR_INVALID_ARG:
        case OXIDE_ERR_WORKSPACE: return {OxideError::Kind::InvalidArgument, msg};
        case OXIDE_ERR_UNSUPPORTED: return {OxideError::Kind::UnsupportedOperation, msg};
        case OXIDE_ERR_LAUNCH: return {OxideError::Kind::KernelLaunchError, msg};
        default: return {OxideError::Kind::CudaError, msg};
    }
}
inline Status check_status(int status) {
    if (status == OXIDE_OK) return Unit{};
    return error_from_status(status);
}
inline Status check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return Unit{};
    std::string msg = std::string(what) + ": " + cudaGetErrorString(e);
    if (e == cudaErrorMemoryAllocation) return OxideError{OxideError::Kind::OutOfMemory, msg};
    return OxideError::cuda(msg);
}

#define OXIDE_TRY(expr)                                   \
    do {                                                  \
        auto oxide_try_r_ = (expr);                       \
        if (oxide_try_r_.is_err()) return oxide_try_r_.error(); \
    } while (0)

// ---- stream -------------------------------------------------------------------------
// The stream the ops of this thread enqueue on (nullptr = legacy default stream).
inline cudaStream_t& current_stream() {
    thread_local cudaStream_t s = nullptr;
    return s;
}

// ---- shapes and dtypes (src/core/dtype.rs) -----------------------------------------------
enum class DType { F32, BF16 };
inline size_t dtype_size(DType d) { return d == DType::F32 ? 4 : 2; }
inline const char* dtype_name(DType d) { return d == DType::F32 ? "f32" : "bf16"; }

class Shape {
  public:
    Shape() = default;
    Shape(std::initializer_list<size_t> d) : dims_(d) {}
    explicit Shape(std::vector<size_t> d) : dims_(std::move(d)) {}
    const std::vector<size_t>& dims() const { return dims_; }
    size_t rank() const { return dims_.size(); }
    size_t elem_count() const {
        size_t n = 1;
        for (size_t d : dims_) n *= d;
        return n;
    }
    bool operator==(const Shape& o) const { return dims_ == o.dims_; }
    bool operator!=(const Shape& o) const { return dims_ != o.dims_; }
    std::string to_string() const { return dims_string(dims_); }
    static std::string dims_string(const std::vector<size_t>& d) {
        std::ostringstream s;
        s << '[';
        for (size_t i = 0; i < d.size(); ++i) s << (i ? ", " : "") << d[i];
        s << ']';
        return s.str();
    }

  private:
    std::vector<size_t> dims_;
};

// ---- device memory ------------------------------------------------------------------------
class DeviceBuffer {
  public:
    static Result<std::shared_ptr<DeviceBuffer>> allocate(size_t bytes, int device) {
        OXIDE_TRY(check_cuda(cudaSetDevice(device), "cudaSetDevice"));
        void* p = nullptr;
        if (bytes) OXIDE_TRY(check_cuda(cudaMalloc(&p, bytes), "cudaMalloc"));
        return std::shared_ptr<DeviceBuffer>(new DeviceBuffer(p, bytes, device));
    }
    ~DeviceBuffer() {
        if (ptr_) cudaFree(ptr_);
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    void* ptr() const { return ptr_; }
    size_t bytes() const { return bytes_; }
    int device() const { return device_; }

  private:
    DeviceBuffer(void* p, size_t b, int d) : ptr_(p), bytes_(b), device_(d) {}
    void* ptr_;
    size_t bytes_;
    int device_;
};

// ---- tensor (src/core/tensor.rs) -------------------------------------------------------------
// Contiguous row-major device tensor; copies share storage like the Rust
// Tensor's Arc<Storage>.
class Tensor {
  public:
    static Result<Tensor> empty(const Shape& shape, DType dtype, int device = 0) {
        auto buf = DeviceBuffer::allocate(shape.elem_count() * dtype_size(dtype), device);
        if (buf.is_err()) return buf.error();
        return Tensor(shape, dtype, std::move(buf).value());
    }
    // Tensor::zeros (src/core/tensor.rs:29)
    static Result<Tensor> zeros(const Shape& shape, DType dtype, int device = 0) {
        auto t = empty(shape, dtype, device);
        if (t.is_err() || !t.value().nbytes()) return t;
        OXIDE_TRY(check_cuda(cudaMemsetAsync(t.value().data(), 0, t.value().nbytes(), current_stream()),
                             "cudaMemsetAsync"));
        return t;
    }
    static Result<Tensor> from_f32(const std::vector<float>& host, const Shape& shape, int device = 0) {
        return from_bytes(host.data(), host.size(), shape, DType::F32, device);
    }
    // bf16 tensor from raw 16-bit patterns.
    static Result<Tensor> from_bf16_bits(const std::vector<uint16_t>& host, const Shape& shape,
                                         int device = 0) {
        return from_bytes(host.data(), host.size(), shape, DType::BF16, device);
    }

    const Shape& shape() const { return shape_; }
    const std::vector<size_t>& dims() const { return shape_.dims(); }
    size_t rank() const { return shape_.rank(); }
    size_t elem_count() const { return shape_.elem_count(); }
    DType dtype() const { return dtype_; }
    int device() const { return buf_->device(); }
    size_t nbytes() const { return elem_count() * dtype_size(dtype_); }
    void* data() const { return buf_->ptr(); }
    template <typename T>
    T* as() const { return static_cast<T*>(buf_->ptr()); }

    // Waits for the current stream, then copies to the host.
    template <typename T>
    Result<std::vector<T>> to_vec() const {
        if (sizeof(T) != dtype_size(dtype_))
            return OxideError{OxideError::Kind::DtypeMismatch,
                              std::string("to_vec element size differs from ") + dtype_name(dtype_)};
        std::vector<T> out(elem_count());
        if (!out.empty()) {
            OXIDE_TRY(check_cuda(cudaMemcpyAsync(out.data(), data(), nbytes(), cudaMemcpyDeviceToHost,
                                                 current_stream()), "cudaMemcpyAsync"));
            OXIDE_TRY(check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize"));
        }
        return out;
    }
    // A view of the same storage with another shape of the same element count.
    Result<Tensor> reshape(const Shape& s) const {
        if (s.elem_count() != elem_count())
            return OxideError::invalid("reshape " + shape_.to_string() + " -> " + s.to_string());
        return Tensor(s, dtype_, buf_);
    }

  private:
    Tensor(Shape s, DType d, std::shared_ptr<DeviceBuffer> b)
        : shape_(std::move(s)), dtype_(d), buf_(std::move(b)) {}
    static Result<Tensor> from_bytes(const void* host, size_t n, const Shape& shape, DType dtype,
                                     int device) {
        if (n != shape.elem_count())
            return OxideError{OxideError::Kind::ShapeMismatch,
                              "data has " + std::to_string(n) + " elements, shape " + shape.to_string()};
        auto t = empty(shape, dtype, device);
        if (t.is_err() || !n) return t;
        OXIDE_TRY(check_cuda(cudaMemcpyAsync(t.value().data(), host, t.value().nbytes(),
                                             cudaMemcpyHostToDevice, current_stream()),
                             "cudaMemcpyAsync"));
        OXIDE_TRY(check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize"));
        return t;
    }

    Shape shape_;
    DType dtype_;
    std::shared_ptr<DeviceBuffer> buf_;
};

// ---- ops (src/ops) ---------------------------------------------------------------------------
namespace ops {
namespace detail {
inline Status same_dtype(const Tensor& a, const Tensor& b, const char* op) {
    if (a.dtype() != b.dtype())
        return OxideError{OxideError::Kind::DtypeMismatch,
                          std::string(op) + ": expected " + dtype_name(a.dtype()) + ", got " +
                              dtype_name(b.dtype())};
    return Unit{};
}
inline Status same_device(const Tensor& a, const Tensor& b, const char* op) {
    if (a.device() != b.device())
        return OxideError{OxideError::Kind::DeviceMismatch,
                          std::string(op) + ": tensors on cuda:" + std::to_string(a.device()) +
                              " and cuda:" + std::to_string(b.device())};
    return Unit{};
}
inline bool bf16(const Tensor& t) { return t.dtype() == DType::BF16; }
}  // namespace detail

// Output shape of a binary op (src/ops/matmul.rs:160-177).
inline Result<std::vector<size_t>> broadcast_shape(const std::vector<size_t>& a,
                                                   const std::vector<size_t>& b) {
    const size_t r = a.size() > b.size() ? a.size() : b.size();
    std::vector<size_t> out(r);
    for (size_t i = 0; i < r; ++i) {
        const size_t da = i < a.size() ? a[a.size() - 1 - i] : 1;
        const size_t db = i < b.size() ? b[b.size() - 1 - i] : 1;
        if (da != db && da != 1 && db != 1)
            return OxideError::invalid("broadcast: shape mismatch " + Shape::dims_string(a) + " and " +
                                       Shape::dims_string(b));
        out[r - 1 - i] = da > db ? da : db;
    }
    return out;
}

// out[i] = a[i % |a|] op b[i % |b|] (src/ops/matmul.rs:136-158).
inline Result<Tensor> binary(int op, const Tensor& a, const Tensor& b) {
    OXIDE_TRY(detail::same_dtype(a, b, "binary"));
    OXIDE_TRY(detail::same_device(a, b, "binary"));
    auto shape = broadcast_shape(a.dims(), b.dims());
    if (shape.is_err()) return shape.error();
    auto out = Tensor::empty(Shape(shape.value()), a.dtype(), a.device());
    if (out.is_err()) return out;
    const Tensor& o = out.value();
    const int rc = detail::bf16(a)
        ? oxide_binary_bf16(op, a.as<oxide_bf16>(), a.elem_count(), b.as<oxide_bf16>(), b.elem_count(),
                            o.as<oxide_bf16>(), o.elem_count(), current_stream())
        : oxide_binary_f32(op, a.as<float>(), a.elem_count(), b.as<float>(), b.elem_count(),
                           o.as<float>(), o.elem_count(), current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}
inline Result<Tensor> add(const Tensor& a, const Tensor& b) { return binary(OXIDE_ADD, a, b); }
inline Result<Tensor> sub(const Tensor& a, const Tensor& b) { return binary(OXIDE_SUB, a, b); }
inline Result<Tensor> mul(const Tensor& a, const Tensor& b) { return binary(OXIDE_MUL, a, b); }
inline Result<Tensor> div(const Tensor& a, const Tensor& b) { return binary(OXIDE_DIV, a, b); }

// x * s (KernelManager::launch_scale, src/cuda_backend/kernels.rs:159-177).
inline Result<Tensor> scale(const Tensor& x, float s) {
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(x)
        ? oxide_scale_bf16(x.as<oxide_bf16>(), out.value().as<oxide_bf16>(), s, x.elem_count(),
                           current_stream())
        : oxide_scale_f32(x.as<float>(), out.value().as<float>(), s, x.elem_count(), current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// silu (src/ops/activation.rs:21-37).
inline Result<Tensor> silu(const Tensor& x) {
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(x)
        ? oxide_silu_bf16(x.as<oxide_bf16>(), out.value().as<oxide_bf16>(), x.elem_count(),
                          current_stream())
        : oxide_silu_f32(x.as<float>(), out.value().as<float>(), x.elem_count(), current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// Unary ops of src/ops/activation.rs (relu, gelu, gelu_quick, sigmoid, tanh)
// and src/ops/math.rs (exp, log, sqrt, pow, clamp, neg, abs): op is an
// oxide_unop; a = pow exponent or clamp minimum, b = clamp maximum.
inline Result<Tensor> unary(int op, const Tensor& x, float a = 0.0f, float b = 0.0f) {
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(x)
        ? oxide_unary_bf16(op, x.as<oxide_bf16>(), out.value().as<oxide_bf16>(), x.elem_count(), a, b,
                           current_stream())
        : oxide_unary_f32(op, x.as<float>(), out.value().as<float>(), x.elem_count(), a, b,
                          current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}
inline Result<Tensor> relu(const Tensor& x) { return unary(OXIDE_RELU, x); }
inline Result<Tensor> gelu(const Tensor& x) { return unary(OXIDE_GELU, x); }
inline Result<Tensor> gelu_quick(const Tensor& x) { return unary(OXIDE_GELU_QUICK, x); }
inline Result<Tensor> sigmoid(const Tensor& x) { return unary(OXIDE_SIGMOID, x); }
inline Result<Tensor> tanh(const Tensor& x) { return unary(OXIDE_TANH, x); }
inline Result<Tensor> exp(const Tensor& x) { return unary(OXIDE_EXP, x); }
inline Result<Tensor> log(const Tensor& x) { return unary(OXIDE_LOG, x); }
inline Result<Tensor> sqrt(const Tensor& x) { return unary(OXIDE_SQRT, x); }
inline Result<Tensor> pow(const Tensor& x, float n) { return unary(OXIDE_POW, x, n); }
inline Result<Tensor> clamp(const Tensor& x, float lo, float hi) { return unary(OXIDE_CLAMP, x, lo, hi); }
inline Result<Tensor> neg(const Tensor& x) { return unary(OXIDE_NEG, x); }
inline Result<Tensor> abs(const Tensor& x) { return unary(OXIDE_ABS, x); }

// mul(silu(gate), up) in one pass (MLP::forward, src/layers/attention.rs:144-145).
inline Result<Tensor> silu_mul(const Tensor& gate, const Tensor& up) {
    OXIDE_TRY(detail::same_dtype(gate, up, "silu_mul"));
    OXIDE_TRY(detail::same_device(gate, up, "silu_mul"));
    if (gate.shape() != up.shape())
        return OxideError{OxideError::Kind::ShapeMismatch,
                          "silu_mul: gate " + gate.shape().to_string() + ", up " + up.shape().to_string()};
    auto out = Tensor::empty(gate.shape(), gate.dtype(), gate.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(gate)
        ? oxide_silu_mul_bf16(gate.as<oxide_bf16>(), up.as<oxide_bf16>(), out.value().as<oxide_bf16>(),
                              gate.elem_count(), current_stream())
        : oxide_silu_mul_f32(gate.as<float>(), up.as<float>(), out.value().as<float>(),
                             gate.elem_count(), current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

namespace detail {
// Argument checks of src/ops/norm.rs:5-19; returns the row length.
inline Result<size_t> norm_cols(const Tensor& x, const Tensor& w) {
    if (x.rank() < 1) return OxideError::invalid("rms_norm requires at least 1D tensor");
    const size_t last = x.dims().back();
    if (w.rank() != 1 || w.dims()[0] != last)
        return OxideError::invalid("rms_norm weight shape " + w.shape().to_string() +
                                   " doesn't match input last dim " + std::to_string(last));
    OXIDE_TRY(same_dtype(x, w, "rms_norm"));
    return last;
}
}  // namespace detail

// rms_norm (src/ops/norm.rs:4-51).
inline Result<Tensor> rms_norm(const Tensor& x, const Tensor& w, float eps) {
    auto cols = detail::norm_cols(x, w);
    if (cols.is_err()) return cols.error();
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const size_t c = cols.value(), rows = c ? x.elem_count() / c : 0;
    const int rc = detail::bf16(x)
        ? oxide_rms_norm_bf16(x.as<oxide_bf16>(), w.as<oxide_bf16>(), out.value().as<oxide_bf16>(), rows,
                              c, eps, current_stream())
        : oxide_rms_norm_f32(x.as<float>(), w.as<float>(), out.value().as<float>(), rows, c, eps,
                             current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// layer_norm (src/ops/norm.rs:53-117), with the reference's argument checks.
inline Result<Tensor> layer_norm(const Tensor& x, const Tensor& w, const Tensor& b, float eps) {
    if (x.rank() < 1) return OxideError::invalid("layer_norm requires at least 1D tensor");
    const size_t last = x.dims().back();
    if (w.rank() != 1 || w.dims()[0] != last)
        return OxideError::invalid("layer_norm weight shape " + w.shape().to_string() +
                                   " doesn't match input last dim " + std::to_string(last));
    if (b.rank() != 1 || b.dims()[0] != last)
        return OxideError::invalid("layer_norm bias shape " + b.shape().to_string() +
                                   " doesn't match input last dim " + std::to_string(last));
    OXIDE_TRY(detail::same_dtype(x, w, "layer_norm"));
    OXIDE_TRY(detail::same_dtype(x, b, "layer_norm"));
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const size_t rows = last ? x.elem_count() / last : 0;
    const int rc = detail::bf16(x)
        ? oxide_layer_norm_bf16(x.as<oxide_bf16>(), w.as<oxide_bf16>(), b.as<oxide_bf16>(),
                                out.value().as<oxide_bf16>(), rows, last, eps, current_stream())
        : oxide_layer_norm_f32(x.as<float>(), w.as<float>(), b.as<float>(), out.value().as<float>(), rows,
                               last, eps, current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// repeat_kv (src/ops/attention.rs:161-201): [b, kv_heads, s, d] -> [b, kv_heads * n_rep, s, d].
inline Result<Tensor> repeat_kv(const Tensor& x, size_t n_rep) {
    if (x.rank() < 4)
        return OxideError::invalid("repeat_kv requires 4D tensor (batch, heads, seq_len, head_dim)");
    std::vector<size_t> d = x.dims();
    const size_t b = d[0], h = d[1], s = d[2], hd = (b && h && s) ? x.elem_count() / (b * h * s) : 0;
    d[1] *= n_rep;
    auto out = Tensor::empty(Shape(d), x.dtype(), x.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(x)
        ? oxide_repeat_kv_bf16(x.as<oxide_bf16>(), out.value().as<oxide_bf16>(), b, h, s, hd, n_rep,
                               current_stream())
        : oxide_repeat_kv_f32(x.as<float>(), out.value().as<float>(), b, h, s, hd, n_rep, current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// (h, y): h = x + r, y = rms_norm(h) (src/layers/transformer.rs:64-67).
inline Result<std::pair<Tensor, Tensor>> add_rms_norm(const Tensor& x, const Tensor& r,
                                                      const Tensor& w, float eps) {
    auto cols = detail::norm_cols(x, w);
    if (cols.is_err()) return cols.error();
    if (x.shape() != r.shape())
        return OxideError{OxideError::Kind::ShapeMismatch,
                          "add_rms_norm: x " + x.shape().to_string() + ", residual " + r.shape().to_string()};
    OXIDE_TRY(detail::same_dtype(x, r, "add_rms_norm"));
    auto h = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (h.is_err()) return h.error();
    auto y = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (y.is_err()) return y.error();
    const size_t c = cols.value(), rows = c ? x.elem_count() / c : 0;
    const int rc = detail::bf16(x)
        ? oxide_add_rms_norm_bf16(x.as<oxide_bf16>(), r.as<oxide_bf16>(), w.as<oxide_bf16>(),
                                  h.value().as<oxide_bf16>(), y.value().as<oxide_bf16>(), rows, c, eps,
                                  current_stream())
        : oxide_add_rms_norm_f32(x.as<float>(), r.as<float>(), w.as<float>(), h.value().as<float>(),
                                 y.value().as<float>(), rows, c, eps, current_stream());
    OXIDE_TRY(check_status(rc));
    return std::make_pair(std::move(h).value(), std::move(y).value());
}

// softmax along `dim` (src/ops/activation.rs:76-124).
inline Result<Tensor> softmax(const Tensor& x, size_t dim) {
    if (dim >= x.rank())
        return OxideError::invalid("softmax dim " + std::to_string(dim) + " out of range for rank " +
                                   std::to_string(x.rank()));
    size_t outer = 1, inner = 1;
    for (size_t i = 0; i < dim; ++i) outer *= x.dims()[i];
    for (size_t i = dim + 1; i < x.rank(); ++i) inner *= x.dims()[i];
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(x)
        ? oxide_softmax_bf16(x.as<oxide_bf16>(), out.value().as<oxide_bf16>(), outer, x.dims()[dim],
                             inner, current_stream())
        : oxide_softmax_f32(x.as<float>(), out.value().as<float>(), outer, x.dims()[dim], inner,
                            current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// Options of scale_mask_softmax: the additive mask and the per-row valid
// length (per-sequence KV lengths and/or a causal block of q_len rows).
struct MaskOptions {
    const Tensor* mask = nullptr;  // f32, added as mask[j % mask.elem_count()]
    const int32_t* lens = nullptr; // device int32, one per group of rows_per_len rows
    size_t rows_per_len = 1;
    size_t causal_q_len = 0;
};

// softmax(x * scale + mask) over the last dim: the scale/mask/softmax block of
// scaled_dot_product_attention (src/ops/attention.rs:41,60,63-79).
inline Result<Tensor> scale_mask_softmax(const Tensor& x, float scale, const MaskOptions& m = {}) {
    if (x.rank() < 1) return OxideError::invalid("scale_mask_softmax requires at least 1D tensor");
    if (m.mask && m.mask->dtype() != DType::F32)
        return OxideError{OxideError::Kind::DtypeMismatch, "scale_mask_softmax: mask must be f32"};
    const size_t cols = x.dims().back(), rows = cols ? x.elem_count() / cols : 0;
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const float* mp = m.mask ? m.mask->as<float>() : nullptr;
    const size_t ml = m.mask ? m.mask->elem_count() : 0;
    const int rc = detail::bf16(x)
        ? oxide_scale_mask_softmax_bf16(x.as<oxide_bf16>(), out.value().as<oxide_bf16>(), rows, cols,
                                        scale, mp, ml, m.lens, m.rows_per_len, m.causal_q_len,
                                        current_stream())
        : oxide_scale_mask_softmax_f32(x.as<float>(), out.value().as<float>(), rows, cols, scale, mp,
                                       ml, m.lens, m.rows_per_len, m.causal_q_len, current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// apply_rotary_emb (src/ops/attention.rs:96-159): x [..., seq_len, head_dim]
// head-major, cos/sin f32 [seq_len, head_dim/2], position = sequence index.
inline Result<Tensor> apply_rotary_emb(const Tensor& x, const Tensor& cos, const Tensor& sin) {
    if (x.rank() < 3) return OxideError::invalid("apply_rotary_emb requires at least 3D tensor");
    const size_t seq_len = x.dims()[x.rank() - 2], head_dim = x.dims().back(), half = head_dim / 2;
    const std::vector<size_t> want = {seq_len, half};
    if (cos.dims() != want)
        return OxideError::invalid("cos shape " + cos.shape().to_string() + " doesn't match expected " +
                                   Shape::dims_string(want));
    if (sin.dims() != want)
        return OxideError::invalid("sin shape " + sin.shape().to_string() + " doesn't match expected " +
                                   Shape::dims_string(want));
    if (cos.dtype() != DType::F32 || sin.dtype() != DType::F32)
        return OxideError{OxideError::Kind::DtypeMismatch, "apply_rotary_emb: cos/sin must be f32"};
    auto out = Tensor::empty(x.shape(), x.dtype(), x.device());
    if (out.is_err()) return out;
    const size_t heads = (seq_len && head_dim) ? x.elem_count() / (seq_len * head_dim) : 0;
    const int rc = detail::bf16(x)
        ? oxide_rope_bf16(x.as<oxide_bf16>(), out.value().as<oxide_bf16>(), heads, nullptr, nullptr, 0,
                          cos.as<float>(), sin.as<float>(), seq_len, nullptr, seq_len, head_dim, 1,
                          current_stream())
        : oxide_rope_f32(x.as<float>(), out.value().as<float>(), heads, nullptr, nullptr, 0,
                         cos.as<float>(), sin.as<float>(), seq_len, nullptr, seq_len, head_dim, 1,
                         current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// q and k of MultiHeadAttention::forward (src/layers/attention.rs:88-94) in
// one launch, token-major [tokens, heads, head_dim], positions (device int32,
// may be null: position = token index) indexing the cos/sin tables.
inline Result<std::pair<Tensor, Tensor>> rope_qk(const Tensor& q, const Tensor& k, const Tensor& cos,
                                                 const Tensor& sin, const int32_t* positions = nullptr) {
    if (q.rank() != 3 || k.rank() != 3 || q.dims()[0] != k.dims()[0] || q.dims()[2] != k.dims()[2])
        return OxideError::invalid("rope_qk: q " + q.shape().to_string() + " and k " + k.shape().to_string() +
                                   " must be [tokens, heads, head_dim] with equal tokens and head_dim");
    OXIDE_TRY(detail::same_dtype(q, k, "rope_qk"));
    const size_t head_dim = q.dims()[2];
    if (cos.rank() != 2 || cos.dims()[1] != head_dim / 2 || cos.shape() != sin.shape())
        return OxideError::invalid("rope_qk: cos/sin shape " + cos.shape().to_string() +
                                   " doesn't match [*, " + std::to_string(head_dim / 2) + "]");
    auto qo = Tensor::empty(q.shape(), q.dtype(), q.device());
    if (qo.is_err()) return qo.error();
    auto ko = Tensor::empty(k.shape(), k.dtype(), k.device());
    if (ko.is_err()) return ko.error();
    const int rc = detail::bf16(q)
        ? oxide_rope_bf16(q.as<oxide_bf16>(), qo.value().as<oxide_bf16>(), q.dims()[1], k.as<oxide_bf16>(),
                          ko.value().as<oxide_bf16>(), k.dims()[1], cos.as<float>(), sin.as<float>(),
                          cos.dims()[0], positions, q.dims()[0], head_dim, 0, current_stream())
        : oxide_rope_f32(q.as<float>(), qo.value().as<float>(), q.dims()[1], k.as<float>(),
                         ko.value().as<float>(), k.dims()[1], cos.as<float>(), sin.as<float>(),
                         cos.dims()[0], positions, q.dims()[0], head_dim, 0, current_stream());
    OXIDE_TRY(check_status(rc));
    return std::make_pair(std::move(qo).value(), std::move(ko).value());
}

// Row argmax over the last dim -> u32 indices (a tensor of shape dims[:-1],
// returned as raw u32 on the host side through to_vec<uint32_t>()).
inline Result<std::vector<uint32_t>> argmax(const Tensor& x) {
    if (x.rank() < 1) return OxideError::invalid("argmax requires at least 1D tensor");
    const size_t cols = x.dims().back(), rows = cols ? x.elem_count() / cols : 0;
    auto idx = DeviceBuffer::allocate(rows * sizeof(uint32_t), x.device());
    if (idx.is_err()) return idx.error();
    uint32_t* ip = static_cast<uint32_t*>(idx.value()->ptr());
    const int rc = detail::bf16(x)
        ? oxide_argmax_rows_bf16(x.as<oxide_bf16>(), rows, cols, ip, current_stream())
        : oxide_argmax_rows_f32(x.as<float>(), rows, cols, ip, current_stream());
    OXIDE_TRY(check_status(rc));
    std::vector<uint32_t> host(rows);
    if (rows) {
        OXIDE_TRY(check_cuda(cudaMemcpyAsync(host.data(), ip, rows * 4, cudaMemcpyDeviceToHost,
                                             current_stream()), "cudaMemcpyAsync"));
        OXIDE_TRY(check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize"));
    }
    return host;
}

// Whole-tensor sum / max / sum of squares (f64), returned to the host.
inline Result<double> reduce(const Tensor& x, int op) {
    auto ws = DeviceBuffer::allocate(oxide_reduce_workspace_bytes(x.elem_count()) + sizeof(double),
                                     x.device());
    if (ws.is_err()) return ws.error();
    char* base = static_cast<char*>(ws.value()->ptr());
    double* out = reinterpret_cast<double*>(base);
    void* scratch = base + sizeof(double);
    const uint64_t sb = oxide_reduce_workspace_bytes(x.elem_count());
    const int rc = detail::bf16(x)
        ? oxide_reduce_bf16(op, x.as<oxide_bf16>(), x.elem_count(), out, scratch, sb, current_stream())
        : oxide_reduce_f32(op, x.as<float>(), x.elem_count(), out, scratch, sb, current_stream());
    OXIDE_TRY(check_status(rc));
    double v = 0;
    OXIDE_TRY(check_cuda(cudaMemcpyAsync(&v, out, sizeof v, cudaMemcpyDeviceToHost, current_stream()),
                         "cudaMemcpyAsync"));
    OXIDE_TRY(check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize"));
    return v;
}
inline Result<double> sum(const Tensor& x) { return reduce(x, OXIDE_RED_SUM); }
inline Result<double> max(const Tensor& x) { return reduce(x, OXIDE_RED_MAX); }
inline Result<double> sum_sq(const Tensor& x) { return reduce(x, OXIDE_RED_SUMSQ); }

// Per-row sum / max / sum of squares over the last dim -> f32 tensor dims[:-1].
inline Result<Tensor> reduce_rows(const Tensor& x, int op) {
    if (x.rank() < 1) return OxideError::invalid("reduce_rows requires at least 1D tensor");
    const size_t cols = x.dims().back(), rows = cols ? x.elem_count() / cols : 0;
    std::vector<size_t> od(x.dims().begin(), x.dims().end() - 1);
    auto out = Tensor::empty(Shape(od), DType::F32, x.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(x)
        ? oxide_reduce_rows_bf16(op, x.as<oxide_bf16>(), rows, cols, out.value().as<float>(),
                                 current_stream())
        : oxide_reduce_rows_f32(op, x.as<float>(), rows, cols, out.value().as<float>(), current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}

// One decode step of attention over a KV cache (src/layers/attention.rs:96-99
// for one query token): q [batch, q_heads, head_dim], caches
// [batch, kv_heads, max_seq, head_dim], lens (device int32 [batch], may be
// null: every position) -> out [batch, q_heads, head_dim].  The GQA head map
// of repeat_kv is applied without materialising it.
inline Result<Tensor> decode_attention(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache,
                                       const int32_t* lens = nullptr) {
    if (q.rank() != 3 || k_cache.rank() != 4 || k_cache.shape() != v_cache.shape() ||
        q.dims()[0] != k_cache.dims()[0] || q.dims()[2] != k_cache.dims()[3])
        return OxideError::invalid("decode_attention: q " + q.shape().to_string() + " and caches " +
                                   k_cache.shape().to_string() + " must be [b, hq, d] and [b, hkv, max_seq, d]");
    OXIDE_TRY(detail::same_dtype(q, k_cache, "decode_attention"));
    OXIDE_TRY(detail::same_dtype(q, v_cache, "decode_attention"));
    const size_t b = q.dims()[0], hq = q.dims()[1], d = q.dims()[2];
    const size_t hkv = k_cache.dims()[1], max_seq = k_cache.dims()[2];
    auto out = Tensor::empty(q.shape(), q.dtype(), q.device());
    if (out.is_err()) return out;
    const uint64_t wb = oxide_decode_attention_workspace_bytes(b, hq, max_seq, d);
    auto ws = DeviceBuffer::allocate(wb ? wb : 16, q.device());
    if (ws.is_err()) return ws.error();
    const float scale = 1.0f / std::sqrt((float)d);
    const int rc = detail::bf16(q)
        ? oxide_decode_attention_bf16(q.as<oxide_bf16>(), k_cache.as<oxide_bf16>(), v_cache.as<oxide_bf16>(),
                                      lens, out.value().as<oxide_bf16>(), b, hq, hkv, max_seq, d, scale,
                                      ws.value()->ptr(), wb, current_stream())
        : oxide_decode_attention_f32(q.as<float>(), k_cache.as<float>(), v_cache.as<float>(), lens,
                                     out.value().as<float>(), b, hq, hkv, max_seq, d, scale, ws.value()->ptr(), wb,
                                     current_stream());
    OXIDE_TRY(check_status(rc));
    OXIDE_TRY(check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize"));  // ws lifetime
    return out;
}

// softmax_with_temperature (src/tokenizer.rs:166-180) over the last dim ->
// f32 probabilities of the same shape.
inline Result<Tensor> softmax_with_temperature(const Tensor& logits, float temperature) {
    if (logits.rank() < 1) return OxideError::invalid("softmax_with_temperature requires at least 1D tensor");
    const size_t vocab = logits.dims().back(), rows = vocab ? logits.elem_count() / vocab : 0;
    auto out = Tensor::empty(logits.shape(), DType::F32, logits.device());
    if (out.is_err()) return out;
    const int rc = detail::bf16(logits)
        ? oxide_softmax_with_temperature_bf16(logits.as<oxide_bf16>(), out.value().as<float>(), rows, vocab,
                                              temperature, current_stream())
        : oxide_softmax_with_temperature_f32(logits.as<float>(), out.value().as<float>(), rows, vocab,
                                             temperature, current_stream());
    OXIDE_TRY(check_status(rc));
    return out;
}
}  // namespace ops

// InferenceParams (src/tokenizer.rs:145-162) with the reference's defaults.
struct InferenceParams {
    size_t max_new_tokens = 100;
    float temperature = 1.0f;
    float top_p = 1.0f;
    size_t top_k = 50;
    float repetition_penalty = 1.0f;
};

// The token step of the generation loop (src/pipeline.rs:181-205) for every
// row of logits [..., vocab]: softmax_with_temperature, then sample_top_p when
// top_p < 1, else sample_top_k.  uniforms holds one draw in [0, 1) per row --
// the reference's fastrand::f32() -- so the caller keeps the generator.  A
// row whose probabilities hold a NaN gives OXIDE_SAMPLE_INVALID (the
// reference's sort panics there).
inline Result<std::vector<uint32_t>> sample_next_token(const Tensor& logits, const std::vector<float>& uniforms,
                                                       const InferenceParams& params = {}) {
    if (logits.rank() < 1) return OxideError::invalid("sample_next_token requires at least 1D tensor");
    const size_t vocab = logits.dims().back();
    size_t rows = 1;
    for (size_t i = 0; i + 1 < logits.rank(); ++i) rows *= logits.dims()[i];
    if (uniforms.size() != rows)
        return OxideError::invalid("sample_next_token: " + std::to_string(uniforms.size()) +
                                   " uniforms for " + std::to_string(rows) + " rows");
    auto buf = DeviceBuffer::allocate(rows * (sizeof(float) + sizeof(uint32_t)) + 16, logits.device());
    if (buf.is_err()) return buf.error();
    float* u = static_cast<float*>(buf.value()->ptr());
    uint32_t* tok = reinterpret_cast<uint32_t*>(u + rows);
    std::vector<uint32_t> host(rows);
    if (rows == 0) return host;
    OXIDE_TRY(check_cuda(cudaMemcpyAsync(u, uniforms.data(), rows * sizeof(float), cudaMemcpyHostToDevice,
                                         current_stream()), "cudaMemcpyAsync"));
    const int rc = logits.dtype() == DType::BF16
        ? oxide_sample_bf16(logits.as<oxide_bf16>(), rows, vocab, params.temperature, params.top_k, params.top_p,
                            u, tok, nullptr, current_stream())
        : oxide_sample_f32(logits.as<float>(), rows, vocab, params.temperature, params.top_k, params.top_p, u,
                           tok, nullptr, current_stream());
    OXIDE_TRY(check_status(rc));
    OXIDE_TRY(check_cuda(cudaMemcpyAsync(host.data(), tok, rows * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                         current_stream()), "cudaMemcpyAsync"));
    OXIDE_TRY(check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize"));
    return host;
}

// precompute_rope_cache (src/models/mistral.rs:91-115): f32 (cos, sin)
// tables [max_pos, head_dim/2] built on the host, then uploaded.
inline Result<std::pair<Tensor, Tensor>> precompute_rope_cache(float theta, size_t head_dim,
                                                               size_t max_pos, int device = 0) {
    const size_t half = head_dim / 2;
    std::vector<float> c(max_pos * half), s(max_pos * half);
    OXIDE_TRY(check_status(oxide_rope_table_host_f32(theta, head_dim, max_pos, c.data(), s.data())));
    auto ct = Tensor::from_f32(c, Shape{max_pos, half}, device);
    if (ct.is_err()) return ct.error();
    auto st = Tensor::from_f32(s, Shape{max_pos, half}, device);
    if (st.is_err()) return st.error();
    return std::make_pair(std::move(ct).value(), std::move(st).value());
}

// KVCache (src/cache/kv_cache.rs): per-layer device caches [batch, kv_heads,
// max_seq_len, head_dim]; update() appends with one kernel at the layer's own
// length (the reference's single counter, advanced by every layer's update,
// would place layer 1's tokens after layer 0's).
class KvCache {
  public:
    static Result<KvCache> create(size_t num_layers, size_t batch, size_t kv_heads, size_t head_dim,
                                  size_t max_seq_len, DType dtype = DType::F32, int device = 0) {
        KvCache c;
        c.batch_ = batch;
        c.heads_ = kv_heads;
        c.head_dim_ = head_dim;
        c.max_ = max_seq_len;
        c.len_.assign(num_layers, 0);
        for (size_t l = 0; l < num_layers; ++l) {
            auto k = Tensor::zeros(Shape{batch, kv_heads, max_seq_len, head_dim}, dtype, device);
            if (k.is_err()) return k.error();
            auto v = Tensor::zeros(Shape{batch, kv_heads, max_seq_len, head_dim}, dtype, device);
            if (v.is_err()) return v.error();
            c.k_.push_back(std::move(k).value());
            c.v_.push_back(std::move(v).value());
        }
        return c;
    }
    Status update(size_t layer, const Tensor& key, const Tensor& value) {
        if (layer >= k_.size())
            return OxideError::invalid("Layer index " + std::to_string(layer) + " out of range for " +
                                       std::to_string(k_.size()) + " layers");
        const Tensor& kc = k_[layer];
        if (key.shape() != value.shape() || key.rank() != 4 || key.dims()[0] != batch_ ||
            key.dims()[1] != heads_ || key.dims()[3] != head_dim_ || key.dtype() != kc.dtype() ||
            value.dtype() != kc.dtype())
            return OxideError::invalid("key/value " + key.shape().to_string() + " do not match the cache " +
                                       kc.shape().to_string());
        const size_t cur = len_[layer], add = key.dims()[2];
        if (cur + add > max_)
            return OxideError::invalid("KV cache overflow: " + std::to_string(cur + add) + " > " +
                                       std::to_string(max_));
        const int rc = detail_bf16(kc)
            ? oxide_kv_cache_append_bf16(kc.as<oxide_bf16>(), v_[layer].as<oxide_bf16>(), key.as<oxide_bf16>(),
                                         value.as<oxide_bf16>(), batch_, heads_, max_, head_dim_, cur, add,
                                         current_stream())
            : oxide_kv_cache_append_f32(kc.as<float>(), v_[layer].as<float>(), key.as<float>(), value.as<float>(),
                                        batch_, heads_, max_, head_dim_, cur, add, current_stream());
        OXIDE_TRY(check_status(rc));
        len_[layer] = cur + add;
        return Unit{};
    }
    const Tensor& k_cache(size_t layer) const { return k_[layer]; }
    const Tensor& v_cache(size_t layer) const { return v_[layer]; }
    size_t seq_len(size_t layer) const { return len_[layer]; }
    size_t current_seq_len() const { return len_.empty() ? 0 : len_[0]; }
    size_t max_seq_len() const { return max_; }
    size_t num_layers() const { return k_.size(); }
    void clear() { std::fill(len_.begin(), len_.end(), 0); }
    bool is_full() const { return current_seq_len() >= max_; }
    size_t get_cache_size() const {
        return k_.empty() ? 0 : 2 * k_[0].nbytes() * k_.size();
    }

  private:
    static bool detail_bf16(const Tensor& t) { return t.dtype() == DType::BF16; }
    KvCache() = default;
    std::vector<Tensor> k_, v_;
    std::vector<size_t> len_;
    size_t batch_ = 0, heads_ = 0, head_dim_ = 0, max_ = 0;
};

// ---- launcher-level interface (src/cuda_backend) ------------------------------------------------
// KernelManager (src/cuda_backend/kernels.rs:75-376): launchers over caller-owned
// device buffers, asynchronous on the manager's stream, errors as strings.
using LaunchResult = Result<Unit>;

class KernelManager {
  public:
    explicit KernelManager(cudaStream_t stream = nullptr) : stream_(stream) {}
    cudaStream_t stream() const { return stream_; }

    LaunchResult launch_vecadd(const float* a, const float* b, float* c, size_t n) const {
        return wrap("vecadd", oxide_add_f32(a, b, c, n, stream_));
    }
    LaunchResult launch_sub(const float* a, const float* b, float* c, size_t n) const {
        return wrap("sub", oxide_sub_f32(a, b, c, n, stream_));
    }
    LaunchResult launch_mul(const float* a, const float* b, float* c, size_t n) const {
        return wrap("mul", oxide_binary_f32(OXIDE_MUL, a, n, b, n, c, n, stream_));
    }
    LaunchResult launch_div(const float* a, const float* b, float* c, size_t n) const {
        return wrap("div", oxide_div_f32(a, b, c, n, stream_));
    }
    LaunchResult launch_scale(const float* input, float* output, float scale, size_t n) const {
        return wrap("scale", oxide_scale_f32(input, output, scale, n, stream_));
    }
    LaunchResult launch_silu(const float* input, float* output, size_t n) const {
        return wrap("silu", oxide_silu_f32(input, output, n, stream_));
    }
    LaunchResult launch_relu(const float* input, float* output, size_t n) const {
        return wrap("relu", oxide_relu_f32(input, output, n, stream_));
    }
    LaunchResult launch_gelu(const float* input, float* output, size_t n) const {
        return wrap("gelu", oxide_gelu_f32(input, output, n, stream_));
    }
    LaunchResult launch_sigmoid(const float* input, float* output, size_t n) const {
        return wrap("sigmoid", oxide_sigmoid_f32(input, output, n, stream_));
    }
    LaunchResult launch_tanh(const float* input, float* output, size_t n) const {
        return wrap("tanh", oxide_tanh_f32(input, output, n, stream_));
    }
    LaunchResult launch_layer_norm(const float* input, const float* weight, const float* bias,
                                   float* output, size_t num_rows, size_t num_cols, float eps) const {
        return wrap("layer_norm",
                    oxide_layer_norm_f32(input, weight, bias, output, num_rows, num_cols, eps, stream_));
    }
    LaunchResult launch_rms_norm(const float* input, const float* weight, float* output,
                                 size_t num_rows, size_t num_cols, float eps) const {
        return wrap("rms_norm", oxide_rms_norm_f32(input, weight, output, num_rows, num_cols, eps, stream_));
    }
    LaunchResult launch_softmax(const float* input, float* output, size_t num_rows,
                                size_t num_cols) const {
        return wrap("softmax", oxide_softmax_f32(input, output, num_rows, num_cols, 1, stream_));
    }

  private:
    static LaunchResult wrap(const char* what, int rc) {
        if (rc == OXIDE_OK) return Unit{};
        OxideError e = error_from_status(rc);
        e.message = std::string(what) + " launch failed: " + e.message;
        return e;
    }
    cudaStream_t stream_;
};

// CudaBackend (src/cuda_backend/mod.rs:43-140): device selection, f32 buffers,
// host<->device copies, and the kernel manager.
class CudaBackend {
  public:
    static Result<CudaBackend> create(int device_id) {
        int n = 0;
        OXIDE_TRY(check_cuda(cudaGetDeviceCount(&n), "cudaGetDeviceCount"));
        if (device_id < 0 || device_id >= n)
            return OxideError{OxideError::Kind::DeviceError, "no CUDA device " + std::to_string(device_id)};
        OXIDE_TRY(check_cuda(cudaSetDevice(device_id), "cudaSetDevice"));
        return CudaBackend(device_id);
    }
    int device() const { return device_; }
    const KernelManager& kernels() const { return kernels_; }
    Result<Tensor> allocate_f32(size_t len) const { return Tensor::zeros(Shape{len}, DType::F32, device_); }
    Result<Tensor> copy_host_to_device(const std::vector<float>& host) const {
        return Tensor::from_f32(host, Shape{host.size()}, device_);
    }
    Result<std::vector<float>> copy_device_to_host(const Tensor& t) const { return t.to_vec<float>(); }
    Status synchronize() const { return check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize"); }

  private:
    explicit CudaBackend(int d) : device_(d) {}
    int device_;
    KernelManager kernels_;
};

}  // namespace oxide
