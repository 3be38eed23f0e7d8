// Tests of the C++ host layer (include/oxide_host.hpp) against the CPU oracle.
//
// They follow the reference's own tests where it has one (the CudaBackend
// allocation + host/device round trip of src/cuda_backend/mod.rs:218-243) and
// otherwise check each op of src/ops through the Rust-shaped interface:
// new output per call, InvalidArgument with the reference's message on bad
// shapes, results equal to the oracle's (bit for bit where the contract says
// so, else within the stated tolerance).
//
//   test_host_ops            run every test; device tests are skipped (and
//                            reported) when no CUDA device is visible
//   test_host_ops --host     host-only tests
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "oxide_host.hpp"
#include "oxide_oracle.h"

using namespace oxide;

namespace {

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

struct TestCase {
    const char* name;
    bool device;
    std::function<void()> fn;
};
std::vector<TestCase>& registry() {
    static std::vector<TestCase> r;
    return r;
}
struct Reg {
    Reg(const char* n, bool d, std::function<void()> f) { registry().push_back({n, d, std::move(f)}); }
};
#define HOST_TEST(name) \
    static void name(); \
    static Reg reg_##name(#name, false, name); \
    static void name()
#define DEVICE_TEST(name) \
    static void name(); \
    static Reg reg_##name(#name, true, name); \
    static void name()
#define EXPECT(cond)                                                                           \
    do {                                                                                       \
        if (!(cond))                                                                           \
            throw Failure(std::string(__FILE__) + ":" + std::to_string(__LINE__) + ": " + #cond); \
    } while (0)

template <typename T>
T unwrap(Result<T> r, const char* what = "op") {
    if (r.is_err()) throw Failure(std::string(what) + " failed: " + r.error().to_string());
    return std::move(r).value();
}
template <typename T>
OxideError expect_err(Result<T> r) {
    if (r.is_ok()) throw Failure("expected an error");
    return r.error();
}

const int kThreads = 1;

std::vector<float> randn(size_t n, unsigned seed, float scale = 1.0f) {
    std::mt19937 g(seed);
    std::normal_distribution<float> d(0.0f, 1.0f);
    std::vector<float> v(n);
    for (auto& x : v) x = d(g) * scale;
    return v;
}
std::vector<float> uniform(size_t n, unsigned seed, float lo, float hi) {
    std::mt19937 g(seed);
    std::uniform_real_distribution<float> d(lo, hi);
    std::vector<float> v(n);
    for (auto& x : v) x = d(g);
    return v;
}
std::vector<uint16_t> to_bf16(const std::vector<float>& v) {
    std::vector<uint16_t> o(v.size());
    for (size_t i = 0; i < v.size(); ++i) o[i] = orc_f32_to_bf16(v[i]);
    return o;
}

uint32_t bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
int64_t ordered(float f) {
    const int32_t i = static_cast<int32_t>(bits(f));
    return i < 0 ? static_cast<int64_t>(INT32_MIN) - i : i;
}
int64_t ordered16(uint16_t h) { return h & 0x8000 ? -static_cast<int64_t>(h & 0x7fff) : h; }

void expect_bits_equal(const std::vector<float>& got, const std::vector<float>& ref) {
    EXPECT(got.size() == ref.size());
    for (size_t i = 0; i < got.size(); ++i)
        if (bits(got[i]) != bits(ref[i]))
            throw Failure("element " + std::to_string(i) + ": " + std::to_string(got[i]) + " != " +
                          std::to_string(ref[i]));
}
void expect_ulp(const std::vector<float>& got, const std::vector<float>& ref, int64_t max_ulp) {
    EXPECT(got.size() == ref.size());
    for (size_t i = 0; i < got.size(); ++i)
        if (std::llabs(ordered(got[i]) - ordered(ref[i])) > max_ulp)
            throw Failure("element " + std::to_string(i) + " differs by more than " +
                          std::to_string(max_ulp) + " ulp");
}
void expect_ulp16(const std::vector<uint16_t>& got, const std::vector<uint16_t>& ref, int64_t max_ulp) {
    EXPECT(got.size() == ref.size());
    for (size_t i = 0; i < got.size(); ++i)
        if (std::llabs(ordered16(got[i]) - ordered16(ref[i])) > max_ulp)
            throw Failure("bf16 element " + std::to_string(i) + " differs by more than " +
                          std::to_string(max_ulp) + " ulp");
}
void expect_close_rel(const std::vector<float>& got, const std::vector<float>& ref, double rel) {
    EXPECT(got.size() == ref.size());
    for (size_t i = 0; i < got.size(); ++i) {
        const double e = std::fabs(static_cast<double>(got[i]) - ref[i]);
        if (e > rel * std::fabs(static_cast<double>(ref[i])) + 1e-38)
            throw Failure("element " + std::to_string(i) + ": " + std::to_string(got[i]) + " vs " +
                          std::to_string(ref[i]));
    }
}

Tensor dev(const std::vector<float>& v, Shape s) { return unwrap(Tensor::from_f32(v, std::move(s)), "upload"); }
Tensor dev16(const std::vector<uint16_t>& v, Shape s) {
    return unwrap(Tensor::from_bf16_bits(v, std::move(s)), "upload");
}
std::vector<float> host(const Tensor& t) { return unwrap(t.to_vec<float>(), "download"); }
std::vector<uint16_t> host16(const Tensor& t) { return unwrap(t.to_vec<uint16_t>(), "download"); }

// ---- host-only ------------------------------------------------------------------------

HOST_TEST(broadcast_shape_follows_reference_rules) {
    EXPECT((unwrap(ops::broadcast_shape({8, 4096}, {4096})) == std::vector<size_t>{8, 4096}));
    EXPECT((unwrap(ops::broadcast_shape({3, 1, 64}, {5, 64})) == std::vector<size_t>{3, 5, 64}));
    EXPECT((unwrap(ops::broadcast_shape({}, {7})) == std::vector<size_t>{7}));
    const OxideError e = expect_err(ops::broadcast_shape({2, 3}, {4}));
    EXPECT(e.kind == OxideError::Kind::InvalidArgument);
    EXPECT(e.message == "broadcast: shape mismatch [2, 3] and [4]");
    EXPECT(e.to_string() == "Invalid argument: broadcast: shape mismatch [2, 3] and [4]");
}

HOST_TEST(status_codes_map_to_error_kinds) {
    EXPECT(error_from_status(OXIDE_ERR_INVALID_ARG).kind == OxideError::Kind::InvalidArgument);
    EXPECT(error_from_status(OXIDE_ERR_UNSUPPORTED).kind == OxideError::Kind::UnsupportedOperation);
    EXPECT(error_from_status(OXIDE_ERR_LAUNCH).kind == OxideError::Kind::KernelLaunchError);
    EXPECT(error_from_status(OXIDE_ERR_CUDA).kind == OxideError::Kind::CudaError);
    EXPECT(check_status(OXIDE_OK).is_ok());
}

HOST_TEST(launcher_rejects_bad_arguments_before_any_launch) {
    KernelManager km;
    // null buffers with n > 0: argument error, reported like cudarc launch errors
    auto r = km.launch_vecadd(nullptr, nullptr, nullptr, 16);
    EXPECT(r.is_err());
    EXPECT(r.error().kind == OxideError::Kind::InvalidArgument);
    EXPECT(r.error().message.rfind("vecadd launch failed: ", 0) == 0);
    // n = 0 is a valid no-op
    EXPECT(km.launch_vecadd(nullptr, nullptr, nullptr, 0).is_ok());
    // an injected failure is reported and nothing is launched
    oxide_debug_fail_next("oxide_rms_norm_f32");
    r = km.launch_rms_norm(nullptr, nullptr, nullptr, 4, 4, 1e-5f);
    EXPECT(r.is_err() && r.error().kind == OxideError::Kind::CudaError);
    EXPECT(r.error().message.find("injected") != std::string::npos);
}

HOST_TEST(rope_table_matches_oracle) {
    const size_t d = 128, p = 64;
    std::vector<float> c(p * d / 2), s(p * d / 2), oc(c.size()), os(s.size());
    EXPECT(oxide_rope_table_host_f32(1e6f, d, p, c.data(), s.data()) == OXIDE_OK);
    orc_rope_table_f32(1e6f, d, p, oc.data(), os.data());
    expect_bits_equal(c, oc);
    expect_bits_equal(s, os);
}

// ---- device ---------------------------------------------------------------------------

// src/cuda_backend/mod.rs:218-243: allocate 1024 floats, round-trip 0..1024.
DEVICE_TEST(backend_allocation_and_round_trip) {
    CudaBackend backend = unwrap(CudaBackend::create(0), "CudaBackend::create");
    Tensor buffer = unwrap(backend.allocate_f32(1024));
    EXPECT(buffer.elem_count() == 1024);
    std::vector<float> host_data(1024);
    for (int i = 0; i < 1024; ++i) host_data[i] = static_cast<float>(i);
    Tensor device_buf = unwrap(backend.copy_host_to_device(host_data));
    std::vector<float> host_back = unwrap(backend.copy_device_to_host(device_buf));
    EXPECT(host_back[0] == 0.0f);
    EXPECT(host_back[1023] == 1023.0f);
    EXPECT(unwrap(backend.copy_device_to_host(buffer))[511] == 0.0f);  // zeros
    EXPECT(backend.synchronize().is_ok());
}

DEVICE_TEST(binary_ops_with_broadcast_match_oracle) {
    const auto a = randn(3 * 64, 1), b = randn(5 * 64, 2);
    const Tensor ta = dev(a, {3, 1, 64}), tb = dev(b, {5, 64});
    const int opsel[] = {OXIDE_ADD, OXIDE_SUB, OXIDE_MUL, OXIDE_DIV};
    for (int op : opsel) {
        Tensor out = unwrap(ops::binary(op, ta, tb));
        EXPECT((out.dims() == std::vector<size_t>{3, 5, 64}));
        std::vector<float> ref(out.elem_count());
        orc_binary_f32(op, a.data(), a.size(), b.data(), b.size(), ref.data(), ref.size(), kThreads);
        expect_bits_equal(host(out), ref);
    }
    // row-broadcast multiply [rows, cols] * [cols] and bf16 add
    const auto x = randn(37 * 256, 3), s = uniform(256, 4, 0.5f, 1.5f);
    std::vector<float> ref(x.size());
    orc_binary_f32(OXIDE_MUL, x.data(), x.size(), s.data(), s.size(), ref.data(), ref.size(), kThreads);
    expect_bits_equal(host(unwrap(ops::mul(dev(x, {37, 256}), dev(s, {256})))), ref);
    const auto xb = to_bf16(x), yb = to_bf16(randn(x.size(), 5));
    std::vector<uint16_t> rb(x.size());
    orc_binary_bf16(OXIDE_ADD, xb.data(), xb.size(), yb.data(), yb.size(), rb.data(), rb.size(), kThreads);
    EXPECT(host16(unwrap(ops::add(dev16(xb, {37, 256}), dev16(yb, {37, 256})))) == rb);
    // shape and dtype errors
    EXPECT(expect_err(ops::add(dev(a, {3, 64}), dev(b, {5, 64}))).kind == OxideError::Kind::InvalidArgument);
    EXPECT(expect_err(ops::add(dev(x, {37, 256}), dev16(yb, {37, 256}))).kind ==
           OxideError::Kind::DtypeMismatch);
}

DEVICE_TEST(silu_and_silu_mul_match_oracle) {
    const size_t n = 4099;  // not a multiple of the vector width
    const auto g = randn(n, 6, 4.0f), u = randn(n, 7);
    std::vector<float> ref(n);
    orc_silu_f32(g.data(), ref.data(), n, kThreads);
    expect_ulp(host(unwrap(ops::silu(dev(g, {n})))), ref, 8);
    orc_silu_mul_f32(g.data(), u.data(), ref.data(), n, kThreads);
    expect_ulp(host(unwrap(ops::silu_mul(dev(g, {n}), dev(u, {n})))), ref, 8);
    const auto gb = to_bf16(g), ub = to_bf16(u);
    std::vector<uint16_t> rb(n);
    orc_silu_mul_bf16(gb.data(), ub.data(), rb.data(), n, kThreads);
    expect_ulp16(host16(unwrap(ops::silu_mul(dev16(gb, {n}), dev16(ub, {n})))), rb, 1);
    EXPECT(expect_err(ops::silu_mul(dev(g, {n}), dev(u, {1, n}))).kind == OxideError::Kind::ShapeMismatch);
}

DEVICE_TEST(rms_norm_matches_oracle_and_checks_weight_shape) {
    const size_t rows = 33, cols = 4096;
    const auto x = randn(rows * cols, 8), w = uniform(cols, 9, 0.5f, 1.5f);
    std::vector<float> ref(x.size());
    orc_rms_norm_f32(x.data(), w.data(), ref.data(), rows, cols, 1e-5f, kThreads);
    expect_close_rel(host(unwrap(ops::rms_norm(dev(x, {rows, cols}), dev(w, {cols}), 1e-5f))), ref, 1e-5);
    const auto xb = to_bf16(x), wb = to_bf16(w);
    std::vector<uint16_t> rb(x.size());
    orc_rms_norm_bf16(xb.data(), wb.data(), rb.data(), rows, cols, 1e-5f, kThreads);
    expect_ulp16(host16(unwrap(ops::rms_norm(dev16(xb, {rows, cols}), dev16(wb, {cols}), 1e-5f))), rb, 1);
    const OxideError e = expect_err(ops::rms_norm(dev(x, {rows, cols}), dev(uniform(cols / 2, 22, 0.5f, 1.5f), {cols / 2}), 1e-5f));
    EXPECT(e.kind == OxideError::Kind::InvalidArgument);
    EXPECT(e.message == "rms_norm weight shape [2048] doesn't match input last dim 4096");
}

DEVICE_TEST(add_rms_norm_matches_unfused_pair) {
    const size_t rows = 17, cols = 4096;
    const auto x = to_bf16(randn(rows * cols, 10)), r = to_bf16(randn(rows * cols, 11)),
               w = to_bf16(uniform(cols, 12, 0.5f, 1.5f));
    std::vector<uint16_t> h(x.size()), y(x.size());
    orc_add_rms_norm_bf16(x.data(), r.data(), w.data(), h.data(), y.data(), rows, cols, 1e-5f, kThreads);
    auto hy = unwrap(ops::add_rms_norm(dev16(x, {rows, cols}), dev16(r, {rows, cols}), dev16(w, {cols}), 1e-5f));
    EXPECT(host16(hy.first) == h);  // the residual is bit-exact
    expect_ulp16(host16(hy.second), y, 1);
    // fused == add then rms_norm through the same layer
    Tensor h2 = unwrap(ops::add(dev16(x, {rows, cols}), dev16(r, {rows, cols})));
    EXPECT(host16(unwrap(ops::rms_norm(h2, dev16(w, {cols}), 1e-5f))) == host16(hy.second));
}

DEVICE_TEST(softmax_any_dim_matches_oracle) {
    const size_t a = 4, d = 37, b = 3;
    const auto x = randn(a * d * b, 13, 3.0f);
    std::vector<float> ref(x.size());
    orc_softmax_f32(x.data(), ref.data(), a, d, b, kThreads);  // dim = 1 of [4, 37, 3]
    expect_close_rel(host(unwrap(ops::softmax(dev(x, {a, d, b}), 1))), ref, 1e-5);
    orc_softmax_f32(x.data(), ref.data(), a * d, b, 1, kThreads);  // last dim
    expect_close_rel(host(unwrap(ops::softmax(dev(x, {a, d, b}), 2))), ref, 1e-5);
    const OxideError e = expect_err(ops::softmax(dev(x, {a, d, b}), 3));
    EXPECT(e.message == "softmax dim 3 out of range for rank 3");
}

DEVICE_TEST(scale_mask_softmax_with_kv_lengths_matches_oracle) {
    const size_t rows = 8, cols = 1000;
    const auto x = randn(rows * cols, 14, 11.3f);
    const std::vector<int32_t> lens = {1000, 517, 1, 0};  // per pair of rows
    int32_t* dl = nullptr;
    EXPECT(cudaMalloc(&dl, lens.size() * 4) == cudaSuccess);
    EXPECT(cudaMemcpy(dl, lens.data(), lens.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess);
    ops::MaskOptions m;
    m.lens = dl;
    m.rows_per_len = 2;
    const float scale = 1.0f / std::sqrt(128.0f);
    Tensor out = unwrap(ops::scale_mask_softmax(dev(x, {rows, cols}), scale, m));
    std::vector<float> ref(x.size());
    orc_scale_mask_softmax_f32(x.data(), ref.data(), rows, cols, scale, nullptr, 0, lens.data(), 2, 0,
                               kThreads);
    const auto got = host(out);
    cudaFree(dl);
    expect_close_rel(got, ref, 1e-5);
    for (size_t j = 0; j < cols; ++j) EXPECT(got[6 * cols + j] == 0.0f);  // length 0: zeros
}

DEVICE_TEST(rotary_embedding_matches_oracle) {
    const size_t heads = 4, seq = 16, hd = 128;
    auto [cos_t, sin_t] = unwrap(precompute_rope_cache(1e6f, hd, seq));
    std::vector<float> oc(seq * hd / 2), os(oc.size());
    orc_rope_table_f32(1e6f, hd, seq, oc.data(), os.data());
    expect_bits_equal(host(cos_t), oc);
    // apply_rotary_emb: head-major [heads, seq, head_dim]
    const auto x = randn(heads * seq * hd, 15);
    std::vector<float> ref(x.size());
    orc_rope_f32(x.data(), ref.data(), seq, heads, hd, 1, oc.data(), os.data(), nullptr, kThreads);
    expect_bits_equal(host(unwrap(ops::apply_rotary_emb(dev(x, {1, heads, seq, hd}), cos_t, sin_t))), ref);
    // q and k in one launch, token-major, bf16
    const auto q = to_bf16(randn(seq * 8 * hd, 16)), k = to_bf16(randn(seq * 2 * hd, 17));
    auto qk = unwrap(ops::rope_qk(dev16(q, {seq, 8, hd}), dev16(k, {seq, 2, hd}), cos_t, sin_t));
    std::vector<uint16_t> rq(q.size()), rk(k.size());
    orc_rope_bf16(q.data(), rq.data(), seq, 8, hd, 0, oc.data(), os.data(), nullptr, kThreads);
    orc_rope_bf16(k.data(), rk.data(), seq, 2, hd, 0, oc.data(), os.data(), nullptr, kThreads);
    EXPECT(host16(qk.first) == rq);
    EXPECT(host16(qk.second) == rk);
    const OxideError e = expect_err(ops::apply_rotary_emb(dev(x, {heads, seq, hd}), sin_t, dev(oc, {seq * 2, hd / 4})));
    EXPECT(e.message == "sin shape [32, 32] doesn't match expected [16, 64]");
}

DEVICE_TEST(argmax_and_reductions_match_oracle) {
    const size_t rows = 9, cols = 32000;
    auto x = randn(rows * cols, 18);
    x[1 * cols + 5] = 50.0f;
    x[1 * cols + 900] = 50.0f;  // tie: the lowest index wins
    std::vector<uint32_t> ref(rows);
    orc_argmax_rows_f32(x.data(), rows, cols, ref.data(), kThreads);
    const Tensor tx = dev(x, {rows, cols});
    EXPECT(unwrap(ops::argmax(tx)) == ref);
    EXPECT(ref[1] == 5);
    for (int op : {OXIDE_RED_SUM, OXIDE_RED_MAX, OXIDE_RED_SUMSQ}) {
        const double want = orc_reduce_f32(op, x.data(), x.size(), kThreads);
        const double got = unwrap(ops::reduce(tx, op));
        double mag = 0;
        for (float v : x) mag += op == OXIDE_RED_SUMSQ ? double(v) * v : std::fabs(double(v));
        EXPECT(op == OXIDE_RED_MAX ? got == want : std::fabs(got - want) <= 1e-5 * mag);
        std::vector<float> rr(rows);
        orc_reduce_rows_f32(op, x.data(), rows, cols, rr.data(), kThreads);
        const auto gr = host(unwrap(ops::reduce_rows(tx, op)));
        for (size_t i = 0; i < rows; ++i) {
            double m = 0;
            for (size_t j = 0; j < cols; ++j) {
                const double v = x[i * cols + j];
                m += op == OXIDE_RED_SUMSQ ? v * v : std::fabs(v);
            }
            EXPECT(op == OXIDE_RED_MAX ? gr[i] == rr[i] : std::fabs(double(gr[i]) - rr[i]) <= 1e-5 * m);
        }
    }
}

DEVICE_TEST(kernel_manager_launchers_match_oracle) {
    CudaBackend backend = unwrap(CudaBackend::create(0));
    const KernelManager& km = backend.kernels();
    const size_t rows = 64, cols = 4096, n = rows * cols;
    const auto a = randn(n, 19), b = randn(n, 20), w = uniform(cols, 21, 0.5f, 1.5f);
    const Tensor ta = dev(a, {n}), tb = dev(b, {n}), tw = dev(w, {cols});
    Tensor out = unwrap(backend.allocate_f32(n));
    std::vector<float> ref(n);
    EXPECT(km.launch_vecadd(ta.as<float>(), tb.as<float>(), out.as<float>(), n).is_ok());
    orc_binary_f32(OXIDE_ADD, a.data(), n, b.data(), n, ref.data(), n, kThreads);
    expect_bits_equal(host(out), ref);
    EXPECT(km.launch_div(ta.as<float>(), tb.as<float>(), out.as<float>(), n).is_ok());
    orc_binary_f32(OXIDE_DIV, a.data(), n, b.data(), n, ref.data(), n, kThreads);
    expect_bits_equal(host(out), ref);
    EXPECT(km.launch_scale(ta.as<float>(), out.as<float>(), 0.125f, n).is_ok());
    orc_scale_f32(a.data(), ref.data(), 0.125f, n, kThreads);
    expect_bits_equal(host(out), ref);
    EXPECT(km.launch_rms_norm(ta.as<float>(), tw.as<float>(), out.as<float>(), rows, cols, 1e-5f).is_ok());
    orc_rms_norm_f32(a.data(), w.data(), ref.data(), rows, cols, 1e-5f, kThreads);
    expect_close_rel(host(out), ref, 1e-5);
    EXPECT(km.launch_softmax(ta.as<float>(), out.as<float>(), rows, cols).is_ok());
    orc_softmax_f32(a.data(), ref.data(), rows, cols, 1, kThreads);
    expect_close_rel(host(out), ref, 1e-5);
    EXPECT(backend.synchronize().is_ok());
}

DEVICE_TEST(unary_ops_and_layer_norm_match_oracle) {
    const size_t n = 3001;
    const auto x = randn(n, 23, 3.0f);
    std::vector<float> ref(n);
    const Tensor tx = dev(x, {n});
    orc_unary_f32(ORC_RELU, x.data(), ref.data(), n, 0.0f, 0.0f, kThreads);
    expect_bits_equal(host(unwrap(ops::relu(tx))), ref);
    orc_unary_f32(ORC_TANH, x.data(), ref.data(), n, 0.0f, 0.0f, kThreads);
    expect_ulp(host(unwrap(ops::tanh(tx))), ref, 4);
    orc_unary_f32(ORC_GELU_QUICK, x.data(), ref.data(), n, 0.0f, 0.0f, kThreads);
    expect_ulp(host(unwrap(ops::gelu_quick(tx))), ref, 8);
    orc_unary_f32(ORC_CLAMP, x.data(), ref.data(), n, -1.0f, 2.0f, kThreads);
    expect_bits_equal(host(unwrap(ops::clamp(tx, -1.0f, 2.0f))), ref);
    EXPECT(expect_err(ops::clamp(tx, 2.0f, -1.0f)).kind == OxideError::Kind::InvalidArgument);
    // KernelManager::launch_sigmoid on raw buffers
    KernelManager km;
    Tensor out = unwrap(Tensor::empty(Shape{n}, DType::F32));
    EXPECT(km.launch_sigmoid(tx.as<float>(), out.as<float>(), n).is_ok());
    orc_unary_f32(ORC_SIGMOID, x.data(), ref.data(), n, 0.0f, 0.0f, kThreads);
    expect_ulp(host(out), ref, 8);
    // layer_norm: constant rows give the bias; shape errors carry the reference's message
    const size_t rows = 6, cols = 768;
    const auto w = uniform(cols, 24, 0.5f, 1.5f), b = uniform(cols, 25, -0.5f, 0.5f);
    const Tensor tw = dev(w, {cols}), tb = dev(b, {cols});
    std::vector<float> c(rows * cols, 2.5f);
    const auto y = host(unwrap(ops::layer_norm(dev(c, {rows, cols}), tw, tb, 1e-5f)));
    for (size_t r = 0; r < rows; ++r)
        for (size_t i = 0; i < cols; ++i) EXPECT(bits(y[r * cols + i]) == bits(b[i]));
    const OxideError e =
        expect_err(ops::layer_norm(dev(c, {rows, cols}), tw, dev(uniform(10, 26, 0.0f, 1.0f), {10}), 1e-5f));
    EXPECT(e.message == "layer_norm bias shape [10] doesn't match input last dim 768");
    const auto xr = randn(rows * cols, 27, 2.0f);
    std::vector<float> lref(xr.size());
    orc_layer_norm_f32(xr.data(), w.data(), b.data(), lref.data(), rows, cols, 1e-5f, kThreads);
    const auto lgot = host(unwrap(ops::layer_norm(dev(xr, {rows, cols}), tw, tb, 1e-5f)));
    for (size_t i = 0; i < lref.size(); ++i)
        EXPECT(std::fabs(lgot[i] - lref[i]) <= 1e-5f * (std::fabs(lref[i] - b[i % cols]) + std::fabs(b[i % cols])) + 1e-6f);
}

DEVICE_TEST(repeat_kv_and_kv_cache_match_oracle) {
    const size_t b = 2, h = 3, s = 5, d = 64, rep = 4;
    const auto x = randn(b * h * s * d, 28);
    std::vector<float> ref(x.size() * rep);
    orc_repeat_kv(x.data(), ref.data(), b, h, s, d, rep, 4);
    const Tensor out = unwrap(ops::repeat_kv(dev(x, {b, h, s, d}), rep));
    EXPECT((out.dims() == std::vector<size_t>{b, h * rep, s, d}));
    expect_bits_equal(host(out), ref);
    // cache: two appends (prefill of 3 tokens, then 1) equal one append of 4
    KvCache cache = unwrap(KvCache::create(2, b, h, d, 8));
    const auto k1 = randn(b * h * 3 * d, 29), v1 = randn(b * h * 3 * d, 30);
    const auto k2 = randn(b * h * 1 * d, 31), v2 = randn(b * h * 1 * d, 32);
    EXPECT(cache.update(1, dev(k1, {b, h, 3, d}), dev(v1, {b, h, 3, d})).is_ok());
    EXPECT(cache.update(1, dev(k2, {b, h, 1, d}), dev(v2, {b, h, 1, d})).is_ok());
    EXPECT(cache.seq_len(1) == 4 && cache.seq_len(0) == 0);
    std::vector<float> kref(b * h * 8 * d, 0.0f), vref(kref.size(), 0.0f);
    EXPECT(orc_kv_append(kref.data(), vref.data(), k1.data(), v1.data(), b, h, 8, d, 0, 3, 4) == 0);
    EXPECT(orc_kv_append(kref.data(), vref.data(), k2.data(), v2.data(), b, h, 8, d, 3, 1, 4) == 0);
    expect_bits_equal(host(cache.k_cache(1)), kref);
    expect_bits_equal(host(cache.v_cache(1)), vref);
    const auto big = randn(b * h * 5 * d, 33);
    const Status st = cache.update(1, dev(big, {b, h, 5, d}), dev(big, {b, h, 5, d}));
    EXPECT(st.is_err() && st.error().message == "KV cache overflow: 9 > 8");
    EXPECT(cache.update(2, dev(k2, {b, h, 1, d}), dev(v2, {b, h, 1, d})).error().message ==
           "Layer index 2 out of range for 2 layers");
}

DEVICE_TEST(decode_attention_and_sampling_match_oracle) {
    // one decode step over a cache of 40 positions, 8 query heads on 2 kv heads
    const size_t b = 2, hq = 8, hkv = 2, m = 40, d = 128;
    const auto q = randn(b * hq * d, 40), kc = randn(b * hkv * m * d, 41), vc = randn(b * hkv * m * d, 42);
    const std::vector<int32_t> lens = {40, 17};
    int32_t* dl = nullptr;
    EXPECT(cudaMalloc(&dl, sizeof(int32_t) * b) == cudaSuccess);
    EXPECT(cudaMemcpy(dl, lens.data(), sizeof(int32_t) * b, cudaMemcpyHostToDevice) == cudaSuccess);
    const Tensor out = unwrap(ops::decode_attention(dev(q, {b, hq, d}), dev(kc, {b, hkv, m, d}),
                                                    dev(vc, {b, hkv, m, d}), dl));
    std::vector<float> ref(q.size());
    orc_decode_attention_f32(q.data(), kc.data(), vc.data(), lens.data(), ref.data(), b, hq, hkv, m, d,
                             1.0f / std::sqrt((float)d), 1);
    const auto got = host(out);
    for (size_t i = 0; i < got.size(); ++i) EXPECT(std::fabs(got[i] - ref[i]) <= 1e-5f * (1.0f + std::fabs(ref[i])));
    cudaFree(dl);
    // sampling: the reference's defaults (top-k 50) and a top-p nucleus
    const size_t rows = 4, vocab = 5000;
    auto logits = randn(rows * vocab, 43);
    for (auto& v : logits) v *= 3.0f;
    const std::vector<float> u = {0.1f, 0.5f, 0.0f, 0.97f};
    const Tensor lt = dev(logits, {rows, vocab});
    // the kernel's own probabilities, walked by the reference's loops (the oracle)
    const auto gp = host(unwrap(ops::softmax_with_temperature(lt, 1.0f)));
    for (const auto& [k, p] : std::vector<std::pair<size_t, float>>{{50, 1.0f}, {1, 1.0f}, {50, 0.8f}}) {
        InferenceParams params;
        params.top_k = k;
        params.top_p = p;
        const auto tok = unwrap(sample_next_token(lt, u, params));
        for (size_t r = 0; r < rows; ++r) EXPECT(tok[r] == orc_sample_probs(gp.data() + r * vocab, vocab, k, p, u[r]));
    }
    const auto probs = host(unwrap(ops::softmax_with_temperature(lt, 0.7f)));
    std::vector<float> pref(logits.size());
    orc_softmax_temperature_f32(logits.data(), rows, vocab, 0.7f, pref.data(), 1);
    for (size_t i = 0; i < probs.size(); ++i) EXPECT(std::fabs(probs[i] - pref[i]) <= 2e-5f * pref[i] + 1e-12f);
    EXPECT(sample_next_token(lt, {0.5f}).error().message == "sample_next_token: 1 uniforms for 4 rows");
}

}  // namespace

int main(int argc, char** argv) {
    const bool host_only = argc > 1 && std::string(argv[1]) == "--host";
    int ndev = 0;
    const bool have_device = !host_only && cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0;
    int passed = 0, failed = 0, skipped = 0;
    for (const TestCase& t : registry()) {
        if (t.device && !have_device) {
            ++skipped;
            std::printf("SKIP %s (no CUDA device)\n", t.name);
            continue;
        }
        try {
            t.fn();
            ++passed;
            std::printf("PASS %s\n", t.name);
        } catch (const std::exception& e) {
            ++failed;
            std::printf("FAIL %s: %s\n", t.name, e.what());
        }
    }
    std::printf("%d passed, %d failed, %d skipped\n", passed, failed, skipped);
    return failed ? 1 : 0;
}
