// oxide_pipe.cpp -- host-buffer execution of one op with overlapped copies.
//
// The reference's ops consume and produce host tensors (src/ops/*: inputs
// read through Storage::as_f32_slice, outputs from Tensor::zeros), and its GPU
// backend moves data with CudaBackend::copy_host_to_device /
// copy_device_to_host (src/cuda_backend/mod.rs:76-85).  A pipeline runs one
// op on host buffers end to end: the rows are cut into chunks, chunk c goes to
// stream c % depth, and on each stream the host->device copy, the kernel and
// the device->host copy of a chunk are enqueued in order.  With depth >= 3 the
// upload of one chunk, the kernel of the next and the download of a third
// overlap, so the op runs at the PCIe copy rate rather than copy + compute.
//
// Staging buffers are allocated once in oxide_pipe_create; the op calls only
// enqueue copies and kernels and wait for their own streams.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <numeric>
#include <vector>

#include "oxide_ops.h"

namespace oxide {
int set_error(int code, const char* fmt, ...);
int injected_failure(const char* op);
}  // namespace oxide

struct oxide_pipe {
    int device = 0;
    uint64_t chunk_bytes = 0;
    int depth = 0;
    std::vector<cudaStream_t> streams;
    std::vector<void*> in0, in1, out;  // per-stream staging, chunk_bytes each
    void* bc0 = nullptr;               // broadcast operands, chunk_bytes each
    void* bc1 = nullptr;
    cudaEvent_t bc_ready = nullptr;
    std::mutex mu;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int cuda_fail(const char* op, cudaError_t e) {
    return oxide::set_error(OXIDE_ERR_CUDA, "%s: %s", op, cudaGetErrorString(e));
}

#define PIPE_CUDA(op, call)                    \
    do {                                       \
        cudaError_t _e = (call);               \
        if (_e != cudaSuccess) return cuda_fail(op, _e); \
    } while (0)

// Enqueue one step of a chunk; on failure record the status and stop
// enqueueing (the caller still drains the streams before returning).
#define STEP(call)                                          \
    do {                                                    \
        if (rc == OXIDE_OK) {                               \
            cudaError_t _e = (call);                        \
            if (_e != cudaSuccess) rc = cuda_fail(op, _e);  \
        }                                                   \
    } while (0)

void release(oxide_pipe* p) {
    for (cudaStream_t s : p->streams)
        if (s) cudaStreamSynchronize(s);
    for (void* b : p->in0) cudaFree(b);
    for (void* b : p->in1) cudaFree(b);
    for (void* b : p->out) cudaFree(b);
    if (p->bc0) cudaFree(p->bc0);
    if (p->bc1) cudaFree(p->bc1);
    if (p->bc_ready) cudaEventDestroy(p->bc_ready);
    for (cudaStream_t s : p->streams)
        if (s) cudaStreamDestroy(s);
}

// Wait for every stream of the pipe; report the first error.
int drain(oxide_pipe* p, const char* op) {
    int rc = OXIDE_OK;
    for (cudaStream_t s : p->streams) {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess && rc == OXIDE_OK) rc = cuda_fail(op, e);
    }
    return rc;
}

// Upload the broadcast operands (if any) on stream 0 and make every stream
// wait for them.
int upload_bcast(oxide_pipe* p, const char* op, const void* h0, uint64_t b0, const void* h1,
                 uint64_t b1) {
    if (!h0 && !h1) return OXIDE_OK;
    if (h0) PIPE_CUDA(op, cudaMemcpyAsync(p->bc0, h0, b0, cudaMemcpyHostToDevice, p->streams[0]));
    if (h1) PIPE_CUDA(op, cudaMemcpyAsync(p->bc1, h1, b1, cudaMemcpyHostToDevice, p->streams[0]));
    PIPE_CUDA(op, cudaEventRecord(p->bc_ready, p->streams[0]));
    for (int i = 1; i < p->depth; ++i)
        PIPE_CUDA(op, cudaStreamWaitEvent(p->streams[i], p->bc_ready, 0));
    return OXIDE_OK;
}

}  // namespace

extern "C" {

int oxide_pipe_create(int device, uint64_t chunk_bytes, int depth, oxide_pipe_t* out) {
    const char* op = "oxide_pipe_create";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!out) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null output pointer", op);
    *out = nullptr;
    if (depth < 1 || depth > 16)
        return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: depth must be in [1, 16]", op);
    if (chunk_bytes < 4096 || chunk_bytes % 256)
        return oxide::set_error(OXIDE_ERR_INVALID_ARG,
                                "%s: chunk_bytes must be >= 4096 and a multiple of 256", op);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: no CUDA device %d", op, device);
    }
    DeviceGuard g(device);
    auto* p = new oxide_pipe();
    p->device = device;
    p->chunk_bytes = chunk_bytes;
    p->depth = depth;
    p->streams.assign(depth, nullptr);
    p->in0.assign(depth, nullptr);
    p->in1.assign(depth, nullptr);
    p->out.assign(depth, nullptr);
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < depth && e == cudaSuccess; ++i) {
        e = cudaStreamCreateWithFlags(&p->streams[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaMalloc(&p->in0[i], chunk_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&p->in1[i], chunk_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&p->out[i], chunk_bytes);
    }
    if (e == cudaSuccess) e = cudaMalloc(&p->bc0, chunk_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&p->bc1, chunk_bytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->bc_ready, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        int rc = cuda_fail(op, e);
        release(p);
        delete p;
        return rc;
    }
    *out = p;
    return OXIDE_OK;
}

int oxide_pipe_destroy(oxide_pipe_t p) {
    if (!p) return OXIDE_OK;
    {
        DeviceGuard g(p->device);
        std::lock_guard<std::mutex> lk(p->mu);
        release(p);
    }
    delete p;
    return OXIDE_OK;
}

int oxide_pipe_binary_f32(oxide_pipe_t p, int bop, const float* a, uint64_t na, const float* b,
                          uint64_t nb, float* out, uint64_t n) {
    const char* op = "oxide_pipe_binary_f32";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (n == 0) return OXIDE_OK;
    if (!a || !b || !out) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    if (na < 1 || nb < 1 || na > n || nb > n || n % na || n % nb)
        return oxide::set_error(OXIDE_ERR_INVALID_ARG,
                                "%s: operand lengths must divide the output length", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t cap = p->chunk_bytes / sizeof(float);
    // Chunks must hold whole periods of every broadcast operand.
    uint64_t period = 1;
    if (na < n) period = std::lcm(period, na);
    if (nb < n) period = std::lcm(period, nb);
    if (period > cap)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED,
                                "%s: broadcast period %llu exceeds the pipe chunk", op,
                                (unsigned long long)period);
    const uint64_t chunk = cap / period * period;
    int rc = upload_bcast(p, op, na < n ? a : nullptr, na * sizeof(float), nb < n ? b : nullptr,
                          nb * sizeof(float));
    if (rc) {
        drain(p, op);
        return rc;
    }
    uint64_t c = 0;
    for (uint64_t lo = 0; lo < n && rc == OXIDE_OK; lo += chunk, ++c) {
        const uint64_t cnt = n - lo < chunk ? n - lo : chunk;
        const int s = (int)(c % p->depth);
        cudaStream_t st = p->streams[s];
        const float* da = static_cast<const float*>(p->bc0);
        const float* db = static_cast<const float*>(p->bc1);
        if (na == n) {
            STEP(cudaMemcpyAsync(p->in0[s], a + lo, cnt * 4, cudaMemcpyHostToDevice, st));
            da = static_cast<const float*>(p->in0[s]);
        }
        if (nb == n) {
            STEP(cudaMemcpyAsync(p->in1[s], b + lo, cnt * 4, cudaMemcpyHostToDevice, st));
            db = static_cast<const float*>(p->in1[s]);
        }
        if (rc == OXIDE_OK) rc = oxide_binary_f32(bop, da, na == n ? cnt : na, db, nb == n ? cnt : nb,
                              static_cast<float*>(p->out[s]), cnt, st);
        STEP(cudaMemcpyAsync(out + lo, p->out[s], cnt * 4, cudaMemcpyDeviceToHost, st));
    }
    int rc2 = drain(p, op);
    return rc ? rc : rc2;
}

int oxide_pipe_silu_mul_f32(oxide_pipe_t p, const float* gate, const float* up, float* out,
                            uint64_t n) {
    const char* op = "oxide_pipe_silu_mul_f32";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (n == 0) return OXIDE_OK;
    if (!gate || !up || !out) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t chunk = p->chunk_bytes / sizeof(float);
    int rc = OXIDE_OK;
    uint64_t c = 0;
    for (uint64_t lo = 0; lo < n && rc == OXIDE_OK; lo += chunk, ++c) {
        const uint64_t cnt = n - lo < chunk ? n - lo : chunk;
        const int s = (int)(c % p->depth);
        cudaStream_t st = p->streams[s];
        STEP(cudaMemcpyAsync(p->in0[s], gate + lo, cnt * 4, cudaMemcpyHostToDevice, st));
        STEP(cudaMemcpyAsync(p->in1[s], up + lo, cnt * 4, cudaMemcpyHostToDevice, st));
        if (rc == OXIDE_OK) rc = oxide_silu_mul_f32(static_cast<const float*>(p->in0[s]),
                                static_cast<const float*>(p->in1[s]),
                                static_cast<float*>(p->out[s]), cnt, st);
        STEP(cudaMemcpyAsync(out + lo, p->out[s], cnt * 4, cudaMemcpyDeviceToHost, st));
    }
    int rc2 = drain(p, op);
    return rc ? rc : rc2;
}

int oxide_pipe_rms_norm_f32(oxide_pipe_t p, const float* x, const float* w, float* out,
                            uint64_t rows, uint64_t cols, float eps) {
    const char* op = "oxide_pipe_rms_norm_f32";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (rows == 0) return OXIDE_OK;
    if (!x || !w || !out) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    if (cols == 0 || cols * sizeof(float) > p->chunk_bytes)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED, "%s: a row must fit in one pipe chunk", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t rows_per = p->chunk_bytes / (cols * sizeof(float));
    int rc = upload_bcast(p, op, w, cols * sizeof(float), nullptr, 0);
    if (rc) {
        drain(p, op);
        return rc;
    }
    uint64_t c = 0;
    for (uint64_t r0 = 0; r0 < rows && rc == OXIDE_OK; r0 += rows_per, ++c) {
        const uint64_t nr = rows - r0 < rows_per ? rows - r0 : rows_per;
        const int s = (int)(c % p->depth);
        cudaStream_t st = p->streams[s];
        const uint64_t bytes = nr * cols * sizeof(float);
        STEP(cudaMemcpyAsync(p->in0[s], x + r0 * cols, bytes, cudaMemcpyHostToDevice, st));
        if (rc == OXIDE_OK) rc = oxide_rms_norm_f32(static_cast<const float*>(p->in0[s]),
                                static_cast<const float*>(p->bc0), static_cast<float*>(p->out[s]),
                                nr, cols, eps, st);
        STEP(cudaMemcpyAsync(out + r0 * cols, p->out[s], bytes, cudaMemcpyDeviceToHost, st));
    }
    int rc2 = drain(p, op);
    return rc ? rc : rc2;
}

}  // extern "C"
