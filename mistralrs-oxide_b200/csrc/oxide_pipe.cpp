// oxide_pipe.cpp -- host-buffer execution of ops with overlapped copies.
//
// The reference's ops consume and produce host tensors (src/ops/*: inputs
// read through Storage::as_f32_slice, outputs from Tensor::zeros), and its GPU
// backend moves data with CudaBackend::copy_host_to_device /
// copy_device_to_host (src/cuda_backend/mod.rs:76-85).  A pipeline runs ops on
// host buffers end to end: the rows are cut into chunks, chunk c goes to the
// next stream in round-robin order, and on each stream the host->device copy,
// the kernel(s) and the device->host copy of a chunk are enqueued in order.
// With depth >= 3 the upload of one chunk, the kernel of the next and the
// download of a third overlap, so an op runs at the PCIe copy rate rather
// than copy + compute.
//
// Staging buffers are allocated once in oxide_pipe_create; the op calls only
// enqueue copies and kernels.  By default each op waits for its own streams
// before returning.  In deferred mode (oxide_pipe_defer) op calls return once
// their work is enqueued and oxide_pipe_sync waits for all of it, so the
// uploads of one op overlap the downloads of the one before; the round-robin
// stream order carries over from op to op, and stream order alone keeps a
// staging buffer from being refilled before its download has left.
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
    bool defer = false;
    uint64_t next = 0;  // round-robin position of the next chunk
    std::vector<cudaStream_t> streams;
    std::vector<void*> in0, in1, out, out2;  // per-stream staging, chunk_bytes each
    std::vector<cudaEvent_t> tail;           // per-stream marker for the broadcast barrier
    void* bc0 = nullptr;                     // broadcast operands, chunk_bytes each
    void* bc1 = nullptr;
    void* bc2 = nullptr;
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
// Enqueue a library entry point (returns an oxide status).
#define KSTEP(call)                       \
    do {                                  \
        if (rc == OXIDE_OK) rc = (call);  \
    } while (0)

void release(oxide_pipe* p) {
    for (cudaStream_t s : p->streams)
        if (s) cudaStreamSynchronize(s);
    for (auto* v : {&p->in0, &p->in1, &p->out, &p->out2})
        for (void* b : *v) cudaFree(b);
    for (void* b : {p->bc0, p->bc1, p->bc2})
        if (b) cudaFree(b);
    for (cudaEvent_t e : p->tail)
        if (e) cudaEventDestroy(e);
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

// End of an op call: an error always drains (nothing of the call may still
// run after it returns); otherwise drain unless the pipe is deferred.
int finish(oxide_pipe* p, const char* op, int rc) {
    if (rc != OXIDE_OK) {
        drain(p, op);
        return rc;
    }
    return p->defer ? OXIDE_OK : drain(p, op);
}

// Upload the broadcast operands (if any) on stream 0 and make every stream
// wait for them.  Stream 0 first waits for the work already enqueued on the
// other streams: in deferred mode an earlier op's kernels may still read the
// broadcast buffers this upload overwrites.
int upload_bcast(oxide_pipe* p, const char* op, const void* h0, uint64_t b0, const void* h1,
                 uint64_t b1, const void* h2 = nullptr, uint64_t b2 = 0) {
    if (!h0 && !h1 && !h2) return OXIDE_OK;
    for (int i = 1; i < p->depth; ++i) {
        PIPE_CUDA(op, cudaEventRecord(p->tail[i], p->streams[i]));
        PIPE_CUDA(op, cudaStreamWaitEvent(p->streams[0], p->tail[i], 0));
    }
    if (h0) PIPE_CUDA(op, cudaMemcpyAsync(p->bc0, h0, b0, cudaMemcpyHostToDevice, p->streams[0]));
    if (h1) PIPE_CUDA(op, cudaMemcpyAsync(p->bc1, h1, b1, cudaMemcpyHostToDevice, p->streams[0]));
    if (h2) PIPE_CUDA(op, cudaMemcpyAsync(p->bc2, h2, b2, cudaMemcpyHostToDevice, p->streams[0]));
    PIPE_CUDA(op, cudaEventRecord(p->bc_ready, p->streams[0]));
    for (int i = 1; i < p->depth; ++i)
        PIPE_CUDA(op, cudaStreamWaitEvent(p->streams[i], p->bc_ready, 0));
    return OXIDE_OK;
}

// The staging set of the next chunk in round-robin order.
struct Stage {
    cudaStream_t st;
    void *in0, *in1, *out, *out2;
};
Stage next_stage(oxide_pipe* p) {
    const int s = (int)(p->next++ % (uint64_t)p->depth);
    return Stage{p->streams[s], p->in0[s], p->in1[s], p->out[s], p->out2[s]};
}

template <typename T>
T* as(void* v) {
    return static_cast<T*>(v);
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
    p->tail.assign(depth, nullptr);
    for (auto* v : {&p->in0, &p->in1, &p->out, &p->out2}) v->assign(depth, nullptr);
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < depth && e == cudaSuccess; ++i) {
        e = cudaStreamCreateWithFlags(&p->streams[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->tail[i], cudaEventDisableTiming);
        for (auto* v : {&p->in0, &p->in1, &p->out, &p->out2})
            if (e == cudaSuccess) e = cudaMalloc(&(*v)[i], chunk_bytes);
    }
    for (void** b : {&p->bc0, &p->bc1, &p->bc2})
        if (e == cudaSuccess) e = cudaMalloc(b, chunk_bytes);
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

int oxide_pipe_defer(oxide_pipe_t p, int on) {
    const char* op = "oxide_pipe_defer";
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    std::lock_guard<std::mutex> lk(p->mu);
    int rc = OXIDE_OK;
    if (!on && p->defer) {  // leaving deferred mode completes what is queued
        DeviceGuard g(p->device);
        rc = drain(p, op);
    }
    p->defer = on != 0;
    return rc;
}

int oxide_pipe_sync(oxide_pipe_t p) {
    const char* op = "oxide_pipe_sync";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    return drain(p, op);
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
    for (uint64_t lo = 0; lo < n && rc == OXIDE_OK; lo += chunk) {
        const uint64_t cnt = n - lo < chunk ? n - lo : chunk;
        const Stage s = next_stage(p);
        const float* da = as<const float>(p->bc0);
        const float* db = as<const float>(p->bc1);
        if (na == n) {
            STEP(cudaMemcpyAsync(s.in0, a + lo, cnt * 4, cudaMemcpyHostToDevice, s.st));
            da = as<const float>(s.in0);
        }
        if (nb == n) {
            STEP(cudaMemcpyAsync(s.in1, b + lo, cnt * 4, cudaMemcpyHostToDevice, s.st));
            db = as<const float>(s.in1);
        }
        KSTEP(oxide_binary_f32(bop, da, na == n ? cnt : na, db, nb == n ? cnt : nb, as<float>(s.out), cnt,
                               s.st));
        STEP(cudaMemcpyAsync(out + lo, s.out, cnt * 4, cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
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
    for (uint64_t lo = 0; lo < n && rc == OXIDE_OK; lo += chunk) {
        const uint64_t cnt = n - lo < chunk ? n - lo : chunk;
        const Stage s = next_stage(p);
        STEP(cudaMemcpyAsync(s.in0, gate + lo, cnt * 4, cudaMemcpyHostToDevice, s.st));
        STEP(cudaMemcpyAsync(s.in1, up + lo, cnt * 4, cudaMemcpyHostToDevice, s.st));
        KSTEP(oxide_silu_mul_f32(as<const float>(s.in0), as<const float>(s.in1), as<float>(s.out), cnt, s.st));
        STEP(cudaMemcpyAsync(out + lo, s.out, cnt * 4, cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
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
    for (uint64_t r0 = 0; r0 < rows && rc == OXIDE_OK; r0 += rows_per) {
        const uint64_t nr = rows - r0 < rows_per ? rows - r0 : rows_per;
        const Stage s = next_stage(p);
        const uint64_t bytes = nr * cols * sizeof(float);
        STEP(cudaMemcpyAsync(s.in0, x + r0 * cols, bytes, cudaMemcpyHostToDevice, s.st));
        KSTEP(oxide_rms_norm_f32(as<const float>(s.in0), as<const float>(p->bc0), as<float>(s.out), nr, cols,
                                 eps, s.st));
        STEP(cudaMemcpyAsync(out + r0 * cols, s.out, bytes, cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
}

int oxide_pipe_add_mul_rowbcast_f32(oxide_pipe_t p, const float* a, const float* b, const float* s_host,
                                    float* h, float* y, uint64_t rows, uint64_t cols) {
    const char* op = "oxide_pipe_add_mul_rowbcast_f32";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (rows == 0) return OXIDE_OK;
    if (!a || !b || !s_host || !h || !y) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    if (cols == 0 || cols * sizeof(float) > p->chunk_bytes)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED, "%s: a row must fit in one pipe chunk", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t rows_per = p->chunk_bytes / (cols * sizeof(float));
    int rc = upload_bcast(p, op, s_host, cols * sizeof(float), nullptr, 0);
    for (uint64_t r0 = 0; r0 < rows && rc == OXIDE_OK; r0 += rows_per) {
        const uint64_t nr = rows - r0 < rows_per ? rows - r0 : rows_per;
        const Stage s = next_stage(p);
        const uint64_t n = nr * cols, bytes = n * sizeof(float), off = r0 * cols;
        STEP(cudaMemcpyAsync(s.in0, a + off, bytes, cudaMemcpyHostToDevice, s.st));
        STEP(cudaMemcpyAsync(s.in1, b + off, bytes, cudaMemcpyHostToDevice, s.st));
        KSTEP(oxide_add_f32(as<const float>(s.in0), as<const float>(s.in1), as<float>(s.out), n, s.st));
        KSTEP(oxide_mul_rowbcast_f32(as<const float>(s.out), as<const float>(p->bc0), as<float>(s.out2), nr, cols,
                                     s.st));
        STEP(cudaMemcpyAsync(h + off, s.out, bytes, cudaMemcpyDeviceToHost, s.st));
        STEP(cudaMemcpyAsync(y + off, s.out2, bytes, cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
}

}  // extern "C"

// h = x + r, y = rms_norm(h) on host rows (f32 and bf16 share the body).
template <typename T, typename F>
static int pipe_add_rms_norm(const char* op, oxide_pipe_t p, const T* x, const T* r, const T* w, T* h, T* y,
                             uint64_t rows, uint64_t cols, float eps, F kernel) {
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (rows == 0) return OXIDE_OK;
    if (!x || !r || !w || !h || !y) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    if (cols == 0 || cols * sizeof(T) > p->chunk_bytes)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED, "%s: a row must fit in one pipe chunk", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t rows_per = p->chunk_bytes / (cols * sizeof(T));
    int rc = upload_bcast(p, op, w, cols * sizeof(T), nullptr, 0);
    for (uint64_t r0 = 0; r0 < rows && rc == OXIDE_OK; r0 += rows_per) {
        const uint64_t nr = rows - r0 < rows_per ? rows - r0 : rows_per;
        const Stage s = next_stage(p);
        const uint64_t bytes = nr * cols * sizeof(T), off = r0 * cols;
        STEP(cudaMemcpyAsync(s.in0, x + off, bytes, cudaMemcpyHostToDevice, s.st));
        STEP(cudaMemcpyAsync(s.in1, r + off, bytes, cudaMemcpyHostToDevice, s.st));
        KSTEP(kernel(as<const T>(s.in0), as<const T>(s.in1), as<const T>(p->bc0), as<T>(s.out), as<T>(s.out2), nr,
                     cols, eps, s.st));
        STEP(cudaMemcpyAsync(h + off, s.out, bytes, cudaMemcpyDeviceToHost, s.st));
        STEP(cudaMemcpyAsync(y + off, s.out2, bytes, cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
}

extern "C" {

int oxide_pipe_add_rms_norm_f32(oxide_pipe_t p, const float* x, const float* r, const float* w, float* h,
                                float* y, uint64_t rows, uint64_t cols, float eps) {
    return pipe_add_rms_norm<float>("oxide_pipe_add_rms_norm_f32", p, x, r, w, h, y, rows, cols, eps,
                                    oxide_add_rms_norm_f32);
}
int oxide_pipe_add_rms_norm_bf16(oxide_pipe_t p, const oxide_bf16* x, const oxide_bf16* r, const oxide_bf16* w,
                                 oxide_bf16* h, oxide_bf16* y, uint64_t rows, uint64_t cols, float eps) {
    return pipe_add_rms_norm<oxide_bf16>("oxide_pipe_add_rms_norm_bf16", p, x, r, w, h, y, rows, cols, eps,
                                         oxide_add_rms_norm_bf16);
}

int oxide_pipe_argmax_rows_f32(oxide_pipe_t p, const float* x, uint64_t rows, uint64_t cols, uint32_t* idx) {
    const char* op = "oxide_pipe_argmax_rows_f32";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (rows == 0) return OXIDE_OK;
    if (!x || !idx) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    if (cols == 0 || cols * sizeof(float) > p->chunk_bytes)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED, "%s: a row must fit in one pipe chunk", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t rows_per = p->chunk_bytes / (cols * sizeof(float));
    int rc = OXIDE_OK;
    for (uint64_t r0 = 0; r0 < rows && rc == OXIDE_OK; r0 += rows_per) {
        const uint64_t nr = rows - r0 < rows_per ? rows - r0 : rows_per;
        const Stage s = next_stage(p);
        STEP(cudaMemcpyAsync(s.in0, x + r0 * cols, nr * cols * sizeof(float), cudaMemcpyHostToDevice, s.st));
        KSTEP(oxide_argmax_rows_f32(as<const float>(s.in0), nr, cols, as<uint32_t>(s.out), s.st));
        STEP(cudaMemcpyAsync(idx + r0, s.out, nr * sizeof(uint32_t), cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
}

int oxide_pipe_scale_mask_softmax_f32(oxide_pipe_t p, const float* x, float* out, uint64_t rows, uint64_t cols,
                                      float scale, const float* mask, uint64_t mask_len, const int32_t* lens,
                                      uint64_t rows_per_len, uint64_t causal_q_len) {
    const char* op = "oxide_pipe_scale_mask_softmax_f32";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (rows == 0) return OXIDE_OK;
    if (!x || !out) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    if (lens && rows_per_len == 0)
        return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: rows_per_len must be >= 1 with lens", op);
    if (mask && (mask_len == 0 || mask_len * sizeof(float) > p->chunk_bytes))
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED, "%s: mask must be non-empty and fit in one pipe chunk", op);
    const uint64_t groups = lens ? (rows + rows_per_len - 1) / rows_per_len : 0;
    if (groups * sizeof(int32_t) > p->chunk_bytes)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED, "%s: lens must fit in one pipe chunk", op);
    // Chunks hold whole lens groups and whole causal blocks, so chunk-local
    // rows keep their group (r / rows_per_len) and query (r % causal_q_len).
    uint64_t unit = 1;
    if (lens) unit = std::lcm(unit, rows_per_len);
    if (causal_q_len) unit = std::lcm(unit, causal_q_len);
    const uint64_t cap_rows = cols && cols * sizeof(float) <= p->chunk_bytes ? p->chunk_bytes / (cols * sizeof(float)) : 0;
    if (cap_rows < unit)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED,
                                "%s: %llu rows of %llu keys (one lens group / causal block) exceed the pipe chunk",
                                op, (unsigned long long)unit, (unsigned long long)cols);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t rows_per = cap_rows / unit * unit;
    int rc = upload_bcast(p, op, mask, mask_len * sizeof(float), lens, groups * sizeof(int32_t));
    const size_t pitch = cols * sizeof(float);
    for (uint64_t r0 = 0; r0 < rows && rc == OXIDE_OK; r0 += rows_per) {
        const uint64_t nr = rows - r0 < rows_per ? rows - r0 : rows_per;
        const Stage s = next_stage(p);
        if (lens) {
            // Upload only the keys the kernel reads: the first lens[g] of each
            // row of group g, one strided copy per group.
            for (uint64_t gr = r0; gr < r0 + nr && rc == OXIDE_OK; gr += rows_per_len) {
                const int64_t lg = lens[gr / rows_per_len];
                const uint64_t valid = lg <= 0 ? 0 : ((uint64_t)lg < cols ? (uint64_t)lg : cols);
                const uint64_t h = (r0 + nr - gr) < rows_per_len ? (r0 + nr - gr) : rows_per_len;
                if (valid)
                    STEP(cudaMemcpy2DAsync(as<float>(s.in0) + (gr - r0) * cols, pitch, x + gr * cols, pitch,
                                           valid * sizeof(float), h, cudaMemcpyHostToDevice, s.st));
            }
        } else {
            STEP(cudaMemcpyAsync(s.in0, x + r0 * cols, nr * pitch, cudaMemcpyHostToDevice, s.st));
        }
        KSTEP(oxide_scale_mask_softmax_f32(as<const float>(s.in0), as<float>(s.out), nr, cols, scale,
                                           mask ? as<const float>(p->bc0) : nullptr, mask_len,
                                           lens ? as<const int32_t>(p->bc1) + r0 / rows_per_len : nullptr,
                                           rows_per_len, causal_q_len, s.st));
        STEP(cudaMemcpyAsync(out + r0 * cols, s.out, nr * pitch, cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
}

int oxide_pipe_rope_bf16(oxide_pipe_t p, const oxide_bf16* q, oxide_bf16* q_out, uint64_t q_heads,
                         const oxide_bf16* k, oxide_bf16* k_out, uint64_t k_heads, const float* cos_t,
                         const float* sin_t, uint64_t table_rows, const int32_t* positions, uint64_t tokens,
                         uint64_t head_dim) {
    const char* op = "oxide_pipe_rope_bf16";
    if (int inj = oxide::injected_failure(op)) return inj;
    if (!p) return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pipe", op);
    if (tokens == 0) return OXIDE_OK;
    if (!q || !q_out || !cos_t || !sin_t || (k && !k_out))
        return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: null pointer", op);
    if (!k) k_heads = 0;
    if (head_dim < 2 || head_dim % 2 || q_heads == 0 || table_rows == 0)
        return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: bad head_dim, head count or table", op);
    if (!positions && table_rows < tokens)
        return oxide::set_error(OXIDE_ERR_INVALID_ARG, "%s: table_rows < tokens without positions", op);
    const uint64_t half = head_dim / 2;
    const uint64_t qtok = q_heads * head_dim * sizeof(oxide_bf16), ktok = k_heads * head_dim * sizeof(oxide_bf16);
    const uint64_t tab = table_rows * half * sizeof(float);
    if (qtok > p->chunk_bytes || ktok > p->chunk_bytes || tab > p->chunk_bytes ||
        tokens * sizeof(int32_t) > p->chunk_bytes)
        return oxide::set_error(OXIDE_ERR_UNSUPPORTED, "%s: a token's heads, the tables and the positions must "
                                "each fit in one pipe chunk", op);
    std::lock_guard<std::mutex> lk(p->mu);
    DeviceGuard g(p->device);
    const uint64_t per = p->chunk_bytes / (qtok > ktok ? qtok : ktok);
    int rc = upload_bcast(p, op, cos_t, tab, sin_t, tab, positions, positions ? tokens * sizeof(int32_t) : 0);
    for (uint64_t t0 = 0; t0 < tokens && rc == OXIDE_OK; t0 += per) {
        const uint64_t nt = tokens - t0 < per ? tokens - t0 : per;
        const Stage s = next_stage(p);
        const uint64_t qoff = t0 * q_heads * head_dim, koff = t0 * k_heads * head_dim;
        STEP(cudaMemcpyAsync(s.in0, q + qoff, nt * qtok, cudaMemcpyHostToDevice, s.st));
        if (k) STEP(cudaMemcpyAsync(s.in1, k + koff, nt * ktok, cudaMemcpyHostToDevice, s.st));
        // Without positions token t uses table row t: offset the tables by the
        // chunk's first token (table_rows >= tokens, checked above).
        const float* c = as<const float>(p->bc0);
        const float* sn = as<const float>(p->bc1);
        uint64_t trows = table_rows;
        const int32_t* pos = positions ? as<const int32_t>(p->bc2) + t0 : nullptr;
        if (!positions) {
            c += t0 * half;
            sn += t0 * half;
            trows = table_rows - t0;
        }
        KSTEP(oxide_rope_bf16(as<const oxide_bf16>(s.in0), as<oxide_bf16>(s.in0), q_heads,
                              k ? as<const oxide_bf16>(s.in1) : nullptr, k ? as<oxide_bf16>(s.in1) : nullptr, k_heads,
                              c, sn, trows, pos, nt, head_dim, 0, s.st));
        STEP(cudaMemcpyAsync(q_out + qoff, s.in0, nt * qtok, cudaMemcpyDeviceToHost, s.st));
        if (k) STEP(cudaMemcpyAsync(k_out + koff, s.in1, nt * ktok, cudaMemcpyDeviceToHost, s.st));
    }
    return finish(p, op, rc);
}

}  // extern "C"
