// oxide_runtime.cu -- status codes, per-thread error messages, host-side
// fault injection and cached device attributes shared by every entry point.
//
// The status convention mirrors the reference's error model
// (src/cuda_backend/errors.rs:10-31 CudaError, src/error.rs:3-45 OxideError):
// every failure is returned to the caller, none aborts the process.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "oxide_common.cuh"

namespace oxide {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* op) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return OXIDE_OK;
    return set_error(OXIDE_ERR_LAUNCH, "%s: launch failed: %s", op, cudaGetErrorString(e));
}

// Fault injection: one armed operation name, consumed by the first matching
// entry point.  Guarded by a mutex; the fast path is one relaxed atomic load.
static std::atomic<bool> g_inject_armed{false};
static std::mutex g_inject_mu;
static std::string g_inject_op;

int injected_failure(const char* op) {
    if (!g_inject_armed.load(std::memory_order_relaxed)) return 0;
    std::lock_guard<std::mutex> lk(g_inject_mu);
    if (!g_inject_armed.load(std::memory_order_relaxed)) return 0;
    if (g_inject_op == "*" || g_inject_op == op) {
        g_inject_armed.store(false, std::memory_order_relaxed);
        g_inject_op.clear();
        return set_error(OXIDE_ERR_INJECTED, "%s: injected failure", op);
    }
    return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("OXIDE_NO_PDL");
        return !(v && v[0] == '1');
    }();
    return on;
}

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int resident_blocks(const void* kernel, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, std::pair<const void*, std::pair<int, size_t>>>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    auto key = std::make_pair(dev, std::make_pair(kernel, std::make_pair(threads, smem)));
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
            cudaSuccess ||
        per_sm <= 0) {
        cudaGetLastError();  // clear the sticky-free error of a failed query
        per_sm = 1;
    }
    int blocks = per_sm * sm_count();
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = blocks;
    return blocks;
}

bool ensure_dyn_smem(const void* kernel, size_t smem) {
    if (smem <= 48 * 1024) return true;
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, size_t> done;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_pair(dev, kernel);
    std::lock_guard<std::mutex> lk(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= smem) return true;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    done[key] = smem;
    return true;
}

// Driver API entry points, resolved through the runtime (the library links
// only the static CUDA runtime, not libcuda directly).  nullptr if absent.
void* driver_fn(const char* symbol) {
    static std::mutex mu;
    static std::map<std::string, void*> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(symbol);
    if (it != cache.end()) return it->second;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint(symbol, &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        fn = nullptr;
    }
    cache[symbol] = fn;
    return fn;
}

// Unique id of the calling thread's current CUDA context (cuCtxGetId): a
// context created after a cudaDeviceReset gets a new id even where the
// driver reuses the old handle's address.  0 if there is none or the driver
// lacks the call.
unsigned long long current_context_id() {
    typedef int (*GetCurrent)(void**);
    typedef int (*GetId)(void*, unsigned long long*);
    static GetCurrent get_current = reinterpret_cast<GetCurrent>(driver_fn("cuCtxGetCurrent"));
    static GetId get_id = reinterpret_cast<GetId>(driver_fn("cuCtxGetId"));
    if (!get_current || !get_id) return 0;
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
    return id;
}

// Self-test: RowDiv(b)(a) against the IEEE quotient for every pair (a_i, b_j).
// out[0] counts the mismatching pairs, out[1] keeps the smallest mismatching
// pair index (i * nb + j); the caller sets out = {0, UINT64_MAX} first.
__global__ void __launch_bounds__(256)
    selftest_rowdiv_kernel(const float* a, uint64_t na, const float* b, uint64_t nb,
                           unsigned long long* out) {
    pdl_begin();
    const uint64_t total = na * nb;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = t / nb, j = t % nb;
        const RowDiv d(b[j]);
        const float q = d(a[i]);
        const float ref = __fdiv_rn(a[i], b[j]);
        const bool same = __float_as_uint(q) == __float_as_uint(ref) || (q != q && ref != ref);
        if (!same) {
            atomicAdd(&out[0], 1ull);
            atomicMin(&out[1], (unsigned long long)t);
        }
    }
}

}  // namespace oxide

extern "C" {

int oxide_selftest_rowdiv(const float* a, uint64_t na, const float* b, uint64_t nb,
                          unsigned long long* out, oxide_stream_t stream) {
    const char* name = "oxide_selftest_rowdiv";
    OXIDE_INJECT(name);
    OXIDE_REQUIRE(out, name, "null output pointer");
    if (na == 0 || nb == 0) return OXIDE_OK;
    OXIDE_REQUIRE(a && b, name, "null pointer");
    OXIDE_REQUIRE(na <= UINT64_MAX / nb, name, "na * nb overflows");
    oxide::launch_k(oxide::selftest_rowdiv_kernel, oxide::sm_count() * 8, 256, 0, stream, a, na, b, nb, out);
    return oxide::check_launch(name);
}

const char* oxide_status_string(int status) {
    switch (status) {
        case OXIDE_OK: return "OXIDE_OK";
        case OXIDE_ERR_INVALID_ARG: return "OXIDE_ERR_INVALID_ARG";
        case OXIDE_ERR_LAUNCH: return "OXIDE_ERR_LAUNCH";
        case OXIDE_ERR_UNSUPPORTED: return "OXIDE_ERR_UNSUPPORTED";
        case OXIDE_ERR_CUDA: return "OXIDE_ERR_CUDA";
        case OXIDE_ERR_WORKSPACE: return "OXIDE_ERR_WORKSPACE";
        case OXIDE_ERR_INJECTED: return "OXIDE_ERR_INJECTED";
        case OXIDE_ERR_TIMEOUT: return "OXIDE_ERR_TIMEOUT";
        default: return "OXIDE_ERR_UNKNOWN";
    }
}

const char* oxide_last_error(void) { return oxide::g_last_error; }

const char* oxide_version(void) { return "oxide-b200 0.1.0 (sm_100a)"; }

void oxide_debug_fail_next(const char* op) {
    std::lock_guard<std::mutex> lk(oxide::g_inject_mu);
    if (op == nullptr) {
        oxide::g_inject_op.clear();
        oxide::g_inject_armed.store(false);
    } else {
        oxide::g_inject_op = op;
        oxide::g_inject_armed.store(true);
    }
}

}  // extern "C"
