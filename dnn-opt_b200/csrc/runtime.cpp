// Host runtime: device contexts, per-stream workspace, staging buffers,
// status bookkeeping and host-side fault injection.
#include "runtime.h"

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>

namespace dnnopt_b200 {

namespace {

thread_local int t_last_status = DNNOPT_STATUS_SUCCESS;
std::atomic<uint64_t> g_launches{0};

std::mutex g_ctx_mu;
std::unordered_map<int, std::unique_ptr<DeviceContext>> g_ctx;

// Fault injection state: pending counts per site (1..3).
std::mutex g_fault_mu;
int g_fault_pending[4] = {0, 0, 0, 0};
bool g_fault_env_read = false;

void read_fault_env_locked() {
    if (g_fault_env_read) return;
    g_fault_env_read = true;
    const char* s = std::getenv("DNNOPT_FAULT_INJECT");
    if (!s) return;
    int site = 0, count = 0;
    if (std::sscanf(s, "%d:%d", &site, &count) == 2 && site >= 1 && site <= 3 && count > 0)
        g_fault_pending[site] = count;
}

template <typename T>
cudaError_t grow(T** p, size_t* have, size_t need) {
    if (need <= *have) return cudaSuccess;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    size_t alloc = need + need / 4;   // grow geometrically to avoid churn
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), alloc * sizeof(T));
    if (e != cudaSuccess) { *p = nullptr; return e; }
    *have = alloc;
    return cudaSuccess;
}

}  // namespace

int set_status(int st) {
    t_last_status = st;
    return st;
}

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return set_status(DNNOPT_STATUS_SUCCESS);
    if (e == cudaErrorMemoryAllocation) return set_status(DNNOPT_STATUS_ALLOC_FAILED);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
        return set_status(DNNOPT_STATUS_NO_DEVICE);
    return set_status(DNNOPT_STATUS_CUDA_ERROR);
}

void note_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

int check_injected_fault(int site) {
    std::lock_guard<std::mutex> lk(g_fault_mu);
    read_fault_env_locked();
    if (site < 1 || site > 3 || g_fault_pending[site] <= 0) return DNNOPT_STATUS_SUCCESS;
    --g_fault_pending[site];
    return DNNOPT_STATUS_INJECTED_FAULT;
}

DeviceContext* current_context(int* status) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *status = cuda_status(e == cudaErrorInvalidDevice ? cudaErrorNoDevice : e);
        if (*status == DNNOPT_STATUS_CUDA_ERROR) *status = set_status(DNNOPT_STATUS_NO_DEVICE);
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    auto it = g_ctx.find(dev);
    if (it != g_ctx.end()) { *status = DNNOPT_STATUS_SUCCESS; return it->second.get(); }
    auto ctx = std::make_unique<DeviceContext>();
    ctx->device = dev;
    e = cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) { *status = cuda_status(e); return nullptr; }
    e = cudaStreamCreateWithFlags(&ctx->default_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) { *status = cuda_status(e); return nullptr; }
    DeviceContext* raw = ctx.get();
    g_ctx.emplace(dev, std::move(ctx));
    *status = DNNOPT_STATUS_SUCCESS;
    return raw;
}

int ensure_workspace(DeviceContext* ctx, cudaStream_t stream, size_t ws_floats, size_t counters,
                     size_t quant_bytes, Workspace** out) {
    int inj = check_injected_fault(1);
    if (inj != DNNOPT_STATUS_SUCCESS) return set_status(inj);
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    Workspace& w = ctx->ws[stream];
    cudaError_t e;
    if (!w.err) {
        // err (word 0), absmax (words 4-5), the conv prep's grid-barrier
        // count and generation (words 6-7), scales (words 8-11) and the conv
        // prep's two absmax slots (words 12-15) share one small
        // zero-initialised allocation.
        void* small = nullptr;
        e = cudaMalloc(&small, 64);
        if (e != cudaSuccess) return cuda_status(e);
        e = cudaMemsetAsync(small, 0, 64, stream);
        if (e != cudaSuccess) { cudaFree(small); return cuda_status(e); }
        w.err = static_cast<uint32_t*>(small);
        w.absmax = w.err + 4;
        w.scales = reinterpret_cast<float*>(w.err + 8);
    }
    if ((e = grow(&w.ws, &w.ws_floats, ws_floats)) != cudaSuccess) return cuda_status(e);
    if (counters > w.n_counters) {
        size_t old = w.n_counters;
        (void)old;
        if ((e = grow(&w.counters, &w.n_counters, counters)) != cudaSuccess) return cuda_status(e);
        // Tickets must start at zero; kernels leave them at zero.
        e = cudaMemsetAsync(w.counters, 0, w.n_counters * sizeof(uint32_t), stream);
        if (e != cudaSuccess) return cuda_status(e);
    }
    if (quant_bytes > w.quant_bytes) {
        unsigned char* q = static_cast<unsigned char*>(w.quant);
        if ((e = grow(&q, &w.quant_bytes, quant_bytes)) != cudaSuccess) return cuda_status(e);
        w.quant = q;
    }
    *out = &w;
    return DNNOPT_STATUS_SUCCESS;
}

int ensure_stage(DeviceContext* ctx, int slot, size_t bytes, void** out) {
    int inj = check_injected_fault(1);
    if (inj != DNNOPT_STATUS_SUCCESS) return set_status(inj);
    unsigned char* p = static_cast<unsigned char*>(ctx->stage[slot]);
    cudaError_t e = grow(&p, &ctx->stage_bytes[slot], bytes);
    ctx->stage[slot] = p;
    if (e != cudaSuccess) return cuda_status(e);
    *out = p;
    return DNNOPT_STATUS_SUCCESS;
}

PtrKind classify_pointer(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return PtrKind::Host;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return PtrKind::Device;
    return PtrKind::Host;
}

}  // namespace dnnopt_b200

using namespace dnnopt_b200;

extern "C" {

int dnnopt_get_last_error(void) { return t_last_status; }

const char* dnnopt_status_string(int s) {
    switch (s) {
        case DNNOPT_STATUS_SUCCESS: return "success";
        case DNNOPT_STATUS_INVALID_VALUE: return "invalid value";
        case DNNOPT_STATUS_NOT_SUPPORTED: return "not supported";
        case DNNOPT_STATUS_CUDA_ERROR: return "CUDA error";
        case DNNOPT_STATUS_ALLOC_FAILED: return "allocation failed";
        case DNNOPT_STATUS_NO_DEVICE: return "no CUDA device";
        case DNNOPT_STATUS_KERNEL_TIMEOUT: return "in-kernel wait timed out";
        case DNNOPT_STATUS_INJECTED_FAULT: return "injected fault";
        case DNNOPT_STATUS_EXCEEDS_SCRATCH: return "request exceeds the fixed scratch area";
        default: return "unknown status";
    }
}

uint64_t dnnopt_launch_count(void) { return g_launches.load(); }

int dnnopt_debug_inject_fault(int site, int count) {
    if (site < 1 || site > 3 || count < 0) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    std::lock_guard<std::mutex> lk(g_fault_mu);
    read_fault_env_locked();
    g_fault_pending[site] = count;
    return set_status(DNNOPT_STATUS_SUCCESS);
}

int dnnopt_set_stream(void* stream) {
    int st;
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->user_stream = static_cast<cudaStream_t>(stream);
    ctx->user_stream_set = stream != nullptr;
    return set_status(DNNOPT_STATUS_SUCCESS);
}

}  // extern "C"
