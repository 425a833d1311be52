// Host runtime internals: per-device context, per-stream workspace, pinned /
// device staging for host-pointer calls, status bookkeeping and host-side
// fault injection.  Internal to libdnnopt_b200.so.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "dnnopt_b200.h"

namespace dnnopt_b200 {

// Scratch owned by one (device, stream) pair.  Everything grows on demand and
// is freed at process exit.
struct Workspace {
    float* ws = nullptr;            // split-K partial strips
    size_t ws_floats = 0;
    uint32_t* counters = nullptr;   // split-K tickets (kept zero between launches)
    size_t n_counters = 0;
    uint32_t* err = nullptr;        // bounded-wait error word
    uint32_t* absmax = nullptr;     // [2] absmax bit patterns (FP32-API int8), [2..3] grid-barrier words
    float* scales = nullptr;        // [2] sA, sB
    void* quant = nullptr;          // quantised copies of A and B
    size_t quant_bytes = 0;
};

struct DeviceContext {
    int device = -1;
    int num_sms = 0;
    cudaStream_t default_stream = nullptr;   // library-owned non-blocking stream
    cudaStream_t user_stream = nullptr;      // set by dnnopt_set_stream (host API)
    bool user_stream_set = false;
    std::mutex mu;                           // serialises host-API calls on this device
    std::unordered_map<cudaStream_t, Workspace> ws;
    // Device staging for host-pointer calls (host API).
    void* stage[4] = {nullptr, nullptr, nullptr, nullptr};
    size_t stage_bytes[4] = {0, 0, 0, 0};
    // Pinned host word that receives the stream's kernel error word in the
    // same stream as the result copy (host API), so a call syncs once.
    uint32_t* host_err = nullptr;
};

// Returns the context of the current device (creating it), or nullptr with
// *status set.
DeviceContext* current_context(int* status);

// Workspace for `stream` sized for at least the given amounts.
int ensure_workspace(DeviceContext* ctx, cudaStream_t stream, size_t ws_floats, size_t counters,
                     size_t quant_bytes, Workspace** out);

int ensure_stage(DeviceContext* ctx, int slot, size_t bytes, void** out);

// Status helpers.
int set_status(int st);                 // records as the thread's last status
int cuda_status(cudaError_t e);         // maps a CUDA error to a status (and records it)
void note_launch(int n = 1);            // library kernel launch counter

// Host-side fault injection (tests): returns DNNOPT_STATUS_INJECTED_FAULT
// while an injected fault of `site` is pending.
int check_injected_fault(int site);

// Pointer classification for host-API calls.
enum class PtrKind { Device, Host };
PtrKind classify_pointer(const void* p);

}  // namespace dnnopt_b200
