// Peer-GPU plumbing for the fused all-gather (one process per GPU):
//   * the bounded wait kernel that holds a stream until every rank's flag
//     has reached the call's number;
//   * device buffers that other processes can map (CUDA IPC handles).
// Every wait here is bounded by %globaltimer; a flag that never arrives
// turns into an error word and a DNNOPT_STATUS_KERNEL_TIMEOUT status, never a
// hung stream.
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

// Launched as a programmatic dependent of the kernel before it on the
// stream (the fused GEMM), so its spin overlaps that kernel's tail; the
// griddepcontrol.wait at the end keeps it from completing before that kernel.
// It releases its own dependents at entry: they launch early and wait (in
// their griddepcontrol.wait) for this kernel's completion, which hides their
// launch latency.
__global__ void __launch_bounds__(32)
peer_wait_kernel(const uint32_t* __restrict__ flag, int world, uint32_t epoch, uint32_t* seq,
                 uint64_t timeout_ns, uint32_t* err) {
    pdl_launch_dependents();
    const int q = threadIdx.x;
    const uint32_t want = seq ? *seq + 1u : epoch;
    if (q < world) {
        const uint64_t t0 = global_timer_ns();
        // Call numbers increase by one per call; the signed difference tolerates wrap.
        while (static_cast<int32_t>(ld_acquire_sys_u32(&flag[q]) - want) < 0) {
            if (global_timer_ns() - t0 > timeout_ns) {
                record_kernel_error(err, kKerrPeerTimeout);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
    pdl_wait();
    if (seq && q == 0) *seq = want;   // read by the next call's GEMM (stream order)
}

}  // namespace

cudaError_t launch_peer_wait(const uint32_t* flag, int world, uint32_t epoch, uint32_t* seq,
                             uint64_t timeout_ns, uint32_t* err, cudaStream_t s) {
    if (!flag || world < 1 || world > kAllGatherMaxRanks) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, 1);
    cfg.blockDim = dim3(32, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, peer_wait_kernel, flag, world, epoch, seq, timeout_ns, err);
}

}  // namespace dnnopt_b200
