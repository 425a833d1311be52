// Device-side helpers shared by the sm_100a kernels: scalar conversions,
// mbarrier / TMA / tcgen05 PTX wrappers, and the bounded-wait error flag.
//
// Every spin-wait in this library is bounded.  When a wait gives up it records
// a code in a device error word (passed to the kernel by the host and read back
// after the launch) and returns, so a lost arrival turns into an error status
// instead of a hung GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace dnnopt_b200 {

// ---------------------------------------------------------------------------
// Error word written by bounded waits.
// ---------------------------------------------------------------------------
enum KernelErrorCode : uint32_t {
    kKerrNone = 0,
    kKerrMbarTimeout = 1,      // an mbarrier wait exceeded its iteration limit
    kKerrTmemAlloc = 2,        // TMEM allocation returned an unusable address
    kKerrPeerTimeout = 3,      // a peer GPU's flag did not arrive within the limit
};

__device__ __forceinline__ void record_kernel_error(uint32_t* err, uint32_t code) {
    if (err) atomicCAS(err, 0u, code);
}

// Upper bound on the wait for one mbarrier phase.  A healthy pipeline
// completes a phase within microseconds; 2 s of %globaltimer only trips on a
// lost arrival.
constexpr uint64_t kMbarTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// Scalar conversions
// ---------------------------------------------------------------------------
// The bias pass of the oneDNN entry (integration/onednn/0001-dnnopt-integration.patch:355-362:
// C[i,j] += bias[i] on the column-major C, i.e. bias[n] on the row-major view),
// fused into the FP32 epilogues as its own rounding after alpha*acc + beta*C.
__device__ __forceinline__ float add_bias(float v, const float* bias, int64_t n) {
    return bias ? __fadd_rn(v, __ldg(bias + n)) : v;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Round-to-nearest-even FP32 -> BF16 bits, identical to the reference's
// bfloat16_t(float) constructor (include/dnnopt/gemm/gemm_types.h:18-24),
// including its treatment of NaN payloads and overflow.
__device__ __forceinline__ uint16_t f32_to_bf16_bits_ref(float f) {
    uint32_t u = __float_as_uint(f);
    uint32_t round = 0x7FFFu + ((u >> 16) & 1u);
    return static_cast<uint16_t>((u + round) >> 16);
}

__device__ __forceinline__ float round_to_bf16(float f) {
    return bf16_bits_to_f32(f32_to_bf16_bits_ref(f));
}

// Two OCP E4M3FN bytes (low byte = element 0) -> two exact FP32 values.
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint16_t two) {
    __half2_raw h;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(*reinterpret_cast<uint32_t*>(&h)) : "h"(two));
    __half2 hv = *reinterpret_cast<__half2*>(&h);
    return __half22float2(hv);
}

// ---------------------------------------------------------------------------
// Shared-memory address / mbarrier wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or `hint_ns` elapses, instead of re-issuing the probe.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records the error
// word) when the limit is reached.  `abort_flag` lets the other roles of a
// warp-specialised kernel skip their remaining waits once one has failed.
// Between probes the thread sleeps in hardware (suspend-time hint, woken when
// the phase completes), so waiting warps take no issue slots or shared-memory
// bandwidth from the warps that feed the tensor cores (measured on B200: 128
// threads polling without the hint slowed a TMA + tcgen05 pipeline's stages
// from about 0.3 to 0.55 us each).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile uint32_t* abort_flag, uint32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (abort_flag && *abort_flag) return false;
        if ((i & 15u) == 0 && global_timer_ns() - t0 > kMbarTimeoutNs) break;
    }
    record_kernel_error(err, kKerrMbarTimeout);
    if (abort_flag) *abort_flag = 1u;
    return false;
}

// The same wait for a whole warp: lane 0 waits, the result is broadcast.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               volatile uint32_t* abort_flag, uint32_t* err) {
    uint32_t ok = 0;
    if ((threadIdx.x & 31u) == 0) ok = mbar_wait(bar, parity, abort_flag, err) ? 1u : 0u;
    return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor): every load lands in the issuing CTA's shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory, completing on `bar`
// (complete_tx).  Both addresses 16-byte aligned, `bytes` a multiple of 16.
// Efficient for copies of a few KB; at ~0.5 KB the per-copy cost dominates.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes,
                                             uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int32_t x,
                                             int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
        "r"(smem_u32(smem_src)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/f16 inputs, f32 accumulate).
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma previously issued by this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// canonical 128-byte-swizzled layout: rows of 128 B (64 bf16 along K), eight
// rows per 1024-B swizzle atom, atoms stacked densely along M/N.
//   bits  0-13 start address >> 4
//   bits 16-29 leading byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout: 2 = SWIZZLE_128B
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor, kind::f16 with BF16 A/B, F32 D, both K-major.
//   bits 4-5 D format (1 = F32); 7-9 A format (1 = BF16); 10-12 B format;
//   15/16 A/B major (0 = K); 17-22 N >> 3; 24-28 M >> 4.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Flag and counter accesses with explicit scope (peer GPUs signal each other
// through mapped memory).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void st_relaxed_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu_u32(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---------------------------------------------------------------------------
// Thread-block clusters (distributed shared memory) and programmatic
// dependent launch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
    return v;
}

// Programmatic dependent launch: wait until the preceding grid on the stream
// has completed and its memory is visible (no-op without the launch
// attribute), and allow the next grid to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
        "elect.sync rx|px, %1;\n\t"
        "@px mov.s32 %0, 1;\n\t}"
        : "+r"(pred)
        : "r"(0xFFFFFFFFu));
    return pred != 0;
}

}  // namespace dnnopt_b200
