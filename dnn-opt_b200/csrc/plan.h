// Plan selector: the B200 replacement of the reference's shape dispatcher
// (src/gemm/gemm.cpp:168-455) and CPU autotuner (src/gemm/gemm_autotune.cpp,
// src/autotune/shape_cache.cpp).  For each (kind, shape, layout) it picks a
// kernel family and its launch shape (split-K factor or grid), optionally by
// timing candidates (autotune), and caches the choice.
#pragma once

#include <cstdint>
#include <string>

#include "kernels.h"

namespace dnnopt_b200 {

enum class Kind : int {
    F32 = 0,        // gemm_fp32
    BF16F32 = 1,    // gemm_bf16_bf16bf16f32
    F32BF16R = 2,   // gemm_bf16 (FP32 API)
    F32S8Q = 3,     // gemm_int8 (FP32 API)
    S8S32 = 4,      // gemm_int8_int8int8int32
    E4M3BF16 = 5,   // config-5 decode-FFN weight GEMM
    RE4E5 = 6,      // gemm_fp8_e4m3
    RE5E5 = 7,      // gemm_fp8_e5m2
};

enum class KernelId : int {
    GemvKn = 0,     // small-M split-K, B K x N
    GemvNk = 1,     // small-M dot form, B N x K
    TileF32 = 2,    // general SIMT FP32-accumulate GEMM (gemm_simt.cu)
    TileS8 = 3,     // general SIMT int8 tile
    Bf16Tc = 4,     // tcgen05 tall-skinny BF16
    GemvNkRows = 5, // dot form over 8-row blocks of A (M > 8)
    GemvKnCluster = 6,  // small-M split-K, splits reduced in a thread-block cluster
    GemvRows = 7,   // small-M dot form with A in registers (aligned B rows, K <= 512 chunks)
    E4m3Tc = 8,     // config-5 e4m3 weights on tcgen05 (kind::f8f6f4), 8-row blocks of A
    GemvSlab = 9,   // small-M column slab, B K x N: whole K per CTA, no split-K reduction
    GemvPanel = 10, // small-M FP32 row panels, B K x N: 512-byte row segments, cluster K reduction
    GemvRowsBulk = 11,  // GemvRows with B rows staged by bulk copies in a shared-memory ring
    GemmTc = 12,    // general tcgen05 GEMM, both operands by TMA (int8 kind::i8, bf16 kind::f16)
};

struct Plan {
    KernelId kernel = KernelId::TileF32;
    GemvKnPlan kn{};
    GemvNkPlan nk{};
    E4m3TcPlan e4{};
    GemmSimtPlan simt{};
    TcPlan tc{};
    int slab_w = 8;      // GemvSlab: columns per CTA (8 or 16)
    int panel_w = 128;   // GemvPanel: columns per CTA (128 or 256)
    int panel_splits = 8;  // GemvPanel: K-ranges per panel = cluster size (1, 2, 4, 8)
    bool tuned = false;
};

struct DeviceInfo {
    int num_sms = 148;
    bool have_device = false;
};

// splits_hint <= 0: heuristic.  allow_cluster: may choose the cluster variant
// (splits <= 16, kchunk <= gemv_kn_cluster_max_chunk()).
GemvKnPlan kn_plan_for(Kind kind, const GemmArgs& g, const DeviceInfo& info, int splits_hint,
                       bool allow_cluster = true);
// The split rule behind kn_plan_for as a pure function of the shape, the M
// class, the B vector width, the kernel's resident CTAs per SM and the SM
// count (shared with the allocation-free entry point, which caches its own
// occupancy figures).
GemvKnPlan kn_plan_rule(const GemmArgs& g, int mt, int vec4, int occ, int num_sms, int splits_hint,
                        bool allow_cluster);
GemvNkPlan nk_plan_for(Kind kind, const GemmArgs& g, const DeviceInfo& info, int grid_hint);

// Heuristic plan (no timing).  Needs no device when info.have_device is false
// (occupancy is then estimated).
Plan heuristic_plan(Kind kind, const GemmArgs& g, const DeviceInfo& info);
const char* kernel_name(KernelId k);
std::string describe_plan(Kind kind, const GemmArgs& g, const Plan& p);

// Autotune cache: LRU of 256 plans keyed by FNV-1a, persisted as "DNNAUTO"
// version 5.
bool autotune_enabled();
void set_autotune_enabled(bool on);
uint64_t plan_key(Kind kind, const GemmArgs& g, int vec);
bool cache_lookup(uint64_t key, Plan* out);
void cache_store(uint64_t key, const Plan& p, float time_us);
int cache_save(const char* path);
int cache_load(const char* path);
int cache_entries();

// Element sizes of A and B for a kind (bytes).
int elem_bytes_a(Kind k);
int elem_bytes_b(Kind k);

}  // namespace dnnopt_b200
