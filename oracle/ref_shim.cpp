// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// Link shim for building the reference's portable (non-ARM) GEMM path on an
// x86 host.  The reference's ARM-only layers (hwcaps detection, the
// micro-benchmark autotuner and the packed driver) either do not compile on
// x86 or deadlock there (the autotuner re-enters a non-recursive mutex while
// benchmarking: reference src/gemm/gemm_autotune.cpp:130,164).  This shim
// replaces exactly those entry points:
//
//   * detect_arm_hwcaps()            -> an empty profile (no NEON/SVE/SME)
//   * get_autotuned_profile()        -> the generic-default tuning profile
//   * get_current_thresholds()       -> the reference's default thresholds
//                                       (src/gemm/gemm.cpp:268-272)
//   * select_gemm_kernel()           -> kPacked (unused on x86: the switch that
//                                       reads it is under __ARM_NEON)
//   * get_autotuned_blocking_params()-> never reached (registry is empty)
//   * gemm_driver_generic()          -> never reached (registry is empty)
//
// With no micro-kernels registered (none of the NEON/SVE/SME TUs are built),
// dispatch_via_registry() returns false and every gemm_fp32() call resolves to
// the reference's own gemm_naive_fp32 (src/gemm/gemm.cpp:88-100, :376), which
// is the x86 path the reference itself takes once the autotuner is bypassed.
#include "dnnopt/arm_hwcaps.h"
#include "dnnopt/cpu_tuning_profile.h"
#include "dnnopt/gemm/gemm_autotune.h"
#include "dnnopt/gemm/gemm_driver_generic.h"

#include <cstdio>
#include <cstdlib>
#include <string>

namespace dnnopt {

const ArmHwProfile& detect_arm_hwcaps() {
    static ArmHwProfile p = [] {
        ArmHwProfile q;
        q.cpu_name = "x86-64 host (oracle shim)";
        q.num_cores = 1;
        return q;
    }();
    return p;
}

void print_hwcaps_summary(const ArmHwProfile& profile) {
    std::printf("%s\n", profile.cpu_name.c_str());
}

std::string platform_tag(const ArmHwProfile&) { return "x86_oracle_shim"; }

const CpuTuningProfile& get_autotuned_profile() {
    return lookup_tuning_profile(detect_arm_hwcaps());
}

ThresholdSelection get_current_thresholds() {
    ThresholdSelection t{};
    t.small_m_bound = 8;
    t.wide_n_bound = 48;
    t.unpacked_thresh = 4 * 1024 * 1024;
    t.valid = true;
    return t;
}

GemmKernelId select_gemm_kernel(int, int, int, GemmDataType) {
    return GemmKernelId::kPacked;
}

GemmBlockingParams get_autotuned_blocking_params(int, int, int, int, int, int, int, int) {
    std::fprintf(stderr, "oracle shim: packed driver is not part of the x86 oracle build\n");
    std::abort();
}

void gemm_driver_generic(int, int, int, float, const float*, int, const float*, int,
                         float, float*, int, const GemmDriverConfig&) {
    std::fprintf(stderr, "oracle shim: packed driver is not part of the x86 oracle build\n");
    std::abort();
}

}  // namespace dnnopt
