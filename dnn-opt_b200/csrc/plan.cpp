// Plan selector and autotune cache.
//
// Dispatch rules (B200 re-statement of src/gemm/gemm.cpp:168-455, where the
// reference routes by M < small_m_bound (8), N >= wide_n_bound and K):
//   * FP32, M <= 8, B stored K x N, N >= 512, K <= 2048
//                                    -> GemvPanel (64-column panels read as
//                                      whole row segments, K ranges summed by
//                                      the last CTA of each panel)
//   * M <= 8 and B stored K x N      -> GemvSlab (whole K per 8-column CTA) for
//                                      K <= 2048 and 512 <= N <= 8192, where a
//                                      split-K reduction costs more than the B
//                                      stream; else GemvKn (split-K streaming
//                                      GEMV, splits reduced by a ticketed last
//                                      CTA) or, when autotune measures it faster,
//                                      GemvKnCluster (splits reduced in a
//                                      thread-block cluster) or GemvSlab
//   * M <= 8 and B stored N x K      -> GemvRows (dot form, A in registers;
//                                      autotune also times GemvRowsBulk, B rows
//                                      by bulk copy into a shared ring) / GemvNk
//   * BF16, large M, N <= 256        -> Bf16Tc  (tcgen05 tall-skinny, B resident)
//   * BF16 M > 8 otherwise, int8 M > 8 (TMA-aligned operands)
//                                    -> GemmTc  (tcgen05, both operands by TMA)
//   * config-5 e4m3 with M > 8       -> GemvNkRows (dot form per 8-row block)
//   * anything else                  -> TileF32 / TileS8 (general SIMT tiles)
// The split-K factor is chosen so that the grid is one wave of resident CTAs
// (strips x splits ~= occupancy x SMs), never below 32 K-rows per split;
// autotune times {s, s/2, 2s, 1} in both variants and keeps the fastest.
#include "plan.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <list>
#include <map>
#include <mutex>
#include <unordered_map>
#include <utility>
#include <vector>

namespace dnnopt_b200 {

namespace {

int mt_for(int M) { return M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8)); }

In in_a(Kind k) {
    switch (k) {
        case Kind::BF16F32: return In::BF16;
        case Kind::F32BF16R: return In::F32R;
        case Kind::RE4E5: return In::RE4;
        case Kind::RE5E5: return In::RE5;
        default: return In::F32;
    }
}
In in_b(Kind k) {
    switch (k) {
        case Kind::BF16F32: return In::BF16;
        case Kind::F32BF16R: return In::F32R;
        case Kind::RE4E5:
        case Kind::RE5E5: return In::RE5;
        default: return In::F32;
    }
}

DotKind dot_kind(Kind k) {
    switch (k) {
        case Kind::S8S32: return DotKind::S8S32;
        case Kind::F32S8Q: return DotKind::S8DQ;
        case Kind::E4M3BF16: return DotKind::E4M3;
        case Kind::BF16F32: return DotKind::BF16;
        default: return DotKind::F32;
    }
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int kn_occupancy(Kind kind, int mt, int vec4, const DeviceInfo& info) {
    if (!info.have_device) return 3;
    static std::mutex mu;
    static std::map<int, int> memo;
    int key = static_cast<int>(kind) * 100 + mt * 10 + vec4;
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
    int occ = 0;
    if (gemv_kn_occupancy(in_a(kind), in_b(kind), mt, vec4, &occ) != cudaSuccess || occ < 1) {
        cudaGetLastError();
        occ = 1;
    }
    memo[key] = occ;
    return occ;
}

// Occupancy queries are memoised: the planner runs on every call, and the
// CUDA occupancy calculator costs microseconds.  Keys hold everything the
// answer depends on (kernel template arguments and the shared-memory size,
// which is set by K up to the kernels' pass length).
int memo_occupancy(int64_t key, const std::function<cudaError_t(int*)>& query) {
    static std::mutex mu;
    static std::map<int64_t, int> memo;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return 1; }
    key = key * 64 + dev;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = memo.find(key);
        if (it != memo.end()) return it->second;
    }
    int occ = 0;
    if (query(&occ) != cudaSuccess || occ < 1) {
        cudaGetLastError();
        occ = 1;
    }
    std::lock_guard<std::mutex> lk(mu);
    memo[key] = occ;
    return occ;
}

int slab_occupancy(Kind kind, int mt, int w, int K, const DeviceInfo& info) {
    if (!info.have_device) return 8;   // no device: plan names only, 8-column slabs
    const int kk = K < 1024 ? K : 1024;
    const int64_t key = ((static_cast<int64_t>(kind) * 16 + mt) * 32 + w) * 2048 + kk;
    return memo_occupancy(key * 4 + 1, [&](int* occ) {
        return gemv_slab_occupancy(in_a(kind), in_b(kind), mt, w, K, occ);
    });
}

int rows_occupancy(DotKind kind, int mt, int K, const DeviceInfo& info) {
    if (!info.have_device) return 4;
    const int64_t key = (static_cast<int64_t>(kind) * 16 + mt) * (int64_t{1} << 31) + K;
    return memo_occupancy(key * 4 + 2, [&](int* occ) { return gemv_rows_occupancy(kind, mt, K, occ); });
}

int nk_occupancy(DotKind kind, int mt, int vec, int K, const DeviceInfo& info) {
    if (!info.have_device) return 2;
    const int64_t key = ((static_cast<int64_t>(kind) * 16 + mt) * 2 + vec) * (int64_t{1} << 31) + K;
    return memo_occupancy(key * 4 + 3, [&](int* occ) { return gemv_nk_occupancy(kind, mt, vec, K, occ); });
}

// Row-panel GEMV (FP32, B K x N): 64-column panels and the K extent split
// into power-of-two ranges of about 256 rows (at most 8), so a 1024-row B
// gives 4 CTAs per panel.  Measured on B200 on the irregular-N sweep (12
// GEMMs, K = 1024, one stream each, graph replay): 38.1 us against 46.7 for
// the column slabs, 43.1 for 128-column panels in 4 ranges, 44.8 in 8.  Deep
// K (above 2048) stays with split-K.
bool panel_plan(const GemmArgs& g, int* w, int* splits) {
    if (g.K > 2048) return false;
    int s = 1;
    while (s < 8 && g.K / (2 * s) >= 256) s *= 2;
    if (!gemv_panel_supported(g, mt_for(g.M), 64, s)) return false;
    *w = 64;
    *splits = s;
    return true;
}

}  // namespace

int elem_bytes_a(Kind k) {
    switch (k) {
        case Kind::BF16F32:
        case Kind::E4M3BF16: return 2;
        case Kind::S8S32:
        case Kind::RE4E5:
        case Kind::RE5E5: return 1;
        case Kind::F32S8Q: return 1;   // after quantisation
        default: return 4;
    }
}

int elem_bytes_b(Kind k) {
    switch (k) {
        case Kind::BF16F32: return 2;
        case Kind::S8S32:
        case Kind::F32S8Q:
        case Kind::E4M3BF16:
        case Kind::RE4E5:
        case Kind::RE5E5: return 1;
        default: return 4;
    }
}

const char* kernel_name(KernelId k) {
    switch (k) {
        case KernelId::GemvKn: return "gemv_kn_splitk";
        case KernelId::GemvNk: return "gemv_nk_dot";
        case KernelId::TileF32: return "gemm_simt";
        case KernelId::TileS8: return "gemm_tile_s8";
        case KernelId::Bf16Tc: return "gemm_bf16_tcgen05";
        case KernelId::GemvNkRows: return "gemv_nk_dot_rowblocks";
        case KernelId::GemvKnCluster: return "gemv_kn_cluster";
        case KernelId::GemvRows: return "gemv_rows_dot";
        case KernelId::E4m3Tc: return "gemm_e4m3_tcgen05";
        case KernelId::GemvSlab: return "gemv_kn_slab";
        case KernelId::GemvPanel: return "gemv_panel";
        case KernelId::GemvRowsBulk: return "gemv_rows_bulk";
        case KernelId::GemmTc: return "gemm_tcgen05";
    }
    return "?";
}

GemvKnPlan kn_plan_rule(const GemmArgs& g, int mt, int vec4, int occ, int num_sms, int splits_hint,
                        bool allow_cluster) {
    GemvKnPlan p;
    p.mt = mt;
    p.vec4 = vec4;
    p.cluster = 0;
    const int tiles = gemv_kn_tiles(g.N);
    const int max_splits = g.K / 32 > 1 ? g.K / 32 : 1;
    const int cmax = gemv_kn_cluster_max_chunk();
    int splits = splits_hint;
    if (splits <= 0) {
        // One wave of resident CTAs, at most 16 splits of at least 64 rows:
        // measured on B200, more splits only add reduction latency.
        splits = (occ * num_sms) / tiles;
        if (splits > 16) splits = 16;
        if (splits > g.K / 64) splits = g.K / 64;
    }
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    if (allow_cluster) {
        // Cluster variant: at most 16 splits, each at most cmax rows.
        int cs = splits > 16 ? 16 : splits;
        if ((g.K + cs - 1) / cs <= cmax) {
            splits = cs;
            p.cluster = 1;
        }
    }
    int kchunk = (g.K + splits - 1) / splits;
    kchunk = (kchunk + 7) / 8 * 8;
    p.kchunk = kchunk;
    p.splits = (g.K + kchunk - 1) / kchunk;
    return p;
}

GemvKnPlan kn_plan_for(Kind kind, const GemmArgs& g, const DeviceInfo& info, int splits_hint,
                       bool allow_cluster) {
    const int mt = mt_for(g.M);
    const size_t eb = static_cast<size_t>(elem_bytes_b(kind));
    const int vec4 = (aligned(g.B, 4 * eb) && g.ldb % 4 == 0) ? 1 : 0;
    const int occ = splits_hint <= 0 ? kn_occupancy(kind, mt, vec4, info) : 1;
    return kn_plan_rule(g, mt, vec4, occ, info.num_sms, splits_hint, allow_cluster);
}

GemvNkPlan nk_plan_for(Kind kind, const GemmArgs& g, const DeviceInfo& info, int grid_hint) {
    GemvNkPlan p;
    p.mt = mt_for(g.M < 8 ? g.M : 8);
    const size_t eb = static_cast<size_t>(elem_bytes_b(kind));
    p.vec = (aligned(g.B, 16) && (static_cast<size_t>(g.ldb) * eb) % 16 == 0) ? 1 : 0;
    int grid = grid_hint;
    if (grid <= 0) grid = nk_occupancy(dot_kind(kind), p.mt, p.vec, g.K, info) * info.num_sms;
    if (grid > g.N) grid = g.N;
    if (grid < 1) grid = 1;
    p.grid = grid;
    return p;
}

Plan heuristic_plan(Kind kind, const GemmArgs& g, const DeviceInfo& info) {
    Plan p;
    const bool dot_fits = gemv_nk_smem_bytes(dot_kind(kind), mt_for(g.M < 8 ? g.M : 8), g.K) <=
                          kGemvNkMaxSmem;
    switch (kind) {
        case Kind::S8S32:
        case Kind::F32S8Q:
            // Dot form with A in registers: the register-load kernel (config
            // 3: 10.3 us against 10.5 for the bulk-copy ring, which autotune
            // also times).
            if (g.M <= 8 && gemv_rows_supported(dot_kind(kind), g)) {
                p.kernel = KernelId::GemvRows;
                p.nk.mt = mt_for(g.M);
                p.nk.vec = 1;
                p.nk.grid = rows_occupancy(dot_kind(kind), p.nk.mt, g.K, info) * info.num_sms;
            } else if (g.M <= 8 && dot_fits) {
                p.kernel = KernelId::GemvNk;
                p.nk = nk_plan_for(kind, g, info, 0);
            } else if (gemm_tc_supported(TcKind::I8, g)) {
                p.kernel = KernelId::GemmTc;
                p.tc = gemm_tc_plan(TcKind::I8, g, info.num_sms);
            } else {
                p.kernel = KernelId::TileS8;
            }
            return p;
        case Kind::E4M3BF16:
            if (info.have_device) {
                GemmArgs g8 = g;
                g8.M = g.M < 8 ? g.M : 8;
                if (gemm_e4m3_tc_supported(g8)) {
                    p.e4 = gemm_e4m3_tc_plan(g8, info.num_sms);
                    if (p.e4.stages >= 2) {
                        p.kernel = KernelId::E4m3Tc;
                        return p;
                    }
                }
            }
            p.kernel = (g.M <= 8) ? KernelId::GemvNk : KernelId::GemvNkRows;
            p.nk = nk_plan_for(kind, g, info, 0);
            if (!dot_fits) p.kernel = KernelId::TileF32;   // rejected by the caller (no tile path)
            return p;
        default:
            break;
    }
    if (g.M <= 8 && !g.b_trans) {
        p.kn = kn_plan_for(kind, g, info, 0, false);
        p.kernel = p.kn.cluster ? KernelId::GemvKnCluster : KernelId::GemvKn;
        // Measured on B200 (M <= 8, K = 1024, prime N of 1009-4093): the slab
        // form finishes in 0.4-0.8x the split-K time; at K = 4096 split-K wins.
        // 16-column slabs when 8-column ones would need more than one wave of
        // resident CTAs (7 x 4093: 10.7 -> 8.5 us), or for M <= 4 from 1536
        // columns on (3 x 2039: 4.9 -> 3.8 us, 2 x 4093: 6.7 -> 6.1 us);
        // 8 otherwise (narrower N keeps more CTAs: 2 x 1009 at 8 columns
        // takes 2.8 us, at 16 3.7 us).
        if (kind == Kind::F32 && g.N >= 512 && panel_plan(g, &p.panel_w, &p.panel_splits)) {
            p.kernel = KernelId::GemvPanel;
        } else if (g.K <= 2048 && g.N >= 512 && g.N <= 8192) {
            p.kernel = KernelId::GemvSlab;
            const int occ8 = slab_occupancy(kind, p.kn.mt, 8, g.K, info);
            const bool wide = gemv_slab_ctas(g.N, 8) > occ8 * info.num_sms || (p.kn.mt <= 4 && g.N >= 1536);
            p.slab_w = wide ? 16 : 8;
        }
        return p;
    }
    if (kind == Kind::F32 && g.M <= 8 && g.b_trans && gemv_rows_supported(DotKind::F32, g)) {
        p.kernel = KernelId::GemvRows;
        p.nk.mt = mt_for(g.M);
        p.nk.vec = 1;
        p.nk.grid = rows_occupancy(DotKind::F32, p.nk.mt, g.K, info) * info.num_sms;
        return p;
    }
    if (kind == Kind::BF16F32 && g.M <= 8 && g.b_trans && gemv_rows_supported(DotKind::BF16, g)) {
        p.kernel = KernelId::GemvRows;
        p.nk.mt = mt_for(g.M);
        p.nk.vec = 1;
        p.nk.grid = rows_occupancy(DotKind::BF16, p.nk.mt, g.K, info) * info.num_sms;
        return p;
    }
    if (kind == Kind::F32 && g.M <= 8 && g.b_trans && dot_fits) {
        p.kernel = KernelId::GemvNk;
        p.nk = nk_plan_for(kind, g, info, 0);
        return p;
    }
    // BF16 with large M: the tall-skinny kernel while B stays resident in
    // shared memory (N <= 256, K whole); otherwise the streaming tcgen05 GEMM
    // (the tall-skinny kernel would run K in chunks, re-reading C each time).
    if (kind == Kind::BF16F32 && g.M > 8 && info.have_device && gemm_bf16_tc_kchunk(g) == g.K) {
        p.kernel = KernelId::Bf16Tc;
        return p;
    }
    if (kind == Kind::BF16F32 && g.M > 8 && gemm_tc_supported(TcKind::BF16, g)) {
        p.kernel = KernelId::GemmTc;
        p.tc = gemm_tc_plan(TcKind::BF16, g, info.num_sms);
        return p;
    }
    if (kind == Kind::BF16F32 && g.M > 8 && info.have_device && gemm_bf16_tc_kchunk(g) > 0) {
        p.kernel = KernelId::Bf16Tc;   // K in chunks (unaligned operands for the streaming kernel)
        return p;
    }
    p.kernel = KernelId::TileF32;
    p.simt = gemm_simt_plan(g, info.num_sms);
    return p;
}

std::string describe_plan(Kind, const GemmArgs& g, const Plan& p) {
    char buf[160];
    switch (p.kernel) {
        case KernelId::GemvKn:
        case KernelId::GemvKnCluster:
            std::snprintf(buf, sizeof(buf), "%s mt=%d vec4=%d splits=%d kchunk=%d%s",
                          kernel_name(p.kernel), p.kn.mt, p.kn.vec4, p.kn.splits, p.kn.kchunk,
                          p.tuned ? " tuned" : "");
            break;
        case KernelId::GemvNk:
        case KernelId::GemvNkRows:
        case KernelId::GemvRows:
        case KernelId::GemvRowsBulk:
            std::snprintf(buf, sizeof(buf), "%s mt=%d vec=%d grid=%d%s", kernel_name(p.kernel),
                          p.nk.mt, p.nk.vec, p.nk.grid, p.tuned ? " tuned" : "");
            break;
        case KernelId::E4m3Tc:
            std::snprintf(buf, sizeof(buf), "%s splits=%d kc=%d stages=%d", kernel_name(p.kernel),
                          p.e4.splits, p.e4.kc, p.e4.stages);
            break;
        case KernelId::GemvSlab:
            std::snprintf(buf, sizeof(buf), "%s mt=%d w=%d ctas=%d%s", kernel_name(p.kernel), p.kn.mt,
                          p.slab_w, gemv_slab_ctas(g.N, p.slab_w), p.tuned ? " tuned" : "");
            break;
        case KernelId::GemvPanel:
            std::snprintf(buf, sizeof(buf), "%s mt=%d w=%d splits=%d ctas=%d%s", kernel_name(p.kernel), p.kn.mt,
                          p.panel_w, p.panel_splits, gemv_panel_ctas(g.N, p.panel_w, p.panel_splits),
                          p.tuned ? " tuned" : "");
            break;
        case KernelId::GemmTc:
            std::snprintf(buf, sizeof(buf), "%s n=%d splits=%d kblocks=%d", kernel_name(p.kernel), p.tc.n_mma,
                          p.tc.splits, p.tc.kb_per_split);
            break;
        case KernelId::TileF32:
            std::snprintf(buf, sizeof(buf), "%s bm=%d bn=%d splits=%d kchunk=%d", kernel_name(p.kernel),
                          p.simt.bm, p.simt.bn, p.simt.splits, p.simt.kchunk);
            break;
        default:
            std::snprintf(buf, sizeof(buf), "%s", kernel_name(p.kernel));
    }
    return buf;
}

// ---------------------------------------------------------------------------
// Autotune cache
// ---------------------------------------------------------------------------
namespace {

struct Entry {
    int32_t kernel, p0, p1, mt;
    float time_us;
};

// LRU of kCacheCapacity plans (the reference's ShapeCache keeps 256 entries,
// include/dnnopt/autotune/shape_cache.h:139-146): `g_lru` lists keys from the
// most to the least recently used; a lookup hit or a store moves the key to
// the front, a store into a full cache evicts the back.
constexpr size_t kCacheCapacity = 256;
struct Slot {
    Entry e;
    std::list<uint64_t>::iterator pos;
};
std::mutex g_cache_mu;
std::unordered_map<uint64_t, Slot> g_cache;
std::list<uint64_t> g_lru;
int g_autotune = -1;   // -1: read DNNOPT_AUTOTUNE on first query

// Inserts or refreshes `key` (caller holds g_cache_mu).
void cache_put_locked(uint64_t key, const Entry& e) {
    auto it = g_cache.find(key);
    if (it != g_cache.end()) {
        it->second.e = e;
        g_lru.splice(g_lru.begin(), g_lru, it->second.pos);
        return;
    }
    while (g_cache.size() >= kCacheCapacity && !g_lru.empty()) {
        g_cache.erase(g_lru.back());
        g_lru.pop_back();
    }
    g_lru.push_front(key);
    g_cache[key] = Slot{e, g_lru.begin()};
}

// FNV-1a, 64-bit (offset basis 14695981039346656037, prime 1099511628211),
// the hash of the reference's shape keys (src/autotune/shape_cache.cpp:15-24).
uint64_t fnv1a(const void* data, size_t n) {
    const unsigned char* p = static_cast<const unsigned char*>(data);
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) { h ^= p[i]; h *= 1099511628211ull; }
    return h;
}

constexpr char kMagic[8] = {'D', 'N', 'N', 'A', 'U', 'T', 'O', '\0'};
// Reference files are v1-v3 (CPU blocking choices); v4 files of this library
// were keyed with a mistyped offset basis, so v5 marks the FNV-1a keys.
constexpr uint32_t kVersion = 5;

}  // namespace

bool autotune_enabled() {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    if (g_autotune < 0) {
        const char* e = std::getenv("DNNOPT_AUTOTUNE");
        g_autotune = (e && (e[0] == '1' || e[0] == 'y' || e[0] == 'Y')) ? 1 : 0;
    }
    return g_autotune == 1;
}

void set_autotune_enabled(bool on) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    g_autotune = on ? 1 : 0;
}

uint64_t plan_key(Kind kind, const GemmArgs& g, int vec) {
    int64_t k[10] = {static_cast<int64_t>(kind), g.M, g.N, g.K, g.lda, g.ldb, g.ldc,
                     g.a_trans, g.b_trans, vec};
    return fnv1a(k, sizeof(k));
}

bool cache_lookup(uint64_t key, Plan* out) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = g_cache.find(key);
    if (it == g_cache.end()) return false;
    g_lru.splice(g_lru.begin(), g_lru, it->second.pos);
    const Entry& e = it->second.e;
    out->kernel = static_cast<KernelId>(e.kernel);
    out->tuned = true;
    if (out->kernel == KernelId::GemvSlab) {
        out->slab_w = e.p0 == 16 ? 16 : 8;
        out->kn.mt = e.mt;
    } else if (out->kernel == KernelId::GemvPanel) {
        out->panel_w = e.p0 == 64 ? 64 : 128;
        out->panel_splits = e.p1;
        out->kn.mt = e.mt;
    } else if (out->kernel == KernelId::GemvKn || out->kernel == KernelId::GemvKnCluster) {
        out->kn.splits = e.p0;
        out->kn.kchunk = e.p1;
        out->kn.mt = e.mt;
        out->kn.cluster = out->kernel == KernelId::GemvKnCluster ? 1 : 0;
    } else if (out->kernel == KernelId::E4m3Tc) {
        out->e4.splits = e.p0;
        out->e4.kc = e.p1;
        out->e4.stages = e.mt;
    } else {
        out->nk.grid = e.p0;
        out->nk.mt = e.mt;
    }
    return true;
}

void cache_store(uint64_t key, const Plan& p, float time_us) {
    Entry e;
    e.kernel = static_cast<int32_t>(p.kernel);
    if (p.kernel == KernelId::GemvSlab) {
        e.p0 = p.slab_w; e.p1 = 0; e.mt = p.kn.mt;
    } else if (p.kernel == KernelId::GemvPanel) {
        e.p0 = p.panel_w; e.p1 = p.panel_splits; e.mt = p.kn.mt;
    } else if (p.kernel == KernelId::GemvKn || p.kernel == KernelId::GemvKnCluster) {
        e.p0 = p.kn.splits; e.p1 = p.kn.kchunk; e.mt = p.kn.mt;
    } else if (p.kernel == KernelId::E4m3Tc) {
        e.p0 = p.e4.splits; e.p1 = p.e4.kc; e.mt = p.e4.stages;
    }
    else { e.p0 = p.nk.grid; e.p1 = 0; e.mt = p.nk.mt; }
    e.time_us = time_us;
    std::lock_guard<std::mutex> lk(g_cache_mu);
    cache_put_locked(key, e);
}

int cache_save(const char* path) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    FILE* f = std::fopen(path, "wb");
    if (!f) return -1;
    uint32_t n = static_cast<uint32_t>(g_cache.size());
    bool ok = std::fwrite(kMagic, 1, 8, f) == 8 && std::fwrite(&kVersion, 4, 1, f) == 1 &&
              std::fwrite(&n, 4, 1, f) == 1;
    // Least recently used first: loading the file re-inserts in this order,
    // so the recency order survives a save / load round trip.
    for (auto it = g_lru.rbegin(); it != g_lru.rend(); ++it) {
        const Entry& e = g_cache[*it].e;
        ok = ok && std::fwrite(&*it, 8, 1, f) == 1 && std::fwrite(&e, sizeof(Entry), 1, f) == 1;
    }
    ok = (std::fclose(f) == 0) && ok;
    return ok ? static_cast<int>(n) : -1;
}

int cache_load(const char* path) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return -1;
    char magic[8];
    uint32_t ver = 0, n = 0;
    if (std::fread(magic, 1, 8, f) != 8 || std::memcmp(magic, kMagic, 8) != 0 ||
        std::fread(&ver, 4, 1, f) != 1 || ver != kVersion || std::fread(&n, 4, 1, f) != 1 ||
        n > 1000000u) {
        std::fclose(f);
        return -1;
    }
    std::vector<std::pair<uint64_t, Entry>> loaded;
    loaded.reserve(n);
    for (uint32_t i = 0; i < n; ++i) {
        uint64_t key;
        Entry e;
        if (std::fread(&key, 8, 1, f) != 1 || std::fread(&e, sizeof(Entry), 1, f) != 1) {
            std::fclose(f);
            return -1;
        }
        loaded.emplace_back(key, e);
    }
    std::fclose(f);
    // File order is least recently used first; past the capacity the oldest
    // entries are evicted as they would have been.
    std::lock_guard<std::mutex> lk(g_cache_mu);
    for (const auto& kv : loaded) cache_put_locked(kv.first, kv.second);
    return static_cast<int>(loaded.size());
}

int cache_entries() {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    return static_cast<int>(g_cache.size());
}

}  // namespace dnnopt_b200
