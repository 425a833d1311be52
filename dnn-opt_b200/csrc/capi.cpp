// C ABI of libdnnopt_b200.so: argument validation, plan selection (with
// optional autotune), workspace management, host-pointer staging and kernel
// dispatch.  See include/dnnopt_b200.h for the contract of each entry point.
#include <cstdio>
#include <cstring>
#include <string>

#include "kernels.h"
#include "plan.h"
#include "runtime.h"

using namespace dnnopt_b200;

namespace {

GemmArgs to_args(const dnnopt_gemm_desc* d, const void* A, const void* B, void* C) {
    GemmArgs g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.alpha = d->alpha; g.beta = d->beta;
    g.A = A; g.lda = d->lda; g.a_trans = d->trans_a ? 1 : 0;
    g.B = B; g.ldb = d->ldb; g.b_trans = d->trans_b ? 1 : 0;
    g.C = C; g.ldc = d->ldc;
    return g;
}

// B is always N x K for these kinds.
bool b_is_nk(Kind k) { return k == Kind::S8S32 || k == Kind::E4M3BF16; }

// Validates sizes, leading dimensions and pointers.  Returns SUCCESS with
// *noop = true for the reference's silent early return (any of M, N, K == 0).
int validate(Kind kind, const dnnopt_gemm_desc* d, const void* A, const void* B, const void* C,
             bool* noop) {
    *noop = false;
    if (!d) return DNNOPT_STATUS_INVALID_VALUE;
    if (d->M < 0 || d->N < 0 || d->K < 0) return DNNOPT_STATUS_INVALID_VALUE;
    if (d->M == 0 || d->N == 0 || d->K == 0) { *noop = true; return DNNOPT_STATUS_SUCCESS; }
    const bool ta = d->trans_a != 0;
    const bool tb = b_is_nk(kind) ? true : d->trans_b != 0;
    if (d->lda < (ta ? d->M : d->K)) return DNNOPT_STATUS_INVALID_VALUE;
    if (d->ldb < (tb ? d->K : d->N)) return DNNOPT_STATUS_INVALID_VALUE;
    if (d->ldc < d->N) return DNNOPT_STATUS_INVALID_VALUE;
    if (!A || !B || !C) return DNNOPT_STATUS_INVALID_VALUE;
    return DNNOPT_STATUS_SUCCESS;
}

DeviceInfo info_of(const DeviceContext* ctx) {
    DeviceInfo i;
    if (ctx) { i.num_sms = ctx->num_sms; i.have_device = true; }
    return i;
}

// Kernels for a K x N B with M <= 8 (one plan family: interchangeable under autotune).
// Dot-form kernels with A in registers (interchangeable under autotune).
bool is_rows(KernelId k) { return k == KernelId::GemvRows || k == KernelId::GemvRowsBulk; }

bool is_kn(KernelId k) {
    return k == KernelId::GemvKn || k == KernelId::GemvKnCluster || k == KernelId::GemvSlab ||
           k == KernelId::GemvPanel;
}

int vec_of(const Plan& p) {
    if (p.kernel == KernelId::E4m3Tc) return 1;
    return is_kn(p.kernel) ? p.kn.vec4 : p.nk.vec;
}

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

// Launches one plan.  `scales`: per-row scales (e4m3) or {sA, sB} (int8 dequant).
int launch_plan(Kind kind, const GemmArgs& g, const Plan& p, const float* scales,
                DeviceContext* ctx, cudaStream_t s) {
    int inj = check_injected_fault(2);
    if (inj != DNNOPT_STATUS_SUCCESS) return set_status(inj);
    cudaError_t e = cudaSuccess;
    Workspace* w = nullptr;
    int st;
    switch (p.kernel) {
        case KernelId::GemvKn: {
            const size_t wsf = gemv_kn_ws_floats(p.kn, g.N);
            st = ensure_workspace(ctx, s, wsf, static_cast<size_t>(gemv_kn_tiles(g.N)), 0, &w);
            if (st != DNNOPT_STATUS_SUCCESS) return st;
            e = launch_gemv_kn(in_a(kind), in_b(kind), g, p.kn, w->ws, w->counters, s);
            note_launch();
            break;
        }
        case KernelId::GemvKnCluster:
            e = launch_gemv_kn_cluster(in_a(kind), in_b(kind), g, p.kn, s);
            note_launch();
            break;
        case KernelId::GemvSlab:
            if (g.bias) {
                // The slab kernel has no bias epilogue; biased calls (the oneDNN
                // entry) take the split-K kernel of the same plan family.
                const GemvKnPlan kp = kn_plan_for(kind, g, info_of(ctx), 0, false);
                st = ensure_workspace(ctx, s, gemv_kn_ws_floats(kp, g.N),
                                      static_cast<size_t>(gemv_kn_tiles(g.N)), 0, &w);
                if (st != DNNOPT_STATUS_SUCCESS) return st;
                e = launch_gemv_kn(in_a(kind), in_b(kind), g, kp, w->ws, w->counters, s);
                note_launch();
                break;
            }
            e = launch_gemv_slab(in_a(kind), in_b(kind), g, p.kn.mt, p.slab_w, s);
            note_launch();
            break;
        case KernelId::GemvPanel: {
            GemvKnPlan kp = p.kn;
            if (kind != Kind::F32 || !gemv_panel_supported(g, kp.mt, p.panel_w, p.panel_splits))
                return set_status(DNNOPT_STATUS_NOT_SUPPORTED);
            st = ensure_workspace(ctx, s, gemv_panel_ws_floats(g.N, kp.mt, p.panel_w, p.panel_splits),
                                  static_cast<size_t>(gemv_panel_tickets(g.N, p.panel_w)), 0, &w);
            if (st != DNNOPT_STATUS_SUCCESS) return st;
            e = launch_gemv_panel(g, kp.mt, p.panel_w, p.panel_splits, w->ws, w->counters, s);
            note_launch();
            break;
        }
        case KernelId::GemvNk:
            e = launch_gemv_nk(dot_kind(kind), g, p.nk, scales, s);
            note_launch();
            break;
        case KernelId::GemvRows:
            e = launch_gemv_rows(dot_kind(kind), g, p.nk.mt, p.nk.grid, scales, s);
            note_launch();
            break;
        case KernelId::GemvRowsBulk:
            st = ensure_workspace(ctx, s, 0, 0, 0, &w);
            if (st != DNNOPT_STATUS_SUCCESS) return st;
            e = launch_gemv_rows_bulk(dot_kind(kind), g, p.nk.mt, p.nk.grid, scales, w->err, s);
            note_launch();
            break;
        case KernelId::GemvNkRows: {
            const size_t ea = static_cast<size_t>(elem_bytes_a(kind));
            for (int m0 = 0; m0 < g.M && e == cudaSuccess; m0 += 8) {
                GemmArgs r = g;
                r.M = g.M - m0 < 8 ? g.M - m0 : 8;
                r.A = static_cast<const char*>(g.A) +
                      (g.a_trans ? static_cast<size_t>(m0) : static_cast<size_t>(m0) * g.lda) * ea;
                const size_t ec = (kind == Kind::E4M3BF16) ? 2 : 4;
                r.C = static_cast<char*>(g.C) + static_cast<size_t>(m0) * g.ldc * ec;
                GemvNkPlan rp = p.nk;
                rp.mt = r.M <= 1 ? 1 : (r.M <= 2 ? 2 : (r.M <= 4 ? 4 : 8));
                e = launch_gemv_nk(dot_kind(kind), r, rp, scales, s);
                note_launch();
            }
            break;
        }
        case KernelId::E4m3Tc: {
            for (int m0 = 0; m0 < g.M && e == cudaSuccess; m0 += 8) {
                GemmArgs r = g;
                r.M = g.M - m0 < 8 ? g.M - m0 : 8;
                r.A = static_cast<const uint16_t*>(g.A) + static_cast<size_t>(m0) * g.lda;
                r.C = static_cast<uint16_t*>(g.C) + static_cast<size_t>(m0) * g.ldc;
                const size_t wsf = gemm_e4m3_tc_ws_floats(r, p.e4);
                st = ensure_workspace(ctx, s, wsf, static_cast<size_t>((g.N + 127) / 128),
                                      gemm_e4m3_tc_act_bytes(r), &w);
                if (st != DNNOPT_STATUS_SUCCESS) return st;
                e = launch_gemm_e4m3_tc(r, p.e4, scales, w->ws, w->counters, w->quant, w->err, s);
                note_launch(2);
            }
            break;
        }
        case KernelId::GemmTc: {
            const TcKind tk = kind == Kind::BF16F32 ? TcKind::BF16 : TcKind::I8;
            if (kind != Kind::BF16F32 && kind != Kind::S8S32 && kind != Kind::F32S8Q)
                return set_status(DNNOPT_STATUS_NOT_SUPPORTED);
            const size_t wsb = gemm_tc_ws_bytes(g, p.tc);
            st = ensure_workspace(ctx, s, (wsb + 3) / 4, static_cast<size_t>(gemm_tc_tickets(g, p.tc)), 0, &w);
            if (st != DNNOPT_STATUS_SUCCESS) return st;
            e = launch_gemm_tc(tk, dot_kind(kind), g, p.tc, scales, w->ws, w->counters, w->err, ctx->num_sms, s);
            note_launch();
            break;
        }
        case KernelId::TileF32:
            if (kind == Kind::E4M3BF16 || kind == Kind::S8S32 || kind == Kind::F32S8Q)
                return set_status(DNNOPT_STATUS_NOT_SUPPORTED);
            e = launch_gemm_simt(in_a(kind), in_b(kind), g, p.simt, s);
            note_launch();
            break;
        case KernelId::TileS8:
            e = launch_gemm_tile_s8(dot_kind(kind), g, scales, s);
            note_launch();
            break;
        case KernelId::Bf16Tc: {
            st = ensure_workspace(ctx, s, 0, 0, 0, &w);
            if (st != DNNOPT_STATUS_SUCCESS) return st;
            // Deep K: chunks of kc rows, C accumulating (beta = 1 after the first).
            const int kc = gemm_bf16_tc_kchunk(g);
            if (kc < 1) return set_status(DNNOPT_STATUS_NOT_SUPPORTED);
            for (int k0 = 0; k0 < g.K && e == cudaSuccess; k0 += kc) {
                GemmArgs c = g;
                c.K = g.K - k0 < kc ? g.K - k0 : kc;
                c.A = static_cast<const uint16_t*>(g.A) + k0;
                c.B = static_cast<const uint16_t*>(g.B) + (g.b_trans ? static_cast<int64_t>(k0)
                                                                     : static_cast<int64_t>(k0) * g.ldb);
                if (k0 > 0) c.beta = 1.0f;
                e = launch_gemm_bf16_tc(c, ctx->num_sms, w->err, s);
                note_launch();
            }
            break;
        }
    }
    return cuda_status(e);
}

// Times one plan (beta forced to 0, output into `scratch`), microseconds.
float time_plan(Kind kind, GemmArgs g, const Plan& p, const float* scales, DeviceContext* ctx,
                cudaStream_t s, void* scratch) {
    g.beta = 0.0f;
    g.C = scratch;
    g.ldc = g.N;
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess) return 1e30f;
    if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return 1e30f; }
    float best = 1e30f;
    if (launch_plan(kind, g, p, scales, ctx, s) == DNNOPT_STATUS_SUCCESS) {
        for (int r = 0; r < 3; ++r) {
            cudaEventRecord(a, s);
            for (int i = 0; i < 4; ++i) launch_plan(kind, g, p, scales, ctx, s);
            cudaEventRecord(b, s);
            if (cudaEventSynchronize(b) != cudaSuccess) break;
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, a, b);
            if (ms * 250.0f < best) best = ms * 250.0f;
        }
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaGetLastError();
    return best;
}

Plan get_plan(Kind kind, const GemmArgs& g, DeviceContext* ctx, cudaStream_t s,
              const float* scales) {
    const DeviceInfo info = info_of(ctx);
    Plan h = heuristic_plan(kind, g, info);
    const bool tunable = is_kn(h.kernel) || h.kernel == KernelId::GemvNk || is_rows(h.kernel) ||
                         h.kernel == KernelId::E4m3Tc;
    if (!tunable) return h;
    const uint64_t key = plan_key(kind, g, vec_of(h));
    Plan c = h;
    if (cache_lookup(key, &c) && (c.kernel == h.kernel || (is_kn(c.kernel) && is_kn(h.kernel)) ||
                                  (is_rows(c.kernel) && is_rows(h.kernel)))) {
        // Layout-derived fields come from the current call.
        if (is_kn(c.kernel)) c.kn.vec4 = h.kn.vec4;
        else if (c.kernel != KernelId::E4m3Tc) c.nk.vec = h.nk.vec;
        // A loaded plan that does not fit this call (a hand-written or stale
        // file) gives way to the heuristic one.
        if (c.kernel == KernelId::GemvPanel &&
            (kind != Kind::F32 || !gemv_panel_supported(g, c.kn.mt, c.panel_w, c.panel_splits)))
            return h;
        return c;
    }
    if (!autotune_enabled() || !ctx) return h;

    // Candidates around the heuristic choice.
    constexpr int kMaxCands = 24;
    Plan cands[kMaxCands];
    int nc = 0;
    if (is_kn(h.kernel)) {
        if (kind == Kind::F32) {
            for (int pw : {64, 128})
                for (int ps : {1, 2, 4, 8}) {
                    if (!gemv_panel_supported(g, h.kn.mt, pw, ps) || nc >= kMaxCands - 8) continue;
                    Plan q = h;
                    q.kernel = KernelId::GemvPanel;
                    q.kn = kn_plan_for(kind, g, info, 0, false);
                    q.panel_w = pw;
                    q.panel_splits = ps;
                    cands[nc++] = q;
                }
        }
        for (int w : {8, 16}) {
            Plan slab = h;
            slab.kernel = KernelId::GemvSlab;
            slab.kn = kn_plan_for(kind, g, info, 0, false);
            slab.slab_w = w;
            cands[nc++] = slab;
        }
        const GemvKnPlan ws_plan = kn_plan_for(kind, g, info, 0, false);
        const int tries[6] = {h.kn.splits, h.kn.splits / 2, h.kn.splits * 2, 1,
                              ws_plan.splits, ws_plan.splits * 2};
        for (int t : tries) {
            if (t < 1) continue;
            for (int cl = 0; cl < 2; ++cl) {
                Plan q = h;
                q.kn = kn_plan_for(kind, g, info, t, cl == 1);
                if ((cl == 1) != (q.kn.cluster == 1)) continue;
                q.kernel = q.kn.cluster ? KernelId::GemvKnCluster : KernelId::GemvKn;
                bool dup = false;
                for (int i = 0; i < nc; ++i)
                    dup = dup || (cands[i].kn.splits == q.kn.splits && cands[i].kernel == q.kernel);
                if (!dup && nc < kMaxCands) cands[nc++] = q;
            }
        }
    } else if (h.kernel == KernelId::E4m3Tc) {
        GemmArgs g8 = g;
        g8.M = g.M < 8 ? g.M : 8;
        const int s0 = h.e4.splits;
        const int tries[6] = {s0, s0 / 2, s0 * 2, 1, 2, 4};
        const int depths[2] = {2, 3};
        for (int t : tries)
            for (int d : depths) {
                if (t < 1 || t > 32) continue;
                Plan q = h;
                q.e4 = gemm_e4m3_tc_plan_splits(g8, t, d);
                if (q.e4.stages < 2) continue;
                bool dup = false;
                for (int i = 0; i < nc; ++i)
                    dup = dup || (cands[i].e4.splits == q.e4.splits && cands[i].e4.stages == q.e4.stages);
                if (!dup && nc < kMaxCands) cands[nc++] = q;
            }
    } else if (is_rows(h.kernel)) {
        // Register-load rows kernel at its occupancy grid and half of it, and
        // the bulk-copy ring at its own occupancy grid.
        const int g0 = h.nk.grid;
        for (int t : {g0, g0 / 2}) {
            if (t < 1) continue;
            Plan q = h;
            q.nk.grid = t;
            cands[nc++] = q;
        }
        if (gemv_rows_bulk_supported(dot_kind(kind), g)) {
            Plan q = h;
            q.kernel = KernelId::GemvRowsBulk;
            int occ = 1;
            if (gemv_rows_bulk_occupancy(dot_kind(kind), h.nk.mt, g.K, &occ) != cudaSuccess || occ < 1) {
                cudaGetLastError();
                occ = 1;
            }
            q.nk.grid = occ * info.num_sms;
            cands[nc++] = q;
        }
    } else {
        const int g0 = h.nk.grid;
        const int tries[3] = {g0, g0 / 2, g0 * 2};
        for (int t : tries) {
            if (t < 1) continue;
            Plan q = h;
            q.nk = nk_plan_for(kind, g, info, t);
            bool dup = false;
            for (int i = 0; i < nc; ++i) dup = dup || cands[i].nk.grid == q.nk.grid;
            if (!dup) cands[nc++] = q;
        }
    }
    const size_t out_bytes = static_cast<size_t>(g.M) * g.N * 4;
    Workspace* w = nullptr;
    if (ensure_workspace(ctx, s, 0, 0, out_bytes, &w) != DNNOPT_STATUS_SUCCESS) return h;
    float best_t = 1e30f;
    Plan best = h;
    for (int i = 0; i < nc; ++i) {
        float t = time_plan(kind, g, cands[i], scales, ctx, s, w->quant);
        if (t < best_t) { best_t = t; best = cands[i]; }
    }
    best.tuned = true;
    cache_store(key, best, best_t);
    return best;
}

// Device-pointer dispatch for one call (validation already done, not a no-op).
int run_device(Kind kind, const GemmArgs& g0, const float* scales, DeviceContext* ctx,
               cudaStream_t s) {
    GemmArgs g = g0;
    if (b_is_nk(kind)) g.b_trans = 1;
    if (kind == Kind::F32S8Q) {
        // Quantise (absmax -> scales -> int8 copies), then the int8 GEMM with a
        // dequantising epilogue.
        const size_t qa = static_cast<size_t>(g.M) * g.K;
        const size_t qb = static_cast<size_t>(g.N) * g.K;
        Workspace* w = nullptr;
        int st = ensure_workspace(ctx, s, 0, 0, qa + qb + 16, &w);
        if (st != DNNOPT_STATUS_SUCCESS) return st;
        int inj = check_injected_fault(2);
        if (inj != DNNOPT_STATUS_SUCCESS) return set_status(inj);
        int8_t* q = static_cast<int8_t*>(w->quant);
        cudaError_t e = launch_absmax2(g, w->absmax, s);
        note_launch();
        if (e == cudaSuccess) { e = launch_quantize_s8(g, w->absmax, w->scales, q, q + qa, s); note_launch(); }
        if (e != cudaSuccess) return cuda_status(e);
        GemmArgs gq = g;
        gq.A = q; gq.lda = g.K; gq.a_trans = 0;
        gq.B = q + qa; gq.ldb = g.K; gq.b_trans = 1;
        Plan p = get_plan(kind, gq, ctx, s, w->scales);
        return launch_plan(kind, gq, p, w->scales, ctx, s);
    }
    Plan p = get_plan(kind, g, ctx, s, scales);
    return launch_plan(kind, g, p, scales, ctx, s);
}

int device_entry(Kind kind, const dnnopt_gemm_desc* d, const void* A, const void* B, void* C,
                 const float* scales, void* stream) {
    bool noop;
    int st = validate(kind, d, A, B, C, &noop);
    if (st != DNNOPT_STATUS_SUCCESS || noop) return set_status(st);
    if (kind == Kind::E4M3BF16 && !scales) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    return run_device(kind, to_args(d, A, B, C), scales, ctx, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Host-signature entry points: host or device pointers, synchronous.
// ---------------------------------------------------------------------------
struct Operand {
    const void* user;
    size_t bytes;     // span of the stored matrix in bytes
    bool in, out;     // copied to / from the device
};

size_t span_bytes(int rows, int cols, int ld, size_t eb) {
    if (rows <= 0 || cols <= 0) return 0;
    return (static_cast<size_t>(rows - 1) * ld + cols) * eb;
}

int host_entry(Kind kind, const dnnopt_gemm_desc* d, const void* A, const void* B, void* C,
               const float* scales) {
    bool noop;
    int st = validate(kind, d, A, B, C, &noop);
    if (st != DNNOPT_STATUS_SUCCESS || noop) return set_status(st);
    if (kind == Kind::E4M3BF16 && !scales) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaStream_t s = ctx->user_stream_set ? ctx->user_stream : ctx->default_stream;

    const bool ta = d->trans_a != 0, tb = b_is_nk(kind) || d->trans_b != 0;
    const size_t ea = (kind == Kind::F32 || kind == Kind::F32BF16R || kind == Kind::F32S8Q) ? 4
                      : (kind == Kind::BF16F32 || kind == Kind::E4M3BF16) ? 2 : 1;
    const size_t eb = (kind == Kind::F32 || kind == Kind::F32BF16R || kind == Kind::F32S8Q) ? 4
                      : (kind == Kind::BF16F32) ? 2 : 1;
    const size_t ec = (kind == Kind::S8S32) ? 4 : (kind == Kind::E4M3BF16 ? 2 : 4);
    // C is staged in when beta != 0, and whenever its rows are padded (ldc > N):
    // the whole span is copied back, so the padding must make the round trip.
    const bool reads_c =
        (kind != Kind::S8S32 && kind != Kind::E4M3BF16 && d->beta != 0.0f) || d->ldc > d->N;
    Operand ops[4] = {
        {A, ta ? span_bytes(d->K, d->M, d->lda, ea) : span_bytes(d->M, d->K, d->lda, ea), true, false},
        {B, tb ? span_bytes(d->N, d->K, d->ldb, eb) : span_bytes(d->K, d->N, d->ldb, eb), true, false},
        {C, span_bytes(d->M, d->N, d->ldc, ec), reads_c, true},
        {scales, kind == Kind::E4M3BF16 ? static_cast<size_t>(d->N) * 4 : 0, true, false},
    };
    const void* dev[4] = {A, B, C, scales};
    for (int i = 0; i < 4; ++i) {
        if (!ops[i].user || ops[i].bytes == 0) continue;
        if (classify_pointer(ops[i].user) == PtrKind::Device) continue;
        void* buf = nullptr;
        st = ensure_stage(ctx, i, ops[i].bytes, &buf);
        if (st != DNNOPT_STATUS_SUCCESS) return st;
        dev[i] = buf;
        if (ops[i].in) {
            int inj = check_injected_fault(3);
            if (inj != DNNOPT_STATUS_SUCCESS) return set_status(inj);
            cudaError_t e = cudaMemcpyAsync(buf, ops[i].user, ops[i].bytes, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_status(e);
        }
    }
    GemmArgs g = to_args(d, dev[0], dev[1], const_cast<void*>(dev[2]));
    st = run_device(kind, g, static_cast<const float*>(dev[3]), ctx, s);
    if (st != DNNOPT_STATUS_SUCCESS) {
        cudaStreamSynchronize(s);
        return set_status(st);
    }
    if (dev[2] != C) {
        cudaError_t e = cudaMemcpyAsync(C, dev[2], ops[2].bytes, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return cuda_status(e);
    }
    // Bounded in-kernel waits report through the stream's error word: read it
    // in the same stream, into a pinned word, so the call synchronises once.
    auto it = ctx->ws.find(s);
    const bool check_err = it != ctx->ws.end() && it->second.err;
    if (check_err && !ctx->host_err) {
        void* h = nullptr;
        if (cudaHostAlloc(&h, sizeof(uint32_t), cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            h = nullptr;
        }
        ctx->host_err = static_cast<uint32_t*>(h);
    }
    uint32_t code = 0;
    if (check_err && ctx->host_err) {
        *ctx->host_err = 0u;
        cudaError_t e = cudaMemcpyAsync(ctx->host_err, it->second.err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return cuda_status(e);
    }
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    if (check_err) {
        if (ctx->host_err) {
            code = *ctx->host_err;
        } else {
            e = cudaMemcpy(&code, it->second.err, sizeof(code), cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) return cuda_status(e);
        }
        if (code != 0) {
            // Clears the error word and the conv prep's grid-barrier and
            // absmax words (a timed-out barrier may have left them set).
            cudaMemset(it->second.err, 0, 16 * sizeof(uint32_t));
            return set_status(DNNOPT_STATUS_KERNEL_TIMEOUT);
        }
    }
    return set_status(DNNOPT_STATUS_SUCCESS);
}

dnnopt_gemm_desc make_desc(int M, int N, int K, float alpha, int lda, int ldb, float beta,
                           int ldc) {
    dnnopt_gemm_desc d;
    d.M = M; d.N = N; d.K = K;
    d.lda = lda; d.ldb = ldb; d.ldc = ldc;
    d.alpha = alpha; d.beta = beta;
    d.trans_a = 0; d.trans_b = 0;
    return d;
}

int g_num_threads = 0;

// ---- oneDNN entry (integration/onednn/0001-dnnopt-integration.patch:279-365) ----
struct ColMajorArgs {
    bool ta, tb;
    int64_t M, N, K, lda, ldb, ldc;
    float alpha, beta;
};

// Argument checks of the column-major entry.  Returns SUCCESS with *noop for
// M == 0 or N == 0 (the entry's early return).
int colmajor_parse(const char* transa, const char* transb, const int64_t* M, const int64_t* N,
                   const int64_t* K, const float* alpha, const int64_t* lda, const int64_t* ldb,
                   const float* beta, const int64_t* ldc, ColMajorArgs* a, bool* noop) {
    *noop = false;
    if (!transa || !transb || !M || !N || !K || !alpha || !lda || !ldb || !beta || !ldc)
        return DNNOPT_STATUS_INVALID_VALUE;
    // Packed operands: dnnl_unimplemented in the reference (:284-286).
    if (*transa == 'P' || *transa == 'p' || *transb == 'P' || *transb == 'p')
        return DNNOPT_STATUS_NOT_SUPPORTED;
    if (*M < 0 || *N < 0 || *K < 0) return DNNOPT_STATUS_INVALID_VALUE;
    if (*M == 0 || *N == 0) { *noop = true; return DNNOPT_STATUS_SUCCESS; }
    a->ta = *transa == 'T' || *transa == 't';
    a->tb = *transb == 'T' || *transb == 't';
    a->M = *M; a->N = *N; a->K = *K;
    a->lda = *lda; a->ldb = *ldb; a->ldc = *ldc;
    a->alpha = *alpha; a->beta = *beta;
    if (a->ldc < 1) return DNNOPT_STATUS_INVALID_VALUE;
    if (a->K > 0) {
        if (a->lda < (a->ta ? a->K : a->M) || a->ldb < (a->tb ? a->N : a->K))
            return DNNOPT_STATUS_INVALID_VALUE;
        const int64_t kIntMax = 2147483647;
        if (a->M > kIntMax || a->N > kIntMax || a->K > kIntMax || a->lda > kIntMax ||
            a->ldb > kIntMax)
            return DNNOPT_STATUS_NOT_SUPPORTED;
    }
    return DNNOPT_STATUS_SUCCESS;
}

// Bytes each column-major operand spans.
size_t colmajor_span(int64_t rows, int64_t cols, int64_t ld) {
    if (rows <= 0 || cols <= 0) return 0;
    return static_cast<size_t>((cols - 1) * ld + rows) * sizeof(float);
}

// Device pointers, stream-ordered.  The column-major GEMM is the row-major one
// with the operands swapped, RowMajor(op B, op A, N, M, K, B, ldb, A, lda, C, ldc)
// (:306-329); transposes are kernel flags, not copies.  ldc >= M: the bias is
// fused into the GEMM's epilogue.  ldc < M (:330-353): the GEMM writes a dense
// N x M scratch that is copied back in the entry's order.
int colmajor_device(const ColMajorArgs& a, const float* A, const float* B, float* C,
                    const float* bias, DeviceContext* ctx, cudaStream_t s) {
    if (a.K == 0) {
        cudaError_t e = launch_colmajor_k0(C, bias, a.M, a.N, a.ldc, a.beta, s);
        note_launch();
        return cuda_status(e);
    }
    GemmArgs g;
    g.M = static_cast<int>(a.N); g.N = static_cast<int>(a.M); g.K = static_cast<int>(a.K);
    g.alpha = a.alpha; g.beta = a.beta;
    g.A = B; g.lda = a.ldb; g.a_trans = a.tb ? 1 : 0;
    g.B = A; g.ldb = a.lda; g.b_trans = a.ta ? 1 : 0;
    if (a.ldc >= a.M) {
        g.C = C; g.ldc = a.ldc; g.bias = bias;
        return run_device(Kind::F32, g, nullptr, ctx, s);
    }
    Workspace* w = nullptr;
    const size_t tmp_bytes = static_cast<size_t>(a.M) * a.N * sizeof(float);
    int st = ensure_workspace(ctx, s, 0, 0, tmp_bytes, &w);
    if (st != DNNOPT_STATUS_SUCCESS) return st;
    float* tmp = static_cast<float*>(w->quant);
    if (a.beta != 0.0f) {
        cudaError_t e = launch_colmajor_gather(tmp, C, a.M, a.N, a.ldc, s);
        note_launch();
        if (e != cudaSuccess) return cuda_status(e);
    }
    g.C = tmp; g.ldc = a.M;
    st = run_device(Kind::F32, g, nullptr, ctx, s);
    if (st != DNNOPT_STATUS_SUCCESS) return st;
    cudaError_t e = launch_colmajor_writeback(C, tmp, a.M, bias, a.M, a.N, a.ldc, s);
    note_launch();
    return cuda_status(e);
}

// ---- Conv3D (reference src/conv/conv3d.cpp) --------------------------------
// Geometry and argument checks; *noop for the reference's early return
// (N, IC or OC <= 0) and for an empty output.
int conv3d_geom(int precision, const dnnopt_conv3d_params* p, int post_op, Conv3dGeom* g, bool* noop) {
    *noop = false;
    if (!p || precision < DNNOPT_CONV3D_FP32 || precision > DNNOPT_CONV3D_INT8 ||
        post_op < DNNOPT_POSTOP_NONE || post_op > DNNOPT_POSTOP_RELU6)
        return DNNOPT_STATUS_INVALID_VALUE;
    if (p->N <= 0 || p->OC <= 0 || p->IC <= 0) { *noop = true; return DNNOPT_STATUS_SUCCESS; }
    if (p->ID < 0 || p->IH < 0 || p->IW < 0 || p->KD < 1 || p->KH < 1 || p->KW < 1 ||
        p->stride_d < 1 || p->stride_h < 1 || p->stride_w < 1 || p->pad_d < 0 || p->pad_h < 0 ||
        p->pad_w < 0)
        return DNNOPT_STATUS_INVALID_VALUE;
    Conv3dGeom q;
    q.N = p->N; q.IC = p->IC; q.ID = p->ID; q.IH = p->IH; q.IW = p->IW; q.OC = p->OC;
    q.KD = p->KD; q.KH = p->KH; q.KW = p->KW;
    q.sd = p->stride_d; q.sh = p->stride_h; q.sw = p->stride_w;
    q.pd = p->pad_d; q.ph = p->pad_h; q.pw = p->pad_w;
    // Conv3DParams::OD/OH/OW (include/dnnopt/conv/conv3d.h:26-32), C integer division.
    q.OD = (q.ID + 2 * q.pd - q.KD) / q.sd + 1;
    q.OH = (q.IH + 2 * q.ph - q.KH) / q.sh + 1;
    q.OW = (q.IW + 2 * q.pw - q.KW) / q.sw + 1;
    if (q.OD <= 0 || q.OH <= 0 || q.OW <= 0) { *noop = true; return DNNOPT_STATUS_SUCCESS; }
    const int64_t taps = static_cast<int64_t>(q.KD) * q.KH * q.KW;
    q.M = static_cast<int64_t>(q.N) * q.OD * q.OH * q.OW;
    q.K = taps * q.IC;
    if (taps > kConv3dMaxTaps || q.M > 2147483647 || q.K > 2147483647)
        return DNNOPT_STATUS_NOT_SUPPORTED;
    *g = q;
    return DNNOPT_STATUS_SUCCESS;
}

// Device pointers, stream-ordered: scales (INT8), column matrix and filter in
// the compute precision, the library GEMM (FP32 / BF16 -> FP32 / INT8 ->
// INT32, filter as the N x K operand), then bias, dequantisation and post-op.
int conv3d_device(int precision, const Conv3dGeom& g, const float* in, const float* f, const float* bias,
                  float* out, int op, DeviceContext* ctx, cudaStream_t s) {
    // FP32 with IC % 4 == 0: one implicit-GEMM launch that gathers the column
    // matrix tile by tile from the input (no M x K scratch), bias and post-op
    // in its epilogue.
    if (precision == DNNOPT_CONV3D_FP32 && gemm_simt_conv_ok(g, in, f)) {
        const cudaError_t e = launch_gemm_simt_conv(g, in, f, bias, op, out, ctx->num_sms, s);
        note_launch();
        return cuda_status(e);
    }
    const size_t eb = precision == DNNOPT_CONV3D_FP32 ? 4 : (precision == DNNOPT_CONV3D_BF16 ? 2 : 1);
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    // BF16 / INT8 with stride 1 and channel rows of a 32-byte multiple: the
    // operands converted (or quantised) once, then one implicit tcgen05 launch
    // with bias, dequantisation and post-op in its epilogue.
    if (precision != DNNOPT_CONV3D_FP32 && conv3d_tc_ok(g, precision)) {
        const size_t cb = precision == DNNOPT_CONV3D_BF16 ? 2 : 1;
        const int64_t cf = static_cast<int64_t>(g.OC) * g.K;
        const size_t in_b = up(conv3d_tc_input_bytes(g, precision)), f_b = up(static_cast<size_t>(cf) * cb);
        Workspace* w = nullptr;
        int st = ensure_workspace(ctx, s, 0, 0, in_b + f_b, &w);
        if (st != DNNOPT_STATUS_SUCCESS) return st;
        char* base = static_cast<char*>(w->quant);
        // INT8 prep: grid-barrier words = the two spare absmax words, absmax
        // slots = the four words after the scales.
        cudaError_t e = launch_conv3d_tc_prep(g, precision, in, f, base, base + in_b, w->absmax + 2,
                                              reinterpret_cast<uint32_t*>(w->scales) + 4, w->scales, w->err,
                                              ctx->num_sms, s);
        note_launch();
        if (e == cudaSuccess) {
            e = launch_conv3d_tc(g, precision, base, base + in_b, w->scales, bias, op, out, w->err, ctx->num_sms, s);
            note_launch();
        }
        return cuda_status(e);
    }
    // INT8 with IC % 16 == 0 and M >= 64: the dp4a kernel gathers 16-byte
    // channel segments from the quantised input, so no column matrix (the
    // workspace buffers are 256-byte aligned, so only the geometry decides).
    // When the column matrix can feed the tcgen05 GEMM (dense int8 rows of a
    // 16-byte multiple), materialising it and running kind::i8 beats the
    // dp4a implicit GEMM (the column matrix write costs less than the dp4a
    // arithmetic), so the implicit form is kept for the other shapes.
    GemmArgs probe{};
    probe.M = static_cast<int>(g.M); probe.N = g.OC; probe.K = static_cast<int>(g.K);
    // The column matrix and the quantised filter live in the 256-byte aligned
    // workspace: only the geometry decides (the address is never dereferenced).
    const void* ws_like = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
    probe.A = ws_like; probe.lda = g.K; probe.B = ws_like; probe.ldb = g.K; probe.b_trans = 1;
    probe.C = out; probe.ldc = g.OC;
    const bool tc8 = precision == DNNOPT_CONV3D_INT8 && g.M > 8 && gemm_tc_supported(TcKind::I8, probe);
    const bool implicit8 = precision == DNNOPT_CONV3D_INT8 && !tc8 && gemm_tile_s8_conv_ok(g, nullptr, nullptr);
    const size_t col_b = implicit8 ? 0 : up(static_cast<size_t>(g.M) * g.K * eb);
    const size_t flt_b = precision ? up(static_cast<size_t>(g.OC) * g.K * eb) : 0;
    const size_t acc_b = precision == DNNOPT_CONV3D_INT8 && !implicit8 ? up(static_cast<size_t>(g.M) * g.OC * 4) : 0;
    const int64_t nin = static_cast<int64_t>(g.N) * g.ID * g.IH * g.IW * g.IC;
    // BF16 / INT8 with whole 16-byte channel chunks: the input is converted
    // once into the workspace and im2col copies its chunks.
    const bool copy = precision != DNNOPT_CONV3D_FP32 && conv3d_copy_im2col_ok(g, precision);
    const size_t in_b = copy ? up(static_cast<size_t>(nin) * eb) : 0;
    Workspace* w = nullptr;
    int st = ensure_workspace(ctx, s, 0, 0, col_b + flt_b + acc_b + in_b, &w);
    if (st != DNNOPT_STATUS_SUCCESS) return st;
    char* base = static_cast<char*>(w->quant);
    void* col = base;
    void* fq = base + col_b;
    int32_t* acc = reinterpret_cast<int32_t*>(base + col_b + flt_b);
    void* inq = base + col_b + flt_b + acc_b;
    const int64_t nf = static_cast<int64_t>(g.OC) * g.K;
    cudaError_t e = cudaSuccess;
    if (implicit8) {   // absmax; scales + quantised input and filter; GEMM with the epilogue
        e = launch_conv3d_absmax_quant(in, nin, f, nf, w->absmax, w->scales, static_cast<int8_t*>(inq),
                                       static_cast<int8_t*>(fq), s);
        note_launch(2);
        if (e == cudaSuccess) {
            e = launch_gemm_tile_s8_conv(g, static_cast<const int8_t*>(inq), static_cast<const int8_t*>(fq),
                                         w->scales, bias, op, out, s);
            note_launch();
        }
        return cuda_status(e);
    }
    if (precision == DNNOPT_CONV3D_INT8) {
        e = launch_conv3d_scales(in, nin, f, nf, w->absmax, w->scales, s);
        note_launch(2);
        if (e != cudaSuccess) return cuda_status(e);
    }
    if (copy) {
        e = launch_conv3d_filter(precision, in, inq, nin, w->scales, s, 2);
        note_launch();
        if (e == cudaSuccess) e = launch_conv3d_im2col_copy(g, precision, inq, col, s);
    } else {
        e = launch_conv3d_im2col(g, precision, in, col, w->scales, s);
    }
    note_launch();
    if (e == cudaSuccess && precision != DNNOPT_CONV3D_FP32) {
        e = launch_conv3d_filter(precision, f, fq, nf, w->scales, s);
        note_launch();
    }
    if (e != cudaSuccess) return cuda_status(e);
    GemmArgs ga;
    ga.M = static_cast<int>(g.M); ga.N = g.OC; ga.K = static_cast<int>(g.K);
    ga.alpha = 1.0f; ga.beta = 0.0f;
    ga.A = col; ga.lda = g.K; ga.a_trans = 0;
    ga.B = precision == DNNOPT_CONV3D_FP32 ? static_cast<const void*>(f) : fq;
    ga.ldb = g.K; ga.b_trans = 1;
    ga.C = precision == DNNOPT_CONV3D_INT8 ? static_cast<void*>(acc) : static_cast<void*>(out);
    ga.ldc = g.OC;
    const Kind kind = precision == DNNOPT_CONV3D_FP32 ? Kind::F32
                      : (precision == DNNOPT_CONV3D_BF16 ? Kind::BF16F32 : Kind::S8S32);
    st = run_device(kind, ga, nullptr, ctx, s);
    if (st != DNNOPT_STATUS_SUCCESS) return st;
    if (precision == DNNOPT_CONV3D_INT8 || bias || op != DNNOPT_POSTOP_NONE) {
        e = launch_conv3d_post(out, precision == DNNOPT_CONV3D_INT8 ? acc : nullptr, w->scales, bias, g.M,
                               g.OC, op, s);
        note_launch();
    }
    return cuda_status(e);
}

}  // namespace

extern "C" {

// ---- reference-signature (host or device pointers, synchronous) ----------
int dnnopt_gemm_fp32(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
                     int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, alpha, lda, ldb, beta, ldc);
    return host_entry(Kind::F32, &d, A, B, C, nullptr);
}

int dnnopt_gemm_bf16(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
                     int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, alpha, lda, ldb, beta, ldc);
    return host_entry(Kind::F32BF16R, &d, A, B, C, nullptr);
}

int dnnopt_gemm_bf16_bf16bf16f32(int M, int N, int K, float alpha, const uint16_t* A, int lda,
                                 const uint16_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, alpha, lda, ldb, beta, ldc);
    return host_entry(Kind::BF16F32, &d, A, B, C, nullptr);
}

int dnnopt_gemm_int8(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
                     int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, alpha, lda, ldb, beta, ldc);
    return host_entry(Kind::F32S8Q, &d, A, B, C, nullptr);
}

int dnnopt_gemm_int8_int8int8int32(int M, int N, int K, const int8_t* A, int lda, const int8_t* B,
                                   int ldb, int32_t* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, 1.0f, lda, ldb, 0.0f, ldc);
    return host_entry(Kind::S8S32, &d, A, B, C, nullptr);
}

int dnnopt_gemm_fp8_e4m3(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                         const uint8_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, alpha, lda, ldb, beta, ldc);
    return host_entry(Kind::RE4E5, &d, A, B, C, nullptr);
}

int dnnopt_gemm_fp8_e5m2(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                         const uint8_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, alpha, lda, ldb, beta, ldc);
    return host_entry(Kind::RE5E5, &d, A, B, C, nullptr);
}

int dnnopt_gemm_fp8(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
                    int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, alpha, lda, ldb, beta, ldc);
    bool noop;
    int st = validate(Kind::F32, &d, A, B, C, &noop);
    if (st != DNNOPT_STATUS_SUCCESS || noop) return set_status(st);
    // Quantise with the reference codecs on the device, then gemm_fp8_e4m3.
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    const size_t qa = static_cast<size_t>(M) * K, qb = static_cast<size_t>(K) * N;
    void* dA = nullptr;
    void* dB = nullptr;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        cudaStream_t s = ctx->user_stream_set ? ctx->user_stream : ctx->default_stream;
        const void* src[2] = {A, B};
        const size_t bytes[2] = {span_bytes(M, K, lda, 4), span_bytes(K, N, ldb, 4)};
        for (int i = 0; i < 2; ++i) {
            if (classify_pointer(src[i]) == PtrKind::Device) {
                (i == 0 ? dA : dB) = const_cast<void*>(src[i]);
                continue;
            }
            void* buf = nullptr;
            st = ensure_stage(ctx, i, bytes[i], &buf);
            if (st != DNNOPT_STATUS_SUCCESS) return st;
            cudaError_t e = cudaMemcpyAsync(buf, src[i], bytes[i], cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_status(e);
            (i == 0 ? dA : dB) = buf;
        }
        void* q = nullptr;
        st = ensure_stage(ctx, 3, qa + qb, &q);
        if (st != DNNOPT_STATUS_SUCCESS) return st;
        GemmArgs g = to_args(&d, dA, dB, C);
        cudaError_t e = launch_quantize_ref_fp8(g, static_cast<uint8_t*>(q),
                                                static_cast<uint8_t*>(q) + qa, s);
        note_launch();
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_status(e);
        dA = q;
        dB = static_cast<uint8_t*>(q) + qa;
    }
    // dA/dB are device buffers now (stage slot 3); the call below only stages C.
    dnnopt_gemm_desc dq = make_desc(M, N, K, alpha, K, N, beta, ldc);
    return host_entry(Kind::RE4E5, &dq, dA, dB, C, nullptr);
}

int dnnopt_has_fp8_support(void) { return 1; }

int dnnopt_gemm_f32_desc(const dnnopt_gemm_desc* d, const float* A, const float* B, float* C) {
    return host_entry(Kind::F32, d, A, B, C, nullptr);
}

int dnnopt_conv3d(int precision, const dnnopt_conv3d_params* p, const float* input,
                  const float* filter, const float* bias, float* output, int post_op) {
    Conv3dGeom g;
    bool noop;
    int st = conv3d_geom(precision, p, post_op, &g, &noop);
    if (st != DNNOPT_STATUS_SUCCESS || noop) return set_status(st);
    if (!input || !filter || !output) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaStream_t s = ctx->user_stream_set ? ctx->user_stream : ctx->default_stream;
    const size_t nin = static_cast<size_t>(g.N) * g.ID * g.IH * g.IW * g.IC;
    Operand ops[4] = {
        {input, nin * sizeof(float), true, false},
        {filter, static_cast<size_t>(g.OC) * g.K * sizeof(float), true, false},
        {bias, bias ? static_cast<size_t>(g.OC) * sizeof(float) : 0, true, false},
        {output, static_cast<size_t>(g.M) * g.OC * sizeof(float), false, true},
    };
    const void* dev[4] = {input, filter, bias, output};
    for (int i = 0; i < 4; ++i) {
        if (!ops[i].user || ops[i].bytes == 0) continue;
        if (classify_pointer(ops[i].user) == PtrKind::Device) continue;
        void* buf = nullptr;
        st = ensure_stage(ctx, i, ops[i].bytes, &buf);
        if (st != DNNOPT_STATUS_SUCCESS) return st;
        dev[i] = buf;
        if (ops[i].in) {
            cudaError_t e = cudaMemcpyAsync(buf, ops[i].user, ops[i].bytes, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_status(e);
        }
    }
    st = conv3d_device(precision, g, static_cast<const float*>(dev[0]), static_cast<const float*>(dev[1]),
                       static_cast<const float*>(dev[2]), static_cast<float*>(const_cast<void*>(dev[3])),
                       post_op, ctx, s);
    if (st != DNNOPT_STATUS_SUCCESS) {
        cudaStreamSynchronize(s);
        return set_status(st);
    }
    if (dev[3] != output) {
        cudaError_t e = cudaMemcpyAsync(output, dev[3], ops[3].bytes, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return cuda_status(e);
    }
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    return set_status(DNNOPT_STATUS_SUCCESS);
}

int dnnopt_sgemm_colmajor(const char* transa, const char* transb, const int64_t* M,
                          const int64_t* N, const int64_t* K, const float* alpha, const float* A,
                          const int64_t* lda, const float* B, const int64_t* ldb,
                          const float* beta, float* C, const int64_t* ldc, const float* bias) {
    ColMajorArgs a;
    bool noop;
    int st = colmajor_parse(transa, transb, M, N, K, alpha, lda, ldb, beta, ldc, &a, &noop);
    if (st != DNNOPT_STATUS_SUCCESS || noop) return set_status(st);
    if (!C || (a.K > 0 && (!A || !B))) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaStream_t s = ctx->user_stream_set ? ctx->user_stream : ctx->default_stream;
    // The K == 0 path reads C whatever beta is; otherwise C is read for
    // beta != 0, and staged in whenever its columns are padded (ldc > M) so
    // that the padding survives the copy back of the whole span.
    const bool reads_c = a.K == 0 || a.beta != 0.0f || a.ldc > a.M;
    Operand ops[4] = {
        {A, a.K > 0 ? (a.ta ? colmajor_span(a.K, a.M, a.lda) : colmajor_span(a.M, a.K, a.lda)) : 0,
         true, false},
        {B, a.K > 0 ? (a.tb ? colmajor_span(a.N, a.K, a.ldb) : colmajor_span(a.K, a.N, a.ldb)) : 0,
         true, false},
        {C, colmajor_span(a.M, a.N, a.ldc), reads_c, true},
        {bias, bias ? static_cast<size_t>(a.M) * sizeof(float) : 0, true, false},
    };
    const void* dev[4] = {A, B, C, bias};
    for (int i = 0; i < 4; ++i) {
        if (!ops[i].user || ops[i].bytes == 0) continue;
        if (classify_pointer(ops[i].user) == PtrKind::Device) continue;
        void* buf = nullptr;
        st = ensure_stage(ctx, i, ops[i].bytes, &buf);
        if (st != DNNOPT_STATUS_SUCCESS) return st;
        dev[i] = buf;
        if (ops[i].in) {
            cudaError_t e = cudaMemcpyAsync(buf, ops[i].user, ops[i].bytes, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_status(e);
        }
    }
    st = colmajor_device(a, static_cast<const float*>(dev[0]), static_cast<const float*>(dev[1]),
                         static_cast<float*>(const_cast<void*>(dev[2])),
                         static_cast<const float*>(dev[3]), ctx, s);
    if (st != DNNOPT_STATUS_SUCCESS) {
        cudaStreamSynchronize(s);
        return set_status(st);
    }
    if (dev[2] != C) {
        cudaError_t e = cudaMemcpyAsync(C, dev[2], ops[2].bytes, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return cuda_status(e);
    }
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    return set_status(DNNOPT_STATUS_SUCCESS);
}

int dnnopt_saxpy(int N, float alpha, const float* X, int incX, float* Y, int incY) {
    if (N <= 0 || alpha == 0.0f) return set_status(DNNOPT_STATUS_SUCCESS);   // reference early return
    if (!X || !Y || incX < 0 || incY < 0) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    int st;
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaStream_t s = ctx->user_stream_set ? ctx->user_stream : ctx->default_stream;
    const size_t xb = (static_cast<size_t>(N - 1) * incX + 1) * 4;
    const size_t yb = (static_cast<size_t>(N - 1) * incY + 1) * 4;
    const float* dx = X;
    float* dy = Y;
    if (classify_pointer(X) == PtrKind::Host) {
        void* b = nullptr;
        if ((st = ensure_stage(ctx, 0, xb, &b)) != DNNOPT_STATUS_SUCCESS) return st;
        cudaError_t e = cudaMemcpyAsync(b, X, xb, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_status(e);
        dx = static_cast<const float*>(b);
    }
    if (classify_pointer(Y) == PtrKind::Host) {
        void* b = nullptr;
        if ((st = ensure_stage(ctx, 2, yb, &b)) != DNNOPT_STATUS_SUCCESS) return st;
        cudaError_t e = cudaMemcpyAsync(b, Y, yb, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_status(e);
        dy = static_cast<float*>(b);
    }
    cudaError_t e = launch_saxpy(N, alpha, dx, incX, dy, incY, s);
    note_launch();
    if (e == cudaSuccess && dy != Y) e = cudaMemcpyAsync(Y, dy, yb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return cuda_status(e);
}

int dnnopt_gemm_e4m3_bf16(int M, int N, int K, const uint16_t* A, int lda, const uint8_t* W,
                          int ldw, const float* scale, uint16_t* C, int ldc) {
    dnnopt_gemm_desc d = make_desc(M, N, K, 1.0f, lda, ldw, 0.0f, ldc);
    return host_entry(Kind::E4M3BF16, &d, A, W, C, scale);
}

void dnnopt_gemm_set_num_threads(int n) { g_num_threads = n < 0 ? 0 : n; }
int dnnopt_gemm_get_num_threads(void) { return g_num_threads > 0 ? g_num_threads : 1; }

// ---- device-pointer entry points ------------------------------------------
int dnnopt_cuda_conv3d(int precision, const dnnopt_conv3d_params* p, const float* input,
                       const float* filter, const float* bias, float* output, int post_op,
                       void* stream) {
    Conv3dGeom g;
    bool noop;
    int st = conv3d_geom(precision, p, post_op, &g, &noop);
    if (st != DNNOPT_STATUS_SUCCESS || noop) return set_status(st);
    if (!input || !filter || !output) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    return set_status(conv3d_device(precision, g, input, filter, bias, output, post_op, ctx,
                                    static_cast<cudaStream_t>(stream)));
}

int dnnopt_cuda_sgemm_colmajor(const char* transa, const char* transb, const int64_t* M,
                               const int64_t* N, const int64_t* K, const float* alpha,
                               const float* A, const int64_t* lda, const float* B,
                               const int64_t* ldb, const float* beta, float* C, const int64_t* ldc,
                               const float* bias, void* stream) {
    ColMajorArgs a;
    bool noop;
    int st = colmajor_parse(transa, transb, M, N, K, alpha, lda, ldb, beta, ldc, &a, &noop);
    if (st != DNNOPT_STATUS_SUCCESS || noop) return set_status(st);
    if (!C || (a.K > 0 && (!A || !B))) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    return set_status(colmajor_device(a, A, B, C, bias, ctx, static_cast<cudaStream_t>(stream)));
}

int dnnopt_cuda_gemm_f32(const dnnopt_gemm_desc* d, const float* A, const float* B, float* C,
                         void* stream) {
    return device_entry(Kind::F32, d, A, B, C, nullptr, stream);
}
int dnnopt_cuda_gemm_bf16f32(const dnnopt_gemm_desc* d, const uint16_t* A, const uint16_t* B,
                             float* C, void* stream) {
    return device_entry(Kind::BF16F32, d, A, B, C, nullptr, stream);
}
int dnnopt_cuda_gemm_f32_bf16round(const dnnopt_gemm_desc* d, const float* A, const float* B,
                                   float* C, void* stream) {
    return device_entry(Kind::F32BF16R, d, A, B, C, nullptr, stream);
}
int dnnopt_cuda_gemm_f32_s8quant(const dnnopt_gemm_desc* d, const float* A, const float* B,
                                 float* C, void* stream) {
    return device_entry(Kind::F32S8Q, d, A, B, C, nullptr, stream);
}
int dnnopt_cuda_gemm_s8s32(const dnnopt_gemm_desc* d, const int8_t* A, const int8_t* B,
                           int32_t* C, void* stream) {
    return device_entry(Kind::S8S32, d, A, B, C, nullptr, stream);
}
int dnnopt_cuda_gemm_e4m3bf16(const dnnopt_gemm_desc* d, const uint16_t* A, const uint8_t* W,
                              const float* scale, uint16_t* C, void* stream) {
    return device_entry(Kind::E4M3BF16, d, A, W, C, scale, stream);
}
int dnnopt_cuda_gemm_refe4m3_e5m2(const dnnopt_gemm_desc* d, const uint8_t* A, const uint8_t* B,
                                  float* C, void* stream) {
    return device_entry(Kind::RE4E5, d, A, B, C, nullptr, stream);
}
int dnnopt_cuda_gemm_refe5m2_e5m2(const dnnopt_gemm_desc* d, const uint8_t* A, const uint8_t* B,
                                  float* C, void* stream) {
    return device_entry(Kind::RE5E5, d, A, B, C, nullptr, stream);
}

// ---- multi-GPU --------------------------------------------------------------
int dnnopt_peer_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    *ptr = nullptr;
    int st;
    if (!current_context(&st)) return st;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_status(DNNOPT_STATUS_ALLOC_FAILED);
    }
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_status(e);
    }
    *ptr = p;
    return set_status(DNNOPT_STATUS_SUCCESS);
}

int dnnopt_peer_free(void* ptr) {
    if (!ptr) return set_status(DNNOPT_STATUS_SUCCESS);
    return cuda_status(cudaFree(ptr));
}

int dnnopt_ipc_handle(const void* ptr, unsigned char handle[64]) {
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    if (!ptr || !handle) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return cuda_status(e);
    std::memcpy(handle, &h, sizeof(h));
    return set_status(DNNOPT_STATUS_SUCCESS);
}

int dnnopt_ipc_open(const unsigned char handle[64], void** ptr) {
    if (!handle || !ptr) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    *ptr = nullptr;
    int st;
    if (!current_context(&st)) return st;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int dnnopt_ipc_close(void* ptr) {
    if (!ptr) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    return cuda_status(cudaIpcCloseMemHandle(ptr));
}

int dnnopt_cuda_gemm_e4m3bf16_allgather(const dnnopt_gemm_desc* d, const uint16_t* A,
                                        const uint8_t* W, const float* scale,
                                        const dnnopt_allgather_desc* ag, void* stream) {
    if (!ag || ag->world < 1 || ag->world > DNNOPT_MAX_RANKS || ag->rank < 0 || ag->rank >= ag->world ||
        !ag->seq || ag->out_stride % 2 != 0)
        return set_status(DNNOPT_STATUS_INVALID_VALUE);
    for (int q = 0; q < ag->world; ++q)
        if (!ag->out[q] || !ag->flags[q]) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    bool noop;
    int st = validate(Kind::E4M3BF16, d, A, W, ag->out[ag->rank], &noop);
    if (st != DNNOPT_STATUS_SUCCESS) return set_status(st);
    if (noop || !scale || static_cast<int64_t>(d->ldc) < static_cast<int64_t>(ag->world) * d->N)
        return set_status(DNNOPT_STATUS_INVALID_VALUE);
    if (d->M > 8) return set_status(DNNOPT_STATUS_NOT_SUPPORTED);
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GemmArgs g = to_args(d, A, W, ag->out[ag->rank]);
    g.b_trans = 1;
    Plan p = get_plan(Kind::E4M3BF16, g, ctx, s, scale);
    if (p.kernel != KernelId::E4m3Tc) return set_status(DNNOPT_STATUS_NOT_SUPPORTED);
    int inj = check_injected_fault(2);
    if (inj != DNNOPT_STATUS_SUCCESS) return set_status(inj);
    const size_t tiles = static_cast<size_t>((g.N + 127) / 128);
    Workspace* w = nullptr;
    st = ensure_workspace(ctx, s, gemm_e4m3_tc_ws_floats(g, p.e4), tiles + 1,
                          gemm_e4m3_tc_act_bytes(g), &w);
    if (st != DNNOPT_STATUS_SUCCESS) return st;
    AllGatherArgs a;
    a.world = ag->world;
    a.rank = ag->rank;
    for (int q = 0; q < kAllGatherMaxRanks; ++q) {
        a.out[q] = q < ag->world ? ag->out[q] : nullptr;
        a.flag[q] = q < ag->world ? ag->flags[q] : nullptr;
    }
    a.done = w->counters + tiles;      // the tile tickets occupy counters[0, tiles)
    a.seq = ag->seq;
    a.out_stride_elems = static_cast<int64_t>(ag->out_stride / 2);
    cudaError_t e = launch_gemm_e4m3_tc(g, p.e4, scale, w->ws, w->counters, w->quant, w->err, s, &a);
    note_launch(2);
    if (e == cudaSuccess) {
        e = launch_peer_wait(ag->flags[ag->rank], ag->world, 0u, ag->seq, 2000000000ull /* 2 s */,
                             w->err, s);
        note_launch();
    }
    return cuda_status(e);
}

int dnnopt_cuda_peer_wait(const unsigned int* flags, int world, unsigned int epoch,
                          unsigned int timeout_us, void* stream) {
    if (!flags || world < 1 || world > DNNOPT_MAX_RANKS) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    int st;
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Workspace* w = nullptr;
    st = ensure_workspace(ctx, s, 0, 0, 0, &w);
    if (st != DNNOPT_STATUS_SUCCESS) return st;
    cudaError_t e = launch_peer_wait(flags, world, epoch, nullptr,
                                     static_cast<uint64_t>(timeout_us) * 1000ull, w->err, s);
    note_launch();
    return cuda_status(e);
}

int dnnopt_stream_status(void* stream) {
    int st;
    DeviceContext* ctx = current_context(&st);
    if (!ctx) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    auto it = ctx->ws.find(s);
    if (it != ctx->ws.end() && it->second.err) {
        uint32_t code = 0;
        e = cudaMemcpy(&code, it->second.err, sizeof(code), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_status(e);
        if (code != 0) {
            // Clears the error word and the conv prep's grid-barrier and
            // absmax words (a timed-out barrier may have left them set).
            cudaMemset(it->second.err, 0, 16 * sizeof(uint32_t));
            return set_status(DNNOPT_STATUS_KERNEL_TIMEOUT);
        }
    }
    return set_status(DNNOPT_STATUS_SUCCESS);
}

// ---- plan / autotune --------------------------------------------------------
int dnnopt_plan_describe(int kind, const dnnopt_gemm_desc* d, char* buf, int len) {
    if (!d || !buf || len <= 0 || kind < 0 || kind > 7) return set_status(DNNOPT_STATUS_INVALID_VALUE);
    Kind k = static_cast<Kind>(kind);
    GemmArgs g = to_args(d, nullptr, nullptr, nullptr);
    if (b_is_nk(k)) g.b_trans = 1;
    DeviceInfo info;
    int dev = -1;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int st;
        DeviceContext* ctx = current_context(&st);
        if (ctx) info = info_of(ctx);
    } else {
        cudaGetLastError();
    }
    std::string s = describe_plan(k, g, heuristic_plan(k, g, info));
    std::snprintf(buf, static_cast<size_t>(len), "%s", s.c_str());
    return set_status(DNNOPT_STATUS_SUCCESS);
}

int dnnopt_autotune_enable(int on) {
    set_autotune_enabled(on != 0);
    return set_status(DNNOPT_STATUS_SUCCESS);
}
int dnnopt_autotune_save(const char* path) {
    if (!path) return -1;
    return cache_save(path);
}
int dnnopt_autotune_load(const char* path) {
    if (!path) return -1;
    return cache_load(path);
}
int dnnopt_autotune_entries(void) { return cache_entries(); }

}  // extern "C"
