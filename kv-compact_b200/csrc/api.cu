// api.cu — the drop-in C ABI (include/kv-compact-api.h) over the device engine.
//
// Host pointers in, malloc'd host arrays out, as in the reference
// (src/kv-compact-api.cpp:333-1268). Each call stages its inputs to the
// current CUDA device, runs the pipeline of engine.cu on that device's
// stream, computes the quality stats on the device and copies the results
// back. Calls are serialised per device by the context mutex and may run
// concurrently on different devices.
#include <stdlib.h>

#include <algorithm>
#include <chrono>
#include <vector>

#include "engine.h"

namespace {

using clk = std::chrono::steady_clock;
double ms_since(clk::time_point t0) {
    return std::chrono::duration<double, std::milli>(clk::now() - t0).count();
}

// arena slots: 0-2 engine scratch, 4 metrics, 3/6 fp32 K/V (ping-pong), 5 io, 7 quantised io

// Returning from a call with an upload still in flight on the copy stream
// would let the caller reuse its input buffers too early, and one with a
// download in flight would let it free result arrays still being written:
// every return path waits for both streams (a no-op on the success path,
// which has already drained them).
struct io_stream_guard {
    kvc_ctx * ctx;
    ~io_stream_guard() {
        cudaStreamSynchronize(ctx->copy_stream);
        for (auto gs : ctx->group_stream) cudaStreamSynchronize(gs);
        cudaStreamSynchronize(ctx->d2h_stream);
    }
};
enum { SLOT_KV_A = 3, SLOT_IO = 5, SLOT_KV_B = 6, SLOT_QIO = 7 };

struct dev_out {
    kvc_plan plan;
    int * sel = nullptr;
    float * beta = nullptr;
    float * cv = nullptr;
    float * Q = nullptr;      // top-level queries on the device
    float * rkv_w = nullptr;  // R-KV weights on the device (null: none)
    std::vector<float> w;     // their host copy (source of the upload)
    float * d_res = nullptr;  // metric triples on the device (null: no metrics)
    int pairs = 0;
    std::vector<float> h_res; // their host copy
    kv_compact_stats stats{};
};

// Device->host copies through the pinned staging buffer: every copy is
// queued on the stream, one wait, then the staged bytes are spread over host
// threads into the (freshly malloc'd) destinations.
struct d2h_piece { void * host; const void * dev; size_t bytes; };
int gather_to_host(kvc_ctx * ctx, const std::vector<d2h_piece> & v) {
    size_t tot = 0;
    for (const auto & x : v) tot += (x.bytes + 255) & ~(size_t)255;
    void * pin;
    int rc;
    if ((rc = kvc_pinned(ctx, tot, &pin))) return rc;
    std::vector<kvc_copy_piece> pieces;
    size_t off = 0;
    for (const auto & x : v) {
        if (!x.bytes) continue;
        if (kvc_is_pinned(x.host)) {          // page-locked result array: copy straight into it
            KVC_CUDA(cudaMemcpyAsync(x.host, x.dev, x.bytes, cudaMemcpyDeviceToHost, ctx->stream));
            continue;
        }
        KVC_CUDA(cudaMemcpyAsync((char *)pin + off, x.dev, x.bytes, cudaMemcpyDeviceToHost, ctx->stream));
        pieces.push_back({x.host, (char *)pin + off, x.bytes});
        off += (x.bytes + 255) & ~(size_t)255;
    }
    if ((rc = kvc_wait(ctx))) return rc;
    kvc_parallel_copy(pieces);
    return KVC_OK;
}

// After the stream has drained and h_res holds the triples: stats of the call.
void finish_dev(kvc_ctx * ctx, dev_out * d) {
    kvc_phase_ms ph;
    kvc_phase_collect(ctx, &ph);
    d->stats.scoring_ms = ph.scoring_ms;
    d->stats.nnls_ms = ph.refit_ms;
    if (d->d_res) kvc_metrics_reduce(d->h_res.data(), d->pairs, &d->stats);
}

// Device side of one call, part 1: the io arena (Q | R-KV weights | sel |
// beta | C_v, sized from out->plan), the top-level queries (uploaded, or
// sampled from dK, which must then be resident) and the R-KV weights.
int stage_call(kvc_ctx * ctx, const float * dK, const float * hQ, int T, int H, int dk, int dv,
               const kv_compact_params & p, dev_out * out) {
    const kvc_plan & pl = out->plan;
    const int ek = H * dk;
    const int t = pl.t_total;
    const bool rkv = p.reasoning && p.reasoning->classifier;
    size_t nQ = (size_t)pl.nq_top * ek, nW = rkv ? (size_t)T : 0;
    size_t bytes = (nQ + nW + (size_t)t + (size_t)H * t + (size_t)H * t * dv + 64) * 4;
    void * a;
    int rc;
    if ((rc = kvc_arena(ctx, SLOT_IO, bytes, &a))) return rc;
    float * base = (float *)a;
    out->Q = base;
    float * dW = out->Q + ((nQ + 31) & ~31ULL);
    out->sel = (int *)(dW + ((nW + 31) & ~31ULL));
    out->beta = (float *)(out->sel + ((t + 31) & ~31));
    out->cv = out->beta + (((size_t)H * t + 31) & ~31ULL);
    out->rkv_w = rkv ? dW : nullptr;
    cudaStream_t st = ctx->stream;
    if (pl.top_cheap) {
        if ((rc = kvc_launch_cheap_q(dK, T, ek, pl.nq_top, out->Q, st))) return rc;
    } else {
        KVC_CUDA(cudaMemcpyAsync(out->Q, hQ, nQ * 4, cudaMemcpyHostToDevice, st));
    }
    if (rkv) {
        out->w.resize(T);
        const kv_compact_reasoning & r = *p.reasoning;
        for (int j = 0; j < T; j++) {
            int ty = r.classifier(j + r.token_offset, r.classifier_data);
            out->w[j] = ty == KV_TOKEN_THINKING ? r.thinking_weight
                                                : (ty == KV_TOKEN_TRANSITION ? r.transition_weight : 1.0f);
        }
        KVC_CUDA(cudaMemcpyAsync(dW, out->w.data(), (size_t)T * 4, cudaMemcpyHostToDevice, st));
    }
    return KVC_OK;
}

// Part 2: the engine over the layer (`io`: inputs still on the host, results
// emitted group by group) and, with `want_metrics`, the quality-metric
// kernels, leaving the triples in out->d_res.
int run_call(kvc_ctx * ctx, const float * dK, const float * dV, int H, int dk, int dv, const kv_compact_params & p,
             dev_out * out, bool want_metrics, kvc_stream_io * io) {
    const kvc_plan & pl = out->plan;
    kvc_layer_job job;
    job.K = dK;
    job.V = dV;
    job.Q = out->Q;
    job.rkv_w = out->rkv_w;
    job.plan = &pl;
    job.io = io;
    job.out.sel = out->sel;
    job.out.beta = out->beta;
    job.out.cv = out->cv;
    job.out.t_total = pl.t_total;
    int rc;
    kvc_phase_ms ph;
    if ((rc = kvc_engine_run(ctx, p, H, dk, dv, &job, 1, &ph, want_metrics))) return rc;
    if (want_metrics) {
        out->pairs = kvc_metric_pairs(H, pl.nq_top);
        void * a9;
        if ((rc = kvc_arena(ctx, 9, ((size_t)out->pairs * 3 + 64) * 4, &a9))) return rc;
        out->d_res = (float *)a9;
        out->h_res.assign((size_t)out->pairs * 3, 0.0f);
        if ((rc = kvc_engine_metrics_launch(ctx, job, H, dk, dv, out->d_res))) return rc;
    }
    return KVC_OK;
}

// Compact one layer whose fp32 K/V are already on the device.
int compact_dev(kvc_ctx * ctx, const float * dK, const float * dV, const float * hQ, int T, int n_q, int H,
                int dk, int dv, const kv_compact_params & p, dev_out * out, bool want_metrics) {
    int rc = kvc_make_plan(T, n_q, hQ == nullptr, H, dk, dv, p, &out->plan);
    if (rc) return rc;
    if ((rc = stage_call(ctx, dK, hQ, T, H, dk, dv, p, out))) return rc;
    return run_call(ctx, dK, dV, H, dk, dv, p, out, want_metrics, nullptr);
}

// Result arrays of a drop-in call, filled group by group: an array holds
// `rows` rows of `row_bytes` bytes copied from `dev` on the d2h stream,
// straight into `host` when it is a page-locked pool block, else into pinned
// staging that is copied over once everything has arrived. An array of
// `count` > 1 parts (one per head, `host_pitch` / `dev_pitch` bytes apart)
// goes in one 2D copy per group: with uploads running in the other
// direction, the copy engines lose much of their throughput to many small
// copies, and one 2D copy per array family keeps a group to five copies.
struct host_outputs {
    struct array {
        void * host; const char * dev; size_t row_bytes;
        int count; size_t host_pitch, dev_pitch;
        char * stage;
    };
    std::vector<array> arrays;
    int rows = 0;
    char * extra = nullptr;   // pinned staging of `extra_bytes` for one more download (metric triples)

    void add(void * host, const void * dev, size_t row_bytes, int count = 1, size_t host_pitch = 0,
             size_t dev_pitch = 0) {
        arrays.push_back({host, (const char *)dev, row_bytes, count, host_pitch, dev_pitch, nullptr});
    }
    size_t bytes_of(const array & x) const {
        return x.count > 1 ? (size_t)x.count * x.host_pitch : (size_t)rows * x.row_bytes;
    }
    // Staging for the arrays that are not page-locked and for the extra
    // download (before anything is queued).
    int prepare(kvc_ctx * ctx, int n_rows, size_t extra_bytes) {
        rows = n_rows;
        size_t need = (extra_bytes + 255) & ~(size_t)255;
        for (const array & x : arrays)
            if (!kvc_is_pinned(x.host)) need += (bytes_of(x) + 255) & ~(size_t)255;
        void * pin;
        int rc;
        if ((rc = kvc_pinned(ctx, need, &pin))) return rc;
        extra = (char *)pin;
        size_t off = (extra_bytes + 255) & ~(size_t)255;
        for (array & x : arrays)
            if (!kvc_is_pinned(x.host)) {
                x.stage = (char *)pin + off;
                off += (bytes_of(x) + 255) & ~(size_t)255;
            }
        return KVC_OK;
    }
    // Copy rows [r0, r1) once stream `st` reaches its current point.
    int emit(kvc_ctx * ctx, int r0, int r1, cudaStream_t st) {
        if (r1 <= r0) return KVC_OK;
        cudaEvent_t e = kvc_sync_event(ctx);
        KVC_CUDA(cudaEventRecord(e, st));
        KVC_CUDA(cudaStreamWaitEvent(ctx->d2h_stream, e, 0));
        for (const array & x : arrays) {
            char * dst = (x.stage ? x.stage : (char *)x.host) + (size_t)r0 * x.row_bytes;
            const char * src = x.dev + (size_t)r0 * x.row_bytes;
            const size_t w = (size_t)(r1 - r0) * x.row_bytes;
            if (x.count > 1)
                KVC_CUDA(cudaMemcpy2DAsync(dst, x.host_pitch, src, x.dev_pitch, w, x.count, cudaMemcpyDeviceToHost,
                                           ctx->d2h_stream));
            else
                KVC_CUDA(cudaMemcpyAsync(dst, src, w, cudaMemcpyDeviceToHost, ctx->d2h_stream));
        }
        kvc_trace(ctx, "d" + std::to_string(r1), ctx->d2h_stream);
        return KVC_OK;
    }
    // The compute stream waits for every queued download (so one kvc_wait
    // covers both).
    int join(kvc_ctx * ctx) {
        cudaEvent_t e = kvc_sync_event(ctx);
        KVC_CUDA(cudaEventRecord(e, ctx->d2h_stream));
        KVC_CUDA(cudaStreamWaitEvent(ctx->stream, e, 0));
        return KVC_OK;
    }
    // After the wait: staged arrays to their destinations.
    void unstage() const {
        std::vector<kvc_copy_piece> pieces;
        for (const array & x : arrays)
            if (x.stage) pieces.push_back({x.host, x.stage, bytes_of(x)});
        if (!pieces.empty()) kvc_parallel_copy(pieces);
    }
};

// Number of upload/compute/download groups for a call moving `in_bytes` of
// inputs over `n_units` chunks: about one group per 32 MB of input, at most
// 8 (KVC_STREAM_GROUPS overrides, for tuning). On one cfg4 layer (218 MB of
// Q8_0 K/V) 5 to 8 groups give 5.5-5.6 ms per call, one group 8.0 ms.
int stream_groups(size_t in_bytes, size_t n_units) {
    long long g = (long long)(in_bytes / ((size_t)32 << 20));
    if (const char * e = getenv("KVC_STREAM_GROUPS")) g = atoll(e);
    g = std::min<long long>(std::max<long long>(g, 1), 8);
    return (int)std::min<long long>(g, (long long)std::max<size_t>(n_units, 1));
}

// Size ratio of consecutive groups: 3/4, so the last groups (whose refit
// and download are left when the uploads end) are the small ones
// (KVC_STREAM_RATIO overrides, for tuning).
double stream_ratio() {
    const char * e = getenv("KVC_STREAM_RATIO");
    double q = e ? atof(e) : 0.75;
    return (q > 0.0 && q <= 4.0) ? q : 0.75;
}

// End of a drop-in call: the compute stream joins the downloads, the metric
// triples come back through the staging, one polled wait, then the staged
// arrays are copied over and the stats finished.
int finish_call(kvc_ctx * ctx, dev_out & d, host_outputs & outs) {
    int rc;
    if ((rc = outs.join(ctx))) return rc;
    const size_t rb = d.h_res.size() * sizeof(float);
    if (d.d_res && rb) KVC_CUDA(cudaMemcpyAsync(outs.extra, d.d_res, rb, cudaMemcpyDeviceToHost, ctx->stream));
    kvc_trace(ctx, "done", ctx->stream);
    if ((rc = kvc_wait(ctx))) return rc;
    kvc_trace_dump(ctx);
    if (d.d_res && rb) memcpy(d.h_res.data(), outs.extra, rb);
    outs.unstage();
    finish_dev(ctx, &d);
    return KVC_OK;
}

// Result arrays of a kv_compact_result for t kept keys, in the reference's
// layout (selected_indices[t], beta[h][t], C_v[h][t*d_v]). The heads of
// beta and of C_v are slices of one block each (t resp. t*d_v floats apart),
// so a group of rows goes back in one 2D copy per family; the *_free
// functions release the blocks.
void alloc_result_arrays(kv_compact_result * r, int t, int H, int dv) {
    const size_t tp = (size_t)std::max(t, 1);
    r->t = t;
    r->n_head_kv = H;
    r->selected_indices = (int *)kvc_hmalloc(tp * sizeof(int));
    r->beta = (float **)malloc((size_t)H * sizeof(float *));
    r->C_v = (float **)malloc((size_t)H * sizeof(float *));
    float * bb = (float *)kvc_hmalloc((size_t)H * tp * sizeof(float));
    float * cb = (float *)kvc_hmalloc((size_t)H * tp * dv * sizeof(float));
    for (int h = 0; h < H; h++) {
        r->beta[h] = bb + (size_t)h * tp;
        r->C_v[h] = cb + (size_t)h * tp * dv;
    }
}

// The same, registered with `outs` for the group-by-group downloads.
void alloc_result(kv_compact_result * r, const dev_out & d, int H, int dv, host_outputs * outs) {
    const int t = d.plan.t_total;
    alloc_result_arrays(r, t, H, dv);
    outs->add(r->selected_indices, d.sel, sizeof(int));
    if (H > 0 && t > 0) {
        outs->add(r->beta[0], d.beta, sizeof(float), H, (size_t)t * sizeof(float), (size_t)t * sizeof(float));
        outs->add(r->C_v[0], d.cv, (size_t)dv * sizeof(float), H, (size_t)t * dv * sizeof(float),
                  (size_t)t * dv * sizeof(float));
    }
}

// Allocate the reference's result arrays and copy the outputs (plus the
// metric triples and any `extra` pieces) back; finishes d's stats.
int fill_result(kvc_ctx * ctx, dev_out & d, int H, int dv, kv_compact_result * r,
                const std::vector<d2h_piece> & extra = {}) {
    const int t = d.plan.t_total;
    alloc_result_arrays(r, t, H, dv);
    std::vector<d2h_piece> v;
    v.push_back({r->selected_indices, d.sel, (size_t)t * 4});
    if (H > 0) {
        v.push_back({r->beta[0], d.beta, (size_t)H * t * 4});
        v.push_back({r->C_v[0], d.cv, (size_t)H * t * dv * 4});
    }
    for (const auto & x : extra) v.push_back(x);
    if (d.d_res) v.push_back({d.h_res.data(), d.d_res, d.h_res.size() * sizeof(float)});
    int rc = gather_to_host(ctx, v);
    if (rc) return rc;
    finish_dev(ctx, &d);
    return KVC_OK;
}

void free_result_arrays(kv_compact_result * r) {
    if (!r) return;
    kvc_hfree(r->selected_indices);
    r->selected_indices = NULL;
    if (r->beta) {
        if (r->n_head_kv > 0) kvc_hfree(r->beta[0]);     // block holding every head
        free(r->beta);
        r->beta = NULL;
    }
    if (r->C_v) {
        if (r->n_head_kv > 0) kvc_hfree(r->C_v[0]);
        free(r->C_v);
        r->C_v = NULL;
    }
    r->t = 0;
    r->n_head_kv = 0;
}

kv_compact_params defaults() {
    kv_compact_params p;
    memset(&p, 0, sizeof(p));
    p.target_ratio = 0.5f;
    p.target_count = 0;
    p.use_sensitivity = 0;
    p.ridge = 1e-6f;
    p.nnls_max_iter = 200;
    p.refine_rounds = 0;
    p.use_diversity = 0;
    p.diversity_strength = 0.5f;
    p.n_shared_prefix = 0;
    p.use_cheap_qref = 0;
    p.skip_beta = 1;
    p.score_method = 1;
    p.use_omp = 0;
    p.omp_k_choice = 1;
    p.omp_refit_interval = 1;
    p.nnls_method = 1;
    p.nnls_pgd_iters = 0;
    p.chunk_size = 0;
    p.n_threads = 0;
    p.layer_filter = NULL;
    p.layer_filter_data = NULL;
    p.reasoning = NULL;
    return p;
}

}  // namespace

extern "C" {

KVC_EXPORT kv_compact_params kv_compact_params_default(void) { return defaults(); }

KVC_EXPORT int kv_compact(const float * K_all, const float * V_all, const float * Q_ref_all, int T, int n_q, int n_head_kv,
               int d_k, int d_v, const kv_compact_params * params, kv_compact_result * result) {
    if (!K_all || !V_all || !result) return KVC_ERR_NULL;
    if (T <= 0 || n_head_kv <= 0 || d_k <= 0 || d_v <= 0) return KVC_ERR_DIMS;
    const auto t0 = clk::now();
    kv_compact_params p = params ? *params : defaults();
    if (!(p.use_cheap_qref || !Q_ref_all) && n_q <= 0) return KVC_ERR_DIMS;
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    io_stream_guard cg{ctx};
    const int H = n_head_kv, ek = H * d_k, ev = H * d_v;
    const float * hQ = (p.use_cheap_qref || !Q_ref_all) ? nullptr : Q_ref_all;
    dev_out d;
    if ((rc = kvc_make_plan(T, n_q, hQ == nullptr, H, d_k, d_v, p, &d.plan))) return rc;
    kvc_trace(ctx, "call", ctx->stream);
    void * a;
    if ((rc = kvc_arena(ctx, SLOT_KV_A, ((size_t)T * ek + (size_t)T * ev + 64) * 4, &a))) return rc;
    float * dK = (float *)a;
    float * dV = dK + (((size_t)T * ek + 31) & ~31ULL);
    kvc_stream_io io;
    io.k = {(const uint8_t *)K_all, (uint8_t *)dK, (size_t)ek * 4, -1};
    io.v = {(const uint8_t *)V_all, (uint8_t *)dV, (size_t)ev * 4, -1};
    io.max_groups = stream_groups((size_t)T * (ek + ev) * 4, d.plan.units.size());
    io.size_ratio = stream_ratio();
    if (d.plan.top_cheap) {        // the top-level queries sample all of K: it goes up first, in full
        KVC_CUDA(cudaMemcpyAsync(dK, K_all, (size_t)T * ek * 4, cudaMemcpyHostToDevice, ctx->stream));
        io.k_resident = true;
    }
    if ((rc = stage_call(ctx, dK, hQ, T, H, d_k, d_v, p, &d))) return rc;
    host_outputs outs;
    alloc_result(result, d, H, d_v, &outs);
    auto fail = [&](int code) {
        for (auto gs : ctx->group_stream) cudaStreamSynchronize(gs);
        cudaStreamSynchronize(ctx->d2h_stream);
        free_result_arrays(result);
        return code;
    };
    if ((rc = outs.prepare(ctx, d.plan.t_total, (size_t)kvc_metric_pairs(H, d.plan.nq_top) * 3 * sizeof(float))))
        return fail(rc);
    io.emit = [&](int r0, int r1, cudaStream_t s) { return outs.emit(ctx, r0, r1, s); };
    if ((rc = run_call(ctx, dK, dV, H, d_k, d_v, p, &d, true, &io))) return fail(rc);
    if ((rc = finish_call(ctx, d, outs))) return fail(rc);
    result->stats = d.stats;
    result->stats.elapsed_ms = ms_since(t0);
    kvc_resolve_timers(ctx);
    return KVC_OK;
}

KVC_EXPORT void kv_compact_result_free(kv_compact_result * result) { free_result_arrays(result); }

KVC_EXPORT int kv_compact_multi_round(const float * K_all, const float * V_all, const float * Q_ref_all, int T, int n_q,
                           int n_head_kv, int d_k, int d_v, const kv_compact_params * params, int n_rounds,
                           kv_compact_result * result, kv_compact_stats * per_round_stats) {
    if (!K_all || !V_all || !result) return KVC_ERR_NULL;
    if (T <= 0 || n_head_kv <= 0 || d_k <= 0 || d_v <= 0) return KVC_ERR_DIMS;
    if (n_rounds < 1) return KVC_ERR_ROUNDS;
    kv_compact_params p = params ? *params : defaults();
    if (!Q_ref_all && !p.use_cheap_qref) return KVC_ERR_NULL;
    if (Q_ref_all && n_q <= 0 && !p.use_cheap_qref) return KVC_ERR_DIMS;
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    const int H = n_head_kv, ek = H * d_k, ev = H * d_v;
    cudaStream_t st = ctx->stream;

    // original K/V stay resident for the final metrics (slot KV_A); rounds
    // ping-pong between two further buffers inside slot KV_B.
    void * a;
    size_t nk = ((size_t)T * ek + 31) & ~31ULL, nv = ((size_t)T * ev + 31) & ~31ULL;
    if ((rc = kvc_arena(ctx, SLOT_KV_A, (nk + nv) * 4, &a))) return rc;
    float * oK = (float *)a;
    float * oV = oK + nk;
    KVC_CUDA(cudaMemcpyAsync(oK, K_all, (size_t)T * ek * 4, cudaMemcpyHostToDevice, st));
    KVC_CUDA(cudaMemcpyAsync(oV, V_all, (size_t)T * ev * 4, cudaMemcpyHostToDevice, st));
    void * b;
    if ((rc = kvc_arena(ctx, SLOT_KV_B, 2 * (nk + nv) * 4 + 1024, &b))) return rc;
    float * pK[2] = {(float *)b, (float *)b + nk + nv};
    float * pV[2] = {pK[0] + nk, pK[1] + nk};
    KVC_CUDA(cudaMemcpyAsync(pK[0], oK, (size_t)T * ek * 4, cudaMemcpyDeviceToDevice, st));
    KVC_CUDA(cudaMemcpyAsync(pV[0], oV, (size_t)T * ev * 4, cudaMemcpyDeviceToDevice, st));

    // queries of the final metrics (src/kv-compact-api.cpp:1011-1023)
    int nq_mr = n_q;
    std::vector<float> qmr;
    const bool cheap = p.use_cheap_qref || !Q_ref_all;
    if (cheap) {
        nq_mr = T / 2;
        if (nq_mr > 64) nq_mr = 64;
        if (nq_mr < 4) nq_mr = 4;
        if (nq_mr > T) nq_mr = T;
    }
    std::vector<int> orig(T);
    for (int i = 0; i < T; i++) orig[i] = i;
    int cur_T = T, cur = 0;
    dev_out d;
    for (int r = 0; r < n_rounds; r++) {
        int nq_r = nq_mr < cur_T ? nq_mr : cur_T;
        d = dev_out();
        if ((rc = compact_dev(ctx, pK[cur], pV[cur], cheap ? nullptr : Q_ref_all, cur_T, nq_r, H, d_k, d_v, p,
                              &d, true)))
            return rc;
        const int nT = d.plan.t_total;
        std::vector<int> sel(nT);
        if ((rc = gather_to_host(ctx, {{sel.data(), d.sel, (size_t)nT * 4},
                                       {d.h_res.data(), d.d_res, d.h_res.size() * sizeof(float)}})))
            return rc;
        finish_dev(ctx, &d);
        if (per_round_stats) per_round_stats[r] = d.stats;
        std::vector<int> no(nT);
        for (int j = 0; j < nT; j++) no[j] = orig[sel[j]];
        if (r == n_rounds - 1) {
            const kv_compact_stats keep = d.stats;     // already complete
            d.d_res = nullptr;
            if ((rc = fill_result(ctx, d, H, d_v, result))) return rc;
            memcpy(result->selected_indices, no.data(), (size_t)nT * sizeof(int));
            result->stats = keep;
        } else {
            const int nxt = cur ^ 1;
            if ((rc = kvc_launch_gather_rows(pK[cur], ek, d.sel, nT, ek, pK[nxt], ek, st))) return rc;
            if ((rc = kvc_launch_encode_heads(d.cv, H, nT, nT, d_v, 0, (uint8_t *)pV[nxt], (size_t)ev * 4, st))) return rc;
            cur = nxt;
        }
        orig.swap(no);
        cur_T = nT;
    }
    // final metrics against the original cache (src/kv-compact-api.cpp:1105-1108)
    {
        kvc_plan mp;
        mp.T = T;
        mp.nq_top = nq_mr;
        mp.t_total = result->t;
        void * c;
        size_t need = ((size_t)nq_mr * ek + (size_t)result->t + (size_t)H * result->t +
                       (size_t)H * result->t * d_v + 128) * 4;
        if ((rc = kvc_arena(ctx, SLOT_QIO, need, &c))) return rc;
        float * mQ = (float *)c;
        int * msel = (int *)(mQ + (((size_t)nq_mr * ek + 31) & ~31ULL));
        float * mbeta = (float *)(msel + ((result->t + 31) & ~31));
        float * mcv = mbeta + (((size_t)H * result->t + 31) & ~31ULL);
        if (cheap) {
            if ((rc = kvc_launch_cheap_q(oK, T, ek, nq_mr, mQ, st))) return rc;
        } else {
            KVC_CUDA(cudaMemcpyAsync(mQ, Q_ref_all, (size_t)nq_mr * ek * 4, cudaMemcpyHostToDevice, st));
        }
        KVC_CUDA(cudaMemcpyAsync(msel, result->selected_indices, (size_t)result->t * 4, cudaMemcpyHostToDevice, st));
        KVC_CUDA(cudaMemcpyAsync(mbeta, d.beta, (size_t)H * result->t * 4, cudaMemcpyDeviceToDevice, st));
        KVC_CUDA(cudaMemcpyAsync(mcv, d.cv, (size_t)H * result->t * d_v * 4, cudaMemcpyDeviceToDevice, st));
        kvc_layer_job job;
        job.K = oK;
        job.V = oV;
        job.Q = mQ;
        job.plan = &mp;
        job.out.sel = msel;
        job.out.beta = mbeta;
        job.out.cv = mcv;
        job.out.t_total = result->t;
        kv_compact_stats s = result->stats;
        if ((rc = kvc_engine_metrics(ctx, job, H, d_k, d_v, &s))) return rc;
        result->stats.avg_cosine_sim = s.avg_cosine_sim;
        result->stats.avg_mse = s.avg_mse;
        result->stats.avg_agreement = s.avg_agreement;
    }
    kvc_resolve_timers(ctx);
    return KVC_OK;
}

KVC_EXPORT int kv_quant_row_elements(int type, size_t row_bytes) { return kvc_row_elements(type, row_bytes); }
KVC_EXPORT size_t kv_quant_row_bytes(int type, int n_elements) { return kvc_row_bytes(type, n_elements); }

KVC_EXPORT int kv_dequantize_row(const uint8_t * src, int type, size_t row_bytes, float * dst, int max_elements) {
    int n = kvc_row_elements(type, row_bytes);
    if (n > max_elements) n = max_elements;
    kvc_host_decode_row(src, type, dst, (size_t)n);
    return n;
}

KVC_EXPORT size_t kv_quantize_row(const float * src, int type, int n_elements, uint8_t * dst) {
    return kvc_host_encode_row(src, type, dst, n_elements);
}

KVC_EXPORT int kv_compact_quantized(const uint8_t * K_quant, const uint8_t * V_quant, const float * Q_ref_all, int k_type,
                         int v_type, size_t k_row_bytes, size_t v_row_bytes, int T, int n_q, int n_head_kv,
                         int d_k, int d_v, const kv_compact_params * params, kv_compact_quant_result * result) {
    if (!K_quant || !V_quant || !result) return KVC_ERR_NULL;
    if (T <= 0 || n_head_kv <= 0 || d_k <= 0 || d_v <= 0) return KVC_ERR_DIMS;
    const int H = n_head_kv, ek = H * d_k, ev = H * d_v;
    if (kvc_row_elements(k_type, k_row_bytes) != ek || kvc_row_elements(v_type, v_row_bytes) != ev)
        return KVC_ERR_ROWSIZE;
    const auto t0 = clk::now();
    kv_compact_params p = params ? *params : defaults();
    if (!(p.use_cheap_qref || !Q_ref_all) && n_q <= 0) return KVC_ERR_DIMS;
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    io_stream_guard cg{ctx};
    cudaStream_t st = ctx->stream;
    const float * hQ = (p.use_cheap_qref || !Q_ref_all) ? nullptr : Q_ref_all;
    dev_out d;
    if ((rc = kvc_make_plan(T, n_q, hQ == nullptr, H, d_k, d_v, p, &d.plan))) return rc;
    kvc_trace(ctx, "call", ctx->stream);
    const int t = d.plan.t_total;
    size_t nk = ((size_t)T * ek + 31) & ~31ULL, nv = ((size_t)T * ev + 31) & ~31ULL;
    size_t qk = ((size_t)T * k_row_bytes + 255) & ~255ULL, qv = ((size_t)T * v_row_bytes + 255) & ~255ULL;
    void * a;
    if ((rc = kvc_arena(ctx, SLOT_KV_A, (nk + nv) * 4 + qk + qv, &a))) return rc;
    float * dK = (float *)a;
    float * dV = dK + nk;
    uint8_t * qK = (uint8_t *)(dV + nv);
    uint8_t * qV = qK + qk;
    void * b;
    size_t ob = (((size_t)t * k_row_bytes + 255) & ~255ULL) + (size_t)t * v_row_bytes + 256;
    if ((rc = kvc_arena(ctx, SLOT_QIO, ob, &b))) return rc;
    uint8_t * oK = (uint8_t *)b;
    uint8_t * oV = oK + (((size_t)t * k_row_bytes + 255) & ~255ULL);
    kvc_stream_io io;
    io.k = {K_quant, qK, k_row_bytes, k_type};
    io.v = {V_quant, qV, v_row_bytes, v_type};
    io.max_groups = stream_groups((size_t)T * (k_row_bytes + v_row_bytes), d.plan.units.size());
    io.size_ratio = stream_ratio();
    if (d.plan.top_cheap) {        // the top-level queries sample all of K: it goes up first, in full
        KVC_CUDA(cudaMemcpyAsync(qK, K_quant, (size_t)T * k_row_bytes, cudaMemcpyHostToDevice, st));
        kvc_stage_timer tm(ctx, KVC_ST_DECODE, 1);
        if ((rc = kvc_launch_decode(qK, k_row_bytes, k_type, dK, T, ek, st))) return rc;
        io.k_resident = true;
    }
    // K stays in its block format when nothing needs it decoded (tensor-core
    // scoring, K_out re-encoded from the stored rows)
    io.k_blocks_only = !io.k_resident && kvc_k_blocks_only(p, d.plan, k_type, k_row_bytes, qK, H, d_k);
    if ((rc = stage_call(ctx, dK, hQ, T, H, d_k, d_v, p, &d))) return rc;
    memset(result, 0, sizeof(*result));
    host_outputs outs;
    alloc_result(&result->base, d, H, d_v, &outs);
    result->k_type = k_type;
    result->v_type = v_type;
    result->k_row_bytes = k_row_bytes;
    result->v_row_bytes = v_row_bytes;
    result->K_out = (uint8_t *)kvc_hmalloc(std::max<size_t>((size_t)t * k_row_bytes, 1));
    result->V_out = (uint8_t *)kvc_hmalloc(std::max<size_t>((size_t)t * v_row_bytes, 1));
    outs.add(result->K_out, oK, k_row_bytes);
    outs.add(result->V_out, oV, v_row_bytes);
    auto fail = [&](int code) {
        for (auto gs : ctx->group_stream) cudaStreamSynchronize(gs);
        cudaStreamSynchronize(ctx->d2h_stream);
        free_result_arrays(&result->base);
        kvc_hfree(result->K_out);
        result->K_out = NULL;
        kvc_hfree(result->V_out);
        result->V_out = NULL;
        return code;
    };
    if ((rc = outs.prepare(ctx, t, (size_t)kvc_metric_pairs(H, d.plan.nq_top) * 3 * sizeof(float))))
        return fail(rc);
    // kept rows [r0, r1): K_out re-encodes the original (dequantised) rows at
    // the selected positions, V_out the refitted values C_v; then both go
    // back with the group's indices, beta and C_v
    io.emit = [&](int r0, int r1, cudaStream_t s) {
        int e;
        {
            kvc_stage_timer tm(ctx, KVC_ST_REQUANT, 2, s);
            e = io.k_blocks_only
                    ? kvc_launch_transcode_gather(qK, k_row_bytes, d.sel + r0, r1 - r0, ek, k_type,
                                                  oK + (size_t)r0 * k_row_bytes, k_row_bytes, s)
                    : kvc_launch_encode_gather(dK, (size_t)ek, d.sel + r0, r1 - r0, ek, k_type,
                                               oK + (size_t)r0 * k_row_bytes, k_row_bytes, s);
            if (e) return e;
            if ((e = kvc_launch_encode_heads(d.cv + (size_t)r0 * d_v, H, t, r1 - r0, d_v, v_type,
                                             oV + (size_t)r0 * v_row_bytes, v_row_bytes, s)))
                return e;
        }
        return outs.emit(ctx, r0, r1, s);
    };
    if ((rc = run_call(ctx, dK, dV, H, d_k, d_v, p, &d, true, &io))) return fail(rc);
    if ((rc = finish_call(ctx, d, outs))) return fail(rc);
    result->base.stats = d.stats;
    result->base.stats.elapsed_ms = ms_since(t0);
    kvc_resolve_timers(ctx);
    return KVC_OK;
}

KVC_EXPORT void kv_compact_quant_result_free(kv_compact_quant_result * result) {
    if (!result) return;
    free_result_arrays(&result->base);
    kvc_hfree(result->K_out);
    result->K_out = NULL;
    kvc_hfree(result->V_out);
    result->V_out = NULL;
}

}  // extern "C"
