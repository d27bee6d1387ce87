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
// would let the caller reuse its input buffers too early: every return path
// waits for that stream (a no-op once the engine has consumed the upload).
struct copy_stream_guard {
    kvc_ctx * ctx;
    ~copy_stream_guard() { cudaStreamSynchronize(ctx->copy_stream); }
};
enum { SLOT_KV_A = 3, SLOT_IO = 5, SLOT_KV_B = 6, SLOT_QIO = 7 };

struct dev_out {
    kvc_plan plan;
    int * sel = nullptr;
    float * beta = nullptr;
    float * cv = nullptr;
    float * Q = nullptr;      // top-level queries on the device
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

// Compact one layer whose fp32 K/V are already on the device.
// V may still be on the host (`v_host`, `v_bytes`): the engine uploads it to
// `v_dev` on the copy stream while the scoring runs, and decodes it into dV
// when `v_quant` (== v_dev) is given.
int compact_dev(kvc_ctx * ctx, const float * dK, const float * dV, const float * hQ, int T, int n_q, int H,
                int dk, int dv, const kv_compact_params & p, dev_out * out, bool want_metrics,
                const void * v_host = nullptr, void * v_dev = nullptr, size_t v_bytes = 0,
                const uint8_t * v_quant = nullptr, size_t v_rb = 0, int v_type = 0) {
    int rc = kvc_make_plan(T, n_q, hQ == nullptr, H, dk, dv, p, &out->plan);
    if (rc) return rc;
    const kvc_plan & pl = out->plan;
    const int ek = H * dk;
    const int t = pl.t_total;
    const bool rkv = p.reasoning && p.reasoning->classifier;
    // io arena: Q | rkv weights | sel | beta | cv
    size_t nQ = (size_t)pl.nq_top * ek, nW = rkv ? (size_t)T : 0;
    size_t bytes = (nQ + nW + (size_t)t + (size_t)H * t + (size_t)H * t * dv + 64) * 4;
    void * a;
    if ((rc = kvc_arena(ctx, SLOT_IO, bytes, &a))) return rc;
    float * base = (float *)a;
    float * dQ = base;
    float * dW = dQ + ((nQ + 31) & ~31ULL);
    int * dsel = (int *)(dW + ((nW + 31) & ~31ULL));
    float * dbeta = (float *)(dsel + ((t + 31) & ~31));
    float * dcv = dbeta + (((size_t)H * t + 31) & ~31ULL);
    cudaStream_t st = ctx->stream;
    if (pl.top_cheap) {
        if ((rc = kvc_launch_cheap_q(dK, T, ek, pl.nq_top, dQ, st))) return rc;
    } else {
        KVC_CUDA(cudaMemcpyAsync(dQ, hQ, nQ * 4, cudaMemcpyHostToDevice, st));
    }
    std::vector<float> w;
    if (rkv) {
        w.resize(T);
        const kv_compact_reasoning & r = *p.reasoning;
        for (int j = 0; j < T; j++) {
            int ty = r.classifier(j + r.token_offset, r.classifier_data);
            w[j] = ty == KV_TOKEN_THINKING ? r.thinking_weight : (ty == KV_TOKEN_TRANSITION ? r.transition_weight : 1.0f);
        }
        KVC_CUDA(cudaMemcpyAsync(dW, w.data(), (size_t)T * 4, cudaMemcpyHostToDevice, st));
    }
    kvc_layer_job job;
    job.K = dK;
    job.V = dV;
    job.Q = dQ;
    job.rkv_w = rkv ? dW : nullptr;
    job.plan = &pl;
    job.v_host = v_host;
    job.v_dev = v_dev;
    job.v_bytes = v_bytes;
    job.v_quant = v_quant;
    job.v_row_bytes = v_rb;
    job.v_type = v_type;
    job.out.sel = dsel;
    job.out.beta = dbeta;
    job.out.cv = dcv;
    job.out.t_total = t;
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
    out->sel = dsel;
    out->beta = dbeta;
    out->cv = dcv;
    out->Q = dQ;
    return KVC_OK;
}

// Allocate the reference's result arrays and copy the outputs (plus the
// metric triples and any `extra` pieces) back; finishes d's stats.
int fill_result(kvc_ctx * ctx, dev_out & d, int H, int dv, kv_compact_result * r,
                const std::vector<d2h_piece> & extra = {}) {
    const int t = d.plan.t_total;
    r->t = t;
    r->n_head_kv = H;
    r->selected_indices = (int *)kvc_hmalloc((size_t)std::max(t, 1) * sizeof(int));
    r->beta = (float **)malloc((size_t)H * sizeof(float *));
    r->C_v = (float **)malloc((size_t)H * sizeof(float *));
    for (int h = 0; h < H; h++) {
        r->beta[h] = (float *)kvc_hmalloc((size_t)std::max(t, 1) * sizeof(float));
        r->C_v[h] = (float *)kvc_hmalloc((size_t)std::max(t, 1) * dv * sizeof(float));
    }
    std::vector<d2h_piece> v;
    v.push_back({r->selected_indices, d.sel, (size_t)t * 4});
    for (int h = 0; h < H; h++) {
        v.push_back({r->beta[h], d.beta + (size_t)h * t, (size_t)t * 4});
        v.push_back({r->C_v[h], d.cv + (size_t)h * t * dv, (size_t)t * dv * 4});
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
        for (int h = 0; h < r->n_head_kv; h++) kvc_hfree(r->beta[h]);
        free(r->beta);
        r->beta = NULL;
    }
    if (r->C_v) {
        for (int h = 0; h < r->n_head_kv; h++) kvc_hfree(r->C_v[h]);
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
    copy_stream_guard cg{ctx};
    const int H = n_head_kv, ek = H * d_k, ev = H * d_v;
    void * a;
    if ((rc = kvc_arena(ctx, SLOT_KV_A, ((size_t)T * ek + (size_t)T * ev + 64) * 4, &a))) return rc;
    float * dK = (float *)a;
    float * dV = dK + (((size_t)T * ek + 31) & ~31ULL);
    // K now; V is uploaded by the engine on the copy stream, overlapping the scoring
    KVC_CUDA(cudaMemcpyAsync(dK, K_all, (size_t)T * ek * 4, cudaMemcpyHostToDevice, ctx->stream));
    const float * hQ = (p.use_cheap_qref || !Q_ref_all) ? nullptr : Q_ref_all;
    dev_out d;
    if ((rc = compact_dev(ctx, dK, dV, hQ, T, n_q, H, d_k, d_v, p, &d, true, V_all, dV, (size_t)T * ev * 4)))
        return rc;
    if ((rc = fill_result(ctx, d, H, d_v, result))) return rc;
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
            if ((rc = kvc_launch_encode_heads(d.cv, H, nT, d_v, 0, (uint8_t *)pV[nxt], (size_t)ev * 4, st))) return rc;
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
    copy_stream_guard cg{ctx};
    cudaStream_t st = ctx->stream;
    size_t nk = ((size_t)T * ek + 31) & ~31ULL, nv = ((size_t)T * ev + 31) & ~31ULL;
    size_t qk = ((size_t)T * k_row_bytes + 255) & ~255ULL, qv = ((size_t)T * v_row_bytes + 255) & ~255ULL;
    void * a;
    if ((rc = kvc_arena(ctx, SLOT_KV_A, (nk + nv) * 4 + qk + qv, &a))) return rc;
    float * dK = (float *)a;
    float * dV = dK + nk;
    uint8_t * qK = (uint8_t *)(dV + nv);
    uint8_t * qV = qK + qk;
    // K now; the engine uploads V on the copy stream once its own small
    // uploads are queued, and decodes it just before the first stage that
    // reads it (the scoring overlaps the upload)
    KVC_CUDA(cudaMemcpyAsync(qK, K_quant, (size_t)T * k_row_bytes, cudaMemcpyHostToDevice, st));
    {
        kvc_stage_timer tm(ctx, KVC_ST_DECODE, 1);
        if ((rc = kvc_launch_decode(qK, k_row_bytes, k_type, dK, T, ek, st))) return rc;
    }
    memset(&result->base, 0, sizeof(result->base));
    const float * hQ = (p.use_cheap_qref || !Q_ref_all) ? nullptr : Q_ref_all;
    dev_out d;
    if ((rc = compact_dev(ctx, dK, dV, hQ, T, n_q, H, d_k, d_v, p, &d, true, V_quant, qV,
                          (size_t)T * v_row_bytes, qV, v_row_bytes, v_type)))
        return rc;
    const int t = d.plan.t_total;
    void * b;
    size_t ob = (((size_t)t * k_row_bytes + 255) & ~255ULL) + (size_t)t * v_row_bytes + 256;
    if ((rc = kvc_arena(ctx, SLOT_QIO, ob, &b))) return rc;
    uint8_t * oK = (uint8_t *)b;
    uint8_t * oV = oK + (((size_t)t * k_row_bytes + 255) & ~255ULL);
    {
        kvc_stage_timer tm(ctx, KVC_ST_REQUANT, 2);
        if ((rc = kvc_launch_encode_gather(dK, (size_t)ek, d.sel, t, ek, k_type, oK, k_row_bytes, st))) return rc;
        if ((rc = kvc_launch_encode_heads(d.cv, H, t, d_v, v_type, oV, v_row_bytes, st))) return rc;
    }
    result->k_type = k_type;
    result->v_type = v_type;
    result->k_row_bytes = k_row_bytes;
    result->v_row_bytes = v_row_bytes;
    result->K_out = (uint8_t *)kvc_hmalloc(std::max<size_t>((size_t)t * k_row_bytes, 1));
    result->V_out = (uint8_t *)kvc_hmalloc(std::max<size_t>((size_t)t * v_row_bytes, 1));
    if ((rc = fill_result(ctx, d, H, d_v, &result->base,
                          {{result->K_out, oK, (size_t)t * k_row_bytes}, {result->V_out, oV, (size_t)t * v_row_bytes}})))
        return rc;
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
