// batched.cu — whole-model, device-resident compaction (include/kvc-batched.h).
//
// All filtered layers are decoded to fp32 once, planned, and handed to the
// engine as one job list, so every pipeline stage is a single launch over
// all (layer, chunk) units of the model.
#include <algorithm>
#include <vector>

#include "../../include/kvc-batched.h"
#include "engine.h"

namespace {
enum { SLOT_BATCH_KV = 3, SLOT_BATCH_IO = 5 };

bool layer_on(const kvc_model_desc * m, const kv_compact_params & p, int l) {
    if (!p.layer_filter) return true;
    return p.layer_filter(l, m->n_layers, p.layer_filter_data) != 0;
}

int check(const kvc_model_desc * m, const kvc_layer_desc * L) {
    if (!m || !L) return KVC_ERR_NULL;
    if (m->T <= 0 || m->n_head_kv <= 0 || m->d_k <= 0 || m->d_v <= 0 || m->n_layers <= 0) return KVC_ERR_DIMS;
    if (kvc_row_elements(m->k_type, m->k_row_bytes) != m->n_head_kv * m->d_k ||
        kvc_row_elements(m->v_type, m->v_row_bytes) != m->n_head_kv * m->d_v)
        return KVC_ERR_ROWSIZE;
    return KVC_OK;
}

// Cache positions of layer l (its own n_tokens, else the model's T).
int layer_T(const kvc_model_desc * m, const kvc_layer_desc & Ld) {
    return Ld.n_tokens > 0 ? Ld.n_tokens : m->T;
}

kv_compact_params params_or_default(const kv_compact_params * p) {
    return p ? *p : kv_compact_params_default();
}
}  // namespace

extern "C" {

KVC_EXPORT uint64_t kvc_launch_count(void) {
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    return ctx ? ctx->launches : 0;
}

KVC_EXPORT int kvc_profile(int enable, double * stage_ms, uint64_t * stage_launches, int n) {
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    kvc_resolve_timers(ctx);
    for (int i = 0; i < n && i < KVC_N_STAGES; i++) {
        if (stage_ms) stage_ms[i] = ctx->stage_ms[i];
        if (stage_launches) stage_launches[i] = ctx->stage_launches[i];
    }
    for (int i = 0; i < KVC_N_STAGES; i++) { ctx->stage_ms[i] = 0.0; ctx->stage_launches[i] = 0; }
    ctx->profiling = enable;
    return KVC_N_STAGES;
}

KVC_EXPORT int kvc_plan_layers(const kvc_model_desc * m, const kvc_layer_desc * L, const kv_compact_params * params,
                    int * t_out) {
    int rc = check(m, L);
    if (rc) return rc;
    if (!t_out) return KVC_ERR_NULL;
    kv_compact_params p = params_or_default(params);
    for (int l = 0; l < m->n_layers; l++) {
        t_out[l] = 0;
        if (!layer_on(m, p, l)) continue;
        const bool qn = p.use_cheap_qref || !L[l].Q_ref;
        if (!L[l].K || !L[l].V) return KVC_ERR_NULL;
        if (L[l].n_tokens < 0) return KVC_ERR_DIMS;
        kvc_plan pl;
        if ((rc = kvc_make_plan(layer_T(m, L[l]), L[l].n_q, qn, m->n_head_kv, m->d_k, m->d_v, p, &pl))) return rc;
        t_out[l] = pl.t_total;
    }
    return KVC_OK;
}

KVC_EXPORT int kvc_compact_layers_dev(const kvc_model_desc * m, const kvc_layer_desc * L, const kv_compact_params * params,
                           kvc_layer_result * R, int want_stats) {
    int rc = check(m, L);
    if (rc) return rc;
    if (!R) return KVC_ERR_NULL;
    kv_compact_params p = params_or_default(params);
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaStream_t st = ctx->stream;
    const int H = m->n_head_kv, dk = m->d_k, dv = m->d_v, T = m->T;
    const int ek = H * dk, ev = H * dv;
    const bool rkv = p.reasoning && p.reasoning->classifier;

    std::vector<int> on;
    for (int l = 0; l < m->n_layers; l++) {
        R[l].t = 0;
        if (layer_on(m, p, l)) on.push_back(l);
    }
    const int n = (int)on.size();
    if (n == 0) return KVC_OK;
    std::vector<kvc_plan> plans(n);
    for (int i = 0; i < n; i++) {
        const int l = on[i];
        if (!L[l].K || !L[l].V) return KVC_ERR_NULL;
        if (L[l].n_tokens < 0 || (rkv && layer_T(m, L[l]) != T)) return KVC_ERR_DIMS;
        const bool qn = p.use_cheap_qref || !L[l].Q_ref;
        if ((rc = kvc_make_plan(layer_T(m, L[l]), L[l].n_q, qn, H, dk, dv, p, &plans[i]))) return rc;
    }
    // fp32 caches of every filtered layer (each T_l rows), plus generated
    // cheap queries and R-KV weights
    std::vector<size_t> kv_off(n + 1, 0);
    for (int i = 0; i < n; i++) {
        const size_t Tl = (size_t)layer_T(m, L[on[i]]);
        kv_off[i + 1] = kv_off[i] + ((Tl * ek + 31) & ~31ULL) + ((Tl * ev + 31) & ~31ULL);
    }
    void * a;
    if ((rc = kvc_arena(ctx, SLOT_BATCH_KV, kv_off[n] * 4, &a))) return rc;
    float * F = (float *)a;
    size_t io = 0;
    for (int i = 0; i < n; i++) if (plans[i].top_cheap) io += (((size_t)plans[i].nq_top * ek) + 31) & ~31ULL;
    if (rkv) io += (size_t)T + 32;
    void * b = nullptr;
    if ((rc = kvc_arena(ctx, SLOT_BATCH_IO, io * 4 + 256, &b))) return rc;
    float * io_p = (float *)b;
    float * dW = nullptr;
    if (rkv) {
        std::vector<float> w(T);
        const kv_compact_reasoning & r = *p.reasoning;
        for (int j = 0; j < T; j++) {
            int ty = r.classifier(j + r.token_offset, r.classifier_data);
            w[j] = ty == KV_TOKEN_THINKING ? r.thinking_weight : (ty == KV_TOKEN_TRANSITION ? r.transition_weight : 1.0f);
        }
        dW = io_p;
        io_p += ((size_t)T + 31) & ~31ULL;
        KVC_CUDA(cudaMemcpyAsync(dW, w.data(), (size_t)T * 4, cudaMemcpyHostToDevice, st));
    }
    // K is decoded to fp32 unless every layer reads it only in its block
    // format (then K_out is re-encoded from the stored rows)
    bool k_blocks = true;
    for (int i = 0; i < n && k_blocks; i++)
        k_blocks = kvc_k_blocks_only(p, plans[i], m->k_type, m->k_row_bytes, L[on[i]].K, H, dk);
    std::vector<kvc_layer_job> jobs(n);
    for (int i = 0; i < n; i++) {
        const int l = on[i], Tl = layer_T(m, L[l]);
        float * dK = F + kv_off[i];
        float * dV = dK + (((size_t)Tl * ek + 31) & ~31ULL);
        if (!k_blocks) {
            kvc_stage_timer tm(ctx, KVC_ST_DECODE, 1);
            if ((rc = kvc_launch_decode((const uint8_t *)L[l].K, m->k_row_bytes, m->k_type, dK, Tl, ek, st))) return rc;
        }
        kvc_layer_job & J = jobs[i];
        J.K = dK;
        J.Kq = (const uint8_t *)L[l].K;     // scored from its block bytes where the format allows
        J.k_row_bytes = m->k_row_bytes;
        J.k_type = m->k_type;
        J.V = dV;                  // decoded by the engine unless it reads V in its block format
        J.Vq = (const uint8_t *)L[l].V;
        J.v_row_bytes = m->v_row_bytes;
        J.v_type = m->v_type;
        J.v_decoded = false;
        if (plans[i].top_cheap) {
            float * q = io_p;
            io_p += (((size_t)plans[i].nq_top * ek) + 31) & ~31ULL;
            if ((rc = kvc_launch_cheap_q(dK, Tl, ek, plans[i].nq_top, q, st))) return rc;
            ctx->launches += 1;
            J.Q = q;
        } else {
            J.Q = L[l].Q_ref;
        }
        J.rkv_w = dW;
        J.plan = &plans[i];
        if (!R[l].selected_indices || !R[l].beta || !R[l].C_v) return KVC_ERR_NULL;
        J.out.sel = R[l].selected_indices;
        J.out.beta = R[l].beta;
        J.out.cv = R[l].C_v;
        J.out.t_total = plans[i].t_total;
    }
    kvc_phase_ms ph;
    if ((rc = kvc_engine_run(ctx, p, H, dk, dv, jobs.data(), n, want_stats ? &ph : nullptr, want_stats != 0)))
        return rc;
    // requantisation and metric kernels of every layer, then one wait
    std::vector<int> pair_off(n + 1, 0);
    for (int i = 0; i < n; i++) pair_off[i + 1] = pair_off[i] + (want_stats ? kvc_metric_pairs(H, plans[i].nq_top) : 0);
    float * d_res = nullptr;
    if (want_stats) {
        void * a9;
        if ((rc = kvc_arena(ctx, 9, ((size_t)pair_off[n] * 3 + 64) * 4, &a9))) return rc;
        d_res = (float *)a9;
    }
    std::vector<const float *> m_parts;
    std::vector<int> m_chunks;
    std::vector<float *> m_res;
    // requantisation of every layer in one launch per codec where the
    // layers allow it (else per layer below)
    bool rq_done = false;
    {
        std::vector<const uint8_t *> ks(n);
        std::vector<const int *> sl(n);
        std::vector<int> ts(n);
        std::vector<uint8_t *> kd(n), vd(n);
        std::vector<const float *> cvs(n);
        bool all_k = true, all_v = true, any_k = false, any_v = false;
        for (int i = 0; i < n; i++) {
            const int l = on[i];
            ks[i] = (const uint8_t *)L[l].K;
            sl[i] = R[l].selected_indices;
            ts[i] = plans[i].t_total;
            kd[i] = R[l].K_out;
            vd[i] = R[l].V_out;
            cvs[i] = R[l].C_v;
            all_k = all_k && kd[i];
            all_v = all_v && vd[i];
            any_k = any_k || kd[i];
            any_v = any_v || vd[i];
        }
        if (k_blocks && all_k == any_k && all_v == any_v && (any_k || any_v)) {
            kvc_stage_timer tm(ctx, KVC_ST_REQUANT, (any_k ? 1 : 0) + (any_v ? 1 : 0));
            rc = kvc_launch_requant_batch(n, ks.data(), sl.data(), ts.data(), any_k ? kd.data() : nullptr,
                                          m->k_row_bytes, ek, m->k_type, cvs.data(), any_v ? vd.data() : nullptr,
                                          m->v_row_bytes, H, dv, m->v_type, st);
            if (rc == KVC_OK) rq_done = true;
            else if (rc != KVC_ERR_SHAPE) return rc;
        }
    }
    for (int i = 0; i < n; i++) {
        const int l = on[i];
        const int t = plans[i].t_total;
        R[l].t = t;
        if (R[l].K_out && !rq_done) {
            kvc_stage_timer tm(ctx, KVC_ST_REQUANT, 1);
            rc = k_blocks ? kvc_launch_transcode_gather((const uint8_t *)L[l].K, m->k_row_bytes,
                                                        R[l].selected_indices, t, ek, m->k_type, R[l].K_out,
                                                        m->k_row_bytes, st)
                          : kvc_launch_encode_gather(jobs[i].K, (size_t)ek, R[l].selected_indices, t, ek,
                                                     m->k_type, R[l].K_out, m->k_row_bytes, st);
            if (rc) return rc;
        }
        if (R[l].V_out && !rq_done) {
            kvc_stage_timer tm(ctx, KVC_ST_REQUANT, 1);
            if ((rc = kvc_launch_encode_heads(R[l].C_v, H, t, t, dv, m->v_type, R[l].V_out, m->v_row_bytes, st)))
                return rc;
        }
        memset(&R[l].stats, 0, sizeof(R[l].stats));
        if (!want_stats) continue;
        if (jobs[i].out.mpart && plans[i].nq_top == plans[0].nq_top) {   // merged below, all layers at once
            m_parts.push_back(jobs[i].out.mpart);
            m_chunks.push_back(jobs[i].out.n_chunks);
            m_res.push_back(d_res + (size_t)pair_off[i] * 3);
        } else if ((rc = kvc_engine_metrics_launch(ctx, jobs[i], H, dk, dv, d_res + (size_t)pair_off[i] * 3))) {
            return rc;
        }
    }
    if (!m_parts.empty()) {
        kvc_stage_timer tm(ctx, KVC_ST_METRICS, 1);
        if ((rc = kvc_launch_metric_merge_batch(m_parts.data(), m_chunks.data(), m_res.data(), (int)m_parts.size(), H,
                                                plans[0].nq_top, dv, st)))
            return rc;
    }
    if ((rc = kvc_wait(ctx))) return rc;
    if (want_stats) {
        std::vector<float> h((size_t)pair_off[n] * 3);
        KVC_CUDA(cudaMemcpyAsync(h.data(), d_res, h.size() * sizeof(float), cudaMemcpyDeviceToHost, st));
        kvc_phase_collect(ctx, &ph);
        for (int i = 0; i < n; i++) {
            const int l = on[i];
            kvc_metrics_reduce(h.data() + (size_t)pair_off[i] * 3, pair_off[i + 1] - pair_off[i], &R[l].stats);
            R[l].stats.scoring_ms = ph.scoring_ms / n;
            R[l].stats.nnls_ms = ph.refit_ms / n;
        }
    }
    kvc_resolve_timers(ctx);
    return KVC_OK;
}

KVC_EXPORT int kvc_quantize_rows_dev(const float * src, size_t src_stride, int type, int rows, int n, uint8_t * dst,
                                     size_t dst_row_bytes) {
    if (!src || !dst) return KVC_ERR_NULL;
    if (rows < 0 || n <= 0) return KVC_ERR_DIMS;
    if (kvc_row_bytes(type, n) > dst_row_bytes) return KVC_ERR_ROWSIZE;
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    {
        kvc_stage_timer tm(ctx, KVC_ST_REQUANT, 1);
        if ((rc = kvc_launch_encode_gather(src, src_stride, nullptr, rows, n, type, dst, dst_row_bytes, ctx->stream)))
            return rc;
    }
    KVC_CUDA(cudaStreamSynchronize(ctx->stream));
    kvc_resolve_timers(ctx);
    return KVC_OK;
}

KVC_EXPORT int kvc_dequantize_rows_dev(const uint8_t * src, size_t src_row_bytes, int type, int rows, int n,
                                       float * dst) {
    if (!src || !dst) return KVC_ERR_NULL;
    if (rows < 0 || n <= 0) return KVC_ERR_DIMS;
    if (kvc_row_elements(type, src_row_bytes) < n) return KVC_ERR_ROWSIZE;
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    {
        kvc_stage_timer tm(ctx, KVC_ST_DECODE, 1);
        if ((rc = kvc_launch_decode(src, src_row_bytes, type, dst, rows, n, ctx->stream))) return rc;
    }
    KVC_CUDA(cudaStreamSynchronize(ctx->stream));
    kvc_resolve_timers(ctx);
    return KVC_OK;
}

}  // extern "C"
