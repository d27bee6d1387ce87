// state_ref.cpp — CPU checker for kvc_state_compact (test infrastructure;
// never linked into libkvc.so).
//
// The reference's state path lives in its headers and its CLI. The headers
// (include/kv-compact-state.h: parsed_kv_state::parse, build_compacted_state;
// include/kv-compact-math.h: mat_mul_ABt, softmax_importance_fused,
// exp_softmax_importance_fused, compute_head_sensitivity,
// accumulate_weighted_importance, nnls_solve, least_squares_solve,
// compute_beta_direction) are compiled here from where they lie (oracle/
// Makefile, target `ref`). The CLI (src/kv-compact.cpp) needs llama.cpp and
// cannot be built, so the steps it takes on a parsed state are restated
// below, each with the lines it follows:
//   reference queries = K rows of the last n_ref cells            :274-277, 452
//   per compacted layer and head: S = Q K^T * 1/sqrt(d_k),
//     softmax + importance, global max (or sensitivity-weighted sum) :456-556
//   top-t over all cells (partial_sort, then ascending)             :558-566
//   per layer and head: X = softmax(S[:, sel] + beta), Y = A V_h,
//     C_v = least_squares_solve(X, Y)                               :592-640
//   layers left out keep their V rows at the kept cells             :580-590
//   beta directions, then build_compacted_state                     :655-690, 786-792
// With fold_beta the beta of each layer and head is the API's
// Lawson-Hanson fit (src/kv-compact-api.cpp:812-831) instead of the CLI's 0.
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <numeric>
#include <vector>

#include "kv-compact-math.h"
#include "kv-compact-state.h"

extern "C" {

// layer_mask: n_layer flags of the layers to compact, or NULL for every layer
// parsed_kv_state::is_compactable_layer accepts with the first such layer's
// widths. gimp_out (optional, cell_count floats): the global importance the
// selection ranked. Returns 0 or the negative codes of kvc_state_compact.
int state_ref_compact(const uint8_t * in, size_t n, int n_head_kv, uint32_t n_pos_per_embd, float ratio,
                      int n_ref, int score_method, int use_sensitivity, const int * layer_mask, int fold_beta,
                      float ridge, uint8_t ** out, size_t * out_n, int * sel_out, int * t_out, float * gimp_out) {
    if (!in || !out || !out_n || n_head_kv <= 0) return -1;
    parsed_kv_state st;
    if (!st.parse(in, n, n_pos_per_embd)) return -20;
    if (st.n_stream == 0 || st.streams[0].cell_count == 0 || st.streams[0].n_layer == 0) return -20;
    for (uint32_t s = 1; s < st.n_stream; s++)
        if (st.streams[s].cell_count) return -21;
    const auto & sd = st.streams[0];
    const int T = (int)sd.cell_count, L = (int)sd.n_layer, H = n_head_kv;

    // layers compacted and their widths
    std::vector<int> on(L, 0);
    int ek = -1, ev = -1;
    for (int l = 0; l < L; l++) {
        const bool want = layer_mask ? layer_mask[l] != 0 : st.is_compactable_layer(0, l, H);
        if (!want) continue;
        if (!st.is_compactable_layer(0, l, H)) return -4;
        const int k = sd.layers[l].n_embd_k_gqa(), v = sd.layers[l].n_embd_v_gqa_computed();
        if (ek < 0) { ek = k; ev = v; }
        if (k != ek || v != ev) {
            if (layer_mask) return -4;
            continue;
        }
        on[l] = 1;
    }
    if (ek < 0) return -4;
    for (int l = 0; l < L; l++)
        if (sd.layers[l].n_embd_k_gqa() != ek || sd.layers[l].n_embd_v_gqa_computed() != ev) return -21;
    const int d_k = ek / H, d_v = ev / H;

    const int t = std::max(1, (int)(T * ratio));
    if (n_ref <= 0) n_ref = std::max(16, T / 4);
    n_ref = std::min(n_ref, T);
    const int ref_start = T - n_ref;
    const float inv_sqrt_dk = 1.0f / sqrtf((float)d_k);

    struct head_cache { std::vector<float> scores, attn, expv, rsum; };
    std::vector<std::vector<head_cache>> hc(L);
    std::vector<float> global(T, 0.0f);
    std::vector<std::vector<float>> head_imp;
    std::vector<float> sens;
    std::vector<float> q(n_ref * d_k), k(T * d_k);
    for (int l = 0; l < L; l++) {
        if (!on[l]) continue;
        const auto & ld = sd.layers[l];
        hc[l].resize(H);
        for (int h = 0; h < H; h++) {
            auto & c = hc[l][h];
            c.scores.resize((size_t)n_ref * T);
            c.attn.resize((size_t)n_ref * T);
            for (int i = 0; i < n_ref; i++)
                memcpy(q.data() + i * d_k, ld.K.data() + (size_t)(ref_start + i) * ek + h * d_k, d_k * 4);
            for (int j = 0; j < T; j++) memcpy(k.data() + (size_t)j * d_k, ld.K.data() + (size_t)j * ek + h * d_k, d_k * 4);
            mat_mul_ABt(q.data(), k.data(), c.scores.data(), n_ref, T, d_k);
            for (size_t i = 0; i < c.scores.size(); i++) c.scores[i] *= inv_sqrt_dk;
            std::vector<float> imp(T);
            if (fold_beta) {
                c.expv.resize((size_t)n_ref * T);
                c.rsum.resize(n_ref);
                exp_softmax_importance_fused(c.scores.data(), c.expv.data(), c.rsum.data(), c.attn.data(),
                                             imp.data(), n_ref, T, score_method);
            } else {
                softmax_importance_fused(c.scores.data(), c.attn.data(), imp.data(), n_ref, T, score_method);
            }
            if (use_sensitivity) {
                sens.push_back(compute_head_sensitivity(c.attn.data(), n_ref, T));
                head_imp.push_back(std::move(imp));
            } else {
                for (int j = 0; j < T; j++)
                    if (imp[j] > global[j]) global[j] = imp[j];
            }
        }
    }
    if (use_sensitivity) accumulate_weighted_importance(head_imp, sens, T, (int)sens.size(), global.data());
    if (gimp_out) memcpy(gimp_out, global.data(), (size_t)T * sizeof(float));
    std::vector<int> sel(T);
    std::iota(sel.begin(), sel.end(), 0);
    std::partial_sort(sel.begin(), sel.begin() + t, sel.end(),
                      [&](int a, int b) { return global[a] > global[b]; });
    sel.resize(t);
    std::sort(sel.begin(), sel.end());

    std::vector<std::vector<std::vector<float>>> cv_all(L), beta_all(L), dirs(L);
    std::vector<float> vbuf((size_t)T * d_v);
    for (int l = 0; l < L; l++) {
        const auto & ld = sd.layers[l];
        cv_all[l].resize(H);
        beta_all[l].resize(H);
        dirs[l].resize(H);
        for (int h = 0; h < H; h++) {
            auto & cv = cv_all[l][h];
            auto & beta = beta_all[l][h];
            cv.resize((size_t)t * d_v);
            beta.assign(t, 0.0f);
            dirs[l][h].assign(d_k, 0.0f);
            if (!on[l]) {
                for (int j = 0; j < t; j++)
                    memcpy(cv.data() + (size_t)j * d_v, ld.V.data() + (size_t)sel[j] * ev + h * d_v, d_v * 4);
                continue;
            }
            const auto & c = hc[l][h];
            if (fold_beta) {
                std::vector<float> M((size_t)n_ref * t), w(t);
                for (int i = 0; i < n_ref; i++)
                    for (int j = 0; j < t; j++) M[(size_t)i * t + j] = c.expv[(size_t)i * T + sel[j]];
                nnls_solve(M.data(), c.rsum.data(), w.data(), n_ref, t, 200);
                for (int j = 0; j < t; j++) beta[j] = logf(std::max(1e-12f, w[j]));
                std::vector<float> qh((size_t)n_ref * d_k);
                for (int i = 0; i < n_ref; i++)
                    memcpy(qh.data() + (size_t)i * d_k, ld.K.data() + (size_t)(ref_start + i) * ek + h * d_k, d_k * 4);
                compute_beta_direction(qh.data(), n_ref, d_k, dirs[l][h].data(), ridge);
            }
            std::vector<float> X((size_t)n_ref * t), Y((size_t)n_ref * d_v);
            for (int i = 0; i < n_ref; i++)
                for (int j = 0; j < t; j++) X[(size_t)i * t + j] = c.scores[(size_t)i * T + sel[j]] + beta[j];
            softmax_rows(X.data(), n_ref, t);
            for (int j = 0; j < T; j++) memcpy(vbuf.data() + (size_t)j * d_v, ld.V.data() + (size_t)j * ev + h * d_v, d_v * 4);
            mat_mul_AB(c.attn.data(), vbuf.data(), Y.data(), n_ref, T, d_v);
            least_squares_solve(X.data(), Y.data(), cv.data(), n_ref, t, d_v, ridge);
        }
    }
    std::vector<uint8_t> res = fold_beta
        ? build_compacted_state(st, sel, cv_all, H, d_k, d_v, n_pos_per_embd, beta_all, dirs)
        : build_compacted_state(st, sel, cv_all, H, d_k, d_v, n_pos_per_embd);
    *out = (uint8_t *)malloc(res.size() ? res.size() : 1);
    memcpy(*out, res.data(), res.size());
    *out_n = res.size();
    if (sel_out) memcpy(sel_out, sel.data(), (size_t)t * sizeof(int));
    if (t_out) *t_out = t;
    return 0;
}

void state_ref_free(void * p) { free(p); }

// Layout summary by the reference's parser (for the host-side parse checks).
int state_ref_inspect(const uint8_t * in, size_t n, uint32_t n_pos_per_embd, uint32_t * out4, size_t * trailing) {
    parsed_kv_state st;
    if (!st.parse(in, n, n_pos_per_embd)) return -20;
    out4[0] = st.n_stream;
    out4[1] = st.n_stream ? st.streams[0].cell_count : 0;
    out4[2] = st.n_stream ? st.streams[0].v_trans : 0;
    out4[3] = st.n_stream ? st.streams[0].n_layer : 0;
    *trailing = st.trailing_data.size();
    return 0;
}

}  // extern "C"
