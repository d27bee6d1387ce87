// state.cu — compaction of a saved llama.cpp sequence state (kvc-state.h).
//
// Host: a walk of the state's layout with the checks of the reference's
// parser (include/kv-compact-state.h:104-222: every read bounds-checked, row
// data sized cell_count * row bytes, transposed V n_embd * cell_count
// elements) that records offsets only; the bulk K/V bytes then go to the
// device in one copy and are decoded there by the library's codecs (a
// transposed V is decoded as n_embd rows of cell_count values and transposed).
// Every compacted layer is one unchunked unit of the engine whose reference
// queries are the K rows of the last n_ref cells (src/kv-compact.cpp:
// 274-277, 452). The engine's shared-selection mode keeps one set of cells
// for all layers: the top-t of the importance aggregated over every layer
// and head (src/kv-compact.cpp:470-566). Each layer then refits its values
// for that set (:592-640); layers left out keep their V rows (:580-590).
// With fold_beta the engine also fits beta (Lawson-Hanson, as the API's
// nnls_method 0) and K' = K + (beta * sqrt(d_k)) * v is written, v solving
// (Q^T Q + ridge I) v = Q^T 1 in fp64 for the layer's reference queries Q
// (compute_beta_direction, include/kv-compact-math.h:636-640;
// build_compacted_state, include/kv-compact-state.h:715-729).
// Writer (build_compacted_state, :645-810): cell records of the kept cells
// copied byte for byte, K rows re-encoded in their type, V rows from C_v in
// their type (or transposed, n_embd rows of t values), empty streams and the
// trailing bytes copied. The encoded sections are built on the device and
// copied into the output, whose headers the host writes.
#include <math.h>
#include <stdlib.h>

#include <algorithm>
#include <vector>

#include "../../include/kvc-state.h"
#include "engine.h"

namespace {

enum { ERR_FORMAT = -20, ERR_LAYOUT = -21 };
enum { SLOT_ST_IN = 10, SLOT_ST_F = 11, SLOT_ST_OUT = 12, SLOT_ST_ENC = 13 };

struct st_layer {
    int32_t k_type = 0, v_type = 0;
    uint64_t k_row = 0, v_row = 0;   // bytes per row (V: non-transposed only)
    uint32_t v_el = 0, v_embd = 0;   // transposed V: bytes per value, values per cell
    size_t k_data = 0, v_data = 0;   // offsets of the row data in the input
    int ek = 0, ev = 0;              // values per cell
};

struct st_layout {
    uint32_t n_stream = 0, cells = 0, v_trans = 0, n_layer = 0;
    std::vector<size_t> cell_off, cell_len;   // stream 0's cell records
    std::vector<st_layer> L;
    size_t kv_begin = 0, kv_end = 0;          // stream 0's first K row data .. end of its last V data
    size_t trailing = 0;                      // offset of the bytes after the KV section
};

template <typename T>
bool rd(const uint8_t * base, size_t size, size_t & pos, T & v) {
    if (pos + sizeof(T) > size) return false;
    memcpy(&v, base + pos, sizeof(T));
    pos += sizeof(T);
    return true;
}

bool known_type(int32_t t) { return t == 0 || t == 1 || t == 2 || t == 3 || t == 8; }

// Walk of the state's layout (offsets only). Streams after the first must be empty.
int walk(const uint8_t * d, size_t size, uint32_t n_pos_per_embd, st_layout * o) {
    size_t pos = 0;
    if (!rd(d, size, pos, o->n_stream)) return ERR_FORMAT;
    for (uint32_t s = 0; s < o->n_stream; s++) {
        uint32_t cc = 0;
        if (!rd(d, size, pos, cc)) return ERR_FORMAT;
        if (cc == 0) continue;
        if (s > 0) return ERR_LAYOUT;
        o->cells = cc;
        o->cell_off.resize(cc);
        o->cell_len.resize(cc);
        for (uint32_t c = 0; c < cc; c++) {
            const size_t at = pos;
            int32_t p;
            uint32_t n_seq;
            if (!rd(d, size, pos, p) || !rd(d, size, pos, n_seq)) return ERR_FORMAT;
            if (n_pos_per_embd > 1) {
                int32_t x, y;
                if (!rd(d, size, pos, x) || !rd(d, size, pos, y)) return ERR_FORMAT;
            }
            if ((size - pos) / 4 < n_seq) return ERR_FORMAT;
            pos += (size_t)n_seq * 4;
            o->cell_off[c] = at;
            o->cell_len[c] = pos - at;
        }
        if (!rd(d, size, pos, o->v_trans) || !rd(d, size, pos, o->n_layer)) return ERR_FORMAT;
        o->L.resize(o->n_layer);
        for (auto & ld : o->L) {
            if (!rd(d, size, pos, ld.k_type) || !rd(d, size, pos, ld.k_row)) return ERR_FORMAT;
            if (ld.k_row && cc > (size - pos) / ld.k_row) return ERR_FORMAT;
            if (!known_type(ld.k_type)) return ERR_LAYOUT;
            ld.k_data = pos;
            ld.ek = kvc_row_elements(ld.k_type, ld.k_row);
            pos += (size_t)cc * ld.k_row;
        }
        if (o->n_layer) o->kv_begin = o->L[0].k_data;
        for (auto & ld : o->L) {
            if (!o->v_trans) {
                if (!rd(d, size, pos, ld.v_type) || !rd(d, size, pos, ld.v_row)) return ERR_FORMAT;
                if (ld.v_row && cc > (size - pos) / ld.v_row) return ERR_FORMAT;
                if (!known_type(ld.v_type)) return ERR_LAYOUT;
                ld.v_data = pos;
                ld.ev = kvc_row_elements(ld.v_type, ld.v_row);
                pos += (size_t)cc * ld.v_row;
            } else {
                if (!rd(d, size, pos, ld.v_type) || !rd(d, size, pos, ld.v_el) || !rd(d, size, pos, ld.v_embd))
                    return ERR_FORMAT;
                const size_t bytes = (size_t)ld.v_embd * cc * ld.v_el;
                if (ld.v_el && (size_t)ld.v_embd * cc > (size - pos) / ld.v_el) return ERR_FORMAT;
                if (ld.v_type != 0 && ld.v_type != 1) return ERR_LAYOUT;   // transposed V: F32 / F16 values
                if (ld.v_el != (ld.v_type == 0 ? 4u : 2u)) return ERR_LAYOUT;
                ld.v_data = pos;
                ld.ev = (int)ld.v_embd;
                pos += bytes;
            }
        }
        o->kv_end = pos;
    }
    o->trailing = pos;
    return KVC_OK;
}

// dst [cols x rows] = src [rows x cols]^T, 32x32 tiles.
__global__ void k_transpose(const float * __restrict__ src, int rows, int cols, float * __restrict__ dst) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = src[(long long)r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[(long long)c * rows + r] = tile[threadIdx.x][i];
    }
}

int launch_transpose(const float * src, int rows, int cols, float * dst, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return KVC_OK;
    k_transpose<<<dim3((cols + 31) / 32, (rows + 31) / 32), dim3(32, 8), 0, st>>>(src, rows, cols, dst);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

// Direction of the beta fold for (layer, head) = blockIdx.x, blockIdx.y:
// (Q^T Q + ridge I) v = Q^T 1 in fp64 by Cholesky, Q the layer's reference
// queries of the head ([n_ref x d_k], rows `ek` apart). G in `work`.
__global__ void __launch_bounds__(256) k_beta_dir(const float * const * __restrict__ q_rows, int n_ref, int ek,
                                                  int dk, float ridge, double * __restrict__ work,
                                                  float * __restrict__ dirs) {
    const int l = blockIdx.x, h = blockIdx.y, H = gridDim.y;
    const float * Q = q_rows[l] + (long long)h * dk;
    double * G = work + ((long long)l * H + h) * ((long long)dk * dk + dk);
    double * b = G + (long long)dk * dk;
    for (int e = threadIdx.x; e < dk * dk; e += blockDim.x) {
        const int i = e / dk, j = e % dk;
        if (j > i) continue;
        double acc = 0.0;
        for (int q = 0; q < n_ref; q++) acc = fma((double)Q[(long long)q * ek + i], (double)Q[(long long)q * ek + j], acc);
        if (i == j) acc += (double)ridge;
        G[i * dk + j] = acc;
    }
    for (int i = threadIdx.x; i < dk; i += blockDim.x) {
        double acc = 0.0;
        for (int q = 0; q < n_ref; q++) acc += (double)Q[(long long)q * ek + i];
        b[i] = acc;
    }
    __syncthreads();
    // right-looking Cholesky on the lower triangle
    __shared__ double piv;
    for (int k = 0; k < dk; k++) {
        if (threadIdx.x == 0) {
            const double a = G[k * dk + k];
            piv = a > 0.0 ? sqrt(a) : 0.0;
            G[k * dk + k] = piv;
        }
        __syncthreads();
        const double pk = piv;
        for (int i = k + 1 + threadIdx.x; i < dk; i += blockDim.x) G[i * dk + k] = pk > 0.0 ? G[i * dk + k] / pk : 0.0;
        __syncthreads();
        for (int e = threadIdx.x; e < (dk - k - 1) * (dk - k - 1); e += blockDim.x) {
            const int i = k + 1 + e / (dk - k - 1), j = k + 1 + e % (dk - k - 1);
            if (j <= i) G[i * dk + j] -= G[i * dk + k] * G[j * dk + k];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < dk; i++) {                  // L y = b
            double s = b[i];
            for (int j = 0; j < i; j++) s -= G[i * dk + j] * b[j];
            b[i] = G[i * dk + i] > 0.0 ? s / G[i * dk + i] : 0.0;
        }
        for (int i = dk - 1; i >= 0; i--) {             // L^T v = y
            double s = b[i];
            for (int j = i + 1; j < dk; j++) s -= G[j * dk + i] * b[j];
            b[i] = G[i * dk + i] > 0.0 ? s / G[i * dk + i] : 0.0;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < dk; i += blockDim.x) dirs[((long long)l * H + h) * dk + i] = (float)b[i];
}

// K' rows of one layer: row j = K[sel[j]] + fl(fl(beta[h][j] * scale) * dir[h][d])
// per value (h, d) in the reference's rounding order (build_compacted_state,
// kv-compact-state.h:715-729); beta / dir null: a zero beta, as the reference
// folds it for layers left out (K + 0).
__global__ void k_fold_rows(const float * __restrict__ K, int ek, const int * __restrict__ sel, int t, int dk,
                            const float * __restrict__ beta, const float * __restrict__ dir, float scale,
                            float * __restrict__ out) {
    const long long total = (long long)t * ek;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int j = (int)(i / ek), e = (int)(i - (long long)j * ek);
        const int h = e / dk, d = e - h * dk;
        const float k = K[(long long)sel[j] * ek + e];
        const float bs = beta ? __fmul_rn(beta[(long long)h * t + j], scale) : 0.0f;
        const float dv = dir ? dir[(long long)h * dk + d] : 0.0f;
        out[i] = __fadd_rn(k, __fmul_rn(bs, dv));
    }
}

// [ev x t] values of a transposed V: column j of value e is head h = e / dv's
// C_v row j (or, cv null, the layer's V row sel[j]).
__global__ void k_v_columns(const float * __restrict__ cv, const float * __restrict__ V, const int * __restrict__ sel,
                            int t, int ev, int dv, float * __restrict__ out) {
    const long long total = (long long)t * ev;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int e = (int)(i / t), j = (int)(i - (long long)e * t);
        const int h = e / dv, c = e - h * dv;
        out[i] = cv ? cv[((long long)h * t + j) * dv + c] : V[(long long)sel[j] * ev + e];
    }
}

int grid_of(long long work) {
    long long g = (work + 255) / 256;
    return (int)std::max<long long>(1, std::min<long long>(g, 148LL * 16));
}

}  // namespace

extern "C" {

KVC_EXPORT kvc_state_params kvc_state_params_default(void) {
    kvc_state_params p;
    memset(&p, 0, sizeof(p));
    p.n_pos_per_embd = 1;
    p.target_ratio = 0.2f;
    p.score_method = 0;
    p.ridge = 1e-6f;
    return p;
}

KVC_EXPORT int kvc_state_inspect(const uint8_t * state, size_t size, uint32_t n_pos_per_embd, kvc_state_info * info) {
    if (!state || !info) return KVC_ERR_NULL;
    st_layout lo;
    const int rc = walk(state, size, n_pos_per_embd, &lo);
    memset(info, 0, sizeof(*info));
    if (rc) return rc;
    info->n_stream = lo.n_stream;
    info->cell_count = lo.cells;
    info->v_trans = lo.v_trans;
    info->n_layer = lo.n_layer;
    info->trailing_bytes = size - lo.trailing;
    return KVC_OK;
}

KVC_EXPORT void kvc_state_free(void * p) { kvc_hfree(p); }

KVC_EXPORT int kvc_state_compact(const uint8_t * state, size_t size, const kvc_state_params * params,
                                 uint8_t ** out_state, size_t * out_size, int ** out_selected,
                                 kvc_state_info * info) {
    if (!state || !params || !out_state || !out_size) return KVC_ERR_NULL;
    const kvc_state_params & sp = *params;
    const int H = sp.n_head_kv;
    if (H <= 0 || !(sp.target_ratio > 0.0f && sp.target_ratio < 1.0f) || sp.score_method < 0 || sp.score_method > 2)
        return KVC_ERR_DIMS;
    st_layout lo;
    int rc = walk(state, size, sp.n_pos_per_embd, &lo);
    if (rc) return rc;
    if (lo.cells == 0 || lo.n_layer == 0) return ERR_FORMAT;
    const int T = (int)lo.cells, NL = (int)lo.n_layer;

    // layers compacted: the filter's (each must split into H heads), else
    // every layer that splits with the first such layer's widths
    std::vector<int> on(NL, 0);
    int ek = -1, ev = -1;
    for (int l = 0; l < NL; l++) {
        const st_layer & ld = lo.L[l];
        const bool splits = ld.ek > 0 && ld.ev > 0 && ld.ek % H == 0 && ld.ev % H == 0;
        const bool want = sp.layer_filter ? sp.layer_filter(l, NL, sp.layer_filter_data) != 0 : splits;
        if (!want) continue;
        if (!splits) return KVC_ERR_ROWSIZE;
        if (ek < 0) { ek = ld.ek; ev = ld.ev; }
        if (ld.ek != ek || ld.ev != ev) {
            if (sp.layer_filter) return KVC_ERR_ROWSIZE;
            continue;
        }
        on[l] = 1;
    }
    if (ek < 0) return KVC_ERR_ROWSIZE;
    for (int l = 0; l < NL; l++)                       // the writer needs one geometry for every layer
        if (lo.L[l].ek != ek || lo.L[l].ev != ev) return ERR_LAYOUT;
    const int dk = ek / H, dv = ev / H;
    if (dk > KVC_MAX_D || dv > KVC_MAX_D) return KVC_ERR_SHAPE;
    const int t = std::max(1, (int)((float)T * sp.target_ratio));
    int n_ref = sp.n_ref_queries > 0 ? sp.n_ref_queries : std::max(16, T / 4);
    n_ref = std::min(n_ref, T);
    const int ref_start = T - n_ref;
    std::vector<int> comp;
    for (int l = 0; l < NL; l++)
        if (on[l]) comp.push_back(l);
    const int NC = (int)comp.size();

    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return rc;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaStream_t st = ctx->stream;

    // ---- device buffers: input KV bytes; fp32 K/V of every layer (+ room
    // for a transposed V's rows); per compacted layer sel | beta | C_v;
    // pointers, fold directions and their fp64 work; encoder inputs
    const size_t in_bytes = lo.kv_end - lo.kv_begin;
    const size_t kv_f = ((size_t)T * ek + 31) / 32 * 32, vv_f = ((size_t)T * ev + 31) / 32 * 32;
    void * a_in, * a_f, * a_out, * a_enc;
    if ((rc = kvc_arena(ctx, SLOT_ST_IN, in_bytes, &a_in))) return rc;
    if ((rc = kvc_arena(ctx, SLOT_ST_F, ((size_t)NL * (kv_f + vv_f) + vv_f) * 4, &a_f))) return rc;
    const size_t sel_n = ((size_t)t + 31) / 32 * 32, beta_n = ((size_t)H * t + 31) / 32 * 32,
                 cv_n = ((size_t)H * t * dv + 31) / 32 * 32;
    const size_t per_layer_out = sel_n + beta_n + cv_n;
    const size_t dir_n = ((size_t)NL * H * dk + 31) / 32 * 32;
    const size_t work_d = (size_t)NL * H * ((size_t)dk * dk + dk);
    if ((rc = kvc_arena(ctx, SLOT_ST_OUT, ((size_t)std::max(NC, 1) * per_layer_out + dir_n + NL * 2 + 64) * 4 +
                                              (sp.fold_beta ? work_d * 8 : 0), &a_out)))
        return rc;
    // encoded output sections of every layer: K rows, then V (rows or transposed values)
    std::vector<size_t> kenc_off(NL), venc_off(NL), kenc_len(NL), venc_len(NL);
    size_t enc_total = 0;
    for (int l = 0; l < NL; l++) {
        const st_layer & ld = lo.L[l];
        kenc_off[l] = enc_total;
        kenc_len[l] = (size_t)t * ld.k_row;
        enc_total += (kenc_len[l] + 255) & ~(size_t)255;
    }
    for (int l = 0; l < NL; l++) {
        const st_layer & ld = lo.L[l];
        venc_off[l] = enc_total;
        venc_len[l] = lo.v_trans ? (size_t)ev * t * ld.v_el : (size_t)t * ld.v_row;
        enc_total += (venc_len[l] + 255) & ~(size_t)255;
    }
    const size_t tmp_f = std::max((size_t)t * ek, (size_t)t * ev);
    if ((rc = kvc_arena(ctx, SLOT_ST_ENC, enc_total + tmp_f * 4 + 256, &a_enc))) return rc;
    uint8_t * d_in = (uint8_t *)a_in;
    float * d_K0 = (float *)a_f;
    auto dK = [&](int l) { return d_K0 + (size_t)l * (kv_f + vv_f); };
    auto dV = [&](int l) { return d_K0 + (size_t)l * (kv_f + vv_f) + kv_f; };
    float * d_vtmp = d_K0 + (size_t)NL * (kv_f + vv_f);
    float * d_o = (float *)a_out;
    auto dsel = [&](int c) { return (int *)(d_o + (size_t)c * per_layer_out); };
    auto dbeta = [&](int c) { return d_o + (size_t)c * per_layer_out + sel_n; };
    auto dcv = [&](int c) { return d_o + (size_t)c * per_layer_out + sel_n + beta_n; };
    float * d_dirs = d_o + (size_t)std::max(NC, 1) * per_layer_out;
    const float ** d_qrows = (const float **)(d_dirs + dir_n);
    double * d_work = (double *)(((uintptr_t)(d_qrows + NL) + 255) & ~(uintptr_t)255);
    uint8_t * d_enc = (uint8_t *)a_enc;
    float * d_tmp = (float *)(d_enc + enc_total);

    // ---- upload and decode every layer
    KVC_CUDA(cudaMemcpyAsync(d_in, state + lo.kv_begin, in_bytes, cudaMemcpyHostToDevice, st));
    for (int l = 0; l < NL; l++) {
        const st_layer & ld = lo.L[l];
        if ((rc = kvc_launch_decode(d_in + (ld.k_data - lo.kv_begin), ld.k_row, ld.k_type, dK(l), T, ek, st))) return rc;
        if (!lo.v_trans) {
            if ((rc = kvc_launch_decode(d_in + (ld.v_data - lo.kv_begin), ld.v_row, ld.v_type, dV(l), T, ev, st)))
                return rc;
        } else {
            if ((rc = kvc_launch_decode(d_in + (ld.v_data - lo.kv_begin), (size_t)T * ld.v_el, ld.v_type, d_vtmp, ev,
                                        T, st)))
                return rc;
            if ((rc = launch_transpose(d_vtmp, ev, T, dV(l), st))) return rc;
        }
    }

    // ---- one unit per compacted layer, one shared selection
    kv_compact_params p = kv_compact_params_default();
    p.score_method = sp.score_method;
    p.use_sensitivity = sp.use_sensitivity;
    p.skip_beta = sp.fold_beta ? 0 : 1;
    p.nnls_method = 0;
    p.nnls_max_iter = 200;
    p.ridge = sp.ridge;
    std::vector<kvc_plan> plans(NC);
    std::vector<kvc_layer_job> jobs(NC);
    for (int c = 0; c < NC; c++) {
        const int l = comp[c];
        kvc_plan & pl = plans[c];
        pl.T = T;
        pl.nq_top = n_ref;
        pl.chunk = T;
        pl.t_total = t;
        pl.units.push_back(kvc_plan_unit{0, T, t, 0, n_ref, 0});
        kvc_layer_job & J = jobs[c];
        J.K = dK(l);
        J.V = dV(l);
        J.Q = dK(l) + (size_t)ref_start * ek;
        J.plan = &pl;
        J.out.sel = dsel(c);
        J.out.beta = dbeta(c);
        J.out.cv = dcv(c);
        J.out.t_total = t;
    }
    kvc_shared_sel shared{t};
    if (NC > 0 && (rc = kvc_engine_run(ctx, p, H, dk, dv, jobs.data(), NC, nullptr, false, &shared))) return rc;

    // ---- beta directions (fold only), K' / K rows, V rows or columns
    const float scale = sqrtf((float)dk);
    if (sp.fold_beta && NC > 0) {
        std::vector<const float *> qr(NL, nullptr);
        for (int c = 0; c < NC; c++) qr[c] = dK(comp[c]) + (size_t)ref_start * ek;
        KVC_CUDA(cudaMemcpyAsync(d_qrows, qr.data(), NL * sizeof(float *), cudaMemcpyHostToDevice, st));
        k_beta_dir<<<dim3(NC, H), 256, 0, st>>>(d_qrows, n_ref, ek, dk, sp.ridge, d_work, d_dirs);
        KVC_CUDA(cudaGetLastError());
    }
    const int * sel0 = NC > 0 ? dsel(0) : nullptr;
    if (!sel0) return KVC_ERR_ROWSIZE;
    for (int l = 0; l < NL; l++) {
        const st_layer & ld = lo.L[l];
        const int c = on[l] ? (int)(std::find(comp.begin(), comp.end(), l) - comp.begin()) : -1;
        uint8_t * ko = d_enc + kenc_off[l];
        if (sp.fold_beta) {
            k_fold_rows<<<grid_of((long long)t * ek), 256, 0, st>>>(dK(l), ek, sel0, t, dk, c >= 0 ? dbeta(c) : nullptr,
                                                                    c >= 0 ? d_dirs + (size_t)c * H * dk : nullptr,
                                                                    scale, d_tmp);
            KVC_CUDA(cudaGetLastError());
            if ((rc = kvc_launch_encode_gather(d_tmp, (size_t)ek, nullptr, t, ek, ld.k_type, ko, ld.k_row, st))) return rc;
        } else if ((rc = kvc_launch_encode_gather(dK(l), (size_t)ek, sel0, t, ek, ld.k_type, ko, ld.k_row, st))) {
            return rc;
        }
        uint8_t * vo = d_enc + venc_off[l];
        if (!lo.v_trans) {
            if (c >= 0) rc = kvc_launch_encode_heads(dcv(c), H, t, t, dv, ld.v_type, vo, ld.v_row, st);
            else rc = kvc_launch_encode_gather(dV(l), (size_t)ev, sel0, t, ev, ld.v_type, vo, ld.v_row, st);
            if (rc) return rc;
        } else {
            k_v_columns<<<grid_of((long long)t * ev), 256, 0, st>>>(c >= 0 ? dcv(c) : nullptr, dV(l), sel0, t, ev, dv,
                                                                     d_tmp);
            KVC_CUDA(cudaGetLastError());
            if ((rc = kvc_launch_encode_gather(d_tmp, (size_t)t, nullptr, ev, t, ld.v_type, vo, (size_t)t * ld.v_el, st)))
                return rc;
        }
    }

    // ---- output: host headers and cell records, device sections copied in
    std::vector<int> sel(t);
    KVC_CUDA(cudaMemcpyAsync(sel.data(), sel0, (size_t)t * sizeof(int), cudaMemcpyDeviceToHost, st));
    if ((rc = kvc_wait(ctx))) return rc;
    size_t cells_bytes = 0;
    for (int j = 0; j < t; j++) cells_bytes += lo.cell_len[sel[j]];
    size_t total = 4 + 4 + cells_bytes + 8;
    for (int l = 0; l < NL; l++) total += 12 + kenc_len[l];
    for (int l = 0; l < NL; l++) total += 12 + venc_len[l];     // [v_type][v_size_row] or [v_type][v_size_el][n_embd_v]
    total += (size_t)(lo.n_stream - 1) * 4 + (size - lo.trailing);
    uint8_t * out = (uint8_t *)kvc_hmalloc(total);
    if (!out) return KVC_ERR_OOM;
    size_t w = 0;
    auto put = [&](const void * src, size_t n) { memcpy(out + w, src, n); w += n; };
    struct piece { size_t dst; const uint8_t * src; size_t n; };
    std::vector<piece> pieces;
    put(&lo.n_stream, 4);
    const uint32_t tt = (uint32_t)t;
    put(&tt, 4);
    for (int j = 0; j < t; j++) put(state + lo.cell_off[sel[j]], lo.cell_len[sel[j]]);
    put(&lo.v_trans, 4);
    put(&lo.n_layer, 4);
    for (int l = 0; l < NL; l++) {
        put(&lo.L[l].k_type, 4);
        put(&lo.L[l].k_row, 8);
        pieces.push_back({w, d_enc + kenc_off[l], kenc_len[l]});
        w += kenc_len[l];
    }
    for (int l = 0; l < NL; l++) {
        put(&lo.L[l].v_type, 4);
        if (!lo.v_trans) {
            put(&lo.L[l].v_row, 8);
        } else {
            const uint32_t ne = (uint32_t)(H * dv);
            put(&lo.L[l].v_el, 4);
            put(&ne, 4);
        }
        pieces.push_back({w, d_enc + venc_off[l], venc_len[l]});
        w += venc_len[l];
    }
    const uint32_t zero = 0;
    for (uint32_t s = 1; s < lo.n_stream; s++) put(&zero, 4);
    put(state + lo.trailing, size - lo.trailing);
    if (w != total) {                                  // the size computed above must be the size written
        kvc_hfree(out);
        return ERR_FORMAT;
    }
    for (const piece & pc : pieces)
        if (pc.n) KVC_CUDA(cudaMemcpyAsync(out + pc.dst, pc.src, pc.n, cudaMemcpyDeviceToHost, st));
    if ((rc = kvc_wait(ctx))) {
        kvc_hfree(out);
        return rc;
    }
    *out_state = out;
    *out_size = w;
    if (out_selected) {
        int * so = (int *)kvc_hmalloc((size_t)t * sizeof(int));
        memcpy(so, sel.data(), (size_t)t * sizeof(int));
        *out_selected = so;
    }
    if (info) {
        memset(info, 0, sizeof(*info));
        info->n_stream = lo.n_stream;
        info->cell_count = lo.cells;
        info->v_trans = lo.v_trans;
        info->n_layer = lo.n_layer;
        info->n_compacted = NC;
        info->t = t;
        info->n_ref_queries = n_ref;
        info->trailing_bytes = size - lo.trailing;
    }
    kvc_resolve_timers(ctx);
    return KVC_OK;
}

}  // extern "C"
