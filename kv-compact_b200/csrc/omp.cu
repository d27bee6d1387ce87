// omp.cu — orthogonal-matching-pursuit key selection (use_omp) on the device.
//
// The reference (include/kv-compact-math.h:832-950, called from
// src/kv-compact-api.cpp:687-715) selects keys greedily by attention mass:
//   CE = sum over heads of the exp-scores E_h[q][j] = expf(S_h[q][j] - max_j),
//   CS = sum over heads of their row sums (sequential over j);
//   repeat until t keys are chosen: residual r = CS - cur; corr[j] = CE[:,j].r
//   over the unchosen keys; take the k_choice largest (first maximum on ties);
//   every refit_interval-th round (and at the end) refit the weights of the
//   chosen keys by the clamped least-squares NNLS (normal equations + 1e-10
//   ridge, Gaussian elimination with partial pivoting, clamp at 1e-12,
//   optional projected-gradient steps) and set cur = CE[:,chosen] w; in the
//   other rounds new keys get weight 1e-12. The chosen keys, sorted by
//   position, are the selection (the weights are not used further).
// Each of these quantities depends on the previous rounds through argmax
// decisions, so they are computed here in the reference's fp32 operation
// order: every sum that the reference runs sequentially is a sequential loop
// of explicitly rounded multiply/add in one thread (parallel only across
// independent sums), argmax reductions resolve ties to the lowest index, and
// the elimination updates each element with the same two roundings.
//
//   k_omp_exp     one CTA per unit: row max and sequential row sum of every
//                 (head, query) row of the raw scores, then CE and CS.
//                 Runs between the scoring and the softmax (which overwrites S).
//   k_omp_select  one CTA per unit: the greedy loop; working arrays in the
//                 unit's scratch (kvc_omp_floats).
#include "engine.h"

#include <math.h>

namespace {
constexpr int OT = 256;   // threads of both kernels

// e^x rounded to float from the double-precision exponential: the correctly
// rounded result except when e^x lies within ~1e-16 relative of a rounding
// boundary between two floats — the result the reference's libm expf returns.
// The greedy loop below branches on these values, so a last-bit difference
// (the single-precision expf is within 2 ulp) could change the selection.
__device__ __forceinline__ float exp_f(float x) { return (float)exp((double)x); }

struct omp_ws {           // per-unit working arrays (floats unless noted)
    float *CE, *CS, *cur, *res, *corr, *M, *AtA, *Atb, *aug, *w, *prev, *pu, *pv, *pg, *fcol, *rmx, *rrs;
    int *order, *mask;
};

__host__ __device__ inline long long omp_floats(int C, int t, int nq, int H) {
    return (long long)nq * C + 4LL * nq + C + (long long)nq * t + (long long)t * t + t + (long long)t * (t + 1) +
           6LL * t + 2LL * H * nq + t + C + 64;
}

__device__ omp_ws omp_layout(float * base, int C, int t, int nq, int H) {
    omp_ws w;
    float * p = base;
    w.CE = p; p += (long long)nq * C;
    w.CS = p; p += nq;
    w.cur = p; p += nq;
    w.res = p; p += nq;
    w.pv = p; p += nq;
    w.corr = p; p += C;
    w.M = p; p += (long long)nq * t;
    w.AtA = p; p += (long long)t * t;
    w.Atb = p; p += t;
    w.aug = p; p += (long long)t * (t + 1);
    w.w = p; p += t;
    w.prev = p; p += t;
    w.pu = p; p += t;
    w.pg = p; p += t;
    w.fcol = p; p += t;
    w.rmx = p; p += (long long)H * nq;
    w.rrs = p; p += (long long)H * nq;
    w.order = reinterpret_cast<int *>(p); p += t;
    w.mask = reinterpret_cast<int *>(p);
    return w;
}
}  // namespace

size_t kvc_omp_floats(int C, int t, int nq, int H) { return (size_t)omp_floats(C, t, nq, H); }

// Exp-scores summed over heads (CE) and their row sums (CS), from the raw
// scores S of the unit (src/kv-compact-api.cpp:632-649 with math.h:142-196:
// per row mx = first element then the maximum, e = expf(s - mx), sum over j in
// order; then the per-head arrays accumulated in head order).
__global__ void __launch_bounds__(OT) k_omp_exp(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                float * __restrict__ fs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active || u.omp_off < 0) return;
    const int C = u.C, nq = u.nq, H = P.H;
    omp_ws W = omp_layout(fs + u.omp_off, C, u.t, nq, H);
    for (int r = threadIdx.x; r < H * nq; r += OT) {
        const int h = r / nq, i = r - h * nq;
        const float * row = fs + u.s_off + ((long long)h * nq + i) * C;
        float mx = row[0];
        for (int j = 1; j < C; j++) if (row[j] > mx) mx = row[j];
        float s = 0.0f;
        for (int j = 0; j < C; j++) s = __fadd_rn(s, exp_f(__fsub_rn(row[j], mx)));
        W.rmx[r] = mx;
        W.rrs[r] = s;
    }
    __syncthreads();
    for (long long e = threadIdx.x; e < (long long)nq * C; e += OT) {
        const int i = (int)(e / C), j = (int)(e - (long long)i * C);
        float acc = 0.0f;
        for (int h = 0; h < H; h++) {
            const float v = fs[u.s_off + ((long long)h * nq + i) * C + j];
            acc = __fadd_rn(acc, exp_f(__fsub_rn(v, W.rmx[h * nq + i])));
        }
        W.CE[e] = acc;
    }
    for (int i = threadIdx.x; i < nq; i += OT) {
        float acc = 0.0f;
        for (int h = 0; h < H; h++) acc = __fadd_rn(acc, W.rrs[h * nq + i]);
        W.CS[i] = acc;
    }
}

namespace {
// Largest value among the threads' candidates, ties to the lowest index
// (a sequential scan with strict '>' keeps the first maximum). Candidates with
// idx < 0 take no part. Every thread returns the winner's index (-1: none).
__device__ int block_argmax(float v, int idx, float * sv, int * si) {
    for (int o = 16; o; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (i2 >= 0 && (idx < 0 || v2 > v || (v2 == v && i2 < idx))) { v = v2; idx = i2; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();                               // the previous use of sv/si is over
    if (lane == 0) { sv[warp] = v; si[warp] = idx; }
    __syncthreads();
    v = sv[0];
    idx = si[0];
    for (int k = 1; k < OT / 32; k++) {
        const float v2 = sv[k];
        const int i2 = si[k];
        if (i2 >= 0 && (idx < 0 || v2 > v || (v2 == v && i2 < idx))) { v = v2; idx = i2; }
    }
    return idx;
}

// One scalar computed by thread 0, then seen by every thread.
__device__ float block_bcast(float v, float * slot) {
    __syncthreads();
    if (threadIdx.x == 0) *slot = v;
    __syncthreads();
    return *slot;
}

// In-place Gaussian elimination with partial pivoting on [n x (n+1)] and back
// substitution into x (math.h:359-397 as restated in the oracle): pivots with
// |pivot| < 1e-12 are skipped and their unknowns set to skip_value.
__device__ void gauss_solve(float * aug, int n, float * x, float skip_value, float * fcol, float * sv, int * si) {
    const int wd = n + 1;
    for (int c = 0; c < n; c++) {
        float best = -1.0f;
        int bi = -1;
        for (int r = c + threadIdx.x; r < n; r += OT) {
            const float v = fabsf(aug[(long long)r * wd + c]);
            if (bi < 0 || v > best) { best = v; bi = r; }
        }
        const int pr = block_argmax(best, bi, sv, si);
        if (pr != c && pr >= 0)
            for (int j = threadIdx.x; j < wd; j += OT) {
                const float tmp = aug[(long long)c * wd + j];
                aug[(long long)c * wd + j] = aug[(long long)pr * wd + j];
                aug[(long long)pr * wd + j] = tmp;
            }
        __syncthreads();
        const float piv = aug[(long long)c * wd + c];
        if (fabsf(piv) < 1e-12f) continue;           // uniform: every thread read the same value
        for (int r = c + 1 + threadIdx.x; r < n; r += OT) fcol[r] = __fdiv_rn(aug[(long long)r * wd + c], piv);
        __syncthreads();
        const int span = wd - c;
        for (long long e = threadIdx.x; e < (long long)(n - c - 1) * span; e += OT) {
            const int r = c + 1 + (int)(e / span), j = c + (int)(e % span);
            aug[(long long)r * wd + j] = __fsub_rn(aug[(long long)r * wd + j], __fmul_rn(fcol[r], aug[(long long)c * wd + j]));
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        for (int c = n - 1; c >= 0; c--) {
            const float piv = aug[(long long)c * wd + c];
            if (fabsf(piv) < 1e-12f) { x[c] = skip_value; continue; }
            float v = aug[(long long)c * wd + n];
            for (int r = c + 1; r < n; r++) v = __fsub_rn(v, __fmul_rn(aug[(long long)c * wd + r], x[r]));
            x[c] = __fdiv_rn(v, piv);
        }
    }
    __syncthreads();
}
}  // namespace

namespace {
// Clamped least squares with optional projected-gradient steps on
// A [m x n] w ~= b (math.h:683-806 as restated in the oracle, eps = 1e-12).
__device__ void nnls_pgd(const float * A, const float * b, int m, int n, int iters, const omp_ws & W,
                         float * sv, int * si, float * slot) {
    const float eps = 1e-12f;
    for (long long e = threadIdx.x; e < (long long)n * n; e += OT) {   // AtA, sequential over rows
        const int i = (int)(e / n), j = (int)(e % n);
        float s = 0.0f;
        for (int k = 0; k < m; k++) s = __fadd_rn(s, __fmul_rn(A[(long long)k * n + i], A[(long long)k * n + j]));
        W.AtA[e] = s;
    }
    for (int i = threadIdx.x; i < n; i += OT) {
        float s = 0.0f;
        for (int k = 0; k < m; k++) s = __fadd_rn(s, __fmul_rn(A[(long long)k * n + i], b[k]));
        W.Atb[i] = s;
    }
    __syncthreads();
    const int wd = n + 1;
    for (long long e = threadIdx.x; e < (long long)n * wd; e += OT) {
        const int i = (int)(e / wd), j = (int)(e % wd);
        float v = (j < n) ? W.AtA[(long long)i * n + j] : W.Atb[i];
        if (j == i) v = __fadd_rn(v, 1e-10f);
        W.aug[e] = v;
    }
    __syncthreads();
    gauss_solve(W.aug, n, W.w, eps, W.fcol, sv, si);
    for (int i = threadIdx.x; i < n; i += OT) if (W.w[i] < eps) W.w[i] = eps;
    __syncthreads();
    if (iters <= 0) return;
    const float u0 = __fdiv_rn(1.0f, sqrtf((float)n));
    for (int j = threadIdx.x; j < n; j += OT) W.pu[j] = u0;
    __syncthreads();
    for (int pw = 0; pw < 3; pw++) {                                    // power iteration for the step size
        for (int i = threadIdx.x; i < m; i += OT) {
            float acc = 0.0f;
            for (int j = 0; j < n; j++) acc = __fadd_rn(acc, __fmul_rn(A[(long long)i * n + j], W.pu[j]));
            W.pv[i] = acc;
        }
        __syncthreads();
        float vn = 0.0f;
        if (threadIdx.x == 0) {
            for (int i = 0; i < m; i++) vn = __fadd_rn(vn, __fmul_rn(W.pv[i], W.pv[i]));
            vn = sqrtf(vn);
        }
        vn = block_bcast(vn, slot);
        if (vn < 1e-12f) break;
        for (int i = threadIdx.x; i < m; i += OT) W.pv[i] = __fdiv_rn(W.pv[i], vn);
        __syncthreads();
        for (int j = threadIdx.x; j < n; j += OT) {
            float acc = 0.0f;
            for (int i = 0; i < m; i++) acc = __fadd_rn(acc, __fmul_rn(A[(long long)i * n + j], W.pv[i]));
            W.pu[j] = acc;
        }
        __syncthreads();
        float un = 0.0f;
        if (threadIdx.x == 0) {
            for (int j = 0; j < n; j++) un = __fadd_rn(un, __fmul_rn(W.pu[j], W.pu[j]));
            un = sqrtf(un);
        }
        un = block_bcast(un, slot);
        if (un < 1e-12f) break;
        for (int j = threadIdx.x; j < n; j += OT) W.pu[j] = __fdiv_rn(W.pu[j], un);
        __syncthreads();
    }
    for (int i = threadIdx.x; i < n; i += OT) {                         // (AtA u)_i
        float acc = 0.0f;
        for (int j = 0; j < n; j++) acc = __fadd_rn(acc, __fmul_rn(W.AtA[(long long)i * n + j], W.pu[j]));
        W.pg[i] = acc;
    }
    __syncthreads();
    float L = 0.0f;
    if (threadIdx.x == 0) {
        for (int i = 0; i < n; i++) L = __fadd_rn(L, __fmul_rn(W.pu[i], W.pg[i]));
        if (L < 1e-6f) L = 1e-6f;
    }
    L = block_bcast(L, slot);
    const float eta = __fdiv_rn(1.0f, L);
    for (int it = 0; it < iters; it++) {
        for (int i = threadIdx.x; i < n; i += OT) {
            float acc = 0.0f;
            for (int j = 0; j < n; j++) acc = __fadd_rn(acc, __fmul_rn(W.AtA[(long long)i * n + j], W.w[j]));
            W.pg[i] = __fsub_rn(acc, W.Atb[i]);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += OT) {
            float v = __fsub_rn(W.w[i], __fmul_rn(eta, W.pg[i]));
            W.w[i] = v < eps ? eps : v;
        }
        __syncthreads();
    }
}
}  // namespace

// The greedy selection of one unit (math.h:832-950 as restated in the oracle).
__global__ void __launch_bounds__(OT) k_omp_select(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                   float * __restrict__ fs, int * __restrict__ is,
                                                   const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active || u.omp_off < 0) return;
    const int C = u.C, nq = u.nq, t = u.t;
    omp_ws W = omp_layout(fs + u.omp_off, C, t, nq, P.H);
    __shared__ float sv[OT / 32];
    __shared__ int si[OT / 32];
    __shared__ float slot;
    const int kc = P.omp_k_choice, refit = P.omp_refit_interval;
    for (int i = threadIdx.x; i < nq; i += OT) W.cur[i] = 0.0f;
    for (int j = threadIdx.x; j < C; j += OT) W.mask[j] = 0;
    __syncthreads();
    int nsel = 0, nprev = 0, iter = 0;
    // every round adds at least one key unless no finite correlation is left;
    // the bound only ends that degenerate case (where the reference would spin)
    while (nsel < t && iter <= C + t) {
        for (int i = threadIdx.x; i < nq; i += OT) W.res[i] = __fsub_rn(W.CS[i], W.cur[i]);
        __syncthreads();
        for (int j = threadIdx.x; j < C; j += OT) {
            float c = 0.0f;
            if (!W.mask[j])
                for (int i = 0; i < nq; i++) c = __fadd_rn(c, __fmul_rn(W.CE[(long long)i * C + j], W.res[i]));
            W.corr[j] = c;
        }
        __syncthreads();
        int k_sel = kc < t - nsel ? kc : t - nsel;
        if (k_sel > C - nsel) k_sel = C - nsel;
        if (k_sel <= 0) break;
        for (int k = 0; k < k_sel; k++) {
            float best = 0.0f;
            int bi = -1;
            for (int j = threadIdx.x; j < C; j += OT) {
                if (W.mask[j]) continue;
                const float c = W.corr[j];
                if (c > -1e30f && (bi < 0 || c > best)) { best = c; bi = j; }
            }
            const int b = block_argmax(best, bi, sv, si);
            if (b < 0) break;                    // (uniform) no candidate left this round
            if (threadIdx.x == 0) {
                W.order[nsel] = b;
                W.mask[b] = 1;
                W.corr[b] = -1e30f;
            }
            nsel++;
            __syncthreads();
        }
        const int ct = nsel;
        const bool solve = (refit <= 1) || (iter % refit == 0) || (ct == t);
        if (solve) {
            for (long long e = threadIdx.x; e < (long long)nq * ct; e += OT) {
                const int i = (int)(e / ct), j = (int)(e % ct);
                W.M[e] = W.CE[(long long)i * C + W.order[j]];
            }
            __syncthreads();
            nnls_pgd(W.M, W.CS, nq, ct, P.nnls_pgd_iters, W, sv, si, &slot);
            for (int j = threadIdx.x; j < ct; j += OT) W.prev[j] = W.w[j];
            nprev = ct;
            for (int i = threadIdx.x; i < nq; i += OT) {
                float acc = 0.0f;
                for (int j = 0; j < ct; j++) acc = __fadd_rn(acc, __fmul_rn(W.M[(long long)i * ct + j], W.w[j]));
                W.cur[i] = acc;
            }
        } else {
            for (int j = nprev + threadIdx.x; j < ct; j += OT) W.prev[j] = 1e-12f;
            nprev = ct;
            __syncthreads();
            for (int i = threadIdx.x; i < nq; i += OT) {
                float acc = 0.0f;
                for (int j = 0; j < ct; j++)
                    acc = __fadd_rn(acc, __fmul_rn(W.CE[(long long)i * C + W.order[j]], W.prev[j]));
                W.cur[i] = acc;
            }
        }
        __syncthreads();
        iter++;
    }
    // chosen keys in position order (distinct), as chunk-local and global indices
    if (threadIdx.x == 0) {
        for (int a = 1; a < nsel; a++) {
            const int key = W.order[a];
            int b = a - 1;
            while (b >= 0 && W.order[b] > key) { W.order[b + 1] = W.order[b]; b--; }
            W.order[b + 1] = key;
        }
    }
    __syncthreads();
    int * sel = is + u.sel_off;
    const kvc_layer_out lo = outs[u.layer];
    for (int j = threadIdx.x; j < t; j += OT) {
        const int v = j < nsel ? W.order[j] : 0;
        sel[j] = v;
        lo.sel[u.out_off + j] = u.token_base + v;
    }
}

int kvc_launch_omp_exp(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    k_omp_exp<<<n_units, OT, 0, st>>>(d_units, P, fs);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_omp_select(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs, int * is,
                          const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    k_omp_select<<<n_units, OT, 0, st>>>(d_units, P, fs, is, d_outs);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
