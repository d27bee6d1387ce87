// nnls.cu — beta fit (NNLS) and worst-key refinement on the device.
//
// Beta (src/kv-compact-api.cpp:812-831): per (unit, head), M[q][j] =
// exp(S[q][sel_j] - rowmax[q]) (the reference's exp-scores), b[q] = row sum
// of exp-scores over the chunk; w = NNLS(M, b); beta_j = log(max(1e-12, w_j)).
//
//   k_nnls_gram  A = M^T M and c = M^T b in fp64 (32x32 tiles over t x t),
//                M formed on the fly from the raw S[:, sel] block.
//   k_nnls_lh    Lawson-Hanson (include/kv-compact-math.h:283-452) with the
//                reference's decision rules: entering variable = first
//                largest positive dual (KKT threshold 1e-10), feasibility
//                s_P > 0, step alpha = min w/(w - s + 1e-30), variables with
//                |w| < 1e-12 leave P, subproblem ridge 1e-10, final clamp at
//                1e-12. The subproblem is solved with a Cholesky factor of
//                A[P,P] kept in insertion order: a new variable appends one
//                row (O(p^2)); when variables leave P the factor is rebuilt.
//   k_nnls_pgd   nnls_method 1 (math.h:683-806): (A + 1e-10 I) w = c by
//                Cholesky, clamp at 1e-12, then the optional projected
//                gradient steps with the 3-step power-iteration step size.
// The reference solves these systems in fp32 by Gaussian elimination; here
// they run in fp64, so where the fp32 result is dominated by rounding the
// two can differ (tolerance-checked by the parity tests, not bit-checked).
//
// Refinement (src/kv-compact-api.cpp:852-946), k_refine, one CTA per unit:
// key_value[j] = sum_h mean_q X_h[q][j]^2 with X_h = softmax(S[:, sel] + beta)
// (the X of the last solve; the reference recomputes this softmax per key),
// worst = first minimum, best unused = first maximum importance outside the
// kept set, stop when best <= 0.5 * importance(worst), else swap, re-sort,
// and the following beta / X / C_v stages re-solve the unit.
#include "engine.h"

#include <math.h>

namespace {
constexpr int NT = 32;

// doubles per (unit, head): A [t x t] | c [t] | packed L [t(t+1)/2] | work [4t + n_q]
__host__ __device__ inline long long kvc_nnls_stride(int t, int nq) {
    return (long long)t * t + t + (long long)t * (t + 1) / 2 + 4LL * t + nq;
}

__device__ __forceinline__ const float * sraw(const kvc_unit & u, const float * fs, int h) {
    return fs + u.x_off + (long long)h * u.nq * u.t;   // raw S[:, sel] before the X softmax
}
}  // namespace

// A (t x t) and c (t) per (unit, head), fp64; nn region: [A | c | L | work].
__global__ void __launch_bounds__(256) k_nnls_gram(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                   const float * __restrict__ fs, double * __restrict__ gs) {
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y, t = u.t, nq = u.nq;
    const int tn = (t + NT - 1) / NT;
    const int nc = tn * tn;
    if ((int)blockIdx.x > nc) return;
    const float * S = sraw(u, fs, h);
    const float * rmax = fs + u.row_off + (long long)h * 2 * nq;
    const float * rsum = rmax + nq;
    const long long stride = (long long)kvc_nnls_stride(t, nq);
    double * A = gs + u.g_off + (long long)h * stride;
    double * c = A + (long long)t * t;
    if ((int)blockIdx.x == nc) {
        // c = M^T b
        for (int j = threadIdx.x; j < t; j += blockDim.x) {
            double acc = 0.0;
            for (int q = 0; q < nq; q++) {
                float m = expf(__fsub_rn(S[(long long)q * t + j], rmax[q]));
                acc = fma((double)m, (double)rsum[q], acc);
            }
            c[j] = acc;
        }
        return;
    }
    const int a0 = (blockIdx.x / tn) * NT, b0 = (blockIdx.x % tn) * NT;
    if (b0 > a0) return;
    __shared__ double As[NT][NT + 1];
    __shared__ double Bs[NT][NT + 1];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    double acc[2][2] = {{0, 0}, {0, 0}};
    for (int k0 = 0; k0 < nq; k0 += NT) {
        for (int e = tid; e < NT * NT; e += 256) {
            int kk = e / NT, r = e % NT;
            int q = k0 + kk;
            double xa = 0.0, xb = 0.0;
            if (q < nq) {
                if (a0 + r < t) xa = (double)expf(__fsub_rn(S[(long long)q * t + a0 + r], rmax[q]));
                if (b0 + r < t) xb = (double)expf(__fsub_rn(S[(long long)q * t + b0 + r], rmax[q]));
            }
            As[kk][r] = xa;
            Bs[kk][r] = xb;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < NT; kk++) {
            double x0 = As[kk][ty * 2], x1 = As[kk][ty * 2 + 1];
            double y0 = Bs[kk][tx * 2], y1 = Bs[kk][tx * 2 + 1];
            acc[0][0] = fma(x0, y0, acc[0][0]);
            acc[0][1] = fma(x0, y1, acc[0][1]);
            acc[1][0] = fma(x1, y0, acc[1][0]);
            acc[1][1] = fma(x1, y1, acc[1][1]);
        }
        __syncthreads();
    }
    for (int i = 0; i < 2; i++)
        for (int j = 0; j < 2; j++) {
            int a = a0 + ty * 2 + i, b = b0 + tx * 2 + j;
            if (a < t && b < t && b <= a) {
                A[(long long)a * t + b] = acc[i][j];
                A[(long long)b * t + a] = acc[i][j];
            }
        }
}

namespace {
// warp-level helpers (one warp runs the sequential parts of a solver)
__device__ __forceinline__ double warp_sum_d(double v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Append variable `var` as row p of the packed factor L (insertion order in
// `ord`): L[p][m] = (A[var][ord[m]] - sum L[p][k] L[m][k]) / L[m][m], then the
// diagonal. Returns false when the new pivot is not positive.
__device__ bool chol_append(double * L, const double * A, int t, const int * ord, int p, int var, double ridge) {
    const int lane = threadIdx.x & 31;
    double * Lp = L + (long long)p * (p + 1) / 2;
    for (int m = 0; m < p; m++) {
        const double * Lm = L + (long long)m * (m + 1) / 2;
        double part = 0.0;
        for (int k = lane; k < m; k += 32) part = fma(Lp[k], Lm[k], part);
        double s = warp_sum_d(part);
        if (lane == 0) {
            double v = A[(long long)var * t + ord[m]] - s;
            Lp[m] = (Lm[m] > 0.0) ? v / Lm[m] : 0.0;
        }
        __syncwarp();
    }
    double part = 0.0;
    for (int k = lane; k < p; k += 32) part = fma(Lp[k], Lp[k], part);
    double s = warp_sum_d(part);
    double d = A[(long long)var * t + var] + ridge - s;
    bool ok = d > 0.0 && isfinite(d);
    if (lane == 0) Lp[p] = ok ? sqrt(d) : 0.0;
    __syncwarp();
    return ok;
}

// Solve L L^T s = rhs over the p variables (rhs in y, result in y).
__device__ void chol_solve(const double * L, double * y, int p) {
    const int lane = threadIdx.x & 31;
    for (int i = 0; i < p; i++) {                 // forward, row-oriented
        const double * Li = L + (long long)i * (i + 1) / 2;
        double part = 0.0;
        for (int k = lane; k < i; k += 32) part = fma(Li[k], y[k], part);
        double s = warp_sum_d(part);
        if (lane == 0) y[i] = (Li[i] > 0.0) ? (y[i] - s) / Li[i] : 0.0;
        __syncwarp();
    }
    for (int i = p - 1; i >= 0; i--) {            // backward, column-oriented on row i
        const double * Li = L + (long long)i * (i + 1) / 2;
        double si = 0.0;
        if (lane == 0) {
            si = (Li[i] > 0.0) ? y[i] / Li[i] : 0.0;
            y[i] = si;
        }
        si = __shfl_sync(0xffffffffu, si, 0);
        for (int k = lane; k < i; k += 32) y[k] -= Li[k] * si;
        __syncwarp();
    }
}
}  // namespace

// One warp per (unit, head); vectors in shared memory, A and L in global.
__global__ void __launch_bounds__(32) k_nnls_lh(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                double * __restrict__ gs, const kvc_layer_out * __restrict__ outs,
                                                int max_t) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    const int h = blockIdx.y, t = u.t;
    const long long stride = (long long)kvc_nnls_stride(t, u.nq);
    const double * A = gs + u.g_off + (long long)h * stride;
    const double * c = A + (long long)t * t;
    double * L = const_cast<double *>(c) + t;
    double * wk = L + (long long)t * (t + 1) / 2;   // work space
    double * w = wk, * grad = wk + t, * y = wk + 2 * t;
    int * ord = reinterpret_cast<int *>(wk + 3 * t);        // P in insertion order
    extern __shared__ unsigned char inP[];                  // [max_t]
    const int lane = threadIdx.x;
    const int max_iter = P.nnls_max_iter;
    for (int i = lane; i < t; i += 32) { w[i] = 0.0; grad[i] = -c[i]; inP[i] = 0; }
    __syncwarp();
    int p = 0;
    for (int outer = 0; outer < max_iter; outer++) {
        // entering variable: first index of the largest positive dual
        float best = 0.0f;
        int bi = -1;
        for (int i = lane; i < t; i += 32) {
            float dual = (float)(-grad[i]);
            if (!inP[i] && dual > best) { best = dual; bi = i; }
        }
        for (int o = 16; o; o >>= 1) {
            float b2 = __shfl_xor_sync(0xffffffffu, best, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (b2 > best || (b2 == best && i2 >= 0 && (bi < 0 || i2 < bi))) { best = b2; bi = i2; }
        }
        if (bi < 0 || best < 1e-10f) break;
        if (lane == 0) { inP[bi] = 1; ord[p] = bi; }
        __syncwarp();
        chol_append(L, A, t, ord, p, bi, 1e-10);
        p++;
        for (int inner = 0; inner < max_iter; inner++) {
            for (int m = lane; m < p; m += 32) y[m] = c[ord[m]];
            __syncwarp();
            chol_solve(L, y, p);                        // y[m] = s at variable ord[m]
            bool feas = true;
            for (int m = lane; m < p; m += 32) if (!(y[m] > 0.0)) feas = false;
            feas = __all_sync(0xffffffffu, feas);
            if (feas) {
                for (int i = lane; i < t; i += 32) w[i] = 0.0;
                __syncwarp();
                for (int m = lane; m < p; m += 32) w[ord[m]] = y[m];
                __syncwarp();
                break;
            }
            double alpha = 1.0;
            for (int m = lane; m < p; m += 32) {
                const int k = ord[m];
                if (y[m] <= 0.0) {
                    double a = w[k] / (w[k] - y[m] + 1e-30);
                    if (a < alpha) alpha = a;
                }
            }
            for (int o = 16; o; o >>= 1) alpha = fmin(alpha, __shfl_xor_sync(0xffffffffu, alpha, o));
            // w += alpha (s - w); variables outside P have s = w = 0
            for (int m = lane; m < p; m += 32) {
                const int k = ord[m];
                w[k] += alpha * (y[m] - w[k]);
            }
            __syncwarp();
            // drop near-zero variables, keep the survivors' order, rebuild L
            int np = 0;
            for (int m = 0; m < p; m++) {
                const int k = ord[m];
                const bool keep = fabs(w[k]) >= 1e-12;
                if (!keep) {
                    if (lane == 0) { w[k] = 0.0; inP[k] = 0; }
                } else {
                    if (lane == 0) ord[np] = k;
                    np++;
                }
                __syncwarp();
            }
            if (np != p) {
                p = np;
                for (int m = 0; m < p; m++) chol_append(L, A, t, ord, m, ord[m], 1e-10);
            }
        }
        // grad = A w - c
        for (int i = 0; i < t; i++) {
            double part = 0.0;
            for (int k = lane; k < t; k += 32) part = fma(A[(long long)i * t + k], w[k], part);
            double s = warp_sum_d(part);
            if (lane == 0) grad[i] = s - c[i];
        }
        __syncwarp();
    }
    const kvc_layer_out lo = outs[u.layer];
    float * beta = lo.beta + (long long)h * lo.t_total + u.out_off;
    for (int i = lane; i < t; i += 32) {
        float wf = (float)w[i];
        if (wf < 1e-12f) wf = 1e-12f;
        beta[i] = logf(wf > 1e-12f ? wf : 1e-12f);
    }
    (void)max_t;
}

// nnls_method 1: clamped ridge least squares + optional projected gradient.
__global__ void __launch_bounds__(32) k_nnls_pgd(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                 const float * __restrict__ fs, double * __restrict__ gs,
                                                 const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    const int h = blockIdx.y, t = u.t, nq = u.nq;
    const long long stride = (long long)kvc_nnls_stride(t, nq);
    const double * A = gs + u.g_off + (long long)h * stride;
    const double * c = A + (long long)t * t;
    double * L = const_cast<double *>(c) + t;
    double * wk = L + (long long)t * (t + 1) / 2;
    double * w = wk, * g = wk + t, * uu = wk + 2 * t, * vv = wk + 4 * t;
    int * ord = reinterpret_cast<int *>(wk + 3 * t);
    const int lane = threadIdx.x;
    const double eps = 1e-12;
    for (int i = lane; i < t; i += 32) ord[i] = i;
    __syncwarp();
    for (int m = 0; m < t; m++) chol_append(L, A, t, ord, m, m, 1e-10);
    for (int i = lane; i < t; i += 32) w[i] = c[i];
    __syncwarp();
    chol_solve(L, w, t);
    for (int i = lane; i < t; i += 32) {
        const double * Li = L + (long long)i * (i + 1) / 2;
        if (!(Li[i] > 0.0)) w[i] = eps;             // singular pivot -> eps, as the reference
        if (w[i] < eps) w[i] = eps;
    }
    __syncwarp();
    if (P.nnls_pgd_iters > 0) {
        // step 1/L with L = u^T A u, u from 3 power iterations on M (math.h:754-790)
        const float * S = sraw(u, fs, h);
        const float * rmax = fs + u.row_off + (long long)h * 2 * nq;
        for (int i = lane; i < t; i += 32) uu[i] = 1.0 / sqrt((double)t);
        __syncwarp();
        for (int pw = 0; pw < 3; pw++) {
            for (int q = 0; q < nq; q++) {              // v = M u
                double part = 0.0;
                for (int j = lane; j < t; j += 32)
                    part = fma((double)expf(__fsub_rn(S[(long long)q * t + j], rmax[q])), uu[j], part);
                const double sq = warp_sum_d(part);
                if (lane == 0) vv[q] = sq;
            }
            __syncwarp();
            double part = 0.0;
            for (int q = lane; q < nq; q += 32) part = fma(vv[q], vv[q], part);
            const double vn = sqrt(warp_sum_d(part));
            if (vn < 1e-12) break;
            for (int q = lane; q < nq; q += 32) vv[q] /= vn;
            __syncwarp();
            for (int j = lane; j < t; j += 32) {        // u = M^T v
                double acc = 0.0;
                for (int q = 0; q < nq; q++)
                    acc = fma((double)expf(__fsub_rn(S[(long long)q * t + j], rmax[q])), vv[q], acc);
                uu[j] = acc;
            }
            __syncwarp();
            part = 0.0;
            for (int j = lane; j < t; j += 32) part = fma(uu[j], uu[j], part);
            const double un = sqrt(warp_sum_d(part));
            if (un < 1e-12) break;
            for (int j = lane; j < t; j += 32) uu[j] /= un;
            __syncwarp();
        }
        double Lest = 0.0;
        for (int i = 0; i < t; i++) {
            double part = 0.0;
            for (int k = lane; k < t; k += 32) part = fma(A[(long long)i * t + k], uu[k], part);
            Lest = fma(uu[i], warp_sum_d(part), Lest);
        }
        if (Lest < 1e-6) Lest = 1e-6;
        const double eta = 1.0 / Lest;
        for (int it = 0; it < P.nnls_pgd_iters; it++) {
            for (int i = 0; i < t; i++) {
                double part = 0.0;
                for (int k = lane; k < t; k += 32) part = fma(A[(long long)i * t + k], w[k], part);
                const double sg = warp_sum_d(part);
                if (lane == 0) g[i] = sg - c[i];
            }
            __syncwarp();
            for (int i = lane; i < t; i += 32) {
                const double v = w[i] - eta * g[i];
                w[i] = v < eps ? eps : v;
            }
            __syncwarp();
        }
    }
    const kvc_layer_out lo = outs[u.layer];
    float * beta = lo.beta + (long long)h * lo.t_total + u.out_off;
    for (int i = lane; i < t; i += 32) {
        float wf = (float)w[i];
        beta[i] = logf(wf > 1e-12f ? wf : 1e-12f);
    }
}

// Worst-key swap, one CTA per unit (see the file header).
__global__ void __launch_bounds__(256) k_refine(kvc_unit * __restrict__ units, kvc_params_dev P,
                                                const float * __restrict__ fs, int * __restrict__ is,
                                                const kvc_layer_out * __restrict__ outs) {
    kvc_unit & U = units[blockIdx.x];
    const kvc_unit u = U;
    if (!u.active) return;
    const int t = u.t, C = u.C, nq = u.nq;
    __shared__ float rv[32];
    __shared__ int ri[32];
    __shared__ int s_worst, s_best, s_stop;
    if (t >= C) { if (threadIdx.x == 0) U.active = 0; return; }
    int * sel = is + u.sel_off;
    int * flags = is + u.c_off;
    const float * gimp = fs + u.imp_off + (long long)2 * P.H * C;
    const float inv_nq = 1.0f;
    (void)inv_nq;
    // key value and first minimum
    float bv = INFINITY;
    int bi = 0x7fffffff;
    for (int j = threadIdx.x; j < t; j += blockDim.x) {
        float kv = 0.0f;
        for (int h = 0; h < P.H; h++) {
            const float * X = fs + u.x_off + (long long)h * nq * t;
            float e = 0.0f;
            for (int q = 0; q < nq; q++) { float x = X[(long long)q * t + j]; e = __fadd_rn(e, __fmul_rn(x, x)); }
            kv = __fadd_rn(kv, __fdiv_rn(e, (float)nq));
        }
        if (kv < bv) { bv = kv; bi = j; }
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int o = 16; o; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (v2 < bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; }
    }
    if (lane == 0) { rv[w] = bv; ri[w] = bi; }
    for (int j = threadIdx.x; j < C; j += blockDim.x) flags[j] = 0;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = rv[0];
        int i = ri[0];
        for (int k = 1; k < nw; k++) if (rv[k] < b || (rv[k] == b && ri[k] < i)) { b = rv[k]; i = ri[k]; }
        s_worst = i;
    }
    for (int j = threadIdx.x; j < t; j += blockDim.x) flags[sel[j]] = 1;
    __syncthreads();
    // best unused: first maximum importance outside the kept set (> -1)
    float gb = -1.0f;
    int gi = 0x7fffffff;
    for (int j = threadIdx.x; j < C; j += blockDim.x)
        if (!flags[j] && gimp[j] > gb) { gb = gimp[j]; gi = j; }
    for (int o = 16; o; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, gb, o);
        int i2 = __shfl_xor_sync(0xffffffffu, gi, o);
        if (v2 > gb || (v2 == gb && i2 < gi)) { gb = v2; gi = i2; }
    }
    __syncthreads();
    if (lane == 0) { rv[w] = gb; ri[w] = gi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = rv[0];
        int i = ri[0];
        for (int k = 1; k < nw; k++) if (rv[k] > b || (rv[k] == b && ri[k] < i)) { b = rv[k]; i = ri[k]; }
        const int worst_pos = sel[s_worst];
        s_best = (i == 0x7fffffff) ? -1 : i;
        s_stop = (s_best < 0) || !(b > __fmul_rn(gimp[worst_pos], 0.5f));
        if (!s_stop) {
            flags[worst_pos] = 0;
            flags[s_best] = 1;
        } else {
            U.active = 0;
        }
    }
    __syncthreads();
    if (s_stop) return;
    // emit the new kept set in ascending order
    const kvc_layer_out lo = outs[u.layer];
    __shared__ int sh[33];
    int base = 0;
    for (int j0 = 0; j0 < C; j0 += blockDim.x) {
        const int j = j0 + threadIdx.x;
        const int f = (j < C) ? flags[j] : 0;
        int x = f;
        for (int o = 1; o < 32; o <<= 1) { int y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
        __syncthreads();
        if (lane == 31) sh[w] = x;
        __syncthreads();
        if (w == 0) {
            int s = (lane < nw) ? sh[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) { int y = __shfl_up_sync(0xffffffffu, s, o); if (lane >= o) s += y; }
            if (lane < nw) sh[lane] = s;
        }
        __syncthreads();
        const int pos = base + ((w > 0) ? sh[w - 1] : 0) + x - f;
        const int tot = sh[nw - 1];
        if (f && pos < t) {
            sel[pos] = j;
            lo.sel[u.out_off + pos] = u.token_base + j;
        }
        base += tot;
        __syncthreads();
    }
}

size_t kvc_nnls_doubles_per_head(int t, int nq) { return (size_t)kvc_nnls_stride(t, nq); }

int kvc_launch_beta(const kvc_unit * d_units, int n_units, int max_nq, int max_t, const kvc_params_dev & P,
                    float * fs, int * is, double * gs, const kvc_layer_out * d_outs, cudaStream_t st) {
    (void)max_nq;
    (void)is;
    if (n_units <= 0) return KVC_OK;
    const int tn = (max_t + NT - 1) / NT;
    k_nnls_gram<<<dim3(tn * tn + 1, P.H, n_units), 256, 0, st>>>(d_units, P, fs, gs);
    KVC_CUDA(cudaGetLastError());
    if (P.nnls_method == 0) {
        k_nnls_lh<<<dim3(n_units, P.H), 32, (size_t)max_t, st>>>(d_units, P, gs, d_outs, max_t);
    } else {
        k_nnls_pgd<<<dim3(n_units, P.H), 32, 0, st>>>(d_units, P, fs, gs, d_outs);
    }
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_refine(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs,
                      int * is, const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    k_refine<<<n_units, 256, 0, st>>>(const_cast<kvc_unit *>(d_units), P, fs, is, d_outs);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
