// lsq.cu — value refit C_v = argmin ||X C - Y||^2 + ridge ||C||^2 per (unit, head).
//
// The reference solves the primal normal equations (X^T X + ridge I) C = X^T Y
// by fp32 Gaussian elimination (include/kv-compact-math.h:463-557). With
// n_q < t the primal matrix has rank <= n_q, so its smallest t - n_q
// eigenvalues equal the ridge (1e-6) and fp32 rounding in those directions is
// amplified ~1e6x: the reference's C_v carries noise of ~1e-2 relative in the
// null space of X. This stage solves the same ridge problem accurately:
//   * t <= n_q: primal,  G = X^T X + ridge I  [t x t],  C = G^-1 X^T Y
//   * n_q < t:  dual,    G = X X^T + ridge I  [n_q x n_q], C = X^T G^-1 Y
//     (identical in exact arithmetic: (X^T X + rI)^-1 X^T = X^T (X X^T + rI)^-1)
// with the Gram matrix accumulated in fp64 from the fp32 X (products of two
// fp32 values are exact in fp64), an fp64 Cholesky factorisation and fp64
// triangular solves. A non-positive pivot marks its unknown singular and
// zeroes it, the counterpart of the reference skipping pivots below 1e-12.
//
// The dense products run as one batched fp64 GEMM launch each (k_dgemm,
// 64x64 tiles, 4x4 per thread, over every (unit, head)):
//   GRAM  G = X X^T (dual) or X^T X (primal), + ridge on the diagonal
//   RHS   R = X^T Y                          (primal only)
//   OUT   C_v = X^T Z                        (dual only)
// and the latency-bound part runs one CTA per (unit, head):
//   k_lsq_factor  Cholesky of G in shared memory (n <= 128) + both triangular
//                 solves for all d_v right-hand sides in registers; writes Z
//                 (dual) or C_v (primal).
//   k_chol_solve  the same for n > 128 or d_v > 128, G in global memory.
#include "kvc_internal.h"

#include <math.h>

namespace {
constexpr int GT = 32;
constexpr int FN = 128;   // max unknowns of the shared-memory path (k_lsq_factor)
constexpr int FC = 8;     // right-hand-side columns per warp in k_lsq_factor (16 warps)
}

enum { DG_GRAM = 0, DG_RHS = 1, DG_OUT = 2 };
constexpr int DT = 64, DK = 16;

// One 64x64 tile of C = A B per CTA for the (unit, head, mode) problem.
__global__ void __launch_bounds__(256) k_dgemm(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                               const float * __restrict__ fs, double * __restrict__ gs,
                                               const kvc_layer_out * __restrict__ outs, int mode) {
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y;
    const int nq = u.nq, t = u.t, dv = P.dv;
    const bool dual = nq < t;
    const int n = dual ? nq : t;
    if ((mode == DG_RHS && dual) || (mode == DG_OUT && !dual)) return;
    if (mode != DG_GRAM && (n > FN || dv > FN)) return;     // k_chol_solve does its own
    int M, N, K;
    if (mode == DG_GRAM) { M = n; N = n; K = dual ? t : nq; }
    else { M = t; N = dv; K = nq; }
    const int tn = (N + DT - 1) / DT, tm = (M + DT - 1) / DT;
    if ((int)blockIdx.x >= tm * tn) return;
    const int m0 = (blockIdx.x / tn) * DT, n0 = (blockIdx.x % tn) * DT;
    if (mode == DG_GRAM && n0 > m0) return;          // lower tiles; mirrored on store
    const float * X = fs + u.x_off + (long long)h * nq * t;
    const float * Y = fs + u.y_off + (long long)h * nq * dv;
    const double * Z = gs + u.z_off + (long long)h * n * dv;

    __shared__ __align__(16) double As[DK][DT + 2];
    __shared__ __align__(16) double Bs[DK][DT + 2];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const bool rows = (mode == DG_GRAM && dual);     // operands are rows of X (k contiguous)
    double acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
    for (int k0 = 0; k0 < K; k0 += DK) {
        for (int e = tid; e < DT * DK; e += 256) {
            int mm, kk;
            if (rows) { mm = e / DK; kk = e % DK; } else { kk = e / DT; mm = e % DT; }
            const int m = m0 + mm, k = k0 + kk;
            double v = 0.0;
            if (m < M && k < K) v = rows ? (double)X[(long long)m * t + k] : (double)X[(long long)k * t + m];
            As[kk][mm] = v;
        }
        for (int e = tid; e < DT * DK; e += 256) {
            int nn, kk;
            if (rows) { nn = e / DK; kk = e % DK; } else { kk = e / DT; nn = e % DT; }
            const int c = n0 + nn, k = k0 + kk;
            double v = 0.0;
            if (c < N && k < K) {
                if (mode == DG_GRAM) v = dual ? (double)X[(long long)c * t + k] : (double)X[(long long)k * t + c];
                else if (mode == DG_RHS) v = (double)Y[(long long)k * dv + c];
                else v = Z[(long long)k * dv + c];
            }
            Bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < DK; kk++) {
            const double2 a01 = *reinterpret_cast<const double2 *>(&As[kk][ty * 4]);
            const double2 a23 = *reinterpret_cast<const double2 *>(&As[kk][ty * 4 + 2]);
            const double2 b01 = *reinterpret_cast<const double2 *>(&Bs[kk][tx * 4]);
            const double2 b23 = *reinterpret_cast<const double2 *>(&Bs[kk][tx * 4 + 2]);
            const double av[4] = {a01.x, a01.y, a23.x, a23.y};
            const double bv[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
    if (mode == DG_GRAM) {
        double * G = gs + u.g_off + (long long)h * n * n;
        const double ridge = (double)P.ridge;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int a = m0 + ty * 4 + i, b = n0 + tx * 4 + j;
                if (a < n && b < n && b <= a) {
                    const double v = acc[i][j] + (a == b ? ridge : 0.0);
                    G[(long long)a * n + b] = v;
                    G[(long long)b * n + a] = v;
                }
            }
    } else if (mode == DG_RHS) {
        double * R = gs + u.z_off + (long long)h * n * dv;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int a = m0 + ty * 4 + i, c = n0 + tx * 4 + j;
                if (a < M && c < N) R[(long long)a * dv + c] = acc[i][j];
            }
    } else {
        const kvc_layer_out lo = outs[u.layer];
        float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int a = m0 + ty * 4 + i, c = n0 + tx * 4 + j;
                if (a < M && c < N) cv[(long long)a * dv + c] = (float)acc[i][j];
            }
    }
}

// Panel width for n unknowns: keeps the n x PW fp64 panel within 96 KB.
__host__ __device__ inline int lsq_panel(int n) { return n <= 384 ? 32 : (n <= 1536 ? 8 : 4); }

__global__ void __launch_bounds__(256) k_chol_solve(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                    const float * __restrict__ fs, double * __restrict__ gs,
                                                    const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    const int h = blockIdx.y;
    const int nq = u.nq, t = u.t, dv = P.dv;
    const bool dual = nq < t;
    const int n = dual ? nq : t;
    if (n <= FN && dv <= FN) return;           // handled by k_lsq_factor
    const int PW = lsq_panel(n);
    const float * X = fs + u.x_off + (long long)h * nq * t;
    const float * Y = fs + u.y_off + (long long)h * nq * dv;
    const kvc_layer_out lo = outs[u.layer];
    float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
    double * Gg = gs + u.g_off + (long long)h * n * n;

    extern __shared__ double sm[];
    const bool g_in_smem = n <= 128;
    double * G = g_in_smem ? sm : Gg;
    double * B = g_in_smem ? sm + (size_t)n * n : sm;        // [n][PW]
    __shared__ double s_piv;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;

    if (g_in_smem)
        for (int e = tid; e < n * n; e += nt) G[e] = Gg[e];
    __syncthreads();

    // ---- Cholesky, lower triangle in place (row-major, G[i*n+j], j <= i)
    for (int k = 0; k < n; k++) {
        if (tid == 0) {
            double d = G[(long long)k * n + k];
            double l = (d > 0.0 && isfinite(d)) ? sqrt(d) : 0.0;
            G[(long long)k * n + k] = l;
            s_piv = l;
        }
        __syncthreads();
        const double l = s_piv;
        for (int i = k + 1 + tid; i < n; i += nt)
            G[(long long)i * n + k] = (l > 0.0) ? G[(long long)i * n + k] / l : 0.0;
        __syncthreads();
        for (int i = k + 1 + warp; i < n; i += nw) {
            const double lik = G[(long long)i * n + k];
            for (int j = k + 1 + lane; j <= i; j += 32)
                G[(long long)i * n + j] -= lik * G[(long long)j * n + k];
        }
        __syncthreads();
    }

    for (int c0 = 0; c0 < dv; c0 += PW) {
        const int pw = min(PW, dv - c0);
        // ---- right-hand side panel
        if (dual) {
            for (int e = tid; e < n * PW; e += nt) {
                int a = e / PW, c = e % PW;
                B[e] = (c < pw) ? (double)Y[(long long)a * dv + c0 + c] : 0.0;
            }
        } else {
            for (int e = tid; e < n * PW; e += nt) {
                int a = e / PW, c = e % PW;
                double acc = 0.0;
                if (c < pw)
                    for (int q = 0; q < nq; q++)
                        acc = fma((double)X[(long long)q * t + a], (double)Y[(long long)q * dv + c0 + c], acc);
                B[e] = acc;
            }
        }
        __syncthreads();
        // ---- forward: L w = b
        for (int k = 0; k < n; k++) {
            const double l = G[(long long)k * n + k];
            if (tid < PW) B[k * PW + tid] = (l > 0.0) ? B[k * PW + tid] / l : 0.0;
            __syncthreads();
            for (int e = tid; e < (n - k - 1) * PW; e += nt) {
                int i = k + 1 + e / PW, c = e % PW;
                B[i * PW + c] -= G[(long long)i * n + k] * B[k * PW + c];
            }
            __syncthreads();
        }
        // ---- backward: L^T z = w
        for (int k = n - 1; k >= 0; k--) {
            const double l = G[(long long)k * n + k];
            if (tid < PW) B[k * PW + tid] = (l > 0.0) ? B[k * PW + tid] / l : 0.0;
            __syncthreads();
            for (int e = tid; e < k * PW; e += nt) {
                int i = e / PW, c = e % PW;
                B[i * PW + c] -= G[(long long)k * n + i] * B[k * PW + c];
            }
            __syncthreads();
        }
        // ---- output
        if (dual) {
            for (int e = tid; e < t * pw; e += nt) {
                int j = e / pw, c = e % pw;
                double acc = 0.0;
                for (int a = 0; a < nq; a++)
                    acc = fma((double)X[(long long)a * t + j], B[a * PW + c], acc);
                cv[(long long)j * dv + c0 + c] = (float)acc;
            }
        } else {
            for (int e = tid; e < n * pw; e += nt) {
                int a = e / pw, c = e % pw;
                cv[(long long)a * dv + c0 + c] = (float)B[a * PW + c];
            }
        }
        __syncthreads();
    }
}


// ---------------------------------------------------------------------------
// Factor + solve, n = min(n_q, t) <= 128 and d_v <= 128, one CTA of 16 warps
// per (unit, head). G (fp64, from k_dgemm) is copied to shared memory with an
// odd row stride so column walks hit distinct banks, and factorised with a
// right-looking Cholesky whose steps are spread over all 16 warps. The
// right-hand sides (Y for the dual, X^T Y from
// k_dgemm for the primal) stay in registers: warp w owns columns [8w, 8w+8),
// lane l rows l, l+32, l+64, l+96, and both triangular solves run
// warp-synchronously with reciprocal pivots. The result Z (dual, consumed by
// the OUT GEMM) or C_v (primal) is written to global memory.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512, 1) k_lsq_factor(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                       const float * __restrict__ fs, double * __restrict__ gs,
                                                       const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    const int nq = u.nq, t = u.t, dv = P.dv;
    const bool dual = nq < t;
    const int n = dual ? nq : t;
    if (n > FN || dv > FN) return;            // handled by k_chol_solve
    const int h = blockIdx.y;
    const float * Y = fs + u.y_off + (long long)h * nq * dv;
    const double * Gg = gs + u.g_off + (long long)h * n * n;
    double * Zg = gs + u.z_off + (long long)h * n * dv;        // primal: holds X^T Y on entry

    extern __shared__ double G[];
    const int ld = n + 1;
    double * rinv = G + n * ld;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
    for (int e = tid; e < n * n; e += nthr) G[(e / n) * ld + (e % n)] = Gg[e];
    __syncthreads();

    // Right-looking Cholesky, every step parallel over the whole CTA. Each
    // thread derives the pivot reciprocal itself (no extra barrier); the
    // scaled column goes to colk first so the rank-1 update never reads a
    // column entry another thread is rewriting. Two barriers per column.
    double * colk = rinv + FN;                     // [n]
    for (int k = 0; k < n; k++) {
        const double d = G[k * ld + k];
        const double l = (d > 0.0 && isfinite(d)) ? sqrt(d) : 0.0;
        const double il = (l > 0.0) ? 1.0 / l : 0.0;
        for (int i = k + 1 + tid; i < n; i += nthr) colk[i] = G[i * ld + k] * il;
        if (tid == 0) rinv[k] = il;
        __syncthreads();                           // every thread has read the pivot
        if (tid == 0) G[k * ld + k] = l;
        const int m = n - k - 1;                   // trailing size
        for (int e = tid; e < m * m; e += nthr) {
            const int i = k + 1 + e / m, j = k + 1 + e % m;
            if (j <= i) G[i * ld + j] -= colk[i] * colk[j];
        }
        for (int i = k + 1 + tid; i < n; i += nthr) G[i * ld + k] = colk[i];
        __syncthreads();
    }

    const int c0 = warp * FC;
    double b[4][FC];
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int r = lane + 32 * s;
#pragma unroll
        for (int c = 0; c < FC; c++) {
            double v = 0.0;
            if (r < n && c0 + c < dv) v = dual ? (double)Y[(long long)r * dv + c0 + c] : Zg[(long long)r * dv + c0 + c];
            b[s][c] = v;
        }
    }
#pragma unroll
    for (int S = 0; S < 4; S++) {
        for (int kk = 0; kk < 32; kk++) {
            const int k = 32 * S + kk;
            if (k >= n) break;
            const double il = rinv[k];
            double z[FC];
#pragma unroll
            for (int c = 0; c < FC; c++) z[c] = __shfl_sync(0xffffffffu, b[S][c] * il, kk);
            if (lane == kk) {
#pragma unroll
                for (int c = 0; c < FC; c++) b[S][c] = z[c];
            }
#pragma unroll
            for (int s2 = S; s2 < 4; s2++) {
                const int r = lane + 32 * s2;
                if (r > k && r < n) {
                    const double l = G[r * ld + k];
#pragma unroll
                    for (int c = 0; c < FC; c++) b[s2][c] -= l * z[c];
                }
            }
        }
    }
#pragma unroll
    for (int S = 3; S >= 0; S--) {
        for (int kk = 31; kk >= 0; kk--) {
            const int k = 32 * S + kk;
            if (k >= n) continue;
            const double il = rinv[k];
            double z[FC];
#pragma unroll
            for (int c = 0; c < FC; c++) z[c] = __shfl_sync(0xffffffffu, b[S][c] * il, kk);
            if (lane == kk) {
#pragma unroll
                for (int c = 0; c < FC; c++) b[S][c] = z[c];
            }
#pragma unroll
            for (int s2 = 0; s2 <= S; s2++) {
                const int r = lane + 32 * s2;
                if (r < k) {
                    const double l = G[k * ld + r];
#pragma unroll
                    for (int c = 0; c < FC; c++) b[s2][c] -= l * z[c];
                }
            }
        }
    }
    if (dual) {
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int r = lane + 32 * s;
            if (r >= n) continue;
#pragma unroll
            for (int c = 0; c < FC; c++)
                if (c0 + c < dv) Zg[(long long)r * dv + c0 + c] = b[s][c];
        }
    } else {
        const kvc_layer_out lo = outs[u.layer];
        float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int r = lane + 32 * s;
            if (r >= n) continue;
#pragma unroll
            for (int c = 0; c < FC; c++)
                if (c0 + c < dv) cv[(long long)r * dv + c0 + c] = (float)b[s][c];
        }
    }
}

size_t kvc_lsq_smem_bytes(int n) {
    size_t pw = (size_t)lsq_panel(n);
    size_t b = (size_t)n * pw * sizeof(double);
    if (n <= 128) b += (size_t)n * n * sizeof(double);
    return b;
}

int kvc_launch_lsq(const kvc_unit * d_units, int n_units, int max_n, int max_t, size_t smem_bytes,
                   const kvc_params_dev & P, const float * fs, double * gs,
                   const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    const int tg = (max_n + DT - 1) / DT;
    k_dgemm<<<dim3(tg * tg, P.H, n_units), 256, 0, st>>>(d_units, P, fs, gs, d_outs, DG_GRAM);
    KVC_CUDA(cudaGetLastError());
    const int to = ((max_t + DT - 1) / DT) * ((P.dv + DT - 1) / DT);
    k_dgemm<<<dim3(to, P.H, n_units), 256, 0, st>>>(d_units, P, fs, gs, d_outs, DG_RHS);
    KVC_CUDA(cudaGetLastError());
    const size_t fast_smem = (size_t)(FN * (FN + 1) + 2 * FN) * sizeof(double);
    KVC_CUDA(cudaFuncSetAttribute(k_lsq_factor, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fast_smem));
    k_lsq_factor<<<dim3(n_units, P.H), 512, fast_smem, st>>>(d_units, P, fs, gs, d_outs);
    KVC_CUDA(cudaGetLastError());
    k_dgemm<<<dim3(to, P.H, n_units), 256, 0, st>>>(d_units, P, fs, gs, d_outs, DG_OUT);
    KVC_CUDA(cudaGetLastError());
    if (max_n > FN || P.dv > FN) {
        KVC_CUDA(cudaFuncSetAttribute(k_chol_solve, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
        k_chol_solve<<<dim3(n_units, P.H), 256, smem_bytes, st>>>(d_units, P, fs, gs, d_outs);
        KVC_CUDA(cudaGetLastError());
    }
    return KVC_OK;
}
