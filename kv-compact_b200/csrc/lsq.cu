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
// k_gram:       32x32 fp64 tiles of G, grid over all tiles of all (unit, head)
// k_chol_solve: one CTA per (unit, head); G in shared memory when n <= 128,
//               right-hand sides in panels of PW columns.
#include "kvc_internal.h"

#include <math.h>

namespace {
constexpr int GT = 32;
constexpr int FN = 128;   // max unknowns of the fast path (k_lsq_small)
constexpr int FC = 8;     // right-hand-side columns per warp in k_lsq_small (16 warps)
}

__global__ void __launch_bounds__(256) k_gram(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                              const float * __restrict__ fs, double * __restrict__ gs) {
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y;
    const int nq = u.nq, t = u.t;
    const bool dual = nq < t;
    const int n = dual ? nq : t, inner = dual ? t : nq;
    const int tn = (n + GT - 1) / GT;
    if ((int)blockIdx.x >= tn * tn) return;
    const int a0 = (blockIdx.x / tn) * GT, b0 = (blockIdx.x % tn) * GT;
    if (b0 > a0) return;                     // lower tiles only; mirrored on store
    const float * X = fs + u.x_off + (long long)h * nq * t;
    double * G = gs + u.g_off + (long long)h * n * n;
    __shared__ double As[GT][GT + 1];
    __shared__ double Bs[GT][GT + 1];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    double acc[2][2] = {{0, 0}, {0, 0}};
    for (int k0 = 0; k0 < inner; k0 += GT) {
        for (int e = tid; e < GT * GT; e += 256) {
            int r = e / GT, c = e % GT;       // r: operand index, c: inner offset
            int a = a0 + r, b = b0 + r, k = k0 + c;
            float xa = 0.0f, xb = 0.0f;
            if (k < inner) {
                if (dual) {
                    if (a < n) xa = X[(long long)a * t + k];
                    if (b < n) xb = X[(long long)b * t + k];
                } else {
                    if (a < n) xa = X[(long long)k * t + a];
                    if (b < n) xb = X[(long long)k * t + b];
                }
            }
            As[c][r] = (double)xa;
            Bs[c][r] = (double)xb;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < GT; kk++) {
            double x0 = As[kk][ty * 2], x1 = As[kk][ty * 2 + 1];
            double y0 = Bs[kk][tx * 2], y1 = Bs[kk][tx * 2 + 1];
            acc[0][0] = fma(x0, y0, acc[0][0]);
            acc[0][1] = fma(x0, y1, acc[0][1]);
            acc[1][0] = fma(x1, y0, acc[1][0]);
            acc[1][1] = fma(x1, y1, acc[1][1]);
        }
        __syncthreads();
    }
    const double ridge = (double)P.ridge;
    for (int i = 0; i < 2; i++)
        for (int j = 0; j < 2; j++) {
            int a = a0 + ty * 2 + i, b = b0 + tx * 2 + j;
            if (a < n && b < n && b <= a) {
                double v = acc[i][j] + (a == b ? ridge : 0.0);
                G[(long long)a * n + b] = v;
                G[(long long)b * n + a] = v;
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
    if (n <= FN && dv <= FN) return;           // handled by k_lsq_small
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
// Fast path: n = min(n_q, t) <= 128 and d_v <= 128, one CTA of 16 warps per
// (unit, head). G (fp64) lives in shared memory and is factorised with a
// 32-column blocked Cholesky (3 block-wide barriers per block column). The
// right-hand sides stay in registers: warp w owns columns [8w, 8w+8), lane l
// owns rows l, l+32, l+64, l+96, and both triangular solves run
// warp-synchronously (no block barriers). Z then replaces G in shared memory
// for the dual product C_v = X^T Z.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512, 1) k_lsq_small(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                      const float * __restrict__ fs, const double * __restrict__ gs,
                                                      const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    const int nq = u.nq, t = u.t, dv = P.dv;
    const bool dual = nq < t;
    const int n = dual ? nq : t;
    if (n > FN || dv > FN) return;            // handled by k_chol_solve
    const int h = blockIdx.y;
    const float * X = fs + u.x_off + (long long)h * nq * t;
    const float * Y = fs + u.y_off + (long long)h * nq * dv;
    const kvc_layer_out lo = outs[u.layer];
    float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
    const double * Gg = gs + u.g_off + (long long)h * n * n;

    extern __shared__ double G[];              // [n][n], later Z [n][dv]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < n * n; e += blockDim.x) G[e] = Gg[e];
    __syncthreads();

    // ---- blocked Cholesky, lower triangle, row-major G[i*n + j]
    for (int kb = 0; kb < n; kb += 32) {
        const int nb = min(32, n - kb);
        if (warp == 0) {
            for (int k = kb; k < kb + nb; k++) {
                double d = G[k * n + k];
                double l = (d > 0.0 && isfinite(d)) ? sqrt(d) : 0.0;
                __syncwarp();
                if (lane == 0) G[k * n + k] = l;
                const int i = kb + lane;
                if (i > k && i < kb + nb) G[i * n + k] = (l > 0.0) ? G[i * n + k] / l : 0.0;
                __syncwarp();
                if (i > k && i < kb + nb) {
                    const double lik = G[i * n + k];
                    for (int j = k + 1; j <= i; j++) G[i * n + j] -= lik * G[j * n + k];
                }
                __syncwarp();
            }
        }
        __syncthreads();
        // panel below the diagonal block: L_ik = (A_ik - sum_{m<k} L_im L_km) / L_kk
        for (int i = kb + nb + tid; i < n; i += blockDim.x) {
            for (int k = kb; k < kb + nb; k++) {
                double v = G[i * n + k];
                for (int m = kb; m < k; m++) v -= G[i * n + m] * G[k * n + m];
                const double l = G[k * n + k];
                G[i * n + k] = (l > 0.0) ? v / l : 0.0;
            }
        }
        __syncthreads();
        // trailing update of the lower triangle
        const int r0 = kb + nb, m = n - r0;
        for (int e = tid; e < m * m; e += blockDim.x) {
            const int i = r0 + e / m, j = r0 + e % m;
            if (j > i) continue;
            double v = G[i * n + j];
            for (int q = kb; q < kb + nb; q++) v -= G[i * n + q] * G[j * n + q];
            G[i * n + j] = v;
        }
        __syncthreads();
    }

    // ---- right-hand sides in registers
    const int c0 = warp * FC;
    double b[4][FC];
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int r = lane + 32 * s;
#pragma unroll
        for (int c = 0; c < FC; c++) {
            double v = 0.0;
            if (r < n && c0 + c < dv) {
                if (dual) {
                    v = (double)Y[(long long)r * dv + c0 + c];
                } else {
                    for (int q = 0; q < nq; q++)
                        v = fma((double)X[(long long)q * t + r], (double)Y[(long long)q * dv + c0 + c], v);
                }
            }
            b[s][c] = v;
        }
    }
    // ---- forward: L w = b. Row k = 32*S + kk lives in slot S of lane kk;
    // S is a compile-time loop index so b never needs dynamic indexing.
#pragma unroll
    for (int S = 0; S < 4; S++) {
        for (int kk = 0; kk < 32; kk++) {
            const int k = 32 * S + kk;
            if (k >= n) break;
            const double lkk = G[k * n + k];
            double z[FC];
#pragma unroll
            for (int c = 0; c < FC; c++) {
                const double v = (lkk > 0.0) ? b[S][c] / lkk : 0.0;
                z[c] = __shfl_sync(0xffffffffu, v, kk);
            }
            if (lane == kk) {
#pragma unroll
                for (int c = 0; c < FC; c++) b[S][c] = z[c];
            }
#pragma unroll
            for (int s2 = S; s2 < 4; s2++) {
                const int r = lane + 32 * s2;
                if (r > k && r < n) {
                    const double l = G[r * n + k];
#pragma unroll
                    for (int c = 0; c < FC; c++) b[s2][c] -= l * z[c];
                }
            }
        }
    }
    // ---- backward: L^T x = w
#pragma unroll
    for (int S = 3; S >= 0; S--) {
        for (int kk = 31; kk >= 0; kk--) {
            const int k = 32 * S + kk;
            if (k >= n) continue;
            const double lkk = G[k * n + k];
            double z[FC];
#pragma unroll
            for (int c = 0; c < FC; c++) {
                const double v = (lkk > 0.0) ? b[S][c] / lkk : 0.0;
                z[c] = __shfl_sync(0xffffffffu, v, kk);
            }
            if (lane == kk) {
#pragma unroll
                for (int c = 0; c < FC; c++) b[S][c] = z[c];
            }
#pragma unroll
            for (int s2 = 0; s2 <= S; s2++) {
                const int r = lane + 32 * s2;
                if (r < k) {
                    const double l = G[k * n + r];
#pragma unroll
                    for (int c = 0; c < FC; c++) b[s2][c] -= l * z[c];
                }
            }
        }
    }
    if (!dual) {
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int r = lane + 32 * s;
            if (r >= n) continue;
#pragma unroll
            for (int c = 0; c < FC; c++)
                if (c0 + c < dv) cv[(long long)r * dv + c0 + c] = (float)b[s][c];
        }
        return;
    }
    __syncthreads();                            // every warp is done with L
    double * Z = G;                             // [n][dv]
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int r = lane + 32 * s;
        if (r >= n) continue;
#pragma unroll
        for (int c = 0; c < FC; c++)
            if (c0 + c < dv) Z[r * dv + c0 + c] = b[s][c];
    }
    __syncthreads();
    // ---- C_v[j][cb:cb+16] = sum_a X[a][j] Z[a][cb:cb+16]
    const int nblk = (dv + 15) / 16;
    for (int e = tid; e < t * nblk; e += blockDim.x) {
        const int j = e % t, cb = (e / t) * 16;
        double acc[16];
#pragma unroll
        for (int c = 0; c < 16; c++) acc[c] = 0.0;
        for (int a = 0; a < nq; a++) {
            const double x = (double)X[(long long)a * t + j];
            const double * zr = Z + a * dv + cb;
#pragma unroll
            for (int c = 0; c < 16; c++) acc[c] = fma(x, zr[c < dv - cb ? c : 0], acc[c]);
        }
#pragma unroll
        for (int c = 0; c < 16; c++)
            if (cb + c < dv) cv[(long long)j * dv + cb + c] = (float)acc[c];
    }
}

size_t kvc_lsq_smem_bytes(int n) {
    size_t pw = (size_t)lsq_panel(n);
    size_t b = (size_t)n * pw * sizeof(double);
    if (n <= 128) b += (size_t)n * n * sizeof(double);
    return b;
}

int kvc_launch_lsq(const kvc_unit * d_units, int n_units, int max_n, size_t smem_bytes,
                   const kvc_params_dev & P, const float * fs, double * gs,
                   const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    int tn = (max_n + GT - 1) / GT;
    k_gram<<<dim3(tn * tn, P.H, n_units), 256, 0, st>>>(d_units, P, fs, gs);
    KVC_CUDA(cudaGetLastError());
    const size_t fast_smem = (size_t)FN * FN * sizeof(double);
    KVC_CUDA(cudaFuncSetAttribute(k_lsq_small, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fast_smem));
    k_lsq_small<<<dim3(n_units, P.H), 512, fast_smem, st>>>(d_units, P, fs, gs, d_outs);
    KVC_CUDA(cudaGetLastError());
    if (max_n > FN || P.dv > FN) {
        KVC_CUDA(cudaFuncSetAttribute(k_chol_solve, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
        k_chol_solve<<<dim3(n_units, P.H), 256, smem_bytes, st>>>(d_units, P, fs, gs, d_outs);
        KVC_CUDA(cudaGetLastError());
    }
    return KVC_OK;
}
