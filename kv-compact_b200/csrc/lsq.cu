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
constexpr int FN = 128;   // max unknowns of the shared-memory path (k_lsq_factor)
constexpr int FC = 8;     // right-hand-side columns per warp in k_lsq_factor (16 warps)
}

enum { DG_GRAM = 0, DG_RHS = 1, DG_OUT = 2 };
constexpr int DT = 64, DK = 8;

// One 64x64 tile of C = A B per CTA of 64 threads for the (unit, head, mode)
// problem. Thread (ty, tx) of the 8x8 grid owns rows 2ty + 16i + {0,1} and
// columns 2tx + 16j + {0,1} (i, j < 4): per k step it reads four double2 of
// A and four of B from shared memory for 64 DFMA, and the double2 reads of a
// quarter-warp cover 128 contiguous bytes. Shared tiles are double-buffered;
// the next k slab is fetched into registers while the current one is used.
__global__ void __launch_bounds__(64) k_dgemm(const kvc_unit * __restrict__ units, kvc_params_dev P,
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

    __shared__ __align__(16) double As[2][DK][DT];
    __shared__ __align__(16) double Bs[2][DK][DT];
    const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
    const bool rows = (mode == DG_GRAM && dual);     // operands are rows of X (k contiguous)
    // thread tid fetches row/column tid of the tile for the DK k values of a
    // slab (conflict-free shared stores; `rows` operands read DK consecutive
    // floats of one row per thread, which L1 coalesces across the slab)
    double ra[DK], rb[DK];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int r = 0; r < DK; r++) {
            const int m = m0 + tid, c = n0 + tid, k = k0 + r;
            double va = 0.0, vb = 0.0;
            if (k < K) {
                if (m < M) va = rows ? (double)X[(long long)m * t + k] : (double)X[(long long)k * t + m];
                if (c < N) {
                    if (mode == DG_GRAM) vb = dual ? (double)X[(long long)c * t + k] : (double)X[(long long)k * t + c];
                    else if (mode == DG_RHS) vb = (double)Y[(long long)k * dv + c];
                    else vb = Z[(long long)k * dv + c];
                }
            }
            ra[r] = va;
            rb[r] = vb;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int r = 0; r < DK; r++) {
            As[buf][r][tid] = ra[r];
            Bs[buf][r][tid] = rb[r];
        }
    };
    double acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0;
    fetch(0);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += DK) {
        const bool more = k0 + DK < K;
        if (more) fetch(k0 + DK);
#pragma unroll
        for (int kk = 0; kk < DK; kk++) {
            double av[8], bv[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const double2 a2 = *reinterpret_cast<const double2 *>(&As[buf][kk][2 * ty + 16 * i]);
                const double2 b2 = *reinterpret_cast<const double2 *>(&Bs[buf][kk][2 * tx + 16 * i]);
                av[2 * i] = a2.x; av[2 * i + 1] = a2.y;
                bv[2 * i] = b2.x; bv[2 * i + 1] = b2.y;
            }
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        if (more) stash(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
    auto row_of = [&](int i) { return m0 + 2 * ty + 16 * (i >> 1) + (i & 1); };
    auto col_of = [&](int j) { return n0 + 2 * tx + 16 * (j >> 1) + (j & 1); };
    if (mode == DG_GRAM) {
        double * G = gs + u.g_off + (long long)h * n * n;
        const double ridge = (double)P.ridge;
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int a = row_of(i), b = col_of(j);
                if (a < n && b < n && b <= a) {
                    const double v = acc[i][j] + (a == b ? ridge : 0.0);
                    G[(long long)a * n + b] = v;
                    G[(long long)b * n + a] = v;
                }
            }
    } else if (mode == DG_RHS) {
        double * R = gs + u.z_off + (long long)h * n * dv;
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int a = row_of(i), c = col_of(j);
                if (a < M && c < N) R[(long long)a * dv + c] = acc[i][j];
            }
    } else {
        const kvc_layer_out lo = outs[u.layer];
        float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int a = row_of(i), c = col_of(j);
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
// warp-synchronously with reciprocal pivots, the solved row of each step
// broadcast to the warp through a shared-memory slot. The result Z (dual, consumed by
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
    // thread derives the pivot and its reciprocal itself from one rsqrt (no
    // extra barrier); the scaled column goes to colk first so the rank-1
    // update never reads a column entry another thread is rewriting. The
    // update of the lower trailing triangle gives row i to warp (i mod 16)
    // and its columns to the lanes (contiguous, conflict-free). Two barriers
    // per column.
    double * colk = rinv + FN;                     // [n]
    const int nwarp = nthr >> 5;
    for (int k = 0; k < n; k++) {
        const double d = G[k * ld + k];
        const bool pos = d > 0.0 && isfinite(d);
        const double il = pos ? rsqrt(d) : 0.0;
        for (int i = k + 1 + tid; i < n; i += nthr) colk[i] = G[i * ld + k] * il;
        if (tid == 0) rinv[k] = il;
        __syncthreads();                           // every thread has read the pivot
        if (tid == 0) G[k * ld + k] = pos ? d * il : 0.0;
        for (int i = k + 1 + warp; i < n; i += nwarp) {
            const double ci = colk[i];
            double * Gi = G + i * ld;
            for (int j = k + 1 + lane; j <= i; j += 32) Gi[j] -= ci * colk[j];
            if (lane == 0) Gi[k] = ci;
        }
        __syncthreads();
    }

    const int c0 = warp * FC;
    double * zb = colk + FN + warp * FC;           // this warp's broadcast slot
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
            if (lane == kk) {
                const double il = rinv[k];
#pragma unroll
                for (int c = 0; c < FC; c++) {
                    b[S][c] *= il;
                    zb[c] = b[S][c];
                }
            }
            __syncwarp();
            double z[FC];
#pragma unroll
            for (int c = 0; c < FC; c += 2) {
                const double2 v = *reinterpret_cast<const double2 *>(zb + c);
                z[c] = v.x;
                z[c + 1] = v.y;
            }
            __syncwarp();
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
            if (lane == kk) {
                const double il = rinv[k];
#pragma unroll
                for (int c = 0; c < FC; c++) {
                    b[S][c] *= il;
                    zb[c] = b[S][c];
                }
            }
            __syncwarp();
            double z[FC];
#pragma unroll
            for (int c = 0; c < FC; c += 2) {
                const double2 v = *reinterpret_cast<const double2 *>(zb + c);
                z[c] = v.x;
                z[c + 1] = v.y;
            }
            __syncwarp();
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
    k_dgemm<<<dim3(tg * tg, P.H, n_units), 64, 0, st>>>(d_units, P, fs, gs, d_outs, DG_GRAM);
    KVC_CUDA(cudaGetLastError());
    const int to = ((max_t + DT - 1) / DT) * ((P.dv + DT - 1) / DT);
    k_dgemm<<<dim3(to, P.H, n_units), 64, 0, st>>>(d_units, P, fs, gs, d_outs, DG_RHS);
    KVC_CUDA(cudaGetLastError());
    const size_t fast_smem = (size_t)(FN * (FN + 1) + 2 * FN + 16 * FC) * sizeof(double);
    KVC_CUDA(cudaFuncSetAttribute(k_lsq_factor, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fast_smem));
    k_lsq_factor<<<dim3(n_units, P.H), 512, fast_smem, st>>>(d_units, P, fs, gs, d_outs);
    KVC_CUDA(cudaGetLastError());
    k_dgemm<<<dim3(to, P.H, n_units), 64, 0, st>>>(d_units, P, fs, gs, d_outs, DG_OUT);
    KVC_CUDA(cudaGetLastError());
    if (max_n > FN || P.dv > FN) {
        KVC_CUDA(cudaFuncSetAttribute(k_chol_solve, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
        k_chol_solve<<<dim3(n_units, P.H), 256, smem_bytes, st>>>(d_units, P, fs, gs, d_outs);
        KVC_CUDA(cudaGetLastError());
    }
    return KVC_OK;
}
