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
// fp32 values are exact in fp64) and an fp64 solve. A non-positive pivot marks
// its unknown singular and zeroes it, the counterpart of the reference
// skipping pivots below 1e-12.
//
// The dense products run as one batched fp64 GEMM launch each (k_dgemm on
// the fp64 tensor cores, 64x64 tiles, over every (unit, head)):
//   GRAM  G = X X^T (dual) or X^T X (primal), + ridge on the diagonal
//   RHS   R = X^T Y                          (primal only)
//   OUT   C_v = X^T Z                        (dual only)
// and the solve runs one CTA per (unit, head):
//   k_lsq_factor  block Gauss-Jordan elimination of [G | R] (four unknowns
//                 per step, rank-4 updates on the fp64 tensor cores) with G in
//                 shared memory and R in MMA fragments (n <= 128, d_v <= 128);
//                 writes Z (dual) or C_v (primal).
//   k_chol_solve  Cholesky + triangular solves for n > 128 or d_v > 128,
//                 G in global memory.
#include "kvc_internal.h"

#include <math.h>

namespace {
constexpr int FN = 128;   // max unknowns of the shared-memory path (k_lsq_factor)
}

enum { DG_GRAM = 0, DG_RHS = 1, DG_OUT = 2 };

// In-place inverse of a symmetric 4x4 block, read from its upper triangle,
// by its adjugate (cofactor expansion over the 2x2 minors of the top and
// bottom row pairs) divided by the determinant; only the ten distinct
// entries of the symmetric inverse are formed (the pivot blocks of the
// elimination are the symmetric Schur complements of G + ridge I, equal to
// their transposes up to rounding). Returns false, leaving `a` unchanged,
// unless the block is positive definite by Sylvester's criterion (leading
// minors > 0) with a finite determinant.
__device__ __forceinline__ bool inverse4_sym(double (&a)[4][4]) {
    const double a00 = a[0][0], a01 = a[0][1], a02 = a[0][2], a03 = a[0][3];
    const double a11 = a[1][1], a12 = a[1][2], a13 = a[1][3], a22 = a[2][2], a23 = a[2][3], a33 = a[3][3];
    const double s0 = a00 * a11 - a01 * a01, s1 = a00 * a12 - a01 * a02, s2 = a00 * a13 - a01 * a03;
    const double s3 = a01 * a12 - a11 * a02, s4 = a01 * a13 - a11 * a03, s5 = a02 * a13 - a12 * a03;
    const double c5 = a22 * a33 - a23 * a23, c4 = a12 * a33 - a13 * a23, c3 = a12 * a23 - a13 * a22;
    const double c2 = a02 * a33 - a03 * a23, c1 = a02 * a23 - a03 * a22, c0 = a02 * a13 - a03 * a12;
    const double det = s0 * c5 - s1 * c4 + s2 * c3 + s3 * c2 - s4 * c1 + s5 * c0;
    const double m3 = a00 * (a11 * a22 - a12 * a12) - a01 * (a01 * a22 - a12 * a02) + a02 * (a01 * a12 - a11 * a02);
    if (!(a00 > 0.0 && s0 > 0.0 && m3 > 0.0 && det > 0.0 && isfinite(det))) return false;
    const double id = 1.0 / det;
    const double b00 = (a11 * c5 - a12 * c4 + a13 * c3) * id, b01 = (-a01 * c5 + a02 * c4 - a03 * c3) * id;
    const double b02 = (a13 * s5 - a23 * s4 + a33 * s3) * id, b03 = (-a12 * s5 + a22 * s4 - a23 * s3) * id;
    const double b11 = (a00 * c5 - a02 * c2 + a03 * c1) * id, b12 = (-a03 * s5 + a23 * s2 - a33 * s1) * id;
    const double b13 = (a02 * s5 - a22 * s2 + a23 * s1) * id, b22 = (a03 * s4 - a13 * s2 + a33 * s0) * id;
    const double b23 = (-a02 * s4 + a12 * s2 - a23 * s0) * id, b33 = (a02 * s3 - a12 * s1 + a22 * s0) * id;
    a[0][0] = b00; a[0][1] = a[1][0] = b01; a[0][2] = a[2][0] = b02; a[0][3] = a[3][0] = b03;
    a[1][1] = b11; a[1][2] = a[2][1] = b12; a[1][3] = a[3][1] = b13;
    a[2][2] = b22; a[2][3] = a[3][2] = b23; a[3][3] = b33;
    return true;
}

constexpr int DT = 64, DK = 16, DLD = 72;   // CTA tile, k slab, shared row stride (doubles)

// D (8x8) += A (8x4) B (4x8) on the fp64 tensor cores (warp-wide). Lane l
// holds A[l/4][l%4], B[l%4][l/4] and D[l/4][2(l%4) + {0,1}].
__device__ __forceinline__ void dmma(double (&c)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(c[0]), "+d"(c[1]) : "d"(a), "d"(b));
}

// One 64x64 tile of C = A B per CTA of 4 warps for the (unit, head, mode)
// problem, on the fp64 tensor cores (mma m8n8k4): each warp owns a 32x32
// quarter = 4x4 accumulator tiles, and per k step of 4 loads four A and four
// B fragments from shared memory for 16 MMAs. Operands are staged as
// [k][row] slabs of 16 k (row stride 72 doubles: fragment loads hit every
// bank twice, the minimum for 32 doubles), double-buffered, the next slab
// fetched into registers while the current one is multiplied. Thread t
// fetches row t % 64 of the slab for 8 consecutive k, so the shared stores of
// a warp are 32 consecutive doubles and the global loads run along the
// source's contiguous dimension or stay within one 32-byte sector per row.
__global__ void __launch_bounds__(128) k_dgemm(const kvc_unit * __restrict__ units, kvc_params_dev P,
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

    __shared__ __align__(16) double As[2][DK][DLD];
    __shared__ __align__(16) double Bs[2][DK][DLD];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
    const int fr = tid & 63, fk = (tid >> 6) * 8;       // fetch: row fr, k fk..fk+7 of the slab
    const bool rows = (mode == DG_GRAM && dual);       // operands are rows of X (k contiguous)
    double ra[8], rb[8];
    auto fetch = [&](int k0) {
        const int m = m0 + fr, c = n0 + fr;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int k = k0 + fk + e;
            double va = 0.0, vb = 0.0;
            if (k < K) {
                if (m < M) va = rows ? (double)X[(long long)m * t + k] : (double)X[(long long)k * t + m];
                if (c < N) {
                    if (mode == DG_GRAM) vb = dual ? (double)X[(long long)c * t + k] : (double)X[(long long)k * t + c];
                    else if (mode == DG_RHS) vb = (double)Y[(long long)k * dv + c];
                    else vb = Z[(long long)k * dv + c];
                }
            }
            ra[e] = va;
            rb[e] = vb;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            As[buf][fk + e][fr] = ra[e];
            Bs[buf][fk + e][fr] = rb[e];
        }
    };
    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j][0] = acc[i][j][1] = 0.0;
    fetch(0);
    stash(0);
    __syncthreads();
    int buf = 0;
    const int fm = lane >> 2, fq = lane & 3;
    for (int k0 = 0; k0 < K; k0 += DK) {
        const bool more = k0 + DK < K;
        if (more) fetch(k0 + DK);
#pragma unroll
        for (int kk = 0; kk < DK; kk += 4) {
            double a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                a[i] = As[buf][kk + fq][wm + 8 * i + fm];
                b[i] = Bs[buf][kk + fq][wn + 8 * i + fm];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) dmma(acc[i][j], a[i], b[j]);
        }
        if (more) stash(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
    if (mode == DG_GRAM) {
        double * G = gs + u.g_off + (long long)h * n * n;
        const double ridge = (double)P.ridge;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < 2; v++) {
                    const int a = m0 + wm + 8 * i + fm, b = n0 + wn + 8 * j + 2 * fq + v;
                    if (a < n && b < n && b <= a) {
                        const double x = acc[i][j][v] + (a == b ? ridge : 0.0);
                        G[(long long)a * n + b] = x;
                        G[(long long)b * n + a] = x;
                    }
                }
    } else if (mode == DG_RHS) {
        double * R = gs + u.z_off + (long long)h * n * dv;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < 2; v++) {
                    const int a = m0 + wm + 8 * i + fm, c = n0 + wn + 8 * j + 2 * fq + v;
                    if (a < M && c < N) R[(long long)a * dv + c] = acc[i][j][v];
                }
    } else {
        const kvc_layer_out lo = outs[u.layer];
        float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < 2; v++) {
                    const int a = m0 + wm + 8 * i + fm, c = n0 + wn + 8 * j + 2 * fq + v;
                    if (a < M && c < N) cv[(long long)a * dv + c] = (float)acc[i][j][v];
                }
    }
}

// Same products with the operands staged by cp.async in a three-slab ring
// (requires t and d_v multiples of 4, so every 16-byte chunk of X, Y and Z rows
// is aligned). Operands stay in their source layout in shared memory — rows of
// X ([m][k], stride 20 floats) for the dual Gram matrix, [k][m] rows (stride
// 72) otherwise — and are widened to fp64 as the MMA fragments are read
// (exact). Two slabs are in flight while the third is multiplied. Chunks that
// straddle the end of a row or of K copy only their valid bytes (the rest is
// zero-filled), so nothing outside X, Y or Z is read and no stray k term
// enters a product.
constexpr int AK_LD = DK + 4;        // [m][k] fp32 rows
constexpr int AM_LD = DT + 8;        // [k][m] rows (fp32 or fp64)
constexpr int DG_NST = 3;
constexpr int DG_STAGE_F = DT * AK_LD > DK * AM_LD ? DT * AK_LD : DK * AM_LD;   // floats per fp32 operand slab

size_t kvc_dgemm_async_smem() {
    // per stage: A (fp32) + B (fp32, or fp64 for Z)
    return (size_t)DG_NST * (DG_STAGE_F * sizeof(float) + DK * AM_LD * sizeof(double));
}

__device__ __forceinline__ void dg_cp16(void * smem, const void * gmem, int bytes) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(sa), "l"(gmem), "r"(bytes) : "memory");
}

// One instantiation per product (MODE: DG_GRAM, DG_RHS, DG_OUT), so the Gram
// product's triangle logic costs the other products nothing.
template <int MODE>
__global__ void __launch_bounds__(128) k_dgemm_async(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                     const float * __restrict__ fs, double * __restrict__ gs,
                                                     const kvc_layer_out * __restrict__ outs) {
    constexpr int mode = MODE;
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
    if (mode == DG_GRAM && n0 > m0) return;
    const float * X = fs + u.x_off + (long long)h * nq * t;
    const float * Y = fs + u.y_off + (long long)h * nq * dv;
    const double * Z = gs + u.z_off + (long long)h * n * dv;

    extern __shared__ __align__(16) unsigned char dgsm[];
    float * Asm = reinterpret_cast<float *>(dgsm);                                  // [NST][DG_STAGE_F]
    double * Bsm = reinterpret_cast<double *>(dgsm + DG_NST * DG_STAGE_F * sizeof(float));  // [NST][DK*AM_LD]
    const bool arows = (mode == DG_GRAM && dual);      // A = rows of X ([m][k])
    const bool brows = arows;                          // B = rows of X too (X X^T)
    const bool bz = (mode == DG_OUT);                  // B = Z (fp64)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
    const int fm = lane >> 2, fq = lane & 3;

    // one slab: A 64 x 16 fp32 = 256 chunks, B 256 (fp32) or 512 (fp64) chunks of 16 bytes
    auto issue = [&](int k0, int b) {
        float * As = Asm + b * DG_STAGE_F;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int c = tid + 128 * i;               // 0..255
            int bytes = 0;
            const float * src = X;
            float * dst;
            if (arows) {                               // row m = c / 4, k quad c % 4
                const int mm = c >> 2, kq = (c & 3) * 4, m = m0 + mm, k = k0 + kq;
                dst = As + mm * AK_LD + kq;
                if (m < M && k < K) { bytes = 4 * min(4, K - k); src = X + (long long)m * t + k; }
            } else {                                   // k row c / 16, m quad c % 16
                const int kk = c >> 4, mq = (c & 15) * 4, k = k0 + kk, m = m0 + mq;
                dst = As + kk * AM_LD + mq;
                if (k < K && m < M) { bytes = 4 * min(4, M - m); src = X + (long long)k * t + m; }
            }
            dg_cp16(dst, src, bytes);
        }
        if (bz) {
            double * Bs = Bsm + b * (DK * AM_LD);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int c = tid + 128 * i;           // 0..511: k row c / 32, n pair c % 32
                const int kk = c >> 5, np = (c & 31) * 2, k = k0 + kk, nn = n0 + np;
                int bytes = 0;
                const double * src = Z;
                if (k < K && nn < N) { bytes = 8 * min(2, N - nn); src = Z + (long long)k * dv + nn; }
                dg_cp16(Bs + kk * AM_LD + np, src, bytes);
            }
        } else {
            float * Bs = reinterpret_cast<float *>(Bsm + b * (DK * AM_LD));
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int c = tid + 128 * i;
                int bytes = 0;
                const float * src = X;
                float * dst;
                if (brows) {
                    const int nn = c >> 2, kq = (c & 3) * 4, col = n0 + nn, k = k0 + kq;
                    dst = Bs + nn * AK_LD + kq;
                    if (col < N && k < K) { bytes = 4 * min(4, K - k); src = X + (long long)col * t + k; }
                } else {
                    const int kk = c >> 4, nq4 = (c & 15) * 4, k = k0 + kk, col = n0 + nq4;
                    dst = Bs + kk * AM_LD + nq4;
                    if (k < K && col < N) {
                        bytes = 4 * min(4, N - col);
                        src = (mode == DG_RHS) ? Y + (long long)k * dv + col : X + (long long)k * t + col;
                    }
                }
                dg_cp16(dst, src, bytes);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j][0] = acc[i][j][1] = 0.0;
    // a Gram tile on the diagonal keeps only its lower triangle: the warp
    // whose 32 x 32 block lies above it skips its products, and the two
    // warps on it skip their 8 x 8 tiles above it (the store drops them)
    const bool diag = mode == DG_GRAM && m0 == n0;
    const bool skip_all = diag && wn > wm, lower_only = diag && wn == wm;
    const int nslab = (K + DK - 1) / DK;
    issue(0, 0);
    if (nslab > 1) issue(DK, 1);
    for (int s = 0; s < nslab; s++) {
        if (s + 1 < nslab) asm volatile("cp.async.wait_group 1;" ::: "memory");
        else asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();                               // slab s visible; slab s-1 no longer read
        if (s + 2 < nslab) issue((s + 2) * DK, (s + 2) % DG_NST);
        const int b = s % DG_NST;
        const float * As = Asm + b * DG_STAGE_F;
        const double * Bd = Bsm + b * (DK * AM_LD);
        const float * Bf = reinterpret_cast<const float *>(Bd);
        if (skip_all) continue;
#pragma unroll
        for (int kk = 0; kk < DK; kk += 4) {
            double a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int m = wm + 8 * i + fm, nn = wn + 8 * i + fm, k = kk + fq;
                a[i] = arows ? (double)As[m * AK_LD + k] : (double)As[k * AM_LD + m];
                bb[i] = bz ? Bd[k * AM_LD + nn] : (brows ? (double)Bf[nn * AK_LD + k] : (double)Bf[k * AM_LD + nn]);
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (!lower_only || j <= i) dmma(acc[i][j], a[i], bb[j]);
        }
    }
    if (mode == DG_GRAM) {
        double * G = gs + u.g_off + (long long)h * n * n;
        const double ridge = (double)P.ridge;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < 2; v++) {
                    const int a = m0 + wm + 8 * i + fm, b = n0 + wn + 8 * j + 2 * fq + v;
                    if (a < n && b < n && b <= a) {
                        const double x = acc[i][j][v] + (a == b ? ridge : 0.0);
                        G[(long long)a * n + b] = x;
                        G[(long long)b * n + a] = x;
                    }
                }
    } else if (mode == DG_RHS) {
        double * R = gs + u.z_off + (long long)h * n * dv;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < 2; v++) {
                    const int a = m0 + wm + 8 * i + fm, c = n0 + wn + 8 * j + 2 * fq + v;
                    if (a < M && c < N) R[(long long)a * dv + c] = acc[i][j][v];
                }
    } else {
        const kvc_layer_out lo = outs[u.layer];
        float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < 2; v++) {
                    const int a = m0 + wm + 8 * i + fm, c = n0 + wn + 8 * j + 2 * fq + v;
                    if (a < M && c < N) cv[(long long)a * dv + c] = (float)acc[i][j][v];
                }
    }
}

// Panel width for n unknowns: keeps the n x PW fp64 panel within 96 KB.
// Right-hand-side columns per panel of k_chol_solve: n x panel doubles of
// shared memory (at most 192 KB up to KVC_LSQ_MAX_N unknowns).
__host__ __device__ inline int lsq_panel(int n) {
    return n <= 384 ? 32 : (n <= 1536 ? 8 : (n <= 6144 ? 4 : (n <= 12288 ? 2 : 1)));
}

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
// Solve, n = min(n_q, t) <= 128 and d_v <= 128, one CTA of 16 warps per
// (unit, head): block Gauss-Jordan elimination of [G | R] in diagonal order
// without pivoting (R = Y for the dual, X^T Y from k_dgemm for the primal),
// four unknowns per step, on the fp64 tensor cores. G is symmetric positive
// definite (Gram matrix + ridge), for which elimination in diagonal order is
// stable.
// Step k (unknowns k..k+3): P = G[k..k+3][k..k+3] is inverted in registers
// (adjugate, or Gauss-Jordan when P is not positive definite); a pivot that is not positive and finite marks its unknown
// singular (its row of P^-1 is zeroed, so it drops out and ends at zero — the
// reference skips pivots below 1e-12). The pivot rows become P^-1 (pivot rows
// of G and R); every other row i loses M[i] x (the new pivot rows), with
// M[i] = G[i][k..k+3]. That rank-4 update is an m8n8k4 MMA per 8x8 tile: G's
// tiles right of the block (read from and written back to shared memory) and
// all of R (held in MMA accumulator fragments, warp w owning a 32x32 quarter-
// block). Two barriers per step; no triangular dependency chains. n is
// padded to a multiple of 8 with identity rows, which stay untouched.
// After the last step R holds G^-1 R: Z (dual, consumed by the OUT product) or
// C_v (primal) is written to global memory.
// ---------------------------------------------------------------------------
constexpr int GLD = FN + 8;     // G row stride: the 16-byte C-tile loads of a quarter-warp hit 8 bank groups
constexpr int PLD = FN + 4;     // pivot-row stride: B-fragment loads hit every bank twice

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
    const int n8 = (n + 7) & ~7;

    extern __shared__ __align__(16) double G[];   // [n8][GLD]
    double * PR = G + FN * GLD;                  // [4][PLD] new pivot rows of G
    double * RR = PR + 4 * PLD;                  // [4][PLD] new pivot rows of R
    double * RP = RR + 4 * PLD;                  // [4][PLD] old pivot rows of R
    double * M = RP + 4 * PLD;                   // [FN][4]  multipliers (0 on pivot rows)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int fr = lane >> 2, fq = lane & 3;     // MMA fragment row / k index of this lane
    const int wr = warp >> 2, wc = warp & 3;     // this warp's quarter-block of R
    if (n == n8 && (n & 1) == 0 && ((((uintptr_t)Gg) & 15) == 0)) {
        // rows of G straight into shared memory, 16 bytes per asynchronous
        // copy, all in flight at once (one CTA per SM: nothing else hides
        // this load); the copies complete before the first barrier
        const int per_row = n >> 1;
        for (int e = tid; e < n * per_row; e += 512) {
            const int i = e / per_row, c = (e - i * per_row) * 2;
            const uint32_t sa = (uint32_t)__cvta_generic_to_shared(G + i * GLD + c);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(sa), "l"(Gg + (long long)i * n + c) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
        for (int e = tid; e < n8 * n8; e += 512) {
            const int i = e / n8, j = e - i * n8;
            G[i * GLD + j] = (i < n && j < n) ? Gg[(long long)i * n + j] : (i == j ? 1.0 : 0.0);
        }
    }
    double acc[4][4][2];
#pragma unroll
    for (int rt = 0; rt < 4; rt++)
#pragma unroll
        for (int ct = 0; ct < 4; ct++)
#pragma unroll
            for (int v = 0; v < 2; v++) {
                const int row = 32 * wr + 8 * rt + fr, col = 32 * wc + 8 * ct + 2 * fq + v;
                double x = 0.0;
                if (row < n && col < dv) x = dual ? (double)Y[(long long)row * dv + col] : Zg[(long long)row * dv + col];
                acc[rt][ct][v] = x;
            }
    // rows kk .. kk+3 of R (held in this warp's fragments) into RP: the old
    // pivot rows of R for step kk, taken as soon as the previous step is done
    auto extract_rp = [&](int kk) {
        if (kk >= n8 || wr != (kk >> 5)) return;
        const int prt_ = (kk >> 3) & 3, pr0_ = kk & 7;
        if (fr < pr0_ || fr >= pr0_ + 4) return;
#pragma unroll
        for (int rt = 0; rt < 4; rt++)
            if (rt == prt_)
#pragma unroll
                for (int ct = 0; ct < 4; ct++)
#pragma unroll
                    for (int v = 0; v < 2; v++) RP[(fr - pr0_) * PLD + 32 * wc + 8 * ct + 2 * fq + v] = acc[rt][ct][v];
    };
    extract_rp(0);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();

    for (int k = 0; k < n8; k += 4) {
        const int jt0 = (k + 4) >> 3;            // first column tile of G still needed
        const int prt = (k >> 3) & 3, pr0 = k & 7;
        // ---- A (one barrier): warps 0-3 invert the pivot block P and write the
        // new pivot rows of G (P^-1 G[k..k+3][j], into PR and into G itself) and
        // of R (P^-1 RP, into RR), one column per thread; warps 4-7 meanwhile
        // copy the multipliers M. A step costs 4.3k cycles without the overlap
        // (A 1.7k, of which 0.4k the multipliers; a second barrier 0.4k).
        if (tid < 128) {
            double T[4][4];
#pragma unroll
            for (int q = 0; q < 4; q++)
#pragma unroll
                for (int c = 0; c < 4; c++) T[q][c] = G[(k + q) * GLD + k + c];
            // (no barrier: P's own columns of G are not rewritten below)
            // inverse of the pivot block: the adjugate over the determinant
            // (one division, a short dependency chain) when the block is
            // positive definite, which every pivot block of G + ridge I is;
            // otherwise in-place Gauss-Jordan inversion, where a skipped
            // (non-positive) pivot leaves its row and column to be zeroed
            if (!inverse4_sym(T)) {
            bool skip[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const double piv = T[q][q];
                skip[q] = !(piv > 0.0 && isfinite(piv));
                if (skip[q]) continue;
                const double ip = 1.0 / piv;
                T[q][q] = 1.0;
#pragma unroll
                for (int c = 0; c < 4; c++) T[q][c] *= ip;
#pragma unroll
                for (int r2 = 0; r2 < 4; r2++) {
                    if (r2 == q) continue;
                    const double f = T[r2][q];
                    T[r2][q] = 0.0;
#pragma unroll
                    for (int c = 0; c < 4; c++) T[r2][c] = fma(-f, T[q][c], T[r2][c]);
                }
            }
#pragma unroll
            for (int q = 0; q < 4; q++)
                if (skip[q])
#pragma unroll
                    for (int c = 0; c < 4; c++) T[q][c] = T[c][q] = 0.0;
            }
            const int j = 8 * jt0 + tid;
            if (j < n8) {
                double g[4];
#pragma unroll
                for (int q = 0; q < 4; q++) g[q] = G[(k + q) * GLD + j];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const double x = fma(T[q][0], g[0], fma(T[q][1], g[1], fma(T[q][2], g[2], T[q][3] * g[3])));
                    PR[q * PLD + j] = x;
                    // the pivot block's own columns are dead after this step;
                    // leaving them unwritten lets every thread read P without
                    // a barrier (tile updates below give them zero multipliers)
                    if (j >= k + 4) G[(k + q) * GLD + j] = x;
                }
            }
            double rp[4];
#pragma unroll
            for (int q = 0; q < 4; q++) rp[q] = RP[q * PLD + tid];
#pragma unroll
            for (int q = 0; q < 4; q++)
                RR[q * PLD + tid] = fma(T[q][0], rp[0], fma(T[q][1], rp[1], fma(T[q][2], rp[2], T[q][3] * rp[3])));
        } else if (tid < 256) {                  // rows past n8 get zero multipliers too
            const int r = tid - 128;
            const bool zero = (r >= k && r < k + 4) || r >= n8;
#pragma unroll
            for (int q = 0; q < 4; q++) M[r * 4 + q] = zero ? 0.0 : G[r * GLD + k + q];
        }
        __syncthreads();
        // ---- B: rank-4 updates (pivot rows have zero multipliers). The 16
        // independent MMAs of this warp's R tiles are interleaved, two at a
        // time, with the load -> MMA -> store chains of its G tiles (row
        // tile `warp`, column tiles from jt0, two at a time), so the tensor
        // pipe works on R while a G chain waits.
        {
            double am[4], bb[4];
#pragma unroll
            for (int rt = 0; rt < 4; rt++) am[rt] = -M[(32 * wr + 8 * rt + fr) * 4 + fq];
#pragma unroll
            for (int ct = 0; ct < 4; ct++) bb[ct] = RR[fq * PLD + 32 * wc + 8 * ct + fr];
            const bool grow = 8 * warp < n8;
            const double amg = grow ? -M[(8 * warp + fr) * 4 + fq] : 0.0;
            const int nct = n8 >> 3;
#pragma unroll
            for (int it = 0; it < 8; it++) {
                const int ct0 = jt0 + 2 * it;
                if (grow && ct0 < nct) {
                    const int ct1 = min(ct0 + 1, nct - 1);
                    double2 * cp0 = reinterpret_cast<double2 *>(G + (8 * warp + fr) * GLD + 8 * ct0 + 2 * fq);
                    double2 * cp1 = reinterpret_cast<double2 *>(G + (8 * warp + fr) * GLD + 8 * ct1 + 2 * fq);
                    const double b0 = PR[fq * PLD + 8 * ct0 + fr], b1 = PR[fq * PLD + 8 * ct1 + fr];
                    const double2 c0 = *cp0, c1 = *cp1;
                    double cc0[2] = {c0.x, c0.y}, cc1[2] = {c1.x, c1.y};
                    dmma(cc0, amg, b0);
                    dmma(cc1, amg, b1);
                    *cp0 = make_double2(cc0[0], cc0[1]);
                    if (ct0 + 1 < nct) *cp1 = make_double2(cc1[0], cc1[1]);
                }
                dmma(acc[(2 * it) >> 2][(2 * it) & 3], am[(2 * it) >> 2], bb[(2 * it) & 3]);
                dmma(acc[(2 * it + 1) >> 2][(2 * it + 1) & 3], am[(2 * it + 1) >> 2], bb[(2 * it + 1) & 3]);
            }
            if (wr == (k >> 5) && fr >= pr0 && fr < pr0 + 4) {
#pragma unroll
                for (int rt = 0; rt < 4; rt++)
                    if (rt == prt)
#pragma unroll
                        for (int ct = 0; ct < 4; ct++)
#pragma unroll
                            for (int v = 0; v < 2; v++)
                                acc[rt][ct][v] = RR[(fr - pr0) * PLD + 32 * wc + 8 * ct + 2 * fq + v];
            }
            extract_rp(k + 4);
        }
        __syncthreads();
    }

    const kvc_layer_out lo = outs[u.layer];
    float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
#pragma unroll
    for (int rt = 0; rt < 4; rt++)
#pragma unroll
        for (int ct = 0; ct < 4; ct++)
#pragma unroll
            for (int v = 0; v < 2; v++) {
                const int row = 32 * wr + 8 * rt + fr, col = 32 * wc + 8 * ct + 2 * fq + v;
                if (row >= n || col >= dv) continue;
                if (dual) Zg[(long long)row * dv + col] = acc[rt][ct][v];
                else cv[(long long)row * dv + col] = (float)acc[rt][ct][v];
            }
}

size_t kvc_lsq_smem_bytes(int n) {
    size_t pw = (size_t)lsq_panel(n);
    size_t b = (size_t)n * pw * sizeof(double);
    if (n <= 128) b += (size_t)n * n * sizeof(double);
    return b;
}

static int launch_dgemm(dim3 grid, const kvc_unit * d_units, const kvc_params_dev & P, const float * fs,
                        double * gs, const kvc_layer_out * d_outs, int mode, bool aligned, cudaStream_t st) {
    if (aligned) {
        const size_t sm = kvc_dgemm_async_smem();
        auto kern = mode == DG_GRAM ? k_dgemm_async<DG_GRAM> : (mode == DG_RHS ? k_dgemm_async<DG_RHS>
                                                                               : k_dgemm_async<DG_OUT>);
        KVC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        kern<<<grid, 128, sm, st>>>(d_units, P, fs, gs, d_outs);
    } else {
        k_dgemm<<<grid, 128, 0, st>>>(d_units, P, fs, gs, d_outs, mode);
    }
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_lsq_gram(const kvc_unit * d_units, int n_units, int max_n, int max_t, const kvc_params_dev & P,
                        const float * fs, double * gs, const kvc_layer_out * d_outs, const kvc_unit * d_primal,
                        int n_primal, bool aligned, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    const int tg = (max_n + DT - 1) / DT;
    int rc;
    if ((rc = launch_dgemm(dim3(tg * tg, P.H, n_units), d_units, P, fs, gs, d_outs, DG_GRAM, aligned, st))) return rc;
    if (n_primal > 0) {
        const int to = ((max_t + DT - 1) / DT) * ((P.dv + DT - 1) / DT);
        if ((rc = launch_dgemm(dim3(to, P.H, n_primal), d_primal, P, fs, gs, d_outs, DG_RHS, aligned, st))) return rc;
    }
    return KVC_OK;
}

int kvc_launch_lsq_factor(const kvc_unit * d_units, int n_units, int max_n, size_t smem_bytes,
                          const kvc_params_dev & P, const float * fs, double * gs,
                          const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    const size_t fast_smem = (size_t)(FN * GLD + 12 * PLD + 4 * FN + 16) * sizeof(double);
    KVC_CUDA(cudaFuncSetAttribute(k_lsq_factor, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fast_smem));
    k_lsq_factor<<<dim3(n_units, P.H), 512, fast_smem, st>>>(d_units, P, fs, gs, d_outs);
    KVC_CUDA(cudaGetLastError());
    if (max_n > FN || P.dv > FN) {
        KVC_CUDA(cudaFuncSetAttribute(k_chol_solve, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
        k_chol_solve<<<dim3(n_units, P.H), 256, smem_bytes, st>>>(d_units, P, fs, gs, d_outs);
        KVC_CUDA(cudaGetLastError());
    }
    return KVC_OK;
}

int kvc_launch_lsq_out(const kvc_unit * d_units, int n_units, int max_t, const kvc_params_dev & P,
                       const float * fs, double * gs, const kvc_layer_out * d_outs, bool any_dual, bool aligned,
                       cudaStream_t st) {
    if (n_units <= 0 || !any_dual) return KVC_OK;
    const int to = ((max_t + DT - 1) / DT) * ((P.dv + DT - 1) / DT);
    return launch_dgemm(dim3(to, P.H, n_units), d_units, P, fs, gs, d_outs, DG_OUT, aligned, st);
}
