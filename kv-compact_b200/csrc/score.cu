// score.cu — reference scoring, row softmax + key importance, refit target Y.
//
// Stage 1, k_score: S[q][j] = (sum_d Q[q][d] * K[key(j)][d]) * (1/sqrt(d_k))
//   The reference computes each dot product as a sequential fp32 sum over d
//   with a separate multiply per term, then scales (include/kv-compact-math.h:
//   44-54, src/kv-compact-api.cpp:618-628). Key selection ranks keys by values
//   derived from S, and a different summation order moves S by ~1e-6 relative,
//   which is enough to reorder keys whose importances differ by less than
//   that. So every S element here is accumulated in exactly the reference's
//   order with explicitly rounded multiply and add: S is bit-identical to the
//   reference's. The kernel is a 128x128 (or 64x256) tile SIMT GEMM whose
//   inner loop runs over d in order for 64 independent accumulators per thread.
//   The refit's S[:, sel] is gathered from S afterwards (k_gather_x,
//   k_gather_softmax_x), bit for bit these scores.
//
// Stage 2, k_softmax_importance: row softmax statistics with max shift and
//   1/(sum + 1e-12) (math.h:201-248), kept for the beta fit and the metrics;
//   per-key importance aggregates A over the queries in query order (max,
//   RMS or mean), plus the per-key max used by sensitivity weighting
//   (math.h:579-594). S itself is never overwritten: every consumer of A
//   forms it from S and the row statistics (softmax_entry), so the refit's
//   S[:, sel] is a gather (k_gather_x) instead of a second scoring pass.
//
// Stage 3, k_pv: Y_h = A_h V_h (math.h:70-80 via src/kv-compact-api.cpp:754-783),
//   a 64x64-tile SIMT GEMM with fp32 FMA (Y only feeds the least-squares
//   right-hand side, which is tolerance-checked); the tensor-core version is
//   k_pv_tc (pv_tc.cu).
#include "engine.h"

#include <math.h>
#include <stdlib.h>

namespace {

constexpr int SB = 64, SK = 32, ST = 256;

// Position of cheap reference query qi of n within a chunk of C tokens
// (src/kv-compact-api.cpp:140-146): floor(((qi+1)/(n+1))^2 * (C-1)).
__device__ __forceinline__ int cheap_pos(int qi, int n, int C) {
    float fr = __fdiv_rn((float)(qi + 1), (float)(n + 1));
    fr = __fmul_rn(fr, fr);
    int pos = (int)__fmul_rn(fr, (float)(C - 1));
    if (pos >= C) pos = C - 1;
    if (pos < 0) pos = 0;
    return pos;
}

__device__ __forceinline__ const float * qrow_ptr(const kvc_unit & u, int q, int h, int ek, int dk) {
    if (u.qmode == 0) return u.Q + (long long)q * ek + (long long)h * dk;
    return u.K + (long long)cheap_pos(q, u.nq, u.C) * ek + (long long)h * dk;
}

// Load rows [0, NR) of a [NR x SK] slab starting at column d0 into shared
// memory transposed (dst[k][row]); zero outside bounds. 256 threads: thread
// tid takes row tid % NR and SK*NR/256 consecutive columns of it in float4
// pieces, so a warp's transposed stores hit 32 consecutive rows.
template <int NR>
__device__ __forceinline__ void load_rows(float (*dst)[NR + 4], const float * const * rowp, int d0, int dk,
                                          bool vec_ok) {
    constexpr int PER = SK * NR / ST;        // floats per thread: 16 (NR=128) or 32 (NR=256) or 8 (NR=64)
    const int r = threadIdx.x % NR;
    const int c0 = (threadIdx.x / NR) * PER;
    const float * p = rowp[r];
#pragma unroll
    for (int i = 0; i < PER; i += 4) {
        const int c = c0 + i;
        float v[4];
        if (p && vec_ok && d0 + c + 4 <= dk) {
            const float4 a = *reinterpret_cast<const float4 *>(p + d0 + c);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; e++) v[e] = (p && d0 + c + e < dk) ? p[d0 + c + e] : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 4; e++) dst[c + e][r] = v[e];
    }
}

}  // namespace

// Epilogue of both scoring kernels: S = acc * (1/sqrt(d_k)) into the S block;
// mode 2 also writes, per row and CTA
// key tile, the maximum of the row's scores in the tile (exact: a maximum
// does not depend on order), from which the importance kernel takes the row
// maxima without a pass over S. Rows of a tile are shared by the NTX = TK/8
// lanes with the same ty (a half-warp or a warp), reduced with shuffles.
template <int TQ, int TK>
__device__ __forceinline__ void store_scores(const kvc_unit & u, const kvc_params_dev & P, float * fs,
                                             const float (&acc)[8][8], int mode, int ncols, int q0, int j0, int ty,
                                             int tx, int h) {
    constexpr int NTX = TK / 8;
    const int ld = ncols;
    float * out = fs + u.s_off + (long long)h * u.nq * u.C;
    const bool vst = (ld & 3) == 0 && ((((uintptr_t)out) & 15) == 0);
    const int ntile = (u.C + 127) / 128;
    float * pm = fs + u.pm_off + (long long)h * u.nq * ntile;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int q = q0 + (i < 4 ? 4 * ty + i : TQ / 2 + 4 * ty + i - 4);
        float * row = out + (long long)q * ld;
        float mx = -INFINITY;
#pragma unroll
        for (int hb = 0; hb < 2; hb++) {
            const int c = j0 + hb * (TK / 2) + 4 * tx;
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                v[e] = __fmul_rn(acc[i][4 * hb + e], P.isd);
                if (c + e < ncols) mx = fmaxf(mx, v[e]);
            }
            if (q >= u.nq) continue;
            if (vst && c + 4 <= ncols) {
                *reinterpret_cast<float4 *>(row + c) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++)
                    if (c + e < ncols) row[c + e] = v[e];
            }
        }
        if (mode == 2) {
#pragma unroll
            for (int o = NTX / 2; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (tx == 0 && q < u.nq) pm[(long long)q * ntile + j0 / TK] = mx;
        }
    }
}

// mode 0: all C keys of the chunk -> S block (ld C); mode 2: the same plus
// the row maxima of each key tile (store_scores)
// CTA tile TQ queries x TK keys (TQ*TK = 16384), 256 threads, 8x8 outputs per
// thread: rows 4ty+{0..3} and TQ/2+4ty+{0..3}, columns 4tx+{0..3} and
// TK/2+4tx+{0..3}, so both operand reads per d are two conflict-free
// float4 loads for 64 multiply-add pairs. Each output is one accumulator
// updated in d order: acc = fl(acc + fl(q*k)).
template <int TQ>
__global__ void __launch_bounds__(ST, 2) k_score(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                 float * __restrict__ fs, int mode) {
    constexpr int TK = 16384 / TQ;
    constexpr int NTX = TK / 8;               // threads along keys
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y;
    const int ncols = u.C;
    const int tq = (u.nq + TQ - 1) / TQ, tk = (ncols + TK - 1) / TK;
    if ((int)blockIdx.x >= tq * tk) return;
    const int q0 = (blockIdx.x / tk) * TQ, j0 = (blockIdx.x % tk) * TK;
    const int ek = P.H * P.dk, dk = P.dk;

    __shared__ __align__(16) float Qs[SK][TQ + 4];
    __shared__ __align__(16) float Ks[SK][TK + 4];
    __shared__ const float * qp[TQ];
    __shared__ const float * kp[TK];
    const int tid = threadIdx.x;
    for (int i = tid; i < TQ + TK; i += ST) {
        if (i < TQ) {
            const int q = q0 + i;
            qp[i] = q < u.nq ? qrow_ptr(u, q, h, ek, dk) : nullptr;
        } else {
            const int j = j0 + i - TQ;
            if (j < ncols) {
                const int key = j;
                kp[i - TQ] = u.K + (long long)key * ek + (long long)h * dk;
            } else {
                kp[i - TQ] = nullptr;
            }
        }
    }
    __syncthreads();
    const bool vec_ok = ((ek & 3) == 0) && ((dk & 3) == 0) &&
                        ((((uintptr_t)u.K) & 15) == 0) && (u.qmode == 1 || (((uintptr_t)u.Q) & 15) == 0);
    const int ty = tid / NTX, tx = tid % NTX;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

    for (int d0 = 0; d0 < dk; d0 += SK) {
        load_rows<TQ>(Qs, qp, d0, dk, vec_ok);
        load_rows<TK>(Ks, kp, d0, dk, vec_ok);
        __syncthreads();
        const int kend = min(SK, dk - d0);
        if (kend == SK) {
#pragma unroll 4
            for (int kk = 0; kk < SK; kk++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&Qs[kk][4 * ty]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&Qs[kk][TQ / 2 + 4 * ty]);
                const float4 b0 = *reinterpret_cast<const float4 *>(&Ks[kk][4 * tx]);
                const float4 b1 = *reinterpret_cast<const float4 *>(&Ks[kk][TK / 2 + 4 * tx]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
            }
        } else {
            for (int kk = 0; kk < kend; kk++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&Qs[kk][4 * ty]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&Qs[kk][TQ / 2 + 4 * ty]);
                const float4 b0 = *reinterpret_cast<const float4 *>(&Ks[kk][4 * tx]);
                const float4 b1 = *reinterpret_cast<const float4 *>(&Ks[kk][TK / 2 + 4 * tx]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
            }
        }
        __syncthreads();
    }
    store_scores<TQ, TK>(u, P, fs, acc, mode, ncols, q0, j0, ty, tx, h);
}

// Same tile, operands staged with cp.async (requires 16-byte aligned rows:
// d_k and H*d_k multiples of 4 and aligned K/Q bases). Two staging buffers
// keep the next slab's rows in flight while the current slab is multiplied;
// each slab is transposed shared-to-shared into the [k][row] layout the
// float4 operand reads need. The arithmetic is that of k_score<128>.
constexpr int AS_LD = SK + 4;   // staged row stride (floats): conflict-free float4 reads across rows

__device__ __forceinline__ void cp_async16(void * smem, const void * gmem, int src_bytes) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(sa), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

size_t kvc_score_async_smem() {
    return sizeof(float) * (2 * 2 * 128 * AS_LD + 2 * SK * (128 + 4));
}

__global__ void __launch_bounds__(ST, 2) k_score_async(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                       float * __restrict__ fs, int mode) {
    constexpr int TQ = 128, TK = 128, NTX = TK / 8;
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y;
    const int ncols = u.C;
    const int tq = (u.nq + TQ - 1) / TQ, tk = (ncols + TK - 1) / TK;
    if ((int)blockIdx.x >= tq * tk) return;
    const int q0 = (blockIdx.x / tk) * TQ, j0 = (blockIdx.x % tk) * TK;
    const int ek = P.H * P.dk, dk = P.dk;

    extern __shared__ __align__(16) float dsm[];
    float * Sq = dsm;                                   // [2][TQ][AS_LD] staged Q rows
    float * Sk = Sq + 2 * TQ * AS_LD;                   // [2][TK][AS_LD] staged K rows
    float (*Qs)[TQ + 4] = reinterpret_cast<float (*)[TQ + 4]>(Sk + 2 * TK * AS_LD);
    float (*Ks)[TK + 4] = reinterpret_cast<float (*)[TK + 4]>(Sk + 2 * TK * AS_LD + SK * (TQ + 4));
    __shared__ const float * qp[TQ];
    __shared__ const float * kp[TK];
    const int tid = threadIdx.x;
    if (tid < TQ) {
        const int q = q0 + tid;
        qp[tid] = q < u.nq ? qrow_ptr(u, q, h, ek, dk) : nullptr;
    } else {
        const int j = j0 + tid - TQ;
        if (j < ncols) {
            const int key = j;
            kp[tid - TQ] = u.K + (long long)key * ek + (long long)h * dk;
        } else {
            kp[tid - TQ] = nullptr;
        }
    }
    __syncthreads();
    auto issue = [&](int d0, int b) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int e = tid + ST * i, r = e >> 3, c = (e & 7) * 4;
            const float * pq = qp[r];
            const float * pk = kp[r];
            const int bq = (pq && d0 + c < dk) ? 16 : 0, bk = (pk && d0 + c < dk) ? 16 : 0;
            cp_async16(Sq + (b * TQ + r) * AS_LD + c, bq ? pq + d0 + c : fs, bq);
            cp_async16(Sk + (b * TK + r) * AS_LD + c, bk ? pk + d0 + c : fs, bk);
        }
        cp_async_commit();
    };
    const int ty = tid / NTX, tx = tid % NTX;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
    const int nslab = (dk + SK - 1) / SK;
    issue(0, 0);
    if (nslab > 1) issue(SK, 1);
    for (int s = 0; s < nslab; s++) {
        const int b = s & 1;
        if (s + 1 < nslab) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();                                // slab s staged; the previous slab's products are done
        {
            const int r = tid & (TQ - 1), c0 = (tid >> 7) * 16;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 vq = *reinterpret_cast<const float4 *>(Sq + (b * TQ + r) * AS_LD + c0 + 4 * i);
                const float4 vk = *reinterpret_cast<const float4 *>(Sk + (b * TK + r) * AS_LD + c0 + 4 * i);
                Qs[c0 + 4 * i + 0][r] = vq.x; Qs[c0 + 4 * i + 1][r] = vq.y;
                Qs[c0 + 4 * i + 2][r] = vq.z; Qs[c0 + 4 * i + 3][r] = vq.w;
                Ks[c0 + 4 * i + 0][r] = vk.x; Ks[c0 + 4 * i + 1][r] = vk.y;
                Ks[c0 + 4 * i + 2][r] = vk.z; Ks[c0 + 4 * i + 3][r] = vk.w;
            }
        }
        __syncthreads();                                // operands ready; staging buffer b free again
        if (s + 2 < nslab) issue((s + 2) * SK, b);
        const int kend = min(SK, dk - s * SK);
        if (kend == SK) {
#pragma unroll 4
            for (int kk = 0; kk < SK; kk++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&Qs[kk][4 * ty]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&Qs[kk][TQ / 2 + 4 * ty]);
                const float4 b0 = *reinterpret_cast<const float4 *>(&Ks[kk][4 * tx]);
                const float4 b1 = *reinterpret_cast<const float4 *>(&Ks[kk][TK / 2 + 4 * tx]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
            }
        } else {
            for (int kk = 0; kk < kend; kk++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&Qs[kk][4 * ty]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&Qs[kk][TQ / 2 + 4 * ty]);
                const float4 b0 = *reinterpret_cast<const float4 *>(&Ks[kk][4 * tx]);
                const float4 b1 = *reinterpret_cast<const float4 *>(&Ks[kk][TK / 2 + 4 * tx]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
            }
        }
    }
    store_scores<TQ, TK>(u, P, fs, acc, mode, ncols, q0, j0, ty, tx, h);
}

// A[q][j] of the row softmax, formed from the raw score s, the row max m
// and inv = 1 / (row exp-sum + 1e-12) with the reference's arithmetic
// (math.h:201-248): e = expf(s - m), A = e * inv. The scores stay in place;
// every consumer of A (importance, Y = A V) forms it with this function.
__device__ __forceinline__ float softmax_entry(float s, float m, float inv) {
    return __fmul_rn(expf(__fsub_rn(s, m)), inv);
}
__device__ __forceinline__ float softmax_inv(float sum) { return __fdiv_rn(1.0f, __fadd_rn(sum, 1e-12f)); }

// One CTA per (unit, head); S is left intact. Phase 1: one warp per row —
// row max, exp-sum (the second read of the row comes from L1), kept as the
// row statistics. Phase 2: one thread per key — A formed from S and the row
// statistics, aggregated over queries in query order (max, RMS or mean),
// plus the per-key max used by sensitivity weighting (math.h:579-594).
constexpr int SMI_ROWS = 2048;   // row statistics held in shared memory (more rows: read from global)

__global__ void __launch_bounds__(256) k_softmax_importance(const kvc_unit * __restrict__ units,
                                                           kvc_params_dev P, float * __restrict__ fs) {
    const kvc_unit u = units[blockIdx.y];
    const int h = blockIdx.x;
    const int C = u.C, nq = u.nq;
    const float * S = fs + u.s_off + (long long)h * nq * C;
    float * rmax = fs + u.row_off + (long long)h * 2 * nq;
    float * rsum = rmax + nq;
    __shared__ float sm_m[SMI_ROWS], sm_inv[SMI_ROWS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int q = warp; q < nq; q += nw) {
        const float * row = S + (long long)q * C;
        float m = row[0];
        for (int j = lane; j < C; j += 32) { float v = row[j]; if (v > m) m = v; }
        for (int o = 16; o; o >>= 1) { float v = __shfl_xor_sync(0xffffffffu, m, o); if (v > m) m = v; }
        float s = 0.0f;
        for (int j = lane; j < C; j += 32) s = __fadd_rn(s, expf(__fsub_rn(row[j], m)));
        for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) {
            rmax[q] = m;
            rsum[q] = s;
            if (q < SMI_ROWS) { sm_m[q] = m; sm_inv[q] = softmax_inv(s); }
        }
    }
    __syncthreads();
    float * imp = fs + u.imp_off + (long long)h * C;
    float * cmax = fs + u.imp_off + (long long)(P.H + h) * C;
    const float inv_m = __fdiv_rn(1.0f, (float)nq);
    constexpr int QB = 8;                    // rows whose loads are in flight together
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        float acc = 0.0f, mx = 0.0f;
        for (int q0 = 0; q0 < nq; q0 += QB) {
            float v[QB];
#pragma unroll
            for (int k = 0; k < QB; k++) v[k] = q0 + k < nq ? S[(long long)(q0 + k) * C + j] : 0.0f;
#pragma unroll
            for (int k = 0; k < QB; k++) {       // aggregated in query order
                const int q = q0 + k;
                if (q >= nq) break;
                const float m = q < SMI_ROWS ? sm_m[q] : rmax[q];
                const float inv = q < SMI_ROWS ? sm_inv[q] : softmax_inv(rsum[q]);
                const float w = softmax_entry(v[k], m, inv);
                if (P.score_method == 0) { if (w > acc) acc = w; }
                else if (P.score_method == 1) acc = __fadd_rn(acc, __fmul_rn(w, w));
                else acc = __fadd_rn(acc, w);
                if (w > mx) mx = w;
            }
        }
        if (P.score_method == 1) acc = sqrtf(__fmul_rn(acc, inv_m));
        else if (P.score_method == 2) acc = __fmul_rn(acc, inv_m);
        imp[j] = acc;
        cmax[j] = mx;
    }
}

// Single pass over S for chunks of at most RI_THREADS * RI_MAX_CPT keys and
// SMI_ROWS queries, with the row maxima from the scoring epilogue (mode 2):
// the CTA walks the rows in blocks of RI_RB, each thread holding its
// columns' scores of the block (the next block already loading) and turning
// them into exponentials in place; one CTA-wide reduction per block gives
// the rows' exp-sums, then A = e * inv (softmax_entry's arithmetic) is
// aggregated per key in query order as k_softmax_importance aggregates it.
// S is read once from memory and exp evaluated once per entry. Measured on
// a cfg4 step: one row per block and 4 CTAs per SM 1.86 ms; 2 rows, 3 CTAs
// 2.02; 2 rows, 4 CTAs 2.19; 4 rows, 2 CTAs 2.27; 1 row, 6 CTAs 2.15.
// RI_CPT columns per thread, the smallest instantiation that covers the
// chunk (a 1,280-key chunk takes 5: no thread evaluates dead columns).
constexpr int RI_THREADS = 256, RI_MAX_CPT = 8;

template <int RI_RB, int MINB, int RI_CPT>
__global__ void __launch_bounds__(RI_THREADS, MINB) k_row_importance(const kvc_unit * __restrict__ units,
                                                                  kvc_params_dev P, float * __restrict__ fs,
                                                                  int tile_keys) {
    const kvc_unit u = units[blockIdx.y];
    const int h = blockIdx.x, C = u.C, nq = u.nq, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const float * S = fs + u.s_off + (long long)h * nq * C;
    const int ntile_alloc = (C + 127) / 128, ntile = (C + tile_keys - 1) / tile_keys;
    const float * pm = fs + u.pm_off + (long long)h * nq * ntile_alloc;
    float * rmax = fs + u.row_off + (long long)h * 2 * nq;
    float * rsum = rmax + nq;
    __shared__ float sm_m[SMI_ROWS];
    __shared__ float red[2][RI_RB][RI_THREADS / 32];
    for (int q = tid; q < nq; q += RI_THREADS) {
        float m = pm[(long long)q * ntile_alloc];
        for (int k = 1; k < ntile; k++) m = fmaxf(m, pm[(long long)q * ntile_alloc + k]);
        sm_m[q] = m;
    }
    __syncthreads();
    auto load_block = [&](int q0, float (&dst)[RI_RB][RI_CPT]) {
#pragma unroll
        for (int r = 0; r < RI_RB; r++) {
            const float * row = S + (long long)(q0 + r) * C;
#pragma unroll
            for (int c = 0; c < RI_CPT; c++) {
                const int j = tid + RI_THREADS * c;
                dst[r][c] = (q0 + r < nq && j < C) ? row[j] : 0.0f;
            }
        }
    };
    float cur[RI_RB][RI_CPT], nxt[RI_RB][RI_CPT], acc[RI_CPT], mx[RI_CPT];
#pragma unroll
    for (int c = 0; c < RI_CPT; c++) { acc[c] = 0.0f; mx[c] = 0.0f; }
    load_block(0, cur);
    for (int q0 = 0, blk = 0; q0 < nq; q0 += RI_RB, blk ^= 1) {
        if (q0 + RI_RB < nq) load_block(q0 + RI_RB, nxt);
        float sl[RI_RB];
#pragma unroll
        for (int r = 0; r < RI_RB; r++) {
            const float m = q0 + r < nq ? sm_m[q0 + r] : 0.0f;
            sl[r] = 0.0f;
#pragma unroll
            for (int c = 0; c < RI_CPT; c++) {
                const int j = tid + RI_THREADS * c;
                cur[r][c] = j < C ? expf(__fsub_rn(cur[r][c], m)) : 0.0f;
                sl[r] = __fadd_rn(sl[r], cur[r][c]);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) sl[r] = __fadd_rn(sl[r], __shfl_xor_sync(0xffffffffu, sl[r], o));
        }
        if (lane == 0)
#pragma unroll
            for (int r = 0; r < RI_RB; r++) red[blk][r][warp] = sl[r];
        __syncthreads();
#pragma unroll
        for (int r = 0; r < RI_RB; r++) {
            const int q = q0 + r;
            if (q >= nq) break;
            float tot = red[blk][r][0];
#pragma unroll
            for (int w = 1; w < RI_THREADS / 32; w++) tot = __fadd_rn(tot, red[blk][r][w]);
            const float inv = softmax_inv(tot);
            if (tid == 0) { rmax[q] = sm_m[q]; rsum[q] = tot; }
#pragma unroll
            for (int c = 0; c < RI_CPT; c++) {       // aggregated in query order
                const float w = __fmul_rn(cur[r][c], inv);
                if (P.score_method == 0) { if (w > acc[c]) acc[c] = w; }
                else if (P.score_method == 1) acc[c] = __fadd_rn(acc[c], __fmul_rn(w, w));
                else acc[c] = __fadd_rn(acc[c], w);
                if (P.use_sensitivity && w > mx[c]) mx[c] = w;     // read only by sensitivity weighting
            }
        }
#pragma unroll
        for (int r = 0; r < RI_RB; r++)
#pragma unroll
            for (int c = 0; c < RI_CPT; c++) cur[r][c] = nxt[r][c];
    }
    float * imp = fs + u.imp_off + (long long)h * C;
    float * cmax = fs + u.imp_off + (long long)(P.H + h) * C;
    const float inv_m = __fdiv_rn(1.0f, (float)nq);
#pragma unroll
    for (int c = 0; c < RI_CPT; c++) {
        const int j = tid + RI_THREADS * c;
        if (j >= C) continue;
        float a = acc[c];
        if (P.score_method == 1) a = sqrtf(__fmul_rn(a, inv_m));
        else if (P.score_method == 2) a = __fmul_rn(a, inv_m);
        imp[j] = a;
        if (P.use_sensitivity) cmax[j] = mx[c];
    }
}

// X block of the refit: X[q][j] = S[q][sel[j]], the raw scores of the kept
// keys (the same values the scoring computed, bit for bit); one warp per row.
__global__ void __launch_bounds__(256) k_gather_x(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                  float * __restrict__ fs, const int * __restrict__ is) {
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y, nq = u.nq, t = u.t, C = u.C;
    const int * sel = is + u.sel_off;
    const float * S = fs + u.s_off + (long long)h * nq * C;
    float * X = fs + u.x_off + (long long)h * nq * t;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int q = blockIdx.x * 8 + warp; q < nq; q += gridDim.x * 8) {
        const float * row = S + (long long)q * C;
        float * xr = X + (long long)q * t;
        for (int j = lane; j < t; j += 32) xr[j] = row[sel[j]];
    }
    (void)P;
}

// Y_h [nq x dv] = A_h [nq x C] . V_h [C x dv]; 64x64 output tile per CTA.
__global__ void __launch_bounds__(ST) k_pv(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                           float * __restrict__ fs, int from_scores) {
    const kvc_unit u = units[blockIdx.z];
    const int h = blockIdx.y;
    const int dv = P.dv, ev = P.H * P.dv, nq = u.nq, C = u.C;
    const int tq = (nq + SB - 1) / SB, tn = (dv + SB - 1) / SB;
    if ((int)blockIdx.x >= tq * tn) return;
    const int q0 = (blockIdx.x / tn) * SB, n0 = (blockIdx.x % tn) * SB;
    const float * S = fs + u.s_off + (long long)h * nq * C;    // A, or raw scores A is formed from
    const float * rmax = fs + u.row_off + (long long)h * 2 * nq;
    const float * V = u.V + (long long)h * dv;
    float * Y = fs + u.y_off + (long long)h * nq * dv;

    __shared__ float As[SK][SB + 4];   // [k][row]
    __shared__ float Vs[SK][SB + 4];   // [k][col]
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int ar = tid >> 2, aq = q0 + ar;                    // the A row this thread stages
    const bool rs = from_scores && aq < nq;
    const float am = rs ? rmax[aq] : 0.0f, ainv = rs ? softmax_inv(rmax[nq + aq]) : 0.0f;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < C; k0 += SK) {
        // A tile: 64 rows x 32 k; thread -> row tid/4, 8 consecutive k
        {
            const int c = (tid & 3) * 8;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                int k = k0 + c + i;
                float a = 0.0f;
                if (aq < nq && k < C) {
                    a = S[(long long)aq * C + k];
                    if (from_scores) a = softmax_entry(a, am, ainv);
                }
                As[c + i][ar] = a;
            }
        }
        // V tile: 32 k x 64 cols; thread -> k tid/8, 8 consecutive cols
        {
            int r = tid >> 3, c = (tid & 7) * 8;
            int k = k0 + r;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                int n = n0 + c + i;
                Vs[r][c + i] = (k < C && n < dv) ? V[(long long)k * ev + n] : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < SK; kk++) {
            float4 a = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
            float4 b = *reinterpret_cast<const float4 *>(&Vs[kk][tx * 4]);
            float av[4] = {a.x, a.y, a.z, a.w};
            float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int q = q0 + ty * 4 + i;
        if (q >= nq) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int n = n0 + tx * 4 + j;
            if (n < dv) Y[(long long)q * dv + n] = acc[i][j];
        }
    }
}

// Row softmax of X = S[:, sel] + beta in place (math.h:83-100 via
// src/kv-compact-api.cpp:834-840); one warp per row.
__global__ void __launch_bounds__(256) k_softmax_x(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                   float * __restrict__ fs, const float * __restrict__ beta_all,
                                                   const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y;
    const int t = u.t, nq = u.nq;
    const kvc_layer_out lo = outs[u.layer];
    const float * beta = lo.beta + (long long)h * lo.t_total + u.out_off;
    float * X = fs + u.x_off + (long long)h * nq * t;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int q = blockIdx.x * nw + warp; q < nq; q += gridDim.x * nw) {
        float * row = X + (long long)q * t;
        float m = -INFINITY;
        bool first = true;
        for (int j = lane; j < t; j += 32) {
            float v = __fadd_rn(row[j], beta[j]);
            row[j] = v;
            if (first || v > m) { m = v; first = false; }
        }
        for (int o = 16; o; o >>= 1) { float v = __shfl_xor_sync(0xffffffffu, m, o); if (v > m) m = v; }
        float s = 0.0f;
        for (int j = lane; j < t; j += 32) {
            float e = expf(__fsub_rn(row[j], m));
            row[j] = e;
            s = __fadd_rn(s, e);
        }
        for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        float inv = __fdiv_rn(1.0f, __fadd_rn(s, 1e-12f));
        for (int j = lane; j < t; j += 32) row[j] = __fmul_rn(row[j], inv);
        if (lane == 0 && u.xs_off > 0) {     // kept for the chunk-merged quality metrics
            float * xs = fs + u.xs_off + (long long)h * 2 * nq;
            xs[q] = m;
            xs[nq + q] = s;
        }
    }
    (void)beta_all;
}

// X = softmax(S[:, sel]) without a bias (skip_beta): the gather of
// k_gather_x and the row softmax of k_softmax_x in one pass, one warp per
// row (the raw row block is never written to memory and read back). Adding a
// zero beta changes no exponential, so X is bit for bit that of the two
// kernels.
__global__ void __launch_bounds__(256) k_gather_softmax_x(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                          float * __restrict__ fs, const int * __restrict__ is) {
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y, nq = u.nq, t = u.t, C = u.C;
    const int * sel = is + u.sel_off;
    const float * S = fs + u.s_off + (long long)h * nq * C;
    float * X = fs + u.x_off + (long long)h * nq * t;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int q = blockIdx.x * 8 + warp; q < nq; q += gridDim.x * 8) {
        const float * src = S + (long long)q * C;
        float * row = X + (long long)q * t;
        float m = -INFINITY;
        bool first = true;
        for (int j = lane; j < t; j += 32) {
            const float v = src[sel[j]];
            row[j] = v;
            if (first || v > m) { m = v; first = false; }
        }
        for (int o = 16; o; o >>= 1) { float v = __shfl_xor_sync(0xffffffffu, m, o); if (v > m) m = v; }
        float sm = 0.0f;
        for (int j = lane; j < t; j += 32) {
            const float e = expf(__fsub_rn(row[j], m));
            row[j] = e;
            sm = __fadd_rn(sm, e);
        }
        for (int o = 16; o; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
        const float inv = __fdiv_rn(1.0f, __fadd_rn(sm, 1e-12f));
        for (int j = lane; j < t; j += 32) row[j] = __fmul_rn(row[j], inv);
        if (lane == 0 && u.xs_off > 0) {     // kept for the chunk-merged quality metrics
            float * xs = fs + u.xs_off + (long long)h * 2 * nq;
            xs[q] = m;
            xs[nq + q] = sm;
        }
    }
    (void)P;
}

// k_gather_softmax_x with the row in registers (t <= 32 R): each lane
// gathers its R values of S[q][sel[j]] (j = lane, lane + 32, ...) at once,
// with sel staged in shared memory for all the CTA's rows, and X is written
// once. Same order of every operation as k_gather_softmax_x (bit-identical).
template <int R>
__global__ void __launch_bounds__(256) k_gather_softmax_x_reg(const kvc_unit * __restrict__ units,
                                                              float * __restrict__ fs, const int * __restrict__ is) {
    const kvc_unit u = units[blockIdx.z];
    if (!u.active) return;
    const int h = blockIdx.y, nq = u.nq, t = u.t, C = u.C;
    __shared__ int ssel[32 * R];
    for (int j = threadIdx.x; j < t; j += 256) ssel[j] = is[u.sel_off + j];
    __syncthreads();
    const float * S = fs + u.s_off + (long long)h * nq * C;
    float * X = fs + u.x_off + (long long)h * nq * t;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int q = blockIdx.x * 8 + warp; q < nq; q += gridDim.x * 8) {
        const float * src = S + (long long)q * C;
        float v[R];
#pragma unroll
        for (int i = 0; i < R; i++) {
            const int j = lane + 32 * i;
            v[i] = j < t ? src[ssel[j]] : 0.0f;
        }
        float m = -INFINITY;
        bool first = true;
#pragma unroll
        for (int i = 0; i < R; i++)
            if (lane + 32 * i < t && (first || v[i] > m)) { m = v[i]; first = false; }
        for (int o = 16; o; o >>= 1) { float w = __shfl_xor_sync(0xffffffffu, m, o); if (w > m) m = w; }
        float sm = 0.0f;
#pragma unroll
        for (int i = 0; i < R; i++)
            if (lane + 32 * i < t) {
                v[i] = expf(__fsub_rn(v[i], m));
                sm = __fadd_rn(sm, v[i]);
            }
        for (int o = 16; o; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
        const float inv = __fdiv_rn(1.0f, __fadd_rn(sm, 1e-12f));
        float * row = X + (long long)q * t;
#pragma unroll
        for (int i = 0; i < R; i++)
            if (lane + 32 * i < t) row[lane + 32 * i] = __fmul_rn(v[i], inv);
        if (lane == 0 && u.xs_off > 0) {     // kept for the chunk-merged quality metrics
            float * xs = fs + u.xs_off + (long long)h * 2 * nq;
            xs[q] = m;
            xs[nq + q] = sm;
        }
    }
}

int kvc_launch_gather_softmax_x(const kvc_unit * d_units, int n_units, int max_nq, int max_t, const kvc_params_dev & P,
                                float * fs, const int * is, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    const int gx = (max_nq + 7) / 8 < 16 ? (max_nq + 7) / 8 : 16;
    if (max_t <= 256) k_gather_softmax_x_reg<8><<<dim3(gx, P.H, n_units), 256, 0, st>>>(d_units, fs, is);
    else if (max_t <= 512) k_gather_softmax_x_reg<16><<<dim3(gx, P.H, n_units), 256, 0, st>>>(d_units, fs, is);
    else k_gather_softmax_x<<<dim3(gx, P.H, n_units), 256, 0, st>>>(d_units, P, fs, is);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_score(const kvc_unit * d_units, int n_units, int max_nq, int max_cols,
                     const kvc_params_dev & P, float * fs, int mode, cudaStream_t st,
                     bool rows_aligned) {
    if (n_units <= 0) return KVC_OK;
    if (max_nq > 64 && rows_aligned) {
        const int tiles = ((max_nq + 127) / 128) * ((max_cols + 127) / 128);
        const size_t sm = kvc_score_async_smem();
        KVC_CUDA(cudaFuncSetAttribute(k_score_async, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        k_score_async<<<dim3(tiles, P.H, n_units), ST, sm, st>>>(d_units, P, fs, mode);
    } else if (max_nq > 64) {
        const int tiles = ((max_nq + 127) / 128) * ((max_cols + 127) / 128);
        k_score<128><<<dim3(tiles, P.H, n_units), ST, 0, st>>>(d_units, P, fs, mode);
    } else {
        const int tiles = ((max_nq + 63) / 64) * ((max_cols + 255) / 256);
        k_score<64><<<dim3(tiles, P.H, n_units), ST, 0, st>>>(d_units, P, fs, mode);
    }
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_gather_x(const kvc_unit * d_units, int n_units, int max_nq, const kvc_params_dev & P, float * fs,
                        const int * is, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    const int gx = (max_nq + 7) / 8 < 16 ? (max_nq + 7) / 8 : 16;
    k_gather_x<<<dim3(gx, P.H, n_units), 256, 0, st>>>(d_units, P, fs, is);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_score_tile_keys(int max_nq, bool rows_aligned) {
    return (max_nq > 64) ? 128 : 256;            // k_score_async / k_score<128>: 128; k_score<64>: 256
    (void)rows_aligned;
}

int kvc_launch_softmax_importance(const kvc_unit * d_units, int n_units, int max_nq, int max_C, int tile_keys,
                                  const kvc_params_dev & P, float * fs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    if (tile_keys > 0 && max_C <= RI_THREADS * RI_MAX_CPT && max_nq <= SMI_ROWS) {
        const dim3 grid(P.H, n_units);
        const int cpt = (max_C + RI_THREADS - 1) / RI_THREADS;
        if (cpt <= 2) k_row_importance<1, 4, 2><<<grid, RI_THREADS, 0, st>>>(d_units, P, fs, tile_keys);
        else if (cpt <= 4) k_row_importance<1, 4, 4><<<grid, RI_THREADS, 0, st>>>(d_units, P, fs, tile_keys);
        else if (cpt <= 5) k_row_importance<1, 4, 5><<<grid, RI_THREADS, 0, st>>>(d_units, P, fs, tile_keys);
        else k_row_importance<1, 4, 8><<<grid, RI_THREADS, 0, st>>>(d_units, P, fs, tile_keys);
        KVC_CUDA(cudaGetLastError());
        return KVC_OK;
    }
    k_softmax_importance<<<dim3(P.H, n_units), 256, 0, st>>>(d_units, P, fs);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_pv(const kvc_unit * d_units, int n_units, int max_nq, const kvc_params_dev & P,
                  float * fs, bool from_scores, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    if (kvc_pv_tc_ok(max_nq, P.dv)) return kvc_launch_pv_tc(d_units, n_units, P, fs, from_scores, st);
    int tiles = ((max_nq + SB - 1) / SB) * ((P.dv + SB - 1) / SB);
    k_pv<<<dim3(tiles, P.H, n_units), ST, 0, st>>>(d_units, P, fs, from_scores ? 1 : 0);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_softmax_x(const kvc_unit * d_units, int n_units, int max_nq, const kvc_params_dev & P,
                         float * fs, const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    int rows_per_cta = 8;
    int gx = (max_nq + rows_per_cta - 1) / rows_per_cta;
    k_softmax_x<<<dim3(gx, P.H, n_units), 256, 0, st>>>(d_units, P, fs, nullptr, d_outs);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
