// metrics.cu — kv_compact_stats quality fields (src/kv-compact-api.cpp:239-325).
//
// For the first min(H,4) heads and min(n_q,32) reference queries: the
// attention output over all T original keys/values ("orig") and over the kept
// keys (scores + beta) with the refitted values C_v ("comp"); then cosine,
// MSE and argmax agreement per (head, query). The reference loops query by
// query; here the 32 queries of a head are processed together so every key
// and value row is read once per head:
//   k_mscore    scores of 32 queries x 128 keys per CTA, sequential fp32 dot
//               then the scale (+ beta for comp), as the reference computes them
//   k_msoftmax  one CTA per (side, head, query) row: max, exp, sum, normalise
//   k_mpv       split-K weighted sum of value rows, partial [32 x d_v] per CTA
//   k_mfinal    fixed-order reduction of the partials, cosine/MSE/argmax
// The per-pair triples are summed on the host in the reference's order.
#include "kvc_internal.h"

#include <math.h>

namespace {
constexpr int MQ = 32;       // queries per head
constexpr int MK = 128;      // keys per scoring CTA
constexpr int MD = 32;       // d slab
constexpr int PK = 32;       // keys per value tile
}  // namespace

struct kvc_metric_args {
    const float * K;       // [T x ek]
    const float * V;       // [T x ev]
    const float * Q;       // [nq x ek]
    const int * sel;       // [t] global positions
    const float * beta;    // [H][t]
    const float * cv;      // [H][t][dv]
    int T, t, nq, H, dk, dv, mh, mq, nsplit;
    float isd;
    float * S;             // [2][mh][mq][ld] scores -> weights
    float * part;          // [2][nsplit][mh][mq][dv]
    float * res;           // [mh*mq][3]
    long long ld;          // max(T, t)
};

__global__ void __launch_bounds__(256) k_mscore(kvc_metric_args a) {
    const int side = blockIdx.z, h = blockIdx.y;
    const int n = side == 0 ? a.T : a.t;
    const int j0 = blockIdx.x * MK;
    if (j0 >= n) return;
    const int ek = a.H * a.dk;
    __shared__ float Qs[MD][MQ + 4];
    __shared__ float Ks[MD][MK + 4];
    __shared__ const float * kp[MK];
    const int tid = threadIdx.x;
    if (tid < MK) {
        int j = j0 + tid;
        if (j < n) {
            long long row = side == 0 ? j : a.sel[j];
            kp[tid] = a.K + row * ek + (long long)h * a.dk;
        } else {
            kp[tid] = nullptr;
        }
    }
    __syncthreads();
    const int ty = tid >> 5, tx = tid & 31;   // 8 x 32 threads: 4 queries x 4 keys each
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    for (int d0 = 0; d0 < a.dk; d0 += MD) {
        for (int e = tid; e < MQ * MD; e += 256) {
            int q = e / MD, c = e % MD;
            Qs[c][q] = (q < a.mq && d0 + c < a.dk) ? a.Q[(long long)q * ek + (long long)h * a.dk + d0 + c] : 0.0f;
        }
        for (int e = tid; e < MK * MD; e += 256) {
            int r = e / MD, c = e % MD;
            const float * p = kp[r];
            Ks[c][r] = (p && d0 + c < a.dk) ? p[d0 + c] : 0.0f;
        }
        __syncthreads();
        const int kend = min(MD, a.dk - d0);
        for (int kk = 0; kk < kend; kk++) {
            float4 qv = *reinterpret_cast<const float4 *>(&Qs[kk][ty * 4]);
            float qa[4] = {qv.x, qv.y, qv.z, qv.w};
            float kb[4] = {Ks[kk][tx], Ks[kk][tx + 32], Ks[kk][tx + 64], Ks[kk][tx + 96]};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(qa[i], kb[j]));
        }
        __syncthreads();
    }
    const float * bh = a.beta + (long long)h * a.t;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int q = ty * 4 + i;
        if (q >= a.mq) continue;
        float * row = a.S + (((long long)side * a.mh + h) * a.mq + q) * a.ld;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int c = j0 + tx + 32 * j;
            if (c < n) {
                float s = __fmul_rn(acc[i][j], a.isd);
                if (side == 1) s = __fadd_rn(s, bh[c]);
                row[c] = s;
            }
        }
    }
}

__global__ void __launch_bounds__(1024) k_msoftmax(kvc_metric_args a) {
    const int side = blockIdx.z, h = blockIdx.y, q = blockIdx.x;
    const int n = side == 0 ? a.T : a.t;
    float * row = a.S + (((long long)side * a.mh + h) * a.mq + q) * a.ld;
    __shared__ float sh[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float m = -INFINITY;
    for (int j = threadIdx.x; j < n; j += blockDim.x) m = fmaxf(m, row[j]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sh[w] = m;
    __syncthreads();
    m = sh[0];
    for (int i = 1; i < nw; i++) m = fmaxf(m, sh[i]);
    __syncthreads();
    float s = 0.0f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        float e = expf(__fsub_rn(row[j], m));
        row[j] = e;
        s = __fadd_rn(s, e);
    }
    for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) sh[w] = s;
    __syncthreads();
    s = 0.0f;
    for (int i = 0; i < nw; i++) s = __fadd_rn(s, sh[i]);
    const float inv = __fdiv_rn(1.0f, __fadd_rn(s, 1e-12f));
    for (int j = threadIdx.x; j < n; j += blockDim.x) row[j] = __fmul_rn(row[j], inv);
}

// partial[side][split][h][q][c] = sum over the split's keys of w[q][j] * row_j[c].
// 256 threads = 8 query groups x 32 column groups; a thread owns queries
// 4qg..4qg+3 and columns 4cg..4cg+3 (+128 when d_v > 128): per key it reads
// one float4 of weights (broadcast in the warp) and one or two float4 of
// values, for 16 or 32 FMAs.
__global__ void __launch_bounds__(256) k_mpv(kvc_metric_args a) {
    const int side = blockIdx.z, h = blockIdx.y, split = blockIdx.x;
    const int n = side == 0 ? a.T : a.t;
    const long long per = (n + a.nsplit - 1) / a.nsplit;
    const long long jb = split * per, je = min((long long)n, jb + per);
    const int dv = a.dv, ev = a.H * a.dv;
    __shared__ __align__(16) float Ws[PK][MQ];
    __shared__ __align__(16) float Vs[PK][KVC_MAX_D];
    const float * W = a.S + ((long long)side * a.mh + h) * a.mq * a.ld;
    const int tid = threadIdx.x, qg = tid >> 5, cg = tid & 31;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < 8; c++) acc[i][c] = 0.0f;
    const bool hi = dv > 128;
    for (long long j0 = jb; j0 < je; j0 += PK) {
        for (int e = tid; e < MQ * PK; e += 256) {
            const int qq = e / PK, jj = e % PK;
            const long long j = j0 + jj;
            Ws[jj][qq] = (qq < a.mq && j < je) ? W[(long long)qq * a.ld + j] : 0.0f;
        }
        for (int e = tid; e < PK * dv; e += 256) {
            const int jj = e / dv, c = e % dv;
            const long long j = j0 + jj;
            float v = 0.0f;
            if (j < je) v = side == 0 ? a.V[j * ev + (long long)h * dv + c] : a.cv[((long long)h * a.t + j) * dv + c];
            Vs[jj][c] = v;
        }
        __syncthreads();
        const int jn = (int)min((long long)PK, je - j0);
        for (int jj = 0; jj < jn; jj++) {
            const float4 w4 = *reinterpret_cast<const float4 *>(&Ws[jj][4 * qg]);
            const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
            float vv[8];
            if (4 * cg < dv) {
                const float4 v4 = *reinterpret_cast<const float4 *>(&Vs[jj][4 * cg]);
                vv[0] = v4.x; vv[1] = v4.y; vv[2] = v4.z; vv[3] = v4.w;
            } else {
                vv[0] = vv[1] = vv[2] = vv[3] = 0.0f;
            }
            if (hi && 128 + 4 * cg < dv) {
                const float4 v4 = *reinterpret_cast<const float4 *>(&Vs[jj][128 + 4 * cg]);
                vv[4] = v4.x; vv[5] = v4.y; vv[6] = v4.z; vv[7] = v4.w;
            } else {
                vv[4] = vv[5] = vv[6] = vv[7] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int c = 0; c < 8; c++) acc[i][c] = fmaf(wv[i], vv[c], acc[i][c]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int q = 4 * qg + i;
        if (q >= a.mq) continue;
        float * out = a.part + ((((long long)side * a.nsplit + split) * a.mh + h) * a.mq + q) * dv;
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const int col = (c < 4) ? 4 * cg + c : 128 + 4 * cg + (c - 4);
            if (col < dv && (c < 4 || hi)) out[col] = acc[i][c];
        }
    }
}

__global__ void __launch_bounds__(256) k_mfinal(kvc_metric_args a) {
    const int pair = blockIdx.x;
    const int h = pair / a.mq, q = pair % a.mq;
    const int dv = a.dv;
    __shared__ float oo[KVC_MAX_D], co[KVC_MAX_D];
    for (int c = threadIdx.x; c < dv; c += blockDim.x) {
        float so = 0.0f, sc = 0.0f;
        for (int s = 0; s < a.nsplit; s++) {
            so = __fadd_rn(so, a.part[((((long long)0 * a.nsplit + s) * a.mh + h) * a.mq + q) * dv + c]);
            sc = __fadd_rn(sc, a.part[((((long long)1 * a.nsplit + s) * a.mh + h) * a.mq + q) * dv + c]);
        }
        oo[c] = so;
        co[c] = sc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float dp = 0.0f, no = 0.0f, nc = 0.0f, mse = 0.0f;
        for (int d = 0; d < dv; d++) {
            dp = __fadd_rn(dp, __fmul_rn(oo[d], co[d]));
            no = __fadd_rn(no, __fmul_rn(oo[d], oo[d]));
            nc = __fadd_rn(nc, __fmul_rn(co[d], co[d]));
        }
        for (int d = 0; d < dv; d++) {
            float df = __fsub_rn(oo[d], co[d]);
            mse = __fadd_rn(mse, __fmul_rn(df, df));
        }
        int ao = 0, ac = 0;
        for (int d = 1; d < dv; d++) {
            if (oo[d] > oo[ao]) ao = d;
            if (co[d] > co[ac]) ac = d;
        }
        a.res[pair * 3 + 0] = __fdiv_rn(dp, __fadd_rn(sqrtf(__fmul_rn(no, nc)), 1e-8f));
        a.res[pair * 3 + 1] = __fdiv_rn(mse, (float)dv);
        a.res[pair * 3 + 2] = (ao == ac) ? 1.0f : 0.0f;
    }
}

int kvc_metric_pairs(int H, int nq) { return (H < 4 ? H : 4) * (nq < 32 ? nq : 32); }

size_t kvc_metric_scratch_floats(int H, int nq, int T, int t, int dv) {
    const long long mh = H < 4 ? H : 4, mq = nq < 32 ? nq : 32;
    const long long ld = T > t ? T : t;
    const long long nsplit = 128;
    return (size_t)(2 * mh * mq * ld + 2 * nsplit * mh * mq * dv + mh * mq * 3 + 64);
}

int kvc_launch_metrics(const float * K, const float * V, const float * Q, int T, int nq, int H, int dk, int dv,
                       const int * sel, const float * beta, const float * cv, int t, float isd,
                       float * scratch, float * res, cudaStream_t st) {
    kvc_metric_args a;
    a.K = K; a.V = V; a.Q = Q; a.sel = sel; a.beta = beta; a.cv = cv;
    a.T = T; a.t = t; a.nq = nq; a.H = H; a.dk = dk; a.dv = dv;
    a.mh = H < 4 ? H : 4;
    a.mq = nq < 32 ? nq : 32;
    a.nsplit = 128;
    a.isd = isd;
    a.ld = T > t ? T : t;
    a.S = scratch;
    a.part = scratch + 2LL * a.mh * a.mq * a.ld;
    a.res = res;
    if (a.mh * a.mq <= 0) return KVC_OK;
    const int nblk = (int)((a.ld + MK - 1) / MK);
    k_mscore<<<dim3(nblk, a.mh, 2), 256, 0, st>>>(a);
    KVC_CUDA(cudaGetLastError());
    k_msoftmax<<<dim3(a.mq, a.mh, 2), 1024, 0, st>>>(a);
    KVC_CUDA(cudaGetLastError());
    k_mpv<<<dim3(a.nsplit, a.mh, 2), 256, 0, st>>>(a);
    KVC_CUDA(cudaGetLastError());
    k_mfinal<<<a.mh * a.mq, 128, 0, st>>>(a);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
