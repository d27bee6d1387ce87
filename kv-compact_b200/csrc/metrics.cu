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
//
// Chunk-merged form (the pipeline already holds what the metric needs). When
// every chunk of a layer scored the layer's own reference queries, chunk k
// has, per (head, query): the row max m_k and exp-sum s_k of its scores, its
// attention output Y_k = softmax_k(S) V_k, and the same three for the kept
// keys, m'_k, s'_k and X_k C_v,k with X = softmax(S[:, sel] + beta). A softmax
// over all T keys is the exp(m_k - M)-weighted merge of the chunk softmaxes
// (M = max_k m_k), so
//   orig = sum_k e^(m_k-M) (s_k + 1e-12) Y_k / (sum_k e^(m_k-M) s_k + 1e-12)
// and comp likewise from the kept-key terms. k_metric_partial stores the
// per-chunk terms after the last solve, k_metric_merge combines them in fp64
// and finishes cosine/MSE/argmax like k_mfinal. This is the same quantity in a
// different summation order (agreement with the direct form ~1e-6 relative);
// it replaces a second pass over all T keys and values per layer.
#include "kvc_internal.h"

#include <math.h>

namespace {
constexpr int MQ = 32;       // queries per head
constexpr int MK = 128;      // keys per scoring CTA
constexpr int MD = 32;       // d slab
constexpr int PK = 32;       // keys per value tile
constexpr int MWLD = PK + 4;  // row stride of a staged X tile (floats)

// 16-byte asynchronous global -> shared copy of `bytes` (0..16) valid bytes, the rest zero-filled.
__device__ __forceinline__ void mcp16(void * smem, const void * gmem, int bytes) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(sa), "l"(gmem), "r"(bytes) : "memory");
}
// dynamic shared memory of k_metric_partial: two X tiles and two C_v tiles
inline size_t metric_partial_smem(bool hi) {
    return (size_t)(2 * 32 * (32 + 4) + 2 * 32 * (hi ? 256 : 128)) * sizeof(float);
}
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

// cosine, MSE and argmax agreement of one (head, query) pair from its two
// d_v-vectors in shared memory (src/kv-compact-api.cpp:285-318); thread 0.
__device__ void metric_triple(const float * oo, const float * co, int dv, float * res) {
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
    res[0] = __fdiv_rn(dp, __fadd_rn(sqrtf(__fmul_rn(no, nc)), 1e-8f));
    res[1] = __fdiv_rn(mse, (float)dv);
    res[2] = (ao == ac) ? 1.0f : 0.0f;
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
    if (threadIdx.x == 0) metric_triple(oo, co, dv, a.res + pair * 3);
}

// ---- chunk-merged form ------------------------------------------------------
// Record of one (chunk, head, query): m, s, m', s', Y[d_v], (X C_v)[d_v];
// records are laid out [chunk][head][query].
__host__ __device__ inline int metric_rec(int dv) { return 4 + 2 * dv; }

// grid (units, min(H,4)): per-chunk terms of the first min(n_q,32) queries.
// Runs for every unit of a layer that has a record buffer, active or not
// (a unit that stopped refining keeps the X and C_v of its last solve).
// HI: d_v > 128, each thread also owns columns 128 + 4 cg .. +3 (otherwise
// those accumulators would only ever add products of zero).
template <bool HI>
__global__ void __launch_bounds__(256, HI ? 2 : 4) k_metric_partial(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                        const float * __restrict__ fs,
                                                        const kvc_layer_out * __restrict__ outs) {
    constexpr int NC = HI ? 8 : 4;
    const kvc_unit u = units[blockIdx.x];
    const kvc_layer_out lo = outs[u.layer];
    if (lo.mpart == nullptr || u.qmode != 0) return;
    const int h = blockIdx.y, nq = u.nq, t = u.t, dv = P.dv;
    const int mh = P.H < 4 ? P.H : 4, mq = nq < MQ ? nq : MQ;
    const int rec = metric_rec(dv);
    float * out = lo.mpart + ((long long)u.chunk * mh + h) * mq * rec;
    const float * rmax = fs + u.row_off + (long long)h * 2 * nq;
    const float * xs = fs + u.xs_off + (long long)h * 2 * nq;
    const float * Y = fs + u.y_off + (long long)h * nq * dv;
    const float * X = fs + u.x_off + (long long)h * nq * t;
    const float * cv = lo.cv + ((long long)h * lo.t_total + u.out_off) * dv;
    const int tid = threadIdx.x;
    if (tid < mq) {
        out[(long long)tid * rec + 0] = rmax[tid];
        out[(long long)tid * rec + 1] = rmax[nq + tid];
        out[(long long)tid * rec + 2] = xs[tid];
        out[(long long)tid * rec + 3] = xs[nq + tid];
    }
    for (int e = tid; e < mq * dv; e += 256) {
        const int q = e / dv, c = e % dv;
        out[(long long)q * rec + 4 + c] = Y[(long long)q * dv + c];
    }
    // (X C_v)[q][c]: 8 query groups x 32 column groups, 4 queries x 4 (or 8)
    // columns a thread. Tiles of PK kept keys — X's [q][j] rows and C_v's
    // [j][c] rows, both in their own layout — arrive by 16-byte asynchronous
    // copies into two buffers, the next tile in flight while the current one
    // is multiplied; keys are summed in the same order either way.
    constexpr int DVP = HI ? 2 * 128 : 128;
    extern __shared__ __align__(16) float msm[];
    float * Wt = msm;                                  // [2][MQ][MWLD]
    float * Vt = msm + 2 * MQ * MWLD;                  // [2][PK][DVP]
    const int qg = tid >> 5, cg = tid & 31;
    float acc[4][NC];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < NC; c++) acc[i][c] = 0.0f;
    const bool vec = (t % 4 == 0) && (dv % 4 == 0) && ((((uintptr_t)X) | ((uintptr_t)cv)) & 15) == 0;
    auto stage = [&](int j0, int b) {
        float * W = Wt + b * MQ * MWLD;
        float * V = Vt + b * PK * DVP;
        if (vec) {
            for (int e = tid; e < MQ * (PK / 4); e += 256) {
                const int qq = e / (PK / 4), c4 = e % (PK / 4), j = j0 + 4 * c4;
                const int bytes = (qq < mq && j < t) ? 4 * min(4, t - j) : 0;
                mcp16(W + qq * MWLD + 4 * c4, bytes ? X + (long long)qq * t + j : X, bytes);
            }
            for (int e = tid; e < PK * (dv / 4); e += 256) {
                const int jj = e / (dv / 4), c4 = e % (dv / 4), j = j0 + jj;
                const int bytes = j < t ? 16 : 0;
                mcp16(V + jj * DVP + 4 * c4, bytes ? cv + (long long)j * dv + 4 * c4 : cv, bytes);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        } else {
            for (int e = tid; e < MQ * PK; e += 256) {
                const int qq = e / PK, jj = e % PK;
                W[qq * MWLD + jj] = (qq < mq && j0 + jj < t) ? X[(long long)qq * t + j0 + jj] : 0.0f;
            }
            for (int e = tid; e < PK * dv; e += 256) {
                const int jj = e / dv, c = e % dv;
                V[jj * DVP + c] = (j0 + jj < t) ? cv[(long long)(j0 + jj) * dv + c] : 0.0f;
            }
        }
    };
    const int nst = (t + PK - 1) / PK;
    if (nst > 0) stage(0, 0);
    for (int st = 0; st < nst; st++) {
        const int j0 = st * PK, b = st & 1;
        if (st + 1 < nst) stage(j0 + PK, b ^ 1);
        if (vec) {
            if (st + 1 < nst) asm volatile("cp.async.wait_group 1;" ::: "memory");
            else asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const float * W = Wt + b * MQ * MWLD;
        const float * V = Vt + b * PK * DVP;
        const int jn = min(PK, t - j0);
#pragma unroll 4
        for (int jj = 0; jj < jn; jj++) {
            float wv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) wv[i] = W[(4 * qg + i) * MWLD + jj];
            float vv[NC];
            if (4 * cg < dv) {
                const float4 v4 = *reinterpret_cast<const float4 *>(V + jj * DVP + 4 * cg);
                vv[0] = v4.x; vv[1] = v4.y; vv[2] = v4.z; vv[3] = v4.w;
            } else {
                vv[0] = vv[1] = vv[2] = vv[3] = 0.0f;
            }
            if (HI) {
                if (128 + 4 * cg < dv) {
                    const float4 v4 = *reinterpret_cast<const float4 *>(V + jj * DVP + 128 + 4 * cg);
                    vv[NC - 4] = v4.x; vv[NC - 3] = v4.y; vv[NC - 2] = v4.z; vv[NC - 1] = v4.w;
                } else {
                    vv[NC - 4] = vv[NC - 3] = vv[NC - 2] = vv[NC - 1] = 0.0f;
                }
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int c = 0; c < NC; c++) acc[i][c] = fmaf(wv[i], vv[c], acc[i][c]);
        }
        __syncthreads();                            // buffer b is restaged two tiles later
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int q = 4 * qg + i;
        if (q >= mq) continue;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int col = (c < 4) ? 4 * cg + c : 128 + 4 * cg + (c - 4);
            if (col < dv) out[(long long)q * rec + 4 + dv + col] = acc[i][c];
        }
    }
}

// grid min(H,4) * min(n_q,32): merge the chunk records of one (head, query)
// pair in fp64, then the metric triple. The per-chunk weights
// e^(m_k - M) (s_k + 1e-12) (and their kept-key counterparts) are computed
// once into shared memory (up to MERGE_SMEM_CHUNKS chunks; beyond that they
// are recomputed per column).
constexpr int MERGE_SMEM_CHUNKS = 2048;

__device__ __forceinline__ void metric_merge_pair(const float * __restrict__ mpart, int n_chunks, int mh, int mq,
                                                  int dv, float * __restrict__ res, const int pair) {
    const int h = pair / mq, q = pair % mq;
    const int rec = metric_rec(dv);
    const long long cstride = (long long)mh * mq * rec;
    const float * r0 = mpart + ((long long)h * mq + q) * rec;
    extern __shared__ double wsh[];              // [2][n_chunks] orig / comp weights
    __shared__ float red[2][32];
    __shared__ double dred[2][32];
    __shared__ float oo[KVC_MAX_D], co[KVC_MAX_D];
    float M = -INFINITY, Mc = -INFINITY;
    for (int k = threadIdx.x; k < n_chunks; k += blockDim.x) {
        M = fmaxf(M, r0[k * cstride + 0]);
        Mc = fmaxf(Mc, r0[k * cstride + 2]);
    }
    for (int o = 16; o; o >>= 1) {
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        Mc = fmaxf(Mc, __shfl_xor_sync(0xffffffffu, Mc, o));
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) { red[0][w] = M; red[1][w] = Mc; }
    __syncthreads();
    M = red[0][0];
    Mc = red[1][0];
    for (int i = 1; i < nw; i++) { M = fmaxf(M, red[0][i]); Mc = fmaxf(Mc, red[1][i]); }
    const bool cached = n_chunks <= MERGE_SMEM_CHUNKS;
    double d_o = 0.0, d_c = 0.0;                 // denominators: sum_k e^(m_k - M) s_k
    for (int k = threadIdx.x; k < n_chunks; k += blockDim.x) {
        const float * r = r0 + k * cstride;
        const double eo = exp((double)r[0] - (double)M), ec = exp((double)r[2] - (double)Mc);
        d_o += eo * (double)r[1];
        d_c += ec * (double)r[3];
        if (cached) {
            wsh[k] = eo * ((double)r[1] + 1e-12);
            wsh[n_chunks + k] = ec * ((double)r[3] + 1e-12);
        }
    }
    for (int o = 16; o; o >>= 1) {
        d_o += __shfl_xor_sync(0xffffffffu, d_o, o);
        d_c += __shfl_xor_sync(0xffffffffu, d_c, o);
    }
    if (lane == 0) { dred[0][w] = d_o; dred[1][w] = d_c; }
    __syncthreads();
    d_o = 0.0;
    d_c = 0.0;
    for (int i = 0; i < nw; i++) { d_o += dred[0][i]; d_c += dred[1][i]; }
    for (int c = threadIdx.x; c < dv; c += blockDim.x) {
        double no = 0.0, nc = 0.0;
        for (int k = 0; k < n_chunks; k++) {
            const float * r = r0 + k * cstride;
            double wo, wc;
            if (cached) {
                wo = wsh[k];
                wc = wsh[n_chunks + k];
            } else {
                wo = exp((double)r[0] - (double)M) * ((double)r[1] + 1e-12);
                wc = exp((double)r[2] - (double)Mc) * ((double)r[3] + 1e-12);
            }
            no = fma(wo, (double)r[4 + c], no);
            nc = fma(wc, (double)r[4 + dv + c], nc);
        }
        oo[c] = (float)(no / (d_o + 1e-12));
        co[c] = (float)(nc / (d_c + 1e-12));
    }
    __syncthreads();
    if (threadIdx.x == 0) metric_triple(oo, co, dv, res + pair * 3);
}

__global__ void __launch_bounds__(256) k_metric_merge(const float * __restrict__ mpart, int n_chunks, int mh,
                                                      int mq, int dv, float * __restrict__ res) {
    metric_merge_pair(mpart, n_chunks, mh, mq, dv, res, blockIdx.x);
}

// Several layers' merges in one launch (grid.y = layer): the per-layer
// launches each ran one short wave of min(H,4) x min(n_q,32) CTAs.
constexpr int MERGE_BATCH = 32;
struct kvc_merge_batch {
    const float * mpart[MERGE_BATCH];
    float * res[MERGE_BATCH];
    int n_chunks[MERGE_BATCH];
};

__global__ void __launch_bounds__(256) k_metric_merge_batch(const kvc_merge_batch b, int mh, int mq, int dv) {
    const int l = blockIdx.y;
    metric_merge_pair(b.mpart[l], b.n_chunks[l], mh, mq, dv, b.res[l], blockIdx.x);
}

int kvc_launch_metric_merge(const float * mpart, int n_chunks, int H, int nq, int dv, float * res, cudaStream_t st);

int kvc_launch_metric_merge_batch(const float * const * mparts, const int * n_chunks, float * const * res, int n,
                                  int H, int nq, int dv, cudaStream_t st) {
    const int mh = H < 4 ? H : 4, mq = nq < 32 ? nq : 32;
    if (mh * mq <= 0) return KVC_OK;
    for (int l = 0; l < n; l++)
        if (n_chunks[l] > MERGE_SMEM_CHUNKS) {        // uncached weights: one launch per layer
            for (int i = 0; i < n; i++) {
                int rc = kvc_launch_metric_merge(mparts[i], n_chunks[i], H, nq, dv, res[i], st);
                if (rc) return rc;
            }
            return KVC_OK;
        }
    for (int l0 = 0; l0 < n; l0 += MERGE_BATCH) {
        kvc_merge_batch b;
        memset(&b, 0, sizeof(b));
        const int nl = n - l0 < MERGE_BATCH ? n - l0 : MERGE_BATCH;
        int max_chunks = 1;
        for (int i = 0; i < nl; i++) {
            b.mpart[i] = mparts[l0 + i];
            b.res[i] = res[l0 + i];
            b.n_chunks[i] = n_chunks[l0 + i];
            if (n_chunks[l0 + i] <= 0) return KVC_ERR_SHAPE;
            if (n_chunks[l0 + i] > max_chunks) max_chunks = n_chunks[l0 + i];
        }
        const size_t sm = 2 * (size_t)max_chunks * sizeof(double);     // every layer's weights cached
        k_metric_merge_batch<<<dim3(mh * mq, nl), 256, sm, st>>>(b, mh, mq, dv);
        KVC_CUDA(cudaGetLastError());
    }
    return KVC_OK;
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

size_t kvc_metric_partial_floats(int n_chunks, int H, int nq, int dv) {
    const long long mh = H < 4 ? H : 4, mq = nq < 32 ? nq : 32;
    return (size_t)(n_chunks * mh * mq * metric_rec(dv));
}

int kvc_launch_metric_partial(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, const float * fs,
                              const kvc_layer_out * d_outs, cudaStream_t st) {
    const int mh = P.H < 4 ? P.H : 4;
    if (n_units <= 0 || mh <= 0) return KVC_OK;
    if (P.dv > 128) {
        KVC_CUDA(cudaFuncSetAttribute(k_metric_partial<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)metric_partial_smem(true)));
        k_metric_partial<true><<<dim3(n_units, mh), 256, metric_partial_smem(true), st>>>(d_units, P, fs, d_outs);
    } else {
        k_metric_partial<false><<<dim3(n_units, mh), 256, metric_partial_smem(false), st>>>(d_units, P, fs, d_outs);
    }
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_metric_merge(const float * mpart, int n_chunks, int H, int nq, int dv, float * res, cudaStream_t st) {
    const int mh = H < 4 ? H : 4, mq = nq < 32 ? nq : 32;
    if (mh * mq <= 0 || n_chunks <= 0) return KVC_OK;
    const size_t sm = n_chunks <= MERGE_SMEM_CHUNKS ? 2 * (size_t)n_chunks * sizeof(double) : 0;
    k_metric_merge<<<mh * mq, 256, sm, st>>>(mpart, n_chunks, mh, mq, dv, res);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
