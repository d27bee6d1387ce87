// metrics.cu — kv_compact_stats quality fields (src/kv-compact-api.cpp:239-325).
//
// For each of the first min(H,4) heads and min(n_q,32) reference queries:
// the attention output over all T original keys and values, and the output
// over the kept keys (scores + beta) and refitted values C_v; then cosine,
// MSE and argmax agreement. One CTA per (head, query) pair; the per-pair
// triples are summed on the host in the reference's (head, query) order.
#include "kvc_internal.h"

#include <math.h>

namespace {
__device__ float blk_max(float v, float * sh) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = -INFINITY;
    for (int i = 0; i < nw; i++) r = fmaxf(r, sh[i]);
    __syncthreads();
    return r;
}
__device__ float blk_sum(float v, float * sh) {
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = 0.0f;
    for (int i = 0; i < nw; i++) r = __fadd_rn(r, sh[i]);
    __syncthreads();
    return r;
}

// softmax over n scores in buf (in place) then out[d] = sum_j w_j * row_j[d]
__device__ void attend(float * buf, int n, const float * rows, long long row_stride, const int * idx,
                       int dv, float * out, float * sh) {
    float m = -INFINITY;
    for (int j = threadIdx.x; j < n; j += blockDim.x) m = fmaxf(m, buf[j]);
    m = blk_max(m, sh);
    float s = 0.0f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        float e = expf(__fsub_rn(buf[j], m));
        buf[j] = e;
        s = __fadd_rn(s, e);
    }
    s = blk_sum(s, sh);
    const float inv = __fdiv_rn(1.0f, __fadd_rn(s, 1e-12f));
    __syncthreads();
    for (int d = threadIdx.x; d < dv; d += blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < n; j++) {
            long long r = idx ? (long long)idx[j] : (long long)j;
            acc = fmaf(__fmul_rn(buf[j], inv), rows[r * row_stride + d], acc);
        }
        out[d] = acc;
    }
    __syncthreads();
}
}  // namespace

// Q: [nq x H*dk] top-level queries; sel: [t] global positions; beta [H][t];
// cv [H][t][dv]; res: [pairs][3]; scratch: [pairs][max(T,t)] floats.
__global__ void __launch_bounds__(256) k_metrics(const float * __restrict__ K, const float * __restrict__ V,
                                                 const float * __restrict__ Q, int T, int nq, int H, int dk,
                                                 int dv, const int * __restrict__ sel,
                                                 const float * __restrict__ beta, const float * __restrict__ cv,
                                                 int t, float isd, float * __restrict__ scratch,
                                                 float * __restrict__ res) {
    const int mq = nq < 32 ? nq : 32;
    const int pair = blockIdx.x;
    const int h = pair / mq, qi = pair % mq;
    const int ek = H * dk, ev = H * dv;
    const float * q = Q + (long long)qi * ek + (long long)h * dk;
    float * buf = scratch + (long long)pair * (T > t ? T : t);
    __shared__ float sh[32];
    __shared__ float oo[KVC_MAX_D], co[KVC_MAX_D];

    for (int j = threadIdx.x; j < T; j += blockDim.x) {
        const float * k = K + (long long)j * ek + (long long)h * dk;
        float acc = 0.0f;
        for (int d = 0; d < dk; d++) acc = __fadd_rn(acc, __fmul_rn(q[d], k[d]));
        buf[j] = __fmul_rn(acc, isd);
    }
    __syncthreads();
    attend(buf, T, V + (long long)h * dv, ev, nullptr, dv, oo, sh);

    const float * bh = beta + (long long)h * t;
    for (int j = threadIdx.x; j < t; j += blockDim.x) {
        const float * k = K + (long long)sel[j] * ek + (long long)h * dk;
        float acc = 0.0f;
        for (int d = 0; d < dk; d++) acc = __fadd_rn(acc, __fmul_rn(q[d], k[d]));
        buf[j] = __fadd_rn(__fmul_rn(acc, isd), bh[j]);
    }
    __syncthreads();
    attend(buf, t, cv + (long long)h * t * dv, dv, nullptr, dv, co, sh);

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
        res[pair * 3 + 0] = __fdiv_rn(dp, __fadd_rn(sqrtf(__fmul_rn(no, nc)), 1e-8f));
        res[pair * 3 + 1] = __fdiv_rn(mse, (float)dv);
        res[pair * 3 + 2] = (ao == ac) ? 1.0f : 0.0f;
    }
}

int kvc_metric_pairs(int H, int nq) { return (H < 4 ? H : 4) * (nq < 32 ? nq : 32); }

int kvc_launch_metrics(const float * K, const float * V, const float * Q, int T, int nq, int H, int dk, int dv,
                       const int * sel, const float * beta, const float * cv, int t, float isd,
                       float * scratch, float * res, cudaStream_t st) {
    int pairs = kvc_metric_pairs(H, nq);
    if (pairs <= 0) return KVC_OK;
    k_metrics<<<pairs, 256, 0, st>>>(K, V, Q, T, nq, H, dk, dv, sel, beta, cv, t, isd, scratch, res);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
