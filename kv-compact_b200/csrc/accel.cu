// accel.cu — the CUDA accelerator seam (include/kv-compact-accel-cuda.h),
// built on the engine's scoring (k_score) and refit-target (k_pv) kernels.
// Sizes are formed in size_t after the head width is bounded, and an error
// that follows queued copies drains the stream before returning (the copies
// read the caller's host buffers).
#include <limits.h>

#include <vector>

#include "../../include/kv-compact-accel-cuda.h"
#include "engine.h"

namespace {
enum { SLOT_SEAM = 4 };

kvc_params_dev seam_params(int H, int dk, int dv, float scale) {
    kvc_params_dev P;
    memset(&P, 0, sizeof(P));
    P.H = H;
    P.dk = dk;
    P.dv = dv;
    P.isd = scale;
    return P;
}

// Whether H heads of width d fit the kernels (d <= KVC_MAX_D, H*d an int).
bool width_ok(int H, int d) { return d <= KVC_MAX_D && (size_t)H * (size_t)d <= (size_t)INT_MAX; }

// Error return once work is queued on `st`.
int fail_after_queue(cudaStream_t st) {
    cudaStreamSynchronize(st);
    cudaGetLastError();
    return -1;
}

int put_unit(kvc_ctx * ctx, const kvc_unit & u) {
    if (ctx->units_cap < 1) {
        ctx->units_cap = 16;
        KVC_CUDA(cudaMalloc(&ctx->d_units, ctx->units_cap * sizeof(kvc_unit)));
    }
    KVC_CUDA(cudaMemcpyAsync(ctx->d_units, &u, sizeof(u), cudaMemcpyHostToDevice, ctx->stream));
    return KVC_OK;
}

// scores of H heads: S_h = scale * Q_h K_h^T, written to host buffers out[h].
int scores(const float * Q, const float * K, float ** out, int nq, int T, int H, int dk, float scale) {
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!width_ok(H, dk)) return -1;
    const int ek = H * dk;
    size_t nQ = ((size_t)nq * ek + 31) & ~31ULL, nK = ((size_t)T * ek + 31) & ~31ULL;
    size_t nS = (size_t)H * nq * (size_t)T;
    void * a;
    if (kvc_arena(ctx, SLOT_SEAM, (nQ + nK + nS) * 4, &a)) return -1;
    float * dQ = (float *)a;
    float * dK = dQ + nQ;
    float * dS = dK + nK;
    cudaStream_t st = ctx->stream;
    if (cudaMemcpyAsync(dQ, Q, (size_t)nq * ek * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail_after_queue(st);
    if (cudaMemcpyAsync(dK, K, (size_t)T * ek * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail_after_queue(st);
    kvc_unit u;
    memset(&u, 0, sizeof(u));
    u.K = dK;
    u.Q = dQ;
    u.C = T;
    u.t = T;
    u.nq = nq;
    u.active = 1;
    u.s_off = (long long)(dS - dQ);
    if (put_unit(ctx, u)) return fail_after_queue(st);
    kvc_params_dev P = seam_params(H, dk, dk, scale);
    if (kvc_launch_score(ctx->d_units, 1, nq, T, P, dQ, 0, st)) return fail_after_queue(st);
    ctx->launches += 1;
    for (int h = 0; h < H; h++)
        if (cudaMemcpyAsync(out[h], dS + (size_t)h * nq * T, (size_t)nq * T * 4, cudaMemcpyDeviceToHost, st) !=
            cudaSuccess)
            return fail_after_queue(st);
    return cudaStreamSynchronize(st) == cudaSuccess ? 0 : -1;
}
}  // namespace

extern "C" {

KVC_EXPORT int kv_compact_cuda_available(void) {
    int rc;
    return kvc_get_ctx(&rc) ? 1 : 0;
}

KVC_EXPORT int kv_compact_cuda_mat_mul_ABt_scaled(const float * A, const float * B, float * C, int m, int n, int k,
                                       float scale) {
    if (!A || !B || !C || m <= 0 || n <= 0 || k <= 0) return -1;
    float * out[1] = {C};
    return scores(A, B, out, m, n, 1, k, scale);
}

KVC_EXPORT int kv_compact_cuda_score_all_heads(const float * Q_ref, const float * K_all, float ** scores_out, int n_q,
                                    int T, int n_head_kv, int d_k, float scale) {
    if (!Q_ref || !K_all || !scores_out || n_q <= 0 || T <= 0 || n_head_kv <= 0 || d_k <= 0) return -1;
    return scores(Q_ref, K_all, scores_out, n_q, T, n_head_kv, d_k, scale);
}

KVC_EXPORT int kv_compact_cuda_refit_target_all_heads(const float * const * W, const float * V_all, float ** Y_out, int n_q,
                                           int T, int n_head_kv, int d_v) {
    if (!W || !V_all || !Y_out || n_q <= 0 || T <= 0 || n_head_kv <= 0 || d_v <= 0) return -1;
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!width_ok(n_head_kv, d_v)) return -1;
    const int H = n_head_kv, ev = H * d_v;
    size_t nW = ((size_t)H * n_q * (size_t)T + 31) & ~31ULL, nV = ((size_t)T * ev + 31) & ~31ULL;
    size_t nY = (size_t)H * n_q * d_v;
    void * a;
    if (kvc_arena(ctx, SLOT_SEAM, (nW + nV + nY) * 4, &a)) return -1;
    float * dW = (float *)a;
    float * dV = dW + nW;
    float * dY = dV + nV;
    cudaStream_t st = ctx->stream;
    for (int h = 0; h < H; h++)
        if (cudaMemcpyAsync(dW + (size_t)h * n_q * T, W[h], (size_t)n_q * T * 4, cudaMemcpyHostToDevice, st) !=
            cudaSuccess)
            return fail_after_queue(st);
    if (cudaMemcpyAsync(dV, V_all, (size_t)T * ev * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail_after_queue(st);
    kvc_unit u;
    memset(&u, 0, sizeof(u));
    u.V = dV;
    u.C = T;
    u.nq = n_q;
    u.active = 1;
    u.s_off = 0;
    u.y_off = (long long)(dY - dW);
    if (put_unit(ctx, u)) return fail_after_queue(st);
    kvc_params_dev P = seam_params(H, d_v, d_v, 1.0f);
    if (kvc_launch_pv(ctx->d_units, 1, n_q, P, dW, false, st)) return fail_after_queue(st);
    ctx->launches += 1;
    for (int h = 0; h < H; h++)
        if (cudaMemcpyAsync(Y_out[h], dY + (size_t)h * n_q * d_v, (size_t)n_q * d_v * 4, cudaMemcpyDeviceToHost,
                            st) != cudaSuccess)
            return fail_after_queue(st);
    return cudaStreamSynchronize(st) == cudaSuccess ? 0 : -1;
}

KVC_EXPORT void kv_compact_cuda_pool_free(void) {
    int rc;
    kvc_ctx * ctx = kvc_get_ctx(&rc);
    if (!ctx) return;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaStreamSynchronize(ctx->stream);
    for (int s = 0; s < (int)(sizeof(ctx->arena) / sizeof(ctx->arena[0])); s++) {
        if (ctx->arena[s]) cudaFree(ctx->arena[s]);
        ctx->arena[s] = nullptr;
        ctx->arena_cap[s] = 0;
    }
    kvc_hpool_release();
}

}  // extern "C"
