/*
 * kv-compact-accel-cuda.h — the compaction library's accelerator seam on CUDA.
 *
 * Same entry points, argument meaning and return convention (0 = done,
 * -1 = no usable device) as the reference's HIP seam
 * (fabiantax/kv-compact include/kv-compact-accel.h:22-55), renamed
 * kv_compact_hip_* -> kv_compact_cuda_*. All pointers are HOST pointers;
 * each call stages its operands to the current CUDA device (sm_100a) and
 * copies the result back. The scoring entry points produce the reference's
 * CPU-path values bit for bit (sequential fp32 dot products, then the scale).
 *
 * A build of the reference that defines the HIP seam can link against
 * libkvc.so by mapping each kv_compact_hip_* name onto the kv_compact_cuda_*
 * entry point of the same arguments (a macro or a one-line forwarding
 * function per name).
 */
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

/* 1 when a device that runs the library's sm_100a kernels is present
 * (reference kv-compact-accel.h:22). */
int kv_compact_cuda_available(void);

/* C[m x n] = scale * A[m x k] B[n x k]^T (reference kv-compact-accel.h:24-26). */
int kv_compact_cuda_mat_mul_ABt_scaled(const float * A, const float * B, float * C,
                                       int m, int n, int k, float scale);

/* scores_out[h][qi*T + ki] = scale * Q_ref[qi, h, :] . K_all[ki, h, :]
 * for every head (reference kv-compact-accel.h:38-40). */
int kv_compact_cuda_score_all_heads(const float * Q_ref, const float * K_all, float ** scores_out,
                                    int n_q, int T, int n_head_kv, int d_k, float scale);

/* Y_out[h] = W_per_head[h] (n_q x T) . V_h (T x d_v), V_h the head-h columns
 * of V_all [T x n_head_kv*d_v] (reference kv-compact-accel.h:50-52). */
int kv_compact_cuda_refit_target_all_heads(const float * const * W_per_head, const float * V_all,
                                           float ** Y_out, int n_q, int T, int n_head_kv, int d_v);

/* Release the device buffers the seam keeps between calls
 * (reference kv-compact-accel.h:55). */
void kv_compact_cuda_pool_free(void);

/* kv_compact_cuda_score_all_heads for callers that cannot let the library
 * allocate device memory (an engine that has reserved all of HBM for its own
 * allocator, or a path that must not pay cudaMalloc's latency and implicit
 * synchronisation). No counterpart in the reference. Same arguments and the
 * same bit-identical scores; staging lives in a 16 MiB array compiled into
 * the library (held by every GPU that loads it), so it needs
 * n_q*H*d_k + T*H*d_k + H*n_q*T floats (each part rounded up to 64) <=
 * 4,194,304 and returns -13 with a message beyond that; -1 on bad arguments
 * (d_k > 256 among them) or no sm_100 device. The first call on a device looks up the array's
 * address (make it before any stream capture). Calls share the array: calls
 * from this process are serialised, calls overlapping on the GPU race. */
int kv_compact_cuda_score_all_heads_noalloc(const float * Q_ref, const float * K_all,
                                            float ** scores_out, int n_q, int T,
                                            int n_head_kv, int d_k, float scale);

#ifdef __cplusplus
}
#endif
