/*
 * kvc-batched.h — device-resident, whole-model compaction (no reference
 * counterpart: the reference is called once per layer with host arrays; this
 * entry point runs every filtered layer of a model in one batched pass over
 * caches that already live in GPU memory).
 *
 * Semantics per layer are exactly kv_compact_quantized() of
 * kv-compact-api.h with the same params (dequant -> compact -> requant), and
 * params->layer_filter, when set, decides which layers are compacted, as the
 * reference's callers do with kv_compact_should_compact_layer().
 *
 * All pointers in kvc_layer_desc / kvc_layer_result are DEVICE pointers of
 * the current CUDA device. The library's work runs on a blocking stream, so
 * it starts after all work the caller queued on the legacy default stream;
 * inputs written on other non-blocking streams must be synchronised by the
 * caller first. Calls return after the work has completed.
 *
 * Limits: d_k, d_v <= 256; min(n_q, t) <= 24576 per chunk with skip_beta
 * and no OMP selection, <= 3072 otherwise; H <= 64 with use_sensitivity.
 * Violations return -13.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "kv-compact-api.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kvc_model_desc {
    int    n_layers;
    int    T;            /* cache positions per layer */
    int    n_head_kv;
    int    d_k;
    int    d_v;
    int    k_type;       /* KV_TYPE_* of the K rows */
    int    v_type;       /* KV_TYPE_* of the V rows */
    size_t k_row_bytes;  /* bytes per K row (n_head_kv*d_k values) */
    size_t v_row_bytes;
} kvc_model_desc;

typedef struct kvc_layer_desc {
    const void *  K;      /* device [T_l x k_row_bytes] */
    const void *  V;      /* device [T_l x v_row_bytes] */
    const float * Q_ref;  /* device [n_q x n_head_kv*d_k] fp32, or NULL (cheap queries) */
    int           n_q;
    int           n_tokens; /* T_l, this layer's cache positions; 0 = model->T. Layers
                               of different lengths (e.g. slices of a model's layers
                               on one GPU) share one call; R-KV weighting
                               (params->reasoning) needs every T_l = model->T */
} kvc_layer_desc;

typedef struct kvc_layer_result {
    int       t;                 /* kept positions (0 for filtered-out layers) */
    int *     selected_indices;  /* device [t] ascending positions */
    float *   beta;              /* device [n_head_kv x t] */
    float *   C_v;               /* device [n_head_kv x t x d_v] */
    uint8_t * K_out;             /* device [t x k_row_bytes]; NULL skips the requant */
    uint8_t * V_out;             /* device [t x v_row_bytes]; NULL skips the requant */
    kv_compact_stats stats;      /* quality fields filled when want_stats != 0 */
} kvc_layer_result;

/* t of every layer (0 where the filter skips it); returns 0 or an error code. */
int kvc_plan_layers(const kvc_model_desc * model, const kvc_layer_desc * layers,
                    const kv_compact_params * params, int * t_out);

/* Compact all filtered layers. results[l] must hold device buffers sized
 * from kvc_plan_layers(). Returns 0 or a negative error code. */
int kvc_compact_layers_dev(const kvc_model_desc * model, const kvc_layer_desc * layers,
                           const kv_compact_params * params, kvc_layer_result * results,
                           int want_stats);

/* Row codecs on device memory, bit-identical to kv_quantize_row /
 * kv_dequantize_row: rows x n values, src rows src_stride floats apart
 * (quantize) or src_row_bytes apart (dequantize). */
int kvc_quantize_rows_dev(const float * src, size_t src_stride, int type, int rows, int n,
                          uint8_t * dst, size_t dst_row_bytes);
int kvc_dequantize_rows_dev(const uint8_t * src, size_t src_row_bytes, int type, int rows, int n,
                            float * dst);

/* Kernels this process has launched through the library so far. */
uint64_t kvc_launch_count(void);

/* Per-stage device timing of the current device's library stream: copies the
 * accumulated milliseconds and launch counts of up to n stages (decode, score,
 * softmax+importance, select, refit target, beta, X build, LS Gram products,
 * refinement, metrics, requant, LS factor+solve, LS output product) into the
 * arrays (either may be NULL), resets
 * them, and turns event timing on (enable != 0) or off. Returns the number of
 * stages, or a negative error code. */
int kvc_profile(int enable, double * stage_ms, uint64_t * stage_launches, int n);

#ifdef __cplusplus
}
#endif
