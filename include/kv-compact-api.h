/*
 * kv-compact-api.h — drop-in C ABI of the B200 compaction library (libkvc.so).
 *
 * Every type and function here keeps the name, field order, field types and
 * calling convention of the reference's public header
 * (fabiantax/kv-compact include/kv-compact-api.h), so a program or a ctypes
 * binding written against the reference links against libkvc.so unchanged.
 * Each declaration cites the reference line it stands in for.
 *
 * What differs is underneath: inputs are staged to the GPU, the compaction
 * runs as sm_100a kernels, and results come back into malloc'd host arrays
 * with the same ownership rules as the reference (free them with the *_free
 * functions, which null the pointers and tolerate a second call).
 *
 * Return codes (reference src/kv-compact-api.cpp:369-392,990-997,1201):
 *    0  success
 *   -1  a required pointer is NULL
 *   -2  bad dimensions (T, n_head_kv, d_k, d_v <= 0; n_q <= 0 with explicit Q)
 *   -3  n_rounds < 1 (multi-round only)
 *   -4  quantised row size does not match n_head_kv * d
 * Codes added by this library (disjoint from the above):
 *  -10  no CUDA device / the library's kernels cannot run on it
 *  -11  device memory allocation failed
 *  -12  a CUDA launch or copy failed (the CUDA error is logged to stderr)
 *  -13  a shape outside what the kernels support (see kvc-batched.h limits)
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Layer filters (reference include/kv-compact-api.h:51-87) ----------
 * Caller-side helpers: the library never calls them, callers loop over
 * layers and ask kv_compact_should_compact_layer() which ones to compact. */
typedef int (*kv_layer_filter_fn)(int layer_idx, int n_layers, void * user_data);

/* Every layer is compacted. */
static inline int kv_layer_filter_all(int layer_idx, int n_layers, void * user_data) {
    (void)layer_idx; (void)n_layers; (void)user_data;
    return 1;
}

/* Layers (interval-1), (2*interval-1), ... are compacted; user_data carries
 * the interval as an integer. interval <= 0 compacts every layer. */
static inline int kv_layer_filter_periodic(int layer_idx, int n_layers, void * user_data) {
    int interval = (int)(intptr_t)user_data;
    (void)n_layers;
    if (interval <= 0) return 1;
    return ((layer_idx + 1) % interval) == 0;
}

/* Explicit, ascending list of layers to compact. */
typedef struct kv_layer_list {
    const int * layers;
    int         n_layers;
} kv_layer_list;

static inline int kv_layer_filter_explicit(int layer_idx, int n_layers, void * user_data) {
    const kv_layer_list * list = (const kv_layer_list *)user_data;
    (void)n_layers;
    if (!list || !list->layers) return 1;
    for (int i = 0; i < list->n_layers; i++) {
        if (list->layers[i] == layer_idx) return 1;
        if (list->layers[i] > layer_idx) break;
    }
    return 0;
}

/* ---- Reasoning-aware weighting (reference include/kv-compact-api.h:98-127) */
typedef enum {
    KV_TOKEN_ANSWER     = 0,
    KV_TOKEN_THINKING   = 1,
    KV_TOKEN_TRANSITION = 2
} kv_token_type;

/* Called once per cache position (position + token_offset) on the host. */
typedef int (*kv_token_classifier_fn)(int token_pos, void * user_data);

typedef struct kv_compact_reasoning {
    kv_token_classifier_fn classifier;      /* NULL disables the weighting     */
    void *                 classifier_data;
    float                  thinking_weight;   /* importance multiplier          */
    float                  transition_weight; /* importance multiplier          */
    int                    token_offset;      /* added to each position         */
} kv_compact_reasoning;

/* ---- Parameters (reference include/kv-compact-api.h:133-215) -----------
 * 22 fields; the layout is relied on by ctypes mirrors of the reference. */
typedef struct kv_compact_params {
    float  target_ratio;        /* kept fraction when target_count == 0       */
    int    target_count;        /* > 0: keep exactly this many (per call)     */
    int    use_sensitivity;     /* sensitivity-weighted head aggregation      */
    float  ridge;               /* ridge added to the LS normal equations     */
    int    nnls_max_iter;       /* Lawson-Hanson outer/inner iteration cap    */
    int    refine_rounds;       /* worst-key swap rounds                       */
    int    use_diversity;       /* greedy cosine-diversity selection          */
    float  diversity_strength;  /* penalty weight in [0,1]                     */
    int    n_shared_prefix;     /* leading positions always kept              */
    int    use_cheap_qref;      /* reference queries sampled from K           */
    int    skip_beta;           /* beta = 0, no NNLS                           */
    int    score_method;        /* 0 max, 1 rms, 2 mean over queries           */
    int    use_omp;             /* orthogonal-matching-pursuit selection      */
    int    omp_k_choice;        /* keys added per OMP iteration               */
    int    omp_refit_interval;  /* OMP NNLS refit period                      */
    int    nnls_method;         /* 0 Lawson-Hanson, 1 clamped LS (+PGD)       */
    int    nnls_pgd_iters;      /* projected-gradient steps after clamping    */
    int    chunk_size;          /* 0 auto, -1 never chunk, > 0 explicit       */
    int    n_threads;           /* host threads for staging (0 = all)         */
    kv_layer_filter_fn     layer_filter;
    void *                 layer_filter_data;
    kv_compact_reasoning * reasoning;
} kv_compact_params;

/* ---- Results (reference include/kv-compact-api.h:221-241) -------------- */
typedef struct kv_compact_stats {
    float  avg_cosine_sim;  /* compacted vs full attention output, <=4 heads x <=32 queries */
    float  avg_mse;
    float  avg_agreement;   /* fraction of queries whose output argmax agrees */
    double elapsed_ms;      /* whole call */
    double scoring_ms;      /* scoring + selection phase (device time) */
    double nnls_ms;         /* beta + value-refit phase (device time) */
} kv_compact_stats;

typedef struct kv_compact_result {
    int      t;                 /* kept positions                           */
    int      n_head_kv;
    int    * selected_indices;  /* [t], ascending original positions        */
    float ** beta;              /* [n_head_kv] -> [t]                        */
    float ** C_v;               /* [n_head_kv] -> [t * d_v] refitted values */
    kv_compact_stats stats;
} kv_compact_result;

/* reference include/kv-compact-api.h:248 */
kv_compact_params kv_compact_params_default(void);

/* One layer, all KV heads (reference include/kv-compact-api.h:264-270).
 * K_all/V_all: [T x n_head_kv*d] host fp32, Q_ref_all: [n_q x n_head_kv*d_k]
 * host fp32 (may be NULL with use_cheap_qref). */
int kv_compact(const float * K_all, const float * V_all, const float * Q_ref_all,
               int T, int n_q, int n_head_kv, int d_k, int d_v,
               const kv_compact_params * params, kv_compact_result * result);

/* Repeated compaction of the previous round's (K_sel, C_v)
 * (reference include/kv-compact-api.h:288-296). */
int kv_compact_multi_round(const float * K_all, const float * V_all, const float * Q_ref_all,
                           int T, int n_q, int n_head_kv, int d_k, int d_v,
                           const kv_compact_params * params, int n_rounds,
                           kv_compact_result * result, kv_compact_stats * per_round_stats);

/* reference include/kv-compact-api.h:299 */
void kv_compact_result_free(kv_compact_result * result);

/* ---- Quantised caches (reference include/kv-compact-api.h:306-358) ----- */
typedef enum {
    KV_TYPE_F32  = 0,
    KV_TYPE_F16  = 1,
    KV_TYPE_Q4_0 = 2,
    KV_TYPE_Q4_1 = 3,
    KV_TYPE_Q8_0 = 8
} kv_data_type;

#define KV_COMPACT_BLOCK_SIZE 32

typedef struct kv_compact_quant_result {
    kv_compact_result base;
    int               k_type;
    int               v_type;
    uint8_t *         K_out;       /* [t x k_row_bytes] selected K rows, requantised */
    uint8_t *         V_out;       /* [t x v_row_bytes] C_v rows, requantised        */
    size_t            k_row_bytes;
    size_t            v_row_bytes;
} kv_compact_quant_result;

/* dequant -> compact -> requant (reference include/kv-compact-api.h:347-355) */
int kv_compact_quantized(const uint8_t * K_quant, const uint8_t * V_quant,
                         const float * Q_ref_all, int k_type, int v_type,
                         size_t k_row_bytes, size_t v_row_bytes,
                         int T, int n_q, int n_head_kv, int d_k, int d_v,
                         const kv_compact_params * params,
                         kv_compact_quant_result * result);

/* reference include/kv-compact-api.h:358 */
void kv_compact_quant_result_free(kv_compact_quant_result * result);

/* Row codecs (reference include/kv-compact-api.h:366-378). Host-side, same
 * bytes as the device codecs. */
int    kv_dequantize_row(const uint8_t * src, int type, size_t row_bytes,
                         float * dst, int max_elements);
size_t kv_quantize_row(const float * src, int type, int n_elements, uint8_t * dst);
int    kv_quant_row_elements(int type, size_t row_bytes);
size_t kv_quant_row_bytes(int type, int n_elements);

/* Caller-side layer loop helpers (reference include/kv-compact-api.h:381-396). */
static inline int kv_compact_count_layers(kv_layer_filter_fn filter, void * filter_data,
                                          int n_layers) {
    if (!filter) return n_layers;
    int count = 0;
    for (int l = 0; l < n_layers; l++)
        if (filter(l, n_layers, filter_data)) count++;
    return count;
}

static inline int kv_compact_should_compact_layer(const kv_compact_params * params,
                                                  int layer_idx, int n_layers) {
    if (!params || !params->layer_filter) return 1;
    return params->layer_filter(layer_idx, n_layers, params->layer_filter_data);
}

#ifdef __cplusplus
}
#endif
