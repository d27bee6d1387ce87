/*
 * kvc-state.h — compaction of a saved llama.cpp sequence state.
 *
 * The reference's state path is C++ in headers and in its CLI:
 *   parsed_kv_state::parse            include/kv-compact-state.h:104-222
 *   build_compacted_state             include/kv-compact-state.h:645-810
 *   compute_beta_direction            include/kv-compact-math.h:636-640
 *   cross-layer global key selection  src/kv-compact.cpp:456-590
 *   per-layer value refit             src/kv-compact.cpp:592-640
 * A llama.cpp state keeps one list of cells per stream, so every layer of the
 * compacted state must keep the same cells: the selection is global (one
 * top-t over all cells of the importance aggregated over every compacted
 * layer and head) and each layer then refits its values for that selection.
 * kvc_state_compact() runs all of it on the current CUDA device in one call:
 * the state's K/V rows are uploaded once and decoded on the device (the
 * transposed V layout is transposed there), the scoring, selection and refit
 * run over all compacted layers as one batch, and the compacted state is
 * written by device encoders into the reference's byte layout.
 *
 * State layout (llama_state_seq_get_data, one or more streams):
 *   [n_stream:u32] per stream:
 *     [cell_count:u32] per cell: [pos:i32][n_seq_id:u32]([x:i32][y:i32] when
 *       n_pos_per_embd > 1)[seq_id:i32 * n_seq_id]
 *     [v_trans:u32][n_layer:u32]
 *     per layer: [k_type:i32][k_size_row:u64][rows]
 *     per layer: non-transposed [v_type:i32][v_size_row:u64][rows]
 *                transposed     [v_type:i32][v_size_el:u32][n_embd_v:u32][n_embd_v x cells]
 *   [trailing bytes, e.g. a recurrent-state section, copied unchanged]
 *
 * Error codes: 0 OK; -1 null argument; -2 bad parameter; -4 a compacted
 * layer's K/V width is not n_head_kv * d; -20 malformed or truncated state;
 * -21 unsupported layout (more than one non-empty stream; quantised
 * transposed V); -13 shape beyond the engine's limits (d > 256; min(n_ref,
 * t) > 24576, or > 3072 with the beta fit; all compacted layers must fit one
 * device batch); -10..-12
 * no device / CUDA failure.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "kv-compact-api.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kvc_state_params {
    int                n_head_kv;       /* KV heads of the compacted layers */
    uint32_t           n_pos_per_embd;  /* 1; 4 for M-RoPE / IMROPE models (cells carry x, y) */
    float              target_ratio;    /* keep max(1, (int)(cells * ratio)) cells, 0 < ratio < 1 */
    int                n_ref_queries;   /* queries = K rows of the last n cells; 0: max(16, cells / 4) */
    int                score_method;    /* per-head importance: 0 max (the CLI's), 1 RMS, 2 mean */
    int                use_sensitivity; /* global importance sum_{layer,head} s * imp (else the max) */
    int                fold_beta;       /* fit beta by NNLS and fold it into K along the direction v
                                           with Q_ref v ~ 1 (else beta = 0 and K rows unchanged) */
    float              ridge;           /* ridge of the value refit and of the beta direction */
    kv_layer_filter_fn layer_filter;    /* attention layers; NULL: every layer whose K and V split
                                           into n_head_kv heads of the first such layer's widths */
    void *             layer_filter_data;
} kvc_state_params;

/* Defaults: ratio 0.2, n_ref_queries 0, score_method 0, no sensitivity, no
 * beta, ridge 1e-6, n_pos_per_embd 1, n_head_kv 0 (must be set). */
kvc_state_params kvc_state_params_default(void);

typedef struct kvc_state_info {
    uint32_t n_stream;
    uint32_t cell_count;      /* cells of stream 0 */
    uint32_t v_trans;
    uint32_t n_layer;
    int      n_compacted;     /* layers whose values were refitted (others keep their rows) */
    int      t;               /* cells kept */
    int      n_ref_queries;
    size_t   trailing_bytes;  /* bytes after the KV section */
} kvc_state_info;

/* Layout of a state without a device: stream, cell and layer counts.
 * Returns 0 or -20 / -21. */
int kvc_state_inspect(const uint8_t * state, size_t size, uint32_t n_pos_per_embd, kvc_state_info * info);

/* Compact stream 0 of `state`. On success *out_state (size *out_size) is the
 * compacted state, to be released with kvc_state_free; if out_selected is
 * not NULL it receives the kept cell indices (ascending, info->t of them,
 * also released with kvc_state_free). */
int kvc_state_compact(const uint8_t * state, size_t size, const kvc_state_params * params,
                      uint8_t ** out_state, size_t * out_size, int ** out_selected, kvc_state_info * info);

void kvc_state_free(void * p);

#ifdef __cplusplus
}
#endif
