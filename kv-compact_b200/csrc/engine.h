// engine.h — host-side planning and the device pipeline over (layer, chunk) units.
#pragma once

#include <functional>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kv-compact-api.h"
#include "kvc_internal.h"

#define KVC_N_STAGES 13
#define KVC_GROUP_STREAMS 4

// One chunk of one layer as the reference's kv_compact would process it.
struct kvc_plan_unit {
    int start;    // first token
    int C;        // tokens
    int t;        // kept keys
    int prefix;   // forced leading keys (<= t)
    int nq;       // reference queries used by this chunk
    int qmode;    // 0: top-level queries, 1: cheap queries from this chunk's keys
};

struct kvc_plan {
    int T = 0;
    int nq_top = 0;        // n_q_used of the top-level call
    bool top_cheap = false;// top-level queries are sampled from the full K
    int chunk = 0;         // effective chunk size (T when unchunked)
    int t_total = 0;
    std::vector<kvc_plan_unit> units;
};

// Mirrors src/kv-compact-api.cpp:369-437 and the per-chunk sub-call sizing
// (:466-498 + :382-409). Returns 0 or a negative reference error code.
int kvc_make_plan(int T, int n_q, bool q_null, int H, int dk, int dv, const kv_compact_params & p,
                  kvc_plan * out);

// Host-resident inputs and outputs of a drop-in call (single job). The
// engine cuts the layer's chunks into groups and overlaps, group by group,
// the upload of K/V rows (context copy stream), the compute, and the
// download of finished output rows (context d2h stream, queued by `emit`):
//   copy stream:    K_0 V_0 K_1 V_1 ...   (queued once the call's small
//                                          uploads are queued, so they go first)
//   group stream g: [wait K_g] decode K_g, scoring/selection of group g,
//                   [wait V_g] decode V_g, refit of group g, emit(g)
//   d2h stream:     results of group g while later groups compute
// Groups run on KVC_GROUP_STREAMS streams in turn, so the kernels of
// different groups (many of them one short wave each) share the SMs; group
// sizes may shrink geometrically so the work left after the last upload
// (the refit and download of the last group) is small. Each group then has
// scratch of its own; when the whole layer's scratch does not fit the
// device, groups run one after the other on the compute stream instead.
// A group's rows are the token rows its chunks cover; its output rows are
// the kept-key rows [r0, r1) of the layer's result arrays.
struct kvc_stream_io {
    // One input matrix: rows of `row_bytes` host bytes at `host`, staged at
    // `stage` (device, same row layout). type < 0: the rows are fp32 and
    // `stage` is the job's K / V itself; otherwise quantised rows decoded
    // into the job's K / V after the upload.
    struct input {
        const uint8_t * host = nullptr;
        uint8_t * stage = nullptr;
        size_t row_bytes = 0;
        int type = -1;
    } k, v;
    bool k_resident = false;   // K already uploaded and decoded in full (top-level cheap queries)
    bool k_blocks_only = false; // K is read only in its block format (kvc_k_blocks_only): not decoded
    int max_groups = 1;        // upper bound on the number of groups
    double size_ratio = 1.0;   // size of group g+1 / size of group g
    // Queue whatever consumes output rows [r0, r1) (requantisation, copies
    // to the host) on stream `st`, after the group's results.
    std::function<int(int r0, int r1, cudaStream_t st)> emit;
};

// Whether a layer's pipeline reads K only in its stored block format: the
// tensor-core scoring takes it (kvc_score_tc_ok) and nothing needs fp32 K
// rows (no cheap queries, which sample K rows; no diversity greedy, which
// compares K rows; the quality metrics come from the per-chunk records).
// K_out is then re-encoded from the stored rows (kvc_launch_transcode_gather).
bool kvc_k_blocks_only(const kv_compact_params & p, const struct kvc_plan & pl, int k_type, size_t k_row_bytes,
                       const void * k_base, int H, int dk);

// Device-side job for one layer: fp32 caches resident on the device.
struct kvc_layer_job {
    const float * K = nullptr;      // [T x H*dk]
    const uint8_t * Kq = nullptr;   // or K's rows in their block format [T x k_row_bytes] (device), if kept
    size_t k_row_bytes = 0;
    int k_type = -1;
    const float * V = nullptr;      // [T x H*dv] (holds the decoded rows once v_decoded)
    const uint8_t * Vq = nullptr;   // or V's rows in their block format [T x v_row_bytes] (device)
    size_t v_row_bytes = 0;
    int v_type = -1;
    bool v_decoded = true;          // false: V is only in Vq (or the io stage) so far
    const float * Q = nullptr;      // [nq_top x H*dk] top-level queries
    const float * rkv_w = nullptr;  // [T] device R-KV weights or null
    const kvc_plan * plan = nullptr;
    kvc_layer_out out{};            // device outputs (sel, beta, cv, t_total)
    kvc_stream_io * io = nullptr;   // host-resident inputs/outputs (single-job drop-in calls)
};

struct kvc_phase_ms {
    double scoring_ms = 0.0;
    double refit_ms = 0.0;
};

// Per-device state: stream, events and grow-only scratch arenas.
struct kvc_ctx {
    int device = -1;
    cudaStream_t stream = nullptr;
    cudaStream_t copy_stream = nullptr;         // host->device uploads overlapping compute
    cudaStream_t d2h_stream = nullptr;          // device->host results overlapping compute
    cudaStream_t group_stream[KVC_GROUP_STREAMS] = {};   // groups of a streamed call, round robin
    cudaEvent_t ev[4] = {};
    std::vector<cudaEvent_t> sync_ev;           // cross-stream ordering events (no timing), grow-only
    size_t sync_used = 0;
    std::mutex mu;
    void * arena[16] = {};          // slots: 0-2 engine scratch, 3-9 API / batched / seam, 10-13 state path
    size_t arena_cap[16] = {};
    kvc_unit * d_units = nullptr;
    size_t units_cap = 0;
    kvc_layer_out * d_outs = nullptr;
    size_t outs_cap = 0;
    uint64_t launches = 0;          // kernel launches issued (for the bench)
    // optional per-stage device timing (kvc_profile_*): events around each stage
    int profiling = 0;
    double stage_ms[KVC_N_STAGES] = {};
    uint64_t stage_launches[KVC_N_STAGES] = {};
    std::vector<cudaEvent_t> ev_pool;            // reused timing events
    std::vector<std::pair<int, int>> pending;    // (stage, first event index) awaiting resolution
    size_t ev_used = 0;
    // scoring/refit phase events of kvc_engine_run (three per batch), read by kvc_phase_collect
    std::vector<cudaEvent_t> ph_ev;
    size_t ph_used = 0;
    // pinned host staging for device->host results (grow-only)
    void * pinned = nullptr;
    size_t pinned_cap = 0;
    // KVC_TRACE=1: timeline of the streamed drop-in calls (kvc_trace / kvc_trace_dump)
    bool trace = false;
    std::vector<cudaEvent_t> trace_ev;
    std::vector<std::string> trace_label;
    size_t trace_used = 0;
};

// Wait until all work queued on ctx->stream has finished, polling its
// completion instead of sleeping in the driver: the calling thread resumes as
// soon as the device is done (no wake-up latency between dependent steps).
int kvc_wait(kvc_ctx * ctx);

// Next cross-stream ordering event of the context (reset with sync_used = 0
// at the start of a call, once no earlier event is still pending).
cudaEvent_t kvc_sync_event(kvc_ctx * ctx);

// With KVC_TRACE=1 in the environment: mark `label` on stream `st` (a timing
// event), and after the call's final wait print the marks of the call to
// stderr in milliseconds since its first mark. No-ops otherwise.
void kvc_trace(kvc_ctx * ctx, const std::string & label, cudaStream_t st);
void kvc_trace_dump(kvc_ctx * ctx);

// Grow the pinned staging buffer to at least `bytes`.
int kvc_pinned(kvc_ctx * ctx, size_t bytes, void ** out);

// Host memcpy of many (dst, src, bytes) pieces spread over worker threads
// (first-touch page faults of fresh malloc'd outputs dominate a single thread).
struct kvc_copy_piece { void * dst; const void * src; size_t bytes; };
void kvc_parallel_copy(const std::vector<kvc_copy_piece> & pieces);

// Result arrays of the drop-in API (hostpool.cu): page-locked blocks from a
// pool when available (else malloc); kvc_hfree returns them to the pool.
void * kvc_hmalloc(size_t bytes);
void kvc_hfree(void * p);
bool kvc_is_pinned(const void * p);
void kvc_hpool_release();

// Accumulate the elapsed times of the stages recorded since the last call
// (waits for the last recorded event).
void kvc_resolve_timers(kvc_ctx * ctx);

// Stage ids for per-stage timing.
enum {
    KVC_ST_DECODE = 0, KVC_ST_SCORE, KVC_ST_SOFTMAX, KVC_ST_SELECT, KVC_ST_PV, KVC_ST_BETA,
    KVC_ST_XBUILD, KVC_ST_LSQ, KVC_ST_REFINE, KVC_ST_METRICS, KVC_ST_REQUANT, KVC_ST_LSQ_FACTOR,
    KVC_ST_LSQ_OUT,
};

// Brackets one stage with events on `st` (default ctx->stream) when profiling is on.
struct kvc_stage_timer {
    kvc_ctx * ctx;
    int stage;
    cudaStream_t stream;
    int first = -1;
    kvc_stage_timer(kvc_ctx * c, int s, int n_launch, cudaStream_t st = nullptr);
    ~kvc_stage_timer();
};

// Context of the current CUDA device (created on first use). nullptr if no device.
kvc_ctx * kvc_get_ctx(int * rc);

// Grow arena slot `slot` to at least `bytes` (device memory).
int kvc_arena(kvc_ctx * ctx, int slot, size_t bytes, void ** out);

// Run the compaction pipeline over all units of `jobs` on ctx->stream.
// Outputs land in each job's `out` buffers. Stream-ordered, no host sync. With
// `phase`, the scoring and refit phases are bracketed by events; read them
// with kvc_phase_collect once the stream has drained.
// With `metric_partials`, layers whose chunks all scored the layer's own
// queries also get per-chunk quality-metric records (jobs[l].out.mpart, in
// arena slot 8, valid until the next run), which kvc_engine_metrics merges
// instead of re-reading the whole cache.
// With `shared`, every job is one unchunked unit over the same T positions
// and they all keep one selection: the top-t of the importance aggregated
// over every job and head (the llama.cpp state path, kvc-state.h). All jobs
// must fit one batch; diversity and OMP selection are not available there.
struct kvc_shared_sel {
    int t;                          // positions kept in every job
};
int kvc_engine_run(kvc_ctx * ctx, const kv_compact_params & p, int H, int dk, int dv,
                   kvc_layer_job * jobs, int n_jobs, kvc_phase_ms * phase, bool metric_partials,
                   const kvc_shared_sel * shared = nullptr);

// Scoring / refit milliseconds of the kvc_engine_run calls since the last
// collection (the stream must have drained).
void kvc_phase_collect(kvc_ctx * ctx, kvc_phase_ms * phase);

// Quality metrics of one layer: launch the kernels that leave the
// (cosine, MSE, agreement) triple of each of the kvc_metric_pairs() (head,
// query) pairs in d_res (stream-ordered), then average the triples on the
// host in reference order.
int kvc_engine_metrics_launch(kvc_ctx * ctx, const kvc_layer_job & job, int H, int dk, int dv, float * d_res);
void kvc_metrics_reduce(const float * h_res, int pairs, kv_compact_stats * st);
// Both, with a wait in between.
int kvc_engine_metrics(kvc_ctx * ctx, const kvc_layer_job & job, int H, int dk, int dv,
                       kv_compact_stats * st);

// Launchers (kernels in score.cu, select.cu, lsq.cu, nnls.cu, metrics.cu).
// rows_aligned: every K / Q row the units read starts on a 16-byte boundary
// (H*d_k and d_k multiples of 4, 16-byte aligned bases) — enables the
// asynchronous-copy variant.
// S = Q K^T / sqrt(d_k) of every (unit, head); mode 2 also writes the row
// maxima of each key tile (for the one-pass importance kernel).
int kvc_launch_score(const kvc_unit * d_units, int n_units, int max_nq, int max_cols,
                     const kvc_params_dev & P, float * fs, int mode, cudaStream_t st,
                     bool rows_aligned = false);
// Key tile of the scoring kernel kvc_launch_score picks (the granularity of
// its mode-2 row maxima).
int kvc_score_tile_keys(int max_nq, bool rows_aligned);
// Row statistics and per-key importance. tile_keys > 0: the scores were
// written in mode 2 with that key tile (one pass over S when the chunks are
// small enough); 0: the kernel finds the row maxima itself.
int kvc_launch_softmax_importance(const kvc_unit * d_units, int n_units, int max_nq, int max_C, int tile_keys,
                                  const kvc_params_dev & P, float * fs, cudaStream_t st);
// X block of the refit: the raw scores of the kept keys, S[:, sel].
int kvc_launch_gather_x(const kvc_unit * d_units, int n_units, int max_nq, const kvc_params_dev & P, float * fs,
                        const int * is, cudaStream_t st);
// X = softmax(S[:, sel]) in one pass (no beta).
int kvc_launch_gather_softmax_x(const kvc_unit * d_units, int n_units, int max_nq, int max_t, const kvc_params_dev & P,
                                float * fs, const int * is, cudaStream_t st);
// Y = A V per (unit, head). from_scores: the S region holds raw scores and A
// is formed from them and the row statistics (the engine); else it holds A.
int kvc_launch_pv(const kvc_unit * d_units, int n_units, int max_nq, const kvc_params_dev & P,
                  float * fs, bool from_scores, cudaStream_t st);
bool kvc_pv_tc_ok(int max_nq, int dv);
int kvc_launch_pv_tc(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs, bool from_scores,
                     cudaStream_t st);
int kvc_tc_take_error(cudaStream_t st);

// Scoring on the tcgen05 tensor cores from K's stored block bytes
// (score_tc.cu). kvc_score_tc_ok: whether the format, row layout, head
// dimension and query count take that path (KVC_EXACT_SCORES=1 keeps the
// bit-exact SIMT kernels); fills the geometry the launch needs.
struct kvc_score_tc_geom {
    int k_type = -1;      // 8 Q8_0, 2 Q4_0, 1 F16
    int seg = 0;          // bytes of one head in a K row
    int raww = 0;         // TMA box width in bytes
};
bool kvc_score_tc_ok(int k_type, size_t k_row_bytes, const void * k_base, int H, int dk, int max_nq,
                     kvc_score_tc_geom * g);
size_t kvc_score_tc_map_bytes();
// Encode the TMA map of one layer's K (or V) rows into `map` (kvc_score_tc_map_bytes()
// bytes, 64-byte aligned); `fused`: the box height of the fused kernel's tiles.
int kvc_score_tc_make_map(void * map, const uint8_t * k_base, size_t k_row_bytes, int rows, int raww, bool fused);
// S (and, mode 2, each row's maximum in pm slot 0) of every (unit, head);
// d_maps[layer] = the TMA map of the layer's K rows.
int kvc_launch_score_tc(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs,
                        const void * d_maps, const kvc_score_tc_geom & g, int mode, cudaStream_t st);
int kvc_score_tc_take_error(cudaStream_t st);
// Scoring fused with the refit target Y = softmax(S) V (d_k = d_v = 128, V
// in Q8_0 / Q4_0 rows read by TMA): whether it applies (fills V's geometry),
// and the launch (Y into each unit's y_off block; no separate refit-target
// pass). Opt-in with KVC_FUSED_PV=1: on cfg4 it measured slower (7.6 ms per
// step) than the separate scoring and refit-target kernels (3.0 + 3.4 ms).
bool kvc_score_pv_tc_ok(int dk, int dv, int max_nq, const kvc_score_tc_geom & kg, int v_type, size_t v_row_bytes,
                        const void * v_base, int H, kvc_score_tc_geom * vg);
int kvc_launch_score_pv_tc(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs,
                           const void * d_kmaps, const void * d_vmaps, const kvc_score_tc_geom & kg,
                           const kvc_score_tc_geom & vg, int mode, cudaStream_t st);
int kvc_launch_softmax_x(const kvc_unit * d_units, int n_units, int max_nq, const kvc_params_dev & P,
                         float * fs, const kvc_layer_out * d_outs, cudaStream_t st);
int kvc_launch_aggregate(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs,
                         cudaStream_t st);
int kvc_launch_select(const kvc_unit * d_units, int n_units, int max_C, const kvc_params_dev & P, float * fs,
                      int * is, const kvc_layer_out * d_outs, cudaStream_t st);
// One selection for every unit (each spanning positions 0..T-1): global
// importance over all units and heads into gimp (sensitivities of each
// (unit, head) into sens when P.use_sensitivity), top-t of it by the unit
// d_all (one unit over gimp, its selection at is + d_all->sel_off ==
// all_sel), then broadcast to every unit and its layer's output indices.
int kvc_launch_shared_select(const kvc_unit * d_units, int n_units, const kvc_unit * d_all, const kvc_params_dev & P,
                             float * fs, int * is, float * gimp, float * sens, const int * all_sel, int T, int t,
                             const kvc_layer_out * d_outs, cudaStream_t st);
size_t kvc_lsq_smem_bytes(int n);
// LS refit in three launches: Gram (and primal right-hand side) products,
// factorisation + solves, output product (dual form).
// `any_primal` / `any_dual`: whether some unit solves the primal (t <= n_q) /
// dual form; launches only one form needs are skipped otherwise.
// `aligned`: every unit's t and d_v are multiples of 4 (asynchronous-copy variant).
// Gram matrices of every unit; the primal right-hand side X^T Y of the units
// in d_primal[0 .. n_primal) (copies of the primal ones among d_units).
int kvc_launch_lsq_gram(const kvc_unit * d_units, int n_units, int max_n, int max_t, const kvc_params_dev & P,
                        const float * fs, double * gs, const kvc_layer_out * d_outs, const kvc_unit * d_primal,
                        int n_primal, bool aligned, cudaStream_t st);
int kvc_launch_lsq_factor(const kvc_unit * d_units, int n_units, int max_n, size_t smem_bytes,
                          const kvc_params_dev & P, const float * fs, double * gs,
                          const kvc_layer_out * d_outs, cudaStream_t st);
int kvc_launch_lsq_out(const kvc_unit * d_units, int n_units, int max_t, const kvc_params_dev & P,
                       const float * fs, double * gs, const kvc_layer_out * d_outs, bool any_dual, bool aligned,
                       cudaStream_t st);
int kvc_metric_pairs(int H, int nq);
size_t kvc_metric_scratch_floats(int H, int nq, int T, int t, int dv);
int kvc_launch_metrics(const float * K, const float * V, const float * Q, int T, int nq, int H, int dk, int dv,
                       const int * sel, const float * beta, const float * cv, int t, float isd,
                       float * scratch, float * res, cudaStream_t st);
size_t kvc_metric_partial_floats(int n_chunks, int H, int nq, int dv);
int kvc_launch_metric_partial(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, const float * fs,
                              const kvc_layer_out * d_outs, cudaStream_t st);
int kvc_launch_metric_merge(const float * mpart, int n_chunks, int H, int nq, int dv, float * res, cudaStream_t st);
// The merges of n layers (all with H heads, nq_top queries, d_v) in as few launches as possible.
int kvc_launch_metric_merge_batch(const float * const * mparts, const int * n_chunks, float * const * res, int n,
                                  int H, int nq, int dv, cudaStream_t st);
size_t kvc_omp_floats(int C, int t, int nq, int H);
int kvc_launch_omp_exp(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs, cudaStream_t st);
int kvc_launch_omp_select(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs, int * is,
                          const kvc_layer_out * d_outs, cudaStream_t st);
int kvc_launch_gather_rows(const float * src, int src_stride, const int * idx, int rows, int n,
                           float * dst, int dst_stride, cudaStream_t st);
int kvc_launch_cheap_q(const float * K, int T, int ek, int nq, float * Q, cudaStream_t st);
int kvc_launch_beta(const kvc_unit * d_units, int n_units, int max_nq, int max_t, const kvc_params_dev & P,
                    float * fs, int * is, double * gs, const kvc_layer_out * d_outs, cudaStream_t st);
size_t kvc_nnls_doubles_per_head(int t, int nq);
int kvc_launch_refine(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs,
                      int * is, const kvc_layer_out * d_outs, cudaStream_t st);
