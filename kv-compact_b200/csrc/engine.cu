// engine.cu — planning, per-device context and the stage pipeline.
//
// Pipeline over a flat list of units (one per (layer, chunk), all heads):
//   scoring phase:  k_score -> k_softmax_importance -> k_aggregate -> k_select
//   refit phase:    k_pv (Y) -> k_gather_x (S[:,sel]) -> beta (NNLS, optional)
//                   -> k_softmax_x (X) -> k_dgemm + k_lsq_factor (C_v)
//                   -> refinement rounds (optional)
// Every stage is one launch over all units of the batch, so a whole model
// (all filtered layers) is a handful of launches that fill the 148 SMs.
#include "engine.h"

#include <math.h>
#include <limits.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <thread>

// ---------------------------------------------------------------------------
// planning (host)
// ---------------------------------------------------------------------------
static int cheap_nq(int T) {                 // src/kv-compact-api.cpp:384-387
    int n = T / 2;
    if (n > 64) n = 64;
    if (n < 4) n = 4;
    if (n > T) n = T;
    return n;
}

static int size_t_for(int T, const kv_compact_params & p) {   // :396-409
    int t;
    if (p.target_count > 0) {
        t = p.target_count < T ? p.target_count : T;
    } else {
        t = (int)((float)T * p.target_ratio);
        if (t < 1) t = 1;
        if (t > T) t = T;
    }
    if (p.n_shared_prefix > t) t = p.n_shared_prefix < T ? p.n_shared_prefix : T;
    return t;
}

static int clamp_prefix(int prefix, int t) {
    if (prefix <= 0) return 0;
    return prefix < t ? prefix : t;
}

bool kvc_k_blocks_only(const kv_compact_params & p, const kvc_plan & pl, int k_type, size_t k_row_bytes,
                       const void * k_base, int H, int dk) {
    if (p.use_diversity || pl.top_cheap || pl.units.empty()) return false;
    int max_nq = 1;
    for (const kvc_plan_unit & u : pl.units) {
        if (u.qmode != 0 || u.nq != pl.nq_top) return false;
        max_nq = std::max(max_nq, u.nq);
    }
    return kvc_score_tc_ok(k_type, k_row_bytes, k_base, H, dk, max_nq, nullptr);
}

int kvc_make_plan(int T, int n_q, bool q_null, int H, int dk, int dv, const kv_compact_params & p,
                  kvc_plan * out) {
    if (T <= 0 || H <= 0 || dk <= 0 || dv <= 0) return KVC_ERR_DIMS;
    kvc_plan pl;
    pl.T = T;
    if (p.use_cheap_qref || q_null) {
        pl.top_cheap = true;
        pl.nq_top = cheap_nq(T);
    } else {
        if (n_q <= 0) return KVC_ERR_DIMS;
        pl.nq_top = n_q;
    }
    const int t_top = size_t_for(T, p);

    int cs = p.chunk_size;                   // :417-437
    if (cs == 0) {
        float re = (p.target_count > 0) ? (float)p.target_count / (float)T : p.target_ratio;
        if (re <= 0.0f) re = 0.5f;
        if (re > 1.0f) re = 1.0f;
        int et = (int)((float)T * re);
        if (et > 256) {
            cs = (int)(256.0f / re);
            if (cs < 64) cs = 64;
            if (cs >= T) cs = T;
        } else {
            cs = T;
        }
    } else if (cs < 0) {
        cs = T;
    }
    pl.chunk = cs;

    if (cs >= T) {
        kvc_plan_unit u;
        u.start = 0;
        u.C = T;
        u.t = t_top;
        u.prefix = clamp_prefix(p.n_shared_prefix, t_top);
        u.nq = pl.nq_top;
        u.qmode = 0;
        pl.units.push_back(u);
        pl.t_total = t_top;
    } else {
        int nc = (T + cs - 1) / cs;
        pl.t_total = 0;
        for (int c = 0; c < nc; c++) {
            kvc_plan_unit u;
            u.start = c * cs;
            int end = u.start + cs;
            if (end > T) end = T;
            u.C = end - u.start;
            kv_compact_params cp = p;
            cp.chunk_size = -1;
            if (c > 0) cp.n_shared_prefix = 0;
            if (cp.n_shared_prefix > u.C) cp.n_shared_prefix = u.C;
            if (p.use_cheap_qref) {
                u.qmode = 1;
                u.nq = cheap_nq(u.C);
            } else {
                u.qmode = 0;
                u.nq = pl.nq_top;
            }
            u.t = size_t_for(u.C, cp);
            u.prefix = clamp_prefix(cp.n_shared_prefix, u.t);
            pl.units.push_back(u);
            pl.t_total += u.t;
        }
    }
    *out = std::move(pl);
    return KVC_OK;
}

// ---------------------------------------------------------------------------
// context and arenas
// ---------------------------------------------------------------------------
static std::mutex g_ctx_mu;
static kvc_ctx * g_ctx[64];

// Host-side failure injection for tests: KVC_FAULT_INJECT=alloc makes every
// scratch request fail as an exhausted device would (-11), =nodev makes the
// library see no usable device (-10). Read on every call, so a test can turn
// it on and off around single calls; nothing is injected on the GPU.
static bool fault_injected(const char * what) {
    const char * e = getenv("KVC_FAULT_INJECT");
    return e && strcmp(e, what) == 0;
}

kvc_ctx * kvc_get_ctx(int * rc) {
    int dev = -1, n = 0;
    if (fault_injected("nodev")) {
        if (rc) *rc = KVC_ERR_NODEV;
        return nullptr;
    }
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        if (rc) *rc = KVC_ERR_NODEV;
        return nullptr;
    }
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        if (rc) *rc = KVC_ERR_NODEV;
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    if (!g_ctx[dev]) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess || prop.major < 10) {
            fprintf(stderr, "[kvc] device %d (sm_%d%d) cannot run sm_100a kernels\n", dev, prop.major, prop.minor);
            if (rc) *rc = KVC_ERR_NODEV;
            return nullptr;
        }
        kvc_ctx * c = new kvc_ctx();
        c->device = dev;
        // A blocking stream: its work is ordered after everything the caller
        // queued on the legacy default stream (e.g. PyTorch producing the
        // device caches the batched API reads) and vice versa.
        if (cudaStreamCreate(&c->stream) != cudaSuccess) {
            delete c;
            if (rc) *rc = KVC_ERR_CUDA;
            return nullptr;
        }
        for (auto & e : c->ev) cudaEventCreate(&e);
        if (cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&c->d2h_stream, cudaStreamNonBlocking) != cudaSuccess) {
            delete c;
            if (rc) *rc = KVC_ERR_CUDA;
            return nullptr;
        }
        bool ok = true;
        for (auto & gs : c->group_stream) ok = ok && cudaStreamCreateWithFlags(&gs, cudaStreamNonBlocking) == cudaSuccess;
        if (!ok) {
            delete c;
            if (rc) *rc = KVC_ERR_CUDA;
            return nullptr;
        }
        const char * tr = getenv("KVC_TRACE");
        c->trace = tr && atoi(tr) > 0;
        g_ctx[dev] = c;
    }
    if (rc) *rc = KVC_OK;
    return g_ctx[dev];
}

int kvc_arena(kvc_ctx * ctx, int slot, size_t bytes, void ** out) {
    if (fault_injected("alloc")) {
        fprintf(stderr, "[kvc] injected allocation failure (KVC_FAULT_INJECT=alloc)\n");
        return KVC_ERR_OOM;
    }
    if (bytes == 0) bytes = 256;
    if (ctx->arena_cap[slot] < bytes) {
        if (ctx->arena[slot]) {
            KVC_CUDA(cudaStreamSynchronize(ctx->stream));
            cudaFree(ctx->arena[slot]);
            ctx->arena[slot] = nullptr;
            ctx->arena_cap[slot] = 0;
        }
        size_t cap = bytes + bytes / 8;
        KVC_CUDA(cudaMalloc(&ctx->arena[slot], cap));
        ctx->arena_cap[slot] = cap;
    }
    *out = ctx->arena[slot];
    return KVC_OK;
}

int kvc_wait(kvc_ctx * ctx) {
    KVC_CUDA(cudaEventRecord(ctx->ev[0], ctx->stream));
    cudaError_t e;
    while ((e = cudaEventQuery(ctx->ev[0])) == cudaErrorNotReady) {
    }
    KVC_CUDA(e);
    int te = kvc_tc_take_error(ctx->stream);
    if (!te) te = kvc_score_tc_take_error(ctx->stream);
    if (te) {
        fprintf(stderr, "[kvc] tensor-core kernel reported error %d (bounded wait ran out)\n", te);
        return KVC_ERR_CUDA;
    }
    return KVC_OK;
}

void kvc_trace(kvc_ctx * ctx, const std::string & label, cudaStream_t st) {
    if (!ctx->trace) return;
    if (ctx->trace_used == ctx->trace_ev.size()) {
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        ctx->trace_ev.push_back(e);
        ctx->trace_label.emplace_back();
    }
    ctx->trace_label[ctx->trace_used] = label;
    cudaEventRecord(ctx->trace_ev[ctx->trace_used++], st);
}

void kvc_trace_dump(kvc_ctx * ctx) {
    if (!ctx->trace || ctx->trace_used == 0) return;
    std::string line = "[kvc trace]";
    for (size_t i = 0; i < ctx->trace_used; i++) {
        float ms = 0.0f;
        cudaEventSynchronize(ctx->trace_ev[i]);
        cudaEventElapsedTime(&ms, ctx->trace_ev[0], ctx->trace_ev[i]);
        char buf[96];
        snprintf(buf, sizeof buf, " %s=%.3f", ctx->trace_label[i].c_str(), ms);
        line += buf;
    }
    fprintf(stderr, "%s\n", line.c_str());
    ctx->trace_used = 0;
}

cudaEvent_t kvc_sync_event(kvc_ctx * ctx) {
    if (ctx->sync_used == ctx->sync_ev.size()) {
        cudaEvent_t e = nullptr;
        cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
        ctx->sync_ev.push_back(e);
    }
    return ctx->sync_ev[ctx->sync_used++];
}

int kvc_pinned(kvc_ctx * ctx, size_t bytes, void ** out) {
    if (bytes == 0) bytes = 256;
    if (ctx->pinned_cap < bytes) {
        if (ctx->pinned) {
            KVC_CUDA(cudaStreamSynchronize(ctx->stream));
            cudaFreeHost(ctx->pinned);
            ctx->pinned = nullptr;
            ctx->pinned_cap = 0;
        }
        size_t cap = bytes + bytes / 8;
        KVC_CUDA(cudaHostAlloc(&ctx->pinned, cap, cudaHostAllocDefault));
        ctx->pinned_cap = cap;
    }
    *out = ctx->pinned;
    return KVC_OK;
}

void kvc_parallel_copy(const std::vector<kvc_copy_piece> & pieces) {
    size_t total = 0;
    for (const auto & pc : pieces) total += pc.bytes;
    unsigned hw = std::thread::hardware_concurrency();
    int nt = (int)std::min<size_t>(std::max(1u, std::min(hw, 16u)), total / (4u << 20) + 1);
    if (nt <= 1) {
        for (const auto & pc : pieces) memcpy(pc.dst, pc.src, pc.bytes);
        return;
    }
    // split the concatenated byte range evenly; thread i copies [i*per, (i+1)*per)
    const size_t per = (total + nt - 1) / nt;
    auto work = [&](int i) {
        size_t lo = (size_t)i * per, hi = std::min(total, lo + per), pos = 0;
        for (const auto & pc : pieces) {
            size_t a = std::max(lo, pos), b = std::min(hi, pos + pc.bytes);
            if (a < b) memcpy((char *)pc.dst + (a - pos), (const char *)pc.src + (a - pos), b - a);
            pos += pc.bytes;
            if (pos >= hi) break;
        }
    };
    std::vector<std::thread> th;
    for (int i = 1; i < nt; i++) th.emplace_back(work, i);
    work(0);
    for (auto & x : th) x.join();
}

static cudaEvent_t phase_event(kvc_ctx * ctx) {
    if (ctx->ph_used == ctx->ph_ev.size()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        ctx->ph_ev.push_back(e);
    }
    return ctx->ph_ev[ctx->ph_used++];
}

void kvc_phase_collect(kvc_ctx * ctx, kvc_phase_ms * phase) {
    double a = 0.0, b = 0.0;
    for (size_t i = 0; i + 2 < ctx->ph_used; i += 3) {
        float x = 0.0f, y = 0.0f;
        cudaEventElapsedTime(&x, ctx->ph_ev[i], ctx->ph_ev[i + 1]);
        cudaEventElapsedTime(&y, ctx->ph_ev[i + 1], ctx->ph_ev[i + 2]);
        a += x;
        b += y;
    }
    ctx->ph_used = 0;
    if (phase) {
        phase->scoring_ms = a;
        phase->refit_ms = b;
    }
}

static cudaEvent_t next_event(kvc_ctx * ctx, int * idx) {
    if (ctx->ev_used == ctx->ev_pool.size()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        ctx->ev_pool.push_back(e);
    }
    *idx = (int)ctx->ev_used;
    return ctx->ev_pool[ctx->ev_used++];
}

kvc_stage_timer::kvc_stage_timer(kvc_ctx * c, int s, int n_launch, cudaStream_t st)
    : ctx(c), stage(s), stream(st ? st : c->stream) {
    ctx->launches += (uint64_t)n_launch;
    ctx->stage_launches[s] += (uint64_t)n_launch;
    if (!ctx->profiling) return;
    cudaEventRecord(next_event(ctx, &first), stream);
}

kvc_stage_timer::~kvc_stage_timer() {
    if (first < 0) return;
    int second;
    cudaEventRecord(next_event(ctx, &second), stream);
    ctx->pending.push_back({stage, first});
}

void kvc_resolve_timers(kvc_ctx * ctx) {
    if (ctx->pending.empty()) { ctx->ev_used = 0; return; }
    cudaEventSynchronize(ctx->ev_pool[ctx->ev_used - 1]);
    for (auto & pr : ctx->pending) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ctx->ev_pool[pr.second], ctx->ev_pool[pr.second + 1]);
        ctx->stage_ms[pr.first] += ms;
    }
    ctx->pending.clear();
    ctx->ev_used = 0;
}

// ---------------------------------------------------------------------------
// small utility kernels
// ---------------------------------------------------------------------------
__global__ void k_gather_rows(const float * __restrict__ src, int ss, const int * __restrict__ idx, int rows,
                              int n, float * __restrict__ dst, int ds) {
    long long total = (long long)rows * n;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        long long r = i / n;
        int c = (int)(i - r * n);
        dst[r * ds + c] = src[(long long)idx[r] * ss + c];
    }
}

int kvc_launch_gather_rows(const float * src, int ss, const int * idx, int rows, int n, float * dst, int ds,
                           cudaStream_t st) {
    if (rows <= 0 || n <= 0) return KVC_OK;
    long long work = (long long)rows * n;
    int g = (int)std::min<long long>((work + 255) / 256, 148LL * 32);
    k_gather_rows<<<g, 256, 0, st>>>(src, ss, idx, rows, n, dst, ds);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

// Cheap reference queries: rows of K at floor(((i+1)/(n+1))^2 (T-1))
// (src/kv-compact-api.cpp:132-152).
__global__ void k_cheap_q(const float * __restrict__ K, int T, int ek, int nq, float * __restrict__ Q) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)nq * ek;
         i += (long long)gridDim.x * blockDim.x) {
        int qi = (int)(i / ek), c = (int)(i % ek);
        float fr = __fdiv_rn((float)(qi + 1), (float)(nq + 1));
        fr = __fmul_rn(fr, fr);
        int pos = (int)__fmul_rn(fr, (float)(T - 1));
        if (pos >= T) pos = T - 1;
        if (pos < 0) pos = 0;
        Q[i] = K[(long long)pos * ek + c];
    }
}

int kvc_launch_cheap_q(const float * K, int T, int ek, int nq, float * Q, cudaStream_t st) {
    long long work = (long long)nq * ek;
    int g = (int)std::min<long long>((work + 255) / 256, 148LL * 8);
    k_cheap_q<<<g, 256, 0, st>>>(K, T, ek, nq, Q);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

// ---------------------------------------------------------------------------
// pipeline
// ---------------------------------------------------------------------------
static inline long long al32(long long x) { return (x + 31) & ~31LL; }

struct unit_sizes {
    long long fs, is, gs;
};

static unit_sizes sizes_of(const kvc_plan_unit & u, int H, int dv, bool omp) {
    unit_sizes s;
    const int n = std::min(u.nq, u.t);
    s.fs = al32((long long)H * u.nq * u.C) + al32((long long)H * u.nq * ((u.C + 127) / 128)) +
           al32((long long)(2 * H + 1) * u.C) + al32((long long)2 * H * u.nq) +
           al32((long long)H * u.nq * dv) + al32((long long)H * u.nq * u.t) + al32((long long)2 * H * u.nq);
    if (omp) s.fs += al32((long long)kvc_omp_floats(u.C, u.t, u.nq, H));
    s.is = al32(u.t) + al32(4LL * u.C);
    s.gs = al32((long long)H * n * n) + al32((long long)H * n * dv);
    return s;
}

int kvc_engine_run(kvc_ctx * ctx, const kv_compact_params & p, int H, int dk, int dv,
                   kvc_layer_job * jobs, int n_jobs, kvc_phase_ms * phase, bool metric_partials,
                   const kvc_shared_sel * shared) {
    if (n_jobs <= 0) return KVC_OK;
    cudaStream_t st = ctx->stream;
    const int T_sh = shared ? jobs[0].plan->T : 0;
    if (shared) {                                // one unchunked unit per job, all over the same positions
        if (p.use_diversity || p.use_omp) return KVC_ERR_SHAPE;
        for (int l = 0; l < n_jobs; l++) {
            const kvc_plan & pl = *jobs[l].plan;
            if (jobs[l].io || pl.units.size() != 1 || pl.T != T_sh || pl.units[0].C != T_sh ||
                pl.units[0].t != shared->t || pl.units[0].start != 0)
                return KVC_ERR_SHAPE;
        }
    }
    if (p.use_sensitivity && H > 64) return KVC_ERR_SHAPE;
    if (dk > KVC_MAX_D || dv > KVC_MAX_D) return KVC_ERR_SHAPE;

    kvc_params_dev P;
    P.H = H; P.dk = dk; P.dv = dv;
    P.score_method = p.score_method;
    P.skip_beta = p.skip_beta;
    P.use_sensitivity = p.use_sensitivity;
    P.use_diversity = p.use_diversity;
    P.diversity_strength = p.diversity_strength;
    P.nnls_method = p.nnls_method;
    P.nnls_max_iter = p.nnls_max_iter;
    P.nnls_pgd_iters = p.nnls_pgd_iters;
    P.ridge = p.ridge;
    P.isd = 1.0f / sqrtf((float)dk);
    P.use_omp = p.use_omp ? 1 : 0;
    P.omp_k_choice = p.omp_k_choice;
    P.omp_refit_interval = p.omp_refit_interval;

    // ---- layer outputs table
    const size_t n_outs = (size_t)n_jobs + (shared ? 1 : 0);     // + the shared selection's own entry
    if (ctx->outs_cap < n_outs) {
        if (ctx->d_outs) { KVC_CUDA(cudaStreamSynchronize(st)); cudaFree(ctx->d_outs); }
        ctx->outs_cap = n_outs * 2;
        KVC_CUDA(cudaMalloc(&ctx->d_outs, ctx->outs_cap * sizeof(kvc_layer_out)));
    }
    std::vector<kvc_layer_out> outs(n_jobs);
    for (int l = 0; l < n_jobs; l++) {
        jobs[l].out.n_chunks = (int)jobs[l].plan->units.size();
        jobs[l].out.mpart = nullptr;
    }
    // per-chunk metric records for layers whose chunks all used the layer's queries
    if (metric_partials) {
        size_t mp_total = 0;
        std::vector<size_t> mp_off(n_jobs, (size_t)-1);
        for (int l = 0; l < n_jobs; l++) {
            const kvc_plan & pl = *jobs[l].plan;
            bool own_q = !pl.units.empty();
            for (const kvc_plan_unit & pu : pl.units) own_q = own_q && pu.qmode == 0 && pu.nq == pl.nq_top;
            if (!own_q) continue;
            mp_off[l] = mp_total;
            mp_total += (kvc_metric_partial_floats((int)pl.units.size(), H, pl.nq_top, dv) + 63) & ~(size_t)63;
        }
        if (mp_total) {
            void * a8;
            int rc8;
            if ((rc8 = kvc_arena(ctx, 8, mp_total * 4, &a8))) return rc8;
            for (int l = 0; l < n_jobs; l++)
                if (mp_off[l] != (size_t)-1) jobs[l].out.mpart = (float *)a8 + mp_off[l];
        }
    }
    for (int l = 0; l < n_jobs; l++) outs[l] = jobs[l].out;
    KVC_CUDA(cudaMemcpyAsync(ctx->d_outs, outs.data(), n_jobs * sizeof(kvc_layer_out), cudaMemcpyHostToDevice, st));
    for (int l = 0; l < n_jobs; l++)
        if (outs[l].t_total > 0)
            KVC_CUDA(cudaMemsetAsync(outs[l].beta, 0, (size_t)H * outs[l].t_total * sizeof(float), st));

    // ---- flat unit list, split into batches that fit the scratch budget
    struct ref { int l, i; };
    std::vector<ref> all;
    for (int l = 0; l < n_jobs; l++)
        for (int i = 0; i < (int)jobs[l].plan->units.size(); i++) all.push_back({l, i});

    kvc_stream_io * io = nullptr;
    for (int l = 0; l < n_jobs; l++)
        if (jobs[l].io) {
            if (n_jobs > 1) return KVC_ERR_SHAPE;   // host-resident inputs: single-job calls only
            io = jobs[l].io;
            jobs[l].v_decoded = io->v.type < 0;     // fp32 rows land in V as they are
        }
    // V stays in its block format when every job has it in one format and
    // the tensor-core refit-target kernel takes every unit: that kernel
    // decodes the values it reads, and no fp32 copy of V is written (the
    // direct quality metrics decode V on their own when they run).
    // KVC_DECODE_V=1 decodes V first instead.
    {
        int max_nq_all = 1, ty = -1;
        size_t rb = 0;
        bool ok = !shared && getenv("KVC_DECODE_V") == nullptr;
        for (int l = 0; l < n_jobs && ok; l++) {
            for (const kvc_plan_unit & pu : jobs[l].plan->units) max_nq_all = std::max(max_nq_all, pu.nq);
            const bool streamed = jobs[l].io != nullptr;
            const int t_l = streamed ? jobs[l].io->v.type : jobs[l].v_type;
            const size_t rb_l = streamed ? jobs[l].io->v.row_bytes : jobs[l].v_row_bytes;
            const bool src = streamed ? jobs[l].io->v.stage != nullptr : jobs[l].Vq != nullptr;
            ok = src && (t_l == 8 || t_l == 2 || t_l == 3) && (l == 0 || (t_l == ty && rb_l == rb));
            ty = t_l;
            rb = rb_l;
        }
        ok = ok && kvc_pv_tc_ok(max_nq_all, dv);
        P.v_type = ok ? ty : -1;
        P.v_rb = ok ? (long long)rb : 0;
    }
    const bool v_blocks = P.v_type >= 0;
    // Scores on the tensor cores, read from K's stored block bytes
    // (score_tc.cu), when every job has them on the device in one supported
    // format; else the bit-exact SIMT kernels over the fp32 K.
    kvc_score_tc_geom tcg;
    bool tc_score = !shared;
    {
        int max_nq_all = 1;
        for (int l = 0; l < n_jobs; l++)
            for (const kvc_plan_unit & pu : jobs[l].plan->units) max_nq_all = std::max(max_nq_all, pu.nq);
        for (int l = 0; l < n_jobs && tc_score; l++) {
            const bool streamed = jobs[l].io != nullptr;
            const uint8_t * kb = streamed ? jobs[l].io->k.stage : jobs[l].Kq;
            const int kt = streamed ? jobs[l].io->k.type : jobs[l].k_type;
            const size_t krb = streamed ? jobs[l].io->k.row_bytes : jobs[l].k_row_bytes;
            kvc_score_tc_geom g;
            tc_score = kb != nullptr && kvc_score_tc_ok(kt, krb, kb, H, dk, max_nq_all, &g) &&
                       (l == 0 || (g.k_type == tcg.k_type && g.seg == tcg.seg && g.raww == tcg.raww));
            if (l == 0) tcg = g;
        }
    }
    for (int l = 0; l < n_jobs; l++)             // undecoded K needs the tensor-core scoring
        if (jobs[l].io && jobs[l].io->k_blocks_only && !tc_score) return KVC_ERR_SHAPE;
    // The refit target Y = softmax(S) V in the scoring pass itself when V's
    // rows are in one block format the fused kernel reads (score_tc.cu)
    kvc_score_tc_geom vg;
    bool fused_pv = tc_score && v_blocks && !P.use_omp;
    {
        int max_nq_all = 1;
        for (int l = 0; l < n_jobs; l++)
            for (const kvc_plan_unit & pu : jobs[l].plan->units) max_nq_all = std::max(max_nq_all, pu.nq);
        for (int l = 0; l < n_jobs && fused_pv; l++) {
            const bool streamed = jobs[l].io != nullptr;
            const uint8_t * vb = streamed ? jobs[l].io->v.stage : jobs[l].Vq;
            kvc_score_tc_geom g;
            fused_pv = vb != nullptr &&
                       kvc_score_pv_tc_ok(dk, dv, max_nq_all, tcg, (int)P.v_type, (size_t)P.v_rb, vb, H, &g) &&
                       (l == 0 || (g.seg == vg.seg && g.raww == vg.raww));
            if (l == 0) vg = g;
        }
    }
    void * d_maps = nullptr;
    if (tc_score) {                               // one TMA map per job (layer): its K rows as bytes x rows
        const size_t mb = kvc_score_tc_map_bytes();
        std::vector<uint64_t> maps((size_t)n_jobs * mb / 8);
        for (int l = 0; l < n_jobs; l++) {
            const bool streamed = jobs[l].io != nullptr;
            const uint8_t * kb = streamed ? jobs[l].io->k.stage : jobs[l].Kq;
            const size_t krb = streamed ? jobs[l].io->k.row_bytes : jobs[l].k_row_bytes;
            int rcm;
            if ((rcm = kvc_score_tc_make_map(maps.data() + (size_t)l * mb / 8, kb, krb, jobs[l].plan->T, tcg.raww,
                                             fused_pv)))
                return rcm;
        }
        if (fused_pv) {                           // then one per job for V's rows
            maps.resize((size_t)2 * n_jobs * mb / 8);
            for (int l = 0; l < n_jobs; l++) {
                const bool streamed = jobs[l].io != nullptr;
                const uint8_t * vb = streamed ? jobs[l].io->v.stage : jobs[l].Vq;
                int rcm;
                if ((rcm = kvc_score_tc_make_map(maps.data() + (size_t)(n_jobs + l) * mb / 8, vb, (size_t)P.v_rb,
                                                 jobs[l].plan->T, vg.raww, true)))
                    return rcm;
            }
        }
        const size_t nmaps = fused_pv ? 2 * (size_t)n_jobs : (size_t)n_jobs;
        int rcm;
        if ((rcm = kvc_arena(ctx, 14, nmaps * mb, &d_maps))) return rcm;
        KVC_CUDA(cudaMemcpyAsync(d_maps, maps.data(), nmaps * mb, cudaMemcpyHostToDevice, st));
    }
    const void * d_vmaps = fused_pv ? (const void *)((const uint8_t *)d_maps + (size_t)n_jobs * kvc_score_tc_map_bytes())
                                    : nullptr;
    if (io && !v_blocks) jobs[0].v_decoded = true;  // arrive() decodes every group's rows
    for (int l = 0; l < n_jobs && !v_blocks; l++) {
        kvc_layer_job & J = jobs[l];
        if (J.io || J.v_decoded) continue;
        if (!J.Vq || !J.V) return KVC_ERR_NULL;
        kvc_stage_timer tm(ctx, KVC_ST_DECODE, 1);
        int rcd;
        if ((rcd = kvc_launch_decode(J.Vq, J.v_row_bytes, J.v_type, const_cast<float *>(J.V), J.plan->T, H * dv, st)))
            return rcd;
        J.v_decoded = true;
    }
    // a streamed job is cut into at most io->max_groups groups of consecutive
    // units whose sizes shrink by io->size_ratio from one to the next (each
    // at least one unit); group_end[g] is one past the last unit of group g
    std::vector<size_t> group_end;
    if (io && io->max_groups > 1 && all.size() > 1) {
        const int g_n = (int)std::min<size_t>((size_t)io->max_groups, all.size());
        const double q = io->size_ratio > 0.0 ? io->size_ratio : 1.0;
        double wsum = 0.0, w = 1.0;
        for (int g = 0; g < g_n; g++, w *= q) wsum += w;
        size_t end = 0;
        w = 1.0;
        double acc = 0.0;
        for (int g = 0; g < g_n; g++, w *= q) {
            acc += w;
            size_t e = (g == g_n - 1) ? all.size() : (size_t)llround(acc / wsum * (double)all.size());
            e = std::max(e, end + 1);
            e = std::min(e, all.size() - (size_t)(g_n - 1 - g));     // leave one unit per later group
            group_end.push_back(e);
            end = e;
        }
    } else {
        group_end.push_back(all.size());
    }

    // Scratch of all units at once, counted as the batch loop below places it.
    // When the arenas already hold that much (every call after the first on
    // the same shapes) the whole job is one batch (or, streamed, groups with
    // scratch of their own) and the device is not queried: cudaMemGetInfo can
    // take tens of milliseconds on a busy host.
    long long fs_all = 0, is_all = 0, gs_all = 0;
    for (int l = 0; l < n_jobs; l++)
        if (jobs[l].rkv_w) fs_all += al32(jobs[l].plan->T);
    for (const ref & rf : all) {
        const kvc_plan_unit & pu = jobs[rf.l].plan->units[rf.i];
        const unit_sizes us = sizes_of(pu, H, dv, p.use_omp != 0);
        fs_all += us.fs;
        is_all += us.is;
        const int n = std::min(pu.nq, pu.t);
        long long gper = (long long)n * n;
        if (!p.skip_beta) gper = std::max<long long>(gper, (long long)kvc_nnls_doubles_per_head(pu.t, pu.nq));
        gs_all += al32((long long)H * gper) + al32((long long)H * n * dv);
    }
    long long env_cap = 0;
    // KVC_SCRATCH_BUDGET_MB caps the scratch of one batch (testing the
    // multi-batch path, or leaving room for other users of the device)
    if (const char * env = getenv("KVC_SCRATCH_BUDGET_MB")) env_cap = atoll(env) << 20;
    long long budget;
    if (env_cap <= 0 && (size_t)fs_all * 4 <= ctx->arena_cap[0] && (size_t)is_all * 4 <= ctx->arena_cap[1] &&
        (size_t)gs_all * 8 <= ctx->arena_cap[2]) {
        budget = LLONG_MAX;
    } else {
        size_t free_b = 0, total_b = 0;
        cudaMemGetInfo(&free_b, &total_b);
        budget = (long long)std::min<size_t>((size_t)(free_b * 0.6), (size_t)48 << 30);
        // bytes already held by our arenas can be reused
        budget += (long long)(ctx->arena_cap[0] + ctx->arena_cap[1] + ctx->arena_cap[2]);
        if (env_cap > 0) budget = std::min(budget, env_cap);
    }

    if (phase) ctx->ph_used = 0;
    ctx->sync_used = 0;
    bool rows_aligned = (dk % 4) == 0 && ((H * dk) % 4) == 0;
    for (int l = 0; l < n_jobs; l++)
        rows_aligned = rows_aligned && (((uintptr_t)jobs[l].K) & 15) == 0 && (((uintptr_t)jobs[l].Q) & 15) == 0;

    // Groups of a streamed job run concurrently (scoring of one beside the
    // refit of the previous) when the whole job's scratch fits: each group
    // then keeps scratch of its own.
    const bool concurrent = io && (fs_all * 4 + is_all * 4 + gs_all * 8) <= budget;

    // ---- batches of consecutive units, each within the scratch budget; a
    // streamed job is also cut into at most io->max_groups groups. All
    // batches are laid out before anything is queued, so the arenas grow
    // once and every unit table goes up in one copy ahead of the bulk rows.
    struct batch {
        std::vector<kvc_unit> U;
        size_t u0 = 0;                           // first entry in the device unit table
        long long fs = 0, is = 0, gs = 0;        // scratch end offsets
        std::vector<long long> w_base;           // R-KV weights at the front of the float arena
        int max_nq = 1, max_C = 1, max_t = 1, max_n = 1;
        bool any_primal = false, any_dual = false, lsq_aligned = true;
        size_t lsq_smem = 0;
        size_t p0 = 0;                           // its primal units' copies in the device unit table
        int n_primal = 0;
        int row0 = 0, row1 = 0;                  // token rows (streamed job)
        int out0 = 0, out1 = 0;                  // kept-key rows (streamed job)
    };
    std::vector<batch> B;
    long long max_fs = 0, max_is = 0, max_gs = 0;
    size_t pos = 0;
    while (pos < all.size()) {
        batch bt;
        bt.lsq_aligned = (dv % 4) == 0;
        if (concurrent && !B.empty()) {          // continue after the previous group's scratch
            bt.fs = B.back().fs;
            bt.is = B.back().is;
            bt.gs = B.back().gs;
            bt.w_base = B[0].w_base;
        } else {
            bt.w_base.assign(n_jobs, -1);
            for (int l = 0; l < n_jobs; l++)
                if (jobs[l].rkv_w) { bt.w_base[l] = bt.fs; bt.fs += al32(jobs[l].plan->T); }
        }
        const size_t first = pos;
        size_t gi = 0;
        while (group_end[gi] <= first) gi++;
        while (pos < group_end[gi]) {
            const kvc_plan_unit & pu = jobs[all[pos].l].plan->units[all[pos].i];
            unit_sizes s = sizes_of(pu, H, dv, p.use_omp != 0);
            long long bytes = (bt.fs + s.fs) * 4 + (bt.is + s.is) * 4 + (bt.gs + s.gs) * 8;
            if (pos > first && bytes > budget) break;
            const kvc_layer_job & J = jobs[all[pos].l];
            const int ek = H * dk, ev = H * dv;
            kvc_unit u;
            memset(&u, 0, sizeof(u));
            u.K = J.K + (long long)pu.start * ek;
            if (v_blocks)
                u.Vq = (J.io ? J.io->v.stage : J.Vq) + (long long)pu.start * P.v_rb;
            else
                u.V = J.V + (long long)pu.start * ev;
            u.Q = J.Q;
            u.C = pu.C; u.t = pu.t; u.prefix = pu.prefix; u.nq = pu.nq; u.qmode = pu.qmode;
            u.layer = all[pos].l;
            int off = 0;
            for (int k = 0; k < all[pos].i; k++) off += J.plan->units[k].t;
            u.out_off = off;
            u.token_base = pu.start;
            u.active = 1;
            u.chunk = all[pos].i;
            u.s_off = bt.fs; bt.fs += al32((long long)H * pu.nq * pu.C);
            u.pm_off = bt.fs; bt.fs += al32((long long)H * pu.nq * ((pu.C + 127) / 128));
            u.imp_off = bt.fs; bt.fs += al32((long long)(2 * H + 1) * pu.C);
            u.row_off = bt.fs; bt.fs += al32((long long)2 * H * pu.nq);
            u.y_off = bt.fs; bt.fs += al32((long long)H * pu.nq * dv);
            u.x_off = bt.fs; bt.fs += al32((long long)H * pu.nq * pu.t);
            u.xs_off = bt.fs; bt.fs += al32((long long)2 * H * pu.nq);
            u.omp_off = -1;
            if (p.use_omp) { u.omp_off = bt.fs; bt.fs += al32((long long)kvc_omp_floats(pu.C, pu.t, pu.nq, H)); }
            u.w_off = bt.w_base[u.layer] >= 0 ? bt.w_base[u.layer] + pu.start : -1;
            u.sel_off = bt.is; bt.is += al32(pu.t);
            u.c_off = bt.is; bt.is += al32(4LL * pu.C);
            const int n = std::min(pu.nq, pu.t);
            if (n > ((p.skip_beta && !p.use_omp) ? KVC_LSQ_MAX_N : KVC_NNLS_MAX_N)) return KVC_ERR_SHAPE;
            long long gper = (long long)n * n;
            if (!p.skip_beta) gper = std::max<long long>(gper, (long long)kvc_nnls_doubles_per_head(pu.t, pu.nq));
            u.g_off = bt.gs; bt.gs += al32((long long)H * gper);
            u.z_off = bt.gs; bt.gs += al32((long long)H * n * dv);
            bt.max_nq = std::max(bt.max_nq, pu.nq);
            bt.max_C = std::max(bt.max_C, pu.C);
            bt.max_t = std::max(bt.max_t, pu.t);
            bt.max_n = std::max(bt.max_n, n);
            if (pu.nq < pu.t) bt.any_dual = true;
            else { bt.any_primal = true; bt.n_primal++; }
            if (pu.t % 4) bt.lsq_aligned = false;
            bt.lsq_smem = std::max(bt.lsq_smem, kvc_lsq_smem_bytes(n));
            if (bt.U.empty()) { bt.row0 = pu.start; bt.out0 = off; }
            bt.row1 = pu.start + pu.C;
            bt.out1 = off + pu.t;
            bt.U.push_back(u);
            pos++;
        }
        bt.u0 = first;
        max_fs = std::max(max_fs, bt.fs);
        max_is = std::max(max_is, bt.is);
        max_gs = std::max(max_gs, bt.gs);
        B.push_back(std::move(bt));
    }
    // shared selection: global importance, per-(job, head) sensitivities, and
    // a unit over all T positions whose selection every job then takes
    long long sh_gimp = 0, sh_sens = 0, sh_sel = 0;
    kvc_unit sh_unit;
    memset(&sh_unit, 0, sizeof(sh_unit));
    if (shared) {
        if (B.size() != 1) return KVC_ERR_SHAPE;
        batch & bt = B[0];
        sh_gimp = bt.fs; bt.fs += al32(T_sh);
        sh_sens = bt.fs; bt.fs += al32((long long)n_jobs * H);
        sh_sel = bt.is; bt.is += al32(shared->t);
        sh_unit.c_off = bt.is; bt.is += al32(4LL * T_sh);
        sh_unit.sel_off = sh_sel;
        sh_unit.imp_off = sh_gimp - 2LL * H * T_sh;  // the select kernel reads fs + imp_off + 2*H*C
        sh_unit.C = T_sh;
        sh_unit.t = shared->t;
        sh_unit.layer = n_jobs;
        sh_unit.active = 1;
        max_fs = std::max(max_fs, bt.fs);
        max_is = std::max(max_is, bt.is);
    }
    void * a0; void * a1; void * a2;
    int rc;
    if ((rc = kvc_arena(ctx, 0, (size_t)max_fs * 4, &a0))) return rc;
    if ((rc = kvc_arena(ctx, 1, (size_t)max_is * 4, &a1))) return rc;
    if ((rc = kvc_arena(ctx, 2, (size_t)max_gs * 8, &a2))) return rc;
    float * F = (float *)a0;
    int * I = (int *)a1;
    double * G = (double *)a2;
    // the unit table: every batch's units, the shared-selection unit, then a
    // copy of each batch's primal units (the primal right-hand side product
    // launches over those alone)
    size_t n_primal_all = 0;
    for (const batch & bt : B) n_primal_all += bt.n_primal;
    const size_t n_table = all.size() + (shared ? 1 : 0) + n_primal_all;
    if (ctx->units_cap < n_table) {
        if (ctx->d_units) { KVC_CUDA(cudaStreamSynchronize(st)); cudaFree(ctx->d_units); }
        ctx->units_cap = n_table * 2;
        KVC_CUDA(cudaMalloc(&ctx->d_units, ctx->units_cap * sizeof(kvc_unit)));
    }
    {
        std::vector<kvc_unit> table;
        table.reserve(n_table);
        for (const batch & bt : B) table.insert(table.end(), bt.U.begin(), bt.U.end());
        if (shared) table.push_back(sh_unit);
        for (batch & bt : B) {
            bt.p0 = table.size();
            for (const kvc_unit & u : bt.U)
                if (u.nq >= u.t) table.push_back(u);
        }
        KVC_CUDA(cudaMemcpyAsync(ctx->d_units, table.data(), table.size() * sizeof(kvc_unit),
                                 cudaMemcpyHostToDevice, st));
    }
    if (shared) {                                 // the shared unit's output entry: its selection slot
        kvc_layer_out so;
        memset(&so, 0, sizeof(so));
        so.sel = I + sh_sel;
        so.t_total = shared->t;
        so.n_chunks = 1;
        KVC_CUDA(cudaMemcpyAsync(ctx->d_outs + n_jobs, &so, sizeof(so), cudaMemcpyHostToDevice, st));
    }

    // ---- bulk uploads of a streamed job, group by group on the copy stream.
    // The copy engine serves uploads in the order they become ready: the bulk
    // rows wait for everything queued so far on the compute stream (the small
    // uploads above and the caller's), or they would go ahead of them.
    std::vector<cudaEvent_t> ev_k(B.size(), nullptr), ev_v(B.size(), nullptr);
    if (io) {
        kvc_trace(ctx, "queued", st);
        cudaEvent_t e0 = kvc_sync_event(ctx);
        KVC_CUDA(cudaEventRecord(e0, st));
        KVC_CUDA(cudaStreamWaitEvent(ctx->copy_stream, e0, 0));
        for (size_t bi = 0; bi < B.size(); bi++) {
            const size_t r0 = (size_t)B[bi].row0, nr = (size_t)(B[bi].row1 - B[bi].row0);
            if (!io->k_resident) {
                KVC_CUDA(cudaMemcpyAsync(io->k.stage + r0 * io->k.row_bytes, io->k.host + r0 * io->k.row_bytes,
                                         nr * io->k.row_bytes, cudaMemcpyHostToDevice, ctx->copy_stream));
                ev_k[bi] = kvc_sync_event(ctx);
                KVC_CUDA(cudaEventRecord(ev_k[bi], ctx->copy_stream));
                kvc_trace(ctx, "k" + std::to_string(bi), ctx->copy_stream);
            }
            KVC_CUDA(cudaMemcpyAsync(io->v.stage + r0 * io->v.row_bytes, io->v.host + r0 * io->v.row_bytes,
                                     nr * io->v.row_bytes, cudaMemcpyHostToDevice, ctx->copy_stream));
            ev_v[bi] = kvc_sync_event(ctx);
            KVC_CUDA(cudaEventRecord(ev_v[bi], ctx->copy_stream));
            kvc_trace(ctx, "v" + std::to_string(bi), ctx->copy_stream);
        }
    }
    // rows [r0, r1) of a streamed input are on the device once `e` is reached;
    // quantised rows are then decoded into the job's fp32 matrix
    auto arrive = [&](cudaEvent_t e, const kvc_stream_io::input & in, const float * dst, int ncols, int r0,
                      int r1, cudaStream_t s) -> int {
        KVC_CUDA(cudaStreamWaitEvent(s, e, 0));
        if (in.type < 0 || (v_blocks && &in == &io->v) || (io->k_blocks_only && &in == &io->k))
            return KVC_OK;                                                 // used as they are
        kvc_stage_timer tm(ctx, KVC_ST_DECODE, 1, s);
        return kvc_launch_decode(in.stage + (size_t)r0 * in.row_bytes, in.row_bytes, in.type,
                                 const_cast<float *>(dst) + (size_t)r0 * ncols, r1 - r0, ncols, s);
    };

    // scoring phase of one batch: scores, softmax + importance, selection
    auto scoring = [&](const batch & bt, cudaStream_t s) -> int {
        const int nu = (int)bt.U.size();
        const kvc_unit * du = ctx->d_units + bt.u0;
        int e;
        {
            kvc_stage_timer tm(ctx, KVC_ST_SCORE, 1, s);
            // fused: Y = softmax(S) V comes out of the same launch (timed as scoring)
            e = fused_pv ? kvc_launch_score_pv_tc(du, nu, P, F, d_maps, d_vmaps, tcg, vg, 2, s)
                : tc_score ? kvc_launch_score_tc(du, nu, P, F, d_maps, tcg, 2, s)
                           : kvc_launch_score(du, nu, bt.max_nq, bt.max_C, P, F, 2, s, rows_aligned);
            if (e) return e;
        }
        if (P.use_omp) {                             // needs the raw scores: before the softmax
            kvc_stage_timer tm(ctx, KVC_ST_SELECT, 1, s);
            if ((e = kvc_launch_omp_exp(du, nu, P, F, s))) return e;
        }
        {
            // the tensor-core scoring leaves each row's maximum over the whole chunk
            kvc_stage_timer tm(ctx, KVC_ST_SOFTMAX, 1, s);
            const int tile_keys = tc_score ? bt.max_C : kvc_score_tile_keys(bt.max_nq, rows_aligned);
            if ((e = kvc_launch_softmax_importance(du, nu, bt.max_nq, bt.max_C, tile_keys, P, F, s))) return e;
        }
        kvc_stage_timer tm(ctx, KVC_ST_SELECT, 2, s);
        if ((e = kvc_launch_aggregate(du, nu, P, F, s))) return e;
        if (P.use_omp) return kvc_launch_omp_select(du, nu, P, F, I, ctx->d_outs, s);
        return kvc_launch_select(du, nu, bt.max_C, P, F, I, ctx->d_outs, s);
    };
    // refit phase: Y, then per refinement round X (and beta) and the LS
    // solve for C_v, then the per-chunk metric records
    auto refit = [&](const batch & bt, cudaStream_t s) -> int {
        const int nu = (int)bt.U.size();
        const kvc_unit * du = ctx->d_units + bt.u0;
        const int max_nq = bt.max_nq, max_t = bt.max_t, max_n = bt.max_n;
        int e;
        if (!fused_pv) {
            kvc_stage_timer tm(ctx, KVC_ST_PV, 1, s);
            if ((e = kvc_launch_pv(du, nu, max_nq, P, F, true, s))) return e;
        }
        for (int r = 0; r <= p.refine_rounds; r++) {
            if (r > 0) {
                kvc_stage_timer tm(ctx, KVC_ST_REFINE, 1, s);
                if ((e = kvc_launch_refine(du, nu, P, F, I, ctx->d_outs, s))) return e;
            }
            if (p.skip_beta) {
                kvc_stage_timer tm(ctx, KVC_ST_XBUILD, 1, s);     // X = softmax(S[:, sel]), one pass
                if ((e = kvc_launch_gather_softmax_x(du, nu, max_nq, max_t, P, F, I, s))) return e;
            } else {
                {
                    kvc_stage_timer tm(ctx, KVC_ST_XBUILD, 1, s); // raw S[:, sel], gathered from S
                    if ((e = kvc_launch_gather_x(du, nu, max_nq, P, F, I, s))) return e;
                }
                {
                    kvc_stage_timer tm(ctx, KVC_ST_BETA, 2, s);
                    if ((e = kvc_launch_beta(du, nu, max_nq, max_t, P, F, I, G, ctx->d_outs, s))) return e;
                }
                kvc_stage_timer tm(ctx, KVC_ST_XBUILD, 1, s);     // X = softmax(S[:, sel] + beta)
                if ((e = kvc_launch_softmax_x(du, nu, max_nq, P, F, ctx->d_outs, s))) return e;
            }
            {
                kvc_stage_timer tm(ctx, KVC_ST_LSQ, bt.any_primal ? 2 : 1, s);
                if ((e = kvc_launch_lsq_gram(du, nu, max_n, max_t, P, F, G, ctx->d_outs, ctx->d_units + bt.p0,
                                             bt.n_primal,
                                             bt.lsq_aligned, s)))
                    return e;
            }
            {
                kvc_stage_timer tm(ctx, KVC_ST_LSQ_FACTOR, (max_n > 128 || dv > 128) ? 2 : 1, s);
                if ((e = kvc_launch_lsq_factor(du, nu, max_n, bt.lsq_smem, P, F, G, ctx->d_outs, s))) return e;
            }
            {
                kvc_stage_timer tm(ctx, KVC_ST_LSQ_OUT, bt.any_dual ? 1 : 0, s);
                if ((e = kvc_launch_lsq_out(du, nu, max_t, P, F, G, ctx->d_outs, bt.any_dual, bt.lsq_aligned, s)))
                    return e;
            }
        }
        if (metric_partials) {
            kvc_stage_timer tm(ctx, KVC_ST_METRICS, 1, s);
            if ((e = kvc_launch_metric_partial(du, nu, P, F, ctx->d_outs, s))) return e;
        }
        return KVC_OK;
    };
    auto weights = [&](const batch & bt, cudaStream_t s) -> int {
        for (int l = 0; l < n_jobs; l++)
            if (bt.w_base[l] >= 0)
                KVC_CUDA(cudaMemcpyAsync(F + bt.w_base[l], jobs[l].rkv_w, (size_t)jobs[l].plan->T * 4,
                                         cudaMemcpyDeviceToDevice, s));
        return KVC_OK;
    };

    if (concurrent) {
        // group g on group stream g % KVC_GROUP_STREAMS: its scoring as soon
        // as its K rows are in, its refit once its V rows are in; the streams
        // start after everything queued so far on the compute stream, which
        // joins them all at the end
        if ((rc = weights(B[0], st))) return rc;
        cudaEvent_t e_setup = kvc_sync_event(ctx);
        KVC_CUDA(cudaEventRecord(e_setup, st));
        const size_t n_streams = std::min<size_t>(B.size(), KVC_GROUP_STREAMS);
        for (size_t i = 0; i < n_streams; i++) KVC_CUDA(cudaStreamWaitEvent(ctx->group_stream[i], e_setup, 0));
        for (size_t bi = 0; bi < B.size(); bi++) {
            const batch & bt = B[bi];
            cudaStream_t gs = ctx->group_stream[bi % KVC_GROUP_STREAMS];
            if (ev_k[bi] && (rc = arrive(ev_k[bi], io->k, jobs[0].K, H * dk, bt.row0, bt.row1, gs))) return rc;
            if (fused_pv && (rc = arrive(ev_v[bi], io->v, jobs[0].V, H * dv, bt.row0, bt.row1, gs))) return rc;
            if (phase) KVC_CUDA(cudaEventRecord(phase_event(ctx), gs));
            if ((rc = scoring(bt, gs))) return rc;
            kvc_trace(ctx, "s" + std::to_string(bi), gs);
            if (phase) KVC_CUDA(cudaEventRecord(phase_event(ctx), gs));
            if (!fused_pv && (rc = arrive(ev_v[bi], io->v, jobs[0].V, H * dv, bt.row0, bt.row1, gs))) return rc;
            if ((rc = refit(bt, gs))) return rc;
            if (phase) KVC_CUDA(cudaEventRecord(phase_event(ctx), gs));
            kvc_trace(ctx, "r" + std::to_string(bi), gs);
            if (io->emit && (rc = io->emit(bt.out0, bt.out1, gs))) return rc;
        }
        for (size_t i = 0; i < n_streams; i++) {
            cudaEvent_t ej = kvc_sync_event(ctx);
            KVC_CUDA(cudaEventRecord(ej, ctx->group_stream[i]));
            KVC_CUDA(cudaStreamWaitEvent(st, ej, 0));
        }
        return KVC_OK;
    }
    // scoring phase of the shared selection: scores and importances of every
    // unit, then one selection for all of them
    auto scoring_shared = [&](const batch & bt, cudaStream_t s) -> int {
        const int nu = (int)bt.U.size();
        const kvc_unit * du = ctx->d_units + bt.u0;
        int e;
        {
            kvc_stage_timer tm(ctx, KVC_ST_SCORE, 1, s);
            if ((e = kvc_launch_score(du, nu, bt.max_nq, bt.max_C, P, F, 2, s, rows_aligned))) return e;
        }
        {
            kvc_stage_timer tm(ctx, KVC_ST_SOFTMAX, 1, s);
            if ((e = kvc_launch_softmax_importance(du, nu, bt.max_nq, bt.max_C,
                                                   kvc_score_tile_keys(bt.max_nq, rows_aligned), P, F, s)))
                return e;
        }
        kvc_stage_timer tm(ctx, KVC_ST_SELECT, P.use_sensitivity ? 4 : 3, s);
        return kvc_launch_shared_select(du, nu, ctx->d_units + all.size(), P, F, I, F + sh_gimp, F + sh_sens,
                                        I + sh_sel, T_sh, shared->t, ctx->d_outs, s);
    };
    for (size_t bi = 0; bi < B.size(); bi++) {
        const batch & bt = B[bi];
        if ((rc = weights(bt, st))) return rc;
        if (io && ev_k[bi] && (rc = arrive(ev_k[bi], io->k, jobs[0].K, H * dk, bt.row0, bt.row1, st))) return rc;
        if (io && fused_pv && (rc = arrive(ev_v[bi], io->v, jobs[0].V, H * dv, bt.row0, bt.row1, st))) return rc;
        if (phase) KVC_CUDA(cudaEventRecord(phase_event(ctx), st));
        if ((rc = shared ? scoring_shared(bt, st) : scoring(bt, st))) return rc;
        if (phase) KVC_CUDA(cudaEventRecord(phase_event(ctx), st));
        if (io && !fused_pv && (rc = arrive(ev_v[bi], io->v, jobs[0].V, H * dv, bt.row0, bt.row1, st))) return rc;
        if ((rc = refit(bt, st))) return rc;
        if (phase) KVC_CUDA(cudaEventRecord(phase_event(ctx), st));
        if (io) kvc_trace(ctx, "r" + std::to_string(bi), st);
        if (io && io->emit && (rc = io->emit(bt.out0, bt.out1, st))) return rc;
    }
    return KVC_OK;
}

int kvc_engine_metrics_launch(kvc_ctx * ctx, const kvc_layer_job & job, int H, int dk, int dv, float * d_res) {
    const kvc_plan & pl = *job.plan;
    const int t = job.out.t_total;
    int rc;
    kvc_stage_timer tm(ctx, KVC_ST_METRICS, job.out.mpart ? 1 : 4);
    if (job.out.mpart)              // merge the per-chunk records of the last run
        return kvc_launch_metric_merge(job.out.mpart, job.out.n_chunks, H, pl.nq_top, dv, d_res, ctx->stream);
    if (!job.v_decoded) {           // the run read V in its block format: decode it for the direct metrics
        const bool streamed = job.io != nullptr;
        const uint8_t * src = streamed ? job.io->v.stage : job.Vq;
        if (!src || !job.V) return KVC_ERR_NULL;
        if ((rc = kvc_launch_decode(src, streamed ? job.io->v.row_bytes : job.v_row_bytes,
                                    streamed ? job.io->v.type : job.v_type, const_cast<float *>(job.V), pl.T,
                                    H * dv, ctx->stream)))
            return rc;
    }
    const size_t nf = kvc_metric_scratch_floats(H, pl.nq_top, pl.T, t, dv);
    void * a4;
    if ((rc = kvc_arena(ctx, 4, nf * 4, &a4))) return rc;
    const float isd = 1.0f / sqrtf((float)dk);
    return kvc_launch_metrics(job.K, job.V, job.Q, pl.T, pl.nq_top, H, dk, dv, job.out.sel, job.out.beta,
                              job.out.cv, t, isd, (float *)a4, d_res, ctx->stream);
}

int kvc_engine_metrics(kvc_ctx * ctx, const kvc_layer_job & job, int H, int dk, int dv, kv_compact_stats * st) {
    const int pairs = kvc_metric_pairs(H, job.plan->nq_top);
    void * a9;
    int rc;
    if ((rc = kvc_arena(ctx, 9, ((size_t)pairs * 3 + 64) * 4, &a9))) return rc;
    if ((rc = kvc_engine_metrics_launch(ctx, job, H, dk, dv, (float *)a9))) return rc;
    if ((rc = kvc_wait(ctx))) return rc;
    std::vector<float> h((size_t)pairs * 3);
    KVC_CUDA(cudaMemcpyAsync(h.data(), a9, h.size() * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    kvc_metrics_reduce(h.data(), pairs, st);
    return KVC_OK;
}

// Average the per-pair (cosine, MSE, agreement) triples in the reference's
// order (src/kv-compact-api.cpp:319-324).
void kvc_metrics_reduce(const float * h, int pairs, kv_compact_stats * st) {
    if (getenv("KVC_DEBUG_METRICS"))
        fprintf(stderr, "[kvc] metrics pairs=%d first (cos,mse,agree)=(%g,%g,%g)\n", pairs, h[0], h[1], h[2]);
    float sc = 0.0f, sm = 0.0f;
    int agree = 0;
    for (int i = 0; i < pairs; i++) {
        sc += h[i * 3 + 0];
        sm += h[i * 3 + 1];
        agree += h[i * 3 + 2] > 0.5f ? 1 : 0;
    }
    st->avg_cosine_sim = sc / (float)pairs;
    st->avg_mse = sm / (float)pairs;
    st->avg_agreement = (float)agree / (float)pairs;
}
