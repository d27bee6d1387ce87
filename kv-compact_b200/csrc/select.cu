// select.cu — per-unit key selection.
//
// k_aggregate: global importance of each key of a unit (src/kv-compact-api.cpp:
//   651-684): the max over heads, or the sensitivity-weighted sum over heads
//   (include/kv-compact-math.h:579-618), times the R-KV class weight.
//
// k_select_topt: the t - prefix most important non-prefix keys, plus the
//   prefix (src/kv-compact-api.cpp:717-743). A 4-pass 8-bit radix select over
//   order-preserving uint32 keys finds the exact k-th largest importance.
//   When keys tie exactly at that threshold and not all tied keys fit, the
//   reference's choice among them is whatever libstdc++'s std::partial_sort
//   heap leaves behind; the kernel then replays that heap selection (the
//   classic hole-sifting binary heap, on one thread over the unit's
//   importances in shared memory) so exact ties resolve as they do there.
//   Selected positions are emitted in ascending order by a block-wide scan.
//
// k_select_diverse: greedy cosine-diversity selection (src/kv-compact-api.cpp:
//   175-233): t - prefix sequential steps, each an argmax of
//   imp*(1 - strength*penalty) (first index wins ties) followed by a
//   penalty update with the cosine between the chosen key and every unused
//   key over the full n_embd = H*d_k row. Dot products and norms keep the
//   reference's sequential fp32 order; norms are computed once per key.
#include "engine.h"

#include <math.h>

#include <algorithm>

namespace {

__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions for blockDim.x <= 1024 (multiple of 32).
__device__ float block_max(float v, float * sh) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = (threadIdx.x < nw) ? sh[threadIdx.x] : -INFINITY;
    if (w == 0) r = warp_max(r);
    if (threadIdx.x == 0) sh[0] = r;
    __syncthreads();
    r = sh[0];
    __syncthreads();
    return r;
}
__device__ float block_sum(float v, float * sh) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = (threadIdx.x < nw) ? sh[threadIdx.x] : 0.0f;
    if (w == 0) r = warp_sum(r);
    if (threadIdx.x == 0) sh[0] = r;
    __syncthreads();
    r = sh[0];
    __syncthreads();
    return r;
}

// Exclusive scan of one int per thread; returns the prefix, total in *tot.
__device__ int block_scan(int v, int * sh, int * tot) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = (lane < nw) ? sh[lane] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < nw) sh[lane] = s;
    }
    __syncthreads();
    int base = (w > 0) ? sh[w - 1] : 0;
    *tot = sh[nw - 1];
    __syncthreads();
    return base + x - v;
}

// --- libstdc++-compatible heap selection (one thread) ----------------------
struct HeapCtx {
    const float * imp;
    __device__ bool before(int a, int b) const { return imp[a] > imp[b]; }
};

__device__ void heap_push_up(int * h, int hole, int top, int val, const HeapCtx & c) {
    int parent = (hole - 1) / 2;
    while (hole > top && c.before(h[parent], val)) {
        h[hole] = h[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    h[hole] = val;
}

__device__ void heap_adjust(int * h, int hole, int len, int val, const HeapCtx & c) {
    int top = hole, child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (c.before(h[child], h[child - 1])) child--;
        h[hole] = h[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        h[hole] = h[child - 1];
        hole = child - 1;
    }
    heap_push_up(h, hole, top, val, c);
}

// Heap-select the k best of candidates first..C-1 (indices into imp).
__device__ void heap_select(int * heap, int first, int C, int k, const float * imp) {
    HeapCtx c{imp};
    for (int i = 0; i < k; i++) heap[i] = first + i;
    if (k >= 2) {
        for (int parent = (k - 2) / 2;; parent--) {
            heap_adjust(heap, parent, k, heap[parent], c);
            if (parent == 0) break;
        }
    }
    for (int i = first + k; i < C; i++)
        if (c.before(i, heap[0])) heap_adjust(heap, 0, k, i, c);
}

}  // namespace

__global__ void __launch_bounds__(256) k_aggregate(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                   float * __restrict__ fs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    const int C = u.C, H = P.H;
    float * gimp = fs + u.imp_off + (long long)2 * H * C;
    __shared__ float red[32];
    __shared__ float sens[64];
    if (P.use_sensitivity) {
        for (int h = 0; h < H; h++) {
            const float * cm = fs + u.imp_off + (long long)(H + h) * C;
            float mx = 0.0f, sm = 0.0f;
            for (int j = threadIdx.x; j < C; j += blockDim.x) {
                float v = cm[j];
                if (v > mx) mx = v;
                sm = __fadd_rn(sm, v);
            }
            mx = block_max(mx, red);
            sm = block_sum(sm, red);
            if (threadIdx.x == 0 && h < 64) {
                float mean = __fdiv_rn(sm, (float)C);
                sens[h] = __fdiv_rn(mx, __fadd_rn(mean, 1e-12f));
            }
        }
        __syncthreads();
    }
    const float * w = u.w_off >= 0 ? fs + u.w_off : nullptr;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        float g = 0.0f;
        for (int h = 0; h < H; h++) {
            float v = fs[u.imp_off + (long long)h * C + j];
            if (P.use_sensitivity) g = __fadd_rn(g, __fmul_rn(sens[h < 64 ? h : 63], v));
            else if (v > g) g = v;
        }
        if (w) g = __fmul_rn(g, w[j]);
        gimp[j] = g;
    }
}

// Emit the flagged positions of a unit in ascending order.
__device__ void emit_selected(const kvc_unit & u, const int * flags, int * sel,
                              const kvc_layer_out & lo, int * shi) {
    int base = 0;
    for (int j0 = 0; j0 < u.C; j0 += blockDim.x) {
        int j = j0 + threadIdx.x;
        int f = (j < u.C) ? flags[j] : 0;
        int tot;
        int pos = block_scan(f, shi, &tot);
        if (f && base + pos < u.t) {
            sel[base + pos] = j;
            lo.sel[u.out_off + base + pos] = u.token_base + j;
        }
        base += tot;
    }
}

__global__ void __launch_bounds__(1024) k_select_topt(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                      float * __restrict__ fs, int * __restrict__ is,
                                                      const kvc_layer_out * __restrict__ outs, int smem_floats) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    extern __shared__ float dyn[];
    __shared__ int hist[256];
    __shared__ int shi[33];
    __shared__ uint32_t s_prefix;
    __shared__ int s_k, s_gt, s_eq;
    const int C = u.C, pc = u.prefix, k = u.t - u.prefix, ncand = C - pc;
    const float * gimp = fs + u.imp_off + (long long)2 * P.H * C;
    int * flags = is + u.c_off;
    int * sel = is + u.sel_off;
    const kvc_layer_out lo = outs[u.layer];

    if (k <= 0 || k >= ncand) {
        for (int j = threadIdx.x; j < C; j += blockDim.x) flags[j] = (j < pc || k > 0) ? 1 : 0;
        __syncthreads();
        emit_selected(u, flags, sel, lo, shi);
        return;
    }
    if (threadIdx.x == 0) { s_prefix = 0; s_k = k; s_gt = 0; s_eq = 0; }
    for (int pass = 0; pass < 4; pass++) {
        const int shift = 24 - 8 * pass;
        for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
        __syncthreads();
        const uint32_t pre = s_prefix;
        const uint32_t hmask = (pass == 0) ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
        for (int j = pc + threadIdx.x; j < C; j += blockDim.x) {
            uint32_t key = kvc_fkey(gimp[j]);
            if ((key & hmask) == (pre & hmask)) atomicAdd(&hist[(key >> shift) & 0xFF], 1);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int kk = s_k, cum = 0, b = 255;
            for (; b > 0; b--) {
                if (cum + hist[b] >= kk) break;
                cum += hist[b];
            }
            s_gt += cum;
            s_k = kk - cum;
            s_prefix = pre | ((uint32_t)b << shift);
            s_eq = hist[b];
        }
        __syncthreads();
    }
    const uint32_t kth = s_prefix;
    const int need = k - s_gt;
    if (need == s_eq) {
        for (int j = threadIdx.x; j < C; j += blockDim.x)
            flags[j] = (j < pc) ? 1 : (kvc_fkey(gimp[j]) >= kth ? 1 : 0);
    } else {
        // exact ties straddle the cut: replay the reference's heap selection
        for (int j = threadIdx.x; j < C; j += blockDim.x) flags[j] = (j < pc) ? 1 : 0;
        const float * imp = gimp;
        int * heap = is + u.c_off + C;
        if (C + k <= smem_floats) {
            float * simp = dyn;
            for (int j = threadIdx.x; j < C; j += blockDim.x) simp[j] = gimp[j];
            imp = simp;
            heap = reinterpret_cast<int *>(dyn + C);
        }
        __syncthreads();
        if (threadIdx.x == 0) heap_select(heap, pc, C, k, imp);
        __syncthreads();
        for (int i = threadIdx.x; i < k; i += blockDim.x) flags[heap[i]] = 1;
    }
    __syncthreads();
    emit_selected(u, flags, sel, lo, shi);
}

__global__ void __launch_bounds__(1024) k_select_diverse(const kvc_unit * __restrict__ units,
                                                         kvc_params_dev P, float * __restrict__ fs,
                                                         int * __restrict__ is,
                                                         const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.x];
    if (!u.active) return;
    const int C = u.C, t = u.t, pc = u.prefix;
    const int ek = P.H * P.dk;
    const float * gimp = fs + u.imp_off + (long long)2 * P.H * C;
    int * used = is + u.c_off;
    float * pen = reinterpret_cast<float *>(is + u.c_off + C);
    float * nrm = reinterpret_cast<float *>(is + u.c_off + 2 * (long long)C);
    int * order = is + u.c_off + 3 * (long long)C;
    int * sel = is + u.sel_off;
    const kvc_layer_out lo = outs[u.layer];
    extern __shared__ float ks[];           // the chosen key row (ek floats)
    __shared__ float rs[32];
    __shared__ int ri[32];
    __shared__ int shi[33];
    __shared__ int s_best;

    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        used[j] = j < pc ? 1 : 0;
        pen[j] = 0.0f;
        const float * kj = u.K + (long long)j * ek;
        float n2 = 0.0f;
        for (int d = 0; d < ek; d++) n2 = __fadd_rn(n2, __fmul_rn(kj[d], kj[d]));
        nrm[j] = sqrtf(n2);
    }
    for (int j = threadIdx.x; j < pc; j += blockDim.x) order[j] = j;
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int n = pc;
    while (n < t) {
        float bs = -1e30f;
        int bi = 0x7fffffff;
        for (int j = threadIdx.x; j < C; j += blockDim.x) {
            if (used[j]) continue;
            float sc = __fmul_rn(gimp[j], __fsub_rn(1.0f, __fmul_rn(P.diversity_strength, pen[j])));
            if (sc > bs) { bs = sc; bi = j; }   // ascending j per thread: first max kept
        }
        for (int o = 16; o; o >>= 1) {
            float s2 = __shfl_xor_sync(0xffffffffu, bs, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (s2 > bs || (s2 == bs && i2 < bi)) { bs = s2; bi = i2; }
        }
        if (lane == 0) { rs[w] = bs; ri[w] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            float b = rs[0];
            int i = ri[0];
            for (int k = 1; k < nw; k++)
                if (rs[k] > b || (rs[k] == b && ri[k] < i)) { b = rs[k]; i = ri[k]; }
            s_best = (b > -1e30f && i != 0x7fffffff) ? i : -1;
            if (s_best >= 0) { used[s_best] = 1; order[n] = s_best; }
        }
        __syncthreads();
        const int best = s_best;
        if (best < 0) break;
        n++;
        const float * kb = u.K + (long long)best * ek;
        for (int d = threadIdx.x; d < ek; d += blockDim.x) ks[d] = kb[d];
        __syncthreads();
        const float ns = __fadd_rn(nrm[best], 1e-8f);
        for (int j = threadIdx.x; j < C; j += blockDim.x) {
            if (used[j]) continue;
            const float * kj = u.K + (long long)j * ek;
            float dot = 0.0f;
            for (int d = 0; d < ek; d++) dot = __fadd_rn(dot, __fmul_rn(ks[d], kj[d]));
            float cs = __fdiv_rn(dot, __fadd_rn(__fmul_rn(ns, nrm[j]), 1e-8f));
            if (cs > pen[j]) pen[j] = cs;
        }
        __syncthreads();
    }
    // ascending order of the chosen positions
    for (int j = threadIdx.x; j < C; j += blockDim.x) used[j] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) used[order[i]] = 1;
    __syncthreads();
    emit_selected(u, used, sel, lo, shi);
}

// ---- one selection shared by every unit of a call ---------------------------
// (the llama.cpp state path: one unit per layer spanning all cells; the cells
// kept must be the same in every layer, src/kv-compact.cpp:470-566)

// Sensitivity of each (unit, head): max_j cmax[j] / (mean_j cmax[j] + 1e-12)
// of the per-key maximum attention (include/kv-compact-math.h:579-594),
// reduced as k_aggregate reduces it.
__global__ void __launch_bounds__(256) k_unit_head_sens(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                                        const float * __restrict__ fs, float * __restrict__ sens) {
    const kvc_unit u = units[blockIdx.y];
    const int h = blockIdx.x, C = u.C, H = P.H;
    __shared__ float red[32];
    const float * cm = fs + u.imp_off + (long long)(H + h) * C;
    float mx = 0.0f, sm = 0.0f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        const float v = cm[j];
        if (v > mx) mx = v;
        sm = __fadd_rn(sm, v);
    }
    mx = block_max(mx, red);
    sm = block_sum(sm, red);
    if (threadIdx.x == 0) sens[blockIdx.y * H + h] = __fdiv_rn(mx, __fadd_rn(__fdiv_rn(sm, (float)C), 1e-12f));
}

// Importance of every position over all units and heads: the maximum of the
// per-head importances, or (with sensitivity weighting) the sum of s * imp
// accumulated unit by unit, head by head, as the reference accumulates it
// layer by layer (accumulate_weighted_importance, math.h:607-618).
__global__ void __launch_bounds__(256) k_global_importance(const kvc_unit * __restrict__ units, int n_units,
                                                           kvc_params_dev P, const float * __restrict__ fs,
                                                           const float * __restrict__ sens, int T,
                                                           float * __restrict__ gimp) {
    extern __shared__ long long imp_base[];         // per unit: offset of its head-0 importance
    for (int i = threadIdx.x; i < n_units; i += blockDim.x) imp_base[i] = units[i].imp_off;
    __syncthreads();
    const int H = P.H;
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < T; j += (long long)gridDim.x * blockDim.x) {
        float g = 0.0f;
        for (int i = 0; i < n_units; i++)
            for (int h = 0; h < H; h++) {
                const float v = fs[imp_base[i] + (long long)h * T + j];
                if (P.use_sensitivity) g = __fadd_rn(g, __fmul_rn(sens[i * H + h], v));
                else if (v > g) g = v;
            }
        gimp[j] = g;
    }
}

// The shared selection (positions 0..T-1, ascending) into every unit's
// selection slot and its layer's output indices.
__global__ void k_broadcast_sel(const kvc_unit * __restrict__ units, int * __restrict__ is,
                                const int * __restrict__ sel, int t, const kvc_layer_out * __restrict__ outs) {
    const kvc_unit u = units[blockIdx.y];
    const kvc_layer_out lo = outs[u.layer];
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < t; j += gridDim.x * blockDim.x) {
        is[u.sel_off + j] = sel[j];
        lo.sel[u.out_off + j] = u.token_base + sel[j];
    }
}

int kvc_launch_shared_select(const kvc_unit * d_units, int n_units, const kvc_unit * d_all, const kvc_params_dev & P,
                             float * fs, int * is, float * gimp, float * sens, const int * all_sel, int T, int t,
                             const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    if (P.use_sensitivity) {
        k_unit_head_sens<<<dim3(P.H, n_units), 256, 0, st>>>(d_units, P, fs, sens);
        KVC_CUDA(cudaGetLastError());
    }
    const int g = (int)std::min<long long>(((long long)T + 255) / 256, 148LL * 8);
    k_global_importance<<<g, 256, (size_t)n_units * sizeof(long long), st>>>(d_units, n_units, P, fs, sens, T, gimp);
    KVC_CUDA(cudaGetLastError());
    kvc_params_dev Ps = P;                          // plain top-t over all positions
    Ps.use_diversity = 0;
    int rc;
    if ((rc = kvc_launch_select(d_all, 1, T, Ps, fs, is, d_outs, st))) return rc;
    const int gx = (t + 255) / 256 < 64 ? (t + 255) / 256 : 64;
    k_broadcast_sel<<<dim3(gx > 0 ? gx : 1, n_units), 256, 0, st>>>(d_units, is, all_sel, t, d_outs);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_aggregate(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs,
                         cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    k_aggregate<<<n_units, 256, 0, st>>>(d_units, P, fs);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_select(const kvc_unit * d_units, int n_units, int max_C, const kvc_params_dev & P, float * fs,
                      int * is, const kvc_layer_out * d_outs, cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    if (P.use_diversity) {
        size_t sm = (size_t)P.H * P.dk * sizeof(float);
        if (sm > 48 * 1024) KVC_CUDA(cudaFuncSetAttribute(k_select_diverse, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        k_select_diverse<<<n_units, 1024, sm, st>>>(d_units, P, fs, is, d_outs);
    } else {
        // importances + heap in shared memory when they fit (2 * max_C floats)
        size_t want = (size_t)2 * max_C * sizeof(float);
        size_t cap = 160 * 1024;
        size_t sm = want < cap ? want : cap;
        if (sm > 48 * 1024) KVC_CUDA(cudaFuncSetAttribute(k_select_topt, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        k_select_topt<<<n_units, 1024, sm, st>>>(d_units, P, fs, is, d_outs, (int)(sm / sizeof(float)));
    }
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
