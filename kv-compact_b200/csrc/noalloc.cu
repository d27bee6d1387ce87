// noalloc.cu — multi-head scoring that allocates no device memory.
//
// kv_compact_cuda_score_all_heads stages its host operands and the scores in
// device buffers it allocates on first use and keeps. Some callers cannot let
// a library allocate: serving engines that reserve all of HBM for their own
// allocator, or paths that must not add the latency and device-wide
// synchronisation of cudaMalloc/cudaFree. This variant runs the same scoring
// kernel (k_score) with its staging buffers and work-unit descriptor in a
// file-scope __device__ array instead, so it never calls cudaMalloc, cudaFree
// or any allocating routine.
//
// The array (KVC_NOALLOC_SCRATCH_FLOATS floats, 16 MiB) is part of the
// library image: every GPU that loads libkvc.so holds it until the process
// exits. A call needs n_q*H*d_k + T*H*d_k + H*n_q*T floats (each region
// rounded up to 64 floats); larger sizes are rejected with -13 and a message.
// Host code cannot use the array's name as a device address, so on the first
// call on each device (with that device current) the address is looked up
// with cudaGetSymbolAddress and cached; make that first call before any stream
// capture. All calls share the array and it keeps the last call's contents;
// every region is fully overwritten before it is read, so nothing has to start
// at zero. Calls made from this process are serialised by a mutex; calls that
// overlap on the GPU from elsewhere (another thread bypassing it, or another
// stream still reading a previous result) race on the array.
#include <limits.h>

#include <mutex>

#include "engine.h"

#define KVC_NOALLOC_SCRATCH_FLOATS (4u << 20)   // 4,194,304 floats = 16 MiB

static __device__ __align__(256) float kvc_noalloc_scratch[KVC_NOALLOC_SCRATCH_FLOATS];
static __device__ __align__(256) kvc_unit kvc_noalloc_unit;

namespace {
std::mutex g_mu;
float * g_scratch[64];        // device address of kvc_noalloc_scratch, per device
kvc_unit * g_unit[64];        // device address of kvc_noalloc_unit, per device

inline size_t up64(size_t n) { return (n + 63) & ~size_t(63); }
}  // namespace

extern "C" KVC_EXPORT int kv_compact_cuda_score_all_heads_noalloc(const float * Q_ref, const float * K_all,
                                                                   float ** scores_out, int n_q, int T,
                                                                   int n_head_kv, int d_k, float scale) {
    if (!Q_ref || !K_all || !scores_out || n_q <= 0 || T <= 0 || n_head_kv <= 0 || d_k <= 0) return -1;
    int dev = -1, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return -1; }
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major < 10) {
        cudaGetLastError();
        return -1;
    }
    // every product in size_t, and the head width bounded before it is used
    // as an int, so absurd arguments cannot wrap into a size that passes
    if (d_k > KVC_MAX_D || (size_t)n_head_kv * (size_t)d_k > (size_t)INT_MAX) return -1;
    const int H = n_head_kv, ek = H * d_k;
    const size_t nQ = up64((size_t)n_q * (size_t)ek), nK = up64((size_t)T * (size_t)ek);
    const size_t nS = up64((size_t)H * (size_t)n_q * (size_t)T);
    if (nQ + nK + nS > KVC_NOALLOC_SCRATCH_FLOATS) {
        fprintf(stderr,
                "[kvc] kv_compact_cuda_score_all_heads_noalloc: n_q=%d T=%d heads=%d d_k=%d needs %zu floats of "
                "scratch, the static array holds %u\n",
                n_q, T, H, d_k, nQ + nK + nS, KVC_NOALLOC_SCRATCH_FLOATS);
        return KVC_ERR_SHAPE;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch[dev]) {
        void * a = nullptr;
        void * b = nullptr;
        if (cudaGetSymbolAddress(&a, kvc_noalloc_scratch) != cudaSuccess ||
            cudaGetSymbolAddress(&b, kvc_noalloc_unit) != cudaSuccess) {
            fprintf(stderr, "[kvc] cudaGetSymbolAddress failed for the no-allocation scratch on device %d\n", dev);
            cudaGetLastError();
            return -1;
        }
        g_scratch[dev] = (float *)a;
        g_unit[dev] = (kvc_unit *)b;
    }
    float * base = g_scratch[dev];
    float * dQ = base;
    float * dK = dQ + nQ;
    float * dS = dK + nK;
    cudaStream_t st = cudaStreamPerThread;
    // An error after copies were queued waits for the stream first: the
    // copies read the caller's host buffers, which the caller may release
    // as soon as this call returns.
    auto fail = [st]() {
        cudaStreamSynchronize(st);
        cudaGetLastError();
        return -1;
    };
    if (cudaMemcpyAsync(dQ, Q_ref, (size_t)n_q * ek * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) return fail();
    if (cudaMemcpyAsync(dK, K_all, (size_t)T * ek * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) return fail();
    kvc_unit u;
    memset(&u, 0, sizeof(u));
    u.K = dK;
    u.Q = dQ;
    u.C = T;
    u.t = T;
    u.nq = n_q;
    u.active = 1;
    u.s_off = (long long)(dS - base);
    if (cudaMemcpyAsync(g_unit[dev], &u, sizeof(u), cudaMemcpyHostToDevice, st) != cudaSuccess) return fail();
    kvc_params_dev P;
    memset(&P, 0, sizeof(P));
    P.H = H;
    P.dk = d_k;
    P.dv = d_k;
    P.isd = scale;
    if (kvc_launch_score(g_unit[dev], 1, n_q, T, P, base, 0, st) != KVC_OK) return fail();
    for (int h = 0; h < H; h++)
        if (cudaMemcpyAsync(scores_out[h], dS + (size_t)h * n_q * T, (size_t)n_q * T * 4, cudaMemcpyDeviceToHost,
                            st) != cudaSuccess)
            return fail();
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    return 0;
}
