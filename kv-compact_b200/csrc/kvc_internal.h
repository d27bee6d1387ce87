// kvc_internal.h — shared definitions of the B200 compaction engine.
//
// A "unit" is one (layer, chunk) of a compaction call with all of its KV
// heads: the reference compacts each chunk independently (src/kv-compact-api.cpp:
// 462-499) and shares one key selection across the heads of a call
// (src/kv-compact-api.cpp:651-744), so a unit is the natural piece of work
// for one kernel stage. Every stage runs over a flat list of units.
//
// Device layout (all row-major, resident in HBM):
//   K, V          [T x H*d] fp32 per layer (dequantised once if stored quantised)
//   S             per (unit, head) [n_q x C] raw scores (kept: consumers of the
//                 softmax A form it from S and the row statistics)
//   imp           per (unit, head) [C] importance, plus [C] aggregated per unit
//   Y             per (unit, head) [n_q x d_v] = A_h V_h
//   X             per (unit, head) [n_q x t]   = softmax(S[:, sel] + beta)
//   G             per (unit, head) [n x n] fp64, n = min(n_q, t)
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#define KVC_HD __host__ __device__ __forceinline__
// Public entry points keep default visibility; everything else is hidden.
#define KVC_EXPORT __attribute__((visibility("default")))

// Return codes added by this library (kv-compact-api.h lists them).
enum {
    KVC_OK = 0,
    KVC_ERR_NULL = -1,
    KVC_ERR_DIMS = -2,
    KVC_ERR_ROUNDS = -3,
    KVC_ERR_ROWSIZE = -4,
    KVC_ERR_NODEV = -10,
    KVC_ERR_OOM = -11,
    KVC_ERR_CUDA = -12,
    KVC_ERR_SHAPE = -13,
};

#define KVC_CUDA(call)                                                               \
    do {                                                                             \
        cudaError_t e_ = (call);                                                     \
        if (e_ != cudaSuccess) {                                                     \
            fprintf(stderr, "[kvc] CUDA error %s at %s:%d: %s\n", cudaGetErrorName(e_), \
                    __FILE__, __LINE__, cudaGetErrorString(e_));                     \
            return (e_ == cudaErrorMemoryAllocation) ? KVC_ERR_OOM : KVC_ERR_CUDA;   \
        }                                                                            \
    } while (0)

// Largest head dimension the kernels are instantiated for.
#define KVC_MAX_D 256
// Most unknowns of one least-squares solve (min(n_q, t) of a chunk): the
// global-memory Cholesky's right-hand-side panel must fit shared memory.
// The beta fit and OMP selection keep their own bound (KVC_NNLS_MAX_N).
#define KVC_LSQ_MAX_N 24576
#define KVC_NNLS_MAX_N 3072
// Most layers of one batched requantisation launch (kvc_launch_requant_batch).
#define KVC_RQ_MAX_LAYERS 64

struct kvc_unit {
    const float * K;      // first row of the chunk, row stride ek = H*d_k
    const float * V;      // first row of the chunk, row stride ev = H*d_v
    const float * Q;      // first reference-query row (qmode 0), row stride ek
    const uint8_t * Vq;   // or null: first V row in its block format (kvc_params_dev::v_type, v_rb), V unused
    int C;                // tokens in the chunk
    int t;                // keys kept
    int prefix;           // positions 0..prefix-1 always kept (prefix <= t)
    int nq;               // reference queries
    int qmode;            // 0: rows of Q; 1: cheap queries = K rows of the chunk
    int layer;            // output layer slot
    int out_off;          // first output slot of this unit within the layer
    int token_base;       // chunk start within the layer (added to indices)
    int active;           // refinement: 0 once the unit stopped swapping
    int chunk;            // chunk index within its layer
    long long s_off;      // floats: raw scores S, H blocks of nq*C
    long long imp_off;    // floats: 2H+1 blocks of C (per head, per-head column max, aggregated)
    long long row_off;    // floats: H blocks of nq (row max / row sum)
    long long y_off;      // floats: H blocks of nq*dv
    long long x_off;      // floats: H blocks of nq*t
    long long g_off;      // doubles: H blocks of n*n (NNLS: its own per-head stride)
    long long z_off;      // doubles: H blocks of n*d_v (dual Z, or primal X^T Y)
    long long sel_off;    // ints: t selected chunk-local positions
    long long w_off;      // floats: C R-KV weights (or -1: none)
    long long c_off;      // ints/floats: C per-candidate scratch (selection)
    long long xs_off;     // floats: H blocks of 2*nq (row max, row sum of X before normalising)
    long long omp_off;    // floats: OMP selection working arrays (omp.cu), or -1
    long long pm_off;     // floats: H blocks of nq x ceil(C/128) row maxima of the score tiles (mode 2)
};

struct kvc_layer_out {
    int * sel;            // [t_total] global positions (device)
    float * beta;         // [H][t_total]
    float * cv;           // [H][t_total][d_v]
    int t_total;
    int n_chunks;         // units of this layer
    float * mpart;        // per-chunk quality-metric partials, or null (metrics.cu)
};

struct kvc_params_dev {
    int H, dk, dv;
    int score_method;     // 0 max, 1 rms, 2 mean
    int skip_beta;
    int use_sensitivity;
    int use_diversity;
    float diversity_strength;
    int nnls_method;
    int nnls_max_iter;
    int nnls_pgd_iters;
    float ridge;
    float isd;            // 1/sqrtf(d_k), computed as the reference does
    int use_omp;
    int omp_k_choice;
    int omp_refit_interval;
    int v_type;           // block format of the units' Vq rows (8 Q8_0, 2 Q4_0, 3 Q4_1)
    long long v_rb;       // bytes per Vq row
};

// f32 arithmetic that is never contracted into FMA, on host and device.
KVC_HD float kvc_mul(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
KVC_HD float kvc_add(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}
KVC_HD float kvc_sub(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fsub_rn(a, b);
#else
    return a - b;
#endif
}
KVC_HD float kvc_div(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fdiv_rn(a, b);
#else
    return a / b;
#endif
}

// Order-preserving map of a float onto uint32 (larger float -> larger key).
KVC_HD uint32_t kvc_fkey(float f) {
    uint32_t u;
#ifdef __CUDA_ARCH__
    u = __float_as_uint(f);
#else
    memcpy(&u, &f, 4);
#endif
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---- codecs (codec.cu) ----------------------------------------------------
int kvc_row_elements(int type, size_t row_bytes);
size_t kvc_row_bytes(int type, int n);
int kvc_block_bytes(int type);
void kvc_host_decode_row(const uint8_t * src, int type, float * dst, size_t n);
size_t kvc_host_encode_row(const float * src, int type, uint8_t * dst, int n);
int kvc_launch_decode(const uint8_t * src, size_t src_row_bytes, int type, float * dst,
                      int rows, int n, cudaStream_t st);
int kvc_launch_encode_gather(const float * src, size_t src_stride, const int * rows_idx,
                             int rows, int n, int type, uint8_t * dst, size_t dst_row_bytes,
                             cudaStream_t st);
// Output row r = encode(decode(src row idx[r])) straight from the stored
// rows (K_out without an fp32 copy of K), bit-identical to decoding first.
int kvc_launch_transcode_gather(const uint8_t * src, size_t src_rb, const int * idx, int rows, int n, int type,
                                uint8_t * dst, size_t dst_rb, cudaStream_t st);
// V_out rows 0..rows-1 from cv[h][j][:] (heads t rows apart).
int kvc_launch_encode_heads(const float * cv, int H, int t, int rows, int dv, int type, uint8_t * dst,
                            size_t dst_row_bytes, cudaStream_t st);
// The K_out transcode (k_dst != nullptr) and the V_out encode (v_dst !=
// nullptr) of n layers in one launch each, the same bytes as the per-layer
// kvc_launch_transcode_gather / kvc_launch_encode_heads. Returns
// KVC_ERR_SHAPE, launching nothing, where a layer needs the general kernels
// (types, row sizes, alignment; more than KVC_RQ_MAX_LAYERS layers).
int kvc_launch_requant_batch(int n, const uint8_t * const * k_src, const int * const * sel, const int * t,
                             uint8_t * const * k_dst, size_t k_rb, int ek, int k_type, const float * const * cv,
                             uint8_t * const * v_dst, size_t v_rb, int H, int dv, int v_type, cudaStream_t st);
