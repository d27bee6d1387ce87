// pv_tc.cu — refit target Y_h = A_h V_h on the tcgen05 tensor cores.
//
// Y is the right-hand side of the value refit (src/kv-compact-api.cpp:754-783,
// include/kv-compact-math.h:70-80): A = softmax weights of the chunk's
// reference queries [n_q x C], V = the chunk's value rows of head h
// [C x d_v]. The refit tolerates fp32-level rounding (never bit-compared), so
// the product runs on the tensor cores in kind::tf32 with the 3xTF32 split:
// every fp32 operand x ~= hi + lo, hi = x rounded to TF32, lo = (x - hi)
// rounded to TF32 (both exactly representable for the tensor core), and
//   A V ~= A_lo V_hi + A_hi V_lo + A_hi V_hi
// accumulated in fp32 in TMEM — relative error ~1e-6, the same order as an
// fp32 SIMT product.
//
// One CTA of 4 warps per (unit, head): M = 128 query rows (zero-padded),
// N = d_v, K = the chunk's keys in stages of 16. Per stage every thread loads
// its share of A (float4 along keys) and V (coalesced along d_v) into
// registers, splits it and stores hi/lo tiles into shared memory in the
// K-major no-swizzle canonical layout; thread 0 issues the six MMAs of the
// stage and commits them to the stage buffer's mbarrier. Two stage buffers:
// the loads of stage s+1 are in flight while the tensor core works on stage
// s, and a buffer is rewritten only after its mbarrier reports that the MMAs
// reading it completed. Every mbarrier wait is bounded; a wait that runs out
// records an error (kvc_tc_take_error) and the CTA frees its TMEM and stops.
#include "engine.h"
#include "tc_sm100.h"

#include <cuda_fp16.h>

namespace {
constexpr int PV_M = 128;                    // tile rows (queries)
constexpr int PV_KS = 16;                    // keys per stage
constexpr int PV_LBO = 128;                  // bytes between 16-byte K chunks (one core matrix)
constexpr int PV_SBO = (PV_KS / 4) * PV_LBO; // bytes between 8-row groups
constexpr uint32_t PV_POLLS = 1u << 20;      // bound of every mbarrier wait

__device__ int g_tc_error;                   // first error code of a tcgen05 kernel (0: none)

template <int DV>
constexpr uint32_t pv_stage_bytes() { return 2u * (PV_M / 8) * PV_SBO + 2u * (DV / 8) * PV_SBO; }
template <int DV>
constexpr uint32_t pv_tmem_cols() { return DV <= 32 ? 32 : (DV <= 64 ? 64 : (DV <= 128 ? 128 : 256)); }
}  // namespace

// Raw bytes of value n of head h in a V row kept in its block format (VT: 8
// Q8_0, 2 Q4_0, 3 Q4_1; head h's values start at block h * DV / 32), packed
// for key slot e of a four-key unit: the code byte into byte e of w[0], the
// block's fp16 scale into half e & 1 of w[1 + e / 2], the Q4_1 minimum into
// half e & 1 of w[3 + e / 2].
template <int VT, int DV>
__device__ __forceinline__ void vq_raw(const uint8_t * __restrict__ row, int h, int n, int e, uint32_t * w) {
    constexpr int BB = VT == 8 ? 34 : (VT == 2 ? 18 : 20);
    const uint8_t * blk = row + (h * (DV / 32) + (n >> 5)) * BB;
    const int i = n & 31;
    const uint32_t code = VT == 8 ? blk[2 + i] : blk[(VT == 2 ? 2 : 4) + (i >> 1)];
    w[0] |= code << (8 * e);
    w[1 + (e >> 1)] |= (uint32_t)(*reinterpret_cast<const unsigned short *>(blk)) << (16 * (e & 1));
    if (VT == 3) w[3 + (e >> 1)] |= (uint32_t)(*reinterpret_cast<const unsigned short *>(blk + 2)) << (16 * (e & 1));
}

// The value of key slot e from vq_raw's packing, with the arithmetic of the
// codec's decode (separately rounded multiply and add): the same fp32 value a
// decoded V row holds. An empty slot (zero scale and minimum) gives 0.
template <int VT>
__device__ __forceinline__ float vq_cook(const uint32_t * w, int n, int e) {
    const float d = __half2float(__ushort_as_half((unsigned short)(w[1 + (e >> 1)] >> (16 * (e & 1)))));
    const uint32_t q = (w[0] >> (8 * e)) & 0xFFu;
    if (VT == 8) return __fmul_rn(d, (float)(int8_t)q);
    const uint32_t nib = (n & 1) ? q >> 4 : q & 0xFu;
    if (VT == 2) return __fmul_rn(d, __fsub_rn((float)nib, 8.0f));
    const float m = __half2float(__ushort_as_half((unsigned short)(w[3 + (e >> 1)] >> (16 * (e & 1)))));
    return __fadd_rn(__fmul_rn(d, (float)nib), m);
}

// One (unit, head) tile. FULL: every query row exists (n_q = 128), every
// stage holds 16 keys and the score rows are 16-byte aligned, so the loads
// and conversions run without per-element bounds predicates (measured on a
// cfg4 batch: 2.67 ms against 3.49 ms with the predicates). VT: 0 when V is
// an fp32 matrix (u.V), else the block format of u.Vq's rows, decoded here
// (no fp32 copy of V is written or read: on the cfg4 batch 2.92 ms, against
// 2.66 ms plus about 1.3 ms for decoding V first).
template <int DV, bool FULL, int VT>
__device__ __forceinline__ void pv_tile(const kvc_unit & u, const int h, const kvc_params_dev & P,
                                        float * __restrict__ fs, const int from_scores, uint8_t * smem,
                                        uint64_t * mbar, uint32_t * tmem_slot_p) {
    using namespace kvc_tc;
    constexpr int NPB = DV / 32;                       // (row, k-quad) pairs of V per thread and stage
    constexpr uint32_t A_BYTES = (PV_M / 8) * PV_SBO;  // one A tile (hi or lo)
    constexpr uint32_t B_BYTES = (DV / 8) * PV_SBO;    // one B tile
    constexpr uint32_t STAGE = pv_stage_bytes<DV>();
    constexpr uint32_t NCOLS = pv_tmem_cols<DV>();
    const int ev = P.H * DV, nq = u.nq, C = u.C;
    const float * A = fs + u.s_off + (long long)h * nq * C;     // A, or raw scores A is formed from
    const float * rmax = fs + u.row_off + (long long)h * 2 * nq;
    const float * V = VT ? nullptr : u.V + (long long)h * DV;
    float * Y = fs + u.y_off + (long long)h * nq * DV;
    uint32_t & tmem_slot = *tmem_slot_p;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) tmem_alloc(&tmem_slot, NCOLS);
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_init_fence();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_slot;
    constexpr uint32_t IDESC = idesc_tf32(PV_M, DV);
    const int nst = (C + PV_KS - 1) / PV_KS;
    const bool avec = ((C & 3) == 0) && ((((uintptr_t)A) & 15) == 0);

    // row statistics of the four A rows this thread stages (the same rows in every stage)
    float am[4], ainv[4];
#pragma unroll
    for (int it = 0; it < 4; it++) {
        const int idx = it * 128 + tid;
        const int r = ((idx >> 5) << 3) | (idx & 7);
        const bool rs = from_scores && r < nq;
        am[it] = rs ? rmax[r] : 0.0f;
        ainv[it] = rs ? __fdiv_rn(1.0f, __fadd_rn(rmax[nq + r], 1e-12f)) : 0.0f;
    }
    // from scores: A = exp(s - m) * inv, the softmax of score.cu with the
    // hardware exponential (Y only feeds the least-squares right-hand side and
    // the quality metrics, both tolerance-checked; its relative error stays
    // near 1e-6, like the 3xTF32 products); else the given weights; zero
    // outside the tile
    auto a_entry = [&](float sv, int it, bool live) {
        if (!FULL && !live) return 0.0f;
        return from_scores ? __fmul_rn(__expf(__fsub_rn(sv, am[it])), ainv[it]) : sv;
    };
    // two register sets: the stages s+1 and s+2 are in flight while stage s
    // is converted into shared memory (one stage of loads per thread alone
    // leaves too few bytes in flight to keep HBM busy)
    float4 ra[2][4];
    float rb[2][NPB][4];                               // fp32 V (VT 0)
    // block-format V (VT != 0): the raw bytes, turned into values only when
    // the stage is stored (two stages after the loads were issued), so no
    // warp waits on its V loads: [0] = the four codes (key e in byte e),
    // [1], [2] = the fp16 scales of keys 0-1 and 2-3, [3], [4] = their Q4_1
    // minima
    uint32_t rv[2][NPB][VT == 3 ? 5 : 3];
    auto load = [&](int s, int p) {
        const int k0 = s * PV_KS;
#pragma unroll
        for (int it = 0; it < 4; it++) {               // A rows: a quarter-warp covers 8 rows of one k-quad
            const int idx = it * 128 + tid;
            const int r = ((idx >> 5) << 3) | (idx & 7), kq = (idx >> 3) & 3;
            const int k = k0 + 4 * kq;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (FULL) {
                v = *reinterpret_cast<const float4 *>(A + (long long)r * C + k);
            } else if (r < nq) {
                const float * p = A + (long long)r * C + k;
                if (avec && k + 4 <= C) {
                    v = *reinterpret_cast<const float4 *>(p);
                } else {
                    if (k + 0 < C) v.x = p[0];
                    if (k + 1 < C) v.y = p[1];
                    if (k + 2 < C) v.z = p[2];
                    if (k + 3 < C) v.w = p[3];
                }
            }
            ra[p][it] = v;
        }
#pragma unroll
        for (int pb = 0; pb < NPB; pb++) {             // V: lanes run along d_v (coalesced rows)
            const int idx = pb * 128 + tid;
            const int n = idx % DV, kq = idx / DV;
            const int k = k0 + 4 * kq;
            if (VT) {
                uint32_t w[VT == 3 ? 5 : 3] = {};
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    if (!FULL && k + e >= C) continue;          // zero scale (and minimum): value 0
                    vq_raw<VT, DV>(u.Vq + (long long)(k + e) * P.v_rb, h, n, e, w);
                }
#pragma unroll
                for (int i = 0; i < (VT == 3 ? 5 : 3); i++) rv[p][pb][i] = w[i];
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++) rb[p][pb][e] = (!FULL && k + e >= C) ? 0.0f : V[(long long)(k + e) * ev + n];
            }
        }
    };
    auto store = [&](int b, int s, int p) {
        uint8_t * base = smem + b * STAGE;
#pragma unroll
        for (int it = 0; it < 4; it++) {
            const int idx = it * 128 + tid;
            const int r = ((idx >> 5) << 3) | (idx & 7), kq = (idx >> 3) & 3;
            const int k = s * PV_KS + 4 * kq;
            const uint32_t off = (r >> 3) * PV_SBO + kq * PV_LBO + (r & 7) * 16;
            const bool rl = r < nq;
            const float a0 = a_entry(ra[p][it].x, it, rl && k + 0 < C), a1 = a_entry(ra[p][it].y, it, rl && k + 1 < C);
            const float a2 = a_entry(ra[p][it].z, it, rl && k + 2 < C), a3 = a_entry(ra[p][it].w, it, rl && k + 3 < C);
            float4 hi, lo;
            tf32_split(a0, hi.x, lo.x);
            tf32_split(a1, hi.y, lo.y);
            tf32_split(a2, hi.z, lo.z);
            tf32_split(a3, hi.w, lo.w);
            *reinterpret_cast<float4 *>(base + off) = hi;
            *reinterpret_cast<float4 *>(base + A_BYTES + off) = lo;
        }
#pragma unroll
        for (int pb = 0; pb < NPB; pb++) {
            const int idx = pb * 128 + tid;
            const int n = idx % DV, kq = idx / DV;
            const uint32_t off = (n >> 3) * PV_SBO + kq * PV_LBO + (n & 7) * 16;
            float v[4];
            if (VT) {
#pragma unroll
                for (int e = 0; e < 4; e++) v[e] = vq_cook<VT>(rv[p][pb], n, e);
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++) v[e] = rb[p][pb][e];
            }
            float4 hi, lo;
            tf32_split(v[0], hi.x, lo.x);
            tf32_split(v[1], hi.y, lo.y);
            tf32_split(v[2], hi.z, lo.z);
            tf32_split(v[3], hi.w, lo.w);
            *reinterpret_cast<float4 *>(base + 2 * A_BYTES + off) = hi;
            *reinterpret_cast<float4 *>(base + 2 * A_BYTES + B_BYTES + off) = lo;
        }
    };

    load(0, 0);
    if (nst > 1) load(1, 1);
    int s = 0, err = 0;
    for (; s < nst; s++) {
        const int b = s & 1;                      // stage buffer = register set
        bool ok = true;
        if (s >= 2) ok = mbar_wait(&mbar[b], (uint32_t)(((s - 2) >> 1) & 1), PV_POLLS);
        if (b == 0) {
            store(0, s, 0);
            if (s + 2 < nst) load(s + 2, 0);
        } else {
            store(1, s, 1);
            if (s + 2 < nst) load(s + 2, 1);
        }
        fence_smem_to_async();
        if (__syncthreads_or(!ok)) {          // every thread takes the same decision
            err = 1;
            break;
        }
        if (tid == 0) {
            fence_after_sync();
            const uint32_t sa = smem_u32(smem + b * STAGE);
#pragma unroll
            for (int ks = 0; ks < PV_KS / 8; ks++) {
                const uint32_t ko = ks * 2 * PV_LBO;
                const uint64_t ahi = sdesc(sa + ko, PV_LBO, PV_SBO);
                const uint64_t alo = sdesc(sa + A_BYTES + ko, PV_LBO, PV_SBO);
                const uint64_t bhi = sdesc(sa + 2 * A_BYTES + ko, PV_LBO, PV_SBO);
                const uint64_t blo = sdesc(sa + 2 * A_BYTES + B_BYTES + ko, PV_LBO, PV_SBO);
                mma_tf32(tmem, alo, bhi, IDESC, (s | ks) != 0);
                mma_tf32(tmem, ahi, blo, IDESC, 1u);
                mma_tf32(tmem, ahi, bhi, IDESC, 1u);
            }
            commit(&mbar[b]);
        }
    }
    // the last issued commit covers every MMA of the CTA
    const int last = s - 1;
    bool ok = true;
    if (last >= 0) ok = mbar_wait(&mbar[last & 1], (uint32_t)((last >> 1) & 1), PV_POLLS);
    if (__syncthreads_or(!ok)) err |= 2;
    fence_after_sync();
    if (!err) {
        const int q = 32 * warp + lane;
#pragma unroll
        for (int c0 = 0; c0 < DV; c0 += 16) {
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
            if (q < nq) {
                float4 * dst = reinterpret_cast<float4 *>(Y + (long long)q * DV + c0);
#pragma unroll
                for (int i = 0; i < 4; i++) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
        }
    } else if (tid == 0) {
        atomicCAS(&g_tc_error, 0, 100 + err);
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_free(tmem, NCOLS);
}

template <int DV>
__global__ void __launch_bounds__(128) k_pv_tc(const kvc_unit * __restrict__ units, kvc_params_dev P,
                                               float * __restrict__ fs, int from_scores) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ uint32_t tmem_slot;
    const kvc_unit u = units[blockIdx.x];
    const int h = blockIdx.y;
    const float * A = fs + u.s_off + (long long)h * u.nq * u.C;
    const bool full = u.nq == PV_M && (u.C % PV_KS) == 0 && ((((uintptr_t)A) & 15) == 0);
    if (!u.Vq) {
        if (full) pv_tile<DV, true, 0>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
        else pv_tile<DV, false, 0>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
    } else if (P.v_type == 8) {
        if (full) pv_tile<DV, true, 8>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
        else pv_tile<DV, false, 8>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
    } else if (P.v_type == 2) {
        if (full) pv_tile<DV, true, 2>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
        else pv_tile<DV, false, 2>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
    } else {
        if (full) pv_tile<DV, true, 3>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
        else pv_tile<DV, false, 3>(u, h, P, fs, from_scores, smem, mbar, &tmem_slot);
    }
}

// Whether k_pv_tc handles this shape (else the SIMT k_pv does).
bool kvc_pv_tc_ok(int max_nq, int dv) {
    return max_nq <= PV_M && (dv == 64 || dv == 128 || dv == 256) && getenv("KVC_NO_TC") == nullptr;
}

int kvc_launch_pv_tc(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs, bool from_scores,
                     cudaStream_t st) {
    if (n_units <= 0) return KVC_OK;
    const dim3 grid(n_units, P.H);
    switch (P.dv) {
        case 64: {
            const uint32_t sm = 2 * pv_stage_bytes<64>();
            KVC_CUDA(cudaFuncSetAttribute(k_pv_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
            k_pv_tc<64><<<grid, 128, sm, st>>>(d_units, P, fs, from_scores ? 1 : 0);
            break;
        }
        case 128: {
            const uint32_t sm = 2 * pv_stage_bytes<128>();
            KVC_CUDA(cudaFuncSetAttribute(k_pv_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
            k_pv_tc<128><<<grid, 128, sm, st>>>(d_units, P, fs, from_scores ? 1 : 0);
            break;
        }
        case 256: {
            const uint32_t sm = 2 * pv_stage_bytes<256>();
            KVC_CUDA(cudaFuncSetAttribute(k_pv_tc<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
            k_pv_tc<256><<<grid, 128, sm, st>>>(d_units, P, fs, from_scores ? 1 : 0);
            break;
        }
        default:
            return KVC_ERR_SHAPE;
    }
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

// Read and clear the error code left by a tcgen05 kernel (stream must be idle).
int kvc_tc_take_error(cudaStream_t st) {
    int h = 0;
    const int zero = 0;
    if (cudaMemcpyFromSymbolAsync(&h, g_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return -1;
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    if (h && cudaMemcpyToSymbolAsync(g_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) == cudaSuccess)
        cudaStreamSynchronize(st);
    return h;
}
