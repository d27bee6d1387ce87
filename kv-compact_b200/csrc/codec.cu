// codec.cu — F32/F16/Q8_0/Q4_0/Q4_1 row codecs, bit-exact with the reference.
//
// The reference codecs (include/kv-compact-state.h:326-629) define:
//   * F16 decode: exact IEEE half -> float (subnormals normalised, NaN payload kept)
//   * F16 encode: mantissa TRUNCATION (no rounding), exponent < -10 -> +-0,
//     overflow and NaN -> +-inf
//   * Q8_0 (34 B / 32 values): d = f16trunc(amax/127), q = (int8)roundf(clamp(x*127/amax))
//   * Q4_0 (18 B): d = f16trunc(amax/7), q = clamp(roundf(x*7/amax + 8)), nibbles lo|hi<<4
//   * Q4_1 (20 B): d = f16trunc((max-min)/15), m = f16trunc(min),
//     q = clamp(roundf((x-min)*15/(max-min)))
// The block functions below are __host__ __device__ so the host entry points
// (kv_quantize_row / kv_dequantize_row) and the device kernels share one
// definition. Every multiply/add is an explicit round-to-nearest operation
// (kvc_mul/kvc_add), never contracted, because the reference (x86-64 without
// FMA) rounds after each operation.
#include "kvc_internal.h"

#include <math.h>

#include <algorithm>

#define QK 32

KVC_HD float kvc_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int ee = 1;
            while (!(m & 0x400u)) { m <<= 1; ee--; }
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(ee + 112) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
#ifdef __CUDA_ARCH__
    return __uint_as_float(bits);
#else
    float f;
    memcpy(&f, &bits, 4);
    return f;
#endif
}

KVC_HD uint16_t kvc_f2h_trunc(float v) {
#ifdef __CUDA_ARCH__
    uint32_t f = __float_as_uint(v);
#else
    uint32_t f;
    memcpy(&f, &v, 4);
#endif
    uint32_t sign = (f >> 16) & 0x8000u;
    int e = (int)((f >> 23) & 0xFFu) - 112;
    uint32_t m = (f >> 13) & 0x3FFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        return (uint16_t)(sign | ((m | 0x400u) >> (1 - e)));
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | m);
}

// max(lo, min(hi, v)) in std::min/std::max operand order (NaN -> hi).
KVC_HD float kvc_clamp(float v, float lo, float hi) {
    float m = (v < hi) ? v : hi;
    return (lo < m) ? m : lo;
}

KVC_HD float kvc_roundf(float x) { return roundf(x); }

int kvc_block_bytes(int type) {
    switch (type) {
    case 0: return 4;
    case 1: return 2;
    case 8: return 34;
    case 2: return 18;
    case 3: return 20;
    default: return 4;
    }
}

static bool is_block(int type) { return type == 8 || type == 2 || type == 3; }

int kvc_row_elements(int type, size_t row_bytes) {
    if (type == 0) return (int)(row_bytes / 4);
    if (type == 1) return (int)(row_bytes / 2);
    if (is_block(type)) return (int)(row_bytes / (size_t)kvc_block_bytes(type)) * QK;
    return (int)(row_bytes / 4);
}

size_t kvc_row_bytes(int type, int n) {
    if (type == 0) return (size_t)n * 4;
    if (type == 1) return (size_t)n * 2;
    if (is_block(type)) return (size_t)(n / QK) * (size_t)kvc_block_bytes(type);
    return (size_t)n * 4;
}

// ---- one 32-value block ---------------------------------------------------
KVC_HD uint16_t ld16(const uint8_t * p) { return (uint16_t)(p[0] | (p[1] << 8)); }
KVC_HD void st16(uint8_t * p, uint16_t v) { p[0] = (uint8_t)(v & 0xFF); p[1] = (uint8_t)(v >> 8); }

KVC_HD void decode_block(const uint8_t * b, int type, float * o) {
    float d = kvc_h2f(ld16(b));
    if (type == 8) {
        for (int i = 0; i < QK; i++) o[i] = kvc_mul(d, (float)(int8_t)b[2 + i]);
    } else if (type == 2) {
        for (int i = 0; i < QK / 2; i++) {
            uint8_t q = b[2 + i];
            o[2 * i] = kvc_mul(d, kvc_sub((float)(q & 0xF), 8.0f));
            o[2 * i + 1] = kvc_mul(d, kvc_sub((float)(q >> 4), 8.0f));
        }
    } else {
        float m = kvc_h2f(ld16(b + 2));
        for (int i = 0; i < QK / 2; i++) {
            uint8_t q = b[4 + i];
            o[2 * i] = kvc_add(kvc_mul(d, (float)(q & 0xF)), m);
            o[2 * i + 1] = kvc_add(kvc_mul(d, (float)(q >> 4)), m);
        }
    }
}

KVC_HD void encode_block(const float * x, int type, uint8_t * o) {
    if (type == 8 || type == 2) {
        float amax = 0.0f;
        for (int i = 0; i < QK; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
        float lim = (type == 8) ? 127.0f : 7.0f;
        float d = kvc_div(amax, lim);
        st16(o, kvc_f2h_trunc(d));
        float id = (d != 0.0f) ? kvc_div(lim, amax) : 0.0f;
        if (type == 8) {
            for (int i = 0; i < QK; i++)
                o[2 + i] = (uint8_t)(int8_t)kvc_roundf(kvc_clamp(kvc_mul(x[i], id), -128.0f, 127.0f));
        } else {
            for (int i = 0; i < QK / 2; i++) {
                float v0 = kvc_add(kvc_mul(x[2 * i], id), 8.0f);
                float v1 = kvc_add(kvc_mul(x[2 * i + 1], id), 8.0f);
                uint8_t q0 = (uint8_t)kvc_clamp(kvc_roundf(v0), 0.0f, 15.0f);
                uint8_t q1 = (uint8_t)kvc_clamp(kvc_roundf(v1), 0.0f, 15.0f);
                o[2 + i] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    } else {
        float lo = x[0], hi = x[0];
        for (int i = 1; i < QK; i++) { if (x[i] < lo) lo = x[i]; if (x[i] > hi) hi = x[i]; }
        float rng = kvc_sub(hi, lo);
        float d = kvc_div(rng, 15.0f);
        st16(o, kvc_f2h_trunc(d));
        st16(o + 2, kvc_f2h_trunc(lo));
        float id = (d != 0.0f) ? kvc_div(15.0f, rng) : 0.0f;
        for (int i = 0; i < QK / 2; i++) {
            float v0 = kvc_mul(kvc_sub(x[2 * i], lo), id);
            float v1 = kvc_mul(kvc_sub(x[2 * i + 1], lo), id);
            uint8_t q0 = (uint8_t)kvc_clamp(kvc_roundf(v0), 0.0f, 15.0f);
            uint8_t q1 = (uint8_t)kvc_clamp(kvc_roundf(v1), 0.0f, 15.0f);
            o[4 + i] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

// ---- host rows -------------------------------------------------------------
void kvc_host_decode_row(const uint8_t * src, int type, float * dst, size_t n) {
    if (type == 0) { memcpy(dst, src, n * 4); return; }
    if (type == 1) {
        for (size_t i = 0; i < n; i++) dst[i] = kvc_h2f(ld16(src + 2 * i));
        return;
    }
    if (!is_block(type)) { memset(dst, 0, n * 4); return; }
    size_t nb = n / QK, bb = (size_t)kvc_block_bytes(type);
    for (size_t b = 0; b < nb; b++) decode_block(src + b * bb, type, dst + b * QK);
}

size_t kvc_host_encode_row(const float * src, int type, uint8_t * dst, int n) {
    if (type == 0) { memcpy(dst, src, (size_t)n * 4); return (size_t)n * 4; }
    if (type == 1) {
        for (int i = 0; i < n; i++) st16(dst + 2 * i, kvc_f2h_trunc(src[i]));
        return (size_t)n * 2;
    }
    if (!is_block(type)) return 0;
    int nb = n / QK, bb = kvc_block_bytes(type);
    for (int b = 0; b < nb; b++) encode_block(src + b * QK, type, dst + (size_t)b * bb);
    return (size_t)nb * (size_t)bb;
}

// ---- device kernels --------------------------------------------------------
// Block formats run 8 threads per 32-value block, 4 values per thread, so a
// warp covers 4 consecutive blocks: it reads their bytes contiguously and
// writes (decode) or reads (encode) 512 contiguous bytes of floats. Every
// value goes through the same arithmetic as decode_block / encode_block.

// Values 4*sub .. 4*sub+3 of one block.
__device__ __forceinline__ void decode_quad(const uint8_t * b, int type, int sub, float * o) {
    const float d = kvc_h2f(ld16(b));
    if (type == 8) {
        const uint16_t w0 = ld16(b + 2 + 4 * sub), w1 = ld16(b + 4 + 4 * sub);
        const int8_t q[4] = {(int8_t)(w0 & 0xFF), (int8_t)(w0 >> 8), (int8_t)(w1 & 0xFF), (int8_t)(w1 >> 8)};
#pragma unroll
        for (int i = 0; i < 4; i++) o[i] = kvc_mul(d, (float)q[i]);
    } else if (type == 2) {
        const uint16_t w = ld16(b + 2 + 2 * sub);
        const uint8_t q0 = (uint8_t)(w & 0xFF), q1 = (uint8_t)(w >> 8);
        o[0] = kvc_mul(d, kvc_sub((float)(q0 & 0xF), 8.0f));
        o[1] = kvc_mul(d, kvc_sub((float)(q0 >> 4), 8.0f));
        o[2] = kvc_mul(d, kvc_sub((float)(q1 & 0xF), 8.0f));
        o[3] = kvc_mul(d, kvc_sub((float)(q1 >> 4), 8.0f));
    } else {
        const float m = kvc_h2f(ld16(b + 2));
        const uint16_t w = ld16(b + 4 + 2 * sub);
        const uint8_t q0 = (uint8_t)(w & 0xFF), q1 = (uint8_t)(w >> 8);
        o[0] = kvc_add(kvc_mul(d, (float)(q0 & 0xF)), m);
        o[1] = kvc_add(kvc_mul(d, (float)(q0 >> 4)), m);
        o[2] = kvc_add(kvc_mul(d, (float)(q1 & 0xF)), m);
        o[3] = kvc_add(kvc_mul(d, (float)(q1 >> 4)), m);
    }
}

// IT: the index type of the flat quad index — 32-bit whenever the launch's
// quads fit (the row / block split then costs a 32-bit division instead of
// a 64-bit one, which dominated these memory-bound loops).
template <typename IT>
__global__ void k_decode_blocks(const uint8_t * __restrict__ src, size_t rb, int type,
                                float * __restrict__ dst, int rows, int n) {
    const int nb = n / QK;
    const IT total = (IT)rows * (IT)nb * 8;
    const int bb = (type == 8) ? 34 : (type == 2 ? 18 : 20);
    for (IT i = (IT)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (IT)gridDim.x * blockDim.x) {
        const IT gb = i >> 3;
        const int sub = (int)(i & 7);
        const IT r = gb / (IT)nb;
        const int b = (int)(gb - r * (IT)nb);
        float o[4];
        decode_quad(src + (size_t)r * rb + (size_t)b * bb, type, sub, o);
        float * q = dst + (long long)r * n + (long long)b * QK + 4 * sub;
        if ((((uintptr_t)q) & 15) == 0) {
            *reinterpret_cast<float4 *>(q) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
            for (int k = 0; k < 4; k++) q[k] = o[k];
        }
    }
}

__global__ void k_decode_elems(const uint8_t * __restrict__ src, size_t rb, int type,
                               float * __restrict__ dst, int rows, int n) {
    long long total = (long long)rows * n;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        long long r = i / n;
        int e = (int)(i - r * n);
        const uint8_t * p = src + r * rb;
        if (type == 1) {
            dst[i] = kvc_h2f(ld16(p + 2 * e));
        } else if (type == 0) {
            float v;
            memcpy(&v, p + 4 * e, 4);
            dst[i] = v;
        } else {
            dst[i] = 0.0f;
        }
    }
}

// Packed rows (row bytes = blocks x block bytes, 16-byte aligned source): the
// tensor is one run of blocks. A CTA takes 64 blocks at a time: their bytes
// come in as 16-byte loads (the next span's already in flight while this one
// decodes), staged in shared memory, and each thread decodes 8 values of one
// block into two float4 stores. Measured on a cfg4 K (12 x 101,120 rows of
// 1,024 Q8_0 values): 1.25 ms against 1.44 ms for k_decode_blocks, whose
// per-thread byte loads straight from global memory cost more instructions.
template <int TYPE>
__global__ void __launch_bounds__(256) k_decode_span(const uint8_t * __restrict__ src, float * __restrict__ dst,
                                                     long long nblocks) {
    constexpr int BB = TYPE == 8 ? 34 : (TYPE == 2 ? 18 : 20);
    constexpr int SPB = 64, SB = SPB * BB, NV = SB / 16;
    static_assert(SB % 16 == 0, "a span is whole 16-byte pieces");
    __shared__ __align__(16) uint8_t sb[2][SB];
    const long long nsp = (nblocks + SPB - 1) / SPB;
    auto fetch = [&](long long sp, uint4 & r) {
        const long long b0 = sp * SPB;
        if (sp >= nsp || threadIdx.x >= NV) return;
        const int nbytes = (int)min((long long)SPB, nblocks - b0) * BB, o = threadIdx.x * 16;
        if (o + 16 <= nbytes) r = *reinterpret_cast<const uint4 *>(src + b0 * BB + o);
    };
    uint4 r = make_uint4(0, 0, 0, 0);
    long long sp = blockIdx.x;
    fetch(sp, r);
    for (int buf = 0; sp < nsp; sp += gridDim.x, buf ^= 1) {
        const long long b0 = sp * SPB;
        const int nb = (int)min((long long)SPB, nblocks - b0), nbytes = nb * BB;
        if (threadIdx.x < NV) {
            const int o = threadIdx.x * 16;
            if (o + 16 <= nbytes) *reinterpret_cast<uint4 *>(sb[buf] + o) = r;
            else
                for (int i = o; i < nbytes && i < o + 16; i++) sb[buf][i] = src[b0 * BB + i];
        }
        r = make_uint4(0, 0, 0, 0);
        fetch(sp + gridDim.x, r);
        __syncthreads();        // this span staged; the buffer written next was last read two spans ago
        const int blk = threadIdx.x >> 2, part = threadIdx.x & 3;
        if (blk < nb) {
            float o[8];
            decode_quad(sb[buf] + blk * BB, TYPE, 2 * part, o);
            decode_quad(sb[buf] + blk * BB, TYPE, 2 * part + 1, o + 4);
            float4 * q = reinterpret_cast<float4 *>(dst + (b0 + blk) * QK + 8 * part);
            q[0] = make_float4(o[0], o[1], o[2], o[3]);
            q[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
    }
}

static int grid_for(long long work, int threads) {
    long long g = (work + threads - 1) / threads;
    if (g > 148LL * 64) g = 148LL * 64;
    if (g < 1) g = 1;
    return (int)g;
}

int kvc_launch_decode(const uint8_t * src, size_t rb, int type, float * dst, int rows, int n,
                      cudaStream_t st) {
    if (rows <= 0 || n <= 0) return KVC_OK;
    if (is_block(type) && rb == (size_t)(n / QK) * (size_t)kvc_block_bytes(type) && (((uintptr_t)src) & 15) == 0 &&
        (((uintptr_t)dst) & 15) == 0) {
        const long long nblocks = (long long)rows * (n / QK);
        if (nblocks == 0) return KVC_OK;
        const long long nsp = (nblocks + 63) / 64;
        const int grid = (int)std::min<long long>(nsp, 148LL * 32);
        if (type == 8) k_decode_span<8><<<grid, 256, 0, st>>>(src, dst, nblocks);
        else if (type == 2) k_decode_span<2><<<grid, 256, 0, st>>>(src, dst, nblocks);
        else k_decode_span<3><<<grid, 256, 0, st>>>(src, dst, nblocks);
    } else if (is_block(type)) {
        long long work = (long long)rows * (n / QK) * 8;
        if (work + (long long)148 * 64 * 256 + 64 < (1LL << 32))   // the last grid-stride step stays below 2^32
            k_decode_blocks<uint32_t><<<grid_for(work, 256), 256, 0, st>>>(src, rb, type, dst, rows, n);
        else
            k_decode_blocks<unsigned long long><<<grid_for(work, 256), 256, 0, st>>>(src, rb, type, dst, rows, n);
    } else {
        long long work = (long long)rows * n;
        k_decode_elems<<<grid_for(work, 256), 256, 0, st>>>(src, rb, type, dst, rows, n);
    }
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

// Encode values 4*sub .. 4*sub+3 of a block held by the 8 lanes of an
// aligned lane group (x: this lane's 4 values, x0: the block's first value);
// the block statistics are combined with shuffles inside the group.
__device__ __forceinline__ void encode_quad(const float * x, float x0, int type, int sub, uint8_t * o) {
    if (type == 8 || type == 2) {
        float amax = 0.0f;                               // NaN never wins: skipped as in encode_block
#pragma unroll
        for (int i = 0; i < 4; i++) { const float a = fabsf(x[i]); if (a > amax) amax = a; }
#pragma unroll
        for (int off = 4; off; off >>= 1) {
            const float b = __shfl_xor_sync(0xffffffffu, amax, off, 8);
            if (b > amax) amax = b;
        }
        const float lim = (type == 8) ? 127.0f : 7.0f;
        const float d = kvc_div(amax, lim);
        if (sub == 0) st16(o, kvc_f2h_trunc(d));
        const float id = (d != 0.0f) ? kvc_div(lim, amax) : 0.0f;
        if (type == 8) {
            uint8_t q[4];
#pragma unroll
            for (int i = 0; i < 4; i++) q[i] = (uint8_t)(int8_t)kvc_roundf(kvc_clamp(kvc_mul(x[i], id), -128.0f, 127.0f));
            st16(o + 2 + 4 * sub, (uint16_t)(q[0] | (q[1] << 8)));
            st16(o + 4 + 4 * sub, (uint16_t)(q[2] | (q[3] << 8)));
        } else {
            uint8_t q[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                q[i] = (uint8_t)kvc_clamp(kvc_roundf(kvc_add(kvc_mul(x[i], id), 8.0f)), 0.0f, 15.0f);
            st16(o + 2 + 2 * sub, (uint16_t)((q[0] | (q[1] << 4)) | ((q[2] | (q[3] << 4)) << 8)));
        }
    } else {
        float lo = x0, hi = x0;                          // a NaN first value poisons both, as in encode_block
#pragma unroll
        for (int i = 0; i < 4; i++) { if (x[i] < lo) lo = x[i]; if (x[i] > hi) hi = x[i]; }
#pragma unroll
        for (int off = 4; off; off >>= 1) {
            const float a = __shfl_xor_sync(0xffffffffu, lo, off, 8);
            const float b = __shfl_xor_sync(0xffffffffu, hi, off, 8);
            if (a < lo) lo = a;
            if (b > hi) hi = b;
        }
        const float rng = kvc_sub(hi, lo);
        const float d = kvc_div(rng, 15.0f);
        if (sub == 0) {
            st16(o, kvc_f2h_trunc(d));
            st16(o + 2, kvc_f2h_trunc(lo));
        }
        const float id = (d != 0.0f) ? kvc_div(15.0f, rng) : 0.0f;
        uint8_t q[4];
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = (uint8_t)kvc_clamp(kvc_roundf(kvc_mul(kvc_sub(x[i], lo), id)), 0.0f, 15.0f);
        st16(o + 4 + 2 * sub, (uint16_t)((q[0] | (q[1] << 4)) | ((q[2] | (q[3] << 4)) << 8)));
    }
}

__device__ __forceinline__ bool dev_is_block(int type) { return type == 8 || type == 2 || type == 3; }

// Block formats: thread i handles quarter `i & 7` of block `i >> 3`. The
// loop bound is rounded up to whole warps so every lane of a group reaches
// the shuffles; lanes past the end only take part in them.
__device__ __forceinline__ long long warp_round(long long n) { return (n + 31) & ~31LL; }

// K_out rows: row j = src[rows_idx[j]] (fp32, stride src_stride) re-encoded.
template <typename IT>
__global__ void k_encode_gather(const float * __restrict__ src, size_t stride,
                                const int * __restrict__ idx, int rows, int n, int type,
                                uint8_t * __restrict__ dst, size_t drb) {
    if (dev_is_block(type)) {
        const int nb = n / QK, bb = (type == 8) ? 34 : (type == 2 ? 18 : 20);
        const IT total = (IT)rows * (IT)nb * 8, total_w = (total + 31) & ~(IT)31;
        for (IT i = (IT)blockIdx.x * blockDim.x + threadIdx.x; i < total_w; i += (IT)gridDim.x * blockDim.x) {
            const bool live = i < total;
            const IT gb = live ? (i >> 3) : 0;
            const int sub = (int)(i & 7);
            const IT r = gb / (IT)nb;
            const int b = (int)(gb - r * (IT)nb);
            const float * row = src + (idx ? (long long)idx[r] : (long long)r) * (long long)stride + (long long)b * QK;
            float x[4];
            if ((((uintptr_t)(row + 4 * sub)) & 15) == 0) {
                const float4 v = *reinterpret_cast<const float4 *>(row + 4 * sub);
                x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
            } else {
#pragma unroll
                for (int k = 0; k < 4; k++) x[k] = row[4 * sub + k];
            }
            uint8_t tmp[34];
            uint8_t * o = live ? dst + (size_t)r * drb + (size_t)b * bb : tmp;
            encode_quad(x, row[0], type, sub, o);
        }
        return;
    }
    const IT total = (IT)rows * (IT)n;
    for (IT i = (IT)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (IT)gridDim.x * blockDim.x) {
        const IT r = i / (IT)n;
        const int e = (int)(i - r * (IT)n);
        const float v = src[(idx ? (long long)idx[r] : (long long)r) * (long long)stride + e];
        uint8_t * o = dst + (size_t)r * drb;
        if (type == 1) st16(o + 2 * e, kvc_f2h_trunc(v));
        else memcpy(o + 4 * e, &v, 4);
    }
}

// V_out rows: row j (of `rows`), element e = h*dv + k comes from
// cv[h][j][k], heads `t` rows apart.
template <typename IT>
__global__ void k_encode_heads(const float * __restrict__ cv, int H, int t, int rows, int dv, int type,
                               uint8_t * __restrict__ dst, size_t drb) {
    const int n = H * dv;
    if (dev_is_block(type)) {
        const int nb = n / QK, bb = (type == 8) ? 34 : (type == 2 ? 18 : 20);
        const IT total = (IT)rows * (IT)nb * 8, total_w = (total + 31) & ~(IT)31;
        for (IT i = (IT)blockIdx.x * blockDim.x + threadIdx.x; i < total_w; i += (IT)gridDim.x * blockDim.x) {
            const bool live = i < total;
            const IT gb = live ? (i >> 3) : 0;
            const int sub = (int)(i & 7);
            const IT j = gb / (IT)nb;
            const int b = (int)(gb - j * (IT)nb);
            float x[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int e = b * QK + 4 * sub + k;
                const int h = e / dv, c = e - h * dv;
                x[k] = cv[((long long)h * t + j) * dv + c];
            }
            const int e0 = b * QK, h0 = e0 / dv;
            const float x0 = cv[((long long)h0 * t + j) * dv + (e0 - h0 * dv)];
            uint8_t tmp[34];
            uint8_t * o = live ? dst + (size_t)j * drb + (size_t)b * bb : tmp;
            encode_quad(x, x0, type, sub, o);
        }
        return;
    }
    const IT total = (IT)rows * (IT)n;
    for (IT i = (IT)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (IT)gridDim.x * blockDim.x) {
        const IT j = i / (IT)n;
        const int b = (int)(i - j * (IT)n);
        const int h = b / dv, c = b - h * dv;
        const float v = cv[((long long)h * t + j) * dv + c];
        uint8_t * o = dst + j * drb;
        if (type == 1) st16(o + 2 * b, kvc_f2h_trunc(v));
        else memcpy(o + 4 * b, &v, 4);
    }
}

// Encode 8 values (part `part` of 4) of a block held by the 4 lanes of an
// aligned lane group, into the block's bytes at o: the arithmetic of
// encode_quad / encode_block, with the block statistics combined by
// shuffles inside the group (maxima and minima do not depend on order).
template <int TYPE>
__device__ __forceinline__ void encode_oct(const float (&x)[8], float x0, int part, uint8_t * o) {
    auto st = [](uint8_t * q, uint16_t v) { *reinterpret_cast<uint16_t *>(q) = v; };
    if (TYPE == 8 || TYPE == 2) {
        float amax = 0.0f;                               // NaN never wins: skipped as in encode_block
#pragma unroll
        for (int i = 0; i < 8; i++) { const float a = fabsf(x[i]); if (a > amax) amax = a; }
#pragma unroll
        for (int off = 2; off; off >>= 1) {
            const float b = __shfl_xor_sync(0xffffffffu, amax, off, 4);
            if (b > amax) amax = b;
        }
        const float lim = (TYPE == 8) ? 127.0f : 7.0f;
        const float d = kvc_div(amax, lim);
        if (part == 0) st(o, kvc_f2h_trunc(d));
        const float id = (d != 0.0f) ? kvc_div(lim, amax) : 0.0f;
        if (TYPE == 8) {
            uint8_t q[8];
#pragma unroll
            for (int i = 0; i < 8; i++) q[i] = (uint8_t)(int8_t)kvc_roundf(kvc_clamp(kvc_mul(x[i], id), -128.0f, 127.0f));
#pragma unroll
            for (int i = 0; i < 4; i++) st(o + 2 + 8 * part + 2 * i, (uint16_t)(q[2 * i] | (q[2 * i + 1] << 8)));
        } else {
            uint8_t q[8];
#pragma unroll
            for (int i = 0; i < 8; i++) q[i] = (uint8_t)kvc_clamp(kvc_roundf(kvc_add(kvc_mul(x[i], id), 8.0f)), 0.0f, 15.0f);
#pragma unroll
            for (int i = 0; i < 2; i++)
                st(o + 2 + 4 * part + 2 * i,
                   (uint16_t)((q[4 * i] | (q[4 * i + 1] << 4)) | ((q[4 * i + 2] | (q[4 * i + 3] << 4)) << 8)));
        }
    } else {
        float lo = x0, hi = x0;                          // a NaN first value poisons both, as in encode_block
#pragma unroll
        for (int i = 0; i < 8; i++) { if (x[i] < lo) lo = x[i]; if (x[i] > hi) hi = x[i]; }
#pragma unroll
        for (int off = 2; off; off >>= 1) {
            const float a = __shfl_xor_sync(0xffffffffu, lo, off, 4);
            const float b = __shfl_xor_sync(0xffffffffu, hi, off, 4);
            if (a < lo) lo = a;
            if (b > hi) hi = b;
        }
        const float rng = kvc_sub(hi, lo);
        const float d = kvc_div(rng, 15.0f);
        if (part == 0) {
            st(o, kvc_f2h_trunc(d));
            st(o + 2, kvc_f2h_trunc(lo));
        }
        const float id = (d != 0.0f) ? kvc_div(15.0f, rng) : 0.0f;
        uint8_t q[8];
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = (uint8_t)kvc_clamp(kvc_roundf(kvc_mul(kvc_sub(x[i], lo), id)), 0.0f, 15.0f);
#pragma unroll
        for (int i = 0; i < 2; i++)
            st(o + 4 + 4 * part + 2 * i,
               (uint16_t)((q[4 * i] | (q[4 * i + 1] << 4)) | ((q[4 * i + 2] | (q[4 * i + 3] << 4)) << 8)));
    }
}

// Packed block rows out (row bytes = blocks x block bytes, 16-byte aligned
// destination): a CTA encodes 64 blocks at a time, 4 threads a block and 8
// values a thread read as two float4, into shared memory, and writes the
// span's bytes out as 16-byte stores (one thread per 16 bytes) instead of the
// 2-byte stores of k_encode_gather / k_encode_heads. HEADS = 0: block b of
// output row r holds values 32b.. of source row idx[r] (or r); HEADS = 1:
// output row r is row r of every head of cv ([H][t][dv], d_v a multiple of
// 32, so a block lies within one head).
template <int TYPE, int HEADS>
__global__ void __launch_bounds__(256) k_encode_span(const float * __restrict__ src, size_t stride,
                                                     const int * __restrict__ idx, int t, int dv, int nb,
                                                     long long nblocks, uint8_t * __restrict__ dst) {
    constexpr int BB = TYPE == 8 ? 34 : (TYPE == 2 ? 18 : 20);
    constexpr int SPB = 64, SB = SPB * BB, NV = SB / 16;
    static_assert(SB % 16 == 0, "a span is whole 16-byte pieces");
    __shared__ __align__(16) uint8_t sb[SB + BB + 14];   // + a block that lanes past the end write, never read
    const int blk = threadIdx.x >> 2, part = threadIdx.x & 3;
    for (long long sp = blockIdx.x; sp * SPB < nblocks; sp += gridDim.x) {
        const long long b0 = sp * SPB;
        const int nbk = (int)min((long long)SPB, nblocks - b0);
        const bool live = blk < nbk;
        float x[8];
        if (live) {
            const long long gb = b0 + blk, r = gb / nb;
            const int b = (int)(gb - r * nb);
            const float * p;
            if (HEADS) {
                const int e0 = b * QK, h = e0 / dv;
                p = src + ((long long)h * t + r) * dv + (e0 - h * dv) + 8 * part;
            } else {
                p = src + (idx ? (long long)idx[r] : r) * (long long)stride + (long long)b * QK + 8 * part;
            }
            const float4 u0 = *reinterpret_cast<const float4 *>(p), u1 = *reinterpret_cast<const float4 *>(p + 4);
            x[0] = u0.x; x[1] = u0.y; x[2] = u0.z; x[3] = u0.w;
            x[4] = u1.x; x[5] = u1.y; x[6] = u1.z; x[7] = u1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = 0.0f;
        }
        const float x0 = __shfl_sync(0xffffffffu, x[0], threadIdx.x & 28);   // the block's first value
        encode_oct<TYPE>(x, x0, part, sb + (live ? blk * BB : SB));
        __syncthreads();
        const int nbytes = nbk * BB;
        uint8_t * d = dst + b0 * BB;
        if (threadIdx.x < NV) {
            const int o = threadIdx.x * 16;
            if (o + 16 <= nbytes) *reinterpret_cast<uint4 *>(d + o) = *reinterpret_cast<const uint4 *>(sb + o);
            else
                for (int i = o; i < nbytes && i < o + 16; i++) d[i] = sb[i];
        }
        __syncthreads();
    }
}

template <int HEADS>
static void launch_encode_span(int type, const float * src, size_t stride, const int * idx, int t, int dv, int nb,
                               long long nblocks, uint8_t * dst, cudaStream_t st) {
    const int grid = (int)std::min<long long>((nblocks + 63) / 64, 148LL * 32);
    if (type == 8) k_encode_span<8, HEADS><<<grid, 256, 0, st>>>(src, stride, idx, t, dv, nb, nblocks, dst);
    else if (type == 2) k_encode_span<2, HEADS><<<grid, 256, 0, st>>>(src, stride, idx, t, dv, nb, nblocks, dst);
    else k_encode_span<3, HEADS><<<grid, 256, 0, st>>>(src, stride, idx, t, dv, nb, nblocks, dst);
}

int kvc_launch_encode_gather(const float * src, size_t stride, const int * idx, int rows, int n,
                             int type, uint8_t * dst, size_t drb, cudaStream_t st) {
    if (rows <= 0) return KVC_OK;
    if (is_block(type) && n >= QK && n % QK == 0 && drb == (size_t)(n / QK) * (size_t)kvc_block_bytes(type) &&
        stride % 4 == 0 && (((uintptr_t)src) & 15) == 0 && (((uintptr_t)dst) & 15) == 0) {
        launch_encode_span<0>(type, src, stride, idx, 0, 0, n / QK, (long long)rows * (n / QK), dst, st);
        KVC_CUDA(cudaGetLastError());
        return KVC_OK;
    }
    long long work = (long long)rows * (is_block(type) ? (n / QK) * 8 : n);
    if (work + (long long)148 * 64 * 256 + 64 < (1LL << 32))   // the last grid-stride step stays below 2^32
        k_encode_gather<uint32_t><<<grid_for(work, 256), 256, 0, st>>>(src, stride, idx, rows, n, type, dst, drb);
    else
        k_encode_gather<unsigned long long><<<grid_for(work, 256), 256, 0, st>>>(src, stride, idx, rows, n, type, dst,
                                                                              drb);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

int kvc_launch_encode_heads(const float * cv, int H, int t, int rows, int dv, int type, uint8_t * dst,
                            size_t drb, cudaStream_t st) {
    if (rows <= 0) return KVC_OK;
    if (is_block(type) && dv % QK == 0 && drb == (size_t)((H * dv) / QK) * (size_t)kvc_block_bytes(type) &&
        (((uintptr_t)cv) & 15) == 0 && (((uintptr_t)dst) & 15) == 0) {
        launch_encode_span<1>(type, cv, 0, nullptr, t, dv, (H * dv) / QK, (long long)rows * ((H * dv) / QK), dst, st);
        KVC_CUDA(cudaGetLastError());
        return KVC_OK;
    }
    long long work = (long long)rows * (is_block(type) ? ((H * dv) / QK) * 8 : H * dv);
    if (work + (long long)148 * 64 * 256 + 64 < (1LL << 32))   // the last grid-stride step stays below 2^32
        k_encode_heads<uint32_t><<<grid_for(work, 256), 256, 0, st>>>(cv, H, t, rows, dv, type, dst, drb);
    else
        k_encode_heads<unsigned long long><<<grid_for(work, 256), 256, 0, st>>>(cv, H, t, rows, dv, type, dst, drb);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

// Rows re-encoded straight from their stored bytes: output row r =
// encode(decode(source row idx[r])) block by block with decode_block /
// encode_block, the same arithmetic the decode and encode kernels use, so the
// bytes equal those of decoding every row to fp32 first and re-encoding the
// kept ones. One thread per 32-value block (a warp covers consecutive blocks
// of a row: contiguous bytes in and out); F16 / F32 rows per value.
__global__ void __launch_bounds__(256) k_transcode_gather(const uint8_t * __restrict__ src, size_t srb,
                                                          const int * __restrict__ idx, int rows, int nb, int type,
                                                          uint8_t * __restrict__ dst, size_t drb) {
    const long long total = (long long)rows * nb;
    const int bb = type == 8 ? 34 : (type == 2 ? 18 : (type == 3 ? 20 : (type == 1 ? 2 : 4)));
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / nb;
        const int b = (int)(i - r * nb);
        const uint8_t * s = src + (size_t)idx[r] * srb + (size_t)b * bb;
        uint8_t * o = dst + (size_t)r * drb + (size_t)b * bb;
        if (type == 1) {
            st16(o, kvc_f2h_trunc(kvc_h2f(ld16(s))));
        } else if (type == 0) {
            o[0] = s[0]; o[1] = s[1]; o[2] = s[2]; o[3] = s[3];
        } else {
            float x[QK];
            decode_block(s, type, x);
            encode_block(x, type, o);
        }
    }
}

// The same for block formats with 16-byte multiple rows: one warp per output
// row. The source row's bytes come into shared memory by 16-byte loads, each
// lane re-encodes whole blocks there (decode_block / encode_block over
// shared memory), and the row goes out by 16-byte stores.
constexpr int TR_WARPS = 8, TR_MAX_RB = 2176;        // rows up to 2,176 bytes (e.g. 64 Q8_0 blocks)
template <int TYPE>
__global__ void __launch_bounds__(TR_WARPS * 32) k_transcode_rows(const uint8_t * __restrict__ src, size_t rb,
                                                                  const int * __restrict__ idx, int rows, int nb,
                                                                  uint8_t * __restrict__ dst) {
    constexpr int BB = TYPE == 8 ? 34 : (TYPE == 2 ? 18 : 20);
    __shared__ __align__(16) uint8_t sin[TR_WARPS][TR_MAX_RB], sout[TR_WARPS][TR_MAX_RB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = (int)(rb / 16);
    for (long long r = (long long)blockIdx.x * TR_WARPS + warp; r < rows; r += (long long)gridDim.x * TR_WARPS) {
        const uint4 * s = reinterpret_cast<const uint4 *>(src + (size_t)idx[r] * rb);
        for (int i = lane; i < nv; i += 32) reinterpret_cast<uint4 *>(sin[warp])[i] = s[i];
        __syncwarp();
        for (int b = lane; b < nb; b += 32) {
            float x[QK];
            decode_block(sin[warp] + b * BB, TYPE, x);
            encode_block(x, TYPE, sout[warp] + b * BB);
        }
        __syncwarp();
        uint4 * o = reinterpret_cast<uint4 *>(dst + (size_t)r * rb);
        for (int i = lane; i < nv; i += 32) o[i] = reinterpret_cast<const uint4 *>(sout[warp])[i];
        __syncwarp();
    }
}

// Every layer of a call in one launch (the per-layer launches of a whole
// model are 10-30 us each and spend part of that in their tail): a table of
// up to KVC_RQ_MAX_LAYERS layers, passed by value, with the first work item
// of each layer (rows for the transcode, 64-block spans for the encode);
// each work item is done exactly as by the per-layer kernels.
struct kvc_rq_batch {
    int n;
    long long start[KVC_RQ_MAX_LAYERS + 1];
    const void * src[KVC_RQ_MAX_LAYERS];
    const int * idx[KVC_RQ_MAX_LAYERS];
    uint8_t * dst[KVC_RQ_MAX_LAYERS];
    int t[KVC_RQ_MAX_LAYERS];
};

template <int TYPE>
__global__ void __launch_bounds__(TR_WARPS * 32) k_transcode_rows_batch(const __grid_constant__ kvc_rq_batch B,
                                                                        size_t rb, int nb) {
    constexpr int BB = TYPE == 8 ? 34 : (TYPE == 2 ? 18 : 20);
    __shared__ __align__(16) uint8_t sin[TR_WARPS][TR_MAX_RB], sout[TR_WARPS][TR_MAX_RB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = (int)(rb / 16);
    int l = 0;
    for (long long g = (long long)blockIdx.x * TR_WARPS + warp; g < B.start[B.n]; g += (long long)gridDim.x * TR_WARPS) {
        while (g >= B.start[l + 1]) l++;           // rows only increase along the loop
        const long long r = g - B.start[l];
        const uint4 * s = reinterpret_cast<const uint4 *>((const uint8_t *)B.src[l] + (size_t)B.idx[l][r] * rb);
        for (int i = lane; i < nv; i += 32) reinterpret_cast<uint4 *>(sin[warp])[i] = s[i];
        __syncwarp();
        for (int b = lane; b < nb; b += 32) {
            float x[QK];
            decode_block(sin[warp] + b * BB, TYPE, x);
            encode_block(x, TYPE, sout[warp] + b * BB);
        }
        __syncwarp();
        uint4 * o = reinterpret_cast<uint4 *>(B.dst[l] + (size_t)r * rb);
        for (int i = lane; i < nv; i += 32) o[i] = reinterpret_cast<const uint4 *>(sout[warp])[i];
        __syncwarp();
    }
}

// k_encode_span<TYPE, 1> over every layer: span sp of layer l covers blocks
// 64 (sp - start[l]) .. of that layer's t rows x nb blocks.
template <int TYPE>
__global__ void __launch_bounds__(256) k_encode_heads_batch(const __grid_constant__ kvc_rq_batch B, int dv, int nb) {
    constexpr int BB = TYPE == 8 ? 34 : (TYPE == 2 ? 18 : 20);
    constexpr int SPB = 64, SB = SPB * BB, NV = SB / 16;
    __shared__ __align__(16) uint8_t sb[SB + BB + 14];
    const int blk = threadIdx.x >> 2, part = threadIdx.x & 3;
    int l = 0;
    for (long long sp = blockIdx.x; sp < B.start[B.n]; sp += gridDim.x) {
        while (sp >= B.start[l + 1]) l++;
        const int t = B.t[l];
        const long long nblocks = (long long)t * nb;
        const long long b0 = (sp - B.start[l]) * SPB;
        const int nbk = (int)min((long long)SPB, nblocks - b0);
        const bool live = blk < nbk;
        float x[8];
        if (live) {
            const long long gb = b0 + blk, r = gb / nb;
            const int b = (int)(gb - r * nb);
            const int e0 = b * QK, h = e0 / dv;
            const float * p = (const float *)B.src[l] + ((long long)h * t + r) * dv + (e0 - h * dv) + 8 * part;
            const float4 u0 = *reinterpret_cast<const float4 *>(p), u1 = *reinterpret_cast<const float4 *>(p + 4);
            x[0] = u0.x; x[1] = u0.y; x[2] = u0.z; x[3] = u0.w;
            x[4] = u1.x; x[5] = u1.y; x[6] = u1.z; x[7] = u1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = 0.0f;
        }
        const float x0 = __shfl_sync(0xffffffffu, x[0], threadIdx.x & 28);
        encode_oct<TYPE>(x, x0, part, sb + (live ? blk * BB : SB));
        __syncthreads();
        const int nbytes = nbk * BB;
        uint8_t * d = B.dst[l] + b0 * BB;
        if (threadIdx.x < NV) {
            const int o = threadIdx.x * 16;
            if (o + 16 <= nbytes) *reinterpret_cast<uint4 *>(d + o) = *reinterpret_cast<const uint4 *>(sb + o);
            else
                for (int i = o; i < nbytes && i < o + 16; i++) d[i] = sb[i];
        }
        __syncthreads();
    }
}

int kvc_launch_requant_batch(int n, const uint8_t * const * k_src, const int * const * sel, const int * t,
                             uint8_t * const * k_dst, size_t k_rb, int ek, int k_type, const float * const * cv,
                             uint8_t * const * v_dst, size_t v_rb, int H, int dv, int v_type, cudaStream_t st) {
    if (n <= 0) return KVC_OK;
    if (n > KVC_RQ_MAX_LAYERS) return KVC_ERR_SHAPE;
    const bool k_on = k_dst != nullptr, v_on = v_dst != nullptr;
    if (k_on && !(is_block(k_type) && k_rb % 16 == 0 && k_rb <= (size_t)TR_MAX_RB &&
                  k_rb == (size_t)(ek / QK) * (size_t)kvc_block_bytes(k_type)))
        return KVC_ERR_SHAPE;
    if (v_on && !(is_block(v_type) && dv % QK == 0 && v_rb == (size_t)((H * dv) / QK) * (size_t)kvc_block_bytes(v_type)))
        return KVC_ERR_SHAPE;
    for (int i = 0; i < n; i++) {
        if (k_on && ((((uintptr_t)k_src[i]) | ((uintptr_t)k_dst[i])) & 15)) return KVC_ERR_SHAPE;
        if (v_on && ((((uintptr_t)cv[i]) | ((uintptr_t)v_dst[i])) & 15)) return KVC_ERR_SHAPE;
    }
    if (k_on) {
        kvc_rq_batch B{};
        B.n = n;
        for (int i = 0; i < n; i++) {
            B.start[i + 1] = B.start[i] + t[i];
            B.src[i] = k_src[i];
            B.idx[i] = sel[i];
            B.dst[i] = k_dst[i];
            B.t[i] = t[i];
        }
        const int grid = (int)std::min<long long>((B.start[n] + TR_WARPS - 1) / TR_WARPS, 148LL * 8);
        if (grid > 0) {
            if (k_type == 8) k_transcode_rows_batch<8><<<grid, TR_WARPS * 32, 0, st>>>(B, k_rb, ek / QK);
            else if (k_type == 2) k_transcode_rows_batch<2><<<grid, TR_WARPS * 32, 0, st>>>(B, k_rb, ek / QK);
            else k_transcode_rows_batch<3><<<grid, TR_WARPS * 32, 0, st>>>(B, k_rb, ek / QK);
            KVC_CUDA(cudaGetLastError());
        }
    }
    if (v_on) {
        const int nb = (H * dv) / QK;
        kvc_rq_batch B{};
        B.n = n;
        for (int i = 0; i < n; i++) {
            B.start[i + 1] = B.start[i] + ((long long)t[i] * nb + 63) / 64;
            B.src[i] = cv[i];
            B.idx[i] = nullptr;
            B.dst[i] = v_dst[i];
            B.t[i] = t[i];
        }
        const int grid = (int)std::min<long long>(B.start[n], 148LL * 32);
        if (grid > 0) {
            if (v_type == 8) k_encode_heads_batch<8><<<grid, 256, 0, st>>>(B, dv, nb);
            else if (v_type == 2) k_encode_heads_batch<2><<<grid, 256, 0, st>>>(B, dv, nb);
            else k_encode_heads_batch<3><<<grid, 256, 0, st>>>(B, dv, nb);
            KVC_CUDA(cudaGetLastError());
        }
    }
    return KVC_OK;
}

int kvc_launch_transcode_gather(const uint8_t * src, size_t src_rb, const int * idx, int rows, int n, int type,
                                uint8_t * dst, size_t dst_rb, cudaStream_t st) {
    if (rows <= 0) return KVC_OK;
    if (is_block(type) && src_rb == dst_rb && src_rb % 16 == 0 && src_rb <= (size_t)TR_MAX_RB &&
        src_rb == (size_t)(n / QK) * (size_t)kvc_block_bytes(type) && (((uintptr_t)src) & 15) == 0 &&
        (((uintptr_t)dst) & 15) == 0) {
        const int grid = (int)std::min<long long>(((long long)rows + TR_WARPS - 1) / TR_WARPS, 148LL * 8);
        if (type == 8) k_transcode_rows<8><<<grid, TR_WARPS * 32, 0, st>>>(src, src_rb, idx, rows, n / QK, dst);
        else if (type == 2) k_transcode_rows<2><<<grid, TR_WARPS * 32, 0, st>>>(src, src_rb, idx, rows, n / QK, dst);
        else k_transcode_rows<3><<<grid, TR_WARPS * 32, 0, st>>>(src, src_rb, idx, rows, n / QK, dst);
        KVC_CUDA(cudaGetLastError());
        return KVC_OK;
    }
    const int nb = is_block(type) ? n / QK : n;
    const long long work = (long long)rows * nb;
    const int grid = (int)std::min<long long>((work + 255) / 256, 148LL * 16);
    k_transcode_gather<<<grid, 256, 0, st>>>(src, src_rb, idx, rows, nb, type, dst, dst_rb);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}
