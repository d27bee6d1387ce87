/*
 * kvc_oracle.c — CPU restatement of the kv-compact compaction path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * library: tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may load it; the product (libkvc.so) never does.
 *
 * It restates, in plain C, the algorithm of fabiantax/kv-compact's Linux CPU
 * path (OpenMP + Gaussian elimination; that path has no BLAS on Linux). Each
 * function cites the reference file:line it follows. The floating-point
 * operations are kept in the reference's order (sequential fp32 sums, no
 * fused multiply-add: gcc for x86-64 without -march emits none, and the
 * Makefile passes -ffp-contract=off), so for the same inputs this file and
 * the reference compiled here produce bit-identical outputs. That claim is
 * pinned by tests/test_oracle_golden.py against fixtures that
 * tests/golden/make_golden.py generates by running the reference itself.
 *
 * Exported names carry an "oracle_" prefix so this library and the product
 * can be loaded into one process.
 */
#define _POSIX_C_SOURCE 199309L
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../include/kv-compact-api.h"

#define QK 32

/* ========================================================================
 * Codecs — reference include/kv-compact-state.h:326-629
 * ====================================================================== */

/* IEEE half -> float, exact (state.h:465-500). */
static float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            /* subnormal half: normalise the mantissa */
            int32_t ee = 1;
            while (!(m & 0x400u)) { m <<= 1; ee--; }
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(ee + 112) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> half by mantissa truncation (state.h:508-525): no rounding,
 * exponent below -10 flushes to signed zero, overflow (and NaN) to inf. */
static uint16_t orc_f32_to_f16(float v) {
    uint32_t f;
    memcpy(&f, &v, 4);
    uint32_t sign = (f >> 16) & 0x8000u;
    int32_t e = (int32_t)((f >> 23) & 0xFFu) - 112;
    uint32_t m = (f >> 13) & 0x3FFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        return (uint16_t)(sign | ((m | 0x400u) >> (1 - e)));
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | m);
}

static int orc_block_bytes(int type) {           /* state.h:326-333 */
    switch (type) {
    case KV_TYPE_F32: return 4;
    case KV_TYPE_F16: return 2;
    case KV_TYPE_Q8_0: return 34;
    case KV_TYPE_Q4_0: return 18;
    case KV_TYPE_Q4_1: return 20;
    default: return 4;
    }
}

static int orc_is_block_type(int type) {
    return type == KV_TYPE_Q8_0 || type == KV_TYPE_Q4_0 || type == KV_TYPE_Q4_1;
}

int oracle_quant_row_elements(int type, size_t row_bytes) {   /* state.h:343-352 */
    if (type == KV_TYPE_F32) return (int)(row_bytes / 4);
    if (type == KV_TYPE_F16) return (int)(row_bytes / 2);
    if (orc_is_block_type(type)) return (int)(row_bytes / (size_t)orc_block_bytes(type)) * QK;
    return (int)(row_bytes / 4);
}

size_t oracle_quant_row_bytes(int type, int n) {              /* api.cpp:1159-1167 */
    if (type == KV_TYPE_F32) return (size_t)n * 4;
    if (type == KV_TYPE_F16) return (size_t)n * 2;
    if (orc_is_block_type(type)) return (size_t)(n / QK) * (size_t)orc_block_bytes(type);
    return (size_t)n * 4;
}

/* Decode n values of one row (state.h:355-421). */
static void orc_decode_row(const uint8_t * src, int type, float * dst, size_t n) {
    if (type == KV_TYPE_F32) { memcpy(dst, src, n * 4); return; }
    if (type == KV_TYPE_F16) {
        for (size_t i = 0; i < n; i++) {
            uint16_t h; memcpy(&h, src + 2 * i, 2);
            dst[i] = orc_f16_to_f32(h);
        }
        return;
    }
    if (!orc_is_block_type(type)) { memset(dst, 0, n * 4); return; }
    size_t nb = n / QK, bb = (size_t)orc_block_bytes(type);
    for (size_t b = 0; b < nb; b++) {
        const uint8_t * blk = src + b * bb;
        float * o = dst + b * QK;
        uint16_t dh; memcpy(&dh, blk, 2);
        float d = orc_f16_to_f32(dh);
        if (type == KV_TYPE_Q8_0) {
            const int8_t * q = (const int8_t *)(blk + 2);
            for (int i = 0; i < QK; i++) o[i] = d * (float)q[i];
        } else if (type == KV_TYPE_Q4_0) {
            const uint8_t * q = blk + 2;
            for (int i = 0; i < QK / 2; i++) {
                o[2 * i]     = d * ((float)(q[i] & 0xF) - 8.0f);
                o[2 * i + 1] = d * ((float)(q[i] >> 4) - 8.0f);
            }
        } else {
            uint16_t mh; memcpy(&mh, blk + 2, 2);
            float m = orc_f16_to_f32(mh);
            const uint8_t * q = blk + 4;
            for (int i = 0; i < QK / 2; i++) {
                o[2 * i]     = d * (float)(q[i] & 0xF) + m;
                o[2 * i + 1] = d * (float)(q[i] >> 4) + m;
            }
        }
    }
}

/* max(lo, min(hi, v)) with the operand order of std::min/std::max, so a NaN
 * v maps to hi exactly as at state.h:543,563-564,588-589. */
static float orc_clampf(float v, float lo, float hi) {
    float m = (v < hi) ? v : hi;
    return (lo < m) ? m : lo;
}

/* Encode one row (state.h:528-629). Returns bytes written. */
static size_t orc_encode_row(const float * src, int type, uint8_t * dst, int n) {
    if (type == KV_TYPE_F32) { memcpy(dst, src, (size_t)n * 4); return (size_t)n * 4; }
    if (type == KV_TYPE_F16) {
        for (int i = 0; i < n; i++) {
            uint16_t h = orc_f32_to_f16(src[i]);
            memcpy(dst + 2 * i, &h, 2);
        }
        return (size_t)n * 2;
    }
    if (!orc_is_block_type(type)) return 0;
    int nb = n / QK, bb = orc_block_bytes(type);
    for (int b = 0; b < nb; b++) {
        const float * x = src + b * QK;
        uint8_t * o = dst + (size_t)b * bb;
        if (type == KV_TYPE_Q8_0) {                           /* state.h:528-545 */
            float amax = 0.0f;
            for (int i = 0; i < QK; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
            float d = amax / 127.0f;
            uint16_t dh = orc_f32_to_f16(d);
            memcpy(o, &dh, 2);
            float id = (d != 0.0f) ? 127.0f / amax : 0.0f;
            for (int i = 0; i < QK; i++)
                ((int8_t *)(o + 2))[i] = (int8_t)roundf(orc_clampf(x[i] * id, -128.0f, 127.0f));
        } else if (type == KV_TYPE_Q4_0) {                    /* state.h:548-567 */
            float amax = 0.0f;
            for (int i = 0; i < QK; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
            float d = amax / 7.0f;
            uint16_t dh = orc_f32_to_f16(d);
            memcpy(o, &dh, 2);
            float id = (d != 0.0f) ? 7.0f / amax : 0.0f;
            for (int i = 0; i < QK / 2; i++) {
                float v0 = x[2 * i] * id + 8.0f, v1 = x[2 * i + 1] * id + 8.0f;
                uint8_t q0 = (uint8_t)orc_clampf(roundf(v0), 0.0f, 15.0f);
                uint8_t q1 = (uint8_t)orc_clampf(roundf(v1), 0.0f, 15.0f);
                o[2 + i] = (uint8_t)(q0 | (q1 << 4));
            }
        } else {                                              /* state.h:570-592 */
            float lo = x[0], hi = x[0];
            for (int i = 1; i < QK; i++) { if (x[i] < lo) lo = x[i]; if (x[i] > hi) hi = x[i]; }
            float d = (hi - lo) / 15.0f;
            uint16_t dh = orc_f32_to_f16(d), mh = orc_f32_to_f16(lo);
            memcpy(o, &dh, 2);
            memcpy(o + 2, &mh, 2);
            float id = (d != 0.0f) ? 15.0f / (hi - lo) : 0.0f;
            for (int i = 0; i < QK / 2; i++) {
                float v0 = (x[2 * i] - lo) * id, v1 = (x[2 * i + 1] - lo) * id;
                uint8_t q0 = (uint8_t)orc_clampf(roundf(v0), 0.0f, 15.0f);
                uint8_t q1 = (uint8_t)orc_clampf(roundf(v1), 0.0f, 15.0f);
                o[4 + i] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
    return (size_t)nb * (size_t)bb;
}

int oracle_dequantize_row(const uint8_t * src, int type, size_t row_bytes, float * dst, int max_el) {
    int n = oracle_quant_row_elements(type, row_bytes);         /* api.cpp:1169-1175 */
    if (n > max_el) n = max_el;
    orc_decode_row(src, type, dst, (size_t)n);
    return n;
}

size_t oracle_quantize_row(const float * src, int type, int n, uint8_t * dst) {
    return orc_encode_row(src, type, dst, n);                   /* api.cpp:1177-1180 */
}

/* ========================================================================
 * Dense kernels — reference include/kv-compact-math.h
 * ====================================================================== */

/* Row softmax with max shift and 1/(sum+1e-12) (math.h:83-100). */
static void orc_softmax_rows(float * a, int m, int n) {
    for (int i = 0; i < m; i++) {
        float * r = a + (size_t)i * n;
        float mx = r[0];
        for (int j = 1; j < n; j++) if (r[j] > mx) mx = r[j];
        float s = 0.0f;
        for (int j = 0; j < n; j++) { r[j] = expf(r[j] - mx); s += r[j]; }
        float inv = 1.0f / (s + 1e-12f);
        for (int j = 0; j < n; j++) r[j] *= inv;
    }
}

/* Row softmax plus per-column importance (math.h:142-248). exp_out/row_sums
 * may be NULL. agg: 0 max, 1 rms, 2 mean over rows. */
static void orc_softmax_importance(const float * s, float * exp_out, float * row_sums,
                                   float * sm_out, float * imp, int m, int n, int agg) {
    memset(imp, 0, (size_t)n * 4);
    for (int i = 0; i < m; i++) {
        const float * r = s + (size_t)i * n;
        float * sm = sm_out + (size_t)i * n;
        float mx = r[0];
        for (int j = 1; j < n; j++) if (r[j] > mx) mx = r[j];
        float sum = 0.0f;
        for (int j = 0; j < n; j++) {
            float e = expf(r[j] - mx);
            sm[j] = e;
            if (exp_out) exp_out[(size_t)i * n + j] = e;
            sum += e;
        }
        if (row_sums) row_sums[i] = sum;
        float inv = 1.0f / (sum + 1e-12f);
        for (int j = 0; j < n; j++) {
            float w = sm[j] * inv;
            sm[j] = w;
            if (agg == 0) { if (w > imp[j]) imp[j] = w; }
            else if (agg == 1) imp[j] += w * w;
            else imp[j] += w;
        }
    }
    if (agg == 1) {
        float inv_m = 1.0f / (float)m;
        for (int j = 0; j < n; j++) imp[j] = sqrtf(imp[j] * inv_m);
    } else if (agg == 2) {
        float inv_m = 1.0f / (float)m;
        for (int j = 0; j < n; j++) imp[j] *= inv_m;
    }
}

/* In-place Gaussian elimination with partial pivoting on an augmented
 * [n x (n+p)] system, the shared core of math.h:359-397, 494-557, 717-744.
 * Pivots with |pivot| < 1e-12 are skipped; on back substitution their
 * unknowns are set to `skip_value`. x is [n x p]. */
static void orc_gauss_solve(float * aug, int n, int p, float * x, float skip_value) {
    int w = n + p;
    for (int c = 0; c < n; c++) {
        int pr = c;
        float best = fabsf(aug[(size_t)c * w + c]);
        for (int r = c + 1; r < n; r++) {
            float v = fabsf(aug[(size_t)r * w + c]);
            if (v > best) { best = v; pr = r; }
        }
        if (pr != c)
            for (int j = 0; j < w; j++) {
                float t = aug[(size_t)c * w + j];
                aug[(size_t)c * w + j] = aug[(size_t)pr * w + j];
                aug[(size_t)pr * w + j] = t;
            }
        float piv = aug[(size_t)c * w + c];
        if (fabsf(piv) < 1e-12f) continue;
        for (int r = c + 1; r < n; r++) {
            float f = aug[(size_t)r * w + c] / piv;
            for (int j = c; j < w; j++) aug[(size_t)r * w + j] -= f * aug[(size_t)c * w + j];
        }
    }
    for (int c = n - 1; c >= 0; c--) {
        float piv = aug[(size_t)c * w + c];
        if (fabsf(piv) < 1e-12f) {
            for (int j = 0; j < p; j++) x[(size_t)c * p + j] = skip_value;
            continue;
        }
        for (int j = 0; j < p; j++) {
            float v = aug[(size_t)c * w + n + j];
            for (int r = c + 1; r < n; r++) v -= aug[(size_t)c * w + r] * x[(size_t)r * p + j];
            x[(size_t)c * p + j] = v / piv;
        }
    }
}

/* AtA (n x n) and Atb (n x p) with sequential sums over m (math.h:288-304). */
static void orc_normal_eq(const float * A, const float * b, int m, int n, int p,
                          float * AtA, float * Atb) {
    for (int i = 0; i < n; i++)
        for (int j = 0; j < n; j++) {
            float s = 0.0f;
            for (int k = 0; k < m; k++) s += A[(size_t)k * n + i] * A[(size_t)k * n + j];
            AtA[(size_t)i * n + j] = s;
        }
    for (int i = 0; i < n; i++)
        for (int l = 0; l < p; l++) {
            float s = 0.0f;
            for (int k = 0; k < m; k++) s += A[(size_t)k * n + i] * b[(size_t)k * p + l];
            Atb[(size_t)i * p + l] = s;
        }
}

/* Ridge least squares by normal equations + GE (math.h:463-557).
 * A [m x n], b [m x p] -> x [n x p]. */
void oracle_least_squares(const float * A, const float * b, float * x,
                          int m, int n, int p, float ridge) {
    float * AtA = (float *)malloc((size_t)n * n * 4);
    float * Atb = (float *)malloc((size_t)n * p * 4);
    float * aug = (float *)malloc((size_t)n * (n + p) * 4);
    orc_normal_eq(A, b, m, n, p, AtA, Atb);
    for (int i = 0; i < n; i++) AtA[(size_t)i * n + i] += ridge;
    for (int i = 0; i < n; i++) {
        memcpy(aug + (size_t)i * (n + p), AtA + (size_t)i * n, (size_t)n * 4);
        memcpy(aug + (size_t)i * (n + p) + n, Atb + (size_t)i * p, (size_t)p * 4);
    }
    orc_gauss_solve(aug, n, p, x, 0.0f);
    free(AtA); free(Atb); free(aug);
}

/* Lawson-Hanson NNLS, min ||A w - b||, w >= 0 (math.h:283-452).
 * A [m x n], b [m]. Returns the number of outer iterations taken. */
int oracle_nnls_lh(const float * A, const float * b, float * w, int m, int n, int max_iter) {
    float * AtA = (float *)malloc((size_t)n * n * 4);
    float * Atb = (float *)malloc((size_t)n * 4);
    float * grad = (float *)malloc((size_t)n * 4);
    float * s = (float *)calloc((size_t)n, 4);
    float * aug = (float *)malloc((size_t)n * (n + 1) * 4);
    float * sP = (float *)malloc((size_t)n * 4);
    int * P = (int *)malloc((size_t)n * sizeof(int));
    unsigned char * inP = (unsigned char *)calloc((size_t)n, 1);
    int outer_done = 0;

    orc_normal_eq(A, b, m, n, 1, AtA, Atb);
    for (int i = 0; i < n; i++) { w[i] = 0.0f; grad[i] = -Atb[i]; }

    for (int outer = 0; outer < max_iter; outer++) {
        int ti = -1;
        float best = 0.0f;
        for (int i = 0; i < n; i++)
            if (!inP[i] && (-grad[i]) > best) { best = -grad[i]; ti = i; }
        if (ti < 0 || best < 1e-10f) break;
        outer_done = outer + 1;
        inP[ti] = 1;

        for (int inner = 0; inner < max_iter; inner++) {
            int np = 0;
            for (int i = 0; i < n; i++) if (inP[i]) P[np++] = i;
            int wd = np + 1;
            for (int i = 0; i < np; i++) {
                for (int j = 0; j < np; j++) aug[(size_t)i * wd + j] = AtA[(size_t)P[i] * n + P[j]];
                aug[(size_t)i * wd + i] += 1e-10f;
                aug[(size_t)i * wd + np] = Atb[P[i]];
            }
            orc_gauss_solve(aug, np, 1, sP, 0.0f);
            for (int i = 0; i < n; i++) s[i] = 0.0f;
            for (int i = 0; i < np; i++) s[P[i]] = sP[i];

            int feasible = 1;
            for (int i = 0; i < np; i++) if (sP[i] <= 0.0f) { feasible = 0; break; }
            if (feasible) { for (int i = 0; i < n; i++) w[i] = s[i]; break; }

            float alpha = 1.0f;
            for (int i = 0; i < np; i++) {
                int k = P[i];
                if (s[k] <= 0.0f) {
                    float a = w[k] / (w[k] - s[k] + 1e-30f);
                    if (a < alpha) alpha = a;
                }
            }
            for (int i = 0; i < n; i++) w[i] += alpha * (s[i] - w[i]);
            for (int i = 0; i < np; i++) {
                int k = P[i];
                if (fabsf(w[k]) < 1e-12f) { w[k] = 0.0f; inP[k] = 0; }
            }
        }
        for (int i = 0; i < n; i++) {
            float acc = 0.0f;
            for (int j = 0; j < n; j++) acc += AtA[(size_t)i * n + j] * w[j];
            grad[i] = acc - Atb[i];
        }
    }
    for (int i = 0; i < n; i++) if (w[i] < 1e-12f) w[i] = 1e-12f;
    free(AtA); free(Atb); free(grad); free(s); free(aug); free(sP); free(P); free(inP);
    return outer_done;
}

/* Clamped least squares + optional projected gradient (math.h:683-806). */
void oracle_nnls_pgd(const float * A, const float * b, float * w, int m, int n,
                     float eps, int iters) {
    float * AtA = (float *)malloc((size_t)n * n * 4);
    float * Atb = (float *)malloc((size_t)n * 4);
    float * aug = (float *)malloc((size_t)n * (n + 1) * 4);
    orc_normal_eq(A, b, m, n, 1, AtA, Atb);
    for (int i = 0; i < n; i++) {
        memcpy(aug + (size_t)i * (n + 1), AtA + (size_t)i * n, (size_t)n * 4);
        aug[(size_t)i * (n + 1) + i] += 1e-10f;
        aug[(size_t)i * (n + 1) + n] = Atb[i];
    }
    orc_gauss_solve(aug, n, 1, w, eps);
    for (int i = 0; i < n; i++) if (w[i] < eps) w[i] = eps;
    if (iters > 0) {
        float * u = (float *)malloc((size_t)n * 4);
        float * v = (float *)malloc((size_t)m * 4);
        float * g = (float *)malloc((size_t)n * 4);
        for (int i = 0; i < n; i++) u[i] = 1.0f / sqrtf((float)n);
        for (int pw = 0; pw < 3; pw++) {
            for (int i = 0; i < m; i++) {
                float acc = 0.0f;
                for (int j = 0; j < n; j++) acc += A[(size_t)i * n + j] * u[j];
                v[i] = acc;
            }
            float vn = 0.0f;
            for (int i = 0; i < m; i++) vn += v[i] * v[i];
            vn = sqrtf(vn);
            if (vn < 1e-12f) break;
            for (int i = 0; i < m; i++) v[i] /= vn;
            for (int j = 0; j < n; j++) {
                float acc = 0.0f;
                for (int i = 0; i < m; i++) acc += A[(size_t)i * n + j] * v[i];
                u[j] = acc;
            }
            float un = 0.0f;
            for (int j = 0; j < n; j++) un += u[j] * u[j];
            un = sqrtf(un);
            if (un < 1e-12f) break;
            for (int j = 0; j < n; j++) u[j] /= un;
        }
        float L = 0.0f;
        for (int i = 0; i < n; i++) {
            float acc = 0.0f;
            for (int j = 0; j < n; j++) acc += AtA[(size_t)i * n + j] * u[j];
            L += u[i] * acc;
        }
        if (L < 1e-6f) L = 1e-6f;
        float eta = 1.0f / L;
        for (int it = 0; it < iters; it++) {
            for (int i = 0; i < n; i++) {
                float acc = 0.0f;
                for (int j = 0; j < n; j++) acc += AtA[(size_t)i * n + j] * w[j];
                g[i] = acc - Atb[i];
            }
            for (int i = 0; i < n; i++) { w[i] -= eta * g[i]; if (w[i] < eps) w[i] = eps; }
        }
        free(u); free(v); free(g);
    }
    free(AtA); free(Atb); free(aug);
}

/* Orthogonal matching pursuit on attention mass (math.h:832-950). */
static void orc_omp_select(const float * E, const float * rs, int T, int nq, int t,
                           int * sel, float * w_out, int kc, int refit, int pgd_iters) {
    unsigned char * mask = (unsigned char *)calloc((size_t)T, 1);
    float * cur = (float *)calloc((size_t)nq, 4);
    float * res = (float *)malloc((size_t)nq * 4);
    float * corr = (float *)malloc((size_t)T * 4);
    int * order = (int *)malloc((size_t)(t > 0 ? t : 1) * sizeof(int));
    float * prev = (float *)malloc((size_t)(t > 0 ? t : 1) * 4);
    float * M = (float *)malloc((size_t)nq * (t > 0 ? t : 1) * 4);
    float * w = (float *)malloc((size_t)(t > 0 ? t : 1) * 4);
    int nsel = 0, nprev = 0, iter = 0;

    while (nsel < t) {
        for (int i = 0; i < nq; i++) res[i] = rs[i] - cur[i];
        for (int j = 0; j < T; j++) {
            corr[j] = 0.0f;
            if (mask[j]) continue;
            float c = 0.0f;
            for (int i = 0; i < nq; i++) c += E[(size_t)i * T + j] * res[i];
            corr[j] = c;
        }
        int k_sel = kc < t - nsel ? kc : t - nsel;
        if (k_sel > T - nsel) k_sel = T - nsel;
        if (k_sel <= 0) break;
        for (int k = 0; k < k_sel; k++) {
            int best = -1;
            float bc = -1e30f;
            for (int j = 0; j < T; j++) {
                if (mask[j]) continue;
                if (corr[j] > bc) { bc = corr[j]; best = j; }
            }
            if (best < 0) break;
            order[nsel++] = best;
            mask[best] = 1;
            corr[best] = -1e30f;
        }
        int ct = nsel;
        int solve = (refit <= 1) || (iter % refit == 0) || (ct == t);
        if (solve) {
            for (int i = 0; i < nq; i++)
                for (int j = 0; j < ct; j++) M[(size_t)i * ct + j] = E[(size_t)i * T + order[j]];
            oracle_nnls_pgd(M, rs, w, nq, ct, 1e-12f, pgd_iters);
            memcpy(prev, w, (size_t)ct * 4);
            nprev = ct;
            for (int i = 0; i < nq; i++) {
                float acc = 0.0f;
                for (int j = 0; j < ct; j++) acc += M[(size_t)i * ct + j] * w[j];
                cur[i] = acc;
            }
        } else {
            for (int j = nprev; j < ct; j++) prev[j] = 1e-12f;
            nprev = ct;
            for (int i = 0; i < nq; i++) {
                float acc = 0.0f;
                for (int j = 0; j < ct; j++) acc += E[(size_t)i * T + order[j]] * prev[j];
                cur[i] = acc;
            }
        }
        iter++;
    }
    /* ascending by position, weights follow (indices are distinct) */
    for (int a = 1; a < nsel; a++) {
        int key = order[a]; float wv = prev[a]; int b = a - 1;
        while (b >= 0 && order[b] > key) { order[b + 1] = order[b]; prev[b + 1] = prev[b]; b--; }
        order[b + 1] = key; prev[b + 1] = wv;
    }
    for (int j = 0; j < nsel; j++) { sel[j] = order[j]; w_out[j] = j < nprev ? prev[j] : 1e-12f; }
    for (int j = nsel; j < t; j++) { sel[j] = 0; w_out[j] = 1e-12f; }
    free(mask); free(cur); free(res); free(corr); free(order); free(prev); free(M); free(w);
}

/* ========================================================================
 * Top-t selection with the tie order of libstdc++'s std::partial_sort
 * (binary-heap select over [first, middle) then the rest), which the
 * reference uses at src/kv-compact-api.cpp:727,738. Only the SET of the
 * first t entries matters (they are re-sorted by position afterwards), and
 * that set depends on the heap's sift order when importances tie exactly.
 * ====================================================================== */
typedef struct { const float * imp; } orc_cmp_ctx;

/* "a ranks before b": higher importance first */
static int orc_before(const orc_cmp_ctx * c, int a, int b) { return c->imp[a] > c->imp[b]; }

static void orc_heap_push_up(int * h, long hole, long top, int val, const orc_cmp_ctx * c) {
    long parent = (hole - 1) / 2;
    while (hole > top && orc_before(c, h[parent], val)) {
        h[hole] = h[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    h[hole] = val;
}

/* sift the hole at `hole` down to a leaf along the preferred child, then
 * push `val` back up — the classic hole-based adjust of the STL heap. */
static void orc_heap_adjust(int * h, long hole, long len, int val, const orc_cmp_ctx * c) {
    long top = hole, child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (orc_before(c, h[child], h[child - 1])) child--;
        h[hole] = h[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        h[hole] = h[child - 1];
        hole = child - 1;
    }
    orc_heap_push_up(h, hole, top, val, c);
}

static void orc_partial_select(int * a, long middle, long last, const float * imp) {
    orc_cmp_ctx c = { imp };
    if (middle <= 0) return;
    if (middle >= 2) {
        long parent = (middle - 2) / 2;
        for (;;) {
            orc_heap_adjust(a, parent, middle, a[parent], &c);
            if (parent == 0) break;
            parent--;
        }
    }
    for (long i = middle; i < last; i++) {
        if (orc_before(&c, a[i], a[0])) {
            int v = a[i];
            a[i] = a[0];
            orc_heap_adjust(a, 0, middle, v, &c);
        }
    }
}

static int orc_int_cmp(const void * x, const void * y) {
    int a = *(const int *)x, b = *(const int *)y;
    return (a > b) - (a < b);
}

/* Greedy cosine-diversity selection (src/kv-compact-api.cpp:175-233).
 * Rows of K are the full n_embd-wide key rows (all heads). */
static void orc_select_diverse(const float * imp, const float * K, int T, int t, int n_embd,
                               float strength, int n_prefix, int * out, int * n_out) {
    unsigned char * used = (unsigned char *)calloc((size_t)T, 1);
    float * pen = (float *)calloc((size_t)T, 4);
    int n = 0;
    int pc = n_prefix < t ? n_prefix : t;
    for (int j = 0; j < pc; j++) { out[n++] = j; used[j] = 1; }
    while (n < t) {
        int best = -1;
        float bs = -1e30f;
        for (int j = 0; j < T; j++) {
            if (used[j]) continue;
            float sc = imp[j] * (1.0f - strength * pen[j]);
            if (sc > bs) { bs = sc; best = j; }
        }
        if (best < 0) break;
        out[n++] = best;
        used[best] = 1;
        const float * ks = K + (size_t)best * n_embd;
        float ns = 0.0f;
        for (int d = 0; d < n_embd; d++) ns += ks[d] * ks[d];
        ns = sqrtf(ns) + 1e-8f;
        for (int j = 0; j < T; j++) {
            if (used[j]) continue;
            const float * kj = K + (size_t)j * n_embd;
            float dot = 0.0f, nj = 0.0f;
            for (int d = 0; d < n_embd; d++) { dot += ks[d] * kj[d]; nj += kj[d] * kj[d]; }
            float cs = dot / (ns * sqrtf(nj) + 1e-8f);
            if (cs > pen[j]) pen[j] = cs;
        }
    }
    qsort(out, (size_t)n, sizeof(int), orc_int_cmp);
    *n_out = n;
    free(used); free(pen);
}

/* Quadratically spaced K rows as proxy queries (src/kv-compact-api.cpp:132-152). */
static float * orc_cheap_qref(const float * K, int T, int n_embd, int nq) {
    float * Q = (float *)malloc((size_t)nq * n_embd * 4);
    for (int qi = 0; qi < nq; qi++) {
        float fr = (float)(qi + 1) / (float)(nq + 1);
        fr = fr * fr;
        int pos = (int)(fr * (float)(T - 1));
        if (pos >= T) pos = T - 1;
        if (pos < 0) pos = 0;
        memcpy(Q + (size_t)qi * n_embd, K + (size_t)pos * n_embd, (size_t)n_embd * 4);
    }
    return Q;
}

static int orc_cheap_nq(int T) {                      /* src/kv-compact-api.cpp:384-387 */
    int n = T / 2;
    if (n > 64) n = 64;
    if (n < 4) n = 4;
    if (n > T) n = T;
    return n;
}

/* Full-vs-compacted attention quality on <=4 heads x <=32 queries
 * (src/kv-compact-api.cpp:239-325). */
static void orc_quality(const float * K, const float * V, const float * Q, int T, int nq,
                        int H, int dk, int dv, const kv_compact_result * r, kv_compact_stats * st) {
    float isd = 1.0f / sqrtf((float)dk);
    int t = r->t, ek = H * dk, ev = H * dv;
    float sc = 0.0f, sm = 0.0f;
    int agree = 0, total = 0;
    int mh = H < 4 ? H : 4, mq = nq < 32 ? nq : 32;
    float * os = (float *)malloc((size_t)T * 4);
    float * cs = (float *)malloc((size_t)(t > 0 ? t : 1) * 4);
    float * oo = (float *)malloc((size_t)dv * 4);
    float * co = (float *)malloc((size_t)dv * 4);
    for (int h = 0; h < mh; h++)
        for (int qi = 0; qi < mq; qi++) {
            const float * q = Q + (size_t)qi * ek + (size_t)h * dk;
            for (int j = 0; j < T; j++) {
                const float * k = K + (size_t)j * ek + (size_t)h * dk;
                float dot = 0.0f;
                for (int d = 0; d < dk; d++) dot += q[d] * k[d];
                os[j] = dot * isd;
            }
            orc_softmax_rows(os, 1, T);
            for (int d = 0; d < dv; d++) oo[d] = 0.0f;
            for (int j = 0; j < T; j++) {
                const float * v = V + (size_t)j * ev + (size_t)h * dv;
                for (int d = 0; d < dv; d++) oo[d] += os[j] * v[d];
            }
            for (int j = 0; j < t; j++) {
                const float * k = K + (size_t)r->selected_indices[j] * ek + (size_t)h * dk;
                float dot = 0.0f;
                for (int d = 0; d < dk; d++) dot += q[d] * k[d];
                cs[j] = dot * isd + r->beta[h][j];
            }
            orc_softmax_rows(cs, 1, t);
            for (int d = 0; d < dv; d++) co[d] = 0.0f;
            for (int j = 0; j < t; j++)
                for (int d = 0; d < dv; d++) co[d] += cs[j] * r->C_v[h][(size_t)j * dv + d];
            float dp = 0.0f, no = 0.0f, nc = 0.0f;
            for (int d = 0; d < dv; d++) { dp += oo[d] * co[d]; no += oo[d] * oo[d]; nc += co[d] * co[d]; }
            sc += dp / (sqrtf(no * nc) + 1e-8f);
            float mse = 0.0f;
            for (int d = 0; d < dv; d++) { float df = oo[d] - co[d]; mse += df * df; }
            sm += mse / (float)dv;
            int ao = 0, ac = 0;
            for (int d = 1; d < dv; d++) { if (oo[d] > oo[ao]) ao = d; if (co[d] > co[ac]) ac = d; }
            if (ao == ac) agree++;
            total++;
        }
    st->avg_cosine_sim = sc / (float)total;
    st->avg_mse = sm / (float)total;
    st->avg_agreement = (float)agree / (float)total;
    free(os); free(cs); free(oo); free(co);
}

static double orc_now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e3 + (double)ts.tv_nsec * 1e-6;
}

static void orc_result_alloc(kv_compact_result * r, int t, int H, int dv) {
    r->t = t;
    r->n_head_kv = H;
    r->selected_indices = (int *)malloc((size_t)(t > 0 ? t : 1) * sizeof(int));
    r->beta = (float **)malloc((size_t)H * sizeof(float *));
    r->C_v = (float **)malloc((size_t)H * sizeof(float *));
    for (int h = 0; h < H; h++) {
        r->beta[h] = (float *)malloc((size_t)(t > 0 ? t : 1) * 4);
        r->C_v[h] = (float *)malloc((size_t)(t > 0 ? t : 1) * dv * 4);
    }
}

void oracle_result_free(kv_compact_result * r) {             /* api.cpp:1113-1137 */
    if (!r) return;
    free(r->selected_indices);
    r->selected_indices = NULL;
    if (r->beta) { for (int h = 0; h < r->n_head_kv; h++) free(r->beta[h]); free(r->beta); r->beta = NULL; }
    if (r->C_v) { for (int h = 0; h < r->n_head_kv; h++) free(r->C_v[h]); free(r->C_v); r->C_v = NULL; }
    r->t = 0;
    r->n_head_kv = 0;
}

kv_compact_params oracle_params_default(void) {               /* api.cpp:333-358 */
    kv_compact_params p;
    memset(&p, 0, sizeof(p));
    p.target_ratio = 0.5f;
    p.ridge = 1e-6f;
    p.nnls_max_iter = 200;
    p.diversity_strength = 0.5f;
    p.skip_beta = 1;
    p.score_method = 1;
    p.omp_k_choice = 1;
    p.omp_refit_interval = 1;
    p.nnls_method = 1;
    return p;
}

/* Optional trace of the last unchunked body's global importance, used by
 * the parity tests to classify selection mismatches by importance gap. */
static float * g_trace_imp = NULL;
static int g_trace_cap = 0;
static int g_trace_len = 0;
static int g_trace_base = 0;   /* chunk start of the body being traced */

/* Record the global importance of every key of the next call into buf
 * (position j of the layer -> buf[j]); pass NULL to stop tracing. */
void oracle_trace_importance(float * buf, int cap) {
    g_trace_imp = buf; g_trace_cap = cap; g_trace_len = 0; g_trace_base = 0;
}
int oracle_trace_len(void) { return g_trace_len; }

/* Test aid: with `on`, the next calls stop after the key selection (indices
 * only; beta and C_v zero, stats zero), for shapes whose refit the oracle
 * would take minutes to solve while the parity tests need only the
 * selection and the traced importances. */
static int g_select_only = 0;
void oracle_select_only(int on) { g_select_only = on; }

/* beta for one head: w from NNLS on exp-scores, beta = log(max(1e-12, w))
 * (src/kv-compact-api.cpp:812-831). */
static void orc_beta_head(const float * E, const float * rs, const int * sel, int nq, int T,
                          int t, const kv_compact_params * p, float * beta) {
    float * M = (float *)malloc((size_t)nq * t * 4);
    float * w = (float *)malloc((size_t)t * 4);
    for (int qi = 0; qi < nq; qi++)
        for (int j = 0; j < t; j++) M[(size_t)qi * t + j] = E[(size_t)qi * T + sel[j]];
    if (p->nnls_method == 0) oracle_nnls_lh(M, rs, w, nq, t, p->nnls_max_iter);
    else oracle_nnls_pgd(M, rs, w, nq, t, 1e-12f, p->nnls_pgd_iters);
    for (int j = 0; j < t; j++) beta[j] = logf(w[j] > 1e-12f ? w[j] : 1e-12f);
    free(M); free(w);
}

/* C_v for one head: X = softmax(S[:, sel] + beta), LS against Y
 * (src/kv-compact-api.cpp:833-848). */
static void orc_refit_head(const float * S, const float * Y, const int * sel, const float * beta,
                           int nq, int T, int t, int dv, float ridge, float * cv) {
    float * X = (float *)malloc((size_t)nq * t * 4);
    for (int qi = 0; qi < nq; qi++)
        for (int j = 0; j < t; j++) X[(size_t)qi * t + j] = S[(size_t)qi * T + sel[j]] + beta[j];
    orc_softmax_rows(X, nq, t);
    oracle_least_squares(X, Y, cv, nq, t, dv, ridge);
    free(X);
}

/* The unchunked body of kv_compact (src/kv-compact-api.cpp:562-978). */
static int orc_compact_body(const float * K, const float * V, const float * Q, int T, int nq,
                            int H, int dk, int dv, int t, const kv_compact_params * p,
                            kv_compact_result * res) {
    double t0 = orc_now_ms();
    int ek = H * dk, ev = H * dv;
    float isd = 1.0f / sqrtf((float)dk);
    int need_exp = !p->skip_beta || p->use_omp;
    size_t nqT = (size_t)nq * T;

    float ** S = (float **)malloc((size_t)H * sizeof(float *));
    float ** A = (float **)malloc((size_t)H * sizeof(float *));
    float ** E = (float **)calloc((size_t)H, sizeof(float *));
    float ** RS = (float **)calloc((size_t)H, sizeof(float *));
    float * gimp = (float *)calloc((size_t)T, 4);
    float * himp = (float *)malloc((size_t)T * 4);
    float * sens = (float *)malloc((size_t)H * 4);
    float ** pimp = (float **)calloc((size_t)H, sizeof(float *));

    /* scores: sequential dot over d, then the separate 1/sqrt(d) scale
     * (math.h:44-54; api.cpp:618-628) */
    for (int h = 0; h < H; h++) {
        S[h] = (float *)malloc(nqT * 4);
        A[h] = (float *)malloc(nqT * 4);
        for (int qi = 0; qi < nq; qi++) {
            const float * q = Q + (size_t)qi * ek + (size_t)h * dk;
            for (int j = 0; j < T; j++) {
                const float * k = K + (size_t)j * ek + (size_t)h * dk;
                float acc = 0.0f;
                for (int d = 0; d < dk; d++) acc += q[d] * k[d];
                S[h][(size_t)qi * T + j] = acc;
            }
        }
        for (size_t i = 0; i < nqT; i++) S[h][i] *= isd;
    }
    /* softmax + importance, head aggregation (api.cpp:632-666) */
    for (int h = 0; h < H; h++) {
        if (need_exp) { E[h] = (float *)malloc(nqT * 4); RS[h] = (float *)malloc((size_t)nq * 4); }
        orc_softmax_importance(S[h], E[h], RS[h], A[h], himp, nq, T, p->score_method);
        if (p->use_sensitivity) {
            /* math.h:579-594 */
            float sum = 0.0f, mx = 0.0f;
            for (int j = 0; j < T; j++) {
                float cm = 0.0f;
                for (int qi = 0; qi < nq; qi++) { float v = A[h][(size_t)qi * T + j]; if (v > cm) cm = v; }
                sum += cm;
                if (cm > mx) mx = cm;
            }
            float mean = sum / (float)T;
            sens[h] = mx / (mean + 1e-12f);
            pimp[h] = (float *)malloc((size_t)T * 4);
            memcpy(pimp[h], himp, (size_t)T * 4);
        } else {
            for (int j = 0; j < T; j++) if (himp[j] > gimp[j]) gimp[j] = himp[j];
        }
    }
    if (p->use_sensitivity)                                   /* math.h:607-618 */
        for (int h = 0; h < H; h++)
            for (int j = 0; j < T; j++) gimp[j] += sens[h] * pimp[h][j];

    if (p->reasoning && p->reasoning->classifier) {            /* api.cpp:672-684 */
        int off = p->reasoning->token_offset;
        for (int j = 0; j < T; j++) {
            int ty = p->reasoning->classifier(j + off, p->reasoning->classifier_data);
            float w = 1.0f;
            if (ty == KV_TOKEN_THINKING) w = p->reasoning->thinking_weight;
            else if (ty == KV_TOKEN_TRANSITION) w = p->reasoning->transition_weight;
            gimp[j] *= w;
        }
    }
    if (g_trace_imp) {
        for (int j = 0; j < T && g_trace_base + j < g_trace_cap; j++) g_trace_imp[g_trace_base + j] = gimp[j];
        if (g_trace_base + T > g_trace_len) g_trace_len = g_trace_base + T;
    }

    /* selection (api.cpp:687-744) */
    int * sel = (int *)malloc((size_t)(t > 0 ? t : 1) * sizeof(int));
    float * omp_w = NULL;
    if (p->use_omp) {
        float * CE = (float *)calloc(nqT, 4);
        float * CS = (float *)calloc((size_t)nq, 4);
        for (int h = 0; h < H; h++) {
            for (size_t i = 0; i < nqT; i++) CE[i] += E[h][i];
            for (int i = 0; i < nq; i++) CS[i] += RS[h][i];
        }
        omp_w = (float *)malloc((size_t)t * 4);
        orc_omp_select(CE, CS, T, nq, t, sel, omp_w, p->omp_k_choice, p->omp_refit_interval,
                       p->nnls_pgd_iters);
        free(CE); free(CS);
    } else if (p->use_diversity) {
        int nout = 0;
        orc_select_diverse(gimp, K, T, t, ek, p->diversity_strength, p->n_shared_prefix, sel, &nout);
    } else {
        int pc = p->n_shared_prefix > 0 ? (p->n_shared_prefix < t ? p->n_shared_prefix : t) : 0;
        int ncand = T - pc;
        int * cand = (int *)malloc((size_t)(ncand > 0 ? ncand : 1) * sizeof(int));
        for (int j = 0; j < ncand; j++) cand[j] = pc + j;
        orc_partial_select(cand, t - pc, ncand, gimp);
        for (int j = 0; j < pc; j++) sel[j] = j;
        for (int j = 0; j < t - pc; j++) sel[pc + j] = cand[j];
        qsort(sel, (size_t)t, sizeof(int), orc_int_cmp);
        free(cand);
    }
    double t_score = orc_now_ms() - t0;
    double t1 = orc_now_ms();
    if (g_select_only) {
        orc_result_alloc(res, t, H, dv);
        memcpy(res->selected_indices, sel, (size_t)t * sizeof(int));
        for (int h = 0; h < H; h++) {
            memset(res->beta[h], 0, (size_t)t * 4);
            memset(res->C_v[h], 0, (size_t)t * dv * 4);
        }
        memset(&res->stats, 0, sizeof(res->stats));
        for (int h = 0; h < H; h++) { free(S[h]); free(A[h]); free(E[h]); free(RS[h]); free(pimp[h]); }
        free(S); free(A); free(E); free(RS); free(pimp);
        free(gimp); free(himp); free(sens); free(sel); free(omp_w);
        return 0;
    }

    /* Y_h = A_h V_h with sequential sums over T (math.h:70-80) */
    float ** Y = (float **)malloc((size_t)H * sizeof(float *));
    float * vb = (float *)malloc((size_t)T * dv * 4);
    for (int h = 0; h < H; h++) {
        Y[h] = (float *)malloc((size_t)nq * dv * 4);
        for (int j = 0; j < T; j++) memcpy(vb + (size_t)j * dv, V + (size_t)j * ev + (size_t)h * dv, (size_t)dv * 4);
        for (int qi = 0; qi < nq; qi++)
            for (int d = 0; d < dv; d++) {
                float acc = 0.0f;
                for (int j = 0; j < T; j++) acc += A[h][(size_t)qi * T + j] * vb[(size_t)j * dv + d];
                Y[h][(size_t)qi * dv + d] = acc;
            }
    }
    free(vb);

    float ** B = (float **)malloc((size_t)H * sizeof(float *));
    float ** CV = (float **)malloc((size_t)H * sizeof(float *));
    for (int h = 0; h < H; h++) {
        B[h] = (float *)calloc((size_t)(t > 0 ? t : 1), 4);
        CV[h] = (float *)malloc((size_t)(t > 0 ? t : 1) * dv * 4);
        if (!p->skip_beta) orc_beta_head(E[h], RS[h], sel, nq, T, t, p, B[h]);
        orc_refit_head(S[h], Y[h], sel, B[h], nq, T, t, dv, p->ridge, CV[h]);
    }

    /* worst-key swap refinement (api.cpp:852-946) */
    if (p->refine_rounds > 0 && t < T) {
        unsigned char * is_sel = (unsigned char *)calloc((size_t)T, 1);
        for (int j = 0; j < t; j++) is_sel[sel[j]] = 1;
        float * kv = (float *)malloc((size_t)t * 4);
        float * err = (float *)malloc((size_t)t * 4);
        float * row = (float *)malloc((size_t)t * 4);
        for (int rr = 0; rr < p->refine_rounds; rr++) {
            for (int j = 0; j < t; j++) kv[j] = 0.0f;
            for (int h = 0; h < H; h++) {
                for (int j = 0; j < t; j++) err[j] = 0.0f;
                for (int qi = 0; qi < nq; qi++) {
                    for (int j = 0; j < t; j++) row[j] = S[h][(size_t)qi * T + sel[j]] + B[h][j];
                    orc_softmax_rows(row, 1, t);
                    for (int j = 0; j < t; j++) err[j] += row[j] * row[j];
                }
                for (int j = 0; j < t; j++) kv[j] += err[j] / (float)nq;
            }
            int worst = 0;
            for (int j = 1; j < t; j++) if (kv[j] < kv[worst]) worst = j;
            int bu = -1;
            float bi = -1.0f;
            for (int j = 0; j < T; j++) if (!is_sel[j] && gimp[j] > bi) { bi = gimp[j]; bu = j; }
            if (bu < 0) break;
            if (bi <= gimp[sel[worst]] * 0.5f) break;
            is_sel[sel[worst]] = 0;
            is_sel[bu] = 1;
            sel[worst] = bu;
            qsort(sel, (size_t)t, sizeof(int), orc_int_cmp);
            for (int h = 0; h < H; h++) {
                if (p->skip_beta) memset(B[h], 0, (size_t)t * 4);
                else orc_beta_head(E[h], RS[h], sel, nq, T, t, p, B[h]);
                orc_refit_head(S[h], Y[h], sel, B[h], nq, T, t, dv, p->ridge, CV[h]);
            }
        }
        free(is_sel); free(kv); free(err); free(row);
    }
    double t_nnls = orc_now_ms() - t1;

    orc_result_alloc(res, t, H, dv);
    memcpy(res->selected_indices, sel, (size_t)t * sizeof(int));
    for (int h = 0; h < H; h++) {
        memcpy(res->beta[h], B[h], (size_t)t * 4);
        memcpy(res->C_v[h], CV[h], (size_t)t * dv * 4);
    }
    orc_quality(K, V, Q, T, nq, H, dk, dv, res, &res->stats);
    res->stats.elapsed_ms = orc_now_ms() - t0;
    res->stats.scoring_ms = t_score;
    res->stats.nnls_ms = t_nnls;

    for (int h = 0; h < H; h++) {
        free(S[h]); free(A[h]); free(E[h]); free(RS[h]); free(pimp[h]);
        free(Y[h]); free(B[h]); free(CV[h]);
    }
    free(S); free(A); free(E); free(RS); free(pimp); free(Y); free(B); free(CV);
    free(gimp); free(himp); free(sens); free(sel); free(omp_w);
    return 0;
}

/* kv_compact: validation, Q choice, t sizing, chunk geometry, merge
 * (src/kv-compact-api.cpp:360-560). */
int oracle_kv_compact(const float * K, const float * V, const float * Q, int T, int n_q,
                      int H, int dk, int dv, const kv_compact_params * params,
                      kv_compact_result * res) {
    if (!K || !V || !res) return -1;
    if (T <= 0 || H <= 0 || dk <= 0 || dv <= 0) return -2;
    kv_compact_params p = params ? *params : oracle_params_default();
    int ek = H * dk, ev = H * dv;

    float * cheap = NULL;
    const float * Qu = Q;
    int nq = n_q;
    if (p.use_cheap_qref || !Q) {
        nq = orc_cheap_nq(T);
        cheap = orc_cheap_qref(K, T, ek, nq);
        Qu = cheap;
    } else if (n_q <= 0) {
        return -2;
    }

    int t;
    if (p.target_count > 0) t = p.target_count < T ? p.target_count : T;
    else {
        t = (int)((float)T * p.target_ratio);
        if (t < 1) t = 1;
        if (t > T) t = T;
    }
    if (p.n_shared_prefix > t) t = p.n_shared_prefix < T ? p.n_shared_prefix : T;

    int cs = p.chunk_size;
    if (cs == 0) {
        float re = p.target_count > 0 ? (float)p.target_count / (float)T : p.target_ratio;
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

    if (cs >= T) {
        int rc = orc_compact_body(K, V, Qu, T, nq, H, dk, dv, t, &p, res);
        free(cheap);
        return rc;
    }

    double t0 = orc_now_ms();
    int nc = (T + cs - 1) / cs;
    kv_compact_result * cr = (kv_compact_result *)calloc((size_t)nc, sizeof(kv_compact_result));
    int rc = 0;
    for (int c = 0; c < nc && rc == 0; c++) {
        int st = c * cs, en = st + cs;
        if (en > T) en = T;
        int cT = en - st;
        kv_compact_params cp = p;
        cp.chunk_size = -1;
        cp.n_threads = 1;
        if (c > 0) cp.n_shared_prefix = 0;
        if (cp.n_shared_prefix > cT) cp.n_shared_prefix = cT;
        kv_compact_reasoning rz;
        if (cp.reasoning) { rz = *cp.reasoning; rz.token_offset += st; cp.reasoning = &rz; }
        g_trace_base = st;
        rc = oracle_kv_compact(K + (size_t)st * ek, V + (size_t)st * ev, Qu, cT, nq, H, dk, dv,
                               &cp, &cr[c]);
    }
    g_trace_base = 0;
    if (rc != 0) {
        for (int c = 0; c < nc; c++) oracle_result_free(&cr[c]);
        free(cr); free(cheap);
        return rc;
    }
    int tot = 0;
    for (int c = 0; c < nc; c++) tot += cr[c].t;
    orc_result_alloc(res, tot, H, dv);
    int off = 0;
    double ssum = 0.0, nsum = 0.0;
    for (int c = 0; c < nc; c++) {
        for (int j = 0; j < cr[c].t; j++) res->selected_indices[off + j] = cr[c].selected_indices[j] + c * cs;
        for (int h = 0; h < H; h++) {
            memcpy(res->beta[h] + off, cr[c].beta[h], (size_t)cr[c].t * 4);
            memcpy(res->C_v[h] + (size_t)off * dv, cr[c].C_v[h], (size_t)cr[c].t * dv * 4);
        }
        off += cr[c].t;
        ssum += cr[c].stats.scoring_ms;
        nsum += cr[c].stats.nnls_ms;
    }
    orc_quality(K, V, Qu, T, nq, H, dk, dv, res, &res->stats);
    res->stats.elapsed_ms = orc_now_ms() - t0;
    res->stats.scoring_ms = ssum;
    res->stats.nnls_ms = nsum;
    for (int c = 0; c < nc; c++) oracle_result_free(&cr[c]);
    free(cr);
    free(cheap);
    return 0;
}

/* Repeated compaction (src/kv-compact-api.cpp:980-1111). */
int oracle_kv_compact_multi_round(const float * K, const float * V, const float * Q, int T,
                                  int n_q, int H, int dk, int dv, const kv_compact_params * params,
                                  int n_rounds, kv_compact_result * res, kv_compact_stats * prs) {
    if (!K || !V || !res) return -1;
    if (T <= 0 || H <= 0 || dk <= 0 || dv <= 0) return -2;
    if (n_rounds < 1) return -3;
    kv_compact_params pc = params ? *params : oracle_params_default();
    if (!Q && !pc.use_cheap_qref) return -1;
    if (Q && n_q <= 0 && !pc.use_cheap_qref) return -2;
    int ek = H * dk, ev = H * dv;
    int * orig = (int *)malloc((size_t)T * sizeof(int));
    for (int i = 0; i < T; i++) orig[i] = i;
    float * cK = (float *)malloc((size_t)T * ek * 4);
    float * cV = (float *)malloc((size_t)T * ev * 4);
    memcpy(cK, K, (size_t)T * ek * 4);
    memcpy(cV, V, (size_t)T * ev * 4);
    int cT = T;
    float * cheap = NULL;
    const float * Qm = Q;
    int nqm = n_q;
    if (pc.use_cheap_qref || !Q) {
        nqm = orc_cheap_nq(T);
        cheap = orc_cheap_qref(K, T, ek, nqm);
        Qm = cheap;
    }
    for (int r = 0; r < n_rounds; r++) {
        int nqr = nqm < cT ? nqm : cT;
        kv_compact_result rr;
        memset(&rr, 0, sizeof(rr));
        int rc = oracle_kv_compact(cK, cV, Qm, cT, nqr, H, dk, dv, params, &rr);
        if (rc != 0) {
            oracle_result_free(&rr);
            free(orig); free(cK); free(cV); free(cheap);
            return rc;
        }
        if (prs) prs[r] = rr.stats;
        int nT = rr.t;
        int * no = (int *)malloc((size_t)(nT > 0 ? nT : 1) * sizeof(int));
        float * nK = (float *)malloc((size_t)(nT > 0 ? nT : 1) * ek * 4);
        float * nV = (float *)malloc((size_t)(nT > 0 ? nT : 1) * ev * 4);
        for (int j = 0; j < nT; j++) {
            int s = rr.selected_indices[j];
            no[j] = orig[s];
            memcpy(nK + (size_t)j * ek, cK + (size_t)s * ek, (size_t)ek * 4);
            for (int h = 0; h < H; h++)
                memcpy(nV + (size_t)j * ev + (size_t)h * dv, rr.C_v[h] + (size_t)j * dv, (size_t)dv * 4);
        }
        if (r == n_rounds - 1) {
            orc_result_alloc(res, nT, H, dv);
            memcpy(res->selected_indices, no, (size_t)nT * sizeof(int));
            for (int h = 0; h < H; h++) {
                memcpy(res->beta[h], rr.beta[h], (size_t)nT * 4);
                memcpy(res->C_v[h], rr.C_v[h], (size_t)nT * dv * 4);
            }
            res->stats = rr.stats;
        }
        oracle_result_free(&rr);
        free(cK); free(cV); free(orig);
        cK = nK; cV = nV; orig = no; cT = nT;
    }
    orc_quality(K, V, Qm, T, nqm, H, dk, dv, res, &res->stats);
    free(orig); free(cK); free(cV); free(cheap);
    return 0;
}

/* dequant -> compact -> requant (src/kv-compact-api.cpp:1182-1257). */
int oracle_kv_compact_quantized(const uint8_t * Kq, const uint8_t * Vq, const float * Q,
                                int kt, int vt, size_t krb, size_t vrb, int T, int n_q, int H,
                                int dk, int dv, const kv_compact_params * params,
                                kv_compact_quant_result * res) {
    if (!Kq || !Vq || !res) return -1;
    if (T <= 0 || H <= 0 || dk <= 0 || dv <= 0) return -2;
    int ek = H * dk, ev = H * dv;
    if (oracle_quant_row_elements(kt, krb) != ek || oracle_quant_row_elements(vt, vrb) != ev) return -4;
    float * Kf = (float *)malloc((size_t)T * ek * 4);
    float * Vf = (float *)malloc((size_t)T * ev * 4);
    for (int i = 0; i < T; i++) {
        orc_decode_row(Kq + (size_t)i * krb, kt, Kf + (size_t)i * ek, (size_t)ek);
        orc_decode_row(Vq + (size_t)i * vrb, vt, Vf + (size_t)i * ev, (size_t)ev);
    }
    memset(&res->base, 0, sizeof(res->base));
    int rc = oracle_kv_compact(Kf, Vf, Q, T, n_q, H, dk, dv, params, &res->base);
    if (rc != 0) { free(Kf); free(Vf); return rc; }
    int t = res->base.t;
    res->k_type = kt; res->v_type = vt; res->k_row_bytes = krb; res->v_row_bytes = vrb;
    res->K_out = (uint8_t *)malloc((size_t)(t > 0 ? t : 1) * krb);
    res->V_out = (uint8_t *)malloc((size_t)(t > 0 ? t : 1) * vrb);
    for (int j = 0; j < t; j++)
        orc_encode_row(Kf + (size_t)res->base.selected_indices[j] * ek, kt, res->K_out + (size_t)j * krb, ek);
    float * row = (float *)malloc((size_t)ev * 4);
    for (int j = 0; j < t; j++) {
        for (int h = 0; h < H; h++) memcpy(row + (size_t)h * dv, res->base.C_v[h] + (size_t)j * dv, (size_t)dv * 4);
        orc_encode_row(row, vt, res->V_out + (size_t)j * vrb, ev);
    }
    free(row); free(Kf); free(Vf);
    return 0;
}

void oracle_quant_result_free(kv_compact_quant_result * r) {   /* api.cpp:1259-1266 */
    if (!r) return;
    oracle_result_free(&r->base);
    free(r->K_out); r->K_out = NULL;
    free(r->V_out); r->V_out = NULL;
}

/* Per-unit softmax/importance exposed for element-level kernel parity:
 * scores S [m x n] -> softmax A, importance imp (math.h:142-248). */
void oracle_softmax_importance(const float * S, float * A, float * imp, float * row_sums,
                               int m, int n, int agg) {
    float * E = row_sums ? (float *)malloc((size_t)m * n * 4) : NULL;
    orc_softmax_importance(S, E, row_sums, A, imp, m, n, agg);
    free(E);
}
