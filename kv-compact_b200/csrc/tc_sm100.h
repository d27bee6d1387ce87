// tc_sm100.h — thin inline-PTX wrappers for the 5th-generation tensor cores
// (tcgen05) and shared-memory mbarriers on sm_100a.
//
// Operand tiles live in shared memory in the K-major, no-swizzle canonical
// layout: "core matrices" of 8 rows x 16 bytes stored contiguously (128 B),
// consecutive 16-byte K chunks LBO bytes apart, consecutive 8-row groups SBO
// bytes apart. The accumulator lives in tensor memory (TMEM): row i of a
// 128-row tile is TMEM lane i, column j is TMEM column base + j, and warp w
// of the CTA may read lanes [32w, 32w + 32).
#pragma once

#include <stdint.h>

namespace kvc_tc {

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Shared-memory matrix descriptor (sm_100 format: version 1, no swizzle).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;                       // descriptor version for sm_100
    return d;                                     // base offset 0, layout SWIZZLE_NONE
}

// Instruction descriptor of kind::tf32: fp32 accumulate, both operands
// TF32 and K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4)                      // D format F32
         | (2u << 7)                      // A format TF32
         | (2u << 10)                     // B format TF32
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// Arrive once on the mbarrier when all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void commit(uint64_t * mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(mbar)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t * slot, uint32_t ncols) {     // one full warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {       // the allocating warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes made visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_smem_to_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float * v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void mbar_init(uint64_t * mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(mbar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Wait for the completion of the mbarrier phase with the given parity, at
// most `limit` polls. Returns false when the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t * mbar, uint32_t parity, uint32_t limit) {
    const uint32_t a = smem_u32(mbar);
    for (uint32_t i = 0; i < limit; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// Instruction descriptor of kind::f16 with f16 operands: fp32 accumulate,
// A and B both F16 and K-major, M x N tile (A/B format 0 = F16).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                      // D format F32
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T in kind::f16, issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// 16 consecutive fp32 columns of this thread's TMEM lane, without waiting:
// several loads can be in flight before one tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t * r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 consecutive fp32 columns into this thread's TMEM lane (then tmem_wait_st
// before the values are relied on).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t * r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
           "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// One arrival on the mbarrier (release semantics at CTA scope).
__device__ __forceinline__ void mbar_arrive(uint64_t * mbar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(mbar)) : "memory");
}

// 32 bytes (8 consecutive fp32, 32-byte aligned) in one access: a whole
// 32-byte sector per thread.
__device__ __forceinline__ void st_global_v8(float * p, const float * v) {
    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 :: "l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                 : "memory");
}

// Arm the mbarrier for one arrival (this thread's) plus `bytes` of
// asynchronous-copy transactions.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * mbar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(mbar)), "r"(bytes) : "memory");
}

// 2-D tiled TMA load of one box of the tensor map at `tmap` (a global-memory
// CUtensorMap) into shared memory, completing on `mbar`. x is the innermost
// coordinate (its byte offset must be a multiple of 16), y the row. No
// multicast: the box lands in this CTA's shared memory only.
__device__ __forceinline__ void tma_load_2d(void * dst, const void * tmap, int x, int y, uint64_t * mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(mbar)) : "memory");
}

// The same wait for a role that may wait long (a producer ahead of its
// consumer): after the first polls it sleeps `ns` nanoseconds between polls,
// leaving the issue slots to the warps that have work. At most `limit` polls.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t * mbar, uint32_t parity, uint32_t limit, uint32_t ns) {
    const uint32_t a = smem_u32(mbar);
    for (uint32_t i = 0; i < limit; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
        if (i >= 4) __nanosleep(ns);
    }
    return false;
}

// Round an fp32 value to the nearest TF32 value (10 explicit mantissa bits,
// ties away from zero), returned as fp32 with the 13 low bits clear — the
// tensor core then reads it exactly.
__device__ __forceinline__ float tf32_round(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// Split x into a TF32 head and a TF32 tail: hi = round(x), lo = round(x - hi)
// (x - hi is exact in fp32). |x - hi - lo| <= 2^-22 |x|, and rounding both
// parts to nearest keeps the split unbiased (plain truncation would shrink
// every product by up to 2^-20 in the same direction).
__device__ __forceinline__ void tf32_split(float x, float & hi, float & lo) {
    hi = tf32_round(x);
    lo = tf32_round(__fsub_rn(x, hi));
}

}  // namespace kvc_tc
