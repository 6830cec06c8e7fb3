// pa_common.cuh - small sm_100a building blocks shared by the phone-attn kernels: mbarriers with bounded waits,
// 1-D bulk (TMA engine) copies, f16 packing, byte permutes and the warp-level f16 and s8 MMAs.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace pa {

// error codes written to the device status word (the host reads it after the stream is synchronised)
enum : int { ST_OK = 0, ST_TIMEOUT_FULL = 1, ST_TIMEOUT_EMPTY = 2, ST_TIMEOUT_DRAIN = 3, ST_BAD_ARGS = 4,
             ST_TIMEOUT_PEER = 5 };   // a rank's partial did not arrive in time (peer-store exchange)

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// orders this thread's generic-proxy shared-memory accesses with its following async-proxy (bulk copy) ones
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for phase `parity` of an mbarrier, giving up after timeout_ns of wall time or as soon as *abort is set
// (abort may be null).
// Returns true once the phase completed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t timeout_ns,
                                                  const volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 63) {
            if (abort != nullptr && *abort) return false;
            if (globaltimer_ns() - t0 > timeout_ns) return false;
        }
    }
}

// 1-D bulk copy global -> this CTA's shared memory, completing on an mbarrier (no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory loads by 32-bit shared address. They are plain C++ loads (not volatile asm), so the compiler may
// schedule them early, e.g. a tile's V words under the softmax of its scores; the mbarrier waits and fences above
// carry "memory" clobbers, so no load moves across a wait for the data it reads.
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    return *reinterpret_cast<const uint32_t *>(__cvta_shared_to_generic(addr));
}
// the same at a compile-time byte offset from base
template <int OFF>
__device__ __forceinline__ uint32_t lds32o(uint32_t base) {
    return *reinterpret_cast<const uint32_t *>(__cvta_shared_to_generic(base + OFF));
}
__device__ __forceinline__ uint32_t lds16(uint32_t addr) {
    return *reinterpret_cast<const uint16_t *>(__cvta_shared_to_generic(addr));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// (a & b) | c
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// two fp32 -> f16x2 (lo = a, hi = b), round to nearest even
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(d) : "f"(a), "f"(b));
    return d;
}

// 2^x (MUFU ex2, flush-to-zero)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// transpose of an 8x8 b16 matrix held in mma fragment order (one .b32 per lane)
__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(x));
    return d;
}

// four 8x8 b16 matrices from shared memory in mma fragment order; lane l gives the 16-byte row address of matrix l/8,
// row l%8 (volatile: the compiler keeps it after the mbarrier wait for the data)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// the same, each matrix transposed
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D += A(16x16, f16, row) * B(16x8, f16, col), fp32 accumulate
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A(16x32, s8, row) * B(32x8, s8, col), exact int32 (a fresh accumulator: one call is one 32-value dot product
// per (row, column)). Fragments: a0/a2 = row g, k 4t..4t+3 / 16+4t..; a1/a3 = row g+8; b0/b1 = k 4t.. / 16+4t.., column g;
// d0,d1 = row g, columns 2t, 2t+1; d2,d3 = row g+8.
__device__ __forceinline__ void mma16832_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                            uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
// f16 bits (low 16 of x) -> fp32, exact
__device__ __forceinline__ float h2f_bits(uint32_t x) { return __half2float(__ushort_as_half((unsigned short) x)); }

constexpr float LOG2E = 1.4426950408889634f;
constexpr float M_EMPTY = -1e30f;   // running max before any key (as scripts/sme/sme_attn.c:281)

}  // namespace pa
