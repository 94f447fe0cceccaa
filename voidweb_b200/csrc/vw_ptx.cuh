// vw_ptx.cuh -- thin inline-PTX helpers for sm_100a: mbarriers, TMA tensor
// and bulk copies, warp-level tensor-core fragments (ldmatrix / movmatrix /
// mma.sync), and bounded waits.  Every wait here gives up after a deadline on
// the SM's cycle counter so that no kernel can hang a GPU; the caller records
// the failure in the pool's device error word and unwinds.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace vw {

// Device error word bits (read back by vw_pool_check).
enum : uint32_t {
    kDevErrBlockId = 1u << 0,     // block id >= num_blocks in a table or pair list
    kDevErrSeqLen = 1u << 1,      // seq_len == 0 or longer than the block table row
    kDevErrTimeout = 1u << 2,     // a bounded wait gave up
    kDevErrSlot = 1u << 3,        // append slot outside the pool
    kDevErrLaunch = 1u << 4,      // unusable launch (dynamic shared memory not 1024-B aligned)
};

// Wait deadline in SM cycles: 4e9 cycles is about 2 s at the 1965 MHz maximum
// clock and at most about 4 s at any clock the part runs a kernel at; kernels
// here run for microseconds.  The cycle counter is read in a few cycles, unlike
// %globaltimer, so polling it does not delay the waiter's wake-up.
constexpr uint64_t kWaitDeadlineCycles = 4000000000ull;

__device__ __forceinline__ uint64_t cycles() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Suspend-time hint of the waits, in ns: a waiting thread sleeps at most this
// long before it rechecks (0: the hardware's own limit).  With the hint the
// FP8 decode of the Llama-3-8B batch measured 4028 against 3751 GB/s and the
// Qwen decode 4535 against 4512 (20, 200 and 2000 ns alike).
#ifndef VW_MBAR_SUSPEND_HINT_NS
#define VW_MBAR_SUSPEND_HINT_NS 200
#endif

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
#if VW_MBAR_SUSPEND_HINT_NS > 0
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"((uint32_t)VW_MBAR_SUSPEND_HINT_NS)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
#endif
    return ok != 0;
}

// Wait until the phase with the given parity has completed, or until the
// deadline (cycles(), see kWaitDeadlineCycles) passes.  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline) {
    if (mbar_try_wait(bar, parity)) return true;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (cycles() > deadline) return false;
    }
}

// ---- TMA / bulk copies (no multicast anywhere, no L2 eviction hints) -------

// 2-D tiled tensor load; the box and swizzle come from the tensor map.  A
// negative or out-of-range coordinate reads the map's zero fill.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1),
          "r"(smem_u32(bar))
        : "memory");
}

// 3-D tiled tensor load (same rules as the 2-D form).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
          "r"(smem_u32(bar))
        : "memory");
}

// Untiled bulk copy global -> shared; both addresses 16-B aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-B aligned) into L2.  A hint:
// it reads nothing into the CTA and orders nothing.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                 ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- programmatic dependent launch -------------------------------------------

// Wait until the preceding grid on the stream has completed and its memory is
// visible (no-op when the kernel was not launched as a programmatic dependent).
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Let the next programmatic dependent grid start launching.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- named barrier among a subset of warps ---------------------------------

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- warp-level tensor-core fragments ---------------------------------------

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// D = A(16x16, row) * B(16x8, col) + C, f32 accumulate.
template <bool kBF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    if constexpr (kBF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
            "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
            "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// Pack two f32 into a 16-bit pair (lo in bits 0..15), round to nearest even.
template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    if constexpr (kBF16)
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- 16-bit element helpers --------------------------------------------------

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    float f;
    asm("{ .reg .f16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((uint16_t)h));
    return f;
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
    return r;
}

__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
    uint16_t r;
    asm("{ .reg .f16 t; cvt.rn.f16.f32 t, %1; mov.b16 %0, t; }" : "=h"(r) : "f"(f));
    return r;
}

}  // namespace vw
