// Tensor Memory Accelerator (TMA) helpers for sm_100a: 2-D tiled tensor
// maps built through the driver entry point (no libcuda link), mbarrier
// transaction barriers, and bounded waits.
//
// Every wait on an mbarrier gives up after kSpinLimit polls: it records the
// failure in the library's per-device status word (read back with
// sl_device_status) and lets the kernel return, instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace slb {

// 2-D fp32 row-major matrix [rows, cols] -> tensor map with box
// [box_rows, box_cols].  Returns false if the driver entry point is missing
// or the encode fails (caller falls back to the non-TMA kernel).
bool make_tmap_2d(CUtensorMap* map, const float* base, int64_t rows, int64_t cols,
                  int box_rows, int box_cols, bool swizzle128 = false);

// Per-device status word owned by the library (bit 0 = a bounded wait timed
// out); allocated on first use on the current device.
unsigned* device_status_word();

constexpr long long kSpinLimit = 1LL << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Plain arrive (one count) on an mbarrier.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Returns false on timeout (and raises bit 0 of *status).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned phase, unsigned* status,
                                          long long spin_limit = kSpinLimit) {
    const uint32_t a = smem_addr(bar);
    for (long long it = 0; it < spin_limit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(phase)
            : "memory");
        if (done) return true;
    }
    atomicOr(status, 1u);
    return false;
}

// TMA 2-D tile load: box at (col x, row y) into shared memory, completing
// `bytes` on `bar`.  x * sizeof(float) must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// L2 eviction-priority policies for TMA loads (createpolicy): evict_first
// for an operand each byte of which is read once (streamed), evict_last for
// one that later CTAs read again, so the stream does not push it out of L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// TMA 2-D tile load with an L2 cache policy (see above).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, int x, int y,
                                                 uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// 1-D bulk copy global -> shared (no multicast), completing `bytes` on
// `bar`.  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* src, unsigned bytes,
                                             uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(smem_dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

}  // namespace slb
