// Shared-memory barriers and bulk asynchronous copies (sm_90+ PTX), shared by
// the tensor-core scorer and the weight-streaming products.  Every wait is
// bounded: it reports failure instead of spinning forever.
#pragma once

#include <cstdint>

namespace popkv {

constexpr int kMaxWaitPolls = 1 << 20;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Generic-proxy shared-memory accesses are ordered before later async-proxy
// (bulk copy, tensor core) accesses of the same memory.
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(mbar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Bounded wait for the phase with the given parity; false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, int polls = kMaxWaitPolls) {
    const uint32_t addr = smem_addr(mbar);
    for (int i = 0; i < polls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t"
            ".reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t"
            "}\n"
            : "=r"(done) : "r"(addr), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
    asm volatile(
        "{\n\t"
        ".reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t"
        "}\n" :: "r"(smem_addr(mbar)) : "memory");
}

// Arrive on the barrier and announce `bytes` of copies that complete on it.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* mbar, uint32_t bytes) {
    asm volatile(
        "{\n\t"
        ".reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t"
        "}\n" :: "r"(smem_addr(mbar)), "r"(bytes) : "memory");
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global to this CTA's shared memory, completing on `mbar`; the destination is this CTA only.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(mbar)) : "memory");
}

}  // namespace popkv
