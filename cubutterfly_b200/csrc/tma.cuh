// tma.cuh -- bulk-copy (TMA) and mbarrier helpers for persistent tile pipelines.
//
// A pipeline keeps STAGES input tiles in flight per CTA: one thread issues
// cp.async.bulk global->shared copies that complete on an mbarrier; all
// threads wait for the barrier's phase, consume the tile, and the slot is
// refilled with the tile STAGES iterations ahead.  Every wait is bounded: on
// expiry the kernel records an error code in a device word and leaves the
// loop (no trap, no endless spin).
#pragma once

#include "common.cuh"

namespace cubf::tma {

// ~2^22 polls with a growing nanosleep back-off: well over a second, far
// beyond any healthy copy latency.
constexpr uint32_t kWaitPolls = 1u << 22;
constexpr unsigned kErrTimeout = 1u;

CUBF_DEV uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

CUBF_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make the initialised barriers visible to the async (TMA) proxy.
CUBF_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

CUBF_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

CUBF_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
        "r"(bytes)
        : "memory");
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned) completing on `bar`.
CUBF_DEV void bulk_load(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

CUBF_DEV bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for the phase with `parity` to complete.  Returns false on
// expiry.
CUBF_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
    uint32_t sleep = 0;
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_test(bar, parity)) return true;
        if (i > 64) {
            __nanosleep(sleep);
            sleep = sleep < 256 ? sleep + 32 : 256;
        }
    }
    return false;
}

CUBF_DEV void record_error(unsigned* err, unsigned code) {
    if (err) atomicOr(err, code);
}

// Abort path of a ring pipeline whose iteration k gave up waiting: records
// the error and waits (bounded) for the copies still in flight -- iterations
// k .. k+STAGES-1 that have a tile -- so that none lands after the CTA
// leaves.  Called by the issuing thread only.
template <int STAGES>
CUBF_DEV void abort_ring(uint64_t* bar, int k, size_t first_tile, size_t tile_stride, size_t tiles,
                         unsigned* err) {
    record_error(err, kErrTimeout);
    for (int j = k; j < k + STAGES; ++j) {
        if (first_tile + static_cast<size_t>(j) * tile_stride >= tiles) break;
        mbar_wait(&bar[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1));
    }
}

}  // namespace cubf::tma
