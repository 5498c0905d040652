// common.cuh -- device helpers shared by the sm_100a butterfly kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#define CUBF_DEV __device__ __forceinline__

namespace cubf {

// ---- compile-time bit helpers ------------------------------------------
constexpr int popc32(uint32_t x) {
    int c = 0;
    for (int i = 0; i < 32; ++i) c += (x >> i) & 1u;
    return c;
}
constexpr uint32_t lowmask(int n) { return n <= 0 ? 0u : (n >= 32 ? ~0u : ((1u << n) - 1u)); }
// Bit position of the j-th set bit of m (j counted from the least significant).
constexpr int nth_bit(uint32_t m, int j) {
    for (int b = 0; b < 32; ++b)
        if ((m >> b) & 1u) {
            if (j == 0) return b;
            --j;
        }
    return -1;
}
// Scatter the low bits of x into the set bits of m (parallel bit deposit).
constexpr uint32_t deposit(uint32_t x, uint32_t m) {
    uint32_t r = 0;
    int src = 0;
    for (int b = 0; b < 32; ++b)
        if ((m >> b) & 1u) {
            r |= ((x >> src) & 1u) << b;
            ++src;
        }
    return r;
}

// Parallel bit extract: gather the bits of x selected by m into the low bits.
constexpr uint32_t extract(uint32_t x, uint32_t m) {
    uint32_t r = 0;
    int dst = 0;
    for (int b = 0; b < 32; ++b)
        if ((m >> b) & 1u) {
            r |= ((x >> b) & 1u) << dst;
            ++dst;
        }
    return r;
}

// deposit(r, m) for every r < E, as a compile-time table (indexing it with an
// unrolled loop counter folds to immediates).
template <int E>
struct Offsets {
    uint32_t v[E];
};
template <int E>
constexpr Offsets<E> make_offsets(uint32_t m) {
    Offsets<E> o{};
    for (int r = 0; r < E; ++r) o.v[r] = deposit(static_cast<uint32_t>(r), m);
    return o;
}

// Runtime deposit of x into the compile-time mask M (unrolled; used once per
// exchange group, not per element).
template <uint32_t M, int BITS>
CUBF_DEV uint32_t deposit_rt(uint32_t x) {
    uint32_t r = 0;
    int src = 0;
#pragma unroll
    for (int b = 0; b < BITS; ++b) {
        if ((M >> b) & 1u) {
            r |= ((x >> src) & 1u) << b;
            ++src;
        }
    }
    return r;
}

// ---- storage <-> compute conversions --------------------------------------
template <typename S, typename C>
struct Convert;
template <>
struct Convert<float, float> {
    static CUBF_DEV float load(float x) { return x; }
    static CUBF_DEV float store(float x) { return x; }
};
template <>
struct Convert<__nv_bfloat16, float> {
    static CUBF_DEV float load(__nv_bfloat16 x) { return __bfloat162float(x); }
    static CUBF_DEV __nv_bfloat16 store(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Convert<__half, float> {
    static CUBF_DEV float load(__half x) { return __half2float(x); }
    static CUBF_DEV __half store(float x) { return __float2half_rn(x); }
};
template <>
struct Convert<uint32_t, uint32_t> {
    static CUBF_DEV uint32_t load(uint32_t x) { return x; }
    static CUBF_DEV uint32_t store(uint32_t x) { return x; }
};
template <>
struct Convert<unsigned long long, unsigned long long> {
    static CUBF_DEV unsigned long long load(unsigned long long x) { return x; }
    static CUBF_DEV unsigned long long store(unsigned long long x) { return x; }
};

// 16-byte vector of storage elements.
template <typename T>
struct alignas(16) Vec16 {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

// L2 residency hints for the tile passes.  A single-pass transform streams
// (evict-first both ways); in a multi-pass chain run on an L2-sized chunk the
// intermediate is stored evict-last so the next pass reads it from L2, and the
// final pass streams its output.
enum CacheMode : int { kStream = 0, kChainFirst = 1, kChainLast = 2, kChainMiddle = 3 };

// Programmatic dependent launch (launch_dependent in launch_util.cuh): a
// kernel launched that way may be scheduled while the kernel before it on
// the stream still runs; pdl_begin() waits until that kernel has completed
// and its writes are visible, then lets the kernel after this one be
// scheduled the same way.  Called first, before any global memory access, so
// the kernel's semantics are those of an ordinary stream-ordered launch; what
// it gains is the launch and CTA scheduling latency between back-to-back
// kernels.  Both instructions are no-ops in a kernel launched without the
// attribute.
CUBF_DEV void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Bulk prefetch of [p, p + bytes) into L2 (one instruction; p 16-byte
// aligned, bytes a multiple of 16).  One-shot kernels issue it for the tile
// the CTA one resident wave later will read, so DRAM keeps streaming while
// the current wave computes.
CUBF_DEV void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch of the rows [first, first + count) x row_bytes of the tile that
// CTA blockIdx.x + stride will process (thread 0 only; stride 0 disables).
CUBF_DEV void prefetch_next_wave(const void* base, size_t tile_bytes, size_t last_bytes, unsigned stride) {
    if (stride == 0 || threadIdx.x != 0) return;
    const size_t next = static_cast<size_t>(blockIdx.x) + stride;
    if (next >= gridDim.x) return;
    const size_t bytes = next + 1 == gridDim.x ? last_bytes : tile_bytes;
    const unsigned char* p = static_cast<const unsigned char*>(base) + next * tile_bytes;
    for (size_t off = 0; off < bytes; off += size_t{1} << 20) {
        const size_t n = bytes - off < (size_t{1} << 20) ? bytes - off : (size_t{1} << 20);
        prefetch_l2(p + off, static_cast<uint32_t>(n));
    }
}

// The same for an explicit (virtual) CTA `block` of `grid` run by threads
// vtid = 0..: the persistent chain kernel runs tile passes as queue items.
CUBF_DEV void prefetch_wave_of(const void* base, size_t tile_bytes, size_t last_bytes, unsigned stride,
                               size_t block, size_t grid, uint32_t vtid) {
    if (stride == 0 || vtid != 0) return;
    const size_t next = block + stride;
    if (next >= grid) return;
    const size_t bytes = next + 1 == grid ? last_bytes : tile_bytes;
    const unsigned char* p = static_cast<const unsigned char*>(base) + next * tile_bytes;
    for (size_t off = 0; off < bytes; off += size_t{1} << 20) {
        const size_t n = bytes - off < (size_t{1} << 20) ? bytes - off : (size_t{1} << 20);
        prefetch_l2(p + off, static_cast<uint32_t>(n));
    }
}

CUBF_DEV uint64_t l2_policy(bool keep) {
    uint64_t p;
    if (keep)
        asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    else
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
CUBF_DEV uint4 ld16_hint(const void* p, uint64_t pol) {
    uint4 r;
    asm volatile("ld.global.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(pol));
    return r;
}
// The same load served by L2 only (not L1): data another CTA wrote earlier in
// the same kernel (the persistent chain kernel's second pass).
CUBF_DEV uint4 ld16_hint_cg(const void* p, uint64_t pol) {
    uint4 r;
    asm volatile("ld.global.cg.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(pol)
                 : "memory");
    return r;
}
CUBF_DEV void st16_hint(void* p, uint4 v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v4.u32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w), "l"(pol)
                 : "memory");
}

// Streaming loads/stores: the transforms touch each byte once, so keep them
// out of L1 and mark them evict-first in L2.
template <typename T>
CUBF_DEV Vec16<T> ldg_stream(const Vec16<T>* p) {
    Vec16<T> r;
    uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
    *reinterpret_cast<uint4*>(&r) = u;
    return r;
}
template <typename T>
CUBF_DEV void stg_stream(Vec16<T>* p, const Vec16<T>& v) {
    __stcs(reinterpret_cast<uint4*>(p), *reinterpret_cast<const uint4*>(&v));
}

}  // namespace cubf
