// launch_bitwise.cu -- instantiations and launchers of the FWHT / zeta tile kernels.
//
// Compiled once per (operator, storage) pair: the translation unit is built
// with CUBF_BW_OP and CUBF_BW_TYPE defined, so the instantiation sets compile
// in parallel.  launch_bitwise_dispatch.cpp routes a BwVariant to the unit.
#include "bitwise.cuh"
#include "chain.cuh"
#include "fwht.cuh"
#include "kernels.hpp"
#include "launch_util.cuh"

#include <algorithm>


#ifndef CUBF_BW_OP
#error "CUBF_BW_OP must be defined (0 fwht, 1 subset zeta, 2 superset zeta)"
#endif
#ifndef CUBF_BW_TYPE
#error "CUBF_BW_TYPE must be defined (0 f32, 1 bf16, 2 f16, 3 u32, 4 u64)"
#endif

namespace cubf {
namespace {

#if CUBF_BW_OP == 0
using Op = bw::FwhtOp;
#elif CUBF_BW_OP == 1
using Op = bw::ZetaOp<false>;
#else
using Op = bw::ZetaOp<true>;
#endif

#if CUBF_BW_TYPE == 0
using TS = float;
using TC = float;
#elif CUBF_BW_TYPE == 1
using TS = __nv_bfloat16;
using TC = float;
#elif CUBF_BW_TYPE == 2
using TS = __half;
using TC = float;
#elif CUBF_BW_TYPE == 3
using TS = uint32_t;
using TC = uint32_t;
#else
using TS = unsigned long long;
using TC = unsigned long long;
#endif

// Values per thread: 64 (LOGE 6) for 4-byte compute, 32 for 8-byte compute.
constexpr int kLogE = sizeof(TC) == 8 ? 5 : 6;
constexpr int kLogW = sizeof(TS) == 8 ? 3 : (sizeof(TS) == 4 ? 4 : 5);  // 64-byte column blocks
constexpr int kMaxContig = sizeof(TC) == 8 ? 13 : 14;
constexpr int kMaxStrided = sizeof(TC) == 8 ? 9 : 10;

#if CUBF_BW_OP == 0
// FWHT tiles: one thread per row up to 64 values (no exchange), rows of 128
// over 4 threads of 32 values (shuffle finish: fewer registers, more resident
// warps), then 64 values per thread; rows narrower than one 16-byte vector
// use the generic kernel.
constexpr int fwht_log_e(int logh) { return logh <= 6 ? logh : (logh == 7 ? 5 : 6); }
constexpr bool fwht_pair_kernel(int logh) { return (1 << logh) * static_cast<int>(sizeof(TS)) >= 16; }

template <int LOGH>
struct FwhtEntry {
    static constexpr int LOGE = fwht_log_e(LOGH);
    using S = fwht::FwhtShape<TS, LOGH, LOGE>;
    static constexpr bool kShuffle = fwht::ShuffleFinish<S>::value;
    static constexpr int SMEM = kShuffle ? 0 : S::SMEM_BYTES;
    static LaunchShape shape() {
        LaunchShape s;
        s.threads = S::TPB;
        s.smem_bytes = SMEM;
        s.units_per_cta = S::TILES;
        s.elems_per_thread = S::E;
        s.exchanges = kShuffle ? 0 : S::G.count - 1 + (S::STAGE_OUT ? 1 : 0);
        return s;
    }
    static cudaError_t launch(const void* in, void* out, std::size_t outer, std::size_t inner, bool inverse,
                              float scale, int cache_mode, cudaStream_t stream) {
        (void)inverse;  // FWHT is its own inverse up to the scale
        (void)cache_mode;
        if (inner != 1) return cudaErrorInvalidValue;
        if (outer == 0) return cudaSuccess;
        auto kernel = fwht::fwht_tile_kernel<TS, LOGH, LOGE>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, S::TPB, SMEM, &grid_cap);
        if (e != cudaSuccess) return e;
        const std::size_t blocks = (outer + S::TILES - 1) / S::TILES;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        const unsigned stride = blocks > static_cast<std::size_t>(grid_cap) ? grid_cap : 0;
        return launch_dependent(kernel, static_cast<unsigned>(blocks), S::TPB, SMEM, stream, static_cast<const TS*>(in),
                                static_cast<TS*>(out), outer, scale, stride);
    }
};
#endif

template <int LOGH, int LOGW>
struct Entry {
    using S = bw::TileShape<TS, TC, LOGH, LOGW, kLogE>;
    static LaunchShape shape() {
        LaunchShape s;
        s.threads = S::TPB;
        s.smem_bytes = S::SMEM_BYTES;
        s.units_per_cta = S::TILES;
        s.elems_per_thread = S::E;
        s.exchanges = S::G.count - 1;
        return s;
    }
    static cudaError_t launch(const void* in, void* out, std::size_t outer, std::size_t inner, bool inverse,
                              float scale, int cache_mode, cudaStream_t stream) {
        auto kernel = bw::bitwise_tile_kernel<Op, TS, TC, LOGH, LOGW, kLogE>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, S::TPB, S::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        if ((inner >> LOGW) == 0 || (inner & (inner - 1)) != 0) return cudaErrorInvalidValue;
        if (LOGW == 0 && inner != 1) return cudaErrorInvalidValue;
        int log_inner = 0;
        while ((std::size_t{1} << log_inner) < inner) ++log_inner;
        const std::size_t tiles = outer * (inner >> LOGW);
        const std::size_t blocks = (tiles + S::TILES - 1) / S::TILES;
        if (blocks == 0) return cudaSuccess;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        // contiguous passes that stream from DRAM prefetch one resident wave ahead
        const bool streams_in = LOGW == 0 && (cache_mode == kStream || cache_mode == kChainFirst);
        const unsigned stride = streams_in && blocks > static_cast<std::size_t>(grid_cap) ? grid_cap : 0;
        return launch_dependent(kernel, static_cast<unsigned>(blocks), S::TPB, S::SMEM_BYTES, stream,
                                static_cast<const TS*>(in), static_cast<TS*>(out), outer, log_inner, inverse ? 1 : 0,
                                scale, cache_mode, stride);
    }
};

using LaunchFn = cudaError_t (*)(const void*, void*, std::size_t, std::size_t, bool, float, int, cudaStream_t);
using ShapeFn = LaunchShape (*)();

#if CUBF_BW_OP == 0
template <int H>
constexpr LaunchFn contig_launch() {
    if constexpr (fwht_pair_kernel(H)) return FwhtEntry<H>::launch;
    else return Entry<H, 0>::launch;
}
template <int H>
constexpr ShapeFn contig_shape() {
    if constexpr (fwht_pair_kernel(H)) return FwhtEntry<H>::shape;
    else return Entry<H, 0>::shape;
}
#else
template <int H>
constexpr LaunchFn contig_launch() { return Entry<H, 0>::launch; }
template <int H>
constexpr ShapeFn contig_shape() { return Entry<H, 0>::shape; }
#endif

template <int... H>
struct Contig {
    static constexpr LaunchFn launch[] = {contig_launch<H>()...};
    static constexpr ShapeFn shape[] = {contig_shape<H>()...};
};
template <int... H>
struct Strided {
    static constexpr LaunchFn launch[] = {Entry<H, kLogW>::launch...};
    static constexpr ShapeFn shape[] = {Entry<H, kLogW>::shape...};
};

#if CUBF_BW_OP == 0
// FWHT: one contiguous pass per row (N <= 2^14).
using C = Contig<1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14>;
using T = Strided<1>;
constexpr bool kHasStrided = false;
#else
#if CUBF_BW_TYPE == 4
using C = Contig<1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13>;
using T = Strided<1, 2, 3, 4, 5, 6, 7, 8, 9>;
#else
using C = Contig<1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14>;
using T = Strided<1, 2, 3, 4, 5, 6, 7, 8, 9, 10>;
#endif
constexpr bool kHasStrided = true;
#endif

#if CUBF_BW_OP != 0
// Chunk-overlapped two-pass chains (csrc/chain.cuh): pass A is the widest
// contiguous tile, pass B any strided one; C + 1 step launches on `stream`.
template <int H1>
struct ChainEntry {
    static constexpr int H0 = kMaxContig;
    using K = bw::ChainShape<Op, TS, TC, H0, H1, kLogW, kLogE>;
    using A = typename K::A;
    using B = typename K::B;
    static cudaError_t launch(const BwChain& c, const void* in, void* out, cudaStream_t stream) {
        if constexpr (!K::kValid) {
            return cudaErrorInvalidValue;
        } else {
            if (c.n != (std::size_t{1} << (H0 + H1)) || c.chunk == 0 || c.batch == 0) return cudaErrorInvalidValue;
            auto kernel = bw::bitwise_chain_step_kernel<Op, TS, TC, H0, H1, kLogW, kLogE>;
            static KernelSetup setup;
            int grid_cap = 0;
            cudaError_t e = setup_kernel(setup, kernel, K::TPB, K::SMEM_BYTES, &grid_cap);
            if (e != cudaSuccess) return e;
            auto a_blocks = [&](std::size_t nb) {
                return (((nb * (c.n >> H0)) + A::TILES - 1) / A::TILES + K::SUB_A - 1) / K::SUB_A;
            };
            auto b_blocks = [&](std::size_t nb) {
                return (((nb * ((std::size_t{1} << H0) >> kLogW)) + B::TILES - 1) / B::TILES + K::SUB_B - 1) / K::SUB_B;
            };
            const std::size_t chunks = (c.batch + c.chunk - 1) / c.chunk;
            const std::size_t chunk_elems = c.chunk * c.n;
            const TS* src = static_cast<const TS*>(in);
            TS* dst = static_cast<TS*>(out);
            for (std::size_t k = 0; k <= chunks; ++k) {
                bw::ChainStep st{};
                st.inverse = c.inverse ? 1 : 0;
                st.scale_b = c.scale;
                st.log_inner_b = H0;
                if (k < chunks) {
                    const std::size_t nb = std::min(c.chunk, c.batch - k * c.chunk);
                    st.a_in = src + k * chunk_elems;
                    st.a_out = dst + k * chunk_elems;
                    st.a_outer = nb * (c.n >> H0);
                    st.a_blocks = static_cast<unsigned>(a_blocks(nb));
                }
                if (k > 0) {
                    const std::size_t nb = std::min(c.chunk, c.batch - (k - 1) * c.chunk);
                    st.b_buf = dst + (k - 1) * chunk_elems;
                    st.b_outer = nb;
                    st.b_blocks = static_cast<unsigned>(b_blocks(nb));
                }
                const std::size_t total = static_cast<std::size_t>(st.a_blocks) + st.b_blocks;
                if (total > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
                // a half wave ahead while both roles share a step (measured best: 737 vs 760-762 us)
                st.prefetch_stride = st.b_blocks ? static_cast<unsigned>(grid_cap / 2) : static_cast<unsigned>(grid_cap);
                if ((e = launch_dependent(kernel, static_cast<unsigned>(total), K::TPB, K::SMEM_BYTES, stream, st)) !=
                    cudaSuccess)
                    return e;
            }
            return cudaSuccess;
        }
    }
};
template <int... H>
struct Chains {
    static constexpr cudaError_t (*launch[])(const BwChain&, const void*, void*, cudaStream_t) = {
        ChainEntry<H>::launch...};
};
#if CUBF_BW_TYPE == 4
using CH = Chains<1, 2, 3, 4, 5, 6, 7, 8, 9>;
#else
using CH = Chains<1, 2, 3, 4, 5, 6, 7, 8, 9, 10>;
#endif
#endif

}  // namespace

#define CUBF_CAT2(a, b) a##b
#define CUBF_CAT(a, b) CUBF_CAT2(a, b)
#define CUBF_UNIT CUBF_CAT(CUBF_CAT(bw_unit_, CUBF_BW_OP), CUBF_CAT(_, CUBF_BW_TYPE))

// Unit entry points (named per operator/type so all units link together).
LaunchShape CUBF_CAT(CUBF_UNIT, _shape)(int log_h, int log_w) {
    if (log_w == 0 && log_h >= 1 && log_h <= kMaxContig) return C::shape[log_h - 1]();
    if (kHasStrided && log_w == kLogW && log_h >= 1 && log_h <= kMaxStrided) return T::shape[log_h - 1]();
    return {};
}

cudaError_t CUBF_CAT(CUBF_UNIT, _launch)(int log_h, int log_w, const void* in, void* out, std::size_t outer,
                                         std::size_t inner, bool inverse, float scale, int cache_mode,
                                         cudaStream_t stream) {
    if (log_w == 0 && log_h >= 1 && log_h <= kMaxContig)
        return C::launch[log_h - 1](in, out, outer, inner, inverse, scale, cache_mode, stream);
    if (kHasStrided && log_w == kLogW && log_h >= 1 && log_h <= kMaxStrided)
        return T::launch[log_h - 1](in, out, outer, inner, inverse, scale, cache_mode, stream);
    return cudaErrorInvalidValue;
}

cudaError_t CUBF_CAT(CUBF_UNIT, _chain)(const BwChain& c, const void* in, void* out, cudaStream_t stream) {
#if CUBF_BW_OP != 0
    if (c.log_h0 == kMaxContig && c.log_h1 >= 1 && c.log_h1 <= kMaxStrided)
        return CH::launch[c.log_h1 - 1](c, in, out, stream);
#else
    (void)c, (void)in, (void)out, (void)stream;
#endif
    return cudaErrorInvalidValue;
}

}  // namespace cubf
