// launch_fft.cu -- instantiations and launchers of the FFT kernels.
#include "fft.cuh"
#include "kernels.hpp"
#include "launch_util.cuh"

#include <cstdint>

namespace cubf {
namespace {

template <int LOGN>
LaunchShape shape_of() {
    using S = fft::LocalShape<LOGN>;
    LaunchShape s;
    s.threads = S::TPB;
    s.smem_bytes = S::SMEM_BYTES;
    s.units_per_cta = S::TPC;
    s.elems_per_thread = S::E;
    s.exchanges = S::NPASS - 1;
    return s;
}

constexpr int kStages = 2;

// Persistent TMA-pipelined variant for rows of at least 2 KB (LOGN >= 8).
template <int LOGN>
cudaError_t launch_tma(const void* in, void* out, std::size_t batch, const void* tw, bool inverse, float scale,
                       cudaStream_t stream, unsigned* err) {
    using S = fft::LocalShape<LOGN>;
    using T = fft::TmaShape<LOGN, kStages>;
    auto kernel = fft::fft_tma_kernel<LOGN, kStages>;
    static KernelSetup setup;
    int grid_cap = 0;
    cudaError_t e = setup_kernel(setup, kernel, S::TPB, T::SMEM_BYTES, &grid_cap);
    if (e != cudaSuccess) return e;
    const std::size_t tiles = (batch + S::TPC - 1) / S::TPC;
    if (tiles == 0) return cudaSuccess;
    const unsigned grid = static_cast<unsigned>(tiles < static_cast<std::size_t>(grid_cap) ? tiles : grid_cap);
    kernel<<<grid, S::TPB, T::SMEM_BYTES, stream>>>(static_cast<const float2*>(in), static_cast<float2*>(out), batch,
                                                    static_cast<const float2*>(tw), inverse ? 1 : 0, scale, err);
    return cudaGetLastError();
}

template <int LOGN>
cudaError_t launch(const void* in, void* out, std::size_t batch, const void* tw, bool inverse, float scale,
                   cudaStream_t stream, unsigned* err) {
    using S = fft::LocalShape<LOGN>;
    if constexpr (LOGN >= 8 && LOGN <= 12) {
        // bulk copies need 16-byte aligned rows (always: N * 8 bytes, N >= 2)
        if ((reinterpret_cast<std::uintptr_t>(in) & 15) == 0)
            return launch_tma<LOGN>(in, out, batch, tw, inverse, scale, stream, err);
    }
    auto kernel = fft::fft_local_kernel<LOGN>;
    static KernelSetup setup;
    int grid_cap = 0;
    cudaError_t e = setup_kernel(setup, kernel, S::TPB, S::SMEM_BYTES, &grid_cap);
    if (e != cudaSuccess) return e;
    const std::size_t blocks = (batch + S::TPC - 1) / S::TPC;
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
    kernel<<<static_cast<unsigned>(blocks), S::TPB, S::SMEM_BYTES, stream>>>(
        static_cast<const float2*>(in), static_cast<float2*>(out), batch, static_cast<const float2*>(tw),
        inverse ? 1 : 0, scale);
    return cudaGetLastError();
}

using LaunchFn = cudaError_t (*)(const void*, void*, std::size_t, const void*, bool, float, cudaStream_t, unsigned*);
using ShapeFn = LaunchShape (*)();

template <int... L>
struct Table {
    static constexpr LaunchFn launch_fns[] = {launch<L>...};
    static constexpr ShapeFn shape_fns[] = {shape_of<L>...};
};
using Local = Table<1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13>;

template <int LOGR>
struct GlobalEntry {
    using G = fft::GlobalPassShape<LOGR>;
    static LaunchShape shape() {
        LaunchShape s;
        s.threads = G::TPB;
        s.smem_bytes = G::SMEM_BYTES;
        s.units_per_cta = G::C;
        s.elems_per_thread = G::S::E;
        s.exchanges = G::S::NPASS + 1;
        return s;
    }
    static cudaError_t launch(const void* src, void* dst, int log_n, int ns_bits, std::size_t batch,
                              const void* tw1024, const FftOuterTables& outer, bool conj_in, bool conj_out,
                              float scale, cudaStream_t stream) {
        auto kernel = fft::fft_global_pass_kernel<LOGR>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, G::TPB, G::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        if (log_n < LOGR || ((std::size_t{1} << (log_n - LOGR)) % G::C) != 0) return cudaErrorInvalidValue;
        const std::size_t blocks = batch * ((std::size_t{1} << (log_n - LOGR)) / G::C);
        if (blocks == 0) return cudaSuccess;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        fft::OuterTwiddles ot{static_cast<const double2*>(outer.lo), static_cast<const double2*>(outer.hi),
                              outer.split};
        kernel<<<static_cast<unsigned>(blocks), G::TPB, G::SMEM_BYTES, stream>>>(
            static_cast<const float2*>(src), static_cast<float2*>(dst), log_n, ns_bits, batch,
            static_cast<const float2*>(tw1024), 10 - LOGR, ot, conj_in ? 1 : 0, conj_out ? 1 : 0, scale);
        return cudaGetLastError();
    }
};
using GlobalLaunch = cudaError_t (*)(const void*, void*, int, int, std::size_t, const void*, const FftOuterTables&,
                                     bool, bool, float, cudaStream_t);
using GlobalShape = LaunchShape (*)();
template <int... L>
struct GlobalTable {
    static constexpr GlobalLaunch launch_fns[] = {GlobalEntry<L>::launch...};
    static constexpr GlobalShape shape_fns[] = {GlobalEntry<L>::shape...};
};
using Global = GlobalTable<4, 5, 6, 7, 8, 9, 10>;

}  // namespace

LaunchShape fft_global_pass_shape(int log_r) {
    if (log_r < kFftPassMinLog || log_r > kFftPassMaxLog) return {};
    return Global::shape_fns[log_r - kFftPassMinLog]();
}

cudaError_t launch_fft_global_pass(int log_r, const void* src, void* dst, int log_n, int ns_bits,
                                   std::size_t batch, const void* tw1024, const FftOuterTables& outer, bool conj_in,
                                   bool conj_out, float scale, cudaStream_t stream) {
    if (log_r < kFftPassMinLog || log_r > kFftPassMaxLog) return cudaErrorInvalidValue;
    return Global::launch_fns[log_r - kFftPassMinLog](src, dst, log_n, ns_bits, batch, tw1024, outer, conj_in,
                                                      conj_out, scale, stream);
}

LaunchShape fft_local_shape(int log_n) {
    if (log_n < 1 || log_n > kFftLocalMaxLog) return {};
    return Local::shape_fns[log_n - 1]();
}

cudaError_t launch_fft_local(int log_n, const void* in, void* out, std::size_t batch, const void* twiddles,
                             bool inverse, float scale, cudaStream_t stream, unsigned* err) {
    if (log_n < 1 || log_n > kFftLocalMaxLog) return cudaErrorInvalidValue;
    return Local::launch_fns[log_n - 1](in, out, batch, twiddles, inverse, scale, stream, err);
}

}  // namespace cubf
