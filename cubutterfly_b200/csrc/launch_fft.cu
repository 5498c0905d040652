// launch_fft.cu -- instantiations and launchers of the FFT kernels.
#include "fft.cuh"
#include "fft_pair.cuh"
#include "kernels.hpp"
#include "launch_util.cuh"

#include <cmath>
#include <cstdint>
#include <vector>

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

// Column-pair f32x2 kernel; its twiddle table follows the 2N floats of W_N.
template <int LOGN>
cudaError_t launch_pair(const void* in, void* out, std::size_t batch, const void* tw, bool inverse, float scale,
                        cudaStream_t stream) {
    using S = fft::PairShape<LOGN>;
    const float4* table = reinterpret_cast<const float4*>(static_cast<const float*>(tw) + 2 * S::N);
    auto kernel = fft::fft_pair_kernel<LOGN>;
    static KernelSetup setup;
    int grid_cap = 0;
    cudaError_t e = setup_kernel(setup, kernel, S::TPB, S::SMEM_BYTES, &grid_cap);
    if (e != cudaSuccess) return e;
    const std::size_t blocks = (batch + S::TPC - 1) / S::TPC;
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
    // prefetch one resident wave ahead when the grid has more than one wave
    const unsigned stride = blocks > static_cast<std::size_t>(grid_cap) ? grid_cap : 0;
    return launch_dependent(kernel, static_cast<unsigned>(blocks), S::TPB, S::SMEM_BYTES, stream,
                            static_cast<const float4*>(in), static_cast<float4*>(out), batch, table, inverse ? 1 : 0,
                            scale, stride);
}

template <int LOGN>
cudaError_t launch(const void* in, void* out, std::size_t batch, const void* tw, bool inverse, float scale,
                   cudaStream_t stream) {
    using S = fft::LocalShape<LOGN>;
    if constexpr (LOGN >= kFftPairMinLog && LOGN <= kFftPairMaxLog) {
        if (((reinterpret_cast<std::uintptr_t>(in) | reinterpret_cast<std::uintptr_t>(out)) & 15) == 0)
            return launch_pair<LOGN>(in, out, batch, tw, inverse, scale, stream);
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

using LaunchFn = cudaError_t (*)(const void*, void*, std::size_t, const void*, bool, float, cudaStream_t);
using ShapeFn = LaunchShape (*)();

template <int... L>
struct Table {
    static constexpr LaunchFn launch_fns[] = {launch<L>...};
    static constexpr ShapeFn shape_fns[] = {shape_of<L>...};
};
using Local = Table<1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13>;

template <int LOGR, int CW = 0>
struct GlobalEntry {
    using G = fft::GlobalPassShape<LOGR, CW>;
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
                              float scale, cudaStream_t stream, int log_v, int outer_shift) {
        auto kernel = fft::fft_global_pass_kernel<LOGR, CW>;
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
            static_cast<const float2*>(tw1024), 10 - LOGR, ot, conj_in ? 1 : 0, conj_out ? 1 : 0, scale, log_v,
            blocks > static_cast<std::size_t>(grid_cap) ? static_cast<unsigned>(grid_cap) : 0u, outer_shift);
        return cudaGetLastError();
    }
};
// Register-direct variants of the same pass (fft.cuh): the first pass of
// radix >= 2^8, and every pass whose Ns is at least its column count.
template <int LOGR, bool FIRST, int CW = 0>
struct RegEntry {
    using G = fft::GlobalRegShape<LOGR, CW>;
    static bool eligible(int log_n, int ns_bits, int log_v) {
        if (log_n > 31) return false;  // 32-bit offsets within a transform
        if (FIRST) return ns_bits == 0 && log_v == 0 && G::T >= 16 && log_n >= LOGR + G::LOG_C;
        return ns_bits >= G::LOG_C && log_n >= ns_bits + LOGR;
    }
    static cudaError_t launch(const void* src, void* dst, int log_n, int ns_bits, std::size_t batch,
                              const void* tw1024, const FftOuterTables& outer, bool conj_in, bool conj_out,
                              float scale, cudaStream_t stream, int log_v, int outer_shift) {
        const std::size_t blocks = batch * ((std::size_t{1} << (log_n - LOGR)) >> G::LOG_C);
        return run(src, dst, log_n, ns_bits, blocks, tw1024, outer, conj_in, conj_out, scale, stream, log_v,
                   outer_shift, fft::RegChunk{0, 0, 0, 0, 0});
    }
    // `blocks` tiles of the pass (the chained plans run their chunks through
    // the chain-step kernel of csrc/fft_chain.cu instead)
    static cudaError_t run(const void* src, void* dst, int log_n, int ns_bits, std::size_t blocks,
                           const void* tw1024, const FftOuterTables& outer, bool conj_in, bool conj_out, float scale,
                           cudaStream_t stream, int log_v, int outer_shift, const fft::RegChunk& chunk) {
        if constexpr (FIRST && G::T < 16) {
            return cudaErrorInvalidValue;  // never eligible: runs of T < 16 values
        } else {
        auto kernel = fft::fft_global_reg_kernel<LOGR, FIRST, CW, false>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, G::TPB, G::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        if (blocks == 0) return cudaSuccess;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        fft::OuterTwiddles ot{static_cast<const double2*>(outer.lo), static_cast<const double2*>(outer.hi),
                              outer.split};
        const unsigned prefetch = blocks > static_cast<std::size_t>(grid_cap) ? static_cast<unsigned>(grid_cap) : 0u;
        return launch_dependent(kernel, static_cast<unsigned>(blocks), G::TPB, G::SMEM_BYTES, stream,
                                static_cast<const float2*>(src), static_cast<float2*>(dst), log_n, ns_bits,
                                static_cast<const float2*>(tw1024), ot, conj_in ? 1 : 0, conj_out ? 1 : 0, scale,
                                log_v, prefetch, outer_shift, chunk);
        }
    }
    static LaunchShape shape() {
        LaunchShape s;
        s.threads = G::TPB;
        s.smem_bytes = G::SMEM_BYTES;
        s.units_per_cta = G::C;
        s.elems_per_thread = G::S::E;
        s.exchanges = G::S::NPASS - 1;
        return s;
    }
};

using GlobalLaunch = cudaError_t (*)(const void*, void*, int, int, std::size_t, const void*, const FftOuterTables&,
                                     bool, bool, float, cudaStream_t, int, int);
using GlobalShape = LaunchShape (*)();
template <int... L>
struct GlobalTable {
    static constexpr GlobalLaunch launch_fns[] = {GlobalEntry<L>::launch...};
    static constexpr GlobalShape shape_fns[] = {GlobalEntry<L>::shape...};
};
using Global = GlobalTable<4, 5, 6, 7, 8, 9, 10>;
template <int... L>
struct RegTable {
    static constexpr bool (*first_ok[])(int, int, int) = {RegEntry<L, true>::eligible...};
    static constexpr bool (*later_ok[])(int, int, int) = {RegEntry<L, false>::eligible...};
    static constexpr GlobalLaunch first_fns[] = {RegEntry<L, true>::launch...};
    static constexpr GlobalLaunch later_fns[] = {RegEntry<L, false>::launch...};
};
using Reg = RegTable<4, 5, 6, 7, 8, 9, 10>;
// 32-column variants (256-byte runs) of radix 2^6..2^8, for arrays far larger
// than L2 (2^26 values and more): measured on 2^30 points (8+8+7+7) 12.3 ms against 14.6 ms
// with 16 columns, on 2^24 points 3 % slower
template <int... L>
struct RegWideTable {
    static constexpr bool (*first_ok[])(int, int, int) = {RegEntry<L, true, 32>::eligible...};
    static constexpr bool (*later_ok[])(int, int, int) = {RegEntry<L, false, 32>::eligible...};
    static constexpr GlobalLaunch first_fns[] = {RegEntry<L, true, 32>::launch...};
    static constexpr GlobalLaunch later_fns[] = {RegEntry<L, false, 32>::launch...};
};
using RegWide = RegWideTable<6, 7, 8>;
constexpr int kRegWideMinLog = 26;

// 8-column variants of the large radices (64-byte runs, two CTAs per SM at 2^10)
template <int... L>
struct NarrowTable {
    static constexpr GlobalLaunch launch_fns[] = {GlobalEntry<L, kFftBlockChunk>::launch...};
    static constexpr GlobalShape shape_fns[] = {GlobalEntry<L, kFftBlockChunk>::shape...};
};
using Narrow = NarrowTable<8, 9, 10>;

template <int LOGR>
struct DeinterleaveEntry {
    using G = fft::GlobalPassShape<LOGR, kFftBlockChunk>;
    static LaunchShape shape() { return GlobalEntry<LOGR, kFftBlockChunk>::shape(); }
    static cudaError_t launch(const void* src, void* dst, int log_len, int log_v, std::size_t m0,
                              const void* tw1024, bool conj_in, cudaStream_t stream) {
        auto kernel = fft::fft_deinterleave_pass_kernel<LOGR, kFftBlockChunk>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, G::TPB, G::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        if (log_len < LOGR || log_v < 3) return cudaErrorInvalidValue;
        const std::size_t blocks = std::size_t{1} << (log_len - LOGR);
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        kernel<<<static_cast<unsigned>(blocks), G::TPB, G::SMEM_BYTES, stream>>>(
            static_cast<const float2*>(src), static_cast<float2*>(dst), log_len, log_v, m0,
            static_cast<const float2*>(tw1024), 10 - LOGR, conj_in ? 1 : 0);
        return cudaGetLastError();
    }
};
template <int... L>
struct DeinterleaveTable {
    static constexpr cudaError_t (*launch_fns[])(const void*, void*, int, int, std::size_t, const void*, bool,
                                                 cudaStream_t) = {DeinterleaveEntry<L>::launch...};
    static constexpr GlobalShape shape_fns[] = {DeinterleaveEntry<L>::shape...};
};
using Deinterleave = DeinterleaveTable<8, 9, 10>;

}  // namespace

LaunchShape fft_global_pass_shape(int log_r) {
    if (log_r < kFftPassMinLog || log_r > kFftPassMaxLog) return {};
    return Global::shape_fns[log_r - kFftPassMinLog]();
}

cudaError_t launch_fft_global_pass(int log_r, const void* src, void* dst, int log_n, int ns_bits,
                                   std::size_t batch, const void* tw1024, const FftOuterTables& outer, bool conj_in,
                                   bool conj_out, float scale, cudaStream_t stream, int log_v, int outer_shift,
                                   bool narrow) {
    if (log_r < kFftPassMinLog || log_r > kFftPassMaxLog) return cudaErrorInvalidValue;
    if (log_v < 0 || log_v > log_n - log_r || outer_shift < 0) return cudaErrorInvalidValue;
    if (narrow) {
        if (!fft_global_pass_narrow_available(log_r)) return cudaErrorInvalidValue;
        return Narrow::launch_fns[log_r - 8](src, dst, log_n, ns_bits, batch, tw1024, outer, conj_in, conj_out, scale,
                                             stream, log_v, outer_shift);
    }
    const int i = log_r - kFftPassMinLog;
    if (log_n <= 31 && (batch << log_n) >= (std::size_t{1} << kRegWideMinLog) && log_r >= 6 && log_r <= 8) {
        const int k = log_r - 6;
        if (RegWide::first_ok[k](log_n, ns_bits, log_v))
            return RegWide::first_fns[k](src, dst, log_n, ns_bits, batch, tw1024, outer, conj_in, conj_out, scale,
                                         stream, log_v, outer_shift);
        if (RegWide::later_ok[k](log_n, ns_bits, log_v))
            return RegWide::later_fns[k](src, dst, log_n, ns_bits, batch, tw1024, outer, conj_in, conj_out, scale,
                                         stream, log_v, outer_shift);
    }
    if (Reg::first_ok[i](log_n, ns_bits, log_v))
        return Reg::first_fns[i](src, dst, log_n, ns_bits, batch, tw1024, outer, conj_in, conj_out, scale, stream,
                                 log_v, outer_shift);
    if (Reg::later_ok[i](log_n, ns_bits, log_v))
        return Reg::later_fns[i](src, dst, log_n, ns_bits, batch, tw1024, outer, conj_in, conj_out, scale, stream,
                                 log_v, outer_shift);
    return Global::launch_fns[i](src, dst, log_n, ns_bits, batch, tw1024, outer, conj_in, conj_out, scale, stream,
                                 log_v, outer_shift);
}

bool fft_chain_pass_available(int log_r) { return log_r >= kFftChainMinLog && log_r <= kFftChainMaxLog; }

bool fft_global_pass_narrow_available(int log_r) { return log_r >= 8 && log_r <= kFftPassMaxLog; }

LaunchShape fft_global_pass_narrow_shape(int log_r) {
    return fft_global_pass_narrow_available(log_r) ? Narrow::shape_fns[log_r - 8]() : LaunchShape{};
}

LaunchShape fft_deinterleave_shape(int log_r) {
    if (log_r < kFftDeinterleaveMinLog || log_r > kFftPassMaxLog) return {};
    return Deinterleave::shape_fns[log_r - kFftDeinterleaveMinLog]();
}

cudaError_t launch_fft_deinterleave_pass(int log_r, const void* src, void* dst, int log_len, int log_v,
                                         std::size_t m0, const void* tw1024, bool conj_in, cudaStream_t stream) {
    if (log_r < kFftDeinterleaveMinLog || log_r > kFftPassMaxLog) return cudaErrorInvalidValue;
    return Deinterleave::launch_fns[log_r - kFftDeinterleaveMinLog](src, dst, log_len, log_v, m0, tw1024, conj_in,
                                                                    stream);
}

std::vector<float> fft_local_twiddles(int log_n) {
    constexpr double kPi = 3.141592653589793238462643383279502884;
    const std::size_t n = std::size_t{1} << log_n;
    std::vector<float> tw(2 * n);
    for (std::size_t k = 0; k < n; ++k) {
        // exp(-2 pi i k / N) in double, rounded once (reference butterfly.cu:1502-1514)
        const double a = -2.0 * kPi * static_cast<double>(k) / static_cast<double>(n);
        tw[2 * k] = static_cast<float>(std::cos(a));
        tw[2 * k + 1] = static_cast<float>(std::sin(a));
    }
    if (log_n >= kFftPairMinLog && log_n <= kFftPairMaxLog) {
        // column-pair table: pass p >= 1, radix index r in [1, R), column pair
        // jp < NS/2 -> (re, re, im, im) of W_{NS R}^{c r} for columns c = 2jp, 2jp+1
        const int npass = (log_n + 3) / 4;
        int ns_bits = 0;
        for (int p = 0; p < npass; ++p) {
            const int rb = log_n / npass + (p < log_n % npass ? 1 : 0);
            if (p > 0) {
                const std::size_t ns = std::size_t{1} << ns_bits, len = ns << rb;
                for (std::size_t r = 1; r < (std::size_t{1} << rb); ++r)
                    for (std::size_t jp = 0; jp < ns / 2; ++jp) {
                        const double a0 = -2.0 * kPi * static_cast<double>((2 * jp * r) % len) / len;
                        const double a1 = -2.0 * kPi * static_cast<double>(((2 * jp + 1) * r) % len) / len;
                        tw.push_back(static_cast<float>(std::cos(a0)));
                        tw.push_back(static_cast<float>(std::cos(a1)));
                        tw.push_back(static_cast<float>(std::sin(a0)));
                        tw.push_back(static_cast<float>(std::sin(a1)));
                    }
            }
            ns_bits += rb;
        }
    }
    return tw;
}

LaunchShape fft_local_shape(int log_n) {
    if (log_n < 1 || log_n > kFftLocalMaxLog) return {};
    return Local::shape_fns[log_n - 1]();
}

cudaError_t launch_fft_local(int log_n, const void* in, void* out, std::size_t batch, const void* twiddles,
                             bool inverse, float scale, cudaStream_t stream) {
    if (log_n < 1 || log_n > kFftLocalMaxLog) return cudaErrorInvalidValue;
    return Local::launch_fns[log_n - 1](in, out, batch, twiddles, inverse, scale, stream);
}

}  // namespace cubf
