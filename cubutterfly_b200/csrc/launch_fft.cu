// launch_fft.cu -- instantiations and launchers of the FFT kernels.
#include "fft.cuh"
#include "kernels.hpp"

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

template <int LOGN>
cudaError_t launch(const void* in, void* out, std::size_t batch, const void* tw, bool inverse, float scale,
                   cudaStream_t stream) {
    using S = fft::LocalShape<LOGN>;
    auto kernel = fft::fft_local_kernel<LOGN>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured = true;
    }
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

}  // namespace

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
