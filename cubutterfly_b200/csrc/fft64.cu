// fft64.cu -- complex fp64 FFT, radix 2 (the reference's numeric FP64 plans;
// arithmetic of cuntt::reference_fft<Complex64>, src/butterfly_reference.cpp:435-473).
//
// The input is bit-reversal permuted (bitrev.cu), then stage s (half = 2^s)
// combines a = x[base + o], b = x[base + half + o] into a + w b, a - w b with
// w = exp(-+ pi i o / half), taken from a per-plan table of W_N^k computed in
// double with the same angle rounding (k = o N / (2 half)).  Products and sums
// round separately in the reference's order, so results are bit-identical to
// it.  The low min(L, 11) stages run in one shared-memory tile pass over
// 2^11-point blocks; each higher stage is one in-place pass; a normalised
// inverse scales by 1/N (exact) in the last pass.
#include "kernels.hpp"

#include <cuda_runtime.h>

namespace cubf {
namespace {

constexpr int kThreads = 256;
constexpr int kTileLog = 11;

__device__ __forceinline__ void butterfly(double2& a, double2& b, double2 w, double scale) {
    const double vr = __dsub_rn(__dmul_rn(b.x, w.x), __dmul_rn(b.y, w.y));
    const double vi = __dadd_rn(__dmul_rn(b.x, w.y), __dmul_rn(b.y, w.x));
    const double2 x = a;
    a = make_double2(__dmul_rn(__dadd_rn(x.x, vr), scale), __dmul_rn(__dadd_rn(x.y, vi), scale));
    b = make_double2(__dmul_rn(__dsub_rn(x.x, vr), scale), __dmul_rn(__dsub_rn(x.y, vi), scale));
}

// Stages 0 .. tile_log - 1 of consecutive 2^tile_log-point blocks (in place).
__global__ void __launch_bounds__(kThreads)
    fft64_tile_kernel(double2* data, const double2* __restrict__ tw, int log_n, int tile_log, double last_scale) {
    extern __shared__ __align__(16) unsigned char raw[];
    double2* tile = reinterpret_cast<double2*>(raw);
    const size_t n = size_t{1} << tile_log;
    double2* block = data + static_cast<size_t>(blockIdx.x) * n;
    for (size_t i = threadIdx.x; i < n; i += kThreads) tile[i] = block[i];
    __syncthreads();
    for (int s = 0; s < tile_log; ++s) {
        const size_t half = size_t{1} << s;
        const double scale = s + 1 == log_n ? last_scale : 1.0;
        for (size_t p = threadIdx.x; p < n / 2; p += kThreads) {
            const size_t o = p & (half - 1);
            const size_t lo = ((p >> s) << (s + 1)) | o;
            butterfly(tile[lo], tile[lo + half], __ldg(tw + (o << (log_n - 1 - s))), scale);
        }
        __syncthreads();
    }
    for (size_t i = threadIdx.x; i < n; i += kThreads) block[i] = tile[i];
}

__global__ void __launch_bounds__(kThreads)
    fft64_stage_kernel(double2* data, const double2* __restrict__ tw, int log_n, int s, size_t pairs, double scale) {
    const size_t half = size_t{1} << s;
    for (size_t p = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; p < pairs;
         p += static_cast<size_t>(gridDim.x) * kThreads) {
        const size_t o = p & (half - 1);
        const size_t lo = ((p >> s) << (s + 1)) | o;
        butterfly(data[lo], data[lo + half], __ldg(tw + (o << (log_n - 1 - s))), scale);
    }
}

}  // namespace

cudaError_t launch_fft64(int log_n, const void* in, void* out, std::size_t batch, const void* twiddles,
                         double scale, cudaStream_t stream) {
    if (log_n < 1 || log_n > 30) return cudaErrorInvalidValue;
    cudaError_t e = launch_bitrev(16, log_n, in, out, batch, stream);
    if (e != cudaSuccess) return e;
    double2* data = static_cast<double2*>(out);
    const double2* tw = static_cast<const double2*>(twiddles);
    const int tile_log = log_n < kTileLog ? log_n : kTileLog;
    const std::size_t blocks = batch << (log_n - tile_log);
    if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
    const int smem = 16 << tile_log;
    fft64_tile_kernel<<<static_cast<unsigned>(blocks), kThreads, smem, stream>>>(data, tw, log_n, tile_log, scale);
    e = cudaGetLastError();
    const std::size_t pairs = (batch << log_n) / 2;
    std::size_t grid = (pairs + kThreads - 1) / kThreads;
    if (grid > 148 * 32) grid = 148 * 32;
    for (int s = tile_log; s < log_n && e == cudaSuccess; ++s) {
        fft64_stage_kernel<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(data, tw, log_n, s, pairs,
                                                                               s + 1 == log_n ? scale : 1.0);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace cubf
