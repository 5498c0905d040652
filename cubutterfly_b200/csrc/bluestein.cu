// bluestein.cu -- arbitrary-length complex FFT as a power-of-two convolution.
//
// With nk = (n^2 + k^2 - (k - n)^2) / 2 the length-N DFT becomes
//   X[k] = c[k] * sum_n (x[n] c[n]) conj(c[k - n]),   c[j] = exp(s i pi j^2 / N),
// s = -1 forward, +1 inverse: a linear convolution of a[n] = x[n] c[n] with
// b[j] = conj(c[j]), |j| < N.  It runs as a cyclic convolution of M >= 2N - 1
// points (M a power of two): a zero-padded to M, b wrapped (b[M - j] = b[j]),
//   X = c * IDFT_M( DFT_M(a) * DFT_M(b) ) / M.
// DFT_M(b) / M (and 1/N for a normalised inverse) is computed once per plan in
// fp64; the two M-point transforms are the library's own power-of-two FFT
// plans, in place in the workspace.  Chirp angles reduce j^2 mod 2N in
// integers, so pi (j^2 mod 2N) / N stays in [0, 2 pi) for every length.
//
// The NTT of any length N (u64 words, prime q with 2N | q - 1 and M | q - 1)
// is the same identity over Z_q with psi a primitive 2N-th root in place of
// exp(-i pi / N): c[j] = psi^(j^2 mod 2N), b[j] = c[j]^-1, and
// X[k] = c[k] sum_n x[n] c[n] b[k - n] = sum_n x[n] (psi^2)^(nk) exactly; the
// M-point cyclic convolution runs on the library's power-of-two NTT plans
// (natural -> bit-reversed forward, bit-reversed -> natural inverse with
// 1/M, so the product needs no reordering).
#include "kernels.hpp"

#include <cuda_runtime.h>

namespace cubf {
namespace {

constexpr int kThreads = 256;

template <typename T2>
struct Complex;
template <>
struct Complex<float2> {
    static __device__ __forceinline__ float2 mul(float2 a, float2 b) {
        return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
    }
    static __device__ __forceinline__ float2 from(double2 v) {
        return make_float2(static_cast<float>(v.x), static_cast<float>(v.y));
    }
    static __device__ __forceinline__ float2 zero() { return make_float2(0.f, 0.f); }
};
template <>
struct Complex<double2> {
    static __device__ __forceinline__ double2 mul(double2 a, double2 b) {
        return make_double2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
    }
    static __device__ __forceinline__ double2 from(double2 v) { return v; }
    static __device__ __forceinline__ double2 zero() { return make_double2(0.0, 0.0); }
};

unsigned grid_for(std::size_t count) {
    const std::size_t blocks = (count + kThreads - 1) / kThreads;
    return static_cast<unsigned>(blocks < 148u * 32u ? blocks : 148u * 32u);
}

// exp(sign i pi (j^2 mod 2N) / N) in fp64
__device__ __forceinline__ double2 chirp(std::size_t j, std::size_t n, double sign) {
    const unsigned long long r = static_cast<unsigned long long>((static_cast<unsigned __int128>(j) * j) % (2 * n));
    double s, c;
    sincospi(static_cast<double>(r) / static_cast<double>(n), &s, &c);
    return make_double2(c, sign * s);
}

// chirp table c[j], j < n
template <typename T2>
__global__ void __launch_bounds__(kThreads) chirp_table_kernel(T2* table, std::size_t n, double sign) {
    for (std::size_t j = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; j < n;
         j += static_cast<std::size_t>(gridDim.x) * kThreads)
        table[j] = Complex<T2>::from(chirp(j, n, sign));
}

// the wrapped convolution kernel b (fp64): conj(c[j]) at j and M - j for j < n, zero elsewhere
__global__ void __launch_bounds__(kThreads) kernel_taps_kernel(double2* b, std::size_t n, std::size_t m, double sign) {
    for (std::size_t j = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; j < m;
         j += static_cast<std::size_t>(gridDim.x) * kThreads) {
        const std::size_t t = j < n ? j : (m - j < n ? m - j : m);
        b[j] = t < m ? chirp(t, n, -sign) : make_double2(0.0, 0.0);
    }
}

// spectrum = B * scale, rounded once to the storage precision
template <typename T2>
__global__ void __launch_bounds__(kThreads) scale_spectrum_kernel(const double2* bd, T2* spectrum, std::size_t m,
                                                                  double scale) {
    for (std::size_t j = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; j < m;
         j += static_cast<std::size_t>(gridDim.x) * kThreads)
        spectrum[j] = Complex<T2>::from(make_double2(bd[j].x * scale, bd[j].y * scale));
}

// work[b][j] = x[b][j] c[j] (j < n), 0 (n <= j < M)
template <typename T2>
__global__ void __launch_bounds__(kThreads)
    pack_kernel(const T2* in, std::size_t is, std::size_t ibs, T2* work, const T2* table, std::size_t n, std::size_t m,
                std::size_t batch) {
    const std::size_t total = m * batch;
    for (std::size_t idx = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<std::size_t>(gridDim.x) * kThreads) {
        const std::size_t b = idx / m, j = idx - b * m;
        work[idx] = j < n ? Complex<T2>::mul(in[b * ibs + j * is], table[j]) : Complex<T2>::zero();
    }
}

// work[b][k] *= spectrum[k]
template <typename T2>
__global__ void __launch_bounds__(kThreads) multiply_kernel(T2* work, const T2* spectrum, std::size_t m,
                                                            std::size_t batch) {
    const std::size_t total = m * batch;
    for (std::size_t idx = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<std::size_t>(gridDim.x) * kThreads)
        work[idx] = Complex<T2>::mul(work[idx], spectrum[idx & (m - 1)]);
}

// out[b][k] = work[b][k] c[k], k < n
template <typename T2>
__global__ void __launch_bounds__(kThreads)
    unpack_kernel(const T2* work, T2* out, std::size_t os, std::size_t obs, const T2* table, std::size_t n,
                  std::size_t m, std::size_t batch) {
    const std::size_t total = n * batch;
    for (std::size_t idx = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<std::size_t>(gridDim.x) * kThreads) {
        const std::size_t b = idx / n, k = idx - b * n;
        out[b * obs + k * os] = Complex<T2>::mul(work[b * m + k], table[k]);
    }
}

// ---- NTT (u64 words, prime q < 2^63) ----------------------------------------
// Shoup product a w mod q for any 64-bit a and w < q (wq = floor(w 2^64 / q)):
// the remainder estimate lies in [0, 2q).
__device__ __forceinline__ std::uint64_t mul_shoup(std::uint64_t a, std::uint64_t w, std::uint64_t wq,
                                                   std::uint64_t q) {
    const std::uint64_t r = a * w - __umul64hi(a, wq) * q;
    return r >= q ? r - q : r;
}

// work[b][j] = (x[b][j] mod q) c[j] (j < n), 0 (n <= j < M)
__global__ void __launch_bounds__(kThreads)
    ntt_pack_kernel(const std::uint64_t* in, std::size_t is, std::size_t ibs, std::uint64_t* work,
                    const std::uint64_t* chirp, const std::uint64_t* chirp_q, std::size_t n, std::size_t m,
                    std::size_t batch, std::uint64_t q, std::uint64_t unit_q) {
    const std::size_t total = m * batch;
    for (std::size_t idx = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<std::size_t>(gridDim.x) * kThreads) {
        const std::size_t b = idx / m, j = idx - b * m;
        std::uint64_t v = 0;
        if (j < n) v = mul_shoup(mul_shoup(in[b * ibs + j * is], 1, unit_q, q), chirp[j], chirp_q[j], q);
        work[idx] = v;
    }
}

__global__ void __launch_bounds__(kThreads)
    ntt_multiply_kernel(std::uint64_t* work, const std::uint64_t* spectrum, const std::uint64_t* spectrum_q,
                        std::size_t m, std::size_t batch, std::uint64_t q) {
    const std::size_t total = m * batch;
    for (std::size_t idx = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<std::size_t>(gridDim.x) * kThreads) {
        const std::size_t k = idx & (m - 1);
        work[idx] = mul_shoup(work[idx], spectrum[k], spectrum_q[k], q);
    }
}

__global__ void __launch_bounds__(kThreads)
    ntt_unpack_kernel(const std::uint64_t* work, std::uint64_t* out, std::size_t os, std::size_t obs,
                      const std::uint64_t* chirp, const std::uint64_t* chirp_q, std::size_t n, std::size_t m,
                      std::size_t batch, std::uint64_t q) {
    const std::size_t total = n * batch;
    for (std::size_t idx = static_cast<std::size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<std::size_t>(gridDim.x) * kThreads) {
        const std::size_t b = idx / n, k = idx - b * n;
        out[b * obs + k * os] = mul_shoup(work[b * m + k], chirp[k], chirp_q[k], q);
    }
}

}  // namespace

cudaError_t launch_bluestein_ntt_pack(const void* in, std::size_t is, std::size_t ibs, void* work, const void* chirp,
                                      const void* chirp_q, std::size_t n, std::size_t m, std::size_t batch,
                                      std::uint64_t q, std::uint64_t unit_q, cudaStream_t stream) {
    ntt_pack_kernel<<<grid_for(m * batch), kThreads, 0, stream>>>(
        static_cast<const std::uint64_t*>(in), is, ibs, static_cast<std::uint64_t*>(work),
        static_cast<const std::uint64_t*>(chirp), static_cast<const std::uint64_t*>(chirp_q), n, m, batch, q, unit_q);
    return cudaGetLastError();
}

cudaError_t launch_bluestein_ntt_multiply(void* work, const void* spectrum, const void* spectrum_q, std::size_t m,
                                          std::size_t batch, std::uint64_t q, cudaStream_t stream) {
    ntt_multiply_kernel<<<grid_for(m * batch), kThreads, 0, stream>>>(
        static_cast<std::uint64_t*>(work), static_cast<const std::uint64_t*>(spectrum),
        static_cast<const std::uint64_t*>(spectrum_q), m, batch, q);
    return cudaGetLastError();
}

cudaError_t launch_bluestein_ntt_unpack(const void* work, void* out, std::size_t os, std::size_t obs,
                                        const void* chirp, const void* chirp_q, std::size_t n, std::size_t m,
                                        std::size_t batch, std::uint64_t q, cudaStream_t stream) {
    ntt_unpack_kernel<<<grid_for(n * batch), kThreads, 0, stream>>>(
        static_cast<const std::uint64_t*>(work), static_cast<std::uint64_t*>(out), os, obs,
        static_cast<const std::uint64_t*>(chirp), static_cast<const std::uint64_t*>(chirp_q), n, m, batch, q);
    return cudaGetLastError();
}

cudaError_t launch_bluestein_tables(bool f64, std::size_t n, std::size_t m, bool inverse, void* chirp_table,
                                    void* taps, cudaStream_t stream) {
    const double sign = inverse ? 1.0 : -1.0;
    if (f64)
        chirp_table_kernel<double2><<<grid_for(n), kThreads, 0, stream>>>(static_cast<double2*>(chirp_table), n, sign);
    else
        chirp_table_kernel<float2><<<grid_for(n), kThreads, 0, stream>>>(static_cast<float2*>(chirp_table), n, sign);
    kernel_taps_kernel<<<grid_for(m), kThreads, 0, stream>>>(static_cast<double2*>(taps), n, m, sign);
    return cudaGetLastError();
}

cudaError_t launch_bluestein_spectrum(bool f64, const void* taps_spectrum, void* spectrum, std::size_t m,
                                      double scale, cudaStream_t stream) {
    const auto* bd = static_cast<const double2*>(taps_spectrum);
    if (f64)
        scale_spectrum_kernel<double2><<<grid_for(m), kThreads, 0, stream>>>(bd, static_cast<double2*>(spectrum), m,
                                                                              scale);
    else
        scale_spectrum_kernel<float2><<<grid_for(m), kThreads, 0, stream>>>(bd, static_cast<float2*>(spectrum), m,
                                                                            scale);
    return cudaGetLastError();
}

cudaError_t launch_bluestein_pack(bool f64, const void* in, std::size_t is, std::size_t ibs, void* work,
                                  const void* chirp_table, std::size_t n, std::size_t m, std::size_t batch,
                                  cudaStream_t stream) {
    if (f64)
        pack_kernel<double2><<<grid_for(m * batch), kThreads, 0, stream>>>(
            static_cast<const double2*>(in), is, ibs, static_cast<double2*>(work),
            static_cast<const double2*>(chirp_table), n, m, batch);
    else
        pack_kernel<float2><<<grid_for(m * batch), kThreads, 0, stream>>>(
            static_cast<const float2*>(in), is, ibs, static_cast<float2*>(work),
            static_cast<const float2*>(chirp_table), n, m, batch);
    return cudaGetLastError();
}

cudaError_t launch_bluestein_multiply(bool f64, void* work, const void* spectrum, std::size_t m, std::size_t batch,
                                      cudaStream_t stream) {
    if (f64)
        multiply_kernel<double2><<<grid_for(m * batch), kThreads, 0, stream>>>(
            static_cast<double2*>(work), static_cast<const double2*>(spectrum), m, batch);
    else
        multiply_kernel<float2><<<grid_for(m * batch), kThreads, 0, stream>>>(
            static_cast<float2*>(work), static_cast<const float2*>(spectrum), m, batch);
    return cudaGetLastError();
}

cudaError_t launch_bluestein_unpack(bool f64, const void* work, void* out, std::size_t os, std::size_t obs,
                                    const void* chirp_table, std::size_t n, std::size_t m, std::size_t batch,
                                    cudaStream_t stream) {
    if (f64)
        unpack_kernel<double2><<<grid_for(n * batch), kThreads, 0, stream>>>(
            static_cast<const double2*>(work), static_cast<double2*>(out), os, obs,
            static_cast<const double2*>(chirp_table), n, m, batch);
    else
        unpack_kernel<float2><<<grid_for(n * batch), kThreads, 0, stream>>>(
            static_cast<const float2*>(work), static_cast<float2*>(out), os, obs,
            static_cast<const float2*>(chirp_table), n, m, batch);
    return cudaGetLastError();
}

}  // namespace cubf
