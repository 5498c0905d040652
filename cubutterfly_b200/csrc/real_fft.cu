// real_fft.cu -- R2C / C2R on top of an N/2-point complex FFT.
//
// A real signal x of N points read as N/2 complex values z[n] = x[2n] + i x[2n+1]
// has Z = DFT_{N/2}(z) = E + i O with E, O the DFTs of the even and odd
// samples, and the half spectrum of x is
//   X[k] = E[k] + W^k O[k],  E[k] = (Z[k] + conj Z[N/2-k]) / 2,
//                            O[k] = -i (Z[k] - conj Z[N/2-k]) / 2,   k = 0..N/2,
// (indices mod N/2, W = exp(-2 pi i / N)).  The inverse runs the same algebra
// backwards: Z[k] = E[k] + i O[k] with E[k] = (X[k] + conj X[N/2-k]) / 2 and
// O[k] = W^-k (X[k] - conj X[N/2-k]) / 2, then an unnormalised inverse DFT of
// N/2 points yields (N/2) z, so the caller's scale carries the factor 2.
// Twiddles W^k, k = 0..N/2, come from a per-plan table computed in double.
#include "kernels.hpp"

#include <cuda_runtime.h>

namespace cubf {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Bin k of the half spectrum from Z[k] and conj Z[N/2 - k] (indices mod N/2).
__device__ __forceinline__ float2 r2c_bin(float2 zk, float2 zm, float2 w, float scale) {
    const float2 e = make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y - zm.y));
    const float2 d = make_float2(0.5f * (zk.x - zm.x), 0.5f * (zk.y + zm.y));  // (Z[k] - conj Z[-k]) / 2
    const float2 o = make_float2(d.y, -d.x);                                      // -i d
    const float2 t = cmul(w, o);
    return make_float2((e.x + t.x) * scale, (e.y + t.y) * scale);
}

// Bins k and N/2 - k read the same two values, so one thread makes both
// (k = 0 .. N/4): every spectrum value is read once.
__global__ void __launch_bounds__(kThreads) r2c_post_kernel(const float2* z, float2* x, const float2* tw, size_t half,
                                                            size_t batch, size_t out_bs, float scale) {
    const size_t per = half / 2 + 1, total = per * batch;
    for (size_t idx = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * kThreads) {
        const size_t b = idx / per, k = idx - b * per;
        const float2* zb = z + b * half;
        float2* xb = x + b * out_bs;
        const float2 a = zb[k];
        const float2 m = zb[k == 0 ? 0 : half - k];
        xb[k] = r2c_bin(a, m, tw[k], scale);
        if (half - k != k) xb[half - k] = r2c_bin(m, a, tw[half - k], scale);
    }
}

// z[k] from X[k] and conj X[N/2 - k]; z[k] and z[N/2 - k] share their reads.
__device__ __forceinline__ float2 c2r_value(float2 xk, float2 xm, float2 w, float scale) {
    const float2 e = make_float2(0.5f * (xk.x + xm.x), 0.5f * (xk.y - xm.y));
    const float2 d = make_float2(0.5f * (xk.x - xm.x), 0.5f * (xk.y + xm.y));
    const float2 o = cmul(make_float2(w.x, -w.y), d);  // W^-k d
    return make_float2((e.x - o.y) * scale, (e.y + o.x) * scale);  // E + i O
}

__global__ void __launch_bounds__(kThreads) c2r_pre_kernel(const float2* x, float2* z, const float2* tw, size_t half,
                                                           size_t batch, size_t in_bs, float scale) {
    const size_t per = half / 2 + 1, total = per * batch;
    for (size_t idx = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * kThreads) {
        const size_t b = idx / per, k = idx - b * per;
        const float2* xb = x + b * in_bs;
        float2* zb = z + b * half;
        const float2 xk = xb[k], xm = xb[half - k];  // conj of xm taken in c2r_value
        zb[k] = c2r_value(xk, xm, tw[k], scale);
        if (k != 0 && half - k != k) zb[half - k] = c2r_value(xm, xk, tw[half - k], scale);
    }
}

unsigned grid_for(size_t work) {
    size_t blocks = (work + kThreads - 1) / kThreads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    return static_cast<unsigned>(blocks ? blocks : 1);
}

}  // namespace

cudaError_t launch_r2c_post(const void* z, void* x, const void* twiddles, std::size_t half, std::size_t batch,
                            std::size_t out_batch_stride, float scale, cudaStream_t stream) {
    r2c_post_kernel<<<grid_for((half / 2 + 1) * batch), kThreads, 0, stream>>>(
        static_cast<const float2*>(z), static_cast<float2*>(x), static_cast<const float2*>(twiddles), half, batch,
        out_batch_stride, scale);
    return cudaGetLastError();
}

cudaError_t launch_c2r_pre(const void* x, void* z, const void* twiddles, std::size_t half, std::size_t batch,
                           std::size_t in_batch_stride, float scale, cudaStream_t stream) {
    c2r_pre_kernel<<<grid_for((half / 2 + 1) * batch), kThreads, 0, stream>>>(
        static_cast<const float2*>(x), static_cast<float2*>(z), static_cast<const float2*>(twiddles), half, batch,
        in_batch_stride, scale);
    return cudaGetLastError();
}

}  // namespace cubf
