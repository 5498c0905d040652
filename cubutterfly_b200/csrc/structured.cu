// structured.cu -- the structured 2x2 butterfly (reference STRUCTURED_2X2,
// cuntt::reference_structured_2x2, src/butterfly_reference.cpp:541-591).
//
// Stage s (s = 0 .. L-1, applied in that order) maps every pair (l, r) whose
// indices differ in bit s to (m00 l + m01 r, m10 l + m11 r) with the stage's
// matrix.  The low min(L, 12) stages run in one shared-memory tile pass per
// 2^12-element block; each higher stage is one in-place pass over pairs
// 2^s apart.  Products and sums round separately (no fused multiply-add), in
// the reference's stage order, so results are bit-identical to it.
#include "kernels.hpp"

#include <cuda_runtime.h>

namespace cubf {
namespace {

constexpr int kThreads = 256;
constexpr int kTileLog = 12;

template <typename T>
struct Coef;
template <>
struct Coef<float> {
    static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
    static __device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
    static __host__ __device__ __forceinline__ float get(const StructuredStages& m, int s, int k) { return m.f32[s][k]; }
};
template <>
struct Coef<double> {
    static __device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
    static __device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
    static __host__ __device__ __forceinline__ double get(const StructuredStages& m, int s, int k) { return m.f64[s][k]; }
};

template <typename T>
__device__ __forceinline__ void stage_pair(T& l, T& r, T m00, T m01, T m10, T m11) {
    using C = Coef<T>;
    const T a = l, b = r;
    l = C::add(C::mul(m00, a), C::mul(m01, b));
    r = C::add(C::mul(m10, a), C::mul(m11, b));
}

// Stages 0 .. tile_log - 1 of consecutive 2^tile_log-element blocks.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    structured_tile_kernel(const T* in, T* out, int tile_log, StructuredStages m) {
    extern __shared__ __align__(16) unsigned char raw[];
    T* tile = reinterpret_cast<T*>(raw);
    const size_t n = size_t{1} << tile_log;
    const T* src = in + static_cast<size_t>(blockIdx.x) * n;
    T* dst = out + static_cast<size_t>(blockIdx.x) * n;
    for (size_t i = threadIdx.x; i < n; i += kThreads) tile[i] = src[i];
    __syncthreads();
    for (int s = 0; s < tile_log; ++s) {
        const T m00 = Coef<T>::get(m, s, 0), m01 = Coef<T>::get(m, s, 1), m10 = Coef<T>::get(m, s, 2),
                m11 = Coef<T>::get(m, s, 3);
        const size_t half = size_t{1} << s;
        for (size_t p = threadIdx.x; p < n / 2; p += kThreads) {
            const size_t lo = ((p >> s) << (s + 1)) | (p & (half - 1));
            stage_pair(tile[lo], tile[lo + half], m00, m01, m10, m11);
        }
        __syncthreads();
    }
    for (size_t i = threadIdx.x; i < n; i += kThreads) dst[i] = tile[i];
}

// Stage s >= kTileLog over `pairs` pairs of the whole batch, in place.
template <typename T>
__global__ void __launch_bounds__(kThreads) structured_stage_kernel(T* data, int s, size_t pairs, T m00, T m01, T m10,
                                                                     T m11) {
    const size_t half = size_t{1} << s;
    for (size_t p = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; p < pairs;
         p += static_cast<size_t>(gridDim.x) * kThreads) {
        const size_t lo = ((p >> s) << (s + 1)) | (p & (half - 1));
        stage_pair(data[lo], data[lo + half], m00, m01, m10, m11);
    }
}

template <typename T>
cudaError_t launch_typed(int log_n, const void* in, void* out, std::size_t batch, const StructuredStages& m,
                         cudaStream_t stream) {
    const int tile_log = log_n < kTileLog ? log_n : kTileLog;
    const std::size_t blocks = batch << (log_n - tile_log);
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
    const int smem = static_cast<int>(sizeof(T)) << tile_log;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(structured_tile_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem);
        if (e != cudaSuccess) return e;
    }
    structured_tile_kernel<T><<<static_cast<unsigned>(blocks), kThreads, smem, stream>>>(
        static_cast<const T*>(in), static_cast<T*>(out), tile_log, m);
    cudaError_t e = cudaGetLastError();
    const std::size_t pairs = (batch << log_n) / 2;
    std::size_t grid = (pairs + kThreads - 1) / kThreads;
    if (grid > 148 * 32) grid = 148 * 32;
    for (int s = tile_log; s < log_n && e == cudaSuccess; ++s) {
        structured_stage_kernel<T><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
            static_cast<T*>(out), s, pairs, Coef<T>::get(m, s, 0), Coef<T>::get(m, s, 1), Coef<T>::get(m, s, 2),
            Coef<T>::get(m, s, 3));
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace

cudaError_t launch_structured(int elem_bytes, int log_n, const void* in, void* out, std::size_t batch,
                              const StructuredStages& stages, cudaStream_t stream) {
    if (log_n < 1 || log_n > kStructuredMaxLog) return cudaErrorInvalidValue;
    return elem_bytes == 4 ? launch_typed<float>(log_n, in, out, batch, stages, stream)
                           : launch_typed<double>(log_n, in, out, batch, stages, stream);
}

}  // namespace cubf
