// unaligned.cu -- element-granular FWHT and zeta for caller buffers that are
// element-aligned but not 16-byte aligned.
//
// The reference's cubutterflyExecute accepts any non-null element pointer
// (src/c_api.cpp:4998-5004), e.g. a row-slice view at an odd offset; the tile
// kernels of this build move 16-byte vectors.  For such pointers the executor
// runs these instead (complex FFTs and NTTs need nothing: their kernels move
// whole elements, and the local FFT already takes its float2 path):
//
// * FWHT with FP32 arithmetic and one rounding to storage (FINAL_STORAGE):
//   one CTA per row of up to 2^14 values, the row held in shared memory as
//   fp32, stages 0 .. L-1, then `scale` and the narrowing store -- the
//   reference's widen / FP32 FWHT / scale / narrow contract.
// * Subset / superset zeta (wrap-around integers, so stage order does not
//   change a bit): rows of up to 2^13 (u64) / 2^14 (u32) values the same way;
//   longer rows are copied to the output (when out of place) and then
//   transformed there in place, one element-granular launch per stage.
#include "bitwise.cuh"
#include "kernels.hpp"

#include <cuda_runtime.h>

namespace cubf {
namespace {

constexpr int kThreads = 512;

template <typename TS>
__device__ __forceinline__ float widen(TS x) {
    return Convert<TS, float>::load(x);
}
template <typename TS>
__device__ __forceinline__ TS narrow(float x) {
    return Convert<TS, float>::store(x);
}

template <typename TS>
__global__ void __launch_bounds__(kThreads)
    fwht_rows_unaligned_kernel(const TS* in, TS* out, int log_n, size_t rows, float scale) {
    extern __shared__ float srow[];
    const size_t n = size_t{1} << log_n;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const TS* src = in + row * n;
        TS* dst = out + row * n;
        for (size_t i = threadIdx.x; i < n; i += blockDim.x) srow[i] = widen(src[i]);
        __syncthreads();
        for (int s = 0; s < log_n; ++s) {
            const size_t h = size_t{1} << s;
            for (size_t k = threadIdx.x; k < n / 2; k += blockDim.x) {
                const size_t i = ((k >> s) << (s + 1)) | (k & (h - 1));
                const float a = srow[i], b = srow[i + h];
                srow[i] = a + b;
                srow[i + h] = a - b;
            }
            __syncthreads();
        }
        for (size_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = narrow<TS>(srow[i] * scale);
        __syncthreads();  // the row buffer is free for the next row
    }
}

template <typename T, bool SUPERSET>
__device__ __forceinline__ void zeta_pair(T& lo, T& hi, bool inverse) {
    if (SUPERSET)
        lo = inverse ? lo - hi : lo + hi;
    else
        hi = inverse ? hi - lo : hi + lo;
}

template <typename T, bool SUPERSET>
__global__ void __launch_bounds__(kThreads)
    zeta_rows_unaligned_kernel(const T* in, T* out, int log_n, size_t rows, int inverse) {
    extern __shared__ unsigned char sraw[];
    T* srow = reinterpret_cast<T*>(sraw);
    const size_t n = size_t{1} << log_n;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* src = in + row * n;
        T* dst = out + row * n;
        for (size_t i = threadIdx.x; i < n; i += blockDim.x) srow[i] = src[i];
        __syncthreads();
        for (int s = 0; s < log_n; ++s) {
            const size_t h = size_t{1} << s;
            for (size_t k = threadIdx.x; k < n / 2; k += blockDim.x) {
                const size_t i = ((k >> s) << (s + 1)) | (k & (h - 1));
                zeta_pair<T, SUPERSET>(srow[i], srow[i + h], inverse != 0);
            }
            __syncthreads();
        }
        for (size_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = srow[i];
        __syncthreads();
    }
}

// One stage of an in-place zeta over `batch` rows of 2^log_n values.
template <typename T, bool SUPERSET>
__global__ void __launch_bounds__(256)
    zeta_stage_unaligned_kernel(T* data, int log_n, int s, size_t pairs, int inverse) {
    const size_t h = size_t{1} << s;
    for (size_t k = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < pairs;
         k += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = k >> (log_n - 1), kk = k & ((size_t{1} << (log_n - 1)) - 1);
        T* r = data + (row << log_n);
        const size_t i = ((kk >> s) << (s + 1)) | (kk & (h - 1));
        zeta_pair<T, SUPERSET>(r[i], r[i + h], inverse != 0);
    }
}

unsigned grid_of(size_t units, int per_sm) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t cap = static_cast<size_t>(sms) * per_sm;
    return static_cast<unsigned>(units < cap ? (units ? units : 1) : cap);
}

template <typename TS>
cudaError_t fwht_typed(int log_n, const void* in, void* out, size_t rows, float scale, cudaStream_t stream) {
    const int smem = static_cast<int>(sizeof(float) << log_n);
    auto kernel = fwht_rows_unaligned_kernel<TS>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
    }
    kernel<<<grid_of(rows, 2), kThreads, smem, stream>>>(static_cast<const TS*>(in), static_cast<TS*>(out), log_n,
                                                          rows, scale);
    return cudaGetLastError();
}

template <typename T, bool SUPERSET>
cudaError_t zeta_typed(int log_n, const void* in, void* out, size_t batch, bool inverse, cudaStream_t stream) {
    const size_t row_bytes = sizeof(T) << log_n;
    if (row_bytes <= 64 * 1024) {
        auto kernel = zeta_rows_unaligned_kernel<T, SUPERSET>;
        const int smem = static_cast<int>(row_bytes);
        if (smem > 48 * 1024) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
        }
        kernel<<<grid_of(batch, 2), kThreads, smem, stream>>>(static_cast<const T*>(in), static_cast<T*>(out), log_n,
                                                               batch, inverse ? 1 : 0);
        return cudaGetLastError();
    }
    if (in != out) {
        const cudaError_t e = cudaMemcpyAsync(out, in, row_bytes * batch, cudaMemcpyDeviceToDevice, stream);
        if (e != cudaSuccess) return e;
    }
    const size_t pairs = batch << (log_n - 1);
    const unsigned grid = grid_of((pairs + 255) / 256, 16);
    for (int s = 0; s < log_n; ++s) {
        zeta_stage_unaligned_kernel<T, SUPERSET><<<grid, 256, 0, stream>>>(static_cast<T*>(out), log_n, s, pairs,
                                                                           inverse ? 1 : 0);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

cudaError_t launch_fwht_unaligned(BwType type, int log_n, const void* in, void* out, std::size_t rows, float scale,
                                  cudaStream_t stream) {
    if (log_n < 1 || log_n > 14) return cudaErrorInvalidValue;
    switch (type) {
        case BwType::F32: return fwht_typed<float>(log_n, in, out, rows, scale, stream);
        case BwType::BF16: return fwht_typed<__nv_bfloat16>(log_n, in, out, rows, scale, stream);
        case BwType::F16: return fwht_typed<__half>(log_n, in, out, rows, scale, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_zeta_unaligned(BwType type, bool superset, int log_n, const void* in, void* out,
                                  std::size_t batch, bool inverse, cudaStream_t stream) {
    if (log_n < 1 || log_n > 30) return cudaErrorInvalidValue;
    if (type == BwType::U32)
        return superset ? zeta_typed<uint32_t, true>(log_n, in, out, batch, inverse, stream)
                        : zeta_typed<uint32_t, false>(log_n, in, out, batch, inverse, stream);
    if (type == BwType::U64)
        return superset ? zeta_typed<unsigned long long, true>(log_n, in, out, batch, inverse, stream)
                        : zeta_typed<unsigned long long, false>(log_n, in, out, batch, inverse, stream);
    return cudaErrorInvalidValue;
}

}  // namespace cubf
