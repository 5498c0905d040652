// fwht_native.cu -- FWHT with native low-precision stage storage: bf16 or fp16
// values rounded to their storage type after every stage (the reference's
// LowFwhtOperator<Storage, Native = true>, src/operator_traits.cuh:114-154).
//
// Stage s (s = 0 .. L-1, in that order) maps (l, r) to (l + r, l - r) with
// correctly rounded storage-precision add / sub.  A normalised inverse halves
// every stage: after the butterfly when both operands have headroom
// (magnitude bits <= 0x7e7f bf16 / 0x73ff fp16), before it otherwise.  The low
// min(L, 12) stages run in one shared-memory tile pass, each higher stage as
// one in-place pass.
#include "kernels.hpp"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace cubf {
namespace {

constexpr int kThreads = 256;
constexpr int kTileLog = 12;

template <typename T>
struct Low;
template <>
struct Low<__nv_bfloat16> {
    static constexpr unsigned short kLimit = 0x7e7f;
    static __device__ __forceinline__ __nv_bfloat16 add(__nv_bfloat16 a, __nv_bfloat16 b) { return __hadd_rn(a, b); }
    static __device__ __forceinline__ __nv_bfloat16 sub(__nv_bfloat16 a, __nv_bfloat16 b) { return __hsub_rn(a, b); }
    static __device__ __forceinline__ __nv_bfloat16 mul(__nv_bfloat16 a, __nv_bfloat16 b) { return __hmul_rn(a, b); }
    static __device__ __forceinline__ __nv_bfloat16 half() { return __float2bfloat16_rn(0.5f); }
    static __device__ __forceinline__ unsigned short bits(__nv_bfloat16 v) { return __bfloat16_as_ushort(v) & 0x7fff; }
};
template <>
struct Low<__half> {
    static constexpr unsigned short kLimit = 0x73ff;
    static __device__ __forceinline__ __half add(__half a, __half b) { return __hadd_rn(a, b); }
    static __device__ __forceinline__ __half sub(__half a, __half b) { return __hsub_rn(a, b); }
    static __device__ __forceinline__ __half mul(__half a, __half b) { return __hmul_rn(a, b); }
    static __device__ __forceinline__ __half half() { return __float2half_rn(0.5f); }
    static __device__ __forceinline__ unsigned short bits(__half v) { return __half_as_ushort(v) & 0x7fff; }
};

template <typename T>
__device__ __forceinline__ void butterfly(T& l, T& r, bool normalize) {
    using L = Low<T>;
    const bool after = normalize && L::bits(l) <= L::kLimit && L::bits(r) <= L::kLimit;
    if (normalize && !after) {
        l = L::mul(l, L::half());
        r = L::mul(r, L::half());
    }
    const T a = l, b = r;
    l = L::add(a, b);
    r = L::sub(a, b);
    if (after) {
        l = L::mul(l, L::half());
        r = L::mul(r, L::half());
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) native_tile_kernel(const T* in, T* out, int tile_log, int normalize) {
    extern __shared__ __align__(16) unsigned char raw[];
    T* tile = reinterpret_cast<T*>(raw);
    const size_t n = size_t{1} << tile_log;
    const T* src = in + static_cast<size_t>(blockIdx.x) * n;
    T* dst = out + static_cast<size_t>(blockIdx.x) * n;
    for (size_t i = threadIdx.x; i < n; i += kThreads) tile[i] = src[i];
    __syncthreads();
    for (int s = 0; s < tile_log; ++s) {
        const size_t half = size_t{1} << s;
        for (size_t p = threadIdx.x; p < n / 2; p += kThreads) {
            const size_t lo = ((p >> s) << (s + 1)) | (p & (half - 1));
            butterfly(tile[lo], tile[lo + half], normalize != 0);
        }
        __syncthreads();
    }
    for (size_t i = threadIdx.x; i < n; i += kThreads) dst[i] = tile[i];
}

template <typename T>
__global__ void __launch_bounds__(kThreads) native_stage_kernel(T* data, int s, size_t pairs, int normalize) {
    const size_t half = size_t{1} << s;
    for (size_t p = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; p < pairs;
         p += static_cast<size_t>(gridDim.x) * kThreads) {
        const size_t lo = ((p >> s) << (s + 1)) | (p & (half - 1));
        butterfly(data[lo], data[lo + half], normalize != 0);
    }
}

template <typename T>
cudaError_t launch_typed(int log_n, const void* in, void* out, std::size_t batch, bool normalize,
                         cudaStream_t stream) {
    const int tile_log = log_n < kTileLog ? log_n : kTileLog;
    const std::size_t blocks = batch << (log_n - tile_log);
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
    const int smem = static_cast<int>(sizeof(T)) << tile_log;
    native_tile_kernel<T><<<static_cast<unsigned>(blocks), kThreads, smem, stream>>>(
        static_cast<const T*>(in), static_cast<T*>(out), tile_log, normalize ? 1 : 0);
    cudaError_t e = cudaGetLastError();
    const std::size_t pairs = (batch << log_n) / 2;
    std::size_t grid = (pairs + kThreads - 1) / kThreads;
    if (grid > 148 * 32) grid = 148 * 32;
    for (int s = tile_log; s < log_n && e == cudaSuccess; ++s) {
        native_stage_kernel<T><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(static_cast<T*>(out), s, pairs,
                                                                                    normalize ? 1 : 0);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace

cudaError_t launch_fwht_native(bool bf16, int log_n, const void* in, void* out, std::size_t batch, bool normalize,
                               cudaStream_t stream) {
    if (log_n < 1 || log_n > 30) return cudaErrorInvalidValue;
    return bf16 ? launch_typed<__nv_bfloat16>(log_n, in, out, batch, normalize, stream)
                : launch_typed<__half>(log_n, in, out, batch, normalize, stream);
}

}  // namespace cubf
