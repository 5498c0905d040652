// bitrev.cu -- boundary kernels of the main ABI: the bit-reversal permutation
// of packed batches of 2^L elements (logical orders) and the strided gather /
// scatter that stages a strided or padded layout through a packed buffer.
//
// Serves the bit-reversed logical orders of the main ABI (semantic contract
// src/semantic_contract.cpp:257-271: a bit-reversed axis stores logical index
// i at position bitrev(i)).  For L >= 10 the index is split as (a, m, b) with
// 5-bit a and b: element (a, m, b) moves to (rev b, rev m, rev a), so the
// 32 x 32 tile of middle index m maps onto the tile of middle index rev(m) with
// rows and columns exchanged and reversed.  One CTA loads both tiles m and
// rev(m) through shared memory and writes both, so every CTA writes exactly
// the addresses it read and the permutation runs in place as well; rows are
// 32 consecutive elements, so loads and stores are coalesced.  Shorter
// transforms swap element pairs directly.
#include "common.cuh"
#include "kernels.hpp"

#include <cstdint>

namespace cubf {
namespace {

constexpr int kTileBits = 5;
constexpr int kTile = 1 << kTileBits;
constexpr int kThreads = 256;

CUBF_DEV uint32_t rev_bits(uint32_t x, int bits) { return bits ? __brev(x) >> (32 - bits) : 0u; }

template <typename T>
__global__ void __launch_bounds__(kThreads) bitrev_tiled_kernel(const T* in, T* out, int log_n) {
    __shared__ T s[2][kTile][kTile + 1];  // +1 column: the transposed reads hit distinct banks
    const int mid_bits = log_n - 2 * kTileBits;
    const size_t blk = blockIdx.x;
    const uint32_t m = static_cast<uint32_t>(blk & ((size_t{1} << mid_bits) - 1));
    const uint32_t mr = rev_bits(m, mid_bits);
    if (mr < m) return;  // the pair is handled by the CTA of the smaller index
    const bool pair = mr != m;
    const size_t n = size_t{1} << log_n;
    const size_t base = (blk >> mid_bits) * n;
    const size_t row = size_t{1} << (log_n - kTileBits);  // distance between rows a and a + 1
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const T* src = in + base;
    T* dst = out + base;
#pragma unroll
    for (int a = warp; a < kTile; a += kThreads / 32) {
        s[0][a][lane] = src[a * row + (static_cast<size_t>(m) << kTileBits) + lane];
        if (pair) s[1][a][lane] = src[a * row + (static_cast<size_t>(mr) << kTileBits) + lane];
    }
    __syncthreads();
    const uint32_t rl = rev_bits(lane, kTileBits);
#pragma unroll
    for (int a = warp; a < kTile; a += kThreads / 32) {
        const uint32_t ra = rev_bits(a, kTileBits);
        dst[a * row + (static_cast<size_t>(mr) << kTileBits) + lane] = s[0][rl][ra];
        if (pair) dst[a * row + (static_cast<size_t>(m) << kTileBits) + lane] = s[1][rl][ra];
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) bitrev_small_kernel(const T* in, T* out, int log_n, size_t total) {
    const size_t idx = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (idx >= total) return;
    const size_t n = size_t{1} << log_n;
    const size_t base = idx & ~(n - 1);
    const uint32_t i = static_cast<uint32_t>(idx & (n - 1));
    const uint32_t j = rev_bits(i, log_n);
    if (j < i) return;  // each pair is swapped by its smaller index
    const T a = in[base + i], b = in[base + j];
    out[base + j] = a;
    out[base + i] = b;
}

template <typename T>
cudaError_t launch_typed(int log_n, const void* in, void* out, std::size_t batch, cudaStream_t stream) {
    const T* src = static_cast<const T*>(in);
    T* dst = static_cast<T*>(out);
    if (log_n >= 2 * kTileBits) {
        const std::size_t blocks = batch << (log_n - 2 * kTileBits);
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        bitrev_tiled_kernel<T><<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(src, dst, log_n);
    } else {
        const std::size_t total = batch << log_n;
        const std::size_t blocks = (total + kThreads - 1) / kThreads;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        bitrev_small_kernel<T><<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(src, dst, log_n, total);
    }
    return cudaGetLastError();
}

// out[b * obs + i * os] = in[b * ibs + i * is] for i < n, b < batch.
template <typename T>
__global__ void __launch_bounds__(kThreads) strided_copy_kernel(const T* in, size_t is, size_t ibs, T* out, size_t os,
                                                                 size_t obs, size_t n, size_t total) {
    for (size_t idx = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * kThreads) {
        const size_t b = idx / n, i = idx - b * n;
        out[b * obs + i * os] = in[b * ibs + i * is];
    }
}

// Up to three axes and a batch: element (b, i0, i1, i2) moves from
// b * ibs + sum_k i_k * is_k to b * obs + sum_k i_k * os_k.
struct NdLayout {
    size_t ext[3];
    size_t is[3];
    size_t os[3];
    size_t ibs, obs;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) strided_copy_nd_kernel(const T* in, T* out, NdLayout l, size_t total) {
    for (size_t idx = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * kThreads) {
        size_t r = idx;
        const size_t i2 = r % l.ext[2];
        r /= l.ext[2];
        const size_t i1 = r % l.ext[1];
        r /= l.ext[1];
        const size_t i0 = r % l.ext[0];
        const size_t b = r / l.ext[0];
        out[b * l.obs + i0 * l.os[0] + i1 * l.os[1] + i2 * l.os[2]] =
            in[b * l.ibs + i0 * l.is[0] + i1 * l.is[1] + i2 * l.is[2]];
    }
}

template <typename T>
cudaError_t copy_nd_typed(const void* in, void* out, const NdLayout& l, size_t batch, cudaStream_t stream) {
    const std::size_t total = batch * l.ext[0] * l.ext[1] * l.ext[2];
    if (total == 0) return cudaSuccess;
    std::size_t blocks = (total + kThreads - 1) / kThreads;
    if (blocks > 148 * 64) blocks = 148 * 64;
    strided_copy_nd_kernel<T><<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(static_cast<const T*>(in),
                                                                                        static_cast<T*>(out), l, total);
    return cudaGetLastError();
}

template <typename T>
cudaError_t copy_typed(const void* in, std::size_t is, std::size_t ibs, void* out, std::size_t os, std::size_t obs,
                       std::size_t n, std::size_t batch, cudaStream_t stream) {
    const std::size_t total = n * batch;
    std::size_t blocks = (total + kThreads - 1) / kThreads;
    if (blocks > 148 * 64) blocks = 148 * 64;  // grid-stride beyond 64 blocks per SM
    strided_copy_kernel<T><<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(
        static_cast<const T*>(in), is, ibs, static_cast<T*>(out), os, obs, n, total);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_strided_copy(int elem_bytes, const void* in, std::size_t in_stride, std::size_t in_batch_stride,
                                void* out, std::size_t out_stride, std::size_t out_batch_stride, std::size_t n,
                                std::size_t batch, cudaStream_t stream) {
    if (n == 0 || batch == 0) return cudaSuccess;
    switch (elem_bytes) {
        case 2:
            return copy_typed<std::uint16_t>(in, in_stride, in_batch_stride, out, out_stride, out_batch_stride, n,
                                             batch, stream);
        case 4:
            return copy_typed<std::uint32_t>(in, in_stride, in_batch_stride, out, out_stride, out_batch_stride, n,
                                             batch, stream);
        case 8:
            return copy_typed<unsigned long long>(in, in_stride, in_batch_stride, out, out_stride, out_batch_stride,
                                                  n, batch, stream);
        case 16:
            return copy_typed<uint4>(in, in_stride, in_batch_stride, out, out_stride, out_batch_stride, n, batch,
                                     stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_strided_copy_nd(int elem_bytes, int dims, const std::size_t* extents, const void* in,
                                   const std::size_t* in_strides, std::size_t in_batch_stride, void* out,
                                   const std::size_t* out_strides, std::size_t out_batch_stride, std::size_t batch,
                                   cudaStream_t stream) {
    if (dims < 1 || dims > 3) return cudaErrorInvalidValue;
    NdLayout l{};
    const int pad = 3 - dims;  // leading unit axes
    for (int k = 0; k < 3; ++k) {
        const int a = k - pad;
        l.ext[k] = a >= 0 ? extents[a] : 1;
        l.is[k] = a >= 0 ? in_strides[a] : 0;
        l.os[k] = a >= 0 ? out_strides[a] : 0;
    }
    l.ibs = in_batch_stride;
    l.obs = out_batch_stride;
    switch (elem_bytes) {
        case 2: return copy_nd_typed<std::uint16_t>(in, out, l, batch, stream);
        case 4: return copy_nd_typed<std::uint32_t>(in, out, l, batch, stream);
        case 8: return copy_nd_typed<unsigned long long>(in, out, l, batch, stream);
        case 16: return copy_nd_typed<uint4>(in, out, l, batch, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_bitrev(int elem_bytes, int log_n, const void* in, void* out, std::size_t batch,
                          cudaStream_t stream) {
    if (log_n < 0 || log_n > 31) return cudaErrorInvalidValue;
    if (batch == 0 || log_n == 0) {
        if (in != out && batch != 0)
            return cudaMemcpyAsync(out, in, batch * static_cast<std::size_t>(elem_bytes), cudaMemcpyDeviceToDevice,
                                   stream);
        return cudaSuccess;
    }
    switch (elem_bytes) {
        case 2: return launch_typed<std::uint16_t>(log_n, in, out, batch, stream);
        case 4: return launch_typed<std::uint32_t>(log_n, in, out, batch, stream);
        case 8: return launch_typed<unsigned long long>(log_n, in, out, batch, stream);
        case 16: return launch_typed<uint4>(log_n, in, out, batch, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace cubf
