// real_adapter.cu -- the main ABI's legacy real-FFT adapter entry points
// (reference include/cubutterfly/cubutterfly.h:188-194, src/real_fft_adapter.cu):
//   cubutterflyPackRealFp32        complex[i] = (scale * real[i], 0)
//   cubutterflyExpandHermitianFp32 rebuild a height x width complex spectrum
//                                  of a real 2-D signal from its
//                                  height x (width / 2 + 1) half, using
//                                  X[r][c] = conj(X[(height - r) % height][width - c])
// Both return 0, 1 for invalid arguments, or the CUDA launch status.
#include <cubutterfly/cubutterfly.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace {

constexpr int kThreads = 256;

// Four real values per thread in, two 16-byte complex pairs out.
__global__ void __launch_bounds__(kThreads) pack_real_kernel(const float* in, float2* out, size_t n, float scale) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    const bool vec = (reinterpret_cast<uintptr_t>(in) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    if (vec) {
        const size_t quads = n / 4;
        for (size_t q = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; q < quads; q += stride) {
            const float4 v = reinterpret_cast<const float4*>(in)[q];
            float4* o = reinterpret_cast<float4*>(out) + 2 * q;
            o[0] = make_float4(v.x * scale, 0.f, v.y * scale, 0.f);
            o[1] = make_float4(v.z * scale, 0.f, v.w * scale, 0.f);
        }
        for (size_t i = 4 * quads + static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride)
            out[i] = make_float2(in[i] * scale, 0.f);
        return;
    }
    for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride)
        out[i] = make_float2(in[i] * scale, 0.f);
}

__global__ void __launch_bounds__(kThreads)
    expand_hermitian_kernel(const float2* half, float2* full, size_t height, size_t width, size_t total) {
    const size_t hw = width / 2 + 1;
    for (size_t idx = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * kThreads) {
        const size_t c = idx % width;
        const size_t rest = idx / width;
        const size_t r = rest % height;
        const float2* plane = half + (rest / height) * height * hw;
        if (c < hw) {
            full[idx] = plane[r * hw + c];
        } else {
            const float2 v = plane[((height - r) % height) * hw + (width - c)];
            full[idx] = make_float2(v.x, -v.y);
        }
    }
}

unsigned grid_for(size_t work) {
    size_t blocks = (work + kThreads - 1) / kThreads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    return static_cast<unsigned>(blocks ? blocks : 1);
}

}  // namespace

extern "C" int cubutterflyPackRealFp32(const float* input, void* output, size_t elements, float scale,
                                       uint64_t stream) {
    if (input == nullptr || output == nullptr || elements == 0) return 1;
    pack_real_kernel<<<grid_for((elements + 3) / 4), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        input, static_cast<float2*>(output), elements, scale);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int cubutterflyExpandHermitianFp32(const void* half, void* full, uint32_t height, uint32_t width,
                                              size_t batch, uint64_t stream) {
    if (half == nullptr || full == nullptr || height == 0 || width == 0 || batch == 0) return 1;
    const size_t total = batch * static_cast<size_t>(height) * width;
    expand_hermitian_kernel<<<grid_for(total), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const float2*>(half), static_cast<float2*>(full), height, width, total);
    return static_cast<int>(cudaGetLastError());
}
