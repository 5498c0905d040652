// fwht_native.cu -- FWHT with native low-precision stage storage: bf16 or fp16
// values rounded to their storage type after every stage (the reference's
// LowFwhtOperator<Storage, Native = true>, src/operator_traits.cuh:114-154).
//
// Stage s (s = 0 .. L-1, in that order) maps (l, r) to (l + r, l - r) with
// correctly rounded storage-precision add / sub.  A normalised inverse halves
// every stage: after the butterfly when both operands have headroom
// (magnitude bits <= 0x7e7f bf16 / 0x73ff fp16), before it otherwise.  The low
// min(L, 12) stages run in one tile pass (rows of 4096 in register phases
// over packed pairs, shorter rows in shared memory), each higher stage as one
// in-place pass.
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

// Two stage-storage values per 32-bit word (lanes: the lower address low).
template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
    using P = __nv_bfloat162;
    static __device__ __forceinline__ P add(P a, P b) { return __hadd2_rn(a, b); }
    static __device__ __forceinline__ P sub(P a, P b) { return __hsub2_rn(a, b); }
    static __device__ __forceinline__ P swap(P a) { return __lowhigh2highlow(a); }
    static __device__ __forceinline__ P lows(P a, P b) { return __lows2bfloat162(a, b); }
    static __device__ __forceinline__ __nv_bfloat16 lane(uint32_t u, int i) {
        return __ushort_as_bfloat16(static_cast<unsigned short>(u >> (16 * i)));
    }
    static __device__ __forceinline__ uint32_t join(__nv_bfloat16 a, __nv_bfloat16 b) {
        return __bfloat16_as_ushort(a) | (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
    }
};
template <>
struct Pack<__half> {
    using P = __half2;
    static __device__ __forceinline__ P add(P a, P b) { return __hadd2_rn(a, b); }
    static __device__ __forceinline__ P sub(P a, P b) { return __hsub2_rn(a, b); }
    static __device__ __forceinline__ P swap(P a) { return __lowhigh2highlow(a); }
    static __device__ __forceinline__ P lows(P a, P b) { return __lows2half2(a, b); }
    static __device__ __forceinline__ __half lane(uint32_t u, int i) {
        return __ushort_as_half(static_cast<unsigned short>(u >> (16 * i)));
    }
    static __device__ __forceinline__ uint32_t join(__half a, __half b) {
        return __half_as_ushort(a) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
    }
};

template <typename P>
__device__ __forceinline__ P to_pair(uint32_t u) {
    P p;
    memcpy(&p, &u, 4);
    return p;
}
template <typename P>
__device__ __forceinline__ uint32_t to_word(P p) {
    uint32_t u;
    memcpy(&u, &p, 4);
    return u;
}

// Two butterflies at once: lanes of `l` pair with the same lanes of `r`.
// A normalised inverse decides halving per element pair, so it runs lane by
// lane through the scalar butterfly.
template <typename T>
__device__ __forceinline__ void butterfly2(uint32_t& l, uint32_t& r, bool normalize) {
    using K = Pack<T>;
    using P = typename K::P;
    if (!normalize) {
        const P a = to_pair<P>(l), b = to_pair<P>(r);
        l = to_word(K::add(a, b));
        r = to_word(K::sub(a, b));
        return;
    }
    T l0 = K::lane(l, 0), l1 = K::lane(l, 1), r0 = K::lane(r, 0), r1 = K::lane(r, 1);
    butterfly(l0, r0, true);
    butterfly(l1, r1, true);
    l = K::join(l0, l1);
    r = K::join(r0, r1);
}

// Stage 0 inside one word: lanes (a, b) -> (a + b, a - b).
template <typename T>
__device__ __forceinline__ void butterfly_in_word(uint32_t& u, bool normalize) {
    using K = Pack<T>;
    using P = typename K::P;
    if (!normalize) {
        const P x = to_pair<P>(u), y = K::swap(x);
        u = to_word(K::lows(K::add(x, y), K::sub(x, y)));
        return;
    }
    T a = K::lane(u, 0), b = K::lane(u, 1);
    butterfly(a, b, true);
    u = K::join(a, b);
}

// Rows of 4096 values (the first 12 stages of any longer row), 128 threads
// per row, two rows per CTA, 32 values per thread as 16 words paired over
// index bit 0.  Stages run in register phases in ascending order, the same
// order and roundings as the reference: bits 0-4 (the thread's 32 consecutive
// values, 64-byte loads), bits 5-8 and bits 9-11 after exchanges of 32-bit
// words through shared memory (4 words of padding per 16 keep the 16-byte
// writes conflict free), results stored as 8-byte runs.
template <typename T>
__global__ void __launch_bounds__(256) native_row4096_kernel(const T* in, T* out, size_t rows, int normalize) {
    __shared__ __align__(16) uint32_t exchange[2][2048 + 512];
    const int t = threadIdx.x & 127;
    const size_t row = static_cast<size_t>(blockIdx.x) * 2 + (threadIdx.x >> 7);
    const bool active = row < rows;
    const T* src = in + (active ? row : 0) * 4096;
    T* dst = out + (active ? row : 0) * 4096;
    uint32_t* w = exchange[threadIdx.x >> 7];
    const bool nz = normalize != 0;
    auto padded = [](int word) { return word + ((word >> 4) << 2); };
    uint32_t v[16];
    {  // phase A: values t * 32 + e
        const uint4* s4 = reinterpret_cast<const uint4*>(src + t * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 a = active ? s4[q] : make_uint4(0, 0, 0, 0);
            v[4 * q] = a.x;
            v[4 * q + 1] = a.y;
            v[4 * q + 2] = a.z;
            v[4 * q + 3] = a.w;
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) butterfly_in_word<T>(v[k], nz);
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int k = 0; k < 16; ++k)
                if (!(k & (1 << b))) butterfly2<T>(v[k], v[k | (1 << b)], nz);
        uint4* wa = reinterpret_cast<uint4*>(w + padded(t * 16));
#pragma unroll
        for (int q = 0; q < 4; ++q) wa[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    __syncthreads();
    {  // phase B: thread (hi, lo) holds words (hi << 8) | (k << 4) | lo, k = index bits 5-8
        const int lo = t & 15, hi = t >> 4;
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = w[padded((hi << 8) | (k << 4) | lo)];
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int k = 0; k < 16; ++k)
                if (!(k & (1 << b))) butterfly2<T>(v[k], v[k | (1 << b)], nz);
#pragma unroll
        for (int k = 0; k < 16; ++k) w[padded((hi << 8) | (k << 4) | lo)] = v[k];
    }
    __syncthreads();
    // phase C: thread t = index bits 2-8; word (c << 8) | (t << 1) | b1, register (c << 1) | b1
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint2 p = *reinterpret_cast<const uint2*>(w + padded((c << 8) | (t << 1)));
        v[2 * c] = p.x;
        v[2 * c + 1] = p.y;
    }
#pragma unroll
    for (int b = 1; b < 4; ++b)
#pragma unroll
        for (int k = 0; k < 16; ++k)
            if (!(k & (1 << b))) butterfly2<T>(v[k], v[k | (1 << b)], nz);
    if (!active) return;
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint2*>(dst + ((c << 9) | (t << 2))) = make_uint2(v[2 * c], v[2 * c + 1]);
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
    if (tile_log == 12) {
        native_row4096_kernel<T><<<static_cast<unsigned>((blocks + 1) / 2), 256, 0, stream>>>(
            static_cast<const T*>(in), static_cast<T*>(out), blocks, normalize ? 1 : 0);
    } else {
        const int smem = static_cast<int>(sizeof(T)) << tile_log;
        native_tile_kernel<T><<<static_cast<unsigned>(blocks), kThreads, smem, stream>>>(
            static_cast<const T*>(in), static_cast<T*>(out), tile_log, normalize ? 1 : 0);
    }
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
