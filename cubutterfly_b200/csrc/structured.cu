// structured.cu -- the structured 2x2 butterfly (reference STRUCTURED_2X2,
// cuntt::reference_structured_2x2, src/butterfly_reference.cpp:541-591).
//
// Stage s (s = 0 .. L-1, applied in that order) maps every pair (l, r) whose
// indices differ in bit s to (m00 l + m01 r, m10 l + m11 r) with the stage's
// matrix.  The low min(L, 12) stages run in one shared-memory tile pass per
// 2^12-element block; higher stages in groups of up to eight per in-place
// column pass (64-byte column runs of the rows those stages pair).  Products and sums round separately (no fused multiply-add), in
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

// COUNT stages from FIRST on the 32 register values of a thread, stage
// FIRST + i pairing registers whose index differs in bit REGBIT + i.
template <typename T, int FIRST, int COUNT, int REGBIT>
__device__ __forceinline__ void row_stages(T (&v)[32], const StructuredStages& m) {
#pragma unroll
    for (int i = 0; i < COUNT; ++i) {
        const T m00 = Coef<T>::get(m, FIRST + i, 0), m01 = Coef<T>::get(m, FIRST + i, 1),
                m10 = Coef<T>::get(m, FIRST + i, 2), m11 = Coef<T>::get(m, FIRST + i, 3);
#pragma unroll
        for (int k = 0; k < 32; ++k)
            if (!(k & (1 << (REGBIT + i)))) stage_pair(v[k], v[k | (1 << (REGBIT + i))], m00, m01, m10, m11);
    }
}

// Stages 0 .. 11 of 4096-element blocks, 128 threads per block, 32 values per
// thread in registers: stages 0-4 on the thread's 32 consecutive values,
// 5-9 and 10-11 after exchanges through shared memory (one word of padding
// per 32 keeps every exchange access conflict free for 4-byte values), in the
// reference's order with its roundings.
template <typename T>
__global__ void __launch_bounds__(128) structured_row4096_kernel(const T* in, T* out, StructuredStages m) {
    __shared__ __align__(16) T tile[4096 + 128];
    const int t = threadIdx.x;
    const T* src = in + static_cast<size_t>(blockIdx.x) * 4096;
    T* dst = out + static_cast<size_t>(blockIdx.x) * 4096;
    auto at = [](int j) { return j + (j >> 5); };
    T v[32];
    // phase A: values t * 32 + e (bits 0-4)
#pragma unroll
    for (int q = 0; q < 32 * static_cast<int>(sizeof(T)) / 16; ++q) {
        const uint4 w = reinterpret_cast<const uint4*>(src + t * 32)[q];
        memcpy(&v[q * 16 / sizeof(T)], &w, 16);
    }
    row_stages<T, 0, 5, 0>(v, m);
#pragma unroll
    for (int e = 0; e < 32; ++e) tile[at(t * 32 + e)] = v[e];
    __syncthreads();
    // phase B: thread (hi, lo) = index bits (10-11, 0-4); register k = bits 5-9
    const int lo = t & 31, hi = t >> 5;
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = tile[at((hi << 10) | (k << 5) | lo)];
    row_stages<T, 5, 5, 0>(v, m);
#pragma unroll
    for (int k = 0; k < 32; ++k) tile[at((hi << 10) | (k << 5) | lo)] = v[k];
    __syncthreads();
    // phase C: thread t = index bits 3-9; register k = (bits 10-11) << 3 | bits 0-2
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = tile[at(((k >> 3) << 10) | (t << 3) | (k & 7))];
    row_stages<T, 10, 2, 3>(v, m);
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int q = 0; q < 8 * static_cast<int>(sizeof(T)) / 16; ++q) {
            uint4 w;
            memcpy(&w, &v[c * 8 + q * 16 / sizeof(T)], 16);
            reinterpret_cast<uint4*>(dst + ((c << 10) | (t << 3)))[q] = w;
        }
}

// Stages s0 .. s0 + g - 1 (s0 >= 12, g <= 8) in one in-place pass: a CTA
// takes kCols adjacent columns (64-byte runs) of the 2^g rows 2^s0 apart that
// those stages pair, applies the stages in order in shared memory and writes
// the tile back.
constexpr int kColGroup = 8;
template <typename T>
__global__ void __launch_bounds__(kThreads) structured_column_kernel(T* data, int s0, int g, StructuredStages m) {
    constexpr int kCols = 64 / static_cast<int>(sizeof(T));
    extern __shared__ __align__(16) unsigned char raw[];
    T* tile = reinterpret_cast<T*>(raw);  // [2^g rows][kCols]
    const size_t tiles_per_block = (size_t{1} << s0) / kCols;
    const size_t blk = blockIdx.x / tiles_per_block;
    T* base = data + (blk << (s0 + g)) + (blockIdx.x % tiles_per_block) * kCols;
    const int n = kCols << g;
    for (int i = threadIdx.x; i < n; i += kThreads) tile[i] = base[(static_cast<size_t>(i / kCols) << s0) + i % kCols];
    __syncthreads();
    for (int k = 0; k < g; ++k) {
        const int st = s0 + k;
        const T m00 = Coef<T>::get(m, st, 0), m01 = Coef<T>::get(m, st, 1), m10 = Coef<T>::get(m, st, 2),
                m11 = Coef<T>::get(m, st, 3);
        const int half = 1 << k;
        for (int p = threadIdx.x; p < n / 2; p += kThreads) {
            const int c = p % kCols, q = p / kCols;
            const int r = ((q >> k) << (k + 1)) | (q & (half - 1));
            stage_pair(tile[r * kCols + c], tile[(r + half) * kCols + c], m00, m01, m10, m11);
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < n; i += kThreads) base[(static_cast<size_t>(i / kCols) << s0) + i % kCols] = tile[i];
}

// Eight stages s0 .. s0 + 7 (s0 >= 12) in one in-place pass with the values
// in registers: a CTA of 16 x kCols threads takes kCols adjacent columns
// (64-byte runs) of the 256 rows 2^s0 apart; thread (group g, column c) holds
// rows 16 g + i (stages s0 .. s0 + 3 in registers), then, after one exchange
// through padded shared memory, rows 16 i + g (stages s0 + 4 .. s0 + 7).
template <typename T>
__global__ void __launch_bounds__(16 * (64 / sizeof(T))) structured_column8_kernel(T* data, int s0, StructuredStages m) {
    constexpr int kCols = 64 / static_cast<int>(sizeof(T));
    __shared__ T tile[256 * (kCols + 1)];
    const size_t tiles_per_block = (size_t{1} << s0) / kCols;
    const size_t blk = blockIdx.x / tiles_per_block;
    T* base = data + (blk << (s0 + 8)) + (blockIdx.x % tiles_per_block) * kCols;
    const int c = threadIdx.x % kCols, g = threadIdx.x / kCols;
    T v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = base[(static_cast<size_t>(16 * g + i) << s0) + c];
    auto stages = [&](int first) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int st = first + b;
            const T m00 = Coef<T>::get(m, st, 0), m01 = Coef<T>::get(m, st, 1), m10 = Coef<T>::get(m, st, 2),
                    m11 = Coef<T>::get(m, st, 3);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (!(i & (1 << b))) stage_pair(v[i], v[i | (1 << b)], m00, m01, m10, m11);
        }
    };
    stages(s0);
#pragma unroll
    for (int i = 0; i < 16; ++i) tile[(16 * g + i) * (kCols + 1) + c] = v[i];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = tile[(16 * i + g) * (kCols + 1) + c];
    stages(s0 + 4);
#pragma unroll
    for (int i = 0; i < 16; ++i) base[(static_cast<size_t>(16 * i + g) << s0) + c] = v[i];
}

template <typename T>
cudaError_t launch_tile(int tile_log, const void* in, void* out, std::size_t blocks, const StructuredStages& m,
                        cudaStream_t stream) {
    const int smem = static_cast<int>(sizeof(T)) << tile_log;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(structured_tile_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem);
        if (e != cudaSuccess) return e;
    }
    structured_tile_kernel<T><<<static_cast<unsigned>(blocks), kThreads, smem, stream>>>(
        static_cast<const T*>(in), static_cast<T*>(out), tile_log, m);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_typed(int log_n, const void* in, void* out, std::size_t batch, const StructuredStages& m,
                         cudaStream_t stream) {
    const int tile_log = log_n < kTileLog ? log_n : kTileLog;
    const std::size_t blocks = batch << (log_n - tile_log);
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
    cudaError_t e = cudaSuccess;
    if (tile_log == 12) {
        structured_row4096_kernel<T><<<static_cast<unsigned>(blocks), 128, 0, stream>>>(static_cast<const T*>(in),
                                                                                        static_cast<T*>(out), m);
        e = cudaGetLastError();
    } else {
        e = launch_tile<T>(tile_log, in, out, blocks, m, stream);
    }
    // higher stages in groups of up to kColGroup per in-place column pass
    constexpr int kCols = 64 / static_cast<int>(sizeof(T));
    for (int s0 = tile_log; s0 < log_n && e == cudaSuccess;) {
        const int g = log_n - s0 < kColGroup ? log_n - s0 : kColGroup;
        const std::size_t ctas = (batch << (log_n - s0 - g)) * ((std::size_t{1} << s0) / kCols);
        if (ctas > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        if (g == kColGroup) {
            structured_column8_kernel<T><<<static_cast<unsigned>(ctas), 16 * kCols, 0, stream>>>(static_cast<T*>(out),
                                                                                               s0, m);
            e = cudaGetLastError();
            s0 += g;
            continue;
        }
        structured_column_kernel<T><<<static_cast<unsigned>(ctas), kThreads, static_cast<int>(sizeof(T)) * (kCols << g),
                                      stream>>>(static_cast<T*>(out), s0, g, m);
        e = cudaGetLastError();
        s0 += g;
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
