// fft64.cu -- complex fp64 FFT, radix 2 (the reference's numeric FP64 plans;
// arithmetic of cuntt::reference_fft<Complex64>, src/butterfly_reference.cpp:435-473).
//
// The input is bit-reversal permuted (bitrev.cu), then stage s (half = 2^s)
// combines a = x[base + o], b = x[base + half + o] into a + w b, a - w b with
// w = exp(-+ pi i o / half), taken from a per-plan table of W_N^k computed in
// double with the same angle rounding (k = o N / (2 half)).  Products and sums
// round separately in the reference's order, so results are bit-identical to
// it.  The low min(L, 11) stages run in one shared-memory tile pass over
// 2^11-point blocks; higher stages in groups of up to eight per in-place
// column pass (128-byte column runs of the rows those stages pair); a
// normalised inverse scales by 1/N (exact) in the last stage.
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

// COUNT stages from FIRST on a thread's 16 register values: stage FIRST + i
// pairs registers whose index differs in bit REGBIT + i; `index(k)` is the
// transform index of register k (for the pair's twiddle offset).
template <int FIRST, int COUNT, int REGBIT, typename Index>
__device__ __forceinline__ void row_stages(double2 (&v)[16], const double2* __restrict__ tw, int log_n,
                                           double last_scale, Index index) {
#pragma unroll
    for (int i = 0; i < COUNT; ++i) {
        const int st = FIRST + i;
        const double scale = st + 1 == log_n ? last_scale : 1.0;
        const size_t half = size_t{1} << st;
#pragma unroll
        for (int k = 0; k < 16; ++k)
            if (!(k & (1 << (REGBIT + i)))) {
                const size_t o = index(k) & (half - 1);
                butterfly(v[k], v[k | (1 << (REGBIT + i))], __ldg(tw + (o << (log_n - 1 - st))), scale);
            }
    }
}

// Stages 0 .. 10 of 2048-point blocks (in place), 128 threads per block, 16
// values per thread in registers: stages 0-3 on the thread's 16 consecutive
// values, 4-7 and 8-10 after exchanges through shared memory (one value of
// padding per 16), with the twiddles, order and roundings of the per-stage
// form.
__global__ void __launch_bounds__(128)
    fft64_row2048_kernel(double2* data, const double2* __restrict__ tw, int log_n, double last_scale) {
    __shared__ __align__(16) double2 tile[2048 + 128];
    const int t = threadIdx.x;
    double2* block = data + static_cast<size_t>(blockIdx.x) * 2048;
    auto at = [](int j) { return j + (j >> 4); };
    double2 v[16];
    // phase A: values t * 16 + e (bits 0-3)
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = block[t * 16 + e];
    row_stages<0, 4, 0>(v, tw, log_n, last_scale, [&](int k) { return static_cast<size_t>(t * 16 + k); });
#pragma unroll
    for (int e = 0; e < 16; ++e) tile[at(t * 16 + e)] = v[e];
    __syncthreads();
    // phase B: thread (hi, lo) = index bits (8-10, 0-3); register k = bits 4-7
    const int lo = t & 15, hi = t >> 4;
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = tile[at((hi << 8) | (k << 4) | lo)];
    row_stages<4, 4, 0>(v, tw, log_n, last_scale,
                        [&](int k) { return static_cast<size_t>((hi << 8) | (k << 4) | lo); });
#pragma unroll
    for (int k = 0; k < 16; ++k) tile[at((hi << 8) | (k << 4) | lo)] = v[k];
    __syncthreads();
    // phase C: thread t = index bits 1-7; register k = (bits 8-10) << 1 | bit 0
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = tile[at(((k >> 1) << 8) | (t << 1) | (k & 1))];
    row_stages<8, 3, 1>(v, tw, log_n, last_scale,
                        [&](int k) { return static_cast<size_t>(((k >> 1) << 8) | (t << 1) | (k & 1)); });
#pragma unroll
    for (int k = 0; k < 16; ++k) block[((k >> 1) << 8) | (t << 1) | (k & 1)] = v[k];
}

// Stages s0 .. s0 + g - 1 (s0 >= 11, g <= 8) in one in-place pass: a CTA
// takes kCols adjacent columns (128-byte runs) of the 2^g rows 2^s0 apart
// that those stages pair and applies them in order in shared memory, with the
// per-stage twiddles and arithmetic of the single-stage form.
constexpr int kColGroup = 8;
constexpr int kCols = 8;
// Eight stages s0 .. s0 + 7 (s0 >= 11) in one in-place pass with the values
// in registers: 128 threads take kCols adjacent columns of the 256 rows 2^s0
// apart; thread (group g, column c) holds rows 16 g + i for stages s0 ..
// s0 + 3 and, after one exchange through padded shared memory, rows 16 i + g
// for stages s0 + 4 .. s0 + 7, with the twiddles of the per-stage form.
__global__ void __launch_bounds__(128)
    fft64_column8_kernel(double2* data, const double2* __restrict__ tw, int log_n, int s0, double last_scale) {
    __shared__ __align__(16) double2 tile[256 * (kCols + 1)];
    const size_t tiles_per_block = (size_t{1} << s0) / kCols;
    const size_t blk = blockIdx.x / tiles_per_block;
    const size_t col = (blockIdx.x % tiles_per_block) * kCols + threadIdx.x % kCols;
    double2* base = data + (blk << (s0 + 8)) + col;
    const int g = threadIdx.x / kCols, c = threadIdx.x % kCols;
    double2 v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = base[static_cast<size_t>(16 * g + i) << s0];
    // row(i): the row of register i; stage s0 + first + b pairs registers differing in bit b
    auto stages = [&](int first, auto row) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int st = s0 + first + b;
            const double scale = st + 1 == log_n ? last_scale : 1.0;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (!(i & (1 << b))) {
                    const size_t r = static_cast<size_t>(row(i));
                    const size_t o = ((r & ((size_t{1} << (first + b)) - 1)) << s0) | col;
                    butterfly(v[i], v[i | (1 << b)], __ldg(tw + (o << (log_n - 1 - st))), scale);
                }
        }
    };
    stages(0, [&](int i) { return 16 * g + i; });
#pragma unroll
    for (int i = 0; i < 16; ++i) tile[(16 * g + i) * (kCols + 1) + c] = v[i];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = tile[(16 * i + g) * (kCols + 1) + c];
    stages(4, [&](int i) { return 16 * i + g; });
#pragma unroll
    for (int i = 0; i < 16; ++i) base[static_cast<size_t>(16 * i + g) << s0] = v[i];
}

__global__ void __launch_bounds__(kThreads)
    fft64_column_kernel(double2* data, const double2* __restrict__ tw, int log_n, int s0, int g, double last_scale) {
    extern __shared__ __align__(16) unsigned char raw[];
    double2* tile = reinterpret_cast<double2*>(raw);  // [2^g rows][kCols]
    const size_t tiles_per_block = (size_t{1} << s0) / kCols;
    const size_t blk = blockIdx.x / tiles_per_block;
    const size_t c0 = (blockIdx.x % tiles_per_block) * kCols;
    double2* base = data + (blk << (s0 + g)) + c0;
    const int n = kCols << g;
    for (int i = threadIdx.x; i < n; i += kThreads) tile[i] = base[(static_cast<size_t>(i / kCols) << s0) + i % kCols];
    __syncthreads();
    for (int k = 0; k < g; ++k) {
        const int st = s0 + k;
        const double scale = st + 1 == log_n ? last_scale : 1.0;
        const int half = 1 << k;
        for (int p = threadIdx.x; p < n / 2; p += kThreads) {
            const int c = p % kCols, q = p / kCols;
            const int r = ((q >> k) << (k + 1)) | (q & (half - 1));
            // offset of the pair's low element within its 2^(st+1) group
            const size_t o = (static_cast<size_t>(r & (half - 1)) << s0) | (c0 + c);
            butterfly(tile[r * kCols + c], tile[(r + half) * kCols + c], __ldg(tw + (o << (log_n - 1 - st))), scale);
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < n; i += kThreads) base[(static_cast<size_t>(i / kCols) << s0) + i % kCols] = tile[i];
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
    if (tile_log == 11) {
        fft64_row2048_kernel<<<static_cast<unsigned>(blocks), 128, 0, stream>>>(data, tw, log_n, scale);
    } else {
        const int smem = 16 << tile_log;
        fft64_tile_kernel<<<static_cast<unsigned>(blocks), kThreads, smem, stream>>>(data, tw, log_n, tile_log, scale);
    }
    e = cudaGetLastError();
    for (int s0 = tile_log; s0 < log_n && e == cudaSuccess;) {
        const int g = log_n - s0 < kColGroup ? log_n - s0 : kColGroup;
        const std::size_t ctas = (batch << (log_n - s0 - g)) * ((std::size_t{1} << s0) / kCols);
        if (ctas > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        if (g == kColGroup) {
            fft64_column8_kernel<<<static_cast<unsigned>(ctas), 128, 0, stream>>>(data, tw, log_n, s0, scale);
            e = cudaGetLastError();
            s0 += g;
            continue;
        }
        fft64_column_kernel<<<static_cast<unsigned>(ctas), kThreads, 16 * (kCols << g), stream>>>(data, tw, log_n, s0,
                                                                                                g, scale);
        e = cudaGetLastError();
        s0 += g;
    }
    return e;
}

}  // namespace cubf
