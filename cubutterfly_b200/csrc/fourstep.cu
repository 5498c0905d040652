// fourstep.cu -- twiddle and transpose steps of the four-step (distributed) FFT.
//
// A length-N = N1 * N2 FFT split over ranks runs column FFTs of length N1,
// multiplies element (k1, n2) by W_N^(k1 n2), exchanges, and runs row FFTs of
// length N2.  The twiddle kernel applies the middle multiply to a rank's block:
// data[i][j] *= W_N^((row_offset + i) (col_offset + j)), the exponent reduced
// mod N in integers and the twiddle formed in fp64 from two exact tables
// (W_N^e = hi[e >> s] * lo[e & (2^s - 1)]) before one rounding to fp32.  The
// transpose kernel moves 32 x 32 tiles of complex64 through shared memory
// (coalesced 256-byte row segments on both sides) for the final reordering.
#include <cubutterfly/cubutterfly_b200.h>

#include "fft.cuh"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace cubf {
void set_last_error(const std::string& message);
}

namespace {

// Generic path: two table-formed twiddles per float4 (any cols >= 2).
__global__ void fourstep_twiddle_kernel(float4* data, size_t pairs, int log_cols, size_t row_offset,
                                        size_t col_offset, int log_n, cubf::fft::OuterTwiddles tw, int conj) {
    const size_t nmask = (size_t{1} << log_n) - 1;
    const size_t cmask = (size_t{1} << log_cols) - 1;
    for (size_t p = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; p < pairs;
         p += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t idx = 2 * p;  // two complex values per float4
        const size_t row = row_offset + (idx >> log_cols);
        const size_t col = col_offset + (idx & cmask);
        float4 v = __ldcs(data + p);
        float2 w0 = cubf::fft::outer_twiddle(tw, (row * col) & nmask);
        float2 w1 = cubf::fft::outer_twiddle(tw, (row * (col + 1)) & nmask);
        if (conj) {
            w0.y = -w0.y;
            w1.y = -w1.y;
        }
        const float2 a = cubf::fft::cmul(make_float2(v.x, v.y), w0);
        const float2 b = cubf::fft::cmul(make_float2(v.z, v.w), w1);
        __stcs(data + p, make_float4(a.x, a.y, b.x, b.y));
    }
}

// Rows of at least 64 columns: a warp covers 64 consecutive columns (32
// float4, one coalesced 512-byte access) of one row per step and walks kSteps
// steps along the row; each thread's two twiddles start from the tables and
// advance by W^(64 row) in fp64 (one complex multiply each per step).
constexpr int kTwiddleSteps = 16;
__global__ void fourstep_twiddle_rows_kernel(float4* data, int log_cols, size_t rows, size_t row_offset,
                                             size_t col_offset, int log_n, cubf::fft::OuterTwiddles tw, int conj,
                                             int steps) {
    const size_t nmask = (size_t{1} << log_n) - 1;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const size_t warps_per_row = (size_t{1} << (log_cols - 6)) / static_cast<size_t>(steps);
    const size_t r = warp / warps_per_row;
    if (r >= rows) return;
    const size_t c0 = (warp % warps_per_row) * static_cast<size_t>(steps) * 64 + 2 * static_cast<size_t>(lane);
    const size_t row = row_offset + r;
    const size_t col = col_offset + c0;
    double2 wa = cubf::fft::outer_twiddle_d(tw, (row * col) & nmask);
    double2 wb = cubf::fft::outer_twiddle_d(tw, (row * (col + 1)) & nmask);
    const double2 step = cubf::fft::outer_twiddle_d(tw, (row * 64) & nmask);
    const double sgn = conj ? -1.0 : 1.0;
    float4* p = data + ((r << log_cols) + c0) / 2;
    for (int s = 0; s < steps; ++s) {
        const float4 v = __ldcs(p + 32 * s);
        const float2 a = cubf::fft::cmul(make_float2(v.x, v.y),
                                         make_float2(static_cast<float>(wa.x), static_cast<float>(sgn * wa.y)));
        const float2 b = cubf::fft::cmul(make_float2(v.z, v.w),
                                         make_float2(static_cast<float>(wb.x), static_cast<float>(sgn * wb.y)));
        __stcs(p + 32 * s, make_float4(a.x, a.y, b.x, b.y));
        wa = cubf::fft::cmul_d(wa, step);
        wb = cubf::fft::cmul_d(wb, step);
    }
}

// out[b][c][r] = in[b][r][c]; 32 x 32 tiles, 32 x 8 threads, batch in z.
__global__ void transpose_c64_kernel(const float2* __restrict__ in, float2* __restrict__ out, size_t rows,
                                     size_t cols) {
    __shared__ float2 tile[32][33];
    const size_t base = static_cast<size_t>(blockIdx.z) * rows * cols;
    const size_t r0 = static_cast<size_t>(blockIdx.y) * 32, c0 = static_cast<size_t>(blockIdx.x) * 32;
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        const size_t r = r0 + threadIdx.y + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[threadIdx.y + i][threadIdx.x] = __ldcs(in + base + r * cols + c);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        const size_t c = c0 + threadIdx.y + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) __stcs(out + base + c * rows + r, tile[threadIdx.x][threadIdx.y + i]);
    }
}

// out[b][a][c] = in[a][b][c] for (A, B, C) blocks of complex64, C a
// multiple of 2 (16-byte moves).  When in_self / out_self are set, source
// block a == self is read from in_self ([B][C]) and destination block
// b == self is written to out_self ([A][C]) instead -- a rank's own block of
// an all-to-all never has to pass through the exchange buffers.
__global__ void permute_blocks_c64_kernel(const float4* __restrict__ in, const float4* __restrict__ in_self,
                                          float4* __restrict__ out, float4* __restrict__ out_self, size_t self,
                                          size_t A, size_t B, size_t c4) {
    const size_t runs = A * B;
    for (size_t run = blockIdx.x; run < runs; run += gridDim.x) {
        const size_t a = run / B, b = run % B;
        const float4* src = (in_self && a == self) ? in_self + b * c4 : in + run * c4;
        float4* dst = (out_self && b == self) ? out_self + a * c4 : out + (b * A + a) * c4;
        for (size_t i = threadIdx.x; i < c4; i += blockDim.x) __stcs(dst + i, __ldcs(src + i));
    }
}

struct Tables {
    double2* lo = nullptr;
    double2* hi = nullptr;
    int split = 0;
    ~Tables() {
        if (lo) cudaFree(lo);
        if (hi) cudaFree(hi);
    }
};

std::mutex g_mutex;
std::map<std::pair<int, int>, std::unique_ptr<Tables>> g_tables;  // (device, log n)

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

const Tables& tables_for(int log_n) {
    int dev = 0;
    check(cudaGetDevice(&dev), "current device");
    std::lock_guard<std::mutex> lock(g_mutex);
    auto& slot = g_tables[{dev, log_n}];
    if (slot) return *slot;
    auto t = std::make_unique<Tables>();
    constexpr double kPi = 3.141592653589793238462643383279502884;
    t->split = (log_n + 1) / 2;
    const std::size_t nlo = std::size_t{1} << t->split, nhi = std::size_t{1} << (log_n - t->split);
    const double n = std::ldexp(1.0, log_n);
    std::vector<double> lo(2 * nlo), hi(2 * nhi);
    for (std::size_t k = 0; k < nlo; ++k) {
        const double a = -2.0 * kPi * static_cast<double>(k) / n;
        lo[2 * k] = std::cos(a);
        lo[2 * k + 1] = std::sin(a);
    }
    for (std::size_t k = 0; k < nhi; ++k) {
        const double a = -2.0 * kPi * static_cast<double>(k << t->split) / n;
        hi[2 * k] = std::cos(a);
        hi[2 * k + 1] = std::sin(a);
    }
    check(cudaMalloc(&t->lo, nlo * sizeof(double2)), "twiddle table allocation");
    check(cudaMalloc(&t->hi, nhi * sizeof(double2)), "twiddle table allocation");
    check(cudaMemcpy(t->lo, lo.data(), nlo * sizeof(double2), cudaMemcpyHostToDevice), "twiddle upload");
    check(cudaMemcpy(t->hi, hi.data(), nhi * sizeof(double2), cudaMemcpyHostToDevice), "twiddle upload");
    slot = std::move(t);
    return *slot;
}

}  // namespace

namespace cubf {
// W_N^k tables of the four-step twiddles (per device and log N, built once).
fft::OuterTwiddles fourstep_twiddle_tables(int log_n) {
    const Tables& t = tables_for(log_n);
    return fft::OuterTwiddles{t.lo, t.hi, t.split};
}
}  // namespace cubf

extern "C" cubutterflyStatus_t cubutterflyB200FourStepTwiddle(void* data, size_t rows, size_t cols,
                                                             size_t row_offset, size_t col_offset, size_t n,
                                                             int inverse, cudaStream_t stream) {
    try {
        cubf::set_last_error("");
        if (!data || rows == 0 || cols < 2 || (cols & (cols - 1)) || n == 0 || (n & (n - 1)))
            throw std::invalid_argument("four-step twiddle needs non-null data, rows > 0, power-of-two cols >= 2 and n");
        if (reinterpret_cast<std::uintptr_t>(data) % 16)
            throw std::invalid_argument("four-step twiddle data must be 16-byte aligned");
        int log_n = 0, log_cols = 0;
        while ((std::size_t{1} << log_n) < n) ++log_n;
        while ((std::size_t{1} << log_cols) < cols) ++log_cols;
        if (log_n > 40) throw std::invalid_argument("four-step twiddle length is limited to 2^40");
        const Tables& t = tables_for(log_n);
        const cubf::fft::OuterTwiddles ot{t.lo, t.hi, t.split};
        if (log_cols >= 6) {
            const std::size_t chunks = cols / 64;
            const int steps = static_cast<int>(chunks < kTwiddleSteps ? chunks : kTwiddleSteps);
            const std::size_t warps = rows * (chunks / static_cast<std::size_t>(steps));
            const std::size_t blocks = (warps * 32 + 255) / 256;
            if (blocks > 0x7fffffffULL) throw std::invalid_argument("four-step twiddle grid is too large");
            fourstep_twiddle_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
                static_cast<float4*>(data), log_cols, rows, row_offset, col_offset, log_n, ot, inverse ? 1 : 0, steps);
        } else {
            const std::size_t pairs = rows * cols / 2;
            int dev = 0, sms = 0;
            check(cudaGetDevice(&dev), "current device");
            check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
            const std::size_t want = (pairs + 255) / 256;
            const unsigned grid =
                static_cast<unsigned>(want < static_cast<std::size_t>(sms) * 16 ? want : sms * 16);
            fourstep_twiddle_kernel<<<grid, 256, 0, stream>>>(static_cast<float4*>(data), pairs, log_cols, row_offset,
                                                               col_offset, log_n, ot, inverse ? 1 : 0);
        }
        check(cudaGetLastError(), "four-step twiddle launch");
        return CUBUTTERFLY_STATUS_SUCCESS;
    } catch (const std::invalid_argument& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::exception& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_CUDA_ERROR;
    }
}

extern "C" cubutterflyStatus_t cubutterflyB200TransposeC64(const void* input, void* output, size_t batch, size_t rows,
                                                          size_t cols, cudaStream_t stream) {
    try {
        cubf::set_last_error("");
        if (!input || !output || batch == 0 || rows == 0 || cols == 0)
            throw std::invalid_argument("transpose needs non-null buffers and nonzero batch, rows and cols");
        if (input == output) throw std::invalid_argument("transpose must be out of place");
        const std::size_t ty = (rows + 31) / 32, tx = (cols + 31) / 32;
        if (tx > 0x7fffffffULL || ty > 65535 || batch > 65535)
            throw std::invalid_argument("transpose grid exceeds the launch limits (rows/32 and batch <= 65535)");
        transpose_c64_kernel<<<dim3(static_cast<unsigned>(tx), static_cast<unsigned>(ty), static_cast<unsigned>(batch)),
                               dim3(32, 8), 0, stream>>>(static_cast<const float2*>(input), static_cast<float2*>(output),
                                                         rows, cols);
        check(cudaGetLastError(), "transpose launch");
        return CUBUTTERFLY_STATUS_SUCCESS;
    } catch (const std::invalid_argument& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::exception& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_CUDA_ERROR;
    }
}

extern "C" cubutterflyStatus_t cubutterflyB200PermuteBlocksC64(const void* input, const void* input_self,
                                                              void* output, void* output_self, size_t self,
                                                              size_t a, size_t b, size_t c, cudaStream_t stream) {
    try {
        cubf::set_last_error("");
        if (!input || !output || a == 0 || b == 0 || c == 0 || c % 2)
            throw std::invalid_argument("block permute needs non-null buffers, nonzero A and B and an even C");
        for (const void* ptr : {input, input_self, static_cast<const void*>(output), static_cast<const void*>(output_self)})
            if (reinterpret_cast<std::uintptr_t>(ptr) % 16)
                throw std::invalid_argument("block permute buffers must be 16-byte aligned");
        if (input == output) throw std::invalid_argument("block permute must be out of place");
        int dev = 0, sms = 0;
        check(cudaGetDevice(&dev), "current device");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
        const std::size_t runs = a * b;
        const unsigned grid = static_cast<unsigned>(runs < static_cast<std::size_t>(sms) * 8 ? runs : sms * 8);
        permute_blocks_c64_kernel<<<grid, 256, 0, stream>>>(
            static_cast<const float4*>(input), static_cast<const float4*>(input_self), static_cast<float4*>(output),
            static_cast<float4*>(output_self), self, a, b, c / 2);
        check(cudaGetLastError(), "block permute launch");
        return CUBUTTERFLY_STATUS_SUCCESS;
    } catch (const std::invalid_argument& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::exception& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_CUDA_ERROR;
    }
}
