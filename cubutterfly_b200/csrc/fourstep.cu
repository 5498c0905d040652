// fourstep.cu -- twiddle step of the four-step (distributed) FFT.
//
// A length-N = N1 * N2 FFT split over ranks runs column FFTs of length N1,
// multiplies element (n2, k1) by W_N^(n2 k1), exchanges, and runs row FFTs of
// length N2.  This kernel applies the middle multiply to a rank's block of
// rows: data[j][k] *= W_N^((row_offset + j) k), the exponent reduced mod N in
// integers and the twiddle formed in fp64 from two exact tables (W_N^e =
// hi[e >> s] * lo[e & (2^s - 1)]) before one rounding to fp32.
#include <cubutterfly/cubutterfly_b200.h>

#include "fft.cuh"

#include <cuda_runtime.h>

#include <cmath>
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

__global__ void fourstep_twiddle_kernel(float4* data, size_t pairs, int log_cols, size_t row_offset, int log_n,
                                        cubf::fft::OuterTwiddles tw, int conj) {
    const size_t nmask = (size_t{1} << log_n) - 1;
    const size_t cmask = (size_t{1} << log_cols) - 1;
    for (size_t p = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; p < pairs;
         p += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t idx = 2 * p;  // two complex values per float4
        const size_t j = idx >> log_cols;
        const size_t k = idx & cmask;
        const size_t row = row_offset + j;
        float4 v = __ldcs(data + p);
        float2 w0 = cubf::fft::outer_twiddle(tw, (row * k) & nmask);
        float2 w1 = cubf::fft::outer_twiddle(tw, (row * (k + 1)) & nmask);
        if (conj) {
            w0.y = -w0.y;
            w1.y = -w1.y;
        }
        const float2 a = cubf::fft::cmul(make_float2(v.x, v.y), w0);
        const float2 b = cubf::fft::cmul(make_float2(v.z, v.w), w1);
        __stcs(data + p, make_float4(a.x, a.y, b.x, b.y));
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

extern "C" cubutterflyStatus_t cubutterflyB200FourStepTwiddle(void* data, size_t rows, size_t cols,
                                                             size_t row_offset, size_t n, int inverse,
                                                             cudaStream_t stream) {
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
        const std::size_t pairs = rows * cols / 2;
        int dev = 0, sms = 0;
        check(cudaGetDevice(&dev), "current device");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
        const std::size_t want = (pairs + 255) / 256;
        const unsigned grid = static_cast<unsigned>(want < static_cast<std::size_t>(sms) * 16 ? want : sms * 16);
        fourstep_twiddle_kernel<<<grid, 256, 0, stream>>>(static_cast<float4*>(data), pairs, log_cols, row_offset,
                                                           log_n, cubf::fft::OuterTwiddles{t.lo, t.hi, t.split},
                                                           inverse ? 1 : 0);
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
