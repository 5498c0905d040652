// calibrate.cu -- integer roof of the NTT butterfly on this device.
//
// The RNS / cyclic NTT tile passes are bound by 64-bit integer multiplies
// (three per Shoup product), not by HBM.  To report how close a pass comes to
// that roof, cubutterflyB200NttButterflyPeak measures the rate at which the
// device executes the exact forward lazy (Harvey) Cooley-Tukey butterfly the
// passes use (ntt::ntt_group: reduce_2q, mul_shoup_lazy, add, sub + 2q), on
// values held in registers: no loads, no stores, no shared-memory exchange,
// enough independent butterflies per thread and resident warps per SM to keep
// the integer pipes issuing every cycle.  The result is butterflies per
// second for the whole device.
#include <cubutterfly/cubutterfly_b200.h>

#include "ntt.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <string>

namespace {

using cubf::ntt::u64;

constexpr int kValues = 16;   // residues per thread, as in the 2^8-point tiles
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads, 4)
    butterfly_peak_kernel(u64* sink, u64 q, u64 w0, u64 wq0, int rounds) {
    u64 v[kValues];
#pragma unroll
    for (int r = 0; r < kValues; ++r) v[r] = (threadIdx.x * 131u + r * 7919u + blockIdx.x) % q;
    u64 w = w0, wq = wq0;
    for (int it = 0; it < rounds; ++it) {
        // four radix-2 stages over the 16 registers (pairs at distance 8, 4,
        // 2, 1): 32 butterflies, as one register group of a tile takes them
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int h = 8 >> s;
#pragma unroll
            for (int r0 = 0; r0 < kValues; ++r0) {
                if (r0 & h) continue;
                const int r1 = r0 | h;
                const u64 a = cubf::ntt::reduce_2q(v[r0], 2 * q);
                const u64 t = cubf::ntt::mul_shoup_lazy(v[r1], w, wq, q);
                v[r0] = a + t;
                v[r1] = a - t + 2 * q;
            }
        }
        // a data-independent change of root keeps the compiler from
        // hoisting anything out of the loop
        w ^= static_cast<u64>(it & 1);
        wq ^= static_cast<u64>(it & 1) << 7;
    }
    u64 acc = 0;
#pragma unroll
    for (int r = 0; r < kValues; ++r) acc ^= v[r];
    if (acc == 0x5a5a5a5a5a5a5a5aull) sink[0] = acc;  // never true in practice; keeps the work live
}

}  // namespace

namespace cubf {
void set_last_error(const std::string& message);
}

extern "C" cubutterflyStatus_t cubutterflyB200NttButterflyPeak(unsigned long long modulus, double* per_second) {
    if (per_second == nullptr || modulus < 3 || modulus >= (1ull << 62)) {
        cubf::set_last_error("per_second must be non-null and the modulus in [3, 2^62)");
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    }
    auto fail = [](cudaError_t e) {
        cubf::set_last_error(std::string("butterfly peak: ") + cudaGetErrorString(e));
        cudaGetLastError();
        return CUBUTTERFLY_STATUS_CUDA_ERROR;
    };
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(e);
    // w = 3 mod q with its Shoup quotient floor(3 * 2^64 / q)
    const u64 q = modulus, w = 3 % q;
    const u64 wq = static_cast<u64>((static_cast<unsigned __int128>(w) << 64) / q);
    cudaStream_t s = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    u64* sink = nullptr;
    double best = 0.0;
    if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess) return fail(e);
    if ((e = cudaEventCreate(&a)) == cudaSuccess && (e = cudaEventCreate(&b)) == cudaSuccess &&
        (e = cudaMalloc(&sink, sizeof(u64))) == cudaSuccess) {
        const unsigned grid = static_cast<unsigned>(sms) * 8u;  // two waves of 4 CTAs per SM
        const int rounds = 2048;
        for (int trial = 0; trial < 4 && e == cudaSuccess; ++trial) {
            cudaEventRecord(a, s);
            butterfly_peak_kernel<<<grid, kThreads, 0, s>>>(sink, q, w, wq, rounds);
            cudaEventRecord(b, s);
            if ((e = cudaEventSynchronize(b)) != cudaSuccess) break;
            float ms = 0;
            cudaEventElapsedTime(&ms, a, b);
            const double butterflies = static_cast<double>(grid) * kThreads * rounds * 4 * (kValues / 2);
            if (trial > 0 && ms > 0) best = std::max(best, butterflies / (ms * 1e-3));  // trial 0 warms up
        }
        if (e == cudaSuccess) e = cudaGetLastError();
    }
    if (sink) cudaFree(sink);
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    cudaStreamDestroy(s);
    if (e != cudaSuccess) return fail(e);
    *per_second = best;
    return CUBUTTERFLY_STATUS_SUCCESS;
}
