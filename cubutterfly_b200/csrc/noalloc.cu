// noalloc.cu -- allocation-free entry point for the multi-pass FFT.
//
// Some callers cannot allocate device memory at all: code running under a
// fixed memory budget or a custom pool that owns every byte, plug-in hosts
// that forbid cudaMalloc/cudaFree on their threads, or latency-critical paths
// where an allocation (and its implicit synchronisation) is not acceptable.
// They can still run the multi-pass global FFT, which needs scratch beyond its
// input and output, through cubutterflyB200FftC2CNoAlloc: the scratch and the
// twiddle tables live in the file-scope device arrays below, which every GPU
// that loads this library holds until the process exits.
//
// Set-up: the first call on a device (with that device current) resolves the
// arrays' device addresses with cudaGetSymbolAddress, uploads the twiddle
// tables once and waits for that upload to land (so the first call's kernels
// read complete tables on any stream, blocking or not); make that first call
// before any stream capture.  Calls after it issue kernel launches only.  All calls share one scratch array and it keeps
// the previous call's contents; nothing in it needs to start at zero (every
// scratch word is written by a pass before any pass reads it).  Calls whose
// execution overlaps on the GPU (different streams, or other host threads)
// race on the shared scratch: serialise them on one stream.
#include <cubutterfly/cubutterfly_b200.h>

#include "kernels.hpp"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace {

// Largest scratch this entry point offers: 16 MiB, i.e. n * batch <= 2^21
// complex values.  Passes alternate between the scratch and the output so the
// last one lands in the output; an in-place transform therefore needs an even
// pass count (n <= 2^20, two passes of at most 2^10), and n = 2^21 (three
// passes) runs out of place only.
constexpr std::size_t kScratchBytes = std::size_t{16} << 20;
constexpr int kMinLog = 14;  // below this the single-kernel FFT needs no scratch
constexpr int kMaxLog = 21;

// Outer twiddle tables of every supported length, packed: for log n = L,
// lo = W_N^k (k < 2^split) then hi = W_N^(k << split), split = ceil(L / 2).
constexpr int split_of(int l) { return (l + 1) / 2; }
constexpr int entries_of(int l) { return (1 << split_of(l)) + (1 << (l - split_of(l))); }
constexpr int offset_of(int l) {
    int o = 0;
    for (int i = kMinLog; i < l; ++i) o += entries_of(i);
    return o;
}
constexpr int kOuterEntries = offset_of(kMaxLog + 1);

static __device__ __align__(256) unsigned char g_fft_scratch[kScratchBytes];
static __device__ __align__(256) double2 g_fft_outer[kOuterEntries];
static __device__ __align__(256) float2 g_fft_tw1024[1024];

// Host images of the tables (static storage: no heap use on any call path).
double h_outer[2 * kOuterEntries];
float h_tw1024[2 * 1024];

constexpr int kMaxDevices = 64;
struct DeviceSlots {
    bool ready = false;
    unsigned char* scratch = nullptr;
    double2* outer = nullptr;
    float2* tw1024 = nullptr;
};
DeviceSlots g_slots[kMaxDevices];
bool g_host_tables = false;
std::mutex g_setup_mutex;

struct Failure : std::runtime_error {
    Failure(cubutterflyStatus_t s, const std::string& m) : std::runtime_error(m), status(s) {}
    cubutterflyStatus_t status;
};

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw Failure(CUBUTTERFLY_STATUS_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

void fill_host_tables() {
    constexpr double kPi = 3.141592653589793238462643383279502884;
    for (int l = kMinLog; l <= kMaxLog; ++l) {
        const int split = split_of(l);
        const double n = std::ldexp(1.0, l);
        double* lo = h_outer + 2 * offset_of(l);
        double* hi = lo + 2 * (1 << split);
        for (int k = 0; k < (1 << split); ++k) {
            const double a = -2.0 * kPi * static_cast<double>(k) / n;
            lo[2 * k] = std::cos(a);
            lo[2 * k + 1] = std::sin(a);
        }
        for (int k = 0; k < (1 << (l - split)); ++k) {
            const double a = -2.0 * kPi * static_cast<double>(static_cast<std::size_t>(k) << split) / n;
            hi[2 * k] = std::cos(a);
            hi[2 * k + 1] = std::sin(a);
        }
    }
    for (int k = 0; k < 1024; ++k) {
        const double a = -2.0 * kPi * static_cast<double>(k) / 1024.0;
        h_tw1024[2 * k] = static_cast<float>(std::cos(a));
        h_tw1024[2 * k + 1] = static_cast<float>(std::sin(a));
    }
    g_host_tables = true;
}

// Once per device, with that device current: device addresses of the arrays
// (host code must not use the symbols themselves as pointers) and the tables.
const DeviceSlots& device_setup() {
    int dev = 0;
    check(cudaGetDevice(&dev), "current device");
    if (dev < 0 || dev >= kMaxDevices)
        throw Failure(CUBUTTERFLY_STATUS_NOT_SUPPORTED, "device index beyond the allocation-free table");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceSlots& s = g_slots[dev];
    if (s.ready) return s;
    if (!g_host_tables) fill_host_tables();
    void* p = nullptr;
    check(cudaGetSymbolAddress(&p, g_fft_scratch), "scratch symbol address");
    s.scratch = static_cast<unsigned char*>(p);
    check(cudaGetSymbolAddress(&p, g_fft_outer), "twiddle symbol address");
    s.outer = static_cast<double2*>(p);
    check(cudaGetSymbolAddress(&p, g_fft_tw1024), "twiddle symbol address");
    s.tw1024 = static_cast<float2*>(p);
    check(cudaMemcpyToSymbol(g_fft_outer, h_outer, sizeof(h_outer)), "twiddle upload");
    check(cudaMemcpyToSymbol(g_fft_tw1024, h_tw1024, sizeof(h_tw1024)), "twiddle upload");
    // A pageable-source copy may return before its DMA lands, and kernels on a
    // non-blocking stream do not wait for the legacy stream it ran on.
    check(cudaStreamSynchronize(cudaStreamLegacy), "twiddle upload wait");
    s.ready = true;
    return s;
}

}  // namespace

namespace cubf {
// The library's thread-local last-error text (c_api.cpp), so failures of this
// entry point read back through cubutterflyGetLastErrorString.
void set_last_error(const std::string& message);
}  // namespace cubf

extern "C" cubutterflyStatus_t cubutterflyB200FftC2CNoAlloc(const void* input, void* output, size_t n,
                                                           size_t batch, int inverse, int normalize,
                                                           cudaStream_t stream) {
    try {
        cubf::set_last_error("");
        if (input == nullptr || output == nullptr)
            throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE, "input and output must be non-null");
        if ((reinterpret_cast<std::uintptr_t>(input) | reinterpret_cast<std::uintptr_t>(output)) % 16 != 0)
            throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE, "input and output must be 16-byte aligned");
        if (n == 0 || (n & (n - 1)) != 0)
            throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE, "length must be a power of two");
        int l = 0;
        while ((std::size_t{1} << l) < n) ++l;
        if (l < kMinLog || l > kMaxLog)
            throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE,
                          "allocation-free FFT lengths are 2^14 .. 2^21 (shorter lengths need no scratch: use "
                          "cubutterflyExecute)");
        if (batch == 0) throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE, "batch must be positive");
        const int np = (l + cubf::kFftPassMaxLog - 1) / cubf::kFftPassMaxLog;
        const bool in_place = input == output;
        if (in_place && np % 2 == 1)
            throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE,
                          "in-place allocation-free FFTs go up to 2^20 points; run 2^21 points out of place");
        const std::size_t bytes = n * 8;
        if (batch > kScratchBytes / bytes)
            throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE,
                          "n * batch exceeds the 16 MiB allocation-free scratch (2^21 complex values)");
        const std::size_t total = bytes * batch;
        {
            // pass 0 writes while it reads: partly overlapping buffers would
            // corrupt the input before every element of it is read
            const auto a = reinterpret_cast<std::uintptr_t>(input);
            const auto b = reinterpret_cast<std::uintptr_t>(output);
            if (!in_place && a < b + total && b < a + total)
                throw Failure(CUBUTTERFLY_STATUS_INVALID_VALUE,
                              "input and output overlap: pass the same pointer for an in-place transform or "
                              "disjoint buffers");
        }
        const DeviceSlots& s = device_setup();
        const cubf::FftOuterTables outer{s.outer + offset_of(l), s.outer + offset_of(l) + (1 << split_of(l)),
                                         split_of(l)};
        const float scale = (inverse && normalize) ? 1.0f / static_cast<float>(n) : 1.0f;
        // Same pass schedule and buffer ping-pong as a planned multi-pass FFT;
        // the scratch array stands in for the caller workspace.
        const void* src = input;
        int ns = 0;
        for (int i = 0; i < np; ++i) {
            const int log_r = l / np + (i < l % np ? 1 : 0);
            void* dst = (np - 1 - i) % 2 == 0 ? output : static_cast<void*>(s.scratch);
            const bool last = i + 1 == np;
            check(cubf::launch_fft_global_pass(log_r, src, dst, l, ns, batch, s.tw1024, outer, inverse && i == 0,
                                               inverse && last, last ? scale : 1.0f, stream),
                  "FFT pass launch");
            src = dst;
            ns += log_r;
        }
        return CUBUTTERFLY_STATUS_SUCCESS;
    } catch (const Failure& f) {
        cubf::set_last_error(f.what());
        return f.status;
    } catch (const std::exception& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_INTERNAL_ERROR;
    } catch (...) {
        cubf::set_last_error("unrecognized exception");
        return CUBUTTERFLY_STATUS_INTERNAL_ERROR;
    }
}
