// ntt_adapter.hpp -- HEonGPU's word64 per-polynomial RNS NTT served by this
// library's RNS plans.
//
// Mirrors the reference's adapters/heongpu/ntt_adapter.hpp:9-76: the same
// namespace, switches, counters, execution modes and orderings, and the
// gpuntt::cubutterfly_GPU_* wrappers HEonGPU's call sites are patched to.
// An enabled adapter never falls back to GPU-NTT: a request it cannot serve
// throws.  Plans are prepared on the first call of a request (which reads the
// moduli, root tables and orders from device memory and synchronises the
// stream); freeze before timing or CUDA graph capture so a plan miss throws
// instead of preparing.  Root tables, moduli and streams must outlive the
// cached plans; clear the cache after synchronising.  State is per host
// thread, as in the reference.
#pragma once

#include <cstddef>
#include <stdexcept>

#if __has_include(<gpuntt/ntt_merge/ntt.cuh>)
#include <gpuntt/ntt_merge/ntt.cuh>
#define CUBUTTERFLY_HEONGPU_HAVE_GPUNTT 1
#else
#include "gpuntt_types.hpp"
#define CUBUTTERFLY_HEONGPU_HAVE_GPUNTT 0
#endif

#define CUBUTTERFLY_HEONGPU_API __attribute__((visibility("default")))

namespace cubutterfly_heongpu {
CUBUTTERFLY_HEONGPU_API void set_enabled(bool enabled);
CUBUTTERFLY_HEONGPU_API bool enabled();
CUBUTTERFLY_HEONGPU_API void freeze_plans(bool freeze);
CUBUTTERFLY_HEONGPU_API void reset_counters();
CUBUTTERFLY_HEONGPU_API std::size_t replacement_calls();
CUBUTTERFLY_HEONGPU_API std::size_t replacement_polynomials();
CUBUTTERFLY_HEONGPU_API void clear_cache();

// NativeRns: one RNS plan over every polynomial of the call (domains shared
// by equal (q, psi)); Grouped: one RNS plan per modulus.
enum class Execution { NativeRns, Grouped };
CUBUTTERFLY_HEONGPU_API void set_execution(Execution execution);
CUBUTTERFLY_HEONGPU_API Execution get_execution();
CUBUTTERFLY_HEONGPU_API const char* execution_name(Execution execution);

// Which modulus each of the `batch` polynomials uses and where it lives:
//   Contiguous  polynomial b at b * N, modulus b % modulus_count;
//   Modulus     polynomial b at b * N, modulus order[b % modulus_count];
//   Polynomial  polynomial b at order[b] * N, modulus b % modulus_count.
enum class Ordering { Contiguous, Modulus, Polynomial };

// Negacyclic NTT of `batch` polynomials of 2^cfg.n_power words: forward takes
// natural coefficients to bit-reversed evaluations, inverse the reverse
// (scaled by N^-1).  roots[m * N + bitrev(j)] = psi_m^j (psi_m^-j for the
// inverse tables), as HEonGPU stores them.
CUBUTTERFLY_HEONGPU_API void transform(Data64* input, Data64* output, Root64* roots, Modulus64* moduli,
                                       gpuntt::ntt_rns_configuration<Data64> config, int batch, int modulus_count,
                                       Ordering ordering = Ordering::Contiguous, int* order = nullptr);
}  // namespace cubutterfly_heongpu

namespace gpuntt {
namespace cubutterfly_detail {
[[noreturn]] inline void no_gpuntt() {
    throw std::logic_error("cubutterfly HEonGPU adapter is disabled and GPU-NTT is not linked");
}
}  // namespace cubutterfly_detail

#if CUBUTTERFLY_HEONGPU_HAVE_GPUNTT
#define CUBUTTERFLY_HEONGPU_FALLBACK(call) return call
#else
#define CUBUTTERFLY_HEONGPU_FALLBACK(call) cubutterfly_detail::no_gpuntt()
#endif

inline void cubutterfly_GPU_NTT(Data64* input, Data64* output, Root64* roots, Modulus64* moduli,
                                ntt_rns_configuration<Data64> cfg, int batch, int count) {
    if (!cubutterfly_heongpu::enabled()) CUBUTTERFLY_HEONGPU_FALLBACK(GPU_NTT(input, output, roots, moduli, cfg, batch, count));
    cfg.ntt_type = FORWARD;  // GPU-NTT's entry points name the direction
    cubutterfly_heongpu::transform(input, output, roots, moduli, cfg, batch, count);
}
inline void cubutterfly_GPU_INTT(Data64* input, Data64* output, Root64* roots, Modulus64* moduli,
                                 ntt_rns_configuration<Data64> cfg, int batch, int count) {
    if (!cubutterfly_heongpu::enabled()) CUBUTTERFLY_HEONGPU_FALLBACK(GPU_INTT(input, output, roots, moduli, cfg, batch, count));
    cfg.ntt_type = INVERSE;
    cubutterfly_heongpu::transform(input, output, roots, moduli, cfg, batch, count);
}
inline void cubutterfly_GPU_NTT_Inplace(Data64* input, Root64* roots, Modulus64* moduli,
                                        ntt_rns_configuration<Data64> cfg, int batch, int count) {
    if (!cubutterfly_heongpu::enabled()) CUBUTTERFLY_HEONGPU_FALLBACK(GPU_NTT_Inplace(input, roots, moduli, cfg, batch, count));
    cfg.ntt_type = FORWARD;
    cubutterfly_heongpu::transform(input, input, roots, moduli, cfg, batch, count);
}
inline void cubutterfly_GPU_INTT_Inplace(Data64* input, Root64* roots, Modulus64* moduli,
                                         ntt_rns_configuration<Data64> cfg, int batch, int count) {
    if (!cubutterfly_heongpu::enabled()) CUBUTTERFLY_HEONGPU_FALLBACK(GPU_INTT_Inplace(input, roots, moduli, cfg, batch, count));
    cfg.ntt_type = INVERSE;
    cubutterfly_heongpu::transform(input, input, roots, moduli, cfg, batch, count);
}
// The ordered variants keep the configuration's direction.
inline void cubutterfly_GPU_NTT_Modulus_Ordered_Inplace(Data64* input, Root64* roots, Modulus64* moduli,
                                                        ntt_rns_configuration<Data64> cfg, int batch, int count,
                                                        int* order) {
    if (!cubutterfly_heongpu::enabled())
        CUBUTTERFLY_HEONGPU_FALLBACK(GPU_NTT_Modulus_Ordered_Inplace(input, roots, moduli, cfg, batch, count, order));
    cubutterfly_heongpu::transform(input, input, roots, moduli, cfg, batch, count,
                                   cubutterfly_heongpu::Ordering::Modulus, order);
}
inline void cubutterfly_GPU_NTT_Poly_Ordered_Inplace(Data64* input, Root64* roots, Modulus64* moduli,
                                                     ntt_rns_configuration<Data64> cfg, int batch, int count,
                                                     int* order) {
    if (!cubutterfly_heongpu::enabled())
        CUBUTTERFLY_HEONGPU_FALLBACK(GPU_NTT_Poly_Ordered_Inplace(input, roots, moduli, cfg, batch, count, order));
    cubutterfly_heongpu::transform(input, input, roots, moduli, cfg, batch, count,
                                   cubutterfly_heongpu::Ordering::Polynomial, order);
}
#undef CUBUTTERFLY_HEONGPU_FALLBACK
}  // namespace gpuntt
