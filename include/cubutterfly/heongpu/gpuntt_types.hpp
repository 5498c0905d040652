// gpuntt_types.hpp -- the GPU-NTT names the HEonGPU adapter binds, for builds
// without GPU-NTT on the include path.
//
// HEonGPU's NTT layer is GPU-NTT (gpuntt/ntt_merge/ntt.cuh).  The adapter uses
// only these of its names: the 64-bit word types, the modulus record's
// `value`, and the RNS configuration's direction, layout, reduction
// polynomial, zero padding, 1/N table and stream.  A HEonGPU build includes
// GPU-NTT's own header instead (ntt_adapter.hpp picks it when present), so
// only the member names below matter, not their order.
#pragma once

#include <cuda_runtime_api.h>

#include <cstdint>

using Data64 = std::uint64_t;
using Root64 = std::uint64_t;
using Ninverse64 = std::uint64_t;

// A word64 modulus: the value and its Barrett constants.
struct Modulus64 {
    Data64 value = 0;
    Data64 bit = 0;
    Data64 mu = 0;
};

namespace gpuntt {
enum type { FORWARD, INVERSE };
enum NTTLayout { PerPolynomial, PerCoefficient };
enum class ReductionPolynomial { X_N_plus, X_N_minus };

template <typename T>
struct ntt_rns_configuration {
    int n_power = 0;
    type ntt_type = FORWARD;
    NTTLayout ntt_layout = PerPolynomial;
    ReductionPolynomial reduction_poly = ReductionPolynomial::X_N_plus;
    bool zero_padding = false;
    T* mod_inverse = nullptr;  // device: N^-1 mod q per modulus (inverse transforms)
    cudaStream_t stream = nullptr;
};
}  // namespace gpuntt
