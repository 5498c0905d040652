// descriptor.hpp -- transform semantics behind cubutterflyDescriptor_t.
//
// The fields, defaults, validation rules and the two JSON schemas
// ("cubutterfly-descriptor-v1" wrapping "cubutterfly-semantic-v1") are the
// reference's descriptor contract (src/semantic_contract.hpp:11-43,
// src/semantic_contract.cpp:189-406) so that descriptors serialised by either
// library load in the other.  Everything here is CPU-only.
#pragma once

#include <cubutterfly/cubutterfly.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include <nlohmann/json.hpp>

namespace cubf {

using Json = nlohmann::json;

// Default NTT modulus of the reference (include/cuntt/ntt.hpp:17).
constexpr std::uint64_t kDefaultModulus = 1152921504606584833ULL;

// Thrown for requests that are valid semantics but have no executable lowering
// in this build; mapped to CUBUTTERFLY_STATUS_NOT_SUPPORTED.
struct Unsupported : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void require(bool ok, const char* message) {
    if (!ok) throw std::invalid_argument(message);
}
inline void require(bool ok, const std::string& message) {
    if (!ok) throw std::invalid_argument(message);
}

struct Descriptor {
    cubutterflyOperator_t op = CUBUTTERFLY_OPERATOR_FFT;
    cubutterflyDataType_t storage = CUBUTTERFLY_DATA_COMPLEX_FP32;
    cubutterflyComputeType_t compute = CUBUTTERFLY_COMPUTE_FP32;
    cubutterflyDirection_t direction = CUBUTTERFLY_DIRECTION_FORWARD;
    cubutterflyPlacement_t placement = CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE;
    cubutterflyLengthMode_t length_mode = CUBUTTERFLY_LENGTH_STANDARD;
    cubutterflyExecutionMode_t execution_mode = CUBUTTERFLY_EXECUTION_AUTO;
    cubutterflyFftTransformType_t fft_type = CUBUTTERFLY_FFT_C2C;
    double fft_output_scale = 1.0;
    double output_scale = 1.0;
    cubutterflyOutputRounding_t output_rounding = CUBUTTERFLY_ROUNDING_STAGE_STORAGE;
    cubutterflyArithmeticPolicy_t arithmetic_policy = CUBUTTERFLY_ARITHMETIC_STRICT;
    cubutterflyAlgorithmPolicy_t algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
    std::string explicit_algorithm;
    std::uint32_t rank = 1;
    std::vector<std::size_t> extents{256};
    std::vector<std::size_t> input_strides;
    std::vector<std::size_t> output_strides;
    std::size_t input_batch_stride = 0;
    std::size_t output_batch_stride = 0;
    std::size_t batch = 1;
    bool normalize_inverse = true;
    std::uint64_t modulus = kDefaultModulus;
    std::uint32_t word_bits = 64;
    cubutterflyNttLayout_t input_ntt_layout = CUBUTTERFLY_NTT_LAYOUT_NATURAL;
    cubutterflyNttLayout_t output_ntt_layout = CUBUTTERFLY_NTT_LAYOUT_NATURAL;
    std::vector<std::vector<cubutterflyMatrix2x2_t>> stage_matrices = std::vector<std::vector<cubutterflyMatrix2x2_t>>(3);
    std::vector<cubutterflyLogicalOrder_t> input_orders;
    std::vector<cubutterflyLogicalOrder_t> output_orders;
};

// Validated, canonical copy (packed strides resolved, orders expanded, compute
// type resolved, inverse normalisation canonicalised).  Throws
// std::invalid_argument on an invalid description.
Descriptor normalize(const Descriptor& d);
Json semantic_json(const Descriptor& d);
Json descriptor_json(const Descriptor& d);
Descriptor descriptor_from_json(const Json& j);
// Static lowering check of this build: {"status": "eligible"|"missing-lowering", "gaps": [...]}.
Json capabilities(const Descriptor& d);
std::vector<std::size_t> input_extents(const Descriptor& d);
std::vector<std::size_t> output_extents(const Descriptor& d);
// Rank-one batches interleaved element-wise: element n of transform b at
// n * batch + b (stride = batch, batch stride 1), batch a power of two >= 2,
// N >= 16 and N * batch >= 2^12 (a pass tile takes >= 16 columns).  The
// layout of the columns of a row-major matrix.
bool interleaved_batches(const Descriptor& d);
// Rank one, element stride 1, batch stride N on both sides.
bool packed_layout(const Descriptor& d);
bool layout_nonoverlapping(const std::vector<std::size_t>& extents, const std::vector<std::size_t>& strides,
                           std::size_t batch, std::size_t batch_stride);
std::size_t storage_bytes(cubutterflyDataType_t t);
bool is_pow2(std::size_t n);
unsigned log2_exact(std::size_t n);

}  // namespace cubf

// The opaque C handle is the descriptor itself.
struct cubutterflyDescriptor : cubf::Descriptor {};
