// descriptor.cpp -- validation, canonical JSON and static capabilities.
//
// The validation rules restate the reference's normalize_descriptor
// (src/semantic_contract.cpp:189-318) so that the same descriptors are
// INVALID_VALUE in both libraries; the JSON field names and schema strings are
// the reference's (semantic_contract.cpp:320-406) so serialised descriptors are
// interchangeable.  capabilities() reports what THIS build executes.
#include "descriptor.hpp"

#include <algorithm>
#include <cmath>
#include <limits>
#include <numeric>
#include <unordered_set>
#include <utility>

namespace cubf {
namespace {

template <typename E>
void check_enum(E value, int last) {
    require(static_cast<int>(value) >= 0 && static_cast<int>(value) <= last, "invalid descriptor enum");
}

std::size_t mul_checked(std::size_t a, std::size_t b) {
    require(b == 0 || a <= std::numeric_limits<std::size_t>::max() / b, "descriptor span overflows size_t");
    return a * b;
}
std::size_t add_checked(std::size_t a, std::size_t b) {
    require(a <= std::numeric_limits<std::size_t>::max() - b, "descriptor span overflows size_t");
    return a + b;
}
std::size_t next_pow2(std::size_t n) {
    require(n != 0, "zero extent");
    std::size_t p = 1;
    while (p < n) p = mul_checked(p, 2);
    return p;
}

std::vector<std::size_t> side(const Descriptor& d, bool input) {
    require(d.rank > 0 && d.extents.size() == d.rank, "rank and shape mismatch");
    std::vector<std::size_t> e = d.extents;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    // Zero-extended embedding pads the forward input / inverse output side.
    if (d.length_mode == CUBUTTERFLY_LENGTH_ZERO_EXTENDED_EMBEDDING && input == inverse)
        for (auto& n : e) n = next_pow2(n);
    if (d.op == CUBUTTERFLY_OPERATOR_FFT &&
        ((input && d.fft_type == CUBUTTERFLY_FFT_C2R) || (!input && d.fft_type == CUBUTTERFLY_FFT_R2C)))
        e.back() = e.back() / 2 + 1;
    return e;
}

enum class Proof { Disjoint, Overlap, Unknown };

// Non-overlap proof of a strided batched layout: sorted-stride hierarchy first,
// then a pairwise lattice collision test, then bounded enumeration.
Proof prove_layout(const std::vector<std::size_t>& extents, const std::vector<std::size_t>& strides,
                   std::size_t batch, std::size_t batch_stride) {
    require(!extents.empty() && extents.size() == strides.size() && batch > 0 && batch_stride > 0,
            "invalid layout dimensions");
    std::vector<std::pair<std::size_t, std::size_t>> dims;  // (stride, extent)
    std::size_t span = 1;
    for (std::size_t a = 0; a < extents.size(); ++a) {
        require(extents[a] > 0 && strides[a] > 0, "layout extents and strides must be positive");
        span = add_checked(span, mul_checked(extents[a] - 1, strides[a]));
        if (extents[a] > 1) dims.emplace_back(strides[a], extents[a]);
    }
    add_checked(span, mul_checked(batch - 1, batch_stride));
    if (batch > 1) dims.emplace_back(batch_stride, batch);
    std::sort(dims.begin(), dims.end());
    std::size_t covered = 1;
    bool nested = true;
    for (const auto& [stride, extent] : dims) {
        if (stride < covered) nested = false;
        covered = add_checked(covered, mul_checked(extent - 1, stride));
    }
    if (nested) return Proof::Disjoint;
    for (std::size_t a = 0; a < dims.size(); ++a)
        for (std::size_t b = a + 1; b < dims.size(); ++b) {
            const std::size_t g = std::gcd(dims[a].first, dims[b].first);
            if (dims[a].second - 1 >= dims[b].first / g && dims[b].second - 1 >= dims[a].first / g)
                return Proof::Overlap;
        }
    constexpr std::size_t kLimit = 65536;
    std::size_t points = 1;
    for (const auto& dim : dims) {
        if (dim.second > kLimit / points) return Proof::Unknown;
        points *= dim.second;
    }
    std::unordered_set<std::size_t> seen;
    seen.reserve(points);
    for (std::size_t i = 0; i < points; ++i) {
        std::size_t rest = i, address = 0;
        for (const auto& dim : dims) {
            address += (rest % dim.second) * dim.first;
            rest /= dim.second;
        }
        if (!seen.insert(address).second) return Proof::Overlap;
    }
    return Proof::Disjoint;
}

void resolve_layout(std::vector<std::size_t>& strides, std::size_t& batch_stride,
                    const std::vector<std::size_t>& extents, std::size_t batch) {
    if (strides.empty()) {
        strides.resize(extents.size());
        std::size_t s = 1;
        for (std::size_t a = extents.size(); a-- > 0;) {
            strides[a] = s;
            s = mul_checked(s, extents[a]);
        }
    }
    require(strides.size() == extents.size(), "stride rank mismatch");
    std::size_t span = 1;
    for (std::size_t a = 0; a < extents.size(); ++a) {
        require(strides[a] > 0, "axis stride must be nonzero");
        span = add_checked(span, mul_checked(extents[a] - 1, strides[a]));
    }
    if (!batch_stride) batch_stride = span;
    require(prove_layout(extents, strides, batch, batch_stride) != Proof::Overlap, "descriptor layout overlaps");
}

void resolve_orders(std::vector<cubutterflyLogicalOrder_t>& orders, const std::vector<std::size_t>& extents) {
    if (orders.empty()) orders.assign(extents.size(), CUBUTTERFLY_ORDER_NATURAL);
    require(orders.size() == extents.size(), "logical order rank mismatch");
    for (std::size_t a = 0; a < orders.size(); ++a) {
        check_enum(orders[a], 1);
        require(orders[a] == CUBUTTERFLY_ORDER_NATURAL || is_pow2(extents[a]),
                "bit reversal requires a power-of-two side extent");
    }
}

// ---- JSON readers (strict: exact field sets, range-checked integers) -------
void exact_fields(const Json& v, std::initializer_list<const char*> names) {
    require(v.is_object() && v.size() == names.size(), "JSON fields mismatch");
    for (const char* n : names) require(v.contains(n), "missing JSON field");
}
std::uint64_t json_uint(const Json& v, std::uint64_t maximum) {
    require(v.is_number_integer(), "JSON integer required");
    std::uint64_t r;
    if (v.is_number_unsigned()) {
        r = v.get<std::uint64_t>();
    } else {
        const auto s = v.get<std::int64_t>();
        require(s >= 0, "JSON integer out of range");
        r = static_cast<std::uint64_t>(s);
    }
    require(r <= maximum, "JSON integer out of range");
    return r;
}
template <typename T>
T json_int(const Json& v) {
    return static_cast<T>(json_uint(v, std::numeric_limits<T>::max()));
}
template <typename E>
E json_enum(const Json& v, int last) {
    return static_cast<E>(json_uint(v, static_cast<std::uint64_t>(last)));
}
std::vector<std::size_t> json_sizes(const Json& v) {
    require(v.is_array(), "JSON array required");
    std::vector<std::size_t> r;
    for (const auto& x : v) r.push_back(json_int<std::size_t>(x));
    return r;
}
std::vector<cubutterflyLogicalOrder_t> json_orders(const Json& v) {
    require(v.is_array(), "JSON order array required");
    std::vector<cubutterflyLogicalOrder_t> r;
    for (const auto& x : v) r.push_back(json_enum<cubutterflyLogicalOrder_t>(x, 1));
    return r;
}
double json_real(const Json& v) {
    require(v.is_number(), "JSON number required");
    const double r = v.get<double>();
    require(std::isfinite(r), "JSON number must be finite");
    return r;
}

bool low_precision(cubutterflyDataType_t s) {
    return s == CUBUTTERFLY_DATA_FP16 || s == CUBUTTERFLY_DATA_BF16 || s == CUBUTTERFLY_DATA_COMPLEX_FP16 ||
           s == CUBUTTERFLY_DATA_COMPLEX_BF16;
}

}  // namespace

bool is_pow2(std::size_t n) { return n && !(n & (n - 1)); }
unsigned log2_exact(std::size_t n) {
    unsigned l = 0;
    while ((std::size_t{1} << l) < n) ++l;
    return l;
}

std::size_t storage_bytes(cubutterflyDataType_t t) {
    switch (t) {
        case CUBUTTERFLY_DATA_FP16:
        case CUBUTTERFLY_DATA_BF16: return 2;
        case CUBUTTERFLY_DATA_FP32:
        case CUBUTTERFLY_DATA_COMPLEX_FP16:
        case CUBUTTERFLY_DATA_COMPLEX_BF16:
        case CUBUTTERFLY_DATA_UINT32: return 4;
        case CUBUTTERFLY_DATA_FP64:
        case CUBUTTERFLY_DATA_COMPLEX_FP32:
        case CUBUTTERFLY_DATA_UINT64: return 8;
        case CUBUTTERFLY_DATA_COMPLEX_FP64: return 16;
    }
    throw std::invalid_argument("invalid storage type");
}

std::vector<std::size_t> input_extents(const Descriptor& d) { return side(d, true); }
std::vector<std::size_t> output_extents(const Descriptor& d) { return side(d, false); }

bool interleaved_batches(const Descriptor& d) {
    return d.rank == 1 && d.batch >= 2 && (d.batch & (d.batch - 1)) == 0 && d.extents.size() == 1 &&
           d.extents[0] >= 16 && d.extents[0] * d.batch >= 4096 && d.input_strides == std::vector<std::size_t>{d.batch} &&
           d.output_strides == std::vector<std::size_t>{d.batch} && d.input_batch_stride == 1 &&
           d.output_batch_stride == 1;
}

bool packed_layout(const Descriptor& d) {
    return d.rank == 1 && d.extents.size() == 1 && d.input_strides == std::vector<std::size_t>{1} &&
           d.output_strides == std::vector<std::size_t>{1} && d.input_batch_stride == d.extents[0] &&
           d.output_batch_stride == d.extents[0];
}

bool layout_nonoverlapping(const std::vector<std::size_t>& extents, const std::vector<std::size_t>& strides,
                           std::size_t batch, std::size_t batch_stride) {
    return prove_layout(extents, strides, batch, batch_stride) == Proof::Disjoint;
}

Descriptor normalize(const Descriptor& source) {
    Descriptor d = source;
    check_enum(d.op, 5);
    check_enum(d.storage, 9);
    check_enum(d.compute, 4);
    check_enum(d.direction, 1);
    check_enum(d.placement, 1);
    check_enum(d.length_mode, 1);
    check_enum(d.execution_mode, 2);
    check_enum(d.fft_type, 2);
    check_enum(d.algorithm_policy, 2);
    check_enum(d.input_ntt_layout, 2);
    check_enum(d.output_ntt_layout, 2);
    require((d.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) == !d.explicit_algorithm.empty(),
            "explicit selection policy and algorithm must be supplied together");
    require(d.rank > 0 && d.extents.size() == d.rank, "rank and shape mismatch");
    require(d.batch > 0, "batch must be positive");
    for (auto n : d.extents) require(n > 0, "extent must be positive");
    require(std::isfinite(d.fft_output_scale), "FFT output scale must be finite");
    require(std::isfinite(d.output_scale), "output scale must be finite");
    check_enum(d.output_rounding, 1);
    check_enum(d.arithmetic_policy, 1);
    if (d.arithmetic_policy == CUBUTTERFLY_ARITHMETIC_ALLOW_FP16_MMA)
        require(d.op == CUBUTTERFLY_OPERATOR_FWHT && d.storage == CUBUTTERFLY_DATA_FP16 &&
                    d.compute == CUBUTTERFLY_COMPUTE_NATIVE && d.rank == 1 &&
                    d.direction == CUBUTTERFLY_DIRECTION_FORWARD &&
                    d.placement == CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE && d.output_scale == 1.0 &&
                    d.output_rounding == CUBUTTERFLY_ROUNDING_STAGE_STORAGE,
                "FP16 MMA policy currently supports rank-one forward out-of-place native FP16 FWHT only");

    const bool real = d.storage <= CUBUTTERFLY_DATA_FP64;
    const bool complex = d.storage >= CUBUTTERFLY_DATA_COMPLEX_FP16 && d.storage <= CUBUTTERFLY_DATA_COMPLEX_FP64;
    const bool integer = d.storage >= CUBUTTERFLY_DATA_UINT32;
    const bool low = low_precision(d.storage);
    const auto natural_compute =
        integer ? (d.storage == CUBUTTERFLY_DATA_UINT32 ? CUBUTTERFLY_COMPUTE_UINT32 : CUBUTTERFLY_COMPUTE_UINT64)
                : ((d.storage == CUBUTTERFLY_DATA_FP64 || d.storage == CUBUTTERFLY_DATA_COMPLEX_FP64)
                       ? CUBUTTERFLY_COMPUTE_FP64
                       : CUBUTTERFLY_COMPUTE_FP32);
    require(d.compute == CUBUTTERFLY_COMPUTE_NATIVE ||
                (integer ? (d.compute == CUBUTTERFLY_COMPUTE_UINT32 || d.compute == CUBUTTERFLY_COMPUTE_UINT64)
                         : (d.compute == CUBUTTERFLY_COMPUTE_FP32 || d.compute == CUBUTTERFLY_COMPUTE_FP64)),
            "compute domain is incompatible with storage");
    // Low-precision NATIVE keeps its meaning (stage-storage arithmetic).
    if (d.compute == CUBUTTERFLY_COMPUTE_NATIVE && !low) d.compute = natural_compute;

    if (d.op == CUBUTTERFLY_OPERATOR_FFT) {
        require(d.fft_type == CUBUTTERFLY_FFT_C2C ? complex : real, "FFT transform and storage are incompatible");
        if (d.fft_type != CUBUTTERFLY_FFT_C2C)
            require((d.fft_type == CUBUTTERFLY_FFT_R2C) == (d.direction == CUBUTTERFLY_DIRECTION_FORWARD),
                    "R2C requires forward direction and C2R requires inverse direction");
    } else {
        require(d.fft_type == CUBUTTERFLY_FFT_C2C && d.fft_output_scale == 1.0,
                "FFT parameters require FFT operator");
        if (d.op == CUBUTTERFLY_OPERATOR_NTT) require(integer, "NTT requires integer storage");
    }
    if (d.op != CUBUTTERFLY_OPERATOR_FFT && d.op != CUBUTTERFLY_OPERATOR_NTT &&
        d.length_mode == CUBUTTERFLY_LENGTH_STANDARD)
        for (auto n : d.extents) require(is_pow2(n), "butterfly extent must be power of two");
    if (d.op == CUBUTTERFLY_OPERATOR_NTT) {
        require(d.word_bits == (d.storage == CUBUTTERFLY_DATA_UINT32 ? 32U : 64U), "NTT word bits must match storage");
        require(d.modulus > 2 && (d.modulus & 1) &&
                    (d.word_bits == 64 || d.modulus <= std::numeric_limits<std::uint32_t>::max()),
                "invalid NTT modulus");
    } else {
        require(d.modulus == kDefaultModulus && d.word_bits == 64, "modulus and word bits require NTT operator");
        require(d.input_ntt_layout == CUBUTTERFLY_NTT_LAYOUT_NATURAL &&
                    d.output_ntt_layout == CUBUTTERFLY_NTT_LAYOUT_NATURAL,
                "NTT layouts require NTT operator");
    }
    const auto in = side(d, true), out = side(d, false);
    resolve_orders(d.input_orders, in);
    resolve_orders(d.output_orders, out);
    // The legacy rank-one bit-reversed NTT layout is the bit-reversed logical order.
    for (bool is_input : {true, false}) {
        auto& layout = is_input ? d.input_ntt_layout : d.output_ntt_layout;
        auto& orders = is_input ? d.input_orders : d.output_orders;
        const auto& extents = is_input ? in : out;
        if (layout == CUBUTTERFLY_NTT_LAYOUT_BIT_REVERSED) {
            require(d.rank == 1 && is_pow2(extents[0]), "legacy bit reversal requires rank-one power-of-two shape");
            const auto& given = is_input ? source.input_orders : source.output_orders;
            require(given.empty() || given[0] == CUBUTTERFLY_ORDER_BIT_REVERSED,
                    "legacy bit reversal conflicts with explicit logical order");
            orders[0] = CUBUTTERFLY_ORDER_BIT_REVERSED;
            layout = CUBUTTERFLY_NTT_LAYOUT_NATURAL;
        }
    }
    if (d.input_ntt_layout == CUBUTTERFLY_NTT_LAYOUT_APPT_STATIC ||
        d.output_ntt_layout == CUBUTTERFLY_NTT_LAYOUT_APPT_STATIC) {
        auto natural = [](const std::vector<cubutterflyLogicalOrder_t>& o) {
            return std::all_of(o.begin(), o.end(), [](auto x) { return x == CUBUTTERFLY_ORDER_NATURAL; });
        };
        require(natural(d.input_orders) && natural(d.output_orders),
                "APPT layout cannot be combined with logical bit reversal");
    }
    resolve_layout(d.input_strides, d.input_batch_stride, in, d.batch);
    resolve_layout(d.output_strides, d.output_batch_stride, out, d.batch);
    d.stage_matrices.resize(std::max<std::size_t>(3, std::max<std::size_t>(d.rank, d.stage_matrices.size())));
    for (std::size_t axis = 0; axis < d.stage_matrices.size(); ++axis) {
        const auto& ms = d.stage_matrices[axis];
        require(axis < d.rank || ms.empty(), "matrices supplied beyond rank");
        require(d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2 || ms.empty(), "matrices require structured operator");
        if (d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2 && axis < d.rank)
            require(ms.size() == 1 || ms.size() == log2_exact(next_pow2(d.extents[axis])),
                    "structured axis requires one matrix or one per stage");
        for (const auto& m : ms) {
            require(std::isfinite(m.m00) && std::isfinite(m.m01) && std::isfinite(m.m10) && std::isfinite(m.m11),
                    "matrix entries must be finite");
            if (d.direction == CUBUTTERFLY_DIRECTION_INVERSE) {
                const double det = m.m00 * m.m11 - m.m01 * m.m10;
                require(std::isfinite(det) && det != 0, "inverse matrix must be nonsingular");
            }
        }
    }
    if (d.direction == CUBUTTERFLY_DIRECTION_FORWARD)
        d.normalize_inverse = false;
    else if (d.op == CUBUTTERFLY_OPERATOR_NTT)
        d.normalize_inverse = true;
    else if (d.op == CUBUTTERFLY_OPERATOR_SUBSET_ZETA || d.op == CUBUTTERFLY_OPERATOR_SUPERSET_ZETA ||
             d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2)
        d.normalize_inverse = false;
    if (d.arithmetic_policy == CUBUTTERFLY_ARITHMETIC_ALLOW_FP16_MMA)
        require(d.length_mode == CUBUTTERFLY_LENGTH_STANDARD && is_pow2(d.extents[0]) &&
                    d.input_strides == std::vector<std::size_t>{1} && d.output_strides == d.input_strides &&
                    d.input_batch_stride == d.extents[0] && d.output_batch_stride == d.extents[0] &&
                    d.input_orders == std::vector<cubutterflyLogicalOrder_t>{CUBUTTERFLY_ORDER_NATURAL} &&
                    d.output_orders == d.input_orders,
                "FP16 MMA policy currently requires packed natural power-of-two layout");
    return d;
}

Json semantic_json(const Descriptor& source) {
    const Descriptor d = normalize(source);
    Json matrices = Json::array();
    for (std::size_t axis = 0; axis < d.rank; ++axis) {
        Json list = Json::array();
        for (const auto& m : d.stage_matrices[axis]) list.push_back({m.m00, m.m01, m.m10, m.m11});
        matrices.push_back(std::move(list));
    }
    auto orders = [](const std::vector<cubutterflyLogicalOrder_t>& o) {
        Json a = Json::array();
        for (auto x : o) a.push_back(static_cast<int>(x));
        return a;
    };
    const bool ntt = d.op == CUBUTTERFLY_OPERATOR_NTT;
    Json r{{"schema", "cubutterfly-semantic-v1"},
           {"operator", int(d.op)},
           {"storage", int(d.storage)},
           {"compute", int(d.compute)},
           {"shape", d.extents},
           {"batch", d.batch},
           {"inverse", int(d.direction)},
           {"normalize_inverse", d.normalize_inverse},
           {"placement", int(d.placement)},
           {"fft_type", int(d.fft_type)},
           {"fft_output_scale", d.fft_output_scale},
           {"length_mode", int(d.length_mode)},
           {"input_strides", d.input_strides},
           {"output_strides", d.output_strides},
           {"input_batch_stride", d.input_batch_stride},
           {"output_batch_stride", d.output_batch_stride},
           {"input_orders", orders(d.input_orders)},
           {"output_orders", orders(d.output_orders)},
           {"ntt_input_layout", int(d.input_ntt_layout)},
           {"ntt_output_layout", int(d.output_ntt_layout)},
           {"modulus", ntt ? Json(d.modulus) : Json(nullptr)},
           {"word_bits", ntt ? Json(d.word_bits) : Json(nullptr)},
           {"matrices", matrices}};
    if (d.output_scale != 1.0) r["output_scale"] = d.output_scale;
    if (d.arithmetic_policy != CUBUTTERFLY_ARITHMETIC_STRICT) r["arithmetic_policy"] = int(d.arithmetic_policy);
    if (d.output_rounding != CUBUTTERFLY_ROUNDING_STAGE_STORAGE) r["output_rounding"] = int(d.output_rounding);
    return r;
}

Json descriptor_json(const Descriptor& source) {
    const Descriptor d = normalize(source);
    return {{"schema", "cubutterfly-descriptor-v1"},
            {"semantics", semantic_json(d)},
            {"selection",
             {{"execution_mode", int(d.execution_mode)},
              {"algorithm_policy", int(d.algorithm_policy)},
              {"explicit_algorithm", d.explicit_algorithm}}}};
}

Descriptor descriptor_from_json(const Json& v) {
    exact_fields(v, {"schema", "semantics", "selection"});
    require(v.at("schema").is_string() && v.at("schema") == "cubutterfly-descriptor-v1", "invalid descriptor schema");
    const Json& s = v.at("semantics");
    require(s.is_object(), "JSON semantics object required");
    Json required = s;
    required.erase("output_scale");
    required.erase("output_rounding");
    required.erase("arithmetic_policy");
    exact_fields(required, {"schema", "operator", "storage", "compute", "shape", "batch", "inverse",
                            "normalize_inverse", "placement", "fft_type", "fft_output_scale", "length_mode",
                            "input_strides", "output_strides", "input_batch_stride", "output_batch_stride",
                            "modulus", "word_bits", "matrices", "input_orders", "output_orders",
                            "ntt_input_layout", "ntt_output_layout"});
    require(s.at("schema").is_string() && s.at("schema") == "cubutterfly-semantic-v1", "invalid semantic schema");
    Descriptor d;
    d.op = json_enum<cubutterflyOperator_t>(s.at("operator"), 5);
    d.storage = json_enum<cubutterflyDataType_t>(s.at("storage"), 9);
    d.compute = json_enum<cubutterflyComputeType_t>(s.at("compute"), 4);
    d.direction = json_enum<cubutterflyDirection_t>(s.at("inverse"), 1);
    d.placement = json_enum<cubutterflyPlacement_t>(s.at("placement"), 1);
    d.fft_type = json_enum<cubutterflyFftTransformType_t>(s.at("fft_type"), 2);
    d.length_mode = json_enum<cubutterflyLengthMode_t>(s.at("length_mode"), 1);
    d.input_ntt_layout = json_enum<cubutterflyNttLayout_t>(s.at("ntt_input_layout"), 2);
    d.output_ntt_layout = json_enum<cubutterflyNttLayout_t>(s.at("ntt_output_layout"), 2);
    d.extents = json_sizes(s.at("shape"));
    require(d.extents.size() <= std::numeric_limits<std::uint32_t>::max(), "JSON rank out of range");
    d.rank = static_cast<std::uint32_t>(d.extents.size());
    d.batch = json_int<std::size_t>(s.at("batch"));
    d.input_strides = json_sizes(s.at("input_strides"));
    d.output_strides = json_sizes(s.at("output_strides"));
    d.input_batch_stride = json_int<std::size_t>(s.at("input_batch_stride"));
    d.output_batch_stride = json_int<std::size_t>(s.at("output_batch_stride"));
    d.input_orders = json_orders(s.at("input_orders"));
    d.output_orders = json_orders(s.at("output_orders"));
    require(s.at("normalize_inverse").is_boolean(), "JSON boolean required");
    d.normalize_inverse = s.at("normalize_inverse").get<bool>();
    d.fft_output_scale = json_real(s.at("fft_output_scale"));
    if (s.contains("arithmetic_policy"))
        d.arithmetic_policy = json_enum<cubutterflyArithmeticPolicy_t>(s.at("arithmetic_policy"), 1);
    if (s.contains("output_scale")) d.output_scale = json_real(s.at("output_scale"));
    if (s.contains("output_rounding"))
        d.output_rounding = json_enum<cubutterflyOutputRounding_t>(s.at("output_rounding"), 1);
    if (d.op == CUBUTTERFLY_OPERATOR_NTT) {
        d.modulus = json_int<std::uint64_t>(s.at("modulus"));
        d.word_bits = json_int<std::uint32_t>(s.at("word_bits"));
    } else {
        require(s.at("modulus").is_null() && s.at("word_bits").is_null(), "non-NTT modulus fields must be null");
    }
    const Json& matrices = s.at("matrices");
    require(matrices.is_array() && matrices.size() == d.rank, "JSON matrix rank mismatch");
    d.stage_matrices.assign(std::max<std::size_t>(3, d.rank), {});
    for (std::size_t axis = 0; axis < d.rank; ++axis) {
        require(matrices[axis].is_array(), "JSON matrix list required");
        for (const auto& m : matrices[axis]) {
            require(m.is_array() && m.size() == 4, "JSON matrix requires four entries");
            d.stage_matrices[axis].push_back({json_real(m[0]), json_real(m[1]), json_real(m[2]), json_real(m[3])});
        }
    }
    const Json& sel = v.at("selection");
    exact_fields(sel, {"execution_mode", "algorithm_policy", "explicit_algorithm"});
    d.execution_mode = json_enum<cubutterflyExecutionMode_t>(sel.at("execution_mode"), 2);
    d.algorithm_policy = json_enum<cubutterflyAlgorithmPolicy_t>(sel.at("algorithm_policy"), 2);
    require(sel.at("explicit_algorithm").is_string(), "JSON algorithm string required");
    d.explicit_algorithm = sel.at("explicit_algorithm").get<std::string>();
    return normalize(d);
}

// What this build lowers: rank-one, packed, standard-length power-of-two
// transforms of the four hot-path operator families.
Json capabilities(const Descriptor& source) {
    const Descriptor d = normalize(source);
    Json gaps = Json::array();
    auto gap = [&](const char* code, const char* reason) { gaps.push_back({{"code", code}, {"reason", reason}}); };
    // Ranks two and three run as compositions of rank-one plans: FFT and NTT
    // one per axis (innermost first, the other axes transposed innermost
    // through the workspace), FWHT and zeta as one transform over the
    // concatenated index bits (the tensor product of the per-axis transforms).
    if (d.rank > 3) gap("rank-lowering", "ranks above three are not built");
    // xD execution (reference src/c_api.cpp:4289-4365) needs rank two or
    // more; where its lowering is unavailable the reference itself runs the
    // composite path, which is what ranks two and three execute here.
    if (d.execution_mode == CUBUTTERFLY_EXECUTION_XD && d.rank < 2)
        gap("execution-policy", "xD execution requires rank at least two");
    // Zero-extended embedding (the forward input / inverse output zero-padded
    // to the next power of two) runs staged through a packed buffer of the
    // padded length: rank one, out of place.
    const bool embedded = d.length_mode == CUBUTTERFLY_LENGTH_ZERO_EXTENDED_EMBEDDING;
    if (embedded) {
        if (d.rank != 1) gap("length-lowering", "zero-extended embedding is built for rank one");
        if (d.placement == CUBUTTERFLY_PLACEMENT_IN_PLACE)
            gap("length-lowering", "zero-extended embedding executes out of place");
        if (d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type != CUBUTTERFLY_FFT_C2C)
            gap("length-lowering", "zero-extended embedding is built for complex FFTs");
        if (!std::all_of(d.input_orders.begin(), d.input_orders.end(),
                         [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; }) ||
            !std::all_of(d.output_orders.begin(), d.output_orders.end(),
                         [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; }))
            gap("order-lowering", "zero-extended embedding executes natural logical orders");
    }
    // Standard-length complex FFTs and u64 NTTs of other lengths run as
    // Bluestein convolutions over power-of-two transforms (reference
    // src/bluestein_fft.cu, src/bluestein_ntt.cu): C2C / u64, ranks one and
    // two, natural orders, any layout.
    const bool arbitrary = d.length_mode == CUBUTTERFLY_LENGTH_STANDARD &&
                           std::any_of(d.extents.begin(), d.extents.end(), [](std::size_t e) { return !is_pow2(e); });
    if (arbitrary) {
        if (d.op == CUBUTTERFLY_OPERATOR_NTT && d.storage != CUBUTTERFLY_DATA_UINT64)
            gap("arbitrary-word-lowering", "Bluestein NTT executes uint64 words");
        if (d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type != CUBUTTERFLY_FFT_C2C)
            gap("arbitrary-length-lowering", "non-power-of-two R2C/C2R transforms are not built");
        if (d.rank > 2) gap("rank-bluestein-lowering", "rank-three Bluestein composition is not built");
        if (!std::all_of(d.input_orders.begin(), d.input_orders.end(),
                         [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; }) ||
            !std::all_of(d.output_orders.begin(), d.output_orders.end(),
                         [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; }))
            gap("order-lowering", "non-power-of-two FFTs execute natural logical orders");
    }
    const bool bluestein = arbitrary && (d.op == CUBUTTERFLY_OPERATOR_FFT || d.op == CUBUTTERFLY_OPERATOR_NTT);
    for (auto n : d.extents)
        if ((!is_pow2(n) && !embedded && !bluestein) || n < 2)
            gap("length-lowering", "extents must be powers of two of at least two");
    // R2C / C2R: rank one, fp32, packed, out of place, over an N/2-point
    // complex FFT (N >= 4)
    const bool real_fft = d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type != CUBUTTERFLY_FFT_C2C;
    // (ranks two and three: real rows of the innermost axis, then C2C over
    // the outer axes of the half spectrum, as the reference's RealFFT)
    if (real_fft) {
        if (d.rank > 3) gap("real-fft-lowering", "R2C/C2R transforms are built for ranks one to three");
        if (d.storage != CUBUTTERFLY_DATA_FP32)
            gap("real-fft-lowering", "R2C/C2R transforms execute FP32 real storage");
        if (d.extents.back() < 4) gap("real-fft-lowering", "R2C/C2R transforms need at least four points");
        if (d.placement == CUBUTTERFLY_PLACEMENT_IN_PLACE)
            gap("real-fft-lowering", "R2C/C2R transforms execute out of place");
        const auto ri = side(d, true), ro = side(d, false);
        auto packed = [](const std::vector<std::size_t>& e) {
            std::vector<std::size_t> st(e.size(), 1);
            for (std::size_t k = e.size() - 1; k-- > 0;) st[k] = st[k + 1] * e[k + 1];
            return st;
        };
        auto volume = [](const std::vector<std::size_t>& e) {
            std::size_t v = 1;
            for (auto x : e) v *= x;
            return v;
        };
        if (d.input_strides != packed(ri) || d.output_strides != packed(ro) || d.input_batch_stride != volume(ri) ||
            d.output_batch_stride != volume(ro))
            gap("layout-lowering", "R2C/C2R transforms execute packed batches");
        if (!std::isfinite(static_cast<float>(d.fft_output_scale)))
            gap("fft-scale-lowering", "FFT output scale must be representable as finite FP32");
    }
    if (d.fft_type == CUBUTTERFLY_FFT_C2C && d.fft_output_scale != 1.0)
        gap("fft-scale-lowering", "additional FFT output scaling requires R2C/C2R");
    const auto in = input_extents(d), out = output_extents(d);
    // FWHT and zeta of rank > 1 transform the flattened index; FFT and NTT
    // each axis (bounded by the largest axis)
    std::size_t n = 1, longest = 1;
    for (auto e : d.extents) {
        if (embedded) e = next_pow2(e);  // the padded (physical) length
        if (bluestein && !is_pow2(e)) e = next_pow2(2 * e - 1);  // the convolution length
        n *= e;
        longest = std::max(longest, e);
    }
    if (d.op == CUBUTTERFLY_OPERATOR_FFT || d.op == CUBUTTERFLY_OPERATOR_NTT) n = longest;
    if (d.rank > 1 && !std::all_of(d.input_orders.begin(), d.input_orders.end(),
                                   [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; }))
        gap("order-lowering", "bit-reversed logical orders are built for rank-one transforms");
    if (d.rank > 1 && !std::all_of(d.output_orders.begin(), d.output_orders.end(),
                                   [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; }))
        gap("order-lowering", "bit-reversed logical orders are built for rank-one transforms");
    const bool packed = d.rank == 1 && d.input_strides == std::vector<std::size_t>{1} &&
                        d.output_strides == std::vector<std::size_t>{1} && d.input_batch_stride == in[0] &&
                        d.output_batch_stride == out[0];
    // Other rank-one strided or padded layouts are staged through a packed
    // workspace buffer (gather, packed passes, scatter); FFT batches
    // interleaved element-wise run natively.
    const bool interleaved = d.op == CUBUTTERFLY_OPERATOR_FFT && d.storage == CUBUTTERFLY_DATA_COMPLEX_FP32 &&
                             interleaved_batches(d);
    const bool natural_in = std::all_of(d.input_orders.begin(), d.input_orders.end(),
                                        [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; });
    const bool natural_out = std::all_of(d.output_orders.begin(), d.output_orders.end(),
                                         [](auto o) { return o == CUBUTTERFLY_ORDER_NATURAL; });
    // Bit-reversed orders run as bit-reversal permutations of packed batches.
    if ((!natural_in || !natural_out) && interleaved && !packed)
        gap("order-lowering", "bit-reversed logical orders are not built for interleaved FFT batches");
    // ALLOW_FP16_MMA only permits tensor-core arithmetic: the reference keeps
    // its strict selection when no calibrated MMA candidate wins
    // (src/mapping_selector.cpp:13-42), so the policy itself is no gap here
    // (normalize limits it to native FP16 FWHT, a storage gap of this build).
    const bool epilogue = d.output_scale != 1.0 || d.output_rounding != CUBUTTERFLY_ROUNDING_STAGE_STORAGE;
    switch (d.op) {
        case CUBUTTERFLY_OPERATOR_FFT:
            if (!(d.storage == CUBUTTERFLY_DATA_COMPLEX_FP64 && d.compute == CUBUTTERFLY_COMPUTE_FP64 && !real_fft) &&
                ((d.storage != CUBUTTERFLY_DATA_COMPLEX_FP32 && !real_fft) || d.compute != CUBUTTERFLY_COMPUTE_FP32))
                gap("storage-lowering",
                    "FFT executes complex FP32 (FP32 for R2C/C2R) with FP32 compute, or complex FP64 with FP64 compute");
            if (epilogue) gap("output-epilogue-lowering", "output epilogues apply to FWHT only");
            if (n > (std::size_t{1} << 30)) gap("length-lowering", "FFT length is limited to 2^30");
            break;
        case CUBUTTERFLY_OPERATOR_FWHT: {
            // FP64 runs as the structured 2x2 butterfly with H_2 in every stage
            // (bit-identical to the reference's double FWHT), no epilogue
            const bool f64 = d.storage == CUBUTTERFLY_DATA_FP64 && d.compute == CUBUTTERFLY_COMPUTE_FP64;
            if (f64) {
                if (epilogue) gap("output-epilogue-lowering", "FP64 FWHT takes no output epilogue");
                if (!natural_in || !natural_out) gap("order-lowering", "FP64 FWHT executes natural logical orders");
                break;
            }
            // bf16 / fp16 with NATIVE compute: stage-storage rounding (the
            // reference's default low-precision FWHT), no epilogue
            const bool native_low = (d.storage == CUBUTTERFLY_DATA_BF16 || d.storage == CUBUTTERFLY_DATA_FP16) &&
                                    d.compute == CUBUTTERFLY_COMPUTE_NATIVE &&
                                    d.output_rounding == CUBUTTERFLY_ROUNDING_STAGE_STORAGE;
            if (native_low) {
                if (d.output_scale != 1.0)
                    gap("output-epilogue-lowering", "native low-precision FWHT takes no output scale");
                if (!natural_in || !natural_out)
                    gap("order-lowering", "native low-precision FWHT executes natural logical orders");
                break;
            }
            const bool f32 = d.storage == CUBUTTERFLY_DATA_FP32 && d.compute == CUBUTTERFLY_COMPUTE_FP32;
            const bool low = (d.storage == CUBUTTERFLY_DATA_BF16 || d.storage == CUBUTTERFLY_DATA_FP16) &&
                             d.compute == CUBUTTERFLY_COMPUTE_FP32 &&
                             d.output_rounding == CUBUTTERFLY_ROUNDING_FINAL_STORAGE;
            if (!f32 && !low)
                gap("storage-lowering",
                    "FWHT executes FP32 storage, or BF16/FP16 storage with FP32 compute and final-storage rounding");
            if (epilogue && !low && !(f32 && d.output_rounding == CUBUTTERFLY_ROUNDING_STAGE_STORAGE))
                gap("output-epilogue-lowering", "output epilogue requires FP32 compute");
            if (!std::isfinite(static_cast<float>(d.output_scale)))
                gap("output-scale-lowering", "output scale must be representable as finite FP32");
            if (n > (std::size_t{1} << 15)) gap("length-lowering", "FWHT length is limited to 2^15");
            break;
        }
        case CUBUTTERFLY_OPERATOR_SUBSET_ZETA:
        case CUBUTTERFLY_OPERATOR_SUPERSET_ZETA:
            if (d.storage != CUBUTTERFLY_DATA_UINT32 && d.storage != CUBUTTERFLY_DATA_UINT64)
                gap("storage-lowering", "zeta kernels require uint32 or uint64 storage");
            if (epilogue) gap("output-epilogue-lowering", "output epilogues apply to FWHT only");
            if (n > (std::size_t{1} << 30)) gap("length-lowering", "zeta length is limited to 2^30");
            break;
        case CUBUTTERFLY_OPERATOR_NTT:
            // Cyclic NTT over uint32 / uint64 words (word bits = storage
            // bits, checked by normalize); modulus primality, q < 2^63 and
            // 2^log_n | q - 1 are plan-time validation (INVALID_VALUE), as
            // in the reference's plan constructor.
            if (epilogue) gap("output-epilogue-lowering", "output epilogues apply to FWHT only");
            if (n > (std::size_t{1} << 20))
                gap("length-lowering", "NTT length is limited to 2^20 (the reference's direct NTT range)");
            break;
        case CUBUTTERFLY_OPERATOR_STRUCTURED_2X2:
            // fp32 / fp64 storage computed in its own precision; ranks two and
            // three run over the flattened index with the axes' stage lists
            // concatenated (innermost axis = lowest bits)
            if ((d.storage != CUBUTTERFLY_DATA_FP32 || d.compute != CUBUTTERFLY_COMPUTE_FP32) &&
                (d.storage != CUBUTTERFLY_DATA_FP64 || d.compute != CUBUTTERFLY_COMPUTE_FP64))
                gap("storage-lowering", "structured 2x2 executes FP32 or FP64 storage in its own precision");
            if (!natural_in || !natural_out) gap("order-lowering", "structured 2x2 executes natural logical orders");
            if (epilogue) gap("output-epilogue-lowering", "output epilogues apply to FWHT only");
            if (n > (std::size_t{1} << 30)) gap("length-lowering", "structured 2x2 length is limited to 2^30");
            break;
    }
    if (!layout_nonoverlapping(in, d.input_strides, d.batch, d.input_batch_stride) ||
        !layout_nonoverlapping(out, d.output_strides, d.batch, d.output_batch_stride))
        gap("layout-proof-unavailable", "non-overlap of this layout was not established by bounded validation");
    return {{"schema", "cubutterfly-capabilities-v1"},
            {"semantic_contract", semantic_json(d)},
            {"status", gaps.empty() ? "eligible" : "missing-lowering"},
            {"gaps", gaps},
            {"validation_scope", "CPU structural semantics and static lowering constraints of cubutterfly_b200"},
            {"boundary_adapter", false},
            {"performance_verified", false}};
}

}  // namespace cubf
