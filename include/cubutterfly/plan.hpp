// plan.hpp -- header-only C++ owners over the C ABI of cubutterfly_b200.
//
// The C++ interface of the reference's include/cubutterfly/plan.hpp:12-221:
// cubutterfly::check, Transform, PlanOptions, Context, Descriptor and Plan
// with the same members and meaning, so C++ callers switch by relinking.
// Every failure of the C ABI becomes std::runtime_error("<status>: <last
// error>").  A Plan created with allocate_workspace (the default) owns a
// cudaMalloc'd workspace of exactly the size the plan reports; pass false to
// supply one with set_workspace.
#pragma once

#include <cubutterfly/cubutterfly.h>

#include <cstdint>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace cuntt {
// The library's default NTT modulus (the descriptor default).
inline constexpr std::uint64_t kDefaultModulus = 1152921504606584833ULL;
}  // namespace cuntt

namespace cubutterfly {

inline void check(cubutterflyStatus_t status) {
    if (status == CUBUTTERFLY_STATUS_SUCCESS) return;
    const char* detail = cubutterflyGetLastErrorString();
    std::string message = cubutterflyGetStatusString(status);
    if (detail && *detail) message += std::string(": ") + detail;
    throw std::runtime_error(message);
}

// What to compute; how is the planner's choice (PlanOptions).
struct Transform {
    cubutterflyOperator_t op = CUBUTTERFLY_OPERATOR_FFT;
    cubutterflyDataType_t storage = CUBUTTERFLY_DATA_COMPLEX_FP32;
    cubutterflyComputeType_t compute = CUBUTTERFLY_COMPUTE_NATIVE;
    std::vector<std::size_t> extents{256};
    std::size_t batch = 1;
    std::vector<std::size_t> input_strides, output_strides;  // empty: packed
    std::size_t input_batch_stride = 0, output_batch_stride = 0;
    bool inverse = false, normalize_inverse = true, in_place = false;
    cubutterflyLengthMode_t length_mode = CUBUTTERFLY_LENGTH_STANDARD;
    std::uint64_t modulus = cuntt::kDefaultModulus;
    std::uint32_t word_bits = 64;
    cubutterflyNttLayout_t input_order = CUBUTTERFLY_NTT_LAYOUT_NATURAL;   // legacy NTT layouts
    cubutterflyNttLayout_t output_order = CUBUTTERFLY_NTT_LAYOUT_NATURAL;
    std::vector<cubutterflyLogicalOrder_t> input_orders, output_orders;  // per axis; empty: natural
    std::vector<std::vector<cubutterflyMatrix2x2_t>> stage_matrices;     // per axis (structured 2x2)
    cubutterflyExecutionMode_t execution_mode = CUBUTTERFLY_EXECUTION_AUTO;
    cubutterflyFftTransformType_t fft_type = CUBUTTERFLY_FFT_C2C;
    double fft_output_scale = 1.0;
    double output_scale = 1.0;
    cubutterflyOutputRounding_t output_rounding = CUBUTTERFLY_ROUNDING_STAGE_STORAGE;
    cubutterflyArithmeticPolicy_t arithmetic_policy = CUBUTTERFLY_ARITHMETIC_STRICT;
};

struct PlanOptions {
    cubutterflyAlgorithmPolicy_t policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
    std::string mapping;  // non-empty: EXPLICIT with this mapping JSON / pass list / algorithm name
    bool allocate_workspace = true;
    cubutterflyExecutionMode_t execution_mode = CUBUTTERFLY_EXECUTION_AUTO;  // AUTO: Transform's
};

// A handle (stream, plan-cache path, log callback), shared by the plans made from it.
class Context {
    struct Handle {
        cubutterflyHandle_t raw = nullptr;
        Handle() { check(cubutterflyCreate(&raw)); }
        ~Handle() { cubutterflyDestroy(raw); }
        Handle(const Handle&) = delete;
        Handle& operator=(const Handle&) = delete;
    };
    std::shared_ptr<Handle> handle_ = std::make_shared<Handle>();

  public:
    void set_stream(cudaStream_t stream) { check(cubutterflySetStream(handle_->raw, stream)); }
    void set_cache_path(const std::string& path) { check(cubutterflySetCachePath(handle_->raw, path.c_str())); }
    void set_logger(cubutterflyLogCallback_t logger, void* user = nullptr) {
        check(cubutterflySetLogCallback(handle_->raw, logger, user));
    }
    cubutterflyHandle_t native_handle() const noexcept { return handle_->raw; }
};

namespace detail {
// Two-call string query: size (with the terminating NUL), then the text.
template <typename Object, typename Query>
std::string query_text(Object object, Query query) {
    std::size_t bytes = 0;
    check(query(object, nullptr, &bytes));
    std::string text(bytes, '\0');
    check(query(object, text.data(), &bytes));
    while (!text.empty() && text.back() == '\0') text.pop_back();
    return text;
}
}  // namespace detail

class Descriptor {
    struct Release {
        void operator()(cubutterflyDescriptor_t d) const noexcept { cubutterflyDestroyDescriptor(d); }
    };
    std::unique_ptr<std::remove_pointer_t<cubutterflyDescriptor_t>, Release> raw_;

    Descriptor() {
        cubutterflyDescriptor_t d = nullptr;
        check(cubutterflyCreateDescriptor(&d));
        raw_.reset(d);
    }

  public:
    Descriptor(const Transform& t, const PlanOptions& options = {}) : Descriptor() {
        const cubutterflyDescriptor_t d = native_handle();
        const std::size_t rank = t.extents.size();
        if (rank > std::numeric_limits<std::uint32_t>::max())
            throw std::invalid_argument("rank exceeds the uint32 C ABI range");
        for (std::size_t count : {t.input_strides.size(), t.output_strides.size(), t.input_orders.size(),
                                  t.output_orders.size()})
            if (count != 0 && count != rank) throw std::invalid_argument("one entry is required per axis");
        const bool legacy_layouts =
            t.input_order != CUBUTTERFLY_NTT_LAYOUT_NATURAL || t.output_order != CUBUTTERFLY_NTT_LAYOUT_NATURAL;
        if (legacy_layouts && t.op != CUBUTTERFLY_OPERATOR_NTT)
            throw std::invalid_argument("legacy NTT layouts require an NTT operator");
        if (t.op != CUBUTTERFLY_OPERATOR_NTT && (t.modulus != cuntt::kDefaultModulus || t.word_bits != 64))
            throw std::invalid_argument("modulus and word_bits require an NTT operator");
        if (legacy_layouts && (!t.input_orders.empty() || !t.output_orders.empty()))
            throw std::invalid_argument("legacy NTT layouts and logical orders are ambiguous");
        check(cubutterflySetOperator(d, t.op));
        check(cubutterflySetDataType(d, t.storage, t.compute));
        check(cubutterflySetShape(d, static_cast<std::uint32_t>(rank), t.extents.data(), t.batch));
        check(cubutterflySetExecutionMode(
            d, options.execution_mode != CUBUTTERFLY_EXECUTION_AUTO ? options.execution_mode : t.execution_mode));
        check(cubutterflySetFftTransformType(d, t.fft_type));
        check(cubutterflySetFftOutputScale(d, t.fft_output_scale));
        check(cubutterflySetOutputScale(d, t.output_scale));
        check(cubutterflySetOutputRounding(d, t.output_rounding));
        check(cubutterflySetArithmeticPolicy(d, t.arithmetic_policy));
        check(cubutterflySetStrides(d, t.input_strides.empty() ? nullptr : t.input_strides.data(),
                                    t.input_batch_stride, t.output_strides.empty() ? nullptr : t.output_strides.data(),
                                    t.output_batch_stride));
        check(cubutterflySetDirection(d, t.inverse ? CUBUTTERFLY_DIRECTION_INVERSE : CUBUTTERFLY_DIRECTION_FORWARD,
                                      t.normalize_inverse ? 1 : 0));
        check(cubutterflySetPlacement(d, t.in_place ? CUBUTTERFLY_PLACEMENT_IN_PLACE : CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE));
        check(cubutterflySetLengthMode(d, t.length_mode));
        check(cubutterflySetAlgorithmPolicy(d, options.mapping.empty() ? options.policy : CUBUTTERFLY_ALGORITHM_EXPLICIT,
                                            options.mapping.c_str()));
        if (t.op == CUBUTTERFLY_OPERATOR_NTT) {
            check(cubutterflySetModulus(d, t.modulus, t.word_bits));
            check(cubutterflySetNttLayouts(d, t.input_order, t.output_order));
        }
        if (!legacy_layouts)
            check(cubutterflySetLogicalOrders(d, t.input_orders.empty() ? nullptr : t.input_orders.data(),
                                              t.output_orders.empty() ? nullptr : t.output_orders.data()));
        for (std::size_t axis = 0; axis < t.stage_matrices.size(); ++axis) {
            if (t.stage_matrices[axis].empty()) continue;
            check(cubutterflySetStageMatrices(d, static_cast<std::uint32_t>(axis), t.stage_matrices[axis].data(),
                                              t.stage_matrices[axis].size()));
        }
    }
    Descriptor(Descriptor&&) noexcept = default;
    Descriptor& operator=(Descriptor&&) noexcept = default;
    Descriptor(const Descriptor&) = delete;
    Descriptor& operator=(const Descriptor&) = delete;

    static Descriptor from_json(const std::string& json) {
        Descriptor d;
        check(cubutterflyDescriptorSetJson(d.native_handle(), json.c_str()));
        return d;
    }
    void validate() const { check(cubutterflyDescriptorValidate(native_handle())); }
    std::string json() const { return detail::query_text(native_handle(), cubutterflyDescriptorGetJson); }
    std::string capabilities_json() const {
        return detail::query_text(native_handle(), cubutterflyDescriptorGetCapabilities);
    }
    cubutterflyDescriptor_t native_handle() const noexcept { return raw_.get(); }
};

class Plan {
    struct Owned {
        Context context;
        cubutterflyPlan_t raw = nullptr;
        void* workspace = nullptr;
        explicit Owned(const Context& c) : context(c) {}
        ~Owned() {
            cubutterflyDestroyPlan(raw);
            if (workspace) cudaFree(workspace);
        }
        Owned(const Owned&) = delete;
        Owned& operator=(const Owned&) = delete;
    };
    std::unique_ptr<Owned> owned_;

    std::size_t size_of(cubutterflyStatus_t (*query)(cubutterflyPlan_t, std::size_t*)) const {
        std::size_t bytes = 0;
        check(query(owned_->raw, &bytes));
        return bytes;
    }

  public:
    Plan(const Context& context, const Transform& transform, const PlanOptions& options = {})
        : Plan(context, Descriptor(transform, options), options.allocate_workspace) {}
    Plan(const Context& context, const Descriptor& descriptor, bool allocate_workspace = true)
        : owned_(std::make_unique<Owned>(context)) {
        check(cubutterflyCreatePlan(context.native_handle(), descriptor.native_handle(), &owned_->raw));
        const std::size_t bytes = workspace_size();
        if (allocate_workspace && bytes) {
            const cudaError_t e = cudaMalloc(&owned_->workspace, bytes);
            if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
            check(cubutterflyPlanSetWorkspace(owned_->raw, owned_->workspace, bytes));
        }
    }
    Plan(Plan&&) noexcept = default;
    Plan& operator=(Plan&&) noexcept = default;
    Plan(const Plan&) = delete;
    Plan& operator=(const Plan&) = delete;

    std::size_t workspace_size() const { return size_of(cubutterflyPlanGetWorkspaceSize); }
    std::size_t input_size() const { return size_of(cubutterflyPlanGetInputSize); }
    std::size_t output_size() const { return size_of(cubutterflyPlanGetOutputSize); }
    void set_workspace(void* pointer, std::size_t bytes) { check(cubutterflyPlanSetWorkspace(owned_->raw, pointer, bytes)); }
    void execute(const void* input, void* output) {
        check(cubutterflyExecute(owned_->context.native_handle(), owned_->raw, input, output));
    }
    void execute_steady(const void* input, void* output) {
        check(cubutterflyExecuteSteady(owned_->context.native_handle(), owned_->raw, input, output));
    }
    std::string mapping_json() const { return detail::query_text(owned_->raw, cubutterflyPlanGetMappingJson); }
    std::string descriptor_json() const { return detail::query_text(owned_->raw, cubutterflyPlanGetDescriptorJson); }
    std::string selection_reason() const { return detail::query_text(owned_->raw, cubutterflyPlanGetSelectionReason); }
    std::string algorithm_name() const { return detail::query_text(owned_->raw, cubutterflyPlanGetAlgorithmName); }
    cubutterflySelectionSource_t selection_source() const {
        cubutterflySelectionSource_t source;
        check(cubutterflyPlanGetSelectionSource(owned_->raw, &source));
        return source;
    }
    cubutterflyPlan_t native_handle() const noexcept { return owned_->raw; }
};

}  // namespace cubutterfly
