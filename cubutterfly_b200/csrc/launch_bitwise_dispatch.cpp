// launch_bitwise_dispatch.cpp -- routes a BwVariant to its compiled unit.
#include "kernels.hpp"

namespace cubf {

#define CUBF_DECLARE_UNIT(OP, TY)                                                                       \
    LaunchShape bw_unit_##OP##_##TY##_shape(int log_h, int log_w);                                      \
    cudaError_t bw_unit_##OP##_##TY##_launch(int log_h, int log_w, const void* in, void* out,          \
                                             std::size_t outer, std::size_t inner, bool inverse,       \
                                             float scale, int cache_mode, cudaStream_t stream);        \
    cudaError_t bw_unit_##OP##_##TY##_chain(const BwChain& c, const void* in, void* out, cudaStream_t stream);
CUBF_DECLARE_UNIT(0, 0)
CUBF_DECLARE_UNIT(0, 1)
CUBF_DECLARE_UNIT(0, 2)
CUBF_DECLARE_UNIT(1, 3)
CUBF_DECLARE_UNIT(1, 4)
CUBF_DECLARE_UNIT(2, 3)
CUBF_DECLARE_UNIT(2, 4)
#undef CUBF_DECLARE_UNIT

namespace {
using ShapeFn = LaunchShape (*)(int, int);
using LaunchFn = cudaError_t (*)(int, int, const void*, void*, std::size_t, std::size_t, bool, float, int,
                                 cudaStream_t);
using ChainFn = cudaError_t (*)(const BwChain&, const void*, void*, cudaStream_t);
struct Unit {
    ShapeFn shape;
    LaunchFn launch;
    ChainFn chain;
};
Unit unit_of(BwOp op, BwType type) {
    switch (op) {
        case BwOp::Fwht:
            if (type == BwType::F32) return {bw_unit_0_0_shape, bw_unit_0_0_launch, bw_unit_0_0_chain};
            if (type == BwType::BF16) return {bw_unit_0_1_shape, bw_unit_0_1_launch, bw_unit_0_1_chain};
            if (type == BwType::F16) return {bw_unit_0_2_shape, bw_unit_0_2_launch, bw_unit_0_2_chain};
            break;
        case BwOp::ZetaSubset:
            if (type == BwType::U32) return {bw_unit_1_3_shape, bw_unit_1_3_launch, bw_unit_1_3_chain};
            if (type == BwType::U64) return {bw_unit_1_4_shape, bw_unit_1_4_launch, bw_unit_1_4_chain};
            break;
        case BwOp::ZetaSuperset:
            if (type == BwType::U32) return {bw_unit_2_3_shape, bw_unit_2_3_launch, bw_unit_2_3_chain};
            if (type == BwType::U64) return {bw_unit_2_4_shape, bw_unit_2_4_launch, bw_unit_2_4_chain};
            break;
    }
    return {nullptr, nullptr, nullptr};
}
}  // namespace

const char* bw_type_name(BwType t) {
    switch (t) {
        case BwType::F32: return "f32";
        case BwType::BF16: return "bf16";
        case BwType::F16: return "f16";
        case BwType::U32: return "u32";
        case BwType::U64: return "u64";
    }
    return "?";
}
std::size_t bw_type_bytes(BwType t) {
    switch (t) {
        case BwType::BF16:
        case BwType::F16: return 2;
        case BwType::F32:
        case BwType::U32: return 4;
        case BwType::U64: return 8;
    }
    return 0;
}
int bw_strided_log_w(BwType t) { return bw_type_bytes(t) == 8 ? 3 : (bw_type_bytes(t) == 4 ? 4 : 5); }
int bw_max_contiguous_log(BwType t) { return t == BwType::U64 ? 13 : 14; }
int bw_max_strided_log(BwType t) { return t == BwType::U64 ? 9 : 10; }

bool bw_available(const BwVariant& v) { return bw_shape(v).threads > 0; }

LaunchShape bw_shape(const BwVariant& v) {
    const Unit u = unit_of(v.op, v.type);
    return u.shape ? u.shape(v.log_h, v.log_w) : LaunchShape{};
}

cudaError_t launch_bw(const BwVariant& v, const void* in, void* out, std::size_t outer, std::size_t inner,
                      bool inverse, float scale, int cache_mode, cudaStream_t stream) {
    const Unit u = unit_of(v.op, v.type);
    if (!u.launch) return cudaErrorInvalidValue;
    return u.launch(v.log_h, v.log_w, in, out, outer, inner, inverse, scale, cache_mode, stream);
}

bool bw_chain_available(BwOp op, BwType type, int log_h0, int log_h1) {
    return op != BwOp::Fwht && unit_of(op, type).chain != nullptr && log_h0 == bw_max_contiguous_log(type) &&
           log_h1 >= 1 && log_h1 <= bw_max_strided_log(type);
}

cudaError_t launch_bw_chain(BwOp op, BwType type, const BwChain& c, const void* in, void* out, cudaStream_t stream) {
    const Unit u = unit_of(op, type);
    if (!u.chain || op == BwOp::Fwht) return cudaErrorInvalidValue;
    return u.chain(c, in, out, stream);
}

}  // namespace cubf
