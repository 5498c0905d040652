// launch_ntt_dispatch.cpp -- routes NTT launches to the 32- or 64-bit word
// object of launch_ntt.cu.
#include "kernels.hpp"

namespace cubf {
namespace detail {
LaunchShape ntt_shape_w64(const NttVariant& v);
LaunchShape ntt_shape_w32(const NttVariant& v);
cudaError_t launch_ntt_w64(const NttVariant& v, const NttLaunch& a, cudaStream_t stream);
cudaError_t launch_ntt_w32(const NttVariant& v, const NttLaunch& a, cudaStream_t stream);
}  // namespace detail

bool ntt_available(const NttVariant& v) { return v.log_n >= kNttMinLog && v.log_n <= kNttMaxLog; }

bool ntt_single_available(int log_n) { return log_n >= 1 && log_n <= kNttSingleMaxLog; }

LaunchShape ntt_shape(const NttVariant& v) {
    return v.word32 ? detail::ntt_shape_w32(v) : detail::ntt_shape_w64(v);
}

cudaError_t launch_ntt(const NttVariant& v, const NttLaunch& a, cudaStream_t stream) {
    if (a.reduce_input && a.tables.unit_q == nullptr) return cudaErrorInvalidValue;
    return v.word32 ? detail::launch_ntt_w32(v, a, stream) : detail::launch_ntt_w64(v, a, stream);
}

}  // namespace cubf
