// launch_ntt.cu -- instantiations and launchers of the RNS NTT tile passes.
#include "kernels.hpp"
#include "launch_util.cuh"
#include "ntt.cuh"

namespace cubf {
namespace {

template <int L, bool STRIDED, bool INV, bool LAZY>
struct Entry {
    using S = ntt::PassShape<L, STRIDED, INV, LAZY>;
    static LaunchShape shape() {
        LaunchShape s;
        s.threads = S::TPB;
        s.smem_bytes = S::SMEM_BYTES;
        s.units_per_cta = S::COLS;
        s.elems_per_thread = S::E;
        s.exchanges = S::Gs::COUNT - 1;
        return s;
    }
    static cudaError_t launch(const std::uint64_t* in, std::uint64_t* out, const NttPolyDesc* polys,
                              std::size_t poly_count, const NttTables& t, bool in_is_out, bool final_pass,
                              bool final_scale, cudaStream_t stream) {
        auto kernel = ntt::ntt_pass_kernel<L, STRIDED, INV, LAZY>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, S::TPB, S::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        constexpr std::size_t groups = (std::size_t{1} << (L - S::B)) / S::COLS;
        const std::size_t blocks = poly_count * groups;
        if (blocks == 0) return cudaSuccess;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        ntt::DomainTables tab{reinterpret_cast<const ntt::u64*>(t.roots),
                              reinterpret_cast<const ntt::u64*>(t.quotients),
                              reinterpret_cast<const ntt::u64*>(t.moduli), reinterpret_cast<const ntt::u64*>(t.n_inv),
                              reinterpret_cast<const ntt::u64*>(t.n_inv_q)};
        kernel<<<static_cast<unsigned>(blocks), S::TPB, S::SMEM_BYTES, stream>>>(
            reinterpret_cast<const ntt::u64*>(in), reinterpret_cast<ntt::u64*>(out),
            reinterpret_cast<const ntt::PolyDesc*>(polys), tab, in_is_out ? 1 : 0, final_pass ? 1 : 0,
            final_scale ? 1 : 0);
        return cudaGetLastError();
    }
};

using LaunchFn = cudaError_t (*)(const std::uint64_t*, std::uint64_t*, const NttPolyDesc*, std::size_t,
                                 const NttTables&, bool, bool, bool, cudaStream_t);
using ShapeFn = LaunchShape (*)();

template <bool STRIDED, bool INV, bool LAZY, int... L>
struct Row {
    static constexpr LaunchFn launch[] = {Entry<L, STRIDED, INV, LAZY>::launch...};
    static constexpr ShapeFn shape[] = {Entry<L, STRIDED, INV, LAZY>::shape...};
};
#define CUBF_NTT_LOGS 12, 13, 14, 15, 16, 17, 18, 19, 20
// [inverse][strided][lazy]
template <bool INV, bool STRIDED>
struct Rows {
    using Strict = Row<STRIDED, INV, false, CUBF_NTT_LOGS>;
    using Lazy = Row<STRIDED, INV, true, CUBF_NTT_LOGS>;
};

static_assert(sizeof(NttPolyDesc) == sizeof(ntt::PolyDesc), "poly descriptor layout");

int slot(const NttVariant& v) {
    if (v.log_n < kNttMinLog || v.log_n > kNttMaxLog) return -1;
    return v.log_n - kNttMinLog;
}

}  // namespace

bool ntt_available(const NttVariant& v) { return slot(v) >= 0; }

LaunchShape ntt_shape(const NttVariant& v) {
    const int s = slot(v);
    if (s < 0) return {};
    ShapeFn const* t;
    if (!v.inverse)
        t = v.strided ? (v.lazy ? Rows<false, true>::Lazy::shape : Rows<false, true>::Strict::shape)
                      : (v.lazy ? Rows<false, false>::Lazy::shape : Rows<false, false>::Strict::shape);
    else
        t = v.strided ? (v.lazy ? Rows<true, true>::Lazy::shape : Rows<true, true>::Strict::shape)
                      : (v.lazy ? Rows<true, false>::Lazy::shape : Rows<true, false>::Strict::shape);
    return t[s]();
}

cudaError_t launch_ntt_pass(const NttVariant& v, const std::uint64_t* in, std::uint64_t* out,
                            const NttPolyDesc* polys, std::size_t poly_count, const NttTables& tables,
                            bool in_is_out, bool final_pass, bool final_scale, cudaStream_t stream) {
    const int s = slot(v);
    if (s < 0) return cudaErrorInvalidValue;
    LaunchFn const* t;
    if (!v.inverse)
        t = v.strided ? (v.lazy ? Rows<false, true>::Lazy::launch : Rows<false, true>::Strict::launch)
                      : (v.lazy ? Rows<false, false>::Lazy::launch : Rows<false, false>::Strict::launch);
    else
        t = v.strided ? (v.lazy ? Rows<true, true>::Lazy::launch : Rows<true, true>::Strict::launch)
                      : (v.lazy ? Rows<true, false>::Lazy::launch : Rows<true, false>::Strict::launch);
    return t[s](in, out, polys, poly_count, tables, in_is_out, final_pass, final_scale, stream);
}

}  // namespace cubf
