// launch_ntt.cu -- instantiations and launchers of the NTT tile kernels for
// one storage word, chosen by CUBF_NTT_WORD (32 or 64; one object each).
// 64-bit words carry strict and lazy variants (lazy needs every modulus
// < 2^62); 32-bit words always have q < 2^32 and use the lazy variants only.
#include "kernels.hpp"
#include "launch_util.cuh"
#include "ntt.cuh"

#ifndef CUBF_NTT_WORD
#define CUBF_NTT_WORD 64
#endif

namespace cubf {
namespace {

#if CUBF_NTT_WORD == 64
using Word = ntt::u64;
constexpr bool kHasStrict = true;
#else
using Word = unsigned int;
constexpr bool kHasStrict = false;
#endif

ntt::DomainTables device_tables(const NttTables& t) {
    return {reinterpret_cast<const ntt::u64*>(t.root_pairs), reinterpret_cast<const ntt::u64*>(t.moduli),
            reinterpret_cast<const ntt::u64*>(t.n_inv),      reinterpret_cast<const ntt::u64*>(t.n_inv_q),
            reinterpret_cast<const ntt::u64*>(t.unit_q)};
}

template <int L, bool STRIDED, bool INV, bool LAZY, int D = 0>
struct Entry {
    using S = ntt::PassShape<L, STRIDED, INV, LAZY, D>;
    static LaunchShape shape() {
        LaunchShape s;
        s.threads = S::TPB;
        s.smem_bytes = S::SMEM_BYTES;
        s.units_per_cta = S::COLS;
        s.elems_per_thread = S::E;
        s.exchanges = S::Gs::COUNT - 1;
        return s;
    }
    static cudaError_t launch(const NttLaunch& a, cudaStream_t stream) {
        auto kernel = ntt::ntt_pass_kernel<L, STRIDED, INV, LAZY, Word, D>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, S::TPB, S::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        constexpr std::size_t groups = (std::size_t{1} << (L - S::B)) / S::COLS;
        const std::size_t blocks = a.count * groups;
        if (blocks == 0) return cudaSuccess;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        // an ordinary launch: as a programmatic dependent (launch_dependent)
        // the two passes measured slower on config 2 (44.5 against 43.2 us)
        kernel<<<static_cast<unsigned>(blocks), S::TPB, S::SMEM_BYTES, stream>>>(
            static_cast<const Word*>(a.in), static_cast<Word*>(a.out),
            reinterpret_cast<const ntt::PolyDesc*>(a.polys), device_tables(a.tables), a.in_is_out ? 1 : 0,
            a.final_pass ? 1 : 0, a.final_scale ? 1 : 0, a.reduce_input ? 1 : 0);
        return cudaGetLastError();
    }
};

template <int L, bool INV, bool LAZY>
struct SingleEntry {
    using S = ntt::SingleShape<L, INV, LAZY>;
    static LaunchShape shape() {
        LaunchShape s;
        s.threads = S::TPB;
        s.smem_bytes = S::SMEM_BYTES;
        s.units_per_cta = S::COLS;
        s.elems_per_thread = S::E;
        s.exchanges = S::Gs::COUNT - 1;
        return s;
    }
    static cudaError_t launch(const NttLaunch& a, cudaStream_t stream) {
        auto kernel = ntt::ntt_single_kernel<L, INV, LAZY, Word>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, S::TPB, S::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        const std::size_t blocks = (a.count + S::COLS - 1) / S::COLS;
        if (blocks == 0) return cudaSuccess;
        if (blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        kernel<<<static_cast<unsigned>(blocks), S::TPB, S::SMEM_BYTES, stream>>>(
            static_cast<const Word*>(a.in), static_cast<Word*>(a.out), a.count, device_tables(a.tables),
            a.final_scale ? 1 : 0, a.reduce_input ? 1 : 0);
        return cudaGetLastError();
    }
};

using LaunchFn = cudaError_t (*)(const NttLaunch&, cudaStream_t);
using ShapeFn = LaunchShape (*)();

template <bool STRIDED, bool INV, bool LAZY, int... L>
struct Row {
    static constexpr LaunchFn launch[] = {Entry<L, STRIDED, INV, LAZY>::launch...};
    static constexpr ShapeFn shape[] = {Entry<L, STRIDED, INV, LAZY>::shape...};
};
template <int D, bool STRIDED, bool INV, int... L>
struct SplitRow {
    static constexpr LaunchFn launch[] = {Entry<L, STRIDED, INV, true, D>::launch...};
    static constexpr ShapeFn shape[] = {Entry<L, STRIDED, INV, true, D>::shape...};
};
template <bool INV, bool LAZY, int... L>
struct SingleRow {
    static constexpr LaunchFn launch[] = {SingleEntry<L, INV, LAZY>::launch...};
    static constexpr ShapeFn shape[] = {SingleEntry<L, INV, LAZY>::shape...};
};
#define CUBF_NTT_LOGS 12, 13, 14, 15, 16, 17, 18, 19, 20
#define CUBF_NTT_SINGLE_LOGS 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11
static_assert(kNttSingleMaxLog == 11 && kNttMinLog == 12, "instantiated length ranges");

// Pass tables [inverse][strided][lazy]; 32-bit words map strict requests to lazy.
#define CUBF_NTT_SPLIT_LOGS 14, 15, 16, 17, 18
static_assert(kNttSplitMinLog == 14 && kNttSplitMaxLog == 18, "instantiated split range");

template <typename Fn, bool FOR_SHAPE>
Fn pick_split(const NttVariant& v) {
    const int s = v.log_n - kNttSplitMinLog;
#define CUBF_PICK(D, STR, INV)                                                             \
    if constexpr (FOR_SHAPE) return SplitRow<D, STR, INV, CUBF_NTT_SPLIT_LOGS>::shape[s];   \
    else return SplitRow<D, STR, INV, CUBF_NTT_SPLIT_LOGS>::launch[s];
    if (v.split > 0) {
        if (v.strided) {
            if (v.inverse) { CUBF_PICK(1, true, true) } else { CUBF_PICK(1, true, false) }
        } else {
            if (v.inverse) { CUBF_PICK(1, false, true) } else { CUBF_PICK(1, false, false) }
        }
    } else {
        if (v.strided) {
            if (v.inverse) { CUBF_PICK(-1, true, true) } else { CUBF_PICK(-1, true, false) }
        } else {
            if (v.inverse) { CUBF_PICK(-1, false, true) } else { CUBF_PICK(-1, false, false) }
        }
    }
#undef CUBF_PICK
}

template <typename Fn, bool FOR_SHAPE>
Fn pick_pass(const NttVariant& v) {
    const bool lazy = v.lazy || !kHasStrict;
    if (v.split != 0) return pick_split<Fn, FOR_SHAPE>(v);
    const int s = v.log_n - kNttMinLog;
#define CUBF_PICK(INV, STR)                                                                              \
    if (lazy) {                                                                                          \
        if constexpr (FOR_SHAPE) return Row<STR, INV, true, CUBF_NTT_LOGS>::shape[s];                    \
        else return Row<STR, INV, true, CUBF_NTT_LOGS>::launch[s];                                       \
    } else {                                                                                             \
        if constexpr (FOR_SHAPE) return Row<STR, INV, !kHasStrict, CUBF_NTT_LOGS>::shape[s];             \
        else return Row<STR, INV, !kHasStrict, CUBF_NTT_LOGS>::launch[s];                                \
    }
    if (!v.inverse) {
        if (v.strided) { CUBF_PICK(false, true) } else { CUBF_PICK(false, false) }
    } else {
        if (v.strided) { CUBF_PICK(true, true) } else { CUBF_PICK(true, false) }
    }
#undef CUBF_PICK
}

template <typename Fn, bool FOR_SHAPE>
Fn pick_single(const NttVariant& v) {
    const bool lazy = v.lazy || !kHasStrict;
    const int s = v.log_n - 1;
#define CUBF_PICK(INV)                                                                            \
    if (lazy) {                                                                                   \
        if constexpr (FOR_SHAPE) return SingleRow<INV, true, CUBF_NTT_SINGLE_LOGS>::shape[s];     \
        else return SingleRow<INV, true, CUBF_NTT_SINGLE_LOGS>::launch[s];                        \
    } else {                                                                                      \
        if constexpr (FOR_SHAPE) return SingleRow<INV, !kHasStrict, CUBF_NTT_SINGLE_LOGS>::shape[s]; \
        else return SingleRow<INV, !kHasStrict, CUBF_NTT_SINGLE_LOGS>::launch[s];                 \
    }
    if (!v.inverse) {
        CUBF_PICK(false)
    } else {
        CUBF_PICK(true)
    }
#undef CUBF_PICK
}

}  // namespace

namespace detail {
#if CUBF_NTT_WORD == 64
#define CUBF_NTT_FN(name) name##_w64
#else
#define CUBF_NTT_FN(name) name##_w32
#endif

LaunchShape CUBF_NTT_FN(ntt_shape)(const NttVariant& v) {
    if (!ntt_split_available(v.log_n, v.split, v.lazy || !kHasStrict)) return {};
    if (v.log_n >= kNttMinLog && v.log_n <= kNttMaxLog) return pick_pass<ShapeFn, true>(v)();
    if (v.log_n >= 1 && v.log_n <= kNttSingleMaxLog) return pick_single<ShapeFn, true>(v)();
    return {};
}

cudaError_t CUBF_NTT_FN(launch_ntt)(const NttVariant& v, const NttLaunch& a, cudaStream_t stream) {
    if (!ntt_split_available(v.log_n, v.split, v.lazy || !kHasStrict)) return cudaErrorInvalidValue;
    if (v.log_n >= kNttMinLog && v.log_n <= kNttMaxLog) return pick_pass<LaunchFn, false>(v)(a, stream);
    if (v.log_n >= 1 && v.log_n <= kNttSingleMaxLog) return pick_single<LaunchFn, false>(v)(a, stream);
    return cudaErrorInvalidValue;
}
#undef CUBF_NTT_FN
}  // namespace detail

}  // namespace cubf
