// fft_pair.cuh -- in-CTA complex fp32 FFT on column pairs (f32x2 Stockham).
//
// Same transform and pass schedule as fft_local_kernel (Stockham autosort,
// radix <= 16 passes, natural order in and out, forward kernels serving the
// inverse through conj(FFT(conj(x)))), organised for the packed fp32 pipe:
// every thread processes two adjacent columns j, j+1 of each pass together,
// holding them split by component -- one 64-bit register pair with
// (re_j, re_j+1) and one with (im_j, im_j+1).  Every complex add, subtract
// and multiply of the radix codelets then acts on both columns with one
// add/sub/mul/fma.rn.f32x2, the multiply by -i is a renaming, and the
// shared-memory exchange keeps separate real and imaginary planes so both
// columns move with one 64-bit access.  Inter-pass twiddles come from a
// per-plan table in global memory (L1-resident): one 16-byte entry
// (re_j, re_j+1, im_j, im_j+1) per column pair and radix index, each value
// computed in double and rounded once to fp32.
#pragma once

#include "f32x2.cuh"

#include <type_traits>
#include <utility>

namespace cubf::fft {

using f32x2::P;
using f32x2::pk;
using f32x2::up;

// Two complex values (columns j and j+1), split by component.
struct CP {
    P re, im;
};

CUBF_DEV CP cp_add(CP a, CP b) { return {f32x2::add2(a.re, b.re), f32x2::add2(a.im, b.im)}; }
CUBF_DEV CP cp_sub(CP a, CP b) { return {f32x2::sub2(a.re, b.re), f32x2::sub2(a.im, b.im)}; }

// a * w for per-column twiddles w = (re pair, im pair).
CUBF_DEV CP cp_mul(CP a, CP w) {
    using namespace f32x2;
    return {sub2(mul2(a.re, w.re), mul2(a.im, w.im)), fma2(a.re, w.im, mul2(a.im, w.re))};
}

// W_16^k = exp(-2 pi i k / 16) for k < 8: the constants of fft.cuh's w16.
struct W16 {
    static constexpr float c1 = 0.923879532511286756128f;  // cos(pi/8)
    static constexpr float s1 = 0.382683432365089771728f;  // sin(pi/8)
    static constexpr float r2 = 0.707106781186547524401f;  // sqrt(2)/2
    static constexpr float re[8] = {1.f, c1, r2, s1, 0.f, -s1, -r2, -c1};
    static constexpr float im[8] = {0.f, -s1, -r2, -c1, -1.f, -c1, -r2, -s1};
};

// Radix-2 butterfly (e, o) -> (e + W_16^K o, e - W_16^K o) on both columns.
template <int K>
CUBF_DEV void cp_bfly(CP& e, CP& o) {
    using namespace f32x2;
    if constexpr (K == 0) {
        const CP x = cp_add(e, o), y = cp_sub(e, o);
        e = x;
        o = y;
    } else if constexpr (K == 4) {
        // W_16^4 o = -i o = (o.im, -o.re)
        const CP x = {add2(e.re, o.im), sub2(e.im, o.re)};
        const CP y = {sub2(e.re, o.im), add2(e.im, o.re)};
        e = x;
        o = y;
    } else {
        const P wr = pk(W16::re[K], W16::re[K]);
        const P wi = pk(W16::im[K], W16::im[K]);
        const CP t = {sub2(mul2(o.re, wr), mul2(o.im, wi)), fma2(o.re, wi, mul2(o.im, wr))};
        const CP x = cp_add(e, t), y = cp_sub(e, t);
        e = x;
        o = y;
    }
}

// In-register forward DFT of length R on v[0..R) (natural order in and out),
// recursive radix-2 DIT as Dft<R> in fft.cuh.
template <int R>
struct PairDft {
    template <int... K>
    static CUBF_DEV void combine(CP* e, CP* o, std::integer_sequence<int, K...>) {
        (cp_bfly<K * (16 / R)>(e[K], o[K]), ...);
    }
    static CUBF_DEV void run(CP* v) {
        CP e[R / 2], o[R / 2];
#pragma unroll
        for (int i = 0; i < R / 2; ++i) {
            e[i] = v[2 * i];
            o[i] = v[2 * i + 1];
        }
        PairDft<R / 2>::run(e);
        PairDft<R / 2>::run(o);
        combine(e, o, std::make_integer_sequence<int, R / 2>{});
#pragma unroll
        for (int k = 0; k < R / 2; ++k) {
            v[k] = e[k];
            v[k + R / 2] = o[k];
        }
    }
};
template <>
struct PairDft<1> {
    static CUBF_DEV void run(CP*) {}
};

// Shape of the column-pair kernel for 2^LOGN points: T = N/32 threads per
// transform (16 values of each of 2 columns per pass), ceil(LOGN/4) passes.
template <int LOGN>
struct PairShape {
    static constexpr int N = 1 << LOGN;
    static constexpr int T = N / 32;
    static constexpr int NPASS = (LOGN + 3) / 4;
    static constexpr int radix_bits(int p) { return LOGN / NPASS + (p < LOGN % NPASS ? 1 : 0); }
    static constexpr int ns_bits(int p) {
        int s = 0;
        for (int i = 0; i < p; ++i) s += radix_bits(i);
        return s;
    }
    static constexpr int TPB = T >= 128 ? T : 128;
    static constexpr int TPC = TPB / T;  // transforms per CTA
    // One real and one imaginary plane per transform.  Element i lives at
    // pad(i) = i + 2 (i / 32): two floats of padding per 32 spread the
    // strided exchange stores over the banks while keeping 64-bit granules
    // aligned, and pad(i + 32 m) = pad(i) + 34 m, so every access is a
    // per-thread base plus a compile-time offset.
    static CUBF_DEV int pad(int i) { return i + ((i >> 5) << 1); }
    static constexpr int PLANE = N + N / 16 + 2;
    static constexpr int SMEM_BYTES = TPC * 2 * PLANE * 4;
    // Twiddle table: for each pass p >= 1, (R_p - 1) x (NS_p / 2) entries.
    static constexpr int tw_offset(int p) {
        int o = 0;
        for (int i = 1; i < p; ++i) o += ((1 << radix_bits(i)) - 1) * ((1 << ns_bits(i)) / 2);
        return o;
    }
    static constexpr int TW_ENTRIES = tw_offset(NPASS);
    static_assert(LOGN >= 5 && LOGN <= 13, "column-pair kernel covers 2^5 .. 2^13 points");
};

// Offset of element base + off in a padded plane, given pad(base); when
// base's low five bits and off cannot carry into bit 5 the padding of off
// adds on its own (off a multiple of 32, or base + off within one 32-block).
template <int OFF, bool SAME_BLOCK>
CUBF_DEV int pad_add(int pbase, int base) {
    if constexpr (OFF % 32 == 0) return pbase + OFF + ((OFF >> 5) << 1);
    else if constexpr (SAME_BLOCK) return pbase + OFF;
    else return base + OFF + (((base + OFF) >> 5) << 1);
}

template <int N, int... I>
struct Unroll {
    template <typename F>
    static CUBF_DEV void run(F&& f) {
        if constexpr (sizeof...(I) < N) Unroll<N, I..., sizeof...(I)>::run(f);
        else (f(std::integral_constant<int, I>{}), ...);
    }
};

// Pass P, load half: the R inputs x[j + r N/R] of columns j, j+1 (j even),
// the inter-pass twiddles, the radix-R codelets.  `gload(i)` reads HBM (pass
// 0); later passes read the padded planes.
template <int LOGN, int P, typename GLoad, typename AfterLoad>
CUBF_DEV void pair_pass_load(CP (&v)[16], int q, const float4* __restrict__ tw, const float* pre,
                             const float* pim, GLoad gload, AfterLoad after_load) {
    using S = PairShape<LOGN>;
    constexpr int RB = S::radix_bits(P);
    constexpr int R = 1 << RB;
    constexpr int NS = 1 << S::ns_bits(P);
    constexpr int SUB = 16 / R;
    constexpr int STEP = S::N / R;
#pragma unroll
    for (int u = 0; u < SUB; ++u) {
        const int j = 2 * (q + S::T * u);
        if constexpr (P == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) v[u * R + r] = gload(j + r * STEP);
            if (u == SUB - 1) after_load();  // global loads of this thread are issued
        } else {
            const int pj = S::pad(j);
            Unroll<R>::run([&](auto rc) {
                constexpr int r = decltype(rc)::value;
                const int a = pad_add<r * STEP, false>(pj, j);
                v[u * R + r] = CP{*reinterpret_cast<const f32x2::P*>(pre + a), *reinterpret_cast<const f32x2::P*>(pim + a)};
            });
        }
    }
    if constexpr (NS > 1) {
#pragma unroll
        for (int u = 0; u < SUB; ++u) {
            const int jp = (2 * (q + S::T * u) & (NS - 1)) >> 1;
            const float4* t = tw + S::tw_offset(P) + jp;
#pragma unroll
            for (int r = 1; r < R; ++r) {
                const ulonglong2 w = __ldg(reinterpret_cast<const ulonglong2*>(t + (r - 1) * (NS / 2)));
                v[u * R + r] = cp_mul(v[u * R + r], CP{w.x, w.y});
            }
        }
    }
#pragma unroll
    for (int u = 0; u < SUB; ++u) PairDft<R>::run(&v[u * R]);
}

// Pass P, store half: output k of column j goes to (j / NS) NS R + (j mod NS)
// + k NS.  Columns j and j+1 are adjacent there when NS >= 2 (one 64-bit
// store per plane); in pass 0 (NS = 1) they are R apart.  The last pass
// writes HBM through `gstore(i, x)` (i even, both columns).
template <int LOGN, int P, typename GStore>
CUBF_DEV void pair_pass_store(const CP (&v)[16], int q, float* pre, float* pim, GStore gstore) {
    using S = PairShape<LOGN>;
    constexpr int RB = S::radix_bits(P);
    constexpr int R = 1 << RB;
    constexpr int NSB = S::ns_bits(P);
    constexpr int NS = 1 << NSB;
    constexpr int SUB = 16 / R;
    constexpr bool LAST = P == S::NPASS - 1;
#pragma unroll
    for (int u = 0; u < SUB; ++u) {
        const int j = 2 * (q + S::T * u);
        const int hi = (j >> NSB) << (NSB + RB);
        const int base = hi + (j & (NS - 1));
        if constexpr (LAST) {
#pragma unroll
            for (int k = 0; k < R; ++k) gstore(base + k * NS, v[u * R + k]);
        } else if constexpr (NS >= 2) {
            // hi is a multiple of NS R >= 32; (j mod NS) + k NS stays inside a
            // 32-block when NS < 32 (NS divides 32), else k NS is a multiple of 32
            static_assert(NS * R >= 32, "exchange planes assume NS R >= 32");
            const int pb = (NS >= 32) ? S::pad(base) : base + ((hi >> 5) << 1);
            Unroll<R>::run([&](auto kc) {
                constexpr int k = decltype(kc)::value;
                constexpr int off = k * NS;
                const int a = NS >= 32 ? pad_add<off, false>(pb, base) : pb + off + ((off >> 5) << 1);
                *reinterpret_cast<f32x2::P*>(pre + a) = v[u * R + k].re;
                *reinterpret_cast<f32x2::P*>(pim + a) = v[u * R + k].im;
            });
        } else {
            // pass 0: column j at j R + k, column j + 1 at j R + R + k; with
            // R >= 16 both stay in the 32-block of j R (j even)
            const int pb = S::pad(base);
            Unroll<R>::run([&](auto kc) {
                constexpr int k = decltype(kc)::value;
                float r0, r1, m0, m1;
                up(v[u * R + k].re, r0, r1);
                up(v[u * R + k].im, m0, m1);
                const int a0 = R >= 16 ? pb + k : S::pad(base + k);
                const int a1 = R >= 16 ? pb + R + k : S::pad(base + R + k);
                pre[a0] = r0;
                pre[a1] = r1;
                pim[a0] = m0;
                pim[a1] = m1;
            });
        }
    }
}

template <int LOGN, int P>
struct PairPasses {
    template <typename GLoad, typename GStore, typename AfterLoad>
    static CUBF_DEV void run(CP (&v)[16], int q, const float4* __restrict__ tw, float* pre, float* pim,
                             GLoad gload, GStore gstore, AfterLoad after_load) {
        using S = PairShape<LOGN>;
        pair_pass_load<LOGN, P>(v, q, tw, pre, pim, gload, after_load);
        if constexpr (P == S::NPASS - 1) {
            pair_pass_store<LOGN, P>(v, q, pre, pim, gstore);
        } else {
            if constexpr (P > 0) __syncthreads();  // every read of this pass is done
            pair_pass_store<LOGN, P>(v, q, pre, pim, gstore);
            __syncthreads();
            PairPasses<LOGN, P + 1>::run(v, q, tw, pre, pim, gload, gstore, after_load);
        }
    }
};

template <int LOGN>
constexpr int pair_min_blocks() {
    constexpr int tpb = PairShape<LOGN>::TPB;
    return 512 / tpb > 0 ? 512 / tpb : 1;
}

// Batch rows of 2^LOGN packed complex64 (16-byte aligned rows), natural order
// in and out; `inverse` conjugates on load and store, `scale` multiplies the
// outputs.  in may equal out (each transform is read completely before any
// of its outputs is written).
template <int LOGN>
__global__ void __launch_bounds__(PairShape<LOGN>::TPB, pair_min_blocks<LOGN>())
    fft_pair_kernel(const float4* in, float4* out, size_t batch, const float4* __restrict__ tw, int inverse,
                    float scale, unsigned prefetch_stride) {
    using S = PairShape<LOGN>;
    extern __shared__ __align__(16) float smem_f[];
    pdl_begin();
    const int c = threadIdx.x / S::T;
    const int q = threadIdx.x % S::T;
    const size_t row = static_cast<size_t>(blockIdx.x) * S::TPC + c;
    const bool active = row < batch;
    const float4* src = in + (active ? row : 0) * (S::N / 2);
    float4* dst = out + (active ? row : 0) * (S::N / 2);
    float* pre = smem_f + c * 2 * S::PLANE;
    float* pim = pre + S::PLANE;
    const P im_sign = inverse ? pk(-1.f, -1.f) : pk(1.f, 1.f);
    const P s_re = pk(scale, scale);
    const P s_im = inverse ? pk(-scale, -scale) : s_re;
    const bool plain_load = !inverse;
    const bool plain_store = !inverse && scale == 1.0f;
    auto gload = [&](int i) -> CP {
        const float4 f = active ? __ldcs(src + (i >> 1)) : make_float4(0.f, 0.f, 0.f, 0.f);
        CP x{pk(f.x, f.z), pk(f.y, f.w)};
        if (!plain_load) x.im = f32x2::mul2(x.im, im_sign);
        return x;
    };
    auto gstore = [&](int i, CP x) {
        if (!plain_store) {
            x.re = f32x2::mul2(x.re, s_re);
            x.im = f32x2::mul2(x.im, s_im);
        }
        float r0, r1, m0, m1;
        up(x.re, r0, r1);
        up(x.im, m0, m1);
        if (active) __stcs(dst + (i >> 1), make_float4(r0, m0, r1, m1));
    };
    // once this CTA's loads are out, prefetch the tile of the CTA one wave later into L2
    auto after_load = [&]() {
        constexpr size_t tile_bytes = size_t{S::TPC} * S::N * 8;
        const size_t rem = batch % S::TPC;
        prefetch_next_wave(in, tile_bytes, rem ? rem * S::N * 8 : tile_bytes, prefetch_stride);
    };
    CP v[16];
    PairPasses<LOGN, 0>::run(v, q, tw, pre, pim, gload, gstore, after_load);
}

}  // namespace cubf::fft
