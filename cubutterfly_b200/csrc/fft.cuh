// fft.cuh -- complex fp32 FFT kernels for sm_100a (Stockham autosort).
//
// Semantics follow the reference FftOperator / reference_fft
// (src/operator_traits.cuh:223-283, src/butterfly_reference.cpp:392-433):
// X[k] = sum_n x[n] exp(-2 pi i n k / N) forward, +i inverse, optional 1/N.
// The arithmetic organisation is new: Stockham autosort passes of radix 16
// (register codelets built from radix-2 DIT splits with exact-rounded
// constants), natural order in and out with no bit-reversal pass, one HBM
// read and one HBM write per element, twiddles W_N^k from a table computed in
// double on the host and rounded once to fp32 (as butterfly.cu:1502-1514).
// The inverse transform is conj(FFT(conj(x))): the conjugation is folded into
// the load and store so one set of forward kernels serves both directions.
#pragma once

#include "common.cuh"

namespace cubf::fft {

constexpr int log2_const(int x) {
    int l = 0;
    while ((1 << l) < x) ++l;
    return l;
}

CUBF_DEV float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
CUBF_DEV float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
CUBF_DEV float2 cmul(float2 a, float2 b) {
    return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
CUBF_DEV float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }

// W_16^k = exp(-2 pi i k / 16), k in [0, 16), as exact-rounded fp32 pairs.
CUBF_DEV float2 w16(int k) {
    constexpr float c1 = 0.923879532511286756128f;  // cos(pi/8)
    constexpr float s1 = 0.382683432365089771728f;  // sin(pi/8)
    constexpr float r2 = 0.707106781186547524401f;  // sqrt(2)/2
    switch (k & 15) {
        case 0: return make_float2(1.f, 0.f);
        case 1: return make_float2(c1, -s1);
        case 2: return make_float2(r2, -r2);
        case 3: return make_float2(s1, -c1);
        case 4: return make_float2(0.f, -1.f);
        case 5: return make_float2(-s1, -c1);
        case 6: return make_float2(-r2, -r2);
        case 7: return make_float2(-c1, -s1);
        case 8: return make_float2(-1.f, 0.f);
        case 9: return make_float2(-c1, s1);
        case 10: return make_float2(-r2, r2);
        case 11: return make_float2(-s1, c1);
        case 12: return make_float2(0.f, 1.f);
        case 13: return make_float2(s1, c1);
        case 14: return make_float2(r2, r2);
        default: return make_float2(c1, s1);
    }
}

// Multiply by W_16^k with the trivial cases free of multiplies.
CUBF_DEV float2 mul_w16(float2 a, int k) {
    switch (k & 15) {
        case 0: return a;
        case 4: return make_float2(a.y, -a.x);    // * -i
        case 8: return make_float2(-a.x, -a.y);   // * -1
        case 12: return make_float2(-a.y, a.x);   // * +i
        default: return cmul(a, w16(k));
    }
}

// In-register forward DFT of length R (R = 1, 2, 4, 8, 16) on v[0..R), natural
// order in and out: X[k] = E[k] + W_R^k O[k], X[k + R/2] = E[k] - W_R^k O[k].
template <int R>
struct Dft {
    static CUBF_DEV void run(float2* v) {
        float2 e[R / 2], o[R / 2];
#pragma unroll
        for (int i = 0; i < R / 2; ++i) {
            e[i] = v[2 * i];
            o[i] = v[2 * i + 1];
        }
        Dft<R / 2>::run(e);
        Dft<R / 2>::run(o);
#pragma unroll
        for (int k = 0; k < R / 2; ++k) {
            const float2 t = mul_w16(o[k], k * (16 / R));
            v[k] = cadd(e[k], t);
            v[k + R / 2] = csub(e[k], t);
        }
    }
};
template <>
struct Dft<2> {
    static CUBF_DEV void run(float2* v) {
        const float2 a = v[0], b = v[1];
        v[0] = cadd(a, b);
        v[1] = csub(a, b);
    }
};
template <>
struct Dft<1> {
    static CUBF_DEV void run(float2*) {}
};

// Twiddles W_N^k from two small tables in shared memory: W_N^k =
// hi[k >> 6] * lo[k & 63], both factors exact-rounded fp32 (one extra product
// rounding, far below the fp32 FFT error).  N/64 + 64 entries.
template <int LOGN>
struct TwiddleTable {
    static constexpr int LO_BITS = LOGN < 6 ? LOGN : 6;
    static constexpr int NLO = 1 << LO_BITS;
    static constexpr int NHI = 1 << (LOGN - LO_BITS);
    static constexpr int ENTRIES = NLO + NHI;
    static constexpr int BYTES = ENTRIES * 8;
    const float2* lo;
    const float2* hi;
    // fill from a global table of W_M^k (M = N << log_stride), so entry k of
    // this table is tw[k << log_stride]; all threads of the CTA take part
    static CUBF_DEV TwiddleTable load(float2* smem, const float2* __restrict__ tw, int log_stride = 0) {
        for (int i = threadIdx.x; i < NLO; i += blockDim.x) smem[i] = __ldg(tw + (i << log_stride));
        for (int i = threadIdx.x; i < NHI; i += blockDim.x)
            smem[NLO + i] = __ldg(tw + ((i << LO_BITS) << log_stride));
        return TwiddleTable{smem, smem + NLO};
    }
    CUBF_DEV float2 operator()(int k) const {
        if constexpr (NHI == 1) return lo[k];
        else return cmul(hi[k >> LO_BITS], lo[k & (NLO - 1)]);
    }
};

// Pass schedule of an in-CTA transform of 2^LOGN points: ceil(LOGN/4) passes,
// radix bits balanced so every pass has radix <= 16.
template <int LOGN>
struct LocalShape {
    static constexpr int N = 1 << LOGN;
    static constexpr int LOGE = LOGN < 4 ? LOGN : 4;  // values held per thread (log)
    static constexpr int E = 1 << LOGE;
    static constexpr int T = N / E;  // threads per transform
    static constexpr int NPASS = (LOGN + 3) / 4;
    static constexpr int radix_bits(int p) { return LOGN / NPASS + (p < LOGN % NPASS ? 1 : 0); }
    static constexpr int ns_bits(int p) {
        int s = 0;
        for (int i = 0; i < p; ++i) s += radix_bits(i);
        return s;
    }
    // Shared-memory index with one float2 of padding per 16 (bank spread).
    static CUBF_DEV int pad(int i) { return i + (i >> 4); }
    static constexpr int PADDED = N + N / 16;
    static constexpr int TPB = T >= 128 ? T : 128;  // threads per CTA
    static constexpr int TPC = TPB / T;             // transforms per CTA
    static constexpr bool DOUBLE_BUFFER = LOGN <= 12;
    static constexpr int SMEM_BYTES = (DOUBLE_BUFFER ? 2 : 1) * TPC * PADDED * 8 + TwiddleTable<LOGN>::BYTES;
};

// One Stockham pass P of a 2^LOGN transform, split in two halves so the
// caller can place a barrier between the reads and the writes of a pass:
// load R values per sub-DFT, apply the inter-pass twiddle
// W_{Ns R}^{(j mod Ns) r} = W_N^{(j mod Ns) r N/(Ns R)}, run the register DFT;
// then store with the Stockham autosort index.
template <int LOGN, int P, typename Twiddle, typename Load>
CUBF_DEV void pass_load_tw(float2 (&v)[LocalShape<LOGN>::E], int th, Twiddle twf, Load load) {
    using S = LocalShape<LOGN>;
    constexpr int RB = S::radix_bits(P);
    constexpr int R = 1 << RB;
    constexpr int NSB = S::ns_bits(P);
    constexpr int NS = 1 << NSB;
    constexpr int SUB = S::E / R;  // sub-DFTs per thread
#pragma unroll
    for (int u = 0; u < SUB; ++u) {
        const int j = th + S::T * u;
#pragma unroll
        for (int r = 0; r < R; ++r) v[u * R + r] = load(j + r * (S::N / R));
    }
#pragma unroll
    for (int u = 0; u < SUB; ++u) {
        const int j = th + S::T * u;
        if (NS > 1) {
            const int jm = j & (NS - 1);
#pragma unroll
            for (int r = 1; r < R; ++r) v[u * R + r] = cmul(v[u * R + r], twf(jm, r));
        }
        Dft<R>::run(&v[u * R]);
    }
}

// twf(jm, r) = W_{Ns R}^{jm r} = W_N^{(jm r) N / (Ns R)} from a TwiddleTable
template <int LOGN, int P, typename Load>
CUBF_DEV void pass_load(float2 (&v)[LocalShape<LOGN>::E], int th, const TwiddleTable<LOGN>& tw, Load load) {
    using S = LocalShape<LOGN>;
    constexpr int SHIFT = LOGN - S::ns_bits(P) - S::radix_bits(P);
    pass_load_tw<LOGN, P>(v, th, [&](int jm, int r) { return tw((jm * r) << SHIFT); }, load);
}

template <int LOGN, int P, typename Store>
CUBF_DEV void pass_store(const float2 (&v)[LocalShape<LOGN>::E], int th, Store store) {
    using S = LocalShape<LOGN>;
    constexpr int RB = S::radix_bits(P);
    constexpr int R = 1 << RB;
    constexpr int NSB = S::ns_bits(P);
    constexpr int NS = 1 << NSB;
    constexpr int SUB = S::E / R;
#pragma unroll
    for (int u = 0; u < SUB; ++u) {
        const int j = th + S::T * u;
        const int base = ((j >> NSB) << (NSB + RB)) + (j & (NS - 1));
#pragma unroll
        for (int r = 0; r < R; ++r) store(base + r * NS, v[u * R + r]);
    }
}

// Runs passes P..NPASS-1; pass 0 reads HBM, the last pass writes HBM, the
// passes in between exchange through shared memory.
template <int LOGN, int P, bool DB = LocalShape<LOGN>::DOUBLE_BUFFER>
struct Passes {
    template <typename GLoad, typename GStore>
    static CUBF_DEV void run(float2 (&v)[LocalShape<LOGN>::E], int th, const TwiddleTable<LOGN>& tw,
                             float2* buf0, float2* buf1, GLoad gload, GStore gstore) {
        using S = LocalShape<LOGN>;
        if constexpr (P == 0) {
            pass_load<LOGN, 0>(v, th, tw, gload);
        } else {
            const float2* rb = ((P - 1) & 1) ? buf1 : buf0;
            pass_load<LOGN, P>(v, th, tw, [&](int i) { return rb[S::pad(i)]; });
        }
        if constexpr (P == S::NPASS - 1) {
            pass_store<LOGN, P>(v, th, gstore);
        } else {
            if constexpr (!DB && P > 0) __syncthreads();  // reads done before overwrite
            float2* wb = (P & 1) ? buf1 : buf0;
            pass_store<LOGN, P>(v, th, [&](int i, float2 x) { wb[S::pad(i)] = x; });
            __syncthreads();
            Passes<LOGN, P + 1, DB>::run(v, th, tw, buf0, buf1, gload, gstore);
        }
    }
};

// Whole transform in one CTA: batch rows of 2^LOGN packed complex64, natural
// in/out.  `inverse` conjugates on load and store; `scale` multiplies outputs.
template <int LOGN>
__global__ void __launch_bounds__(LocalShape<LOGN>::TPB)
    fft_local_kernel(const float2* in, float2* out, size_t batch,
                     const float2* __restrict__ tw, int inverse, float scale) {
    using S = LocalShape<LOGN>;
    extern __shared__ float2 smem[];
    const int c = threadIdx.x / S::T;
    const int th = threadIdx.x % S::T;
    const size_t row = static_cast<size_t>(blockIdx.x) * S::TPC + c;
    const bool active = row < batch;
    const float2* src = in + row * S::N;
    float2* dst = out + row * S::N;
    float2* buf0 = smem + c * S::PADDED;
    float2* buf1 = S::DOUBLE_BUFFER ? buf0 + S::TPC * S::PADDED : buf0;
    const auto twt = TwiddleTable<LOGN>::load(smem + (S::DOUBLE_BUFFER ? 2 : 1) * S::TPC * S::PADDED, tw);
    __syncthreads();
    const float sgn = inverse ? -1.f : 1.f;
    float2 v[S::E];
    auto gload = [&](int i) -> float2 {
        float2 x = active ? __ldcs(src + i) : make_float2(0.f, 0.f);
        x.y *= sgn;
        return x;
    };
    auto gstore = [&](int i, float2 x) {
        if (active) __stcs(dst + i, make_float2(x.x * scale, x.y * sgn * scale));
    };
    Passes<LOGN, 0>::run(v, th, twt, buf0, buf1, gload, gstore);
}

// ---- multi-pass global Stockham (N > 2^13) -----------------------------------
//
// Pass p of radix R = 2^LOGR over a length-N transform (Ns = 2^ns_bits is the
// product of the earlier radices): for j < N/R, take x[j + n N/R] (n < R),
// multiply by the outer twiddle W_{Ns R}^{(j mod Ns) n}, run the length-R DFT,
// and write y[(j / Ns) Ns R + (j mod Ns) + k Ns].  A CTA takes C >= 16
// adjacent columns j, so every global access is a run of at least 128 bytes:
// it loads the C x R tile into shared memory with the outer twiddle applied,
// runs the in-CTA Stockham passes of LocalShape<LOGR> on each column in the
// same buffer, and scatters the result with a mapping that keeps global
// stores contiguous.  Outer twiddles come from a fp64 recurrence per column
// (one two-level table lookup for the start and one for the step, then fp64
// products), rounded once to fp32.
template <int LOGR, int CW = 0>
struct GlobalPassShape {
    using S = LocalShape<LOGR>;
    static constexpr int R = 1 << LOGR;
    // columns per CTA: CW when given, else >= 16 (runs of >= 128 bytes)
    static constexpr int C = CW ? CW : (S::T >= 16 ? 16 : 256 / S::T);
    static constexpr int TPB = C * S::T;
    static constexpr int RS = S::PADDED + 1;                 // padded row stride (float2)
    static constexpr int TILE = C * R;
    static constexpr int SMEM_BYTES = C * RS * 8 + TwiddleTable<LOGR>::BYTES;
    static_assert(LOGR >= 4 && TPB <= 1024, "global pass radix must be 16..1024");
};

struct OuterTwiddles {
    const double2* lo;  // W_N^k, k < 2^split
    const double2* hi;  // W_N^(k << split)
    int split;
};

CUBF_DEV double2 outer_twiddle_d(const OuterTwiddles& t, size_t k) {
    const double2 a = __ldg(t.lo + (k & ((size_t{1} << t.split) - 1)));
    const double2 b = __ldg(t.hi + (k >> t.split));
    return make_double2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
CUBF_DEV float2 outer_twiddle(const OuterTwiddles& t, size_t k) {
    const double2 w = outer_twiddle_d(t, k);
    return make_float2(static_cast<float>(w.x), static_cast<float>(w.y));
}
CUBF_DEV double2 cmul_d(double2 a, double2 b) {
    return make_double2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// In-place in-CTA passes on one shared-memory buffer: load, barrier, store,
// barrier, per pass.
template <int LOGR, int P>
struct GlobalColumnPasses {
    static CUBF_DEV void run(float2 (&v)[LocalShape<LOGR>::E], int th, const TwiddleTable<LOGR>& tw, float2* row) {
        using S = LocalShape<LOGR>;
        if constexpr (P < S::NPASS) {
            pass_load<LOGR, P>(v, th, tw, [&](int i) { return row[S::pad(i)]; });
            __syncthreads();
            pass_store<LOGR, P>(v, th, [&](int i, float2 x) { row[S::pad(i)] = x; });
            __syncthreads();
            GlobalColumnPasses<LOGR, P + 1>::run(v, th, tw, row);
        }
    }
};

// Interleaved batches (log_v > 0): 2^log_v transforms stored as vector
// elements -- element n of transform l at n 2^log_v + l -- form one array of
// 2^log_n = N 2^log_v values.  A pass over it is the same Stockham pass with
// Ns scaled by 2^log_v (the caller passes ns_bits including log_v), except
// that the outer twiddle depends on the transform index (j mod Ns) >> log_v
// only and is a power of W_N (the outer tables hold W_N).
//
// `outer_shift` > 0 serves a transform of 2^log_n points from outer tables of
// W_M, M = 2^(log_n + outer_shift) (W_N = W_M^(2^outer_shift)).
template <int LOGR, int CW = 0>
__global__ void __launch_bounds__(GlobalPassShape<LOGR, CW>::TPB)
    fft_global_pass_kernel(const float2* src, float2* dst, int log_n, int ns_bits, size_t batch,
                           const float2* __restrict__ tw_r, int tw_log_stride, OuterTwiddles outer, int conj_in,
                           int conj_out, float scale, int log_v, unsigned prefetch_stride, int outer_shift) {
    using G = GlobalPassShape<LOGR, CW>;
    using S = typename G::S;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2* a = reinterpret_cast<float2*>(smem_raw);
    const auto twt = TwiddleTable<LOGR>::load(a + G::C * G::RS, tw_r, tw_log_stride);
    const size_t n = size_t{1} << log_n;
    const size_t cols = n >> LOGR;  // j range
    const size_t ctas_per_batch = cols / G::C;
    const size_t bidx = blockIdx.x / ctas_per_batch;
    const size_t j0 = (blockIdx.x % ctas_per_batch) * G::C;
    const size_t ns = size_t{1} << ns_bits;
    const float2* sb = src + bidx * n;
    float2* db = dst + bidx * n;
    const float in_sgn = conj_in ? -1.f : 1.f;
    const int tshift = log_n - ns_bits - LOGR + outer_shift;         // W_{Ns R}^m = W_M^(m << tshift)
    const size_t tmask = (size_t{1} << (log_n - log_v + outer_shift)) - 1;  // exponents are taken mod M
    // 1. coalesced tile load (runs of C elements), outer twiddle applied.
    //    Thread t handles column c = t % C and rows r = t / C + k (TPB / C).
    {
        constexpr int RSTEP = G::TPB / G::C;
        const int c = threadIdx.x % G::C;
        const size_t j = j0 + c;
        const size_t jm = (j & (ns - 1)) >> log_v;
        const int r0 = threadIdx.x / G::C;
        const bool twiddled = ns_bits > log_v;
        double2 w = make_double2(1.0, 0.0), step = make_double2(1.0, 0.0);
        if (twiddled) {
            w = outer_twiddle_d(outer, ((jm * static_cast<size_t>(r0)) << tshift) & tmask);
            step = outer_twiddle_d(outer, ((jm * static_cast<size_t>(RSTEP)) << tshift) & tmask);
        }
#pragma unroll 4
        for (int r = r0; r < G::R; r += RSTEP) {
            float2 x = __ldcs(sb + j + static_cast<size_t>(r) * cols);
            x.y *= in_sgn;
            if (twiddled) {
                x = cmul(x, make_float2(static_cast<float>(w.x), static_cast<float>(w.y)));
                w = cmul_d(w, step);
            }
            a[c * G::RS + S::pad(r)] = x;
        }
    }
    // loads issued: prefetch the tile of the CTA one resident wave later into L2, one C-column row segment
    // (a run of C * 8 bytes) per thread and row
    if (prefetch_stride != 0 && blockIdx.x + static_cast<size_t>(prefetch_stride) < gridDim.x) {
        const size_t nb = blockIdx.x + static_cast<size_t>(prefetch_stride);
        const float2* nsrc = src + (nb / ctas_per_batch) * n + (nb % ctas_per_batch) * G::C;
        for (int r = threadIdx.x; r < G::R; r += G::TPB) prefetch_l2(nsrc + static_cast<size_t>(r) * cols, G::C * 8);
    }
    __syncthreads();
    // 2. length-R DFT of each column, in place in shared memory
    {
        const int c = threadIdx.x / S::T;
        const int th = threadIdx.x % S::T;
        float2 v[S::E];
        GlobalColumnPasses<LOGR, 0>::run(v, th, twt, a + c * G::RS);
    }
    // 3. scatter: element (c, k) -> y[(j / Ns) Ns R + (j mod Ns) + k Ns], with
    //    the fastest index chosen so consecutive threads write consecutive words
    constexpr int LOG_C = log2_const(G::C);
    const int log_ne = ns_bits < LOG_C ? ns_bits : LOG_C;  // runs of min(Ns, C) columns are contiguous
    const int ne_mask = (1 << log_ne) - 1;
    const float out_sgn = conj_out ? -1.f : 1.f;
    float2* dcol = db + ((j0 >> ns_bits) << (ns_bits + LOGR)) + (j0 & (ns - 1));
#pragma unroll 4
    for (int idx = threadIdx.x; idx < G::TILE; idx += G::TPB) {
        const int c_lo = idx & ne_mask;
        const int k = (idx >> log_ne) & (G::R - 1);
        const int c = ((idx >> (log_ne + LOGR)) << log_ne) | c_lo;
        // j = j0 + c; j0 is a multiple of C, so (j mod Ns) and (j / Ns) split as below
        const size_t o = (static_cast<size_t>(c >> ns_bits) << (ns_bits + LOGR)) + (c & (ns - 1)) +
                         static_cast<size_t>(k) * ns;
        const float2 x = a[c * G::RS + S::pad(k)];
        __stcs(dcol + o, make_float2(x.x * scale, x.y * out_sgn * scale));
    }
}

// ---- register-direct global pass ----------------------------------------------
//
// The same Stockham pass as fft_global_pass_kernel, for the shapes every plan
// uses (the first pass, Ns = 1, and passes with Ns >= C), with the tile never
// staged whole in shared memory: the first in-CTA register phase loads its
// column values straight from HBM and applies the outer twiddle in registers,
// the last one writes straight to HBM, and only the exchanges between the
// in-CTA phases use shared memory (one exchange up to radix 2^8).  A column
// of R values is served by T = R / 16 threads of 16 values each.  Loads put
// the C columns of a CTA on consecutive threads, so a warp reads whole
// C-column runs of two or more rows; stores do the same for Ns >= C (runs of
// C columns at row stride Ns), and for Ns = 1, where column j's R outputs are
// contiguous at y[j R], the last phase puts the column's T threads on
// consecutive lanes (T >= 16: 128-byte runs).  Per point that is one global
// load, one global store and one shared-memory round trip per exchange,
// against the staged kernel's three shared-memory round trips and its
// per-element scatter index arithmetic.
template <int LOGR, int CW = 0>
struct GlobalRegShape {
    using S = LocalShape<LOGR>;
    static constexpr int R = 1 << LOGR;
    static constexpr int T = S::T;  // threads per column
    // columns per CTA: CW when given, else runs of >= 128 bytes
    static constexpr int C = CW ? CW : (T >= 8 ? 16 : 128 / T);
    static constexpr int LOG_C = log2_const(C);
    static constexpr int TPB = C * T;
    static constexpr int RS = S::PADDED + 1;  // padded column stride (float2)
    static constexpr bool EXCHANGE = S::NPASS > 1;
    static constexpr int TILE_BYTES = EXCHANGE ? C * RS * 8 : 0;
    // W_R^m for m < R (phases with columns on consecutive threads: one
    // twiddle per half-warp, a broadcast), and for the first pass's last
    // phase the same values as [r][jm] rows (consecutive jm on consecutive
    // lanes: conflict-free)
    static constexpr int TW_BYTES = EXCHANGE ? 2 * R * 8 : 0;
    static constexpr int SMEM_BYTES = TILE_BYTES + TW_BYTES;
    static constexpr int MINB = 1024 / TPB;  // 64 registers per thread
    static_assert(LOGR >= 4 && TPB <= 1024 && TPB >= 128, "register-direct pass radix must be 16..1024");
};

// In-place in-CTA phases 1 .. NPASS-2 of the register-direct pass; `full`
// holds W_R^m, m < R.
template <int LOGR, int P>
struct GlobalRegMiddle {
    static CUBF_DEV void run(float2 (&v)[LocalShape<LOGR>::E], int th, const float2* full, float2* col) {
        using S = LocalShape<LOGR>;
        if constexpr (P < S::NPASS - 1) {
            constexpr int SHIFT = LOGR - S::ns_bits(P) - S::radix_bits(P);
            pass_load_tw<LOGR, P>(v, th, [&](int jm, int r) { return full[(jm * r) << SHIFT]; },
                                  [&](int i) { return col[S::pad(i)]; });
            __syncthreads();
            pass_store<LOGR, P>(v, th, [&](int i, float2 x) { col[S::pad(i)] = x; });
            __syncthreads();
            GlobalRegMiddle<LOGR, P + 1>::run(v, th, full, col);
        }
    }
};

// With CHUNKED, the tiles cover a chunk of a pass's column tiles (the
// L2-chained pass pairs of the "fft-l2-chain" plans, run by the chain-step
// kernel of fft_chain.cu): tile b starts at column base + (b mod
// tiles_per_run) C + (b / tiles_per_run) run_stride of the pass's single
// transform.  `src_l2`: the source is an intermediate an earlier launch left
// in L2; each 128-byte line is discarded from L2 once the tile holds its
// values (never written back to HBM).  `dst_l2`: the destination is such an
// intermediate (stored with an L2 evict-last policy).
struct RegChunk {
    uint32_t base;
    uint32_t tiles_per_run;  // 0: every tile of every transform, in order
    uint32_t run_stride;
    int src_l2;
    int dst_l2;
};

CUBF_DEV void discard_l2_line(const void* p) {
    asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}

// FIRST: Ns = 1 (and no interleaving; T >= 16), the tile's output is C R
// contiguous values; otherwise Ns >= C.  Offsets within one transform (or one
// interleaved array) are 32-bit: 2^log_n <= 2^31.
//
// reg_pass_tile is the body of one CTA of the pass: tile `vblock` of a grid
// of `vgrid` tiles, run by threads tid < TPB over the shared memory at
// `smem`.  fft_global_reg_kernel runs one tile per CTA; the chain-step kernel
// (fft_chain_step_kernel) runs tiles of two passes side by side.  ROLE fixes
// a chunked tile's L2 flags at compile time: 1 the first pass of a chain
// pair (HBM source, L2-kept destination), 2 the second (L2 source, HBM
// destination); 0 takes them from `chunk`.
template <int LOGR, bool FIRST, int CW, bool CHUNKED, int ROLE = 0>
CUBF_DEV void reg_pass_tile(const float2* src, float2* dst, int log_n, int ns_bits, const float2* __restrict__ tw1024,
                            const OuterTwiddles& outer, int conj_in, int conj_out, float scale, int log_v,
                            unsigned prefetch_stride, int outer_shift, const RegChunk& chunk, size_t vblock,
                            size_t vgrid, int tid, unsigned char* smem_raw) {
    using G = GlobalRegShape<LOGR, CW>;
    using S = typename G::S;
    constexpr int RB0 = S::radix_bits(0);
    constexpr int RA = 1 << RB0;        // radix of the first register phase
    constexpr int SUB0 = S::E / RA;     // its sub-DFTs per thread
    constexpr int ROWSTEP = G::R / RA;  // row distance within a first-phase sub-DFT
    constexpr int PL = S::NPASS - 1;    // last register phase
    float2* a = reinterpret_cast<float2*>(smem_raw);
    float2* full = a + G::TILE_BYTES / 8;
    float2* rows = full + G::R;
    if constexpr (G::EXCHANGE) {
        // W_R^m = W_1024^(m 2^(10 - LOGR)); rows[r NsL + jm] = W_R^(jm r) for the last phase
        constexpr int NSL = 1 << S::ns_bits(PL);
        for (int m = tid; m < G::R; m += G::TPB) {
            full[m] = __ldg(tw1024 + (m << (10 - LOGR)));
            const int r = m / NSL, jm = m % NSL;
            rows[m] = __ldg(tw1024 + (((jm * r) & (G::R - 1)) << (10 - LOGR)));
        }
    }
    const uint32_t cols = 1u << (log_n - LOGR);
    const uint32_t ctas_per_batch = cols >> G::LOG_C;
    // (transform, first column) of tile b of this launch
    auto tile_origin = [&](size_t b, size_t& t, uint32_t& j) {
        if (CHUNKED) {
            t = 0;
            j = chunk.base + ((static_cast<uint32_t>(b) % chunk.tiles_per_run) << G::LOG_C) +
                (static_cast<uint32_t>(b) / chunk.tiles_per_run) * chunk.run_stride;
        } else {
            t = b / ctas_per_batch;
            j = static_cast<uint32_t>(b % ctas_per_batch) << G::LOG_C;
        }
    };
    size_t bidx;
    uint32_t j0;
    tile_origin(vblock, bidx, j0);
    const uint32_t ns = 1u << ns_bits;
    float2 v[S::E];
    // phase 0: straight from HBM, columns on consecutive threads
    const int c0 = tid & (G::C - 1);
    const int th0 = tid >> G::LOG_C;
    {
        const float2* col = src + (bidx << log_n) + j0 + c0;
        const uint32_t rstep = ROWSTEP * cols;
#pragma unroll
        for (int u = 0; u < SUB0; ++u) {
            const uint32_t off = static_cast<uint32_t>(th0 + S::T * u) * cols;
#pragma unroll
            for (int r = 0; r < RA; ++r) v[u * RA + r] = __ldcs(col + (off + r * rstep));
        }
    }
    if (prefetch_stride != 0 && vblock + static_cast<size_t>(prefetch_stride) < vgrid) {
        size_t nt;
        uint32_t nj;
        tile_origin(vblock + static_cast<size_t>(prefetch_stride), nt, nj);
        const float2* nsrc = src + (nt << log_n) + nj;
        for (int r = tid; r < G::R; r += G::TPB) prefetch_l2(nsrc + static_cast<uint32_t>(r) * cols, G::C * 8);
    }
    if (conj_in) {
#pragma unroll
        for (int i = 0; i < S::E; ++i) v[i].y = -v[i].y;
    }
    if (!FIRST && ns_bits > log_v) {
        // outer twiddle W_{Ns R}^{jm i} of row i = j + r ROWSTEP: a fp64 start
        // and step per sub-DFT, a fp64 recurrence, each factor rounded once
        const size_t jm = ((j0 + c0) & (ns - 1)) >> log_v;
        const int tshift = log_n - ns_bits - LOGR + outer_shift;
        const size_t tmask = (size_t{1} << (log_n - log_v + outer_shift)) - 1;
        const double2 step = outer_twiddle_d(outer, ((jm * ROWSTEP) << tshift) & tmask);
#pragma unroll
        for (int u = 0; u < SUB0; ++u) {
            const int j = th0 + S::T * u;
            double2 w = outer_twiddle_d(outer, ((jm * static_cast<size_t>(j)) << tshift) & tmask);
#pragma unroll
            for (int r = 0; r < RA; ++r) {
                v[u * RA + r] = cmul(v[u * RA + r], make_float2(static_cast<float>(w.x), static_cast<float>(w.y)));
                if (r + 1 < RA) w = cmul_d(w, step);
            }
        }
    }
#pragma unroll
    for (int u = 0; u < SUB0; ++u) Dft<RA>::run(&v[u * RA]);
    const bool src_l2 = CHUNKED && (ROLE == 0 ? chunk.src_l2 != 0 : ROLE == 2);
    const bool dst_l2 = CHUNKED && (ROLE == 0 ? chunk.dst_l2 != 0 : ROLE == 1);
    // Once every thread of the tile has loaded its values (after the first
    // exchange's barrier), drop the tile's source lines from L2 without
    // writing them back: R rows of C = 32 columns, two 128-byte lines per
    // row, one line per thread (TPB = 2R).  The addresses come from the
    // thread index, not from the loads, so none stays live across the DFTs
    // (reusing the load addresses there cost ~100 bytes of spills a thread).
    static_assert(!CHUNKED || (G::EXCHANGE && G::TPB == 2 * G::R), "chunked tiles discard one line per thread");
    auto discard_source = [&]() {
        const uint32_t row = static_cast<uint32_t>(tid) >> 1;
        discard_l2_line(src + (bidx << log_n) + j0 + row * cols + (static_cast<uint32_t>(tid) & 1u) * 16u);
    };
    // the output's column base: y[(J / Ns) Ns R + (J mod Ns) + k Ns] with
    // J = j0 + c, j0 a multiple of C; Ns = 1 reduces it to y[J R + k]
    float2* dbase = dst + (bidx << log_n) + (((j0 >> ns_bits) << (ns_bits + LOGR)) + (j0 & (ns - 1)));
    const float out_sgn = conj_out ? -1.f : 1.f;
    const bool plain = scale == 1.f && !conj_out;
    const uint64_t keep = dst_l2 ? l2_policy(true) : 0;
    auto emit = [&](float2* p, float2 x) {
        const float2 y = plain ? x : make_float2(x.x * scale, x.y * out_sgn * scale);
        if (dst_l2)
            asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(p), "f"(y.x), "f"(y.y),
                         "l"(keep)
                         : "memory");
        else
            __stcs(p, y);
    };
    if constexpr (!G::EXCHANGE) {
        // one register phase (radix 16, Ns >= C): output k of column c0 at k Ns
        static_assert(!FIRST, "the first pass needs the exchange to reach contiguous runs");
        float2* d = dbase + c0;
        pass_store<LOGR, 0>(v, th0, [&](int k, float2 x) { emit(d + static_cast<uint32_t>(k) * ns, x); });
    } else {
        pass_store<LOGR, 0>(v, th0, [&](int i, float2 x) { a[c0 * G::RS + S::pad(i)] = x; });
        __syncthreads();
        if (src_l2) discard_source();
        GlobalRegMiddle<LOGR, 1>::run(v, th0, full, a + c0 * G::RS);
        constexpr int SHIFT = LOGR - S::ns_bits(PL) - S::radix_bits(PL);
        constexpr int NSL = 1 << S::ns_bits(PL);
        if constexpr (FIRST) {
            // a column's threads on consecutive lanes: y[J R + k] in runs of T
            const int c1 = tid / S::T;
            const int th1 = tid % S::T;
            const float2* col = a + c1 * G::RS;
            pass_load_tw<LOGR, PL>(v, th1, [&](int jm, int r) { return rows[r * NSL + jm]; },
                                   [&](int i) { return col[S::pad(i)]; });
            float2* d = dbase + c1 * G::R;
            pass_store<LOGR, PL>(v, th1, [&](int k, float2 x) { emit(d + k, x); });
        } else {
            const float2* col = a + c0 * G::RS;
            pass_load_tw<LOGR, PL>(v, th0, [&](int jm, int r) { return full[(jm * r) << SHIFT]; },
                                   [&](int i) { return col[S::pad(i)]; });
            float2* d = dbase + c0;
            pass_store<LOGR, PL>(v, th0, [&](int k, float2 x) { emit(d + static_cast<uint32_t>(k) * ns, x); });
        }
    }
}

template <int LOGR, bool FIRST, int CW = 0, bool CHUNKED = false>
__global__ void __launch_bounds__(GlobalRegShape<LOGR, CW>::TPB, GlobalRegShape<LOGR, CW>::MINB)
    fft_global_reg_kernel(const float2* src, float2* dst, int log_n, int ns_bits, const float2* __restrict__ tw1024,
                          OuterTwiddles outer, int conj_in, int conj_out, float scale, int log_v,
                          unsigned prefetch_stride, int outer_shift, RegChunk chunk) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    pdl_begin();
    reg_pass_tile<LOGR, FIRST, CW, CHUNKED>(src, dst, log_n, ns_bits, tw1024, outer, conj_in, conj_out, scale, log_v,
                                            prefetch_stride, outer_shift, chunk, blockIdx.x, gridDim.x,
                                            static_cast<int>(threadIdx.x), smem_raw);
}



// ---- L2-blocked large transform: first pass of the decimated transforms ------
//
// A transform of N = V L points runs as V transforms of L points over the
// decimated sequences x_m[i] = x[m + V i] (m < V), then one radix-V Stockham
// pass with Ns = L that combines them (Cooley-Tukey, decimation in time).
// The V decimated transforms are taken CW at a time, a chunk whose L-point
// data fits in L2: this kernel runs the first Stockham pass (Ns = 1, radix
// R = 2^LOGR) of transforms m0 .. m0 + CW - 1 of a chunk, reading x in runs of
// CW adjacent values (the transforms interleave element by element) and
// writing each transform's pass output contiguously (dst + (m - m0) L), kept
// in L2 for the chunk's next pass.  CTA b takes column j = b of every
// transform of the chunk: rows x_m[j + r L / R], r < R.
template <int LOGR, int CW>
__global__ void __launch_bounds__(GlobalPassShape<LOGR, CW>::TPB,
                                  1024 / GlobalPassShape<LOGR, CW>::TPB > 0 ? 1024 / GlobalPassShape<LOGR, CW>::TPB : 1)
    fft_deinterleave_pass_kernel(const float2* src, float2* dst, int log_len, int log_v, size_t m0,
                                 const float2* __restrict__ tw_r, int tw_log_stride, int conj_in) {
    using G = GlobalPassShape<LOGR, CW>;
    using S = typename G::S;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2* a = reinterpret_cast<float2*>(smem_raw);
    const auto twt = TwiddleTable<LOGR>::load(a + G::C * G::RS, tw_r, tw_log_stride);
    const size_t len = size_t{1} << log_len;
    const size_t cols = len >> LOGR;
    const size_t j = blockIdx.x;
    const float in_sgn = conj_in ? -1.f : 1.f;
    {
        constexpr int RSTEP = G::TPB / CW;
        const int c = threadIdx.x % CW;
        const float2* s = src + m0 + c + (j << log_v);
#pragma unroll 4
        for (int r = threadIdx.x / CW; r < G::R; r += RSTEP) {
            float2 x = __ldcs(s + ((static_cast<size_t>(r) * cols) << log_v));
            x.y *= in_sgn;
            a[c * G::RS + S::pad(r)] = x;
        }
    }
    __syncthreads();
    {
        const int c = threadIdx.x / S::T;
        const int th = threadIdx.x % S::T;
        float2 v[S::E];
        GlobalColumnPasses<LOGR, 0>::run(v, th, twt, a + c * G::RS);
    }
    // y_m[j R + k] -> dst[(m - m0) L + j R + k]: contiguous in k; kept in L2
    const uint64_t keep = l2_policy(true);
#pragma unroll 4
    for (int idx = threadIdx.x; idx < CW * G::R; idx += G::TPB) {
        const int c = idx >> LOGR, k = idx & (G::R - 1);
        const float2 x = a[c * G::RS + S::pad(k)];
        float2* p = dst + static_cast<size_t>(c) * len + j * G::R + k;
        asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(p), "f"(x.x), "f"(x.y), "l"(keep)
                     : "memory");
    }
}

}  // namespace cubf::fft
