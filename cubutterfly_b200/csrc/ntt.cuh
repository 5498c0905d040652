// ntt.cuh -- RNS word64 NTT kernels for sm_100a.
//
// Forward negacyclic NTT, natural input, bit-reversed output, one modulus per
// polynomial, as served by the reference's RNS ABI (RnsPlan, include/cuntt/
// rns_ntt.hpp:97-131; fused CT core src/rns_fused_ctgs.cuh:55-224).  The
// negacyclic twist is folded into the Cooley-Tukey stages: stage s pairs
// elements j and j + N/2^(s+1) and multiplies by psi^bitrev(2^s + (j >> (L-s)))
// (the "psi_rev" root schedule), so output is bit-reversed with no extra pass.
// The inverse (Gentleman-Sande with psi^-bitrev, natural output from a
// bit-reversed input, scaled by N^-1) uses the same tile machinery.
//
// The L = log2 N stages are split into two tile passes: pass 1 transforms the
// top L1 index bits of every column (strided tiles, C adjacent columns per CTA
// for coalescing), pass 2 the low L2 bits of contiguous chunks.  Inside a tile
// each thread keeps 2^LOGE residues in registers; successive register groups
// of LOGE index bits are reached through shared memory.  Products use Shoup's
// method with per-root precomputed quotients floor(w 2^64 / q), so a modular
// multiply is one 64-bit high product and two low products; q < 2^63.
//
// The same passes serve the cyclic single-modulus NTT of the main ABI
// (cuntt::Plan, include/cuntt/ntt.hpp:432): with the cyclic root schedule the
// Cooley-Tukey passes map natural input to bit-reversed output and the
// Gentleman-Sande passes bit-reversed input to natural output, for either
// direction (the root table carries omega or omega^-1).  Storage words may be
// 32 or 64 bits wide; arithmetic is 64-bit throughout.  Transforms of at most
// 2^11 points run as one tile per transform (ntt_single_kernel).
#pragma once

#include "common.cuh"

namespace cubf::ntt {

using u64 = unsigned long long;

CUBF_DEV u64 mul_shoup(u64 a, u64 w, u64 wq, u64 q) {
    const u64 hi = __umul64hi(a, wq);
    const u64 r = a * w - hi * q;  // in [0, 2q)
    return r >= q ? r - q : r;
}
CUBF_DEV u64 add_mod(u64 a, u64 b, u64 q) {
    const u64 s = a + b;
    return s >= q ? s - q : s;
}
CUBF_DEV u64 sub_mod(u64 a, u64 b, u64 q) { return a >= b ? a - b : a + q - b; }

// Lazy (Harvey) arithmetic for q < 2^62: Shoup's product without its final
// correction lands in [0, 2q) for any 64-bit input, and butterflies keep
// values in [0, 4q) (forward) or [0, 2q) (inverse) so most conditional
// subtractions disappear; outputs are reduced to [0, q) once, when written.
CUBF_DEV u64 mul_shoup_lazy(u64 a, u64 w, u64 wq, u64 q) { return a * w - __umul64hi(a, wq) * q; }
CUBF_DEV u64 reduce_2q(u64 a, u64 q2) { return a >= q2 ? a - q2 : a; }
CUBF_DEV u64 canonical_4q(u64 a, u64 q) { return reduce_2q(reduce_2q(a, 2 * q), q); }
// x mod q for any 64-bit x: Shoup's product with w = 1 and uq = floor(2^64 / q)
// estimates the quotient to within one, so one conditional subtraction
// remains.  The main-ABI NTT reduces its input words with it, as the
// reference's reference_ntt does (src/reference.cpp:601-603).
CUBF_DEV u64 reduce_word(u64 x, u64 uq, u64 q) { return reduce_2q(x - __umul64hi(x, uq) * q, q); }

// Per-polynomial binding of an RNS plan: offsets into the caller's buffers and
// the domain whose modulus and root tables it uses.
struct PolyDesc {
    u64 in_off;
    u64 out_off;
    uint32_t domain;
    uint32_t pad_;
};

struct DomainTables {
    // [domains][N] pairs {w, floor(w 2^64 / q)}: forward w = psi^bitrev(i),
    // inverse psi^-bitrev(i); one 16-byte load fetches a root and its quotient
    const u64* root_pairs;
    const u64* moduli;    // [domains]
    const u64* n_inv;     // [domains] N^-1 mod q (inverse only)
    const u64* n_inv_q;   // Shoup quotient of n_inv
    const u64* unit_q;    // [domains] floor(2^64 / q), read when input words are reduced
};

// Register group g of a tile with B index bits: registers hold the LOGE
// consecutive bits starting at lo(g); the stage bits of the group are the
// not-yet-processed ones.  Forward processes bits top-down, inverse bottom-up.
template <int B, int LOGE, bool INV>
struct NttGroups {
    static constexpr int E = 1 << LOGE;
    static constexpr int COUNT = (B + LOGE - 1) / LOGE;
    static constexpr int lo(int g) {
        if (!INV) {
            const int top = B - g * LOGE;  // exclusive top of new bits
            return top - LOGE < 0 ? 0 : top - LOGE;
        }
        const int start = g * LOGE;
        return start + LOGE > B ? B - LOGE : start;
    }
    // new (stage) bits of group g, as a mask of tile bits
    static constexpr uint32_t stage(int g) {
        if (!INV) {
            const int top = B - g * LOGE;
            const int bot = top - LOGE < 0 ? 0 : top - LOGE;
            return lowmask(top) & ~lowmask(bot);
        }
        const int bot = g * LOGE;
        const int top = bot + LOGE > B ? B : bot + LOGE;
        return lowmask(top) & ~lowmask(bot);
    }
    static constexpr uint32_t reg(int g) { return lowmask(LOGE) << lo(g); }
};

template <int B_, int LOGE_, int COLS_, bool STRIDED_, bool INV_, bool LAZY_, bool STAGEABLE_ = true>
struct NttShape {
    static constexpr bool LAZY = LAZY_;
    static constexpr int B = B_;
    static constexpr int LOGE = LOGE_;
    static constexpr int E = 1 << LOGE;
    static constexpr int COLS = COLS_;  // tiles per CTA
    static constexpr bool STRIDED = STRIDED_;
    static constexpr bool INV = INV_;
    static constexpr int TPT = 1 << (B - LOGE);
    static constexpr int TPB = TPT * COLS;
    using Gs = NttGroups<B, LOGE, INV>;
    static constexpr int TILE = 1 << B;
    // strided tiles live column-interleaved ([row][col]); contiguous tiles
    // row-major with one word of padding per 16.
    static CUBF_DEV int sidx(int col, uint32_t i) {
        if constexpr (STRIDED)
            return static_cast<int>(i) * COLS + col;
        else
            return col * (TILE + TILE / 16) + static_cast<int>(i + (i >> 4));
    }
    static constexpr int XCH_BYTES = (STRIDED ? TILE * COLS : COLS * (TILE + TILE / 16)) * 8;
    // Root pairs a CTA stages into shared memory before its stages run: the
    // strided pass's tiles all use entries 1 .. 2^B - 1 of the table; the
    // contiguous pass's COLS tiles use, for local stage ls, COLS 2^ls
    // consecutive entries from 2^(off+ls) + first_tile 2^ls.
    // Staged for the strided pass only (2^B - 1 pairs shared by every tile);
    // the contiguous pass's COLS (2^B - 1) pairs would take a 16-tile CTA's
    // occupancy from four CTAs per SM to two (measured slower: 53.3 vs 46.5 us
    // at 32 x 2^16), so its stages read the global pairs, kept L2-resident.
    static constexpr int STAGE_PAIRS = STRIDED ? (TILE - 1) : COLS * (TILE - 1);
    static constexpr bool STAGE = STAGEABLE_ && STRIDED;
    static constexpr int ROOT_PAIRS = STAGE ? STAGE_PAIRS : 0;
    static constexpr int SMEM_BYTES = XCH_BYTES + ROOT_PAIRS * 16;
    // Resident CTAs to ask for: as many as the register file holds with up
    // to 16 residues per thread in 64 registers, but no more than shared
    // memory admits (the register cap would only cost hoisting).
    static constexpr int SMEM_CTAS = (227 * 1024) / SMEM_BYTES;
    static constexpr int REG_CTAS = (E <= 16 && TPB <= 1024) ? 1024 / TPB : 1;
    static constexpr int MINB = SMEM_CTAS < REG_CTAS ? (SMEM_CTAS > 0 ? SMEM_CTAS : 1) : REG_CTAS;
};

// Butterflies of group G on the registers of one thread.  i = tpart | (r << lo)
// is the tile row of register r; the root of the pair at tile bit b (local
// stage ls = B-1-b forward) is roots[2^(off+ls) + (hi << ls) + (i >> (b+1))].
// Root pair k with an L2 evict-last hint: the tables (16 bytes per root) stay
// resident across calls while the coefficient streams pass through.
// The tables are read-only for the kernel's lifetime, so the load is not
// volatile: the compiler may issue it ahead of the butterflies that come
// before its use.
CUBF_DEV ulonglong2 load_root_pair(const u64* __restrict__ pairs, u64 k, uint64_t pol) {
    ulonglong2 r;
    asm("ld.global.nc.L2::cache_hint.v2.u64 {%0, %1}, [%2], %3;"
        : "=l"(r.x), "=l"(r.y)
        : "l"(pairs + 2 * k), "l"(pol));
    return r;
}

// Coefficient words with an L2 hint (evict-first streams, evict-last for the
// intermediate the second pass reads back).
template <typename T>
CUBF_DEV T load_word(const T* p, uint64_t pol) {
    if constexpr (sizeof(T) == 8) {
        unsigned long long v;
        asm volatile("ld.global.L2::cache_hint.u64 %0, [%1], %2;" : "=l"(v) : "l"(p), "l"(pol));
        return static_cast<T>(v);
    } else {
        unsigned v;
        asm volatile("ld.global.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
        return static_cast<T>(v);
    }
}
template <typename T>
CUBF_DEV void store_word(T* p, T v, uint64_t pol) {
    if constexpr (sizeof(T) == 8)
        asm volatile("st.global.L2::cache_hint.u64 [%0], %1, %2;" ::"l"(p), "l"(static_cast<unsigned long long>(v)),
                     "l"(pol)
                     : "memory");
    else
        asm volatile("st.global.L2::cache_hint.u32 [%0], %1, %2;" ::"l"(p), "r"(static_cast<unsigned>(v)), "l"(pol)
                     : "memory");
}

// Roots of the tile passes come from the CTA's staged copy in shared memory
// (`sroots`, laid out as NttShape::ROOT_PAIRS describes); the whole-transform
// kernel reads the global pairs directly (`sroots` null).
template <typename S, int G>
CUBF_DEV void ntt_group(u64 (&v)[S::E], uint32_t tpart, u64 hi, int off, const u64* __restrict__ pairs,
                        uint64_t tab_pol, const ulonglong2* sroots, int col, u64 q) {
    using Gs = typename S::Gs;
    constexpr int LO = Gs::lo(G);
    constexpr uint32_t STAGE = Gs::stage(G);
#pragma unroll
    for (int jj = 0; jj < S::LOGE; ++jj) {
        const int j = S::INV ? jj : S::LOGE - 1 - jj;  // forward: top-down
        const int b = LO + j;
        if ((STAGE >> b) & 1u) {
            const int ls = S::B - 1 - b;
            const u64 head = (u64{1} << (off + ls)) + (hi << ls) + (tpart >> (b + 1));
#pragma unroll
            for (int rh = 0; rh < (S::E >> (j + 1)); ++rh) {
                const u64 k = head + static_cast<u64>(rh);
                ulonglong2 wp;
                if (sroots != nullptr) {
                    const uint32_t x = (tpart >> (b + 1)) + static_cast<uint32_t>(rh);
                    const int local = S::STRIDED ? (1 << ls) - 1 + static_cast<int>(x)
                                                 : (S::COLS << ls) - S::COLS + (col << ls) + static_cast<int>(x);
                    wp = sroots[local];
                } else {
                    wp = load_root_pair(pairs, k, tab_pol);
                }
                const u64 w = wp.x, wq = wp.y;
#pragma unroll
                for (int rl = 0; rl < (1 << j); ++rl) {
                    const int r0 = (rh << (j + 1)) | rl;
                    const int r1 = r0 | (1 << j);
                    if constexpr (!S::INV && S::LAZY) {
                        // Cooley-Tukey, inputs and outputs in [0, 4q)
                        const u64 a = reduce_2q(v[r0], 2 * q);
                        const u64 t = mul_shoup_lazy(v[r1], w, wq, q);
                        v[r0] = a + t;
                        v[r1] = a - t + 2 * q;
                    } else if constexpr (S::INV && S::LAZY) {
                        // Gentleman-Sande, inputs and outputs in [0, 2q)
                        const u64 a = v[r0], c = v[r1];
                        v[r0] = reduce_2q(a + c, 2 * q);
                        v[r1] = mul_shoup_lazy(a - c + 2 * q, w, wq, q);
                    } else if constexpr (!S::INV) {
                        // Cooley-Tukey: (a + w b, a - w b)
                        const u64 t = mul_shoup(v[r1], w, wq, q);
                        const u64 a = v[r0];
                        v[r0] = add_mod(a, t, q);
                        v[r1] = sub_mod(a, t, q);
                    } else {
                        // Gentleman-Sande: (a + b, (a - b) w)
                        const u64 a = v[r0], c = v[r1];
                        v[r0] = add_mod(a, c, q);
                        v[r1] = mul_shoup(sub_mod(a, c, q), w, wq, q);
                    }
                }
            }
        }
    }
}

template <typename S, int G>
CUBF_DEV void ntt_groups(u64 (&v)[S::E], u64* sbuf, int col, uint32_t t, u64 hi, int off,
                         const u64* __restrict__ pairs, uint64_t tab_pol, const ulonglong2* sroots, u64 q) {
    using Gs = typename S::Gs;
    if constexpr (G < Gs::COUNT) {
        if constexpr (G > 0) {
            constexpr uint32_t RP = Gs::reg(G - 1), RN = Gs::reg(G);
            constexpr Offsets<S::E> OP = make_offsets<S::E>(RP);
            constexpr Offsets<S::E> ON = make_offsets<S::E>(RN);
            if constexpr (G > 1) __syncthreads();
            const uint32_t tp = deposit_rt<lowmask(S::B) & ~RP, S::B>(t);
#pragma unroll
            for (int r = 0; r < S::E; ++r) sbuf[S::sidx(col, tp | OP.v[r])] = v[r];
            __syncthreads();
            const uint32_t tn = deposit_rt<lowmask(S::B) & ~RN, S::B>(t);
#pragma unroll
            for (int r = 0; r < S::E; ++r) v[r] = sbuf[S::sidx(col, tn | ON.v[r])];
        }
        const uint32_t tpart = deposit_rt<lowmask(S::B) & ~Gs::reg(G), S::B>(t);
        ntt_group<S, G>(v, tpart, hi, off, pairs, tab_pol, sroots, col, q);
        ntt_groups<S, G + 1>(v, sbuf, col, t, hi, off, pairs, tab_pol, sroots, q);
    }
}

// Tile geometry of the two passes of a 2^L transform: the strided pass covers
// the top ceil(L/2) + D index bits, the contiguous pass the low floor(L/2) - D
// bits (D = 0 by default; the RNS tuner also tries D = -1 and +1).
constexpr int strided_bits(int L, int D = 0) { return (L + 1) / 2 + D; }
constexpr int contiguous_bits(int L, int D = 0) { return L / 2 - D; }
// 8 residues per thread up to 8-bit passes: 16 registers of values leave room
// for more resident warps, which hide the root-load and multiply latency
// better than the fewer exchanges of 16 residues per thread do (config 2,
// 8+8: 38.9 against 42.4 us); 32 above.
constexpr int log_e_for(int b) { return b <= 8 ? 3 : 5; }
// CTAs of 128 threads: strided passes take 8 adjacent columns (64-byte rows
// of uint64), contiguous passes pack tiles up to 128 threads.  Config 2
// (32 x 2^16) then runs 1024 CTAs per pass, seven per SM at most, and the
// SMs finish together: 43.2 us against 47.2 us with 256-thread CTAs (512
// CTAs, three or four per SM); 64-thread contiguous CTAs 43.8 us, 64-thread
// CTAs in both passes 45.9 us.
constexpr int cols_for(int b, bool strided) {
    return strided ? 8 : ((128 >> (b - log_e_for(b))) > 0 ? (128 >> (b - log_e_for(b))) : 1);
}
template <int L, bool STRIDED, bool INV, bool LAZY, int D = 0>
using PassShape = NttShape<STRIDED ? strided_bits(L, D) : contiguous_bits(L, D),
                           log_e_for(STRIDED ? strided_bits(L, D) : contiguous_bits(L, D)),
                           cols_for(STRIDED ? strided_bits(L, D) : contiguous_bits(L, D), STRIDED), STRIDED, INV, LAZY>;

// One tile pass over every polynomial of a 2^L transform.  Forward runs the
// strided pass (stages 0..B1-1) then the contiguous pass; inverse runs them in
// the opposite order.  `in_is_out` makes the pass read the output buffer (the
// second pass is in place); `final_pass` marks the pass that writes the
// result (lazy variants reduce to [0, q) there), and with `final_scale` the
// final inverse pass scales by N^-1.  LAZY requires every modulus < 2^62.
// Results are written by store_result: reduced to [0, q) on the final pass of
// a lazy variant, scaled by N^-1 when `final_scale` is set.
template <bool INV, bool LAZY>
CUBF_DEV u64 final_value(u64 v, u64 q, bool final_pass, bool scale, u64 ni, u64 niq) {
    if (scale) return mul_shoup(v, ni, niq, q);  // exact for any 64-bit v
    if (LAZY && final_pass) return INV ? reduce_2q(v, q) : canonical_4q(v, q);
    return v;
}

// T is the storage word (unsigned int or u64); `reduce_input` reduces each
// loaded word modulo q first, so any 64-bit input is accepted.
template <int L, bool STRIDED, bool INV, bool LAZY, typename T, int D = 0>
__global__ void __launch_bounds__(PassShape<L, STRIDED, INV, LAZY, D>::TPB, PassShape<L, STRIDED, INV, LAZY, D>::MINB)
    ntt_pass_kernel(const T* in, T* out, const PolyDesc* __restrict__ polys, DomainTables tab, int in_is_out,
                    int final_pass, int final_scale, int reduce_input) {
    using S = PassShape<L, STRIDED, INV, LAZY, D>;
    using Gs = typename S::Gs;
    constexpr int B = S::B;
    constexpr int COLS = S::COLS;
    constexpr int LOWB = STRIDED ? L - B : 0;  // index bits below this pass's bits
    constexpr size_t N = size_t{1} << L;
    constexpr size_t GROUPS = (N >> B) / COLS;  // CTAs per polynomial
    extern __shared__ __align__(16) unsigned char smem_raw[];
    u64* sbuf = reinterpret_cast<u64*>(smem_raw);

    const size_t p = blockIdx.x / GROUPS;
    const uint32_t g = static_cast<uint32_t>(blockIdx.x % GROUPS);
    const PolyDesc pd = polys[p];
    const u64 q = tab.moduli[pd.domain];
    const u64* pairs = tab.root_pairs + 2 * static_cast<size_t>(pd.domain) * N;
    const uint64_t tab_pol = l2_policy(true);
    // the first pass streams its input and keeps its output (read back by the
    // second pass) in L2; the final pass streams both ways
    const uint64_t ld_pol = l2_policy(false);
    const uint64_t st_pol = l2_policy(!final_pass);
    // stage this CTA's root pairs (asynchronous copies, overlapping the
    // coefficient loads below; the tables are kept in L2 across calls)
    ulonglong2* sroots = S::STAGE ? reinterpret_cast<ulonglong2*>(smem_raw + S::XCH_BYTES) : nullptr;
    if constexpr (S::STAGE) {
        const int off_s = STRIDED ? 0 : L - B;
        for (int i = threadIdx.x; i < S::ROOT_PAIRS; i += S::TPB) {
            size_t k;
            if constexpr (STRIDED) {
                k = static_cast<size_t>(i) + 1;
            } else {
                int ls = 0;
#pragma unroll
                for (int s2 = 1; s2 < B; ++s2)
                    if (i >= (COLS << s2) - COLS) ls = s2;
                const int j = i - ((COLS << ls) - COLS);
                k = (size_t{1} << (off_s + ls)) + ((static_cast<size_t>(g) * COLS) << ls) + static_cast<size_t>(j);
            }
            const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(sroots + i));
            asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst),
                         "l"(pairs + 2 * k), "l"(tab_pol)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    const T* src = in_is_out ? static_cast<const T*>(out) + pd.out_off : in + pd.in_off;
    T* dst = out + pd.out_off;

    int col;
    uint32_t t;
    if constexpr (STRIDED) {
        col = threadIdx.x % COLS;  // adjacent threads -> adjacent columns (coalesced)
        t = threadIdx.x / COLS;
    } else {
        col = threadIdx.x / S::TPT;
        t = threadIdx.x % S::TPT;
    }
    const uint32_t tile = g * COLS + col;
    // Tile row i lives at (i << LOWB) | tile (strided) or (tile << B) | i.
    const T* tsrc = src + (STRIDED ? tile : (static_cast<size_t>(tile) << B));
    T* tdst = dst + (STRIDED ? tile : (static_cast<size_t>(tile) << B));
    constexpr int SHIFT = STRIDED ? LOWB : 0;
    const int off = STRIDED ? 0 : L - B;
    const u64 hi = STRIDED ? 0 : static_cast<u64>(tile);

    u64 v[S::E];
    {
        constexpr uint32_t R0 = Gs::reg(0);
        constexpr Offsets<S::E> O0 = make_offsets<S::E>(R0);
        const uint32_t tp = deposit_rt<lowmask(B) & ~R0, B>(t);
        const T* ts = tsrc + (static_cast<size_t>(tp) << SHIFT);
#pragma unroll
        for (int r = 0; r < S::E; ++r) v[r] = static_cast<u64>(load_word(ts + (static_cast<size_t>(O0.v[r]) << SHIFT), ld_pol));
        if (reduce_input) {
            const u64 uq = tab.unit_q[pd.domain];
#pragma unroll
            for (int r = 0; r < S::E; ++r) v[r] = reduce_word(v[r], uq, q);
        }
    }
    if constexpr (S::STAGE) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // every thread's staged roots are visible
    }
    ntt_groups<S, 0>(v, sbuf, col, t, hi, off, pairs, tab_pol, sroots, q);
    constexpr uint32_t RF = Gs::reg(Gs::COUNT - 1);
    constexpr Offsets<S::E> OF = make_offsets<S::E>(RF);
    const uint32_t tf = deposit_rt<lowmask(B) & ~RF, B>(t);
    T* td = tdst + (static_cast<size_t>(tf) << SHIFT);
    const u64 ni = final_scale ? tab.n_inv[pd.domain] : 0, niq = final_scale ? tab.n_inv_q[pd.domain] : 0;
#pragma unroll
    for (int r = 0; r < S::E; ++r)
        store_word(td + (static_cast<size_t>(OF.v[r]) << SHIFT),
                   static_cast<T>(final_value<INV, LAZY>(v[r], q, final_pass, final_scale, ni, niq)), st_pol);
}

// Whole transforms of 2^L <= 2^11 points as single tiles, COLS transforms
// per CTA, packed batch (transform p at p * 2^L), one domain.
constexpr int single_log_e(int L) { return L < log_e_for(L) ? L : log_e_for(L); }
constexpr int single_cols(int L) { return 256 >> (L - single_log_e(L)); }
template <int L, bool INV, bool LAZY>
using SingleShape = NttShape<L, single_log_e(L), single_cols(L), false, INV, LAZY, false>;

template <int L, bool INV, bool LAZY, typename T>
__global__ void __launch_bounds__(SingleShape<L, INV, LAZY>::TPB, SingleShape<L, INV, LAZY>::MINB)
    ntt_single_kernel(const T* in, T* out, size_t count, DomainTables tab, int final_scale, int reduce_input) {
    using S = SingleShape<L, INV, LAZY>;
    using Gs = typename S::Gs;
    constexpr size_t N = size_t{1} << L;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    u64* sbuf = reinterpret_cast<u64*>(smem_raw);
    const int col = threadIdx.x / S::TPT;
    const uint32_t t = threadIdx.x % S::TPT;
    const size_t p = static_cast<size_t>(blockIdx.x) * S::COLS + col;
    const bool active = p < count;  // idle columns still take part in the block barriers
    const u64 q = tab.moduli[0];

    u64 v[S::E];
    {
        constexpr uint32_t R0 = Gs::reg(0);
        constexpr Offsets<S::E> O0 = make_offsets<S::E>(R0);
        const T* ts = in + p * N + deposit_rt<lowmask(L) & ~R0, L>(t);
        const u64 uq = reduce_input ? tab.unit_q[0] : 0;
#pragma unroll
        for (int r = 0; r < S::E; ++r) {
            v[r] = active ? static_cast<u64>(ts[O0.v[r]]) : 0;
            if (reduce_input) v[r] = reduce_word(v[r], uq, q);
        }
    }
    ntt_groups<S, 0>(v, sbuf, col, t, 0, 0, tab.root_pairs, l2_policy(true), nullptr, q);
    if (!active) return;
    constexpr uint32_t RF = Gs::reg(Gs::COUNT - 1);
    constexpr Offsets<S::E> OF = make_offsets<S::E>(RF);
    T* td = out + p * N + deposit_rt<lowmask(L) & ~RF, L>(t);
    const u64 ni = final_scale ? tab.n_inv[0] : 0, niq = final_scale ? tab.n_inv_q[0] : 0;
#pragma unroll
    for (int r = 0; r < S::E; ++r)
        td[OF.v[r]] = static_cast<T>(final_value<INV, LAZY>(v[r], q, true, final_scale, ni, niq));
}

}  // namespace cubf::ntt
