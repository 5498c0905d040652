// bitwise.cuh -- FWHT and subset/superset zeta kernels for sm_100a.
//
// Both transforms are products of commuting per-bit stages: stage b pairs the
// elements whose indices differ in bit b.  The reference runs them stage by
// stage (FwhtOperator / BooleanZetaOperator, src/operator_traits.cuh:88-112 and
// :364-398; reference_fwht / reference_subset_zeta, butterfly_reference.cpp:349,
// :475).  Because the stages commute, this kernel applies any set of index bits
// in one pass over a TILE of 2^(LOGH+LOGW) elements: LOGH transformed "row"
// bits over W = 2^LOGW contiguous, untouched "column" positions.  Each thread
// holds E = 2^LOGE values in registers; the tile's bits are covered by a few
// register groups: group 1 is loaded straight from HBM with 16-byte vectors
// (bits 0..LOGV-1 plus the top bits), later groups are reached through one
// shared-memory exchange each.  A transform longer than one tile runs as
// several tile passes (a contiguous pass over the low bits, then strided
// passes over the high bits with coalesced column blocks), each pass reading
// and writing HBM once.
#pragma once

#include "common.cuh"

namespace cubf::bw {

// ---- operators --------------------------------------------------------------
// apply(lo, hi): lo has the stage bit clear, hi has it set.  apply2 does two
// independent butterflies (lo0, hi0), (lo1, hi1) at once; for FWHT in fp32 it
// issues Blackwell's packed add.f32x2 / sub.f32x2 (two lanes per instruction).
struct FwhtOp {
    static constexpr bool kPacked = true;
    template <typename T>
    static CUBF_DEV void apply(T& lo, T& hi, int) {
        const T a = lo, b = hi;
        lo = a + b;
        hi = a - b;
    }
    static CUBF_DEV void apply2(float& lo0, float& lo1, float& hi0, float& hi1, int) {
        float s0, s1, d0, d1;
        asm("{\n\t.reg .b64 a, b, s, d;\n\t"
            "mov.b64 a, {%4, %5};\n\t"
            "mov.b64 b, {%6, %7};\n\t"
            "add.rn.f32x2 s, a, b;\n\t"
            "sub.rn.f32x2 d, a, b;\n\t"
            "mov.b64 {%0, %1}, s;\n\t"
            "mov.b64 {%2, %3}, d;\n\t}"
            : "=f"(s0), "=f"(s1), "=f"(d0), "=f"(d1)
            : "f"(lo0), "f"(lo1), "f"(hi0), "f"(hi1));
        lo0 = s0;
        lo1 = s1;
        hi0 = d0;
        hi1 = d1;
    }
};

// x * scale for two fp32 values with one packed multiply.
CUBF_DEV void scale2(float& a, float& b, float s) {
    float o0, o1;
    asm("{\n\t.reg .b64 x, y, z;\n\t"
        "mov.b64 x, {%2, %3};\n\t"
        "mov.b64 y, {%4, %4};\n\t"
        "mul.rn.f32x2 z, x, y;\n\t"
        "mov.b64 {%0, %1}, z;\n\t}"
        : "=f"(o0), "=f"(o1)
        : "f"(a), "f"(b), "f"(s));
    a = o0;
    b = o1;
}
template <bool SUPERSET>
struct ZetaOp {
    static constexpr bool kPacked = false;
    // subset: f[S | bit] += f[S]; superset: f[S] += f[S | bit]; inverse subtracts.
    template <typename T>
    static CUBF_DEV void apply(T& lo, T& hi, int inverse) {
        if constexpr (SUPERSET)
            lo = inverse ? lo - hi : lo + hi;
        else
            hi = inverse ? hi - lo : hi + lo;
    }
};

// ---- register-group plan (compile time) -------------------------------------
struct Groups {
    uint32_t reg[4];    // tile-index bits held in registers by each group
    uint32_t stage[4];  // bits transformed while in that group
    int count;
};

constexpr int log2_const(int x) {
    int l = 0;
    while ((1 << l) < x) ++l;
    return l;
}

constexpr int popcount_const(uint32_t x) {
    int n = 0;
    for (; x; x &= x - 1) ++n;
    return n;
}

// Register groups of a tile of 2^(LOGH+LOGW) elements, LOGE register bits
// per thread.  Group 1 holds the LOGV vector bits (16-byte loads) and the
// top bits.  Each later group takes the remaining stage bits (the previous
// group's lane bits first) and fills its register set with, in order: the
// vector bits if it is the final group (16-byte stores), the previous
// group's lane bits (its lowest five thread bits), then bits above those.
// With the writer's lane bits as the reader's lowest register bits, the
// scalar shared-memory stores of an exchange hit 32 distinct banks.
template <int LOGH, int LOGW, int LOGE, int LOGV>
constexpr Groups lane_fill_groups() {
    Groups g{};
    constexpr int LT = LOGH + LOGW;
    const uint32_t full = lowmask(LT);
    const uint32_t transform = lowmask(LOGH) << LOGW;
    const uint32_t g1 = lowmask(LOGV) | (lowmask(LOGE - LOGV) << (LT - (LOGE - LOGV)));
    g.reg[0] = g1;
    g.stage[0] = g1 & transform;
    uint32_t done = g.stage[0];
    int k = 1;
    while ((transform & ~done) != 0u && k < 4) {
        const uint32_t rem = transform & ~done;
        const uint32_t thread_bits = full & ~g.reg[k - 1];
        uint32_t lanes = 0;
        int nl = 0, top = -1;
        for (int b = 0; b < LT && nl < 5; ++b)
            if ((thread_bits >> b) & 1u) {
                lanes |= 1u << b;
                ++nl;
                top = b;
            }
        const bool last = popcount_const(rem) <= LOGE;
        uint32_t take = 0;
        int cnt = 0;
        for (int b = 0; b < LT && cnt < LOGE; ++b)
            if (((rem & lanes) >> b) & 1u) {
                take |= 1u << b;
                ++cnt;
            }
        for (int b = 0; b < LT && cnt < LOGE; ++b)
            if (((rem & ~take) >> b) & 1u) {
                take |= 1u << b;
                ++cnt;
            }
        uint32_t reg = take;
        if (last)
            for (int b = 0; b < LOGV && cnt < LOGE; ++b)
                if (!((reg >> b) & 1u)) {
                    reg |= 1u << b;
                    ++cnt;
                }
        for (int b = 0; b < LT && cnt < LOGE; ++b)
            if (((lanes & ~reg) >> b) & 1u) {
                reg |= 1u << b;
                ++cnt;
            }
        for (int b = top + 1; b < LT && cnt < LOGE; ++b)
            if (!((reg >> b) & 1u)) {
                reg |= 1u << b;
                ++cnt;
            }
        for (int b = 0; b < LT && cnt < LOGE; ++b)
            if (!((reg >> b) & 1u)) {
                reg |= 1u << b;
                ++cnt;
            }
        g.reg[k] = reg;
        g.stage[k] = take;
        done |= take;
        ++k;
    }
    g.count = k;
    return g;
}

// A plan is well formed when every group holds exactly LOGE register bits,
// each stage bit belongs to its group, and the stages cover every
// transformed bit once.
template <int LOGH, int LOGW, int LOGE>
constexpr bool well_formed(const Groups& g) {
    if (g.count < 1 || g.count > 4) return false;
    uint32_t acc = 0;
    for (int k = 0; k < g.count; ++k) {
        if (popcount_const(g.reg[k]) != LOGE || (g.stage[k] & ~g.reg[k]) != 0u || (acc & g.stage[k]) != 0u)
            return false;
        acc |= g.stage[k];
    }
    return acc == (lowmask(LOGH) << LOGW);
}

// Alternative plan: every later group holds all of the previous group's
// lane bits and takes stage bits only in the remaining slots, finishing
// (with the vector bits) as soon as the rest fits.  Costs a group more on
// some tiles but makes every exchange conflict free by construction.
template <int LOGH, int LOGW, int LOGE, int LOGV>
constexpr Groups lanes_first_groups() {
    Groups g{};
    constexpr int LT = LOGH + LOGW;
    const uint32_t full = lowmask(LT);
    const uint32_t transform = lowmask(LOGH) << LOGW;
    const uint32_t g1 = lowmask(LOGV) | (lowmask(LOGE - LOGV) << (LT - (LOGE - LOGV)));
    g.reg[0] = g1;
    g.stage[0] = g1 & transform;
    uint32_t done = g.stage[0];
    int k = 1;
    while ((transform & ~done) != 0u && k < 4) {
        const uint32_t rem = transform & ~done;
        const uint32_t thread_bits = full & ~g.reg[k - 1];
        uint32_t reg = 0;
        int nl = 0, top = -1;
        for (int b = 0; b < LT && nl < 5; ++b)
            if ((thread_bits >> b) & 1u) {
                reg |= 1u << b;
                ++nl;
                top = b;
            }
        if (nl > LOGE) return Groups{};
        const uint32_t need = (rem | lowmask(LOGV)) & ~reg;
        if (popcount_const(need) + nl <= LOGE) {
            reg |= need;
            int cnt = popcount_const(reg);
            for (int b = top + 1; b < LT && cnt < LOGE; ++b)
                if (!((reg >> b) & 1u)) {
                    reg |= 1u << b;
                    ++cnt;
                }
            for (int b = 0; b < LT && cnt < LOGE; ++b)
                if (!((reg >> b) & 1u)) {
                    reg |= 1u << b;
                    ++cnt;
                }
        } else {
            int cnt = nl;
            for (int b = 0; b < LT && cnt < LOGE; ++b)
                if (((rem & ~reg) >> b) & 1u) {
                    reg |= 1u << b;
                    ++cnt;
                }
            for (int b = top + 1; b < LT && cnt < LOGE; ++b)
                if (!((reg >> b) & 1u)) {
                    reg |= 1u << b;
                    ++cnt;
                }
            for (int b = 0; b < LT && cnt < LOGE; ++b)
                if (!((reg >> b) & 1u)) {
                    reg |= 1u << b;
                    ++cnt;
                }
        }
        if ((reg & rem) == 0u || popcount_const(reg) != LOGE) return Groups{};
        g.reg[k] = reg;
        g.stage[k] = reg & rem;
        done |= reg & rem;
        ++k;
    }
    g.count = (transform & ~done) == 0u ? k : 0;
    return g;
}

// Shared-memory cost of a plan: (passes, wavefronts).  Passes are the
// exchanges plus the output staging when the final group cannot store
// 16-byte vectors.  Wavefronts are those of one warp's scalar stores and
// 16-byte loads per pass, from an exact bank model of lanes 0..31 (banks
// shift uniformly with the register index, so register 0 stands for all).
struct SmemCost {
    int passes;
    int waves;
};

// Max distinct 32-bit words per bank among `n` lanes accessing `width`
// bytes each at byte addresses a[] (wider accesses issue in phases of
// 128 bytes).
constexpr int bank_waves(const uint32_t (&a)[32], int width) {
    const int per_phase = width <= 4 ? 32 : 128 / width;
    int total = 0;
    for (int p0 = 0; p0 < 32; p0 += per_phase) {
        int worst = 0;
        for (int bank = 0; bank < 32; ++bank) {
            uint32_t words[32] = {};
            int nw = 0;
            for (int l = p0; l < p0 + per_phase; ++l)
                for (int w = 0; w < (width <= 4 ? 1 : width / 4); ++w) {
                    const uint32_t word = (a[l] >> 2) + static_cast<uint32_t>(w);
                    if (static_cast<int>(word % 32u) != bank) continue;
                    bool seen = false;
                    for (int i = 0; i < nw; ++i) seen = seen || words[i] == word;
                    if (!seen) words[nw++] = word;
                }
            worst = nw > worst ? nw : worst;
        }
        total += worst;
    }
    return total;
}

template <int LT, int LOGE>
constexpr uint32_t layout_addr(uint32_t e, uint32_t rn, int pad, int tile, int tile_elems, int esize) {
    const uint32_t row = extract(e, lowmask(LT) & ~rn);
    const uint32_t j = extract(e, rn);
    return (static_cast<uint32_t>(tile * tile_elems) + row * static_cast<uint32_t>((1 << LOGE) + pad) + j) *
           static_cast<uint32_t>(esize);
}

template <int LT, int LOGE>
constexpr int pass_waves(uint32_t writer, uint32_t reader, int pad, int tile_elems, int esize) {
    constexpr int TPT = 1 << (LT - LOGE);
    uint32_t a[32] = {};
    for (int l = 0; l < 32; ++l) {
        const int tile = l / TPT, t = l % TPT;
        a[l] = layout_addr<LT, LOGE>(deposit(static_cast<uint32_t>(t), lowmask(LT) & ~writer), reader, pad, tile,
                                     tile_elems, esize);
    }
    const int stores = (1 << LOGE) * bank_waves(a, esize);
    for (int l = 0; l < 32; ++l) {
        const int tile = l / TPT, t = l % TPT;
        a[l] = layout_addr<LT, LOGE>(deposit(static_cast<uint32_t>(t), lowmask(LT) & ~reader), reader, pad, tile,
                                     tile_elems, esize);
    }
    const int per_load = 16 / esize;
    const int loads = ((1 << LOGE) >= per_load ? (1 << LOGE) / per_load : 1) * bank_waves(a, 16);
    return stores + loads;
}

template <int LOGH, int LOGW, int LOGE, int LOGV, int TS_BYTES, int TC_BYTES>
constexpr SmemCost smem_cost(const Groups& g) {
    constexpr int LT = LOGH + LOGW;
    constexpr int E = 1 << LOGE;
    constexpr int TPT = 1 << (LT - LOGE);
    SmemCost c{0, 0};
    if (!well_formed<LOGH, LOGW, LOGE>(g)) return SmemCost{1 << 20, 1 << 20};
    const int padc = 16 / TC_BYTES, pads = 16 / TS_BYTES;
    const int xch_elems = TPT * (E + padc);
    for (int k = 1; k < g.count; ++k) {
        ++c.passes;
        c.waves += pass_waves<LT, LOGE>(g.reg[k - 1], g.reg[k], padc, xch_elems, TC_BYTES);
    }
    const bool vec_final = LOGV > 0 && (g.reg[g.count - 1] & lowmask(LOGV)) == lowmask(LOGV);
    if (LOGV > 0 && !vec_final) {
        ++c.passes;
        const int out_elems = TPT * (E + pads);
        const int tile_elems = (xch_elems * TC_BYTES > out_elems * TS_BYTES ? xch_elems * TC_BYTES
                                                                           : out_elems * TS_BYTES) /
                               TS_BYTES;
        c.waves += pass_waves<LT, LOGE>(g.reg[g.count - 1], g.reg[0], pads, tile_elems, TS_BYTES);
    }
    return c;
}

// The plan a tile uses: the fewer shared-memory passes, then the fewer
// wavefronts.
template <int LOGH, int LOGW, int LOGE, int LOGV, int TS_BYTES, int TC_BYTES>
constexpr Groups make_groups() {
    constexpr Groups a = lane_fill_groups<LOGH, LOGW, LOGE, LOGV>();
    constexpr Groups b = lanes_first_groups<LOGH, LOGW, LOGE, LOGV>();
    constexpr SmemCost ca = smem_cost<LOGH, LOGW, LOGE, LOGV, TS_BYTES, TC_BYTES>(a);
    constexpr SmemCost cb = smem_cost<LOGH, LOGW, LOGE, LOGV, TS_BYTES, TC_BYTES>(b);
    if constexpr (cb.passes < ca.passes || (cb.passes == ca.passes && cb.waves < ca.waves))
        return b;
    else
        return a;
}

template <typename TS_, typename TC_, int LOGH_, int LOGW_, int LOGE_>
struct TileShape {
    using TS = TS_;
    using TC = TC_;
    static constexpr int LOGH = LOGH_;
    static constexpr int LOGW = LOGW_;
    static constexpr int LT = LOGH + LOGW;
    static constexpr int LOGE = LOGE_ < LT ? LOGE_ : LT;
    static constexpr int E = 1 << LOGE;
    static constexpr int TPT = 1 << (LT - LOGE);  // threads per tile
    static constexpr int VEC_BITS = log2_const(16 / sizeof(TS));
    // Vector loads need bits 0..LOGV-1 contiguous in memory.
    // 16-byte vectors only: bits 0..VEC_BITS-1 must be register bits and be
    // contiguous in memory (contiguous tiles, or at least that many columns).
    static constexpr int LOGV = (LOGE >= VEC_BITS && (LOGW == 0 || LOGW >= VEC_BITS)) ? VEC_BITS : 0;
    static constexpr int V = 1 << LOGV;
    static constexpr Groups G = make_groups<LOGH, LOGW, LOGE, LOGV, sizeof(TS), sizeof(TC)>();
    static_assert(well_formed<LOGH, LOGW, LOGE>(G), "register groups must be well formed");
    static constexpr int TPB = TPT >= 128 ? TPT : 128;
    static constexpr int TILES = TPB / TPT;  // tiles per CTA
    // Final group stores 16-byte vectors when it holds bits 0..LOGV-1;
    // otherwise the narrowed results go back through shared memory into the
    // group-1 layout and leave as 16-byte vectors (STAGE_OUT).
    static constexpr bool VEC_STORE = LOGV > 0 && (G.reg[G.count - 1] & lowmask(LOGV)) == lowmask(LOGV);
    static constexpr bool STAGE_OUT = LOGV > 0 && !VEC_STORE;
    // Exchange layout ("reader-contiguous"): the E values a thread reads in
    // the next group are contiguous (16-byte loads), rows of E padded by one
    // 16-byte chunk so consecutive readers start in different banks.
    static constexpr int PADC = 16 / static_cast<int>(sizeof(TC));
    static constexpr int PADS = 16 / static_cast<int>(sizeof(TS));
    static constexpr int XCH_BYTES = TPT * (E + PADC) * static_cast<int>(sizeof(TC));
    static constexpr int OUT_BYTES = STAGE_OUT ? TPT * (E + PADS) * static_cast<int>(sizeof(TS)) : 0;
    static constexpr int TILE_SMEM = G.count > 1 || STAGE_OUT ? (XCH_BYTES > OUT_BYTES ? XCH_BYTES : OUT_BYTES) : 0;
    static constexpr int SMEM_BYTES = TILES * TILE_SMEM;
    // Offset (in elements) of tile element e in a buffer laid out for a
    // reader whose register bits are RN.
    template <uint32_t RN, int PAD>
    static CUBF_DEV int xaddr(uint32_t e) {
        return static_cast<int>(extract(e, lowmask(LT) & ~RN) * (E + PAD) + extract(e, RN));
    }
};

// Apply the stages STAGE (tile-index bits) of a group whose registers hold the
// tile-index bits REG: register bit j pairs v[r] with v[r | 1 << j].
template <typename Op, int LOGE, uint32_t REG, uint32_t STAGE, typename TC>
CUBF_DEV void apply_group(TC (&v)[1 << LOGE], int inverse) {
    constexpr uint32_t RSTAGE = extract(STAGE, REG);
#pragma unroll
    for (int j = 0; j < LOGE; ++j) {
        if ((RSTAGE >> j) & 1u) {
            if constexpr (Op::kPacked && std::is_same<TC, float>::value && LOGE >= 2) {
                // pair butterflies along register bit k (0, or 1 for the stage on bit 0)
                const int k = j == 0 ? 1 : 0;
#pragma unroll
                for (int r = 0; r < (1 << LOGE); ++r)
                    if (!((r >> j) & 1) && !((r >> k) & 1))
                        Op::apply2(v[r], v[r | (1 << k)], v[r | (1 << j)], v[r | (1 << j) | (1 << k)], inverse);
            } else {
#pragma unroll
                for (int r = 0; r < (1 << LOGE); ++r)
                    if (!((r >> j) & 1)) Op::apply(v[r], v[r | (1 << j)], inverse);
            }
        }
    }
}

// 16-byte shared-memory vector access of N elements of T.
template <typename T>
CUBF_DEV void lds16(const T* p, T* out) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    *reinterpret_cast<uint4*>(out) = u;
}

// Shared-memory exchange into group K and its stages, then the rest.
template <typename Op, typename S, int K>
CUBF_DEV void exchange_groups(typename S::TC (&v)[S::E], typename S::TC* tbuf, uint32_t t, int inverse) {
    if constexpr (K < S::G.count) {
        constexpr uint32_t RP = S::G.reg[K - 1];
        constexpr uint32_t RN = S::G.reg[K];
        constexpr Offsets<S::E> OP = make_offsets<S::E>(RP);
        constexpr Offsets<S::E> ON = make_offsets<S::E>(RN);
        (void)ON;
        if constexpr (K > 1) __syncthreads();  // previous exchange's reads are done
        const uint32_t tp = deposit_rt<lowmask(S::LT) & ~RP, S::LT>(t);
#pragma unroll
        for (int r = 0; r < S::E; ++r) tbuf[S::template xaddr<RN, S::PADC>(tp | OP.v[r])] = v[r];
        __syncthreads();
        // the reader's E values are contiguous: row t, padded
        const typename S::TC* row = tbuf + static_cast<int>(t) * (S::E + S::PADC);
        if constexpr (S::E >= S::PADC) {
#pragma unroll
            for (int r = 0; r < S::E; r += S::PADC) lds16(row + r, &v[r]);
        } else {
#pragma unroll
            for (int r = 0; r < S::E; ++r) v[r] = row[r];
        }
        apply_group<Op, S::LOGE, RN, S::G.stage[K]>(v, inverse);
        exchange_groups<Op, S, K + 1>(v, tbuf, t, inverse);
    }
}

// One tile pass.  The input is `outer` independent arrays of H x 2^log_inner
// elements (H = 2^LOGH transformed rows, row stride 2^log_inner); a tile is H
// rows by W = 2^LOGW adjacent columns.  LOGW == 0 is the contiguous case (row
// stride 1, log_inner ignored).  `in` and `out` may alias (every tile reads all its elements before
// writing any).  Floating-point results are multiplied by `scale` before the
// final narrowing (the FINAL_STORAGE epilogue).
//
// tile_pass is the work of one CTA of such a pass: CTA `vblock` of `vgrid`,
// run by threads vtid = 0 .. TPB-1 with its shared memory at `smem_raw`.  The
// one-shot kernel below passes blockIdx / threadIdx; the persistent chain
// kernel passes queue items.  COHERENT reads through L2 only (data that other
// CTAs of the same launch wrote).
template <typename Op, typename TS, typename TC, int LOGH, int LOGW, int LOGE, bool COHERENT>
CUBF_DEV void tile_pass(const TS* in, TS* out, size_t outer, int log_inner, int inverse, float scale, int cache_mode,
                        unsigned prefetch_stride, size_t vblock, size_t vgrid, uint32_t vtid,
                        unsigned char* smem_raw) {
    using S = TileShape<TS, TC, LOGH, LOGW, LOGE>;
    constexpr Groups G = S::G;
    constexpr int LT = S::LT;

    const int local = vtid / S::TPT;
    const uint32_t t = vtid % S::TPT;
    // Contiguous tiles (LOGW == 0) have row stride 1; strided tiles 2^log_inner.
    const int li = LOGW == 0 ? 0 : log_inner;
    const size_t col_blocks = size_t{1} << (li - LOGW);
    const size_t tile = vblock * S::TILES + local;
    const bool active = tile < outer * col_blocks;
    const size_t o = active ? tile >> (li - LOGW) : 0;
    const size_t cb = active ? tile & (col_blocks - 1) : 0;
    const size_t base = (o << (li + LOGH)) + (cb << LOGW);
    const TS* tin = in + base;
    TS* tout = out + base;
    // Offset of tile element e from the tile base (32-bit: tiles are < 2^31 elements apart only in base).
    auto addr = [&](uint32_t e) -> size_t {
        if constexpr (LOGW == 0)
            return e;
        else
            return (static_cast<size_t>(e >> LOGW) << li) + (e & lowmask(LOGW));
    };
    TC* tbuf = reinterpret_cast<TC*>(smem_raw + local * S::TILE_SMEM);

    // L2 policies: the input of a chain's first pass and the last pass's
    // output are not read again; chain intermediates are kept.
    const uint64_t ld_pol = l2_policy(false);
    const uint64_t st_pol = l2_policy(cache_mode == kChainFirst || cache_mode == kChainMiddle);
    TC v[S::E];
    {  // group 1: 16-byte vector loads along bits 0..LOGV-1
        constexpr uint32_t R0 = G.reg[0];
        constexpr Offsets<S::E> O0 = make_offsets<S::E>(R0);
        const uint32_t te = deposit_rt<lowmask(LT) & ~R0, LT>(t);
#pragma unroll
        for (int q = 0; q < S::E / S::V; ++q) {
            const uint32_t e = te | O0.v[q * S::V];
            if constexpr (S::V > 1) {
                Vec16<TS> x;
                if (active) {
                    const uint4 w = COHERENT ? ld16_hint_cg(tin + addr(e), ld_pol) : ld16_hint(tin + addr(e), ld_pol);
                    x = *reinterpret_cast<const Vec16<TS>*>(&w);
                } else {
#pragma unroll
                    for (int i = 0; i < S::V; ++i) x.v[i] = TS{};
                }
#pragma unroll
                for (int i = 0; i < S::V; ++i) v[q * S::V + i] = Convert<TS, TC>::load(x.v[i]);
            } else {
                v[q] = Convert<TS, TC>::load(active ? (COHERENT ? __ldcg(tin + addr(e)) : tin[addr(e)]) : TS{});
            }
        }
    }
    if constexpr (LOGW == 0) {  // loads issued: prefetch the rows of the CTA one resident wave later
        constexpr size_t row_bytes = (size_t{1} << LOGH) * sizeof(TS);
        const size_t rem = outer % S::TILES;
        prefetch_wave_of(in, S::TILES * row_bytes, (rem ? rem : S::TILES) * row_bytes, prefetch_stride, vblock, vgrid,
                         vtid);
    }
    apply_group<Op, S::LOGE, G.reg[0], G.stage[0]>(v, inverse);
    exchange_groups<Op, S, 1>(v, tbuf, t, inverse);

    constexpr uint32_t RF = G.reg[G.count - 1];
    constexpr Offsets<S::E> OF = make_offsets<S::E>(RF);
    const uint32_t tf = deposit_rt<lowmask(LT) & ~RF, LT>(t);
    if constexpr (std::is_same<TC, float>::value) {
        if (scale != 1.0f) {
#pragma unroll
            for (int r = 0; r < S::E; r += 2) scale2(v[r], v[r + 1], scale);
        }
    }
    auto narrow = [&](TC x) -> TS { return Convert<TS, TC>::store(x); };
    if constexpr (S::STAGE_OUT) {
        // narrowed values -> shared memory in the group-1 (vector) layout ->
        // 16-byte stores; the buffer is the exchange buffer, reused
        constexpr uint32_t R0 = G.reg[0];
        TS* obuf = reinterpret_cast<TS*>(tbuf);
        if constexpr (G.count > 1) __syncthreads();  // exchange reads are done
#pragma unroll
        for (int r = 0; r < S::E; ++r) obuf[S::template xaddr<R0, S::PADS>(tf | OF.v[r])] = narrow(v[r]);
        __syncthreads();
        if (!active) return;
        constexpr Offsets<S::E> O0 = make_offsets<S::E>(R0);
        const uint32_t te = deposit_rt<lowmask(LT) & ~R0, LT>(t);
        const TS* row = obuf + static_cast<int>(t) * (S::E + S::PADS);
#pragma unroll
        for (int q = 0; q < S::E / S::V; ++q) {
            Vec16<TS> x;
            lds16(row + q * S::V, x.v);
            st16_hint(tout + addr(te | O0.v[q * S::V]), *reinterpret_cast<const uint4*>(&x), st_pol);
        }
        return;
    }
    if (!active) return;
    if constexpr (S::VEC_STORE) {
#pragma unroll
        for (int q = 0; q < S::E / S::V; ++q) {
            Vec16<TS> x;
#pragma unroll
            for (int i = 0; i < S::V; ++i) x.v[i] = narrow(v[q * S::V + i]);
            st16_hint(tout + addr(tf | OF.v[q * S::V]), *reinterpret_cast<const uint4*>(&x), st_pol);
        }
    } else {
#pragma unroll
        for (int r = 0; r < S::E; ++r) tout[addr(tf | OF.v[r])] = narrow(v[r]);
    }
}


template <typename Op, typename TS, typename TC, int LOGH, int LOGW, int LOGE>
__global__ void __launch_bounds__(TileShape<TS, TC, LOGH, LOGW, LOGE>::TPB,
                                  (512 / TileShape<TS, TC, LOGH, LOGW, LOGE>::TPB > 0
                                       ? 512 / TileShape<TS, TC, LOGH, LOGW, LOGE>::TPB
                                       : 1))
    bitwise_tile_kernel(const TS* in, TS* out, size_t outer, int log_inner, int inverse, float scale,
                        int cache_mode, unsigned prefetch_stride) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    pdl_begin();
    tile_pass<Op, TS, TC, LOGH, LOGW, LOGE, false>(in, out, outer, log_inner, inverse, scale, cache_mode,
                                                   prefetch_stride, blockIdx.x, gridDim.x, threadIdx.x, smem_raw);
}

}  // namespace cubf::bw
