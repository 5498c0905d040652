// fwht.cuh -- FWHT tile kernel with fp32 compute held in packed register pairs.
//
// Same tile/group schedule as bitwise_tile_kernel (contiguous rows; group 1
// loaded with 16-byte vectors, later groups through a conflict-free padded
// shared-memory exchange), specialised for the FWHT butterfly in fp32:
// values live as 64-bit pairs (register bits 0 of the group), so every stage
// on register bits >= 1 is one add.f32x2 + one sub.f32x2 per two butterflies
// and the output scale is one mul.f32x2 per pair -- the Blackwell packed fp32
// pipe, with no repacking between stages.  Storage is bf16, fp16 or fp32;
// results are scaled and rounded once (the FINAL_STORAGE epilogue of the
// reference's FP16 path, src/butterfly.cu:1451-1470, :1882-1897).
#pragma once

#include "bitwise.cuh"
#include "f32x2.cuh"

namespace cubf::fwht {

using namespace cubf::f32x2;

// Storage <-> pair conversions (16-bit types pack two elements per word).
template <typename TS>
struct PairIO;
template <>
struct PairIO<__nv_bfloat16> {
    // word holds elements (2i, 2i+1) in its (low, high) halves
    static CUBF_DEV P widen(uint32_t w) { return pk(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u)); }
    static CUBF_DEV uint32_t narrow(P p) {
        float lo, hi;
        up(p, lo, hi);
        uint32_t r;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
        return r;
    }
};
template <>
struct PairIO<__half> {
    static CUBF_DEV P widen(uint32_t w) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w);
        return pk(__low2float(h), __high2float(h));
    }
    static CUBF_DEV uint32_t narrow(P p) {
        float lo, hi;
        up(p, lo, hi);
        uint32_t r;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
        return r;
    }
};

template <typename TS, int LOGH, int LOGE>
using FwhtShape = bw::TileShape<TS, float, LOGH, 0, LOGE>;

// Rows of at most 4 threads finish their thread bits with warp shuffles: the
// partner's value arrives over the lane crossbar and the butterfly is
// own * (+1 | -1) + partner (exact), one packed FMA per pair.
template <typename S>
struct ShuffleFinish {
    static constexpr bool value = S::TPT > 1 && S::TPT <= 4;
};

template <typename S>
CUBF_DEV void shuffle_stages(P (&v)[S::E / 2], uint32_t t) {
    constexpr uint32_t R0 = S::G.reg[0];
    constexpr uint32_t THREAD_BITS = lowmask(S::LT) & ~R0;  // tile bits held across lanes
#pragma unroll
    for (int k = 0; k < S::LT - S::LOGE; ++k) {
        // k-th thread bit <-> lane bit k of t (threads of a tile are adjacent lanes)
        const float s = ((t >> k) & 1u) ? -1.f : 1.f;
        const P sgn = pk(s, s);
        (void)THREAD_BITS;
#pragma unroll
        for (int i = 0; i < S::E / 2; ++i) {
            float a, b;
            up(v[i], a, b);
            const float pa = __shfl_xor_sync(0xffffffffu, a, 1 << k);
            const float pb = __shfl_xor_sync(0xffffffffu, b, 1 << k);
            v[i] = fma2(v[i], sgn, pk(pa, pb));
        }
    }
}

// Stages STAGE of a group with register bits REG on pair registers.
template <int LOGE, uint32_t REG, uint32_t STAGE>
CUBF_DEV void pair_stages(P (&v)[(1 << LOGE) / 2]) {
    constexpr uint32_t RS = extract(STAGE, REG);
    constexpr int NP = (1 << LOGE) / 2;
#pragma unroll
    for (int j = 0; j < LOGE; ++j) {
        if ((RS >> j) & 1u) {
            if (j == 0) {
#pragma unroll
                for (int i = 0; i < NP; ++i) {
                    float a, b;
                    up(v[i], a, b);
                    v[i] = pk(a + b, a - b);
                }
            } else {
                const int m = 1 << (j - 1);
#pragma unroll
                for (int i = 0; i < NP; ++i)
                    if (!(i & m)) {
                        const P a = v[i], b = v[i | m];
                        v[i] = add2(a, b);
                        v[i | m] = sub2(a, b);
                    }
            }
        }
    }
}

template <typename S, int K>
CUBF_DEV void pair_exchanges(P (&v)[S::E / 2], float* tbuf, uint32_t t) {
    if constexpr (K < S::G.count) {
        constexpr uint32_t RP = S::G.reg[K - 1];
        constexpr uint32_t RN = S::G.reg[K];
        constexpr Offsets<S::E> OP = make_offsets<S::E>(RP);
        if constexpr (K > 1) __syncthreads();
        const uint32_t tp = deposit_rt<lowmask(S::LT) & ~RP, S::LT>(t);
#pragma unroll
        for (int i = 0; i < S::E / 2; ++i) {
            float a, b;
            up(v[i], a, b);
            tbuf[S::template xaddr<RN, 4>(tp | OP.v[2 * i])] = a;
            tbuf[S::template xaddr<RN, 4>(tp | OP.v[2 * i + 1])] = b;
        }
        __syncthreads();
        const float* row = tbuf + static_cast<int>(t) * (S::E + 4);
        if constexpr (S::E >= 4) {
#pragma unroll
            for (int i = 0; i < S::E / 2; i += 2) {
                const ulonglong2 w = *reinterpret_cast<const ulonglong2*>(row + 2 * i);
                v[i] = w.x;
                v[i + 1] = w.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < S::E / 2; ++i) v[i] = pk(row[2 * i], row[2 * i + 1]);
        }
        pair_stages<S::LOGE, RN, S::G.stage[K]>(v);
        pair_exchanges<S, K + 1>(v, tbuf, t);
    }
}

// Resident CTAs per SM the register allocation must allow: as many as the
// exchange buffers fit in shared memory (1 KB per CTA is reserved by the
// runtime), at most 8, and no fewer registers than 88 per thread (64 values
// in 32 register pairs plus addressing; tighter bounds spill).
template <typename TS, int LOGH, int LOGE>
constexpr int fwht_min_blocks() {
    using S = FwhtShape<TS, LOGH, LOGE>;
    constexpr int smem = ShuffleFinish<S>::value ? 0 : S::SMEM_BYTES;
    constexpr int by_smem = (228 * 1024) / (smem + 1024);
    constexpr int by_regs = 65536 / (S::TPB * 88);
    constexpr int b = by_smem < by_regs ? by_smem : by_regs;
    return b > 8 ? 8 : (b < 1 ? 1 : b);
}

// Group-1 input of one thread: the 16-byte vectors of row `tin` it holds
// (zeros for an inactive row).
template <typename TS, int LOGH, int LOGE>
CUBF_DEV void fwht_load(const TS* tin, bool active, uint32_t t, uint4 (&w)[FwhtShape<TS, LOGH, LOGE>::E /
                                                                          FwhtShape<TS, LOGH, LOGE>::V]) {
    using S = FwhtShape<TS, LOGH, LOGE>;
    constexpr uint32_t R0 = S::G.reg[0];
    constexpr Offsets<S::E> O0 = make_offsets<S::E>(R0);
    const uint32_t te = deposit_rt<lowmask(S::LT) & ~R0, S::LT>(t);
#pragma unroll
    for (int q = 0; q < S::E / S::V; ++q)
        w[q] = active ? __ldg(reinterpret_cast<const uint4*>(tin + (te | O0.v[q * S::V]))) : make_uint4(0, 0, 0, 0);
}

// One row of 2^LOGH elements (per thread-group of the CTA) from its loaded
// group-1 vectors `w`; results go to `tout` (the row in HBM).  Every thread
// of the CTA must call it (it contains barriers when the row spans several
// threads' exchanges).
template <typename TS, int LOGH, int LOGE>
CUBF_DEV void fwht_row(const uint4 (&w)[FwhtShape<TS, LOGH, LOGE>::E / FwhtShape<TS, LOGH, LOGE>::V], TS* tout,
                       bool active, uint32_t t, float* tbuf, float scale) {
    using S = FwhtShape<TS, LOGH, LOGE>;
    constexpr bw::Groups G = S::G;
    constexpr int LT = S::LT;
    constexpr int NP = S::E / 2;
    P v[NP];
    {
#pragma unroll
        for (int q = 0; q < S::E / S::V; ++q) {
            if constexpr (sizeof(TS) == 4) {
                v[q * 2] = (static_cast<P>(w[q].y) << 32) | w[q].x;
                v[q * 2 + 1] = (static_cast<P>(w[q].w) << 32) | w[q].z;
            } else {
                v[q * 4 + 0] = PairIO<TS>::widen(w[q].x);
                v[q * 4 + 1] = PairIO<TS>::widen(w[q].y);
                v[q * 4 + 2] = PairIO<TS>::widen(w[q].z);
                v[q * 4 + 3] = PairIO<TS>::widen(w[q].w);
            }
        }
    }
    pair_stages<S::LOGE, G.reg[0], G.stage[0]>(v);
    constexpr bool kShuffle = ShuffleFinish<S>::value;
    if constexpr (kShuffle)
        shuffle_stages<S>(v, t);
    else
        pair_exchanges<S, 1>(v, tbuf, t);

    if (scale != 1.0f) {
        const P s2 = pk(scale, scale);
#pragma unroll
        for (int i = 0; i < NP; ++i) v[i] = mul2(v[i], s2);
    }
    constexpr uint32_t RF = kShuffle ? G.reg[0] : G.reg[G.count - 1];
    constexpr Offsets<S::E> OF = make_offsets<S::E>(RF);
    const uint32_t tf = deposit_rt<lowmask(LT) & ~RF, LT>(t);
    if constexpr (kShuffle || S::VEC_STORE) {
        if (!active) return;
#pragma unroll
        for (int q = 0; q < S::E / S::V; ++q) {
            uint4 w;
            if constexpr (sizeof(TS) == 4) {
                w = make_uint4(static_cast<uint32_t>(v[q * 2]), static_cast<uint32_t>(v[q * 2] >> 32),
                               static_cast<uint32_t>(v[q * 2 + 1]), static_cast<uint32_t>(v[q * 2 + 1] >> 32));
            } else {
                w = make_uint4(PairIO<TS>::narrow(v[q * 4]), PairIO<TS>::narrow(v[q * 4 + 1]),
                               PairIO<TS>::narrow(v[q * 4 + 2]), PairIO<TS>::narrow(v[q * 4 + 3]));
            }
            __stcs(reinterpret_cast<uint4*>(tout + (tf | OF.v[q * S::V])), w);
        }
    } else {
        // Results leave through shared memory in the group-1 layout so that
        // global stores are 16-byte vectors.
        constexpr uint32_t R0 = G.reg[0];
        constexpr int PADS = 16 / static_cast<int>(sizeof(TS));
        if constexpr (G.count > 1) __syncthreads();
        if constexpr (sizeof(TS) == 2) {
            uint16_t* obuf = reinterpret_cast<uint16_t*>(tbuf);
#pragma unroll
            for (int i = 0; i < NP; ++i) {
                const uint32_t w = PairIO<TS>::narrow(v[i]);
                obuf[S::template xaddr<R0, PADS>(tf | OF.v[2 * i])] = static_cast<uint16_t>(w);
                obuf[S::template xaddr<R0, PADS>(tf | OF.v[2 * i + 1])] = static_cast<uint16_t>(w >> 16);
            }
        } else {
#pragma unroll
            for (int i = 0; i < NP; ++i) {
                float a, b;
                up(v[i], a, b);
                tbuf[S::template xaddr<R0, PADS>(tf | OF.v[2 * i])] = a;
                tbuf[S::template xaddr<R0, PADS>(tf | OF.v[2 * i + 1])] = b;
            }
        }
        __syncthreads();
        if (!active) return;
        constexpr Offsets<S::E> O0 = make_offsets<S::E>(R0);
        const uint32_t te = deposit_rt<lowmask(LT) & ~R0, LT>(t);
        const TS* orow = reinterpret_cast<const TS*>(tbuf) + static_cast<int>(t) * (S::E + PADS);
#pragma unroll
        for (int q = 0; q < S::E / S::V; ++q)
            __stcs(reinterpret_cast<uint4*>(tout + (te | O0.v[q * S::V])),
                   *reinterpret_cast<const uint4*>(orow + q * S::V));
    }
}

// Contiguous rows of 2^LOGH elements, `rows` of them; in may equal out.
template <typename TS, int LOGH, int LOGE>
__global__ void __launch_bounds__(FwhtShape<TS, LOGH, LOGE>::TPB, fwht_min_blocks<TS, LOGH, LOGE>())
    fwht_tile_kernel(const TS* in, TS* out, size_t rows, float scale, unsigned prefetch_stride) {
    using S = FwhtShape<TS, LOGH, LOGE>;
    static_assert(S::E >= 2 && S::V * sizeof(TS) == 16, "FWHT tiles move 16-byte vectors");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    pdl_begin();
    const int local = threadIdx.x / S::TPT;
    const uint32_t t = threadIdx.x % S::TPT;
    const size_t row = static_cast<size_t>(blockIdx.x) * S::TILES + local;
    const bool active = row < rows;
    const TS* tin = in + (active ? row : 0) * (size_t{1} << LOGH);
    TS* tout = out + (active ? row : 0) * (size_t{1} << LOGH);
    float* tbuf = reinterpret_cast<float*>(smem_raw + local * S::TILE_SMEM);
    uint4 w[S::E / S::V];
    fwht_load<TS, LOGH, LOGE>(tin, active, t, w);
    {  // loads issued: prefetch the tile of the CTA one resident wave later into L2
        constexpr size_t row_bytes = (size_t{1} << LOGH) * sizeof(TS);
        const size_t rem = rows % S::TILES;
        prefetch_next_wave(in, S::TILES * row_bytes, (rem ? rem : S::TILES) * row_bytes, prefetch_stride);
    }
    fwht_row<TS, LOGH, LOGE>(w, tout, active, t, tbuf, scale);
}

}  // namespace cubf::fwht
