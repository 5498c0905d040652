// chain.cuh -- two tile passes over a batch chunked to L2, overlapped chunk by chunk.
//
// A zeta transform longer than one tile runs as a contiguous pass over its
// low index bits (A) and a strided pass over the high bits (B), chunk by
// chunk so that each chunk's intermediate is still in L2 when B reads it
// (the reference's SharedIterative groups, src/shared_iterative.cuh:49-144,
// run one launch per group over the whole batch instead).  B of chunk c needs
// all of A of chunk c; A of chunk c+1 is independent of both.  So the chain
// runs as C + 1 launches on one stream, step k holding the CTAs of B(k-1) and
// of A(k) side by side:
//
//     [A(0)] [B(0) | A(1)] [B(1) | A(2)] ... [B(C-2) | A(C-1)] [B(C-1)]
//
// Stream order gives B(k) its dependency on A(k) (the step before); within a
// step the two roles share the SMs, A streaming from DRAM while B reads L2.
// A step's B CTAs come first (lower block indices are dispatched first), so
// B drains chunk k-1 from L2 while A's CTAs, which follow, fill it with chunk
// k; each A CTA prefetches into L2 the A tile about one resident wave of A
// work later.  Measured on config 3 (2^24 x 16 u32, one B200): B first 727-737
// us, B and A alternating in proportion 856 us, A first 853 us, the first half
// or three quarters of B first and the rest alternating 798 / 765 us.  No CTA
// waits on another; nothing is allocated or synchronised.
//
// One CTA of the step kernel runs SUB = TPB_K / TPB virtual CTAs of its pass
// side by side (tile_pass with virtual block and thread indices), so passes
// with different CTA sizes share one kernel.
#pragma once

#include "bitwise.cuh"

namespace cubf::bw {

struct ChainStep {
    const void* a_in;        // A: input of chunk k (unused when a_blocks == 0)
    void* a_out;             // A: output of chunk k (the intermediate)
    size_t a_outer;          // A: `outer` of tile_pass (contiguous tiles)
    unsigned a_blocks;       // A: CTAs of the step kernel
    void* b_buf;             // B: chunk k-1, in place (unused when b_blocks == 0)
    size_t b_outer;          // B: `outer` of tile_pass (strided tiles)
    unsigned b_blocks;       // B: CTAs of the step kernel
    int log_inner_b;         // B: row stride bits (= pass A's tile bits)
    int inverse;
    float scale_b;           // the final pass's output scale
    unsigned prefetch_stride;  // A: prefetch the A CTA this many A CTAs later (0: off)
};

template <typename Op, typename TS, typename TC, int H0, int H1, int LOGW1, int LOGE>
struct ChainShape {
    using A = TileShape<TS, TC, H0, 0, LOGE>;
    using B = TileShape<TS, TC, H1, LOGW1, LOGE>;
    static constexpr int TPB = A::TPB > B::TPB ? A::TPB : B::TPB;
    static constexpr int SUB_A = TPB / A::TPB;
    static constexpr int SUB_B = TPB / B::TPB;
    static constexpr int SMEM_A = SUB_A * A::SMEM_BYTES;
    static constexpr int SMEM_B = SUB_B * B::SMEM_BYTES;
    static constexpr int SMEM_BYTES = SMEM_A > SMEM_B ? SMEM_A : SMEM_B;
    static constexpr bool kValid = TPB % A::TPB == 0 && TPB % B::TPB == 0;
};

template <typename Op, typename TS, typename TC, int H0, int H1, int LOGW1, int LOGE>
__global__ void __launch_bounds__(ChainShape<Op, TS, TC, H0, H1, LOGW1, LOGE>::TPB,
                                  512 / ChainShape<Op, TS, TC, H0, H1, LOGW1, LOGE>::TPB)
    bitwise_chain_step_kernel(ChainStep s) {
    using K = ChainShape<Op, TS, TC, H0, H1, LOGW1, LOGE>;
    using A = typename K::A;
    using B = typename K::B;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    pdl_begin();
    const size_t b = blockIdx.x;
    // the step's B CTAs first: they drain chunk k-1 from L2 before the A
    // CTAs that come after them fill it with chunk k
    const bool role_b = b < s.b_blocks;
    if (role_b) {
        const int sub = static_cast<int>(threadIdx.x) / B::TPB;
        const size_t vgrid = (s.b_outer * (size_t{1} << (s.log_inner_b - LOGW1)) + B::TILES - 1) / B::TILES;
        TS* buf = static_cast<TS*>(s.b_buf);
        tile_pass<Op, TS, TC, H1, LOGW1, LOGE, false>(buf, buf, s.b_outer, s.log_inner_b, s.inverse, s.scale_b,
                                                      kChainLast, 0, b * K::SUB_B + sub, vgrid,
                                                      threadIdx.x % B::TPB, smem_raw + sub * B::SMEM_BYTES);
    } else {
        const int sub = static_cast<int>(threadIdx.x) / A::TPB;
        const size_t vgrid = (s.a_outer + A::TILES - 1) / A::TILES;
        const size_t vblock = (b - s.b_blocks) * K::SUB_A + sub;
        tile_pass<Op, TS, TC, H0, 0, LOGE, false>(static_cast<const TS*>(s.a_in), static_cast<TS*>(s.a_out),
                                                  s.a_outer, 0, s.inverse, 1.0f, kChainFirst,
                                                  s.prefetch_stride * K::SUB_A, vblock, vgrid, threadIdx.x % A::TPB,
                                                  smem_raw + sub * A::SMEM_BYTES);
    }
}

}  // namespace cubf::bw
