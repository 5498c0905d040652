// fft_chain.cu -- chain steps of the L2-chained FFT plans ("fft-l2-chain").
//
// An L2-chained plan runs the four Stockham passes of a long transform as two
// pass pairs; each pair goes chunk by chunk so that the pair's second pass
// (B) reads the chunk its first pass (A) wrote while the chunk is still in L2.
// B of chunk k needs all of A of chunk k; A of chunk k+1 needs nothing of
// either, and their memory is disjoint (chunks own disjoint column sets of
// both the source and the destination).  So a pair of C chunks runs as C + 1
// launches on one stream, step k holding the tiles of B(k-1) and of A(k):
//
//     [A(0)] [B(0) | A(1)] [B(1) | A(2)] ... [B(C-2) | A(C-1)] [B(C-1)]
//
// Within a step the two roles share the SMs: A streams its chunk from HBM
// into L2 while B drains the previous chunk from L2 to HBM.  Steps are
// launched as programmatic dependents of the step before (PDL).  Only the
// CTAs that read what earlier steps wrote wait for them (griddepcontrol.wait:
// the previous grid complete and its writes visible) -- B always, A on the
// first step of a pair (pair two reads all of pair one; pair one's first
// step reads the caller's input).  A CTA lets the next step launch once it
// has started and, if it waits, once its wait is over, so a step's CTAs that
// do not wait run beside the step before at most, whose memory they do not
// touch, never beside an older one.  A(k+1) thus starts on SMs that step k's
// tail leaves idle.  A's CTAs come first in the grid (lower block indices are
// dispatched first); B's follow.  Every step has a waiting CTA, so steps
// still complete in stream order.
//
// A step CTA runs SUB = TPB / TPB_pass tiles of its role side by side
// (reg_pass_tile with virtual block and thread indices), so passes of
// different CTA sizes (radix 2^7: 256 threads, 2^8: 512) share one kernel.
// No CTA waits on another; nothing is allocated.
#include "fft.cuh"
#include "kernels.hpp"
#include "launch_util.cuh"

namespace cubf {
namespace fft {

struct ChainStepArgs {
    // role A: the pair's first pass over chunk k
    const float2* a_src;
    float2* a_dst;
    RegChunk a_chunk;
    int a_ns_bits;
    int a_conj_in;
    unsigned a_blocks;  // CTAs of the step kernel
    unsigned a_tiles;   // pass tiles (a_blocks x SUB_A)
    unsigned a_prefetch;
    int a_wait;  // A reads what the previous kernel wrote
    // role B: the pair's second pass over chunk k-1
    const float2* b_src;
    float2* b_dst;
    RegChunk b_chunk;
    int b_ns_bits;
    int b_conj_out;
    float b_scale;
    unsigned b_blocks;
    unsigned b_tiles;
    int log_n;
    const float2* tw1024;
    OuterTwiddles outer;
};

template <int LA, bool FA, int LB>
struct ChainStepShape {
    using GA = GlobalRegShape<LA, 32>;
    using GB = GlobalRegShape<LB, 32>;
    static constexpr int TPB = GA::TPB > GB::TPB ? GA::TPB : GB::TPB;
    static constexpr int SUB_A = TPB / GA::TPB;
    static constexpr int SUB_B = TPB / GB::TPB;
    static constexpr int SMEM_A = SUB_A * GA::SMEM_BYTES;
    static constexpr int SMEM_B = SUB_B * GB::SMEM_BYTES;
    static constexpr int SMEM_BYTES = SMEM_A > SMEM_B ? SMEM_A : SMEM_B;
    static constexpr int MINB = 1024 / TPB;  // 64 registers per thread, as the single passes
    static_assert(TPB % GA::TPB == 0 && TPB % GB::TPB == 0, "pass CTA sizes must divide the step's");
    static_assert(GA::SMEM_BYTES % 16 == 0 && GB::SMEM_BYTES % 16 == 0, "tile slices stay 16-byte aligned");
};

template <int LA, bool FA, int LB>
__global__ void __launch_bounds__(ChainStepShape<LA, FA, LB>::TPB, ChainStepShape<LA, FA, LB>::MINB)
    fft_chain_step_kernel(ChainStepArgs s) {
    using K = ChainStepShape<LA, FA, LB>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // The next step may launch once every CTA of this one has passed the
    // trigger; a CTA that waits triggers after its wait, so the next step's
    // CTAs that do not wait never run beside a step older than this one.
    const size_t b = blockIdx.x;
    if (b >= s.a_blocks) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        constexpr int TB = K::GB::TPB;
        const int sub = static_cast<int>(threadIdx.x) / TB;
        reg_pass_tile<LB, false, 32, true, 2>(s.b_src, s.b_dst, s.log_n, s.b_ns_bits, s.tw1024, s.outer, 0,
                                           s.b_conj_out, s.b_scale, 0, 0u, 0, s.b_chunk,
                                           (b - s.a_blocks) * K::SUB_B + sub,
                                           s.b_tiles, static_cast<int>(threadIdx.x) % TB,
                                           smem_raw + sub * K::GB::SMEM_BYTES);
    } else {
        if (s.a_wait) asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        constexpr int TA = K::GA::TPB;
        const int sub = static_cast<int>(threadIdx.x) / TA;
        reg_pass_tile<LA, FA, 32, true, 1>(s.a_src, s.a_dst, s.log_n, s.a_ns_bits, s.tw1024, s.outer, s.a_conj_in, 0,
                                        1.0f, 0, s.a_prefetch, 0, s.a_chunk, b * K::SUB_A + sub,
                                        s.a_tiles, static_cast<int>(threadIdx.x) % TA,
                                        smem_raw + sub * K::GA::SMEM_BYTES);
    }
}

}  // namespace fft

namespace {

template <int LA, bool FA, int LB>
struct ChainStepEntry {
    using K = fft::ChainStepShape<LA, FA, LB>;
    static cudaError_t launch(const FftChainRole& a, const FftChainRole& b, int log_n, const void* tw1024,
                              const FftOuterTables& outer, cudaStream_t stream) {
        auto kernel = fft::fft_chain_step_kernel<LA, FA, LB>;
        static KernelSetup setup;
        int grid_cap = 0;
        cudaError_t e = setup_kernel(setup, kernel, K::TPB, K::SMEM_BYTES, &grid_cap);
        if (e != cudaSuccess) return e;
        const std::size_t a_tiles = static_cast<std::size_t>(a.chunk.tiles_per_run) * a.chunk.runs;
        const std::size_t b_tiles = static_cast<std::size_t>(b.chunk.tiles_per_run) * b.chunk.runs;
        if (a_tiles % K::SUB_A != 0 || b_tiles % K::SUB_B != 0) return cudaErrorInvalidValue;
        const std::size_t a_blocks = a_tiles / K::SUB_A, b_blocks = b_tiles / K::SUB_B;
        if (a_blocks + b_blocks == 0) return cudaSuccess;
        if (a_blocks + b_blocks > 0x7fffffffULL) return cudaErrorInvalidConfiguration;
        fft::ChainStepArgs s{};
        s.a_src = static_cast<const float2*>(a.src);
        s.a_dst = static_cast<float2*>(a.dst);
        s.a_chunk = fft::RegChunk{a.chunk.base, a.chunk.tiles_per_run, a.chunk.run_stride, 0, 1};
        s.a_ns_bits = a.ns_bits;
        s.a_conj_in = a.conj_in ? 1 : 0;
        s.a_blocks = static_cast<unsigned>(a_blocks);
        s.a_tiles = static_cast<unsigned>(a_tiles);
        // an A tile prefetches the A tile one resident wave of the step later
        s.a_prefetch = static_cast<unsigned>(grid_cap) * K::SUB_A;
        s.b_src = static_cast<const float2*>(b.src);
        s.b_dst = static_cast<float2*>(b.dst);
        s.b_chunk = fft::RegChunk{b.chunk.base, b.chunk.tiles_per_run, b.chunk.run_stride, 1, 0};
        s.b_ns_bits = b.ns_bits;
        s.b_conj_out = b.conj_out ? 1 : 0;
        s.b_scale = b.scale;
        s.b_blocks = static_cast<unsigned>(b_blocks);
        s.b_tiles = static_cast<unsigned>(b_tiles);
        s.log_n = log_n;
        s.tw1024 = static_cast<const float2*>(tw1024);
        s.outer = fft::OuterTwiddles{static_cast<const double2*>(outer.lo), static_cast<const double2*>(outer.hi),
                                     outer.split};
        s.a_wait = a.wait ? 1 : 0;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(static_cast<unsigned>(a_blocks + b_blocks));
        cfg.blockDim = dim3(K::TPB);
        cfg.dynamicSmemBytes = K::SMEM_BYTES;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kernel, s);
    }
};

using StepLaunch = cudaError_t (*)(const FftChainRole&, const FftChainRole&, int, const void*,
                                   const FftOuterTables&, cudaStream_t);
// [a_log_r - 6][b_log_r - 6] for a pair whose first pass is not the
// transform's first (pair two), and [b_log_r - 6] for pair one (A radix 2^8).
constexpr StepLaunch kLaterSteps[3][3] = {
    {ChainStepEntry<6, false, 6>::launch, ChainStepEntry<6, false, 7>::launch, ChainStepEntry<6, false, 8>::launch},
    {ChainStepEntry<7, false, 6>::launch, ChainStepEntry<7, false, 7>::launch, ChainStepEntry<7, false, 8>::launch},
    {ChainStepEntry<8, false, 6>::launch, ChainStepEntry<8, false, 7>::launch, ChainStepEntry<8, false, 8>::launch}};
constexpr StepLaunch kFirstSteps[3] = {ChainStepEntry<8, true, 6>::launch, ChainStepEntry<8, true, 7>::launch,
                                       ChainStepEntry<8, true, 8>::launch};

}  // namespace

cudaError_t launch_fft_chain_step(const FftChainRole& a, const FftChainRole& b, int log_n, const void* tw1024,
                                  const FftOuterTables& outer, cudaStream_t stream) {
    if (!fft_chain_pass_available(a.log_r) || !fft_chain_pass_available(b.log_r) || log_n > 31)
        return cudaErrorInvalidValue;
    const bool first = a.ns_bits == 0;
    if (first && a.log_r != kFftChainMaxLog) return cudaErrorInvalidValue;  // the first pass writes 128-byte runs
    if ((!first && a.ns_bits < kFftChainColumnsLog) || b.ns_bits < kFftChainColumnsLog) return cudaErrorInvalidValue;
    const int ia = a.log_r - kFftChainMinLog, ib = b.log_r - kFftChainMinLog;
    return first ? kFirstSteps[ib](a, b, log_n, tw1024, outer, stream)
                 : kLaterSteps[ia][ib](a, b, log_n, tw1024, outer, stream);
}

}  // namespace cubf
