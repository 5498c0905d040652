// kernels.hpp -- host-side view of the compiled sm_100a kernel variants.
//
// Every kernel is a template instantiated for a fixed tile geometry; the
// planner enumerates only the variants listed here and the executor launches
// them through these functions.  No CUDA types beyond cudaStream_t appear.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace cubf {

struct LaunchShape {
    int threads = 0;           // per CTA
    int smem_bytes = 0;        // dynamic shared memory per CTA
    int units_per_cta = 0;     // transforms / tiles handled by one CTA
    int elems_per_thread = 0;  // register-resident values per thread
    int exchanges = 0;         // shared-memory exchanges per tile
};

// ---- FFT (complex fp32) ------------------------------------------------------
constexpr int kFftLocalMaxLog = 13;
// Lengths served by the column-pair (f32x2) kernel.
constexpr int kFftPairMinLog = 5;
constexpr int kFftPairMaxLog = 13;
// Twiddle table of a local plan: W_N^k (k < N, interleaved complex fp32),
// followed for the column-pair lengths by its per-pass column-pair entries.
std::vector<float> fft_local_twiddles(int log_n);
LaunchShape fft_local_shape(int log_n);
cudaError_t launch_fft_local(int log_n, const void* in, void* out, std::size_t batch, const void* twiddles,
                             bool inverse, float scale, cudaStream_t stream);

// Multi-pass global Stockham for N > 2^13: radix 2^4..2^10 per pass.
constexpr int kFftPassMinLog = 4;
constexpr int kFftPassMaxLog = 10;
struct FftOuterTables {
    const void* lo;  // double2 W_N^k, k < 2^split
    const void* hi;  // double2 W_N^(k << split)
    int split;
};
LaunchShape fft_global_pass_shape(int log_r);
// tw1024: float2 W_1024^k, k < 1024 (the in-CTA twiddles of every radix).
// log_v > 0: 2^log_v interleaved transforms (element n of transform l at
// n 2^log_v + l) treated as one array of 2^log_n values; ns_bits then
// includes log_v and `outer` holds W for the transform length 2^(log_n-log_v).
// `outer_shift` > 0: `outer` holds W for 2^(log_n - log_v + outer_shift)
// points (one table set serves the shorter transforms of a blocked plan).
// `narrow`: 8 columns per CTA (64-byte runs, half the shared memory) where
// fft_global_pass_narrow_available(log_r).
// A chunk of one Stockham pass's column tiles (the L2-chained pass pairs of
// the "fft-l2-chain" plans): tile b covers columns base + (b mod tiles_per_run)
// 32 + (b / tiles_per_run) run_stride of one transform, b < tiles_per_run runs.
// src_l2: the source is an L2-resident intermediate (its lines are discarded
// once read); dst_l2: the destination is one (kept in L2).
struct FftChunk {
    std::uint32_t base;
    std::uint32_t tiles_per_run;
    std::uint32_t run_stride;
    std::uint32_t runs;
    bool src_l2;
    bool dst_l2;
};
constexpr int kFftChainMinLog = 6;       // pass radices of the chained plans
constexpr int kFftChainMaxLog = 8;
constexpr int kFftChainColumnsLog = 5;   // 32 columns per CTA
bool fft_chain_pass_available(int log_r);
// One role of a chain step (csrc/fft_chain.cu): a pass of radix 2^log_r with
// Ns = 2^ns_bits over one chunk; a chunk with zero runs leaves the role out.
// Role A (the pair's first pass) writes an L2-kept intermediate and may
// conjugate its input; role B (the second pass) reads one and may conjugate
// and scale its output.  `wait`: role A reads what the previous kernel on
// the stream wrote (role B always does).
struct FftChainRole {
    const void* src;
    void* dst;
    int log_r;
    int ns_bits;
    bool conj_in;
    bool conj_out;
    float scale;
    FftChunk chunk;
    bool wait;
};
// Step k of an L2-chained pass pair: B over chunk k-1 and A over chunk k in
// one launch (A's radix 2^8 when it is the transform's first pass).
cudaError_t launch_fft_chain_step(const FftChainRole& a, const FftChainRole& b, int log_n, const void* tw1024,
                                  const FftOuterTables& outer, cudaStream_t stream);
cudaError_t launch_fft_global_pass(int log_r, const void* src, void* dst, int log_n, int ns_bits,
                                   std::size_t batch, const void* tw1024, const FftOuterTables& outer, bool conj_in,
                                   bool conj_out, float scale, cudaStream_t stream, int log_v = 0,
                                   int outer_shift = 0, bool narrow = false);
bool fft_global_pass_narrow_available(int log_r);
LaunchShape fft_global_pass_narrow_shape(int log_r);

// L2-blocked transforms (csrc/fft.cuh, fft_deinterleave_pass_kernel): the
// first pass (radix 2^log_r, Ns = 1) of transforms m0 .. m0 + 7 of 2^log_v
// transforms of 2^log_len points interleaved element by element in `src`;
// each transform's pass output goes contiguously to dst + (m - m0) 2^log_len
// with an L2 evict-last hint.  log_r in kFftDeinterleaveMinLog .. 10.
constexpr int kFftBlockChunk = 8;
constexpr int kFftDeinterleaveMinLog = 8;
LaunchShape fft_deinterleave_shape(int log_r);
cudaError_t launch_fft_deinterleave_pass(int log_r, const void* src, void* dst, int log_len, int log_v,
                                         std::size_t m0, const void* tw1024, bool conj_in, cudaStream_t stream);

// ---- FWHT / zeta tile passes --------------------------------------------------
enum class BwOp { Fwht = 0, ZetaSubset = 1, ZetaSuperset = 2 };
enum class BwType { F32 = 0, BF16 = 1, F16 = 2, U32 = 3, U64 = 4 };
struct BwVariant {
    BwOp op;
    BwType type;
    int log_h;  // transformed bits per tile
    int log_w;  // adjacent columns per tile (0: contiguous rows)
};
const char* bw_type_name(BwType t);
std::size_t bw_type_bytes(BwType t);
// Fixed column width of strided passes for a storage type (64-byte segments).
int bw_strided_log_w(BwType t);
int bw_max_contiguous_log(BwType t);
int bw_max_strided_log(BwType t);
bool bw_available(const BwVariant& v);
LaunchShape bw_shape(const BwVariant& v);
// outer arrays of (2^log_h x inner) elements; the pass transforms the 2^log_h
// axis.  in may equal out.  cache_mode: 0 streaming single pass, 1 first pass
// of a chain (output kept in L2), 2 last pass of a chain, 3 middle pass.
cudaError_t launch_bw(const BwVariant& v, const void* in, void* out, std::size_t outer, std::size_t inner,
                      bool inverse, float scale, int cache_mode, cudaStream_t stream);

// Chunk-overlapped two-pass chain (csrc/chain.cuh), zeta operators: pass A
// over the low log_h0 = bw_max_contiguous_log bits (contiguous tiles), pass B
// over the remaining log_h1 bits (strided tiles), the batch cut into chunks of
// `chunk` transforms whose intermediate stays in L2; chunks + 1 launches on
// `stream`, step k running B of chunk k-1 beside A of chunk k.
struct BwChain {
    std::size_t n = 0, batch = 0, chunk = 0;
    int log_h0 = 0, log_h1 = 0;
    bool inverse = false;
    float scale = 1.0f;
};
bool bw_chain_available(BwOp op, BwType type, int log_h0, int log_h1);

// Element-granular FWHT (FP32 arithmetic, one rounding to storage; rows of up
// to 2^14) and zeta (any length) for buffers that are element-aligned but not
// 16-byte aligned (csrc/unaligned.cu); `in` may equal `out`.
cudaError_t launch_fwht_unaligned(BwType type, int log_n, const void* in, void* out, std::size_t rows, float scale,
                                  cudaStream_t stream);
cudaError_t launch_zeta_unaligned(BwType type, bool superset, int log_n, const void* in, void* out,
                                  std::size_t batch, bool inverse, cudaStream_t stream);
cudaError_t launch_bw_chain(BwOp op, BwType type, const BwChain& c, const void* in, void* out, cudaStream_t stream);

// ---- FWHT on the tensor cores (tcgen05) ------------------------------------------
// 4096-point bf16 rows as H_64 (x) H_64 contractions (csrc/fwht_tc.cu); in may
// equal out.  `status` (nullable; device-visible, normally mapped pinned host
// memory) receives bit 0 when a bounded MMA-completion wait expired and bit 1
// when the dynamic shared memory was not 1 KiB aligned (the output is then
// not written); the kernel only ever sets bits.
bool fwht_tc_available(int log_n, BwType type);
LaunchShape fwht_tc_shape();
cudaError_t launch_fwht_tc(const void* in, void* out, std::size_t rows, float scale, unsigned int* status,
                           cudaStream_t stream);

// ---- structured 2x2 butterfly (csrc/structured.cu) ---------------------------------
constexpr int kStructuredMaxLog = 30;
// Per-stage matrices (m00, m01, m10, m11), already inverted for an inverse
// transform, in both storage precisions (fp32 values are the fp64 ones cast).
struct StructuredStages {
    float f32[kStructuredMaxLog][4];
    double f64[kStructuredMaxLog][4];
};
// `batch` packed transforms of 2^log_n fp32 (elem_bytes 4) or fp64 (8)
// values; in may equal out.  One tile pass plus one pass per stage >= 12.
cudaError_t launch_structured(int elem_bytes, int log_n, const void* in, void* out, std::size_t batch,
                              const StructuredStages& stages, cudaStream_t stream);

// ---- complex fp64 FFT, radix 2 (csrc/fft64.cu) ---------------------------------------
// twiddles: W_N^k (double2), k < N/2, conjugated for an inverse; scale: 1 or
// 1/N (normalised inverse).  in may equal out.
cudaError_t launch_fft64(int log_n, const void* in, void* out, std::size_t batch, const void* twiddles,
                         double scale, cudaStream_t stream);

// ---- FWHT with native bf16 / fp16 stage storage (csrc/fwht_native.cu) -------------
// Every stage rounds to the storage type; `normalize` halves each stage (an
// inverse normalised by 1/N).  in may equal out.
cudaError_t launch_fwht_native(bool bf16, int log_n, const void* in, void* out, std::size_t batch, bool normalize,
                               cudaStream_t stream);

// ---- arbitrary-length complex FFT (Bluestein, csrc/bluestein.cu) ------------------
// f64 selects complex fp64 (double2) buffers, else complex fp32 (float2).
// tables: chirp_table[j] = exp(s i pi j^2 / n), j < n (s = -1 forward, +1
// inverse), in the storage precision; taps (fp64, m values) = the wrapped
// conj(chirp) of the m-point cyclic convolution.
cudaError_t launch_bluestein_tables(bool f64, std::size_t n, std::size_t m, bool inverse, void* chirp_table,
                                    void* taps, cudaStream_t stream);
// spectrum = taps_spectrum (fp64) * scale, in the storage precision
cudaError_t launch_bluestein_spectrum(bool f64, const void* taps_spectrum, void* spectrum, std::size_t m,
                                      double scale, cudaStream_t stream);
// work (m per transform, packed) = input * chirp, zero-padded
cudaError_t launch_bluestein_pack(bool f64, const void* in, std::size_t in_stride, std::size_t in_batch_stride,
                                  void* work, const void* chirp_table, std::size_t n, std::size_t m, std::size_t batch,
                                  cudaStream_t stream);
// work *= spectrum (per transform)
cudaError_t launch_bluestein_multiply(bool f64, void* work, const void* spectrum, std::size_t m, std::size_t batch,
                                      cudaStream_t stream);
// NTT over u64 words: pack reduces the input mod q (unit_q = floor(2^64 / q))
// and multiplies by the chirp; multiply by the convolution spectrum; unpack
// multiplies by the output chirp.  Every multiplier comes with its Shoup
// quotient table.
cudaError_t launch_bluestein_ntt_pack(const void* in, std::size_t in_stride, std::size_t in_batch_stride, void* work,
                                      const void* chirp, const void* chirp_q, std::size_t n, std::size_t m,
                                      std::size_t batch, std::uint64_t q, std::uint64_t unit_q, cudaStream_t stream);
cudaError_t launch_bluestein_ntt_multiply(void* work, const void* spectrum, const void* spectrum_q, std::size_t m,
                                          std::size_t batch, std::uint64_t q, cudaStream_t stream);
cudaError_t launch_bluestein_ntt_unpack(const void* work, void* out, std::size_t out_stride,
                                        std::size_t out_batch_stride, const void* chirp, const void* chirp_q,
                                        std::size_t n, std::size_t m, std::size_t batch, std::uint64_t q,
                                        cudaStream_t stream);
// output = work[0 .. n) * chirp
cudaError_t launch_bluestein_unpack(bool f64, const void* work, void* out, std::size_t out_stride,
                                    std::size_t out_batch_stride, const void* chirp_table, std::size_t n,
                                    std::size_t m, std::size_t batch, cudaStream_t stream);

// ---- real FFTs over an N/2-point complex FFT (csrc/real_fft.cu) -------------------
// twiddles: W_N^k (complex fp32), k = 0..half.  R2C: z (batch x half, packed)
// -> x (half + 1 per transform at out_batch_stride), times scale.  C2R: x ->
// z with the factor 2 of the half-length inverse and the caller's scales in
// `scale`.
cudaError_t launch_r2c_post(const void* z, void* x, const void* twiddles, std::size_t half, std::size_t batch,
                            std::size_t out_batch_stride, float scale, cudaStream_t stream);
cudaError_t launch_c2r_pre(const void* x, void* z, const void* twiddles, std::size_t half, std::size_t batch,
                           std::size_t in_batch_stride, float scale, cudaStream_t stream);

// ---- NTT tile passes (RNS ABI and the main-ABI cyclic NTT) ----------------------
struct NttPolyDesc {
    std::uint64_t in_off;
    std::uint64_t out_off;
    std::uint32_t domain;
    std::uint32_t pad_;
};
// root_pairs: [domains][N] pairs {root, Shoup quotient of root} (16 bytes,
// 16-byte aligned), so one vector load fetches both.
struct NttTables {
    const std::uint64_t* root_pairs;
    const std::uint64_t* moduli;
    const std::uint64_t* n_inv;
    const std::uint64_t* n_inv_q;
    const std::uint64_t* unit_q = nullptr;  // floor(2^64 / q); needed when input words are reduced
};
struct NttVariant {
    int log_n;            // transform length 2^log_n
    bool strided;         // top bits (strided columns) or low bits (contiguous chunks)
    bool inverse;         // Gentleman-Sande (bit-reversed in, natural out) vs Cooley-Tukey
    bool lazy;            // Harvey lazy reduction (every modulus < 2^62)
    bool word32 = false;  // 32-bit storage words (moduli < 2^32, always lazy)
    int split = 0;        // strided pass bits ceil(L/2) + split (0; +-1 where ntt_split_available)
};
// One launch of a pass (2^12 .. 2^20: strided or contiguous tile pass over the
// polynomials of `polys`, a DEVICE array of `count` entries) or of a
// whole-transform tile (2^1 .. 2^11: `count` packed transforms, domain 0,
// `polys` unused).
struct NttLaunch {
    const void* in = nullptr;
    void* out = nullptr;
    const NttPolyDesc* polys = nullptr;
    std::size_t count = 0;
    NttTables tables{};
    bool in_is_out = false;     // read the output buffer at the output offsets
    bool final_pass = false;    // this pass writes the result (lazy: reduce to [0, q))
    bool final_scale = false;   // multiply the result by N^-1
    bool reduce_input = false;  // reduce input words modulo q on load
};
constexpr int kNttSingleMaxLog = 11;
constexpr int kNttMinLog = 12;
constexpr int kNttMaxLog = 20;
inline int ntt_pass_bits(int log_n, bool strided, int split = 0) {
    return strided ? (log_n + 1) / 2 + split : log_n / 2 - split;
}
// Pass-split alternatives (lazy arithmetic, 2^14 .. 2^18, split -1 or +1).
constexpr int kNttSplitMinLog = 14, kNttSplitMaxLog = 18;
inline bool ntt_split_available(int log_n, int split, bool lazy) {
    return split == 0 || (lazy && (split == 1 || split == -1) && log_n >= kNttSplitMinLog && log_n <= kNttSplitMaxLog);
}
// Two tile passes exist for 2^12 .. 2^20.
bool ntt_available(const NttVariant& v);
// A whole-transform tile exists for 2^1 .. 2^11.
bool ntt_single_available(int log_n);
LaunchShape ntt_shape(const NttVariant& v);
cudaError_t launch_ntt(const NttVariant& v, const NttLaunch& a, cudaStream_t stream);

// ---- bit-reversal permutation ------------------------------------------------------
// out[b][rev(i)] = in[b][i] for `batch` packed transforms of 2^log_n elements
// of elem_bytes (2, 4, 8 or 16) each.  in may equal out (pairs of tiles are swapped
// by one CTA).
cudaError_t launch_bitrev(int elem_bytes, int log_n, const void* in, void* out, std::size_t batch,
                          cudaStream_t stream);
// out[b * out_batch_stride + i * out_stride] = in[b * in_batch_stride + i * in_stride]
// for i < n, b < batch (elements of elem_bytes 2, 4 or 8; strides in elements).
cudaError_t launch_strided_copy(int elem_bytes, const void* in, std::size_t in_stride, std::size_t in_batch_stride,
                                void* out, std::size_t out_stride, std::size_t out_batch_stride, std::size_t n,
                                std::size_t batch, cudaStream_t stream);
// The same over dims = 1..3 axes (extents, per-axis strides in elements).
cudaError_t launch_strided_copy_nd(int elem_bytes, int dims, const std::size_t* extents, const void* in,
                                   const std::size_t* in_strides, std::size_t in_batch_stride, void* out,
                                   const std::size_t* out_strides, std::size_t out_batch_stride, std::size_t batch,
                                   cudaStream_t stream);

}  // namespace cubf
