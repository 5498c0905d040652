// planner.hpp -- B200 hardware profile, mappings and the stage partitioner.
//
// Replaces the reference's selection stack (mapping_selector.cpp:9-46 ->
// plan_registry.cpp:551-1292 -> a Python static ranker subprocess) with a C++
// planner: the stage set of a transform is partitioned into HBM passes, each
// pass a compiled tile kernel whose on-chip footprint fits the hardware
// profile; candidates are ranked by a roofline cost model (bytes moved per
// pass against the profile's HBM bandwidth, integer/FP issue time and launch
// latency), and the MEASURE policy times the best finalists on the device.
#pragma once

#include "descriptor.hpp"
#include "kernels.hpp"

#include <string>
#include <vector>

namespace cubf {

// Capacity and throughput facts of the target (reference hardware_model.hpp:35-113).
struct HardwareProfile {
    std::string name = "NVIDIA B200";
    int cc_major = 10;
    int cc_minor = 0;
    int sm_count = 148;
    int smem_per_block_optin = 232448;  // 227 KB
    int smem_per_sm = 233472;           // 228 KB
    int regs_per_sm = 65536;
    int max_threads_per_sm = 2048;
    std::size_t l2_bytes = 126ull << 20;
    std::size_t global_bytes = 0;
    double hbm_gbs = 6450.0;     // measured STREAM-style copy on this platform
    double sm_clock_ghz = 1.9;   // boost clock under memory-bound load
    double launch_us = 2.5;      // per-kernel launch + drain
    std::string source = "builtin";
    Json to_json() const;
    std::string fingerprint() const;
};

// The profile of the current device: env CUBUTTERFLY_HARDWARE_MODEL (a JSON
// file) overrides; otherwise live device properties over B200 defaults; with
// no device, the builtin B200 profile.
HardwareProfile resolve_profile();
HardwareProfile profile_from_json(const Json& j);

enum class PassKind {
    FftLocal,
    FftGlobal,
    BitwiseTile,
    NttStrided,
    NttContiguous,
    NttSingle,
    FwhtTensor,
    StructuredTile,
    StructuredStage,
    NativeTile,
    NativeStage,
    Fft64Tile,
    Fft64Stage,
    FftDeinterleave,  // L2-blocked FFT: first pass of a chunk of decimated transforms
    FftChain,         // L2-chained FFT: a pass run chunk by chunk, its pair partner reading it from L2
    FftGlobalNarrow   // L2-blocked FFT: the combining pass (8 columns per CTA)
};

struct Pass {
    PassKind kind = PassKind::BitwiseTile;
    int log_h = 0;      // transformed index bits
    int log_w = 0;      // adjacent untouched columns per tile (bitwise)
    int log_inner = 0;  // log2 of the row stride of this pass (bitwise); Ns bits (global FFT)
    LaunchShape shape;
};

struct Mapping {
    std::string family;  // "fft-stockham-local", "fwht-tile", "zeta-tile", "ntt-tile-ct", ...
    std::vector<Pass> passes;
    // Logical-order boundary: bit-reversal permutation of the input before
    // the first pass and of the output after the last.
    bool permute_input = false;
    bool permute_output = false;
    // Strided or padded layout: gathered into a packed buffer at the start of
    // the workspace (staged_bytes), transformed there in place, scattered out.
    bool staged = false;
    std::size_t staged_bytes = 0;
    std::size_t workspace_bytes = 0;
    double predicted_us = 0.0;
    std::string label;  // replaces the derived name when set (composite plans)
    std::string name() const;
    Json to_json() const;
};

struct PlanRequest {
    Descriptor d;  // normalised
    int log_n = 0;
    // FFT batches interleaved element-wise (element stride = batch, batch
    // stride 1): log2 of the batch, else 0.  Always planned as global passes.
    int log_v = 0;
    BwType bw_type = BwType::F32;
    BwOp bw_op = BwOp::Fwht;
    // Bit-reversal permutations the logical orders require (see
    // resolve_orders); a permuted input makes the core run in place.
    bool permute_input = false;
    bool permute_output = false;
    // A strided or padded layout runs staged through a packed buffer (the
    // core then runs in place on it).
    bool staged = false;
    // NTT: Gentleman-Sande passes (bit-reversed input to natural output)
    // instead of Cooley-Tukey (natural input to bit-reversed output).
    bool ntt_gs = false;
    bool ntt_word32 = false;  // uint32 storage
    bool ntt_lazy = false;    // modulus < 2^62
    // FWHT on bf16 / fp16 with NATIVE compute: every stage rounds to storage
    bool fwht_native = false;
    bool fft64 = false;  // complex fp64 FFT (radix-2 passes)
};

// Fill the order-dependent fields of a request from its descriptor:
//   FFT            bit-reversed input / output -> permute before / after;
//   FWHT, zeta     both commute with bit reversal (H and the subset order are
//                  invariant under reversing the bit positions), so equal
//                  orders need nothing and unequal ones one permutation of
//                  the output;
//   NTT            natural -> bit-reversed runs Cooley-Tukey, bit-reversed ->
//                  natural Gentleman-Sande; equal orders permute the input
//                  and then run Gentleman-Sande (natural) or Cooley-Tukey
//                  (bit-reversed).
void resolve_orders(PlanRequest& r);

// The tensor-core FWHT (4096-point bf16 rows as H_64 (x) H_64 on tcgen05).
Mapping fwht_tc_mapping(const PlanRequest& r, const HardwareProfile& hw);
// The NTT passes of the request (one whole-transform tile up to 2^11, else
// the strided and contiguous passes in execution order).
Mapping ntt_mapping(const PlanRequest& r, const HardwareProfile& hw);
// Multi-pass global FFT with the given radix bits per pass.
Mapping fft_global_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::vector<int>& parts);
// L2-blocked FFT of long transforms (family "fft-l2-blocked"): parts are the
// radix bits of the passes of each decimated transform of L = N / V points
// (the first one the de-interleaving pass), then log V, the radix of the
// final combining pass.  Two HBM round trips whatever the pass count.
Mapping fft_blocked_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::vector<int>& parts);
// L2-chained FFT (family "fft-l2-chain"): four Stockham passes of radix
// 2^6..2^8 run as two pairs; each pair runs chunk by chunk (32 MiB of values),
// the second pass of a chunk reading the first one's output from L2 and
// discarding it there, so each pair costs one HBM round trip.  Out of place,
// packed, natural order.
Mapping fft_chain_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::vector<int>& parts);
// Values per chunk of an L2-chained pass pair (32 MiB of complex fp32).
constexpr int kFftChainChunkLog = 22;
// Every legal mapping of the request, ranked best first by the static model.
std::vector<Mapping> enumerate_mappings(const PlanRequest& r, const HardwareProfile& hw);
// Parse an EXPLICIT mapping: the JSON of Mapping::to_json, or a pass list
// "h0+h1+..." of transformed bits per pass (bitwise operators).
Mapping parse_explicit_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::string& text);

}  // namespace cubf
