// planner.cpp -- hardware profile, pass partitioning and static ranking.
#include "planner.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <fstream>
#include <functional>
#include <sstream>

namespace cubf {

Json HardwareProfile::to_json() const {
    return {{"schema", "cubutterfly-b200-hardware-v1"},
            {"name", name},
            {"cc_major", cc_major},
            {"cc_minor", cc_minor},
            {"sm_count", sm_count},
            {"smem_per_block_optin", smem_per_block_optin},
            {"smem_per_sm", smem_per_sm},
            {"regs_per_sm", regs_per_sm},
            {"max_threads_per_sm", max_threads_per_sm},
            {"l2_bytes", l2_bytes},
            {"global_bytes", global_bytes},
            {"hbm_gbs", hbm_gbs},
            {"sm_clock_ghz", sm_clock_ghz},
            {"launch_us", launch_us},
            {"source", source}};
}

std::string HardwareProfile::fingerprint() const {
    std::ostringstream o;
    o << name << "|sm_" << cc_major << cc_minor << "|" << sm_count << "SM|" << smem_per_block_optin << "|"
      << global_bytes;
    return o.str();
}

HardwareProfile profile_from_json(const Json& j) {
    HardwareProfile p;
    require(j.is_object(), "hardware profile must be a JSON object");
    auto get = [&](const char* k, auto& field) {
        if (j.contains(k)) field = j.at(k).get<std::decay_t<decltype(field)>>();
    };
    get("name", p.name);
    get("cc_major", p.cc_major);
    get("cc_minor", p.cc_minor);
    get("sm_count", p.sm_count);
    get("smem_per_block_optin", p.smem_per_block_optin);
    get("smem_per_sm", p.smem_per_sm);
    get("regs_per_sm", p.regs_per_sm);
    get("max_threads_per_sm", p.max_threads_per_sm);
    get("l2_bytes", p.l2_bytes);
    get("global_bytes", p.global_bytes);
    get("hbm_gbs", p.hbm_gbs);
    get("sm_clock_ghz", p.sm_clock_ghz);
    get("launch_us", p.launch_us);
    require(p.sm_count > 0 && p.smem_per_block_optin > 0 && p.hbm_gbs > 0 && p.sm_clock_ghz > 0,
            "hardware profile capacities must be positive");
    p.source = "file";
    return p;
}

HardwareProfile resolve_profile() {
    if (const char* path = std::getenv("CUBUTTERFLY_HARDWARE_MODEL"); path && *path) {
        std::ifstream in(path);
        require(static_cast<bool>(in), std::string("cannot read CUBUTTERFLY_HARDWARE_MODEL file ") + path);
        Json j;
        in >> j;
        HardwareProfile p = profile_from_json(j);
        p.source = std::string("file:") + path;
        return p;
    }
    HardwareProfile p;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        return p;  // builtin B200 profile
    }
    int dev = 0;
    cudaDeviceProp prop{};
    if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
        cudaGetLastError();
        return p;
    }
    p.name = prop.name;
    p.cc_major = prop.major;
    p.cc_minor = prop.minor;
    p.sm_count = prop.multiProcessorCount;
    p.smem_per_block_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
    p.smem_per_sm = static_cast<int>(prop.sharedMemPerMultiprocessor);
    p.regs_per_sm = prop.regsPerMultiprocessor;
    p.max_threads_per_sm = prop.maxThreadsPerMultiProcessor;
    p.l2_bytes = static_cast<std::size_t>(prop.l2CacheSize);
    p.global_bytes = prop.totalGlobalMem;
    // Bandwidth: the B200 figure measured on this platform unless the device
    // is not a B200, then the bus-width x clock estimate at 80 %.
    int mem_clock_khz = 0, bus_bits = 0;
    cudaDeviceGetAttribute(&mem_clock_khz, cudaDevAttrMemoryClockRate, dev);
    cudaDeviceGetAttribute(&bus_bits, cudaDevAttrGlobalMemoryBusWidth, dev);
    if (p.cc_major != 10 && mem_clock_khz > 0 && bus_bits > 0)
        p.hbm_gbs = 0.8 * 2.0 * mem_clock_khz * 1e3 * (bus_bits / 8.0) / 1e9;
    p.source = "device";
    return p;
}

// ---------------------------------------------------------------------------
namespace {

struct Cost {
    double us = 0;
};

double pass_time_us(const HardwareProfile& hw, double elems, double store_bytes, double compute_bytes,
                    int stages, int exchanges, double alu_ops_per_elem_stage, double eff) {
    const double bytes = 2.0 * elems * store_bytes;
    const double t_mem = bytes / (hw.hbm_gbs * 1e3 * eff);
    const double lanes = hw.sm_count * 128.0 * hw.sm_clock_ghz * 1e3;  // ops per us
    const double t_alu = elems * stages * alu_ops_per_elem_stage / lanes;
    const double smem_bpus = hw.sm_count * 128.0 * hw.sm_clock_ghz * 1e3;  // bytes per us
    const double t_smem = elems * exchanges * 2.0 * compute_bytes / smem_bpus;
    return std::max({t_mem, t_alu, t_smem}) + hw.launch_us;
}

bool fits(const LaunchShape& s, const HardwareProfile& hw) {
    return s.threads > 0 && s.threads <= 1024 && s.smem_bytes <= hw.smem_per_block_optin;
}

std::size_t compute_bytes_of(BwType t) { return t == BwType::U64 ? 8 : 4; }

double bw_alu_cost(BwOp op, BwType t) {
    // adds per element per stage (FWHT: one add or sub; zeta: half the
    // elements update; 64-bit integer adds take two issue slots)
    const double base = op == BwOp::Fwht ? 1.0 : 0.5;
    return t == BwType::U64 ? 2.0 * base : base;
}

Mapping bitwise_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::vector<int>& parts) {
    Mapping m;
    m.family = r.bw_op == BwOp::Fwht ? "fwht-tile" : "zeta-tile";
    const double elems = static_cast<double>(r.d.batch) * std::ldexp(1.0, r.log_n);
    int done = 0;
    for (std::size_t i = 0; i < parts.size(); ++i) {
        Pass p;
        p.kind = PassKind::BitwiseTile;
        p.log_h = parts[i];
        p.log_w = i == 0 ? 0 : bw_strided_log_w(r.bw_type);
        p.log_inner = done;
        require(p.log_h >= 1, "mapping pass must transform at least one bit");
        if (i > 0 && p.log_inner < p.log_w)
            throw Unsupported("strided pass needs at least " + std::to_string(p.log_w) + " lower index bits");
        p.shape = bw_shape({r.bw_op, r.bw_type, p.log_h, p.log_w});
        if (!fits(p.shape, hw))
            throw Unsupported("no compiled tile kernel for pass of " + std::to_string(p.log_h) + " bits");
        m.predicted_us += pass_time_us(hw, elems, static_cast<double>(bw_type_bytes(r.bw_type)),
                                       static_cast<double>(compute_bytes_of(r.bw_type)), p.log_h, p.shape.exchanges,
                                       bw_alu_cost(r.bw_op, r.bw_type), i == 0 ? 0.92 : 0.85);
        m.passes.push_back(p);
        done += parts[i];
    }
    require(done == r.log_n, "mapping passes must cover every stage exactly once");
    return m;
}

void compositions(int total, int first_max, int rest_max, int max_parts, std::vector<int>& cur,
                  std::vector<std::vector<int>>& out) {
    if (total == 0) {
        out.push_back(cur);
        return;
    }
    if (static_cast<int>(cur.size()) == max_parts) return;
    const int lim = cur.empty() ? first_max : rest_max;
    for (int h = std::min(lim, total); h >= 1; --h) {
        cur.push_back(h);
        compositions(total - h, first_max, rest_max, max_parts, cur, out);
        cur.pop_back();
    }
}

}  // namespace

void resolve_orders(PlanRequest& r) {
    const Descriptor& d = r.d;
    const bool rin = !d.input_orders.empty() && d.input_orders[0] == CUBUTTERFLY_ORDER_BIT_REVERSED;
    const bool rout = !d.output_orders.empty() && d.output_orders[0] == CUBUTTERFLY_ORDER_BIT_REVERSED;
    r.permute_input = r.permute_output = r.ntt_gs = false;
    switch (d.op) {
        case CUBUTTERFLY_OPERATOR_FFT:
            r.permute_input = rin;
            r.permute_output = rout;
            break;
        case CUBUTTERFLY_OPERATOR_NTT:
            // (N, R): CT.  (R, N): GS.  (N, N): permute, then bit-reversed
            // input -> GS.  (R, R): permute, then natural input -> CT.
            r.permute_input = rin == rout;
            r.ntt_gs = rin != rout ? rin : !rin;
            r.ntt_word32 = d.storage == CUBUTTERFLY_DATA_UINT32;
            r.ntt_lazy = d.modulus < (std::uint64_t{1} << 62);
            break;
        default:
            r.permute_output = rin != rout;
            break;
    }
}

namespace {
double permutation_us(const PlanRequest& r, const HardwareProfile& hw, double elem_bytes) {
    const double bytes = 2.0 * static_cast<double>(r.d.batch) * std::ldexp(1.0, r.log_n) * elem_bytes;
    return bytes / (hw.hbm_gbs * 1e3 * 0.8) + hw.launch_us;
}
void add_boundary(Mapping& m, const PlanRequest& r, const HardwareProfile& hw) {
    m.permute_input = r.permute_input;
    m.permute_output = r.permute_output;
    const double esz = static_cast<double>(storage_bytes(r.d.storage));
    m.predicted_us += (m.permute_input ? permutation_us(r, hw, esz) : 0.0) +
                      (m.permute_output ? permutation_us(r, hw, esz) : 0.0);
    m.staged = r.staged;
    if (m.staged) {
        const std::size_t bytes = r.d.batch * (std::size_t{1} << r.log_n) * storage_bytes(r.d.storage);
        m.staged_bytes = (bytes + 255) / 256 * 256;  // the core's own workspace follows, 256-byte aligned
        m.workspace_bytes += m.staged_bytes;
        m.predicted_us += 2.0 * permutation_us(r, hw, esz);  // gather + scatter
    }
}
}  // namespace

Mapping fwht_tc_mapping(const PlanRequest& r, const HardwareProfile& hw) {
    Mapping m;
    m.family = "fwht-tcgen05";
    const double elems = static_cast<double>(r.d.batch) * std::ldexp(1.0, r.log_n);
    for (int i = 0; i < 2; ++i) {
        Pass p;
        p.kind = PassKind::FwhtTensor;
        p.log_h = r.log_n / 2;
        p.shape = fwht_tc_shape();
        m.passes.push_back(p);
    }
    if (!fits(m.passes[0].shape, hw)) throw Unsupported("tensor-core FWHT tile does not fit the device");
    // one HBM pass; ranked behind the single-pass SIMT tile by the static
    // model (the MEASURE policy or an explicit mapping selects it)
    m.predicted_us = 1.05 * pass_time_us(hw, elems, 2.0, 4.0, r.log_n, 1, 0.5, 0.92);
    return m;
}

Mapping ntt_mapping(const PlanRequest& r, const HardwareProfile& hw) {
    Mapping m;
    m.family = r.ntt_gs ? "ntt-tile-gs" : "ntt-tile-ct";
    const int l = r.log_n;
    const double elems = static_cast<double>(r.d.batch) * std::ldexp(1.0, l);
    const double esz = r.ntt_word32 ? 4.0 : 8.0;
    // 64-bit Shoup butterflies: ~20 integer issue slots per element and stage
    // on the half-rate integer pipe
    const double alu = r.ntt_lazy ? 40.0 : 48.0;
    auto add = [&](PassKind kind, int bits, int inner, bool strided) {
        Pass p;
        p.kind = kind;
        p.log_h = bits;
        p.log_inner = inner;
        p.shape = ntt_shape({l, strided, r.ntt_gs, r.ntt_lazy, r.ntt_word32});
        if (!fits(p.shape, hw)) throw Unsupported("NTT tile does not fit the device");
        m.predicted_us += pass_time_us(hw, elems, esz, 8.0, bits, p.shape.exchanges, alu, 0.85);
        m.passes.push_back(p);
    };
    if (ntt_single_available(l)) {
        add(PassKind::NttSingle, l, 0, false);
    } else if (ntt_available({l, true, r.ntt_gs, r.ntt_lazy, r.ntt_word32})) {
        const int sb = ntt_pass_bits(l, true), cb = ntt_pass_bits(l, false);
        if (!r.ntt_gs) {
            add(PassKind::NttStrided, sb, cb, true);
            add(PassKind::NttContiguous, cb, 0, false);
        } else {
            add(PassKind::NttContiguous, cb, 0, false);
            add(PassKind::NttStrided, sb, cb, true);
        }
    } else {
        throw Unsupported("NTT length must be 2^1 .. 2^" + std::to_string(kNttMaxLog) + " in this build");
    }
    return m;
}

Mapping fft_global_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::vector<int>& parts) {
    Mapping m;
    m.family = "fft-stockham-global";
    const Descriptor& d = r.d;
    const double elems = static_cast<double>(d.batch) * std::ldexp(1.0, r.log_n);
    int ns = 0;
    for (int bits : parts) {
        require(bits >= kFftPassMinLog && bits <= kFftPassMaxLog, "FFT pass radix must be 2^4 .. 2^10");
        Pass p;
        p.kind = PassKind::FftGlobal;
        p.log_h = bits;
        p.log_inner = ns;
        p.shape = fft_global_pass_shape(bits);
        require(fits(p.shape, hw), "FFT pass tile does not fit the device");
        // a CTA takes units_per_cta adjacent columns of the (N 2^log_v) / R
        const std::size_t cols = std::size_t{1} << (r.log_n + r.log_v - bits);
        if (cols % static_cast<std::size_t>(p.shape.units_per_cta) != 0)
            throw Unsupported("FFT pass of " + std::to_string(bits) + " bits needs more columns than this transform has");
        // Measured on a B200: passes the register-direct kernel takes (a first
        // pass of radix >= 2^8, later passes with Ns >= 16 columns) run at
        // 0.8-0.95 of the copy rate up to radix 2^8 (2^30 as 8+7+7+8: 11.2
        // ms), radix 2^9 at ~0.74, radix 2^10 (one 1024-thread CTA per SM) at
        // ~0.5; the staged kernel (first passes below radix 2^8, 0 < Ns < 16)
        // at ~0.55 (2^28 as 7+7+7+7: 3.22 ms, as 8+7+7+6: 2.70 ms).
        const int nsb = ns + r.log_v;
        const bool direct = (nsb == 0 && bits >= 8) || nsb >= 4;
        const double eff = !direct ? 0.55 : (bits >= 10 ? 0.5 : (bits == 9 ? 0.74 : 0.9));
        m.predicted_us += pass_time_us(hw, elems, 8.0, 8.0, bits, p.shape.exchanges, 2.5 / 2.0, eff);
        m.passes.push_back(p);
        ns += bits;
    }
    require(ns == r.log_n, "FFT passes must cover every stage exactly once");
    // a permuted input lands in the output buffer and the passes run in place
    const bool in_place = d.placement == CUBUTTERFLY_PLACEMENT_IN_PLACE || r.permute_input || r.staged;
    const std::size_t bytes = d.batch * (std::size_t{1} << r.log_n) * 8;
    m.workspace_bytes = bytes * ((in_place && parts.size() % 2 == 1) ? 2 : 1);
    return m;
}

Mapping fft_blocked_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::vector<int>& parts) {
    const Descriptor& d = r.d;
    require(d.op == CUBUTTERFLY_OPERATOR_FFT && r.log_v == 0 && !r.fft64, "L2-blocked FFT serves packed complex fp32");
    require(parts.size() >= 2, "L2-blocked FFT needs decimated-transform passes and a combining pass");
    const int log_vb = parts.back();
    const int log_len = r.log_n - log_vb;
    if (!fft_global_pass_narrow_available(log_vb) || parts.front() < kFftDeinterleaveMinLog ||
        parts.front() > kFftPassMaxLog)
        throw Unsupported("L2-blocked FFT: first and combining passes must be radix 2^8 .. 2^10");
    const std::size_t chunk_bytes = std::size_t{kFftBlockChunk} << (log_len + 3);
    if (static_cast<double>(chunk_bytes) > 0.55 * static_cast<double>(hw.l2_bytes))
        throw Unsupported("L2-blocked FFT: a chunk of decimated transforms does not fit L2");
    Mapping m;
    m.family = "fft-l2-blocked";
    const double elems = static_cast<double>(d.batch) * std::ldexp(1.0, r.log_n);
    int ns = 0;
    for (std::size_t i = 0; i + 1 < parts.size(); ++i) {
        const int bits = parts[i];
        require(bits >= kFftPassMinLog && bits <= kFftPassMaxLog, "FFT pass radix must be 2^4 .. 2^10");
        Pass p;
        p.kind = i == 0 ? PassKind::FftDeinterleave : PassKind::FftGlobal;
        p.log_h = bits;
        p.log_inner = ns;
        p.shape = i == 0 ? fft_deinterleave_shape(bits) : fft_global_pass_shape(bits);
        require(fits(p.shape, hw), "FFT pass tile does not fit the device");
        if ((std::size_t{1} << (log_len - bits)) % static_cast<std::size_t>(p.shape.units_per_cta) != 0 && i > 0)
            throw Unsupported("L2-blocked FFT: decimated transforms too short for this pass");
        // only the first pass reads HBM and only the last writes it; the
        // rest move data through L2 (counted at a quarter of the HBM cost).
        // Efficiency is what a B200 measured: these passes move 64- and
        // 128-byte runs at megabyte strides (de-interleave 58 us, chunk pass
        // 64 us per 64 MiB chunk of a 2^30 transform, about 2.2 TB/s).
        const bool first = i == 0, last = i + 2 == parts.size();
        const double share = (first ? 0.5 : 0.125) + (last ? 0.5 : 0.125);
        const double eff = 0.34;
        m.predicted_us += share * pass_time_us(hw, elems, 8.0, 8.0, bits, p.shape.exchanges, 2.5 / 2.0, eff);
        m.passes.push_back(p);
        ns += bits;
    }
    require(ns == log_len, "L2-blocked FFT passes must cover every stage exactly once");
    Pass f;
    f.kind = PassKind::FftGlobalNarrow;
    f.log_h = log_vb;
    f.log_inner = log_len;
    f.shape = fft_global_pass_narrow_shape(log_vb);
    require(fits(f.shape, hw), "FFT pass tile does not fit the device");
    // measured: the 8-column radix-2^10 combining pass of 2^30 points, 8.6 ms (2.0 TB/s)
    m.predicted_us += pass_time_us(hw, elems, 8.0, 8.0, log_vb, f.shape.exchanges, 2.5 / 2.0, 0.31);
    m.passes.push_back(f);
    // blocks of decimated-transform results (one transform of the batch at a
    // time), then one or two chunk staging buffers
    m.workspace_bytes = (std::size_t{8} << r.log_n) + chunk_bytes * (parts.size() > 3 ? 2 : 1);
    return m;
}

Mapping fft_chain_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::vector<int>& parts) {
    const Descriptor& d = r.d;
    require(d.op == CUBUTTERFLY_OPERATOR_FFT && r.log_v == 0 && !r.fft64, "L2-chained FFT serves packed complex fp32");
    if (d.placement == CUBUTTERFLY_PLACEMENT_IN_PLACE || r.permute_input || r.staged)
        throw Unsupported("L2-chained FFT runs out of place on packed natural-order buffers");
    if (parts.size() != 4) throw Unsupported("L2-chained FFT runs four passes (two chained pairs)");
    int total = 0;
    for (int b : parts) {
        if (!fft_chain_pass_available(b)) throw Unsupported("L2-chained FFT passes are radix 2^6 .. 2^8");
        total += b;
    }
    require(total == r.log_n, "FFT passes must cover every stage exactly once");
    // the first pass writes whole columns as 128-byte runs of 16 threads
    if (parts[0] != kFftChainMaxLog) throw Unsupported("L2-chained FFT: the first pass is radix 2^8");
    // each pair's chunks: 32-column tiles of at least one run
    const int key1 = r.log_n - parts[0] - parts[1], key2 = parts[0] + parts[1];
    if (std::min(key1, kFftChainChunkLog - parts[0] - parts[1]) < kFftChainColumnsLog ||
        std::min(key2, kFftChainChunkLog - parts[2] - parts[3]) < kFftChainColumnsLog)
        throw Unsupported("L2-chained FFT: transform too short for 32-column chunks");
    if (static_cast<double>(std::size_t{8} << kFftChainChunkLog) > 0.35 * static_cast<double>(hw.l2_bytes))
        throw Unsupported("L2-chained FFT: a chunk does not fit L2");
    Mapping m;
    m.family = "fft-l2-chain";
    const double elems = static_cast<double>(d.batch) * std::ldexp(1.0, r.log_n);
    int ns = 0;
    for (int bits : parts) {
        Pass p;
        p.kind = PassKind::FftChain;
        p.log_h = bits;
        p.log_inner = ns;
        p.shape = fft_global_pass_shape(bits);
        require(fits(p.shape, hw), "FFT pass tile does not fit the device");
        // measured on a B200 with both passes of a pair in each chain step
        // (PDL between steps): a pair moves ~1.1x its ideal DRAM bytes (the
        // intermediate stays in L2), but the steps run at ~2.6-3 TB/s, so the
        // plan only matches the Stockham plan (2^30: 11.4-11.8 ms against
        // 11.75; 2^28: 2.79 against 2.71 ms; 2^26: 0.72 against 0.67 ms),
        // i.e. each pass at ~0.45 of HBM speed on its full traffic
        m.predicted_us += pass_time_us(hw, elems, 8.0, 8.0, bits, p.shape.exchanges, 2.5 / 2.0, 0.45);
        m.passes.push_back(p);
        ns += bits;
    }
    m.workspace_bytes = (std::size_t{8} << r.log_n) + 128;  // the intermediate, aligned up to a 128-byte line
    return m;
}

std::string Mapping::name() const {
    if (!label.empty()) return label;
    std::ostringstream o;
    if (staged) o << "gather+";
    if (permute_input) o << "bitrev+";
    o << family << "[";
    for (std::size_t i = 0; i < passes.size(); ++i) {
        if (i) o << "+";
        o << passes[i].log_h;
    }
    o << "]";
    if (permute_output) o << "+bitrev";
    if (staged) o << "+scatter";
    return o.str();
}

Json Mapping::to_json() const {
    Json ps = Json::array();
    for (const auto& p : passes) {
        const char* kernel = "bitwise_tile";
        switch (p.kind) {
            case PassKind::FftLocal: kernel = "fft_local"; break;
            case PassKind::FftGlobal: kernel = "fft_global_pass"; break;
            case PassKind::NttStrided: kernel = "ntt_pass_strided"; break;
            case PassKind::NttContiguous: kernel = "ntt_pass_contiguous"; break;
            case PassKind::NttSingle: kernel = "ntt_single"; break;
            case PassKind::FwhtTensor: kernel = "fwht_tcgen05"; break;
            case PassKind::StructuredTile: kernel = "structured_tile"; break;
            case PassKind::StructuredStage: kernel = "structured_column"; break;
            case PassKind::NativeTile: kernel = "fwht_native_tile"; break;
            case PassKind::NativeStage: kernel = "fwht_native_stage"; break;
            case PassKind::Fft64Tile: kernel = "fft64_tile"; break;
            case PassKind::Fft64Stage: kernel = "fft64_column"; break;
            case PassKind::FftDeinterleave: kernel = "fft_deinterleave_pass"; break;
            case PassKind::FftGlobalNarrow: kernel = "fft_global_pass_narrow"; break;
            case PassKind::FftChain: kernel = "fft_chain_pass"; break;
            default: break;
        }
        ps.push_back({{"kernel", kernel},
                      {"log_h", p.log_h},
                      {"log_w", p.log_w},
                      {"log_inner", p.log_inner},
                      {"threads", p.shape.threads},
                      {"smem_bytes", p.shape.smem_bytes},
                      {"units_per_cta", p.shape.units_per_cta},
                      {"elems_per_thread", p.shape.elems_per_thread},
                      {"exchanges", p.shape.exchanges}});
    }
    return {{"schema", "cubutterfly-b200-mapping-v1"},
            {"family", family},
            {"name", name()},
            {"passes", ps},
            {"boundary",
             {{"input_bit_reversal", permute_input},
              {"output_bit_reversal", permute_output},
              {"staged_layout", staged},
              {"staged_bytes", staged_bytes}}},
            {"workspace_bytes", workspace_bytes},
            {"predicted_us", predicted_us}};
}

namespace {
std::vector<Mapping> enumerate_core(const PlanRequest& r, const HardwareProfile& hw);
}

std::vector<Mapping> enumerate_mappings(const PlanRequest& r, const HardwareProfile& hw) {
    std::vector<Mapping> out = enumerate_core(r, hw);
    for (auto& m : out) add_boundary(m, r, hw);
    return out;
}

namespace {
std::vector<Mapping> enumerate_core(const PlanRequest& r, const HardwareProfile& hw) {
    std::vector<Mapping> out;
    if (r.d.op == CUBUTTERFLY_OPERATOR_NTT) {
        out.push_back(ntt_mapping(r, hw));
        return out;
    }
    if (r.d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2 || r.fwht_native || r.fft64) {
        // one shared-memory tile pass for the low 12 (fp64 FFT: 11) stages
        const bool native = r.fwht_native;
        Mapping m;
        m.family = r.fft64 ? "fft64-radix2" : native ? "fwht-native" : "structured-2x2";
        const int tile = std::min(r.log_n, r.fft64 ? 11 : 12);
        const double esz = static_cast<double>(storage_bytes(r.d.storage));
        const double elems = static_cast<double>(r.d.batch) * std::ldexp(1.0, r.log_n);
        Pass t;
        t.kind = r.fft64 ? PassKind::Fft64Tile : native ? PassKind::NativeTile : PassKind::StructuredTile;
        t.log_h = tile;
        t.shape.threads = 256;
        t.shape.smem_bytes = static_cast<int>(esz) << tile;
        t.shape.units_per_cta = 1;
        m.passes.push_back(t);
        m.predicted_us += pass_time_us(hw, elems, esz, esz, tile, tile, 3.0, 0.7);
        // higher stages: one pass each (native), or column passes of up to
        // eight stages (structured, fp64 FFT)
        const int group = native ? 1 : 8;
        for (int s = tile; s < r.log_n;) {
            Pass g;
            g.kind = r.fft64 ? PassKind::Fft64Stage : native ? PassKind::NativeStage : PassKind::StructuredStage;
            g.log_h = std::min(group, r.log_n - s);
            g.log_inner = s;
            g.shape.threads = 256;
            m.passes.push_back(g);
            m.predicted_us += pass_time_us(hw, elems, esz, esz, g.log_h, 0, 3.0, 0.7);
            s += g.log_h;
        }
        out.push_back(m);
        return out;
    }
    const Descriptor& d = r.d;
    if (d.op == CUBUTTERFLY_OPERATOR_FFT && (r.log_n > kFftLocalMaxLog || r.log_v > 0)) {
        if (r.log_n < kFftPassMinLog)
            throw Unsupported("interleaved FFT batches need at least 2^" + std::to_string(kFftPassMinLog) + " points");
        // Multi-pass global Stockham: for each cap on the radix bits of a
        // pass, ceil(L / cap) passes with balanced radices; and a radix-2^8
        // first pass (the register-direct kernel's first pass) followed by
        // balanced passes in ascending radix.
        std::vector<std::vector<int>> partitions;
        for (int cap = kFftPassMaxLog; cap >= 7; --cap) {
            const int np = (r.log_n + cap - 1) / cap;
            std::vector<int> parts;
            for (int i = 0; i < np; ++i) parts.push_back(r.log_n / np + (i < r.log_n % np ? 1 : 0));
            partitions.push_back(parts);
        }
        if (r.log_v == 0 && r.log_n >= 8 + kFftPassMinLog) {
            const int rest = r.log_n - 8;
            for (int np = (rest + 7) / 8; np <= (rest + 5) / 6; ++np) {
                std::vector<int> parts;
                for (int i = 0; i < np; ++i) parts.push_back(rest / np + (i < rest % np ? 1 : 0));
                std::sort(parts.begin(), parts.end());
                parts.insert(parts.begin(), 8);
                // ahead of the balanced partitions: on equal cost the radix-2^8
                // first pass wins (2^30: 8+7+7+8 11.2 ms, 8+8+7+7 11.55 ms)
                partitions.insert(partitions.begin() + (np - (rest + 7) / 8), parts);
            }
        }
        for (const auto& parts : partitions) {
            if (*std::min_element(parts.begin(), parts.end()) < kFftPassMinLog ||
                *std::max_element(parts.begin(), parts.end()) > kFftPassMaxLog)
                continue;
            bool dup = false;
            for (const auto& m : out) {
                std::vector<int> have;
                for (const auto& ps : m.passes) have.push_back(ps.log_h);
                if (have == parts) dup = true;
            }
            if (dup) continue;
            try {
                out.push_back(fft_global_mapping(r, hw, parts));
            } catch (const Unsupported&) {
            }
        }
        // L2-blocked plans of long transforms: V = 2^10 decimated transforms,
        // their L = N / V points in balanced passes of at most 2^10
        if (r.log_v == 0 && !r.fft64 && r.log_n >= 24 && r.log_n <= 30) {
            const int log_len = r.log_n - 10;
            const int np = (log_len + kFftPassMaxLog - 1) / kFftPassMaxLog;
            std::vector<int> parts;
            for (int i = 0; i < np; ++i) parts.push_back(log_len / np + (i < log_len % np ? 1 : 0));
            parts.push_back(10);
            try {
                out.push_back(fft_blocked_mapping(r, hw, parts));
            } catch (const Unsupported&) {
            }
        }
        // L2-chained plans: radix 2^8 first, the rest in three balanced passes
        if (r.log_v == 0 && !r.fft64 && r.log_n >= 26 && r.log_n <= 31) {
            const int rest = r.log_n - kFftChainMaxLog;
            std::vector<int> parts{kFftChainMaxLog};
            for (int i = 0; i < 3; ++i) parts.push_back(rest / 3 + (i < rest % 3 ? 1 : 0));
            try {
                out.push_back(fft_chain_mapping(r, hw, parts));
            } catch (const Unsupported&) {
            }
        }
        if (out.empty()) throw Unsupported("no global FFT pass partition fits this transform");
        std::stable_sort(out.begin(), out.end(),
                         [](const Mapping& a, const Mapping& b) { return a.predicted_us < b.predicted_us; });
        return out;
    }
    if (d.op == CUBUTTERFLY_OPERATOR_FFT) {
        Mapping m;
        m.family = "fft-stockham-local";
        Pass p;
        p.kind = PassKind::FftLocal;
        p.log_h = r.log_n;
        p.shape = fft_local_shape(r.log_n);
        require(fits(p.shape, hw), "FFT tile does not fit the device");
        m.passes.push_back(p);
        const double elems = static_cast<double>(d.batch) * std::ldexp(1.0, r.log_n);
        // 5 N log N flops per transform on FMA lanes (2 flops per lane-op)
        m.predicted_us = pass_time_us(hw, elems, 8.0, 8.0, r.log_n, p.shape.exchanges, 2.5 / 2.0, 0.9);
        out.push_back(m);
        return out;
    }
    if (r.bw_op == BwOp::Fwht && fwht_tc_available(r.log_n, r.bw_type)) out.push_back(fwht_tc_mapping(r, hw));
    // Bitwise operators: every composition of log N into tile passes.
    std::vector<std::vector<int>> parts;
    std::vector<int> cur;
    const int first_max = std::min(bw_max_contiguous_log(r.bw_type), r.log_n);
    const int rest_max = r.bw_op == BwOp::Fwht ? 0 : bw_max_strided_log(r.bw_type);
    compositions(r.log_n, first_max, rest_max, 4, cur, parts);
    for (const auto& p : parts) {
        try {
            out.push_back(bitwise_mapping(r, hw, p));
        } catch (const Unsupported&) {
        }
    }
    if (out.empty()) throw Unsupported("no tile partition of " + std::to_string(r.log_n) + " stages fits");
    std::stable_sort(out.begin(), out.end(),
                     [](const Mapping& a, const Mapping& b) { return a.predicted_us < b.predicted_us; });
    return out;
}
}  // namespace

namespace {
Mapping parse_core(const PlanRequest& r, const HardwareProfile& hw, const std::string& text);
}

Mapping parse_explicit_mapping(const PlanRequest& r, const HardwareProfile& hw, const std::string& text) {
    Mapping m = parse_core(r, hw, text);
    add_boundary(m, r, hw);
    return m;
}

namespace {
Mapping parse_core(const PlanRequest& r, const HardwareProfile& hw, const std::string& text) {
    std::vector<int> parts;
    if (!text.empty() && text.front() == '{') {
        const Json j = Json::parse(text);
        require(j.is_object() && j.value("schema", "") == "cubutterfly-b200-mapping-v1",
                "explicit mapping must use schema cubutterfly-b200-mapping-v1");
        require(j.at("passes").is_array(), "explicit mapping passes must be an array");
        for (const auto& p : j.at("passes")) parts.push_back(p.at("log_h").get<int>());
        if (j.value("family", "") == "fwht-tcgen05") return parse_core(r, hw, "fwht-tcgen05[6+6]");
        if (j.value("family", "") == "fft-l2-blocked") return fft_blocked_mapping(r, hw, parts);
        if (j.value("family", "") == "fft-l2-chain") return fft_chain_mapping(r, hw, parts);
    } else {
        std::string body = text;
        const auto lb = body.find('['), rb = body.rfind(']');
        if (lb != std::string::npos && rb != std::string::npos && rb > lb) body = body.substr(lb + 1, rb - lb - 1);
        std::stringstream ss(body);
        std::string item;
        while (std::getline(ss, item, '+')) {
            require(!item.empty() && item.find_first_not_of("0123456789") == std::string::npos,
                    "explicit mapping must be JSON or a '+'-separated list of pass bit counts");
            parts.push_back(std::stoi(item));
        }
    }
    require(!parts.empty(), "explicit mapping has no passes");
    if (r.d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2 || r.fwht_native || r.fft64)
        return enumerate_core(r, hw).front();
    if (r.d.op == CUBUTTERFLY_OPERATOR_FFT) {
        if (text.find("fft-l2-blocked") != std::string::npos) return fft_blocked_mapping(r, hw, parts);
        if (text.find("fft-l2-chain") != std::string::npos) return fft_chain_mapping(r, hw, parts);
        if (r.log_n > kFftLocalMaxLog || r.log_v > 0) return fft_global_mapping(r, hw, parts);
        require(parts.size() == 1 && parts[0] == r.log_n, "FFT up to 2^13 is one local pass of log N bits");
        return enumerate_core(r, hw).front();
    }
    if (r.d.op == CUBUTTERFLY_OPERATOR_NTT) {
        Mapping m = ntt_mapping(r, hw);
        std::vector<int> planned;
        for (const auto& p : m.passes) planned.push_back(p.log_h);
        if (parts != planned) throw Unsupported("explicit NTT mapping must be the planned pass split " + m.name());
        return m;
    }
    if (r.bw_op == BwOp::Fwht && text.find("tcgen05") != std::string::npos) {
        if (!fwht_tc_available(r.log_n, r.bw_type))
            throw Unsupported("the tensor-core FWHT serves 4096-point bf16 rows");
        return fwht_tc_mapping(r, hw);
    }
    if (r.bw_op == BwOp::Fwht) require(parts.size() == 1, "FWHT executes as a single tile pass");
    return bitwise_mapping(r, hw, parts);
}
}  // namespace

}  // namespace cubf
