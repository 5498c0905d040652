// rns_api.cpp -- the cubutterflyRns* C ABI over the B200 NTT tile passes.
//
// Contract (reference src/rns_c_api.cpp:18-112, src/rns_tuning.cpp:117-250):
// status 0 ok / 1 invalid argument or state / 2 runtime failure, thread-local
// error text, strict schema-v1 config JSON with unknown-key rejection,
// Prepare once outside stream capture with a prefer/require/refresh mapping
// cache, Execute asynchronous and allocation-free with alignment and aliasing
// checks.  The mapping space is the B200 one: a two-pass split of the index
// bits (strided top bits, contiguous low bits) with compiled tile kernels.
#include <cuntt/rns_c_api.h>

#include "descriptor.hpp"
#include "kernels.hpp"
#include "modarith.hpp"
#include "planner.hpp"

#include <cuda_runtime_api.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <limits>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

using u64 = std::uint64_t;
using cubf::Json;

thread_local std::string last_error;

void require(bool ok, const std::string& message) {
    if (!ok) throw std::invalid_argument(message);
}
void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string("RNS ") + what + ": " + cudaGetErrorString(e));
    }
}

using cubf::modarith::bitrev;
using cubf::modarith::is_prime;
using cubf::modarith::mulmod;
using cubf::modarith::powmod;
using cubf::modarith::shoup;

struct Domain {
    u64 modulus = 0;
    u64 root = 0;
};
struct Polynomial {
    std::uint32_t domain = 0;
    std::size_t input_offset = 0;
    std::size_t output_offset = 0;
};
struct Config {
    std::uint32_t log_n = 12;
    bool inverse = false;
    bool negacyclic = true;
    bool input_bitrev = false;
    bool output_bitrev = true;
    std::vector<Domain> domains;
    std::vector<Polynomial> polynomials;
};

// ---- strict JSON (schema_version 1) -------------------------------------------
template <typename T>
T json_uint(const Json& v) {
    require(v.is_number_unsigned() || v.is_number_integer(), "RNS JSON integer field has invalid type");
    if (v.is_number_integer() && !v.is_number_unsigned())
        require(v.get<std::int64_t>() >= 0, "RNS JSON integer field must be nonnegative");
    const u64 x = v.get<u64>();
    require(x <= std::numeric_limits<T>::max(), "RNS JSON integer field overflows");
    return static_cast<T>(x);
}
void only_fields(const Json& v, std::initializer_list<const char*> allowed, const char* what) {
    require(v.is_object(), std::string("RNS JSON ") + what + " must be an object");
    for (auto it = v.begin(); it != v.end(); ++it)
        require(std::find_if(allowed.begin(), allowed.end(), [&](const char* a) { return it.key() == a; }) !=
                    allowed.end(),
                std::string("unknown RNS JSON ") + what + " field: " + it.key());
}
bool json_bool(const Json& v, const char* what) {
    require(v.is_boolean(), std::string("RNS JSON ") + what + " must be boolean");
    return v.get<bool>();
}
std::string json_enum(const Json& v, std::initializer_list<const char*> choices) {
    require(v.is_string(), "RNS JSON enum must be a string");
    const auto s = v.get<std::string>();
    for (const char* c : choices)
        if (s == c) return s;
    throw std::invalid_argument("invalid RNS JSON enum: " + s);
}

Config parse_config(const std::string& text) {
    const Json j = Json::parse(text);
    require(j.is_object() && j.contains("schema_version") && json_uint<unsigned>(j.at("schema_version")) == 1,
            "unsupported RNS JSON schema_version");
    only_fields(j, {"schema_version", "log_n", "inverse", "ring", "input_order", "output_order", "domains",
                    "polynomials"},
                "config");
    Config c;
    c.log_n = json_uint<std::uint32_t>(j.at("log_n"));
    c.inverse = json_bool(j.at("inverse"), "inverse");
    c.negacyclic = json_enum(j.at("ring"), {"cyclic", "negacyclic"}) == "negacyclic";
    c.input_bitrev = json_enum(j.at("input_order"), {"natural", "bit_reversed"}) == "bit_reversed";
    c.output_bitrev = json_enum(j.at("output_order"), {"natural", "bit_reversed"}) == "bit_reversed";
    require(j.at("domains").is_array() && j.at("polynomials").is_array(),
            "RNS domains and polynomials must be arrays");
    for (const auto& d : j.at("domains")) {
        only_fields(d, {"modulus", "root"}, "domain");
        c.domains.push_back({json_uint<u64>(d.at("modulus")), json_uint<u64>(d.at("root"))});
    }
    for (const auto& p : j.at("polynomials")) {
        only_fields(p, {"domain", "input_offset", "output_offset"}, "polynomial");
        c.polynomials.push_back({json_uint<std::uint32_t>(p.at("domain")), json_uint<std::size_t>(p.at("input_offset")),
                                 json_uint<std::size_t>(p.at("output_offset"))});
    }
    return c;
}

Json config_json(const Config& c) {
    Json ds = Json::array(), ps = Json::array();
    for (const auto& d : c.domains) ds.push_back({{"modulus", d.modulus}, {"root", d.root}});
    for (const auto& p : c.polynomials)
        ps.push_back({{"domain", p.domain}, {"input_offset", p.input_offset}, {"output_offset", p.output_offset}});
    return {{"schema_version", 1},
            {"log_n", c.log_n},
            {"inverse", c.inverse},
            {"ring", c.negacyclic ? "negacyclic" : "cyclic"},
            {"input_order", c.input_bitrev ? "bit_reversed" : "natural"},
            {"output_order", c.output_bitrev ? "bit_reversed" : "natural"},
            {"domains", ds},
            {"polynomials", ps}};
}

void validate(const Config& c) {
    require(c.log_n >= 1 && c.log_n <= 30, "RNS log_n must be in [1, 30]");
    require(!c.domains.empty(), "RNS plan needs at least one domain");
    require(!c.polynomials.empty(), "RNS plan needs at least one polynomial");
    const u64 n = u64{1} << c.log_n;
    for (const auto& d : c.domains) {
        require(d.modulus > 2 && d.modulus < (u64{1} << 63), "RNS modulus must be in (2, 2^63)");
        require(is_prime(d.modulus), "RNS modulus must be prime");
        const u64 order = c.negacyclic ? 2 * n : n;
        require((d.modulus - 1) % order == 0, "RNS modulus does not admit a root of the required order");
        require(d.root > 0 && d.root < d.modulus, "RNS root must be a canonical residue");
        require(powmod(d.root, order, d.modulus) == 1 && powmod(d.root, order / 2, d.modulus) == d.modulus - 1,
                "RNS root is not primitive of the required order");
    }
    std::vector<std::pair<std::size_t, std::size_t>> outs;
    for (const auto& p : c.polynomials) {
        require(p.domain < c.domains.size(), "RNS polynomial refers to a missing domain");
        require(p.input_offset <= std::numeric_limits<std::size_t>::max() - n &&
                    p.output_offset <= std::numeric_limits<std::size_t>::max() - n,
                "RNS offset overflows");
        outs.emplace_back(p.output_offset, p.output_offset + n);
    }
    std::sort(outs.begin(), outs.end());
    for (std::size_t i = 1; i < outs.size(); ++i)
        require(outs[i].first >= outs[i - 1].second, "RNS output intervals must be disjoint");
}

struct DeviceBuffer {
    void* ptr = nullptr;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() {
        if (ptr) cudaFree(ptr);
    }
    void upload(const void* host, std::size_t bytes) {
        check(cudaMalloc(&ptr, bytes), "table allocation");
        check(cudaMemcpy(ptr, host, bytes, cudaMemcpyHostToDevice), "table upload");
    }
    template <typename T>
    T* as() const {
        return static_cast<T*>(ptr);
    }
};

}  // namespace

struct cubutterflyRnsPlanOpaque {
    Config config;
    int device = 0;
    bool prepared = false;
    bool in_place = false;
    bool needs_scratch = false;
    bool lazy = false;  // every modulus < 2^62: Harvey lazy butterflies allowed
    // The mapping Prepare chose: pass split (strided bits ceil(L/2) + split)
    // and arithmetic (lazy or fully reduced Shoup products).
    int split = 0;
    bool use_lazy = false;
    Json candidates = Json::array();  // Prepare's timings, {mapping, kernel_ms}
    std::size_t scratch_bytes = 0;
    DeviceBuffer root_pairs, moduli, n_inv, n_inv_q, polys, polys_scratch, scratch;
    cubf::NttTables tables{};
    // Prepare results
    bool cache_hit = false;
    std::string cache_key;
    std::string source = "unprepared";
    double kernel_ms = 0.0;

    Json mapping_json() const { return mapping_json_for(split, use_lazy); }

    Json mapping_json_for(int sp, bool lz) const {
        const int l = static_cast<int>(config.log_n);
        const auto s1 = cubf::ntt_shape({l, true, config.inverse, lz, false, sp});
        const auto s2 = cubf::ntt_shape({l, false, config.inverse, lz, false, sp});
        return {{"schema_version", 1},
                {"core_family", "b200_two_pass_tile"},
                {"split", sp},
                {"strided_bits", cubf::ntt_pass_bits(l, true, sp)},
                {"contiguous_bits", cubf::ntt_pass_bits(l, false, sp)},
                {"strided_threads", s1.threads},
                {"contiguous_threads", s2.threads},
                {"strided_columns", s1.units_per_cta},
                {"contiguous_tiles", s2.units_per_cta},
                {"values_per_thread", s1.elems_per_thread},
                {"arithmetic", lz ? "shoup-lazy" : "shoup"},
                {"order", config.inverse ? "contiguous_then_strided" : "strided_then_contiguous"}};
    }

    void build() {
        const Config& c = config;
        const int l = static_cast<int>(c.log_n);
        if (!cubf::ntt_available({l, true, c.inverse}))
            throw std::invalid_argument("RNS log_n must be in [" + std::to_string(cubf::kNttMinLog) + ", " +
                                        std::to_string(cubf::kNttMaxLog) + "] in this build");
        // The tile passes map natural input to bit-reversed output (forward)
        // and bit-reversed input to natural output (inverse).
        require(c.input_bitrev == c.inverse && c.output_bitrev == !c.inverse,
                "this build executes forward natural->bit_reversed and inverse bit_reversed->natural RNS NTTs");
        const std::size_t n = std::size_t{1} << l;
        const std::size_t dn = c.domains.size();
        std::vector<u64> r(dn * n), rq(dn * n), m(dn), ni(dn), niq(dn);
        lazy = true;
        for (std::size_t d = 0; d < dn; ++d) {
            const u64 q = c.domains[d].modulus;
            m[d] = q;
            lazy = lazy && q < (u64{1} << 62);
            // Forward stage s, block i uses root table entry k = 2^s + i.
            //   negacyclic: psi^bitrev_L(k)
            //   cyclic:     omega^(bitrev_s(i) * 2^(L-1-s)), omega = root
            // Inverse (Gentleman-Sande) uses the modular inverses.
            u64 base = c.domains[d].root;
            if (c.inverse) base = powmod(base, q - 2, q);
            std::vector<u64> pw(n);
            pw[0] = 1;
            for (std::size_t j = 1; j < n; ++j) pw[j] = mulmod(pw[j - 1], base, q);
            r[d * n + 0] = 1;
            for (int s = 0; s < l; ++s)
                for (std::size_t i = 0; i < (std::size_t{1} << s); ++i) {
                    const std::size_t k = (std::size_t{1} << s) + i;
                    std::size_t e;
                    if (c.negacyclic)
                        e = bitrev(k, l);
                    else
                        e = bitrev(i, s) << (l - 1 - s);
                    r[d * n + k] = pw[e];
                }
            for (std::size_t k = 0; k < n; ++k) rq[d * n + k] = shoup(r[d * n + k], q);
            ni[d] = powmod(static_cast<u64>(n), q - 2, q);
            niq[d] = shoup(ni[d], q);
        }
        use_lazy = lazy;
        check(cudaGetDevice(&device), "current device");
        std::vector<u64> rp(2 * r.size());
        for (std::size_t k = 0; k < r.size(); ++k) {
            rp[2 * k] = r[k];
            rp[2 * k + 1] = rq[k];
        }
        root_pairs.upload(rp.data(), rp.size() * 8);
        moduli.upload(m.data(), m.size() * 8);
        n_inv.upload(ni.data(), ni.size() * 8);
        n_inv_q.upload(niq.data(), niq.size() * 8);
        tables = {root_pairs.as<u64>(), moduli.as<u64>(), n_inv.as<u64>(), n_inv_q.as<u64>()};
        std::vector<cubf::NttPolyDesc> pd, ps;
        for (std::size_t p = 0; p < c.polynomials.size(); ++p) {
            const auto& x = c.polynomials[p];
            pd.push_back({x.input_offset, x.output_offset, x.domain, 0});
            ps.push_back({x.input_offset, p * n, x.domain, 0});  // pass 1 into private scratch
        }
        polys.upload(pd.data(), pd.size() * sizeof(cubf::NttPolyDesc));
        polys_scratch.upload(ps.data(), ps.size() * sizeof(cubf::NttPolyDesc));
    }

    // In-place execution with permuted offsets lets one polynomial's first
    // pass overwrite another's unread input: route pass 1 through scratch.
    bool aliasing_needs_scratch() const {
        for (const auto& p : config.polynomials)
            if (p.input_offset != p.output_offset) return true;
        return false;
    }

    void launch(const u64* in, u64* out, cudaStream_t stream) {
        const int l = static_cast<int>(config.log_n);
        const std::size_t count = config.polynomials.size();
        const bool inv = config.inverse;
        const cubf::NttVariant first{l, !inv, inv, use_lazy, false, split}, second{l, inv, inv, use_lazy, false, split};
        cubf::NttLaunch a1, a2;
        a1.count = a2.count = count;
        a1.tables = a2.tables = tables;
        a2.final_pass = true;
        a2.final_scale = inv;
        if (needs_scratch) {
            // pass 1 into private scratch; pass 2 reads scratch (its out_off)
            // and writes the caller's output
            u64* tmp = scratch.as<u64>();
            a1.in = in;
            a1.out = tmp;
            a1.polys = polys_scratch.as<cubf::NttPolyDesc>();
            a2.in = tmp;
            a2.out = out;
            a2.polys = polys_scratch_to_out();
        } else {
            a1.in = in;
            a1.out = out;
            a1.polys = a2.polys = polys.as<cubf::NttPolyDesc>();
            a2.in = out;
            a2.out = out;
            a2.in_is_out = true;
        }
        check(cubf::launch_ntt(first, a1, stream), "pass 1 launch");
        check(cubf::launch_ntt(second, a2, stream), "pass 2 launch");
    }

    DeviceBuffer polys_s2o;
    const cubf::NttPolyDesc* polys_scratch_to_out() const { return polys_s2o.as<cubf::NttPolyDesc>(); }

    void prepare_scratch() {
        needs_scratch = in_place && aliasing_needs_scratch();
        if (!needs_scratch) return;
        const std::size_t n = std::size_t{1} << config.log_n;
        scratch_bytes = config.polynomials.size() * n * 8;
        check(cudaMalloc(&scratch.ptr, scratch_bytes), "scratch allocation");
        std::vector<cubf::NttPolyDesc> s2o;
        for (std::size_t p = 0; p < config.polynomials.size(); ++p)
            s2o.push_back({p * n, config.polynomials[p].output_offset, config.polynomials[p].domain, 0});
        polys_s2o.upload(s2o.data(), s2o.size() * sizeof(cubf::NttPolyDesc));
    }
};

namespace {

template <typename F>
int guarded(F&& body) noexcept {
    try {
        last_error.clear();
        body();
        return 0;
    } catch (const std::invalid_argument& e) {
        try {
            last_error = e.what();
        } catch (...) {
        }
        return 1;
    } catch (const Json::exception& e) {
        try {
            last_error = e.what();
        } catch (...) {
        }
        return 1;
    } catch (const std::exception& e) {
        try {
            last_error = e.what();
        } catch (...) {
        }
        return 2;
    } catch (...) {
        try {
            last_error = "unknown RNS failure";
        } catch (...) {
        }
        return 2;
    }
}

std::string cache_key_for(const Json& identity) {
    u64 h = 14695981039346656037ULL;  // FNV-1a over the canonical identity text
    for (unsigned char b : identity.dump()) {
        h ^= b;
        h *= 1099511628211ULL;
    }
    std::ostringstream o;
    o << "rns-b200-v1-" << std::hex << std::setfill('0') << std::setw(16) << h;
    return o.str();
}

double time_plan(cubutterflyRnsPlanOpaque& p, cudaStream_t stream, unsigned reps) {
    const std::size_t n = std::size_t{1} << p.config.log_n;
    std::size_t span_in = 0, span_out = 0;
    for (const auto& x : p.config.polynomials) {
        span_in = std::max(span_in, x.input_offset + n);
        span_out = std::max(span_out, x.output_offset + n);
    }
    DeviceBuffer a, b;
    const std::size_t words = std::max(span_in, span_out);
    check(cudaMalloc(&a.ptr, words * 8), "tuning buffer");
    check(cudaMemsetAsync(a.ptr, 0, words * 8, stream), "tuning buffer init");
    u64* out = a.as<u64>();
    if (!p.in_place) {
        check(cudaMalloc(&b.ptr, words * 8), "tuning buffer");
        out = b.as<u64>();
    }
    cudaEvent_t e0, e1;
    check(cudaEventCreate(&e0), "event");
    check(cudaEventCreate(&e1), "event");
    p.launch(a.as<u64>(), out, stream);
    check(cudaEventRecord(e0, stream), "event record");
    for (unsigned i = 0; i < reps; ++i) p.launch(a.as<u64>(), out, stream);
    check(cudaEventRecord(e1, stream), "event record");
    check(cudaEventSynchronize(e1), "event sync");
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return ms / reps;
}

}  // namespace

extern "C" {

const char* cubutterflyRnsLastError(void) { return last_error.c_str(); }

int cubutterflyRnsCreate(const char* config_json, cubutterflyRnsPlan* result) {
    return guarded([&] {
        require(result != nullptr, "result must be non-null");
        *result = nullptr;
        require(config_json != nullptr, "config JSON must be non-null");
        auto plan = std::make_unique<cubutterflyRnsPlanOpaque>();
        plan->config = parse_config(config_json);
        validate(plan->config);
        plan->build();
        *result = plan.release();
    });
}

int cubutterflyRnsPrepare(cubutterflyRnsPlan plan, int placement, const char* cache_directory, int policy,
                          unsigned repetitions, void* stream_ptr) {
    return guarded([&] {
        require(plan != nullptr, "plan must be non-null");
        require(!plan->prepared, "plan is already prepared; create another plan to retune");
        require(placement == 0 || placement == 1, "invalid placement");
        require(policy >= 0 && policy <= 2, "invalid cache policy");
        require(repetitions > 0, "repetitions must be positive");
        const std::string dir = cache_directory ? cache_directory : "";
        require(!(dir.empty() && policy == 1), "RNS Require policy needs a nonempty cache_directory");
        auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        check(cudaStreamIsCapturing(stream, &cap), "capture query");
        require(cap == cudaStreamCaptureStatusNone, "RNS preparation must run outside CUDA Graph capture");
        plan->in_place = placement == 1;
        plan->prepare_scratch();
        int dev = 0;
        cudaDeviceProp prop{};
        check(cudaGetDevice(&dev), "device");
        check(cudaGetDeviceProperties(&prop, dev), "device properties");
        const Json identity{{"request", config_json(plan->config)},
                            {"placement", plan->in_place ? "in_place" : "separate"},
                            {"hardware",
                             {{"name", prop.name},
                              {"total_global_memory", prop.totalGlobalMem},
                              {"cc_major", prop.major},
                              {"cc_minor", prop.minor},
                              {"multiprocessor_count", prop.multiProcessorCount}}},
                            {"protocol", {{"name", "rns_b200_event_timing_v1"}, {"repetitions", repetitions}}}};
        plan->cache_key = cache_key_for(identity);
        const std::string path = dir.empty() ? "" : dir + "/" + plan->cache_key + ".json";
        if (!path.empty() && policy != 2) {
            std::ifstream in(path);
            if (in) {
                Json rec;
                in >> rec;
                if (rec.at("identity") != identity)
                    throw std::runtime_error("RNS cache identity mismatch: " + path);
                // the record's mapping (split and arithmetic) must be one this
                // build executes for this request
                const Json& m = rec.at("mapping");
                const int sp = m.value("split", 0);
                const bool lz = m.value("arithmetic", "") == "shoup-lazy";
                if ((lz && !plan->lazy) || m != plan->mapping_json_for(sp, lz) ||
                    cubf::ntt_shape({static_cast<int>(plan->config.log_n), true, plan->config.inverse, lz, false, sp})
                            .threads == 0)
                    throw std::runtime_error("RNS cache mapping is not executable by this build: " + path);
                plan->split = sp;
                plan->use_lazy = lz;
                plan->candidates = rec.value("candidates", Json::array());
                plan->kernel_ms = rec.at("kernel_ms").get<double>();
                require(std::isfinite(plan->kernel_ms) && plan->kernel_ms > 0, "invalid RNS cache kernel_ms");
                plan->cache_hit = true;
                plan->source = "prepared_cache_timing_only";
                plan->prepared = true;
                return;
            }
        }
        if (policy == 1) throw std::runtime_error("required RNS prepared cache record is missing: " + path);
        // Candidate search: the pass splits this build has for the length
        // (strided bits ceil(L/2) - 1, + 0, + 1) with lazy arithmetic where
        // every modulus allows it, and the fully reduced arithmetic at the
        // default split; each timed with CUDA events over `repetitions`
        // executions.  The plan's mapping changes only once every candidate
        // has been timed.
        const int l = static_cast<int>(plan->config.log_n);
        std::vector<std::pair<int, bool>> cands;
        for (const int sp : {0, -1, 1})
            for (const bool lz : {true, false}) {
                if (lz && !plan->lazy) continue;
                if (!cubf::ntt_split_available(l, sp, lz)) continue;
                if (cubf::ntt_shape({l, true, plan->config.inverse, lz, false, sp}).threads == 0) continue;
                cands.emplace_back(sp, lz);
            }
        const int keep_split = plan->split;
        const bool keep_lazy = plan->use_lazy;
        Json timings = Json::array();
        double best = 0.0;
        std::pair<int, bool> best_c = cands.front();
        try {
            for (const auto& c : cands) {
                plan->split = c.first;
                plan->use_lazy = c.second;
                const double ms = time_plan(*plan, stream, repetitions);
                timings.push_back({{"mapping", plan->mapping_json()}, {"kernel_ms", ms}});
                if (timings.size() == 1 || ms < best) {
                    best = ms;
                    best_c = c;
                }
            }
        } catch (...) {
            plan->split = keep_split;
            plan->use_lazy = keep_lazy;
            throw;
        }
        plan->split = best_c.first;
        plan->use_lazy = best_c.second;
        plan->candidates = timings;
        plan->kernel_ms = best;
        plan->source = path.empty() ? "uncached_event_timing" : "event_timing";
        if (!path.empty()) {
            ::mkdir(dir.c_str(), 0755);
            const Json rec{{"schema_version", 1},
                           {"identity", identity},
                           {"mapping", plan->mapping_json()},
                           {"kernel_ms", plan->kernel_ms},
                           {"candidates", plan->candidates},
                           {"source", plan->source}};
            const std::string tmp = path + ".tmp";
            {
                std::ofstream out(tmp, std::ios::trunc);
                require(static_cast<bool>(out), "cannot write RNS cache " + tmp);
                out << rec.dump(2) << "\n";
            }
            if (std::rename(tmp.c_str(), path.c_str()) != 0)
                throw std::runtime_error("cannot publish RNS cache record " + path);
        }
        plan->prepared = true;
    });
}

int cubutterflyRnsExecute(cubutterflyRnsPlan plan, const uint64_t* input, uint64_t* output, void* stream) {
    return guarded([&] {
        require(plan != nullptr && plan->prepared, "plan must be prepared");
        require(input != nullptr && output != nullptr, "device pointers must be non-null");
        require(reinterpret_cast<std::uintptr_t>(input) % 8 == 0 && reinterpret_cast<std::uintptr_t>(output) % 8 == 0,
                "device pointers must be uint64 aligned");
        require((input == output) == plan->in_place, "pointer aliasing does not match prepared placement");
        plan->launch(input, output, reinterpret_cast<cudaStream_t>(stream));
    });
}

int cubutterflyRnsInfoJson(cubutterflyRnsPlan plan, char* buffer, size_t* bytes) {
    return guarded([&] {
        require(plan != nullptr && bytes != nullptr, "plan and bytes must be non-null");
        const Json info{{"prepared", plan->prepared},
                        {"workspace_bytes", plan->scratch_bytes},
                        {"request", config_json(plan->config)},
                        {"mapping", plan->mapping_json()},
                        {"placement", plan->in_place ? "in_place" : "separate"},
                        {"cache_hit", plan->cache_hit},
                        {"cache_key", plan->cache_key},
                        {"source", plan->source},
                        {"kernel_ms", plan->kernel_ms},
                        {"candidates", plan->candidates}};
        const std::string text = info.dump();
        const std::size_t capacity = *bytes;
        *bytes = text.size() + 1;
        if (!buffer) return;
        require(capacity >= *bytes, "info JSON buffer is too small");
        std::memcpy(buffer, text.c_str(), *bytes);
    });
}

int cubutterflyRnsDestroy(cubutterflyRnsPlan plan) {
    return guarded([&] { delete plan; });
}

}  // extern "C"
