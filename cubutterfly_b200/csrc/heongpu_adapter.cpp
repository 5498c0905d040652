// heongpu_adapter.cpp -- HEonGPU's word64 RNS NTT calls served by RNS plans of
// this library (the scalar adapter of reference adapters/heongpu/ntt_adapter.cu).
//
// A call names `batch` polynomials, a modulus for each (through the ordering)
// and HEonGPU's per-modulus root tables.  The first call of a request reads the
// moduli, tables and orders from device memory, checks that every table is the
// bit-reversed power table of a primitive 2N-th root psi (and, for inverse
// calls, that the 1/N table holds N^-1), and prepares RNS plans whose domains
// are those (q, psi): one plan over all polynomials (native-rns) or one per
// modulus (grouped).  Later calls of the same request only execute them.
#include <cubutterfly/cubutterfly.h>
#include <cubutterfly/cubutterfly_b200.h>
#include <cubutterfly/heongpu/ntt_adapter.hpp>
#include <cuntt/rns_c_api.h>

#include "modarith.hpp"

#include <nlohmann/json.hpp>

#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <iostream>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <tuple>
#include <vector>

namespace cubutterfly_heongpu {
namespace {

using U64 = std::uint64_t;
namespace ma = cubf::modarith;

thread_local bool active = false;
thread_local bool frozen = false;
thread_local Execution execution = Execution::NativeRns;
thread_local std::size_t calls = 0, polynomials = 0;

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

void check_rns(int status, const char* what) {
    if (status == 0) return;
    const std::string message = std::string(what) + ": " + cubutterflyRnsLastError();
    if (status == 1) throw std::invalid_argument(message);
    throw std::runtime_error(message);
}

// Device metadata read at preparation (synchronises the caller's stream).
template <class T>
std::vector<T> fetch(const T* device, std::size_t count, cudaStream_t stream) {
    std::vector<T> host(count);
    check(cudaMemcpyAsync(host.data(), device, count * sizeof(T), cudaMemcpyDeviceToHost, stream),
          "adapter metadata read");
    check(cudaStreamSynchronize(stream), "adapter metadata read");
    return host;
}

// psi of one modulus from HEonGPU's table, entry bitrev(j) = root^j: the
// forward table holds the powers of psi, the inverse table those of psi^-1
// (reference ntt_adapter.cu:39-56).  Throws unless root is a primitive 2N-th
// root of a word64 NTT prime below 2^62 and every entry matches.
U64 table_psi(U64 q, const std::vector<U64>& table, int log_n, bool inverse) {
    const std::size_t n = std::size_t{1} << log_n;
    if (q < 3 || q >= (U64{1} << 62) || (q - 1) % (2 * U64(n)))
        throw std::invalid_argument("adapter requires a word64 NTT prime below 2^62 with a 2N-th root");
    const U64 root = table[n / 2];  // bitrev(1)
    const U64 psi = inverse ? ma::powmod(root, q - 2, q) : root;
    if (ma::powmod(psi, n, q) != q - 1 || ma::powmod(psi, 2 * U64(n), q) != 1)
        throw std::invalid_argument("adapter table is not a primitive negacyclic root");
    U64 power = 1;
    for (std::size_t j = 0; j < n; ++j) {
        if (table[ma::bitrev(j, log_n)] != power)
            throw std::invalid_argument("unsupported HEonGPU twiddle table representation");
        power = ma::mulmod(power, root, q);
    }
    return psi;
}

struct RnsPlan {
    cubutterflyRnsPlan handle = nullptr;
    RnsPlan() = default;
    RnsPlan(const RnsPlan&) = delete;
    RnsPlan& operator=(const RnsPlan&) = delete;
    ~RnsPlan() {
        if (handle) cubutterflyRnsDestroy(handle);
    }
};

// Preparation options of the reference's prepare_rns
// (adapters/heongpu/rns_preparation.hpp:17-40): mapping cache directory and
// policy, and the confirmation repetitions, from the environment.
void prepare(RnsPlan& plan, bool in_place, cudaStream_t stream) {
    std::string directory;
    if (const char* v = std::getenv("CUBUTTERFLY_RNS_CACHE")) directory = v;
    int policy = 0;
    if (const char* v = std::getenv("CUBUTTERFLY_RNS_CACHE_POLICY")) {
        const std::string s(v);
        if (s == "prefer")
            policy = 0;
        else if (s == "require")
            policy = 1;
        else if (s == "refresh")
            policy = 2;
        else
            throw std::invalid_argument("CUBUTTERFLY_RNS_CACHE_POLICY must be prefer, require or refresh");
    }
    unsigned repetitions = 3;
    if (const char* v = std::getenv("CUBUTTERFLY_RNS_TUNE_REPETITIONS")) {
        char* end = nullptr;
        errno = 0;
        const unsigned long r = std::strtoul(v, &end, 10);
        if (errno || end == v || *end != '\0' || r == 0 || r > 1000)
            throw std::invalid_argument("CUBUTTERFLY_RNS_TUNE_REPETITIONS must be an integer in [1,1000]");
        repetitions = static_cast<unsigned>(r);
    }
    check_rns(cubutterflyRnsPrepare(plan.handle, in_place ? 1 : 0, directory.c_str(), policy, repetitions, stream),
              "adapter RNS prepare");
}

struct Domain {
    U64 q, psi;
};
struct Placement {
    std::uint32_t domain;
    std::size_t offset;
};

std::unique_ptr<RnsPlan> make_plan(int log_n, bool inverse, const std::vector<Domain>& domains,
                                   const std::vector<Placement>& polys, bool in_place, cudaStream_t stream) {
    nlohmann::json ds = nlohmann::json::array(), ps = nlohmann::json::array();
    for (const auto& d : domains) ds.push_back({{"modulus", d.q}, {"root", d.psi}});
    for (const auto& p : polys) ps.push_back({{"domain", p.domain}, {"input_offset", p.offset}, {"output_offset", p.offset}});
    const nlohmann::json config = {{"schema_version", 1},
                                   {"log_n", log_n},
                                   {"inverse", inverse},
                                   {"ring", "negacyclic"},
                                   {"input_order", inverse ? "bit_reversed" : "natural"},
                                   {"output_order", inverse ? "natural" : "bit_reversed"},
                                   {"domains", ds},
                                   {"polynomials", ps}};
    auto plan = std::make_unique<RnsPlan>();
    check_rns(cubutterflyRnsCreate(config.dump().c_str(), &plan->handle), "adapter RNS plan");
    prepare(*plan, in_place, stream);
    std::size_t bytes = 0;
    check_rns(cubutterflyRnsInfoJson(plan->handle, nullptr, &bytes), "adapter RNS info");
    std::string info(bytes, '\0');
    check_rns(cubutterflyRnsInfoJson(plan->handle, info.data(), &bytes), "adapter RNS info");
    const auto j = nlohmann::json::parse(info.c_str());
    std::cerr << "ntt_adapter_plan,N=" << (std::size_t{1} << log_n) << ",B=" << polys.size()
              << ",execution=" << execution_name(execution) << ",domains=" << domains.size()
              << ",placement=" << (in_place ? "in-place" : "separate") << ",inverse=" << inverse
              << ",mapping=" << (j.contains("mapping") ? j.at("mapping").dump() : std::string("{}")) << '\n';
    return plan;
}

using Key = std::tuple<int, std::uintptr_t, std::uintptr_t, std::uintptr_t, std::uintptr_t, std::uintptr_t, int, int,
                       int, int, int, int, bool>;
struct Prepared {
    std::vector<std::unique_ptr<RnsPlan>> plans;
};
thread_local std::map<Key, Prepared> cache;

Prepared prepare_request(Data64* source, Data64* destination, Root64* roots, Modulus64* moduli,
                         const gpuntt::ntt_rns_configuration<Data64>& cfg, int batch, int modulus_count,
                         Ordering ordering, int* order) {
    const int log_n = cfg.n_power;
    const std::size_t n = std::size_t{1} << log_n;
    const bool inverse = cfg.ntt_type == gpuntt::INVERSE;
    std::vector<int> indices;
    if (ordering != Ordering::Contiguous)
        indices = fetch(order, static_cast<std::size_t>(ordering == Ordering::Modulus ? modulus_count : batch),
                        cfg.stream);
    // modulus index -> polynomial positions, in call order
    std::map<int, std::vector<int>> groups;
    std::set<int> seen;
    for (int b = 0; b < batch; ++b) {
        const int m = ordering == Ordering::Modulus ? indices[b % modulus_count] : b % modulus_count;
        const int p = ordering == Ordering::Polynomial ? indices[b] : b;
        if (m < 0 || p < 0 || !seen.insert(p).second)
            throw std::invalid_argument("negative or overlapping ordered polynomial request");
        groups[m].push_back(p);
    }
    Prepared prepared;
    std::vector<Domain> domains;
    std::map<std::pair<U64, U64>, std::uint32_t> domain_of;
    std::vector<Placement> all;
    const bool in_place = source == destination;
    for (const auto& [m, positions] : groups) {
        const U64 q = fetch(moduli + m, 1, cfg.stream)[0].value;
        const U64 psi = table_psi(q, fetch(roots + static_cast<std::size_t>(m) * n, n, cfg.stream), log_n, inverse);
        if (inverse && fetch(cfg.mod_inverse + m, 1, cfg.stream)[0] != ma::powmod(U64(n) % q, q - 2, q))
            throw std::invalid_argument("inverse NTT normalization differs from 1/N");
        if (execution == Execution::Grouped) {
            std::vector<Placement> polys;
            for (const int p : positions) polys.push_back({0, static_cast<std::size_t>(p) * n});
            prepared.plans.push_back(make_plan(log_n, inverse, {{q, psi}}, polys, in_place, cfg.stream));
        } else {
            const auto found = domain_of.emplace(std::make_pair(q, psi), static_cast<std::uint32_t>(domains.size()));
            if (found.second) domains.push_back({q, psi});
            for (const int p : positions) all.push_back({found.first->second, static_cast<std::size_t>(p) * n});
        }
    }
    if (execution == Execution::NativeRns)
        prepared.plans.push_back(make_plan(log_n, inverse, domains, all, in_place, cfg.stream));
    return prepared;
}

}  // namespace

void set_enabled(bool value) { active = value; }
bool enabled() { return active; }
void freeze_plans(bool value) { frozen = value; }
void reset_counters() { calls = polynomials = 0; }
std::size_t replacement_calls() { return calls; }
std::size_t replacement_polynomials() { return polynomials; }
void clear_cache() {
    cache.clear();
    frozen = false;
}

void set_execution(Execution value) {
    if (value != Execution::NativeRns && value != Execution::Grouped)
        throw std::invalid_argument("invalid HEonGPU NTT execution mode");
    execution = value;
}
Execution get_execution() { return execution; }
const char* execution_name(Execution value) {
    switch (value) {
        case Execution::NativeRns:
            return "native-rns";
        case Execution::Grouped:
            return "grouped";
    }
    throw std::invalid_argument("invalid HEonGPU NTT execution mode");
}

// Request checks of reference ntt_adapter.cu:245-258; the RNS tile passes of
// this build serve 2^12..2^20 in both execution modes (no implicit fallback).
void transform(Data64* source, Data64* destination, Root64* roots, Modulus64* moduli,
               gpuntt::ntt_rns_configuration<Data64> cfg, int batch, int modulus_count, Ordering ordering,
               int* order) {
    if (cfg.ntt_layout != gpuntt::PerPolynomial || cfg.zero_padding ||
        (ordering != Ordering::Contiguous && ordering != Ordering::Modulus && ordering != Ordering::Polynomial) ||
        cfg.reduction_poly != gpuntt::ReductionPolynomial::X_N_plus ||
        (cfg.ntt_type != gpuntt::FORWARD && cfg.ntt_type != gpuntt::INVERSE) || cfg.n_power < 1 ||
        cfg.n_power > 26 || batch <= 0 || modulus_count <= 0 || !source || !destination || !roots || !moduli ||
        (ordering != Ordering::Contiguous && !order) || (cfg.ntt_type == gpuntt::INVERSE && !cfg.mod_inverse))
        throw std::invalid_argument("unsupported or invalid HEonGPU NTT adapter request");
    if (cfg.n_power < 12 || cfg.n_power > 20)
        throw std::invalid_argument("the RNS tile passes support logN 12..20; no implicit fallback");
    int device = 0;
    check(cudaGetDevice(&device), "adapter device identity");
    const Key key{device,
                  reinterpret_cast<std::uintptr_t>(cfg.stream),
                  reinterpret_cast<std::uintptr_t>(roots),
                  reinterpret_cast<std::uintptr_t>(moduli),
                  reinterpret_cast<std::uintptr_t>(order),
                  reinterpret_cast<std::uintptr_t>(cfg.mod_inverse),
                  cfg.n_power,
                  static_cast<int>(cfg.ntt_type),
                  batch,
                  modulus_count,
                  static_cast<int>(ordering),
                  static_cast<int>(execution),
                  source == destination};
    auto found = cache.find(key);
    if (found == cache.end()) {
        if (frozen) throw std::runtime_error("NTT adapter plan miss during frozen measurement/capture");
        found = cache.emplace(key, prepare_request(source, destination, roots, moduli, cfg, batch, modulus_count,
                                                   ordering, order))
                    .first;
    }
    ++calls;
    polynomials += static_cast<std::size_t>(batch);
    for (const auto& plan : found->second.plans)
        check_rns(cubutterflyRnsExecute(plan->handle, source, destination, cfg.stream), "adapter RNS execute");
}

}  // namespace cubutterfly_heongpu

// ---- C entry points (the adapter driven with plain pointers) -----------------
namespace cubf {
void set_last_error(const std::string& message);
}  // namespace cubf

namespace {
template <typename F>
cubutterflyStatus_t guarded(F&& body) noexcept {
    try {
        cubf::set_last_error("");
        body();
        return CUBUTTERFLY_STATUS_SUCCESS;
    } catch (const std::invalid_argument& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::logic_error& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_INTERNAL_ERROR;
    } catch (const std::bad_alloc& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_ALLOC_FAILED;
    } catch (const std::exception& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_BACKEND_ERROR;
    } catch (...) {
        cubf::set_last_error("unrecognized exception");
        return CUBUTTERFLY_STATUS_INTERNAL_ERROR;
    }
}
}  // namespace

extern "C" cubutterflyStatus_t cubutterflyB200HeongpuTransform(const uint64_t* input, uint64_t* output,
                                                              const uint64_t* roots, const void* moduli,
                                                              const uint64_t* mod_inverse, int n_power, int inverse,
                                                              int batch, int modulus_count, int ordering,
                                                              const int* order, int execution, cudaStream_t stream) {
    return guarded([&] {
        namespace h = cubutterfly_heongpu;
        if (ordering < 0 || ordering > 2) throw std::invalid_argument("ordering must be 0, 1 or 2");
        if (execution < 0 || execution > 1) throw std::invalid_argument("execution must be 0 or 1");
        gpuntt::ntt_rns_configuration<Data64> cfg;
        cfg.n_power = n_power;
        cfg.ntt_type = inverse ? gpuntt::INVERSE : gpuntt::FORWARD;
        cfg.mod_inverse = const_cast<Data64*>(mod_inverse);
        cfg.stream = stream;
        h::set_execution(execution ? h::Execution::Grouped : h::Execution::NativeRns);
        h::transform(const_cast<Data64*>(input), output, const_cast<Root64*>(roots),
                     static_cast<Modulus64*>(const_cast<void*>(moduli)), cfg, batch, modulus_count,
                     static_cast<h::Ordering>(ordering), const_cast<int*>(order));
    });
}

extern "C" cubutterflyStatus_t cubutterflyB200HeongpuControl(int freeze, int clear_cache, int reset_counters,
                                                            size_t* calls, size_t* polynomials) {
    return guarded([&] {
        namespace h = cubutterfly_heongpu;
        if (clear_cache) h::clear_cache();
        if (freeze >= 0) h::freeze_plans(freeze != 0);
        if (calls) *calls = h::replacement_calls();
        if (polynomials) *polynomials = h::replacement_polynomials();
        if (reset_counters) h::reset_counters();
    });
}
