// c_api.cpp -- the cubutterfly* C ABI over the B200 planner and kernels.
//
// Contract (reference src/c_api.cpp): exceptions never cross the ABI;
// protect() maps them to status codes with a thread-local last error
// (reference c_api.cpp:121-163); string queries use the two-call NULL-buffer
// protocol (:497-520); workspace is caller-owned (:4890-4995); execution is
// asynchronous on the handle stream, allocation-free, with the in-place /
// out-of-place pointer rule (:5002-5004).
#include <cubutterfly/cubutterfly.h>
#include <cubutterfly/cubutterfly_b200.h>

#include "descriptor.hpp"
#include "kernels.hpp"
#include "modarith.hpp"
#include "planner.hpp"

#include <cuda_runtime_api.h>
#include <fcntl.h>
#include <sys/file.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <new>
#include <sstream>
#include <string>
#include <vector>

struct cubutterflyHandle {
    cudaStream_t stream = nullptr;
    cubutterflyLogCallback_t logger = nullptr;
    void* logger_data = nullptr;
    std::string cache_path;
};

struct cubutterflyPlan {
    cubf::Descriptor desc;
    cubf::PlanRequest req;
    cubf::Mapping mapping;
    cubf::HardwareProfile hw;
    cubutterflySelectionSource_t source = CUBUTTERFLY_SELECTION_STATIC_MODEL;
    std::string reason;
    std::size_t input_bytes = 0;
    std::size_t output_bytes = 0;
    void* workspace = nullptr;
    std::size_t workspace_size = 0;
    void* twiddles = nullptr;  // FFT: W_N^k, k < N (local) or W_1024^k (global passes), complex fp32
    void* outer_lo = nullptr;  // global FFT: double2 W_N^k, k < 2^split
    void* outer_hi = nullptr;  // global FFT: double2 W_N^(k << split)
    int outer_split = 0;
    // NTT: one allocation holding the {root, Shoup quotient} pairs, the
    // per-modulus constants and the per-transform offsets of the tile passes.
    void* ntt_block = nullptr;
    cubf::NttTables ntt_tables{};
    const cubf::NttPolyDesc* ntt_polys = nullptr;
    int device = 0;
    // Device-side status word of plans whose kernels wait on the device (the
    // tensor-core FWHT): mapped pinned host memory the kernel ORs failure
    // bits into, read (and cleared) by the next Execute without a sync.
    unsigned int* status_host = nullptr;
    unsigned int* status_dev = nullptr;
    cudaStream_t steady_stream = nullptr;
    bool steady_ready = false;
    // Rank two and three: packed rank-one child plans.  FFT / NTT: one per
    // axis, innermost first, each run in place on a packed copy of the tensor
    // (axes other than the innermost transposed innermost through a second
    // buffer).  FWHT / zeta: one child over the flattened index, on the
    // caller's buffers when both layouts are packed (`flat`).
    struct Axis {
        std::unique_ptr<cubutterflyPlan> plan;
        std::size_t n = 0, outer = 0, inner = 0;  // length; blocks before and elements after the axis
        std::size_t ws_offset = 0;                // child workspace inside this plan's workspace
    };
    std::vector<Axis> axes;
    bool flat = false;
    std::size_t packed_bytes = 0;  // one packed copy of the tensor (256-byte aligned)
    // R2C / C2R: axes[0] is the N/2-point complex FFT; the half-length
    // spectrum lives at the start of the workspace (packed_bytes).
    bool embedded = false;  // zero-extended embedding: axes[0] transforms the padded rows in place
    cubf::StructuredStages structured{};  // structured 2x2: per-stage matrices (inverted for an inverse plan)
    cubutterflyFftTransformType_t real_kind = CUBUTTERFLY_FFT_C2C;
    bool real_nd = false;  // rank-two / rank-three R2C / C2R: axes[0] rows, axes[1] outer axes
    // FFT composites of packed tensors whose outer axes qualify as
    // interleaved batches (`direct`): the innermost axis runs from the input
    // into the output, every other axis in place there as `groups` blocks of
    // interleaved transforms -- no gather, transposes or scatter.
    bool direct = false;
    std::size_t groups = 1;
    void* real_tw = nullptr;  // W_N^k, k = 0..N/2, complex fp32
    // Arbitrary-length FFT (Bluestein): axes[0] / axes[1] are the forward and
    // unnormalised inverse conv-point FFTs, in place on the work buffer at the
    // start of the workspace; bluestein_tables holds the chirp (n values) and,
    // 256-byte aligned after it, the scaled convolution spectrum (conv values).
    bool bluestein = false;
    std::size_t conv = 0;
    void* bluestein_tables = nullptr;
    // Extents the plan transforms physically (padded or convolution lengths),
    // when they differ from the descriptor's.
    std::vector<std::size_t> physical;
    ~cubutterflyPlan() {
        if (twiddles) cudaFree(twiddles);
        if (outer_lo) cudaFree(outer_lo);
        if (outer_hi) cudaFree(outer_hi);
        if (ntt_block) cudaFree(ntt_block);
        if (real_tw) cudaFree(real_tw);
        if (bluestein_tables) cudaFree(bluestein_tables);
        if (status_host) cudaFreeHost(status_host);
    }
};

namespace {

thread_local std::string last_error;

struct CudaFailure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

std::size_t align256(std::size_t v) { return (v + 255) / 256 * 256; }

template <typename F>
cubutterflyStatus_t protect(F&& body) noexcept {
    try {
        last_error.clear();
        body();
        return CUBUTTERFLY_STATUS_SUCCESS;
    } catch (const cubf::Unsupported& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_NOT_SUPPORTED;
    } catch (const CudaFailure& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_CUDA_ERROR;
    } catch (const std::invalid_argument& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::overflow_error& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::bad_alloc& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_ALLOC_FAILED;
    } catch (const nlohmann::json::exception& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::logic_error& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_INTERNAL_ERROR;
    } catch (const std::runtime_error& e) {
        last_error = e.what();
        return CUBUTTERFLY_STATUS_BACKEND_ERROR;
    } catch (...) {
        last_error = "unrecognized exception";
        return CUBUTTERFLY_STATUS_INTERNAL_ERROR;
    }
}

using cubf::require;

void copy_text(const std::string& value, char* dst, std::size_t* bytes) {
    require(bytes != nullptr, "size query pointer must be non-null");
    const std::size_t need = value.size() + 1;
    if (dst == nullptr) {
        *bytes = need;
        return;
    }
    require(*bytes >= need, "destination string buffer is too small");
    std::memcpy(dst, value.c_str(), need);
    *bytes = need;
}

cubf::Descriptor& desc_of(cubutterflyDescriptor_t d) {
    require(d != nullptr, "descriptor must be non-null");
    return *d;
}

void log_event(const cubutterflyHandle* h, cubutterflyLogLevel_t level, const char* event, const std::string& msg) {
    if (h && h->logger) h->logger(level, event, msg.c_str(), h->logger_data);
}

// ---- plan cache: {"schema", "entries": {key: mapping-json}} ------------------
std::string workload_key(const cubutterflyPlan& p) {
    std::ostringstream o;
    o << cubf::semantic_json(p.desc).dump() << "|" << p.hw.fingerprint();
    return o.str();
}

class FileLock {
  public:
    explicit FileLock(const std::string& path) {
        fd_ = ::open((path + ".lock").c_str(), O_CREAT | O_RDWR, 0644);
        if (fd_ >= 0) ::flock(fd_, LOCK_EX);
    }
    ~FileLock() {
        if (fd_ >= 0) {
            ::flock(fd_, LOCK_UN);
            ::close(fd_);
        }
    }

  private:
    int fd_ = -1;
};

cubf::Json read_cache(const std::string& path) {
    std::ifstream in(path);
    if (!in) return {{"schema", "cubutterfly-b200-plan-cache-v1"}, {"entries", cubf::Json::object()}};
    cubf::Json j;
    in >> j;
    require(j.is_object() && j.value("schema", "") == "cubutterfly-b200-plan-cache-v1" && j.contains("entries"),
            "plan cache file has an unknown format: " + path);
    return j;
}

bool lookup_cache(const std::string& path, const std::string& key, std::string& mapping) {
    if (path.empty()) return false;
    FileLock lock(path);
    const cubf::Json j = read_cache(path);
    const auto& e = j.at("entries");
    if (!e.contains(key)) return false;
    mapping = e.at(key).at("mapping").dump();
    return true;
}

void store_cache(const std::string& path, const std::string& key, const cubf::Mapping& m, double us) {
    if (path.empty()) return;
    FileLock lock(path);
    cubf::Json j = read_cache(path);
    j["entries"][key] = {{"mapping", m.to_json()}, {"measured_us", us}};
    const std::string tmp = path + ".tmp";
    {
        std::ofstream out(tmp, std::ios::trunc);
        require(static_cast<bool>(out), "cannot write plan cache " + path);
        out << j.dump(1) << "\n";
    }
    require(std::rename(tmp.c_str(), path.c_str()) == 0, "cannot publish plan cache " + path);
}

// ---- execution ----------------------------------------------------------------
// Cyclic NTT (cuntt::Plan semantics, include/cuntt/ntt.hpp:432; reference_ntt
// src/reference.cpp:584-630): input words reduced modulo q on load, the
// inverse always scaled by N^-1.
void launch_ntt(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out, cudaStream_t stream) {
    const auto& d = p.desc;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    const int l = p.req.log_n;
    const bool gs = p.req.ntt_gs;
    cubf::NttLaunch a;
    a.count = d.batch;
    a.tables = p.ntt_tables;
    a.polys = p.ntt_polys;
    a.in = in;
    a.out = out;
    a.reduce_input = true;
    if (m.passes.size() == 1) {
        a.final_pass = true;
        a.final_scale = inverse;
        check_cuda(cubf::launch_ntt({l, false, gs, p.req.ntt_lazy, p.req.ntt_word32}, a, stream), "NTT launch");
        return;
    }
    check_cuda(cubf::launch_ntt({l, !gs, gs, p.req.ntt_lazy, p.req.ntt_word32}, a, stream), "NTT pass 1 launch");
    a.in = out;
    a.in_is_out = true;
    a.reduce_input = false;
    a.final_pass = true;
    a.final_scale = inverse;
    check_cuda(cubf::launch_ntt({l, gs, gs, p.req.ntt_lazy, p.req.ntt_word32}, a, stream), "NTT pass 2 launch");
}

void launch_core(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out, void* ws,
                 cudaStream_t stream);

// The boundary around the core passes, on packed batches: a bit-reversed
// input is permuted into the output buffer first (the core then runs in place
// there), a bit-reversed output is permuted in place last.  `ws` is the
// core's workspace.
void launch_packed(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out, void* ws,
                   cudaStream_t stream) {
    const auto& d = p.desc;
    const int esz = static_cast<int>(cubf::storage_bytes(d.storage));
    const void* core_in = in;
    if (m.permute_input) {
        check_cuda(cubf::launch_bitrev(esz, p.req.log_n, in, out, d.batch, stream), "input permutation launch");
        core_in = out;
    }
    launch_core(p, m, core_in, out, ws, stream);
    if (m.permute_output)
        check_cuda(cubf::launch_bitrev(esz, p.req.log_n, out, out, d.batch, stream), "output permutation launch");
}

void launch_mapping(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out,
                    cudaStream_t stream);

// Row-major packed strides of the extents.
std::vector<std::size_t> packed_strides(const std::vector<std::size_t>& ext) {
    std::vector<std::size_t> st(ext.size(), 1);
    for (std::size_t k = ext.size(); k-- > 1;) st[k - 1] = st[k] * ext[k];
    return st;
}

// Rank two and three (reference composite execution, src/c_api.cpp:4533-4650:
// one axis plan per dimension, innermost first).
void launch_composite(const cubutterflyPlan& p, const void* in, void* out, cudaStream_t stream) {
    const auto& d = p.desc;
    unsigned char* ws = static_cast<unsigned char*>(p.workspace);
    if (p.direct) {
        const void* src = in;
        for (const auto& ax : p.axes) {
            auto& c = *ax.plan;
            c.workspace = ws + ax.ws_offset;
            launch_mapping(c, c.mapping, src, out, stream);
            src = out;
        }
        return;
    }
    if (p.flat) {
        auto& c = *p.axes.front().plan;
        c.workspace = ws + p.axes.front().ws_offset;
        launch_mapping(c, c.mapping, in, out, stream);
        return;
    }
    const int esz = static_cast<int>(cubf::storage_bytes(d.storage));
    const int dims = static_cast<int>(d.rank);
    const auto ps = packed_strides(d.extents);
    std::size_t volume = 1;
    for (auto e : d.extents) volume *= e;
    unsigned char* a = ws;
    unsigned char* b = ws + p.packed_bytes;
    check_cuda(cubf::launch_strided_copy_nd(esz, dims, d.extents.data(), in, d.input_strides.data(),
                                            d.input_batch_stride, a, ps.data(), volume, d.batch, stream),
               "composite gather launch");
    for (const auto& ax : p.axes) {
        auto& c = *ax.plan;
        c.workspace = ws + ax.ws_offset;
        if (ax.inner == 1) {
            launch_mapping(c, c.mapping, a, a, stream);
            continue;
        }
        // [outer][n][inner] <-> [outer][inner][n]
        const std::size_t ext[2] = {ax.n, ax.inner};
        const std::size_t by_axis[2] = {ax.inner, 1}, axis_last[2] = {1, ax.n};
        const std::size_t block = ax.n * ax.inner;
        check_cuda(cubf::launch_strided_copy_nd(esz, 2, ext, a, by_axis, block, b, axis_last, block, ax.outer, stream),
                   "composite transpose launch");
        launch_mapping(c, c.mapping, b, b, stream);
        check_cuda(cubf::launch_strided_copy_nd(esz, 2, ext, b, axis_last, block, a, by_axis, block, ax.outer, stream),
                   "composite transpose launch");
    }
    check_cuda(cubf::launch_strided_copy_nd(esz, dims, d.extents.data(), a, ps.data(), volume, out,
                                            d.output_strides.data(), d.output_batch_stride, d.batch, stream),
               "composite scatter launch");
}

// A strided or padded layout is gathered into the packed buffer at the start
// of the workspace, transformed there in place and scattered to the output
// layout (the reference's general strided boundary, src/general_kernels.cu).
// R2C: the real input read as N/2 complex values -> complex FFT into the
// workspace -> split into N/2 + 1 bins.  C2R: bins -> N/2 complex values in
// the workspace -> inverse complex FFT written as the real output.
void launch_real(const cubutterflyPlan& p, const void* in, void* out, cudaStream_t stream) {
    const auto& d = p.desc;
    const std::size_t half = d.extents[0] / 2;
    unsigned char* ws = static_cast<unsigned char*>(p.workspace);
    auto& c = *p.axes.front().plan;
    c.workspace = ws + p.axes.front().ws_offset;
    if (p.real_kind == CUBUTTERFLY_FFT_R2C) {
        launch_mapping(c, c.mapping, in, ws, stream);
        check_cuda(cubf::launch_r2c_post(ws, out, p.real_tw, half, d.batch, d.output_batch_stride,
                                         static_cast<float>(d.fft_output_scale), stream),
                   "R2C split launch");
        return;
    }
    double scale = 2.0 * d.fft_output_scale;  // the half-length inverse yields (N/2) z
    if (d.normalize_inverse) scale /= static_cast<double>(d.extents[0]);
    check_cuda(cubf::launch_c2r_pre(in, ws, p.real_tw, half, d.batch, d.input_batch_stride, static_cast<float>(scale),
                                    stream),
               "C2R merge launch");
    launch_mapping(c, c.mapping, ws, out, stream);
}

// Zero-extended embedding: rows of N logical elements in a packed buffer of
// P = next_pow2(N) per row.  Forward: zero the buffer, gather the N inputs,
// transform, write all P outputs.  Inverse: gather the P inputs, transform,
// write the first N outputs of each row.
void launch_embedded(const cubutterflyPlan& p, const void* in, void* out, cudaStream_t stream) {
    const auto& d = p.desc;
    const int esz = static_cast<int>(cubf::storage_bytes(d.storage));
    const std::size_t n = d.extents[0], pn = p.axes.front().n;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    unsigned char* ws = static_cast<unsigned char*>(p.workspace);
    auto& c = *p.axes.front().plan;
    c.workspace = ws + p.axes.front().ws_offset;
    if (!inverse) check_cuda(cudaMemsetAsync(ws, 0, d.batch * pn * esz, stream), "embedding zero fill");
    check_cuda(cubf::launch_strided_copy(esz, in, d.input_strides[0], d.input_batch_stride, ws, 1, pn,
                                         inverse ? pn : n, d.batch, stream),
               "embedding gather launch");
    launch_mapping(c, c.mapping, ws, ws, stream);
    check_cuda(cubf::launch_strided_copy(esz, ws, 1, pn, out, d.output_strides[0], d.output_batch_stride,
                                         inverse ? n : pn, d.batch, stream),
               "embedding scatter launch");
}

// Bluestein: pack (input x chirp, zero-padded) -> forward conv-point FFT ->
// x spectrum -> inverse conv-point FFT -> unpack (x chirp) into the output
// layout.  Input and output may alias: the pack completes before the unpack.
// Table layout of a Bluestein NTT plan: pack chirp, its Shoup quotients,
// unpack chirp (x N^-1 for an inverse), its quotients (n words each), then
// the convolution spectrum and its quotients (conv words each), every part
// 256-byte aligned.
struct NttChirpTables {
    std::size_t pack, pack_q, unpack, unpack_q, spectrum, spectrum_q, bytes;
    NttChirpTables(std::size_t n, std::size_t m) {
        const std::size_t a = align256(n * 8), b = align256(m * 8);
        pack = 0;
        pack_q = a;
        unpack = 2 * a;
        unpack_q = 3 * a;
        spectrum = 4 * a;
        spectrum_q = 4 * a + b;
        bytes = 4 * a + 2 * b;
    }
};

void launch_bluestein_ntt(const cubutterflyPlan& p, const void* in, void* out, cudaStream_t stream) {
    const auto& d = p.desc;
    const std::size_t n = d.extents[0], m = p.conv;
    const std::uint64_t q = d.modulus;
    const NttChirpTables t(n, m);
    unsigned char* ws = static_cast<unsigned char*>(p.workspace);
    const unsigned char* tb = static_cast<const unsigned char*>(p.bluestein_tables);
    const std::uint64_t unit_q = static_cast<std::uint64_t>((static_cast<unsigned __int128>(1) << 64) / q);
    check_cuda(cubf::launch_bluestein_ntt_pack(in, d.input_strides[0], d.input_batch_stride, ws, tb + t.pack,
                                               tb + t.pack_q, n, m, d.batch, q, unit_q, stream),
               "Bluestein NTT pack launch");
    for (std::size_t i = 0; i < 2; ++i) {
        auto& c = *p.axes[i].plan;
        c.workspace = ws + p.axes[i].ws_offset;
        launch_mapping(c, c.mapping, ws, ws, stream);
        if (i == 0)
            check_cuda(cubf::launch_bluestein_ntt_multiply(ws, tb + t.spectrum, tb + t.spectrum_q, m, d.batch, q,
                                                           stream),
                       "Bluestein NTT multiply launch");
    }
    check_cuda(cubf::launch_bluestein_ntt_unpack(ws, out, d.output_strides[0], d.output_batch_stride, tb + t.unpack,
                                                 tb + t.unpack_q, n, m, d.batch, q, stream),
               "Bluestein NTT unpack launch");
}

void launch_bluestein(const cubutterflyPlan& p, const void* in, void* out, cudaStream_t stream) {
    const auto& d = p.desc;
    if (d.op == CUBUTTERFLY_OPERATOR_NTT) {
        launch_bluestein_ntt(p, in, out, stream);
        return;
    }
    const bool f64 = d.storage == CUBUTTERFLY_DATA_COMPLEX_FP64;
    const std::size_t n = d.extents[0], m = p.conv, esz = cubf::storage_bytes(d.storage);
    unsigned char* ws = static_cast<unsigned char*>(p.workspace);
    const unsigned char* chirp = static_cast<const unsigned char*>(p.bluestein_tables);
    const unsigned char* spectrum = chirp + align256(n * esz);
    check_cuda(cubf::launch_bluestein_pack(f64, in, d.input_strides[0], d.input_batch_stride, ws, chirp, n, m,
                                           d.batch, stream),
               "Bluestein pack launch");
    for (std::size_t i = 0; i < 2; ++i) {
        auto& c = *p.axes[i].plan;
        c.workspace = ws + p.axes[i].ws_offset;
        launch_mapping(c, c.mapping, ws, ws, stream);
        if (i == 0)
            check_cuda(cubf::launch_bluestein_multiply(f64, ws, spectrum, m, d.batch, stream),
                       "Bluestein multiply launch");
    }
    check_cuda(cubf::launch_bluestein_unpack(f64, ws, out, d.output_strides[0], d.output_batch_stride, chirp, n, m,
                                             d.batch, stream),
               "Bluestein unpack launch");
}

void launch_real_nd(const cubutterflyPlan& p, const void* in, void* out, cudaStream_t stream) {
    unsigned char* ws = static_cast<unsigned char*>(p.workspace);
    auto& rows = *p.axes[0].plan;
    auto& axes = *p.axes[1].plan;
    rows.workspace = axes.workspace = ws + p.axes[0].ws_offset;
    if (p.desc.fft_type == CUBUTTERFLY_FFT_R2C) {
        launch_mapping(rows, rows.mapping, in, ws, stream);
        launch_mapping(axes, axes.mapping, ws, out, stream);
    } else {
        launch_mapping(axes, axes.mapping, in, ws, stream);
        launch_mapping(rows, rows.mapping, ws, out, stream);
    }
}

void launch_mapping(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out,
                    cudaStream_t stream) {
    if (p.real_nd) {
        launch_real_nd(p, in, out, stream);
        return;
    }
    if (p.bluestein) {
        launch_bluestein(p, in, out, stream);
        return;
    }
    if (p.embedded) {
        launch_embedded(p, in, out, stream);
        return;
    }
    if (p.real_kind != CUBUTTERFLY_FFT_C2C) {
        launch_real(p, in, out, stream);
        return;
    }
    if (!p.axes.empty()) {
        launch_composite(p, in, out, stream);
        return;
    }
    if (!m.staged) {
        launch_packed(p, m, in, out, p.workspace, stream);
        return;
    }
    const auto& d = p.desc;
    const int esz = static_cast<int>(cubf::storage_bytes(d.storage));
    const std::size_t n = d.extents[0];
    unsigned char* ws = static_cast<unsigned char*>(p.workspace);
    // Out of place, a packed side needs no copy: the core reads the packed
    // input or writes the packed output directly (every core also runs out of
    // place, and its workspace was sized for the in-place form).
    const bool packed_in = d.input_strides[0] == 1 && d.input_batch_stride == n;
    const bool packed_out = d.output_strides[0] == 1 && d.output_batch_stride == n;
    if (in != out && packed_in) {
        launch_packed(p, m, in, ws, ws + m.staged_bytes, stream);
    } else {
        check_cuda(cubf::launch_strided_copy(esz, in, d.input_strides[0], d.input_batch_stride, ws, 1, n, n, d.batch,
                                             stream),
                   "layout gather launch");
        if (in != out && packed_out) {
            launch_packed(p, m, ws, out, ws + m.staged_bytes, stream);
            return;
        }
        launch_packed(p, m, ws, ws, ws + m.staged_bytes, stream);
    }
    check_cuda(cubf::launch_strided_copy(esz, ws, 1, n, out, d.output_strides[0], d.output_batch_stride, n, d.batch,
                                         stream),
               "layout scatter launch");
}

// Transforms per L2 chunk of a chained bitwise plan (the whole batch for a
// single pass).
std::size_t chain_chunk(const cubutterflyPlan& p, const cubf::Mapping& m) {
    if (m.passes.size() < 2) return p.desc.batch;
    const std::size_t transform_bytes = p.desc.extents[0] * cubf::bw_type_bytes(p.req.bw_type);
    const std::size_t budget = std::max<std::size_t>(p.hw.l2_bytes * 2 / 5, 1);
    return std::max<std::size_t>(1, budget / transform_bytes);
}

// Bitwise tile passes: the first reads the input, the rest run in place.
// Multi-pass chains run chunk by chunk (every pass over a chunk of transforms
// sized to stay in L2, so the intermediate one pass writes is read by the
// next from L2 instead of HBM).  Two-pass chains over several chunks overlap
// pass A of chunk c+1 with pass B of chunk c, one launch per step
// (csrc/chain.cuh); other chains launch pass by pass, chunk by chunk.  All
// launches go to the caller's stream.
void enqueue_chain(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out,
                   cudaStream_t stream, double scale) {
    const auto& d = p.desc;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    const std::size_t n = d.extents[0];
    const std::size_t transform_bytes = n * cubf::bw_type_bytes(p.req.bw_type);
    const bool chained = m.passes.size() > 1;
    const std::size_t chunk = chain_chunk(p, m);
    if (m.passes.size() == 2 && d.batch > chunk &&
        cubf::bw_chain_available(p.req.bw_op, p.req.bw_type, m.passes[0].log_h, m.passes[1].log_h)) {
        cubf::BwChain c;
        c.n = n;
        c.batch = d.batch;
        c.chunk = chunk;
        c.log_h0 = m.passes[0].log_h;
        c.log_h1 = m.passes[1].log_h;
        c.inverse = inverse;
        c.scale = static_cast<float>(scale);
        check_cuda(cubf::launch_bw_chain(p.req.bw_op, p.req.bw_type, c, in, out, stream), "chain launch");
        return;
    }
    for (std::size_t b0 = 0; b0 < d.batch; b0 += chunk) {
        const std::size_t nb = std::min(chunk, d.batch - b0);
        const void* src = static_cast<const unsigned char*>(in) + b0 * transform_bytes;
        void* dst = static_cast<unsigned char*>(out) + b0 * transform_bytes;
        for (std::size_t i = 0; i < m.passes.size(); ++i) {
            const auto& ps = m.passes[i];
            const bool last = i + 1 == m.passes.size();
            const std::size_t inner = std::size_t{1} << ps.log_inner;
            const std::size_t outer = nb * (n >> (ps.log_inner + ps.log_h));
            const std::size_t inner_arg = ps.log_w == 0 ? 1 : inner;
            const std::size_t outer_arg = ps.log_w == 0 ? outer * inner : outer;
            const int mode = !chained ? 0 : (i == 0 ? 1 : (last ? 2 : 3));
            check_cuda(cubf::launch_bw({p.req.bw_op, p.req.bw_type, ps.log_h, ps.log_w}, src, dst, outer_arg,
                                       inner_arg, inverse, last ? static_cast<float>(scale) : 1.0f, mode, stream),
                       "tile pass launch");
            src = dst;
        }
    }
}

// L2-blocked FFT (mapping family "fft-l2-blocked", planner.hpp): each
// transform of N = V L points runs as V decimated transforms of L points,
// taken kFftBlockChunk at a time -- their first pass de-interleaves from the
// input into an L2-resident staging buffer, the rest run there, the last
// writes the block of results -- then one radix-V pass with Ns = L combines
// the blocks into the natural-order output.  Workspace: the blocks (N
// values), then one or two chunk staging buffers.
void launch_fft_blocked(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out, void* core_ws,
                        float scale, cudaStream_t stream) {
    const auto& d = p.desc;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    const int log_n = p.req.log_n;
    const int log_vb = m.passes.back().log_h;
    const int log_len = log_n - log_vb;
    const std::size_t n = std::size_t{1} << log_n, len = std::size_t{1} << log_len;
    const std::size_t chunk = cubf::kFftBlockChunk;
    auto* ws = static_cast<float2*>(core_ws);
    float2* blocks = ws;
    float2* stage[2] = {ws + n, ws + n + chunk * len};
    const cubf::FftOuterTables outer{p.outer_lo, p.outer_hi, p.outer_split};
    const std::size_t nsub = m.passes.size() - 1;
    for (std::size_t b = 0; b < d.batch; ++b) {
        const float2* src = static_cast<const float2*>(in) + b * n;
        float2* dst = static_cast<float2*>(out) + b * n;
        for (std::size_t m0 = 0; m0 < (std::size_t{1} << log_vb); m0 += chunk) {
            float2* target = blocks + m0 * len;
            const void* cur = nsub == 1 ? static_cast<void*>(target) : static_cast<void*>(stage[0]);
            check_cuda(cubf::launch_fft_deinterleave_pass(m.passes[0].log_h, src, const_cast<void*>(cur), log_len, log_vb,
                                                          m0, p.twiddles, inverse, stream),
                       "FFT de-interleave pass launch");
            for (std::size_t i = 1; i < nsub; ++i) {
                const bool last = i + 1 == nsub;
                void* next = last ? static_cast<void*>(target) : static_cast<void*>(stage[i & 1]);
                check_cuda(cubf::launch_fft_global_pass(m.passes[i].log_h, cur, next, log_len, m.passes[i].log_inner,
                                                        chunk, p.twiddles, outer, false, false, 1.0f, stream, 0, log_vb),
                           "FFT chunk pass launch");
                cur = next;
            }
        }
        check_cuda(cubf::launch_fft_global_pass(log_vb, blocks, dst, log_n, log_len, 1, p.twiddles, outer, false,
                                                inverse, scale, stream, 0, 0, true),
                   "FFT combining pass launch");
    }
}

// L2-chained FFT (mapping family "fft-l2-chain", planner.hpp): passes 0+1
// and then 2+3 of the Stockham plan, each pair chunk by chunk.  A chunk of a
// pair is a set of "keys" -- the column bits the two passes share -- chosen
// so that the second pass of the chunk reads exactly what the first one wrote:
// pair one (Ns = 1) keys on the columns' high n - b0 - b1 bits, pair two on
// the low b0 + b1 bits.  The first pass writes the workspace with an L2
// evict-last policy, the second reads it back from L2 and discards its lines,
// so each pair reads and writes HBM once.  Tiles of 32 columns; a chunk holds
// 2^22 values.  A pair of C chunks runs as C + 1 chain steps
// (launch_fft_chain_step, csrc/fft_chain.cu): step k runs the pair's first
// pass over chunk k beside its second pass over chunk k-1, each step a
// programmatic dependent launch of the one before.
void launch_fft_chain(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out, void* core_ws,
                      float scale, cudaStream_t stream) {
    const auto& d = p.desc;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    const int ln = p.req.log_n;
    const std::size_t n = std::size_t{1} << ln;
    const int b0 = m.passes[0].log_h, b1 = m.passes[1].log_h, b2 = m.passes[2].log_h, b3 = m.passes[3].log_h;
    const int tl = cubf::kFftChainColumnsLog;
    const cubf::FftOuterTables outer{p.outer_lo, p.outer_hi, p.outer_split};
    auto role = [&](int i, const void* src, void* dst, const cubf::FftChunk& c) {
        const bool last = i == 3;
        return cubf::FftChainRole{src, dst, m.passes[i].log_h, m.passes[i].log_inner, inverse && i == 0,
                                  inverse && last, last ? scale : 1.0f, c, false};
    };
    const cubf::FftChunk none{0, 0, 0, 0, false, false};
    // one pair over `chunks` chunks: chunk c's A and B roles from make(c)
    auto pair = [&](std::uint32_t chunks, auto make_a, auto make_b) {
        for (std::uint32_t k = 0; k <= chunks; ++k) {
            const cubf::FftChainRole a = k < chunks ? make_a(k) : make_a(0);
            const cubf::FftChainRole b = k > 0 ? make_b(k - 1) : make_b(0);
            cubf::FftChainRole ra = a, rb = b;
            if (k == chunks) ra.chunk = none;
            if (k == 0) rb.chunk = none;
            ra.wait = k == 0;  // the pair's first step reads what came before it
            check_cuda(cubf::launch_fft_chain_step(ra, rb, ln, p.twiddles, outer, stream), "FFT chain step launch");
        }
    };
    for (std::size_t b = 0; b < d.batch; ++b) {
        const float2* src = static_cast<const float2*>(in) + b * n;
        float2* dst = static_cast<float2*>(out) + b * n;
        // the intermediate starts on a 128-byte line: the second pass of a
        // pair drops whole lines of it from L2
        float2* ws = reinterpret_cast<float2*>((reinterpret_cast<std::uintptr_t>(core_ws) + 127) &
                                               ~std::uintptr_t{127});
        // pair one: key h < 2^(n - b0 - b1); pass 0 columns r 2^(n-b0-b1) + h (r < 2^b1),
        // pass 1 columns h 2^b0 + k (k < 2^b0)
        {
            const int kb = ln - b0 - b1;
            const int fl = std::min(kb, cubf::kFftChainChunkLog - b0 - b1);
            pair(
                1u << (kb - fl),
                [&](std::uint32_t c) {
                    const std::uint32_t h0 = c << fl;
                    return role(0, src, ws, {h0, 1u << (fl - tl), 1u << kb, 1u << b1, false, true});
                },
                [&](std::uint32_t c) {
                    const std::uint32_t h0 = c << fl;
                    return role(1, ws, dst, {h0 << b0, 1u << (fl + b0 - tl), 0, 1, true, false});
                });
        }
        // pair two: key l < 2^(b0 + b1); pass 2 columns r 2^s + l (r < 2^b3),
        // pass 3 columns k 2^s + l (k < 2^b2), s = b0 + b1
        {
            const int s = b0 + b1;
            const int fl = std::min(s, cubf::kFftChainChunkLog - b2 - b3);
            pair(
                1u << (s - fl),
                [&](std::uint32_t c) {
                    return role(2, dst, ws, {c << fl, 1u << (fl - tl), 1u << s, 1u << b3, false, true});
                },
                [&](std::uint32_t c) {
                    return role(3, ws, dst, {c << fl, 1u << (fl - tl), 1u << s, 1u << b2, true, false});
                });
        }
    }
}

void launch_core(const cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out, void* core_ws,
                 cudaStream_t stream) {
    const auto& d = p.desc;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    const std::size_t n = d.extents[0];
    if (d.op == CUBUTTERFLY_OPERATOR_NTT) {
        launch_ntt(p, m, in, out, stream);
        return;
    }
    // Caller buffers that are element-aligned but not 16-byte aligned (the
    // reference accepts any element pointer): complex FFTs and NTTs move whole
    // elements already; FWHT and zeta take their element-granular kernels
    // (csrc/unaligned.cu); the stage-storage kernels below have none.
    const bool vec16 = ((reinterpret_cast<std::uintptr_t>(in) | reinterpret_cast<std::uintptr_t>(out)) & 15) == 0;
    if (!vec16 && (p.req.fwht_native || d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2))
        throw cubf::Unsupported(std::string(p.req.fwht_native ? "stage-storage FWHT" : "structured 2x2") +
                                " plans need 16-byte aligned input and output buffers");
    if (p.req.fwht_native) {
        check_cuda(cubf::launch_fwht_native(d.storage == CUBUTTERFLY_DATA_BF16, p.req.log_n, in, out, d.batch,
                                            inverse && d.normalize_inverse, stream),
                   "native FWHT launch");
        return;
    }
    if (d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2) {
        check_cuda(cubf::launch_structured(static_cast<int>(cubf::storage_bytes(d.storage)), p.req.log_n, in, out,
                                           d.batch, p.structured, stream),
                   "structured launch");
        return;
    }
    if (p.req.fft64) {
        const double scale = (inverse && d.normalize_inverse) ? 1.0 / static_cast<double>(n) : 1.0;
        check_cuda(cubf::launch_fft64(p.req.log_n, in, out, d.batch, p.twiddles, scale, stream), "FP64 FFT launch");
        return;
    }
    if (d.op == CUBUTTERFLY_OPERATOR_FFT) {
        const float scale = (inverse && d.normalize_inverse) ? 1.0f / static_cast<float>(n) : 1.0f;
        if (m.passes.front().kind == cubf::PassKind::FftLocal) {
            check_cuda(cubf::launch_fft_local(p.req.log_n, in, out, d.batch, p.twiddles, inverse, scale, stream),
                       "FFT launch");
            return;
        }
        if (m.family == "fft-l2-blocked") {
            launch_fft_blocked(p, m, in, out, core_ws, scale, stream);
            return;
        }
        if (m.family == "fft-l2-chain") {
            launch_fft_chain(p, m, in, out, core_ws, scale, stream);
            return;
        }
        // Global passes ping-pong between the output and the workspace so the
        // last pass lands in `out`; an in-place plan with an odd pass count
        // starts in a second workspace half.
        const std::size_t np = m.passes.size();
        const std::size_t bytes = d.batch * n * 8 * p.groups;
        unsigned char* ws = static_cast<unsigned char*>(core_ws);
        const bool in_place = in == out;
        const cubf::FftOuterTables outer{p.outer_lo, p.outer_hi, p.outer_split};
        const void* src = in;
        for (std::size_t i = 0; i < np; ++i) {
            void* dst;
            if ((np - 1 - i) % 2 == 0)
                dst = (in_place && i == 0 && np > 1) ? ws + bytes : out;
            else
                dst = ws;
            const bool last = i + 1 == np;
            const auto& ps = m.passes[i];
            // interleaved batches run as one array of N * batch values
            const int lv = p.req.log_v;
            check_cuda(cubf::launch_fft_global_pass(ps.log_h, src, dst, p.req.log_n + lv, ps.log_inner + lv,
                                                    lv ? p.groups : d.batch, p.twiddles, outer, inverse && i == 0,
                                                    inverse && last, last ? scale : 1.0f, stream, lv),
                       "FFT pass launch");
            src = dst;
        }
        return;
    }
    double scale = 1.0;
    if (d.op == CUBUTTERFLY_OPERATOR_FWHT) {
        scale = d.output_scale;
        if (inverse && d.normalize_inverse) scale /= static_cast<double>(n);
    }
    if (!vec16) {
        if (d.op == CUBUTTERFLY_OPERATOR_FWHT)
            check_cuda(cubf::launch_fwht_unaligned(p.req.bw_type, p.req.log_n, in, out, d.batch,
                                                   static_cast<float>(scale), stream),
                       "element-granular FWHT launch");
        else
            check_cuda(cubf::launch_zeta_unaligned(p.req.bw_type, p.req.bw_op == cubf::BwOp::ZetaSuperset,
                                                   p.req.log_n, in, out, d.batch, inverse, stream),
                       "element-granular zeta launch");
        return;
    }
    if (m.passes.front().kind == cubf::PassKind::FwhtTensor) {
        check_cuda(cubf::launch_fwht_tc(in, out, d.batch, static_cast<float>(scale), p.status_dev, stream),
                   "tensor FWHT launch");
        return;
    }
    enqueue_chain(p, m, in, out, stream, scale);
}


double time_mapping(cubutterflyPlan& p, const cubf::Mapping& m, const void* in, void* out, cudaStream_t stream,
                    int reps) {
    cudaEvent_t a, b;
    check_cuda(cudaEventCreate(&a), "event");
    check_cuda(cudaEventCreate(&b), "event");
    launch_mapping(p, m, in, out, stream);  // warm-up
    check_cuda(cudaEventRecord(a, stream), "event record");
    for (int i = 0; i < reps; ++i) launch_mapping(p, m, in, out, stream);
    check_cuda(cudaEventRecord(b, stream), "event record");
    check_cuda(cudaEventSynchronize(b), "event sync");
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return 1000.0 * ms / reps;
}

// Root table of the cyclic NTT with the reference's root convention
// (find_primitive_power_of_two_root(log N, q); the inverse uses its modular
// inverse, src/reference.cpp:597-600), followed by q, N^-1, its Shoup
// quotient, floor(2^64 / q) and the per-transform offsets.
void build_ntt_tables(cubutterflyPlan& p) {
    namespace ma = cubf::modarith;
    const auto& d = p.desc;
    const int l = p.req.log_n;
    const std::uint64_t q = d.modulus;
    // validate_config of the reference's NTT plans (src/ntt.cu): a prime
    // modulus below 2^63 with 2^log_n | q - 1 (the root search checks the rest)
    require(q < (std::uint64_t{1} << 63), "NTT modulus must be below 2^63");
    const std::size_t n = std::size_t{1} << l;
    std::uint64_t root = ma::primitive_root_of_two_power(static_cast<unsigned>(l), q);
    if (d.direction == CUBUTTERFLY_DIRECTION_INVERSE) root = ma::powmod(root, q - 2, q);
    std::vector<std::uint64_t> words(2 * n + 4), roots(n), quots(n);
    ma::cyclic_root_table(l, q, root, roots.data(), quots.data());
    for (std::size_t k = 0; k < n; ++k) {  // {root, quotient} pairs
        words[2 * k] = roots[k];
        words[2 * k + 1] = quots[k];
    }
    const std::uint64_t ni = ma::powmod(static_cast<std::uint64_t>(n), q - 2, q);
    words[2 * n + 0] = q;
    words[2 * n + 1] = ni;
    words[2 * n + 2] = ma::shoup(ni, q);
    words[2 * n + 3] = static_cast<std::uint64_t>((static_cast<unsigned __int128>(1) << 64) / q);
    std::vector<cubf::NttPolyDesc> polys;
    if (!cubf::ntt_single_available(l)) {
        polys.resize(d.batch);
        for (std::size_t b = 0; b < d.batch; ++b) polys[b] = {b * n, b * n, 0, 0};
    }
    const std::size_t table_bytes = words.size() * 8, poly_bytes = polys.size() * sizeof(cubf::NttPolyDesc);
    check_cuda(cudaMalloc(&p.ntt_block, table_bytes + poly_bytes), "NTT table allocation");
    check_cuda(cudaMemcpy(p.ntt_block, words.data(), table_bytes, cudaMemcpyHostToDevice), "NTT table upload");
    auto* base = static_cast<std::uint64_t*>(p.ntt_block);
    if (poly_bytes) {
        check_cuda(cudaMemcpy(base + words.size(), polys.data(), poly_bytes, cudaMemcpyHostToDevice),
                   "NTT offsets upload");
        p.ntt_polys = reinterpret_cast<const cubf::NttPolyDesc*>(base + words.size());
    }
    p.ntt_tables = {base, base + 2 * n, base + 2 * n + 1, base + 2 * n + 2, base + 2 * n + 3};
}

// Per-stage matrices of a structured 2x2 plan: one shared matrix or one per
// stage; an inverse plan uses each matrix's inverse, computed in double as the
// reference does (src/butterfly_reference.cpp:560-570).
void build_structured(cubutterflyPlan& p) {
    const auto& ms = p.desc.stage_matrices.at(0);
    const int l = p.req.log_n;
    require(ms.size() == 1 || ms.size() == static_cast<std::size_t>(l),
            "structured 2x2 requires one matrix or one matrix per stage");
    require(l <= cubf::kStructuredMaxLog, "structured 2x2 length is limited to 2^30");
    for (int s = 0; s < l; ++s) {
        const auto& m = ms.size() == 1 ? ms[0] : ms[s];
        double a = m.m00, b = m.m01, c = m.m10, e = m.m11;
        if (p.desc.direction == CUBUTTERFLY_DIRECTION_INVERSE) {
            const double det = m.m00 * m.m11 - m.m01 * m.m10;
            require(std::isfinite(det) && det != 0.0, "structured 2x2 inverse requires nonsingular matrices");
            a = m.m11 / det;
            b = -m.m01 / det;
            c = -m.m10 / det;
            e = m.m00 / det;
        }
        const double v[4] = {a, b, c, e};
        for (int k = 0; k < 4; ++k) {
            p.structured.f64[s][k] = v[k];
            p.structured.f32[s][k] = static_cast<float>(v[k]);
        }
    }
}

void build_tables(cubutterflyPlan& p) {
    if (p.desc.op == CUBUTTERFLY_OPERATOR_NTT) {
        build_ntt_tables(p);
        return;
    }
    if (p.desc.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2) {
        build_structured(p);
        return;
    }
    if (p.desc.op != CUBUTTERFLY_OPERATOR_FFT) return;
    constexpr double kPi = 3.141592653589793238462643383279502884;
    if (p.req.fft64) {
        // W_N^k, k < N/2, with the reference's angle rounding: ((+-pi) * o) / half
        // for stage half and offset o equals ((+-pi) * 2k) / N exactly (powers of two)
        const std::size_t n = p.desc.extents[0];
        const double sign = p.desc.direction == CUBUTTERFLY_DIRECTION_INVERSE ? 1.0 : -1.0;
        std::vector<double> tw(n);  // n / 2 complex entries
        for (std::size_t k = 0; k < n / 2; ++k) {
            const double angle = sign * kPi * static_cast<double>(2 * k) / static_cast<double>(n);
            tw[2 * k] = std::cos(angle);
            tw[2 * k + 1] = std::sin(angle);
        }
        check_cuda(cudaMalloc(&p.twiddles, std::max<std::size_t>(tw.size(), 2) * sizeof(double)),
                   "twiddle table allocation");
        check_cuda(cudaMemcpy(p.twiddles, tw.data(), tw.size() * sizeof(double), cudaMemcpyHostToDevice),
                   "twiddle table upload");
        return;
    }
    // every candidate of a request is global or every one is local
    const bool global = p.req.log_n > cubf::kFftLocalMaxLog || p.req.log_v > 0;
    if (global) {
        // exp(-2 pi i k / N) for the outer twiddles, in double: lo k < 2^split, hi k << split
        const int l = p.req.log_n;
        const int split = (l + 1) / 2;
        const std::size_t nlo = std::size_t{1} << split, nhi = std::size_t{1} << (l - split);
        const double n_d = std::ldexp(1.0, l);
        std::vector<double> lo(2 * nlo), hi(2 * nhi);
        for (std::size_t k = 0; k < nlo; ++k) {
            const double a = -2.0 * kPi * static_cast<double>(k) / n_d;
            lo[2 * k] = std::cos(a);
            lo[2 * k + 1] = std::sin(a);
        }
        for (std::size_t k = 0; k < nhi; ++k) {
            const double a = -2.0 * kPi * static_cast<double>(k << split) / n_d;
            hi[2 * k] = std::cos(a);
            hi[2 * k + 1] = std::sin(a);
        }
        check_cuda(cudaMalloc(&p.outer_lo, lo.size() * 8), "twiddle table allocation");
        check_cuda(cudaMalloc(&p.outer_hi, hi.size() * 8), "twiddle table allocation");
        check_cuda(cudaMemcpy(p.outer_lo, lo.data(), lo.size() * 8, cudaMemcpyHostToDevice), "twiddle upload");
        check_cuda(cudaMemcpy(p.outer_hi, hi.data(), hi.size() * 8, cudaMemcpyHostToDevice), "twiddle upload");
        p.outer_split = split;
    }
    const std::vector<float> tw = cubf::fft_local_twiddles(global ? 10 : p.req.log_n);
    check_cuda(cudaMalloc(&p.twiddles, tw.size() * sizeof(float)), "twiddle table allocation");
    check_cuda(cudaMemcpy(p.twiddles, tw.data(), tw.size() * sizeof(float), cudaMemcpyHostToDevice),
               "twiddle table upload");
}

cubf::PlanRequest make_request(const cubf::Descriptor& d) {
    cubf::PlanRequest r;
    r.d = d;
    r.log_n = static_cast<int>(cubf::log2_exact(d.extents[0]));
    if (d.op == CUBUTTERFLY_OPERATOR_FFT && d.storage == CUBUTTERFLY_DATA_COMPLEX_FP32 && cubf::interleaved_batches(d))
        r.log_v = static_cast<int>(cubf::log2_exact(d.batch));
    r.fft64 = d.op == CUBUTTERFLY_OPERATOR_FFT && d.storage == CUBUTTERFLY_DATA_COMPLEX_FP64;
    switch (d.op) {
        case CUBUTTERFLY_OPERATOR_FWHT:
            r.bw_op = cubf::BwOp::Fwht;
            r.bw_type = d.storage == CUBUTTERFLY_DATA_BF16   ? cubf::BwType::BF16
                        : d.storage == CUBUTTERFLY_DATA_FP16 ? cubf::BwType::F16
                                                             : cubf::BwType::F32;
            break;
        case CUBUTTERFLY_OPERATOR_SUBSET_ZETA:
        case CUBUTTERFLY_OPERATOR_SUPERSET_ZETA:
            r.bw_op = d.op == CUBUTTERFLY_OPERATOR_SUBSET_ZETA ? cubf::BwOp::ZetaSubset : cubf::BwOp::ZetaSuperset;
            r.bw_type = d.storage == CUBUTTERFLY_DATA_UINT64 ? cubf::BwType::U64 : cubf::BwType::U32;
            break;
        default:
            break;
    }
    cubf::resolve_orders(r);
    r.staged = !cubf::packed_layout(d) && r.log_v == 0;
    r.fwht_native = d.op == CUBUTTERFLY_OPERATOR_FWHT &&
                    (d.storage == CUBUTTERFLY_DATA_BF16 || d.storage == CUBUTTERFLY_DATA_FP16) &&
                    d.compute == CUBUTTERFLY_COMPUTE_NATIVE;
    return r;
}

// An algorithm name of the reference's own catalogue ("ntt-shared-iterative",
// "bluestein-cufft-power2-core", ...): lower-case words joined by '-', no
// pass list, bracketed family or JSON.  Those name kernels of the reference
// build; a plan that asks for one here runs this build's best mapping.
bool reference_algorithm_name(const std::string& s) {
    if (s.empty() || s.front() < 'a' || s.front() > 'z' || s.find('-') == std::string::npos) return false;
    return std::all_of(s.begin(), s.end(), [](char c) { return (c >= 'a' && c <= 'z') || (c >= '0' && c <= '9') || c == '-'; });
}

void select_mapping(cubutterflyHandle* h, cubutterflyPlan& p) {
    const auto& d = p.desc;
    if (d.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT && reference_algorithm_name(d.explicit_algorithm)) {
        p.mapping = cubf::enumerate_mappings(p.req, p.hw).front();
        p.source = CUBUTTERFLY_SELECTION_STATIC_MODEL;
        p.reason = "explicit reference algorithm '" + d.explicit_algorithm +
                   "' names a kernel family of the reference build; the static model's " + p.mapping.name() +
                   " executes it here";
        return;
    }
    if (d.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) {
        p.mapping = cubf::parse_explicit_mapping(p.req, p.hw, d.explicit_algorithm);
        p.source = CUBUTTERFLY_SELECTION_EXPLICIT;
        p.reason = "explicit mapping " + p.mapping.name();
        return;
    }
    auto ranked = cubf::enumerate_mappings(p.req, p.hw);
    if (d.algorithm_policy == CUBUTTERFLY_ALGORITHM_DEFAULT) {
        std::string cached;
        if (h && lookup_cache(h->cache_path, workload_key(p), cached)) {
            p.mapping = cubf::parse_explicit_mapping(p.req, p.hw, cached);
            p.source = CUBUTTERFLY_SELECTION_USER_CACHE;
            p.reason = "plan cache hit " + p.mapping.name();
            return;
        }
        p.mapping = ranked.front();
        p.source = CUBUTTERFLY_SELECTION_STATIC_MODEL;
        std::ostringstream o;
        o << "static roofline model over " << ranked.size() << " partitions on " << p.hw.name << " ("
          << p.hw.source << "): " << p.mapping.name() << " predicted " << p.mapping.predicted_us << " us";
        p.reason = o.str();
        return;
    }
    // MEASURE: time up to four finalists on private device buffers.
    const std::size_t finalists = std::min<std::size_t>(4, ranked.size());
    const std::size_t bytes = std::max(p.input_bytes, p.output_bytes);
    void* a = nullptr;
    void* b = nullptr;
    check_cuda(cudaMalloc(&a, bytes), "measure buffer");
    std::unique_ptr<void, void (*)(void*)> ga(a, [](void* x) { cudaFree(x); });
    check_cuda(cudaMalloc(&b, bytes), "measure buffer");
    std::unique_ptr<void, void (*)(void*)> gb(b, [](void* x) { cudaFree(x); });
    check_cuda(cudaMemset(a, 0, bytes), "measure buffer init");
    // a private workspace for the finalists (the caller's is set after planning)
    std::size_t ws_bytes = 0;
    for (std::size_t i = 0; i < finalists; ++i) ws_bytes = std::max(ws_bytes, ranked[i].workspace_bytes);
    void* ws = nullptr;
    if (ws_bytes) check_cuda(cudaMalloc(&ws, ws_bytes), "measure workspace");
    std::unique_ptr<void, void (*)(void*)> gws(ws, [](void* x) {
        if (x) cudaFree(x);
    });
    p.workspace = ws;
    cudaStream_t s = h ? h->stream : nullptr;
    double best = 1e300;
    std::size_t best_i = 0;
    for (std::size_t i = 0; i < finalists; ++i) {
        const double us = time_mapping(p, ranked[i], a, b, s, 5);
        if (us < best) {
            best = us;
            best_i = i;
        }
    }
    check_cuda(cudaStreamSynchronize(s), "measure drain");
    p.workspace = nullptr;
    p.mapping = ranked[best_i];
    p.source = CUBUTTERFLY_SELECTION_RUNTIME_MEASURED;
    std::ostringstream o;
    o << "measured " << finalists << " finalists: " << p.mapping.name() << " " << best << " us";
    p.reason = o.str();
    if (h) store_cache(h->cache_path, workload_key(p), p.mapping, best);
}

}  // namespace

namespace cubf {
}  // namespace cubf

namespace {

// Bytes spanned by a layout: its largest element offset + 1.
std::size_t layout_span(const cubf::Descriptor& d, const std::vector<std::size_t>& ext,
                        const std::vector<std::size_t>& str, std::size_t bs) {
    std::size_t last = (d.batch - 1) * bs;
    for (std::size_t a = 0; a < ext.size(); ++a) last += (ext[a] - 1) * str[a];
    return (last + 1) * cubf::storage_bytes(d.storage);
}

std::unique_ptr<cubutterflyPlan> create_rank1(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    auto p = std::make_unique<cubutterflyPlan>();
    p->desc = d;
    p->input_bytes = layout_span(d, cubf::input_extents(d), d.input_strides, d.input_batch_stride);
    p->output_bytes = layout_span(d, cubf::output_extents(d), d.output_strides, d.output_batch_stride);
    p->req = make_request(d);
    p->hw = cubf::resolve_profile();
    check_cuda(cudaGetDevice(&p->device), "current device");
    if (d.op == CUBUTTERFLY_OPERATOR_FWHT && cubf::fwht_tc_available(p->req.log_n, p->req.bw_type)) {
        void* host = nullptr;
        check_cuda(cudaHostAlloc(&host, sizeof(unsigned int), cudaHostAllocMapped), "device status word");
        p->status_host = static_cast<unsigned int*>(host);
        *p->status_host = 0;
        void* dev = nullptr;
        check_cuda(cudaHostGetDevicePointer(&dev, host, 0), "device status word address");
        p->status_dev = static_cast<unsigned int*>(dev);
    }
    build_tables(*p);  // before selection: MEASURE executes the candidates
    select_mapping(handle, *p);
    return p;
}

// A complex FFT whose length is not a power of two (standard length mode).
bool arbitrary_fft(const cubf::Descriptor& d) {
    return d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type == CUBUTTERFLY_FFT_C2C &&
           d.length_mode == CUBUTTERFLY_LENGTH_STANDARD &&
           std::any_of(d.extents.begin(), d.extents.end(), [](std::size_t e) { return !cubf::is_pow2(e); });
}

// The least power of two >= 2n - 1.
std::size_t bluestein_length(std::size_t n) {
    std::size_t m = 1;
    while (m < 2 * n - 1) m <<= 1;
    return m;
}

// The forward power-of-two child of a rank-one Bluestein plan: the packed
// batch of convolution-length transforms, in place on the work buffer.
cubf::Descriptor bluestein_child(const cubf::Descriptor& d) {
    cubf::Descriptor c = d;
    const std::size_t m = bluestein_length(d.extents[0]);
    c.extents = {m};
    c.input_strides = c.output_strides = {1};
    c.input_batch_stride = c.output_batch_stride = m;
    c.input_orders = c.output_orders = {CUBUTTERFLY_ORDER_NATURAL};
    c.placement = CUBUTTERFLY_PLACEMENT_IN_PLACE;
    c.direction = CUBUTTERFLY_DIRECTION_FORWARD;
    c.normalize_inverse = false;
    if (c.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) {
        c.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
        c.explicit_algorithm.clear();
    }
    return cubf::normalize(c);
}

struct DeviceTemp {
    void* ptr = nullptr;
    explicit DeviceTemp(std::size_t bytes) { check_cuda(cudaMalloc(&ptr, bytes), "Bluestein set-up allocation"); }
    ~DeviceTemp() {
        if (ptr) cudaFree(ptr);
    }
    DeviceTemp(const DeviceTemp&) = delete;
    DeviceTemp& operator=(const DeviceTemp&) = delete;
};

// Rank-one arbitrary-length complex FFT (reference src/bluestein_fft.cu with
// its own power-of-two core): conv = the least power of two >= 2n - 1; the
// convolution spectrum is computed once here in fp64 (taps on the device,
// an fp64 conv-point FFT plan of this library, scaled by 1 / conv and, for a
// normalised inverse, 1 / n) and rounded once to the storage precision.
std::unique_ptr<cubutterflyPlan> create_bluestein(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    auto p = std::make_unique<cubutterflyPlan>();
    p->desc = d;
    p->bluestein = true;
    p->input_bytes = layout_span(d, cubf::input_extents(d), d.input_strides, d.input_batch_stride);
    p->output_bytes = layout_span(d, cubf::output_extents(d), d.output_strides, d.output_batch_stride);
    p->hw = cubf::resolve_profile();
    check_cuda(cudaGetDevice(&p->device), "current device");
    const std::size_t n = d.extents[0];
    const std::size_t m = bluestein_length(n);
    p->conv = m;
    p->physical = {m};
    const bool f64 = d.storage == CUBUTTERFLY_DATA_COMPLEX_FP64;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    const std::size_t esz = cubf::storage_bytes(d.storage);
    const std::size_t work_bytes = align256(m * d.batch * esz);
    cubf::Descriptor c = bluestein_child(d);
    std::size_t child_ws = 0;
    for (auto dir : {CUBUTTERFLY_DIRECTION_FORWARD, CUBUTTERFLY_DIRECTION_INVERSE}) {
        c.direction = dir;
        cubutterflyPlan::Axis ax;
        ax.plan = create_rank1(handle, cubf::normalize(c));
        ax.n = m;
        ax.outer = d.batch;
        ax.inner = 1;
        ax.ws_offset = work_bytes;
        child_ws = std::max(child_ws, ax.plan->mapping.workspace_bytes);
        p->axes.push_back(std::move(ax));
    }
    p->mapping.family = "bluestein";
    p->mapping.label = "bluestein[" + std::to_string(m) + ":" + p->axes[0].plan->mapping.name() + "]";
    p->mapping.workspace_bytes = work_bytes + align256(child_ws);
    p->source = p->axes[0].plan->source;
    p->reason = "non-power-of-two FFT of " + std::to_string(n) + " points as a " + std::to_string(m) +
                "-point cyclic convolution (Bluestein): " + p->axes[0].plan->reason;

    // per-plan tables
    check_cuda(cudaMalloc(&p->bluestein_tables, align256(n * esz) + m * esz), "Bluestein table allocation");
    unsigned char* chirp = static_cast<unsigned char*>(p->bluestein_tables);
    cubf::Descriptor k = c;
    k.storage = CUBUTTERFLY_DATA_COMPLEX_FP64;
    k.compute = CUBUTTERFLY_COMPUTE_FP64;
    k.batch = 1;
    k.direction = CUBUTTERFLY_DIRECTION_FORWARD;
    k.placement = CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE;
    k.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
    auto kp = create_rank1(handle, cubf::normalize(k));
    DeviceTemp temp(2 * align256(m * 16) + align256(kp->mapping.workspace_bytes) + 256);
    unsigned char* taps = static_cast<unsigned char*>(temp.ptr);
    unsigned char* taps_spectrum = taps + align256(m * 16);
    kp->workspace = taps_spectrum + align256(m * 16);
    cudaStream_t s = nullptr;
    check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "Bluestein set-up stream");
    try {
        check_cuda(cubf::launch_bluestein_tables(f64, n, m, inverse, chirp, taps, s), "Bluestein table launch");
        launch_mapping(*kp, kp->mapping, taps, taps_spectrum, s);
        const double scale = (1.0 / static_cast<double>(m)) *
                             (inverse && d.normalize_inverse ? 1.0 / static_cast<double>(n) : 1.0);
        check_cuda(cubf::launch_bluestein_spectrum(f64, taps_spectrum, chirp + align256(n * esz), m, scale, s),
                   "Bluestein spectrum launch");
        check_cuda(cudaStreamSynchronize(s), "Bluestein set-up");
    } catch (...) {
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
        throw;
    }
    cudaStreamDestroy(s);
    return p;
}

// A u64 NTT whose length is not a power of two.
bool arbitrary_ntt(const cubf::Descriptor& d) {
    return d.op == CUBUTTERFLY_OPERATOR_NTT && d.length_mode == CUBUTTERFLY_LENGTH_STANDARD &&
           std::any_of(d.extents.begin(), d.extents.end(), [](std::size_t e) { return !cubf::is_pow2(e); });
}

// Rank-one arbitrary-length NTT over u64 words (reference
// src/bluestein_ntt.cu): psi = the reference's primitive 2n-th root (its
// inverse for an inverse plan), chirps psi^(j^2 mod 2n), the wrapped inverse
// chirps as convolution taps, the conv-point cyclic convolution on this
// library's power-of-two NTT plans.  X[k] = sum_j x[j] (psi^2)^(jk) exactly,
// times n^-1 for an inverse.  Needs a prime q < 2^63 with 2n | q - 1 and
// conv | q - 1 (INVALID_VALUE otherwise, as the reference).
std::unique_ptr<cubutterflyPlan> create_bluestein_ntt(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    namespace ma = cubf::modarith;
    auto p = std::make_unique<cubutterflyPlan>();
    p->desc = d;
    p->bluestein = true;
    p->input_bytes = layout_span(d, cubf::input_extents(d), d.input_strides, d.input_batch_stride);
    p->output_bytes = layout_span(d, cubf::output_extents(d), d.output_strides, d.output_batch_stride);
    p->hw = cubf::resolve_profile();
    check_cuda(cudaGetDevice(&p->device), "current device");
    const std::size_t n = d.extents[0];
    const std::size_t m = bluestein_length(n);
    const std::uint64_t q = d.modulus;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    p->conv = m;
    p->physical = {m};
    require(q < (std::uint64_t{1} << 63), "NTT modulus must be below 2^63");
    std::uint64_t psi = ma::primitive_root_of_order(2 * n, q);  // validates q and 2n | q - 1
    require((q - 1) % m == 0, "modulus does not admit the power-of-two Bluestein convolution root");
    if (inverse) psi = ma::powmod(psi, q - 2, q);
    // children: forward natural -> bit-reversed, inverse bit-reversed -> natural (x conv^-1)
    cubf::Descriptor c = bluestein_child(d);
    c.output_orders = {CUBUTTERFLY_ORDER_BIT_REVERSED};
    const std::size_t work_bytes = align256(m * d.batch * 8);
    std::size_t child_ws = 0;
    for (int i = 0; i < 2; ++i) {
        cubf::Descriptor ci = c;
        if (i == 1) {
            ci.direction = CUBUTTERFLY_DIRECTION_INVERSE;
            ci.input_orders = {CUBUTTERFLY_ORDER_BIT_REVERSED};
            ci.output_orders = {CUBUTTERFLY_ORDER_NATURAL};
        }
        cubutterflyPlan::Axis ax;
        ax.plan = create_rank1(handle, cubf::normalize(ci));
        ax.n = m;
        ax.outer = d.batch;
        ax.inner = 1;
        ax.ws_offset = work_bytes;
        child_ws = std::max(child_ws, ax.plan->mapping.workspace_bytes);
        p->axes.push_back(std::move(ax));
    }
    p->mapping.family = "bluestein-ntt";
    p->mapping.label = "bluestein-ntt[" + std::to_string(m) + ":" + p->axes[0].plan->mapping.name() + "]";
    p->mapping.workspace_bytes = work_bytes + align256(child_ws);
    p->source = p->axes[0].plan->source;
    p->reason = "non-power-of-two NTT of " + std::to_string(n) + " points as a " + std::to_string(m) +
                "-point cyclic convolution (Bluestein) over power-of-two NTT plans";

    // host tables
    const NttChirpTables t(n, m);
    std::vector<std::uint64_t> host(t.bytes / 8, 0);
    const std::uint64_t n_inv = inverse ? ma::powmod(n % q, q - 2, q) : 1;
    std::vector<std::uint64_t> taps(m, 0);
    for (std::size_t j = 0; j < n; ++j) {
        const auto e = static_cast<std::uint64_t>((static_cast<unsigned __int128>(j) * j) % (2 * n));
        const std::uint64_t cj = ma::powmod(psi, e, q);
        const std::uint64_t uj = ma::mulmod(cj, n_inv, q);
        host[t.pack / 8 + j] = cj;
        host[t.pack_q / 8 + j] = ma::shoup(cj, q);
        host[t.unpack / 8 + j] = uj;
        host[t.unpack_q / 8 + j] = ma::shoup(uj, q);
        const std::uint64_t bj = ma::powmod(cj, q - 2, q);
        taps[j] = bj;
        if (j) taps[m - j] = bj;
    }
    check_cuda(cudaMalloc(&p->bluestein_tables, t.bytes), "Bluestein NTT table allocation");
    unsigned char* tb = static_cast<unsigned char*>(p->bluestein_tables);
    // the taps' spectrum, in the forward child's (bit-reversed) order
    cubf::Descriptor k = c;
    k.batch = 1;
    k.input_batch_stride = k.output_batch_stride = m;
    k.placement = CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE;
    auto kp = create_rank1(handle, cubf::normalize(k));
    DeviceTemp temp(align256(m * 8) + align256(kp->mapping.workspace_bytes) + 256);
    unsigned char* dtaps = static_cast<unsigned char*>(temp.ptr);
    kp->workspace = dtaps + align256(m * 8);
    cudaStream_t s = nullptr;
    check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "Bluestein set-up stream");
    try {
        check_cuda(cudaMemcpyAsync(dtaps, taps.data(), m * 8, cudaMemcpyHostToDevice, s), "Bluestein taps upload");
        launch_mapping(*kp, kp->mapping, dtaps, tb + t.spectrum, s);
        check_cuda(cudaMemcpyAsync(host.data() + t.spectrum / 8, tb + t.spectrum, m * 8, cudaMemcpyDeviceToHost, s),
                   "Bluestein spectrum read");
        check_cuda(cudaStreamSynchronize(s), "Bluestein set-up");
        for (std::size_t j = 0; j < m; ++j) host[t.spectrum_q / 8 + j] = ma::shoup(host[t.spectrum / 8 + j], q);
        check_cuda(cudaMemcpyAsync(tb, host.data(), t.bytes, cudaMemcpyHostToDevice, s), "Bluestein table upload");
        check_cuda(cudaStreamSynchronize(s), "Bluestein set-up");
    } catch (...) {
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
        throw;
    }
    cudaStreamDestroy(s);
    return p;
}

// A rank-one plan of any supported length.
std::unique_ptr<cubutterflyPlan> create_axis(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    if (arbitrary_fft(d)) return create_bluestein(handle, d);
    if (arbitrary_ntt(d)) return create_bluestein_ntt(handle, d);
    return create_rank1(handle, d);
}

// The rank-one child descriptors of a rank-two or rank-three descriptor.
struct AxisSpec {
    cubf::Descriptor d;
    std::size_t n, outer, inner;
    std::size_t axis = 0;  // descriptor axis (FFT / NTT children)
};
// skip_innermost: leave the innermost axis untransformed (the outer axes of a
// multi-rank real FFT, whose innermost axis is the half spectrum).
std::vector<AxisSpec> composite_axes(const cubf::Descriptor& d, bool& flat, bool skip_innermost = false) {
    cubf::Descriptor c = d;
    c.rank = 1;
    c.input_orders = c.output_orders = {CUBUTTERFLY_ORDER_NATURAL};
    c.input_ntt_layout = c.output_ntt_layout = CUBUTTERFLY_NTT_LAYOUT_NATURAL;
    c.input_strides = c.output_strides = {1};
    c.stage_matrices.assign(3, {});
    if (c.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) {  // a pass list names one rank-one plan
        c.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
        c.explicit_algorithm.clear();
    }
    std::size_t volume = 1;
    for (auto e : d.extents) volume *= e;
    const bool packed_in = d.input_strides == packed_strides(d.extents) && d.input_batch_stride == volume;
    const bool packed_out = d.output_strides == packed_strides(d.extents) && d.output_batch_stride == volume;
    std::vector<AxisSpec> axes;
    if (d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2) {
        // the structured transform of a row-major tensor is the one of the
        // flattened index whose stages are the innermost axis's, then the next
        std::vector<cubutterflyMatrix2x2_t> flat_stages;
        for (std::size_t k = d.rank; k-- > 0;) {
            const auto& ms = d.stage_matrices.at(k);
            const unsigned bits = cubf::log2_exact(d.extents[k]);
            require(ms.size() == 1 || ms.size() == bits, "structured axis requires one matrix or one per stage");
            for (unsigned s = 0; s < bits; ++s) flat_stages.push_back(ms.size() == 1 ? ms[0] : ms[s]);
        }
        c.stage_matrices.assign(3, {});
        c.stage_matrices[0] = flat_stages;
    }
    if (d.op == CUBUTTERFLY_OPERATOR_FWHT || d.op == CUBUTTERFLY_OPERATOR_SUBSET_ZETA ||
        d.op == CUBUTTERFLY_OPERATOR_SUPERSET_ZETA || d.op == CUBUTTERFLY_OPERATOR_STRUCTURED_2X2) {
        // H_N0 (x) H_N1 (x) ... = H_(N0 N1 ...) on the row-major index, and
        // likewise for the subset / superset order: one transform of the
        // concatenated index bits
        flat = packed_in && packed_out;
        c.extents = {volume};
        c.input_batch_stride = c.output_batch_stride = volume;
        if (!flat) c.placement = CUBUTTERFLY_PLACEMENT_IN_PLACE;
        axes.push_back({c, volume, d.batch, 1});
        return axes;
    }
    flat = false;
    c.placement = CUBUTTERFLY_PLACEMENT_IN_PLACE;  // children run in place on the workspace copies
    for (std::size_t k = d.rank; k-- > 0;) {
        if (skip_innermost && k + 1 == d.rank) continue;
        std::size_t outer = d.batch, inner = 1;
        for (std::size_t j = 0; j < k; ++j) outer *= d.extents[j];
        for (std::size_t j = k + 1; j < d.rank; ++j) inner *= d.extents[j];
        AxisSpec a{c, d.extents[k], outer, inner, k};
        a.d.extents = {d.extents[k]};
        a.d.batch = outer * inner;
        a.d.input_batch_stride = a.d.output_batch_stride = d.extents[k];
        axes.push_back(a);
    }
    return axes;
}

std::unique_ptr<cubutterflyPlan> create_composite(cubutterflyHandle* handle, const cubf::Descriptor& d,
                                                  bool skip_innermost = false) {
    auto p = std::make_unique<cubutterflyPlan>();
    p->desc = d;
    p->input_bytes = layout_span(d, cubf::input_extents(d), d.input_strides, d.input_batch_stride);
    p->output_bytes = layout_span(d, cubf::output_extents(d), d.output_strides, d.output_batch_stride);
    p->hw = cubf::resolve_profile();
    check_cuda(cudaGetDevice(&p->device), "current device");
    std::size_t volume = 1;
    for (auto e : d.extents) volume *= e;
    p->packed_bytes = align256(d.batch * volume * cubf::storage_bytes(d.storage));
    bool flat = false;
    auto specs = composite_axes(d, flat, skip_innermost);
    p->flat = flat;
    // direct FFT composite: packed complex fp32 tensors, power-of-two axes,
    // every outer axis an interleaved batch (n >= 16, n * inner >= 2^12)
    if (d.op == CUBUTTERFLY_OPERATOR_FFT && d.storage == CUBUTTERFLY_DATA_COMPLEX_FP32 && !flat && !skip_innermost &&
        d.input_strides == packed_strides(d.extents) && d.output_strides == packed_strides(d.extents) &&
        d.input_batch_stride == volume && d.output_batch_stride == volume &&
        std::all_of(d.extents.begin(), d.extents.end(), [](std::size_t e) { return cubf::is_pow2(e); }) &&
        std::all_of(specs.begin(), specs.end(),
                    [](const AxisSpec& a) {
                        return a.inner == 1 ||
                               (a.n >= 16 && a.n * a.inner >= 4096 && a.n * a.inner <= (std::size_t{1} << 30));
                    })) {
        p->direct = true;
        std::size_t ws_bytes = 0;
        std::ostringstream name;
        name << "composite-direct[";
        for (std::size_t i = 0; i < specs.size(); ++i) {
            cubf::Descriptor c = specs[i].d;
            if (specs[i].inner > 1) {  // interleaved: element stride = inner, transforms 1 apart
                c.batch = specs[i].inner;
                c.input_strides = c.output_strides = {specs[i].inner};
                c.input_batch_stride = c.output_batch_stride = 1;
            }
            cubutterflyPlan::Axis ax;
            ax.plan = create_rank1(handle, cubf::normalize(c));
            if (specs[i].inner > 1) {
                ax.plan->groups = specs[i].outer;
                ax.plan->mapping.workspace_bytes *= specs[i].outer;
            }
            ax.n = specs[i].n;
            ax.outer = specs[i].outer;
            ax.inner = specs[i].inner;
            ax.ws_offset = 0;
            ws_bytes = std::max(ws_bytes, ax.plan->mapping.workspace_bytes);
            name << (i ? "," : "") << "axis" << specs[i].axis << ":" << ax.plan->mapping.name();
            p->axes.push_back(std::move(ax));
        }
        name << "]";
        p->mapping.family = "composite";
        p->mapping.label =
            d.execution_mode == CUBUTTERFLY_EXECUTION_XD ? "xd[" + name.str() + "]" : name.str();
        p->mapping.workspace_bytes = ws_bytes;
        p->source = p->axes.front().plan->source;
        p->reason = "rank-" + std::to_string(d.rank) +
                    " FFT: the innermost axis from the input, every outer axis in place as interleaved batches";
        return p;
    }
    const bool two_buffers = d.op == CUBUTTERFLY_OPERATOR_FFT || d.op == CUBUTTERFLY_OPERATOR_NTT;
    std::size_t offset = flat ? 0 : p->packed_bytes * (two_buffers ? 2 : 1);
    std::ostringstream name, reason;
    name << "composite[";
    cubutterflySelectionSource_t source = CUBUTTERFLY_SELECTION_STATIC_MODEL;
    for (std::size_t i = 0; i < specs.size(); ++i) {
        cubutterflyPlan::Axis ax;
        ax.plan = create_axis(handle, cubf::normalize(specs[i].d));
        ax.n = specs[i].n;
        ax.outer = specs[i].outer;
        ax.inner = specs[i].inner;
        ax.ws_offset = offset;
        offset += align256(ax.plan->mapping.workspace_bytes);
        const std::string label = flat || (specs.size() == 1 && !skip_innermost) ? "flat"
                                                                                 : "axis" + std::to_string(specs[i].axis);
        name << (i ? "," : "") << label << ":" << ax.plan->mapping.name();
        reason << (i ? "; " : "") << label << ": " << ax.plan->reason;
        if (ax.plan->source != CUBUTTERFLY_SELECTION_STATIC_MODEL) source = ax.plan->source;
        p->axes.push_back(std::move(ax));
    }
    name << "]";
    if (!flat && p->axes.size() == d.rank) {  // per-axis children, innermost first
        p->physical = d.extents;
        for (std::size_t i = 0; i < p->axes.size(); ++i)
            if (!p->axes[i].plan->physical.empty()) p->physical[d.rank - 1 - i] = p->axes[i].plan->physical[0];
    }
    p->mapping.family = "composite";
    // xD execution requests run as this composite (the reference's own path
    // where its xD lowering does not apply); the name keeps the xD prefix
    p->mapping.label = d.execution_mode == CUBUTTERFLY_EXECUTION_XD ? "xd[" + name.str() + "]" : name.str();
    p->mapping.workspace_bytes = offset;
    p->source = source;
    p->reason = "rank-" + std::to_string(d.rank) + " composition of rank-one plans: " + reason.str();
    return p;
}

// The N/2-point complex FFT under an R2C / C2R descriptor.
cubf::Descriptor real_child(const cubf::Descriptor& d) {
    cubf::Descriptor c = d;
    c.fft_type = CUBUTTERFLY_FFT_C2C;
    c.storage = CUBUTTERFLY_DATA_COMPLEX_FP32;
    c.compute = CUBUTTERFLY_COMPUTE_FP32;
    c.extents = {d.extents[0] / 2};
    c.input_strides = c.output_strides = {1};
    c.input_batch_stride = c.output_batch_stride = d.extents[0] / 2;
    c.normalize_inverse = false;  // C2R folds 2 / N into its merge step
    c.fft_output_scale = 1.0;
    c.placement = CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE;
    if (c.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) {
        c.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
        c.explicit_algorithm.clear();
    }
    return cubf::normalize(c);
}

// R2C / C2R over an N/2-point complex FFT child plan.
std::unique_ptr<cubutterflyPlan> create_real(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    auto p = std::make_unique<cubutterflyPlan>();
    p->desc = d;
    p->real_kind = d.fft_type;
    p->input_bytes = layout_span(d, cubf::input_extents(d), d.input_strides, d.input_batch_stride) *
                     (d.fft_type == CUBUTTERFLY_FFT_C2R ? 2 : 1);
    p->output_bytes = layout_span(d, cubf::output_extents(d), d.output_strides, d.output_batch_stride) *
                      (d.fft_type == CUBUTTERFLY_FFT_R2C ? 2 : 1);
    p->hw = cubf::resolve_profile();
    check_cuda(cudaGetDevice(&p->device), "current device");
    const std::size_t n = d.extents[0], half = n / 2;
    const cubf::Descriptor c = real_child(d);
    p->packed_bytes = align256(d.batch * half * 8);
    cubutterflyPlan::Axis ax;
    ax.plan = create_rank1(handle, c);
    ax.n = half;
    ax.outer = d.batch;
    ax.inner = 1;
    ax.ws_offset = p->packed_bytes;
    p->mapping.family = d.fft_type == CUBUTTERFLY_FFT_R2C ? "fft-r2c" : "fft-c2r";
    p->mapping.label = p->mapping.family + "[" + ax.plan->mapping.name() + "]";
    p->mapping.workspace_bytes = p->packed_bytes + align256(ax.plan->mapping.workspace_bytes);
    p->source = ax.plan->source;
    p->reason = std::string(d.fft_type == CUBUTTERFLY_FFT_R2C ? "R2C" : "C2R") + " over an N/2-point complex FFT: " +
                ax.plan->reason;
    p->axes.push_back(std::move(ax));
    // W_N^k = exp(-2 pi i k / N), k = 0..N/2, computed in double, rounded once
    constexpr double kPi = 3.141592653589793238462643383279502884;
    std::vector<float> tw(2 * (half + 1));
    for (std::size_t k = 0; k <= half; ++k) {
        const double a = -2.0 * kPi * static_cast<double>(k) / static_cast<double>(n);
        tw[2 * k] = static_cast<float>(std::cos(a));
        tw[2 * k + 1] = static_cast<float>(std::sin(a));
    }
    check_cuda(cudaMalloc(&p->real_tw, tw.size() * sizeof(float)), "real twiddle allocation");
    check_cuda(cudaMemcpy(p->real_tw, tw.data(), tw.size() * sizeof(float), cudaMemcpyHostToDevice),
               "real twiddle upload");
    return p;
}

// The row transform of a rank-two / rank-three real FFT: the rank-one real
// transform of every innermost line, packed, carrying the output scale (and
// the outer axes' share of a normalised inverse's 1 / N).
cubf::Descriptor real_rows(const cubf::Descriptor& d) {
    const bool r2c = d.fft_type == CUBUTTERFLY_FFT_R2C;
    const bool inverse = d.direction == CUBUTTERFLY_DIRECTION_INVERSE;
    const std::size_t nl = d.extents.back(), h = nl / 2 + 1;
    std::size_t outer = 1;
    for (std::size_t k = 0; k + 1 < d.rank; ++k) outer *= d.extents[k];
    cubf::Descriptor r = d;
    r.rank = 1;
    r.extents = {nl};
    r.batch = d.batch * outer;
    r.input_strides = r.output_strides = {1};
    r.input_batch_stride = r2c ? nl : h;
    r.output_batch_stride = r2c ? h : nl;
    r.input_orders = r.output_orders = {CUBUTTERFLY_ORDER_NATURAL};
    r.stage_matrices.assign(3, {});
    r.execution_mode = CUBUTTERFLY_EXECUTION_AUTO;
    r.fft_output_scale = d.fft_output_scale * (inverse && d.normalize_inverse ? 1.0 / static_cast<double>(outer) : 1.0);
    if (r.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) {
        r.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
        r.explicit_algorithm.clear();
    }
    return cubf::normalize(r);
}

// The outer axes of a rank-two / rank-three real FFT: C2C over the packed
// half-spectrum tensor, whose innermost axis the composite leaves untouched.
cubf::Descriptor real_outer(const cubf::Descriptor& d) {
    const std::size_t h = d.extents.back() / 2 + 1;
    std::size_t outer = 1;
    for (std::size_t k = 0; k + 1 < d.rank; ++k) outer *= d.extents[k];
    cubf::Descriptor c = d;
    c.fft_type = CUBUTTERFLY_FFT_C2C;
    c.storage = CUBUTTERFLY_DATA_COMPLEX_FP32;
    c.compute = CUBUTTERFLY_COMPUTE_FP32;
    c.extents.back() = h;
    c.input_strides = c.output_strides = packed_strides(c.extents);
    c.input_batch_stride = c.output_batch_stride = outer * h;
    c.input_orders = c.output_orders = std::vector<cubutterflyLogicalOrder_t>(d.rank, CUBUTTERFLY_ORDER_NATURAL);
    c.normalize_inverse = false;
    c.fft_output_scale = 1.0;
    c.placement = CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE;
    c.execution_mode = CUBUTTERFLY_EXECUTION_AUTO;
    if (c.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) {
        c.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
        c.explicit_algorithm.clear();
    }
    return cubf::normalize(c);
}

// Rank-two and rank-three R2C / C2R (the reference's RealFFT,
// python/cubutterfly/real_fft.py): axes[0] the rank-one real transform of
// the innermost axis over every row, axes[1] a C2C composite over the outer
// axes of the half-spectrum tensor (its innermost axis untouched).  R2C runs
// rows then outer axes, C2R the reverse, through a packed half tensor at the
// start of the workspace; the output scale (and a normalised inverse's 1 / N)
// is applied once, by the row transform.
std::unique_ptr<cubutterflyPlan> create_real_nd(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    auto p = std::make_unique<cubutterflyPlan>();
    p->desc = d;
    p->real_nd = true;
    p->input_bytes = layout_span(d, cubf::input_extents(d), d.input_strides, d.input_batch_stride) *
                     (d.fft_type == CUBUTTERFLY_FFT_C2R ? 2 : 1);
    p->output_bytes = layout_span(d, cubf::output_extents(d), d.output_strides, d.output_batch_stride) *
                      (d.fft_type == CUBUTTERFLY_FFT_R2C ? 2 : 1);
    p->hw = cubf::resolve_profile();
    check_cuda(cudaGetDevice(&p->device), "current device");
    const bool r2c = d.fft_type == CUBUTTERFLY_FFT_R2C;
    const std::size_t nl = d.extents.back(), h = nl / 2 + 1;
    std::size_t outer = 1;
    for (std::size_t k = 0; k + 1 < d.rank; ++k) outer *= d.extents[k];
    const cubf::Descriptor r = real_rows(d), c = real_outer(d);
    p->packed_bytes = align256(d.batch * outer * h * 8);
    cubutterflyPlan::Axis rows, axes;
    rows.plan = create_real(handle, r);
    axes.plan = create_composite(handle, c, true);
    rows.n = nl;
    axes.n = h;
    rows.outer = axes.outer = d.batch;
    rows.inner = axes.inner = 1;
    rows.ws_offset = axes.ws_offset = p->packed_bytes;
    p->mapping.family = r2c ? "fft-r2c" : "fft-c2r";
    p->mapping.label = p->mapping.family + "-rank" + std::to_string(d.rank) + "[rows:" + rows.plan->mapping.name() +
                       "," + axes.plan->mapping.name() + "]";
    p->mapping.workspace_bytes =
        p->packed_bytes + align256(std::max(rows.plan->mapping.workspace_bytes, axes.plan->mapping.workspace_bytes));
    p->source = rows.plan->source;
    p->reason = std::string(r2c ? "R2C" : "C2R") + " of rank " + std::to_string(d.rank) +
                ": rank-one real rows, then C2C outer axes of the half spectrum: " + rows.plan->reason;
    p->axes.push_back(std::move(rows));
    p->axes.push_back(std::move(axes));
    return p;
}

// FP64 FWHT as the structured 2x2 butterfly: H_2 = [[1, 1], [1, -1]] in every
// stage (1 * x is exact, so each stage is (l + r, l - r) as in the reference's
// double FWHT); an inverse normalised by 1/N halves every stage instead, which
// is exact for a power-of-two N.
std::unique_ptr<cubutterflyPlan> create_fwht64(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    cubf::Descriptor s = d;
    s.op = CUBUTTERFLY_OPERATOR_STRUCTURED_2X2;
    const bool halve = d.direction == CUBUTTERFLY_DIRECTION_INVERSE && d.normalize_inverse;
    const double h = halve ? 0.5 : 1.0;
    s.direction = CUBUTTERFLY_DIRECTION_FORWARD;
    s.normalize_inverse = false;
    s.stage_matrices.assign(3, {});
    for (std::size_t k = 0; k < d.rank; ++k) s.stage_matrices[k] = {cubutterflyMatrix2x2_t{h, h, h, -h}};
    s = cubf::normalize(s);
    auto p = s.rank == 1 ? create_rank1(handle, s) : create_composite(handle, s);
    p->mapping.label = "fwht-f64:" + p->mapping.name();
    return p;
}

// Zero-extended embedding over a packed plan of the padded length.
std::unique_ptr<cubutterflyPlan> create_embedded(cubutterflyHandle* handle, const cubf::Descriptor& d) {
    auto p = std::make_unique<cubutterflyPlan>();
    p->desc = d;
    p->embedded = true;
    p->input_bytes = layout_span(d, cubf::input_extents(d), d.input_strides, d.input_batch_stride);
    p->output_bytes = layout_span(d, cubf::output_extents(d), d.output_strides, d.output_batch_stride);
    p->hw = cubf::resolve_profile();
    check_cuda(cudaGetDevice(&p->device), "current device");
    std::size_t pn = 1;
    while (pn < d.extents[0]) pn <<= 1;
    cubf::Descriptor c = d;
    c.length_mode = CUBUTTERFLY_LENGTH_STANDARD;
    c.extents = {pn};
    c.input_strides = c.output_strides = {1};
    c.input_batch_stride = c.output_batch_stride = pn;
    c.placement = CUBUTTERFLY_PLACEMENT_IN_PLACE;
    if (c.algorithm_policy == CUBUTTERFLY_ALGORITHM_EXPLICIT) {
        c.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
        c.explicit_algorithm.clear();
    }
    p->packed_bytes = align256(d.batch * pn * cubf::storage_bytes(d.storage));
    cubutterflyPlan::Axis ax;
    ax.plan = create_rank1(handle, cubf::normalize(c));
    ax.n = pn;
    p->physical = {pn};
    ax.outer = d.batch;
    ax.inner = 1;
    ax.ws_offset = p->packed_bytes;
    p->mapping.family = "zero-extended";
    p->mapping.label = "zero-extended[" + ax.plan->mapping.name() + "]";
    p->mapping.workspace_bytes = p->packed_bytes + align256(ax.plan->mapping.workspace_bytes);
    p->source = ax.plan->source;
    p->reason = "zero-extended embedding of " + std::to_string(d.extents[0]) + " points into " + std::to_string(pn) +
                ": " + ax.plan->reason;
    p->axes.push_back(std::move(ax));
    return p;
}

// Mapping JSON of a composite plan: its children, in execution order.
cubf::Json composite_json(const cubutterflyPlan& p) {
    cubf::Json axes = cubf::Json::array();
    for (const auto& ax : p.axes)
        axes.push_back({{"length", ax.n}, {"outer", ax.outer}, {"inner", ax.inner},
                        {"mapping", ax.plan->mapping.to_json()}});
    return {{"schema", "cubutterfly-b200-mapping-v1"},
            {"family", p.mapping.family},
            {"name", p.mapping.name()},
            {"flat", p.flat},
            {"axes", axes},
            {"workspace_bytes", p.mapping.workspace_bytes}};
}

}  // namespace

namespace cubf {
void set_last_error(const std::string& message) { last_error = message; }
}  // namespace cubf

extern "C" {

const char* cubutterflyGetStatusString(cubutterflyStatus_t status) {
    switch (status) {
        case CUBUTTERFLY_STATUS_SUCCESS: return "CUBUTTERFLY_STATUS_SUCCESS";
        case CUBUTTERFLY_STATUS_INVALID_VALUE: return "CUBUTTERFLY_STATUS_INVALID_VALUE";
        case CUBUTTERFLY_STATUS_INVALID_TYPE: return "CUBUTTERFLY_STATUS_INVALID_TYPE";
        case CUBUTTERFLY_STATUS_NOT_SUPPORTED: return "CUBUTTERFLY_STATUS_NOT_SUPPORTED";
        case CUBUTTERFLY_STATUS_ALLOC_FAILED: return "CUBUTTERFLY_STATUS_ALLOC_FAILED";
        case CUBUTTERFLY_STATUS_CUDA_ERROR: return "CUBUTTERFLY_STATUS_CUDA_ERROR";
        case CUBUTTERFLY_STATUS_BACKEND_ERROR: return "CUBUTTERFLY_STATUS_BACKEND_ERROR";
        case CUBUTTERFLY_STATUS_INTERNAL_ERROR: return "CUBUTTERFLY_STATUS_INTERNAL_ERROR";
    }
    return "CUBUTTERFLY_STATUS_UNKNOWN";
}

const char* cubutterflyGetLastErrorString(void) { return last_error.c_str(); }

cubutterflyStatus_t cubutterflyGetVersion(int* major, int* minor, int* patch) {
    return protect([&] {
        require(major && minor && patch, "version pointers must be non-null");
        *major = CUBUTTERFLY_VERSION_MAJOR;
        *minor = CUBUTTERFLY_VERSION_MINOR;
        *patch = CUBUTTERFLY_VERSION_PATCH;
    });
}

cubutterflyStatus_t cubutterflyCreate(cubutterflyHandle_t* handle) {
    return protect([&] {
        require(handle != nullptr, "handle pointer must be non-null");
        *handle = new cubutterflyHandle();
    });
}

cubutterflyStatus_t cubutterflyDestroy(cubutterflyHandle_t handle) {
    return protect([&] { delete handle; });
}

cubutterflyStatus_t cubutterflySetStream(cubutterflyHandle_t handle, cudaStream_t stream) {
    return protect([&] {
        require(handle != nullptr, "handle must be non-null");
        handle->stream = stream;
    });
}

cubutterflyStatus_t cubutterflyGetStream(cubutterflyHandle_t handle, cudaStream_t* stream) {
    return protect([&] {
        require(handle != nullptr && stream != nullptr, "handle and stream pointer must be non-null");
        *stream = handle->stream;
    });
}

cubutterflyStatus_t cubutterflySetLogCallback(cubutterflyHandle_t handle, cubutterflyLogCallback_t callback,
                                              void* user_data) {
    return protect([&] {
        require(handle != nullptr, "handle must be non-null");
        handle->logger = callback;
        handle->logger_data = user_data;
    });
}

cubutterflyStatus_t cubutterflySetCachePath(cubutterflyHandle_t handle, const char* path) {
    return protect([&] {
        require(handle != nullptr, "handle must be non-null");
        handle->cache_path = path ? path : "";
    });
}

// cubutterflyPackRealFp32 and cubutterflyExpandHermitianFp32 live in real_adapter.cu.

cubutterflyStatus_t cubutterflyCreateDescriptor(cubutterflyDescriptor_t* descriptor) {
    return protect([&] {
        require(descriptor != nullptr, "descriptor pointer must be non-null");
        *descriptor = new cubutterflyDescriptor();
    });
}

cubutterflyStatus_t cubutterflyDestroyDescriptor(cubutterflyDescriptor_t descriptor) {
    return protect([&] { delete descriptor; });
}

cubutterflyStatus_t cubutterflySetOperator(cubutterflyDescriptor_t d, cubutterflyOperator_t op) {
    return protect([&] {
        require(static_cast<int>(op) >= 0 && static_cast<int>(op) <= 5, "invalid operator");
        desc_of(d).op = op;
    });
}

cubutterflyStatus_t cubutterflySetDataType(cubutterflyDescriptor_t d, cubutterflyDataType_t storage,
                                           cubutterflyComputeType_t compute) {
    return protect([&] {
        require(static_cast<int>(storage) >= 0 && static_cast<int>(storage) <= 9, "invalid storage type");
        require(static_cast<int>(compute) >= 0 && static_cast<int>(compute) <= 4, "invalid compute type");
        desc_of(d).storage = storage;
        desc_of(d).compute = compute;
    });
}

cubutterflyStatus_t cubutterflySetShape(cubutterflyDescriptor_t d, uint32_t rank, const size_t* extents,
                                        size_t batch) {
    return protect([&] {
        require(rank > 0 && extents != nullptr, "rank must be positive and extents non-null");
        require(batch > 0, "batch must be positive");
        auto& x = desc_of(d);
        x.rank = rank;
        x.extents.assign(extents, extents + rank);
        x.batch = batch;
        x.input_strides.clear();
        x.output_strides.clear();
        x.input_orders.clear();
        x.output_orders.clear();
        x.stage_matrices.assign(std::max<std::size_t>(3, rank), {});
    });
}

cubutterflyStatus_t cubutterflySetExecutionMode(cubutterflyDescriptor_t d, cubutterflyExecutionMode_t mode) {
    return protect([&] {
        require(static_cast<int>(mode) >= 0 && static_cast<int>(mode) <= 2, "invalid execution mode");
        desc_of(d).execution_mode = mode;
    });
}

cubutterflyStatus_t cubutterflySetFftTransformType(cubutterflyDescriptor_t d, cubutterflyFftTransformType_t type) {
    return protect([&] {
        require(static_cast<int>(type) >= 0 && static_cast<int>(type) <= 2, "invalid FFT transform type");
        desc_of(d).fft_type = type;
    });
}

cubutterflyStatus_t cubutterflySetFftOutputScale(cubutterflyDescriptor_t d, double scale) {
    return protect([&] {
        require(std::isfinite(scale), "FFT output scale must be finite");
        desc_of(d).fft_output_scale = scale;
    });
}

cubutterflyStatus_t cubutterflySetOutputScale(cubutterflyDescriptor_t d, double scale) {
    return protect([&] {
        require(std::isfinite(scale), "output scale must be finite");
        desc_of(d).output_scale = scale;
    });
}

cubutterflyStatus_t cubutterflySetArithmeticPolicy(cubutterflyDescriptor_t d, cubutterflyArithmeticPolicy_t policy) {
    return protect([&] {
        require(static_cast<int>(policy) >= 0 && static_cast<int>(policy) <= 1, "invalid arithmetic policy");
        desc_of(d).arithmetic_policy = policy;
    });
}

cubutterflyStatus_t cubutterflySetOutputRounding(cubutterflyDescriptor_t d, cubutterflyOutputRounding_t rounding) {
    return protect([&] {
        require(static_cast<int>(rounding) >= 0 && static_cast<int>(rounding) <= 1, "invalid output rounding");
        desc_of(d).output_rounding = rounding;
    });
}

cubutterflyStatus_t cubutterflySetStrides(cubutterflyDescriptor_t d, const size_t* input_strides,
                                          size_t input_batch_stride, const size_t* output_strides,
                                          size_t output_batch_stride) {
    return protect([&] {
        auto& x = desc_of(d);
        const std::size_t rank = x.extents.size();
        x.input_strides = input_strides ? std::vector<std::size_t>(input_strides, input_strides + rank)
                                        : std::vector<std::size_t>{};
        x.output_strides = output_strides ? std::vector<std::size_t>(output_strides, output_strides + rank)
                                          : std::vector<std::size_t>{};
        x.input_batch_stride = input_batch_stride;
        x.output_batch_stride = output_batch_stride;
    });
}

cubutterflyStatus_t cubutterflySetLogicalOrders(cubutterflyDescriptor_t d, const cubutterflyLogicalOrder_t* in,
                                                const cubutterflyLogicalOrder_t* out) {
    return protect([&] {
        auto& x = desc_of(d);
        const std::size_t rank = x.extents.size();
        x.input_orders = in ? std::vector<cubutterflyLogicalOrder_t>(in, in + rank)
                            : std::vector<cubutterflyLogicalOrder_t>{};
        x.output_orders = out ? std::vector<cubutterflyLogicalOrder_t>(out, out + rank)
                              : std::vector<cubutterflyLogicalOrder_t>{};
    });
}

cubutterflyStatus_t cubutterflyDescriptorValidate(cubutterflyDescriptor_t d) {
    return protect([&] { (void)cubf::normalize(desc_of(d)); });
}

cubutterflyStatus_t cubutterflyDescriptorGetJson(cubutterflyDescriptor_t d, char* json, size_t* bytes) {
    return protect([&] { copy_text(cubf::descriptor_json(desc_of(d)).dump(), json, bytes); });
}

cubutterflyStatus_t cubutterflyDescriptorSetJson(cubutterflyDescriptor_t d, const char* json) {
    return protect([&] {
        require(json != nullptr, "JSON text must be non-null");
        auto& x = desc_of(d);
        cubf::Descriptor parsed = cubf::descriptor_from_json(cubf::Json::parse(json));
        x = cubutterflyDescriptor{parsed};  // atomic replacement
    });
}

cubutterflyStatus_t cubutterflyDescriptorGetCapabilities(cubutterflyDescriptor_t d, char* json, size_t* bytes) {
    return protect([&] { copy_text(cubf::capabilities(desc_of(d)).dump(), json, bytes); });
}

cubutterflyStatus_t cubutterflySetDirection(cubutterflyDescriptor_t d, cubutterflyDirection_t direction,
                                            int normalize_inverse) {
    return protect([&] {
        require(static_cast<int>(direction) >= 0 && static_cast<int>(direction) <= 1, "invalid direction");
        desc_of(d).direction = direction;
        desc_of(d).normalize_inverse = normalize_inverse != 0;
    });
}

cubutterflyStatus_t cubutterflySetPlacement(cubutterflyDescriptor_t d, cubutterflyPlacement_t placement) {
    return protect([&] {
        require(static_cast<int>(placement) >= 0 && static_cast<int>(placement) <= 1, "invalid placement");
        desc_of(d).placement = placement;
    });
}

cubutterflyStatus_t cubutterflySetLengthMode(cubutterflyDescriptor_t d, cubutterflyLengthMode_t mode) {
    return protect([&] {
        require(static_cast<int>(mode) >= 0 && static_cast<int>(mode) <= 1, "invalid length mode");
        desc_of(d).length_mode = mode;
    });
}

cubutterflyStatus_t cubutterflySetAlgorithmPolicy(cubutterflyDescriptor_t d, cubutterflyAlgorithmPolicy_t policy,
                                                  const char* explicit_algorithm) {
    return protect([&] {
        require(static_cast<int>(policy) >= 0 && static_cast<int>(policy) <= 2, "invalid algorithm policy");
        auto& x = desc_of(d);
        x.algorithm_policy = policy;
        x.explicit_algorithm = explicit_algorithm ? explicit_algorithm : "";
    });
}

cubutterflyStatus_t cubutterflySetModulus(cubutterflyDescriptor_t d, uint64_t modulus, uint32_t word_bits) {
    return protect([&] {
        require(word_bits == 32 || word_bits == 64, "word bits must be 32 or 64");
        desc_of(d).modulus = modulus;
        desc_of(d).word_bits = word_bits;
    });
}

cubutterflyStatus_t cubutterflySetNttLayouts(cubutterflyDescriptor_t d, cubutterflyNttLayout_t in,
                                             cubutterflyNttLayout_t out) {
    return protect([&] {
        require(static_cast<int>(in) >= 0 && static_cast<int>(in) <= 2 && static_cast<int>(out) >= 0 &&
                    static_cast<int>(out) <= 2,
                "invalid NTT layout");
        desc_of(d).input_ntt_layout = in;
        desc_of(d).output_ntt_layout = out;
    });
}

cubutterflyStatus_t cubutterflySetStageMatrices(cubutterflyDescriptor_t d, uint32_t axis,
                                                const cubutterflyMatrix2x2_t* matrices, size_t count) {
    return protect([&] {
        auto& x = desc_of(d);
        require(axis < x.rank, "matrix axis out of range");
        require(count == 0 || matrices != nullptr, "matrices must be non-null");
        if (x.stage_matrices.size() < std::max<std::size_t>(3, x.rank)) x.stage_matrices.resize(std::max<std::size_t>(3, x.rank));
        x.stage_matrices[axis].assign(matrices, matrices + count);
    });
}

cubutterflyStatus_t cubutterflyCreatePlan(cubutterflyHandle_t handle, cubutterflyDescriptor_t descriptor,
                                          cubutterflyPlan_t* plan) {
    return protect([&] {
        require(handle != nullptr && plan != nullptr, "handle and plan pointer must be non-null");
        *plan = nullptr;
        const cubf::Descriptor d = cubf::normalize(desc_of(descriptor));
        const cubf::Json caps = cubf::capabilities(d);
        if (caps.at("status") != "eligible") {
            const auto& gap = caps.at("gaps").at(0);
            throw cubf::Unsupported(gap.at("code").get<std::string>() + ": " + gap.at("reason").get<std::string>());
        }
        auto p = d.op == CUBUTTERFLY_OPERATOR_FWHT && d.storage == CUBUTTERFLY_DATA_FP64
                     ? create_fwht64(handle, d)
                 : d.length_mode == CUBUTTERFLY_LENGTH_ZERO_EXTENDED_EMBEDDING ? create_embedded(handle, d)
                 : d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type != CUBUTTERFLY_FFT_C2C
                     ? (d.rank == 1 ? create_real(handle, d) : create_real_nd(handle, d))
                 : d.rank == 1                                                        ? create_axis(handle, d)
                                                                                      : create_composite(handle, d);
        log_event(handle, CUBUTTERFLY_LOG_INFO, "plan-selected", p->reason);
        if (p->source == CUBUTTERFLY_SELECTION_STATIC_MODEL) {
            // no measurement backs this choice on this device: say so, and
            // how to get one (the reference's "workload-profile-miss" event)
            log_event(handle, CUBUTTERFLY_LOG_WARNING, "workload-profile-miss",
                      "no measured mapping for this workload on " + p->hw.name + "; using the static model's " +
                          p->reason + "; select MEASURE with a cache path to calibrate it");
        }
        *plan = p.release();
    });
}

cubutterflyStatus_t cubutterflyDestroyPlan(cubutterflyPlan_t plan) {
    return protect([&] { delete plan; });
}

cubutterflyStatus_t cubutterflyPlanGetDescriptorJson(cubutterflyPlan_t plan, char* json, size_t* bytes) {
    return protect([&] {
        require(plan != nullptr, "plan must be non-null");
        copy_text(cubf::descriptor_json(plan->desc).dump(), json, bytes);
    });
}

cubutterflyStatus_t cubutterflyPlanGetWorkspaceSize(cubutterflyPlan_t plan, size_t* bytes) {
    return protect([&] {
        require(plan != nullptr && bytes != nullptr, "plan and size pointer must be non-null");
        *bytes = plan->mapping.workspace_bytes;
    });
}

cubutterflyStatus_t cubutterflyPlanGetInputSize(cubutterflyPlan_t plan, size_t* bytes) {
    return protect([&] {
        require(plan != nullptr && bytes != nullptr, "plan and size pointer must be non-null");
        *bytes = plan->input_bytes;
    });
}

cubutterflyStatus_t cubutterflyPlanGetOutputSize(cubutterflyPlan_t plan, size_t* bytes) {
    return protect([&] {
        require(plan != nullptr && bytes != nullptr, "plan and size pointer must be non-null");
        *bytes = plan->output_bytes;
    });
}

cubutterflyStatus_t cubutterflyPlanGetPhysicalExtents(cubutterflyPlan_t plan, size_t* extents, uint32_t capacity) {
    return protect([&] {
        require(plan != nullptr && extents != nullptr, "plan and extents must be non-null");
        require(capacity >= plan->desc.rank, "extent capacity is smaller than the rank");
        for (std::size_t a = 0; a < plan->desc.rank; ++a)
            extents[a] = plan->physical.empty() ? plan->desc.extents[a] : plan->physical[a];
    });
}

cubutterflyStatus_t cubutterflyPlanGetSelectionSource(cubutterflyPlan_t plan, cubutterflySelectionSource_t* source) {
    return protect([&] {
        require(plan != nullptr && source != nullptr, "plan and source pointer must be non-null");
        *source = plan->source;
    });
}

cubutterflyStatus_t cubutterflyPlanGetAlgorithmName(cubutterflyPlan_t plan, char* name, size_t* bytes) {
    return protect([&] {
        require(plan != nullptr, "plan must be non-null");
        copy_text(plan->mapping.name(), name, bytes);
    });
}

cubutterflyStatus_t cubutterflyPlanGetSelectionReason(cubutterflyPlan_t plan, char* reason, size_t* bytes) {
    return protect([&] {
        require(plan != nullptr, "plan must be non-null");
        copy_text(plan->reason, reason, bytes);
    });
}

cubutterflyStatus_t cubutterflyPlanGetMappingJson(cubutterflyPlan_t plan, char* json, size_t* bytes) {
    return protect([&] {
        require(plan != nullptr, "plan must be non-null");
        cubf::Json j = plan->axes.empty() ? plan->mapping.to_json() : composite_json(*plan);
        j["hardware"] = plan->hw.to_json();
        copy_text(j.dump(), json, bytes);
    });
}

cubutterflyStatus_t cubutterflyPlanGetNttLayoutInfo(cubutterflyPlan_t plan, cubutterflyNttLayoutInfo_t* info) {
    return protect([&] {
        require(plan != nullptr && info != nullptr, "plan and info must be non-null");
        // The reference reports layout info only for its APPT static-layout
        // NTT cores (src/c_api.cpp:4843-4870); this build executes natural
        // and bit-reversed orders only.
        throw cubf::Unsupported("NTT layout info describes APPT static layouts, which this build does not execute");
    });
}

cubutterflyStatus_t cubutterflyPlanSetWorkspace(cubutterflyPlan_t plan, void* workspace, size_t bytes) {
    return protect([&] {
        require(plan != nullptr, "plan must be non-null");
        require(bytes >= plan->mapping.workspace_bytes, "workspace is smaller than the plan requires");
        require(plan->mapping.workspace_bytes == 0 || workspace != nullptr, "workspace must be non-null");
        require(reinterpret_cast<std::uintptr_t>(workspace) % 16 == 0, "workspace must be 16-byte aligned");
        plan->workspace = workspace;
        plan->workspace_size = bytes;
    });
}

namespace {
// The device-status words of a plan and of its child plans, OR-ed.
unsigned int device_status(const cubutterflyPlan& p) {
    unsigned int bits = p.status_host ? *reinterpret_cast<volatile unsigned int*>(p.status_host) : 0u;
    for (const auto& a : p.axes)
        if (a.plan) bits |= device_status(*a.plan);
    return bits;
}

void clear_device_status(cubutterflyPlan& p) {
    if (p.status_host) *reinterpret_cast<volatile unsigned int*>(p.status_host) = 0u;
    for (auto& a : p.axes)
        if (a.plan) clear_device_status(*a.plan);
}

// Caller pointers must be aligned to their element (the reference's contract:
// any element pointer of a cudaMalloc'd buffer); real FFT data moves as
// float2 pairs, so its real side needs 8 bytes.
void check_element_alignment(const cubutterflyPlan& p, const void* input, const void* output) {
    const auto& d = p.desc;
    std::size_t in_align = cubf::storage_bytes(d.storage), out_align = in_align;
    if (d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type != CUBUTTERFLY_FFT_C2C) in_align = out_align = 8;
    require(reinterpret_cast<std::uintptr_t>(input) % in_align == 0,
            "input must be aligned to its element (" + std::to_string(in_align) + " bytes)");
    require(reinterpret_cast<std::uintptr_t>(output) % out_align == 0,
            "output must be aligned to its element (" + std::to_string(out_align) + " bytes)");
}

// A failure that an earlier launch of this plan recorded on the device (a
// bounded wait that expired: that launch's output is invalid) is the status
// of the next call on the plan; reporting it clears it.
void report_device_status(cubutterflyPlan& p) {
    const unsigned int bits = device_status(p);
    if (bits == 0) return;
    clear_device_status(p);
    std::ostringstream o;
    o << "an earlier launch of this plan failed on the device (status bits 0x" << std::hex << bits
      << "): "
      << ((bits & 1u) ? "a tensor-core completion wait expired" : "kernel launch invariant violated")
      << "; that launch's output is invalid";
    throw std::runtime_error(o.str());
}
}  // namespace

cubutterflyStatus_t cubutterflyExecute(cubutterflyHandle_t handle, cubutterflyPlan_t plan, const void* input,
                                       void* output) {
    return protect([&] {
        require(handle != nullptr && plan != nullptr, "handle and plan must be non-null");
        report_device_status(*plan);
        require(input != nullptr && output != nullptr, "input and output must be non-null");
        const bool in_place = plan->desc.placement == CUBUTTERFLY_PLACEMENT_IN_PLACE;
        require(in_place == (input == output),
                in_place ? "in-place plans require input == output" : "out-of-place plans require input != output");
        require(plan->mapping.workspace_bytes == 0 || plan->workspace != nullptr, "plan workspace is not set");
        check_element_alignment(*plan, input, output);
        launch_mapping(*plan, plan->mapping, input, output, handle->stream);
        plan->steady_stream = handle->stream;
        plan->steady_ready = true;
    });
}

cubutterflyStatus_t cubutterflyExecuteSteady(cubutterflyHandle_t handle, cubutterflyPlan_t plan, const void* input,
                                             void* output) {
    if (!handle || !plan || !plan->steady_ready || plan->steady_stream != handle->stream)
        return cubutterflyExecute(handle, plan, input, output);
    return protect([&] {
        report_device_status(*plan);
        const bool in_place = plan->desc.placement == CUBUTTERFLY_PLACEMENT_IN_PLACE;
        require(input != nullptr && output != nullptr && in_place == (input == output),
                "pointer aliasing does not match the plan placement");
        check_element_alignment(*plan, input, output);
        launch_mapping(*plan, plan->mapping, input, output, handle->stream);
    });
}

cubutterflyStatus_t cubutterflyB200PlanGetDeviceStatus(cubutterflyPlan_t plan, unsigned int* bits) {
    return protect([&] {
        require(plan != nullptr && bits != nullptr, "plan and bits must be non-null");
        *bits = device_status(*plan);
    });
}

cubutterflyStatus_t cubutterflyB200PlanInjectDeviceStatus(cubutterflyPlan_t plan, unsigned int bits) {
    return protect([&] {
        require(plan != nullptr, "plan must be non-null");
        cubutterflyPlan* p = plan;
        while (p->status_host == nullptr && p->axes.size() == 1 && p->axes[0].plan) p = p->axes[0].plan.get();
        if (p->status_host == nullptr)
            throw cubf::Unsupported("plan has no device status word (only tensor-core FWHT plans wait on the device)");
        *reinterpret_cast<volatile unsigned int*>(p->status_host) |= bits;
    });
}

cubutterflyStatus_t cubutterflyB200RankMappings(cubutterflyDescriptor_t descriptor, const char* hardware_json,
                                               char* json, size_t* bytes) {
    return protect([&] {
        const cubf::Descriptor d = cubf::normalize(desc_of(descriptor));
        const cubf::Json caps = cubf::capabilities(d);
        if (caps.at("status") != "eligible") {
            const auto& gap = caps.at("gaps").at(0);
            throw cubf::Unsupported(gap.at("code").get<std::string>() + ": " + gap.at("reason").get<std::string>());
        }
        const cubf::HardwareProfile hw = hardware_json ? cubf::profile_from_json(cubf::Json::parse(hardware_json))
                                                       : cubf::resolve_profile();
        cubf::Json out = cubf::Json::array();
        // the best mapping of a rank-one child (its power-of-two core for a
        // Bluestein axis)
        auto child_mapping = [&](const cubf::Descriptor& c) -> cubf::Json {
            if (!arbitrary_fft(c) && !arbitrary_ntt(c))
                return cubf::enumerate_mappings(make_request(c), hw).front().to_json();
            cubf::Descriptor k = bluestein_child(c);
            if (c.op == CUBUTTERFLY_OPERATOR_NTT) {
                k.output_orders = {CUBUTTERFLY_ORDER_BIT_REVERSED};
                k = cubf::normalize(k);
            }
            return {{"family", c.op == CUBUTTERFLY_OPERATOR_NTT ? "bluestein-ntt" : "bluestein"},
                    {"convolution_length", k.extents[0]},
                    {"core", cubf::enumerate_mappings(make_request(k), hw).front().to_json()}};
        };
        if ((arbitrary_fft(d) || arbitrary_ntt(d)) && d.rank == 1) {
            cubf::Json axes = cubf::Json::array();
            axes.push_back({{"length", d.extents[0]}, {"outer", d.batch}, {"inner", 1}, {"mapping", child_mapping(d)}});
            out.push_back({{"schema", "cubutterfly-b200-mapping-v1"},
                           {"family", d.op == CUBUTTERFLY_OPERATOR_NTT ? "bluestein-ntt" : "bluestein"},
                           {"axes", axes}});
        } else if (d.length_mode == CUBUTTERFLY_LENGTH_ZERO_EXTENDED_EMBEDDING) {
            cubf::Descriptor c = d;
            std::size_t pn = 1;
            while (pn < d.extents[0]) pn <<= 1;
            c.length_mode = CUBUTTERFLY_LENGTH_STANDARD;
            c.extents = {pn};
            c.input_strides = c.output_strides = {1};
            c.input_batch_stride = c.output_batch_stride = pn;
            c.placement = CUBUTTERFLY_PLACEMENT_IN_PLACE;
            c.algorithm_policy = CUBUTTERFLY_ALGORITHM_DEFAULT;
            c.explicit_algorithm.clear();
            c = cubf::normalize(c);
            cubf::Json axes = cubf::Json::array();
            axes.push_back({{"length", pn}, {"outer", d.batch}, {"inner", 1},
                            {"mapping", cubf::enumerate_mappings(make_request(c), hw).front().to_json()}});
            out.push_back({{"schema", "cubutterfly-b200-mapping-v1"}, {"family", "zero-extended"}, {"axes", axes}});
        } else if (d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type != CUBUTTERFLY_FFT_C2C && d.rank > 1) {
            const cubf::Descriptor r = real_rows(d), c = real_outer(d);
            cubf::Json axes = cubf::Json::array();
            axes.push_back({{"length", d.extents.back()}, {"outer", r.batch}, {"inner", 1},
                            {"mapping", cubf::enumerate_mappings(make_request(real_child(r)), hw).front().to_json()}});
            bool flat = false;
            for (const auto& a : composite_axes(c, flat, true)) {
                const cubf::Descriptor ca = cubf::normalize(a.d);
                axes.push_back({{"length", a.n}, {"outer", a.outer}, {"inner", a.inner}, {"mapping", child_mapping(ca)}});
            }
            out.push_back({{"schema", "cubutterfly-b200-mapping-v1"},
                           {"family", d.fft_type == CUBUTTERFLY_FFT_R2C ? "fft-r2c" : "fft-c2r"},
                           {"axes", axes}});
        } else if (d.op == CUBUTTERFLY_OPERATOR_FFT && d.fft_type != CUBUTTERFLY_FFT_C2C) {
            const cubf::Descriptor c = real_child(d);
            cubf::Json axes = cubf::Json::array();
            axes.push_back({{"length", c.extents[0]}, {"outer", d.batch}, {"inner", 1},
                            {"mapping", cubf::enumerate_mappings(make_request(c), hw).front().to_json()}});
            out.push_back({{"schema", "cubutterfly-b200-mapping-v1"},
                           {"family", d.fft_type == CUBUTTERFLY_FFT_R2C ? "fft-r2c" : "fft-c2r"},
                           {"axes", axes}});
        } else if (d.rank == 1) {
            for (const auto& m : cubf::enumerate_mappings(make_request(d), hw)) out.push_back(m.to_json());
        } else {
            // a composite: the best mapping of every child, in execution order
            bool flat = false;
            cubf::Json axes = cubf::Json::array();
            for (const auto& a : composite_axes(d, flat)) {
                const cubf::Descriptor c = cubf::normalize(a.d);
                axes.push_back({{"length", a.n}, {"outer", a.outer}, {"inner", a.inner}, {"mapping", child_mapping(c)}});
            }
            out.push_back({{"schema", "cubutterfly-b200-mapping-v1"}, {"family", "composite"}, {"flat", flat},
                           {"axes", axes}});
        }
        copy_text(out.dump(), json, bytes);
    });
}

}  // extern "C"
