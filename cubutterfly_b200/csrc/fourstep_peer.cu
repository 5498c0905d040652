// fourstep_peer.cu -- the data movement of the distributed four-step FFT done
// by kernels that store straight into the other ranks' buffers.
//
// The four-step transform (N = N1 x N2 over P ranks, rank r holding rows
// r N1/P .. of the row-major N1 x N2 matrix; n1p = N1/P, n2p = N2/P) has three
// all-to-all exchanges.  Each exchange here is one kernel that reads this
// rank's local data once and writes every element to its final place in the
// destination rank's buffer: buffers of other GPUs are CUDA IPC mappings
// (cudaIpcOpenMemHandle) reached over NVLink by ordinary stores, so the
// permutes, the twiddle multiply and the final transpose around the exchanges
// cost no separate pass.  No loads from peer memory, no multicast.
//
//   scatter_columns:   x[i][q n2p + j]                -> block_q[(r n1p + i) n2p + j]
//   scatter_rows:      spec[k1][j] W_N^(k1 (r n2p + j)) -> rows_q[i N2 + r n2p + j],  k1 = q n1p + i
//   scatter_transpose: out[i][q n2p + j]              -> result_q[j N1 + r n1p + i]
//
// Each also runs on a part -- columns [c0, c0 + w) of every rank's block, or
// rows [i0, i0 + m) of `out` -- so the exchanges can be pipelined against the
// FFT stages: a column part of the block is laid out as its own N1 x w
// matrix at element offset c0 N1 (a complete interleaved batch for the
// column FFT), and a column part of spec is N1 x w.
//
// A rank may start reading a buffer that peers wrote only after every rank's
// kernel has finished (the caller orders them with a collective).
#include <cubutterfly/cubutterfly_b200.h>

#include "fft.cuh"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

namespace cubf {
void set_last_error(const std::string& message);
fft::OuterTwiddles fourstep_twiddle_tables(int log_n);  // fourstep.cu
}

namespace {

constexpr int kMaxRanks = 8;

struct PeerPtrs {
    float2* p[kMaxRanks];
};

// One CTA per (row i, destination q) run of w values, 16-byte moves: columns
// [c0, c0 + w) of destination q's block, stored as the part's N1 x w matrix.
__global__ void scatter_columns_kernel(const float4* __restrict__ x, PeerPtrs dest, int ranks, int rank, size_t n1p,
                                       size_t n2p, size_t c0, size_t w) {
    const size_t runs = n1p * static_cast<size_t>(ranks);
    const size_t w4 = w / 2, n1 = n1p * static_cast<size_t>(ranks);
    for (size_t run = blockIdx.x; run < runs; run += gridDim.x) {
        const size_t i = run / ranks;
        const int q = static_cast<int>(run % ranks);
        const float4* src = x + ((i * ranks + q) * n2p + c0) / 2;
        float4* dst = reinterpret_cast<float4*>(dest.p[q]) + (c0 * n1 + (static_cast<size_t>(rank) * n1p + i) * w) / 2;
        for (size_t t = threadIdx.x; t < w4; t += blockDim.x) dst[t] = __ldcs(src + t);
    }
    __threadfence_system();  // this thread's peer stores are visible system-wide
}

// A warp covers 64 consecutive columns of one spec row per step and walks
// `steps` steps along the row; twiddles start from the fp64 tables and advance
// by W^(64 k1) in fp64 (one rounding each).  spec (the part) is N1 x w,
// w >= 64; its column j is column c0 + j of this rank's N2/P.
__global__ void scatter_rows_kernel(const float4* __restrict__ spec, PeerPtrs dest, int rank, size_t n1,
                                    size_t n1p, size_t n2p, int log_w, size_t c0, size_t n2, int log_n,
                                    cubf::fft::OuterTwiddles tw, int conj, int steps) {
    const size_t nmask = (size_t{1} << log_n) - 1;
    const size_t w = size_t{1} << log_w;
    const int lane = threadIdx.x & 31;
    const size_t warps_per_row = (w >> 6) / static_cast<size_t>(steps);
    const size_t ranks = n1 / n1p;
    const size_t items = n1 * warps_per_row, grid_warps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
    for (size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; warp < items;
         warp += grid_warps) {
    // rows taken round-robin over the destination ranks, so the CTAs in
    // flight write to every rank at once (local HBM and NVLink together)
    const size_t slot = warp / warps_per_row;
    const size_t k1 = (slot % ranks) * n1p + slot / ranks;
    const size_t j0 = (warp % warps_per_row) * static_cast<size_t>(steps) * 64 + 2 * static_cast<size_t>(lane);
    const size_t col = static_cast<size_t>(rank) * n2p + c0 + j0;  // n2 index of this thread's first value
    double2 wa = cubf::fft::outer_twiddle_d(tw, (k1 * col) & nmask);
    double2 wb = cubf::fft::outer_twiddle_d(tw, (k1 * (col + 1)) & nmask);
    const double2 step = cubf::fft::outer_twiddle_d(tw, (k1 * 64) & nmask);
    const double sgn = conj ? -1.0 : 1.0;
    const int q = static_cast<int>(k1 / n1p);
    const size_t i = k1 % n1p;
    const float4* s = spec + ((k1 << log_w) + j0) / 2;
    float4* d = reinterpret_cast<float4*>(dest.p[q]) + (i * n2 + col) / 2;
    // four steps' loads in flight before their multiplies and peer stores
    for (int t0 = 0; t0 < steps; t0 += 4) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = t0 + u < steps ? __ldcs(s + 32 * (t0 + u)) : make_float4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (t0 + u >= steps) break;
            const float2 a = cubf::fft::cmul(make_float2(v[u].x, v[u].y),
                                             make_float2(static_cast<float>(wa.x), static_cast<float>(sgn * wa.y)));
            const float2 b = cubf::fft::cmul(make_float2(v[u].z, v[u].w),
                                             make_float2(static_cast<float>(wb.x), static_cast<float>(sgn * wb.y)));
            d[32 * (t0 + u)] = make_float4(a.x, a.y, b.x, b.y);
            wa = cubf::fft::cmul_d(wa, step);
            wb = cubf::fft::cmul_d(wb, step);
        }
    }
    }
    __threadfence_system();
}

// Tiles of 128 values along i by 32 along k2 through shared memory: read as
// 256-byte row segments of `out` (n1p x n2, row-major), written as 32 runs of
// 128 consecutive i (1 KiB each) in the destination shard -- long runs keep
// the writes that cross NVLink and land in the peer's HBM efficient.  A tile
// lies in one destination block (n2p a multiple of 32).
constexpr int kTileI = 128, kTileK = 32;
__global__ void __launch_bounds__(256) scatter_transpose_kernel(const float2* __restrict__ out, PeerPtrs dest,
                                                                int rank, size_t n1, size_t n1p, size_t n2p,
                                                                size_t n2, size_t row0, size_t row_tiles) {
    __shared__ float2 tile[kTileI][kTileK + 1];
    const size_t ranks = n2 / n2p, per_rank = n2p / kTileK, tx = n2 / kTileK;
    const size_t tiles = tx * row_tiles;
    const int x = threadIdx.x & 31, y = threadIdx.x >> 5;  // 32 x 8
    for (size_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        // column tiles taken round-robin over the destination ranks (adjacent
        // tiles write to different ranks)
        const size_t bx = t % tx, by = t / tx;
        const size_t ct = (bx % ranks) * per_rank + bx / ranks;
        const size_t i0 = row0 + by * kTileI, c0 = ct * kTileK;
        __syncthreads();  // the previous tile's reads of `tile` are done
#pragma unroll
        for (int r = 0; r < kTileI; r += 8) tile[r + y][x] = __ldcs(out + (i0 + r + y) * n2 + c0 + x);
        __syncthreads();
        const int q = static_cast<int>(c0 / n2p);
        const size_t jb = c0 % n2p;
        const int i = threadIdx.x & (kTileI - 1), half = threadIdx.x >> 7;  // two destination rows per pass
        float2* d = dest.p[q] + static_cast<size_t>(rank) * n1p + i0 + i;
#pragma unroll
        for (int k = 0; k < kTileK; k += 2) d[(jb + k + half) * n1] = tile[i][k + half];
    }
    __threadfence_system();
}

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

bool pow2(std::size_t v) { return v != 0 && (v & (v - 1)) == 0; }
// CTAs per SM of a scatter launch: the caller's bound (a pipelined schedule
// leaves room for a concurrent FFT stage), else 8 (the whole GPU).
int per_sm(int ctas_per_sm) {
    if (ctas_per_sm < 0 || ctas_per_sm > 32) throw std::invalid_argument("ctas_per_sm must be 0 (default) .. 32");
    return ctas_per_sm ? ctas_per_sm : 8;
}
int log2_of(std::size_t v) {
    int l = 0;
    while ((std::size_t{1} << l) < v) ++l;
    return l;
}

// Shared checks: P power of two in [2, 8], rank < P, shapes powers of two,
// every destination pointer non-null and 16-byte aligned.
PeerPtrs peers_of(void* const* dest, int ranks, int rank) {
    if (ranks < 2 || ranks > kMaxRanks || !pow2(static_cast<std::size_t>(ranks)) || rank < 0 || rank >= ranks)
        throw std::invalid_argument("peer scatter needs 2, 4 or 8 ranks and 0 <= rank < ranks");
    if (!dest) throw std::invalid_argument("peer scatter needs the destination pointers of every rank");
    PeerPtrs p{};
    for (int q = 0; q < ranks; ++q) {
        if (!dest[q] || reinterpret_cast<std::uintptr_t>(dest[q]) % 16)
            throw std::invalid_argument("peer scatter destinations must be non-null and 16-byte aligned");
        p.p[q] = static_cast<float2*>(dest[q]);
    }
    return p;
}

template <typename F>
cubutterflyStatus_t guarded(F&& f) {
    try {
        cubf::set_last_error("");
        f();
        return CUBUTTERFLY_STATUS_SUCCESS;
    } catch (const std::invalid_argument& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_INVALID_VALUE;
    } catch (const std::exception& e) {
        cubf::set_last_error(e.what());
        return CUBUTTERFLY_STATUS_CUDA_ERROR;
    }
}

}  // namespace

extern "C" cubutterflyStatus_t cubutterflyB200PeerBufferCreate(size_t bytes, void** ptr, void* ipc_handle) {
    return guarded([&] {
        if (!ptr || !ipc_handle || bytes == 0) throw std::invalid_argument("peer buffer needs bytes > 0 and outputs");
        void* p = nullptr;
        check(cudaMalloc(&p, bytes), "peer buffer allocation");
        cudaIpcMemHandle_t h;
        const cudaError_t e = cudaIpcGetMemHandle(&h, p);
        if (e != cudaSuccess) {
            cudaFree(p);
            check(e, "IPC handle of the peer buffer");
        }
        std::memcpy(ipc_handle, &h, sizeof(h));
        *ptr = p;
    });
}

extern "C" cubutterflyStatus_t cubutterflyB200PeerBufferOpen(const void* ipc_handle, void** ptr) {
    return guarded([&] {
        if (!ptr || !ipc_handle) throw std::invalid_argument("peer buffer open needs a handle and an output");
        cudaIpcMemHandle_t h;
        std::memcpy(&h, ipc_handle, sizeof(h));
        check(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "IPC open of a peer buffer");
    });
}

extern "C" cubutterflyStatus_t cubutterflyB200PeerBufferClose(void* ptr) {
    return guarded([&] {
        if (!ptr) throw std::invalid_argument("peer buffer close needs a pointer");
        check(cudaIpcCloseMemHandle(ptr), "IPC close of a peer buffer");
    });
}

extern "C" cubutterflyStatus_t cubutterflyB200PeerBufferDestroy(void* ptr) {
    return guarded([&] {
        if (!ptr) throw std::invalid_argument("peer buffer destroy needs a pointer");
        check(cudaFree(ptr), "peer buffer free");
    });
}

extern "C" cubutterflyStatus_t cubutterflyB200FourStepScatterColumns(const void* x, void* const* dest, int ranks,
                                                                    int rank, size_t n1, size_t n2, size_t c0,
                                                                    size_t width, int ctas_per_sm,
                                                                    cudaStream_t stream) {
    return guarded([&] {
        const PeerPtrs p = peers_of(dest, ranks, rank);
        const int k = per_sm(ctas_per_sm);
        if (!x || reinterpret_cast<std::uintptr_t>(x) % 16 || !pow2(n1) || !pow2(n2) ||
            n1 < static_cast<std::size_t>(ranks) || n2 < 2 * static_cast<std::size_t>(ranks))
            throw std::invalid_argument("column scatter needs an aligned source and power-of-two N1, N2 >= 2P");
        const std::size_t n1p = n1 / ranks, n2p = n2 / ranks;
        if (!pow2(width) || width < 2 || c0 % width || c0 + width > n2p)
            throw std::invalid_argument("column scatter part: power-of-two width >= 2 dividing c0, c0 + width <= N2/P");
        int dev = 0, sms = 0;
        check(cudaGetDevice(&dev), "current device");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
        const std::size_t runs = n1p * ranks;
        const std::size_t cap = static_cast<std::size_t>(sms) * static_cast<std::size_t>(k);
        const unsigned grid = static_cast<unsigned>(runs < cap ? runs : cap);
        scatter_columns_kernel<<<grid, 256, 0, stream>>>(static_cast<const float4*>(x), p, ranks, rank, n1p, n2p, c0,
                                                          width);
        check(cudaGetLastError(), "column scatter launch");
    });
}

extern "C" cubutterflyStatus_t cubutterflyB200FourStepScatterRows(const void* spec, void* const* dest, int ranks,
                                                                 int rank, size_t n1, size_t n2, size_t c0,
                                                                 size_t width, int inverse, int ctas_per_sm,
                                                                 cudaStream_t stream) {
    return guarded([&] {
        const PeerPtrs p = peers_of(dest, ranks, rank);
        const int k = per_sm(ctas_per_sm);
        if (!spec || reinterpret_cast<std::uintptr_t>(spec) % 16 || !pow2(n1) || !pow2(n2) ||
            n2 < 64 * static_cast<std::size_t>(ranks) || n1 < static_cast<std::size_t>(ranks))
            throw std::invalid_argument("row scatter needs an aligned source, power-of-two N1 >= P and N2 >= 64 P");
        const std::size_t n1p = n1 / ranks, n2p = n2 / ranks;
        if (!pow2(width) || width < 64 || c0 % width || c0 + width > n2p)
            throw std::invalid_argument("row scatter part: power-of-two width >= 64 dividing c0, c0 + width <= N2/P");
        const int log_n = log2_of(n1) + log2_of(n2);
        if (log_n > 40) throw std::invalid_argument("four-step length is limited to 2^40");
        const cubf::fft::OuterTwiddles ot = cubf::fourstep_twiddle_tables(log_n);
        const std::size_t chunks = width / 64;
        const int steps = static_cast<int>(chunks < 16 ? chunks : 16);
        const std::size_t warps = n1 * (chunks / static_cast<std::size_t>(steps));
        int dev = 0, sms = 0;
        check(cudaGetDevice(&dev), "current device");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
        const std::size_t cap = static_cast<std::size_t>(sms) * static_cast<std::size_t>(k);
        const std::size_t want = (warps * 32 + 255) / 256;
        const std::size_t blocks = want < cap ? want : cap;
        scatter_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            static_cast<const float4*>(spec), p, rank, n1, n1p, n2p, log2_of(width), c0, n2, log_n, ot, inverse ? 1 : 0,
            steps);
        check(cudaGetLastError(), "row scatter launch");
    });
}

extern "C" cubutterflyStatus_t cubutterflyB200FourStepScatterTranspose(const void* out, void* const* dest, int ranks,
                                                                      int rank, size_t n1, size_t n2, size_t row0,
                                                                      size_t rows, int ctas_per_sm,
                                                                      cudaStream_t stream) {
    return guarded([&] {
        const PeerPtrs p = peers_of(dest, ranks, rank);
        const int k = per_sm(ctas_per_sm);
        if (!out || !pow2(n1) || !pow2(n2) || n1 < kTileI * static_cast<std::size_t>(ranks) ||
            n2 < kTileK * static_cast<std::size_t>(ranks))
            throw std::invalid_argument("transpose scatter needs power-of-two N1 >= 128 P and N2 >= 32 P");
        const std::size_t n1p = n1 / ranks, n2p = n2 / ranks;
        if (rows == 0 || rows % kTileI || row0 % kTileI || row0 + rows > n1p)
            throw std::invalid_argument("transpose scatter part: rows and row0 multiples of 128, row0 + rows <= N1/P");
        const std::size_t tiles = (n2 / kTileK) * (rows / kTileI);
        int dev = 0, sms = 0;
        check(cudaGetDevice(&dev), "current device");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
        const std::size_t cap = static_cast<std::size_t>(sms) * static_cast<std::size_t>(k);
        scatter_transpose_kernel<<<static_cast<unsigned>(tiles < cap ? tiles : cap), 256, 0, stream>>>(
            static_cast<const float2*>(out), p, rank, n1, n1p, n2p, n2, row0, rows / kTileI);
        check(cudaGetLastError(), "transpose scatter launch");
    });
}
