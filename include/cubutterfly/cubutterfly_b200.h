/*
 * cubutterfly_b200.h -- extensions of the B200 build beyond the reference ABI.
 *
 * Nothing here replaces a reference entry point; callers of the reference
 * header need none of it.  Symbols use the cubutterflyB200 prefix.
 */
#ifndef CUBUTTERFLY_B200_EXT_H
#define CUBUTTERFLY_B200_EXT_H

#include <cubutterfly/cubutterfly.h>

#ifdef __cplusplus
extern "C" {
#endif

/* CPU-only planner preview (no counterpart in the reference ABI; the
 * reference exposes its static ranking only through a Python subprocess,
 * scripts/rank_static_candidates.py).  Writes a JSON array of every legal
 * mapping of the descriptor, best first, as the DEFAULT policy would rank it
 * under `hardware_json` (a cubutterfly-b200-hardware-v1 object; NULL selects
 * the current device or the builtin B200 profile).  Two-call size protocol. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200RankMappings(cubutterflyDescriptor_t descriptor,
                                                              const char* hardware_json, char* json,
                                                              size_t* bytes);

/* Twiddle step of the four-step FFT (no counterpart in the reference ABI;
 * used by cubutterfly_b200.distributed for one transform split across GPUs).
 * data: `rows` x `cols` complex fp32, row-major, 16-byte aligned, cols a
 * power of two >= 2; multiplies element (i, j) by
 * W_n^((row_offset + i) (col_offset + j)), W_n = exp(-2 pi i/n) (conjugated
 * when `inverse`), with the twiddle formed in fp64 and rounded once.  The
 * first call per (device, n) uploads its tables. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200FourStepTwiddle(void* data, size_t rows, size_t cols,
                                                                 size_t row_offset, size_t col_offset, size_t n,
                                                                 int inverse, cudaStream_t stream);

/* Block permute of complex fp32 data (no counterpart in the reference ABI;
 * the four-step FFT's packing around its all-to-alls): output[b][a][:] =
 * input[a][b][:] for A x B blocks of C values (C even, buffers 16-byte
 * aligned, out of place).  If `input_self` is non-null, source block
 * a == self is read from input_self ([B][C]) instead; if `output_self` is
 * non-null, destination block b == self is written to output_self ([A][C]). */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PermuteBlocksC64(const void* input, const void* input_self,
                                                                  void* output, void* output_self, size_t self,
                                                                  size_t a, size_t b, size_t c,
                                                                  cudaStream_t stream);

/* Batched complex fp32 transpose (no counterpart in the reference ABI; the
 * four-step FFT's final reordering): output[b][c][r] = input[b][r][c] for
 * `batch` row-major rows x cols matrices, out of place, asynchronous on
 * `stream`; rows / 32 and batch at most 65535. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200TransposeC64(const void* input, void* output, size_t batch,
                                                              size_t rows, size_t cols, cudaStream_t stream);

/* Peer buffers and peer-store exchanges of the four-step FFT over P ranks
 * (no counterpart in the reference ABI; cubutterfly_b200.distributed with
 * transport "peer").  A rank allocates its exchange buffers with
 * cubutterflyB200PeerBufferCreate (device memory plus its 64-byte CUDA IPC
 * handle), sends the handles to the other ranks, which map them with
 * cubutterflyB200PeerBufferOpen (unmap: ...Close; free: ...Destroy).  The
 * scatter kernels then read this rank's data once and store every value
 * straight into its destination rank's buffer (dest[q], q < ranks; dest[rank]
 * is this rank's own buffer) over NVLink: ordinary stores, no loads from peer
 * memory.  N = n1 x n2 split over ranks = 2, 4 or 8 (n1p = n1/ranks,
 * n2p = n2/ranks, powers of two), this rank = `rank`; each call covers a part:
 * columns j in [c0, c0 + width) of N2/P (ScatterColumns, ScatterRows) or rows
 * i in [row0, row0 + rows) of n1p (ScatterTranspose); the whole exchange is
 * c0 = 0, width = n2p, or row0 = 0, rows = n1p:
 *   ScatterColumns:   x[i][q n2p + j] (n1p x n2)   -> dest[q][c0 n1 + (rank n1p + i) width + j - c0]
 *   ScatterRows:      spec[k1][j - c0] (n1 x width) times W_N^(k1 (rank n2p + j)), conjugated when
 *                     `inverse`                    -> dest[k1 / n1p][(k1 % n1p) n2 + rank n2p + j]
 *   ScatterTranspose: out[i][q n2p + j] (n1p x n2) -> dest[q][j n1 + rank n1p + i]
 * `ctas_per_sm` bounds the launch to that many CTAs per SM (0: 8, the whole
 * GPU), so a pipelined schedule can run an FFT stage beside it.
 * Every buffer holds N / ranks values, 16-byte aligned; ScatterTranspose needs
 * n1 >= 128 ranks, ScatterRows n2 >= 64 ranks.  A rank reads what
 * the others stored only after all of them finished (order them with a
 * collective). */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PeerBufferCreate(size_t bytes, void** ptr, void* ipc_handle);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PeerBufferOpen(const void* ipc_handle, void** ptr);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PeerBufferClose(void* ptr);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PeerBufferDestroy(void* ptr);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200FourStepScatterColumns(const void* x, void* const* dest, int ranks,
                                                                        int rank, size_t n1, size_t n2, size_t c0,
                                                                        size_t width, int ctas_per_sm,
                                                                        cudaStream_t stream);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200FourStepScatterRows(const void* spec, void* const* dest, int ranks,
                                                                     int rank, size_t n1, size_t n2, size_t c0,
                                                                     size_t width, int inverse, int ctas_per_sm,
                                                                     cudaStream_t stream);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200FourStepScatterTranspose(const void* out, void* const* dest,
                                                                          int ranks, int rank, size_t n1, size_t n2,
                                                                          size_t row0, size_t rows, int ctas_per_sm,
                                                                          cudaStream_t stream);

/* Device-side failure status of a plan (no counterpart in the reference ABI;
 * the reference's kernels never wait on the device).  The tensor-core FWHT
 * mapping waits on its own MMA completions with bounded waits; when one
 * expires the launch stops, frees its tensor memory and records bit 0 in the
 * plan's status word (bit 1: a launch invariant failed), and its output is
 * invalid.  The next cubutterflyExecute / ExecuteSteady on that plan returns
 * CUBUTTERFLY_STATUS_BACKEND_ERROR with the reason and clears the word.
 * GetDeviceStatus reads the word (plan and child plans, OR-ed) without
 * clearing or synchronising: it is final once the plan's stream has been
 * synchronised.  Plans of other mappings always read 0. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PlanGetDeviceStatus(cubutterflyPlan_t plan, unsigned int* bits);

/* Host-side test hook (no counterpart in the reference ABI): ORs `bits` into
 * the plan's device status word as a failing launch would, so that callers
 * can test their handling of the failure path without making a kernel fail.
 * CUBUTTERFLY_STATUS_NOT_SUPPORTED for plans without a status word. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PlanInjectDeviceStatus(cubutterflyPlan_t plan, unsigned int bits);

/* Integer roof of the NTT butterfly (no counterpart in the reference ABI;
 * a measurement aid).  Runs the forward lazy Cooley-Tukey butterfly of the
 * NTT tile passes (Shoup product, values in [0, 4q)) from registers on every
 * SM of the current device and writes the best rate seen, in butterflies per
 * second, to *per_second.  modulus in [3, 2^62).  Synchronous (about 0.1 s);
 * call it outside timed regions and stream capture. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200NttButterflyPeak(unsigned long long modulus, double* per_second);

/* Allocation-free complex fp32 FFT (no counterpart in the reference ABI).
 * For callers that cannot allocate device memory -- fixed memory budgets or
 * pools that own every byte, hosts that forbid cudaMalloc/cudaFree on their
 * threads, latency-critical paths -- and so cannot provide the workspace a
 * planned multi-pass FFT needs.  Runs the same multi-pass kernels as a
 * cubutterflyCreatePlan/Execute FFT (forward or inverse, optional 1/N,
 * natural order, in place when input == output) with scratch in a 16 MiB
 * device array inside the library: n a power of two in [2^14, 2^21],
 * n * batch <= 2^21 complex values; in place (input == output) up to
 * n = 2^20, n = 2^21 out of place only; input and output either equal or
 * disjoint.  Other sizes return CUBUTTERFLY_STATUS_INVALID_VALUE.  Pointers
 * 16-byte aligned.  Allocates nothing.  The first call on a device sets up
 * that device (symbol addresses, twiddle upload, a wait for the upload) and
 * should precede any stream capture.  Every call shares the scratch: calls that overlap on the GPU
 * race, so serialise them on one stream. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200FftC2CNoAlloc(const void* input, void* output, size_t n,
                                                               size_t batch, int inverse, int normalize,
                                                               cudaStream_t stream);

/* The HEonGPU NTT adapter (reference adapters/heongpu/ntt_adapter.hpp, C++
 * API in cubutterfly/heongpu/ntt_adapter.hpp) driven with plain pointers:
 * cubutterfly_heongpu::transform of `batch` negacyclic word64 polynomials of
 * 2^n_power coefficients.  Device arrays: moduli, modulus_count records of
 * three 64-bit words {value, bit, mu} (GPU-NTT's Modulus64); roots,
 * modulus_count tables of 2^n_power words whose entry bitrev(j) is psi^j
 * (forward) or psi^-j (inverse); mod_inverse, N^-1 per modulus (inverse
 * only); order (orderings 1 and 2).  ordering: 0 contiguous, 1 modulus
 * order, 2 polynomial order; execution: 0 one RNS plan (native-rns), 1 one
 * plan per modulus (grouped).  The first call of a request prepares plans
 * (device metadata reads, a stream synchronisation); later calls only
 * launch. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200HeongpuTransform(const uint64_t* input, uint64_t* output,
                                                                  const uint64_t* roots, const void* moduli,
                                                                  const uint64_t* mod_inverse, int n_power,
                                                                  int inverse, int batch, int modulus_count,
                                                                  int ordering, const int* order, int execution,
                                                                  cudaStream_t stream);
/* Adapter switches of the calling thread: clear_cache (non-zero) drops every
 * prepared plan and unfreezes; freeze 1 / 0 sets the frozen state (a plan
 * miss then fails instead of preparing), -1 leaves it; calls / polynomials
 * (optional) receive the counters, then reset_counters (non-zero) zeroes
 * them. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200HeongpuControl(int freeze, int clear_cache, int reset_counters,
                                                                size_t* calls, size_t* polynomials);

#ifdef __cplusplus
}
#endif

#endif /* CUBUTTERFLY_B200_EXT_H */
