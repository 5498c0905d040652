// fwht_tc.cu -- FWHT of 4096-point bf16 rows on the 5th-generation tensor
// cores (tcgen05.mma, accumulators in tensor memory).
//
// H_4096 = H_64 (x) H_64 on the index i = a + 64 b: two dense contractions
// against the 64 x 64 Hadamard matrix (entries +-1, exact in bf16).  Two rows
// form one M = 128 tile (row r of the pair, 64 vectors each):
//
//   stage 1  A1[m = a + 64 r][k = b] = x_r[a + 64 b]     bf16, straight from
//            HBM (MN-major: 8 consecutive a share one 16-byte chunk, so the
//            row's 16-byte chunks land in the canonical layout with cp.async)
//            D1 = A1 . H_64  (128 x 64 fp32 in TMEM)      -- H along b
//   stage 2  A2[m' = b' + 64 r][k = a] = D1[a + 64 r][b']  split into
//            bf16 hi + lo (x = hi + lo to 2^-18 relative), written by the
//            thread that owns TMEM lane a + 64 r as 16-byte chunks of 8
//            consecutive b'
//            D2 = A2hi . H_64 + A2lo . H_64                -- H along a
//   output   thread of lane b' + 64 r holds out_r[a' + 64 b'], a' = 0..63:
//            64 consecutive elements, scaled, rounded once to bf16 and
//            stored as 16-byte vectors.
//
// The input is exact in bf16, so stage 1 is exact up to fp32 accumulation;
// stage 2's hi/lo split keeps ~18 significant bits, so results agree with the
// FP32 FINAL_STORAGE contract (widen, FP32 FWHT, scale, round once) except
// for rare last-bit differences.  One thread issues the MMAs; completion is
// signalled through an mbarrier by tcgen05.commit.  Every wait is bounded:
// on expiry the CTA records an error, stops, and still frees its TMEM.
//
// Per 128-thread group: two A1 buffers (the next pair's rows stream in with
// cp.async while the current pair computes; a consumed A1 buffer then holds
// the stage-2 hi operand) and the lo operand / output staging buffer, 50 KiB,
// plus 64 TMEM columns; one CTA of four groups per SM (H_64 is shared).
#include "common.cuh"
#include "f32x2.cuh"
#include "kernels.hpp"
#include "launch_util.cuh"

#include <cstdint>

namespace cubf::fwht_tc {
namespace {

// Kernels that allocate tensor memory get one resident CTA per SM, so one CTA
// runs kGroups independent 128-thread groups (named barriers, their own
// buffers, mbarrier and 64 TMEM columns), each streaming its own row pairs.
constexpr int kGroups = 4;
constexpr int kGroupThreads = 128;
constexpr int kThreads = kGroups * kGroupThreads;
constexpr int kN = 4096;
constexpr uint32_t kTileBytes = 128 * 64 * 2;  // one M = 128, K = 64 bf16 operand
// Operand layouts: the canonical 128-byte-swizzled forms (1 KiB atoms of 8
// rows x 128 bytes, 16-byte chunk c of row j stored at chunk c ^ j), which
// the tensor core reads without bank conflicts.
//   A (MN-major): atom rows are K, each row 64 consecutive M values; K atoms
//   at kSBO, M atoms (64 rows) at kLBO:
//     (m, k) -> (m / 64) kLBO + (k / 8) kSBO + (k % 8) 128 + (((m % 64) / 8) ^ (k % 8)) 16 + (m % 8) 2
//   B = H_64 (K-major): atom rows are N, each row the 64 K values; N atoms at 1 KiB:
//     (n, k) -> (n / 8) 1024 + (n % 8) 128 + ((k / 8) ^ (n % 8)) 16 + (k % 8) 2
constexpr uint32_t kSBO = 1024;
constexpr uint32_t kLBO = 8192;
constexpr uint32_t kBSBO = 1024;
constexpr uint32_t kSwizzle128 = 2;  // descriptor layout type
// Output staging: 64 segments of 128 bytes per row at a 144-byte pitch.
constexpr uint32_t kStagePitch = 144;
constexpr uint32_t kStageRow = 64 * kStagePitch;
constexpr uint32_t kStageBytes = 2 * kStageRow;  // >= kTileBytes: also the lo operand
static_assert(kStageBytes >= kTileBytes, "the lo buffer holds an operand");
constexpr uint32_t kGroupCols = 128;  // two 64-column accumulators: pair k and pair k + 1
constexpr uint32_t kTmemCols = 512;   // power of two >= kGroups * kGroupCols
static_assert(kGroups * kGroupCols <= kTmemCols, "TMEM columns");
// Instruction descriptor: D f32 (bits 4-5 = 1), A and B bf16 (7-9, 10-12 = 1),
// A MN-major (bit 15), B K-major, N = 64 (bits 17-22 = N >> 3), M = 128
// (bits 24-28 = M >> 4).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kSpinLimit = 1u << 22;

// a1[k & 1] holds pair k's rows, then (dead after stage 1) its stage-2 hi
// operand; lo holds the lo operand and then the output staging.
struct GroupSmem {
    alignas(1024) uint8_t a1[2][kTileBytes];
    alignas(1024) uint8_t lo[kStageBytes];
    alignas(8) unsigned long long mbar[2];  // [0]: stage-1 MMAs done, [1]: stage-2 MMAs done
    uint32_t abort;
};
struct Smem {
    GroupSmem g[kGroups];
    alignas(1024) uint8_t b[64 * 64 * 2];
    uint32_t tmem_base;
};


// Failure report to the plan's status word (mapped pinned host memory): a
// plain system-visible store, not an atomic -- atomics on mapped host memory
// are not atomic from the host's side, and any nonzero value is a failure.
CUBF_DEV void record_status(unsigned int* status, unsigned int code) {
    if (status == nullptr) return;
    *reinterpret_cast<volatile unsigned int*>(status) = code;
    __threadfence_system();
}

CUBF_DEV uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// Shared-memory matrix descriptor: start, leading and stride byte offsets
// (16-byte units), version 1, base offset 0 (atoms 1 KiB aligned), 128-byte swizzle.
CUBF_DEV uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           (static_cast<uint64_t>(kSwizzle128) << 61);
}
CUBF_DEV uint32_t a_chunk(uint32_t m, uint32_t k) {  // byte offset of the chunk holding (m .. m + 7, k)
    return (m >> 6) * kLBO + (k >> 3) * kSBO + (k & 7) * 128 + ((((m & 63) >> 3) ^ (k & 7)) << 4);
}

CUBF_DEV void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

CUBF_DEV void mma_commit(uint32_t mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
                 : "memory");
}

CUBF_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CUBF_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
CUBF_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bounded wait on an mbarrier phase; false when the limit expired.
CUBF_DEV bool mbar_wait(uint32_t mbar, uint32_t phase) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, P1;\n\t}"
            : "=r"(done)
            : "r"(mbar), "r"(phase)
            : "memory");
        if (done) return true;
    }
    return false;
}

CUBF_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
CUBF_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

CUBF_DEV uint32_t pack_bf16(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Stage the 16-byte chunks of rows 2p, 2p+1 into A1 (zeros past the last row).
CUBF_DEV void load_pair(const __nv_bfloat16* in, size_t rows, size_t pair, uint8_t* a1, int lt) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const int q = lt + kGroupThreads * c;  // chunk of the pair, 0..1023
        const int r = q >> 9, g = q & 511;
        const size_t row = 2 * pair + r;
        const bool ok = row < rows;
        const __nv_bfloat16* src = in + (ok ? row : 0) * kN + g * 8;
        // element a + 64 b: chunk g holds a = 8 (g % 8) .. +7 of b = g / 8; m = a + 64 r, k = b
        const uint32_t dst = smem_addr(a1) + a_chunk(8 * (g & 7) + 64 * r, g >> 3);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
                     : "memory");
    }
}

// Barrier of one 128-thread group (ids 1..kGroups; 0 is __syncthreads).
CUBF_DEV void group_sync(int g) { asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kGroupThreads) : "memory"); }

__global__ void __launch_bounds__(kThreads, 1)
    fwht4096_tc_kernel(const __nv_bfloat16* in, __nv_bfloat16* out, size_t rows, float scale,
                       unsigned int* status) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int grp = tid / kGroupThreads, lt = tid % kGroupThreads;
    GroupSmem& gs = sm.g[grp];
    // the swizzle acts on absolute shared-memory address bits: atoms must be 1 KiB aligned
    const size_t pairs = (smem_addr(smem_raw) & 1023u) ? 0 : (rows + 1) / 2;
    if (pairs == 0 && rows != 0 && tid == 0) record_status(status, 2u);

    const size_t first = static_cast<size_t>(blockIdx.x) * kGroups + grp;
    const size_t stride = static_cast<size_t>(gridDim.x) * kGroups;
    // the first two pairs stream in while the CTA sets up
    if (first < pairs) load_pair(in, rows, first, gs.a1[0], lt);
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (first + stride < pairs) load_pair(in, rows, first + stride, gs.a1[1], lt);
    asm volatile("cp.async.commit_group;" ::: "memory");

    // H_64 as the K-major B operand, shared by the groups
    for (int e = tid; e < 64 * 64; e += kThreads) {
        const int n = e >> 6, k = e & 63;
        const float h = (__popc(n & k) & 1) ? -1.f : 1.f;
        *reinterpret_cast<__nv_bfloat16*>(sm.b + (n >> 3) * kBSBO + (n & 7) * 128 + (((k >> 3) ^ (n & 7)) << 4) +
                                          (k & 7) * 2) = __float2bfloat16(h);
    }
    const uint32_t mbar1 = smem_addr(&gs.mbar[0]), mbar2 = smem_addr(&gs.mbar[1]);
    if (lt == 0) {
        gs.abort = 0;
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mbar1) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mbar2) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&sm.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_proxy_async();  // H_64 stores visible to the tensor core
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sm.tmem_base + grp * kGroupCols;  // this group's two accumulators
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;  // this warp's TMEM lanes
    const uint32_t b_addr = smem_addr(sm.b);
    const int r = lt >> 6;   // row of the pair owned by this thread's TMEM lane
    const int lm = lt & 63;  // a (stage 1) or b' (stage 2)
    uint32_t ph1 = 0, ph2 = 0;

    // Pipeline per group: while pair k's stage-2 MMAs run, pair k+1's rows
    // (loaded one pair ahead) go through their stage-1 MMAs into the other
    // accumulator; pair k+2's rows stream into pair k's buffer once its
    // stage-2 MMAs have read it.
    auto issue_stage1 = [&](int buf, uint32_t d) {
        const uint32_t a = smem_addr(gs.a1[buf]);
#pragma unroll
        for (int s = 0; s < 4; ++s)
            mma_bf16(d, smem_desc(a + 2 * s * kSBO, kLBO, kSBO), smem_desc(b_addr + 32 * s, 16, kBSBO), s > 0);
        mma_commit(mbar1);
    };
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // the first pair has landed
    fence_proxy_async();
    group_sync(grp);
    if (first < pairs && lt == 0) {
        fence_after_sync();
        issue_stage1(0, tmem);
    }
    int k = 0;
    for (size_t pair = first; pair < pairs; pair += stride, ++k) {
        const int buf = k & 1;
        const uint32_t d = tmem + 64 * buf, dn = tmem + 64 * (buf ^ 1);

        // ---- stage-1 results of pair k -> stage-2 operands ----
        if (!mbar_wait(mbar1, ph1)) gs.abort = 1;
        ph1 ^= 1;
        fence_after_sync();
        uint8_t* hi = gs.a1[buf];  // pair k's rows are consumed: its stage-2 hi operand goes here
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            uint32_t v[2][16];
            tmem_ld16(d + lane_off + 32 * half, v[0]);
            tmem_ld16(d + lane_off + 32 * half + 16, v[1]);
            tmem_wait_ld();
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                const int q = 2 * half + qq;
                // columns b' = 16 q .. 16 q + 15 of lane a + 64 r -> A2 rows b' + 64 r, k = a
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float x0 = __uint_as_float(v[qq][8 * h + 2 * e]);
                        const float x1 = __uint_as_float(v[qq][8 * h + 2 * e + 1]);
                        hw[e] = pack_bf16(x0, x1);
                        // exact residuals x - hi (one packed subtract), rounded once
                        const f32x2::P res = f32x2::sub2(f32x2::pk(x0, x1), f32x2::pk(__uint_as_float(hw[e] << 16),
                                                                                      __uint_as_float(hw[e] & 0xffff0000u)));
                        float l0, l1;
                        f32x2::up(res, l0, l1);
                        lw[e] = pack_bf16(l0, l1);
                    }
                    const uint32_t off = a_chunk(16 * q + 8 * h + 64 * r, lm);  // rows b' .. b' + 7, k = a
                    *reinterpret_cast<uint4*>(hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(gs.lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                }
            }
        }
        fence_proxy_async();
        fence_before_sync();
        group_sync(grp);
        if (gs.abort) break;

        // ---- stage 2 of pair k: D = A2hi . H_64 + A2lo . H_64 (H along a) ----
        if (lt == 0) {
            fence_after_sync();
            const uint32_t ah = smem_addr(hi), al = smem_addr(gs.lo);
#pragma unroll
            for (int s = 0; s < 4; ++s)
                mma_bf16(d, smem_desc(ah + 2 * s * kSBO, kLBO, kSBO), smem_desc(b_addr + 32 * s, 16, kBSBO), s > 0);
#pragma unroll
            for (int s = 0; s < 4; ++s)
                mma_bf16(d, smem_desc(al + 2 * s * kSBO, kLBO, kSBO), smem_desc(b_addr + 32 * s, 16, kBSBO), 1);
            mma_commit(mbar2);
        }
        // ---- stage 1 of pair k + 1 (rows landed one iteration ago) ----
        const bool more = pair + stride < pairs;
        if (more) {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            fence_proxy_async();
            group_sync(grp);
            if (lt == 0) {
                fence_after_sync();
                issue_stage1(buf ^ 1, dn);
            }
        }
        if (!mbar_wait(mbar2, ph2)) gs.abort = 1;
        ph2 ^= 1;
        fence_after_sync();
        // pair k's buffer is free: stream pair k + 2's rows into it
        if (pair + 2 * stride < pairs) load_pair(in, rows, pair + 2 * stride, gs.a1[buf], lt);
        asm volatile("cp.async.commit_group;" ::: "memory");
        {
            // lane b' + 64 r holds out_r[64 b' .. 64 b' + 63]: scale, round, and stage the
            // 128-byte segment at pitch kStagePitch (conflict-free), then copy the two
            // rows out with coalesced 16-byte loads and stores
            uint8_t* stage = gs.lo;  // free once stage 2 is done
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t v[2][16];
                tmem_ld16(d + lane_off + 32 * half, v[0]);
                tmem_ld16(d + lane_off + 32 * half + 16, v[1]);
                tmem_wait_ld();
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    uint32_t w[8];
                    const f32x2::P s2 = f32x2::pk(scale, scale);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        float y0, y1;
                        f32x2::up(f32x2::mul2(f32x2::pk(__uint_as_float(v[qq][2 * e]), __uint_as_float(v[qq][2 * e + 1])), s2),
                                  y0, y1);
                        w[e] = pack_bf16(y0, y1);
                    }
                    uint8_t* seg = stage + r * kStageRow + lm * kStagePitch + 32 * (2 * half + qq);
                    *reinterpret_cast<uint4*>(seg) = make_uint4(w[0], w[1], w[2], w[3]);
                    *reinterpret_cast<uint4*>(seg + 16) = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
            group_sync(grp);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = lt + kGroupThreads * i;  // 16-byte chunk of the pair, 0..1023
                const int rr = c >> 9, cc = c & 511;
                const size_t row = 2 * pair + rr;
                const uint4 w = *reinterpret_cast<const uint4*>(stage + rr * kStageRow + (cc >> 3) * kStagePitch +
                                                                (cc & 7) * 16);
                if (row < rows && !gs.abort) __stcs(reinterpret_cast<uint4*>(out + row * kN) + cc, w);
            }
        }
        fence_before_sync();
        group_sync(grp);  // staging read and TMEM reads done before they are overwritten
        if (gs.abort) break;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // no copy still in flight at exit
    if (gs.abort && lt == 0) {
        // bounded: let outstanding MMA batches drain before TMEM is freed
        mbar_wait(mbar1, ph1);
        mbar_wait(mbar2, ph2);
        record_status(status, 1u);
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sm.tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace
}  // namespace cubf::fwht_tc

namespace cubf {

bool fwht_tc_available(int log_n, BwType type) { return log_n == 12 && type == BwType::BF16; }

LaunchShape fwht_tc_shape() {
    LaunchShape s;
    s.threads = fwht_tc::kThreads;
    s.smem_bytes = static_cast<int>(sizeof(fwht_tc::Smem));
    s.units_per_cta = 2 * fwht_tc::kGroups;
    s.elems_per_thread = 64;
    s.exchanges = 1;
    return s;
}

cudaError_t launch_fwht_tc(const void* in, void* out, std::size_t rows, float scale, unsigned int* status,
                           cudaStream_t stream) {
    using namespace fwht_tc;
    static KernelSetup setup;
    int grid_cap = 0;
    const int smem = static_cast<int>(sizeof(Smem));
    cudaError_t e = setup_kernel(setup, fwht4096_tc_kernel, kThreads, smem, &grid_cap, true);
    if (e != cudaSuccess) return e;
    const std::size_t pairs = (rows + 1) / 2;
    if (pairs == 0) return cudaSuccess;
    const std::size_t want = (pairs + kGroups - 1) / kGroups;  // CTAs that have a pair for every group
    const std::size_t grid = want < static_cast<std::size_t>(grid_cap) ? want : static_cast<std::size_t>(grid_cap);
    fwht4096_tc_kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(
        static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), rows, scale, status);
    return cudaGetLastError();
}

}  // namespace cubf
