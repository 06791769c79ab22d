// gemm_tc.cu -- F16-weight mul_mat on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the prefill-shaped mul_mat of the reference: matrix_mult_avx512
// (kernels/x86/matrix_mult_avx512.asm:118-282) behind simd_matmul_f16's convert-then-GEMM
// (src/simd/simd_matmul.cpp:428-480), and the upstream F16 path the hook actually falls back
// to for F16 weights (src/simd/ggml-cpu-simd.c:1314-1465: src1 narrowed to f16, then
// ggml_vec_dot_f16 with fp32 accumulation).
//
// Y[n][m] = sum_k W[m][k] * f16(X[n][k]) with W: M x K f16 (K contiguous), X: N x K f32,
// Y: N x M f32 (ggml dst layout).  Two launches per call:
//   1. narrow X to f16 into the workspace (the same round-to-nearest-even the reference's
//      F16 path applies to src1);
//   2. a persistent warp-specialised GEMM, one CTA per SM, output tile (128*MT) x BN:
//        warp 0   TMA producer: (128*MT)x64 W box + BNx64 X box per stage (128-byte
//                 swizzle, K-major), STAGES-deep mbarrier ring;
//        warp 1   MMA issuer (one thread): MT x tcgen05.mma.cta_group::1.kind::f16
//                 (M = 128, N = BN, K = 16) per K step, the MT M-tiles sharing the X tile,
//                 fp32 accumulators in TMEM; commits free smem stages and publish
//                 finished accumulators;
//        warps 2-9 epilogue: tcgen05.ld 32 lanes x 32 columns; each 32 x 32 block is
//                 written to a per-warp shared-memory staging buffer in Y's own order
//                 (32 consecutive m per column n) and stored with one TMA tensor store
//                 (cp.async.bulk.tensor, bulk group), so a warp's drain costs 32 shared
//                 stores per block instead of 32 global ones, and the TMEM accumulator is
//                 released as soon as it has been read.  Two warps per TMEM lane quarter
//                 split the columns.  Y without 16-byte alignment (and split-K partial
//                 tiles) take plain coalesced global stores.
//      When two accumulator sets fit in TMEM (2*MT*BN <= 512 columns) the epilogue of
//      tile t overlaps the MMAs of tile t+1.  MT = 2 (256 x 256 per SM) needs 64 KB of
//      operands per 1024 MMA cycles instead of 48 KB per 512 for 128 x 256, which is what
//      bounds this kernel (every TMA copy fills only its own CTA).  Every mbarrier wait is
//      bounded (MLZC_DEVERR_WAIT_TIMEOUT).
// Small tile counts split K across CTAs: each split stores its partial tile to the
// workspace and the split that finishes a tile last sums the partials in split order, so
// results are bitwise reproducible.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;                       // one 128-byte swizzle atom of f16
constexpr int kEpiWarps = 8;       // two warps per TMEM lane quarter, each draining half the columns
constexpr int kGemmThreads = 64 + kEpiWarps * 32;
constexpr int kSmemMax = 232448;             // dynamic shared memory per block (227 KB)
constexpr int kSmemFixed = 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kStgBytes = 32 * 32 * 4;  // one 32 x 32 f32 staging block of the epilogue

// ------------------------------------------------------------------ PTX wrappers

using ptx::bulk_load;
using ptx::global_ns;
using ptx::kWaitNs;
using ptx::mbar_arrive;
using ptx::mbar_expect_tx;
using ptx::mbar_init;
using ptx::mbar_try_wait;
using ptx::mbar_wait;
using ptx::smem_u32;

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Tiled TMA store of a box from shared memory into the current bulk group (committed by
// bulk_commit); elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N of this thread's bulk groups still read their shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// UMMA shared-memory descriptor of a K-major tile written by TMA with 128-byte swizzle:
// rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);   // start address        [0, 14)
    d |= (uint64_t)1 << 16;                     // leading byte offset  [16, 30) (unused: swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset   [32, 46): 8 rows x 128 B
    d |= (uint64_t)1 << 46;                     // descriptor version   [46, 48) = 1 on sm_100
    d |= (uint64_t)2 << 61;                     // layout: SWIZZLE_128B [61, 64)
    return d;
}

// Instruction descriptor, kind::f16: A = B = f16, D = f32, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4)                             // D format f32        [4, 6)
           | (0u << 7) | (0u << 10)              // A, B format f16     [7, 10), [10, 13)
           | (0u << 15) | (0u << 16)             // A, B K-major        15, 16
           | ((uint32_t)(N >> 3) << 17)          // N / 8               [17, 23)
           | ((uint32_t)(M >> 4) << 24);         // M / 16              [24, 29)
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// --------------------------------------------------------------------- kernels

// MT M-tiles of 128 rows share one BN-column X tile per stage: an SM computes a
// (128*MT) x BN output tile with MT UMMAs per K step.  The per-SM operand feed per MMA
// cycle falls with MT (48 KB per 512 MMA cycles for 128x256, 64 KB per 1024 for 256x256),
// which is what bounds this kernel with per-CTA operand loads.
template <int BN, int MT>
struct TileCfg {
    static constexpr int kRows = BM * MT;
    static constexpr uint32_t kABytes = (uint32_t)kRows * BK * 2;
    static constexpr uint32_t kBBytes = (uint32_t)BN * BK * 2;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    // epilogue staging: two blocks per warp when that still leaves three pipeline stages
    static constexpr int kStgBufs = (kSmemMax - kSmemFixed - 2 * kEpiWarps * (int)kStgBytes) / (int)kStageBytes >= 3 ? 2 : 1;
    static constexpr uint32_t kStgTotal = (uint32_t)kEpiWarps * kStgBufs * kStgBytes;
    static constexpr int kStagesFit = (kSmemMax - kSmemFixed - (int)kStgTotal) / (int)kStageBytes;
    static constexpr int kStages = kStagesFit > 12 ? 12 : kStagesFit;
    static constexpr int kAccCols = MT * BN;                           // one accumulator set
    static constexpr int kBufs = 2 * kAccCols <= 512 ? 2 : 1;          // double-buffered when TMEM allows
    static constexpr uint32_t kTmemCols = kBufs * kAccCols < 32 ? 32u
                                          : (kBufs * kAccCols <= 64 ? 64u
                                          : (kBufs * kAccCols <= 128 ? 128u
                                          : (kBufs * kAccCols <= 256 ? 256u : 512u)));
    static constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kStgTotal + kSmemFixed;
    static_assert(kStages >= 2, "pipeline needs two stages");
    static_assert(kSmemBytes <= (size_t)kSmemMax, "shared memory");
};

constexpr int kGemmMaxPeers = 7;   // other ranks of an 8-GPU row-sharded call

struct GemmArgs {
    float* y;
    size_t y_cs;          // bytes between output columns (tokens)
    int M, N, K;
    int num_m, num_n;     // tiles ((128*MT) x BN)
    int kblocks;          // BK blocks of the whole K
    int splits;           // K splits; > 1: partial tiles in `part`, the last split to finish sums them
    int num_work;         // num_m * num_n * splits
    const uint8_t* x16t;  // narrowed activations, one pre-swizzled BN x 64 block per (n-block, k-block)
    float* part;          // [splits][tiles][BN][128*MT] partial accumulators (splits > 1)
    int* tile_count;      // per tile: splits finished (zeroed by the narrowing kernel)
    unsigned int* err;
    int tma_store;        // 1: Y is written through tmY (16-byte aligned Y and column stride)
    // Row-sharded mul_mat: every finished tile also goes to this rank's slice in the slot of
    // the call's epoch parity of each other rank (peer memory over NVLink), so the exchange
    // overlaps the remaining tiles.  npeer = 0: a plain GEMM.
    int npeer;
    float* pslot[2][kGemmMaxPeers];   // [parity][peer]: the slice, [N][M] with column stride pcs
    size_t pcs;
    const uint32_t* epoch;            // this rank's last completed epoch (the call's is + 1)
    // Optional per-row output scale (powers of two from the quantised-weight path, whose
    // f16 rows may be stored scaled down); nullptr: none.
    const float* row_scale;
};

// The peers' slices as TMA store targets ([parity][peer], same box as tmY).
struct PeerMaps {
    CUtensorMap m[2][kGemmMaxPeers];
};

template <int BN, int MT>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmY,
                   const __grid_constant__ PeerMaps pm, GemmArgs g) {
    using C = TileCfg<BN, MT>;
    constexpr int STAGES = C::kStages;
    constexpr int NBUF = C::kBufs;
    constexpr int ROWS = C::kRows;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smA = smem;
    uint8_t* smB = smem + STAGES * C::kABytes;
    float* stg_all = reinterpret_cast<float*>(smem + STAGES * C::kStageBytes);   // epilogue staging
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::kStageBytes + C::kStgTotal);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    volatile int* last_flag = abort_flag + 1;   // "this CTA sums the current split tile"

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tfull[b]), 1);
            mbar_init(smem_u32(&tempty[b]), kEpiWarps);   // one arrival per epilogue warp
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        tma_prefetch_desc(&tmA);
        if (g.tma_store) tma_prefetch_desc(&tmY);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(C::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    // set-up above overlaps the previous kernel's tail; operands and outputs wait for it
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();

    const int tiles = g.num_m * g.num_n;
    const int kper = (g.kblocks + g.splits - 1) / g.splits;   // k-blocks per split
    auto work_coords = [&](int w, int& m0, int& n0, int& kb0, int& kb1) {
        const int tile = w % tiles;
        const int split = w / tiles;
        // N-tiles fastest: the CTAs in flight share each W tile (read from DRAM once per
        // round, by all its N-tiles together) and all of X stays in L2
        m0 = (tile / g.num_n) * ROWS;
        n0 = (tile % g.num_n) * BN;
        kb0 = split * kper;
        kb1 = min(kb0 + kper, g.kblocks);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            uint32_t it = 0;
            bool ok = true;
            for (int w = blockIdx.x; w < g.num_work && ok; w += gridDim.x) {
                int m0, n0, kb0, kb1;
                work_coords(w, m0, n0, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1, abort_flag, g.err)) { ok = false; break; }
                    const uint32_t fb = smem_u32(&full[s]);
                    mbar_expect_tx(fb, C::kStageBytes);
                    tma_load_2d(smem_u32(smA + s * C::kABytes), &tmA, fb, kb * BK, m0);
                    bulk_load(smem_u32(smB + s * C::kBBytes),
                              g.x16t + ((size_t)(n0 / BN) * g.kblocks + kb) * C::kBBytes, C::kBBytes, fb);
                }
            }
            if (!ok) {
                // let the copies already issued land before the CTA's smem goes away
                const uint32_t issued = it;
                for (uint32_t j = issued > (uint32_t)STAGES ? issued - STAGES : 0; j < issued; ++j) {
                    const uint64_t t0 = global_ns();
                    while (!mbar_try_wait(smem_u32(&full[j % STAGES]), (j / STAGES) & 1) && global_ns() - t0 < kWaitNs) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            constexpr uint32_t idesc = umma_idesc_f16(BM, BN);
            uint32_t it = 0, t = 0;
            bool ok = true;
            uint32_t last_commit_bar = 0, last_commit_parity = 0;
            for (int w = blockIdx.x; w < g.num_work && ok; w += gridDim.x, ++t) {
                int m0, n0, kb0, kb1;
                work_coords(w, m0, n0, kb0, kb1);
                const uint32_t b = NBUF == 2 ? (t & 1) : 0;
                const uint32_t aph = NBUF == 2 ? ((t >> 1) & 1) : (t & 1);
                if (!mbar_wait(smem_u32(&tempty[b]), aph ^ 1, abort_flag, g.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + b * C::kAccCols;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(smem_u32(&full[s]), ph, abort_flag, g.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = umma_desc_sw128(smem_u32(smA + s * C::kABytes));
                    const uint64_t bd = umma_desc_sw128(smem_u32(smB + s * C::kBBytes));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
#pragma unroll
                        for (int i = 0; i < MT; ++i) {
                            // M-tile i starts 128 rows (16 KB, = 1024 in the encoded address) later;
                            // +32 bytes along K inside the swizzle atom = +2 in the encoded address
                            umma_f16(d_tmem + i * BN, ad + (uint64_t)i * (BM * BK * 2 >> 4) + 2 * k, bd + 2 * k, idesc,
                                     (kb > kb0 || k > 0) ? 1u : 0u);
                        }
                    }
                    umma_commit(smem_u32(&empty[s]));
                    last_commit_bar = smem_u32(&empty[s]);
                    last_commit_parity = ph;
                }
                if (!ok) break;
                umma_commit(smem_u32(&tfull[b]));
            }
            if (!ok && last_commit_bar) {
                // wait (bounded) for the MMAs already issued before the TMEM is released
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(last_commit_bar, last_commit_parity) && global_ns() - t0 < kWaitNs) {
                }
            }
        }
    } else {
        // ---------------- epilogue: TMEM -> registers -> Y (or the split partials)
        const int quarter = warp & 3;            // TMEM lanes [32*quarter, 32*quarter + 32)
        constexpr int NSUB = kEpiWarps / 4;      // warps per TMEM lane quarter
        const int sub = (warp - 2) >> 2;         // which of them this warp is
        // columns per TMEM load: 32, or BN for the 16-wide tile; G loads are issued before
        // one wait, so the drain pays the TMEM load latency once per G x 32 columns
        constexpr int kCols = BN < 32 ? BN : 32;
        constexpr int kChunks = BN < 32 ? 1 : BN / 32;
        // chunk groups of G go round-robin to the NSUB warps of a quarter
        constexpr int G = kChunks >= 2 * NSUB ? 2 : 1;
        constexpr int NSTG = C::kStgBufs;
        float* stg = stg_all + (size_t)(warp - 2) * NSTG * (kStgBytes / 4);
        // TMA stores: full 32 x 32 blocks, whole tiles (no split partials)
        const bool tma_out = (kCols == 32) && g.tma_store && g.splits == 1;
        // the call's epoch parity (the previous call's wait kernel advanced the epoch before
        // this kernel's pdl_wait returned)
        const int par = g.npeer ? (int)((*reinterpret_cast<const volatile uint32_t*>(g.epoch) + 1) & 1) : 0;
        uint32_t nst = 0;                        // staging blocks this warp has stored
        uint32_t t = 0;
        for (int w = blockIdx.x; w < g.num_work; w += gridDim.x, ++t) {
            int m0, n0, kb0, kb1;
            work_coords(w, m0, n0, kb0, kb1);
            const uint32_t b = NBUF == 2 ? (t & 1) : 0;
            const uint32_t aph = NBUF == 2 ? ((t >> 1) & 1) : (t & 1);
            if (!mbar_wait(smem_u32(&tfull[b]), aph, abort_flag, g.err)) break;
            tc_fence_after();
            const int tile = w % tiles;
            const int split = w / tiles;
            float* mypart = g.part + ((size_t)split * tiles + tile) * (size_t)(ROWS * BN);
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                const int row = i * BM + quarter * 32 + lane;   // row of the tile this thread owns
                const int m = m0 + row;
                char* ybase = reinterpret_cast<char*>(g.y) + (size_t)m * 4;
                // whole tiles only (split partials are scaled in the fix-up below)
                const float rsc = (g.row_scale && g.splits == 1 && m < g.M) ? ptx::ld_act(g.row_scale + m) : 1.0f;
#pragma unroll 1
                for (int c0 = sub * G; c0 < kChunks; c0 += NSUB * G) {
                    uint32_t r[G][32];
                    // a group may run past the last chunk when kChunks is not a multiple of G:
                    // those chunks are neither loaded nor stored (they would be columns of
                    // the next accumulator and of the neighbouring tile)
#pragma unroll
                    for (int gg = 0; gg < G; ++gg)
                        if (c0 + gg < kChunks)
                            tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + b * C::kAccCols + i * BN +
                                          (c0 + gg) * 32,
                                      r[gg]);
                    tmem_ld_wait();
                    if (rsc != 1.0f) {
#pragma unroll
                        for (int gg = 0; gg < G; ++gg)
#pragma unroll
                            for (int j = 0; j < 32; ++j) r[gg][j] = __float_as_uint(__uint_as_float(r[gg][j]) * rsc);
                    }
#pragma unroll
                    for (int gg = 0; gg < G; ++gg) {
                        if (c0 + gg >= kChunks) continue;
                        const int c = (c0 + gg) * 32;
                        if (tma_out) {
                            // block (32 rows of this lane quarter x 32 columns) -> staging in
                            // Y's order (column-major over m), then one tensor store
                            float* buf = stg + (nst % NSTG) * (kStgBytes / 4);
                            if (nst >= (uint32_t)NSTG) {
                                if (lane == 0) bulk_wait_read<NSTG - 1>();
                                __syncwarp();
                            }
#pragma unroll
                            for (int j = 0; j < 32; ++j) buf[j * 32 + lane] = __uint_as_float(r[gg][j]);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                const int bx = m0 + i * BM + quarter * 32, by = n0 + c;
                                tma_store_2d(&tmY, smem_u32(buf), bx, by);
                                for (int r = 0; r < g.npeer; ++r) tma_store_2d(&pm.m[par][r], smem_u32(buf), bx, by);
                                bulk_commit();
                            }
                            ++nst;
                        } else if (g.splits == 1) {
                            if (m < g.M) {
#pragma unroll
                                for (int j = 0; j < kCols; ++j) {
                                    const int n = n0 + c + j;
                                    if (n < g.N) *reinterpret_cast<float*>(ybase + (size_t)n * g.y_cs) = __uint_as_float(r[gg][j]);
                                }
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < kCols; ++j) mypart[(size_t)(c + j) * ROWS + row] = __uint_as_float(r[gg][j]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tempty[b]));
            if (g.splits > 1) {
                // Deterministic split-K: the split that finishes a tile last sums all of the
                // tile's partials in split order 0..S-1 (no CTA ever waits for another).
                __threadfence();
                asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
                if (threadIdx.x == 64) {
                    const int done = atomicAdd(&g.tile_count[tile], 1);
                    *last_flag = (done == g.splits - 1) ? 1 : 0;
                }
                asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
                if (*last_flag) {
                    __threadfence();
                    // 4 consecutive rows per thread (one float4 per split and column), the
                    // epilogue's 128 threads spread over ROWS/4 row groups x the columns.
                    constexpr int RG = ROWS / 4;                 // row groups (32 or 64)
                    constexpr int CG = (kEpiWarps * 32) / RG;    // column phases (4 or 2)
                    const int et = threadIdx.x - 64;
                    const int r4 = (et % RG) * 4;
                    const int cg = et / RG;
                    const float* p0 = g.part + (size_t)tile * (ROWS * BN) + r4;
                    const size_t sstride = (size_t)tiles * (ROWS * BN);
                    const int ncols = min(BN, g.N - n0);
                    const int mrow = m0 + r4;
                    const bool vec_store = mrow + 3 < g.M && ((reinterpret_cast<uintptr_t>(g.y) | g.y_cs) % 16 == 0);
                    float rs4[4] = {1.0f, 1.0f, 1.0f, 1.0f};
                    if (g.row_scale && mrow < g.M)
                        for (int q = 0; q < 4 && mrow + q < g.M; ++q) rs4[q] = ptx::ld_act(g.row_scale + mrow + q);
                    if (mrow < g.M) {
#pragma unroll 1
                        for (int c = cg; c < ncols; c += 4 * CG) {
                            float4 acc[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                            for (int sp = 0; sp < g.splits; ++sp) {
                                float4 v[4];
#pragma unroll
                                for (int u = 0; u < 4; ++u) {
                                    const int cc = c + u * CG;
                                    v[u] = cc < ncols ? __ldcg(reinterpret_cast<const float4*>(p0 + sp * sstride + (size_t)cc * ROWS))
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                                }
#pragma unroll
                                for (int u = 0; u < 4; ++u) {
                                    acc[u].x += v[u].x; acc[u].y += v[u].y; acc[u].z += v[u].z; acc[u].w += v[u].w;
                                }
                            }
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                acc[u].x *= rs4[0]; acc[u].y *= rs4[1]; acc[u].z *= rs4[2]; acc[u].w *= rs4[3];
                            }
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int cc = c + u * CG;
                                if (cc >= ncols) continue;
                                float* dst = reinterpret_cast<float*>(reinterpret_cast<char*>(g.y) + (size_t)(n0 + cc) * g.y_cs) + mrow;
                                if (vec_store) {
                                    *reinterpret_cast<float4*>(dst) = acc[u];
                                } else {
                                    const float a4[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
                                    for (int q = 0; q < 4 && mrow + q < g.M; ++q) dst[q] = a4[q];
                                }
                                for (int r = 0; r < g.npeer; ++r) {
                                    // the slices are dense, 16-byte aligned [N][M] (M % 4 == 0)
                                    float* pd = reinterpret_cast<float*>(reinterpret_cast<char*>(g.pslot[par][r]) +
                                                                         (size_t)(n0 + cc) * g.pcs) + mrow;
                                    *reinterpret_cast<float4*>(pd) = acc[u];
                                }
                            }
                        }
                    }
                }
            }
        }
    }

    // the epilogue's tensor stores read shared memory until they complete
    if (warp >= 2 && lane == 0) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::kTmemCols)
                     : "memory");
    }
}

// X (N x K f32, column stride x_cs bytes) -> f16 (round-to-nearest-even) in the layout the
// GEMM's X stages use: one contiguous BN x 64 block per (n-block, k-block), rows of 128
// bytes with the 16-byte chunks XOR-swizzled by (row % 8) -- the image a 128-byte-swizzle
// TMA box would leave in shared memory, so each stage is a single bulk copy.  Rows past N
// and columns past K are zero.  Also zeroes the split-K tile counters.
__global__ void narrow_f16_kernel(const char* x, size_t x_cs, int N, int K, uint8_t* __restrict__ x16t,
                                  int BN, int num_n, int kblocks, int vec, int* __restrict__ tile_count, int ntiles) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // X may come from, and X16 / the counters be in use by, the previous kernel
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ntiles; i += gridDim.x * blockDim.x) tile_count[i] = 0;
    const int cpr = kblocks * 8;                          // 16-byte chunks per padded row
    const int64_t total = (int64_t)num_n * BN * cpr;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int n = (int)(i / cpr);
        const int ch = (int)(i % cpr);
        const int k0 = ch * 8;
        float v[8];
        if (n < N) {
            const float* xr = reinterpret_cast<const float*>(x + (size_t)n * x_cs);
            if (vec && k0 + 8 <= K) {
                const float4 a = ptx::ld_act(reinterpret_cast<const float4*>(xr + k0));
                const float4 b = ptx::ld_act(reinterpret_cast<const float4*>(xr + k0 + 4));
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = (k0 + e < K) ? ptx::ld_act(xr + k0 + e) : 0.0f;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = 0.0f;
        }
        uint4 o;
        __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
        __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
        o.x = *reinterpret_cast<uint32_t*>(&h0);
        o.y = *reinterpret_cast<uint32_t*>(&h1);
        o.z = *reinterpret_cast<uint32_t*>(&h2);
        o.w = *reinterpret_cast<uint32_t*>(&h3);
        const int nb = n / BN, r = n % BN, kb = ch / 8, c16 = ch % 8;
        const size_t off = (((size_t)nb * kblocks + kb) * BN + r) * 128 + (size_t)((c16 ^ (r & 7)) * 16);
        *reinterpret_cast<uint4*>(x16t + off) = o;
    }
}

// ------------------------------------------------------------------ host side

// 2-D f16 tensor map: rows of `inner` elements, `rows` rows `row_bytes` apart; box
// `box_rows` x 64 elements with 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return MLZC_OK;
}

// 2-D f32 tensor map of Y (ggml dst: N columns of M floats, y_cs bytes apart), 32 x 32
// boxes, no swizzle: the epilogue's staging blocks.
int make_y_map(CUtensorMap* map, float* y, uint64_t M, uint64_t N, uint64_t y_cs) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {M, N};
    const cuuint64_t strides[1] = {y_cs};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled (Y) failed (%d)", (int)r);
    return MLZC_OK;
}

struct GemmPlan {
    int MT, BN, num_m, num_n, kblocks, splits;
    size_t x16, counters, partials;   // workspace segments (bytes)
    size_t total() const { return x16 + counters + partials; }
};

// Measured cost of one work unit on B200 (SM clocks, 148 SMs), per tile shape (MT, BN):
// cycles per 64-deep k-block, and fixed cycles per unit (pipeline fill, and the epilogue
// drain where only one accumulator set fits in TMEM).  Least-squares fit over the
// Llama-3 projection shapes (3072x3072, 1024x3072, 8192x3072, 3072x8192) at 512 and 2048
// tokens, narrowing excluded.  Only shapes that won somewhere are candidates.  A K split
// also writes its partial tile and the last split reads them all back: priced at the
// store-bound drain rate (~10 bytes per cycle per SM).
struct ShapeCost {
    int mt, bn;
    double kb_cycles, unit_cycles;
};
constexpr ShapeCost kShapeCosts[] = {
    {2, 256, 1076.0, 31962.0}, {2, 192, 1119.0, 16248.0}, {1, 256, 561.0, 17288.0},
    {1, 128, 581.0, 5909.0},   {1, 96, 596.0, 8882.0},
};
constexpr double kSplitBytesPerCycle = 10.0;
// K splits for wide problems: few tiles over a long K (the row shards of the sharded FFN,
// e.g. 1024 x 28672 at 256 tokens) measured fastest with 4 to 8 splits.
constexpr int kMaxWideSplits = 8;

// Tile shape (MT M-tiles of 128 rows x BN columns per CTA) and K split for a problem.
// Wide problems (N >= 128) minimise rounds x measured unit cost over the candidates, with
// at most kMaxWideSplits K splits (a split's partial tile goes through the workspace); narrow ones
// (decode) use the narrowest BN that holds N and split K to occupy the SMs.
GemmPlan plan_gemm(int64_t M, int64_t K, int64_t N, int sm_count) {
    GemmPlan p{};
    p.kblocks = (int)((K + BK - 1) / BK);
    p.MT = 1;
    p.splits = 1;
    if (N >= 128) {
        double best = 1e300;
        for (const ShapeCost& sc : kShapeCosts)
            for (int sp = 1; sp <= kMaxWideSplits; ++sp) {
                if (sp > 1 && p.kblocks / sp < 4) break;
                const long tiles = (long)((M + BM * sc.mt - 1) / (BM * sc.mt)) * ((N + sc.bn - 1) / sc.bn);
                const long rounds = (tiles * sp + sm_count - 1) / sm_count;
                const int kper = (p.kblocks + sp - 1) / sp;
                const double split_io = sp > 1 ? 2.0 * sc.mt * BM * sc.bn * 4 / kSplitBytesPerCycle : 0.0;
                const double cost = (double)rounds * (kper * sc.kb_cycles + sc.unit_cycles + split_io);
                if (cost < best * 0.999) {
                    best = cost;
                    p.MT = sc.mt;
                    p.BN = sc.bn;
                    p.splits = sp;
                }
            }
    } else {
        p.BN = N <= 16 ? 16 : (N <= 32 ? 32 : (N <= 64 ? 64 : 128));
        const int tiles = (int)((M + BM - 1) / BM) * (int)((N + p.BN - 1) / p.BN);
        if (tiles * 2 <= sm_count) p.splits = std::max(1, std::min(sm_count / tiles, p.kblocks / 4));
    }
    p.num_m = (int)((M + BM * p.MT - 1) / (BM * p.MT));
    p.num_n = (int)((N + p.BN - 1) / p.BN);
    const int tiles = p.num_m * p.num_n;
    if (p.splits > 1) {
        // every split must own >= 1 k-block: an empty split would add a stale accumulator
        const int kper = (p.kblocks + p.splits - 1) / p.splits;
        p.splits = (p.kblocks + kper - 1) / kper;
    }
    p.x16 = ((size_t)p.num_n * p.BN * p.kblocks * BK * 2 + 255) / 256 * 256;
    p.counters = p.splits > 1 ? ((size_t)tiles * 4 + 255) / 256 * 256 : 0;
    p.partials = p.splits > 1 ? (size_t)p.splits * tiles * BM * p.MT * p.BN * 4 : 0;
    return p;
}

int current_sm_count() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;   // B200
    }
    return sms;
}

template <int BN, int MT>
int launch_tile(const DeviceCtx* c, const CUtensorMap& ta, const CUtensorMap& ty, const PeerMaps& pm, GemmArgs g,
                cudaStream_t s) {
    using Cfg = TileCfg<BN, MT>;
    static bool attr_set[64] = {};
    const int dev = c->device < 64 ? c->device : 63;
    if (!attr_set[dev]) {
        MLZC_CUDA_TRY(cudaFuncSetAttribute(gemm_f16_tc_kernel<BN, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)Cfg::kSmemBytes));
        attr_set[dev] = true;
    }
    const int grid = std::min(g.num_work, c->sm_count);
    MLZC_CUDA_TRY(launch_pdl(gemm_f16_tc_kernel<BN, MT>, dim3(grid), dim3(kGemmThreads), Cfg::kSmemBytes, s, ta, ty, pm, g));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

}  // namespace

size_t gemm_f16_workspace_bytes(int64_t M, int64_t K, int64_t N) { return plan_gemm(M, K, N, current_sm_count()).total(); }

bool gemm_f16_applicable(int64_t M, int64_t K, int64_t N, const void* w, size_t w_row_bytes, const float*, size_t,
                         const float*, size_t) {
    if (M < 1 || K < 1 || N < 1) return false;
    if ((uintptr_t)w % 16 != 0 || w_row_bytes % 16 != 0) return false;   // TMA base / stride rules
    if (M > (1ll << 31) - 1 || N > (1ll << 31) - 1 || K > (1ll << 31) - 1) return false;
    return true;
}

namespace {

int launch_gemm_f16_impl(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                         size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                         cudaStream_t s, const GemmPeers* peers, const float* row_scale) {
    const GemmPlan pl = plan_gemm(M, K, N, c->sm_count);
    const size_t need = pl.total();
    if (!ws || ws_bytes < need)
        return fail(MLZC_ERR_NOMEM, "mul_mat (tensor-core path): workspace of %zu bytes needed, %zu given", need, ws_bytes);
    char* wsc = static_cast<char*>(ws);
    uint8_t* x16t = reinterpret_cast<uint8_t*>(wsc);
    int* counters = reinterpret_cast<int*>(wsc + pl.x16);
    float* partials = reinterpret_cast<float*>(wsc + pl.x16 + pl.counters);
    const int tiles = pl.num_m * pl.num_n;
    {
        const int vec = ((uintptr_t)x % 16 == 0 && x_col_bytes % 16 == 0) ? 1 : 0;
        const int64_t total = (int64_t)pl.num_n * pl.BN * pl.kblocks * 8;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)c->sm_count * 8));
        MLZC_CUDA_TRY(launch_pdl(narrow_f16_kernel, dim3(grid), dim3(256), 0, s, reinterpret_cast<const char*>(x), x_col_bytes, (int)N, (int)K, x16t,
                                               pl.BN, pl.num_n, pl.kblocks, vec, counters, pl.splits > 1 ? tiles : 0));
        MLZC_CUDA_TRY(cudaGetLastError());
        count_launch();
    }
    const int BN = pl.BN;
    CUtensorMap ta;
    int st = make_map(&ta, w, (uint64_t)K, (uint64_t)M, w_row_bytes, (uint32_t)(BM * pl.MT));
    if (st != MLZC_OK) return st;

    GemmArgs g{};
    g.y = y;
    g.y_cs = y_col_bytes;
    g.M = (int)M;
    g.N = (int)N;
    g.K = (int)K;
    g.num_m = pl.num_m;
    g.num_n = pl.num_n;
    g.kblocks = pl.kblocks;
    g.err = c->err;
    g.splits = pl.splits;
    g.num_work = tiles * pl.splits;
    g.x16t = x16t;
    g.part = partials;
    g.tile_count = counters;
    g.row_scale = row_scale;
    // Y through TMA stores: base and column stride 16-byte aligned (the tensor-map rules)
    CUtensorMap ty;
    std::memset(&ty, 0, sizeof ty);
    g.tma_store = ((uintptr_t)y % 16 == 0 && y_col_bytes % 16 == 0 && pl.splits == 1 && pl.BN >= 32) ? 1 : 0;
    if (g.tma_store) {
        st = make_y_map(&ty, y, (uint64_t)M, (uint64_t)N, y_col_bytes);
        if (st != MLZC_OK) return st;
    }
    PeerMaps pm;
    std::memset(&pm, 0, sizeof pm);
    if (peers) {
        // tiles reach the peers through the TMA stores or the split fix-up; the plain
        // per-thread store path has no peer form
        if (!g.tma_store && pl.splits == 1) return fail(MLZC_ERR_UNSUPPORTED, "GEMM peer stores: Y not TMA-storable");
        if (peers->npeer > kGemmMaxPeers || M % 4 || peers->pcs % 16)
            return fail(MLZC_ERR_UNSUPPORTED, "GEMM peer stores: layout not taken");
        g.npeer = peers->npeer;
        g.pcs = peers->pcs;
        g.epoch = peers->epoch;
        for (int par = 0; par < 2; ++par)
            for (int r = 0; r < peers->npeer; ++r) {
                g.pslot[par][r] = peers->slot[par][r];
                if (g.tma_store && (st = make_y_map(&pm.m[par][r], peers->slot[par][r], (uint64_t)M, (uint64_t)N,
                                                    peers->pcs)) != MLZC_OK)
                    return st;
            }
    }
    if (pl.MT == 2) return BN == 192 ? launch_tile<192, 2>(c, ta, ty, pm, g, s) : launch_tile<256, 2>(c, ta, ty, pm, g, s);
    switch (BN) {
        case 16: return launch_tile<16, 1>(c, ta, ty, pm, g, s);
        case 32: return launch_tile<32, 1>(c, ta, ty, pm, g, s);
        case 64: return launch_tile<64, 1>(c, ta, ty, pm, g, s);
        case 96: return launch_tile<96, 1>(c, ta, ty, pm, g, s);
        case 128: return launch_tile<128, 1>(c, ta, ty, pm, g, s);
        default: return launch_tile<256, 1>(c, ta, ty, pm, g, s);
    }
}

}  // namespace

int launch_gemm_f16(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                    size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                    cudaStream_t s) {
    return launch_gemm_f16_impl(c, w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes, ws, ws_bytes, s, nullptr,
                                nullptr);
}

int launch_gemm_f16_row_scaled(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                               const float* x, size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws,
                               size_t ws_bytes, const float* row_scale, cudaStream_t s) {
    return launch_gemm_f16_impl(c, w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes, ws, ws_bytes, s, nullptr,
                                row_scale);
}

int launch_gemm_f16_peers(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                          size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                          const GemmPeers& peers, cudaStream_t s) {
    return launch_gemm_f16_impl(c, w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes, ws, ws_bytes, s, &peers,
                                nullptr);
}

}  // namespace mlzc
