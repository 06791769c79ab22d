// q4k_ring.cu -- decode-shaped Q4_K mul_mat for 5 <= N <= 8 activation columns as a
// persistent kernel fed by a TMA ring (q4k_ring_xs_kernel): the activations are prepared once
// per call (q4k_prep_kernel's f16 B fragments and sub-block sums) and each stage carries its
// blocks' fragments next to the weight box.  (N <= 4 takes the int8 path, q4k_i8.cu.)
//
// Replaces, for these shapes, the Q4_K branch of ggml_simd_try_mul_mat
// (src/simd/ggml_simd_hook.cpp:188-231, 238-299): one simd_vec_dot_q4_k_q8_k
// (src/simd/kernels/x86/vec/vec_dot_q4_k_q8_k_avx2.asm:38-266) per (row, column).  The
// arithmetic is that of q4k_mma.cu (exact f16 sc*q dequant, f16 activations, fp32 MMA
// accumulation, the min term as an MMA pair); what changes is how the bytes arrive.
//
// Design (HBM-bound: every block byte is read once):
//   - A tile is 16 weight rows (the MMA's M) times all of K.  Each CTA owns whole tiles
//     (t = blockIdx.x, + gridDim.x, ...), so no partial row crosses CTAs and nothing is
//     merged after the kernel.
//   - A producer warp streams the tile's blocks into a 2-stage shared-memory ring with TMA:
//     a stage is 8 consecutive K blocks of the 16 rows (one 2-d box of 16 rows x 1152
//     contiguous bytes) plus those blocks' prepared activations (bulk copies from the
//     workspace).  Two CTAs per SM.
//   - Eight consumer warps each take one block of every stage: the header and their
//     32-byte nibble chunk for rows g and g + 8, the (sc, m) unpack, LOP3 + HFMA2 dequant
//     and the MMAs.
//   - At the end of a tile the eight warps' partial rows are summed in warp order through
//     shared memory (one named barrier per tile; double-buffered), so results repeat bit
//     for bit.
//   - Every mbarrier wait is bounded; a consumer that gives up keeps taking the named
//     barriers (so no warp is left waiting on them) and no output is written.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "internal.h"
#include "ptx.cuh"
#include "q4k.cuh"

namespace mlzc {
namespace {

using ptx::mma16816;
using q4k::deq_hi;
using q4k::deq_lo;
using q4k::h2u;
using q4k::RowScales;

constexpr int kRWarps = 8;                                 // consumer warps
constexpr int kRThreads = (kRWarps + 1) * 32;              // + the producer warp
constexpr int kTileRows = 16;                              // rows per tile (MMA M)
constexpr int kStageBlocks = kRWarps;                      // K blocks per stage, one per consumer warp
constexpr int kBoxBytes = kTileRows * q4k::kBlockBytes;    // 2304: one block of the tile's 16 rows
constexpr uint32_t kStageBytes = kStageBlocks * kBoxBytes; // 18432
constexpr int kU64PerBlock = q4k::kBlockBytes / 8;         // a block in the map's 8-byte elements

struct RingParams {
    const char* x;               // activations, column n at x + n * x_cs (f32)
    size_t x_cs;
    char* y;                     // output, column n at y + n * y_cs (f32)
    size_t y_cs;
    int M, nblk, N, tiles;       // tiles = ceil(M / 16)
    int early;                   // 1: the producer may load blocks before pdl_wait()
    const uint4* xf;             // prepared B fragments (q4k_prep_kernel layout), shared-X form only
    const uint2* xs;             // prepared sub-block sums, shared-X form only
    unsigned int* err;           // device error word (bounded waits)
    CUtensorMap tm_w;            // W as 8-byte elements: [M][nblk * 18], box 18 x 16
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// The 256 consumer threads only (the producer warp never takes it).
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kRWarps * 32) : "memory"); }

__device__ __forceinline__ uint32_t word_of(const uint4& a, const uint4& b, int wi) {
    switch (wi) {
        case 0: return a.x;
        case 1: return a.y;
        case 2: return a.z;
        case 3: return a.w;
        case 4: return b.x;
        case 5: return b.y;
        case 6: return b.z;
        default: return b.w;
    }
}

// Streaming shared-X stage: the 16 x 8-block weight box, then the 8 blocks' prepared B
// fragments (4 KB each) and sub-block sums (256 B each) of the single column tile.
constexpr uint32_t kXsStageBytes = kStageBytes + kStageBlocks * (4096 + 256);   // 53248
constexpr int kXsStages = 2;

// Producer of the streaming shared-X form: as ring_producer, and each stage also gets its
// blocks' prepared activations by bulk copy from the workspace -- after pdl_wait(), since the
// prep kernel wrote them (in the weights-first mode the first weight box goes out before it).
__device__ __forceinline__ void ring_producer_xs(const RingParams& p, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                                 volatile int* abort_flag, int my_tiles, int nst) {
    const int G = gridDim.x;
    bool waited = !p.early;
    if (waited) ptx::pdl_wait();
    const int total = my_tiles * nst;
    int issued = 0;
    for (int it = 0; it < total; ++it) {
        const int s = it % kXsStages;
        const uint32_t ph = (it / kXsStages) & 1;
        if (!ptx::mbar_wait(ptx::smem_u32(&empty[s]), ph ^ 1, abort_flag, p.err)) break;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const int ti = it / nst, si = it % nst;
        const int m0 = ((int)blockIdx.x + ti * G) * kTileRows;
        const int kb0 = si * kStageBlocks;
        const int nb = min(kStageBlocks, p.nblk - kb0);   // the fragment copies stop at the row end
        const uint32_t fb = ptx::smem_u32(&full[s]);
        const uint32_t st = ptx::smem_u32(ring + (size_t)s * kXsStageBytes);
        ptx::mbar_expect_tx(fb, kStageBytes + (uint32_t)nb * (4096 + 256));
        tma_load_2d(st, &p.tm_w, fb, kb0 * kU64PerBlock, m0);
        if (!waited) {
            ptx::pdl_wait();
            waited = true;
        }
        ptx::bulk_load(st + kStageBytes, reinterpret_cast<const char*>(p.xf) + (size_t)kb0 * 4096, (uint32_t)nb * 4096, fb);
        ptx::bulk_load(st + kStageBytes + kStageBlocks * 4096, reinterpret_cast<const char*>(p.xs) + (size_t)kb0 * 256,
                       (uint32_t)nb * 256, fb);
        issued = it + 1;
    }
    volatile int no_abort = 0;
    for (int s = 0; s < kXsStages && s < issued; ++s) {
        const int last = s + (issued - 1 - s) / kXsStages * kXsStages;
        ptx::mbar_wait(ptx::smem_u32(&full[s]), (last / kXsStages) & 1, &no_abort, p.err);
    }
}

// Shared-X form (3 <= N <= 8): the activations were prepared once for the call by
// q4k_prep_kernel (f16 B fragments and sub-block sums, one 8-column tile), and each stage
// carries its 8 blocks' fragments and sums next to the weight box, so the activations cost a
// re-read from L2 per tile instead of a conversion per CTA.  Two stages, two CTAs per SM;
// shared memory aligned to 128 bytes (enough for the non-swizzled weight box) so both fit.
constexpr size_t ring_xs_smem_bytes() {
    return 128 + (size_t)kXsStages * kXsStageBytes + 2 * (size_t)kRWarps * kTileRows * 8 * 4 + (2 * kXsStages + 1) * 8 + 16;
}

__global__ void __launch_bounds__(kRThreads, 2)
q4k_ring_xs_kernel(const __grid_constant__ RingParams p) {
    constexpr int NT = 1;                                  // one 8-column MMA tile
    constexpr int kStagesX = kXsStages;
    constexpr uint32_t kSB = kXsStageBytes;                // stage stride
    constexpr int kRedX = kRWarps * kTileRows * 8 * NT;   // one set of the warps' partial tiles
    extern __shared__ uint8_t q4x_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q4x_smem_raw) + 127) & ~uintptr_t(127));
    uint8_t* ring = smem;
    float* red = reinterpret_cast<float*>(smem + (size_t)kStagesX * kSB);
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kRedX);
    uint64_t* empty = full + kStagesX;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStagesX);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesX; ++s) {
            ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
            ptx::mbar_init(ptx::smem_u32(&empty[s]), kRWarps);
        }
        *abort_flag = 0;
        ptx::mbar_init_fence();
    }
    __syncthreads();
    ptx::pdl_launch_dependents();

    const int G = gridDim.x;
    const int nst = (p.nblk + kStageBlocks - 1) / kStageBlocks;
    const int my_tiles = (int)blockIdx.x < p.tiles ? (p.tiles - 1 - (int)blockIdx.x) / G + 1 : 0;
    if (warp == kRWarps) {
        if (lane == 0) ring_producer_xs(p, ring, full, empty, abort_flag, my_tiles, nst);
        return;
    }

    // ---------------- consumers
    ptx::pdl_wait();   // the writes of Y come after the previous kernel
    bool ok = true;

    const int g = lane >> 2;
    const int q4 = lane & 3;
    const uint32_t ring_u32 = ptx::smem_u32(ring);
    int it = 0;
    for (int ti = 0; ti < my_tiles; ++ti) {
        const int m0 = ((int)blockIdx.x + ti * G) * kTileRows;
        float y[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t) y[t][0] = y[t][1] = y[t][2] = y[t][3] = 0.0f;
        for (int si = 0; si < nst; ++si, ++it) {
            const int s = it % kStagesX;
            const uint32_t ph = (it / kStagesX) & 1;
            if (ok && !ptx::mbar_wait(ptx::smem_u32(&full[s]), ph, abort_flag, p.err)) ok = false;
            if (!ok) continue;
            const int kb = si * kStageBlocks + warp;
            if (kb < p.nblk) {
                const uint32_t bb = ring_u32 + (uint32_t)s * kSB + (uint32_t)warp * q4k::kBlockBytes;
                const uint32_t r0 = bb + (uint32_t)g * (kStageBlocks * q4k::kBlockBytes), r1 = r0 + 8 * (kStageBlocks * q4k::kBlockBytes);
                const uint4 h0 = lds128(r0), h1 = lds128(r1);
                const uint4 a0w = lds128(r0 + 16 + 32 * q4), b0w = lds128(r0 + 32 + 32 * q4);
                const uint4 a1w = lds128(r1 + 16 + 32 * q4), b1w = lds128(r1 + 32 + 32 * q4);
                RowScales s0, s1;
                q4k::row_scales2(h0, h1, q4, s0, s1);
                // this block's fragments and sums, in the stage after the weights
                const uint4* xst = reinterpret_cast<const uint4*>(ring + (size_t)s * kSB + kStageBytes);
                const uint2* sst = reinterpret_cast<const uint2*>(ring + (size_t)s * kSB + kStageBytes + kStageBlocks * 4096);
                const uint4* xb[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    xb[t] = xst + (size_t)(t * kStageBlocks + warp) * 256 + q4 * 8 + g;
                float acc[NT][2][4];
#pragma unroll
                for (int t = 0; t < NT; ++t)
#pragma unroll
                    for (int c = 0; c < 2; ++c) acc[t][c][0] = acc[t][c][1] = acc[t][c][2] = acc[t][c][3] = 0.0f;
#pragma unroll
                for (int pr = 0; pr < 8; ++pr) {
                    uint4 xv[NT];
#pragma unroll
                    for (int t = 0; t < NT; ++t) xv[t] = xb[t][pr * 32];
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        const int stp = 2 * pr + h2, wi = stp & 7;
                        const uint32_t w0 = word_of(a0w, b0w, wi), w1 = word_of(a1w, b1w, wi);
                        uint32_t a0, a1, a2, a3;
                        if (stp < 8) {
                            a0 = deq_lo(w0, s0);
                            a1 = deq_lo(w1, s1);
                            a2 = deq_lo(w0 >> 8, s0);
                            a3 = deq_lo(w1 >> 8, s1);
                        } else {
                            a0 = deq_hi(w0, s0);
                            a1 = deq_hi(w1, s1);
                            a2 = deq_hi(w0 >> 8, s0);
                            a3 = deq_hi(w1 >> 8, s1);
                        }
#pragma unroll
                        for (int t = 0; t < NT; ++t)
                            mma16816(acc[t][h2], a0, a1, a2, a3, h2 ? xv[t].z : xv[t].x, h2 ? xv[t].w : xv[t].y);
                    }
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    // min term: sum_j m_j S_j with S as f16 hi + lo
                    const uint2 sv = sst[(t * kStageBlocks + warp) * 32 + q4 * 8 + g];
                    float mn[4] = {0.f, 0.f, 0.f, 0.f}, ml[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(mn, s0.mpair, s1.mpair, 0u, 0u, sv.x, 0u);
                    mma16816(ml, s0.mpair, s1.mpair, 0u, 0u, sv.y, 0u);
                    y[t][0] += s0.d * (acc[t][0][0] + acc[t][1][0]) - s0.dmin * (mn[0] + ml[0]);
                    y[t][1] += s0.d * (acc[t][0][1] + acc[t][1][1]) - s0.dmin * (mn[1] + ml[1]);
                    y[t][2] += s1.d * (acc[t][0][2] + acc[t][1][2]) - s1.dmin * (mn[2] + ml[2]);
                    y[t][3] += s1.d * (acc[t][0][3] + acc[t][1][3]) - s1.dmin * (mn[3] + ml[3]);
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&empty[s]));
        }
        // ---- the eight warps' partial tiles -> rows of Y, summed in warp order
        float* rb = red + (ti & 1) * kRedX;
        float* mine = rb + warp * (kTileRows * 8 * NT);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            mine[t * 128 + g * 8 + 2 * q4] = y[t][0];
            mine[t * 128 + g * 8 + 2 * q4 + 1] = y[t][1];
            mine[t * 128 + (g + 8) * 8 + 2 * q4] = y[t][2];
            mine[t * 128 + (g + 8) * 8 + 2 * q4 + 1] = y[t][3];
        }
        consumer_sync();
        const int tid = threadIdx.x;
        if (ok && tid < kTileRows * p.N && !*abort_flag) {
            const int r = tid & (kTileRows - 1), c = tid >> 4;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kRWarps; ++w) v += rb[w * (kTileRows * 8 * NT) + (c >> 3) * 128 + r * 8 + (c & 7)];
            if (m0 + r < p.M) reinterpret_cast<float*>(p.y + (size_t)c * p.y_cs)[m0 + r] = v;
        }
    }
}


// Resident CTAs of a ring kernel with `smem` bytes, over all SMs (the kernel's shared-memory
// limit is raised to the device's opt-in maximum once per device; occupancy is queried once
// per device and size; one cache per kernel instantiation).
template <typename Kern>
int ring_slots(Kern kernel, size_t smem, int* out) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, size_t>, int> cache;
    static std::map<std::tuple<const void*, int>, bool> attr_set;
    int dev = 0;
    MLZC_CUDA_TRY(cudaGetDevice(&dev));
    const void* key = reinterpret_cast<const void*>(kernel);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({key, dev, smem});
    if (it != cache.end()) {
        *out = it->second;
        return MLZC_OK;
    }
    if (!attr_set[{key, dev}]) {
        int optin = 0;
        MLZC_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        MLZC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
        attr_set[{key, dev}] = true;
    }
    int occ = 0, sms = 0;
    MLZC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kRThreads, smem));
    MLZC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (occ < 1) return fail(MLZC_ERR_CUDA, "Q4_K ring kernel does not fit on an SM");
    cache[{key, dev, smem}] = occ * sms;
    *out = occ * sms;
    return MLZC_OK;
}

int launch_ring_xs(const DeviceCtx* c, RingParams& p, cudaStream_t s) {
    const size_t smem = ring_xs_smem_bytes();
    int slots = 0;
    const int st = ring_slots(q4k_ring_xs_kernel, smem, &slots);
    if (st != MLZC_OK) return st;
    const int grid = std::min(p.tiles, slots);
    p.err = c->err;
    MLZC_CUDA_TRY(launch_pdl(q4k_ring_xs_kernel, dim3((unsigned)grid), dim3(kRThreads), smem, s, p));
    count_launch();
    return MLZC_OK;
}

// Everything but the activation source (p.x / p.xf, p.xs), which the two forms set.
int make_ring_params(const void* w, size_t w_row_bytes, int64_t M, int64_t K, int64_t N, float* y, size_t y_col_bytes,
                     RingParams* out) {
    if ((uintptr_t)w % 16 || w_row_bytes % 16) return fail(MLZC_ERR_INVALID, "Q4_K: weights must be 16-byte aligned");
    auto enc = tensor_map_encoder();
    if (!enc) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    RingParams& p = *out;
    p = RingParams{};
    p.y = reinterpret_cast<char*>(y);
    p.y_cs = y_col_bytes;
    p.M = (int)M;
    p.nblk = (int)(K / q4k::kQK);
    p.N = (int)N;
    p.tiles = (int)((M + kTileRows - 1) / kTileRows);
    p.early = weights_before_wait() ? 1 : 0;
    const cuuint64_t dims[2] = {(cuuint64_t)p.nblk * kU64PerBlock, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)w_row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(kU64PerBlock * kStageBlocks), (cuuint32_t)kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&p.tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MLZC_ERR_INVALID, "Q4_K ring: weight rows not expressible as a TMA map (%d)", (int)r);
    return MLZC_OK;
}

}  // namespace

bool q4k_ring_xs_applicable(int64_t M, int64_t K, int64_t N) {
    // Measured on B200 (us, this form / a register-only decode kernel): N = 8:
    // 4096 x 4096 6.9 / 8.0, 14336 x 4096 16.4 / 19.4, 4096 x 14336 16.5 / 25.0.
    return N >= 5 && N <= 8 && K % q4k::kQK == 0 && M >= 1 && M <= (int64_t)1 << 30;
}

int launch_q4k_ring_xs(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                       const uint4* xf, const uint2* xs, int64_t N, float* y, size_t y_col_bytes, cudaStream_t s) {
    if (!q4k_ring_xs_applicable(M, K, N)) return fail(MLZC_ERR_UNSUPPORTED, "Q4_K ring: shape not taken");
    if ((uintptr_t)xf % 16 || (uintptr_t)xs % 16) return fail(MLZC_ERR_INVALID, "Q4_K ring: workspace not 16-byte aligned");
    RingParams p;
    const int st = make_ring_params(w, w_row_bytes, M, K, N, y, y_col_bytes, &p);
    if (st != MLZC_OK) return st;
    p.xf = xf;
    p.xs = xs;
    return launch_ring_xs(c, p, s);
}

}  // namespace mlzc
