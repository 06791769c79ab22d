// q4k_i8.cu -- decode-shaped Q4_K mul_mat (1 <= N <= 4 activation columns) on the 8-bit
// integer tensor-core path, as a stream-K persistent kernel fed by a TMA ring.
//
// Replaces, for N <= 4, the Q4_K branch of ggml_simd_try_mul_mat
// (src/simd/ggml_simd_hook.cpp:188-231, 238-299): quantize_row_q8_k_reference (:109-148)
// of each activation column, then one simd_vec_dot_q4_k_q8_k
// (src/simd/kernels/x86/vec/vec_dot_q4_k_q8_k_avx2.asm:38-266) per (row, column).
//
// Arithmetic.  Each 256-value block of an activation column is quantised to two int8
// vectors with one f32 scale s: x ~= s * (hi + lo / 254), hi = rint(x / s) with
// s = max|x| / 127, lo = rint(254 (x - s hi) / s).  The error is below s / 508 per value
// (about 1.5e-5 of the block's largest value), far inside the parity tolerance of the
// dequantised-F32 product; the reference's own Q8_K rounding is 64x coarser.  A Q4_K
// sub-block j (32 weights, 6-bit scale sc_j and min m_j) is then exactly one
// mma.sync.m16n8k32 u8 x s8 -> s32: the weight nibbles are the u8 operand as they lie
// (one LOP3 keeps the low nibbles of four bytes, one the high nibbles, which read as 16 q),
// and the hi and lo vectors of up to four columns are the eight B columns.  Each
// sub-block's integer sums are scaled by sc_j with one IMAD per accumulator and summed in
// int32 (no overflow: |sum| < 2^29); per block the row gets
//   y += d * s / 16 * (HI + LO / 254) - dmin * sum_j m_j S_j,
// with the sub-block sums S_j of the unquantised activations (f16 hi + lo) against m_j
// (f16) in one m16n8k16 MMA.  About 1.3 thread instructions per weight, against ~3.4 for the
// f16 dequant path.
//
// Schedule.  A unit is 16 weight rows x 8 K blocks (one TMA box of 16 x 1152 bytes); the
// units of all row tiles are numbered tile-major and every CTA takes an equal contiguous
// range of them (stream-K), so no SM idles while another finishes a tile.  A producer warp
// fills a shared-memory ring with each unit's weight box plus, by one bulk copy, the unit's
// prepared activation record (act_i8::prep_kernel writes one record per 8 blocks).  Eight
// consumer warps each take one block of a unit.  At the end of a tile (or of the CTA's
// range) the warps' partial rows are summed in warp order through shared memory and added
// into Y (zeroed by the prep kernel) with red.global.add.  The grid is capped so that every
// CTA's range is at least nst - 1 units long (nst = units per tile): no range then lies
// strictly inside a tile, a tile has at most two pieces, and 0 + a + b = 0 + b + a exactly,
// so results repeat bit for bit with no fix-up pass, counter or fence (a counter-and-slot
// merge measured 3-5 us slower per call: its fence and atomic round trips sat on every
// CTA's critical path).
//
// Bank conflicts.  With K a multiple of 2048 the weight box is loaded as a 3-d view
// (16 x 9 x 128-byte lines per stage) with the 128-byte swizzle, and the MMA rows g = 0..7
// read tile rows 0, 2, 4, 6, 1, 3, 5, 7 (+8): every 8-byte nibble load of a half-warp then
// touches distinct banks (a plain box puts all 16 rows on the same banks, 1152 being a
// multiple of 128).  Other K use the plain box.
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
#include "act_i8.cuh"

namespace mlzc {
namespace {

constexpr int kQK = 256;                                   // weights per Q4_K block
constexpr int kBlk = 144;                                  // bytes per Q4_K block
constexpr int kWarps = 8;                                  // consumer warps = blocks per unit
constexpr int kThreads = (kWarps + 1) * 32;                // + the producer warp
constexpr int kTileRows = 16;
constexpr uint32_t kBoxBytes = kTileRows * kWarps * kBlk;  // 18432: one unit's weights
constexpr int kU64PerBlock = kBlk / 8;                     // 18
// activation records: act_i8.cuh with 8 sums (32-value sub-blocks) per block
using act_i8::kVarStride;
__host__ __device__ constexpr uint32_t rec_bytes(int nct) { return act_i8::rec_bytes(nct, 8); }
__host__ __device__ constexpr uint32_t rec_scale_off(int nct) { return act_i8::rec_scale_off(nct); }
__host__ __device__ constexpr uint32_t rec_sum_off(int nct) { return act_i8::rec_sum_off(nct); }

__host__ __device__ constexpr int stages_for(int nct) { return nct <= 2 ? 4 : 2; }

struct I8Params {
    const char* rec;             // prepared records, unit column si at rec + si * rbytes
    char* y;                     // output, column n at y + n * y_cs (f32)
    size_t y_cs;
    unsigned int* err;           // device error word (bounded waits)
    long long units;             // tiles * nst
    int M, nblk, nst, N, tiles;
    int early;                   // 1: the producer may load weights before pdl_wait()
    CUtensorMap tm_w;
};

// Dynamic shared memory: ring of weight boxes (1024-aligned for the swizzle), the records,
// the double-buffered reduction tiles, barriers.
constexpr size_t i8_smem_bytes(int nct) {
    return 1024 + (size_t)stages_for(nct) * (kBoxBytes + rec_bytes(nct)) + 2 * (size_t)kWarps * kTileRows * nct * 4 +
           2 * (size_t)stages_for(nct) * 8 + 32;
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

// d = a (16 x 32 u8) . b (32 x 8 s8), fresh s32 accumulators.  Fragments per the PTX ISA:
// lane l holds A rows l/4 and l/4 + 8 at k 4(l%4)..+3 (a0, a1) and 16 + 4(l%4)..+3 (a2, a3),
// B column l/4 at the same k (b0, b1), D rows l/4, l/4 + 8 x columns 2(l%4), +1.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory"); }

__device__ __forceinline__ void red_add(float* p, float v) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Offset in a stage of byte `o` of tile row `r` (1152 bytes per row), plain or as the
// 128-byte-swizzled image of the 3-d box (line L = 9 r + o / 128, 16-byte unit u of the
// line stored at u ^ (L & 7)).
template <bool SWZ>
__device__ __forceinline__ uint32_t box_off(int r, int o) {
    if constexpr (!SWZ) return (uint32_t)(r * (kWarps * kBlk) + o);
    const int L = 9 * r + (o >> 7);
    const int u = (o >> 4) & 7;
    return (uint32_t)(L * 128 + ((u ^ (L & 7)) << 4) + (o & 15));
}

// CTA c's units [first_unit(c), first_unit(c + 1)).
__device__ __forceinline__ long long first_unit(long long c, long long U, long long G) { return c * U / G; }

// ------------------------------------------------------------------ main kernel
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

template <int NCT, bool SWZ>
__global__ void __launch_bounds__(kThreads, 2) q4k_i8_kernel(const __grid_constant__ I8Params p) {
    constexpr int NV = 2 * NCT;
    constexpr int S = stages_for(NCT);
    constexpr uint32_t RB = rec_bytes(NCT);
    extern __shared__ uint8_t i8_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(i8_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* boxes = smem;                                        // S x 18432
    uint8_t* recs = boxes + (size_t)S * kBoxBytes;                // S x RB
    float* red = reinterpret_cast<float*>(recs + (size_t)S * RB); // 2 x [8 warps][16 rows][NCT]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kWarps * kTileRows * NCT);
    uint64_t* empty = full + S;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
            ptx::mbar_init(ptx::smem_u32(&empty[s]), kWarps);
        }
        *abort_flag = 0;
        ptx::mbar_init_fence();
    }
    __syncthreads();
    ptx::pdl_launch_dependents();

    const long long U = p.units, G = gridDim.x, c = blockIdx.x;
    const long long u0 = first_unit(c, U, G), u1 = first_unit(c + 1, U, G);

    if (warp == kWarps) {
        // ---------------- producer
        if (lane != 0) return;
        auto load_weights = [&](int s, long long u) {
            const int tile = (int)(u / p.nst), si = (int)(u % p.nst);
            const uint32_t fb = ptx::smem_u32(&full[s]);
            ptx::mbar_expect_tx(fb, kBoxBytes + RB);
            const uint32_t dst = ptx::smem_u32(boxes + (size_t)s * kBoxBytes);
            if constexpr (SWZ)
                tma_load_3d(dst, &p.tm_w, fb, 0, si * 9, tile * kTileRows);
            else
                tma_load_2d(dst, &p.tm_w, fb, si * kWarps * kU64PerBlock, tile * kTileRows);
        };
        auto load_record = [&](int s, long long u) {
            const int si = (int)(u % p.nst);
            ptx::bulk_load(ptx::smem_u32(recs + (size_t)s * RB), p.rec + (size_t)si * RB, RB, ptx::smem_u32(&full[s]));
        };
        // weights-first mode: the first S units' weight boxes go out before the wait (the
        // ring's slots are free at the start), their records after it (the prep kernel's output)
        const int pro = p.early ? (int)(u1 - u0 < S ? u1 - u0 : S) : 0;
        for (int i = 0; i < pro; ++i) load_weights(i, u0 + i);
        ptx::pdl_wait();
        for (int i = 0; i < pro; ++i) load_record(i, u0 + i);
        int issued = pro;
        int it = pro;
        for (long long u = u0 + pro; u < u1; ++u, ++it) {
            const int s = it % S;
            const uint32_t ph = (it / S) & 1;
            if (!ptx::mbar_wait(ptx::smem_u32(&empty[s]), ph ^ 1, abort_flag, p.err)) break;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            load_weights(s, u);
            load_record(s, u);
            issued = it + 1;
        }
        // no copy may still be landing when the CTA exits (bounded)
        volatile int no_abort = 0;
        for (int s = 0; s < S && s < issued; ++s) {
            const int last = s + (issued - 1 - s) / S * S;
            ptx::mbar_wait(ptx::smem_u32(&full[s]), (last / S) & 1, &no_abort, p.err);
        }
        return;
    }

    // ---------------- consumers
    ptx::pdl_wait();   // Y (zeroed by the prep kernel) comes after the previous kernels
    const int g = lane >> 2, t = lane & 3;
    // MMA rows g and g + 8 read tile rows y0 and y0 + 8 (bank-conflict-free order for the
    // swizzled box)
    const int y0 = SWZ ? ((g & 3) * 2 + (g >> 2)) : g;
    const int y1 = y0 + 8;
    const int ob = warp * kBlk;   // this warp's block in the unit's rows
    const uint32_t hoff0 = box_off<SWZ>(y0, ob), hoff1 = box_off<SWZ>(y1, ob);
    uint32_t aoff0[4], aoff1[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        aoff0[ch] = box_off<SWZ>(y0, ob + 16 + 32 * ch + 8 * t);
        aoff1[ch] = box_off<SWZ>(y1, ob + 16 + 32 * ch + 8 * t);
    }
    const bool bv = g < NV;   // this lane's B column is a real vector
    const uint32_t boff = (uint32_t)((bv ? g : 0) * kVarStride + warp * kQK + 8 * t);
    const int tn = t < NCT ? t : NCT - 1;
    const uint32_t scoff = rec_scale_off(NCT) + (uint32_t)(tn * 8 + warp) * 4;
    const uint32_t smoff = rec_sum_off(NCT) + (uint32_t)((warp * NV + (bv ? g : 0)) * 16 + 4 * t);
    const uint32_t box_base = ptx::smem_u32(boxes), rec_base = ptx::smem_u32(recs);
    const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
    const uint32_t msel = (t & 1) ? 0x5342u : 0x5140u;

    const int tid = threadIdx.x;
    bool ok = true;
    int it = 0, flushes = 0;
    float ya0 = 0.0f, ya1 = 0.0f;   // rows y0, y1 of column t
    long long u = u0;
    int tile = (int)(u0 / p.nst), si = (int)(u0 % p.nst);
    while (u < u1) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (ok && !ptx::mbar_wait(ptx::smem_u32(&full[s]), ph, abort_flag, p.err)) ok = false;
        const int kb = si * kWarps + warp;
        if (ok && kb < p.nblk) {
            const uint32_t W = box_base + (uint32_t)s * kBoxBytes;
            const uint32_t R = rec_base + (uint32_t)s * RB;
            const uint4 h0 = lds128(W + hoff0), h1 = lds128(W + hoff1);
            uint2 wa[4], wb[4], bx[8];
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                wa[ch] = lds64(W + aoff0[ch]);
                wb[ch] = lds64(W + aoff1[ch]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) bx[j] = bv ? lds64(R + boff + 32 * j) : make_uint2(0u, 0u);
            const uint32_t sraw = bv ? lds32(R + smoff) : 0u;
            const float sb = __uint_as_float(lds32(R + scoff));
            // 6-bit scales and mins of the eight sub-blocks, four per word
            const uint32_t sc03a = h0.y & 0x3F3F3F3Fu, sc03b = h1.y & 0x3F3F3F3Fu;
            const uint32_t sc47a = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
            const uint32_t sc47b = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
            int acc_e[4] = {0, 0, 0, 0}, acc_o[4] = {0, 0, 0, 0};
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const uint32_t wsa = ch < 2 ? sc03a : sc47a, wsb = ch < 2 ? sc03b : sc47b;
                const int je = (2 * ch) & 3, jo = (2 * ch + 1) & 3;
                const int sea = (int)__byte_perm(wsa, 0u, 0x4440u | je), seb = (int)__byte_perm(wsb, 0u, 0x4440u | je);
                const int soa = (int)__byte_perm(wsa, 0u, 0x4440u | jo), sob = (int)__byte_perm(wsb, 0u, 0x4440u | jo);
                int d[4];
                mma_u8s8(d, wa[ch].x & 0x0F0F0F0Fu, wb[ch].x & 0x0F0F0F0Fu, wa[ch].y & 0x0F0F0F0Fu,
                         wb[ch].y & 0x0F0F0F0Fu, bx[2 * ch].x, bx[2 * ch].y);
                acc_e[0] += d[0] * sea;
                acc_e[1] += d[1] * sea;
                acc_e[2] += d[2] * seb;
                acc_e[3] += d[3] * seb;
                mma_u8s8(d, wa[ch].x & 0xF0F0F0F0u, wb[ch].x & 0xF0F0F0F0u, wa[ch].y & 0xF0F0F0F0u,
                         wb[ch].y & 0xF0F0F0F0u, bx[2 * ch + 1].x, bx[2 * ch + 1].y);
                acc_o[0] += d[0] * soa;
                acc_o[1] += d[1] * soa;
                acc_o[2] += d[2] * sob;
                acc_o[3] += d[3] * sob;
            }
            // min term: sum_j m_j S_j (rows y0, y1; S as f16 hi + lo / 2048 in columns 2t, 2t + 1)
            const uint32_t m03a = h0.z & 0x3F3F3F3Fu, m03b = h1.z & 0x3F3F3F3Fu;
            const uint32_t m47a = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
            const uint32_t m47b = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
            const uint32_t mpa = q4k::h2u(__hsub2(q4k::u2h(__byte_perm(t < 2 ? m03a : m47a, 0x6464u, msel)), k1024));
            const uint32_t mpb = q4k::h2u(__hsub2(q4k::u2h(__byte_perm(t < 2 ? m03b : m47b, 0x6464u, msel)), k1024));
            float mn[4] = {0.f, 0.f, 0.f, 0.f};
            ptx::mma16816(mn, mpa, mpb, 0u, 0u, sraw, 0u);
            const float2 dd0 = __half22float2(q4k::u2h(h0.x)), dd1 = __half22float2(q4k::u2h(h1.x));
            const float f = sb * (1.0f / 16.0f);
            const float hi0 = (float)(acc_e[0] * 16 + acc_o[0]), lo0 = (float)(acc_e[1] * 16 + acc_o[1]);
            const float hi1 = (float)(acc_e[2] * 16 + acc_o[2]), lo1 = (float)(acc_e[3] * 16 + acc_o[3]);
            ya0 += dd0.x * f * fmaf(lo0, 1.0f / 254.0f, hi0) - dd0.y * fmaf(mn[1], 1.0f / 2048.0f, mn[0]);
            ya1 += dd1.x * f * fmaf(lo1, 1.0f / 254.0f, hi1) - dd1.y * fmaf(mn[3], 1.0f / 2048.0f, mn[2]);
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&empty[s]));
        ++it;
        ++u;
        const bool tile_end = ++si == p.nst || u == u1;
        if (!tile_end) continue;
        // ---- flush tile `tile`: the eight warps' partial rows, summed in warp order
        float* rb = red + (flushes & 1) * (kWarps * kTileRows * NCT);
        ++flushes;
        if (t < NCT) {
            rb[(warp * kTileRows + y0) * NCT + t] = ya0;
            rb[(warp * kTileRows + y1) * NCT + t] = ya1;
        }
        consumer_sync();
        const int r = tid & (kTileRows - 1), n = tid >> 4;
        const int m0 = tile * kTileRows;
        if (tid < kTileRows * p.N && ok && !*abort_flag && m0 + r < p.M) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += rb[(w * kTileRows + r) * NCT + n];
            red_add(reinterpret_cast<float*>(p.y + (size_t)n * p.y_cs) + m0 + r, v);
        }
        ya0 = ya1 = 0.0f;
        ++tile;
        si = 0;
    }
}

// Resident CTAs of an instantiation over all SMs (shared-memory limit raised once per
// device; cached per kernel, device and size).
template <typename Kern>
int i8_slots(Kern kernel, size_t smem, int* out) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int>, int> cache;
    int dev = 0;
    MLZC_CUDA_TRY(cudaGetDevice(&dev));
    const void* key = reinterpret_cast<const void*>(kernel);
    std::lock_guard<std::mutex> lk(mu);
    auto f = cache.find({key, dev});
    if (f != cache.end()) {
        *out = f->second;
        return MLZC_OK;
    }
    MLZC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int occ = 0, sms = 0;
    MLZC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kThreads, smem));
    MLZC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (occ < 1) return fail(MLZC_ERR_CUDA, "Q4_K int8 kernel does not fit on an SM");
    cache[{key, dev}] = occ * sms;
    *out = occ * sms;
    return MLZC_OK;
}

template <int NCT, bool SWZ>
int launch_main(const DeviceCtx* c, I8Params& p, cudaStream_t s) {
    const size_t smem = i8_smem_bytes(NCT);
    int slots = 0;
    const int st = i8_slots(q4k_i8_kernel<NCT, SWZ>, smem, &slots);
    if (st != MLZC_OK) return st;
    // ranges of at least nst - 1 units: at most two pieces per tile (see the file comment)
    const long long cap = p.nst > 1 ? p.units / (p.nst - 1) : p.units;
    // 92 % of the resident slots: the free ones let the next call's kernels start during this
    // one's tail (B200 sweep of 34-100 % on the C3 / C6 steps: 92 % best at batch 1, 2 and 4,
    // e.g. C3 batch 1 27.0 vs 28.5 us per step, C6 batch 1 34.3 vs 36.3)
    const long long use = std::max<long long>(1, (long long)slots * 23 / 25);
    const int grid = (int)std::max<long long>(1, std::min<long long>({p.units, use, cap}));
    p.err = c->err;
    MLZC_CUDA_TRY(launch_pdl(q4k_i8_kernel<NCT, SWZ>, dim3((unsigned)grid), dim3(kThreads), smem, s, p));
    count_launch();
    return MLZC_OK;
}

int nct_of(int64_t N) { return N <= 1 ? 1 : N <= 2 ? 2 : 4; }

struct I8Ws {
    uint32_t rbytes;
    size_t rec;
    size_t total() const { return rec; }
};

I8Ws i8_ws(int64_t K, int64_t N) {
    I8Ws w;
    const int nblk = (int)(K / kQK), nst = (nblk + kWarps - 1) / kWarps;
    w.rbytes = rec_bytes(nct_of(N));
    w.rec = ((size_t)nst * w.rbytes + 255) / 256 * 256;
    return w;
}

}  // namespace

bool q4k_i8_applicable(int64_t M, int64_t K, int64_t N) {
    return N >= 1 && N <= 4 && K >= kQK && K % kQK == 0 && M >= 1 && M <= ((int64_t)1 << 30) &&
           K / kQK <= ((int64_t)1 << 24);
}

size_t q4k_i8_workspace_bytes(int64_t K, int64_t N) { return i8_ws(K, N).total(); }

int launch_q4k_i8(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                  size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                  cudaStream_t s) {
    if (!q4k_i8_applicable(M, K, N)) return fail(MLZC_ERR_UNSUPPORTED, "Q4_K int8 path: shape not taken");
    if ((uintptr_t)w % 16 || w_row_bytes % 16 || (uintptr_t)x % 16 || x_col_bytes % 16)
        return fail(MLZC_ERR_INVALID, "Q4_K: weights and activations must be 16-byte aligned");
    const I8Ws q = i8_ws(K, N);
    if (!ws || ws_bytes < q.total() || (uintptr_t)ws % 16)
        return fail(MLZC_ERR_NOMEM, "Q4_K: workspace of %zu bytes needed, %zu given", q.total(), ws_bytes);
    auto enc = tensor_map_encoder();
    if (!enc) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    char* wsc = static_cast<char*>(ws);
    const int nct = nct_of(N);
    I8Params p{};
    p.rec = wsc;
    p.y = reinterpret_cast<char*>(y);
    p.y_cs = y_col_bytes;
    p.M = (int)M;
    p.nblk = (int)(K / kQK);
    p.nst = (p.nblk + kWarps - 1) / kWarps;
    p.N = (int)N;
    p.tiles = (int)((M + kTileRows - 1) / kTileRows);
    p.units = (long long)p.tiles * p.nst;
    p.early = weights_before_wait() ? 1 : 0;
    // 128-byte-swizzled 3-d view when a row is whole 128-byte lines of whole units
    const bool swz = p.nblk % kWarps == 0;
    CUresult r;
    if (swz) {
        const cuuint64_t dims[3] = {16, (cuuint64_t)p.nblk * kBlk / 128, (cuuint64_t)M};
        const cuuint64_t strides[2] = {128, (cuuint64_t)w_row_bytes};
        const cuuint32_t box[3] = {16, 9, (cuuint32_t)kTileRows};
        const cuuint32_t estr[3] = {1, 1, 1};
        r = enc(&p.tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(w), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[2] = {(cuuint64_t)p.nblk * kU64PerBlock, (cuuint64_t)M};
        const cuuint64_t strides[1] = {(cuuint64_t)w_row_bytes};
        const cuuint32_t box[2] = {(cuuint32_t)(kU64PerBlock * kWarps), (cuuint32_t)kTileRows};
        const cuuint32_t estr[2] = {1, 1};
        r = enc(&p.tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return fail(MLZC_ERR_INVALID, "Q4_K: weight rows not expressible as a TMA map (%d)", (int)r);
    {
        const int items = p.nst * kWarps * nct;
        // one warp per record item; at least enough threads to zero Y in a few passes
        const long long zero_ctas = std::min<long long>(148, ((long long)M * N + 2047) / 2048);
        const unsigned pg = (unsigned)std::max<long long>((items + 7) / 8, zero_ctas);
        MLZC_CUDA_TRY(launch_pdl(act_i8::prep_kernel<8>, dim3(pg), dim3(256), 0, s,
                                 reinterpret_cast<const char*>(x), x_col_bytes, (int)N, nct, p.nblk, p.nst, q.rbytes,
                                 wsc, p.y, p.y_cs, p.M));
        count_launch();
    }
    if (nct == 1) return swz ? launch_main<1, true>(c, p, s) : launch_main<1, false>(c, p, s);
    if (nct == 2) return swz ? launch_main<2, true>(c, p, s) : launch_main<2, false>(c, p, s);
    return swz ? launch_main<4, true>(c, p, s) : launch_main<4, false>(c, p, s);
}

}  // namespace mlzc
