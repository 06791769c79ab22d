// q6k_i8.cu -- decode-shaped Q6_K mul_mat (1 <= N <= 4 activation columns) on the 8-bit
// integer tensor-core path, as a stream-K persistent kernel fed by a TMA ring.
//
// Replaces, for N <= 4, the Q6_K branch of ggml_simd_try_mul_mat
// (src/simd/ggml_simd_hook.cpp:282-288, the K-quant path of :234-301): Q8_K activations
// and one simd_vec_dot_q6_k_q8_k (src/simd/kernels/x86/vec/vec_dot_q6_k_q8_k_avx2.asm) per
// (row, column).  The parity bar is the dequantised-F32 product.
//
// Q6_K block (GGUF, 210 bytes per 256 weights): ql[128] @0, qh[64] @128, int8 scales[16]
// @192 (one per 16 weights), f16 d @208.  Weight p = 128 h + 32 qd + l (half h, quadrant qd,
// l < 32): q = nibble (qd / 2) of ql[64 h + 32 (qd % 2) + l] | bits (2 qd, 2 qd + 1) of
// qh[32 h + l] << 4, w = d * scales[8 h + 2 qd + l / 16] * (q - 32).
//
// Arithmetic.  Activations as int8 hi + lo per 256-value block (act_i8.cuh).  A quadrant
// (32 weights: two scale groups) is one mma.sync.m16n8k32 u8 x s8 -> s32 with the 6-bit q
// as the u8 operand (built from a ql word and a qh word by masks and shifts, four weights per
// 32-bit word) and the B columns split by group: for column n, B column 4 n + 2 grp + v holds
// vector v (hi / lo) of the group-grp half of the quadrant's values and zeros in the other
// half, so each accumulator column is one (group, hi / lo) sum.  A lane keeps the columns of
// one group parity and scales them by that group's int8 scale with one IMAD each (|sum| <
// 2^28 over a block).  One column fills half of the B columns, so there the other half carries
// the next quadrant and quadrant pairs accumulate in one MMA chain (q6_block_spread: half the
// scaling IMADs and scale extractions; 14.6 vs 15.0 us on 14336 x 4096).  The -32 offset is -32 d sum_g sc_g S_g with the group sums S_g of
// the unquantised activations (f16 hi + lo / 2048) against the scales (exact f16) in one m16n8k16
// MMA per block.  Per block the row gets d * s * (HI + LO / 254) - 32 d sum_g sc_g S_g.
//
// Schedule: as q4k_i8.cu (16-row x 8-block units, tile-major stream-K over CTAs, a TMA
// ring carrying each unit's weight box and activation record, eight consumer warps taking
// one block each, two-piece red.add merges into Y zeroed by the prep kernel).  A unit's
// rows are 1680 bytes (a multiple of 16 but not of 128, so no swizzle is needed: rows fall
// 4 banks apart and the 4-byte loads of a warp touch distinct banks).  Blocks at odd
// positions of a unit are 2-byte aligned only: their 4-byte fields are read as the two
// aligned words around them joined by a funnel shift.
//
// Needs K a multiple of 1024 (a row of whole 8-byte TMA elements) and 16-byte row strides;
// other shapes take q6k.cu.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "act_i8.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int kQK = 256;
constexpr int kBlk = 210;
constexpr int kWarps = 8;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kTileRows = 16;
constexpr int kRowBytes = kWarps * kBlk;                    // 1680: one unit row
constexpr uint32_t kBoxBytes = kTileRows * kRowBytes;       // 26880
constexpr int kU64PerUnit = kRowBytes / 8;                  // 210
constexpr int kGpb = 16;                                    // scale groups per block
using act_i8::kVarStride;

__host__ __device__ constexpr uint32_t rec_bytes(int nct) { return act_i8::rec_bytes(nct, kGpb); }
__host__ __device__ constexpr int stages_for(int nct) { return nct <= 1 ? 3 : 2; }

struct I8Params {
    const char* rec;
    char* y;
    size_t y_cs;
    unsigned int* err;
    long long units;
    int M, nblk, nst, N, tiles;
    int early;
    CUtensorMap tm_w;
};

constexpr size_t i8_smem_bytes(int nct) {
    return 128 + (size_t)stages_for(nct) * (kBoxBytes + rec_bytes(nct)) +
           2 * (size_t)kWarps * kTileRows * nct * 2 * 4 + 2 * (size_t)stages_for(nct) * 8 + 32;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
// The 4-byte field at a: aligned (ODD = false), or at a 2-mod-4 address (the two aligned
// words around it, joined).
template <bool ODD>
__device__ __forceinline__ uint32_t ldw(uint32_t a) {
    if constexpr (!ODD) return lds32(a);
    return __funnelshift_r(lds32(a - 2), lds32(a + 2), 16);
}

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// d += a . b (same fragments as mma_u8s8)
__device__ __forceinline__ void mma_u8s8_acc(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory"); }
__device__ __forceinline__ void red_add(float* p, float v) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ long long first_unit(long long c, long long U, long long G) { return c * U / G; }

// prmt with sign replication: selector nibbles 8 | b copy the sign of byte b.
__device__ __forceinline__ int prmt_sx(uint32_t x, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(x), "r"(sel));
    return (int)d;
}

// Two int8 (bytes 0, 1 of x) -> exact f16 pair.
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t x) {
    const uint32_t u = __byte_perm(x ^ 0x8080u, 0x6464u, 0x5140u);
    __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&u),
                        __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
    return *reinterpret_cast<uint32_t*>(&h);
}

// Per block of one warp: rows y0 = g and y0 + 8 (addresses r0, r1 of the block's first byte)
// against the unit record R; accumulates into ya[j][0..1] (batch column n = 2 j + t / 2 of
// group parity t & 1, rows y0 and y1).
template <int NCT, bool ODD>
__device__ __forceinline__ void q6_block(uint32_t r0, uint32_t r1, uint32_t R, int warp, int g, int t,
                                         float (&ya)[(NCT + 1) / 2][2]) {
    constexpr int NV = 2 * NCT;
    constexpr int NT = (NCT + 1) / 2;            // 8-column B tiles (two columns each)
    const int p = t & 1;
    // scales: 16 int8 per row, as four words; the group a lane uses in quadrant qd of half h
    // is 8 h + 2 qd + p: byte 2 (qd & 1) + p of word 2 h + qd / 2
    uint32_t sw0[4], sw1[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sw0[i] = ldw<ODD>(r0 + 192 + 4 * i);
        sw1[i] = ldw<ODD>(r1 + 192 + 4 * i);
    }
    // sign-extending byte selectors for bytes p and 2 + p
    const uint32_t b_lo = (uint32_t)p, b_hi = (uint32_t)(2 + p);
    const uint32_t sel_lo = b_lo | ((8u | b_lo) << 4) | ((8u | b_lo) << 8) | ((8u | b_lo) << 12);
    const uint32_t sel_hi = b_hi | ((8u | b_hi) << 4) | ((8u | b_hi) << 8) | ((8u | b_hi) << 12);
    int acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        // qh words (l = 4 t.., 16 + 4 t..) and ql words of quadrants 0 / 2 and 1 / 3
        const uint32_t u00 = ldw<ODD>(r0 + 128 + 32 * h + 4 * t), u01 = ldw<ODD>(r0 + 128 + 32 * h + 16 + 4 * t);
        const uint32_t u10 = ldw<ODD>(r1 + 128 + 32 * h + 4 * t), u11 = ldw<ODD>(r1 + 128 + 32 * h + 16 + 4 * t);
        const uint32_t wa00 = ldw<ODD>(r0 + 64 * h + 4 * t), wa01 = ldw<ODD>(r0 + 64 * h + 16 + 4 * t);
        const uint32_t wb00 = ldw<ODD>(r0 + 64 * h + 32 + 4 * t), wb01 = ldw<ODD>(r0 + 64 * h + 48 + 4 * t);
        const uint32_t wa10 = ldw<ODD>(r1 + 64 * h + 4 * t), wa11 = ldw<ODD>(r1 + 64 * h + 16 + 4 * t);
        const uint32_t wb10 = ldw<ODD>(r1 + 64 * h + 32 + 4 * t), wb11 = ldw<ODD>(r1 + 64 * h + 48 + 4 * t);
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
            auto q6 = [&](uint32_t wa, uint32_t wb, uint32_t u) -> uint32_t {
                const uint32_t w = (qd & 1) ? wb : wa;
                const uint32_t nib = (qd & 2) ? ((w >> 4) & 0x0F0F0F0Fu) : (w & 0x0F0F0F0Fu);
                const uint32_t hb = (qd == 0 ? (u << 4) : qd == 1 ? (u << 2) : qd == 2 ? u : (u >> 2)) & 0x30303030u;
                return nib | hb;
            };
            const uint32_t a0 = q6(wa00, wb00, u00), a1 = q6(wa10, wb10, u10);
            const uint32_t a2 = q6(wa01, wb01, u01), a3 = q6(wa11, wb11, u11);
            const int si = 2 * h + (qd >> 1);
            const int sc0 = prmt_sx(sw0[si], (qd & 1) ? sel_hi : sel_lo);
            const int sc1 = prmt_sx(sw1[si], (qd & 1) ? sel_hi : sel_lo);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                // B column g of tile j: column n = 2 j + g / 4, group (g / 2) & 1, vector g & 1
                const int n = 2 * j + (g >> 2), grp = (g >> 1) & 1, v = g & 1;
                uint32_t bw = 0u;
                if (n < NCT) bw = lds32(R + (uint32_t)((2 * n + v) * kVarStride + warp * kQK + 128 * h + 32 * qd + 16 * grp + 4 * t));
                int d[4];
                mma_u8s8(d, a0, a1, a2, a3, grp ? 0u : bw, grp ? bw : 0u);
                acc[j][0] += d[0] * sc0;
                acc[j][1] += d[1] * sc0;
                acc[j][2] += d[2] * sc1;
                acc[j][3] += d[3] * sc1;
            }
        }
    }
    // -32 d sum_g sc_g S_g: A = the scales as f16 (rows y0, y1; k = group), B = the sums
    // (f16 hi + lo of column n in B columns 2 n, 2 n + 1); lane t gets column t's pair
    const uint32_t swa0 = t < 2 ? sw0[0] : sw0[1], swb0 = t < 2 ? sw0[2] : sw0[3];
    const uint32_t swa1 = t < 2 ? sw1[0] : sw1[1], swb1 = t < 2 ? sw1[2] : sw1[3];
    const int sh = 16 * (t & 1);
    const uint32_t ma0 = i8x2_to_h2(swa0 >> sh), ma2 = i8x2_to_h2(swb0 >> sh);   // row y0: groups 2t.., 2t+8..
    const uint32_t ma1 = i8x2_to_h2(swa1 >> sh), ma3 = i8x2_to_h2(swb1 >> sh);   // row y1
    uint32_t sb0 = 0u, sb1 = 0u;
    if (g < NV) {
        const uint32_t so = R + act_i8::rec_sum_off(NCT) + (uint32_t)((warp * NV + g) * kGpb * 2 + 4 * t);
        sb0 = lds32(so);
        sb1 = lds32(so + 16);
    }
    float mn[4] = {0.f, 0.f, 0.f, 0.f};
    ptx::mma16816(mn, ma0, ma1, ma2, ma3, sb0, sb1);
    const float d0 = __half2float(__ushort_as_half((unsigned short)lds16(r0 + 208)));
    const float d1 = __half2float(__ushort_as_half((unsigned short)lds16(r1 + 208)));
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int n = 2 * j + (t >> 1);
        // the min term of column n sits in lane (g, n); the group-parity-0 lane adds it
        const float m0 = __shfl_sync(0xffffffffu, fmaf(mn[1], 1.0f / 2048.0f, mn[0]), 4 * g + (n & 3));
        const float m1 = __shfl_sync(0xffffffffu, fmaf(mn[3], 1.0f / 2048.0f, mn[2]), 4 * g + (n & 3));
        if (n < NCT) {
            const float s = __uint_as_float(lds32(R + act_i8::rec_scale_off(NCT) + (uint32_t)(n * 8 + warp) * 4));
            const float hi0 = (float)acc[j][0], lo0 = (float)acc[j][1];
            const float hi1 = (float)acc[j][2], lo1 = (float)acc[j][3];
            ya[j][0] += d0 * (s * fmaf(lo0, 1.0f / 254.0f, hi0) - (p == 0 ? 32.0f * m0 : 0.0f));
            ya[j][1] += d1 * (s * fmaf(lo1, 1.0f / 254.0f, hi1) - (p == 0 ? 32.0f * m1 : 0.0f));
        }
    }
}

// One activation column: the four B columns the column needs (2 groups x hi / lo) fill half
// of an MMA, so the other half carries the next quadrant -- B column 4 qp + 2 grp + v holds
// group grp of vector v for the quadrants qd % 2 == qp and zeros for the others -- and the
// quadrant pairs (0, 1), (2, 3) of each half accumulate in one MMA chain.  Lane t's C columns
// are then quadrant parity t / 2, group t % 2: its scale is byte t of one scale word, and it
// scales one chain (4 IMADs) where the one-tile form scales every quadrant with lanes of zero
// columns.  Accumulates this lane's share of rows y0, y1 into ya[0..1] (summed over the quad
// at the flush; lane t = 0 carries the -32 offset).
template <bool ODD>
__device__ __forceinline__ void q6_block_spread(uint32_t r0, uint32_t r1, uint32_t R, int warp, int g, int t,
                                                float (&ya)[2]) {
    const int bqp = g >> 2, bgrp = (g >> 1) & 1, bvec = g & 1;
    uint32_t sw0[4], sw1[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sw0[i] = ldw<ODD>(r0 + 192 + 4 * i);
        sw1[i] = ldw<ODD>(r1 + 192 + 4 * i);
    }
    const uint32_t sel = (uint32_t)t | ((8u | t) << 4) | ((8u | t) << 8) | ((8u | t) << 12);
    const uint32_t boff = R + (uint32_t)(bvec * kVarStride + warp * kQK + 16 * bgrp + 4 * t);
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t u00 = ldw<ODD>(r0 + 128 + 32 * h + 4 * t), u01 = ldw<ODD>(r0 + 128 + 32 * h + 16 + 4 * t);
        const uint32_t u10 = ldw<ODD>(r1 + 128 + 32 * h + 4 * t), u11 = ldw<ODD>(r1 + 128 + 32 * h + 16 + 4 * t);
        const uint32_t wa00 = ldw<ODD>(r0 + 64 * h + 4 * t), wa01 = ldw<ODD>(r0 + 64 * h + 16 + 4 * t);
        const uint32_t wb00 = ldw<ODD>(r0 + 64 * h + 32 + 4 * t), wb01 = ldw<ODD>(r0 + 64 * h + 48 + 4 * t);
        const uint32_t wa10 = ldw<ODD>(r1 + 64 * h + 4 * t), wa11 = ldw<ODD>(r1 + 64 * h + 16 + 4 * t);
        const uint32_t wb10 = ldw<ODD>(r1 + 64 * h + 32 + 4 * t), wb11 = ldw<ODD>(r1 + 64 * h + 48 + 4 * t);
        int d[2][4];
        // chains c = quadrants (0, 1) and (2, 3), their MMAs interleaved
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int qd = 2 * c + jj;
                auto q6 = [&](uint32_t wa, uint32_t wb, uint32_t u) -> uint32_t {
                    const uint32_t w = (qd & 1) ? wb : wa;
                    const uint32_t nib = (qd & 2) ? ((w >> 4) & 0x0F0F0F0Fu) : (w & 0x0F0F0F0Fu);
                    const uint32_t hb = (qd == 0 ? (u << 4) : qd == 1 ? (u << 2) : qd == 2 ? u : (u >> 2)) & 0x30303030u;
                    return nib | hb;
                };
                const uint32_t a0 = q6(wa00, wb00, u00), a1 = q6(wa10, wb10, u10);
                const uint32_t a2 = q6(wa01, wb01, u01), a3 = q6(wa11, wb11, u11);
                const uint32_t bw = bqp == jj ? lds32(boff + (uint32_t)(128 * h + 32 * qd)) : 0u;
                if (jj == 0)
                    mma_u8s8(d[c], a0, a1, a2, a3, bgrp ? 0u : bw, bgrp ? bw : 0u);
                else
                    mma_u8s8_acc(d[c], a0, a1, a2, a3, bgrp ? 0u : bw, bgrp ? bw : 0u);
            }
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            // group 8 h + 2 (2 c + t / 2) + t % 2 = 8 h + 4 c + t: byte t of word 2 h + c
            const int sc0 = prmt_sx(sw0[2 * h + c], sel), sc1 = prmt_sx(sw1[2 * h + c], sel);
            acc[0] += d[c][0] * sc0;
            acc[1] += d[c][1] * sc0;
            acc[2] += d[c][2] * sc1;
            acc[3] += d[c][3] * sc1;
        }
    }
    // -32 d sum_g sc_g S_g as in q6_block (lane t = 0 holds column 0's pair)
    const uint32_t swa0 = t < 2 ? sw0[0] : sw0[1], swb0 = t < 2 ? sw0[2] : sw0[3];
    const uint32_t swa1 = t < 2 ? sw1[0] : sw1[1], swb1 = t < 2 ? sw1[2] : sw1[3];
    const int sh = 16 * (t & 1);
    const uint32_t ma0 = i8x2_to_h2(swa0 >> sh), ma2 = i8x2_to_h2(swb0 >> sh);
    const uint32_t ma1 = i8x2_to_h2(swa1 >> sh), ma3 = i8x2_to_h2(swb1 >> sh);
    uint32_t sb0 = 0u, sb1 = 0u;
    if (g < 2) {
        const uint32_t so = R + act_i8::rec_sum_off(1) + (uint32_t)((warp * 2 + g) * kGpb * 2 + 4 * t);
        sb0 = lds32(so);
        sb1 = lds32(so + 16);
    }
    float mn[4] = {0.f, 0.f, 0.f, 0.f};
    ptx::mma16816(mn, ma0, ma1, ma2, ma3, sb0, sb1);
    const float d0 = __half2float(__ushort_as_half((unsigned short)lds16(r0 + 208)));
    const float d1 = __half2float(__ushort_as_half((unsigned short)lds16(r1 + 208)));
    const float s = __uint_as_float(lds32(R + act_i8::rec_scale_off(1) + (uint32_t)warp * 4));
    const float m0 = t == 0 ? 32.0f * fmaf(mn[1], 1.0f / 2048.0f, mn[0]) : 0.0f;
    const float m1 = t == 0 ? 32.0f * fmaf(mn[3], 1.0f / 2048.0f, mn[2]) : 0.0f;
    ya[0] += d0 * (s * fmaf((float)acc[1], 1.0f / 254.0f, (float)acc[0]) - m0);
    ya[1] += d1 * (s * fmaf((float)acc[3], 1.0f / 254.0f, (float)acc[2]) - m1);
}

template <int NCT>
__global__ void __launch_bounds__(kThreads, 2) q6k_i8_kernel(const __grid_constant__ I8Params p) {
    constexpr int S = stages_for(NCT);
    constexpr int NT = (NCT + 1) / 2;
    constexpr uint32_t RB = rec_bytes(NCT);
    extern __shared__ uint8_t q6i8_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q6i8_smem_raw) + 127) & ~uintptr_t(127));
    uint8_t* boxes = smem;                                        // S x 26880
    uint8_t* recs = boxes + (size_t)S * kBoxBytes;                // S x RB
    float* red = reinterpret_cast<float*>(recs + (size_t)S * RB); // 2 x [8 warps][16 rows][NCT][2 parities]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kWarps * kTileRows * NCT * 2);
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
        if (lane != 0) return;
        auto load_weights = [&](int s, long long u) {
            const int tile = (int)(u / p.nst), si = (int)(u % p.nst);
            const uint32_t fb = ptx::smem_u32(&full[s]);
            ptx::mbar_expect_tx(fb, kBoxBytes + RB);
            tma_load_2d(ptx::smem_u32(boxes + (size_t)s * kBoxBytes), &p.tm_w, fb, si * kU64PerUnit, tile * kTileRows);
        };
        auto load_record = [&](int s, long long u) {
            const int si = (int)(u % p.nst);
            ptx::bulk_load(ptx::smem_u32(recs + (size_t)s * RB), p.rec + (size_t)si * RB, RB, ptx::smem_u32(&full[s]));
        };
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
        volatile int no_abort = 0;
        for (int s = 0; s < S && s < issued; ++s) {
            const int last = s + (issued - 1 - s) / S * S;
            ptx::mbar_wait(ptx::smem_u32(&full[s]), (last / S) & 1, &no_abort, p.err);
        }
        return;
    }

    ptx::pdl_wait();   // Y (zeroed by the prep kernel) comes after the previous kernels
    const int g = lane >> 2, t = lane & 3;
    const uint32_t box_base = ptx::smem_u32(boxes), rec_base = ptx::smem_u32(recs);
    const int tid = threadIdx.x;
    bool ok = true;
    int it = 0, flushes = 0;
    float ya[NT][2];
#pragma unroll
    for (int j = 0; j < NT; ++j) ya[j][0] = ya[j][1] = 0.0f;
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
            const uint32_t r0 = W + (uint32_t)(g * kRowBytes + warp * kBlk), r1 = r0 + 8 * kRowBytes;
            if constexpr (NCT == 1) {
                if (warp & 1)
                    q6_block_spread<true>(r0, r1, R, warp, g, t, ya[0]);
                else
                    q6_block_spread<false>(r0, r1, R, warp, g, t, ya[0]);
            } else {
                if (warp & 1)
                    q6_block<NCT, true>(r0, r1, R, warp, g, t, ya);
                else
                    q6_block<NCT, false>(r0, r1, R, warp, g, t, ya);
            }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&empty[s]));
        ++it;
        ++u;
        const bool tile_end = ++si == p.nst || u == u1;
        if (!tile_end) continue;
        // ---- flush: the warps' partial rows (two group parities each), summed in a fixed order
        float* rb = red + (flushes & 1) * (kWarps * kTileRows * NCT * 2);
        ++flushes;
        if constexpr (NCT == 1) {
            // the quad's four shares of column 0: pairs (t, t + 2) here, the two sums below
            const float v0 = ya[0][0] + __shfl_xor_sync(0xffffffffu, ya[0][0], 2);
            const float v1 = ya[0][1] + __shfl_xor_sync(0xffffffffu, ya[0][1], 2);
            if (t < 2) {
                rb[(warp * kTileRows + g) * 2 + t] = v0;
                rb[(warp * kTileRows + g + 8) * 2 + t] = v1;
            }
            ya[0][0] = ya[0][1] = 0.0f;
        } else {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int n = 2 * j + (t >> 1);
                if (n < NCT) {
                    rb[((warp * kTileRows + g) * NCT + n) * 2 + (t & 1)] = ya[j][0];
                    rb[((warp * kTileRows + g + 8) * NCT + n) * 2 + (t & 1)] = ya[j][1];
                }
                ya[j][0] = ya[j][1] = 0.0f;
            }
        }
        consumer_sync();
        const int r = tid & (kTileRows - 1), n = tid >> 4;
        const int m0 = tile * kTileRows;
        if (tid < kTileRows * p.N && ok && !*abort_flag && m0 + r < p.M) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w)
                v += rb[((w * kTileRows + r) * NCT + n) * 2] + rb[((w * kTileRows + r) * NCT + n) * 2 + 1];
            red_add(reinterpret_cast<float*>(p.y + (size_t)n * p.y_cs) + m0 + r, v);
        }
        ++tile;
        si = 0;
    }
}

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
    if (occ < 1) return fail(MLZC_ERR_CUDA, "Q6_K int8 kernel does not fit on an SM");
    cache[{key, dev}] = occ * sms;
    *out = occ * sms;
    return MLZC_OK;
}

template <int NCT>
int launch_main(const DeviceCtx* c, I8Params& p, cudaStream_t s) {
    const size_t smem = i8_smem_bytes(NCT);
    int slots = 0;
    const int st = i8_slots(q6k_i8_kernel<NCT>, smem, &slots);
    if (st != MLZC_OK) return st;
    // ranges of at least nst - 1 units: at most two pieces per tile (0 + a + b = 0 + b + a)
    const long long cap = p.nst > 1 ? p.units / (p.nst - 1) : p.units;
    // 92 % of the resident slots: the free ones let the next call's kernels start during this
    // one's tail (B200 sweep of 34-100 % on the C3 / C6 steps: 92 % best at batch 1, 2 and 4,
    // e.g. C3 batch 1 27.0 vs 28.5 us per step, C6 batch 1 34.3 vs 36.3)
    const long long use = std::max<long long>(1, (long long)slots * 23 / 25);
    const int grid = (int)std::max<long long>(1, std::min<long long>({p.units, use, cap}));
    p.err = c->err;
    MLZC_CUDA_TRY(launch_pdl(q6k_i8_kernel<NCT>, dim3((unsigned)grid), dim3(kThreads), smem, s, p));
    count_launch();
    return MLZC_OK;
}

int nct_of(int64_t N) { return N <= 1 ? 1 : N <= 2 ? 2 : 4; }

size_t rec_total(int64_t K, int64_t N) {
    const int nblk = (int)(K / kQK), nst = (nblk + kWarps - 1) / kWarps;
    return ((size_t)nst * rec_bytes(nct_of(N)) + 255) / 256 * 256;
}

}  // namespace

bool q6k_i8_applicable(int64_t M, int64_t K, int64_t N) {
    return N >= 1 && N <= 4 && K >= 1024 && K % 1024 == 0 && M >= 1 && M <= ((int64_t)1 << 30) &&
           K / kQK <= ((int64_t)1 << 24);
}

size_t q6k_i8_workspace_bytes(int64_t K, int64_t N) { return rec_total(K, N); }

int launch_q6k_i8(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                  size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                  cudaStream_t s) {
    if (!q6k_i8_applicable(M, K, N)) return fail(MLZC_ERR_UNSUPPORTED, "Q6_K int8 path: shape not taken");
    if ((uintptr_t)w % 16 || w_row_bytes % 16 || (uintptr_t)x % 16 || x_col_bytes % 16)
        return fail(MLZC_ERR_UNSUPPORTED, "Q6_K int8 path: needs 16-byte aligned rows");
    const size_t need = rec_total(K, N);
    if (!ws || ws_bytes < need || (uintptr_t)ws % 16)
        return fail(MLZC_ERR_NOMEM, "Q6_K: workspace of %zu bytes needed, %zu given", need, ws_bytes);
    auto enc = tensor_map_encoder();
    if (!enc) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const int nct = nct_of(N);
    I8Params p{};
    p.rec = static_cast<const char*>(ws);
    p.y = reinterpret_cast<char*>(y);
    p.y_cs = y_col_bytes;
    p.M = (int)M;
    p.nblk = (int)(K / kQK);
    p.nst = (p.nblk + kWarps - 1) / kWarps;
    p.N = (int)N;
    p.tiles = (int)((M + kTileRows - 1) / kTileRows);
    p.units = (long long)p.tiles * p.nst;
    p.early = weights_before_wait() ? 1 : 0;
    const cuuint64_t dims[2] = {(cuuint64_t)p.nblk * kBlk / 8, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)w_row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)kU64PerUnit, (cuuint32_t)kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&p.tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MLZC_ERR_UNSUPPORTED, "Q6_K int8 path: rows not expressible as a TMA map (%d)", (int)r);
    {
        const int items = p.nst * kWarps * nct;
        const long long zero_ctas = std::min<long long>(148, ((long long)M * N + 2047) / 2048);
        const unsigned pg = (unsigned)std::max<long long>((items + 7) / 8, zero_ctas);
        MLZC_CUDA_TRY(launch_pdl(act_i8::prep_kernel<kGpb>, dim3(pg), dim3(256), 0, s, reinterpret_cast<const char*>(x),
                                 x_col_bytes, (int)N, nct, p.nblk, p.nst, rec_bytes(nct), static_cast<char*>(ws), p.y,
                                 p.y_cs, p.M));
        count_launch();
    }
    if (nct == 1) return launch_main<1>(c, p, s);
    if (nct == 2) return launch_main<2>(c, p, s);
    return launch_main<4>(c, p, s);
}

}  // namespace mlzc
