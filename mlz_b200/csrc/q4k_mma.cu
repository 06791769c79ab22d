// q4k_mma.cu -- Q4_K-weight mul_mat on the tensor cores (mma.sync m16n8k16, f16 x f16 -> f32).
//
// Replaces the Q4_K branch of ggml_simd_try_mul_mat (src/simd/ggml_simd_hook.cpp:188-231,
// 238-299): one simd_vec_dot_q4_k_q8_k (kernels/x86/vec/vec_dot_q4_k_q8_k_avx2.asm:38-266)
// per (row, column) over Q8_K-quantised activations.  Here the activations keep f32
// precision up to one f16 rounding (the parity bar is the dequantised-f32 product).
//
// Q4_K block (GGUF, 144 bytes per 256 weights): d (f16) @0, dmin (f16) @2, twelve bytes of
// packed 6-bit (sc, m) for the 8 sub-blocks of 32 @4, 128 nibble bytes @16 where byte b of
// 32-byte chunk c holds element b of sub-block 2c (low nibble) and of sub-block 2c+1 (high
// nibble).  Weight = d * sc_j * q - dmin * m_j, so per block and activation column
//     y += d * sum_i (sc_j q_i) x_i  -  dmin * sum_j m_j S_j,    S_j = sum_{i in j} x_i.
//
// Tensor-core form, weights as A (16 rows per MMA), activations as B (8 columns):
//   * sc_j * q_i is an integer <= 945, exact in f16.  A nibble pair becomes that f16 pair
//     with one LOP3 (0x6400 exponent trick: the bits read as 1024 + q, or 1024 + 16 q for a
//     high nibble) and one HFMA2 (* sc - 1024 sc, or * sc/16 - 64 sc; exact), so a whole
//     block accumulates in one MMA chain with no per-sub-block rescaling; d scales the sum.
//   * The k order inside a block is permuted so that quad thread q (lane % 4) holds exactly
//     chunk q, i.e. sub-blocks 2q and 2q+1: a thread unpacks only those two (sc, m) pairs per
//     row, and sums S_j for them from the activations it loaded itself.
//   * The min term is one more MMA pair per block: A = m_j (exact) at k = 2q, 2q+1, B = S_j
//     split into f16 hi + lo parts.
// Activations are rounded to f16 once (relative error <= 2^-11 per element, random across
// the sum).  A CTA = 8 warps over 32 rows x 8 columns; warps take the K blocks in turn,
// prefetch the next block's weights into registers, and the CTA sums the warps' partial
// rows in a fixed order (results repeat bit for bit).
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

using ptx::mma16816;

constexpr int kQK = 256;
constexpr int kQ4KBytes = 144;
constexpr int kQWarps = 8;
constexpr int kQThreads = kQWarps * 32;
constexpr int kQRows = 32;     // rows per CTA: two 16-row MMA tiles
constexpr int kQCols = 8;      // activation columns per CTA: one 8-column MMA tile

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// One row's share of a block for this thread: header (d, dmin, scales) and its 32-byte chunk.
struct RowBlock {
    uint4 hdr, qa, qb;
};

__device__ __forceinline__ RowBlock load_row_block(const char* blk, int q4) {
    RowBlock r;
    r.hdr = ld_stream(blk);
    r.qa = ld_stream(blk + 16 + 32 * q4);
    r.qb = ld_stream(blk + 16 + 32 * q4 + 16);
    return r;
}

// Per row and block: the HFMA2 constants that turn nibble bits into sc * q for sub-blocks
// 2c (low nibbles) and 2c+1 (high nibbles), the (m_2c, m_2c+1) pair, and d, dmin.
struct RowScales {
    __half2 mul_lo, add_lo, mul_hi, add_hi;
    uint32_t mpair;
    float d, dmin;
};

__device__ __forceinline__ RowScales row_scales(const uint4& hdr, int c) {
    // scale bytes s[0..11] = hdr.y (s0-s3), hdr.z (s4-s7), hdr.w (s8-s11); this thread needs
    // sub-blocks j = 2c, 2c+1, i.e. byte pair j' = 2 (c & 1), +1 of each word
    const int sh = 16 * (c & 1);
    const uint32_t A = (hdr.y >> sh) & 0xFFFFu, B = (hdr.z >> sh) & 0xFFFFu, Cw = (hdr.w >> sh) & 0xFFFFu;
    uint32_t sc2, m2;
    if (c < 2) {   // j < 4: sc = s[j] & 63, m = s[j+4] & 63
        sc2 = A & 0x3F3Fu;
        m2 = B & 0x3F3Fu;
    } else {       // j >= 4: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4, m = (s[j+4] >> 4) | (s[j] >> 6) << 4
        sc2 = (Cw & 0x0F0Fu) | ((A >> 2) & 0x3030u);
        m2 = ((Cw >> 4) & 0x0F0Fu) | ((B >> 2) & 0x3030u);
    }
    const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
    const __half2 sch = __hsub2(u2h(__byte_perm(sc2, 0x6464u, 0x5140)), k1024);   // (sc_2c, sc_2c+1)
    RowScales r;
    r.mpair = h2u(__hsub2(u2h(__byte_perm(m2, 0x6464u, 0x5140)), k1024));          // (m_2c, m_2c+1)
    const __half2 lo = __low2half2(sch), hi = __high2half2(sch);
    r.mul_lo = lo;
    r.add_lo = __hmul2(lo, __float2half2_rn(-1024.0f));
    r.mul_hi = __hmul2(hi, __float2half2_rn(0.0625f));
    r.add_hi = __hmul2(hi, __float2half2_rn(-64.0f));
    const __half2 dd = u2h(hdr.x);
    r.d = __low2float(dd);
    r.dmin = __high2float(dd);
    return r;
}

// sc * q for the nibble pair (bytes 0 and 2 of w) of the low or high half.
__device__ __forceinline__ uint32_t deq_lo(uint32_t w, const RowScales& s) {
    return h2u(__hfma2(u2h((w & 0x000F000Fu) | 0x64006400u), s.mul_lo, s.add_lo));
}
__device__ __forceinline__ uint32_t deq_hi(uint32_t w, const RowScales& s) {
    return h2u(__hfma2(u2h((w & 0x00F000F0u) | 0x64006400u), s.mul_hi, s.add_hi));
}

__device__ __forceinline__ uint32_t word_of(const RowBlock& r, int wi) {
    switch (wi) {
        case 0: return r.qa.x;
        case 1: return r.qa.y;
        case 2: return r.qa.z;
        case 3: return r.qa.w;
        case 4: return r.qb.x;
        case 5: return r.qb.y;
        case 6: return r.qb.z;
        default: return r.qb.w;
    }
}

__global__ void __launch_bounds__(kQThreads)
q4k_mma_kernel(const char* __restrict__ W, size_t w_rs, int M, int nblk, const char* __restrict__ X, size_t x_cs,
               int N, char* __restrict__ Y, size_t y_cs) {
    __shared__ float red[kQWarps][kQRows * kQCols];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int q4 = lane & 3;
    const int m0 = blockIdx.y * kQRows;
    const int n0 = blockIdx.x * kQCols;

    // rows of this thread: tile t, half h -> m0 + 16 t + g + 8 h (clamped for loads)
    const char* rowp[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = min(m0 + 16 * (i >> 1) + g + 8 * (i & 1), M - 1);
        rowp[i] = W + (size_t)r * w_rs;
    }
    const bool col_ok = n0 + g < N;
    const float* xcol = reinterpret_cast<const float*>(X + (size_t)(col_ok ? n0 + g : 0) * x_cs);

    float y[2][4] = {};
    RowBlock cur[4], nxt[4];
    int kb = warp;
    if (kb < nblk) {
#pragma unroll
        for (int i = 0; i < 4; ++i) cur[i] = load_row_block(rowp[i] + (size_t)kb * kQ4KBytes, q4);
    }
    for (; kb < nblk; kb += kQWarps) {
        const int kn = kb + kQWarps;
        if (kn < nblk) {
#pragma unroll
            for (int i = 0; i < 4; ++i) nxt[i] = load_row_block(rowp[i] + (size_t)kn * kQ4KBytes, q4);
        }
        RowScales sc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[i] = row_scales(cur[i].hdr, q4);

        float acc[2][4] = {};
        float S[2] = {0.0f, 0.0f};
        const float4* xb = reinterpret_cast<const float4*>(xcol + (size_t)kb * kQK + 64 * q4);
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
            float4 xv[8];
#pragma unroll
            for (int wi = 0; wi < 8; ++wi) xv[wi] = col_ok ? xb[8 * hi + wi] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int wi = 0; wi < 8; ++wi) {
                S[hi] += (xv[wi].x + xv[wi].y) + (xv[wi].z + xv[wi].w);
                const uint32_t b0 = h2u(__floats2half2_rn(xv[wi].x, xv[wi].z));
                const uint32_t b1 = h2u(__floats2half2_rn(xv[wi].y, xv[wi].w));
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const uint32_t w0 = word_of(cur[2 * t], wi), w1 = word_of(cur[2 * t + 1], wi);
                    uint32_t a0, a1, a2, a3;
                    if (hi == 0) {
                        a0 = deq_lo(w0, sc[2 * t]);
                        a1 = deq_lo(w1, sc[2 * t + 1]);
                        a2 = deq_lo(w0 >> 8, sc[2 * t]);
                        a3 = deq_lo(w1 >> 8, sc[2 * t + 1]);
                    } else {
                        a0 = deq_hi(w0, sc[2 * t]);
                        a1 = deq_hi(w1, sc[2 * t + 1]);
                        a2 = deq_hi(w0 >> 8, sc[2 * t]);
                        a3 = deq_hi(w1 >> 8, sc[2 * t + 1]);
                    }
                    mma16816(acc[t], a0, a1, a2, a3, b0, b1);
                }
            }
        }
        // min term: sum_j m_j S_j with S as f16 hi + lo
        const __half2 Sh = __floats2half2_rn(S[0], S[1]);
        const float2 Shf = __half22float2(Sh);
        const uint32_t bs_hi = h2u(Sh), bs_lo = h2u(__floats2half2_rn(S[0] - Shf.x, S[1] - Shf.y));
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            float mn[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(mn, sc[2 * t].mpair, sc[2 * t + 1].mpair, 0u, 0u, bs_hi, 0u);
            mma16816(mn, sc[2 * t].mpair, sc[2 * t + 1].mpair, 0u, 0u, bs_lo, 0u);
            // rows g (e = 0, 1) and g + 8 (e = 2, 3)
            y[t][0] += sc[2 * t].d * acc[t][0] - sc[2 * t].dmin * mn[0];
            y[t][1] += sc[2 * t].d * acc[t][1] - sc[2 * t].dmin * mn[1];
            y[t][2] += sc[2 * t + 1].d * acc[t][2] - sc[2 * t + 1].dmin * mn[2];
            y[t][3] += sc[2 * t + 1].d * acc[t][3] - sc[2 * t + 1].dmin * mn[3];
        }
        if (kn < nblk) {
#pragma unroll
            for (int i = 0; i < 4; ++i) cur[i] = nxt[i];
        }
    }

    // partial rows of every warp -> fixed-order sum
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int r = 16 * t + g;
        red[warp][r * kQCols + 2 * q4] = y[t][0];
        red[warp][r * kQCols + 2 * q4 + 1] = y[t][1];
        red[warp][(r + 8) * kQCols + 2 * q4] = y[t][2];
        red[warp][(r + 8) * kQCols + 2 * q4 + 1] = y[t][3];
    }
    __syncthreads();
    const int r = threadIdx.x % kQRows, cidx = threadIdx.x / kQRows;
    if (m0 + r < M && n0 + cidx < N) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kQWarps; ++w) v += red[w][r * kQCols + cidx];
        reinterpret_cast<float*>(Y + (size_t)(n0 + cidx) * y_cs)[m0 + r] = v;
    }
}

}  // namespace

int launch_q4k_mma(const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x, size_t x_col_bytes,
                   int64_t N, float* y, size_t y_col_bytes, cudaStream_t s) {
    if (K % kQK != 0) return fail(MLZC_ERR_INVALID, "Q4_K: K=%lld is not a multiple of 256", (long long)K);
    if ((uintptr_t)w % 16 || w_row_bytes % 16 || (uintptr_t)x % 16 || x_col_bytes % 16)
        return fail(MLZC_ERR_INVALID, "Q4_K: weights and activations must be 16-byte aligned");
    if (M > INT32_MAX / 2 || K / kQK > INT32_MAX) return fail(MLZC_ERR_INVALID, "Q4_K: dimensions too large");
    const dim3 grid((unsigned)((N + kQCols - 1) / kQCols), (unsigned)((M + kQRows - 1) / kQRows));
    if (grid.y > 65535u) return fail(MLZC_ERR_INVALID, "Q4_K: M=%lld beyond %d rows", (long long)M, 65535 * kQRows);
    q4k_mma_kernel<<<grid, kQThreads, 0, s>>>(static_cast<const char*>(w), w_row_bytes, (int)M, (int)(K / kQK),
                                              reinterpret_cast<const char*>(x), x_col_bytes, (int)N,
                                              reinterpret_cast<char*>(y), y_col_bytes);
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

}  // namespace mlzc
