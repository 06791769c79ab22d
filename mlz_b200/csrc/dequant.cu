// dequant.cu -- Q4_K / Q6_K weights at prefill sizes: the rows are dequantised to f16 once
// per call into the workspace, then the tcgen05 F16 GEMM (gemm_tc.cu) runs on them.
//
// Replaces, for many activation columns, the K-quant branch of ggml_simd_try_mul_mat
// (src/simd/ggml_simd_hook.cpp:234-301: one simd_vec_dot_q4_k_q8_k / _q6_k_q8_k per (row,
// column)).  The decode kernels (q4k_i8.cu, q4k_ring.cu, q4k_mma.cu, q6k_i8.cu, q6k.cu)
// stream the blocks once per group of at most 16 columns; with hundreds of columns that is
// hundreds of passes over W, while dequantise + GEMM reads the blocks once, writes and reads
// 2 bytes per weight, and runs the contraction on the tensor cores (compute-bound there).
//
// Arithmetic: each weight is formed in f32 exactly as the dequantised-F32 reference forms it
// -- Q4_K (d sc) q - (dmin m), Q6_K (d sc) (q - 32), the GGUF layouts restated in the file
// headers of q4k_mma.cu and q6k.cu -- and rounded to f16 (RNE): relative error <= 2^-11 per
// weight, the same as the f16 rounding of the activations the GEMM applies.
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int kQK = 256;
constexpr int kQ4KBytes = 144;
constexpr int kQ6KBytes = 210;

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// A row's weights are rounded to f16 after scaling by 2^-e, the smallest power of two that
// brings the row's largest possible |w| (from its block scales) within the f16 range; e = 0
// for every row of a real model, where the f16 weights are the RNE roundings of the f32
// dequantised ones.  row_scale[m] = 2^e, and the GEMM's epilogue multiplies those rows of Y
// back (exact: powers of two).
__device__ __forceinline__ int row_exponent(float bound) {
    if (!(bound > 65504.0f)) return 0;   // (also NaN / inf scales: left to propagate)
    int e = 0;
    const float f = frexpf(bound / 65504.0f, &e);   // bound / 65504 = f 2^e, f in [0.5, 1)
    return f == 0.5f ? e - 1 : e;
}

// One CTA per row at a time (grid-stride over rows): the row's exponent from its block headers
// -- |w| <= |d| 63 15 + |dmin| 63 (Q4_K), |w| <= |d| 128 32 (Q6_K) -- reduced over the CTA,
// row_scale[m] = 2^e, then the row's weights times 2^-e, one block per warp at a time.  The
// headers' cache lines are read again by the dequantisation right after, from L1 / L2.
constexpr int kDqThreads = 128;

template <bool Q6>
__device__ __forceinline__ float block_bound(const unsigned char* blk) {
    if constexpr (Q6) {
        return fabsf(__half2float(__ushort_as_half((unsigned short)(blk[208] | (blk[209] << 8))))) * 4096.0f;
    } else {
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk)));
        const float dmin = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk + 2)));
        return fabsf(d) * 945.0f + fabsf(dmin) * 63.0f;
    }
}

// Q4_K: lane l of a warp writes 16-byte chunk l of a block's 512-byte f16 image (positions
// 8 l .. 8 l + 7: sub-block j = l / 4, 8 bytes of its nibbles), so a warp's store is one
// contiguous block.  The loads of kDqU blocks are issued before any is converted.
struct Q4Raw {
    uint32_t dd;      // d | dmin << 16 (f16 bits)
    uint32_t s0, s1;  // the scale bytes sub-block j needs
    uint2 q;          // 8 bytes of nibbles
};
__device__ __forceinline__ Q4Raw q4k_load(const unsigned char* blk, int l) {
    const int j = l >> 2, c = j >> 1;
    Q4Raw r;
    r.dd = *reinterpret_cast<const uint32_t*>(blk);
    const unsigned char* sc = blk + 4;
    // j < 4: sc[j] & 63, sc[j + 4] & 63; else sc[j + 4], sc[j - 4] >> 6, sc[j] >> 6
    r.s0 = j < 4 ? sc[j] : sc[j + 4];
    r.s1 = j < 4 ? sc[j + 4] : (uint32_t)sc[j - 4] | ((uint32_t)sc[j] << 8);
    r.q = *reinterpret_cast<const uint2*>(blk + 16 + 32 * c + 8 * (l & 3));
    return r;
}
// Four bytes of x (0..255 each) -> exact floats: each byte under the 2^23 exponent, minus 2^23.
__device__ __forceinline__ void bytes_to_f32(uint32_t x, float (&f)[4]) {
#pragma unroll
    for (int b = 0; b < 4; ++b)
        f[b] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7650u | (uint32_t)b)) - 8388608.0f;
}

// w = (d sc) q - (dmin m) in f32: d sc and dmin m are exact (11 x 6 bits), and so is (d sc) q
// (4 more bits), so one FMA rounds exactly where the product-then-difference does.
__device__ __forceinline__ uint4 q4k_convert(const Q4Raw& r, int l, float sc_row, bool scaled) {
    const int j = l >> 2, hi = j & 1;
    const float d = __half2float(__ushort_as_half((unsigned short)(r.dd & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(r.dd >> 16)));
    int s, m;
    if (j < 4) {
        s = r.s0 & 63;
        m = r.s1 & 63;
    } else {
        s = (r.s0 & 0x0F) | (((r.s1 & 0xFF) >> 6) << 4);
        m = (r.s0 >> 4) | (((r.s1 >> 8) >> 6) << 4);
    }
    const float dj = d * (float)s, mj = dmin * (float)m;
    const uint32_t x0 = (hi ? r.q.x >> 4 : r.q.x) & 0x0F0F0F0Fu, x1 = (hi ? r.q.y >> 4 : r.q.y) & 0x0F0F0F0Fu;
    float f[8];
    float (&f0)[4] = *reinterpret_cast<float(*)[4]>(&f[0]);
    float (&f1)[4] = *reinterpret_cast<float(*)[4]>(&f[4]);
    bytes_to_f32(x0, f0);
    bytes_to_f32(x1, f1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        f[i] = fmaf(dj, f[i], -mj);
        if (scaled) f[i] *= sc_row;
    }
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

// Q6_K: lane l writes positions p = 8 l .. 8 l + 7 (h = p / 128, quadrant k, l0 = p % 32; scale
// group p / 16).  Q6_K blocks are 2-byte aligned only: the 8-byte runs are read as 2-byte words.
struct Q6Raw {
    uint32_t dsc;            // d (f16 bits) | scale byte << 16
    uint32_t ql[2], qh[2];   // the 8 bytes of low nibbles and high bits, as two words each
};
__device__ __forceinline__ Q6Raw q6k_load(const unsigned char* blk, int l) {
    const int p0 = 8 * l, h = p0 / 128, k = (p0 % 128) / 32, l0 = p0 % 32;
    const unsigned short* ql = reinterpret_cast<const unsigned short*>(blk + 64 * h + 32 * (k % 2) + l0);
    const unsigned short* qh = reinterpret_cast<const unsigned short*>(blk + 128 + 32 * h + l0);
    Q6Raw r;
    r.dsc = (uint32_t)*reinterpret_cast<const unsigned short*>(blk + 208) | ((uint32_t)blk[192 + (l >> 1)] << 16);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        r.ql[i] = (uint32_t)ql[2 * i] | ((uint32_t)ql[2 * i + 1] << 16);
        r.qh[i] = (uint32_t)qh[2 * i] | ((uint32_t)qh[2 * i + 1] << 16);
    }
    return r;
}
// w = (d sc) (q - 32) = fma(d sc, q, -32 d sc): the exact product rounded once either way.
__device__ __forceinline__ uint4 q6k_convert(const Q6Raw& r, int l, float sc_row, bool scaled) {
    const int p0 = 8 * l, k = (p0 % 128) / 32;
    const float d = __half2float(__ushort_as_half((unsigned short)(r.dsc & 0xFFFF)));
    const float ds = d * (float)(signed char)(r.dsc >> 16);
    float f[8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t q = ((r.ql[i] >> (4 * (k / 2))) & 0x0F0F0F0Fu) | (((r.qh[i] >> (2 * k)) & 0x03030303u) << 4);
        float (&fi)[4] = *reinterpret_cast<float(*)[4]>(&f[4 * i]);
        bytes_to_f32(q, fi);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        f[i] = fmaf(ds, f[i], -32.0f * ds);
        if (scaled) f[i] *= sc_row;
    }
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

constexpr int kDqU = 4;   // blocks per warp in flight

template <bool Q6>
__global__ void __launch_bounds__(kDqThreads) dequant_f16_kernel(const char* __restrict__ W, size_t w_rs, int M, int nblk,
                                                                 char* __restrict__ out, size_t out_rs,
                                                                 float* __restrict__ row_scale) {
    constexpr int kBlk = Q6 ? kQ6KBytes : kQ4KBytes;
    constexpr int kWarps = kDqThreads / 32;
    using Raw = typename std::conditional<Q6, Q6Raw, Q4Raw>::type;
    __shared__ float wmax[kWarps];
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // the previous kernel may still read the workspace
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    for (int m = blockIdx.x; m < M; m += gridDim.x) {
        const unsigned char* row = reinterpret_cast<const unsigned char*>(W + (size_t)m * w_rs);
        float bound = 0.0f;
        for (int kb = t; kb < nblk; kb += kDqThreads) bound = fmaxf(bound, block_bound<Q6>(row + (size_t)kb * kBlk));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bound = fmaxf(bound, __shfl_xor_sync(0xffffffffu, bound, o));
        if (lane == 0) wmax[warp] = bound;
        __syncthreads();
        bound = wmax[0];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) bound = fmaxf(bound, wmax[w]);
        __syncthreads();   // wmax is rewritten for the next row
        const int e = row_exponent(bound);
        const float sc_row = ldexpf(1.0f, -e);
        if (t == 0) row_scale[m] = ldexpf(1.0f, e);
        uint4* orow = reinterpret_cast<uint4*>(out + (size_t)m * out_rs);
        for (int kb0 = warp; kb0 < nblk; kb0 += kWarps * kDqU) {
            Raw r[kDqU];
#pragma unroll
            for (int u = 0; u < kDqU; ++u) {
                const int kb = kb0 + u * kWarps;
                if (kb < nblk) {
                    if constexpr (Q6)
                        r[u] = q6k_load(row + (size_t)kb * kBlk, lane);
                    else
                        r[u] = q4k_load(row + (size_t)kb * kBlk, lane);
                }
            }
#pragma unroll
            for (int u = 0; u < kDqU; ++u) {
                const int kb = kb0 + u * kWarps;
                if (kb < nblk) {
                    if constexpr (Q6)
                        orow[(size_t)kb * 32 + lane] = q6k_convert(r[u], lane, sc_row, e != 0);
                    else
                        orow[(size_t)kb * 32 + lane] = q4k_convert(r[u], lane, sc_row, e != 0);
                }
            }
        }
    }
}

constexpr size_t w16_bytes(int64_t M, int64_t K) { return ((size_t)M * (size_t)K * 2 + 255) / 256 * 256; }
constexpr size_t rs_bytes(int64_t M) { return ((size_t)M * 4 + 255) / 256 * 256; }

}  // namespace

bool quant_gemm_applicable(int w_type, int64_t M, int64_t K, int64_t N) {
    // below ~4 M weights the blocks stay in L2 across the decode kernels' passes (256 x 4096,
    // N = 128: 9.2 us there, 18.6 us through the f16 image)
    return (w_type == MLZC_TYPE_Q4_K || w_type == MLZC_TYPE_Q6_K) && N >= kQuantGemmMinN && K % kQK == 0 && M >= 1 &&
           M <= ((int64_t)1 << 30) && K <= ((int64_t)1 << 30) && M * K >= ((int64_t)1 << 22);
}

size_t quant_gemm_workspace_bytes(int64_t M, int64_t K, int64_t N) {
    return w16_bytes(M, K) + rs_bytes(M) + gemm_f16_workspace_bytes(M, K, N);
}

int launch_quant_gemm(const DeviceCtx* c, int w_type, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                      const float* x, size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws,
                      size_t ws_bytes, cudaStream_t s) {
    if (!quant_gemm_applicable(w_type, M, K, N)) return fail(MLZC_ERR_UNSUPPORTED, "quantised GEMM: shape not taken");
    const size_t need = quant_gemm_workspace_bytes(M, K, N);
    if (!ws || ws_bytes < need || (uintptr_t)ws % 16)
        return fail(MLZC_ERR_NOMEM, "quantised GEMM: workspace of %zu bytes (16-byte aligned) needed, %zu given", need,
                    ws_bytes);
    const int nblk = (int)(K / kQK);
    char* w16 = static_cast<char*>(ws);
    float* row_scale = reinterpret_cast<float*>(w16 + w16_bytes(M, K));
    const size_t rs16 = (size_t)K * 2;
    {
        // one CTA per row at a time
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(M, 148 * 16));
        const char* wc = static_cast<const char*>(w);
        if (w_type == MLZC_TYPE_Q4_K) {
            if ((uintptr_t)w % 16 || w_row_bytes % 16)
                return fail(MLZC_ERR_INVALID, "Q4_K: weights must be 16-byte aligned");
            MLZC_CUDA_TRY(launch_pdl(dequant_f16_kernel<false>, dim3(grid), dim3(kDqThreads), 0, s, wc, w_row_bytes,
                                     (int)M, nblk, w16, rs16, row_scale));
        } else {
            MLZC_CUDA_TRY(launch_pdl(dequant_f16_kernel<true>, dim3(grid), dim3(kDqThreads), 0, s, wc, w_row_bytes,
                                     (int)M, nblk, w16, rs16, row_scale));
        }
        count_launch();
    }
    const size_t off = w16_bytes(M, K) + rs_bytes(M);
    return launch_gemm_f16_row_scaled(c, w16, rs16, M, K, x, x_col_bytes, N, y, y_col_bytes,
                                      static_cast<char*>(ws) + off, ws_bytes - off, row_scale, s);
}

}  // namespace mlzc
