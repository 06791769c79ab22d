// gemv_mma.cu -- skinny F16-weight mul_mat (2..16 activation columns) on the tensor cores.
//
// Replaces, for F16 weights and few activation columns, the upstream F16 path the hook falls
// back to (src/simd/ggml-cpu-simd.c:1314-1465: src1 rounded to f16, then ggml_vec_dot_f16 per
// (row, column) with fp32 accumulation).  That arithmetic -- f16 x f16 products summed in
// fp32 -- is what mma.sync.m16n8k16.f32.f16.f16.f32 computes.
//
// HBM-bound: every weight byte is read once, in 16-byte loads, straight into the A operand
// with no ALU work.  Inside each 32-value chunk of K the k order is permuted so that quad
// thread q (lane % 4) owns values 8q .. 8q+7 of a row -- one 16-byte load -- which are its A
// fragments of two consecutive k-steps (pairs (0,1), (2,3) for the first, (4,5), (6,7) for
// the second).  The activations of the same values (two float4 per column) are rounded to
// f16 pairs for the B fragments.  A CTA = 8 warps over 16 MT rows x 8 NT columns; each warp
// takes a contiguous eighth of K (long sequential runs per row), keeps U chunks of loads in
// flight ahead of its MMAs, and the CTA sums the warps' partial tiles in a fixed order
// (results repeat bit for bit).
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

using ptx::mma16816;

constexpr int kSkWarps = 8;
constexpr int kSkThreads = kSkWarps * 32;
constexpr int kChunkK = 32;    // k values per chunk: two MMA k-steps

__device__ __forceinline__ uint4 ld_w16(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int MT, int NT, int U>
__global__ void __launch_bounds__(kSkThreads)
gemv_f16_mma_kernel(const char* __restrict__ W, size_t w_rs, int M, int K, const char* X, size_t x_cs,
                    int N, char* __restrict__ Y, size_t y_cs, int early) {
    constexpr int ROWS = 16 * MT, COLS = 8 * NT;
    __shared__ float red[ROWS * COLS];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int q4 = lane & 3;
    const int m0 = blockIdx.x * ROWS;
    const int n0 = blockIdx.y * COLS;

    // this thread's rows (tile t, half h -> m0 + 16 t + 8 h + g) and columns (tile nt -> n0 + 8 nt + g),
    // clamped for loads; the clamped rows and columns are never stored
    const char* wrow[MT][2];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) wrow[t][h] = W + (size_t)min(m0 + 16 * t + 8 * h + g, M - 1) * w_rs + 16 * q4;
    const char* xcol[NT];
    bool xok[NT];   // this lane's B column is a real one
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        // with one column tile the lanes past N load nothing (N = 2: 6 of 8 lanes; measured
        // 11.7 -> 10.6 us on 8192 x 3072); with two tiles (N > 8) the predicate measured slower
        xok[nt] = NT > 1 || n0 + 8 * nt + g < N;
        xcol[nt] = X + (size_t)min(n0 + 8 * nt + g, N - 1) * x_cs + 32 * q4;
    }

    ptx::pdl_launch_dependents();
    if (!early) ptx::pdl_wait();
    const int nch = (K + kChunkK - 1) / kChunkK;
    const int c_begin = (int)((int64_t)nch * warp / kSkWarps);
    const int c_end = (int)((int64_t)nch * (warp + 1) / kSkWarps);

    float acc[MT][NT][4] = {};
    for (int c0 = c_begin; c0 < c_end; c0 += U) {
        uint4 wv[U][MT][2];
        float4 xv[U][NT][2];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c0 + u;
            // K % 8 == 0, so this thread's 8-value group is wholly inside K or wholly past it
            const bool ok = c < c_end && c * kChunkK + 8 * q4 < K;
#pragma unroll
            for (int t = 0; t < MT; ++t)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    wv[u][t][h] = ok ? ld_w16(wrow[t][h] + (size_t)c * (kChunkK * 2)) : make_uint4(0, 0, 0, 0);
        }
        // (f16 weights are never an output of these kernels: with early != 0 their first loads
        // overlap the previous kernel's tail; the activations never do)
        if (c0 == c_begin) ptx::pdl_wait();
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c0 + u;
            const bool ok = c < c_end && c * kChunkK + 8 * q4 < K;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float4* xp = reinterpret_cast<const float4*>(xcol[nt] + (size_t)c * (kChunkK * 4));
                xv[u][nt][0] = ok && xok[nt] ? ptx::ld_act(xp) : make_float4(0.f, 0.f, 0.f, 0.f);
                xv[u][nt][1] = ok && xok[nt] ? ptx::ld_act(xp + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                uint32_t b0[NT], b1[NT];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const float4 v = xv[u][nt][s];
                    b0[nt] = pack_h2(v.x, v.y);
                    b1[nt] = pack_h2(v.z, v.w);
                }
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    const uint32_t a0 = s ? wv[u][t][0].z : wv[u][t][0].x;
                    const uint32_t a2 = s ? wv[u][t][0].w : wv[u][t][0].y;
                    const uint32_t a1 = s ? wv[u][t][1].z : wv[u][t][1].x;
                    const uint32_t a3 = s ? wv[u][t][1].w : wv[u][t][1].y;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) mma16816(acc[t][nt], a0, a1, a2, a3, b0[nt], b1[nt]);
                }
            }
        }
    }

    ptx::pdl_wait();   // (again, for warps whose K range was empty)
    // fixed-order sum of the warps' tiles through one shared buffer (warp 7 first)
    for (int w = kSkWarps - 1; w >= 0; --w) {
        if (warp == w) {
#pragma unroll
            for (int t = 0; t < MT; ++t)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int r = 16 * t + g + 8 * (e >> 1);
                        const int cc = 8 * nt + 2 * q4 + (e & 1);
                        float* p = &red[cc * ROWS + r];
                        *p = (w == kSkWarps - 1 ? 0.0f : *p) + acc[t][nt][e];
                    }
        }
        __syncthreads();
    }
    for (int idx = threadIdx.x; idx < ROWS * COLS; idx += kSkThreads) {
        const int r = idx % ROWS, cc = idx / ROWS;
        if (m0 + r < M && n0 + cc < N) reinterpret_cast<float*>(Y + (size_t)(n0 + cc) * y_cs)[m0 + r] = red[cc * ROWS + r];
    }
}

template <int MT, int NT, int U>
int launch_sk(const char* w, size_t w_rs, int64_t M, int64_t K, const char* x, size_t x_cs, int64_t N, char* y,
              size_t y_cs, cudaStream_t s) {
    const dim3 grid((unsigned)((M + 16 * MT - 1) / (16 * MT)), (unsigned)((N + 8 * NT - 1) / (8 * NT)));
    MLZC_CUDA_TRY(launch_pdl(gemv_f16_mma_kernel<MT, NT, U>, grid, dim3(kSkThreads), 0, s, w, w_rs, (int)M, (int)K, x,
                             x_cs, (int)N, y, y_cs, weights_before_wait() ? 1 : 0));
    count_launch();
    return MLZC_OK;
}

}  // namespace

bool gemv_f16_mma_applicable(int64_t M, int64_t K, int64_t N, const void* w, size_t w_row_bytes, const float* x,
                             size_t x_col_bytes) {
    return N >= 2 && N <= 16 && K % 8 == 0 && M <= (1ll << 30) && K <= (1ll << 30) && (uintptr_t)w % 16 == 0 &&
           w_row_bytes % 16 == 0 && (uintptr_t)x % 16 == 0 && x_col_bytes % 16 == 0;
}

int launch_gemv_f16_mma(const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x, size_t x_col_bytes,
                        int64_t N, float* y, size_t y_col_bytes, cudaStream_t s) {
    const char* wc = static_cast<const char*>(w);
    const char* xc = reinterpret_cast<const char*>(x);
    char* yc = reinterpret_cast<char*>(y);
    // measured on B200 (8192 x 3072, us for U = 2 / 3 / 4 chunks in flight per warp): N = 2
    // 10.6 / 9.7 / 10.5, N = 4 10.9 / 10.0 / 10.2, N = 8 11.4 / 10.8 / 10.4; 16-row CTAs beat
    // 32-row ones up to 8 columns; beyond 16 columns the tcgen05 GEMM is faster.  A later
    // sweep of MT {1, 2, 4} x U {2, 3, 4, 6} (graph-replayed, weights rotated past L2) kept
    // those and found U = 4 better for N <= 4 on matrices from ~40 M weights (14336 x 4096,
    // N = 4: 22.6 vs 24.3 us) and MT = 2, U = 4 for 9..16 columns (N = 16: 12.8 vs 13.3 us
    // on 8192 x 3072, 28.7 vs 31.9 on 14336 x 4096).
    if (N <= 4) {
        if (M * K >= (int64_t)40 << 20) return launch_sk<1, 1, 4>(wc, w_row_bytes, M, K, xc, x_col_bytes, N, yc, y_col_bytes, s);
        return launch_sk<1, 1, 3>(wc, w_row_bytes, M, K, xc, x_col_bytes, N, yc, y_col_bytes, s);
    }
    if (N <= 8) return launch_sk<1, 1, 4>(wc, w_row_bytes, M, K, xc, x_col_bytes, N, yc, y_col_bytes, s);
    return launch_sk<2, 2, 4>(wc, w_row_bytes, M, K, xc, x_col_bytes, N, yc, y_col_bytes, s);
}

}  // namespace mlzc
