// q6k.cu -- Q6_K-weight mul_mat on the tensor cores (mma.sync m16n8k16, f16 x f16 -> f32).
//
// Replaces the Q6_K branch of ggml_simd_try_mul_mat (src/simd/ggml_simd_hook.cpp:282-288,
// the K-quant path of :234-301): one simd_vec_dot_q6_k_q8_k
// (src/simd/kernels/x86/vec/vec_dot_q6_k_q8_k_avx2.asm) per (row, column) over Q8_K
// activations.  As for Q4_K, the activations keep f32 precision up to one f16 rounding;
// the parity bar is the dequantised-F32 product.
//
// Q6_K block (GGUF, 210 bytes per 256 weights; block size src/bench_simd.zig:34-40):
// ql[128] @0, qh[64] @128, int8 scales[16] @192 (one per 16 weights), f16 d @208.
// Element p (h = p / 128, r = p % 128, k = r / 32, l = r % 32): 6-bit u = nibble k/2 of
// ql[64h + 32(k%2) + l] | (bits 2k, 2k+1 of qh[32h + l]) << 4, w = d * scales[p/16] * (u-32).
//
// Tensor-core form: one MMA k-step per 16-weight scale group s (so the group's integer
// scale multiplies the k-step's fp32 result, exactly), d once per block.  In group s a
// quad thread q holds the 4 weights i = 4q .. 4q+3 of each of its rows, which are the four
// bytes of one 32-bit word of ql (and of qh): bytes 0, 2 form one f16 pair and bytes 1, 3
// the other, each built with masks and shifts as 0x6400 | u (= 1024 + u, exact) and
// re-centred by one HSUB2 (- 1056).  The activations of the same positions (x0, x2),
// (x1, x3) are the B fragments.
//
// A 210-byte block is only 2-byte aligned when its index is odd: a 4-byte field there is
// read as the two aligned words around it, joined with a funnel shift.  W must be 4-byte
// aligned (so the first block of row 0 is), and no word read lies outside a block except
// the 2 bytes before an odd block, which belong to the block before it.
//
// CTA = 8 warps over 32 rows (two MMA tiles) x 8 * NT columns; warps take the blocks in
// turn and the CTA sums the warps' partial rows in a fixed order (results repeat bit for
// bit).
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

using ptx::mma16816;

constexpr int kQK = 256;
constexpr int kQ6KBytes = 210;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 32;

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ uint32_t ld_w32(const char* p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// 32-bit field at p (p 2-byte aligned; `mis` = p % 4, 0 or 2)
__device__ __forceinline__ uint32_t ld_field(const char* p, int mis) {
    if (mis == 0) return ld_w32(p);
    const uint32_t lo = ld_w32(p - 2), hi = ld_w32(p + 2);
    return __funnelshift_r(lo, hi, 16);
}

// One row's share of a block for a quad thread q4: ql words of the 8 16-byte chunks (word
// q4 of each), qh words of the 4 chunks, the 16 scale bytes and d.
struct Q6Row {
    uint32_t ql[8], qh[4], sc[4];
    float d;
};

__device__ __forceinline__ void load_row(const char* blk, int q4, Q6Row& r) {
    const int mis = (int)(reinterpret_cast<uintptr_t>(blk) & 3);
#pragma unroll
    for (int c = 0; c < 8; ++c) r.ql[c] = ld_field(blk + 16 * c + 4 * q4, mis);
#pragma unroll
    for (int c = 0; c < 4; ++c) r.qh[c] = ld_field(blk + 128 + 16 * c + 4 * q4, mis);
#pragma unroll
    for (int c = 0; c < 4; ++c) r.sc[c] = ld_field(blk + 192 + 4 * c, mis);
    unsigned short dh;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(dh) : "l"(blk + 208));
    r.d = __half2float(__ushort_as_half(dh));
}

// The two f16 pairs of group s of a row: (i = 4q, 4q+2) and (4q+1, 4q+3), as q = u - 32.
template <int S>
__device__ __forceinline__ void deq_group(const Q6Row& r, uint32_t& pa, uint32_t& pb) {
    constexpr int h = S >> 3, k = (S >> 1) & 3, b = S & 1;
    constexpr int c = 4 * h + 2 * (k & 1) + b, ch = 2 * h + b, nib = k >> 1;
    const uint32_t ql = nib ? (r.ql[c] >> 4) : r.ql[c];
    // qh bits 2k, 2k+1 of each byte -> bits 4, 5 of the byte
    const uint32_t qh = (2 * k <= 4) ? (r.qh[ch] << (4 - 2 * k)) : (r.qh[ch] >> (2 * k - 4));
    const uint32_t fa = (ql & 0x000F000Fu) | (qh & 0x00300030u) | 0x64006400u;
    const uint32_t fb = ((ql >> 8) & 0x000F000Fu) | ((qh >> 8) & 0x00300030u) | 0x64006400u;
    const __half2 bias = __halves2half2(__ushort_as_half(0x6420), __ushort_as_half(0x6420));   // 1056
    pa = h2u(__hsub2(u2h(fa), bias));
    pb = h2u(__hsub2(u2h(fb), bias));
}

__device__ __forceinline__ float sc_of(const Q6Row& r, int s) {
    return (float)(int)(int8_t)(r.sc[s >> 2] >> (8 * (s & 3)));
}

template <int S, int NT>
__device__ __forceinline__ void group_step(const Q6Row (&rw)[4], const uint32_t (&bx)[NT][2], float (&acc)[NT][2][4]) {
    uint32_t pa[4], pb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) deq_group<S>(rw[i], pa[i], pb[i]);
    float sc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[i] = sc_of(rw[i], S);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            float tmp[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(tmp, pa[2 * t], pa[2 * t + 1], pb[2 * t], pb[2 * t + 1], bx[nt][0], bx[nt][1]);
            acc[nt][t][0] += sc[2 * t] * tmp[0];
            acc[nt][t][1] += sc[2 * t] * tmp[1];
            acc[nt][t][2] += sc[2 * t + 1] * tmp[2];
            acc[nt][t][3] += sc[2 * t + 1] * tmp[3];
        }
    }
}

template <int S, int NT>
__device__ __forceinline__ void group_run(const Q6Row (&rw)[4], const float* const (&xc)[NT], const bool (&cok)[NT],
                                          float (&acc)[NT][2][4]) {
    uint32_t bx[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float4 v = cok[nt] ? ptx::ld_act(reinterpret_cast<const float4*>(xc[nt] + 16 * S)) : make_float4(0.f, 0.f, 0.f, 0.f);
        bx[nt][0] = h2u(__floats2half2_rn(v.x, v.z));
        bx[nt][1] = h2u(__floats2half2_rn(v.y, v.w));
    }
    group_step<S, NT>(rw, bx, acc);
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
q6k_mma_kernel(const char* __restrict__ W, size_t w_rs, int M, int nblk, const char* X, size_t x_cs, int N,
               char* __restrict__ Y, size_t y_cs, int early) {
    constexpr int COLS = 8 * NT;
    __shared__ float red[kWarps][kRows * COLS];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int q4 = lane & 3;
    const int m0 = blockIdx.y * kRows;
    const int n0 = blockIdx.x * COLS;

    // rows of this thread: tile t, half e -> m0 + 16 t + g + 8 e (clamped for loads)
    const char* rowp[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = min(m0 + 16 * (i >> 1) + g + 8 * (i & 1), M - 1);
        rowp[i] = W + (size_t)r * w_rs;
    }
    const float* xcol[NT];
    bool cok[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        cok[nt] = n0 + 8 * nt + g < N;
        xcol[nt] = reinterpret_cast<const float*>(X + (size_t)(cok[nt] ? n0 + 8 * nt + g : 0) * x_cs) + 4 * q4;
    }

    float y[NT][2][4] = {};
    ptx::pdl_launch_dependents();
    // Q6_K blocks are never an output of this library's kernels: with early != 0 the first
    // block's loads overlap the previous kernel's tail; activations and writes come after it
    if (!early) ptx::pdl_wait();
    Q6Row rw[4], nx[4];
    int kb = warp;
    if (kb < nblk) {
#pragma unroll
        for (int i = 0; i < 4; ++i) load_row(rowp[i] + (size_t)kb * kQ6KBytes, q4, rw[i]);
    }
    ptx::pdl_wait();
    for (; kb < nblk; kb += kWarps) {
        // the next block's fields are in flight while this one is computed
        const int kn = kb + kWarps;
        if (kn < nblk) {
#pragma unroll
            for (int i = 0; i < 4; ++i) load_row(rowp[i] + (size_t)kn * kQ6KBytes, q4, nx[i]);
        }
        float acc[NT][2][4] = {};
        const float* xc[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xc[nt] = xcol[nt] + (size_t)kb * kQK;
        group_run<0, NT>(rw, xc, cok, acc);
        group_run<1, NT>(rw, xc, cok, acc);
        group_run<2, NT>(rw, xc, cok, acc);
        group_run<3, NT>(rw, xc, cok, acc);
        group_run<4, NT>(rw, xc, cok, acc);
        group_run<5, NT>(rw, xc, cok, acc);
        group_run<6, NT>(rw, xc, cok, acc);
        group_run<7, NT>(rw, xc, cok, acc);
        group_run<8, NT>(rw, xc, cok, acc);
        group_run<9, NT>(rw, xc, cok, acc);
        group_run<10, NT>(rw, xc, cok, acc);
        group_run<11, NT>(rw, xc, cok, acc);
        group_run<12, NT>(rw, xc, cok, acc);
        group_run<13, NT>(rw, xc, cok, acc);
        group_run<14, NT>(rw, xc, cok, acc);
        group_run<15, NT>(rw, xc, cok, acc);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                y[nt][t][0] += rw[2 * t].d * acc[nt][t][0];
                y[nt][t][1] += rw[2 * t].d * acc[nt][t][1];
                y[nt][t][2] += rw[2 * t + 1].d * acc[nt][t][2];
                y[nt][t][3] += rw[2 * t + 1].d * acc[nt][t][3];
            }
        if (kn < nblk) {
#pragma unroll
            for (int i = 0; i < 4; ++i) rw[i] = nx[i];
        }
    }

    // partial rows of every warp -> fixed-order sum
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int r = 16 * t + g;
            red[warp][r * COLS + 8 * nt + 2 * q4] = y[nt][t][0];
            red[warp][r * COLS + 8 * nt + 2 * q4 + 1] = y[nt][t][1];
            red[warp][(r + 8) * COLS + 8 * nt + 2 * q4] = y[nt][t][2];
            red[warp][(r + 8) * COLS + 8 * nt + 2 * q4 + 1] = y[nt][t][3];
        }
    __syncthreads();
    for (int e = threadIdx.x; e < kRows * COLS; e += kThreads) {
        const int r = e % kRows, cidx = e / kRows;
        if (m0 + r < M && n0 + cidx < N) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += red[w][r * COLS + cidx];
            reinterpret_cast<float*>(Y + (size_t)(n0 + cidx) * y_cs)[m0 + r] = v;
        }
    }
}

}  // namespace

int launch_q6k(const DeviceCtx*, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
               size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, cudaStream_t s) {
    const int nblk = (int)(K / kQK);
    const int NT = N > 8 ? 2 : 1;
    const int cols = 8 * NT;
    const dim3 grid((unsigned)((N + cols - 1) / cols), (unsigned)((M + kRows - 1) / kRows));
    if (grid.y > 65535u) return fail(MLZC_ERR_INVALID, "mul_mat (Q6_K): M too large");
    const int early = weights_before_wait() ? 1 : 0;
    const char* W = static_cast<const char*>(w);
    const char* X = reinterpret_cast<const char*>(x);
    char* Y = reinterpret_cast<char*>(y);
    if (NT == 2)
        MLZC_CUDA_TRY(launch_pdl(q6k_mma_kernel<2>, grid, dim3(kThreads), 0, s, W, w_row_bytes, (int)M, nblk, X,
                                 x_col_bytes, (int)N, Y, y_col_bytes, early));
    else
        MLZC_CUDA_TRY(launch_pdl(q6k_mma_kernel<1>, grid, dim3(kThreads), 0, s, W, w_row_bytes, (int)M, nblk, X,
                                 x_col_bytes, (int)N, Y, y_col_bytes, early));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

}  // namespace mlzc
