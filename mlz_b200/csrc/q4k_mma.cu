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
#include "q4k.cuh"

namespace mlzc {
namespace {

using ptx::mma16816;
using q4k::RowScales;
using q4k::deq_hi;
using q4k::deq_lo;
using q4k::h2u;

constexpr int kQK = q4k::kQK;
constexpr int kQ4KBytes = q4k::kBlockBytes;
constexpr int kQWarps = 8;
constexpr int kQThreads = kQWarps * 32;
constexpr int kQRows = 32;     // rows per CTA: two 16-row MMA tiles

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

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

// Activation prep: X (N x K f32) rounded to f16 once, in the order the B fragments use,
// plus the sub-block sums as f16 hi + lo pairs.  One thread per (column, block, quad slot
// q, k-step s = 8 hi + wi): the values e = 64q + 32 hi + 4 wi + {0, 2} go to b0 and {1, 3}
// to b1; the 8 k-steps of a half (16 consecutive threads per (column, block, q): lanes 0-7
// hi = 0, 8-15 hi = 1) sum S_2q+hi by shuffles.  Columns past N are zero.
//   xf: [n-tile][block][k-step pair p][q][g] uint4 = (b0, b1) of steps 2p, 2p + 1
//       (g = column within the 8-column tile): the 32 lanes (g, q) of a warp read one
//       k-step pair of a block as 512 contiguous bytes, from global or shared memory
//   xs: [n-tile][block][q][g] uint2 (hi pair, lo pair)
__global__ void q4k_prep_kernel(const char* X, size_t x_cs, int N, int n_pad, int nblk,
                                uint2* __restrict__ xf, uint2* __restrict__ xs) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // X may come from, and the workspace be in use by, the previous kernel
    const int64_t total = (int64_t)n_pad * nblk * 64;     // a multiple of 32: whole warps
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int st = (int)(i & 15);
        const int q = (int)((i >> 4) & 3);
        const int64_t r = i >> 6;
        const int n = (int)(r % n_pad);
        const int kb = (int)(r / n_pad);
        const int nt = n >> 3, g = n & 7;
        const int hi = st >> 3, wi = st & 7;
        const int64_t slot = (((int64_t)nt * nblk + kb) * 4 + q) * 8 + g;
        const int64_t fslot = ((((int64_t)nt * nblk + kb) * 8 + (st >> 1)) * 4 + q) * 8 + g;
        const float4* src = reinterpret_cast<const float4*>(X + (size_t)(n < N ? n : 0) * x_cs) + (size_t)kb * (kQK / 4) + 16 * q;
        const float4 v = n < N ? ptx::ld_act(src + 8 * hi + wi) : make_float4(0.f, 0.f, 0.f, 0.f);
        const __half2 b0 = __floats2half2_rn(v.x, v.z), b1 = __floats2half2_rn(v.y, v.w);
        xf[fslot * 2 + (st & 1)] = make_uint2(h2u(b0), h2u(b1));
        const float2 f0 = __half22float2(b0), f1 = __half22float2(b1);
        float S = (f0.x + f0.y) + (f1.x + f1.y);
        S += __shfl_xor_sync(0xffffffffu, S, 1);
        S += __shfl_xor_sync(0xffffffffu, S, 2);
        S += __shfl_xor_sync(0xffffffffu, S, 4);
        const float S1 = __shfl_down_sync(0xffffffffu, S, 8);   // lane st = 0 gets the hi = 1 sum
        if (st == 0) {
            const __half2 sh = __floats2half2_rn(S, S1);
            const float2 shf = __half22float2(sh);
            xs[slot] = make_uint2(h2u(sh), h2u(__floats2half2_rn(S - shf.x, S1 - shf.y)));
        }
    }
}

// Main kernel (N > 8): a CTA = 8 warps over 32 rows (two 16-row MMA tiles) x 8 NT columns; warps
// take the K blocks in turn.  Per block a warp loads its rows' headers and nibble chunks
// (12 16-byte loads per thread) and the prepared activation fragments (one 16-byte load
// per k-step pair and column tile, pipelined one pair ahead), so per weight value the
// work is the LOP3 + HFMA2 dequant and a share of one MMA.  With one column tile the
// registers stay at <= 128, so two CTAs (16 warps) share an SM and hide the load latency.
template <int NT>
__global__ void __launch_bounds__(kQThreads, NT == 1 ? 2 : 1)
q4k_mma_kernel(const char* __restrict__ W, size_t w_rs, int M, int nblk, const uint2* xf,
               const uint2* xs, int N, char* __restrict__ Y, size_t y_cs, int early) {
    constexpr int COLS = 8 * NT;
    __shared__ float red[kQRows * COLS];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int q4 = lane & 3;
    const int m0 = blockIdx.y * kQRows;
    const int ntile0 = blockIdx.x * NT;

    // rows of this thread: tile t, half h -> m0 + 16 t + g + 8 h (clamped for loads)
    const char* rowp[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = min(m0 + 16 * (i >> 1) + g + 8 * (i & 1), M - 1);
        rowp[i] = W + (size_t)r * w_rs;
    }

    float y[NT][2][4] = {};
    ptx::pdl_launch_dependents();
    if (!early) ptx::pdl_wait();
    for (int kb = warp; kb < nblk; kb += kQWarps) {
        RowBlock cur[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) cur[i] = load_row_block(rowp[i] + (size_t)kb * kQ4KBytes, q4);
        // Q4_K blocks are never an output of these kernels; the prepared activations are
        if (kb == warp) ptx::pdl_wait();
        const uint4* xfrag[NT];
        uint2 sv[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int64_t slot = (((int64_t)(ntile0 + nt) * nblk + kb) * 4 + q4) * 8 + g;
            xfrag[nt] = reinterpret_cast<const uint4*>(xf) + ((((int64_t)(ntile0 + nt) * nblk + kb) * 8) * 4 + q4) * 8 + g;
            sv[nt] = ptx::ld_act(xs + slot);
        }
        uint4 xp[2][NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xp[0][nt] = ptx::ld_act(xfrag[nt]);
        RowScales sc[4];   // rows g, g + 8 of tile 0, then of tile 1
        q4k::row_scales2(cur[0].hdr, cur[1].hdr, q4, sc[0], sc[1]);
        q4k::row_scales2(cur[2].hdr, cur[3].hdr, q4, sc[2], sc[3]);

        float acc[NT][2][4] = {};
#pragma unroll
        for (int p = 0; p < 8; ++p) {          // k-step pairs 2p, 2p+1
            if (p < 7) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) xp[(p + 1) & 1][nt] = ptx::ld_act(xfrag[nt] + (p + 1) * 32);
            }
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                const int st = 2 * p + h2, hi = st >> 3, wi = st & 7;
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
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const uint4 x = xp[p & 1][nt];
                        mma16816(acc[nt][t], a0, a1, a2, a3, h2 ? x.z : x.x, h2 ? x.w : x.y);
                    }
                }
            }
        }
        // min term: sum_j m_j S_j (S as f16 hi + lo), then d and dmin
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                float mn[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(mn, sc[2 * t].mpair, sc[2 * t + 1].mpair, 0u, 0u, sv[nt].x, 0u);
                mma16816(mn, sc[2 * t].mpair, sc[2 * t + 1].mpair, 0u, 0u, sv[nt].y, 0u);
                y[nt][t][0] += sc[2 * t].d * acc[nt][t][0] - sc[2 * t].dmin * mn[0];
                y[nt][t][1] += sc[2 * t].d * acc[nt][t][1] - sc[2 * t].dmin * mn[1];
                y[nt][t][2] += sc[2 * t + 1].d * acc[nt][t][2] - sc[2 * t + 1].dmin * mn[2];
                y[nt][t][3] += sc[2 * t + 1].d * acc[nt][t][3] - sc[2 * t + 1].dmin * mn[3];
            }
    }

    ptx::pdl_wait();   // (again, for warps without a block)
    // fixed-order sum of the warps' partial rows through one shared buffer (warp 7 first)
    for (int w = kQWarps - 1; w >= 0; --w) {
        if (warp == w) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int t = 0; t < 2; ++t)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int r = 16 * t + g + 8 * (e >> 1);
                        const int cc = 8 * nt + 2 * q4 + (e & 1);
                        float* pp = &red[cc * kQRows + r];
                        *pp = (w == kQWarps - 1 ? 0.0f : *pp) + y[nt][t][e];
                    }
        }
        __syncthreads();
    }
    const int n0 = ntile0 * 8;
    for (int idx = threadIdx.x; idx < kQRows * COLS; idx += kQThreads) {
        const int r = idx % kQRows, cc = idx / kQRows;
        if (m0 + r < M && n0 + cc < N) reinterpret_cast<float*>(Y + (size_t)(n0 + cc) * y_cs)[m0 + r] = red[cc * kQRows + r];
    }
}

struct Q4kWs {
    int n_pad, nblk;
    size_t xf_bytes, xs_bytes;
};

Q4kWs q4k_ws(int64_t K, int64_t N) {
    Q4kWs w;
    // whole 8-column tiles; pairs of them for the batched kernel (N > 8)
    w.n_pad = N <= 8 ? 8 : (int)((N + 15) / 16 * 16);
    w.nblk = (int)(K / kQK);
    w.xf_bytes = ((size_t)w.n_pad * w.nblk * 4 * 16 * sizeof(uint2) + 255) / 256 * 256;
    w.xs_bytes = ((size_t)w.n_pad * w.nblk * 4 * sizeof(uint2) + 255) / 256 * 256;
    return w;
}

}  // namespace

size_t q4k_workspace_bytes(int64_t K, int64_t N) {
    if (q4k_i8_applicable(1, K, N)) return q4k_i8_workspace_bytes(K, N);
    // prepared activations: the shared-X ring (5 <= N <= 8) and the batched kernel (N > 8,
    // and any shape the int8 path does not take)
    const Q4kWs w = q4k_ws(K, N);
    return w.xf_bytes + w.xs_bytes;
}

int launch_q4k_mma(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                   size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
    if (K % kQK != 0) return fail(MLZC_ERR_INVALID, "Q4_K: K=%lld is not a multiple of 256", (long long)K);
    if ((uintptr_t)w % 16 || w_row_bytes % 16 || (uintptr_t)x % 16 || x_col_bytes % 16)
        return fail(MLZC_ERR_INVALID, "Q4_K: weights and activations must be 16-byte aligned");
    if (M > INT32_MAX / 2 || K / kQK > INT32_MAX / 64 || N > INT32_MAX / 64)
        return fail(MLZC_ERR_INVALID, "Q4_K: dimensions too large");
    const char* wc = static_cast<const char*>(w);
    const char* xc = reinterpret_cast<const char*>(x);
    char* yc = reinterpret_cast<char*>(y);
    // N <= 4: the int8 path; 5 <= N <= 8: the shared-X ring; N > 8: the batched kernel
    if (q4k_i8_applicable(M, K, N))
        return launch_q4k_i8(c, w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes, ws, ws_bytes, s);
    const bool xstream = q4k_ring_xs_applicable(M, K, N);
    const Q4kWs q = q4k_ws(K, N);
    if (!ws || ws_bytes < q.xf_bytes + q.xs_bytes || (uintptr_t)ws % 16)
        return fail(MLZC_ERR_NOMEM, "Q4_K: workspace of %zu bytes needed, %zu given", q.xf_bytes + q.xs_bytes, ws_bytes);
    uint2* xf = static_cast<uint2*>(ws);
    uint2* xs = reinterpret_cast<uint2*>(static_cast<char*>(ws) + q.xf_bytes);
    {
        const int64_t total = (int64_t)q.n_pad * q.nblk * 64;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 148 * 16));
        MLZC_CUDA_TRY(launch_pdl(q4k_prep_kernel, dim3(grid), dim3(256), 0, s, xc, x_col_bytes, (int)N, q.n_pad, q.nblk,
                                 xf, xs));
        count_launch();
    }
    if (xstream)
        return launch_q4k_ring_xs(c, w, w_row_bytes, M, K, reinterpret_cast<const uint4*>(xf), xs, N, y, y_col_bytes, s);
    const dim3 grid((unsigned)((N + 15) / 16), (unsigned)((M + kQRows - 1) / kQRows));
    if (grid.y > 65535u) return fail(MLZC_ERR_INVALID, "Q4_K: M=%lld beyond %d rows", (long long)M, 65535 * kQRows);
    MLZC_CUDA_TRY(launch_pdl(q4k_mma_kernel<2>, grid, dim3(kQThreads), 0, s, wc, w_row_bytes, (int)M, q.nblk, xf, xs,
                             (int)N, yc, y_col_bytes, weights_before_wait() ? 1 : 0));
    count_launch();
    return MLZC_OK;
}

}  // namespace mlzc
