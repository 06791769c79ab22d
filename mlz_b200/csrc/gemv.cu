// gemv.cu -- decode-shaped mul_mat (few activation columns) on the CUDA cores.
//
// Replaces the per-row dot products of the reference: matrix_mult_avx512's k-loop
// (kernels/x86/matrix_mult_avx512.asm:165-181) reached through simd_matmul_f32
// (src/simd/simd_matmul.cpp:214-251), the upstream F16 vec_dot path the hook falls back
// to (src/simd/ggml-cpu-simd.c:1145-1244).
//
// Design (HBM-bound: every weight byte is read exactly once):
//   - one warp owns ROWS consecutive weight rows; its 32 lanes stride over K in 16-byte
//     chunks, so every load instruction of the warp reads 512 contiguous bytes per row;
//   - weights are streamed with L1::no_allocate loads (never re-read), activations with
//     weak L1-cached loads (they are re-read by every warp of a CTA and stay in L1/L2);
//   - fp32 accumulation per lane, butterfly shuffle reduction at the end;
//   - the ROWS rows of a warp share each activation load, which keeps the L1 traffic
//     per FMA at or below one byte.
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <type_traits>

#include "internal.h"
#include "peer.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ float2 h2_to_f2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
}

__device__ __forceinline__ float round_to_f16(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Unpacks 8 weights of one 16-byte chunk to f32 (F16 weights: 8 values per chunk).
struct WF16 {
    static constexpr int kPerChunk = 8;
    static constexpr bool kRoundX = true;
    static constexpr bool kNcWeights = true;   // f16 weights are never an output of these kernels
    __device__ __forceinline__ static void unpack(const uint4& v, float* w) {
        float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), c = h2_to_f2(v.z), d = h2_to_f2(v.w);
        w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y;
        w[4] = c.x; w[5] = c.y; w[6] = d.x; w[7] = d.y;
    }
    __device__ __forceinline__ static float scalar(const char* row, int64_t k) {
        return __half2float(reinterpret_cast<const __half*>(row)[k]);
    }
};

// F32 weights: 4 values per chunk, activations used as they are.
struct WF32 {
    static constexpr int kPerChunk = 4;
    static constexpr bool kRoundX = false;
    static constexpr bool kNcWeights = false;  // f32 weights may be an earlier call's output
    __device__ __forceinline__ static void unpack(const uint4& v, float* w) {
        w[0] = __uint_as_float(v.x); w[1] = __uint_as_float(v.y);
        w[2] = __uint_as_float(v.z); w[3] = __uint_as_float(v.w);
    }
    __device__ __forceinline__ static float scalar(const char* row, int64_t k) {
        return reinterpret_cast<const float*>(row)[k];
    }
};

// Vectorised kernel: requires 16-byte aligned rows/columns and K % kPerChunk == 0.
// Each lane keeps ROWS x U 16-byte weight loads in flight (U chunks 32 apart), which is
// what hides the HBM latency: ~128 KB in flight per SM at ROWS = 2, U = 4.
// early != 0 (f16 weights only): the first weight loads are issued before pdl_wait().
// KW = 1: each warp owns ROWS rows over all of K.  KW = 2, 4, 8: KW warps share a group of
// ROWS rows, warp w of the group takes every KW-th stretch of 32 * U chunks, and the CTA sums
// each group's KW partial rows in warp order -- more, shorter streams in flight per row.
// PEER (row-sharded mul_mat, one column): instead of Y, every output row goes to this
// rank's slice in the epoch's slot of every rank's exchange region (peer memory over
// NVLink); the wait kernel that follows on the stream signals and gathers.
template <class WT, int NB, int ROWS, int U, int KW, bool PEER>
__global__ void __launch_bounds__(kThreads)
gemv_vec_kernel(const char* __restrict__ W, size_t w_rs, int64_t M, int64_t K,
                const char* X, size_t x_cs, int ncols,
                char* __restrict__ Y, size_t y_cs, int early, PeerView pv) {
    constexpr int CH = WT::kPerChunk;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // KW warps share a group of ROWS rows (KW = 1: a warp per group), kWarps / KW groups per CTA
    const int grp = warp / KW;
    const int64_t row0 = ((int64_t)blockIdx.x * (kWarps / KW) + grp) * ROWS;
    const int kw = warp % KW;
    ptx::pdl_launch_dependents();
    if (KW == 1 && row0 >= M) return;   // (KW > 1: every warp takes the CTA barrier below)
    bool waited = false;
    if (!(WT::kNcWeights && early)) {
        ptx::pdl_wait();
        waited = true;
    }

    const char* wrow[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; r++) wrow[r] = W + (size_t)min(row0 + r, M - 1) * w_rs;

    float acc[ROWS][NB];
#pragma unroll
    for (int r = 0; r < ROWS; r++)
#pragma unroll
        for (int n = 0; n < NB; n++) acc[r][n] = 0.0f;

    const int64_t nchunk = K / CH;
    for (int64_t base = (int64_t)kw * 32 * U; base < nchunk; base += (int64_t)32 * U * KW) {
        uint4 wv[ROWS][U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t c = base + lane + 32 * u;
#pragma unroll
            for (int r = 0; r < ROWS; r++)
                wv[r][u] = c >= nchunk ? make_uint4(0, 0, 0, 0) : ptx::ld_weight16<WT::kNcWeights>(wrow[r] + (size_t)c * 16);
        }
        // the first weight loads are in flight while the previous kernel finishes; the
        // activations (and every write) come after it
        if (!waited) {
            ptx::pdl_wait();
            waited = true;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t c = base + lane + 32 * u;
            if (c >= nchunk) break;
            float wf[ROWS][CH];
#pragma unroll
            for (int r = 0; r < ROWS; r++) WT::unpack(wv[r][u], wf[r]);
#pragma unroll
            for (int n = 0; n < NB; n++) {
                if (n < ncols) {
                    const float4* xp = reinterpret_cast<const float4*>(X + (size_t)n * x_cs) + c * (CH / 4);
                    float xf[CH];
#pragma unroll
                    for (int q = 0; q < CH / 4; q++) {
                        const float4 t = ptx::ld_act(xp + q);
                        xf[4 * q + 0] = t.x; xf[4 * q + 1] = t.y; xf[4 * q + 2] = t.z; xf[4 * q + 3] = t.w;
                    }
                    if (WT::kRoundX) {
#pragma unroll
                        for (int i = 0; i < CH; i++) xf[i] = round_to_f16(xf[i]);
                    }
#pragma unroll
                    for (int r = 0; r < ROWS; r++)
#pragma unroll
                        for (int i = 0; i < CH; i++) acc[r][n] = fmaf(wf[r][i], xf[i], acc[r][n]);
                }
            }
        }
    }
    if (!waited) ptx::pdl_wait();
    uint32_t e = 0;
    if (PEER) e = peer_epoch(pv);   // after the wait: the previous call's wait kernel advanced it
    auto put = [&](int n, int64_t row, float v) {
        if (PEER) {
            // this rank's own rows straight into Y, the other ranks' slots over NVLink
            const size_t off = peer_slice_offset(pv, e) + (size_t)row * 4;   // [N = 1][m_loc]
            for (int r = 0; r < pv.G; ++r) {
                if (r == pv.rank) reinterpret_cast<float*>(Y)[row] = v;
                else *reinterpret_cast<float*>(pv.base[r] + off) = v;
            }
        } else {
            reinterpret_cast<float*>(Y + (size_t)n * y_cs)[row] = v;
        }
    };
    if (KW == 1) {
#pragma unroll
        for (int r = 0; r < ROWS; r++)
#pragma unroll
            for (int n = 0; n < NB; n++) {
                const float v = warp_sum(acc[r][n]);
                if (lane == 0 && n < ncols && row0 + r < M) put(n, row0 + r, v);
            }
    } else {
        __shared__ float red[kWarps][ROWS * NB];
#pragma unroll
        for (int r = 0; r < ROWS; r++)
#pragma unroll
            for (int n = 0; n < NB; n++) {
                const float v = warp_sum(acc[r][n]);
                if (lane == 0) red[warp][r * NB + n] = v;
            }
        __syncthreads();
        if (threadIdx.x < (kWarps / KW) * ROWS * NB) {
            const int gi = threadIdx.x / (ROWS * NB), e = threadIdx.x % (ROWS * NB);
            const int r = e / NB, n = e % NB;
            const int64_t rg = ((int64_t)blockIdx.x * (kWarps / KW) + gi) * ROWS;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < KW; ++w) v += red[gi * KW + w][e];
            if (n < ncols && rg + r < M) put(n, rg + r, v);
        }
    }
}

// Scalar kernel for any alignment / K: one warp per row, columns in sequence.
template <class WT>
__global__ void __launch_bounds__(kThreads)
gemv_scalar_kernel(const char* __restrict__ W, size_t w_rs, int64_t M, int64_t K,
                   const char* __restrict__ X, size_t x_cs, int64_t N,
                   char* __restrict__ Y, size_t y_cs) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (row >= M) return;
    const char* wr = W + (size_t)row * w_rs;
    for (int64_t n = 0; n < N; n++) {
        const float* xc = reinterpret_cast<const float*>(X + (size_t)n * x_cs);
        float acc = 0.0f;
        for (int64_t k = lane; k < K; k += 32) {
            float xv = xc[k];
            if (WT::kRoundX) xv = round_to_f16(xv);
            acc = fmaf(WT::scalar(wr, k), xv, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) reinterpret_cast<float*>(Y + (size_t)n * y_cs)[row] = acc;
    }
}

// KW warps of a CTA split the K of each row group whenever K is long enough for every warp
// to keep its loads in flight: measured on B200 (us per call, KW = 8 / one warp per 2 rows):
// 8192 x 28672 68.3 / 73.5, 28672 x 8192 65.0 / 74.6 (7.2 TB/s of weights).

// SM count of the current device (queried once per device).
int sm_count_cached() {
    static std::atomic<int> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 148;
    }
    int v = cached[dev].load(std::memory_order_relaxed);
    if (!v) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
            cudaGetLastError();
            v = 148;
        }
        cached[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

template <class WT, int NB, bool PEER = false>
int launch_vec(const char* w, size_t w_rs, int64_t M, int64_t K, const char* x, size_t x_cs,
               int ncols, char* y, size_t y_cs, cudaStream_t s, const PeerView& pv = PeerView{}) {
    constexpr int ROWS = 2;
    constexpr int U = NB <= 2 ? 4 : 2;
    const int early = weights_before_wait() ? 1 : 0;
    // the most warps per row group (KW) for which each still has a full set of loads in flight
    const int64_t chunks = K / WT::kPerChunk;
    const int kw = chunks >= (int64_t)32 * U * 8 ? 8 : chunks >= (int64_t)32 * U * 4 ? 4 : chunks >= (int64_t)32 * U * 2 ? 2 : 1;
    const int64_t rows_per_cta = (int64_t)(kWarps / kw) * ROWS;
    const unsigned grid = (unsigned)((M + rows_per_cta - 1) / rows_per_cta);
    auto go = [&](auto kern, unsigned g) {
        return launch_pdl(kern, dim3(g), dim3(kThreads), 0, s, w, w_rs, M, K, x, x_cs, ncols, y, y_cs, early, pv);
    };
    cudaError_t e;
    if constexpr (NB == 1 && std::is_same<WT, WF16>::value) {
        // Matrices of fewer than ~16 CTAs per SM at the shape above (C1's 8192 x 3072, the row
        // shards of the sharded FFN): 4 rows per group, 2 loads in flight, and the KW that
        // brings the grid nearest ~3.5 CTAs per SM.  Swept on B200 over ROWS {1, 2, 4} x
        // U {2, 3, 4, 6, 8} x KW {1, 2, 4, 8} (us per call, graph-replayed, weights rotated
        // past L2; this shape / the one above): 8192 x 3072 8.1 / 10.1, 3584 x 8192 9.9 /
        // 10.4, 2048 x 28672 18.1 / 20.7; at 7168 x 8192 and above the shape above wins.
        const int64_t sms = sm_count_cached();
        if ((int64_t)grid < 16 * sms) {
            int best_kw = 0;
            int64_t best_grid = 0;
            for (int k2 = 1; k2 <= 8; k2 *= 2) {
                if (chunks < (int64_t)64 * k2) break;   // every warp one full 2-chunk step
                const int64_t g2 = (M + (int64_t)(kWarps / k2) * 4 - 1) / ((int64_t)(kWarps / k2) * 4);
                if (!best_kw || std::llabs(2 * g2 - 7 * sms) < std::llabs(2 * best_grid - 7 * sms)) {
                    best_kw = k2;
                    best_grid = g2;
                }
            }
            if (best_kw && 2 * best_grid >= 5 * sms) {
                const unsigned g2 = (unsigned)best_grid;
                if (best_kw == 8) e = go(gemv_vec_kernel<WT, 1, 4, 2, 8, PEER>, g2);
                else if (best_kw == 4) e = go(gemv_vec_kernel<WT, 1, 4, 2, 4, PEER>, g2);
                else if (best_kw == 2) e = go(gemv_vec_kernel<WT, 1, 4, 2, 2, PEER>, g2);
                else e = go(gemv_vec_kernel<WT, 1, 4, 2, 1, PEER>, g2);
                MLZC_CUDA_TRY(e);
                count_launch();
                return MLZC_OK;
            }
        }
    }
    if (kw == 8) e = go(gemv_vec_kernel<WT, NB, ROWS, U, 8, PEER>, grid);
    else if (kw == 4) e = go(gemv_vec_kernel<WT, NB, ROWS, U, 4, PEER>, grid);
    else if (kw == 2) e = go(gemv_vec_kernel<WT, NB, ROWS, U, 2, PEER>, grid);
    else e = go(gemv_vec_kernel<WT, NB, ROWS, U, 1, PEER>, grid);
    MLZC_CUDA_TRY(e);
    count_launch();
    return MLZC_OK;
}

template <class WT>
int run_gemv(const void* w, size_t w_rs, int64_t M, int64_t K, const float* x, size_t x_cs,
             int64_t N, float* y, size_t y_cs, cudaStream_t s) {
    const char* wc = static_cast<const char*>(w);
    const char* xc = reinterpret_cast<const char*>(x);
    char* yc = reinterpret_cast<char*>(y);
    const bool aligned = ((uintptr_t)w % 16 == 0) && ((uintptr_t)x % 16 == 0) && (w_rs % 16 == 0) &&
                         (x_cs % 16 == 0) && (K % WT::kPerChunk == 0);
    if (!aligned) {
        const unsigned grid = (unsigned)((M + kWarps - 1) / kWarps);
        gemv_scalar_kernel<WT><<<grid, kThreads, 0, s>>>(wc, w_rs, M, K, xc, x_cs, N, yc, y_cs);
        count_launch();
        MLZC_CUDA_TRY(cudaGetLastError());
        return MLZC_OK;
    }
    for (int64_t n0 = 0; n0 < N; n0 += 8) {
        const int nc = (int)std::min<int64_t>(8, N - n0);
        const char* xn = xc + (size_t)n0 * x_cs;
        char* yn = yc + (size_t)n0 * y_cs;
        int st;
        if (nc == 1) st = launch_vec<WT, 1>(wc, w_rs, M, K, xn, x_cs, nc, yn, y_cs, s);
        else if (nc == 2) st = launch_vec<WT, 2>(wc, w_rs, M, K, xn, x_cs, nc, yn, y_cs, s);
        else if (nc <= 4) st = launch_vec<WT, 4>(wc, w_rs, M, K, xn, x_cs, nc, yn, y_cs, s);
        else st = launch_vec<WT, 8>(wc, w_rs, M, K, xn, x_cs, nc, yn, y_cs, s);
        if (st != MLZC_OK) return st;
    }
    return MLZC_OK;
}

// F16 decode GEMV whose outputs go straight to every rank's exchange slot (see PEER).
int gemv_f16_peer(const void* w, size_t w_rs, int64_t M, int64_t K, const float* x, const PeerView& pv,
                  float* y_own, cudaStream_t s) {
    const bool aligned = ((uintptr_t)w % 16 == 0) && ((uintptr_t)x % 16 == 0) && (w_rs % 16 == 0) &&
                         (K % WF16::kPerChunk == 0);
    if (!aligned || M < 1 || K < 1) return MLZC_ERR_UNSUPPORTED;   // caller takes the two-kernel path
    return launch_vec<WF16, 1, true>(static_cast<const char*>(w), w_rs, M, K, reinterpret_cast<const char*>(x),
                                     (size_t)K * 4, 1, reinterpret_cast<char*>(y_own), 0, s, pv);
}

// gathered [G][N][m_loc] -> dst [N][G * m_loc] (column stride dst_cs bytes): one CTA row per
// (rank slice r, column n) -- blockIdx.y = r * N + n -- threads over m, float4 when the
// slices and the destination are 16-byte aligned.
__global__ void gather_permute_kernel(const float* src, char* __restrict__ dst, size_t dst_cs, int N,
                                      int64_t m_loc, int vec) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // the gathered slices come from the all-gather
    const int64_t rn = blockIdx.y;
    const int64_t n = rn % N, r = rn / N;
    const float* srow = src + rn * m_loc;
    float* drow = reinterpret_cast<float*>(dst + (size_t)n * dst_cs) + r * m_loc;
    if (vec) {
        const int64_t m4 = m_loc / 4;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m4; i += (int64_t)gridDim.x * blockDim.x)
            reinterpret_cast<float4*>(drow)[i] = ptx::ld_act(reinterpret_cast<const float4*>(srow) + i);
    } else {
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m_loc; i += (int64_t)gridDim.x * blockDim.x)
            drow[i] = ptx::ld_act(srow + i);
    }
}

}  // namespace

int launch_gemv_f16_peer(const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                         const PeerView& pv, float* y_own, cudaStream_t s) {
    return gemv_f16_peer(w, w_row_bytes, M, K, x, pv, y_own, s);
}

int launch_gather_permute(const float* src, float* dst, size_t dst_col_bytes, int G, int64_t N,
                          int64_t m_loc, cudaStream_t s) {
    if ((int64_t)G * N == 0 || m_loc == 0) return MLZC_OK;
    if ((int64_t)G * N > 65535) return fail(MLZC_ERR_INVALID, "gather: %lld slices x columns", (long long)(G * N));
    const int vec = (m_loc % 4 == 0 && (uintptr_t)src % 16 == 0 && (uintptr_t)dst % 16 == 0 && dst_col_bytes % 16 == 0) ? 1 : 0;
    const int64_t per_row = vec ? m_loc / 4 : m_loc;
    const unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>((per_row + 255) / 256, 64));
    MLZC_CUDA_TRY(launch_pdl(gather_permute_kernel, dim3(gx, (unsigned)(G * N)), dim3(256), 0, s, src,
                             reinterpret_cast<char*>(dst), dst_col_bytes, (int)N, m_loc, vec));
    count_launch();
    MLZC_CUDA_TRY(cudaGetLastError());
    return MLZC_OK;
}

int launch_gemv(const DeviceCtx*, int w_type, const void* w, size_t w_row_bytes, int64_t M,
                int64_t K, const float* x, size_t x_col_bytes, int64_t N, float* y,
                size_t y_col_bytes, cudaStream_t s) {
    if (w_type == MLZC_TYPE_F16)
        return run_gemv<WF16>(w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes, s);
    if (w_type == MLZC_TYPE_F32)
        return run_gemv<WF32>(w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes, s);
    return fail(MLZC_ERR_UNSUPPORTED, "gemv: weight type %d", w_type);
}

}  // namespace mlzc
