// fa_quant.cu -- flash-attention decode over a quantised KV cache (Q8_0 or Q4_0 K and V).
//
// Replaces the quantised-KV branches of flash_attn_dispatch (src/simd/flash_attention.cpp
// :112-248: simd_flash_attn_q8_0_avx512 / _q4_0_avx512, i.e. the FA2 skeleton
// flash_attn_fa2_skeleton_avx512.inc with the DEQUANT_K_DOT_BLOCK / DEQUANT_V_ACCUM_BLOCK
// macros of kernels/x86/flash/flash_attn_q8_0_avx512.asm and flash_attn_q4_0_avx512.asm).
// Element d of a row: Q8_0 (34-byte blocks of 32) = f16 d * int8 q; Q4_0 (18-byte blocks of
// 32) = f16 d * (nibble - 8), values 0-15 in the low nibbles, 16-31 in the high ones.  The
// score order is the F16 kernel's: s = <q * scale, k> + mask, softcap, + ALiBi.
//
// Design (split-K flash decoding on the CUDA cores; the rows are 136 / 72 bytes for
// D = 128, not 16-byte multiples, so no TMA map describes them):
//   - a CTA (128 threads) owns one segment -- one sequence, one KV head, up to 8 query rows
//     sharing it (GQA packing, as the F16 kernel) -- and one contiguous range of its
//     64-key tiles (grid.x = splits);
//   - per tile the CTA copies the 64 raw K and V rows into shared memory with 4-byte loads
//     (coalesced over each row), thread t scores key t % 64 for rows t / 64, +2, +4, +6
//     (int8 / nibble -> f32 per element, block scale once per 32), each warp updates the
//     online softmax of two rows, and thread t accumulates output dims t (+128) of every
//     row from the dequantised V;
//   - each CTA writes one partial record (m, l, O) per row; a combine kernel merges a
//     segment's records in split order (results repeat bit for bit).
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int kQThreads = 128;
constexpr int kQTile = 64;     // keys per tile
constexpr int kQRows = 8;      // query rows per segment

struct FaqParams {
    const char* q;
    const char* k;
    const char* v;
    const char* mask;
    char* dst;
    float* part;               // [nB][segments][splits][kQRows][D + 2]
    const int32_t* kv_len;
    int64_t q_nb1, q_nb2, q_nb3;
    int64_t k_nb1, k_nb2, k_nb3;
    int64_t v_nb1, v_nb2, v_nb3;
    int64_t m_nb0, m_nb1, m_nb2, m_nb3;
    int64_t d_nb1, d_nb2, d_nb3;
    int n_kv, n_q, n_head_q, n_head_kv;
    int G, rows_total, n_rgroups, n_hidx, HR, packed;
    int splits, tiles_per_split;
    int b_base, nB;
    float scale, softcap, alibi_p2inv;
    int use_softcap;
};

template <int TYPE>
struct KvFormat;
template <>
struct KvFormat<8> {   // Q8_0
    static constexpr int kBlockBytes = 34;
    __device__ __forceinline__ static float elem(const unsigned char* blk, int i) {
        return (float)(int)(signed char)blk[2 + i];
    }
};
template <>
struct KvFormat<2> {   // Q4_0
    static constexpr int kBlockBytes = 18;
    __device__ __forceinline__ static float elem(const unsigned char* blk, int i) {
        const unsigned b = blk[2 + (i & 15)];
        return (float)((int)(i < 16 ? (b & 15u) : (b >> 4)) - 8);
    }
};

__device__ __forceinline__ float blk_scale(const unsigned char* blk) {
    return __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
}

// Copies `rows` rows of `rb` bytes (row j at src + j * stride, 4-byte aligned) into shared
// memory at dst + j * rb; rows past `valid` are zero.
__device__ __forceinline__ void copy_rows(unsigned char* dst, const char* src, int64_t stride, int rb, int valid) {
    const int wpr = rb / 4;
    for (int i = threadIdx.x; i < kQTile * wpr; i += kQThreads) {
        const int j = i / wpr, w = i - j * wpr;
        uint32_t v = 0;
        if (j < valid) v = ptx::ld_act(reinterpret_cast<const int*>(src + (int64_t)j * stride) + w);
        reinterpret_cast<uint32_t*>(dst + j * rb)[w] = v;
    }
}

template <int D, int TYPE>
__global__ void __launch_bounds__(kQThreads)
fa_quant_kernel(const FaqParams p) {
    using F = KvFormat<TYPE>;
    constexpr int NB = D / 32;                  // blocks per row
    constexpr int RB = NB * F::kBlockBytes;     // bytes per row
    constexpr int DU = D / kQThreads;           // output dims per thread (1 or 2)
    static_assert(D % kQThreads == 0 || D == 64, "head dim");
    extern __shared__ __align__(16) unsigned char fq_smem[];
    float* q_s = reinterpret_cast<float*>(fq_smem);                   // [kQRows][D], * scale
    float* p_s = q_s + kQRows * D;                                    // [kQRows][kQTile]
    float* st_s = p_s + kQRows * kQTile;                              // [kQRows][3]: m, l, corr
    unsigned char* k_s = reinterpret_cast<unsigned char*>(st_s + kQRows * 4);
    unsigned char* v_s = k_s + kQTile * RB;

    ptx::pdl_launch_dependents();
    ptx::pdl_wait();
    const int t = threadIdx.x;
    const int split = blockIdx.x;
    const int seg = blockIdx.y;
    const int ib = p.b_base + blockIdx.z;
    const int hidx = seg / p.n_rgroups, rg = seg % p.n_rgroups;
    const int head_base = p.packed ? hidx * p.G : hidx;
    const int ihkv = p.packed ? hidx : hidx * p.n_head_kv / p.n_head_q;
    const int r0 = rg * kQRows;
    const int nrows = min(kQRows, p.rows_total - r0);
    const int L = p.kv_len ? min(p.kv_len[ib], p.n_kv) : p.n_kv;

    // query rows of the segment, scaled
    for (int i = t; i < kQRows * D; i += kQThreads) {
        const int r = i / D, d = i - r * D;
        float v = 0.0f;
        if (r < nrows) {
            const int rr = r0 + r, iq = rr / p.G, ihq = head_base + rr % p.G;
            v = ptx::ld_act(reinterpret_cast<const float*>(p.q + iq * p.q_nb1 + ihq * p.q_nb2 + ib * p.q_nb3) + d) * p.scale;
        }
        q_s[i] = v;
    }
    if (t < kQRows) {
        st_s[t * 4 + 0] = -INFINITY;
        st_s[t * 4 + 1] = 0.0f;
    }
    float O[kQRows][DU > 0 ? DU : 1];
#pragma unroll
    for (int r = 0; r < kQRows; ++r)
#pragma unroll
        for (int u = 0; u < (DU > 0 ? DU : 1); ++u) O[r][u] = 0.0f;

    const char* kbase = p.k + ihkv * p.k_nb2 + ib * p.k_nb3;
    const char* vbase = p.v + ihkv * p.v_nb2 + ib * p.v_nb3;
    const int tile0 = split * p.tiles_per_split;
    const int tile1 = min(tile0 + p.tiles_per_split, (L + kQTile - 1) / kQTile);
    const int warp = t >> 5, lane = t & 31;
    for (int tile = tile0; tile < tile1; ++tile) {
        const int j0 = tile * kQTile;
        const int valid = min(kQTile, L - j0);
        __syncthreads();   // the previous tile's K/V/P are no longer read
        copy_rows(k_s, kbase + (int64_t)j0 * p.k_nb1, p.k_nb1, RB, valid);
        copy_rows(v_s, vbase + (int64_t)j0 * p.v_nb1, p.v_nb1, RB, valid);
        __syncthreads();
        // scores: key jj = t % 64, rows t / 64 + 2 i
        {
            const int jj = t & (kQTile - 1);
            const int rbase = t / kQTile;               // 0 or 1
            float acc[kQRows / 2];
#pragma unroll
            for (int i = 0; i < kQRows / 2; ++i) acc[i] = 0.0f;
            const unsigned char* krow = k_s + jj * RB;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const unsigned char* blk = krow + b * F::kBlockBytes;
                float part[kQRows / 2];
#pragma unroll
                for (int i = 0; i < kQRows / 2; ++i) part[i] = 0.0f;
#pragma unroll 8
                for (int e = 0; e < 32; ++e) {
                    const float kv = F::elem(blk, e);
#pragma unroll
                    for (int i = 0; i < kQRows / 2; ++i) part[i] = fmaf(q_s[(rbase + 2 * i) * D + b * 32 + e], kv, part[i]);
                }
                const float ds = blk_scale(blk);
#pragma unroll
                for (int i = 0; i < kQRows / 2; ++i) acc[i] = fmaf(ds, part[i], acc[i]);
            }
            const int j = j0 + jj;
#pragma unroll
            for (int i = 0; i < kQRows / 2; ++i) {
                const int r = rbase + 2 * i;
                float a = acc[i];
                if (j < L && r < nrows) {
                    const int rr = r0 + r, iq = rr / p.G, ihq = head_base + rr % p.G;
                    if (p.mask)
                        a += ptx::ld_act(reinterpret_cast<const float*>(p.mask + iq * p.m_nb1 + (int64_t)j * p.m_nb0 +
                                                                        ihq * p.m_nb2 + ib * p.m_nb3));
                    if (p.use_softcap) a = p.softcap * tanhf(a / p.softcap);
                    if (p.alibi_p2inv != 0.0f) a += exp2f(p.alibi_p2inv * (float)(ihq + 1)) * (float)(j - iq);
                } else {
                    a = -INFINITY;
                }
                p_s[r * kQTile + jj] = a;
            }
        }
        __syncthreads();
        // online softmax: warp w updates rows w and w + 4
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = warp + 4 * h;
            const float a0 = p_s[r * kQTile + lane], a1 = p_s[r * kQTile + lane + 32];
            float mx = fmaxf(a0, a1);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_old = st_s[r * 4 + 0];
            const float m_new = fmaxf(m_old, mx);
            // a row with no visible key so far keeps m = -inf and p = 0
            const float corr = m_new == -INFINITY ? 1.0f : __expf(m_old - m_new);
            const float e0 = m_new == -INFINITY ? 0.0f : __expf(a0 - m_new);
            const float e1 = m_new == -INFINITY ? 0.0f : __expf(a1 - m_new);
            p_s[r * kQTile + lane] = e0;
            p_s[r * kQTile + lane + 32] = e1;
            float sum = e0 + e1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                st_s[r * 4 + 0] = m_new;
                st_s[r * 4 + 1] = st_s[r * 4 + 1] * corr + sum;
                st_s[r * 4 + 2] = corr;
            }
        }
        __syncthreads();
        // O[r][d] = O[r][d] * corr[r] + sum_j p[r][j] * v[j][d]
#pragma unroll
        for (int u = 0; u < (DU > 0 ? DU : 1); ++u) {
            const int d = t + u * kQThreads;
            if (D == 64 && d >= 64) break;
            const int b = d / 32, e = d % 32;
#pragma unroll
            for (int r = 0; r < kQRows; ++r) O[r][u] *= st_s[r * 4 + 2];
            for (int jj = 0; jj < valid; ++jj) {
                const unsigned char* blk = v_s + jj * RB + b * F::kBlockBytes;
                const float vv = blk_scale(blk) * F::elem(blk, e);
#pragma unroll
                for (int r = 0; r < kQRows; ++r) O[r][u] = fmaf(p_s[r * kQTile + jj], vv, O[r][u]);
            }
        }
    }
    __syncthreads();
    // partial record per row: m, l, O[D]
    float* rec = p.part + ((((size_t)blockIdx.z * p.HR + seg) * p.splits + split) * kQRows) * (D + 2);
#pragma unroll
    for (int u = 0; u < (DU > 0 ? DU : 1); ++u) {
        const int d = t + u * kQThreads;
        if (D == 64 && d >= 64) break;
#pragma unroll
        for (int r = 0; r < kQRows; ++r) rec[r * (D + 2) + 2 + d] = O[r][u];
    }
    if (t < kQRows) {
        rec[t * (D + 2) + 0] = st_s[t * 4 + 0];
        rec[t * (D + 2) + 1] = st_s[t * 4 + 1];
    }
}

// Merges a segment's split records row by row (split order), writes dst.
template <int D>
__global__ void fa_quant_combine_kernel(const FaqParams p) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();
    const int seg = blockIdx.y, ib = p.b_base + blockIdx.z;
    const int hidx = seg / p.n_rgroups, rg = seg % p.n_rgroups;
    const int head_base = p.packed ? hidx * p.G : hidx;
    const int r = blockIdx.x, rr = rg * kQRows + r;
    if (rr >= p.rows_total) return;
    const int iq = rr / p.G, ihq = head_base + rr % p.G;
    const float* rec0 = p.part + (((size_t)blockIdx.z * p.HR + seg) * p.splits * kQRows + r) * (D + 2);
    const size_t sstride = (size_t)kQRows * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, ptx::ld_act(rec0 + s * sstride));
    float* out = reinterpret_cast<float*>(p.dst + iq * p.d_nb1 + ihq * p.d_nb2 + ib * p.d_nb3);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float Ls = 0.0f, Os = 0.0f;
        if (M != -INFINITY) {
            for (int s = 0; s < p.splits; ++s) {
                const float* rec = rec0 + s * sstride;
                const float m = ptx::ld_act(rec);
                if (m == -INFINITY) continue;   // an empty split (all keys masked or past L)
                const float w = __expf(m - M);
                Ls += w * ptx::ld_act(rec + 1);
                Os += w * ptx::ld_act(rec + 2 + d);
            }
        }
        out[d] = Ls > 0.0f ? Os / Ls : 0.0f;
    }
}

struct FaqPlan {
    FaqParams p;
    size_t smem, ws_bytes;
    int slice;
};

int faq_plan(const mlzc_fa_desc* d, int sm_count, FaqPlan* out) {
    FaqPlan pl{};
    FaqParams& p = pl.p;
    const int Hq = (int)d->n_head_q, Hkv = (int)d->n_head_kv, D = (int)d->head_dim_k;
    p.packed = (Hq % Hkv == 0) ? 1 : 0;
    p.G = p.packed ? Hq / Hkv : 1;
    p.n_q = (int)d->n_queries;
    p.rows_total = p.G * p.n_q;
    p.n_rgroups = (p.rows_total + kQRows - 1) / kQRows;
    p.n_kv = (int)d->n_kv;
    p.n_head_q = Hq;
    p.n_head_kv = Hkv;
    p.n_hidx = p.packed ? Hkv : Hq;
    p.HR = p.n_hidx * p.n_rgroups;
    pl.slice = (int)std::min<int64_t>(d->batch_size, 65535);
    const int tiles = std::max(1, (p.n_kv + kQTile - 1) / kQTile);
    // about 4 CTAs per SM over the launch, at least 2 tiles per split where possible
    const int64_t segs = (int64_t)pl.slice * p.HR;
    int splits = (int)std::min<int64_t>(tiles, std::max<int64_t>(1, (4LL * sm_count + segs - 1) / segs));
    p.tiles_per_split = (tiles + splits - 1) / splits;
    p.splits = (tiles + p.tiles_per_split - 1) / p.tiles_per_split;
    const int RB = (int)fa_row_bytes(d->k_type, D);
    pl.smem = (size_t)(kQRows * D + kQRows * kQTile + kQRows * 4) * 4 + 2 * (size_t)kQTile * RB;
    pl.ws_bytes = (size_t)pl.slice * p.HR * p.splits * kQRows * (D + 2) * 4;
    *out = pl;
    return MLZC_OK;
}

template <int D, int TYPE>
int faq_launch(const FaqPlan& pl, cudaStream_t s) {
    static bool attr[64] = {};
    int dev = 0;
    MLZC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        MLZC_CUDA_TRY(cudaFuncSetAttribute(fa_quant_kernel<D, TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)pl.smem));
        attr[dev] = true;
    }
    const dim3 g((unsigned)pl.p.splits, (unsigned)pl.p.HR, (unsigned)pl.p.nB);
    MLZC_CUDA_TRY(launch_pdl(fa_quant_kernel<D, TYPE>, g, dim3(kQThreads), pl.smem, s, pl.p));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    const dim3 gc((unsigned)kQRows, (unsigned)pl.p.HR, (unsigned)pl.p.nB);
    MLZC_CUDA_TRY(launch_pdl(fa_quant_combine_kernel<D>, gc, dim3(std::min(D, 128)), 0, s, pl.p));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

template <int TYPE>
int faq_dispatch(const FaqPlan& pl, int D, cudaStream_t s) {
    if (D == 64) return faq_launch<64, TYPE>(pl, s);
    if (D == 128) return faq_launch<128, TYPE>(pl, s);
    return faq_launch<256, TYPE>(pl, s);
}

}  // namespace

int faq_workspace_bytes(const mlzc_fa_desc* d, int sm_count, size_t* out) {
    FaqPlan pl;
    const int st = faq_plan(d, sm_count, &pl);
    *out = st == MLZC_OK ? pl.ws_bytes : 0;
    return st;
}

int launch_flash_attn_quant(int sm_count, const mlzc_fa_desc* d, void* ws, size_t ws_bytes, cudaStream_t s) {
    FaqPlan pl;
    int st = faq_plan(d, sm_count, &pl);
    if (st != MLZC_OK) return st;
    if (pl.ws_bytes > ws_bytes || !ws)
        return fail(MLZC_ERR_NOMEM, "flash_attn: workspace of %zu bytes needed, %zu given", pl.ws_bytes, ws_bytes);
    if ((reinterpret_cast<uintptr_t>(ws) & 15) != 0) return fail(MLZC_ERR_INVALID, "flash_attn: workspace not 16-byte aligned");
    FaqParams& p = pl.p;
    p.q = reinterpret_cast<const char*>(d->q);
    p.k = static_cast<const char*>(d->k);
    p.v = static_cast<const char*>(d->v);
    p.mask = reinterpret_cast<const char*>(d->mask);
    p.dst = reinterpret_cast<char*>(d->dst);
    p.part = static_cast<float*>(ws);
    p.kv_len = d->kv_len;
    p.q_nb1 = d->q_nb[1]; p.q_nb2 = d->q_nb[2]; p.q_nb3 = d->q_nb[3];
    p.k_nb1 = d->k_nb[1]; p.k_nb2 = d->k_nb[2]; p.k_nb3 = d->k_nb[3];
    p.v_nb1 = d->v_nb[1]; p.v_nb2 = d->v_nb[2]; p.v_nb3 = d->v_nb[3];
    p.m_nb0 = d->mask_nb[0]; p.m_nb1 = d->mask_nb[1]; p.m_nb2 = d->mask_nb[2]; p.m_nb3 = d->mask_nb[3];
    p.d_nb1 = d->dst_nb[1]; p.d_nb2 = d->dst_nb[2]; p.d_nb3 = d->dst_nb[3];
    p.scale = d->scale;
    p.use_softcap = (d->mode & MLZC_FA_MODE_SOFTCAP) && d->logit_softcap != 0.0f;
    p.softcap = d->logit_softcap;
    if (d->mode & MLZC_FA_MODE_ALIBI) {
        int p2 = 1;
        while (p2 < p.n_head_q) p2 <<= 1;
        p.alibi_p2inv = -8.0f / (float)p2;
    } else {
        p.alibi_p2inv = 0.0f;
    }
    const int D = (int)d->head_dim_k;
    for (int64_t b0 = 0; b0 < d->batch_size; b0 += pl.slice) {
        p.b_base = (int)b0;
        p.nB = (int)std::min<int64_t>(pl.slice, d->batch_size - b0);
        st = d->k_type == MLZC_TYPE_Q8_0 ? faq_dispatch<8>(pl, D, s) : faq_dispatch<2>(pl, D, s);
        if (st != MLZC_OK) return st;
    }
    return MLZC_OK;
}

}  // namespace mlzc
