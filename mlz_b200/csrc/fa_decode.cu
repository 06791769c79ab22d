// fa_decode.cu -- flash-attention decode over an F16 KV cache.
//
// Replaces the F16 branch of flash_attn_dispatch (src/simd/flash_attention.cpp:143-150):
// simd_flash_attn_f16_avx512 = the FA2 skeleton (kernels/x86/flash/
// flash_attn_fa2_skeleton_avx512.inc:394-842) with the F16 macros of
// flash_attn_f16_avx512.asm:46-82.  The reference gives every (query, head, batch) work
// item to one CPU thread and walks its keys in tiles of 64 with an online softmax.
//
// GPU design (HBM-bound: every K/V byte is read once):
//   - Grouped-query packing: the G = n_head_q / n_head_kv query heads (times n_queries)
//     that share a KV head are the columns of one MMA tile (up to 8 query rows), so each
//     K/V row is read once for all of them.  A "segment" is one (sequence, kv head, row
//     group) and its keys are cut into 64-key tiles.
//   - Persistent, stream-K balanced: a grid of (SMs x resident CTAs) walks the tiles of
//     all segments in one global order, each CTA taking an equal contiguous range, so a
//     ragged batch costs only its real keys and no CTA idles while another finishes.  A
//     CTA's range covers whole segments or parts of them ("pieces"); at the end of a piece
//     every consumer warp writes a partial (max, sum, unnormalised O) record of its rows,
//     and the combine kernel merges a row's records in CTA then warp order, so results
//     repeat bit for bit.
//   - A producer warp streams K and V tiles into a shared-memory ring with TMA (4-d tensor
//     maps over the ggml strides, 64-dim boxes with 128-byte swizzle), across piece
//     boundaries without a pause.
//   - Four consumer warps own 16 keys of every tile.  Scores S^T = K . Q^T and the update
//     O^T += V^T . P^T run on the tensor cores (mma.sync m16n8k16, f16 operands, f32
//     accumulators in registers): keys fill the MMA's M side (16) and the query rows its
//     N side (8), and the S^T accumulators become the P^T operand through an in-register
//     8x8 transpose (movmatrix).  With 3-8 query rows per KV head the tcgen05 MMA's
//     minimum M of 64 would be mostly padding and every online-softmax rescale would go
//     through TMEM; here the accumulators stay in registers and the tensor pipe stays far
//     below its bound (D/4 MMAs per 16 keys).
//     fp32-level accuracy: Q and P are split into f16 hi + lo parts (two MMAs each), K
//     and V are f16 already.  Online softmax (max / rescale / exp) in fp32 per warp.
//   - Every mbarrier wait is bounded (MLZC_DEVERR_WAIT_TIMEOUT).
// Score order (flash_attention.cpp:339-363): s = <q*scale, k>, + mask, softcap, + ALiBi.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int kFaWarps = 4;                          // consumer warps
constexpr int kFaThreads = (kFaWarps + 1) * 32;      // + one producer warp
constexpr int kTile = 64;                            // keys per shared-memory stage
constexpr int kWarpKeys = kTile / kFaWarps;          // 16 keys per consumer warp and tile
constexpr int kRows = 8;                             // query rows per segment (the MMA's N)
constexpr int kBox = 64;                             // dims per TMA box (128 bytes, swizzled)
constexpr int kMaxBatch = 1024;                      // sequences per launch (prefix table in smem)

template <int D>
struct FaCfg {
    static constexpr int kBoxes = D / kBox;
    static constexpr uint32_t kOperandBytes = kBoxes * kTile * 128;   // K or V of one tile
    static constexpr uint32_t kStageBytes = 2 * kOperandBytes;
    static constexpr int kStages = D == 64 ? 4 : 3;
    static constexpr uint32_t kPrefBytes = ((kMaxBatch + 1) * 4 + 15) / 16 * 16;
    static constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + kPrefBytes + 128;
};

struct __align__(64) FaParams {
    const char* q;
    const char* mask;
    char* dst;
    float* part;                 // partial records: (CTAs + segments) x warps x kRows x (D + 2)
    int* pref_out;               // the prefix table, for the combine kernel
    const int32_t* kv_len;       // per sequence, or nullptr (every sequence has n_kv keys)
    int64_t q_nb1, q_nb2, q_nb3;
    int64_t m_nb0, m_nb1, m_nb2, m_nb3;
    int64_t d_nb1, d_nb2, d_nb3;
    int n_kv, n_q, n_head_q, n_head_kv;
    int G;                       // query heads per row group
    int rows_total;              // G * n_q
    int n_rgroups;               // ceil(rows_total / kRows)
    int n_hidx;                  // kv heads (packed) or query heads
    int HR;                      // segments per sequence: n_hidx * n_rgroups
    int b_base, nB;              // sequences [b_base, b_base + nB) in this launch
    int packed;                  // 1: a segment's heads share one kv head; 0: one query head
    float scale, softcap, alibi_p2inv;  // alibi_p2inv = -8 / P (0 = no ALiBi)
    int use_softcap;
    int k_hmul, k_bmul, v_hmul, v_bmul;   // 0 where K / V is shared across heads / sequences
    unsigned int* err;           // device error word (bounded waits)
    CUtensorMap tm_k, tm_v;      // [B][Hkv][n_kv][D] with 64 x 64 swizzled boxes
};

// Row r of a row group -> (query position, query head).
__device__ __forceinline__ void row_coords(const FaParams& p, int head_base, int r, int& iq, int& ihq) {
    iq = r / p.G;
    ihq = head_base + r % p.G;
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z,
                                            int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

using ptx::mma16816;
using ptx::movtrans;
using ptx::split_h2;


// Address of the 16-byte chunk `chunk` (of 8 dims) of key row `key` in a tile operand
// stored as kBoxes boxes of [64 keys][128 bytes] with the TMA 128-byte swizzle.
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int key, int chunk) {
    return base + (uint32_t)((chunk >> 3) * (kTile * 128) + key * 128 + (((chunk & 7) ^ (key & 7)) << 4));
}


__device__ __forceinline__ int seq_len(const FaParams& p, int b) {
    return p.kv_len ? min(max(ptx::ld_act(p.kv_len + p.b_base + b), 0), p.n_kv) : p.n_kv;
}

// CTA of global tile t when W tiles are cut into P equal contiguous ranges
// [c W / P, (c + 1) W / P).
__device__ __forceinline__ int cta_of_tile(int64_t t, int64_t W, int P) {
    return (int)(((t + 1) * P - 1) / W);
}

// Position in the global tile order: sequence b, segment sl of the sequence, tile j of
// the segment (nb tiles).  Segments of a sequence come in (head index, row group) order.
struct Walk {
    int b, sl, j, nb;
    __device__ __forceinline__ void init(const int* pref, int nB, int HR, int64_t t) {
        int lo = 0, hi = nB - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if ((int64_t)HR * pref[mid] <= t) lo = mid; else hi = mid - 1;
        }
        b = lo;
        nb = pref[b + 1] - pref[b];
        const int64_t u = t - (int64_t)HR * pref[b];
        sl = (int)(u / nb);
        j = (int)(u % nb);
    }
    __device__ __forceinline__ void next(const int* pref, int nB, int HR) {
        if (++j < nb) return;
        j = 0;
        if (++sl < HR) return;
        sl = 0;
        do { ++b; } while (b < nB && pref[b + 1] == pref[b]);
        if (b < nB) nb = pref[b + 1] - pref[b];
    }
};

// Score and value steps per tile and warp, in the transposed form that puts keys on the
// MMA's M side (16) and the query rows on N (8):
//   S^T [16 keys x 8 rows]  = K [16 keys x D] . Q^T [D x 8 rows]      (D/16 k-steps)
//   O^T [D x 8 rows]       += V^T [D x 16 keys] . P^T [16 keys x 8 rows]
// Fragment ownership (g = lane/4, q = lane%4): S^T element (key g or g+8, row 2q or 2q+1),
// O^T element (dim 16t + g or +8, row 2q or 2q+1): every lane keeps two query rows.
// GEN = false is plain decode (no mask, softcap or ALiBi): the score path carries no
// branches for them.
template <int D, bool GEN>
__global__ void __launch_bounds__(kFaThreads)
fa_decode_kernel(const __grid_constant__ FaParams p) {
    using C = FaCfg<D>;
    constexpr int STAGES = C::kStages;
    constexpr int KS = D / 16;                   // 16-dim steps (QK) and 16-dim output tiles (PV)
    extern __shared__ uint8_t fa_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    int* pref = reinterpret_cast<int*>(smem + STAGES * C::kStageBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::kStageBytes + C::kPrefBytes);
    uint64_t* empty = full + STAGES;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + STAGES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int q4 = lane & 3;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
            ptx::mbar_init(ptx::smem_u32(&empty[s]), kFaWarps);
        }
        *abort_flag = 0;
        ptx::mbar_init_fence();
    }
    // the set-up above overlaps the previous kernel's tail; kv_len, Q, K, V and the outputs
    // wait for it
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();
    // prefix table: pref[b] = tiles of one segment summed over sequences < b
    if (warp == 0) {
        int run = 0;
        for (int base = 0; base < p.nB; base += 32) {
            const int b = base + lane;
            const int nb = b < p.nB ? (seq_len(p, b) + kTile - 1) / kTile : 0;
            int x = nb;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (b < p.nB) pref[b + 1] = run + x;
            run += __shfl_sync(0xffffffffu, x, 31);
        }
        if (lane == 0) pref[0] = 0;
    }
    __syncthreads();
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i <= p.nB; i += kFaThreads) p.pref_out[i] = pref[i];

    const int64_t W = (int64_t)p.HR * pref[p.nB];
    const int P = gridDim.x;
    const int64_t t_begin = W * blockIdx.x / P;
    const int64_t t_end = W * (blockIdx.x + 1) / P;
    const int count = (int)(t_end - t_begin);
    if (count <= 0) return;

    if (warp == kFaWarps) {
        // ---------------- producer: K and V tiles into the ring with TMA
        if (lane == 0) {
            Walk w;
            w.init(pref, p.nB, p.HR, t_begin);
            for (int i = 0; i < count; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (i / STAGES) & 1;
                if (!ptx::mbar_wait(ptx::smem_u32(&empty[s]), ph ^ 1, abort_flag, p.err)) break;
                // the consumers read this stage with ldmatrix (generic proxy); order those
                // reads, which the empty barrier has made visible here, before the TMA
                // (async proxy) overwrites the stage
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                const int hidx = w.sl / p.n_rgroups;
                const int kvh = p.packed ? hidx : (int)((int64_t)hidx * p.n_head_kv / p.n_head_q);
                const uint32_t fb = ptx::smem_u32(&full[s]);
                const uint32_t st = ptx::smem_u32(ring + s * C::kStageBytes);
                const int j0 = w.j * kTile;
                ptx::mbar_expect_tx(fb, C::kStageBytes);
#pragma unroll
                for (int bx = 0; bx < C::kBoxes; ++bx) {
                    tma_load_4d(st + bx * (kTile * 128), &p.tm_k, fb, bx * kBox, j0, kvh * p.k_hmul,
                                (p.b_base + w.b) * p.k_bmul);
                    tma_load_4d(st + C::kOperandBytes + bx * (kTile * 128), &p.tm_v, fb, bx * kBox, j0,
                                kvh * p.v_hmul, (p.b_base + w.b) * p.v_bmul);
                }
                w.next(pref, p.nB, p.HR);
            }
        }
        return;
    }

    // ---------------- consumers: 16 keys of every tile per warp
    const int mat = lane >> 3;                   // ldmatrix: matrix whose row this lane addresses
    const int kw = warp * kWarpKeys;
    const int k_key = kw + (lane & 7) + 8 * (mat & 1);     // K: matrices (keys, dims) = (0,0) (8,0) (0,8) (8,8)
    const int k_half = mat >> 1;
    const int v_key = kw + (lane & 7) + 8 * (mat >> 1);    // V^T: matrices (dims, keys) = (0,0) (8,0) (0,8) (8,8)
    const int v_half = mat & 1;

    Walk w;
    w.init(pref, p.nB, p.HR, t_begin);
    // per-piece state
    int L = 0, ib = 0, head_base = 0, rg = 0, nrows = 0;
    int iq_r[2] = {0, 0}, ihq_r[2] = {0, 0};
    bool row_ok[2] = {false, false};
    float slope[2] = {0.0f, 0.0f};
    uint32_t qf[KS][4];
    float m_row[2], l_row[2];
    float o[KS][4];

    for (int i = 0; i < count; ++i) {
        if (i == 0 || w.j == 0) {
            // ---- a new piece: segment (w.b, w.sl)
            ib = p.b_base + w.b;
            L = seq_len(p, w.b);
            const int hidx = w.sl / p.n_rgroups;
            rg = w.sl % p.n_rgroups;
            head_base = p.packed ? hidx * p.G : hidx;
            nrows = min(kRows, p.rows_total - rg * kRows);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = 2 * q4 + h;
                row_ok[h] = r < nrows;
                row_coords(p, head_base, rg * kRows + (row_ok[h] ? r : 0), iq_r[h], ihq_r[h]);
                slope[h] = p.alibi_p2inv != 0.0f ? exp2f(p.alibi_p2inv * (float)(ihq_r[h] + 1)) : 0.0f;
                m_row[h] = -INFINITY;
                l_row[h] = 0.0f;
            }
            // B fragments of Q^T (pre-scaled, f16 hi + lo): row g, dims 16 ks + {2 q4, +1, +8, +9}
            const float* qr = nullptr;
            if (g < nrows) {
                int iq, ihq;
                row_coords(p, head_base, rg * kRows + g, iq, ihq);
                qr = reinterpret_cast<const float*>(p.q + iq * p.q_nb1 + ihq * p.q_nb2 + ib * p.q_nb3);
            }
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int d0 = 16 * ks + 2 * q4;
                float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
                if (qr) {
                    x0 = ptx::ld_act(qr + d0) * p.scale;
                    x1 = ptx::ld_act(qr + d0 + 1) * p.scale;
                    x2 = ptx::ld_act(qr + d0 + 8) * p.scale;
                    x3 = ptx::ld_act(qr + d0 + 9) * p.scale;
                }
                split_h2(x0, x1, qf[ks][0], qf[ks][2]);
                split_h2(x2, x3, qf[ks][1], qf[ks][3]);
            }
#pragma unroll
            for (int t = 0; t < KS; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
        }

        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!ptx::mbar_wait(ptx::smem_u32(&full[s]), ph, abort_flag, p.err)) return;   // all consumers stop here
        const uint32_t kbuf = ptx::smem_u32(ring + s * C::kStageBytes);
        const uint32_t vbuf = kbuf + C::kOperandBytes;
        const int j0 = w.j * kTile;
        if (j0 + kw + kWarpKeys > L) {
            // V rows past the sequence's last key may hold any bits (NaN included) and
            // 0 * NaN in P . V would poison O: zero this warp's rows of them
            const int first = max(0, L - j0 - kw);
            uint8_t* vgen = ring + s * C::kStageBytes + C::kOperandBytes;
            for (int idx = lane; idx < (kWarpKeys - first) * (D / 8); idx += 32) {
                const int key = kw + first + idx / (D / 8);
                const int c = idx % (D / 8);
                *reinterpret_cast<uint4*>(vgen + (tile_addr(vbuf, key, c) - vbuf)) = make_uint4(0, 0, 0, 0);
            }
            // these generic writes precede the next TMA write into the stage
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        }

        // S^T = K . Q^T in four independent accumulator chains (Q hi / lo x even / odd
        // 16-dim steps), summed at the end
        float acc[4][4] = {};
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(tile_addr(kbuf, k_key, 2 * ks + k_half), a0, a1, a2, a3);
            mma16816(acc[2 * (ks & 1)], a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
            mma16816(acc[2 * (ks & 1) + 1], a0, a1, a2, a3, qf[ks][2], qf[ks][3]);
        }
        // mask / softcap / ALiBi / validity; element e: key g + 8 (e >> 1), row 2 q4 + (e & 1)
        float sc[4];
        float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int h = e & 1;
            const int j = j0 + kw + g + 8 * (e >> 1);
            float a = (acc[0][e] + acc[2][e]) + (acc[1][e] + acc[3][e]);
            if (j < L && row_ok[h]) {
                if constexpr (GEN) {
                    if (p.mask)
                        a += ptx::ld_act(reinterpret_cast<const float*>(p.mask + iq_r[h] * p.m_nb1 + (int64_t)j * p.m_nb0 +
                                                            ihq_r[h] * p.m_nb2 + ib * p.m_nb3));
                    if (p.use_softcap) a = p.softcap * tanhf(a / p.softcap);
                    if (p.alibi_p2inv != 0.0f) a += slope[h] * (float)(j - iq_r[h]);
                }
            } else {
                a = -INFINITY;
            }
            sc[e] = a;
            tmax[h] = fmaxf(tmax[h], a);
        }
        float corr[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 4));
            tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 8));
            tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 16));
            const float mnew = fmaxf(m_row[h], tmax[h]);
            corr[h] = (mnew == -INFINITY) ? 1.0f : __expf(m_row[h] - mnew);
            m_row[h] = mnew;
            l_row[h] *= corr[h];
        }
        if (corr[0] != 1.0f || corr[1] != 1.0f) {
#pragma unroll
            for (int t2 = 0; t2 < KS; ++t2) {
                o[t2][0] *= corr[0]; o[t2][1] *= corr[1];
                o[t2][2] *= corr[0]; o[t2][3] *= corr[1];
            }
        }
        float pe[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int h = e & 1;
            pe[e] = (sc[e] == -INFINITY) ? 0.0f : __expf(sc[e] - m_row[h]);
            l_row[h] += pe[e];
        }
        // P^T (keys x rows) as f16 hi + lo, transposed in registers into B fragments
        uint32_t h0, l0, h1, l1;
        split_h2(pe[0], pe[1], h0, l0);      // key g
        split_h2(pe[2], pe[3], h1, l1);      // key g + 8
        const uint32_t bh0 = movtrans(h0), bh1 = movtrans(h1);
        const uint32_t bl0 = movtrans(l0), bl1 = movtrans(l1);
        // O^T += V^T . P^T
#pragma unroll
        for (int dt = 0; dt < KS; ++dt) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(tile_addr(vbuf, v_key, 2 * dt + v_half), a0, a1, a2, a3);
            mma16816(o[dt], a0, a1, a2, a3, bh0, bh1);
            mma16816(o[dt], a0, a1, a2, a3, bl0, bl1);
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&empty[s]));

        const bool seg_end = (w.j == w.nb - 1);
        if (seg_end || i == count - 1) {
            // ---- end of the piece: this warp's (max, sum, unnormalised O) of its rows
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                l_row[h] += __shfl_xor_sync(0xffffffffu, l_row[h], 4);
                l_row[h] += __shfl_xor_sync(0xffffffffu, l_row[h], 8);
                l_row[h] += __shfl_xor_sync(0xffffffffu, l_row[h], 16);
            }
            float* rec = p.part + (((int64_t)blockIdx.x + (int64_t)w.b * p.HR + w.sl) * kFaWarps + warp) * kRows * (D + 2);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (!row_ok[h]) continue;
                float* rr = rec + (2 * q4 + h) * (D + 2);
                if (g == 0) { rr[0] = m_row[h]; rr[1] = l_row[h]; }
#pragma unroll
                for (int dt = 0; dt < KS; ++dt) {
                    rr[2 + 16 * dt + g] = o[dt][h];
                    rr[2 + 16 * dt + g + 8] = o[dt][2 + h];
                }
            }
        }
        w.next(pref, p.nB, p.HR);
    }
}

// Writes every output row: merges the per-warp records of the CTAs that held pieces of its
// segment, in CTA then warp order (zeros for an empty sequence).  One CTA of D threads per
// row, latency-lean: record headers are read in parallel (one per thread), the maximum and
// the weighted sum come from block reductions, then each thread sums its dimension over
// the records with independent loads.
template <int D>
__global__ void __launch_bounds__(D)
fa_combine_kernel(const __grid_constant__ FaParams p, int P) {
    constexpr int NW = D / 32;
    __shared__ float s_e[D];          // record weights of the current chunk
    __shared__ float s_red[NW];
    __shared__ float s_bcast;
    const int row = blockIdx.x;
    const int hidx = blockIdx.y;
    const int b = blockIdx.z;
    const int t = threadIdx.x;
    const int lane = t & 31, wid = t >> 5;
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // the partial records come from the decode kernel
    const int* pref = p.pref_out;
    const int nb = ptx::ld_act(pref + b + 1) - ptx::ld_act(pref + b);
    const int rg = row / kRows, r = row % kRows;
    const int sl = hidx * p.n_rgroups + rg;
    const int ib = p.b_base + b;
    const int head_base = p.packed ? hidx * p.G : hidx;
    int iq, ihq;
    row_coords(p, head_base, row, iq, ihq);
    float* dr = reinterpret_cast<float*>(p.dst + iq * p.d_nb1 + ihq * p.d_nb2 + ib * p.d_nb3);
    if (nb == 0) {
        dr[t] = 0.0f;
        return;
    }
    const int64_t W = (int64_t)p.HR * ptx::ld_act(pref + p.nB);
    const int64_t T = (int64_t)p.HR * ptx::ld_act(pref + b) + (int64_t)sl * nb;
    const int cf = cta_of_tile(T, W, P);
    const int nrec = (cta_of_tile(T + nb - 1, W, P) - cf + 1) * kFaWarps;
    const float* base = p.part + (((int64_t)cf + (int64_t)b * p.HR + sl) * kFaWarps * kRows + r) * (D + 2);
    // record q = (CTA cf + q / kFaWarps, warp q % kFaWarps) sits at base + q * kRows * (D + 2);
    // CTAs with an empty range (more CTAs than tiles) wrote none
    auto rec_m = [&](int q) {
        const int64_t c = cf + q / kFaWarps;
        return (W * c / P == W * (c + 1) / P) ? -INFINITY : ptx::ld_act(base + (int64_t)q * kRows * (D + 2));
    };
    auto block_reduce = [&](float v, bool is_max) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float u = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, u) : v + u;
        }
        if (lane == 0) s_red[wid] = v;
        __syncthreads();
        if (t == 0) {
            float a = s_red[0];
            for (int w = 1; w < NW; ++w) a = is_max ? fmaxf(a, s_red[w]) : a + s_red[w];
            s_bcast = a;
        }
        __syncthreads();
        const float res = s_bcast;
        __syncthreads();
        return res;
    };
    float mloc = -INFINITY;
    for (int q = t; q < nrec; q += D) mloc = fmaxf(mloc, rec_m(q));
    const float M = block_reduce(mloc, true);
    if (M == -INFINITY) {
        dr[t] = 0.0f;
        return;
    }
    float Ls = 0.0f, Os = 0.0f;
    for (int q0 = 0; q0 < nrec; q0 += D) {
        const int q = q0 + t;
        float e = 0.0f, lw = 0.0f;
        if (q < nrec) {
            const float m = rec_m(q);
            if (m != -INFINITY) {
                e = __expf(m - M);
                lw = e * ptx::ld_act(base + (int64_t)q * kRows * (D + 2) + 1);
            }
        }
        s_e[t] = e;
        Ls += block_reduce(lw, false);   // also orders the s_e writes before the reads below
        const int n = min(D, nrec - q0);
        int k = 0;
        // a record of weight 0 is not read: an empty-range CTA's slot holds stale bits
        for (; k + 4 <= n; k += 4) {
            const float* o0 = base + (int64_t)(q0 + k) * kRows * (D + 2) + 2 + t;
            const float e0 = s_e[k], e1 = s_e[k + 1], e2 = s_e[k + 2], e3 = s_e[k + 3];
            const float v0 = e0 != 0.0f ? ptx::ld_act(o0) : 0.0f;
            const float v1 = e1 != 0.0f ? ptx::ld_act(o0 + kRows * (D + 2)) : 0.0f;
            const float v2 = e2 != 0.0f ? ptx::ld_act(o0 + 2 * kRows * (D + 2)) : 0.0f;
            const float v3 = e3 != 0.0f ? ptx::ld_act(o0 + 3 * kRows * (D + 2)) : 0.0f;
            Os += e0 * v0;
            Os += e1 * v1;
            Os += e2 * v2;
            Os += e3 * v3;
        }
        for (; k < n; ++k)
            if (s_e[k] != 0.0f) Os += s_e[k] * ptx::ld_act(base + (int64_t)(q0 + k) * kRows * (D + 2) + 2 + t);
        __syncthreads();   // s_e is rewritten by the next chunk
    }
    dr[t] = Ls > 0.0f ? Os / Ls : 0.0f;
}

// Resident CTAs of the decode kernel per SM on the current device (sets the kernel's
// shared-memory attributes on first use).
// The per-device cache is atomic: two host threads may make their first call at the same
// time (on one device or on different ones); both then set the same attributes and store
// the same value.
template <int D>
int fa_ctas_per_sm(int* out) {
    static std::atomic<int> cached[64];
    int dev = 0;
    MLZC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(MLZC_ERR_INVALID, "flash_attn: device %d beyond 64", dev);
    if (!cached[dev].load(std::memory_order_acquire)) {
        constexpr size_t smem = FaCfg<D>::kSmemBytes;
        for (auto* k : {fa_decode_kernel<D, false>, fa_decode_kernel<D, true>}) {
            MLZC_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            MLZC_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                               (int)cudaSharedmemCarveoutMaxShared));
        }
        int occ = 0, occ_gen = 0;
        MLZC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fa_decode_kernel<D, false>, kFaThreads, smem));
        MLZC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_gen, fa_decode_kernel<D, true>, kFaThreads, smem));
        occ = std::min(occ, occ_gen);
        int sms = 0;
        MLZC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        if (occ < 1) return fail(MLZC_ERR_CUDA, "flash_attn: decode kernel does not fit on an SM");
        cached[dev].store(occ * sms, std::memory_order_release);
    }
    *out = cached[dev].load(std::memory_order_acquire);
    return MLZC_OK;
}

struct FaPlan {
    FaParams p;
    int ctas;          // decode grid (persistent)
    int slice;         // sequences per launch
    size_t pref_bytes;
    size_t ws_bytes;
};

int make_plan(const mlzc_fa_desc* d, FaPlan* out) {
    FaPlan pl{};
    FaParams& p = pl.p;
    const int Hq = (int)d->n_head_q, Hkv = (int)d->n_head_kv;
    const int D = (int)d->head_dim_k;
    p.packed = (Hq % Hkv == 0) ? 1 : 0;
    p.G = p.packed ? Hq / Hkv : 1;
    p.n_q = (int)d->n_queries;
    p.rows_total = p.G * p.n_q;
    p.n_rgroups = (p.rows_total + kRows - 1) / kRows;
    p.n_kv = (int)d->n_kv;
    p.n_head_q = Hq;
    p.n_head_kv = Hkv;
    p.n_hidx = p.packed ? Hkv : Hq;
    p.HR = p.n_hidx * p.n_rgroups;
    pl.slice = (int)std::min<int64_t>(d->batch_size, kMaxBatch);
    int resident = 0;
    int st = MLZC_OK;
    if (D == 64) st = fa_ctas_per_sm<64>(&resident);
    else if (D == 128) st = fa_ctas_per_sm<128>(&resident);
    else if (D == 256) st = fa_ctas_per_sm<256>(&resident);
    else return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: head_dim %d (64, 128, 256 supported)", D);
    if (st != MLZC_OK) return st;
    const int64_t tiles_max = (int64_t)pl.slice * p.HR * ((p.n_kv + kTile - 1) / kTile);
    pl.ctas = (int)std::max<int64_t>(1, std::min<int64_t>(resident, tiles_max));
    pl.pref_bytes = ((size_t)(pl.slice + 1) * sizeof(int) + 255) / 256 * 256;
    pl.ws_bytes = pl.pref_bytes + ((size_t)pl.ctas + (size_t)pl.slice * p.HR) * kFaWarps * kRows *
                                      (size_t)(d->head_dim_v + 2) * sizeof(float);
    *out = pl;
    return MLZC_OK;
}

// 4-d f16 map of a K or V tensor (ggml dims [D, n_kv, Hkv, B], byte strides nb[1..3]) with
// 64 x 64 boxes in the 128-byte swizzle (the layout tile_addr() reads).  A dimension with
// stride 0 (one K/V shared by every head or sequence) gets extent 1 in the map and its
// coordinate multiplier (*hmul, *bmul) is 0; a tensor map cannot hold a 0 stride.
int encode_kv_map(CUtensorMap* map, const void* base, int64_t D, int64_t n_kv, int64_t hkv, int64_t B, const size_t* nb,
                  int* hmul, int* bmul) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(MLZC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if (nb[1] == 0) return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: K/V with a 0 key stride");
    const bool hb = (hkv == 1 || nb[2] == 0), bb = (B == 1 || nb[3] == 0);
    *hmul = hb ? 0 : 1;
    *bmul = bb ? 0 : 1;
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)n_kv, hb ? 1u : (cuuint64_t)hkv, bb ? 1u : (cuuint64_t)B};
    // strides of extent-1 dimensions are never stepped; keep them legal
    const cuuint64_t st1 = nb[1];
    const cuuint64_t st2 = hb ? st1 * (cuuint64_t)n_kv : nb[2];
    const cuuint64_t st3 = bb ? st2 * dims[2] : nb[3];
    const cuuint64_t strides[3] = {st1, st2, st3};
    const cuuint32_t box[4] = {(cuuint32_t)kBox, (cuuint32_t)kTile, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: K/V strides not expressible as a TMA map (%d)", (int)r);
    return MLZC_OK;
}

}  // namespace

namespace {
int current_sms() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        sms = 148;
    }
    return sms;
}
}  // namespace

int fa_workspace_bytes(const mlzc_fa_desc* d, size_t* out) {
    if (d->k_type != MLZC_TYPE_F16) return faq_workspace_bytes(d, current_sms(), out);
    FaPlan pl;
    const int st = make_plan(d, &pl);
    *out = st == MLZC_OK ? pl.ws_bytes : 0;
    return st;
}

namespace {

// Error word of calls made without a library context (the allocation-free entry point):
// a device variable of this module, so it needs no allocation either.
__device__ unsigned int g_fa_static_err;
std::mutex g_fa_err_mu;
unsigned int* g_fa_err_addr[64] = {};

unsigned int* static_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_fa_err_mu);
    if (!g_fa_err_addr[dev]) {
        void* a = nullptr;
        if (cudaGetSymbolAddress(&a, g_fa_static_err) != cudaSuccess) return nullptr;
        g_fa_err_addr[dev] = static_cast<unsigned int*>(a);
    }
    return g_fa_err_addr[dev];
}

template <int D>
int fa_launch(const FaPlan& pl, cudaStream_t s) {
    const bool gen = pl.p.mask || pl.p.use_softcap || pl.p.alibi_p2inv != 0.0f;
    if (gen)
        MLZC_CUDA_TRY(launch_pdl(fa_decode_kernel<D, true>, dim3(pl.ctas), dim3(kFaThreads), FaCfg<D>::kSmemBytes, s, pl.p));
    else
        MLZC_CUDA_TRY(launch_pdl(fa_decode_kernel<D, false>, dim3(pl.ctas), dim3(kFaThreads), FaCfg<D>::kSmemBytes, s, pl.p));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    const dim3 g((unsigned)pl.p.rows_total, (unsigned)pl.p.n_hidx, (unsigned)pl.p.nB);
    MLZC_CUDA_TRY(launch_pdl(fa_combine_kernel<D>, g, dim3(D), 0, s, pl.p, pl.ctas));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

}  // namespace

int fa_take_static_errors(unsigned int* out) {
    *out = 0;
    unsigned int* a = static_error_word();
    if (!a) return MLZC_OK;
    unsigned int v = 0;
    MLZC_CUDA_TRY(cudaMemcpy(&v, a, sizeof v, cudaMemcpyDeviceToHost));
    if (v) MLZC_CUDA_TRY(cudaMemset(a, 0, sizeof v));
    *out = v;
    return MLZC_OK;
}

int launch_flash_attn(const DeviceCtx* c, const mlzc_fa_desc* d, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (d->k_type != MLZC_TYPE_F16) return launch_flash_attn_quant(c ? c->sm_count : current_sms(), d, ws, ws_bytes, s);
    FaPlan pl;
    int st = make_plan(d, &pl);
    if (st != MLZC_OK) return st;
    if (pl.ws_bytes > ws_bytes || !ws)
        return fail(MLZC_ERR_NOMEM, "flash_attn: workspace of %zu bytes needed, %zu given", pl.ws_bytes, ws_bytes);
    if ((reinterpret_cast<uintptr_t>(ws) & 15) != 0) return fail(MLZC_ERR_INVALID, "flash_attn: workspace not 16-byte aligned");
    FaParams& p = pl.p;
    p.q = reinterpret_cast<const char*>(d->q);
    p.mask = reinterpret_cast<const char*>(d->mask);
    p.dst = reinterpret_cast<char*>(d->dst);
    p.pref_out = static_cast<int*>(ws);
    p.part = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.pref_bytes);
    p.kv_len = d->kv_len;
    p.q_nb1 = d->q_nb[1]; p.q_nb2 = d->q_nb[2]; p.q_nb3 = d->q_nb[3];
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
    p.err = c ? c->err : static_error_word();
    if (!p.err) return fail(MLZC_ERR_CUDA, "flash_attn: no device error word");
    if (d->n_kv > 0) {
        st = encode_kv_map(&p.tm_k, d->k, d->head_dim_k, d->n_kv, d->n_head_kv, d->batch_size, d->k_nb, &p.k_hmul,
                           &p.k_bmul);
        if (st != MLZC_OK) return st;
        st = encode_kv_map(&p.tm_v, d->v, d->head_dim_v, d->n_kv, d->n_head_kv, d->batch_size, d->v_nb, &p.v_hmul,
                           &p.v_bmul);
        if (st != MLZC_OK) return st;
    }
    const int D = (int)d->head_dim_k;
    for (int64_t b0 = 0; b0 < d->batch_size; b0 += pl.slice) {
        p.b_base = (int)b0;
        p.nB = (int)std::min<int64_t>(pl.slice, d->batch_size - b0);
        if (D == 64) st = fa_launch<64>(pl, s);
        else if (D == 128) st = fa_launch<128>(pl, s);
        else st = fa_launch<256>(pl, s);
        if (st != MLZC_OK) return st;
    }
    return MLZC_OK;
}

}  // namespace mlzc

// ======================================================================
// Allocation-free flash-attention decode (mlzc_flash_attn_dev_noalloc).
//
// Some callers cannot allocate device memory for each call: code that runs where a
// cudaMalloc would synchronise the device or be refused (a host callback, a thread that
// must never block behind other streams, an engine whose memory is fully budgeted up
// front), or a binding that simply has no allocator to hand us a workspace.  For them
// this variant keeps the decode kernel's prefix table and partial records in one fixed
// scratch array that lives in the library's device image instead of a caller workspace.
//
// The array is a file-scope __device__ variable, so every GPU that loads this library
// holds kNoAllocScratchBytes of it until the process exits, whether or not the entry
// point is used.  Host code cannot use the array's name as a device address (on the host
// it names a stand-in object), so the device address is looked up with
// cudaGetSymbolAddress -- once per device, on the first call made while that device is
// current, and cached.  That first call therefore does the set-up; make it before any
// stream capture.
//
// Every call shares the one array and it keeps whatever the previous call left in it.
// Nothing in it has to start at zero: each call writes every partial record it later
// reads.  Calls whose kernels overlap on the GPU (on different streams, or from several
// host threads) race on the array and corrupt each other's results; serialise them.
// ======================================================================
namespace mlzc {
namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;   // 16 MiB per device
static __device__ __align__(256) float g_fa_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};

}  // namespace
}  // namespace mlzc

extern "C" int mlzc_flash_attn_dev_noalloc(const mlzc_fa_desc* desc, void* stream) {
    using namespace mlzc;
    int st = check_fa_args(desc);
    if (st != MLZC_OK) return st;
    size_t need = 0;
    st = fa_workspace_bytes(desc, &need);
    if (st != MLZC_OK) return st;
    if (need > kNoAllocScratchBytes)
        return fail(MLZC_ERR_NOMEM,
                    "flash_attn (allocation-free): this call needs %zu bytes of split scratch but the fixed "
                    "scratch holds %zu; use mlzc_flash_attn_dev with a workspace",
                    need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    {
        int dev = 0;
        MLZC_CUDA_TRY(cudaGetDevice(&dev));
        if (dev < 0 || dev >= kNoAllocMaxDevices)
            return fail(MLZC_ERR_INVALID, "flash_attn (allocation-free): device %d beyond %d", dev, kNoAllocMaxDevices);
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_addr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_fa_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(flash-attention scratch)");
            g_noalloc_addr[dev] = p;
        }
        scratch = g_noalloc_addr[dev];
    }
    return launch_flash_attn(nullptr, desc, scratch, kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
}
