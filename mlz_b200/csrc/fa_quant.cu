// fa_quant.cu -- flash-attention decode over a quantised KV cache (Q8_0, Q4_0, Q4_1, Q5_0,
// Q5_1 or IQ4_NL K and V) or an F32 one.
//
// Replaces the quantised-KV and F32 branches of flash_attn_dispatch
// (src/simd/flash_attention.cpp:112-248: simd_flash_attn_<type>_avx512, i.e. the FA2
// skeleton flash_attn_fa2_skeleton_avx512.inc with the DEQUANT_K_DOT_BLOCK /
// DEQUANT_V_ACCUM_BLOCK macros of kernels/x86/flash/flash_attn_<type>_avx512.asm).
// Element d of a row, per 32-value block (GGUF layouts; values 0-15 in the low nibbles,
// 16-31 in the high ones; Q5_x: bit d of the 32-bit qh is value d's fifth bit):
//   Q8_0 (34 B)  f16 d * int8 q            Q4_0 (18 B)   d * (nibble - 8)
//   Q4_1 (20 B)  d * nibble + f16 m        Q5_0 (22 B)   d * (q5 - 16)
//   Q5_1 (24 B)  d * q5 + m                IQ4_NL (18 B) d * code_book[nibble]
//   F32          the value itself (head_dim 64 or 128)
// The score order is the F16 kernel's: s = <q * scale, k> + mask, softcap, + ALiBi.
//
// Design (split-K flash decoding on the tensor cores; the rows are 72-136 bytes for D = 128,
// not 16-byte multiples, so no TMA map describes them):
//   - a CTA (four warps) owns one segment -- one sequence, one KV head, up to 8 query rows
//     sharing it (GQA packing, as the F16 kernel) -- and one contiguous range of up to
//     tiles_per_split 64-key tiles (grid.x = splits; CTAs past a sequence's end only write
//     an empty record);
//   - the raw K and V rows of each tile stream into a 2-stage shared-memory ring with
//     cp.async (16-byte chunks when a head's rows are contiguous, else 8- or 4-byte
//     pieces per row; rows past the sequence's end are zero-filled);
//   - warp w owns keys 16 w .. 16 w + 15 of every tile, with its own online softmax.
//     Scores S^T = K . Q^T and the update O^T += V^T . P^T run on mma.sync m16n8k16 (keys
//     on M for S, dims on M for O, up to 8 query rows on N), Q and P split into f16 hi + lo
//     as in the F16 kernel.  The quantised values enter as exact f16 integers (int8, or a
//     nibble with its fifth bit OR-ed into the mantissa, minus the type's offset: one LOP3
//     + PRMT + HSUB2 / HFMA2 per pair; IQ4_NL through a shared-memory table from a byte to
//     the f16 pair of its two code-book values) and the f16 block scales d are applied in
//     f32: per key and 32-dim block on the score partial sums, and per key and block on P
//     before the V^T . P^T step -- the reference's own order (q . (d k) as (q . k) d per
//     block).  A block minimum m adds m * (the block's sum of the scaled query) to a score
//     and sum_keys p * m to every dim of the block of O (kept per lane, rescaled with O,
//     added at the end).  F32 values are split into f16 hi + lo like Q and P;
//   - at the end the four warps' (max, sum, O) states are merged through shared memory into
//     one partial record per row and a combine kernel merges a segment's records in split
//     order (results repeat bit for bit).
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
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
    int kcopy, vcopy;          // copy width of a tile's rows: 16 (contiguous rows), 8 or 4
};

using ptx::mma16816;
using ptx::movtrans;
using ptx::split_h2;

// Block layouts (ggml type ids; 32 values per block, GGUF element order: value i < 16 in
// the low nibble of quant byte i, value i >= 16 in the high nibble of byte i - 16; Q5_x:
// bit i of the 32-bit qh is value i's fifth bit).  kQs / kQh: byte offsets of the quants and
// of qh (-1: none); kMin: a block minimum m (f16 at offset 2) is added to every value.
template <int TYPE>
struct KvFormat;
template <>
struct KvFormat<0> {   // F32 rows, taken 32 values (128 bytes) at a time; no scale
    static constexpr int kBlockBytes = 128, kQs = 0, kQh = -1;
    static constexpr bool kMin = false;
};
template <>
struct KvFormat<8> {   // Q8_0: f16 d, 32 int8; d * q
    static constexpr int kBlockBytes = 34, kQs = 2, kQh = -1;
    static constexpr bool kMin = false;
};
template <>
struct KvFormat<2> {   // Q4_0: f16 d, 16 bytes of nibbles; d * (q - 8)
    static constexpr int kBlockBytes = 18, kQs = 2, kQh = -1;
    static constexpr bool kMin = false;
};
template <>
struct KvFormat<3> {   // Q4_1: f16 d, f16 m, 16 bytes of nibbles; d * q + m
    static constexpr int kBlockBytes = 20, kQs = 4, kQh = -1;
    static constexpr bool kMin = true;
};
template <>
struct KvFormat<6> {   // Q5_0: f16 d, u32 qh, 16 bytes of nibbles; d * (q5 - 16)
    static constexpr int kBlockBytes = 22, kQs = 6, kQh = 2;
    static constexpr bool kMin = false;
};
template <>
struct KvFormat<7> {   // Q5_1: f16 d, f16 m, u32 qh, 16 bytes of nibbles; d * q5 + m
    static constexpr int kBlockBytes = 24, kQs = 8, kQh = 4;
    static constexpr bool kMin = true;
};
template <>
struct KvFormat<20> {  // IQ4_NL: f16 d, 16 bytes of 4-bit codes; d * kIq4nl[q]
    static constexpr int kBlockBytes = 18, kQs = 2, kQh = -1;
    static constexpr bool kMin = false;
};

// IQ4_NL's non-linear code book (the GGUF table, the LUT of
// kernels/x86/flash/flash_attn_iq4_nl_avx512.asm:34-35).
__constant__ int8_t kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

constexpr int kQStages = 2;

__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 lds_f2(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float lds_f16(uint32_t a) { return __half2float(__ushort_as_half((unsigned short)lds_u16(a))); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Two int8 values (bytes 0 and 1 of x) -> exact f16 pair: bias to unsigned, place under the
// 1024 exponent (0x64 bytes), subtract 1024 + 128.
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t x) {
    const uint32_t u = __byte_perm(x ^ 0x8080u, 0x6464u, 0x5140u);
    return h2_bits(__hsub2(bits_h2(u), __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480))));
}
// A nibble pair in f16 form -- u = (byte0, 0x64, byte1, 0x64) as two halves, from one key's
// u16 load (prmt) or from two keys' (pair_cols) -- plus the pair's fifth bits already placed
// (hb: bits 4 / 20 for low nibbles, 8 / 24 for high ones; 0 for 4-bit types) -> the exact
// f16 pair of the type's integer values: q - 8 (Q4_0), q (Q4_1, Q5_1 with its fifth bit),
// q5 - 16 (Q5_0).  Low nibbles read as 1024 + q, high ones as 1024 + 16 q.
template <int TYPE, bool HI>
__device__ __forceinline__ uint32_t nib_to_h2(uint32_t u, uint32_t hb) {
    if constexpr (!HI) {
        constexpr unsigned short kSub = TYPE == 2 ? 0x6408 : (TYPE == 6 ? 0x6410 : 0x6400);   // 1032 / 1040 / 1024
        const __half2 k = __halves2half2(__ushort_as_half(kSub), __ushort_as_half(kSub));
        return h2_bits(__hsub2(bits_h2((u & 0xFF0FFF0Fu) | hb), k));
    } else {
        constexpr unsigned short kAdd = TYPE == 2 ? 0xD480 : (TYPE == 6 ? 0xD500 : 0xD400);   // -72 / -80 / -64
        const __half2 k = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));   // 1/16
        const __half2 c = __halves2half2(__ushort_as_half(kAdd), __ushort_as_half(kAdd));
        return h2_bits(__hfma2(bits_h2((u & 0xFFF0FFF0u) | hb), k, c));
    }
}
// Fifth bits of one key's pair: bits s, s + 1 of h to bits 4 and 20 (low nibbles) or 8 and
// 24 (high nibbles).  v * (2^4 + 2^19) puts bit 0 of v at 4 and bit 1 at 20 (and copies at 19
// and 5 that the mask drops); likewise 2^8 + 2^23 for 8 and 24.
__device__ __forceinline__ uint32_t fifth_lo(uint32_t h, int s) { return (((h >> s) & 3u) * 0x80010u) & 0x100010u; }
__device__ __forceinline__ uint32_t fifth_hi(uint32_t h, int s) { return (((h >> s) & 3u) * 0x800100u) & 0x1000100u; }
// The 32-bit qh of a block at a 2-byte-aligned shared address.
__device__ __forceinline__ uint32_t lds_qh(uint32_t a) { return __byte_perm(lds_u16(a), lds_u16(a + 2), 0x5410); }
// IQ4_NL: the f16 pair (value of the low nibble, value of the high nibble) of byte x, from
// the 256-entry table at shared address tab.
__device__ __forceinline__ uint32_t iq4_byte(uint32_t tab, uint32_t x) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(tab + 4 * x));
    return v;
}

// Column pair (bytes 0 of a and b) and (bytes 1 of a and b) of two keys' u16 loads.
__device__ __forceinline__ void pair_cols(uint32_t a, uint32_t b, uint32_t& c0, uint32_t& c1) {
    const uint32_t z = __byte_perm(a, b, 0x5410u);   // a.b0 a.b1 b.b0 b.b1
    c0 = __byte_perm(z, 0x6464u, 0x4240u);           // a.b0 64 b.b0 64
    c1 = __byte_perm(z, 0x6464u, 0x4341u);           // a.b1 64 b.b1 64
}

__device__ __forceinline__ void cp_async(uint32_t dst, const void* src, int bytes, int src_bytes) {
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
    else if (bytes == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Issues the copies of `valid` rows (of RB bytes, row j at src + j * stride) into dst
// (rows packed at RB); rows valid..63 are zero-filled.  mode 16: the 64 rows are one
// contiguous 16-byte-aligned range; 8 / 4: per-row pieces of that width.
template <int RB>
__device__ __forceinline__ void copy_tile(uint32_t dst, const char* src, int64_t stride, int valid, int mode) {
    if (mode == 16) {
        constexpr int kChunks = kQTile * RB / 16;
        const int vb = valid * RB;
        for (int c = threadIdx.x; c < kChunks; c += kQThreads) {
            const int off = 16 * c;
            const int n = min(16, max(0, vb - off));
            cp_async(dst + off, src + (n > 0 ? off : 0), 16, n);
        }
    } else {
        const int w = mode;
        const int per = RB / w;
        for (int i = threadIdx.x; i < kQTile * per; i += kQThreads) {
            const int j = i / per, c = i - j * per;
            const bool ok = j < valid;
            cp_async(dst + j * RB + c * w, src + (ok ? (int64_t)j * stride + c * w : 0), w, ok ? w : 0);
        }
    }
}

template <int D, int TYPE, bool GEN>
__global__ void __launch_bounds__(kQThreads)
fa_quant_kernel(const FaqParams p) {
    using F = KvFormat<TYPE>;
    constexpr int NB = D / 32;                  // blocks per row
    constexpr int RB = NB * F::kBlockBytes;     // bytes per row
    constexpr int KS = D / 16;                  // 16-dim steps
    constexpr uint32_t kTileBytes = kQTile * RB;
    extern __shared__ __align__(16) unsigned char fq_smem[];
    // [stage][K, V] raw tiles (the merge area [4 warps][8 rows][D + 2] once they are done),
    // then the Q^T fragment table [KS][32 lanes] x uint4 (hi0, hi1, lo0, lo1), the block sums
    // of the scaled query rows [NB][8] (types with a block minimum) and the IQ4_NL byte table
    constexpr uint32_t kRing = kQStages * 2 * kTileBytes;
    constexpr uint32_t kMerge = 4 * kQRows * (D + 2) * 4;
    constexpr uint32_t kQtabOff = kRing > kMerge ? kRing : kMerge;
    const uint32_t ring = ptx::smem_u32(fq_smem);
    uint4* qtab = reinterpret_cast<uint4*>(fq_smem + kQtabOff);
    float* qsum = reinterpret_cast<float*>(fq_smem + kQtabOff + KS * 32 * 16);
    uint32_t* iqtab = reinterpret_cast<uint32_t*>(fq_smem + kQtabOff + KS * 32 * 16 + 256);
    float* mrg = reinterpret_cast<float*>(fq_smem);   // after the last tile (ring drained)

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, g = lane >> 2, q4 = lane & 3;
    const int split = blockIdx.x, seg = blockIdx.y, ib = p.b_base + blockIdx.z;
    const int hidx = seg / p.n_rgroups, rg = seg % p.n_rgroups;
    const int head_base = p.packed ? hidx * p.G : hidx;
    const int ihkv = p.packed ? hidx : hidx * p.n_head_kv / p.n_head_q;
    const int r0 = rg * kQRows;
    const int nrows = min(kQRows, p.rows_total - r0);

    ptx::pdl_launch_dependents();
    ptx::pdl_wait();
    const int L = p.kv_len ? min(max(ptx::ld_act(p.kv_len + ib), 0), p.n_kv) : p.n_kv;
    const int tile0 = split * p.tiles_per_split;
    const int tile1 = min(tile0 + p.tiles_per_split, (L + kQTile - 1) / kQTile);
    float* rec = p.part + ((((size_t)blockIdx.z * p.HR + seg) * p.splits + split) * kQRows) * (D + 2);
    if (tile0 >= tile1) {
        // no key of this split: an empty record (the combine skips it)
        if (t < kQRows) { rec[t * (D + 2)] = -INFINITY; rec[t * (D + 2) + 1] = 0.0f; }
        return;
    }
    const char* kbase = p.k + ihkv * p.k_nb2 + ib * p.k_nb3;
    const char* vbase = p.v + ihkv * p.v_nb2 + ib * p.v_nb3;
    auto load_tile = [&](int tile, int stage) {
        const int j0 = tile * kQTile;
        const int valid = min(kQTile, L - j0);
        const uint32_t dk = ring + (uint32_t)stage * 2 * kTileBytes;
        copy_tile<RB>(dk, kbase + (int64_t)j0 * p.k_nb1, p.k_nb1, valid, p.kcopy);
        copy_tile<RB>(dk + kTileBytes, vbase + (int64_t)j0 * p.v_nb1, p.v_nb1, valid, p.vcopy);
    };
    const int ntiles = tile1 - tile0;
#pragma unroll
    for (int i = 0; i < kQStages - 1; ++i) {
        if (i < ntiles) load_tile(tile0 + i, i);
        cp_commit();
    }
    // Q^T fragments (scaled, f16 hi + lo): entry (ks, lane) = row g, dims 16 ks + {2 q4, +1, +8, +9}
    for (int e = t; e < KS * 32; e += kQThreads) {
        const int ks = e >> 5, l = e & 31, gr = l >> 2, qq = l & 3;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        if (gr < nrows) {
            const int rr = r0 + gr, iq = rr / p.G, ihq = head_base + rr % p.G;
            const float* qr = reinterpret_cast<const float*>(p.q + iq * p.q_nb1 + ihq * p.q_nb2 + ib * p.q_nb3);
            const int d0 = 16 * ks + 2 * qq;
            x[0] = ptx::ld_act(qr + d0) * p.scale;
            x[1] = ptx::ld_act(qr + d0 + 1) * p.scale;
            x[2] = ptx::ld_act(qr + d0 + 8) * p.scale;
            x[3] = ptx::ld_act(qr + d0 + 9) * p.scale;
        }
        uint4 f;
        split_h2(x[0], x[1], f.x, f.z);
        split_h2(x[2], x[3], f.y, f.w);
        qtab[e] = f;
    }
    if constexpr (F::kMin) {
        // sum over each block's 32 dims of the scaled query: the block minimum m adds
        // m * sum to a score (value = d q + m)
        for (int e = t; e < NB * kQRows; e += kQThreads) {
            const int b = e / kQRows, gr = e % kQRows;
            float sum = 0.0f;
            if (gr < nrows) {
                const int rr = r0 + gr, iq = rr / p.G, ihq = head_base + rr % p.G;
                const float* qr = reinterpret_cast<const float*>(p.q + iq * p.q_nb1 + ihq * p.q_nb2 + ib * p.q_nb3);
                for (int d = 32 * b; d < 32 * b + 32; ++d) sum += ptx::ld_act(qr + d) * p.scale;
            }
            qsum[e] = sum;
        }
    }
    if constexpr (TYPE == 20) {
        // byte x -> f16 pair (code book value of its low nibble, of its high nibble)
        for (int x = t; x < 256; x += kQThreads)
            iqtab[x] = (uint32_t)__half_as_ushort(__float2half_rn((float)kIq4nl[x & 15])) |
                       ((uint32_t)__half_as_ushort(__float2half_rn((float)kIq4nl[x >> 4])) << 16);
    }
    const uint32_t iqtab_u = ptx::smem_u32(iqtab);
    // per-lane row state: rows 2 q4 and 2 q4 + 1
    int iq_r[2], ihq_r[2];
    bool row_ok[2];
    float slope[2], m_row[2], l_row[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int r = 2 * q4 + h;
        row_ok[h] = r < nrows;
        const int rr = r0 + (row_ok[h] ? r : 0);
        iq_r[h] = rr / p.G;
        ihq_r[h] = head_base + rr % p.G;
        slope[h] = p.alibi_p2inv != 0.0f ? exp2f(p.alibi_p2inv * (float)(ihq_r[h] + 1)) : 0.0f;
        m_row[h] = -INFINITY;
        l_row[h] = 0.0f;
    }
    float o[KS][4];
#pragma unroll
    for (int d = 0; d < KS; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
    // block-minimum part of O (sum over this lane's keys of p * m per block and row; its
    // lanes' sums are joined into o at the end)
    float macc[F::kMin ? NB : 1][2];
#pragma unroll
    for (int b = 0; b < (F::kMin ? NB : 1); ++b) macc[b][0] = macc[b][1] = 0.0f;
    const int kw = warp * 16;
    const uint32_t qtab_u = ptx::smem_u32(qtab) + (uint32_t)lane * 16;

    for (int i = 0; i < ntiles; ++i) {
        cp_wait<kQStages - 2>();
        __syncthreads();   // tile i has landed for every thread; stage (i - 1) % S is free
        if (i + kQStages - 1 < ntiles) load_tile(tile0 + i + kQStages - 1, (i + kQStages - 1) % kQStages);
        cp_commit();
        const uint32_t kb = ring + (uint32_t)(i % kQStages) * 2 * kTileBytes;
        const uint32_t vb = kb + kTileBytes;
        const int j0 = (tile0 + i) * kQTile;
        // ---- S^T (keys kw + g, kw + g + 8; rows 2 q4, +1): per block, two 16-dim steps
        const uint32_t kr0 = kb + (uint32_t)(kw + g) * RB, kr1 = kr0 + 8 * RB;
        float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float th[4] = {0.f, 0.f, 0.f, 0.f}, tl[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t o0 = kr0 + b * F::kBlockBytes + F::kQs, o1 = kr1 + b * F::kBlockBytes + F::kQs;
            if constexpr (TYPE == 0) {
                // f32 keys as f16 hi + lo: K.Q = Khi.Qhi + Khi.Qlo + Klo.Qhi (the dropped
                // Klo.Qlo term is ~2^-22 relative)
#pragma unroll
                for (int st = 0; st < 2; ++st) {
                    const uint32_t e0 = o0 + 4 * (16 * st + 2 * q4), e1 = o1 + 4 * (16 * st + 2 * q4);
                    const float2 k0 = lds_f2(e0), k1 = lds_f2(e1), k2 = lds_f2(e0 + 32), k3 = lds_f2(e1 + 32);
                    uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
                    split_h2(k0.x, k0.y, h0, l0);
                    split_h2(k1.x, k1.y, h1, l1);
                    split_h2(k2.x, k2.y, h2, l2);
                    split_h2(k3.x, k3.y, h3, l3);
                    const uint4 qf = lds_v4(qtab_u + (uint32_t)(2 * b + st) * 512);
                    mma16816(th, h0, h1, h2, h3, qf.x, qf.y);
                    mma16816(tl, h0, h1, h2, h3, qf.z, qf.w);
                    mma16816(tl, l0, l1, l2, l3, qf.x, qf.y);
                }
            } else if constexpr (TYPE == 8) {
#pragma unroll
                for (int st = 0; st < 2; ++st) {
                    const uint32_t a0 = i8x2_to_h2(lds_u16(o0 + 16 * st + 2 * q4));
                    const uint32_t a1 = i8x2_to_h2(lds_u16(o1 + 16 * st + 2 * q4));
                    const uint32_t a2 = i8x2_to_h2(lds_u16(o0 + 16 * st + 2 * q4 + 8));
                    const uint32_t a3 = i8x2_to_h2(lds_u16(o1 + 16 * st + 2 * q4 + 8));
                    const uint4 qf = lds_v4(qtab_u + (uint32_t)(2 * b + st) * 512);
                    mma16816(th, a0, a1, a2, a3, qf.x, qf.y);
                    mma16816(tl, a0, a1, a2, a3, qf.z, qf.w);
                }
            } else {
                // nibble types: low nibbles are dims 0-15 of the block, high nibbles dims 16-31;
                // w0 / w2: key g, bytes 2 q4 (+1) / 2 q4 + 8 (+9); w1 / w3: key g + 8
                const uint32_t w[4] = {lds_u16(o0 + 2 * q4), lds_u16(o1 + 2 * q4), lds_u16(o0 + 2 * q4 + 8),
                                       lds_u16(o1 + 2 * q4 + 8)};
                uint32_t lo[4], hi[4];
                if constexpr (TYPE == 20) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t t0 = iq4_byte(iqtab_u, w[k] & 0xFFu), t1 = iq4_byte(iqtab_u, w[k] >> 8);
                        lo[k] = __byte_perm(t0, t1, 0x5410u);
                        hi[k] = __byte_perm(t0, t1, 0x7632u);
                    }
                } else {
                    uint32_t hl[4] = {0u, 0u, 0u, 0u}, hh[4] = {0u, 0u, 0u, 0u};
                    if constexpr (F::kQh >= 0) {
                        // fifth bits of this lane's values: bits 2 q4 + {0, 1, 8, 9, 16, 17, 24, 25}
                        const uint32_t h0 = lds_qh(kr0 + b * F::kBlockBytes + F::kQh) >> (2 * q4);
                        const uint32_t h1 = lds_qh(kr1 + b * F::kBlockBytes + F::kQh) >> (2 * q4);
                        hl[0] = fifth_lo(h0, 0); hl[1] = fifth_lo(h1, 0);
                        hl[2] = fifth_lo(h0, 8); hl[3] = fifth_lo(h1, 8);
                        hh[0] = fifth_hi(h0, 16); hh[1] = fifth_hi(h1, 16);
                        hh[2] = fifth_hi(h0, 24); hh[3] = fifth_hi(h1, 24);
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t u = __byte_perm(w[k], 0x6464u, 0x5140u);
                        lo[k] = nib_to_h2<TYPE, false>(u, hl[k]);
                        hi[k] = nib_to_h2<TYPE, true>(u, hh[k]);
                    }
                }
                {
                    const uint4 qf = lds_v4(qtab_u + (uint32_t)(2 * b) * 512);
                    mma16816(th, lo[0], lo[1], lo[2], lo[3], qf.x, qf.y);
                    mma16816(tl, lo[0], lo[1], lo[2], lo[3], qf.z, qf.w);
                }
                {
                    const uint4 qf = lds_v4(qtab_u + (uint32_t)(2 * b + 1) * 512);
                    mma16816(th, hi[0], hi[1], hi[2], hi[3], qf.x, qf.y);
                    mma16816(tl, hi[0], hi[1], hi[2], hi[3], qf.z, qf.w);
                }
            }
            const float d0 = TYPE == 0 ? 1.0f : lds_f16(kr0 + b * F::kBlockBytes);
            const float d1 = TYPE == 0 ? 1.0f : lds_f16(kr1 + b * F::kBlockBytes);
            sacc[0] = fmaf(d0, th[0] + tl[0], sacc[0]);
            sacc[1] = fmaf(d0, th[1] + tl[1], sacc[1]);
            sacc[2] = fmaf(d1, th[2] + tl[2], sacc[2]);
            sacc[3] = fmaf(d1, th[3] + tl[3], sacc[3]);
            if constexpr (F::kMin) {
                const float m0 = lds_f16(kr0 + b * F::kBlockBytes + 2), m1 = lds_f16(kr1 + b * F::kBlockBytes + 2);
                const float2 qs = *reinterpret_cast<const float2*>(qsum + b * kQRows + 2 * q4);   // rows 2 q4, + 1
                sacc[0] = fmaf(m0, qs.x, sacc[0]);
                sacc[1] = fmaf(m0, qs.y, sacc[1]);
                sacc[2] = fmaf(m1, qs.x, sacc[2]);
                sacc[3] = fmaf(m1, qs.y, sacc[3]);
            }
        }
        // ---- mask / softcap / ALiBi / validity; element e: key g + 8 (e >> 1), row 2 q4 + (e & 1)
        float sc[4], tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int h = e & 1;
            const int j = j0 + kw + g + 8 * (e >> 1);
            float a = sacc[e];
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
            for (int d = 0; d < KS; ++d) {
                o[d][0] *= corr[0]; o[d][1] *= corr[1];
                o[d][2] *= corr[0]; o[d][3] *= corr[1];
            }
            if constexpr (F::kMin) {
#pragma unroll
                for (int b = 0; b < NB; ++b) { macc[b][0] *= corr[0]; macc[b][1] *= corr[1]; }
            }
        }
        float pe[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int h = e & 1;
            pe[e] = (sc[e] == -INFINITY) ? 0.0f : __expf(sc[e] - m_row[h]);
            l_row[h] += pe[e];
        }
        // ---- O^T += V^T . (P d_V)^T, per 32-dim block.  Within a 16-dim output tile, MMA
        // row g is dim 2 g and row g + 8 dim 2 g + 1 (so a lane's pair of loads feeds both).
        const uint32_t vk0 = vb + (uint32_t)(kw + 2 * q4) * RB;    // keys 2 q4, 2 q4 + 1
        const uint32_t vk8 = vk0 + 8 * RB;                          // keys 2 q4 + 8, + 9
        const uint32_t vd0 = vb + (uint32_t)(kw + g) * RB, vd8 = vd0 + 8 * RB;   // keys g, g + 8 (scales)
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float dv0 = TYPE == 0 ? 1.0f : lds_f16(vd0 + b * F::kBlockBytes);
            const float dv8 = TYPE == 0 ? 1.0f : lds_f16(vd8 + b * F::kBlockBytes);
            uint32_t h0, l0, h1, l1;
            split_h2(pe[0] * dv0, pe[1] * dv0, h0, l0);   // key g
            split_h2(pe[2] * dv8, pe[3] * dv8, h1, l1);   // key g + 8
            const uint32_t bh0 = movtrans(h0), bh1 = movtrans(h1), bl0 = movtrans(l0), bl1 = movtrans(l1);
            const uint32_t base0 = vk0 + b * F::kBlockBytes + F::kQs + 2 * g, base8 = vk8 + b * F::kBlockBytes + F::kQs + 2 * g;
            if constexpr (TYPE == 0) {
                // f32 values as f16 hi + lo: V.P = Vhi.Phi + Vhi.Plo + Vlo.Phi
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const uint32_t e = 4 * (32 * b + 16 * hf + 2 * g);   // dims 2 g, 2 g + 1 of the tile
                    const float2 va = lds_f2(vk0 + e), vb2 = lds_f2(vk0 + RB + e);   // keys 2 q4, 2 q4 + 1
                    const float2 vc = lds_f2(vk8 + e), vd = lds_f2(vk8 + RB + e);    // keys 2 q4 + 8, + 9
                    uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
                    split_h2(va.x, vb2.x, h0, l0);
                    split_h2(va.y, vb2.y, h1, l1);
                    split_h2(vc.x, vd.x, h2, l2);
                    split_h2(vc.y, vd.y, h3, l3);
                    mma16816(o[2 * b + hf], h0, h1, h2, h3, bh0, bh1);
                    mma16816(o[2 * b + hf], h0, h1, h2, h3, bl0, bl1);
                    mma16816(o[2 * b + hf], l0, l1, l2, l3, bh0, bh1);
                }
            } else if constexpr (TYPE == 8) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t c00, c01, c80, c81;
                    pair_cols(lds_u16(base0 + 16 * hf) ^ 0x8080u, lds_u16(base0 + RB + 16 * hf) ^ 0x8080u, c00, c01);
                    pair_cols(lds_u16(base8 + 16 * hf) ^ 0x8080u, lds_u16(base8 + RB + 16 * hf) ^ 0x8080u, c80, c81);
                    const __half2 k = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
                    const uint32_t a0 = h2_bits(__hsub2(bits_h2(c00), k)), a1 = h2_bits(__hsub2(bits_h2(c01), k));
                    const uint32_t a2 = h2_bits(__hsub2(bits_h2(c80), k)), a3 = h2_bits(__hsub2(bits_h2(c81), k));
                    mma16816(o[2 * b + hf], a0, a1, a2, a3, bh0, bh1);
                    mma16816(o[2 * b + hf], a0, a1, a2, a3, bl0, bl1);
                }
            } else {
                // fragments (dims 2 g | 2 g + 1 of keys 2 q4, 2 q4 + 1 | 2 q4 + 8, 2 q4 + 9):
                // low nibbles -> o[2 b] (dims 0-15 of the block), high nibbles -> o[2 b + 1]
                uint32_t lo[4], hi[4];
                if constexpr (TYPE == 20) {
                    const uint32_t x[4] = {lds_u16(base0), lds_u16(base0 + RB), lds_u16(base8), lds_u16(base8 + RB)};
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        const uint32_t a = x[2 * pr], c = x[2 * pr + 1];
                        const uint32_t ta0 = iq4_byte(iqtab_u, a & 0xFFu), ta1 = iq4_byte(iqtab_u, a >> 8);
                        const uint32_t tc0 = iq4_byte(iqtab_u, c & 0xFFu), tc1 = iq4_byte(iqtab_u, c >> 8);
                        lo[2 * pr] = __byte_perm(ta0, tc0, 0x5410u);
                        lo[2 * pr + 1] = __byte_perm(ta1, tc1, 0x5410u);
                        hi[2 * pr] = __byte_perm(ta0, tc0, 0x7632u);
                        hi[2 * pr + 1] = __byte_perm(ta1, tc1, 0x7632u);
                    }
                } else {
                    uint32_t c[4];
                    pair_cols(lds_u16(base0), lds_u16(base0 + RB), c[0], c[1]);
                    pair_cols(lds_u16(base8), lds_u16(base8 + RB), c[2], c[3]);
                    uint32_t hl[4] = {0u, 0u, 0u, 0u}, hh[4] = {0u, 0u, 0u, 0u};
                    if constexpr (F::kQh >= 0) {
                        // fifth bits 2 g, 2 g + 1 (low) and 16 + 2 g, 17 + 2 g (high) of the four keys
                        const uint32_t qa = lds_qh(vk0 + b * F::kBlockBytes + F::kQh) >> (2 * g);
                        const uint32_t qb = lds_qh(vk0 + RB + b * F::kBlockBytes + F::kQh) >> (2 * g);
                        const uint32_t qc = lds_qh(vk8 + b * F::kBlockBytes + F::kQh) >> (2 * g);
                        const uint32_t qd = lds_qh(vk8 + RB + b * F::kBlockBytes + F::kQh) >> (2 * g);
                        // byte 0 (bits 2 g, 2 g + 1) and byte 2 (16 + 2 g, 17 + 2 g) of two keys' qh
                        // side by side: bit j of key A's byte at j, of key B's at 16 + j
                        const uint32_t zab = __byte_perm(qa, qb, 0x5410u), zcd = __byte_perm(qc, qd, 0x5410u);
                        const uint32_t zab2 = __byte_perm(qa, qb, 0x7632u), zcd2 = __byte_perm(qc, qd, 0x7632u);
                        hl[0] = (zab & 0x00010001u) << 4; hl[1] = (zab & 0x00020002u) << 3;
                        hl[2] = (zcd & 0x00010001u) << 4; hl[3] = (zcd & 0x00020002u) << 3;
                        hh[0] = (zab2 & 0x00010001u) << 8; hh[1] = (zab2 & 0x00020002u) << 7;
                        hh[2] = (zcd2 & 0x00010001u) << 8; hh[3] = (zcd2 & 0x00020002u) << 7;
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        lo[k] = nib_to_h2<TYPE, false>(c[k], hl[k]);
                        hi[k] = nib_to_h2<TYPE, true>(c[k], hh[k]);
                    }
                }
                mma16816(o[2 * b], lo[0], lo[1], lo[2], lo[3], bh0, bh1);
                mma16816(o[2 * b], lo[0], lo[1], lo[2], lo[3], bl0, bl1);
                mma16816(o[2 * b + 1], hi[0], hi[1], hi[2], hi[3], bh0, bh1);
                mma16816(o[2 * b + 1], hi[0], hi[1], hi[2], hi[3], bl0, bl1);
            }
            if constexpr (F::kMin) {
                const float mv0 = lds_f16(vd0 + b * F::kBlockBytes + 2), mv8 = lds_f16(vd8 + b * F::kBlockBytes + 2);
                macc[b][0] = fmaf(pe[0], mv0, fmaf(pe[2], mv8, macc[b][0]));
                macc[b][1] = fmaf(pe[1], mv0, fmaf(pe[3], mv8, macc[b][1]));
            }
        }
    }
    cp_wait<0>();
    if constexpr (F::kMin) {
        // the block-minimum part: summed over the warp's keys (the lanes sharing q4), added to
        // every dim of the block
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v = macc[b][h];
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                v += __shfl_xor_sync(0xffffffffu, v, 8);
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                o[2 * b][h] += v; o[2 * b][2 + h] += v;
                o[2 * b + 1][h] += v; o[2 * b + 1][2 + h] += v;
            }
        }
    }
    // ---- merge the four warps' states into one record per row
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        l_row[h] += __shfl_xor_sync(0xffffffffu, l_row[h], 4);
        l_row[h] += __shfl_xor_sync(0xffffffffu, l_row[h], 8);
        l_row[h] += __shfl_xor_sync(0xffffffffu, l_row[h], 16);
    }
    __syncthreads();   // the ring and the Q table are no longer read
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float* mr = mrg + (warp * kQRows + 2 * q4 + h) * (D + 2);
        if (g == 0) { mr[0] = m_row[h]; mr[1] = l_row[h]; }
        // tile d: MMA rows g, g + 8 = dims 16 d + 2 g, + 1
#pragma unroll
        for (int d = 0; d < KS; ++d) {
            mr[2 + 16 * d + 2 * g] = o[d][h];
            mr[2 + 16 * d + 2 * g + 1] = o[d][2 + h];
        }
    }
    __syncthreads();
    for (int e = t; e < kQRows * (D + 2); e += kQThreads) {
        const int r = e / (D + 2), c = e - r * (D + 2);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, mrg[(w * kQRows + r) * (D + 2)]);
        float v;
        if (c == 0) {
            v = M;
        } else {
            v = 0.0f;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float m = mrg[(w * kQRows + r) * (D + 2)];
                if (m != -INFINITY) v += __expf(m - M) * mrg[(w * kQRows + r) * (D + 2) + c];
            }
        }
        rec[e] = v;
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
    // Splits of 4..64 tiles, sized for ~T CTAs per SM over the launch if every sequence had
    // n_kv keys: ragged batches then still fill several waves (CTAs past a sequence's end
    // exit at once), and the partial records stay a few percent of the K/V bytes.  T per
    // type, measured on B200 over T in {2 .. 32} on the C7 batch (us per call, chosen T / 8):
    // Q4_0 12 (44.5 / 53.2), Q5_1 12 (66.7 / 82.5), F32 6 (157 / 163); Q8_0, Q4_1, Q5_0 and
    // IQ4_NL 8 (12 was level for Q8_0 and Q5_0, 9-15 % slower for Q4_1 and IQ4_NL).
    const int64_t segs = (int64_t)pl.slice * p.HR;
    const int64_t T = (d->k_type == MLZC_TYPE_Q4_0 || d->k_type == MLZC_TYPE_Q5_1) ? 12
                      : d->k_type == MLZC_TYPE_F32                                 ? 6
                                                                                   : 8;
    const int64_t want = (int64_t)tiles * segs / std::max<int64_t>(1, T * sm_count);
    p.tiles_per_split = (int)std::min<int64_t>(std::max<int64_t>(4, want), 64);
    p.tiles_per_split = std::min(p.tiles_per_split, tiles);
    p.splits = (tiles + p.tiles_per_split - 1) / p.tiles_per_split;
    if (p.splits > 65535) return fail(MLZC_ERR_INVALID, "flash_attn: too many key tiles");
    const int RB = (int)fa_row_bytes(d->k_type, D);
    // the merge area of the four warps reuses the ring
    const size_t ring = (size_t)kQStages * 2 * kQTile * RB;
    // + the Q^T fragment table, the query block sums (256 bytes) and the IQ4_NL byte table (1 KB)
    pl.smem = std::max(ring, (size_t)4 * kQRows * (D + 2) * 4) + (size_t)(D / 16) * 32 * 16 + 256 + 1024;
    pl.ws_bytes = (size_t)pl.slice * p.HR * p.splits * kQRows * (D + 2) * 4;
    *out = pl;
    return MLZC_OK;
}

template <int D, int TYPE, bool GEN>
int faq_launch(const FaqPlan& pl, cudaStream_t s) {
    static std::atomic<bool> attr[64] = {};
    int dev = 0;
    MLZC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr[dev].load()) {
        // the largest dynamic size any call of this instantiation asks for (the ring and
        // table depend on D and the type only)
        MLZC_CUDA_TRY(cudaFuncSetAttribute(fa_quant_kernel<D, TYPE, GEN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)pl.smem));
        if (dev >= 0 && dev < 64) attr[dev].store(true);
    }
    const dim3 g((unsigned)pl.p.splits, (unsigned)pl.p.HR, (unsigned)pl.p.nB);
    MLZC_CUDA_TRY(launch_pdl(fa_quant_kernel<D, TYPE, GEN>, g, dim3(kQThreads), pl.smem, s, pl.p));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    const dim3 gc((unsigned)kQRows, (unsigned)pl.p.HR, (unsigned)pl.p.nB);
    MLZC_CUDA_TRY(launch_pdl(fa_quant_combine_kernel<D>, gc, dim3(std::min(D, 128)), 0, s, pl.p));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

template <int TYPE, bool GEN>
int faq_dispatch(const FaqPlan& pl, int D, cudaStream_t s) {
    if (D == 64) return faq_launch<64, TYPE, GEN>(pl, s);
    if (D == 128) return faq_launch<128, TYPE, GEN>(pl, s);
    if constexpr (TYPE == 0) {
        // f32 rows of 256 dims: two stages of 64-key K and V tiles are 256 KB (the gate declines it)
        return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: F32 K/V with head_dim %d", D);
    } else {
        return faq_launch<256, TYPE, GEN>(pl, s);
    }
}

// Widest cp.async piece every row of a tile can be copied with: 16 when a head's rows are
// contiguous and 16-byte aligned (a tile is then one range), else 8 or 4 per row.
int copy_mode(const void* base, int64_t nb1, int64_t nb2, int64_t nb3, int rb) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    if (nb1 == rb && a % 16 == 0 && nb2 % 16 == 0 && nb3 % 16 == 0) return 16;
    if (rb % 8 == 0 && a % 8 == 0 && nb1 % 8 == 0 && nb2 % 8 == 0 && nb3 % 8 == 0) return 8;
    return 4;
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
    const int RB = (int)fa_row_bytes(d->k_type, D);
    p.kcopy = copy_mode(d->k, d->k_nb[1], d->k_nb[2], d->k_nb[3], RB);
    p.vcopy = copy_mode(d->v, d->v_nb[1], d->v_nb[2], d->v_nb[3], RB);
    const bool gen = p.mask != nullptr || p.use_softcap || p.alibi_p2inv != 0.0f;
    for (int64_t b0 = 0; b0 < d->batch_size; b0 += pl.slice) {
        p.b_base = (int)b0;
        p.nB = (int)std::min<int64_t>(pl.slice, d->batch_size - b0);
        switch (d->k_type) {
            case MLZC_TYPE_F32: st = gen ? faq_dispatch<0, true>(pl, D, s) : faq_dispatch<0, false>(pl, D, s); break;
            case MLZC_TYPE_Q8_0: st = gen ? faq_dispatch<8, true>(pl, D, s) : faq_dispatch<8, false>(pl, D, s); break;
            case MLZC_TYPE_Q4_0: st = gen ? faq_dispatch<2, true>(pl, D, s) : faq_dispatch<2, false>(pl, D, s); break;
            case MLZC_TYPE_Q4_1: st = gen ? faq_dispatch<3, true>(pl, D, s) : faq_dispatch<3, false>(pl, D, s); break;
            case MLZC_TYPE_Q5_0: st = gen ? faq_dispatch<6, true>(pl, D, s) : faq_dispatch<6, false>(pl, D, s); break;
            case MLZC_TYPE_Q5_1: st = gen ? faq_dispatch<7, true>(pl, D, s) : faq_dispatch<7, false>(pl, D, s); break;
            case MLZC_TYPE_IQ4_NL:
                st = gen ? faq_dispatch<20, true>(pl, D, s) : faq_dispatch<20, false>(pl, D, s);
                break;
            default: return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: K/V type %d", d->k_type);
        }
        if (st != MLZC_OK) return st;
    }
    return MLZC_OK;
}

}  // namespace mlzc
