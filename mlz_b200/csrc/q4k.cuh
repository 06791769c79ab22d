// q4k.cuh -- Q4_K block arithmetic shared by the Q4_K kernels: the exact f16 dequant of a
// nibble pair (sc * q as one LOP3 + one HFMA2) and the per-row scale unpack.
//
// Q4_K block (GGUF, 144 bytes per 256 weights): d (f16) @0, dmin (f16) @2, twelve bytes of
// packed 6-bit (sc, m) for the 8 sub-blocks of 32 @4, 128 nibble bytes @16 where byte b of
// 32-byte chunk c holds element b of sub-block 2c (low nibble) and of sub-block 2c+1 (high
// nibble).  The 6-bit (sc, m) unpack is that of src/simd/kernels/x86/vec/
// vec_dot_q4_k_q8_k_avx2.asm:101-150 (get_scale_min_k4), done for two sub-blocks at once.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace mlzc {
namespace q4k {

constexpr int kQK = 256;          // weights per block
constexpr int kBlockBytes = 144;  // bytes per block

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Per row and block: the HFMA2 constants that turn nibble bits into sc * q for sub-blocks
// 2c (low nibbles) and 2c+1 (high nibbles), the (m_2c, m_2c+1) pair, and d, dmin.
struct RowScales {
    __half2 mul_lo, add_lo, mul_hi, add_hi;
    uint32_t mpair;
    float d, dmin;
};

// The scale constants of rows g (header h0) and g + 8 (header h1) for sub-blocks j = 2c,
// 2c + 1.  Scale bytes s[0..11] = hdr.y (s0-s3), hdr.z (s4-s7), hdr.w (s8-s11); this
// thread needs byte pair j' = 2 (c & 1), +1 of each word, and one byte permute per word
// packs both rows' pairs into one register (row g in bytes 0-1, row g + 8 in bytes 2-3),
// so the 6-bit unpack runs once for the two rows:
//   j < 4:  sc = s[j] & 63, m = s[j+4] & 63
//   j >= 4: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4, m = (s[j+4] >> 4) | (s[j] >> 6) << 4
__device__ __forceinline__ void row_scales2(const uint4& h0, const uint4& h1, int c, RowScales& s0, RowScales& s1) {
    const uint32_t sel = (c & 1) ? 0x7632u : 0x5410u;
    const uint32_t A = __byte_perm(h0.y, h1.y, sel), B = __byte_perm(h0.z, h1.z, sel), Cw = __byte_perm(h0.w, h1.w, sel);
    uint32_t sc, m;
    if (c < 2) {
        sc = A & 0x3F3F3F3Fu;
        m = B & 0x3F3F3F3Fu;
    } else {
        sc = (Cw & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u);
        m = ((Cw >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u);
    }
    const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
    const uint32_t selr[2] = {0x5140u, 0x5342u};
    RowScales* out[2] = {&s0, &s1};
    const uint4* hd[2] = {&h0, &h1};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const __half2 sch = __hsub2(u2h(__byte_perm(sc, 0x6464u, selr[r])), k1024);
        RowScales& o = *out[r];
        o.mpair = h2u(__hsub2(u2h(__byte_perm(m, 0x6464u, selr[r])), k1024));
        const __half2 lo = __low2half2(sch), hi = __high2half2(sch);
        o.mul_lo = lo;
        o.add_lo = __hmul2(lo, __float2half2_rn(-1024.0f));
        o.mul_hi = __hmul2(hi, __float2half2_rn(0.0625f));
        o.add_hi = __hmul2(hi, __float2half2_rn(-64.0f));
        const __half2 dd = u2h(hd[r]->x);
        o.d = __low2float(dd);
        o.dmin = __high2float(dd);
    }
}

// (w & mask) | 0x64006400 as one LOP3 with the magic constant in a register (written as two
// C operations, each with an immediate, it measured as two integer instructions per call).
template <uint32_t kMask>
__device__ __forceinline__ uint32_t nib_f16x2(uint32_t w) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "n"(kMask), "r"(0x64006400u));
    return d;
}
__device__ __forceinline__ uint32_t deq_lo(uint32_t w, const RowScales& s) {
    return h2u(__hfma2(u2h(nib_f16x2<0x000F000Fu>(w)), s.mul_lo, s.add_lo));
}
__device__ __forceinline__ uint32_t deq_hi(uint32_t w, const RowScales& s) {
    return h2u(__hfma2(u2h(nib_f16x2<0x00F000F0u>(w)), s.mul_hi, s.add_hi));
}

}  // namespace q4k
}  // namespace mlzc
