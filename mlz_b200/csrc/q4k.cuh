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
