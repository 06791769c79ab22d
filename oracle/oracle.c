/*
 * oracle.c -- CPU restatement of MLz's src/simd mul_mat / Q4_K / flash-attention
 * decode math.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and the
 * CPU-baseline leg of bench.py link this file; the shipped CUDA library never does.
 *
 * Two kinds of functions live here:
 *   ora_*   exact checkers.  fp64 accumulation, plain C, no SIMD.  These define
 *           "the right answer" for the GPU kernels.
 *   base_*  timed CPU baselines.  AVX-512 / AVX2 restatements of the reference's
 *           own loop structure, threaded over all host cores the way the reference
 *           hook splits rows.  They are what bench.py reports as the CPU number.
 *
 * Citations are path:line inside the MLz project.
 *
 * Parity status: the reference ships no golden vectors or known-answer tests for
 * any of these kernels (src/bench_simd.zig:90-99 only times random bytes).  The Q4_K
 * dequantisation is pinned against the gguf 0.19.0 Python decoder (fixtures under
 * tests/golden/); flash-attention decode is pinned against the reference's own
 * flash_attn_quantized (src/simd/flash_attention.cpp:291-410) compiled from source
 * into oracle/_ref.  The F16 GEMM contract (upstream ggml_vec_dot_f16, not vendored
 * with the reference) is unpinned beyond the reference's scalar matmul fallback.
 *
 * Build: see oracle/Makefile (-O2 -ffp-contract=off so that the f32 dequant is
 * bit-identical to the gguf decoder's numpy arithmetic).
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------------- */
/* IEEE binary16 <-> binary32 (portable, round-to-nearest-even)               */
/* ------------------------------------------------------------------------- */

/* Same contract as F16C vcvtph2ps and as the scalar path of convert_f16_to_f32
 * (src/simd/simd_matmul.cpp:318-365): exact widening, subnormals kept. */
float ora_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
        }
    } else if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Round-to-nearest-even narrowing, the contract of F16C vcvtps2ph with imm 0 and
 * of upstream ggml_cpu_fp32_to_fp16, which the reference's F16 mul_mat path applies
 * to every activation (src/simd/ggml-cpu-simd.c:215-220, 1314-1350). */
uint16_t ora_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) {                       /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477FF000u) {                       /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7C00u);
    }
    if (ax < 0x38800000u) {                        /* below smallest normal half */
        if (ax < 0x33000000u) return (uint16_t)sign;   /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;                     /* biased f32 exponent */
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e;                 /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

void ora_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = ora_f32_to_f16(src[i]);
}

void ora_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = ora_f16_to_f32(src[i]);
}

/* ------------------------------------------------------------------------- */
/* mul_mat in ggml layout                                                     */
/*   W  : M rows of K weights, row m at W + m*w_row_bytes (src0, ne = [K, M])  */
/*   X  : N columns of K f32, column n at X + n*x_col_bytes (src1, ne = [K, N])*/
/*   Y  : N x M, element (m, n) at Y[n*M + m]   (dst, ne = [M, N], nb1 = 4M)   */
/* Layout contract: src/simd/ggml-cpu-simd.c:1246-1300 (GGML_ASSERTs on nb).  */
/* ------------------------------------------------------------------------- */

/* F16 weights.  With round_x != 0 the activations are first narrowed to f16, which
 * is what the reference's actual F16 path does (type_traits_cpu[F16].vec_dot_type =
 * F16, src/simd/ggml-cpu-simd.c:215-220, conversion loop :1314-1350); products are
 * then exact and summed in fp64. */
void ora_mul_mat_f16(const uint16_t* W, size_t w_row_bytes, int64_t M, int64_t K,
                     const float* X, size_t x_col_bytes, int64_t N,
                     double* Y, int round_x) {
    double* xd = (double*)malloc(sizeof(double) * (size_t)(K * (N > 0 ? N : 1)));
    double* wd = (double*)malloc(sizeof(double) * (size_t)(K > 0 ? K : 1));
    for (int64_t n = 0; n < N; n++) {
        const float* xc = (const float*)((const char*)X + n * x_col_bytes);
        for (int64_t k = 0; k < K; k++) {
            xd[n * K + k] = round_x ? (double)ora_f16_to_f32(ora_f32_to_f16(xc[k])) : (double)xc[k];
        }
    }
    for (int64_t m = 0; m < M; m++) {
        const uint16_t* wr = (const uint16_t*)((const char*)W + m * w_row_bytes);
        for (int64_t k = 0; k < K; k++) wd[k] = (double)ora_f16_to_f32(wr[k]);
        for (int64_t n = 0; n < N; n++) {
            const double* xn = xd + n * K;
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += wd[k] * xn[k];
            Y[n * M + m] = acc;
        }
    }
    free(xd);
    free(wd);
}

/* F32 weights: the hook's F32 branch (src/simd/ggml_simd_hook.cpp:304-311) routed to
 * simd_matmul_f32 (src/simd/simd_matmul.cpp:214-251), here with ggml's real layout. */
void ora_mul_mat_f32(const float* W, size_t w_row_bytes, int64_t M, int64_t K,
                     const float* X, size_t x_col_bytes, int64_t N, double* Y) {
    for (int64_t n = 0; n < N; n++) {
        const float* xc = (const float*)((const char*)X + n * x_col_bytes);
        for (int64_t m = 0; m < M; m++) {
            const float* wr = (const float*)((const char*)W + m * w_row_bytes);
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += (double)wr[k] * (double)xc[k];
            Y[n * M + m] = acc;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Q4_K super-blocks (GGUF layout, 144 bytes per 256 weights)                 */
/*   @0 d (f16)  @2 dmin (f16)  @4 scales[12] (6-bit sc/m x 8)  @16 qs[128]    */
/* Field offsets: src/simd/kernels/x86/vec/vec_dot_q4_k_q8_k_avx2.asm:80-150.  */
/* ------------------------------------------------------------------------- */

#define ORA_QK_K 256
#define ORA_Q4K_BYTES 144
#define ORA_Q8K_BYTES 292
#define ORA_Q6K_BYTES 210

/* 6-bit scale/min unpack of sub-block j, as the AVX2 kernel does it
 * (vec_dot_q4_k_q8_k_avx2.asm:101-150). */
void ora_q4k_scale_min(const uint8_t* scales, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = scales[j] & 63;
        *m = scales[j + 4] & 63;
    } else {
        *sc = (scales[j + 4] & 0x0F) | ((scales[j - 4] >> 6) << 4);
        *m = (scales[j + 4] >> 4) | ((scales[j] >> 6) << 4);
    }
}

/* Dequantise one row of K/256 blocks to f32.  Nibble order is GGUF's: in each
 * 64-value chunk c, qs[32c+l] holds value 64c+l in its low nibble (sub-block 2c)
 * and value 64c+32+l in its high nibble (sub-block 2c+1).  The f32 arithmetic
 * (d*sc)*q - (dmin*m) matches the gguf 0.19.0 decoder bit for bit. */
void ora_q4k_dequant_row(const uint8_t* blocks, int64_t K, float* out) {
    const int64_t nb = K / ORA_QK_K;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * ORA_Q4K_BYTES;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        const float d = ora_f16_to_f32(dh);
        const float dmin = ora_f16_to_f32(mh);
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + 16;
        float* o = out + b * ORA_QK_K;
        for (int c = 0; c < 4; c++) {
            int sc0, m0, sc1, m1;
            ora_q4k_scale_min(scales, 2 * c, &sc0, &m0);
            ora_q4k_scale_min(scales, 2 * c + 1, &sc1, &m1);
            const float d0 = d * (float)sc0, mm0 = dmin * (float)m0;
            const float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
            for (int l = 0; l < 32; l++) {
                const uint8_t q = qs[32 * c + l];
                o[64 * c + l] = d0 * (float)(q & 0x0F) - mm0;
                o[64 * c + 32 + l] = d1 * (float)(q >> 4) - mm1;
            }
        }
    }
}

/* Q4_K weight x f32 activation, fp64 accumulation of the dequantised f32 weights:
 * the "dequantised F32 product" the Q4_K parity gate is defined against. */
void ora_mul_mat_q4k(const uint8_t* W, size_t w_row_bytes, int64_t M, int64_t K,
                     const float* X, size_t x_col_bytes, int64_t N, double* Y) {
    float* wf = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t m = 0; m < M; m++) {
        ora_q4k_dequant_row(W + m * w_row_bytes, K, wf);
        for (int64_t n = 0; n < N; n++) {
            const float* xc = (const float*)((const char*)X + n * x_col_bytes);
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += (double)wf[k] * (double)xc[k];
            Y[n * M + m] = acc;
        }
    }
    free(wf);
}

/* Q6_K (GGUF, 210 bytes per 256 weights): ql[128] @0 (low 4 bits), qh[64] @128 (high 2
 * bits), 16 int8 scales @192 (one per 16 weights), f16 d @208.  Element p of a block
 * (h = p / 128, r = p % 128, l = r % 32, k = r / 32): low bits = nibble k / 2 of
 * ql[64h + 32 (k % 2) + l], high bits = bits 2k, 2k+1 of qh[32h + l]; q = (lo | hi << 4)
 * - 32; w = (d * scales[p / 16]) * q in f32 -- the layout and arithmetic of the gguf
 * 0.19.0 decoder (gguf/quants.py Q6_K.dequantize_blocks), bit for bit.  The reference
 * hook routes Q6_K weights like Q4_K (src/simd/ggml_simd_hook.cpp:282-288; block size
 * src/bench_simd.zig:34-40). */
void ora_q6k_dequant_row(const uint8_t* blocks, int64_t K, float* out) {
    const int64_t nb = K / ORA_QK_K;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * ORA_Q6K_BYTES;
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        uint16_t dh;
        memcpy(&dh, blk + 208, 2);
        const float d = ora_f16_to_f32(dh);
        float* o = out + b * ORA_QK_K;
        for (int p = 0; p < ORA_QK_K; p++) {
            const int h = p / 128, r = p % 128, l = r % 32, k = r / 32;
            const int lo = (ql[64 * h + 32 * (k % 2) + l] >> (4 * (k / 2))) & 0x0F;
            const int hi = (qh[32 * h + l] >> (2 * k)) & 0x03;
            const int q = (lo | (hi << 4)) - 32;
            const float ds = d * (float)sc[p / 16];
            o[p] = ds * (float)q;
        }
    }
}

/* Q6_K weight x f32 activation, fp64 accumulation of the dequantised f32 weights (the
 * dequantised-F32 product the Q6_K parity gate is defined against). */
void ora_mul_mat_q6k(const uint8_t* W, size_t w_row_bytes, int64_t M, int64_t K,
                     const float* X, size_t x_col_bytes, int64_t N, double* Y) {
    float* wf = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t m = 0; m < M; m++) {
        ora_q6k_dequant_row(W + m * w_row_bytes, K, wf);
        for (int64_t n = 0; n < N; n++) {
            const float* xc = (const float*)((const char*)X + n * x_col_bytes);
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += (double)wf[k] * (double)xc[k];
            Y[n * M + m] = acc;
        }
    }
    free(wf);
}

/* F32 -> Q8_K (292 bytes: f32 d, 256 x int8, 16 x int16 bsums), restating
 * quantize_row_q8_k_reference (src/simd/ggml_simd_hook.cpp:109-148): d = amax/127,
 * q = round-half-away(x/d), bsums over groups of 16. */
void ora_quantize_row_q8k(const float* x, int64_t K, uint8_t* out) {
    const int64_t nb = K / ORA_QK_K;
    for (int64_t b = 0; b < nb; b++) {
        const float* xb = x + b * ORA_QK_K;
        uint8_t* blk = out + b * ORA_Q8K_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < ORA_QK_K; j++) {
            const float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        memcpy(blk, &d, 4);
        int8_t* qs = (int8_t*)(blk + 4);
        for (int j = 0; j < ORA_QK_K; j++) qs[j] = (int8_t)roundf(xb[j] * id);
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += qs[16 * g + l];
            const int16_t s16 = (int16_t)s;
            memcpy(blk + 260 + 2 * g, &s16, 2);
        }
    }
}

/* Q4_K . Q8_K super-block dot: sum_b y.d * (d * sum_j sc_j <q4_j, q8_j>
 * - dmin * sum_j m_j (bsum_2j + bsum_2j+1)), the math of
 * vec_dot_q4_k_q8_k_avx2.asm:72-234, with the nibble order and y.d of GGUF
 * (the reference kernels' nibble interleave differs from GGUF). */
float ora_vec_dot_q4k_q8k(int64_t K, const uint8_t* vx, const uint8_t* vy) {
    const int64_t nb = K / ORA_QK_K;
    float sum = 0.0f;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* x = vx + b * ORA_Q4K_BYTES;
        const uint8_t* y = vy + b * ORA_Q8K_BYTES;
        uint16_t dh, mh;
        float dy;
        memcpy(&dh, x, 2);
        memcpy(&mh, x + 2, 2);
        memcpy(&dy, y, 4);
        const float sd = ora_f16_to_f32(dh) * dy;
        const float smin = ora_f16_to_f32(mh) * dy;
        const int8_t* q8 = (const int8_t*)(y + 4);
        for (int j = 0; j < 8; j++) {
            int sc, m;
            ora_q4k_scale_min(x + 4, j, &sc, &m);
            const uint8_t* qs = x + 16 + 32 * (j / 2);
            const int shift = (j & 1) ? 4 : 0;
            int dot = 0;
            for (int l = 0; l < 32; l++) dot += ((qs[l] >> shift) & 0x0F) * q8[32 * j + l];
            int16_t b0, b1;
            memcpy(&b0, y + 260 + 4 * j, 2);
            memcpy(&b1, y + 262 + 4 * j, 2);
            sum += (float)dot * (sd * (float)sc);
            sum -= (smin * (float)m) * (float)(b0 + b1);
        }
    }
    return sum;
}

/* ------------------------------------------------------------------------- */
/* Flash-attention decode (one query position per sequence in the tests, but  */
/* any n_q is accepted).  Byte strides follow flash_attn_config_t             */
/* (src/simd/flash_attention.h:65-114); the loop restates the FA2 skeleton     */
/* (kernels/x86/flash/flash_attn_fa2_skeleton_avx512.inc:394-842) and the      */
/* readable statement flash_attn_quantized (src/simd/flash_attention.cpp:291-410)*/
/* in fp64 with exact exp.  Score order: dot*scale, + mask, softcap, + ALiBi.  */
/* Mask element (iq, j) is at iq*mask_nb1 + j*mask_nb0 (the skeleton's indexing,*/
/* :618-636; flash_attention.cpp:352 transposes it).                          */
/* ------------------------------------------------------------------------- */

typedef struct {
    int64_t head_dim_k, head_dim_v, n_queries, n_kv, n_head_q, n_head_kv, batch_size;
    float scale, logit_softcap, max_bias;
    uint32_t mode;                  /* bit 0x08 ALiBi, 0x10 softcap, as FA_MODE_* */
    const float* q;                 /* f32 */
    const uint16_t* k;              /* f16 */
    const uint16_t* v;              /* f16 */
    const float* mask;              /* f32 or NULL */
    float* dst;                     /* f32 */
    size_t q_nb[4], k_nb[4], v_nb[4], mask_nb[4], dst_nb[4];
    const int32_t* kv_len;          /* per batch element, NULL = n_kv for all */
    int32_t kv_type;                /* K/V element type (ggml ids): 0 F32, 1 F16, 8 Q8_0, 2 Q4_0,
                                       3 Q4_1, 6 Q5_0, 7 Q5_1, 20 IQ4_NL */
} ora_fa_t;

/* Bytes of one 32-value block of a quantised KV-cache type (ggml ids), 0 for F16. */
static int64_t ora_kv_block_bytes(int32_t type) {
    switch (type) {
        case 8: return 34;   /* Q8_0   */
        case 2: return 18;   /* Q4_0   */
        case 3: return 20;   /* Q4_1   */
        case 6: return 22;   /* Q5_0   */
        case 7: return 24;   /* Q5_1   */
        case 20: return 18;  /* IQ4_NL */
        default: return 0;
    }
}

/* The 16 values of IQ4_NL's non-linear 4-bit code (the GGUF table, also the LUT of
 * flash_attn_iq4_nl_avx512.asm:34-35). */
static const int8_t ora_iq4nl_values[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                            1, 13, 25, 38, 53, 69, 89, 113};

/* One 32-value block of a quantised KV row as f32, in the GGUF element order (value i < 16
 * from the low nibble of quant byte i, value i >= 16 from the high nibble of byte i - 16;
 * Q5_x: bit i of the 32-bit qh is value i's fifth bit).  Each value is formed in f32 as the
 * gguf 0.19.0 decoders (gguf/quants.py) and the reference's DEQUANT_K_DOT_BLOCK macros form it:
 *   Q8_0  (34 B: f16 d, 32 int8)              d * q
 *   Q4_0  (18 B: f16 d, 16 B nibbles)         d * (q - 8)      flash_attn_q4_0_avx512.asm
 *   Q4_1  (20 B: f16 d, f16 m, 16 B nibbles)  d * q + m        flash_attn_q4_1_avx512.asm:7-13
 *   Q5_0  (22 B: f16 d, u32 qh, 16 B)         d * (q5 - 16)    flash_attn_q5_0_avx512.asm:9-15
 *   Q5_1  (24 B: f16 d, f16 m, u32 qh, 16 B)  d * q5 + m       flash_attn_q5_1_avx512.asm:7-14
 *   IQ4_NL (18 B: f16 d, 16 B nibbles)        d * table[q]     flash_attn_iq4_nl_avx512.asm:7-13
 * (d * q is exact in f32, so d * q + m has one rounding whether or not it is fused.) */
static void ora_kv_block(const unsigned char* blk, int32_t type, float* o) {
    const float d = ora_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    if (type == 8) {
        for (int i = 0; i < 32; i++) o[i] = d * (float)(int8_t)blk[2 + i];
        return;
    }
    float m = 0.0f;
    const unsigned char* qs = blk + 2;
    uint32_t qh = 0;
    if (type == 3 || type == 7) {
        m = ora_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        qs = blk + 4;
    }
    if (type == 6 || type == 7) {
        const unsigned char* h = type == 6 ? blk + 2 : blk + 4;
        qh = (uint32_t)h[0] | ((uint32_t)h[1] << 8) | ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
        qs = h + 4;
    }
    for (int i = 0; i < 32; i++) {
        const int q4 = i < 16 ? (qs[i] & 0x0F) : (qs[i - 16] >> 4);
        const int q5 = q4 | (int)(((qh >> i) & 1u) << 4);
        switch (type) {
            case 2: o[i] = d * (float)(q4 - 8); break;
            case 3: o[i] = d * (float)q4 + m; break;
            case 6: o[i] = d * (float)(q5 - 16); break;
            case 7: o[i] = d * (float)q5 + m; break;
            default: o[i] = d * (float)ora_iq4nl_values[q4]; break;   /* 20: IQ4_NL */
        }
    }
}

/* Element d of a K or V row of type `type` (0 = F32, 1 = F16, or a quantised type above) as
 * f32. */
static float ora_kv_elem(const char* row, int64_t d, int32_t type) {
    const int64_t bb = ora_kv_block_bytes(type);
    if (bb) {
        float blk[32];
        ora_kv_block((const unsigned char*)row + (d / 32) * bb, type, blk);
        return blk[d % 32];
    }
    if (type == 0) {
        float f;
        memcpy(&f, row + 4 * d, 4);
        return f;
    }
    uint16_t h;
    memcpy(&h, row + 2 * d, 2);
    return ora_f16_to_f32(h);
}

/* A whole K/V row of type `type` (dv values) as f32, block by block (the same products as
 * ora_kv_elem, so the same bits). */
void ora_kv_row(const char* row, int64_t dv, int32_t type, float* out) {
    const int64_t bb = ora_kv_block_bytes(type);
    if (bb) {
        for (int64_t b = 0; b < dv / 32; b++) ora_kv_block((const unsigned char*)row + b * bb, type, out + 32 * b);
        return;
    }
    for (int64_t d = 0; d < dv; d++) out[d] = ora_kv_elem(row, d, type);
}

static double ora_alibi_slope(int64_t h, int64_t n_heads, float max_bias) {
    /* flash_attention.cpp:278-285 fixes max_bias at 8 (base 2^(-8/n)); the
     * restatement keeps that constant: the reference ignores max_bias's value. */
    (void)max_bias;
    int64_t p2 = 1;
    while (p2 < n_heads) p2 <<= 1;
    const double base = pow(2.0, -8.0 / (double)p2);
    return pow(base, (double)(h + 1));
}

void ora_flash_attn(const ora_fa_t* c) {
    const int64_t DK = c->head_dim_k, DV = c->head_dim_v;
    double* s = (double*)malloc(sizeof(double) * (size_t)(c->n_kv > 0 ? c->n_kv : 1));
    double* o = (double*)malloc(sizeof(double) * (size_t)DV);
    float* row = (float*)malloc(sizeof(float) * (size_t)(DK > DV ? DK : DV));   /* one decoded K / V row */
    for (int64_t ib = 0; ib < c->batch_size; ib++) {
        const int64_t L = c->kv_len ? c->kv_len[ib] : c->n_kv;
        for (int64_t ihq = 0; ihq < c->n_head_q; ihq++) {
            const int64_t ihkv = ihq * c->n_head_kv / c->n_head_q;
            const double slope = (c->mode & 0x08u) ? ora_alibi_slope(ihq, c->n_head_q, c->max_bias) : 0.0;
            for (int64_t iq = 0; iq < c->n_queries; iq++) {
                const float* qr = (const float*)((const char*)c->q + iq * c->q_nb[1] + ihq * c->q_nb[2] + ib * c->q_nb[3]);
                float* dr = (float*)((char*)c->dst + iq * c->dst_nb[1] + ihq * c->dst_nb[2] + ib * c->dst_nb[3]);
                double mx = -INFINITY;
                for (int64_t j = 0; j < L; j++) {
                    const char* kr = (const char*)c->k + j * c->k_nb[1] + ihkv * c->k_nb[2] + ib * c->k_nb[3];
                    double dot = 0.0;
                    ora_kv_row(kr, DK, c->kv_type, row);
                    for (int64_t d = 0; d < DK; d++) dot += (double)qr[d] * (double)row[d];
                    double sj = dot * (double)c->scale;
                    if (c->mask) {
                        sj += (double)*(const float*)((const char*)c->mask + iq * c->mask_nb[1] + j * c->mask_nb[0]);
                    }
                    if (c->mode & 0x10u) sj = (double)c->logit_softcap * tanh(sj / (double)c->logit_softcap);
                    if (c->mode & 0x08u) sj += slope * (double)(j - iq);
                    s[j] = sj;
                    if (sj > mx) mx = sj;
                }
                for (int64_t d = 0; d < DV; d++) o[d] = 0.0;
                double l = 0.0;
                if (L > 0 && mx > -INFINITY) {
                    for (int64_t j = 0; j < L; j++) {
                        const double p = exp(s[j] - mx);
                        l += p;
                        const char* vr = (const char*)c->v + j * c->v_nb[1] + ihkv * c->v_nb[2] + ib * c->v_nb[3];
                        ora_kv_row(vr, DV, c->kv_type, row);
                        for (int64_t d = 0; d < DV; d++) o[d] += p * (double)row[d];
                    }
                }
                for (int64_t d = 0; d < DV; d++) dr[d] = l > 0.0 ? (float)(o[d] / l) : 0.0f;
            }
        }
    }
    free(s);
    free(o);
    free(row);
}

/* ========================================================================= */
/* Timed CPU baselines                                                        */
/* ========================================================================= */

typedef void (*base_task_fn)(void* arg, int ith, int nth);
typedef struct { base_task_fn fn; void* arg; int ith, nth; } base_thread_t;

static void* base_thread_main(void* p) {
    base_thread_t* t = (base_thread_t*)p;
    t->fn(t->arg, t->ith, t->nth);
    return NULL;
}

/* ggml-style fork/join: every thread gets (ith, nth) and picks its own rows. */
static void base_parallel(base_task_fn fn, void* arg, int nth) {
    if (nth < 1) nth = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nth);
    base_thread_t* ts = (base_thread_t*)malloc(sizeof(base_thread_t) * (size_t)nth);
    for (int i = 0; i < nth; i++) {
        ts[i].fn = fn; ts[i].arg = arg; ts[i].ith = i; ts[i].nth = nth;
        if (i > 0) pthread_create(&th[i], NULL, base_thread_main, &ts[i]);
    }
    base_thread_main(&ts[0]);
    for (int i = 1; i < nth; i++) pthread_join(th[i], NULL);
    free(th);
    free(ts);
}

int base_has_avx512(void) {
#if defined(__x86_64__)
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw");
#else
    return 0;
#endif
}

int base_has_avx2(void) {
#if defined(__x86_64__)
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && __builtin_cpu_supports("f16c");
#else
    return 0;
#endif
}

/* C[M x N] = A[M x K] . B[K x N], row-major f32, the loop of matrix_mult_avx512
 * (kernels/x86/matrix_mult_avx512.asm:118-282): per row, 64-column tiles held in
 * four zmm accumulators, A[i][k] broadcast and FMA'd over k ascending, masked
 * remainder columns. */
#if defined(__x86_64__)
__attribute__((target("avx512f,avx512bw,fma")))
static void base_matrix_mult_avx512(const float* A, const float* B, float* C,
                                    int64_t M, int64_t N, int64_t K) {
    for (int64_t i = 0; i < M; i++) {
        const float* a = A + i * K;
        float* c = C + i * N;
        int64_t j = 0;
        for (; j + 64 <= N; j += 64) {
            __m512 c0 = _mm512_setzero_ps(), c1 = _mm512_setzero_ps();
            __m512 c2 = _mm512_setzero_ps(), c3 = _mm512_setzero_ps();
            for (int64_t k = 0; k < K; k++) {
                const __m512 av = _mm512_set1_ps(a[k]);
                const float* b = B + k * N + j;
                c0 = _mm512_fmadd_ps(av, _mm512_loadu_ps(b), c0);
                c1 = _mm512_fmadd_ps(av, _mm512_loadu_ps(b + 16), c1);
                c2 = _mm512_fmadd_ps(av, _mm512_loadu_ps(b + 32), c2);
                c3 = _mm512_fmadd_ps(av, _mm512_loadu_ps(b + 48), c3);
            }
            _mm512_storeu_ps(c + j, c0);
            _mm512_storeu_ps(c + j + 16, c1);
            _mm512_storeu_ps(c + j + 32, c2);
            _mm512_storeu_ps(c + j + 48, c3);
        }
        for (; j < N; j += 16) {
            const int64_t rem = N - j < 16 ? N - j : 16;
            const __mmask16 mk = (__mmask16)((1u << rem) - 1u);
            __m512 c0 = _mm512_setzero_ps();
            for (int64_t k = 0; k < K; k++) {
                const __m512 av = _mm512_set1_ps(a[k]);
                c0 = _mm512_fmadd_ps(av, _mm512_maskz_loadu_ps(mk, B + k * N + j), c0);
            }
            _mm512_mask_storeu_ps(c + j, mk, c0);
        }
    }
}

/* AVX2 twin (matrix_mult_avx2.asm:71-332: 32-column tiles). */
__attribute__((target("avx2,fma")))
static void base_matrix_mult_avx2(const float* A, const float* B, float* C,
                                  int64_t M, int64_t N, int64_t K) {
    for (int64_t i = 0; i < M; i++) {
        const float* a = A + i * K;
        float* c = C + i * N;
        int64_t j = 0;
        for (; j + 32 <= N; j += 32) {
            __m256 c0 = _mm256_setzero_ps(), c1 = _mm256_setzero_ps();
            __m256 c2 = _mm256_setzero_ps(), c3 = _mm256_setzero_ps();
            for (int64_t k = 0; k < K; k++) {
                const __m256 av = _mm256_set1_ps(a[k]);
                const float* b = B + k * N + j;
                c0 = _mm256_fmadd_ps(av, _mm256_loadu_ps(b), c0);
                c1 = _mm256_fmadd_ps(av, _mm256_loadu_ps(b + 8), c1);
                c2 = _mm256_fmadd_ps(av, _mm256_loadu_ps(b + 16), c2);
                c3 = _mm256_fmadd_ps(av, _mm256_loadu_ps(b + 24), c3);
            }
            _mm256_storeu_ps(c + j, c0);
            _mm256_storeu_ps(c + j + 8, c1);
            _mm256_storeu_ps(c + j + 16, c2);
            _mm256_storeu_ps(c + j + 24, c3);
        }
        for (; j < N; j++) {
            float acc = 0.0f;
            for (int64_t k = 0; k < K; k++) acc += a[k] * B[k * N + j];
            c[j] = acc;
        }
    }
}

__attribute__((target("avx2,f16c")))
static void base_f16_to_f32(const uint16_t* s, float* d, int64_t n) {
    int64_t i = 0;
    for (; i + 8 <= n; i += 8) _mm256_storeu_ps(d + i, _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(s + i))));
    for (; i < n; i++) d[i] = ora_f16_to_f32(s[i]);
}

__attribute__((target("avx2,f16c")))
static void base_f32_to_f16(const float* s, uint16_t* d, int64_t n) {
    int64_t i = 0;
    for (; i + 8 <= n; i += 8) _mm_storeu_si128((__m128i*)(d + i), _mm256_cvtps_ph(_mm256_loadu_ps(s + i), 0));
    for (; i < n; i++) d[i] = ora_f32_to_f16(s[i]);
}
#endif

static void base_matrix_mult_scalar(const float* A, const float* B, float* C,
                                    int64_t M, int64_t N, int64_t K) {
    memset(C, 0, sizeof(float) * (size_t)(M * N));
    for (int64_t i = 0; i < M; i++)
        for (int64_t k = 0; k < K; k++) {
            const float a = A[i * K + k];
            for (int64_t j = 0; j < N; j++) C[i * N + j] += a * B[k * N + j];
        }
}

static void base_matrix_mult(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K) {
#if defined(__x86_64__)
    if (base_has_avx512()) { base_matrix_mult_avx512(A, B, C, M, N, K); return; }
    if (base_has_avx2()) { base_matrix_mult_avx2(A, B, C, M, N, K); return; }
#endif
    base_matrix_mult_scalar(A, B, C, M, N, K);
}

typedef struct {
    const uint16_t* W; size_t w_row_bytes; int64_t M, K;
    const float* Bt;        /* K x N row-major, already f16-rounded f32 */
    int64_t N;
    float* Y;               /* N x M (ggml dst) */
} base_f16_task_t;

/* One thread's share of simd_matmul_f16 (src/simd/simd_matmul.cpp:428-480):
 * rows [ith*ceil(M/nth), ...), convert the W slice to f32, run the f32 GEMM on it,
 * write the slice's outputs. */
static void base_f16_worker(void* p, int ith, int nth) {
    base_f16_task_t* t = (base_f16_task_t*)p;
    const int64_t rpt = (t->M + nth - 1) / nth;
    const int64_t r0 = (int64_t)ith * rpt;
    const int64_t r1 = r0 + rpt < t->M ? r0 + rpt : t->M;
    if (r0 >= r1) return;
    const int64_t lm = r1 - r0;
    float* A = (float*)aligned_alloc(64, (size_t)((lm * t->K * 4 + 63) / 64 * 64));
    float* C = (float*)aligned_alloc(64, (size_t)((lm * t->N * 4 + 63) / 64 * 64));
    for (int64_t i = 0; i < lm; i++) {
        const uint16_t* wr = (const uint16_t*)((const char*)t->W + (r0 + i) * t->w_row_bytes);
#if defined(__x86_64__)
        if (base_has_avx2()) base_f16_to_f32(wr, A + i * t->K, t->K); else
#endif
        ora_f16_to_f32_array(wr, A + i * t->K, t->K);
    }
    base_matrix_mult(A, t->Bt, C, lm, t->N, t->K);
    for (int64_t i = 0; i < lm; i++)
        for (int64_t n = 0; n < t->N; n++) t->Y[n * t->M + r0 + i] = C[i * t->N + n];
    free(A);
    free(C);
}

/* Timed baseline for F16 mul_mat in ggml layout: X narrowed to f16 (the contract of
 * the reference's F16 path) and transposed to the K x N operand matrix_mult expects,
 * then simd_matmul_f16's convert-then-GEMM row split over nth threads. */
void base_mul_mat_f16(const uint16_t* W, size_t w_row_bytes, int64_t M, int64_t K,
                      const float* X, size_t x_col_bytes, int64_t N, float* Y, int nth) {
    float* Bt = (float*)aligned_alloc(64, (size_t)((K * N * 4 + 63) / 64 * 64));
    uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)K);
    float* tf = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t n = 0; n < N; n++) {
        const float* xc = (const float*)((const char*)X + n * x_col_bytes);
#if defined(__x86_64__)
        if (base_has_avx2()) { base_f32_to_f16(xc, tmp, K); base_f16_to_f32(tmp, tf, K); } else
#endif
        { ora_f32_to_f16_array(xc, tmp, K); ora_f16_to_f32_array(tmp, tf, K); }
        for (int64_t k = 0; k < K; k++) Bt[k * N + n] = tf[k];
    }
    free(tmp);
    free(tf);
    base_f16_task_t t = {W, w_row_bytes, M, K, Bt, N, Y};
    base_parallel(base_f16_worker, &t, nth);
    free(Bt);
}

/* --- Q4_K x Q8_K ------------------------------------------------------- */

#if defined(__x86_64__)
/* AVX2 restatement of vec_dot_q4_k_q8_k_avx2.asm:72-234 (scalar scale unpack,
 * vpmaddubsw/vpmaddwd sub-block dots, fp32 FMA accumulate), with GGUF nibble
 * order: sub-block 2c is the low nibbles of qs[32c..32c+32), 2c+1 the high ones. */
__attribute__((target("avx2,fma,f16c")))
static float base_vec_dot_q4k_q8k_avx2(int64_t K, const uint8_t* vx, const uint8_t* vy) {
    const int64_t nb = K / ORA_QK_K;
    const __m256i lo = _mm256_set1_epi8(0x0F);
    const __m256i ones = _mm256_set1_epi16(1);
    __m256 acc = _mm256_setzero_ps();
    float mins = 0.0f;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* x = vx + b * ORA_Q4K_BYTES;
        const uint8_t* y = vy + b * ORA_Q8K_BYTES;
        uint16_t dh, mh;
        float dy;
        memcpy(&dh, x, 2);
        memcpy(&mh, x + 2, 2);
        memcpy(&dy, y, 4);
        const float sd = ora_f16_to_f32(dh) * dy;
        const float smin = ora_f16_to_f32(mh) * dy;
        for (int c = 0; c < 4; c++) {
            const __m256i q = _mm256_loadu_si256((const __m256i*)(x + 16 + 32 * c));
            const __m256i q0 = _mm256_and_si256(q, lo);
            const __m256i q1 = _mm256_and_si256(_mm256_srli_epi16(q, 4), lo);
            const __m256i y0 = _mm256_loadu_si256((const __m256i*)(y + 4 + 64 * c));
            const __m256i y1 = _mm256_loadu_si256((const __m256i*)(y + 4 + 64 * c + 32));
            const __m256i p0 = _mm256_madd_epi16(_mm256_maddubs_epi16(q0, y0), ones);
            const __m256i p1 = _mm256_madd_epi16(_mm256_maddubs_epi16(q1, y1), ones);
            int sc0, m0, sc1, m1;
            ora_q4k_scale_min(x + 4, 2 * c, &sc0, &m0);
            ora_q4k_scale_min(x + 4, 2 * c + 1, &sc1, &m1);
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p0), _mm256_set1_ps(sd * (float)sc0), acc);
            acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p1), _mm256_set1_ps(sd * (float)sc1), acc);
            int16_t bs[4];
            memcpy(bs, y + 260 + 8 * c, 8);
            mins += smin * ((float)m0 * (float)(bs[0] + bs[1]) + (float)m1 * (float)(bs[2] + bs[3]));
        }
    }
    __m128 s = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    s = _mm_hadd_ps(s, s);
    s = _mm_hadd_ps(s, s);
    return _mm_cvtss_f32(s) - mins;
}
#endif

typedef struct {
    const uint8_t* W; size_t w_row_bytes; int64_t M, K;
    const float* X; size_t x_col_bytes; int64_t N;
    float* Y;
} base_q4k_task_t;

/* One thread of ggml_simd_try_mul_mat's K-quant branch
 * (src/simd/ggml_simd_hook.cpp:234-301): each thread quantises ALL of src1 to
 * Q8_K, then runs its M-row share, one vec_dot per (m, n). */
static void base_q4k_worker(void* p, int ith, int nth) {
    base_q4k_task_t* t = (base_q4k_task_t*)p;
    const int64_t mpt = (t->M + nth - 1) / nth;
    const int64_t m0 = (int64_t)ith * mpt < t->M ? (int64_t)ith * mpt : t->M;
    const int64_t m1 = m0 + mpt < t->M ? m0 + mpt : t->M;
    if (m0 >= m1) return;
    const size_t qrow = (size_t)(t->K / ORA_QK_K) * ORA_Q8K_BYTES;
    uint8_t* q8 = (uint8_t*)malloc(qrow * (size_t)t->N);
    for (int64_t n = 0; n < t->N; n++)
        ora_quantize_row_q8k((const float*)((const char*)t->X + n * t->x_col_bytes), t->K, q8 + n * qrow);
    for (int64_t m = m0; m < m1; m++) {
        const uint8_t* wr = t->W + m * t->w_row_bytes;
        for (int64_t n = 0; n < t->N; n++) {
            float r;
#if defined(__x86_64__)
            if (base_has_avx2()) r = base_vec_dot_q4k_q8k_avx2(t->K, wr, q8 + n * qrow); else
#endif
            r = ora_vec_dot_q4k_q8k(t->K, wr, q8 + n * qrow);
            t->Y[n * t->M + m] = r;
        }
    }
    free(q8);
}

void base_mul_mat_q4k(const uint8_t* W, size_t w_row_bytes, int64_t M, int64_t K,
                      const float* X, size_t x_col_bytes, int64_t N, float* Y, int nth) {
    base_q4k_task_t t = {W, w_row_bytes, M, K, X, x_col_bytes, N, Y};
    base_parallel(base_q4k_worker, &t, nth);
}

/* Q6_K . Q8_K super-block dot: sum_b y.d * d * sum_g sc_g * sum_{i in g} (q_i - 32) q8_i,
 * the math of vec_dot_q6_k_q8_k (src/simd/kernels/x86/vec/vec_dot_q6_k_q8_k_avx2.asm),
 * with GGUF's element order; integer sums per group of 16, one float scale per block. */
static float base_vec_dot_q6k_q8k(int64_t K, const uint8_t* vx, const uint8_t* vy) {
    const int64_t nb = K / ORA_QK_K;
    float sum = 0.0f;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = vx + b * ORA_Q6K_BYTES;
        const uint8_t* yb = vy + b * ORA_Q8K_BYTES;
        float yd;
        memcpy(&yd, yb, 4);
        const int8_t* q8 = (const int8_t*)(yb + 4);
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        uint16_t dh;
        memcpy(&dh, blk + 208, 2);
        int8_t q6[256];
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 32; l++) {
                const uint8_t a = ql[64 * h + l], c = ql[64 * h + 32 + l], e = qh[32 * h + l];
                q6[128 * h + l] = (int8_t)(((a & 0x0F) | ((e & 3) << 4)) - 32);
                q6[128 * h + 32 + l] = (int8_t)(((c & 0x0F) | (((e >> 2) & 3) << 4)) - 32);
                q6[128 * h + 64 + l] = (int8_t)(((a >> 4) | (((e >> 4) & 3) << 4)) - 32);
                q6[128 * h + 96 + l] = (int8_t)(((c >> 4) | (((e >> 6) & 3) << 4)) - 32);
            }
        int isum = 0;
        for (int g = 0; g < 16; g++) {
            int gs = 0;
            for (int i = 0; i < 16; i++) gs += (int)q6[16 * g + i] * (int)q8[16 * g + i];
            isum += (int)sc[g] * gs;
        }
        sum += yd * ora_f16_to_f32(dh) * (float)isum;
    }
    return sum;
}

static void base_q6k_worker(void* p, int ith, int nth) {
    base_q4k_task_t* t = (base_q4k_task_t*)p;
    const int64_t mpt = (t->M + nth - 1) / nth;
    const int64_t m0 = (int64_t)ith * mpt < t->M ? (int64_t)ith * mpt : t->M;
    const int64_t m1 = m0 + mpt < t->M ? m0 + mpt : t->M;
    if (m0 >= m1) return;
    const size_t qrow = (size_t)(t->K / ORA_QK_K) * ORA_Q8K_BYTES;
    uint8_t* q8 = (uint8_t*)malloc(qrow * (size_t)t->N);
    for (int64_t n = 0; n < t->N; n++)
        ora_quantize_row_q8k((const float*)((const char*)t->X + n * t->x_col_bytes), t->K, q8 + n * qrow);
    for (int64_t m = m0; m < m1; m++) {
        const uint8_t* wr = t->W + m * t->w_row_bytes;
        for (int64_t n = 0; n < t->N; n++) t->Y[n * t->M + m] = base_vec_dot_q6k_q8k(t->K, wr, q8 + n * qrow);
    }
    free(q8);
}

void base_mul_mat_q6k(const uint8_t* W, size_t w_row_bytes, int64_t M, int64_t K,
                      const float* X, size_t x_col_bytes, int64_t N, float* Y, int nth) {
    base_q4k_task_t t = {W, w_row_bytes, M, K, X, x_col_bytes, N, Y};
    base_parallel(base_q6k_worker, &t, nth);
}

/* --- Flash-attention decode, F16 K/V ------------------------------------ */

typedef struct { const ora_fa_t* c; } base_fa_task_t;

#if defined(__x86_64__)
/* One work item of the AVX-512 FA2 skeleton with F16 K/V macros
 * (flash_attn_fa2_skeleton_avx512.inc:426-842, flash_attn_f16_avx512.asm:46-82):
 * KV tiles of 64, per-key f16->f32 dot with the f32 query, tile max, online
 * rescale of O and the running sum, fused exp + PV accumulate, final 1/sum. */
__attribute__((target("avx512f,avx512bw,fma")))
static void base_fa_item_avx512(const ora_fa_t* c, int64_t ib, int64_t ihq, int64_t iq) {
    enum { TILE = 64 };
    const int64_t DK = c->head_dim_k, DV = c->head_dim_v;
    const int64_t ihkv = ihq * c->n_head_kv / c->n_head_q;
    const int64_t L = c->kv_len ? c->kv_len[ib] : c->n_kv;
    const float* qr = (const float*)((const char*)c->q + iq * c->q_nb[1] + ihq * c->q_nb[2] + ib * c->q_nb[3]);
    const char* kb = (const char*)c->k + ihkv * c->k_nb[2] + ib * c->k_nb[3];
    const char* vb = (const char*)c->v + ihkv * c->v_nb[2] + ib * c->v_nb[3];
    float* dr = (float*)((char*)c->dst + iq * c->dst_nb[1] + ihq * c->dst_nb[2] + ib * c->dst_nb[3]);
    float O[256] __attribute__((aligned(64)));
    float sc[TILE];
    for (int64_t d = 0; d < DV; d++) O[d] = 0.0f;
    float mx = -INFINITY, sum = 0.0f;
    for (int64_t t0 = 0; t0 < L; t0 += TILE) {
        const int64_t t1 = t0 + TILE < L ? t0 + TILE : L;
        float tmax = -INFINITY;
        for (int64_t j = t0; j < t1; j++) {
            const uint16_t* kr = (const uint16_t*)(kb + j * c->k_nb[1]);
            __m512 acc = _mm512_setzero_ps();
            for (int64_t d = 0; d < DK; d += 16) {
                const __m512 kf = _mm512_cvtph_ps(_mm256_loadu_si256((const __m256i*)(kr + d)));
                acc = _mm512_fmadd_ps(kf, _mm512_loadu_ps(qr + d), acc);
            }
            float s = _mm512_reduce_add_ps(acc) * c->scale;
            if (c->mask) s += *(const float*)((const char*)c->mask + iq * c->mask_nb[1] + j * c->mask_nb[0]);
            sc[j - t0] = s;
            if (s > tmax) tmax = s;
        }
        const float nmx = mx > tmax ? mx : tmax;
        const float corr = expf(mx - nmx);
        sum *= corr;
        mx = nmx;
        const __m512 cv = _mm512_set1_ps(corr);
        for (int64_t d = 0; d < DV; d += 16) _mm512_store_ps(O + d, _mm512_mul_ps(cv, _mm512_load_ps(O + d)));
        for (int64_t j = t0; j < t1; j++) {
            const float p = expf(sc[j - t0] - mx);
            sum += p;
            const __m512 pv = _mm512_set1_ps(p);
            const uint16_t* vr = (const uint16_t*)(vb + j * c->v_nb[1]);
            for (int64_t d = 0; d < DV; d += 16) {
                const __m512 vf = _mm512_cvtph_ps(_mm256_loadu_si256((const __m256i*)(vr + d)));
                _mm512_store_ps(O + d, _mm512_fmadd_ps(pv, vf, _mm512_load_ps(O + d)));
            }
        }
    }
    const float inv = sum != 0.0f ? 1.0f / sum : 0.0f;
    for (int64_t d = 0; d < DV; d++) dr[d] = sum != 0.0f ? O[d] * inv : 0.0f;
}
#endif

#if defined(__x86_64__)
/* The same FA2 loop for quantised K/V (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL): each key /
 * value row is first dequantised to f32 (the DEQUANT_K_DOT_BLOCK / DEQUANT_V_ACCUM_BLOCK
 * steps of kernels/x86/flash/flash_attn_<type>_avx512.asm), then dotted / accumulated. */
__attribute__((target("avx512f,avx512bw,fma")))
static void base_fa_item_q_avx512(const ora_fa_t* c, int64_t ib, int64_t ihq, int64_t iq) {
    enum { TILE = 64 };
    const int64_t DK = c->head_dim_k, DV = c->head_dim_v;
    const int64_t ihkv = ihq * c->n_head_kv / c->n_head_q;
    const int64_t L = c->kv_len ? c->kv_len[ib] : c->n_kv;
    const float* qr = (const float*)((const char*)c->q + iq * c->q_nb[1] + ihq * c->q_nb[2] + ib * c->q_nb[3]);
    const char* kb = (const char*)c->k + ihkv * c->k_nb[2] + ib * c->k_nb[3];
    const char* vb = (const char*)c->v + ihkv * c->v_nb[2] + ib * c->v_nb[3];
    float* dr = (float*)((char*)c->dst + iq * c->dst_nb[1] + ihq * c->dst_nb[2] + ib * c->dst_nb[3]);
    float O[256] __attribute__((aligned(64)));
    float row[256] __attribute__((aligned(64)));
    float sc[TILE];
    for (int64_t d = 0; d < DV; d++) O[d] = 0.0f;
    float mx = -INFINITY, sum = 0.0f;
    for (int64_t t0 = 0; t0 < L; t0 += TILE) {
        const int64_t t1 = t0 + TILE < L ? t0 + TILE : L;
        float tmax = -INFINITY;
        for (int64_t j = t0; j < t1; j++) {
            ora_kv_row(kb + j * c->k_nb[1], DK, c->kv_type, row);
            __m512 acc = _mm512_setzero_ps();
            for (int64_t d = 0; d < DK; d += 16) acc = _mm512_fmadd_ps(_mm512_load_ps(row + d), _mm512_loadu_ps(qr + d), acc);
            float s = _mm512_reduce_add_ps(acc) * c->scale;
            if (c->mask) s += *(const float*)((const char*)c->mask + iq * c->mask_nb[1] + j * c->mask_nb[0]);
            sc[j - t0] = s;
            if (s > tmax) tmax = s;
        }
        const float nmx = mx > tmax ? mx : tmax;
        const float corr = expf(mx - nmx);
        sum *= corr;
        mx = nmx;
        const __m512 cv = _mm512_set1_ps(corr);
        for (int64_t d = 0; d < DV; d += 16) _mm512_store_ps(O + d, _mm512_mul_ps(cv, _mm512_load_ps(O + d)));
        for (int64_t j = t0; j < t1; j++) {
            const float p = expf(sc[j - t0] - mx);
            sum += p;
            ora_kv_row(vb + j * c->v_nb[1], DV, c->kv_type, row);
            const __m512 pv = _mm512_set1_ps(p);
            for (int64_t d = 0; d < DV; d += 16)
                _mm512_store_ps(O + d, _mm512_fmadd_ps(pv, _mm512_load_ps(row + d), _mm512_load_ps(O + d)));
        }
    }
    const float inv = sum != 0.0f ? 1.0f / sum : 0.0f;
    for (int64_t d = 0; d < DV; d++) dr[d] = sum != 0.0f ? O[d] * inv : 0.0f;
}
#endif

static void base_fa_worker(void* p, int ith, int nth) {
    const ora_fa_t* c = ((base_fa_task_t*)p)->c;
    const int64_t nqh = c->n_queries * c->n_head_q;
    const int64_t total = nqh * c->batch_size;
    /* work split of the skeleton (:394-422): [total*ith/nth, total*(ith+1)/nth) */
    const int64_t w0 = total * ith / nth, w1 = total * (ith + 1) / nth;
    for (int64_t w = w0; w < w1; w++) {
        const int64_t ib = w / nqh, rem = w % nqh;
        const int64_t ihq = rem / c->n_queries, iq = rem % c->n_queries;
#if defined(__x86_64__)
        if (base_has_avx512() && c->head_dim_k % 16 == 0 && c->head_dim_v % 16 == 0 && c->head_dim_v <= 256) {
            if (c->kv_type == 1) base_fa_item_avx512(c, ib, ihq, iq);
            else base_fa_item_q_avx512(c, ib, ihq, iq);
            continue;
        }
#endif
        /* portable fallback: reuse the exact checker on a one-item view */
        ora_fa_t one = *c;
        one.batch_size = 1; one.n_head_q = 1; one.n_queries = 1;
        one.n_head_kv = 1;
        const int64_t ihkv = ihq * c->n_head_kv / c->n_head_q;
        one.q = (const float*)((const char*)c->q + iq * c->q_nb[1] + ihq * c->q_nb[2] + ib * c->q_nb[3]);
        one.k = (const uint16_t*)((const char*)c->k + ihkv * c->k_nb[2] + ib * c->k_nb[3]);
        one.v = (const uint16_t*)((const char*)c->v + ihkv * c->v_nb[2] + ib * c->v_nb[3]);
        one.dst = (float*)((char*)c->dst + iq * c->dst_nb[1] + ihq * c->dst_nb[2] + ib * c->dst_nb[3]);
        one.kv_len = c->kv_len ? c->kv_len + ib : NULL;
        one.mask = c->mask ? (const float*)((const char*)c->mask + iq * c->mask_nb[1]) : NULL;
        one.mode = 0;
        ora_flash_attn(&one);
    }
}

void base_flash_attn(const ora_fa_t* c, int nth) {
    base_fa_task_t t = {c};
    base_parallel(base_fa_worker, &t, nth);
}
