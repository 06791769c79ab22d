// ref_shim.cpp -- link shim that lets the reference's own C++ sources
// (src/simd/flash_attention.cpp, src/simd/simd_matmul.cpp) build as a stand-alone
// shared library in oracle/_ref.  TEST INFRASTRUCTURE ONLY.
//
// The reference's x86 kernels are NASM sources and nasm is not installed, so the
// assembly entry points those two files reference are provided here as inert stubs
// that only count how often they were reached.  The tests call exclusively
// reference code paths that never reach them (flash_attn_quantized, and
// simd_matmul_f32 below its M*N*K < 512 scalar threshold,
// src/simd/simd_matmul.cpp:217-223) and assert that the counter stays 0.
//
// The two callbacks below adapt flash_attn_quantized (src/simd/flash_attention.cpp
// :291-410, whose K dot product is a ggml_vec_dot_t) to F16 keys and an f32 query:
// "from_float" copies the query unchanged and "vec_dot" is an f16 x f32 dot, so the
// reference loop computes exactly the F16-KV attention of its F16 assembly kernel
// (flash_attn_f16_avx512.asm:46-82: f16 K widened to f32, f32 Q); an f32 x f32 "vec_dot"
// does the same for F32 K/V (its F32 value branch).
#include <cstddef>
#include <cstdint>
#include <cstring>

#include "flash_attention.h"
#include "simd_matmul.h"

extern "C" {

int mlzref_stub_hits = 0;

#define MLZREF_STUB_MM(name)                                                   \
    void name(const float*, const float*, float*, size_t, size_t, size_t) {   \
        mlzref_stub_hits++;                                                    \
    }
MLZREF_STUB_MM(matrix_mult_avx2)
MLZREF_STUB_MM(matrix_mult_avx512)

#define MLZREF_STUB_FA(name) \
    void name(const flash_attn_config_t*) { mlzref_stub_hits++; }
#define MLZREF_STUB_FA2(t) MLZREF_STUB_FA(simd_flash_attn_##t##_avx2) MLZREF_STUB_FA(simd_flash_attn_##t##_avx512)
MLZREF_STUB_FA2(f32)
MLZREF_STUB_FA2(f16)
MLZREF_STUB_FA2(q4_0)
MLZREF_STUB_FA2(q4_1)
MLZREF_STUB_FA2(q5_0)
MLZREF_STUB_FA2(q5_1)
MLZREF_STUB_FA2(q8_0)
MLZREF_STUB_FA2(iq4_nl)
MLZREF_STUB_FA2(q2_k)
MLZREF_STUB_FA2(q3_k)
MLZREF_STUB_FA2(q4_k)
MLZREF_STUB_FA2(q5_k)
MLZREF_STUB_FA2(q6_k)
MLZREF_STUB_FA2(q8_k)

static float mlzref_h2f(uint16_t h) {
    // IEEE binary16 -> binary32 widening (exact).
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

static void mlzref_from_float_copy(const float* src, void* dst, int64_t k) {
    std::memcpy(dst, src, sizeof(float) * (size_t)k);
}

static void mlzref_vec_dot_f16_f32(int n, float* s, size_t, const void* vx, size_t,
                                   const void* vy, size_t, int) {
    const uint16_t* k = (const uint16_t*)vx;
    const float* q = (const float*)vy;
    float acc = 0.0f;
    for (int i = 0; i < n; i++) acc += mlzref_h2f(k[i]) * q[i];
    *s = acc;
}

// Run the reference's flash_attn_quantized on F16 K/V with an f32 query.
void mlzref_flash_attn_f16(const flash_attn_config_t* cfg) {
    flash_attn_quantized(cfg, mlzref_vec_dot_f16_f32, mlzref_from_float_copy,
                         sizeof(float) * (size_t)cfg->head_dim_k);
}

// The f32 x f32 dot of ggml's F32 vec_dot (k ascending, one float accumulator).
static void mlzref_vec_dot_f32_f32(int n, float* s, size_t, const void* vx, size_t,
                                   const void* vy, size_t, int) {
    const float* k = (const float*)vx;
    const float* q = (const float*)vy;
    float acc = 0.0f;
    for (int i = 0; i < n; i++) acc += k[i] * q[i];
    *s = acc;
}

// Run the reference's flash_attn_quantized on F32 K/V (its F32 value branch,
// flash_attention.cpp:391-393) with an f32 query.
void mlzref_flash_attn_f32(const flash_attn_config_t* cfg) {
    flash_attn_quantized(cfg, mlzref_vec_dot_f32_f32, mlzref_from_float_copy,
                         sizeof(float) * (size_t)cfg->head_dim_k);
}

size_t mlzref_config_size(void) { return sizeof(flash_attn_config_t); }

}  // extern "C"
