// ref_hook_shim.cpp -- compiles the reference's src/simd/ggml_simd_hook.cpp in place
// (included from the reference tree, nothing copied) against the minimal ggml declarations
// of oracle/ref_include, so that its file-local quantize_row_q8_k_reference
// (ggml_simd_hook.cpp:109-148) can produce golden Q8_K blocks.  TEST INFRASTRUCTURE ONLY.
// The hook's assembly dot products (NASM, not buildable here) are inert stubs counted in
// mlzref_stub_hits; the wrapper below never reaches them.
#include "ggml_simd_hook.cpp"

extern "C" {

extern int mlzref_stub_hits;

#define MLZREF_STUB_DOT(name) \
    void name(int, float*, const void*, const void*) { mlzref_stub_hits++; }
#define MLZREF_STUB_DOT2(t) MLZREF_STUB_DOT(simd_vec_dot_##t##_avx2) MLZREF_STUB_DOT(simd_vec_dot_##t##_avx512)
MLZREF_STUB_DOT2(q4_0_q8_0)
MLZREF_STUB_DOT2(q8_0_q8_0)
MLZREF_STUB_DOT2(q2_k_q8_k)
MLZREF_STUB_DOT2(q3_k_q8_k)
MLZREF_STUB_DOT2(q4_k_q8_k)
MLZREF_STUB_DOT2(q6_k_q8_k)
MLZREF_STUB_DOT2(q8_k_q8_k)

// The reference's F32 -> Q8_K quantiser on one row of k values (k a multiple of 256).
void mlzref_quantize_row_q8k(const float* x, void* y, int k) { quantize_row_q8_k_reference(x, y, k); }

}  // extern "C"
