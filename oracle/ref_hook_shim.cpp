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

// The reference's hook itself, ggml_simd_try_mul_mat (ggml_simd_hook.cpp:153-315), on one
// MUL_MAT node -- weights W (M rows of K values of type w_type, row stride w_row_bytes),
// activations X (N columns of K floats), dst Y (N columns of M floats) -- called once per
// thread index 0..nth-1 in turn, as ggml's threadpool would.  Returns the AND of the
// threads' answers (1 handled, 0 fall back).
int mlzref_try_mul_mat(int w_type, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                       int64_t N, float* y, int nth) {
    ggml_tensor s0{}, s1{}, d{};
    s0.type = (ggml_type)w_type;
    s0.ne[0] = K; s0.ne[1] = M; s0.ne[2] = s0.ne[3] = 1;
    s0.nb[0] = w_type == GGML_TYPE_F32 ? 4 : 2; s0.nb[1] = w_row_bytes; s0.nb[2] = s0.nb[3] = w_row_bytes * (size_t)M;
    s0.data = const_cast<void*>(w);
    s1.type = GGML_TYPE_F32;
    s1.ne[0] = K; s1.ne[1] = N; s1.ne[2] = s1.ne[3] = 1;
    s1.nb[0] = 4; s1.nb[1] = 4 * (size_t)K; s1.nb[2] = s1.nb[3] = 4 * (size_t)K * (size_t)N;
    s1.data = const_cast<float*>(x);
    d.type = GGML_TYPE_F32;
    d.ne[0] = M; d.ne[1] = N; d.ne[2] = d.ne[3] = 1;
    d.nb[0] = 4; d.nb[1] = 4 * (size_t)M; d.nb[2] = d.nb[3] = 4 * (size_t)M * (size_t)N;
    d.src[0] = &s0;
    d.src[1] = &s1;
    d.data = y;
    int all = 1;
    for (int ith = 0; ith < nth; ++ith) {
        ggml_compute_params p{ith, nth};
        all &= ggml_simd_try_mul_mat(&p, &d);
    }
    return all;
}

}  // extern "C"
