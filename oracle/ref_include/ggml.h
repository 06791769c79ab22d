// Minimal declarations for compiling the reference's src/simd/ggml_simd_hook.cpp in
// place (oracle/_ref, test infrastructure only).  The upstream ggml headers the hook
// includes are not part of the reference tree; the hook only needs the type ids, the
// tensor fields it reads and the compute parameters (ith, nth), declared here with
// ggml's ids and field names.
#pragma once
#include <cstddef>
#include <cstdint>

enum ggml_type {
    GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6, GGML_TYPE_Q5_1 = 7, GGML_TYPE_Q8_0 = 8, GGML_TYPE_Q8_1 = 9,
    GGML_TYPE_Q2_K = 10, GGML_TYPE_Q3_K = 11, GGML_TYPE_Q4_K = 12, GGML_TYPE_Q5_K = 13,
    GGML_TYPE_Q6_K = 14, GGML_TYPE_Q8_K = 15
};

#define GGML_MAX_SRC 10
#define GGML_MAX_OP_PARAMS 64

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)];
    struct ggml_tensor* src[GGML_MAX_SRC];
    void* data;
};
