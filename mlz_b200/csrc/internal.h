// internal.h -- shared declarations of the mlzc library (host and device side).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/mlzc.h"

namespace mlzc {

// Records `status` and a printf-style message as the calling thread's last error and
// returns `status`, so call sites read `return fail(MLZC_ERR_INVALID, "...")`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Maps a CUDA error to MLZC_ERR_CUDA with the failing call's name.
int cuda_fail(cudaError_t e, const char* what);

#define MLZC_CUDA_TRY(call)                                  \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return ::mlzc::cuda_fail(e_, #call); \
    } while (0)

// Per-device state, created on first use of the device.
struct DeviceCtx {
    int device = -1;
    int sm_count = 0;
    unsigned int* err = nullptr;      // kernel error word (MLZC_DEVERR_* bits)
    cudaStream_t stream = nullptr;    // stream of the host-pointer entry points (compute)
    cudaStream_t h2d = nullptr;       // host -> device copies of the host-pointer calls
    cudaStream_t d2h = nullptr;       // device -> host copies of the host-pointer calls
    static constexpr int kEvents = 8;
    cudaEvent_t ev[kEvents] = {};     // chunk hand-offs between the three streams
};

// Context of `device` (creating it if needed); nullptr + last error on failure.
DeviceCtx* device_ctx(int device);
// Context of the calling thread's current device.
DeviceCtx* current_ctx();

// The driver's cuTensorMapEncodeTiled (looked up once), or nullptr if the driver lacks it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Counts one kernel launch (read by mlzc_launch_count).
void count_launch(int n = 1);

// Process-wide launch-overlap mode (MLZC_OVERLAP_*), set by mlzc_set_launch_overlap.
int overlap_mode();
// True when weight loads may be issued before pdl_wait() (MLZC_OVERLAP_WEIGHTS).
inline bool weights_before_wait() { return overlap_mode() == MLZC_OVERLAP_WEIGHTS; }

// Bounded-wait budget for every spin loop in the kernels (mbarrier polls).
constexpr long long kSpinLimit = 1ll << 26;

// ---- launchers (asynchronous; return MLZC_OK or a status with the message set) ----

// CUDA-core GEMV/skinny GEMM for F16 or F32 weights, any N (column chunks).
int launch_gemv(const DeviceCtx* c, int w_type, const void* w, size_t w_row_bytes,
                int64_t M, int64_t K, const float* x, size_t x_col_bytes, int64_t N,
                float* y, size_t y_col_bytes, cudaStream_t s);

// Skinny F16 mul_mat (2 <= N <= 16) on the tensor cores (mma.sync).
bool gemv_f16_mma_applicable(int64_t M, int64_t K, int64_t N, const void* w, size_t w_row_bytes,
                             const float* x, size_t x_col_bytes);
int launch_gemv_f16_mma(const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                        size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, cudaStream_t s);

// Q4_K dequant-dot on the tensor cores (mma.sync), any N: an activation prep launch (f16
// fragments + sub-block sums into the workspace) and the main kernel.
size_t q4k_workspace_bytes(int64_t K, int64_t N);
int launch_q4k_mma(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                   const float* x, size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes,
                   void* ws, size_t ws_bytes, cudaStream_t s);
// Decode-shaped Q4_K, N <= 2 (N <= 4 with many short rows): persistent kernel fed by a TMA
// ring, activations converted once per CTA into shared memory.
// The tcgen05 GEMM of a row-sharded call that also stores every finished tile into this
// rank's slice of each other rank's exchange slot (both parities given; the kernel picks
// the call's by the device epoch).  MLZC_ERR_UNSUPPORTED when Y or the layout does not fit.
struct GemmPeers {
    int npeer;
    float* slot[2][7];
    size_t pcs;                 // column stride of the slices (bytes)
    const uint32_t* epoch;      // this rank's completed-epoch counter
};
int launch_gemm_f16_peers(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                          size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                          const GemmPeers& peers, cudaStream_t s);
// F16 mul_mat dispatch helpers shared with the sharded path.
bool mul_mat_uses_gemm(int w_type, int64_t M, int64_t K, int64_t N, const void* w, size_t w_rs, const float* x,
                       size_t x_cs, const float* y, size_t y_cs);

// Q4_K, 1 <= N <= 4: int8 tensor-core path (activations quantised to int8 hi + lo per
// block by a prep launch), stream-K over 16-row x 8-block units.
bool q4k_i8_applicable(int64_t M, int64_t K, int64_t N);
size_t q4k_i8_workspace_bytes(int64_t K, int64_t N);
int launch_q4k_i8(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                  size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                  cudaStream_t s);
// Q6_K, 1 <= N <= 4, K a multiple of 1024: the same int8 path (q6k_i8.cu).
bool q6k_i8_applicable(int64_t M, int64_t K, int64_t N);
size_t q6k_i8_workspace_bytes(int64_t K, int64_t N);
int launch_q6k_i8(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                  size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws, size_t ws_bytes,
                  cudaStream_t s);
// Q4_K / Q6_K with at least kQuantGemmMinN columns and 4 M weights: the rows dequantised to
// f16 in the workspace (read once), then the tcgen05 F16 GEMM (dequant.cu).
constexpr int64_t kQuantGemmMinN = 64;
bool quant_gemm_applicable(int w_type, int64_t M, int64_t K, int64_t N);
size_t quant_gemm_workspace_bytes(int64_t M, int64_t K, int64_t N);
int launch_quant_gemm(const DeviceCtx* c, int w_type, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                      const float* x, size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws,
                      size_t ws_bytes, cudaStream_t s);
// The same ring for 5 <= N <= 8 (where it wins), fed by activations prepared once per call
// (q4k_prep_kernel's xf / xs) that travel with each stage.
bool q4k_ring_xs_applicable(int64_t M, int64_t K, int64_t N);
int launch_q4k_ring_xs(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                       const uint4* xf, const uint2* xs, int64_t N, float* y, size_t y_col_bytes,
                       cudaStream_t s);

// tcgen05/TMEM GEMM for F16 weights (activations narrowed to f16 in the workspace).
size_t gemm_f16_workspace_bytes(int64_t M, int64_t K, int64_t N);
bool gemm_f16_applicable(int64_t M, int64_t K, int64_t N, const void* w, size_t w_row_bytes,
                         const float* x, size_t x_col_bytes, const float* y, size_t y_col_bytes);
int launch_gemm_f16(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M,
                    int64_t K, const float* x, size_t x_col_bytes, int64_t N, float* y,
                    size_t y_col_bytes, void* ws, size_t ws_bytes, cudaStream_t s);
// The same with Y row m multiplied by row_scale[m] (the quantised-weight path, dequant.cu).
int launch_gemm_f16_row_scaled(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                               const float* x, size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, void* ws,
                               size_t ws_bytes, const float* row_scale, cudaStream_t s);

// Flash-attention decode (persistent stream-K over key tiles + combine).  The workspace
// size depends on the current device (its resident CTA count).
int fa_workspace_bytes(const mlzc_fa_desc* d, size_t* out);
// Quantised KV cache (Q8_0 / Q4_0 K and V): split-K CUDA-core decode + combine (fa_quant.cu).
int faq_workspace_bytes(const mlzc_fa_desc* d, int sm_count, size_t* out);
int launch_flash_attn_quant(int sm_count, const mlzc_fa_desc* d, void* ws, size_t ws_bytes, cudaStream_t s);
// Bytes of one K or V row of head_dim values of ggml type `type` (F16, Q8_0, Q4_0).
// Bytes of one 32-value block of a quantised KV-cache type (GGUF layouts), 0 for other types.
inline size_t kv_block_bytes(int32_t type) {
    switch (type) {
        case MLZC_TYPE_Q8_0: return 34;
        case MLZC_TYPE_Q4_0: return 18;
        case MLZC_TYPE_Q4_1: return 20;
        case MLZC_TYPE_Q5_0: return 22;
        case MLZC_TYPE_Q5_1: return 24;
        case MLZC_TYPE_IQ4_NL: return 18;
        default: return 0;
    }
}
inline size_t fa_row_bytes(int32_t type, int64_t head_dim) {
    const size_t bb = kv_block_bytes(type);
    if (bb) return (size_t)(head_dim / 32) * bb;
    return (size_t)head_dim * (type == MLZC_TYPE_F32 ? 4 : 2);
}
int launch_flash_attn(const DeviceCtx* c, const mlzc_fa_desc* d, void* ws, size_t ws_bytes,
                      cudaStream_t s);

// Reads and clears the error word used by flash-attention calls made without a library
// context (the allocation-free entry point) on the current device.
int fa_take_static_errors(unsigned int* out);

// Dispatch of one validated mul_mat to the kernel that fits its shape (GEMV, Q4_K,
// tensor-core GEMM); asynchronous on `s`.
int mul_mat_run(DeviceCtx* c, int w_type, const void* w, size_t w_rs, int64_t M, int64_t K,
                const float* x, size_t x_cs, int64_t N, float* y, size_t y_cs, void* ws,
                size_t ws_bytes, cudaStream_t s);
size_t mul_mat_workspace(int w_type, int64_t M, int64_t K, int64_t N);

// dst[n][r*m_loc + m] = src[r][n][m] for r < G: reorders all-gathered row slices into the
// ggml [N][M] layout.
int launch_gather_permute(const float* src, float* dst, size_t dst_col_bytes, int G, int64_t N,
                          int64_t m_loc, cudaStream_t s);

// Q4_K / Q6_K: 256-weight super-blocks of 144 / 210 bytes.
inline bool is_kquant(int w_type) { return w_type == MLZC_TYPE_Q4_K || w_type == MLZC_TYPE_Q6_K; }
// Bytes of one dense row of K weights of type w_type.
inline size_t dense_row_bytes(int w_type, int64_t K) {
    if (w_type == MLZC_TYPE_Q4_K) return (size_t)(K / 256) * 144;
    if (w_type == MLZC_TYPE_Q6_K) return (size_t)(K / 256) * 210;
    return (size_t)K * (w_type == MLZC_TYPE_F16 ? 2 : 4);
}

// Q6_K dequant-dot on the tensor cores (mma.sync), any N; no workspace.
int launch_q6k(const DeviceCtx* c, const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
               size_t x_col_bytes, int64_t N, float* y, size_t y_col_bytes, cudaStream_t s);

// Shape / type gate shared by the device entry point and the hook.
int check_mul_mat_args(int w_type, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                       const float* x, size_t x_col_bytes, int64_t N, const float* y,
                       size_t y_col_bytes);
int check_fa_args(const mlzc_fa_desc* d);

}  // namespace mlzc
