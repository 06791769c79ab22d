// runtime.cpp -- host side of the mlzc C ABI: errors, device contexts, argument gates,
// kernel dispatch, and the ggml-hook-level entry points with host buffers.
//
// The hook entry points mirror the reference's dispatch layer:
//   ggml_simd_try_mul_mat  (src/simd/ggml_simd_hook.cpp:153-315)  -> mlzc_try_mul_mat
//   ggml_simd_try_flash_attn (src/simd/ggml_simd_hook.cpp:317-375) -> mlzc_try_flash_attn
// Same return contract (1 = handled, 0 = let the CPU path run), same caller (every ggml
// threadpool thread of the node).  Where the reference splits M rows over the threads
// (:177-185), the GPU version lets thread 0 issue the whole node and hands its answer to
// the other threads, so that a fallback is always taken by all threads together.
#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace mlzc {

namespace {
thread_local std::string g_last_error;
thread_local int g_last_status = MLZC_OK;   // status of the calling thread's last fail()

std::mutex g_ctx_mu;
std::vector<std::unique_ptr<DeviceCtx>> g_ctx;   // indexed by device id
int g_hook_device = 0;                           // device of the hook-level entry points
}  // namespace

namespace {
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_overlap{MLZC_OVERLAP_SAFE};
}  // namespace

void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int overlap_mode() { return g_overlap.load(std::memory_order_relaxed); }

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    g_last_status = status;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? MLZC_ERR_NOMEM : MLZC_ERR_CUDA, "%s: %s (%s)", what,
                cudaGetErrorString(e), cudaGetErrorName(e));
}

DeviceCtx* device_ctx(int device) {
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess) { cuda_fail(e, "cudaGetDeviceCount"); return nullptr; }
    if (device < 0 || device >= ndev) { fail(MLZC_ERR_INVALID, "device %d out of range (%d devices)", device, ndev); return nullptr; }
    if ((int)g_ctx.size() < ndev) g_ctx.resize(ndev);
    if (g_ctx[device]) return g_ctx[device].get();
    int prev = 0;
    cudaGetDevice(&prev);
    auto c = std::make_unique<DeviceCtx>();
    c->device = device;
    bool ok = cudaSetDevice(device) == cudaSuccess;
    ok = ok && cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device) == cudaSuccess;
    ok = ok && cudaMalloc(&c->err, sizeof(unsigned int)) == cudaSuccess;
    ok = ok && cudaMemset(c->err, 0, sizeof(unsigned int)) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&c->h2d, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&c->d2h, cudaStreamNonBlocking) == cudaSuccess;
    for (int i = 0; ok && i < DeviceCtx::kEvents; ++i)
        ok = cudaEventCreateWithFlags(&c->ev[i], cudaEventDisableTiming) == cudaSuccess;
    cudaSetDevice(prev);
    if (!ok) { fail(MLZC_ERR_CUDA, "creating the context of device %d failed: %s", device, cudaGetErrorString(cudaGetLastError())); return nullptr; }
    g_ctx[device] = std::move(c);
    return g_ctx[device].get();
}

DeviceCtx* current_ctx() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { cuda_fail(e, "cudaGetDevice"); return nullptr; }
    return device_ctx(dev);
}

int check_mul_mat_args(int w_type, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                       const float* x, size_t x_col_bytes, int64_t N, const float* y,
                       size_t y_col_bytes) {
    if (w_type != MLZC_TYPE_F16 && w_type != MLZC_TYPE_F32 && w_type != MLZC_TYPE_Q4_K && w_type != MLZC_TYPE_Q6_K)
        return fail(MLZC_ERR_UNSUPPORTED, "mul_mat: weight type %d not handled (F32=0, F16=1, Q4_K=12, Q6_K=14)",
                    w_type);
    if (M < 0 || K < 0 || N < 0) return fail(MLZC_ERR_INVALID, "mul_mat: negative dimension");
    if (M == 0 || N == 0) return MLZC_OK;
    if (K > 0 && (!w || !x)) return fail(MLZC_ERR_INVALID, "mul_mat: null W or X");
    if (!y) return fail(MLZC_ERR_INVALID, "mul_mat: null Y");
    // alignment the kernels need of W and its row stride: the element (f16 / f32), a
    // 4-byte word for the quantised blocks (Q6_K rows themselves are 2-byte multiples)
    const size_t esz = w_type == MLZC_TYPE_F16 ? 2 : 4;
    const size_t rs_align = w_type == MLZC_TYPE_Q6_K ? 2 : esz;
    const size_t min_row = dense_row_bytes(w_type, K);
    if (is_kquant(w_type) && K % 256 != 0)
        return fail(MLZC_ERR_INVALID, "mul_mat: Q4_K / Q6_K need K %% 256 == 0 (K=%lld)", (long long)K);
    if (w_row_bytes < min_row) return fail(MLZC_ERR_INVALID, "mul_mat: w_row_bytes %zu < row size %zu", w_row_bytes, min_row);
    if (x_col_bytes < (size_t)K * 4) return fail(MLZC_ERR_INVALID, "mul_mat: x_col_bytes %zu < 4*K", x_col_bytes);
    if (y_col_bytes < (size_t)M * 4 || y_col_bytes % 4) return fail(MLZC_ERR_INVALID, "mul_mat: y_col_bytes %zu must be >= 4*M and a multiple of 4", y_col_bytes);
    if ((uintptr_t)y % 4 || (uintptr_t)x % 4 || (uintptr_t)w % esz || x_col_bytes % 4 || w_row_bytes % rs_align)
        return fail(MLZC_ERR_INVALID, "mul_mat: pointers / strides not aligned to their element size");
    return MLZC_OK;
}

int check_fa_args(const mlzc_fa_desc* d) {
    if (!d) return fail(MLZC_ERR_INVALID, "flash_attn: null descriptor");
    // quantised caches and F32 go to the cp.async-ring kernel (rows of 4-byte-aligned pieces)
    const bool f32 = d->k_type == MLZC_TYPE_F32;
    const bool quant = kv_block_bytes(d->k_type) != 0 || f32;
    if ((d->k_type != MLZC_TYPE_F16 && !quant) || d->v_type != d->k_type)
        return fail(MLZC_ERR_UNSUPPORTED,
                    "flash_attn: K/V types %d/%d (both F16, F32, Q8_0, Q4_0, Q4_1, Q5_0, Q5_1 or IQ4_NL)", d->k_type,
                    d->v_type);
    if (d->head_dim_k != d->head_dim_v) return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: DK != DV");
    if (d->head_dim_k != 64 && d->head_dim_k != 128 && d->head_dim_k != 256)
        return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: head_dim %lld (64, 128, 256 supported)", (long long)d->head_dim_k);
    if (f32 && d->head_dim_k == 256)
        return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: F32 K/V with head_dim 256 (64, 128 supported)");
    if (d->n_queries <= 0 || d->n_kv < 0 || d->n_head_q <= 0 || d->n_head_kv <= 0 || d->batch_size <= 0)
        return fail(MLZC_ERR_INVALID, "flash_attn: empty or negative dimension");
    if (d->n_head_kv > d->n_head_q) return fail(MLZC_ERR_INVALID, "flash_attn: more KV heads than query heads");
    if (d->n_kv > (1 << 30) || d->batch_size > 65535 || d->n_queries * d->n_head_q > (1 << 20))
        return fail(MLZC_ERR_INVALID, "flash_attn: dimension too large");
    if (!d->q || !d->dst || (d->n_kv > 0 && (!d->k || !d->v))) return fail(MLZC_ERR_INVALID, "flash_attn: null tensor");
    if ((uintptr_t)d->q % 16 || d->q_nb[1] % 16 || d->q_nb[2] % 16 || d->q_nb[3] % 16 || d->q_nb[0] != 4)
        return fail(MLZC_ERR_INVALID, "flash_attn: q rows must be contiguous f32 on 16-byte boundaries");
    if (quant) {
        // rows of blocks (nb[0] = block bytes, ggml's convention), 4-byte aligned
        const size_t bb = f32 ? 4 : kv_block_bytes(d->k_type);   // nb[0]: block (or element) bytes
        if ((uintptr_t)d->k % 4 || (uintptr_t)d->v % 4 || d->k_nb[1] % 4 || d->v_nb[1] % 4 || d->k_nb[2] % 4 ||
            d->v_nb[2] % 4 || d->k_nb[3] % 4 || d->v_nb[3] % 4 || d->k_nb[0] != bb || d->v_nb[0] != bb)
            return fail(MLZC_ERR_INVALID, "flash_attn: quantised / F32 K/V rows must be contiguous on 4-byte boundaries");
    } else if ((uintptr_t)d->k % 16 || (uintptr_t)d->v % 16 || d->k_nb[1] % 16 || d->v_nb[1] % 16 ||
               d->k_nb[2] % 16 || d->v_nb[2] % 16 || d->k_nb[3] % 16 || d->v_nb[3] % 16 || d->k_nb[0] != 2 ||
               d->v_nb[0] != 2) {
        return fail(MLZC_ERR_INVALID, "flash_attn: K/V rows must be contiguous f16 on 16-byte boundaries");
    }
    if (d->dst_nb[0] != 4 || (uintptr_t)d->dst % 4) return fail(MLZC_ERR_INVALID, "flash_attn: dst rows must be contiguous f32");
    if (d->mask && (d->mask_nb[0] % 4 || (uintptr_t)d->mask % 4)) return fail(MLZC_ERR_INVALID, "flash_attn: mask must be f32-aligned");
    if ((d->mode & MLZC_FA_MODE_SOFTCAP) && d->logit_softcap == 0.0f)
        return fail(MLZC_ERR_INVALID, "flash_attn: SOFTCAP mode with softcap 0");
    return MLZC_OK;
}

namespace {

// Minimum activation columns for which the tensor-core GEMM beats the CUDA-core GEMV.
constexpr int64_t kGemmMinN = 8;

bool use_gemm(int w_type, int64_t M, int64_t K, int64_t N, const void* w, size_t w_rs,
              const float* x, size_t x_cs, const float* y, size_t y_cs) {
    return w_type == MLZC_TYPE_F16 && N >= kGemmMinN && gemm_f16_applicable(M, K, N, w, w_rs, x, x_cs, y, y_cs);
}

}  // namespace

bool mul_mat_uses_gemm(int w_type, int64_t M, int64_t K, int64_t N, const void* w, size_t w_rs, const float* x,
                       size_t x_cs, const float* y, size_t y_cs) {
    return w_type == MLZC_TYPE_F16 && !gemv_f16_mma_applicable(M, K, N, w, w_rs, x, x_cs) &&
           use_gemm(w_type, M, K, N, w, w_rs, x, x_cs, y, y_cs);
}

namespace {

int mul_mat_dispatch(DeviceCtx* c, int w_type, const void* w, size_t w_rs, int64_t M, int64_t K,
                     const float* x, size_t x_cs, int64_t N, float* y, size_t y_cs, void* ws,
                     size_t ws_bytes, cudaStream_t s) {
    if (M == 0 || N == 0) return MLZC_OK;
    if (K == 0) {
        // empty contraction: Y = 0
        if (y_cs == (size_t)M * 4) {
            MLZC_CUDA_TRY(cudaMemsetAsync(y, 0, (size_t)N * y_cs, s));
        } else {
            MLZC_CUDA_TRY(cudaMemset2DAsync(y, y_cs, 0, (size_t)M * 4, (size_t)N, s));
        }
        return MLZC_OK;
    }
    // prefill-sized batches of quantised weights: dequantise once, then the tcgen05 GEMM
    if (quant_gemm_applicable(w_type, M, K, N))
        return launch_quant_gemm(c, w_type, w, w_rs, M, K, x, x_cs, N, y, y_cs, ws, ws_bytes, s);
    if (w_type == MLZC_TYPE_Q4_K) return launch_q4k_mma(c, w, w_rs, M, K, x, x_cs, N, y, y_cs, ws, ws_bytes, s);
    if (w_type == MLZC_TYPE_Q6_K) {
        if ((uintptr_t)x % 16 || x_cs % 16)
            return fail(MLZC_ERR_INVALID, "mul_mat (Q6_K): activation columns must be 16-byte aligned");
        // decode shapes with 16-byte rows: the int8 path; the rest (and rows only 2-byte
        // aligned) the f16 tensor-core kernel
        if (q6k_i8_applicable(M, K, N) && (uintptr_t)w % 16 == 0 && w_rs % 16 == 0)
            return launch_q6k_i8(c, w, w_rs, M, K, x, x_cs, N, y, y_cs, ws, ws_bytes, s);
        return launch_q6k(c, w, w_rs, M, K, x, x_cs, N, y, y_cs, s);
    }
    if (w_type == MLZC_TYPE_F16 && gemv_f16_mma_applicable(M, K, N, w, w_rs, x, x_cs))
        return launch_gemv_f16_mma(w, w_rs, M, K, x, x_cs, N, y, y_cs, s);
    if (use_gemm(w_type, M, K, N, w, w_rs, x, x_cs, y, y_cs))
        return launch_gemm_f16(c, w, w_rs, M, K, x, x_cs, N, y, y_cs, ws, ws_bytes, s);
    return launch_gemv(c, w_type, w, w_rs, M, K, x, x_cs, N, y, y_cs, s);
}

size_t mul_mat_ws(int w_type, int64_t M, int64_t K, int64_t N) {
    if (quant_gemm_applicable(w_type, M, K, N)) return quant_gemm_workspace_bytes(M, K, N);
    if (w_type == MLZC_TYPE_Q4_K) return K % 256 == 0 ? q4k_workspace_bytes(K, N) : 0;
    if (w_type == MLZC_TYPE_Q6_K) return q6k_i8_applicable(M, K, N) ? q6k_i8_workspace_bytes(K, N) : 0;
    // N in [8, 16] normally takes the skinny tensor-core path (no workspace), but the
    // tcgen05 GEMM it falls back to for unaligned operands needs one
    if (w_type == MLZC_TYPE_F16 && N >= kGemmMinN) return gemm_f16_workspace_bytes(M, K, N);
    return 0;
}

}  // namespace

int mul_mat_run(DeviceCtx* c, int w_type, const void* w, size_t w_rs, int64_t M, int64_t K,
                const float* x, size_t x_cs, int64_t N, float* y, size_t y_cs, void* ws,
                size_t ws_bytes, cudaStream_t s) {
    return mul_mat_dispatch(c, w_type, w, w_rs, M, K, x, x_cs, N, y, y_cs, ws, ws_bytes, s);
}

size_t mul_mat_workspace(int w_type, int64_t M, int64_t K, int64_t N) { return mul_mat_ws(w_type, M, K, N); }

}  // namespace mlzc

using namespace mlzc;

// ============================================================ runtime entry points

extern "C" const char* mlzc_last_error(void) { return g_last_error.c_str(); }

extern "C" int mlzc_version(void) { return MLZC_VERSION; }

extern "C" int mlzc_launch_count(uint64_t* out_count) {
    if (!out_count) return fail(MLZC_ERR_INVALID, "null out_count");
    *out_count = g_launches.load(std::memory_order_relaxed);
    return MLZC_OK;
}

extern "C" int mlzc_set_launch_overlap(int mode) {
    if (mode != MLZC_OVERLAP_OFF && mode != MLZC_OVERLAP_SAFE && mode != MLZC_OVERLAP_WEIGHTS)
        return fail(MLZC_ERR_INVALID, "launch overlap mode %d (0, 1 or 2)", mode);
    g_overlap.store(mode, std::memory_order_relaxed);
    return MLZC_OK;
}

extern "C" int mlzc_get_launch_overlap(int* out_mode) {
    if (!out_mode) return fail(MLZC_ERR_INVALID, "null out_mode");
    *out_mode = overlap_mode();
    return MLZC_OK;
}

extern "C" int mlzc_init(int device) {
    g_last_status = MLZC_OK;
    DeviceCtx* c = device_ctx(device);
    if (!c) return g_last_status != MLZC_OK ? g_last_status : MLZC_ERR_CUDA;
    g_hook_device = device;
    return MLZC_OK;
}

extern "C" int mlzc_weight_cache_clear(void);

extern "C" int mlzc_shutdown(void) {
    mlzc_weight_cache_clear();
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    for (auto& c : g_ctx) {
        if (!c) continue;
        cudaSetDevice(c->device);
        if (c->stream) cudaStreamDestroy(c->stream);
        if (c->h2d) cudaStreamDestroy(c->h2d);
        if (c->d2h) cudaStreamDestroy(c->d2h);
        for (cudaEvent_t e : c->ev)
            if (e) cudaEventDestroy(e);
        if (c->err) cudaFree(c->err);
    }
    g_ctx.clear();
    cudaSetDevice(prev);
    return MLZC_OK;
}

extern "C" int mlzc_device_errors(int device, uint32_t* out_bits) {
    if (!out_bits) return fail(MLZC_ERR_INVALID, "null out_bits");
    // No context is created here: a process that only used the allocation-free entry
    // point has none, and reading its error word must not allocate either.
    DeviceCtx* c = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_ctx_mu);
        int ndev = 0;
        cudaError_t e = cudaGetDeviceCount(&ndev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
        if (device < 0 || device >= ndev) return fail(MLZC_ERR_INVALID, "device %d out of range (%d devices)", device, ndev);
        if (device < (int)g_ctx.size()) c = g_ctx[device].get();
    }
    int prev = 0;
    cudaGetDevice(&prev);
    MLZC_CUDA_TRY(cudaSetDevice(device));
    unsigned int v = 0, vs = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (c && e == cudaSuccess) e = cudaMemcpy(&v, c->err, sizeof v, cudaMemcpyDeviceToHost);
    if (c && e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof v);
    int st = e == cudaSuccess ? fa_take_static_errors(&vs) : MLZC_OK;
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "mlzc_device_errors");
    if (st != MLZC_OK) return st;
    *out_bits = v | vs;
    return MLZC_OK;
}

extern "C" int mlzc_mul_mat_workspace_bytes(int w_type, int64_t M, int64_t K, int64_t N, size_t* out_bytes) {
    if (!out_bytes) return fail(MLZC_ERR_INVALID, "null out_bytes");
    *out_bytes = mul_mat_ws(w_type, M, K, N);
    return MLZC_OK;
}

extern "C" int mlzc_mul_mat_dev(int w_type, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                                const float* x, size_t x_col_bytes, int64_t N, float* y,
                                size_t y_col_bytes, void* workspace, size_t workspace_bytes,
                                void* stream) {
    int st = check_mul_mat_args(w_type, w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes);
    if (st != MLZC_OK) return st;
    DeviceCtx* c = current_ctx();
    if (!c) return MLZC_ERR_CUDA;
    return mul_mat_dispatch(c, w_type, w, w_row_bytes, M, K, x, x_col_bytes, N, y, y_col_bytes, workspace,
                            workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int mlzc_flash_attn_workspace_bytes(const mlzc_fa_desc* desc, size_t* out_bytes) {
    if (!out_bytes) return fail(MLZC_ERR_INVALID, "null out_bytes");
    int st = check_fa_args(desc);
    if (st != MLZC_OK) return st;
    return fa_workspace_bytes(desc, out_bytes);
}

extern "C" int mlzc_flash_attn_dev(const mlzc_fa_desc* desc, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    int st = check_fa_args(desc);
    if (st != MLZC_OK) return st;
    DeviceCtx* c = current_ctx();
    if (!c) return MLZC_ERR_CUDA;
    return launch_flash_attn(c, desc, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

// ============================================================ host-pointer level

namespace {

struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    int ensure(size_t want) {
        if (want <= bytes) return MLZC_OK;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        size_t sz = want + want / 4 + 256;
        MLZC_CUDA_TRY(cudaMalloc(&ptr, sz));
        bytes = sz;
        return MLZC_OK;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

// Device-side arena of the synchronous host-pointer calls on one device.
struct HostArena {
    std::mutex mu;
    DeviceBuffer x, y, ws, q, k, v, mask, dst, kvlen;
};

std::mutex g_arena_mu;
std::map<int, std::unique_ptr<HostArena>> g_arena;

HostArena* arena(int device) {
    std::lock_guard<std::mutex> lk(g_arena_mu);
    auto& a = g_arena[device];
    if (!a) a = std::make_unique<HostArena>();
    return a.get();
}

// Makes `device` current for the lifetime of the object.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int device) {
        cudaGetDevice(&prev);
        ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Copies N columns of `row_bytes` bytes, `src_stride` apart, into a dense device buffer.
int h2d_cols(void* dst, const void* src, size_t row_bytes, size_t src_stride, int64_t n, cudaStream_t s) {
    if (src_stride == row_bytes) {
        MLZC_CUDA_TRY(cudaMemcpyAsync(dst, src, row_bytes * (size_t)n, cudaMemcpyHostToDevice, s));
    } else {
        MLZC_CUDA_TRY(cudaMemcpy2DAsync(dst, row_bytes, src, src_stride, row_bytes, (size_t)n, cudaMemcpyHostToDevice, s));
    }
    return MLZC_OK;
}

int d2h_cols(void* dst, size_t dst_stride, const void* src, size_t row_bytes, int64_t n, cudaStream_t s) {
    if (dst_stride == row_bytes) {
        MLZC_CUDA_TRY(cudaMemcpyAsync(dst, src, row_bytes * (size_t)n, cudaMemcpyDeviceToHost, s));
    } else {
        MLZC_CUDA_TRY(cudaMemcpy2DAsync(dst, dst_stride, src, row_bytes, row_bytes, (size_t)n, cudaMemcpyDeviceToHost, s));
    }
    return MLZC_OK;
}

}  // namespace

struct mlzc_weight_s {
    int device = 0;
    int type = 0;
    int64_t M = 0, K = 0;
    size_t row_bytes = 0;
    void* dev = nullptr;
};

extern "C" int mlzc_weight_upload(int device, int w_type, const void* host, size_t row_bytes, int64_t M,
                                  int64_t K, mlzc_weight* out) {
    if (!out) return fail(MLZC_ERR_INVALID, "null out");
    *out = nullptr;
    int st = check_mul_mat_args(w_type, host, row_bytes, M, K, reinterpret_cast<const float*>(16), (size_t)K * 4, 1,
                                reinterpret_cast<const float*>(16), (size_t)M * 4);
    if (st != MLZC_OK) return st;
    if (M * K > 0 && !host) return fail(MLZC_ERR_INVALID, "null host weights");
    DeviceCtx* c = device_ctx(device);
    if (!c) return MLZC_ERR_CUDA;
    DeviceGuard g(device);
    if (!g.ok) return fail(MLZC_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    const size_t dense = dense_row_bytes(w_type, K);
    // keep rows 16-byte aligned on the device so the vector paths apply
    const size_t dev_row = (dense + 15) / 16 * 16;
    auto w = std::make_unique<mlzc_weight_s>();
    w->device = device;
    w->type = w_type;
    w->M = M;
    w->K = K;
    w->row_bytes = dev_row;
    if (M > 0 && dev_row > 0) {
        MLZC_CUDA_TRY(cudaMalloc(&w->dev, dev_row * (size_t)M));
        cudaError_t e;
        if (dev_row == row_bytes)
            e = cudaMemcpy(w->dev, host, dev_row * (size_t)M, cudaMemcpyHostToDevice);
        else
            e = cudaMemcpy2D(w->dev, dev_row, host, row_bytes, dense, (size_t)M, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(w->dev);
            return cuda_fail(e, "weight upload");
        }
    }
    *out = w.release();
    return MLZC_OK;
}

extern "C" int mlzc_weight_free(mlzc_weight w) {
    if (!w) return MLZC_OK;
    if (w->dev) {
        DeviceGuard g(w->device);
        cudaFree(w->dev);
    }
    delete w;
    return MLZC_OK;
}

namespace {
constexpr int kPipeChunks = 4;          // column chunks of a wide host-pointer call
constexpr int64_t kPipeMinCols = 128;   // no chunk narrower than this
}  // namespace

extern "C" int mlzc_mul_mat(mlzc_weight w, const float* x, size_t x_col_bytes, int64_t N, float* y,
                            size_t y_col_bytes) {
    if (!w) return fail(MLZC_ERR_INVALID, "null weight handle");
    const int64_t M = w->M, K = w->K;
    if (N < 0) return fail(MLZC_ERR_INVALID, "negative N");
    if (N == 0 || M == 0) return MLZC_OK;
    if (!x || !y) return fail(MLZC_ERR_INVALID, "null X or Y");
    if (x_col_bytes < (size_t)K * 4 || y_col_bytes < (size_t)M * 4)
        return fail(MLZC_ERR_INVALID, "column strides smaller than a column");
    DeviceCtx* c = device_ctx(w->device);
    if (!c) return MLZC_ERR_CUDA;
    DeviceGuard g(w->device);
    if (!g.ok) return fail(MLZC_ERR_CUDA, "cudaSetDevice(%d) failed", w->device);
    HostArena* a = arena(w->device);
    std::lock_guard<std::mutex> lk(a->mu);
    const size_t xb = (size_t)K * 4, yb = (size_t)M * 4;
    int st;
    if ((st = a->x.ensure(xb * (size_t)N + 16)) != MLZC_OK) return st;
    if ((st = a->y.ensure(yb * (size_t)N + 16)) != MLZC_OK) return st;
    // Column chunks flow through three streams: copy in (h2d), compute (stream), copy out
    // (d2h).  Chunk i + 1 uploads while chunk i computes and chunk i - 1 downloads; PCIe
    // carries both directions at once.  Narrow calls (decode) are one chunk.
    const int64_t nc = N >= 2 * kPipeMinCols ? std::max<int64_t>(kPipeMinCols, (N + kPipeChunks - 1) / kPipeChunks) : N;
    const int nchunks = (int)((N + nc - 1) / nc);
    const size_t wsb = mul_mat_ws(w->type, M, K, nc);
    if ((st = a->ws.ensure(wsb)) != MLZC_OK) return st;
    char* xd = static_cast<char*>(a->x.ptr);
    char* yd = static_cast<char*>(a->y.ptr);
    const char* xh = reinterpret_cast<const char*>(x);
    char* yh = reinterpret_cast<char*>(y);
    for (int i = 0; i < nchunks; ++i) {
        const int64_t c0 = (int64_t)i * nc, n = std::min(nc, N - c0);
        cudaEvent_t up = c->ev[(2 * i) % DeviceCtx::kEvents], done = c->ev[(2 * i + 1) % DeviceCtx::kEvents];
        if ((st = h2d_cols(xd + c0 * xb, xh + c0 * x_col_bytes, xb, x_col_bytes, n, c->h2d)) != MLZC_OK) return st;
        MLZC_CUDA_TRY(cudaEventRecord(up, c->h2d));
        MLZC_CUDA_TRY(cudaStreamWaitEvent(c->stream, up, 0));
        // dense device columns: the column stride is K floats
        st = mul_mat_dispatch(c, w->type, w->dev, w->row_bytes, M, K, reinterpret_cast<const float*>(xd + c0 * xb), xb,
                              n, reinterpret_cast<float*>(yd + c0 * yb), yb, a->ws.ptr, a->ws.bytes, c->stream);
        if (st != MLZC_OK) return st;
        MLZC_CUDA_TRY(cudaEventRecord(done, c->stream));
        MLZC_CUDA_TRY(cudaStreamWaitEvent(c->d2h, done, 0));
        if ((st = d2h_cols(yh + c0 * y_col_bytes, y_col_bytes, yd + c0 * yb, yb, n, c->d2h)) != MLZC_OK) return st;
    }
    MLZC_CUDA_TRY(cudaStreamSynchronize(c->d2h));
    return MLZC_OK;
}

extern "C" int mlzc_host_register(void* ptr, size_t bytes) {
    if (!ptr || !bytes) return fail(MLZC_ERR_INVALID, "host_register: null or empty range");
    const cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterPortable);
    if (e == cudaErrorHostMemoryAlreadyRegistered) {
        cudaGetLastError();
        return MLZC_OK;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostRegister");
    return MLZC_OK;
}

extern "C" int mlzc_host_unregister(void* ptr) {
    if (!ptr) return fail(MLZC_ERR_INVALID, "host_unregister: null pointer");
    const cudaError_t e = cudaHostUnregister(ptr);
    if (e == cudaErrorHostMemoryNotRegistered) {
        cudaGetLastError();
        return MLZC_OK;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostUnregister");
    return MLZC_OK;
}

// ---------------------------------------------------------------- hook level

namespace {

// One in-flight ggml node shared by its nth threads.
struct NodeTicket {
    int result = 0;
    bool done = false;
    int consumed = 0;
};
std::mutex g_node_mu;
std::condition_variable g_node_cv;
std::unordered_map<const void*, NodeTicket> g_nodes;

// Thread 0 runs `work` (returning 1/0); every thread returns that value.  The ticket is
// dropped once all nth threads have read it, before ggml's post-node barrier releases
// any of them into the next evaluation of the same node.
template <class F>
int run_node(const void* key, int ith, int nth, F&& work) {
    if (nth <= 1) return work();
    std::unique_lock<std::mutex> lk(g_node_mu);
    if (ith == 0) {
        lk.unlock();
        const int r = work();
        lk.lock();
        NodeTicket& t = g_nodes[key];
        t.result = r;
        t.done = true;
        g_node_cv.notify_all();
    } else {
        g_node_cv.wait(lk, [&] {
            auto it = g_nodes.find(key);
            return it != g_nodes.end() && it->second.done;
        });
    }
    NodeTicket& t = g_nodes[key];
    const int r = t.result;
    if (++t.consumed == nth) g_nodes.erase(key);
    return r;
}

using WeightKey = std::tuple<const void*, int, int64_t, int64_t, size_t, int>;
struct CachedWeight {
    mlzc_weight w = nullptr;
    uint64_t fingerprint = 0;
};
std::mutex g_wcache_mu;
std::map<WeightKey, CachedWeight> g_wcache;

// FNV-1a over 64-byte samples at the start, middle and end of the host buffer.  ggml
// weights are immutable for a model's lifetime, so (pointer, type, shape) identifies
// them; the fingerprint catches a buffer reused for other data at the same address
// (e.g. after a model reload) without hashing the whole tensor on every call.
uint64_t fingerprint(const void* data, size_t bytes) {
    const unsigned char* p = static_cast<const unsigned char*>(data);
    uint64_t h = 1469598103934665603ull;
    const size_t win = bytes < 64 ? bytes : 64;
    const size_t offs[3] = {0, bytes / 2 - (bytes / 2 >= win / 2 ? win / 2 : 0), bytes - win};
    for (size_t o : offs)
        for (size_t i = 0; i < win; ++i) h = (h ^ p[o + i]) * 1099511628211ull;
    return h;
}

mlzc_weight cached_weight(const mlzc_tensor* src0, int device, int* status) {
    const WeightKey key{src0->data, src0->type, src0->ne[0], src0->ne[1], src0->nb[1], device};
    const size_t row = dense_row_bytes(src0->type, src0->ne[0]);
    const size_t bytes = src0->ne[1] > 0 ? (size_t)(src0->ne[1] - 1) * src0->nb[1] + row : 0;
    const uint64_t fp = bytes ? fingerprint(src0->data, bytes) : 0;
    std::lock_guard<std::mutex> lk(g_wcache_mu);
    auto it = g_wcache.find(key);
    if (it != g_wcache.end()) {
        if (it->second.fingerprint == fp) return it->second.w;
        mlzc_weight_free(it->second.w);
        g_wcache.erase(it);
    }
    mlzc_weight w = nullptr;
    *status = mlzc_weight_upload(device, src0->type, src0->data, src0->nb[1], src0->ne[1], src0->ne[0], &w);
    if (*status != MLZC_OK) return nullptr;
    g_wcache[key] = CachedWeight{w, fp};
    return w;
}

// The type / shape gate of ggml_simd_try_mul_mat (ggml_simd_hook.cpp:154-164), extended
// with the layout checks ggml_compute_forward_mul_mat asserts (ggml-cpu-simd.c:1273-1288).
// Deterministic in the tensor metadata, so all threads of a node agree.
bool mul_mat_gate(const mlzc_tensor* s0, const mlzc_tensor* s1, const mlzc_tensor* d) {
    if (!s0 || !s1 || !d || !s0->data || !s1->data || !d->data) return false;
    if (d->type != MLZC_TYPE_F32 || s1->type != MLZC_TYPE_F32) return false;
    if (s0->type != MLZC_TYPE_F32 && s0->type != MLZC_TYPE_F16 && !is_kquant(s0->type)) return false;
    if (s1->ne[0] != s0->ne[0]) return false;
    if (d->ne[0] != s0->ne[1] || d->ne[1] != s1->ne[1]) return false;
    for (int i = 2; i < 4; i++)
        if (s0->ne[i] != 1 || s1->ne[i] != 1 || d->ne[i] != 1) return false;
    // nb[0] of a quantised ggml tensor is its block size in bytes
    const size_t esz0 = s0->type == MLZC_TYPE_F16 ? 2 : (s0->type == MLZC_TYPE_F32 ? 4 : dense_row_bytes(s0->type, 256));
    if (s0->nb[0] != esz0 || s1->nb[0] != 4 || d->nb[0] != 4) return false;
    if (is_kquant(s0->type) && s0->ne[0] % 256 != 0) return false;
    return true;
}

}  // namespace

extern "C" int mlzc_weight_cache_clear(void) {
    std::lock_guard<std::mutex> lk(g_wcache_mu);
    for (auto& kv : g_wcache) mlzc_weight_free(kv.second.w);
    g_wcache.clear();
    return MLZC_OK;
}

extern "C" int mlzc_try_mul_mat(const mlzc_tensor* src0, const mlzc_tensor* src1, mlzc_tensor* dst, int ith,
                                int nth) {
    if (!mul_mat_gate(src0, src1, dst)) return 0;
    if (nth < 1 || ith < 0 || ith >= nth) return 0;
    return run_node(dst->data, ith, nth, [&]() -> int {
        int st = MLZC_OK;
        mlzc_weight w = cached_weight(src0, g_hook_device, &st);
        if (!w) return 0;
        st = mlzc_mul_mat(w, static_cast<const float*>(src1->data), src1->nb[1], src1->ne[1],
                          static_cast<float*>(dst->data), dst->nb[1]);
        return st == MLZC_OK ? 1 : 0;
    });
}

namespace {
// Byte extent of a 4-d view with element size `esz` and innermost extent ne0.
size_t extent(int64_t ne0, size_t esz, int64_t n1, size_t nb1, int64_t n2, size_t nb2, int64_t n3, size_t nb3) {
    if (ne0 <= 0 || n1 <= 0 || n2 <= 0 || n3 <= 0) return 0;
    return (size_t)(n1 - 1) * nb1 + (size_t)(n2 - 1) * nb2 + (size_t)(n3 - 1) * nb3 + (size_t)ne0 * esz;
}
}  // namespace

extern "C" int mlzc_try_flash_attn(const mlzc_fa_desc* desc, int ith, int nth) {
    if (check_fa_args(desc) != MLZC_OK) return 0;
    if (nth < 1 || ith < 0 || ith >= nth) return 0;
    return run_node(desc->dst, ith, nth, [&]() -> int {
        const int device = g_hook_device;
        DeviceCtx* c = device_ctx(device);
        if (!c) return 0;
        DeviceGuard g(device);
        if (!g.ok) return 0;
        HostArena* a = arena(device);
        std::lock_guard<std::mutex> lk(a->mu);
        const mlzc_fa_desc& d = *desc;
        const size_t qb = extent(d.head_dim_k, 4, d.n_queries, d.q_nb[1], d.n_head_q, d.q_nb[2], d.batch_size, d.q_nb[3]);
        const size_t kb = extent((int64_t)fa_row_bytes(d.k_type, d.head_dim_k), 1, d.n_kv, d.k_nb[1], d.n_head_kv,
                                 d.k_nb[2], d.batch_size, d.k_nb[3]);
        const size_t vb = extent((int64_t)fa_row_bytes(d.v_type, d.head_dim_v), 1, d.n_kv, d.v_nb[1], d.n_head_kv,
                                 d.v_nb[2], d.batch_size, d.v_nb[3]);
        const size_t db = extent(d.head_dim_v, 4, d.n_queries, d.dst_nb[1], d.n_head_q, d.dst_nb[2], d.batch_size, d.dst_nb[3]);
        const size_t mb = d.mask ? extent(d.n_kv, 4, d.n_queries, d.mask_nb[1], d.n_head_q, d.mask_nb[2], d.batch_size, d.mask_nb[3]) : 0;
        if (d.mask && d.mask_nb[0] != 4) return 0;
        mlzc_fa_desc dd = d;
        size_t wsb = 0;
        if (fa_workspace_bytes(&d, &wsb) != MLZC_OK) return 0;
        cudaStream_t s = c->stream;
        if (a->q.ensure(qb) || a->k.ensure(kb) || a->v.ensure(vb) || a->dst.ensure(db) || a->ws.ensure(wsb)) return 0;
        if (mb && a->mask.ensure(mb)) return 0;
        if (d.kv_len && a->kvlen.ensure((size_t)d.batch_size * 4)) return 0;
        if (cudaMemcpyAsync(a->q.ptr, d.q, qb, cudaMemcpyHostToDevice, s) != cudaSuccess) return 0;
        // dst may be a strided view: seed the device copy so bytes between rows survive
        if (cudaMemcpyAsync(a->dst.ptr, d.dst, db, cudaMemcpyHostToDevice, s) != cudaSuccess) return 0;
        if (kb && cudaMemcpyAsync(a->k.ptr, d.k, kb, cudaMemcpyHostToDevice, s) != cudaSuccess) return 0;
        if (vb && cudaMemcpyAsync(a->v.ptr, d.v, vb, cudaMemcpyHostToDevice, s) != cudaSuccess) return 0;
        if (mb && cudaMemcpyAsync(a->mask.ptr, d.mask, mb, cudaMemcpyHostToDevice, s) != cudaSuccess) return 0;
        if (d.kv_len && cudaMemcpyAsync(a->kvlen.ptr, d.kv_len, (size_t)d.batch_size * 4, cudaMemcpyHostToDevice, s) != cudaSuccess) return 0;
        dd.q = static_cast<const float*>(a->q.ptr);
        dd.k = a->k.ptr;
        dd.v = a->v.ptr;
        dd.mask = mb ? static_cast<const float*>(a->mask.ptr) : nullptr;
        dd.dst = static_cast<float*>(a->dst.ptr);
        dd.kv_len = d.kv_len ? static_cast<const int32_t*>(a->kvlen.ptr) : nullptr;
        if (launch_flash_attn(c, &dd, a->ws.ptr, a->ws.bytes, s) != MLZC_OK) return 0;
        if (cudaMemcpyAsync(d.dst, a->dst.ptr, db, cudaMemcpyDeviceToHost, s) != cudaSuccess) return 0;
        if (cudaStreamSynchronize(s) != cudaSuccess) return 0;
        return 1;
    });
}
