/*
 * mlzc.h -- C ABI of the B200 (sm_100a) implementation of MLz's src/simd hot path.
 *
 * The library (mlz_b200/libmlzc.so) replaces the CPU kernels behind MLz's ggml hook:
 *   - F16 / F32 weight x F32 activation mul_mat (decode GEMV and prefill GEMM),
 *   - Q4_K super-block weight x F32 activation mul_mat (dequant-dot),
 *   - F16-KV flash-attention decode with grouped-query heads,
 *   - row-sharded mul_mat over several GPUs of one node (NCCL all-gather of slices).
 *
 * Conventions (all entry points):
 *   - Every function returns an int status: MLZC_OK (0) on success, a negative
 *     MLZC_ERR_* on failure.  Nothing aborts or traps; mlzc_last_error() gives a
 *     human-readable message for the calling thread's last failure.
 *   - Plain pointers and sizes only.  "stream" is a cudaStream_t passed as void*
 *     (NULL = the legacy default stream).  "_dev" functions take device pointers and
 *     are asynchronous on that stream; the others take host pointers and return when
 *     the result is in host memory.
 *   - Tensors use ggml's layout: ne[0] is the contiguous axis, nb[] are byte strides.
 *     For mul_mat: W has ne = [K, M] (row m at w + m*w_row_bytes), X has ne = [K, N]
 *     (column n at x + n*x_col_bytes), Y has ne = [M, N] (element (m, n) at
 *     y + n*y_col_bytes + 4*m).  This is the contract ggml_compute_forward_mul_mat
 *     asserts (src/simd/ggml-cpu-simd.c:1273-1288 in the MLz tree).
 *   - Type ids are ggml_type values: F32 = 0, F16 = 1, Q4_K = 12, Q6_K = 14.
 *   - F16 weights: activations are narrowed to f16 (round-to-nearest-even) and the
 *     products are accumulated in fp32, which is the contract of the reference's
 *     F16 path (type_traits_cpu[F16].vec_dot_type = F16, ggml-cpu-simd.c:215-220).
 *     F32 weights: activations stay f32, fp32 accumulation.  Q4_K / Q6_K weights:
 *     activations rounded to f16 once, exact f16 dequant of the quants, fp32 accumulation
 *     (within 2e-3 of the dequantised-F32 product).
 *   - The first call that touches a device creates its context (a small device
 *     allocation); make that call, or mlzc_init(), before any stream capture.
 */
#ifndef MLZC_H
#define MLZC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLZC_VERSION 1

enum mlzc_status {
    MLZC_OK = 0,
    MLZC_ERR_INVALID = -1,      /* bad pointer, size, stride or alignment */
    MLZC_ERR_UNSUPPORTED = -2,  /* type / shape combination this library does not take */
    MLZC_ERR_CUDA = -3,         /* a CUDA runtime call failed */
    MLZC_ERR_NOMEM = -4,        /* device or pinned allocation failed, or workspace too small */
    MLZC_ERR_DEVICE = -5,       /* a kernel reported an error (see mlzc_device_errors) */
    MLZC_ERR_COMM = -6          /* NCCL failure or timeout */
};

/* ggml type ids (GGML_TYPE_*); Q4_1, Q5_0, Q5_1 and IQ4_NL are used as KV-cache types only. */
enum mlzc_type {
    MLZC_TYPE_F32 = 0, MLZC_TYPE_F16 = 1, MLZC_TYPE_Q4_0 = 2, MLZC_TYPE_Q4_1 = 3, MLZC_TYPE_Q5_0 = 6,
    MLZC_TYPE_Q5_1 = 7, MLZC_TYPE_Q8_0 = 8, MLZC_TYPE_Q4_K = 12, MLZC_TYPE_Q6_K = 14, MLZC_TYPE_IQ4_NL = 20
};

/* Attention mode bits; same values as FA_MODE_* (src/simd/flash_attention.h:43-49). */
#define MLZC_FA_MODE_GQA_BATCH 0x04u
#define MLZC_FA_MODE_ALIBI 0x08u
#define MLZC_FA_MODE_SOFTCAP 0x10u

/* Kernel error bits reported by mlzc_device_errors(). */
#define MLZC_DEVERR_WAIT_TIMEOUT 0x1u  /* a bounded mbarrier / flag wait gave up */
#define MLZC_DEVERR_BAD_SHAPE 0x2u     /* a kernel saw a shape its launch did not promise */

/* ---------------------------------------------------------------- runtime */

/* Number of kernels this library has launched in this process (all devices).  A
 * diagnostics counter with no counterpart in the reference; benchmarks read it around a
 * timed region. */
int mlzc_launch_count(uint64_t* out_count);

/* Launch overlap (programmatic dependent launch).  With MLZC_OVERLAP_SAFE (the default)
 * each kernel of a call may start while the previous kernel of its stream finishes and
 * does its set-up then, but reads and writes global memory only after that kernel has
 * completed: any producer of W, X or the workspace is safe.  MLZC_OVERLAP_WEIGHTS also
 * issues the first weight (W) loads of the decode-shaped kernels before that point; use it
 * only when no kernel still running on the stream writes W (model weights), the case of
 * a decode loop.  MLZC_OVERLAP_OFF launches every kernel in plain stream order.  The mode
 * is process-wide and read at each launch (so at capture time for CUDA graphs).
 * No counterpart in the reference (its CPU kernels have no launches to overlap). */
#define MLZC_OVERLAP_OFF 0
#define MLZC_OVERLAP_SAFE 1
#define MLZC_OVERLAP_WEIGHTS 2
int mlzc_set_launch_overlap(int mode);
int mlzc_get_launch_overlap(int* out_mode);

/* Message of the calling thread's last failed call ("" if none). */
const char* mlzc_last_error(void);
int mlzc_version(void);
/* Create the context of CUDA device `device` (idempotent). */
int mlzc_init(int device);
/* Release every context, cached weight and workspace this library holds. */
int mlzc_shutdown(void);
/* Read and clear the kernel error word of `device` (MLZC_DEVERR_* bits), together with the
 * word of the allocation-free entry point.  Synchronises the device.  It creates no
 * context and allocates nothing, so callers of mlzc_flash_attn_dev_noalloc can use it. */
int mlzc_device_errors(int device, uint32_t* out_bits);

/* Failure-path self-test: launches one small kernel on `device` that waits on an
 * mbarrier nothing arrives on, through the same bounded wait every kernel uses, with a
 * limit of `limit_us` microseconds (1 .. 2 000 000).  The wait gives up, the kernel sets
 * MLZC_DEVERR_WAIT_TIMEOUT in the device error word and returns, and *out_gave_up is 1;
 * the context stays usable.  Synchronous.  No counterpart in the reference (its kernels
 * have no waits). */
int mlzc_selftest_wait_timeout(int device, uint32_t limit_us, int* out_gave_up);

/* --------------------------------------------------- device-pointer kernels */

/* Workspace (device bytes) that mlzc_mul_mat_dev needs for this shape; 0 if none. */
int mlzc_mul_mat_workspace_bytes(int w_type, int64_t M, int64_t K, int64_t N, size_t* out_bytes);

/* Y = W . X in ggml layout (see the header comment), on `stream`.
 * Replaces: ggml_simd_try_mul_mat's compute branches (src/simd/ggml_simd_hook.cpp:188-311),
 * simd_matmul_f32 (src/simd/simd_matmul.cpp:214-251), simd_matmul_f16 (:428-480), and the
 * upstream F16 vec_dot path the hook falls back to (src/simd/ggml-cpu-simd.c:1314-1465).
 * Pointers and strides need only their element alignment; 16-byte aligned W and X with
 * 16-byte multiple strides take the vectorised kernels, anything else a slower exact
 * path.  Q4_K needs K % 256 == 0 and 16-byte aligned blocks and activation columns;
 * Q6_K (210-byte blocks, ggml_simd_hook.cpp:282-288 routes them with Q4_K) needs
 * K % 256 == 0, a 4-byte aligned W with an even row stride, and 16-byte aligned
 * activation columns.
 * `workspace` may be NULL when the query above returned 0. */
int mlzc_mul_mat_dev(int w_type, const void* w, size_t w_row_bytes, int64_t M, int64_t K,
                     const float* x, size_t x_col_bytes, int64_t N,
                     float* y, size_t y_col_bytes,
                     void* workspace, size_t workspace_bytes, void* stream);

/* F32 activations -> Q8_K blocks, on `stream`: column n of X (K floats at
 * x + n*x_col_bytes, K % 256 == 0) becomes K/256 blocks of 292 bytes at
 * out + n*out_col_bytes (f32 d = amax/127, 256 int8 q = round(x/d), 16 int16 sums of 16
 * consecutive q).  Bit-identical to the reference on finite inputs.
 * Replaces: quantize_row_q8_k_reference (src/simd/ggml_simd_hook.cpp:109-148), run by the
 * hook on each activation column before the Q4_K dot products (:197-204, :244-251). */
int mlzc_quantize_q8k_dev(const float* x, size_t x_col_bytes, int64_t K, int64_t N, void* out,
                          size_t out_col_bytes, void* stream);

/* One flash-attention call.  Field names and meaning follow flash_attn_config_t
 * (src/simd/flash_attention.h:65-114); pointers are DEVICE pointers for
 * mlzc_flash_attn_dev and HOST pointers for mlzc_try_flash_attn.
 * Q: f32, ne = [DK, n_queries, n_head_q, batch]; K/V: f16, ne = [DK|DV, n_kv,
 * n_head_kv, batch]; mask: f32 [n_kv, n_queries] added to the scaled scores (NULL =
 * none); dst: f32, element (d, iq, ihq, ib) at d*4 + iq*dst_nb[1] + ihq*dst_nb[2] +
 * ib*dst_nb[3].  kv_len (extension): int32 per batch element, keys at positions
 * >= kv_len[ib] are not read (NULL = n_kv for every element); this is how a ragged
 * batch of sequences is expressed without a mask.
 * Score of key j for query iq of head ihq: s = scale * <q, k_j>; s += mask(iq, j);
 * if MLZC_FA_MODE_SOFTCAP: s = softcap * tanh(s / softcap); if MLZC_FA_MODE_ALIBI:
 * s += slope(ihq) * (j - iq) with slope = 2^(-8/P)^(ihq+1), P = n_head_q rounded up to a
 * power of two (the order and slope of flash_attention.cpp:339-363).  KV head of query
 * head ihq: ihq * n_head_kv / n_head_q.  Rows with no visible key produce zeros. */
typedef struct {
    int64_t head_dim_k, head_dim_v, n_queries, n_kv, n_head_q, n_head_kv, batch_size;
    float scale, logit_softcap, max_bias;
    uint32_t mode;
    const float* q;
    const void* k;
    const void* v;
    const float* mask;
    float* dst;
    size_t q_nb[4], k_nb[4], v_nb[4], mask_nb[4], dst_nb[4];
    int32_t k_type, v_type;   /* both F16, both F32 (DK <= 128) or both one quantised KV type
                                 (Q8_0 Q4_0 Q4_1 Q5_0 Q5_1 IQ4_NL) */
    const int32_t* kv_len;    /* NULL or batch_size entries (device memory for _dev) */
} mlzc_fa_desc;

/* Workspace (device bytes) mlzc_flash_attn_dev needs for this call. */
int mlzc_flash_attn_workspace_bytes(const mlzc_fa_desc* desc, size_t* out_bytes);

/* Flash-attention on device pointers.
 * Replaces: flash_attn_dispatch's F16/F16 branch (src/simd/flash_attention.cpp:143-150)
 * -> simd_flash_attn_f16_avx512 (kernels/x86/flash/flash_attn_f16_avx512.asm + the FA2
 * skeleton flash_attn_fa2_skeleton_avx512.inc:394-842).
 * Requirements: DK == DV in {64, 128, 256}; contiguous f16 K/V rows whose strides
 * (nb[1..3]) are multiples of 16 bytes; contiguous, 16-byte aligned f32 q rows.
 * Quantised KV cache (the Q8_0, Q4_0, Q4_1, Q5_0, Q5_1 and IQ4_NL branches of
 * flash_attn_dispatch, flash_attention.cpp:112-248 -> simd_flash_attn_<type>_avx512,
 * kernels/x86/flash/flash_attn_<type>_avx512.asm): K and V rows of 32-value blocks in the
 * GGUF layouts (nb[0] = the block size, as ggml sets it), 4-byte aligned with 4-byte
 * multiple strides.  Element: Q8_0 (34 B) f16 d * int8 q; Q4_0 (18 B) d * (nibble - 8);
 * Q4_1 (20 B) d * nibble + f16 m; Q5_0 (22 B) d * (q5 - 16); Q5_1 (24 B) d * q5 + m, q5 the
 * nibble with its fifth bit from the block's 32-bit qh; IQ4_NL (18 B) d * table[nibble].
 * F32 K/V (flash_attn_dispatch's F32 branch -> simd_flash_attn_f32_avx512), head_dim 64 or
 * 128: contiguous f32 rows (nb[0] = 4) on 4-byte boundaries with 4-byte multiple strides. */
int mlzc_flash_attn_dev(const mlzc_fa_desc* desc, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Same computation as mlzc_flash_attn_dev, for callers that cannot allocate device memory
 * per call (a host callback, a thread that must not block on a device-wide allocation, an
 * engine with a fixed memory budget, a binding without an allocator).  No counterpart in
 * the reference.  It allocates nothing: the split partials go to a fixed 16 MiB scratch
 * array inside the library's device image, held by every GPU that loads the library until
 * the process exits.  Calls needing more than that (mlzc_flash_attn_workspace_bytes)
 * fail with MLZC_ERR_NOMEM.  The first call on a device does that device's set-up, with
 * the device current: it looks up the array's device address and sets the decode
 * kernel's shared-memory attributes (once each); make it before any stream capture.  All
 * calls share the array, so calls that overlap on the GPU race; serialise them.  A kernel
 * whose bounded wait gave up reports MLZC_DEVERR_WAIT_TIMEOUT in a device word that
 * mlzc_device_errors reads and clears (without allocating). */
int mlzc_flash_attn_dev_noalloc(const mlzc_fa_desc* desc, void* stream);

/* ------------------------------------------------ host-pointer (hook) level */

/* The subset of struct ggml_tensor the hook reads. */
typedef struct {
    int32_t type;
    int64_t ne[4];
    size_t nb[4];
    void* data;
} mlzc_tensor;

/* Drop-in body for ggml_simd_try_mul_mat (src/simd/ggml_simd_hook.cpp:153-315): called by
 * every ggml threadpool thread (ith of nth) for the same MUL_MAT node.  Returns 1 when the
 * node was computed on the GPU (dst written) and 0 when the caller must fall back to the
 * CPU path.  All nth threads of a node receive the same answer, so a fallback is taken by
 * all of them together (the upstream path has barriers inside).  Thread 0 does the GPU
 * work: weights are uploaded on first use and cached on the device keyed by
 * (src0->data, type, ne, nb); X is copied in and Y copied out on every call.
 * ne[2] / ne[3] broadcast of ggml is not taken (returns 0 when ne[2] or ne[3] != 1). */
int mlzc_try_mul_mat(const mlzc_tensor* src0, const mlzc_tensor* src1, mlzc_tensor* dst,
                     int ith, int nth);

/* Drop-in body for ggml_simd_try_flash_attn (src/simd/ggml_simd_hook.cpp:317-375) with
 * host pointers in `desc`; same 1 / 0 contract and thread rule as mlzc_try_mul_mat. */
int mlzc_try_flash_attn(const mlzc_fa_desc* desc, int ith, int nth);

/* Device-resident weights for callers that manage their own tensors (the engine). */
typedef struct mlzc_weight_s* mlzc_weight;
int mlzc_weight_upload(int device, int w_type, const void* host, size_t row_bytes,
                       int64_t M, int64_t K, mlzc_weight* out);
int mlzc_weight_free(mlzc_weight w);
/* Y = W . X with X, Y in HOST memory (pinned or pageable).  Synchronous.  Calls with
 * N >= 256 columns are cut into up to 4 column chunks whose uploads, compute and
 * downloads overlap on three streams. */
int mlzc_mul_mat(mlzc_weight w, const float* x, size_t x_col_bytes, int64_t N,
                 float* y, size_t y_col_bytes);
/* Drop every weight cached by mlzc_try_mul_mat (e.g. when a model is unloaded). */
int mlzc_weight_cache_clear(void);

/* Page-lock an existing host range (e.g. ggml's compute buffer, which holds every src1 and
 * dst the hook sees) so the host-pointer calls copy it by DMA, overlapping the upload of
 * one column chunk with the compute and download of the others; pageable memory is copied
 * through a driver staging buffer, one direction at a time.  Idempotent; unregister
 * before freeing the range.  No counterpart in the reference (its buffers never leave the
 * host). */
int mlzc_host_register(void* ptr, size_t bytes);
int mlzc_host_unregister(void* ptr);

/* ---------------------------------------------------- multi-GPU (one node) */

typedef struct mlzc_comm_s* mlzc_comm;
#define MLZC_UNIQUE_ID_BYTES 128
/* Rank 0 creates the id and the caller distributes it to every rank. */
int mlzc_comm_unique_id(void* out_id);
/* Collective over `nranks` processes, one GPU each; `timeout_ms` bounds every wait. */
int mlzc_comm_init(int nranks, int rank, int device, const void* unique_id, int timeout_ms,
                   mlzc_comm* out);
int mlzc_comm_destroy(mlzc_comm comm);

/* Workspace for mlzc_mul_mat_sharded_dev. */
int mlzc_mul_mat_sharded_workspace_bytes(mlzc_comm comm, int w_type, int64_t M_total,
                                         int64_t K, int64_t N, size_t* out_bytes);

/* Row-sharded mul_mat: this rank holds rows [r*M_total/G, (r+1)*M_total/G) of W
 * (w_shard, M_total % G == 0) and computes that slice of Y; the slices are all-gathered
 * so that every rank ends with the full Y (ggml layout, M_total rows).  No counterpart
 * in the reference (it has no multi-GPU path).  The slices travel through the ranks'
 * exchange regions in peer memory over NVLink (the decode GEMV and the prefill GEMM store
 * their outputs straight into every rank's slot; a wait kernel then signals, waits and
 * gathers), or through an NCCL all-gather on `stream` where the peer regions could not be
 * set up.  Every rank makes the same calls in the same order. */
int mlzc_mul_mat_sharded_dev(mlzc_comm comm, int w_type, const void* w_shard,
                             size_t w_row_bytes, int64_t M_total, int64_t K,
                             const float* x, size_t x_col_bytes, int64_t N,
                             float* y, size_t y_col_bytes,
                             void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLZC_H */
