// quant.cu -- F32 -> Q8_K activation quantisation on the GPU.
//
// Replaces quantize_row_q8_k_reference (src/simd/ggml_simd_hook.cpp:109-148), which the
// reference hook runs on every ggml thread for every activation column before its Q4_K
// dot products (:197-204, :244-251).  Block layout (292 bytes per 256 values): f32 d at 0,
// 256 int8 quants at 4, 16 int16 group sums at 260.  Arithmetic, step for step as the
// reference: amax = max |x| (NaN ignored, as its `>` comparison does), d = amax / 127
// (IEEE division), id = d ? 1 / d : 0, q = round-half-away-from-zero(x * id) with no
// fused multiply-add, sums of 16 consecutive quants.  The results are bit-identical to
// the reference on finite inputs.
//
// One warp per block: each lane loads 8 consecutive values (two 16-byte loads when the
// column is 16-byte aligned), the amax is a shuffle reduction, lane pairs add their group
// sums.  HBM-bound: 1024 bytes read and 292 written per block.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int kQ8KBytes = 292;
constexpr int kQ8Warps = 8;   // blocks per CTA

__global__ void __launch_bounds__(kQ8Warps * 32)
quantize_q8k_kernel(const char* __restrict__ x, size_t x_cs, int nblk, int N, uint8_t* __restrict__ out, size_t out_cs,
                    int vec) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // X may be the previous kernel's output
    const int lane = threadIdx.x & 31;
    const int64_t total = (int64_t)nblk * N;
    for (int64_t wb = (int64_t)blockIdx.x * kQ8Warps + (threadIdx.x >> 5); wb < total;
         wb += (int64_t)gridDim.x * kQ8Warps) {
        const int n = (int)(wb / nblk), b = (int)(wb % nblk);
        const float* xb = reinterpret_cast<const float*>(x + (size_t)n * x_cs) + (size_t)b * 256 + lane * 8;
        float v[8];
        if (vec) {
            const float4 a = ptx::ld_act(reinterpret_cast<const float4*>(xb));
            const float4 c = ptx::ld_act(reinterpret_cast<const float4*>(xb) + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = ptx::ld_act(xb + e);
        }
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) amax = fabsf(v[e]) > amax ? fabsf(v[e]) : amax;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float t = __shfl_xor_sync(0xffffffffu, amax, o);
            amax = t > amax ? t : amax;
        }
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint32_t w0 = 0, w1 = 0;
        int sum = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int q = (int)roundf(__fmul_rn(v[e], id));
            sum += q;
            const uint32_t byte = (uint32_t)(q & 0xFF);
            if (e < 4) w0 |= byte << (8 * e);
            else w1 |= byte << (8 * (e - 4));
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);   // lanes 2g, 2g + 1 hold group g
        uint8_t* blk = out + (size_t)n * out_cs + (size_t)b * kQ8KBytes;
        if (lane == 0) *reinterpret_cast<float*>(blk) = d;
        uint32_t* qs = reinterpret_cast<uint32_t*>(blk + 4 + lane * 8);
        qs[0] = w0;
        qs[1] = w1;
        if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(blk + 260 + lane) = (int16_t)sum;
    }
}

}  // namespace
}  // namespace mlzc

using namespace mlzc;

extern "C" int mlzc_quantize_q8k_dev(const float* x, size_t x_col_bytes, int64_t K, int64_t N, void* out,
                                     size_t out_col_bytes, void* stream) {
    if (K < 0 || N < 0) return fail(MLZC_ERR_INVALID, "quantize_q8k: negative dimension");
    if (K % 256 != 0) return fail(MLZC_ERR_INVALID, "quantize_q8k: K %% 256 != 0 (K=%lld)", (long long)K);
    if (K == 0 || N == 0) return MLZC_OK;
    if (!x || !out) return fail(MLZC_ERR_INVALID, "quantize_q8k: null pointer");
    const int64_t nblk = K / 256;
    if (x_col_bytes < (size_t)K * 4 || x_col_bytes % 4 || (uintptr_t)x % 4)
        return fail(MLZC_ERR_INVALID, "quantize_q8k: x columns must hold K aligned floats");
    if (out_col_bytes < (size_t)nblk * kQ8KBytes || out_col_bytes % 4 || (uintptr_t)out % 4)
        return fail(MLZC_ERR_INVALID, "quantize_q8k: out columns must hold K/256 blocks of 292 bytes, 4-byte aligned");
    if (nblk > (1 << 30) || N > (1 << 30)) return fail(MLZC_ERR_INVALID, "quantize_q8k: too large");
    DeviceCtx* c = current_ctx();
    if (!c) return MLZC_ERR_CUDA;
    const int vec = ((uintptr_t)x % 16 == 0 && x_col_bytes % 16 == 0) ? 1 : 0;
    const int64_t blocks = nblk * N;
    const int grid = (int)std::min<int64_t>((blocks + kQ8Warps - 1) / kQ8Warps, (int64_t)c->sm_count * 16);
    MLZC_CUDA_TRY(launch_pdl(quantize_q8k_kernel, dim3(grid), dim3(kQ8Warps * 32), 0, static_cast<cudaStream_t>(stream),
                             reinterpret_cast<const char*>(x), x_col_bytes, (int)nblk, (int)N,
                             static_cast<uint8_t*>(out), out_col_bytes, vec));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}
