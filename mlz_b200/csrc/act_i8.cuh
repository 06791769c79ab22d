// act_i8.cuh -- activations as int8 hi + lo per 256-value block, for the int8 tensor-core
// decode paths (q4k_i8.cu, q6k_i8.cu).
//
// Each 256-value block of an activation column becomes one f32 scale s = max|x| / 127 and two
// int8 vectors: hi = rint(x / s), lo = rint(254 (x - s hi) / s), so x ~= s (hi + lo / 254) with
// an error below s / 508 per value.  The prep kernel writes one record per 8 blocks (a "unit"
// column of the weight tiles), which the main kernels' rings carry stage by stage:
//   [NV][2080] int8: vector 2n = hi, 2n + 1 = lo of column n, block w at 256 w (the 32 pad
//                    bytes make the B-fragment loads of a half-warp hit distinct banks)
//   [NCT][8] f32:    the scale s of each (column, block)
//   [8][NV][GPB] f16: the sums of the unquantised values over each of the GPB groups of a
//                    block (256 / GPB values each): f16 hi part in vector 2n, the rest times
//                    2048 in vector 2n + 1 (sum = hi + lo / 2048)
// with NCT columns (N padded to 1, 2 or 4; padded columns are zeros) and NV = 2 NCT.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace mlzc {
namespace act_i8 {

constexpr int kVarStride = 2080;

__host__ __device__ constexpr uint32_t rec_bytes(int nct, int gpb) {
    return (uint32_t)(2 * nct * kVarStride + nct * 32 + 8 * 2 * nct * gpb * 2);
}
__host__ __device__ constexpr uint32_t rec_scale_off(int nct) { return (uint32_t)(2 * nct * kVarStride); }
__host__ __device__ constexpr uint32_t rec_sum_off(int nct) { return rec_scale_off(nct) + (uint32_t)(nct * 32); }

// One warp per (block kb < nst * 8, column n < nct): quantises the block's 256 values,
// sums its GPB groups and writes them into unit kb / 8's record (zeros for blocks past the
// row and columns past N).  Also zeroes Y (M rows of N columns), which the main kernels add
// their pieces into.
template <int GPB>
__global__ void __launch_bounds__(256) prep_kernel(const char* __restrict__ x, size_t x_cs, int N, int nct, int nblk,
                                                   int nst, uint32_t rbytes, char* __restrict__ rec,
                                                   char* __restrict__ y, size_t y_cs, int M) {
    constexpr int kLanesPerGroup = 32 / GPB;   // each lane holds 8 consecutive values
    static_assert(kLanesPerGroup >= 1 && 32 % GPB == 0, "groups of 8 values or more");
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // x comes from, and the records and Y may still be read by, the previous kernel
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)M * N;
         i += (long long)gridDim.x * blockDim.x)
        reinterpret_cast<float*>(y + (size_t)(i / M) * y_cs)[i % M] = 0.0f;
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (item >= nst * 8 * nct) return;
    const int kb = item / nct, n = item % nct;
    float v[8];
    if (kb < nblk && n < N) {
        const float4* p = reinterpret_cast<const float4*>(x + (size_t)n * x_cs) + (size_t)kb * 64 + 2 * lane;
        const float4 a = ptx::ld_act(p), b = ptx::ld_act(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    float amax = 0.0f, sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        amax = fmaxf(amax, fabsf(v[i]));
        sum += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
#pragma unroll
    for (int o = 1; o < kLanesPerGroup; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float s = amax / 127.0f;
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int h = __float2int_rn(v[i] * inv);
        const float r = fmaf(-s, (float)h, v[i]);
        const int l = max(-127, min(127, __float2int_rn(r * inv * 254.0f)));
        hw[i >> 2] |= ((uint32_t)h & 0xFFu) << (8 * (i & 3));
        lw[i >> 2] |= ((uint32_t)l & 0xFFu) << (8 * (i & 3));
    }
    char* r = rec + (size_t)(kb >> 3) * rbytes;
    const int w = kb & 7;
    *reinterpret_cast<uint2*>(r + (2 * n) * kVarStride + w * 256 + 8 * lane) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(r + (2 * n + 1) * kVarStride + w * 256 + 8 * lane) = make_uint2(lw[0], lw[1]);
    if (lane == 0) reinterpret_cast<float*>(r + rec_scale_off(nct))[n * 8 + w] = s;
    if ((lane & (kLanesPerGroup - 1)) == 0) {
        // the lo part scaled by 2^11 so that it stays a normal f16 (consumers weight its
        // column by 2^-11): hi + lo / 2048 = sum to ~2^-22 relative, and 4x the inputs gives
        // exactly 4x both parts
        const __half sh = __float2half_rn(sum);
        const __half sl = __float2half_rn((sum - __half2float(sh)) * 2048.0f);
        __half* sp = reinterpret_cast<__half*>(r + rec_sum_off(nct));
        sp[(w * 2 * nct + 2 * n) * GPB + lane / kLanesPerGroup] = sh;
        sp[(w * 2 * nct + 2 * n + 1) * GPB + lane / kLanesPerGroup] = sl;
    }
}

}  // namespace act_i8
}  // namespace mlzc
