// ptx.cuh -- inline-PTX helpers shared by the kernels: mbarriers with bounded waits and
// bulk (TMA engine) copies into shared memory.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "internal.h"

namespace mlzc {
namespace ptx {

constexpr uint64_t kWaitNs = 2000000000ull;   // 2 s bound on any single mbarrier wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Slow path of mbar_wait: polls until the phase completes, gives up after `limit_ns`
// (kWaitNs for every kernel; setting the error word and `abort_flag`) or as soon as
// another thread of the CTA set `abort_flag`.
__device__ __noinline__ inline bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                   unsigned int* err, uint64_t limit_ns = kWaitNs) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 31) == 0) {
            if (*abort_flag) return false;
            if (global_ns() - t0 > limit_ns) {
                atomicOr(err, MLZC_DEVERR_WAIT_TIMEOUT);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Waits for the phase of parity `parity` of `bar` (bounded, see mbar_wait_slow).  The
// common case -- the phase has already completed -- stays inline, with no call.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, unsigned int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, abort_flag, err);
}

// Contiguous bulk copy global -> shared (16-byte aligned, size a multiple of 16), completing
// `bytes` on the mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// c += a . b for one m16n8k16 tile: A 16x16 and B 16x8 f16 fragments, f32 accumulators
// (fragment ownership per the PTX ISA: lane l holds rows l/4 and l/4 + 8, k pairs 2(l%4)
// and 2(l%4) + 8 of A; k pairs of column l/4 of B; rows l/4, l/4 + 8 x columns 2(l%4), +1
// of C).
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// f16 hi + lo split of two floats: x ~= hi + lo with |x - hi - lo| ~ 2^-22 |x|.
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_h2(x0 - hf.x, x1 - hf.y);
}

// Transposes an 8x8 f16 matrix held as the standard mma fragment (lane: row lane/4,
// columns 2*(lane%4) and +1).
__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// Programmatic dependent launch: a kernel launched with the programmatic-serialization
// attribute may start while the previous kernel of the stream finishes; it must call
// pdl_wait() before it reads anything the previous kernel may have written or writes
// anything the previous kernel may still read.  pdl_launch_dependents() lets the next such
// kernel start early (its own pdl_wait() still waits for this whole grid).  After the
// wait the previous grid's writes are visible to ordinary (weak) loads -- ld_act() below,
// TMA and bulk copies -- but not to the non-coherent read-only path (__ldg,
// ld.global.nc), which assumes data unchanged for the kernel's whole life and which a
// compiler may also hoist above the wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Loads of data that an earlier kernel of the stream may have written (activations,
// prepared operands, partial records): weak ld.global, cached in L1 for reuse within the
// kernel.  volatile keeps them in program order after pdl_wait().
__device__ __forceinline__ float ld_act(const float* p) {
    float v;
    asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float4 ld_act(const float4* p) {
    float4 v;
    asm volatile("ld.global.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ int ld_act(const int* p) {
    int v;
    asm volatile("ld.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_act(const uint2* p) {
    uint2 v;
    asm volatile("ld.global.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_act(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// 16-byte weight load, streamed (never re-read, not allocated in L1).  `nc` = the weights
// cannot be an output of a kernel still running on the stream (read-only path); otherwise
// a weak coherent load.
template <bool nc>
__device__ __forceinline__ uint4 ld_weight16(const void* p) {
    uint4 v;
    if constexpr (nc)
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(p));
    else
        asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(p));
    return v;
}

}  // namespace ptx

// Launches `kernel` with programmatic stream serialization allowed (see pdl_wait), unless
// the launch-overlap mode is MLZC_OVERLAP_OFF.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap_mode() == MLZC_OVERLAP_OFF ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
}  // namespace mlzc
