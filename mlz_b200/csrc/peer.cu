// peer.cu -- all-gather of row-sharded mul_mat slices through peer (NVLink) memory.
//
// The reference has no multi-GPU path.  For the row-sharded mul_mat every rank computes
// the Y slice of its M/G weight rows; instead of an NCCL all-gather, two small kernels move
// the slices through a symmetric exchange region that every rank allocated and opened on
// every peer at communicator set-up (CUDA IPC over NVLink / NVSwitch):
//   push: the rank's slice [N][m_loc] is stored into slot[parity] of every rank (itself
//         included) at offset rank * slice_stride -- 16-byte stores straight into peer
//         memory -- then the last CTA to finish releases this rank's epoch flag on every
//         rank (a system-scope fence orders all CTAs' stores before it);
//   wait: one thread per CTA acquires the G flags of the epoch (bounded by %globaltimer:
//         MLZC_DEVERR_WAIT_TIMEOUT and no output on expiry), then the CTAs copy the slots
//         into Y in ggml order (y[n][r * m_loc + m] = slot[r][n][m]); the last CTA to
//         finish advances the epoch counter.
// Epochs live in device memory (so a CUDA graph of the calls replays correctly); the two
// slots alternate by epoch parity, which is safe because a rank pushes epoch e + 2 only
// after its wait for e + 1, which needs every rank's push of e + 1, which each rank's
// stream issues after its own wait (and copy) of e.  No TMA and no multicast touch peer
// memory: plain st.global / ld.global.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "internal.h"
#include "peer.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    return *reinterpret_cast<const volatile uint32_t*>(p);
}

__global__ void __launch_bounds__(256)
peer_push_kernel(const uint4* __restrict__ slice, size_t chunks, PeerView pv) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // the slice is the previous kernel's output
    PeerHeader* me = reinterpret_cast<PeerHeader*>(pv.base[pv.rank]);
    const uint32_t e = ld_volatile(&me->epoch) + 1;
    const size_t slot_off = kPeerHeaderBytes + (size_t)(e & 1) * pv.slot_bytes + (size_t)pv.rank * pv.slice_stride;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = ptx::ld_act(slice + i);
        for (int r = 0; r < pv.G; ++r) reinterpret_cast<uint4*>(pv.base[r] + slot_off)[i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int done = atomicAdd(&me->push_done, 1u);
        if (done == gridDim.x - 1) {
            me->push_done = 0;
            __threadfence_system();
            for (int r = 0; r < pv.G; ++r)
                st_release_sys(&reinterpret_cast<PeerHeader*>(pv.base[r])->flag[e & 1][pv.rank], e);
        }
    }
}

__global__ void __launch_bounds__(256)
peer_wait_kernel(PeerView pv, int N, int m_loc, float* __restrict__ y, size_t y_cs, unsigned int* err) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // this rank's push has completed; Y may be read by the previous kernel
    PeerHeader* me = reinterpret_cast<PeerHeader*>(pv.base[pv.rank]);
    __shared__ int ok;
    const uint32_t e = ld_volatile(&me->epoch) + 1;
    if (threadIdx.x == 0) {
        ok = 1;
        const uint64_t t0 = ptx::global_ns();
        for (int r = 0; r < pv.G && ok; ++r) {
            while (ld_acquire_sys(&me->flag[e & 1][r]) != e) {
                if (ptx::global_ns() - t0 > ptx::kWaitNs) {
                    atomicOr(err, MLZC_DEVERR_WAIT_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (ok) {
        const char* slots = pv.base[pv.rank] + kPeerHeaderBytes + (size_t)(e & 1) * pv.slot_bytes;
        const int64_t total = (int64_t)pv.G * N * m_loc;
        const bool vec = (m_loc % 4 == 0) && (y_cs % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
        if (vec) {
            const int64_t total4 = total / 4;
            const int q = m_loc / 4;
            for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
                const int m4 = (int)(i % q);
                const int64_t rn = i / q;
                const int n = (int)(rn % N), r = (int)(rn / N);
                const float4 v = ptx::ld_act(reinterpret_cast<const float4*>(slots + (size_t)r * pv.slice_stride +
                                                                              ((size_t)n * m_loc + 4 * m4) * 4));
                *reinterpret_cast<float4*>(reinterpret_cast<char*>(y) + (size_t)n * y_cs + ((size_t)r * m_loc + 4 * m4) * 4) = v;
            }
        } else {
            for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
                const int m = (int)(i % m_loc);
                const int64_t rn = i / m_loc;
                const int n = (int)(rn % N), r = (int)(rn / N);
                const float v = ptx::ld_act(reinterpret_cast<const float*>(slots + (size_t)r * pv.slice_stride) +
                                            (size_t)n * m_loc + m);
                reinterpret_cast<float*>(reinterpret_cast<char*>(y) + (size_t)n * y_cs)[(size_t)r * m_loc + m] = v;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();   // this CTA's read of the epoch happens before its count
        const unsigned int done = atomicAdd(&me->wait_done, 1u);
        if (done == gridDim.x - 1) {   // every CTA has read the epoch: advance it
            me->wait_done = 0;
            me->epoch = e;
        }
    }
}

}  // namespace

int launch_peer_allgather(const PeerView& pv, const float* slice, int N, int m_loc, float* y, size_t y_cs,
                          unsigned int* err, int sm_count, cudaStream_t s) {
    const size_t chunks = pv.slice_stride / 16;
    const int gp = (int)std::max<size_t>(1, std::min<size_t>((chunks + 255) / 256, (size_t)sm_count));
    MLZC_CUDA_TRY(launch_pdl(peer_push_kernel, dim3(gp), dim3(256), 0, s, reinterpret_cast<const uint4*>(slice), chunks, pv));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    const int64_t total = (int64_t)pv.G * N * m_loc;
    const int gw = (int)std::max<int64_t>(1, std::min<int64_t>((total / 4 + 255) / 256, (int64_t)sm_count));
    MLZC_CUDA_TRY(launch_pdl(peer_wait_kernel, dim3(gw), dim3(256), 0, s, pv, N, m_loc, y, y_cs, err));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

}  // namespace mlzc
