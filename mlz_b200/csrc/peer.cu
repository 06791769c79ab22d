// peer.cu -- all-gather of row-sharded mul_mat slices through peer (NVLink) memory.
//
// The reference has no multi-GPU path.  For the row-sharded mul_mat every rank computes
// the Y slice of its M/G weight rows; instead of an NCCL all-gather, two small kernels move
// the slices through a symmetric exchange region that every rank allocated and opened on
// every peer at communicator set-up (CUDA IPC over NVLink / NVSwitch):
//   push: the rank's slice [N][m_loc] is stored into slot[parity] of every rank (itself
//         included) at offset rank * slice_stride -- 16-byte stores straight into peer
//         memory.  For decode (one column) the GEMV itself does these stores (gemv.cu)
//         and there is no push kernel;
//   wait: its CTA 0 first releases this rank's epoch flag on every rank (release stores at
//         system scope; the kernel that stored the slice has completed), then one warp per
//         CTA acquires the G flags of the epoch (bounded by %globaltimer:
//         MLZC_DEVERR_WAIT_TIMEOUT and no output on expiry), the CTAs copy the slots into
//         Y in ggml order (y[n][r * m_loc + m] = slot[r][n][m]), and the last CTA to finish
//         advances the epoch counter.
// Epochs live in device memory (so a CUDA graph of the calls replays correctly); the two
// slots alternate by epoch parity, which is safe because a rank pushes epoch e + 2 only
// after its wait for e + 1, which needs every rank's push of e + 1, which each rank's
// stream issues after its own wait (and copy) of e.  Peer memory is only ever written (plain
// stores here and in the decode GEMV, TMA tensor stores in the prefill GEMM's epilogue) and
// read back by its owner: no copy engine load or cluster-wide broadcast reads another GPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "internal.h"
#include "peer.h"
#include "ptx.cuh"

namespace mlzc {
namespace {

constexpr int kPeerPiece = 2048;   // floats per CTA pass of the slot -> Y copy

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(256)
peer_push_kernel(const uint4* __restrict__ slice, size_t chunks, PeerView pv) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // the slice is the previous kernel's output
    const size_t off = peer_slice_offset(pv, peer_epoch(pv));
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = ptx::ld_act(slice + i);
        for (int r = 0; r < pv.G; ++r) reinterpret_cast<uint4*>(pv.base[r] + off)[i] = v;
    }
}

// The kernel before this one on the stream (the push kernel, the fused decode GEMV or the
// fused GEMM) stored this rank's slice into every rank's slot and has completed: G threads of
// CTA 0 release this rank's flag on the G ranks, then every CTA waits for all G flags and
// copies the slots into Y.
__global__ void __launch_bounds__(256)
peer_wait_kernel(PeerView pv, int N, int m_loc, float* __restrict__ y, size_t y_cs, unsigned int* err, int skip_self) {
    ptx::pdl_launch_dependents();
    ptx::pdl_wait();   // this rank's slice stores have completed; Y may be read by the previous kernel
    PeerHeader* me = reinterpret_cast<PeerHeader*>(pv.base[pv.rank]);
    __shared__ int ok;
    const uint32_t e = peer_epoch(pv);
    if (blockIdx.x == 0 && threadIdx.x < pv.G) {
        // message passing: the slice stores were completed by the kernel before this one (its
        // grid finished before pdl_wait returned), and each flag is a release store at system
        // scope; a reader acquires the flag before it reads the slot.  One thread per rank: a
        // single thread's release stores would each wait for the previous remote store to
        // complete (one NVLink round trip per rank).  (A sequentially consistent system fence
        // here measured 1.9 us per call and orders nothing more.)
        st_release_sys(&reinterpret_cast<PeerHeader*>(pv.base[threadIdx.x])->flag[e & 1][pv.rank], e);
    }
    if (threadIdx.x < 32) {
        // lane r polls rank r's flag: the G acquires overlap instead of taking one round trip
        // each (bounded; every lane gives up together)
        const int lane = threadIdx.x;
        bool mine = lane >= pv.G;
        const uint64_t t0 = ptx::global_ns();
        bool timed_out = false;
        while (!__all_sync(0xffffffffu, mine)) {
            if (!mine) mine = ld_acquire_sys(&me->flag[e & 1][lane]) == e;
            if (__any_sync(0xffffffffu, ptx::global_ns() - t0 > ptx::kWaitNs)) {
                timed_out = true;
                break;
            }
        }
        if (lane == 0) {
            ok = timed_out ? 0 : 1;
            if (timed_out) atomicOr(err, MLZC_DEVERR_WAIT_TIMEOUT);
        }
    }
    __syncthreads();
    if (ok) {
        // pieces of kPeerPiece floats of the (rank r, column n) rows: y[n][r*m_loc + m]
        const char* slots = pv.base[pv.rank] + kPeerHeaderBytes + (size_t)(e & 1) * pv.slot_bytes;
        // skip_self: this rank's slice is already in Y (its GEMM stored it there)
        const int nr = skip_self ? pv.G - 1 : pv.G;
        const int per_row = (m_loc + kPeerPiece - 1) / kPeerPiece;
        const int pieces = nr * N * per_row;
        const bool vec = (m_loc % 4 == 0) && (y_cs % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
        for (int pc = blockIdx.x; pc < pieces; pc += gridDim.x) {
            const int rn = pc / per_row, m0 = (pc - rn * per_row) * kPeerPiece;
            const int ri = rn / N, n = rn - ri * N;
            const int r = skip_self && ri >= pv.rank ? ri + 1 : ri;
            const int m1 = min(m_loc, m0 + kPeerPiece);
            const float* src = reinterpret_cast<const float*>(slots + (size_t)r * pv.slice_stride) + (size_t)n * m_loc;
            float* dst = reinterpret_cast<float*>(reinterpret_cast<char*>(y) + (size_t)n * y_cs) + (size_t)r * m_loc;
            if (vec) {
                for (int m4 = m0 / 4 + threadIdx.x; m4 < m1 / 4; m4 += blockDim.x)
                    reinterpret_cast<float4*>(dst)[m4] = ptx::ld_act(reinterpret_cast<const float4*>(src) + m4);
            } else {
                for (int m = m0 + threadIdx.x; m < m1; m += blockDim.x) dst[m] = ptx::ld_act(src + m);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // acq_rel: this CTA's read of the epoch happens before its count, and the last CTA's
        // epoch store after every count
        const unsigned int done = atom_add_acq_rel_gpu(&me->wait_done, 1u);
        if (done == gridDim.x - 1) {   // every CTA has read the epoch: advance it
            me->wait_done = 0;
            me->epoch = e;
        }
    }
}

}  // namespace

int launch_peer_wait(const PeerView& pv, int N, int m_loc, float* y, size_t y_cs, unsigned int* err, int sm_count,
                     cudaStream_t s, bool skip_self) {
    // one CTA pass per piece of kPeerPiece floats (a multiple of 4) of each (rank, column) row,
    // at most 4 CTAs per SM: a one-column gather spreads over many SMs
    const int64_t pieces = (int64_t)(skip_self ? pv.G - 1 : pv.G) * N * ((m_loc + kPeerPiece - 1) / kPeerPiece);
    const int gw = (int)std::max<int64_t>(1, std::min<int64_t>(pieces, (int64_t)sm_count * 4));
    MLZC_CUDA_TRY(launch_pdl(peer_wait_kernel, dim3(gw), dim3(256), 0, s, pv, N, m_loc, y, y_cs, err, skip_self ? 1 : 0));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return MLZC_OK;
}

int launch_peer_allgather(const PeerView& pv, const float* slice, int N, int m_loc, float* y, size_t y_cs,
                          unsigned int* err, int sm_count, cudaStream_t s) {
    const size_t chunks = pv.slice_stride / 16;
    const int gp = (int)std::max<size_t>(1, std::min<size_t>((chunks + 255) / 256, (size_t)sm_count));
    MLZC_CUDA_TRY(launch_pdl(peer_push_kernel, dim3(gp), dim3(256), 0, s, reinterpret_cast<const uint4*>(slice), chunks, pv));
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    return launch_peer_wait(pv, N, m_loc, y, y_cs, err, sm_count, s);
}

}  // namespace mlzc
