// peer.h -- layout of the symmetric exchange region of the peer-memory all-gather (peer.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace mlzc {

constexpr int kPeerMaxRanks = 16;
constexpr size_t kPeerHeaderBytes = 4096;

// Start of every rank's exchange region: the epoch flags released by the ranks' wait
// kernels (flag[parity][rank] = the epoch of that rank's last slice of that parity) and
// this rank's own counters.
struct PeerHeader {
    uint32_t flag[2][kPeerMaxRanks];
    uint32_t epoch;        // last completed epoch (advanced by the wait kernel)
    uint32_t wait_done;    // CTAs of the current wait kernel that finished
};
static_assert(sizeof(PeerHeader) <= kPeerHeaderBytes, "header");

// Kernel-side view of the exchange: every rank's region (this process's mapping), the
// slot size of one parity and the per-rank slice stride inside a slot.
struct PeerView {
    char* base[kPeerMaxRanks];
    int G, rank;
    size_t slot_bytes;
    size_t slice_stride;   // bytes, a multiple of 16 >= N * m_loc * 4
};

// Pushes `slice` ([N][m_loc] f32, slice_stride bytes incl. padding) to every rank and
// gathers all slices into y ([N][G * m_loc], column stride y_cs) on stream s.
int launch_peer_allgather(const PeerView& pv, const float* slice, int N, int m_loc, float* y, size_t y_cs,
                          unsigned int* err, int sm_count, cudaStream_t s);
// The wait and copy half alone, after a kernel that stored this rank's slice into every
// rank's slot itself (the push kernel, or the fused decode GEMV), or into the other ranks'
// slots and its own rows of Y (the fused GEMM: skip_self); it first releases this rank's
// flag on every rank.
int launch_peer_wait(const PeerView& pv, int N, int m_loc, float* y, size_t y_cs, unsigned int* err, int sm_count,
                     cudaStream_t s, bool skip_self = false);

#ifdef __CUDACC__
// Epoch of the call in flight, read by every CTA of the kernels of one call.
__device__ __forceinline__ uint32_t peer_epoch(const PeerView& pv) {
    return *reinterpret_cast<const volatile uint32_t*>(&reinterpret_cast<const PeerHeader*>(pv.base[pv.rank])->epoch) + 1;
}
// Byte offset, inside any rank's region, of this rank's slice in the slot of epoch e.
__device__ __forceinline__ size_t peer_slice_offset(const PeerView& pv, uint32_t e) {
    return kPeerHeaderBytes + (size_t)(e & 1) * pv.slot_bytes + (size_t)pv.rank * pv.slice_stride;
}
#endif

// Decode GEMV (one activation column, F16 weights) that stores every output row into this
// rank's rows of Y (y_own) and into every other rank's slot (gemv.cu); MLZC_ERR_UNSUPPORTED
// when the operands do not fit its vectorised form (the caller then takes the slice + push
// path).
int launch_gemv_f16_peer(const void* w, size_t w_row_bytes, int64_t M, int64_t K, const float* x,
                         const PeerView& pv, float* y_own, cudaStream_t s);

}  // namespace mlzc
