// peer.h -- layout of the symmetric exchange region of the peer-memory all-gather (peer.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace mlzc {

constexpr int kPeerMaxRanks = 16;
constexpr size_t kPeerHeaderBytes = 4096;

// Start of every rank's exchange region: the epoch flags written by the ranks' push
// kernels (flag[parity][rank] = epoch of that rank's last push of that parity) and this
// rank's own counters.
struct PeerHeader {
    uint32_t flag[2][kPeerMaxRanks];
    uint32_t epoch;        // last completed epoch (advanced by the wait kernel)
    uint32_t push_done;    // CTAs of the current push kernel that finished their stores
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

}  // namespace mlzc
