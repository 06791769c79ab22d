// comm.cpp -- row-sharded mul_mat over the GPUs of one node (one process per GPU).
//
// The reference has no multi-GPU path (its only parallelism is the ggml CPU threadpool).
// A weight matrix that splits by rows is sharded so that rank r holds rows
// [r*M/G, (r+1)*M/G); every rank computes its slice of Y with the single-GPU kernels and
// an NCCL all-gather over NVLink assembles the full Y on every rank.
//
// NCCL is resolved at run time with dlopen: a process that already loaded an NCCL (for
// instance through torch.distributed) keeps using that one, and the rest of the library
// has no NCCL dependency at all.  Communicators are created non-blocking and every host
// wait on them is bounded by the caller's timeout, after which the communicator is aborted
// and MLZC_ERR_COMM returned.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <algorithm>
#include <vector>
#include <cstring>
#include <mutex>
#include <thread>

#include "internal.h"
#include "peer.h"

namespace mlzc {
namespace {

struct NcclApi {
    void* handle = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

std::once_flag g_nccl_once;
NcclApi g_nccl;

template <class T>
void sym(void* h, const char* name, T& fn) {
    fn = reinterpret_cast<T>(dlsym(h, name));
}

const NcclApi* nccl() {
    std::call_once(g_nccl_once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        g_nccl.handle = h;
        sym(h, "ncclGetUniqueId", g_nccl.GetUniqueId);
        sym(h, "ncclCommInitRankConfig", g_nccl.CommInitRankConfig);
        sym(h, "ncclCommDestroy", g_nccl.CommDestroy);
        sym(h, "ncclCommAbort", g_nccl.CommAbort);
        sym(h, "ncclCommGetAsyncError", g_nccl.CommGetAsyncError);
        sym(h, "ncclAllGather", g_nccl.AllGather);
        sym(h, "ncclAllReduce", g_nccl.AllReduce);
        sym(h, "ncclGetErrorString", g_nccl.GetErrorString);
        g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRankConfig && g_nccl.CommDestroy && g_nccl.CommAbort &&
                    g_nccl.CommGetAsyncError && g_nccl.AllGather && g_nccl.AllReduce && g_nccl.GetErrorString;
    });
    return g_nccl.ok ? &g_nccl : nullptr;
}

int nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
    return fail(MLZC_ERR_COMM, "%s: %s", what, api ? api->GetErrorString(r) : "NCCL unavailable");
}

}  // namespace
}  // namespace mlzc

using namespace mlzc;

struct mlzc_comm_s {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0;
    int timeout_ms = 0;
    bool broken = false;
    // peer-memory all-gather (peer.cu): this rank's exchange region and every rank's, as
    // mapped in this process (peer regions opened from their CUDA IPC handles)
    bool peer_ok = false;
    void* region = nullptr;
    char* base[mlzc::kPeerMaxRanks] = {};
    size_t slot_bytes = 0;
};

namespace {

// Polls a non-blocking communicator until its pending operation leaves ncclInProgress:
// spinning for the first 100 us (an enqueue normally completes within microseconds), then
// sleeping 50 us between polls, bounded by the communicator's timeout.
int wait_comm(const NcclApi* api, mlzc_comm c, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = api->CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) { c->broken = true; return nccl_fail(api, r, what); }
        if (st == ncclSuccess) return MLZC_OK;
        if (st != ncclInProgress) { c->broken = true; return nccl_fail(api, st, what); }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (c->timeout_ms > 0 && ms > c->timeout_ms) {
            c->broken = true;
            api->CommAbort(c->comm);
            c->comm = nullptr;
            return fail(MLZC_ERR_COMM, "%s: no progress within %d ms; communicator aborted", what, c->timeout_ms);
        }
        const auto us = std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
        if (us > 100) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

namespace {

// Enqueue-and-wait helpers for the set-up collectives (non-blocking communicator).
int enq_done(const NcclApi* api, mlzc_comm c, ncclResult_t r, const char* what) {
    if (r != ncclSuccess && r != ncclInProgress) {
        c->broken = true;
        return nccl_fail(api, r, what);
    }
    return r == ncclInProgress ? wait_comm(api, c, what) : MLZC_OK;
}

void peer_release(mlzc_comm c) {
    for (int r = 0; r < c->nranks && r < kPeerMaxRanks; ++r)
        if (r != c->rank && c->base[r]) cudaIpcCloseMemHandle(c->base[r]);
    if (c->region) cudaFree(c->region);
    c->region = nullptr;
    for (auto& b : c->base) b = nullptr;
    c->peer_ok = false;
}

// Symmetric exchange region for the peer-memory all-gather: allocated here, its CUDA IPC
// handle all-gathered over the communicator, every peer's region opened (peer access over
// NVLink), and the outcome agreed on by all ranks (an all-reduce of the local result), so
// every rank takes the same gather path.  MLZ_SHARDED_GATHER=nccl keeps NCCL's all-gather;
// MLZ_PEER_SLOT_MB sets the slot size (64 MB per parity by default).
int peer_setup(const NcclApi* api, mlzc_comm c) {
    const char* mode = getenv("MLZ_SHARDED_GATHER");
    if ((mode && std::strcmp(mode, "nccl") == 0) || c->nranks > kPeerMaxRanks) return MLZC_OK;   // same on every rank
    const char* mb = getenv("MLZ_PEER_SLOT_MB");
    c->slot_bytes = (size_t)(mb ? std::max(1, atoi(mb)) : 64) << 20;
    cudaStream_t s = nullptr;
    MLZC_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    int local_ok = 1;
    cudaIpcMemHandle_t mine{};
    if (cudaMalloc(&c->region, kPeerHeaderBytes + 2 * c->slot_bytes) != cudaSuccess ||
        cudaMemset(c->region, 0, kPeerHeaderBytes) != cudaSuccess || cudaIpcGetMemHandle(&mine, c->region) != cudaSuccess) {
        cudaGetLastError();
        local_ok = 0;
    }
    // handles of all ranks (64 bytes each) through a device buffer
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    char* dh = nullptr;
    int* dflag = nullptr;
    int st = MLZC_OK;
    std::vector<char> all((size_t)c->nranks * hb);
    if (cudaMalloc(&dh, hb * (size_t)(c->nranks + 1)) != cudaSuccess || cudaMalloc(&dflag, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        st = fail(MLZC_ERR_NOMEM, "peer exchange set-up: device buffers");
    }
    if (st == MLZC_OK && cudaMemcpy(dh + (size_t)c->nranks * hb, &mine, hb, cudaMemcpyHostToDevice) != cudaSuccess)
        st = fail(MLZC_ERR_CUDA, "peer exchange set-up: copy of the handle");
    if (st == MLZC_OK)
        st = enq_done(api, c, api->AllGather(dh + (size_t)c->nranks * hb, dh, hb, ncclUint8, c->comm, s), "ncclAllGather (handles)");
    if (st == MLZC_OK && (cudaStreamSynchronize(s) != cudaSuccess ||
                          cudaMemcpy(all.data(), dh, all.size(), cudaMemcpyDeviceToHost) != cudaSuccess))
        st = fail(MLZC_ERR_CUDA, "peer exchange set-up: handle read-back");
    if (st == MLZC_OK) {
        c->base[c->rank] = static_cast<char*>(c->region);
        for (int r = 0; r < c->nranks && local_ok; ++r) {
            if (r == c->rank) continue;
            cudaIpcMemHandle_t h;
            std::memcpy(&h, all.data() + (size_t)r * hb, hb);
            void* p = nullptr;
            if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                local_ok = 0;
            } else {
                c->base[r] = static_cast<char*>(p);
            }
        }
        // every rank must agree: minimum of the local outcomes
        int agreed = 0;
        if (cudaMemcpy(dflag, &local_ok, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
            st = fail(MLZC_ERR_CUDA, "peer exchange set-up: flag copy");
        if (st == MLZC_OK) st = enq_done(api, c, api->AllReduce(dflag, dflag, 1, ncclInt32, ncclMin, c->comm, s), "ncclAllReduce (peer set-up)");
        if (st == MLZC_OK && (cudaStreamSynchronize(s) != cudaSuccess ||
                              cudaMemcpy(&agreed, dflag, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess))
            st = fail(MLZC_ERR_CUDA, "peer exchange set-up: flag read-back");
        c->peer_ok = st == MLZC_OK && agreed == 1;
    }
    if (dh) cudaFree(dh);
    if (dflag) cudaFree(dflag);
    cudaStreamDestroy(s);
    if (!c->peer_ok) peer_release(c);
    return st;
}

}  // namespace

extern "C" int mlzc_comm_unique_id(void* out_id) {
    if (!out_id) return fail(MLZC_ERR_INVALID, "null id buffer");
    const NcclApi* api = nccl();
    if (!api) return fail(MLZC_ERR_COMM, "libnccl.so.2 could not be loaded");
    static_assert(sizeof(ncclUniqueId) == MLZC_UNIQUE_ID_BYTES, "unique id size");
    ncclUniqueId id;
    ncclResult_t r = api->GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(api, r, "ncclGetUniqueId");
    std::memcpy(out_id, &id, sizeof id);
    return MLZC_OK;
}

extern "C" int mlzc_comm_init(int nranks, int rank, int device, const void* unique_id, int timeout_ms,
                              mlzc_comm* out) {
    if (!out || !unique_id) return fail(MLZC_ERR_INVALID, "null argument");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(MLZC_ERR_INVALID, "rank %d of %d", rank, nranks);
    const NcclApi* api = nccl();
    if (!api) return fail(MLZC_ERR_COMM, "libnccl.so.2 could not be loaded");
    if (!device_ctx(device)) return MLZC_ERR_CUDA;
    MLZC_CUDA_TRY(cudaSetDevice(device));
    auto* c = new mlzc_comm_s;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    c->timeout_ms = timeout_ms;
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = api->CommInitRankConfig(&c->comm, nranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return nccl_fail(api, r, "ncclCommInitRankConfig");
    }
    int st = wait_comm(api, c, "ncclCommInitRankConfig");
    if (st != MLZC_OK) {
        if (c->comm) api->CommAbort(c->comm);
        delete c;
        return st;
    }
    st = peer_setup(api, c);
    if (st != MLZC_OK) {
        api->CommAbort(c->comm);
        delete c;
        return st;
    }
    *out = c;
    return MLZC_OK;
}

extern "C" int mlzc_comm_destroy(mlzc_comm c) {
    if (!c) return MLZC_OK;
    if (c->peer_ok) {
        // this rank's kernels are done with the exchange (every peer's push into this
        // region completed before this rank's last wait kernel could finish)
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(c->device);
        cudaDeviceSynchronize();
        peer_release(c);
        cudaSetDevice(prev);
    }
    const NcclApi* api = nccl();
    if (api && c->comm) {
        if (c->broken) api->CommAbort(c->comm);
        else api->CommDestroy(c->comm);
    }
    delete c;
    return MLZC_OK;
}

extern "C" int mlzc_mul_mat_sharded_workspace_bytes(mlzc_comm c, int w_type, int64_t M_total, int64_t K,
                                                    int64_t N, size_t* out_bytes) {
    if (!c || !out_bytes) return fail(MLZC_ERR_INVALID, "null argument");
    if (M_total % c->nranks) return fail(MLZC_ERR_INVALID, "M_total %lld not divisible by %d ranks", (long long)M_total, c->nranks);
    const int64_t m_loc = M_total / c->nranks;
    const size_t mm = (mul_mat_workspace(w_type, m_loc, K, N) + 255) / 256 * 256;
    const size_t slice = ((size_t)N * m_loc * 4 + 255) / 256 * 256;
    const size_t gathered = (size_t)c->nranks * N * m_loc * 4;
    *out_bytes = mm + slice + gathered;
    return MLZC_OK;
}

extern "C" int mlzc_mul_mat_sharded_dev(mlzc_comm c, int w_type, const void* w_shard, size_t w_row_bytes,
                                        int64_t M_total, int64_t K, const float* x, size_t x_col_bytes, int64_t N,
                                        float* y, size_t y_col_bytes, void* workspace, size_t workspace_bytes,
                                        void* stream) {
    if (!c || !c->comm) return fail(MLZC_ERR_COMM, "communicator missing or aborted");
    const NcclApi* api = nccl();
    if (!api) return fail(MLZC_ERR_COMM, "libnccl.so.2 could not be loaded");
    size_t need = 0;
    int st = mlzc_mul_mat_sharded_workspace_bytes(c, w_type, M_total, K, N, &need);
    if (st != MLZC_OK) return st;
    if (workspace_bytes < need || (need && !workspace))
        return fail(MLZC_ERR_NOMEM, "sharded mul_mat: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    const int64_t m_loc = M_total / c->nranks;
    st = check_mul_mat_args(w_type, w_shard, w_row_bytes, m_loc, K, x, x_col_bytes, N, y, y_col_bytes);
    if (st != MLZC_OK) return st;
    if (y_col_bytes < (size_t)M_total * 4) return fail(MLZC_ERR_INVALID, "y_col_bytes smaller than a full column");
    DeviceCtx* ctx = device_ctx(c->device);
    if (!ctx) return MLZC_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(workspace);
    const size_t mm = (mul_mat_workspace(w_type, m_loc, K, N) + 255) / 256 * 256;
    const size_t slice_bytes = ((size_t)N * m_loc * 4 + 255) / 256 * 256;
    float* slice = reinterpret_cast<float*>(ws + mm);
    float* gathered = reinterpret_cast<float*>(ws + mm + slice_bytes);
    const bool peer = c->peer_ok && (size_t)c->nranks * slice_bytes <= c->slot_bytes;
    PeerView pv{};
    if (peer) {
        for (int r = 0; r < c->nranks; ++r) pv.base[r] = c->base[r];
        pv.G = c->nranks;
        pv.rank = c->rank;
        pv.slot_bytes = c->slot_bytes;
        pv.slice_stride = slice_bytes;
        // decode (one column, F16): one kernel computes the slice and stores it into every
        // rank's slot over NVLink as it goes; then the wait-and-copy kernel
        // this rank's rows of Y
        float* y_own = reinterpret_cast<float*>(reinterpret_cast<char*>(y) + (size_t)c->rank * m_loc * 4);
        if (N == 1 && w_type == MLZC_TYPE_F16) {
            st = launch_gemv_f16_peer(w_shard, w_row_bytes, m_loc, K, x, pv, y_own, s);
            if (st == MLZC_OK)
                return launch_peer_wait(pv, (int)N, (int)m_loc, y, y_col_bytes, ctx->err, ctx->sm_count, s, true);
            if (st != MLZC_ERR_UNSUPPORTED) return st;
        }
        // prefill (the tcgen05 GEMM): its epilogue stores every finished tile into its rows of Y
        // and into this rank's slice of each other rank's slot, so the exchange overlaps the
        // remaining tiles; the wait kernel then copies only the other ranks' slices
        if (c->nranks - 1 <= 7 &&
            mul_mat_uses_gemm(w_type, m_loc, K, N, w_shard, w_row_bytes, x, x_col_bytes, y_own, y_col_bytes)) {
            GemmPeers gp{};
            gp.npeer = c->nranks - 1;
            gp.pcs = (size_t)m_loc * 4;
            gp.epoch = &reinterpret_cast<const PeerHeader*>(c->base[c->rank])->epoch;
            for (int par = 0; par < 2; ++par)
                for (int r = 0, i = 0; r < c->nranks; ++r) {
                    if (r == c->rank) continue;
                    gp.slot[par][i++] = reinterpret_cast<float*>(c->base[r] + kPeerHeaderBytes + (size_t)par * c->slot_bytes +
                                                                 (size_t)c->rank * slice_bytes);
                }
            st = launch_gemm_f16_peers(ctx, w_shard, w_row_bytes, m_loc, K, x, x_col_bytes, N, y_own, y_col_bytes, ws, mm,
                                       gp, s);
            if (st == MLZC_OK)
                return launch_peer_wait(pv, (int)N, (int)m_loc, y, y_col_bytes, ctx->err, ctx->sm_count, s, true);
            if (st != MLZC_ERR_UNSUPPORTED) return st;
        }
    }
    // This rank's slice, dense [N][m_loc].
    st = mul_mat_run(ctx, w_type, w_shard, w_row_bytes, m_loc, K, x, x_col_bytes, N, slice, (size_t)m_loc * 4,
                     ws, mm, s);
    if (st != MLZC_OK) return st;
    if (peer) return launch_peer_allgather(pv, slice, (int)N, (int)m_loc, y, y_col_bytes, ctx->err, ctx->sm_count, s);
    const bool direct = (N == 1);  // one column: slices land at their final place in y
    ncclResult_t r = api->AllGather(slice, direct ? static_cast<void*>(y) : static_cast<void*>(gathered),
                                    (size_t)N * m_loc, ncclFloat32, c->comm, s);
    if (r != ncclSuccess && r != ncclInProgress) {
        c->broken = true;
        return nccl_fail(api, r, "ncclAllGather");
    }
    // ncclInProgress: the collective may not be in the stream yet, so it must finish
    // enqueueing before anything that reads its output is launched
    if (r == ncclInProgress && (st = wait_comm(api, c, "ncclAllGather")) != MLZC_OK) return st;
    if (!direct) return launch_gather_permute(gathered, y, y_col_bytes, c->nranks, N, m_loc, s);
    return MLZC_OK;
}
