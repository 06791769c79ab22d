// fa_decode.cu -- flash-attention decode over an F16 KV cache.
//
// Replaces the F16 branch of flash_attn_dispatch (src/simd/flash_attention.cpp:143-150):
// simd_flash_attn_f16_avx512 = the FA2 skeleton (kernels/x86/flash/
// flash_attn_fa2_skeleton_avx512.inc:394-842) with the F16 macros of
// flash_attn_f16_avx512.asm:46-82.  The reference gives every (query, head, batch) work
// item to one CPU thread and walks its keys in tiles of 64 with an online softmax.
//
// GPU design (HBM-bound: every K/V byte is read once):
//   - Grouped-query packing: the G = n_head_q / n_head_kv query heads (times n_queries)
//     that share a KV head are one "row group"; a CTA serves RG of those rows, so each
//     K/V row is read once for all of them.
//   - Split-K ("flash decoding"): the keys of a sequence are cut into chunks of
//     kChunk positions, one CTA per (chunk, row group, kv head, sequence); chunks past a
//     sequence's kv_len exit at once, so a ragged batch costs only its real keys.
//   - Inside a CTA each warp runs its own online softmax over every 4th group of 4 keys:
//     8 lanes per key, each lane holding D/8 query dims (pre-scaled) and D/8 output dims
//     in registers; scores are reduced over the 8 lanes with shuffles, K/V rows are
//     loaded as 16-byte vectors one step ahead of their use.
//   - The 4 warps' (max, sum, O) states merge in shared memory; a CTA then writes its
//     partial (max, sum, unnormalised O) to the workspace, and the combine kernel merges
//     the chunks of each row.  With a single chunk the CTA writes the final row itself.
// Score order (flash_attention.cpp:339-363): s = <q*scale, k>, + mask, softcap, + ALiBi.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "internal.h"

namespace mlzc {
namespace {

constexpr int kFaWarps = 4;
constexpr int kFaThreads = kFaWarps * 32;
constexpr int kLanesPerKey = 8;
constexpr int kKeysPerWarpStep = 32 / kLanesPerKey;             // 4
constexpr int kKeysPerCtaStep = kKeysPerWarpStep * kFaWarps;    // 16
constexpr int kChunk = 256;                                     // keys per CTA

struct FaParams {
    const char* q;
    const char* k;
    const char* v;
    const char* mask;
    char* dst;
    float* part;                 // workspace partials, or nullptr when nsplit == 1
    const int32_t* kv_len;
    int64_t q_nb1, q_nb2, q_nb3;
    int64_t k_nb1, k_nb2, k_nb3;
    int64_t v_nb1, v_nb2, v_nb3;
    int64_t m_nb0, m_nb1, m_nb2, m_nb3;
    int64_t d_nb1, d_nb2, d_nb3;
    int n_kv, n_q, n_head_q, n_head_kv;
    int G;                       // query heads per row group
    int rows_total;              // G * n_q
    int n_rgroups;               // ceil(rows_total / RG)
    int nsplit;
    int packed;                  // 1: grid.y walks kv heads; 0: grid.y walks query heads
    float scale, softcap, alibi_p2inv;  // alibi_p2inv = -8 / P (0 = no ALiBi)
    int use_softcap;
};

__device__ __forceinline__ void f16x8_to_f32(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 ld_kv16(const char* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

// Row r of a row group -> (query position, query head).
__device__ __forceinline__ void row_coords(const FaParams& p, int head_base, int r, int& iq, int& ihq) {
    iq = r / p.G;
    ihq = head_base + r % p.G;
}

template <int D, int RG>
__global__ void __launch_bounds__(kFaThreads)
fa_decode_kernel(FaParams p) {
    constexpr int DL = D / kLanesPerKey;      // dims per lane
    constexpr int NV = DL / 8;                // 16-byte vectors per lane per row
    static_assert(DL % 8 == 0, "D must be a multiple of 64");

    const int split = blockIdx.x;
    const int rg = blockIdx.y % p.n_rgroups;
    const int hidx = blockIdx.y / p.n_rgroups;
    const int ib = blockIdx.z;
    const int kvh = p.packed ? hidx : (int)((int64_t)hidx * p.n_head_kv / p.n_head_q);
    const int head_base = p.packed ? hidx * p.G : hidx;

    const int L = p.kv_len ? min(p.kv_len[ib], p.n_kv) : p.n_kv;
    const int k0 = split * kChunk;
    const int k1 = min(k0 + kChunk, L);

    if (k0 >= L && p.nsplit > 1) return;   // chunk past this sequence's keys: no record

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int sub = lane & (kLanesPerKey - 1);    // dims [sub*DL, sub*DL + DL)
    const int kslot = lane / kLanesPerKey;        // which of the warp's 4 keys

    // rows of this CTA
    int iq_r[RG], ihq_r[RG];
    bool valid[RG];
#pragma unroll
    for (int r = 0; r < RG; r++) {
        const int row = rg * RG + r;
        valid[r] = row < p.rows_total;
        row_coords(p, head_base, valid[r] ? row : 0, iq_r[r], ihq_r[r]);
    }

    // query slice in registers, pre-scaled
    float qv[RG][DL];
#pragma unroll
    for (int r = 0; r < RG; r++) {
        const float* qr = reinterpret_cast<const float*>(p.q + iq_r[r] * p.q_nb1 + ihq_r[r] * p.q_nb2 + ib * p.q_nb3);
#pragma unroll
        for (int i = 0; i < DL; i += 4) {
            const float4 t = *reinterpret_cast<const float4*>(qr + sub * DL + i);
            qv[r][i] = t.x * p.scale; qv[r][i + 1] = t.y * p.scale;
            qv[r][i + 2] = t.z * p.scale; qv[r][i + 3] = t.w * p.scale;
        }
    }
    float slope[RG];
#pragma unroll
    for (int r = 0; r < RG; r++) slope[r] = p.alibi_p2inv != 0.0f ? exp2f(p.alibi_p2inv * (float)(ihq_r[r] + 1)) : 0.0f;

    float m[RG], l[RG], o[RG][DL];
#pragma unroll
    for (int r = 0; r < RG; r++) {
        m[r] = -INFINITY;
        l[r] = 0.0f;
#pragma unroll
        for (int i = 0; i < DL; i++) o[r][i] = 0.0f;
    }

    const char* kbase = p.k + kvh * p.k_nb2 + ib * p.k_nb3 + sub * DL * 2;
    const char* vbase = p.v + kvh * p.v_nb2 + ib * p.v_nb3 + sub * DL * 2;

    // key handled by this lane at step t: k0 + t*16 + warp*4 + kslot
    int j = k0 + warp * kKeysPerWarpStep + kslot;
    uint4 kn[NV], vn[NV];
#pragma unroll
    for (int u = 0; u < NV; u++) { kn[u] = make_uint4(0, 0, 0, 0); vn[u] = kn[u]; }
    if (j < k1) {
#pragma unroll
        for (int u = 0; u < NV; u++) {
            kn[u] = ld_kv16(kbase + (int64_t)j * p.k_nb1 + u * 16);
            vn[u] = ld_kv16(vbase + (int64_t)j * p.v_nb1 + u * 16);
        }
    }
    for (int jb = k0 + warp * kKeysPerWarpStep; jb < k1; jb += kKeysPerCtaStep) {
        const bool live = j < k1;
        uint4 kc[NV], vc[NV];
#pragma unroll
        for (int u = 0; u < NV; u++) { kc[u] = kn[u]; vc[u] = vn[u]; }
        const int jn = j + kKeysPerCtaStep;
        if (jn < k1) {
#pragma unroll
            for (int u = 0; u < NV; u++) {
                kn[u] = ld_kv16(kbase + (int64_t)jn * p.k_nb1 + u * 16);
                vn[u] = ld_kv16(vbase + (int64_t)jn * p.v_nb1 + u * 16);
            }
        } else {
#pragma unroll
            for (int u = 0; u < NV; u++) { kn[u] = make_uint4(0, 0, 0, 0); vn[u] = kn[u]; }
        }
        // scores of this lane's key for the RG rows
        float kf[DL];
#pragma unroll
        for (int u = 0; u < NV; u++) f16x8_to_f32(kc[u], kf + 8 * u);
        float s[RG];
#pragma unroll
        for (int r = 0; r < RG; r++) {
            float a = 0.0f;
#pragma unroll
            for (int i = 0; i < DL; i++) a = fmaf(qv[r][i], kf[i], a);
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            a += __shfl_xor_sync(0xffffffffu, a, 2);
            a += __shfl_xor_sync(0xffffffffu, a, 4);
            s[r] = a;
        }
#pragma unroll
        for (int r = 0; r < RG; r++) {
            float sr = s[r];
            if (p.mask) {
                const int jj = live ? j : k0;
                sr += *reinterpret_cast<const float*>(p.mask + iq_r[r] * p.m_nb1 + (int64_t)jj * p.m_nb0 +
                                                     ihq_r[r] * p.m_nb2 + ib * p.m_nb3);
            }
            if (p.use_softcap) sr = p.softcap * tanhf(sr / p.softcap);
            if (p.alibi_p2inv != 0.0f) sr += slope[r] * (float)(j - iq_r[r]);
            s[r] = live ? sr : -INFINITY;
        }
        // warp-wide max over the 4 keys of the step, online rescale, accumulate PV
        float vf[DL];
#pragma unroll
        for (int u = 0; u < NV; u++) f16x8_to_f32(vc[u], vf + 8 * u);
#pragma unroll
        for (int r = 0; r < RG; r++) {
            float mx = fmaxf(s[r], __shfl_xor_sync(0xffffffffu, s[r], 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(m[r], mx);
            if (mnew == -INFINITY) continue;          // nothing visible yet (warp-uniform)
            if (mnew > m[r]) {                        // warp-uniform branch
                const float corr = __expf(m[r] - mnew);
                l[r] *= corr;
#pragma unroll
                for (int i = 0; i < DL; i++) o[r][i] *= corr;
                m[r] = mnew;
            }
            const float pr = __expf(s[r] - mnew);
            l[r] += pr;
#pragma unroll
            for (int i = 0; i < DL; i++) o[r][i] = fmaf(pr, vf[i], o[r][i]);
        }
        j = jn;
    }

    // merge the 4 key slots of the warp (same m within a warp; sum l and o)
#pragma unroll
    for (int r = 0; r < RG; r++) {
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 8);
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 16);
#pragma unroll
        for (int i = 0; i < DL; i++) {
            o[r][i] += __shfl_xor_sync(0xffffffffu, o[r][i], 8);
            o[r][i] += __shfl_xor_sync(0xffffffffu, o[r][i], 16);
        }
    }

    // merge the warps through shared memory
    __shared__ float sm_m[kFaWarps][RG], sm_l[kFaWarps][RG];
    __shared__ float sm_o[kFaWarps][RG][D];
    if (lane < kLanesPerKey) {
#pragma unroll
        for (int r = 0; r < RG; r++) {
#pragma unroll
            for (int i = 0; i < DL; i++) sm_o[warp][r][sub * DL + i] = o[r][i];
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < RG; r++) { sm_m[warp][r] = m[r]; sm_l[warp][r] = l[r]; }
    }
    __syncthreads();

    const int rows_here = RG;
    for (int idx = threadIdx.x; idx < rows_here * D; idx += kFaThreads) {
        const int r = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kFaWarps; w++) M = fmaxf(M, sm_m[w][r]);
        float Ls = 0.0f, Os = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kFaWarps; w++) {
                const float e = __expf(sm_m[w][r] - M);
                Ls += sm_l[w][r] * e;
                Os += sm_o[w][r][d] * e;
            }
        }
        const int row = rg * RG + r;
        if (row >= p.rows_total) continue;
        int iq, ihq;
        row_coords(p, head_base, row, iq, ihq);
        if (p.nsplit == 1) {
            float* dr = reinterpret_cast<float*>(p.dst + iq * p.d_nb1 + ihq * p.d_nb2 + ib * p.d_nb3);
            dr[d] = Ls > 0.0f ? Os / Ls : 0.0f;
        } else {
            // partial record: [m, l, o[0..D)] per (ib, hidx, row, split)
            const int64_t n_hidx = gridDim.y / p.n_rgroups;
            const int64_t rec = (((int64_t)ib * n_hidx + hidx) * p.rows_total + row) * p.nsplit + split;
            float* pr = p.part + rec * (D + 2);
            if (d == 0) { pr[0] = M; pr[1] = Ls; }
            pr[2 + d] = Os;
        }
    }
}

// Merges the chunk partials of every (sequence, head index, row): one CTA per row.
template <int D>
__global__ void __launch_bounds__(D)
fa_combine_kernel(FaParams p, int n_hidx) {
    const int row = blockIdx.x;
    const int hidx = blockIdx.y;
    const int ib = blockIdx.z;
    const int d = threadIdx.x;
    const int64_t rec0 = (((int64_t)ib * n_hidx + hidx) * p.rows_total + row) * p.nsplit;
    const float* base = p.part + rec0 * (D + 2);
    const int L = p.kv_len ? min(p.kv_len[ib], p.n_kv) : p.n_kv;
    const int used = min(p.nsplit, (L + kChunk - 1) / kChunk);
    float M = -INFINITY;
    for (int s = 0; s < used; s++) M = fmaxf(M, base[(int64_t)s * (D + 2)]);
    float Ls = 0.0f, Os = 0.0f;
    if (M != -INFINITY) {
        for (int s = 0; s < used; s++) {
            const float* pr = base + (int64_t)s * (D + 2);
            const float e = __expf(pr[0] - M);
            Ls += pr[1] * e;
            Os += pr[2 + d] * e;
        }
    }
    const int head_base = p.packed ? hidx * p.G : hidx;
    int iq, ihq;
    row_coords(p, head_base, row, iq, ihq);
    float* dr = reinterpret_cast<float*>(p.dst + iq * p.d_nb1 + ihq * p.d_nb2 + ib * p.d_nb3);
    dr[d] = Ls > 0.0f ? Os / Ls : 0.0f;
}

struct FaPlan {
    FaParams p;
    int RG;
    int n_hidx;
    dim3 grid;
    size_t ws_bytes;
};

FaPlan make_plan(const mlzc_fa_desc* d) {
    FaPlan pl{};
    FaParams& p = pl.p;
    const int Hq = (int)d->n_head_q, Hkv = (int)d->n_head_kv;
    p.packed = (Hq % Hkv == 0) ? 1 : 0;
    p.G = p.packed ? Hq / Hkv : 1;
    p.n_q = (int)d->n_queries;
    p.rows_total = p.G * p.n_q;
    pl.RG = p.rows_total >= 4 ? 4 : (p.rows_total >= 2 ? 2 : 1);
    p.n_rgroups = (p.rows_total + pl.RG - 1) / pl.RG;
    p.n_kv = (int)d->n_kv;
    p.n_head_q = Hq;
    p.n_head_kv = Hkv;
    p.nsplit = std::max(1, (p.n_kv + kChunk - 1) / kChunk);
    pl.n_hidx = p.packed ? Hkv : Hq;
    pl.grid = dim3((unsigned)p.nsplit, (unsigned)(p.n_rgroups * pl.n_hidx), (unsigned)d->batch_size);
    const int64_t D = d->head_dim_v;
    pl.ws_bytes = p.nsplit > 1
        ? (size_t)d->batch_size * pl.n_hidx * p.rows_total * p.nsplit * (D + 2) * sizeof(float)
        : 0;
    return pl;
}

}  // namespace

size_t fa_workspace_bytes(const mlzc_fa_desc* d) { return make_plan(d).ws_bytes; }

int launch_flash_attn(const DeviceCtx*, const mlzc_fa_desc* d, void* ws, size_t ws_bytes,
                      cudaStream_t s) {
    FaPlan pl = make_plan(d);
    if (pl.ws_bytes > ws_bytes || (pl.ws_bytes && !ws))
        return fail(MLZC_ERR_NOMEM, "flash_attn: workspace of %zu bytes needed, %zu given", pl.ws_bytes, ws_bytes);
    FaParams& p = pl.p;
    p.q = reinterpret_cast<const char*>(d->q);
    p.k = static_cast<const char*>(d->k);
    p.v = static_cast<const char*>(d->v);
    p.mask = reinterpret_cast<const char*>(d->mask);
    p.dst = reinterpret_cast<char*>(d->dst);
    p.part = static_cast<float*>(ws);
    p.kv_len = d->kv_len;
    p.q_nb1 = d->q_nb[1]; p.q_nb2 = d->q_nb[2]; p.q_nb3 = d->q_nb[3];
    p.k_nb1 = d->k_nb[1]; p.k_nb2 = d->k_nb[2]; p.k_nb3 = d->k_nb[3];
    p.v_nb1 = d->v_nb[1]; p.v_nb2 = d->v_nb[2]; p.v_nb3 = d->v_nb[3];
    p.m_nb0 = d->mask_nb[0]; p.m_nb1 = d->mask_nb[1]; p.m_nb2 = d->mask_nb[2]; p.m_nb3 = d->mask_nb[3];
    p.d_nb1 = d->dst_nb[1]; p.d_nb2 = d->dst_nb[2]; p.d_nb3 = d->dst_nb[3];
    p.scale = d->scale;
    p.use_softcap = (d->mode & MLZC_FA_MODE_SOFTCAP) && d->logit_softcap != 0.0f;
    p.softcap = d->logit_softcap;
    if (d->mode & MLZC_FA_MODE_ALIBI) {
        int p2 = 1;
        while (p2 < p.n_head_q) p2 <<= 1;
        p.alibi_p2inv = -8.0f / (float)p2;
    } else {
        p.alibi_p2inv = 0.0f;
    }
    const int D = (int)d->head_dim_k;
#define MLZC_FA_LAUNCH(DD, RGV) fa_decode_kernel<DD, RGV><<<pl.grid, kFaThreads, 0, s>>>(p)
#define MLZC_FA_RG(DD)                                  \
    do {                                                \
        if (pl.RG == 4) MLZC_FA_LAUNCH(DD, 4);          \
        else if (pl.RG == 2) MLZC_FA_LAUNCH(DD, 2);     \
        else MLZC_FA_LAUNCH(DD, 1);                     \
    } while (0)
    if (D == 64) MLZC_FA_RG(64);
    else if (D == 128) MLZC_FA_RG(128);
    else if (D == 256) MLZC_FA_RG(256);
    else return fail(MLZC_ERR_UNSUPPORTED, "flash_attn: head_dim %d (64, 128, 256 supported)", D);
#undef MLZC_FA_RG
#undef MLZC_FA_LAUNCH
    MLZC_CUDA_TRY(cudaGetLastError());
    count_launch();
    if (p.nsplit > 1) {
        const dim3 g((unsigned)p.rows_total, (unsigned)pl.n_hidx, (unsigned)d->batch_size);
        if (D == 64) fa_combine_kernel<64><<<g, 64, 0, s>>>(p, pl.n_hidx);
        else if (D == 128) fa_combine_kernel<128><<<g, 128, 0, s>>>(p, pl.n_hidx);
        else fa_combine_kernel<256><<<g, 256, 0, s>>>(p, pl.n_hidx);
        MLZC_CUDA_TRY(cudaGetLastError());
        count_launch();
    }
    return MLZC_OK;
}

}  // namespace mlzc

// ======================================================================
// Allocation-free flash-attention decode (mlzc_flash_attn_dev_noalloc).
//
// Some callers cannot allocate device memory for each call: code that runs where a
// cudaMalloc would synchronise the device or be refused (a host callback, a thread that
// must never block behind other streams, an engine whose memory is fully budgeted up
// front), or a binding that simply has no allocator to hand us a workspace.  For them
// this variant keeps the split-K partials of the decode kernel in one fixed scratch
// array that lives in the library's device image instead of a caller workspace.
//
// The array is a file-scope __device__ variable, so every GPU that loads this library
// holds kNoAllocScratchBytes of it until the process exits, whether or not the entry
// point is used.  Host code cannot use the array's name as a device address (on the host
// it names a stand-in object), so the device address is looked up with
// cudaGetSymbolAddress -- once per device, on the first call made while that device is
// current, and cached.  That first call therefore does the set-up; make it before any
// stream capture.
//
// Every call shares the one array and it keeps whatever the previous call left in it.
// Nothing in it has to start at zero: each call writes every partial record it later
// reads.  Calls whose kernels overlap on the GPU (on different streams, or from several
// host threads) race on the array and corrupt each other's results; serialise them.
// ======================================================================
namespace mlzc {
namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;   // 16 MiB per device
static __device__ __align__(256) float g_fa_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};

}  // namespace
}  // namespace mlzc

extern "C" int mlzc_flash_attn_dev_noalloc(const mlzc_fa_desc* desc, void* stream) {
    using namespace mlzc;
    int st = check_fa_args(desc);
    if (st != MLZC_OK) return st;
    const size_t need = fa_workspace_bytes(desc);
    if (need > kNoAllocScratchBytes)
        return fail(MLZC_ERR_NOMEM,
                    "flash_attn (allocation-free): this call needs %zu bytes of split scratch but the fixed "
                    "scratch holds %zu; use mlzc_flash_attn_dev with a workspace",
                    need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    if (need > 0) {
        int dev = 0;
        MLZC_CUDA_TRY(cudaGetDevice(&dev));
        if (dev < 0 || dev >= kNoAllocMaxDevices)
            return fail(MLZC_ERR_INVALID, "flash_attn (allocation-free): device %d beyond %d", dev, kNoAllocMaxDevices);
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_addr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_fa_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(flash-attention scratch)");
            g_noalloc_addr[dev] = p;
        }
        scratch = g_noalloc_addr[dev];
    }
    return launch_flash_attn(nullptr, desc, scratch, kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
}
