// selftest.cu -- exercises the failure path every kernel's bounded waits share, without
// a fault: a kernel waits on an mbarrier that nothing ever arrives on, through the same
// ptx::mbar_wait_slow the GEMM, flash-attention and Q4_K ring kernels use, with a short
// limit.  The wait gives up, sets MLZC_DEVERR_WAIT_TIMEOUT in the device error word and
// the kernel returns normally, so the context stays usable.
#include "ptx.cuh"

namespace mlzc {
namespace {

__global__ void wait_selftest_kernel(unsigned int* err, uint64_t limit_ns, int* state) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        ptx::mbar_init(ptx::smem_u32(&bar), 1);   // one arrival completes phase 0 -- none comes
        abort_flag = 0;
        ptx::mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool done = ptx::mbar_wait_slow(ptx::smem_u32(&bar), 0, &abort_flag, err, limit_ns);
        *state = done ? 1 : 2;
    }
}

}  // namespace
}  // namespace mlzc

using namespace mlzc;

extern "C" int mlzc_selftest_wait_timeout(int device, uint32_t limit_us, int* out_gave_up) {
    if (!out_gave_up) return fail(MLZC_ERR_INVALID, "null out_gave_up");
    *out_gave_up = 0;
    if (limit_us == 0 || limit_us > 2000000u) return fail(MLZC_ERR_INVALID, "limit_us %u (1 .. 2000000)", limit_us);
    DeviceCtx* c = device_ctx(device);
    if (!c) return MLZC_ERR_CUDA;
    int prev = 0;
    cudaGetDevice(&prev);
    MLZC_CUDA_TRY(cudaSetDevice(device));
    int* state = nullptr;
    int host_state = 0;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&state), sizeof(int), c->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(state, 0, sizeof(int), c->stream);
    if (e == cudaSuccess) {
        wait_selftest_kernel<<<1, 32, 0, c->stream>>>(c->err, (uint64_t)limit_us * 1000ull, state);
        e = cudaGetLastError();
        count_launch();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(&host_state, state, sizeof(int), cudaMemcpyDeviceToHost, c->stream);
    if (state) cudaFreeAsync(state, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "mlzc_selftest_wait_timeout");
    if (host_state == 0) return fail(MLZC_ERR_DEVICE, "self-test kernel did not report");
    *out_gave_up = host_state == 2 ? 1 : 0;
    return MLZC_OK;
}
