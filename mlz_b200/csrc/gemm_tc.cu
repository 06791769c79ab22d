// gemm_tc.cu -- tensor-core (tcgen05 / TMEM) GEMM for F16 weights.  Placeholder until
// the kernel lands: reports "not applicable" so every F16 shape takes the CUDA-core path.
#include "internal.h"

namespace mlzc {

size_t gemm_f16_workspace_bytes(int64_t, int64_t, int64_t) { return 0; }

bool gemm_f16_applicable(int64_t, int64_t, int64_t, const void*, size_t, const float*, size_t,
                         const float*, size_t) {
    return false;
}

int launch_gemm_f16(const DeviceCtx*, const void*, size_t, int64_t, int64_t, const float*, size_t,
                    int64_t, float*, size_t, void*, size_t, cudaStream_t) {
    return fail(MLZC_ERR_UNSUPPORTED, "tensor-core GEMM not built");
}

}  // namespace mlzc
