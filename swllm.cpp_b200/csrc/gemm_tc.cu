// gemm_tc.cu -- tensor-core dequant-GEMM (tcgen05) for prefill-sized M.
#include <cuda_runtime.h>

#include "gemm_tc.h"
#include "swq_device.cuh"

namespace swq {

bool gemm_tc_supported(int, int, int, int) { return false; }

cudaError_t gemm_tc_launch(int, const void*, const float*, float*, int, int, int, int, int, cudaStream_t) {
    return cudaErrorNotSupported;
}

SWQ_DEFINE_STATUS_FETCH(gemm_tc)

}  // namespace swq
