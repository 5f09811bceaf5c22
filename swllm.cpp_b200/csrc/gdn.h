// gdn.h -- internal interface of the GatedDeltaNet decode step (host side).
#pragma once

#include <cuda_runtime.h>

namespace swq {

cudaError_t gdn_step_launch(const float* qkv, int ld_qkv, const float* z, const float* beta, const float* alpha,
                            const float* dt, const float* a, const float* conv_w, const float* norm_w, float* S,
                            float* conv, float* y, int rows, int n_k, int n_v, int k_hd, int v_hd, int cw,
                            cudaStream_t s);
int gdn_max_head_dim();

}  // namespace swq
