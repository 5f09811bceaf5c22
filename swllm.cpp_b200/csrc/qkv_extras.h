// qkv_extras.h -- launcher of the q/k/v bias adds and per-head q/k RMSNorm
// (qkv_extras.cu).  Any of the bias / norm pointers may be null; the caller
// (api.cu) checks the sizes.
#pragma once

#include <cuda_runtime.h>

namespace swq {

cudaError_t qkv_extras_launch(float* q, float* k, float* v, const float* bq, const float* bk, const float* bv,
                              const float* q_norm, const float* k_norm, int q_dim, int kv_dim, int head_dim,
                              float eps, int rows, int ldq, int ldk, int ldv, cudaStream_t s);

}  // namespace swq
