// prefill.h -- launchers of the prefill kernels (prefill.cu).  Rows m = s *
// seq_len + p of the activation buffers are token p of sequence s, at
// position pos0 + p.  The callers check every size (api.cu).
#pragma once

#include <cuda_runtime.h>

namespace swq {

cudaError_t rope_kv_prefill_launch(float* q, const float* k, const float* v, float* kcache, float* vcache, int pos0,
                                   int seq_len, const float* freqs, int q_dim, int kv_dim, int head_dim,
                                   int rope_dim, int neox, int rows, int max_seq, int ldq, int ldk, int ldv,
                                   cudaStream_t s);
// head_dim 32, 64, 128 or 256.
cudaError_t attention_prefill_launch(float* out, const float* q, const float* kcache, const float* vcache, int pos0,
                                     int seq_len, int rows, int num_heads, int num_kv_heads, int head_dim,
                                     int max_seq, int ldq, int ldo, cudaStream_t s, int form = 3);
// form: 3 = tensor cores on K/V converted to fp16 pairs once per call (scratch from
// libswq's pool), 2 = tensor cores converting each tile (fp16 operand pairs), 1 = the fp32
// tiled CUDA-core form, 0 = one warp per row and head (other head dims always)

}  // namespace swq
