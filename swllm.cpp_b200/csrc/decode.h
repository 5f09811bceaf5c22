// decode.h -- launchers of the decode-step kernels (decode.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace swq {

// out = rmsnorm(x) per row; with y (not null) x += y first, in place.
cudaError_t rmsnorm_launch(float* out, float* x, const float* y, const float* w, int n, float eps, int rows,
                           cudaStream_t s);
cudaError_t rope_kv_launch(float* q, const float* k, const float* v, float* kcache, float* vcache, const int* pos,
                           const float* freqs, int q_dim, int kv_dim, int head_dim, int rope_dim, int neox, int rows,
                           int max_seq, int ldq, int ldk, int ldv, int num_sms, cudaStream_t s);
// Context splits of attention_launch for `rows` sequences.
int attention_splits(int rows, int num_kv_heads, int max_seq, int num_sms);
// Workspace bytes: per-split partials plus one completion counter per
// (sequence, kv head); zero-filled before first use, left zeroed by every call.
size_t attention_workspace(int num_heads, int num_kv_heads, int head_dim, int rows, int splits);
cudaError_t attention_launch(float* out, const float* q, const float* kcache, const float* vcache, const int* pos,
                             void* workspace, int num_heads, int num_kv_heads, int head_dim, int rows, int max_seq,
                             int splits, int ldq, cudaStream_t s);
cudaError_t silu_mul_launch(float* out, const float* gate, const float* up, int n, int rows, int ld, int num_sms,
                            cudaStream_t s);
cudaError_t add_launch(float* x, const float* y, int64_t n, int num_sms, cudaStream_t s);
cudaError_t embed_launch(float* x, const float* table, const int* tokens, int dim, int vocab, int rows,
                         cudaStream_t s);
cudaError_t argmax_launch(const float* logits, int n, int rows, int* tokens, int* history, const int* step,
                          cudaStream_t s);
cudaError_t advance_launch(int* pos, int* step, cudaStream_t s);

}  // namespace swq
