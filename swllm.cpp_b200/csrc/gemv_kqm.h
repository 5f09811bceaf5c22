// gemv_kqm.h -- Q4_K / Q6_K GEMVs of 2..32 activation rows, each weight read
// once for all rows, exact products on the tensor cores (gemv_kqm.cu): host
// interface.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "gemm_tc.h"  // ActArgs

namespace swq {

// Whether the batched K-quant GEMV serves Y[M x N] = X[M x K] . W^T (type
// Q4_K or Q6_K, 2 <= M <= min(max_m, 32), K a multiple of 256, W 16-byte
// aligned, Q6_K rows 16-byte aligned).
bool gemv_kqm_supported(int type, const void* W, int M, int N, int K, int max_m, int num_sms, int smem_optin);
// Scratch of one call: the activation table, sums of squares, split partials
// and counters (256-byte aligned base).
size_t gemv_kqm_workspace_bytes(int type, int M, int N, int K, int num_sms, int smem_optin);
// Two launches on s (the table, then the GEMV), both programmatic dependents
// of their predecessor; cudaErrorInvalidValue when ws is missing, misaligned
// or short.
cudaError_t gemv_kqm_launch(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                            const ActArgs& act, int early, int num_sms, int smem_optin, void* ws, size_t ws_bytes,
                            cudaStream_t s);
cudaError_t status_fetch_gemv_kqm(unsigned* out, cudaStream_t s);
// Shared-memory KB of one split's activation table (K splits follow from it)
// and consumer warps per 16-row tile (0: automatic).
void gemv_kqm_tune(int table_kb, int group);

}  // namespace swq
