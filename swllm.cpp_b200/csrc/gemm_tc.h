// gemm_tc.h -- tensor-core (tcgen05) dequant-GEMM for prefill-sized M.
#pragma once

#include <cuda_runtime.h>

namespace swq {

// Activation prologue of the conversion to fp16 (kinds as swq_act.kind): the
// input row m of the GEMM is
//   RMSNORM: x = X[m] (+ R[m]), then x * normw; 1/sqrt(mean(x^2) + eps) goes
//            into the row's output scale, and x is written to sum_out when given
//   SWIGLU:  silu(X[m*ld + k]) * X[m*ld + K + k]
struct ActArgs {
    int kind = 0;  // 0 none, 1 RMSNORM, 2 SWIGLU
    const float* R = nullptr;
    const float* normw = nullptr;
    float eps = 0.f;
    float* sum_out = nullptr;
    int ld = 0;  // X row stride in elements (0: K)
    const int* rows_dev = nullptr;  // device row count: rows at or past it are not converted
};

// Stream-ordered scratch from libswq's pool on the current device (kept for
// the next call once freed).
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t s);
cudaError_t scratch_free(void* p, cudaStream_t s);
// True when the tcgen05 GEMM serves this problem.
bool gemm_tc_supported(int type, const void* W, int M, int N, int K, int refcpu);
// Y[M x N] = X[M x K] . W[N x K]^T on tensor cores.
cudaError_t gemm_tc_launch(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                           int refcpu, int num_sms, cudaStream_t s, const ActArgs& act = ActArgs{});
// The same with the fp16 copy of X in libswq's fixed device array instead of a
// stream-ordered allocation (swq_gemm_noalloc); M * K must fit that array.
cudaError_t gemm_tc_launch_noalloc(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                                   int refcpu, int num_sms, cudaStream_t s, const ActArgs& act = ActArgs{});
// The same with the scratch in a caller-owned workspace (256-byte aligned,
// at least gemm_tc_workspace_bytes); cudaErrorInvalidValue when it is not.
size_t gemm_tc_workspace_bytes(int M, int N, int K, int num_sms);
cudaError_t gemm_tc_launch_ws(int type, const void* W, const float* X, float* Y, int M, int N, int K, int refcpu,
                              int num_sms, cudaStream_t s, const ActArgs& act, void* ws, size_t ws_bytes);
// MoE grouped GEMM: expert e multiplies rows offsets[e] .. offsets[e+1]-1 of X
// (rows x K) by the GGUF matrix wptrs[e] (N x K) into the same rows of Y.
// wptrs and offsets are device arrays of n_experts and n_experts + 1 entries.
// refcpu: Q2_K in the reference CPU routine's activation order.
// mean_rows > 0 picks the token tile (else rows / n_experts); live_rows, when
// given, is a device count past which X is not read (offsets non-decreasing).
// w_all != nullptr: stacked experts, expert e is rows e*N .. e*N+N-1 of the
// n_experts*N x K matrix at w_all (wptrs unused).
cudaError_t gemm_tc_grouped_launch(int type, const void* const* wptrs, const int* offsets, const float* X, float* Y,
                                   int n_experts, int rows, int N, int K, int refcpu, int num_sms, cudaStream_t s,
                                   int mean_rows = 0, const int* live_rows = nullptr, const void* w_all = nullptr);
cudaError_t status_fetch_gemm_tc(unsigned* out, cudaStream_t s);

// SWQ_OPT_EARLY_WEIGHT_PREFETCH for the tensor-core GEMM: 1 lets its weight
// loads start before the previous kernel on the stream completes.
void gemm_tc_set_early_prefetch(int on);

}  // namespace swq
