// dropin_backend.cpp -- the rest of the reference's CUDA backend interface for
// the drop-in build (TEST INFRASTRUCTURE ONLY).
//
// With LLM_USE_CUDA the reference's Compute (src/tensor.h:20-28) declares
// these functions, defined in its src/cuda_kernels.cu.  In the drop-in build
// the quantized matmul goes to libswq (oracle/make_dropin.py); these element-
// wise operations run the reference's own CPU routines on the same host
// buffers, so the model's results differ from the CPU build only where libswq
// computes.  Compiled with the derived tensor.h ahead of the reference's.
#include "tensor.h"

bool cuda_check_gpu() { return true; }

void cuda_matmul(float* out, const float* a, const float* b, int M, int N, int K) {
    cpu_matmul(out, a, b, M, N, K);
}

void cuda_matmul_transposed_weight(float* out, const float* x, const float* w, int N, int K) {
    cpu_matmul_transposed(out, x, w, N, K);
}

void cuda_rmsnorm(float* out, const float* x, const float* w, int n, float eps) { cpu_rmsnorm(out, x, w, n, eps); }

void cuda_softmax(float* x, int n) { cpu_softmax(x, n); }

void cuda_silu_elementwise_mul(float* out, const float* gate, const float* up, int n) {
    cpu_silu_elementwise_mul(out, gate, up, n);
}

void cuda_rope(float* q, float* k, int q_dim, int k_dim, int head_dim, int pos, float theta) {
    cpu_rope(q, k, q_dim, k_dim, head_dim, pos, theta);
}

void cuda_add(float* out, const float* a, const float* b, int n) { cpu_add(out, a, b, n); }

// libswq calls of the drop-in branch that returned an error (each printed).
extern "C" int dropin_errors(void) { return g_swq_dropin_errors; }

// Drops the libswq context and every weight it holds (call after freeing a
// model: its file buffer's address may come back for the next one).
extern "C" void dropin_reset(void) {
    swq_ctx_destroy(g_swq_dropin_ctx);
    g_swq_dropin_ctx = nullptr;
}
