// ref_shim.cpp -- C ABI over the reference's own src/tensor.h, compiled from
// the reference sources where they lie (see oracle/Makefile).  TEST
// INFRASTRUCTURE ONLY: it pins the C restatement in swq_oracle.c and serves as
// the timed CPU baseline ("kind": "reference").  It is never part of libswq.
//
// Every entry point calls straight into the reference's code:
//   ref_dequantize          -> dequantize()                   src/tensor.h:451
//   ref_matmul_transposed_q -> Compute::matmul_transposed_q    src/tensor.h:1212
//                              (Backend::CPU: the fused per-format routines)
//   ref_matmul_transposed   -> cpu_matmul_transposed          src/tensor.h:548
//   ref_fp16_to_fp32        -> fp16_to_fp32                   src/tensor.h:33
//   ref_type_size / ref_block_size -> ggml_type_size / ggml_block_size
//                                                             src/gguf.h:60,89
#include <cstdint>
#include <cstddef>

#include "tensor.h"

extern "C" {

void ref_dequantize(unsigned type, const void* src, float* dst, long long n) {
    dequantize(src, dst, static_cast<int64_t>(n), static_cast<GGMLType>(type));
}

void ref_matmul_transposed_q(unsigned type, float* out, const float* x,
                             const void* w, int N, int K) {
    Compute compute(Backend::CPU);
    QuantWeight qw;
    qw.data = w;
    qw.type = static_cast<GGMLType>(type);
    compute.matmul_transposed_q(out, x, qw, N, K);
}

void ref_matmul_transposed(float* out, const float* x, const float* w, int N, int K) {
    cpu_matmul_transposed(out, x, w, N, K);
}

float ref_fp16_to_fp32(unsigned short h) { return fp16_to_fp32(h); }

size_t ref_type_size(unsigned type) { return ggml_type_size(static_cast<GGMLType>(type)); }

size_t ref_block_size(unsigned type) { return ggml_block_size(static_cast<GGMLType>(type)); }

int ref_max_threads(void) {
#ifdef LLM_USE_OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void ref_set_threads(int n) {
#ifdef LLM_USE_OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

}  // extern "C"
