// gemv.h -- internal launch interface of the libswq kernels (host side).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace swq {

struct DeviceInfo {
    int device = -1;
    int num_sms = 0;
    int smem_per_block_optin = 0;
    int smem_per_sm = 0;
    int cc_major = 0, cc_minor = 0;
};

// Activation prologue kinds (values of swq_act.kind).
enum : int { ACT_NONE = 0, ACT_RMSNORM = 1, ACT_SWIGLU = 2 };

struct GemvLaunch {
    int type;
    const void* W;
    const float* X;
    float* Y;
    int M, N, K;
    int refcpu;  // Q2_K reference-CPU activation order
    int early;   // weight prefetch before the programmatic dependency
    int num_sms;
    int smem_per_block_optin;
    int smem_per_sm;
    int smem_kb;   // CTA shared-memory budget in KB (0: automatic)
    int stage_kb;  // largest weight stage in KB (0: 96)
    int ctas_per_sm;  // 0: automatic
    int xf = 1;       // fp32 activations (else 16-bit fixed point)
    int imma = 1;     // M = 1: exact integer dot products on the tensor cores (1: Q6_K, 2: Q4_K too)
    // activation prologue (ACT_*); ld = X row stride in elements (0: K, SWIGLU: 2K)
    int act = ACT_NONE;
    const float* R = nullptr;
    const float* normw = nullptr;
    float eps = 0.f;
    float* sum_out = nullptr;
    int ld = 0;
};

// Fused dequant + GEMV for M <= 8 activation rows.
cudaError_t gemv_launch(const GemvLaunch& L, cudaStream_t s);
// The single-row form with integer tensor-core dot products (gemv_imma.cu):
// whether it takes this launch, and the launch.
bool gemv_imma_supported(const GemvLaunch& L);
cudaError_t gemv_imma_launch(const GemvLaunch& L, cudaStream_t s);
// The single-row Q4_K / Q6_K form with integer tensor-core sub-block sums and
// one conversion per super-block (gemv_kq.cu; SWQ_OPT_GEMV_INT_MMA >= 2).
bool gemv_kq_supported(const GemvLaunch& L);
cudaError_t gemv_kq_launch(const GemvLaunch& L, cudaStream_t s);
// Device status bit of an input a kernel skipped because it was misaligned
// (DEV_BAD_ALIGN in the device code).
constexpr unsigned kStatusBadAlign = 32u;

// Grouped GEMV (MoE decode): expert e multiplies rows offsets[e] ..
// offsets[e+1]-1 of X by its GGUF matrix wptrs[e] (device arrays); every expert
// matrix 16-byte aligned (a misaligned one is skipped and flagged).
// adaptive: rows per pass chosen per expert on the device (4, 2 or 1) instead
// of from the mean rows_total / n_experts.  w_all: stacked experts (expert e
// at w_all + e * N * row bytes; wptrs unused).
cudaError_t grouped_gemv_launch(int type, const void* const* wptrs, const int* offsets, const float* X, float* Y,
                                int n_experts, int rows_total, int N, int K, int refcpu, int smem_optin,
                                cudaStream_t s, bool adaptive = false, const void* w_all = nullptr);
// Shared-memory bytes of the per-CTA activation prep for padded row count MT.
size_t gemv_smem_x_bytes(int type, int MT, int K, bool xf);

// Bit-exact dequantization of nblocks whole blocks.
cudaError_t dequant_launch(int type, const void* src, float* dst, int64_t nblocks, int num_sms,
                           cudaStream_t s);

// Device status words of each translation unit (bounded-wait timeouts).
cudaError_t status_fetch_gemv(unsigned* out, cudaStream_t s);
cudaError_t status_fetch_dequant(unsigned* out, cudaStream_t s);
cudaError_t status_fetch_gemv_imma(unsigned* out, cudaStream_t s);
cudaError_t status_fetch_gemv_kq(unsigned* out, cudaStream_t s);

}  // namespace swq
