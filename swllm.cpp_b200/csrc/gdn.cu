// gdn.cu -- one decode step of a GatedDeltaNet (linear attention) layer on
// the device, after its projections (sm_100a).
//
// Follows the reference's Qwen3.5 branch of Model::forward
// (src/model.h:369-513) from the projection outputs to the input of the
// output projection:
//   6. causal depthwise conv1d over the value channels: the channel's
//      history shifts left by one, the new value enters last, out = sum_w
//      conv_w[d][w] * hist[w]                                 (:421-440)
//   7. per value head h (key head h mod n_k): decay = exp(-exp(a_h) *
//      sigmoid(alpha_h) [* sigmoid(dt_h)]), beta = sigmoid(beta_h) (1 without
//      the projection); pred = S^T k; S = decay S + beta k (v - pred)^T;
//      y = S^T q, S of [k_hd x v_hd] per head                  (:442-487)
//   8. per head RMSNorm of y (eps 1e-5) times ssm_norm          (:489-499)
//   9. y *= sigmoid(z)                                         (:501-504)
// Every product and sum is rounded as the reference's loops round them
// (separate multiplies and adds, sums in index order), except the head
// norm's sum of squares, which is a tree over the head's threads.
//
// One CTA per (row, value head), one thread per value column j: thread j
// owns column j of the head's state (k_hd floats at stride v_hd, coalesced
// across the warp), its conv channel and its output.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/swq.h"
#include "gdn.h"
#include "swq_device.cuh"

namespace swq {

namespace {

constexpr int GDN_MAX_HD = 1024;

struct GdnArgs {
    const float* qkv;   // [rows, ld_qkv]: q (key_dim), k (key_dim), v (value_dim)
    int ld_qkv;
    const float* z;     // [rows, value_dim] or null (the reference then gates with sigmoid(0))
    const float* beta;  // [rows, n_v] raw projections, each may be null
    const float* alpha;
    const float* dt;
    const float* a;       // [n_v] or null
    const float* conv_w;  // [value_dim, cw] or null (no conv)
    const float* norm_w;  // [value_dim] or null
    float* S;             // [rows, n_v, k_hd, v_hd]
    float* conv;          // [rows, value_dim, cw]
    float* y;             // [rows, value_dim]
    int n_k, n_v, k_hd, v_hd, cw;
};

__device__ __forceinline__ float sigm(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

__global__ void gdn_step_kernel(const GdnArgs a) {
    extern __shared__ float sh[];  // q[k_hd], k[k_hd], red[32]
    float* qs = sh;
    float* ks = sh + a.k_hd;
    float* red = ks + a.k_hd;
    const int h = blockIdx.x, row = blockIdx.y, j = threadIdx.x;
    const int key_dim = a.n_k * a.k_hd, value_dim = a.n_v * a.v_hd;
    const float* qkv = a.qkv + static_cast<size_t>(row) * a.ld_qkv;
    const int kh = h % a.n_k;
    for (int i = j; i < a.k_hd; i += blockDim.x) {
        qs[i] = qkv[kh * a.k_hd + i];
        ks[i] = qkv[key_dim + kh * a.k_hd + i];
    }
    const bool live = j < a.v_hd;
    const int d = h * a.v_hd + j;
    // 6. conv1d of this value channel
    float v = 0.f;
    if (live) {
        v = qkv[2 * key_dim + d];
        if (a.conv_w != nullptr && a.cw > 0) {
            float* hist = a.conv + (static_cast<size_t>(row) * value_dim + d) * a.cw;
            for (int w = 0; w + 1 < a.cw; ++w) hist[w] = hist[w + 1];
            hist[a.cw - 1] = v;
            const float* cwp = a.conv_w + static_cast<size_t>(d) * a.cw;
            float s = 0.f;
            for (int w = 0; w < a.cw; ++w) s = __fadd_rn(s, __fmul_rn(cwp[w], hist[w]));
            v = s;
        }
    }
    // 7. gates of head h
    const size_t gi = static_cast<size_t>(row) * a.n_v + h;
    const float base = a.a ? expf(a.a[h]) : 1.0f;
    const float ag = a.alpha ? sigm(a.alpha[gi]) : 1.0f;
    float log_decay = __fmul_rn(-base, ag);
    if (a.dt) log_decay = __fmul_rn(log_decay, sigm(a.dt[gi]));
    const float decay = expf(log_decay);
    const float beta = a.beta ? sigm(a.beta[gi]) : 1.0f;
    __syncthreads();
    float y = 0.f;
    if (live) {
        float* Sc = a.S + (gi * a.k_hd) * a.v_hd + j;
        float pred = 0.f;
        for (int i = 0; i < a.k_hd; ++i) pred = __fadd_rn(pred, __fmul_rn(Sc[static_cast<size_t>(i) * a.v_hd], ks[i]));
        const float delta = __fsub_rn(v, pred);
        for (int i = 0; i < a.k_hd; ++i) {
            float* p = Sc + static_cast<size_t>(i) * a.v_hd;
            const float s = __fadd_rn(__fmul_rn(decay, *p), __fmul_rn(__fmul_rn(beta, ks[i]), delta));
            *p = s;
            y = __fadd_rn(y, __fmul_rn(s, qs[i]));
        }
    }
    // 8. per-head RMSNorm
    if (a.norm_w != nullptr) {
        float sq = live ? __fmul_rn(y, y) : 0.f;
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if ((j & 31) == 0) red[j >> 5] = sq;
        __syncthreads();
        float ss = 0.f;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) ss += red[w];
        ss = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(a.v_hd)), 1e-5f)));
        if (live) y = __fmul_rn(__fmul_rn(y, ss), a.norm_w[d]);
    }
    // 9. gate
    if (live) {
        const float zg = a.z ? sigm(a.z[static_cast<size_t>(row) * value_dim + d]) : sigm(0.0f);
        a.y[static_cast<size_t>(row) * value_dim + d] = __fmul_rn(y, zg);
    }
}

}  // namespace

cudaError_t gdn_step_launch(const float* qkv, int ld_qkv, const float* z, const float* beta, const float* alpha,
                            const float* dt, const float* a, const float* conv_w, const float* norm_w, float* S,
                            float* conv, float* y, int rows, int n_k, int n_v, int k_hd, int v_hd, int cw,
                            cudaStream_t s) {
    GdnArgs g{qkv, ld_qkv, z, beta, alpha, dt, a, conv_w, norm_w, S, conv, y, n_k, n_v, k_hd, v_hd, cw};
    const int threads = (v_hd + 31) / 32 * 32;
    const size_t smem = (2 * static_cast<size_t>(k_hd) + 32) * sizeof(float);
    gdn_step_kernel<<<dim3(n_v, rows), threads, smem, s>>>(g);
    return cudaGetLastError();
}

int gdn_max_head_dim() { return GDN_MAX_HD; }

}  // namespace swq
