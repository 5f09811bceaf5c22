// qkv_extras.cu -- the optional steps between the q/k/v projections and RoPE
// in the reference's dense forward (src/model.h:291-318): bias adds
// (q += bq, k += bk, v += bv; Compute::add) and the per-head RMSNorm of q and
// k with one [head_dim] weight shared by the heads (Compute::rmsnorm,
// src/tensor.h:1028-1033), in that order.  Models without them (Llama) never
// launch this kernel.
//
// One CTA per (row, head segment): the segments are the heads of q (when q has
// a bias or a norm), then of k, then of v (bias only).  Each CTA works on one
// head_dim slice of one row in place: bias add and sum of squares in one
// pass, then the scale.
#include <cuda_runtime.h>
#include <math.h>

#include "qkv_extras.h"

namespace swq {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

constexpr int QX_THREADS = 128;

struct QkvExtras {
    float *q, *k, *v;
    const float *bq, *bk, *bv, *qn, *kn;
    int sq, sk, sv;        // segments (heads) of q, k, v that have work
    int head_dim, ldq, ldk, ldv;
    float eps;
};

__global__ void __launch_bounds__(QX_THREADS) qkv_extras_kernel(const QkvExtras a) {
    __shared__ float red[QX_THREADS / 32];
    const int row = blockIdx.x, seg = blockIdx.y, hd = a.head_dim;
    float* x;
    const float* bias;
    const float* w;
    int h;
    if (seg < a.sq) {
        h = seg;
        x = a.q + static_cast<size_t>(row) * a.ldq + h * hd;
        bias = a.bq;
        w = a.qn;
    } else if (seg < a.sq + a.sk) {
        h = seg - a.sq;
        x = a.k + static_cast<size_t>(row) * a.ldk + h * hd;
        bias = a.bk;
        w = a.kn;
    } else {
        h = seg - a.sq - a.sk;
        x = a.v + static_cast<size_t>(row) * a.ldv + h * hd;
        bias = a.bv;
        w = nullptr;
    }
    const float* b = bias ? bias + h * hd : nullptr;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hd; i += QX_THREADS) {
        float t = x[i];
        if (b) {
            t = t + b[i];
            x[i] = t;
        }
        ss = fmaf(t, t, ss);
    }
    if (!w) return;  // the same for the whole CTA
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < QX_THREADS / 32; ++i) tot += red[i];
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(hd) + a.eps);
    for (int i = threadIdx.x; i < hd; i += QX_THREADS) x[i] = x[i] * scale * w[i];
}

}  // namespace

cudaError_t qkv_extras_launch(float* q, float* k, float* v, const float* bq, const float* bk, const float* bv,
                              const float* q_norm, const float* k_norm, int q_dim, int kv_dim, int head_dim,
                              float eps, int rows, int ldq, int ldk, int ldv, cudaStream_t s) {
    QkvExtras a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.bq = bq;
    a.bk = bk;
    a.bv = bv;
    a.qn = q_norm;
    a.kn = k_norm;
    a.sq = (bq || q_norm) ? q_dim / head_dim : 0;
    a.sk = (bk || k_norm) ? kv_dim / head_dim : 0;
    a.sv = bv ? kv_dim / head_dim : 0;
    a.head_dim = head_dim;
    a.ldq = ldq;
    a.ldk = ldk;
    a.ldv = ldv;
    a.eps = eps;
    const int segs = a.sq + a.sk + a.sv;
    if (segs == 0 || rows == 0) return cudaSuccess;
    if (segs > 65535) return cudaErrorInvalidConfiguration;
    qkv_extras_kernel<<<dim3(rows, segs), QX_THREADS, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace swq
