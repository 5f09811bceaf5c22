// prefill.cu -- the two steps of a batched prefill forward that differ from a
// decode step: RoPE + KV append at one position per row, and causal
// attention.  Everything else in a prefill (embedding rows, RMSNorm, the
// projections as M-row tensor-core GEMMs, SiLU-mul) runs the decode step's
// kernels on M = sequences x tokens rows.
//
// The reference has no batched prefill: it calls Model::forward once per
// prompt token (src/main.cpp:284-287), so token p of the prompt sees
// positions 0..pos0+p of its own cache (src/model.h:329-361).  Here the
// prompt's P tokens of each of S sequences are rows m = s*P + p of one
// [S*P x n] buffer; row m is position pos0 + p of sequence s.
//
// KV cache layout as in decode.cu: [sequence s][position t][kv_dim] per layer.
#include <cuda_runtime.h>
#include <math.h>

#include <cstdint>

#include "prefill.h"

namespace swq {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// RoPE on q (in place) and k of row m at position pos0 + m % seq_len, then k
// and v into the cache of sequence m / seq_len at that position.  Pairs and
// angles as decode.cu's rope_kv_kernel (the same cosf / sinf of pos * freqs[i]),
// so a prefilled position holds the same keys as a decoded one.
// Grid: (rows, blocks over the row's items); every index below is bounded by
// q_dim, kv_dim (the row) and max_seq (the cache, checked on the host).
__global__ void rope_kv_prefill_kernel(float* __restrict__ q, const float* __restrict__ k,
                                       const float* __restrict__ v, float* __restrict__ kcache,
                                       float* __restrict__ vcache, int pos0, int seq_len,
                                       const float* __restrict__ freqs, int q_dim, int kv_dim, int head_dim,
                                       int rope_dim, int neox, int max_seq, int ldq, int ldk, int ldv) {
    const int m = blockIdx.x;
    const int seq = m / seq_len, pos = pos0 + m % seq_len;
    const int half = rope_dim / 2;
    const int qpairs = (q_dim / head_dim) * half, kpairs = (kv_dim / head_dim) * half;
    float* qb = q + static_cast<size_t>(m) * ldq;
    const float* kb = k + static_cast<size_t>(m) * ldk;
    const float* vb = v + static_cast<size_t>(m) * ldv;
    float* kc = kcache + (static_cast<size_t>(seq) * max_seq + pos) * kv_dim;
    float* vc = vcache + (static_cast<size_t>(seq) * max_seq + pos) * kv_dim;
    for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < qpairs + kpairs + kv_dim; i += gridDim.y * blockDim.x) {
        if (i < qpairs + kpairs) {
            const bool isq = i < qpairs;
            const int j = isq ? i : i - qpairs;
            const int h = j / half, r = j % half;
            const int i0 = h * head_dim + (neox ? r : 2 * r);
            const int i1 = h * head_dim + (neox ? r + half : 2 * r + 1);
            const float angle = static_cast<float>(pos) * freqs[r];
            const float c = cosf(angle), s = sinf(angle);
            if (isq) {
                const float a = qb[i0], bb = qb[i1];
                qb[i0] = a * c - bb * s;
                qb[i1] = a * s + bb * c;
            } else {
                const float a = kb[i0], bb = kb[i1];
                kc[i0] = a * c - bb * s;
                kc[i1] = a * s + bb * c;
            }
        } else {
            const int d = i - qpairs - kpairs;
            vc[d] = vb[d];
        }
    }
    if (rope_dim < head_dim) {  // dimensions past rope_dim are not rotated: k as is
        for (int d = blockIdx.y * blockDim.x + threadIdx.x; d < kv_dim; d += gridDim.y * blockDim.x)
            if (d % head_dim >= rope_dim) kc[d] = kb[d];
    }
}

constexpr int PF_WARPS = 8;

// Causal attention, one warp per (row m, query head h): scores
// q.k_t / sqrt(head_dim) over t = 0 .. pos0 + m % seq_len of the row's
// sequence, softmax, sum of softmax * v_t (src/model.h:329-361), as one
// online-softmax pass in position order.  Lane l holds elements
// l*PER .. l*PER+PER-1 of the head (PER = head_dim / 32).  Warps past M x H
// return at once; every cache read is below position pos0 + seq_len <= max_seq.
template <int PER>
__global__ void __launch_bounds__(PF_WARPS * 32) attention_prefill_kernel(
    float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ kcache,
    const float* __restrict__ vcache, int pos0, int seq_len, int rows, int num_heads, int num_kv_heads,
    int max_seq, int ldq, int ldo) {
    constexpr int HD = 32 * PER;
    const int lane = threadIdx.x & 31;
    const long long w = static_cast<long long>(blockIdx.x) * PF_WARPS + (threadIdx.x >> 5);
    if (w >= static_cast<long long>(rows) * num_heads) return;
    const int m = static_cast<int>(w / num_heads), h = static_cast<int>(w % num_heads);
    const int seq = m / seq_len, n_ctx = pos0 + m % seq_len + 1;
    const int kvh = h / (num_heads / num_kv_heads);
    const int kv_dim = num_kv_heads * HD;
    const float* qh = q + static_cast<size_t>(m) * ldq + h * HD + lane * PER;
    const float* kbase = kcache + static_cast<size_t>(seq) * max_seq * kv_dim + kvh * HD + lane * PER;
    const float* vbase = vcache + static_cast<size_t>(seq) * max_seq * kv_dim + kvh * HD + lane * PER;
    float qr[PER], acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        qr[i] = qh[i];
        acc[i] = 0.f;
    }
    const float sqrt_hd = sqrtf(static_cast<float>(HD));
    float mx = -INFINITY, l = 0.f;
    for (int t = 0; t < n_ctx; ++t) {
        const float* kt = kbase + static_cast<size_t>(t) * kv_dim;
        const float* vt = vbase + static_cast<size_t>(t) * kv_dim;
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < PER; ++i) d += qr[i] * kt[i];
        const float s = warp_sum(d) / sqrt_hd;
        const float mnew = fmaxf(mx, s);
        const float corr = expf(mx - mnew);  // 0 on the first position (mx = -inf)
        const float p = expf(s - mnew);
        l = l * corr + p;
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[i] = acc[i] * corr + p * vt[i];
        mx = mnew;
    }
    float* oh = out + static_cast<size_t>(m) * ldo + h * HD + lane * PER;
    const float inv_l = 1.f / l;
#pragma unroll
    for (int i = 0; i < PER; ++i) oh[i] = acc[i] * inv_l;
}

}  // namespace

cudaError_t rope_kv_prefill_launch(float* q, const float* k, const float* v, float* kcache, float* vcache, int pos0,
                                   int seq_len, const float* freqs, int q_dim, int kv_dim, int head_dim,
                                   int rope_dim, int neox, int rows, int max_seq, int ldq, int ldk, int ldv,
                                   cudaStream_t s) {
    const int items = (q_dim / head_dim + kv_dim / head_dim) * (rope_dim / 2) + kv_dim;
    const int gy = (items + 255) / 256;
    if (gy > 65535) return cudaErrorInvalidConfiguration;
    rope_kv_prefill_kernel<<<dim3(rows, gy), 256, 0, s>>>(q, k, v, kcache, vcache, pos0, seq_len, freqs, q_dim,
                                                          kv_dim, head_dim, rope_dim, neox, max_seq, ldq, ldk, ldv);
    return cudaGetLastError();
}

cudaError_t attention_prefill_launch(float* out, const float* q, const float* kcache, const float* vcache, int pos0,
                                     int seq_len, int rows, int num_heads, int num_kv_heads, int head_dim,
                                     int max_seq, int ldq, int ldo, cudaStream_t s) {
    const long long warps = static_cast<long long>(rows) * num_heads;
    const long long blocks = (warps + PF_WARPS - 1) / PF_WARPS;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const dim3 grid(static_cast<unsigned>(blocks)), block(PF_WARPS * 32);
    switch (head_dim / 32) {
        case 1: attention_prefill_kernel<1><<<grid, block, 0, s>>>(out, q, kcache, vcache, pos0, seq_len, rows,
                                                                   num_heads, num_kv_heads, max_seq, ldq, ldo);
            break;
        case 2: attention_prefill_kernel<2><<<grid, block, 0, s>>>(out, q, kcache, vcache, pos0, seq_len, rows,
                                                                   num_heads, num_kv_heads, max_seq, ldq, ldo);
            break;
        case 4: attention_prefill_kernel<4><<<grid, block, 0, s>>>(out, q, kcache, vcache, pos0, seq_len, rows,
                                                                   num_heads, num_kv_heads, max_seq, ldq, ldo);
            break;
        case 8: attention_prefill_kernel<8><<<grid, block, 0, s>>>(out, q, kcache, vcache, pos0, seq_len, rows,
                                                                   num_heads, num_kv_heads, max_seq, ldq, ldo);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace swq
