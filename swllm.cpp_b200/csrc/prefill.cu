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


// Causal attention for a whole prompt, tiled (the form used for head_dim 64
// and 128): CTA = (64 query rows of one sequence, query head h), 256 threads.
// Q rows live in shared memory; key/value positions 0 .. the tile's last
// query position stream through in tiles of 64.  Thread (ty, tx), ty =
// t / 16, tx = t % 16, owns scores S[ty + 16 i][tx + 16 j] (i, j < 4) of a
// tile and output rows ty + 16 i, dims 4 tx .. 4 tx + 3 (+ 64 for head_dim
// 128).  Online softmax per row (the 16 threads of a row are 16 lanes of one
// warp: max and sum by shuffles), masked causally (key t <= the row's
// position).  fp32 throughout, like the reference's loops
// (src/model.h:329-361); the sums run in another order.
template <int HD>
__global__ void __launch_bounds__(256) attention_prefill_tiled(
    float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ kcache,
    const float* __restrict__ vcache, int pos0, int seq_len, int num_heads, int num_kv_heads, int max_seq, int ldq,
    int ldo) {
    constexpr int BM = 64, BN = 64, KS = HD + 4;  // K rows padded: 16 consecutive rows hit distinct banks
    constexpr int DPT = HD / 16;                  // output dims per thread (4 or 8)
    extern __shared__ float psm[];
    float* Qs = psm;             // [BM][HD]
    float* Ks = Qs + BM * HD;    // [BN][KS]
    float* Vs = Ks + BN * KS;    // [BN][HD]
    float* Ps = Vs + BN * HD;    // [BM][BN + 1]
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    // heavier (later) query tiles first: the causal work grows with the tile
    const int qt = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int p0 = qt * BM;
    const int nrow = min(BM, seq_len - p0);
    const int kvh = h / (num_heads / num_kv_heads);
    const int kv_dim = num_kv_heads * HD;
    const size_t m0 = static_cast<size_t>(seq) * seq_len + p0;
    for (int i = tid; i < BM * HD / 4; i += 256) {
        const int r = i / (HD / 4), c = (i % (HD / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nrow) {
            const float* src = q + (m0 + r) * ldq + h * HD + c;
            v = make_float4(src[0], src[1], src[2], src[3]);
        }
        *reinterpret_cast<float4*>(Qs + r * HD + c) = v;
    }
    const float* kb = kcache + static_cast<size_t>(seq) * max_seq * kv_dim + kvh * HD;
    const float* vb = vcache + static_cast<size_t>(seq) * max_seq * kv_dim + kvh * HD;
    const float sqrt_hd = sqrtf(static_cast<float>(HD));
    float mrow[4], lrow[4], acc[4][DPT];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        mrow[i] = -INFINITY;
        lrow[i] = 0.f;
#pragma unroll
        for (int d = 0; d < DPT; ++d) acc[i][d] = 0.f;
    }
    const int last = pos0 + p0 + nrow - 1;  // last key position any row of the tile sees
    for (int t0 = 0; t0 <= last; t0 += BN) {
        __syncthreads();  // the previous tile's K, V, P are consumed
        for (int i = tid; i < BN * HD / 4; i += 256) {
            const int r = i / (HD / 4), c = (i % (HD / 4)) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (t0 + r <= last) {
                const float* ks = kb + static_cast<size_t>(t0 + r) * kv_dim + c;
                const float* vs = vb + static_cast<size_t>(t0 + r) * kv_dim + c;
                kv = make_float4(ks[0], ks[1], ks[2], ks[3]);
                vv = make_float4(vs[0], vs[1], vs[2], vs[3]);
            }
            *reinterpret_cast<float4*>(Ks + r * KS + c) = kv;
            *reinterpret_cast<float4*>(Vs + r * HD + c) = vv;
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            float4 qa[4], ka[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(Qs + (ty + 16 * i) * HD + d);
#pragma unroll
            for (int j = 0; j < 4; ++j) ka[j] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * j) * KS + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float s = sc[i][j];
                    s = fmaf(qa[i].x, ka[j].x, s);
                    s = fmaf(qa[i].y, ka[j].y, s);
                    s = fmaf(qa[i].z, ka[j].z, s);
                    s = fmaf(qa[i].w, ka[j].w, s);
                    sc[i][j] = s;
                }
        }
        // mask, online softmax per row, P into shared memory
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            const int qpos = pos0 + p0 + r;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int t = t0 + tx + 16 * j;
                sc[i][j] = (r < nrow && t <= qpos) ? sc[i][j] / sqrt_hd : -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mnew = fmaxf(mrow[i], mx);
            // rows with nothing unmasked yet keep m = -inf: scale 1, p = 0
            const float corr = mnew == -INFINITY ? 1.f : expf(mrow[i] - mnew);
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float pv = mnew == -INFINITY ? 0.f : expf(sc[i][j] - mnew);
                Ps[r * (BN + 1) + tx + 16 * j] = pv;
                ps += pv;
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            lrow[i] = lrow[i] * corr + ps;
            mrow[i] = mnew;
#pragma unroll
            for (int dd = 0; dd < DPT; ++dd) acc[i][dd] *= corr;
        }
        __syncthreads();
        // O += P V
        const int kmax = min(BN, last - t0 + 1);
        for (int kk = 0; kk < kmax; ++kk) {
            const float4 v0 = *reinterpret_cast<const float4*>(Vs + kk * HD + 4 * tx);
            float4 v1 = v0;
            if constexpr (DPT == 8) v1 = *reinterpret_cast<const float4*>(Vs + kk * HD + 64 + 4 * tx);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pv = Ps[(ty + 16 * i) * (BN + 1) + kk];
                acc[i][0] = fmaf(pv, v0.x, acc[i][0]);
                acc[i][1] = fmaf(pv, v0.y, acc[i][1]);
                acc[i][2] = fmaf(pv, v0.z, acc[i][2]);
                acc[i][3] = fmaf(pv, v0.w, acc[i][3]);
                if constexpr (DPT == 8) {
                    acc[i][4] = fmaf(pv, v1.x, acc[i][4]);
                    acc[i][5] = fmaf(pv, v1.y, acc[i][5]);
                    acc[i][6] = fmaf(pv, v1.z, acc[i][6]);
                    acc[i][7] = fmaf(pv, v1.w, acc[i][7]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = ty + 16 * i;
        if (r >= nrow) continue;
        float* o = out + (m0 + r) * ldo + h * HD;
        const float inv = 1.f / lrow[i];
#pragma unroll
        for (int dd = 0; dd < DPT; ++dd) o[(dd < 4 ? 4 * tx : 64 + 4 * tx - 4) + dd] = acc[i][dd] * inv;
    }
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
    if ((head_dim == 64 || head_dim == 128) && seq_len > 0 && rows % seq_len == 0 && (ldq % 4) == 0 &&
        (reinterpret_cast<uintptr_t>(q) & 15u) == 0 && (num_kv_heads * head_dim) % 4 == 0) {
        const int nseq = rows / seq_len;
        const dim3 grid((seq_len + 63) / 64, num_heads, nseq);
        if (nseq > 65535 || num_heads > 65535) return cudaErrorInvalidConfiguration;
        const size_t smem = (64 * head_dim + 64 * (head_dim + 4) + 64 * head_dim + 64 * 65) * sizeof(float);
        cudaError_t e;
        if (head_dim == 128) {
            e = cudaFuncSetAttribute(attention_prefill_tiled<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            attention_prefill_tiled<128><<<grid, 256, smem, s>>>(out, q, kcache, vcache, pos0, seq_len, num_heads,
                                                                  num_kv_heads, max_seq, ldq, ldo);
        } else {
            e = cudaFuncSetAttribute(attention_prefill_tiled<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            attention_prefill_tiled<64><<<grid, 256, smem, s>>>(out, q, kcache, vcache, pos0, seq_len, num_heads,
                                                                 num_kv_heads, max_seq, ldq, ldo);
        }
        return cudaGetLastError();
    }
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
