// decode.cu -- the device-resident decode step around the quantized GEMVs:
// embedding row, RMSNorm, RoPE + KV-cache append, decode attention, SiLU-mul,
// residual add, argmax (the reference's Model::forward, src/model.h:257-543,
// with its Compute helpers, src/tensor.h:1028-1180).
//
// All activations are fp32, as in the reference.  B sequences decode in step
// (same position), row b of every [B x n] buffer belongs to sequence b.  The
// position lives in device memory (`pos`, advanced by swq_decode_advance) so a
// whole decode step can be captured once in a CUDA graph and replayed.
//
// KV cache layout (fp32): [layer][sequence b][position t][kv_dim].
#include <cuda_runtime.h>
#include <math.h>

#include <cstdint>

#include "decode.h"

namespace swq {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// RMSNorm of each row: out = x * (1 / sqrt(mean(x^2) + eps)) * w
// (src/tensor.h:1028-1033).  One CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(float* __restrict__ out, const float* __restrict__ x,
                                                      const float* __restrict__ w, int n, float eps) {
    const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
    float* orow = out + static_cast<size_t>(blockIdx.x) * n;
    __shared__ float part[8];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) part[0] = v;
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(part[0] / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = xr[i] * scale * w[i];
}

// RoPE on q (in place) and k, then k and v into the cache at `pos`.
// Interleaved pairs (2i, 2i+1) (src/tensor.h:1068-1107) or, with neox, pairs
// (i, i + rope_dim/2) (src/tensor.h:1121-1161); angle = pos * freqs[i].
// One thread per rotated pair (q heads, then k heads), plus v copies.
__global__ void rope_kv_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                               float* __restrict__ kcache, float* __restrict__ vcache, const int* __restrict__ pos_p,
                               const float* __restrict__ freqs, int q_dim, int kv_dim, int head_dim, int rope_dim,
                               int neox, int max_seq) {
    const int b = blockIdx.y;
    const int pos = *pos_p;
    const int half = rope_dim / 2;
    const int qpairs = (q_dim / head_dim) * half, kpairs = (kv_dim / head_dim) * half;
    float* qb = q + static_cast<size_t>(b) * q_dim;
    const float* kb = k + static_cast<size_t>(b) * kv_dim;
    const float* vb = v + static_cast<size_t>(b) * kv_dim;
    float* kc = kcache + (static_cast<size_t>(b) * max_seq + pos) * kv_dim;
    float* vc = vcache + (static_cast<size_t>(b) * max_seq + pos) * kv_dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < qpairs + kpairs + kv_dim; i += gridDim.x * blockDim.x) {
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
    // dimensions past rope_dim are not rotated: copy k as is
    if (rope_dim < head_dim) {
        for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < kv_dim; d += gridDim.x * blockDim.x)
            if (d % head_dim >= rope_dim) kc[d] = kb[d];
    }
}

// Decode attention, split over the context: CTA (split, kv head, sequence)
// handles timesteps [split*chunk, ...) for the kv_mul query heads that share
// the kv head (src/model.h:329-361: score = q.k / sqrt(head_dim), softmax over
// t <= pos, out = sum softmax * v).  Writes per split the running max m, the
// sum l of exp(score - m) and the unnormalised output; attn_combine merges them.
constexpr int ATT_THREADS = 128;

// MUL query heads per kv head, PER = head_dim / 32 elements per lane.
template <int MUL, int PER>
__global__ void __launch_bounds__(ATT_THREADS) attn_split_kernel(
    const float* __restrict__ q, const float* __restrict__ kcache, const float* __restrict__ vcache,
    const int* __restrict__ pos_p, float* __restrict__ part_o, float* __restrict__ part_ml, int num_heads,
    int num_kv_heads, int max_seq, int chunk) {
    constexpr int HD = 32 * PER;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int nsplit = gridDim.x;
    const int kv_dim = num_kv_heads * HD;
    const int n_ctx = *pos_p + 1;
    const int t0 = split * chunk, t1 = min(n_ctx, t0 + chunk);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(HD));
    __shared__ float s_m[ATT_THREADS / 32][MUL], s_l[ATT_THREADS / 32][MUL];
    __shared__ float s_o[ATT_THREADS / 32][MUL][HD];

    float qv[MUL][PER], acc[MUL][PER], m[MUL], l[MUL];
#pragma unroll
    for (int j = 0; j < MUL; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
        const float* qh = q + (static_cast<size_t>(b) * num_heads + kvh * MUL + j) * HD;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            acc[j][e] = 0.f;
            qv[j][e] = qh[e * 32 + lane];
        }
    }
    const float* kbase = kcache + static_cast<size_t>(b) * max_seq * kv_dim + kvh * HD;
    const float* vbase = vcache + static_cast<size_t>(b) * max_seq * kv_dim + kvh * HD;
    for (int t = t0 + warp; t < t1; t += ATT_THREADS / 32) {
        const float* kt = kbase + static_cast<size_t>(t) * kv_dim;
        const float* vt = vbase + static_cast<size_t>(t) * kv_dim;
        float kk[PER], vv[PER];
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            kk[e] = kt[e * 32 + lane];
            vv[e] = vt[e * 32 + lane];
        }
#pragma unroll
        for (int j = 0; j < MUL; ++j) {
            float sdot = 0.f;
#pragma unroll
            for (int e = 0; e < PER; ++e) sdot = fmaf(qv[j][e], kk[e], sdot);
            const float score = warp_sum(sdot) * inv_sqrt;
            const float mn = fmaxf(m[j], score);
            const float corr = expf(m[j] - mn), pexp = expf(score - mn);
            l[j] = l[j] * corr + pexp;
#pragma unroll
            for (int e = 0; e < PER; ++e) acc[j][e] = fmaf(pexp, vv[e], acc[j][e] * corr);
            m[j] = mn;
        }
    }
    // merge the warps of the CTA
#pragma unroll
    for (int j = 0; j < MUL; ++j) {
        if (lane == 0) {
            s_m[warp][j] = m[j];
            s_l[warp][j] = l[j];
        }
#pragma unroll
        for (int e = 0; e < PER; ++e) s_o[warp][j][e * 32 + lane] = acc[j][e];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < MUL * HD; idx += ATT_THREADS) {
        const int j = idx / HD, d = idx % HD;
        float mm = -INFINITY;
        for (int w = 0; w < ATT_THREADS / 32; ++w) mm = fmaxf(mm, s_m[w][j]);
        float ll = 0.f, oo = 0.f;
        for (int w = 0; w < ATT_THREADS / 32; ++w) {
            const float c = s_m[w][j] == -INFINITY ? 0.f : expf(s_m[w][j] - mm);
            ll += s_l[w][j] * c;
            oo += s_o[w][j][d] * c;
        }
        const size_t slot = (static_cast<size_t>(b) * num_heads + kvh * MUL + j) * nsplit + split;
        part_o[slot * HD + d] = oo;
        if (d == 0) {
            part_ml[2 * slot] = mm;
            part_ml[2 * slot + 1] = ll;
        }
    }
}

// out[b, h*head_dim + d] = sum_s o_s * exp(m_s - M) / sum_s l_s * exp(m_s - M)
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                    float* __restrict__ out, int num_heads, int head_dim, int nsplit) {
    const int h = blockIdx.x, b = blockIdx.y;
    const size_t base = (static_cast<size_t>(b) * num_heads + h) * nsplit;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_ml[2 * (base + s)]);
    float L = 0.f;
    for (int s = 0; s < nsplit; ++s) {
        const float ms = part_ml[2 * (base + s)];
        if (ms != -INFINITY) L += part_ml[2 * (base + s) + 1] * expf(ms - M);
    }
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float o = 0.f;
        for (int s = 0; s < nsplit; ++s) {
            const float ms = part_ml[2 * (base + s)];
            if (ms != -INFINITY) o += part_o[(base + s) * head_dim + d] * expf(ms - M);
        }
        out[(static_cast<size_t>(b) * num_heads + h) * head_dim + d] = o / L;
    }
}

// out[r, i] = silu(gate[r*ld + i]) * up[r*ld + i], silu(x) = x / (1 + exp(-x))
// (src/tensor.h:1050-1064); out is rows x n, row-major.
__global__ void silu_mul_kernel(float* __restrict__ out, const float* __restrict__ gate, const float* __restrict__ up,
                                int n, int rows, int ld) {
    const int64_t total = static_cast<int64_t>(n) * rows;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / n, c = i - r * n;
        const float g = gate[r * ld + c];
        out[i] = g / (1.0f + expf(-g)) * up[r * ld + c];
    }
}

// x += y (the residual adds of src/model.h:363, 541).
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] += y[i];
}

// x[b] = table[token[b]] (fp32 rows, src/model.h:265).
__global__ void embed_kernel(float* __restrict__ x, const float* __restrict__ table, const int* __restrict__ tokens,
                             int dim) {
    const int b = blockIdx.y;
    const float* row = table + static_cast<size_t>(tokens[b]) * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        x[static_cast<size_t>(b) * dim + i] = row[i];
}

// Greedy next token: the first index of the row maximum.  One CTA per row;
// writes tokens[b] and, when history is given, history[step * B + b].
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int n, int* __restrict__ tokens,
                                                      int* __restrict__ history, const int* __restrict__ step_p) {
    const int b = blockIdx.x;
    const float* row = logits + static_cast<size_t>(b) * n;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = row[i];
        if (v > best || (v == best && i < bi)) { best = v; bi = i; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int nw = blockDim.x >> 5;
        best = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
        bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        if (threadIdx.x == 0) {
            tokens[b] = bi;
            if (history) history[static_cast<size_t>(*step_p) * gridDim.x + b] = bi;
        }
    }
}

__global__ void advance_kernel(int* pos, int* step) {
    *pos += 1;
    if (step) *step += 1;
}

int grid_for(int64_t n, int num_sms) {
    const int64_t g = (n + 255) / 256;
    return static_cast<int>(g < 4LL * num_sms ? (g > 0 ? g : 1) : 4LL * num_sms);
}

}  // namespace

cudaError_t rmsnorm_launch(float* out, const float* x, const float* w, int n, float eps, int rows, cudaStream_t s) {
    rmsnorm_kernel<<<rows, 256, 0, s>>>(out, x, w, n, eps);
    return cudaGetLastError();
}

cudaError_t rope_kv_launch(float* q, const float* k, const float* v, float* kcache, float* vcache, const int* pos,
                           const float* freqs, int q_dim, int kv_dim, int head_dim, int rope_dim, int neox, int rows,
                           int max_seq, int num_sms, cudaStream_t s) {
    const int items = (q_dim / head_dim + kv_dim / head_dim) * (rope_dim / 2) + kv_dim;
    const dim3 grid(static_cast<unsigned>(grid_for(items, num_sms)), static_cast<unsigned>(rows));
    rope_kv_kernel<<<grid, 256, 0, s>>>(q, k, v, kcache, vcache, pos, freqs, q_dim, kv_dim, head_dim, rope_dim, neox,
                                        max_seq);
    return cudaGetLastError();
}

int attention_splits(int rows, int num_kv_heads, int max_seq, int num_sms) {
    int splits = (2 * num_sms + rows * num_kv_heads - 1) / (rows * num_kv_heads);
    splits = splits < 1 ? 1 : splits;
    const int max_splits = (max_seq + 15) / 16;  // at least 16 positions per split
    return splits > max_splits ? max_splits : splits;
}

template <int MUL>
static cudaError_t attn_split_per(int per, dim3 grid, cudaStream_t s, const float* q, const float* kc, const float* vc,
                                  const int* pos, float* po, float* pml, int nh, int nkv, int max_seq, int chunk) {
    switch (per) {
        case 2: attn_split_kernel<MUL, 2><<<grid, ATT_THREADS, 0, s>>>(q, kc, vc, pos, po, pml, nh, nkv, max_seq, chunk); break;
        case 4: attn_split_kernel<MUL, 4><<<grid, ATT_THREADS, 0, s>>>(q, kc, vc, pos, po, pml, nh, nkv, max_seq, chunk); break;
        case 8: attn_split_kernel<MUL, 8><<<grid, ATT_THREADS, 0, s>>>(q, kc, vc, pos, po, pml, nh, nkv, max_seq, chunk); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t attention_launch(float* out, const float* q, const float* kcache, const float* vcache, const int* pos,
                             float* part_o, float* part_ml, int num_heads, int num_kv_heads, int head_dim, int rows,
                             int max_seq, int splits, cudaStream_t s) {
    if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || head_dim % 32 != 0) return cudaErrorInvalidValue;
    const int mul = num_heads / num_kv_heads, per = head_dim / 32;
    const int chunk = (max_seq + splits - 1) / splits;
    const dim3 grid(splits, num_kv_heads, rows);
    cudaError_t e;
    switch (mul) {
        case 1: e = attn_split_per<1>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, num_heads, num_kv_heads, max_seq, chunk); break;
        case 2: e = attn_split_per<2>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, num_heads, num_kv_heads, max_seq, chunk); break;
        case 4: e = attn_split_per<4>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, num_heads, num_kv_heads, max_seq, chunk); break;
        case 8: e = attn_split_per<8>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, num_heads, num_kv_heads, max_seq, chunk); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    attn_combine_kernel<<<dim3(num_heads, rows), 128, 0, s>>>(part_o, part_ml, out, num_heads, head_dim, splits);
    return cudaGetLastError();
}

cudaError_t silu_mul_launch(float* out, const float* gate, const float* up, int n, int rows, int ld, int num_sms,
                            cudaStream_t s) {
    silu_mul_kernel<<<grid_for(static_cast<int64_t>(n) * rows, num_sms), 256, 0, s>>>(out, gate, up, n, rows, ld);
    return cudaGetLastError();
}

cudaError_t add_launch(float* x, const float* y, int64_t n, int num_sms, cudaStream_t s) {
    add_kernel<<<grid_for(n, num_sms), 256, 0, s>>>(x, y, n);
    return cudaGetLastError();
}

cudaError_t embed_launch(float* x, const float* table, const int* tokens, int dim, int rows, cudaStream_t s) {
    embed_kernel<<<dim3((dim + 255) / 256, rows), 256, 0, s>>>(x, table, tokens, dim);
    return cudaGetLastError();
}

cudaError_t argmax_launch(const float* logits, int n, int rows, int* tokens, int* history, const int* step,
                          cudaStream_t s) {
    argmax_kernel<<<rows, 1024, 0, s>>>(logits, n, tokens, history, step);
    return cudaGetLastError();
}

cudaError_t advance_launch(int* pos, int* step, cudaStream_t s) {
    advance_kernel<<<1, 1, 0, s>>>(pos, step);
    return cudaGetLastError();
}

}  // namespace swq
