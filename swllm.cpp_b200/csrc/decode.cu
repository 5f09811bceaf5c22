// decode.cu -- the device-resident decode step around the quantized GEMVs:
// embedding row, RMSNorm (alone or fused with the residual add before it),
// RoPE + KV-cache append, decode attention, SiLU-mul, residual add, argmax
// (the reference's Model::forward, src/model.h:257-543, with its Compute
// helpers, src/tensor.h:1028-1180).
//
// All activations are fp32, as in the reference.  B sequences decode in step
// (same position); row b of every [B x n] buffer belongs to sequence b.  The
// position lives in device memory (`pos`, advanced by advance_kernel) so a
// whole decode step can be captured once in a CUDA graph and replayed.
//
// KV cache layout (fp32): [layer][sequence b][position t][kv_dim].
//
// Every kernel here is launched as a programmatic dependent of the kernel
// before it on the stream: it is resident early and begins with
// griddepcontrol.wait, so nothing here touches memory before its predecessor
// completed.  It lets its own dependents launch (griddepcontrol.launch_dependents)
// only once its work is done: the GEMV that usually follows spreads one CTA per
// SM over a GPU that no longer holds the previous GEMV's CTAs.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <cstdint>

#include "decode.h"
#include "swq_device.cuh"

namespace swq {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over the CTA (blockDim.x a multiple of 32, at most 1024); every thread
// gets the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float u = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        u = warp_sum(u);
        if (threadIdx.x == 0) red[32] = u;
    }
    __syncthreads();
    return red[32];
}

// RMSNorm of each row, optionally after the residual add x += y:
//   out = x / sqrt(mean(x^2) + eps) * w      (src/tensor.h:1028-1033)
// One CTA per row; VEC: n % 4 == 0 and 16-byte aligned rows.  With y, x is
// updated in place first (src/model.h:363-366 and 519-520 in one pass).
template <bool VEC, bool ADD>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(float* __restrict__ out, float* __restrict__ x,
                                                       const float* __restrict__ y, const float* __restrict__ w,
                                                       int n, float eps) {
    pdl_wait_primary();
    __shared__ float red[33];
    float* xr = x + static_cast<size_t>(blockIdx.x) * n;
    const float* yr = ADD ? y + static_cast<size_t>(blockIdx.x) * n : nullptr;
    float* orow = out + static_cast<size_t>(blockIdx.x) * n;
    float ss = 0.f;
    if (VEC) {
        float4* x4 = reinterpret_cast<float4*>(xr);
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
            float4 a = x4[i];
            if (ADD) {
                const float4 b = reinterpret_cast<const float4*>(yr)[i];
                a.x += b.x;
                a.y += b.y;
                a.z += b.z;
                a.w += b.w;
                x4[i] = a;
            }
            ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            float a = xr[i];
            if (ADD) {
                a += yr[i];
                xr[i] = a;
            }
            ss = fmaf(a, a, ss);
        }
    }
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    if (VEC) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        const float4* w4 = reinterpret_cast<const float4*>(w);
        float4* o4 = reinterpret_cast<float4*>(orow);
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
            const float4 a = x4[i], g = w4[i];
            o4[i] = make_float4(a.x * scale * g.x, a.y * scale * g.y, a.z * scale * g.z, a.w * scale * g.w);
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = xr[i] * scale * w[i];
    }
}

// RoPE on q (in place) and k, then k and v into the cache at `pos`.
// Interleaved pairs (2i, 2i+1) (src/tensor.h:1068-1107) or, with neox, pairs
// (i, i + rope_dim/2) (src/tensor.h:1121-1161); angle = pos * freqs[i].
// Row b of q / k / v starts at b * ldq / ldk / ldv.
__global__ void rope_kv_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                               float* __restrict__ kcache, float* __restrict__ vcache, const int* __restrict__ pos_p,
                               const float* __restrict__ freqs, int q_dim, int kv_dim, int head_dim, int rope_dim,
                               int neox, int max_seq, int ldq, int ldk, int ldv) {
    pdl_wait_primary();
    const int b = blockIdx.y;
    const int pos = *pos_p;
    const int half = rope_dim / 2;
    const int qpairs = (q_dim / head_dim) * half, kpairs = (kv_dim / head_dim) * half;
    float* qb = q + static_cast<size_t>(b) * ldq;
    const float* kb = k + static_cast<size_t>(b) * ldk;
    const float* vb = v + static_cast<size_t>(b) * ldv;
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
// handles a slice of the timesteps for the MUL query heads that share the
// kv head (src/model.h:329-361: score = q.k / sqrt(head_dim), softmax over
// t <= pos, out = sum softmax * v), keeping a running max m, the sum l of
// exp(score - m) and the unnormalised output.  Each CTA writes its partial
// (m, l, o) per head; the last CTA of a (sequence, kv head) to finish -- an
// atomic count in the workspace, reset by that CTA -- merges the splits.
constexpr int ATT_MAXSPLIT = 64;  // the merge keeps MUL x splits weights in the partial buffer

// Warps per CTA and consecutive positions a warp takes at once; the CTA's
// per-warp partials (NW x MUL x head_dim floats) stay within 32 KB.
template <int MUL, int PER>
struct AttCfg {
    static constexpr int NW = MUL * PER <= 32 ? 8 : 4;
    static constexpr int U = PER <= 4 ? 8 : 4;
    static constexpr int THREADS = NW * 32;
    static constexpr int MINCHUNK = NW * U;  // positions per split at least
};

// MUL query heads per kv head, PER = head_dim / 32 elements per lane.
// The live context [0, pos] is cut into ns = ceil(n_ctx / chunk) splits of
// chunk = max(MINCHUNK, ceil(n_ctx / gridDim.x)) positions (worked out on the
// device from pos, so a captured launch adapts to the position); CTAs past ns
// return at once.  Inside a split, warp w takes positions w U .. w U + U - 1,
// then the next NW U: all their K and V loads are issued before any
// arithmetic, then one online-softmax update per query head for the U scores.
template <int MUL, int PER>
__global__ void __launch_bounds__(AttCfg<MUL, PER>::THREADS) attn_kernel(
    const float* __restrict__ q, const float* __restrict__ kcache, const float* __restrict__ vcache,
    const int* __restrict__ pos_p, float* __restrict__ part_o, float* __restrict__ part_ml,
    unsigned* __restrict__ done, float* __restrict__ out, int num_heads, int num_kv_heads, int max_seq, int ldq) {
    pdl_wait_primary();
    using C = AttCfg<MUL, PER>;
    constexpr int HD = 32 * PER;
    constexpr int NW = C::NW, U = C::U, NT = C::THREADS;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int ns_grid = gridDim.x;  // slot stride of the partials
    const int kv_dim = num_kv_heads * HD;
    const int n_ctx = min(*pos_p + 1, max_seq);
    const int chunk = max(C::MINCHUNK, (n_ctx + ns_grid - 1) / ns_grid);
    const int nsplit = (n_ctx + chunk - 1) / chunk;
    if (split >= nsplit) return;
    const int t0 = split * chunk, t1 = min(n_ctx, t0 + chunk);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(HD));
    __shared__ float s_m[NW][MUL], s_l[NW][MUL];
    __shared__ float s_o[NW][MUL][HD];
    __shared__ unsigned s_last;

    float qv[MUL][PER], acc[MUL][PER], m[MUL], l[MUL];
#pragma unroll
    for (int j = 0; j < MUL; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
        const float* qh = q + static_cast<size_t>(b) * ldq + (kvh * MUL + j) * HD;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            acc[j][e] = 0.f;
            qv[j][e] = qh[e * 32 + lane] * inv_sqrt;
        }
    }
    const float* kbase = kcache + static_cast<size_t>(b) * max_seq * kv_dim + kvh * HD;
    const float* vbase = vcache + static_cast<size_t>(b) * max_seq * kv_dim + kvh * HD;
    for (int tb = t0 + warp * U; tb < t1; tb += NW * U) {
        float kk[U][PER], vv[U][PER];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = min(tb + u, t1 - 1);  // past the end: a repeat, masked below
            const float* kt = kbase + static_cast<size_t>(t) * kv_dim;
            const float* vt = vbase + static_cast<size_t>(t) * kv_dim;
#pragma unroll
            for (int e = 0; e < PER; ++e) {
                kk[u][e] = __ldcg(kt + e * 32 + lane);
                vv[u][e] = __ldcg(vt + e * 32 + lane);
            }
        }
#pragma unroll
        for (int j = 0; j < MUL; ++j) {
            float sc[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < PER; ++e) d = fmaf(qv[j][e], kk[u][e], d);
                sc[u] = d;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                for (int u = 0; u < U; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
            }
            float mn = m[j];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (tb + u >= t1) sc[u] = -INFINITY;
                mn = fmaxf(mn, sc[u]);
            }
            const float corr = expf(m[j] - mn);
            float ps = 0.f;
#pragma unroll
            for (int e = 0; e < PER; ++e) acc[j][e] *= corr;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float pe = expf(sc[u] - mn);
                ps += pe;
#pragma unroll
                for (int e = 0; e < PER; ++e) acc[j][e] = fmaf(pe, vv[u][e], acc[j][e]);
            }
            l[j] = l[j] * corr + ps;
            m[j] = mn;
        }
    }
    // merge the warps of the CTA into this split's partial
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
    for (int idx = threadIdx.x; idx < MUL * HD; idx += NT) {
        const int j = idx / HD, d = idx % HD;
        float mm = -INFINITY;
        for (int w = 0; w < NW; ++w) mm = fmaxf(mm, s_m[w][j]);
        float ll = 0.f, oo = 0.f;
        for (int w = 0; w < NW; ++w) {
            const float c = s_m[w][j] == -INFINITY ? 0.f : expf(s_m[w][j] - mm);
            ll += s_l[w][j] * c;
            oo += s_o[w][j][d] * c;
        }
        const size_t slot = (static_cast<size_t>(b) * num_heads + kvh * MUL + j) * ns_grid + split;
        part_o[slot * HD + d] = oo;
        if (d == 0) {
            part_ml[2 * slot] = mm;
            part_ml[2 * slot + 1] = ll;
        }
    }
    // the last split of this (sequence, kv head) merges all splits
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* cnt = done + static_cast<size_t>(b) * num_kv_heads + kvh;
        s_last = atomicAdd(cnt, 1u) == static_cast<unsigned>(nsplit - 1);
        if (s_last) *cnt = 0u;  // ready for the next call
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // weight of split s for head j: exp(m_s - M) / sum_s' l_s' exp(m_s' - M)
    float* s_w = &s_o[0][0][0];  // MUL x nsplit (nsplit <= ATT_MAXSPLIT)
    for (int j = warp; j < MUL; j += NW) {
        const size_t base = (static_cast<size_t>(b) * num_heads + kvh * MUL + j) * ns_grid;
        float M = -INFINITY;
        for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, __ldcg(&part_ml[2 * (base + s)]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.f;
        for (int s = lane; s < nsplit; s += 32) {
            const float ms = __ldcg(&part_ml[2 * (base + s)]);
            const float c = ms == -INFINITY ? 0.f : expf(ms - M);
            s_w[j * nsplit + s] = c;
            L += __ldcg(&part_ml[2 * (base + s) + 1]) * c;
        }
        L = warp_sum(L);
        for (int s = lane; s < nsplit; s += 32) s_w[j * nsplit + s] /= L;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < MUL * HD; idx += NT) {
        const int j = idx / HD, d = idx % HD;
        const size_t base = (static_cast<size_t>(b) * num_heads + kvh * MUL + j) * ns_grid;
        // eight partials in flight per batch (the loads do not wait on the sum)
        float o = 0.f;
        for (int s0 = 0; s0 < nsplit; s0 += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = s0 + u < nsplit ? __ldcg(&part_o[(base + s0 + u) * HD + d]) : 0.f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (s0 + u < nsplit) o = fmaf(v[u], s_w[j * nsplit + s0 + u], o);
        }
        out[(static_cast<size_t>(b) * num_heads + kvh * MUL + j) * HD + d] = o;
    }
}

// out[r, i] = silu(gate[r*ld + i]) * up[r*ld + i], silu(x) = x / (1 + exp(-x))
// (src/tensor.h:1050-1064); out is rows x n, row-major.
__global__ void silu_mul_kernel(float* __restrict__ out, const float* __restrict__ gate, const float* __restrict__ up,
                                int n, int rows, int ld, int vec) {
    pdl_wait_primary();
    // rows over grid y, columns over grid x; 4 columns per thread when every
    // row of the three arrays starts 16-byte aligned
    for (int r = blockIdx.y; r < rows; r += gridDim.y) {
        const float* g = gate + static_cast<size_t>(r) * ld;
        const float* u = up + static_cast<size_t>(r) * ld;
        float* o = out + static_cast<size_t>(r) * n;
        if (vec) {
            for (int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x); c < n; c += 4 * gridDim.x * blockDim.x) {
                const float4 gv = *reinterpret_cast<const float4*>(g + c);
                const float4 uv = *reinterpret_cast<const float4*>(u + c);
                float4 ov;
                ov.x = gv.x / (1.0f + expf(-gv.x)) * uv.x;
                ov.y = gv.y / (1.0f + expf(-gv.y)) * uv.y;
                ov.z = gv.z / (1.0f + expf(-gv.z)) * uv.z;
                ov.w = gv.w / (1.0f + expf(-gv.w)) * uv.w;
                *reinterpret_cast<float4*>(o + c) = ov;
            }
        } else {
            for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
                const float gv = g[c];
                o[c] = gv / (1.0f + expf(-gv)) * u[c];
            }
        }
    }
}

// x += y (the residual adds of src/model.h:363, 541).
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
    pdl_wait_primary();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] += y[i];
}

// x[b] = table[token[b]] (fp32 rows, src/model.h:265); a token id outside
// [0, vocab) reads row 0.
__global__ void embed_kernel(float* __restrict__ x, const float* __restrict__ table, const int* __restrict__ tokens,
                             int dim, int vocab) {
    pdl_wait_primary();
    const int b = blockIdx.y;
    const int tok = tokens[b];
    const float* row = table + static_cast<size_t>(tok >= 0 && tok < vocab ? tok : 0) * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        x[static_cast<size_t>(b) * dim + i] = row[i];
}

__device__ __forceinline__ void better(float v, int i, float& best, int& bi) {
    if (v > best || (v == best && i < bi)) {
        best = v;
        bi = i;
    }
}

// Greedy next token: the first index of the row maximum.  One CTA per row;
// writes tokens[b] and, when history is given, history[step * B + b].
template <bool VEC>
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int n, int* __restrict__ tokens,
                                                      int* __restrict__ history, const int* __restrict__ step_p) {
    pdl_wait_primary();
    const int b = blockIdx.x;
    const float* row = logits + static_cast<size_t>(b) * n;
    // index 0 until a larger value is seen: a row of NaN still yields a valid token
    float best = -INFINITY;
    int bi = 0;
    if (VEC) {
        const float4* r4 = reinterpret_cast<const float4*>(row);
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
            const float4 v = r4[i];
            better(v.x, 4 * i, best, bi);
            better(v.y, 4 * i + 1, best, bi);
            better(v.z, 4 * i + 2, best, bi);
            better(v.w, 4 * i + 3, best, bi);
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) better(row[i], i, best, bi);
    }
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        better(__shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o), best, bi);
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int nw = blockDim.x >> 5;
        best = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
        bi = threadIdx.x < nw ? si[threadIdx.x] : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            better(__shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o), best, bi);
        if (threadIdx.x == 0) {
            tokens[b] = bi;
            if (history) history[static_cast<size_t>(*step_p) * gridDim.x + b] = bi;
        }
    }
}

__global__ void advance_kernel(int* pos, int* step) {
    pdl_wait_primary();
    *pos += 1;
    if (step) *step += 1;
}

// Launch as a programmatic dependent of the previous kernel on the stream.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

int grid_for(int64_t n, int num_sms) {
    const int64_t g = (n + 255) / 256;
    return static_cast<int>(g < 4LL * num_sms ? (g > 0 ? g : 1) : 4LL * num_sms);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define ERR_RET(call)                            \
    do {                                         \
        const cudaError_t e_ = (call);           \
        if (e_ != cudaSuccess) return e_;        \
    } while (0)

}  // namespace

cudaError_t rmsnorm_launch(float* out, float* x, const float* y, const float* w, int n, float eps, int rows,
                           cudaStream_t s) {
    const bool vec = n % 4 == 0 && aligned16(out) && aligned16(x) && aligned16(w) && (!y || aligned16(y));
    const int threads = std::min(1024, std::max(32, ((vec ? n / 4 : n) + 31) / 32 * 32));
    if (y) {
        if (vec) ERR_RET(launch_pdl(rmsnorm_kernel<true, true>, dim3(rows), dim3(threads), s, out, x, y, w, n, eps));
        else ERR_RET(launch_pdl(rmsnorm_kernel<false, true>, dim3(rows), dim3(threads), s, out, x, y, w, n, eps));
    } else {
        if (vec) ERR_RET(launch_pdl(rmsnorm_kernel<true, false>, dim3(rows), dim3(threads), s, out, x, nullptr, w, n, eps));
        else ERR_RET(launch_pdl(rmsnorm_kernel<false, false>, dim3(rows), dim3(threads), s, out, x, nullptr, w, n, eps));
    }
    return cudaGetLastError();
}

cudaError_t rope_kv_launch(float* q, const float* k, const float* v, float* kcache, float* vcache, const int* pos,
                           const float* freqs, int q_dim, int kv_dim, int head_dim, int rope_dim, int neox, int rows,
                           int max_seq, int ldq, int ldk, int ldv, int num_sms, cudaStream_t s) {
    const int items = (q_dim / head_dim + kv_dim / head_dim) * (rope_dim / 2) + kv_dim;
    const dim3 grid(static_cast<unsigned>(grid_for(items, num_sms)), static_cast<unsigned>(rows));
    ERR_RET(launch_pdl(rope_kv_kernel, dim3(grid), dim3(256), s, q, k, v, kcache, vcache, pos, freqs, q_dim, kv_dim, head_dim, rope_dim, neox, max_seq, ldq, ldk, ldv));
    return cudaGetLastError();
}

int attention_splits(int rows, int num_kv_heads, int max_seq, int num_sms) {
    int splits = (2 * num_sms + rows * num_kv_heads - 1) / (rows * num_kv_heads);
    splits = splits < 1 ? 1 : splits;
    int max_splits = (max_seq + 31) / 32;  // at least 32 positions per split
    max_splits = max_splits < ATT_MAXSPLIT ? max_splits : ATT_MAXSPLIT;
    return splits > max_splits ? max_splits : splits;
}

size_t attention_workspace(int num_heads, int num_kv_heads, int head_dim, int rows, int splits) {
    const size_t slots = static_cast<size_t>(rows) * num_heads * splits;
    return slots * (static_cast<size_t>(head_dim) + 2) * sizeof(float) +
           static_cast<size_t>(rows) * num_kv_heads * sizeof(unsigned);
}

template <int MUL>
static cudaError_t attn_per(int per, dim3 grid, cudaStream_t s, const float* q, const float* kc, const float* vc,
                            const int* pos, float* po, float* pml, unsigned* done, float* out, int nh, int nkv,
                            int max_seq, int ldq) {
    switch (per) {
        case 2:
            ERR_RET(launch_pdl(attn_kernel<MUL, 2>, dim3(grid), dim3(AttCfg<MUL, 2>::THREADS), s, q, kc, vc, pos, po, pml, done, out, nh, nkv, max_seq, ldq));
            break;
        case 4:
            ERR_RET(launch_pdl(attn_kernel<MUL, 4>, dim3(grid), dim3(AttCfg<MUL, 4>::THREADS), s, q, kc, vc, pos, po, pml, done, out, nh, nkv, max_seq, ldq));
            break;
        case 8:
            ERR_RET(launch_pdl(attn_kernel<MUL, 8>, dim3(grid), dim3(AttCfg<MUL, 8>::THREADS), s, q, kc, vc, pos, po, pml, done, out, nh, nkv, max_seq, ldq));
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t attention_launch(float* out, const float* q, const float* kcache, const float* vcache, const int* pos,
                             void* workspace, int num_heads, int num_kv_heads, int head_dim, int rows, int max_seq,
                             int splits, int ldq, cudaStream_t s) {
    if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || head_dim % 32 != 0) return cudaErrorInvalidValue;
    const int mul = num_heads / num_kv_heads, per = head_dim / 32;
    const dim3 grid(splits, num_kv_heads, rows);
    float* part_o = static_cast<float*>(workspace);
    float* part_ml = part_o + static_cast<size_t>(rows) * num_heads * splits * head_dim;
    unsigned* done = reinterpret_cast<unsigned*>(part_ml + static_cast<size_t>(rows) * num_heads * splits * 2);
    switch (mul) {
        case 1: return attn_per<1>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, done, out, num_heads, num_kv_heads, max_seq, ldq);
        case 2: return attn_per<2>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, done, out, num_heads, num_kv_heads, max_seq, ldq);
        case 4: return attn_per<4>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, done, out, num_heads, num_kv_heads, max_seq, ldq);
        case 8: return attn_per<8>(per, grid, s, q, kcache, vcache, pos, part_o, part_ml, done, out, num_heads, num_kv_heads, max_seq, ldq);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t silu_mul_launch(float* out, const float* gate, const float* up, int n, int rows, int ld, int num_sms,
                            cudaStream_t s) {
    const int vec = (n % 4 == 0 && ld % 4 == 0 && ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(gate) |
                                                    reinterpret_cast<uintptr_t>(up)) & 15u) == 0) ? 1 : 0;
    const int per = vec ? 4 * 256 : 256;
    int gx = (n + per - 1) / per;
    int gy = std::min(rows, 65535);
    // about four CTAs per SM in all, at least one column block per row
    const int want = std::max(1, 4 * num_sms / std::max(1, gy));
    gx = std::max(1, std::min(gx, want));
    ERR_RET(launch_pdl(silu_mul_kernel, dim3(gx, gy), dim3(256), s, out, gate, up, n, rows, ld, vec));
    return cudaGetLastError();
}

cudaError_t add_launch(float* x, const float* y, int64_t n, int num_sms, cudaStream_t s) {
    ERR_RET(launch_pdl(add_kernel, dim3(grid_for(n, num_sms)), dim3(256), s, x, y, n));
    return cudaGetLastError();
}

cudaError_t embed_launch(float* x, const float* table, const int* tokens, int dim, int vocab, int rows,
                         cudaStream_t s) {
    ERR_RET(launch_pdl(embed_kernel, dim3((dim + 255) / 256, rows), dim3(256), s, x, table, tokens, dim, vocab));
    return cudaGetLastError();
}

cudaError_t argmax_launch(const float* logits, int n, int rows, int* tokens, int* history, const int* step,
                          cudaStream_t s) {
    if (n % 4 == 0 && aligned16(logits))
        ERR_RET(launch_pdl(argmax_kernel<true>, dim3(rows), dim3(1024), s, logits, n, tokens, history, step));
    else
        ERR_RET(launch_pdl(argmax_kernel<false>, dim3(rows), dim3(1024), s, logits, n, tokens, history, step));
    return cudaGetLastError();
}

cudaError_t advance_launch(int* pos, int* step, cudaStream_t s) {
    ERR_RET(launch_pdl(advance_kernel, dim3(1), dim3(1), s, pos, step));
    return cudaGetLastError();
}

}  // namespace swq
