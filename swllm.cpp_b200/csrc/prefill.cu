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
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <cstdint>

#include "gemm_tc.h"  // scratch_alloc / scratch_free
#include "prefill.h"
#include "swq_device.cuh"

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


// Causal attention for a whole prompt on the tensor cores (head_dim 64 and
// 128): CTA = (64 query rows of one sequence, query head h), 4 warps of 16
// rows; key/value positions stream through shared memory in tiles of 64.
//
// Operands are fp16 pairs: a row x of Q or K is scaled by 2^(13 - E) (E: its
// largest binary exponent) and split x = h + l (h = fp16 of the scaled
// value, l = fp16 of the rest: 22 bits relative to the row's largest
// element); S = Q K^T takes h.h + h.l + l.h on m16n8k16 MMAs with fp32
// accumulation, then the row scales 2^(E - 13) and 1 / sqrt(head_dim) in
// fp32.  P = exp(S - m) (online softmax per row in fp32) and V are split the
// same way (V unscaled, except rows past 2^15 in magnitude, scaled down by a
// power of two that P takes back) for O += P V.  Every product is exact; the
// dropped l.l terms sit 2^-22 below the kept ones.  The reference's loops
// (src/model.h:329-361) round every product and sum in fp32 instead.
//
// Fragments: Q (A) and K (B of S) as 32-bit shared loads (rows padded to
// HD + 8 halves: the 8 rows x 4 pairs of a fragment hit 32 distinct banks);
// P (A of O) straight from the S accumulators; V (B of O) by ldmatrix.trans
// from its row-major tile.
namespace amma {

__device__ __forceinline__ uint32_t lds32(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const __half* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ uint32_t h2(float a, float b) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Split a and b into fp16 h (returned) and l (lo).
__device__ __forceinline__ uint32_t split2(float a, float b, uint32_t& lo) {
    const __half2 hv = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(hv);
    lo = h2(a - hf.x, b - hf.y);
    return *reinterpret_cast<const uint32_t*>(&hv);
}

// One row of HD fp32 values (src; null = zeros), 8 lanes (sub = lane & 7) of
// HD / 8 each, into h / l rows of shared memory.  SCALE_TO_TOP: scaled to
// below 2^13, *aux = 2^(E - 13) (NaN for a non-finite row); else unscaled
// unless the row reaches 2^15 (then scaled down, *aux = the factor back).
template <int HD, bool SCALE_TO_TOP>
__device__ __forceinline__ void stage_row(const float* src, __half* dh, __half* dl, float* aux, int sub) {
    constexpr int PER = HD / 8;
    float v[PER];
    if (src) {
#pragma unroll
        for (int i = 0; i < PER; i += 4) {
            const float4 f = *reinterpret_cast<const float4*>(src + sub * PER + i);
            v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) v[i] = 0.f;
    }
    float mx = 0.f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        mx = fmaxf(mx, fabsf(v[i]));
        bad |= !(fabsf(v[i]) <= 3.402823466e38f);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad ? 1 : 0, o) != 0;
    }
    const int E = max(((__float_as_int(mx) >> 23) & 0xFF) - 126, -100);  // mx < 2^E
    float up, back;
    if (SCALE_TO_TOP) {
        up = __int_as_float((127 + 13 - E) << 23);
        back = __int_as_float((127 + E - 13) << 23);
    } else {
        const int k = max(E - 15, 0);
        up = __int_as_float((127 - k) << 23);
        back = __int_as_float((127 + k) << 23);
    }
    if (bad) {
        up = 0.f;
        back = __int_as_float(0x7fc00000);
    }
    uint32_t H[PER / 2], L[PER / 2];
#pragma unroll
    for (int i = 0; i < PER; i += 2) H[i / 2] = split2(v[i] * up, v[i + 1] * up, L[i / 2]);
    if (dh == nullptr) return;  // a row past the end (the shuffles above need all 8 lanes)
#pragma unroll
    for (int i = 0; i < PER / 2; i += 2) {
        *reinterpret_cast<uint2*>(dh + sub * PER + 2 * i) = make_uint2(H[i], H[i + 1]);
        *reinterpret_cast<uint2*>(dl + sub * PER + 2 * i) = make_uint2(L[i], L[i + 1]);
    }
    if (sub == 0) *aux = back;
}

// 16 bytes global -> shared, asynchronous; src_bytes 0 fills zeros (a row past
// the context) and reads nothing.
__device__ __forceinline__ void cp16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp8(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace amma

template <int HD>
__global__ void __launch_bounds__(128, 2) attention_prefill_mma(
    float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ kcache,
    const float* __restrict__ vcache, int pos0, int seq_len, int num_heads, int num_kv_heads, int max_seq, int ldq,
    int ldo) {
    using namespace amma;
    constexpr int BM = 64, BN = 64, ST = HD + 8;  // row stride in halves
    constexpr int NB = BN / 8, ND = HD / 8, KS = HD / 16;
    extern __shared__ __align__(16) uint8_t amsm[];
    __half* Qh = reinterpret_cast<__half*>(amsm);
    __half* Ql = Qh + BM * ST;
    __half* Kh = Ql + BM * ST;
    __half* Kl = Kh + BN * ST;
    __half* Vh = Kl + BN * ST;
    __half* Vl = Vh + BN * ST;
    float* qinv = reinterpret_cast<float*>(Vl + BN * ST);
    float* kinv = qinv + BM;
    float* vmul = kinv + BN;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int sub = lane & 7, rsub = lane >> 3;  // staging: 4 rows per warp pass, 8 lanes a row
    // heavier (later) query tiles first: the causal work grows with the tile
    const int qt = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int p0 = qt * BM;
    const int nrow = min(BM, seq_len - p0);
    const int kvh = h / (num_heads / num_kv_heads);
    const int kv_dim = num_kv_heads * HD;
    const size_t m0 = static_cast<size_t>(seq) * seq_len + p0;
    for (int r = 4 * warp + rsub; r < BM; r += 16)
        stage_row<HD, true>(r < nrow ? q + (m0 + r) * ldq + h * HD : nullptr, Qh + r * ST, Ql + r * ST, qinv + r,
                            sub);
    const float* kb = kcache + static_cast<size_t>(seq) * max_seq * kv_dim + kvh * HD;
    const float* vb = vcache + static_cast<size_t>(seq) * max_seq * kv_dim + kvh * HD;
    const float rsqrt_hd = 1.0f / sqrtf(static_cast<float>(HD));
    const int r0 = 16 * warp + g, r1 = r0 + 8;  // this lane's two query rows in the tile
    const int qpos0 = pos0 + p0 + r0, qpos1 = pos0 + p0 + r1;
    const bool live0 = r0 < nrow, live1 = r1 < nrow;
    float O[ND][4];
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) O[nd][0] = O[nd][1] = O[nd][2] = O[nd][3] = 0.f;
    float m_0 = -INFINITY, m_1 = -INFINITY, l_0 = 0.f, l_1 = 0.f;
    const int last = pos0 + p0 + nrow - 1;  // last key position any row of the tile sees
    for (int t0 = 0; t0 <= last; t0 += BN) {
        __syncthreads();  // the previous tile's K and V are consumed (and Q staged)
        for (int r = 4 * warp + rsub; r < BN; r += 16) {
            const bool in = t0 + r <= last;
            stage_row<HD, true>(in ? kb + static_cast<size_t>(t0 + r) * kv_dim : nullptr, Kh + r * ST, Kl + r * ST,
                                kinv + r, sub);
            stage_row<HD, false>(in ? vb + static_cast<size_t>(t0 + r) * kv_dim : nullptr, Vh + r * ST, Vl + r * ST,
                                 vmul + r, sub);
        }
        __syncthreads();
        // S = Q K^T for this warp's 16 rows x 64 keys
        float S[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) S[nb][0] = S[nb][1] = S[nb][2] = S[nb][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int c = ks * 16 + 2 * t;
            uint32_t ah[4], al[4];
            ah[0] = lds32(Qh + r0 * ST + c);
            ah[1] = lds32(Qh + r1 * ST + c);
            ah[2] = lds32(Qh + r0 * ST + c + 8);
            ah[3] = lds32(Qh + r1 * ST + c + 8);
            al[0] = lds32(Ql + r0 * ST + c);
            al[1] = lds32(Ql + r1 * ST + c);
            al[2] = lds32(Ql + r0 * ST + c + 8);
            al[3] = lds32(Ql + r1 * ST + c + 8);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                const __half* kh = Kh + (nb * 8 + g) * ST + c;
                const __half* kl = Kl + (nb * 8 + g) * ST + c;
                const uint32_t bh0 = lds32(kh), bh1 = lds32(kh + 8), bl0 = lds32(kl), bl1 = lds32(kl + 8);
                mma16816(S[nb], ah, bh0, bh1);
                mma16816(S[nb], ah, bl0, bl1);
                mma16816(S[nb], al, bh0, bh1);
            }
        }
        // scores, causal mask, online softmax (rows r0, r1: the 4 lanes t of a row)
        const float qs0 = qinv[r0] * rsqrt_hd, qs1 = qinv[r1] * rsqrt_hd;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int j = nb * 8 + 2 * t + c, key = t0 + j;
                const float ki = kinv[j];
                S[nb][c] = (live0 && key <= qpos0) ? S[nb][c] * ki * qs0 : -INFINITY;
                S[nb][2 + c] = (live1 && key <= qpos1) ? S[nb][2 + c] * ki * qs1 : -INFINITY;
                mx0 = fmaxf(mx0, S[nb][c]);
                mx1 = fmaxf(mx1, S[nb][2 + c]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m_0, mx0), mn1 = fmaxf(m_1, mx1);
        // rows with nothing unmasked yet keep m = -inf: scale 1, p = 0
        const float corr0 = mn0 == -INFINITY ? 1.f : expf(m_0 - mn0);
        const float corr1 = mn1 == -INFINITY ? 1.f : expf(m_1 - mn1);
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                S[nb][c] = mn0 == -INFINITY ? 0.f : expf(S[nb][c] - mn0);
                S[nb][2 + c] = mn1 == -INFINITY ? 0.f : expf(S[nb][2 + c] - mn1);
                ps0 += S[nb][c];
                ps1 += S[nb][2 + c];
            }
        }
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
        l_0 = l_0 * corr0 + ps0;
        l_1 = l_1 * corr1 + ps1;
        m_0 = mn0;
        m_1 = mn1;
#pragma unroll
        for (int nd = 0; nd < ND; ++nd) {
            O[nd][0] *= corr0;
            O[nd][1] *= corr0;
            O[nd][2] *= corr1;
            O[nd][3] *= corr1;
        }
        // O += P V, 16 keys per k-step (n-blocks 2kk and 2kk + 1 of S)
#pragma unroll
        for (int kk = 0; kk < NB / 2; ++kk) {
            const float va0 = vmul[kk * 16 + 2 * t], va1 = vmul[kk * 16 + 2 * t + 1];
            const float vb0 = vmul[kk * 16 + 8 + 2 * t], vb1 = vmul[kk * 16 + 8 + 2 * t + 1];
            uint32_t ph[4], pl[4];
            ph[0] = split2(S[2 * kk][0] * va0, S[2 * kk][1] * va1, pl[0]);
            ph[1] = split2(S[2 * kk][2] * va0, S[2 * kk][3] * va1, pl[1]);
            ph[2] = split2(S[2 * kk + 1][0] * vb0, S[2 * kk + 1][1] * vb1, pl[2]);
            ph[3] = split2(S[2 * kk + 1][2] * vb0, S[2 * kk + 1][3] * vb1, pl[3]);
            // ldmatrix.trans rows: keys kk*16 + (lane / 8 % 2) * 8 + lane % 8, dims 8 (nd + lane / 16)
            const int vrow = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
            for (int nd = 0; nd < ND; nd += 2) {
                const int vcol = 8 * (nd + (lane >> 4));
                uint32_t bh[4], bl[4];
                ldsm_x4_t(bh, Vh + vrow * ST + vcol);
                ldsm_x4_t(bl, Vl + vrow * ST + vcol);
                mma16816(O[nd], ph, bh[0], bh[1]);
                mma16816(O[nd], ph, bl[0], bl[1]);
                mma16816(O[nd], pl, bh[0], bh[1]);
                mma16816(O[nd + 1], ph, bh[2], bh[3]);
                mma16816(O[nd + 1], ph, bl[2], bl[3]);
                mma16816(O[nd + 1], pl, bh[2], bh[3]);
            }
        }
    }
    const float inv0 = 1.f / l_0, inv1 = 1.f / l_1;
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
        const int d = nd * 8 + 2 * t;
        if (live0)
            *reinterpret_cast<float2*>(out + (m0 + r0) * ldo + h * HD + d) =
                make_float2(O[nd][0] * inv0, O[nd][1] * inv0);
        if (live1)
            *reinterpret_cast<float2*>(out + (m0 + r1) * ldo + h * HD + d) =
                make_float2(O[nd][2] * inv1, O[nd][3] * inv1);
    }
}


// The K and V rows of every sequence's context as fp16 pairs, once per layer:
// row record [k h | k l | v h | v l] (HD halves each) per (sequence, KV head,
// position), scales [(kinv, vmul)] per row -- what attention_prefill_mma's
// staging computes for every query tile, computed once for all of them.
// One warp per 4 rows (8 lanes a row).
template <int HD>
__global__ void __launch_bounds__(256) kv_pairs_kernel(const float* __restrict__ kcache,
                                                       const float* __restrict__ vcache, __half* __restrict__ pairs,
                                                       float* __restrict__ scales, int n_ctx, int num_kv_heads,
                                                       int max_seq, long long total) {
    using namespace amma;
    const int lane = threadIdx.x & 31, sub = lane & 7;
    const long long row = (static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * 4 + (lane >> 3);
    const bool live = row < total;
    const long long r = live ? row : 0;
    const int t = static_cast<int>(r % n_ctx);
    const long long sh = r / n_ctx;  // sequence * num_kv_heads + kv head
    const int kvh = static_cast<int>(sh % num_kv_heads);
    const long long seq = sh / num_kv_heads;
    const size_t off = (static_cast<size_t>(seq) * max_seq + t) * (static_cast<size_t>(num_kv_heads) * HD) +
                       static_cast<size_t>(kvh) * HD;
    __half* rec = pairs + static_cast<size_t>(r) * 4 * HD;
    stage_row<HD, true>(kcache + off, live ? rec : nullptr, rec + HD, scales + 2 * r, sub);
    stage_row<HD, false>(vcache + off, live ? rec + 2 * HD : nullptr, rec + 3 * HD, scales + 2 * r + 1, sub);
}

// attention_prefill_mma's arithmetic on the pairs of kv_pairs_kernel: 32-key
// tiles, copied asynchronously into two shared-memory stages (the next tile
// lands while this one is computed), no conversion in the loop.
template <int HD>
__global__ void __launch_bounds__(128, 2) attention_prefill_pairs(
    float* __restrict__ out, const float* __restrict__ q, const __half* __restrict__ pairs,
    const float* __restrict__ scales, int pos0, int seq_len, int num_heads, int num_kv_heads, int n_ctx, int ldq,
    int ldo) {
    using namespace amma;
    constexpr int BM = 64, BN = 32, ST = HD + 8;  // row stride in halves
    constexpr int NB = BN / 8, ND = HD / 8, KS = HD / 16, CH = HD / 8;  // CH: 16-byte chunks of a row part
    constexpr int STAGE = 4 * BN * ST;                                   // halves of one stage (k h, k l, v h, v l)
    extern __shared__ __align__(16) uint8_t apsm[];
    __half* Qh = reinterpret_cast<__half*>(apsm);
    __half* Ql = Qh + BM * ST;
    __half* KV = Ql + BM * ST;                                      // [stage][part][BN][ST]
    float* qinv = reinterpret_cast<float*>(KV + 2 * STAGE);          // [BM]
    float* scl = qinv + BM;                                          // [stage][BN][2]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int sub = lane & 7, rsub = lane >> 3;
    const int qt = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int p0 = qt * BM;
    const int nrow = min(BM, seq_len - p0);
    const int kvh = h / (num_heads / num_kv_heads);
    const size_t m0 = static_cast<size_t>(seq) * seq_len + p0;
    const long long base = (static_cast<long long>(seq) * num_kv_heads + kvh) * n_ctx;  // first pair row
    const int last = pos0 + p0 + nrow - 1;  // last key position any row of the tile sees
    const int ntile = last / BN + 1;
    auto load = [&](int tile, int stage) {
        const int t0 = tile * BN;
        __half* dst = KV + stage * STAGE;
        for (int c = threadIdx.x; c < BN * 4 * CH; c += 128) {
            const int r = c / (4 * CH), part = (c / CH) % 4, o = c % CH;
            const bool in = t0 + r < n_ctx;
            const __half* src = pairs + (static_cast<size_t>(base + (in ? t0 + r : 0)) * 4 + part) * HD + o * 8;
            cp16(dst + (part * BN + r) * ST + o * 8, src, in ? 16 : 0);
        }
        if (threadIdx.x < BN) {
            const int r = threadIdx.x;
            const bool in = t0 + r < n_ctx;
            cp8(scl + stage * 2 * BN + 2 * r, scales + 2 * (base + (in ? t0 + r : 0)), in ? 8 : 0);
        }
        cp_commit();
    };
    load(0, 0);
    for (int r = 4 * warp + rsub; r < BM; r += 16)
        stage_row<HD, true>(r < nrow ? q + (m0 + r) * ldq + h * HD : nullptr, Qh + r * ST, Ql + r * ST, qinv + r,
                            sub);
    const float rsqrt_hd = 1.0f / sqrtf(static_cast<float>(HD));
    const int r0 = 16 * warp + g, r1 = r0 + 8;
    const int qpos0 = pos0 + p0 + r0, qpos1 = pos0 + p0 + r1;
    const bool live0 = r0 < nrow, live1 = r1 < nrow;
    float O[ND][4];
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) O[nd][0] = O[nd][1] = O[nd][2] = O[nd][3] = 0.f;
    float m_0 = -INFINITY, m_1 = -INFINITY, l_0 = 0.f, l_1 = 0.f;
    for (int tile = 0; tile < ntile; ++tile) {
        const int stage = tile & 1, t0 = tile * BN;
        if (tile + 1 < ntile) {
            load(tile + 1, stage ^ 1);
            cp_wait<1>();  // this tile's group has landed
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const __half* Kh = KV + stage * STAGE;
        const __half* Kl = Kh + BN * ST;
        const __half* Vh = Kl + BN * ST;
        const __half* Vl = Vh + BN * ST;
        const float* sc = scl + stage * 2 * BN;
        float S[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) S[nb][0] = S[nb][1] = S[nb][2] = S[nb][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int c = ks * 16 + 2 * t;
            uint32_t ah[4], al[4];
            ah[0] = lds32(Qh + r0 * ST + c);
            ah[1] = lds32(Qh + r1 * ST + c);
            ah[2] = lds32(Qh + r0 * ST + c + 8);
            ah[3] = lds32(Qh + r1 * ST + c + 8);
            al[0] = lds32(Ql + r0 * ST + c);
            al[1] = lds32(Ql + r1 * ST + c);
            al[2] = lds32(Ql + r0 * ST + c + 8);
            al[3] = lds32(Ql + r1 * ST + c + 8);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                const __half* kh = Kh + (nb * 8 + g) * ST + c;
                const __half* kl = Kl + (nb * 8 + g) * ST + c;
                const uint32_t bh0 = lds32(kh), bh1 = lds32(kh + 8), bl0 = lds32(kl), bl1 = lds32(kl + 8);
                mma16816(S[nb], ah, bh0, bh1);
                mma16816(S[nb], ah, bl0, bl1);
                mma16816(S[nb], al, bh0, bh1);
            }
        }
        const float qs0 = qinv[r0] * rsqrt_hd, qs1 = qinv[r1] * rsqrt_hd;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int j = nb * 8 + 2 * t + c, key = t0 + j;
                const float ki = sc[2 * j];
                S[nb][c] = (live0 && key <= qpos0) ? S[nb][c] * ki * qs0 : -INFINITY;
                S[nb][2 + c] = (live1 && key <= qpos1) ? S[nb][2 + c] * ki * qs1 : -INFINITY;
                mx0 = fmaxf(mx0, S[nb][c]);
                mx1 = fmaxf(mx1, S[nb][2 + c]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m_0, mx0), mn1 = fmaxf(m_1, mx1);
        const float corr0 = mn0 == -INFINITY ? 1.f : expf(m_0 - mn0);
        const float corr1 = mn1 == -INFINITY ? 1.f : expf(m_1 - mn1);
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                S[nb][c] = mn0 == -INFINITY ? 0.f : expf(S[nb][c] - mn0);
                S[nb][2 + c] = mn1 == -INFINITY ? 0.f : expf(S[nb][2 + c] - mn1);
                ps0 += S[nb][c];
                ps1 += S[nb][2 + c];
            }
        }
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
        l_0 = l_0 * corr0 + ps0;
        l_1 = l_1 * corr1 + ps1;
        m_0 = mn0;
        m_1 = mn1;
#pragma unroll
        for (int nd = 0; nd < ND; ++nd) {
            O[nd][0] *= corr0;
            O[nd][1] *= corr0;
            O[nd][2] *= corr1;
            O[nd][3] *= corr1;
        }
#pragma unroll
        for (int kk = 0; kk < NB / 2; ++kk) {
            const float va0 = sc[2 * (kk * 16 + 2 * t) + 1], va1 = sc[2 * (kk * 16 + 2 * t + 1) + 1];
            const float vb0 = sc[2 * (kk * 16 + 8 + 2 * t) + 1], vb1 = sc[2 * (kk * 16 + 8 + 2 * t + 1) + 1];
            uint32_t ph[4], pl[4];
            ph[0] = split2(S[2 * kk][0] * va0, S[2 * kk][1] * va1, pl[0]);
            ph[1] = split2(S[2 * kk][2] * va0, S[2 * kk][3] * va1, pl[1]);
            ph[2] = split2(S[2 * kk + 1][0] * vb0, S[2 * kk + 1][1] * vb1, pl[2]);
            ph[3] = split2(S[2 * kk + 1][2] * vb0, S[2 * kk + 1][3] * vb1, pl[3]);
            const int vrow = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
            for (int nd = 0; nd < ND; nd += 2) {
                const int vcol = 8 * (nd + (lane >> 4));
                uint32_t bh[4], bl[4];
                ldsm_x4_t(bh, Vh + vrow * ST + vcol);
                ldsm_x4_t(bl, Vl + vrow * ST + vcol);
                mma16816(O[nd], ph, bh[0], bh[1]);
                mma16816(O[nd], ph, bl[0], bl[1]);
                mma16816(O[nd], pl, bh[0], bh[1]);
                mma16816(O[nd + 1], ph, bh[2], bh[3]);
                mma16816(O[nd + 1], ph, bl[2], bl[3]);
                mma16816(O[nd + 1], pl, bh[2], bh[3]);
            }
        }
        __syncthreads();  // this stage is read out: the load after next may overwrite it
    }
    const float inv0 = 1.f / l_0, inv1 = 1.f / l_1;
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
        const int d = nd * 8 + 2 * t;
        if (live0)
            *reinterpret_cast<float2*>(out + (m0 + r0) * ldo + h * HD + d) =
                make_float2(O[nd][0] * inv0, O[nd][1] * inv0);
        if (live1)
            *reinterpret_cast<float2*>(out + (m0 + r1) * ldo + h * HD + d) =
                make_float2(O[nd][2] * inv1, O[nd][3] * inv1);
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
                                     int max_seq, int ldq, int ldo, cudaStream_t s, int form) {
    const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const bool mma_ok = (head_dim == 64 || head_dim == 128) && seq_len > 0 && rows % seq_len == 0 &&
                        (ldq % 4) == 0 && (ldo % 2) == 0 && a16(q) && a16(kcache) && a16(vcache) &&
                        (reinterpret_cast<uintptr_t>(out) & 7u) == 0 && (num_kv_heads * head_dim) % 4 == 0;
    if (form >= 3 && mma_ok) {
        // K/V as fp16 pairs once for the layer (stream-ordered scratch), then
        // the double-buffered tensor-core attention over them
        const int nseq = rows / seq_len;
        const int n_ctx = pos0 + seq_len;
        const dim3 grid((seq_len + 63) / 64, num_heads, nseq);
        if (nseq > 65535 || num_heads > 65535) return cudaErrorInvalidConfiguration;
        const long long total = static_cast<long long>(nseq) * num_kv_heads * n_ctx;
        const size_t pair_bytes = (static_cast<size_t>(total) * 4 * head_dim * sizeof(__half) + 255) / 256 * 256;
        const size_t bytes = pair_bytes + static_cast<size_t>(total) * 2 * sizeof(float);
        const long long blocks = (total + 31) / 32;
        if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
        void* buf = nullptr;
        cudaError_t e = scratch_alloc(&buf, bytes, s);
        if (e != cudaSuccess) return e;
        __half* pairs = static_cast<__half*>(buf);
        float* scales = reinterpret_cast<float*>(static_cast<uint8_t*>(buf) + pair_bytes);
        const int ST = head_dim + 8;
        const size_t smem = (2 * 64 * ST + 2 * 4 * 32 * ST) * sizeof(__half) + (64 + 2 * 2 * 32) * sizeof(float);
        if (head_dim == 128) {
            kv_pairs_kernel<128><<<static_cast<unsigned>(blocks), 256, 0, s>>>(kcache, vcache, pairs, scales, n_ctx,
                                                                                num_kv_heads, max_seq, total);
            e = cudaFuncSetAttribute(attention_prefill_pairs<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e == cudaSuccess)
                attention_prefill_pairs<128><<<grid, 128, smem, s>>>(out, q, pairs, scales, pos0, seq_len, num_heads,
                                                                      num_kv_heads, n_ctx, ldq, ldo);
        } else {
            kv_pairs_kernel<64><<<static_cast<unsigned>(blocks), 256, 0, s>>>(kcache, vcache, pairs, scales, n_ctx,
                                                                               num_kv_heads, max_seq, total);
            e = cudaFuncSetAttribute(attention_prefill_pairs<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e == cudaSuccess)
                attention_prefill_pairs<64><<<grid, 128, smem, s>>>(out, q, pairs, scales, pos0, seq_len, num_heads,
                                                                     num_kv_heads, n_ctx, ldq, ldo);
        }
        if (e == cudaSuccess) e = cudaGetLastError();
        const cudaError_t e2 = scratch_free(buf, s);
        return e != cudaSuccess ? e : e2;
    }
    if (form >= 2 && mma_ok) {
        const int nseq = rows / seq_len;
        const dim3 grid((seq_len + 63) / 64, num_heads, nseq);
        if (nseq > 65535 || num_heads > 65535) return cudaErrorInvalidConfiguration;
        const size_t smem = 6 * 64 * (head_dim + 8) * sizeof(__half) + 3 * 64 * sizeof(float);
        cudaError_t e;
        if (head_dim == 128) {
            e = cudaFuncSetAttribute(attention_prefill_mma<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            attention_prefill_mma<128><<<grid, 128, smem, s>>>(out, q, kcache, vcache, pos0, seq_len, num_heads,
                                                                num_kv_heads, max_seq, ldq, ldo);
        } else {
            e = cudaFuncSetAttribute(attention_prefill_mma<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            attention_prefill_mma<64><<<grid, 128, smem, s>>>(out, q, kcache, vcache, pos0, seq_len, num_heads,
                                                               num_kv_heads, max_seq, ldq, ldo);
        }
        return cudaGetLastError();
    }
    if (form >= 1 && (head_dim == 64 || head_dim == 128) && seq_len > 0 && rows % seq_len == 0 && (ldq % 4) == 0 &&
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
