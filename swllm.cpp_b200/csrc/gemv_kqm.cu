// gemv_kqm.cu -- K-quant GEMVs of 2..32 activation rows (batched decode):
// Y[M x N] = X[M x K] . W[N x K]^T for Q4_K and Q6_K, every weight read once
// for all M rows, products exact on the tensor cores (sm_100a).
//
// Replaces M calls of cpu_matmul_transposed_q4_k / _q6_k
// (src/tensor.h:769-856) behind Compute::matmul_transposed_q
// (src/tensor.h:1212) -- the rows of a batched decode step.  The reference
// evaluates, per row, in fp32
//     Q4_K: y = sum_b sum_j sum_{k in j} (d_b sc_j q_k - dmin_b m_j) x_k
//     Q6_K: y = sum_b sum_j sum_{k in j} d_b sc_j (q_k - 32) x_k
// Here, per super-block b of 256 weights and activation row:
//     x_k 2^(14 - E_b) = h_k + l_k, two fp16 numbers (E_b: the row's largest
//     binary exponent in the super-block; h_k = fp16 of the scaled value,
//     l_k = fp16 of the rest, 22 bits in all)
// and on m16n8k16 f16 MMAs with fp32 accumulation
//     Q4_K: C = sum_k (sc_j q_k) (h_k + l_k)   (sc_j q_k <= 945: exact in fp16)
//           C' = sum_j m_j X'_j                (X'_j: the sub-block sums of the
//                                               scaled x, split the same way)
//           y += 2^(E_b - 14) (d_b C - 32 dmin_b C')
//     Q6_K: C_j = sum_{k in j} (q_k - 32) (h_k + l_k), y += 2^(E_b - 14) d_b
//           sum_j sc_j C_j (the scale applied in fp32: (q - 32) sc can
//           exceed fp16's exact integers)
// Every product is exact; the MMA sums 16 products at a time in fp32.  Error
// sources: the 22-bit split of x relative to the super-block's largest
// element (fewer bits for blocks below 2^-117, see prep_kernel), the MMA's
// and the epilogue's fp32 sums -- the reference rounds every product and
// addition instead.
//
// Two launches:
//   prep_kernel   X -> the B-fragment table: per super-block and k-step of 16
//                 elements, per block of 8 activation rows, h and l as fp16
//                 in fragment order; the sub-block sums for the Q4_K mins; per
//                 row the super-block scale 2^(E_b - 14); (RMSNORM) the
//                 per-super-block sums of squares.  One warp per (row,
//                 super-block); the activation prologues of the other GEMV
//                 forms run here.
//   gemv_kqm_kernel  persistent CTAs over (row range, K split): a producer warp
//                 streams 16-row weight boxes through a shared-memory ring
//                 (TMA, no multicast); consumer warps in groups of GW, a group
//                 per 16-row tile, each warp a share of the tile's
//                 super-blocks; a group sums its warps' rows in warp order.
//                 K is split so that a split's table fits shared memory: a
//                 CTA either runs every split of its rows in turn (adding into
//                 Y in split order) or one split, with the splits of a row
//                 range summed in split order by the CTA that finishes last.
// Every wait is bounded.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "gemv.h"
#include "gemv_kqm.h"
#include "swq_device.cuh"

namespace swq {
namespace kqm {

constexpr int TR = 16;  // weight rows per tile (the MMA's M)
constexpr int MAX_STAGES = 16;
// Table record of one super-block per block of 8 activation rows: B
// fragments of x (16 k-steps x h, l x 32 lanes x 8 bytes), B fragments of the
// sub-block sums for the Q4_K mins (h, l x 32 lanes x 4 bytes), per row the
// scale 2^(E_b - 14).
constexpr int FRAG_UNIT = 16 * 2 * 256;
constexpr int MINF_UNIT = 2 * 128;
constexpr int XS_UNIT = 8 * 4;
constexpr int REC_UNIT = FRAG_UNIT + MINF_UNIT + XS_UNIT;

template <int T>
struct Fmt;
template <>
struct Fmt<Q4_K> {
    static constexpr int BB = 144;
};
template <>
struct Fmt<Q6_K> {
    static constexpr int BB = 210;
};

struct PrepParams {
    const float* X;
    int ld;  // row stride of X in elements
    uint8_t* tab;
    float* rsq;  // [8 NCB][nb] sums of squares (RMSNORM), or null
    unsigned* cnt;
    int ncnt;  // split counters of the GEMV, zeroed here
    int M, K, nb;
    int act;
    const float* R;  // RMSNORM residual, row stride K
    const float* normw;
    float* sum_out;  // RMSNORM: x = X + R written here (row stride K)
    int vec;         // all of X, R, normw, sum_out 16-byte aligned with 4-multiple strides
};

struct Params {
    const uint8_t* W;
    float* Y;
    const uint8_t* tab;
    const float* rsq;
    float* part;    // [S][8 NCB][N] split partials (SC > 1)
    unsigned* cnt;  // [G] split arrivals (SC > 1)
    int N, K, nb, M, ldy;
    int G, S, SC, kbs;  // row groups, K splits, CTAs per row group (1 or S), super-blocks per split
    int KC, cs, stage_bytes, stages;
    uint32_t stage_magic;  // ceil(2^32 / stages)
    int GW;                // consumer warps per tile group
    int early;
    int rms;
    float eps;
    uint32_t off_rs, off_tab, off_part, off_ring;
};

// D = A . B (+ C): m16n8k16, fp16 operands, fp32 accumulation
__device__ __forceinline__ void mma_acc(float (&d)[4], const uint32_t (&a)[4], uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}
__device__ __forceinline__ void mma_zero(float (&d)[4], const uint32_t (&a)[4], uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "f"(0.0f));
}

__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
    const __half2 r = __hadd2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
    const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b),
                              *reinterpret_cast<const __half2*>(&c));
    return *reinterpret_cast<const uint32_t*>(&r);
}

// fp16 bit patterns: 1024 + n is 0x6400 | n for 0 <= n < 1024
constexpr uint32_t H2_1024 = 0x64006400u;
constexpr uint32_t H2_M1024 = 0xE400E400u;      // -1024
constexpr uint32_t H2_M1056 = 0xE420E420u;      // -1056
constexpr uint32_t H2_SIXTEENTH = 0x2C002C00u;  // 1/16
constexpr uint32_t H2_M64 = 0xD400D400u;        // -64

// Quant values of bytes 0..3 of a weight word as the A operand's fp16 pairs
// (byte 0, byte 2) and (byte 1, byte 3) -- the k order of the table's B
// fragments.  Q4_K low nibbles times the sub-block scale: (1024 + q) sc -
// 1024 sc (kS = (sc, sc), kB = -1024 (sc, sc)); high nibbles:
// (1024 + 16 q) sc / 16 - 64 sc.  One rounding of an exact result below
// 1024: exact.
__device__ __forceinline__ void nib_lo(uint32_t w, uint32_t kS, uint32_t kB, uint32_t& p02, uint32_t& p13) {
    p02 = hfma2_u((w & 0x000F000Fu) | H2_1024, kS, kB);
    p13 = hfma2_u(((w >> 8) & 0x000F000Fu) | H2_1024, kS, kB);
}
__device__ __forceinline__ void nib_hi(uint32_t w, uint32_t kS16, uint32_t kB64, uint32_t& p02, uint32_t& p13) {
    p02 = hfma2_u((w & 0x00F000F0u) | H2_1024, kS16, kB64);
    p13 = hfma2_u(((w >> 8) & 0x00F000F0u) | H2_1024, kS16, kB64);
}

// (n, n) in fp16 for a small integer n (0 <= n < 1024)
__device__ __forceinline__ uint32_t h2_int(uint32_t n) { return hadd2_u((n | (n << 16)) | H2_1024, H2_M1024); }

// Four 6-bit values (bytes 0..3 of w), minus 32, as fp16 pairs (byte 0,
// byte 2) and (byte 1, byte 3), exact.
__device__ __forceinline__ void six_pairs(uint32_t w, uint32_t& p02, uint32_t& p13) {
    p02 = hadd2_u((w & 0x003F003Fu) | H2_1024, H2_M1056);
    p13 = hadd2_u(((w >> 8) & 0x003F003Fu) | H2_1024, H2_M1056);
}

__device__ __forceinline__ void tma_box(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                        uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t cnt) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(cnt) : "memory");
}

// 16-byte global -> shared copy, asynchronous (completed by cp_async_wait)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// First row of tile `tile` of [r_begin, r_end): a last tile that would run past
// r_end starts lower (rows the previous tile also read) when the range holds a
// whole tile, so no tile reads another CTA's rows.
__device__ __forceinline__ int tile_row0(int tile, int r_begin, int r_end) {
    const int r0 = r_begin + tile * TR;
    return (r0 + TR > r_end && r_end - TR >= r_begin) ? r_end - TR : r0;
}

__device__ __forceinline__ void ld8(const float* p, float (&v)[8], bool vec) {
    if (vec) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        const float4 c = __ldg(reinterpret_cast<const float4*>(p + 4));
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __ldg(p + i);
    }
}

__device__ __forceinline__ void st8(float* p, const float (&v)[8], bool vec) {
    if (vec) {
        reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = v[i];
    }
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Record of super-block b (REC_UNIT * NCB bytes):
//   frag [k-step s][row block cb][h, l][lane 32] x 8 bytes: lane (g, t) holds
//        elements e = 16 s + 4t + (0..3) of activation row 8 cb + g as the
//        MMA's B pairs (e0, e2) in b0 (k = 2t, 2t + 1) and (e1, e3) in b1
//        (k = 2t + 8, 2t + 9) -- the order of the A operands built from
//        weight words (bytes 0, 2 and 1, 3)
//   minf [row block cb][h, l][lane 32] x 4 bytes: lane (g, t) holds the sums
//        of the scaled x over sub-blocks 2t and 2t + 1 of 32 elements, times
//        2^-5 (the B operand of the Q4_K mins: k = 2t, 2t + 1; k >= 8 is zero)
//   xs   [8 NCB] fp32: 2^(E_b - 14), NaN for a super-block with a non-finite
//        value
// One warp per (row m, super-block b); lane l takes elements 8l .. 8l + 7.
template <int NCB>
__global__ void __launch_bounds__(256) prep_kernel(const PrepParams p) {
    pdl_launch_dependents();
    pdl_wait_primary();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int i = threadIdx.x; i < p.ncnt; i += blockDim.x) p.cnt[i] = 0u;
    const int b = blockIdx.x;
    const int m = blockIdx.y * 8 + warp;
    if (m >= 8 * NCB) return;
    const bool vec = p.vec != 0;
    uint8_t* rec = p.tab + static_cast<size_t>(b) * (REC_UNIT * NCB);
    const int e0 = 256 * b + 8 * lane;
    float v[8];
    float sq = 0.f;
    if (m < p.M) {
        const float* xr = p.X + static_cast<size_t>(m) * p.ld;
        if (p.act == ACT_SWIGLU) {
            float gt[8], up[8];
            ld8(xr + e0, gt, vec);
            ld8(xr + p.K + e0, up, vec);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = gt[i] / (1.0f + expf(-gt[i])) * up[i];
        } else {
            ld8(xr + e0, v, vec);
            if (p.act == ACT_RMSNORM) {
                if (p.R) {
                    float r[8];
                    ld8(p.R + static_cast<size_t>(m) * p.K + e0, r, vec);
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] += r[i];
                }
                if (p.sum_out) st8(p.sum_out + static_cast<size_t>(m) * p.K + e0, v, vec);
                float w[8];
                ld8(p.normw + e0, w, vec);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    sq = fmaf(v[i], v[i], sq);
                    v[i] *= w[i];
                }
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float mx = 0.f;
    bool nonfinite = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        mx = fmaxf(mx, fabsf(v[i]));
        nonfinite |= !(fabsf(v[i]) <= 3.402823466e38f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
    }
    nonfinite = __any_sync(0xffffffffu, nonfinite);
    // E: mx < 2^E; the scaled values stay below 2^14 (fp16 max 65504), the
    // scaled sums of 32 times 2^-5 too.  E >= -100 keeps the scale factors
    // normal floats: a super-block whose largest element is below 2^-117
    // keeps fewer than 22 bits (its low part turns fp16-subnormal).  Beside
    // blocks of normal magnitude that is far under fp32's resolution of the
    // row's sums; a row made only of such blocks loses relative accuracy
    // (about 1e-4 at fp32's smallest normals, 1e-2 for subnormal rows).
    const int E = max(((__float_as_int(mx) >> 23) & 0xFF) - 126, -100);
    const float up_s = nonfinite ? 0.f : __int_as_float((127 + 14 - E) << 23);
    float u[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) u[i] = v[i] * up_s;
    // h and l of elements (0, 2), (1, 3), (4, 6), (5, 7)
    uint32_t H[4], L[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int i0 = (q >> 1) * 4 + (q & 1);
        const __half2 h = __floats2half2_rn(u[i0], u[i0 + 2]);
        const float2 hf = __half22float2(h);
        H[q] = *reinterpret_cast<const uint32_t*>(&h);
        L[q] = pack_h2(u[i0] - hf.x, u[i0 + 2] - hf.y);
    }
    const int cb = m >> 3, g = m & 7, s = lane >> 1, t0 = 2 * (lane & 1);
    uint8_t* fh = rec + ((s * NCB + cb) * 2) * 256;
    *reinterpret_cast<uint2*>(fh + (4 * g + t0) * 8) = make_uint2(H[0], H[1]);
    *reinterpret_cast<uint2*>(fh + (4 * g + t0 + 1) * 8) = make_uint2(H[2], H[3]);
    *reinterpret_cast<uint2*>(fh + 256 + (4 * g + t0) * 8) = make_uint2(L[0], L[1]);
    *reinterpret_cast<uint2*>(fh + 256 + (4 * g + t0 + 1) * 8) = make_uint2(L[2], L[3]);
    // sums of 32 (sub-block j on lanes 4j .. 4j + 3), scaled by 2^-5 more
    float s8 = ((u[0] + u[1]) + (u[2] + u[3])) + ((u[4] + u[5]) + (u[6] + u[7]));
    s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
    s8 += __shfl_xor_sync(0xffffffffu, s8, 2);
    const float xa = __shfl_sync(0xffffffffu, s8, 8 * (lane & 3)) * 0.03125f;
    const float xb = __shfl_sync(0xffffffffu, s8, 8 * (lane & 3) + 4) * 0.03125f;
    if (lane < 4) {
        const __half2 h = __floats2half2_rn(xa, xb);
        const float2 hf = __half22float2(h);
        uint8_t* mf = rec + FRAG_UNIT * NCB + cb * 256 + (4 * g + lane) * 4;
        *reinterpret_cast<uint32_t*>(mf) = *reinterpret_cast<const uint32_t*>(&h);
        *reinterpret_cast<uint32_t*>(mf + 128) = pack_h2(xa - hf.x, xb - hf.y);
    }
    if (lane == 0) {
        float* xs = reinterpret_cast<float*>(rec + (FRAG_UNIT + MINF_UNIT) * NCB);
        xs[m] = nonfinite ? __int_as_float(0x7fc00000) : __int_as_float((127 + E - 14) << 23);
        if (p.rsq) p.rsq[static_cast<size_t>(m) * p.nb + b] = sq;
    }
}

// B fragment of k-step s, row block cb (h at +0, l at +256)
template <int NCB>
__device__ __forceinline__ const uint8_t* frag(const uint8_t* rec, int s, int cb, int lane) {
    return rec + ((s * NCB + cb) * 2) * 256 + lane * 8;
}

// One Q4_K item: super-block rows g (bA) and g + 8 (bB) of a tile, table
// record rec.  The sub-block scales are folded into the A operands (q sc is
// exact in fp16), so one chain of MMAs per row block and h / l sums the whole
// super-block; the mins are one more MMA pair (A: the 8 mins, B: the sums of
// 32).  acc[cb][i]: row g (i < 2) or g + 8, activation row 8 cb + 2t + (i & 1).
template <int NCB>
__device__ __forceinline__ void item_q4k(const uint8_t* bA, const uint8_t* bB, const uint8_t* rec, int lane,
                                         float (&acc)[NCB][4]) {
    const int t = lane & 3;
    const uint4 hA = lds_u128(bA), hB = lds_u128(bB);
    // 6-bit scales (get_scale_min_k4, src/tensor.h:218-227): sub-blocks 0..3
    // in bytes 0..3, 4..7 from bytes 8..11 with the high bits of 0..3
    const uint32_t sloA = hA.y & 0x3F3F3F3Fu, shiA = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
    const uint32_t sloB = hB.y & 0x3F3F3F3Fu, shiB = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
    float Ch[NCB][4], Cl[NCB][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t wA0 = *reinterpret_cast<const uint32_t*>(bA + 16 + 32 * c + 4 * t);
        const uint32_t wA1 = *reinterpret_cast<const uint32_t*>(bA + 16 + 32 * c + 16 + 4 * t);
        const uint32_t wB0 = *reinterpret_cast<const uint32_t*>(bB + 16 + 32 * c + 4 * t);
        const uint32_t wB1 = *reinterpret_cast<const uint32_t*>(bB + 16 + 32 * c + 16 + 4 * t);
        const uint32_t wsA = (c < 2 ? sloA : shiA) >> (16 * (c & 1)), wsB = (c < 2 ? sloB : shiB) >> (16 * (c & 1));
        // (sc, sc) of the unit's two sub-blocks, rows A and B
        const uint32_t kAl = h2_int(wsA & 0xFFu), kAh = h2_int((wsA >> 8) & 0xFFu);
        const uint32_t kBl = h2_int(wsB & 0xFFu), kBh = h2_int((wsB >> 8) & 0xFFu);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t kA = half ? kAh : kAl, kB = half ? kBh : kBl;
            const uint32_t kA1 = half ? hmul2_u(kA, H2_SIXTEENTH) : kA, kB1 = half ? hmul2_u(kB, H2_SIXTEENTH) : kB;
            const uint32_t kA0 = hmul2_u(kA, half ? H2_M64 : H2_M1024), kB0 = hmul2_u(kB, half ? H2_M64 : H2_M1024);
#pragma unroll
            for (int gr = 0; gr < 2; ++gr) {
                uint32_t a[4];
                const uint32_t wa = gr ? wA1 : wA0, wb = gr ? wB1 : wB0;
                if (half) {
                    nib_hi(wa, kA1, kA0, a[0], a[2]);
                    nib_hi(wb, kB1, kB0, a[1], a[3]);
                } else {
                    nib_lo(wa, kA1, kA0, a[0], a[2]);
                    nib_lo(wb, kB1, kB0, a[1], a[3]);
                }
                const int s = 4 * c + 2 * half + gr;
#pragma unroll
                for (int cb = 0; cb < NCB; ++cb) {
                    const uint8_t* f = frag<NCB>(rec, s, cb, lane);
                    const uint2 bh = *reinterpret_cast<const uint2*>(f);
                    const uint2 bl = *reinterpret_cast<const uint2*>(f + 256);
                    if (s == 0) {
                        mma_zero(Ch[cb], a, bh);
                        mma_zero(Cl[cb], a, bl);
                    } else {
                        mma_acc(Ch[cb], a, bh);
                        mma_acc(Cl[cb], a, bl);
                    }
                }
            }
        }
    }
    // mins m_j of sub-blocks 2t, 2t + 1 (bytes 4..7, or the high nibbles of
    // 8..11 with the high bits of 4..7) as the A pair of k = 2t, 2t + 1
    const uint32_t mwA = t < 2 ? hA.z : (((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u));
    const uint32_t mwB = t < 2 ? hB.z : (((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u));
    const uint32_t mA = (mwA >> (16 * (t & 1))) & 0x3F3Fu, mB = (mwB >> (16 * (t & 1))) & 0x3F3Fu;
    uint32_t am[4];
    am[0] = hadd2_u(((mA & 0xFFu) | ((mA & 0xFF00u) << 8)) | H2_1024, H2_M1024);
    am[1] = hadd2_u(((mB & 0xFFu) | ((mB & 0xFF00u) << 8)) | H2_1024, H2_M1024);
    am[2] = 0u;
    am[3] = 0u;
    const float2 dmA = __half22float2(*reinterpret_cast<const __half2*>(&hA.x));
    const float2 dmB = __half22float2(*reinterpret_cast<const __half2*>(&hB.x));
    const float* xs = reinterpret_cast<const float*>(rec + (FRAG_UNIT + MINF_UNIT) * NCB);
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) {
        const uint8_t* mf = rec + FRAG_UNIT * NCB + cb * 256 + lane * 4;
        float Cm[4];
        mma_zero(Cm, am, make_uint2(*reinterpret_cast<const uint32_t*>(mf), 0u));
        mma_acc(Cm, am, make_uint2(*reinterpret_cast<const uint32_t*>(mf + 128), 0u));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float e = xs[8 * cb + 2 * t + i];
            // d sum_j sc_j C_j - 32 dmin sum_j m_j X'_j (the sums carry 2^-5)
            acc[cb][i] = fmaf(e, fmaf(dmA.x, Ch[cb][i] + Cl[cb][i], -32.0f * dmA.y * Cm[i]), acc[cb][i]);
            acc[cb][2 + i] =
                fmaf(e, fmaf(dmB.x, Ch[cb][2 + i] + Cl[cb][2 + i], -32.0f * dmB.y * Cm[2 + i]), acc[cb][2 + i]);
        }
    }
}

// 32-bit word at a block offset that is a multiple of 4 for a block at a
// 2-byte aligned address (ODD: 2 mod 4), from two aligned words.
template <bool ODD>
__device__ __forceinline__ uint32_t ld32(const uint8_t* q) {
    if constexpr (!ODD) {
        return *reinterpret_cast<const uint32_t*>(q);
    } else {
        const uint32_t* a = reinterpret_cast<const uint32_t*>(q - 2);
        return __funnelshift_r(a[0], a[1], 16);
    }
}

__device__ __forceinline__ int sext8(uint32_t w, int byte) {
    return static_cast<int>(static_cast<int8_t>(static_cast<uint8_t>(w >> (8 * byte))));
}

// One Q6_K item (ql[128] @0, qh[64] @128, int8 scales[16] @192, fp16 d @208,
// src/tensor.h:398-432).  Unit c = (nn, h), plane p: the 16 elements
// 128 nn + 32 p + 16 h + .. of sub-block j = 8 nn + 2 p + h, which is also
// k-step j of the table; lane t holds elements 4t .. 4t + 3 of rows g, g + 8.
template <int NCB, bool ODD>
__device__ __forceinline__ void item_q6k(const uint8_t* bA, const uint8_t* bB, const uint8_t* rec, int lane,
                                         float (&acc)[NCB][4]) {
    const int t = lane & 3;
    float T[NCB][4];
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) T[cb][0] = T[cb][1] = T[cb][2] = T[cb][3] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int nn = c >> 1, h = c & 1;
        const int o = 64 * nn + 16 * h + 4 * t;
        const uint32_t L0A = ld32<ODD>(bA + o), L1A = ld32<ODD>(bA + o + 32);
        const uint32_t HA = ld32<ODD>(bA + 128 + 32 * nn + 16 * h + 4 * t);
        const uint32_t L0B = ld32<ODD>(bB + o), L1B = ld32<ODD>(bB + o + 32);
        const uint32_t HB = ld32<ODD>(bB + 128 + 32 * nn + 16 * h + 4 * t);
        const uint32_t SA0 = ld32<ODD>(bA + 192 + 8 * nn), SA1 = ld32<ODD>(bA + 192 + 8 * nn + 4);
        const uint32_t SB0 = ld32<ODD>(bB + 192 + 8 * nn), SB1 = ld32<ODD>(bB + 192 + 8 * nn + 4);
#pragma unroll
        for (int pl = 0; pl < 4; ++pl) {
            const uint32_t PA = pl == 0   ? (L0A & 0x0F0F0F0Fu) | ((HA << 4) & 0x30303030u)
                                : pl == 1 ? (L1A & 0x0F0F0F0Fu) | ((HA << 2) & 0x30303030u)
                                : pl == 2 ? ((L0A >> 4) & 0x0F0F0F0Fu) | (HA & 0x30303030u)
                                          : ((L1A >> 4) & 0x0F0F0F0Fu) | ((HA >> 2) & 0x30303030u);
            const uint32_t PB = pl == 0   ? (L0B & 0x0F0F0F0Fu) | ((HB << 4) & 0x30303030u)
                                : pl == 1 ? (L1B & 0x0F0F0F0Fu) | ((HB << 2) & 0x30303030u)
                                : pl == 2 ? ((L0B >> 4) & 0x0F0F0F0Fu) | (HB & 0x30303030u)
                                          : ((L1B >> 4) & 0x0F0F0F0Fu) | ((HB >> 2) & 0x30303030u);
            uint32_t a[4];
            six_pairs(PA, a[0], a[2]);
            six_pairs(PB, a[1], a[3]);
            const int jl = 2 * pl + h;  // sub-block within the half: byte jl of the half's 8 scales
            const float sA = static_cast<float>(sext8(jl < 4 ? SA0 : SA1, jl & 3));
            const float sB = static_cast<float>(sext8(jl < 4 ? SB0 : SB1, jl & 3));
            const int s = 8 * nn + jl;
#pragma unroll
            for (int cb = 0; cb < NCB; ++cb) {
                const uint8_t* f = frag<NCB>(rec, s, cb, lane);
                float C[4];
                mma_zero(C, a, *reinterpret_cast<const uint2*>(f));
                mma_acc(C, a, *reinterpret_cast<const uint2*>(f + 256));
                T[cb][0] = fmaf(sA, C[0], T[cb][0]);
                T[cb][1] = fmaf(sA, C[1], T[cb][1]);
                T[cb][2] = fmaf(sB, C[2], T[cb][2]);
                T[cb][3] = fmaf(sB, C[3], T[cb][3]);
            }
        }
    }
    const float dA = __half2float(*reinterpret_cast<const __half*>(bA + 208));
    const float dB = __half2float(*reinterpret_cast<const __half*>(bB + 208));
    const float* xs = reinterpret_cast<const float*>(rec + (FRAG_UNIT + MINF_UNIT) * NCB);
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float e = xs[8 * cb + 2 * t + i];
            acc[cb][i] = fmaf(dA * e, T[cb][i], acc[cb][i]);
            acc[cb][2 + i] = fmaf(dB * e, T[cb][2 + i], acc[cb][2 + i]);
        }
    }
}

// Splits of CTA column sc: s = sc, sc + SC, ... < S; split s covers
// super-blocks [s kbs, min(nb, (s + 1) kbs)) in chunks of KC.
__device__ __forceinline__ int split_blocks(const Params& p, int s) { return min(p.kbs, p.nb - s * p.kbs); }

template <int T, int NCB, int NCW>
__global__ void __launch_bounds__((NCW + 1) * 32, 1) gemv_kqm_kernel(const Params p,
                                                                    const __grid_constant__ CUtensorMap tmap) {
    constexpr int BB = Fmt<T>::BB;
    constexpr int REC = REC_UNIT * NCB;
    constexpr int MB = 8 * NCB;   // activation rows of the table (M padded)
    constexpr int NT = NCW * 32;  // consumer threads
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + MAX_STAGES;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + MAX_STAGES);
    volatile int* last_flag = abort_flag + 1;
    float* s_rs = reinterpret_cast<float*>(smem + p.off_rs);
    uint8_t* tab = smem + p.off_tab;
    float* part = reinterpret_cast<float*>(smem + p.off_part);  // [NCW][MB][TR]
    uint8_t* ring = smem + p.off_ring;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gi = blockIdx.x / p.SC, sc = blockIdx.x % p.SC;
    const int rlo = p.N / p.G, rex = p.N % p.G;
    const int r_begin = gi * rlo + min(gi, rex);
    const int r_end = r_begin + rlo + (gi < rex ? 1 : 0);
    const int ntiles = (r_end - r_begin + TR - 1) / TR;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], p.KC);  // one arrival per item (super-block) of the stage
        }
        *abort_flag = 0;
        *last_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == NCW) {
        // ------------------------------------------------------------ producer
        if (!p.early) pdl_wait_primary();
        const uint64_t pol = l2_policy_evict_first();
        int st = 0;
        bool stop = false;
        for (int s = sc; s < p.S && !stop; s += p.SC) {
            const int nbl = split_blocks(p, s), nch = (nbl + p.KC - 1) / p.KC;
            for (int tile = 0; tile < ntiles && !stop; ++tile) {
                for (int ch = 0; ch < nch; ++ch, ++st) {
                    const int slot = st % p.stages;
                    if (st >= p.stages &&
                        (!mbar_wait_bounded(&empty[slot], ((st / p.stages) - 1) & 1, DEV_TIMEOUT_EMPTY) ||
                         *abort_flag)) {
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    if (lane == 0) {
                        // the box starts on the 16-byte boundary at or below the
                        // chunk's first block (Q6_K blocks are 210 bytes)
                        const int byte0 = (s * p.kbs + ch * p.KC) * BB;
                        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(p.stage_bytes));
                        tma_box(ring + static_cast<size_t>(slot) * p.stage_bytes, &tmap, (byte0 & ~15) / 8,
                                tile_row0(tile, r_begin, r_end), &full[slot], pol);
                    }
                    __syncwarp();
                }
            }
        }
        if (lane == 0) {
            // Drain: no copy of this CTA may still be writing shared memory.
            const int issued = st;
            for (int s = 0; s < p.stages && s < issued; ++s) {
                const int last = issued - 1 - ((issued - 1 - s) % p.stages);
                mbar_wait_bounded(&full[s], (last / p.stages) & 1, DEV_TIMEOUT_DRAIN);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    pdl_wait_primary();
    for (int m = threadIdx.x; m < MB; m += NT) {
        float rs = 1.f;
        if (p.rms) {
            float tq = 0.f;
            for (int b = 0; b < p.nb; ++b) tq += p.rsq[static_cast<size_t>(m) * p.nb + b];
            rs = 1.0f / sqrtf(tq / static_cast<float>(p.K) + p.eps);
        }
        s_rs[m] = rs;
    }
    const int GW = p.GW, NG = NCW / GW;
    const int grp = warp / GW, jw = warp % GW;
    const int g = lane >> 2, t = lane & 3;
    int st = 0;
    bool ok = true;
    int js = 0;
    const int nsplit = (p.S - sc + p.SC - 1) / p.SC;
    for (int s = sc; s < p.S; s += p.SC, ++js) {
        const int nbl = split_blocks(p, s), nch = (nbl + p.KC - 1) / p.KC;
        // this split's table records, once every consumer is done with the last
        named_bar_sync(1, NT);
        {
            const uint8_t* src = p.tab + static_cast<size_t>(s) * p.kbs * REC;
            const int n16 = nbl * (REC / 16);
            for (int i = threadIdx.x; i < n16; i += NT) cp_async16(tab + 16 * i, src + 16 * i);
            cp_async_wait();
        }
        named_bar_sync(1, NT);
        for (int tile = grp; tile < ntiles; tile += NG) {
            float acc[NCB][4];
#pragma unroll
            for (int cb = 0; cb < NCB; ++cb) acc[cb][0] = acc[cb][1] = acc[cb][2] = acc[cb][3] = 0.f;
            for (int sb = jw; sb < nbl; sb += GW) {
                const int ch = sb / p.KC, sbl = sb - ch * p.KC;
                const uint32_t stg = static_cast<uint32_t>(st + tile * nch + ch);
                const uint32_t qs = __umulhi(stg, p.stage_magic);  // stg / stages
                const int slot = static_cast<int>(stg - qs * static_cast<uint32_t>(p.stages));
                if (ok && !*abort_flag) {
                    if (!mbar_wait_bounded(&full[slot], qs & 1u, DEV_TIMEOUT_FULL)) {
                        *abort_flag = 1;
                        ok = false;
                    }
                } else {
                    ok = false;
                }
                ok = __all_sync(0xffffffffu, ok);  // the item's MMAs need the whole warp
                if (ok) {
                    const int lead = ((s * p.kbs + ch * p.KC) * BB) & 15;
                    const uint8_t* bA = ring + static_cast<size_t>(slot) * p.stage_bytes + g * p.cs + lead + sbl * BB;
                    const uint8_t* bB = bA + 8 * p.cs;
                    const uint8_t* rec = tab + static_cast<size_t>(sb) * REC;
                    if constexpr (T == Q4_K) {
                        item_q4k<NCB>(bA, bB, rec, lane, acc);
                    } else if (((lead >> 1) + sbl) & 1) {  // block at 2 mod 4
                        item_q6k<NCB, true>(bA, bB, rec, lane, acc);
                    } else {
                        item_q6k<NCB, false>(bA, bB, rec, lane, acc);
                    }
                    // the stage's slot is free once all its items are done; the
                    // item that ends a short last chunk also accounts for the
                    // missing ones
                    const int kc = min(p.KC, nbl - ch * p.KC);
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cnt(&empty[slot], sbl == kc - 1 ? static_cast<uint32_t>(p.KC - kc + 1) : 1u);
                }
            }
            const int row0 = tile_row0(tile, r_begin, r_end);
            if (GW == 1) {  // the warp owns the tile: its lanes write their outputs
                if (ok && !*abort_flag) {
#pragma unroll
                    for (int cb = 0; cb < NCB; ++cb) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int m = 8 * cb + 2 * t + (i & 1), row = row0 + g + 8 * (i >> 1);
                            if (m >= p.M || row < r_begin + tile * TR || row >= r_end) continue;
                            float v = acc[cb][i];
                            if (p.SC == 1) {
                                float* y = p.Y + static_cast<size_t>(m) * p.ldy + row;
                                if (js > 0) v += *y;
                                if (js == nsplit - 1) v *= s_rs[m];
                                *y = v;
                            } else {
                                p.part[(static_cast<size_t>(s) * MB + m) * p.N + row] = v;
                            }
                        }
                    }
                }
                continue;
            }
            // this warp's rows of the tile: part[warp][m][row]
            float* pw = part + warp * (MB * TR);
#pragma unroll
            for (int cb = 0; cb < NCB; ++cb) {
#pragma unroll
                for (int i = 0; i < 4; ++i) pw[(8 * cb + 2 * t + (i & 1)) * TR + g + 8 * (i >> 1)] = acc[cb][i];
            }
            named_bar_sync(2 + grp, GW * 32);
            if (ok && !*abort_flag) {
                for (int e = lane + 32 * jw; e < MB * TR; e += GW * 32) {
                    const int m = e / TR, r = e % TR, row = row0 + r;
                    if (m >= p.M || row < r_begin + tile * TR || row >= r_end) continue;
                    const float* pb = part + (grp * GW) * (MB * TR) + e;
                    float v = 0.f;
                    for (int w = 0; w < GW; ++w) v += pb[w * (MB * TR)];
                    if (p.SC == 1) {
                        float* y = p.Y + static_cast<size_t>(m) * p.ldy + row;
                        if (js > 0) v += *y;
                        if (js == nsplit - 1) v *= s_rs[m];
                        *y = v;
                    } else {
                        p.part[(static_cast<size_t>(s) * MB + m) * p.N + row] = v;
                    }
                }
            }
            named_bar_sync(2 + grp, GW * 32);  // the group's partials are reused by its next tile
        }
        st += ntiles * nch;
    }
    if (p.SC == 1) return;
    // Splits in different CTAs: the CTA that completes a row range last sums
    // its S partials in split order.
    __threadfence();
    named_bar_sync(1, NT);
    if (threadIdx.x == 0) {
        const bool good = !*abort_flag;
        *last_flag = (good && atomicAdd(&p.cnt[gi], 1u) == static_cast<unsigned>(p.S - 1)) ? 1 : 0;
    }
    named_bar_sync(1, NT);
    if (!*last_flag) return;
    __threadfence();
    // four outputs per thread and pass, all their partials requested before
    // the first store (the loads of one pass are independent)
    const int rows = r_end - r_begin, total = p.M * rows;
    for (int e0 = threadIdx.x; e0 < total; e0 += 4 * NT) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        size_t off[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = min(e0 + u * NT, total - 1);
            off[u] = static_cast<size_t>(e / rows) * p.N + r_begin + e % rows;
        }
        for (int s = 0; s < p.S; ++s) {
            const float* ps = p.part + static_cast<size_t>(s) * MB * p.N;
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] += __ldcg(ps + off[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = e0 + u * NT;
            if (e >= total) break;
            const int m = e / rows, row = r_begin + e % rows;
            p.Y[static_cast<size_t>(m) * p.ldy + row] = v[u] * s_rs[m];
        }
    }
    if (threadIdx.x == 0) p.cnt[gi] = 0u;
}

}  // namespace kqm

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

using EncodeTiledKqm = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledKqm encode_kqm() {
    static EncodeTiledKqm fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledKqm>(f);
    });
    return fn;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// smem row stride >= bytes, an odd number of 16-byte units (the 8 rows of a
// fragment start in 8 distinct 16-byte bank groups)
int padded_stride(int bytes) {
    int s = static_cast<int>(align_up(static_cast<size_t>(bytes), 16));
    while (((s / 16) & 1) == 0) s += 16;
    return s;
}

// Blocks of 8 activation rows of the kernel that serves M rows.
int ncb_for(int M) {
    for (int ncb : {1, 2, 4})
        if (8 * ncb >= M) return ncb;
    return 0;
}

std::atomic<int> g_table_kb{0};  // KB of one split's table (SWQ_OPT_GEMV_BATCH_TABLE_KB, 0: automatic)
std::atomic<int> g_group{0};     // consumer warps per tile (SWQ_OPT_GEMV_BATCH_GROUP, 0: automatic)
constexpr size_t kSplitPartialLimit = 16u << 20;  // partials of CTA-parallel splits (stay in L2)

// K split and CTA layout for a table of at most table_kb KB per split.
struct KqmSplit {
    int kbs, S, SC, G, tiles_cta;
    size_t part_bytes;
};

KqmSplit split_for(int table_kb, size_t rec, int nb, int N, int MB, int num_sms) {
    KqmSplit q{};
    const int kbs_max = std::max<int>(1, static_cast<int>(static_cast<size_t>(table_kb) * 1024 / rec));
    const int S0 = (nb + kbs_max - 1) / kbs_max;
    q.kbs = (nb + S0 - 1) / S0;
    q.S = (nb + q.kbs - 1) / q.kbs;  // no empty split
    const int tiles = (N + kqm::TR - 1) / kqm::TR;
    q.part_bytes = static_cast<size_t>(q.S) * MB * N * sizeof(float);
    if (q.S > 1 && q.part_bytes <= kSplitPartialLimit && num_sms / q.S >= 1) {
        q.SC = q.S;
        q.G = std::max(1, std::min(tiles, num_sms / q.S));
    } else {
        q.SC = 1;
        q.G = std::max(1, std::min(tiles, num_sms));
    }
    const int rows_cta = (N + q.G - 1) / q.G;
    q.tiles_cta = (rows_cta + kqm::TR - 1) / kqm::TR;
    return q;
}

struct KqmPlan {
    kqm::Params p;
    int NCB = 0, NCW = 0, grid = 0;
    uint32_t smem = 0;
    size_t off_tab = 0, off_rsq = 0, off_part = 0, off_cnt = 0, ws_bytes = 0;
};

bool plan_kqm_at(int type, int M, int N, int K, int num_sms, int smem_optin, int table_kb, KqmPlan& P) {
    using namespace kqm;
    const int BB = type == Q4_K ? 144 : 210;
    Params& p = P.p;
    p = Params{};
    P.NCB = ncb_for(M);
    if (P.NCB == 0 || K <= 0 || K % 256 != 0 || N <= 0) return false;
    P.NCW = P.NCB >= 4 ? 8 : 16;
    const int MB = 8 * P.NCB;  // table rows (M padded)
    const size_t rec = static_cast<size_t>(REC_UNIT) * P.NCB;
    p.N = N;
    p.K = K;
    p.nb = K / 256;
    p.M = M;
    p.ldy = N;
    const KqmSplit q = split_for(table_kb, rec, p.nb, N, MB, num_sms);
    p.kbs = q.kbs;
    p.S = q.S;
    p.SC = q.SC;
    p.G = q.G;
    const size_t part_bytes = q.part_bytes;
    P.grid = p.G * p.SC;
    p.KC = std::min(p.kbs, 8);
    const int nch_max = (p.kbs + p.KC - 1) / p.KC;
    // Q6_K: a chunk's box starts up to 14 bytes below its first block
    p.cs = padded_stride(p.KC * BB + (BB % 16 ? 14 : 0));
    if (p.cs / 8 > 256) return false;  // the box's inner extent limit
    p.stage_bytes = TR * p.cs;
    // Warps per tile group: a power of two up to the split's super-blocks (or
    // the tuned value), at most 8 groups (named barriers 2..9).  A group waits
    // for the stages of its next tile while the others hold theirs, so the
    // ring holds at least one tile's stages per group: a wait then never
    // reaches a slot more than one lap ahead (an mbarrier parity wait cannot
    // tell that lap from the previous one).
    // Automatically: at least two tiles per group (a group neither idles nor
    // ends on a lone last tile), at least two warps per group, at most the
    // split's super-blocks (B200: the 8-row LM head 128256 x 4096 Q6_K takes
    // 150 us with groups of 4 warps, 176 us with 8).
    int gw = 1;
    while (gw < P.NCW && gw * q.tiles_cta < 2 * P.NCW) gw *= 2;
    gw = std::max(gw, 2);
    while (gw > 1 && gw > p.kbs) gw /= 2;
    if (g_group.load() > 0) gw = std::min(g_group.load(), P.NCW);
    while ((gw > 1 && P.NCW / gw > 8) || P.NCW % gw != 0) gw *= 2;
    const uint32_t budget = static_cast<uint32_t>(smem_optin) - 1024u;
    const int need = q.tiles_cta * nch_max * (p.SC == 1 ? p.S : 1);
    uint32_t off = 0;
    for (;; gw *= 2) {
        off = static_cast<uint32_t>(2 * MAX_STAGES * 8 + 16);
        p.off_rs = off;
        off += static_cast<uint32_t>(MB * 4);
        off = static_cast<uint32_t>(align_up(off, 128));
        p.off_tab = off;
        off += static_cast<uint32_t>(p.kbs * rec);
        off = static_cast<uint32_t>(align_up(off, 16));
        p.off_part = off;
        if (gw > 1) off += static_cast<uint32_t>(P.NCW * MB * TR * 4);
        off = static_cast<uint32_t>(align_up(off, 128));
        p.off_ring = off;
        if (off + 2u * p.stage_bytes > budget) return false;
        p.stages = std::max(2, std::min<int>({static_cast<int>((budget - off) / p.stage_bytes), MAX_STAGES, need}));
        if (p.stages >= std::min(need, (P.NCW / gw) * nch_max)) break;
        if (gw >= P.NCW) return false;
    }
    p.GW = gw;
    p.stage_magic = static_cast<uint32_t>((0x100000000ull + static_cast<uint64_t>(p.stages) - 1) /
                                          static_cast<uint64_t>(p.stages));
    P.smem = off + static_cast<uint32_t>(p.stages) * p.stage_bytes;
    // workspace: table records, sums of squares, split partials, counters
    size_t ws = 0;
    P.off_tab = ws;
    ws = align_up(ws + static_cast<size_t>(p.nb) * rec, 256);
    P.off_rsq = ws;
    ws = align_up(ws + static_cast<size_t>(MB) * p.nb * sizeof(float), 256);
    P.off_part = ws;
    if (p.SC > 1) ws = align_up(ws + part_bytes, 256);
    P.off_cnt = ws;
    ws = align_up(ws + static_cast<size_t>(p.G) * sizeof(unsigned), 256);
    P.ws_bytes = ws;
    return true;
}

// Table size: the tuned value, else 72 KB (8 super-blocks per split for up
// to 8 rows, 4 for 16), or 144 KB for 9..16 rows where each CTA still gets 8
// tiles or more (8 super-blocks per split: half the splits and per-tile sums;
// on B200 gate+up 28672 x 4096 at 16 rows 57.8 -> 48.2 us; slower on small
// matrices, whose CTAs then hold few tiles).
bool plan_kqm(int type, int M, int N, int K, int num_sms, int smem_optin, KqmPlan& P) {
    if (g_table_kb.load() > 0) return plan_kqm_at(type, M, N, K, num_sms, smem_optin, g_table_kb.load(), P);
    if (ncb_for(M) == 2 && K > 0 && K % 256 == 0 && N > 0) {
        const size_t rec = static_cast<size_t>(kqm::REC_UNIT) * 2;
        if (split_for(144, rec, K / 256, N, 16, num_sms).tiles_cta >= 8 &&
            plan_kqm_at(type, M, N, K, num_sms, smem_optin, 144, P))
            return true;
    }
    return plan_kqm_at(type, M, N, K, num_sms, smem_optin, 72, P);
}

bool kqm_shape_ok(int type, const void* W, int M, int N, int K, int max_m) {
    if (type != Q4_K && type != Q6_K) return false;
    if (M < 2 || M > std::min(max_m, 32) || N <= 0 || K <= 0 || K % 256 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(W) & 15u) != 0) return false;
    if (type == Q6_K && (K / 256) % 8 != 0) return false;  // rows of 210-byte blocks 16-byte aligned
    return encode_kqm() != nullptr;
}

template <int T, int NCB>
cudaError_t launch_t(const KqmPlan& P, const kqm::PrepParams& pp, const CUtensorMap& tmap, cudaStream_t s) {
    constexpr int NCW = NCB >= 4 ? 8 : 16;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(pp.nb, NCB);
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, kqm::prep_kernel<NCB>, pp);
        if (e != cudaSuccess) return e;
    }
    auto kern = kqm::gemv_kqm_kernel<T, NCB, NCW>;
    static thread_local int set_dev = -1;
    static thread_local uint32_t set_smem = 0;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != set_dev || P.smem > set_smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(P.smem));
        if (e != cudaSuccess) return e;
        set_dev = dev;
        set_smem = P.smem;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(P.grid);
    cfg.blockDim = dim3((NCW + 1) * 32);
    cfg.dynamicSmemBytes = P.smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, P.p, tmap);
}

template <int T>
cudaError_t launch_ncb(const KqmPlan& P, const kqm::PrepParams& pp, const CUtensorMap& tmap, cudaStream_t s) {
    switch (P.NCB) {
        case 1: return launch_t<T, 1>(P, pp, tmap, s);
        case 2: return launch_t<T, 2>(P, pp, tmap, s);
        case 4: return launch_t<T, 4>(P, pp, tmap, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

void gemv_kqm_tune(int table_kb, int group) {
    g_table_kb = std::max(8, table_kb);
    g_group = group;
}

bool gemv_kqm_supported(int type, const void* W, int M, int N, int K, int max_m, int num_sms, int smem_optin) {
    if (!kqm_shape_ok(type, W, M, N, K, max_m)) return false;
    KqmPlan P;
    return plan_kqm(type, M, N, K, num_sms, smem_optin, P);
}

size_t gemv_kqm_workspace_bytes(int type, int M, int N, int K, int num_sms, int smem_optin) {
    KqmPlan P;
    if (!plan_kqm(type, M, N, K, num_sms, smem_optin, P)) return 0;
    return P.ws_bytes;
}

cudaError_t gemv_kqm_launch(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                            const ActArgs& act, int early, int num_sms, int smem_optin, void* ws, size_t ws_bytes,
                            cudaStream_t s) {
    KqmPlan P;
    if (!plan_kqm(type, M, N, K, num_sms, smem_optin, P)) return cudaErrorNotSupported;
    if (ws == nullptr || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0 || ws_bytes < P.ws_bytes)
        return cudaErrorInvalidValue;
    uint8_t* base = static_cast<uint8_t*>(ws);
    kqm::Params& p = P.p;
    const int BB = type == Q4_K ? 144 : 210;
    const int row_bytes = (K / 256) * BB;
    p.W = static_cast<const uint8_t*>(W);
    p.Y = Y;
    p.tab = base + P.off_tab;
    p.rsq = act.kind == ACT_RMSNORM ? reinterpret_cast<const float*>(base + P.off_rsq) : nullptr;
    p.part = p.SC > 1 ? reinterpret_cast<float*>(base + P.off_part) : nullptr;
    p.cnt = reinterpret_cast<unsigned*>(base + P.off_cnt);
    p.early = early;
    p.rms = act.kind == ACT_RMSNORM ? 1 : 0;
    p.eps = act.eps;

    kqm::PrepParams pp{};
    pp.X = X;
    pp.ld = act.ld > 0 ? act.ld : K;
    pp.tab = base + P.off_tab;
    pp.rsq = act.kind == ACT_RMSNORM ? reinterpret_cast<float*>(base + P.off_rsq) : nullptr;
    pp.cnt = p.cnt;
    pp.ncnt = p.G;
    pp.M = M;
    pp.K = K;
    pp.nb = K / 256;
    pp.act = act.kind;
    pp.R = act.R;
    pp.normw = act.normw;
    pp.sum_out = act.sum_out;
    const auto a16 = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    pp.vec = (a16(X) && a16(act.R) && a16(act.normw) && a16(act.sum_out) && pp.ld % 4 == 0 && K % 4 == 0) ? 1 : 0;

    CUtensorMap tmap;
    std::memset(&tmap, 0, sizeof(tmap));
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 8), static_cast<cuuint64_t>(N)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(p.cs / 8), static_cast<cuuint32_t>(kqm::TR)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = encode_kqm()(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(W), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    return type == Q4_K ? launch_ncb<Q4_K>(P, pp, tmap, s) : launch_ncb<Q6_K>(P, pp, tmap, s);
}

SWQ_DEFINE_STATUS_FETCH(gemv_kqm)

}  // namespace swq
