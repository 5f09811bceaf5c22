// gemv_kq.cu -- single-row K-quant GEMVs y = W . x (Q4_K, Q6_K) with exact
// integer sub-block dot products on the tensor cores and one floating-point
// conversion per super-block (sm_100a).
//
// Replaces cpu_matmul_transposed_q4_k / _q6_k (src/tensor.h:769-856) behind
// Compute::matmul_transposed_q (src/tensor.h:1212) for the decode
// projections.  The reference evaluates, per row, in fp32
//     Q4_K: y = sum_b sum_j sum_{k in j} (d_b sc_j q_k - dmin_b m_j) x_k
//           (super-block b of 256 weights, sub-block j of 32, 6-bit sc_j,
//           m_j, 4-bit q_k)
//     Q6_K: y = sum_b sum_j sum_{k in j} d_b sc_j (q_k - 32) x_k
//           (sub-block j of 16, int8 sc_j, 6-bit q_k)
// Here the same sums are formed as
//     Q4_K: y = sum_b [ d_b * sum_j sc_j S_j  -  dmin_b * sum_j m_j X_j ]
//     Q6_K: y = sum_b d_b * [ sum_j sc_j S_j  -  32 * sum_j sc_j X_j ]
//     S_j = sum_{k in j} q_k x_k  (exact: integers),  X_j = sum_{k in j} x_k,
// with x held per super-block as a 30-bit fixed-point number
// x_k = Z_k 2^(E_b - 30) (E_b: the super-block's largest binary exponent) and
// Z_k split into four signed 8-bit limbs.  One mma.sync m16n8k32
// (u8 x s8 -> s32) multiplies 16 weight rows by the four limbs of 32
// activations; the products and the int32 sums are exact; the sub-block scale
// sc_j is applied with an integer multiply-add, so a whole super-block is
// summed exactly in int32 and converted to fp32 once.  Error sources: the
// activation rounding (|dx| <= 2^(E_b - 31), below fp32's rounding of the
// super-block's largest element), one conversion per super-block and the fp32
// accumulation over super-blocks -- the reference rounds every product and
// every addition instead.
//
// Why tensor cores in a bandwidth-bound kernel: on CUDA cores every weight
// costs a byte permute, a float add and a multiply-add (plus the activation
// loads); at 4.5-6.6 bits per weight that issue rate, not HBM, bounds a
// decode GEMV.  Here a masked word of four quant bytes is an MMA operand.
//
// Structure: persistent CTA per SM (balanced contiguous row ranges), 16-row
// tiles (the MMA's M).  One producer warp issues every stage of the CTA --
// a TMA box of 16 rows x KC super-blocks, landing at a padded row stride --
// into a shared-memory ring, requesting weights before griddepcontrol.wait
// (they are immutable inputs).
// The consumer warps first turn x into the limb table (after the wait), then
// take (tile, super-block) items round-robin; a warp sums its items of a tile
// in registers; the rows are finally summed over the warps in warp order
// (deterministic).  Every wait is bounded.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "formats.cuh"
#include "gemv.h"
#include "swq_device.cuh"

namespace swq {
namespace kq {

// NCW consumer warps + one producer warp: 16 (two CTAs per SM) or 8 (up to
// four CTAs per SM, for more kernels in flight at once)
template <int NCW>
struct Shape {
    static constexpr int THREADS = (NCW + 1) * 32;
};
constexpr int TR = 16;  // rows per tile (the MMA's M)
constexpr int MAX_STAGES = 16;

// Per format: block bytes, the largest K (the limb table holds K / 64 * 256
// bytes of shared memory), the blocks a row must come in for 16-byte aligned
// rows, sub-block sums per super-block.
template <int T>
struct KQ;
template <>
struct KQ<Q4_K> {
    static constexpr int BB = 144, MAX_K = 8192, ALIGN_NB = 2, SUMS = 8;
};
template <>
struct KQ<Q6_K> {
    static constexpr int BB = 210, MAX_K = 16384, ALIGN_NB = 8, SUMS = 16;
};

struct Params {
    const uint8_t* W;
    const float* X;
    float* Y;
    int N, K, nb, row_bytes;
    int KC, nchunks;  // super-blocks per chunk, chunks per row
    int cs;           // shared-memory bytes of one row of a chunk (KC * 144, padded)
    int stage_bytes;  // TR * cs
    int stages;
    uint32_t stage_magic;  // ceil(2^32 / stages): st / stages = umulhi(st, stage_magic) for st < 2^28
    int early;
    int x_vec;  // activation rows 16-byte aligned
    uint32_t off_xt, off_xe, off_xsum, off_part, off_ring;
    // activation prologue (ACT_*), as in the CUDA-core GEMV:
    //   RMSNORM: x = X (+ R), then x * normw; the outputs scale by 1 / rms(x);
    //            CTA 0 writes x to sum_out when given
    //   SWIGLU:  x_k = silu(X[k]) * X[K + k]
    int act;
    const float* R;
    const float* normw;
    float eps;
    float* sum_out;
};

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One stage: a box of TR rows x (cs / 8) 8-byte elements of the weight matrix
// (tensor map over [N rows][row_bytes / 8]); rows and bytes past the matrix
// read as zeros.  The box's inner extent is the padded row stride, so the rows
// land at that stride in shared memory.  Into this CTA only.
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

// First row of tile `tile` of the CTA's range [r_begin, r_end): a last tile
// that would run past r_end starts lower (on rows the previous tile just
// read) when the range holds a whole tile, so no tile reads another CTA's rows.
__device__ __forceinline__ int tile_row0(int tile, int r_begin, int r_end) {
    const int r0 = r_begin + tile * TR;
    return (r0 + TR > r_end && r_end - TR >= r_begin) ? r_end - TR : r0;
}

// 8 consecutive floats (two float4 loads when VEC)
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

// Limb table of x, one warp per super-block b, lane l taking the 8 elements
// 256 b + 8 l .. + 7.
//
// Q4_K MMA operand order: lane (g, t) of a fragment loads the 8 quant bytes
// 8t .. 8t + 7 of a unit's 32 (one 64-bit load per row) as its A words for
// k = 4t .. 4t + 3 and k = 16 + 4t .. 16 + 4t + 3, so B row k holds the
// activation of quant byte 8t + i (k = 4t + i) or 8t + 4 + i (k = 16 + 4t + i).
// Low nibbles are the unit's first 32 elements (MMA 0, output columns 0..3
// = limbs 0..3), high nibbles its last 32 (MMA 1, columns 4..7).
//   xt: Q4_K -- per unit, per lane (g, t): 8 bytes, limb (g mod 4) of the
//       8 activations of quant bytes 8t .. 8t + 7 of the low-nibble half
//       (g < 4, MMA 0) or of the high-nibble half (g >= 4, MMA 1); the other
//       MMA's operand of that lane is zero (masked in the consumer).
//       Q6_K -- per unit (nn, h) = 64 elements in 4 planes of 16 (plane p:
//       elements 128 nn + 32 p + 16 h .. + 15, sub-block 8 nn + 2 p + h),
//       per MMA m (planes 2m, 2m + 1), per lane (g, t): 4 bytes, limb (g mod
//       4) of elements 4t .. 4t + 3 of plane 2m (g < 4) or 2m + 1 (g >= 4).
//   xe: per super-block 2^(E_b - 30) (NaN when the super-block holds a
//       non-finite value, so that it propagates).
//   xsum: per sub-block j, sum(x) over its elements (fp32, fixed order), 16
//       slots per super-block.
template <int T, int NCW>
__device__ __forceinline__ void prep_x(const Params& p, uint8_t* xt, float* xe, float* xsum, int warp, int lane,
                                       float& sq) {
    const bool rms = p.act == ACT_RMSNORM;
    for (int b = warp; b < p.nb; b += NCW) {
        const int e0 = 256 * b + 8 * lane;
        float v[8];
        if (p.act == ACT_SWIGLU) {
            float gt[8], up[8];
            ld8(p.X + e0, gt, p.x_vec);
            ld8(p.X + p.K + e0, up, p.x_vec);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = gt[i] / (1.0f + expf(-gt[i])) * up[i];
        } else {
            ld8(p.X + e0, v, p.x_vec);
            if (rms) {
                if (p.R) {
                    float r[8];
                    ld8(p.R + e0, r, p.x_vec);
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] += r[i];
                }
                if (p.sum_out && blockIdx.x == 0) {
                    if (p.x_vec) {
                        reinterpret_cast<float4*>(p.sum_out + e0)[0] = make_float4(v[0], v[1], v[2], v[3]);
                        reinterpret_cast<float4*>(p.sum_out + e0)[1] = make_float4(v[4], v[5], v[6], v[7]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) p.sum_out[e0 + i] = v[i];
                    }
                }
                float w[8];
                ld8(p.normw + e0, w, p.x_vec);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    sq = fmaf(v[i], v[i], sq);
                    v[i] *= w[i];
                }
            }
        }
        float mx = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
        bool nonfinite = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) nonfinite |= !(fabsf(v[i]) <= 3.402823466e38f);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        nonfinite = __any_sync(0xffffffffu, nonfinite);
        // E: mx < 2^E; Z = x 2^(30 - E) lies in (-2^30, 2^30).  E stays >= -96
        // so that both scale factors are normal floats: a super-block whose
        // largest element is below 2^-97 keeps fewer bits.  Beside blocks of
        // normal magnitude that is far under fp32's resolution of the row's
        // sum; a row made only of such blocks loses accuracy (about 1e-3 at
        // 1e-35, most of the value at fp32's smallest normals).
        const int ebits = (__float_as_int(mx) >> 23) & 0xFF;
        const int E = max(ebits - 126, -96);
        const float up_s = nonfinite ? 0.f : __int_as_float((127 + 30 - E) << 23);  // 2^(30 - E)
        uint32_t Z[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            // signed base-256 digits: bytes of Y = Z + 0x808080 with the low
            // three biased by 128 (byte ^ 0x80 = byte - 128 as int8), the top
            // byte as is; |Z| < 2^30 keeps the top digit within -64..64.
            const int z = __float2int_rn(v[i] * up_s);
            Z[i] = (static_cast<uint32_t>(z) + 0x808080u) ^ 0x808080u;
        }
        // 4 x 4 byte transposes: limb n of elements 0..3 and of 4..7
        uint32_t L0[4], L1[4];
        {
            const uint32_t a = __byte_perm(Z[0], Z[1], 0x5140), c = __byte_perm(Z[0], Z[1], 0x7362);
            const uint32_t e = __byte_perm(Z[2], Z[3], 0x5140), f = __byte_perm(Z[2], Z[3], 0x7362);
            L0[0] = __byte_perm(a, e, 0x5410);
            L0[1] = __byte_perm(a, e, 0x7632);
            L0[2] = __byte_perm(c, f, 0x5410);
            L0[3] = __byte_perm(c, f, 0x7632);
        }
        {
            const uint32_t a = __byte_perm(Z[4], Z[5], 0x5140), c = __byte_perm(Z[4], Z[5], 0x7362);
            const uint32_t e = __byte_perm(Z[6], Z[7], 0x5140), f = __byte_perm(Z[6], Z[7], 0x7362);
            L1[0] = __byte_perm(a, e, 0x5410);
            L1[1] = __byte_perm(a, e, 0x7632);
            L1[2] = __byte_perm(c, f, 0x5410);
            L1[3] = __byte_perm(c, f, 0x7632);
        }
        float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        if constexpr (T == Q4_K) {
            // lane = (unit c, half m, quarter t): element 64 c + 32 m + 8 t + i
            const int c = lane >> 3, m = (lane >> 2) & 1, t = lane & 3;
            uint8_t* tu = xt + static_cast<size_t>(4 * b + c) * 256;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                const int ln = 4 * (n + 4 * m) + t;  // fragment lane of limb n
                *reinterpret_cast<uint2*>(tu + ln * 8) = make_uint2(L0[n], L1[n]);
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (t == 0) xsum[16 * b + 2 * c + m] = s;
        } else {
            // lane = (half nn, plane pp, h, quarter pair): element
            // 128 nn + 32 pp + 16 h + 4 t + i with t = t0 (i < 4) or t0 + 1
            const int nn = lane >> 4, pp = (lane >> 2) & 3, h = (lane & 3) >> 1, t0 = 2 * (lane & 1);
            uint8_t* tu = xt + static_cast<size_t>(4 * b + 2 * nn + h) * 256 + (pp >> 1) * 128;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                const int ln = 4 * (n + 4 * (pp & 1)) + t0;  // fragment lane of limb n
                *reinterpret_cast<uint32_t*>(tu + ln * 4) = L0[n];
                *reinterpret_cast<uint32_t*>(tu + (ln + 1) * 4) = L1[n];
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            if ((lane & 1) == 0) xsum[16 * b + 8 * nn + 2 * pp + h] = s;
        }
        if (lane == 0) xe[b] = nonfinite ? __int_as_float(0x7fc00000) : __int_as_float((127 + E - 30) << 23);
    }
}


// 32-bit word at a block offset that is a multiple of 4: blocks of 210 bytes
// (Q6_K) sit at 2-byte aligned addresses every other block (ODD), read as two
// aligned words and a funnel shift.
template <bool ODD>
__device__ __forceinline__ uint32_t ld32(const uint8_t* q) {
    if constexpr (!ODD) {
        return *reinterpret_cast<const uint32_t*>(q);
    } else {
        const uint32_t* a = reinterpret_cast<const uint32_t*>(q - 2);
        return __funnelshift_r(a[0], a[1], 16);
    }
}

// One Q4_K item: super-block sb of the tile's rows g (bA) and g + 8 (bB),
// limb table xu of the super-block (this lane's slot), sub-block sums xj.
__device__ __forceinline__ void item_q4k(const uint8_t* bA, const uint8_t* bB, const uint8_t* xu, const float* xj,
                                         float xs, int t, int par, uint32_t lo_mask, float lw0, float lw1,
                                         float& accA, float& accB) {
    const uint4 hA = lds_u128(bA), hB = lds_u128(bB);
    // 6-bit scales of sub-blocks 2c + par (get_scale_min_k4,
    // src/tensor.h:218-227): c < 2 from bytes 0..3, c >= 2 from 8..11 with the
    // high bits of 0..3; shifted so that unit c's scale is byte 0 (c even) or
    // 2 (c odd).
    const uint32_t sloA = (hA.y & 0x3F3F3F3Fu) >> (8 * par);
    const uint32_t shiA = ((hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u)) >> (8 * par);
    const uint32_t sloB = (hB.y & 0x3F3F3F3Fu) >> (8 * par);
    const uint32_t shiB = ((hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u)) >> (8 * par);
    int T0 = 0, T1 = 0, T2 = 0, T3 = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint2 wA = *reinterpret_cast<const uint2*>(bA + 16 + 32 * c + 8 * t);
        const uint2 wB = *reinterpret_cast<const uint2*>(bB + 16 + 32 * c + 8 * t);
        const uint2 bx = *reinterpret_cast<const uint2*>(xu + c * 256);
        int d[4] = {0, 0, 0, 0};
        mma_u8s8(d, wA.x & 0x0F0F0F0Fu, wB.x & 0x0F0F0F0Fu, wA.y & 0x0F0F0F0Fu, wB.y & 0x0F0F0F0Fu, bx.x & lo_mask,
                 bx.y & lo_mask);
        mma_u8s8(d, wA.x & 0xF0F0F0F0u, wB.x & 0xF0F0F0F0u, wA.y & 0xF0F0F0F0u, wB.y & 0xF0F0F0F0u, bx.x & ~lo_mask,
                 bx.y & ~lo_mask);
        const uint32_t wsA = c < 2 ? sloA : shiA, wsB = c < 2 ? sloB : shiB;
        const int scA = static_cast<int>((wsA >> (16 * (c & 1))) & 0xFFu);
        const int scB = static_cast<int>((wsB >> (16 * (c & 1))) & 0xFFu);
        T0 += scA * d[0];
        T1 += scA * d[1];
        T2 += scB * d[2];
        T3 += scB * d[3];
    }
    const float vA = fmaf(static_cast<float>(T1), lw1, static_cast<float>(T0) * lw0) * xs;
    const float vB = fmaf(static_cast<float>(T3), lw1, static_cast<float>(T2) * lw0) * xs;
    const float2 dmA = __half22float2(*reinterpret_cast<const __half2*>(&hA.x));
    const float2 dmB = __half22float2(*reinterpret_cast<const __half2*>(&hB.x));
    // mins of sub-blocks 2t and 2t + 1 (bytes 4..7, or 8..11 high nibbles with
    // the high bits of 4..7), times their sums of x
    const uint32_t mnA =
        (t < 2 ? (hA.z & 0x3F3F3F3Fu) : (((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u))) >> (16 * (t & 1));
    const uint32_t mnB =
        (t < 2 ? (hB.z & 0x3F3F3F3Fu) : (((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u))) >> (16 * (t & 1));
    const float2 x2 = *reinterpret_cast<const float2*>(xj + 2 * t);
    const float mmA = fmaf(static_cast<float>((mnA >> 8) & 0xFFu), x2.y, static_cast<float>(mnA & 0xFFu) * x2.x);
    const float mmB = fmaf(static_cast<float>((mnB >> 8) & 0xFFu), x2.y, static_cast<float>(mnB & 0xFFu) * x2.x);
    accA = fmaf(-dmA.y, mmA, fmaf(dmA.x, vA, accA));
    accB = fmaf(-dmB.y, mmB, fmaf(dmB.x, vB, accB));
}

__device__ __forceinline__ int sext8(uint32_t w, int byte) {
    return static_cast<int>(static_cast<int8_t>(static_cast<uint8_t>(w >> (8 * byte))));
}

// One Q6_K item (src/tensor.h:398-432 layout: ql[128] @0, qh[64] @128,
// int8 scales[16] @192, fp16 d @208).  Unit c = (half nn, h): lane t holds
// the four 6-bit values at l = 16 h + 4t .. + 3 of each plane p (elements
// 128 nn + 32 p + l, sub-block 8 nn + 2 p + h).  MMA 0 takes planes 0 and 1,
// MMA 1 planes 2 and 3; this lane's output columns belong to plane 2m + par.
template <bool ODD>
__device__ __forceinline__ void item_q6k(const uint8_t* bA, const uint8_t* bB, const uint8_t* xu, const float* xj,
                                         float xs, int t, int par, uint32_t lo_mask, float lw0, float lw1,
                                         float& accA, float& accB) {
    uint32_t SA[4], SB[4];  // scale words, shifted so that byte h is sub-block 4q + 2 par + h
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        SA[q] = ld32<ODD>(bA + 192 + 4 * q) >> (16 * par);
        SB[q] = ld32<ODD>(bB + 192 + 4 * q) >> (16 * par);
    }
    int T0 = 0, T1 = 0, T2 = 0, T3 = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int nn = c >> 1, h = c & 1;
        const int o = 64 * nn + 16 * h + 4 * t;
        const uint32_t L0A = ld32<ODD>(bA + o), L1A = ld32<ODD>(bA + o + 32);
        const uint32_t HA = ld32<ODD>(bA + 128 + 32 * nn + 16 * h + 4 * t);
        const uint32_t L0B = ld32<ODD>(bB + o), L1B = ld32<ODD>(bB + o + 32);
        const uint32_t HB = ld32<ODD>(bB + 128 + 32 * nn + 16 * h + 4 * t);
        const uint32_t bx0 = *reinterpret_cast<const uint32_t*>(xu + c * 256);
        const uint32_t bx1 = *reinterpret_cast<const uint32_t*>(xu + c * 256 + 128);
        int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};
        mma_u8s8(d0, (L0A & 0x0F0F0F0Fu) | ((HA << 4) & 0x30303030u), (L0B & 0x0F0F0F0Fu) | ((HB << 4) & 0x30303030u),
                 (L1A & 0x0F0F0F0Fu) | ((HA << 2) & 0x30303030u), (L1B & 0x0F0F0F0Fu) | ((HB << 2) & 0x30303030u),
                 bx0 & lo_mask, bx0 & ~lo_mask);
        mma_u8s8(d1, ((L0A >> 4) & 0x0F0F0F0Fu) | (HA & 0x30303030u), ((L0B >> 4) & 0x0F0F0F0Fu) | (HB & 0x30303030u),
                 ((L1A >> 4) & 0x0F0F0F0Fu) | ((HA >> 2) & 0x30303030u),
                 ((L1B >> 4) & 0x0F0F0F0Fu) | ((HB >> 2) & 0x30303030u), bx1 & lo_mask, bx1 & ~lo_mask);
        const int sA0 = sext8(SA[2 * nn], h), sA1 = sext8(SA[2 * nn + 1], h);
        const int sB0 = sext8(SB[2 * nn], h), sB1 = sext8(SB[2 * nn + 1], h);
        T0 += sA0 * d0[0] + sA1 * d1[0];
        T1 += sA0 * d0[1] + sA1 * d1[1];
        T2 += sB0 * d0[2] + sB1 * d1[2];
        T3 += sB0 * d0[3] + sB1 * d1[3];
    }
    const float vA = fmaf(static_cast<float>(T1), lw1, static_cast<float>(T0) * lw0) * xs;
    const float vB = fmaf(static_cast<float>(T3), lw1, static_cast<float>(T2) * lw0) * xs;
    // zero point 32: sub-blocks 4t .. 4t + 3 of this lane, sum_j sc_j X_j
    const uint32_t zA = ld32<ODD>(bA + 192 + 4 * t), zB = ld32<ODD>(bB + 192 + 4 * t);
    const float4 x4 = *reinterpret_cast<const float4*>(xj + 4 * t);
    float mA = static_cast<float>(sext8(zA, 0)) * x4.x, mB = static_cast<float>(sext8(zB, 0)) * x4.x;
    mA = fmaf(static_cast<float>(sext8(zA, 1)), x4.y, mA);
    mB = fmaf(static_cast<float>(sext8(zB, 1)), x4.y, mB);
    mA = fmaf(static_cast<float>(sext8(zA, 2)), x4.z, mA);
    mB = fmaf(static_cast<float>(sext8(zB, 2)), x4.z, mB);
    mA = fmaf(static_cast<float>(sext8(zA, 3)), x4.w, mA);
    mB = fmaf(static_cast<float>(sext8(zB, 3)), x4.w, mB);
    const float dA = __half2float(*reinterpret_cast<const __half*>(bA + 208));
    const float dB = __half2float(*reinterpret_cast<const __half*>(bB + 208));
    accA = fmaf(dA, fmaf(-32.0f, mA, vA), accA);
    accB = fmaf(dB, fmaf(-32.0f, mB, vB), accB);
}

template <int T, int NCW>
__global__ void __launch_bounds__(Shape<NCW>::THREADS, NCW == 16 ? 2 : 3)
    gemv_kq_kernel(const Params p, const __grid_constant__ CUtensorMap tmap) {
    constexpr int BB = KQ<T>::BB;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + MAX_STAGES;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + MAX_STAGES);
    uint8_t* xt = smem + p.off_xt;
    float* xe = reinterpret_cast<float*>(smem + p.off_xe);
    float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);
    float* part = reinterpret_cast<float*>(smem + p.off_part);  // [tile][NCW][TR]
    uint8_t* ring = smem + p.off_ring;
    __shared__ float s_sq[NCW];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, bi = blockIdx.x;
    const int rlo = p.N / G, rex = p.N % G;
    const int r_begin = bi * rlo + min(bi, rex);
    const int r_end = r_begin + rlo + (bi < rex ? 1 : 0);
    const int ntiles = (r_end - r_begin + TR - 1) / TR;
    const int nstage = ntiles * p.nchunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], p.KC);  // one arrival per item (super-block) of the stage
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == NCW) {
        // ------------------------------------------------------------ producer
        if (!p.early) pdl_wait_primary();
        const uint64_t pol = l2_policy_evict_first();
        int issued = 0;
        for (int st = 0; st < nstage; ++st, ++issued) {
            const int s = st % p.stages;
            if (st >= p.stages) {
                if (!mbar_wait_bounded(&empty[s], ((st / p.stages) - 1) & 1, DEV_TIMEOUT_EMPTY) || *abort_flag) {
                    *abort_flag = 1;
                    break;
                }
            }
            const int tile = st / p.nchunks, ch = st % p.nchunks;
            uint8_t* dst = ring + static_cast<size_t>(s) * p.stage_bytes;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(p.stage_bytes));
                tma_box(dst, &tmap, ch * p.KC * BB / 8, tile_row0(tile, r_begin, r_end), &full[s], pol);
            }
            __syncwarp();
        }
        if (lane == 0) {
            // Drain: no copy of this CTA may still be writing shared memory.
            for (int s = 0; s < p.stages && s < issued; ++s) {
                const int last = issued - 1 - ((issued - 1 - s) % p.stages);
                mbar_wait_bounded(&full[s], (last / p.stages) & 1, DEV_TIMEOUT_DRAIN);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    pdl_wait_primary();
    float sq = 0.f;
    prep_x<T, NCW>(p, xt, xe, xsum, warp, lane, sq);
    if (p.act == ACT_RMSNORM) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) s_sq[warp] = sq;
    }
    // Work split.  nb >= NCW: warp w multiplies super-blocks w, w + NCW, ...
    // of every tile -- exactly the ones it prepared, so it needs no other
    // warp's table entries and no CTA barrier, and it writes its partial of
    // every tile.  nb < NCW: R = NCW / nb warps share each super-block
    // (replica r = w / nb takes tiles r, r + R, ...) after a barrier that
    // publishes the table; warps past R * nb only take part in the barriers.
    const bool own = p.nb >= NCW;
    const int R = own ? 1 : NCW / p.nb;
    const int sb0 = own ? warp : warp % p.nb;
    const int t0 = own ? 0 : warp / p.nb;
    if (own) {
        __syncwarp();
    } else {
        for (int i = threadIdx.x; i < ntiles * NCW * TR; i += NCW * 32) part[i] = 0.f;
        named_bar_sync(1, NCW * 32);
    }

    const int g = lane >> 2, t = lane & 3;
    const int par = t >> 1;  // output columns 4..7: Q4_K the high-nibble sub-block, Q6_K the odd plane
    // limb weights of this lane's two output columns (limbs 2 (t & 1) and
    // 2 (t & 1) + 1); Q4_K high nibbles are read in place (x 16)
    const float lw0 = ((t & 1) ? 65536.0f : 1.0f) * (T == Q4_K && par ? 0.0625f : 1.0f);
    const float lw1 = lw0 * 256.0f;
    const uint32_t lo_mask = g < 4 ? 0xFFFFFFFFu : 0u;  // this lane's B column is in MMA 0's half
    const int ch0 = sb0 / p.KC, sbl0 = sb0 - ch0 * p.KC;
    bool ok = true;
    for (int tile = (own || warp < R * p.nb) ? t0 : ntiles; tile < ntiles; tile += R) {
        float accA = 0.f, accB = 0.f;  // rows g, g + 8 of the tile
        int ch = ch0, sbl = sbl0;
        for (int sb = sb0; sb < p.nb; sb += NCW) {
            const uint32_t st = static_cast<uint32_t>(tile * p.nchunks + ch);
            const uint32_t q = __umulhi(st, p.stage_magic);  // st / stages
            const int s = static_cast<int>(st - q * static_cast<uint32_t>(p.stages));
            if (!mbar_wait_bounded(&full[s], q & 1u, DEV_TIMEOUT_FULL) || *abort_flag) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            const uint8_t* bA = ring + static_cast<size_t>(s) * p.stage_bytes + g * p.cs + sbl * BB;
            const uint8_t* bB = bA + 8 * p.cs;
            const uint8_t* xu = xt + static_cast<size_t>(4 * sb) * 256 + lane * (T == Q4_K ? 8 : 4);
            const float* xj = xsum + 16 * sb;
            if constexpr (T == Q4_K) {
                item_q4k(bA, bB, xu, xj, xe[sb], t, par, lo_mask, lw0, lw1, accA, accB);
            } else if (sbl & 1) {  // the chunk starts on a 16-byte boundary: odd blocks at 2 mod 4
                item_q6k<true>(bA, bB, xu, xj, xe[sb], t, par, lo_mask, lw0, lw1, accA, accB);
            } else {
                item_q6k<false>(bA, bB, xu, xj, xe[sb], t, par, lo_mask, lw0, lw1, accA, accB);
            }
            // the stage's slot is free once all its items are done; the item
            // that ends a short last chunk also accounts for the missing ones
            const int kc = min(p.KC, p.nb - ch * p.KC);
            __syncwarp();
            if (lane == 0) mbar_arrive_cnt(&empty[s], sbl == kc - 1 ? static_cast<uint32_t>(p.KC - kc + 1) : 1u);
            sbl += NCW;
            while (sbl >= p.KC) {
                sbl -= p.KC;
                ++ch;
            }
        }
        if (!ok) break;
        accA += __shfl_xor_sync(0xffffffffu, accA, 1);
        accA += __shfl_xor_sync(0xffffffffu, accA, 2);
        accB += __shfl_xor_sync(0xffffffffu, accB, 1);
        accB += __shfl_xor_sync(0xffffffffu, accB, 2);
        if (t == 0) {
            part[(tile * NCW + warp) * TR + g] = accA;
            part[(tile * NCW + warp) * TR + g + 8] = accB;
        }
    }
    // Every consumer warp reaches this one barrier exactly once (also after
    // a timeout), then the rows are summed over the warps in warp order.
    named_bar_sync(1, NCW * 32);
    if (!ok || *abort_flag) return;
    float rs = 1.f;
    if (p.act == ACT_RMSNORM) {
        float tq = 0.f;
        for (int w = 0; w < NCW; ++w) tq += s_sq[w];
        rs = 1.0f / sqrtf(tq / static_cast<float>(p.K) + p.eps);
    }
    for (int r = threadIdx.x; r < ntiles * TR; r += NCW * 32) {
        const int tile = r / TR;
        const int row = tile_row0(tile, r_begin, r_end) + (r % TR);
        if (row < r_begin + tile * TR || row >= r_end) continue;  // another tile's row, or past the range
        const float* pb = part + tile * NCW * TR + (r % TR);
        float y = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; ++w) y += pb[w * TR];
        p.Y[row] = y * rs;
    }
}

}  // namespace kq

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

using EncodeTiledKq = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledKq encode_kq() {
    static EncodeTiledKq fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledKq>(f);
    });
    return fn;
}

uint32_t align_up4(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// smem row stride >= bytes, a multiple of 16 with an odd number of 16-byte
// units, so the 8 rows of a fragment start in 8 distinct 16-byte bank groups
int padded_stride_kq(int bytes) {
    int s = static_cast<int>(align_up4(static_cast<uint32_t>(bytes), 16u));
    while (((s / 16) & 1) == 0) s += 16;
    return s;
}

struct KqPlan {
    kq::Params p;
    int grid;
    int ncw;  // consumer warps per CTA
    uint32_t smem;
};

// Shared-memory plan: limb table, scales, sums, per-warp row partials, then
// as many ring stages as the budget holds (two CTAs per SM when at least 3
// stages fit in half an SM).
template <int T>
bool plan_kq(const GemvLaunch& L, KqPlan& P) {
    using namespace kq;
    constexpr int BB = KQ<T>::BB;
    Params& p = P.p;
    p = Params{};
    p.W = static_cast<const uint8_t*>(L.W);
    p.X = L.X;
    p.Y = L.Y;
    p.N = L.N;
    p.K = L.K;
    p.nb = L.K / 256;
    p.row_bytes = p.nb * BB;
    p.early = L.early;
    p.act = L.act;
    p.R = L.R;
    p.normw = L.normw;
    p.eps = L.eps;
    p.sum_out = L.sum_out;
    const bool al = (reinterpret_cast<uintptr_t>(L.X) & 15u) == 0 &&
                    (L.R == nullptr || (reinterpret_cast<uintptr_t>(L.R) & 15u) == 0) &&
                    (L.normw == nullptr || (reinterpret_cast<uintptr_t>(L.normw) & 15u) == 0) &&
                    (L.sum_out == nullptr || (reinterpret_cast<uintptr_t>(L.sum_out) & 15u) == 0);
    p.x_vec = al ? 1 : 0;
    P.grid = std::max(1, std::min(L.num_sms, (L.N + 1) / 2));
    const int rows_cta = (L.N + P.grid - 1) / P.grid;
    const int tiles_cta = (rows_cta + TR - 1) / TR;
    const int units = L.K / 64;
    uint32_t off = static_cast<uint32_t>(2 * MAX_STAGES * 8 + 16);
    off = align_up4(off, 128);
    p.off_xt = off;
    off += static_cast<uint32_t>(units) * 256u;
    p.off_xe = off;
    off += static_cast<uint32_t>(p.nb) * 4u;
    off = align_up4(off, 16);
    p.off_xsum = off;
    off += static_cast<uint32_t>(p.nb) * 64u;  // 16 sub-block sums per super-block
    p.off_part = off;
    // CTAs per SM: automatic (two CTAs of 16 consumer warps), or forced
    // (SWQ_OPT_GEMV_CTAS_PER_SM: 1-2 with 16 warps, 3-4 with 8)
    const int ctas = L.ctas_per_sm > 0 ? std::min(L.ctas_per_sm, 4) : 0;
    P.ncw = ctas >= 3 ? 8 : 16;
    off += static_cast<uint32_t>(tiles_cta) * P.ncw * TR * 4u;
    off = align_up4(off, 128);
    p.off_ring = off;
    // chunks of at most 8 super-blocks (1152 or 1680 bytes of each of the 16
    // rows; the box's inner extent, the padded stride, stays under its limit
    // of 256 eight-byte elements, and a chunk starts on an 8-byte element)
    p.KC = std::min(8, p.nb);
    p.nchunks = (p.nb + p.KC - 1) / p.KC;
    p.cs = padded_stride_kq(p.KC * BB);
    p.stage_bytes = TR * p.cs;
    int need = tiles_cta * p.nchunks;
    const uint32_t cap = static_cast<uint32_t>(L.smem_per_block_optin) - 1024u;
    const uint32_t half = static_cast<uint32_t>(L.smem_per_sm) / 2u - 2048u;  // two CTAs per SM
    uint32_t budget = half;
    if (ctas > 0) {
        budget = std::min(cap, static_cast<uint32_t>(L.smem_per_sm) / static_cast<uint32_t>(ctas) - 1280u);
    } else if (off + 3u * p.stage_bytes > budget && off + static_cast<uint32_t>(need) * p.stage_bytes > budget) {
        // chunks of 4 super-blocks keep two CTAs per SM when that fits three
        // stages (a long activation table); else one CTA.  Only where 4
        // blocks are a multiple of 16 bytes (Q4_K, not Q6_K): a chunk's
        // first 8-byte element x must satisfy x * 8 = 0 mod 16 for the TMA.
        const int cs4 = padded_stride_kq(4 * BB);
        if (p.KC == 8 && (4 * BB) % 16 == 0 && off + 3u * static_cast<uint32_t>(TR * cs4) <= budget) {
            p.KC = 4;
            p.nchunks = (p.nb + 3) / 4;
            p.cs = cs4;
            p.stage_bytes = TR * p.cs;
            need = tiles_cta * p.nchunks;
        } else {
            budget = cap;
        }
    }
    // TMA: every chunk starts on a 16-byte boundary of its row
    if ((p.KC * BB) % 16 != 0) return false;
    if (off + 2u * p.stage_bytes > budget) return false;
    p.stages = std::max(2, std::min<int>({static_cast<int>((budget - off) / p.stage_bytes), MAX_STAGES, need}));
    p.stage_magic = static_cast<uint32_t>((0x100000000ull + static_cast<uint64_t>(p.stages) - 1) /
                                          static_cast<uint64_t>(p.stages));
    P.smem = off + static_cast<uint32_t>(p.stages) * p.stage_bytes;
    return true;
}

}  // namespace

template <int T>
static bool kq_supported_t(const GemvLaunch& L) {
    if (L.M != 1 || !L.xf || L.imma < 2) return false;
    if (L.K <= 0 || L.K % 256 != 0 || L.K > kq::KQ<T>::MAX_K) return false;
    if (L.act != ACT_NONE && L.act != ACT_RMSNORM && L.act != ACT_SWIGLU) return false;
    if (L.act == ACT_RMSNORM && L.normw == nullptr) return false;
    if ((reinterpret_cast<uintptr_t>(L.W) & 15u) != 0) return false;
    if ((L.K / 256) % kq::KQ<T>::ALIGN_NB != 0) return false;  // rows 16-byte aligned
    if (encode_kq() == nullptr) return false;
    KqPlan P;
    return plan_kq<T>(L, P);
}

bool gemv_kq_supported(const GemvLaunch& L) {
    switch (L.type) {
        case Q4_K: return kq_supported_t<Q4_K>(L);
        case Q6_K: return kq_supported_t<Q6_K>(L);
        default: return false;
    }
}

template <int T>
static cudaError_t kq_launch_t(const GemvLaunch& L, cudaStream_t stream) {
    KqPlan P;
    if (!plan_kq<T>(L, P)) return cudaErrorInvalidConfiguration;
    const kq::Params& p = P.p;
    CUtensorMap tmap;
    std::memset(&tmap, 0, sizeof(tmap));
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.row_bytes / 8), static_cast<cuuint64_t>(L.N)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.row_bytes)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(p.cs / 8), static_cast<cuuint32_t>(kq::TR)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = encode_kq()(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(L.W), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    auto kern = P.ncw == 16 ? kq::gemv_kq_kernel<T, 16> : kq::gemv_kq_kernel<T, 8>;
    static thread_local int set_dev[2] = {-1, -1};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int ki = P.ncw == 16 ? 0 : 1;
    if (dev != set_dev[ki]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 L.smem_per_block_optin - 1024);
        if (e != cudaSuccess) return e;
        set_dev[ki] = dev;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(P.grid);
    cfg.blockDim = dim3((P.ncw + 1) * 32);
    cfg.dynamicSmemBytes = P.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, tmap);
}

cudaError_t gemv_kq_launch(const GemvLaunch& L, cudaStream_t s) {
    switch (L.type) {
        case Q4_K: return kq_launch_t<Q4_K>(L, s);
        case Q6_K: return kq_launch_t<Q6_K>(L, s);
        default: return cudaErrorInvalidValue;
    }
}

SWQ_DEFINE_STATUS_FETCH(gemv_kq)

}  // namespace swq
