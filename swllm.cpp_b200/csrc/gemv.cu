// gemv.cu -- fused dequant + GEMV/small-M GEMM on GGUF blocks (sm_100a).
//
// Y[m][i] = sum_k X[m][k] * W[i][k] for m < M (M <= 8), i < N, W in GGUF
// blocks.  Replaces the per-format CPU routines cpu_matmul_transposed_*
// (src/tensor.h:570-1025) behind Compute::matmul_transposed_q
// (src/tensor.h:1212).
//
// Design (HBM-bound streaming):
//  * Persistent grid of one CTA per SM; CTA b owns a contiguous, balanced range
//    of rows.  Shared memory per CTA stays under half an SM so the CTAs of the
//    next kernel on the stream (programmatic dependent launch) fit beside it
//    and start streaming their weights while this one finishes.
//  * Last warp = producer: one lane moves raw blocks into shared-memory stages
//    with the TMA -- one 1-D bulk copy per stage of whole rows, or one 2-D
//    tensor-map copy per stage of row chunks (into this CTA only, L2 evict-first)
//    -- completing on per-stage mbarriers.  Weights are requested before
//    griddepcontrol.wait (they are immutable inputs).  When a CTA's rows fit
//    in shared memory every stage gets its own slot and all of them are in
//    flight at once.
//  * NCW consumer warps, one or two rows per warp per stage (two rows share
//    each activation load and run two dot-product chains side by side).  A
//    lane owns one unit (32 or 64 elements): it decodes the quant bits into
//    packed small integers and dots each part with the activation row, held
//    in shared memory as 16-bit fixed point (per-32-element scale), with dp2a.
//  * The activation prep runs once per CTA after griddepcontrol.wait into a
//    unit-chunk-major layout: for each group of 32 consecutive units, chunk j
//    of all 32 units is one contiguous 512-byte plane, so a lane's loads are
//    base + compile-time offsets and a warp's loads never conflict on banks.
//    Each (unit, part) also gets its activation scale and integer sum.
//  * Every wait is bounded; on timeout the kernel records it in the device
//    status word, drains its own copies and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <numeric>

#include "formats.cuh"
#include "gemv.h"
#include "swq_device.cuh"

namespace swq {

enum : int { MODE_PLAIN = 0, MODE_BULK_ROWS = 1, MODE_TMAP = 2 };

// 8 consecutive floats (two float4 loads when VEC), and the store of 8
__device__ __forceinline__ void load8(const float* p, float (&v)[8], bool vec) {
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
__device__ __forceinline__ void store8(float* p, const float (&v)[8], bool vec) {
    if (vec) {
        reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = v[i];
    }
}

struct GemvParams {
    const uint8_t* W;
    const float* X;
    float* Y;
    int M, N, K;
    int nb;           // blocks per row
    int row_bytes;    // nb * BB
    int KC;           // blocks per chunk
    int nchunks;      // chunks per row
    int row_stride;   // bytes between rows inside a stage
    int rg;           // rows per stage
    int stage_bytes;  // rg * row_stride, 16-aligned
    int stages;
    int mode;    // MODE_*
    int refcpu;  // Q2_K reference-CPU activation order
    int early;   // weight prefetch before griddepcontrol.wait
    int x_vec;   // X rows 16-byte aligned: float4 activation loads
    int xstride; // bytes per activation row in shared memory
    uint32_t off_xq, off_ring;  // smem offsets
    // activation prologue (ACT_*): the GEMV's input row m is
    //   RMSNORM: x = X[m] (+ R[m]), then x * normw (the 1/rms of x scales the
    //            outputs of row m); CTA 0 writes x to sum_out when given
    //   SWIGLU:  silu(X[m*ld + k]) * X[m*ld + K + k]
    int act;
    const float* R;
    const float* normw;
    float eps;
    float* sum_out;
    int ld;  // X row stride in elements (SWIGLU), else K
};

// dp2a with a signed 16-bit pair and four 8-bit values, unsigned or signed.
template <bool SIGNED>
__device__ __forceinline__ int dp2a_lo(int a, uint32_t b, int c) {
    int d;
    if (SIGNED) asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    else asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
template <bool SIGNED>
__device__ __forceinline__ int dp2a_hi(int a, uint32_t b, int c) {
    int d;
    if (SIGNED) asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    else asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 2-D tiled TMA load of a box of the weight bytes (tensor map over 8-byte
// elements: inner = row bytes / 8, outer = rows).  Into this CTA only.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Activation layout in shared memory, per activation row: units in groups of
// 32; a group holds CPU chunk planes (32 x 16 B each: 8 int16 values of one
// unit) then PARTS meta planes (32 x 8 B each: scale bits, integer sum).
template <int T>
struct XLay {
    using F = Fmt<T>;
    static constexpr int CPU = F::UE / 8;                         // chunks per unit
    static constexpr int CPP = F::PE / 8;                         // chunks per part
    static constexpr int GB = 32 * (F::UE * 2 + F::PARTS * 8);    // bytes per group
    static constexpr int META = 32 * 16 * CPU;                    // offset of the meta planes
    __host__ __device__ static int row_bytes(int K) { return ((K / F::UE + 31) / 32) * GB; }
    __device__ static uint32_t chunk_off(int u) { return (u >> 5) * GB + (u & 31) * 16; }
    __device__ static uint32_t meta_off(int u) { return (u >> 5) * GB + META + (u & 31) * 8; }
};

// Consumer warps per CTA for a padded activation-row count.
template <int MT>
struct Cfg {
    static constexpr int NCW = MT <= 2 ? 12 : 8;
    static constexpr int RPW = MT == 1 ? 2 : 1;  // rows per consumer warp per stage
    static constexpr int RGMAX = NCW * RPW;      // rows per stage at most
    static constexpr int THREADS = (NCW + 1) * 32;
};

// ---------------------------------------------------------------------------
// fp32 activations (the default): x stays fp32 as in the reference, every
// quant byte becomes an exact float, the products are exact in the FMA and only
// the fp32 accumulation rounds -- as in cpu_matmul_transposed_* (src/tensor.h:
// 570-1025), which rounds each product as well.
//
// Layout per activation row: units in groups of 32; a group holds NW chunk
// planes (32 lanes x 16 B: the 4 fp32 activations of one decoded word of each
// unit), then, for formats with a min (Q2_K, Q4_K, Q5_K), PARTS planes of the
// part sums sum(x) (32 x 4 B).  A lane's loads are base + compile-time offsets
// and a warp's never share a bank.
// ---------------------------------------------------------------------------
template <int T>
struct XLayF {
    using F = Fmt<T>;
    static constexpr int NW = F::UE / 4;                           // chunks (words) per unit
    static constexpr int WPP = NW / F::PARTS;                      // words per part
    static constexpr int MPL = F::MIN ? F::PARTS : 0;              // meta planes
    static constexpr int GB = 32 * (16 * NW + 4 * MPL);            // bytes per group
    static constexpr int META = 32 * 16 * NW;                      // offset of the meta planes
    __host__ __device__ static int row_bytes(int K) { return ((K / F::UE + 31) / 32) * GB; }
    __device__ static uint32_t chunk_off(int u) { return (u >> 5) * GB + (u & 31) * 16; }
    __device__ static uint32_t meta_off(int u) { return (u >> 5) * GB + META + (u & 31) * 4; }
};

// Quant byte b -> float (b - z), exact: the byte is placed in the low mantissa
// of 2^23 (one byte permute), then 2^23 + z is subtracted (one packed add for
// two elements).  Bytes 0, 1 of word w -> lo, bytes 2, 3 -> hi.
__device__ __forceinline__ void word_to_f2(uint32_t w, float2 bias, float2& lo, float2& hi) {
    lo = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650)),
                                __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7651))), bias);
    hi = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7652)),
                                __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7653))), bias);
}

// Zero point of part pt in the units of its bytes (signed bytes are read as
// byte ^ 0x80, i.e. value + 128).
template <int T>
__device__ __forceinline__ float2 part_bias(int pt) {
    using F = Fmt<T>;
    const float z = 8388608.0f + static_cast<float>(F::QSIGNED ? 128 : F::ioff(pt));
    return make_float2(-z, -z);
}

template <int T, int MT>
__device__ __forceinline__ void unit_dotf(const uint8_t* blk, int c, int u, const uint8_t* xs, int xstride,
                                          float (&acc)[MT]) {
    using F = Fmt<T>;
    using XL = XLayF<T>;
    constexpr int NW = XL::NW, WPP = XL::WPP;
    uint32_t q[NW];
    float wd[F::PARTS], wm[F::PARTS];
    F::decode(blk, c, q, wd, wm);
    const uint32_t co = XL::chunk_off(u);
#pragma unroll
    for (int pt = 0; pt < F::PARTS; ++pt) {
        const float2 bias = part_bias<T>(pt);
        float2 S[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) S[m] = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < WPP; ++i) {
            float2 lo, hi;
            word_to_f2(F::QSIGNED ? (q[pt * WPP + i] ^ 0x80808080u) : q[pt * WPP + i], bias, lo, hi);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + m * xstride + co + (pt * WPP + i) * 512);
                S[m] = __ffma2_rn(make_float2(xv.x, xv.y), lo, S[m]);
                S[m] = __ffma2_rn(make_float2(xv.z, xv.w), hi, S[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float t = wd[pt] * (S[m].x + S[m].y);
            if (F::MIN)
                t = fmaf(-wm[pt], *reinterpret_cast<const float*>(xs + m * xstride + XL::meta_off(u) + pt * 128), t);
            acc[m] += t;
        }
    }
}

// The same unit position in two rows, sharing every activation load.
template <int T, int MT>
__device__ __forceinline__ void unit_dotf2(const uint8_t* blkA, const uint8_t* blkB, int c, int u, const uint8_t* xs,
                                           int xstride, float (&accA)[MT], float (&accB)[MT]) {
    using F = Fmt<T>;
    using XL = XLayF<T>;
    constexpr int NW = XL::NW, WPP = XL::WPP;
    uint32_t qa[NW], qb[NW];
    float wda[F::PARTS], wma[F::PARTS], wdb[F::PARTS], wmb[F::PARTS];
    F::decode(blkA, c, qa, wda, wma);
    F::decode(blkB, c, qb, wdb, wmb);
    const uint32_t co = XL::chunk_off(u);
#pragma unroll
    for (int pt = 0; pt < F::PARTS; ++pt) {
        const float2 bias = part_bias<T>(pt);
        float2 SA[MT], SB[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) SA[m] = SB[m] = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < WPP; ++i) {
            float2 alo, ahi, blo, bhi;
            word_to_f2(F::QSIGNED ? (qa[pt * WPP + i] ^ 0x80808080u) : qa[pt * WPP + i], bias, alo, ahi);
            word_to_f2(F::QSIGNED ? (qb[pt * WPP + i] ^ 0x80808080u) : qb[pt * WPP + i], bias, blo, bhi);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + m * xstride + co + (pt * WPP + i) * 512);
                const float2 x01 = make_float2(xv.x, xv.y), x23 = make_float2(xv.z, xv.w);
                SA[m] = __ffma2_rn(x01, alo, SA[m]);
                SB[m] = __ffma2_rn(x01, blo, SB[m]);
                SA[m] = __ffma2_rn(x23, ahi, SA[m]);
                SB[m] = __ffma2_rn(x23, bhi, SB[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float ta = wda[pt] * (SA[m].x + SA[m].y);
            float tb = wdb[pt] * (SB[m].x + SB[m].y);
            if (F::MIN) {
                const float I = *reinterpret_cast<const float*>(xs + m * xstride + XL::meta_off(u) + pt * 128);
                ta = fmaf(-wma[pt], I, ta);
                tb = fmaf(-wmb[pt], I, tb);
            }
            accA[m] += ta;
            accB[m] += tb;
        }
    }
}

// 4 consecutive floats (one float4 load when VEC)
__device__ __forceinline__ void load4(const float* p, float (&v)[4], bool vec) {
    if (vec) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __ldg(p + i);
    }
}

// Activation rows -> the fp32 layout, with the prologue (RMSNORM: (x + r) * w,
// the squares of x + r summed per row into sqm; SWIGLU: silu(g) * u).  Item =
// 4 consecutive elements of one row = one chunk; PE/4 consecutive items (one
// part) sum their elements by shuffles for the meta plane.
template <int T, int MT>
__device__ __forceinline__ void prep_xf(const GemvParams& p, uint8_t* xq, int ctid, int nct, float (&sqm)[MT]) {
    using F = Fmt<T>;
    using XL = XLayF<T>;
    const bool refcpu = p.refcpu != 0;
    const bool rms = p.act == ACT_RMSNORM;
    const int ipr = p.K / 4;  // items per row
    const int items = MT * ipr;
    constexpr int GL = F::PE / 4;  // lanes of one part
    for (int base = 0; base < items; base += nct) {
        const int it = base + ctid;
        const bool act = it < items;
        const int mm = (MT == 1 || !act) ? 0 : it / ipr;
        const int kk = act ? (it - mm * ipr) * 4 : 0;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (act && mm < p.M) {
            const size_t xo = static_cast<size_t>(mm) * p.ld + kk;
            load4(p.X + xo, v, p.x_vec);
            if (p.act == ACT_SWIGLU) {
                float g[4];
                load4(p.X + xo + p.K, g, p.x_vec);
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = v[i] / (1.0f + expf(-v[i])) * g[i];
            } else if (rms) {
                const size_t ro = static_cast<size_t>(mm) * p.K + kk;
                if (p.R) {
                    float r[4];
                    load4(p.R + ro, r, p.x_vec);
#pragma unroll
                    for (int i = 0; i < 4; ++i) v[i] += r[i];
                }
                if (p.sum_out && blockIdx.x == 0) {
                    if (p.x_vec) *reinterpret_cast<float4*>(p.sum_out + ro) = make_float4(v[0], v[1], v[2], v[3]);
                    else for (int i = 0; i < 4; ++i) p.sum_out[ro + i] = v[i];
                }
                float sq = 0.f, w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) sq = fmaf(v[i], v[i], sq);
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m == mm) sqm[m] += sq;
                load4(p.normw + kk, w, p.x_vec);
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] *= w[i];
            }
        }
        float psum = 0.f;
        if (F::MIN) {
            psum = (v[0] + v[1]) + (v[2] + v[3]);
#pragma unroll
            for (int o = 1; o < GL; o <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        }
        if (act) {
            const int kb = kk / F::QK, kq = kk - kb * F::QK;
            int c, p0, j;
            const int np = F::item_dest(kq & ~7, refcpu, c, p0, j);
            const int wi = 2 * j + ((kq >> 2) & 1);  // word of the part
            const int u = kb * F::UPB + c;
            uint8_t* xrow = xq + static_cast<size_t>(mm) * p.xstride;
            const float4 v4 = make_float4(v[0], v[1], v[2], v[3]);
            for (int t = 0; t < np; ++t) {
                *reinterpret_cast<float4*>(xrow + XL::chunk_off(u) + ((p0 + t) * XL::WPP + wi) * 512) = v4;
                if (F::MIN && wi % GL == 0)
                    *reinterpret_cast<float*>(xrow + XL::meta_off(u) + (p0 + t) * 128) = psum;
            }
        }
    }
}

// One unit of one row: decode the quant bits, dot every part with every
// activation row, add into acc.
template <int T, int MT>
__device__ __forceinline__ void unit_dot(const uint8_t* blk, int c, int u, const uint8_t* xq, int xstride,
                                         float (&acc)[MT]) {
    using F = Fmt<T>;
    using XL = XLay<T>;
    constexpr int NW = F::UE / 4, WPP = NW / F::PARTS;
    uint32_t q[NW];
    float wd[F::PARTS], wm[F::PARTS];
    F::decode(blk, c, q, wd, wm);
    const uint32_t co = XL::chunk_off(u), mo = XL::meta_off(u);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const uint8_t* xg = xq + static_cast<size_t>(m) * xstride + co;
        const uint8_t* xm = xq + static_cast<size_t>(m) * xstride + mo;
#pragma unroll
        for (int pt = 0; pt < F::PARTS; ++pt) {
            const int2 mt = *reinterpret_cast<const int2*>(xm + pt * 256);
            int S0 = 0, S1 = 0;
#pragma unroll
            for (int j = 0; j < XL::CPP; ++j) {
                const uint4 v = lds_u128(xg + (pt * XL::CPP + j) * 512);
                const uint32_t w0 = q[pt * WPP + 2 * j], w1 = q[pt * WPP + 2 * j + 1];
                S0 = dp2a_lo<F::QSIGNED>(static_cast<int>(v.x), w0, S0);
                S1 = dp2a_hi<F::QSIGNED>(static_cast<int>(v.y), w0, S1);
                S0 = dp2a_lo<F::QSIGNED>(static_cast<int>(v.z), w1, S0);
                S1 = dp2a_hi<F::QSIGNED>(static_cast<int>(v.w), w1, S1);
            }
            float t = wd[pt] * static_cast<float>(S0 + S1 - F::ioff(pt) * mt.y);
            if (F::MIN) t = fmaf(-wm[pt], static_cast<float>(mt.y), t);
            acc[m] = fmaf(__int_as_float(mt.x), t, acc[m]);
        }
    }
}

// The same unit position in two rows: the activation loads are shared and
// the two dot-product chains run side by side.
template <int T, int MT>
__device__ __forceinline__ void unit_dot2(const uint8_t* blkA, const uint8_t* blkB, int c, int u,
                                          const uint8_t* xq, int xstride, float (&accA)[MT], float (&accB)[MT]) {
    using F = Fmt<T>;
    using XL = XLay<T>;
    constexpr int NW = F::UE / 4, WPP = NW / F::PARTS;
    uint32_t qa[NW], qb[NW];
    float wda[F::PARTS], wma[F::PARTS], wdb[F::PARTS], wmb[F::PARTS];
    F::decode(blkA, c, qa, wda, wma);
    F::decode(blkB, c, qb, wdb, wmb);
    const uint32_t co = XL::chunk_off(u), mo = XL::meta_off(u);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const uint8_t* xg = xq + static_cast<size_t>(m) * xstride + co;
        const uint8_t* xm = xq + static_cast<size_t>(m) * xstride + mo;
#pragma unroll
        for (int pt = 0; pt < F::PARTS; ++pt) {
            const int2 mt = *reinterpret_cast<const int2*>(xm + pt * 256);
            int A0 = 0, A1 = 0, B0 = 0, B1 = 0;
#pragma unroll
            for (int j = 0; j < XL::CPP; ++j) {
                const uint4 v = lds_u128(xg + (pt * XL::CPP + j) * 512);
                const uint32_t a0 = qa[pt * WPP + 2 * j], a1 = qa[pt * WPP + 2 * j + 1];
                const uint32_t b0 = qb[pt * WPP + 2 * j], b1 = qb[pt * WPP + 2 * j + 1];
                A0 = dp2a_lo<F::QSIGNED>(static_cast<int>(v.x), a0, A0);
                B0 = dp2a_lo<F::QSIGNED>(static_cast<int>(v.x), b0, B0);
                A1 = dp2a_hi<F::QSIGNED>(static_cast<int>(v.y), a0, A1);
                B1 = dp2a_hi<F::QSIGNED>(static_cast<int>(v.y), b0, B1);
                A0 = dp2a_lo<F::QSIGNED>(static_cast<int>(v.z), a1, A0);
                B0 = dp2a_lo<F::QSIGNED>(static_cast<int>(v.z), b1, B0);
                A1 = dp2a_hi<F::QSIGNED>(static_cast<int>(v.w), a1, A1);
                B1 = dp2a_hi<F::QSIGNED>(static_cast<int>(v.w), b1, B1);
            }
            const float xs = __int_as_float(mt.x);
            const int I = mt.y;
            float ta = wda[pt] * static_cast<float>(A0 + A1 - F::ioff(pt) * I);
            float tb = wdb[pt] * static_cast<float>(B0 + B1 - F::ioff(pt) * I);
            if (F::MIN) {
                ta = fmaf(-wma[pt], static_cast<float>(I), ta);
                tb = fmaf(-wmb[pt], static_cast<float>(I), tb);
            }
            accA[m] = fmaf(xs, ta, accA[m]);
            accB[m] = fmaf(xs, tb, accB[m]);
        }
    }
}

template <int MT>
__device__ __forceinline__ void row_store(float (&acc)[MT], int lane, float* Y, int M, int N, int row,
                                          const float* rscale) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        float v = acc[m];
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if (lane == 0 && m < M) Y[static_cast<size_t>(m) * N + row] = rscale ? v * rscale[m] : v;
        acc[m] = 0.f;
    }
}

// First W row of the tensor-map box of the row group starting at rg: rg, or
// r_end - RG when the group is short and the CTA has RG rows before r_end.
__device__ __forceinline__ int tmap_row0(int rg, int r_begin, int r_end, int RG) {
    return (rg + RG > r_end && r_end - RG >= r_begin) ? r_end - RG : rg;
}

template <int T, int MT, bool XF>
__global__ void __launch_bounds__(Cfg<MT>::THREADS, 2)
    gemv_kernel(const GemvParams p, const __grid_constant__ CUtensorMap tmap) {
    using F = Fmt<T>;
    using XL = XLay<T>;
    constexpr int NCW = Cfg<MT>::NCW;
    constexpr int UPB = F::UPB, QK = F::QK, BB = F::BB, PE = F::PE;

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + p.stages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + p.stages);
    uint8_t* xq = smem + p.off_xq;
    uint8_t* ring = smem + p.off_ring;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int RG = p.rg;

    const int G = gridDim.x, b = blockIdx.x;
    const int rlo = p.N / G, rex = p.N % G;
    const int r_begin = b * rlo + min(b, rex);
    const int r_end = r_begin + rlo + (b < rex ? 1 : 0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
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
        int it = 0;
        bool ok = true;
        for (int rg = r_begin; rg < r_end && ok; rg += RG) {
            const int rows = min(RG, r_end - rg);
            for (int ch = 0; ch < p.nchunks; ++ch, ++it) {
                const int s = it % p.stages;
                if (it >= p.stages) {
                    if (!mbar_wait_bounded(&empty[s], ((it / p.stages) - 1) & 1, DEV_TIMEOUT_EMPTY) ||
                        *abort_flag) {
                        ok = false;
                        *abort_flag = 1;
                        break;
                    }
                }
                const int kb0 = ch * p.KC;
                const int kc = min(p.KC, p.nb - kb0);
                const uint32_t bytes_row = static_cast<uint32_t>(kc * BB);
                uint8_t* dst = ring + static_cast<size_t>(s) * p.stage_bytes;
                if (p.mode == MODE_TMAP) {
                    if (lane == 0) {
                        // The box is always full: RG rows x KC blocks (rows past N
                        // read zeros).  A last group shorter than RG starts lower,
                        // on rows of this CTA's previous group (just read, so
                        // L2 hits) rather than past r_end on the next CTA's rows.
                        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(p.KC * BB * RG));
                        tma_load_2d(dst, &tmap, kb0 * BB / 8, tmap_row0(rg, r_begin, r_end, RG), &full[s], pol);
                    }
                } else if (p.mode == MODE_BULK_ROWS) {
                    if (lane == 0) {
                        const uint8_t* src = p.W + static_cast<size_t>(rg) * p.row_bytes;
                        mbar_arrive_expect_tx(&full[s], bytes_row * rows);
                        bulk_g2s(dst, src, bytes_row * rows, &full[s], pol);
                    }
                } else {
                    const uint8_t* src = p.W + static_cast<size_t>(rg) * p.row_bytes + static_cast<size_t>(kb0) * BB;
                    for (int r = 0; r < rows; ++r) {
                        const uint8_t* sr = src + static_cast<size_t>(r) * p.row_bytes;
                        uint8_t* dr = dst + r * p.row_stride;
                        for (uint32_t i = lane; i < bytes_row; i += 32) dr[i] = __ldg(sr + i);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[s]);
                }
            }
        }
        if (p.mode != MODE_PLAIN && lane == 0) {
            // Drain: no TMA copy of this CTA may still be writing shared memory.
            const int issued = it;
            for (int s = 0; s < p.stages && s < issued; ++s) {
                const int last = issued - 1 - ((issued - 1 - s) % p.stages);
                mbar_wait_bounded(&full[s], (last / p.stages) & 1, DEV_TIMEOUT_DRAIN);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    pdl_wait_primary();
    constexpr int NCT = NCW * 32;
    const int ctid = threadIdx.x;
    const bool refcpu = p.refcpu != 0;
    const bool rms = p.act == ACT_RMSNORM;
    __shared__ float s_sq[NCW][MT];  // RMSNORM: each warp's sum of squares of each input row
    float sqm[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sqm[m] = 0.f;

    // Activation prep.  fp32 (XF): item = 4 consecutive elements (prep_xf).
    // 16-bit fixed point: item = 8 consecutive elements of one row (one 16-byte
    // chunk of one unit part).  Four lanes hold one 32-element block (scale);
    // PE/8 lanes one part (integer sum).  Loads for two items per thread are
    // issued before any arithmetic.
    if constexpr (XF) {
        prep_xf<T, MT>(p, xq, ctid, NCT, sqm);
    } else {
        const int ipr = p.K / 8;  // items per row (multiple of 4)
        const int items = MT * ipr;
        for (int base = 0; base < items; base += 2 * NCT) {
            float v[2][8];
            int mm[2], kk[2];
            bool act[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int it = base + h * NCT + ctid;
                act[h] = it < items;
                mm[h] = (MT == 1 || !act[h]) ? 0 : it / ipr;
                kk[h] = act[h] ? (it - mm[h] * ipr) * 8 : 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) v[h][i] = 0.f;
                if (act[h] && mm[h] < p.M) {
                    const size_t xo = static_cast<size_t>(mm[h]) * p.ld + kk[h];
                    load8(p.X + xo, v[h], p.x_vec);
                    if (p.act == ACT_SWIGLU) {
                        float u[8];
                        load8(p.X + xo + p.K, u, p.x_vec);
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[h][i] = v[h][i] / (1.0f + expf(-v[h][i])) * u[i];
                    } else if (rms) {
                        const size_t ro = static_cast<size_t>(mm[h]) * p.K + kk[h];
                        if (p.R) {
                            float r[8];
                            load8(p.R + ro, r, p.x_vec);
#pragma unroll
                            for (int i = 0; i < 8; ++i) v[h][i] += r[i];
                        }
                        if (p.sum_out && blockIdx.x == 0) store8(p.sum_out + ro, v[h], p.x_vec);
                        float sq = 0.f, w[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) sq = fmaf(v[h][i], v[h][i], sq);
#pragma unroll
                        for (int m = 0; m < MT; ++m)
                            if (m == mm[h]) sqm[m] += sq;
                        load8(p.normw + kk[h], w, p.x_vec);
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[h][i] *= w[i];
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float a = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[h][i]));
                a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
                a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
                // |v| <= a, so |v * inv| <= 32767 (to within the approximate
                // reciprocal) and rounds into the int16 range.
                const bool live = a > 1e-30f;
                const float inv = live ? __fdividef(32767.0f, a) : 0.f;
                // |v * inv| <= 32767: adding 1.5 * 2^23 rounds to the nearest integer
                // in the low mantissa bits (exact, ties to even).
                int xi[8], sum = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    xi[i] = __float_as_int(fmaf(v[h][i], inv, 12582912.0f)) - 0x4B400000;
                    sum += xi[i];
                }
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                if (PE == 32) sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                if (act[h]) {
                    uint4 pk;
                    pk.x = __byte_perm(xi[0], xi[1], 0x5410);
                    pk.y = __byte_perm(xi[2], xi[3], 0x5410);
                    pk.z = __byte_perm(xi[4], xi[5], 0x5410);
                    pk.w = __byte_perm(xi[6], xi[7], 0x5410);
                    const float sc = live ? a * (1.0f / 32767.0f) : 0.f;
                    const int kb = kk[h] / QK, kq = kk[h] - kb * QK;
                    int c, p0, j;
                    const int np = F::item_dest(kq, refcpu, c, p0, j);
                    uint8_t* xrow = xq + static_cast<size_t>(mm[h]) * p.xstride;
                    const int u = kb * UPB + c;
                    for (int t = 0; t < np; ++t) {
                        *reinterpret_cast<uint4*>(xrow + XL::chunk_off(u) + ((p0 + t) * XL::CPP + j) * 512) = pk;
                        if (j == 0)
                            *reinterpret_cast<int2*>(xrow + XL::meta_off(u) + (p0 + t) * 256) =
                                make_int2(__float_as_int(sc), sum);
                    }
                }
            }
        }
    }
    if (rms) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float t = sqm[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            if ((ctid & 31) == 0) s_sq[ctid >> 5][m] = t;
        }
    }
    named_bar_sync(1, NCT);
    // RMSNORM: outputs of row m scale by 1 / sqrt(mean(x^2) + eps); the warps'
    // sums are added in warp order, so every CTA and every run agree.
    float rsv[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        float t = 0.f;
        if (rms)
            for (int w = 0; w < NCW; ++w) t += s_sq[w][m];
        rsv[m] = rms ? 1.0f / sqrtf(t / static_cast<float>(p.K) + p.eps) : 1.f;
    }
    const float* rsc = rms ? rsv : nullptr;

    float accA[MT], accB[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) accA[m] = accB[m] = 0.f;

    int s = 0;
    uint32_t phase = 0;
    bool ok = true;
    if (p.nchunks == 1) {
        // Whole rows per stage: warp w takes rows w, w + NCW, w + 2 NCW, ... of
        // the stage, two at a time, and stores each result right away.
        for (int rg = r_begin; rg < r_end && ok; rg += RG) {
            const int rows = min(RG, r_end - rg);
            if (!mbar_wait_bounded(&full[s], phase, DEV_TIMEOUT_FULL) || *abort_flag) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            const int nu = p.nb * UPB;
            const uint8_t* stage = ring + static_cast<size_t>(s) * p.stage_bytes;
            for (int r0 = warp; r0 < rows; r0 += 2 * NCW) {
                const uint8_t* rowA = stage + r0 * p.row_stride;
                if (r0 + NCW < rows) {
                    const uint8_t* rowB = rowA + NCW * p.row_stride;
                    for (int uu = lane; uu < nu; uu += 32) {
                        const int kbl = uu / UPB, c = uu - kbl * UPB;
                        if constexpr (XF) unit_dotf2<T, MT>(rowA + kbl * BB, rowB + kbl * BB, c, uu, xq, p.xstride, accA, accB);
                        else unit_dot2<T, MT>(rowA + kbl * BB, rowB + kbl * BB, c, uu, xq, p.xstride, accA, accB);
                    }
                    row_store<MT>(accA, lane, p.Y, p.M, p.N, rg + r0, rsc);
                    row_store<MT>(accB, lane, p.Y, p.M, p.N, rg + r0 + NCW, rsc);
                } else {
#pragma unroll 2
                    for (int uu = lane; uu < nu; uu += 32) {
                        const int kbl = uu / UPB, c = uu - kbl * UPB;
                        if constexpr (XF) unit_dotf<T, MT>(rowA + kbl * BB, c, uu, xq, p.xstride, accA);
                        else unit_dot<T, MT>(rowA + kbl * BB, c, uu, xq, p.xstride, accA);
                    }
                    row_store<MT>(accA, lane, p.Y, p.M, p.N, rg + r0, rsc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == p.stages) {
                s = 0;
                phase ^= 1u;
            }
        }
        return;
    }
    // Row chunks: each warp keeps its (at most two) rows across the chunks.
    for (int rg = r_begin; rg < r_end && ok; rg += RG) {
        const int rows = min(RG, r_end - rg);
        const bool hasA = warp < rows, hasB = warp + NCW < rows;
        for (int ch = 0; ch < p.nchunks; ++ch) {
            if (!mbar_wait_bounded(&full[s], phase, DEV_TIMEOUT_FULL) || *abort_flag) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            const int kb0 = ch * p.KC;
            const int kc = min(p.KC, p.nb - kb0);
            const int nu = kc * UPB;
            const int shift = p.mode == MODE_TMAP ? rg - tmap_row0(rg, r_begin, r_end, RG) : 0;
            const uint8_t* stage = ring + static_cast<size_t>(s) * p.stage_bytes + static_cast<size_t>(shift) * p.row_stride;
            const uint8_t* rowA = stage + warp * p.row_stride;
            const uint8_t* rowB = stage + (warp + NCW) * p.row_stride;
            if (hasB) {
                for (int uu = lane; uu < nu; uu += 32) {
                    const int kbl = uu / UPB, c = uu - kbl * UPB;
                    if constexpr (XF)
                        unit_dotf2<T, MT>(rowA + kbl * BB, rowB + kbl * BB, c, kb0 * UPB + uu, xq, p.xstride, accA, accB);
                    else
                        unit_dot2<T, MT>(rowA + kbl * BB, rowB + kbl * BB, c, kb0 * UPB + uu, xq, p.xstride, accA, accB);
                }
            } else if (hasA) {
#pragma unroll 2
                for (int uu = lane; uu < nu; uu += 32) {
                    const int kbl = uu / UPB, c = uu - kbl * UPB;
                    if constexpr (XF) unit_dotf<T, MT>(rowA + kbl * BB, c, kb0 * UPB + uu, xq, p.xstride, accA);
                    else unit_dot<T, MT>(rowA + kbl * BB, c, kb0 * UPB + uu, xq, p.xstride, accA);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == p.stages) {
                s = 0;
                phase ^= 1u;
            }
        }
        if (!ok) break;
        if (hasA) row_store<MT>(accA, lane, p.Y, p.M, p.N, rg + warp, rsc);
        if (hasB) row_store<MT>(accB, lane, p.Y, p.M, p.N, rg + warp + NCW, rsc);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <int T>
static uint32_t x_area_bytes_t(int MT, int K, bool xf) {
    return static_cast<uint32_t>(MT) *
           static_cast<uint32_t>(xf ? XLayF<T>::row_bytes(K) : XLay<T>::row_bytes(K));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

template <int T, int MT, bool XF>
static cudaError_t launch_t(const GemvLaunch& L, cudaStream_t stream) {
    using F = Fmt<T>;
    constexpr int RGMAX = Cfg<MT>::RGMAX;
    GemvParams p{};
    p.W = static_cast<const uint8_t*>(L.W);
    p.X = L.X;
    p.Y = L.Y;
    p.M = L.M;
    p.N = L.N;
    p.K = L.K;
    p.nb = L.K / F::QK;
    p.row_bytes = p.nb * F::BB;
    p.refcpu = L.refcpu;
    p.early = L.early;
    p.act = L.act;
    p.R = L.R;
    p.normw = L.normw;
    p.eps = L.eps;
    p.sum_out = L.sum_out;
    p.ld = L.ld > 0 ? L.ld : (L.act == ACT_SWIGLU ? 2 * L.K : L.K);
    // float4 activation loads: every row start 16-byte aligned (K % 32 == 0)
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    p.x_vec = (al(L.X) && al(L.R) && al(L.normw) && al(L.sum_out) && p.ld % 4 == 0) ? 1 : 0;
    p.xstride = XF ? XLayF<T>::row_bytes(L.K) : XLay<T>::row_bytes(L.K);

    const int per_sm = L.ctas_per_sm > 0 ? L.ctas_per_sm : 1;
    const int grid = std::max(1, std::min(L.num_sms * per_sm, L.N));
    const int rows_cta = (L.N + grid - 1) / grid;

    // Shared memory: barriers | activations | ring.
    uint32_t off = 2 * 16 * 8 + 16;
    off = align_up(off, 128);
    p.off_xq = off;
    off += x_area_bytes_t<T>(MT, L.K, XF);
    off = align_up(off, 128);
    p.off_ring = off;
    // (1 KB stays free for the kernel's static shared memory)
    const uint32_t smem_cap = static_cast<uint32_t>(L.smem_per_block_optin) - 1024;
    // Two CTAs per SM: this kernel's and the next one's.
    // Two CTAs per SM (this kernel's and the next one's) must fit beside each
    // other with their static shared memory and the 1 KB the SM reserves per CTA.
    constexpr uint32_t kStatic = 1024 + sizeof(float) * Cfg<MT>::NCW * MT;
    const uint32_t half_sm = static_cast<uint32_t>(L.smem_per_sm) / 2 - kStatic;
    uint32_t budget = (off + 32 * 1024 <= half_sm) ? half_sm : smem_cap;
    if (per_sm > 1) budget = std::min(smem_cap, static_cast<uint32_t>(L.smem_per_sm) / per_sm - kStatic);
    if (L.smem_kb > 0) budget = std::min(smem_cap, static_cast<uint32_t>(L.smem_kb) * 1024u);
    if (off >= budget) return cudaErrorInvalidConfiguration;
    const uint32_t ring_cap = budget - off;

    const bool aligned = (reinterpret_cast<uintptr_t>(L.W) & 15u) == 0 && (p.row_bytes % 16) == 0;
    const int al_blocks = 16 / std::gcd(F::BB, 16);
    const uint32_t kStageCap = L.stage_kb > 0 ? static_cast<uint32_t>(L.stage_kb) * 1024u : 96u * 1024u;
    bool chosen = false;
    CUtensorMap tmap;
    std::memset(&tmap, 0, sizeof(tmap));

    if (aligned) {
        // Whole rows, one contiguous bulk copy per stage; every stage its own
        // slot when the CTA's rows fit (then usually a single stage).
        constexpr int kRowsMax = 4 * Cfg<MT>::NCW;
        const int min_rows = std::min(rows_cta, Cfg<MT>::NCW);  // at least one row per warp
        for (int ngroups = (rows_cta + kRowsMax - 1) / kRowsMax; ngroups <= rows_cta; ++ngroups) {
            const int rg = (rows_cta + ngroups - 1) / ngroups;
            if (rg < min_rows) break;
            const uint32_t sb = static_cast<uint32_t>(rg) * p.row_bytes;
            if (sb > kStageCap) continue;
            int stages;
            if (ngroups <= 8 && static_cast<uint32_t>(ngroups) * sb <= ring_cap)
                stages = ngroups;  // resident: every row group in flight at once
            else if (2 * sb <= ring_cap)
                stages = std::min<int>(static_cast<int>(ring_cap / sb), 8);
            else
                continue;
            p.mode = MODE_BULK_ROWS;
            p.KC = p.nb;
            p.nchunks = 1;
            p.rg = rg;
            p.row_stride = p.row_bytes;
            p.stage_bytes = static_cast<int>(sb);
            p.stages = stages;
            chosen = true;
            break;
        }
        // Row chunks through a 2-D tensor map (box inner <= 256 x 8 bytes).
        EncodeTiledFn enc = chosen ? nullptr : encode_fn();
        if (!chosen && enc && (p.row_bytes % 8) == 0) {
            int KC = std::min(2048 / F::BB, std::max(al_blocks, static_cast<int>((ring_cap / 2) / (RGMAX * F::BB))));
            KC = KC / al_blocks * al_blocks;
            while (KC >= al_blocks && p.nb % KC != 0) KC -= al_blocks;
            // Fewer rows per stage when two stages of RGMAX rows do not fit (at
            // least one row per consumer warp).  Tensor copies land on
            // 128-byte aligned slots.
            int rgt = RGMAX;
            if (KC >= al_blocks) {
                const int fit_rows = static_cast<int>((ring_cap / 2 - 128) / (KC * F::BB));
                rgt = std::min(RGMAX, fit_rows);
            }
            const uint32_t sb = align_up(static_cast<uint32_t>(rgt) * KC * F::BB, 128);
            if (KC >= al_blocks && KC < p.nb && KC * F::BB <= 2048 && rgt >= Cfg<MT>::NCW &&
                ring_cap >= 2 * sb) {
                const int nchunks = p.nb / KC;
                const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.row_bytes / 8), static_cast<cuuint64_t>(L.N)};
                const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.row_bytes)};
                const cuuint32_t box[2] = {static_cast<cuuint32_t>(KC * F::BB / 8), static_cast<cuuint32_t>(rgt)};
                const cuuint32_t estr[2] = {1, 1};
                CUresult r = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(L.W), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
                if (r == CUDA_SUCCESS) {
                    p.mode = MODE_TMAP;
                    p.KC = KC;
                    p.nchunks = nchunks;
                    p.rg = rgt;
                    p.row_stride = KC * F::BB;
                    p.stage_bytes = static_cast<int>(sb);
                    const int need = ((rows_cta + rgt - 1) / rgt) * nchunks;
                    p.stages = std::max(2, std::min({static_cast<int>(ring_cap / sb), 8, need}));
                    chosen = true;
                }
            }
        }
    }
    if (!chosen) {
        // Plain loads by the producer warp: any alignment.
        int KC = static_cast<int>((28 * 1024) / (RGMAX * F::BB));
        KC = std::max(al_blocks, KC / al_blocks * al_blocks);
        if (KC >= p.nb) KC = p.nb;
        p.mode = MODE_PLAIN;
        p.KC = KC;
        p.nchunks = (p.nb + KC - 1) / KC;
        p.row_stride = static_cast<int>(align_up(static_cast<uint32_t>(KC * F::BB), 16));
        p.rg = std::min(RGMAX, static_cast<int>(ring_cap / 2 / p.row_stride));
        if (p.rg < 1) return cudaErrorInvalidConfiguration;
        p.stage_bytes = p.rg * p.row_stride;
        const int need = ((rows_cta + p.rg - 1) / p.rg) * p.nchunks;
        p.stages = std::max(2, std::min({static_cast<int>(ring_cap / p.stage_bytes), 8, need}));
    }
    const uint32_t smem = off + static_cast<uint32_t>(p.stages) * p.stage_bytes;
    auto kern = gemv_kernel<T, MT, XF>;
    // The attribute is per device: raise it once to the opt-in maximum.
    static thread_local int set_dev = -1;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != set_dev) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_cap));
        if (e != cudaSuccess) return e;
        set_dev = dev;
    }

    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(Cfg<MT>::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, tmap);
}

// fp32 activations (L.xf) for up to 4 rows when they fit the budget below;
// else (or with L.xf = 0) 16-bit fixed-point activations.
constexpr uint32_t kXfMaxBytes = 120u * 1024u;

template <int T>
static cudaError_t launch_fmt(const GemvLaunch& L, cudaStream_t s) {
    const int mt = L.M <= 1 ? 1 : L.M <= 2 ? 2 : L.M <= 4 ? 4 : 8;
    if (L.xf && mt <= 4 && x_area_bytes_t<T>(mt, L.K, true) <= kXfMaxBytes) {
        if (mt == 1) return launch_t<T, 1, true>(L, s);
        if (mt == 2) return launch_t<T, 2, true>(L, s);
        return launch_t<T, 4, true>(L, s);
    }
    if (mt == 1) return launch_t<T, 1, false>(L, s);
    if (mt == 2) return launch_t<T, 2, false>(L, s);
    if (mt == 4) return launch_t<T, 4, false>(L, s);
    return launch_t<T, 8, false>(L, s);
}

template <int T>
static size_t smem_x_bytes_fmt(int MT, int K, bool xf) {
    if (xf && MT <= 4 && x_area_bytes_t<T>(MT, K, true) <= kXfMaxBytes) return x_area_bytes_t<T>(MT, K, true);
    return x_area_bytes_t<T>(MT, K, false);
}

size_t gemv_smem_x_bytes(int type, int MT, int K, bool xf) {
    switch (type) {
        case Q4_0: return smem_x_bytes_fmt<Q4_0>(MT, K, xf);
        case Q8_0: return smem_x_bytes_fmt<Q8_0>(MT, K, xf);
        case Q2_K: return smem_x_bytes_fmt<Q2_K>(MT, K, xf);
        case Q3_K: return smem_x_bytes_fmt<Q3_K>(MT, K, xf);
        case Q4_K: return smem_x_bytes_fmt<Q4_K>(MT, K, xf);
        case Q5_K: return smem_x_bytes_fmt<Q5_K>(MT, K, xf);
        case Q6_K: return smem_x_bytes_fmt<Q6_K>(MT, K, xf);
        default: return 0;
    }
}

cudaError_t gemv_launch(const GemvLaunch& L, cudaStream_t s) {
    if (L.imma >= 2 && gemv_kq_supported(L)) return gemv_kq_launch(L, s);
    if (L.imma && gemv_imma_supported(L)) return gemv_imma_launch(L, s);
    switch (L.type) {
        case Q4_0: return launch_fmt<Q4_0>(L, s);
        case Q8_0: return launch_fmt<Q8_0>(L, s);
        case Q2_K: return launch_fmt<Q2_K>(L, s);
        case Q3_K: return launch_fmt<Q3_K>(L, s);
        case Q4_K: return launch_fmt<Q4_K>(L, s);
        case Q5_K: return launch_fmt<Q5_K>(L, s);
        case Q6_K: return launch_fmt<Q6_K>(L, s);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// Grouped GEMV (MoE decode): expert e multiplies its rows offsets[e] ..
// offsets[e+1]-1 of X (few per expert) by its own GGUF matrix wptrs[e].
// CTA (chunk, e) takes W rows [64 chunk, 64 chunk + 64) of expert e: an
// expert without rows costs one early exit, and no other expert's weights
// are read.  The expert's activation rows are converted MT at a time into the
// GEMV's shared-memory layout (16-bit fixed point per 32-element block), then
// each warp dots whole W rows read straight from global memory (a lane per
// unit, the same decoders and dp2a chains as gemv_kernel).  The unit decoders
// read 32-bit words, so every expert matrix must start on a 16-byte boundary:
// an expert that does not is skipped and recorded (DEV_BAD_ALIGN) for
// swq_check, never read misaligned.
// ---------------------------------------------------------------------------

static_assert(DEV_BAD_ALIGN == kStatusBadAlign, "status bit shared with the host");

struct GroupedGemvParams {
    const uint8_t* const* wptrs;
    const int* offsets;
    const float* X;
    float* Y;
    int n_experts, rows_total, N, K, nb, row_bytes, xstride, refcpu, x_vec, adaptive;
    const uint8_t* w_all;  // stacked experts: expert e at w_all + e * N * row_bytes (wptrs unused)
};

constexpr int GG_WARPS = 8;
constexpr int GG_ROWS = 64;  // W rows per CTA

// rows (<= MT) activation rows of length K at X (row stride K) -> the GEMV's
// shared-memory layout at xq; rows MT-rows .. MT-1 are zero.  Every thread of
// the CTA takes part (full-warp shuffles); nthreads is a multiple of 32.
template <int T, int MT>
__device__ void prep_x_rows(const float* X, int K, int rows, uint8_t* xq, int xstride, bool refcpu, bool vec,
                            int tid, int nthreads) {
    using F = Fmt<T>;
    using XL = XLay<T>;
    const int ipr = K / 8;  // items per row (multiple of 4: K % 32 == 0)
    const int items = MT * ipr;
    for (int base = 0; base < items; base += nthreads) {
        const int it = base + tid;
        const bool act = it < items;
        const int mm = act ? it / ipr : 0;
        const int kk = act ? (it - mm * ipr) * 8 : 0;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
        if (act && mm < rows) load8(X + static_cast<size_t>(mm) * K + kk, v, vec);
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[i]));
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
        const bool live = a > 1e-30f;
        const float inv = live ? __fdividef(32767.0f, a) : 0.f;
        int xi[8], sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            xi[i] = __float_as_int(fmaf(v[i], inv, 12582912.0f)) - 0x4B400000;
            sum += xi[i];
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if (F::PE == 32) sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (act) {
            uint4 pk;
            pk.x = __byte_perm(xi[0], xi[1], 0x5410);
            pk.y = __byte_perm(xi[2], xi[3], 0x5410);
            pk.z = __byte_perm(xi[4], xi[5], 0x5410);
            pk.w = __byte_perm(xi[6], xi[7], 0x5410);
            const float sc = live ? a * (1.0f / 32767.0f) : 0.f;
            const int kb = kk / F::QK, kq = kk - kb * F::QK;
            int c, p0, j;
            const int np = F::item_dest(kq, refcpu, c, p0, j);
            uint8_t* xrow = xq + static_cast<size_t>(mm) * xstride;
            const int u = kb * F::UPB + c;
            for (int t = 0; t < np; ++t) {
                *reinterpret_cast<uint4*>(xrow + XL::chunk_off(u) + ((p0 + t) * XL::CPP + j) * 512) = pk;
                if (j == 0)
                    *reinterpret_cast<int2*>(xrow + XL::meta_off(u) + (p0 + t) * 256) =
                        make_int2(__float_as_int(sc), sum);
            }
        }
    }
}

// One pass over `mrows` (<= MTP) activation rows of expert matrix W.
template <int T, int MTP>
__device__ __forceinline__ void grouped_pass(const GroupedGemvParams& p, const uint8_t* W, int m0, int mrows, int r0,
                                             int r1, uint8_t* xq) {
    using F = Fmt<T>;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nu = p.nb * F::UPB;
    prep_x_rows<T, MTP>(p.X + static_cast<size_t>(m0) * p.K, p.K, mrows, xq, p.xstride, p.refcpu != 0,
                        p.x_vec != 0, threadIdx.x, GG_WARPS * 32);
    __syncthreads();
    for (int row = r0 + warp; row < r1; row += GG_WARPS) {
        float acc[MTP];
#pragma unroll
        for (int m = 0; m < MTP; ++m) acc[m] = 0.f;
        const uint8_t* wr = W + static_cast<size_t>(row) * p.row_bytes;
        for (int uu = lane; uu < nu; uu += 32) {
            const int kbl = uu / F::UPB, c = uu - kbl * F::UPB;
            unit_dot<T, MTP>(wr + kbl * F::BB, c, uu, xq, p.xstride, acc);
        }
        row_store<MTP>(acc, lane, p.Y + static_cast<size_t>(m0) * p.N, mrows, p.N, row, nullptr);
    }
    __syncthreads();  // the next pass overwrites xq
}

// MT rows per pass; with p.adaptive (MT = 4) each expert's rows are taken in
// passes of 4, 2 or 1 by how many remain, so an expert with one row costs one
// row's work.  A row's result does not depend on the pass it is in.
template <int T, int MT>
__global__ void __launch_bounds__(GG_WARPS * 32) grouped_gemv_kernel(const GroupedGemvParams p) {
    extern __shared__ __align__(128) uint8_t xq[];
    pdl_wait_primary();  // X and the offsets may come from the previous kernels
    const int e = blockIdx.y;
    const int a = min(max(p.offsets[e], 0), p.rows_total);
    const int b = max(a, min(max(p.offsets[e + 1], 0), p.rows_total));
    const int r0 = blockIdx.x * GG_ROWS;
    if (b <= a || r0 >= p.N) return;
    const int r1 = min(p.N, r0 + GG_ROWS);
    const uint8_t* W = p.w_all ? p.w_all + static_cast<size_t>(e) * p.N * p.row_bytes : p.wptrs[e];
    if (reinterpret_cast<uintptr_t>(W) & 15u) {
        if (threadIdx.x == 0) atomicOr(&g_swq_dev_status, DEV_BAD_ALIGN);
        return;
    }
    for (int m0 = a; m0 < b;) {
        const int rem = b - m0;
        if (MT == 4 && p.adaptive && rem < 3) {
            if (rem == 2) {
                grouped_pass<T, 2>(p, W, m0, 2, r0, r1, xq);
                m0 += 2;
            } else {
                grouped_pass<T, 1>(p, W, m0, 1, r0, r1, xq);
                m0 += 1;
            }
        } else {
            grouped_pass<T, MT>(p, W, m0, min(MT, rem), r0, r1, xq);
            m0 += MT;
        }
    }
}

template <int T, int MT>
static cudaError_t launch_grouped_gemv_t(const GroupedGemvParams& p0, int smem_optin, cudaStream_t s) {
    GroupedGemvParams p = p0;
    p.xstride = XLay<T>::row_bytes(p.K);
    const size_t smem = static_cast<size_t>(MT) * p.xstride;  // 16-bit fixed-point activations
    if (smem > static_cast<size_t>(smem_optin)) return cudaErrorInvalidConfiguration;
    auto kern = grouped_gemv_kernel<T, MT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const dim3 grid(static_cast<unsigned>((p.N + GG_ROWS - 1) / GG_ROWS), static_cast<unsigned>(p.n_experts));
    kern<<<grid, GG_WARPS * 32, smem, s>>>(p);
    return cudaGetLastError();
}

template <int T>
static cudaError_t launch_grouped_gemv_fmt(const GroupedGemvParams& p, int mt, int smem_optin, cudaStream_t s) {
    if (mt <= 1) return launch_grouped_gemv_t<T, 1>(p, smem_optin, s);
    if (mt <= 2) return launch_grouped_gemv_t<T, 2>(p, smem_optin, s);
    return launch_grouped_gemv_t<T, 4>(p, smem_optin, s);
}

cudaError_t grouped_gemv_launch(int type, const void* const* wptrs, const int* offsets, const float* X, float* Y,
                                int n_experts, int rows_total, int N, int K, int refcpu, int smem_optin,
                                cudaStream_t s, bool adaptive, const void* w_all) {
    GroupedGemvParams p{};
    p.w_all = static_cast<const uint8_t*>(w_all);
    p.wptrs = reinterpret_cast<const uint8_t* const*>(wptrs);
    p.offsets = offsets;
    p.X = X;
    p.Y = Y;
    p.n_experts = n_experts;
    p.rows_total = rows_total;
    p.N = N;
    p.K = K;
    p.refcpu = refcpu;
    p.x_vec = (reinterpret_cast<uintptr_t>(X) & 15u) == 0 ? 1 : 0;
    // activation rows per pass: the mean rows per expert (1, 2 or 4), or 4
    // with the pass size chosen per expert on the device
    p.adaptive = adaptive ? 1 : 0;
    const int mt = adaptive ? 4 : (rows_total + n_experts - 1) / n_experts;
    switch (type) {
        case Q4_0: p.nb = K / Fmt<Q4_0>::QK; p.row_bytes = p.nb * Fmt<Q4_0>::BB; return launch_grouped_gemv_fmt<Q4_0>(p, mt, smem_optin, s);
        case Q8_0: p.nb = K / Fmt<Q8_0>::QK; p.row_bytes = p.nb * Fmt<Q8_0>::BB; return launch_grouped_gemv_fmt<Q8_0>(p, mt, smem_optin, s);
        case Q2_K: p.nb = K / Fmt<Q2_K>::QK; p.row_bytes = p.nb * Fmt<Q2_K>::BB; return launch_grouped_gemv_fmt<Q2_K>(p, mt, smem_optin, s);
        case Q3_K: p.nb = K / Fmt<Q3_K>::QK; p.row_bytes = p.nb * Fmt<Q3_K>::BB; return launch_grouped_gemv_fmt<Q3_K>(p, mt, smem_optin, s);
        case Q4_K: p.nb = K / Fmt<Q4_K>::QK; p.row_bytes = p.nb * Fmt<Q4_K>::BB; return launch_grouped_gemv_fmt<Q4_K>(p, mt, smem_optin, s);
        case Q5_K: p.nb = K / Fmt<Q5_K>::QK; p.row_bytes = p.nb * Fmt<Q5_K>::BB; return launch_grouped_gemv_fmt<Q5_K>(p, mt, smem_optin, s);
        case Q6_K: p.nb = K / Fmt<Q6_K>::QK; p.row_bytes = p.nb * Fmt<Q6_K>::BB; return launch_grouped_gemv_fmt<Q6_K>(p, mt, smem_optin, s);
        default: return cudaErrorInvalidValue;
    }
}

SWQ_DEFINE_STATUS_FETCH(gemv)

}  // namespace swq
