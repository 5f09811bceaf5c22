// gemv_imma.cu -- single-row GEMV y = W . x for Q4_K and Q6_K with exact
// integer sub-block dot products on the tensor cores (sm_100a).
//
// Replaces cpu_matmul_transposed_q4_k / _q6_k (src/tensor.h:769-856) for the
// decode projections.  The reference accumulates (d*sc*q - dmin*m) * x in
// fp32, one rounding per product and per add.  Here every quant value is an
// exact small integer and x is held as a 30-bit fixed-point number per part
// (a 16- or 32-element sub-block sharing one weight scale): x = X * 2^(E-30)
// with E the part's largest binary exponent, X split into four signed 8-bit
// limbs.  One mma.sync m16n8k32 (u8 x s8 -> s32) multiplies 16 weight rows by
// the four limbs of 32 activations; the int32 sums are exact.  Per part the
// epilogue forms S = sum q * x in fp32 from the limb sums (two limbs at a
// time, exact below 2^24), and adds wd * S - (wd * z + wm) * sum(x) -- the
// same expression as the other kernels, with the product sums exact instead
// of rounded.  Measured error against a float64 evaluation is that of fp32
// accumulation (~1e-7 relative).
//
// Why the tensor cores on a memory-bound kernel: the CUDA-core form spends
// about three instructions per weight (byte -> float, the multiply-add, the
// zero point); here a masked word of four quant bytes is already a valid int8
// A fragment and one MMA does 4096 multiply-adds.  Measured on B200 against
// the fp32 CUDA-core kernel (dependent launches, rotating weights): faster
// for Q6_K (4096 x 14336: 20.6 vs 22.4 us; 128256 x 4096: 121 vs 169 us),
// slower for Q4_K (the per-sub-block epilogue, ~5 instructions per weight
// row and part, dominates at 4.5 bits per weight), so the default routes Q6_K
// here and Q4_K to the CUDA-core kernel (SWQ_OPT_GEMV_INT_MMA).
//
// Structure: a persistent CTA per SM owns a contiguous row range, processed
// as 16-row tiles (the MMA M).  One producer warp moves each tile's rows, a
// K-chunk at a time, into a shared-memory ring with per-row TMA bulk copies
// (the row stride in shared memory is padded so that the eight rows of a
// fragment fall on distinct banks); weights are requested before
// griddepcontrol.wait (they are immutable inputs).  The consumer warps first
// turn x into limb fragments (after the wait), then split each stage's
// 64-element groups among themselves; per tile, the warps' row partials are
// summed in warp order (deterministic).  Every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "formats.cuh"
#include "gemv.h"
#include "swq_device.cuh"

namespace swq {
namespace imma {

constexpr int NCW = 16;                   // consumer warps
constexpr int THREADS = (NCW + 1) * 32;   // + one producer warp
constexpr int TR = 16;                    // rows per tile (the MMA's M)
constexpr int MAX_K = 16384;              // x fragments: K / 64 * 256 bytes of shared memory

// Per-format view for this kernel.  A 64-element unit of a block gives eight
// words (four quant bytes each) to each of two MMAs of K = 32.  Lane t of a
// fragment owns words t and 4 + t of each MMA.
//   P16: parts of 16 elements (two per MMA: columns 0..3 and 4..7 of the MMA's
//        output take the limbs of the even and odd part); else parts of 32
//        (MMA 0 -> columns 0..3, MMA 1 -> columns 4..7, one accumulator).
template <int T>
struct Im;

template <>
struct Im<Q4_K> {
    using F = Fmt<Q4_K>;
    static constexpr bool P16 = false;
    // words t, 4 + t of MMA 0 (low nibbles: part 0) and of MMA 1 (high
    // nibbles in place, x16: part 1)
    __device__ static void words(const uint8_t* blk, int c, int t, uint32_t (&a)[4]) {
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk + 16 + 32 * c + 4 * t);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(blk + 32 + 32 * c + 4 * t);
        a[0] = w0 & 0x0F0F0F0Fu;
        a[1] = w1 & 0x0F0F0F0Fu;
        a[2] = w0 & 0xF0F0F0F0u;
        a[3] = w1 & 0xF0F0F0F0u;
    }
    // weight scale wd and the constant term's factor k of part p (of 2):
    // contribution = wd * S - k * sum(x).  Sub-block j = 2c + p through
    // get_scale_min_k4 (src/tensor.h:218-227); c is the same for a whole warp.
    __device__ static void part(const uint8_t* blk, int c, int p, float& wd, float& k) {
        const uint4 hd = *reinterpret_cast<const uint4*>(blk);
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hd.x));
        uint32_t SC, MN;
        if (c < 2) {
            SC = hd.y & 0x3F3F3F3Fu;
            MN = hd.z & 0x3F3F3F3Fu;
        } else {
            SC = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
            MN = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        }
        const uint32_t sel = 0x7650u + ((2 * c + p) & 3);
        const float sc = __uint_as_float(__byte_perm(SC, 0x4B000000u, sel)) - 8388608.0f;
        const float m = __uint_as_float(__byte_perm(MN, 0x4B000000u, sel)) - 8388608.0f;
        wd = dm.x * sc * (p ? 0.0625f : 1.0f);
        k = dm.y * m;
    }
};

template <>
struct Im<Q6_K> {
    using F = Fmt<Q6_K>;
    static constexpr bool P16 = true;
    // unit c = (half n, h): parts = planes 0..3 (words 4p .. 4p + 3); MMA 0
    // takes planes 0 (columns 0..3) and 1 (4..7), MMA 1 planes 2 and 3.
    __device__ static void words(const uint8_t* blk, int c, int t, uint32_t (&a)[4]) {
        const int n = c >> 1, h = c & 1;
        const uint8_t* ql = blk + 64 * n + 16 * h + 4 * t;
        const uint32_t A = static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(ql)[0]) |
                           (static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(ql)[1]) << 16);
        const uint32_t B = static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(ql + 32)[0]) |
                           (static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(ql + 32)[1]) << 16);
        const uint8_t* qh = blk + 128 + 32 * n + 16 * h + 4 * t;
        const uint32_t H = static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(qh)[0]) |
                           (static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(qh)[1]) << 16);
        a[0] = (A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);         // plane 0
        a[1] = (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);         // plane 1
        a[2] = ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);         // plane 2
        a[3] = ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);  // plane 3
    }
    __device__ static void part(const uint8_t* blk, int c, int p, float& wd, float& k) {
        const int n = c >> 1, h = c & 1;
        const float d = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
        const int s = static_cast<int8_t>(blk[192 + 8 * n + h + 2 * p]);
        wd = d * static_cast<float>(s);
        k = wd * 32.0f;  // zero point 32
    }
};

struct Params {
    const uint8_t* W;
    const float* X;
    float* Y;
    int N, K, nb, row_bytes;
    int KC, nchunks;  // blocks per chunk, chunks per row
    int cs;           // shared-memory bytes of one row of a chunk (KC * BB, padded)
    int stage_bytes;  // TR * cs
    int stages;
    int early;
    int refcpu;
    uint32_t off_xf, off_xs, off_part, off_ring;
};

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One stage: a box of TR rows x (cs / 8) 8-byte elements of the weight matrix
// (tensor map over [N rows][row_bytes / 8]); rows and bytes past the matrix
// read as zeros.  The box's inner size is the padded row stride, so the rows
// land at that stride in shared memory.  Into this CTA only.
__device__ __forceinline__ void tma_box(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                        uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// First row of tile `tile` of the CTA's range [r_begin, r_end): a last tile
// that would run past r_end starts lower (on rows the previous tile just
// read) when the range holds a whole tile, so no tile reads another CTA's rows.
__device__ __forceinline__ int tile_row0(int tile, int r_begin, int r_end) {
    const int r0 = r_begin + tile * TR;
    return (r0 + TR > r_end && r_end - TR >= r_begin) ? r_end - TR : r0;
}

// Signed 8-bit limb of v at byte position (v = sum_l limb_l * 256^l with
// limbs in -128..127): returns the limb and leaves (v - limb) / 256 in v.
__device__ __forceinline__ uint32_t take_limb(int& v) {
    const int l = static_cast<int>(static_cast<int8_t>(v & 0xFF));
    v = (v - l) >> 8;
    return static_cast<uint32_t>(l) & 0xFFu;
}

// x -> fixed-point limbs in the B-fragment layout, plus per part the fixed
// point's scale 2^(E-30) and sum(x).  Item = 4 consecutive elements of one part
// of one unit (PE/4 items per part, consecutive threads).
//   xf: per (unit u, MMA i) 32 words.  P16: words [0,16) hold b0 of lanes
//       g = l (limb l) for the even part, words [16,32) b1 of lanes g = 4 + l
//       for the odd part, index (l * 4 + t).  Else: 16 lanes x 2 words, index
//       (l * 4 + t) * 2 + reg, columns g = l (MMA 0) or 4 + l (MMA 1).
//   xs: per (unit, part) float2 (scale, sum), 4 parts per unit.
template <int T>
__device__ __forceinline__ void prep_x(const Params& p, uint32_t* xf, float2* xs, int tid, int nthreads) {
    using F = Fmt<T>;
    constexpr int PE = F::PE, GL = PE / 4, WPP = F::UE / 4 / F::PARTS;
    const int units = p.K / 64;
    const int items = units * F::PARTS * GL;
    const bool vec = (reinterpret_cast<uintptr_t>(p.X) & 15u) == 0;
    // two items per thread per pass, both loads issued before any arithmetic
    for (int base = 0; base < items; base += 2 * nthreads) {
        float v[2][4];
        int uu[2], pp[2], jj[2];
        bool act[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int it = base + h * nthreads + tid;
            act[h] = it < items;
            jj[h] = it % GL;
            const int up = it / GL;
            pp[h] = up % F::PARTS;
            uu[h] = act[h] ? up / F::PARTS : 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[h][i] = 0.f;
            if (act[h]) {
                const int e = (uu[h] / F::UPB) * F::QK + F::part_elem0(uu[h] % F::UPB, pp[h], p.refcpu != 0) + 4 * jj[h];
                if (vec) {
                    const float4 a = __ldg(reinterpret_cast<const float4*>(p.X + e));
                    v[h][0] = a.x; v[h][1] = a.y; v[h][2] = a.z; v[h][3] = a.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) v[h][i] = __ldg(p.X + e + i);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(fmaxf(fabsf(v[h][0]), fabsf(v[h][1])), fmaxf(fabsf(v[h][2]), fabsf(v[h][3])));
            float sum = (v[h][0] + v[h][1]) + (v[h][2] + v[h][3]);
#pragma unroll
            for (int o = 1; o < GL; o <<= 1) {
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                sum += __shfl_xor_sync(0xffffffffu, sum, o);
            }
            // E: mx < 2^E (normal mx); X = x * 2^(30-E) lies in (-2^30, 2^30).
            // E is kept >= -96 so that both scales stay normal floats (a part
            // below 2^-97 keeps fewer bits, far under fp32's resolution of any
            // sum it joins).  Zero and subnormal-only parts contribute 0; a
            // non-finite part propagates through sum(x).
            const int ebits = (__float_as_int(mx) >> 23) & 0xFF;
            const bool normal = ebits > 0 && ebits < 255;
            const int E = normal ? max(ebits - 126, -96) : 0;
            const float up_s = normal ? __int_as_float((127 + 30 - E) << 23) : 0.f;  // 2^(30-E)
            const float down_s = normal ? __int_as_float((127 + E - 30) << 23) : 0.f;
            if (act[h]) {
                uint32_t lw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    int q = __float2int_rn(v[h][i] * up_s);
#pragma unroll
                    for (int l = 0; l < 3; ++l) lw[l] |= take_limb(q) << (8 * i);
                    lw[3] |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * i);
                }
                const int wd = pp[h] * WPP + jj[h];  // word of the unit
                const int mi = wd >> 3, t = wd & 3, reg = (wd >> 2) & 1;
                uint32_t* dst = xf + (uu[h] * 2 + mi) * 32;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    if (Im<T>::P16) dst[(reg ? 16 : 0) + l * 4 + t] = lw[l];
                    else dst[(l * 4 + t) * 2 + reg] = lw[l];
                }
                if (jj[h] == 0) xs[uu[h] * 4 + pp[h]] = make_float2(down_s, sum);
            }
        }
    }
}

// Group gi of a stage (unit c of block bl of the chunk): A words of the tile
// rows g (rA) and g + 8 (rB), B fragments of the unit's x limbs, two MMAs into
// separate accumulators d[0], d[1] (their output columns are disjoint: MMA 0
// writes columns 0..3 for parts of 32 and columns 0..7 for parts of 16).
template <int T>
__device__ __forceinline__ void mma_group(const uint8_t* rA, const uint8_t* rB, const uint32_t* xf, int kb0, int gi,
                                          int g, int t, int (&d)[2][4]) {
    using F = Fmt<T>;
    constexpr int UPB = F::UPB, BB = F::BB;
    const int bl = gi / UPB, c = gi - bl * UPB;
    const int u = kb0 * UPB + gi;
    uint32_t aA[4], aB[4];
    Im<T>::words(rA + bl * BB, c, t, aA);
    Im<T>::words(rB + bl * BB, c, t, aB);
    const uint32_t* f0 = xf + (u * 2) * 32;
    const uint32_t* f1 = f0 + 32;
    const int l = g & 3;
    uint32_t b00, b01, b10, b11;
    if (Im<T>::P16) {
        const uint32_t even0 = f0[l * 4 + t], odd0 = f0[16 + l * 4 + t];
        const uint32_t even1 = f1[l * 4 + t], odd1 = f1[16 + l * 4 + t];
        b00 = g < 4 ? even0 : 0u;
        b01 = g < 4 ? 0u : odd0;
        b10 = g < 4 ? even1 : 0u;
        b11 = g < 4 ? 0u : odd1;
    } else {
        const uint2 w0 = *reinterpret_cast<const uint2*>(f0 + (l * 4 + t) * 2);
        const uint2 w1 = *reinterpret_cast<const uint2*>(f1 + (l * 4 + t) * 2);
        b00 = g < 4 ? w0.x : 0u;
        b01 = g < 4 ? w0.y : 0u;
        b10 = g < 4 ? 0u : w1.x;
        b11 = g < 4 ? 0u : w1.y;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) d[0][i] = d[1][i] = 0;
    mma_u8s8(d[0], aA[0], aB[0], aA[1], aB[1], b00, b01);
    mma_u8s8(d[1], aA[2], aB[2], aA[3], aB[3], b10, b11);
}

// This lane's columns 2t, 2t+1 are the limbs (2 odd, 2 odd + 1) of part `hi`
// (parts of 32: columns 4..7 of MMA 1 are part 1) and, for parts of 16, of
// part 2 + hi in MMA 1.  Rows g (acc0) and g + 8 (acc1).  Even lanes add the
// constant term once.
template <int T>
__device__ __forceinline__ void epilogue(const uint8_t* rA, const uint8_t* rB, const float2* xs, int kb0, int gi,
                                         bool hi, bool odd, float pair_w, const int (&d)[2][4], float& acc0,
                                         float& acc1) {
    using F = Fmt<T>;
    constexpr int UPB = F::UPB, BB = F::BB;
    const int bl = gi / UPB, c = gi - bl * UPB;
    const int u = kb0 * UPB + gi;
    const uint8_t* bA = rA + bl * BB;
    const uint8_t* bB = rB + bl * BB;
    constexpr int NP = Im<T>::P16 ? 2 : 1;
#pragma unroll
    for (int q = 0; q < NP; ++q) {
        const int pt = Im<T>::P16 ? 2 * q + hi : hi;
        int v0, v1, v2, v3;
        if (Im<T>::P16) {
            v0 = d[q][0]; v1 = d[q][1]; v2 = d[q][2]; v3 = d[q][3];
        } else {  // disjoint columns: the sum is this lane's part
            v0 = d[0][0] + d[1][0]; v1 = d[0][1] + d[1][1]; v2 = d[0][2] + d[1][2]; v3 = d[0][3] + d[1][3];
        }
        const float2 sx = xs[u * 4 + pt];
        float wdA, kA, wdB, kB;
        Im<T>::part(bA, c, pt, wdA, kA);
        Im<T>::part(bB, c, pt, wdB, kB);
        float tA = (wdA * sx.x * pair_w) * static_cast<float>(v0 + 256 * v1);
        float tB = (wdB * sx.x * pair_w) * static_cast<float>(v2 + 256 * v3);
        if (!odd) {
            tA = fmaf(-kA, sx.y, tA);
            tB = fmaf(-kB, sx.y, tB);
        }
        acc0 += tA;
        acc1 += tB;
    }
}

template <int T>
__global__ void __launch_bounds__(THREADS, 2) gemv_imma_kernel(const Params p, const __grid_constant__ CUtensorMap tmap) {
    using F = Fmt<T>;
    constexpr int BB = F::BB, UPB = F::UPB;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + p.stages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + p.stages);
    uint32_t* xf = reinterpret_cast<uint32_t*>(smem + p.off_xf);
    float2* xs = reinterpret_cast<float2*>(smem + p.off_xs);
    float* part = reinterpret_cast<float*>(smem + p.off_part);  // [tile][NCW][TR]
    uint8_t* ring = smem + p.off_ring;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int rlo = p.N / G, rex = p.N % G;
    const int r_begin = b * rlo + min(b, rex);
    const int r_end = r_begin + rlo + (b < rex ? 1 : 0);
    const int ntiles = (r_end - r_begin + TR - 1) / TR;
    const int nstage = ntiles * p.nchunks;

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
    prep_x<T>(p, xf, xs, threadIdx.x, NCW * 32);
    named_bar_sync(1, NCW * 32);

    const int g = lane >> 2, t = lane & 3;
    const bool odd = (t & 1) != 0, hi = t >= 2;
    const float pair_w = odd ? 65536.0f : 1.0f;
    float acc0 = 0.f, acc1 = 0.f;  // rows g and g + 8 of the tile
    bool ok = true;
    for (int st = 0; st < nstage; ++st) {
        const int s = st % p.stages;
        const uint32_t phase = (st / p.stages) & 1;
        if (!mbar_wait_bounded(&full[s], phase, DEV_TIMEOUT_FULL) || *abort_flag) {
            *abort_flag = 1;
            ok = false;
            break;
        }
        const int tile = st / p.nchunks, ch = st % p.nchunks;
        const int kb0 = ch * p.KC, kc = min(p.KC, p.nb - kb0);
        const uint8_t* stage = ring + static_cast<size_t>(s) * p.stage_bytes;
        const uint8_t* rA = stage + g * p.cs;
        const uint8_t* rB = stage + (g + 8) * p.cs;
        for (int gi = warp; gi < kc * UPB; gi += NCW) {
            int d[2][4];
            mma_group<T>(rA, rB, xf, kb0, gi, g, t, d);
            epilogue<T>(rA, rB, xs, kb0, gi, hi, odd, pair_w, d, acc0, acc1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (ch == p.nchunks - 1) {
            // tile done: this warp's partial of each row into its own slot
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            float* pp = part + (tile * NCW + warp) * TR;
            if (t == 0) {
                pp[g] = acc0;
                pp[g + 8] = acc1;
            }
            acc0 = acc1 = 0.f;
        }
    }
    // Every consumer warp reaches this one barrier exactly once (also after
    // a timeout), then the rows are summed over the warps in warp order.
    named_bar_sync(1, NCW * 32);
    if (!ok || *abort_flag) return;
    for (int r = threadIdx.x; r < ntiles * TR; r += NCW * 32) {
        const int tile = r / TR;
        const int row = tile_row0(tile, r_begin, r_end) + (r % TR);
        if (row < r_begin + tile * TR || row >= r_end) continue;  // another tile's row, or past the range
        const float* pb = part + tile * NCW * TR + (r % TR);
        float y = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; ++w) y += pb[w * TR];
        p.Y[row] = y;
    }
}

}  // namespace imma

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static inline uint32_t align_up_u(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

using EncodeTiledImma = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledImma encode_imma() {
    static EncodeTiledImma fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledImma>(f);
    });
    return fn;
}

bool gemv_imma_supported(const GemvLaunch& L) {
    if (L.M != 1 || L.act != ACT_NONE || !L.xf || L.imma <= 0) return false;
    if (L.type != Q6_K && !(L.type == Q4_K && L.imma >= 2)) return false;
    if (L.K <= 0 || L.K % 256 != 0 || L.K > imma::MAX_K) return false;
    if ((reinterpret_cast<uintptr_t>(L.W) & 15u) != 0) return false;
    const int bb = L.type == Q4_K ? 144 : 210;
    const int nb = L.K / 256;
    if ((nb * bb) % 16 != 0) return false;       // rows start 16-byte aligned
    if (L.type == Q6_K && nb % 8 != 0) return false;  // chunks of 8 blocks (1680 bytes)
    return encode_imma() != nullptr;
}

// smem row stride >= bytes, a multiple of 16 with an odd number of 16-byte
// units modulo 8, so the 8 rows of a fragment start in 8 distinct bank groups
static int padded_stride(int bytes) {
    int s = static_cast<int>(align_up_u(static_cast<uint32_t>(bytes), 16u));
    while (((s / 16) & 1) == 0) s += 16;
    return s;
}

template <int T>
static cudaError_t launch_imma_t(const GemvLaunch& L, cudaStream_t stream) {
    using F = Fmt<T>;
    imma::Params p{};
    p.W = static_cast<const uint8_t*>(L.W);
    p.X = L.X;
    p.Y = L.Y;
    p.N = L.N;
    p.K = L.K;
    p.nb = L.K / F::QK;
    p.row_bytes = p.nb * F::BB;
    p.early = L.early;
    p.refcpu = L.refcpu;
    const int units = L.K / 64;
    uint32_t off = static_cast<uint32_t>(2 * 16 * 8 + 16);  // full, empty (16 stages), abort flag
    off = align_up_u(off, 128);
    p.off_xf = off;
    off += static_cast<uint32_t>(units) * 256u;
    p.off_xs = off;
    off += static_cast<uint32_t>(units) * 32u;
    const int grid = std::max(1, std::min(L.num_sms, (L.N + 1) / 2));
    const int rows_cta = (L.N + grid - 1) / grid;
    const int tiles_cta = (rows_cta + imma::TR - 1) / imma::TR;
    p.off_part = off;
    off += static_cast<uint32_t>(tiles_cta) * imma::NCW * imma::TR * 4u;
    off = align_up_u(off, 128);
    p.off_ring = off;
    const uint32_t cap = static_cast<uint32_t>(L.smem_per_block_optin) - 1024u;
    const uint32_t half = static_cast<uint32_t>(L.smem_per_sm) / 2u - 2048u;  // two CTAs per SM
    // Chunks of 8 blocks (2 units per consumer warp per stage; Q6_K needs a
    // multiple of 8 for 16-byte aligned copies), and as many ring slots as the
    // budget holds (up to 16): several stages in flight per SM hide the DRAM
    // latency.  Two CTAs per SM when at least 3 slots fit beside the other.
    const int KC = std::min(8, p.nb);
    p.KC = KC;
    p.nchunks = (p.nb + KC - 1) / KC;
    p.cs = padded_stride(KC * F::BB);
    p.stage_bytes = imma::TR * p.cs;
    const int need = tiles_cta * p.nchunks;
    // one box per stage: TR rows x cs / 8 elements of 8 bytes over [N][row_bytes / 8]
    CUtensorMap tmap;
    std::memset(&tmap, 0, sizeof(tmap));
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.row_bytes / 8), static_cast<cuuint64_t>(L.N)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.row_bytes)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(p.cs / 8), static_cast<cuuint32_t>(imma::TR)};
        const cuuint32_t estr[2] = {1, 1};
        if (p.cs / 8 > 256) return cudaErrorInvalidConfiguration;
        CUresult r = encode_imma()(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(L.W), dims, strides,
                                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    uint32_t budget = half;
    if (off + 3u * p.stage_bytes > budget) budget = cap;
    if (off + 2u * p.stage_bytes > budget) return cudaErrorInvalidConfiguration;
    p.stages = std::max(2, std::min<int>({static_cast<int>((budget - off) / p.stage_bytes), 16, need}));
    const uint32_t smem = off + static_cast<uint32_t>(p.stages) * p.stage_bytes;
    auto kern = imma::gemv_imma_kernel<T>;
    static thread_local int set_dev = -1;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != set_dev) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(cap));
        if (e != cudaSuccess) return e;
        set_dev = dev;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(imma::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, tmap);
}

cudaError_t gemv_imma_launch(const GemvLaunch& L, cudaStream_t s) {
    switch (L.type) {
        case Q4_K: return launch_imma_t<Q4_K>(L, s);
        case Q6_K: return launch_imma_t<Q6_K>(L, s);
        default: return cudaErrorInvalidValue;
    }
}

SWQ_DEFINE_STATUS_FETCH(gemv_imma)

}  // namespace swq
