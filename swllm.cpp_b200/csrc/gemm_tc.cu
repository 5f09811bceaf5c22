// gemm_tc.cu -- tensor-core dequant-GEMM for prefill-sized M (sm_100a, tcgen05).
//
// Y[M x N] = X[M x K] . W[N x K]^T with W in GGUF blocks, X and Y fp32.  The
// reference has no batched quantized path (its prefill is one
// Compute::matmul_transposed_q per token, src/main.cpp:284-287 ->
// src/tensor.h:1212); this kernel is the M-rows-at-once form of it.
//
// Per CTA (persistent, one per SM), output tile = 128 W rows x BN tokens, K in
// steps of 64 (one 128-byte swizzle atom of fp16):
//   X producer   TMA of the fp16 activation tile (64 K x BN tokens, 128-byte
//                swizzled, K-major) per step.
//   MMA issuer   one lane: tcgen05.mma.cta_group::1.kind::f16 (M = 128,
//                N = BN, K = 16) into an fp32 TMEM accumulator.
//   W producer   the GGUF bytes of 256 K elements of the tile's 128 rows per
//                W stage (a 2-D tensor-map copy when rows are 16-byte aligned,
//                else one bulk copy per row).
//   16 dequantizer warps: four lanes per W row, eight rows per warp.
//                Quant bits become fp16 with the
//                0x6400 exponent trick (byte permute, then an exact fp16
//                subtract of the bias and one HFMA2/HMUL2 with the scales) and
//                are stored as the 128-byte-swizzled K-major A operand.
//   4 epilogue warps: tcgen05.ld of the accumulator (TMEM lane quadrant
//                = warp % 4), coalesced fp32 stores of Y.
// The order of the 64 K positions inside a step is whatever makes the
// dequantization cheapest for the format (tc_elem below); the activation
// conversion writes X in the same order, so the products are unchanged.
// Accumulators are double-buffered in TMEM (2 x BN columns) so the epilogue of
// one tile overlaps the MMAs of the next.  Every wait is bounded; on timeout the
// kernel records it, drains what it issued and frees its TMEM.  Every copy lands
// in the issuing CTA only.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>

#include "../../include/swq.h"
#include "formats.cuh"
#include "gemm_tc.h"
#include "swq_device.cuh"

namespace swq {

namespace tc {

constexpr int BM = 128;       // W rows per tile (MMA M)
constexpr int BK = 64;        // K elements per step (one 128-byte swizzle atom of fp16)
constexpr int KG = 256;       // K elements per W stage (4 steps)
constexpr int A_STAGE = BM * BK * 2;  // 16 KB
constexpr int NDQ = 16;       // dequantizer warps
constexpr int PASSES = BM / (8 * NDQ);  // W rows per dequantizer lane
// Warp roles (a warp runs on SM sub-partition warp % 4): warps 0-3 epilogue
// (TMEM lane quadrant = warp), 4 MMA issuer, 5 X producer, 6 W producer, 7 no
// role, 8-23 dequantizers -- four per sub-partition, so the dequantization,
// which sets the pace, uses the issue slots of all four.
constexpr int NWARPS = 8 + NDQ;
constexpr int THREADS = NWARPS * 32;  // 768
constexpr int WARP_MMA = 4, WARP_X = 5, WARP_W = 6, WARP_DQ0 = 8;
__host__ __device__ constexpr int dq_index(int w) { return w >= WARP_DQ0 && w < WARP_DQ0 + NDQ ? w - WARP_DQ0 : -1; }
__host__ __device__ constexpr bool is_epilogue(int w) { return w < 4; }
constexpr uint32_t FULL = 0xffffffffu;
constexpr int TC_MAX_SPLIT = 8;  // split-K parts per output tile at most

// Per-format constants of the W stages.
struct TcFmt {
    int qk, bb;   // elements and bytes per block
    int gbytes;   // bytes of one W stage of one row (256 elements)
    bool f2;      // element order family (tc_elem)
};
__host__ __device__ constexpr TcFmt tc_fmt(int t) {
    return t == Q4_0   ? TcFmt{32, 18, 144, false}
           : t == Q8_0 ? TcFmt{32, 34, 272, false}
           : t == Q2_K ? TcFmt{256, 84, 84, true}
           : t == Q3_K ? TcFmt{256, 110, 110, true}
           : t == Q4_K ? TcFmt{256, 144, 144, false}
           : t == Q5_K ? TcFmt{256, 176, 176, false}
           : t == Q6_K ? TcFmt{256, 210, 210, true}
                       : TcFmt{0, 0, 0, false};
}

// K position p (0..255) of a W stage -> the element of the stage it holds.
// p = 64 s + 32 t + 8 q + i: step s, chunk half t, dequantizer lane q of the
// row, element i of the 16-byte chunk.
//   family 1 (Q4_K, Q5_K, Q8_0, Q4_0): 32-element group 2s + t, inside it
//     16 (i / 4) + 4 q + i % 4 -- low/high nibbles or bytes of words q, q + 4.
//   family 2 (Q2_K, Q3_K, Q6_K): half n = s / 2, plane 2t + i / 4, inside the
//     plane 16 (s % 2) + 4 q + i % 4.
// Family 1 keeps every 32-element block inside its own 32 positions, so a K
// that ends half way through a step still maps positions < K to elements < K.
__host__ __device__ constexpr int tc_elem(bool f2, int p) {
    return f2 ? 128 * ((p >> 6) >> 1) + 32 * (2 * ((p >> 5) & 1) + ((p & 7) >> 2)) + 16 * ((p >> 6) & 1) +
                    4 * ((p >> 3) & 3) + (p & 3)
              : 64 * (p >> 6) + 32 * ((p >> 5) & 1) + 16 * ((p & 7) >> 2) + 4 * ((p >> 3) & 3) + (p & 3);
}

// ---- tcgen05 / UMMA helpers ---------------------------------------------------

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row groups of
// 128-byte rows stacked at 1024 bytes (stride byte offset), version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);       // start address
    d |= static_cast<uint64_t>(1u) << 16;                     // leading byte offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;             // stride byte offset
    d |= static_cast<uint64_t>(1u) << 46;                     // version
    d |= static_cast<uint64_t>(2u) << 61;                     // layout: SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::f16, A = B = fp16, D = fp32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                                   // D format f32
           | (0u << 7) | (0u << 10)                    // A, B fp16
           | (0u << 15) | (0u << 16)                   // K-major
           | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// true on exactly one lane of the (fully active) warp
__device__ __forceinline__ bool elect_one() {
    uint32_t e;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(e));
    return e != 0;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ---- shared-memory reads of the W stage -------------------------------------

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Little-endian word at byte address a: A4 -> a is 4-byte aligned; otherwise
// the word is funnel-shifted out of the two aligned words around it.
template <bool A4>
__device__ __forceinline__ uint32_t ldw(uint32_t a) {
    if constexpr (A4) {
        return lds32(a);
    } else {
        const uint32_t b = a & ~3u;
        return __funnelshift_r(lds32(b), lds32(b + 4), (a & 3u) << 3);
    }
}

// ---- fp16 arithmetic on packed pairs -------------------------------------------

__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<const __half2*>(&u); }
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }
__device__ __forceinline__ uint32_t pack_h2(float a, float b) { return h2u(__floats2half2_rn(a, b)); }
// (1024 + byte0, 1024 + byte1) and (1024 + byte2, 1024 + byte3) as fp16 pairs
__device__ __forceinline__ uint32_t h2b01(uint32_t q) { return __byte_perm(q, 0x64646464u, 0x4140u); }
__device__ __forceinline__ uint32_t h2b23(uint32_t q) { return __byte_perm(q, 0x64646464u, 0x4342u); }
__device__ __forceinline__ uint32_t bc_lo(uint32_t h) { return h2u(__low2half2(u2h(h))); }   // (h.x, h.x)
__device__ __forceinline__ uint32_t bc_hi(uint32_t h) { return h2u(__high2half2(u2h(h))); }  // (h.y, h.y)

// (v - bias) * d + n  and  (v - bias) * d, on fp16 pairs; v - bias is exact.
__device__ __forceinline__ uint32_t fq(uint32_t v, uint32_t bias, uint32_t d, uint32_t n) {
    return h2u(__hfma2(__hsub2(u2h(v), u2h(bias)), u2h(d), u2h(n)));
}
__device__ __forceinline__ uint32_t mq(uint32_t v, uint32_t bias, uint32_t d) {
    return h2u(__hmul2(__hsub2(u2h(v), u2h(bias)), u2h(d)));
}

constexpr uint32_t B1024 = 0x64006400u;  // fp16 1024
constexpr uint32_t B1028 = 0x64046404u;  // 1024 + 4
constexpr uint32_t B1032 = 0x64086408u;  // 1024 + 8
constexpr uint32_t B1056 = 0x64206420u;  // 1024 + 32
constexpr uint32_t B1152 = 0x64806480u;  // 1024 + 128

// fp16 bits (low 16) -> (h, h) pair
__device__ __forceinline__ uint32_t bc_bits(uint32_t b) { return (b & 0xFFFFu) * 0x10001u; }

// ---- per-format dequantization of one W stage, one row, one lane -------------
//
// load(): once per W stage (256 elements of the row), everything the lane needs
// for the stage's four steps -- its quant words and its scales -- into
// registers.  Scales are computed once per block, lane q of a row for part of
// the block, and handed to the row's other lanes (lane q of a row is warp lane
// rr + 8 q); the shuffles run here, on all 32 lanes.  After load() the stage's
// shared memory is no longer read.
// emit(s): the lane's 16 elements of step s as two 16-byte chunks (c0: t = 0,
// c1: t = 1) in the order of tc_elem.  `blk` is the shared-memory byte address
// of the block (256-element formats) or of the 8-block group (Q4_0, Q8_0).

template <int T>
struct Dq;

template <>
struct Dq<Q4_K> {  // d @0, dmin @2, scales[12] @4, qs[128] @16 (src/tensor.h:196-227)
    struct Stage {
        uint32_t wa[4], wb[4];  // qs words q and q + 4 of step s's 32 bytes
        uint32_t dd[4], mm[4];  // (d1, d2), (-m1, -m2) of sub-blocks 2s, 2s + 1
    };
    // (d * sc, -dmin * m) of sub-blocks 2q and 2q + 1
    template <bool A4>
    __device__ static void scales(uint32_t blk, int q, uint32_t& dd, uint32_t& mm) {
        const uint32_t w0 = ldw<A4>(blk), s0 = ldw<A4>(blk + 4), s1 = ldw<A4>(blk + 8), s2 = ldw<A4>(blk + 12);
        const float d = h2f(w0 & 0xFFFFu), dmin = h2f(w0 >> 16);
        uint32_t sc0, m0, sc1, m1;
        scale_min_k4_unit(q, 0, s0, s1, s2, sc0, m0);
        scale_min_k4_unit(q, 1, s0, s1, s2, sc1, m1);
        dd = pack_h2(d * static_cast<float>(sc0), d * static_cast<float>(sc1));
        mm = pack_h2(-(dmin * static_cast<float>(m0)), -(dmin * static_cast<float>(m1)));
    }
    template <bool A4>
    __device__ static void load(uint32_t blk, int q, int rr, Stage& g) {
        uint32_t dd, mm;
        scales<A4>(blk, q, dd, mm);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const uint32_t a = blk + 16 + 32 * s + 4 * q;
            g.wa[s] = ldw<A4>(a);
            g.wb[s] = ldw<A4>(a + 16);
            g.dd[s] = __shfl_sync(FULL, dd, rr + 8 * s);
            g.mm[s] = __shfl_sync(FULL, mm, rr + 8 * s);
        }
    }
    __device__ static void emit(const Stage& g, int s, uint4& c0, uint4& c1) {
        const uint32_t d0 = bc_lo(g.dd[s]), d1 = bc_hi(g.dd[s]), n0 = bc_lo(g.mm[s]), n1 = bc_hi(g.mm[s]);
        const uint32_t wa = g.wa[s], wb = g.wb[s];
        const uint32_t la = wa & 0x0F0F0F0Fu, lb = wb & 0x0F0F0F0Fu;
        const uint32_t ha = (wa >> 4) & 0x0F0F0F0Fu, hb = (wb >> 4) & 0x0F0F0F0Fu;
        c0 = make_uint4(fq(h2b01(la), B1024, d0, n0), fq(h2b23(la), B1024, d0, n0),
                        fq(h2b01(lb), B1024, d0, n0), fq(h2b23(lb), B1024, d0, n0));
        c1 = make_uint4(fq(h2b01(ha), B1024, d1, n1), fq(h2b23(ha), B1024, d1, n1),
                        fq(h2b01(hb), B1024, d1, n1), fq(h2b23(hb), B1024, d1, n1));
    }
};

template <>
struct Dq<Q5_K> {  // d @0, dmin @2, scales[12] @4, qh[32] @16, qs[128] @48 (src/tensor.h:329-365)
    struct Stage {
        uint32_t wa[4], wb[4];  // qs words q and q + 4 of step s's 32 bytes
        uint32_t qa, qb;        // qh bytes of elements 4q .. and 16 + 4q .. (bit j: sub-block j)
        uint32_t dd[4], mm[4];
    };
    template <bool A4>
    __device__ static void load(uint32_t blk, int q, int rr, Stage& g) {
        uint32_t dd, mm;
        Dq<Q4_K>::scales<A4>(blk, q, dd, mm);
        g.qa = ldw<A4>(blk + 16 + 4 * q);
        g.qb = ldw<A4>(blk + 32 + 4 * q);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const uint32_t a = blk + 48 + 32 * s + 4 * q;
            g.wa[s] = ldw<A4>(a);
            g.wb[s] = ldw<A4>(a + 16);
            g.dd[s] = __shfl_sync(FULL, dd, rr + 8 * s);
            g.mm[s] = __shfl_sync(FULL, mm, rr + 8 * s);
        }
    }
    __device__ static void emit(const Stage& g, int s, uint4& c0, uint4& c1) {
        const uint32_t d0 = bc_lo(g.dd[s]), d1 = bc_hi(g.dd[s]), n0 = bc_lo(g.mm[s]), n1 = bc_hi(g.mm[s]);
        const uint32_t wa = g.wa[s], wb = g.wb[s];
        const uint32_t qa = g.qa >> (2 * s), qb = g.qb >> (2 * s);
        // high bit of sub-block 2s + t: bit 2s + t of the qh byte, moved to bit 4
        const uint32_t la = (wa & 0x0F0F0F0Fu) | ((qa << 4) & 0x10101010u);
        const uint32_t lb = (wb & 0x0F0F0F0Fu) | ((qb << 4) & 0x10101010u);
        const uint32_t ha = ((wa >> 4) & 0x0F0F0F0Fu) | ((qa << 3) & 0x10101010u);
        const uint32_t hb = ((wb >> 4) & 0x0F0F0F0Fu) | ((qb << 3) & 0x10101010u);
        c0 = make_uint4(fq(h2b01(la), B1024, d0, n0), fq(h2b23(la), B1024, d0, n0),
                        fq(h2b01(lb), B1024, d0, n0), fq(h2b23(lb), B1024, d0, n0));
        c1 = make_uint4(fq(h2b01(ha), B1024, d1, n1), fq(h2b23(ha), B1024, d1, n1),
                        fq(h2b01(hb), B1024, d1, n1), fq(h2b23(hb), B1024, d1, n1));
    }
};

// Scales of the planes of Q6_K / Q3_K / Q2_K: index 8n + 2kk + hb for plane kk of
// half n and l in 16hb ..; lane q computes indices 4q .. 4q + 3 and holds them as
// a0 = (s[4q], s[4q+2]), a1 = (s[4q+1], s[4q+3]).  Step s (n = s/2, hb = s%2)
// takes a_hb of lane 2n (planes 0, 1) and of lane 2n + 1 (planes 2, 3).
__device__ __forceinline__ void plane_scales(uint32_t a0, uint32_t a1, int rr, uint32_t (&p01)[4],
                                             uint32_t (&p23)[4]) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int n = s >> 1;
        const uint32_t mine = (s & 1) ? a1 : a0;
        p01[s] = __shfl_sync(FULL, mine, rr + 16 * n);
        p23[s] = __shfl_sync(FULL, mine, rr + 16 * n + 8);
    }
}

template <>
struct Dq<Q6_K> {  // ql[128] @0, qh[64] @128, scales[16] (int8) @192, d @208 (src/tensor.h:368-403)
    struct Stage {
        uint32_t wa[4], wb[4], wc[4];  // ql[64n + l], ql[64n + 32 + l], qh[32n + l] for l = 16hb + 4q ..
        uint32_t s01[4], s23[4];       // d * scale of planes (0, 1) and (2, 3)
    };
    template <bool A4>
    __device__ static void load(uint32_t blk, int q, int rr, Stage& g) {
        const uint32_t sw = ldw<A4>(blk + 192 + 4 * q);
        const float d = h2f(ldw<A4>(blk + 208) & 0xFFFFu);
        const float s0 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 0)));
        const float s1 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 1)));
        const float s2 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 2)));
        const float s3 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 3)));
        plane_scales(pack_h2(d * s0, d * s2), pack_h2(d * s1, d * s3), rr, g.s01, g.s23);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int n = s >> 1, hb = s & 1;
            const uint32_t a = blk + 64 * n + 16 * hb + 4 * q;
            g.wa[s] = ldw<A4>(a);
            g.wb[s] = ldw<A4>(a + 32);
            g.wc[s] = ldw<A4>(blk + 128 + 32 * n + 16 * hb + 4 * q);
        }
    }
    __device__ static void emit(const Stage& g, int s, uint4& c0, uint4& c1) {
        const uint32_t sc0 = bc_lo(g.s01[s]), sc1 = bc_hi(g.s01[s]), sc2 = bc_lo(g.s23[s]), sc3 = bc_hi(g.s23[s]);
        const uint32_t wa = g.wa[s], wb = g.wb[s], wc = g.wc[s];
        const uint32_t c4 = wc << 4;  // qh bits 2kk .. 2kk + 1 of each byte to bits 4 .. 5
        const uint32_t p0 = (wa & 0x0F0F0F0Fu) | (c4 & 0x30303030u);
        const uint32_t p1 = (wb & 0x0F0F0F0Fu) | ((c4 >> 2) & 0x30303030u);
        const uint32_t p2 = ((wa >> 4) & 0x0F0F0F0Fu) | (wc & 0x30303030u);
        const uint32_t p3 = ((wb >> 4) & 0x0F0F0F0Fu) | ((wc >> 2) & 0x30303030u);
        c0 = make_uint4(mq(h2b01(p0), B1056, sc0), mq(h2b23(p0), B1056, sc0),
                        mq(h2b01(p1), B1056, sc1), mq(h2b23(p1), B1056, sc1));
        c1 = make_uint4(mq(h2b01(p2), B1056, sc2), mq(h2b23(p2), B1056, sc2),
                        mq(h2b01(p3), B1056, sc3), mq(h2b23(p3), B1056, sc3));
    }
};

template <>
struct Dq<Q2_K> {  // scales[16] @0, qs[64] @16, d @80, dmin @82 (src/tensor.h:232-265)
    struct Stage {
        uint32_t w[4];                         // qs[32n + l], l = 16hb + 4q ..
        uint32_t d01[4], d23[4], m01[4], m23[4];  // (dl, -ml) of planes (0, 1), (2, 3)
    };
    template <bool A4>
    __device__ static void load(uint32_t blk, int q, int rr, Stage& g) {
        const uint32_t sw = ldw<A4>(blk + 4 * q), dw = ldw<A4>(blk + 80);
        const float d = h2f(dw & 0xFFFFu), dmin = h2f(dw >> 16);
        float dl[4], ml[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t b = byte_of(sw, i);
            dl[i] = d * static_cast<float>(b & 15u);
            ml[i] = -(dmin * static_cast<float>(b >> 4));
        }
        plane_scales(pack_h2(dl[0], dl[2]), pack_h2(dl[1], dl[3]), rr, g.d01, g.d23);
        plane_scales(pack_h2(ml[0], ml[2]), pack_h2(ml[1], ml[3]), rr, g.m01, g.m23);
#pragma unroll
        for (int s = 0; s < 4; ++s) g.w[s] = ldw<A4>(blk + 16 + 32 * (s >> 1) + 16 * (s & 1) + 4 * q);
    }
    __device__ static void emit(const Stage& g, int s, uint4& c0, uint4& c1) {
        const uint32_t w = g.w[s];
        const uint32_t p0 = w & 0x03030303u, p1 = (w >> 2) & 0x03030303u;
        const uint32_t p2 = (w >> 4) & 0x03030303u, p3 = (w >> 6) & 0x03030303u;
        const uint32_t e0 = bc_lo(g.d01[s]), e1 = bc_hi(g.d01[s]), e2 = bc_lo(g.d23[s]), e3 = bc_hi(g.d23[s]);
        const uint32_t f0 = bc_lo(g.m01[s]), f1 = bc_hi(g.m01[s]), f2 = bc_lo(g.m23[s]), f3 = bc_hi(g.m23[s]);
        c0 = make_uint4(fq(h2b01(p0), B1024, e0, f0), fq(h2b23(p0), B1024, e0, f0),
                        fq(h2b01(p1), B1024, e1, f1), fq(h2b23(p1), B1024, e1, f1));
        c1 = make_uint4(fq(h2b01(p2), B1024, e2, f2), fq(h2b23(p2), B1024, e2, f2),
                        fq(h2b01(p3), B1024, e3, f3), fq(h2b23(p3), B1024, e3, f3));
    }
};

template <>
struct Dq<Q3_K> {  // hmask[32] @0, qs[64] @32, scales[12] @96, d @108 (src/tensor.h:269-326)
    struct Stage {
        uint32_t wq[4];        // qs[32n + l], l = 16hb + 4q ..
        uint32_t wh0, wh1;     // hmask[l] for hb = 0, 1 (bit 4n + j: plane j of half n)
        uint32_t s01[4], s23[4];
    };
    template <bool A4>
    __device__ static void load(uint32_t blk, int q, int rr, Stage& g) {
        const uint32_t t0 = ldw<A4>(blk + 96), t1 = ldw<A4>(blk + 100), t2 = ldw<A4>(blk + 104);
        const float d = h2f(ldw<A4>(blk + 108) & 0xFFFFu);
        const uint32_t sw = q3k_scale_word(q, t0, t1, t2);
        const float s0 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 0)));
        const float s1 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 1)));
        const float s2 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 2)));
        const float s3 = static_cast<float>(static_cast<int8_t>(byte_of(sw, 3)));
        plane_scales(pack_h2(d * s0, d * s2), pack_h2(d * s1, d * s3), rr, g.s01, g.s23);
        g.wh0 = ldw<A4>(blk + 4 * q);
        g.wh1 = ldw<A4>(blk + 16 + 4 * q);
#pragma unroll
        for (int s = 0; s < 4; ++s) g.wq[s] = ldw<A4>(blk + 32 + 32 * (s >> 1) + 16 * (s & 1) + 4 * q);
    }
    __device__ static void emit(const Stage& g, int s, uint4& c0, uint4& c1) {
        const int n = s >> 1;
        const uint32_t sc0 = bc_lo(g.s01[s]), sc1 = bc_hi(g.s01[s]), sc2 = bc_lo(g.s23[s]), sc3 = bc_hi(g.s23[s]);
        const uint32_t wq = g.wq[s];
        const uint32_t h4 = ((s & 1) ? g.wh1 : g.wh0) >> (4 * n) << 2;  // plane j's bit at bit j + 2
        const uint32_t p0 = (wq & 0x03030303u) | (h4 & 0x04040404u);
        const uint32_t p1 = ((wq >> 2) & 0x03030303u) | ((h4 >> 1) & 0x04040404u);
        const uint32_t p2 = ((wq >> 4) & 0x03030303u) | ((h4 >> 2) & 0x04040404u);
        const uint32_t p3 = ((wq >> 6) & 0x03030303u) | ((h4 >> 3) & 0x04040404u);
        c0 = make_uint4(mq(h2b01(p0), B1028, sc0), mq(h2b23(p0), B1028, sc0),
                        mq(h2b01(p1), B1028, sc1), mq(h2b23(p1), B1028, sc1));
        c1 = make_uint4(mq(h2b01(p2), B1028, sc2), mq(h2b23(p2), B1028, sc2),
                        mq(h2b01(p3), B1028, sc3), mq(h2b23(p3), B1028, sc3));
    }
};

template <>
struct Dq<Q8_0> {  // d @0, qs[32] (int8) @2 (src/tensor.h:157-166); a W stage is 8 blocks
    struct Stage {
        uint32_t d[8];          // (d, d) of block b
        uint32_t wa[8], wb[8];  // quant words q and q + 4 of block b
    };
    template <bool A4>
    __device__ static void load(uint32_t grp, int q, int, Stage& g) {
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const uint32_t a = grp + 34 * b;
            g.d[b] = bc_bits(ldw<A4>(a));
            g.wa[b] = ldw<A4>(a + 2 + 4 * q);
            g.wb[b] = ldw<A4>(a + 18 + 4 * q);
        }
    }
    // block b: bytes as q + 128, then (1152 + q) - 1152
    __device__ static uint4 blk32(const Stage& g, int b) {
        const uint32_t d = g.d[b], wa = g.wa[b] ^ 0x80808080u, wb = g.wb[b] ^ 0x80808080u;
        return make_uint4(mq(h2b01(wa), B1152, d), mq(h2b23(wa), B1152, d), mq(h2b01(wb), B1152, d),
                          mq(h2b23(wb), B1152, d));
    }
    __device__ static void emit(const Stage& g, int s, uint4& c0, uint4& c1) {
        c0 = blk32(g, 2 * s);
        c1 = blk32(g, 2 * s + 1);
    }
};

template <>
struct Dq<Q4_0> {  // d @0, qs[16] @2: element l low nibble of byte l, l + 16 high (src/tensor.h:139-154)
    struct Stage {
        uint32_t d[8], w[8];  // (d, d) and quant word q of block b of the 8-block group
    };
    template <bool A4>
    __device__ static void load(uint32_t grp, int q, int, Stage& g) {
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const uint32_t a = grp + 18 * b;
            g.d[b] = bc_bits(ldw<A4>(a));
            g.w[b] = ldw<A4>(a + 2 + 4 * q);
        }
    }
    __device__ static uint4 blk32(const Stage& g, int b) {
        const uint32_t d = g.d[b], w = g.w[b];
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        return make_uint4(mq(h2b01(lo), B1032, d), mq(h2b23(lo), B1032, d), mq(h2b01(hi), B1032, d),
                          mq(h2b23(hi), B1032, d));
    }
    __device__ static void emit(const Stage& g, int s, uint4& c0, uint4& c1) {
        c0 = blk32(g, 2 * s);
        c1 = blk32(g, 2 * s + 1);
    }
};

struct Params {
    const uint8_t* W;
    float* Y;
    const float* rowscale;  // per X row: 2^k undoing the conversion's scaling
    int M, N, K;
    int row_bytes;
    int n_mtiles, n_ntiles, ksteps;
    int nblocks;      // blocks per row
    int ngroups;      // W stages per tile = ceil(K / 256)
    int stages;       // A/B ring depth
    int wstages;      // W ring depth
    int wp;           // W stage row pitch in shared memory (bytes, 16 x odd)
    int rows_mode;    // 0: one tensor-map copy per W stage; 1: one bulk copy per row
    const uint8_t* w_lo;  // W rounded down to 16 bytes
    const uint8_t* w_hi;  // end of W rounded up to 16 bytes
    // grouped (MoE) mode: expert e multiplies rows offsets[e] .. offsets[e+1]-1
    // of X by its own weights wptrs[e]; offsets are clamped to [0, rows_total]
    // and made non-decreasing on the device.
    const uint8_t* const* wptrs;
    const int* offsets;
    int n_experts;
    int rows_total;
    int stacked;  // grouped: expert e's matrix is rows e*N .. e*N+N-1 of W (wptrs unused)
    int early;  // the W producer may read weights before the previous kernel completes
    // split-K (dense only): each output tile is computed as ksplit work units
    // of gps W stages each; unit u = tile * ksplit + split.  With ksplit > 1
    // every unit writes its partial tile to part[split][M][N], and the unit
    // that finishes a tile last (count in tcount[tile], zeroed by the
    // activation conversion, reset by that unit) sums the partials in split
    // order into Y.
    int ksplit, gps;
    float* part;
    unsigned* tcount;
};

// One output tile: weights, token rows m0 .. m_end-1 (the tile covers m0 .. m0+BN-1),
// W-row tile nt.
struct TileRef {
    const uint8_t* W;
    int m0, m_end, nt;
    int e;  // grouped: the expert
};

__device__ __forceinline__ int clamp_off(const Params& p, int e) { return min(max(p.offsets[e], 0), p.rows_total); }

// Tile index -> TileRef.  Dense: token tile = tile / n_ntiles.  Grouped: tiles are
// numbered expert by expert (tpre[e] = first tile of expert e), ntiles per
// token tile of the expert.
template <bool G, int BN>
__device__ __forceinline__ TileRef tile_ref(const Params& p, const int* tpre, int tile) {
    TileRef r;
    if constexpr (!G) {
        r.nt = tile % p.n_ntiles;
        r.m0 = (tile / p.n_ntiles) * BN;
        r.m_end = p.M;
        r.W = p.W;
        r.e = 0;
    } else {
        int lo = 0, hi = p.n_experts;  // last e with tpre[e] <= tile (empty experts share values)
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (tpre[mid] <= tile) lo = mid; else hi = mid;
        }
        const int local = tile - tpre[lo];
        const int a = clamp_off(p, lo), b = max(a, clamp_off(p, lo + 1));
        r.nt = local % p.n_ntiles;
        r.m0 = a + (local / p.n_ntiles) * BN;
        r.m_end = b;
        r.W = p.stacked ? p.W + static_cast<size_t>(lo) * p.N * p.row_bytes : p.wptrs[lo];
        r.e = lo;
    }
    return r;
}

// Work unit -> (tile, W stage range [g0, g1)).
struct UnitRef {
    int tile, split, g0, g1;
};
__device__ __forceinline__ UnitRef unit_ref(const Params& p, int u) {
    UnitRef r;
    r.tile = u / p.ksplit;
    r.split = u - r.tile * p.ksplit;
    r.g0 = r.split * p.gps;
    r.g1 = min(p.ngroups, r.g0 + p.gps);
    return r;
}

template <int T, int BN, bool A4, bool G>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const Params p, const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap) {
    using D = Dq<T>;
    constexpr TcFmt F = tc_fmt(T);
    constexpr int B_STAGE = BN * BK * 2;
    constexpr uint32_t IDESC = idesc_f16(BM, BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled operands
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S_ = p.stages, SW = p.wstages;
    const int WSTAGE = BM * p.wp;
    uint8_t* a_st = smem;                                   // S x 16 KB
    uint8_t* b_st = a_st + S_ * A_STAGE;                    // S x B_STAGE
    uint8_t* w_st = b_st + S_ * B_STAGE;                    // SW x 128 rows x wp
    // 16 bytes of slack after the W ring: a 2-byte aligned word read at the end
    // of the last row touches the next aligned word.
    uint64_t* bars = reinterpret_cast<uint64_t*>(w_st + SW * WSTAGE + 16);
    uint64_t* full_a = bars;                 // [S] dequantizer warps (NDQ arrivals)
    uint64_t* full_b = bars + S_;            // [S] X TMA bytes
    uint64_t* empty = bars + 2 * S_;         // [S] MMA commit
    uint64_t* wfull = bars + 3 * S_;         // [SW] W bytes (1 or 32 arrivals)
    uint64_t* wempty = wfull + SW;           // [SW] dequantizer warps (NDQ arrivals)
    uint64_t* tfull = wempty + SW;           // [2] MMA commit per tile
    uint64_t* tempty = tfull + 2;            // [2] epilogue warps (4 arrivals)
    uint64_t* drain = tempty + 2;            // final MMA commit before TMEM is freed
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 1) + 1;
    int* tpre = reinterpret_cast<int*>(drain + 2);  // grouped: n_experts + 1 tile offsets

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S_; ++s) {
            mbar_init(&full_a[s], NDQ);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < SW; ++s) {
            mbar_init(&wfull[s], p.rows_mode ? 32 : 1);
            mbar_init(&wempty[s], NDQ);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&tfull[t], 1);
            mbar_init(&tempty[t], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (G) pdl_wait_primary();  // the expert offsets may come from the previous kernels
    if (G && warp == 0) {
        // tiles of expert e = ceil(rows_e / BN) * n_ntiles; tpre = exclusive prefix
        int carry = 0;
        for (int base = 0; base < p.n_experts; base += 32) {
            const int e = base + lane;
            int v = 0;
            if (e < p.n_experts) {
                const int a = clamp_off(p, e), b = max(a, clamp_off(p, e + 1));
                v = ((b - a + BN - 1) / BN) * p.n_ntiles;
            }
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int u = __shfl_up_sync(FULL, v, d);
                if (lane >= d) v += u;
            }
            if (e < p.n_experts) tpre[e + 1] = carry + v;
            carry += __shfl_sync(FULL, v, 31);
        }
        if (lane == 0) tpre[0] = 0;
    }
    if (warp == WARP_MMA) {
        // 2 x BN fp32 columns of TMEM (double-buffered accumulator)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(const_cast<uint32_t*>(tmem_slot))), "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int ntiles = G ? tpre[p.n_experts] : p.n_mtiles * p.n_ntiles * p.ksplit;  // work units
    // Programmatic dependency on the conversion kernel before this one: the
    // roles that read X16 (X producer) or write Y and the split-K buffers
    // (epilogue) wait for it; the W producer, the dequantizers and the MMA
    // touch only the immutable weights and shared memory, so the first W
    // stages stream in while the conversion finishes.  Grouped launches read
    // the expert offsets above, so everything waits.
    if (!G && (!p.early || warp == WARP_X || is_epilogue(warp))) pdl_wait_primary();

    if (warp == WARP_X) {
        // -------------------------------------------------- activation TMA producer
        // The whole warp runs the loop; one elected lane issues the copies.
        int s = 0;
        uint32_t ph = 0;
        int it = 0;  // loads issued
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            if (__shfl_sync(FULL, *abort_flag, 0)) break;
            const UnitRef ur = unit_ref(p, tile);
            const TileRef tr = tile_ref<G, BN>(p, tpre, ur.tile);
            const int ks1 = min(p.ksteps, ur.g1 * (KG / BK));
            bool ok = true;
            for (int ks = ur.g0 * (KG / BK); ks < ks1; ++ks, ++it) {
                const bool got = it < S_ || mbar_wait_bounded(&empty[s], ph ^ 1u, DEV_TIMEOUT_EMPTY);
                if (!__all_sync(FULL, got)) {
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                if (elect_one()) {
                    mbar_arrive_expect_tx(&full_b[s], B_STAGE);
                    tma_load_2d(smem_u32(b_st + s * B_STAGE), &xmap, ks * BK, tr.m0, &full_b[s]);
                }
                __syncwarp();
                if (++s == S_) { s = 0; ph ^= 1u; }
            }
            if (!ok) break;
        }
        // Wait for the last load issued into each stage, so that no copy is
        // still writing shared memory when the CTA exits (immediate unless a
        // wait above gave up).
        for (int i = 0; i < S_ && i < it; ++i) {
            const int idx = it - 1 - i;
            mbar_wait_bounded(&full_b[idx % S_], static_cast<uint32_t>(idx / S_) & 1u, DEV_TIMEOUT_DRAIN);
        }
    } else if (warp == WARP_MMA) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs the loop (warp-uniform descriptors); one elected
        // lane issues the MMAs and the commits that track them.
        int s = 0;
        uint32_t ph = 0;
        int t_local = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t_local) {
            if (__shfl_sync(FULL, *abort_flag, 0)) break;
            const int tb = t_local & 1;
            const uint32_t tph = (t_local >> 1) & 1;
            if (t_local >= 2) {
                const bool got = mbar_wait_bounded(&tempty[tb], tph ^ 1u, DEV_TIMEOUT_MMA);
                if (!__all_sync(FULL, got)) {
                    *abort_flag = 1;
                    break;
                }
            }
            tc_fence_after();
            const uint32_t dt = tmem_base + static_cast<uint32_t>(tb * BN);
            const UnitRef ur = unit_ref(p, tile);
            const int ks0 = ur.g0 * (KG / BK), ks1 = min(p.ksteps, ur.g1 * (KG / BK));
            bool ok = true;
            for (int ks = ks0; ks < ks1; ++ks) {
                const bool got = mbar_wait_bounded(&full_a[s], ph, DEV_TIMEOUT_FULL) &&
                                 mbar_wait_bounded(&full_b[s], ph, DEV_TIMEOUT_FULL);
                if (!__all_sync(FULL, got)) {
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t da = smem_desc_sw128(smem_u32(a_st + s * A_STAGE));
                const uint64_t db = smem_desc_sw128(smem_u32(b_st + s * B_STAGE));
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)  // 32 bytes of K per instruction
                        mma_f16(dt, da + 2 * k, db + 2 * k, IDESC, (ks > ks0 || k) ? 1u : 0u);
                    mma_commit(&empty[s]);
                }
                __syncwarp();
                if (++s == S_) { s = 0; ph ^= 1u; }
            }
            if (!ok) break;
            if (elect_one()) mma_commit(&tfull[tb]);
            __syncwarp();
        }
        // One more commit tracks every MMA the elected lane issued: once it
        // arrives, no tensor-core write to TMEM is in flight.
        if (elect_one()) mma_commit(drain);
        __syncwarp();
        mbar_wait_bounded(drain, 0u, DEV_TIMEOUT_DRAIN);
    } else if (warp == WARP_W) {
        // --------------------------------------------------------- W producer
        const uint64_t pol = l2_policy_evict_first();
        int js = 0;
        uint32_t jph = 0;
        int jt = 0;  // W stages issued
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            if (__shfl_sync(FULL, *abort_flag, 0)) break;
            const UnitRef ur = unit_ref(p, tile);
            const TileRef tr = tile_ref<G, BN>(p, tpre, ur.tile);
            const int row0 = tr.nt * BM;
            const uint8_t* w_hi = G ? reinterpret_cast<const uint8_t*>(
                                          (reinterpret_cast<uintptr_t>(tr.W) + static_cast<size_t>(p.N) * p.row_bytes +
                                           15) & ~uintptr_t(15))
                                    : p.w_hi;
            bool ok = true;
            for (int g = ur.g0; g < ur.g1; ++g, ++jt) {
                const bool got = jt < SW || mbar_wait_bounded(&wempty[js], jph ^ 1u, DEV_TIMEOUT_EMPTY);
                if (!__all_sync(FULL, got)) {
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                const uint32_t dst = smem_u32(w_st + js * WSTAGE);
                const size_t goff = static_cast<size_t>(g) * F.gbytes;
                if (!p.rows_mode) {
                    // one tensor-map box per stage; stacked experts are rows of one map
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&wfull[js], static_cast<uint32_t>(WSTAGE));
                        tma_load_2d(dst, &wmap, static_cast<int>((goff & ~size_t(15)) >> 1),
                                    G ? tr.e * p.N + row0 : row0, &wfull[js]);
                    }
                } else {
                    // Rows lane, lane + 32, lane + 64, lane + 96 of the tile: copy
                    // wp bytes from the 16-byte boundary at or below the row's
                    // stage data, clipped at the end of W rounded up to 16.
                    uint32_t bytes = 0;
                    const uint8_t* src[4];
                    uint32_t len[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int row = row0 + lane + 32 * k;
                        len[k] = 0;
                        src[k] = tr.W;
                        if (row < p.N) {
                            const uint8_t* a = tr.W + static_cast<size_t>(row) * p.row_bytes + goff;
                            const uint8_t* a16 = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(a) &
                                                                                  ~uintptr_t(15));
                            const size_t room = static_cast<size_t>(w_hi - a16);
                            src[k] = a16;
                            len[k] = static_cast<uint32_t>(room < static_cast<size_t>(p.wp) ? room : p.wp);
                            bytes += len[k];
                        }
                    }
                    mbar_arrive_expect_tx(&wfull[js], bytes);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (len[k]) bulk_g2s(w_st + js * WSTAGE + (lane + 32 * k) * p.wp, src[k], len[k], &wfull[js], pol);
                }
                if (++js == SW) { js = 0; jph ^= 1u; }
            }
            if (!ok) break;
        }
        // wait for the last W stage issued into each slot
        if (lane == 0) {
            for (int i = 0; i < SW && i < jt; ++i) {
                const int idx = jt - 1 - i;
                mbar_wait_bounded(&wfull[idx % SW], static_cast<uint32_t>(idx / SW) & 1u, DEV_TIMEOUT_DRAIN);
            }
        }
    } else if (dq_index(warp) >= 0) {
        // ------------------------------------------------------- W dequantizers
        const int rr = lane & 7, q = lane >> 3;
        const int r0 = 8 * dq_index(warp) + rr;  // the lane's tile rows r0 + 8 NDQ p
        int s = 0;
        uint32_t ph = 0;
        int it = 0;
        int js = 0;
        uint32_t jph = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            if (__shfl_sync(FULL, *abort_flag, 0)) break;
            const UnitRef ur = unit_ref(p, tile);
            const TileRef tr = tile_ref<G, BN>(p, tpre, ur.tile);
            const uintptr_t wbase = reinterpret_cast<uintptr_t>(tr.W);
            const int row0 = tr.nt * BM;
            const bool ragged = row0 + BM > p.N;  // last row tile of a ragged N
            bool valid[PASSES];
            uintptr_t rowg[PASSES];
#pragma unroll
            for (int pp = 0; pp < PASSES; ++pp) {
                const int r = r0 + 8 * NDQ * pp;
                valid[pp] = row0 + r < p.N;
                rowg[pp] = wbase + static_cast<uintptr_t>(valid[pp] ? row0 + r : 0) * p.row_bytes;
            }
            bool ok = true;
            for (int g = ur.g0; g < ur.g1 && ok; ++g) {
                const bool gotw = mbar_wait_bounded(&wfull[js], jph, DEV_TIMEOUT_FULL);
                if (!__all_sync(FULL, gotw)) {
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                const uintptr_t goff = static_cast<uintptr_t>(g) * F.gbytes;
                const uint32_t ws = smem_u32(w_st + js * WSTAGE);
                // The whole stage goes to registers, then the slot is handed back
                // to the W producer before any of its steps is dequantized.  A
                // row's stage data starts (its global address mod 16) into its
                // smem row.
                typename D::Stage stg[PASSES];
#pragma unroll
                for (int pp = 0; pp < PASSES; ++pp) {
                    const uint32_t blk =
                        ws + (r0 + 8 * NDQ * pp) * p.wp + static_cast<uint32_t>((rowg[pp] + goff) & 15u);
                    D::template load<A4>(blk, q, rr, stg[pp]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&wempty[js]);
                if (++js == SW) { js = 0; jph ^= 1u; }
                const int nsteps = min(KG / BK, p.ksteps - g * (KG / BK));
#pragma unroll
                for (int st = 0; st < KG / BK; ++st) {
                    if (st >= nsteps) break;
                    const bool got = it < S_ || mbar_wait_bounded(&empty[s], ph ^ 1u, DEV_TIMEOUT_EMPTY);
                    if (!__all_sync(FULL, got)) {  // the warp leaves together
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    // a 32-element block past the end of the row (K % 64 == 32) is zero
                    const bool z1 = F.qk == 32 && g * 8 + 2 * st + 1 >= p.nblocks;
                    const uint32_t as = smem_u32(a_st + s * A_STAGE);
#pragma unroll
                    for (int pp = 0; pp < PASSES; ++pp) {
                        uint4 c0, c1;
                        D::emit(stg[pp], st, c0, c1);
                        const uint4 zero = make_uint4(0, 0, 0, 0);
                        if (ragged && !valid[pp]) { c0 = zero; c1 = zero; }
                        if (z1) c1 = zero;
                        const int r = r0 + 8 * NDQ * pp;
                        const uint32_t line = as + (r >> 3) * 1024 + (r & 7) * 128;
                        sts128(line + ((q ^ (r & 7)) << 4), c0);
                        sts128(line + (((4 + q) ^ (r & 7)) << 4), c1);
                    }
                    fence_async_shared();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full_a[s]);
                    ++it;
                    if (++s == S_) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) break;
        }
    } else if (is_epilogue(warp)) {
        // -------------------------------------------------------------- epilogue
        const int q = warp & 3;        // TMEM lane quadrant
        const int r = 32 * q + lane;   // W row within the tile
        int t_local = 0;
        const bool split = !G && p.ksplit > 1;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t_local) {
            if (__shfl_sync(FULL, *abort_flag, 0)) break;
            const UnitRef ur = unit_ref(p, tile);
            const TileRef tr = tile_ref<G, BN>(p, tpre, ur.tile);
            const int nt = tr.nt;
            const int tb = t_local & 1;
            const uint32_t tph = (t_local >> 1) & 1;
            const bool got = mbar_wait_bounded(&tfull[tb], tph, DEV_TIMEOUT_MMA);
            if (!__all_sync(FULL, got)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int row = nt * BM + r;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(tb * BN);
            float* dst = split ? p.part + static_cast<size_t>(ur.split) * p.M * p.N : p.Y;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tbase + c0, v);
                tmem_wait_ld();
                if (row < p.N) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int tok = tr.m0 + c0 + j;
                        if (tok < tr.m_end)
                            dst[static_cast<size_t>(tok) * p.N + row] =
                                split ? __uint_as_float(v[j]) : __uint_as_float(v[j]) * __ldg(&p.rowscale[tok]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[tb]);
            if (split) {
                // This warp's 32 rows of the tile: the warp that writes its
                // partial last sums all of them, in split order, into Y.  Each
                // warp counts for itself, so no warp ever waits on another.
                __threadfence();
                __syncwarp();
                unsigned last = 0;
                if (lane == 0) {
                    unsigned* cnt = p.tcount + static_cast<size_t>(ur.tile) * 4 + q;
                    last = atomicAdd(cnt, 1u) == static_cast<unsigned>(p.ksplit - 1);
                    if (last) *cnt = 0u;  // ready for the next call
                }
                if (__shfl_sync(FULL, last, 0)) {
                    __threadfence();
                    const int tend = min(tr.m_end, tr.m0 + BN);
                    if (row < p.N) {
                        for (int t0 = tr.m0; t0 < tend; t0 += 4) {
                            float v[4][TC_MAX_SPLIT];
#pragma unroll
                            for (int i = 0; i < 4; ++i)
#pragma unroll
                                for (int sp = 0; sp < TC_MAX_SPLIT; ++sp)
                                    v[i][sp] = (t0 + i < tend && sp < p.ksplit)
                                                   ? __ldcg(&p.part[(static_cast<size_t>(sp) * p.M + t0 + i) * p.N + row])
                                                   : 0.f;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                if (t0 + i >= tend) break;
                                float acc = 0.f;
#pragma unroll
                                for (int sp = 0; sp < TC_MAX_SPLIT; ++sp)
                                    if (sp < p.ksplit) acc += v[i][sp];
                                p.Y[static_cast<size_t>(t0 + i) * p.N + row] = acc * __ldg(&p.rowscale[t0 + i]);
                            }
                        }
                    }
                }
            }
        }
    }

    // Teardown: every role has left its loop (all waits are bounded), the MMA
    // lane has seen its last commit and the producers their last loads.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == WARP_MMA)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * BN));
}

}  // namespace tc

// fp32 -> fp16 activations in the K order of the tensor-core GEMM: within each
// 256-element group, position p holds element tc_elem(F2, p).  Each row is
// first scaled by the power of two 2^-k that brings its largest finite
// magnitude into [2^14, 2^15): no element overflows fp16 (65504) and small
// rows keep fp16's full precision instead of falling into its subnormals;
// rowscale[row] = 2^k undoes it exactly in the epilogue.  All-zero rows and
// rows holding inf keep k = 0.  One CTA per row (grid-stride); 8 positions per thread-step, two
// runs of four consecutive elements (float4 when aligned).
// Four consecutive prologue inputs at k (k % 4 == 0): the value the GEMM
// multiplies (v), and for RMSNORM the sum x = X + R before the weights.
template <bool VEC>
__device__ __forceinline__ float4 ld4(const float* p) {
    if (VEC) return *reinterpret_cast<const float4*>(p);
    return make_float4(p[0], p[1], p[2], p[3]);
}
template <bool VEC>
__device__ __forceinline__ float4 act4(const ActArgs& a, const float* xr, const float* rr, int K, int k, float4& x) {
    x = ld4<VEC>(xr + k);
    if (a.kind == 2) {
        const float4 u = ld4<VEC>(xr + K + k);
        return make_float4(x.x / (1.0f + expf(-x.x)) * u.x, x.y / (1.0f + expf(-x.y)) * u.y,
                           x.z / (1.0f + expf(-x.z)) * u.z, x.w / (1.0f + expf(-x.w)) * u.w);
    }
    if (a.kind == 1) {
        if (rr) {
            const float4 r = ld4<VEC>(rr + k);
            x.x += r.x; x.y += r.y; x.z += r.z; x.w += r.w;
        }
        const float4 w = ld4<VEC>(a.normw + k);
        return make_float4(x.x * w.x, x.y * w.y, x.z * w.z, x.w * w.w);
    }
    return x;
}

// fp32 -> fp16 activations in the K order of the tensor-core GEMM: within each
// 256-element group, position p holds element tc_elem(F2, p).  Each row (after
// the activation prologue) is first scaled by the power of two 2^-k that
// brings its largest finite magnitude into [2^14, 2^15): no element overflows
// fp16 (65504) and small rows keep fp16's full precision instead of falling
// into its subnormals; rowscale[row] = 2^k (times the RMSNORM factor) undoes
// it exactly in the epilogue.  All-zero rows and rows holding inf keep k = 0.
// One CTA per row (grid-stride); 8 positions per thread-step, two runs of four
// consecutive elements (float4 when aligned).
template <bool F2, bool VEC>
__global__ void __launch_bounds__(256) x_to_f16_kernel(const float* __restrict__ X, __half* __restrict__ Xh,
                                                       float* __restrict__ rowscale, int M, int K,
                                                       unsigned* __restrict__ tcount, int ncount, const ActArgs act,
                                                       int q2ref) {
    __shared__ float red[8], red2[8];
    // The GEMM launched after this kernel may start (its weight loads do not
    // depend on this kernel); this kernel itself waits for its predecessor.
    pdl_launch_dependents();
    pdl_wait_primary();
    // split-K tile counters of the GEMM that follows start at zero
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ncount; i += gridDim.x * blockDim.x) tcount[i] = 0u;
    const int ld = act.ld > 0 ? act.ld : K;
    const int Mr = act.rows_dev ? min(M, max(0, *act.rows_dev)) : M;
    for (int row = blockIdx.x; row < Mr; row += gridDim.x) {
        const float* xr = X + static_cast<int64_t>(row) * ld;
        const float* rr = act.R ? act.R + static_cast<int64_t>(row) * K : nullptr;
        float* so = act.sum_out ? act.sum_out + static_cast<int64_t>(row) * K : nullptr;
        float mx = 0.f, ss = 0.f;
        for (int k = 4 * threadIdx.x; k < K; k += 4 * blockDim.x) {
            float4 x;
            const float4 v = act4<VEC>(act, xr, rr, K, k, x);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            if (act.kind == 1) {
                ss = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, fmaf(x.w, x.w, ss))));
                if (so) {
                    if (VEC) *reinterpret_cast<float4*>(so + k) = x;
                    else { so[k] = x.x; so[k + 1] = x.y; so[k + 2] = x.z; so[k + 3] = x.w; }
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            ss += __shfl_xor_sync(0xffffffffu, ss, o);
        }
        if ((threadIdx.x & 31) == 0) {
            red[threadIdx.x >> 5] = mx;
            red2[threadIdx.x >> 5] = ss;
        }
        __syncthreads();
        mx = red[0];
        ss = red2[0];
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
            mx = fmaxf(mx, red[w]);
            ss += red2[w];
        }
        int k = 0;
        if (mx > 0.f && mx <= 3.402823466e38f) k = max(((__float_as_int(mx) >> 23) & 0xFF) - 127 - 14, -100);
        const float sc = __int_as_float((127 - k) << 23);  // 2^-k
        if (threadIdx.x == 0) {
            float rs = __int_as_float((127 + k) << 23);
            if (act.kind == 1) rs *= 1.0f / sqrtf(ss / static_cast<float>(K) + act.eps);
            rowscale[row] = rs;
        }
        for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
            const int p0 = c * 8;
            const int g = p0 & ~255, pp = p0 & 255;
            int e0 = g + tc::tc_elem(F2, pp), e1 = g + tc::tc_elem(F2, pp + 4);
            if (q2ref) {  // Q2_K, reference CPU order: all four planes of a half read x[half + l], l < 32
                e0 = (e0 & ~127) | (e0 & 31);
                e1 = (e1 & ~127) | (e1 & 31);
            }
            float4 x;
            const float4 a = act4<VEC>(act, xr, rr, K, e0, x);
            const float4 b = act4<VEC>(act, xr, rr, K, e1, x);
            uint4 o;
            o.x = tc::pack_h2(a.x * sc, a.y * sc);
            o.y = tc::pack_h2(a.z * sc, a.w * sc);
            o.z = tc::pack_h2(b.x * sc, b.y * sc);
            o.w = tc::pack_h2(b.z * sc, b.w * sc);
            *reinterpret_cast<uint4*>(Xh + static_cast<int64_t>(row) * K + p0) = o;
        }
        __syncthreads();  // red is reused by the next row
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

using EncodeTiledFn2 = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn2() {
    static EncodeTiledFn2 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn2>(f);
    });
    return fn;
}

bool gemm_tc_supported(int type, const void* W, int M, int N, int K, int refcpu) {
    if (tc::tc_fmt(type).qk == 0 || M <= 0 || N <= 0 || K <= 0 || K % 32 != 0) return false;
    // Shared-memory reads of the staged blocks are 2-byte aligned at least.
    if (reinterpret_cast<uintptr_t>(W) % 2 != 0) return false;
    return encode_fn2() != nullptr;
}

// Shared memory of one launch: A/B ring of `stages`, W ring of `wstages`.
// Shared memory of one launch: A/B ring of `stages`, W ring of `wstages`,
// barriers, and `extra` bytes after them (the grouped tile table).
static size_t tc_smem_bytes(int bn, int stages, int wstages, int wp, size_t extra) {
    const size_t bars = static_cast<size_t>(3 * stages + 2 * wstages + 5) * 8 + 8;
    return 1024 + static_cast<size_t>(stages) * (tc::A_STAGE + bn * tc::BK * 2) +
           static_cast<size_t>(wstages) * tc::BM * wp + 16 + bars + extra;
}

// Experts of a grouped launch (device arrays).
struct ExpertSet {
    const uint8_t* const* wptrs;
    const int* offsets;
    int n_experts;
    const uint8_t* w_all = nullptr;  // stacked experts (wptrs unused)
};

// M is the number of X rows (grouped: all experts' rows together).
static std::atomic<int> g_early_prefetch{1};
void gemm_tc_set_early_prefetch(int on) { g_early_prefetch = on ? 1 : 0; }

// Split-K plan of a dense call and its scratch (part: ksplit x M x N floats,
// tcount: 4 counters per output tile).
struct SplitK {
    int ksplit = 1, gps = 0;
    float* part = nullptr;
    unsigned* tcount = nullptr;
};

static int token_tile(int M) { return M <= 64 ? 64 : M <= 128 ? 128 : 256; }

// Output tiles fewer than half the SMs: split K so that about one work unit
// lands on every SM, each unit at least two W stages (512 K), at most
// TC_MAX_SPLIT parts.
static SplitK plan_split(int M, int N, int K, int num_sms) {
    SplitK sk;
    const int tiles = ((M + token_tile(M) - 1) / token_tile(M)) * ((N + tc::BM - 1) / tc::BM);
    const int ngroups = (K + tc::KG - 1) / tc::KG;
    sk.gps = ngroups;
    if (2 * tiles > num_sms) return sk;
    int S = std::min({tc::TC_MAX_SPLIT, num_sms / tiles, ngroups / 2});
    if (S <= 1) return sk;
    sk.gps = (ngroups + S - 1) / S;
    sk.ksplit = (ngroups + sk.gps - 1) / sk.gps;
    return sk;
}
static size_t split_tiles(int M, int N) {
    return static_cast<size_t>((M + token_tile(M) - 1) / token_tile(M)) * ((N + tc::BM - 1) / tc::BM);
}

template <int T, int BN, bool A4, bool G>
static cudaError_t launch_tc(const void* W, const __half* Xh, const float* rowscale, float* Y, int M, int N, int K,
                             int num_sms, cudaStream_t stream, const ExpertSet* ex, const SplitK& sk = SplitK{}) {
    constexpr tc::TcFmt F = tc::tc_fmt(T);
    tc::Params p{};
    p.W = static_cast<const uint8_t*>(W);
    p.Y = Y;
    p.rowscale = rowscale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.nblocks = K / F.qk;
    p.row_bytes = p.nblocks * F.bb;
    p.n_mtiles = (M + BN - 1) / BN;
    p.n_ntiles = (N + tc::BM - 1) / tc::BM;
    p.ksteps = (K + tc::BK - 1) / tc::BK;
    p.ngroups = (K + tc::KG - 1) / tc::KG;
    const uintptr_t w = reinterpret_cast<uintptr_t>(W);
    const bool stacked = G && ex->w_all != nullptr;
    const int wrows = stacked ? ex->n_experts * N : N;  // rows of the weight tensor map
    const size_t wbytes = static_cast<size_t>(wrows) * p.row_bytes;
    p.w_lo = reinterpret_cast<const uint8_t*>(w & ~uintptr_t(15));
    p.w_hi = reinterpret_cast<const uint8_t*>((w + wbytes + 15) & ~uintptr_t(15));
    size_t extra = 0;
    p.early = g_early_prefetch.load(std::memory_order_relaxed);
    p.ksplit = G ? 1 : sk.ksplit;
    p.gps = G || sk.ksplit == 1 ? p.ngroups : sk.gps;
    p.part = sk.part;
    p.tcount = sk.tcount;
    int max_tiles = p.n_mtiles * p.n_ntiles * p.ksplit;
    if constexpr (G) {
        p.wptrs = ex->wptrs;
        p.offsets = ex->offsets;
        p.n_experts = ex->n_experts;
        p.rows_total = M;
        p.stacked = stacked ? 1 : 0;
        extra = static_cast<size_t>(ex->n_experts + 1) * sizeof(int);
        // each expert adds at most one partial token tile
        max_tiles = static_cast<int>(std::min<int64_t>(
            INT32_MAX, static_cast<int64_t>(p.n_ntiles) * ((M + BN - 1) / BN + ex->n_experts)));
    }

    // One 2-D tensor-map copy per W stage needs 16-byte aligned rows; otherwise
    // (and always for grouped launches, whose expert weights are separate
    // allocations) one bulk copy per row from the 16-byte boundary at or below
    // the row's data.
    bool tmap = (!G || stacked) && (w % 16 == 0) && (p.row_bytes % 16 == 0);
    for (int attempt = 0; attempt < 2; ++attempt) {
        const bool offs = !tmap || (F.gbytes % 16 != 0);  // data may start up to 15 bytes into a smem row
        int wp = (F.gbytes + (offs ? 15 : 0) + 15) / 16 * 16;
        if ((wp / 16) % 2 == 0) wp += 16;  // odd multiple of 16: conflict-free across 8 rows
        p.wp = wp;
        p.rows_mode = tmap ? 0 : 1;

        // Deepest A/B ring that fits beside three W stages (two if three leave
        // fewer than three A/B stages).
        p.stages = 0;
        for (int sw : {3, 2}) {
            for (int st = 8; st >= 2; --st) {
                if (tc_smem_bytes(BN, st, sw, wp, extra) <= 227 * 1024) {
                    p.stages = st;
                    p.wstages = sw;
                    break;
                }
            }
            if (p.stages >= 3) break;
        }
        if (p.stages == 0) return cudaErrorInvalidConfiguration;

        CUtensorMap wmap;
        std::memset(&wmap, 0, sizeof(wmap));
        if (tmap) {
            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.row_bytes / 2), static_cast<cuuint64_t>(wrows)};
            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.row_bytes)};
            const cuuint32_t box[2] = {static_cast<cuuint32_t>(wp / 2), static_cast<cuuint32_t>(tc::BM)};
            const cuuint32_t estr[2] = {1, 1};
            CUresult r = encode_fn2()(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(W), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) {
                tmap = false;  // per-row copies need no tensor map
                continue;
            }
        }

        CUtensorMap xmap;
        std::memset(&xmap, 0, sizeof(xmap));
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(tc::BK), static_cast<cuuint32_t>(BN)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = encode_fn2()(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(Xh), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;

        auto kern = tc::gemm_kernel<T, BN, A4, G>;
        static thread_local int set_dev = -1;
        int dev = -1;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev != set_dev) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            if (e != cudaSuccess) return e;
            set_dev = dev;
        }
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(std::max(1, std::min(max_tiles, num_sms)));
        cfg.blockDim = dim3(tc::THREADS);
        cfg.dynamicSmemBytes = tc_smem_bytes(BN, p.stages, p.wstages, p.wp, extra);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, p, xmap, wmap);
    }
    return cudaErrorInvalidValue;
}

template <int T, bool A4>
static cudaError_t launch_tc_bn(const void* W, const __half* Xh, const float* rs, float* Y, int M, int N, int K,
                                int num_sms, cudaStream_t s, const SplitK& sk) {
    if (M <= 64) return launch_tc<T, 64, A4, false>(W, Xh, rs, Y, M, N, K, num_sms, s, nullptr, sk);
    if (M <= 128) return launch_tc<T, 128, A4, false>(W, Xh, rs, Y, M, N, K, num_sms, s, nullptr, sk);
    return launch_tc<T, 256, A4, false>(W, Xh, rs, Y, M, N, K, num_sms, s, nullptr, sk);
}

// Grouped: the token tile follows the mean rows per expert.  Stacked experts
// (one tensor, expert e at rows e*N ..) load each W stage with one tensor-map
// box; separate expert matrices with one bulk copy per row.
template <int T, bool A4>
static cudaError_t launch_tc_grouped_a(const ExpertSet& ex, const __half* Xh, const float* rs, float* Y, int rows,
                                       int N, int K, int num_sms, cudaStream_t s, int mean) {
    const void* W = ex.w_all;
    if (mean <= 64) return launch_tc<T, 64, A4, true>(W, Xh, rs, Y, rows, N, K, num_sms, s, &ex);
    if (mean <= 128) return launch_tc<T, 128, A4, true>(W, Xh, rs, Y, rows, N, K, num_sms, s, &ex);
    return launch_tc<T, 256, A4, true>(W, Xh, rs, Y, rows, N, K, num_sms, s, &ex);
}

template <int T>
static cudaError_t launch_tc_grouped(const ExpertSet& ex, const __half* Xh, const float* rs, float* Y, int rows,
                                     int N, int K, int num_sms, cudaStream_t s, int mean_rows) {
    const int mean = mean_rows > 0 ? mean_rows : (rows + ex.n_experts - 1) / ex.n_experts;
    // Q4_K, Q5_K and Q2_K keep every field of a block 4-byte aligned when W is.
    if constexpr (T == Q4_K || T == Q5_K || T == Q2_K) {
        if (ex.w_all != nullptr && reinterpret_cast<uintptr_t>(ex.w_all) % 4 == 0)
            return launch_tc_grouped_a<T, true>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean);
    }
    return launch_tc_grouped_a<T, false>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean);
}

template <int T>
static cudaError_t launch_tc_fmt(const void* W, const __half* Xh, const float* rs, float* Y, int M, int N, int K,
                                 int num_sms, cudaStream_t s, const SplitK& sk) {
    // Q4_K, Q5_K and Q2_K keep every field of a block 4-byte aligned when W is.
    if constexpr (T == Q4_K || T == Q5_K || T == Q2_K) {
        if (reinterpret_cast<uintptr_t>(W) % 4 == 0)
            return launch_tc_bn<T, true>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
    }
    return launch_tc_bn<T, false>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
}

template <bool F2>
static cudaError_t launch_x_to_f16(const float* X, __half* Xh, float* rowscale, int M, int K, int num_sms,
                                   cudaStream_t s, unsigned* tcount = nullptr, int ncount = 0,
                                   const ActArgs& act = ActArgs{}, int q2ref = 0) {
    const int grid = std::max(1, std::min(M, num_sms * 8));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool vec = al(X) && al(act.R) && al(act.normw) && al(act.sum_out) && (act.ld <= 0 || act.ld % 4 == 0);
    if (vec)
        return cudaLaunchKernelEx(&cfg, x_to_f16_kernel<F2, true>, X, Xh, rowscale, M, K, tcount, ncount, act, q2ref);
    return cudaLaunchKernelEx(&cfg, x_to_f16_kernel<F2, false>, X, Xh, rowscale, M, K, tcount, ncount, act, q2ref);
}

static size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

// Scratch of one call: the fp16 copy of X (M*K halves), M row scales, then
// for a split-K plan the tile counters and the partial products.
static size_t scratch_bytes(int64_t M, int64_t K) { return static_cast<size_t>(M * K) * 2 + static_cast<size_t>(M) * 4; }
static size_t scratch_bytes(int64_t M, int64_t N, int64_t K, const SplitK& sk) {
    size_t b = align16(scratch_bytes(M, K));
    if (sk.ksplit > 1)
        b += align16(split_tiles(static_cast<int>(M), static_cast<int>(N)) * 4 * sizeof(unsigned)) +
             static_cast<size_t>(sk.ksplit) * M * N * sizeof(float);
    return b;
}
// Points sk.tcount and sk.part into the scratch at `base` laid out as above.
static void place_split(SplitK& sk, void* base, int64_t M, int64_t N, int64_t K) {
    if (sk.ksplit <= 1) return;
    uint8_t* b = static_cast<uint8_t*>(base) + align16(scratch_bytes(M, K));
    sk.tcount = reinterpret_cast<unsigned*>(b);
    sk.part = reinterpret_cast<float*>(b + align16(split_tiles(static_cast<int>(M), static_cast<int>(N)) * 4 *
                                                   sizeof(unsigned)));
}

// X -> fp16 into Xh (M*K halves, K order of the format) with row scales rs
// (M floats) and the split-K counters zeroed, then the GEMM.
static cudaError_t gemm_tc_run(int type, const void* W, const float* X, __half* Xh, float* rs, float* Y, int M,
                               int N, int K, int num_sms, cudaStream_t s, const SplitK& sk, const ActArgs& act,
                               int refcpu) {
    const int ncount = sk.ksplit > 1 ? static_cast<int>(split_tiles(M, N) * 4) : 0;
    const int q2ref = (type == Q2_K && refcpu) ? 1 : 0;
    cudaError_t e = tc::tc_fmt(type).f2
                        ? launch_x_to_f16<true>(X, Xh, rs, M, K, num_sms, s, sk.tcount, ncount, act, q2ref)
                        : launch_x_to_f16<false>(X, Xh, rs, M, K, num_sms, s, sk.tcount, ncount, act, q2ref);
    if (e != cudaSuccess) return e;
    switch (type) {
        case Q4_0: return launch_tc_fmt<Q4_0>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
        case Q8_0: return launch_tc_fmt<Q8_0>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
        case Q2_K: return launch_tc_fmt<Q2_K>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
        case Q3_K: return launch_tc_fmt<Q3_K>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
        case Q4_K: return launch_tc_fmt<Q4_K>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
        case Q5_K: return launch_tc_fmt<Q5_K>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
        case Q6_K: return launch_tc_fmt<Q6_K>(W, Xh, rs, Y, M, N, K, num_sms, s, sk);
        default: return cudaErrorInvalidValue;
    }
}

// Stream-ordered pool of the current device for the fp16 copy of X.  The pool
// belongs to libswq and keeps freed memory for the next call (release threshold
// = unlimited), so a call costs no trip to the driver's allocator once the
// largest scratch has been seen.
static cudaError_t scratch_pool(cudaMemPool_t* out) {
    static std::mutex mu;
    static std::map<int, cudaMemPool_t> pools;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    auto it = pools.find(dev);
    if (it == pools.end()) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        if ((e = cudaMemPoolCreate(&pool, &props)) != cudaSuccess) return e;
        uint64_t keep = UINT64_MAX;
        if ((e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep)) != cudaSuccess) return e;
        it = pools.emplace(dev, pool).first;
    }
    *out = it->second;
    return cudaSuccess;
}

cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
    cudaMemPool_t pool = nullptr;
    cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    return cudaMallocFromPoolAsync(p, bytes, pool, s);
}

cudaError_t scratch_free(void* p, cudaStream_t s) { return cudaFreeAsync(p, s); }

cudaError_t gemm_tc_launch(int type, const void* W, const float* X, float* Y, int M, int N, int K, int refcpu,
                           int num_sms, cudaStream_t s, const ActArgs& act) {
    if (!gemm_tc_supported(type, W, M, N, K, refcpu)) return cudaErrorNotSupported;
    const int64_t n = static_cast<int64_t>(M) * K;
    cudaMemPool_t pool = nullptr;
    cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    SplitK sk = plan_split(M, N, K, num_sms);
    __half* Xh = nullptr;
    e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&Xh), scratch_bytes(M, N, K, sk), pool, s);
    if (e != cudaSuccess) return e;
    place_split(sk, Xh, M, N, K);
    e = gemm_tc_run(type, W, X, Xh, reinterpret_cast<float*>(Xh + n), Y, M, N, K, num_sms, s, sk, act, refcpu);
    cudaError_t e2 = cudaFreeAsync(Xh, s);
    return e != cudaSuccess ? e : e2;
}

// Workspace of one call from the caller (swq_gemm_act_ws): the same layout as
// the pool allocation above -- fp16 X, row scales, split-K counters and
// partials -- so each caller (e.g. each decoder) owns its scratch and calls on
// different workspaces never share memory.
size_t gemm_tc_workspace_bytes(int M, int N, int K, int num_sms) {
    return scratch_bytes(M, N, K, plan_split(M, N, K, num_sms));
}

cudaError_t gemm_tc_launch_ws(int type, const void* W, const float* X, float* Y, int M, int N, int K, int refcpu,
                              int num_sms, cudaStream_t s, const ActArgs& act, void* ws, size_t ws_bytes) {
    if (!gemm_tc_supported(type, W, M, N, K, refcpu)) return cudaErrorNotSupported;
    SplitK sk = plan_split(M, N, K, num_sms);
    if (ws == nullptr || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0 || ws_bytes < scratch_bytes(M, N, K, sk))
        return cudaErrorInvalidValue;
    __half* Xh = static_cast<__half*>(ws);
    place_split(sk, Xh, M, N, K);
    return gemm_tc_run(type, W, X, Xh, reinterpret_cast<float*>(Xh + static_cast<int64_t>(M) * K), Y, M, N, K,
                       num_sms, s, sk, act, refcpu);
}

cudaError_t gemm_tc_grouped_launch(int type, const void* const* wptrs, const int* offsets, const float* X, float* Y,
                                   int n_experts, int rows, int N, int K, int refcpu, int num_sms, cudaStream_t s,
                                   int mean_rows, const int* live_rows, const void* w_all) {
    if (tc::tc_fmt(type).qk == 0 || K % 32 != 0 || encode_fn2() == nullptr) return cudaErrorNotSupported;
    const int64_t n = static_cast<int64_t>(rows) * K;
    cudaMemPool_t pool = nullptr;
    cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    __half* Xh = nullptr;
    e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&Xh), scratch_bytes(rows, K), pool, s);
    if (e != cudaSuccess) return e;
    float* rs = reinterpret_cast<float*>(Xh + n);
    const int q2ref = (type == Q2_K && refcpu) ? 1 : 0;
    ActArgs act;
    act.rows_dev = live_rows;
    e = tc::tc_fmt(type).f2 ? launch_x_to_f16<true>(X, Xh, rs, rows, K, num_sms, s, nullptr, 0, act, q2ref)
                            : launch_x_to_f16<false>(X, Xh, rs, rows, K, num_sms, s, nullptr, 0, act, q2ref);
    if (e == cudaSuccess) {
        const ExpertSet ex{reinterpret_cast<const uint8_t* const*>(wptrs), offsets, n_experts,
                           static_cast<const uint8_t*>(w_all)};
        switch (type) {
            case Q4_0: e = launch_tc_grouped<Q4_0>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean_rows); break;
            case Q8_0: e = launch_tc_grouped<Q8_0>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean_rows); break;
            case Q2_K: e = launch_tc_grouped<Q2_K>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean_rows); break;
            case Q3_K: e = launch_tc_grouped<Q3_K>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean_rows); break;
            case Q4_K: e = launch_tc_grouped<Q4_K>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean_rows); break;
            case Q5_K: e = launch_tc_grouped<Q5_K>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean_rows); break;
            case Q6_K: e = launch_tc_grouped<Q6_K>(ex, Xh, rs, Y, rows, N, K, num_sms, s, mean_rows); break;
            default: e = cudaErrorInvalidValue;
        }
    }
    cudaError_t e2 = cudaFreeAsync(Xh, s);
    return e != cudaSuccess ? e : e2;
}

// ---------------------------------------------------------------------------
// Allocation-free variant (swq_gemm_noalloc).  Callers whose process already
// owns the GPU's memory through its own allocator (a serving engine that
// reserves HBM for its KV cache at start-up, a caching allocator that hands
// out every device byte) cannot let this library take a temporary buffer from
// a stream-ordered pool of its own.  For them the fp16 copy of X lives in this fixed array,
// which every GPU that loads libswq holds until the process exits.  In host
// code `g_noalloc_x16` only names the array; its address on a device comes
// from cudaGetSymbolAddress with that device current, looked up once per
// device on that device's first call.  All calls on a device share the array:
// calls whose kernels overlap on the GPU race.  Each call writes every element
// it reads (the tensor map stops at M x K, and M row scales), so nothing needs
// clearing.
// ---------------------------------------------------------------------------

static __device__ __align__(256) uint16_t g_noalloc_x16[SWQ_GEMM_NOALLOC_MAX_X_ELEMS];
// one scale per X row; K >= 32, so M <= SWQ_GEMM_NOALLOC_MAX_X_ELEMS / 32
static __device__ __align__(256) float g_noalloc_rowscale[SWQ_GEMM_NOALLOC_MAX_X_ELEMS / 32];
// split-K partial products and tile counters (a call whose plan does not fit
// runs unsplit)
constexpr size_t NOALLOC_PART_ELEMS = size_t(1) << 22;
constexpr size_t NOALLOC_TCOUNT = 4096;
static __device__ __align__(256) float g_noalloc_part[NOALLOC_PART_ELEMS];
static __device__ __align__(256) unsigned g_noalloc_tcount[NOALLOC_TCOUNT];

struct NoallocArrays {
    void* x16;
    void* rowscale;
    void* part;
    void* tcount;
};

static cudaError_t noalloc_scratch(NoallocArrays* out) {
    static std::mutex mu;
    static std::map<int, NoallocArrays> addr;  // device -> device addresses of the arrays
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    auto it = addr.find(dev);
    if (it == addr.end()) {
        NoallocArrays a{};
        if ((e = cudaGetSymbolAddress(&a.x16, g_noalloc_x16)) != cudaSuccess) return e;
        if ((e = cudaGetSymbolAddress(&a.rowscale, g_noalloc_rowscale)) != cudaSuccess) return e;
        if ((e = cudaGetSymbolAddress(&a.part, g_noalloc_part)) != cudaSuccess) return e;
        if ((e = cudaGetSymbolAddress(&a.tcount, g_noalloc_tcount)) != cudaSuccess) return e;
        it = addr.emplace(dev, a).first;
    }
    *out = it->second;
    return cudaSuccess;
}

cudaError_t gemm_tc_launch_noalloc(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                                   int refcpu, int num_sms, cudaStream_t s, const ActArgs& act) {
    if (!gemm_tc_supported(type, W, M, N, K, refcpu)) return cudaErrorNotSupported;
    if (static_cast<int64_t>(M) * K > SWQ_GEMM_NOALLOC_MAX_X_ELEMS) return cudaErrorInvalidValue;
    NoallocArrays a{};
    cudaError_t e = noalloc_scratch(&a);
    if (e != cudaSuccess) return e;
    SplitK sk = plan_split(M, N, K, num_sms);
    if (sk.ksplit > 1 && (static_cast<size_t>(sk.ksplit) * M * N > NOALLOC_PART_ELEMS ||
                          split_tiles(M, N) * 4 > NOALLOC_TCOUNT)) {
        sk = SplitK{};
        sk.gps = (K + tc::KG - 1) / tc::KG;
    }
    if (sk.ksplit > 1) {
        sk.part = static_cast<float*>(a.part);
        sk.tcount = static_cast<unsigned*>(a.tcount);
    }
    return gemm_tc_run(type, W, X, static_cast<__half*>(a.x16), static_cast<float*>(a.rowscale), Y, M, N, K,
                       num_sms, s, sk, act, refcpu);
}

SWQ_DEFINE_STATUS_FETCH(gemm_tc)

}  // namespace swq
