// gemm_tc.cu -- tensor-core dequant-GEMM for prefill-sized M (sm_100a, tcgen05).
//
// Y[M x N] = X[M x K] . W[N x K]^T with W in GGUF blocks, X and Y fp32.  The
// reference has no batched quantized path (its prefill is one
// Compute::matmul_transposed_q per token, src/main.cpp:284-287 ->
// src/tensor.h:1212); this kernel is the M-rows-at-once form of it.
//
// Per CTA (persistent, one per SM), output tile = 128 W rows x BN tokens:
//   warp 0      TMA producer for the activation tiles (X converted to fp16 once,
//               128-byte swizzled K-major boxes of 64 K x BN tokens); TMEM owner.
//   warp 1      MMA issuer: one lane runs tcgen05.mma.cta_group::1.kind::f16
//               (M = 128, N = BN, K = 16) into an fp32 TMEM accumulator.
//   warps 2-5   W producers: thread i owns W row i of the tile; per 64-element
//               K step it reads that row's GGUF bytes (L2 prefetch a few blocks
//               ahead, one step of register double-buffering), dequantizes to
//               fp16 and stores the 128-byte swizzled K-major A operand.
//   warps 6-9   epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = W rows), coalesced fp32 stores of Y.
// Accumulators are double-buffered in TMEM (2 x BN columns) so the epilogue of
// one tile overlaps the MMAs of the next.  Every wait is bounded; on timeout the
// kernel records it, drains what it issued and frees its TMEM.  Every copy lands
// in the issuing CTA only.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
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
constexpr int BK = 64;        // K elements per stage (one 128-byte swizzle atom of fp16)
constexpr int THREADS = 320;  // 10 warps
constexpr int A_STAGE = BM * BK * 2;  // 16 KB

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

__device__ __forceinline__ void tma_load_2d_nohint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// ---- dequantization of one 64-element K step of one row into fp16 ----------
//
// raw<T>: the bytes a K step needs, loaded from global memory one step ahead;
// emit<T>: eight 16-byte chunks (8 fp16 each) in K order.  Values are the
// reference's element values computed in fp32 and rounded once to fp16.

template <int T>
struct Step;

__device__ __forceinline__ uint32_t g_u32_a4(const uint8_t* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }
__device__ __forceinline__ uint32_t g_u32_a2(const uint8_t* p) {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
    return static_cast<uint32_t>(__ldg(q)) | (static_cast<uint32_t>(__ldg(q + 1)) << 16);
}
__device__ __forceinline__ uint4 g_u128(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

template <>
struct Step<Q4_K> {
    static constexpr int QK = 256, BB = 144;
    struct Raw { uint4 hd, a, b; };
    // row_ptr: start of the row; k0: first element of the step (multiple of 64)
    __device__ static void load(Raw& r, const uint8_t* row, int k0) {
        const uint8_t* blk = row + (k0 >> 8) * BB;
        const int g = (k0 >> 6) & 3;
        r.hd = g_u128(blk);
        r.a = g_u128(blk + 16 + 32 * g);
        r.b = g_u128(blk + 32 + 32 * g);
    }
    __device__ static void emit(const Raw& r, int k0, uint4 (&out)[8]) {
        const int g = (k0 >> 6) & 3;
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&r.hd.x));
        uint32_t sc0, m0, sc1, m1;
        scale_min_k4_unit(g, 0, r.hd.y, r.hd.z, r.hd.w, sc0, m0);
        scale_min_k4_unit(g, 1, r.hd.y, r.hd.z, r.hd.w, sc1, m1);
        const float d1 = dm.x * static_cast<float>(sc0), n1 = -dm.y * static_cast<float>(m0);
        const float d2 = dm.x * static_cast<float>(sc1), n2 = -dm.y * static_cast<float>(m1);
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const bool hi = c >= 4;
            const uint32_t w0 = w[2 * (c & 3)], w1 = w[2 * (c & 3) + 1];
            const float dd = hi ? d2 : d1, nn = hi ? n2 : n1;
            const int sh = hi ? 4 : 0;
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t ww = i < 2 ? w0 : w1;
                const int b0 = 8 * (2 * (i & 1)) + sh, b1 = 8 * (2 * (i & 1) + 1) + sh;
                const float q0 = static_cast<float>((ww >> b0) & 15u), q1 = static_cast<float>((ww >> b1) & 15u);
                o[i] = pack_h2(fmaf(dd, q0, nn), fmaf(dd, q1, nn));
            }
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};

template <>
struct Step<Q5_K> {
    static constexpr int QK = 256, BB = 176;
    struct Raw { uint4 hd, a, b, h0, h1; };
    __device__ static void load(Raw& r, const uint8_t* row, int k0) {
        const uint8_t* blk = row + (k0 >> 8) * BB;
        const int g = (k0 >> 6) & 3;
        r.hd = g_u128(blk);
        r.h0 = g_u128(blk + 16);
        r.h1 = g_u128(blk + 32);
        r.a = g_u128(blk + 48 + 32 * g);
        r.b = g_u128(blk + 64 + 32 * g);
    }
    __device__ static void emit(const Raw& r, int k0, uint4 (&out)[8]) {
        const int g = (k0 >> 6) & 3;
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&r.hd.x));
        uint32_t sc0, m0, sc1, m1;
        scale_min_k4_unit(g, 0, r.hd.y, r.hd.z, r.hd.w, sc0, m0);
        scale_min_k4_unit(g, 1, r.hd.y, r.hd.z, r.hd.w, sc1, m1);
        const float d1 = dm.x * static_cast<float>(sc0), n1 = -dm.y * static_cast<float>(m0);
        const float d2 = dm.x * static_cast<float>(sc1), n2 = -dm.y * static_cast<float>(m1);
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
        const uint32_t h[8] = {r.h0.x, r.h0.y, r.h0.z, r.h0.w, r.h1.x, r.h1.y, r.h1.z, r.h1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const bool hi = c >= 4;
            const int wi = 2 * (c & 3);
            const float dd = hi ? d2 : d1, nn = hi ? n2 : n1;
            const int sh = hi ? 4 : 0, hb = 2 * g + (hi ? 1 : 0);
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t ww = w[wi + (i >> 1)], hh = h[wi + (i >> 1)];
                const int e0 = 2 * (i & 1), e1 = e0 + 1;  // byte within the word
                const uint32_t v0 = ((ww >> (8 * e0 + sh)) & 15u) | (((hh >> (8 * e0 + hb)) & 1u) << 4);
                const uint32_t v1 = ((ww >> (8 * e1 + sh)) & 15u) | (((hh >> (8 * e1 + hb)) & 1u) << 4);
                o[i] = pack_h2(fmaf(dd, static_cast<float>(v0), nn), fmaf(dd, static_cast<float>(v1), nn));
            }
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};

template <>
struct Step<Q6_K> {
    static constexpr int QK = 256, BB = 210;
    // 64 elements = half n, planes 2(g&1) and 2(g&1)+1: ql[64n .. 64n+63],
    // qh[32n .. 32n+31], scales sc[8n .. 8n+7], d.
    struct Raw { uint32_t ql[16], qh[8], s0, s1, d; };
    __device__ static void load(Raw& r, const uint8_t* row, int k0) {
        const uint8_t* blk = row + (k0 >> 8) * BB;
        const int n = (k0 >> 7) & 1;
#pragma unroll
        for (int i = 0; i < 16; ++i) r.ql[i] = g_u32_a2(blk + 64 * n + 4 * i);
#pragma unroll
        for (int i = 0; i < 8; ++i) r.qh[i] = g_u32_a2(blk + 128 + 32 * n + 4 * i);
        r.s0 = g_u32_a2(blk + 192 + 8 * n);
        r.s1 = g_u32_a2(blk + 196 + 8 * n);
        r.d = static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(blk + 208)));
    }
    __device__ static void emit(const Raw& r, int k0, uint4 (&out)[8]) {
        const int g = (k0 >> 6) & 3;
        const int kkb = 2 * (g & 1);  // first plane
        const float d = h2f(r.d);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int kk = kkb + (c >> 2);     // plane
            const int l0 = 8 * (c & 3);        // l of the first element
            const int is = l0 >> 4;
            const int sidx = is + 2 * kk;      // 0..7 within sc[8n ..]
            const int s = static_cast<int8_t>(byte_of(sidx < 4 ? r.s0 : r.s1, sidx & 3));
            const float ds = d * static_cast<float>(s);
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float v[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int l = l0 + 2 * i + e;
                    const int qb = l + 32 * (kk & 1);
                    const uint32_t qlb = byte_of(r.ql[qb >> 2], qb & 3);
                    const uint32_t nib = kk < 2 ? (qlb & 15u) : (qlb >> 4);
                    const uint32_t hb = (byte_of(r.qh[l >> 2], l & 3) >> (2 * kk)) & 3u;
                    v[e] = ds * static_cast<float>(static_cast<int>(nib | (hb << 4)) - 32);
                }
                o[i] = pack_h2(v[0], v[1]);
            }
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};

template <>
struct Step<Q2_K> {
    static constexpr int QK = 256, BB = 84;
    // 64 elements = half n, planes 2(g&1), 2(g&1)+1: qs[32n .. 32n+31],
    // sc[8n .. 8n+7], d, dmin.
    struct Raw { uint32_t qs[8], s0, s1, dd; };
    __device__ static void load(Raw& r, const uint8_t* row, int k0) {
        const uint8_t* blk = row + (k0 >> 8) * BB;
        const int n = (k0 >> 7) & 1;
#pragma unroll
        for (int i = 0; i < 8; ++i) r.qs[i] = g_u32_a4(blk + 16 + 32 * n + 4 * i);
        r.s0 = g_u32_a4(blk + 8 * n);
        r.s1 = g_u32_a4(blk + 8 * n + 4);
        r.dd = g_u32_a4(blk + 80);
    }
    __device__ static void emit(const Raw& r, int k0, uint4 (&out)[8]) {
        const int g = (k0 >> 6) & 3;
        const int jb = 2 * (g & 1);
        const float d = h2f(r.dd & 0xFFFFu), dmin = h2f(r.dd >> 16);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int j = jb + (c >> 2);
            const int e0 = 8 * (c & 3);  // 0..31 within the plane: h = e0 >> 4
            const int h = e0 >> 4;
            const uint32_t s = byte_of((2 * j + h) < 4 ? r.s0 : r.s1, (2 * j + h) & 3);
            const float dl = d * static_cast<float>(s & 15u), nl = -dmin * static_cast<float>(s >> 4);
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int b0 = e0 + 2 * i;  // qs byte index within the 32 (16h + l)
                const uint32_t v0 = (byte_of(r.qs[b0 >> 2], b0 & 3) >> (2 * j)) & 3u;
                const uint32_t v1 = (byte_of(r.qs[(b0 + 1) >> 2], (b0 + 1) & 3) >> (2 * j)) & 3u;
                o[i] = pack_h2(fmaf(dl, static_cast<float>(v0), nl), fmaf(dl, static_cast<float>(v1), nl));
            }
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};

template <>
struct Step<Q3_K> {
    static constexpr int QK = 256, BB = 110;
    struct Raw { uint32_t qs[8], hm[8], t0, t1, t2, d; };
    __device__ static void load(Raw& r, const uint8_t* row, int k0) {
        const uint8_t* blk = row + (k0 >> 8) * BB;
        const int n = (k0 >> 7) & 1;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            r.qs[i] = g_u32_a2(blk + 32 + 32 * n + 4 * i);
            r.hm[i] = g_u32_a2(blk + 4 * i);
        }
        r.t0 = g_u32_a2(blk + 96);
        r.t1 = g_u32_a2(blk + 100);
        r.t2 = g_u32_a2(blk + 104);
        r.d = static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(blk + 108)));
    }
    __device__ static void emit(const Raw& r, int k0, uint4 (&out)[8]) {
        const int g = (k0 >> 6) & 3;
        const int n = g >> 1, jb = 2 * (g & 1);
        const float d = h2f(r.d);
        const uint32_t a_lo = q3k_scale_word(2 * n, r.t0, r.t1, r.t2);
        const uint32_t a_hi = q3k_scale_word(2 * n + 1, r.t0, r.t1, r.t2);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int j = jb + (c >> 2);
            const int e0 = 8 * (c & 3), h = e0 >> 4;
            const int si = 2 * j + h;  // scale index within 8n ..
            const int s = static_cast<int8_t>(byte_of(si < 4 ? a_lo : a_hi, si & 3));
            const float dl = d * static_cast<float>(s);
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float v[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int b = e0 + 2 * i + e;  // 16h + l
                    const int q2 = (byte_of(r.qs[b >> 2], b & 3) >> (2 * j)) & 3;
                    const int hb = (byte_of(r.hm[b >> 2], b & 3) >> (4 * n + j)) & 1;
                    v[e] = dl * static_cast<float>(q2 - (hb ? 0 : 4));
                }
                o[i] = pack_h2(v[0], v[1]);
            }
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};

template <>
struct Step<Q8_0> {
    static constexpr int QK = 32, BB = 34;
    // two blocks (elements k0 .. k0+63); the second may lie past K (valid = 0)
    struct Raw { uint32_t q[16], d0, d1; };
    __device__ static void load(Raw& r, const uint8_t* row, int k0, int K) {
        const uint8_t* b0 = row + (k0 >> 5) * BB;
#pragma unroll
        for (int i = 0; i < 8; ++i) r.q[i] = g_u32_a2(b0 + 2 + 4 * i);
        r.d0 = static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(b0)));
        if (k0 + 32 < K) {
            const uint8_t* b1 = b0 + BB;
#pragma unroll
            for (int i = 0; i < 8; ++i) r.q[8 + i] = g_u32_a2(b1 + 2 + 4 * i);
            r.d1 = static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(b1)));
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) r.q[8 + i] = 0;
            r.d1 = 0;
        }
    }
    __device__ static void emit(const Raw& r, int, uint4 (&out)[8]) {
        const float d0 = h2f(r.d0), d1 = h2f(r.d1);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float d = c < 4 ? d0 : d1;
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = r.q[2 * c + (i >> 1)];
                const int e = 2 * (i & 1);
                o[i] = pack_h2(d * static_cast<float>(static_cast<int8_t>(byte_of(w, e))),
                               d * static_cast<float>(static_cast<int8_t>(byte_of(w, e + 1))));
            }
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};

template <>
struct Step<Q4_0> {
    static constexpr int QK = 32, BB = 18;
    struct Raw { uint32_t q[8], d0, d1; };
    __device__ static void load(Raw& r, const uint8_t* row, int k0, int K) {
        const uint8_t* b0 = row + (k0 >> 5) * BB;
#pragma unroll
        for (int i = 0; i < 4; ++i) r.q[i] = g_u32_a2(b0 + 2 + 4 * i);
        r.d0 = static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(b0)));
        if (k0 + 32 < K) {
            const uint8_t* b1 = b0 + BB;
#pragma unroll
            for (int i = 0; i < 4; ++i) r.q[4 + i] = g_u32_a2(b1 + 2 + 4 * i);
            r.d1 = static_cast<uint32_t>(__ldg(reinterpret_cast<const uint16_t*>(b1)));
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) r.q[4 + i] = 0x88888888u;
            r.d1 = 0;
        }
    }
    __device__ static void emit(const Raw& r, int, uint4 (&out)[8]) {
        const float d0 = h2f(r.d0), d1 = h2f(r.d1);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            // chunk c: block c >> 2; within it elements 8(c&3) .. +7: low nibbles of
            // bytes 0..15 are elements 0..15, high nibbles elements 16..31
            const int blk = c >> 2, cc = c & 3;
            const float d = blk ? d1 : d0;
            const int sh = cc >= 2 ? 4 : 0;
            const int byte0 = 8 * (cc & 1);
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int b = byte0 + 2 * i;
                const uint32_t w0 = r.q[4 * blk + (b >> 2)], w1 = r.q[4 * blk + ((b + 1) >> 2)];
                const int q0 = static_cast<int>((byte_of(w0, b & 3) >> sh) & 15u) - 8;
                const int q1 = static_cast<int>((byte_of(w1, (b + 1) & 3) >> sh) & 15u) - 8;
                o[i] = pack_h2(d * static_cast<float>(q0), d * static_cast<float>(q1));
            }
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};

// Uniform load signature (the 32-element formats need K for a ragged last step).
template <int T>
__device__ __forceinline__ void step_load(typename Step<T>::Raw& r, const uint8_t* row, int k0, int K) {
    if constexpr (T == Q8_0 || T == Q4_0) Step<T>::load(r, row, k0, K);
    else Step<T>::load(r, row, k0);
}

struct Params {
    const uint8_t* W;
    float* Y;
    int M, N, K;
    int row_bytes;
    int n_mtiles, n_ntiles, ksteps;
    int stages;
};

struct Smem {
    uint32_t a_off, b_off, bar_off;
};

template <int T, int BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const Params p, const __grid_constant__ CUtensorMap xmap) {
    using S = Step<T>;
    constexpr int B_STAGE = BN * BK * 2;
    constexpr uint32_t IDESC = idesc_f16(BM, BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled operands
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S_ = p.stages;
    uint8_t* a_st = smem;                                   // S x 16 KB
    uint8_t* b_st = smem + S_ * A_STAGE;                    // S x B_STAGE
    uint64_t* bars = reinterpret_cast<uint64_t*>(b_st + S_ * B_STAGE);
    uint64_t* full_a = bars;              // [S] dequant warps (4 arrivals)
    uint64_t* full_b = bars + S_;         // [S] TMA tx
    uint64_t* empty = bars + 2 * S_;      // [S] MMA commit
    uint64_t* tfull = bars + 3 * S_;      // [2] MMA commit per tile
    uint64_t* tempty = bars + 3 * S_ + 2; // [2] epilogue (4 arrivals)
    uint64_t* drain = bars + 3 * S_ + 4;  // final MMA commit before TMEM is freed
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 3 * S_ + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * S_ + 5) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = p.n_mtiles * p.n_ntiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S_; ++s) {
            mbar_init(&full_a[s], 4);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&tfull[t], 1);
            mbar_init(&tempty[t], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        // 2 x BN fp32 columns of TMEM (double-buffered accumulator)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(const_cast<uint32_t*>(tmem_slot))), "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait_primary();  // X (fp16) is written by the conversion kernel before this one

    if (warp == 0) {
        // ------------------------------------------------ activation TMA producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int it = 0;  // loads issued
            for (int tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x) {
                const int mt = tile / p.n_ntiles;  // token tile
                for (int ks = 0; ks < p.ksteps; ++ks, ++it) {
                    if (it >= S_ && !mbar_wait_bounded(&empty[s], ph ^ 1u, DEV_TIMEOUT_EMPTY)) {
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_b[s], B_STAGE);
                    tma_load_2d_nohint(b_st + s * B_STAGE, &xmap, ks * BK, mt * BN, &full_b[s]);
                    if (++s == S_) { s = 0; ph ^= 1u; }
                }
            }
            // Wait for the last load issued into each stage, so that no copy is
            // still writing shared memory when the CTA exits (immediate unless a
            // wait above gave up).
            for (int i = 0; i < S_ && i < it; ++i) {
                const int idx = it - 1 - i;
                mbar_wait_bounded(&full_b[idx % S_], static_cast<uint32_t>(idx / S_) & 1u, DEV_TIMEOUT_DRAIN);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int t_local = 0;
            for (int tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x, ++t_local) {
                const int tb = t_local & 1;
                const uint32_t tph = (t_local >> 1) & 1;
                if (t_local >= 2 && !mbar_wait_bounded(&tempty[tb], tph ^ 1u, DEV_TIMEOUT_MMA)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t dt = tmem_base + static_cast<uint32_t>(tb * BN);
                bool okk = true;
                for (int ks = 0; ks < p.ksteps; ++ks) {
                    if (!mbar_wait_bounded(&full_a[s], ph, DEV_TIMEOUT_FULL) ||
                        !mbar_wait_bounded(&full_b[s], ph, DEV_TIMEOUT_FULL)) {
                        *abort_flag = 1;
                        okk = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = smem_desc_sw128(smem_u32(a_st + s * A_STAGE));
                    const uint64_t db = smem_desc_sw128(smem_u32(b_st + s * B_STAGE));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)  // 32 bytes of K per instruction
                        mma_f16(dt, da + 2 * k, db + 2 * k, IDESC, (ks | k) ? 1u : 0u);
                    mma_commit(&empty[s]);
                    if (++s == S_) { s = 0; ph ^= 1u; }
                }
                if (!okk) break;
                mma_commit(&tfull[tb]);
            }
            // One more commit tracks every MMA this thread issued: once it
            // arrives, no tensor-core write to TMEM is in flight.
            mma_commit(drain);
            mbar_wait_bounded(drain, 0u, DEV_TIMEOUT_DRAIN);
        }
    } else if (warp < 6) {
        // ------------------------------------------------------- W dequantizers
        const int r = threadIdx.x - 64;  // 0 .. 127: W row of the tile
        int s = 0;
        uint32_t ph = 0;
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            const int nt = tile % p.n_ntiles;
            const int row = nt * BM + r;
            const bool valid = row < p.N;
            const uint8_t* rowp = p.W + static_cast<size_t>(valid ? row : 0) * p.row_bytes;
            typename S::Raw cur, nxt;
            if (valid) step_load<T>(cur, rowp, 0, p.K);
            for (int ks = 0; ks < p.ksteps; ++ks, ++it) {
                const int k0 = ks * BK;
                // L2 prefetch of the block four blocks ahead (once per block)
                if (valid && ((k0 % S::QK) == 0 || S::QK < BK)) {
                    const int kpf = k0 + 4 * (S::QK > BK ? S::QK : BK);
                    if (kpf < p.K) {
                        const uint8_t* pf = rowp + static_cast<size_t>(kpf / S::QK) * S::BB;
                        prefetch_l2(pf);
                        if (S::BB > 128) prefetch_l2(pf + 128);  // still inside the block
                    }
                }
                if (valid && ks + 1 < p.ksteps) step_load<T>(nxt, rowp, k0 + BK, p.K);
                uint4 out[8];
                if (valid) {
                    S::emit(cur, k0, out);
                } else {
#pragma unroll
                    for (int c = 0; c < 8; ++c) out[c] = make_uint4(0, 0, 0, 0);
                }
                const bool got = it < S_ || mbar_wait_bounded(&empty[s], ph ^ 1u, DEV_TIMEOUT_EMPTY);
                if (!__all_sync(0xffffffffu, got)) {  // the warp leaves together
                    *abort_flag = 1;
                    break;
                }
                uint8_t* a = a_st + s * A_STAGE + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(a + ((c ^ (r & 7)) << 4)) = out[c];
                fence_async_shared();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full_a[s]);
                if (++s == S_) { s = 0; ph ^= 1u; }
                cur = nxt;
            }
        }
    } else {
        // -------------------------------------------------------------- epilogue
        const int q = warp & 3;        // TMEM lane quadrant
        const int r = 32 * q + lane;   // W row within the tile
        int t_local = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t_local) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            const int mt = tile / p.n_ntiles, nt = tile % p.n_ntiles;
            const int tb = t_local & 1;
            const uint32_t tph = (t_local >> 1) & 1;
            const bool got = mbar_wait_bounded(&tfull[tb], tph, DEV_TIMEOUT_MMA);
            if (!__all_sync(0xffffffffu, got)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int row = nt * BM + r;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(tb * BN);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tbase + c0, v);
                tmem_wait_ld();
                if (row < p.N) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int tok = mt * BN + c0 + j;
                        if (tok < p.M) p.Y[static_cast<size_t>(tok) * p.N + row] = __uint_as_float(v[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[tb]);
        }
    }

    // Teardown: every role has left its loop (all waits are bounded), the MMA
    // lane has seen its last commit and the TMA lane its last load.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * BN));
}

}  // namespace tc

// fp32 -> fp16 activations (row-major, same shape).
template <bool VEC>
__global__ void __launch_bounds__(256) x_to_f16_kernel(const float* __restrict__ X, __half* __restrict__ Xh,
                                                       int64_t n) {
    const int64_t n4 = n / 4;  // n is a multiple of 32
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 v;
        if (VEC) {
            v = reinterpret_cast<const float4*>(X)[i];
        } else {
            v.x = X[4 * i]; v.y = X[4 * i + 1]; v.z = X[4 * i + 2]; v.w = X[4 * i + 3];
        }
        __half2* o = reinterpret_cast<__half2*>(Xh) + 2 * i;
        o[0] = __floats2half2_rn(v.x, v.y);
        o[1] = __floats2half2_rn(v.z, v.w);
    }
    pdl_launch_dependents();
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

static int type_qk(int t) { return (t == Q4_0 || t == Q8_0) ? 32 : 256; }
static int type_bb(int t) {
    switch (t) {
        case Q4_0: return 18;
        case Q8_0: return 34;
        case Q2_K: return 84;
        case Q3_K: return 110;
        case Q4_K: return 144;
        case Q5_K: return 176;
        case Q6_K: return 210;
        default: return 0;
    }
}

bool gemm_tc_supported(int type, const void* W, int M, int N, int K, int refcpu) {
    if (type_bb(type) == 0 || M <= 0 || N <= 0 || K <= 0 || K % 32 != 0) return false;
    if (refcpu && type == Q2_K) return false;  // the GEMV kernel serves that activation order
    // Weight loads: 16-byte vectors for Q4_K/Q5_K, 4-byte words for Q2_K, 2-byte
    // halves otherwise; every row start keeps the base alignment.
    const uintptr_t w = reinterpret_cast<uintptr_t>(W);
    const uintptr_t need = (type == Q4_K || type == Q5_K) ? 16 : (type == Q2_K ? 4 : 2);
    if (w % need != 0) return false;
    return encode_fn2() != nullptr;
}

template <int T, int BN>
static cudaError_t launch_tc(const void* W, const __half* Xh, float* Y, int M, int N, int K, int num_sms,
                             cudaStream_t stream) {
    tc::Params p{};
    p.W = static_cast<const uint8_t*>(W);
    p.Y = Y;
    p.M = M;
    p.N = N;
    p.K = K;
    p.row_bytes = (K / type_qk(T)) * type_bb(T);
    p.n_mtiles = (M + BN - 1) / BN;
    p.n_ntiles = (N + tc::BM - 1) / tc::BM;
    p.ksteps = (K + tc::BK - 1) / tc::BK;
    constexpr int B_STAGE = BN * tc::BK * 2;
    const int per_stage = tc::A_STAGE + B_STAGE;
    int stages = (200 * 1024) / per_stage;
    stages = std::max(2, std::min(stages, 6));
    p.stages = stages;
    const size_t smem = 1024 + static_cast<size_t>(stages) * per_stage + (3 * stages + 5) * 8 + 16;

    CUtensorMap xmap;
    std::memset(&xmap, 0, sizeof(xmap));
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(tc::BK), static_cast<cuuint32_t>(BN)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn2()(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(Xh), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;

    auto kern = tc::gemm_kernel<T, BN>;
    static thread_local int set_dev = -1;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != set_dev) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        set_dev = dev;
    }
    const int ntiles = p.n_mtiles * p.n_ntiles;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(std::min(ntiles, num_sms));
    cfg.blockDim = dim3(tc::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, xmap);
}

template <int T>
static cudaError_t launch_tc_fmt(const void* W, const __half* Xh, float* Y, int M, int N, int K, int num_sms,
                                 cudaStream_t s) {
    if (M <= 64) return launch_tc<T, 64>(W, Xh, Y, M, N, K, num_sms, s);
    if (M <= 128) return launch_tc<T, 128>(W, Xh, Y, M, N, K, num_sms, s);
    return launch_tc<T, 256>(W, Xh, Y, M, N, K, num_sms, s);
}

// X -> fp16 into Xh (M*K halves), then the GEMM that reads Xh.
static cudaError_t gemm_tc_run(int type, const void* W, const float* X, __half* Xh, float* Y, int M, int N, int K,
                               int num_sms, cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(M) * K;
    const int64_t n4 = n / 4;
    const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(num_sms) * 8));
    if ((reinterpret_cast<uintptr_t>(X) & 15u) == 0)
        x_to_f16_kernel<true><<<std::max(grid, 1), 256, 0, s>>>(X, Xh, n);
    else
        x_to_f16_kernel<false><<<std::max(grid, 1), 256, 0, s>>>(X, Xh, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    switch (type) {
        case Q4_0: return launch_tc_fmt<Q4_0>(W, Xh, Y, M, N, K, num_sms, s);
        case Q8_0: return launch_tc_fmt<Q8_0>(W, Xh, Y, M, N, K, num_sms, s);
        case Q2_K: return launch_tc_fmt<Q2_K>(W, Xh, Y, M, N, K, num_sms, s);
        case Q3_K: return launch_tc_fmt<Q3_K>(W, Xh, Y, M, N, K, num_sms, s);
        case Q4_K: return launch_tc_fmt<Q4_K>(W, Xh, Y, M, N, K, num_sms, s);
        case Q5_K: return launch_tc_fmt<Q5_K>(W, Xh, Y, M, N, K, num_sms, s);
        case Q6_K: return launch_tc_fmt<Q6_K>(W, Xh, Y, M, N, K, num_sms, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemm_tc_launch(int type, const void* W, const float* X, float* Y, int M, int N, int K, int refcpu,
                           int num_sms, cudaStream_t s) {
    if (!gemm_tc_supported(type, W, M, N, K, refcpu)) return cudaErrorNotSupported;
    const int64_t n = static_cast<int64_t>(M) * K;
    __half* Xh = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&Xh), static_cast<size_t>(n) * 2, s);
    if (e != cudaSuccess) return e;
    e = gemm_tc_run(type, W, X, Xh, Y, M, N, K, num_sms, s);
    cudaError_t e2 = cudaFreeAsync(Xh, s);
    return e != cudaSuccess ? e : e2;
}

// ---------------------------------------------------------------------------
// Allocation-free variant (swq_gemm_noalloc).  Callers whose process already
// owns the GPU's memory through its own allocator (a serving engine that
// reserves HBM for its KV cache at start-up, a caching allocator that hands
// out every device byte) cannot let this library take a temporary buffer from
// cudaMallocAsync.  For them the fp16 copy of X lives in this fixed array,
// which every GPU that loads libswq holds until the process exits.  In host
// code `g_noalloc_x16` only names the array; its address on a device comes
// from cudaGetSymbolAddress with that device current, looked up once per
// device on that device's first call.  All calls on a device share the array:
// calls whose kernels overlap on the GPU race.  Each call writes every element
// it reads (the tensor map stops at M x K), so nothing needs clearing.
// ---------------------------------------------------------------------------

static __device__ __align__(256) uint16_t g_noalloc_x16[SWQ_GEMM_NOALLOC_MAX_X_ELEMS];

static cudaError_t noalloc_scratch(__half** out) {
    static std::mutex mu;
    static std::map<int, void*> addr;  // device -> device address of g_noalloc_x16
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    auto it = addr.find(dev);
    if (it == addr.end()) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_x16);
        if (e != cudaSuccess) return e;
        it = addr.emplace(dev, p).first;
    }
    *out = static_cast<__half*>(it->second);
    return cudaSuccess;
}

cudaError_t gemm_tc_launch_noalloc(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                                   int refcpu, int num_sms, cudaStream_t s) {
    if (!gemm_tc_supported(type, W, M, N, K, refcpu)) return cudaErrorNotSupported;
    if (static_cast<int64_t>(M) * K > SWQ_GEMM_NOALLOC_MAX_X_ELEMS) return cudaErrorInvalidValue;
    __half* Xh = nullptr;
    cudaError_t e = noalloc_scratch(&Xh);
    if (e != cudaSuccess) return e;
    return gemm_tc_run(type, W, X, Xh, Y, M, N, K, num_sms, s);
}

SWQ_DEFINE_STATUS_FETCH(gemm_tc)

}  // namespace swq
