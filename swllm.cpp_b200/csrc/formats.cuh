// formats.cuh -- GGUF block formats on the quantized-weight path.
//
// For each format two views of the same block layout:
//
//  * dq_elem(): one element exactly as the reference dequantizer computes it
//    (src/tensor.h:139-432), fp32 with explicit round-to-nearest mul/sub so no
//    FMA contraction changes a bit.  Used by swq_dequant (bit-exact).
//
//  * unit decode for the fused GEMV: a block is split into UPB "units" of UE
//    elements (one lane's work).  decode() turns a unit's quant bits into
//    UE/4 words of four small integers (bytes, unsigned unless QSIGNED).  A
//    unit has PARTS parts; part p covers the PE consecutive block elements
//    starting at part_elem0(c, p), held in words p*WPP .. p*WPP+WPP-1 in
//    element order, and shares one weight scale and one 32-element activation
//    block.  A part's bytes may hold the quant value times a power of two
//    (e.g. a high nibble left in place, x16); wd then carries the inverse
//    factor and ioff(p) (the integer zero point) is in the same scaled units.
//    Activations are 16-bit fixed point, so the dot product is a chain of
//    dp2a instructions:
//        contribution = xs * (wd * (S - ioff(p) * I) - wm * I)
//    with S = sum(q * X) and I = sum(X) over the part.
#pragma once

#include <cuda_fp16.h>

#include "swq_device.cuh"

namespace swq {

// ---- helpers --------------------------------------------------------------------

// get_scale_min_k4 (src/tensor.h:218-227) on the 12-byte field held as three
// little-endian words s0 = bytes 0-3, s1 = bytes 4-7, s2 = bytes 8-11.
__device__ __forceinline__ void scale_min_k4(int j, uint32_t s0, uint32_t s1, uint32_t s2,
                                             uint32_t& sc, uint32_t& m) {
    if (j < 4) {
        sc = byte_of(s0, j) & 63u;
        m = byte_of(s1, j) & 63u;
    } else {
        const int jj = j - 4;
        sc = (byte_of(s2, jj) & 0x0Fu) | ((byte_of(s0, jj) >> 6) << 4);
        m = (byte_of(s2, jj) >> 4) | ((byte_of(s1, jj) >> 6) << 4);
    }
}

// The same for sub-block j = 2c + t (t = 0, 1) without a branch on c, so
// lanes that hold different units of a block do not diverge.
__device__ __forceinline__ void scale_min_k4_unit(int c, int t, uint32_t s0, uint32_t s1, uint32_t s2,
                                                  uint32_t& sc, uint32_t& m) {
    const uint32_t pos = 8u * ((2 * c + t) & 3);
    const uint32_t a0 = __funnelshift_r(s0, 0u, pos) & 0xFFu;  // byte of s0
    const uint32_t a1 = __funnelshift_r(s1, 0u, pos) & 0xFFu;
    const uint32_t a2 = __funnelshift_r(s2, 0u, pos) & 0xFFu;
    const bool hi = c >= 2;
    sc = hi ? ((a2 & 0x0Fu) | ((a0 >> 6) << 4)) : (a0 & 63u);
    m = hi ? ((a2 >> 4) | ((a1 >> 6) << 4)) : (a1 & 63u);
}

// get_scale_min_k4 for sub-blocks 2c and 2c + 1 of a unit, as floats: all 8
// 6-bit scales and mins of the block are assembled bytewise from the 12-byte
// field (s0, s1, s2) in a few word operations, and each selected byte becomes
// an exact float through the low mantissa of 2^23.
__device__ __forceinline__ void scale_min_k4_pair(int c, uint32_t s0, uint32_t s1, uint32_t s2, float& sc0,
                                                  float& m0, float& sc1, float& m1) {
    const uint32_t scl = s0 & 0x3F3F3F3Fu, mnl = s1 & 0x3F3F3F3Fu;  // sub-blocks 0..3
    const uint32_t sch = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);  // 4..7
    const uint32_t mnh = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    const uint32_t SC = c < 2 ? scl : sch, MN = c < 2 ? mnl : mnh;
    const uint32_t sel0 = 0x7650u + ((2 * c) & 3), sel1 = sel0 + 1;
    sc0 = __uint_as_float(__byte_perm(SC, 0x4B000000u, sel0)) - 8388608.0f;
    sc1 = __uint_as_float(__byte_perm(SC, 0x4B000000u, sel1)) - 8388608.0f;
    m0 = __uint_as_float(__byte_perm(MN, 0x4B000000u, sel0)) - 8388608.0f;
    m1 = __uint_as_float(__byte_perm(MN, 0x4B000000u, sel1)) - 8388608.0f;
}

// Q3_K signed scales, src/tensor.h:286-304: word w (0..3) of the unpacked
// 16 scales, each word reduced by 0x20202020 as a whole (byte borrows kept).
__device__ __forceinline__ uint32_t q3k_scale_word(int w, uint32_t t0, uint32_t t1, uint32_t t2) {
    const uint32_t km = 0x03030303u;
    const uint32_t ta = (w < 2) ? t0 : t1;
    const int sh_lo = (w & 1) ? 2 : 0;
    const int sh_hi = 2 * w;
    return ((((ta >> sh_lo) & km) | (((t2 >> sh_hi) & km) << 4))) - 0x20202020u;
}

__device__ __forceinline__ uint32_t ldg_u8(const uint8_t* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t ldg_u16(const uint8_t* p) {
    return static_cast<uint32_t>(__ldg(p)) | (static_cast<uint32_t>(__ldg(p + 1)) << 8);
}

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }

// Hardware fp16 -> fp32 (exact for every finite value); the GEMV's scales.
__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half(static_cast<unsigned short>(bits))); }

template <int T>
struct Fmt;

// =============================================================================
// Q4_0: 32 elements, 18 bytes: d (f16) @0, 16 nibble bytes @2.  src/tensor.h:139
// element j <- low nibble of byte j, element j+16 <- high nibble; value - 8.
// One unit = the block; part 0 = elements 0..15, part 1 = 16..31 (high
// nibbles kept in place, x16).
// =============================================================================
template <>
struct Fmt<Q4_0> {
    static constexpr int QK = 32, BB = 18, UPB = 1, UE = 32, PARTS = 2, PE = 16;
    static constexpr bool MIN = false, QSIGNED = false;
    __host__ __device__ static constexpr int ioff(int p) { return p == 0 ? 8 : 128; }

    __device__ static float dq_elem(const uint8_t* b, int k) {
        const float d = half_bits_to_float(ldg_u16(b));
        const uint32_t v = ldg_u8(b + 2 + (k & 15));
        const int q = (k < 16) ? static_cast<int>(v & 0x0F) : static_cast<int>(v >> 4);
        return fmul(static_cast<float>(q - 8), d);
    }
    __host__ __device__ static int part_elem0(int, int p, bool) { return 16 * p; }
    // 8-element item at block element kk -> (unit, part, chunk in part)
    __host__ __device__ static int item_dest(int kk, bool, int& c, int& p, int& j) {
        c = 0; p = kk >> 4; j = (kk >> 3) & 1; return 1;
    }

    __device__ static void decode(const uint8_t* b, int, uint32_t (&q)[UE / 4], float (&wd)[PARTS],
                                  float (&wm)[PARTS]) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = lds_u32_a2(b + 2 + 4 * i);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            q[i] = w[i] & 0x0F0F0F0Fu;
            q[4 + i] = w[i] & 0xF0F0F0F0u;
        }
        const float d = h2f(*reinterpret_cast<const uint16_t*>(b));
        wd[0] = d;
        wd[1] = d * 0.0625f;
        wm[0] = wm[1] = 0.f;
    }
};

// =============================================================================
// Q8_0: 32 elements, 34 bytes: d @0, 32 x int8 @2.  src/tensor.h:157
// =============================================================================
template <>
struct Fmt<Q8_0> {
    static constexpr int QK = 32, BB = 34, UPB = 1, UE = 32, PARTS = 1, PE = 32;
    static constexpr bool MIN = false, QSIGNED = true;
    __host__ __device__ static constexpr int ioff(int) { return 0; }

    __device__ static float dq_elem(const uint8_t* b, int k) {
        const float d = half_bits_to_float(ldg_u16(b));
        const int q = static_cast<int8_t>(ldg_u8(b + 2 + k));
        return fmul(static_cast<float>(q), d);
    }
    __host__ __device__ static int part_elem0(int, int, bool) { return 0; }
    __host__ __device__ static int item_dest(int kk, bool, int& c, int& p, int& j) {
        c = 0; p = 0; j = kk >> 3; return 1;
    }

    __device__ static void decode(const uint8_t* b, int, uint32_t (&q)[UE / 4], float (&wd)[PARTS],
                                  float (&wm)[PARTS]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = lds_u32_a2(b + 2 + 4 * i);  // signed bytes
        wd[0] = h2f(*reinterpret_cast<const uint16_t*>(b));
        wm[0] = 0.f;
    }
};

// =============================================================================
// Q2_K: 256 elements, 84 bytes: scales[16] @0, qs[64] @16, d @80, dmin @82.
// src/tensor.h:232-265.  Element 128n + 32j + 16h + l <- (qs[32n + 16h + l] >> 2j) & 3,
// scale byte sc[8n + 2j + h] (low nibble: scale, high nibble: min).
// Unit c = (n = c>>1, h = c&1): 64 elements; part j = the 16 elements of
// plane j, its 2-bit values left in place (x 4^j).
// =============================================================================
template <>
struct Fmt<Q2_K> {
    static constexpr int QK = 256, BB = 84, UPB = 4, UE = 64, PARTS = 4, PE = 16;
    static constexpr bool MIN = true, QSIGNED = false;
    __host__ __device__ static constexpr int ioff(int) { return 0; }

    __device__ static float dq_elem(const uint8_t* b, int k) {
        const int n = k >> 7, r = k & 127, j = r >> 5, h = (r >> 4) & 1, l = r & 15;
        const float d = half_bits_to_float(ldg_u16(b + 80));
        const float dmin = half_bits_to_float(ldg_u16(b + 82));
        const uint32_t s = ldg_u8(b + 8 * n + 2 * j + h);
        const float dl = fmul(d, static_cast<float>(s & 0xF));
        const float ml = fmul(dmin, static_cast<float>(s >> 4));
        const uint32_t v = (ldg_u8(b + 16 + 32 * n + 16 * h + l) >> (2 * j)) & 3u;
        return fsub(fmul(dl, static_cast<float>(v)), ml);
    }
    // Part j of unit c holds block elements 128n + 32j + 16h .. +15 (format
    // order).  In the reference-CPU order (cpu_matmul_transposed_q2_k,
    // src/tensor.h:935-945) every plane j reads activations 128n + 16h .. +15.
    __host__ __device__ static int part_elem0(int c, int j, bool refcpu) {
        return 128 * (c >> 1) + (refcpu ? 0 : 32 * j) + 16 * (c & 1);
    }
    // Reference-CPU order: the item feeds parts 0..3 of its unit (or nothing).
    __host__ __device__ static int item_dest(int kk, bool refcpu, int& c, int& p, int& j) {
        const int n = kk >> 7, r = kk & 127;
        c = 2 * n + ((r >> 4) & 1);
        j = (r >> 3) & 1;
        if (!refcpu) { p = r >> 5; return 1; }
        p = 0;
        return r < 32 ? 4 : 0;
    }
    __device__ static void decode(const uint8_t* b, int c, uint32_t (&q)[UE / 4], float (&wd)[PARTS],
                                  float (&wm)[PARTS]) {
        const int n = c >> 1, h = c & 1;
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = lds_u32_a4(b + 16 + 32 * n + 16 * h + 4 * i);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) q[4 * j + i] = w[i] & (0x03030303u << (2 * j));
        const uint32_t s_lo = lds_u32_a4(b + 8 * n);      // sc[8n .. 8n+3]
        const uint32_t s_hi = lds_u32_a4(b + 8 * n + 4);  // sc[8n+4 .. 8n+7]
        const uint32_t dd = lds_u32_a4(b + 80);
        const float d = h2f(dd & 0xFFFFu);
        const float dmin = h2f(dd >> 16);
        constexpr float inv4[4] = {1.0f, 0.25f, 0.0625f, 0.015625f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t s = byte_of(j < 2 ? s_lo : s_hi, 2 * (j & 1) + h);
            wd[j] = d * static_cast<float>(s & 0xF) * inv4[j];
            wm[j] = dmin * static_cast<float>(s >> 4);
        }
    }
};

// =============================================================================
// Q3_K: 256 elements, 110 bytes: hmask[32] @0, qs[64] @32, scales[12] @96, d @108.
// src/tensor.h:269-326.  Element 128n + 32j + 16h + l:
//   v = ((qs[32n + 16h + l] >> 2j) & 3) - (hmask[16h + l] bit (4n + j) ? 0 : 4),
//   scale = scales_i8[8n + 2j + h].
// Decoded as u = q2 | hbit << 2 in 0..7 with zero point 4.
// =============================================================================
template <>
struct Fmt<Q3_K> {
    static constexpr int QK = 256, BB = 110, UPB = 4, UE = 64, PARTS = 4, PE = 16;
    static constexpr bool MIN = false, QSIGNED = false;
    __host__ __device__ static constexpr int ioff(int) { return 4; }

    __device__ static float dq_elem(const uint8_t* b, int k) {
        const int n = k >> 7, r = k & 127, j = r >> 5, h = (r >> 4) & 1, l = r & 15;
        const float d = half_bits_to_float(ldg_u16(b + 108));
        uint32_t t[3];
#pragma unroll
        for (int i = 0; i < 3; ++i)
            t[i] = ldg_u16(b + 96 + 4 * i) | (ldg_u16(b + 98 + 4 * i) << 16);
        const int idx = 8 * n + 2 * j + h;
        const uint32_t sw = q3k_scale_word(idx >> 2, t[0], t[1], t[2]);
        const int sc = static_cast<int8_t>(byte_of(sw, idx & 3));
        const float dl = fmul(d, static_cast<float>(sc));
        const int q2 = static_cast<int>((ldg_u8(b + 32 + 32 * n + 16 * h + l) >> (2 * j)) & 3u);
        const int hb = (ldg_u8(b + 16 * h + l) >> (4 * n + j)) & 1;
        return fmul(dl, static_cast<float>(q2 - (hb ? 0 : 4)));
    }
    __host__ __device__ static int part_elem0(int c, int j, bool) { return 128 * (c >> 1) + 32 * j + 16 * (c & 1); }
    __host__ __device__ static int item_dest(int kk, bool, int& c, int& p, int& j) {
        const int n = kk >> 7, r = kk & 127;
        c = 2 * n + ((r >> 4) & 1); p = r >> 5; j = (r >> 3) & 1; return 1;
    }

    __device__ static void decode(const uint8_t* b, int c, uint32_t (&q)[UE / 4], float (&wd)[PARTS],
                                  float (&wm)[PARTS]) {
        const int n = c >> 1, h = c & 1;
        uint32_t w[4], hm[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[i] = lds_u32_a2(b + 32 + 32 * n + 16 * h + 4 * i);
            hm[i] = lds_u32_a2(b + 16 * h + 4 * i) >> (4 * n);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                q[4 * j + i] = ((w[i] >> (2 * j)) & 0x03030303u) | (((hm[i] >> j) & 0x01010101u) << 2);
        const uint32_t t0 = lds_u32_a2(b + 96), t1 = lds_u32_a2(b + 100), t2 = lds_u32_a2(b + 104);
        const float d = h2f(*reinterpret_cast<const uint16_t*>(b + 108));
        const uint32_t a_lo = q3k_scale_word(2 * n, t0, t1, t2);      // scales 8n .. 8n+3
        const uint32_t a_hi = q3k_scale_word(2 * n + 1, t0, t1, t2);  // scales 8n+4 .. 8n+7
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int s = static_cast<int8_t>(byte_of(j < 2 ? a_lo : a_hi, 2 * (j & 1) + h));
            wd[j] = d * static_cast<float>(s);
            wm[j] = 0.f;
        }
    }
};

// =============================================================================
// Q4_K: 256 elements, 144 bytes: d @0, dmin @2, scales[12] @4, qs[128] @16.
// src/tensor.h:329-358.  64-group g: elements 64g + l (l<32) <- qs[32g+l] & 15
// with (sc, m) pair 2g; elements 64g + 32 + l <- qs[32g+l] >> 4 with pair 2g+1.
// Unit c = group g: part 0 = low nibbles, part 1 = high nibbles kept in place
// (x16).
// =============================================================================
template <>
struct Fmt<Q4_K> {
    static constexpr int QK = 256, BB = 144, UPB = 4, UE = 64, PARTS = 2, PE = 32;
    static constexpr bool MIN = true, QSIGNED = false;
    __host__ __device__ static constexpr int ioff(int) { return 0; }

    __device__ static float dq_elem(const uint8_t* b, int k) {
        const int g = k >> 6, r = k & 63, hi = r >> 5, l = r & 31;
        const float d = half_bits_to_float(ldg_u16(b));
        const float dmin = half_bits_to_float(ldg_u16(b + 2));
        uint32_t s[3];
#pragma unroll
        for (int i = 0; i < 3; ++i)
            s[i] = ldg_u16(b + 4 + 4 * i) | (ldg_u16(b + 6 + 4 * i) << 16);
        uint32_t sc, m;
        scale_min_k4(2 * g + hi, s[0], s[1], s[2], sc, m);
        const float d1 = fmul(d, static_cast<float>(sc));
        const float m1 = fmul(dmin, static_cast<float>(m));
        const uint32_t v = ldg_u8(b + 16 + 32 * g + l);
        const uint32_t qv = hi ? (v >> 4) : (v & 0xF);
        return fsub(fmul(d1, static_cast<float>(qv)), m1);
    }
    __host__ __device__ static int part_elem0(int c, int p, bool) { return 64 * c + 32 * p; }
    __host__ __device__ static int item_dest(int kk, bool, int& c, int& p, int& j) {
        c = kk >> 6; p = (kk >> 5) & 1; j = (kk >> 3) & 3; return 1;
    }

    __device__ static void decode(const uint8_t* b, int c, uint32_t (&q)[UE / 4], float (&wd)[PARTS],
                                  float (&wm)[PARTS]) {
        const uint4 hd = lds_u128(b);
        const uint4 a = lds_u128(b + 16 + 32 * c);
        const uint4 a2 = lds_u128(b + 32 + 32 * c);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, a2.x, a2.y, a2.z, a2.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            q[i] = w[i] & 0x0F0F0F0Fu;
            q[8 + i] = w[i] & 0xF0F0F0F0u;
        }
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hd.x));
        float sc0, m0, sc1, m1;
        scale_min_k4_pair(c, hd.y, hd.z, hd.w, sc0, m0, sc1, m1);
        wd[0] = dm.x * sc0;
        wm[0] = dm.y * m0;
        wd[1] = dm.x * sc1 * 0.0625f;
        wm[1] = dm.y * m1;
    }
};

// =============================================================================
// Q5_K: 256 elements, 176 bytes: d @0, dmin @2, scales[12] @4, qh[32] @16,
// qs[128] @48.  src/tensor.h:361-395.  As Q4_K plus a fifth bit:
// element 64g + l gets +16 when qh[l] bit 2g is set, 64g + 32 + l when bit 2g+1.
// =============================================================================
template <>
struct Fmt<Q5_K> {
    static constexpr int QK = 256, BB = 176, UPB = 4, UE = 64, PARTS = 2, PE = 32;
    static constexpr bool MIN = true, QSIGNED = false;
    __host__ __device__ static constexpr int ioff(int) { return 0; }

    __device__ static float dq_elem(const uint8_t* b, int k) {
        const int g = k >> 6, r = k & 63, hi = r >> 5, l = r & 31;
        const float d = half_bits_to_float(ldg_u16(b));
        const float dmin = half_bits_to_float(ldg_u16(b + 2));
        uint32_t s[3];
#pragma unroll
        for (int i = 0; i < 3; ++i)
            s[i] = ldg_u16(b + 4 + 4 * i) | (ldg_u16(b + 6 + 4 * i) << 16);
        uint32_t sc, m;
        scale_min_k4(2 * g + hi, s[0], s[1], s[2], sc, m);
        const float d1 = fmul(d, static_cast<float>(sc));
        const float m1 = fmul(dmin, static_cast<float>(m));
        const uint32_t v = ldg_u8(b + 48 + 32 * g + l);
        const uint32_t hb = (ldg_u8(b + 16 + l) >> (2 * g + hi)) & 1u;
        const uint32_t qv = (hi ? (v >> 4) : (v & 0xF)) + (hb ? 16u : 0u);
        return fsub(fmul(d1, static_cast<float>(qv)), m1);
    }
    __host__ __device__ static int part_elem0(int c, int p, bool) { return 64 * c + 32 * p; }
    __host__ __device__ static int item_dest(int kk, bool, int& c, int& p, int& j) {
        c = kk >> 6; p = (kk >> 5) & 1; j = (kk >> 3) & 3; return 1;
    }

    __device__ static void decode(const uint8_t* b, int c, uint32_t (&q)[UE / 4], float (&wd)[PARTS],
                                  float (&wm)[PARTS]) {
        const uint4 hd = lds_u128(b);
        const uint4 h0 = lds_u128(b + 16);
        const uint4 h1 = lds_u128(b + 32);
        const uint4 a = lds_u128(b + 48 + 32 * c);
        const uint4 a2 = lds_u128(b + 64 + 32 * c);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, a2.x, a2.y, a2.z, a2.w};
        const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t hb = qh[i] >> (2 * c);
            q[i] = (w[i] & 0x0F0F0F0Fu) | ((hb & 0x01010101u) << 4);
            q[8 + i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | ((hb & 0x02020202u) << 3);
        }
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hd.x));
        float sc0, m0, sc1, m1;
        scale_min_k4_pair(c, hd.y, hd.z, hd.w, sc0, m0, sc1, m1);
        wd[0] = dm.x * sc0;
        wm[0] = dm.y * m0;
        wd[1] = dm.x * sc1;
        wm[1] = dm.y * m1;
    }
};

// =============================================================================
// Q6_K: 256 elements, 210 bytes: ql[128] @0, qh[64] @128, int8 scales[16] @192,
// d @208.  src/tensor.h:398-432.  Half n, l in 0..31, plane k in 0..3:
//   element 128n + 32k + l, 6-bit value from ql[64n + l (+32 for k odd)]
//   (low nibble for k<2, high for k>=2) and bits 2k..2k+1 of qh[32n + l],
//   minus 32; scale sc[8n + l/16 + 2k].
// Unit c = (n = c>>1, h = c&1): l = 16h .. 16h+15, part k = plane k.
// =============================================================================
template <>
struct Fmt<Q6_K> {
    static constexpr int QK = 256, BB = 210, UPB = 4, UE = 64, PARTS = 4, PE = 16;
    static constexpr bool MIN = false, QSIGNED = false;
    __host__ __device__ static constexpr int ioff(int) { return 32; }

    __device__ static float dq_elem(const uint8_t* b, int k) {
        const int n = k >> 7, r = k & 127, kk = r >> 5, l = r & 31, is = l >> 4;
        const float d = half_bits_to_float(ldg_u16(b + 208));
        const uint32_t lo = ldg_u8(b + 64 * n + l + ((kk & 1) ? 32 : 0));
        const uint32_t hh = ldg_u8(b + 128 + 32 * n + l);
        const uint32_t nib = (kk < 2) ? (lo & 0xF) : (lo >> 4);
        const int qv = static_cast<int>(nib | (((hh >> (2 * kk)) & 3u) << 4)) - 32;
        const int sc = static_cast<int8_t>(ldg_u8(b + 192 + 8 * n + is + 2 * kk));
        return fmul(fmul(d, static_cast<float>(sc)), static_cast<float>(qv));
    }
    __host__ __device__ static int part_elem0(int c, int k, bool) { return 128 * (c >> 1) + 32 * k + 16 * (c & 1); }
    __host__ __device__ static int item_dest(int kk, bool, int& c, int& p, int& j) {
        const int n = kk >> 7, r = kk & 127;
        c = 2 * n + ((r >> 4) & 1); p = r >> 5; j = (r >> 3) & 1; return 1;
    }

    __device__ static void decode(const uint8_t* b, int c, uint32_t (&q)[UE / 4], float (&wd)[PARTS],
                                  float (&wm)[PARTS]) {
        const int n = c >> 1, h = c & 1;
        uint32_t A[4], B[4], H[4];
        // 16-byte runs at 2-byte aligned addresses (210-byte blocks); the last
        // run ends at byte 192 of the block, so the extra word stays inside it
        lds_u32x4_a2(b + 64 * n + 16 * h, A);
        lds_u32x4_a2(b + 64 * n + 32 + 16 * h, B);
        lds_u32x4_a2(b + 128 + 32 * n + 16 * h, H);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            q[i] = (A[i] & 0x0F0F0F0Fu) | ((H[i] << 4) & 0x30303030u);
            q[4 + i] = (B[i] & 0x0F0F0F0Fu) | ((H[i] << 2) & 0x30303030u);
            q[8 + i] = ((A[i] >> 4) & 0x0F0F0F0Fu) | (H[i] & 0x30303030u);
            q[12 + i] = ((B[i] >> 4) & 0x0F0F0F0Fu) | ((H[i] >> 2) & 0x30303030u);
        }
        const float d = h2f(*reinterpret_cast<const uint16_t*>(b + 208));
        const uint32_t s_lo = lds_u32_a2(b + 192 + 8 * n);      // sc[8n .. 8n+3]
        const uint32_t s_hi = lds_u32_a2(b + 192 + 8 * n + 4);  // sc[8n+4 .. 8n+7]
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            // scale index 8n + h + 2k
            const int s = static_cast<int8_t>(byte_of(k < 2 ? s_lo : s_hi, 2 * (k & 1) + h));
            wd[k] = d * static_cast<float>(s);
            wm[k] = 0.f;
        }
    }
};

}  // namespace swq
