/*
 * swq_oracle.c -- CPU restatement of swllm.cpp's quantized-weight path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle for the CUDA library
 * (libswq): only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load it.  The product path never calls it and there is no
 * CPU fallback built on it.
 *
 * Every function restates the reference algorithm in plain C, with the same
 * fp32 expression trees and the same accumulation order, so that compiled with
 * -O2 -ffp-contract=off (no FMA contraction, as the reference's own -O2
 * x86-64 build) the results are bit-identical to the reference's.  Parity of
 * this restatement is pinned two ways (tests/test_oracle.py):
 *   - the known-answer blocks of the reference's tests/test_gguf.cpp, and
 *   - golden vectors produced by the reference's own src/tensor.h compiled
 *     from source (oracle/Makefile -> oracle/_ref/), committed under
 *     tests/golden/.
 *
 * Reference citations are src/<file>:<line> inside the swllm.cpp project.
 */
#include <stdint.h>
#include <string.h>
#include <stddef.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* GGMLType ids, src/gguf.h:18-40 (only the formats on this path). */
enum {
    T_Q4_0 = 2, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11,
    T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14
};

/* bytes per block, src/gguf.h:60-86 */
size_t oracle_type_size(int type) {
    switch (type) {
        case T_Q4_0: return 18;
        case T_Q8_0: return 34;
        case T_Q2_K: return 84;
        case T_Q3_K: return 110;
        case T_Q4_K: return 144;
        case T_Q5_K: return 176;
        case T_Q6_K: return 210;
        default: return 0;
    }
}

/* elements per block, src/gguf.h:89-118 */
size_t oracle_block_size(int type) {
    switch (type) {
        case T_Q4_0: case T_Q8_0: return 32;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return 256;
        default: return 0;
    }
}

/* IEEE half -> float by bit manipulation, src/tensor.h:33-58.
 * Subnormals are renormalised; Inf/NaN keep their payload. */
float oracle_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            uint32_t ex = 1;
            while (!(mant & 0x400u)) { mant <<= 1; ex--; }
            mant &= 0x3FFu;
            bits = sign | ((ex + 127u - 15u) << 23) | (mant << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((e + 127u - 15u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float ld_half(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return oracle_fp16_to_fp32(h);
}

/* 6-bit scale/min pair j of the 12-byte K-quant scale field,
 * src/tensor.h:218-227. */
void oracle_get_scale_min_k4(int j, const uint8_t* s, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Q3_K 16 signed scales, src/tensor.h:286-304.  The four 32-bit words are
 * reduced by 0x20202020 as whole words, so a byte below 32 borrows from the
 * next byte; that borrow is part of the reference's result and is kept. */
void oracle_q3k_scales(const uint8_t* sc12, int8_t out[16]) {
    const uint32_t kmask1 = 0x03030303u;
    uint32_t t[3];
    memcpy(t, sc12, 12);
    uint32_t a0 = (t[0] & kmask1) | ((t[2] & kmask1) << 4);
    uint32_t a1 = ((t[0] >> 2) & kmask1) | (((t[2] >> 2) & kmask1) << 4);
    uint32_t a2 = (t[1] & kmask1) | (((t[2] >> 4) & kmask1) << 4);
    uint32_t a3 = ((t[1] >> 2) & kmask1) | (((t[2] >> 6) & kmask1) << 4);
    a0 -= 0x20202020u; a1 -= 0x20202020u; a2 -= 0x20202020u; a3 -= 0x20202020u;
    memcpy(out + 0, &a0, 4);
    memcpy(out + 4, &a1, 4);
    memcpy(out + 8, &a2, 4);
    memcpy(out + 12, &a3, 4);
}

/* ------------------------------------------------------------------------ */
/* Dequantizers                                                              */
/* ------------------------------------------------------------------------ */

/* src/tensor.h:139-154 */
static void dq_q4_0(const uint8_t* p, float* y, int64_t nb) {
    for (int64_t b = 0; b < nb; b++, p += 18, y += 32) {
        float d = ld_half(p);
        for (int j = 0; j < 16; j++) {
            uint8_t v = p[2 + j];
            y[j] = ((int)(v & 0x0F) - 8) * d;
            y[j + 16] = ((int)(v >> 4) - 8) * d;
        }
    }
}

/* src/tensor.h:157-170 */
static void dq_q8_0(const uint8_t* p, float* y, int64_t nb) {
    for (int64_t b = 0; b < nb; b++, p += 34, y += 32) {
        float d = ld_half(p);
        for (int j = 0; j < 32; j++) y[j] = (int8_t)p[2 + j] * d;
    }
}

/* src/tensor.h:232-265 */
static void dq_q2_k(const uint8_t* p, float* y, int64_t nb) {
    for (int64_t b = 0; b < nb; b++, p += 84) {
        const uint8_t* sc = p;
        const uint8_t* q = p + 16;
        float d = ld_half(p + 80), dmin = ld_half(p + 82);
        int is = 0;
        for (int n = 0; n < 256; n += 128) {
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                uint8_t s0 = sc[is++];
                float dl = d * (s0 & 0xF), ml = dmin * (s0 >> 4);
                for (int l = 0; l < 16; l++) *y++ = dl * ((q[l] >> shift) & 3) - ml;
                uint8_t s1 = sc[is++];
                dl = d * (s1 & 0xF); ml = dmin * (s1 >> 4);
                for (int l = 0; l < 16; l++) *y++ = dl * ((q[l + 16] >> shift) & 3) - ml;
                shift += 2;
                if (shift == 8) { shift = 0; q += 32; }
            }
        }
    }
}

/* src/tensor.h:269-326 */
static void dq_q3_k(const uint8_t* p, float* y, int64_t nb) {
    for (int64_t b = 0; b < nb; b++, p += 110, y += 256) {
        const uint8_t* hm = p;
        const uint8_t* q = p + 32;
        float d = ld_half(p + 108);
        int8_t s[16];
        oracle_q3k_scales(p + 96, s);
        uint8_t m = 1;
        for (int n = 0; n < 256; n += 128) {
            int off = (n == 0) ? 0 : 8;
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                float dl0 = d * s[off + 2 * j];
                float dl1 = d * s[off + 2 * j + 1];
                int base = n + 32 * j;
                for (int l = 0; l < 16; l++)
                    y[base + l] = dl0 * ((int)((q[l] >> shift) & 3) - ((hm[l] & m) ? 0 : 4));
                for (int l = 0; l < 16; l++)
                    y[base + 16 + l] = dl1 * ((int)((q[l + 16] >> shift) & 3) - ((hm[l + 16] & m) ? 0 : 4));
                shift += 2;
                if (shift == 8) { shift = 0; q += 32; }
                m <<= 1;
            }
        }
    }
}

/* src/tensor.h:329-358 */
static void dq_q4_k(const uint8_t* p, float* y, int64_t nb) {
    for (int64_t b = 0; b < nb; b++, p += 144, y += 256) {
        float d = ld_half(p), dmin = ld_half(p + 2);
        const uint8_t* s = p + 4;
        const uint8_t* qs = p + 16;
        int is = 0;
        for (int j = 0; j < 256; j += 64) {
            uint8_t sc, m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d1 = d * sc, m1 = dmin * m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d2 = d * sc, m2 = dmin * m;
            const uint8_t* q = qs + (j >> 1);
            for (int l = 0; l < 32; l++) y[j + l] = d1 * (q[l] & 0xF) - m1;
            for (int l = 0; l < 32; l++) y[j + l + 32] = d2 * (q[l] >> 4) - m2;
        }
    }
}

/* src/tensor.h:361-395 */
static void dq_q5_k(const uint8_t* p, float* y, int64_t nb) {
    for (int64_t b = 0; b < nb; b++, p += 176, y += 256) {
        float d = ld_half(p), dmin = ld_half(p + 2);
        const uint8_t* s = p + 4;
        const uint8_t* qh = p + 16;
        const uint8_t* ql = p + 48;
        int is = 0;
        uint8_t u1 = 1, u2 = 2;
        for (int j = 0; j < 256; j += 64) {
            uint8_t sc, m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d1 = d * sc, m1 = dmin * m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d2 = d * sc, m2 = dmin * m;
            const uint8_t* q = ql + (j >> 1);
            for (int l = 0; l < 32; l++) {
                y[j + l] = d1 * ((q[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
                y[j + l + 32] = d2 * ((q[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
            }
            u1 <<= 2; u2 <<= 2;
        }
    }
}

/* src/tensor.h:398-432 */
static void dq_q6_k(const uint8_t* p, float* y, int64_t nb) {
    for (int64_t b = 0; b < nb; b++, p += 210, y += 256) {
        const uint8_t* ql = p;
        const uint8_t* qh = p + 128;
        const int8_t* sc = (const int8_t*)(p + 192);
        float d = ld_half(p + 208);
        for (int n = 0; n < 256; n += 128) {
            const uint8_t* l_ = ql + (n >> 1);
            const uint8_t* h_ = qh + (n >> 2);
            const int8_t* s_ = sc + (n >> 4);
            float* y_ = y + n;
            for (int l = 0; l < 32; l++) {
                int is = l >> 4;
                int8_t q1 = (int8_t)((l_[l] & 0xF) | (((h_[l] >> 0) & 3) << 4)) - 32;
                int8_t q2 = (int8_t)((l_[l + 32] & 0xF) | (((h_[l] >> 2) & 3) << 4)) - 32;
                int8_t q3 = (int8_t)((l_[l] >> 4) | (((h_[l] >> 4) & 3) << 4)) - 32;
                int8_t q4 = (int8_t)((l_[l + 32] >> 4) | (((h_[l] >> 6) & 3) << 4)) - 32;
                y_[l + 0] = d * s_[is + 0] * q1;
                y_[l + 32] = d * s_[is + 2] * q2;
                y_[l + 64] = d * s_[is + 4] * q3;
                y_[l + 96] = d * s_[is + 6] * q4;
            }
        }
    }
}

/* Dispatcher, src/tensor.h:451-497.  Returns 0, or -1 for a type outside
 * this path (the reference prints to stderr and leaves dst untouched). */
int oracle_dequantize(int type, const void* src, float* dst, int64_t n) {
    size_t qk = oracle_block_size(type);
    if (!qk) return -1;
    int64_t nb = n / (int64_t)qk;
    const uint8_t* p = (const uint8_t*)src;
    switch (type) {
        case T_Q4_0: dq_q4_0(p, dst, nb); break;
        case T_Q8_0: dq_q8_0(p, dst, nb); break;
        case T_Q2_K: dq_q2_k(p, dst, nb); break;
        case T_Q3_K: dq_q3_k(p, dst, nb); break;
        case T_Q4_K: dq_q4_k(p, dst, nb); break;
        case T_Q5_K: dq_q5_k(p, dst, nb); break;
        case T_Q6_K: dq_q6_k(p, dst, nb); break;
        default: return -1;
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Fused dequant + GEMV: out[N] = W[N x K] . x[K]                            */
/* ------------------------------------------------------------------------ */

/* src/tensor.h:570-599 */
static float row_q8_0(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 34) {
        float d = ld_half(row);
        const int8_t* v = (const int8_t*)(row + 2);
        const float* xb = x + b * 32;
        float bs = 0.0f;
        for (int j = 0; j < 32; j++) bs += xb[j] * (float)v[j];
        sum += bs * d;
    }
    return sum;
}

/* src/tensor.h:607-640 */
static float row_q4_0(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 18) {
        float d = ld_half(row);
        const uint8_t* nib = row + 2;
        const float* xb = x + b * 32;
        float bs = 0.0f;
        for (int j = 0; j < 16; j++) {
            uint8_t v = nib[j];
            bs += xb[j] * (float)((int)(v & 0x0F) - 8);
            bs += xb[j + 16] * (float)((int)(v >> 4) - 8);
        }
        sum += bs * d;
    }
    return sum;
}

/* src/tensor.h:769-810 */
static float row_q6_k(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 210) {
        const uint8_t* ql = row;
        const uint8_t* qh = row + 128;
        const int8_t* sc = (const int8_t*)(row + 192);
        float d = ld_half(row + 208);
        const float* xb = x + b * 256;
        for (int n = 0; n < 256; n += 128) {
            const uint8_t* l_ = ql + (n >> 1);
            const uint8_t* h_ = qh + (n >> 2);
            const int8_t* s_ = sc + (n >> 4);
            const float* xn = xb + n;
            for (int l = 0; l < 32; l++) {
                int is = l >> 4;
                int8_t q1 = (int8_t)((l_[l] & 0xF) | (((h_[l] >> 0) & 3) << 4)) - 32;
                int8_t q2 = (int8_t)((l_[l + 32] & 0xF) | (((h_[l] >> 2) & 3) << 4)) - 32;
                int8_t q3 = (int8_t)((l_[l] >> 4) | (((h_[l] >> 4) & 3) << 4)) - 32;
                int8_t q4 = (int8_t)((l_[l + 32] >> 4) | (((h_[l] >> 6) & 3) << 4)) - 32;
                sum += d * s_[is + 0] * q1 * xn[l + 0];
                sum += d * s_[is + 2] * q2 * xn[l + 32];
                sum += d * s_[is + 4] * q3 * xn[l + 64];
                sum += d * s_[is + 6] * q4 * xn[l + 96];
            }
        }
    }
    return sum;
}

/* src/tensor.h:817-856 */
static float row_q4_k(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 144) {
        float d = ld_half(row), dmin = ld_half(row + 2);
        const uint8_t* s = row + 4;
        const uint8_t* qs = row + 16;
        const float* xb = x + b * 256;
        int is = 0;
        for (int j = 0; j < 256; j += 64) {
            uint8_t sc, m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d1 = d * sc, m1 = dmin * m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d2 = d * sc, m2 = dmin * m;
            const uint8_t* q = qs + (j >> 1);
            const float* xj = xb + j;
            for (int l = 0; l < 32; l++) {
                sum += (d1 * (q[l] & 0xF) - m1) * xj[l];
                sum += (d2 * (q[l] >> 4) - m2) * xj[l + 32];
            }
        }
    }
    return sum;
}

/* src/tensor.h:863-905 */
static float row_q5_k(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 176) {
        float d = ld_half(row), dmin = ld_half(row + 2);
        const uint8_t* s = row + 4;
        const uint8_t* qh = row + 16;
        const uint8_t* ql = row + 48;
        const float* xb = x + b * 256;
        int is = 0;
        uint8_t u1 = 1, u2 = 2;
        for (int j = 0; j < 256; j += 64) {
            uint8_t sc, m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d1 = d * sc, m1 = dmin * m;
            oracle_get_scale_min_k4(is++, s, &sc, &m);
            float d2 = d * sc, m2 = dmin * m;
            const uint8_t* q = ql + (j >> 1);
            const float* xj = xb + j;
            for (int l = 0; l < 32; l++) {
                sum += (d1 * ((q[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1) * xj[l];
                sum += (d2 * ((q[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2) * xj[l + 32];
            }
            u1 <<= 2; u2 <<= 2;
        }
    }
    return sum;
}

/* src/tensor.h:912-958, restated as written.  Note: the activation index is
 * xb[n + l] / xb[n + l + 16] for all four shift groups j (it does not advance
 * by 32*j), so this routine does NOT equal dequantize_q2_k followed by a dot
 * product.  See oracle_gemv_q2k_dequant_order below for the format order. */
static float row_q2_k_ref_cpu(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 84) {
        const uint8_t* sc = row;
        const uint8_t* q = row + 16;
        float d = ld_half(row + 80), dmin = ld_half(row + 82);
        const float* xb = x + b * 256;
        int is = 0;
        for (int n = 0; n < 256; n += 128) {
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                uint8_t s0 = sc[is++];
                float dl = d * (s0 & 0xF), ml = dmin * (s0 >> 4);
                for (int l = 0; l < 16; l++) {
                    int v = (q[l] >> shift) & 3;
                    sum += (dl * v - ml) * xb[n + l];
                }
                uint8_t s1 = sc[is++];
                dl = d * (s1 & 0xF); ml = dmin * (s1 >> 4);
                for (int l = 0; l < 16; l++) {
                    int v = (q[l + 16] >> shift) & 3;
                    sum += (dl * v - ml) * xb[n + l + 16];
                }
                shift += 2;
                if (shift == 8) { shift = 0; q += 32; }
            }
        }
    }
    return sum;
}

/* Q2_K in the element order of dequantize_q2_k (src/tensor.h:232-265), i.e.
 * the order of the GGUF format and of the reference's CUDA backend, which
 * dequantizes on the host before its SGEMM (src/tensor.h:1219-1223).  Same
 * per-element expression (dl * v - ml) * x, accumulated left to right. */
static float row_q2_k_dq_order(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 84) {
        const uint8_t* sc = row;
        const uint8_t* q = row + 16;
        float d = ld_half(row + 80), dmin = ld_half(row + 82);
        const float* xb = x + b * 256;
        int is = 0;
        for (int n = 0; n < 256; n += 128) {
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                uint8_t s0 = sc[is++];
                float dl = d * (s0 & 0xF), ml = dmin * (s0 >> 4);
                for (int l = 0; l < 16; l++) {
                    int v = (q[l] >> shift) & 3;
                    sum += (dl * v - ml) * xb[n + 32 * j + l];
                }
                uint8_t s1 = sc[is++];
                dl = d * (s1 & 0xF); ml = dmin * (s1 >> 4);
                for (int l = 0; l < 16; l++) {
                    int v = (q[l + 16] >> shift) & 3;
                    sum += (dl * v - ml) * xb[n + 32 * j + l + 16];
                }
                shift += 2;
                if (shift == 8) { shift = 0; q += 32; }
            }
        }
    }
    return sum;
}

/* src/tensor.h:964-1025 */
static float row_q3_k(const uint8_t* row, const float* x, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++, row += 110) {
        const uint8_t* hm = row;
        const uint8_t* q = row + 32;
        float d = ld_half(row + 108);
        const float* xb = x + b * 256;
        int8_t s[16];
        oracle_q3k_scales(row + 96, s);
        uint8_t m = 1;
        for (int n = 0; n < 256; n += 128) {
            int off = (n == 0) ? 0 : 8;
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                float dl0 = d * s[off + 2 * j];
                float dl1 = d * s[off + 2 * j + 1];
                int base = n + 32 * j;
                for (int l = 0; l < 16; l++) {
                    int v0 = ((q[l] >> shift) & 3) - ((hm[l] & m) ? 0 : 4);
                    int v1 = ((q[l + 16] >> shift) & 3) - ((hm[l + 16] & m) ? 0 : 4);
                    sum += dl0 * v0 * xb[base + l];
                    sum += dl1 * v1 * xb[base + l + 16];
                }
                shift += 2;
                if (shift == 8) { shift = 0; q += 32; }
                m <<= 1;
            }
        }
    }
    return sum;
}

typedef float (*row_fn)(const uint8_t*, const float*, int);

static row_fn pick_row(int type, int q2k_ref_cpu) {
    switch (type) {
        case T_Q4_0: return row_q4_0;
        case T_Q8_0: return row_q8_0;
        case T_Q2_K: return q2k_ref_cpu ? row_q2_k_ref_cpu : row_q2_k_dq_order;
        case T_Q3_K: return row_q3_k;
        case T_Q4_K: return row_q4_k;
        case T_Q5_K: return row_q5_k;
        case T_Q6_K: return row_q6_k;
        default: return 0;
    }
}

static int gemv_impl(int type, float* out, const float* x, const void* w,
                     int N, int K, int q2k_ref_cpu) {
    row_fn f = pick_row(type, q2k_ref_cpu);
    size_t qk = oracle_block_size(type), bb = oracle_type_size(type);
    if (!f) return -1;
    int nb = K / (int)qk;
    size_t rb = (size_t)nb * bb;
    const uint8_t* wp = (const uint8_t*)w;
    int i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < N; i++) out[i] = f(wp + (size_t)i * rb, x, nb);
    return 0;
}

/* Compute::matmul_transposed_q CPU branch, src/tensor.h:1228-1277: the fused
 * per-format routine, OpenMP over output rows, one fp32 sum per row. */
int oracle_matmul_transposed_q(int type, float* out, const float* x,
                               const void* w, int N, int K) {
    return gemv_impl(type, out, x, w, N, K, 1);
}

/* Same, with Q2_K in dequantize_q2_k element order (the GGUF format order,
 * equal to the reference CUDA backend's dequantize-then-SGEMM). */
int oracle_matmul_transposed_q_format_order(int type, float* out, const float* x,
                                            const void* w, int N, int K) {
    return gemv_impl(type, out, x, w, N, K, 0);
}

/* M > 1: the reference has no batched quantized path (prefill is a loop of
 * single-token forwards, src/main.cpp:284-287), so Y[m] = W . X[m] for each m. */
int oracle_matmul_q_batched(int type, float* Y, const float* X, const void* w,
                            int M, int N, int K, int format_order) {
    for (int m = 0; m < M; m++) {
        int rc = gemv_impl(type, Y + (size_t)m * N, X + (size_t)m * K, w, N, K,
                           !format_order);
        if (rc) return rc;
    }
    return 0;
}

/* cpu_matmul_transposed, src/tensor.h:548-560 (fp32 weights). */
void oracle_matmul_transposed_f32(float* out, const float* x, const float* w, int N, int K) {
    int i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < N; i++) {
        float sum = 0.0f;
        const float* row = w + (size_t)i * K;
        for (int k = 0; k < K; k++) sum += x[k] * row[k];
        out[i] = sum;
    }
}

int oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}
