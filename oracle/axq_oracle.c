/*
 * CPU oracle for the block-quantized matmul path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of ruwwww/Axon's CPU quantize / dequantize /
 * quantized-matmul algorithms (src/backend/cpu_backend.cpp), written to
 * check the CUDA kernels.  The product never links or calls this file.
 *
 * Exactness notes (these decide bit-exactness of the packed bytes):
 *  - The reference is C++ built for x86-64 without FMA or fast-math, so
 *    every float operation below is a single IEEE-754 binary32 operation;
 *    compile this file with -ffp-contract=off.
 *  - std::max(a,b) is (a<b)?b:a and std::min(a,b) is (b<a)?b:a; the
 *    argument order of each call is kept so NaN inputs behave the same.
 *  - static_cast<int>(float) compiles to cvttss2si on x86-64, which returns
 *    INT_MIN for NaN and for values outside the int range; to_int_x86()
 *    states that rule explicitly (it matters: Q2_K divides by a sub-block
 *    scale that can be 0, giving +-inf or NaN).
 *  - std::round(float) is roundf (halfway cases away from zero).
 */
#include "axq_oracle.h"

#include <limits.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define FMAX(a, b) (((a) < (b)) ? (b) : (a)) /* std::max */
#define FMIN(a, b) (((b) < (a)) ? (b) : (a)) /* std::min */
#define IMAX(a, b) (((a) < (b)) ? (b) : (a))
#define IMIN(a, b) (((b) < (a)) ? (b) : (a))

static int to_int_x86(float f) {
    /* cvttss2si: truncate toward zero; NaN/out-of-range -> 0x80000000. */
    if (f >= -2147483648.0f && f < 2147483648.0f) return (int)f;
    return INT_MIN;
}

/* float_to_half, cpu_backend.cpp:583-595: mantissa truncation; exponents
 * below -14 flush to signed zero, above 15 (NaN included) become inf. */
uint16_t orc_float_to_half(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sign = (u >> 16) & 0x8000u;
    int32_t e = (int32_t)((u >> 23) & 0xFFu) - 127;
    uint32_t mant = u & 0x007FFFFFu;
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    if (e < -14) return (uint16_t)sign;
    return (uint16_t)(sign | ((uint32_t)((e + 15) & 0x1F) << 10) | (mant >> 13));
}

/* half_to_float, cpu_backend.cpp:597-620: fp16 subnormals decode to +-0. */
float orc_half_to_float(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t u;
    if (e == 0) u = sign << 31;
    else if (e == 31) u = (sign << 31) | 0x7F800000u | (mant << 13);
    else u = (sign << 31) | ((e - 15 + 127) << 23) | (mant << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* get_scale_min_k4, cpu_backend.cpp:681-689. */
static void scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* Block layouts (cpu_backend.cpp:624-678), as byte offsets:
 *  Q8_0 34 B: d@0, qs[32]@2          Q4_0 18 B: d@0, qs[16]@2
 *  Q2_K 84 B: d@0 dmin@2 scales[16]@4 qs[64]@20
 *  Q3_K 110 B: hmask[32]@0 qs[64]@32 scales[12]@96 d@108
 *  Q4_K 144 B: d@0 dmin@2 scales[12]@4 qs[128]@16
 *  Q5_K 176 B: d@0 dmin@2 scales[12]@4 qh[32]@16 qs[128]@48
 *  Q6_K 210 B: ql[128]@0 qh[64]@128 scales[16]@192 d@208 */
size_t orc_block_bytes(int fmt) {
    switch (fmt) {
        case ORC_Q8_0: return 34;
        case ORC_Q4_0: return 18;
        case ORC_Q2_K: return 84;
        case ORC_Q3_K: return 110;
        case ORC_Q4_K: return 144;
        case ORC_Q5_K: return 176;
        case ORC_Q6_K: return 210;
        default: return 0;
    }
}

int orc_block_elems(int fmt) {
    switch (fmt) {
        case ORC_Q8_0: case ORC_Q4_0: return 32;
        case ORC_Q2_K: case ORC_Q3_K: case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: return 256;
        default: return 0;
    }
}

size_t orc_quantized_size(size_t numel, int fmt) {
    int be = orc_block_elems(fmt);
    if (!be) return 0;
    return ((numel + (size_t)be - 1) / (size_t)be) * orc_block_bytes(fmt);
}

size_t orc_quantized_size_2d(int64_t rows, int64_t cols, int fmt) {
    int be = orc_block_elems(fmt);
    if (!be) return 0;
    size_t bpr = ((size_t)cols + (size_t)be - 1) / (size_t)be;
    return (size_t)rows * bpr * orc_block_bytes(fmt);
}

/* ---------------------------------------------------------------- pack */

/* quantize_block_q8_0, cpu_backend.cpp:739-752 */
static void pack_q8_0(uint8_t* blk, const float* x, int count) {
    float amax = 0.0f;
    for (int i = 0; i < count; ++i) amax = FMAX(amax, fabsf(x[i]));
    float d = (amax == 0.0f) ? 1.0f : (amax / 127.0f);
    wr16(blk, orc_float_to_half(d));
    for (int i = 0; i < 32; ++i) {
        int8_t q = 0;
        if (i < count) {
            float r = roundf(x[i] / d);
            float c = FMAX(-127.0f, FMIN(127.0f, r));
            q = (int8_t)to_int_x86(c);
        }
        blk[2 + i] = (uint8_t)q;
    }
}

/* quantize_block_q4_0, cpu_backend.cpp:754-773 */
static void pack_q4_0(uint8_t* blk, const float* x, int count) {
    float amax = 0.0f;
    for (int i = 0; i < count; ++i) amax = FMAX(amax, fabsf(x[i]));
    float d = (amax == 0.0f) ? 1.0f : (amax / 8.0f);
    wr16(blk, orc_float_to_half(d));
    for (int i = 0; i < 16; ++i) {
        int lo = 0, hi = 0;
        if (2 * i < count) lo = IMAX(-8, IMIN(7, to_int_x86(roundf(x[2 * i] / d))));
        if (2 * i + 1 < count) hi = IMAX(-8, IMIN(7, to_int_x86(roundf(x[2 * i + 1] / d))));
        blk[2 + i] = (uint8_t)((lo + 8) | ((hi + 8) << 4));
    }
}

/* Shared by Q4_K / Q5_K (cpu_backend.cpp:934-1009, 1011-1090): 8 groups of
 * 32 with an asymmetric range scale `range/levels` and min `-min(g_min,0)`,
 * both re-quantized to 6 bits against their maxima. */
static void kquant_group_stats(const float* x, int count, float levels,
                               float* scales, float* mins, float* max_scale, float* max_min) {
    *max_scale = 0.0f;
    *max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        if (j * 32 >= count) { scales[j] = 0.0f; mins[j] = 0.0f; continue; }
        float lo = x[j * 32], hi = x[j * 32];
        for (int i = 1; i < 32 && j * 32 + i < count; ++i) {
            float v = x[j * 32 + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        float range = hi - lo;
        if (range < 1e-10f) range = 1.0f;
        scales[j] = range / levels;
        float cmin = (lo < 0) ? lo : 0.0f;
        mins[j] = -cmin;
        if (scales[j] > *max_scale) *max_scale = scales[j];
        if (mins[j] > *max_min) *max_min = mins[j];
    }
}

/* 12-byte 6-bit scale/min packing, cpu_backend.cpp:969-980 (inverse of
 * get_scale_min_k4). */
static void kquant_pack_scales(uint8_t* sc12, const float* scales, const float* mins,
                               float iscale, float iscale_m) {
    memset(sc12, 0, 12);
    for (int j = 0; j < 8; ++j) {
        uint8_t ls = (uint8_t)IMIN(63, IMAX(0, to_int_x86(roundf(scales[j] * iscale))));
        uint8_t lm = (uint8_t)IMIN(63, IMAX(0, to_int_x86(roundf(mins[j] * iscale_m))));
        if (j < 4) {
            sc12[j] = ls;
            sc12[j + 4] = lm;
        } else {
            sc12[j + 4] = (uint8_t)((ls & 0xF) | ((lm & 0xF) << 4));
            sc12[j - 4] |= (uint8_t)((ls >> 4) << 6);
            sc12[j] |= (uint8_t)((lm >> 4) << 6);
        }
    }
}

/* Element codes of Q4_K/Q5_K from the fp16-decoded d/dmin and the 6-bit
 * sub-scales (cpu_backend.cpp:984-1000, 1058-1072). */
static void kquant_codes(uint8_t* L, const float* x, int count, const uint8_t* blk_d,
                         const uint8_t* sc12, int maxq) {
    float d_super = orc_half_to_float(rd16(blk_d));
    float m_super = orc_half_to_float(rd16(blk_d + 2));
    for (int j = 0; j < 8; ++j) {
        uint8_t sc, m;
        scale_min_k4(j, sc12, &sc, &m);
        float d_eff = d_super * (float)sc;
        float m_eff = m_super * (float)m;
        if (d_eff < 1e-10f) d_eff = 1.0f;
        for (int i = 0; i < 32 && j * 32 + i < count; ++i) {
            int l = to_int_x86(roundf((x[j * 32 + i] + m_eff) / d_eff));
            L[j * 32 + i] = (uint8_t)IMAX(0, IMIN(maxq, l));
        }
        for (int i = IMAX(0, count - j * 32); i < 32; ++i) L[j * 32 + i] = 0;
    }
}

/* quantize_block_q2_K, cpu_backend.cpp:775-847 */
static void pack_q2_K(uint8_t* blk, const float* x, int count) {
    float sub_scales[16], sub_mins[16];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 16; ++j) {
        if (j * 16 >= count) { sub_scales[j] = 0.0f; sub_mins[j] = 0.0f; continue; }
        float lo = x[j * 16], hi = x[j * 16];
        for (int i = 1; i < 16 && j * 16 + i < count; ++i) {
            float v = x[j * 16 + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        float range = hi - lo;
        if (range < 1e-10f) range = 1.0f;
        sub_scales[j] = range / 3.0f;
        float cmin = (lo < 0) ? lo : 0.0f;
        sub_mins[j] = -cmin;
        if (sub_scales[j] > max_scale) max_scale = sub_scales[j];
        if (sub_mins[j] > max_min) max_min = sub_mins[j];
    }
    float iscale_d = (max_scale > 0.0f) ? 15.0f / max_scale : 0.0f;
    float iscale_m = (max_min > 0.0f) ? 15.0f / max_min : 0.0f;
    wr16(blk + 0, orc_float_to_half(max_scale / 15.0f));
    wr16(blk + 2, orc_float_to_half(max_min / 15.0f));
    uint8_t* scales = blk + 4;
    uint8_t* qs = blk + 20;
    for (int j = 0; j < 16; ++j) {
        int qsc = IMIN(15, IMAX(0, to_int_x86(roundf(sub_scales[j] * iscale_d))));
        int qm = IMIN(15, IMAX(0, to_int_x86(roundf(sub_mins[j] * iscale_m))));
        scales[j] = (uint8_t)(qsc | (qm << 4));
    }
    float d_super = orc_half_to_float(rd16(blk));
    float m_super = orc_half_to_float(rd16(blk + 2));
    uint8_t L[256];
    for (int j = 0; j < 16; ++j) {
        float dv = d_super * (float)(scales[j] & 0xF);
        float mv = m_super * (float)(scales[j] >> 4);
        for (int i = 0; i < 16 && j * 16 + i < count; ++i) {
            int l = to_int_x86(roundf((x[j * 16 + i] + mv) / dv));
            L[j * 16 + i] = (uint8_t)IMAX(0, IMIN(3, l));
        }
        for (int i = IMAX(0, count - j * 16); i < 16; ++i) L[j * 16 + i] = 0;
    }
    memset(qs, 0, 64);
    for (int n = 0; n < 256; n += 128)
        for (int l = 0; l < 32; ++l) {
            int v = 0;
            for (int t = 0; t < 4; ++t)
                if (n + l + 32 * t < count) v |= (L[n + l + 32 * t] & 3) << (2 * t);
            qs[n / 4 + l] = (uint8_t)v;
        }
}

/* quantize_block_q3_K, cpu_backend.cpp:849-932 */
static void pack_q3_K(uint8_t* blk, const float* x, int count) {
    uint8_t* hmask = blk;
    uint8_t* qs = blk + 32;
    uint8_t* scales = blk + 96;
    float sub_scales[16];
    float max_abs = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f;
        for (int i = 0; i < 16 && j * 16 + i < count; ++i) amax = FMAX(amax, fabsf(x[j * 16 + i]));
        sub_scales[j] = (amax < 1e-10f) ? 0.0f : (amax / 4.0f);
        float a = fabsf(sub_scales[j]);
        if (a > max_abs) max_abs = a;
    }
    memset(scales, 0, 12);
    if (max_abs > 0.0f) {
        float iscale = -32.0f / max_abs;
        for (int j = 0; j < 16; ++j) {
            int l = to_int_x86(roundf(iscale * sub_scales[j]));
            l = IMAX(-32, IMIN(31, l)) + 32;
            if (j < 8) scales[j] = (uint8_t)(l & 0xF);
            else scales[j - 8] |= (uint8_t)((l & 0xF) << 4);
            l >>= 4;
            scales[j % 4 + 8] |= (uint8_t)(l << (2 * (j / 4)));
        }
        wr16(blk + 108, orc_float_to_half(1.0f / iscale));
    } else {
        wr16(blk + 108, orc_float_to_half(0.0f));
    }
    int8_t L[256];
    float d_all = orc_half_to_float(rd16(blk + 108));
    for (int j = 0; j < 16; ++j) {
        int sc = (j < 8) ? (scales[j] & 0xF) : (scales[j - 8] >> 4);
        sc = (sc | (((scales[8 + j % 4] >> (2 * (j / 4))) & 3) << 4)) - 32;
        float d_sub = d_all * (float)sc;
        if (fabsf(d_sub) < 1e-10f) d_sub = 1.0f;
        for (int i = 0; i < 16 && j * 16 + i < count; ++i) {
            int l = to_int_x86(roundf(x[j * 16 + i] / d_sub));
            L[j * 16 + i] = (int8_t)IMAX(-4, IMIN(3, l));
        }
        for (int i = IMAX(0, count - j * 16); i < 16; ++i) L[j * 16 + i] = 0;
    }
    memset(hmask, 0, 32);
    memset(qs, 0, 64);
    /* The high bit is written only for elements inside the block's count. */
    for (int j = 0; j < 256 && j < count; ++j)
        if (L[j] + 4 > 3) hmask[j % 32] |= (uint8_t)(1u << (j / 32));
    for (int n = 0; n < 256; n += 128)
        for (int l = 0; l < 32; ++l)
            qs[n / 4 + l] = (uint8_t)((L[n + l] & 3) | ((L[n + l + 32] & 3) << 2) |
                                      ((L[n + l + 64] & 3) << 4) | ((L[n + l + 96] & 3) << 6));
}

/* quantize_block_q4_K, cpu_backend.cpp:934-1009 */
static void pack_q4_K(uint8_t* blk, const float* x, int count) {
    float scales[8], mins[8], max_scale, max_min;
    kquant_group_stats(x, count, 15.0f, scales, mins, &max_scale, &max_min);
    float iscale = (max_scale > 0.0f) ? 63.0f / max_scale : 0.0f;
    float iscale_m = (max_min > 0.0f) ? 63.0f / max_min : 0.0f;
    wr16(blk + 0, orc_float_to_half(max_scale / 63.0f));
    wr16(blk + 2, orc_float_to_half(max_min / 63.0f));
    kquant_pack_scales(blk + 4, scales, mins, iscale, iscale_m);
    uint8_t L[256];
    kquant_codes(L, x, count, blk, blk + 4, 15);
    uint8_t* q = blk + 16;
    for (int j = 0; j < 256; j += 64, q += 32)
        for (int l = 0; l < 32; ++l) q[l] = (uint8_t)(L[j + l] | (L[j + l + 32] << 4));
}

/* quantize_block_q5_K, cpu_backend.cpp:1011-1090 */
static void pack_q5_K(uint8_t* blk, const float* x, int count) {
    float scales[8], mins[8], max_scale, max_min;
    kquant_group_stats(x, count, 31.0f, scales, mins, &max_scale, &max_min);
    float iscale = (max_scale > 0.0f) ? 63.0f / max_scale : 0.0f;
    float iscale_m = (max_min > 0.0f) ? 63.0f / max_min : 0.0f;
    wr16(blk + 0, orc_float_to_half(max_scale / 63.0f));
    wr16(blk + 2, orc_float_to_half(max_min / 63.0f));
    kquant_pack_scales(blk + 4, scales, mins, iscale, iscale_m);
    uint8_t L[256];
    kquant_codes(L, x, count, blk, blk + 4, 31);
    uint8_t* qh = blk + 16;
    uint8_t* q = blk + 48;
    memset(qh, 0, 32);
    uint8_t m1 = 1, m2 = 2;
    for (int j = 0; j < 256; j += 64, q += 32) {
        for (int l = 0; l < 32; ++l) {
            int l1 = L[j + l], l2 = L[j + l + 32];
            if (l1 > 15) { l1 -= 16; qh[l] |= m1; }
            if (l2 > 15) { l2 -= 16; qh[l] |= m2; }
            q[l] = (uint8_t)(l1 | (l2 << 4));
        }
        m1 = (uint8_t)(m1 << 2);
        m2 = (uint8_t)(m2 << 2);
    }
}

/* quantize_block_q6_K, cpu_backend.cpp:1092-1156 */
static void pack_q6_K(uint8_t* blk, const float* x, int count) {
    uint8_t* ql = blk;
    uint8_t* qh = blk + 128;
    int8_t* scales = (int8_t*)(blk + 192);
    float sub_scales[16];
    float max_abs = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f;
        for (int i = 0; i < 16 && j * 16 + i < count; ++i) amax = FMAX(amax, fabsf(x[j * 16 + i]));
        sub_scales[j] = (amax < 1e-10f) ? 0.0f : (amax / 32.0f);
        float a = fabsf(sub_scales[j]);
        if (a > max_abs) max_abs = a;
    }
    if (max_abs < 1e-10f) {
        memset(blk, 0, 210);
        wr16(blk + 208, orc_float_to_half(0.0f));
        return;
    }
    float iscale = -128.0f / max_abs;
    wr16(blk + 208, orc_float_to_half(1.0f / iscale));
    for (int j = 0; j < 16; ++j)
        scales[j] = (int8_t)IMAX(-128, IMIN(127, to_int_x86(roundf(iscale * sub_scales[j]))));
    int8_t L[256];
    float d_all = orc_half_to_float(rd16(blk + 208));
    for (int j = 0; j < 16; ++j) {
        float d_sub = d_all * (float)scales[j];
        if (fabsf(d_sub) < 1e-10f) d_sub = 1.0f;
        for (int i = 0; i < 16 && j * 16 + i < count; ++i) {
            int l = to_int_x86(roundf(x[j * 16 + i] / d_sub));
            L[j * 16 + i] = (int8_t)IMAX(-32, IMIN(31, l));
        }
        for (int i = IMAX(0, count - j * 16); i < 16; ++i) L[j * 16 + i] = 0;
    }
    memset(ql, 0, 128);
    memset(qh, 0, 64);
    for (int n = 0; n < 256; n += 128)
        for (int l = 0; l < 32; ++l) {
            int v0 = L[n + l] + 32, v1 = L[n + l + 32] + 32;
            int v2 = L[n + l + 64] + 32, v3 = L[n + l + 96] + 32;
            ql[n / 2 + l] = (uint8_t)((v0 & 0xF) | ((v2 & 0xF) << 4));
            ql[n / 2 + l + 32] = (uint8_t)((v1 & 0xF) | ((v3 & 0xF) << 4));
            qh[n / 4 + l] = (uint8_t)(((v0 >> 4) & 3) | (((v1 >> 4) & 3) << 2) |
                                      (((v2 >> 4) & 3) << 4) | (((v3 >> 4) & 3) << 6));
        }
}

typedef void (*pack_fn)(uint8_t*, const float*, int);

static pack_fn pack_for(int fmt) {
    switch (fmt) {
        case ORC_Q8_0: return pack_q8_0;
        case ORC_Q4_0: return pack_q4_0;
        case ORC_Q2_K: return pack_q2_K;
        case ORC_Q3_K: return pack_q3_K;
        case ORC_Q4_K: return pack_q4_K;
        case ORC_Q5_K: return pack_q5_K;
        case ORC_Q6_K: return pack_q6_K;
        default: return NULL;
    }
}

int orc_quantize(int fmt, const float* src, int64_t rows, int64_t cols, void* dst) {
    pack_fn fn = pack_for(fmt);
    if (!fn) return -1;
    int be = orc_block_elems(fmt);
    size_t bb = orc_block_bytes(fmt);
    int64_t bpr = (cols + be - 1) / be;
    uint8_t* out = (uint8_t*)dst;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < bpr; ++b) {
            int64_t off = b * be;
            int count = (int)((cols - off) < be ? (cols - off) : be);
            fn(out + (size_t)(r * bpr + b) * bb, src + r * cols + off, count);
        }
    return 0;
}

/* -------------------------------------------------------------- decode */

/* Value of element e (0 <= e < block elems) of one block, computed with
 * exactly the operations of the decode lambdas of cpu_backend.cpp:1340-1504
 * (the same formulas appear in the matmul loops :1699-2060). */
static float decode_elem(int fmt, const uint8_t* blk, int e) {
    switch (fmt) {
        case ORC_Q8_0: /* :1340-1343 */
            return (float)(int8_t)blk[2 + e] * orc_half_to_float(rd16(blk));
        case ORC_Q4_0: { /* :1345-1359 */
            uint8_t byte = blk[2 + e / 2];
            int q = (e & 1) ? ((byte >> 4) - 8) : ((byte & 0xF) - 8);
            return (float)q * orc_half_to_float(rd16(blk));
        }
        case ORC_Q2_K: { /* :1361-1387 */
            float d = orc_half_to_float(rd16(blk));
            float mn = orc_half_to_float(rd16(blk + 2));
            int n = e / 128, j = (e % 128) / 32, l = e % 32;
            uint8_t sc = blk[4 + 8 * n + 2 * j + (l >= 16)];
            float dl = d * (float)(sc & 0xF);
            float ml = mn * (float)(sc >> 4);
            int q = (blk[20 + 32 * n + l] >> (2 * j)) & 3;
            return dl * (float)q - ml;
        }
        case ORC_Q3_K: { /* :1389-1429 */
            float d_all = orc_half_to_float(rd16(blk + 108));
            const uint8_t* sc12 = blk + 96;
            int n = e / 128, j = (e % 128) / 32, l = e % 32;
            int is = 8 * n + 2 * j + (l >= 16);
            int lo4 = (is < 8) ? (sc12[is] & 0xF) : (sc12[is - 8] >> 4);
            int hi2 = (sc12[8 + is % 4] >> (2 * (is / 4))) & 3;
            int sc = (int)(int8_t)(uint8_t)(lo4 | (hi2 << 4)) - 32;
            float dl = d_all * (float)sc;
            int qv = (blk[32 + 32 * n + l] >> (2 * j)) & 3;
            int hbit = (blk[l] >> (4 * n + j)) & 1;
            return dl * (float)(qv - (hbit ? 0 : 4));
        }
        case ORC_Q4_K: { /* :1431-1455 */
            float d = orc_half_to_float(rd16(blk));
            float mn = orc_half_to_float(rd16(blk + 2));
            int g = e / 32, l = e % 32, c = g / 2;
            uint8_t sc, m;
            scale_min_k4(g, blk + 4, &sc, &m);
            float d1 = d * (float)sc, m1 = mn * (float)m;
            uint8_t byte = blk[16 + 32 * c + l];
            int q = (g & 1) ? (byte >> 4) : (byte & 0xF);
            return d1 * (float)q - m1;
        }
        case ORC_Q5_K: { /* :1457-1483 */
            float d = orc_half_to_float(rd16(blk));
            float mn = orc_half_to_float(rd16(blk + 2));
            int g = e / 32, l = e % 32, c = g / 2;
            uint8_t sc, m;
            scale_min_k4(g, blk + 4, &sc, &m);
            float d1 = d * (float)sc, m1 = mn * (float)m;
            uint8_t byte = blk[48 + 32 * c + l];
            int q = ((g & 1) ? (byte >> 4) : (byte & 0xF)) + (((blk[16 + l] >> g) & 1) ? 16 : 0);
            return d1 * (float)q - m1;
        }
        case ORC_Q6_K: { /* :1485-1504 */
            float d = orc_half_to_float(rd16(blk + 208));
            int n = e / 128, t = (e % 128) / 32, l = e % 32;
            const uint8_t* ql = blk + 64 * n;
            const uint8_t* qh = blk + 128 + 32 * n;
            const int8_t* sc = (const int8_t*)(blk + 192 + 8 * n);
            int low = (t == 0) ? (ql[l] & 0xF) : (t == 1) ? (ql[l + 32] & 0xF)
                    : (t == 2) ? (ql[l] >> 4) : (ql[l + 32] >> 4);
            int q = (int)(int8_t)(uint8_t)(low | (((qh[l] >> (2 * t)) & 3) << 4)) - 32;
            return d * (float)sc[l / 16 + 2 * t] * (float)q;
        }
        default:
            return 0.0f;
    }
}

int orc_dequantize(int fmt, const void* src, int64_t rows, int64_t cols, float* dst) {
    int be = orc_block_elems(fmt);
    if (!be) return -1;
    size_t bb = orc_block_bytes(fmt);
    int64_t bpr = (cols + be - 1) / be;
    const uint8_t* in = (const uint8_t*)src;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < bpr; ++b) {
            const uint8_t* blk = in + (size_t)(r * bpr + b) * bb;
            for (int e = 0; e < be && b * be + e < cols; ++e)
                dst[r * cols + b * be + e] = decode_elem(fmt, blk, e);
        }
    return 0;
}

/* -------------------------------------------------------------- matmul */

/* Visit order of the k index inside one 256-element block for the scalar
 * K-quant loops: Q6_K walks four k's (l, l+32, l+64, l+96) per step
 * (cpu_backend.cpp:1835-1851); the others walk k in increasing order. */
static int q6_visit(int step) {
    int n = step / 128, r = step % 128, l = r / 4, t = r % 4;
    return 128 * n + 32 * t + l;
}

int orc_matmul_rows(int fmt, const void* a_q, const float* b, float* out,
                    int64_t M, int64_t K, int64_t N, int64_t row0, int64_t row1) {
    int be = orc_block_elems(fmt);
    if (!be) return -1;
    (void)M;
    size_t bb = orc_block_bytes(fmt);
    int64_t bpr = (K + be - 1) / be;
    const uint8_t* A = (const uint8_t*)a_q;
    for (int64_t i = row0; i < row1; ++i)
        for (int64_t j = 0; j < N; ++j) {
            float sum = 0.0f;
            for (int64_t bk = 0; bk < bpr; ++bk) {
                const uint8_t* blk = A + (size_t)(i * bpr + bk) * bb;
                for (int s = 0; s < be; ++s) {
                    int e = (fmt == ORC_Q6_K) ? q6_visit(s) : s;
                    int64_t k = bk * be + e;
                    if (k >= K) continue;
                    /* Q6_K's `d * sc * q * b` is ((d*sc)*q)*b: decode_elem
                     * already returns (d*sc)*q, so one form covers all. */
                    float w = decode_elem(fmt, blk, e);
                    sum += w * b[k * N + j];
                }
            }
            out[i * N + j] = sum;
        }
    return 0;
}

int orc_matmul(int fmt, const void* a_q, const float* b, float* out,
               int64_t M, int64_t K, int64_t N) {
    return orc_matmul_rows(fmt, a_q, b, out, M, K, N, 0, M);
}

int orc_matmul_f64(int fmt, const void* a_q, const float* b, double* out,
                   int64_t M, int64_t K, int64_t N) {
    int be = orc_block_elems(fmt);
    if (!be) return -1;
    float* w = (float*)malloc(sizeof(float) * (size_t)K);
    if (!w) return -2;
    size_t row_bytes = orc_quantized_size_2d(1, K, fmt);
    for (int64_t i = 0; i < M; ++i) {
        orc_dequantize(fmt, (const uint8_t*)a_q + (size_t)i * row_bytes, 1, K, w);
        for (int64_t j = 0; j < N; ++j) {
            double s = 0.0;
            for (int64_t k = 0; k < K; ++k) s += (double)w[k] * (double)b[k * N + j];
            out[i * N + j] = s;
        }
    }
    free(w);
    return 0;
}
