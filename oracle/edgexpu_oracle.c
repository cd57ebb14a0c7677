/*
 * edgexpu_oracle.c -- CPU restatement of EdgeXPU-LLM's quantized matrix-product path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).  See
 * edgexpu_oracle.h for the reference routine each function restates.  Block layouts
 * (GGUF, "same as llama.cpp" per the reference's gguf_quant.c:8):
 *   Q8_0  34 B : fp16 d @0, int8 qs[32] @2                      (gguf_dot_q8.c:90-96)
 *   Q8_K  292 B: fp32 d @0, int8 qs[256] @4, int16 bsums[16] @260 (gguf_dot_q8.c:98-110)
 *   Q4_K  144 B: fp16 d @0, fp16 dmin @2, 12 B 6-bit scales/mins @4, 128 B nibbles @16
 *                (gguf_quant.c:223-266; nibble byte l of group g holds element 64g+l in the
 *                low half and element 64g+32+l in the high half)
 */
#include "edgexpu_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static float rd_f32(const uint8_t *p) { float v; memcpy(&v, p, 4); return v; }
static uint16_t rd_u16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
static int16_t rd_i16(const uint8_t *p) { int16_t v; memcpy(&v, p, 2); return v; }

/* IEEE binary32 -> binary16, round to nearest even, with subnormals and overflow to inf.
 * This is what the F16C instruction used by the reference (gguf_dot_q8.c:33-35) computes. */
uint16_t eo_fp32_to_fp16(float f) {
    uint32_t x, sign, ax, e, mant, h, rem, half, shift;
    memcpy(&x, &f, 4);
    sign = (x >> 16) & 0x8000u;
    ax = x & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) {                       /* NaN: quiet, keep top payload bits */
        return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
    }
    if (ax >= 0x477FF000u) {                      /* >= 65520 rounds to infinity */
        return (uint16_t)(sign | 0x7C00u);
    }
    e = ax >> 23;
    if (e >= 113u) {                              /* normal binary16 result */
        mant = ax & 0x7FFFFFu;
        h = ((e - 112u) << 10) | (mant >> 13);
        rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
            h++;                                  /* a carry into the exponent is correct */
        }
        return (uint16_t)(sign | h);
    }
    if (e < 102u) {                               /* below 2^-25: rounds to zero */
        return (uint16_t)sign;
    }
    mant = (ax & 0x7FFFFFu) | 0x800000u;          /* subnormal result, unit 2^-24 */
    shift = 126u - e;                             /* 14 .. 24 */
    h = mant >> shift;
    rem = mant & ((1u << shift) - 1u);
    half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (h & 1u))) {
        h++;
    }
    return (uint16_t)(sign | h);
}

/* The reference's non-F16C conversion (gguf_dot_q8.c:64-81): truncates the mantissa and
 * flushes results below the normal range to signed zero. */
uint16_t eo_fp32_to_fp16_trunc(float f) {
    uint32_t x, sign, mant;
    int32_t e;
    memcpy(&x, &f, 4);
    sign = (x >> 16) & 0x8000u;
    e = (int32_t)((x >> 23) & 0xFFu) - 112;
    mant = x & 0x7FFFFFu;
    if (e <= 0) {
        return (uint16_t)sign;
    }
    if (e >= 31) {
        return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | (mant >> 13));
}

float eo_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    float v;
    if (e == 0) {
        v = ldexpf((float)m, -24);                /* zero or subnormal, exact */
        return sign ? -v : v;
    }
    bits = (e == 31u) ? (sign | 0x7F800000u | (m << 13)) : (sign | ((e + 112u) << 23) | (m << 13));
    memcpy(&v, &bits, 4);
    return v;
}

size_t eo_row_bytes(uint32_t type, int n) {
    if (n <= 0) {
        return 0;
    }
    switch (type) {
        case EO_TYPE_Q8_0:
            return (n % EO_QK8_0) ? 0 : (size_t)(n / EO_QK8_0) * EO_Q8_0_BYTES;
        case EO_TYPE_Q4_K:
            return (n % EO_QK_K) ? 0 : (size_t)(n / EO_QK_K) * EO_Q4_K_BYTES;
        default:
            return 0;
    }
}

/* Reference x86 Release path (gguf_dot_q8.c:276-324): d = amax/127 rounded to fp16 (RNE),
 * id = 127/amax (not 1/d), q = round-half-even(x * id) with int8 saturation (packs). */
int eo_quantize_q8_0(const float *x, int n, uint8_t *dst) {
    int b, i;
    if (x == NULL || dst == NULL || n <= 0 || n % EO_QK8_0 != 0) {
        return 0;
    }
    for (b = 0; b < n / EO_QK8_0; b++) {
        const float *xx = x + (size_t)b * EO_QK8_0;
        uint8_t *blk = dst + (size_t)b * EO_Q8_0_BYTES;
        float amax = 0.0f, d, id;
        uint16_t dh;
        for (i = 0; i < EO_QK8_0; i++) {
            amax = fmaxf(amax, fabsf(xx[i]));
        }
        d = amax / 127.0f;
        id = amax != 0.0f ? 127.0f / amax : 0.0f;
        dh = eo_fp32_to_fp16(d);
        memcpy(blk, &dh, 2);
        for (i = 0; i < EO_QK8_0; i++) {
            float p = xx[i] * id;
            float r = nearbyintf(p);              /* default rounding mode: half to even */
            int v;
            if (isnan(r) || r < -128.0f) {
                v = -128;                         /* cvtps_epi32 gives INT_MIN, packs saturates */
            } else if (r > 127.0f) {
                v = 127;
            } else {
                v = (int)r;
            }
            blk[2 + i] = (uint8_t)(int8_t)v;
        }
    }
    return 1;
}

/* Reference generic build (gguf_dot_q8.c:325-357): id = 1/d, lrintf, clamp to +-127, and the
 * truncating fp16 conversion.  Produces different bytes from the x86 Release path. */
int eo_quantize_q8_0_scalar(const float *x, int n, uint8_t *dst) {
    int b, i;
    if (x == NULL || dst == NULL || n <= 0 || n % EO_QK8_0 != 0) {
        return 0;
    }
    for (b = 0; b < n / EO_QK8_0; b++) {
        const float *xx = x + (size_t)b * EO_QK8_0;
        uint8_t *blk = dst + (size_t)b * EO_Q8_0_BYTES;
        float amax = 0.0f, d, id;
        uint16_t dh;
        for (i = 0; i < EO_QK8_0; i++) {
            float ax = fabsf(xx[i]);
            if (ax > amax) {
                amax = ax;
            }
        }
        d = amax / 127.0f;
        id = d > 0.0f ? 1.0f / d : 0.0f;
        dh = eo_fp32_to_fp16_trunc(d);
        memcpy(blk, &dh, 2);
        for (i = 0; i < EO_QK8_0; i++) {
            int v = (int)lrintf(xx[i] * id);
            v = v > 127 ? 127 : (v < -127 ? -127 : v);
            blk[2 + i] = (uint8_t)(int8_t)v;
        }
    }
    return 1;
}

/* gguf_dot_q8.c:360-412: the block scale comes from the SIGNED value of the first element
 * with the largest |x| (strict '>' keeps the first); all-zero blocks are written as zeros. */
int eo_quantize_q8_k(const float *x, int n, uint8_t *dst) {
    int b, j, g;
    if (x == NULL || dst == NULL || n <= 0 || n % EO_QK_K != 0) {
        return 0;
    }
    for (b = 0; b < n / EO_QK_K; b++) {
        const float *xx = x + (size_t)b * EO_QK_K;
        uint8_t *blk = dst + (size_t)b * EO_Q8_K_BYTES;
        int8_t q[EO_QK_K];
        int16_t bs[16];
        float amax = 0.0f, maxv = 0.0f, iscale, d;
        for (j = 0; j < EO_QK_K; j++) {
            float ax = fabsf(xx[j]);
            if (ax > amax) {
                amax = ax;
                maxv = xx[j];
            }
        }
        if (amax == 0.0f) {
            memset(blk, 0, EO_Q8_K_BYTES);
            continue;
        }
        iscale = -127.0f / maxv;
        for (j = 0; j < EO_QK_K; j++) {
            int v = (int)lrintf(iscale * xx[j]);
            q[j] = (int8_t)(v > 127 ? 127 : (v < -127 ? -127 : v));
        }
        for (g = 0; g < 16; g++) {
            int s = 0;
            for (j = 0; j < 16; j++) {
                s += q[g * 16 + j];
            }
            bs[g] = (int16_t)s;
        }
        d = 1.0f / iscale;
        memcpy(blk, &d, 4);
        memcpy(blk + 4, q, EO_QK_K);
        memcpy(blk + 4 + EO_QK_K, bs, sizeof(bs));
    }
    return 1;
}

/* 6-bit scale/min of sub-block j (0..7) from the 12 packed bytes (gguf_quant.c:212-220). */
void eo_q4_k_scale_min(const uint8_t *s, int j, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0Fu) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Q4_K nibble of element e (0..255) inside one super-block's 128 quant bytes. */
static int q4_k_nibble(const uint8_t *qs, int e) {
    int g = e / 64, l = e % 64;
    return l < 32 ? (qs[g * 32 + l] & 0x0F) : (qs[g * 32 + (l - 32)] >> 4);
}

int eo_partials_q8_0(const uint8_t *wrow, const uint8_t *xq, int n, int32_t *ip) {
    int b, j;
    if (wrow == NULL || xq == NULL || ip == NULL || n <= 0 || n % EO_QK8_0 != 0) {
        return 0;
    }
    for (b = 0; b < n / EO_QK8_0; b++) {
        const int8_t *wq = (const int8_t *)(wrow + (size_t)b * EO_Q8_0_BYTES + 2);
        const int8_t *aq = (const int8_t *)(xq + (size_t)b * EO_Q8_0_BYTES + 2);
        int32_t s = 0;
        for (j = 0; j < EO_QK8_0; j++) {
            s += (int32_t)wq[j] * (int32_t)aq[j];
        }
        ip[b] = s;
    }
    return 1;
}

int eo_partials_q4_k(const uint8_t *wrow, const uint8_t *xq, int n, int32_t *sumi, int32_t *summ) {
    int b, j, l;
    if (wrow == NULL || xq == NULL || n <= 0 || n % EO_QK_K != 0) {
        return 0;
    }
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q4_K_BYTES;
        const uint8_t *yb = xq + (size_t)b * EO_Q8_K_BYTES;
        const int8_t *q8 = (const int8_t *)(yb + 4);
        int32_t si = 0, sm = 0;
        for (j = 0; j < 8; j++) {
            uint8_t sc, mn;
            int32_t ip = 0;
            eo_q4_k_scale_min(blk + 4, j, &sc, &mn);
            for (l = 0; l < 32; l++) {
                ip += (int32_t)q4_k_nibble(blk + 16, 32 * j + l) * (int32_t)q8[32 * j + l];
            }
            si += (int32_t)sc * ip;
            sm += (int32_t)mn * ((int32_t)rd_i16(yb + 260 + 4 * j) + (int32_t)rd_i16(yb + 262 + 4 * j));
        }
        if (sumi) sumi[b] = si;
        if (summ) summ[b] = sm;
    }
    return 1;
}

/* gguf_dot_q8.c:467-478: acc += d_w * d_x * (float)ip, one block at a time. */
float eo_dot_q8_0_q8_0(const uint8_t *wrow, const uint8_t *xq, int n) {
    int b, j;
    float acc = 0.0f;
    if (wrow == NULL || xq == NULL || n <= 0 || n % EO_QK8_0 != 0) {
        return 0.0f;
    }
    for (b = 0; b < n / EO_QK8_0; b++) {
        const uint8_t *wb = wrow + (size_t)b * EO_Q8_0_BYTES;
        const uint8_t *xb = xq + (size_t)b * EO_Q8_0_BYTES;
        int32_t ip = 0;
        for (j = 0; j < EO_QK8_0; j++) {
            ip += (int32_t)(int8_t)wb[2 + j] * (int32_t)(int8_t)xb[2 + j];
        }
        acc += eo_fp16_to_fp32(rd_u16(wb)) * eo_fp16_to_fp32(rd_u16(xb)) * (float)ip;
    }
    return acc;
}

/* gguf_dot_q8.c:711-759: per super-block subtract dmin*sum(bsums*m), then add d*(sc*ip) per
 * sub-block. */
float eo_dot_q4_k_q8_k(const uint8_t *wrow, const uint8_t *xq, int n) {
    int b, j, l;
    float acc = 0.0f;
    if (wrow == NULL || xq == NULL || n <= 0 || n % EO_QK_K != 0) {
        return 0.0f;
    }
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q4_K_BYTES;
        const uint8_t *yb = xq + (size_t)b * EO_Q8_K_BYTES;
        const int8_t *q8 = (const int8_t *)(yb + 4);
        float d = eo_fp16_to_fp32(rd_u16(blk)) * rd_f32(yb);
        float dmin = eo_fp16_to_fp32(rd_u16(blk + 2)) * rd_f32(yb);
        int sm = 0;
        for (j = 0; j < 16; j++) {
            uint8_t sc, mn;
            eo_q4_k_scale_min(blk + 4, j / 2, &sc, &mn);
            sm += (int)rd_i16(yb + 260 + 2 * j) * (int)mn;
        }
        acc -= dmin * (float)sm;
        for (j = 0; j < 8; j++) {
            uint8_t sc, mn;
            int32_t ip = 0;
            eo_q4_k_scale_min(blk + 4, j, &sc, &mn);
            for (l = 0; l < 32; l++) {
                ip += (int32_t)q8[32 * j + l] * (int32_t)q4_k_nibble(blk + 16, 32 * j + l);
            }
            acc += d * (float)((int32_t)sc * ip);
        }
    }
    return acc;
}

/* gguf_quant.c:704-752 (scalar dot_u4_f32_32 :596-600): per sub-block of 32,
 * acc += d*sc * sum(q*x) - dmin*m * sum(x). */
float eo_dot_q4_k_f32(const uint8_t *wrow, const float *x, int n) {
    int b, j, l;
    float acc = 0.0f;
    if (wrow == NULL || x == NULL || n <= 0 || n % EO_QK_K != 0) {
        return 0.0f;
    }
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q4_K_BYTES;
        const float *xx = x + (size_t)b * EO_QK_K;
        float d = eo_fp16_to_fp32(rd_u16(blk));
        float mn16 = eo_fp16_to_fp32(rd_u16(blk + 2));
        for (j = 0; j < 8; j++) {
            uint8_t sc, mn;
            float qx = 0.0f, sx = 0.0f;
            eo_q4_k_scale_min(blk + 4, j, &sc, &mn);
            for (l = 0; l < 32; l++) {
                float xv = xx[32 * j + l];
                qx += (float)q4_k_nibble(blk + 16, 32 * j + l) * xv;
                sx += xv;
            }
            acc += (d * (float)sc) * qx - (mn16 * (float)mn) * sx;
        }
    }
    return acc;
}

/* gguf_quant.c:606-670 scalar branch: acc += d * sum(x*q) per block. */
float eo_dot_q8_0_f32(const uint8_t *wrow, const float *x, int n) {
    int b, j;
    float acc = 0.0f;
    if (wrow == NULL || x == NULL || n <= 0 || n % EO_QK8_0 != 0) {
        return 0.0f;
    }
    for (b = 0; b < n / EO_QK8_0; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q8_0_BYTES;
        float s = 0.0f;
        for (j = 0; j < EO_QK8_0; j++) {
            s += x[b * EO_QK8_0 + j] * (float)(int8_t)blk[2 + j];
        }
        acc += eo_fp16_to_fp32(rd_u16(blk)) * s;
    }
    return acc;
}

int eo_dequantize_row(uint32_t type, const uint8_t *wrow, int n, float *dst) {
    int b, j;
    if (wrow == NULL || dst == NULL || eo_row_bytes(type, n) == 0) {
        return 0;
    }
    if (type == EO_TYPE_Q8_0) {                  /* gguf_quant.c:139-155 */
        for (b = 0; b < n / EO_QK8_0; b++) {
            const uint8_t *blk = wrow + (size_t)b * EO_Q8_0_BYTES;
            float d = eo_fp16_to_fp32(rd_u16(blk));
            for (j = 0; j < EO_QK8_0; j++) {
                dst[b * EO_QK8_0 + j] = d * (float)(int8_t)blk[2 + j];
            }
        }
        return 1;
    }
    for (b = 0; b < n / EO_QK_K; b++) {            /* gguf_quant.c:223-266 */
        const uint8_t *blk = wrow + (size_t)b * EO_Q4_K_BYTES;
        float d = eo_fp16_to_fp32(rd_u16(blk));
        float mn16 = eo_fp16_to_fp32(rd_u16(blk + 2));
        for (j = 0; j < EO_QK_K; j++) {
            uint8_t sc, mn;
            eo_q4_k_scale_min(blk + 4, j / 32, &sc, &mn);
            dst[b * EO_QK_K + j] = (d * (float)sc) * (float)q4_k_nibble(blk + 16, j) - mn16 * (float)mn;
        }
    }
    return 1;
}

static void dequant_act(uint32_t type, const uint8_t *xq, int n, double *dst) {
    int b, j;
    if (type == EO_TYPE_Q8_0) {
        for (b = 0; b < n / EO_QK8_0; b++) {
            const uint8_t *blk = xq + (size_t)b * EO_Q8_0_BYTES;
            double d = eo_fp16_to_fp32(rd_u16(blk));
            for (j = 0; j < EO_QK8_0; j++) {
                dst[b * EO_QK8_0 + j] = d * (double)(int8_t)blk[2 + j];
            }
        }
    } else {
        for (b = 0; b < n / EO_QK_K; b++) {
            const uint8_t *blk = xq + (size_t)b * EO_Q8_K_BYTES;
            double d = rd_f32(blk);
            for (j = 0; j < EO_QK_K; j++) {
                dst[b * EO_QK_K + j] = d * (double)(int8_t)blk[4 + j];
            }
        }
    }
}

/* sum_k |w_k * x_k| with the weight dequantized in double (d*sc*q and dmin*m kept separate so
 * the bound also covers the split d*sumi - dmin*summ that every implementation forms). */
static double weight_abs_terms(uint32_t type, const uint8_t *wrow, int n, const double *x) {
    double acc = 0.0;
    int b, j;
    if (type == EO_TYPE_Q8_0) {
        for (b = 0; b < n / EO_QK8_0; b++) {
            const uint8_t *blk = wrow + (size_t)b * EO_Q8_0_BYTES;
            double d = eo_fp16_to_fp32(rd_u16(blk));
            for (j = 0; j < EO_QK8_0; j++) {
                acc += fabs(d * (double)(int8_t)blk[2 + j] * x[b * EO_QK8_0 + j]);
            }
        }
        return acc;
    }
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q4_K_BYTES;
        double d = eo_fp16_to_fp32(rd_u16(blk));
        double mn16 = eo_fp16_to_fp32(rd_u16(blk + 2));
        for (j = 0; j < EO_QK_K; j++) {
            uint8_t sc, mn;
            double xv = x[b * EO_QK_K + j];
            eo_q4_k_scale_min(blk + 4, j / 32, &sc, &mn);
            acc += fabs(d * sc * q4_k_nibble(blk + 16, j) * xv) + fabs(mn16 * mn * xv);
        }
    }
    return acc;
}

double eo_abs_bound_q8(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n) {
    double *xd;
    double r;
    if (eo_row_bytes(type, n) == 0) {
        return 0.0;
    }
    xd = (double *)malloc((size_t)n * sizeof(double));
    if (xd == NULL) {
        return 0.0;
    }
    dequant_act(type, xq, n, xd);
    r = weight_abs_terms(type, wrow, n, xd);
    free(xd);
    return r;
}

double eo_abs_bound_f32(uint32_t type, const uint8_t *wrow, const float *x, int n) {
    double *xd;
    double r;
    int i;
    if (eo_row_bytes(type, n) == 0) {
        return 0.0;
    }
    xd = (double *)malloc((size_t)n * sizeof(double));
    if (xd == NULL) {
        return 0.0;
    }
    for (i = 0; i < n; i++) {
        xd[i] = x[i];
    }
    r = weight_abs_terms(type, wrow, n, xd);
    free(xd);
    return r;
}

static size_t act_bytes(uint32_t type, int n) {
    return type == EO_TYPE_Q8_0 ? (size_t)(n / EO_QK8_0) * EO_Q8_0_BYTES
                                : (size_t)(n / EO_QK_K) * EO_Q8_K_BYTES;
}

static uint8_t *quantize_rows(uint32_t type, const float *x, int m, int n) {
    size_t qb = act_bytes(type, n);
    uint8_t *xq = (uint8_t *)malloc((size_t)m * qb);
    int t;
    if (xq == NULL) {
        return NULL;
    }
    for (t = 0; t < m; t++) {
        if (type == EO_TYPE_Q8_0) {
            eo_quantize_q8_0(x + (size_t)t * n, n, xq + (size_t)t * qb);
        } else {
            eo_quantize_q8_k(x + (size_t)t * n, n, xq + (size_t)t * qb);
        }
    }
    return xq;
}

/* cpu_kernel.c:545-644 for the two in-scope weight types: quantize each token row once
 * (Q8_0 for Q8_0 weights, Q8_K for Q4_K weights), then one integer dot per (row, token). */
int eo_linear_quant_batch(float *out, const float *x, const uint8_t *weight, uint32_t type,
                          const float *bias, int m, int n_out, int n_in) {
    size_t rb = eo_row_bytes(type, n_in), qb;
    uint8_t *xq;
    int o;
    if (out == NULL || x == NULL || weight == NULL || m <= 0 || n_out <= 0 || rb == 0) {
        return 0;
    }
    qb = act_bytes(type, n_in);
    xq = quantize_rows(type, x, m, n_in);
    if (xq == NULL) {
        return 0;
    }
#pragma omp parallel for schedule(static)
    for (o = 0; o < n_out; o++) {
        const uint8_t *wrow = weight + (size_t)o * rb;
        float bv = bias != NULL ? bias[o] : 0.0f;
        int t;
        for (t = 0; t < m; t++) {
            float dot = type == EO_TYPE_Q8_0 ? eo_dot_q8_0_q8_0(wrow, xq + (size_t)t * qb, n_in)
                                             : eo_dot_q4_k_q8_k(wrow, xq + (size_t)t * qb, n_in);
            out[(size_t)t * n_out + o] = bv + dot;
        }
    }
    free(xq);
    return 1;
}

int eo_linear_quant_batch_bound(double *bound, const float *x, const uint8_t *weight, uint32_t type,
                                int m, int n_out, int n_in) {
    size_t rb = eo_row_bytes(type, n_in), qb;
    uint8_t *xq;
    int o;
    if (bound == NULL || x == NULL || weight == NULL || m <= 0 || n_out <= 0 || rb == 0) {
        return 0;
    }
    qb = act_bytes(type, n_in);
    xq = quantize_rows(type, x, m, n_in);
    if (xq == NULL) {
        return 0;
    }
#pragma omp parallel for schedule(static)
    for (o = 0; o < n_out; o++) {
        int t;
        for (t = 0; t < m; t++) {
            bound[(size_t)t * n_out + o] = eo_abs_bound_q8(type, weight + (size_t)o * rb, xq + (size_t)t * qb, n_in);
        }
    }
    free(xq);
    return 1;
}

/* native.c:2292-2401, greedy branch.  Q8_0-class weights see a Q8_0-quantized hidden state
 * (:2317-2319 -> logit_dot_q8 :464-481); Q4_K weights see the fp32 hidden state through
 * dot_q4_k (logit_dot_row :445-462).  Serial semantics of the OpenMP merge (:2373-2383):
 * strictly greater wins, equal scores keep the lowest id, NaN never wins. */
int eo_logits_argmax(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd,
                     int vocab, const float *bias, uint32_t *token_id, float *best_score,
                     float *scores) {
    size_t rb = eo_row_bytes(type, n_embd);
    uint8_t *xq = NULL;
    float *sc;
    float bs = -INFINITY;
    uint32_t best = 0;
    int i;
    if (weight == NULL || hidden == NULL || vocab <= 0 || rb == 0 || token_id == NULL) {
        return 0;
    }
    sc = scores != NULL ? scores : (float *)malloc((size_t)vocab * sizeof(float));
    if (sc == NULL) {
        return 0;
    }
    if (type == EO_TYPE_Q8_0) {
        xq = quantize_rows(type, hidden, 1, n_embd);
        if (xq == NULL) {
            if (scores == NULL) free(sc);
            return 0;
        }
    }
#pragma omp parallel for schedule(static)
    for (i = 0; i < vocab; i++) {
        const uint8_t *wrow = weight + (size_t)i * rb;
        float s = type == EO_TYPE_Q8_0 ? eo_dot_q8_0_q8_0(wrow, xq, n_embd)
                                       : eo_dot_q4_k_f32(wrow, hidden, n_embd);
        if (bias != NULL) {
            s += bias[i];
        }
        sc[i] = s;
    }
    for (i = 0; i < vocab; i++) {
        if (sc[i] > bs) {
            bs = sc[i];
            best = (uint32_t)i;
        }
    }
    *token_id = best;
    if (best_score != NULL) {
        *best_score = bs;
    }
    free(xq);
    if (scores == NULL) {
        free(sc);
    }
    return 1;
}
