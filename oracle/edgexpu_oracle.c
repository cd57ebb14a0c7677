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

size_t eo_block_bytes(uint32_t type) {
    switch (type) {
        case EO_TYPE_Q4_0: return EO_Q4_0_BYTES;
        case EO_TYPE_Q5_0: return EO_Q5_0_BYTES;
        case EO_TYPE_Q8_0: return EO_Q8_0_BYTES;
        case EO_TYPE_Q4_K: return EO_Q4_K_BYTES;
        case EO_TYPE_Q5_K: return EO_Q5_K_BYTES;
        case EO_TYPE_Q6_K: return EO_Q6_K_BYTES;
        default: return 0;
    }
}

int eo_block_elems(uint32_t type) {
    switch (type) {
        case EO_TYPE_Q4_0:
        case EO_TYPE_Q5_0:
        case EO_TYPE_Q8_0: return EO_QK8_0;
        case EO_TYPE_Q4_K:
        case EO_TYPE_Q5_K:
        case EO_TYPE_Q6_K: return EO_QK_K;
        default: return 0;
    }
}

/* gguf_quant.c:468-480 (edgexpu_gguf_row_bytes) for the quantized types of the path. */
size_t eo_row_bytes(uint32_t type, int n) {
    int qk = eo_block_elems(type);
    if (n <= 0 || qk == 0 || n % qk != 0) {
        return 0;
    }
    return (size_t)(n / qk) * eo_block_bytes(type);
}

/* Activation format of the integer dots: Q8_0 for can_dot_q8 types, Q8_K for can_dot_q8k
 * types (gguf_dot_q8.c:414-434, cpu_kernel.c:577-631). */
int eo_act_is_q8_0(uint32_t type) {
    return type == EO_TYPE_Q4_0 || type == EO_TYPE_Q5_0 || type == EO_TYPE_Q8_0;
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

/* ---- per-element integer quant values ------------------------------------------------------
 * The value each integer dot multiplies with the int8 activation, element e of one block. */

/* Q4_K: nibble byte l of group g holds element 64g+l (low half) and 64g+32+l (high half). */
static int q4_k_nibble(const uint8_t *qs, int e) {
    int g = e / 64, l = e % 64;
    return l < 32 ? (qs[g * 32 + l] & 0x0F) : (qs[g * 32 + (l - 32)] >> 4);
}

/* Q4_0 (18 B: fp16 d, 16 nibble bytes): element j < 16 is the low nibble of byte j, element 16+j
 * the high nibble, both offset by 8 (gguf_dot_q8.c:587-592, gguf_quant.c:193-210). */
static int q4_0_value(const uint8_t *blk, int e) {
    const uint8_t *qs = blk + 2;
    return (e < 16 ? (qs[e] & 0x0F) : (qs[e - 16] >> 4)) - 8;
}

/* Q5_0 (22 B: fp16 d, 32 high bits qh, 16 nibble bytes): the fifth bit of element e is bit e of
 * qh; values are offset by 16 (gguf_dot_q8.c:533-540, gguf_quant.c:157-181). */
static int q5_0_value(const uint8_t *blk, int e) {
    uint32_t qh;
    const uint8_t *qs = blk + 6;
    int nib;
    memcpy(&qh, blk + 2, 4);
    nib = e < 16 ? (qs[e] & 0x0F) : (qs[e - 16] >> 4);
    return (nib | (int)(((qh >> e) & 1u) << 4)) - 16;
}

/* Q5_K (176 B: fp16 d, fp16 dmin, 12 scale bytes, qh[32] @16, ql[128] @48): group g = e/64 uses
 * ql bytes 32g.. (low nibbles: sub-block 2g, high: 2g+1) and bit 2g / 2g+1 of qh[l] as the
 * fifth bit (gguf_dot_q8.c:847-860, gguf_quant.c:305-353). */
static int q5_k_value(const uint8_t *blk, int e) {
    int g = e / 64, l = e % 64;
    const uint8_t *qh = blk + 16, *ql = blk + 48 + 32 * g;
    if (l < 32) {
        return (ql[l] & 0x0F) + (((qh[l] >> (2 * g)) & 1) << 4);
    }
    return (ql[l - 32] >> 4) + (((qh[l - 32] >> (2 * g + 1)) & 1) << 4);
}

/* Q6_K (210 B: ql[128], qh[64] @128, int8 scales[16] @192, fp16 d @208): half n = e/128 uses
 * ql[64n..], qh[32n..]; quarter q of the half takes the low/high nibble of ql[l] or ql[l+32]
 * and bits 2q..2q+1 of qh[l]; values are offset by 32 (gguf_dot_q8.c:972-982,
 * gguf_quant.c:269-303). */
static int q6_k_value(const uint8_t *blk, int e) {
    int n = e / 128, r = e % 128, q = r / 32, l = r % 32;
    const uint8_t *ql = blk + 64 * n, *qh = blk + 128 + 32 * n;
    int lo = (q & 1) ? ql[l + 32] : ql[l];
    int nib = (q & 2) ? (lo >> 4) : (lo & 0x0F);
    return (nib | (((qh[l] >> (2 * q)) & 3) << 4)) - 32;
}

/* Weight value of element e of a 32-element block (Q8_0 / Q4_0 / Q5_0). */
static int b32_value(uint32_t type, const uint8_t *blk, int e) {
    if (type == EO_TYPE_Q8_0) {
        return (int8_t)blk[2 + e];
    }
    return type == EO_TYPE_Q4_0 ? q4_0_value(blk, e) : q5_0_value(blk, e);
}

/* Unsigned quant value of element e of a Q4_K / Q5_K super-block (the mins are separate). */
static int kmin_value(uint32_t type, const uint8_t *blk, int e) {
    return type == EO_TYPE_Q4_K ? q4_k_nibble(blk + 16, e) : q5_k_value(blk, e);
}

/* ---- integer partials ------------------------------------------------------------------------ */

int eo_partials_b32(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n, int32_t *ip) {
    size_t bb = eo_block_bytes(type);
    int b, j;
    if (wrow == NULL || xq == NULL || ip == NULL || !eo_act_is_q8_0(type) || eo_row_bytes(type, n) == 0) {
        return 0;
    }
    for (b = 0; b < n / EO_QK8_0; b++) {
        const uint8_t *wb = wrow + (size_t)b * bb;
        const int8_t *aq = (const int8_t *)(xq + (size_t)b * EO_Q8_0_BYTES + 2);
        int32_t s = 0;
        for (j = 0; j < EO_QK8_0; j++) {
            s += (int32_t)b32_value(type, wb, j) * (int32_t)aq[j];
        }
        ip[b] = s;
    }
    return 1;
}

int eo_partials_q8_0(const uint8_t *wrow, const uint8_t *xq, int n, int32_t *ip) {
    return eo_partials_b32(EO_TYPE_Q8_0, wrow, xq, n, ip);
}

/* Q4_K / Q5_K: sumi = sum_j sc_j * sum_l q*q8 over the 8 sub-blocks, summ = sum_j m_j * (bsum_2j +
 * bsum_2j+1).  Q6_K: sumi = sum_{j<16} sc_j * sum_l (q-32)*q8 over the 16-element groups, summ = 0.
 * These are the int32 values the reference's SIMD builds form per super-block. */
int eo_partials_k(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n, int32_t *sumi, int32_t *summ) {
    size_t bb = eo_block_bytes(type);
    int b, j, l;
    if (wrow == NULL || xq == NULL || eo_act_is_q8_0(type) || eo_row_bytes(type, n) == 0) {
        return 0;
    }
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * bb;
        const uint8_t *yb = xq + (size_t)b * EO_Q8_K_BYTES;
        const int8_t *q8 = (const int8_t *)(yb + 4);
        int32_t si = 0, sm = 0;
        if (type == EO_TYPE_Q6_K) {
            const int8_t *sc = (const int8_t *)(blk + 192);
            for (j = 0; j < 16; j++) {
                int32_t ip = 0;
                for (l = 0; l < 16; l++) {
                    ip += (int32_t)q6_k_value(blk, 16 * j + l) * (int32_t)q8[16 * j + l];
                }
                si += (int32_t)sc[j] * ip;
            }
        } else {
            for (j = 0; j < 8; j++) {
                uint8_t sc, mn;
                int32_t ip = 0;
                eo_q4_k_scale_min(blk + 4, j, &sc, &mn);
                for (l = 0; l < 32; l++) {
                    ip += (int32_t)kmin_value(type, blk, 32 * j + l) * (int32_t)q8[32 * j + l];
                }
                si += (int32_t)sc * ip;
                sm += (int32_t)mn * ((int32_t)rd_i16(yb + 260 + 4 * j) + (int32_t)rd_i16(yb + 262 + 4 * j));
            }
        }
        if (sumi) sumi[b] = si;
        if (summ) summ[b] = sm;
    }
    return 1;
}

int eo_partials_q4_k(const uint8_t *wrow, const uint8_t *xq, int n, int32_t *sumi, int32_t *summ) {
    return eo_partials_k(EO_TYPE_Q4_K, wrow, xq, n, sumi, summ);
}

/* ---- float dots with quantized activations (the reference's scalar accumulation order) ---- */

/* gguf_dot_q8.c:467-478 (Q8_0), :529-548 (Q5_0), :584-599 (Q4_0): acc += d_w * d_x * (float)ip
 * one block at a time. */
static float dot_b32_q8_0(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n) {
    size_t bb = eo_block_bytes(type);
    int b, j;
    float acc = 0.0f;
    for (b = 0; b < n / EO_QK8_0; b++) {
        const uint8_t *wb = wrow + (size_t)b * bb;
        const uint8_t *xb = xq + (size_t)b * EO_Q8_0_BYTES;
        int32_t ip = 0;
        for (j = 0; j < EO_QK8_0; j++) {
            ip += (int32_t)b32_value(type, wb, j) * (int32_t)(int8_t)xb[2 + j];
        }
        acc += eo_fp16_to_fp32(rd_u16(wb)) * eo_fp16_to_fp32(rd_u16(xb)) * (float)ip;
    }
    return acc;
}

float eo_dot_q8_0_q8_0(const uint8_t *wrow, const uint8_t *xq, int n) {
    if (wrow == NULL || xq == NULL || eo_row_bytes(EO_TYPE_Q8_0, n) == 0) {
        return 0.0f;
    }
    return dot_b32_q8_0(EO_TYPE_Q8_0, wrow, xq, n);
}

/* gguf_dot_q8.c:711-759 (Q4_K) and :838-893 (Q5_K): per super-block subtract dmin*sum(bsums*m),
 * then add d*(sc*ip) per sub-block.  :984-999 (Q6_K): add d*(sc*ip) per 16-element group. */
static float dot_k_q8_k(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n) {
    size_t bb = eo_block_bytes(type);
    int b, j, l;
    float acc = 0.0f;
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * bb;
        const uint8_t *yb = xq + (size_t)b * EO_Q8_K_BYTES;
        const int8_t *q8 = (const int8_t *)(yb + 4);
        if (type == EO_TYPE_Q6_K) {
            const int8_t *sc = (const int8_t *)(blk + 192);
            float d = eo_fp16_to_fp32(rd_u16(blk + 208)) * rd_f32(yb);
            for (j = 0; j < 16; j++) {
                int32_t ip = 0;
                for (l = 0; l < 16; l++) {
                    ip += (int32_t)q8[16 * j + l] * (int32_t)q6_k_value(blk, 16 * j + l);
                }
                acc += d * (float)((int32_t)sc[j] * ip);
            }
            continue;
        }
        {
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
                    ip += (int32_t)q8[32 * j + l] * (int32_t)kmin_value(type, blk, 32 * j + l);
                }
                acc += d * (float)((int32_t)sc * ip);
            }
        }
    }
    return acc;
}

float eo_dot_q4_k_q8_k(const uint8_t *wrow, const uint8_t *xq, int n) {
    if (wrow == NULL || xq == NULL || eo_row_bytes(EO_TYPE_Q4_K, n) == 0) {
        return 0.0f;
    }
    return dot_k_q8_k(EO_TYPE_Q4_K, wrow, xq, n);
}

/* edgexpu_gguf_dot_quant_q8 / _q8k (gguf_dot_q8.c:1004-1044): the Q8_0-activation dot for
 * Q8_0/Q5_0/Q4_0 weights, the Q8_K-activation dot for Q4_K/Q5_K/Q6_K; 0 for anything else. */
float eo_dot_q8(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n) {
    if (wrow == NULL || xq == NULL || eo_row_bytes(type, n) == 0) {
        return 0.0f;
    }
    return eo_act_is_q8_0(type) ? dot_b32_q8_0(type, wrow, xq, n) : dot_k_q8_k(type, wrow, xq, n);
}

/* ---- float dots in the x86 Release build's order (AVX2 + FMA) ----------------------------------
 * The SIMD branches of gguf_dot_q8.c keep 8 float lanes per row; lane m accumulates, block after
 * block, fma(d_block, (float)P_m, lane) where P_m is an exact int32 partial over bytes 4m..4m+3 of
 * each 32-byte group of the block; the lanes are then summed by hsum_float_8 (:125-131).  The Q4_K
 * mins use 4 more lanes, Q5_K a scalar accumulator.  With the same integer partials and the same
 * float steps the result is bit-identical to that build. */

/* hsum_float_8, gguf_dot_q8.c:125-131: ((v0+v4) + (v2+v6)) + ((v1+v5) + (v3+v7)). */
static float hsum8_dot(const float v[8]) {
    float r0 = v[0] + v[4], r1 = v[1] + v[5], r2 = v[2] + v[6], r3 = v[3] + v[7];
    return (r0 + r2) + (r1 + r3);
}

/* hsum256, gguf_quant.c:488-495: ((v0+v4) + (v1+v5)) + ((v2+v6) + (v3+v7)). */
static float hsum8_quant(const float v[8]) {
    float r0 = v[0] + v[4], r1 = v[1] + v[5], r2 = v[2] + v[6], r3 = v[3] + v[7];
    return (r0 + r1) + (r2 + r3);
}

/* Q8_0 / Q4_0 / Q5_0 (gguf_dot_q8.c:440-452, :486-503, :556-569): d = d_w * d_x per block,
 * P_m = sum of the 4 products of elements 4m..4m+3. */
static float dot_b32_x86(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n) {
    size_t bb = eo_block_bytes(type);
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int b, m, k;
    for (b = 0; b < n / EO_QK8_0; b++) {
        const uint8_t *wb = wrow + (size_t)b * bb;
        const uint8_t *xb = xq + (size_t)b * EO_Q8_0_BYTES;
        float d = eo_fp16_to_fp32(rd_u16(wb)) * eo_fp16_to_fp32(rd_u16(xb));
        for (m = 0; m < 8; m++) {
            int32_t p = 0;
            for (k = 0; k < 4; k++) {
                p += (int32_t)b32_value(type, wb, 4 * m + k) * (int32_t)(int8_t)xb[2 + 4 * m + k];
            }
            lane[m] = fmaf(d, (float)p, lane[m]);
        }
    }
    return hsum8_dot(lane);
}

/* Q4_K / Q5_K / Q6_K (gguf_dot_q8.c:612-664, :772-830, :905-963). */
static float dot_k_x86(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n) {
    size_t bb = eo_block_bytes(type);
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float mins[4] = {0, 0, 0, 0};
    float summs = 0.0f;
    int b, m, j, k, t;
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * bb;
        const uint8_t *yb = xq + (size_t)b * EO_Q8_K_BYTES;
        const int8_t *q8 = (const int8_t *)(yb + 4);
        int32_t p[8];
        if (type == EO_TYPE_Q6_K) {
            const int8_t *sc = (const int8_t *)(blk + 192);
            float d = rd_f32(yb) * eo_fp16_to_fp32(rd_u16(blk + 208));
            for (m = 0; m < 8; m++) {
                int32_t acc = 0;
                for (j = 0; j < 2; j++) {          /* 128-element halves */
                    for (k = 0; k < 4; k++) {      /* 32-element groups, scale per 16 */
                        int32_t s = 0;
                        for (t = 0; t < 4; t++) {
                            int e = 128 * j + 32 * k + 4 * m + t;
                            s += (int32_t)(q6_k_value(blk, e) + 32) * (int32_t)q8[e];
                        }
                        acc += (int32_t)sc[8 * j + 2 * k + (m >= 4)] * s;
                    }
                }
                acc -= 32 * ((int32_t)rd_i16(yb + 260 + 4 * m) * (int32_t)sc[2 * m] +
                             (int32_t)rd_i16(yb + 262 + 4 * m) * (int32_t)sc[2 * m + 1]);
                p[m] = acc;
            }
            for (m = 0; m < 8; m++) {
                lane[m] = fmaf(d, (float)p[m], lane[m]);
            }
            continue;
        }
        {
            float d = rd_f32(yb) * eo_fp16_to_fp32(rd_u16(blk));
            float dmin = -rd_f32(yb) * eo_fp16_to_fp32(rd_u16(blk + 2));
            uint8_t sc[8], mn[8];
            int32_t prod[4];
            for (j = 0; j < 8; j++) {
                eo_q4_k_scale_min(blk + 4, j, &sc[j], &mn[j]);
            }
            for (k = 0; k < 4; k++) {
                int32_t s0 = (int32_t)rd_i16(yb + 260 + 8 * k) + (int32_t)rd_i16(yb + 262 + 8 * k);
                int32_t s1 = (int32_t)rd_i16(yb + 264 + 8 * k) + (int32_t)rd_i16(yb + 266 + 8 * k);
                prod[k] = (int32_t)mn[2 * k] * s0 + (int32_t)mn[2 * k + 1] * s1;
            }
            for (m = 0; m < 8; m++) {
                int32_t acc = 0;
                for (j = 0; j < 4; j++) {          /* 64-element groups: low then high nibbles */
                    int32_t lo = 0, hi = 0;
                    for (t = 0; t < 4; t++) {
                        int e = 64 * j + 4 * m + t;
                        lo += (int32_t)kmin_value(type, blk, e) * (int32_t)q8[e];
                        hi += (int32_t)kmin_value(type, blk, e + 32) * (int32_t)q8[e + 32];
                    }
                    acc += (int32_t)sc[2 * j] * lo + (int32_t)sc[2 * j + 1] * hi;
                }
                p[m] = acc;
            }
            if (type == EO_TYPE_Q4_K) {
                for (k = 0; k < 4; k++) {
                    mins[k] = fmaf(dmin, (float)prod[k], mins[k]);
                }
            } else {
                summs += dmin * (float)(prod[0] + prod[1] + prod[2] + prod[3]);
            }
            for (m = 0; m < 8; m++) {
                lane[m] = fmaf(d, (float)p[m], lane[m]);
            }
        }
    }
    if (type == EO_TYPE_Q4_K) {
        /* :659-661: (m0 + m2) + (m1 + m3), added after the lane sum */
        return hsum8_dot(lane) + ((mins[0] + mins[2]) + (mins[1] + mins[3]));
    }
    if (type == EO_TYPE_Q5_K) {
        return hsum8_dot(lane) + summs;
    }
    return hsum8_dot(lane);
}

float eo_dot_q8_x86(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n) {
    if (wrow == NULL || xq == NULL || eo_row_bytes(type, n) == 0) {
        return 0.0f;
    }
    return eo_act_is_q8_0(type) ? dot_b32_x86(type, wrow, xq, n) : dot_k_x86(type, wrow, xq, n);
}

/* fp32 activations in the x86 order: Q4_K (gguf_quant.c:704-752 with the AVX2 dot_u4_f32_32
 * :545-565: per 32 elements 8 fma lanes over 4 steps and 8 add lanes, each reduced by hsum256;
 * acc += d1*qx - m1*sx) and Q8_0 (:628-645: 8 fma lanes per block, acc += d * hsum256).  The
 * other types have no SIMD branch there: their order is eo_dot_f32's. */
float eo_dot_f32_x86(uint32_t type, const uint8_t *wrow, const float *x, int n) {
    int b, j, i, l;
    float acc = 0.0f;
    if (wrow == NULL || x == NULL || eo_row_bytes(type, n) == 0) {
        return 0.0f;
    }
    if (type == EO_TYPE_Q8_0) {
        for (b = 0; b < n / EO_QK8_0; b++) {
            const uint8_t *blk = wrow + (size_t)b * EO_Q8_0_BYTES;
            const float *xx = x + (size_t)b * EO_QK8_0;
            float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (i = 0; i < EO_QK8_0; i += 8) {
                for (l = 0; l < 8; l++) {
                    v[l] = fmaf((float)(int8_t)blk[2 + i + l], xx[i + l], v[l]);
                }
            }
            acc += eo_fp16_to_fp32(rd_u16(blk)) * hsum8_quant(v);
        }
        return acc;
    }
    if (type != EO_TYPE_Q4_K) {
        return eo_dot_f32(type, wrow, x, n);
    }
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q4_K_BYTES;
        const float *xx = x + (size_t)b * EO_QK_K;
        float d = eo_fp16_to_fp32(rd_u16(blk));
        float mn16 = eo_fp16_to_fp32(rd_u16(blk + 2));
        for (j = 0; j < 8; j++) {              /* sub-block j: low nibbles for even j, high for odd */
            uint8_t sc, mn;
            float vq[8] = {0, 0, 0, 0, 0, 0, 0, 0}, vx[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            eo_q4_k_scale_min(blk + 4, j, &sc, &mn);
            for (i = 0; i < 32; i += 8) {
                for (l = 0; l < 8; l++) {
                    float xv = xx[32 * j + i + l];
                    vq[l] = fmaf((float)q4_k_nibble(blk + 16, 32 * j + i + l), xv, vq[l]);
                    vx[l] = vx[l] + xv;
                }
            }
            acc += (d * (float)sc) * hsum8_quant(vq) - (mn16 * (float)mn) * hsum8_quant(vx);
        }
    }
    return acc;
}

/* ---- float dots with fp32 activations (gguf_quant.c, scalar branches) ---------------------- */

/* gguf_quant.c:704-752 (scalar dot_u4_f32_32 :596-600): per sub-block of 32,
 * acc += d*sc * sum(q*x) - dmin*m * sum(x). */
float eo_dot_q4_k_f32(const uint8_t *wrow, const float *x, int n) {
    int b, j, l;
    float acc = 0.0f;
    if (wrow == NULL || x == NULL || eo_row_bytes(EO_TYPE_Q4_K, n) == 0) {
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
    if (wrow == NULL || x == NULL || eo_row_bytes(EO_TYPE_Q8_0, n) == 0) {
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

/* gguf_quant.c:810-835: acc += d*(q_lo-8)*x[j]; acc += d*(q_hi-8)*x[j+16] for j < 16. */
static float dot_q4_0_f32(const uint8_t *wrow, const float *x, int n) {
    int b, j;
    float acc = 0.0f;
    for (b = 0; b < n / EO_QK8_0; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q4_0_BYTES;
        const float *xx = x + (size_t)b * EO_QK8_0;
        float d = eo_fp16_to_fp32(rd_u16(blk));
        for (j = 0; j < 16; j++) {
            acc += d * (float)q4_0_value(blk, j) * xx[j];
            acc += d * (float)q4_0_value(blk, j + 16) * xx[j + 16];
        }
    }
    return acc;
}

/* gguf_quant.c:672-702: acc += d*(x0*x[j] + x1*x[j+16]) for j < 16. */
static float dot_q5_0_f32(const uint8_t *wrow, const float *x, int n) {
    int b, j;
    float acc = 0.0f;
    for (b = 0; b < n / EO_QK8_0; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q5_0_BYTES;
        const float *xx = x + (size_t)b * EO_QK8_0;
        float d = eo_fp16_to_fp32(rd_u16(blk));
        for (j = 0; j < 16; j++) {
            acc += d * ((float)q5_0_value(blk, j) * xx[j] + (float)q5_0_value(blk, j + 16) * xx[j + 16]);
        }
    }
    return acc;
}

/* gguf_quant.c:837-892: per group of 64 and l < 32, acc += (d1*q0 - m1)*x[l];
 * acc += (d2*q1 - m2)*x[l+32]. */
static float dot_q5_k_f32(const uint8_t *wrow, const float *x, int n) {
    int b, g, l;
    float acc = 0.0f;
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q5_K_BYTES;
        const float *xx = x + (size_t)b * EO_QK_K;
        float d = eo_fp16_to_fp32(rd_u16(blk));
        float mn16 = eo_fp16_to_fp32(rd_u16(blk + 2));
        for (g = 0; g < 4; g++) {
            uint8_t sc1, m1, sc2, m2;
            float d1, dm1, d2, dm2;
            eo_q4_k_scale_min(blk + 4, 2 * g, &sc1, &m1);
            eo_q4_k_scale_min(blk + 4, 2 * g + 1, &sc2, &m2);
            d1 = d * (float)sc1;
            dm1 = mn16 * (float)m1;
            d2 = d * (float)sc2;
            dm2 = mn16 * (float)m2;
            for (l = 0; l < 32; l++) {
                acc += (d1 * (float)q5_k_value(blk, 64 * g + l) - dm1) * xx[64 * g + l];
                acc += (d2 * (float)q5_k_value(blk, 64 * g + 32 + l) - dm2) * xx[64 * g + 32 + l];
            }
        }
    }
    return acc;
}

/* gguf_quant.c:754-794: per half and l < 32, acc += d*sc*q*x for the four quarters in order. */
static float dot_q6_k_f32(const uint8_t *wrow, const float *x, int n) {
    int b, h, l, q;
    float acc = 0.0f;
    for (b = 0; b < n / EO_QK_K; b++) {
        const uint8_t *blk = wrow + (size_t)b * EO_Q6_K_BYTES;
        const int8_t *sc = (const int8_t *)(blk + 192);
        const float *xx = x + (size_t)b * EO_QK_K;
        float d = eo_fp16_to_fp32(rd_u16(blk + 208));
        for (h = 0; h < 2; h++) {
            for (l = 0; l < 32; l++) {
                for (q = 0; q < 4; q++) {
                    int e = 128 * h + 32 * q + l;
                    acc += d * (float)sc[8 * h + l / 16 + 2 * q] * (float)q6_k_value(blk, e) * xx[e];
                }
            }
        }
    }
    return acc;
}

/* edgexpu_gguf_dot_quant (gguf_quant.c:894-918) for the quantized types of the path. */
float eo_dot_f32(uint32_t type, const uint8_t *wrow, const float *x, int n) {
    if (wrow == NULL || x == NULL || eo_row_bytes(type, n) == 0) {
        return 0.0f;
    }
    switch (type) {
        case EO_TYPE_Q8_0: return eo_dot_q8_0_f32(wrow, x, n);
        case EO_TYPE_Q4_0: return dot_q4_0_f32(wrow, x, n);
        case EO_TYPE_Q5_0: return dot_q5_0_f32(wrow, x, n);
        case EO_TYPE_Q4_K: return eo_dot_q4_k_f32(wrow, x, n);
        case EO_TYPE_Q5_K: return dot_q5_k_f32(wrow, x, n);
        case EO_TYPE_Q6_K: return dot_q6_k_f32(wrow, x, n);
        default: return 0.0f;
    }
}

/* ---- dequantization (gguf_quant.c:139-353) ------------------------------------------------- */

/* Element e of one block in double, with the (scale * q) and (min) terms returned separately so
 * a caller can form |d*sc*q*x| + |dmin*m*x|.  Float row dequant rounds as the reference does. */
static void block_terms(uint32_t type, const uint8_t *blk, int e, double *scaled_q, double *min_term) {
    *min_term = 0.0;
    switch (type) {
        case EO_TYPE_Q8_0:
        case EO_TYPE_Q4_0:
        case EO_TYPE_Q5_0:
            *scaled_q = (double)eo_fp16_to_fp32(rd_u16(blk)) * b32_value(type, blk, e);
            return;
        case EO_TYPE_Q6_K:
            *scaled_q = (double)eo_fp16_to_fp32(rd_u16(blk + 208)) * (double)(int8_t)blk[192 + e / 16] *
                        q6_k_value(blk, e);
            return;
        default: {
            uint8_t sc, mn;
            eo_q4_k_scale_min(blk + 4, e / 32, &sc, &mn);
            *scaled_q = (double)eo_fp16_to_fp32(rd_u16(blk)) * sc * kmin_value(type, blk, e);
            *min_term = (double)eo_fp16_to_fp32(rd_u16(blk + 2)) * mn;
            return;
        }
    }
}

/* One row to fp32 with the reference's own float expressions (gguf_quant.c:139-155 Q8_0,
 * :157-181 Q5_0, :193-210 Q4_0, :223-266 Q4_K, :269-303 Q6_K, :305-353 Q5_K). */
int eo_dequantize_row(uint32_t type, const uint8_t *wrow, int n, float *dst) {
    size_t bb = eo_block_bytes(type);
    int qk = eo_block_elems(type);
    int b, e;
    if (wrow == NULL || dst == NULL || eo_row_bytes(type, n) == 0) {
        return 0;
    }
    for (b = 0; b < n / qk; b++) {
        const uint8_t *blk = wrow + (size_t)b * bb;
        float *y = dst + (size_t)b * qk;
        for (e = 0; e < qk; e++) {
            switch (type) {
                case EO_TYPE_Q8_0:
                    y[e] = eo_fp16_to_fp32(rd_u16(blk)) * (float)b32_value(type, blk, e);
                    break;
                case EO_TYPE_Q4_0:              /* ((float)q - 8.0f) * d */
                case EO_TYPE_Q5_0:              /* (float)(q - 16) * d */
                    y[e] = (float)b32_value(type, blk, e) * eo_fp16_to_fp32(rd_u16(blk));
                    break;
                case EO_TYPE_Q6_K:              /* d * (float)sc * (float)q */
                    y[e] = eo_fp16_to_fp32(rd_u16(blk + 208)) * (float)(int8_t)blk[192 + e / 16] *
                           (float)q6_k_value(blk, e);
                    break;
                default: {                      /* (d * sc) * q - (dmin * m) */
                    uint8_t sc, mn;
                    eo_q4_k_scale_min(blk + 4, e / 32, &sc, &mn);
                    y[e] = (eo_fp16_to_fp32(rd_u16(blk)) * (float)sc) * (float)kmin_value(type, blk, e) -
                           eo_fp16_to_fp32(rd_u16(blk + 2)) * (float)mn;
                    break;
                }
            }
        }
    }
    return 1;
}

static void dequant_act(uint32_t type, const uint8_t *xq, int n, double *dst) {
    int b, j;
    if (eo_act_is_q8_0(type)) {
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
    size_t bb = eo_block_bytes(type);
    int qk = eo_block_elems(type);
    double acc = 0.0;
    int b, e;
    for (b = 0; b < n / qk; b++) {
        const uint8_t *blk = wrow + (size_t)b * bb;
        for (e = 0; e < qk; e++) {
            double sq, mt, xv = x[(size_t)b * qk + e];
            block_terms(type, blk, e, &sq, &mt);
            acc += fabs(sq * xv) + fabs(mt * xv);
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

size_t eo_act_row_bytes(uint32_t type, int n) {
    return eo_act_is_q8_0(type) ? (size_t)(n / EO_QK8_0) * EO_Q8_0_BYTES
                                : (size_t)(n / EO_QK_K) * EO_Q8_K_BYTES;
}

static uint8_t *quantize_rows(uint32_t type, const float *x, int m, int n) {
    size_t qb = eo_act_row_bytes(type, n);
    uint8_t *xq = (uint8_t *)malloc((size_t)m * qb);
    int t;
    if (xq == NULL) {
        return NULL;
    }
    for (t = 0; t < m; t++) {
        if (eo_act_is_q8_0(type)) {
            eo_quantize_q8_0(x + (size_t)t * n, n, xq + (size_t)t * qb);
        } else {
            eo_quantize_q8_k(x + (size_t)t * n, n, xq + (size_t)t * qb);
        }
    }
    return xq;
}

/* cpu_kernel.c:545-644 for the quantized weight types: quantize each token row once (Q8_0 for
 * Q8_0/Q5_0/Q4_0 weights, Q8_K for Q4_K/Q5_K/Q6_K), then one integer dot per (row, token). */
int eo_linear_quant_batch(float *out, const float *x, const uint8_t *weight, uint32_t type,
                          const float *bias, int m, int n_out, int n_in) {
    size_t rb = eo_row_bytes(type, n_in), qb;
    uint8_t *xq;
    int o;
    if (out == NULL || x == NULL || weight == NULL || m <= 0 || n_out <= 0 || rb == 0) {
        return 0;
    }
    qb = eo_act_row_bytes(type, n_in);
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
            out[(size_t)t * n_out + o] = bv + eo_dot_q8(type, wrow, xq + (size_t)t * qb, n_in);
        }
    }
    free(xq);
    return 1;
}

/* eo_linear_quant_batch with the dots in the x86 Release build's float order: bit-identical to
 * that build's edgexpu_cpu_linear_quant_batch (out = b + dot, cpu_kernel.c:594-597). */
int eo_linear_quant_batch_x86(float *out, const float *x, const uint8_t *weight, uint32_t type,
                              const float *bias, int m, int n_out, int n_in) {
    size_t rb = eo_row_bytes(type, n_in), qb;
    uint8_t *xq;
    int o;
    if (out == NULL || x == NULL || weight == NULL || m <= 0 || n_out <= 0 || rb == 0) {
        return 0;
    }
    qb = eo_act_row_bytes(type, n_in);
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
            out[(size_t)t * n_out + o] = bv + eo_dot_q8_x86(type, wrow, xq + (size_t)t * qb, n_in);
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
    qb = eo_act_row_bytes(type, n_in);
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

/* native.c:2292-2401, greedy branch.  Q8_0-class weights (can_dot_q8: Q8_0, Q5_0, Q4_0) see a
 * Q8_0-quantized hidden state (:2317-2319 -> logit_dot_q8 :464-481); the K-quants see the fp32
 * hidden state through edgexpu_gguf_dot_quant (logit_dot_row :445-462).  Serial semantics of the
 * OpenMP merge (:2373-2383): strictly greater wins, equal scores keep the lowest id, NaN never
 * wins. */
static int logits_argmax(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                         const float *bias, uint32_t *token_id, float *best_score, float *scores, int x86);

int eo_logits_argmax(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd,
                     int vocab, const float *bias, uint32_t *token_id, float *best_score,
                     float *scores) {
    return logits_argmax(weight, type, hidden, n_embd, vocab, bias, token_id, best_score, scores, 0);
}

/* The same with every score in the x86 Release build's float order (bit-identical scores). */
int eo_logits_argmax_x86(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd,
                         int vocab, const float *bias, uint32_t *token_id, float *best_score,
                         float *scores) {
    return logits_argmax(weight, type, hidden, n_embd, vocab, bias, token_id, best_score, scores, 1);
}

static int logits_argmax(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                         const float *bias, uint32_t *token_id, float *best_score, float *scores, int x86) {
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
    if (eo_act_is_q8_0(type)) {
        xq = quantize_rows(type, hidden, 1, n_embd);
        if (xq == NULL) {
            if (scores == NULL) free(sc);
            return 0;
        }
    }
#pragma omp parallel for schedule(static)
    for (i = 0; i < vocab; i++) {
        const uint8_t *wrow = weight + (size_t)i * rb;
        float s = xq != NULL ? (x86 ? eo_dot_q8_x86(type, wrow, xq, n_embd) : eo_dot_q8(type, wrow, xq, n_embd))
                             : (x86 ? eo_dot_f32_x86(type, wrow, hidden, n_embd) : eo_dot_f32(type, wrow, hidden, n_embd));
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
