/*
 * edgexpu_oracle.h -- CPU restatement of EdgeXPU-LLM's quantized matrix-product path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is compared
 * against.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it;
 * the product (libedgexpu_cuda.so and the C host shim) never links or calls it.
 *
 * Every function restates one reference routine (paths relative to the reference project):
 *   eo_quantize_q8_0        src/gguf_dot_q8.c:269-324  (x86 Release build: AVX2 + F16C branch)
 *   eo_quantize_q8_0_scalar src/gguf_dot_q8.c:325-357  (generic build, truncating fp16 :64-81)
 *   eo_quantize_q8_k        src/gguf_dot_q8.c:360-412
 *   eo_q4_k_scale_min       src/gguf_quant.c:212-220  (== unpack_k4_scales gguf_dot_q8.c:112-124)
 *   eo_dot_q8_0_q8_0        src/gguf_dot_q8.c:436-480  (scalar accumulation order :467-478)
 *   eo_dot_q4_k_q8_k        src/gguf_dot_q8.c:603-762  (scalar accumulation order :711-759)
 *   eo_dot_q4_k_f32         src/gguf_quant.c:704-752 + dot_u4_f32_32 :539-604
 *   eo_dot_q8_0_f32         src/gguf_quant.c:606-670
 *   eo_partials_b32, eo_partials_k, eo_dot_q8
 *                           the integer dots of every quantized type: gguf_dot_q8.c:436-480 (Q8_0),
 *                           :482-550 (Q5_0), :552-601 (Q4_0), :603-762 (Q4_K), :764-895 (Q5_K),
 *                           :897-1002 (Q6_K), dispatch :1004-1044
 *   eo_dot_f32              edgexpu_gguf_dot_quant src/gguf_quant.c:894-918 and the per-type
 *                           scalar dots :606-892
 *   eo_dequantize_row       src/gguf_quant.c:139-353 (one row)
 *   eo_dot_q8_x86           the SIMD branches of gguf_dot_q8.c:436-1002 (AVX2 + FMA float order)
 *   eo_dot_f32_x86          the SIMD branches of gguf_quant.c:539-670 (AVX2 + FMA float order)
 *   eo_linear_quant_batch   src/cpu_kernel.c:545-644
 *   eo_logits_argmax        src/native.c:2292-2401 greedy branch (ties -> lowest id)
 *
 * Integer work (quantized bytes, per-block int32 partials) is bit-exact with the reference's
 * x86 Release build.  Float results follow the reference's scalar accumulation order; the
 * SIMD build sums in a different order, so float comparisons use the tolerance bound
 * eo_abs_bound_* (sum over k of |w_k * x_k|).
 */
#ifndef EDGEXPU_ORACLE_H
#define EDGEXPU_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EO_TYPE_F32 0u
#define EO_TYPE_F16 1u
#define EO_TYPE_Q4_0 2u
#define EO_TYPE_Q5_0 6u
#define EO_TYPE_Q8_0 8u
#define EO_TYPE_Q4_K 12u
#define EO_TYPE_Q5_K 13u
#define EO_TYPE_Q6_K 14u

#define EO_QK8_0 32
#define EO_QK_K 256
#define EO_Q8_0_BYTES 34
#define EO_Q8_K_BYTES 292
#define EO_Q4_K_BYTES 144
#define EO_Q4_0_BYTES 18
#define EO_Q5_0_BYTES 22
#define EO_Q5_K_BYTES 176
#define EO_Q6_K_BYTES 210

uint16_t eo_fp32_to_fp16(float f);          /* IEEE round-to-nearest-even, as F16C */
uint16_t eo_fp32_to_fp16_trunc(float f);    /* the reference's non-F16C fallback */
float eo_fp16_to_fp32(uint16_t h);           /* exact */

size_t eo_block_bytes(uint32_t type);      /* bytes of one GGUF block, 0 if unsupported */
int eo_block_elems(uint32_t type);          /* elements of one GGUF block */
size_t eo_row_bytes(uint32_t type, int n);
int eo_act_is_q8_0(uint32_t type);          /* 1: Q8_0 activations (Q8_0/Q5_0/Q4_0), 0: Q8_K */
size_t eo_act_row_bytes(uint32_t type, int n);

int eo_quantize_q8_0(const float *x, int n, uint8_t *dst);
int eo_quantize_q8_0_scalar(const float *x, int n, uint8_t *dst);
int eo_quantize_q8_k(const float *x, int n, uint8_t *dst);

void eo_q4_k_scale_min(const uint8_t *scales12, int j, uint8_t *sc, uint8_t *mn);

/* Per-block integer partials.  32-element types (Q8_0/Q4_0/Q5_0): ip[b] = sum_{j<32} qw*qx with qw
 * the signed quant value (offset removed).  Q4_K/Q5_K: sumi[b] = sum_j sc_j * ip_j,
 * summ[b] = sum_{j<16} bsums_j * m_{j/2}.  Q6_K: sumi[b] = sum_{j<16} sc_j * ip16_j, summ[b] = 0.
 * These are the int32 values every reference build forms. */
int eo_partials_b32(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n, int32_t *ip);
int eo_partials_k(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n, int32_t *sumi, int32_t *summ);
int eo_partials_q8_0(const uint8_t *wrow, const uint8_t *xq, int n, int32_t *ip);
int eo_partials_q4_k(const uint8_t *wrow, const uint8_t *xq, int n, int32_t *sumi, int32_t *summ);

float eo_dot_q8_0_q8_0(const uint8_t *wrow, const uint8_t *xq, int n);
float eo_dot_q4_k_q8_k(const uint8_t *wrow, const uint8_t *xq, int n);
float eo_dot_q4_k_f32(const uint8_t *wrow, const float *x, int n);
float eo_dot_q8_0_f32(const uint8_t *wrow, const float *x, int n);
float eo_dot_q8(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n);
float eo_dot_f32(uint32_t type, const uint8_t *wrow, const float *x, int n);
/* The same dots in the float order of the reference's x86 Release build (AVX2 + FMA SIMD
 * branches): bit-identical to that build's results. */
float eo_dot_q8_x86(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n);
float eo_dot_f32_x86(uint32_t type, const uint8_t *wrow, const float *x, int n);

/* Tolerance bounds: sum_k |w_k * x_k| with w dequantized and x either the dequantized
 * quantized activation (q8 variants) or the fp32 activation (f32 variant). */
double eo_abs_bound_q8(uint32_t type, const uint8_t *wrow, const uint8_t *xq, int n);
double eo_abs_bound_f32(uint32_t type, const uint8_t *wrow, const float *x, int n);

int eo_dequantize_row(uint32_t type, const uint8_t *wrow, int n, float *dst);

/* out[t*n_out + o] = bias[o] + dot(W_o, quantize(x_t)); returns 0 for unsupported types. */
int eo_linear_quant_batch(float *out, const float *x, const uint8_t *weight, uint32_t type,
                          const float *bias, int m, int n_out, int n_in);
/* The same in the x86 Release build's float order: bit-identical to that build's linear. */
int eo_linear_quant_batch_x86(float *out, const float *x, const uint8_t *weight, uint32_t type,
                              const float *bias, int m, int n_out, int n_in);
/* Same as eo_linear_quant_batch but also returns the per-(token, row) tolerance bound. */
int eo_linear_quant_batch_bound(double *bound, const float *x, const uint8_t *weight, uint32_t type,
                                int m, int n_out, int n_in);

/* Greedy logits: argmax_i (dot(W_i, h) + bias_i), lowest id on ties, NaN scores skipped. */
int eo_logits_argmax(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd,
                     int vocab, const float *bias, uint32_t *token_id, float *best_score,
                     float *scores);

/* The same with the scores in the x86 Release build's float order. */
int eo_logits_argmax_x86(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd,
                         int vocab, const float *bias, uint32_t *token_id, float *best_score,
                         float *scores);

#ifdef __cplusplus
}
#endif

#endif
