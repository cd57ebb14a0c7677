/*
 * ref_driver.c -- drives the REFERENCE's own compiled per-row dots (libedgexpu_ref_*.so) through
 * the greedy logits loop of its src/native.c:2292-2401, which is a static function there and so
 * cannot be called directly.  TEST/BASELINE INFRASTRUCTURE ONLY: used as the reference CPU arm
 * of bench.py and never by the product.
 *
 * The loop keeps the reference's structure: the hidden state is quantized to Q8_0 once when the
 * weight type can take a Q8 dot (native.c:2317-2319), the vocabulary is walked in chunks of
 * 48 MiB of weight rows (native.c:2262-2274, scheduler.h:34), each chunk is split over OpenMP
 * threads with static scheduling, and thread results are merged keeping the higher score and,
 * on equal scores, the lower id (native.c:2364-2385).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "edgexpu/gguf_quant.h"

#define REF_CHUNK_BYTES ((size_t)48u * 1024u * 1024u)

int eoref_logits_greedy(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                        const float *bias, uint32_t *token_id, float *best_score) {
    size_t row_bytes = edgexpu_gguf_row_bytes(type, n_embd);
    size_t chunk;
    uint8_t *xq = NULL;
    uint32_t best = 0;
    float best_s = -INFINITY;
    uint32_t begin;
    if (weight == NULL || hidden == NULL || token_id == NULL || vocab <= 0 || row_bytes == 0) {
        return 0;
    }
    if (edgexpu_gguf_can_dot_q8(type)) {
        xq = (uint8_t *)malloc(edgexpu_gguf_q8_0_nbytes(n_embd));
        if (xq == NULL || !edgexpu_gguf_quantize_q8_0(hidden, n_embd, xq)) {
            free(xq);
            return 0;
        }
    }
    chunk = REF_CHUNK_BYTES / row_bytes;
    if (chunk < 1) {
        chunk = 1;
    }
    for (begin = 0; begin < (uint32_t)vocab; begin += (uint32_t)chunk) {
        uint32_t end = begin + (uint32_t)chunk > (uint32_t)vocab ? (uint32_t)vocab : begin + (uint32_t)chunk;
#pragma omp parallel if ((end - begin) >= 256)
        {
            uint32_t mine = 0;
            float mine_s = -INFINITY;
            uint32_t r;
#pragma omp for nowait schedule(static)
            for (r = begin; r < end; r++) {
                const uint8_t *row = weight + (size_t)r * row_bytes;
                float s = xq != NULL ? edgexpu_gguf_dot_quant_q8(type, row, xq, n_embd)
                                     : edgexpu_gguf_dot_quant(type, row, hidden, n_embd);
                if (bias != NULL) {
                    s += bias[r];
                }
                if (s > mine_s) {
                    mine_s = s;
                    mine = r;
                }
            }
#pragma omp critical
            {
                if (mine_s > best_s || (mine_s == best_s && mine < best)) {
                    best_s = mine_s;
                    best = mine;
                }
            }
        }
    }
    free(xq);
    *token_id = best;
    if (best_score != NULL) {
        *best_score = best_s;
    }
    return 1;
}
