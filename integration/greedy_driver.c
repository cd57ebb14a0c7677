/*
 * greedy_driver.c -- runs the reference's own native session (src/native.c) over a prompt of token
 * ids and n greedy decode steps, through its public API only:
 *   edgexpu_native_init / _load / _ensure_window  (include/edgexpu/native.h)
 *   session->token_ids / token_count               (the fields edgexpu_native_tokenize fills,
 *                                                   native.c:1349-1384; the prompt is ids here)
 *   edgexpu_native_forward_prefill                 (native.c:2061)
 *   edgexpu_native_generate_next, temperature 0    (native.c:2601-2658: greedy)
 * It is compiled unchanged into both builds of the reference runtime: the CPU build
 * (oracle/_ref/libedgexpu_ref_runtime.so, the reference's ids) and the B200 build
 * (integration/_build/libedgexpu_native_b200.so), so both run the same layer loop and differ only
 * in where the quantized matrix products and the greedy logits run.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "edgexpu/native.h"

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + (double)t.tv_nsec * 1e-9;
}

/* Prefill `prompt` (n_prompt ids), then n_new greedy steps.  out_ids gets the generated ids;
 * hidden (nullable, [n_new][n_embd]) the hidden state each step's logits were taken from;
 * seconds[0] / [1] the prefill and decode wall time.  Returns the number of ids generated (the
 * run stops early only at an end-of-sequence id), or -1 with a message in `error`. */
int edgexpu_generate_run(const char *gguf_path, const uint32_t *prompt, int n_prompt, int n_new, float temperature,
                         float top_p, uint32_t *out_ids, float *hidden, int n_embd, double *seconds, char *error,
                         size_t error_size);

int edgexpu_greedy_run(const char *gguf_path, const uint32_t *prompt, int n_prompt, int n_new, uint32_t *out_ids,
                       float *hidden, int n_embd, double *seconds, char *error, size_t error_size) {
    return edgexpu_generate_run(gguf_path, prompt, n_prompt, n_new, 0.0f, 1.0f, out_ids, hidden, n_embd, seconds, error,
                                error_size);
}

/* As edgexpu_greedy_run, with the sampling settings of edgexpu_native_generate_next: temperature
 * <= 1e-4 is greedy, else softmax sampling with top_p (the session's sampler state carries over
 * between calls in one process, as it does in the reference). */
int edgexpu_generate_run(const char *gguf_path, const uint32_t *prompt, int n_prompt, int n_new, float temperature,
                         float top_p, uint32_t *out_ids, float *hidden, int n_embd, double *seconds, char *error,
                         size_t error_size) {
    edgexpu_native_session *s = (edgexpu_native_session *)calloc(1, sizeof *s);
    double t0, t1;
    int i, made = -1;
    if (s == NULL || gguf_path == NULL || prompt == NULL || n_prompt <= 0 || n_new < 0 || out_ids == NULL) {
        snprintf(error, error_size, "greedy_run: invalid arguments");
        free(s);
        return -1;
    }
    edgexpu_native_init(s);
    if (!edgexpu_native_load(s, gguf_path, error, error_size)) {
        goto done;
    }
    if (hidden != NULL && (int)s->gguf.embedding_length != n_embd) {
        snprintf(error, error_size, "greedy_run: model n_embd %u, caller %d", s->gguf.embedding_length, n_embd);
        goto done;
    }
    if (!edgexpu_native_ensure_window(s, n_prompt, n_new, error, error_size)) {
        goto done;
    }
    memcpy(s->token_ids, prompt, (size_t)n_prompt * sizeof(uint32_t));
    s->token_count = n_prompt;
    t0 = now_s();
    if (!edgexpu_native_forward_prefill(s, error, error_size)) {
        goto done;
    }
    t1 = now_s();
    if (seconds != NULL) {
        seconds[0] = t1 - t0;
    }
    made = 0;
    for (i = 0; i < n_new; i++) {
        int stopped = 0;
        if (hidden != NULL) {
            memcpy(hidden + (size_t)i * n_embd, s->last_hidden, (size_t)n_embd * sizeof(float));
        }
        if (!edgexpu_native_generate_next(s, temperature, top_p, &out_ids[i], NULL, 0, &stopped, error, error_size)) {
            made = -1;
            goto done;
        }
        made = i + 1;
        if (stopped) {
            break;
        }
    }
    if (seconds != NULL) {
        seconds[1] = now_s() - t1;
    }
done:
    edgexpu_native_free(s);
    free(s);
    return made;
}
