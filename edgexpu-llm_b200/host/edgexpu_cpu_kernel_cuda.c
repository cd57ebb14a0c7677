/*
 * edgexpu_cpu_kernel_cuda.c -- C host shim: the reference's quantized-linear and activation
 * quantizer entry points, forwarding to the CUDA C ABI.  See include/edgexpu_b200_host.h.
 *
 * Reference counterparts (inside the reference project):
 *   edgexpu_cpu_linear_quant_batch  src/cpu_kernel.c:545-644
 *   edgexpu_cpu_linear_quant        src/cpu_kernel.c:646-656
 *   edgexpu_gguf_quantize_q8_0/_k   src/gguf_dot_q8.c:269-412
 *   edgexpu_gguf_q8_0/_k_nbytes     src/gguf_dot_q8.c:255-267
 *   edgexpu_gguf_can_dot_q8(k)      src/gguf_dot_q8.c:414-434
 *   edgexpu_gguf_dot_quant_q8(k)    src/gguf_dot_q8.c:1004-1044
 *   edgexpu_gguf_dot_quant          src/gguf_quant.c:894-918
 */
#include "../../include/edgexpu_b200_host.h"

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/edgexpu_cuda.h"

#define GGUF_TYPE_F32 0u
#define GGUF_TYPE_F16 1u
#define GGUF_TYPE_Q4_0 2u
#define GGUF_TYPE_Q5_0 6u
#define GGUF_TYPE_Q8_0 8u
#define GGUF_TYPE_Q4_K 12u
#define GGUF_TYPE_Q5_K 13u
#define GGUF_TYPE_Q6_K 14u

static char g_sticky[512];

static void record(const char *what, const char *msg) {
    if (g_sticky[0] == '\0') {
        snprintf(g_sticky, sizeof g_sticky, "%s: %s", what, msg);
    }
}

static void fill_nan(float *out, size_t n) {
    size_t i;
    for (i = 0; i < n; i++) {
        out[i] = NAN;
    }
}

int edgexpu_b200_init(int device, char *error, size_t error_size) {
    return edgexpu_cuda_init(device, error, error_size);
}

/* ---- weight residency: host tensor bytes -> device handle, uploaded once ------------------
 * Open-addressed table keyed by the host address of a tensor's first byte (the reference's mmap
 * offset).  Entries are released by address range when the model file is unmapped. */
typedef struct {
    const uint8_t *host;
    const uint8_t *dev;
    size_t nbytes;
    uint32_t type;
    int n_out;
    int n_in;
    int preloaded; /* part of a model loaded by edgexpu_b200_preload: freed with the model */
} resident_entry;

static resident_entry *g_res;
static size_t g_res_cap;
static size_t g_res_used;

/* Models loaded by edgexpu_b200_preload, by the host range of their file mapping. */
#define MAX_PRELOADED 16
static struct {
    const uint8_t *base;
    size_t size;
    void *model;
} g_models[MAX_PRELOADED];

static size_t res_slot(const uint8_t *host) {
    uint64_t h = (uint64_t)(uintptr_t)host;
    h ^= h >> 33;
    h *= 0xff51afd7ed558ccdull;
    h ^= h >> 33;
    return (size_t)h & (g_res_cap - 1);
}

static int res_grow(void) {
    size_t old_cap = g_res_cap, i;
    resident_entry *old = g_res;
    size_t cap = old_cap ? 2 * old_cap : 1024;
    resident_entry *t = (resident_entry *)calloc(cap, sizeof *t);
    if (t == NULL) {
        return 0;
    }
    g_res = t;
    g_res_cap = cap;
    g_res_used = 0;
    for (i = 0; i < old_cap; i++) {
        if (old[i].host != NULL) {
            size_t k = res_slot(old[i].host);
            while (g_res[k].host != NULL) {
                k = (k + 1) & (cap - 1);
            }
            g_res[k] = old[i];
            g_res_used++;
        }
    }
    free(old);
    return 1;
}

/* Insert host -> dev (the table has room: callers grow it first). */
static void res_insert(const uint8_t *host, const uint8_t *dev, size_t nbytes, uint32_t type, int n_out, int n_in,
                       int preloaded) {
    size_t k = res_slot(host);
    while (g_res[k].host != NULL) {
        k = (k + 1) & (g_res_cap - 1);
    }
    g_res[k].host = host;
    g_res[k].dev = dev;
    g_res[k].nbytes = nbytes;
    g_res[k].type = type;
    g_res[k].n_out = n_out;
    g_res[k].n_in = n_in;
    g_res[k].preloaded = preloaded;
    g_res_used++;
}

static int res_find(const uint8_t *host) {
    size_t k;
    if (g_res_cap == 0) {
        return 0;
    }
    for (k = res_slot(host); g_res[k].host != NULL; k = (k + 1) & (g_res_cap - 1)) {
        if (g_res[k].host == host) {
            return 1;
        }
    }
    return 0;
}

/* Binds the library to EDGEXPU_B200_DEVICE (default 0) on first use; edgexpu_cuda_init returns 1
 * at once when this process already bound that device. */
static int ensure_device(char *error, size_t error_size) {
    const char *env = getenv("EDGEXPU_B200_DEVICE");
    if (edgexpu_cuda_abi_version() != EDGEXPU_CUDA_ABI_VERSION) {
        snprintf(error, error_size, "libedgexpu_cuda ABI %d, expected %d", edgexpu_cuda_abi_version(),
                 EDGEXPU_CUDA_ABI_VERSION);
        return 0;
    }
    return edgexpu_cuda_init(env != NULL ? atoi(env) : 0, error, error_size);
}

const uint8_t *edgexpu_b200_resident(const uint8_t *host, size_t nbytes, uint32_t type, int n_out, int n_in,
                                     char *error, size_t error_size) {
    const uint8_t *dev = NULL;
    size_t k;
    if (host == NULL || nbytes == 0 || n_out <= 0 || n_in <= 0) {
        if (error != NULL && error_size > 0) {
            snprintf(error, error_size, "resident: invalid tensor arguments");
        }
        return NULL;
    }
    if (g_res_cap != 0) {
        for (k = res_slot(host); g_res[k].host != NULL; k = (k + 1) & (g_res_cap - 1)) {
            if (g_res[k].host == host) {
                resident_entry *e = &g_res[k];
                if (e->nbytes == nbytes && e->type == type && e->n_out == n_out && e->n_in == n_in) {
                    return e->dev;
                }
                snprintf(error, error_size, "resident: tensor at %p was uploaded with another shape or type", host);
                return NULL;
            }
        }
    }
    if (!ensure_device(error, error_size)) {
        return NULL;
    }
    if ((g_res_used + 1) * 2 > g_res_cap && !res_grow()) {
        snprintf(error, error_size, "resident: out of host memory");
        return NULL;
    }
    if (!edgexpu_cuda_upload_weight(host, nbytes, type, n_out, n_in, &dev, error, error_size)) {
        return NULL;
    }
    res_insert(host, dev, nbytes, type, n_out, n_in, 0);
    return dev;
}

int edgexpu_b200_preload(const uint8_t *file_map, size_t file_size, const char *path, int window, char *error,
                         size_t error_size) {
    void *model = NULL;
    int i, n, slot = -1;
    if (file_map == NULL || file_size == 0 || path == NULL) {
        snprintf(error, error_size, "preload: invalid arguments");
        return 0;
    }
    for (i = 0; i < MAX_PRELOADED; i++) {
        if (g_models[i].model == NULL) {
            slot = i;
            break;
        }
    }
    if (slot < 0) {
        snprintf(error, error_size, "preload: more than %d models loaded", MAX_PRELOADED);
        return 0;
    }
    if (!ensure_device(error, error_size) || !edgexpu_cuda_gguf_load(path, window, &model, NULL, error, error_size)) {
        return 0;
    }
    n = edgexpu_cuda_gguf_tensor_count(model);
    for (i = 0; i < n; i++) {
        const uint8_t *dev = NULL;
        uint32_t type = 0;
        int64_t n_in = 0, n_out = 0;
        uint64_t off = 0, nbytes = 0;
        if (!edgexpu_cuda_gguf_tensor_at(model, i, NULL, &dev, &type, &n_in, &n_out, &off, &nbytes) || nbytes == 0 ||
            off + nbytes > file_size || res_find(file_map + off)) {
            continue;
        }
        if ((g_res_used + 1) * 2 > g_res_cap && !res_grow()) {
            edgexpu_cuda_gguf_free(model);
            snprintf(error, error_size, "preload: out of host memory");
            return 0;
        }
        res_insert(file_map + off, dev, (size_t)nbytes, type, (int)n_out, (int)n_in, 1);
    }
    g_models[slot].base = file_map;
    g_models[slot].size = file_size;
    g_models[slot].model = model;
    return 1;
}

void edgexpu_b200_release_range(const void *base, size_t size) {
    const uint8_t *lo = (const uint8_t *)base;
    size_t i;
    resident_entry *old = g_res;
    size_t cap = g_res_cap;
    if (base == NULL || size == 0) {
        return;
    }
    /* rebuild the table without the released entries (keeps the probe chains intact) */
    g_res = cap != 0 ? (resident_entry *)calloc(cap, sizeof *g_res) : NULL;
    if (cap != 0 && g_res == NULL) {
        g_res = old;
        return;
    }
    g_res_used = 0;
    for (i = 0; i < cap; i++) {
        if (old[i].host == NULL) {
            continue;
        }
        if (old[i].host >= lo && old[i].host < lo + size) {
            if (!old[i].preloaded) {
                edgexpu_cuda_free_weight(old[i].dev);
            }
            continue;
        }
        {
            size_t k = res_slot(old[i].host);
            while (g_res[k].host != NULL) {
                k = (k + 1) & (cap - 1);
            }
            g_res[k] = old[i];
            g_res_used++;
        }
    }
    free(old);
    for (i = 0; i < MAX_PRELOADED; i++) {
        if (g_models[i].model != NULL && g_models[i].base >= lo && g_models[i].base < lo + size) {
            edgexpu_cuda_gguf_free(g_models[i].model);
            g_models[i].model = NULL;
        }
    }
}

void edgexpu_b200_shutdown(void) {
    int i;
    for (i = 0; i < MAX_PRELOADED; i++) {
        if (g_models[i].model != NULL) {
            edgexpu_cuda_gguf_free(g_models[i].model);
            g_models[i].model = NULL;
        }
    }
    free(g_res);
    g_res = NULL;
    g_res_cap = 0;
    g_res_used = 0;
    edgexpu_cuda_shutdown();
}

const char *edgexpu_b200_last_error(void) {
    return g_sticky;
}

void edgexpu_b200_clear_error(void) {
    g_sticky[0] = '\0';
}

void edgexpu_cpu_linear_quant_batch(float *out, const float *x, const uint8_t *weight, uint32_t type,
                                    const float *bias, int m, int n_out, int n_in) {
    char err[256];
    if (out == NULL || x == NULL || weight == NULL || m <= 0 || n_out <= 0 || n_in <= 0) {
        return; /* cpu_kernel.c:562-564 */
    }
    if (!edgexpu_cuda_linear_quant_batch(out, x, weight, type, bias, m, n_out, n_in, err, sizeof err)) {
        record("edgexpu_cpu_linear_quant_batch", err);
        fill_nan(out, (size_t)m * (size_t)n_out);
    }
}

void edgexpu_cpu_linear_quant(float *out, const float *x, const uint8_t *weight, uint32_t type, const float *bias,
                              int n_out, int n_in) {
    edgexpu_cpu_linear_quant_batch(out, x, weight, type, bias, 1, n_out, n_in);
}

size_t edgexpu_gguf_q8_0_nbytes(int n) {
    return (n <= 0 || n % 32 != 0) ? 0 : (size_t)(n / 32) * 34u;
}

size_t edgexpu_gguf_q8_k_nbytes(int n) {
    return (n <= 0 || n % 256 != 0) ? 0 : (size_t)(n / 256) * 292u;
}

int edgexpu_gguf_can_dot_q8(uint32_t type) {
    return type == GGUF_TYPE_Q4_0 || type == GGUF_TYPE_Q5_0 || type == GGUF_TYPE_Q8_0;
}

int edgexpu_gguf_can_dot_q8k(uint32_t type) {
    return type == GGUF_TYPE_Q4_K || type == GGUF_TYPE_Q5_K || type == GGUF_TYPE_Q6_K;
}

/* One row through the GPU; NaN and the sticky message if the device call fails. */
static float dot_row(const char *what, uint32_t type, const uint8_t *wrow, const void *x, int quantized, int n) {
    char err[256];
    float r = 0.0f;
    if (!edgexpu_cuda_dot_quant(type, wrow, x, quantized, n, &r, err, sizeof err)) {
        record(what, err);
        return NAN;
    }
    return r;
}

float edgexpu_gguf_dot_quant_q8(uint32_t type, const uint8_t *wrow, const uint8_t *x_q8, int n) {
    if (wrow == NULL || x_q8 == NULL || n <= 0 || n % 32 != 0 || !edgexpu_gguf_can_dot_q8(type)) {
        return 0.0f; /* gguf_dot_q8.c:1010-1022 */
    }
    return dot_row("edgexpu_gguf_dot_quant_q8", type, wrow, x_q8, 1, n);
}

float edgexpu_gguf_dot_quant_q8k(uint32_t type, const uint8_t *wrow, const uint8_t *x_q8k, int n) {
    if (wrow == NULL || x_q8k == NULL || n <= 0 || n % 256 != 0 || !edgexpu_gguf_can_dot_q8k(type)) {
        return 0.0f; /* gguf_dot_q8.c:1031-1043 */
    }
    return dot_row("edgexpu_gguf_dot_quant_q8k", type, wrow, x_q8k, 1, n);
}

float edgexpu_gguf_dot_quant(uint32_t type, const uint8_t *row, const float *x, int n) {
    int block;
    if (row == NULL || x == NULL || n <= 0) {
        return 0.0f; /* gguf_quant.c:895-897 */
    }
    switch (type) {
        case GGUF_TYPE_F32:
        case GGUF_TYPE_F16: block = 1; break;
        case GGUF_TYPE_Q4_0:
        case GGUF_TYPE_Q5_0:
        case GGUF_TYPE_Q8_0: block = 32; break;
        case GGUF_TYPE_Q4_K:
        case GGUF_TYPE_Q5_K:
        case GGUF_TYPE_Q6_K: block = 256; break;
        default: return 0.0f; /* gguf_quant.c:915-916 */
    }
    if (n % block != 0) {
        return 0.0f; /* the per-type dots reject unaligned widths */
    }
    return dot_row("edgexpu_gguf_dot_quant", type, row, x, 0, n);
}

int edgexpu_gguf_quantize_q8_0(const float *x, int n, uint8_t *dst) {
    char err[256];
    if (x == NULL || dst == NULL || n <= 0 || n % 32 != 0) {
        return 0; /* gguf_dot_q8.c:272-274 */
    }
    if (!edgexpu_cuda_quantize_q8_0(x, n, dst, err, sizeof err)) {
        record("edgexpu_gguf_quantize_q8_0", err);
        return 0;
    }
    return 1;
}

int edgexpu_gguf_quantize_q8_k(const float *x, int n, uint8_t *dst) {
    char err[256];
    if (x == NULL || dst == NULL || n <= 0 || n % 256 != 0) {
        return 0; /* gguf_dot_q8.c:363-365 */
    }
    if (!edgexpu_cuda_quantize_q8_k(x, n, dst, err, sizeof err)) {
        record("edgexpu_gguf_quantize_q8_k", err);
        return 0;
    }
    return 1;
}

int edgexpu_b200_logits_greedy(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                               const float *bias, uint32_t *token_id, char *error, size_t error_size) {
    if (weight == NULL || hidden == NULL || token_id == NULL || vocab <= 0) {
        if (error != NULL && error_size > 0) {
            snprintf(error, error_size, "logits: missing weight, hidden state or vocab"); /* as native.c:2313-2315 */
        }
        return 0;
    }
    return edgexpu_cuda_logits_argmax(weight, type, hidden, n_embd, vocab, bias, token_id, NULL, error, error_size);
}

int edgexpu_b200_logits_sample(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                               const float *bias, float temperature, float top_p, uint64_t *rng, uint32_t *token_id,
                               char *error, size_t error_size) {
    if (weight == NULL || hidden == NULL || token_id == NULL || rng == NULL || vocab <= 0) {
        if (error != NULL && error_size > 0) {
            snprintf(error, error_size, "logits: missing weight, hidden state or vocab"); /* as native.c:2313-2315 */
        }
        return 0;
    }
    return edgexpu_cuda_logits_sample(weight, type, hidden, n_embd, vocab, bias, temperature, top_p, rng, token_id,
                                      error, error_size);
}
