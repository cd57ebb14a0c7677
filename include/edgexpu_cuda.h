/*
 * edgexpu_cuda.h -- C ABI of libedgexpu_cuda.so, the B200 (sm_100a) implementation of
 * EdgeXPU-LLM's quantized matrix-product path.
 *
 * Plain C types only (no CUDA or torch types): pointers, sizes, and `void *stream` (a
 * cudaStream_t; NULL is the CUDA default stream).  Every entry point returns 1 on
 * success and 0 on failure; failures also leave a message in `error` (when given) and in
 * edgexpu_cuda_last_error().  There is no CPU fallback: without a CUDA device every call
 * fails.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   edgexpu_cuda_linear_quant_batch   edgexpu_cpu_linear_quant_batch   include/edgexpu/cpu_kernel.h:71-80
 *                                     (and edgexpu_cpu_linear_quant    include/edgexpu/cpu_kernel.h:60-68)
 *   edgexpu_cuda_quantize_q8_0        edgexpu_gguf_quantize_q8_0       include/edgexpu/gguf_quant.h:80-81
 *   edgexpu_cuda_quantize_q8_k        edgexpu_gguf_quantize_q8_k       include/edgexpu/gguf_quant.h:85-86
 *   edgexpu_cuda_dot_quant_q8_dev     edgexpu_gguf_dot_quant_q8 / _q8k include/edgexpu/gguf_quant.h:90-102
 *                                     (all rows of a tensor in one call)
 *   edgexpu_cuda_logits_argmax        greedy branch of sample_next_token src/native.c:2355-2400
 *                                     (chunk loop + logit_score src/native.c:500-514)
 *   edgexpu_cuda_upload_weight        per-token staging of load_qweight src/native.c:593-655,
 *                                     stage_copy_bytes src/native.c:350-380 (uploaded once instead)
 *   edgexpu_cuda_dot_quant            edgexpu_gguf_dot_quant_q8 / _q8k  include/edgexpu/gguf_quant.h:90-102
 *                                     and edgexpu_gguf_dot_quant        include/edgexpu/gguf_quant.h:72-77
 *                                     (one row, host activations)
 *   edgexpu_cuda_dequantize_row       edgexpu_gguf_dequantize_row       include/edgexpu/gguf_quant.h:50-58
 *   edgexpu_cuda_dequantize_rows_dev  the token-embedding gather of embedding_row src/native.c:428-443
 *                                     (a batch of rows, device buffers)
 *
 * Weight handles: edgexpu_cuda_upload_weight returns a device address (typed const uint8_t *)
 * that callers keep in edgexpu_qweight.data (include/edgexpu/native.h:23-28) in place of the
 * staging pointer.  Any row of a registered tensor may be passed as `weight` (e.g. a vocab
 * chunk or a tensor-parallel shard), with n_out rows from there.
 *
 * Threading: one device per process; calls are serialised internally.  Host-buffer calls are
 * synchronous; *_dev calls are ordered on `stream` and do not synchronise the host.
 */
#ifndef EDGEXPU_CUDA_H
#define EDGEXPU_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EDGEXPU_CUDA_ABI_VERSION 1

/* GGUF type ids, as EDGEXPU_GGUF_TYPE_* in include/edgexpu/gguf_quant.h:17-24.  The quantized
 * matrix product accepts Q8_0, Q5_0 and Q4_0 weights (Q8_0 activations) and Q4_K, Q5_K and Q6_K
 * weights (Q8_K activations), the pairs of edgexpu_gguf_can_dot_q8 / _q8k; F16 and F32 weights are
 * dotted against the fp32 activations, as the reference's linear does for them. */
#define EDGEXPU_CUDA_TYPE_F32 0u
#define EDGEXPU_CUDA_TYPE_F16 1u
#define EDGEXPU_CUDA_TYPE_Q4_0 2u
#define EDGEXPU_CUDA_TYPE_Q5_0 6u
#define EDGEXPU_CUDA_TYPE_Q8_0 8u
#define EDGEXPU_CUDA_TYPE_Q4_K 12u
#define EDGEXPU_CUDA_TYPE_Q5_K 13u
#define EDGEXPU_CUDA_TYPE_Q6_K 14u

int edgexpu_cuda_abi_version(void);

/* Float order of every float output (linear, single-row dots, logits scores).  No counterpart in
 * the reference.
 *   EDGEXPU_CUDA_ORDER_X86 (the default): bit-identical to the reference's x86 Release build
 *     (AVX2 + FMA): the same exact integer partials summed in the same float steps
 *     (gguf_dot_q8.c:436-1002, gguf_quant.c:539-918).  Every GGUF type; batches stream the weight
 *     once per 8 activation rows.
 *   EDGEXPU_CUDA_ORDER_RELAXED: the same integer partials, float sums in the GEMV's own order, within
 *     1e-5 * sum |w*x| of the reference; Q4_K batches of 64 rows and more run on the tensor-core GEMM.
 * Integer outputs (quantized activations, block partials) are bit-exact in both.  Process-wide. */
#define EDGEXPU_CUDA_ORDER_X86 0
#define EDGEXPU_CUDA_ORDER_RELAXED 1
int edgexpu_cuda_set_float_order(int order);
int edgexpu_cuda_float_order(void);

/* Bind the library to CUDA device `device` (creates its stream and scratch). */
int edgexpu_cuda_init(int device, char *error, size_t error_size);
/* Free every uploaded weight and all scratch; the library can be initialised again. */
int edgexpu_cuda_shutdown(void);
/* Last failure message of this process ("" if none). */
const char *edgexpu_cuda_last_error(void);

/* Copy a packed GGUF tensor (n_out rows of n_in elements, native block layout) to HBM once and
 * return its device handle.  Replaces the per-layer, per-token staging memcpy. */
int edgexpu_cuda_upload_weight(const uint8_t *host, size_t nbytes, uint32_t type, int n_out, int n_in,
                               const uint8_t **handle, char *error, size_t error_size);
/* Register device memory the caller already holds (16-byte aligned, with at least 16 readable
 * bytes past the last row) so it can be passed as `weight`. */
int edgexpu_cuda_register_weight(const void *device_ptr, size_t capacity, uint32_t type, int n_out, int n_in,
                                 char *error, size_t error_size);
/* Forget a handle; frees the memory if it came from edgexpu_cuda_upload_weight. */
int edgexpu_cuda_free_weight(const void *handle);

/* ---- host-buffer entry points (synchronous) ---------------------------------------------- */

/* fp32[n] -> Q8_0 blocks (n/32 * 34 bytes), bytes identical to the reference x86 build. */
int edgexpu_cuda_quantize_q8_0(const float *x, int n, uint8_t *dst, char *error, size_t error_size);
/* fp32[n] -> Q8_K blocks (n/256 * 292 bytes), bytes identical to the reference. */
int edgexpu_cuda_quantize_q8_k(const float *x, int n, uint8_t *dst, char *error, size_t error_size);

/* out[t*n_out + o] = bias[o] + dot(W_o, quantize(x_t)) for t < m, o < n_out; x is [m][n_in]
 * row-major, out is [m][n_out]; bias may be NULL.  Q8_0/Q5_0/Q4_0 weights use Q8_0 activations,
 * Q4_K/Q5_K/Q6_K weights use Q8_K activations (cpu_kernel.c:577-631), F16/F32 weights the fp32
 * activations (:633-643).  The GEMV kernel streams the weight once per 8 activation rows; in the
 * relaxed float order Q4_K batches of 64 rows and more (prefill) run as a tensor-core GEMM
 * (tcgen05 kind::i8) with the same integer partials. */
int edgexpu_cuda_linear_quant_batch(float *out, const float *x, const uint8_t *weight, uint32_t type,
                                    const float *bias, int m, int n_out, int n_in, char *error,
                                    size_t error_size);

/* Greedy next token: argmax over rows i < vocab of dot(W_i, hidden) + bias[i], lowest id on
 * ties.  Q8_0 weights see a Q8_0-quantized hidden state, Q4_K weights the fp32 hidden state
 * (native.c:2317-2319, :445-481).  best_score may be NULL. */
int edgexpu_cuda_logits_argmax(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                               const float *bias, uint32_t *token_id, float *best_score, char *error,
                               size_t error_size);

/* One weight row against one activation row: *result = dot(wrow, x) over n elements.
 * x_quantized = 1: x is a quantized activation row (Q8_0 blocks for Q8_0/Q5_0/Q4_0 weights, Q8_K
 * blocks for Q4_K/Q5_K/Q6_K), as edgexpu_gguf_dot_quant_q8 / _q8k; x_quantized = 0: x is fp32, as
 * edgexpu_gguf_dot_quant (any type above, F16/F32 included).  wrow is a row of a registered tensor
 * or host memory (copied for the call). */
int edgexpu_cuda_dot_quant(uint32_t type, const uint8_t *wrow, const void *x, int x_quantized, int n, float *result,
                           char *error, size_t error_size);

/* Row `row` of a registered tensor (handle = its first row) dequantized to n_in fp32 values in dst
 * (host), bit-identical to the reference's dequantizer (gguf_quant.c:139-353). */
int edgexpu_cuda_dequantize_row(const uint8_t *weight, uint32_t type, int64_t row, int n_in, float *dst, char *error,
                                size_t error_size);

/* ---- device-buffer entry points (ordered on `stream`, no host synchronisation) ----------- */

/* out[i][0..n_in) = row ids[i] of the registered tensor `weight` (its handle) dequantized, for
 * i < n_ids (ids: device int32; NULL = rows 0 .. n_ids-1).  An id outside the tensor gives a NaN
 * row and an error from the next edgexpu_cuda_stream_sync. */
int edgexpu_cuda_dequantize_rows_dev(float *out, const uint8_t *weight, uint32_t type, const int32_t *ids, int n_ids,
                                     int n_in, void *stream);

/* Quantize m rows of n fp32 values into the activation format used with `weight_type`. */
int edgexpu_cuda_quantize_dev(uint32_t weight_type, const float *x, int m, int n, uint8_t *dst, void *stream);

int edgexpu_cuda_linear_quant_batch_dev(float *out, const float *x, const uint8_t *weight, uint32_t type,
                                        const float *bias, int m, int n_out, int n_in, void *stream);

/* n (1..4) tensors that read the same activations (q/k/v, or gate/up) in ONE launch:
 * outs[i][t*n_outs[i] + o] = biases[i][o] + dot(W_i,o, quantize(x_t)).  Same results as n calls of
 * edgexpu_cuda_linear_quant_batch_dev; the reference makes those n calls one by one
 * (native.c:2530-2532, :2576-2577), a single launch streams all n weight tensors back to back.
 * outs, weights, n_outs and biases are host arrays of n entries (biases may be NULL). */
int edgexpu_cuda_linear_quant_multi_dev(int n, float *const *outs, const uint8_t *const *weights, const int *n_outs,
                                        const float *const *biases, uint32_t type, const float *x, int m, int n_in,
                                        void *stream);

/* Same result as edgexpu_cuda_linear_quant_batch_dev, but the call allocates no memory: no
 * cudaMalloc, no cudaFree, no allocating library routine.  It has no counterpart in the reference;
 * it is for callers that cannot allocate once running -- runtimes whose HBM budget is fixed at model
 * load, and decode loops that must not risk the device-wide synchronisation an allocation or free can
 * cause.  Batches of one or two rows use no scratch (the GEMV quantizes them itself); larger batches
 * put their quantized activations in one fixed 1 MiB device array compiled into the library (held on
 * every GPU that loads it until exit), so m * (quantized row bytes) must fit in 1 MiB (e.g. 224 rows of
 * 4096 for Q4_K, 60 rows of 16384 for Q8_0); larger batches are rejected with an error.  The first
 * call on a device looks up the array's device address; make it before any stream capture.  All calls
 * share the array, so calls whose GPU work overlaps (two streams at once) race and must be serialised
 * by the caller.  Meant for decode-sized batches: where the regular entry point would run a Q4_K
 * prefill batch on the tensor-core GEMM (relaxed float order), this one streams the weight once per
 * 8 rows. */
int edgexpu_cuda_linear_quant_batch_noalloc(float *out, const float *x, const uint8_t *weight, uint32_t type,
                                            const float *bias, int m, int n_out, int n_in, void *stream);

/* Rows of pre-quantized activations (xq: m rows of Q8_0 or Q8_K blocks, as from
 * edgexpu_cuda_quantize_dev) against n_out weight rows: the batched counterpart of
 * edgexpu_gguf_dot_quant_q8 / _q8k (include/edgexpu/gguf_quant.h:90-102) with the linear
 * epilogue, out[t*n_out + o] = bias[o] + dot(W_o, xq_t). */
int edgexpu_cuda_dot_quant_q8_dev(float *out, const uint8_t *xq, const uint8_t *weight, uint32_t type,
                                  const float *bias, int m, int n_out, int n_in, void *stream);

/* Writes the argmax key of rows [0, vocab) of `weight` into *key (device).  The key packs the
 * order-preserving bits of the best score (high word) and 0xFFFFFFFF - (row0 + row) (low
 * word), so max over keys from several vocab shards is the global greedy choice. */
int edgexpu_cuda_logits_argmax_dev(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                                   const float *bias, int64_t row0, uint64_t *key, void *stream);

/* Test hook: per-block int32 partials of the production kernel (the GEMV, or for Q4_K with
 * m >= 64 the tensor-core GEMM).  xq holds m pre-quantized activation rows.  Q8_0: partials[t][o][b] = ip.  Q4_K: partials[t][o][b][2] = (sumi, summ). */
int edgexpu_cuda_block_partials_dev(int32_t *partials, const uint8_t *xq, const uint8_t *weight, uint32_t type,
                                    int m, int n_out, int n_in, void *stream);

/* Make sure scratch for m activation rows of n_in elements exists (call before graph capture). */
int edgexpu_cuda_reserve(int m, int n_in, char *error, size_t error_size);

/* Wait for `stream`, then report any device-side timeout recorded by the kernels. */
int edgexpu_cuda_stream_sync(void *stream, char *error, size_t error_size);

/* ---- tensor parallelism: column-sharded linear with the all-reduce inside the GEMV ----------
 * No counterpart in the reference (it is single-process).  One process per GPU.  The o and down
 * projections of a tensor-parallel layer shard their weights by input columns (at 256-element
 * block boundaries, so the Q8_K quantization of each shard is that of the full row), so every rank
 * holds a partial of the whole output.  edgexpu_cuda_linear_quant_batch_tp_dev computes this
 * rank's partial and sums the partials of all ranks in the same launch: every partial output is
 * stored, tagged with the launch's epoch in the same 64-bit word, into every rank's exchange
 * region (CUDA IPC mappings over NVLink), and each CTA waits for the tagged partials of its own
 * rows (bounded; a peer that does not deliver within 2 s sets a status error) and adds them in
 * rank order.  Every rank gets the same bits.  Set-up: tp_init on every rank, exchange the handles (EDGEXPU_CUDA_TP_HANDLE_BYTES
 * each) with any host channel, tp_connect with all `world` handles in rank order, then a barrier.
 * All ranks must make the same sequence of _tp_dev calls, one at a time per process. */
#define EDGEXPU_CUDA_TP_HANDLE_BYTES 64
int edgexpu_cuda_tp_init(int world, int rank, uint8_t *handle_out, char *error, size_t error_size);
int edgexpu_cuda_tp_connect(const uint8_t *handles, char *error, size_t error_size);
int edgexpu_cuda_tp_shutdown(void);
/* out[t*n_out + o] = bias[o] + sum over ranks of dot(W_rank,o, quantize(x_rank,t)); `weight` is this
 * rank's column shard (n_out rows of n_in = its share of the input), x this rank's slice of the
 * activations; bias (full, may be NULL) is applied once.  Rows are processed in launches of up to
 * min(the GEMV's row limit, 65536 / n_out); n_out may be at most 65536. */
int edgexpu_cuda_linear_quant_batch_tp_dev(float *out, const float *x, const uint8_t *weight, uint32_t type,
                                           const float *bias, int m, int n_out, int n_in, void *stream);

/* ---- temperature sampling on the device -------------------------------------------------------
 * edgexpu_cpu_sample_softmax (src/cpu_kernel.c:762-849): softmax of logits[n] in place (the
 * probabilities are written back), the reference's xorshift64 step of *rng (seeded with
 * 0x00ED6E50 when 0), then for top_p in (0, 1) the shortest prefix of the ids ordered by
 * probability (descending, ties by ascending id) whose sum reaches top_p, else all ids in order;
 * *out = the first id of that sequence whose running sum reaches u * (its sum), u = the draw in
 * [0, 1).  Sums in double as the reference's, in a fixed tree order; exp in double rounded to
 * float.  1 on success. */
int edgexpu_cuda_sample_softmax(float *logits, int n, float top_p, uint64_t *rng, uint32_t *out, char *error,
                                size_t error_size);
/* The temperature branch of sample_next_token (src/native.c:2322-2353): every logit score of the
 * resident logits weight (dot + bias, the greedy path's arithmetic and float order) divided by
 * temperature (> 0), then edgexpu_cuda_sample_softmax on the device.  *token_id = the drawn id. */
int edgexpu_cuda_logits_sample(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                               const float *bias, float temperature, float top_p, uint64_t *rng, uint32_t *token_id,
                               char *error, size_t error_size);

/* ---- device-resident model: HBM budget and a GGUF file streamed into HBM --------------------
 * The reference maps the file (src/native.c:115-163), copies each layer into a staging buffer on
 * every use (stage_copy_bytes, native.c:350-380) and admits a model whose working set, KV cache
 * and scratch fit 85 % of RAM (fill_native_plan, src/scheduler.c:320-422).  Here every tensor
 * stays resident, so the plan's weight term is every tensor byte and its limit 85 % of HBM. */
typedef struct edgexpu_cuda_hbm_plan {
    uint64_t weight_bytes;   /* resident tensor bytes (the GGUF data section) */
    uint64_t kv_bytes;       /* 2 * kv_layers * kv_heads * head_dim * window * 4 (scheduler.c:353-359) */
    uint64_t scratch_bytes;  /* min(window, 64) positions of activations (scheduler.c:360-366) */
    uint64_t total_bytes;
    uint64_t limit_bytes;    /* floor(HBM MB * 85 / 100) MB */
    uint64_t file_bytes;
    int window;
    int admitted;
    char reason[256];
} edgexpu_cuda_hbm_plan;
/* Fill `plan` (the terms of fill_native_plan, scheduler.c:320-422, with the weight term and limit
 * above); returns plan->admitted.  Host arithmetic only.  EDGEXPU_BUDGET_DISABLE admits anything,
 * as in the reference; so does a memory size whose 85 % rounds to 0 MB ("device memory unknown"). */
int edgexpu_cuda_hbm_plan_native(uint64_t file_bytes, uint64_t weight_bytes, uint32_t n_kv_layers, uint32_t n_kv_heads,
                                 int head_dim, uint32_t n_embd, uint32_t n_ff, uint32_t n_heads, int window,
                                 uint64_t hbm_total_bytes, edgexpu_cuda_hbm_plan *plan);
/* Parse the GGUF file at `path` (src/gguf.c:359-610), plan its HBM budget for `window` positions
 * (dimensions from the `<arch>.*` keys), and when admitted stream its data section into one HBM
 * arena and register every tensor of a supported type (any row of it is then a valid `weight`).
 * *model receives an opaque handle; `plan` (nullable) the budget, also on refusal (return 0,
 * message = plan reason). */
int edgexpu_cuda_gguf_load(const char *path, int window, void **model, edgexpu_cuda_hbm_plan *plan, char *error,
                           size_t error_size);
int edgexpu_cuda_gguf_tensor_count(const void *model);
/* Tensor `index` of a loaded model: name, device address, GGUF type, row length (n_in), rows
 * (product of the other dimensions), absolute file offset of its first byte, and its byte size
 * (0 when the library does not read that type, so it is not registered). */
int edgexpu_cuda_gguf_tensor_at(const void *model, int index, const char **name, const uint8_t **dev, uint32_t *type,
                                int64_t *n_in, int64_t *n_out, uint64_t *file_offset, uint64_t *nbytes);
/* Index of the tensor called `name`, or -1. */
int edgexpu_cuda_gguf_find(const void *model, const char *name);
/* Metadata value `key` of a loaded model: integers (and an array's element count) in *as_int,
 * numbers in *as_float, strings in *as_str (owned by the model).  Returns GGUF type + 1, or 0 when
 * the key is absent.  Any output may be NULL. */
int edgexpu_cuda_gguf_meta(const void *model, const char *key, uint64_t *as_int, double *as_float, const char **as_str);
/* Unregister the model's tensors and free its arena. */
int edgexpu_cuda_gguf_free(void *model);

/* ---- a llama decoder resident on the device ---------------------------------------------------
 * The reference's layer loop (forward_decode_token, src/native.c:2404-2600) with every op on the
 * device: embedding row, RMSNorm, the q|k|v, o, gate|up and down GEMVs, RoPE, attention over the
 * session's fp32 KV cache, SwiGLU, residual adds, output norm, greedy logits or temperature
 * sampling.  The weights are streamed into HBM by edgexpu_cuda_gguf_load (`window` KV positions
 * planned).  Non-matrix ops restate the reference's float operations; its double sums run in a
 * tree order and exp in double, so they can differ from the reference in the last bit where a
 * value sits next to a float rounding boundary.  Architecture "llama" (RoPE on adjacent pairs). */
int edgexpu_cuda_llama_open(const char *gguf_path, int window, void **session, char *error, size_t error_size);
/* Run tokens[0 .. n_tokens) at positions pos0 .. pos0 + n_tokens - 1 (a prompt, or one decode
 * step), then pick the next token from the output-normed hidden state of the last one: greedy for
 * temperature <= 1e-4 (ties to the lowest id), else softmax sampling with top_p from the xorshift
 * state *rng (edgexpu_cuda_sample_softmax).  last_hidden (nullable, host) receives that hidden
 * state (the reference's session->last_hidden). */
int edgexpu_cuda_llama_forward(void *session, const uint32_t *tokens, int n_tokens, int pos0, float temperature,
                               float top_p, uint64_t *rng, uint32_t *next_token, float *last_hidden, char *error,
                               size_t error_size);
int edgexpu_cuda_llama_close(void *session);

/* Token id encoded in an argmax key (0 when no row had a finite score). */
static inline uint32_t edgexpu_cuda_argmax_key_id(uint64_t key) {
    return key == 0 ? 0u : 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
}

#ifdef __cplusplus
}
#endif

#endif
