/*
 * edgexpu_b200_host.h -- C host shim of libedgexpu_b200_host.so: the reference's own
 * quantized-linear entry points, with bodies that forward to the CUDA C ABI (edgexpu_cuda.h).
 *
 * A maintainer drops this in by deleting the same-named definitions from the reference's
 * src/cpu_kernel.c and src/gguf_dot_q8.c and linking this library; src/native.c's layer loop,
 * src/backend_native.c and the src/arch plugins keep calling the same names.
 *
 * Signatures are identical to the reference (paths inside the reference project):
 *   edgexpu_cpu_linear_quant        include/edgexpu/cpu_kernel.h:60-68
 *   edgexpu_cpu_linear_quant_batch  include/edgexpu/cpu_kernel.h:71-80
 *   edgexpu_gguf_quantize_q8_0      include/edgexpu/gguf_quant.h:80-81
 *   edgexpu_gguf_quantize_q8_k      include/edgexpu/gguf_quant.h:85-86
 *   edgexpu_gguf_q8_0_nbytes        include/edgexpu/gguf_quant.h:80
 *   edgexpu_gguf_q8_k_nbytes        include/edgexpu/gguf_quant.h:85
 *   edgexpu_gguf_can_dot_q8         include/edgexpu/gguf_quant.h:82
 *   edgexpu_gguf_can_dot_q8k        include/edgexpu/gguf_quant.h:87
 *   edgexpu_gguf_dot_quant_q8       include/edgexpu/gguf_quant.h:90-95
 *   edgexpu_gguf_dot_quant_q8k      include/edgexpu/gguf_quant.h:97-102
 *   edgexpu_gguf_dot_quant          include/edgexpu/gguf_quant.h:72-77
 *
 * Error behaviour follows the reference: the void linear entry points return silently on
 * NULL / non-positive arguments (cpu_kernel.c:562-564).  A GPU-side failure (unregistered
 * weight, unsupported type, CUDA error) fills `out` with NaN -- so the finite-RMS check of
 * native.c:2232-2234 stops generation -- and records a sticky message readable through
 * edgexpu_b200_last_error().  The quantizers return 1/0 like the reference.  The single-row dots
 * return 0.0f on bad arguments or an unsupported type, as the reference's dispatch does
 * (gguf_dot_q8.c:1010-1022, :1031-1043; gguf_quant.c:895-917), and NaN plus the sticky message
 * on a GPU-side failure.  Their weight row may be a row of an uploaded tensor (device handle) or
 * host memory such as the reference's mmap'd tensor bytes.
 *
 * The shim adds calls the reference has no counterpart for: init/shutdown of the device, the
 * sticky error, weight residency (edgexpu_b200_resident / _release_range, which replace the
 * per-token staging copy) and the greedy logits call that replaces sample_next_token's chunk loop
 * (src/native.c:2355-2400).  integration/edgexpu_b200.patch shows the four places of
 * src/native.c that call them.
 */
#ifndef EDGEXPU_B200_HOST_H
#define EDGEXPU_B200_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void edgexpu_cpu_linear_quant(float *out, const float *x, const uint8_t *weight, uint32_t type, const float *bias,
                              int n_out, int n_in);
void edgexpu_cpu_linear_quant_batch(float *out, const float *x, const uint8_t *weight, uint32_t type,
                                    const float *bias, int m, int n_out, int n_in);

size_t edgexpu_gguf_q8_0_nbytes(int n);
int edgexpu_gguf_quantize_q8_0(const float *x, int n, uint8_t *dst);
int edgexpu_gguf_can_dot_q8(uint32_t type);
size_t edgexpu_gguf_q8_k_nbytes(int n);
int edgexpu_gguf_quantize_q8_k(const float *x, int n, uint8_t *dst);
int edgexpu_gguf_can_dot_q8k(uint32_t type);
float edgexpu_gguf_dot_quant_q8(uint32_t type, const uint8_t *wrow, const uint8_t *x_q8, int n);
float edgexpu_gguf_dot_quant_q8k(uint32_t type, const uint8_t *wrow, const uint8_t *x_q8k, int n);
float edgexpu_gguf_dot_quant(uint32_t type, const uint8_t *row, const float *x, int n);

/* Binds the shim to a CUDA device.  Optional: edgexpu_b200_resident binds device
 * EDGEXPU_B200_DEVICE (default 0) on first use. */
int edgexpu_b200_init(int device, char *error, size_t error_size);
/* Frees every resident tensor and the device context. */
void edgexpu_b200_shutdown(void);

/* Device handle of a packed GGUF tensor that lives in host memory (the reference's mmap'd tensor
 * bytes, tensor_bytes native.c:165-178): uploaded to HBM on the first call for `host`, the same
 * handle on every later call.  Replaces the per-layer, per-token staging copy of load_qweight
 * (native.c:593-655, stage_copy_bytes :350-380); the handle goes into edgexpu_qweight.data.  NULL
 * and a message in `error` on failure, or when `host` was uploaded with another shape or type. */
const uint8_t *edgexpu_b200_resident(const uint8_t *host, size_t nbytes, uint32_t type, int n_out, int n_in,
                                     char *error, size_t error_size);
/* Called right after the model file is mapped (edgexpu_native_load, native.c:1282-1285): plans the
 * HBM budget of the resident model for `window` positions (edgexpu_cuda_hbm_plan_native: 85 % of
 * HBM, the analogue of admit_session_window native.c:79-92), streams the file's data section into
 * HBM in one pass (edgexpu_cuda_gguf_load), and enters every tensor into the residency table under
 * its address in the mapping [file_map, file_map + file_size), so edgexpu_b200_resident finds it
 * without a copy.  1 on success; 0 and a message in `error` (the budget's reason on refusal). */
int edgexpu_b200_preload(const uint8_t *file_map, size_t file_size, const char *path, int window, char *error,
                         size_t error_size);
/* Frees the resident tensors whose host bytes lie in [base, base + size), and the models preloaded
 * from a mapping there: the model file is being unmapped (edgexpu_native_free, native.c:1203-1233),
 * so a later mapping may reuse the addresses. */
void edgexpu_b200_release_range(const void *base, size_t size);
/* Sticky message of the first failure since the last clear ("" if none). */
const char *edgexpu_b200_last_error(void);
void edgexpu_b200_clear_error(void);

/* Greedy token for the logits weight (tied token_embd or output.weight), as sample_next_token
 * with temperature <= 1e-4.  Returns 1/0 and fills error like the reference's session calls. */
int edgexpu_b200_logits_greedy(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                               const float *bias, uint32_t *token_id, char *error, size_t error_size);
/* Sampled token for temperature > 1e-4, as sample_next_token's temperature branch
 * (native.c:2322-2353 with edgexpu_cpu_sample_softmax, cpu_kernel.c:762-849): scores / temperature,
 * softmax, top_p and the draw from the caller's xorshift state *rng, on the device. */
int edgexpu_b200_logits_sample(const uint8_t *weight, uint32_t type, const float *hidden, int n_embd, int vocab,
                               const float *bias, float temperature, float top_p, uint64_t *rng, uint32_t *token_id,
                               char *error, size_t error_size);

#ifdef __cplusplus
}
#endif

#endif
