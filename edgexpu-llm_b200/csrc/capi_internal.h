// capi_internal.h -- pieces of the C ABI's per-process context shared with other translation units
// of libedgexpu_cuda.so (not exported).
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"

namespace ex {

// GGUF weight types of the path and their activation formats (gguf_dot_q8.c:414-434): Q8_0, Q5_0
// and Q4_0 weights dot against Q8_0 activations, Q4_K, Q5_K and Q6_K against Q8_K.
inline bool acts_are_q8_0(uint32_t type) { return type == TYPE_Q8_0 || type == TYPE_Q5_0 || type == TYPE_Q4_0; }

// Row-stream format of a weight type with quantized activations; false for a type not implemented.
inline bool fmt_of_type(uint32_t type, Fmt* f) {
  switch (type) {
    case TYPE_Q8_0: *f = Fmt::Q8_0xQ8_0; return true;
    case TYPE_Q4_0: *f = Fmt::Q4_0xQ8_0; return true;
    case TYPE_Q5_0: *f = Fmt::Q5_0xQ8_0; return true;
    case TYPE_Q4_K: *f = Fmt::Q4_KxQ8_K; return true;
    case TYPE_Q5_K: *f = Fmt::Q5_KxQ8_K; return true;
    case TYPE_Q6_K: *f = Fmt::Q6_KxQ8_K; return true;
    default: return false;
  }
}

inline Fmt fmt_q8(uint32_t type) {
  Fmt f = Fmt::Q8_0xQ8_0;
  fmt_of_type(type, &f);
  return f;
}

// Format of the greedy-logits dot (native.c:2317-2319, :445-481): the Q8_0-activation types see a
// Q8_0-quantized hidden state, the K-quants the fp32 hidden state (edgexpu_gguf_dot_quant).
inline Fmt logits_fmt(uint32_t type) {
  switch (type) {
    case TYPE_Q4_K: return Fmt::Q4_KxF32;
    case TYPE_Q5_K: return Fmt::Q5_KxF32;
    case TYPE_Q6_K: return Fmt::Q6_KxF32;
    default: return fmt_q8(type);
  }
}

// Quantize m fp32 rows into the activation format of weight type `type`.
inline cudaError_t launch_quantize_for(uint32_t type, const float* x, int m, int n, uint8_t* dst, cudaStream_t st) {
  return acts_are_q8_0(type) ? launch_quantize_q8_0(x, m, n, dst, st) : launch_quantize_q8_k(x, m, n, dst, st);
}

// The lock every entry point holds while it touches the context.
std::recursive_mutex& api_mutex();
// Bind the calling thread to the library's device; 0 (with a message) if edgexpu_cuda_init has not run.
int api_ready(char* error, size_t error_size);
// Check that rows [weight, weight + n_out rows) of width n_in belong to a registered tensor of `type`.
int api_lookup(const uint8_t* weight, uint32_t type, int n_out, int n_in, char* error, size_t error_size);
// Record a failure message (printf-style) for edgexpu_cuda_last_error(); always returns 0.
int api_fail(char* error, size_t error_size, const char* fmt, ...);
const DeviceInfo& api_device_info();
int api_device();
// True when float outputs follow the reference x86 build's order (EDGEXPU_CUDA_ORDER_X86).
bool api_exact_order();
uint32_t* api_status_word();
// The library's stream (the one every synchronous entry point uses).
cudaStream_t api_stream();
// Every logit score (dot + bias, the logits path's activation handling and float order) into scores[vocab].
int api_logit_scores(const uint8_t* weight, uint32_t type, const float* hidden, int n_embd, int vocab, const float* bias,
                     float* scores, cudaStream_t st, char* error, size_t error_size);
// Softmax of io[n] (divided by temperature when > 0) and the reference's draw from *rng; synchronous.
int api_sample(float* io, int n, float temperature, float top_p, uint64_t* rng, uint32_t* out, cudaStream_t st,
               char* error, size_t error_size);
size_t api_row_bytes(uint32_t type, int n);
size_t api_act_row_bytes(uint32_t type, int n);
// Device scratch of at least `bytes` (the library's activation buffer, grown outside stream capture).
void* api_act_scratch(size_t bytes, cudaStream_t st, char* error, size_t error_size);
// Close the tensor-parallel peer mappings and free the local region (tp_p2p.cu); no-op if unused.
void tp_release();

}  // namespace ex
