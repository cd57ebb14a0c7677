// capi_internal.h -- pieces of the C ABI's per-process context shared with other translation units
// of libedgexpu_cuda.so (not exported).
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>

#include "launch.h"

namespace ex {

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
uint32_t* api_status_word();
size_t api_row_bytes(uint32_t type, int n);
size_t api_act_row_bytes(uint32_t type, int n);
// Device scratch of at least `bytes` (the library's activation buffer, grown outside stream capture).
void* api_act_scratch(size_t bytes, cudaStream_t st, char* error, size_t error_size);
// Close the tensor-parallel peer mappings and free the local region (tp_p2p.cu); no-op if unused.
void tp_release();

}  // namespace ex
