// ql_internal.h -- library-internal view of the context, shared by the
// attention API (ql_api.cu) and the model host (ql_model.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

struct ql_ctx {
  int device = 0;
  int num_sms = 0;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  uint32_t* status = nullptr;  // device word raised by kernels
  void* ws = nullptr;          // workspace (staging, split partials, scratch)
  size_t ws_bytes = 0;
  int32_t* counters = nullptr;  // split-merge arrival counters, kept at zero
  size_t counters_n = 0;
};

// Records the message of a failed call (ql_last_error) and returns `code`.
int ql_fail(int code, const char* fmt, ...);
// Reads and clears the context's device status word; QL_ERR_DEVICE with a
// message when a kernel raised a bit.
int ql_check_status(ql_ctx* c);
// The context's reusable device workspace, grown to at least `bytes`
// (growing synchronises the context's stream first).
int ql_ctx_workspace(ql_ctx* c, size_t bytes, void** out);
