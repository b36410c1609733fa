// Per-thread device scope shared by the host entry points that are not tied to
// a model (layer-level calls, tensor_gemm, detect_postprocess_from_pred), the
// thread-local error text behind yb_cuda_last_error(), and helpers that map
// CUDA failures onto status_t.
#pragma once
#include <string>
#include <cuda_runtime.h>
#include "status.h"

namespace yb {

struct DevScope {
  int device = 0;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;
  int num_sms = 148;
};

// Scope of the calling thread's current CUDA device (created on first use).
// Returns nullptr (and sets the error text) when no device is usable.
DevScope* current_scope();

void set_error(const std::string& msg);
const char* last_error();

// Maps a CUDA error to status_t, recording `what` and the CUDA message.
status_t cuda_status(cudaError_t e, const char* what);

// Loads the no-allocation top-k's scratch array and kernels on the current
// device (noalloc.cu); called by yb_cuda_init.
status_t noalloc_prepare_current_device();

// RAII device allocation.
struct DevMem {
  void* p = nullptr;
  size_t bytes = 0;
  DevMem() = default;
  DevMem(const DevMem&) = delete;
  DevMem& operator=(const DevMem&) = delete;
  ~DevMem() {
    if (p) cudaFree(p);
  }
  cudaError_t alloc(size_t n) {
    bytes = n;
    return cudaMalloc(&p, n < 256 ? 256 : n);
  }
  float* f() const { return static_cast<float*>(p); }
};

}  // namespace yb
