#include <cuda_runtime.h>
#include <torch/extension.h>

#include "status.h"

namespace nk {

int* error_word() {
  static int* p = [] {
    int* d = nullptr;
    TORCH_CHECK(cudaMalloc(&d, sizeof(int)) == cudaSuccess, "error_word: cudaMalloc failed");
    TORCH_CHECK(cudaMemset(d, 0, sizeof(int)) == cudaSuccess, "error_word: cudaMemset failed");
    return d;
  }();
  return p;
}

int64_t kernel_status(bool reset) {
  int v = 0;
  TORCH_CHECK(cudaMemcpy(&v, error_word(), sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess,
              "kernel_status: read failed");
  if (reset && v != 0)
    TORCH_CHECK(cudaMemset(error_word(), 0, sizeof(int)) == cudaSuccess, "kernel_status: reset failed");
  return v;
}

static bool g_pdl = false;
bool pdl_enabled() { return g_pdl; }
void set_pdl(bool on) { g_pdl = on; }

}  // namespace nk
