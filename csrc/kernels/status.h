// Device error word shared by the kernels of this extension. A bounded wait
// that runs out writes a nonzero code here instead of hanging the GPU; the
// host reads (and clears) it with kernel_status().
#pragma once
#include <cstdint>
namespace nk {
int* error_word();  // device pointer, allocated once per process
int64_t kernel_status(bool reset);
}
