// Device error word shared by the kernels of this extension. A bounded wait
// that runs out writes a nonzero code here instead of hanging the GPU; the
// host reads (and clears) it with kernel_status().
#pragma once
#include <cstdint>
namespace nk {
int* error_word();  // device pointer, allocated once per process
int64_t kernel_status(bool reset);

// Programmatic dependent launch for the decode chain: while enabled, kernels
// that support it are launched with programmatic stream serialization, so
// their CTAs start (and prefetch weights) while the previous kernel drains;
// each such kernel executes griddepcontrol.wait before touching memory that an
// earlier kernel writes or reads.
bool pdl_enabled();
void set_pdl(bool on);
}
