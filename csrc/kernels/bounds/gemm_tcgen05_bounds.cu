// Debug build of gemm_tcgen05.cu for the `_C_bounds` extension: the tile-index
// checks (NK_IN_BOUNDS in common.cuh) are compiled in.
#define NANOGPT_DEBUG_BOUNDS 1
#include "../gemm_tcgen05.cu"
