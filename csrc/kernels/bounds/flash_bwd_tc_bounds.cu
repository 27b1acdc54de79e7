// Debug build of flash_bwd_tc.cu for the `_C_bounds` extension: the tile-index
// checks (NK_IN_BOUNDS in common.cuh) are compiled in.
#define NANOGPT_DEBUG_BOUNDS 1
#include "../flash_bwd_tc.cu"
