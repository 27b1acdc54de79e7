// Allocation-free C entry point for the flash-attention backward pass.
//
// This entry point has no counterpart in the reference (rs-nanogpt); it is an
// addition of this library.
//
// Who it is for: code that must not allocate GPU memory itself -- for example a
// host runtime that hands this library only pre-planned buffers and forbids
// cudaMalloc / cudaFree (and any library call that allocates) inside its
// compute phase, or a plain-C caller that links the shared object without
// PyTorch and therefore has no caching allocator to borrow scratch from.
// The regular entry point (flash_bwd) takes its scratch buffer from the caller
// as a torch tensor; this one keeps that scratch in a fixed, file-scope device
// array inside the library instead.
//
// Limits and behaviour:
//  * The scratch holds batch * n_head * seq_len floats; at most
//    NANOGPT_NOALLOC_MAX_ROWS (1,048,576 floats = 4 MiB). Larger problems are
//    rejected with NANOGPT_NOALLOC_ERR_TOO_LARGE before anything is launched.
//  * Every GPU that loads the library reserves those 4 MiB until the process
//    exits.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * All calls share the one array and it keeps the previous call's contents.
//    Each call overwrites every entry it reads, so nothing must start at zero,
//    but calls whose GPU work overlaps (different streams without ordering, or
//    different host threads) race on it and must not be issued.
//  * Inputs and outputs are supplied by the caller; head_dim must be 64 or 128,
//    all pointers 16-byte aligned, and batch * n_head at most
//    NANOGPT_NOALLOC_MAX_BATCH_HEADS (65535, the grid.y limit).
//  * A CUDA error already pending when the call starts (from earlier work) is
//    returned as NANOGPT_NOALLOC_ERR_CUDA without clearing it and before
//    anything is queued; each of the three launches is checked on its own and
//    a failed launch stops the sequence.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NANOGPT_NOALLOC_MAX_ROWS (1u << 20)
#define NANOGPT_NOALLOC_MAX_BATCH_HEADS 65535u

#define NANOGPT_NOALLOC_OK 0
#define NANOGPT_NOALLOC_ERR_TOO_LARGE 1
#define NANOGPT_NOALLOC_ERR_BAD_ARG 2
#define NANOGPT_NOALLOC_ERR_CUDA 3

// qkv:  (batch*seq_len, 3*C) bf16, q | k | v column blocks (C = n_head*head_dim)
// out:  (batch*seq_len, C) bf16 forward output; dout: its gradient, same shape
// lse:  (batch, n_head, seq_len) fp32, as written by the forward kernel
// dqkv: (batch*seq_len, 3*C) bf16 output: dQ | dK | dV
// Returns NANOGPT_NOALLOC_OK or an error code; the work is queued on `stream`.
int nanogpt_flash_attention_bwd_noalloc(const void* qkv, const void* out, const void* dout, const float* lse,
                                        void* dqkv, int batch, int seq_len, int n_head, int head_dim,
                                        cudaStream_t stream);

// Human-readable text for a return code of the function above.
const char* nanogpt_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
