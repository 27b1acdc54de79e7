// Warp-level building blocks of the flash-attention kernels: bf16
// m16n8k16 tensor-core MMAs, ldmatrix fragment loads from XOR-swizzled
// shared-memory tiles, and cp.async tile copies with zero fill.
//
// Shared-memory tiles hold rows of HD bf16 (HD * 2 bytes) split in 16-byte
// chunks; chunk c of row r is stored at chunk (c ^ (r & 7)) so that the eight
// row addresses of one ldmatrix phase hit eight different bank groups.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace nk {

template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return uint32_t(row * HD * 2 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill rows beyond the sequence
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Copy `rows` x HD bf16 from global (row stride ld elements) into a swizzled
// tile; rows >= valid_rows are zero-filled. All threads of the CTA take part.
template <int HD, int ROWS, int THREADS>
__device__ __forceinline__ void load_tile(uint32_t smem, const __nv_bfloat16* g, long ld, int valid_rows) {
  constexpr int CHUNKS = HD / 8;
#pragma unroll
  for (int i = threadIdx.x; i < ROWS * CHUNKS; i += THREADS) {
    const int r = i / CHUNKS, c = i % CHUNKS;
    const bool ok = r < valid_rows;
    const __nv_bfloat16* src = g + (ok ? long(r) * ld : 0) + c * 8;
    cp_async16(smem + swz<HD>(r, c), src, ok);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// D (16x8 fp32) += A (16x16 bf16, row) * B (16x8 bf16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A-operand fragment (16 rows x 16 k) from a row-major swizzled tile whose
// rows are the M dimension: rows [r0, r0+16), k columns [k0, k0+16).
template <int HD>
__device__ __forceinline__ void load_a(uint32_t tile, int r0, int k0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  const int r = r0 + (lane & 15), c = (k0 >> 3) + (lane >> 4);
  ldsm_x4(tile + swz<HD>(r, c), a[0], a[1], a[2], a[3]);
}

// A-operand fragment from a tile stored transposed: tile rows are the k
// dimension and tile columns the M dimension (rows [k0, k0+16), cols [m0, m0+16)).
template <int HD>
__device__ __forceinline__ void load_a_t(uint32_t tile, int m0, int k0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  // matrices: (m 0-7,k 0-7) (m 8-15,k 0-7) (m 0-7,k 8-15) (m 8-15,k 8-15)
  const int k = k0 + (lane & 7) + ((lane >> 4) << 3), m = m0 + ((lane >> 3) & 1) * 8;
  ldsm_x4_t(tile + swz<HD>(k, m >> 3), a[0], a[1], a[2], a[3]);
}

// B-operand fragments for two n-tiles (n0..n0+16) and one k-step, from a tile
// whose rows are the N dimension and columns the K dimension (e.g. K for Q K^T).
template <int HD>
__device__ __forceinline__ void load_b_nk(uint32_t tile, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31;
  const int n = n0 + (lane & 7) + ((lane >> 4) << 3), c = (k0 >> 3) + ((lane >> 3) & 1);
  ldsm_x4(tile + swz<HD>(n, c), b[0], b[1], b[2], b[3]);  // b0,b1 of tile n0; b0,b1 of tile n0+8
}

// B-operand fragments for two n-tiles from a tile whose rows are the K
// dimension and columns the N dimension (e.g. V for P V).
template <int HD>
__device__ __forceinline__ void load_b_kn(uint32_t tile, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31;
  const int k = k0 + (lane & 7) + (((lane >> 3) & 1) << 3), c = (n0 >> 3) + (lane >> 4);
  ldsm_x4_t(tile + swz<HD>(k, c), b[0], b[1], b[2], b[3]);
}

}  // namespace nk
