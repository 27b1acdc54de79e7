// Causal flash attention, forward and backward, head_dim 64 or 128, bf16 in /
// bf16 out with fp32 softmax statistics. q/k/v are read in place from the
// fused QKV activation (row stride 3C), so no head transposes are made; the
// output is written in (token, head, dim) order, which is exactly the input
// layout of the c_proj GEMM.
//
// Replaces rs-nanogpt's chunked attention (src/model/flash_attention.rs:48-218):
// same math (softmax(QK^T * scale + causal mask) V, LSE stashed for the
// backward, dS = P o (dP - rowsum(dO o O))), but streamed through registers
// and shared memory with O(T) memory instead of per-chunk temporaries.
//
//   flash_fwd       CTA = 128 query rows of one (batch, head); 8 warps x 16 rows;
//                   K/V tiles of 64 keys double-buffered with cp.async.
//   flash_bwd_dot   D = rowsum(dO o O) per (batch, head, row)            (scratch)
//   flash_bwd_dq    CTA = 128 query rows; dQ = scale * dS K
//   flash_bwd_dkv   CTA = 64 keys; 4 warps x 16 keys; dV = P^T dO, dK = scale * dS^T Q
// The backward recomputes P in both kernels instead of accumulating dQ with
// atomics, so it needs no fp32 dQ buffer.
//
// The LSE is stored in base-2 units of the scaled scores:
// lse2 = log2(sum_j exp2(s_j * scale * log2 e)).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "flash_common.cuh"

namespace nk {

constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long ld_qkv;
  const __nv_bfloat16* o;   // forward output (backward only)
  __nv_bfloat16* out;       // fwd: O; bwd_dq: dQ; bwd_dkv: dK
  __nv_bfloat16* out2;      // bwd_dkv: dV
  long ld_out;
  const __nv_bfloat16* dout;  // dO (backward)
  long ld_do;
  float* lse;
  float* dsum;             // D = rowsum(dO o O)
  int B, H, T;
  float scale, sl2;        // softmax scale, scale * log2(e)
};

__device__ __forceinline__ uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

// ---------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(256) flash_fwd_kernel(const AttnArgs a) {
  constexpr int BM = 128, BN = 64, NT = HD / 8, KS = HD / 16;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + BM * HD * 2;
  const uint32_t sV0 = sK0 + 2 * BN * HD * 2;
  const int qb = gridDim.x - 1 - blockIdx.x;  // heaviest (latest) blocks first
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int q0 = qb * BM;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const long tok0 = long(b) * a.T;
  const __nv_bfloat16* Q = a.q + tok0 * a.ld_qkv + h * HD;
  const __nv_bfloat16* K = a.k + tok0 * a.ld_qkv + h * HD;
  const __nv_bfloat16* V = a.v + tok0 * a.ld_qkv + h * HD;

  load_tile<HD, BM, 256>(sQ, Q + long(q0) * a.ld_qkv, a.ld_qkv, a.T - q0);
  cp_async_commit();
  const int kv_end = min(q0 + BM, a.T);
  const int nkv = (kv_end + BN - 1) / BN;
  load_tile<HD, BN, 256>(sK0, K, a.ld_qkv, a.T);
  load_tile<HD, BN, 256>(sV0, V, a.ld_qkv, a.T);
  cp_async_commit();

  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[KS][4];
  const int r_lo = q0 + warp * 16 + g, r_hi = r_lo + 8;

  for (int j = 0; j < nkv; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkv) {
      const int k0 = (j + 1) * BN;
      load_tile<HD, BN, 256>(sK0 + (buf ^ 1) * BN * HD * 2, K + long(k0) * a.ld_qkv, a.ld_qkv, a.T - k0);
      load_tile<HD, BN, 256>(sV0 + (buf ^ 1) * BN * HD * 2, V + long(k0) * a.ld_qkv, a.ld_qkv, a.T - k0);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) load_a<HD>(sQ, warp * 16, kk * 16, qf[kk]);
    }
    const uint32_t sK = sK0 + buf * BN * HD * 2, sV = sV0 + buf * BN * HD * 2;
    const int k0 = j * BN;
    // Warps whose rows all precede this key block have nothing to do in it.
    if (k0 <= q0 + warp * 16 + 15) {
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bb[4];
          load_b_nk<HD>(sK, np * 16, kk * 16, bb);
          mma16816(s[2 * np], qf[kk], bb[0], bb[1]);
          mma16816(s[2 * np + 1], qf[kk], bb[2], bb[3]);
        }
      }
      float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = k0 + n * 8 + 2 * t4 + (e & 1);
          const int row = e < 2 ? r_lo : r_hi;
          float val = s[n][e] * a.sl2;
          if (col > row || col >= a.T) val = -INFINITY;
          s[n][e] = val;
          mx[e >> 1] = fmaxf(mx[e >> 1], val);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      }
      float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
      for (int r = 0; r < 2; ++r) alpha[r] = exp2f(mrow[r] - mx[r]);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p = exp2f(s[n][e] - mx[e >> 1]);
          s[n][e] = p;
          rs[e >> 1] += p;
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
        lrow[r] = lrow[r] * alpha[r] + rs[r];
        mrow[r] = mx[r];
      }
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        acc[i][0] *= alpha[0]; acc[i][1] *= alpha[0];
        acc[i][2] *= alpha[1]; acc[i][3] *= alpha[1];
      }
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint32_t pa[4] = {pack2(s[2 * kk][0], s[2 * kk][1]), pack2(s[2 * kk][2], s[2 * kk][3]),
                                pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
        for (int np = 0; np < HD / 16; ++np) {
          uint32_t bb[4];
          load_b_kn<HD>(sV, np * 16, kk * 16, bb);
          mma16816(acc[2 * np], pa, bb[0], bb[1]);
          mma16816(acc[2 * np + 1], pa, bb[2], bb[3]);
        }
      }
    }
    __syncthreads();
  }
  // Normalize and store.
  const float inv[2] = {1.f / lrow[0], 1.f / lrow[1]};
  __nv_bfloat16* O = a.out + tok0 * a.ld_out + h * HD;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int col = i * 8 + 2 * t4;
    if (r_lo < a.T)
      *reinterpret_cast<uint32_t*>(O + long(r_lo) * a.ld_out + col) = pack2(acc[i][0] * inv[0], acc[i][1] * inv[0]);
    if (r_hi < a.T)
      *reinterpret_cast<uint32_t*>(O + long(r_hi) * a.ld_out + col) = pack2(acc[i][2] * inv[1], acc[i][3] * inv[1]);
  }
  if (t4 == 0) {
    float* L = a.lse + (long(b) * a.H + h) * a.T;
    if (r_lo < a.T) L[r_lo] = mrow[0] + log2f(lrow[0]);
    if (r_hi < a.T) L[r_hi] = mrow[1] + log2f(lrow[1]);
  }
}

// ---------------------------------------------------------------------------------------------
// D[b,h,t] = sum_d dO[t,h,d] * O[t,h,d]; one warp per (token, head).
template <int HD>
__global__ void flash_bwd_dot_kernel(const AttnArgs a) {
  const long item = long(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (item >= long(a.B) * a.T * a.H) return;
  const long tok = item / a.H;
  const int h = int(item % a.H);
  const __nv_bfloat16* o = a.o + tok * a.ld_out + h * HD;
  const __nv_bfloat16* d = a.dout + tok * a.ld_do + h * HD;
  float s = 0.f;
  for (int c = lane * 2; c < HD; c += 64) {
    float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(o + c));
    float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(d + c));
    s += x.x * y.x + x.y * y.y;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    const int b = int(tok / a.T), t = int(tok % a.T);
    a.dsum[(long(b) * a.H + h) * a.T + t] = s;
  }
}

// ---------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(256) flash_bwd_dq_kernel(const AttnArgs a) {
  constexpr int BM = 128, BN = 64, NT = HD / 8, KS = HD / 16;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sD = sQ + BM * HD * 2;
  const uint32_t sK0 = sD + BM * HD * 2;
  const uint32_t sV0 = sK0 + 2 * BN * HD * 2;
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int q0 = qb * BM;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const long tok0 = long(b) * a.T;
  const __nv_bfloat16* K = a.k + tok0 * a.ld_qkv + h * HD;
  const __nv_bfloat16* V = a.v + tok0 * a.ld_qkv + h * HD;
  load_tile<HD, BM, 256>(sQ, a.q + (tok0 + q0) * a.ld_qkv + h * HD, a.ld_qkv, a.T - q0);
  load_tile<HD, BM, 256>(sD, a.dout + (tok0 + q0) * a.ld_do + h * HD, a.ld_do, a.T - q0);
  cp_async_commit();
  const int kv_end = min(q0 + BM, a.T);
  const int nkv = (kv_end + BN - 1) / BN;
  load_tile<HD, BN, 256>(sK0, K, a.ld_qkv, a.T);
  load_tile<HD, BN, 256>(sV0, V, a.ld_qkv, a.T);
  cp_async_commit();

  const int r_lo = q0 + warp * 16 + g, r_hi = r_lo + 8;
  const float* L = a.lse + (long(b) * a.H + h) * a.T;
  const float* Dp = a.dsum + (long(b) * a.H + h) * a.T;
  const float lse_lo = r_lo < a.T ? L[r_lo] : 0.f, lse_hi = r_hi < a.T ? L[r_hi] : 0.f;
  const float d_lo = r_lo < a.T ? Dp[r_lo] : 0.f, d_hi = r_hi < a.T ? Dp[r_hi] : 0.f;

  float dq[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int j = 0; j < nkv; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkv) {
      const int k0 = (j + 1) * BN;
      load_tile<HD, BN, 256>(sK0 + (buf ^ 1) * BN * HD * 2, K + long(k0) * a.ld_qkv, a.ld_qkv, a.T - k0);
      load_tile<HD, BN, 256>(sV0 + (buf ^ 1) * BN * HD * 2, V + long(k0) * a.ld_qkv, a.ld_qkv, a.T - k0);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + buf * BN * HD * 2, sV = sV0 + buf * BN * HD * 2;
    const int k0 = j * BN;
    if (k0 <= q0 + warp * 16 + 15) {
      float s[8][4], dp[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t qa[4], da[4];
        load_a<HD>(sQ, warp * 16, kk * 16, qa);
        load_a<HD>(sD, warp * 16, kk * 16, da);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bk[4], bv[4];
          load_b_nk<HD>(sK, np * 16, kk * 16, bk);
          load_b_nk<HD>(sV, np * 16, kk * 16, bv);
          mma16816(s[2 * np], qa, bk[0], bk[1]);
          mma16816(s[2 * np + 1], qa, bk[2], bk[3]);
          mma16816(dp[2 * np], da, bv[0], bv[1]);
          mma16816(dp[2 * np + 1], da, bv[2], bv[3]);
        }
      }
      // dS = P o (dP - D)
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = k0 + n * 8 + 2 * t4 + (e & 1);
          const int row = e < 2 ? r_lo : r_hi;
          const float p = (col > row || col >= a.T) ? 0.f : exp2f(s[n][e] * a.sl2 - (e < 2 ? lse_lo : lse_hi));
          s[n][e] = p * (dp[n][e] - (e < 2 ? d_lo : d_hi));
        }
      }
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint32_t sa[4] = {pack2(s[2 * kk][0], s[2 * kk][1]), pack2(s[2 * kk][2], s[2 * kk][3]),
                                pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
        for (int np = 0; np < HD / 16; ++np) {
          uint32_t bb[4];
          load_b_kn<HD>(sK, np * 16, kk * 16, bb);
          mma16816(dq[2 * np], sa, bb[0], bb[1]);
          mma16816(dq[2 * np + 1], sa, bb[2], bb[3]);
        }
      }
    }
    __syncthreads();
  }
  __nv_bfloat16* DQ = a.out + tok0 * a.ld_out + h * HD;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int col = i * 8 + 2 * t4;
    if (r_lo < a.T)
      *reinterpret_cast<uint32_t*>(DQ + long(r_lo) * a.ld_out + col) = pack2(dq[i][0] * a.scale, dq[i][1] * a.scale);
    if (r_hi < a.T)
      *reinterpret_cast<uint32_t*>(DQ + long(r_hi) * a.ld_out + col) = pack2(dq[i][2] * a.scale, dq[i][3] * a.scale);
  }
}

// ---------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(128) flash_bwd_dkv_kernel(const AttnArgs a) {
  constexpr int BN = 64, BQ = 32, NT = HD / 8, KS = HD / 16;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BN * HD * 2;
  const uint32_t sQ0 = sV + BN * HD * 2;
  const uint32_t sO0 = sQ0 + 2 * BQ * HD * 2;  // dO tiles
  float* sL = reinterpret_cast<float*>(smem + 2 * BN * HD * 2 + 4 * BQ * HD * 2);  // [2][BQ] lse
  float* sDs = sL + 2 * BQ;                                                          // [2][BQ] D
  const int kb = blockIdx.x;
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int k0 = kb * BN;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const long tok0 = long(b) * a.T;
  const __nv_bfloat16* Q = a.q + tok0 * a.ld_qkv + h * HD;
  const __nv_bfloat16* DO = a.dout + tok0 * a.ld_do + h * HD;
  const float* L = a.lse + (long(b) * a.H + h) * a.T;
  const float* Dp = a.dsum + (long(b) * a.H + h) * a.T;

  load_tile<HD, BN, 128>(sK, a.k + (tok0 + k0) * a.ld_qkv + h * HD, a.ld_qkv, a.T - k0);
  load_tile<HD, BN, 128>(sV, a.v + (tok0 + k0) * a.ld_qkv + h * HD, a.ld_qkv, a.T - k0);
  const int qt_begin = k0 / BQ, qt_end = (a.T + BQ - 1) / BQ;
  auto load_q = [&](int qt, int buf) {
    const int q0 = qt * BQ;
    load_tile<HD, BQ, 128>(sQ0 + buf * BQ * HD * 2, Q + long(q0) * a.ld_qkv, a.ld_qkv, a.T - q0);
    load_tile<HD, BQ, 128>(sO0 + buf * BQ * HD * 2, DO + long(q0) * a.ld_do, a.ld_do, a.T - q0);
    if (threadIdx.x < BQ) {
      const int r = q0 + threadIdx.x;
      sL[buf * BQ + threadIdx.x] = r < a.T ? L[r] : 0.f;
      sDs[buf * BQ + threadIdx.x] = r < a.T ? Dp[r] : 0.f;
    }
  };
  load_q(qt_begin, 0);
  cp_async_commit();

  float dk[NT][4], dv[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
  const int kr_lo = k0 + warp * 16 + g, kr_hi = kr_lo + 8;  // this thread's key rows

  for (int qt = qt_begin; qt < qt_end; ++qt) {
    const int buf = (qt - qt_begin) & 1;
    __syncthreads();  // previous users of the other buffer are done
    if (qt + 1 < qt_end) {
      load_q(qt + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sQ = sQ0 + buf * BQ * HD * 2, sO = sO0 + buf * BQ * HD * 2;
    const float* lq = sL + buf * BQ;
    const float* dq = sDs + buf * BQ;
    const int q0 = qt * BQ;
    if (q0 + BQ - 1 < k0 + warp * 16) continue;  // every query precedes this warp's keys
    // S^T (16 keys x 32 queries) and dP^T.
    float s[4][4], dp[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t ka[4], va[4];
      load_a<HD>(sK, warp * 16, kk * 16, ka);
      load_a<HD>(sV, warp * 16, kk * 16, va);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t bq[4], bo[4];
        load_b_nk<HD>(sQ, np * 16, kk * 16, bq);
        load_b_nk<HD>(sO, np * 16, kk * 16, bo);
        mma16816(s[2 * np], ka, bq[0], bq[1]);
        mma16816(s[2 * np + 1], ka, bq[2], bq[3]);
        mma16816(dp[2 * np], va, bo[0], bo[1]);
        mma16816(dp[2 * np + 1], va, bo[2], bo[3]);
      }
    }
    float ds[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = n * 8 + 2 * t4 + (e & 1);  // query within the tile
        const int qpos = q0 + qc;
        const int krow = e < 2 ? kr_lo : kr_hi;
        const float p = (krow > qpos || qpos >= a.T || krow >= a.T) ? 0.f : exp2f(s[n][e] * a.sl2 - lq[qc]);
        s[n][e] = p;
        ds[n][e] = p * (dp[n][e] - dq[qc]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q   (contraction over the 32 queries)
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      const uint32_t pa[4] = {pack2(s[2 * kk][0], s[2 * kk][1]), pack2(s[2 * kk][2], s[2 * kk][3]),
                              pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
      const uint32_t sa[4] = {pack2(ds[2 * kk][0], ds[2 * kk][1]), pack2(ds[2 * kk][2], ds[2 * kk][3]),
                              pack2(ds[2 * kk + 1][0], ds[2 * kk + 1][1]), pack2(ds[2 * kk + 1][2], ds[2 * kk + 1][3])};
#pragma unroll
      for (int np = 0; np < HD / 16; ++np) {
        uint32_t bo[4], bq[4];
        load_b_kn<HD>(sO, np * 16, kk * 16, bo);
        load_b_kn<HD>(sQ, np * 16, kk * 16, bq);
        mma16816(dv[2 * np], pa, bo[0], bo[1]);
        mma16816(dv[2 * np + 1], pa, bo[2], bo[3]);
        mma16816(dk[2 * np], sa, bq[0], bq[1]);
        mma16816(dk[2 * np + 1], sa, bq[2], bq[3]);
      }
    }
  }
  __nv_bfloat16* DK = a.out + tok0 * a.ld_out + h * HD;
  __nv_bfloat16* DV = a.out2 + tok0 * a.ld_out + h * HD;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int col = i * 8 + 2 * t4;
    if (kr_lo < a.T) {
      *reinterpret_cast<uint32_t*>(DK + long(kr_lo) * a.ld_out + col) = pack2(dk[i][0] * a.scale, dk[i][1] * a.scale);
      *reinterpret_cast<uint32_t*>(DV + long(kr_lo) * a.ld_out + col) = pack2(dv[i][0], dv[i][1]);
    }
    if (kr_hi < a.T) {
      *reinterpret_cast<uint32_t*>(DK + long(kr_hi) * a.ld_out + col) = pack2(dk[i][2] * a.scale, dk[i][3] * a.scale);
      *reinterpret_cast<uint32_t*>(DV + long(kr_hi) * a.ld_out + col) = pack2(dv[i][2], dv[i][3]);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Host entry points. qkv: (B*T, 3C) bf16 with q | k | v column blocks.

static AttnArgs make_args(torch::Tensor qkv, int64_t B, int64_t T, int64_t H) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1, "attn: bf16 2-D qkv");
  const int64_t C = qkv.size(1) / 3;
  TORCH_CHECK(qkv.size(0) == B * T && C % H == 0, "attn: shape");
  const int HD = int(C / H);
  TORCH_CHECK(HD == 64 || HD == 128, "attn: head_dim must be 64 or 128");
  TORCH_CHECK(qkv.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0, "attn: alignment");
  AttnArgs a{};
  auto base = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.q = base; a.k = base + C; a.v = base + 2 * C;
  a.ld_qkv = qkv.stride(0);
  a.B = int(B); a.H = int(H); a.T = int(T);
  a.scale = 1.f / std::sqrt(float(HD));
  a.sl2 = a.scale * kLog2e;
  return a;
}

template <typename Kernel>
static void set_smem(Kernel k, int bytes) {
  TORCH_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess,
              "attn: cannot reserve shared memory");
}

// out: (B*T, C) bf16; lse: (B, H, T) fp32.
void flash_fwd(torch::Tensor qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t T, int64_t H) {
  AttnArgs a = make_args(qkv, B, T, H);
  const int HD = int(qkv.size(1) / 3 / H);
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(0) == B * T &&
                  out.size(1) == H * HD && out.stride(0) % 8 == 0, "attn: out");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * H * T && lse.is_contiguous(), "attn: lse");
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ld_out = out.stride(0);
  a.lse = lse.data_ptr<float>();
  const at::cuda::CUDAGuard guard(qkv.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid(unsigned((T + 127) / 128), unsigned(B * H));
  if (HD == 128) {
    const int sm = (128 + 4 * 64) * 128 * 2;
    set_smem(flash_fwd_kernel<128>, sm);
    flash_fwd_kernel<128><<<grid, 256, sm, stream>>>(a);
  } else {
    const int sm = (128 + 4 * 64) * 64 * 2;
    set_smem(flash_fwd_kernel<64>, sm);
    flash_fwd_kernel<64><<<grid, 256, sm, stream>>>(a);
  }
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "flash_fwd launch failed");
}

// dqkv: (B*T, 3C) bf16 receives dQ | dK | dV. dsum: (B, H, T) fp32 scratch.
void flash_bwd(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor dsum,
               torch::Tensor dqkv, int64_t B, int64_t T, int64_t H) {
  AttnArgs a = make_args(qkv, B, T, H);
  const int64_t C = qkv.size(1) / 3;
  const int HD = int(C / H);
  TORCH_CHECK(dqkv.sizes() == qkv.sizes() && dqkv.stride(0) == qkv.stride(0) && dqkv.stride(1) == 1, "attn: dqkv");
  TORCH_CHECK(out.stride(1) == 1 && dout.stride(1) == 1 && out.size(1) == C && dout.size(1) == C, "attn: o/do");
  TORCH_CHECK(dsum.scalar_type() == at::kFloat && dsum.numel() == B * H * T, "attn: dsum");
  a.o = reinterpret_cast<const __nv_bfloat16*>(out.data_ptr());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.ld_do = dout.stride(0);
  a.lse = lse.data_ptr<float>();
  a.dsum = dsum.data_ptr<float>();
  const at::cuda::CUDAGuard guard(qkv.device());
  auto stream = at::cuda::getCurrentCUDAStream();

  AttnArgs d = a;
  d.ld_out = out.stride(0);
  const long items = B * T * H;
  if (HD == 128) flash_bwd_dot_kernel<128><<<unsigned((items + 7) / 8), 256, 0, stream>>>(d);
  else flash_bwd_dot_kernel<64><<<unsigned((items + 7) / 8), 256, 0, stream>>>(d);

  auto dbase = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  AttnArgs q = a;
  q.out = dbase;
  q.ld_out = dqkv.stride(0);
  dim3 gq(unsigned((T + 127) / 128), unsigned(B * H));
  AttnArgs kv = a;
  kv.out = dbase + C;
  kv.out2 = dbase + 2 * C;
  kv.ld_out = dqkv.stride(0);
  dim3 gk(unsigned((T + 63) / 64), unsigned(B * H));
  if (HD == 128) {
    const int smq = (2 * 128 + 4 * 64) * 128 * 2, smk = (2 * 64 + 4 * 32) * 128 * 2 + 4 * 32 * 4;
    set_smem(flash_bwd_dq_kernel<128>, smq);
    set_smem(flash_bwd_dkv_kernel<128>, smk);
    flash_bwd_dq_kernel<128><<<gq, 256, smq, stream>>>(q);
    flash_bwd_dkv_kernel<128><<<gk, 128, smk, stream>>>(kv);
  } else {
    const int smq = (2 * 128 + 4 * 64) * 64 * 2, smk = (2 * 64 + 4 * 32) * 64 * 2 + 4 * 32 * 4;
    set_smem(flash_bwd_dq_kernel<64>, smq);
    set_smem(flash_bwd_dkv_kernel<64>, smk);
    flash_bwd_dq_kernel<64><<<gq, 256, smq, stream>>>(q);
    flash_bwd_dkv_kernel<64><<<gk, 128, smk, stream>>>(kv);
  }
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "flash_bwd launch failed");
}

// D = rowsum(dO o O) alone (used by the tcgen05 backward).
void flash_dsum(torch::Tensor out, torch::Tensor dout, torch::Tensor dsum, int64_t B, int64_t T, int64_t H) {
  const int64_t C = out.size(1);
  const int HD = int(C / H);
  TORCH_CHECK(HD == 64 || HD == 128, "flash_dsum: head_dim");
  TORCH_CHECK(out.stride(1) == 1 && dout.stride(1) == 1 && dsum.numel() == B * H * T, "flash_dsum: shapes");
  AttnArgs d{};
  d.o = reinterpret_cast<const __nv_bfloat16*>(out.data_ptr());
  d.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  d.ld_out = out.stride(0);
  d.ld_do = dout.stride(0);
  d.dsum = dsum.data_ptr<float>();
  d.B = int(B); d.H = int(H); d.T = int(T);
  const long items = B * T * H;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (HD == 128) flash_bwd_dot_kernel<128><<<unsigned((items + 7) / 8), 256, 0, stream>>>(d);
  else flash_bwd_dot_kernel<64><<<unsigned((items + 7) / 8), 256, 0, stream>>>(d);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "flash_dsum launch failed");
}

}  // namespace nk

#ifndef NANOGPT_DEBUG_BOUNDS  // the bounds-checked debug extension does not carry the C entry point
// ---------------------------------------------------------------------------------------------
// Allocation-free C entry point (declared and documented in noalloc.h): the same
// three backward kernels, with the D = rowsum(dO o O) scratch taken from a fixed
// file-scope device array instead of a caller-provided tensor.
#include <mutex>

#include "noalloc.h"

static __device__ __align__(256) float g_noalloc_dsum[NANOGPT_NOALLOC_MAX_ROWS];

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoallocMaxDevices] = {};

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }
}  // namespace

extern "C" __attribute__((visibility("default"))) const char* nanogpt_noalloc_error_string(int code) {
  switch (code) {
    case NANOGPT_NOALLOC_OK: return "ok";
    case NANOGPT_NOALLOC_ERR_TOO_LARGE:
      return "batch * n_head * seq_len exceeds the fixed scratch of NANOGPT_NOALLOC_MAX_ROWS (1048576) floats";
    case NANOGPT_NOALLOC_ERR_BAD_ARG:
      return "invalid argument (null or unaligned pointer, head_dim not 64/128, non-positive size, or "
             "batch * n_head above 65535)";
    case NANOGPT_NOALLOC_ERR_CUDA: return "a CUDA runtime call failed (see cudaGetLastError)";
    default: return "unknown error code";
  }
}

extern "C" __attribute__((visibility("default"))) int nanogpt_flash_attention_bwd_noalloc(
    const void* qkv, const void* out, const void* dout, const float* lse, void* dqkv, int batch, int seq_len,
    int n_head, int head_dim, cudaStream_t stream) {
  using namespace nk;
  if (!qkv || !out || !dout || !lse || !dqkv) return NANOGPT_NOALLOC_ERR_BAD_ARG;
  if (!aligned16(qkv) || !aligned16(out) || !aligned16(dout) || !aligned16(dqkv)) return NANOGPT_NOALLOC_ERR_BAD_ARG;
  if (batch <= 0 || seq_len <= 0 || n_head <= 0 || (head_dim != 64 && head_dim != 128))
    return NANOGPT_NOALLOC_ERR_BAD_ARG;
  const size_t rows = size_t(batch) * size_t(n_head) * size_t(seq_len);
  if (rows > NANOGPT_NOALLOC_MAX_ROWS) return NANOGPT_NOALLOC_ERR_TOO_LARGE;
  // The kernels put (batch, head) pairs on grid.y, which holds at most 65535.
  if (size_t(batch) * size_t(n_head) > NANOGPT_NOALLOC_MAX_BATCH_HEADS) return NANOGPT_NOALLOC_ERR_BAD_ARG;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NANOGPT_NOALLOC_ERR_CUDA;
  if (dev < 0 || dev >= kNoallocMaxDevices) return NANOGPT_NOALLOC_ERR_BAD_ARG;
  float* scratch = nullptr;
  {
    // One-time set-up per device, with that device current: the host-side
    // symbol is only a stand-in, the kernels need the device address.
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_dsum) != cudaSuccess || !p) return NANOGPT_NOALLOC_ERR_CUDA;
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_noalloc_ptr[dev];
  }

  const long C = long(n_head) * head_dim;
  AttnArgs a{};
  auto base = static_cast<const __nv_bfloat16*>(qkv);
  a.q = base; a.k = base + C; a.v = base + 2 * C;
  a.ld_qkv = 3 * C;
  a.B = batch; a.H = n_head; a.T = seq_len;
  a.scale = 1.f / std::sqrt(float(head_dim));
  a.sl2 = a.scale * kLog2e;
  a.o = static_cast<const __nv_bfloat16*>(out);
  a.dout = static_cast<const __nv_bfloat16*>(dout);
  a.ld_do = C;
  a.lse = const_cast<float*>(lse);
  a.dsum = scratch;

  AttnArgs d = a;
  d.ld_out = C;
  auto dbase = static_cast<__nv_bfloat16*>(dqkv);
  AttnArgs q = a;
  q.out = dbase;
  q.ld_out = 3 * C;
  AttnArgs kv = a;
  kv.out = dbase + C;
  kv.out2 = dbase + 2 * C;
  kv.ld_out = 3 * C;
  const long items = long(batch) * seq_len * n_head;
  dim3 gq(unsigned((seq_len + 127) / 128), unsigned(batch * n_head));
  dim3 gk(unsigned((seq_len + 63) / 64), unsigned(batch * n_head));
  // An error left pending by earlier, unrelated work is reported without
  // being cleared, before anything is queued, so it is not mistaken for (or
  // hidden by) a failure of this call.
  if (cudaPeekAtLastError() != cudaSuccess) return NANOGPT_NOALLOC_ERR_CUDA;
  const int smq = (2 * 128 + 4 * 64) * head_dim * 2, smk = (2 * 64 + 4 * 32) * head_dim * 2 + 4 * 32 * 4;
  cudaError_t e = cudaSuccess;
  if (head_dim == 128) {
    e = cudaFuncSetAttribute(flash_bwd_dq_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smq);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(flash_bwd_dkv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smk);
  } else {
    e = cudaFuncSetAttribute(flash_bwd_dq_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smq);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(flash_bwd_dkv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smk);
  }
  if (e != cudaSuccess) return NANOGPT_NOALLOC_ERR_CUDA;
  // Each launch is checked on its own; a failed launch stops the sequence, so
  // a later kernel never consumes the output of one that did not run.
  if (head_dim == 128) flash_bwd_dot_kernel<128><<<unsigned((items + 7) / 8), 256, 0, stream>>>(d);
  else flash_bwd_dot_kernel<64><<<unsigned((items + 7) / 8), 256, 0, stream>>>(d);
  if (cudaGetLastError() != cudaSuccess) return NANOGPT_NOALLOC_ERR_CUDA;
  if (head_dim == 128) flash_bwd_dq_kernel<128><<<gq, 256, smq, stream>>>(q);
  else flash_bwd_dq_kernel<64><<<gq, 256, smq, stream>>>(q);
  if (cudaGetLastError() != cudaSuccess) return NANOGPT_NOALLOC_ERR_CUDA;
  if (head_dim == 128) flash_bwd_dkv_kernel<128><<<gk, 128, smk, stream>>>(kv);
  else flash_bwd_dkv_kernel<64><<<gk, 128, smk, stream>>>(kv);
  return cudaGetLastError() == cudaSuccess ? NANOGPT_NOALLOC_OK : NANOGPT_NOALLOC_ERR_CUDA;
}
#endif  // NANOGPT_DEBUG_BOUNDS
