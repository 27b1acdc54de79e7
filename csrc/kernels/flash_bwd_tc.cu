// Causal flash-attention backward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), head_dim 128, seq_len a multiple of 128.
//
// One CTA = one block of 128 keys of one (batch, head). K and V stay in
// shared memory; for every query block j >= the key block (causal) it
//   MMA1  S^T  = K  Q_j^T            -> TMEM [0,128)
//   MMA2  dP^T = V  dO_j^T           -> TMEM [128,256)
//   (compute warps, thread = key row)
//         P^T  = exp2(S^T * scale*log2e - lse2[q])   (causal mask on the diagonal)
//         dS^T = P^T o (dP^T - D[q])
//         P^T goes back to tensor memory (bf16 pairs, over the S^T columns just
//         read); dS^T goes to shared memory.
//   MMA3  dV  += P^T  dO_j           -> TMEM [384,512) (A operand from TMEM)
//   MMA4  dK  += dS^T Q_j            -> TMEM [256,384)
//   MMA5  dQ_j = dS K                -> TMEM [128,256) (dS^T's smem tile read as
//                                       an MN-major A operand: no transpose copy)
//   (drain warps, thread = query row) dQ_j * scale is added to an fp32
//   accumulator with TMA reduce-add tensor stores, staged through dS^T's
//   shared-memory tile once MMA5 has consumed it.
// Q_j / dO_j (and their LSE / D rows) are double-buffered.
// After the last block the compute warps write dK * scale (with the RoPE /
// QK-norm backward when requested) and dV (bf16) into the gradient buffer. A
// final small kernel converts the dQ accumulator to bf16.
//
// Warps: 0 = TMA/bulk loads, 1 = TMEM allocation + MMA issue, 2-9 = compute
// (two per TMEM lane quarter), 10-13 = dQ drain. Every wait is bounded
// (common.cuh).
#include <cstdlib>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "status.h"
#include "tma_host.h"

namespace nk {

namespace fb {
constexpr int HD = 128, BK = 128, BQ = 128;
constexpr int kThreads = 448;  // 2 + 8 compute + 4 drain warps
constexpr int kTile = 128 * 128 * 2;   // 32 KB
constexpr int kSub = 128 * 64 * 2;     // 16 KB swizzle sub-tile
constexpr int kStage = 32 * 32 * 4;  // 4 KB: one drain warp's 32 x 32 fp32 dQ chunk
// K, V, Q x2, dO x2, dS^T (also the dQ drain staging) + LSE/D x2 + barriers.
// No alignment slack: the dynamic shared memory base is checked to be
// 1024-byte aligned at run time (the kernel reports an error otherwise).
constexpr int kSmem = 7 * kTile + 2 * 2 * BQ * 4 + 256;
}  // namespace fb

struct FbArgs {
  __nv_bfloat16* dqkv;  // (B*T, 3C): dK / dV written here
  float* dq_acc;        // (B*T, C) fp32, zeroed by the host
  const float* lse;     // (B, H, T) base-2
  const float* dsum;    // (B, H, T)
  int B, H, T, C;
  float scale, sl2;
  int* err;
  // Optional RoPE + QK-norm backward folded into the dK/dQ write-out:
  // gradients w.r.t. the pre-RoPE k/q (the forward stored y = rms(rope(x))
  // in the QKV buffer and 1/denominator per (row, part, head) in rope_rstd).
  const __nv_bfloat16* qkv;
  const float* rope_rstd;
  const float* rope_cos;
  const float* rope_sin;
  // Measurement switch (NANOGPT_FB_DEBUG; gives wrong gradients when set):
  // bit 0 skips the dQ reduce-add, bit 1 replaces the softmax-gradient math by copies.
  int dbg;
};

__device__ __forceinline__ uint32_t tile_off(int r, int c) {  // 16B chunk c (of 16) in row r, K-major SW128
  return uint32_t((c >> 3) * fb::kSub + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(fb::kThreads, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tmo,
                        const __grid_constant__ CUtensorMap tmq, const FbArgs a) {
  using namespace fb;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if (smem_u32(smem) & 1023) {  // uniform: the whole CTA leaves before any barrier or TMEM use
    if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrTimeoutOther);
    return;
  }
  uint8_t* sK = smem;
  uint8_t* sV = smem + kTile;
  uint8_t* sQ = smem + 2 * kTile;   // [2] query blocks
  uint8_t* sO = smem + 4 * kTile;   // [2] dO blocks
  uint8_t* sS = smem + 6 * kTile;   // dS^T [key][query]; after the dQ product, the drain staging
  float* sL = reinterpret_cast<float*>(smem + 7 * kTile);  // [2] lse2 of the query block
  float* sD = sL + 2 * BQ;                                 // [2] D of the query block
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * kTile + 4 * BQ * 4);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;   // [2]
  uint64_t* qd_empty = bars + 3;  // [2]
  uint64_t* st_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* dq_full = bars + 7;
  uint64_t* dq_free = bars + 8;
  uint64_t* kv_done = bars + 9;
  uint64_t* stage_free = bars + 10;  // the drain's staging reads of dS^T's tile are done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb = blockIdx.x;  // key block; low blocks have the most query blocks
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int nq = a.T / BQ;
  const int nblk = nq - kb;   // query blocks kb .. nq-1
  const long bh = long(b) * a.H + h;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(p_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(kv_done, 1);
    mbar_init(stage_free, 4);
    fence_barrier_init();
    prefetch_tmap(&tm);
    prefetch_tmap(&tmo);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S^T @0, dP^T / dQ @128, dK @256, dV @384

  if (warp == 0) {
    if (lane == 0) {
      const int xq = h * HD, xk = a.C + h * HD, xv = 2 * a.C + h * HD;
      mbar_arrive_expect_tx(kv_full, 2 * kTile);
      for (int s = 0; s < 2; ++s) {
        tma_load_3d(sK + s * kSub, &tm, kv_full, xk + 64 * s, kb * BK, b);
        tma_load_3d(sV + s * kSub, &tm, kv_full, xv + 64 * s, kb * BK, b);
      }
      for (int n = 0; n < nblk; ++n) {
        const int j = kb + n, u = n & 1;
        if (!mbar_wait(&qd_empty[u], ((n >> 1) & 1) ^ 1, kErrTimeoutProducer, a.err)) break;
        mbar_arrive_expect_tx(&qd_full[u], 2 * kTile + 2 * BQ * 4);
        for (int s = 0; s < 2; ++s) {
          tma_load_3d(sQ + u * kTile + s * kSub, &tm, &qd_full[u], xq + 64 * s, j * BQ, b);
          tma_load_3d(sO + u * kTile + s * kSub, &tmo, &qd_full[u], h * HD + 64 * s, j * BQ, b);
        }
        bulk_load(sL + u * BQ, a.lse + bh * a.T + j * BQ, BQ * 4, &qd_full[u]);
        bulk_load(sD + u * BQ, a.dsum + bh * a.T + j * BQ, BQ * 4, &qd_full[u]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_kk = idesc_bf16(128, 128, false, false);  // MMA1, MMA2
      const uint32_t id_kn = idesc_bf16(128, HD, false, true);    // MMA3, MMA4: B MN-major
      const uint32_t id_nn = idesc_bf16(128, HD, true, true);     // MMA5: A and B MN-major
      const uint32_t k = smem_u32(sK), v = smem_u32(sV), ds = smem_u32(sS);
      bool ok = mbar_wait(kv_full, 0, kErrTimeoutMma, a.err);
      for (int n = 0; n < nblk && ok; ++n) {
        const int u = n & 1;
        const uint32_t q = smem_u32(sQ + u * kTile), o = smem_u32(sO + u * kTile);
        if (!mbar_wait(&qd_full[u], (n >> 1) & 1, kErrTimeoutMma, a.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kSub + (kk & 3) * 32;
          umma_bf16(tmem + 0, sw128_desc(k + off, 16, 1024), sw128_desc(q + off, 16, 1024), id_kk, kk > 0);
        }
        // dP^T reuses the columns of the previous dQ (and the compute warps
        // reuse dS^T's tile, the drain's staging): wait until it was drained.
        if (n > 0 && !mbar_wait(dq_free, (n - 1) & 1, kErrTimeoutMma, a.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kSub + (kk & 3) * 32;
          umma_bf16(tmem + 128, sw128_desc(v + off, 16, 1024), sw128_desc(o + off, 16, 1024), id_kk, kk > 0);
        }
        umma_commit(st_full);
        if (!mbar_wait(p_full, n & 1, kErrTimeoutMma, a.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {  // contraction over the 128 queries
          // P^T is in tensor memory: 32 query columns of chunk c packed as bf16
          // pairs in TMEM columns [32c, 32c + 16) (written over S^T).
          umma_bf16_ts(tmem + 384, tmem + 32 * (kk >> 1) + 8 * (kk & 1), sw128_desc(o + kk * 2048, kSub, 1024),
                       id_kn, (n > 0 || kk > 0) ? 1u : 0u);
          const uint32_t aoff = (kk >> 2) * kSub + (kk & 3) * 32;
          umma_bf16(tmem + 256, sw128_desc(ds + aoff, 16, 1024), sw128_desc(q + kk * 2048, kSub, 1024), id_kn,
                    (n > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&qd_empty[u]);  // Q_j / dO_j are no longer read
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {  // contraction over the 128 keys
          umma_bf16(tmem + 128, sw128_desc(ds + kk * 2048, kSub, 1024), sw128_desc(k + kk * 2048, kSub, 1024),
                    id_nn, kk > 0);
        }
        umma_commit(dq_full);
      }
      umma_commit(kv_done);
    }
  } else if (warp < 10) {
    // Compute warps: thread = key row; two warps per TMEM lane quarter, each
    // taking 64 of the block's 128 query columns.
    const int quarter = warp & 3;
    const int half = (warp - 2) / 4;
    const int r = quarter * 32 + lane;
    const int key = kb * BK + r;
    const uint32_t lanes = uint32_t(quarter * 32) << 16;
    bool ok = true;
    // P^T (into tensor memory, over this chunk's own S^T columns) and dS^T
    // (shared memory) for the 32 query columns starting at c * 32.
    auto chunk = [&](int c, int j, bool diag, int u) {
      float s[32], dp[32];
      tmem_ld_32x32(tmem + lanes + c * 32, s);
      tmem_ld_32x32(tmem + lanes + 128 + c * 32, dp);
      const float* L = sL + u * BQ;
      const float* D = sD + u * BQ;
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(L + c * 32 + i);
        const float4 d4 = *reinterpret_cast<const float4*>(D + c * 32 + i);
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
        float pv[4], gv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (a.dbg & 2) { pv[e] = s[i + e]; gv[e] = dp[i + e]; continue; }
          pv[e] = exp2f(fmaf(s[i + e], a.sl2, -lv[e]));
          if (diag && (j * BQ + c * 32 + i + e) < key) pv[e] = 0.f;
          gv[e] = pv[e] * (dp[i + e] - dv4[e]);
        }
        pp[i / 2] = pack_bf16x2(pv[0], pv[1]);
        pp[i / 2 + 1] = pack_bf16x2(pv[2], pv[3]);
        dd[i / 2] = pack_bf16x2(gv[0], gv[1]);
        dd[i / 2 + 1] = pack_bf16x2(gv[2], gv[3]);
      }
      tmem_st_32x16(tmem + lanes + c * 32, pp);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(sS + tile_off(r, c * 4 + q)) = make_uint4(dd[4 * q], dd[4 * q + 1], dd[4 * q + 2], dd[4 * q + 3]);
    };
    for (int n = 0; n < nblk && ok; ++n) {
      const int j = kb + n, u = n & 1;
      if (!mbar_wait(st_full, n & 1, kErrTimeoutEpilogue, a.err)) { ok = false; break; }
      tc_fence_after();
      // st_full of block n comes after the previous block's dQ product and
      // TMEM drain (dP^T waited for it); dS^T's tile is also the drain's
      // staging, so wait for its reads too.
      if (n > 0 && !mbar_wait(stage_free, (n - 1) & 1, kErrTimeoutEpilogue, a.err)) { ok = false; break; }
      if (n == 0) {  // the diagonal block: causal mask
        chunk(2 * half, j, true, u);
        chunk(2 * half + 1, j, true, u);
      } else {
        chunk(2 * half, j, false, u);
        chunk(2 * half + 1, j, false, u);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && mbar_wait(kv_done, 0, kErrTimeoutEpilogue, a.err)) {
      tc_fence_after();
      if (key < a.T && half == 1) {
        __nv_bfloat16* dv = a.dqkv + (long(b) * a.T + key) * 3 * a.C + 2 * a.C + h * HD;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float y[32];
          tmem_ld_32x32(tmem + lanes + 384 + c * 32, y);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(dv + c * 32 + u * 8) = make_uint4(
                pack_bf16x2(y[8 * u], y[8 * u + 1]), pack_bf16x2(y[8 * u + 2], y[8 * u + 3]),
                pack_bf16x2(y[8 * u + 4], y[8 * u + 5]), pack_bf16x2(y[8 * u + 6], y[8 * u + 7]));
        }
      } else if (key < a.T) {
        __nv_bfloat16* dk = a.dqkv + (long(b) * a.T + key) * 3 * a.C + a.C + h * HD;
        // dK = scale * acc; with the RoPE fold, d/dx of y = rms(rope(x)):
        // dr = r (g - y <g, y> / D), then the transposed rotation of the
        // pairs (i, i + 64). Columns are processed 32 + 32 at a time.
        const long row = long(b) * a.T + key;
        const __nv_bfloat16* yk = a.qkv + row * 3 * a.C + a.C + h * HD;
        // Each lane reads its own row of y and of the RoPE tables: 16-byte
        // vector loads (8 bf16 / 4 fp32) keep the warp's cache-line requests
        // per column few.
        auto load8 = [](const __nv_bfloat16* p, float (&v)[8]) {
          const uint4 w = *reinterpret_cast<const uint4*>(p);
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16x2(ws[k]);
            v[2 * k] = f.x;
            v[2 * k + 1] = f.y;
          }
        };
        float dot = 0.f, r = 0.f;
        if (a.rope_rstd) {
          r = a.rope_rstd[row * 2 * a.H + a.H + h];
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            float x[32];
            tmem_ld_32x32(tmem + lanes + 256 + c * 32, x);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              float y[8];
              load8(yk + c * 32 + u * 8, y);
#pragma unroll
              for (int k = 0; k < 8; ++k) dot += y[k] * x[u * 8 + k];
            }
          }
          dot *= a.scale / float(HD);
        }
        const float* crow = a.rope_rstd ? a.rope_cos + long(key) * 64 : nullptr;
        const float* srow = a.rope_rstd ? a.rope_sin + long(key) * 64 : nullptr;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float x1[32], x2[32];
          tmem_ld_32x32(tmem + lanes + 256 + c * 32, x1);
          tmem_ld_32x32(tmem + lanes + 256 + (c + 2) * 32, x2);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float y1[8], y2[8], cs[8], sn[8];
            if (a.rope_rstd) {
              load8(yk + c * 32 + u * 8, y1);
              load8(yk + 64 + c * 32 + u * 8, y2);
#pragma unroll
              for (int k = 0; k < 8; k += 4) {
                const float4 c4 = __ldg(reinterpret_cast<const float4*>(crow + c * 32 + u * 8 + k));
                const float4 s4 = __ldg(reinterpret_cast<const float4*>(srow + c * 32 + u * 8 + k));
                cs[k] = c4.x; cs[k + 1] = c4.y; cs[k + 2] = c4.z; cs[k + 3] = c4.w;
                sn[k] = s4.x; sn[k + 1] = s4.y; sn[k + 2] = s4.z; sn[k + 3] = s4.w;
              }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int i = u * 8 + k;
              float g1 = x1[i] * a.scale, g2 = x2[i] * a.scale;
              if (a.rope_rstd) {
                const float d1 = r * (g1 - y1[k] * dot), d2 = r * (g2 - y2[k] * dot);
                g1 = d1 * cs[k] - d2 * sn[k];  // dx1 = dy1 cos - dy2 sin
                g2 = d1 * sn[k] + d2 * cs[k];  // dx2 = dy1 sin + dy2 cos
              }
              x1[i] = g1;
              x2[i] = g2;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            *reinterpret_cast<uint4*>(dk + c * 32 + u * 8) =
                make_uint4(pack_bf16x2(x1[8 * u], x1[8 * u + 1]), pack_bf16x2(x1[8 * u + 2], x1[8 * u + 3]),
                           pack_bf16x2(x1[8 * u + 4], x1[8 * u + 5]), pack_bf16x2(x1[8 * u + 6], x1[8 * u + 7]));
            *reinterpret_cast<uint4*>(dk + 64 + c * 32 + u * 8) =
                make_uint4(pack_bf16x2(x2[8 * u], x2[8 * u + 1]), pack_bf16x2(x2[8 * u + 2], x2[8 * u + 3]),
                           pack_bf16x2(x2[8 * u + 4], x2[8 * u + 5]), pack_bf16x2(x2[8 * u + 6], x2[8 * u + 7]));
          }
        }
      } else {
        // Lanes past the sequence still take part in the warp-collective loads.
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float x[32];
          tmem_ld_32x32(tmem + lanes + (half ? 384 : 256) + c * 32, x);
        }
      }
    }
  } else {
    // dQ drain warps: thread = query row of the current block. Each warp
    // stages 32 rows x 32 columns of dQ * scale (fp32, 128B-swizzled) and
    // adds them to the fp32 accumulator with one TMA reduce-add; two staging
    // buffers per warp let the next chunk fill while the previous one drains.
    const int quarter = warp & 3;
    const uint32_t lanes = uint32_t(quarter * 32) << 16;
    uint8_t* stage = sS + (warp - 10) * 2 * kStage;  // dS^T's tile: free once dQ = dS K is done
    int chunks = 0;
    for (int n = 0; n < nblk; ++n) {
      const int j = kb + n;
      if (!mbar_wait(dq_full, n & 1, kErrTimeoutEpilogue, a.err)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c, ++chunks) {
        float x[32];
        tmem_ld_32x32(tmem + lanes + 128 + c * 32, x);
        if (a.dbg & 1) continue;
        uint8_t* buf = stage + (chunks & 1) * kStage;
        if (lane == 0 && c >= 2) bulk_wait_read<1>();  // this buffer's previous reduce has read it
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(buf + lane * 128 + ((k ^ (lane & 7)) << 4)) =
              make_float4(x[4 * k] * a.scale, x[4 * k + 1] * a.scale, x[4 * k + 2] * a.scale, x[4 * k + 3] * a.scale);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];"
                       ::"l"(&tmq), "r"(smem_u32(buf)), "r"(h * HD + c * 32), "r"(b * a.T + j * BQ + quarter * 32)
                       : "memory");
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);  // dQ's TMEM columns are free for the next dP^T
      // The staging reads must be done before the compute warps rewrite dS^T.
      if (lane == 0) {
        bulk_wait_read<0>();
        mbar_arrive(stage_free);
      }
    }
    if (lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ accumulator (fp32, (B*T, C)) -> bf16 q columns of dqkv, optionally
// through the RoPE + QK-norm backward. One warp per (token, head); lane l
// owns elements [4l, 4l+4), its rotation partners live in lane l ^ 16.
__global__ void dq_finish_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dqkv, long rows, int T,
                                 int H, int C, const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ rstd,
                                 const float* __restrict__ cos_t, const float* __restrict__ sin_t) {
  const long item = long(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (item >= rows * H) return;
  const long row = item / H;
  const int h = int(item % H);
  const float4 g4 = *reinterpret_cast<const float4*>(acc + row * C + h * 128 + lane * 4);
  float g[4] = {g4.x, g4.y, g4.z, g4.w};
  if (rstd) {
    const uint2 w = *reinterpret_cast<const uint2*>(qkv + row * 3 * C + h * 128 + lane * 4);
    const float2 y0 = unpack_bf16x2(w.x), y1 = unpack_bf16x2(w.y);
    const float y[4] = {y0.x, y0.y, y1.x, y1.y};
    float dot = y[0] * g[0] + y[1] * g[1] + y[2] * g[2] + y[3] * g[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot /= 128.f;
    const float r = rstd[row * 2 * H + h];
    const int pos = int(row % T);
    float dr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) dr[j] = r * (g[j] - y[j] * dot);
    const bool first = lane < 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float partner = __shfl_xor_sync(0xffffffffu, dr[j], 16);
      const int i = (lane & 15) * 4 + j;
      const float cs = cos_t[pos * 64 + i], sn = sin_t[pos * 64 + i];
      g[j] = first ? dr[j] * cs - partner * sn : partner * sn + dr[j] * cs;
    }
  }
  *reinterpret_cast<uint2*>(dqkv + row * 3 * C + h * 128 + lane * 4) =
      make_uint2(pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]));
}

bool flash_bwd_tc_supported(int64_t T, int64_t HD) { return HD == 128 && T % 128 == 0; }

// 3-D map over a (B*T, width) bf16 activation: inner `width` columns, then the
// T rows of one sequence, then B sequences (rows past a sequence read as zeros).
static CUtensorMap seq_map_3d(void* base, int64_t B, int64_t T, int64_t width) {
  CUtensorMap m;
  cuuint64_t dims[3] = {cuuint64_t(width), cuuint64_t(T), cuuint64_t(B)};
  cuuint64_t strides[2] = {cuuint64_t(width * 2), cuuint64_t(T * width * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "flash_bwd_tc: tensor map encode failed ", int(r));
  return m;
}

void flash_dsum(torch::Tensor out, torch::Tensor dout, torch::Tensor dsum, int64_t B, int64_t T, int64_t H);

// The backward's memory-bound preparation: D = rowsum(dO o O) and the zeroed
// fp32 dQ accumulator. Separate so a caller can run it on another stream
// (next to an independent GEMM) and then call flash_bwd_tc with prepared=true.
void flash_bwd_prep(torch::Tensor out, torch::Tensor dout, torch::Tensor dsum, torch::Tensor dq_acc, int64_t B,
                    int64_t T, int64_t H) {
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() && dq_acc.numel() == B * T * out.size(1),
              "flash_bwd_prep: dq_acc");
  const at::cuda::CUDAGuard guard(out.device());
  flash_dsum(out, dout, dsum, B, T, H);
  TORCH_CHECK(cudaMemsetAsync(dq_acc.data_ptr(), 0, size_t(dq_acc.numel()) * 4, at::cuda::getCurrentCUDAStream()) ==
                  cudaSuccess,
              "flash_bwd_prep: memset");
}

// Full backward with the tcgen05 kernel: D precompute and zeroed fp32 dQ
// accumulator (caller's scratch; skipped when `prepared`), the main kernel,
// then dQ -> bf16.
void flash_bwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor dsum,
                  torch::Tensor dq_acc, torch::Tensor dqkv, int64_t B, int64_t T, int64_t H,
                  c10::optional<torch::Tensor> rope_rstd, c10::optional<torch::Tensor> rope_cos,
                  c10::optional<torch::Tensor> rope_sin, bool prepared) {
  using namespace fb;
  const int64_t C = qkv.size(1) / 3;
  TORCH_CHECK(qkv.is_contiguous() && dqkv.is_contiguous() && dout.is_contiguous() && out.is_contiguous(),
              "flash_bwd_tc: contiguous tensors");
  TORCH_CHECK(C == H * HD && qkv.size(0) == B * T && flash_bwd_tc_supported(T, C / H), "flash_bwd_tc: shape");
  TORCH_CHECK(dqkv.sizes() == qkv.sizes() && dout.size(1) == C && out.size(1) == C, "flash_bwd_tc: shapes");
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.numel() == B * T * C && dq_acc.is_contiguous(),
              "flash_bwd_tc: dq_acc");
  TORCH_CHECK(lse.numel() == B * H * T && dsum.numel() == B * H * T, "flash_bwd_tc: lse/dsum");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(lse.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(dsum.data_ptr()) % 16 == 0, "flash_bwd_tc: 16-byte aligned lse/dsum");
  const at::cuda::CUDAGuard guard(qkv.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (!prepared) {
    flash_dsum(out, dout, dsum, B, T, H);
    TORCH_CHECK(cudaMemsetAsync(dq_acc.data_ptr(), 0, size_t(B * T * C) * 4, stream) == cudaSuccess,
                "flash_bwd_tc: memset");
  }
  CUtensorMap tm = seq_map_3d(qkv.data_ptr(), B, T, 3 * C);
  CUtensorMap tmo = seq_map_3d(dout.data_ptr(), B, T, C);
  CUtensorMap tmq;
  {
    cuuint64_t dims[2] = {cuuint64_t(C), cuuint64_t(B * T)};
    cuuint64_t strides[1] = {cuuint64_t(C * 4)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    TORCH_CHECK(reinterpret_cast<uintptr_t>(dq_acc.data_ptr()) % 16 == 0, "flash_bwd_tc: dq_acc alignment");
    CUresult r = encode_tiled_fn()(&tmq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dq_acc.data_ptr(), dims, strides, box,
                                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "flash_bwd_tc: dq tensor map encode failed ", int(r));
  }
  FbArgs a{};
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.dq_acc = dq_acc.data_ptr<float>();
  a.lse = lse.data_ptr<float>();
  a.dsum = dsum.data_ptr<float>();
  a.B = int(B); a.H = int(H); a.T = int(T); a.C = int(C);
  a.scale = 1.f / std::sqrt(float(HD));
  a.sl2 = a.scale * 1.4426950408889634f;
  a.err = error_word();
  if (const char* d = std::getenv("NANOGPT_FB_DEBUG")) a.dbg = std::atoi(d);
  if (rope_rstd.has_value()) {
    TORCH_CHECK(rope_cos.has_value() && rope_sin.has_value() && rope_cos->size(1) == 64 && rope_cos->size(0) >= T &&
                    rope_cos->is_contiguous() && rope_sin->is_contiguous() &&
                    reinterpret_cast<uintptr_t>(rope_cos->data_ptr()) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(rope_sin->data_ptr()) % 16 == 0,
                "flash_bwd_tc: rope tables (T, 64), contiguous, 16-byte aligned");
    a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
    a.rope_rstd = rope_rstd->data_ptr<float>();
    a.rope_cos = rope_cos->data_ptr<float>();
    a.rope_sin = rope_sin->data_ptr<float>();
  }
  static bool configured = false;
  if (!configured) {
    TORCH_CHECK(cudaFuncSetAttribute(flash_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) ==
                    cudaSuccess, "flash_bwd_tc: smem");
    configured = true;
  }
  dim3 grid(unsigned(T / BK), unsigned(B * H));
  flash_bwd_tc_kernel<<<grid, kThreads, kSmem, stream>>>(tm, tmo, tmq, a);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "flash_bwd_tc launch failed");
  const long items = B * T * H;
  dq_finish_kernel<<<unsigned((items + 7) / 8), 256, 0, stream>>>(a.dq_acc, a.dqkv, B * T, int(T), int(H), int(C),
                                                                a.qkv, a.rope_rstd, a.rope_cos, a.rope_sin);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "dq_finish launch failed");
}

}  // namespace nk
