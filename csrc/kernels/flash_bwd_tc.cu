// Causal flash-attention backward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), head_dim 128, seq_len a multiple of 128.
//
// One CTA = one block of 128 keys of one (batch, head). K and V stay in
// shared memory; the CTA walks the query blocks of 64 rows j that can see its
// keys (causal) and for each one
//   S^T  = K  Q_j^T                     (M 128 keys, N 64 queries)
//   dP^T = V  dO_j^T
//   (softmax warps, thread = key row)
//         P^T  = exp2(S^T * scale*log2e - lse2[q])   (causal mask near the diagonal)
//         dS^T = P^T o (dP^T - D[q])
//         P^T goes back to tensor memory (bf16 pairs, over the S^T columns just
//         read); dS^T goes to shared memory.
//   dQ_j^T = K^T dS^T                   (M 128 = head_dim, N 64 queries), into
//                                        the dP^T columns the softmax just read
//   dV  += P^T  dO_j                    (A operand from tensor memory)
//   dK  += dS^T Q_j
//   (drain warps, thread = head-dim lane) dQ_j * scale is added to an fp32
//   accumulator with TMA reduce-add tensor stores.
//
// Tensor memory (512 columns): S^T [0,64) and [64,128) and dP^T / dQ^T
// [128,192) and [192,256) for two query blocks in flight, dK [256,384),
// dV [384,512). With two score buffers the MMA warp issues block j+1's S^T and
// dP^T before block j's gradient products, so the softmax-gradient math of
// block j overlaps five MMAs (those of block j-1 and the scores of j+1) and
// the drain of dQ_{j-1} overlaps three (dV_{j-1}, dK_{j-1}, S_{j+1}); the
// issue order per block is dQ, dV, dK so the drain starts as early as
// possible. Q_j / dO_j (and their LSE / D rows) rotate through three stages.
// After the last block the softmax warps write dK * scale (with the RoPE /
// QK-norm backward when requested) and dV (bf16) into the gradient buffer. A
// final small kernel converts the dQ accumulator to bf16.
//
// Warps: 0 = TMA/bulk loads, 1 = TMEM allocation + MMA issue, 2-9 = softmax
// gradient (two per TMEM lane quarter, 32 query columns each), 10-13 = dQ
// drain. Every wait is bounded (common.cuh).
#include <cstdlib>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "status.h"
#include "tma_host.h"

namespace nk {

namespace fb {
constexpr int HD = 128, BK = 128, BQ = 64, NS = 3;
constexpr int kStage = 32 * 32 * 4;      // 4 KB: one drain warp's 32 x 32 fp32 dQ chunk
constexpr int kThreads = 448;            // 2 + 8 softmax + 4 drain warps
constexpr int kKTile = 128 * 128 * 2;    // 32 KB: K or V (two 64-column sub-tiles)
constexpr int kKSub = 128 * 64 * 2;      // 16 KB
constexpr int kQTile = BQ * 128 * 2;     // 16 KB: one query block of Q or dO
constexpr int kQSub = BQ * 64 * 2;       // 8 KB
constexpr int kDsTile = 128 * BQ * 2;    // 16 KB: dS^T [key][query], one 128-byte-row sub-tile
constexpr int kOffK = 0, kOffV = kKTile, kOffQ = 2 * kKTile, kOffO = kOffQ + NS * kQTile,
              kOffDs = kOffO + NS * kQTile, kOffStage = kOffDs + 2 * kDsTile,
              kOffLD = kOffStage + 4 * 2 * kStage, kOffBar = kOffLD + NS * 2 * BQ * 4;
// No alignment slack: the dynamic shared memory base is checked to be
// 1024-byte aligned at run time (the kernel reports an error otherwise).
constexpr int kSmem = kOffBar + 256;
static_assert(kSmem <= 232448, "shared memory budget");
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
  // bit 0 skips the dQ reduce-add, bit 2 skips the dQ^T MMAs, bit 3 the dV / dK MMAs, bit 4 the S^T / dP^T MMAs,
  // bit 5 makes the MMA warp skip its wait for the dQ^T drain, bit 7 loads only
  // the first stages' Q / dO (later stages are released without a copy), bit 8
  // skips the dK / dV write-out, bit 9 records a timeline (g_fb_trace), bit 13
  // adds dQ with red.global.add from registers instead of TMA reduce-adds, bit 14
  // makes the MMA warp skip its wait for the softmax warps.
  int dbg;
  int st_defer;  // NANOGPT_BWD_ST_DEFER (default 1): see the P^T store in the softmax-gradient warps
};

// Timeline of the first CTA (measurement switch NANOGPT_FB_DEBUG bit 9): per
// query block n, clock64 stamps at slot [n * 16 + k]: k = 0 scores of n + 1
// issued, 1 P of n ready (MMA warp), 2 gradient MMAs of n issued, 3 scores of n
// seen by the softmax warps, 4 softmax of n done, 5 dQ^T of n seen by the
// drain, 6 dQ^T of n read out; softmax internals 8 tensor-memory loads done,
// 9 math done, 10 P^T stored to tensor memory, 11 dS^T stored to shared memory.
__device__ long long g_fb_trace[64 * 16];

template <bool DBG>
__device__ __forceinline__ void fb_stamp(const FbArgs& a, int n, int k) {
  if (DBG && (DBG && (a.dbg & 512)) && blockIdx.x == 0 && blockIdx.y == 0 && n < 64) g_fb_trace[n * 16 + k] = clock64();
}

// DBG: the build with the measurement switches (NANOGPT_FB_DEBUG); the
// production instantiation carries none of their code.
template <bool DBG>
__global__ void __launch_bounds__(fb::kThreads, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tmo,
                        const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmd,
                        const FbArgs a) {
  using namespace fb;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if (smem_u32(smem) & 1023) {  // uniform: the whole CTA leaves before any barrier or TMEM use
    if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrTimeoutOther);
    return;
  }
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  uint8_t* sQ = smem + kOffQ;    // [NS] query blocks
  uint8_t* sO = smem + kOffO;    // [NS] dO blocks
  uint8_t* sDs = smem + kOffDs;  // [2] dS^T tiles
  float* sL = reinterpret_cast<float*>(smem + kOffLD);  // [NS] lse2 of the query block
  float* sD = sL + NS * BQ;                             // [NS] D of the query block
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;    // [NS]
  uint64_t* qd_empty = bars + 1 + NS;   // [NS]
  uint64_t* st_full = bars + 1 + 2 * NS;    // [2] S^T and dP^T of a block are in tensor memory
  uint64_t* p_full = st_full + 2;     // [2] P^T (tensor memory) and dS^T (shared memory) written
  uint64_t* dq_full = p_full + 2;   // [2] dQ^T of a block is in tensor memory
  uint64_t* dq_free = dq_full + 2;   // [2] ... and has been read out by the drain warps
  uint64_t* kv_done = dq_free + 2;
  uint64_t* epi_full = kv_done + 1;  // all 8 softmax warps staged their dK / dV rows
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_full + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb = blockIdx.x;  // key block; low blocks have the most query blocks
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int nq = a.T / BQ;
  const int j0 = kb * (BK / BQ);  // first query block that sees a key of this block
  const int nblk = nq - j0;
  const long bh = long(b) * a.H + h;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&st_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], 4);
    }
    mbar_init(kv_done, 1);
    mbar_init(epi_full, 8);
    fence_barrier_init();
    prefetch_tmap(&tm);
    prefetch_tmap(&tmo);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const int xq = h * HD, xk = a.C + h * HD, xv = 2 * a.C + h * HD;
      mbar_arrive_expect_tx(kv_full, 2 * kKTile);
      for (int s = 0; s < 2; ++s)
        for (int r = 0; r < 2; ++r) {  // 64-row boxes: the second lands 8 KB into the sub-tile
          if (!NK_IN_BOUNDS(kb * BK + 64 * r < a.T && b < a.B && xv + 64 * s < 3 * a.C, a.err)) continue;
          tma_load_3d(sK + s * kKSub + r * kQSub, &tm, kv_full, xk + 64 * s, kb * BK + 64 * r, b);
          tma_load_3d(sV + s * kKSub + r * kQSub, &tm, kv_full, xv + 64 * s, kb * BK + 64 * r, b);
        }
      for (int n = 0; n < nblk; ++n) {
        const int j = j0 + n, st = n % NS;
        if (!mbar_wait(&qd_empty[st], ((n / NS) & 1) ^ 1, kErrTimeoutProducer, a.err)) break;
        if ((DBG && (a.dbg & 128)) && n >= NS) {
          mbar_arrive(&qd_full[st]);
          continue;
        }
        mbar_arrive_expect_tx(&qd_full[st], 2 * kQTile + 2 * BQ * 4);
        if (!NK_IN_BOUNDS(j * BQ + BQ <= a.T && xq + 128 <= a.C, a.err)) break;
        for (int s = 0; s < 2; ++s) {
          tma_load_3d(sQ + st * kQTile + s * kQSub, &tm, &qd_full[st], xq + 64 * s, j * BQ, b);
          tma_load_3d(sO + st * kQTile + s * kQSub, &tmo, &qd_full[st], h * HD + 64 * s, j * BQ, b);
        }
        bulk_load(sL + st * BQ, a.lse + bh * a.T + j * BQ, BQ * 4, &qd_full[st]);
        bulk_load(sD + st * BQ, a.dsum + bh * a.T + j * BQ, BQ * 4, &qd_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, BQ, false, false);  // S^T, dP^T
      const uint32_t id_kn = idesc_bf16(128, HD, false, true);  // dV, dK: B MN-major
      const uint32_t id_q = idesc_bf16(128, BQ, true, true);    // dQ^T: A and B MN-major
      const uint32_t k = smem_u32(sK), v = smem_u32(sV);
      // Base descriptors; every operand below is one of these plus a constant offset.
      const uint64_t dk_km = sw128_desc(k, 16, 1024), dv_km = sw128_desc(v, 16, 1024);
      const uint64_t dk_mn = sw128_desc(k, kKSub, 1024);
      const uint64_t dq_km = sw128_desc(smem_u32(sQ), 16, 1024), do_km = sw128_desc(smem_u32(sO), 16, 1024);
      const uint64_t dq_mn = sw128_desc(smem_u32(sQ), kQSub, 1024), do_mn = sw128_desc(smem_u32(sO), kQSub, 1024);
      const uint64_t dds_km = sw128_desc(smem_u32(sDs), 16, 1024), dds_mn = sw128_desc(smem_u32(sDs), kDsTile, 1024);
      // Scores of block n into buffer n & 1.
      auto scores = [&](int n) -> bool {
        const int st = n % NS, u = n & 1;
        if (!mbar_wait(&qd_full[st], (n / NS) & 1, kErrTimeoutMma, a.err)) return false;
        tc_fence_after();
        const uint32_t qs = st * kQTile;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          if (DBG && (a.dbg & 16)) break;
          const uint32_t ka = (kk >> 2) * kKSub + (kk & 3) * 32, qa = (kk >> 2) * kQSub + (kk & 3) * 32;
          umma_bf16(tmem + 64 * u, desc_advance(dk_km, ka), desc_advance(dq_km, qs + qa), id_s, kk > 0);
        }
        // dP^T reuses the columns of dQ^T of block n - 2: wait until it was drained.
        if (n >= 2 && !(DBG && (a.dbg & 32)) && !mbar_wait(&dq_free[u], ((n - 2) >> 1) & 1, kErrTimeoutMma, a.err))
          return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          if (DBG && (a.dbg & 16)) break;
          const uint32_t ka = (kk >> 2) * kKSub + (kk & 3) * 32, qa = (kk >> 2) * kQSub + (kk & 3) * 32;
          umma_bf16(tmem + 128 + 64 * u, desc_advance(dv_km, ka), desc_advance(do_km, qs + qa), id_s, kk > 0);
        }
        umma_commit(&st_full[u]);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, kErrTimeoutMma, a.err) && scores(0);
      for (int n = 0; n < nblk && ok; ++n) {
        const int st = n % NS, u = n & 1;
        if (n + 1 < nblk && !scores(n + 1)) break;
        fb_stamp<DBG>(a, n, 0);
        if (!(DBG && (a.dbg & 16384)) && !mbar_wait(&p_full[u], (n >> 1) & 1, kErrTimeoutMma, a.err)) break;
        fb_stamp<DBG>(a, n, 1);
        tc_fence_after();
        const uint32_t qs = st * kQTile, dss = u * kDsTile;
#pragma unroll
        for (int kk = 0; kk < BK / 16 && !(DBG && (a.dbg & 4)); ++kk)  // dQ^T = K^T dS^T: contraction over the 128 keys
          umma_bf16(tmem + 128 + 64 * u, desc_advance(dk_mn, kk * 2048), desc_advance(dds_mn, dss + kk * 2048), id_q,
                    kk > 0);
        umma_commit(&dq_full[u]);
#pragma unroll
        for (int kk = 0; kk < BQ / 16 && !(DBG && (a.dbg & 8)); ++kk) {  // contraction over the 64 queries
          // P^T is in tensor memory: 32 query columns of chunk c packed as bf16
          // pairs in TMEM columns [64u + 32c, 64u + 32c + 16) (written over S^T).
          umma_bf16_ts(tmem + 384, tmem + 64 * u + 32 * (kk >> 1) + 8 * (kk & 1), desc_advance(do_mn, qs + kk * 2048),
                       id_kn, (n > 0 || kk > 0) ? 1u : 0u);
          umma_bf16(tmem + 256, desc_advance(dds_km, dss + kk * 32), desc_advance(dq_mn, qs + kk * 2048), id_kn,
                    (n > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&qd_empty[st]);  // Q_j / dO_j / their LSE and D rows are no longer read
        fb_stamp<DBG>(a, n, 2);
      }
      umma_commit(kv_done);
    }
  } else if (warp < 10) {
    // Softmax-gradient warps: thread = key row; two warps per TMEM lane
    // quarter, each taking 32 of the block's 64 query columns.
    const int quarter = warp & 3;
    const int half = (warp - 2) / 4;  // query chunk of this warp
    const int r = quarter * 32 + lane;
    const int key = kb * BK + r;
    const uint32_t lanes = uint32_t(quarter * 32) << 16;
    bool ok = true;
    for (int n = 0; n < nblk && ok; ++n) {
      const int j = j0 + n, u = n & 1, st = n % NS;
      // The block's lse2 / D rows arrived with its Q tile (long before its
      // scores): fetch this warp's 32 + 32 of them into registers now, so the
      // shared-memory loads (which queue behind the tensor cores' operand
      // reads) complete while the warp waits for the scores.
      float lv[32], dv[32];
      if (!mbar_wait(&qd_full[st], (n / NS) & 1, kErrTimeoutEpilogue, a.err)) { ok = false; break; }
      {
        const float4* L4 = reinterpret_cast<const float4*>(sL + st * BQ + 32 * half);
        const float4* D4 = reinterpret_cast<const float4*>(sD + st * BQ + 32 * half);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 l4 = L4[i], d4 = D4[i];
          lv[4 * i] = l4.x; lv[4 * i + 1] = l4.y; lv[4 * i + 2] = l4.z; lv[4 * i + 3] = l4.w;
          dv[4 * i] = d4.x; dv[4 * i + 1] = d4.y; dv[4 * i + 2] = d4.z; dv[4 * i + 3] = d4.w;
        }
      }
      // st_full of block n is committed after every MMA of block n - 2, so
      // dS^T tile u (read by dK / dQ of block n - 2) is free as well.
      if (!mbar_wait(&st_full[u], (n >> 1) & 1, kErrTimeoutEpilogue, a.err)) { ok = false; break; }
      if (warp == 2 && lane == 0) fb_stamp<DBG>(a, n, 3);
      tc_fence_after();
      const bool diag = n < BK / BQ;
      const int q0 = j * BQ + 32 * half;
      uint32_t pp[16], dd[16];
      // Two halves of 16 columns keep the live registers under the budget.
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t sr[16], dr[16];  // both loads in flight, one wait
        tmem_ld_32x16_issue(tmem + lanes + 64 * u + 32 * half + 16 * hh, sr);
        tmem_ld_32x16_issue(tmem + lanes + 128 + 64 * u + 32 * half + 16 * hh, dr);
        tmem_ld_wait16(sr);
        tmem_ld_wait16(dr);
        if (warp == 2 && lane == 0 && hh == 0) fb_stamp<DBG>(a, n, 8);
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          float pv[2], gv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 16 * hh + i + e;
            pv[e] = ex2_approx(fmaf(__uint_as_float(sr[i + e]), a.sl2, -lv[c]));
            if (diag && (q0 + c) < key) pv[e] = 0.f;
            gv[e] = pv[e] * (__uint_as_float(dr[i + e]) - dv[c]);
          }
          pp[(16 * hh + i) / 2] = pack_bf16x2(pv[0], pv[1]);
          dd[(16 * hh + i) / 2] = pack_bf16x2(gv[0], gv[1]);
        }
      }
      if (warp == 2 && lane == 0) fb_stamp<DBG>(a, n, 9);
      // P^T to tensor memory; with st_defer its completion is awaited after the
      // dS^T shared-memory stores below, so the two overlap.
      if (a.st_defer) tmem_st_32x16_issue(tmem + lanes + 64 * u + 32 * half, pp);
      else tmem_st_32x16(tmem + lanes + 64 * u + 32 * half, pp);
      if (warp == 2 && lane == 0) fb_stamp<DBG>(a, n, 10);
      uint8_t* ds = sDs + u * kDsTile;
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 16-byte chunk 4 * half + c of row r, 128-byte swizzle
        const int cc = 4 * half + c;
        *reinterpret_cast<uint4*>(ds + r * 128 + ((cc ^ (r & 7)) << 4)) =
            make_uint4(dd[4 * c], dd[4 * c + 1], dd[4 * c + 2], dd[4 * c + 3]);
      }
      if (warp == 2 && lane == 0) fb_stamp<DBG>(a, n, 11);
      if (a.st_defer) tmem_st_wait();
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (warp == 2 && lane == 0) fb_stamp<DBG>(a, n, 4);
      if (lane == 0) mbar_arrive(&p_full[u]);
    }
    if (ok && mbar_wait(kv_done, 0, kErrTimeoutEpilogue, a.err) && !(DBG && (a.dbg & 256)) &&
        NK_IN_BOUNDS(key < a.T && b < a.B && h < a.H, a.err)) {
      tc_fence_after();
      // dK (warps of chunk 0) and dV (chunk 1) are staged as bf16 tiles in
      // the now idle Q / dO stages, in the 128-byte-swizzled layout of the
      // tensor map's 64 x 64 boxes, and written with TMA tensor stores (one
      // thread per key row writing its own row would scatter every store
      // instruction over 32 rows).
      uint8_t* stg = smem + kOffQ + half * kKTile;
      auto slot = [&](uint8_t* base, int col) {  // 16-byte chunk holding columns [col, col + 8) of row r
        const int ch = col >> 3;
        return base + (ch >> 3) * kKSub + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
      };
      auto put8 = [&](int col, const float* v) {
        *reinterpret_cast<uint4*>(slot(stg, col)) =
            make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                       pack_bf16x2(v[6], v[7]));
      };
      if (half == 1) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float y[32];
          tmem_ld_32x32(tmem + lanes + 384 + c * 32, y);
#pragma unroll
          for (int u = 0; u < 4; ++u) put8(c * 32 + u * 8, y + 8 * u);
        }
      } else {
        // dK = scale * acc; with the RoPE fold, d/dx of y = rms(rope(x)):
        // dr = r (g - y <g, y> / D), then the transposed rotation of the
        // pairs (i, i + 64). y (the stored normalized k) is this CTA's K tile,
        // already in shared memory. Columns are processed 32 + 32 at a time.
        const long row = long(b) * a.T + key;
        auto get8 = [&](int col, float (&v)[8]) {
          const uint4 w = *reinterpret_cast<const uint4*>(slot(sK, col));
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16x2(ws[k]);
            v[2 * k] = f.x;
            v[2 * k + 1] = f.y;
          }
        };
        float dot = 0.f, rr = 0.f;
        if (a.rope_rstd) {
          rr = a.rope_rstd[row * 2 * a.H + a.H + h];
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            float x[32];
            tmem_ld_32x32(tmem + lanes + 256 + c * 32, x);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              float y[8];
              get8(c * 32 + u * 8, y);
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
              get8(c * 32 + u * 8, y1);
              get8(64 + c * 32 + u * 8, y2);
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
                const float d1 = rr * (g1 - y1[k] * dot), d2 = rr * (g2 - y2[k] * dot);
                g1 = d1 * cs[k] - d2 * sn[k];  // dx1 = dy1 cos - dy2 sin
                g2 = d1 * sn[k] + d2 * cs[k];  // dx2 = dy1 sin + dy2 cos
              }
              x1[i] = g1;
              x2[i] = g2;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            put8(c * 32 + u * 8, x1 + 8 * u);
            put8(64 + c * 32 + u * 8, x2 + 8 * u);
          }
        }
      }
      fence_proxy_async();  // the staged tiles are read by the TMA (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(epi_full);
      if (warp == 2 && lane == 0 && mbar_wait(epi_full, 0, kErrTimeoutEpilogue, a.err)) {
        for (int t = 0; t < 2; ++t)  // t = 0: dK, 1: dV
          for (int sub = 0; sub < 2; ++sub)
            for (int rh = 0; rh < 2; ++rh)
              tma_store_3d(&tmd, smem + kOffQ + t * kKTile + sub * kKSub + rh * kQSub, (1 + t) * a.C + h * HD + 64 * sub,
                           kb * BK + 64 * rh, b);
        bulk_commit();
        bulk_wait<0>();  // shared memory must stay valid until the stores are done
      }
    }
  } else {
    // dQ drain warps: thread = head-dim lane (TMEM lane) of dQ^T, 32 query
    // columns per chunk. Each warp stages 32 queries x 32 head dims of
    // dQ * scale (fp32, row-major 128-byte rows: lane t writes word t of every
    // row, conflict-free) and adds them to the fp32 accumulator with one TMA
    // reduce-add; two staging buffers per warp let the next chunk fill while
    // the previous one drains.
    const int quarter = warp & 3;
    const uint32_t lanes = uint32_t(quarter * 32) << 16;
    float* stage = reinterpret_cast<float*>(smem + kOffStage + (warp - 10) * 2 * kStage);
    int chunks = 0;
    for (int n = 0; n < nblk; ++n) {
      const int j = j0 + n, u = n & 1;
      if (!mbar_wait(&dq_full[u], (n >> 1) & 1, kErrTimeoutEpilogue, a.err)) break;
      if (warp == 10 && lane == 0) fb_stamp<DBG>(a, n, 5);
      tc_fence_after();
      uint32_t xr[2][32];
      tmem_ld_32x32_issue(tmem + lanes + 128 + 64 * u, xr[0]);
      tmem_ld_32x32_issue(tmem + lanes + 128 + 64 * u + 32, xr[1]);
      tmem_ld_wait(xr[0]);
      tmem_ld_wait(xr[1]);
      // The dQ^T columns are free for the scores of block n + 2.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[u]);
      if (warp == 10 && lane == 0) fb_stamp<DBG>(a, n, 6);
      if (DBG && (a.dbg & 1)) continue;
      if (DBG && (a.dbg & 8192)) {  // measurement: coalesced red.global.add from registers, no staging
        float* dst = a.dq_acc + (long(b) * a.T + j * BQ) * a.C + h * HD + quarter * 32 + lane;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) atomicAdd(dst + long(32 * c + i) * a.C, __uint_as_float(xr[c][i]) * a.scale);
        continue;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c, ++chunks) {
        float* buf = stage + (chunks & 1) * (kStage / 4);
        if (lane == 0 && chunks >= 2) bulk_wait_read<1>();  // this buffer's previous reduce has read it
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 32; ++i) buf[i * 32 + lane] = __uint_as_float(xr[c][i]) * a.scale;
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          if (NK_IN_BOUNDS(j * BQ + 32 * c < a.T && h * HD + quarter * 32 < a.C, a.err))
          asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];"
                       ::"l"(&tmq), "r"(smem_u32(buf)), "r"(h * HD + quarter * 32), "r"(b * a.T + j * BQ + 32 * c)
                       : "memory");
          bulk_commit();
        }
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
// through the RoPE + QK-norm backward. A warp handles kDqItems (token, head)
// items, issuing all their loads before any arithmetic so several rows'
// memory latencies overlap; in an item lane l owns elements [4l, 4l+4), its
// rotation partners live in lane l ^ 16.
constexpr int kDqItems = 4;
__global__ void dq_finish_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dqkv, long rows, int T,
                                 int H, int C, const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ rstd,
                                 const float* __restrict__ cos_t, const float* __restrict__ sin_t) {
  const long item0 = (long(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32) * kDqItems;
  const int lane = threadIdx.x & 31;
  const long items = rows * H;
  float4 g4[kDqItems];
  uint2 yw[kDqItems];
#pragma unroll
  for (int k = 0; k < kDqItems; ++k) {
    const long item = item0 + k;
    if (item < items) {
      const long row = item / H;
      const int h = int(item % H);
      g4[k] = *reinterpret_cast<const float4*>(acc + row * C + h * 128 + lane * 4);
      if (rstd) yw[k] = *reinterpret_cast<const uint2*>(qkv + row * 3 * C + h * 128 + lane * 4);
    }
  }
#pragma unroll
  for (int k = 0; k < kDqItems; ++k) {
    const long item = item0 + k;
    if (item >= items) break;  // uniform across the warp
    const long row = item / H;
    const int h = int(item % H);
    float g[4] = {g4[k].x, g4[k].y, g4[k].z, g4[k].w};
    if (rstd) {
      const float2 y0 = unpack_bf16x2(yw[k].x), y1 = unpack_bf16x2(yw[k].y);
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
      const float4 cs4 = *reinterpret_cast<const float4*>(cos_t + pos * 64 + (lane & 15) * 4);
      const float4 sn4 = *reinterpret_cast<const float4*>(sin_t + pos * 64 + (lane & 15) * 4);
      const float cs[4] = {cs4.x, cs4.y, cs4.z, cs4.w}, sn[4] = {sn4.x, sn4.y, sn4.z, sn4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float partner = __shfl_xor_sync(0xffffffffu, dr[j], 16);
        g[j] = first ? dr[j] * cs[j] - partner * sn[j] : partner * sn[j] + dr[j] * cs[j];
      }
    }
    *reinterpret_cast<uint2*>(dqkv + row * 3 * C + h * 128 + lane * 4) =
        make_uint2(pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]));
  }
}

// The timeline written under NANOGPT_FB_DEBUG bit 9 (see g_fb_trace).
torch::Tensor flash_bwd_trace() {
  auto out = torch::zeros({64 * 16}, torch::dtype(torch::kInt64));
  TORCH_CHECK(cudaMemcpyFromSymbol(out.data_ptr(), g_fb_trace, sizeof(long long) * 64 * 16) == cudaSuccess,
              "flash_bwd_trace: copy failed");
  return out;
}

bool flash_bwd_tc_supported(int64_t T, int64_t HD) { return HD == 128 && T % 128 == 0; }

// 3-D map over a (B*T, width) bf16 activation: inner `width` columns, then the
// T rows of one sequence, then B sequences (rows past a sequence read as zeros);
// the box is 64 columns x 64 rows.
static CUtensorMap seq_map_3d(void* base, int64_t B, int64_t T, int64_t width) {
  CUtensorMap m;
  cuuint64_t dims[3] = {cuuint64_t(width), cuuint64_t(T), cuuint64_t(B)};
  cuuint64_t strides[2] = {cuuint64_t(width * 2), cuuint64_t(T * width * 2)};
  cuuint32_t box[3] = {64, uint32_t(fb::BQ), 1};
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
// The backward's preparation in one memory pass: D = rowsum(dO o O) per
// (token, head) and the zeroed fp32 dQ accumulator. Half a warp per (token,
// head): each lane reads 8 bf16 of O and of dO (16-byte loads), the 16 lanes
// reduce with shuffles, and each lane clears 8 floats of the head's dQ row.
__global__ void __launch_bounds__(256) flash_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, long ld_o,
                                                             const __nv_bfloat16* __restrict__ dout, long ld_do,
                                                             float* __restrict__ dsum, float* __restrict__ dq_acc,
                                                             long items, int T, int H, int C) {
  const long item = (long(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
  const int sub = threadIdx.x & 15;
  if (item >= items) return;  // items is even per warp half; whole half-warps leave together
  const long tok = item / H;
  const int h = int(item % H);
  const int col = h * 128 + sub * 8;
  const uint4 x = *reinterpret_cast<const uint4*>(o + tok * ld_o + col);
  const uint4 y = *reinterpret_cast<const uint4*>(dout + tok * ld_do + col);
  const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 a = unpack_bf16x2(xs[k]), b = unpack_bf16x2(ys[k]);
    s += a.x * b.x + a.y * b.y;
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  float4* q = reinterpret_cast<float4*>(dq_acc + tok * C + col);
  q[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  q[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (sub == 0) {
    const long b = tok / T, t = tok % T;
    dsum[(b * H + h) * T + t] = s;
  }
}

void flash_bwd_prep(torch::Tensor out, torch::Tensor dout, torch::Tensor dsum, torch::Tensor dq_acc, int64_t B,
                    int64_t T, int64_t H) {
  const int64_t C = out.size(1);
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() && dq_acc.numel() == B * T * C,
              "flash_bwd_prep: dq_acc");
  TORCH_CHECK(C == H * 128 && out.scalar_type() == at::kBFloat16 && dout.scalar_type() == at::kBFloat16 &&
                  out.stride(1) == 1 && dout.stride(1) == 1 && out.stride(0) % 8 == 0 && dout.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(dout.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(dq_acc.data_ptr()) % 16 == 0,
              "flash_bwd_prep: head_dim 128, 16-byte aligned rows");
  TORCH_CHECK(dsum.scalar_type() == at::kFloat && dsum.numel() == B * H * T, "flash_bwd_prep: dsum");
  const at::cuda::CUDAGuard guard(out.device());
  const long items = B * T * H;
  flash_bwd_prep_kernel<<<unsigned((items * 16 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), out.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0), dsum.data_ptr<float>(),
      dq_acc.data_ptr<float>(), items, int(T), int(H), int(C));
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "flash_bwd_prep launch failed");
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
  if (!prepared) flash_bwd_prep(out, dout, dsum, dq_acc, B, T, H);
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
                                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
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
  static const int bwd_st_defer = [] {
    const char* e = std::getenv("NANOGPT_BWD_ST_DEFER");
    return e ? std::atoi(e) : 1;
  }();
  a.st_defer = bwd_st_defer;
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
    TORCH_CHECK(cudaFuncSetAttribute(flash_bwd_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmem) == cudaSuccess &&
                    cudaFuncSetAttribute(flash_bwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmem) == cudaSuccess,
                "flash_bwd_tc: smem");
    configured = true;
  }
  dim3 grid(unsigned(T / BK), unsigned(B * H));
  CUtensorMap tmd = seq_map_3d(dqkv.data_ptr(), B, T, 3 * C);
  if (a.dbg) flash_bwd_tc_kernel<true><<<grid, kThreads, kSmem, stream>>>(tm, tmo, tmq, tmd, a);
  else flash_bwd_tc_kernel<false><<<grid, kThreads, kSmem, stream>>>(tm, tmo, tmq, tmd, a);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "flash_bwd_tc launch failed");
  const long items = B * T * H;
  dq_finish_kernel<<<unsigned((items + 8 * kDqItems - 1) / (8 * kDqItems)), 256, 0, stream>>>(a.dq_acc, a.dqkv, B * T, int(T), int(H), int(C),
                                                                a.qkv, a.rope_rstd, a.rope_cos, a.rope_sin);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "dq_finish launch failed");
}

}  // namespace nk
