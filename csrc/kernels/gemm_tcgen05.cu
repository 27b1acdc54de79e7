// Persistent warp-specialized bf16 GEMM for sm_100a on the 5th-generation
// tensor cores:  C[M,N] (op)= alpha * sum_k A[m,k] * B[n,k].
//
//   warp 0      TMA producer: 128B-swizzled A/B tiles into a STAGES-deep ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: tcgen05.ld from TMEM, fused elementwise op, staged in
//               shared memory and written with TMA tensor stores (two warps per
//               TMEM lane quarter, each owning half the columns)
//
// The fp32 accumulator of a 128 x BN tile lives in tensor memory; two
// accumulator buffers let the epilogue of tile i overlap the MMAs of tile i+1.
// Operands may be K-major or MN-major, which covers the forward pass
// (X W^T), the data gradient (dY W) and the weight gradient (dY^T X) without
// any transposed copies. Split-K (with fp32 vector atomics in the epilogue)
// keeps all 148 SMs busy on the skinny weight-gradient GEMMs.
//
// Replaces the reference's cuBLAS matmuls at rs-nanogpt src/model/linear.rs:46-49
// (Q/K/V/c_proj/c_fc/mlp.c_proj/lm_head) and folds in the ReLU^2 of
// src/model/mlp.rs:32-33 and the residual adds of src/model/block.rs:55-58.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "status.h"
#include <cstdlib>

#include "launch.h"
#include "tma_host.h"

namespace nk {

enum GemmMode : int {
  kStoreBf16 = 0,   // C = alpha*acc
  kRelu2 = 1,       // C = relu(alpha*acc)^2, AUX_OUT = alpha*acc (AUX_OUT optional)
  kDRelu2 = 2,      // C = alpha*acc * 2*relu(AUX)
  kResidual = 3,    // C = alpha*acc + AUX (AUX may alias C)
  kAtomicF32 = 4,   // C(fp32) += alpha*acc   (split-K capable)
  kRopeNorm = 5,    // QKV projection: q and k heads get RoPE + RMSNorm over head_dim, v stored plain
  kAtomicF32T = 6,  // C^T(fp32) += alpha*acc: C is [N, M]; a warp's 32 rows hit 32 adjacent floats
  kDRelu2Act = 7,   // C = alpha*acc * 2*sqrt(AUX), AUX = relu(h)^2 (the ReLU^2 output)
  kLogitsStats = 8, // C = alpha*acc (bf16 logits) + per (row, 128-column group) softmax partials
};

struct GemmArgs {
  int M, N, K;
  int num_m, num_n, splits, kb_per_split, kb_total;
  int a_mn_major, b_mn_major;
  int mode;
  float alpha;
  void* C;
  long ldc;
  const __nv_bfloat16* aux;
  long ld_aux;
  __nv_bfloat16* aux_out;
  long ld_aux_out;
  int* err;
  // kRopeNorm: half-split RoPE at position (row % rope_T), then RMSNorm over
  // each 128-wide head, on columns [0, 2 * rope_C); 1/denominator per
  // (row, part, head) goes to rope_rstd[row * 2H + part * H + head].
  const float* rope_cos;
  const float* rope_sin;
  float* rope_rstd;
  int rope_T, rope_H, rope_C;
  long rope_ld;  // row stride of the transposed (64, >= T) cos/sin tables
  float rope_eps;
  // A (K-major) depends on no earlier kernel (a weight): under programmatic
  // dependent launch its first tiles are fetched before griddepcontrol.wait.
  int a_independent;
  int rotate;  // single-output epilogues rotate through all staging buffers
  // kLogitsStats: (max, sum of exp(v - max)) over the bf16-rounded logits of
  // row r, columns [128 g, 128 g + 128), at stats[r * stats_ld + g].
  float2* stats;
  int stats_ld;
  int trace;  // NANOGPT_GEMM_TRACE: account the MMA warp's waits in g_gemm_trace
};

// Measurement (NANOGPT_GEMM_TRACE=1): per CTA, the MMA warp's cycles waiting
// for a free accumulator (epilogue behind), waiting for operands (loads
// behind), its total cycles, and its tiles. Read with gemm_trace().
__device__ long long g_gemm_trace[1024 * 4];

constexpr int BM = 128, BK = 64, kGroupM = 16;
constexpr int kEpiWarps = 8, kThreads = 64 + 32 * kEpiWarps;

template <int BN, bool PAIR>
struct Smem {
  static constexpr int kBRows = PAIR ? BN / 2 : BN;  // B rows this CTA holds (a pair splits N)
  // Pairs move 2/3 of the bytes per FLOP, so they trade a pipeline stage for
  // four epilogue staging buffers per warp (stores of one chunk overlap the
  // next chunk; the next residual tile is prefetched).
  static constexpr int kStages = PAIR ? 5 : (BN == 128 ? 6 : 4);
  static constexpr int kEpiBufs = PAIR ? 4 : 2;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = kBRows * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTotal = kStages * kStageBytes + kEpiWarps * kEpiBufs * 2048 /*epilogue staging*/ +
                                1024 /*align*/ + 512 /*barriers*/;
};

// Work unit -> (tile row m, tile col n, k-block range). Tiles are rastered in
// groups of kGroupM row-blocks so concurrently running CTAs share B tiles in L2.
__device__ __forceinline__ void unit_coords(const GemmArgs& a, int u, int& m, int& n, int& kb0, int& kb1) {
  const int tiles = a.num_m * a.num_n;
  const int tile = u % tiles, split = u / tiles;
  const int per_group = kGroupM * a.num_n;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gsz = min(a.num_m - first_m, kGroupM);
  const int r = tile % per_group;
  m = first_m + r % gsz;
  n = r / gsz;
  kb0 = split * a.kb_per_split;
  kb1 = min(a.kb_total, kb0 + a.kb_per_split);
}

// Epilogue staging: each epilogue warp owns two 2 KB shared-memory buffers
// holding a 32-row x 32-column bf16 chunk in the TMA 64-byte swizzle layout
// (16-byte chunk j of row r sits at chunk j ^ ((r >> 1) & 3)). Outputs leave
// through TMA tensor stores and the residual / pre-activation input arrives
// through TMA tensor loads, so no thread issues row-scattered global accesses.
constexpr int kStageBufBytes = 2048;

__device__ __forceinline__ uint32_t stg_off(int r, int j) { return uint32_t(r * 64 + ((j ^ ((r >> 1) & 3)) << 4)); }

// Hardware square root (sqrt.approx, ~1 ulp): far below the bf16 rounding of
// the value it scales, and a single instruction where the IEEE-rounded sqrtf
// path costs the epilogue half its throughput.
__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void stage_row_store(uint8_t* buf, int r, const float (&x)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(buf + stg_off(r, j)) =
        make_uint4(pack_bf16x2(x[8 * j], x[8 * j + 1]), pack_bf16x2(x[8 * j + 2], x[8 * j + 3]),
                   pack_bf16x2(x[8 * j + 4], x[8 * j + 5]), pack_bf16x2(x[8 * j + 6], x[8 * j + 7]));
}

__device__ __forceinline__ void stage_row_load(const uint8_t* buf, int r, float (&y)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w = *reinterpret_cast<const uint4*>(buf + stg_off(r, j));
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16x2(ws[k]);
      y[8 * j + 2 * k] = f.x;
      y[8 * j + 2 * k + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void atomic_chunk(const GemmArgs& a, int row, int col0, const float (&v)[32]) {
  if (row >= a.M) return;
  float* c = reinterpret_cast<float*>(a.C) + long(row) * a.ldc + col0;
  if (col0 + 32 <= a.N) {
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      atomicAdd(reinterpret_cast<float4*>(c + i),
                make_float4(a.alpha * v[i], a.alpha * v[i + 1], a.alpha * v[i + 2], a.alpha * v[i + 3]));
  } else {
    for (int i = 0; i < 32 && col0 + i < a.N; ++i) atomicAdd(c + i, a.alpha * v[i]);
  }
}

// Transposed accumulation: element (row, col) goes to C[col * ldc + row]. The
// 32 lanes of a warp hold 32 consecutive rows, so each red.add covers one
// contiguous 128-byte line.
__device__ __forceinline__ void atomic_chunk_t(const GemmArgs& a, int row, int col0, const float (&v)[32]) {
  if (row >= a.M) return;
  float* c = reinterpret_cast<float*>(a.C) + row;
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (col0 + i < a.N) atomicAdd(c + long(col0 + i) * a.ldc, a.alpha * v[i]);
}

// PAIR: a cluster of two CTAs computes a 256 x BN tile with cta_group::2
// MMAs. Each CTA loads its own 128 rows of A and BN/2 rows of B (no
// multicast); the leader (rank 0) issues the MMAs, which read both CTAs'
// shared memory and accumulate each CTA's 128 rows in its own tensor memory.
// Both CTAs' TMA bytes are counted on the leader's full barrier; the leader's
// MMA completion is committed to both CTAs' empty / accumulator-full
// barriers; both CTAs' epilogue warps arrive on the leader's accumulator-empty
// barrier. Per 256 x BN x 64 step the pair moves 64 KB from L2 instead of the
// 96 KB two independent 128 x BN tiles would.
template <int BN, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX,
                     const GemmArgs args) {
  using S = Smem<BN, PAIR>;
  constexpr int kTileM = PAIR ? 2 * BM : BM;
  constexpr int STAGES = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * S::kStageBytes;  // kEpiWarps x kEpiBufs x 2 KB, 1024-aligned
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(staging + kEpiWarps * S::kEpiBufs * kStageBufBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* aux_bar = acc_empty + 2;  // two per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bar + 2 * kEpiWarps);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int units = args.num_m * args.num_n * args.splits;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const int cta_id = PAIR ? int(blockIdx.x) / 2 : int(blockIdx.x);
  const int n_ctas = PAIR ? int(gridDim.x) / 2 : int(gridDim.x);
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    for (int w = 0; w < 2 * kEpiWarps; ++w) mbar_init(&aux_bar[w], 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if (PAIR) tmem_alloc_pair(tmem_slot, 2 * BN);
    else tmem_alloc(tmem_slot, 2 * BN);
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer's barriers exist before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // Weight tiles of the first stages go out before the dependency wait.
      int pre = 0;
      if (!PAIR && args.a_independent && !args.a_mn_major && int(blockIdx.x) < units) {
        int m, n, kb0, kb1;
        unit_coords(args, blockIdx.x, m, n, kb0, kb1);
        for (int kb = kb0; kb < kb1 && pre < STAGES; ++kb, ++pre) {
          mbar_arrive_expect_tx(&full_bar[pre], S::kStageBytes);
          if (NK_IN_BOUNDS(kb * BK < args.K && m * BM < args.M + 2 * BM, args.err))
            tma_load_2d(smem + pre * S::kStageBytes, &tmA, &full_bar[pre], kb * BK, m * BM);
        }
      }
      pdl_wait();
      // (c0, c1) of a bf16 map whose extents are (n0, n1): the inner coordinate
      // must be 16-byte aligned. Boxes of a ragged last tile may start past the
      // extent (TMA fills zeros); the debug build checks that a box starts no
      // further out than one tile.
      auto load = [&](void* dst, const CUtensorMap* map, int stage_, int c0, int c1, int n0, int n1) {
        if (!NK_IN_BOUNDS(c0 % 8 == 0 && c0 >= 0 && c1 >= 0 && c0 < n0 + 2 * BM && c1 < n1 + 2 * BM, args.err)) return;
        if (PAIR) tma_load_2d_pair(dst, map, map_to_cta(&full_bar[stage_], 0), c0, c1);
        else tma_load_2d(dst, map, &full_bar[stage_], c0, c1);
      };
      int issued = 0;
      for (int u = cta_id; u < units && ok; u += n_ctas) {
        int m, n, kb0, kb1;
        unit_coords(args, u, m, n, kb0, kb1);
        const int arow = m * kTileM + int(rank) * BM;        // this CTA's 128 rows of A
        const int brow = n * BN + int(rank) * S::kBRows;     // and its rows of B
        for (int kb = kb0; kb < kb1; ++kb, ++issued) {
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          if (issued >= pre) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, kErrTimeoutProducer, args.err)) { ok = false; break; }
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], (PAIR ? 2 : 1) * S::kStageBytes);
            if (!args.a_mn_major) {
              load(sa, &tmA, stage, kb * BK, arow, args.K, args.M);
            } else {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) load(sa + j * 8192, &tmA, stage, arow + 64 * j, kb * BK, args.M, args.K);
            }
          }
          if (!args.b_mn_major) {
            load(sb, &tmB, stage, kb * BK, brow, args.K, args.N);
          } else {
#pragma unroll
            for (int j = 0; j < S::kBRows / 64; ++j) load(sb + j * 8192, &tmB, stage, brow + 64 * j, kb * BK, args.N, args.K);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = idesc_bf16(kTileM, BN, args.a_mn_major, args.b_mn_major);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      auto commit = [&](uint64_t* bar) {
        if (PAIR) {
          umma_commit_pair(map_to_cta(bar, 0));
          umma_commit_pair(map_to_cta(bar, 1));
        } else {
          umma_commit(bar);
        }
      };
      // Operand descriptors of stage 0; a stage and a 16-deep K step are byte offsets on them.
      const uint32_t sa0 = smem_u32(smem), sb0 = sa0 + S::kABytes;
      const uint64_t a_desc0 = args.a_mn_major ? sw128_desc(sa0, 8192, 1024) : sw128_desc(sa0, 16, 1024);
      const uint64_t b_desc0 = args.b_mn_major ? sw128_desc(sb0, 8192, 1024) : sw128_desc(sb0, 16, 1024);
      const uint32_t a_kstep = args.a_mn_major ? 2048 : 32, b_kstep = args.b_mn_major ? 2048 : 32;
      long long w_acc = 0, w_ld = 0;
      const long long t_begin = clock64();
      for (int u = cta_id; u < units && ok; u += n_ctas, ++local) {
        int m, n, kb0, kb1;
        unit_coords(args, u, m, n, kb0, kb1);
        const int b = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        long long t0 = args.trace ? clock64() : 0;
        if (!mbar_wait(&acc_empty[b], acc_phase ^ 1, kErrTimeoutMma, args.err)) break;
        if (args.trace) w_acc += clock64() - t0;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (args.trace) t0 = clock64();
          if (!mbar_wait(&full_bar[stage], phase, kErrTimeoutMma, args.err)) { ok = false; break; }
          if (args.trace) w_ld += clock64() - t0;
          tc_fence_after();
          const uint32_t so = stage * S::kStageBytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = desc_advance(a_desc0, so + k * a_kstep);
            const uint64_t bd = desc_advance(b_desc0, so + k * b_kstep);
            if (PAIR) umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else umma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        commit(&acc_full[b]);
      }
      if (args.trace && blockIdx.x < 1024) {
        long long* t = g_gemm_trace + blockIdx.x * 4;
        t[0] = w_acc; t[1] = w_ld; t[2] = clock64() - t_begin; t[3] = local;
      }
    }
  } else {
    pdl_wait();                             // the epilogue reads and writes global memory
    const int ew = warp - 2;                // epilogue warp index
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = ew / 4;                // which half of the tile's columns
    constexpr int NB = S::kEpiBufs;
    uint8_t* wbuf = staging + ew * NB * kStageBufBytes;
    // Chunk ck of this warp stages its output in bufO(ck) and its second
    // output / residual input in bufX(ck); with four buffers consecutive
    // chunks alternate between two buffer pairs.
    auto bufO = [&](int ck) { return wbuf + ((2 * ck) % NB) * kStageBufBytes; };
    auto bufX = [&](int ck) { return wbuf + ((2 * ck + 1) % NB) * kStageBufBytes; };
    const bool atomic = args.mode == kAtomicF32 || args.mode == kAtomicF32T;
    const bool need_aux = args.mode == kResidual || args.mode == kDRelu2 || args.mode == kDRelu2Act;
    const bool keep_h = args.mode == kRelu2 && args.aux_out != nullptr;
    // One output and no staged input: every buffer of the warp can hold an
    // output chunk, so NB - 1 stores may still be reading while the next is written.
    const bool single_out = args.rotate && !need_aux && !keep_h;
    auto bufS = [&](int ck) { return single_out ? wbuf + (ck % NB) * kStageBufBytes : bufO(ck); };
    uint32_t aux_ph[2] = {0u, 0u};
    int ck = 0;
    auto issue_aux = [&](int ckk, int col, int row) {  // all lanes call; lane 0 issues
      fence_proxy_async();  // earlier generic reads of the buffer precede the TMA write
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&aux_bar[2 * ew + (ckk & 1)], kStageBufBytes);
        if (NK_IN_BOUNDS(col % 8 == 0 && col >= 0 && col < args.N && row >= 0 && row < args.M + kTileM, args.err))
          tma_load_2d(bufX(ckk), &tmX, &aux_bar[2 * ew + (ckk & 1)], col, row);
      }
    };
    bool ok = true;
    int local = 0;
    auto release_acc = [&](int b) {
      if (PAIR) mbar_arrive_cluster(map_to_cta(&acc_empty[b], 0));
      else mbar_arrive(&acc_empty[b]);
    };
    for (int u = cta_id; u < units && ok; u += n_ctas, ++local) {
      int m, n, kb0, kb1;
      unit_coords(args, u, m, n, kb0, kb1);
      const int b = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[b], acc_phase, kErrTimeoutEpilogue, args.err)) break;
      tc_fence_after();
      const int row0 = m * kTileM + int(rank) * BM + q * 32;
      if (args.mode == kRopeNorm && n * BN + half * 128 < 2 * args.rope_C) {
        // One full q/k head per thread row: 4 TMEM chunks -> RoPE -> RMSNorm -> 4 TMA stores.
        const int colb = n * BN + half * 128;
        const int part = colb / args.rope_C, head = (colb % args.rope_C) / 128;
        const int row = row0 + lane;
        const int pos = (row < args.M ? row : 0) % args.rope_T;
        float hv[128];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          float v[32];
          tmem_ld_32x32(tmem_base + (uint32_t(q * 32) << 16) + b * BN + (half * 4 + c4) * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) hv[c4 * 32 + i] = __bfloat162float(__float2bfloat16(args.alpha * v[i]));
        }
        // Transposed tables: lane l reads position row0 + l, so each load of
        // the warp covers consecutive addresses.
        const float* cr = args.rope_cos + pos;
        const float* sr = args.rope_sin + pos;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float cs = __ldg(cr + i * args.rope_ld), sn = __ldg(sr + i * args.rope_ld);
          const float x1 = hv[i], x2 = hv[i + 64];
          hv[i] = x1 * cs + x2 * sn;       // y1 = x1 cos + x2 sin
          hv[i + 64] = x2 * cs - x1 * sn;  // y2 = x2 cos - x1 sin
          ss += hv[i] * hv[i] + hv[i + 64] * hv[i + 64];
        }
        const float denom = __bfloat162float(__float2bfloat16(sqrtf(ss / 128.f + args.rope_eps)));
        const float inv = 1.f / denom;
        if (row < args.M) args.rope_rstd[long(row) * 2 * args.rope_H + part * args.rope_H + head] = inv;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          float x[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = hv[c4 * 32 + i] * inv;
          uint8_t* sb = bufS(ck);  // same rotation as the plain chunks of this launch
          if (lane == 0) {
            if (single_out) bulk_wait_read<NB - 1>();
            else bulk_wait_read<0>();
          }
          __syncwarp();
          stage_row_store(sb, lane, x);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            // A pair's second CTA can hold only rows past M in the last tile row: nothing to store.
            if (row0 < args.M && NK_IN_BOUNDS(row0 >= 0 && colb + c4 * 32 < args.N, args.err))
              tma_store_2d(&tmC, sb, colb + c4 * 32, row0);
            bulk_commit();
          }
          ++ck;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(b);
        continue;
      }
      const int c_begin = half * (BN / 64), c_end = (half + 1) * (BN / 64);
      if (need_aux && n * BN + c_begin * 32 < args.N) issue_aux(ck, n * BN + c_begin * 32, row0);
      float st_m = -INFINITY, st_s = 0.f;  // kLogitsStats running partials (log2 domain)
#pragma unroll 1
      for (int c = c_begin; c < c_end; ++c) {
        const int col0 = n * BN + c * 32;
        if (col0 >= args.N) break;  // uniform across the warp
        if (need_aux && NB >= 4 && c + 1 < c_end && col0 + 32 < args.N) issue_aux(ck + 1, col0 + 32, row0);
        float v[32];
        tmem_ld_32x32(tmem_base + (uint32_t(q * 32) << 16) + b * BN + c * 32, v);
        if (atomic) {
          if (args.mode == kAtomicF32T) atomic_chunk_t(args, row0 + lane, col0, v);
          else atomic_chunk(args, row0 + lane, col0, v);
          continue;
        }
        float x[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = args.alpha * v[i];
        if (need_aux) {
          if (!mbar_wait(&aux_bar[2 * ew + (ck & 1)], aux_ph[ck & 1], kErrTimeoutEpilogue, args.err)) {
            ok = false;
            break;
          }
          aux_ph[ck & 1] ^= 1;
          float y[32];
          stage_row_load(bufX(ck), lane, y);
          if (args.mode == kDRelu2) {
#pragma unroll
            for (int i = 0; i < 32; ++i)  // d/dh relu(h)^2 = 2 relu(h), on the bf16-rounded upstream grad
              x[i] = __bfloat162float(__float2bfloat16(x[i])) * 2.f * fmaxf(y[i], 0.f);
          } else if (args.mode == kDRelu2Act) {
#pragma unroll
            for (int i = 0; i < 32; ++i)  // relu(h) = sqrt(relu(h)^2): the pre-activation need not be kept
              x[i] = __bfloat162float(__float2bfloat16(x[i])) * 2.f * sqrt_approx(fmaxf(y[i], 0.f));
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) x[i] = __bfloat162float(__float2bfloat16(x[i])) + y[i];
          }
          // NB == 2: the next chunk's residual load reuses this buffer.
          if (NB < 4 && c + 1 < c_end && col0 + 32 < args.N) issue_aux(ck + 1, col0 + 32, row0);
        }
        // The stores that last read this chunk's buffers (NB / 2 chunks ago) are done.
        if (lane == 0) {
          if (single_out) bulk_wait_read<NB - 1>();
          else bulk_wait_read<NB / 2 - 1>();
        }
        __syncwarp();
        if (args.mode == kLogitsStats) {
          // Softmax partials of the values as stored (bf16), in log2 units:
          // m = max(v) * log2e, s = sum 2^(v * log2e - m).
          constexpr float kLog2e = 1.4426950408889634f;
          float cm = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            x[i] = __bfloat162float(__float2bfloat16(x[i]));
            if (col0 + i < args.N) cm = fmaxf(cm, x[i] * kLog2e);
          }
          if (cm > st_m) {
            st_s *= ex2_approx(st_m - cm);  // st_m = -inf at first: st_s is 0 and stays 0
            st_m = cm;
          }
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col0 + i < args.N) st_s += ex2_approx(fmaf(x[i], kLog2e, -st_m));
        }
        if (args.mode == kRelu2) {
          if (keep_h) stage_row_store(bufX(ck), lane, x);  // pre-activation h
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            // Square the bf16-rounded pre-activation, as relu(h)^2 on a bf16 h would.
            const float hr = fmaxf(__bfloat162float(__float2bfloat16(x[i])), 0.f);
            x[i] = hr * hr;
          }
        }
        stage_row_store(bufS(ck), lane, x);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          // (Rows past M inside the last tile are clipped by the TMA store.)
          if (row0 < args.M && NK_IN_BOUNDS(col0 % 8 == 0 && col0 >= 0 && col0 < args.N && row0 >= 0, args.err)) {
            tma_store_2d(&tmC, bufS(ck), col0, row0);
            if (keep_h) tma_store_2d(&tmX, bufX(ck), col0, row0);
          }
          bulk_commit();
        }
        ++ck;
      }
      if (args.mode == kLogitsStats && ok) {
        const int row = row0 + lane, g = (n * BN + half * 128) / 128;
        if (row < args.M && n * BN + half * 128 < args.N) args.stats[long(row) * args.stats_ld + g] = make_float2(st_m, st_s);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) release_acc(b);
    }
    if (lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // no cross-CTA MMA, TMA byte count or arrive is still in flight
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, 2 * BN);
    else tmem_dealloc(tmem_base, 2 * BN);
  }
}

static int num_sms() {
  static int n = [] {
    int dev, v;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

template <int BN, bool PAIR>
static void launch(const GemmArgs& args, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                   const CUtensorMap& tx, cudaStream_t stream) {
  using S = Smem<BN, PAIR>;
  static bool configured = false;
  if (!configured) {
    TORCH_CHECK(cudaFuncSetAttribute(gemm_bf16_kernel<BN, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     S::kTotal) == cudaSuccess,
                "gemm: cannot reserve shared memory");
    configured = true;
  }
  const int units = args.num_m * args.num_n * args.splits;
  if constexpr (!PAIR) {
    const int grid = std::min(units, num_sms());
    TORCH_CHECK(launch_k(gemm_bf16_kernel<BN, false>, dim3(grid), dim3(kThreads), S::kTotal, stream, ta, tb, tc,
                         tx, args) == cudaSuccess,
                "gemm: launch failed");
  } else {
    const int grid = 2 * std::min(units, num_sms() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = S::kTotal;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    TORCH_CHECK(cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<BN, true>, ta, tb, tc, tx, args) == cudaSuccess,
                "gemm: pair launch failed");
  }
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "gemm launch failed");
}

torch::Tensor gemm_trace() {
  auto out = torch::zeros({1024, 4}, torch::dtype(torch::kInt64));
  TORCH_CHECK(cudaMemcpyFromSymbol(out.data_ptr(), g_gemm_trace, sizeof(long long) * 1024 * 4) == cudaSuccess,
              "gemm_trace: copy failed");
  return out;
}

// CTA pairs (cta_group::2) for the large 256-column GEMMs. NANOGPT_GEMM_PAIR:
// unset/1 = where measured faster (below), 0 = never, 2 = for every eligible
// product (measurement switch).
static int pair_mode() {
  static const int mode = [] {
    const char* e = std::getenv("NANOGPT_GEMM_PAIR");
    return e ? std::atoi(e) : 1;
  }();
  return mode;
}

// NANOGPT_GEMM_BALANCE=0 keeps the caller's split count for the split-K
// weight gradients (measurement switch).
static int balance_mode() {
  static const int mode = [] {
    const char* e = std::getenv("NANOGPT_GEMM_BALANCE");
    return e ? std::atoi(e) : 1;
  }();
  return mode;
}

// NANOGPT_GEMM_ROTATE=0 keeps one staging buffer per output chunk (A/B switch).
static int rotate_mode() {
  static const int mode = [] {
    const char* e = std::getenv("NANOGPT_GEMM_ROTATE");
    return e ? std::atoi(e) : 1;
  }();
  return mode;
}

static void check_bf16_2d(const torch::Tensor& t, int64_t rows, int64_t cols, const char* what) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.size(0) == rows && t.size(1) == cols &&
                  t.stride(1) == 1 && (t.stride(0) * 2) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "gemm: bad ", what);
}

// C (op)= alpha * A . B^T with operand layouts:
//   A: a_mn_major ? [K, M] : [M, K]      B: b_mn_major ? [K, N] : [N, K]
void gemm_impl(torch::Tensor A, bool a_mn_major, torch::Tensor B, bool b_mn_major, torch::Tensor C, int64_t mode,
               double alpha, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> aux_out, int64_t splits,
               int64_t block_n, const GemmArgs* rope, bool a_independent = false) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2-D tensors");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm: row-major tensors");
  const int M = int(a_mn_major ? A.size(1) : A.size(0));
  const int K = int(a_mn_major ? A.size(0) : A.size(1));
  const int N = int(b_mn_major ? B.size(1) : B.size(0));
  TORCH_CHECK((b_mn_major ? B.size(0) : B.size(1)) == K, "gemm: K mismatch");
  const bool c_transposed = mode == kAtomicF32T;
  TORCH_CHECK(c_transposed ? (C.size(0) == N && C.size(1) == M) : (C.size(0) == M && C.size(1) == N),
              "gemm: C shape mismatch");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  const bool f32out = mode == kAtomicF32 || mode == kAtomicF32T;
  TORCH_CHECK(C.scalar_type() == (f32out ? at::kFloat : at::kBFloat16), "gemm: C dtype does not fit the mode");
  TORCH_CHECK(splits == 1 || f32out, "gemm: split-K needs the atomic fp32 mode");
  const int elt = f32out ? 4 : 2;
  TORCH_CHECK((C.stride(0) * elt) % 16 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0,
              "gemm: C rows must be 16-byte aligned");

  GemmArgs args{};
  args.M = M; args.N = N; args.K = K;
  args.a_mn_major = a_mn_major; args.b_mn_major = b_mn_major;
  args.mode = int(mode);
  args.alpha = float(alpha);
  args.C = C.data_ptr();
  args.ldc = C.stride(0);
  args.err = error_word();
  args.a_independent = a_independent ? 1 : 0;
  args.rotate = rotate_mode();
  static const int trace = [] {
    const char* e = std::getenv("NANOGPT_GEMM_TRACE");
    return e ? std::atoi(e) : 0;
  }();
  args.trace = trace;
  if (rope && mode == kLogitsStats) {
    args.stats = rope->stats;
    args.stats_ld = rope->stats_ld;
  } else if (rope) {
    args.rope_cos = rope->rope_cos; args.rope_sin = rope->rope_sin; args.rope_rstd = rope->rope_rstd;
    args.rope_T = rope->rope_T; args.rope_ld = rope->rope_ld; args.rope_H = rope->rope_H; args.rope_C = rope->rope_C; args.rope_eps = rope->rope_eps;
  }
  if (mode == kDRelu2 || mode == kDRelu2Act || mode == kResidual) {
    TORCH_CHECK(aux.has_value(), "gemm: mode needs aux");
    check_bf16_2d(*aux, M, N, "aux");
    args.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
    args.ld_aux = aux->stride(0);
  }
  if (mode == kRelu2 && aux_out.has_value()) {
    check_bf16_2d(*aux_out, M, N, "aux_out");
    args.aux_out = reinterpret_cast<__nv_bfloat16*>(aux_out->data_ptr());
    args.ld_aux_out = aux_out->stride(0);
  }
  const int BN = block_n == 128 ? 128 : 256;
  // Pairs measured faster than single-CTA tiles only for the weight-gradient
  // products (both operands MN-major); elsewhere single-CTA tiles win.
  // Measured at the d20 shapes: pairs win for the weight-gradient products
  // (both operands MN-major, +6-20%) and the wide lm_head forward (+6%);
  // single-CTA tiles win or tie elsewhere.
  // Re-measured with MN-major B (the data gradients): pairs +2-8 % on every d20 shape.
  const bool pair_default = b_mn_major || (!a_mn_major && !b_mn_major && N >= 32768);
  const bool pair = BN == 256 && M > BM && mode != kRopeNorm && mode != kAtomicF32T &&
                    (pair_mode() == 2 || (pair_mode() == 1 && pair_default));
  args.num_m = (M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM);
  args.num_n = (N + BN - 1) / BN;
  args.kb_total = (K + BK - 1) / BK;
  int s = int(std::max<int64_t>(1, std::min<int64_t>(splits, args.kb_total)));
  if (mode == kAtomicF32 && s > 1 && balance_mode()) {
    // Split-K weight gradients: among s .. 2s splits take the one whose last
    // round of units leaves the fewest CTAs idle; per-CTA time is modelled as
    // rounds x (k-blocks per unit + 2 for the unit's pipeline fill and flush).
    const long n_ctas = pair ? num_sms() / 2 : num_sms(), tiles = long(args.num_m) * args.num_n;
    long best = -1;
    int best_s = s;
    for (int c = s; c <= 2 * s && c <= args.kb_total; ++c) {
      const long kps = (args.kb_total + c - 1) / c, units = tiles * ((args.kb_total + kps - 1) / kps);
      const long cost = ((units + n_ctas - 1) / n_ctas) * (kps + 2);
      if (best < 0 || cost < best) { best = cost; best_s = c; }
    }
    s = best_s;
  }
  args.kb_per_split = (args.kb_total + s - 1) / s;
  args.splits = (args.kb_total + args.kb_per_split - 1) / args.kb_per_split;

  // Tensor maps: inner dimension first. K-major boxes are 64 (K) x rows;
  // MN-major boxes are 64 (MN) x 64 (K), issued BM/64 or BN/64 times per stage.
  CUtensorMap ta = a_mn_major ? make_tmap_bf16_2d(A.data_ptr(), M, K, A.stride(0), 64, 64)
                              : make_tmap_bf16_2d(A.data_ptr(), K, M, A.stride(0), 64, BM);
  CUtensorMap tb = b_mn_major ? make_tmap_bf16_2d(B.data_ptr(), N, K, B.stride(0), 64, 64)
                              : make_tmap_bf16_2d(B.data_ptr(), K, N, B.stride(0), 64, pair ? BN / 2 : BN);
  // Epilogue maps: 32 x 32 bf16 boxes, 64-byte swizzle (unused in the fp32 atomic mode).
  CUtensorMap tc = ta, tx = ta;
  if (!f32out) {
    tc = make_tmap_bf16_2d_swz(C.data_ptr(), N, M, C.stride(0), 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    if (mode == kResidual || mode == kDRelu2 || mode == kDRelu2Act)
      tx = make_tmap_bf16_2d_swz(aux->data_ptr(), N, M, aux->stride(0), 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    else if (mode == kRelu2 && aux_out.has_value())
      tx = make_tmap_bf16_2d_swz(aux_out->data_ptr(), N, M, aux_out->stride(0), 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  const at::cuda::CUDAGuard guard(A.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (BN == 128) launch<128, false>(args, ta, tb, tc, tx, stream);
  else if (pair) launch<256, true>(args, ta, tb, tc, tx, stream);
  else launch<256, false>(args, ta, tb, tc, tx, stream);
}

void gemm(torch::Tensor A, bool a_mn_major, torch::Tensor B, bool b_mn_major, torch::Tensor C, int64_t mode,
          double alpha, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> aux_out, int64_t splits,
          int64_t block_n) {
  TORCH_CHECK(mode != kRopeNorm, "gemm: use gemm_qkv_rope for the RoPE epilogue");
  TORCH_CHECK(mode >= kStoreBf16 && mode <= kDRelu2Act, "gemm: unknown epilogue mode");
  gemm_impl(A, a_mn_major, B, b_mn_major, C, mode, alpha, aux, aux_out, splits, block_n, nullptr);
}

// logits[M, V] = x[M, K] . w[V, K]^T (bf16) with the softmax partials of each
// row's 128-column groups in stats (M, ceil(V / 128), 2) fp32: the lm_head of
// the fused loss head (the log-sum-exp then needs no pass over the logits).
void gemm_logits_stats(torch::Tensor x, torch::Tensor w, torch::Tensor logits, torch::Tensor stats) {
  const int64_t M = x.size(0), V = w.size(0);
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.dim() == 3 && stats.size(0) >= M &&
                  stats.size(1) == (V + 127) / 128 && stats.size(2) == 2,
              "gemm_logits_stats: stats must be (rows, ceil(V / 128), 2) fp32");
  GemmArgs r{};
  r.stats = reinterpret_cast<float2*>(stats.data_ptr<float>());
  r.stats_ld = int(stats.size(1));
  gemm_impl(x, false, w, false, logits, kLogitsStats, 1.0, c10::nullopt, c10::nullopt, 1, 256, &r);
}

// qkv[M, 3C] = x[M, C] . w[3C, C]^T with RoPE + QK-RMSNorm fused into the
// epilogue for the q and k column blocks (head_dim 128, 3C % 256 == 0).
// cos_t / sin_t are the RoPE tables transposed: (64, >= T), position fastest.
void gemm_qkv_rope(torch::Tensor x, torch::Tensor w, torch::Tensor qkv, torch::Tensor rstd, torch::Tensor cos_t,
                   torch::Tensor sin_t, int64_t T, int64_t H, double eps) {
  const int64_t C = w.size(1);
  TORCH_CHECK(w.size(0) == 3 * C && C == H * 128 && (3 * C) % 256 == 0, "gemm_qkv_rope: shape");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat && cos_t.is_contiguous() &&
                  sin_t.is_contiguous() && cos_t.size(0) == 64 && cos_t.sizes() == sin_t.sizes() &&
                  cos_t.size(1) >= T, "gemm_qkv_rope: transposed rope tables (64, >= T)");
  TORCH_CHECK(rstd.scalar_type() == at::kFloat && rstd.numel() >= x.size(0) * 2 * H, "gemm_qkv_rope: rstd");
  GemmArgs r{};
  r.rope_cos = cos_t.data_ptr<float>();
  r.rope_sin = sin_t.data_ptr<float>();
  r.rope_rstd = rstd.data_ptr<float>();
  r.rope_T = int(T); r.rope_ld = cos_t.size(1); r.rope_H = int(H); r.rope_C = int(C); r.rope_eps = float(eps);
  gemm_impl(x, false, w, false, qkv, kRopeNorm, 1.0, c10::nullopt, c10::nullopt, 1, 256, &r);
}

}  // namespace nk

namespace nk {
// acc[M, N] (fp32) += x[M, K] . w[N, K]^T with the operands swapped (the weight
// rows are the 128-row tile side), split over K, transposed fp32 atomics. The
// weight tiles are independent of earlier kernels (prefetched under PDL).
void gemm_skinny_acc(torch::Tensor w, torch::Tensor x, torch::Tensor acc, int64_t splits) {
  gemm_impl(w, false, x, false, acc, kAtomicF32T, 1.0, c10::nullopt, c10::nullopt, splits, 128, nullptr, true);
}
}  // namespace nk
