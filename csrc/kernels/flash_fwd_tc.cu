// Causal flash-attention forward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), head_dim 128, seq_len a multiple of 256.
//
// One CTA = two 128-row query tiles of one (batch, head); key/value blocks of
// 128. TMEM (512 columns) holds S0, S1 (scores of the two tiles) and O0, O1
// (their output accumulators). Roles:
//   warp 0      TMA loads: Q0, Q1 once, then K_j and V_j per key block
//               (3-D tensor map over the fused QKV buffer; no multicast)
//   warp 1      TMEM allocation + single-thread MMA issue:
//               S_t = Q_t K_j^T, then O_t += P_t V_j
//   warps 2-5   softmax for tile 0, warps 6-9 for tile 1: thread = query row.
//               Reads its S row from TMEM, applies the causal mask on the
//               diagonal block, keeps the running max / sum in registers,
//               writes P (bf16 pairs) back to tensor memory over the S
//               columns it has read (the P V MMA takes its A operand from
//               tensor memory; NANOGPT_FWD_P_TMEM=0 stages P in shared memory
//               instead), and rescales its O row in TMEM only when the row max
//               grew by more than 2^8 since the last rescale (otherwise the
//               stale max is kept, which only scales P and O by the same
//               bounded factor).
// Two tiles per CTA let the tensor core compute one tile's MMAs while the
// other tile's softmax runs.
//
// Output and LSE conventions match flash_attn.cu (LSE in base-2 units of the
// scaled scores), so the backward kernels consume either forward's results.
#include <cstdlib>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "status.h"
#include "tma_host.h"

namespace nk {

namespace fa {
constexpr int HD = 128, BM = 128, BN = 128;
constexpr int kThreads = 320;
constexpr int kTileBytes = BM * HD * 2;      // 32 KB: Q tile, K block, V block or P tile
constexpr int kSubBytes = 128 * 64 * 2;      // 16 KB: one 64-column swizzle sub-tile
constexpr int kSmem = 7 * kTileBytes + 1024 + 256;
constexpr float kRescaleThreshold = 8.0f;    // log2 units
}  // namespace fa

struct FaArgs {
  __nv_bfloat16* out;
  long ld_out;
  float* lse;
  int B, H, T, C;
  float sl2;
  int* err;
  int st_defer;  // P stores to tensor memory waited for once per block (NANOGPT_FWD_ST_DEFER, default 1)
};

// P tile staging: row r, 16-byte chunk c (8 keys) of the 128 keys; sub-tile
// c / 8 covers keys [64 * (c / 8), +64), each row 128 B, 128B-swizzled.
__device__ __forceinline__ uint32_t p_off(int r, int c) {
  return uint32_t((c >> 3) * fa::kSubBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <bool P_TMEM>
__global__ void __launch_bounds__(fa::kThreads, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, const FaArgs a) {
  using namespace fa;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // 2 tiles
  uint8_t* sK = smem + 2 * kTileBytes;      // 2 buffers
  uint8_t* sV = smem + 4 * kTileBytes;
  uint8_t* sP = smem + 5 * kTileBytes;      // 2 tiles (P staged in shared memory)
  // With P in tensor memory the P region holds a second V buffer, so V_{j+1}
  // streams in while P V_j runs (a single buffer put the V load's full
  // latency between P_1 V_j and P_0 V_{j+1} on every key block).
  constexpr int VB = P_TMEM ? 2 : 1;
  auto v_buf = [&](int j) { return (VB == 2 && (j & 1)) ? sP : sV; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [VB]
  uint64_t* v_empty = bars + 7;  // [VB]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;  // [2]
  uint64_t* o_done = bars + 13;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest rows first
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int q0 = qb * 2 * BM;
  const int nblk1 = (q0 + 2 * BM) / BN;       // key blocks of tile 1; tile 0 has one fewer
  const int xq = h * HD, xk = a.C + h * HD, xv = 2 * a.C + h * HD;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VB; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
    }
    fence_barrier_init();
    prefetch_tmap(&tm);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0 @0, S1 @128, O0 @256, O1 @384

  if (warp == 0) {
    // (The debug build skips the loads of an out-of-range tile; the waits on
    // them then run out and the CTA still reaches the final barrier.)
    if (lane == 0 && NK_IN_BOUNDS(q0 + 2 * BM <= a.T && b < a.B && xv + 128 <= 3 * a.C, a.err)) {
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      for (int t = 0; t < 2; ++t)
        for (int s = 0; s < 2; ++s)
          tma_load_3d(sQ + t * kTileBytes + s * kSubBytes, &tm, q_full, xq + 64 * s, q0 + t * BM, b);
      for (int j = 0; j < nblk1; ++j) {
        const int kb = j & 1;
        if (!mbar_wait(&k_empty[kb], ((j >> 1) & 1) ^ 1, kErrTimeoutProducer, a.err)) break;
        mbar_arrive_expect_tx(&k_full[kb], kTileBytes);
        for (int s = 0; s < 2; ++s)
          tma_load_3d(sK + kb * kTileBytes + s * kSubBytes, &tm, &k_full[kb], xk + 64 * s, j * BN, b);
        const int vb = j % VB;
        if (!mbar_wait(&v_empty[vb], ((j / VB) & 1) ^ 1, kErrTimeoutProducer, a.err)) break;
        mbar_arrive_expect_tx(&v_full[vb], kTileBytes);
        for (int s = 0; s < 2; ++s) tma_load_3d(v_buf(j) + s * kSubBytes, &tm, &v_full[vb], xv + 64 * s, j * BN, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Ping-pong: once tile t's softmax of block j is done, issue O_t += P_t V_j
      // and then S_t = Q_t K_{j+1}, so each tile's softmax overlaps the other
      // tile's MMAs. K is double-buffered; V_j is released after PV_1(j).
      const uint32_t id_s = idesc_bf16(BM, BN, false, false);  // Q K^T: both K-major
      const uint32_t id_o = idesc_bf16(BM, HD, false, true);   // P V: V is MN-major (d contiguous)
      const int nblk0 = nblk1 - 1;
      auto issue_s = [&](int t, int j) {
        const uint32_t q = smem_u32(sQ + t * kTileBytes), k = smem_u32(sK + (j & 1) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kSubBytes + (kk & 3) * 32;
          umma_bf16(tmem + t * BN, sw128_desc(q + off, 16, 1024), sw128_desc(k + off, 16, 1024), id_s,
                    kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t p = smem_u32(sP + t * kTileBytes), v = smem_u32(v_buf(j));
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          if constexpr (P_TMEM) {
            // P_t packed as bf16 pairs in TMEM columns [t * BN, t * BN + 64): keys 16 kk.. in 8 columns.
            umma_bf16_ts(tmem + 256 + t * HD, tmem + t * BN + 8 * kk, sw128_desc(v + kk * 2048, kSubBytes, 1024),
                         id_o, (j > 0 || kk > 0) ? 1u : 0u);
          } else {
            const uint32_t poff = (kk >> 2) * kSubBytes + (kk & 3) * 32;
            umma_bf16(tmem + 256 + t * HD, sw128_desc(p + poff, 16, 1024),
                      sw128_desc(v + kk * 2048, kSubBytes, 1024), id_o, (j > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&o_done[t]);
      };
      bool ok = mbar_wait(q_full, 0, kErrTimeoutMma, a.err) && mbar_wait(&k_full[0], 0, kErrTimeoutMma, a.err);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);  // tile 0 has at least one block
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; j < nblk1 && ok; ++j) {
        const bool next = j + 1 < nblk1;  // tile 1 (and tile 0 if j + 1 < nblk0) has block j + 1
        if (!mbar_wait(&v_full[j % VB], (j / VB) & 1, kErrTimeoutMma, a.err)) break;
        if (j < nblk0) {
          if (!mbar_wait(&p_full[0], j & 1, kErrTimeoutMma, a.err)) break;
          tc_fence_after();
          issue_pv(0, j);
        }
        if (next && !mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, kErrTimeoutMma, a.err)) break;
        tc_fence_after();
        if (j + 1 < nblk0) issue_s(0, j + 1);
        if (!mbar_wait(&p_full[1], j & 1, kErrTimeoutMma, a.err)) break;
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(&v_empty[j % VB]);
        if (next) {
          issue_s(1, j + 1);
          umma_commit(&k_empty[(j + 1) & 1]);
        }
      }
    }
  } else {
    // Softmax warpgroups.
    const int t = (warp - 2) / 4;                  // query tile
    const int quarter = warp & 3;                  // TMEM lanes this warp may access
    const int r = quarter * 32 + lane;             // row within the tile
    const int qrow = q0 + t * BM + r;              // absolute query position
    const int nblk = nblk1 - 1 + t;
    const uint32_t t_s = tmem + (uint32_t(quarter * 32) << 16) + t * BN;
    const uint32_t t_o = tmem + (uint32_t(quarter * 32) << 16) + 256 + t * HD;
    uint8_t* P = sP + t * kTileBytes;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk && ok; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, kErrTimeoutEpilogue, a.err)) { ok = false; break; }
      tc_fence_after();
      const bool diag = j == nblk - 1;
      // The whole S row in registers (two 64-column loads): row max, then
      // P = exp2(s * scale*log2e - m) from the same registers. Only the
      // diagonal block needs the causal mask (keys past the query get -inf).
      float sv[BN];
      tmem_ld_32x64(t_s, *reinterpret_cast<float(*)[64]>(sv));
      tmem_ld_32x64(t_s + 64, *reinterpret_cast<float(*)[64]>(sv + 64));
      if (diag) {
        const int lim = qrow - j * BN;  // keys 0..lim of this block are visible
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (i > lim) sv[i] = -INFINITY;
      }
      // Row max over eight independent chains (one chain of 127 dependent
      // max instructions would put its whole latency on the softmax path).
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = sv[k];
#pragma unroll
      for (int i = 8; i < BN; i += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = fmaxf(mx8[k], sv[i + k]);
      const float mraw = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float mx = mraw * a.sl2;  // sl2 > 0: max commutes with the scale
      // The previous P V must be done before P is rewritten or O rescaled.
      if (j > 0 && !mbar_wait(&o_done[t], (j - 1) & 1, kErrTimeoutEpilogue, a.err)) { ok = false; break; }
      tc_fence_after();
      const bool grow = mx > m_used + kRescaleThreshold;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? mx : m_used;
        const float alpha = exp2f(m_used - m_new);  // 0 on the first block, 1 for rows that keep their max
        if (j > 0) {
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld_32x32(t_o + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st_32x32(t_o + c * 32, o);
          }
        }
        l *= alpha;
        m_used = m_new;
      }
      // P = exp2(s - m_used) -> bf16 in shared memory.
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};  // four independent partial sums
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = ex2_approx(fmaf(sv[c * 32 + i], a.sl2, -m_used));
          const float p1 = ex2_approx(fmaf(sv[c * 32 + i + 1], a.sl2, -m_used));
          rs4[(i >> 1) & 3] += p0 + p1;
          pk[i / 2] = pack_bf16x2(p0, p1);
        }
        if constexpr (P_TMEM) {
          // Over this row's own S columns, all of which are already in registers;
          // the four stores overlap the next chunks' math and are waited for once.
          if (a.st_defer) tmem_st_32x16_issue(t_s + 16 * c, pk);
          else tmem_st_32x16(t_s + 16 * c, pk);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(P + p_off(r, c * 4 + q)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                                                                             pk[4 * q + 3]);
        }
      }
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      if constexpr (P_TMEM) {
        if (a.st_defer) tmem_st_wait();
      } else {
        fence_proxy_async();
      }
      // (shared-memory P: the proxy fence makes the generic writes visible to the tensor core)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok && mbar_wait(&o_done[t], (nblk - 1) & 1, kErrTimeoutEpilogue, a.err) && NK_IN_BOUNDS(qrow < a.T, a.err)) {
      tc_fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* orow = a.out + (long(b) * a.T + qrow) * a.ld_out + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tmem_ld_32x32(t_o + c * 32, o);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(orow + c * 32 + q * 8) =
              make_uint4(pack_bf16x2(o[8 * q] * inv, o[8 * q + 1] * inv), pack_bf16x2(o[8 * q + 2] * inv, o[8 * q + 3] * inv),
                         pack_bf16x2(o[8 * q + 4] * inv, o[8 * q + 5] * inv), pack_bf16x2(o[8 * q + 6] * inv, o[8 * q + 7] * inv));
      }
      a.lse[(long(b) * a.H + h) * a.T + qrow] = m_used + log2f(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool flash_fwd_tc_supported(int64_t T, int64_t HD) { return HD == 128 && T % 256 == 0; }

// qkv: (B*T, 3C) bf16; out: (B*T, C) bf16; lse: (B, H, T) fp32.
void flash_fwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t T, int64_t H) {
  using namespace fa;
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous(), "flash_tc: contiguous bf16 qkv");
  const int64_t C = qkv.size(1) / 3;
  TORCH_CHECK(C == H * HD && qkv.size(0) == B * T && flash_fwd_tc_supported(T, C / H), "flash_tc: shape");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(1) == C &&
                  (out.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "flash_tc: out");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * H * T, "flash_tc: lse");
  // 3-D map (inner: 3C columns, then T rows of one sequence, then B sequences):
  // rows past a sequence's end read as zeros instead of the next sequence.
  CUtensorMap m;
  cuuint64_t dims[3] = {cuuint64_t(3 * C), cuuint64_t(T), cuuint64_t(B)};
  cuuint64_t strides[2] = {cuuint64_t(3 * C * 2), cuuint64_t(T * 3 * C * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, qkv.data_ptr(), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "flash_tc: tensor map encode failed ", int(r));
  FaArgs a{};
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ld_out = out.stride(0);
  a.lse = lse.data_ptr<float>();
  a.B = int(B); a.H = int(H); a.T = int(T); a.C = int(C);
  a.sl2 = (1.f / std::sqrt(float(HD))) * 1.4426950408889634f;
  a.err = error_word();
  static const int st_defer = [] {
    const char* e = std::getenv("NANOGPT_FWD_ST_DEFER");
    return e ? std::atoi(e) : 1;
  }();
  a.st_defer = st_defer;
  static const int p_tmem = [] {
    const char* e = std::getenv("NANOGPT_FWD_P_TMEM");
    return e ? std::atoi(e) : 1;
  }();
  static bool configured = false;
  if (!configured) {
    TORCH_CHECK(cudaFuncSetAttribute(flash_fwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) ==
                    cudaSuccess && cudaFuncSetAttribute(flash_fwd_tc_kernel<false>,
                                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) ==
                    cudaSuccess, "flash_tc: smem");
    configured = true;
  }
  const at::cuda::CUDAGuard guard(qkv.device());
  dim3 grid(unsigned(T / 256), unsigned(B * H));
  if (p_tmem) flash_fwd_tc_kernel<true><<<grid, kThreads, kSmem, at::cuda::getCurrentCUDAStream()>>>(m, a);
  else flash_fwd_tc_kernel<false><<<grid, kThreads, kSmem, at::cuda::getCurrentCUDAStream()>>>(m, a);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "flash_fwd_tc launch failed");
}

}  // namespace nk
