// Inference kernels for KV-cache generation:
//   * kv_rope_append   RoPE + QK-RMSNorm of the new rows' q and k (in place in
//                      the fused QKV activation, same math as rope_qknorm_fwd)
//                      and the write of their k, v into the per-layer cache
//                      [B, H, capacity, 128] at each sequence's own position
//                      (rs-nanogpt src/model/kv_cache.rs:62-75 append,
//                      src/model/attention.rs:68-116 rope/norm order).
//   * decode_attention one query row per sequence against its cached prefix
//                      (src/model/flash_attention.rs:282-312): split-KV, every
//                      CTA reduces one chunk of keys of one (sequence, head)
//                      to a partial (max, sum, o[128]); a combine kernel merges
//                      the chunks. Memory bound: K/V rows are streamed once with
//                      16-byte loads, four keys in flight per half-warp.
//   * sample_tokens    on-device next-token choice per row of bf16 logits:
//                      greedy (temperature <= 0: largest logit, last index on
//                      ties, as src/eval/sample.rs:68-77) or top-k at a
//                      temperature (src/eval/sample.rs:123-174): the k-th
//                      largest logit is found by a two-pass radix select on
//                      the 16-bit order key of bf16, ties at the threshold are
//                      taken lowest index first, and one uniform draw per row
//                      (host-generated) picks from the tempered softmax over
//                      the kept logits in index order.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "launch.h"

namespace nk {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float dec_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- KV append ---------------------------------------------------------------

// Warp per (row, head). Row r belongs to sequence r / rows_per_seq at position
// pos_base[s] + r % rows_per_seq; it is cached only when r % rows_per_seq is
// below lens[s] (padding rows of a batched prefill are skipped).
__global__ void kv_rope_append_kernel(__nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ kc,
                                      __nv_bfloat16* __restrict__ vc, const int* __restrict__ pos_base,
                                      const int* __restrict__ lens, int rows, int rows_per_seq, int H, int C, int cap,
                                      const float* __restrict__ cos_t, const float* __restrict__ sin_t, int max_pos,
                                      int do_rope, float eps) {
  const int item = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (item >= rows * H) return;
  const int r = item / H, h = item % H;
  const int s = r / rows_per_seq, t = r % rows_per_seq;
  const int p = (pos_base ? pos_base[s] : 0) + t;
  __nv_bfloat16* row = qkv + long(r) * 3 * C + h * 128 + lane * 4;
  if (do_rope) {
    const int pp = min(p, max_pos - 1);
    const bool first = lane < 16;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      __nv_bfloat16* ptr = row + part * C;
      const uint2 w = *reinterpret_cast<const uint2*>(ptr);
      const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
      const float x[4] = {a.x, a.y, b.x, b.y};
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[j], 16);
        const int i = (lane & 15) * 4 + j;
        const float c = cos_t[pp * 64 + i], sn = sin_t[pp * 64 + i];
        o[j] = first ? x[j] * c + partner * sn : x[j] * c - partner * sn;
      }
      const float ss = dec_warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
      const float denom = __bfloat162float(__float2bfloat16(sqrtf(ss / 128.f + eps)));
      *reinterpret_cast<uint2*>(ptr) =
          make_uint2(pack_bf16x2(o[0] / denom, o[1] / denom), pack_bf16x2(o[2] / denom, o[3] / denom));
    }
    __syncwarp();
  }
  const bool keep = (lens ? t < lens[s] : true) && p < cap;
  if (keep) {
    const long dst = ((long(s) * H + h) * cap + p) * 128 + lane * 4;
    *reinterpret_cast<uint2*>(kc + dst) = *reinterpret_cast<const uint2*>(row + C);
    *reinterpret_cast<uint2*>(vc + dst) = *reinterpret_cast<const uint2*>(row + 2 * C);
  }
}

// ---- decode attention ----------------------------------------------------------

constexpr int kDecThreads = 128;  // 4 warps = 8 half-warps, one key per half-warp
constexpr int kDecUnroll = 4;     // keys in flight per half-warp

__device__ __forceinline__ void bf16x8_to_f32(const uint4 u, float (&f)[8]) {
  float2 t;
  t = unpack_bf16x2(u.x); f[0] = t.x; f[1] = t.y;
  t = unpack_bf16x2(u.y); f[2] = t.x; f[3] = t.y;
  t = unpack_bf16x2(u.z); f[4] = t.x; f[5] = t.y;
  t = unpack_bf16x2(u.w); f[6] = t.x; f[7] = t.y;
}

// grid (splits, H, B). Keys of sequence b are 0 .. pos[b] (inclusive: the
// current token was appended at pos[b]). CTA `split` covers keys
// [split*chunk, (split+1)*chunk). Writes (m, l) and the unnormalised o of
// its chunk (base-2 exponent units), or the final bf16 row when splits == 1.
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ld_qkv, const __nv_bfloat16* __restrict__ kc,
    const __nv_bfloat16* __restrict__ vc, const int* __restrict__ pos, int H, int cap, int chunk, float scale_log2,
    float* __restrict__ part_o, float* __restrict__ part_ml, __nv_bfloat16* __restrict__ out, int ld_out) {
  // No early trigger: this grid spans many waves, and a dependent GEMM's
  // CTAs (a whole SM's shared memory each) would take SMs from it.
  pdl_wait();
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z, S = gridDim.x;
  const int len = min(pos[b] + 1, cap);
  const int k0 = split * chunk, k1 = min(len, k0 + chunk);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int half = lane >> 4, sub = lane & 15;
  const int hw = warp * 2 + half;  // half-warp index 0..7
  __shared__ float sm_o[8][128];
  __shared__ float sm_m[8], sm_l[8];

  float q[8];
  {
    const uint4 u = *reinterpret_cast<const uint4*>(qkv + long(b) * ld_qkv + h * 128 + sub * 8);
    bf16x8_to_f32(u, q);
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] *= scale_log2;
  }
  float m = -1e30f, l = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const long base = (long(b) * H + h) * cap * 128 + sub * 8;
  // The loop bound is uniform across the warp (both half-warps run every
  // iteration) because the 16-lane dot-product reduction shuffles over the
  // full warp; keys past the chunk are masked instead.
  for (int jb = k0 + warp * 2; jb < k1; jb += 8 * kDecUnroll) {
    uint4 ku[kDecUnroll], vu[kDecUnroll];
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      const int j = jb + half + u * 8;
      if (j < k1) {
        ku[u] = __ldg(reinterpret_cast<const uint4*>(kc + base + long(j) * 128));
        vu[u] = __ldg(reinterpret_cast<const uint4*>(vc + base + long(j) * 128));
      } else {
        ku[u] = make_uint4(0, 0, 0, 0);
        vu[u] = make_uint4(0, 0, 0, 0);
      }
    }
    float sc[kDecUnroll];
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      float kf[8];
      bf16x8_to_f32(ku[u], kf);
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(q[i], kf[i], d);
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      sc[u] = (jb + half + u * 8 < k1) ? d : -INFINITY;
    }
    float mx = m;
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) mx = fmaxf(mx, sc[u]);
    const float corr = exp2f(m - mx);
    l *= corr;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] *= corr;
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      const float p = exp2f(sc[u] - mx);
      l += p;
      float vf[8];
      bf16x8_to_f32(vu[u], vf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = fmaf(p, vf[i], o[i]);
    }
    m = mx;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) sm_o[hw][sub * 8 + i] = o[i];
  if (sub == 0) {
    sm_m[hw] = m;
    sm_l[hw] = l;
  }
  __syncthreads();
  // Thread t merges dimension t over the 8 half-warps.
  float M = -1e30f;
#pragma unroll
  for (int i = 0; i < 8; ++i) M = fmaxf(M, sm_m[i]);
  float L = 0.f, O = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float w = exp2f(sm_m[i] - M);
    L += sm_l[i] * w;
    O += sm_o[i][tid] * w;
  }
  if (S == 1) {
    out[long(b) * ld_out + h * 128 + tid] = __float2bfloat16(L > 0.f ? O / L : 0.f);
  } else {
    const long pi = (long(b) * H + h) * S + split;
    part_o[pi * 128 + tid] = O;
    if (tid == 0) {
      part_ml[pi * 2] = M;
      part_ml[pi * 2 + 1] = L;
    }
  }
}

// grid (H, B), 128 threads: merge the splits of one (sequence, head).
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                      const int* __restrict__ pos, int H, int S, int chunk, int cap,
                                      __nv_bfloat16* __restrict__ out, int ld_out) {
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int len = min(pos[b] + 1, cap);
  const int used = min(S, (len + chunk - 1) / chunk);
  const long p0 = (long(b) * H + h) * S;
  float M = -1e30f;
  for (int s = 0; s < used; ++s) M = fmaxf(M, part_ml[(p0 + s) * 2]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < used; ++s) {
    const float w = exp2f(part_ml[(p0 + s) * 2] - M);
    L += part_ml[(p0 + s) * 2 + 1] * w;
    O += part_o[(p0 + s) * 128 + tid] * w;
  }
  out[long(b) * ld_out + h * 128 + tid] = __float2bfloat16(L > 0.f ? O / L : 0.f);
}

// ---- sampling ------------------------------------------------------------------

constexpr int kSampThreads = 512;

__device__ __forceinline__ uint32_t bf16_order_key(uint16_t u) {
  return (u & 0x8000u) ? (~uint32_t(u) & 0xFFFFu) : (uint32_t(u) | 0x8000u);
}

// Exclusive block scan (double) over kSampThreads threads; returns the prefix
// and writes the block total to *total.
__device__ double block_excl_scan(double v, double* sm_warp, double* total) {
  constexpr int kWarps = kSampThreads / 32;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sm_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    double w = lane < kWarps ? sm_warp[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kWarps) sm_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const double before = (warp ? sm_warp[warp - 1] : 0.0) + x - v;
  *total = sm_warp[kWarps - 1];
  __syncthreads();
  return before;
}

// Block-wide sum of an int (every thread gets the total).
__device__ __forceinline__ int block_sum_int(int v, int* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (threadIdx.x % 32 == 0) sm[threadIdx.x / 32] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < kSampThreads / 32; ++w) t += sm[w];
  __syncthreads();
  return t;
}

// One CTA per row. Thread t owns the contiguous logits [t*VPT, t*VPT + VPT)
// (so per-thread sums in index order can be block-scanned); their 16-bit
// order keys live in shared memory, two per word, with thread t's word j at
// t*W + (j ^ (t % 32)) (W = VPT/2, a multiple of 32) so that the 32 lanes of
// a warp reading their j-th words hit 32 different banks.
// Step index of row b is gen_count[b]; its uniform is uniforms[step * B + b];
// the token goes to out_tokens[b * max_steps + step] and next_in[b];
// gen_count[b] advances, and pos[b] too when advance_pos.
// The k-th largest key (tau) is found by a 16-step binary search over the key
// space, each step counting keys >= mid.
__global__ void __launch_bounds__(kSampThreads) sample_tokens_kernel(
    const __nv_bfloat16* __restrict__ logits, int ld, int V, int VPT, float temperature, int top_k,
    const double* __restrict__ uniforms, int B, int max_steps, int* __restrict__ gen_count,
    int* __restrict__ out_tokens, int64_t* __restrict__ next_in, int* __restrict__ pos, int advance_pos) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ uint32_t keys[];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int W = VPT / 2, i0 = tid * VPT, sw = tid & 31;
  const uint32_t* mine = keys + tid * W;
  __shared__ double sm_scan[32];
  __shared__ int sm_int[32];
  __shared__ uint32_t sm_key[32];
  __shared__ int sm_idx[32];
  __shared__ int sm_token;

  {
    const uint16_t* row = reinterpret_cast<const uint16_t*>(logits + long(b) * ld);
    const int words = kSampThreads * W;
    for (int g = tid; g < words; g += kSampThreads) {
      const int i = 2 * g;
      const uint32_t lo = i < V ? bf16_order_key(row[i]) : 0u;
      const uint32_t hi = i + 1 < V ? bf16_order_key(row[i + 1]) : 0u;
      const int t = g / W, j = g % W;
      keys[t * W + (j ^ (t & 31))] = lo | (hi << 16);
    }
  }
  __syncthreads();
#define KEYW(j) mine[(j) ^ sw]

  // Largest key, last index on ties.
  uint32_t best = 0;
  int best_i = -1;
  for (int j = 0; j < W; ++j) {
    const uint32_t w = KEYW(j);
    const uint32_t lo = w & 0xFFFFu, hi = w >> 16;
    const int i = i0 + 2 * j;
    if (i < V && lo >= best) { best = lo; best_i = i; }
    if (i + 1 < V && hi >= best) { best = hi; best_i = i + 1; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t ok = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ok > best || (ok == best && oi > best_i)) { best = ok; best_i = oi; }
  }
  if (lane == 0) { sm_key[warp] = best; sm_idx[warp] = best_i; }
  __syncthreads();
  if (warp == 0) {
    best = lane < kSampThreads / 32 ? sm_key[lane] : 0u;
    best_i = lane < kSampThreads / 32 ? sm_idx[lane] : -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint32_t ok = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ok > best || (ok == best && oi > best_i)) { best = ok; best_i = oi; }
    }
    if (lane == 0) { sm_key[0] = best; sm_token = best_i; }
  }
  __syncthreads();
  const uint32_t max_key = sm_key[0];
  const int step = gen_count[b];

  if (temperature > 0.f) {
    const bool all = top_k <= 0 || top_k >= V;
    uint32_t tau = 0;
    int quota = 0x7FFFFFFF;
    if (!all) {
      // Largest tau with count(key >= tau) >= k (padding keys are 0 and
      // real keys are >= 1, so padding never reaches the count at tau >= 1).
      uint32_t lo = 1, hi = 0xFFFFu;
      while (lo < hi) {
        const uint32_t mid = (lo + hi + 1) >> 1;
        int cnt = 0;
        for (int j = 0; j < W; ++j) {
          const uint32_t w = KEYW(j);
          cnt += ((w & 0xFFFFu) >= mid) + ((w >> 16) >= mid);
        }
        if (block_sum_int(cnt, sm_int) >= top_k) lo = mid;
        else hi = mid - 1;
      }
      tau = lo;
      int gt = 0;
      for (int j = 0; j < W; ++j) {
        const uint32_t w = KEYW(j);
        gt += ((w & 0xFFFFu) > tau) + ((w >> 16) > tau);
      }
      quota = top_k - block_sum_int(gt, sm_int);  // ties at tau that are kept, lowest index first
    }
    int ties = 0;
    if (!all)
      for (int j = 0; j < W; ++j) {
        const uint32_t w = KEYW(j);
        ties += ((w & 0xFFFFu) == tau) + ((w >> 16) == tau);
      }
    double tie_total;
    const int tie_before = int(block_excl_scan(double(ties), sm_scan, &tie_total));
    const float mx = __bfloat162float(__ushort_as_bfloat16(
        uint16_t((max_key & 0x8000u) ? (max_key & 0x7FFFu) : (~max_key & 0xFFFFu))));
    const float sc = kLog2e / temperature;
    // Kept-logit weight exp((x - max) / T), in base 2.
    auto weight = [&](uint32_t k, int i, int& rank_io) -> float {
      if (i >= V) return 0.f;
      bool keep = all || k > tau;
      if (!all && k == tau) keep = rank_io++ < quota;
      if (!keep) return 0.f;
      const uint16_t u = uint16_t((k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu));
      return exp2f((__bfloat162float(__ushort_as_bfloat16(u)) - mx) * sc);
    };
    float wsum = 0.f;
    int rank = tie_before;
    for (int j = 0; j < W; ++j) {
      const uint32_t w = KEYW(j);
      wsum += weight(w & 0xFFFFu, i0 + 2 * j, rank);
      wsum += weight(w >> 16, i0 + 2 * j + 1, rank);
    }
    double total;
    const double before = block_excl_scan(double(wsum), sm_scan, &total);
    const double u = uniforms[long(step < max_steps ? step : max_steps - 1) * B + b];
    const double thr = u * total;
    // The thread whose interval [before, before + wsum) holds thr picks; the
    // last thread with weight also takes thr values lost to rounding.
    if (wsum > 0.f && thr >= before && (thr < before + double(wsum) || before + double(wsum) >= total)) {
      double acc = before;
      int pick = -1, last = -1;
      rank = tie_before;
      for (int e = 0; e < VPT && pick < 0; ++e) {
        const uint32_t w = KEYW(e >> 1);
        const float x = weight((e & 1) ? (w >> 16) : (w & 0xFFFFu), i0 + e, rank);
        if (x > 0.f) {
          last = i0 + e;
          acc += double(x);
          if (acc > thr) pick = i0 + e;
        }
      }
      sm_token = pick >= 0 ? pick : last;
    }
    __syncthreads();
  }
#undef KEYW
  if (tid == 0) {
    const int tok = sm_token;
    if (step < max_steps) out_tokens[long(b) * max_steps + step] = tok;
    next_in[b] = tok;
    gen_count[b] = step + 1;
    if (advance_pos) pos[b] += 1;
  }
}

// ---- skinny GEMM epilogues -------------------------------------------------------

// The decode-path GEMMs run with operands swapped (the weight rows fill the
// 128-row tensor-core tile and the grid; the few token rows are the narrow N
// side), split over K with fp32 atomics straight into acc[M, N] (token-major).
// These kernels read one token row of the accumulator per CTA, zero it for the
// next product and apply the epilogue.

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

// mode 0: out = acc; 1: out = relu(acc)^2 (aux_out = acc when given);
// 3: out = acc + aux. With norm_out, also norm_out = RMSNorm(out) (N <= 2048).
constexpr int kFinThreads = 128;
constexpr int kFinKeep = 4;  // float4 chunks per thread kept for the norm

__global__ void __launch_bounds__(kFinThreads) skinny_finish_kernel(
    float* __restrict__ acc, int N, int mode, __nv_bfloat16* __restrict__ out, int ld_out,
    const __nv_bfloat16* __restrict__ aux, int ld_aux, __nv_bfloat16* __restrict__ aux_out, int ld_aux_out,
    __nv_bfloat16* __restrict__ norm_out, int ld_norm, float eps) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x, tid = threadIdx.x;
  float4* a = reinterpret_cast<float4*>(acc + long(m) * N);
  auto process = [&](int c4) -> float4 {
    const float4 v = a[c4];
    a[c4] = make_float4(0.f, 0.f, 0.f, 0.f);
    float x[4] = {bf16r(v.x), bf16r(v.y), bf16r(v.z), bf16r(v.w)};
    if (mode == 3) {
      const uint2 r = *reinterpret_cast<const uint2*>(aux + long(m) * ld_aux + c4 * 4);
      const float2 r0 = unpack_bf16x2(r.x), r1 = unpack_bf16x2(r.y);
      x[0] = bf16r(x[0] + r0.x); x[1] = bf16r(x[1] + r0.y); x[2] = bf16r(x[2] + r1.x); x[3] = bf16r(x[3] + r1.y);
    } else if (mode == 1) {
      if (aux_out)
        *reinterpret_cast<uint2*>(aux_out + long(m) * ld_aux_out + c4 * 4) =
            make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float h = fmaxf(x[i], 0.f);
        x[i] = bf16r(h * h);
      }
    }
    *reinterpret_cast<uint2*>(out + long(m) * ld_out + c4 * 4) =
        make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    return make_float4(x[0], x[1], x[2], x[3]);
  };
  float4 keep[kFinKeep];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kFinKeep; ++j) {
    const int c4 = tid + j * kFinThreads;
    keep[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c4 < N / 4) {
      keep[j] = process(c4);
      ss += keep[j].x * keep[j].x + keep[j].y * keep[j].y + keep[j].z * keep[j].z + keep[j].w * keep[j].w;
    }
  }
  for (int c4 = tid + kFinKeep * kFinThreads; c4 < N / 4; c4 += kFinThreads) process(c4);  // no norm here
  if (norm_out == nullptr) return;
  __shared__ float red[kFinThreads / 32];
  ss = dec_warp_sum(ss);
  if (tid % 32 == 0) red[tid / 32] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kFinThreads / 32; ++w) tot += red[w];
  // The reference divides by the bf16-rounded denominator.
  const float denom = bf16r(sqrtf(tot / N + eps));
#pragma unroll
  for (int j = 0; j < kFinKeep; ++j) {
    const int c4 = tid + j * kFinThreads;
    if (c4 >= N / 4) break;
    const float4 x = keep[j];
    *reinterpret_cast<uint2*>(norm_out + long(m) * ld_norm + c4 * 4) =
        make_uint2(pack_bf16x2(x.x / denom, x.y / denom), pack_bf16x2(x.z / denom, x.w / denom));
  }
}

// QKV epilogue of a decode step: acc[M, 3C] -> q (RoPE + QK-norm) into the
// qkv buffer, k (RoPE + QK-norm) and v into the caches at position pos[m].
// Warp per (part, head) item; 8 warps per token row.
__global__ void __launch_bounds__(256) qkv_decode_finish_kernel(
    float* __restrict__ acc, int H, int C, __nv_bfloat16* __restrict__ q_out, int ld_q,
    __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, const int* __restrict__ pos, int cap,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int max_pos, float eps) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int p = pos[m];
  const int pp = min(p, max_pos - 1);
  for (int item = warp; item < 3 * H; item += 8) {
    const int part = item / H, h = item % H;
    float4* a = reinterpret_cast<float4*>(acc + long(m) * 3 * C + part * C + h * 128) + lane;
    const float4 v = *a;
    *a = make_float4(0.f, 0.f, 0.f, 0.f);
    float x[4] = {bf16r(v.x), bf16r(v.y), bf16r(v.z), bf16r(v.w)};
    if (part < 2) {
      const bool first = lane < 16;
      float o[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[jj], 16);
        const int i = (lane & 15) * 4 + jj;
        const float c = cos_t[pp * 64 + i], sn = sin_t[pp * 64 + i];
        o[jj] = first ? x[jj] * c + partner * sn : x[jj] * c - partner * sn;
      }
      const float ss = dec_warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
      const float denom = bf16r(sqrtf(ss / 128.f + eps));
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) x[jj] = o[jj] / denom;
    }
    const uint2 w = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    if (part == 0) {
      *reinterpret_cast<uint2*>(q_out + long(m) * ld_q + h * 128 + lane * 4) = w;
    } else if (p < cap) {
      __nv_bfloat16* dst = (part == 1 ? kc : vc) + ((long(m) * H + h) * cap + p) * 128 + lane * 4;
      *reinterpret_cast<uint2*>(dst) = w;
    }
  }
}

void check_i32(const torch::Tensor& t, int64_t n, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous() && t.numel() >= n, what,
              ": contiguous int32 CUDA tensor of at least ", n, " elements");
}

}  // namespace

void kv_rope_append(torch::Tensor qkv, torch::Tensor k_cache, torch::Tensor v_cache, c10::optional<torch::Tensor> pos,
                    c10::optional<torch::Tensor> lens, int64_t rows_per_seq, int64_t H, torch::Tensor cos_t,
                    torch::Tensor sin_t, bool do_rope, double eps) {
  TORCH_CHECK(qkv.is_cuda() && qkv.is_contiguous() && qkv.scalar_type() == at::kBFloat16, "kv_append: bf16 qkv");
  const int64_t rows = qkv.size(0), C = qkv.size(1) / 3;
  TORCH_CHECK(C == H * 128, "kv_append: head_dim must be 128");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  k_cache.sizes() == v_cache.sizes() && k_cache.scalar_type() == at::kBFloat16 &&
                  v_cache.scalar_type() == at::kBFloat16,
              "kv_append: caches are contiguous bf16 [B, H, capacity, 128]");
  TORCH_CHECK(k_cache.size(1) == H && k_cache.size(3) == 128, "kv_append: cache head layout");
  TORCH_CHECK(rows % rows_per_seq == 0 && rows / rows_per_seq <= k_cache.size(0), "kv_append: rows vs batch");
  const int64_t nseq = rows / rows_per_seq;
  if (pos) check_i32(*pos, nseq, "kv_append pos");
  if (lens) check_i32(*lens, nseq, "kv_append lens");
  TORCH_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.size(1) == 64, "kv_append: rope tables");
  const at::cuda::CUDAGuard guard(qkv.device());
  const int warps = 8;
  const int64_t items = rows * H;
  kv_rope_append_kernel<<<(items + warps - 1) / warps, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), pos ? pos->data_ptr<int>() : nullptr,
      lens ? lens->data_ptr<int>() : nullptr, int(rows), int(rows_per_seq), int(H), int(C), int(k_cache.size(2)),
      cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), int(cos_t.size(0)), do_rope ? 1 : 0, float(eps));
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "kv_rope_append launch failed");
}

void decode_attention(torch::Tensor qkv, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor pos,
                      torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml, int64_t chunk) {
  const int64_t B = qkv.size(0), C = qkv.size(1) / 3, H = C / 128;
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1 && C == H * 128, "decode_attention: qkv");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(0) >= B && k_cache.size(1) == H &&
                  k_cache.size(3) == 128 && k_cache.sizes() == v_cache.sizes(),
              "decode_attention: caches are [B, H, capacity, 128]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == B && out.size(1) == C && out.stride(1) == 1,
              "decode_attention: out [B, C] bf16");
  TORCH_CHECK(chunk > 0 && chunk % 8 == 0, "decode_attention: chunk is a positive multiple of 8");
  check_i32(pos, B, "decode_attention pos");
  const int cap = int(k_cache.size(2));
  const int S = int((cap + chunk - 1) / chunk);
  if (S > 1) {
    TORCH_CHECK(part_o.is_contiguous() && part_o.scalar_type() == at::kFloat && part_o.numel() >= B * H * S * 128 &&
                    part_ml.is_contiguous() && part_ml.scalar_type() == at::kFloat && part_ml.numel() >= B * H * S * 2,
                "decode_attention: partial buffers too small");
  }
  const at::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float scale_log2 = float(kLog2e / std::sqrt(128.0));
  launch_k(decode_attn_kernel, dim3(S, H, B), dim3(kDecThreads), 0, st,
           reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), int(qkv.stride(0)),
           reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()),
           reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()), pos.data_ptr<int>(), int(H), cap, int(chunk),
           scale_log2, part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(out.stride(0)));
  if (S > 1)
    launch_k(decode_combine_kernel, dim3(H, B), dim3(128), 0, st, part_o.data_ptr<float>(),
             part_ml.data_ptr<float>(), pos.data_ptr<int>(), int(H), S, int(chunk), cap,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(out.stride(0)));
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "decode_attention launch failed");
}

void sample_tokens(torch::Tensor logits, double temperature, int64_t top_k, torch::Tensor uniforms,
                   torch::Tensor gen_count, torch::Tensor out_tokens, torch::Tensor next_in, torch::Tensor pos,
                   bool advance_pos) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1,
              "sample_tokens: bf16 logits rows");
  const int64_t B = logits.size(0), V = logits.size(1);
  TORCH_CHECK(uniforms.scalar_type() == at::kDouble && uniforms.is_contiguous() && uniforms.dim() == 2 &&
                  uniforms.size(1) == B,
              "sample_tokens: uniforms [max_steps, B] float64");
  const int64_t max_steps = uniforms.size(0);
  check_i32(gen_count, B, "sample_tokens gen_count");
  check_i32(pos, B, "sample_tokens pos");
  TORCH_CHECK(out_tokens.scalar_type() == at::kInt && out_tokens.is_contiguous() &&
                  out_tokens.numel() >= B * max_steps,
              "sample_tokens: out_tokens [B, max_steps] int32");
  TORCH_CHECK(next_in.scalar_type() == at::kLong && next_in.is_contiguous() && next_in.numel() >= B,
              "sample_tokens: next_in int64 [B]");
  // Logits per thread: a multiple of 64 (32 key words, the swizzle period).
  const int vpt = int(((V + kSampThreads - 1) / kSampThreads + 63) / 64 * 64);
  const size_t smem = size_t(kSampThreads) * vpt * 2;
  TORCH_CHECK(smem <= 200 * 1024, "sample_tokens: vocabulary too large for the shared-memory key table");
  static size_t smem_set = 0;
  if (smem > smem_set) {
    TORCH_CHECK(cudaFuncSetAttribute(sample_tokens_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     int(smem)) == cudaSuccess,
                "sample_tokens: shared-memory opt-in failed");
    smem_set = smem;
  }
  const at::cuda::CUDAGuard guard(logits.device());
  launch_k(sample_tokens_kernel, dim3(B), dim3(kSampThreads), smem, at::cuda::getCurrentCUDAStream(),
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), int(logits.stride(0)), int(V), vpt,
      float(temperature), int(top_k), uniforms.data_ptr<double>(), int(B), int(max_steps), gen_count.data_ptr<int>(),
      out_tokens.data_ptr<int>(), next_in.data_ptr<int64_t>(), pos.data_ptr<int>(), advance_pos ? 1 : 0);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "sample_tokens launch failed");
}

void skinny_finish(torch::Tensor acc, torch::Tensor out, int64_t mode, c10::optional<torch::Tensor> aux,
                   c10::optional<torch::Tensor> aux_out, c10::optional<torch::Tensor> norm_out, double eps) {
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.dim() == 2,
              "skinny_finish: acc is a contiguous fp32 [M, N] tensor");
  const int64_t M = acc.size(0), N = acc.size(1);
  TORCH_CHECK(N % 4 == 0, "skinny_finish: N must be a multiple of 4");
  auto check_out = [&](const torch::Tensor& t, const char* what) {
    TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.size(0) == M && t.size(1) == N && t.stride(1) == 1 &&
                    t.stride(0) % 4 == 0,
                "skinny_finish: ", what, " is bf16 [M, N] with 8-byte aligned rows");
  };
  check_out(out, "out");
  TORCH_CHECK(mode == 0 || mode == 1 || mode == 3, "skinny_finish: mode 0, 1 or 3");
  if (mode == 3) {
    TORCH_CHECK(aux.has_value(), "skinny_finish: residual mode needs aux");
    check_out(*aux, "aux");
  }
  if (aux_out) check_out(*aux_out, "aux_out");
  if (norm_out) {
    check_out(*norm_out, "norm_out");
    TORCH_CHECK(N <= 4 * kFinThreads * kFinKeep, "skinny_finish: the fused norm takes N <= 2048");
  }
  const at::cuda::CUDAGuard guard(acc.device());
  launch_k(skinny_finish_kernel, dim3(M), dim3(kFinThreads), 0, at::cuda::getCurrentCUDAStream(),
      acc.data_ptr<float>(), int(N), int(mode), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      int(out.stride(0)), mode == 3 ? reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr()) : nullptr,
      mode == 3 ? int(aux->stride(0)) : 0,
      (mode == 1 && aux_out) ? reinterpret_cast<__nv_bfloat16*>(aux_out->data_ptr()) : nullptr,
      aux_out ? int(aux_out->stride(0)) : 0,
      norm_out ? reinterpret_cast<__nv_bfloat16*>(norm_out->data_ptr()) : nullptr,
      norm_out ? int(norm_out->stride(0)) : 0, float(eps));
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "skinny_finish launch failed");
}

void qkv_decode_finish(torch::Tensor acc, torch::Tensor qkv, torch::Tensor k_cache, torch::Tensor v_cache,
                       torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t, int64_t H, double eps) {
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.dim() == 2,
              "qkv_decode_finish: acc is a contiguous fp32 [M, 3C] tensor");
  const int64_t M = acc.size(0), C = acc.size(1) / 3;
  TORCH_CHECK(C == H * 128, "qkv_decode_finish: head_dim must be 128");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.size(0) == M && qkv.size(1) >= C && qkv.stride(1) == 1 &&
                  qkv.stride(0) % 4 == 0,
              "qkv_decode_finish: q output rows");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.sizes() == v_cache.sizes() &&
                  k_cache.size(0) >= M && k_cache.size(1) == H && k_cache.size(3) == 128 &&
                  k_cache.scalar_type() == at::kBFloat16 && v_cache.scalar_type() == at::kBFloat16,
              "qkv_decode_finish: caches are bf16 [B, H, capacity, 128]");
  check_i32(pos, M, "qkv_decode_finish pos");
  TORCH_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.size(1) == 64, "qkv_decode_finish: tables");
  const at::cuda::CUDAGuard guard(acc.device());
  launch_k(qkv_decode_finish_kernel, dim3(M), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
      acc.data_ptr<float>(), int(H), int(C), reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), int(qkv.stride(0)),
      reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()),
      pos.data_ptr<int>(), int(k_cache.size(2)), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
      int(cos_t.size(0)), float(eps));
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "qkv_decode_finish launch failed");
}

}  // namespace nk
