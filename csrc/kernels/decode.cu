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

constexpr int kSampThreads = 1024;

__device__ __forceinline__ uint32_t bf16_order_key(uint16_t u) {
  return (u & 0x8000u) ? (~uint32_t(u) & 0xFFFFu) : (uint32_t(u) | 0x8000u);
}

// Exclusive block scan (double) over kSampThreads threads; returns the prefix
// and writes the block total to *total (visible to all threads on return).
__device__ double block_excl_scan(double v, double* sm_warp, double* total) {
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
    double w = sm_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sm_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const double before = (warp ? sm_warp[warp - 1] : 0.0) + x - v;
  *total = sm_warp[31];
  __syncthreads();
  return before;
}

// One CTA per row. Step index of row b is gen_count[b]; its uniform is
// uniforms[step * B + b]; the token goes to out_tokens[b * max_steps + step]
// and next_in[b]; gen_count[b] advances, and pos[b] too when advance_pos.
__global__ void __launch_bounds__(kSampThreads) sample_tokens_kernel(
    const __nv_bfloat16* __restrict__ logits, int ld, int V, float temperature, int top_k,
    const double* __restrict__ uniforms, int B, int max_steps, int* __restrict__ gen_count,
    int* __restrict__ out_tokens, int64_t* __restrict__ next_in, int* __restrict__ pos, int advance_pos) {
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const uint16_t* row = reinterpret_cast<const uint16_t*>(logits + long(b) * ld);
  const int seg = (V + kSampThreads - 1) / kSampThreads;
  const int i0 = min(V, tid * seg), i1 = min(V, i0 + seg);
  __shared__ uint32_t hist[256];
  __shared__ double sm_scan[32];
  __shared__ float sm_f[32];
  __shared__ int sm_i[32];
  __shared__ uint32_t sm_sel[4];  // threshold key, quota, token
  __shared__ int sm_token;

  // Largest value (order key) and the last index holding it.
  uint32_t best = 0;
  int best_i = -1;
  for (int i = i0; i < i1; ++i) {
    const uint32_t k = bf16_order_key(row[i]);
    if (k >= best) { best = k; best_i = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t ok = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ok > best || (ok == best && oi > best_i)) { best = ok; best_i = oi; }
  }
  if (lane == 0) { sm_i[warp] = best_i; sm_f[warp] = __uint_as_float(best); }
  __syncthreads();
  if (warp == 0) {
    best = __float_as_uint(sm_f[lane]);
    best_i = sm_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint32_t ok = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ok > best || (ok == best && oi > best_i)) { best = ok; best_i = oi; }
    }
    if (lane == 0) { sm_sel[3] = best; sm_token = best_i; }
  }
  __syncthreads();
  const uint32_t max_key = sm_sel[3];
  const int step = gen_count[b];

  if (temperature > 0.f) {
    // Threshold key tau and how many logits equal to tau are kept.
    const bool all = top_k <= 0 || top_k >= V;
    uint32_t tau = 0, quota = 0xFFFFFFFFu;
    if (!all) {
      for (int i = tid; i < 256; i += kSampThreads) hist[i] = 0;
      __syncthreads();
      for (int i = i0; i < i1; ++i) atomicAdd(&hist[bf16_order_key(row[i]) >> 8], 1u);
      __syncthreads();
      if (tid == 0) {
        uint32_t cum = 0;
        int hb = 255;
        for (; hb > 0; --hb) {
          if (cum + hist[hb] >= uint32_t(top_k)) break;
          cum += hist[hb];
        }
        sm_sel[0] = uint32_t(hb);
        sm_sel[1] = cum;
      }
      __syncthreads();
      const uint32_t hb = sm_sel[0], above = sm_sel[1];
      __syncthreads();
      for (int i = tid; i < 256; i += kSampThreads) hist[i] = 0;
      __syncthreads();
      for (int i = i0; i < i1; ++i) {
        const uint32_t k = bf16_order_key(row[i]);
        if ((k >> 8) == hb) atomicAdd(&hist[k & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t cum = above;
        int lb = 255;
        for (; lb > 0; --lb) {
          if (cum + hist[lb] >= uint32_t(top_k)) break;
          cum += hist[lb];
        }
        sm_sel[0] = (hb << 8) | uint32_t(lb);
        sm_sel[1] = uint32_t(top_k) - cum;  // ties at tau that are kept
      }
      __syncthreads();
      tau = sm_sel[0];
      quota = sm_sel[1];
    }
    // Rank of this thread's first tie among all ties (index order).
    int ties = 0;
    if (!all)
      for (int i = i0; i < i1; ++i) ties += bf16_order_key(row[i]) == tau;
    double tie_total;
    const double tie_before = block_excl_scan(double(ties), sm_scan, &tie_total);
    const float mx = __bfloat162float(__ushort_as_bfloat16(uint16_t((max_key & 0x8000u) ? (max_key & 0x7FFFu)
                                                                                          : (~max_key & 0xFFFFu))));
    const float sc = kLog2e / temperature;
    float wsum = 0.f;
    int rank = int(tie_before);
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = bf16_order_key(row[i]);
      bool keep = all || k > tau;
      if (!all && k == tau) keep = uint32_t(rank++) < quota;
      if (keep) wsum += exp2f((__bfloat162float(__ushort_as_bfloat16(row[i])) - mx) * sc);
    }
    double total;
    const double before = block_excl_scan(double(wsum), sm_scan, &total);
    const double u = uniforms[long(step < max_steps ? step : max_steps - 1) * B + b];
    const double thr = u * total;
    if (wsum > 0.f && thr >= before && (thr < before + double(wsum) || tid == kSampThreads - 1 ||
                                        before + double(wsum) >= total)) {
      double acc = before;
      int pick = -1, last = -1;
      rank = int(tie_before);
      for (int i = i0; i < i1; ++i) {
        const uint32_t k = bf16_order_key(row[i]);
        bool keep = all || k > tau;
        if (!all && k == tau) keep = uint32_t(rank++) < quota;
        if (!keep) continue;
        last = i;
        acc += double(exp2f((__bfloat162float(__ushort_as_bfloat16(row[i])) - mx) * sc));
        if (acc > thr) { pick = i; break; }
      }
      if (pick < 0) pick = last;
      sm_token = pick;  // at most one thread's interval holds thr
    }
    __syncthreads();
  }
  if (tid == 0) {
    const int tok = sm_token;
    if (step < max_steps) out_tokens[long(b) * max_steps + step] = tok;
    next_in[b] = tok;
    gen_count[b] = step + 1;
    if (advance_pos) pos[b] += 1;
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
  decode_attn_kernel<<<dim3(S, H, B), kDecThreads, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), int(qkv.stride(0)),
      reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()), pos.data_ptr<int>(), int(H), cap, int(chunk),
      scale_log2, part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(out.stride(0)));
  if (S > 1)
    decode_combine_kernel<<<dim3(H, B), 128, 0, st>>>(part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                                                      pos.data_ptr<int>(), int(H), S, int(chunk), cap,
                                                      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                      int(out.stride(0)));
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
  const at::cuda::CUDAGuard guard(logits.device());
  sample_tokens_kernel<<<B, kSampThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), int(logits.stride(0)), int(V), float(temperature),
      int(top_k), uniforms.data_ptr<double>(), int(B), int(max_steps), gen_count.data_ptr<int>(),
      out_tokens.data_ptr<int>(), next_in.data_ptr<int64_t>(), pos.data_ptr<int>(), advance_pos ? 1 : 0);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "sample_tokens launch failed");
}

}  // namespace nk
