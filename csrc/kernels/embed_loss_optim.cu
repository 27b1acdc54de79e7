// Memory-bound kernels around the GEMMs:
//   * embedding_fwd/bwd  gather fp32 master rows -> bf16 activations; scatter-add
//                        bf16 row grads into the fp32 gradient with vector atomics
//                        (rs-nanogpt src/model/embedding.rs:33-35, src/model/gpt.rs:103)
//   * softmax_xent       two streaming passes over a chunk of bf16 logits rows: fp32 log-sum-exp,
//                        per-row NLL with ignore_index -1, and (optionally) the
//                        gradient (softmax - onehot) * scale written in place over
//                        the logits (src/model/loss.rs:20-82). Together with the
//                        tcgen05 GEMMs this is the fused lm_head + cross-entropy:
//                        the full (B*T, V) logits are never materialized.
//   * adamw_step         candle AdamW semantics (decoupled decay, bias correction)
//                        on a contiguous slice of the flat master/grad/m/v buffers,
//                        also refreshing the bf16 working copy (src/train/optim.rs)
//   * sumsq              sum of squares for the gradient norm
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace nk {

// ---- embedding --------------------------------------------------------------

__device__ __forceinline__ uint2 embed_load4(const float* row, int c) {
  const float4 f = reinterpret_cast<const float4*>(row)[c];
  return make_uint2(pack_bf16x2(f.x, f.y), pack_bf16x2(f.z, f.w));
}
__device__ __forceinline__ uint2 embed_load4(const __nv_bfloat16* row, int c) {
  return reinterpret_cast<const uint2*>(row)[c];
}

// The table is either the fp32 master or its bf16 working copy (identical
// after rounding: the reference casts the gathered fp32 rows to bf16).
template <typename T>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ idx, const T* __restrict__ wte,
                                     __nv_bfloat16* __restrict__ out, int rows, int C, int V) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const int64_t t = idx[row];
  if (t < 0 || t >= V) return;  // host validates ids; never read out of range
  const T* src = wte + t * C;
  uint2* dst = reinterpret_cast<uint2*>(out + long(row) * C);
  for (int c = lane; c < C / 4; c += 32) dst[c] = embed_load4(src, c);
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ idx, const __nv_bfloat16* __restrict__ dx,
                                     float* __restrict__ grad, int rows, int C, int V) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const int64_t t = idx[row];
  if (t < 0 || t >= V) return;
  const uint2* src = reinterpret_cast<const uint2*>(dx + long(row) * C);
  float4* dst = reinterpret_cast<float4*>(grad + t * C);
  for (int c = lane; c < C / 4; c += 32) {
    uint2 w = src[c];
    float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
    atomicAdd(dst + c, make_float4(a.x, a.y, b.x, b.y));
  }
}

void embedding_fwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor out) {
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous(), "embedding: int64 ids");
  TORCH_CHECK(wte.is_contiguous() && out.is_contiguous(), "embedding: layout");
  const int rows = int(idx.numel()), V = int(wte.size(0)), C = int(wte.size(1));
  TORCH_CHECK(C % 4 == 0 && out.numel() == int64_t(rows) * C, "embedding: shape");
  const at::cuda::CUDAGuard guard(idx.device());
  const int warps = 8;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (wte.scalar_type() == at::kFloat)
    embedding_fwd_kernel<float><<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>(
        idx.data_ptr<int64_t>(), wte.data_ptr<float>(), op, rows, C, V);
  else if (wte.scalar_type() == at::kBFloat16)
    embedding_fwd_kernel<__nv_bfloat16><<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>(
        idx.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(wte.data_ptr()), op, rows, C, V);
  else
    TORCH_CHECK(false, "embedding: fp32 or bf16 table");
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "embedding_fwd launch failed");
}

void embedding_bwd(torch::Tensor idx, torch::Tensor dx, torch::Tensor grad) {
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous() && dx.is_contiguous(), "embedding_bwd: layout");
  TORCH_CHECK(grad.scalar_type() == at::kFloat && grad.is_contiguous(), "embedding_bwd: fp32 grad");
  const int rows = int(idx.numel()), V = int(grad.size(0)), C = int(grad.size(1));
  const at::cuda::CUDAGuard guard(idx.device());
  const int warps = 8;
  embedding_bwd_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dx.data_ptr()), grad.data_ptr<float>(), rows, C,
      V);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "embedding_bwd launch failed");
}

// ---- softmax cross-entropy over a logits chunk ---------------------------------

constexpr int kXentThreads = 512;

template <typename Op>
__device__ __forceinline__ float block_reduce(float v, float* smem, Op op) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  v = smem[0];
  for (int w = 1; w < kXentThreads / 32; ++w) v = op(v, smem[w]);
  return v;
}

// NV = 8-element vectors held in registers per thread (NV * 8 * 512 >= V).
// Online softmax statistics: the running max m and sum s = sum exp(v - m).
__device__ __forceinline__ void xent_absorb8(uint4 w, float& m, float& s) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  float f[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 p = unpack_bf16x2(ws[j]);
    f[2 * j] = p.x;
    f[2 * j + 1] = p.y;
  }
  float cm = f[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) cm = fmaxf(cm, f[j]);
  if (cm > m) {
    s *= __expf(m - cm);  // m = -inf on the first chunk: s is 0 and stays 0
    m = cm;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) s += __expf(f[j] - m);
}

__device__ __forceinline__ void xent_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
  m = mm;
}

// One CTA per row, streaming: pass 1 reads the row once for the online max /
// sum, pass 2 reads it again (an L2 hit: the rows in flight on the GPU, about
// 4 per SM x 128 KB, fit in L2) and writes the gradient in place. No row is
// held in registers, so several rows share an SM and hide each other's latency.
__global__ void __launch_bounds__(kXentThreads, 4) softmax_xent_kernel(
    __nv_bfloat16* logits, long ld, const int64_t* __restrict__ targets, float* __restrict__ nll_out, int V,
    float grad_scale, bool write_grad) {
  __shared__ float red_m[kXentThreads / 32], red_s[kXentThreads / 32];
  __shared__ float bc[2];
  const int row = blockIdx.x;
  __nv_bfloat16* lr = logits + long(row) * ld;
  constexpr int kStep = kXentThreads * 8;
  float m = -INFINITY, s = 0.f;
  int c = threadIdx.x * 8;
  for (; c + 3 * kStep < V; c += 4 * kStep) {
    uint4 w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = *reinterpret_cast<const uint4*>(lr + c + k * kStep);
#pragma unroll
    for (int k = 0; k < 4; ++k) xent_absorb8(w[k], m, s);
  }
  for (; c < V; c += kStep) xent_absorb8(*reinterpret_cast<const uint4*>(lr + c), m, s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    xent_merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) { red_m[warp] = m; red_s[warp] = s; }
  __syncthreads();
  if (warp == 0) {
    m = lane < kXentThreads / 32 ? red_m[lane] : -INFINITY;
    s = lane < kXentThreads / 32 ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      xent_merge(m, s, m2, s2);
    }
    if (lane == 0) { bc[0] = m; bc[1] = s; }
  }
  __syncthreads();
  const float lse = bc[0] + __logf(bc[1]);
  const int64_t t = targets[row];
  const bool valid = t >= 0 && t < V;
  if (threadIdx.x == 0 && nll_out) nll_out[row] = valid ? lse - __bfloat162float(lr[t]) : 0.f;
  if (!write_grad) return;
  __syncthreads();  // lr[t] read above before it is overwritten
  const float sc = valid ? grad_scale : 0.f;
  auto grad8 = [&](uint4 w, int col0) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(ws[j]);
      const int col = col0 + 2 * j;
      const float g0 = __expf(f.x - lse) - (col == t ? 1.f : 0.f);
      const float g1 = __expf(f.y - lse) - (col + 1 == t ? 1.f : 0.f);
      o[j] = pack_bf16x2(g0 * sc, g1 * sc);
    }
    *reinterpret_cast<uint4*>(lr + col0) = make_uint4(o[0], o[1], o[2], o[3]);
  };
  c = threadIdx.x * 8;
  for (; c + 3 * kStep < V; c += 4 * kStep) {
    uint4 w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = *reinterpret_cast<const uint4*>(lr + c + k * kStep);
#pragma unroll
    for (int k = 0; k < 4; ++k) grad8(w[k], c + k * kStep);
  }
  for (; c < V; c += kStep) grad8(*reinterpret_cast<const uint4*>(lr + c), c);
}

// logits: (rows, V) bf16 chunk; targets: (rows,) int64 with -1 = ignore.
// nll (optional): (rows,) fp32 per-row loss (0 where ignored).
void softmax_xent(torch::Tensor logits, torch::Tensor targets, c10::optional<torch::Tensor> nll, double grad_scale,
                  bool write_grad) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1, "xent: logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "xent: int64 targets");
  const int rows = int(logits.size(0)), V = int(logits.size(1));
  TORCH_CHECK(targets.numel() == rows, "xent: targets length");
  TORCH_CHECK(V % 8 == 0 && logits.stride(0) % 8 == 0, "xent: V and row stride must be multiples of 8");
  float* np = nullptr;
  if (nll.has_value()) {
    TORCH_CHECK(nll->scalar_type() == at::kFloat && nll->numel() == rows, "xent: nll");
    np = nll->data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(logits.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto lp = reinterpret_cast<__nv_bfloat16*>(logits.data_ptr());
  softmax_xent_kernel<<<rows, kXentThreads, 0, stream>>>(lp, logits.stride(0), targets.data_ptr<int64_t>(), np, V,
                                                        float(grad_scale), write_grad);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "softmax_xent launch failed");
}

// ---- cross-entropy from the lm_head GEMM's softmax partials ----------------------
//
// The lm_head GEMM (mode kLogitsStats) writes, next to the bf16 logits, the
// (max, sum of 2^(v log2e - max)) of every row's 128-column groups. One CTA
// per row combines the row's partials into the log-sum-exp (a 4 KB read for a
// 65536 vocabulary instead of a pass over the 128 KB row), writes the NLL and,
// for training, makes ONE pass over the row that replaces the logits by the
// gradient (softmax - onehot) * scale. Against the two-pass softmax_xent this
// saves one full read of the logits chunk.

__device__ __forceinline__ void lse2_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * ex2_approx(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * ex2_approx(m2 - mm));
  m = mm;
}

__global__ void __launch_bounds__(kXentThreads, 4) xent_stats_kernel(
    __nv_bfloat16* logits, long ld, const float2* __restrict__ stats, int G, const int64_t* __restrict__ targets,
    float* __restrict__ nll_out, int V, float grad_scale, bool write_grad) {
  __shared__ float red_m[kXentThreads / 32], red_s[kXentThreads / 32];
  __shared__ float bc;
  const int row = blockIdx.x;
  __nv_bfloat16* lr = logits + long(row) * ld;
  float m = -INFINITY, s = 0.f;
  for (int g = threadIdx.x; g < G; g += kXentThreads) {
    const float2 p = stats[long(row) * G + g];
    lse2_merge(m, s, p.x, p.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse2_merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) { red_m[warp] = m; red_s[warp] = s; }
  __syncthreads();
  if (warp == 0) {
    m = lane < kXentThreads / 32 ? red_m[lane] : -INFINITY;
    s = lane < kXentThreads / 32 ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      lse2_merge(m, s, m2, s2);
    }
    if (lane == 0) bc = m + __log2f(s);
  }
  __syncthreads();
  constexpr float kLn2 = 0.6931471805599453f, kLog2e = 1.4426950408889634f;
  const float lse2 = bc;
  const int64_t t = targets[row];
  const bool valid = t >= 0 && t < V;
  if (threadIdx.x == 0 && nll_out) nll_out[row] = valid ? lse2 * kLn2 - __bfloat162float(lr[t]) : 0.f;
  if (!write_grad) return;
  __syncthreads();  // lr[t] read above before it is overwritten
  const float sc = valid ? grad_scale : 0.f;
  constexpr int kStep = kXentThreads * 8;
  auto grad8 = [&](uint4 w, int col0) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(ws[j]);
      const int col = col0 + 2 * j;
      const float g0 = ex2_approx(fmaf(f.x, kLog2e, -lse2)) - (col == t ? 1.f : 0.f);
      const float g1 = ex2_approx(fmaf(f.y, kLog2e, -lse2)) - (col + 1 == t ? 1.f : 0.f);
      o[j] = pack_bf16x2(g0 * sc, g1 * sc);
    }
    *reinterpret_cast<uint4*>(lr + col0) = make_uint4(o[0], o[1], o[2], o[3]);
  };
  int c = threadIdx.x * 8;
  for (; c + 3 * kStep < V; c += 4 * kStep) {
    uint4 w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = *reinterpret_cast<const uint4*>(lr + c + k * kStep);
#pragma unroll
    for (int k = 0; k < 4; ++k) grad8(w[k], c + k * kStep);
  }
  for (; c < V; c += kStep) grad8(*reinterpret_cast<const uint4*>(lr + c), c);
}

// logits: (rows, V) bf16 chunk written by gemm_logits_stats; stats: its
// (rows, ceil(V / 128), 2) partials; targets: (rows,) int64, -1 = ignore.
void xent_from_stats(torch::Tensor logits, torch::Tensor stats, torch::Tensor targets,
                     c10::optional<torch::Tensor> nll, double grad_scale, bool write_grad) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1, "xent: logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "xent: int64 targets");
  const int rows = int(logits.size(0)), V = int(logits.size(1));
  const int G = (V + 127) / 128;
  TORCH_CHECK(targets.numel() == rows, "xent: targets length");
  TORCH_CHECK(V % 8 == 0 && logits.stride(0) % 8 == 0, "xent: V and row stride must be multiples of 8");
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.dim() == 3 && stats.size(0) >= rows &&
                  stats.size(1) == G && stats.size(2) == 2,
              "xent: stats must be (rows, ceil(V / 128), 2) fp32");
  float* np = nullptr;
  if (nll.has_value()) {
    TORCH_CHECK(nll->scalar_type() == at::kFloat && nll->numel() == rows, "xent: nll");
    np = nll->data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(logits.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  xent_stats_kernel<<<rows, kXentThreads, 0, stream>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      reinterpret_cast<const float2*>(stats.data_ptr<float>()), G, targets.data_ptr<int64_t>(), np, V,
      float(grad_scale), write_grad);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "xent_from_stats launch failed");
}

// ---- AdamW -----------------------------------------------------------------------

struct AdamParams {
  float lr, b1, b2, eps, wd, scale_m, scale_v, grad_scale;
};

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ work, long n, AdamParams a) {
  const float decay = 1.f - a.lr * a.wd;
  for (long i = (long(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += long(gridDim.x) * blockDim.x * 4) {
    if (i + 4 <= n) {
      float4 pp = *reinterpret_cast<float4*>(p + i), gg = *reinterpret_cast<const float4*>(g + i);
      float4 mm = *reinterpret_cast<float4*>(m + i), vv = *reinterpret_cast<float4*>(v + i);
      float* P = &pp.x; float* G = &gg.x; float* M = &mm.x; float* Vv = &vv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gj = G[j] * a.grad_scale;
        M[j] = M[j] * a.b1 + gj * (1.f - a.b1);
        Vv[j] = Vv[j] * a.b2 + gj * gj * (1.f - a.b2);
        const float mh = M[j] * a.scale_m, vh = Vv[j] * a.scale_v;
        P[j] = P[j] * decay - (mh / (sqrtf(vh) + a.eps)) * a.lr;
      }
      *reinterpret_cast<float4*>(p + i) = pp;
      *reinterpret_cast<float4*>(m + i) = mm;
      *reinterpret_cast<float4*>(v + i) = vv;
      if (work) *reinterpret_cast<uint2*>(work + i) = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
    } else {
      for (long k = i; k < n; ++k) {
        const float gj = g[k] * a.grad_scale;
        m[k] = m[k] * a.b1 + gj * (1.f - a.b1);
        v[k] = v[k] * a.b2 + gj * gj * (1.f - a.b2);
        p[k] = p[k] * decay - ((m[k] * a.scale_m) / (sqrtf(v[k] * a.scale_v) + a.eps)) * a.lr;
        if (work) work[k] = __float2bfloat16(p[k]);
      }
    }
  }
}

void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> work,
                double lr, double b1, double b2, double eps, double wd, int64_t step, double grad_scale) {
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat, "adamw: fp32");
  const long n = p.numel();
  TORCH_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "adamw: sizes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(p.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0,
              "adamw: 16-byte aligned slices");
  __nv_bfloat16* wp = nullptr;
  if (work.has_value()) {
    TORCH_CHECK(work->scalar_type() == at::kBFloat16 && work->numel() == n, "adamw: work copy");
    wp = reinterpret_cast<__nv_bfloat16*>(work->data_ptr());
  }
  AdamParams a;
  a.lr = float(lr); a.b1 = float(b1); a.b2 = float(b2); a.eps = float(eps); a.wd = float(wd);
  a.scale_m = float(1.0 / (1.0 - std::pow(b1, double(step))));
  a.scale_v = float(1.0 / (1.0 - std::pow(b2, double(step))));
  a.grad_scale = float(grad_scale);
  const at::cuda::CUDAGuard guard(p.device());
  const int threads = 256;
  const long blocks = std::min<long>((n / 4 + threads - 1) / threads + 1, 148 * 16);
  adamw_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), wp, n, a);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "adamw launch failed");
}

// ---- sum of squares -----------------------------------------------------------------

__global__ void sumsq_kernel(const float* __restrict__ x, long n, double* out) {
  __shared__ float red[32];
  float s = 0.f;
  for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += long(gridDim.x) * blockDim.x) s += x[i] * x[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    for (int w = 0; w < int(blockDim.x / 32); ++w) t += red[w];
    atomicAdd(out, t);
  }
}

// out (fp64 scalar tensor) += sum(x^2)
void sumsq(torch::Tensor x, torch::Tensor out) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(), "sumsq: fp32");
  TORCH_CHECK(out.scalar_type() == at::kDouble && out.numel() == 1, "sumsq: fp64 scalar");
  const at::cuda::CUDAGuard guard(x.device());
  sumsq_kernel<<<148 * 4, 512, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(), x.numel(),
                                                                       out.data_ptr<double>());
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "sumsq launch failed");
}

}  // namespace nk
