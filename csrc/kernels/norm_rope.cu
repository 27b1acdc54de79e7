// Row-wise fused kernels of the transformer block, all bf16 in / bf16 out
// with fp32 arithmetic:
//   * rmsnorm_fwd/bwd      y = x / sqrt(mean(x^2) + eps), no gain
//                          (rs-nanogpt src/model/rms_norm.rs:3-8)
//   * rope_qknorm_fwd/bwd  in place on the q and k parts of the fused QKV
//                          GEMM output: half-split RoPE at each token's
//                          position, then RMSNorm over head_dim
//                          (src/model/rope.rs:48-72, src/model/attention.rs:91-92)
// One warp per row; 16-byte vector loads. Rows are `C` wide with C % 256 == 0
// for rmsnorm (8 bf16 per lane per step) and head_dim == 128 for rope.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace nk {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 w = *reinterpret_cast<const uint4*>(p);
  uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = unpack_bf16x2(ws[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                            pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- RMSNorm ---------------------------------------------------------------

template <int VPT>  // 8-element vectors per lane
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                   float* __restrict__ rstd, int rows, int C, long ldx, long ldy, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) {
      load8(xr + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = warp_sum(ss);
  // The reference divides by the bf16-rounded denominator.
  const float denom = __bfloat162float(__float2bfloat16(sqrtf(ss / C + eps)));
  const float r = 1.f / denom;
  if (lane == 0 && rstd) rstd[row] = r;
  __nv_bfloat16* yr = y + row * ldy;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * r;  // within 1 fp32 ulp of v / denom
      store8(yr + c, o);
    }
  }
}

// dx = r * (dy - y * mean(dy * y)),  y = x * r  (r = 1/denom, saved).
// With `accum`, dx is added to the existing contents of dx (residual stream).
template <int VPT>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                                   const float* __restrict__ rstd, __nv_bfloat16* dx, int rows, int C, bool accum) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const long off = long(row) * C;
  const float r = rstd[row];
  // All three inputs of the row (x, dy and, when accumulating, dx) are
  // loaded up front as packed bf16 so their latencies overlap.
  uint4 xw[VPT], gw[VPT], dw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) {
      xw[i] = *reinterpret_cast<const uint4*>(x + off + c);
      gw[i] = *reinterpret_cast<const uint4*>(dy + off + c);
      if (accum) dw[i] = *reinterpret_cast<const uint4*>(dx + off + c);
    }
  }
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) {
      const uint32_t xs[4] = {xw[i].x, xw[i].y, xw[i].z, xw[i].w}, gs[4] = {gw[i].x, gw[i].y, gw[i].z, gw[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 xf = unpack_bf16x2(xs[j]), gf = unpack_bf16x2(gs[j]);
        dot += gf.x * xf.x + gf.y * xf.y;
      }
    }
  }
  dot = warp_sum(dot) * r * r / C;  // r^2 * mean(dy * x)
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) {
      const uint32_t xs[4] = {xw[i].x, xw[i].y, xw[i].z, xw[i].w}, gs[4] = {gw[i].x, gw[i].y, gw[i].z, gw[i].w};
      const uint32_t ds[4] = {dw[i].x, dw[i].y, dw[i].z, dw[i].w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 xf = unpack_bf16x2(xs[j]), gf = unpack_bf16x2(gs[j]);
        float g0 = r * (gf.x - xf.x * dot), g1 = r * (gf.y - xf.y * dot);
        if (accum) {
          const float2 df = unpack_bf16x2(ds[j]);
          g0 += df.x;
          g1 += df.y;
        }
        o[j] = pack_bf16x2(g0, g1);
      }
      *reinterpret_cast<uint4*>(dx + off + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

void rmsnorm_fwd(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> rstd, double eps) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16, "rmsnorm: bf16");
  TORCH_CHECK(x.dim() == 2 && y.sizes() == x.sizes() && x.stride(1) == 1 && y.stride(1) == 1, "rmsnorm: 2-D rows");
  const int rows = int(x.size(0)), C = int(x.size(1));
  TORCH_CHECK(C % 8 == 0 && C <= 8 * 32 * 8, "rmsnorm: C must be a multiple of 8 and <= 2048");
  TORCH_CHECK(x.stride(0) % 8 == 0 && y.stride(0) % 8 == 0, "rmsnorm: 16-byte aligned rows");
  float* r = nullptr;
  if (rstd.has_value()) {
    TORCH_CHECK(rstd->scalar_type() == at::kFloat && rstd->numel() == rows, "rmsnorm: rstd");
    r = rstd->data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int warps = 8, grid = (rows + warps - 1) / warps;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  // Vectors of 8 per lane: the template bound is the smallest that covers C,
  // so no registers are spent on lanes that never load.
  const int vpt = (C / 8 + 31) / 32;
#define RMS_FWD(N) rmsnorm_fwd_kernel<N><<<grid, warps * 32, 0, stream>>>(xp, yp, r, rows, C, x.stride(0), \
                                                                             y.stride(0), float(eps))
  if (vpt <= 2) RMS_FWD(2);
  else if (vpt <= 3) RMS_FWD(3);
  else if (vpt <= 4) RMS_FWD(4);
  else if (vpt <= 5) RMS_FWD(5);
  else if (vpt <= 6) RMS_FWD(6);
  else RMS_FWD(8);
#undef RMS_FWD
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "rmsnorm_fwd launch failed");
}

void rmsnorm_bwd(torch::Tensor x, torch::Tensor dy, torch::Tensor rstd, torch::Tensor dx, bool accum) {
  TORCH_CHECK(x.is_contiguous() && dy.is_contiguous() && dx.is_contiguous(), "rmsnorm_bwd: contiguous");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && dy.scalar_type() == at::kBFloat16 &&
                  dx.scalar_type() == at::kBFloat16, "rmsnorm_bwd: bf16");
  const int rows = int(x.size(0)), C = int(x.size(1));
  TORCH_CHECK(C % 8 == 0 && C <= 2048 && rstd.numel() == rows, "rmsnorm_bwd: shape");
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  // Two warps per block: small blocks fit in the registers a running GEMM
  // leaves free, so the training backward can run this next to a
  // weight-gradient GEMM on another stream.
  const int warps = 2, grid = (rows + warps - 1) / warps;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto gp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto dp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  const int vpt = (C / 8 + 31) / 32;
#define RMS_BWD(N) rmsnorm_bwd_kernel<N><<<grid, warps * 32, 0, stream>>>(xp, gp, rstd.data_ptr<float>(), dp, rows, \
                                                                             C, accum)
  if (vpt <= 2) RMS_BWD(2);
  else if (vpt <= 3) RMS_BWD(3);
  else if (vpt <= 4) RMS_BWD(4);
  else if (vpt <= 5) RMS_BWD(5);
  else if (vpt <= 6) RMS_BWD(6);
  else RMS_BWD(8);
#undef RMS_BWD
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "rmsnorm_bwd launch failed");
}

// ---- RoPE + QK-norm (head_dim 128) -----------------------------------------
// qkv: (tokens, 3C) rows; token index = b * T + t, position = t0 + t.
// Lane l owns elements [4l, 4l+4) of the head; its RoPE partner elements
// (i +- 64) live in lane l ^ 16.

__global__ void rope_qknorm_fwd_kernel(__nv_bfloat16* qkv, float* __restrict__ rstd, const float* __restrict__ cos_t,
                                       const float* __restrict__ sin_t, int tokens, int T, int t0, int H, int C,
                                       float eps) {
  const int item = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;  // (token, part, head)
  const int lane = threadIdx.x % 32;
  if (item >= tokens * 2 * H) return;
  const int token = item / (2 * H), rem = item % (2 * H), part = rem / H, h = rem % H;
  const int pos = t0 + token % T;
  __nv_bfloat16* p = qkv + long(token) * 3 * C + part * C + h * 128 + lane * 4;
  uint2 w = *reinterpret_cast<uint2*>(p);
  float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
  float x[4] = {a.x, a.y, b.x, b.y};
  float o[4];
  const bool first = lane < 16;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[j], 16);
    const int i = (lane & 15) * 4 + j;  // frequency index in [0, 64)
    const float c = cos_t[pos * 64 + i], s = sin_t[pos * 64 + i];
    // y1 = x1 c + x2 s ; y2 = x2 c - x1 s
    o[j] = first ? x[j] * c + partner * s : x[j] * c - partner * s;
  }
  float ss = o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3];
  ss = warp_sum(ss);
  const float denom = __bfloat162float(__float2bfloat16(sqrtf(ss / 128.f + eps)));
  if (lane == 0) rstd[item] = 1.f / denom;
  *reinterpret_cast<uint2*>(p) =
      make_uint2(pack_bf16x2(o[0] / denom, o[1] / denom), pack_bf16x2(o[2] / denom, o[3] / denom));
}

// Backward through y = rms(rope(x)), given y (the forward output, stored in
// place in qkv) and dy (in dqkv); writes dx over dy.
__global__ void rope_qknorm_bwd_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* dqkv,
                                       const float* __restrict__ rstd, const float* __restrict__ cos_t,
                                       const float* __restrict__ sin_t, int tokens, int T, int H, int C) {
  const int item = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (item >= tokens * 2 * H) return;
  const int token = item / (2 * H), rem = item % (2 * H), part = rem / H, h = rem % H;
  const int pos = token % T;
  const long off = long(token) * 3 * C + part * C + h * 128 + lane * 4;
  uint2 wy = *reinterpret_cast<const uint2*>(qkv + off);
  uint2 wg = *reinterpret_cast<const uint2*>(dqkv + off);
  float2 y0 = unpack_bf16x2(wy.x), y1 = unpack_bf16x2(wy.y), g0 = unpack_bf16x2(wg.x), g1 = unpack_bf16x2(wg.y);
  float y[4] = {y0.x, y0.y, y1.x, y1.y}, g[4] = {g0.x, g0.y, g1.x, g1.y};
  const float r = rstd[item];
  float dot = warp_sum(y[0] * g[0] + y[1] * g[1] + y[2] * g[2] + y[3] * g[3]) / 128.f;
  float dr[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) dr[j] = r * (g[j] - y[j] * dot);  // grad w.r.t. the rotated vector
  const bool first = lane < 16;
  float dx[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float partner = __shfl_xor_sync(0xffffffffu, dr[j], 16);
    const int i = (lane & 15) * 4 + j;
    const float c = cos_t[pos * 64 + i], s = sin_t[pos * 64 + i];
    // dx1 = dy1 c - dy2 s ; dx2 = dy1 s + dy2 c
    dx[j] = first ? dr[j] * c - partner * s : partner * s + dr[j] * c;
  }
  *reinterpret_cast<uint2*>(dqkv + off) = make_uint2(pack_bf16x2(dx[0], dx[1]), pack_bf16x2(dx[2], dx[3]));
}

void rope_qknorm_fwd(torch::Tensor qkv, torch::Tensor rstd, torch::Tensor cos_t, torch::Tensor sin_t, int64_t T,
                     int64_t t0, int64_t H, double eps) {
  TORCH_CHECK(qkv.is_contiguous() && qkv.scalar_type() == at::kBFloat16, "rope: contiguous bf16 qkv");
  const int C = int(qkv.size(1) / 3), tokens = int(qkv.size(0));
  TORCH_CHECK(C == H * 128, "rope: head_dim must be 128");
  TORCH_CHECK(rstd.numel() >= tokens * 2 * H && cos_t.size(1) == 64, "rope: shapes");
  TORCH_CHECK(t0 + T <= cos_t.size(0), "rope: positions beyond the table");
  const at::cuda::CUDAGuard guard(qkv.device());
  const int items = tokens * 2 * int(H), warps = 8;
  rope_qknorm_fwd_kernel<<<(items + warps - 1) / warps, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), rstd.data_ptr<float>(), cos_t.data_ptr<float>(),
      sin_t.data_ptr<float>(), tokens, int(T), int(t0), int(H), C, float(eps));
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "rope_qknorm_fwd launch failed");
}

void rope_qknorm_bwd(torch::Tensor qkv, torch::Tensor dqkv, torch::Tensor rstd, torch::Tensor cos_t,
                     torch::Tensor sin_t, int64_t T, int64_t H) {
  TORCH_CHECK(qkv.is_contiguous() && dqkv.is_contiguous(), "rope_bwd: contiguous");
  const int C = int(qkv.size(1) / 3), tokens = int(qkv.size(0));
  TORCH_CHECK(C == H * 128, "rope_bwd: head_dim must be 128");
  const at::cuda::CUDAGuard guard(qkv.device());
  const int items = tokens * 2 * int(H), warps = 8;
  rope_qknorm_bwd_kernel<<<(items + warps - 1) / warps, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
      rstd.data_ptr<float>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), tokens, int(T), int(H), C);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "rope_qknorm_bwd launch failed");
}

}  // namespace nk
