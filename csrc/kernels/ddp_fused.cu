// Fused data-parallel optimizer step over NVLink peer memory:
//   reduce-scatter of the fp32 gradients + AdamW on this rank's shard +
//   all-gather of the updated bf16 working weights, in ONE kernel.
//
// Every rank owns a contiguous shard of the flat parameter buffer. For each
// 4-element vector of its shard a thread
//   1. loads the gradient from every rank's gradient buffer (peer pointers
//      into NVLink-mapped symmetric memory; plain ld.global, no TMA),
//   2. scales the sum by grad_scale / world (the DDP mean, plus the SFT
//      valid-count correction) and accumulates its square for the gradient norm,
//   3. runs the candle AdamW update of its parameter group on the local fp32
//      master, m and v,
//   4. stores the new bf16 weights into every rank's working-copy buffer.
// The transfer of one vector overlaps the math of the others across the
// whole grid; there is no NCCL call.
//
// Cross-GPU ordering uses a signal-pad barrier kernel before (all gradients
// complete) and after (all peers finished reading my gradients and writing my
// weights). Its waits are bounded: on timeout it records an error code and
// returns instead of hanging.
//
// With NVLink SHARP available (multicast objects bound to the symmetric
// buffers) a second kernel does the same step with multimem.ld_reduce /
// multimem.st through the switch instead of per-peer loads and stores.
//
// Replaces rs-nanogpt's per-parameter NCCL AllReduce(Avg) followed by
// candle's AdamW (src/train/dist.rs:327-347, src/train/optim.rs:146-150).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "status.h"

namespace nk {

constexpr int kMaxWorld = 8;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// pads[p] = signal pad of rank p; slot q of a pad holds the epoch rank q reached.
__global__ void ddp_barrier_kernel(uint32_t* const* pads, int rank, int world, uint32_t epoch, int* err) {
  const int p = threadIdx.x;
  if (p >= world) return;
  __threadfence_system();  // everything this rank wrote before is visible first
  st_release_sys(pads[p] + rank, epoch);
  const uint32_t* mine = pads[rank] + p;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (int32_t(ld_acquire_sys(mine) - epoch) < 0) {
    if ((++spins & 1023) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicCAS(err, 0, kErrTimeoutOther);
      return;
    }
  }
}

struct DdpGroup {
  long lo, hi;  // element range of the group
  float lr, b1, b2, eps, wd, scale_m, scale_v;
};

struct DdpArgs {
  const float* const* grads;      // [world] peer gradient buffers
  __nv_bfloat16* const* works;    // [world] peer bf16 working-copy buffers
  float* master;
  float* m;                       // AdamW moments of this rank's shard only:
  float* v;                       //   element i lives at m[i - mv_base]
  long shard_lo, shard_hi;        // this rank's elements, multiples of 4
  long mv_base;
  DdpGroup groups[3];
  int ngroups, world;
  float grad_scale;               // multiplies the summed gradient (includes 1/world)
  double* sumsq;                  // += sum of squared reduced gradients (this shard)
};

template <int W>
__global__ void __launch_bounds__(256) ddp_rs_adam_ag_kernel(const DdpArgs a) {
  __shared__ float red[8];
  float ss = 0.f;
  const long n4 = (a.shard_hi - a.shard_lo) / 4;
  for (long k = long(blockIdx.x) * blockDim.x + threadIdx.x; k < n4; k += long(gridDim.x) * blockDim.x) {
    const long i = a.shard_lo + 4 * k;
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < W; ++p) {
      const float4 x = *reinterpret_cast<const float4*>(a.grads[p] + i);
      g.x += x.x; g.y += x.y; g.z += x.z; g.w += x.w;
    }
    float gv[4] = {g.x * a.grad_scale, g.y * a.grad_scale, g.z * a.grad_scale, g.w * a.grad_scale};
    int gi = 0;
    while (gi + 1 < a.ngroups && i >= a.groups[gi].hi) ++gi;
    const DdpGroup& G = a.groups[gi];
    const bool in_group = i >= G.lo && i < G.hi;  // padding between groups stays untouched
    float4 pp = *reinterpret_cast<float4*>(a.master + i);
    float* const mp = a.m + (i - a.mv_base);
    float* const vp = a.v + (i - a.mv_base);
    float4 mm = *reinterpret_cast<float4*>(mp);
    float4 vv = *reinterpret_cast<float4*>(vp);
    float* P = &pp.x;
    float* M = &mm.x;
    float* V = &vv.x;
    if (in_group) {
      const float decay = 1.f - G.lr * G.wd;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ss += gv[j] * gv[j];
        M[j] = M[j] * G.b1 + gv[j] * (1.f - G.b1);
        V[j] = V[j] * G.b2 + gv[j] * gv[j] * (1.f - G.b2);
        P[j] = P[j] * decay - ((M[j] * G.scale_m) / (sqrtf(V[j] * G.scale_v) + G.eps)) * G.lr;
      }
      *reinterpret_cast<float4*>(a.master + i) = pp;
      *reinterpret_cast<float4*>(mp) = mm;
      *reinterpret_cast<float4*>(vp) = vv;
    }
    const uint2 w = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
#pragma unroll
    for (int p = 0; p < W; ++p) *reinterpret_cast<uint2*>(a.works[p] + i) = w;
  }
  if (a.sumsq) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0;
      for (int w = 0; w < int(blockDim.x / 32); ++w) t += red[w];
      atomicAdd(a.sumsq, t);
    }
  }
}

// NVLS (NVLink SHARP) variant: the switch does the reduction and the
// replication. For each 4-element vector of this rank's shard one
// multimem.ld_reduce on the gradient buffer's multicast address returns the
// sum over all ranks (inbound traffic: the shard once, instead of world - 1
// peer copies of it), and one multimem.st on the working-copy buffer's
// multicast address writes the new bf16 weights into every rank's copy
// (outbound: the shard once). Rank order of the sum is the switch's; the
// AdamW math is the same as in the P2P kernel.
__device__ __forceinline__ float4 multimem_ld_add_v4(const float* mc) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
__device__ __forceinline__ void multimem_st_v2(__nv_bfloat16* mc, uint2 v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(mc), "f"(__uint_as_float(v.x)),
               "f"(__uint_as_float(v.y))
               : "memory");
}
// Accesses through the multicast address alias the unicast buffers that the
// other kernels use; order the two views.
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

__global__ void __launch_bounds__(256) ddp_rs_adam_ag_nvls_kernel(const DdpArgs a, const float* mc_grad,
                                                                   __nv_bfloat16* mc_work) {
  __shared__ float red[8];
  fence_proxy_alias();
  float ss = 0.f;
  const long n4 = (a.shard_hi - a.shard_lo) / 4;
  for (long k = long(blockIdx.x) * blockDim.x + threadIdx.x; k < n4; k += long(gridDim.x) * blockDim.x) {
    const long i = a.shard_lo + 4 * k;
    const float4 g = multimem_ld_add_v4(mc_grad + i);
    float gv[4] = {g.x * a.grad_scale, g.y * a.grad_scale, g.z * a.grad_scale, g.w * a.grad_scale};
    int gi = 0;
    while (gi + 1 < a.ngroups && i >= a.groups[gi].hi) ++gi;
    const DdpGroup& G = a.groups[gi];
    const bool in_group = i >= G.lo && i < G.hi;
    float4 pp = *reinterpret_cast<float4*>(a.master + i);
    float* const mp = a.m + (i - a.mv_base);
    float* const vp = a.v + (i - a.mv_base);
    float4 mm = *reinterpret_cast<float4*>(mp);
    float4 vv = *reinterpret_cast<float4*>(vp);
    float* P = &pp.x;
    float* M = &mm.x;
    float* V = &vv.x;
    if (in_group) {
      const float decay = 1.f - G.lr * G.wd;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ss += gv[j] * gv[j];
        M[j] = M[j] * G.b1 + gv[j] * (1.f - G.b1);
        V[j] = V[j] * G.b2 + gv[j] * gv[j] * (1.f - G.b2);
        P[j] = P[j] * decay - ((M[j] * G.scale_m) / (sqrtf(V[j] * G.scale_v) + G.eps)) * G.lr;
      }
      *reinterpret_cast<float4*>(a.master + i) = pp;
      *reinterpret_cast<float4*>(mp) = mm;
      *reinterpret_cast<float4*>(vp) = vv;
    }
    multimem_st_v2(mc_work + i, make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w)));
  }
  fence_proxy_alias();
  if (a.sumsq) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0;
      for (int w = 0; w < int(blockDim.x / 32); ++w) t += red[w];
      atomicAdd(a.sumsq, t);
    }
  }
}

void ddp_barrier(int64_t pads_dev, int64_t rank, int64_t world, int64_t epoch) {
  TORCH_CHECK(world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world, "ddp_barrier: bad world");
  ddp_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<uint32_t* const*>(pads_dev), int(rank), int(world), uint32_t(epoch), error_word());
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "ddp_barrier launch failed");
}

// groups: (n_groups, 9) float64 rows [lo, hi, lr, b1, b2, eps, wd, scale_m, scale_v]
// m, v: the moments of elements [mv_base, mv_base + m.numel()) (a shard-sized
// slice, or the whole buffer with mv_base 0).
void ddp_rs_adam_ag(int64_t grads_dev, int64_t works_dev, int64_t world, torch::Tensor master, torch::Tensor m,
                    torch::Tensor v, int64_t shard_lo, int64_t shard_hi, torch::Tensor groups, double grad_scale,
                    c10::optional<torch::Tensor> sumsq, int64_t mv_base, int64_t mc_grad, int64_t mc_work,
                    int64_t max_ctas) {
  TORCH_CHECK(world >= 1 && world <= kMaxWorld, "ddp: world size 1..8");
  TORCH_CHECK(master.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat,
              "ddp: fp32 state");
  TORCH_CHECK(shard_lo % 4 == 0 && shard_hi % 4 == 0 && shard_lo <= shard_hi && shard_hi <= master.numel(),
              "ddp: shard bounds must be multiples of 4 inside the buffer");
  TORCH_CHECK(m.numel() == v.numel() && m.is_contiguous() && v.is_contiguous() && mv_base % 4 == 0 &&
                  shard_lo >= mv_base && (shard_hi - mv_base <= m.numel() || shard_hi == shard_lo),
              "ddp: the moment slices must cover the shard");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(m.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(v.data_ptr()) % 16 == 0,
              "ddp: moment slices must be 16-byte aligned");
  TORCH_CHECK(groups.dtype() == at::kDouble && groups.dim() == 2 && groups.size(1) == 9 && groups.size(0) <= 3,
              "ddp: groups table");
  DdpArgs a{};
  a.grads = reinterpret_cast<const float* const*>(grads_dev);
  a.works = reinterpret_cast<__nv_bfloat16* const*>(works_dev);
  a.master = master.data_ptr<float>();
  a.m = m.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.shard_lo = shard_lo;
  a.shard_hi = shard_hi;
  a.mv_base = mv_base;
  a.world = int(world);
  a.grad_scale = float(grad_scale);
  auto g = groups.accessor<double, 2>();
  a.ngroups = int(groups.size(0));
  for (int i = 0; i < a.ngroups; ++i) {
    a.groups[i] = DdpGroup{long(g[i][0]), long(g[i][1]), float(g[i][2]), float(g[i][3]), float(g[i][4]),
                           float(g[i][5]), float(g[i][6]), float(g[i][7]), float(g[i][8])};
    TORCH_CHECK(i == 0 || a.groups[i].lo >= a.groups[i - 1].hi, "ddp: groups must be sorted and disjoint");
  }
  a.sumsq = nullptr;
  if (sumsq.has_value()) {
    TORCH_CHECK(sumsq->scalar_type() == at::kDouble && sumsq->numel() == 1, "ddp: sumsq");
    a.sumsq = sumsq->data_ptr<double>();
  }
  const at::cuda::CUDAGuard guard(master.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const long n4 = (shard_hi - shard_lo) / 4;
  const long cap = max_ctas > 0 ? max_ctas : 148 * 8;
  const int blocks = int(std::max<long>(1, std::min<long>((n4 + 255) / 256, cap)));
  if (mc_grad != 0 && mc_work != 0) {
    TORCH_CHECK(mc_grad % 16 == 0 && mc_work % 16 == 0, "ddp: multicast addresses must be 16-byte aligned");
    ddp_rs_adam_ag_nvls_kernel<<<blocks, 256, 0, stream>>>(a, reinterpret_cast<const float*>(mc_grad),
                                                           reinterpret_cast<__nv_bfloat16*>(mc_work));
    TORCH_CHECK(cudaGetLastError() == cudaSuccess, "ddp_rs_adam_ag (NVLS) launch failed");
    return;
  }
  switch (world) {
    case 1: ddp_rs_adam_ag_kernel<1><<<blocks, 256, 0, stream>>>(a); break;
    case 2: ddp_rs_adam_ag_kernel<2><<<blocks, 256, 0, stream>>>(a); break;
    case 3: ddp_rs_adam_ag_kernel<3><<<blocks, 256, 0, stream>>>(a); break;
    case 4: ddp_rs_adam_ag_kernel<4><<<blocks, 256, 0, stream>>>(a); break;
    case 5: ddp_rs_adam_ag_kernel<5><<<blocks, 256, 0, stream>>>(a); break;
    case 6: ddp_rs_adam_ag_kernel<6><<<blocks, 256, 0, stream>>>(a); break;
    case 7: ddp_rs_adam_ag_kernel<7><<<blocks, 256, 0, stream>>>(a); break;
    default: ddp_rs_adam_ag_kernel<8><<<blocks, 256, 0, stream>>>(a); break;
  }
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "ddp_rs_adam_ag launch failed");
}

}  // namespace nk
