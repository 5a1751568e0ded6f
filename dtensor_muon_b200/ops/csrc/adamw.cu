// Fused multi-tensor Adam / AdamW (one launch per param group).
//
// Same update as torch.optim.adam's single/multi-tensor paths, which the
// reference calls for its "adam"/"adamw" groups (src/muonium/optim/optim.py:642-694):
//   wd coupled:   g += wd * p          decoupled: p *= 1 - lr * wd
//   m = m + (1 - b1) (g - m);  v = b2 v + (1 - b2) g^2;  [amsgrad: vmax = max(vmax, v)]
//   p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// All arithmetic is fp32; each tensor keeps its own dtype (fp32 or bf16) for
// param, grad and both moments. Per-tensor step-size / bias-correction scalars
// come from the host (the step counters live on the CPU, as in torch).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dmb {
namespace {

constexpr int ADAM_THREADS = 256;
// Elements per CTA. Large enough that the per-CTA tensor lookup (a binary search
// over the meta table in global memory) is amortised; on the 1.05 B-param
// embedding/head update this took the kernel from 6.98 to 6.72 ms.
constexpr int ADAM_CHUNK = 65536;
constexpr int META = 10;          // int64 words per tensor

// meta[t] = {p, g, m, v, vmax, numel, dtypes, first_block, f32bits(step_size), f32bits(bc2_sqrt)}
struct AdamArgs {
  const int64_t* meta;
  int ntensors;
  float beta1, beta2, eps, wd, lr;
  int decoupled, amsgrad, maximize;
};

// m / (sqrt(v) / bc2_sqrt + eps) with the hardware approximations (rsqrtf,
// __fdividef; a few ulp): with bf16 states the update moves 14 bytes per element,
// and the IEEE divide and square root made it ALU-bound rather than HBM-bound.
__device__ __forceinline__ float adam_step(float m, float v, float bc2_sqrt, float eps) {
  const float root = v > 0.f ? v * rsqrtf(v) : 0.f;
  return __fdividef(m, root / bc2_sqrt + eps);
}

__device__ __forceinline__ float ld(const void* p, int dt, long long i) {
  return dt == 0 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void st(void* p, int dt, long long i, float v) {
  if (dt == 0)
    reinterpret_cast<float*>(p)[i] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// (256 threads, >= 4 CTAs per SM: caps registers so enough loads are in flight)
__global__ void __launch_bounds__(ADAM_THREADS, 4) adamw_kernel(const AdamArgs a) {
  // Find the tensor this CTA works on (meta[t][7] = first block index, ascending).
  int lo = 0, hi = a.ntensors - 1;
  const int blk = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.meta[(long long)mid * META + 7] <= blk)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int64_t* m = a.meta + (long long)lo * META;
  void* P = reinterpret_cast<void*>(m[0]);
  const void* G = reinterpret_cast<const void*>(m[1]);
  void* M1 = reinterpret_cast<void*>(m[2]);
  void* M2 = reinterpret_cast<void*>(m[3]);
  void* MX = reinterpret_cast<void*>(m[4]);
  const long long n = m[5];
  const int dts = (int)m[6];
  const int dp = dts & 15, dg = (dts >> 4) & 15, dm = (dts >> 8) & 15, dv = (dts >> 12) & 15, dx = (dts >> 16) & 15;
  const float step_size = __int_as_float((int)m[8]);
  const float bc2_sqrt = __int_as_float((int)m[9]);
  const long long start = (long long)(blk - (int)m[7]) * ADAM_CHUNK;
  const long long end = min(n, start + ADAM_CHUNK);
  if ((dts >> 20) & 1) {
    // Vectorised: every array 16-byte aligned and n % 8 == 0.
    for (long long i = start + threadIdx.x * 8; i < end; i += ADAM_THREADS * 8) {
      float g[8], p[8], m1[8], m2[8], mx[8];
      load8(G, dg, i, g);
      load8(P, dp, i, p);
      load8(M1, dm, i, m1);
      load8(M2, dv, i, m2);
      if (a.amsgrad) load8(MX, dx, i, mx);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float gk = a.maximize ? -g[k] : g[k];
        if (a.wd != 0.f) {
          if (a.decoupled)
            p[k] *= 1.f - a.lr * a.wd;
          else
            gk = fmaf(a.wd, p[k], gk);
        }
        m1[k] = fmaf(1.f - a.beta1, gk - m1[k], m1[k]);
        m2[k] = fmaf(a.beta2, m2[k], (1.f - a.beta2) * gk * gk);
        float vv = m2[k];
        if (a.amsgrad) {
          mx[k] = fmaxf(mx[k], m2[k]);
          vv = mx[k];
        }
        p[k] = p[k] - step_size * adam_step(m1[k], vv, bc2_sqrt, a.eps);
      }
      store8(M1, dm, i, m1);
      store8(M2, dv, i, m2);
      if (a.amsgrad) store8(MX, dx, i, mx);
      store8(P, dp, i, p);
    }
    return;
  }
  for (long long i = start + threadIdx.x; i < end; i += ADAM_THREADS) {
    float g = ld(G, dg, i);
    if (a.maximize) g = -g;
    float p = ld(P, dp, i);
    if (a.wd != 0.f) {
      if (a.decoupled)
        p *= 1.f - a.lr * a.wd;
      else
        g = fmaf(a.wd, p, g);
    }
    float m1 = ld(M1, dm, i);
    m1 = fmaf(1.f - a.beta1, g - m1, m1);
    float m2 = ld(M2, dv, i);
    m2 = fmaf(a.beta2, m2, (1.f - a.beta2) * g * g);
    st(M1, dm, i, m1);
    st(M2, dv, i, m2);
    float vv = m2;
    if (a.amsgrad) {
      vv = fmaxf(ld(MX, dx, i), m2);
      st(MX, dx, i, vv);
    }
    p = p - step_size * adam_step(m1, vv, bc2_sqrt, a.eps);
    st(P, dp, i, p);
  }
}

}  // namespace

// meta: CPU int64 [T, 10] as described above (first_block filled here).
void adamw_multi(at::Tensor meta_cpu, double lr, double beta1, double beta2, double eps, double wd, bool decoupled,
                 bool amsgrad, bool maximize, const at::Device& device) {
  TORCH_CHECK(meta_cpu.device().is_cpu() && meta_cpu.scalar_type() == at::kLong && meta_cpu.dim() == 2 &&
              meta_cpu.size(1) == META);
  const int T = meta_cpu.size(0);
  if (T == 0) return;
  auto acc = meta_cpu.accessor<int64_t, 2>();
  int64_t blocks = 0;
  for (int t = 0; t < T; ++t) {
    acc[t][7] = blocks;
    blocks += (acc[t][5] + ADAM_CHUNK - 1) / ADAM_CHUNK;
  }
  if (blocks == 0) return;
  TORCH_CHECK(blocks < (1ll << 31));
  const at::cuda::CUDAGuard guard(device);
  auto meta = meta_cpu.pin_memory().to(device, /*non_blocking=*/true);
  AdamArgs a{};
  a.meta = meta.data_ptr<int64_t>();
  a.ntensors = T;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.wd = wd;
  a.lr = lr;
  a.decoupled = decoupled;
  a.amsgrad = amsgrad;
  a.maximize = maximize;
  adamw_kernel<<<(unsigned)blocks, ADAM_THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  // Keep the pinned staging buffer alive until the copy has been consumed.
  meta.record_stream(at::cuda::getCurrentCUDAStream());
}

}  // namespace dmb
