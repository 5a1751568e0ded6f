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

// meta[t] = {p, g, m, v, vmax, numel, dtypes, first_block, f32bits(step_size), f32bits(1 / bc2_sqrt)}
struct AdamArgs {
  const int64_t* meta;
  int ntensors;
  float beta1, beta2, eps, wd, lr;
  int decoupled, amsgrad, maximize;
};

// m / (sqrt(v) / bc2_sqrt + eps) with the hardware approximations (rsqrtf,
// __fdividef; a few ulp) and the host-computed reciprocal of bc2_sqrt: with bf16
// states the update moves 14 bytes per element, and the IEEE divide and square
// root made it ALU-bound rather than HBM-bound. sqrt(v) is v * rsqrt(v) only for
// finite positive v; 0, +inf and NaN pass through unchanged, as sqrtf gives them.
__device__ __forceinline__ float adam_step(float m, float v, float inv_bc2_sqrt, float eps) {
  const float root = (v > 0.f && v < INFINITY) ? v * rsqrtf(v) : v;
  const float den = fmaf(root, inv_bc2_sqrt, eps);
  // __fdividef returns 0 for a denominator above 2^126; IEEE division keeps m / den there.
  return den < 8.5e37f ? __fdividef(m, den) : m / den;
}

// Eight elements of one array as raw 16-byte words (bf16: one word; fp32: two),
// loaded with the streaming (evict-first) hint: every byte is used once.
struct Raw8 {
  uint4 a, b;
};

__device__ __forceinline__ Raw8 ld_raw(const void* base, int dt, long long i) {
  Raw8 r;
  if (dt == 0) {
    const uint4* q = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(base) + i);
    r.a = __ldcs(q);
    r.b = __ldcs(q + 1);
  } else {
    r.a = __ldcs(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + i));
    r.b = make_uint4(0u, 0u, 0u, 0u);
  }
  return r;
}

__device__ __forceinline__ void unpack(const Raw8& r, int dt, float (&v)[8]) {
  const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
  if (dt == 0) {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __uint_as_float(w[k]);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[2 * k] = bf16_bits_to_float((uint16_t)(w[k] & 0xFFFFu));
      v[2 * k + 1] = bf16_bits_to_float((uint16_t)(w[k] >> 16));
    }
  }
}

__device__ __forceinline__ void st_raw(void* base, int dt, long long i, const float (&v)[8]) {
  if (dt == 0) {
    uint4* q = reinterpret_cast<uint4*>(reinterpret_cast<float*>(base) + i);
    __stcs(q, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3])));
    __stcs(q + 1, make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]), __float_as_uint(v[7])));
  } else {
    __stcs(reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + i),
           make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7])));
  }
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

// (256 threads, >= 2 CTAs per SM: room for two runs of raw loads without spills)
// BF16: every array is bf16 and amsgrad is off (the mixed-precision training
// case); the dtype tests then fold away and each run holds 4 words per array.
template <bool BF16>
__global__ void __launch_bounds__(ADAM_THREADS, BF16 ? 3 : 2) adamw_kernel(const AdamArgs a) {
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
  const int dp = BF16 ? 1 : dts & 15, dg = BF16 ? 1 : (dts >> 4) & 15, dm = BF16 ? 1 : (dts >> 8) & 15,
            dv = BF16 ? 1 : (dts >> 12) & 15, dx = (dts >> 16) & 15;
  const bool amsgrad = !BF16 && a.amsgrad;
  const float step_size = __int_as_float((int)m[8]);
  const float inv_bc2_sqrt = __int_as_float((int)m[9]);
  const long long start = (long long)(blk - (int)m[7]) * ADAM_CHUNK;
  const long long end = min(n, start + ADAM_CHUNK);
  if ((dts >> 20) & 1) {
    // Vectorised (every array 16-byte aligned, n % 8 == 0): each thread owns two
    // 8-element runs per iteration and issues all their loads before any math,
    // so 8 (bf16) to 16 (fp32) independent 16-byte loads per thread are in flight.
    constexpr long long STRIDE = ADAM_THREADS * 8;
    for (long long i0 = start + threadIdx.x * 8; i0 < end; i0 += 2 * STRIDE) {
      Raw8 rg[2], rp[2], rm[2], rv[2], rx[2];
      bool live[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const long long i = i0 + u * STRIDE;
        live[u] = i < end;
        if (live[u]) {
          rg[u] = ld_raw(G, dg, i);
          rp[u] = ld_raw(P, dp, i);
          rm[u] = ld_raw(M1, dm, i);
          rv[u] = ld_raw(M2, dv, i);
          if (amsgrad) rx[u] = ld_raw(MX, dx, i);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!live[u]) continue;
        const long long i = i0 + u * STRIDE;
        float g[8], p[8], m1[8], m2[8], mx[8];
        unpack(rg[u], dg, g);
        unpack(rp[u], dp, p);
        unpack(rm[u], dm, m1);
        unpack(rv[u], dv, m2);
        if (amsgrad) unpack(rx[u], dx, mx);
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
          if (amsgrad) {
            mx[k] = fmaxf(mx[k], m2[k]);
            vv = mx[k];
          }
          p[k] = p[k] - step_size * adam_step(m1[k], vv, inv_bc2_sqrt, a.eps);
        }
        st_raw(M1, dm, i, m1);
        st_raw(M2, dv, i, m2);
        if (amsgrad) st_raw(MX, dx, i, mx);
        st_raw(P, dp, i, p);
      }
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
    p = p - step_size * adam_step(m1, vv, inv_bc2_sqrt, a.eps);
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
  // All-bf16 vector tensors (bit 20 vector path, dtype nibbles 1) without amsgrad take the specialised kernel.
  bool all_bf16 = !amsgrad;
  for (int t = 0; t < T && all_bf16; ++t) all_bf16 = (acc[t][6] & 0x10FFFF) == 0x101111;
  if (all_bf16)
    adamw_kernel<true><<<(unsigned)blocks, ADAM_THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  else
    adamw_kernel<false><<<(unsigned)blocks, ADAM_THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  // Keep the pinned staging buffer alive until the copy has been consumed.
  meta.record_stream(at::cuda::getCurrentCUDAStream());
}

}  // namespace dmb
