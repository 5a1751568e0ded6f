// Block-scaled low-precision momentum for MuonLP (Muon8bit / Muon4bit / MuonFp8).
//
// The reference allocates torchao OptimState8bit / OptimState4bit /
// OptimStateFp8 buffers (src/muonium/optim/optim_lp.py:118-133) but cannot step
// them (tests/optim/test_optim_lp.py:211-222). Here the state is stepped by one
// fused kernel per tensor:
//   dequantize block -> m = beta * m + g -> g' = g + beta * m (Nesterov) ->
//   write g' (bf16, input of the orthogonalisation) -> requantize block.
// Formats (one fp32 scale per `block` consecutive elements):
//   0  fp8 e4m3     code = e4m3(x / s), s = absmax / 448
//   1  8-bit map    code = argmin_k |qmap[k] - x / s|, s = absmax   (256-entry map)
//   2  4-bit map    same with a 16-entry map, two codes per byte (low nibble first)
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dmb {
namespace {

constexpr int LP_THREADS = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < LP_THREADS / 32; ++i) m = fmaxf(m, red[i]);
    red[0] = m;
  }
  __syncthreads();
  return red[0];
}

// Nearest entry of a sorted map (binary search, ties to the lower index).
__device__ __forceinline__ int nearest_code(const float* qmap, int n, float x) {
  int lo = 0, hi = n - 1;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (qmap[mid] <= x)
      lo = mid;
    else
      hi = mid;
  }
  return (fabsf(qmap[hi] - x) < fabsf(x - qmap[lo])) ? hi : lo;
}

__device__ __forceinline__ float decode(const uint8_t* codes, int fmt, long long i, const float* qmap) {
  if (fmt == 0) {
    __nv_fp8_e4m3 c;
    c.__x = codes[i];
    return float(c);
  }
  if (fmt == 1) return qmap[codes[i]];
  const uint8_t byte = codes[i >> 1];
  return qmap[(i & 1) ? (byte >> 4) : (byte & 15)];
}

struct LpArgs {
  uint8_t* codes;
  float* scale;
  const float* qmap_g;
  int fmt, qn;
  long long n;
  int block;
  const void* grad;
  int grad_dtype;
  __nv_bfloat16* gout;  // Nesterov/momentum output, or nullptr
  float momentum;
  int nesterov, maximize, has_grad;
  float* dequant_out;   // optional fp32 dequantised copy (after the update)
  const float* quant_in;  // quantise-only mode: fp32 source
};

// One CTA per quantisation block. Each thread keeps its elements in registers
// between the absmax reduction and the requantisation.
__global__ void __launch_bounds__(LP_THREADS) lp_step_kernel(const LpArgs a) {
  __shared__ float qmap[256];
  __shared__ float red[LP_THREADS / 32];
  for (int i = threadIdx.x; i < a.qn; i += LP_THREADS) qmap[i] = a.qmap_g[i];
  __syncthreads();
  const long long b0 = (long long)blockIdx.x * a.block;
  const int len = (int)min((long long)a.block, a.n - b0);
  constexpr int PER = 16;  // supports block <= LP_THREADS * PER = 4096
  float vals[PER];
  float amax = 0.f;
  const float s_old = a.quant_in ? 0.f : a.scale[blockIdx.x];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int e = threadIdx.x + k * LP_THREADS;
    float m = 0.f;
    if (e < len) {
      const long long i = b0 + e;
      if (a.quant_in) {
        m = a.quant_in[i];
      } else {
        m = decode(a.codes, a.fmt, i, qmap) * s_old;
        if (a.has_grad) {
          float g = a.grad_dtype == 0 ? reinterpret_cast<const float*>(a.grad)[i]
                                      : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.grad)[i]);
          if (a.maximize) g = -g;
          m = fmaf(m, a.momentum, g);
          if (a.gout) a.gout[i] = __float2bfloat16_rn(a.nesterov ? fmaf(m, a.momentum, g) : m);
        }
      }
      if (a.dequant_out) a.dequant_out[i] = m;
    }
    vals[k] = m;
    amax = fmaxf(amax, fabsf(m));
  }
  if (!a.has_grad && !a.quant_in) return;  // dequantise-only
  amax = block_max(amax, red);
  const float s_new = a.fmt == 0 ? amax / 448.f : amax;
  const float inv = s_new > 0.f ? 1.f / s_new : 0.f;
  if (threadIdx.x == 0) a.scale[blockIdx.x] = s_new;
  if (a.fmt == 2) {
    // Two codes per byte: thread handles element pairs (2t, 2t+1) of each 512-chunk.
    __syncthreads();
    // Stage the block through shared memory so pairs can be packed by one thread.
    __shared__ uint8_t c4[4096];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int e = threadIdx.x + k * LP_THREADS;
      if (e < len) c4[e] = (uint8_t)nearest_code(qmap, a.qn, vals[k] * inv);
    }
    __syncthreads();
    for (int e2 = threadIdx.x; e2 < (len + 1) / 2; e2 += LP_THREADS) {
      const uint8_t lo = c4[2 * e2];
      const uint8_t hi = (2 * e2 + 1 < len) ? c4[2 * e2 + 1] : 0;
      a.codes[(b0 >> 1) + e2] = (uint8_t)(lo | (hi << 4));
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int e = threadIdx.x + k * LP_THREADS;
    if (e < len) {
      const float x = vals[k] * inv;
      uint8_t c;
      if (a.fmt == 0) {
        __nv_fp8_e4m3 q(x);
        c = q.__x;
      } else {
        c = (uint8_t)nearest_code(qmap, a.qn, x);
      }
      a.codes[b0 + e] = c;
    }
  }
}

void launch_lp(const LpArgs& a) {
  TORCH_CHECK(a.block > 0 && a.block <= 4096, "MuonLP block size must be in (0, 4096]");
  TORCH_CHECK(a.fmt != 2 || a.block % 2 == 0, "4-bit state needs an even block size");
  const long long nblocks = (a.n + a.block - 1) / a.block;
  if (nblocks == 0) return;
  lp_step_kernel<<<(unsigned)nblocks, LP_THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// Momentum step on a quantised buffer; writes the bf16 orthogonalisation input
// into `gout` (same element order as grad).
void lp_momentum_step(at::Tensor codes, at::Tensor scale, const at::Tensor& qmap, int64_t fmt, int64_t block,
                      const at::Tensor& grad, at::Tensor gout, double momentum, bool nesterov, bool maximize) {
  const at::cuda::CUDAGuard guard(grad.device());
  TORCH_CHECK(grad.is_contiguous() && gout.is_contiguous() && gout.scalar_type() == at::kBFloat16);
  LpArgs a{};
  a.codes = codes.data_ptr<uint8_t>();
  a.scale = scale.data_ptr<float>();
  a.qmap_g = qmap.data_ptr<float>();
  a.fmt = fmt;
  a.qn = qmap.numel();
  a.n = grad.numel();
  a.block = block;
  a.grad = grad.data_ptr();
  a.grad_dtype = grad.scalar_type() == at::kFloat ? 0 : 1;
  TORCH_CHECK(grad.scalar_type() == at::kFloat || grad.scalar_type() == at::kBFloat16);
  a.gout = reinterpret_cast<__nv_bfloat16*>(gout.data_ptr());
  a.momentum = momentum;
  a.nesterov = nesterov;
  a.maximize = maximize;
  a.has_grad = 1;
  launch_lp(a);
}

at::Tensor lp_dequantize(const at::Tensor& codes, const at::Tensor& scale, const at::Tensor& qmap, int64_t fmt,
                         int64_t block, int64_t n) {
  const at::cuda::CUDAGuard guard(codes.device());
  auto out = at::empty({n}, scale.options());
  LpArgs a{};
  a.codes = const_cast<uint8_t*>(codes.data_ptr<uint8_t>());
  a.scale = const_cast<float*>(scale.data_ptr<float>());
  a.qmap_g = qmap.data_ptr<float>();
  a.fmt = fmt;
  a.qn = qmap.numel();
  a.n = n;
  a.block = block;
  a.dequant_out = out.data_ptr<float>();
  launch_lp(a);
  return out;
}

void lp_quantize(const at::Tensor& x, at::Tensor codes, at::Tensor scale, const at::Tensor& qmap, int64_t fmt,
                 int64_t block) {
  const at::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous());
  LpArgs a{};
  a.codes = codes.data_ptr<uint8_t>();
  a.scale = scale.data_ptr<float>();
  a.qmap_g = qmap.data_ptr<float>();
  a.fmt = fmt;
  a.qn = qmap.numel();
  a.n = x.numel();
  a.block = block;
  a.quant_in = x.data_ptr<float>();
  launch_lp(a);
}

}  // namespace dmb
