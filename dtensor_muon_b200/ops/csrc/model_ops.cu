// Fused elementwise kernels of the decoder block (forward and backward).
//
//   rope      rotary embedding on interleaved pairs of [tokens, heads, head_dim]
//             bf16, cos/sin tables in fp32 [seq, head_dim/2]; the backward is
//             the same rotation by -theta (sign = -1). One read, one write.
//   swiglu    h = silu(a) * b (forward) and da, db from dh (backward) in one
//             pass each, fp32 math, bf16 storage.
//
// New relative to the reference (which ships no model); these replace the
// multi-kernel PyTorch compositions of the same math.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dmb {
namespace {

// Each thread handles 8 bf16 values (4 rotation pairs) with 16-byte accesses.
__global__ void rope_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, long long n_vec, int vec_per_row, int heads, int seq,
                            int half, float sign) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_vec) return;
  const long long row = i / vec_per_row;          // (token, head)
  const int pair0 = (int)(i % vec_per_row) * 4;   // first pair index within head_dim/2
  const int s = (int)((row / heads) % seq);
  const float* c = cos_t + (long long)s * half + pair0;
  const float* sn = sin_t + (long long)s * half + pair0;
  uint4 v = x[i];
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float x0 = bf16_bits_to_float((uint16_t)(w[k] & 0xFFFFu));
    const float x1 = bf16_bits_to_float((uint16_t)(w[k] >> 16));
    const float cc = c[k], ss = sign * sn[k];
    w[k] = pack_bf16x2(x0 * cc - x1 * ss, x0 * ss + x1 * cc);
  }
  y[i] = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float sigmoidf_(float a) { return 1.f / (1.f + __expf(-a)); }

__global__ void swiglu_fwd_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b, uint4* __restrict__ h,
                                  long long n_vec) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_vec) return;
  const uint4 va = a[i], vb = b[i];
  const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
  uint32_t out[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float r[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float x = bf16_bits_to_float((uint16_t)(j ? wa[k] >> 16 : wa[k] & 0xFFFFu));
      const float u = bf16_bits_to_float((uint16_t)(j ? wb[k] >> 16 : wb[k] & 0xFFFFu));
      r[j] = x * sigmoidf_(x) * u;
    }
    out[k] = pack_bf16x2(r[0], r[1]);
  }
  h[i] = make_uint4(out[0], out[1], out[2], out[3]);
}

__global__ void swiglu_bwd_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
                                  const uint4* __restrict__ dh, uint4* __restrict__ da, uint4* __restrict__ db,
                                  long long n_vec) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_vec) return;
  const uint4 va = a[i], vb = b[i], vg = dh[i];
  const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w}, wg[4] = {vg.x, vg.y, vg.z, vg.w};
  uint32_t oa[4], ob[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float ra[2], rb[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float x = bf16_bits_to_float((uint16_t)(j ? wa[k] >> 16 : wa[k] & 0xFFFFu));
      const float u = bf16_bits_to_float((uint16_t)(j ? wb[k] >> 16 : wb[k] & 0xFFFFu));
      const float g = bf16_bits_to_float((uint16_t)(j ? wg[k] >> 16 : wg[k] & 0xFFFFu));
      const float sg = sigmoidf_(x);
      const float silu = x * sg;
      ra[j] = g * u * sg * (1.f + x * (1.f - sg));
      rb[j] = g * silu;
    }
    oa[k] = pack_bf16x2(ra[0], ra[1]);
    ob[k] = pack_bf16x2(rb[0], rb[1]);
  }
  da[i] = make_uint4(oa[0], oa[1], oa[2], oa[3]);
  db[i] = make_uint4(ob[0], ob[1], ob[2], ob[3]);
}

void check_bf16_vec(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
              ": contiguous bf16 CUDA tensor expected");
  TORCH_CHECK(t.numel() % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              ": numel must be a multiple of 8 and 16-byte aligned");
}

}  // namespace

// x: [B, S, H, D] bf16 contiguous; cos/sin: [S, D/2] fp32. sign=+1 forward, -1 backward.
at::Tensor rope(const at::Tensor& x, const at::Tensor& cos_t, const at::Tensor& sin_t, double sign) {
  check_bf16_vec(x, "x");
  TORCH_CHECK(x.dim() == 4 && x.size(3) % 8 == 0);
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && cos_t.is_contiguous() && sin_t.is_contiguous());
  const int S = x.size(1), H = x.size(2), D = x.size(3);
  TORCH_CHECK(cos_t.size(0) >= S && cos_t.size(1) == D / 2);
  const at::cuda::CUDAGuard guard(x.device());
  auto y = at::empty_like(x);
  const long long n_vec = x.numel() / 8;
  if (n_vec == 0) return y;
  rope_kernel<<<(unsigned)((n_vec + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(x.data_ptr()), reinterpret_cast<uint4*>(y.data_ptr()), cos_t.data_ptr<float>(),
      sin_t.data_ptr<float>(), n_vec, D / 8, H, S, D / 2, (float)sign);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

at::Tensor swiglu_fwd(const at::Tensor& a, const at::Tensor& b) {
  check_bf16_vec(a, "a");
  check_bf16_vec(b, "b");
  TORCH_CHECK(a.sizes() == b.sizes());
  const at::cuda::CUDAGuard guard(a.device());
  auto h = at::empty_like(a);
  const long long n = a.numel() / 8;
  if (n) {
    swiglu_fwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const uint4*>(a.data_ptr()), reinterpret_cast<const uint4*>(b.data_ptr()),
        reinterpret_cast<uint4*>(h.data_ptr()), n);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return h;
}

std::vector<at::Tensor> swiglu_bwd(const at::Tensor& a, const at::Tensor& b, const at::Tensor& dh) {
  check_bf16_vec(a, "a");
  check_bf16_vec(b, "b");
  check_bf16_vec(dh, "dh");
  const at::cuda::CUDAGuard guard(a.device());
  auto da = at::empty_like(a), db = at::empty_like(b);
  const long long n = a.numel() / 8;
  if (n) {
    swiglu_bwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const uint4*>(a.data_ptr()), reinterpret_cast<const uint4*>(b.data_ptr()),
        reinterpret_cast<const uint4*>(dh.data_ptr()), reinterpret_cast<uint4*>(da.data_ptr()),
        reinterpret_cast<uint4*>(db.data_ptr()), n);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {da, db};
}

}  // namespace dmb

// ---- fused cross entropy over bf16 logits [T, V] (mean over rows) ----------
namespace dmb {
namespace {

constexpr int CE_THREADS = 512;

__device__ __forceinline__ void ce_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  s = (m == -INFINITY ? 0.f : s * expf(m - mx)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - mx));
  m = mx;
}

// One CTA per row: online max / sum-exp over the row (16-byte loads), then
// loss_row = logsumexp - logit[target]; lse kept for the backward.
__global__ void __launch_bounds__(CE_THREADS) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits,
                                                            const int64_t* __restrict__ targets, int V,
                                                            float* __restrict__ loss, float* __restrict__ lse) {
  const long long row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * (long long)V;
  float m = -INFINITY, s = 0.f;
  const int nvec = V / 8;
  for (int v = threadIdx.x; v < nvec; v += CE_THREADS) {
    float f[8];
    load8(x, 1, (long long)v * 8, f);
    float mm = f[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) mm = fmaxf(mm, f[k]);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += expf(f[k] - mm);
    ce_merge(m, s, mm, ss);
  }
  for (int j = nvec * 8 + threadIdx.x; j < V; j += CE_THREADS) ce_merge(m, s, __bfloat162float(x[j]), 1.f);
  __shared__ float sm[CE_THREADS / 32], ss_[CE_THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    ce_merge(m, s, m2, s2);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sm[w] = m;
    ss_[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss_[0];
    for (int i = 1; i < CE_THREADS / 32; ++i) ce_merge(M, S, sm[i], ss_[i]);
    const float l_se = M + logf(S);
    lse[row] = l_se;
    loss[row] = l_se - __bfloat162float(x[targets[row]]);
  }
}

// grad[row, j] = scale * (softmax(row)_j - [j == target]), written as bf16.
__global__ void __launch_bounds__(256) ce_bwd_kernel(const __nv_bfloat16* __restrict__ logits,
                                                     const int64_t* __restrict__ targets,
                                                     const float* __restrict__ lse, int V, float scale,
                                                     const float* __restrict__ gscale, __nv_bfloat16* __restrict__ grad) {
  const long long row = blockIdx.y;
  if (gscale) scale *= *gscale;  // upstream gradient of the mean, read on the device
  const __nv_bfloat16* x = logits + row * (long long)V;
  __nv_bfloat16* g = grad + row * (long long)V;
  const float l_se = lse[row];
  const long long t = targets[row];
  const int nvec = V / 8;
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += gridDim.x * blockDim.x) {
    float f[8];
    load8(x, 1, (long long)v * 8, f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const long long j = (long long)v * 8 + k;
      f[k] = scale * (expf(f[k] - l_se) - (j == t ? 1.f : 0.f));
    }
    store8(g, 1, (long long)v * 8, f);
  }
  if (blockIdx.x == 0)
    for (int j = nvec * 8 + threadIdx.x; j < V; j += blockDim.x)
      g[j] = __float2bfloat16_rn(scale * (expf(__bfloat162float(x[j]) - l_se) - (j == t ? 1.f : 0.f)));
}

}  // namespace

std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& targets) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.is_contiguous() && logits.dim() == 2);
  TORCH_CHECK(targets.is_cuda() && targets.scalar_type() == at::kLong && targets.numel() == logits.size(0));
  TORCH_CHECK(reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0 && logits.size(1) % 8 == 0,
              "cross_entropy_fwd: 16-byte aligned rows (vocab % 8 == 0) expected");
  const at::cuda::CUDAGuard guard(logits.device());
  const int T = logits.size(0), V = logits.size(1);
  auto loss = at::empty({T}, logits.options().dtype(at::kFloat));
  auto lse = at::empty({T}, logits.options().dtype(at::kFloat));
  if (T) {
    ce_fwd_kernel<<<T, CE_THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), V,
        loss.data_ptr<float>(), lse.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {loss, lse};
}

at::Tensor cross_entropy_bwd(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse,
                             double scale, const c10::optional<at::Tensor>& gscale) {
  const at::cuda::CUDAGuard guard(logits.device());
  const int T = logits.size(0), V = logits.size(1);
  auto grad = at::empty_like(logits);
  if (T) {
    const int per_row = std::max(1, std::min(16, (V / 8 + 255) / 256));
    ce_bwd_kernel<<<dim3(per_row, T), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
        V, (float)scale, gscale.has_value() ? gscale->data_ptr<float>() : nullptr,
        reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return grad;
}

}  // namespace dmb
