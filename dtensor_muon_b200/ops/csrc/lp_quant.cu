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

// Dynamic-tree code maps (dynamic_tree_map in optim_lp.py). A map of n
// entries is sorted: P negative magnitudes, Z zeros, P positive magnitudes
// (unsigned: 1 zero, then P). Decade k (0 <= k < V) holds n_k = 2^(V-k-1)
// magnitudes (0.1 + 0.9 (i+1)/n_k) 10^-k, i < n_k. Encoding needs no search:
// the magnitudes <= t (t >= 0) number
//   (n_k - 1) + clamp(floor((t 10^k - 0.1) n_k / 0.9), 0, n_k)
// for t's decade k (t in (10^-(k+1), 10^-k]), and lo = (entries <= x) - 1.
// Float rounding can move that count by one only when t is within rounding of
// a code value, and then either neighbour pair still yields that code. The
// nearer of lo and lo + 1 is taken (ties to lo), as a binary search would.
// Per CTA the map and three per-decade constants live in shared memory.
struct TreeSmem {
  float q[256];    // the map
  float up[8];     // 10^k
  float cnt[8];    // n_k / 0.9
  float lim[8];    // 10^-(k+1): decade k is (lim[k], lim[k-1]]
};

struct TreeMap {
  const TreeSmem* t;
  int n;       // entries (16 or 256)
  int V;       // magnitude bits
  int P;       // positive magnitudes (2^V - 1)
  int zoff;    // entries below the first positive magnitude
  float lim[7];  // decade thresholds 10^-(j+1), kept in registers (the same chain of products as the table)

  __device__ TreeMap(const TreeSmem* sm, int entries, bool sgn) : t(sm), n(entries) {
    const int bits = entries == 256 ? 8 : 4;
    V = sgn ? bits - 1 : bits;
    P = (1 << V) - 1;
    zoff = entries - P;
    float l = 1.f;
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      l *= 0.1f;
      lim[j] = l;
    }
  }
};

// Fill the shared tables (all threads of the CTA call this, then __syncthreads).
__device__ __forceinline__ void tree_smem_fill(TreeSmem* sm, const float* qmap_g, int qn, int V) {
  for (int i = threadIdx.x; i < qn; i += blockDim.x) sm->q[i] = qmap_g[i];
  if (threadIdx.x < 8) {
    const int k = threadIdx.x;
    float up = 1.f, lim = 1.f;
    for (int j = 0; j < k; ++j) up *= 10.f;
    for (int j = 0; j <= k; ++j) lim *= 0.1f;
    sm->up[k] = up;
    sm->cnt[k] = k < V ? (float)(1 << (V - k - 1)) / 0.9f : 0.f;
    sm->lim[k] = lim;
  }
}

__device__ __forceinline__ int tree_count_le(const TreeMap& m, float t) {
  int k = 0;
#pragma unroll
  for (int j = 0; j < 7; ++j) k += (j < m.V - 1 && t <= m.lim[j]) ? 1 : 0;
  // (below the smallest decade the floor is negative and the count is n_k - 1 = 0)
  const int nk = 1 << (m.V - k - 1);
  const float f = floorf(fmaf(t, m.t->up[k], -0.1f) * m.t->cnt[k]);
  return (nk - 1) + (int)fminf(fmaxf(f, 0.f), (float)nk);
}

__device__ __forceinline__ int nearest_code(const TreeMap& m, float x) {
  const int le = x >= 0.f ? m.zoff + tree_count_le(m, x) : m.P - tree_count_le(m, -x);
  const int lo = min(max(le - 1, 0), m.n - 2);
  return (fabsf(m.t->q[lo + 1] - x) < fabsf(x - m.t->q[lo])) ? lo + 1 : lo;
}

// Faster encoding for the persistent vector kernel: a per-CTA table indexed by
// the top bits of |x| (8 exponent + LUT_MBITS mantissa bits, |x| >= 2^-24; below
// that every magnitude is larger). lut[key] = magnitudes <= the bucket's lower
// edge. A bucket is narrower (relative width 2^-8) than the closest pair of
// magnitudes of any supported map (ratio >= 1.007), so at most one magnitude
// lies inside it and one comparison completes the count.
constexpr int LUT_MBITS = 8;
constexpr int LUT_EMIN = 127 - 24;  // biased exponent of the first bucket
constexpr int LUT_N = 25 << LUT_MBITS;

__device__ __forceinline__ int lut_key(float t) {
  const int k = (int)(__float_as_uint(t) >> (23 - LUT_MBITS)) - (LUT_EMIN << LUT_MBITS);
  return min(max(k, 0), LUT_N - 1);
}

// Fill lut[] from the map in shared memory (binary search over the P ascending
// magnitudes q[zoff .. n)); all threads call it, then __syncthreads.
__device__ __forceinline__ void lut_fill(uint8_t* lut, const TreeMap& m) {
  const float* mag = m.t->q + m.zoff;
  for (int i = threadIdx.x; i < LUT_N; i += blockDim.x) {
    const float edge = i == 0 ? 0.f : __uint_as_float((uint32_t)(i + (LUT_EMIN << LUT_MBITS)) << (23 - LUT_MBITS));
    int lo = 0, hi = m.P;  // count of mag <= edge in [lo, hi]
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (mag[mid] <= edge)
        lo = mid + 1;
      else
        hi = mid;
    }
    lut[i] = (uint8_t)lo;
  }
}

__device__ __forceinline__ int nearest_code_lut(const TreeMap& m, const uint8_t* lut, float x) {
  const float t = fabsf(x);
  const int c = lut[lut_key(t)];
  const int cnt = c + ((c < m.P && m.t->q[m.zoff + c] <= t) ? 1 : 0);  // magnitudes <= t
  const int le = x >= 0.f ? m.zoff + cnt : m.P - cnt;
  const int lo = min(max(le - 1, 0), m.n - 2);
  return (fabsf(m.t->q[lo + 1] - x) < fabsf(x - m.t->q[lo])) ? lo + 1 : lo;
}

__device__ __forceinline__ float decode(const uint8_t* codes, int fmt, long long i, const TreeMap& m) {
  if (fmt == 0) {
    __nv_fp8_e4m3 c;
    c.__x = codes[i];
    return float(c);
  }
  if (fmt == 1) return m.t->q[codes[i]];
  const uint8_t byte = codes[i >> 1];
  return m.t->q[(i & 1) ? (byte >> 4) : (byte & 15)];
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

__device__ __forceinline__ float lp_update(const LpArgs& a, float m, float g, long long i) {
  if (a.maximize) g = -g;
  m = fmaf(m, a.momentum, g);
  if (a.gout) a.gout[i] = __float2bfloat16_rn(a.nesterov ? fmaf(m, a.momentum, g) : m);
  return m;
}

// Generic path: one CTA per quantisation block, element e of the block on
// thread e % LP_THREADS; any block size <= 4096 and any alignment.
__global__ void __launch_bounds__(LP_THREADS) lp_step_kernel(const LpArgs a) {
  __shared__ float red[LP_THREADS / 32];
  __shared__ TreeSmem tsm;
  const bool sgn = a.fmt != 0 && __ldg(a.qmap_g) < 0.f;
  const TreeMap tm(&tsm, a.qn, sgn);
  if (a.fmt != 0) tree_smem_fill(&tsm, a.qmap_g, a.qn, tm.V);
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
        m = decode(a.codes, a.fmt, i, tm) * s_old;
        if (a.has_grad) {
          const float g = a.grad_dtype == 0 ? reinterpret_cast<const float*>(a.grad)[i]
                                            : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.grad)[i]);
          m = lp_update(a, m, g, i);
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
    // Two codes per byte: stage the block's codes in shared memory, then pack pairs.
    __shared__ uint8_t c4[4096];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int e = threadIdx.x + k * LP_THREADS;
      if (e < len) c4[e] = (uint8_t)nearest_code(tm, vals[k] * inv);
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
        c = (uint8_t)nearest_code(tm, x);
      }
      a.codes[b0 + e] = c;
    }
  }
}

// Vector path: every thread owns runs of 8 consecutive elements (16-byte bf16
// loads/stores, 8-byte / 4-byte code accesses), so a 2048-element block is one
// 8-element run per thread and a 4096-element block two. Requires block % 8 == 0,
// n % 8 == 0 and 16-byte-aligned element pointers (checked on the host).
constexpr int LP_VEC = 8;
constexpr int LP_RUNS = 4096 / (LP_VEC * LP_THREADS);  // 2

template <int FMT>
__device__ __forceinline__ void decode8(const LpArgs& a, long long i, const TreeMap& tm, float* v) {
  const float* qmap = tm.t->q;
  if constexpr (FMT == 0) {
    const uint2 w = *reinterpret_cast<const uint2*>(a.codes + i);
    const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __nv_fp8_e4m3 c;
      c.__x = (ws[j >> 2] >> (8 * (j & 3))) & 0xff;
      v[j] = float(c);
    }
  } else if constexpr (FMT == 1) {
    const uint2 w = *reinterpret_cast<const uint2*>(a.codes + i);
    const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = qmap[(ws[j >> 2] >> (8 * (j & 3))) & 0xff];
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(a.codes + (i >> 1));
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = qmap[(w >> (4 * j)) & 15];
  }
}

template <int FMT>
__device__ __forceinline__ void encode8(const LpArgs& a, long long i, const TreeMap& tm, const uint8_t* lut,
                                        const float* v, float inv) {
  if constexpr (FMT == 2) {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) w |= (uint32_t)nearest_code_lut(tm, lut, v[j] * inv) << (4 * j);
    *reinterpret_cast<uint32_t*>(a.codes + (i >> 1)) = w;
  } else {
    uint32_t ws[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t c;
      if constexpr (FMT == 0) {
        __nv_fp8_e4m3 q(v[j] * inv);
        c = q.__x;
      } else {
        c = (uint32_t)nearest_code_lut(tm, lut, v[j] * inv);
      }
      ws[j >> 2] |= c << (8 * (j & 3));
    }
    *reinterpret_cast<uint2*>(a.codes + i) = make_uint2(ws[0], ws[1]);
  }
}

template <int FMT>
__global__ void __launch_bounds__(LP_THREADS) lp_step_vec_kernel(const LpArgs a) {
  __shared__ float red[LP_THREADS / 32];
  __shared__ TreeSmem tsm;
  __shared__ uint8_t lut[FMT != 0 ? LUT_N : 1];
  const bool sgn = FMT != 0 && __ldg(a.qmap_g) < 0.f;
  const TreeMap tm(&tsm, a.qn, sgn);
  if (FMT != 0) tree_smem_fill(&tsm, a.qmap_g, a.qn, tm.V);
  __syncthreads();
  if (FMT != 0 && (a.has_grad || a.quant_in)) {
    lut_fill(lut, tm);
    __syncthreads();
  }
  const long long nblocks = (a.n + a.block - 1) / a.block;
  // persistent: the table is built once per CTA and reused for every block
  for (long long blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    const long long b0 = blk * a.block;
    const int len = (int)min((long long)a.block, a.n - b0);
    const float s_old = a.quant_in ? 0.f : a.scale[blk];
    float v[LP_RUNS][LP_VEC];
    float amax = 0.f;
#pragma unroll
    for (int r = 0; r < LP_RUNS; ++r) {
      const int e = (r * LP_THREADS + threadIdx.x) * LP_VEC;
      if (e < len) {
        const long long i = b0 + e;
        if (a.quant_in) {
          const float4 x0 = *reinterpret_cast<const float4*>(a.quant_in + i);
          const float4 x1 = *reinterpret_cast<const float4*>(a.quant_in + i + 4);
          v[r][0] = x0.x; v[r][1] = x0.y; v[r][2] = x0.z; v[r][3] = x0.w;
          v[r][4] = x1.x; v[r][5] = x1.y; v[r][6] = x1.z; v[r][7] = x1.w;
        } else {
          decode8<FMT>(a, i, tm, v[r]);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[r][j] *= s_old;
          if (a.has_grad) {
            float g[8];
            if (a.grad_dtype == 0) {
              const float4 g0 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.grad) + i);
              const float4 g1 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.grad) + i + 4);
              g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w;
              g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
            } else {
              const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.grad) + i);
              const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(h[j]);
                g[2 * j] = f.x;
                g[2 * j + 1] = f.y;
              }
            }
            uint4 out;
            __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float gj = a.maximize ? -g[j] : g[j];
              v[r][j] = fmaf(v[r][j], a.momentum, gj);
              g[j] = a.nesterov ? fmaf(v[r][j], a.momentum, gj) : v[r][j];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = __floats2bfloat162_rn(g[2 * j], g[2 * j + 1]);
            if (a.gout) *reinterpret_cast<uint4*>(a.gout + i) = out;
          }
        }
        if (a.dequant_out) {
          *reinterpret_cast<float4*>(a.dequant_out + i) = make_float4(v[r][0], v[r][1], v[r][2], v[r][3]);
          *reinterpret_cast<float4*>(a.dequant_out + i + 4) = make_float4(v[r][4], v[r][5], v[r][6], v[r][7]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[r][j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[r][j]));
    }
    if (!a.has_grad && !a.quant_in) continue;  // dequantise-only
    amax = block_max(amax, red);
    const float s_new = FMT == 0 ? amax / 448.f : amax;
    const float inv = s_new > 0.f ? 1.f / s_new : 0.f;
    if (threadIdx.x == 0) a.scale[blk] = s_new;
#pragma unroll
    for (int r = 0; r < LP_RUNS; ++r) {
      const int e = (r * LP_THREADS + threadIdx.x) * LP_VEC;
      if (e < len) encode8<FMT>(a, b0 + e, tm, lut, v[r], inv);
    }
  }
}

bool lp_vec_ok(const LpArgs& a) {
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0; };
  if (a.block % LP_VEC != 0 || a.n % LP_VEC != 0) return false;
  if (!al(a.codes, a.fmt == 2 ? 4 : 8)) return false;
  if (a.grad && !al(a.grad, 16)) return false;
  if (a.gout && !al(a.gout, 16)) return false;
  if (a.dequant_out && !al(a.dequant_out, 16)) return false;
  if (a.quant_in && !al(a.quant_in, 16)) return false;
  return true;
}

void launch_lp(LpArgs a) {
  TORCH_CHECK(a.block > 0 && a.block <= 4096, "MuonLP block size must be in (0, 4096]");
  TORCH_CHECK(a.fmt != 2 || a.block % 2 == 0, "4-bit state needs an even block size");
  if (a.fmt != 0) {
    TORCH_CHECK(a.qn == 16 || a.qn == 256, "code map must have 16 or 256 entries");
  }
  const long long nblocks = (a.n + a.block - 1) / a.block;
  if (nblocks == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (lp_vec_ok(a)) {
    // persistent grid: a few CTAs per SM, each looping over blocks
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned grid = (unsigned)std::min<long long>(nblocks, (long long)sms * 6);
    if (a.fmt == 0)
      lp_step_vec_kernel<0><<<grid, LP_THREADS, 0, stream>>>(a);
    else if (a.fmt == 1)
      lp_step_vec_kernel<1><<<grid, LP_THREADS, 0, stream>>>(a);
    else
      lp_step_vec_kernel<2><<<grid, LP_THREADS, 0, stream>>>(a);
  } else {
    lp_step_kernel<<<(unsigned)nblocks, LP_THREADS, 0, stream>>>(a);
  }
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
