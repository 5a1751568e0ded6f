// Memory-bound kernels around the orthogonalisation GEMMs.
//
//   muon_pack      momentum (+Nesterov, maximize) update fused with the bf16
//                  cast, the optional transpose into the N<=M orientation, the
//                  zero padding to a 256-multiple workspace and per-tile
//                  partial sums of squares (for the Frobenius norm).
//                  Reference math: src/muonium/optim/algorithms/muon.py:49-56
//                  (per tensor) and :104-110 (foreach); the stack/transpose/cast
//                  of orthogonalize.py:144 and newton_schulz.py:80-82.
//   norm_finalize  partial sums -> 1 / (||X|| * fac + eps) per matrix
//                  (newton_schulz.py:82, polar_express.py:89).
//   muon_apply     reads the orthogonalised workspace (undoing the transpose),
//                  optional per-row NorMuon scale, cautious / plain decoupled
//                  weight decay and the lr * lr_ratio step, writing the params
//                  in place (muon.py:69-77, :128-140). mode 1 instead writes
//                  the bf16 update to an output tensor (zeropower's result).
//   row_sumsq      per-row (param-row) sums of squares of the update.
//   normuon_finalize  NorMuon's second-moment EMA and Frobenius-preserving
//                  per-row scale (normuon.py:16-55).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>

#include "common.cuh"
#include "no_alloc.h"

namespace dmb {

namespace {

constexpr int TILE = 64;
constexpr int PACK_THREADS = 256;

__device__ __forceinline__ float load_elem(const void* base, int dtype, long long idx) {
  if (dtype == 0) return reinterpret_cast<const float*>(base)[idx];
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
}

__device__ __forceinline__ void store_elem(void* base, int dtype, long long idx, float v) {
  if (dtype == 0)
    reinterpret_cast<float*>(base)[idx] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
}

// Deterministic block sum (fixed shuffle tree + fixed smem order).
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NT / 32; ++i) s += red[i];
    red[0] = s;
  }
  __syncthreads();
  return red[0];
}

struct PackArgs {
  const int64_t* src;  // [B] pointers to the gradient (or plain source) matrices
  const int64_t* buf;  // [B] fp32 momentum matrices, or nullptr
  int src_dtype;       // 0 fp32, 1 bf16
  int R, C;            // logical (param-oriented) matrix shape
  long long ld;        // row stride of each source/buffer matrix, elements
  int transpose;       // workspace holds src^T
  int Np, Mp;          // workspace rows / cols (multiples of TILE = 64; the GEMM layouts use 256)
  float momentum;
  int nesterov, maximize;
  __nv_bfloat16* out;  // [B, Np, Mp]
  float* partial;      // [B, tiles_per_mat]
  int tiles_c;         // workspace tiles along Mp
};

__global__ void __launch_bounds__(PACK_THREADS) muon_pack_kernel(const PackArgs a) {
  __shared__ float tile[TILE][TILE + 1];
  __shared__ float red[PACK_THREADS / 32];
  const int b = blockIdx.y;
  const int wt_r = blockIdx.x / a.tiles_c, wt_c = blockIdx.x % a.tiles_c;
  const int wr0 = wt_r * TILE, wc0 = wt_c * TILE;
  // Source-tile origin in param coordinates.
  const int sr0 = a.transpose ? wc0 : wr0;
  const int sc0 = a.transpose ? wr0 : wc0;
  const void* src = reinterpret_cast<const void*>(a.src[b]);
  float* buf = a.buf ? reinterpret_cast<float*>(a.buf[b]) : nullptr;

  const int j = threadIdx.x & (TILE - 1);
  const int i0 = threadIdx.x >> 6;  // 0..3
  float ss = 0.f;
  const bool any_valid = (sr0 < a.R) && (sc0 < a.C);
#pragma unroll 4
  for (int i = i0; i < TILE; i += PACK_THREADS / TILE) {
    const int r = sr0 + i, c = sc0 + j;
    float v = 0.f;
    if (any_valid && r < a.R && c < a.C) {
      const long long idx = (long long)r * a.ld + c;
      float g = load_elem(src, a.src_dtype, idx);
      if (a.maximize) g = -g;
      if (buf) {
        const float m = fmaf(buf[idx], a.momentum, g);
        buf[idx] = m;
        v = a.nesterov ? fmaf(m, a.momentum, g) : m;
      } else {
        v = g;
      }
      v = __bfloat162float(__float2bfloat16_rn(v));
      ss = fmaf(v, v, ss);
    }
    tile[i][j] = v;
  }
  __syncthreads();
  __nv_bfloat16* out = a.out + (long long)b * a.Np * a.Mp;
#pragma unroll 4
  for (int i = i0; i < TILE; i += PACK_THREADS / TILE) {
    const float v = a.transpose ? tile[j][i] : tile[i][j];
    out[(long long)(wr0 + i) * a.Mp + (wc0 + j)] = __float2bfloat16_rn(v);
  }
  const float tot = block_sum<PACK_THREADS>(ss, red);
  if (threadIdx.x == 0) a.partial[(long long)b * gridDim.x + blockIdx.x] = tot;
}

__global__ void __launch_bounds__(256) norm_finalize_kernel(const float* partial, int nparts, float fac, float eps,
                                                            float* inv_norm, float* norm_out) {
  __shared__ float red[8];
  const int b = blockIdx.x;
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += 256) s += partial[(long long)b * nparts + i];
  const float tot = block_sum<256>(s, red);
  if (threadIdx.x == 0) {
    const float n = sqrtf(tot);
    inv_norm[b] = 1.f / (n * fac + eps);
    if (norm_out) norm_out[b] = n;
  }
}

struct ApplyArgs {
  const __nv_bfloat16* ws;  // [B, Np, Mp]
  int Np, Mp, transpose;
  int R, C;
  long long ld;          // row stride of param / output matrices
  const int64_t* dst;    // [B] param pointers (mode 0)
  int dst_dtype;         // 0 fp32, 1 bf16
  __nv_bfloat16* out;    // mode 1: [B, R, C] contiguous
  const float* rowscale; // [B, R] or nullptr
  const float* mat_scale;// [B] or nullptr (mode 1)
  float lr_eff, wd;
  int cautious, mode;
  int tiles_c;           // param tiles along C
};

__global__ void __launch_bounds__(PACK_THREADS) muon_apply_kernel(const ApplyArgs a) {
  __shared__ float tile[TILE][TILE + 1];
  const int b = blockIdx.y;
  const int pt_r = blockIdx.x / a.tiles_c, pt_c = blockIdx.x % a.tiles_c;
  const int r0 = pt_r * TILE, c0 = pt_c * TILE;
  const int wr0 = a.transpose ? c0 : r0;
  const int wc0 = a.transpose ? r0 : c0;
  const __nv_bfloat16* ws = a.ws + (long long)b * a.Np * a.Mp;
  const int j = threadIdx.x & (TILE - 1);
  const int i0 = threadIdx.x >> 6;
#pragma unroll 4
  for (int i = i0; i < TILE; i += PACK_THREADS / TILE) {
    const int wr = wr0 + i, wc = wc0 + j;
    tile[i][j] = (wr < a.Np && wc < a.Mp) ? __bfloat162float(ws[(long long)wr * a.Mp + wc]) : 0.f;
  }
  __syncthreads();
  const float ms = a.mat_scale ? a.mat_scale[b] : 1.f;
#pragma unroll 4
  for (int i = i0; i < TILE; i += PACK_THREADS / TILE) {
    const int r = r0 + i, c = c0 + j;
    if (r >= a.R || c >= a.C) continue;
    float u = a.transpose ? tile[j][i] : tile[i][j];
    if (a.rowscale) u *= a.rowscale[(long long)b * a.R + r];
    u *= ms;
    const long long idx = (long long)r * a.ld + c;
    if (a.mode == 1) {
      a.out[(long long)b * a.R * a.C + (long long)r * a.C + c] = __float2bfloat16_rn(u);
      continue;
    }
    void* dst = reinterpret_cast<void*>(a.dst[b]);
    const float pv = load_elem(dst, a.dst_dtype, idx);
    if (a.wd != 0.f) {
      if (a.cautious) {
        if (u * pv > 0.f) u = fmaf(a.wd, pv, u);
      } else {
        u = fmaf(a.wd, pv, u);
      }
    }
    store_elem(dst, a.dst_dtype, idx, fmaf(-a.lr_eff, u, pv));
  }
}


// ---- vectorised variants (16-byte accesses; need C % 8 == 0) -------------
__device__ __forceinline__ void ld8(const void* base, int dt, long long idx, float (&v)[8]) {
  if (dt == 0) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    const float4 x = p[0], y = p[1];
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + idx);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[2 * k] = bf16_bits_to_float((uint16_t)(w[k] & 0xFFFFu));
      v[2 * k + 1] = bf16_bits_to_float((uint16_t)(w[k] >> 16));
    }
  }
}

__device__ __forceinline__ void st8(void* base, int dt, long long idx, const float (&v)[8]) {
  if (dt == 0) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + idx);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + idx) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

// g' for 8 consecutive elements (momentum update in place when buf != null); returns bf16-rounded values.
__device__ __forceinline__ void momentum8(const PackArgs& a, const void* src, float* buf, long long idx, float (&v)[8]) {
  ld8(src, a.src_dtype, idx, v);
  if (a.maximize)
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = -v[k];
  if (buf) {
    float m[8];
    ld8(buf, 0, idx, m);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      m[k] = fmaf(m[k], a.momentum, v[k]);
      v[k] = a.nesterov ? fmaf(m[k], a.momentum, v[k]) : m[k];
    }
    st8(buf, 0, idx, m);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = __bfloat162float(__float2bfloat16_rn(v[k]));
}

// Non-transposed: tile 16 rows x 128 cols, 8 elements per thread.
__global__ void __launch_bounds__(PACK_THREADS) muon_pack_rows_vec(const PackArgs a) {
  __shared__ float red[PACK_THREADS / 32];
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int r = tr * 16 + (threadIdx.x >> 4), c = tc * 128 + (threadIdx.x & 15) * 8;
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float ss = 0.f;
  if (r < a.R && c < a.C) {
    float* buf = a.buf ? reinterpret_cast<float*>(a.buf[b]) : nullptr;
    momentum8(a, reinterpret_cast<const void*>(a.src[b]), buf, (long long)r * a.ld + c, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
  }
  st8(a.out + (long long)b * a.Np * a.Mp, 1, (long long)r * a.Mp + c, v);
  const float tot = block_sum<PACK_THREADS>(ss, red);
  if (threadIdx.x == 0) a.partial[(long long)b * gridDim.x + blockIdx.x] = tot;
}

// Transposed: 64 x 64 tile through shared memory, 16-byte loads and stores.
__global__ void __launch_bounds__(PACK_THREADS) muon_pack_tr_vec(const PackArgs a) {
  __shared__ float tile[TILE][TILE + 1];
  __shared__ float red[PACK_THREADS / 32];
  const int b = blockIdx.y;
  const int wt_r = blockIdx.x / a.tiles_c, wt_c = blockIdx.x % a.tiles_c;
  const int wr0 = wt_r * TILE, wc0 = wt_c * TILE;  // workspace rows = source cols
  const int sr0 = wc0, sc0 = wr0;
  const void* src = reinterpret_cast<const void*>(a.src[b]);
  float* buf = a.buf ? reinterpret_cast<float*>(a.buf[b]) : nullptr;
  const int lane8 = (threadIdx.x & 7) * 8, row = threadIdx.x >> 3;
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int sr = row + it * 32;
    const int r = sr0 + sr, c = sc0 + lane8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (r < a.R && c < a.C) {
      momentum8(a, src, buf, (long long)r * a.ld + c, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[sr][lane8 + k] = v[k];
  }
  __syncthreads();
  __nv_bfloat16* out = a.out + (long long)b * a.Np * a.Mp;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int wr = row + it * 32;  // source column offset
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = tile[lane8 + k][wr];
    st8(out, 1, (long long)(wr0 + wr) * a.Mp + wc0 + lane8, v);
  }
  const float tot = block_sum<PACK_THREADS>(ss, red);
  if (threadIdx.x == 0) a.partial[(long long)b * gridDim.x + blockIdx.x] = tot;
}

__device__ __forceinline__ void apply8(const ApplyArgs& a, int b, int r, int c, float (&u)[8]) {
  const float rs = (a.rowscale ? a.rowscale[(long long)b * a.R + r] : 1.f) * (a.mat_scale ? a.mat_scale[b] : 1.f);
  void* dst = reinterpret_cast<void*>(a.dst[b]);
  const long long idx = (long long)r * a.ld + c;
  float p[8];
  ld8(dst, a.dst_dtype, idx, p);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float x = u[k] * rs;
    if (a.wd != 0.f) {
      if (!a.cautious || x * p[k] > 0.f) x = fmaf(a.wd, p[k], x);
    }
    p[k] = fmaf(-a.lr_eff, x, p[k]);
  }
  st8(dst, a.dst_dtype, idx, p);
}

__global__ void __launch_bounds__(PACK_THREADS) muon_apply_rows_vec(const ApplyArgs a) {
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int r = tr * 16 + (threadIdx.x >> 4), c = tc * 128 + (threadIdx.x & 15) * 8;
  if (r >= a.R || c >= a.C) return;
  float u[8];
  ld8(a.ws + (long long)b * a.Np * a.Mp, 1, (long long)r * a.Mp + c, u);
  apply8(a, b, r, c, u);
}

__global__ void __launch_bounds__(PACK_THREADS) muon_apply_tr_vec(const ApplyArgs a) {
  __shared__ float tile[TILE][TILE + 1];
  const int b = blockIdx.y;
  const int pt_r = blockIdx.x / a.tiles_c, pt_c = blockIdx.x % a.tiles_c;
  const int r0 = pt_r * TILE, c0 = pt_c * TILE;  // param tile; workspace rows = param cols
  const __nv_bfloat16* ws = a.ws + (long long)b * a.Np * a.Mp;
  const int lane8 = (threadIdx.x & 7) * 8, row = threadIdx.x >> 3;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int wr = row + it * 32;
    float v[8];
    ld8(ws, 1, (long long)(c0 + wr) * a.Mp + r0 + lane8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[wr][lane8 + k] = v[k];
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int i = row + it * 32;
    const int r = r0 + i, c = c0 + lane8;
    if (r >= a.R || c >= a.C) continue;
    float u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) u[k] = tile[lane8 + k][i];
    apply8(a, b, r, c, u);
  }
}

// rowsq[b, r] = sum_c u[b, r, c]^2 with u read from the (possibly transposed) workspace.
__global__ void __launch_bounds__(256) row_sumsq_rows_kernel(const __nv_bfloat16* ws, int Np, int Mp, int R, int C,
                                                             float* rowsq) {
  const int b = blockIdx.y;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + w;
  if (r >= R) return;
  const __nv_bfloat16* row = ws + (long long)b * Np * Mp + (long long)r * Mp;
  float s = 0.f;
  for (int c = l; c < C; c += 32) {
    const float v = __bfloat162float(row[c]);
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (l == 0) rowsq[(long long)b * R + r] = s;
}

__global__ void __launch_bounds__(256) row_sumsq_cols_kernel(const __nv_bfloat16* ws, int Np, int Mp, int R, int C,
                                                             float* rowsq) {
  // Transposed workspace: param row r is workspace column r; sum over workspace rows 0..C-1.
  __shared__ float part[8][33];
  const int b = blockIdx.y;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int r = blockIdx.x * 32 + tx;
  const __nv_bfloat16* base = ws + (long long)b * Np * Mp;
  float s = 0.f;
  if (r < R)
    for (int i = ty; i < C; i += 8) {
      const float v = __bfloat162float(base[(long long)i * Mp + r]);
      s = fmaf(v, v, s);
    }
  part[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && r < R) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += part[k][tx];
    rowsq[(long long)b * R + r] = t;
  }
}

// NorMuon: v_new = lerp(v, rowsq / C, 1 - beta2); u /= sqrt(v_new) + 1e-8; then
// rescale so ||u||_F is unchanged. Writes v_new into the state and the per-row
// factor into rowscale.
__global__ void __launch_bounds__(256) normuon_finalize_kernel(const float* rowsq, const int64_t* vptrs, int R,
                                                               int C, float beta2, float* rowscale) {
  __shared__ float red[8];
  const int b = blockIdx.x;
  float* v = reinterpret_cast<float*>(vptrs[b]);
  const float* rs = rowsq + (long long)b * R;
  float s_old = 0.f, s_new = 0.f;
  const float w = 1.f - beta2;
  for (int r = threadIdx.x; r < R; r += 256) {
    const float q = rs[r];
    const float nn = q / (float)C;
    const float vo = v[r];
    const float vn = vo + w * (nn - vo);
    v[r] = vn;
    const float inv = 1.f / (sqrtf(vn) + 1e-8f);
    rowscale[(long long)b * R + r] = inv;
    s_old += q;
    s_new += q * inv * inv;
  }
  const float t_old = block_sum<256>(s_old, red);
  const float t_new = block_sum<256>(s_new, red);
  const float fac = sqrtf(t_old) / fmaxf(sqrtf(t_new), 1e-8f);
  for (int r = threadIdx.x; r < R; r += 256) rowscale[(long long)b * R + r] *= fac;
}

}  // namespace

// Packs B matrices (pointers in `src`, optional fp32 momentum `buf`) into the
// bf16 workspace `out` [B, Np, Mp]; returns per-tile partial sums of squares.
at::Tensor muon_pack_ex(const at::Tensor& src_ptrs, const c10::optional<at::Tensor>& buf_ptrs, int64_t src_dtype_code,
                        int64_t R, int64_t C, int64_t ld, bool transpose, at::Tensor& out, double momentum,
                        bool nesterov, bool maximize, bool vec_ok) {
  TORCH_CHECK(out.is_cuda() && out.dim() == 3 && out.scalar_type() == at::kBFloat16 && out.is_contiguous());
  const int B = out.size(0), Np = out.size(1), Mp = out.size(2);
  TORCH_CHECK(Np % TILE == 0 && Mp % TILE == 0);
  TORCH_CHECK(src_ptrs.numel() == B && src_ptrs.scalar_type() == at::kLong && src_ptrs.is_cuda());
  const int64_t N = transpose ? C : R, M = transpose ? R : C;
  TORCH_CHECK(N <= Np && M <= Mp, "workspace too small");
  const at::cuda::CUDAGuard guard(out.device());
  const int tiles_r = Np / TILE, tiles_c = Mp / TILE;
  auto partial = at::empty({B, tiles_r * tiles_c}, out.options().dtype(at::kFloat));
  PackArgs a{};
  a.src = src_ptrs.data_ptr<int64_t>();
  a.buf = buf_ptrs.has_value() ? buf_ptrs->data_ptr<int64_t>() : nullptr;
  a.src_dtype = (int)src_dtype_code;
  a.R = R;
  a.C = C;
  a.ld = ld;
  a.transpose = transpose ? 1 : 0;
  a.Np = Np;
  a.Mp = Mp;
  a.momentum = (float)momentum;
  a.nesterov = nesterov;
  a.maximize = maximize;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.partial = partial.data_ptr<float>();
  a.tiles_c = tiles_c;
  auto st = at::cuda::getCurrentCUDAStream();
  if (vec_ok && C % 8 == 0 && ld % 8 == 0) {
    if (!transpose) {
      a.tiles_c = Mp / 128;
      auto p2 = at::empty({B, (Np / 16) * a.tiles_c}, out.options().dtype(at::kFloat));
      a.partial = p2.data_ptr<float>();
      muon_pack_rows_vec<<<dim3((Np / 16) * a.tiles_c, B), PACK_THREADS, 0, st>>>(a);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      return p2;
    }
    muon_pack_tr_vec<<<dim3(tiles_r * tiles_c, B), PACK_THREADS, 0, st>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return partial;
  }
  dim3 grid(tiles_r * tiles_c, B);
  muon_pack_kernel<<<grid, PACK_THREADS, 0, st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return partial;
}

// Plain entry points: every matrix pointer is assumed 16-byte aligned (torch allocations).
at::Tensor muon_pack(const at::Tensor& src_ptrs, const c10::optional<at::Tensor>& buf_ptrs, int64_t src_dtype_code,
                     int64_t R, int64_t C, int64_t ld, bool transpose, at::Tensor& out, double momentum,
                     bool nesterov, bool maximize) {
  return muon_pack_ex(src_ptrs, buf_ptrs, src_dtype_code, R, C, ld, transpose, out, momentum, nesterov, maximize,
                      true);
}

// partial [B, P] -> inv_norm [B] = 1 / (sqrt(sum) * fac + eps)
at::Tensor norm_finalize(const at::Tensor& partial, double fac, double eps) {
  const at::cuda::CUDAGuard guard(partial.device());
  const int B = partial.size(0), P = partial.size(1);
  auto inv = at::empty({B}, partial.options());
  norm_finalize_kernel<<<B, 256, 0, at::cuda::getCurrentCUDAStream()>>>(partial.data_ptr<float>(), P, (float)fac,
                                                                          (float)eps, inv.data_ptr<float>(), nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return inv;
}

void muon_apply_ex(const at::Tensor& ws, bool transpose, int64_t R, int64_t C, int64_t ld, const at::Tensor& dst_ptrs,
                   int64_t dst_dtype_code, const c10::optional<at::Tensor>& rowscale,
                   const c10::optional<at::Tensor>& mat_scale, double lr_eff, double wd, bool cautious, bool vec_ok) {
  const at::cuda::CUDAGuard guard(ws.device());
  const int B = ws.size(0);
  ApplyArgs a{};
  a.ws = reinterpret_cast<const __nv_bfloat16*>(ws.data_ptr());
  a.Np = ws.size(1);
  a.Mp = ws.size(2);
  a.transpose = transpose;
  a.R = R;
  a.C = C;
  a.ld = ld;
  a.dst = dst_ptrs.data_ptr<int64_t>();
  a.dst_dtype = (int)dst_dtype_code;
  a.rowscale = rowscale.has_value() ? rowscale->data_ptr<float>() : nullptr;
  a.mat_scale = mat_scale.has_value() ? mat_scale->data_ptr<float>() : nullptr;
  a.lr_eff = (float)lr_eff;
  a.wd = (float)wd;
  a.cautious = cautious;
  a.mode = 0;
  auto st = at::cuda::getCurrentCUDAStream();
  if (vec_ok && C % 8 == 0 && ld % 8 == 0) {
    if (!transpose) {
      a.tiles_c = (C + 127) / 128;
      muon_apply_rows_vec<<<dim3(((R + 15) / 16) * a.tiles_c, B), PACK_THREADS, 0, st>>>(a);
    } else {
      a.tiles_c = (C + TILE - 1) / TILE;
      muon_apply_tr_vec<<<dim3(((R + TILE - 1) / TILE) * a.tiles_c, B), PACK_THREADS, 0, st>>>(a);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  a.tiles_c = (C + TILE - 1) / TILE;
  dim3 grid(((R + TILE - 1) / TILE) * a.tiles_c, B);
  muon_apply_kernel<<<grid, PACK_THREADS, 0, st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void muon_apply(const at::Tensor& ws, bool transpose, int64_t R, int64_t C, int64_t ld, const at::Tensor& dst_ptrs,
                int64_t dst_dtype_code, const c10::optional<at::Tensor>& rowscale,
                const c10::optional<at::Tensor>& mat_scale, double lr_eff, double wd, bool cautious) {
  muon_apply_ex(ws, transpose, R, C, ld, dst_ptrs, dst_dtype_code, rowscale, mat_scale, lr_eff, wd, cautious, true);
}

// Workspace -> contiguous bf16 [B, R, C] (undoing the transpose), optionally
// scaled per matrix.
at::Tensor muon_unpack(const at::Tensor& ws, bool transpose, int64_t R, int64_t C,
                       const c10::optional<at::Tensor>& mat_scale) {
  const at::cuda::CUDAGuard guard(ws.device());
  const int B = ws.size(0);
  auto out = at::empty({B, R, C}, ws.options());
  ApplyArgs a{};
  a.ws = reinterpret_cast<const __nv_bfloat16*>(ws.data_ptr());
  a.Np = ws.size(1);
  a.Mp = ws.size(2);
  a.transpose = transpose;
  a.R = R;
  a.C = C;
  a.ld = C;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.mat_scale = mat_scale.has_value() ? mat_scale->data_ptr<float>() : nullptr;
  a.mode = 1;
  a.tiles_c = (C + TILE - 1) / TILE;
  dim3 grid(((R + TILE - 1) / TILE) * a.tiles_c, B);
  if (B > 0 && R > 0 && C > 0) {
    muon_apply_kernel<<<grid, PACK_THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return out;
}

// Per-param-row sums of squares of the update held in the workspace: [B, R].
at::Tensor row_sumsq(const at::Tensor& ws, bool transpose, int64_t R, int64_t C) {
  const at::cuda::CUDAGuard guard(ws.device());
  const int B = ws.size(0), Np = ws.size(1), Mp = ws.size(2);
  auto out = at::empty({B, R}, ws.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  const auto* w = reinterpret_cast<const __nv_bfloat16*>(ws.data_ptr());
  if (!transpose) {
    row_sumsq_rows_kernel<<<dim3((R + 7) / 8, B), 256, 0, st>>>(w, Np, Mp, R, C, out.data_ptr<float>());
  } else {
    row_sumsq_cols_kernel<<<dim3((R + 31) / 32, B), 256, 0, st>>>(w, Np, Mp, R, C, out.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

at::Tensor normuon_finalize(const at::Tensor& rowsq, const at::Tensor& v_ptrs, int64_t C, double beta2) {
  const at::cuda::CUDAGuard guard(rowsq.device());
  const int B = rowsq.size(0), R = rowsq.size(1);
  auto scale = at::empty_like(rowsq);
  normuon_finalize_kernel<<<B, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      rowsq.data_ptr<float>(), v_ptrs.data_ptr<int64_t>(), R, (int)C, (float)beta2, scale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return scale;
}

// ------------------------------------------------------------------------
// Allocation-free variant of muon_pack (no momentum) + norm_finalize; see
// no_alloc.h. The pointer table and the partial sums live in this array.
namespace {

constexpr size_t kNoAllocPtrBytes = sizeof(int64_t) * kNoAllocMaxBatch;
constexpr size_t kNoAllocScratchBytes = kNoAllocPtrBytes + sizeof(float) * (size_t)kNoAllocMaxPartials;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

__global__ void noalloc_fill_ptrs(int64_t base, int64_t stride_bytes, int batch) {
  int64_t* table = reinterpret_cast<int64_t*>(g_noalloc_scratch);
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < batch; b += gridDim.x * blockDim.x)
    table[b] = base + (int64_t)b * stride_bytes;
}

// Per-device address of g_noalloc_scratch, looked up once with that device current.
unsigned char* noalloc_scratch_ptr(int dev, cudaError_t* err) {
  static unsigned char* addr[64] = {nullptr};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  *err = cudaSuccess;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *err = e;
      return nullptr;
    }
    addr[dev] = static_cast<unsigned char*>(p);
  }
  return addr[dev];
}

}  // namespace
}  // namespace dmb

extern "C" int dmb_pack_normalize_noalloc(const void* src, int src_dtype, int batch, int R, int C, int Np, int Mp,
                                          float fac, float eps, void* out_ws, float* inv_norm,
                                          cudaStream_t stream) {
  using namespace dmb;
  if (!src || !out_ws || !inv_norm || batch <= 0 || R <= 0 || C <= 0) return -1;
  if (src_dtype != 0 && src_dtype != 1) return -1;
  if (Np % TILE != 0 || Mp % TILE != 0) return -1;
  const bool transpose = R > C;
  const int N = transpose ? C : R, M = transpose ? R : C;
  if (N > Np || M > Mp) return -1;
  const long long tiles = (long long)(Np / TILE) * (Mp / TILE);
  if (batch > kNoAllocMaxBatch || tiles * batch > (long long)kNoAllocMaxPartials) return -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  unsigned char* scratch = noalloc_scratch_ptr(dev, &e);
  if (!scratch) return (int)e;
  int64_t* ptrs = reinterpret_cast<int64_t*>(scratch);
  float* partial = reinterpret_cast<float*>(scratch + kNoAllocPtrBytes);

  const int64_t esize = src_dtype == 0 ? 4 : 2;
  noalloc_fill_ptrs<<<(batch + 255) / 256, 256, 0, stream>>>(reinterpret_cast<int64_t>(src), (int64_t)R * C * esize,
                                                              batch);
  // Peek (not Get) after every launch: the error state is left as found, and the
  // first failure is returned before a later kernel could read what it missed.
  if ((e = cudaPeekAtLastError()) != cudaSuccess) return (int)e;
  PackArgs a{};
  a.src = ptrs;
  a.buf = nullptr;
  a.src_dtype = src_dtype;
  a.R = R;
  a.C = C;
  a.ld = C;
  a.transpose = transpose ? 1 : 0;
  a.Np = Np;
  a.Mp = Mp;
  a.momentum = 0.f;
  a.nesterov = 0;
  a.maximize = 0;
  a.out = reinterpret_cast<__nv_bfloat16*>(out_ws);
  a.partial = partial;
  a.tiles_c = Mp / TILE;
  muon_pack_kernel<<<dim3((unsigned)tiles, batch), PACK_THREADS, 0, stream>>>(a);
  if ((e = cudaPeekAtLastError()) != cudaSuccess) return (int)e;
  norm_finalize_kernel<<<batch, 256, 0, stream>>>(partial, (int)tiles, fac, eps, inv_norm, nullptr);
  return (int)cudaPeekAtLastError();
}

