// Owner-compute Muon for dim-0 (FSDP) sharded 2-D matrices over NVLink peer memory.
//
// The reference moves whole matrices to "owner" ranks with a DTensor
// redistribute (an NCCL all-to-all), orthogonalises there and redistributes
// back (src/muonium/orthogonalize/orthogonalize.py:140-155, call sites C4/C5).
// Here both all-to-alls are fused into the memory-bound kernels around the
// owner's GEMMs, through a symmetric buffer every rank can address:
//
//   dist_pack_rows    local momentum / Nesterov on this rank's row shard,
//                     bf16 cast, (transpose,) zero padding, written with P2P
//                     stores straight into the owner's orthogonalisation
//                     workspace (+ per-block partial sums of squares, local)
//   dist_push_sums    per-matrix sum of the partials -> owner's sums[slot][rank]
//                     (and, for NorMuon, this rank's variance rows -> owner)
//   dist_barrier      device-side barrier on flags in the symmetric buffer;
//                     every wait is bounded (error word + return, no hang)
//   dist_apply_rows   P2P loads of this rank's rows of the owner's result
//                     (+ NorMuon row scale), cautious / plain WD, lr step on
//                     the local shard, NorMuon variance rows copied back
//
// The owner itself runs the ordinary local engine (norm_finalize,
// ortho_iterate, row_sumsq / normuon_finalize) on its slots in between.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dmb {

int* device_error_word(int dev);

namespace {

constexpr int T = 64;
constexpr int NT = 256;

__device__ __forceinline__ float ldf(const void* p, int dt, long long i) {
  return dt == 0 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void stf(void* p, int dt, long long i, float v) {
  if (dt == 0)
    reinterpret_cast<float*>(p)[i] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

struct DistArgs {
  const int64_t* grad;  // [B] local shard pointers (rows_local x C)
  const int64_t* buf;   // [B] local fp32 momentum shard pointers
  const int64_t* param; // [B] local param shard pointers
  const int64_t* var;   // [B] local NorMuon variance rows (fp32, rows_local) or nullptr
  const int* owner;     // [B]
  const int* slot;      // [B]
  const int64_t* peer_base;  // [W] symmetric buffer base on every rank
  long long x_off, res_off, sums_off, vbuf_off, rs_off;  // byte offsets of regions
  int grad_dtype, param_dtype;
  int R, C, transpose, Np, Mp;
  int r0, r1;           // this rank's global rows [r0, r1)
  int g1;               // rows handled by pack: [r0, g1) (the rank ending at R also covers the padding)
  int c0, c1;           // this rank's global columns [c0, c1) (FSDP: the whole width)
  int h1;               // columns handled by pack: [c0, h1) (the rank ending at C covers the padding)
  int ldl;              // row stride of the local shard (c1 - c0 for a contiguous shard)
  int rank, world;
  float momentum;
  int nesterov, maximize;
  float* partial;       // [B, nblk] local
  int tiles_c;
  float lr_eff, wd;
  int cautious, has_rowscale;
  int vec_ok;           // host checked: every local pointer is 16-byte aligned
};

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < NT / 32; ++i) s += red[i];
    red[0] = s;
  }
  __syncthreads();
  return red[0];
}

// Tile (64 rows of [r0, g1)) x (64 source columns of [0, Cpad)).
__global__ void __launch_bounds__(NT) dist_pack_rows_kernel(const DistArgs a) {
  __shared__ float tile[T][T + 1];
  __shared__ float red[NT / 32];
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int g0 = a.r0 + tr * T, c0 = a.c0 + tc * T;
  const void* g = reinterpret_cast<const void*>(a.grad[b]);
  float* buf = a.buf ? reinterpret_cast<float*>(a.buf[b]) : nullptr;
  const int j = threadIdx.x & (T - 1), i0 = threadIdx.x >> 6;
  float ss = 0.f;
  for (int i = i0; i < T; i += NT / T) {
    const int gr = g0 + i, c = c0 + j;
    float v = 0.f;
    if (gr < a.r1 && c < a.c1) {
      const long long idx = (long long)(gr - a.r0) * a.ldl + (c - a.c0);
      float gv = ldf(g, a.grad_dtype, idx);
      if (a.maximize) gv = -gv;
      if (buf) {
        const float m = fmaf(buf[idx], a.momentum, gv);
        buf[idx] = m;
        v = a.nesterov ? fmaf(m, a.momentum, gv) : m;
      } else {
        v = gv;
      }
      v = __bfloat162float(__float2bfloat16_rn(v));
      ss = fmaf(v, v, ss);
    }
    tile[i][j] = v;
  }
  __syncthreads();
  __nv_bfloat16* X = reinterpret_cast<__nv_bfloat16*>(a.peer_base[a.owner[b]] + a.x_off) +
                     (long long)a.slot[b] * a.Np * a.Mp;
  if (!a.transpose) {
    // X[gr][c]: row-contiguous stores.
    for (int i = i0; i < T; i += NT / T) {
      const int gr = g0 + i, c = c0 + j;
      if (gr < a.g1 && c < a.h1) X[(long long)gr * a.Mp + c] = __float2bfloat16_rn(tile[i][j]);
    }
  } else {
    // X[c][gr]: consecutive threads walk gr.
    for (int i = i0; i < T; i += NT / T) {
      const int c = c0 + i, gr = g0 + j;
      if (gr < a.g1 && c < a.h1) X[(long long)c * a.Mp + gr] = __float2bfloat16_rn(tile[j][i]);
    }
  }
  const float tot = block_sum(ss, red);
  if (threadIdx.x == 0) a.partial[(long long)b * gridDim.x + blockIdx.x] = tot;
}

__global__ void __launch_bounds__(NT) dist_push_sums_kernel(const DistArgs a, int nblk) {
  __shared__ float red[NT / 32];
  const int b = blockIdx.x;
  float s = 0.f;
  for (int i = threadIdx.x; i < nblk; i += NT) s += a.partial[(long long)b * nblk + i];
  const float tot = block_sum(s, red);
  const int64_t base = a.peer_base[a.owner[b]];
  if (threadIdx.x == 0) reinterpret_cast<float*>(base + a.sums_off)[(long long)a.slot[b] * a.world + a.rank] = tot;
  if (a.var && a.c0 == 0) {  // one writer per row (the rank holding the first column block)
    const float* v = reinterpret_cast<const float*>(a.var[b]);
    float* dst = reinterpret_cast<float*>(base + a.vbuf_off) + (long long)a.slot[b] * a.R;
    for (int r = a.r0 + threadIdx.x; r < a.r1; r += NT) dst[r] = v[r - a.r0];
  }
}

__global__ void __launch_bounds__(NT) dist_apply_rows_kernel(const DistArgs a) {
  __shared__ float tile[T][T + 1];
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int g0 = a.r0 + tr * T, c0 = a.c0 + tc * T;
  const int64_t base = a.peer_base[a.owner[b]];
  const __nv_bfloat16* U = reinterpret_cast<const __nv_bfloat16*>(base + a.res_off) + (long long)a.slot[b] * a.Np * a.Mp;
  const float* rs = a.has_rowscale ? reinterpret_cast<const float*>(base + a.rs_off) + (long long)a.slot[b] * a.R : nullptr;
  const int j = threadIdx.x & (T - 1), i0 = threadIdx.x >> 6;
  if (!a.transpose) {
    for (int i = i0; i < T; i += NT / T) {
      const int gr = g0 + i, c = c0 + j;
      tile[i][j] = (gr < a.r1 && c < a.c1) ? __bfloat162float(U[(long long)gr * a.Mp + c]) : 0.f;
    }
  } else {
    for (int i = i0; i < T; i += NT / T) {
      const int c = c0 + i, gr = g0 + j;
      tile[j][i] = (gr < a.r1 && c < a.c1) ? __bfloat162float(U[(long long)c * a.Mp + gr]) : 0.f;
    }
  }
  __syncthreads();
  void* P = reinterpret_cast<void*>(a.param[b]);
  for (int i = i0; i < T; i += NT / T) {
    const int gr = g0 + i, c = c0 + j;
    if (gr >= a.r1 || c >= a.c1) continue;
    float u = tile[i][j];
    if (rs) u *= rs[gr];
    const long long idx = (long long)(gr - a.r0) * a.ldl + (c - a.c0);
    const float pv = ldf(P, a.param_dtype, idx);
    if (a.wd != 0.f) {
      if (a.cautious) {
        if (u * pv > 0.f) u = fmaf(a.wd, pv, u);
      } else {
        u = fmaf(a.wd, pv, u);
      }
    }
    stf(P, a.param_dtype, idx, fmaf(-a.lr_eff, u, pv));
  }
  // NorMuon: this rank's rows of the updated variance come back from the owner.
  if (a.var && tc == 0) {
    const float* vsrc = reinterpret_cast<const float*>(base + a.vbuf_off) + (long long)a.slot[b] * a.R;
    float* v = reinterpret_cast<float*>(a.var[b]);
    for (int i = threadIdx.x; i < T; i += NT) {
      const int gr = g0 + i;
      if (gr < a.r1) v[gr - a.r0] = vsrc[gr];
    }
  }
}


// ---- vectorised owner-compute kernels (C % 8 == 0, row chunk % 8 == 0) -----
__device__ __forceinline__ void dist_momentum8(const DistArgs& a, const void* g, float* buf, long long idx,
                                               float (&v)[8]) {
  load8(g, a.grad_dtype, idx, v);
  if (a.maximize)
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = -v[k];
  if (buf) {
    float m[8];
    load8(buf, 0, idx, m);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      m[k] = fmaf(m[k], a.momentum, v[k]);
      v[k] = a.nesterov ? fmaf(m[k], a.momentum, v[k]) : m[k];
    }
    store8(buf, 0, idx, m);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = __bfloat162float(__float2bfloat16_rn(v[k]));
}

// Non-transposed: rows [r0, g1) x cols [0, Mp): 16 rows x 128 cols per CTA.
__global__ void __launch_bounds__(NT) dist_pack_rows_vec(const DistArgs a) {
  __shared__ float red[NT / 32];
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int gr = a.r0 + tr * 16 + (threadIdx.x >> 4), c = a.c0 + tc * 128 + (threadIdx.x & 15) * 8;
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float ss = 0.f;
  if (gr < a.r1 && c < a.c1) {
    const long long idx = (long long)(gr - a.r0) * a.ldl + (c - a.c0);
    dist_momentum8(a, reinterpret_cast<const void*>(a.grad[b]), a.buf ? reinterpret_cast<float*>(a.buf[b]) : nullptr,
                   idx, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
  }
  if (gr < a.g1 && c < a.h1) {
    __nv_bfloat16* X = reinterpret_cast<__nv_bfloat16*>(a.peer_base[a.owner[b]] + a.x_off) +
                       (long long)a.slot[b] * a.Np * a.Mp;
    store8(X, 1, (long long)gr * a.Mp + c, v);
  }
  const float tot = block_sum(ss, red);
  if (threadIdx.x == 0) a.partial[(long long)b * gridDim.x + blockIdx.x] = tot;
}

// Transposed: 64 local rows x 64 cols through shared memory; X[c][gr .. gr+7] stored as 16 bytes.
__global__ void __launch_bounds__(NT) dist_pack_tr_vec(const DistArgs a) {
  __shared__ float tile[T][T + 1];
  __shared__ float red[NT / 32];
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int g0 = a.r0 + tr * T, c0 = a.c0 + tc * T;
  const int lane8 = (threadIdx.x & 7) * 8, row = threadIdx.x >> 3;
  const void* g = reinterpret_cast<const void*>(a.grad[b]);
  float* buf = a.buf ? reinterpret_cast<float*>(a.buf[b]) : nullptr;
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int i = row + it * 32;
    const int gr = g0 + i, c = c0 + lane8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (gr < a.r1 && c < a.c1) {
      dist_momentum8(a, g, buf, (long long)(gr - a.r0) * a.ldl + (c - a.c0), v);
#pragma unroll
      for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[i][lane8 + k] = v[k];
  }
  __syncthreads();
  __nv_bfloat16* X = reinterpret_cast<__nv_bfloat16*>(a.peer_base[a.owner[b]] + a.x_off) +
                     (long long)a.slot[b] * a.Np * a.Mp;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int j = row + it * 32;  // column offset within the tile
    const int c = c0 + j, gr = g0 + lane8;
    if (c < a.h1 && gr < a.g1) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = tile[lane8 + k][j];
      store8(X, 1, (long long)c * a.Mp + gr, v);
    }
  }
  const float tot = block_sum(ss, red);
  if (threadIdx.x == 0) a.partial[(long long)b * gridDim.x + blockIdx.x] = tot;
}

__device__ __forceinline__ void dist_apply8(const DistArgs& a, int b, int gr, int c, float (&u)[8], const float* rs) {
  if (rs) {
    const float f = rs[gr];
#pragma unroll
    for (int k = 0; k < 8; ++k) u[k] *= f;
  }
  void* P = reinterpret_cast<void*>(a.param[b]);
  const long long idx = (long long)(gr - a.r0) * a.ldl + (c - a.c0);
  float p[8];
  load8(P, a.param_dtype, idx, p);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float x = u[k];
    if (a.wd != 0.f && (!a.cautious || x * p[k] > 0.f)) x = fmaf(a.wd, p[k], x);
    p[k] = fmaf(-a.lr_eff, x, p[k]);
  }
  store8(P, a.param_dtype, idx, p);
}

__global__ void __launch_bounds__(NT) dist_apply_rows_vec(const DistArgs a) {
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int gr = a.r0 + tr * 16 + (threadIdx.x >> 4), c = a.c0 + tc * 128 + (threadIdx.x & 15) * 8;
  const int64_t base = a.peer_base[a.owner[b]];
  if (a.var && tc == 0 && (threadIdx.x & 15) == 0 && gr < a.r1) {
    const float* vsrc = reinterpret_cast<const float*>(base + a.vbuf_off) + (long long)a.slot[b] * a.R;
    reinterpret_cast<float*>(a.var[b])[gr - a.r0] = vsrc[gr];
  }
  if (gr >= a.r1 || c >= a.c1) return;
  const __nv_bfloat16* U = reinterpret_cast<const __nv_bfloat16*>(base + a.res_off) + (long long)a.slot[b] * a.Np * a.Mp;
  const float* rs = a.has_rowscale ? reinterpret_cast<const float*>(base + a.rs_off) + (long long)a.slot[b] * a.R : nullptr;
  float u[8];
  load8(U, 1, (long long)gr * a.Mp + c, u);
  dist_apply8(a, b, gr, c, u, rs);
}

__global__ void __launch_bounds__(NT) dist_apply_tr_vec(const DistArgs a) {
  __shared__ float tile[T][T + 1];
  const int b = blockIdx.y;
  const int tr = blockIdx.x / a.tiles_c, tc = blockIdx.x % a.tiles_c;
  const int g0 = a.r0 + tr * T, c0 = a.c0 + tc * T;
  const int64_t base = a.peer_base[a.owner[b]];
  const __nv_bfloat16* U = reinterpret_cast<const __nv_bfloat16*>(base + a.res_off) + (long long)a.slot[b] * a.Np * a.Mp;
  const float* rs = a.has_rowscale ? reinterpret_cast<const float*>(base + a.rs_off) + (long long)a.slot[b] * a.R : nullptr;
  const int lane8 = (threadIdx.x & 7) * 8, row = threadIdx.x >> 3;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int j = row + it * 32;  // workspace row = param column c0 + j
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (c0 + j < a.c1 && g0 + lane8 < a.r1) load8(U, 1, (long long)(c0 + j) * a.Mp + g0 + lane8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[j][lane8 + k] = v[k];
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int i = row + it * 32;
    const int gr = g0 + i, c = c0 + lane8;
    if (gr >= a.r1 || c >= a.c1) continue;
    float u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) u[k] = tile[lane8 + k][i];
    dist_apply8(a, b, gr, c, u, rs);
  }
  if (a.var && tc == 0) {
    const float* vsrc = reinterpret_cast<const float*>(base + a.vbuf_off) + (long long)a.slot[b] * a.R;
    for (int i = threadIdx.x; i < T; i += NT) {
      const int gr = g0 + i;
      if (gr < a.r1) reinterpret_cast<float*>(a.var[b])[gr - a.r0] = vsrc[gr];
    }
  }
}

// flags: uint32 [world] at offset 0 of every rank's flag buffer. Rank r
// announces epoch e by writing flags[r] = e on every peer, then waits until
// its own flags[k] >= e for all k. Bounded: gives up after kWaitTimeoutNs.
__global__ void dist_barrier_kernel(const int64_t* flag_base, int rank, int world, unsigned epoch, int* err) {
  const int k = threadIdx.x;
  if (k < world) {
    __threadfence_system();
    unsigned* peer = reinterpret_cast<unsigned*>(flag_base[k]) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peer), "r"(epoch) : "memory");
    const unsigned* mine = reinterpret_cast<const unsigned*>(flag_base[rank]) + k;
    const unsigned long long t0 = global_timer_ns();
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int)(v - epoch) >= 0) break;
      if (global_timer_ns() - t0 > kWaitTimeoutNs) {
        atomicExch(err, (int)kErrPeerTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  __threadfence_system();
}

// Split barrier for pipelined owner compute. flags: uint32 [slots][world] in
// every rank's flag buffer. flag_signal: after this stream's previous work,
// rank announces `epoch` in slot `slot` of every peer (flags[slot][rank] = epoch,
// release at system scope). flag_wait: returns once flags[slot][k] >= epoch for
// every k of this rank's own buffer (acquire); bounded like the barrier.
__global__ void flag_signal_kernel(const int64_t* flag_base, int slot, int rank, int world, unsigned epoch) {
  const int k = threadIdx.x;
  __threadfence_system();
  if (k < world) {
    unsigned* peer = reinterpret_cast<unsigned*>(flag_base[k]) + (long long)slot * world + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peer), "r"(epoch) : "memory");
  }
}

__global__ void flag_wait_kernel(const int64_t* flag_base, int slot, int rank, int world, unsigned epoch, int* err) {
  const int k = threadIdx.x;
  if (k < world) {
    const unsigned* mine = reinterpret_cast<const unsigned*>(flag_base[rank]) + (long long)slot * world + k;
    const unsigned long long t0 = global_timer_ns();
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int)(v - epoch) >= 0) break;
      if (global_timer_ns() - t0 > kWaitTimeoutNs) {
        atomicExch(err, (int)kErrPeerTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  __threadfence_system();
}

}  // namespace

namespace {
DistArgs make_args(const at::Tensor& meta_i64, const at::Tensor& meta_i32, const at::Tensor& peer_base,
                   const std::vector<int64_t>& ints, const std::vector<double>& floats, bool has_buf,
                   bool has_var) {
  // meta_i64: [4, B] grad, buf, param, var pointers; meta_i32: [2, B] owner, slot.
  const int B = meta_i64.size(1);
  DistArgs a{};
  const int64_t* m = meta_i64.data_ptr<int64_t>();
  a.grad = m;
  a.buf = has_buf ? m + B : nullptr;
  a.param = m + 2 * B;
  a.var = has_var ? m + 3 * B : nullptr;
  a.owner = meta_i32.data_ptr<int>();
  a.slot = meta_i32.data_ptr<int>() + B;
  a.peer_base = peer_base.data_ptr<int64_t>();
  // ints: x_off res_off sums_off vbuf_off rs_off grad_dtype param_dtype R C transpose Np Mp r0 r1 g1 rank world
  //       nesterov maximize cautious has_rowscale
  a.x_off = ints[0];
  a.res_off = ints[1];
  a.sums_off = ints[2];
  a.vbuf_off = ints[3];
  a.rs_off = ints[4];
  a.grad_dtype = ints[5];
  a.param_dtype = ints[6];
  a.R = ints[7];
  a.C = ints[8];
  a.transpose = ints[9];
  a.Np = ints[10];
  a.Mp = ints[11];
  a.r0 = ints[12];
  a.r1 = ints[13];
  a.g1 = ints[14];
  a.rank = ints[15];
  a.world = ints[16];
  a.nesterov = ints[17];
  a.maximize = ints[18];
  a.cautious = ints[19];
  a.has_rowscale = ints[20];
  a.vec_ok = ints.size() > 21 ? (int)ints[21] : 0;
  // ints[22..25]: c0 c1 h1 ldl (column block of a 2-D sharded shard); default: all columns
  const int Cpad = a.transpose ? a.Np : a.Mp;
  a.c0 = ints.size() > 25 ? (int)ints[22] : 0;
  a.c1 = ints.size() > 25 ? (int)ints[23] : a.C;
  a.h1 = ints.size() > 25 ? (int)ints[24] : Cpad;
  a.ldl = ints.size() > 25 ? (int)ints[25] : a.C;
  a.momentum = floats[0];
  a.lr_eff = floats[1];
  a.wd = floats[2];
  return a;
}
}  // namespace

// 8-element vector kernels: every row/column edge they touch is a multiple of 8.
bool vec_shape_ok(const DistArgs& a) {
  return a.vec_ok && a.C % 8 == 0 && a.R % 8 == 0 && a.r0 % 8 == 0 && a.r1 % 8 == 0 && a.c0 % 8 == 0 &&
         a.c1 % 8 == 0 && a.h1 % 8 == 0 && a.ldl % 8 == 0;
}

// Phase 1: local momentum + P2P scatter into owners' workspaces, then per-matrix
// sums (and NorMuon variance rows) pushed to the owners.
void dist_pack(const at::Tensor& meta_i64, const at::Tensor& meta_i32, const at::Tensor& peer_base,
               std::vector<int64_t> ints, std::vector<double> floats, bool has_buf, bool has_var) {
  const at::cuda::CUDAGuard guard(meta_i64.device());
  DistArgs a = make_args(meta_i64, meta_i32, peer_base, ints, floats, has_buf, has_var);
  const int B = meta_i64.size(1);
  const int width = a.h1 - a.c0;
  a.tiles_c = (width + T - 1) / T;
  const int rows = a.g1 - a.r0;
  const int tiles_r = rows > 0 ? (rows + T - 1) / T : 0;
  const int nblk = width > 0 ? tiles_r * a.tiles_c : 0;
  auto st = at::cuda::getCurrentCUDAStream();
  const bool vec = vec_shape_ok(a);
  int grid_x = nblk;
  if (vec && !a.transpose) {
    a.tiles_c = (width + 127) / 128;
    grid_x = rows > 0 && width > 0 ? ((rows + 15) / 16) * a.tiles_c : 0;
  }
  auto partial = at::zeros({B, std::max(grid_x, 1)}, meta_i64.options().dtype(at::kFloat));
  a.partial = partial.data_ptr<float>();
  if (grid_x > 0) {
    if (vec && !a.transpose)
      dist_pack_rows_vec<<<dim3(grid_x, B), NT, 0, st>>>(a);
    else if (vec)
      dist_pack_tr_vec<<<dim3(grid_x, B), NT, 0, st>>>(a);
    else
      dist_pack_rows_kernel<<<dim3(grid_x, B), NT, 0, st>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  dist_push_sums_kernel<<<B, NT, 0, st>>>(a, std::max(grid_x, 1));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Phase 3: P2P gather of this rank's rows of the owners' results + apply.
void dist_apply(const at::Tensor& meta_i64, const at::Tensor& meta_i32, const at::Tensor& peer_base,
                std::vector<int64_t> ints, std::vector<double> floats, bool has_var) {
  const at::cuda::CUDAGuard guard(meta_i64.device());
  DistArgs a = make_args(meta_i64, meta_i32, peer_base, ints, floats, false, has_var);
  const int B = meta_i64.size(1);
  const int width = a.c1 - a.c0;
  a.tiles_c = (width + T - 1) / T;
  const int rows = a.r1 - a.r0;
  if (rows <= 0 || width <= 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const bool vec = vec_shape_ok(a);
  if (vec && !a.transpose) {
    a.tiles_c = (width + 127) / 128;
    dist_apply_rows_vec<<<dim3(((rows + 15) / 16) * a.tiles_c, B), NT, 0, st>>>(a);
  } else if (vec) {
    dist_apply_tr_vec<<<dim3(((rows + T - 1) / T) * a.tiles_c, B), NT, 0, st>>>(a);
  } else {
    const int tiles_r = (rows + T - 1) / T;
    dist_apply_rows_kernel<<<dim3(tiles_r * a.tiles_c, B), NT, 0, st>>>(a);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void flag_signal(const at::Tensor& flag_base, int64_t slot, int64_t rank, int64_t world, int64_t epoch) {
  const at::cuda::CUDAGuard guard(flag_base.device());
  TORCH_CHECK(world <= 1024 && slot >= 0);
  flag_signal_kernel<<<1, (int)((world + 31) / 32 * 32), 0, at::cuda::getCurrentCUDAStream()>>>(
      flag_base.data_ptr<int64_t>(), (int)slot, (int)rank, (int)world, (unsigned)epoch);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void flag_wait(const at::Tensor& flag_base, int64_t slot, int64_t rank, int64_t world, int64_t epoch) {
  const at::cuda::CUDAGuard guard(flag_base.device());
  TORCH_CHECK(world <= 1024 && slot >= 0);
  flag_wait_kernel<<<1, (int)((world + 31) / 32 * 32), 0, at::cuda::getCurrentCUDAStream()>>>(
      flag_base.data_ptr<int64_t>(), (int)slot, (int)rank, (int)world, (unsigned)epoch,
      device_error_word(flag_base.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dist_barrier(const at::Tensor& flag_base, int64_t rank, int64_t world, int64_t epoch) {
  const at::cuda::CUDAGuard guard(flag_base.device());
  TORCH_CHECK(world <= 1024);
  dist_barrier_kernel<<<1, (int)((world + 31) / 32 * 32), 0, at::cuda::getCurrentCUDAStream()>>>(
      flag_base.data_ptr<int64_t>(), (int)rank, (int)world, (unsigned)epoch, device_error_word(flag_base.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmb

// ------------------------------------------------------------------------
// FSDP collectives over peer memory (plugged into FSDP2 through its custom
// all-gather / reduce-scatter hooks, parallel/fsdp_comm.py).
// ---- push variants: stores into peers' staging (one barrier per collective)
namespace dmb {
namespace {

// For every rank k: peer_k[off + rank * slot_bytes + i] = src[(per_peer ? k * slot_bytes : 0) + i].
// grid.y walks the peers (rotated by rank so ranks spread over peers); each
// thread keeps 4 independent 16-byte stores in flight; no division in the loop.
__global__ void push_slots_kernel(const uint4* __restrict__ src, const int64_t* peer_base, long long off,
                                  long long slot_vec, int rank, int world, int per_peer) {
  const int k = (blockIdx.y + rank) % world;
  uint4* dst = reinterpret_cast<uint4*>(peer_base[k] + off) + (long long)rank * slot_vec;
  const uint4* s = src + (per_peer ? (long long)k * slot_vec : 0);
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < slot_vec; i += 4 * stride) {
    const uint4 a = s[i], b = s[i + stride], c = s[i + 2 * stride], d = s[i + 3 * stride];
    dst[i] = a;
    dst[i + stride] = b;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; i < slot_vec; i += stride) dst[i] = s[i];
}

// For every rank k: out[k * slot + i] = peer_k[off + k * slot + i] (k == rank reads
// its own staging). The all-gather by pulls: each rank has put its shard into its
// own slot; the result lands straight in the caller's output with no staging copy.
__global__ void pull_slots_kernel(uint4* __restrict__ out, const int64_t* peer_base, long long off, long long slot_vec,
                                  int rank, int world) {
  const int k = (blockIdx.y + rank) % world;
  const uint4* src = reinterpret_cast<const uint4*>(peer_base[k] + off) + (long long)k * slot_vec;
  uint4* dst = out + (long long)k * slot_vec;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < slot_vec; i += 4 * stride) {
    const uint4 a = src[i], b = src[i + stride], c = src[i + 2 * stride], d = src[i + 3 * stride];
    dst[i] = a;
    dst[i + stride] = b;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; i < slot_vec; i += stride) dst[i] = src[i];
}

// In-place all-reduce (sum) of n elements at byte offset `off` of every rank's
// symmetric buffer. Rank r owns chunk r: it sums that chunk over all ranks and
// writes the sum back into every rank's chunk. Two transports:
//  * mc_base != 0 (NVLS): one multimem.ld_reduce through the NVSwitch
//    multicast address returns the sum of all ranks' values, one multimem.st
//    writes it to every rank (the switch reduces and replicates);
//  * otherwise P2P: W 16-byte loads (one per peer), fp32 sum, W stores.
// Callers put a device barrier before (inputs written) and after (results
// visible). Elements are handled 8 (bf16) or 4 (fp32) at a time: 16 bytes.
__device__ __forceinline__ void mm_ld_reduce_bf16x8(const void* mc, uint32_t (&r)[4]) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(mc)
               : "memory");
}
__device__ __forceinline__ void mm_ld_reduce_f32x4(const void* mc, uint32_t (&r)[4]) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(mc)
               : "memory");
}
__device__ __forceinline__ void mm_st_16(void* mc, const uint32_t (&r)[4], int dt) {
  if (dt == 0)
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
  else
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}

__global__ void allreduce_inplace_kernel(const int64_t* peer_base, long long off, long long nvec, int dt, int rank,
                                         int world, long long mc_base) {
  // my chunk of 16-byte vectors
  const long long per = (nvec + world - 1) / world;
  const long long v0 = (long long)rank * per, v1 = min(nvec, v0 + per);
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long v = v0 + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (mc_base != 0) {
    // NVLS: four independent switch reductions in flight per thread, then the broadcasts
    for (; v + 3 * stride < v1; v += 4 * stride) {
      uint32_t r[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const void* mc = reinterpret_cast<const void*>(mc_base + off + (v + u * stride) * 16);
        if (dt == 0)
          mm_ld_reduce_f32x4(mc, r[u]);
        else
          mm_ld_reduce_bf16x8(mc, r[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) mm_st_16(reinterpret_cast<void*>(mc_base + off + (v + u * stride) * 16), r[u], dt);
    }
    for (; v < v1; v += stride) {
      uint32_t r[4];
      void* mc = reinterpret_cast<void*>(mc_base + off + v * 16);
      if (dt == 0)
        mm_ld_reduce_f32x4(mc, r);
      else
        mm_ld_reduce_bf16x8(mc, r);
      mm_st_16(mc, r, dt);
    }
    return;
  }
  for (; v < v1; v += stride) {
    const long long byte = off + v * 16;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < world; ++j) {
      const int k = (j + rank) % world;
      const uint4 w = *reinterpret_cast<const uint4*>(peer_base[k] + byte);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      if (dt == 0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] += __uint_as_float(ws[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[2 * e] += bf16_bits_to_float((uint16_t)(ws[e] & 0xFFFFu));
          acc[2 * e + 1] += bf16_bits_to_float((uint16_t)(ws[e] >> 16));
        }
      }
    }
    uint4 out;
    if (dt == 0)
      out = make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]), __float_as_uint(acc[3]));
    else
      out = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                       pack_bf16x2(acc[6], acc[7]));
    for (int j = 0; j < world; ++j) *reinterpret_cast<uint4*>(peer_base[(j + rank) % world] + byte) = out;
  }
}

__device__ __forceinline__ void mm_scale(uint32_t (&r)[4], int dt, float scale) {
  if (scale == 1.f) return;
  if (dt == 0) {
#pragma unroll
    for (int e = 0; e < 4; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * scale);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bf16_bits_to_float((uint16_t)(r[e] & 0xFFFFu)) * scale;
      const float hi = bf16_bits_to_float((uint16_t)(r[e] >> 16)) * scale;
      r[e] = pack_bf16x2(lo, hi);
    }
  }
}

// Four independent multimem.ld_reduce per thread are issued before any result
// is used: a switch reduction has microseconds of latency, so one in flight per
// thread would leave the NVLink idle.
__global__ void multimem_reduce_to_local_kernel(uint4* __restrict__ out, long long mc, long long nvec, int dt,
                                                float scale) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (; v + 3 * stride < nvec; v += 4 * stride) {
    uint32_t r[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const void* addr = reinterpret_cast<const void*>(mc + (v + u * stride) * 16);
      if (dt == 0)
        mm_ld_reduce_f32x4(addr, r[u]);
      else
        mm_ld_reduce_bf16x8(addr, r[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      mm_scale(r[u], dt, scale);
      out[v + u * stride] = make_uint4(r[u][0], r[u][1], r[u][2], r[u][3]);
    }
  }
  for (; v < nvec; v += stride) {
    uint32_t r[4];
    const void* addr = reinterpret_cast<const void*>(mc + v * 16);
    if (dt == 0)
      mm_ld_reduce_f32x4(addr, r);
    else
      mm_ld_reduce_bf16x8(addr, r);
    mm_scale(r, dt, scale);
    out[v] = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

// out[i] = scale * sum_j staging[j * n + i] (local), dt 0 fp32 / 1 bf16.
__global__ void local_slot_sum_kernel(void* __restrict__ out, const void* __restrict__ staging, long long n, int world,
                                      int dt, float scale) {
  const long long n8 = n / 8;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < n8; v += (long long)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < world; ++j) {
      float x[8];
      load8(staging, dt, (long long)j * n + v * 8, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += x[e];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= scale;
    store8(out, dt, v * 8, acc);
  }
}

}  // namespace

void push_slots(const at::Tensor& src, const at::Tensor& peer_base, int64_t off, int64_t slot_bytes, int64_t rank,
                int64_t world, bool per_peer, int64_t max_ctas) {
  const at::cuda::CUDAGuard guard(src.device());
  TORCH_CHECK(src.is_contiguous() && slot_bytes % 16 == 0 && off % 16 == 0);
  TORCH_CHECK(src.numel() * src.element_size() == (per_peer ? slot_bytes * world : slot_bytes));
  const long long slot_vec = slot_bytes / 16;
  if (slot_vec == 0) return;
  const int per = (int)std::max<long long>(1, std::min<long long>(max_ctas / world, (slot_vec + 1023) / 1024));
  push_slots_kernel<<<dim3(per, (unsigned)world), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(src.data_ptr()), peer_base.data_ptr<int64_t>(), off, slot_vec, (int)rank,
      (int)world, per_peer ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void pull_slots(at::Tensor& out, const at::Tensor& peer_base, int64_t off, int64_t slot_bytes, int64_t rank,
                int64_t world, int64_t max_ctas) {
  const at::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(out.is_contiguous() && slot_bytes % 16 == 0 && off % 16 == 0 &&
              reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0);
  TORCH_CHECK(out.numel() * out.element_size() == slot_bytes * world);
  const long long slot_vec = slot_bytes / 16;
  if (slot_vec == 0) return;
  const int per = (int)std::max<long long>(1, std::min<long long>(max_ctas / world, (slot_vec + 1023) / 1024));
  pull_slots_kernel<<<dim3(per, (unsigned)world), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<uint4*>(out.data_ptr()), peer_base.data_ptr<int64_t>(), off, slot_vec, (int)rank, (int)world);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void allreduce_inplace(const at::Tensor& peer_base, int64_t off, int64_t nbytes, int64_t dtype_code, int64_t rank,
                       int64_t world, int64_t mc_base, int64_t max_ctas) {
  const at::cuda::CUDAGuard guard(peer_base.device());
  TORCH_CHECK(off % 16 == 0 && nbytes % 16 == 0 && (dtype_code == 0 || dtype_code == 1));
  TORCH_CHECK(mc_base % 16 == 0);
  const long long nvec = nbytes / 16;
  if (nvec == 0) return;
  const long long per = (nvec + world - 1) / world;
  const int blocks = (int)std::max<long long>(1, std::min<long long>(max_ctas, (per + 255) / 256));
  allreduce_inplace_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      peer_base.data_ptr<int64_t>(), off, nvec, (int)dtype_code, (int)rank, (int)world, mc_base);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void multimem_reduce_to_local(at::Tensor& out, int64_t mc_addr, double scale, int64_t max_ctas) {
  const at::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(out.is_contiguous() && (out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16));
  const long long nbytes = out.numel() * out.element_size();
  TORCH_CHECK(nbytes % 16 == 0 && mc_addr % 16 == 0 && mc_addr != 0 &&
              reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0);
  const long long nvec = nbytes / 16;
  if (nvec == 0) return;
  const int blocks = (int)std::max<long long>(1, std::min<long long>(max_ctas, (nvec + 255) / 256));
  multimem_reduce_to_local_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<uint4*>(out.data_ptr()), mc_addr, nvec, out.scalar_type() == at::kFloat ? 0 : 1, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void local_slot_sum(at::Tensor& out, const at::Tensor& staging_bytes, int64_t off, int64_t world, double scale,
                    int64_t max_ctas) {
  const at::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(out.is_contiguous() && (out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16));
  const long long n = out.numel();
  TORCH_CHECK(n % 8 == 0 && off % 16 == 0);
  if (n == 0) return;
  const int blocks = (int)std::min<long long>(max_ctas, (n / 8 + 255) / 256);
  local_slot_sum_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr(), static_cast<const char*>(staging_bytes.data_ptr()) + off, n, (int)world,
      out.scalar_type() == at::kFloat ? 0 : 1, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmb

// ---- reduce-scatter fused with the Muon momentum update (FSDP backward) ----
namespace dmb {
namespace {

constexpr int MAX_SEGS = 64;

// seg table (int64 x 5 per segment): offset, numel (valid, unpadded), momentum buffer
// pointer (0: not a Muon parameter), flags (bit0 nesterov, bit1 maximize), momentum as
// float bits. Offsets and numels are multiples of 8.
__global__ void rs_sum_momentum_kernel(void* __restrict__ out, const void* __restrict__ staging, long long n,
                                       int world, int dt, float scale, const int64_t* __restrict__ segs, int nseg) {
  __shared__ int64_t s_off[MAX_SEGS + 1], s_num[MAX_SEGS], s_buf[MAX_SEGS], s_flag[MAX_SEGS];
  __shared__ float s_mom[MAX_SEGS];
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) {
    s_off[i] = segs[i * 5 + 0];
    s_num[i] = segs[i * 5 + 1];
    s_buf[i] = segs[i * 5 + 2];
    s_flag[i] = segs[i * 5 + 3];
    s_mom[i] = __int_as_float((int)segs[i * 5 + 4]);
  }
  if (threadIdx.x == 0) s_off[nseg] = n;
  __syncthreads();
  const long long n8 = n / 8;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < n8; v += (long long)gridDim.x * blockDim.x) {
    const long long e0 = v * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < world; ++j) {
      float x[8];
      load8(staging, dt, (long long)j * n + e0, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += x[e];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= scale;
    int s = 0;
    while (s + 1 < nseg && s_off[s + 1] <= e0) ++s;
    const long long rel = e0 - s_off[s];
    if (s_buf[s] != 0 && rel < s_num[s]) {
      float* buf = reinterpret_cast<float*>(s_buf[s]);
      const float m = s_mom[s];
      const bool nesterov = s_flag[s] & 1, maximize = (s_flag[s] >> 1) & 1;
      float b[8];
      load8(buf, 0, rel, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float g = maximize ? -acc[e] : acc[e];
        b[e] = fmaf(b[e], m, g);
        acc[e] = nesterov ? fmaf(b[e], m, g) : b[e];
      }
      store8(buf, 0, rel, b);
    }
    store8(out, dt, e0, acc);
  }
}

}  // namespace

void rs_sum_momentum(at::Tensor& out, const at::Tensor& staging_bytes, int64_t off, int64_t world, double scale,
                     const at::Tensor& segs, int64_t max_ctas) {
  const at::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(out.is_contiguous() && (out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16));
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 5);
  const int nseg = segs.size(0);
  TORCH_CHECK(nseg >= 1 && nseg <= MAX_SEGS, "rs_sum_momentum: 1..64 segments");
  const long long n = out.numel();
  TORCH_CHECK(n % 8 == 0 && off % 16 == 0);
  if (n == 0) return;
  const int blocks = (int)std::min<long long>(max_ctas, (n / 8 + 255) / 256);
  rs_sum_momentum_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr(), static_cast<const char*>(staging_bytes.data_ptr()) + off, n, (int)world,
      out.scalar_type() == at::kFloat ? 0 : 1, (float)scale, segs.data_ptr<int64_t>(), nseg);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmb
