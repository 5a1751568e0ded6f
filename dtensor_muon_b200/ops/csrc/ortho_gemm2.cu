// 2-SM (cta_group::2) variant of the orthogonalisation GEMM engine.
//
// Same three fused epilogues as ortho_gemm.cu (symmetric Gram, c A A + b A,
// alpha B X + beta X), but a CTA pair (cluster of 2) computes one 256 x 256
// output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16):
//   * each CTA stages its own 128 rows of A and 128 of the 256 B rows/cols,
//     so per-CTA operand traffic per FLOP is 2/3 of the 1-SM 128 x 256 tile
//     and a stage is 32 KiB -> 6 stages in 192 KiB;
//   * both CTAs' TMA loads (plain tile loads, no multicast) complete on the
//     leader CTA's full barrier (cp.async.bulk.tensor ... .cta_group::2);
//   * the leader's single MMA thread issues the pair's MMAs; its commits
//     arrive on both CTAs' barriers (tcgen05.commit ... .multicast::cluster);
//   * each CTA drains its own 128 TMEM lanes; epilogue warps of both CTAs
//     release the accumulator on the leader's barrier (remote arrive).
// Every wait is bounded as in ortho_gemm.cu.
// Reference counterpart: the Triton gram_nd (src/muonium/kernels/gram.py:25-106)
// and the loops of ns_loop_triton / pe_loop_triton (newton_schulz.py:89-103,
// polar_express.py:96-110).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "pair.cuh"

namespace dmb {

int* device_error_word(int dev);
CUtensorMap make_bf16_map_3d(const at::Tensor& t, int box_cols, int box_rows);

namespace {

using namespace pair;

constexpr int TM = 256;  // pair tile rows (128 per CTA)
constexpr int TN = 256;  // pair tile cols
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int A_STAGE = 128 * BK * 2;   // 16 KiB
constexpr int B_STAGE = 128 * BK * 2;   // 16 KiB (this CTA's half of B)
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;

struct Epi2 {
  int tiles_m, tiles_n, tiles_per_batch, total_tiles, num_kb;
  __nv_bfloat16* out;
  long long out_bstride;
  int ldo;
  const __nv_bfloat16* res;
  long long res_bstride;
  int ldr;
  const float* scale;
  float coef_acc, coef_res;
  int acc_pow, res_pow;
  int* err;
};

__device__ __forceinline__ float ipow2(float s, int p) {
  float r = 1.f;
  for (int i = 0; i < p; ++i) r *= s;
  return r;
}

template <bool SYM>
__device__ __forceinline__ void decode2(const Epi2& p, int t, int& b, int& tm, int& tn) {
  b = t / p.tiles_per_batch;
  int r = t - b * p.tiles_per_batch;
  if (SYM) {  // square 256 tiles with tm <= tn; column tn owns tn + 1 tiles
    int c = (int)((sqrtf(8.f * (float)r + 1.f) - 1.f) * 0.5f);
    while ((c + 1) * (c + 2) / 2 <= r) ++c;
    while (c * (c + 1) / 2 > r) --c;
    tn = c;
    tm = r - c * (c + 1) / 2;
  } else {
    tn = r / p.tiles_m;
    tm = r - tn * p.tiles_m;
  }
}

template <bool SYM, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    ortho_gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const Epi2 p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_rank();
  const bool leader = crank == 0;
  const int cid = (int)cluster_id(), ncl = (int)num_clusters();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 16);  // 8 epilogue warps x 2 CTAs
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = cid; ok && t < p.total_tiles; t += ncl) {
      int b, tm, tn;
      decode2<SYM>(p, t, b, tm, tn);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t bar = map_to_cta(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
          tma_load_3d_pair(sA + stage * A_STAGE, &tmA, bar, kb * BK, tm * TM + (int)crank * 128, b);
          if (!B_MN) {
            tma_load_3d_pair(sB + stage * B_STAGE, &tmB, bar, kb * BK, tn * TN + (int)crank * 128, b);
          } else {
#pragma unroll
            for (int q = 0; q < 2; ++q)
              tma_load_3d_pair(sB + stage * B_STAGE + q * (64 * BK * 2), &tmB, bar,
                               tn * TN + (int)crank * 128 + q * 64, kb * BK, b);
          }
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok) {
      const unsigned long long t0 = global_timer_ns();
      while (global_timer_ns() - t0 < 1000000ull) __nanosleep(1000);
    }
  } else if (warp == 1) {
    // ---------------------------------------- MMA issue (leader CTA only) --
    if (leader) {
      constexpr uint32_t IDESC = idesc_bf16_f32(TM, TN, false, B_MN);
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cid; ok && t < p.total_tiles; t += ncl) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * TN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t adesc = smem_desc_sw128(a_base + stage * A_STAGE + k * 32, 16, 1024);
              const uint64_t bdesc =
                  B_MN ? smem_desc_sw128(b_base + stage * B_STAGE + k * 2048, 64 * BK * 2, 1024)
                       : smem_desc_sw128(b_base + stage * B_STAGE + k * 32, 16, 1024);
              mma_pair(d_tmem, adesc, bdesc, IDESC, (kb | k) != 0 ? 1u : 0u);
            }
            commit_pair(&empty[stage]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) commit_pair(&tfull[acc]);
        __syncwarp();
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    // Two warps per TMEM lane quadrant (warp & 3), each draining half of the
    // 256 accumulator columns, so short-K tiles are not epilogue-bound.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t tempty_leader[2] = {map_to_cta(smem_u32(&tempty[0]), 0), map_to_cta(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cid; t < p.total_tiles; t += ncl) {
      int b, tm, tn;
      decode2<SYM>(p, t, b, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err)) break;
      tc_fence_after();
      const float s = p.scale ? p.scale[b] : 1.f;
      const float alpha = p.coef_acc * ipow2(s, p.acc_pow);
      const float beta = p.coef_res * ipow2(s, p.res_pow);
      const int row = tm * TM + (int)crank * 128 + q * 32 + lane;
      __nv_bfloat16* out_b = p.out + (long long)b * p.out_bstride;
      const __nv_bfloat16* res_b = p.res ? p.res + (long long)b * p.res_bstride : nullptr;
#pragma unroll 1
      for (int c = half * (TN / 64); c < (half + 1) * (TN / 64); ++c) {
        uint32_t r[32];
        tmem_ld_32cols(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * TN + c * 32), r);
        const int col0 = tn * TN + c * 32;
        if (SYM && row > col0 + 31) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = alpha * __uint_as_float(r[j]);
        if (res_b) {
          const uint4* rp = reinterpret_cast<const uint4*>(res_b + (long long)row * p.ldr + col0);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 x = __ldg(rp + u);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              v[u * 8 + h * 2 + 0] += beta * bf16_bits_to_float((uint16_t)(w[h] & 0xFFFFu));
              v[u * 8 + h * 2 + 1] += beta * bf16_bits_to_float((uint16_t)(w[h] >> 16));
            }
          }
        }
        if (!SYM || row <= col0) {
          uint4* op = reinterpret_cast<uint4*>(out_b + (long long)row * p.ldo + col0);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 x;
            x.x = pack_bf16x2(v[u * 8 + 0], v[u * 8 + 1]);
            x.y = pack_bf16x2(v[u * 8 + 2], v[u * 8 + 3]);
            x.z = pack_bf16x2(v[u * 8 + 4], v[u * 8 + 5]);
            x.w = pack_bf16x2(v[u * 8 + 6], v[u * 8 + 7]);
            op[u] = x;
          }
          if (SYM) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (row < col0 + j) out_b[(long long)(col0 + j) * p.ldo + row] = __float2bfloat16_rn(v[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = col0 + j;
            if (row <= col) {
              const __nv_bfloat16 hv = __float2bfloat16_rn(v[j]);
              out_b[(long long)row * p.ldo + col] = hv;
              if (row < col) out_b[(long long)col * p.ldo + row] = hv;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(tempty_leader[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

int sm_count(int dev) {
  static int cache[64] = {0};
  if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev];
}

template <bool SYM, bool B_MN>
void launch2(const CUtensorMap& ma, const CUtensorMap& mb, const Epi2& p, cudaStream_t st) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(ortho_gemm2_kernel<SYM, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_BYTES));
    configured[dev] = true;
  }
  const int pairs = std::min(p.total_tiles, sm_count(dev) / 2);
  if (pairs <= 0) return;
  // Cluster shape (2,1,1) comes from __cluster_dims__ on the kernel.
  ortho_gemm2_kernel<SYM, B_MN><<<2 * pairs, THREADS, SMEM_BYTES, st>>>(ma, mb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void fill_common(Epi2& p, at::Tensor& out, const c10::optional<at::Tensor>& res, const c10::optional<at::Tensor>& scale,
                 int B, double coef_acc, double coef_res, int64_t acc_pow, int64_t res_pow) {
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_bstride = out.stride(0);
  p.ldo = out.stride(1);
  if (res.has_value()) {
    TORCH_CHECK(res->sizes() == out.sizes() && res->is_contiguous() && res->scalar_type() == at::kBFloat16);
    p.res = reinterpret_cast<const __nv_bfloat16*>(res->data_ptr());
    p.res_bstride = res->stride(0);
    p.ldr = res->stride(1);
  }
  if (scale.has_value()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->numel() >= B && scale->is_cuda());
    p.scale = scale->data_ptr<float>();
  }
  p.coef_acc = (float)coef_acc;
  p.coef_res = (float)coef_res;
  p.acc_pow = (int)acc_pow;
  p.res_pow = (int)res_pow;
  p.err = device_error_word(out.get_device());
}

void check_ws2(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 3 && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
              ": contiguous bf16 [B,R,C] CUDA tensor expected");
  TORCH_CHECK(t.size(1) % 256 == 0 && t.size(2) % 256 == 0, name, ": rows/cols must be multiples of 256");
}

}  // namespace

void gram_sym2(const at::Tensor& x, at::Tensor& out, const c10::optional<at::Tensor>& res,
               const c10::optional<at::Tensor>& scale, double coef_acc, double coef_res, int64_t acc_pow,
               int64_t res_pow) {
  check_ws2(x, "x");
  check_ws2(out, "out");
  const int B = x.size(0), N = x.size(1), K = x.size(2);
  TORCH_CHECK(out.size(0) == B && out.size(1) == N && out.size(2) == N);
  const at::cuda::CUDAGuard guard(x.device());
  Epi2 p{};
  const int T = N / 256;
  p.tiles_m = T;
  p.tiles_n = T;
  p.tiles_per_batch = T * (T + 1) / 2;
  p.total_tiles = B * p.tiles_per_batch;
  p.num_kb = K / BK;
  fill_common(p, out, res, scale, B, coef_acc, coef_res, acc_pow, res_pow);
  CUtensorMap ma = make_bf16_map_3d(x, BK, 128);
  launch2<true, false>(ma, ma, p, at::cuda::getCurrentCUDAStream());
}

void gemm_ax2(const at::Tensor& a, const at::Tensor& x, at::Tensor& out, const c10::optional<at::Tensor>& res,
              const c10::optional<at::Tensor>& scale, double coef_acc, double coef_res, int64_t acc_pow,
              int64_t res_pow) {
  check_ws2(a, "a");
  check_ws2(x, "x");
  check_ws2(out, "out");
  const int B = x.size(0), N = x.size(1), M = x.size(2);
  TORCH_CHECK(a.size(0) == B && a.size(1) == N && a.size(2) == N && out.sizes() == x.sizes());
  const at::cuda::CUDAGuard guard(x.device());
  Epi2 p{};
  p.tiles_m = N / 256;
  p.tiles_n = M / 256;
  p.tiles_per_batch = p.tiles_m * p.tiles_n;
  p.total_tiles = B * p.tiles_per_batch;
  p.num_kb = N / BK;
  fill_common(p, out, res, scale, B, coef_acc, coef_res, acc_pow, res_pow);
  CUtensorMap ma = make_bf16_map_3d(a, BK, 128);
  CUtensorMap mb = make_bf16_map_3d(x, 64, BK);
  launch2<false, true>(ma, mb, p, at::cuda::getCurrentCUDAStream());
}

}  // namespace dmb
