// Parameter all-gather fused into the forward GEMM (FSDP "all-gather -> first
// forward GEMM" as one kernel).
//
//   out_s[M, N_s] = x[M, K] @ W_s[N_s, K]^T  for up to 4 weights W_s (e.g. the
//   q, k, v projections, or gate and up) that share the input x. Each W_s is
//   row-sharded over `world` ranks: rank r holds rows [r * N_s/W, (r+1) * N_s/W)
//   (FSDP dim-0 shard). The gathered weights land in one local buffer
//   wg[sum N_s, K] (W_s at rows [row0_s, row0_s + N_s)), kept for the backward.
//
// One persistent cta_group::2 kernel does both the gather and the GEMM:
//   * warps 10..13 of every CTA are gather warps. They take 4 KiB pieces of W
//     from one work counter in a fixed order: first this rank's own chunks
//     (its shard -> its symmetric slot for the peers, and -> the local gathered
//     copy `wg`), then the peers' chunks (P2P 16-byte loads from the peer's
//     slot over NVLink -> `wg`). Chunk = 128 rows of wg = one CTA's half of a
//     256-row N tile; the order (own rank first, then rank + 1, ...) comes
//     from a host-built table. Every
//     finished piece bumps its chunk's done counter (release). When the last
//     local piece lands, the rank announces "slot ready for this epoch" to
//     every peer (release store at system scope into the peers' flag arrays).
//     A gather warp reads a peer's slot only after that peer's flag reached
//     this epoch (acquire, bounded wait).
//   * warp 0 (TMA producer) walks output tiles in an order that follows the
//     gather order (tiles whose chunks are all local first), so the MMA starts on
//     local data immediately and each remote chunk is needed only after the
//     gather warps had time to bring it. Before the first TMA load of a B tile
//     it waits (bounded) until its CTA's chunk counter is complete, then
//     issues a proxy fence so the async proxy sees the generic-proxy stores.
//     TMA only ever reads this GPU's own memory (x and wg); nothing is a
//     cluster-multicast load.
//   * warp 1 (leader CTA) issues tcgen05.mma.cta_group::2 into a double-buffered
//     TMEM accumulator; warps 2..9 drain it and store bf16 rows of `out`.
// Work is handed out by a counter, so progress needs only one resident CTA: no
// CTA waits for another CTA that may not have been scheduled yet.
//
// Slots are double-buffered by epoch parity. A rank rewrites slot[e & 1] in
// call e + 2 only after its call e + 1 finished, and call e + 1 cannot finish
// before every peer announced e + 1, which each peer does only after its call
// e (the last reader of slot[e & 1]) finished. Counters are parity-indexed
// too: call e zeroes the other parity's counters for call e + 1.
//
// Every wait is bounded (2 s): on expiry the kernel records an error code in
// the per-device status word and unwinds.
//
// Reference counterpart: none in muonium (it has no model or FSDP forward);
// the unfused baseline is FSDP2's all-gather followed by cuBLAS.
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

constexpr int TM = 256;
constexpr int TN = 256;  // = rows per gather chunk
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int A_STAGE = 128 * BK * 2;
constexpr int B_STAGE = 128 * BK * 2;
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int GATHER_WARPS = 4;
constexpr int THREADS = 320 + 32 * GATHER_WARPS;  // warp 0 TMA, 1 MMA, 2..9 epilogue, 10..13 gather
constexpr int FIRST_GATHER_WARP = 10;
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int PIECE_U = 8;                         // 16-byte loads in flight per lane
constexpr int PIECE_BYTES = 32 * 16 * PIECE_U;     // 4 KiB per warp-piece
constexpr int CHUNK_ROWS = 128;
constexpr int MAX_SEGS = 4;
constexpr int MAX_CHUNKS = 2048;                   // sum N_s <= 262144
constexpr int CTR_STRIDE = 2 + MAX_CHUNKS;         // [ticket, local_done, done[chunk]...]

struct Seg {
  const uint8_t* shard;  // this rank's rows of W_s (local memory)
  __nv_bfloat16* out;    // [M, rows]
  int row0, rows, rpr;   // first row in wg, total rows, rows per rank
  long long slot_off;    // byte offset of W_s's shard inside every rank's slot
};

struct AgArgs {
  int tiles_m, tiles_n, num_kb;
  int rank, world, nseg;
  Seg seg[MAX_SEGS];
  long long row_bytes;       // K * 2
  long long chunk_bytes;     // CHUNK_ROWS * row_bytes
  int ppc;                   // pieces per chunk
  int local_chunks;          // the first local_chunks entries of gather_order are this rank's
  const int* gather_order;   // [tiles_n * 2] chunk ids in gather order
  const int* tile_order;     // [tiles_n] N tiles in processing order
  uint8_t* wg;
  const int64_t* peer_base;  // [world] symmetric data buffers (world > 1)
  long long slot_base;       // this call's slot (parity) in every rank's buffer
  const int64_t* flag_base;  // [world] flag arrays (uint32 per source rank)
  unsigned epoch;
  int* ctr;                  // this call's parity block
  int* ctr_next;             // the other parity block (zeroed here for the next call)
  int* err;
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ int seg_of_row(const AgArgs& p, int row) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < MAX_SEGS; ++i)
    if (i < p.nseg && row >= p.seg[i].row0) s = i;
  return s;
}

__device__ void gather_role(const AgArgs& p, int lane, volatile int* abort_flag) {
  const int total = 2 * p.tiles_n * p.ppc;
  const int local_total = p.local_chunks * p.ppc;
  unsigned long long ready_mask = 0;  // peers seen ready (world <= 64)
  while (true) {
    int t = 0;
    if (lane == 0) t = atomicAdd(p.ctr + 0, 1);
    t = __shfl_sync(0xffffffffu, t, 0);
    if (t >= total || *abort_flag) break;
    const int j = t / p.ppc;
    const int piece = t - j * p.ppc;
    const int chunk = p.gather_order[j];
    const int row = chunk * CHUNK_ROWS;
    const Seg& sg = p.seg[seg_of_row(p, row)];
    const int rr = row - sg.row0;
    const int src_rank = rr / sg.rpr;
    const long long src_off = (long long)(rr - src_rank * sg.rpr) * p.row_bytes;  // inside the rank's shard
    const long long in_chunk = (long long)piece * PIECE_BYTES + lane * 16;
    uint4 v[PIECE_U];
    if (t < local_total) {
      const uint8_t* src = sg.shard + src_off + in_chunk;
#pragma unroll
      for (int u = 0; u < PIECE_U; ++u) v[u] = *reinterpret_cast<const uint4*>(src + u * 512);
      if (p.world > 1) {
        uint8_t* slot = reinterpret_cast<uint8_t*>(p.peer_base[p.rank]) + p.slot_base + sg.slot_off + src_off + in_chunk;
#pragma unroll
        for (int u = 0; u < PIECE_U; ++u) *reinterpret_cast<uint4*>(slot + u * 512) = v[u];
      }
    } else {
      if (!(ready_mask & (1ull << src_rank))) {
        bool ok = true;
        if (lane == 0) {
          const unsigned* f = reinterpret_cast<const unsigned*>(p.flag_base[p.rank]) + src_rank;
          const unsigned long long t0 = global_timer_ns();
          while ((int)(ld_acquire_sys(f) - p.epoch) < 0) {
            if (*abort_flag || global_timer_ns() - t0 > kWaitTimeoutNs) {
              ok = false;
              break;
            }
            __nanosleep(128);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          if (lane == 0) {
            *abort_flag = 1;
            atomicExch(p.err, (int)kErrPeerTimeout);
          }
          break;
        }
        __threadfence_system();
        ready_mask |= 1ull << src_rank;
      }
      const uint8_t* src = reinterpret_cast<const uint8_t*>(p.peer_base[src_rank]) + p.slot_base + sg.slot_off +
                           src_off + in_chunk;
#pragma unroll
      for (int u = 0; u < PIECE_U; ++u) v[u] = *reinterpret_cast<const uint4*>(src + u * 512);
    }
    uint8_t* dst = p.wg + (long long)chunk * p.chunk_bytes + in_chunk;
#pragma unroll
    for (int u = 0; u < PIECE_U; ++u) *reinterpret_cast<uint4*>(dst + u * 512) = v[u];
    fence_proxy_async_global();  // wg is read by TMA (async proxy)
    __threadfence();
    __syncwarp();
    if (lane == 0) {
      atomicAdd(p.ctr + 2 + chunk, 1);
      if (t < local_total && p.world > 1) {
        if (atomicAdd(p.ctr + 1, 1) == local_total - 1) {
          // every local piece is in this rank's slot: announce the epoch to all peers
          __threadfence_system();
          for (int k = 0; k < p.world; ++k) {
            unsigned* f = reinterpret_cast<unsigned*>(p.flag_base[k]) + p.rank;
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(p.epoch) : "memory");
          }
        }
      }
    }
    __syncwarp();
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    ag_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ AgArgs p) {
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
      mbar_init(&tempty[a], 16);
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
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = p.tiles_m * p.tiles_n;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int ready_chunk = -1;
    for (int t = cid; ok && t < total_tiles; t += ncl) {
      const int j = t / p.tiles_m;
      const int tm = t - j * p.tiles_m;
      const int tn = p.tile_order[j];
      if (tn != ready_chunk) {
        if (lane == 0) {
          const int* c = p.ctr + 2 + 2 * tn + (int)crank;  // this CTA loads rows [128 crank, +128) of the tile
          const unsigned long long t0 = global_timer_ns();
          while (ld_acquire_gpu(c) < p.ppc) {
            if (*abort_flag) {
              ok = false;
              break;
            }
            if (global_timer_ns() - t0 > kWaitTimeoutNs) {
              *abort_flag = 1;
              atomicExch(p.err, (int)kErrGemmPipelineTimeout);
              ok = false;
              break;
            }
            __nanosleep(64);
          }
          fence_proxy_async_global();
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        ready_chunk = tn;
      }
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t bar = map_to_cta(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
          tma_load_3d_pair(sA + stage * A_STAGE, &tmA, bar, kb * BK, tm * TM + (int)crank * 128, 0);
          tma_load_3d_pair(sB + stage * B_STAGE, &tmB, bar, kb * BK, tn * TN + (int)crank * 128, 0);
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
      constexpr uint32_t IDESC = idesc_bf16_f32(TM, TN, false, false);
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cid; ok && t < total_tiles; t += ncl) {
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
              const uint64_t bdesc = smem_desc_sw128(b_base + stage * B_STAGE + k * 32, 16, 1024);
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
  } else if (warp < FIRST_GATHER_WARP) {
    // ---------------------------------------------------------- epilogue --
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t tempty_leader[2] = {map_to_cta(smem_u32(&tempty[0]), 0), map_to_cta(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cid; t < total_tiles; t += ncl) {
      const int j = t / p.tiles_m;
      const int tm = t - j * p.tiles_m;
      const int tn = p.tile_order[j];
      const Seg& sg = p.seg[seg_of_row(p, tn * TN)];
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = tm * TM + (int)crank * 128 + q * 32 + lane;
#pragma unroll 1
      for (int c = half * (TN / 64); c < (half + 1) * (TN / 64); ++c) {
        uint32_t r[32];
        tmem_ld_32cols(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * TN + c * 32), r);
        const int col0 = tn * TN - sg.row0 + c * 32;
        uint4* op = reinterpret_cast<uint4*>(sg.out + (long long)row * sg.rows + col0);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 x;
          x.x = pack_bf16x2(__uint_as_float(r[u * 8 + 0]), __uint_as_float(r[u * 8 + 1]));
          x.y = pack_bf16x2(__uint_as_float(r[u * 8 + 2]), __uint_as_float(r[u * 8 + 3]));
          x.z = pack_bf16x2(__uint_as_float(r[u * 8 + 4]), __uint_as_float(r[u * 8 + 5]));
          x.w = pack_bf16x2(__uint_as_float(r[u * 8 + 6]), __uint_as_float(r[u * 8 + 7]));
          op[u] = x;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(tempty_leader[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  } else {
    // ------------------------------------------------------------ gather --
    if (blockIdx.x == 0 && warp == FIRST_GATHER_WARP) {
      for (int i = lane; i < CTR_STRIDE; i += 32) p.ctr_next[i] = 0;
    }
    gather_role(p, lane, abort_flag);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

int sm_count_ag(int dev) {
  static int cache[64] = {0};
  if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev];
}

}  // namespace

// out_s = x @ W_s^T for every segment s, with each W_s gathered from every
// rank's shard into rows [row0_s, row0_s + N_s) of wg (see the top of this file).
// x [M, K], shards[s] [N_s / world, K], wg [sum N_s, K], outs[s] [M, N_s]:
// contiguous bf16 CUDA tensors. order: int32 [2 * tiles_n + tiles_n] device
// table (gather order of the 128-row chunks, own rank's first, then the N-tile
// processing order); local_chunks: how many leading gather entries are local.
// slot_offs[s]: byte offset of shard s inside a rank's slot. peer_base /
// flag_base: int64 [world] device tensors (ignored when world == 1). counters:
// int32 [2 * (2 + 2048)], zero before the first call, owned by one stream.
void ag_gemm(const at::Tensor& x, const std::vector<at::Tensor>& shards, at::Tensor& wg,
             const std::vector<at::Tensor>& outs, const at::Tensor& order, int64_t local_chunks,
             const std::vector<int64_t>& slot_offs, const at::Tensor& peer_base, int64_t slot_base,
             const at::Tensor& flag_base, at::Tensor& counters, int64_t rank, int64_t world, int64_t epoch,
             int64_t max_pairs) {
  auto bf16_2d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
                ": contiguous 2-D bf16 CUDA tensor expected");
  };
  bf16_2d(x, "x");
  bf16_2d(wg, "wg");
  const int64_t M = x.size(0), K = x.size(1), N = wg.size(0);
  const int nseg = (int)shards.size();
  TORCH_CHECK(nseg >= 1 && nseg <= MAX_SEGS && (int)outs.size() == nseg && (int)slot_offs.size() == nseg,
              "1..4 segments with one output and slot offset each");
  TORCH_CHECK(world >= 1 && world <= 64 && rank >= 0 && rank < world, "bad rank/world");
  TORCH_CHECK(M % 256 == 0 && K % 64 == 0 && wg.size(1) == K, "M must be a multiple of 256, K of 64");
  TORCH_CHECK(N % 256 == 0 && N / CHUNK_ROWS <= MAX_CHUNKS, "sum of rows must be a multiple of 256, at most 262144");
  const at::cuda::CUDAGuard guard(x.device());
  const int dev = x.get_device();
  AgArgs p{};
  p.tiles_m = (int)(M / 256);
  p.tiles_n = (int)(N / 256);
  p.num_kb = (int)(K / BK);
  p.rank = (int)rank;
  p.world = (int)world;
  p.nseg = nseg;
  int row0 = 0;
  for (int i = 0; i < nseg; ++i) {
    bf16_2d(shards[i], "shard");
    bf16_2d(outs[i], "out");
    const int64_t rows = shards[i].size(0) * world;
    TORCH_CHECK(shards[i].size(1) == K && shards[i].size(0) % CHUNK_ROWS == 0 && rows % 256 == 0,
                "shard s: [N_s / world, K] with N_s / world a multiple of 128 and N_s a multiple of 256");
    TORCH_CHECK(outs[i].size(0) == M && outs[i].size(1) == rows, "out s must be [M, N_s]");
    TORCH_CHECK(slot_offs[i] % 16 == 0, "slot offsets must be 16-byte aligned");
    p.seg[i].shard = reinterpret_cast<const uint8_t*>(shards[i].data_ptr());
    p.seg[i].out = reinterpret_cast<__nv_bfloat16*>(outs[i].data_ptr());
    p.seg[i].row0 = row0;
    p.seg[i].rows = (int)rows;
    p.seg[i].rpr = (int)shards[i].size(0);
    p.seg[i].slot_off = slot_offs[i];
    row0 += (int)rows;
  }
  TORCH_CHECK(row0 == N, "wg must have sum N_s rows");
  TORCH_CHECK(order.is_cuda() && order.scalar_type() == at::kInt && order.numel() == 3 * p.tiles_n,
              "order: int32 [3 * N / 256]");
  TORCH_CHECK(local_chunks >= 0 && local_chunks <= 2 * p.tiles_n);
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= 2 * CTR_STRIDE,
              "counters: int32 [2 * (2 + 2048)]");
  if (world > 1) {
    TORCH_CHECK(peer_base.is_cuda() && peer_base.scalar_type() == at::kLong && peer_base.numel() == world);
    TORCH_CHECK(flag_base.is_cuda() && flag_base.scalar_type() == at::kLong && flag_base.numel() == world);
    TORCH_CHECK(slot_base % 16 == 0, "slot base must be 16-byte aligned");
  }
  p.row_bytes = K * 2;
  p.chunk_bytes = CHUNK_ROWS * p.row_bytes;
  p.ppc = (int)(p.chunk_bytes / PIECE_BYTES);
  p.local_chunks = (int)local_chunks;
  p.gather_order = order.data_ptr<int>();
  p.tile_order = order.data_ptr<int>() + 2 * p.tiles_n;
  p.wg = reinterpret_cast<uint8_t*>(wg.data_ptr());
  p.peer_base = world > 1 ? peer_base.data_ptr<int64_t>() : nullptr;
  p.slot_base = slot_base;
  p.flag_base = world > 1 ? flag_base.data_ptr<int64_t>() : nullptr;
  p.epoch = (unsigned)epoch;
  int* ctr = counters.data_ptr<int>();
  p.ctr = ctr + (epoch & 1) * CTR_STRIDE;
  p.ctr_next = ctr + ((epoch + 1) & 1) * CTR_STRIDE;
  p.err = device_error_word(dev);

  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(ag_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured[dev] = true;
  }
  auto x3 = x.view({1, M, K});
  auto w3 = wg.view({1, N, K});
  CUtensorMap ma = make_bf16_map_3d(x3, BK, 128);
  CUtensorMap mb = make_bf16_map_3d(w3, BK, 128);
  int pairs = sm_count_ag(dev) / 2;
  if (max_pairs > 0) pairs = std::min<int>(pairs, (int)max_pairs);
  pairs = std::max(1, std::min(pairs, p.tiles_m * p.tiles_n));
  ag_gemm_kernel<<<2 * pairs, THREADS, SMEM_BYTES, at::cuda::getCurrentCUDAStream()>>>(ma, mb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmb
