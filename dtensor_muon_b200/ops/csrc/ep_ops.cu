// Expert-parallel token exchange over NVLink peer memory.
//
// Two row-movement kernels over a symmetric buffer that every rank of the EP
// group can address (new: the reference has no MoE or expert-parallel token
// exchange):
//   ep_scatter_rows  row i of `src` -> rank dst_rank[i], row dst_row[i] of that
//                    rank's receive region (P2P 16-byte stores)
//   ep_gather_rows   row i of `dst` <- rank src_rank[i], row src_row[i] of that
//                    rank's region (P2P 16-byte loads)
// Dispatch is a scatter whose destination rows are pre-sorted by local expert,
// so the receiver's rows are already grouped for the expert GEMMs; combine is
// the matching gather. Backward of each is the other. Synchronisation is the
// bounded device barrier of dist_ops.cu, issued by the caller.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

namespace dmb {
namespace {

__global__ void ep_scatter_rows_kernel(const uint4* __restrict__ src, const int* dst_rank, const int* dst_row,
                                       const int64_t* peer_base, long long off, int vec_per_row) {
  const int i = blockIdx.x;
  uint4* dst = reinterpret_cast<uint4*>(peer_base[dst_rank[i]] + off) + (long long)dst_row[i] * vec_per_row;
  const uint4* s = src + (long long)i * vec_per_row;
  for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) dst[v] = s[v];
}

__global__ void ep_gather_rows_kernel(uint4* __restrict__ dst, const int* src_rank, const int* src_row,
                                      const int64_t* peer_base, long long off, int vec_per_row) {
  const int i = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(peer_base[src_rank[i]] + off) + (long long)src_row[i] * vec_per_row;
  uint4* d = dst + (long long)i * vec_per_row;
  for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) d[v] = s[v];
}

}  // namespace

void ep_scatter_rows(const at::Tensor& src, const at::Tensor& dst_rank, const at::Tensor& dst_row,
                     const at::Tensor& peer_base, int64_t off) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous() && src.dim() == 2);
  const int64_t row_bytes = src.size(1) * src.element_size();
  TORCH_CHECK(row_bytes % 16 == 0 && off % 16 == 0, "rows must be 16-byte multiples");
  const int n = src.size(0);
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(src.device());
  const int vec = row_bytes / 16;
  ep_scatter_rows_kernel<<<n, std::min(256, std::max(32, vec)), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(src.data_ptr()), dst_rank.data_ptr<int>(), dst_row.data_ptr<int>(),
      peer_base.data_ptr<int64_t>(), off, vec);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_gather_rows(at::Tensor& dst, const at::Tensor& src_rank, const at::Tensor& src_row,
                    const at::Tensor& peer_base, int64_t off) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous() && dst.dim() == 2);
  const int64_t row_bytes = dst.size(1) * dst.element_size();
  TORCH_CHECK(row_bytes % 16 == 0 && off % 16 == 0, "rows must be 16-byte multiples");
  const int n = dst.size(0);
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(dst.device());
  const int vec = row_bytes / 16;
  ep_gather_rows_kernel<<<n, std::min(256, std::max(32, vec)), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<uint4*>(dst.data_ptr()), src_rank.data_ptr<int>(), src_row.data_ptr<int>(),
      peer_base.data_ptr<int64_t>(), off, vec);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmb
