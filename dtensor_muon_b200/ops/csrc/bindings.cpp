// Python bindings for the dtensor_muon_b200 sm_100a kernels (module `_C`).
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <mutex>

namespace dmb {

// ---- ortho_gemm.cu
void gram_sym(const at::Tensor& x, at::Tensor& out, const c10::optional<at::Tensor>& res,
              const c10::optional<at::Tensor>& scale, double coef_acc, double coef_res, int64_t acc_pow,
              int64_t res_pow, int64_t max_ctas);
void gemm_ax(const at::Tensor& a, const at::Tensor& x, at::Tensor& out, const c10::optional<at::Tensor>& res,
             const c10::optional<at::Tensor>& scale, double coef_acc, double coef_res, int64_t acc_pow,
             int64_t res_pow, int64_t max_ctas);
at::Tensor ortho_iterate(at::Tensor x, at::Tensor x2, at::Tensor a_ws, at::Tensor b_ws, const at::Tensor& inv_norm,
                         const at::Tensor& coeffs, int64_t max_ctas);
void gram_sym2(const at::Tensor& x, at::Tensor& out, const c10::optional<at::Tensor>& res,
               const c10::optional<at::Tensor>& scale, double coef_acc, double coef_res, int64_t acc_pow,
               int64_t res_pow);
void gemm_ax2(const at::Tensor& a, const at::Tensor& x, at::Tensor& out, const c10::optional<at::Tensor>& res,
              const c10::optional<at::Tensor>& scale, double coef_acc, double coef_res, int64_t acc_pow,
              int64_t res_pow);
void set_gemm_variant(int64_t v);
int64_t get_gemm_variant();
// ---- muon_ops.cu
at::Tensor muon_pack(const at::Tensor& src_ptrs, const c10::optional<at::Tensor>& buf_ptrs, int64_t src_dtype_code,
                     int64_t R, int64_t C, int64_t ld, bool transpose, at::Tensor& out, double momentum,
                     bool nesterov, bool maximize);
at::Tensor muon_pack_ex(const at::Tensor& src_ptrs, const c10::optional<at::Tensor>& buf_ptrs, int64_t src_dtype_code,
                        int64_t R, int64_t C, int64_t ld, bool transpose, at::Tensor& out, double momentum,
                        bool nesterov, bool maximize, bool vec_ok);
void muon_apply_ex(const at::Tensor& ws, bool transpose, int64_t R, int64_t C, int64_t ld, const at::Tensor& dst_ptrs,
                   int64_t dst_dtype_code, const c10::optional<at::Tensor>& rowscale,
                   const c10::optional<at::Tensor>& mat_scale, double lr_eff, double wd, bool cautious, bool vec_ok);
at::Tensor norm_finalize(const at::Tensor& partial, double fac, double eps);
void muon_apply(const at::Tensor& ws, bool transpose, int64_t R, int64_t C, int64_t ld, const at::Tensor& dst_ptrs,
                int64_t dst_dtype_code, const c10::optional<at::Tensor>& rowscale,
                const c10::optional<at::Tensor>& mat_scale, double lr_eff, double wd, bool cautious);
at::Tensor muon_unpack(const at::Tensor& ws, bool transpose, int64_t R, int64_t C,
                       const c10::optional<at::Tensor>& mat_scale);
at::Tensor row_sumsq(const at::Tensor& ws, bool transpose, int64_t R, int64_t C);
at::Tensor normuon_finalize(const at::Tensor& rowsq, const at::Tensor& v_ptrs, int64_t C, double beta2);
// ---- adamw.cu
void adamw_multi(at::Tensor meta_cpu, double lr, double beta1, double beta2, double eps, double wd, bool decoupled,
                 bool amsgrad, bool maximize, const at::Device& device);
// ---- lp_quant.cu
void lp_momentum_step(at::Tensor codes, at::Tensor scale, const at::Tensor& qmap, int64_t fmt, int64_t block,
                      const at::Tensor& grad, at::Tensor gout, double momentum, bool nesterov, bool maximize);
at::Tensor lp_dequantize(const at::Tensor& codes, const at::Tensor& scale, const at::Tensor& qmap, int64_t fmt,
                         int64_t block, int64_t n);
void lp_quantize(const at::Tensor& x, at::Tensor codes, at::Tensor scale, const at::Tensor& qmap, int64_t fmt,
                 int64_t block);

// ---- dist_ops.cu
void dist_pack(const at::Tensor& meta_i64, const at::Tensor& meta_i32, const at::Tensor& peer_base,
               std::vector<int64_t> ints, std::vector<double> floats, bool has_buf, bool has_var);
void dist_apply(const at::Tensor& meta_i64, const at::Tensor& meta_i32, const at::Tensor& peer_base,
                std::vector<int64_t> ints, std::vector<double> floats, bool has_var);
void dist_barrier(const at::Tensor& flag_base, int64_t rank, int64_t world, int64_t epoch);
void push_slots(const at::Tensor& src, const at::Tensor& peer_base, int64_t off, int64_t slot_bytes, int64_t rank,
                int64_t world, bool per_peer, int64_t max_ctas);
void pull_slots(at::Tensor& out, const at::Tensor& peer_base, int64_t off, int64_t slot_bytes, int64_t rank,
                int64_t world, int64_t max_ctas);
void ag_gemm(const at::Tensor& x, const std::vector<at::Tensor>& shards, at::Tensor& wg,
             const std::vector<at::Tensor>& outs, const at::Tensor& order, int64_t local_chunks,
             const std::vector<int64_t>& slot_offs, const at::Tensor& peer_base, int64_t slot_base,
             const at::Tensor& flag_base, at::Tensor& counters, int64_t rank, int64_t world, int64_t epoch,
             int64_t max_pairs);
void allreduce_inplace(const at::Tensor& peer_base, int64_t off, int64_t nbytes, int64_t dtype_code, int64_t rank,
                       int64_t world, int64_t mc_base, int64_t max_ctas);
void flag_signal(const at::Tensor& flag_base, int64_t slot, int64_t rank, int64_t world, int64_t epoch);
void flag_wait(const at::Tensor& flag_base, int64_t slot, int64_t rank, int64_t world, int64_t epoch);
void multimem_reduce_to_local(at::Tensor& out, int64_t mc_addr, double scale, int64_t max_ctas);
void local_slot_sum(at::Tensor& out, const at::Tensor& staging_bytes, int64_t off, int64_t world, double scale,
                    int64_t max_ctas);
void rs_sum_momentum(at::Tensor& out, const at::Tensor& staging_bytes, int64_t off, int64_t world, double scale,
                     const at::Tensor& segs, int64_t max_ctas);


// ---- ep_ops.cu
void ep_scatter_rows(const at::Tensor& src, const at::Tensor& dst_rank, const at::Tensor& dst_row,
                     const at::Tensor& peer_base, int64_t off);
void ep_gather_rows(at::Tensor& dst, const at::Tensor& src_rank, const at::Tensor& src_row,
                    const at::Tensor& peer_base, int64_t off);

// ---- model_ops.cu
at::Tensor rope(const at::Tensor& x, const at::Tensor& cos_t, const at::Tensor& sin_t, double sign);
at::Tensor swiglu_fwd(const at::Tensor& a, const at::Tensor& b);
std::vector<at::Tensor> swiglu_bwd(const at::Tensor& a, const at::Tensor& b, const at::Tensor& dh);
std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& targets);
at::Tensor cross_entropy_bwd(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse,
                             double scale, const c10::optional<at::Tensor>& gscale);

// One status word per device. Kernels whose bounded waits give up write an
// error code here; the host reads and clears it with take_device_error().
int* device_error_word(int dev) {
  static int* words[64] = {nullptr};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    c10::cuda::CUDAGuard g(dev);
    int* p = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
    words[dev] = p;
  }
  return words[dev];
}

int64_t take_device_error(int64_t dev) {
  int* w = device_error_word((int)dev);
  c10::cuda::CUDAGuard g((int)dev);
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
  return v;
}

}  // namespace dmb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dtensor_muon_b200 sm_100a kernels";
  m.def("gram_sym", &dmb::gram_sym);
  m.def("gemm_ax", &dmb::gemm_ax);
  m.def("ortho_iterate", &dmb::ortho_iterate);
  m.def("gram_sym2", &dmb::gram_sym2);
  m.def("gemm_ax2", &dmb::gemm_ax2);
  m.def("set_gemm_variant", &dmb::set_gemm_variant);
  m.def("get_gemm_variant", &dmb::get_gemm_variant);
  m.def("muon_pack", &dmb::muon_pack);
  m.def("muon_pack_ex", &dmb::muon_pack_ex);
  m.def("muon_apply_ex", &dmb::muon_apply_ex);
  m.def("norm_finalize", &dmb::norm_finalize);
  m.def("muon_apply", &dmb::muon_apply);
  m.def("muon_unpack", &dmb::muon_unpack);
  m.def("row_sumsq", &dmb::row_sumsq);
  m.def("normuon_finalize", &dmb::normuon_finalize);
  m.def("adamw_multi", &dmb::adamw_multi);
  m.def("lp_momentum_step", &dmb::lp_momentum_step);
  m.def("lp_dequantize", &dmb::lp_dequantize);
  m.def("lp_quantize", &dmb::lp_quantize);
  m.def("dist_pack", &dmb::dist_pack);
  m.def("dist_apply", &dmb::dist_apply);
  m.def("dist_barrier", &dmb::dist_barrier);
  m.def("push_slots", &dmb::push_slots);
  m.def("local_slot_sum", &dmb::local_slot_sum);
  m.def("pull_slots", &dmb::pull_slots);
  m.def("allreduce_inplace", &dmb::allreduce_inplace);
  m.def("ag_gemm", &dmb::ag_gemm);
  m.def("flag_signal", &dmb::flag_signal);
  m.def("multimem_reduce_to_local", &dmb::multimem_reduce_to_local);
  m.def("flag_wait", &dmb::flag_wait);
  m.def("rs_sum_momentum", &dmb::rs_sum_momentum);
  m.def("ep_scatter_rows", &dmb::ep_scatter_rows);
  m.def("ep_gather_rows", &dmb::ep_gather_rows);
  m.def("rope", &dmb::rope);
  m.def("swiglu_fwd", &dmb::swiglu_fwd);
  m.def("swiglu_bwd", &dmb::swiglu_bwd);
  m.def("cross_entropy_fwd", &dmb::cross_entropy_fwd);
  m.def("cross_entropy_bwd", &dmb::cross_entropy_bwd);
  m.def("take_device_error", &dmb::take_device_error);
}
