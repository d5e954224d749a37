// Python bindings of the femtotron_b200 native extension (module femtotron_b200._C).
#include <torch/extension.h>

namespace ft {
void gemm_tc(const torch::Tensor& A, const torch::Tensor& B, torch::Tensor& D, bool a_mn,
             bool b_mn, int64_t mode, const c10::optional<torch::Tensor>& R,
             const c10::optional<torch::Tensor>& GU, int64_t gate_up_off, torch::Tensor& err);
void rmsnorm_fwd(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& y,
                 torch::Tensor& rstd, double eps);
void rmsnorm_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& w,
                 const torch::Tensor& rstd, torch::Tensor& dx, torch::Tensor& dw_acc);
void rope_apply(torch::Tensor& qk, const torch::Tensor& cos_t, const torch::Tensor& sin_t,
                const c10::optional<torch::Tensor>& pos, int64_t nheads, int64_t head_dim,
                int64_t seq_len, bool inverse);
void swiglu_fwd(const torch::Tensor& gu, torch::Tensor& h, int64_t F);
void swiglu_bwd(const torch::Tensor& dh, const torch::Tensor& gu, torch::Tensor& dgu, int64_t F);
void xent_stats(const torch::Tensor& logits, const torch::Tensor& labels, torch::Tensor& stats,
                int64_t vstart);
void xent_bwd(torch::Tensor& logits, const torch::Tensor& labels, const torch::Tensor& lse,
              const torch::Tensor& grad_scale, int64_t vstart, int64_t ignore_index);
void embed_fwd(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out,
               int64_t vstart);
void embed_bwd(const torch::Tensor& ids, const torch::Tensor& dout, torch::Tensor& dtable,
               int64_t vstart);
void adamw_multi(const std::vector<torch::Tensor>& params, const std::vector<torch::Tensor>& ms,
                 const std::vector<torch::Tensor>& vs, const std::vector<torch::Tensor>& grads,
                 const std::vector<torch::Tensor>& p16s, const std::vector<double>& wds,
                 double lr, double beta1, double beta2, double eps, int64_t step,
                 const c10::optional<torch::Tensor>& grad_scale);
void sumsq_multi(const std::vector<torch::Tensor>& xs, const std::vector<int64_t>& slots,
                 torch::Tensor& out);
torch::Tensor symm_alloc(int64_t nbytes, int64_t device);
torch::Tensor ipc_handle(const torch::Tensor& t);
int64_t ipc_open(const torch::Tensor& handle, int64_t device);
void ipc_close(int64_t ptr);
torch::Tensor tensor_at(int64_t ptr, int64_t numel, torch::ScalarType dtype, int64_t device);
void copy_from_ptrs(const std::vector<int64_t>& dsts, const std::vector<int64_t>& srcs,
                    const std::vector<int64_t>& nbytes);
void gemm_tc_fused(const torch::Tensor& A, const torch::Tensor& B, torch::Tensor& D, bool a_mn,
                   bool b_mn, int64_t mode,
                   const c10::optional<torch::Tensor>& R, const c10::optional<torch::Tensor>& GU,
                   int64_t gate_up_off, torch::Tensor& err, int64_t gate_flags, int64_t gate_op,
                   int64_t gate_epoch, int64_t gate_off, int64_t gate_row_elems,
                   int64_t gate_chunk_elems, const std::vector<int64_t>& scatter_ptrs,
                   int64_t scatter_rows, int64_t m_rot_rows, int64_t reserved_sms);
void wait_flags_geq(const std::vector<int64_t>& addrs, int64_t value, torch::Tensor& err,
                    int64_t timeout_ms, int64_t code);
void rs_adamw(const std::vector<int64_t>& src_ptrs, int64_t base, int64_t n, bool src_f32,
              double scale, bool accumulate, torch::Tensor& grad_shard, bool store_grad,
              const c10::optional<torch::Tensor>& master, const c10::optional<torch::Tensor>& m,
              const c10::optional<torch::Tensor>& v, const c10::optional<torch::Tensor>& p16,
              const c10::optional<torch::Tensor>& segments, double beta1, double beta2,
              double eps, int64_t step);
void stream_write(int64_t addr, int64_t value);
int64_t gate_reserved_sms();
bool nvls_supported(int64_t device);
int64_t nvls_round_size(int64_t device, int64_t world, int64_t nbytes);
int64_t nvls_create(int64_t device, int64_t world, int64_t size);
int64_t nvls_export_fd(int64_t id);
int64_t nvls_import(int64_t device, int64_t world, int64_t size, int64_t fd);
void nvls_add_device(int64_t id);
std::vector<int64_t> nvls_bind_map(int64_t id);
void nvls_close(int64_t id);
void nvls_barrier(int64_t uc_base, int64_t mc_base, int64_t flag_off, int64_t target,
                  torch::Tensor& err, int64_t code, int64_t timeout_ms);
void nvls_reduce_slice(int64_t mc_base, int64_t nbytes, int64_t rank, int64_t world, bool f32,
                       double scale);
void ag_pull(const std::vector<int64_t>& src_ptrs, const std::vector<int64_t>& ready_ptrs,
             torch::Tensor& dst, int64_t chunk_bytes, int64_t chunk_count_ptr, int64_t me,
             int64_t epoch, int64_t ctas, torch::Tensor& err, int64_t timeout_ms);
void rs_pull(const std::vector<int64_t>& src_ptrs, const std::vector<int64_t>& part_ptrs,
             const c10::optional<torch::Tensor>& resid, torch::Tensor& out, int64_t nelem,
             int64_t epoch, torch::Tensor& err, int64_t timeout_ms);
void flash_fwd(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t S,
               int64_t nq, int64_t nkv, int64_t D, torch::Tensor& err);
void flash_fwd_variant(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B,
                       int64_t S, int64_t nq, int64_t nkv, int64_t D, torch::Tensor& err,
                       int64_t variant);
void flash_bwd(const torch::Tensor& qkv, const torch::Tensor& o, const torch::Tensor& dout,
               const torch::Tensor& lse, torch::Tensor& dqkv, int64_t B, int64_t S, int64_t nq,
               int64_t nkv, int64_t D, torch::Tensor& err);
}  // namespace ft

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "femtotron_b200 sm_100a kernels";
  m.def("gemm_tc", &ft::gemm_tc, "tcgen05 GEMM with fused epilogues");
  m.def("rmsnorm_fwd", &ft::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &ft::rmsnorm_bwd);
  m.def("rope_apply", &ft::rope_apply);
  m.def("swiglu_fwd", &ft::swiglu_fwd);
  m.def("swiglu_bwd", &ft::swiglu_bwd);
  m.def("xent_stats", &ft::xent_stats);
  m.def("xent_bwd", &ft::xent_bwd);
  m.def("embed_fwd", &ft::embed_fwd);
  m.def("embed_bwd", &ft::embed_bwd);
  m.def("adamw_multi", &ft::adamw_multi);
  m.def("sumsq_multi", &ft::sumsq_multi);
  m.def("symm_alloc", &ft::symm_alloc);
  m.def("ipc_handle", &ft::ipc_handle);
  m.def("ipc_open", &ft::ipc_open);
  m.def("ipc_close", &ft::ipc_close);
  m.def("tensor_at", &ft::tensor_at);
  m.def("copy_from_ptrs", &ft::copy_from_ptrs);
  m.def("gemm_tc_fused", &ft::gemm_tc_fused);
  m.def("wait_flags_geq", &ft::wait_flags_geq, "bounded wait for peer flags (one warp)");
  m.def("rs_adamw", &ft::rs_adamw, "ZeRO reduce-scatter + fp32 cast/scale + sharded AdamW");
  m.def("stream_write", &ft::stream_write);
  m.def("nvls_supported", &ft::nvls_supported);
  m.def("nvls_round_size", &ft::nvls_round_size);
  m.def("nvls_create", &ft::nvls_create);
  m.def("nvls_export_fd", &ft::nvls_export_fd);
  m.def("nvls_import", &ft::nvls_import);
  m.def("nvls_add_device", &ft::nvls_add_device);
  m.def("nvls_bind_map", &ft::nvls_bind_map);
  m.def("nvls_close", &ft::nvls_close);
  m.def("nvls_barrier", &ft::nvls_barrier, "NVLS barrier: multimem.red + bounded wait");
  m.def("nvls_reduce_slice", &ft::nvls_reduce_slice, "in-switch reduction of this rank's slice (multimem)");
  m.def("gate_reserved_sms", &ft::gate_reserved_sms, "SMs a gated GEMM leaves to the pull kernel");
  m.def("ag_pull", &ft::ag_pull, "tensor-parallel all-gather: SM-driven peer pulls + chunk counters");
  m.def("rs_pull", &ft::rs_pull, "tensor-parallel reduce-scatter: owner pulls and sums peer partials");
  m.def("flash_fwd", &ft::flash_fwd);
  m.def("flash_fwd_variant", &ft::flash_fwd_variant);
  m.def("flash_bwd", &ft::flash_bwd);
}
