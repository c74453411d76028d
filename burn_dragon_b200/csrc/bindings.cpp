// bindings.cpp — Python bindings of the sm_100a extension `_bdh_cuda`.
#include <torch/extension.h>

#include <vector>

namespace bd {
void gemm(int64_t epi, int64_t bn, const at::Tensor& a, bool a_mn, std::vector<int64_t> a_geom,
          const at::Tensor& b, bool b_mn, std::vector<int64_t> b_geom, int64_t M, int64_t N, int64_t K,
          int64_t Z1, int64_t Z2, int64_t splits, bool causal_skip, const at::Tensor& out0,
          const c10::optional<at::Tensor>& out1, const c10::optional<at::Tensor>& aux0,
          const c10::optional<at::Tensor>& aux1, int64_t ld, int64_t sz1, int64_t sz2, int64_t split_stride,
          double alpha, double thr, const c10::optional<at::Tensor>& freq,
          const c10::optional<at::Tensor>& log2_decay, int64_t T, int64_t pos0, int64_t Nh, bool accumulate,
          bool row_decay, int64_t pair, const at::Tensor& err, const c10::optional<std::vector<int64_t>>& scatter,
          const c10::optional<at::Tensor>& acc_src, int64_t src_decay_T, const c10::optional<at::Tensor>& rope_tab);
void rope_table(const at::Tensor& freq, int64_t pos0, int64_t T, const at::Tensor& out);
void ln_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& tokens, int64_t rows, int64_t D,
            const at::Tensor& gamma, const at::Tensor& beta, double eps, const c10::optional<at::Tensor>& y32,
            const c10::optional<at::Tensor>& y16, const at::Tensor& mean, const at::Tensor& rstd, int64_t norm_kind,
            const c10::optional<at::Tensor>& norm_alpha, const c10::optional<at::Tensor>& norm_shift);
at::Tensor ln_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& mean, const at::Tensor& rstd,
                  int64_t rows, int64_t D, const at::Tensor& gamma, int64_t remap_T, int64_t remap_H,
                  const c10::optional<at::Tensor>& dx16, const c10::optional<at::Tensor>& dx32, int64_t norm_kind,
            const c10::optional<at::Tensor>& norm_alpha, const c10::optional<at::Tensor>& norm_shift,
            const c10::optional<at::Tensor>& tokens);
void tail_fwd(const at::Tensor& partial, int64_t nsplit, int64_t split_stride, const at::Tensor& v, int64_t rows,
              int64_t D, const at::Tensor& gamma, const at::Tensor& beta, double eps,
              const c10::optional<at::Tensor>& m_out, const at::Tensor& vout32,
              const c10::optional<at::Tensor>& vout16, const c10::optional<at::Tensor>& st, int64_t norm_kind,
            const c10::optional<at::Tensor>& norm_alpha, const c10::optional<at::Tensor>& norm_shift);
at::Tensor tail_bwd(const at::Tensor& gin, const at::Tensor& v, const at::Tensor& m, const at::Tensor& st,
                    int64_t rows, int64_t D, const at::Tensor& gamma, const at::Tensor& beta, const at::Tensor& dm16,
                    const at::Tensor& dv_res, int64_t norm_kind,
            const c10::optional<at::Tensor>& norm_alpha, const c10::optional<at::Tensor>& norm_shift);
void sum_rows(const at::Tensor& out, const c10::optional<at::Tensor>& base, const at::Tensor& p0, int64_t n0,
              int64_t s0, const c10::optional<at::Tensor>& p1, int64_t n1, int64_t s1, int64_t total);
void cross_entropy(const at::Tensor& logits, const at::Tensor& target, const c10::optional<at::Tensor>& mask,
                   const at::Tensor& inv_count, int64_t rows, int64_t V, const at::Tensor& loss_rows,
                   const at::Tensor& dlogits);
void symmetrize(const at::Tensor& P, const at::Tensor& G, int64_t BH, int64_t T, int64_t H,
                const c10::optional<at::Tensor>& log2_decay);
void adamw(const at::Tensor& p, const at::Tensor& g, const at::Tensor& m, const at::Tensor& v,
           const c10::optional<at::Tensor>& shadow, double lr, double b1, double b2, double eps, double wd,
           double bc1, double bc2, const c10::optional<at::Tensor>& gscale,
           const c10::optional<at::Tensor>& hyper);
void grad_clip_coef(const at::Tensor& g, const at::Tensor& scratch3, double max_norm);
void cast_bf16(const at::Tensor& x, const at::Tensor& y);
void embed_grad(const at::Tensor& tokens, const at::Tensor& g, int64_t rows, int64_t D, const at::Tensor& out,
                bool accumulate, const c10::optional<at::Tensor>& perm, const c10::optional<at::Tensor>& seg);
void rho_step(const at::Tensor& rho, const at::Tensor& q, int64_t q_row_stride, const at::Tensor& v,
              const c10::optional<at::Tensor>& gamma, const at::Tensor& a, int64_t B, int64_t H, int64_t Nh,
              int64_t D);
void scaffold_effective(int64_t key, double stdv, int64_t dist, int64_t rows, int64_t I, int64_t O, int64_t R,
                        const c10::optional<at::Tensor>& A, const c10::optional<at::Tensor>& B,
                        const c10::optional<at::Tensor>& gain, double scale, const c10::optional<at::Tensor>& out16,
                        const c10::optional<at::Tensor>& out32, const c10::optional<at::Tensor>& base32,
                        const c10::optional<at::Tensor>& base_in);
void scaffold_gain_grad(int64_t key, double stdv, int64_t dist, const at::Tensor& dW, const at::Tensor& out);
void scaffold_adapter_grad(int64_t key, double stdv, int64_t dist, int64_t Hm, int64_t I, int64_t O, int64_t R,
                           const at::Tensor& dW, const at::Tensor& A, const at::Tensor& B,
                           const c10::optional<at::Tensor>& base32, double scale, const at::Tensor& dA,
                           const at::Tensor& dB, const c10::optional<at::Tensor>& gain_out, const at::Tensor& work);
int64_t scaffold_adapter_work(int64_t Hm, int64_t I, int64_t O, int64_t R);
int64_t sym_alloc(int64_t bytes, int64_t device);
void sym_free(int64_t ptr, int64_t device);
std::vector<int64_t> ipc_handle(int64_t ptr, int64_t device);
int64_t ipc_open(std::vector<int64_t> handle, int64_t device);
void ipc_close(int64_t ptr, int64_t device);
at::Tensor wrap_ptr(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device);
void peer_barrier(std::vector<int64_t> grad, std::vector<int64_t> param, std::vector<int64_t> shadow,
                  std::vector<int64_t> flags, int64_t rank, int64_t phase, const at::Tensor& err);
void reduce_adamw(std::vector<int64_t> grad, std::vector<int64_t> param, std::vector<int64_t> shadow,
                  std::vector<int64_t> flags, int64_t rank, int64_t lo, int64_t hi, const at::Tensor& m,
                  const at::Tensor& v, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                  const c10::optional<at::Tensor>& hyper);
void tp_reduce_gather(const at::Tensor& slots, std::vector<int64_t> dst, int64_t rank, int64_t rows, int64_t M,
                      int64_t D, int64_t slot_stride);
void tp_scatter_rows(const at::Tensor& src, std::vector<int64_t> slots, int64_t rank, int64_t rows, int64_t M,
                     int64_t D, int64_t slot_stride);
void reduce_mean(std::vector<int64_t> grad, std::vector<int64_t> flags, int64_t rank, int64_t lo, int64_t hi,
                 const at::Tensor& err);
void ddp_step(std::vector<int64_t> grad, std::vector<int64_t> shadow, bool grad_bf16, int64_t rank, int64_t lo,
              int64_t hi, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1, double b2,
              double eps, double wd, const at::Tensor& hyper, const c10::optional<at::Tensor>& coef,
              std::vector<int64_t> gather_master);
void ddp_reduce(std::vector<int64_t> grad, std::vector<int64_t> shadow, bool grad_bf16, int64_t rank, int64_t lo,
                int64_t hi, const at::Tensor& gred, const at::Tensor& sumsq);
void ddp_apply(std::vector<int64_t> grad, std::vector<int64_t> shadow, int64_t rank, int64_t lo, int64_t hi,
               const at::Tensor& gred, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1,
               double b2, double eps, double wd, const at::Tensor& hyper, const at::Tensor& coef,
               std::vector<int64_t> gather_master);
void ddp_norm_exchange(std::vector<int64_t> flags, int64_t rank, const at::Tensor& sumsq, double max_norm,
                       const at::Tensor& out, const at::Tensor& err);
void ddp_epoch_advance(const at::Tensor& flags_local);
void ddp_slot_barrier(std::vector<int64_t> flags, int64_t rank, int64_t slot, const at::Tensor& err);
void ssd_chunk_fwd(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, const at::Tensor& DA,
                   const at::Tensor& S0, const at::Tensor& VS, const at::Tensor& KS, const at::Tensor& CF,
                   int64_t chunk, const at::Tensor& Y, const at::Tensor& SF, const at::Tensor& SC);
void ssd_chunk_bwd(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, const at::Tensor& DA,
                   const at::Tensor& VS, const at::Tensor& KS, const at::Tensor& CF, const at::Tensor& SC,
                   const at::Tensor& DY, const at::Tensor& DSF, int64_t chunk, const at::Tensor& dQ,
                   const at::Tensor& dK, const at::Tensor& dV, const at::Tensor& dDA, const at::Tensor& dS0,
                   const at::Tensor& dVS, const at::Tensor& dKS, const at::Tensor& dCF);
void tp_sum_slots(const at::Tensor& slots, const at::Tensor& out, int64_t world, int64_t n, int64_t slot_stride,
                  const c10::optional<at::Tensor>& add);
void tp_gather_bytes(std::vector<int64_t> dst, int64_t rank, int64_t offset, int64_t nbytes, int64_t device);
void ddp_step_nvls(int64_t mc_grad, int64_t mc_shadow, int64_t mc_master, bool grad_bf16, int64_t world, int64_t lo,
                   int64_t hi, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1,
                   double b2, double eps, double wd, const at::Tensor& hyper, const c10::optional<at::Tensor>& coef);
void ddp_reduce_nvls(int64_t mc_grad, bool grad_bf16, int64_t world, int64_t lo, int64_t hi, const at::Tensor& gred,
                     const at::Tensor& sumsq);
void ddp_apply_nvls(int64_t mc_shadow, int64_t mc_master, int64_t lo, int64_t hi, const at::Tensor& gred,
                    const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1, double b2,
                    double eps, double wd, const at::Tensor& hyper, const at::Tensor& coef);
void set_debug_bounds(int64_t device, const c10::optional<at::Tensor>& word);
void percentile_thresholds(const at::Tensor& values, double q, const at::Tensor& out);
}  // namespace bd

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "burn_dragon_b200 sm_100a kernels (tcgen05 GEMM engine + row kernels)";
  m.def("gemm", &bd::gemm);
  m.def("rope_table", &bd::rope_table);
  // trailing norm arguments: kind 0 LayerNorm, 1 RMSNorm, 2 DynamicTanh, 3 Derf (alpha /
  // shift: 1-element fp32 device tensors of the learnable scalars)
  m.def("ln_fwd", &bd::ln_fwd, py::arg("x"), py::arg("tokens"), py::arg("rows"), py::arg("D"), py::arg("gamma"),
        py::arg("beta"), py::arg("eps"), py::arg("y32"), py::arg("y16"), py::arg("mean"), py::arg("rstd"), py::arg("norm_kind") = 0, py::arg("norm_alpha") = py::none(), py::arg("norm_shift") = py::none());
  m.def("ln_bwd", &bd::ln_bwd, py::arg("dy"), py::arg("x"), py::arg("mean"), py::arg("rstd"), py::arg("rows"),
        py::arg("D"), py::arg("gamma"), py::arg("remap_T"), py::arg("remap_H"), py::arg("dx16"), py::arg("dx32"),
        py::arg("norm_kind") = 0, py::arg("norm_alpha") = py::none(), py::arg("norm_shift") = py::none(),
        py::arg("tokens") = py::none());
  m.def("embed_grad", &bd::embed_grad);
  m.def("tail_fwd", &bd::tail_fwd, py::arg("partial"), py::arg("nsplit"), py::arg("split_stride"), py::arg("v"),
        py::arg("rows"), py::arg("D"), py::arg("gamma"), py::arg("beta"), py::arg("eps"), py::arg("m_out"),
        py::arg("vout32"), py::arg("vout16"), py::arg("st"), py::arg("norm_kind") = 0, py::arg("norm_alpha") = py::none(), py::arg("norm_shift") = py::none());
  m.def("tail_bwd", &bd::tail_bwd, py::arg("gin"), py::arg("v"), py::arg("m"), py::arg("st"), py::arg("rows"),
        py::arg("D"), py::arg("gamma"), py::arg("beta"), py::arg("dm16"), py::arg("dv_res"), py::arg("norm_kind") = 0, py::arg("norm_alpha") = py::none(), py::arg("norm_shift") = py::none());
  m.def("sum_rows", &bd::sum_rows);
  m.def("set_debug_bounds", &bd::set_debug_bounds);
  m.def("cross_entropy", &bd::cross_entropy);
  m.def("symmetrize", &bd::symmetrize);
  m.def("adamw", &bd::adamw);
  m.def("grad_clip_coef", &bd::grad_clip_coef);
  m.def("cast_bf16", &bd::cast_bf16);
  m.def("rho_step", &bd::rho_step);
  m.def("scaffold_effective", &bd::scaffold_effective);
  m.def("scaffold_gain_grad", &bd::scaffold_gain_grad);
  m.def("scaffold_adapter_grad", &bd::scaffold_adapter_grad);
  m.def("scaffold_adapter_work", &bd::scaffold_adapter_work);
  m.def("sym_alloc", &bd::sym_alloc);
  m.def("sym_free", &bd::sym_free);
  m.def("ipc_handle", &bd::ipc_handle);
  m.def("ipc_open", &bd::ipc_open);
  m.def("ipc_close", &bd::ipc_close);
  m.def("wrap_ptr", &bd::wrap_ptr);
  m.def("peer_barrier", &bd::peer_barrier);
  m.def("reduce_adamw", &bd::reduce_adamw);
  m.def("reduce_mean", &bd::reduce_mean);
  m.def("tp_reduce_gather", &bd::tp_reduce_gather);
  m.def("tp_scatter_rows", &bd::tp_scatter_rows);
  m.def("ddp_step", &bd::ddp_step);
  m.def("ddp_step_nvls", &bd::ddp_step_nvls);
  m.def("ddp_reduce_nvls", &bd::ddp_reduce_nvls);
  m.def("ddp_apply_nvls", &bd::ddp_apply_nvls);
  m.def("ddp_reduce", &bd::ddp_reduce);
  m.def("ddp_apply", &bd::ddp_apply);
  m.def("ddp_norm_exchange", &bd::ddp_norm_exchange);
  m.def("ddp_epoch_advance", &bd::ddp_epoch_advance);
  m.def("ddp_slot_barrier", &bd::ddp_slot_barrier);
  m.def("ssd_chunk_fwd", &bd::ssd_chunk_fwd);
  m.def("ssd_chunk_bwd", &bd::ssd_chunk_bwd);
  m.def("tp_sum_slots", &bd::tp_sum_slots);
  m.def("tp_gather_bytes", &bd::tp_gather_bytes);
  m.def("percentile_thresholds", &bd::percentile_thresholds);
}
