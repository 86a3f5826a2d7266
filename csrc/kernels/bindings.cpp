// Python bindings of the sm_100a kernels (module bitresearch_b200._C).
#include <torch/extension.h>

namespace br {
int64_t read_status(int64_t device);
void reset_status(int64_t device);
void gemm_qkv_rope(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, const torch::Tensor& cosT,
                   const torch::Tensor& sinT, torch::Tensor& rq, torch::Tensor& rk, int64_t T, int64_t H, int64_t KV,
                   c10::optional<torch::Tensor> idx, c10::optional<torch::Tensor> ve,
                   c10::optional<torch::Tensor> cur, c10::optional<torch::Tensor> wg,
                   c10::optional<torch::Tensor> gate);
void gemm_launch(const torch::Tensor& a, bool a_mn, int64_t lda, int64_t bsa, const torch::Tensor& b, bool b_mn,
                 int64_t ldb, int64_t bsb, torch::Tensor& c, int64_t ldc, int64_t bsc, int64_t M, int64_t N,
                 int64_t K, int64_t batch, int64_t epi, c10::optional<torch::Tensor> aux, int64_t ld_aux,
                 int64_t bs_aux, double alpha, double beta, int64_t k_splits, int64_t block_n);
void gemm_set_pair(int64_t mode);
int64_t gemm_pair();
void embed_rms_fwd(const torch::Tensor& idx, const torch::Tensor& wte, torch::Tensor& x0, torch::Tensor& rstd);
void ladder_rms_fwd(const torch::Tensor& x, const torch::Tensor& x0, const torch::Tensor& lam_r,
                    const torch::Tensor& lam_0, int64_t layer, torch::Tensor& cur, torch::Tensor& xn,
                    torch::Tensor& rstd);
void rms_fwd(const torch::Tensor& x, torch::Tensor& xn, c10::optional<torch::Tensor> rstd);
void rms_bwd(const torch::Tensor& x, const torch::Tensor& rstd, const torch::Tensor& dy,
             c10::optional<torch::Tensor> dres, c10::optional<torch::Tensor> dx, c10::optional<torch::Tensor> dxb,
             c10::optional<torch::Tensor> rowscale, c10::optional<torch::Tensor> coef,
             c10::optional<torch::Tensor> targets, c10::optional<torch::Tensor> wtab);
void gemm_softcap_ce(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& g, const torch::Tensor& targets,
                     torch::Tensor& partial, torch::Tensor& zt, double cap, bool store);
void ce_finalize(const torch::Tensor& partial, const torch::Tensor& zt, const torch::Tensor& targets, int64_t V,
                 double cap, double scale, c10::optional<torch::Tensor> nats, c10::optional<torch::Tensor> loss_sum,
                 c10::optional<torch::Tensor> rowscale, c10::optional<torch::Tensor> coef,
                 c10::optional<torch::Tensor> x, c10::optional<torch::Tensor> xs, c10::optional<torch::Tensor> dw,
                 c10::optional<torch::Tensor> g);
void ladder_bwd(const torch::Tensor& x, const torch::Tensor& x0, const torch::Tensor& lam_r,
                const torch::Tensor& lam_0, int64_t layer, const torch::Tensor& rstd, const torch::Tensor& dxn,
                const torch::Tensor& dres, c10::optional<torch::Tensor> dgate_in, torch::Tensor& dx,
                torch::Tensor& dx0_acc, torch::Tensor& dlam_r, torch::Tensor& dlam_0, bool first_layer,
                c10::optional<torch::Tensor> dx_b);
void embed_bwd(const torch::Tensor& idx, const torch::Tensor& wte, const torch::Tensor& rstd, const torch::Tensor& dx0,
               torch::Tensor& dwte);
void cast_bf16(const torch::Tensor& x, torch::Tensor& y);
void rope_fwd(torch::Tensor& qkv, int64_t T, int64_t H, int64_t KV, int64_t hd, const torch::Tensor& cosT,
              const torch::Tensor& sinT, torch::Tensor& rq, torch::Tensor& rk, const torch::Tensor& idx,
              c10::optional<torch::Tensor> ve, c10::optional<torch::Tensor> cur, c10::optional<torch::Tensor> wg,
              c10::optional<torch::Tensor> gate);
void rope_bwd(torch::Tensor& dqkv, const torch::Tensor& qkv, int64_t T, int64_t H, int64_t KV, int64_t hd,
              const torch::Tensor& cosT, const torch::Tensor& sinT, const torch::Tensor& rq, const torch::Tensor& rk,
              const torch::Tensor& idx, c10::optional<torch::Tensor> ve, c10::optional<torch::Tensor> gate,
              c10::optional<torch::Tensor> dve, c10::optional<torch::Tensor> dz);
void ve_gate_bwd(const torch::Tensor& cur, const torch::Tensor& dz, const torch::Tensor& wg, torch::Tensor& dwg,
                 torch::Tensor& dgate_in);
void softcap_ce(torch::Tensor& logits, const torch::Tensor& targets, double cap, double scale,
                c10::optional<torch::Tensor> nats, c10::optional<torch::Tensor> loss_sum, bool grad);
void adamw_multi(const std::vector<torch::Tensor>& params, const std::vector<torch::Tensor>& grads,
                 const std::vector<torch::Tensor>& ms, const std::vector<torch::Tensor>& vs,
                 const std::vector<torch::Tensor>& shadows, const std::vector<double>& hyper,
                 c10::optional<torch::Tensor> skip);
int64_t muon_prepare_scratch(int64_t S, int64_t n);
int64_t muon_finish_scratch(int64_t S, int64_t r, int64_t c);
void muon_prepare(const std::vector<torch::Tensor>& grads, const std::vector<torch::Tensor>& moms, double mu,
                  torch::Tensor& X, torch::Tensor& ss, c10::optional<torch::Tensor> skip);
void muon_finish(const torch::Tensor& X, const std::vector<torch::Tensor>& grads,
                 const std::vector<torch::Tensor>& params, const std::vector<torch::Tensor>& secs,
                 const std::vector<torch::Tensor>& shadows, int64_t r, int64_t c, double beta2, double lr, double wd,
                 torch::Tensor& work, c10::optional<torch::Tensor> skip);
void attn_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& o,
              torch::Tensor& lse, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd, int64_t window);
void attn_bwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& o,
              const torch::Tensor& dout, const torch::Tensor& lse, torch::Tensor& dq, torch::Tensor& dk,
              torch::Tensor& dv, torch::Tensor& delta, torch::Tensor& dq_acc, int64_t B, int64_t T, int64_t H,
              int64_t KV, int64_t hd, int64_t window);
void attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t T, int64_t H,
                 int64_t KV, int64_t hd, int64_t window);
void attn_bwd_tc(const torch::Tensor& qkv, const torch::Tensor& o, const torch::Tensor& dout, const torch::Tensor& lse,
                 torch::Tensor& dqkv, torch::Tensor& delta, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd,
                 int64_t window, int64_t which);
torch::Tensor mc_sharpe(int64_t n_paths, int64_t steps, double mu, double sigma, double annual, int64_t seed,
                        int64_t device);
void comm_push(const torch::Tensor& params, const torch::Tensor& peers, int64_t me, const torch::Tensor& chunks,
               int64_t max_blocks);
void comm_signal_peers(const torch::Tensor& flag_peers, int64_t me, int64_t epoch);
void comm_pack_push(const torch::Tensor& grad, const torch::Tensor& recv_peers, int64_t me, int64_t slot_elems,
                    const torch::Tensor& chunks, int64_t wire, double scale, torch::Tensor& bad, int64_t max_blocks);
void comm_signal_all(const torch::Tensor& flag_peers, int64_t me, int64_t slot, int64_t epoch, const torch::Tensor& bad);
void comm_reduce_local(int64_t recv_ptr, int64_t flags_ptr, int64_t npeers, int64_t slot, int64_t epoch,
                       int64_t slot_elems, const torch::Tensor& chunks, torch::Tensor& out, int64_t wire, double scale,
                       int64_t max_blocks, double budget_s);
void comm_agree(int64_t flags_ptr, int64_t npeers, int64_t slot, int64_t epoch, torch::Tensor& skip, double budget_s);
void status_snapshot(torch::Tensor& out, c10::optional<torch::Tensor> skip);
void comm_shadow_refresh(const torch::Tensor& params, int64_t push_flags_ptr, int64_t npeers, int64_t me,
                         int64_t epoch, const torch::Tensor& segs, int64_t max_blocks, double budget_s);
std::tuple<int64_t, torch::Tensor> sym_alloc(int64_t bytes);
int64_t sym_open(const torch::Tensor& handle);
void sym_close(int64_t ptr);
void sym_free(int64_t ptr);
torch::Tensor sym_view(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device);
void comm_pack(const torch::Tensor& src, int64_t send_ptr, int64_t wire, int64_t lo, int64_t hi, double scale,
               torch::Tensor& bad);
void comm_signal(int64_t flag_ptr, int64_t value);
void comm_reduce(const torch::Tensor& peers, const torch::Tensor& flags, int64_t slot, int64_t epoch,
                 const torch::Tensor& chunks, torch::Tensor& out, int64_t wire, double scale, int64_t max_blocks,
                 double budget_s);
void comm_gather(const torch::Tensor& peers, const torch::Tensor& flags, int64_t slot, int64_t epoch,
                 const torch::Tensor& segs, torch::Tensor& local, int64_t max_blocks, double budget_s);
void topk_threshold(const torch::Tensor& grad, const torch::Tensor& err, c10::optional<torch::Tensor> vel, int64_t lo,
                    int64_t hi, double scale, double mu, int64_t sample, double keep_ratio, int64_t seed,
                    bool masking, torch::Tensor& thr_out);
void topk_select(const torch::Tensor& grad, torch::Tensor& err, c10::optional<torch::Tensor> vel,
                 const torch::Tensor& chunks, double scale, double mu, bool masking, const torch::Tensor& thr,
                 int64_t idx_ptr, int64_t val_ptr, int64_t cnt_ptr);
void topk_reduce(const torch::Tensor& peers, const torch::Tensor& flags, int64_t slot, int64_t epoch, int64_t list_off,
                 int64_t cnt_index, torch::Tensor& red, double scale, int64_t max_blocks, double budget_s);
}  // namespace br

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "bitresearch-b200 sm_100a kernels";
  m.def("read_status", &br::read_status);
  m.def("reset_status", &br::reset_status);
  m.def("gemm", &br::gemm_launch);
  m.def("gemm_qkv_rope", &br::gemm_qkv_rope);
  m.def("gemm_set_pair", &br::gemm_set_pair);
  m.def("gemm_pair", &br::gemm_pair);
  m.def("embed_rms_fwd", &br::embed_rms_fwd);
  m.def("ladder_rms_fwd", &br::ladder_rms_fwd);
  m.def("rms_fwd", &br::rms_fwd);
  m.def("rms_bwd", &br::rms_bwd, pybind11::arg("x"), pybind11::arg("rstd"), pybind11::arg("dy"),
        pybind11::arg("dres"), pybind11::arg("dx"), pybind11::arg("dxb"), pybind11::arg("rowscale") = pybind11::none(),
        pybind11::arg("coef") = pybind11::none(), pybind11::arg("targets") = pybind11::none(),
        pybind11::arg("wtab") = pybind11::none());
  m.def("gemm_softcap_ce", &br::gemm_softcap_ce);
  m.def("ce_finalize", &br::ce_finalize, pybind11::arg("partial"), pybind11::arg("zt"), pybind11::arg("targets"),
        pybind11::arg("V"), pybind11::arg("cap"), pybind11::arg("scale"), pybind11::arg("nats") = pybind11::none(),
        pybind11::arg("loss_sum") = pybind11::none(), pybind11::arg("rowscale") = pybind11::none(),
        pybind11::arg("coef") = pybind11::none(), pybind11::arg("x") = pybind11::none(),
        pybind11::arg("xs") = pybind11::none(), pybind11::arg("dw") = pybind11::none(),
        pybind11::arg("g") = pybind11::none());
  m.def("ladder_bwd", &br::ladder_bwd, pybind11::arg("x"), pybind11::arg("x0"), pybind11::arg("lam_r"),
        pybind11::arg("lam_0"), pybind11::arg("layer"), pybind11::arg("rstd"), pybind11::arg("dxn"),
        pybind11::arg("dres"), pybind11::arg("dgate_in"), pybind11::arg("dx"), pybind11::arg("dx0_acc"),
        pybind11::arg("dlam_r"), pybind11::arg("dlam_0"), pybind11::arg("first_layer"),
        pybind11::arg("dx_b") = pybind11::none());
  m.def("embed_bwd", &br::embed_bwd);
  m.def("cast_bf16", &br::cast_bf16);
  m.def("rope_fwd", &br::rope_fwd);
  m.def("rope_bwd", &br::rope_bwd);
  m.def("ve_gate_bwd", &br::ve_gate_bwd);
  m.def("softcap_ce", &br::softcap_ce);
  m.def("adamw_multi", &br::adamw_multi, pybind11::arg("params"), pybind11::arg("grads"), pybind11::arg("ms"),
        pybind11::arg("vs"), pybind11::arg("shadows"), pybind11::arg("hyper"), pybind11::arg("skip") = pybind11::none());
  m.def("muon_prepare", &br::muon_prepare, pybind11::arg("grads"), pybind11::arg("moms"), pybind11::arg("mu"),
        pybind11::arg("X"), pybind11::arg("ss"), pybind11::arg("skip") = pybind11::none());
  m.def("muon_prepare_scratch", &br::muon_prepare_scratch);
  m.def("muon_finish_scratch", &br::muon_finish_scratch);
  m.def("muon_finish", &br::muon_finish, pybind11::arg("X"), pybind11::arg("grads"), pybind11::arg("params"),
        pybind11::arg("secs"), pybind11::arg("shadows"), pybind11::arg("r"), pybind11::arg("c"), pybind11::arg("beta2"),
        pybind11::arg("lr"), pybind11::arg("wd"), pybind11::arg("work"), pybind11::arg("skip") = pybind11::none());
  m.def("attn_fwd", &br::attn_fwd);
  m.def("attn_bwd", &br::attn_bwd);
  m.def("attn_fwd_tc", &br::attn_fwd_tc);
  m.def("attn_bwd_tc", &br::attn_bwd_tc, pybind11::arg("qkv"), pybind11::arg("o"), pybind11::arg("dout"),
        pybind11::arg("lse"), pybind11::arg("dqkv"), pybind11::arg("delta"), pybind11::arg("B"), pybind11::arg("T"),
        pybind11::arg("H"), pybind11::arg("KV"), pybind11::arg("hd"), pybind11::arg("window"),
        pybind11::arg("which") = 0);
  m.def("mc_sharpe", &br::mc_sharpe);
  m.def("comm_push", &br::comm_push);
  m.def("comm_signal_peers", &br::comm_signal_peers);
  m.def("comm_shadow_refresh", &br::comm_shadow_refresh);
  m.def("comm_pack_push", &br::comm_pack_push);
  m.def("comm_signal_all", &br::comm_signal_all);
  m.def("comm_reduce_local", &br::comm_reduce_local);
  m.def("comm_agree", &br::comm_agree);
  m.def("status_snapshot", &br::status_snapshot);
  m.def("sym_alloc", &br::sym_alloc);
  m.def("sym_open", &br::sym_open);
  m.def("sym_close", &br::sym_close);
  m.def("sym_free", &br::sym_free);
  m.def("sym_view", &br::sym_view);
  m.def("comm_pack", &br::comm_pack);
  m.def("comm_signal", &br::comm_signal);
  m.def("comm_reduce", &br::comm_reduce);
  m.def("comm_gather", &br::comm_gather);
  m.def("topk_threshold", &br::topk_threshold);
  m.def("topk_select", &br::topk_select);
  m.def("topk_reduce", &br::topk_reduce);
}
