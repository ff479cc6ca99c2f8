// Python bindings of the sm_100a kernels (one extension module, built in-tree by eagle4_b200/ops/build.py).
#include <torch/extension.h>

namespace e4 {
torch::Tensor gemm_error_word(torch::Device dev);
void gemm_prefill_mode(bool on);
std::vector<torch::Tensor> sampled_walk_sparse(const torch::Tensor& p_cand, const torch::Tensor& row_parent,
                                               const torch::Tensor& row_tok, const torch::Tensor& row_node,
                                               const torch::Tensor& q_store, const torch::Tensor& q_ids,
                                               const torch::Tensor& node_slot, int64_t K, int64_t seed,
                                               const torch::Tensor& round_ctr, int64_t stream);
torch::Tensor shard_residual_mass(const torch::Tensor& logits, int64_t lo, double temperature, const torch::Tensor& mx,
                                  const torch::Tensor& z, const torch::Tensor& final_row,
                                  const torch::Tensor& row_node, const torch::Tensor& q_ids,
                                  const torch::Tensor& r_final, int64_t S, int64_t n);
torch::Tensor shard_draw(const torch::Tensor& logits, int64_t lo, double temperature, const torch::Tensor& mx,
                         const torch::Tensor& z, const torch::Tensor& final_row, const torch::Tensor& row_node,
                         const torch::Tensor& q_ids, const torch::Tensor& r_final, int64_t S, int64_t n,
                         const torch::Tensor& masses, int64_t rank, int64_t seed, const torch::Tensor& round_ctr,
                         int64_t stream);
torch::Tensor moe_experts(const torch::Tensor& latent, const torch::Tensor& chosen, const torch::Tensor& weights,
                          const torch::Tensor& up, const torch::Tensor& down);
void gemm_launch(const torch::Tensor& x, const torch::Tensor& w, int epi, torch::Tensor y, torch::Tensor yf,
                 const torch::Tensor& res, torch::Tensor amax_val, torch::Tensor amax_idx, double fold_eps);
torch::Tensor rmsnorm(const torch::Tensor& x, const torch::Tensor& w, double eps, bool offset);
torch::Tensor concat_norms(const torch::Tensor& e, const torch::Tensor& h, const torch::Tensor& we,
                           const torch::Tensor& wh, double eps);
torch::Tensor embedding(const torch::Tensor& ids, const torch::Tensor& table);
torch::Tensor gated_rmsnorm(const torch::Tensor& o, const torch::Tensor& z, const torch::Tensor& w, double eps,
                            bool gate_first);
torch::Tensor qkv_prepare(const torch::Tensor& qkv, const torch::Tensor& pos, const torch::Tensor& slot,
                          torch::Tensor kc, torch::Tensor vc, const c10::optional<torch::Tensor>& qn,
                          const c10::optional<torch::Tensor>& kn, bool norm_offset, const torch::Tensor& cos_t,
                          const torch::Tensor& sin_t, int64_t Hq, int64_t Hk, int64_t D, int64_t rot, bool gated,
                          double eps);
std::vector<torch::Tensor> argmax_reduce(const torch::Tensor& val, const torch::Tensor& idx, int64_t n_tiles,
                                         int64_t T);
void kv_commit(const torch::Tensor& kp, const torch::Tensor& vp, const torch::Tensor& src, const torch::Tensor& dst,
               int64_t row_elems);
torch::Tensor attention(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc,
                        const torch::Tensor& bt, int64_t page, const torch::Tensor& req, const torch::Tensor& ctx_start,
                        const torch::Tensor& ctx_len, const torch::Tensor& extra, const torch::Tensor& n_extra,
                        double scale, int64_t max_keys, const c10::optional<torch::Tensor>& gate);
torch::Tensor conv_tree(const torch::Tensor& x, const torch::Tensor& cs, const torch::Tensor& slot,
                        const torch::Tensor& parent, const torch::Tensor& w, const torch::Tensor& bias);
void conv_commit(const torch::Tensor& x, torch::Tensor cs, const torch::Tensor& slots, const torch::Tensor& rows,
                 const torch::Tensor& nrows, int64_t W);
void conv_commit_scan(torch::Tensor cs, const torch::Tensor& x, const torch::Tensor& slot, int64_t W,
                      const torch::Tensor& seg);
torch::Tensor gdn_tree(const torch::Tensor& qkv, const torch::Tensor& proj, int64_t z_off, int64_t b_off,
                       int64_t a_off, const torch::Tensor& a_log, const torch::Tensor& dt_bias, torch::Tensor state,
                       const torch::Tensor& slot, const torch::Tensor& parent, const torch::Tensor& norm_w,
                       double eps, int64_t HK, int64_t HV, int64_t K, int64_t V, bool scan,
                       const torch::Tensor& seg);
void gdn_commit_all(const std::vector<torch::Tensor>& qkv, const std::vector<torch::Tensor>& proj,
                    const std::vector<torch::Tensor>& state, const std::vector<torch::Tensor>& conv_state,
                    const std::vector<torch::Tensor>& a_log, const std::vector<torch::Tensor>& dt_bias, int64_t b_off,
                    int64_t a_off, const torch::Tensor& slots, const torch::Tensor& rows, const torch::Tensor& nrows,
                    int64_t HK, int64_t HV, int64_t K, int64_t V, int64_t C, int64_t W);
torch::Tensor mamba_tree(const torch::Tensor& xbc, const torch::Tensor& dt, const torch::Tensor& a_log,
                         const torch::Tensor& dt_bias, const torch::Tensor& dskip, torch::Tensor state,
                         const torch::Tensor& slot, const torch::Tensor& parent, int64_t H, int64_t P, int64_t N,
                         int64_t G, bool scan, const torch::Tensor& seg);
void mamba_commit(const torch::Tensor& xbc, const torch::Tensor& dt, const torch::Tensor& a_log,
                  const torch::Tensor& dt_bias, const torch::Tensor& dskip, torch::Tensor state,
                  const torch::Tensor& slots, const torch::Tensor& rows, const torch::Tensor& nrows, int64_t H,
                  int64_t P, int64_t N, int64_t G);
torch::Tensor gather_dot(const torch::Tensor& h, const torch::Tensor& w, const torch::Tensor& idx);
std::vector<torch::Tensor> softmax_topk(const torch::Tensor& logit, const c10::optional<torch::Tensor>& ids, int64_t K,
                                        double temperature);
std::vector<torch::Tensor> accept_greedy(const torch::Tensor& tid, const torch::Tensor& tokens,
                                         const torch::Tensor& parent, const torch::Tensor& nrows);
std::vector<torch::Tensor> topk_large(const torch::Tensor& scores, int64_t C);
void tree_step(const torch::Tensor& probs, const torch::Tensor& toks, const torch::Tensor& hidden, int64_t bs,
               int64_t K, int64_t step, int64_t layer_start, int64_t parent_col, torch::Tensor scores,
               torch::Tensor tokens, torch::Tensor parents, torch::Tensor front_scores, torch::Tensor front_tokens,
               torch::Tensor front_hidden, torch::Tensor front_nodes, torch::Tensor ancestors, torch::Tensor best,
               torch::Tensor best_prev, torch::Tensor layer_top, torch::Tensor delta_rows, torch::Tensor deltas_out,
               torch::Tensor counter);
void tree_begin(const torch::Tensor& root_probs, const torch::Tensor& root_tokens, const torch::Tensor& root_hidden,
                int64_t bs, int64_t K, bool keep_order, double root_score, torch::Tensor scores, torch::Tensor tokens,
                torch::Tensor front_scores, torch::Tensor front_tokens, torch::Tensor front_hidden,
                torch::Tensor front_nodes, torch::Tensor best, torch::Tensor best_prev, torch::Tensor layer_top,
                torch::Tensor delta_rows, torch::Tensor deltas_out, torch::Tensor counter);
std::vector<torch::Tensor> select_rows(const torch::Tensor& scores, const torch::Tensor& decay,
                                       const torch::Tensor& tokens, const torch::Tensor& parents, int64_t bs,
                                       int64_t n, int64_t K, int64_t count);
int64_t gemm_allreduce(const torch::Tensor& x, const torch::Tensor& w, const torch::Tensor& residual, torch::Tensor y,
                       const std::vector<int64_t>& part, const std::vector<int64_t>& gath,
                       const std::vector<int64_t>& flags, int64_t ctrl, int64_t ldp, int64_t rank,
                       int64_t two_shot_rows);
std::vector<torch::Tensor> sample_children(const torch::Tensor& logits, const torch::Tensor& cand_ids, int64_t K,
                                           double temperature, int64_t seed, const torch::Tensor& round_ctr,
                                           int64_t stream, const c10::optional<torch::Tensor>& front_nodes,
                                           int64_t lanes, torch::Tensor q_store, torch::Tensor q_ids,
                                           torch::Tensor node_slot, int64_t child_base);
std::vector<torch::Tensor> sampled_accept(const torch::Tensor& logits, double temperature,
                                          const torch::Tensor& row_parent, const torch::Tensor& row_tok,
                                          const torch::Tensor& row_node, const torch::Tensor& q_store,
                                          const torch::Tensor& q_ids, const torch::Tensor& node_slot, int64_t K,
                                          int64_t seed, const torch::Tensor& round_ctr, int64_t stream);
void advance_round(torch::Tensor round_ctr);
std::vector<torch::Tensor> verify_rows_meta(const torch::Tensor& prow, const torch::Tensor& toks,
                                            const torch::Tensor& root, const torch::Tensor& L,
                                            const torch::Tensor& slot, const torch::Tensor& block_table, int64_t page);
std::vector<torch::Tensor> draft_step_rows(const torch::Tensor& L, const torch::Tensor& slot,
                                           const torch::Tensor& block_table, torch::Tensor ancestors, int64_t bs,
                                           int64_t K, int64_t s, int64_t page, int64_t window);
torch::Tensor gemm_traced(const torch::Tensor& x, const torch::Tensor& w, int64_t epi);
int64_t sym_alloc(int64_t bytes, int64_t device);
void sym_free(int64_t ptr);
torch::Tensor sym_handle(int64_t ptr);
int64_t sym_open(const torch::Tensor& handle, int64_t device);
void sym_close(int64_t ptr);
torch::Tensor sym_view(int64_t ptr, int64_t offset, int64_t numel, int64_t dtype_code, int64_t device);
void tp_argmax(const torch::Tensor& val, const torch::Tensor& idx, int64_t n_tiles, int64_t lo,
               const std::vector<int64_t>& xbufs, int64_t rank, int64_t max_rows, int64_t channel,
               torch::Tensor out_ids, torch::Tensor out_val, torch::Tensor err);
}  // namespace e4

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "eagle4_b200 sm_100a kernels";
  m.def("error_word", [](int64_t dev) { return e4::gemm_error_word(torch::Device(torch::kCUDA, dev)); });
  m.def("gemm", &e4::gemm_launch, "tcgen05 skinny GEMM with fused epilogue");
  m.def("gemm_prefill_mode", &e4::gemm_prefill_mode);
  m.def("gemm_allreduce", &e4::gemm_allreduce, "row-parallel GEMM fused with its all-reduce and the residual add");
  m.def("sample_children", &e4::sample_children, "Gumbel-top-k children from candidate logits");
  m.def("sampled_accept", &e4::sampled_accept, "recursive tree rejection over the verify rows");
  m.def("advance_round", &e4::advance_round);
  m.def("verify_rows_meta", &e4::verify_rows_meta, "verify row structure of a round");
  m.def("draft_step_rows", &e4::draft_step_rows, "row metadata of one draft step");
  m.def("gemm_traced", &e4::gemm_traced, "one GEMM with per-CTA timestamps (tuning)");
  m.def("sym_alloc", &e4::sym_alloc);
  m.def("sym_free", &e4::sym_free);
  m.def("sym_handle", &e4::sym_handle);
  m.def("sym_open", &e4::sym_open);
  m.def("sym_close", &e4::sym_close);
  m.def("sym_view", &e4::sym_view);
  m.def("tp_argmax", &e4::tp_argmax);
  m.def("rmsnorm", &e4::rmsnorm);
  m.def("concat_norms", &e4::concat_norms);
  m.def("embedding", &e4::embedding);
  m.def("gated_rmsnorm", &e4::gated_rmsnorm);
  m.def("qkv_prepare", &e4::qkv_prepare);
  m.def("argmax_reduce", &e4::argmax_reduce);
  m.def("kv_commit", &e4::kv_commit);
  m.def("attention", &e4::attention);
  m.def("conv_tree", &e4::conv_tree);
  m.def("conv_commit", &e4::conv_commit);
  m.def("conv_commit_scan", &e4::conv_commit_scan);
  m.def("gdn_tree", &e4::gdn_tree);
  m.def("gdn_commit_all", &e4::gdn_commit_all);
  m.def("mamba_tree", &e4::mamba_tree);
  m.def("mamba_commit", &e4::mamba_commit);
  m.def("gather_dot", &e4::gather_dot);
  m.def("softmax_topk", &e4::softmax_topk);
  m.def("accept_greedy", &e4::accept_greedy);
  m.def("topk_large", &e4::topk_large);
  m.def("tree_step", &e4::tree_step);
  m.def("tree_begin", &e4::tree_begin);
  m.def("select_rows", &e4::select_rows);
  m.def("moe_experts", &e4::moe_experts);
  m.def("sampled_walk_sparse", &e4::sampled_walk_sparse);
  m.def("shard_residual_mass", &e4::shard_residual_mass);
  m.def("shard_draw", &e4::shard_draw);
}
