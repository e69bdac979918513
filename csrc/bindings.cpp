// Python bindings for the mimir_b200 sm_100a kernels (module mimir_b200._C).
#include <torch/extension.h>

// elementwise.cu
std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, double eps);
at::Tensor rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor rstd);
std::vector<at::Tensor> add_rmsnorm_fwd(at::Tensor x, at::Tensor delta, double eps);
at::Tensor rmsnorm_bwd_res(at::Tensor dy, at::Tensor x, at::Tensor rstd, at::Tensor dres);
at::Tensor swiglu_fwd(at::Tensor gu);
at::Tensor swiglu_bwd(at::Tensor dp, at::Tensor gu);
at::Tensor rope_qk(at::Tensor gqkv, at::Tensor cos_t, at::Tensor sin_t, at::Tensor pos, int64_t H, int64_t KV);
void rope_qk_bwd(at::Tensor dq, at::Tensor dk, at::Tensor dv, at::Tensor cos_t, at::Tensor sin_t, at::Tensor pos,
                 at::Tensor dgqkv, int64_t H, int64_t KV);
std::vector<at::Tensor> attn_gate_bwd(at::Tensor dy, at::Tensor o, at::Tensor gqkv, at::Tensor dgqkv, int64_t H);
at::Tensor attn_delta(at::Tensor d_o, at::Tensor o, int64_t H);
// loss.cu
std::vector<at::Tensor> ce_fwd(at::Tensor logits, at::Tensor labels);
void ce_bwd_inplace(at::Tensor logits, at::Tensor lse, at::Tensor labels, at::Tensor gscale);
// optim.cu
void adam_atan2_multi(std::vector<at::Tensor> params, std::vector<at::Tensor> grads,
                      c10::optional<std::vector<at::Tensor>> exp_avgs, std::vector<at::Tensor> exp_avg_sqs,
                      c10::optional<std::vector<at::Tensor>> emas, std::vector<double> lrs, std::vector<double> bc1,
                      std::vector<double> bc2_sqrt, double beta1, double beta2, double weight_decay, double ema_decay);
// ngram.cu
at::Tensor ngram_fwd(at::Tensor ids, at::Tensor pos, std::vector<at::Tensor> tables, std::vector<int64_t> orders,
                     int64_t heads, int64_t buckets, at::ScalarType dtype);
at::Tensor ngram_keys(at::Tensor ids, at::Tensor pos, std::vector<int64_t> orders, int64_t heads, int64_t buckets,
                      int64_t width);
void ngram_bwd(at::Tensor dout, at::Tensor ids, at::Tensor pos, at::Tensor sorted_keys, at::Tensor order,
               std::vector<at::Tensor> grads, std::vector<int64_t> orders, int64_t heads, int64_t buckets);
// fmha_fwd.cu
std::vector<at::Tensor> fmha_plan(at::Tensor cu_seqlens, at::Tensor prefix_lens, int64_t numseqs, int64_t total_tokens,
                                  bool is_causal);
std::vector<at::Tensor> fmha_fwd(at::Tensor q_src, int64_t q_col, at::Tensor k_src, int64_t k_col, at::Tensor v_src,
                                 int64_t v_col, c10::optional<at::Tensor> gate_src, int64_t gate_col, int64_t H,
                                 int64_t KV, bool is_causal, at::Tensor cu_seqlens, at::Tensor prefix_lens,
                                 int64_t numseqs, at::Tensor tiles, at::Tensor ntiles);
int64_t fmha_status(at::Device dev);
// fmha_fwd2.cu
std::vector<at::Tensor> fmha_plan2(at::Tensor cu_seqlens, at::Tensor prefix_lens, int64_t numseqs,
                                   int64_t total_tokens, bool is_causal);
std::vector<at::Tensor> fmha_fwd2(at::Tensor q_src, int64_t q_col, at::Tensor k_src, int64_t k_col, at::Tensor v_src,
                                  int64_t v_col, c10::optional<at::Tensor> gate_src, int64_t gate_col, int64_t H,
                                  int64_t KV, bool is_causal, at::Tensor cu_seqlens, at::Tensor prefix_lens,
                                  int64_t numseqs, at::Tensor tiles, at::Tensor ntiles);
// fmha_bwd.cu
std::vector<at::Tensor> fmha_bwd_plan(at::Tensor cu_seqlens, at::Tensor prefix_lens, int64_t numseqs,
                                      int64_t total_tokens, bool is_causal);
std::vector<at::Tensor> fmha_bwd(at::Tensor q_src, int64_t q_col, at::Tensor k_src, int64_t k_col, at::Tensor v_src,
                                 int64_t v_col, at::Tensor d_o, at::Tensor lse, at::Tensor delta, int64_t H,
                                 int64_t KV, bool is_causal, at::Tensor cu_seqlens, at::Tensor prefix_lens,
                                 int64_t numseqs, at::Tensor kv_tiles, at::Tensor kv_ntiles);

// dp_fused.cu
int64_t dp_segment_bytes();
int64_t dp_chunk_elements();
void dp_step(std::vector<int64_t> peer_grads, std::vector<int64_t> peer_weights, at::Tensor segs, int64_t nblocks,
             at::Tensor master, c10::optional<at::Tensor> exp_avg, at::Tensor exp_avg_sq, c10::optional<at::Tensor> ema,
             c10::optional<at::Tensor> reduced, c10::optional<at::Tensor> grad_scale, double b1, double b2,
             double ema_decay, std::vector<int64_t> peer_work, int64_t rank, bool lean);
void dp_reduce(std::vector<int64_t> peer_grads, at::Tensor segs, int64_t nblocks, at::Tensor reduced_out,
               at::Tensor sumsq_out, int64_t rank);
std::vector<at::Tensor> ipc_alloc(int64_t nbytes, int64_t device);
int64_t ipc_open(at::Tensor handle_bytes, int64_t device);
void ipc_close(int64_t ptr, int64_t device);
bool peer_access_possible(int64_t device, int64_t peer);
void zero_bytes(at::Tensor t);
void moe_dispatch(at::Tensor x, at::Tensor rows, at::Tensor dst, std::vector<int64_t> recv, int64_t k,
                  int64_t capacity);
at::Tensor moe_combine(std::vector<int64_t> y, at::Tensor rows, at::Tensor dst, c10::optional<at::Tensor> w,
                       int64_t T, int64_t k, int64_t d, c10::optional<at::Tensor> ys, int64_t capacity);
at::Tensor moe_combine_bwd(at::Tensor dout, at::Tensor w, at::Tensor rows, at::Tensor dst, at::Tensor ys,
                           std::vector<int64_t> dy, int64_t k, int64_t capacity);
int64_t moe_route_status(int64_t device);
void grouped_gemm(at::Tensor a, std::vector<at::Tensor> bs, at::Tensor counts, at::Tensor out, bool b_kn);
void grouped_wgrad(at::Tensor a, at::Tensor b, std::vector<int64_t> rows, std::vector<at::Tensor> grads);
int64_t grouped_gemm_status(int64_t device);
at::Tensor router_topk(at::Tensor scores, int64_t k, c10::optional<at::Tensor> load);
// embedding.cu
at::Tensor embed_fwd(at::Tensor ids, at::Tensor weight, double scale);
void embed_bwd(at::Tensor dout, at::Tensor sorted_ids, at::Tensor order, at::Tensor grad, double scale);
at::Tensor branch_read(at::Tensor s, at::Tensor logits, c10::optional<at::Tensor> gain, at::Tensor alpha);
at::Tensor branch_write(at::Tensor s, at::Tensor u, at::Tensor logits, c10::optional<at::Tensor> gain,
                        at::Tensor alpha);
std::vector<at::Tensor> branch_mix_bwd(at::Tensor grad, at::Tensor s, c10::optional<at::Tensor> u, at::Tensor logits,
                                       c10::optional<at::Tensor> gain, at::Tensor alpha);
at::Tensor invocation_gate_fwd(at::Tensor pre, at::Tensor inj, at::Tensor bias, at::Tensor alpha);
std::vector<at::Tensor> invocation_gate_bwd(at::Tensor dout, at::Tensor pre, at::Tensor inj, at::Tensor bias,
                                            at::Tensor alpha);
at::Tensor goldfish_mask(at::Tensor inputs, at::Tensor supervised, at::Tensor cu_seqlens, int64_t k,
                         int64_t context_width, int64_t seed, std::vector<int64_t> mix);
int64_t embed_status(int64_t device);
// gemm.cu
at::Tensor gemm(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, c10::optional<at::Tensor> out,
                c10::optional<at::Tensor> add, double alpha, double beta, int64_t bn, int64_t group_m,
                int64_t wait_ns, int64_t inject);
std::vector<at::Tensor> gemm_swiglu(at::Tensor x, at::Tensor w_gu, int64_t group_m);
at::Tensor gemm_swiglu_bwd(at::Tensor dy, at::Tensor w_down, at::Tensor gu, int64_t group_m);
int64_t gemm_status(int64_t device);
at::Tensor gemm_allgather(at::Tensor x, std::vector<int64_t> shard_ptrs, int64_t rank, at::Tensor g, at::Tensor flags,
                          int64_t epoch, int64_t wait_ns);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mimir_b200 hand-written sm_100a kernels";
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd);
  m.def("rmsnorm_bwd_res", &rmsnorm_bwd_res);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("rope_qk", &rope_qk);
  m.def("rope_qk_bwd", &rope_qk_bwd);
  m.def("attn_gate_bwd", &attn_gate_bwd);
  m.def("attn_delta", &attn_delta);
  m.def("ce_fwd", &ce_fwd);
  m.def("ce_bwd_inplace", &ce_bwd_inplace);
  m.def("adam_atan2_multi", &adam_atan2_multi);
  m.def("ngram_fwd", &ngram_fwd);
  m.def("ngram_keys", &ngram_keys);
  m.def("ngram_bwd", &ngram_bwd);
  m.def("fmha_plan", &fmha_plan);
  m.def("fmha_fwd", &fmha_fwd);
  m.def("fmha_status", &fmha_status);
  m.def("fmha_plan2", &fmha_plan2);
  m.def("fmha_fwd2", &fmha_fwd2);
  m.def("fmha_bwd_plan", &fmha_bwd_plan);
  m.def("dp_segment_bytes", &dp_segment_bytes);
  m.def("dp_chunk_elements", &dp_chunk_elements);
  m.def("dp_step", &dp_step);
  m.def("dp_reduce", &dp_reduce);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("peer_access_possible", &peer_access_possible);
  m.def("zero_bytes", &zero_bytes);
  m.def("moe_dispatch", &moe_dispatch);
  m.def("moe_combine", &moe_combine);
  m.def("moe_combine_bwd", &moe_combine_bwd);
  m.def("moe_route_status", &moe_route_status);
  m.def("grouped_gemm", &grouped_gemm);
  m.def("grouped_wgrad", &grouped_wgrad);
  m.def("grouped_gemm_status", &grouped_gemm_status);
  m.def("router_topk", &router_topk);
  m.def("gemm", &gemm, py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"), py::arg("out") = py::none(),
        py::arg("add") = py::none(), py::arg("alpha") = 1.0, py::arg("beta") = 0.0, py::arg("bn") = 256,
        py::arg("group_m") = 8, py::arg("wait_ns") = 0, py::arg("inject") = 0);
  m.def("gemm_swiglu", &gemm_swiglu, py::arg("x"), py::arg("w_gu"), py::arg("group_m") = 8);
  m.def("gemm_swiglu_bwd", &gemm_swiglu_bwd, py::arg("dy"), py::arg("w_down"), py::arg("gu"), py::arg("group_m") = 8);
  m.def("gemm_status", &gemm_status);
  m.def("gemm_allgather", &gemm_allgather, py::arg("x"), py::arg("shard_ptrs"), py::arg("rank"), py::arg("g"),
        py::arg("flags"), py::arg("epoch"), py::arg("wait_ns") = 0);
  m.def("embed_fwd", &embed_fwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("embed_status", &embed_status);
  m.def("branch_read", &branch_read);
  m.def("goldfish_mask", &goldfish_mask);
  m.def("invocation_gate_fwd", &invocation_gate_fwd);
  m.def("invocation_gate_bwd", &invocation_gate_bwd);
  m.def("branch_write", &branch_write);
  m.def("branch_mix_bwd", &branch_mix_bwd);
  m.def("fmha_bwd", &fmha_bwd);
}
