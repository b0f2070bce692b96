// Python bindings of the bridge_b200 sm_100a kernels (module bridge_b200._C).
#include <torch/extension.h>

int64_t bb_launch_count();

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps);
std::vector<torch::Tensor> rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd);
std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor res, torch::Tensor w, double eps);
std::vector<torch::Tensor> add_rmsnorm_bwd(torch::Tensor dy, torch::Tensor h, torch::Tensor w, torch::Tensor rstd,
                                           torch::Tensor dh);
void sumsq_into(torch::Tensor x, torch::Tensor out, bool accumulate);
torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w, int64_t start);
void embedding_bwd_acc(torch::Tensor ids, torch::Tensor dy, torch::Tensor grad, int64_t start);
torch::Tensor rmsnorm_bwd_acc(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dres,
                              torch::Tensor dw_acc);
std::vector<torch::Tensor> qk_norm_rope_bwd_acc(torch::Tensor dqo, torch::Tensor dko, torch::Tensor q, torch::Tensor k,
                                                torch::Tensor qw, torch::Tensor kw, torch::Tensor cosb,
                                                torch::Tensor sinb, torch::Tensor rq, torch::Tensor rk,
                                                torch::Tensor dqw_acc, torch::Tensor dkw_acc);
std::vector<torch::Tensor> gated_rmsnorm_fwd(torch::Tensor o, torch::Tensor z, torch::Tensor w, double eps);
std::vector<torch::Tensor> gated_rmsnorm_bwd(torch::Tensor dy, torch::Tensor o, torch::Tensor z, torch::Tensor w,
                                             torch::Tensor rstd);
std::vector<torch::Tensor> l2norm_fwd(torch::Tensor x, double eps);
torch::Tensor l2norm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor rn);
std::vector<torch::Tensor> gdn_gates_fwd(torch::Tensor a, torch::Tensor b, torch::Tensor A_log, torch::Tensor dt);
std::vector<torch::Tensor> gdn_gates_bwd(torch::Tensor dg, torch::Tensor dbeta, torch::Tensor a, torch::Tensor b,
                                         torch::Tensor A_log, torch::Tensor dt);
std::vector<torch::Tensor> qk_norm_rope_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor qw, torch::Tensor kw,
                                            torch::Tensor cosb, torch::Tensor sinb, double eps);
std::vector<torch::Tensor> qk_norm_rope_bwd(torch::Tensor dqo, torch::Tensor dko, torch::Tensor q, torch::Tensor k,
                                            torch::Tensor qw, torch::Tensor kw, torch::Tensor cosb,
                                            torch::Tensor sinb, torch::Tensor rq, torch::Tensor rk);
torch::Tensor swiglu_fwd(torch::Tensor gu);
std::vector<torch::Tensor> moe_route(torch::Tensor logits, int64_t k);
torch::Tensor moe_combine(torch::Tensor ys, torch::Tensor pos, torch::Tensor w, int64_t T);
std::vector<torch::Tensor> moe_combine_bwd(torch::Tensor dy, torch::Tensor ys, torch::Tensor pos, torch::Tensor w);
torch::Tensor moe_route_bwd(torch::Tensor idx, torch::Tensor w, torch::Tensor dw, int64_t E);
torch::Tensor swiglu_bwd(torch::Tensor dy, torch::Tensor gu);
void logprob_stats(torch::Tensor logits, torch::Tensor targets, torch::Tensor inv_temp, int64_t vocab_start,
                   torch::Tensor stats);
std::vector<torch::Tensor> logprob_finalize(torch::Tensor stats);
void logprob_grad_inplace(torch::Tensor logits, torch::Tensor targets, torch::Tensor inv_temp, torch::Tensor lse,
                          torch::Tensor ezn, torch::Tensor dlp, c10::optional<torch::Tensor> dent,
                          int64_t vocab_start);
std::vector<torch::Tensor> ppo_loss_fwd(torch::Tensor x, torch::Tensor old, torch::Tensor adv,
                                        c10::optional<torch::Tensor> w, double denom, double lo, double hi, double c);
void adamw_step(torch::Tensor master, torch::Tensor param, torch::Tensor grad, torch::Tensor m, torch::Tensor v,
                torch::Tensor clip, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2);
std::vector<torch::Tensor> tree_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor pk,
                                         torch::Tensor pv, torch::Tensor cu, torch::Tensor poff, torch::Tensor plen,
                                         int64_t max_seqlen, int64_t max_prefix, double scale);
std::vector<torch::Tensor> tree_attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                         torch::Tensor pk, torch::Tensor pv, torch::Tensor o, torch::Tensor lse,
                                         torch::Tensor cu, torch::Tensor poff, torch::Tensor plen, int64_t max_seqlen,
                                         int64_t max_prefix, double scale, torch::Tensor users_meta, int64_t nspans);

torch::Tensor gemm(torch::Tensor a, torch::Tensor b, bool a_mn, bool b_mn, c10::optional<torch::Tensor> out,
                   bool accumulate);
int64_t gemm_error_code();
torch::Tensor grouped_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor offsets, bool trans_w);
void grouped_gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor offsets, torch::Tensor acc);

std::vector<torch::Tensor> tree_attn_fwd_sm100(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor pk,
                                               torch::Tensor pv, torch::Tensor cu, torch::Tensor poff,
                                               torch::Tensor plen, int64_t max_seqlen, int64_t max_prefix,
                                               double scale);
int64_t attn_error_code();
std::vector<torch::Tensor> tree_attn_bwd_sm100(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                               torch::Tensor pk, torch::Tensor pv, torch::Tensor o, torch::Tensor lse,
                                               torch::Tensor cu, torch::Tensor poff, torch::Tensor plen,
                                               int64_t max_seqlen, int64_t max_prefix, double scale);

std::vector<torch::Tensor> causal_conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                                             c10::optional<torch::Tensor> h0, torch::Tensor cu, int64_t max_len,
                                             bool silu_act);
std::vector<torch::Tensor> causal_conv1d_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                             c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> h0,
                                             c10::optional<torch::Tensor> dhT, torch::Tensor cu, int64_t max_len,
                                             bool silu_act);
std::vector<torch::Tensor> gdr_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                   torch::Tensor beta, c10::optional<torch::Tensor> h0, torch::Tensor chunks,
                                   torch::Tensor seq0, int64_t max_chunks, double scale);
void gdr_phase_profile(bool enable);
void attn_phase_profile(bool enable);
torch::Tensor attn_phase_read();
torch::Tensor gdr_phase_read();
std::vector<torch::Tensor> gdr_bwd(torch::Tensor dout, c10::optional<torch::Tensor> dhT, torch::Tensor q,
                                   torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                                   torch::Tensor ckpt, torch::Tensor wk, torch::Tensor u, torch::Tensor chunks,
                                   torch::Tensor seq0, int64_t max_chunks, bool has_h0, double scale);
std::vector<torch::Tensor> symm_alloc(int64_t nbytes);
int64_t symm_open(torch::Tensor handle);
void symm_close(int64_t ptr);
int64_t symm_pad_bytes();
void symm_barrier(std::vector<int64_t> pads, int64_t rank, int64_t epoch, c10::optional<torch::Tensor> payload,
                  double timeout_s);
void dp_reduce_scatter(std::vector<int64_t> grads, int64_t rank, int64_t offset, int64_t count, double scale,
                       torch::Tensor partials);
void dp_adamw_allgather(torch::Tensor master, torch::Tensor m, torch::Tensor v, torch::Tensor grad_shard,
                        std::vector<int64_t> data, int64_t offset, bool bf16_params, int64_t pad_ptr, double max_norm,
                        double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                        torch::Tensor norm_out);
int64_t symm_error_code();
void p2p_gather_rows(torch::Tensor out, std::vector<int64_t> peers, torch::Tensor src_rank, torch::Tensor src_row);
void p2p_copy(torch::Tensor dst, int64_t src_ptr, int64_t nbytes);
void dp_bucket_signal(std::vector<int64_t> flags, int64_t rank, int64_t max_buckets, int64_t bucket, int64_t epoch);
void dp_bucket_wait(int64_t mine, int64_t n, int64_t max_buckets, int64_t bucket, int64_t epoch, double timeout_s);
void p2p_reduce_rows(torch::Tensor out, std::vector<int64_t> peers, torch::Tensor src_row, bool src_f32,
                     c10::optional<torch::Tensor> add);
torch::Tensor tp_ag_gemm(torch::Tensor gather, torch::Tensor b, bool b_mn, std::vector<int64_t> peers, int64_t rank,
                         int64_t ms, torch::Tensor counters, double timeout_s);
void tp_gemm_rs(torch::Tensor a, torch::Tensor b, bool b_mn, std::vector<int64_t> peers, int64_t rank, int64_t ms,
                double timeout_s);
torch::Tensor tp_sum_slots(torch::Tensor recv, int64_t n, int64_t ms, int64_t N);
void symm_clear_error();

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "bridge_b200 sm_100a kernels";
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd, "h = x + res; y = RMSNorm(h) * w -> (y, rstd, h)");
  m.def("add_rmsnorm_bwd", &add_rmsnorm_bwd, "residual-sum gradient: RMSNorm backward + dh -> (dx, dw)");
  m.def("rmsnorm_bwd_acc", &rmsnorm_bwd_acc, "RMSNorm backward (+ residual grad) with dw accumulated in place");
  m.def("qk_norm_rope_bwd_acc", &qk_norm_rope_bwd_acc, "qk-norm + RoPE backward with weight grads accumulated in place");
  m.def("embedding_fwd", &embedding_fwd, "vocab-parallel embedding lookup (zero rows outside this rank)");
  m.def("embedding_bwd_acc", &embedding_bwd_acc, "embedding backward: scatter-add dy rows into an FP32 grad");
  m.def("sumsq_into", &sumsq_into, "out[0] (+)= sum(x^2), FP32, deterministic");
  m.def("gated_rmsnorm_fwd", &gated_rmsnorm_fwd, "GDN output gate: RMSNorm(o) * w * silu(z)");
  m.def("gated_rmsnorm_bwd", &gated_rmsnorm_bwd);
  m.def("l2norm_fwd", &l2norm_fwd, "row L2 normalisation of a [T, H, D] view");
  m.def("l2norm_bwd", &l2norm_bwd);
  m.def("gdn_gates_fwd", &gdn_gates_fwd, "g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)");
  m.def("gdn_gates_bwd", &gdn_gates_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("moe_route", &moe_route, "MoE top-k routing + stable expert sort (idx, w, counts, offsets, pos, order)");
  m.def("moe_combine", &moe_combine, "y[t] = sum_j w[t,j] ys[pos[t,j]]");
  m.def("moe_combine_bwd", &moe_combine_bwd);
  m.def("moe_route_bwd", &moe_route_bwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("logprob_stats", &logprob_stats);
  m.def("logprob_finalize", &logprob_finalize);
  m.def("logprob_grad_inplace", &logprob_grad_inplace);
  m.def("ppo_loss_fwd", &ppo_loss_fwd);
  m.def("adamw_step", &adamw_step);
  m.def("tree_attn_fwd", &tree_attn_fwd);
  m.def("tree_attn_bwd", &tree_attn_bwd);
  m.def("tree_attn_fwd_sm100", &tree_attn_fwd_sm100, "tcgen05 tree attention forward (head_dim 128)");
  m.def("attn_error_code", &attn_error_code);
  m.def("tree_attn_bwd_sm100", &tree_attn_bwd_sm100, "tcgen05 tree attention backward (head_dim 128)");
  m.def("causal_conv1d_fwd", &causal_conv1d_fwd);
  m.def("causal_conv1d_bwd", &causal_conv1d_bwd);
  m.def("gdr_fwd", &gdr_fwd, "chunked gated delta rule forward (returns o, final state, chunk checkpoints)");
  m.def("gdr_bwd", &gdr_bwd, "chunked gated delta rule backward");
  m.def("attn_phase_profile", &attn_phase_profile, "enable / disable (and clear) tcgen05 attention forward phase timing");
  m.def("attn_phase_read", &attn_phase_read, "attention forward cycles {startup, loop, epilogue, tiles, ctas}");
  m.def("gdr_phase_profile", &gdr_phase_profile, "enable / disable (and clear) gated-delta-rule phase timing");
  m.def("gdr_phase_read", &gdr_phase_read, "summed SM cycles per (kernel, phase) of the gated delta rule");
  m.def("symm_alloc", &symm_alloc, "cudaMalloc + IPC handle (symmetric peer memory)");
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_pad_bytes", &symm_pad_bytes);
  m.def("symm_barrier", &symm_barrier, "cross-GPU barrier over peer signal pads (bounded wait)");
  m.def("dp_reduce_scatter", &dp_reduce_scatter, "P2P-load reduce-scatter of FP32 gradients with scale");
  m.def("dp_adamw_allgather", &dp_adamw_allgather, "AdamW on the local shard + P2P-store parameter all-gather");
  m.def("symm_error_code", &symm_error_code);
  m.def("p2p_gather_rows", &p2p_gather_rows, "out[i] = peer[src_rank[i]][src_row[i]] (P2P loads)");
  m.def("dp_bucket_signal", &dp_bucket_signal, "mark a gradient bucket final on every peer (release store)");
  m.def("dp_bucket_wait", &dp_bucket_wait, "bounded wait until every peer marked the bucket final");
  m.def("p2p_copy", &p2p_copy, "copy-engine copy from a device address (e.g. a peer's symmetric buffer)");
  m.def("p2p_reduce_rows", &p2p_reduce_rows, "out[i] = sum_r peer[r][src_row[i]] (+add) (P2P loads)");
  m.def("symm_clear_error", &symm_clear_error);
  m.def("tp_ag_gemm", &tp_ag_gemm, "all-gather (P2P pull inside the kernel) + tcgen05 GEMM");
  m.def("tp_gemm_rs", &tp_gemm_rs, "tcgen05 GEMM + reduce-scatter (epilogue P2P stores to row owners)");
  m.def("tp_sum_slots", &tp_sum_slots);
  m.def("gemm", &gemm, "tcgen05 GEMM: C (+)= op(A) op(B)^T");
  m.def("gemm_error_code", &gemm_error_code);
  m.def("grouped_gemm", &grouped_gemm, "MoE grouped tcgen05 GEMM (device expert offsets)");
  m.def("grouped_gemm_wgrad", &grouped_gemm_wgrad, "MoE grouped weight gradient, FP32 accumulate");
  m.def("launch_count", &bb_launch_count,
        "kernels launched by this extension so far");
}
