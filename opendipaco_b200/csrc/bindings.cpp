// Python bindings of the sm_100a kernels (module opendipaco_b200._C).
#include <torch/extension.h>

void gemm_bf16(torch::Tensor A, int64_t lda, int64_t sa, bool a_mn, torch::Tensor B, int64_t ldb, int64_t sb,
               bool b_mn, torch::Tensor C, int64_t ldc, int64_t sc, int64_t M, int64_t N, int64_t K, int64_t G,
               int64_t epi, int64_t bn, c10::optional<torch::Tensor> R, int64_t ldr, int64_t sr,
               c10::optional<torch::Tensor> aux, int64_t ldx, int64_t sx, c10::optional<torch::Tensor> part,
               double beta, int64_t f_half, torch::Tensor err, int64_t max_ctas,
               c10::optional<torch::Tensor> sq_part, int64_t sq_ld);
void rmsnorm_fwd(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor y, int64_t sy,
                 torch::Tensor rstd, int64_t M, int64_t H, int64_t G, double eps);
void rmsnorm_fwd_rpw(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor y, int64_t sy,
                     torch::Tensor rstd, int64_t M, int64_t H, int64_t G, double eps, int64_t rows_per_warp);
void rmsnorm_bwd(torch::Tensor x, int64_t sx, torch::Tensor w, int64_t sw, torch::Tensor rstd, torch::Tensor dy,
                 int64_t sdy, c10::optional<torch::Tensor> dres, torch::Tensor dx, int64_t sdx,
                 c10::optional<torch::Tensor> dx16, torch::Tensor dw, int64_t sdw, torch::Tensor work, int64_t M,
                 int64_t H, int64_t G, double beta);
void embedding_fwd(torch::Tensor ids, torch::Tensor E, int64_t se, torch::Tensor out, int64_t M, int64_t H,
                   int64_t G, int64_t V);
void embedding_bwd(torch::Tensor ids, torch::Tensor dx, int64_t sdx, torch::Tensor dE, int64_t se, int64_t M,
                   int64_t H, int64_t G, int64_t V);
void embedding_bwd_sorted(torch::Tensor ids, torch::Tensor dx, int64_t sdx, torch::Tensor dE, int64_t se, int64_t M,
                          int64_t H, int64_t G, int64_t V, torch::Tensor keys, c10::optional<torch::Tensor> rows,
                          c10::optional<torch::Tensor> sq);
void gemm_ce_grad(torch::Tensor A, int64_t lda, int64_t sa, bool a_mn, torch::Tensor B, int64_t ldb, int64_t sb,
                  bool b_mn, torch::Tensor C, int64_t ldc, int64_t sc, int64_t M, int64_t N, int64_t K, int64_t G,
                  double beta, torch::Tensor err, c10::optional<torch::Tensor> sq_part, int64_t sq_ld, int64_t xf,
                  torch::Tensor ob, torch::Tensor labels, torch::Tensor scale, int64_t ms, int64_t split);
void gemm_splitk_reduce(torch::Tensor ws, int64_t S, int64_t G, int64_t M, int64_t N, torch::Tensor C, int64_t ldc,
                        int64_t sc, c10::optional<torch::Tensor> sq_part, int64_t sq_ld, double beta);
void grad_clip_coef_parts(torch::Tensor parts, int64_t nslot, torch::Tensor esq, int64_t M, torch::Tensor grads,
                          int64_t P, torch::Tensor norm_offs, int64_t H, int64_t G, double max_norm, torch::Tensor coef,
                          c10::optional<torch::Tensor> norm_out);
void attention_fwd(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                   torch::Tensor sinT, torch::Tensor o, torch::Tensor lse);
void attention_bwd(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                   torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor dout, torch::Tensor delta,
                   torch::Tensor dqkv);
void attention_fwd_tc(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                      torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor err);
void attention_bwd_tc(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                      torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor dout, torch::Tensor dqkv,
                      torch::Tensor err);
void attention_fwd_flash(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                         torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor err,
                         c10::optional<torch::Tensor> qkr);
void attention_bwd_flash(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                         torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor dout,
                         torch::Tensor delta, torch::Tensor dqkv, torch::Tensor err,
                         c10::optional<torch::Tensor> qkr);
void ce_fused(torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor labels, int64_t M, int64_t V, int64_t G,
              torch::Tensor lse, torch::Tensor row_loss, torch::Tensor loss_sum, torch::Tensor inv_count,
              c10::optional<torch::Tensor> loss_out, torch::Tensor err, c10::optional<torch::Tensor> inv_given,
              c10::optional<torch::Tensor> ob);
void dp_barrier(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, torch::Tensor err);
void dp_grad_reduce_norm(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, int64_t G, int64_t P,
                         int64_t stride, int64_t s0, int64_t s1, torch::Tensor part, double max_norm,
                         torch::Tensor coef, torch::Tensor gnorm, torch::Tensor err);
void dp_adamw(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, int64_t G, int64_t stride,
              int64_t stride16, int64_t s0, int64_t s1, torch::Tensor coef, torch::Tensor sched, double b1, double b2,
              double eps, double wd, torch::Tensor err);
void dp_adam8bit(torch::Tensor tab, torch::Tensor counter, int64_t me, int64_t d, int64_t G, int64_t P, int64_t s0,
                 int64_t s1, torch::Tensor coef, torch::Tensor sched, double b1, double b2, double eps, double wd,
                 torch::Tensor err);
void ce_forward(torch::Tensor part, int64_t T, torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor labels,
                int64_t M, int64_t G, torch::Tensor lse, torch::Tensor row_loss, torch::Tensor loss_sum,
                torch::Tensor inv_count, c10::optional<torch::Tensor> loss_out, c10::optional<torch::Tensor> inv_given);
void ce_backward(torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor lse, torch::Tensor labels,
                 torch::Tensor inv_count, int64_t M, int64_t V, int64_t G);
torch::Tensor cross_entropy_rows(torch::Tensor logits, torch::Tensor target);
void ce_label_count(torch::Tensor labels, int64_t M, int64_t G, torch::Tensor inv_count);
void ce_group_sum(torch::Tensor row_loss, torch::Tensor labels, int64_t M, int64_t G, torch::Tensor loss_sum,
                  torch::Tensor inv_count, c10::optional<torch::Tensor> loss_out, c10::optional<torch::Tensor> inv_given);
void ce_rows_chunk(torch::Tensor logits, int64_t ldl, int64_t sl, torch::Tensor labels, int64_t Mc, int64_t ms,
                   int64_t V, int64_t G, torch::Tensor lse, torch::Tensor row_loss, torch::Tensor inv,
                   c10::optional<torch::Tensor> part, int64_t T, torch::Tensor err, c10::optional<torch::Tensor> ob);
void grad_clip_coef(torch::Tensor grads, int64_t P, int64_t sg, int64_t G, double max_norm, torch::Tensor work,
                    torch::Tensor coef, c10::optional<torch::Tensor> norm_out, c10::optional<torch::Tensor> rows,
                    int64_t r0, int64_t H, int64_t V);
void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor p16, int64_t P,
                int64_t sp, int64_t s16, int64_t G, c10::optional<torch::Tensor> coef, torch::Tensor sched, double b1,
                double b2, double eps, double wd, c10::optional<torch::Tensor> rows, int64_t r0, int64_t H,
                int64_t V);
void adamw_acc_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor p16, int64_t ctas,
                    int64_t sp, int64_t s16, c10::optional<torch::Tensor> coef, torch::Tensor sched, double b1,
                    double b2, double eps, double wd, c10::optional<torch::Tensor> rows, int64_t r0, int64_t H,
                    int64_t V, torch::Tensor regions, int64_t nregs, torch::Tensor entries, bool accumulate);
void adam8bit_step(torch::Tensor p, torch::Tensor g, torch::Tensor mq, torch::Tensor mabs, torch::Tensor vq,
                   torch::Tensor vlo, torch::Tensor vsc, c10::optional<torch::Tensor> coef, torch::Tensor sched,
                   double b1, double b2, double eps, double wd, bool first, c10::optional<torch::Tensor> p16,
                   int64_t blocks_per_group);
void outer_step(torch::Tensor segs, int64_t nseg, torch::Tensor locals, int64_t total_chunks, double lr,
                double momentum, bool nesterov, bool first, c10::optional<torch::Tensor> sq_part,
                c10::optional<torch::Tensor> status);
int64_t outer_chunk_elems();
void outer_nvlink_apply(torch::Tensor keys, int64_t nkeys, int64_t total_chunks, torch::Tensor delta_ptrs,
                        torch::Tensor glob_ptrs, torch::Tensor pads, torch::Tensor mom, int64_t rank, int64_t world,
                        int64_t epoch, double lr, double m, bool nesterov, bool first, torch::Tensor sq_part,
                        torch::Tensor err, c10::optional<torch::Tensor> qd_ptrs,
                        c10::optional<torch::Tensor> qs_ptrs, int64_t kcap, c10::optional<torch::Tensor> status);
void outer_nvlink_topk(torch::Tensor regs, int64_t nregs, int64_t total_blocks, double density, int64_t kcap,
                       torch::Tensor delta, torch::Tensor res, torch::Tensor spi, torch::Tensor spv);
void outer_nvlink_quant(torch::Tensor regs, int64_t nregs, int64_t total_groups, torch::Tensor delta,
                        torch::Tensor res, torch::Tensor qd, torch::Tensor qs);
void outer_nvlink_bcast(torch::Tensor segs, int64_t nseg, torch::Tensor locals, int64_t total_chunks,
                        torch::Tensor pads, int64_t rank, int64_t world, int64_t epoch, torch::Tensor err);
int64_t outer_nvlink_chunk_elems();
int64_t set_peer_wait_ns(int64_t ns);
std::vector<torch::Tensor> quant_int4(torch::Tensor x, bool want_resid);
void dequant_int4(torch::Tensor packed, torch::Tensor scale, int64_t n, int64_t g, torch::Tensor out, double w,
                  bool accumulate);
std::vector<torch::Tensor> quant_int8(torch::Tensor x, bool want_resid);
torch::Tensor robust_combine(torch::Tensor stack, int64_t mode);
torch::Tensor bag_of_tokens(torch::Tensor ids, torch::Tensor offs, torch::Tensor proj);
std::vector<torch::Tensor> kmeans_assign(torch::Tensor x, torch::Tensor c, int64_t topk, bool want_min,
                                         bool want_dist, torch::Tensor err);
std::vector<torch::Tensor> kmeans_cluster_sums(torch::Tensor x, torch::Tensor assign, int64_t K);
void peer_copy(torch::Tensor table, int64_t max_elems);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "opendipaco_b200 sm_100a kernels";
  m.def("gemm_bf16", &gemm_bf16);
  m.def("gemm_splitk_reduce", &gemm_splitk_reduce);
  m.def("gemm_ce_grad", &gemm_ce_grad);
  m.def("grad_clip_coef_parts", &grad_clip_coef_parts);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_fwd_rpw", &rmsnorm_fwd_rpw);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("attention_fwd", &attention_fwd);
  m.def("attention_bwd", &attention_bwd);
  m.def("attention_fwd_tc", &attention_fwd_tc);
  m.def("attention_fwd_flash", &attention_fwd_flash, py::arg("qkv"), py::arg("GB"), py::arg("S"), py::arg("nh"),
        py::arg("nkv"), py::arg("cosT"), py::arg("sinT"), py::arg("o"), py::arg("lse"), py::arg("err"),
        py::arg("qkr") = py::none());
  m.def("attention_bwd_flash", &attention_bwd_flash, py::arg("qkv"), py::arg("GB"), py::arg("S"), py::arg("nh"),
        py::arg("nkv"), py::arg("cosT"), py::arg("sinT"), py::arg("o"), py::arg("lse"), py::arg("dout"),
        py::arg("delta"), py::arg("dqkv"), py::arg("err"), py::arg("qkr") = py::none());
  m.def("ce_fused", &ce_fused, py::arg("logits"), py::arg("ldl"), py::arg("sl"), py::arg("labels"), py::arg("M"),
        py::arg("V"), py::arg("G"), py::arg("lse"), py::arg("row_loss"), py::arg("loss_sum"), py::arg("inv_count"),
        py::arg("loss_out"), py::arg("err"), py::arg("inv_given"), py::arg("ob") = py::none());
  m.def("embedding_bwd_sorted", &embedding_bwd_sorted);
  m.def("dp_barrier", &dp_barrier);
  m.def("dp_grad_reduce_norm", &dp_grad_reduce_norm);
  m.def("dp_adamw", &dp_adamw);
  m.def("dp_adam8bit", &dp_adam8bit);
  m.def("outer_nvlink_quant", &outer_nvlink_quant);
  m.def("outer_nvlink_topk", &outer_nvlink_topk);
  m.def("attention_bwd_tc", &attention_bwd_tc);
  m.def("ce_forward", &ce_forward);
  m.def("ce_backward", &ce_backward);
  m.def("cross_entropy_rows", &cross_entropy_rows);
  m.def("ce_label_count", &ce_label_count);
  m.def("ce_group_sum", &ce_group_sum);
  m.def("ce_rows_chunk", &ce_rows_chunk, py::arg("logits"), py::arg("ldl"), py::arg("sl"), py::arg("labels"),
        py::arg("Mc"), py::arg("ms"), py::arg("V"), py::arg("G"), py::arg("lse"), py::arg("row_loss"), py::arg("inv"),
        py::arg("part"), py::arg("T"), py::arg("err"), py::arg("ob") = py::none());
  m.def("grad_clip_coef", &grad_clip_coef);
  m.def("adamw_step", &adamw_step);
  m.def("adam8bit_step", &adam8bit_step);
  m.def("adamw_acc_step", &adamw_acc_step);
  m.def("outer_step", &outer_step);
  m.def("outer_chunk_elems", &outer_chunk_elems);
  m.def("outer_nvlink_apply", &outer_nvlink_apply);
  m.def("outer_nvlink_bcast", &outer_nvlink_bcast);
  m.def("outer_nvlink_chunk_elems", &outer_nvlink_chunk_elems);
  m.def("set_peer_wait_ns", &set_peer_wait_ns);
  m.def("quant_int4", &quant_int4);
  m.def("dequant_int4", &dequant_int4);
  m.def("quant_int8", &quant_int8);
  m.def("robust_combine", &robust_combine);
  m.def("bag_of_tokens", &bag_of_tokens);
  m.def("kmeans_assign", &kmeans_assign);
  m.def("kmeans_cluster_sums", &kmeans_cluster_sums);
  m.def("peer_copy", &peer_copy);
}
