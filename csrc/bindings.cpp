// pybind11 module `aether_b200._C`: every sm_100a kernel entry point.
#include <torch/extension.h>

#include "host_utils.h"

namespace aether {
// gemm_sm100.cu
int64_t gemm_pair_mode(int64_t mode);
void gemm_bf16(at::Tensor a, at::Tensor b, at::Tensor out, bool a_mn, bool b_mn, std::optional<at::Tensor> bias,
               std::optional<at::Tensor> residual, double alpha, bool accumulate, std::optional<at::Tensor> alpha_t);
// gemm_tp.cu
std::string gemm_tp(std::vector<at::Tensor> a_local, std::vector<at::Tensor> a_ag, std::vector<at::Tensor> b,
             std::vector<at::Tensor> out, std::vector<at::Tensor> residual, std::vector<at::Tensor> push_src,
             std::vector<int64_t> ranks, int64_t tp, int64_t Ml, bool b_mn, int64_t ag_mode, bool rs,
             bool local_copy, std::vector<int64_t> ag_buf, std::vector<int64_t> ag_flag, int64_t ag_mc,
             std::vector<int64_t> rs_buf, std::vector<int64_t> rs_flag, int64_t ag_epoch, int64_t rs_epoch,
             double timeout_s);
std::string gemm_param_gather(std::vector<at::Tensor> a, std::vector<at::Tensor> b, std::vector<at::Tensor> out,
                       std::vector<at::Tensor> shard, std::vector<at::Tensor> ctr, std::vector<int64_t> ranks,
                       int64_t world, int64_t chunk, bool b_mn, std::vector<int64_t> unit_buf,
                       std::vector<int64_t> flags, std::vector<int64_t> ready, int64_t mc, int64_t epoch,
                       double timeout_s);
// norm.cu
void rmsnorm_fwd(at::Tensor x, std::optional<at::Tensor> res, at::Tensor w, at::Tensor y,
                 std::optional<at::Tensor> h_out, std::optional<at::Tensor> rstd, double eps);
void rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, std::optional<at::Tensor> dres,
                 at::Tensor dx, at::Tensor dw_f32, bool accumulate);
void layernorm_fwd(at::Tensor x, std::optional<at::Tensor> res, at::Tensor w, std::optional<at::Tensor> b,
                   at::Tensor y, std::optional<at::Tensor> h_out, at::Tensor mean, at::Tensor rstd, double eps);
void layernorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor mean, at::Tensor rstd,
                   std::optional<at::Tensor> dres, at::Tensor dx, at::Tensor dw_f32, at::Tensor db_f32,
                   bool accumulate);
void softmax_fwd(at::Tensor x, at::Tensor y, double scale);
void softmax_bwd(at::Tensor y, at::Tensor dy, at::Tensor dx, double scale);
// elementwise.cu
void swiglu_fwd(at::Tensor h, at::Tensor act);
void swiglu_bwd(at::Tensor h, at::Tensor dact, at::Tensor dh);
void gelu_fwd(at::Tensor x, at::Tensor y);
void gelu_bwd(at::Tensor x, at::Tensor dy, at::Tensor dx);
void rope_apply(at::Tensor x, at::Tensor pos, at::Tensor cos_t, at::Tensor sin_t, int64_t n_heads, int64_t head_dim,
                bool inverse);
void embedding_fwd(at::Tensor table, at::Tensor ids, at::Tensor out);
void embedding_bwd(at::Tensor dy, at::Tensor ids, at::Tensor dtable_f32);
// loss.cu
void cross_entropy_fused(at::Tensor logits, at::Tensor targets, at::Tensor loss, std::optional<at::Tensor> lse,
                         std::optional<at::Tensor> dlogits, std::optional<at::Tensor> scale_t, double scale,
                         int64_t ignore_index);
void argmax_rows(at::Tensor x, at::Tensor out);
// optim.cu
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, std::optional<at::Tensor> p_bf16, double lr,
                double beta1, double beta2, double eps, double wd, int64_t step, double gscale,
                std::optional<at::Tensor> gscale_t);
void sgd_step(at::Tensor p, at::Tensor g, std::optional<at::Tensor> buf, std::optional<at::Tensor> p_bf16, double lr,
              double momentum, double wd, double gscale, std::optional<at::Tensor> gscale_t);
void grad_norm(at::Tensor g, at::Tensor norm_out, std::optional<at::Tensor> clip_out, double pre_scale,
               double max_norm);
// attention.cu
void attention_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, std::optional<at::Tensor> lse,
                   double scale, bool causal, int64_t causal_offset, int64_t window, double softcap);
void attention_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor dout, at::Tensor lse,
                   at::Tensor dq, at::Tensor dk, at::Tensor dv, double scale, bool causal, int64_t causal_offset,
                   bool use_tc, int64_t window, double softcap);
// attention_sm100.cu
void attention_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, std::optional<at::Tensor> lse,
                      double scale, bool causal, int64_t causal_offset, int64_t window, double softcap);
// gemm_skinny.cu
void skinny_gemm(at::Tensor x, at::Tensor w, at::Tensor acc, int64_t splits, int64_t acc_mc,
                 std::optional<at::Tensor> sig_peers, std::optional<at::Tensor> sig_epoch,
                 std::optional<at::Tensor> sig_done, int64_t sig_rank, int64_t sig_world);
// tp_decode.cu
void tp_vocab_argmax(at::Tensor logits, int64_t n_loc, int64_t col0, at::Tensor flag_peers, at::Tensor ctr,
                     int64_t rows_cap, at::Tensor out, int64_t rank, int64_t world, double timeout_s);
void tp_put_cols(at::Tensor src, int64_t n_loc, int64_t col0, at::Tensor data_peers, int64_t ldd, int64_t rank,
                 int64_t world);
void tp_push_reduce(at::Tensor acc, at::Tensor y, std::optional<at::Tensor> bias, std::optional<at::Tensor> res,
                    std::optional<at::Tensor> w, std::optional<at::Tensor> h, double eps, at::Tensor data_peers,
                    int64_t data_mc, int64_t ld, at::Tensor flag_peers, at::Tensor ctr, int64_t rows_cap,
                    int64_t rank, int64_t world, double timeout_s);
void skinny_gemm_swiglu(at::Tensor x, at::Tensor w, at::Tensor acc, at::Tensor act, at::Tensor tile_cnt,
                        int64_t splits);
void skinny_gemm_qkv(at::Tensor x, at::Tensor w, at::Tensor acc, at::Tensor tile_cnt, std::optional<at::Tensor> bias,
                     at::Tensor qkv, at::Tensor pos, at::Tensor slot, at::Tensor cos_t, at::Tensor sin_t,
                     at::Tensor k_cache, at::Tensor v_cache, int64_t Hq, int64_t Hkv,
                     std::optional<at::Tensor> page_table, int64_t splits);
// gguf_dequant.cu
bool gguf_device_type(int64_t type);
void gguf_dequant(at::Tensor blocks, int64_t type, int64_t rows, int64_t K, at::Tensor out);
// decode_mega.cu
void decode_mega(at::Tensor layers, at::Tensor embed, at::Tensor final_norm, at::Tensor head, int64_t vocab_rows,
                 int64_t vocab_col0, int64_t d, int64_t hq, int64_t hkv, int64_t f, double eps, double scale,
                 at::Tensor tok, at::Tensor pos, at::Tensor slot, at::Tensor seqlen, at::Tensor next,
                 std::optional<at::Tensor> logits, at::Tensor cache0, std::optional<at::Tensor> page_table,
                 at::Tensor x, at::Tensor x2, at::Tensor q, at::Tensor o, at::Tensor act, at::Tensor part,
                 at::Tensor pair_ctr, at::Tensor red0, at::Tensor red1, int64_t red0_mc, int64_t red1_mc,
                 at::Tensor flags, at::Tensor flag_peers, at::Tensor keys, at::Tensor key_peers, int64_t rank,
                 int64_t world, at::Tensor state, double timeout_s, std::optional<at::Tensor> trace,
                 int64_t debug);
// comm.cu
void team_barrier(at::Tensor peer_sig_ptrs, at::Tensor my_sig, at::Tensor epoch, int64_t rank, int64_t world,
                  double timeout_s);
void allreduce_oneshot(at::Tensor peers, at::Tensor out, int64_t world);
void allreduce_nvls(int64_t mc_ptr, int64_t numel, bool is_bf16, int64_t rank, int64_t world);
void dp_reduce_adamw(at::Tensor grad_peers, int64_t grad_mc, at::Tensor param_peers, int64_t param_mc,
                     at::Tensor master, at::Tensor m, at::Tensor v, at::Tensor decay_blocks, int64_t begin, int64_t n,
                     int64_t world, double lr, double beta1, double beta2, double eps, double wd, int64_t step,
                     double gscale, std::optional<at::Tensor> gscale_t);
void skinny_finalize(at::Tensor acc, at::Tensor y, std::optional<at::Tensor> bias, std::optional<at::Tensor> res,
                     bool swiglu, std::optional<at::Tensor> wait_sig, std::optional<at::Tensor> wait_epoch,
                     int64_t wait_rank, int64_t wait_world, double wait_timeout_s);
// decode_attention.cu
void rope_kv_append(at::Tensor qkv, at::Tensor pos, at::Tensor slot, at::Tensor cos_t, at::Tensor sin_t,
                    at::Tensor k_cache, at::Tensor v_cache, int64_t Hq, int64_t Hkv, int64_t D,
                    std::optional<at::Tensor> page_table);
void decode_attention(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor slot, at::Tensor seqlen,
                      at::Tensor out, at::Tensor part_o, at::Tensor part_lse, int64_t Hq, int64_t splits,
                      double scale, std::optional<at::Tensor> counters, std::optional<at::Tensor> page_table,
                      int64_t window, double softcap);
void qkv_finalize_rope(at::Tensor acc, std::optional<at::Tensor> bias, at::Tensor qkv, at::Tensor pos, at::Tensor slot,
                       at::Tensor cos_t, at::Tensor sin_t, at::Tensor k_cache, at::Tensor v_cache, int64_t Hq,
                       int64_t Hkv, int64_t D, std::optional<at::Tensor> page_table);
void finalize_residual_norm(at::Tensor acc, std::optional<at::Tensor> bias, std::optional<at::Tensor> res,
                            at::Tensor y, at::Tensor w, at::Tensor h, double eps,
                            std::optional<at::Tensor> wait_sig, std::optional<at::Tensor> wait_epoch,
                            int64_t wait_rank, int64_t wait_world, double wait_timeout_s);
// gemm_sm100.cu (grouped) and moe.cu
void gemm_grouped(at::Tensor a, at::Tensor w, at::Tensor out, at::Tensor tile_group);
void moe_route(at::Tensor logits, at::Tensor idx, at::Tensor wt, int64_t k, bool softmax_all, bool renorm,
               bool sigmoid, double scale);
// mla.cu
void mla_attention(at::Tensor q_abs, at::Tensor cache, at::Tensor slot, at::Tensor seqlen, at::Tensor out,
                   at::Tensor part_o, at::Tensor part_lse, int64_t splits, double scale);
void mla_prep(at::Tensor kv_a, at::Tensor norm_w, double eps, at::Tensor q, int64_t H, int64_t q_hd, int64_t nope,
              at::Tensor pos, at::Tensor slot, at::Tensor cos_t, at::Tensor sin_t, at::Tensor cache,
              at::Tensor q_abs);
void moe_permute(at::Tensor idx, int64_t E, at::Tensor row_of, at::Tensor src_row, at::Tensor tile_group,
                 int64_t e0);
void moe_gather(at::Tensor x, at::Tensor src_row, at::Tensor X);
void moe_combine(at::Tensor Y, at::Tensor row_of, at::Tensor wt, int64_t k, std::optional<at::Tensor> res,
                 std::optional<at::Tensor> extra, at::Tensor out);
void head_rmsnorm(at::Tensor x, int64_t h0, int64_t nh, int64_t D, at::Tensor w, double eps);
// quant.cu
void quantize_blocks(at::Tensor x, at::Tensor out, int64_t fmt);
void dequantize_blocks(at::Tensor in, at::Tensor y, int64_t fmt);
}  // namespace aether

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace pybind11::literals;
  m.doc() = "aether_b200 sm_100a kernels";
  m.def("gemm_pair_mode", &aether::gemm_pair_mode, "mode"_a,
        "GEMM kernel choice: 0 one-CTA, 1 CTA pair for M, N >= 256, -1 measured default; returns the previous");
  m.def("gemm_bf16", &aether::gemm_bf16, "a"_a, "b"_a, "out"_a, "a_mn"_a, "b_mn"_a, "bias"_a = pybind11::none(),
        "residual"_a = pybind11::none(), "alpha"_a = 1.0, "accumulate"_a = false,
        "alpha_t"_a = pybind11::none());
  m.def("gemm_tp", &aether::gemm_tp, "a_local"_a, "a_ag"_a, "b"_a, "out"_a, "residual"_a, "push_src"_a, "ranks"_a,
        "tp"_a, "Ml"_a, "b_mn"_a, "ag_mode"_a, "rs"_a, "local_copy"_a, "ag_buf"_a, "ag_flag"_a, "ag_mc"_a,
        "rs_buf"_a, "rs_flag"_a, "ag_epoch"_a, "rs_epoch"_a, "timeout_s"_a,
        "tcgen05 GEMM with the TP all-gather / reduce-scatter fused in (sequence-parallel training)");
  m.def("gemm_param_gather", &aether::gemm_param_gather, "a"_a, "b"_a, "out"_a, "shard"_a, "ctr"_a, "ranks"_a,
        "world"_a, "chunk"_a, "b_mn"_a, "unit_buf"_a, "flags"_a, "ready"_a, "mc"_a, "epoch"_a, "timeout_s"_a,
        "tcgen05 GEMM whose weight operand is all-gathered (ZeRO-3) inside the same kernel");
  m.def("rmsnorm_fwd", &aether::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &aether::rmsnorm_bwd);
  m.def("layernorm_fwd", &aether::layernorm_fwd);
  m.def("layernorm_bwd", &aether::layernorm_bwd);
  m.def("softmax_fwd", &aether::softmax_fwd);
  m.def("softmax_bwd", &aether::softmax_bwd);
  m.def("swiglu_fwd", &aether::swiglu_fwd);
  m.def("swiglu_bwd", &aether::swiglu_bwd);
  m.def("gelu_fwd", &aether::gelu_fwd);
  m.def("gelu_bwd", &aether::gelu_bwd);
  m.def("rope_apply", &aether::rope_apply);
  m.def("embedding_fwd", &aether::embedding_fwd);
  m.def("embedding_bwd", &aether::embedding_bwd);
  m.def("cross_entropy_fused", &aether::cross_entropy_fused);
  m.def("argmax_rows", &aether::argmax_rows);
  m.def("adamw_step", &aether::adamw_step);
  m.def("sgd_step", &aether::sgd_step);
  m.def("grad_norm", &aether::grad_norm);
  m.def("attention_fwd", &aether::attention_fwd, "q"_a, "k"_a, "v"_a, "out"_a, "lse"_a, "scale"_a, "causal"_a,
        "causal_offset"_a, "window"_a = 0, "softcap"_a = 0.0);
  m.def("attention_bwd", &aether::attention_bwd, "q"_a, "k"_a, "v"_a, "out"_a, "dout"_a, "lse"_a, "dq"_a, "dk"_a,
        "dv"_a, "scale"_a, "causal"_a, "causal_offset"_a, "use_tc"_a = false, "window"_a = 0, "softcap"_a = 0.0);
  m.def("attention_fwd_tc", &aether::attention_fwd_tc, "q"_a, "k"_a, "v"_a, "out"_a, "lse"_a, "scale"_a, "causal"_a,
        "causal_offset"_a, "window"_a = 0, "softcap"_a = 0.0);
  m.def("skinny_gemm", &aether::skinny_gemm, "x"_a, "w"_a, "acc"_a, "splits"_a = 0, "acc_mc"_a = 0,
        "sig_peers"_a = pybind11::none(), "sig_epoch"_a = pybind11::none(), "sig_done"_a = pybind11::none(),
        "sig_rank"_a = 0, "sig_world"_a = 0);
  m.def("team_barrier", &aether::team_barrier);
  m.def("skinny_gemm_swiglu", &aether::skinny_gemm_swiglu);
  m.def("skinny_gemm_qkv", &aether::skinny_gemm_qkv);
  m.def("gguf_device_type", &aether::gguf_device_type);
  m.def("gguf_dequant", &aether::gguf_dequant);
  m.def("decode_mega", &aether::decode_mega, "layers"_a, "embed"_a, "final_norm"_a, "head"_a, "vocab_rows"_a,
        "vocab_col0"_a, "d"_a, "hq"_a, "hkv"_a, "f"_a, "eps"_a, "scale"_a, "tok"_a, "pos"_a, "slot"_a, "seqlen"_a,
        "next"_a, "logits"_a, "cache0"_a, "page_table"_a, "x"_a, "x2"_a, "q"_a, "o"_a, "act"_a, "part"_a,
        "pair_ctr"_a, "red0"_a, "red1"_a, "red0_mc"_a, "red1_mc"_a, "flags"_a, "flag_peers"_a, "keys"_a,
        "key_peers"_a, "rank"_a, "world"_a, "state"_a, "timeout_s"_a, "trace"_a = pybind11::none(), "debug"_a = 0);
  m.def("tp_vocab_argmax", &aether::tp_vocab_argmax);
  m.def("tp_put_cols", &aether::tp_put_cols);
  m.def("tp_push_reduce", &aether::tp_push_reduce, "acc"_a, "y"_a, "bias"_a, "res"_a, "w"_a, "h"_a, "eps"_a,
        "data_peers"_a, "data_mc"_a, "ld"_a, "flag_peers"_a, "ctr"_a, "rows_cap"_a, "rank"_a, "world"_a,
        "timeout_s"_a);
  m.def("allreduce_oneshot", &aether::allreduce_oneshot);
  m.def("allreduce_nvls", &aether::allreduce_nvls);
  m.def("dp_reduce_adamw", &aether::dp_reduce_adamw);
  m.def("skinny_finalize", &aether::skinny_finalize, "acc"_a, "y"_a, "bias"_a, "res"_a, "swiglu"_a,
        "wait_sig"_a = pybind11::none(), "wait_epoch"_a = pybind11::none(), "wait_rank"_a = 0, "wait_world"_a = 0,
        "wait_timeout_s"_a = 10.0);
  m.def("rope_kv_append", &aether::rope_kv_append, "qkv"_a, "pos"_a, "slot"_a, "cos_t"_a, "sin_t"_a, "k_cache"_a,
        "v_cache"_a, "Hq"_a, "Hkv"_a, "D"_a, "page_table"_a = pybind11::none());
  m.def("decode_attention", &aether::decode_attention, "q"_a, "k_cache"_a, "v_cache"_a, "slot"_a, "seqlen"_a, "out"_a,
        "part_o"_a, "part_lse"_a, "Hq"_a, "splits"_a, "scale"_a, "counters"_a = pybind11::none(),
        "page_table"_a = pybind11::none(), "window"_a = 0, "softcap"_a = 0.0);
  m.def("qkv_finalize_rope", &aether::qkv_finalize_rope, "acc"_a, "bias"_a, "qkv"_a, "pos"_a, "slot"_a, "cos_t"_a,
        "sin_t"_a, "k_cache"_a, "v_cache"_a, "Hq"_a, "Hkv"_a, "D"_a, "page_table"_a = pybind11::none());
  m.def("finalize_residual_norm", &aether::finalize_residual_norm, "acc"_a, "bias"_a, "res"_a, "y"_a, "w"_a, "h"_a,
        "eps"_a, "wait_sig"_a = pybind11::none(), "wait_epoch"_a = pybind11::none(), "wait_rank"_a = 0,
        "wait_world"_a = 0, "wait_timeout_s"_a = 10.0);
  m.def("gemm_grouped", &aether::gemm_grouped, "grouped (MoE) tcgen05 GEMM over 128-row expert tiles");
  m.def("moe_route", &aether::moe_route, "logits"_a, "idx"_a, "wt"_a, "k"_a, "softmax_all"_a, "renorm"_a,
        "sigmoid"_a = false, "scale"_a = 1.0);
  m.def("mla_attention", &aether::mla_attention);
  m.def("mla_prep", &aether::mla_prep);
  m.def("moe_permute", &aether::moe_permute, "idx"_a, "E"_a, "row_of"_a, "src_row"_a, "tile_group"_a, "e0"_a = 0);
  m.def("moe_gather", &aether::moe_gather);
  m.def("moe_combine", &aether::moe_combine);
  m.def("head_rmsnorm", &aether::head_rmsnorm, "in-place per-head RMSNorm (Qwen3 q/k norm)");
  m.def("quantize_blocks", &aether::quantize_blocks, "bf16 -> GGUF Q8_0 (fmt 8) or Q4_0 (fmt 2) blocks");
  m.def("dequantize_blocks", &aether::dequantize_blocks, "GGUF Q8_0 / Q4_0 blocks -> bf16");
  m.def("read_and_clear_status", &aether::read_and_clear_status,
        "Returns (and clears) the device status word set by kernels whose bounded waits expired");
}
