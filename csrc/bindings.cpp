// Python bindings of the sm_100a kernels (module phung5_b200._C).
#include <torch/extension.h>

namespace phx {
void gemm_fp8_block(torch::Tensor xq, torch::Tensor xs, torch::Tensor wq, torch::Tensor ws, torch::Tensor out,
                    torch::Tensor status, int64_t bn, int64_t max_ctas, bool hws, bool pair, int64_t split);
void gemm_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor out, torch::Tensor status, int64_t bn,
               int64_t max_ctas, int64_t split);
void add_rmsnorm_quant(torch::Tensor h, c10::optional<torch::Tensor> delta, torch::Tensor w, double eps,
                       c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> qs,
                       c10::optional<torch::Tensor> out);
void silu_mul_quant(torch::Tensor gu, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> qs,
                    c10::optional<torch::Tensor> out);
void act_quant(torch::Tensor x, torch::Tensor q, torch::Tensor qs);
void rope_kv_write(torch::Tensor qkv, torch::Tensor pos, c10::optional<torch::Tensor> slots, torch::Tensor cos_sin,
                   torch::Tensor q_out, c10::optional<torch::Tensor> k_cache, c10::optional<torch::Tensor> v_cache,
                   int64_t Hq, int64_t Hkv, int64_t D, int64_t page_size);
void paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor pages,
                     torch::Tensor page_indptr, torch::Tensor prefix_len, torch::Tensor q_start,
                     c10::optional<torch::Tensor> tree, torch::Tensor items, torch::Tensor tile_item,
                     torch::Tensor tile_row0, int64_t num_tiles, bool causal, double softmax_scale,
                     c10::optional<torch::Tensor> o_in, c10::optional<torch::Tensor> lse_in,
                     c10::optional<torch::Tensor> o_part, c10::optional<torch::Tensor> lse_part,
                     c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> out_q,
                     c10::optional<torch::Tensor> out_qs);
void paged_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor pages,
                        torch::Tensor page_indptr, torch::Tensor prefix_len, torch::Tensor q_start,
                        c10::optional<torch::Tensor> tree, torch::Tensor items, torch::Tensor tile_item,
                        torch::Tensor tile_row0, int64_t num_tiles, bool causal, double softmax_scale,
                        c10::optional<torch::Tensor> o_in, c10::optional<torch::Tensor> lse_in,
                        c10::optional<torch::Tensor> o_part, c10::optional<torch::Tensor> lse_part,
                        c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> out_q,
                        c10::optional<torch::Tensor> out_qs, torch::Tensor status);
void topk_logprobs(torch::Tensor logits, int64_t k, double temperature, torch::Tensor lp, torch::Tensor idx,
                   c10::optional<torch::Tensor> lse, int64_t vocab_offset);
void gemm_fp8_grouped(torch::Tensor xq, torch::Tensor xs, torch::Tensor wq, torch::Tensor ws, torch::Tensor offsets,
                      torch::Tensor out, torch::Tensor status, bool hws, c10::optional<torch::Tensor> rows);
void gemm_bf16_grouped(torch::Tensor x, torch::Tensor w, torch::Tensor offsets, torch::Tensor out,
                       torch::Tensor status);
void tp_ar_norm(torch::Tensor peer_base, int64_t rank, int64_t world, int64_t M, int64_t H, double eps,
                torch::Tensor w, bool out_bf16, bool push_h, torch::Tensor status, std::vector<int64_t> offsets,
                int64_t s_ld, int64_t off_recv, int64_t mc_base,
                c10::optional<torch::Tensor> phase);
void gemm_scatter(torch::Tensor x, c10::optional<torch::Tensor> xs, torch::Tensor w, c10::optional<torch::Tensor> ws,
                  torch::Tensor peer_base, int64_t off_recv, int64_t rows_per, int64_t rank, torch::Tensor status,
                  bool hws, bool pair, int64_t bn, bool bulk);
void gemm_fp8_swiglu(torch::Tensor xq, torch::Tensor xs, torch::Tensor wq, torch::Tensor ws, torch::Tensor q,
                     torch::Tensor qs, torch::Tensor status);
void moe_combine(torch::Tensor y, torch::Tensor pos, torch::Tensor w, torch::Tensor local, torch::Tensor out);
void tp_allgather(torch::Tensor peer_base, int64_t rank, int64_t world, int64_t nbytes, torch::Tensor status,
                  std::vector<int64_t> offsets, int64_t mc_base);
void gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                   torch::Tensor state, torch::Tensor tok_start, torch::Tensor slot, double scale, torch::Tensor out,
                   bool write_state, c10::optional<torch::Tensor> st_k, c10::optional<torch::Tensor> st_v,
                   c10::optional<torch::Tensor> st_g);
void gdn_fold(torch::Tensor state, torch::Tensor tok_start, torch::Tensor slot, torch::Tensor n_accept,
              torch::Tensor st_k, torch::Tensor st_v, torch::Tensor st_g);
void gdn_gates(torch::Tensor a, torch::Tensor b, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor g,
               torch::Tensor beta);
void causal_conv1d(torch::Tensor x, torch::Tensor window, torch::Tensor w, c10::optional<torch::Tensor> bias,
                   torch::Tensor tok_start, torch::Tensor slot, c10::optional<torch::Tensor> n_commit, torch::Tensor y);
void gated_rmsnorm(torch::Tensor o, torch::Tensor z, torch::Tensor w, double eps, torch::Tensor y);
torch::Tensor raster(torch::Tensor tris, torch::Tensor cols, torch::Tensor vp, int64_t W, int64_t H,
                     std::vector<double> light, double ambient, double diffuse, double exposure, std::vector<double> bg);
void sample_candidates(torch::Tensor logits, int64_t kc, c10::optional<torch::Tensor> temp, int64_t rows_per_temp,
                       int64_t vocab_offset, torch::Tensor cv, torch::Tensor ci, c10::optional<torch::Tensor> cms,
                       torch::Tensor status);
int64_t sample_chunks(int64_t vocab);
void spec_accept(torch::Tensor cv, torch::Tensor ci, int64_t ranks, int64_t nch, int64_t kc, torch::Tensor tokens,
                 torch::Tensor parent, torch::Tensor temp, torch::Tensor top_k, torch::Tensor top_p,
                 torch::Tensor seed, torch::Tensor committed, int64_t D, torch::Tensor acc, torch::Tensor bonus);
torch::Tensor raster_pbr(torch::Tensor tris, torch::Tensor cols, torch::Tensor mats, torch::Tensor vp,
                         std::vector<double> eye, torch::Tensor lights, double ambient, std::vector<double> hemi,
                         double exposure, std::vector<double> bg, int64_t W, int64_t H);
}  // namespace phx

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "phung5_b200 sm_100a kernels";
  m.def("gemm_fp8_block", &phx::gemm_fp8_block);
  m.def("gemm_bf16", &phx::gemm_bf16);
  m.def("gemm_fp8_grouped", &phx::gemm_fp8_grouped);
  m.def("gemm_bf16_grouped", &phx::gemm_bf16_grouped);
  m.def("add_rmsnorm_quant", &phx::add_rmsnorm_quant);
  m.def("silu_mul_quant", &phx::silu_mul_quant);
  m.def("act_quant", &phx::act_quant);
  m.def("rope_kv_write", &phx::rope_kv_write);
  m.def("paged_attention", &phx::paged_attention);
  m.def("paged_attention_tc", &phx::paged_attention_tc);
  m.def("topk_logprobs", &phx::topk_logprobs);
  m.def("tp_ar_norm", &phx::tp_ar_norm);
  m.def("tp_allgather", &phx::tp_allgather);
  m.def("gemm_scatter", &phx::gemm_scatter);
  m.def("moe_combine", &phx::moe_combine);
  m.def("gemm_fp8_swiglu", &phx::gemm_fp8_swiglu);
  m.def("gdn_recurrent", &phx::gdn_recurrent);
  m.def("gdn_fold", &phx::gdn_fold);
  m.def("gdn_gates", &phx::gdn_gates);
  m.def("causal_conv1d", &phx::causal_conv1d);
  m.def("gated_rmsnorm", &phx::gated_rmsnorm);
  m.def("raster", &phx::raster);
  m.def("raster_pbr", &phx::raster_pbr);
  m.def("sample_candidates", &phx::sample_candidates);
  m.def("sample_chunks", &phx::sample_chunks);
  m.def("spec_accept", &phx::spec_accept);
}
