// Python bindings of the sm_100a kernel library (module openmini_v1_b200._C).
#include <torch/extension.h>

void om_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> resid,
             c10::optional<torch::Tensor> workspace, torch::Tensor status, int64_t force_swap,
             int64_t force_splits, std::vector<int64_t> peer);
std::vector<int64_t> om_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t sms, bool allow_split);
void om_gemm_wq(torch::Tensor x, torch::Tensor qtiles, c10::optional<torch::Tensor> scales, int64_t qtype,
                torch::Tensor out, c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> workspace,
                torch::Tensor status, int64_t force_swap, int64_t force_splits, std::vector<int64_t> peer,
                c10::optional<torch::Tensor> sem, std::vector<int64_t> agwait);
void om_rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> delta, torch::Tensor w, torch::Tensor out,
                double eps);
void om_layernorm(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, torch::Tensor out,
                  double eps);
void om_silu_mul(torch::Tensor gu, torch::Tensor out);
void om_gelu(torch::Tensor x, torch::Tensor y);
void om_softmax(torch::Tensor x, torch::Tensor y, double scale);
void om_embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, torch::Tensor status);
void om_rope_kv(torch::Tensor qkv, torch::Tensor positions, torch::Tensor slots, torch::Tensor k_cache,
                torch::Tensor v_cache, torch::Tensor inv_freq, int64_t Hq, int64_t Hkv, int64_t D, int64_t mode,
                torch::Tensor status);
void om_kv_write(torch::Tensor k, torch::Tensor v, torch::Tensor slots, torch::Tensor k_cache,
                 torch::Tensor v_cache);
void om_paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                        torch::Tensor row_seq, torch::Tensor row_ctx, torch::Tensor out, torch::Tensor workspace,
                        int64_t Hq, int64_t max_ctx, double scale, torch::Tensor status);
void om_paged_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                           torch::Tensor row_seq, torch::Tensor row_ctx, torch::Tensor out, torch::Tensor workspace,
                           int64_t Hq, int64_t max_ctx, double scale, torch::Tensor status);
int64_t om_paged_attention_workspace(int64_t rows, int64_t Hq, int64_t D, int64_t max_ctx);
void om_sample(torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_p, torch::Tensor top_k,
               torch::Tensor rng, torch::Tensor out_tok, c10::optional<torch::Tensor> out_logprob,
               c10::optional<torch::Tensor> keep_mask);
void om_repetition_penalty(torch::Tensor logits, torch::Tensor prev, torch::Tensor penalty);
void om_decode_advance(torch::Tensor sampled, torch::Tensor ids, torch::Tensor pos, torch::Tensor ctx,
                       torch::Tensor slots, torch::Tensor bt, torch::Tensor rng, c10::optional<torch::Tensor> hist,
                       torch::Tensor step);
void om_quantize_q4(torch::Tensor w, torch::Tensor q, torch::Tensor scales, c10::optional<torch::Tensor> scales_f16);
void om_dequant_q4(torch::Tensor q, torch::Tensor scales, torch::Tensor out);
void om_quantize_int8(torch::Tensor w, torch::Tensor q, torch::Tensor scale);
void om_dequant_int8(torch::Tensor q, torch::Tensor scale, torch::Tensor out);
void om_gguf_dequant(torch::Tensor raw, int64_t type, torch::Tensor out);

void om_dsa_scores(torch::Tensor qi, torch::Tensor wi, int64_t H, torch::Tensor icache, torch::Tensor bt,
                   torch::Tensor row_seq, torch::Tensor row_ctx, torch::Tensor scores, torch::Tensor status);
void om_dsa_topk(torch::Tensor scores, torch::Tensor row_ctx, int64_t k, torch::Tensor out_idx, torch::Tensor out_n);
void om_dsa_head_reduce(torch::Tensor g, int64_t S, torch::Tensor w, int64_t H, torch::Tensor row_ctx,
                        torch::Tensor scores);
void om_flash_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                      torch::Tensor row_ctx, torch::Tensor tiles, torch::Tensor out, int64_t Hq, double scale,
                      torch::Tensor status, c10::optional<torch::Tensor> lse);
void om_dsa_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor bt,
                      torch::Tensor row_seq, torch::Tensor sel, torch::Tensor sel_n, torch::Tensor out, int64_t Hq,
                      double scale);

#include "common/om_host.h"

int64_t om_symm_alloc(int64_t bytes);
void om_symm_free(int64_t ptr);
torch::Tensor om_symm_handle(int64_t ptr);
int64_t om_symm_open(torch::Tensor handle);
void om_symm_close(int64_t ptr);
torch::Tensor om_symm_view(int64_t ptr, int64_t offset, std::vector<int64_t> shape, int64_t dtype_code);
void om_sp_signal(std::vector<int64_t> bases, int64_t rank, torch::Tensor status);
void om_sp_reduce_norm_gather(std::vector<int64_t> bases, int64_t rank, torch::Tensor h, torch::Tensor w,
                              double eps, int64_t p_off, int64_t x_off, torch::Tensor status, bool push,
                              bool signal);
void om_sp_wait(std::vector<int64_t> bases, int64_t rank, torch::Tensor status);
int64_t om_mla_workspace(int64_t rows, int64_t H, int64_t max_ctx);
void om_mla_decode(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables, torch::Tensor row_seq,
                   torch::Tensor row_ctx, torch::Tensor out, torch::Tensor ws, int64_t max_ctx, double scale,
                   torch::Tensor status);

void om_moe_route(torch::Tensor logits, int64_t k, c10::optional<torch::Tensor> forced, torch::Tensor ids,
                  torch::Tensor wts, torch::Tensor counts);
void om_moe_permute(torch::Tensor x, torch::Tensor ids, torch::Tensor counts, torch::Tensor offsets,
                    torch::Tensor cursor, torch::Tensor row_of, torch::Tensor xp);
void om_moe_combine(torch::Tensor yp, torch::Tensor row_of, torch::Tensor wts, torch::Tensor out, bool add);
void om_grouped_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor offsets, torch::Tensor y, torch::Tensor status);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("launch_count", [] { return (int64_t)om::g_launches.load(); }, "kernel launches issued so far");
  m.doc() = "openmini_v1_b200 sm_100a kernels";
  m.def("gemm", &om_gemm, "bf16 tcgen05 GEMM: out = x @ w^T (+ resid)", py::arg("x"), py::arg("w"),
        py::arg("out"), py::arg("resid") = py::none(), py::arg("workspace") = py::none(), py::arg("status"),
        py::arg("force_swap") = -1, py::arg("force_splits") = 0, py::arg("peer") = std::vector<int64_t>{});
  m.def("gemm_plan", &om_gemm_plan);
  m.def("gemm_wq", &om_gemm_wq, "weight-only quantised tcgen05 GEMM (0 = Q4 block-32, 1 = INT8 per row)",
        py::arg("x"), py::arg("qtiles"), py::arg("scales"), py::arg("qtype"), py::arg("out"),
        py::arg("resid") = py::none(), py::arg("workspace") = py::none(), py::arg("status"),
        py::arg("force_swap") = -1, py::arg("force_splits") = 0, py::arg("peer") = std::vector<int64_t>{},
        py::arg("sem") = py::none(), py::arg("agwait") = std::vector<int64_t>{});
  m.def("rmsnorm", &om_rmsnorm, py::arg("x"), py::arg("delta"), py::arg("w"), py::arg("out"), py::arg("eps"));
  m.def("layernorm", &om_layernorm);
  m.def("silu_mul", &om_silu_mul);
  m.def("gelu", &om_gelu);
  m.def("softmax", &om_softmax);
  m.def("embedding", &om_embedding);
  m.def("rope_kv", &om_rope_kv);
  m.def("kv_write", &om_kv_write);
  m.def("paged_attention", &om_paged_attention);
  m.def("paged_attention_tc", &om_paged_attention_tc, "tcgen05 paged decode attention (head_dim 128)");
  m.def("flash_prefill", &om_flash_prefill, "tcgen05 causal FlashAttention prefill over the paged cache",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_tables"), py::arg("row_ctx"),
        py::arg("tiles"), py::arg("out"), py::arg("Hq"), py::arg("scale"), py::arg("status"),
        py::arg("lse") = py::none());
  m.def("paged_attention_workspace", &om_paged_attention_workspace);
  m.def("sample", &om_sample, py::arg("logits"), py::arg("temperature"), py::arg("top_p"), py::arg("top_k"),
        py::arg("rng"), py::arg("out_tok"), py::arg("out_logprob") = py::none(),
        py::arg("keep_mask") = py::none());
  m.def("repetition_penalty", &om_repetition_penalty);
  m.def("decode_advance", &om_decode_advance);
  m.def("quantize_q4", &om_quantize_q4, py::arg("w"), py::arg("q"), py::arg("scales"),
        py::arg("scales_f16") = py::none());
  m.def("dequant_q4", &om_dequant_q4);
  m.def("quantize_int8", &om_quantize_int8);
  m.def("dequant_int8", &om_dequant_int8);
  m.def("gguf_dequant", &om_gguf_dequant, "GGUF Q4_0 / Q8_0 / Q4_K / Q5_K / Q6_K blocks -> bf16 on the device");
  m.def("dsa_scores", &om_dsa_scores, "DSA indexer scores over the paged indexer-key cache");
  m.def("dsa_topk", &om_dsa_topk, "per-row top-k key positions");
  m.def("dsa_head_reduce", &om_dsa_head_reduce, "indexer scores from the tensor-core head GEMM: relu, weights, mask");
  m.def("dsa_attention", &om_dsa_attention, "attention over selected keys of the paged cache");
  m.def("moe_route", &om_moe_route, "router top-k + softmax weights + per-expert counts");
  m.def("moe_permute", &om_moe_permute, "expert offsets and expert-sorted copy of the activations");
  m.def("moe_combine", &om_moe_combine, "weighted sum of the experts' rows back per token");
  m.def("grouped_gemm", &om_grouped_gemm, "grouped tcgen05 GEMM over expert-sorted rows");
  m.def("symm_alloc", &om_symm_alloc, "device buffer for peer mapping (zeroed)");
  m.def("symm_free", &om_symm_free);
  m.def("symm_handle", &om_symm_handle, "CUDA IPC handle bytes of a symm_alloc buffer");
  m.def("symm_open", &om_symm_open, "map a peer's buffer from its IPC handle");
  m.def("symm_close", &om_symm_close);
  m.def("symm_view", &om_symm_view, "tensor view into a buffer (dtype 0 bf16, 1 fp32, 2 int32)");
  m.def("sp_signal", &om_sp_signal, "publish this rank's partials for the next epoch");
  m.def("sp_reduce_norm_gather", &om_sp_reduce_norm_gather,
        "sum peer partials into own residual rows, RMSNorm, push normed rows to every rank",
        py::arg("bases"), py::arg("rank"), py::arg("h"), py::arg("w"), py::arg("eps"), py::arg("p_off"),
        py::arg("x_off"), py::arg("status"), py::arg("push") = false, py::arg("signal") = false);
  m.def("sp_wait", &om_sp_wait, "wait until every rank pushed its normed rows for this epoch");
  m.def("mla_workspace", &om_mla_workspace, "fp32 workspace floats of mla_decode");
  m.def("mla_decode", &om_mla_decode, "latent attention over a paged 576-wide latent cache (absorbed form)");
}
