// Python bindings of the sm_100a kernels (module gollek_b200_C).
#include <torch/extension.h>

void rms_norm_out(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps);
void fused_add_rms_norm_out(torch::Tensor out, torch::Tensor x, torch::Tensor residual, torch::Tensor w, double eps);
void rope_kv_write_out(torch::Tensor q_out, torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                       c10::optional<torch::Tensor> cache, c10::optional<torch::Tensor> slots, int64_t H, int64_t Hk,
                       int64_t D);
void embedding_out(torch::Tensor out, torch::Tensor ids, torch::Tensor table);
void silu_mul_out(torch::Tensor out, torch::Tensor x);
void paged_decode_attention_out(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables,
                                torch::Tensor seq_lens, double scale, int64_t num_splits,
                                c10::optional<torch::Tensor> workspace);
void paged_prefill_attention_out(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables,
                                 torch::Tensor seq_lens, torch::Tensor query_start, torch::Tensor tiles, double scale);
void gemm_bf16_out(torch::Tensor out, torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> residual,
                   int64_t epi, int64_t bn, c10::optional<torch::Tensor> status, int64_t grid_limit);
void argmax_out(torch::Tensor out, torch::Tensor logits);
void apply_penalties_(torch::Tensor logits, torch::Tensor triples, torch::Tensor rep, torch::Tensor freq,
                      torch::Tensor pres);
void sample_out(torch::Tensor out, torch::Tensor logits, torch::Tensor temps, torch::Tensor top_ks,
                torch::Tensor top_ps, torch::Tensor min_ps, torch::Tensor seeds, torch::Tensor offsets);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "gollek_b200 sm_100a kernels";
  m.def("rms_norm", &rms_norm_out, "RMSNorm (K1)");
  m.def("fused_add_rms_norm", &fused_add_rms_norm_out, "residual add + RMSNorm (K1)");
  m.def("rope_kv_write", &rope_kv_write_out, "QKV split + RoPE + paged KV write (K2)");
  m.def("embedding", &embedding_out, "embedding gather (K13)");
  m.def("silu_mul", &silu_mul_out, "SwiGLU activation");
  m.def("paged_decode_attention", &paged_decode_attention_out, "paged decode attention (K3)");
  m.def("paged_prefill_attention", &paged_prefill_attention_out, "paged prefill attention (K4)");
  m.def("gemm_bf16", &gemm_bf16_out, "tcgen05 bf16 GEMM with fused epilogues (K5/K8)");
  m.def("argmax", &argmax_out, "greedy argmax (K11)");
  m.def("apply_penalties", &apply_penalties_, "repetition/frequency/presence penalties (K11)");
  m.def("sample", &sample_out, "top-k/min-p/top-p sampling (K11)");
}
