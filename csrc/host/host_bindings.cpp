// Python bindings of the host C++ runtime (module gollek_b200_host).
#include <torch/extension.h>

torch::Tensor quantize_q8_0(torch::Tensor x);
torch::Tensor dequantize_q8_0(torch::Tensor raw, int64_t n);
torch::Tensor quantize_q4_k(torch::Tensor x);
torch::Tensor dequantize_q4_k(torch::Tensor raw, int64_t n);
torch::Tensor gguf_dequantize(torch::Tensor raw, int64_t type, int64_t n);
torch::Tensor gguf_quantize(torch::Tensor x, int64_t type);
void register_block_allocator(pybind11::module& m);
void register_forelen(pybind11::module& m);
void register_spec(pybind11::module& m);
void register_grammar(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "gollek_b200 host runtime";
  m.def("quantize_q8_0", &quantize_q8_0);
  m.def("dequantize_q8_0", &dequantize_q8_0);
  m.def("quantize_q4_k", &quantize_q4_k);
  m.def("dequantize_q4_k", &dequantize_q4_k);
  m.def("gguf_dequantize", &gguf_dequantize,
        "dequantize Q4_0/Q4_1/Q5_0/Q5_1/Q2_K/Q3_K/Q5_K/Q6_K blocks (ggml type id) to fp32");
  m.def("gguf_quantize", &gguf_quantize, "quantize fp32 into Q4_0/Q4_1/Q5_0/Q5_1/Q2_K/Q3_K/Q5_K/Q6_K blocks");
  register_block_allocator(m);
  register_forelen(m);
  register_spec(m);
  register_grammar(m);
}
