// pybind11 binding of the reference launcher `llm_fa_forward`
// (llm_fa.cu:1418-1475), compiled together with the reference's own
// llm_fa.cu by oracle/build_ref.py. Baseline infrastructure only.
#include <torch/extension.h>

#include <vector>

std::vector<torch::Tensor> llm_fa_forward(torch::Tensor Q, torch::Tensor K, torch::Tensor V);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("llm_fa_forward", &llm_fa_forward, "reference llm_fa forward (Q, K, V) -> [O, prof, count]");
}
