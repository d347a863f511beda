// pybind11 binding of one reference launcher, compiled together with the
// reference's own .cu source by oracle/build_ref.py. REF_FN names the launcher:
// llm_fa_forward (llm_fa.cu:1418-1475), redist_v6_forward (scaffolding.cu:793)
// or fa4_faux_attn_forward (faux.cu:951); each takes (Q, K, V) and returns
// [O, ...]. Baseline infrastructure only.
#include <torch/extension.h>

#include <vector>

#ifndef REF_FN
#define REF_FN llm_fa_forward
#endif
#define REF_STR2(x) #x
#define REF_STR(x) REF_STR2(x)

std::vector<torch::Tensor> REF_FN(torch::Tensor Q, torch::Tensor K, torch::Tensor V);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def(REF_STR(REF_FN), &REF_FN, "reference launcher (Q, K, V) -> [O, ...]");
}
