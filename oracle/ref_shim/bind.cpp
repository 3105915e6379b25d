// Test infrastructure only: pybind11 module exposing the reference's own
// fa_kla_attention_cpu (ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:36-170),
// compiled from the reference source file where it lies. The reference's
// binding files (backend/cpp/main.cpp, fa_kla_bindings.cpp) are empty, so the
// reference exports nothing by itself; this is the binding it lacks.
#include <torch/extension.h>

torch::Tensor fa_kla_attention_cpu(const torch::Tensor& q_mapped,
                                   const torch::Tensor& k_mapped,
                                   const torch::Tensor& v_reshaped,
                                   const torch::Tensor& temp);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fa_kla_attention_cpu", &fa_kla_attention_cpu,
        "reference FA-KLA CPU kernel (q_mapped, k_mapped, v, temp) -> out");
}
