// Python binding for the reference's SelectiveAdam CUDA kernel -- test
// infrastructure only. oracle/build_ref.py compiles this file together with
// the reference's submodules/clm_kernels/adam.cu (left where it lies in the
// reference tree) into oracle/_ref/. The declaration below matches the
// reference header submodules/clm_kernels/adam.h.
#include <torch/extension.h>

void selective_adam_update(torch::Tensor& param, torch::Tensor& param_grad,
                           torch::Tensor& exp_avg, torch::Tensor& exp_avg_sq,
                           torch::Tensor& tiles_touched, const float lr, const float b1,
                           const float b2, const float eps, const uint32_t N, const uint32_t M);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("selective_adam_update", &selective_adam_update);
}
