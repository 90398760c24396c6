// Python binding of the reference's gsplat 1.0.0 kernels -- TEST
// INFRASTRUCTURE ONLY. oracle/build_ref.py compiles the vendored CUDA sources
// (submodules/gsplat/gsplat/cuda/csrc of the reference tree, read in place)
// with this file into oracle/_ref/gsplat/gsplat_ref*.so, so that the GPU
// parity tests can run the reference projection, SH colors, tile
// intersection and rasterization beside tidegs_b200's. Only the functions
// the engine's render path uses are bound
// (strategies/tide_engine/engine.py:481-561).
#include <torch/extension.h>

#include "bindings.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fully_fused_projection_fwd", &fully_fused_projection_fwd_tensor);
  m.def("fully_fused_projection_bwd", &fully_fused_projection_bwd_tensor);
  m.def("isect_tiles", &isect_tiles_tensor);
  m.def("isect_offset_encode", &isect_offset_encode_tensor);
  m.def("rasterize_to_pixels_fwd", &rasterize_to_pixels_fwd_tensor);
  m.def("rasterize_to_pixels_bwd", &rasterize_to_pixels_bwd_tensor);
  m.def("compute_sh_fwd", &compute_sh_fwd_tensor);
  m.def("compute_sh_bwd", &compute_sh_bwd_tensor);
}
