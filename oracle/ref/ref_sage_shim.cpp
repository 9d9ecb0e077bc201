// TEST INFRASTRUCTURE ONLY: pybind shim exposing the reference's own Sage
// quantizers, the Sage attention and the dense W8A8 attention
// (kernel/csrc/turing/sage/fused.h, attn_cuda_sm75.h),
// compiled from the reference checkout by oracle/ref/build_ref.py into
// oracle/_ref/.  Used to generate golden fixtures on a B200.
#include <torch/extension.h>

#include "attn_cuda_sm75.h"
#include "fused.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("quant_per_block_int8_cuda",
        py::overload_cast<at::Tensor, at::Tensor, at::Tensor, int, int>(&quant_per_block_int8_cuda));
  m.def("quant_per_warp_int8_cuda",
        py::overload_cast<at::Tensor, at::Tensor, at::Tensor, int, int, int>(&quant_per_warp_int8_cuda));
  m.def("quant_qk_rms_rope_int8_cuda", &quant_qk_rms_rope_int8_cuda);
  m.def("qk_int8_sv_f16_accum_f32_attn", &qk_int8_sv_f16_accum_f32_attn);
  m.def("quant_qk_per_warp_int8_rotated_cuda", &quant_qk_per_warp_int8_rotated_cuda);
  m.def("quant_qk_per_warp_int8_rotated_anchored_cuda",
        &quant_qk_per_warp_int8_rotated_anchored_cuda);
  m.def("quantize_v_int8_sm75", &quantize_v_int8_sm75);
  m.def("sol_sparse_online_w8a8_prequantized_attn", &sol_sparse_online_w8a8_prequantized_attn);
}
