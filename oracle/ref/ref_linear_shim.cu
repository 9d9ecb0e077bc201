// TEST INFRASTRUCTURE ONLY: a C shim over the reference's own linear-path
// kernels (kernel/csrc/kernel_api.h, compiled from the reference checkout by
// oracle/ref/build_ref.py into oracle/_ref/libref_linear.so).  It lets the
// golden-fixture generator run the unmodified reference kernels on a B200.
// Nothing in the product links or loads this.
#include <stdexcept>
#include <vector>

#include "kernel_api.h"

namespace K = comfyui_turing_utils::kernels;

namespace {
Tensor mk(const void* p, std::vector<int> shape, Tensor::ScalarType t) {
  Tensor r;
  r.ptr = const_cast<void*>(p);
  r.shape.dataExtent = shape;
  r.scalarType = t;
  r.dev = Device{Device::CUDA, 0};
  return r;
}

template <typename F>
int run(void* stream, F&& f) {
  stackCUDAStreams.push_back(static_cast<cudaStream_t>(stream));
  int rc = 0;
  try {
    f();
  } catch (const std::exception&) {
    rc = 1;
  }
  stackCUDAStreams.pop_back();
  return rc;
}
}  // namespace

extern "C" {

int ref_bf16_convrot(const void* in, int rows, int hidden, int swiglu, int gelu, int int4,
                     int8_t* out, float* scales, void* stream) {
  return run(stream, [&] {
    Tensor x = mk(in, {rows, swiglu ? 2 * hidden : hidden}, Tensor::BF16);
    Tensor o = mk(out, {rows, int4 ? hidden / 2 : hidden}, Tensor::INT8);
    Tensor s = mk(scales, {rows, 1}, Tensor::FP32);
    if (gelu) {
      if (int4) K::turing_bf16_gelu_int4_convrot_quantize(x, o, s, 512);
      else K::turing_bf16_gelu_int8_convrot_quantize(x, o, s, 512);
    } else {
      if (int4) K::turing_bf16_int4_convrot_quantize(x, o, s, swiglu != 0, 512);
      else K::turing_bf16_int8_convrot_quantize(x, o, s, swiglu != 0, 512);
    }
  });
}

int ref_staged_convrot(const void* in, int fp16, int rows, int hidden, int gelu, int int4,
                       void* rotated, float* partial, int8_t* out, float* scales, void* stream) {
  return run(stream, [&] {
    const Tensor::ScalarType t = fp16 ? Tensor::FP16 : Tensor::BF16;
    Tensor x = mk(in, {rows, gelu ? hidden : 2 * hidden}, t);
    Tensor r = mk(rotated, {rows, hidden}, t);
    Tensor pa = mk(partial, {rows, hidden / 256}, Tensor::FP32);
    Tensor o = mk(out, {rows, int4 ? hidden / 2 : hidden}, Tensor::INT8);
    Tensor s = mk(scales, {rows, 1}, Tensor::FP32);
    if (gelu) {
      if (int4) K::turing_gelu_int4_convrot_quantize(x, r, pa, o, s);
      else K::turing_gelu_int8_convrot_quantize(x, r, pa, o, s);
    } else {
      if (int4) K::turing_swiglu_int4_convrot_quantize(x, r, pa, o, s);
      else K::turing_swiglu_int8_convrot_quantize(x, r, pa, o, s);
    }
  });
}

int ref_int8_linear(const int8_t* a, const int8_t* w, const float* a_s, const float* w_s,
                    const float* bias, void* out, int m, int n, int k, void* stream) {
  return run(stream, [&] {
    K::turing_int8_linear(mk(a, {m, k}, Tensor::INT8), mk(w, {n, k}, Tensor::INT8),
                          mk(a_s, {m}, Tensor::FP32), mk(w_s, {n}, Tensor::FP32),
                          bias ? mk(bias, {n}, Tensor::FP32) : Tensor{},
                          mk(out, {m, n}, Tensor::BF16), 0);
  });
}

int ref_w4a8_linear(const int8_t* a, const int8_t* w_packed, const float* a_s, const float* w_s,
                    const float* bias, void* out, int m, int n, int k, void* stream) {
  return run(stream, [&] {
    K::turing_w4a8_linear(mk(a, {m, k}, Tensor::INT8), mk(w_packed, {n, k / 2}, Tensor::INT8),
                          mk(a_s, {m}, Tensor::FP32), mk(w_s, {n}, Tensor::FP32),
                          bias ? mk(bias, {n}, Tensor::FP32) : Tensor{},
                          mk(out, {m, n}, Tensor::BF16), 0);
  });
}

int ref_codebook_linear(const int8_t* a, const int8_t* w_packed, const float* a_s,
                        const uint8_t* gs, const float* c_s, const float* codebook,
                        const float* bias, int8_t* workspace, int chunk_rows, void* out, int m,
                        int n, int k, int group_size, void* stream) {
  return run(stream, [&] {
    K::turing_codebook_w4a8_linear(
        mk(a, {m, k}, Tensor::INT8), mk(w_packed, {n, k / 2}, Tensor::INT8),
        mk(a_s, {m}, Tensor::FP32), mk(gs, {n, k / group_size}, Tensor::INT8),
        mk(c_s, {n}, Tensor::FP32), mk(codebook, {16}, Tensor::FP32),
        bias ? mk(bias, {n}, Tensor::FP32) : Tensor{},
        mk(workspace, {chunk_rows, k}, Tensor::INT8), mk(out, {m, n}, Tensor::BF16), group_size,
        false, 0);
  });
}

int ref_dequant(const int32_t* acc, const float* a_s, const float* w_s, int w_numel, void* out,
                int rows, int cols, void* stream) {
  return run(stream, [&] {
    K::turing_dequantize_int8_bf16(mk(acc, {rows, cols}, Tensor::INT32),
                                   mk(a_s, {rows}, Tensor::FP32), mk(w_s, {w_numel}, Tensor::FP32),
                                   mk(out, {rows, cols}, Tensor::BF16));
  });
}

// dtype: 0 bf16, 1 f16, 2 f32.
static Tensor::ScalarType float_type(int dtype) {
  return dtype == 0 ? Tensor::BF16 : dtype == 1 ? Tensor::FP16 : Tensor::FP32;
}

int ref_segmented_rms_adaln(const void* x, const void* w, const void* scale, const void* shift,
                            const int* segments, void* out, int rows, int hidden, int mod_rows,
                            int n_seg, int dtype, float eps, void* stream) {
  return run(stream, [&] {
    const auto t = float_type(dtype);
    K::turing_segmented_rms_adaln(mk(x, {rows, hidden}, t), mk(w, {hidden}, t),
                                  mk(scale, {mod_rows, hidden}, t), mk(shift, {mod_rows, hidden}, t),
                                  mk(segments, {n_seg, 3}, Tensor::INT32),
                                  mk(out, {rows, hidden}, t), eps);
  });
}

int ref_layer_norm_adaln(const void* x, const void* scale, const void* shift, void* out,
                         int batch, int seq, int hidden, int steps, int dtype, float eps,
                         void* stream) {
  return run(stream, [&] {
    const auto t = float_type(dtype);
    K::turing_layer_norm_adaln(mk(x, {batch, seq, hidden}, t), mk(scale, {batch, steps, hidden}, t),
                               mk(shift, {batch, steps, hidden}, t),
                               mk(out, {batch, seq, hidden}, t), eps);
  });
}

}  // extern "C"
