// Host-side plumbing shared by the translation units of libturing_b200:
// argument checks that become C-ABI error codes, CUDA error checks, device
// properties and TMA descriptor encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "../../include/turing_b200.h"
#include "tb_common.cuh"

namespace tb {

// An argument/shape error (maps to TB_ERR_INVALID) or a CUDA error
// (TB_ERR_CUDA).  The message is what the reference raises for the same
// condition where one exists.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void throw_invalid(const char* msg);
[[noreturn]] void throw_cuda(cudaError_t e, const char* file, int line);

#define TB_REQUIRE(cond, msg)          \
  do {                                 \
    if (!(cond)) ::tb::throw_invalid(msg); \
  } while (0)

#define TB_CUDA_CHECK(expr)                                   \
  do {                                                        \
    cudaError_t tb_e_ = (expr);                               \
    if (tb_e_ != cudaSuccess) ::tb::throw_cuda(tb_e_, __FILE__, __LINE__); \
  } while (0)

void set_last_error(const char* msg);

// Runs `body` and converts exceptions into a status code + thread-local message.
template <typename F>
int guarded(F&& body) {
  try {
    set_last_error("");
    body();
    return TB_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return TB_ERR_INTERNAL;
  }
}

// Registry of per-translation-unit watchdog readers (see tb_tu.cuh).
void register_device_error_reader(int (*reader)());

// Raises TB_ERR_UNSUPPORTED unless the current device is sm_100.
void require_sm100();

int device_sm_count();
int device_cc_major();
size_t device_smem_optin();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// dims/strides innermost first; strides in bytes for dims 1..rank-1.
void encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                       const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                       CUtensorMapSwizzle swizzle);

// Attention launch arguments (sage_attn.cu).  v_scale == null: Sage (16-bit
// V of the output dtype); else W8A8-PV (fp16 V codes, [B, Hk, D] scales).
struct AttnArgs {
  const int8_t* q;
  const int8_t* k;
  const void* v;
  int v_dtype;
  void* out;
  int out_dtype;
  const float* q_scale;
  const float* k_scale;
  float* lse;
  int64_t B, Hq, Hk, Lq, Lk, D;
  int64_t q_sb, q_sh, q_sl, k_sb, k_sh, k_sl, v_sb, v_sh, v_sl, o_sb, o_sh, o_sl;
  int64_t q_tiles_scale, k_tiles_scale;
  int causal;
  float sm_scale;
  const float* v_scale;
};

// Kernels implemented in the other translation units.
void sage_attn_launch(const AttnArgs& a, cudaStream_t stream);
void rot_quant_launch(const void* q, const void* k, int8_t* q_out, int8_t* k_out, float* q_scale,
                      float* k_scale, int32_t* anchors, float* anchor_values, int64_t B,
                      int64_t Hq, int64_t Hk, int64_t Lq, int64_t Lk, int64_t D,
                      const int64_t* strides, int anchor_mode, int nan_code, int dtype,
                      cudaStream_t stream);
void qk_anchor_launch(const void* key, const void* key_norm, const void* freqs,
                      const float* key_rrms, int32_t* anchors, float* anchor_values, int64_t B,
                      int64_t Hk, int64_t Lk, int64_t D, const int64_t* k_strides,
                      const int64_t* freq_strides, int64_t freq_batches, int64_t freq_sequence,
                      int64_t rot_dim, int norm_scope, int split_half, int dtype, float eps,
                      cudaStream_t stream);
void v_quant_launch(const void* v, int dtype, uint16_t* codes_f16, int8_t* codes_cm, float* scale,
                    int64_t B, int64_t H, int64_t L, int64_t D, int64_t Lpad, int64_t sb,
                    int64_t sh, int64_t sl, cudaStream_t stream);
void convrot_check_pointers(const void* input, const void* out, const float* scales, int staged,
                            const void* rotated, const float* partial);
void convrot_quantize_impl(const void* input, int dtype, int64_t rows, int64_t k, int act,
                           int int4, int staged, void* rotated, float* partial, int8_t* out,
                           float* scales, cudaStream_t stream);

}  // namespace tb
