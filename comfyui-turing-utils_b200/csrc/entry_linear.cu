// C entry points of the linear path (GEMMs, dequant epilogue, codebook W4A8)
// and of the Sage quantizers.  Checks follow the reference binding
// (kernel/csrc/bindings.cpp:371-467, 262-369; sage/fused.cu:983-1150).
#include "tb_capi_internal.h"

namespace tb {
void gemm_i8_launch(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                    const float* a_scale, const float* w_scale, const float* bias, void* out,
                    int64_t ldo, int epi, cudaStream_t stream);
void dequant_launch(const int32_t* acc, int64_t acc_stride, const float* a_s, const float* w_s,
                    bool scalar_w, void* out, int rows, int cols, cudaStream_t stream);
void codebook_decode_launch(const int8_t* packed, const uint8_t* group_scale,
                            const float* codebook, int8_t* out, int rows, int k, int group_size,
                            cudaStream_t stream);
void unpack_s4_launch(const int8_t* packed, int8_t* out, int64_t rows, int64_t k,
                      cudaStream_t stream);
void gated_residual_launch(void* x, int64_t x_stride, const void* y, int64_t y_stride,
                           const void* gate, int64_t rows, int64_t cols, cudaStream_t stream);
void sage_quant_launch(const void* input, int dtype, int8_t* out, float* scale, int64_t B,
                       int64_t H, int64_t L, int64_t D, int64_t sb, int64_t sh, int64_t sl,
                       int tile, int64_t num_tiles, int layout, const void* mean,
                       cudaStream_t stream);
void token_mean_launch(const void* input, int dtype, void* mean, int64_t B, int64_t H, int64_t L,
                       int64_t D, int64_t sb, int64_t sh, int64_t sl, int layout,
                       cudaStream_t stream);
}  // namespace tb

using tb::guarded;

extern "C" {

int tb_int8_linear(const int8_t* activation, const int8_t* weight, const float* activation_scale,
                   const float* weight_scale, const float* bias, void* output, int64_t m,
                   int64_t n, int64_t k, int64_t ldo, int tile_policy, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(activation && weight && activation_scale && weight_scale && output,
               "Turing INT8 linear tensors must be CUDA tensors");
    TB_REQUIRE(tile_policy >= 0 && tile_policy <= 5, "invalid Turing INT8 tile policy");
    if (m == 0 || n == 0 || k == 0) return;
    TB_REQUIRE(k % 16 == 0 && n % 8 == 0, "Turing INT8 linear requires K%16=0 and N%8=0");
    tb::require_sm100();
    tb::gemm_i8_launch(activation, weight, m, n, k, activation_scale, weight_scale, bias, output,
                       ldo, 0, static_cast<cudaStream_t>(stream));
  });
}

int tb_int8_gemm_s32(const int8_t* activation, const int8_t* weight, int32_t* accumulator,
                     int64_t m, int64_t n, int64_t k, int64_t acc_stride, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(activation && weight && accumulator, "INT8 GEMM tensors must be CUDA tensors");
    if (m == 0 || n == 0 || k == 0) return;
    TB_REQUIRE(k % 16 == 0 && n % 4 == 0, "INT8 GEMM requires K%16=0 and N%4=0");
    tb::require_sm100();
    tb::gemm_i8_launch(activation, weight, m, n, k, nullptr, nullptr, nullptr, accumulator,
                       acc_stride, 1, static_cast<cudaStream_t>(stream));
  });
}

int tb_dequantize_int8_bf16(const int32_t* accumulator, int64_t acc_stride,
                            const float* activation_scale, const float* weight_scale,
                            int64_t weight_scale_numel, void* output, int64_t rows, int64_t cols,
                            tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(accumulator && activation_scale && weight_scale && output,
               "accumulator and scales must be CUDA tensors");
    TB_REQUIRE(rows > 0 && cols > 0, "INT8 BF16 epilogue dimensions must be positive");
    TB_REQUIRE(acc_stride >= cols, "output_columns must be positive and no larger than the accumulator width");
    TB_REQUIRE(weight_scale_numel == 1 || weight_scale_numel == cols,
               "weight_scale must be scalar or contain one value per output column");
    TB_REQUIRE(rows <= INT32_MAX && cols <= INT32_MAX && acc_stride <= INT32_MAX,
               "INT8 BF16 epilogue dimensions exceed the CUDA kernel range");
    tb::require_sm100();
    tb::dequant_launch(accumulator, acc_stride, activation_scale, weight_scale,
                       weight_scale_numel == 1, output, static_cast<int>(rows),
                       static_cast<int>(cols), static_cast<cudaStream_t>(stream));
  });
}

int tb_gated_residual_add(void* x, int64_t x_stride, const void* y, int64_t y_stride,
                          const void* gate, int64_t rows, int64_t cols, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(x && y, "gated residual add: x and y must be CUDA tensors");
    TB_REQUIRE(rows >= 0 && cols >= 0 && x_stride >= cols && y_stride >= cols,
               "gated residual add: invalid shape or strides");
    if (rows == 0 || cols == 0) return;
    tb::require_sm100();
    tb::gated_residual_launch(x, x_stride, y, y_stride, gate, rows, cols,
                              static_cast<cudaStream_t>(stream));
  });
}

int tb_codebook_w4a8_linear(const int8_t* activation, const int8_t* weight_packed,
                            const float* activation_scale, const uint8_t* group_scale,
                            const float* channel_scale, const float* codebook, const float* bias,
                            int8_t* workspace, int64_t workspace_rows, void* output, int64_t m,
                            int64_t n, int64_t k, int64_t group_size, int inline_decode,
                            int tile_policy, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(activation && weight_packed && activation_scale && group_scale && channel_scale &&
                   codebook && output,
               "all codebook W4A8 tensors must use the same CUDA device");
    if (m == 0 || n == 0 || k == 0) return;
    TB_REQUIRE(k % 16 == 0 && n % 8 == 0 &&
                   (inline_decode || (workspace != nullptr && workspace_rows > 0 &&
                                      workspace_rows % 8 == 0)),
               "Turing codebook W4A8 requires K%16=0, N%8=0, and an 8-row-aligned staged workspace");
    TB_REQUIRE(group_size >= 4 && k % group_size == 0 &&
                   (16 % group_size == 0 || group_size % 16 == 0),
               "unsupported Turing codebook W4A8 group size");
    TB_REQUIRE(tile_policy >= 0 && tile_policy <= 5, "invalid Turing codebook W4A8 tile policy");
    TB_REQUIRE(!inline_decode || workspace != nullptr,
               "the sm_100a codebook W4A8 decodes through the staged workspace; pass one");
    TB_REQUIRE(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX,
               "codebook W4A8 dimensions exceed the CUDA kernel range");
    tb::require_sm100();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t packed_k = k / 2;
    const int64_t gpr = k / group_size;
    // Decode a chunk of weight rows into the workspace, then contract it into
    // the matching output columns (w4a8.cu:1157-1182).
    for (int64_t row = 0; row < n; row += workspace_rows) {
      const int64_t rows = (n - row) < workspace_rows ? (n - row) : workspace_rows;
      tb::codebook_decode_launch(weight_packed + row * packed_k, group_scale + row * gpr,
                                 codebook, workspace, static_cast<int>(rows),
                                 static_cast<int>(k), static_cast<int>(group_size), s);
      tb::gemm_i8_launch(activation, workspace, m, rows, k, activation_scale,
                         channel_scale + row, bias ? bias + row : nullptr,
                         static_cast<__nv_bfloat16*>(output) + row, n, 0, s);
    }
  });
}

int tb_w4a8_linear(const int8_t* activation, const int8_t* weight_packed,
                   const float* activation_scale, const float* weight_scale, const float* bias,
                   int8_t* workspace, int64_t workspace_rows, void* output, int64_t m, int64_t n,
                   int64_t k, int64_t ldo, int tile_policy, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(activation && weight_packed && activation_scale && weight_scale && output,
               "Turing W4A8 tensors must be CUDA tensors");
    TB_REQUIRE(tile_policy >= 0 && tile_policy <= 5, "invalid Turing W4A8 tile policy");
    if (m == 0 || n == 0 || k == 0) return;
    TB_REQUIRE(k % 16 == 0 && n % 8 == 0, "Turing W4A8 linear requires K%16=0 and N%8=0");
    TB_REQUIRE(workspace != nullptr && workspace_rows > 0 && workspace_rows % 8 == 0,
               "Turing W4A8 linear needs an 8-row-aligned int8 weight workspace");
    TB_REQUIRE(ldo >= n, "output row stride must cover N columns");
    tb::require_sm100();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Unpack a chunk of weight rows to int8 in the workspace, then contract it
    // into the matching output columns.
    for (int64_t row = 0; row < n; row += workspace_rows) {
      const int64_t rows = (n - row) < workspace_rows ? (n - row) : workspace_rows;
      tb::unpack_s4_launch(weight_packed + row * (k / 2), workspace, rows, k, s);
      tb::gemm_i8_launch(activation, workspace, m, rows, k, activation_scale, weight_scale + row,
                         bias ? bias + row : nullptr, static_cast<__nv_bfloat16*>(output) + row,
                         ldo, 0, s);
    }
  });
}

int tb_int4_linear(const int8_t* activation_packed, const int8_t* weight_packed,
                   const float* activation_scale, const float* weight_scale, const float* bias,
                   int8_t* activation_workspace, int8_t* weight_workspace,
                   int64_t workspace_rows, void* output, int64_t m, int64_t n, int64_t k,
                   int64_t ldo, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(activation_packed && weight_packed && activation_scale && weight_scale && output,
               "Turing W4A4 tensors must be CUDA tensors");
    if (m == 0 || n == 0 || k == 0) return;
    TB_REQUIRE(k % 16 == 0 && n % 8 == 0, "Turing W4A4 linear requires K%16=0 and N%8=0");
    TB_REQUIRE(activation_workspace != nullptr,
               "Turing W4A4 linear needs an int8 [M, K] activation workspace");
    TB_REQUIRE(weight_workspace != nullptr && workspace_rows > 0 && workspace_rows % 8 == 0,
               "Turing W4A4 linear needs an 8-row-aligned int8 weight workspace");
    TB_REQUIRE(ldo >= n, "output row stride must cover N columns");
    tb::require_sm100();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    tb::unpack_s4_launch(activation_packed, activation_workspace, m, k, s);
    for (int64_t row = 0; row < n; row += workspace_rows) {
      const int64_t rows = (n - row) < workspace_rows ? (n - row) : workspace_rows;
      tb::unpack_s4_launch(weight_packed + row * (k / 2), weight_workspace, rows, k, s);
      tb::gemm_i8_launch(activation_workspace, weight_workspace, m, rows, k, activation_scale,
                         weight_scale + row, bias ? bias + row : nullptr,
                         static_cast<__nv_bfloat16*>(output) + row, ldo, 0, s);
    }
  });
}

static void check_layout_dims(int layout) {
  TB_REQUIRE(layout == TB_LAYOUT_NHD || layout == TB_LAYOUT_HND, "tensor_layout must be 0 or 1");
}

int tb_quant_per_block_int8(const void* input, int dtype, int8_t* output, float* scale, int64_t B,
                            int64_t H, int64_t L, int64_t D, int64_t stride_b, int64_t stride_h,
                            int64_t stride_l, int block_size, int layout, const void* mean,
                            tb_stream_t stream) {
  return guarded([&] {
    check_layout_dims(layout);
    TB_REQUIRE(block_size == 16 || block_size == 32 || block_size == 64 || block_size == 128,
               "block_size must be 16, 32, 64 or 128");
    tb::require_sm100();
    tb::sage_quant_launch(input, dtype, output, scale, B, H, L, D, stride_b, stride_h, stride_l,
                          block_size, (L + block_size - 1) / block_size, layout, mean,
                          static_cast<cudaStream_t>(stream));
  });
}

int tb_quant_per_warp_int8(const void* input, int dtype, int8_t* output, float* scale, int64_t B,
                           int64_t H, int64_t L, int64_t D, int64_t stride_b, int64_t stride_h,
                           int64_t stride_l, int block_size, int warp_block_size, int layout,
                           tb_stream_t stream) {
  return guarded([&] {
    check_layout_dims(layout);
    TB_REQUIRE(block_size == 64 || block_size == 128, "block_size must be 64 or 128");
    TB_REQUIRE(warp_block_size == 16 || warp_block_size == 32 || warp_block_size == 64,
               "warp_block_size must be 16, 32 or 64");
    TB_REQUIRE(block_size % warp_block_size == 0, "block_size must be a multiple of warp_block_size");
    tb::require_sm100();
    // Scale index block * (block/warp) + warp equals the warp tile index; the
    // scale shape [B, H, ceil(L/block) * (block/warp)] pads to whole blocks.
    const int64_t tiles = (L + block_size - 1) / block_size * (block_size / warp_block_size);
    tb::sage_quant_launch(input, dtype, output, scale, B, H, L, D, stride_b, stride_h, stride_l,
                          warp_block_size, tiles, layout, nullptr,
                          static_cast<cudaStream_t>(stream));
  });
}

int tb_token_mean(const void* input, int dtype, void* mean, int64_t B, int64_t H, int64_t L,
                  int64_t D, int64_t stride_b, int64_t stride_h, int64_t stride_l, int layout,
                  tb_stream_t stream) {
  return guarded([&] {
    check_layout_dims(layout);
    tb::require_sm100();
    tb::token_mean_launch(input, dtype, mean, B, H, L, D, stride_b, stride_h, stride_l, layout,
                          static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"

// ------------------------------------------------------------ attention ----

extern "C" int tb_qk_int8_sv_f16_accum_f32_attn(
    const int8_t* q, const int8_t* k, const void* v, int v_dtype, void* out, int out_dtype,
    const float* q_scale, const float* k_scale, float* lse, int64_t B, int64_t Hq, int64_t Hk,
    int64_t Lq, int64_t Lk, int64_t D, const int64_t* strides, int layout, int is_causal,
    int qk_quant_gran, float sm_scale, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(q && k && v && out && q_scale && k_scale && strides,
               "query, key, value, output and scales must be CUDA tensors");
    TB_REQUIRE(layout == TB_LAYOUT_NHD || layout == TB_LAYOUT_HND, "tensor_layout must be 0 or 1");
    TB_REQUIRE(qk_quant_gran == 2, "production Turing Sage requires per-warp Q/K quantization");
    TB_REQUIRE(B > 0 && Hq > 0 && Hk > 0 && Lq > 0 && Lk > 0, "empty Q/K sequences are not supported");
    TB_REQUIRE(Hq % Hk == 0, "num_qo_heads must be divisible by num_kv_heads");
    TB_REQUIRE(Lq <= INT32_MAX && Lk <= INT32_MAX, "sequence length exceeds the kernel range");
    tb::require_sm100();
    tb::AttnArgs a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.v_dtype = v_dtype;
    a.out = out;
    a.out_dtype = out_dtype;
    a.q_scale = q_scale;
    a.k_scale = k_scale;
    a.lse = lse;
    a.B = B;
    a.Hq = Hq;
    a.Hk = Hk;
    a.Lq = Lq;
    a.Lk = Lk;
    a.D = D;
    // strides: q (b, h, l), k (b, h, l), v (b, h, l), o (b, h, l), in elements.
    a.q_sb = strides[0]; a.q_sh = strides[1]; a.q_sl = strides[2];
    a.k_sb = strides[3]; a.k_sh = strides[4]; a.k_sl = strides[5];
    a.v_sb = strides[6]; a.v_sh = strides[7]; a.v_sl = strides[8];
    a.o_sb = strides[9]; a.o_sh = strides[10]; a.o_sl = strides[11];
    a.q_tiles_scale = (Lq + 63) / 64 * 4;
    a.k_tiles_scale = (Lk + 63) / 64;
    a.causal = is_causal;
    a.sm_scale = sm_scale;
    tb::sage_attn_launch(a, static_cast<cudaStream_t>(stream));
  });
}

// ------------------------------------------------------ W8A8-PV attention ----

extern "C" int tb_quant_qk_int8_rotated(const void* query, const void* key, int8_t* query_out,
                                        int8_t* key_out, float* query_scale, float* key_scale,
                                        int32_t* anchors, float* anchor_values, int64_t batch,
                                        int64_t query_heads, int64_t key_heads,
                                        int64_t query_length, int64_t key_length,
                                        int64_t head_dim, const int64_t* strides, int anchor_mode,
                                        int nan_code, int dtype, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(query && key && strides, "query and key must be CUDA tensors");
    tb::require_sm100();
    tb::rot_quant_launch(query, key, query_out, key_out, query_scale, key_scale, anchors,
                         anchor_values, batch, query_heads, key_heads, query_length, key_length,
                         head_dim, strides, anchor_mode, nan_code, dtype,
                         static_cast<cudaStream_t>(stream));
  });
}

extern "C" int tb_qk_anchor_processed(const void* key, const void* key_norm, const void* freqs,
                                      const float* key_rrms, int32_t* anchors,
                                      float* anchor_values, int64_t batch, int64_t key_heads,
                                      int64_t key_length, int64_t head_dim,
                                      const int64_t* key_strides, const int64_t* freq_strides,
                                      int64_t freq_batches, int64_t freq_sequence,
                                      int64_t rot_dim, int norm_scope, int split_half, int dtype,
                                      float epsilon, tb_stream_t stream) {
  return guarded([&] {
    tb::require_sm100();
    tb::qk_anchor_launch(key, key_norm, freqs, key_rrms, anchors, anchor_values, batch, key_heads,
                         key_length, head_dim, key_strides, freq_strides, freq_batches,
                         freq_sequence, rot_dim, norm_scope, split_half, dtype, epsilon,
                         static_cast<cudaStream_t>(stream));
  });
}

extern "C" int tb_quantize_v_int8(const void* value, int dtype, void* codes_f16,
                                  int8_t* codes_channel_major, float* scale, int64_t batch,
                                  int64_t heads, int64_t length, int64_t head_dim,
                                  int64_t padded_length, const int64_t* strides,
                                  tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(value && strides, "value must be a CUDA tensor");
    tb::require_sm100();
    tb::v_quant_launch(value, dtype, static_cast<uint16_t*>(codes_f16), codes_channel_major, scale,
                       batch, heads, length, head_dim, padded_length, strides[0], strides[1],
                       strides[2], static_cast<cudaStream_t>(stream));
  });
}

extern "C" int tb_w8a8_attn(const int8_t* q, const int8_t* k, const void* v_codes,
                            const float* v_scale, void* out, int out_dtype, const float* q_scale,
                            const float* k_scale, int64_t B, int64_t Hq, int64_t Hk, int64_t Lq,
                            int64_t Lk, int64_t D, const int64_t* strides, int is_causal,
                            float sm_scale, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(q && k && v_codes && v_scale && out && q_scale && k_scale && strides,
               "query, key, value codes, output and scales must be CUDA tensors");
    TB_REQUIRE(B > 0 && Hq > 0 && Hk > 0 && Lq > 0 && Lk > 0, "empty Q/K sequences are not supported");
    TB_REQUIRE(Hq % Hk == 0, "prequantized Sol W8A8 Q heads must be divisible by KV heads");
    TB_REQUIRE(Lq <= INT32_MAX && Lk <= INT32_MAX, "sequence length exceeds the kernel range");
    TB_REQUIRE(is_causal == 0 || is_causal == 1, "is_causal must be 0 or 1");
    tb::require_sm100();
    tb::AttnArgs a{};
    a.q = q;
    a.k = k;
    a.v = v_codes;
    a.v_dtype = TB_DTYPE_F16;
    a.out = out;
    a.out_dtype = out_dtype;
    a.q_scale = q_scale;
    a.k_scale = k_scale;
    a.lse = nullptr;
    a.B = B;
    a.Hq = Hq;
    a.Hk = Hk;
    a.Lq = Lq;
    a.Lk = Lk;
    a.D = D;
    a.q_sb = strides[0]; a.q_sh = strides[1]; a.q_sl = strides[2];
    a.k_sb = strides[3]; a.k_sh = strides[4]; a.k_sl = strides[5];
    a.v_sb = strides[6]; a.v_sh = strides[7]; a.v_sl = strides[8];
    a.o_sb = strides[9]; a.o_sh = strides[10]; a.o_sl = strides[11];
    a.q_tiles_scale = (Lq + 63) / 64 * 4;
    a.k_tiles_scale = (Lk + 63) / 64;
    a.causal = is_causal;
    a.sm_scale = sm_scale;
    a.v_scale = v_scale;
    tb::sage_attn_launch(a, static_cast<cudaStream_t>(stream));
  });
}
