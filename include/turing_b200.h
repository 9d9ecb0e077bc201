/*
 * turing_b200.h — C ABI of libturing_b200.so, the sm_100a (B200) implementation
 * of the comfyui-turing-utils quantized DiT path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream) and returns a
 * status code.  On failure the message is available from tb_last_error()
 * (thread-local) and nothing was launched.  Buffers are owned by the caller:
 * outputs and workspaces are allocated by the binding and written in place, as
 * in the reference (kernel/csrc/bindings.cpp:206-210, 350-353, 409-410).
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to the reference project root).  The reference's native interface is the C++
 * ABI in kernel/csrc/kernel_api.h (functions taking `Tensor` PODs,
 * kernel/csrc/tensor_bridge.h:83-236) and the Sage entry points in
 * kernel/csrc/turing/sage/fused.h and attn_cuda_sm75.h; here each `Tensor`
 * becomes a pointer plus the sizes the kernel needs.
 */
#ifndef TURING_B200_H
#define TURING_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define TB_OK 0
#define TB_ERR_INVALID 1     /* argument / shape error (reference: TORCH_CHECK) */
#define TB_ERR_CUDA 2        /* CUDA runtime error at launch */
#define TB_ERR_UNSUPPORTED 3 /* device is not sm_100 */
#define TB_ERR_INTERNAL 4

/* 16-bit floating-point input types. */
#define TB_DTYPE_BF16 0
#define TB_DTYPE_F16 1
#define TB_DTYPE_F32 2  /* norm + AdaLN ops only */

/* Tensor layouts of the Sage entry points (reference: tensor_layout 0/1,
 * kernel/csrc/turing/sage/qk_int_sv_f16_cuda_sm75.cu:1059-1101). */
#define TB_LAYOUT_NHD 0
#define TB_LAYOUT_HND 1

typedef void *tb_stream_t;

/* Exported symbols (the library is built with hidden default visibility). */
#if defined(__GNUC__)
#define TB_API __attribute__((visibility("default")))
#else
#define TB_API
#endif

/* ABI version of this header (bumped on any signature change). */
TB_API int tb_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
TB_API const char *tb_last_error(void);

/* Reads and clears the device-side watchdog word of the current device: 0 if
 * no kernel of this library hit a wait limit since the last call.  No
 * counterpart in the reference (its kernels have no bounded waits). */
TB_API int tb_device_error(int *code_out);

/* ------------------------------------------------ ConvRot quantizers ---- */

/* Alignment (every ConvRot entry below, the allocation-free one included):
 * input, output and the staged form's rotated scratch must be 16-byte
 * aligned, scales and partial_absmax 4-byte aligned (the kernels move 16
 * bytes per access).  Other pointers are rejected with TB_ERR_INVALID before
 * anything is launched. */

/* BF16 row-buffer ConvRot INT8 quantizer: input bf16 [rows, swiglu ? 2*hidden :
 * hidden], output int8 [rows, hidden], scales fp32 [rows].  forced_threads is
 * validated (0/512/768/1024) for signature parity; the kernel sizes its own
 * CTA.  Replaces kernel_api.h:66-70 turing_bf16_int8_convrot_quantize
 * (binding checks kernel/csrc/bindings.cpp:603-646). */
TB_API int tb_bf16_int8_convrot_quantize(const void *input, int64_t rows, int64_t hidden, int swiglu,
                                  int forced_threads, int8_t *output, float *scales,
                                  tb_stream_t stream);

/* As above with packed INT4 output int8 [rows, hidden/2] (low nibble = even
 * column).  Replaces kernel_api.h:72-76 (bindings.cpp:649-688). */
TB_API int tb_bf16_int4_convrot_quantize(const void *input, int64_t rows, int64_t hidden, int swiglu,
                                  int8_t *output, float *scales, tb_stream_t stream);

/* tanh-GELU fused row-buffer quantizers, input bf16 [rows, hidden].
 * Replace kernel_api.h:78-81 and 83-86 (bindings.cpp:690-741). */
TB_API int tb_bf16_gelu_int8_convrot_quantize(const void *input, int64_t rows, int64_t hidden,
                                       int8_t *output, float *scales, tb_stream_t stream);
TB_API int tb_bf16_gelu_int4_convrot_quantize(const void *input, int64_t rows, int64_t hidden,
                                       int8_t *output, float *scales, tb_stream_t stream);

/* Staged (two-pass) ConvRot quantizers with caller-owned scratch:
 * rotated [rows, hidden] of the input dtype and partial_absmax fp32
 * [rows, hidden/256].  dtype TB_DTYPE_BF16 or TB_DTYPE_F16.
 * Replace kernel_api.h:44-48, 50-54, 56-60, 62-64 (bindings.cpp:469-601). */
TB_API int tb_swiglu_int8_convrot_quantize(const void *input, int dtype, int64_t rows, int64_t hidden,
                                    void *rotated, float *partial_absmax, int8_t *output,
                                    float *scales, tb_stream_t stream);
TB_API int tb_swiglu_int4_convrot_quantize(const void *input, int dtype, int64_t rows, int64_t hidden,
                                    void *rotated, float *partial_absmax, int8_t *output,
                                    float *scales, tb_stream_t stream);
TB_API int tb_gelu_int8_convrot_quantize(const void *input, int dtype, int64_t rows, int64_t hidden,
                                  void *rotated, float *partial_absmax, int8_t *output,
                                  float *scales, tb_stream_t stream);
TB_API int tb_gelu_int4_convrot_quantize(const void *input, int dtype, int64_t rows, int64_t hidden,
                                  void *rotated, float *partial_absmax, int8_t *output,
                                  float *scales, tb_stream_t stream);

/* Allocation-free SwiGLU INT8 ConvRot quantizer (staged two-pass form) for
 * callers that cannot allocate device memory when they quantize -- e.g. a host
 * whose memory manager owns all VRAM and forbids untracked allocations, or a
 * path that must not take cudaMalloc's implicit device synchronisation.
 * Same arguments and results as tb_swiglu_int8_convrot_quantize minus the two
 * scratch buffers: the scratch is a fixed 16 MiB array inside the library's
 * device image, reserved on every GPU that loads the library until the process
 * exits.  Limit: rows * hidden * 2 (rounded up to 256) + rows * hidden / 64
 * bytes <= 16 MiB; larger problems are rejected with TB_ERR_INVALID.  The first
 * call on each device looks up the array's device address; make that first
 * call before any stream capture (a new context on the device, e.g. after
 * cudaDeviceReset, repeats the lookup).  All calls share the one array, so
 * calls that overlap on the GPU (different streams without ordering) race on
 * it.  Alignment as for the other ConvRot entries.
 * No counterpart in the reference. */
TB_API int tb_swiglu_int8_convrot_quantize_noalloc(const void *input, int dtype, int64_t rows,
                                                   int64_t hidden, int8_t *output, float *scales,
                                                   tb_stream_t stream);

/* --------------------------------------------------- GEMM + epilogue ---- */

/* W8A8 linear: out[m, n] = bf16(((float)sum_k act[m,k] w[n,k] * a_s[m]) * w_s[n]
 * + bias[n]).  act int8 [m, k], weight int8 [n, k] (K-contiguous rows),
 * activation_scale fp32 [m], weight_scale fp32 [n], bias fp32 [n] or NULL,
 * output bf16 [m, ldo].  Requires k % 16 == 0 and n % 8 == 0.
 * Replaces kernel_api.h:29-35 turing_int8_linear (bindings.cpp:371-421,
 * w4a8.cu:1185-1219). */
TB_API int tb_int8_linear(const int8_t *activation, const int8_t *weight, const float *activation_scale,
                   const float *weight_scale, const float *bias, void *output, int64_t m,
                   int64_t n, int64_t k, int64_t ldo, int tile_policy, tb_stream_t stream);

/* Grouped-codebook W4A8 linear: weight = packed 4-bit codebook indices
 * [n, k/2], group_scale = raw E4M3 bytes [n, k/group_size], channel_scale
 * fp32 [n], codebook fp32 [16].  Weight row w8 = clamp(rint(codebook[idx] *
 * e4m3(group_scale)), -127, 127).  workspace int8 [workspace_rows, k] (the
 * staged decode chunk) may be NULL when inline_decode != 0.
 * Replaces kernel_api.h:15-27 turing_codebook_w4a8_linear
 * (w4a8.cu:1088-1183, bindings.cpp:262-369). */
TB_API int tb_codebook_w4a8_linear(const int8_t *activation, const int8_t *weight_packed,
                            const float *activation_scale, const uint8_t *group_scale,
                            const float *channel_scale, const float *codebook, const float *bias,
                            int8_t *workspace, int64_t workspace_rows, void *output, int64_t m,
                            int64_t n, int64_t k, int64_t group_size, int inline_decode,
                            int tile_policy, tb_stream_t stream);

/* Signed-nibble W4A8 linear: weight_packed [n, k/2] holds two's-complement
 * 4-bit weights, low nibble = even column; each chunk of workspace_rows
 * weight rows (workspace: caller-owned int8 [workspace_rows, k], a multiple of
 * 8) is unpacked to int8 and contracted as tb_int8_linear, writing output
 * columns [row, row + chunk) with row stride ldo.  Requires k % 16 == 0 and
 * n % 8 == 0 (the Python binding pads an N tail to 8, as the reference does).
 * Replaces kernel_api.h:7-13 turing_w4a8_linear (w4a8.cu:34-72, 1000-1086,
 * bindings.cpp:167-259). */
TB_API int tb_w4a8_linear(const int8_t *activation, const int8_t *weight_packed,
                          const float *activation_scale, const float *weight_scale,
                          const float *bias, int8_t *workspace, int64_t workspace_rows,
                          void *output, int64_t m, int64_t n, int64_t k, int64_t ldo,
                          int tile_policy, tb_stream_t stream);

/* W4A4 linear: both operands packed signed 4-bit (low nibble = even column),
 * activation_packed [m, k/2] as written by the INT4 ConvRot quantizers with
 * activation_scale [m] (absmax / 7), weight_packed [n, k/2] with weight_scale
 * [n].  out = bf16(((float)sum_k a4 * w4 * a_s[m]) * w_s[n] + bias[n]).  The
 * activations are unpacked into activation_workspace (int8 [m, k]) and the
 * weights chunk by chunk into weight_workspace (int8 [workspace_rows, k]).
 * Replaces the comfy-kitchen int4_linear call of the plugin's W4A4 path
 * (comfyui_turing_utils/quantization/dispatch.py:791-804); the INT4 codes
 * come from convrot_quant.cu:409-433. */
TB_API int tb_int4_linear(const int8_t *activation_packed, const int8_t *weight_packed,
                          const float *activation_scale, const float *weight_scale,
                          const float *bias, int8_t *activation_workspace,
                          int8_t *weight_workspace, int64_t workspace_rows, void *output,
                          int64_t m, int64_t n, int64_t k, int64_t ldo, tb_stream_t stream);

/* Fused Q/K prologue of the Sage path: RMSNorm (norm_scope 0: over each head's
 * D channels with weight [D]; 1: over all heads of the token with weight
 * [heads * D], rrms scratch query_rrms [B, Lq] / key_rrms [B, Lk]), RoPE as
 * 2x2 rotations from freqs [freq_batches, freq_sequence, 1, rot_dim/2, 2, 2]
 * (freq_strides: batch, sequence, pair, row, col in elements; split_half
 * pairs (p, p + rot_dim/2), else (2p, 2p+1)), then INT8 quantization with the
 * Sage scale layout (norm_scope 2: whole row with query_rrms / key_rrms
 * supplied by the caller, see tb_row_sum_squares): Q per 16-token tile into query_scale [B, Hq, ceil(Lq/64)*4],
 * K per 64-token block into key_scale [B, Hk, ceil(Lk/64)]; codes clamped to
 * +-127.  strides (elements, 16 values): q (b, h, l), k (b, h, l), q_out
 * (b, h, l), k_out (b, h, l), q_scale (b, h), k_scale (b, h); the last
 * dimension is contiguous; Q/K and the norm weights start on 16-byte
 * boundaries, strides are multiples of 8 elements and the INT8 outputs start
 * on 8-byte boundaries.  head_dim 64 or 128, dtype BF16 / F16.  Replaces
 * quant_qk_rms_rope_int8_cuda without the Hadamard/anchor options
 * (kernel/csrc/turing/sage/qk_preprocess.cu:566-753, fused.h:80). */
TB_API int tb_quant_qk_rms_rope_int8(const void *query, const void *key, int8_t *query_out,
                                     int8_t *key_out, float *query_scale, float *key_scale,
                                     const void *query_norm, const void *key_norm,
                                     const void *freqs, float *query_rrms, float *key_rrms,
                                     int64_t batch, int64_t query_heads, int64_t key_heads,
                                     int64_t query_length, int64_t key_length, int64_t head_dim,
                                     const int64_t *strides, const int64_t *freq_strides,
                                     int64_t freq_batches, int64_t freq_sequence, int64_t rot_dim,
                                     int norm_scope, int split_half, int dtype, float epsilon,
                                     tb_stream_t stream);

/* Per-token sum of squares over all heads of one Q or K tensor (elements
 * (b, h, l, 0..head_dim) at b*strides[0] + h*strides[1] + l*strides[2]) into
 * sums [batch, length] fp32, summed in the same order as the row-scope RMS of
 * tb_quant_qk_rms_rope_int8.  For tensor parallelism: each rank sums its own
 * heads, the sums are all-reduced, and the RRMS = rsqrt(sum / (H*D) + eps) is
 * passed to tb_quant_qk_rms_rope_int8 with norm_scope 2.  No counterpart in
 * the reference (its RMS pass, qk_preprocess.cu:203-251, writes the RRMS). */
TB_API int tb_row_sum_squares(const void *input, float *sums, int64_t batch, int64_t heads,
                              int64_t length, int64_t head_dim, const int64_t *strides, int dtype,
                              tb_stream_t stream);

/* ---------------------------------------------------- norm + AdaLN ---- */

/* Segmented RMSNorm + AdaLN: out[r, k] = T(x[r,k] * rsqrt(mean_k x^2 + eps) *
 * w[k] * (1 + scale[m,k]) + shift[m,k]), m = the modulation row of the
 * int32 [start, stop, row] segment holding token r (sorted by stop; 0 when no
 * segment holds r or the row is out of range).  input/output [rows, hidden]
 * contiguous; scale/shift [modulation_rows, hidden] with row strides in
 * elements; dtype TB_DTYPE_BF16 / F16 / F32 for every tensor.  Replaces
 * kernel_api.h:86-92 turing_segmented_rms_adaln (segmented_rms_adaln.cu:135-235,
 * bindings.cpp:734-801). */
TB_API int tb_segmented_rms_adaln(const void *input, const void *weight, const void *scale,
                                  const void *shift, const int32_t *segments, void *output,
                                  int64_t rows, int64_t hidden, int64_t modulation_rows,
                                  int64_t scale_stride, int64_t shift_stride,
                                  int64_t segment_count, int dtype, float epsilon,
                                  tb_stream_t stream);

/* LayerNorm + AdaLN over contiguous [batch, sequence, hidden] with scale/shift
 * [batch, modulation_steps, hidden]: token t of a batch uses modulation step
 * min(t / ceil(sequence / steps), steps - 1); n = T((x - mean) * rsqrt(var +
 * eps)), out = T(float(n) * float(T(1 + scale)) + shift).  Replaces
 * kernel_api.h:94-98 turing_layer_norm_adaln (segmented_rms_adaln.cu:237-306,
 * bindings.cpp:803-849). */
TB_API int tb_layer_norm_adaln(const void *input, const void *scale, const void *shift,
                               void *output, int64_t batch, int64_t sequence, int64_t hidden,
                               int64_t modulation_steps, int dtype, float epsilon,
                               tb_stream_t stream);

/* INT32 accumulator GEMM: acc[m, n] = sum_k act[m,k] * w[n,k] (exact int32),
 * acc row stride acc_stride (elements).  Replaces the INT32 cuBLAS GEMM that
 * the plugin feeds into turing_dequantize_int8_bf16
 * (comfyui_turing_utils/quantization/dispatch.py:481-535); also the
 * accumulator dump used by the bit-exact tests. */
TB_API int tb_int8_gemm_s32(const int8_t *activation, const int8_t *weight, int32_t *accumulator,
                     int64_t m, int64_t n, int64_t k, int64_t acc_stride, tb_stream_t stream);

/* Gated residual add of the DiT block, in place on bf16 rows:
 * x[r, c] = bf16(x[r, c] + y[r, c] * gate[c]) with the product and the sum
 * each rounded to fp32 (gate == NULL: x[r, c] = bf16(x + y)).  x, y and gate
 * 16-byte aligned, cols and both row strides (elements) multiples of 8.  No
 * reference counterpart: the model code around the plugin runs this as
 * torch's `x.addcmul_(y, gate)` on bf16 tensors. */
TB_API int tb_gated_residual_add(void *x, int64_t x_stride, const void *y, int64_t y_stride,
                                 const void *gate, int64_t rows, int64_t cols,
                                 tb_stream_t stream);

/* INT32 -> BF16 dequant epilogue: out[r, c] = bf16((acc[r, c] * a_s[r]) * w_s[c])
 * (w_s scalar when weight_scale_numel == 1).  Replaces kernel_api.h:37-40
 * turing_dequantize_int8_bf16 (bf16_epilogue.cu:147-218). */
TB_API int tb_dequantize_int8_bf16(const int32_t *accumulator, int64_t acc_stride,
                            const float *activation_scale, const float *weight_scale,
                            int64_t weight_scale_numel, void *output, int64_t rows, int64_t cols,
                            tb_stream_t stream);

/* ----------------------------------------------------- Sage quantizers -- */

/* Per-tile INT8 quantization of Q or K.  input [B, H, L, D] (layout HND) or
 * [B, L, H, D] (NHD), last dim contiguous, element strides stride_b / stride_h
 * / stride_l; output int8 contiguous with the input's shape; scale fp32
 * [B, H, ceil(L / tile)] contiguous.  mean: optional bf16/f16 [B, H, D]
 * smoothing mean subtracted before quantization (NULL = none).
 *   tb_quant_per_block_int8: tile = block_size tokens (K, 64) — replaces
 *     fused.h:27-32 quant_per_block_int8_cuda (fused.cu:983-1067).
 *   tb_quant_per_warp_int8: tile = warp_block_size tokens inside block_size
 *     blocks (Q, 64/16), scale [B, H, ceil(L/block)*(block/warp)] — replaces
 *     fused.h:35-41 quant_per_warp_int8_cuda (fused.cu:1070-1150). */
TB_API int tb_quant_per_block_int8(const void *input, int dtype, int8_t *output, float *scale, int64_t B,
                            int64_t H, int64_t L, int64_t D, int64_t stride_b, int64_t stride_h,
                            int64_t stride_l, int block_size, int layout, const void *mean,
                            tb_stream_t stream);
TB_API int tb_quant_per_warp_int8(const void *input, int dtype, int8_t *output, float *scale, int64_t B,
                           int64_t H, int64_t L, int64_t D, int64_t stride_b, int64_t stride_h,
                           int64_t stride_l, int block_size, int warp_block_size, int layout,
                           tb_stream_t stream);

/* Token mean for K smoothing: mean [B, H, D] of the input dtype, accumulated in
 * fp64 and rounded to fp32 then to the input dtype.  Produces the `mean` that
 * the reference's QuantInt8Kernel<..., sub_mean=true> consumes
 * (fused.cu:97-128); the reference has no kernel that computes it. */
TB_API int tb_token_mean(const void *input, int dtype, void *mean, int64_t B, int64_t H, int64_t L,
                  int64_t D, int64_t stride_b, int64_t stride_h, int64_t stride_l, int layout,
                  tb_stream_t stream);

/* ------------------------------------------------------- Sage attention -- */

/* INT8 QK^T / 16-bit PV attention with fp32 accumulation: q, k int8 with
 * per-warp (16-row) Q scales [B, Hq, ceil(Lq/64)*4] and per-block (64-key) K
 * scales [B, Hk, ceil(Lk/64)]; v and out of dtype v_dtype (== out_dtype);
 * strides: 12 element strides (batch, head, token) of q, k, v, out in that
 * order, last dim contiguous; layout TB_LAYOUT_HND or TB_LAYOUT_NHD; D = 128
 * (the binding pads 64 < D < 128); lse: optional [B, Hq, Lq] base-2 log-sum-exp.
 * Replaces attn_cuda_sm75.h:21-31 qk_int8_sv_f16_accum_f32_attn
 * (qk_int_sv_f16_cuda_sm75.cu:984-1123). */
TB_API int tb_qk_int8_sv_f16_accum_f32_attn(const int8_t *q, const int8_t *k, const void *v,
                                            int v_dtype, void *out, int out_dtype,
                                            const float *q_scale, const float *k_scale,
                                            float *lse, int64_t B, int64_t Hq, int64_t Hk,
                                            int64_t Lq, int64_t Lk, int64_t D,
                                            const int64_t *strides, int layout, int is_causal,
                                            int qk_quant_gran, float sm_scale,
                                            tb_stream_t stream);

/* ----------------------------------------------- W8A8-PV attention ---- */

/* Randomized-Hadamard INT8 Q/K of the W8A8 attention: each token row of D = 64
 * or 128 channels becomes H_D diag(sign) x / sqrt(D) (the reference's sign
 * vector and butterfly order), then Q is quantized per 16-token tile into
 * query_scale [B, Hq, ceil(Lq/64)*4] and K per 64-token block into key_scale
 * [B, Hk, ceil(Lk/64)], amax floor 1e-7, scale = amax / 127, codes
 * rni(x * 127 / amax), a NaN coded nan_code (0 or -127).  anchor_mode 0: no
 * K anchor; 1: each (batch, kv head) picks its anchor row from nine sampled
 * keys, writes it to anchors int32 [B, Hk] (or -1) and its values to
 * anchor_values fp32 [B, Hk, D] (zeros for -1), and K minus those values is
 * rotated; 2: anchor_values are given (tb_qk_anchor_processed) and
 * subtracted.  strides (elements, 12 values): q (b, h, l), k (b, h, l),
 * q_out (b, h, l), k_out (b, h, l); last dimension contiguous, Q/K rows
 * 16-byte aligned, the INT8 outputs 8-byte aligned.  dtype BF16 / F16.
 * Replaces quant_qk_per_warp_int8_rotated_anchored_cuda (mode 1) and
 * quant_qk_per_warp_int8_rotated_cuda (mode 0) (kernel/csrc/turing/sage/
 * fused.h:55-78, fused.cu:1252-1287 with the kernels at :201-639), and with
 * mode 2 / nan_code -127 the quantizing half of the fused prologue's rotated
 * form (qk_preprocess.cu:417-563). */
TB_API int tb_quant_qk_int8_rotated(const void *query, const void *key, int8_t *query_out,
                                    int8_t *key_out, float *query_scale, float *key_scale,
                                    int32_t *anchors, float *anchor_values, int64_t batch,
                                    int64_t query_heads, int64_t key_heads, int64_t query_length,
                                    int64_t key_length, int64_t head_dim, const int64_t *strides,
                                    int anchor_mode, int nan_code, int dtype, tb_stream_t stream);

/* The normalizing half of tb_quant_qk_rms_rope_int8 for its Hadamard-rotated
 * form: the same RMSNorm + RoPE (same arguments and checks), but each token's
 * values are written, rounded to the input dtype, to query_out / key_out (16-bit,
 * 16-byte aligned, strides in strides[6..11]) instead of being quantized.
 * Replaces the value computation of quantize_tile<..., Rotate>
 * (kernel/csrc/turing/sage/qk_preprocess.cu:417-537). */
TB_API int tb_qk_rms_rope_apply(const void *query, const void *key, void *query_out,
                                void *key_out, const void *query_norm, const void *key_norm,
                                const void *freqs, float *query_rrms, float *key_rrms,
                                int64_t batch, int64_t query_heads, int64_t key_heads,
                                int64_t query_length, int64_t key_length, int64_t head_dim,
                                const int64_t *strides, const int64_t *freq_strides,
                                int64_t freq_batches, int64_t freq_sequence, int64_t rot_dim,
                                int norm_scope, int split_half, int dtype, float epsilon,
                                tb_stream_t stream);

/* K anchor of the fused prologue's rotated form: nine sampled tokens of each
 * (batch, kv head) normalized and rotated as tb_qk_rms_rope_apply does, with
 * their own RRMS (norm_scope 0: one FMA chain over the channels; 1/2: key_rrms
 * [B, Lk] as written by the row pass), then the anchor rule of
 * tb_quant_qk_int8_rotated; anchors int32 [B, Hk] (row or -1), anchor_values
 * fp32 [B, Hk, D].  key_strides (b, h, l) in elements.  Replaces
 * detect_anchor_kernel (kernel/csrc/turing/sage/qk_preprocess.cu:252-415). */
TB_API int tb_qk_anchor_processed(const void *key, const void *key_norm, const void *freqs,
                                  const float *key_rrms, int32_t *anchors, float *anchor_values,
                                  int64_t batch, int64_t key_heads, int64_t key_length,
                                  int64_t head_dim, const int64_t *key_strides,
                                  const int64_t *freq_strides, int64_t freq_batches,
                                  int64_t freq_sequence, int64_t rot_dim, int norm_scope,
                                  int split_half, int dtype, float epsilon, tb_stream_t stream);

/* Channel-wise INT8 V: per (batch, head, channel) scale = max(amax over the
 * tokens / 127, 1e-12) into scale [B, H, D] fp32 (also the kernels' amax
 * scratch while they run), codes rni(v / scale).  Outputs (at least one):
 * codes_f16 [B, H, L, D] contiguous fp16 holding the integer codes exactly
 * (the operand of tb_w8a8_attn), and/or codes_channel_major int8
 * [B, H, D, padded_length] (padded_length a multiple of 64 >= L, padding 0;
 * the reference's layout without its sm75 16-token fragment permutation).
 * strides: v (b, h, l) in elements; D = 64 or 128; dtype BF16 / F16.
 * Replaces attn_cuda_sm75.h:112-114 quantize_v_int8_sm75
 * (quant_v_int8_cuda_sm75.cu:58-246). */
TB_API int tb_quantize_v_int8(const void *value, int dtype, void *codes_f16,
                              int8_t *codes_channel_major, float *scale, int64_t batch,
                              int64_t heads, int64_t length, int64_t head_dim,
                              int64_t padded_length, const int64_t *strides, tb_stream_t stream);

/* Dense W8A8-PV attention: INT8 Q/K with per-warp Q / per-block K scales (as
 * tb_qk_int8_sv_f16_accum_f32_attn, HND or strided), V as the fp16 codes of
 * tb_quantize_v_int8 with v_scale [B, Hk, D]; per row the softmax reference
 * point is the exact running max minus log2 255, P = rni(2^(s c - m)) in
 * [0, 255] multiplies the V codes exactly, d sums the unrounded p, and
 * out = O / d * v_scale (out_dtype BF16 / F16).  strides: q, k, v_codes, out
 * (b, h, l) in elements; D = 128 (pad 64 < D < 128).  Replaces the dense
 * (force_dense) path of attn_cuda_sm75.h:61-83
 * sol_sparse_online_w8a8_prequantized_attn (sol_sparse_cuda_sm75.cu:709-1394,
 * 2767-2932). */
TB_API int tb_w8a8_attn(const int8_t *q, const int8_t *k, const void *v_codes,
                        const float *v_scale, void *out, int out_dtype, const float *q_scale,
                        const float *k_scale, int64_t B, int64_t Hq, int64_t Hk, int64_t Lq,
                        int64_t Lk, int64_t D, const int64_t *strides, int is_causal,
                        float sm_scale, tb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TURING_B200_H */
