// Memory-bound kernels of the linear path:
//   * INT32 -> BF16 dequant epilogue (kernel/csrc/turing/bf16_epilogue.cu:46-143):
//       out = bf16_rn((acc * a_s[row]) * w_s[col]), w_s scalar or per column;
//   * grouped-codebook W4 -> INT8 decode (kernel/csrc/turing/w4a8.cu:907-973):
//       w8 = clamp(rint(codebook[idx] * e4m3(group_scale)), -127, 127);
//   * signed 4-bit -> INT8 unpack for the W4A8 and W4A4 linears
//     (w4a8.cu:34-72): low nibble = even column, two's-complement nibbles;
//   * the DiT block's gated residual add, x = bf16(x + y * gate[col]) in
//     fp32 with one rounding per operation (what `x.addcmul_(y, gate)` on
//     bf16 tensors computes), in place.
// All move 16-byte vectors per thread with grid-stride loops sized to the SM
// count.
#include <cuda_fp8.h>

#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

template <bool SCALAR_W>
__global__ void __launch_bounds__(256) dequant_vec8_kernel(const int32_t* __restrict__ acc,
                                                           int64_t acc_stride,
                                                           const float* __restrict__ a_s,
                                                           const float* __restrict__ w_s,
                                                           __nv_bfloat16* __restrict__ out,
                                                           int rows, int cols) {
  const int vpr = cols / 8;
  const int64_t total = static_cast<int64_t>(rows) * vpr;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(v / vpr);
    const int col = static_cast<int>(v - static_cast<int64_t>(row) * vpr) * 8;
    const int32_t* src = acc + static_cast<int64_t>(row) * acc_stride + col;
    const int4 x0 = __ldg(reinterpret_cast<const int4*>(src));
    const int4 x1 = __ldg(reinterpret_cast<const int4*>(src + 4));
    const float xs = __ldg(a_s + row);
    float w[8];
    if (SCALAR_W) {
      const float s = __ldg(w_s);
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = s;
    } else {
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(w_s + col));
      const float4 s1 = __ldg(reinterpret_cast<const float4*>(w_s + col + 4));
      w[0] = s0.x; w[1] = s0.y; w[2] = s0.z; w[3] = s0.w;
      w[4] = s1.x; w[5] = s1.y; w[6] = s1.z; w[7] = s1.w;
    }
    const int a[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fmul_rn(__fmul_rn(static_cast<float>(a[j]), xs), w[j]);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * cols + col) =
        make_uint4(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]), pack_bf16x2(r[4], r[5]),
                   pack_bf16x2(r[6], r[7]));
  }
}

template <bool SCALAR_W>
__global__ void __launch_bounds__(256) dequant_scalar_kernel(const int32_t* __restrict__ acc,
                                                             int64_t acc_stride,
                                                             const float* __restrict__ a_s,
                                                             const float* __restrict__ w_s,
                                                             uint16_t* __restrict__ out, int rows,
                                                             int cols) {
  const int64_t total = static_cast<int64_t>(rows) * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / cols);
    const int col = static_cast<int>(i - static_cast<int64_t>(row) * cols);
    const float v = __fmul_rn(__fmul_rn(static_cast<float>(acc[static_cast<int64_t>(row) * acc_stride + col]),
                                        a_s[row]),
                              w_s[SCALAR_W ? 0 : col]);
    out[i] = f32_to_bf16_bits(v);
  }
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}

__device__ __forceinline__ uint32_t decode_byte(float cb, float s) {
  const int q = __float2int_rn(cb * s);
  return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(max(-127, min(127, q)))));
}

// One thread decodes 16 columns (8 packed bytes) of one weight row.
__global__ void __launch_bounds__(256) codebook_decode_kernel(
    const int8_t* __restrict__ packed, const uint8_t* __restrict__ group_scale,
    const float* __restrict__ codebook, int8_t* __restrict__ out, int rows, int k,
    int group_size) {
  __shared__ float cb[16];
  if (threadIdx.x < 16) cb[threadIdx.x] = codebook[threadIdx.x];
  __syncthreads();
  const int vpr = k / 16;
  const int gpr = k / group_size;
  const int64_t total = static_cast<int64_t>(rows) * vpr;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(v / vpr);
    const int col = static_cast<int>(v - static_cast<int64_t>(row) * vpr) * 16;
    const uint2 pk = __ldg(reinterpret_cast<const uint2*>(packed + static_cast<int64_t>(row) * (k / 2) + col / 2));
    const uint8_t* gs = group_scale + static_cast<int64_t>(row) * gpr;
    uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const uint32_t byte = ((e < 8 ? pk.x : pk.y) >> (8 * ((e >> 1) & 3))) & 0xffu;
      const uint32_t code = (e & 1) ? (byte >> 4) : (byte & 0xfu);
      const float s = e4m3_to_f32(__ldg(gs + (col + e) / group_size));
      words[e >> 2] |= decode_byte(cb[code], s) << (8 * (e & 3));
    }
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * k + col) =
        make_uint4(words[0], words[1], words[2], words[3]);
  }
}

// Four codes (nibbles 0..3 of w) looked up in a 16-byte table held in four
// words: two byte permutes pick entries code & 7 from the low and the high
// eight entries, a third takes each byte from the high pick where code >= 8.
__device__ __forceinline__ uint32_t lut16_lookup4(uint32_t w, const uint32_t (&lut)[4]) {
  const uint32_t sel = w & 0x7777u;
  const uint32_t lo = __byte_perm(lut[0], lut[1], sel);
  const uint32_t hi = __byte_perm(lut[2], lut[3], sel);
  return __byte_perm(lo, hi, 0x3210u | ((w >> 1) & 0x4444u));
}

// Codebook decode for group sizes that are multiples of 128: one thread per
// 128 columns of one row, all inside one group, so the group's 16 decoded
// values (decode_byte of each codebook entry with the group scale, the same
// bytes as codebook_decode_kernel) are built once and every nibble is a table
// lookup.
__global__ void __launch_bounds__(256) codebook_decode_lut_kernel(
    const int8_t* __restrict__ packed, const uint8_t* __restrict__ group_scale,
    const float* __restrict__ codebook, int8_t* __restrict__ out, int rows, int k,
    int group_size) {
  __shared__ float cb[16];
  if (threadIdx.x < 16) cb[threadIdx.x] = codebook[threadIdx.x];
  __syncthreads();
  const int cpr = k / 128;
  const int gpr = k / group_size;
  const int64_t total = static_cast<int64_t>(rows) * cpr;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(v / cpr);
    const int col = static_cast<int>(v - static_cast<int64_t>(row) * cpr) * 128;
    const float s = e4m3_to_f32(__ldg(group_scale + static_cast<int64_t>(row) * gpr + col / group_size));
    uint32_t lut[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int c = 0; c < 16; ++c) lut[c >> 2] |= decode_byte(cb[c], s) << (8 * (c & 3));
    // Packed rows are k / 2 bytes (8-byte aligned for k % 16 == 0).
    const uint2* src = reinterpret_cast<const uint2*>(packed + static_cast<int64_t>(row) * (k / 2) + col / 2);
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * k + col);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint2 w = __ldg(src + q);
      dst[q] = make_uint4(lut16_lookup4(w.x, lut), lut16_lookup4(w.x >> 16, lut),
                          lut16_lookup4(w.y, lut), lut16_lookup4(w.y >> 16, lut));
    }
  }
}

// Eight packed nibbles (one 32-bit word, columns 0..7) -> eight int8 values.
// Per byte, (b ^ 8) - 8 sign-extends a nibble b in [0, 15]; __vsub4 keeps the
// four byte lanes independent.  Two byte permutes interleave the even-column
// and odd-column bytes: lo = e0 o0 e1 o1, hi = e2 o2 e3 o3.
__device__ __forceinline__ void unpack_s4_word(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t even = __vsub4((w & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
  const uint32_t odd = __vsub4(((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
  lo = __byte_perm(even, odd, 0x5140);
  hi = __byte_perm(even, odd, 0x7362);
}

// packed holds n_vec 8-byte vectors (16 nibbles each); out receives 16 int8
// per vector.  Rows need no special handling: a row-major [rows, k/2] packed
// matrix maps nibble-for-nibble onto the row-major [rows, k] output.
__global__ void __launch_bounds__(256) unpack_s4_kernel(const uint2* __restrict__ packed,
                                                        uint4* __restrict__ out, int64_t n_vec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_vec;
       i += stride) {
    const uint2 w = __ldg(packed + i);
    uint4 r;
    unpack_s4_word(w.x, r.x, r.y);
    unpack_s4_word(w.y, r.z, r.w);
    out[i] = r;
  }
}

// x[r, c] = bf16_rn(fp32(x) + fp32(y) * fp32(gate[c])) (product and sum each
// rounded to fp32), or bf16_rn(fp32(x) + fp32(y)) without a gate; 8 columns
// (16 bytes) per thread and step.
template <bool GATED>
__global__ void __launch_bounds__(256) gated_residual_kernel(uint16_t* __restrict__ x,
                                                             int64_t x_stride,
                                                             const uint16_t* __restrict__ y,
                                                             int64_t y_stride,
                                                             const uint16_t* __restrict__ gate,
                                                             unsigned int rows,
                                                             unsigned int vpr) {
  const unsigned int total = rows * vpr;
  for (unsigned int v = blockIdx.x * blockDim.x + threadIdx.x; v < total;
       v += gridDim.x * blockDim.x) {
    const unsigned int row = v / vpr;
    const unsigned int col = (v - row * vpr) * 8;
    uint4* px = reinterpret_cast<uint4*>(x + row * x_stride + col);
    const uint4 a = *px;
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(y + row * y_stride + col));
    uint4 g = make_uint4(0u, 0u, 0u, 0u);
    if (GATED) g = __ldg(reinterpret_cast<const uint4*>(gate + col));
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
    const uint32_t wg[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float lo = bf16_bits_to_f32(wb[i] & 0xffffu), hi = bf16_bits_to_f32(wb[i] >> 16);
      if (GATED) {
        lo = __fmul_rn(lo, bf16_bits_to_f32(wg[i] & 0xffffu));
        hi = __fmul_rn(hi, bf16_bits_to_f32(wg[i] >> 16));
      }
      o[i] = pack_bf16x2(__fadd_rn(bf16_bits_to_f32(wa[i] & 0xffffu), lo),
                         __fadd_rn(bf16_bits_to_f32(wa[i] >> 16), hi));
    }
    *px = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

int grid_for(int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

}  // namespace

void dequant_launch(const int32_t* acc, int64_t acc_stride, const float* a_s, const float* w_s,
                    bool scalar_w, void* out, int rows, int cols, cudaStream_t stream) {
  const bool vec = cols % 8 == 0 && acc_stride % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(acc) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
                   (scalar_w || (reinterpret_cast<uintptr_t>(w_s) & 15u) == 0);
  if (vec) {
    const int grid = grid_for(static_cast<int64_t>(rows) * (cols / 8), 256);
    if (scalar_w)
      dequant_vec8_kernel<true><<<grid, 256, 0, stream>>>(acc, acc_stride, a_s, w_s,
                                                          static_cast<__nv_bfloat16*>(out), rows, cols);
    else
      dequant_vec8_kernel<false><<<grid, 256, 0, stream>>>(acc, acc_stride, a_s, w_s,
                                                           static_cast<__nv_bfloat16*>(out), rows, cols);
  } else {
    const int grid = grid_for(static_cast<int64_t>(rows) * cols, 256);
    if (scalar_w)
      dequant_scalar_kernel<true><<<grid, 256, 0, stream>>>(acc, acc_stride, a_s, w_s,
                                                            static_cast<uint16_t*>(out), rows, cols);
    else
      dequant_scalar_kernel<false><<<grid, 256, 0, stream>>>(acc, acc_stride, a_s, w_s,
                                                             static_cast<uint16_t*>(out), rows, cols);
  }
  TB_CUDA_CHECK(cudaGetLastError());
}

void codebook_decode_launch(const int8_t* packed, const uint8_t* group_scale,
                            const float* codebook, int8_t* out, int rows, int k, int group_size,
                            cudaStream_t stream) {
  if (group_size % 128 == 0 && k % 128 == 0) {
    const int grid = grid_for(static_cast<int64_t>(rows) * (k / 128), 256);
    codebook_decode_lut_kernel<<<grid, 256, 0, stream>>>(packed, group_scale, codebook, out, rows,
                                                         k, group_size);
    TB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int grid = grid_for(static_cast<int64_t>(rows) * (k / 16), 256);
  codebook_decode_kernel<<<grid, 256, 0, stream>>>(packed, group_scale, codebook, out, rows, k,
                                                   group_size);
  TB_CUDA_CHECK(cudaGetLastError());
}

void gated_residual_launch(void* x, int64_t x_stride, const void* y, int64_t y_stride,
                           const void* gate, int64_t rows, int64_t cols, cudaStream_t stream) {
  TB_REQUIRE(cols % 8 == 0 && x_stride % 8 == 0 && y_stride % 8 == 0,
             "gated residual add needs columns and row strides divisible by 8");
  TB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(y) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(gate) & 15u) == 0,
             "gated residual add needs 16-byte aligned x, y and gate");
  TB_REQUIRE(rows * (cols / 8) <= INT32_MAX, "gated residual add exceeds the kernel range");
  const int64_t n_vec = rows * (cols / 8);
  if (n_vec == 0) return;
  const int grid = grid_for(n_vec, 256);
  auto* xb = static_cast<uint16_t*>(x);
  auto* yb = static_cast<const uint16_t*>(y);
  auto* gb = static_cast<const uint16_t*>(gate);
  if (gate != nullptr)
    gated_residual_kernel<true><<<grid, 256, 0, stream>>>(xb, x_stride, yb, y_stride, gb,
                                                          static_cast<unsigned int>(rows),
                                                          static_cast<unsigned int>(cols / 8));
  else
    gated_residual_kernel<false><<<grid, 256, 0, stream>>>(xb, x_stride, yb, y_stride, gb,
                                                           static_cast<unsigned int>(rows),
                                                           static_cast<unsigned int>(cols / 8));
  TB_CUDA_CHECK(cudaGetLastError());
}

void unpack_s4_launch(const int8_t* packed, int8_t* out, int64_t rows, int64_t k,
                      cudaStream_t stream) {
  TB_REQUIRE(k % 16 == 0, "signed 4-bit unpack requires K divisible by 16");
  TB_REQUIRE((reinterpret_cast<uintptr_t>(packed) & 7u) == 0 &&
                 (reinterpret_cast<uintptr_t>(out) & 15u) == 0,
             "signed 4-bit unpack requires 8-byte aligned input and 16-byte aligned output");
  const int64_t n_vec = rows * (k / 16);
  if (n_vec == 0) return;
  unpack_s4_kernel<<<grid_for(n_vec, 256), 256, 0, stream>>>(
      reinterpret_cast<const uint2*>(packed), reinterpret_cast<uint4*>(out), n_vec);
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tb
