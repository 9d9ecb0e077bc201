// ConvRot activation quantizer for sm_100a: 256-wide block-Hadamard rotation
// followed by per-token symmetric INT8 (or packed INT4) quantization, with
// optional fused SwiGLU / tanh-GELU on the load.
//
// Semantics follow the reference kernels bit for bit
// (kernel/csrc/turing/convrot_quant.cu:104-156 FHT and activations,
//  :350-444 BF16 row-buffer kernel, :158-291 staged kernels):
//   * the 256-point transform is applied as four radix-4 stages S = 1, 4, 16,
//     64, each output computed as 0.5 * (((x0 +- x1) +- x2) +- x3) in that
//     order, in fp32 with round-to-nearest and no contraction;
//   * the row absmax is taken over the fp32 rotated values, the stored value
//     is bf16 (fp16 for fp16 inputs of the staged form);
//   * scale = max(min(amax, dtype_max) / 127, 1e-30) (row-buffer form) or
//     max(min(amax, dtype_max) * (1/127), 1e-30) (staged form); INT4 uses 7
//     and 1e-10;
//   * INT8 code = clamp(rint(round_dtype(v / round_dtype(scale))), -128, 127),
//     the reference's IEEE divide taken here as a multiply by the correctly
//     rounded reciprocal of round_dtype(scale) (same codes; see
//     quantize16_store); INT4 code = clamp(rint(v * (1/scale)), -7, 7), two
//     per byte, low nibble = even column.
//
// B200 layout: one half-warp owns a 256-group, 16 consecutive elements per
// lane (two 16-byte loads).  Stages S=1 and S=4 run in registers; the group
// is transposed through a bank-conflict-free shared buffer so that lane l
// holds elements l + 16 j; stages S=16 and S=64 then also run in registers.
// The rotated row is kept as bf16 in shared memory (never in HBM) until the
// row scale is known; the quantized codes leave as 16-byte coalesced stores.
// The single-pass form processes rows in pairs (convrot_rowpair_kernel): each
// fp32 value of row A shares a 64-bit register with the same column of row B,
// so every packed f32x2 add / sub / mul does one butterfly step for both rows.
// The 256-point transform is then bound by the FP32 pipe: 14 operations per
// element (four radix-4 stages of 2 + 4 x 3 adds / subs and 4 halvings per 4
// values), which a packed instruction issues in one slot but occupies for two
// pipe cycles.
#include <mutex>

#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

constexpr int kGroup = 256;
constexpr int kTbufStride = 272;  // floats per half-warp transpose buffer (256 + 16 pad)

enum Act { kActNone = 0, kActSwiGLU = 1, kActGelu = 2 };

template <typename T>
__device__ __forceinline__ float elem_to_f32(uint32_t bits16);
template <>
__device__ __forceinline__ float elem_to_f32<__nv_bfloat16>(uint32_t b) {
  return bf16_bits_to_f32(b);
}
template <>
__device__ __forceinline__ float elem_to_f32<__half>(uint32_t b) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
}

template <typename T>
__device__ __forceinline__ uint32_t f32_to_elem_bits(float v);
template <>
__device__ __forceinline__ uint32_t f32_to_elem_bits<__nv_bfloat16>(float v) {
  return f32_to_bf16_bits(v);
}
template <>
__device__ __forceinline__ uint32_t f32_to_elem_bits<__half>(float v) {
  return __half_as_ushort(__float2half_rn(v));
}

template <typename T>
__device__ __forceinline__ float round_to_elem(float v) {
  return elem_to_f32<T>(f32_to_elem_bits<T>(v));
}

// Two floats rounded to T and packed (lo in bits 0..15), with the hardware
// cvt.rn: the same round-to-nearest-even as f32_to_elem_bits, and NaN gives
// the canonical NaN 0x7fff as the reference's float_to_bf16_rn_bits does.
template <typename T>
__device__ __forceinline__ uint32_t pack2_elem(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return pack_bf16x2(lo, hi);
  else return pack_f16x2(lo, hi);
}

template <typename T>
__device__ __forceinline__ float dtype_finite_max();
template <>
__device__ __forceinline__ float dtype_finite_max<__nv_bfloat16>() {
  return 3.38953139e38f;
}
template <>
__device__ __forceinline__ float dtype_finite_max<__half>() {
  return 65504.0f;
}

// Activations exactly as written in the reference so that nvcc forms the same
// expression tree (convrot_quant.cu:137-156).
__device__ __forceinline__ float swiglu_value(float gate, float up) {
  return (gate / (1.0f + expf(-gate))) * up;
}

template <typename T>
__device__ __forceinline__ float gelu_value(float x) {
  constexpr float kAlpha = 0.7978845608028654f;
  constexpr float kBeta = 0.044715f;
  const float activated = 0.5f * x * (1.0f + tanhf(kAlpha * (x + kBeta * x * x * x)));
  return round_to_elem<T>(activated);
}

// One radix-4 butterfly in the reference's operation order.
__device__ __forceinline__ void butterfly4(float& x0, float& x1, float& x2, float& x3) {
  const float s01 = __fadd_rn(x0, x1);
  const float d01 = __fsub_rn(x0, x1);
  const float y0 = __fmul_rn(0.5f, __fsub_rn(__fadd_rn(s01, x2), x3));
  const float y1 = __fmul_rn(0.5f, __fadd_rn(__fsub_rn(s01, x2), x3));
  const float y2 = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(d01, x2), x3));
  // (-x0 + x1) + x2 == x2 - (x0 - x1) exactly (negation is exact).
  const float y3 = __fmul_rn(0.5f, __fadd_rn(__fsub_rn(x2, d01), x3));
  x0 = y0;
  x1 = y1;
  x2 = y2;
  x3 = y3;
}

// Two independent butterflies at once on packed f32x2 registers (lane 0 =
// the first butterfly): every packed add / sub / mul rounds each lane as its
// scalar form does, so the results are the scalar butterfly4's bit for bit.
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpk(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t padd(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t psub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t pmul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t phalf(uint64_t a) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(0x3F0000003F000000ull));
  return r;
}
__device__ __forceinline__ void butterfly4x2(float& a0, float& a1, float& a2, float& a3,
                                             float& b0, float& b1, float& b2, float& b3) {
  const uint64_t x0 = pk(a0, b0), x1 = pk(a1, b1), x2 = pk(a2, b2), x3 = pk(a3, b3);
  const uint64_t s01 = padd(x0, x1);
  const uint64_t d01 = psub(x0, x1);
  const uint64_t y0 = phalf(psub(padd(s01, x2), x3));
  const uint64_t y1 = phalf(padd(psub(s01, x2), x3));
  const uint64_t y2 = phalf(padd(padd(d01, x2), x3));
  const uint64_t y3 = phalf(padd(psub(x2, d01), x3));
  unpk(y0, a0, b0);
  unpk(y1, a1, b1);
  unpk(y2, a2, b2);
  unpk(y3, a3, b3);
}

// Stage on 4 consecutive registers (S=1 in layout A, S=16 in layout B).
__device__ __forceinline__ void stage_contig(float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; q += 2)
    butterfly4x2(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3],
                 v[4 * q + 4], v[4 * q + 5], v[4 * q + 6], v[4 * q + 7]);
}

// Stage on registers 4 apart (S=4 in layout A, S=64 in layout B).
__device__ __forceinline__ void stage_strided(float (&v)[16]) {
#pragma unroll
  for (int p = 0; p < 4; p += 2)
    butterfly4x2(v[p], v[p + 4], v[p + 8], v[p + 12], v[p + 1], v[p + 5], v[p + 9], v[p + 13]);
}

// Loads the 16 activated fp32 inputs of lane l (elements col..col+15).
template <typename T, int ACT>
__device__ __forceinline__ void load16(const T* __restrict__ row_in, int k, int col,
                                       float (&v)[16]) {
  const uint4* p = reinterpret_cast<const uint4*>(row_in + col);
  uint4 a = __ldg(p);
  uint4 b = __ldg(p + 1);
  uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float x[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[2 * i] = elem_to_f32<T>(w[i] & 0xffffu);
    x[2 * i + 1] = elem_to_f32<T>(w[i] >> 16);
  }
  if constexpr (ACT == kActSwiGLU) {
    const uint4* q = reinterpret_cast<const uint4*>(row_in + k + col);
    uint4 c = __ldg(q);
    uint4 d = __ldg(q + 1);
    uint32_t u[8] = {c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[2 * i] = swiglu_value(x[2 * i], elem_to_f32<T>(u[i] & 0xffffu));
      v[2 * i + 1] = swiglu_value(x[2 * i + 1], elem_to_f32<T>(u[i] >> 16));
    }
  } else if constexpr (ACT == kActGelu) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = gelu_value<T>(x[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = x[i];
  }
}

// Full 256-point rotation of one group held by a half-warp.  On entry lane l
// holds elements 16 l + j in v[j]; on exit it holds elements l + 16 j.
__device__ __forceinline__ void rotate_group(float (&v)[16], float* __restrict__ tbuf, int l) {
  stage_contig(v);   // S = 1
  stage_strided(v);  // S = 4
  const int swz = (l >> 1) & 3;
  float4* row = reinterpret_cast<float4*>(tbuf + 16 * l);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    row[c ^ swz] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
  __syncwarp();
  const int c_read = l >> 2, w_read = l & 3;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int swz_j = (j >> 1) & 3;
    v[j] = tbuf[16 * j + 4 * (c_read ^ swz_j) + w_read];
  }
  __syncwarp();
  stage_contig(v);   // S = 16
  stage_strided(v);  // S = 64
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

struct RowQuantParams {
  const void* input;
  int8_t* output;
  float* scales;
  void* rotated;          // staged form: [rows, k] T scratch
  float* partial_absmax;  // staged form: [rows, k/256]
  int rows;
  int k;
  int rows_per_cta;
};

template <typename T, bool INT4, bool STAGED_SCALE>
__device__ __forceinline__ float row_scale_from_amax(float amax) {
  constexpr float qmax = INT4 ? 7.0f : 127.0f;
  constexpr float floor_v = INT4 ? 1.0e-10f : 1.0e-30f;
  const float clipped = fminf(amax, dtype_finite_max<T>());
  if constexpr (STAGED_SCALE) {
    return fmaxf(__fmul_rn(clipped, 1.0f / qmax), floor_v);
  } else {
    return fmaxf(__fdiv_rn(clipped, qmax), floor_v);
  }
}

// Both halves of a T pair clamped to [-128, 127] with the 16-bit max / min
// (a NaN operand loses, as in fmaxf / fminf, so NaN gives -128); -128 and 127
// are exact in bf16 and fp16, so this equals clamping the widened values.
template <typename T>
__device__ __forceinline__ uint32_t clamp_pair_i8(uint32_t d2) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("{\n\t.reg .b32 t;\n\tmax.bf16x2 t, %1, %2;\n\tmin.bf16x2 %0, t, %3;\n\t}"
        : "=r"(r) : "r"(d2), "r"(0xC300C300u), "r"(0x42FE42FEu));
  } else {
    asm("{\n\t.reg .b32 t;\n\tmax.f16x2 t, %1, %2;\n\tmin.f16x2 %0, t, %3;\n\t}"
        : "=r"(r) : "r"(d2), "r"(0xD800D800u), "r"(0x57F057F0u));
  }
  return r;
}

// Quantizes 16 consecutive rotated elements (bits in `h`) and stores them.
// INT8: the reference divides by the T-rounded scale,
// rint(T(v / T(scale))); here v is multiplied by rcp_rounded =
// __frcp_rn(T(scale)), the correctly rounded reciprocal taken once per row.
// The codes are identical: an exhaustive check over every pair of 16-bit
// values (v, T(scale)) with T(scale) >= 1e-30 -- 1.91e9 bf16 pairs and
// 2.08e9 fp16 pairs -- found no pair whose INT8 code differs from the IEEE
// divide's.  INT4 multiplies by __frcp_rn(scale) as the reference does.
template <typename T, bool INT4>
__device__ __forceinline__ void quantize16_store(const uint32_t (&h)[8], float rcp_rounded,
                                                 float inv_scale, int8_t* __restrict__ dst) {
  if constexpr (INT4) {
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float lo = elem_to_f32<T>(h[i] & 0xffffu);
      const float hi = elem_to_f32<T>(h[i] >> 16);
      // clamp-then-round equals round-then-clamp for integer bounds, and
      // fmaxf(NaN, -7) = -7 reproduces the reference's NaN path.
      const int ql = __float2int_rn(fminf(7.0f, fmaxf(-7.0f, __fmul_rn(lo, inv_scale))));
      const int qh = __float2int_rn(fminf(7.0f, fmaxf(-7.0f, __fmul_rn(hi, inv_scale))));
      const uint32_t byte = (static_cast<uint32_t>(ql) & 0xfu) |
                            ((static_cast<uint32_t>(qh) & 0xfu) << 4);
      packed[i >> 2] |= byte << (8 * (i & 3));
    }
    *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
  } else {
    // d = T(v * rcp) two at a time; then clamp to [-128, 127] (fmaxf maps NaN
    // to -128, as the reference's fminf(127, fmaxf(-128, NaN)) does), and
    // adding 1.5 * 2^23 rounds to the nearest integer, ties to even, exactly
    // as __float2int_rn, leaving the code two's-complement in the low byte.
    // Packed: both multiplies in one mul.rn.f32x2 and both rounding adds in
    // one add.rn.f32x2 (each lane rounds as the scalar form), the clamp on the
    // T pair.
    uint32_t cb[16];
    const uint64_t rcp2 = pk(rcp_rounded, rcp_rounded);
    const uint64_t magic2 = pk(12582912.0f, 12582912.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float lo, hi;
      unpk(pmul(pk(elem_to_f32<T>(h[i] & 0xffffu), elem_to_f32<T>(h[i] >> 16)), rcp2), lo, hi);
      const uint32_t d2 = clamp_pair_i8<T>(pack2_elem<T>(lo, hi));
      unpk(padd(pk(elem_to_f32<T>(d2 & 0xffffu), elem_to_f32<T>(d2 >> 16)), magic2), lo, hi);
      cb[2 * i] = __float_as_uint(lo);
      cb[2 * i + 1] = __float_as_uint(hi);
    }
    uint32_t out[4];
#pragma unroll
    for (int w = 0; w < 4; ++w)
      out[w] = __byte_perm(__byte_perm(cb[4 * w], cb[4 * w + 1], 0x0040),
                           __byte_perm(cb[4 * w + 2], cb[4 * w + 3], 0x0040), 0x5410);
    *reinterpret_cast<uint4*>(dst) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

// Single-pass kernel: rows_per_cta rows per CTA, rotated bf16 row buffer in
// shared memory.  Shared layout: [rows_per_cta * k] row buffer (T bits),
// [halfwarps * kTbufStride] f32 transpose buffers, [rows_per_cta] u32 amax.
template <typename T, int ACT, bool INT4, bool STAGED_SCALE>
__global__ void __launch_bounds__(512) convrot_rowbuffer_kernel(RowQuantParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int R = p.rows_per_cta;
  const int k = p.k;
  const int groups = k / kGroup;
  const int halfwarps = blockDim.x >> 4;
  uint16_t* rowbuf = reinterpret_cast<uint16_t*>(smem);
  float* tbuf_all = reinterpret_cast<float*>(smem + static_cast<size_t>(R) * k * 2);
  unsigned int* row_amax =
      reinterpret_cast<unsigned int*>(tbuf_all + static_cast<size_t>(halfwarps) * kTbufStride);

  const int tid = threadIdx.x;
  const int hw = tid >> 4;
  const int l = tid & 15;
  const int row0 = blockIdx.x * R;
  const int rows_here = min(R, p.rows - row0);
  const int in_width = ACT == kActSwiGLU ? 2 * k : k;
  const T* in = static_cast<const T*>(p.input);
  float* tbuf = tbuf_all + hw * kTbufStride;

  for (int r = tid; r < R; r += blockDim.x) row_amax[r] = 0u;
  __syncthreads();

  // Items (row, group) are taken two per warp so both half-warps of a warp
  // run the same number of iterations (the transpose and the shuffles below
  // are warp-collective); an odd last item leaves one half-warp idle.
  const int items = rows_here * groups;
  // (row, group) of this half-warp's item, advanced by `halfwarps` items per
  // iteration without a division.
  int ir = 0, ig = 2 * (hw >> 1) + (hw & 1);
  while (ig >= groups) {
    ig -= groups;
    ++ir;
  }
  for (int base = 2 * (hw >> 1); base < items; base += halfwarps) {
    const int item = base + (hw & 1);
    const bool active = item < items;
    const int r = active ? ir : 0;
    const int g = active ? ig : 0;
    ig += halfwarps;
    while (ig >= groups) {
      ig -= groups;
      ++ir;
    }
    const T* row_in = in + static_cast<int64_t>(row0 + r) * in_width;
    float v[16];
    load16<T, ACT>(row_in, k, g * kGroup + 16 * l, v);
    rotate_group(v, tbuf, l);
    float amax = 0.0f;
    uint16_t* dst = rowbuf + static_cast<size_t>(r) * k + g * kGroup + l;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      amax = fmaxf(amax, fmaxf(fabsf(v[j]), fabsf(v[j + 1])));
      const uint32_t two = pack2_elem<T>(v[j], v[j + 1]);
      if (active) {
        dst[16 * j] = static_cast<uint16_t>(two & 0xffffu);
        dst[16 * (j + 1)] = static_cast<uint16_t>(two >> 16);
      }
    }
    // Non-negative floats order like their bit patterns.
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o, 16));
    if (active && l == 0) atomicMax(&row_amax[r], __float_as_uint(amax));
  }
  __syncthreads();
  // Per-row constants once per row: scale, RN(1 / T(scale)) and RN(1 / scale),
  // over the row's absmax words (which this overwrites: nothing reads them
  // after the barrier below).
  float* row_rcp = reinterpret_cast<float*>(row_amax);
  for (int r = tid; r < rows_here; r += blockDim.x) {
    const float scale = row_scale_from_amax<T, INT4, STAGED_SCALE>(__uint_as_float(row_amax[r]));
    p.scales[row0 + r] = scale;
    row_rcp[r] = INT4 ? __frcp_rn(scale) : __frcp_rn(round_to_elem<T>(scale));
  }
  __syncthreads();

  // Phase 2: quantize the buffered rows with coalesced 16-element chunks.
  const int chunks_per_row = k / 16;
  const int chunks = rows_here * chunks_per_row;
  int cr = 0, cc = tid;  // (row, chunk in row) of chunk `c`, advanced without a division
  while (cc >= chunks_per_row) {
    cc -= chunks_per_row;
    ++cr;
  }
  for (int c = tid; c < chunks; c += blockDim.x) {
    const int r = cr;
    const int col = cc * 16;
    cc += blockDim.x;
    while (cc >= chunks_per_row) {
      cc -= chunks_per_row;
      ++cr;
    }
    const float rcp = row_rcp[r];
    const uint4* src = reinterpret_cast<const uint4*>(rowbuf + static_cast<size_t>(r) * k + col);
    uint4 a = src[0], b = src[1];
    uint32_t h[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const int64_t row = row0 + r;
    int8_t* dst = INT4 ? p.output + row * (k / 2) + col / 2 : p.output + row * k + col;
    quantize16_store<T, INT4>(h, rcp, rcp, dst);
  }
}

// ---------------------------------------------------------------------------
// Row-pair form of the single-pass kernel: the same arithmetic, two rows per
// packed register.  Every fp32 value lives in a 64-bit register pair whose
// low half is row A's element and whose high half is row B's element at the
// same column, so each add.rn / sub.rn / mul.rn.f32x2 performs one butterfly
// operation for both rows and the pairing never changes between stages (no
// register moves to re-pair values).  A half-warp owns one 256-group of both
// rows; the two half-warps of a warp own neighbouring groups.
//
// Shared layout: the rotated row pair as bf16x2 words (word x = column x,
// low half row A, high half row B), 16-byte chunks XOR-swizzled inside each
// 128-byte line so that the phase-1 word stores and the phase-2 16-byte reads
// are both free of bank conflicts; then one 2 KB transpose buffer per
// half-warp (16 x 16 eight-byte units, chunks swizzled); then the per-row
// absmax words.

// Word index -> swizzled word index of the row-pair buffer.  Inside a
// 128-byte line (32 words, 8 chunks) chunk c is stored at c ^ f(line), with
// f taking line bits 0-1 (spreads four consecutive lines read by eight
// consecutive phase-2 threads) and line bit 3 (separates the two half-warps,
// whose groups are 8 lines apart).
__device__ __forceinline__ int pair_swizzle(int x) {
  const int line = x >> 5;
  const int f = (line & 3) | ((line >> 1) & 4);
  return (line << 5) | ((((x >> 2) & 7) ^ f) << 2) | (x & 3);
}

__device__ __forceinline__ void bfly4_pair(uint64_t& x0, uint64_t& x1, uint64_t& x2,
                                           uint64_t& x3) {
  const uint64_t s01 = padd(x0, x1);
  const uint64_t d01 = psub(x0, x1);
  const uint64_t y0 = phalf(psub(padd(s01, x2), x3));
  const uint64_t y1 = phalf(padd(psub(s01, x2), x3));
  const uint64_t y2 = phalf(padd(padd(d01, x2), x3));
  const uint64_t y3 = phalf(padd(psub(x2, d01), x3));
  x0 = y0;
  x1 = y1;
  x2 = y2;
  x3 = y3;
}

// Full 256-point rotation of one group of both rows.  On entry lane l holds
// elements 16 l + j in v[j]; on exit it holds elements l + 16 j.
__device__ __forceinline__ void rotate_group_pair(uint64_t (&v)[16], uint64_t* __restrict__ tb,
                                                  int l) {
#pragma unroll
  for (int q = 0; q < 4; ++q) bfly4_pair(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int p = 0; p < 4; ++p) bfly4_pair(v[p], v[p + 4], v[p + 8], v[p + 12]);
  // Transpose: row l of the 16 x 16 unit matrix is written as 8 chunks of 16
  // bytes, chunk c at c ^ (l & 7) (eight lanes of a 16-byte store phase hit
  // eight different chunks); column l is read back unit by unit (sixteen
  // lanes read one whole 128-byte row).
  uint4* row = reinterpret_cast<uint4*>(tb + 16 * l);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t a0, a1, b0, b1;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(a0), "=r"(a1) : "l"(v[2 * c]));
    asm("mov.b64 {%0, %1}, %2;" : "=r"(b0), "=r"(b1) : "l"(v[2 * c + 1]));
    row[c ^ (l & 7)] = make_uint4(a0, a1, b0, b1);
  }
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = tb[16 * j + 2 * ((l >> 1) ^ (j & 7)) + (l & 1)];
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 4; ++q) bfly4_pair(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int p = 0; p < 4; ++p) bfly4_pair(v[p], v[p + 4], v[p + 8], v[p + 12]);
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

// Both 16-bit halves of d2 widened to fp32 and added to 1.5 * 2^23 in one
// mixed-precision add each (add.rn.f32.{bf16,f16}: the exact widening, then
// the fp32 round-to-nearest add), equal to widening first and adding after.
template <typename T>
__device__ __forceinline__ void add_magic_pair(uint32_t d2, float& lo, float& hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "add.rn.f32.bf16 %0, l, %3;\n\tadd.rn.f32.bf16 %1, h, %3;\n\t}"
        : "=f"(lo), "=f"(hi) : "r"(d2), "f"(12582912.0f));
  } else {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "add.rn.f32.f16 %0, l, %3;\n\tadd.rn.f32.f16 %1, h, %3;\n\t}"
        : "=f"(lo), "=f"(hi) : "r"(d2), "f"(12582912.0f));
  }
}

// Four consecutive columns of a row pair (h[i] = column i, low half row A)
// quantized to INT8: row A's four codes in `a`, row B's in `b`.  The
// arithmetic per value is quantize16_store's INT8 branch: T(v * rcp), the
// 16-bit pair clamp to [-128, 127], then the 1.5 * 2^23 rounding add.
template <typename T>
__device__ __forceinline__ void quantize4_pair_i8(const uint4& h4, uint64_t rcp2, uint32_t& a,
                                                  uint32_t& b) {
  const uint32_t h[4] = {h4.x, h4.y, h4.z, h4.w};
  uint32_t ca[4], cb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float lo, hi;
    unpk(pmul(pk(elem_to_f32<T>(h[i] & 0xffffu), elem_to_f32<T>(h[i] >> 16)), rcp2), lo, hi);
    const uint32_t d2 = clamp_pair_i8<T>(pack2_elem<T>(lo, hi));
    add_magic_pair<T>(d2, lo, hi);
    ca[i] = __float_as_uint(lo);
    cb[i] = __float_as_uint(hi);
  }
  a = __byte_perm(__byte_perm(ca[0], ca[1], 0x0040), __byte_perm(ca[2], ca[3], 0x0040), 0x5410);
  b = __byte_perm(__byte_perm(cb[0], cb[1], 0x0040), __byte_perm(cb[2], cb[3], 0x0040), 0x5410);
}

// INT4 form: clamp(rint(v * (1 / scale)), -7, 7) per value as
// quantize16_store's INT4 branch; four nibbles per row (low nibble = even
// column) in the low 16 bits of `a` and `b`.
template <typename T>
__device__ __forceinline__ void quantize4_pair_i4(const uint4& h4, uint64_t inv2, uint32_t& a,
                                                  uint32_t& b) {
  const uint32_t h[4] = {h4.x, h4.y, h4.z, h4.w};
  a = 0u;
  b = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float lo, hi;
    unpk(pmul(pk(elem_to_f32<T>(h[i] & 0xffffu), elem_to_f32<T>(h[i] >> 16)), inv2), lo, hi);
    const int qa = __float2int_rn(fminf(7.0f, fmaxf(-7.0f, lo)));
    const int qb = __float2int_rn(fminf(7.0f, fmaxf(-7.0f, hi)));
    a |= (static_cast<uint32_t>(qa) & 0xfu) << (4 * i);
    b |= (static_cast<uint32_t>(qb) & 0xfu) << (4 * i);
  }
}

// The 16 input elements of lane l in both rows of an item, as raw 16-bit
// pairs (two 16-byte loads per row), and their fp32 values.
struct RawPair {
  uint4 a0, a1, b0, b1;
};

template <typename T>
__device__ __forceinline__ void load_raw_pair(const T* row_a, const T* row_b, int col, RawPair& r) {
  const uint4* pa = reinterpret_cast<const uint4*>(row_a + col);
  const uint4* pb = reinterpret_cast<const uint4*>(row_b + col);
  r.a0 = __ldg(pa);
  r.a1 = __ldg(pa + 1);
  r.b0 = __ldg(pb);
  r.b1 = __ldg(pb + 1);
}

template <typename T>
__device__ __forceinline__ void widen16(const uint4& lo, const uint4& hi, float (&v)[16]) {
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = elem_to_f32<T>(w[i] & 0xffffu);
    v[2 * i + 1] = elem_to_f32<T>(w[i] >> 16);
  }
}

// Launch bounds of the row-pair kernel.  The plain form runs at most 8 warps
// per CTA and keeps the next item's loads in flight (80 registers, 3+ CTAs
// per SM); the fused activations run up to 16 warps at 64 registers.
template <int ACT>
struct RowpairBounds {
  static constexpr int kThreads = ACT == 0 ? 256 : 512;
  static constexpr int kMinBlocks = ACT == 0 ? 3 : 2;
};

// rows_per_cta = 2 * row pairs.  Warp items are (row pair, group pair); the
// odd last row of the tensor is paired with itself and its B half dropped.
// Plain form: each warp loads its next item before it rotates the current
// one, so every warp keeps one item's loads in flight behind its arithmetic.
template <typename T, int ACT, bool INT4, bool STAGED_SCALE>
__global__ void __launch_bounds__(RowpairBounds<ACT>::kThreads, RowpairBounds<ACT>::kMinBlocks)
    convrot_rowpair_kernel(RowQuantParams p) {
  constexpr bool kPrefetch = ACT == kActNone;
  extern __shared__ __align__(16) unsigned char smem[];
  const int R = p.rows_per_cta;
  const int k = p.k;
  const int groups = k / kGroup;
  const int gpairs = (groups + 1) >> 1;
  const int warps = blockDim.x >> 5;
  uint32_t* rowbuf = reinterpret_cast<uint32_t*>(smem);
  uint64_t* tb_all = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(R / 2) * k * 4);
  unsigned int* row_amax = reinterpret_cast<unsigned int*>(tb_all + warps * 2 * 256);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int half = (tid >> 4) & 1;
  const int l = tid & 15;
  const int row0 = blockIdx.x * R;
  const int rows_here = min(R, p.rows - row0);
  const int pairs_here = (rows_here + 1) >> 1;
  const int in_width = ACT == kActSwiGLU ? 2 * k : k;
  const T* in = static_cast<const T*>(p.input);
  uint64_t* tb = tb_all + (warp * 2 + half) * 256;
  int lane_sw[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) lane_sw[c] = 4 * ((l >> 2) ^ c) + (l & 3);

  for (int r = tid; r < R; r += blockDim.x) row_amax[r] = 0u;
  __syncthreads();

  // (row pair, group pair) of this warp's item, advanced by `warps` items per
  // iteration without a division.
  const int items = pairs_here * gpairs;
  int ip = 0, igp = warp;
  while (igp >= gpairs) {
    igp -= gpairs;
    ++ip;
  }
  // Source of item (row pair ip_, group pair igp_) for this half-warp; an
  // inactive half (odd group count) re-reads the last group, an odd last row
  // its own row.
  auto item_src = [&](int ip_, int igp_, const T*& ra, const T*& rb, int& col_) {
    const int g_ = 2 * igp_ + half;
    ra = in + static_cast<int64_t>(row0 + 2 * ip_) * in_width;
    rb = 2 * ip_ + 1 < rows_here ? ra + in_width : ra;
    col_ = (g_ < groups ? g_ : groups - 1) * kGroup + 16 * l;
  };
  RawPair nxt;
  if (kPrefetch && warp < items) {
    const T* ra;
    const T* rb;
    int c;
    item_src(ip, igp, ra, rb, c);
    load_raw_pair(ra, rb, c, nxt);
  }
  for (int item = warp; item < items; item += warps) {
    const int rp = ip;
    const int g = 2 * igp + half;
    const T* row_a;
    const T* row_b;
    int col;
    item_src(ip, igp, row_a, row_b, col);
    igp += warps;
    while (igp >= gpairs) {
      igp -= gpairs;
      ++ip;
    }
    const bool active = g < groups;
    const bool has_b = 2 * rp + 1 < rows_here;
    float fa[16], fb[16];
    if constexpr (kPrefetch) {
      const RawPair cur = nxt;
      if (item + warps < items) {  // warp-uniform
        const T* ra;
        const T* rb;
        int c;
        item_src(ip, igp, ra, rb, c);
        load_raw_pair(ra, rb, c, nxt);
      }
      widen16<T>(cur.a0, cur.a1, fa);
      widen16<T>(cur.b0, cur.b1, fb);
    } else {
      load16<T, ACT>(row_a, k, col, fa);
      load16<T, ACT>(row_b, k, col, fb);
    }
    uint64_t v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = pk(fa[j], fb[j]);
    rotate_group_pair(v, tb, l);
    float am_a = 0.0f, am_b = 0.0f;
    // pair_swizzle(rp * k + g * 256 + l + 16 j), spelled out: the group
    // starts on line L0 (a multiple of 8), element l + 16 j sits on line
    // L0 + j / 2 in chunk l / 4 + 4 (j % 2), and f(line) = (j / 2) % 4 plus 4
    // times bit 3 of L0.  So the word is L0 * 32 + 32 (j / 2) + lane_sw[(j / 2)
    // % 4] + 16 ((j % 2) ^ b3), with lane_sw[c] = 4 ((l / 4) ^ c) + l % 4.
    const int line0 = (rp * k + g * kGroup) >> 5;
    const int b3 = (line0 >> 3) & 1;
    uint32_t* dst_even = rowbuf + line0 * 32 + 16 * b3;
    uint32_t* dst_odd = rowbuf + line0 * 32 + 16 * (b3 ^ 1);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      float a0, b0, a1, b1;
      unpk(v[j], a0, b0);
      unpk(v[j + 1], a1, b1);
      am_a = max3f(am_a, fabsf(a0), fabsf(a1));
      am_b = max3f(am_b, fabsf(b0), fabsf(b1));
      if (active) {
        const int off = 32 * (j >> 1) + lane_sw[(j >> 1) & 3];
        dst_even[off] = pack2_elem<T>(a0, b0);
        dst_odd[off] = pack2_elem<T>(a1, b1);
      }
    }
    // Non-negative floats order like their bit patterns; both half-warps
    // hold the same row pair, so one warp-wide maximum serves both.
    const uint32_t wa = warp_max_u32(active ? __float_as_uint(am_a) : 0u);
    const uint32_t wb = warp_max_u32(active ? __float_as_uint(am_b) : 0u);
    if (tid % 32 == 0) {
      atomicMax(&row_amax[2 * rp], wa);
      if (has_b) atomicMax(&row_amax[2 * rp + 1], wb);
    }
  }
  __syncthreads();
  float* row_rcp = reinterpret_cast<float*>(row_amax);
  for (int r = tid; r < rows_here; r += blockDim.x) {
    const float scale = row_scale_from_amax<T, INT4, STAGED_SCALE>(__uint_as_float(row_amax[r]));
    p.scales[row0 + r] = scale;
    row_rcp[r] = INT4 ? __frcp_rn(scale) : __frcp_rn(round_to_elem<T>(scale));
  }
  __syncthreads();

  // Phase 2: sixteen columns of one row pair per thread per iteration.
  const int cpr = k / 16;
  const int chunks = pairs_here * cpr;
  int cr = 0, cc = tid;
  while (cc >= cpr) {
    cc -= cpr;
    ++cr;
  }
  for (int c = tid; c < chunks; c += blockDim.x) {
    const int rp = cr;
    const int col = cc * 16;
    cc += blockDim.x;
    while (cc >= cpr) {
      cc -= cpr;
      ++cr;
    }
    const bool has_b = 2 * rp + 1 < rows_here;
    const float rcp_a = row_rcp[2 * rp];
    const float rcp_b = has_b ? row_rcp[2 * rp + 1] : rcp_a;
    const int xb = rp * k + col;
    const uint64_t rcp2 = pk(rcp_a, rcp_b);
    const int64_t row_a = row0 + 2 * rp;
    uint32_t oa[4], ob[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint4 q = *reinterpret_cast<const uint4*>(rowbuf + pair_swizzle(xb + 4 * s));
      if constexpr (INT4) quantize4_pair_i4<T>(q, rcp2, oa[s], ob[s]);
      else quantize4_pair_i8<T>(q, rcp2, oa[s], ob[s]);
    }
    if constexpr (INT4) {
      const uint2 a = make_uint2(oa[0] | (oa[1] << 16), oa[2] | (oa[3] << 16));
      const uint2 b = make_uint2(ob[0] | (ob[1] << 16), ob[2] | (ob[3] << 16));
      int8_t* dst = p.output + row_a * (k / 2) + col / 2;
      *reinterpret_cast<uint2*>(dst) = a;
      if (has_b) *reinterpret_cast<uint2*>(dst + k / 2) = b;
    } else {
      int8_t* dst = p.output + row_a * k + col;
      *reinterpret_cast<uint4*>(dst) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
      if (has_b) *reinterpret_cast<uint4*>(dst + k) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
    }
  }
}

// Staged form, pass 1: rotate, write the rotated T values to the global
// scratch and one fp32 absmax per (row, group) (convrot_quant.cu:158-211).
template <typename T, int ACT>
__global__ void __launch_bounds__(256) convrot_staged_rotate_kernel(RowQuantParams p) {
  __shared__ __align__(16) float tbuf_all[16 * kTbufStride];
  const int k = p.k;
  const int groups = k / kGroup;
  const int64_t total = static_cast<int64_t>(p.rows) * groups;
  const int hw = threadIdx.x >> 4;
  const int l = threadIdx.x & 15;
  float* tbuf = tbuf_all + hw * kTbufStride;
  const int in_width = ACT == kActSwiGLU ? 2 * k : k;
  const T* in = static_cast<const T*>(p.input);
  uint16_t* rot = static_cast<uint16_t*>(p.rotated);
  // Two items per warp per iteration (see convrot_rowbuffer_kernel).
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * 16 + 2 * (hw >> 1); base < total;
       base += static_cast<int64_t>(gridDim.x) * 16) {
    const int64_t item = base + (hw & 1);
    const bool active = item < total;
    const int64_t row = active ? item / groups : 0;
    const int g = active ? static_cast<int>(item - row * groups) : 0;
    float v[16];
    load16<T, ACT>(in + row * in_width, k, g * kGroup + 16 * l, v);
    rotate_group(v, tbuf, l);
    float amax = 0.0f;
    uint16_t* dst = rot + row * k + g * kGroup + l;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      amax = fmaxf(amax, fabsf(v[j]));
      if (active) dst[16 * j] = static_cast<uint16_t>(f32_to_elem_bits<T>(v[j]));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o, 16));
    if (active && l == 0) p.partial_absmax[row * groups + g] = amax;
  }
}

// Staged form, pass 2: per row, reduce the partial absmax and quantize from
// the rotated scratch (convrot_quant.cu:213-291).  One CTA per row.
template <typename T, bool INT4>
__global__ void __launch_bounds__(256) convrot_staged_quant_kernel(RowQuantParams p) {
  __shared__ float warp_max_s[8];
  const int k = p.k;
  const int groups = k / kGroup;
  const int64_t row = blockIdx.x;
  float amax = 0.0f;
  for (int g = threadIdx.x; g < groups; g += blockDim.x)
    amax = fmaxf(amax, p.partial_absmax[row * groups + g]);
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) warp_max_s[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.0f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) amax = fmaxf(amax, warp_max_s[w]);
  const float scale = row_scale_from_amax<T, INT4, true>(amax);
  const float rcp_rounded = __frcp_rn(round_to_elem<T>(scale));
  const float inv_scale = __frcp_rn(scale);
  if (threadIdx.x == 0) p.scales[row] = scale;
  const uint16_t* rot = static_cast<const uint16_t*>(p.rotated) + row * k;
  for (int col = threadIdx.x * 16; col < k; col += blockDim.x * 16) {
    const uint4* src = reinterpret_cast<const uint4*>(rot + col);
    uint4 a = __ldg(src), b = __ldg(src + 1);
    uint32_t h[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    int8_t* dst = INT4 ? p.output + row * (k / 2) + col / 2 : p.output + row * k + col;
    quantize16_store<T, INT4>(h, rcp_rounded, inv_scale, dst);
  }
}

struct RowbufferLaunch {
  int rows_per_cta;
  int threads;
  size_t smem;
};

RowbufferLaunch plan_rowbuffer(int k) {
  const int groups = k / kGroup;
  int R = groups >= 32 ? 1 : 32 / groups;
  while (R > 1 && static_cast<size_t>(R) * k * 2 > 64 * 1024) R >>= 1;
  const int items = R * groups;
  int halfwarps = items < 32 ? items : 32;
  int threads = halfwarps * 16;
  threads = (threads + 31) / 32 * 32;
  halfwarps = threads / 16;
  RowbufferLaunch L;
  L.rows_per_cta = R;
  L.threads = threads;
  L.smem = static_cast<size_t>(R) * k * 2 + static_cast<size_t>(halfwarps) * kTbufStride * 4 +
           static_cast<size_t>(R) * 4;
  return L;
}

// Row-pair kernel plan: enough row pairs per CTA for about max_warps warp
// items, warps balanced over the items, shared memory = the bf16x2 row-pair
// buffer + 4 KB of transpose buffers per warp + the row absmax words.
// Returns false when that does not fit in one CTA's shared memory.  The plain
// rotation runs best with up to 8 warps per CTA (more, smaller CTAs per SM
// overlap one CTA's loads with another's arithmetic: 380 vs 407 us at
// 75600 x 5120 on a B200); the fused activations, whose tanhf / expf make
// them arithmetic-bound, with up to 16.
bool plan_rowpair(int k, RowbufferLaunch& L, int max_warps) {
  const int groups = k / kGroup;
  const int gpairs = (groups + 1) / 2;
  int pairs = gpairs >= max_warps ? 1 : max_warps / gpairs;
  while (pairs > 1 && static_cast<size_t>(pairs) * k * 4 > 64 * 1024) pairs >>= 1;
  const int items = pairs * gpairs;
  const int iters = (items + max_warps - 1) / max_warps;
  const int warps = (items + iters - 1) / iters;
  L.rows_per_cta = 2 * pairs;
  L.threads = warps * 32;
  L.smem = static_cast<size_t>(pairs) * k * 4 + static_cast<size_t>(warps) * 4096 +
           static_cast<size_t>(2 * pairs) * 4;
  return L.smem <= 200 * 1024;
}

template <typename T, int ACT, bool INT4, bool STAGED_SCALE>
void launch_rowbuffer_t(const void* input, int rows, int k, int8_t* out, float* scales,
                        cudaStream_t stream) {
  RowbufferLaunch P;
  if (plan_rowpair(k, P, ACT == kActNone ? 8 : 16)) {
    RowQuantParams p{};
    p.input = input;
    p.output = out;
    p.scales = scales;
    p.rows = rows;
    p.k = k;
    p.rows_per_cta = P.rows_per_cta;
    auto kernel = convrot_rowpair_kernel<T, ACT, INT4, STAGED_SCALE>;
    if (P.smem > 48 * 1024) {
      TB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(P.smem)));
    }
    const int grid = (rows + P.rows_per_cta - 1) / P.rows_per_cta;
    kernel<<<grid, P.threads, P.smem, stream>>>(p);
    TB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  RowbufferLaunch L = plan_rowbuffer(k);
  RowQuantParams p{};
  p.input = input;
  p.output = out;
  p.scales = scales;
  p.rows = rows;
  p.k = k;
  p.rows_per_cta = L.rows_per_cta;
  auto kernel = convrot_rowbuffer_kernel<T, ACT, INT4, STAGED_SCALE>;
  if (L.smem > 48 * 1024) {
    TB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L.smem)));
  }
  const int grid = (rows + L.rows_per_cta - 1) / L.rows_per_cta;
  kernel<<<grid, L.threads, L.smem, stream>>>(p);
  TB_CUDA_CHECK(cudaGetLastError());
}

template <typename T, int ACT, bool INT4>
void launch_staged_t(const void* input, int rows, int k, void* rotated, float* partial,
                     int8_t* out, float* scales, cudaStream_t stream) {
  RowQuantParams p{};
  p.input = input;
  p.output = out;
  p.scales = scales;
  p.rotated = rotated;
  p.partial_absmax = partial;
  p.rows = rows;
  p.k = k;
  const int64_t items = static_cast<int64_t>(rows) * (k / kGroup);
  int64_t blocks = (items + 15) / 16;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  convrot_staged_rotate_kernel<T, ACT><<<static_cast<int>(blocks), 256, 0, stream>>>(p);
  TB_CUDA_CHECK(cudaGetLastError());
  convrot_staged_quant_kernel<T, INT4><<<rows, 256, 0, stream>>>(p);
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

// The kernels move 16 bytes per load/store (input, codes, rotated scratch)
// and 4 bytes per scale or partial absmax; a sub-allocated pointer off those
// boundaries would be a misaligned access on the device, so it is rejected
// here, before anything is launched.
void convrot_check_pointers(const void* input, const void* out, const float* scales, int staged,
                            const void* rotated, const float* partial) {
  TB_REQUIRE(reinterpret_cast<uintptr_t>(input) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(out) % 16 == 0,
             "ConvRot input and output must be 16-byte aligned");
  TB_REQUIRE(reinterpret_cast<uintptr_t>(scales) % 4 == 0,
             "ConvRot scales must be 4-byte aligned");
  TB_REQUIRE(!staged || (reinterpret_cast<uintptr_t>(rotated) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(partial) % 4 == 0),
             "staged ConvRot scratch must be 16-byte (rotated) and 4-byte (partial) aligned");
}

// Shared dispatcher for both forms.  dtype: TB_DTYPE_BF16 or TB_DTYPE_F16
// (fp16 only for the staged form, as in the reference).
void convrot_quantize_impl(const void* input, int dtype, int64_t rows64, int64_t k64, int act,
                           int int4, int staged, void* rotated, float* partial, int8_t* out,
                           float* scales, cudaStream_t stream) {
  TB_REQUIRE(rows64 > 0 && k64 > 0 && k64 % kGroup == 0,
             "ConvRot width must be positive and divisible by 256");
  TB_REQUIRE(rows64 <= INT32_MAX && k64 <= INT32_MAX,
             "ConvRot dimensions exceed the CUDA kernel range");
  TB_REQUIRE(act >= 0 && act <= 2, "ConvRot activation must be 0 (none), 1 (SwiGLU) or 2 (GELU)");
  TB_REQUIRE(dtype == TB_DTYPE_BF16 || (staged && dtype == TB_DTYPE_F16),
             "ConvRot input must be bfloat16 (float16 only for the staged form)");
  TB_REQUIRE(input != nullptr && out != nullptr && scales != nullptr,
             "ConvRot input, output and scales must be non-null");
  const int rows = static_cast<int>(rows64), k = static_cast<int>(k64);
  TB_REQUIRE(!staged || (rotated != nullptr && partial != nullptr),
             "staged ConvRot requires rotated and partial_absmax scratch");
  convrot_check_pointers(input, out, scales, staged, rotated, partial);
  TB_REQUIRE(static_cast<size_t>(k) * 2 + 32 * kTbufStride * 4 + 64 <= 227 * 1024 || staged,
             "ConvRot row does not fit in shared memory; use the staged form");

#define TB_CONVROT_CASE(T, ACT)                                                             \
  if (staged) {                                                                             \
    if (int4) launch_staged_t<T, ACT, true>(input, rows, k, rotated, partial, out, scales,  \
                                            stream);                                        \
    else launch_staged_t<T, ACT, false>(input, rows, k, rotated, partial, out, scales,      \
                                        stream);                                            \
  } else {                                                                                  \
    if (int4) launch_rowbuffer_t<T, ACT, true, false>(input, rows, k, out, scales, stream); \
    else launch_rowbuffer_t<T, ACT, false, false>(input, rows, k, out, scales, stream);     \
  }
  if (dtype == TB_DTYPE_BF16) {
    if (act == kActNone) { TB_CONVROT_CASE(__nv_bfloat16, kActNone) }
    else if (act == kActSwiGLU) { TB_CONVROT_CASE(__nv_bfloat16, kActSwiGLU) }
    else { TB_CONVROT_CASE(__nv_bfloat16, kActGelu) }
  } else {
    if (act == kActNone) { TB_CONVROT_CASE(__half, kActNone) }
    else if (act == kActSwiGLU) { TB_CONVROT_CASE(__half, kActSwiGLU) }
    else { TB_CONVROT_CASE(__half, kActGelu) }
  }
#undef TB_CONVROT_CASE
}

}  // namespace tb

// ------------------------------------------------------------------------
// Allocation-free staged quantizer.
//
// Some callers cannot allocate device memory at the point where they quantize:
// a host application whose memory manager owns every VRAM byte and forbids
// untracked allocations, code that must not stall on cudaMalloc's implicit
// device synchronisation, or a runtime that has already handed its memory to
// a pool.  For them the staged SwiGLU INT8 quantizer below keeps its scratch
// (the rotated rows and the per-group absmax) in a fixed array that is part of
// this library's device image: it is reserved on every GPU that loads the
// library and held until the process exits.  The caller passes only inputs
// and outputs.
namespace tb {
namespace {

// 16 MiB of scratch: rotated values first, then the fp32 partial absmax.
constexpr size_t kNoAllocScratchBytes = 16u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
// Device address of the array per device ordinal, with the id of the context
// it was looked up in.  A cudaDeviceReset (or any new primary context) loads
// the module again, possibly at another address, and gets a new context id,
// so a changed id triggers a fresh lookup.
struct NoAllocSlot {
  unsigned long long ctx_id;
  void* addr;
};
NoAllocSlot g_noalloc_slot[64] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Id of the calling thread's current context (0 when none is current yet).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  static CtxGetIdFn get_id = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetIdFn>(p);
  }();
  if (get_current == nullptr || get_id == nullptr)
    throw Error(TB_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Looks up the device address of the scratch array for the current device,
// once per device and context.  The array's name is only a host-side
// stand-in; kernels must be given this address.
void* noalloc_scratch_for_current_device() {
  int dev = 0;
  TB_CUDA_CHECK(cudaGetDevice(&dev));
  TB_REQUIRE(dev >= 0 && dev < 64, "device ordinal out of range for the scratch table");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoAllocSlot& slot = g_noalloc_slot[dev];
  const unsigned long long id = current_context_id();
  if (slot.addr == nullptr || id == 0 || id != slot.ctx_id) {
    void* ptr = nullptr;
    TB_CUDA_CHECK(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));  // makes the context current
    slot.addr = ptr;
    slot.ctx_id = current_context_id();
  }
  return slot.addr;
}

}  // namespace
}  // namespace tb

extern "C" int tb_swiglu_int8_convrot_quantize_noalloc(const void* input, int dtype, int64_t rows,
                                                       int64_t hidden, int8_t* output,
                                                       float* scales, tb_stream_t stream) {
  return tb::guarded([&] {
    TB_REQUIRE(input != nullptr && output != nullptr && scales != nullptr,
               "input, output and scales must be CUDA tensors");
    TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16,
               "input must be float16 or bfloat16");
    TB_REQUIRE(rows > 0, "staged ConvRot requires at least one row");
    TB_REQUIRE(hidden > 0 && hidden % 256 == 0,
               "activated SwiGLU width must be positive and divisible by 256");
    TB_REQUIRE(rows <= INT32_MAX && hidden <= INT32_MAX,
               "staged ConvRot dimensions exceed the CUDA kernel range");
    // Scratch: rotated [rows, hidden] (2 bytes each, 256-byte aligned), then
    // partial absmax [rows, hidden / 256] fp32.
    const uint64_t rotated_bytes =
        (static_cast<uint64_t>(rows) * static_cast<uint64_t>(hidden) * 2 + 255) & ~uint64_t{255};
    const uint64_t partial_bytes = static_cast<uint64_t>(rows) * static_cast<uint64_t>(hidden / 256) * 4;
    TB_REQUIRE(rotated_bytes + partial_bytes <= tb::kNoAllocScratchBytes,
               "problem too large for the allocation-free quantizer: rows * hidden * 2 + "
               "rows * hidden / 64 bytes must fit in its 16 MiB scratch; split the rows or use "
               "tb_swiglu_int8_convrot_quantize with caller-owned scratch");
    tb::convrot_check_pointers(input, output, scales, 0, nullptr, nullptr);
    tb::require_sm100();
    unsigned char* scratch = static_cast<unsigned char*>(tb::noalloc_scratch_for_current_device());
    // Nothing in the scratch has to start at zero: the first pass writes every
    // rotated value and every partial absmax before the second pass reads them.
    tb::convrot_quantize_impl(input, dtype, rows, hidden, /*act=*/1, /*int4=*/0, /*staged=*/1,
                              scratch, reinterpret_cast<float*>(scratch + rotated_bytes), output,
                              scales, static_cast<cudaStream_t>(stream));
  });
}
