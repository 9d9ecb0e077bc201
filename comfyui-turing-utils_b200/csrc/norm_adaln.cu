// Norm + AdaLN fusions of the DiT block (kernel/csrc/turing/segmented_rms_adaln.cu):
//
//   segmented RMSNorm + AdaLN (:135-235): for token row r with modulation row
//     m(r) (the [start, stop, row] segment that holds r; 0 when none does or
//     the row is out of range),
//       inv = rsqrt(mean_k(x[r,k]^2) + eps),
//       out[r,k] = T(x[r,k] * inv * w[k] * (1 + scale[m,k]) + shift[m,k]);
//   LayerNorm + AdaLN (:237-306): per row of [batch, sequence, hidden], with
//     the modulation step of the token (sequence split into modulation_steps
//     groups of ceil(sequence / steps) tokens),
//       n = T((x - mean) * rsqrt(var + eps)),  mult = T(1 + scale),
//       out = T(float(n) * float(mult) + shift).
// Statistics are fp32.  LayerNorm rows of 256 * NV 16-bit values (NV <= 24)
// are handled one per warp (layer_norm_adaln_warp_kernel).  Otherwise
// one CTA per row: the row is read from HBM once into
// shared memory (16-byte vectors when the pointers and width allow), reduced
// by warp shuffles, and the output is formed from the staged copy, so each
// element crosses HBM once in each direction.  LayerNorm takes its mean and
// variance in two passes over the staged row (the reference uses a
// single-pass Welford combine; both are fp32 and agree to rounding).
#include <cmath>

#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

constexpr int kNormThreads = 256;
constexpr int kNormWarps = kNormThreads / 32;
// Rows wider than this many bytes are not staged; the second pass then
// re-reads the row (from L2) instead.
constexpr int kMaxStagedBytes = 96 * 1024;

template <typename T>
__device__ __forceinline__ float ld_f(T v);
template <>
__device__ __forceinline__ float ld_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float ld_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T st_f(float v);
template <>
__device__ __forceinline__ float st_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half st_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 st_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Sum over the CTA; every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  __syncthreads();  // red may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormWarps; ++i) t += red[i];
  return t;
}

// Row loader: element k of the row, from the staged copy when there is one.
template <typename T>
struct Row {
  const T* g;   // global row
  const T* s;   // staged row (or null)
  __device__ __forceinline__ float at(int k) const { return ld_f(s ? s[k] : g[k]); }
};

// Copies the row into shared memory with 16-byte vectors (vec) or elements.
template <typename T>
__device__ __forceinline__ void stage_row(const T* g, T* s, int hidden, bool vec) {
  if (vec) {
    constexpr int kW = 16 / sizeof(T);
    const uint4* gv = reinterpret_cast<const uint4*>(g);
    uint4* sv = reinterpret_cast<uint4*>(s);
    for (int i = threadIdx.x; i < hidden / kW; i += kNormThreads) sv[i] = __ldg(gv + i);
  } else {
    for (int i = threadIdx.x; i < hidden; i += kNormThreads) s[i] = g[i];
  }
  __syncthreads();
}

// Modulation row of token `row`: the segment [start, stop) that holds it
// (segments sorted by stop), else -1 (segmented_rms_adaln.cu:115-132).
__device__ __forceinline__ int segment_row(const int* seg, int count, int row) {
  int lo = 0, hi = count;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (row < __ldg(seg + 3 * mid + 1)) hi = mid;
    else lo = mid + 1;
  }
  if (lo >= count || row < __ldg(seg + 3 * lo)) return -1;
  return __ldg(seg + 3 * lo + 2);
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rms_adaln_kernel(
    const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ scale,
    const T* __restrict__ shift, const int* __restrict__ segments, T* __restrict__ out,
    int hidden, int param_rows, int64_t scale_stride, int64_t shift_stride, int seg_count,
    float eps, int staged, int vec) {
  extern __shared__ __align__(16) unsigned char norm_smem[];
  __shared__ float red[kNormWarps];
  const int row = blockIdx.x;
  const T* xr = x + static_cast<int64_t>(row) * hidden;
  T* srow = staged ? reinterpret_cast<T*>(norm_smem) : nullptr;
  if (staged) stage_row(xr, srow, hidden, vec != 0);
  const Row<T> r{xr, srow};
  float ss = 0.0f;
  for (int k = threadIdx.x; k < hidden; k += kNormThreads) {
    const float v = r.at(k);
    ss += v * v;
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
  int m = segment_row(segments, seg_count, row);
  if (m < 0 || m >= param_rows) m = 0;
  const T* sc = scale + static_cast<int64_t>(m) * scale_stride;
  const T* sh = shift + static_cast<int64_t>(m) * shift_stride;
  T* orow = out + static_cast<int64_t>(row) * hidden;
  for (int k = threadIdx.x; k < hidden; k += kNormThreads) {
    const float normalized = r.at(k) * inv;
    const float result = normalized * ld_f(__ldg(w + k)) * (1.0f + ld_f(__ldg(sc + k))) +
                         ld_f(__ldg(sh + k));
    orow[k] = st_f<T>(result);
  }
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) layer_norm_adaln_kernel(
    const T* __restrict__ x, const T* __restrict__ scale, const T* __restrict__ shift,
    T* __restrict__ out, int sequence, int hidden, int steps, float eps, int staged, int vec) {
  extern __shared__ __align__(16) unsigned char norm_smem[];
  __shared__ float red[kNormWarps];
  const int row = blockIdx.x;
  const int batch = row / sequence;
  const int token = row - batch * sequence;
  int mod_token = 0;
  if (steps > 1) {
    const int per = (sequence + steps - 1) / steps;  // tokens per modulation step
    mod_token = min(token / max(per, 1), steps - 1);
  }
  const T* xr = x + static_cast<int64_t>(row) * hidden;
  T* srow = staged ? reinterpret_cast<T*>(norm_smem) : nullptr;
  if (staged) stage_row(xr, srow, hidden, vec != 0);
  const Row<T> r{xr, srow};
  float s = 0.0f;
  for (int k = threadIdx.x; k < hidden; k += kNormThreads) s += r.at(k);
  const float mean = block_sum(s, red) / static_cast<float>(hidden);
  float q = 0.0f;
  for (int k = threadIdx.x; k < hidden; k += kNormThreads) {
    const float d = r.at(k) - mean;
    q += d * d;
  }
  const float var = block_sum(q, red) / static_cast<float>(hidden);
  const float inv_std = rsqrtf(var + eps);
  const int64_t mod = (static_cast<int64_t>(batch) * steps + mod_token) * hidden;
  T* orow = out + static_cast<int64_t>(row) * hidden;
  for (int k = threadIdx.x; k < hidden; k += kNormThreads) {
    const T n = st_f<T>((r.at(k) - mean) * inv_std);
    const T mult = st_f<T>(1.0f + ld_f(__ldg(scale + mod + k)));
    const float result = ld_f(n) * ld_f(mult) + ld_f(__ldg(shift + mod + k));
    orow[k] = st_f<T>(result);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Warp-per-row form for 16-bit rows of hidden = 256 * NV: lane l loads the
// 16-byte chunks l, l + 32, ... of the row (all in flight at once) and parks
// them in its warp's slice of shared memory, so the row crosses HBM once in
// each direction with no CTA barrier; statistics by warp butterflies.  Same formula as
// layer_norm_adaln_kernel (two fp32 passes, then
// out = T(float(T((x - mean) * inv_std)) * float(T(1 + scale)) + shift)); only
// the summation order of the mean and variance differs.
template <typename T>
__device__ __forceinline__ float half_bits_to_f32(uint32_t bits16) {
  return ld_f(__ushort_as_half(static_cast<unsigned short>(bits16)));
}
template <>
__device__ __forceinline__ float half_bits_to_f32<__nv_bfloat16>(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = half_bits_to_f32<T>(w[i] & 0xffffu);
    f[2 * i + 1] = half_bits_to_f32<T>(w[i] >> 16);
  }
}

template <typename T>
__device__ __forceinline__ uint32_t bits_of(T v) {
  return static_cast<uint32_t>(*reinterpret_cast<const unsigned short*>(&v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kWarpRowsPerCta = 8;

template <typename T, int NV>
__global__ void __launch_bounds__(kWarpRowsPerCta * 32, 2) layer_norm_adaln_warp_kernel(
    const T* __restrict__ x, const T* __restrict__ scale, const T* __restrict__ shift,
    T* __restrict__ out, int rows, int sequence, int hidden, int steps, float eps) {
  extern __shared__ __align__(16) unsigned char norm_smem[];
  const int w = threadIdx.x >> 5;
  const int row = blockIdx.x * kWarpRowsPerCta + w;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // warp-uniform
  const int batch = row / sequence;
  const int token = row - batch * sequence;
  int mod_token = 0;
  if (steps > 1) {
    const int per = (sequence + steps - 1) / steps;
    mod_token = min(token / max(per, 1), steps - 1);
  }
  // The warp's row: all NV loads of a lane in flight at once, then parked in
  // this warp's slice of shared memory (lane-owned chunks, no other lane
  // reads them, so no barrier beyond the warp's own program order).
  uint4* srow = reinterpret_cast<uint4*>(norm_smem) + static_cast<size_t>(w) * NV * 32;
  {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * hidden);
    uint4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = __ldg(xr + lane + 32 * i);
#pragma unroll
    for (int i = 0; i < NV; ++i) srow[lane + 32 * i] = v[i];
  }
  float s = 0.0f;
#pragma unroll 4
  for (int i = 0; i < NV; ++i) {
    float f[8];
    unpack8<T>(srow[lane + 32 * i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) s += f[k];
  }
  const float mean = warp_sum(s) / static_cast<float>(hidden);
  float q = 0.0f;
#pragma unroll 4
  for (int i = 0; i < NV; ++i) {
    float f[8];
    unpack8<T>(srow[lane + 32 * i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float d = f[k] - mean;
      q += d * d;
    }
  }
  const float var = warp_sum(q) / static_cast<float>(hidden);
  const float inv_std = rsqrtf(var + eps);
  const int64_t mod = (static_cast<int64_t>(batch) * steps + mod_token) * hidden;
  const uint4* scr = reinterpret_cast<const uint4*>(scale + mod);
  const uint4* shr = reinterpret_cast<const uint4*>(shift + mod);
  uint4* orow = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * hidden);
#pragma unroll 4
  for (int i = 0; i < NV; ++i) {
    float f[8], sc[8], sh[8];
    unpack8<T>(srow[lane + 32 * i], f);
    unpack8<T>(__ldg(scr + lane + 32 * i), sc);
    unpack8<T>(__ldg(shr + lane + 32 * i), sh);
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      uint32_t pair = 0u;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const T n = st_f<T>((f[k + e] - mean) * inv_std);
        const T mult = st_f<T>(1.0f + sc[k + e]);
        const float result = ld_f(n) * ld_f(mult) + sh[k + e];
        pair |= bits_of(st_f<T>(result)) << (16 * e);
      }
      o[k / 2] = pair;
    }
    orow[lane + 32 * i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <typename T, int NV>
void launch_ln_warp(const void* x, const void* scale, const void* shift, void* out, int rows,
                    int seq, int hidden, int steps, float eps, cudaStream_t stream) {
  const int grid = (rows + kWarpRowsPerCta - 1) / kWarpRowsPerCta;
  const size_t smem = static_cast<size_t>(kWarpRowsPerCta) * NV * 32 * 16;
  auto kern = layer_norm_adaln_warp_kernel<T, NV>;
  if (smem > 48 * 1024)
    TB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
  kern<<<grid, kWarpRowsPerCta * 32, smem, stream>>>(
      static_cast<const T*>(x), static_cast<const T*>(scale), static_cast<const T*>(shift),
      static_cast<T*>(out), rows, seq, hidden, steps, eps);
  TB_CUDA_CHECK(cudaGetLastError());
}

// The warp-per-row form for hidden = 256 * NV, NV in {4, 8, 12, 16, 20,
// 24} (1024 ... 6144 columns), 16-bit types and 16-byte aligned tensors;
// false when it does not apply.
template <typename T>
bool try_ln_warp(const void* x, const void* scale, const void* shift, void* out, int rows,
                 int seq, int hidden, int steps, float eps, cudaStream_t stream) {
  if (hidden % 256 != 0 || !aligned16(x) || !aligned16(scale) || !aligned16(shift) ||
      !aligned16(out))
    return false;
  switch (hidden / 256) {
    case 4: launch_ln_warp<T, 4>(x, scale, shift, out, rows, seq, hidden, steps, eps, stream); return true;
    case 8: launch_ln_warp<T, 8>(x, scale, shift, out, rows, seq, hidden, steps, eps, stream); return true;
    case 12: launch_ln_warp<T, 12>(x, scale, shift, out, rows, seq, hidden, steps, eps, stream); return true;
    case 16: launch_ln_warp<T, 16>(x, scale, shift, out, rows, seq, hidden, steps, eps, stream); return true;
    case 20: launch_ln_warp<T, 20>(x, scale, shift, out, rows, seq, hidden, steps, eps, stream); return true;
    case 24: launch_ln_warp<T, 24>(x, scale, shift, out, rows, seq, hidden, steps, eps, stream); return true;
    default: return false;
  }
}

int elem_bytes(int dtype) { return dtype == TB_DTYPE_F32 ? 4 : 2; }


template <typename T, typename K, typename... Args>
void launch_with_smem(K kern, int rows, size_t smem, cudaStream_t stream, Args... args) {
  if (smem > 48 * 1024)
    TB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
  kern<<<rows, kNormThreads, smem, stream>>>(args...);
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace
}  // namespace tb

using tb::guarded;

extern "C" int tb_segmented_rms_adaln(const void* input, const void* weight, const void* scale,
                                      const void* shift, const int32_t* segments, void* output,
                                      int64_t rows, int64_t hidden, int64_t modulation_rows,
                                      int64_t scale_stride, int64_t shift_stride,
                                      int64_t segment_count, int dtype, float epsilon,
                                      tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(input && weight && scale && shift && segments && output,
               "all segmented RMSNorm+AdaLN tensors must use the same CUDA device");
    TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16 || dtype == TB_DTYPE_F32,
               "segmented RMSNorm+AdaLN requires float16, bfloat16, or float32 input");
    TB_REQUIRE(rows > 0 && hidden > 0, "segmented RMSNorm+AdaLN input dimensions must be positive");
    TB_REQUIRE(modulation_rows > 0, "scale must be [modulation_rows, hidden]");
    TB_REQUIRE(segment_count > 0, "segments must contain at least one row");
    TB_REQUIRE(rows <= INT32_MAX && hidden <= INT32_MAX && modulation_rows <= INT32_MAX &&
                   segment_count <= INT32_MAX,
               "segmented RMSNorm+AdaLN dimensions exceed the CUDA kernel range");
    TB_REQUIRE(std::isfinite(epsilon) && epsilon > 0.0f,
               "RMSNorm epsilon must be finite and positive");
    tb::require_sm100();
    const int eb = tb::elem_bytes(dtype);
    const size_t row_bytes = static_cast<size_t>(hidden) * eb;
    const int staged = row_bytes <= static_cast<size_t>(tb::kMaxStagedBytes);
    const int vec = staged && (row_bytes % 16 == 0) && tb::aligned16(input);
    const size_t smem = staged ? (row_bytes + 15) / 16 * 16 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int r = static_cast<int>(rows), hd = static_cast<int>(hidden);
    const int pr = static_cast<int>(modulation_rows), sc = static_cast<int>(segment_count);
    if (dtype == TB_DTYPE_BF16) {
      using T = __nv_bfloat16;
      tb::launch_with_smem<T>(tb::rms_adaln_kernel<T>, r, smem, s, static_cast<const T*>(input),
                              static_cast<const T*>(weight), static_cast<const T*>(scale),
                              static_cast<const T*>(shift), segments, static_cast<T*>(output), hd,
                              pr, scale_stride, shift_stride, sc, epsilon, staged, vec);
    } else if (dtype == TB_DTYPE_F16) {
      using T = __half;
      tb::launch_with_smem<T>(tb::rms_adaln_kernel<T>, r, smem, s, static_cast<const T*>(input),
                              static_cast<const T*>(weight), static_cast<const T*>(scale),
                              static_cast<const T*>(shift), segments, static_cast<T*>(output), hd,
                              pr, scale_stride, shift_stride, sc, epsilon, staged, vec);
    } else {
      using T = float;
      tb::launch_with_smem<T>(tb::rms_adaln_kernel<T>, r, smem, s, static_cast<const T*>(input),
                              static_cast<const T*>(weight), static_cast<const T*>(scale),
                              static_cast<const T*>(shift), segments, static_cast<T*>(output), hd,
                              pr, scale_stride, shift_stride, sc, epsilon, staged, vec);
    }
  });
}

extern "C" int tb_layer_norm_adaln(const void* input, const void* scale, const void* shift,
                                   void* output, int64_t batch, int64_t sequence, int64_t hidden,
                                   int64_t modulation_steps, int dtype, float epsilon,
                                   tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(input && scale && shift && output,
               "LayerNorm+AdaLN tensors must use the same CUDA device");
    TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16 || dtype == TB_DTYPE_F32,
               "LayerNorm+AdaLN requires float16, bfloat16, or float32 input");
    TB_REQUIRE(batch > 0 && sequence > 0 && hidden > 0 && modulation_steps > 0,
               "LayerNorm+AdaLN dimensions must be positive");
    TB_REQUIRE(batch * sequence <= INT32_MAX && hidden <= INT32_MAX &&
                   modulation_steps <= INT32_MAX,
               "LayerNorm+AdaLN dimensions exceed the CUDA kernel range");
    TB_REQUIRE(std::isfinite(epsilon) && epsilon > 0.0f,
               "LayerNorm epsilon must be finite and positive");
    tb::require_sm100();
    const int eb = tb::elem_bytes(dtype);
    const size_t row_bytes = static_cast<size_t>(hidden) * eb;
    const int staged = row_bytes <= static_cast<size_t>(tb::kMaxStagedBytes);
    const int vec = staged && (row_bytes % 16 == 0) && tb::aligned16(input);
    const size_t smem = staged ? (row_bytes + 15) / 16 * 16 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int rows = static_cast<int>(batch * sequence);
    const int seq = static_cast<int>(sequence), hd = static_cast<int>(hidden);
    const int steps = static_cast<int>(modulation_steps);
    if (dtype == TB_DTYPE_BF16 &&
        tb::try_ln_warp<__nv_bfloat16>(input, scale, shift, output, rows, seq, hd, steps,
                                       epsilon, s))
      return;
    if (dtype == TB_DTYPE_F16 &&
        tb::try_ln_warp<__half>(input, scale, shift, output, rows, seq, hd, steps, epsilon, s))
      return;
    if (dtype == TB_DTYPE_BF16) {
      using T = __nv_bfloat16;
      tb::launch_with_smem<T>(tb::layer_norm_adaln_kernel<T>, rows, smem, s,
                              static_cast<const T*>(input), static_cast<const T*>(scale),
                              static_cast<const T*>(shift), static_cast<T*>(output), seq, hd,
                              steps, epsilon, staged, vec);
    } else if (dtype == TB_DTYPE_F16) {
      using T = __half;
      tb::launch_with_smem<T>(tb::layer_norm_adaln_kernel<T>, rows, smem, s,
                              static_cast<const T*>(input), static_cast<const T*>(scale),
                              static_cast<const T*>(shift), static_cast<T*>(output), seq, hd,
                              steps, epsilon, staged, vec);
    } else {
      using T = float;
      tb::launch_with_smem<T>(tb::layer_norm_adaln_kernel<T>, rows, smem, s,
                              static_cast<const T*>(input), static_cast<const T*>(scale),
                              static_cast<const T*>(shift), static_cast<T*>(output), seq, hd,
                              steps, epsilon, staged, vec);
    }
  });
}
