// Sage Q/K INT8 quantizers for sm_100a (memory-bound).
//
// Per tile of T tokens x D channels of one (batch, head)
// (kernel/csrc/turing/sage/fused.cu:66-200, QuantInt8Kernel):
//   amax  = max(1e-7, max |x - mean|)          (mean only when smoothing K)
//   scale = amax / 127                          -> scale[b, h, tile]
//   q     = cvt.rni.sat.s8((x - mean) * (127 / amax))
// The reference builds this extension with --use_fast_math, so its two
// divides are approximate; this implementation (and the CPU oracle) use the
// IEEE divides, which is the one definition the bit-exact tests pin.
// Tiles: Q per 16-token warp tile inside 64-token blocks (scale index
// block*4 + warp, quant.py:95-115), K per 64-token block.
//
// Token mean for K smoothing: per (batch, head, channel), summed in fp64 so
// the result does not depend on the reduction order, divided by L, rounded to
// fp32 and then to the input dtype (the mean that QuantInt8Kernel<...,
// sub_mean=true> subtracts, fused.cu:97-128).
#include <type_traits>

#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

template <typename T>
__device__ __forceinline__ float to_f32(uint32_t bits);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(uint32_t b) {
  return bf16_bits_to_f32(b);
}
template <>
__device__ __forceinline__ float to_f32<__half>(uint32_t b) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
}

__device__ __forceinline__ uint32_t cvt_s8(float x) {
  uint32_t r;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r & 0xffu;
}

struct QuantParams {
  const void* in;
  int8_t* out;
  float* scale;
  const void* mean;  // [B, H, D] or null
  int H, L;
  int64_t in_sb, in_sh, in_sl;   // input strides (elements)
  int64_t out_sb, out_sh, out_sl;
  int tiles;                     // scale entries per (b, h)
};

// grid (tiles, H, B), 256 threads; thread t handles packs of 8 channels.
template <typename T, int D, int TILE, bool MEAN>
__global__ void __launch_bounds__(256) quant_tile_kernel(QuantParams p) {
  constexpr int kTPR = D / 8;                 // threads per token row
  constexpr int kRowsPerPass = 256 / kTPR;    // token rows covered by one pass
  constexpr int kPasses = (TILE + kRowsPerPass - 1) / kRowsPerPass;
  __shared__ float warp_amax[8];
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x;
  const int c8 = (t % kTPR) * 8;
  const int r0 = t / kTPR;
  const T* in = static_cast<const T*>(p.in);
  float mean_v[8];
  if constexpr (MEAN) {
    const uint4 m = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.mean) +
                                                         (static_cast<int64_t>(b) * p.H + h) * D + c8));
    const uint32_t mw[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mean_v[2 * i] = to_f32<T>(mw[i] & 0xffffu);
      mean_v[2 * i + 1] = to_f32<T>(mw[i] >> 16);
    }
  }
  float x[kPasses][8];
  float amax = 0.0000001f;
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int row = r0 + ps * kRowsPerPass;
    const int tok = tile * TILE + row;
    if (row < TILE && tok < p.L) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(
          in + b * p.in_sb + h * p.in_sh + static_cast<int64_t>(tok) * p.in_sl + c8));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[ps][2 * i] = to_f32<T>(w[i] & 0xffffu);
        x[ps][2 * i + 1] = to_f32<T>(w[i] >> 16);
      }
      if constexpr (MEAN) {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[ps][i] = __fsub_rn(x[ps][i], mean_v[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[ps][i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[ps][i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((t & 31) == 0) warp_amax[t >> 5] = amax;
  __syncthreads();
  amax = warp_amax[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, warp_amax[w]);
  if (t == 0) p.scale[(static_cast<int64_t>(b) * p.H + h) * p.tiles + tile] = __fdiv_rn(amax, 127.0f);
  const float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int row = r0 + ps * kRowsPerPass;
    const int tok = tile * TILE + row;
    if (row < TILE && tok < p.L) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lo |= cvt_s8(__fmul_rn(x[ps][i], inv)) << (8 * i);
        hi |= cvt_s8(__fmul_rn(x[ps][4 + i], inv)) << (8 * i);
      }
      *reinterpret_cast<uint2*>(p.out + b * p.out_sb + h * p.out_sh +
                                static_cast<int64_t>(tok) * p.out_sl + c8) = make_uint2(lo, hi);
    }
  }
}

struct MeanParams {
  const void* in;
  void* mean;
  int H, L;
  int64_t sb, sh, sl;
};

template <typename T, int D>
__global__ void __launch_bounds__(1024) token_mean_kernel(MeanParams p) {
  constexpr int kTPR = D / 8;             // threads per token row (8 channels each)
  constexpr int kStripes = 1024 / kTPR;   // token stripes per CTA
  constexpr int kStripesPerWarp = 32 / kTPR;
  constexpr int kInFlight = 8;  // 170 us at configs[1]' K (4: 186 us, 1: 291 us)
  __shared__ double partial[32][D + 1];   // one row of channel sums per warp
  const int h = blockIdx.x, b = blockIdx.y;
  const int t = threadIdx.x;
  const int c8 = (t % kTPR) * 8;
  const int stripe = t / kTPR;
  const T* in = static_cast<const T*>(p.in) + b * p.sb + h * p.sh;
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  auto add_row = [&](const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] += static_cast<double>(to_f32<T>(w[i] & 0xffffu));
      acc[2 * i + 1] += static_cast<double>(to_f32<T>(w[i] >> 16));
    }
  };
  // kInFlight of this thread's token rows are loaded before any is added (one
  // CTA per head keeps only a few CTAs on the GPU, so each thread keeps
  // several loads in flight); the rows are still added in increasing token
  // order.
  int tok = stripe;
  for (; tok + (kInFlight - 1) * kStripes < p.L; tok += kInFlight * kStripes) {
    uint4 v[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u)
      v[u] = __ldg(reinterpret_cast<const uint4*>(in + static_cast<int64_t>(tok + u * kStripes) * p.sl + c8));
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) add_row(v[u]);
  }
  for (; tok < p.L; tok += kStripes)
    add_row(__ldg(reinterpret_cast<const uint4*>(in + static_cast<int64_t>(tok) * p.sl + c8)));
  // Fold the stripes that share a warp, then the warps, in a fixed order.
#pragma unroll
  for (int o = kTPR; o < 32; o <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  (void)kStripesPerWarp;
  if ((t & 31) < kTPR) {
#pragma unroll
    for (int i = 0; i < 8; ++i) partial[t >> 5][c8 + i] = acc[i];
  }
  __syncthreads();
  if (t < D) {
    double s = 0.0;
    for (int w = 0; w < 32; ++w) s += partial[w][t];
    const float m = static_cast<float>(s / static_cast<double>(p.L));
    uint16_t bits;
    if constexpr (std::is_same<T, __half>::value) {
      bits = __half_as_ushort(__float2half_rn(m));
    } else {
      bits = f32_to_bf16_bits(m);
    }
    static_cast<uint16_t*>(p.mean)[(static_cast<int64_t>(b) * p.H + h) * D + t] = bits;
  }
}

template <typename T, int D, int TILE>
void launch_quant_t(const QuantParams& p, int B, bool mean, cudaStream_t stream) {
  dim3 grid(p.tiles, p.H, B);
  if (mean) quant_tile_kernel<T, D, TILE, true><<<grid, 256, 0, stream>>>(p);
  else quant_tile_kernel<T, D, TILE, false><<<grid, 256, 0, stream>>>(p);
  TB_CUDA_CHECK(cudaGetLastError());
}

void check_qk_input(const void* input, int dtype, int64_t B, int64_t H, int64_t L, int64_t D,
                    int64_t sb, int64_t sh, int64_t sl, int layout) {
  TB_REQUIRE(input != nullptr, "input must be a CUDA tensor");
  TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16, "Only half and bfloat16 are supported");
  TB_REQUIRE(layout == TB_LAYOUT_NHD || layout == TB_LAYOUT_HND, "tensor_layout must be 0 or 1");
  TB_REQUIRE(B > 0 && H > 0 && L > 0, "empty Q/K sequences are not supported");
  TB_REQUIRE(D == 64 || D == 128, "Unsupported head_dim (the quantizers take 64 or 128)");
  TB_REQUIRE(B <= 65535 && H <= 65535 && L <= INT32_MAX, "Q/K dimensions exceed the kernel range");
  TB_REQUIRE(sb % 8 == 0 && sh % 8 == 0 && sl % 8 == 0 &&
                 (reinterpret_cast<uintptr_t>(input) & 15u) == 0,
             "Q/K rows must be 16-byte aligned (last dimension contiguous)");
}

}  // namespace

void sage_quant_launch(const void* input, int dtype, int8_t* out, float* scale, int64_t B,
                       int64_t H, int64_t L, int64_t D, int64_t sb, int64_t sh, int64_t sl,
                       int tile, int64_t num_tiles, int layout, const void* mean,
                       cudaStream_t stream) {
  check_qk_input(input, dtype, B, H, L, D, sb, sh, sl, layout);
  TB_REQUIRE(out != nullptr && scale != nullptr, "output and scale must be CUDA tensors");
  QuantParams p{};
  p.in = input;
  p.out = out;
  p.scale = scale;
  p.mean = mean;
  p.H = static_cast<int>(H);
  p.L = static_cast<int>(L);
  p.in_sb = sb;
  p.in_sh = sh;
  p.in_sl = sl;
  // The output is contiguous with the input's shape in the given layout.
  if (layout == TB_LAYOUT_HND) {
    p.out_sl = D;
    p.out_sh = L * D;
    p.out_sb = H * L * D;
  } else {
    p.out_sh = D;
    p.out_sl = H * D;
    p.out_sb = L * H * D;
  }
  // num_tiles >= ceil(L / tile): the per-warp Q layout pads the sequence to
  // whole 64-token blocks and writes a scale (amax floor 1e-7) for every
  // warp tile of the padded blocks, as the reference grid does.
  TB_REQUIRE(num_tiles >= (L + tile - 1) / tile && num_tiles <= INT32_MAX,
             "scale layout is smaller than the quantization tiles");
  p.tiles = static_cast<int>(num_tiles);
  const bool m = mean != nullptr;
  const int b = static_cast<int>(B);
#define TB_Q(T)                                                        \
  if (D == 128) {                                                      \
    if (tile == 16) launch_quant_t<T, 128, 16>(p, b, m, stream);      \
    else if (tile == 32) launch_quant_t<T, 128, 32>(p, b, m, stream); \
    else if (tile == 64) launch_quant_t<T, 128, 64>(p, b, m, stream); \
    else launch_quant_t<T, 128, 128>(p, b, m, stream);                \
  } else {                                                             \
    if (tile == 16) launch_quant_t<T, 64, 16>(p, b, m, stream);       \
    else if (tile == 32) launch_quant_t<T, 64, 32>(p, b, m, stream);  \
    else if (tile == 64) launch_quant_t<T, 64, 64>(p, b, m, stream);  \
    else launch_quant_t<T, 64, 128>(p, b, m, stream);                 \
  }
  TB_REQUIRE(tile == 16 || tile == 32 || tile == 64 || tile == 128,
             "quantization tile must be 16, 32, 64 or 128 tokens");
  if (dtype == TB_DTYPE_BF16) {
    TB_Q(__nv_bfloat16)
  } else {
    TB_Q(__half)
  }
#undef TB_Q
}

void token_mean_launch(const void* input, int dtype, void* mean, int64_t B, int64_t H, int64_t L,
                       int64_t D, int64_t sb, int64_t sh, int64_t sl, int layout,
                       cudaStream_t stream) {
  check_qk_input(input, dtype, B, H, L, D, sb, sh, sl, layout);
  TB_REQUIRE(mean != nullptr, "mean must be a CUDA tensor");
  MeanParams p{};
  p.in = input;
  p.mean = mean;
  p.H = static_cast<int>(H);
  p.L = static_cast<int>(L);
  p.sb = sb;
  p.sh = sh;
  p.sl = sl;
  dim3 grid(static_cast<unsigned>(H), static_cast<unsigned>(B));
  if (dtype == TB_DTYPE_BF16) {
    if (D == 128) token_mean_kernel<__nv_bfloat16, 128><<<grid, 1024, 0, stream>>>(p);
    else token_mean_kernel<__nv_bfloat16, 64><<<grid, 1024, 0, stream>>>(p);
  } else {
    if (D == 128) token_mean_kernel<__half, 128><<<grid, 1024, 0, stream>>>(p);
    else token_mean_kernel<__half, 64><<<grid, 1024, 0, stream>>>(p);
  }
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tb
