// Quantizers of the dense W8A8-PV attention for sm_100a (memory-bound).
//
// Q/K (kernel/csrc/turing/sage/fused.cu:201-398, 406-556, 559-639):
//   K anchor   per (batch, kv head): nine keys at rows s * (L - 1) / 8; the one
//              nearest their mean becomes the anchor when subtracting it
//              lowers the samples' energy and grows their range by at most
//              12.5 %; otherwise -1 (no subtraction).  The fused prologue's
//              variant (qk_preprocess.cu:252-415) samples the normalized +
//              rotated keys instead (qk_anchor_kernel).
//   rotation   x -> H_D diag(sign) x / sqrt(D) over the D = 64 / 128 channels
//              of a token (Sylvester Walsh-Hadamard, the sign vector of the
//              reference), K minus its anchor's values first (the raw anchor
//              row, or the prologue's processed sample).
//   codes      per tile (Q: 16 tokens, K: 64 tokens) amax = max(1e-7, |x|),
//              scale = amax / 127, q = rni_sat(x * (127 / amax)); a NaN codes
//              as 0 (fused.cu's cvt.rni.sat.s8) or -127 (the prologue's clamp
//              of nearbyintf, qk_preprocess.cu:43-47).
// V (quant_v_int8_cuda_sm75.cu:58-164): per (batch, head, channel) over all
//   tokens, scale = max(amax / 127, 1e-12), q = rni_sat(v * (1 / scale)).
//
// Bit-exactness: the butterflies run in the reference's stage order (channel
// bit 0 first, bit 6 last), each lo' = lo + hi, hi' = lo - hi in fp32, and
// the anchor statistics use its reduction order (per-thread fmaf chains, warp
// shfl_down trees, the four warps summed in order), so the codes, scales and
// anchor choices are the reference's.  Divides are IEEE (the reference's
// extension is built with --use_fast_math; the CPU oracle fixes IEEE).
//
// Layout of the rotation: the 4 lanes of a token row hold packs r, r+4, r+8,
// r+12 of 8 channels (r = lane % 4), so channel bits 0-2 and 5-6 are
// butterflies inside a lane and bits 3-4 are two xor-shuffles; each load
// instruction reads 64 contiguous bytes of 8 rows.
#include <type_traits>

#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

template <typename T>
__device__ __forceinline__ float lo_f(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(w << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
}
template <typename T>
__device__ __forceinline__ float hi_f(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(w & 0xffff0000u);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&x)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = lo_f<T>(w[i]);
    x[2 * i + 1] = hi_f<T>(w[i]);
  }
}

// Low byte = rni_sat_s8(v) for |v| <= 127 * (1 + 2^-23), or nan_code for a
// NaN: adding 1.5 * 2^23 rounds to the nearest integer, ties to even, and
// leaves it two's-complement in the low byte.
__device__ __forceinline__ uint32_t code_bits(float v, float nan_code) {
  return __float_as_uint(__fadd_rn(v == v ? v : nan_code, 12582912.0f));
}
__device__ __forceinline__ uint32_t pack_codes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Bit c of the 128-bit word, clear = channel c negated (fused.cu:205-213).
__device__ constexpr uint32_t kRotSigns[4] = {0x1035997bu, 0x8087f5eeu, 0xee2e4e1au,
                                              0x71132418u};

// ------------------------------------------------------------ K anchor ----

struct AnchorParams {
  const void* k;
  int32_t* anchors;  // [B, Hk]
  float* values;     // [B, Hk, D]: the anchor rows, zeros for -1
  int H, L;
  int64_t sb, sh, sl;
};

constexpr int kAnchorSamples = 9;

__device__ __forceinline__ float tree_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float tree_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_down_sync(0xffffffffu, v, o));
  return v;
}

// The anchor choice over samp[9][D] (filled by the caller, synced), run by the
// 128 threads of the CTA (thread t owns channel t); writes the row index (or
// -1) and the anchor's values (zeros for -1).
template <int D>
__device__ __forceinline__ void anchor_select(const float (*samp)[D], int L, int32_t* anchor,
                                              float* values) {
  __shared__ float w_oe[4], w_om[4], w_be[4], w_bm[4];
  __shared__ float w_cd[kAnchorSamples][4];
  __shared__ int best_sh;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float oe = 0.0f, om = 0.0f;
  float cd[kAnchorSamples];
#pragma unroll
  for (int s = 0; s < kAnchorSamples; ++s) cd[s] = 0.0f;
  if (t < D) {
    float sum = 0.0f;
#pragma unroll
    for (int s = 0; s < kAnchorSamples; ++s) {
      const float v = samp[s][t];
      oe = fmaf(v, v, oe);
      om = fmaxf(om, fabsf(v));
      sum += v;
    }
#pragma unroll
    for (int s = 0; s < kAnchorSamples; ++s) {
      const float dist = fmaf(9.0f, samp[s][t], -sum);  // 9 * x is exact
      cd[s] = fmaf(dist, dist, cd[s]);
    }
  }
  oe = tree_sum(oe);
  om = tree_max(om);
#pragma unroll
  for (int s = 0; s < kAnchorSamples; ++s) cd[s] = tree_sum(cd[s]);
  if (lane == 0) {
    w_oe[warp] = oe;
    w_om[warp] = om;
#pragma unroll
    for (int s = 0; s < kAnchorSamples; ++s) w_cd[s][warp] = cd[s];
  }
  __syncthreads();
  if (t == 0) {
    int best = 0;
    float best_d = 3.402823466e+38F;
    for (int s = 0; s < kAnchorSamples; ++s) {
      float d = 0.0f;
      for (int w = 0; w < 4; ++w) d += w_cd[s][w];
      if (d < best_d) {
        best = s;
        best_d = d;
      }
    }
    best_sh = best;
  }
  __syncthreads();
  const int best = best_sh;
  float be = 0.0f, bm = 0.0f;
  if (t < D) {
    const float a = samp[best][t];
#pragma unroll
    for (int s = 0; s < kAnchorSamples; ++s) {
      const float r = samp[s][t] - a;
      be = fmaf(r, r, be);
      bm = fmaxf(bm, fabsf(r));
    }
  }
  be = tree_sum(be);
  bm = tree_max(bm);
  if (lane == 0) {
    w_be[warp] = be;
    w_bm[warp] = bm;
  }
  __syncthreads();
  if (t == 0) {
    float toe = 0.0f, tom = 0.0f, tbe = 0.0f, tbm = 0.0f;
    for (int w = 0; w < 4; ++w) {
      toe += w_oe[w];
      tom = fmaxf(tom, w_om[w]);
      tbe += w_be[w];
      tbm = fmaxf(tbm, w_bm[w]);
    }
    const bool keep = tbe < toe && tbm <= tom * 1.125f;
    *anchor = keep ? static_cast<int32_t>(static_cast<int64_t>(best) * (L - 1) / (kAnchorSamples - 1))
                   : -1;
    best_sh = keep ? best : -1;
  }
  __syncthreads();
  if (t < D) values[t] = best_sh >= 0 ? samp[best_sh][t] : 0.0f;
}

// Anchor of the raw keys.  grid (Hk, B), 128 threads.
template <typename T, int D>
__global__ void __launch_bounds__(128) k_anchor_kernel(AnchorParams p) {
  __shared__ float samp[kAnchorSamples][D];
  const int h = blockIdx.x, b = blockIdx.y;
  const T* kh = static_cast<const T*>(p.k) + b * p.sb + h * p.sh;
  for (int i = threadIdx.x; i < kAnchorSamples * D; i += 128) {
    const int s = i / D, c = i - s * D;
    const int64_t row = static_cast<int64_t>(s) * (p.L - 1) / (kAnchorSamples - 1);
    const T v = kh[row * p.sl + c];
    if constexpr (std::is_same<T, __nv_bfloat16>::value) samp[s][c] = __bfloat162float(v);
    else samp[s][c] = __half2float(v);
  }
  __syncthreads();
  anchor_select<D>(samp, p.L, p.anchors + b * p.H + h,
                   p.values + (static_cast<int64_t>(b) * p.H + h) * D);
}

// Anchor of the fused prologue's normalized + rotated keys
// (detect_anchor_kernel, qk_preprocess.cu:252-415).  Each sampled token gets
// its own RRMS (row scope: the row RRMS; head scope: one FMA chain over the
// channels in order, then the correctly rounded 1/sqrt), then
// n = T(x * rrms * w) and, on the first rot_dim channels,
// v = T(fma(f[row][1], n(second), f[row][0] * n(first))).  grid (Hk, B), 128 threads.
struct ProcAnchorParams {
  const void* k;
  const void* norm;      // [D] (head scope) or [Hk * D] (row scope)
  const void* freqs;     // valid memory even when rot_dim == 0
  const float* rrms;     // row scope: [B, L]; else unused (valid memory)
  int32_t* anchors;      // [B, Hk]
  float* values;         // [B, Hk, D]
  int H, L, rot_dim, split_half, row_scope, f_batches, f_seq;
  int64_t sb, sh, sl;
  int64_t f_b, f_s, f_p, f_r, f_c;
  float eps;
};

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(v);
  else return __half2float(v);
}
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(v));
  else return __half2float(__float2half_rn(v));
}

template <typename T, int D>
__global__ void __launch_bounds__(128) qk_anchor_kernel(ProcAnchorParams p) {
  __shared__ float samp[kAnchorSamples][D];
  __shared__ float rr[kAnchorSamples];
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  const T* kh = static_cast<const T*>(p.k) + b * p.sb + h * p.sh;
  const T* w = static_cast<const T*>(p.norm) + (p.row_scope ? h * D : 0);
  if (t < kAnchorSamples) {
    const int tok = static_cast<int>(static_cast<int64_t>(t) * (p.L - 1) / (kAnchorSamples - 1));
    if (p.row_scope) {
      rr[t] = p.rrms[static_cast<int64_t>(b) * p.L + tok];
    } else {
      float sum = 0.0f;
      for (int c = 0; c < D; ++c) {
        const float v = to_f(kh[static_cast<int64_t>(tok) * p.sl + c]);
        sum = fmaf(v, v, sum);
      }
      rr[t] = __frsqrt_rn(__fdiv_rn(sum, static_cast<float>(D)) + p.eps);
    }
  }
  __syncthreads();
  if (t < D) {
    const int half = p.rot_dim / 2;
    const T* fr = static_cast<const T*>(p.freqs);
    for (int s = 0; s < kAnchorSamples; ++s) {
      const int tok = static_cast<int>(static_cast<int64_t>(s) * (p.L - 1) / (kAnchorSamples - 1));
      const T* row = kh + static_cast<int64_t>(tok) * p.sl;
      const float rs = rr[s];
      float v = round_to<T>(to_f(row[t]) * rs * to_f(w[t]));
      if (t < p.rot_dim) {
        const int pair = p.split_half ? (t < half ? t : t - half) : t / 2;
        const int first = p.split_half ? pair : 2 * pair;
        const int second = p.split_half ? pair + half : first + 1;
        const int comp = p.split_half ? (t >= half) : (t & 1);
        const float x0 = round_to<T>(to_f(row[first]) * rs * to_f(w[first]));
        const float x1 = round_to<T>(to_f(row[second]) * rs * to_f(w[second]));
        const int64_t fbase = static_cast<int64_t>(p.f_batches == 1 ? 0 : b) * p.f_b +
                              static_cast<int64_t>(p.f_seq == 1 ? 0 : tok) * p.f_s +
                              static_cast<int64_t>(pair) * p.f_p + comp * p.f_r;
        v = round_to<T>(fmaf(to_f(fr[fbase + p.f_c]), x1, to_f(fr[fbase]) * x0));
      }
      samp[s][t] = v;
    }
  }
  __syncthreads();
  anchor_select<D>(samp, p.L, p.anchors + b * p.H + h,
                   p.values + (static_cast<int64_t>(b) * p.H + h) * D);
}

// --------------------------------------------------- rotated Q/K codes ----

struct RotParams {
  const void* in[2];      // Q, K
  int8_t* out[2];
  float* scale[2];        // Q: [B, Hq, blocks*4]; K: [B, Hk, blocks]
  const float* anchor_values;  // [B, Hk, D] subtracted from K (zeros: none) or null
  float nan_code;              // code of a NaN: 0 or -127
  int heads[2], length[2], blocks[2];
  int64_t s_b[2], s_h[2], s_l[2];   // input strides (elements)
  int64_t o_b[2], o_h[2], o_l[2];   // output strides
};

// Butterfly of one pair in place: (lo, hi) -> (lo + hi, lo - hi).
__device__ __forceinline__ void bfly(float& lo, float& hi) {
  const float a = lo, c = hi;
  lo = __fadd_rn(a, c);
  hi = __fsub_rn(a, c);
}

// grid (Q tasks + K tasks, B), 128 threads; a task is one 64-token block of
// one head.  Warp w covers tokens 16w..16w+15 of the block (one Q scale tile);
// lane l holds token rows l/4 and l/4 + 8 of them, packs r + 4k (r = l % 4).
template <typename T, int D>
__global__ void __launch_bounds__(128) rot_quant_kernel(const RotParams a) {
  constexpr int NP = D / 32;  // packs per lane
  __shared__ float warp_amax[4];
  const int b = blockIdx.y;
  int task = blockIdx.x;
  const int which = task < a.heads[0] * a.blocks[0] ? 0 : 1;
  if (which == 1) task -= a.heads[0] * a.blocks[0];
  const int h = task / a.blocks[which];
  const int blk = task - h * a.blocks[which];
  const int L = a.length[which];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane & 3;
  const T* in = static_cast<const T*>(a.in[which]) + b * a.s_b[which] + h * a.s_h[which];
  const bool anchored = which == 1 && a.anchor_values != nullptr;
  float anc[NP][8];
  if (anchored) {
    const float* av = a.anchor_values + (static_cast<int64_t>(b) * a.heads[1] + h) * D;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      const float4 lo4 = __ldg(reinterpret_cast<const float4*>(av + 8 * (r + 4 * k)));
      const float4 hi4 = __ldg(reinterpret_cast<const float4*>(av + 8 * (r + 4 * k) + 4));
      anc[k][0] = lo4.x; anc[k][1] = lo4.y; anc[k][2] = lo4.z; anc[k][3] = lo4.w;
      anc[k][4] = hi4.x; anc[k][5] = hi4.y; anc[k][6] = hi4.z; anc[k][7] = hi4.w;
    }
  }
  float v[2][NP][8];
  float amax = 0.0000001f;
#pragma unroll
  for (int ps = 0; ps < 2; ++ps) {
    const int tok = blk * 64 + warp * 16 + ps * 8 + (lane >> 2);
    if (tok < L) {
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        load8(in + static_cast<int64_t>(tok) * a.s_l[which] + 8 * (r + 4 * k), v[ps][k]);
        if (anchored) {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[ps][k][e] = __fsub_rn(v[ps][k][e], anc[k][e]);
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < NP; ++k)
#pragma unroll
        for (int e = 0; e < 8; ++e) v[ps][k][e] = 0.0f;
    }
    // Signs: channel 8 (r + 4k) + e is negated when bit e of byte r of word k
    // is clear.
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      const uint32_t keep = kRotSigns[k] >> (8 * r);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        v[ps][k][e] = __uint_as_float(__float_as_uint(v[ps][k][e]) ^ ((~keep >> e & 1u) << 31));
    }
    // Channel bits 0, 1, 2: inside the pack.
#pragma unroll
    for (int span = 1; span < 8; span <<= 1)
#pragma unroll
      for (int k = 0; k < NP; ++k)
#pragma unroll
        for (int base = 0; base < 8; base += 2 * span)
#pragma unroll
          for (int o = 0; o < span; ++o) bfly(v[ps][k][base + o], v[ps][k][base + o + span]);
    // Channel bits 3, 4: across the 4 lanes of the row.
#pragma unroll
    for (int bit = 1; bit < 4; bit <<= 1) {
#pragma unroll
      for (int k = 0; k < NP; ++k)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float other = __shfl_xor_sync(0xffffffffu, v[ps][k][e], bit);
          v[ps][k][e] = (r & bit) ? __fsub_rn(other, v[ps][k][e]) : __fadd_rn(v[ps][k][e], other);
        }
    }
    // Channel bits 5 (and 6 for D = 128): across the lane's packs.
#pragma unroll
    for (int kb = 1; kb < NP; kb <<= 1)
#pragma unroll
      for (int k = 0; k < NP; ++k)
        if (!(k & kb)) {
#pragma unroll
          for (int e = 0; e < 8; ++e) bfly(v[ps][k][e], v[ps][k + kb][e]);
        }
    constexpr float kNorm = D == 64 ? 0.125f : 0.08838834764831845f;
#pragma unroll
    for (int k = 0; k < NP; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[ps][k][e] = __fmul_rn(v[ps][k][e], kNorm);
        amax = fmaxf(amax, fabsf(v[ps][k][e]));
      }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float* scale = a.scale[which] + (static_cast<int64_t>(b) * a.heads[which] + h) *
                                      (which == 0 ? a.blocks[0] * 4 : a.blocks[1]);
  if (which == 1) {
    // K: one tile of 64 tokens over the four warps.
    if (lane == 0) warp_amax[warp] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(warp_amax[0], warp_amax[1]), fmaxf(warp_amax[2], warp_amax[3]));
    if (threadIdx.x == 0) scale[blk] = __fdiv_rn(amax, 127.0f);
  } else if (lane == 0) {
    scale[blk * 4 + warp] = __fdiv_rn(amax, 127.0f);
  }
  const float inv = __fdiv_rn(127.0f, amax);
  int8_t* out = a.out[which] + b * a.o_b[which] + h * a.o_h[which];
#pragma unroll
  for (int ps = 0; ps < 2; ++ps) {
    const int tok = blk * 64 + warp * 16 + ps * 8 + (lane >> 2);
    if (tok >= L) continue;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      uint32_t cb[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) cb[e] = code_bits(__fmul_rn(v[ps][k][e], inv), a.nan_code);
      *reinterpret_cast<uint2*>(out + static_cast<int64_t>(tok) * a.o_l[which] + 8 * (r + 4 * k)) =
          make_uint2(pack_codes(cb[0], cb[1], cb[2], cb[3]), pack_codes(cb[4], cb[5], cb[6], cb[7]));
    }
  }
}

// ------------------------------------------------------------ V codes -----

struct VParams {
  const void* v;
  uint16_t* codes_f16;  // [B, H, L, D] contiguous or null
  int8_t* codes_cm;     // [B, H, D, Lpad] contiguous or null
  float* scale;         // [B, H, D]: amax bits while the kernels run
  int H, L, Lpad;
  int64_t sb, sh, sl;
};

constexpr int kVChunk = 64;  // tokens per CTA

// grid (ceil(L / kVChunk), B * H), 256 threads: D / 8 lanes per token row.
template <typename T, int D>
__global__ void __launch_bounds__(256) v_amax_kernel(VParams p) {
  constexpr int kTPR = D / 8, kRows = 256 / kTPR;
  __shared__ float part[kRows][D];
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int c8 = (threadIdx.x % kTPR) * 8, row = threadIdx.x / kTPR;
  const T* vh = static_cast<const T*>(p.v) + b * p.sb + h * p.sh;
  float m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int tok = blockIdx.x * kVChunk + row; tok < min(p.L, (blockIdx.x + 1) * kVChunk); tok += kRows) {
    float x[8];
    load8(vh + static_cast<int64_t>(tok) * p.sl + c8, x);
#pragma unroll
    for (int e = 0; e < 8; ++e) m[e] = fmaxf(m[e], fabsf(x[e]));
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[row][c8 + e] = m[e];
  __syncthreads();
  if (threadIdx.x < D) {
    float mx = 0.0f;
    for (int r2 = 0; r2 < kRows; ++r2) mx = fmaxf(mx, part[r2][threadIdx.x]);
    // Non-negative floats order like their bit patterns.
    atomicMax(reinterpret_cast<unsigned int*>(p.scale) + static_cast<int64_t>(bh) * D + threadIdx.x,
              __float_as_uint(mx));
  }
}

// Same grid: codes of the chunk, from the finished channel maxima.
template <typename T, int D>
__global__ void __launch_bounds__(256) v_codes_kernel(VParams p) {
  constexpr int kTPR = D / 8, kRows = 256 / kTPR;
  __shared__ float inv_sh[D];
  __shared__ int8_t tile[D][kVChunk + 4];
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int c8 = (threadIdx.x % kTPR) * 8, row = threadIdx.x / kTPR;
  const int t0 = blockIdx.x * kVChunk;
  if (threadIdx.x < D) {
    const float amax = __uint_as_float(
        reinterpret_cast<const unsigned int*>(p.scale)[static_cast<int64_t>(bh) * D + threadIdx.x]);
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-12f);
    inv_sh[threadIdx.x] = __frcp_rn(sc);
  }
  __syncthreads();
  const T* vh = static_cast<const T*>(p.v) + b * p.sb + h * p.sh;
  for (int i = row; i < kVChunk; i += kRows) {
    const int tok = t0 + i;
    uint32_t cb[8];
    if (tok < p.L) {
      float x[8];
      load8(vh + static_cast<int64_t>(tok) * p.sl + c8, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) cb[e] = code_bits(__fmul_rn(x[e], inv_sh[c8 + e]), 0.0f) & 0xffu;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) cb[e] = 0;
    }
    if (p.codes_f16 != nullptr && tok < p.L) {
      // Exact fp16 of the signed code c: 0x6400 | (c + 128) is the fp16 1024 +
      // (c + 128) (exponent 10, one unit per step), minus 1152.
      uint32_t w[4];
#pragma unroll
      for (int i2 = 0; i2 < 4; ++i2) {
        const uint32_t biased = (0x6400u | (cb[2 * i2] ^ 0x80u)) | ((0x6400u | (cb[2 * i2 + 1] ^ 0x80u)) << 16);
        const __half2 hv = __hsub2(*reinterpret_cast<const __half2*>(&biased), __float2half2_rn(1152.0f));
        w[i2] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      *reinterpret_cast<uint4*>(p.codes_f16 + (static_cast<int64_t>(bh) * p.L + tok) * D + c8) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (p.codes_cm != nullptr) {
#pragma unroll
      for (int e = 0; e < 8; ++e) tile[c8 + e][i] = static_cast<int8_t>(cb[e]);
    }
  }
  if (p.codes_cm != nullptr) {
    __syncthreads();
    // Channel rows of kVChunk tokens: 16 lanes x 4 bytes per row.
    for (int i = threadIdx.x; i < D * (kVChunk / 4); i += 256) {
      const int c = i / (kVChunk / 4), q4 = i - c * (kVChunk / 4);
      if (t0 + 4 * q4 >= p.Lpad) continue;
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) w |= static_cast<uint32_t>(static_cast<uint8_t>(tile[c][4 * q4 + j])) << (8 * j);
      *reinterpret_cast<uint32_t*>(p.codes_cm + (static_cast<int64_t>(bh) * D + c) * p.Lpad + t0 + 4 * q4) = w;
    }
  }
}

// scale = max(amax / 127, 1e-12) in place.
__global__ void v_scale_kernel(float* scale, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) scale[i] = fmaxf(__fdiv_rn(__uint_as_float(reinterpret_cast<unsigned int*>(scale)[i]), 127.0f), 1.0e-12f);
}

void check_rows(const void* p, int64_t sb, int64_t sh, int64_t sl, const char* msg) {
  TB_REQUIRE(p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && sb % 8 == 0 &&
                 sh % 8 == 0 && sl % 8 == 0,
             msg);
}

}  // namespace

void rot_quant_launch(const void* q, const void* k, int8_t* q_out, int8_t* k_out, float* q_scale,
                      float* k_scale, int32_t* anchors, float* anchor_values, int64_t B,
                      int64_t Hq, int64_t Hk, int64_t Lq, int64_t Lk, int64_t D,
                      const int64_t* s, int anchor_mode, int nan_code, int dtype,
                      cudaStream_t stream) {
  TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16,
             "Turing W8A8 Q/K must be float16 or bfloat16");
  TB_REQUIRE(D == 64 || D == 128, "the rotated quantizer takes head_dim 64 or 128 (pad first)");
  TB_REQUIRE(B > 0 && Hq > 0 && Hk > 0 && Lq > 0 && Lk > 0, "empty Q/K sequences are not supported");
  TB_REQUIRE(B <= 65535 && Lq <= INT32_MAX && Lk <= INT32_MAX, "Q/K dimensions exceed the kernel range");
  check_rows(q, s[0], s[1], s[2], "Q rows must be 16-byte aligned (last dimension contiguous)");
  check_rows(k, s[3], s[4], s[5], "K rows must be 16-byte aligned (last dimension contiguous)");
  TB_REQUIRE(q_out && k_out && (reinterpret_cast<uintptr_t>(q_out) & 7u) == 0 &&
                 (reinterpret_cast<uintptr_t>(k_out) & 7u) == 0 && s[6] % 8 == 0 && s[7] % 8 == 0 &&
                 s[8] % 8 == 0 && s[9] % 8 == 0 && s[10] % 8 == 0 && s[11] % 8 == 0,
             "INT8 Q/K outputs must start on 8-byte boundaries with strides of 8 elements");
  TB_REQUIRE(q_scale && k_scale, "scales must be CUDA tensors");
  TB_REQUIRE(anchor_mode >= 0 && anchor_mode <= 2,
             "anchor_mode must be 0 (none), 1 (detect from K) or 2 (values given)");
  TB_REQUIRE(anchor_mode == 0 || ((reinterpret_cast<uintptr_t>(anchor_values) & 15u) == 0 &&
                                  anchor_values != nullptr),
             "K anchor values must be a 16-byte aligned float32 [B, Hk, D] CUDA tensor");
  TB_REQUIRE(anchor_mode != 1 || anchors != nullptr, "K anchor scratch must be a CUDA tensor");
  TB_REQUIRE(nan_code == 0 || nan_code == -127, "nan_code must be 0 or -127");
  RotParams a{};
  a.in[0] = q;
  a.in[1] = k;
  a.out[0] = q_out;
  a.out[1] = k_out;
  a.scale[0] = q_scale;
  a.scale[1] = k_scale;
  a.anchor_values = anchor_mode ? anchor_values : nullptr;
  a.nan_code = static_cast<float>(nan_code);
  a.heads[0] = static_cast<int>(Hq);
  a.heads[1] = static_cast<int>(Hk);
  a.length[0] = static_cast<int>(Lq);
  a.length[1] = static_cast<int>(Lk);
  a.blocks[0] = static_cast<int>((Lq + 63) / 64);
  a.blocks[1] = static_cast<int>((Lk + 63) / 64);
  for (int w = 0; w < 2; ++w) {
    a.s_b[w] = s[3 * w];
    a.s_h[w] = s[3 * w + 1];
    a.s_l[w] = s[3 * w + 2];
    a.o_b[w] = s[6 + 3 * w];
    a.o_h[w] = s[6 + 3 * w + 1];
    a.o_l[w] = s[6 + 3 * w + 2];
  }
  const int64_t tasks = Hq * a.blocks[0] + Hk * a.blocks[1];
  TB_REQUIRE(tasks <= INT32_MAX, "Q/K dimensions exceed the kernel range");
  const dim3 grid(static_cast<unsigned>(tasks), static_cast<unsigned>(B));
  if (anchor_mode == 1) {
    AnchorParams ap{k, anchors, anchor_values, static_cast<int>(Hk), static_cast<int>(Lk),
                    s[3], s[4], s[5]};
    const dim3 ag(static_cast<unsigned>(Hk), static_cast<unsigned>(B));
    TB_REQUIRE(Hk <= 65535, "K head count exceeds the grid range");
    if (dtype == TB_DTYPE_BF16) {
      if (D == 128) k_anchor_kernel<__nv_bfloat16, 128><<<ag, 128, 0, stream>>>(ap);
      else k_anchor_kernel<__nv_bfloat16, 64><<<ag, 128, 0, stream>>>(ap);
    } else {
      if (D == 128) k_anchor_kernel<__half, 128><<<ag, 128, 0, stream>>>(ap);
      else k_anchor_kernel<__half, 64><<<ag, 128, 0, stream>>>(ap);
    }
    TB_CUDA_CHECK(cudaGetLastError());
  }
  if (dtype == TB_DTYPE_BF16) {
    if (D == 128) rot_quant_kernel<__nv_bfloat16, 128><<<grid, 128, 0, stream>>>(a);
    else rot_quant_kernel<__nv_bfloat16, 64><<<grid, 128, 0, stream>>>(a);
  } else {
    if (D == 128) rot_quant_kernel<__half, 128><<<grid, 128, 0, stream>>>(a);
    else rot_quant_kernel<__half, 64><<<grid, 128, 0, stream>>>(a);
  }
  TB_CUDA_CHECK(cudaGetLastError());
}

void qk_anchor_launch(const void* key, const void* key_norm, const void* freqs,
                      const float* key_rrms, int32_t* anchors, float* anchor_values, int64_t B,
                      int64_t Hk, int64_t Lk, int64_t D, const int64_t* k_strides,
                      const int64_t* freq_strides, int64_t freq_batches, int64_t freq_sequence,
                      int64_t rot_dim, int norm_scope, int split_half, int dtype, float eps,
                      cudaStream_t stream) {
  TB_REQUIRE(key && key_norm && anchors && anchor_values && k_strides,
             "K, its norm weight and the anchor outputs must be CUDA tensors");
  TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16, "K must be float16 or bfloat16");
  TB_REQUIRE(D == 64 || D == 128, "fused Q/K preprocessing requires head_dim 64 or 128");
  TB_REQUIRE(B > 0 && Hk > 0 && Lk > 0 && B <= 65535 && Hk <= 65535 && Lk <= INT32_MAX,
             "K dimensions must be positive and within the CUDA grid range");
  TB_REQUIRE(norm_scope >= 0 && norm_scope <= 2, "norm_scope must be 0, 1 or 2");
  TB_REQUIRE(norm_scope == 0 || key_rrms != nullptr, "row RRMS of K must be provided");
  TB_REQUIRE(rot_dim >= 0 && rot_dim <= D && rot_dim % 2 == 0,
             "rot_dim must be even and within head_dim");
  TB_REQUIRE(rot_dim == 0 || (freqs && freq_strides),
             "RoPE frequencies are required when rot_dim > 0");
  ProcAnchorParams p{};
  p.k = key;
  p.norm = key_norm;
  // Pointers the kernel does not use at run time still name readable memory.
  p.freqs = rot_dim > 0 ? freqs : key;
  p.rrms = norm_scope ? key_rrms : static_cast<const float*>(key);
  p.anchors = anchors;
  p.values = anchor_values;
  p.H = static_cast<int>(Hk);
  p.L = static_cast<int>(Lk);
  p.rot_dim = static_cast<int>(rot_dim);
  p.split_half = split_half;
  p.row_scope = norm_scope ? 1 : 0;
  p.sb = k_strides[0];
  p.sh = k_strides[1];
  p.sl = k_strides[2];
  if (rot_dim > 0) {
    p.f_b = freq_strides[0]; p.f_s = freq_strides[1]; p.f_p = freq_strides[2];
    p.f_r = freq_strides[3]; p.f_c = freq_strides[4];
    p.f_batches = static_cast<int>(freq_batches);
    p.f_seq = static_cast<int>(freq_sequence);
  } else {
    p.f_batches = p.f_seq = 1;
  }
  p.eps = eps;
  const dim3 grid(static_cast<unsigned>(Hk), static_cast<unsigned>(B));
  if (dtype == TB_DTYPE_BF16) {
    if (D == 128) qk_anchor_kernel<__nv_bfloat16, 128><<<grid, 128, 0, stream>>>(p);
    else qk_anchor_kernel<__nv_bfloat16, 64><<<grid, 128, 0, stream>>>(p);
  } else {
    if (D == 128) qk_anchor_kernel<__half, 128><<<grid, 128, 0, stream>>>(p);
    else qk_anchor_kernel<__half, 64><<<grid, 128, 0, stream>>>(p);
  }
  TB_CUDA_CHECK(cudaGetLastError());
}

void v_quant_launch(const void* v, int dtype, uint16_t* codes_f16, int8_t* codes_cm, float* scale,
                    int64_t B, int64_t H, int64_t L, int64_t D, int64_t Lpad, int64_t sb,
                    int64_t sh, int64_t sl, cudaStream_t stream) {
  TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16, "Turing W8A8 V must be FP16 or BF16");
  TB_REQUIRE(D == 64 || D == 128, "the V quantizer takes head_dim 64 or 128 (pad first)");
  TB_REQUIRE(B > 0 && H > 0 && L > 0 && L <= INT32_MAX, "V must hold at least one token");
  TB_REQUIRE(B * H <= 65535, "batch * heads exceeds the grid range");
  check_rows(v, sb, sh, sl, "V rows must be 16-byte aligned (head dimension contiguous)");
  TB_REQUIRE(codes_f16 != nullptr || codes_cm != nullptr, "no V code output given");
  TB_REQUIRE(codes_f16 == nullptr || (reinterpret_cast<uintptr_t>(codes_f16) & 15u) == 0,
             "fp16 V codes must be 16-byte aligned");
  TB_REQUIRE(codes_cm == nullptr || ((reinterpret_cast<uintptr_t>(codes_cm) & 3u) == 0 &&
                                     Lpad % 64 == 0 && Lpad >= L && Lpad <= INT32_MAX),
             "Turing W8A8 quantized V must be [B,H,D,ceil(N/64)*64]");
  TB_REQUIRE(scale != nullptr, "V scale must be a CUDA tensor");
  VParams p{v, codes_f16, codes_cm, scale, static_cast<int>(H), static_cast<int>(L),
            static_cast<int>(Lpad), sb, sh, sl};
  const int64_t n = B * H * D;
  TB_CUDA_CHECK(cudaMemsetAsync(scale, 0, sizeof(float) * n, stream));
  const int64_t tok_span = codes_cm != nullptr ? Lpad : L;
  const dim3 grid(static_cast<unsigned>((tok_span + kVChunk - 1) / kVChunk), static_cast<unsigned>(B * H));
  const dim3 grid_amax(static_cast<unsigned>((L + kVChunk - 1) / kVChunk), static_cast<unsigned>(B * H));
#define TB_VQ(T, DD)                                                  \
  {                                                                   \
    v_amax_kernel<T, DD><<<grid_amax, 256, 0, stream>>>(p);           \
    v_codes_kernel<T, DD><<<grid, 256, 0, stream>>>(p);               \
  }
  if (dtype == TB_DTYPE_BF16) {
    if (D == 128) TB_VQ(__nv_bfloat16, 128) else TB_VQ(__nv_bfloat16, 64)
  } else {
    if (D == 128) TB_VQ(__half, 128) else TB_VQ(__half, 64)
  }
#undef TB_VQ
  v_scale_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(scale, n);
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tb
