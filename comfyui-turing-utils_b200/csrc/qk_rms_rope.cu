// Fused Q/K prologue of the Sage attention path: RMSNorm (per head, or over the
// whole row of all heads) with an affine weight, RoPE as 2x2 rotations, and
// the per-tile INT8 quantization of the Sage contract (Q per 16-token warp
// tile, K per 64-token block).  Reference: kernel/csrc/turing/sage/
// qk_preprocess.cu:151-201 (per-element processing), :203-251 (row RMS),
// :417-563 (tile quantizer), :566-753 (launcher).  For the Hadamard /
// anchor variant that feeds the W8A8 attention the kernel writes the
// normalized + rotated values instead of codes (tb_qk_rms_rope_apply); the
// anchor and the rotated quantization run in w8a8_quant.cu.
//
// Per element of token t, channel c of a head (T = the input dtype):
//   n(c)  = T(x[c] * rrms * w[c])            rrms = rsqrt(sum_c x^2 / D + eps)
//   (sum of squares in the reference's order: an FMA chain per 8-channel pack
//   and an XOR tree over the packs, or, row scope, its block reduction)
//   c >= rot_dim: v = n(c); otherwise, with the pair (first, second) of c
//   (interleaved: (2p, 2p+1); split-half: (p, p + rot_dim/2)) and the pair's
//   2x2 matrix f[row][col] (row = which member c is):
//   v = T(fma(f[row][1], n(second), f[row][0] * n(first)))
// Then per tile: amax = max(1e-7, max |v|), scale = amax / 127,
// q = clamp(rint(v * (127 / amax)), -127, 127) (NaN -> -127).
// The reciprocal square root and the divides are correctly rounded
// (__frsqrt_rn, IEEE division); the reference's attention extension is built
// with fast-math and uses the hardware approximations, so its codes can differ
// by one where a product lands on a rounding boundary.
//
// Work layout (HBM-bound: each Q/K element is read once and its INT8 code
// written once; row scope adds one read for the row RMS pass):
//   * row_rrms_kernel: one CTA per 16 tokens; a thread owns one 16-byte pack
//     of channels and one residue class of heads (head mod 256/D), keeping the
//     reference's per-thread FMA chain for each of its 8 channels; the 256
//     chains of a token are then folded in the reference's warp/block order.
//   * qk_rms_rope_kernel: one CTA per (64-token block, head, Q or K); a thread
//     owns one 16-byte pack per 16 or 32 tokens, normalizes it once, rotates
//     interleaved pairs in registers (split-half partners go through shared
//     memory), and the Q warp tiles / K block take their max from one
//     CTA-wide exchange.
#include <cmath>

#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

constexpr int kQkThreads = 256;
constexpr int kQkBlock = 64;      // tokens per CTA (one K block, four Q warp tiles)
constexpr int kRowTokens = 16;    // tokens per CTA of the row RMS pass

template <typename T>
__device__ __forceinline__ float round_t(float v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(v));
  else return __half2float(__float2half_rn(v));
}

// 16-bit element k (0..7) of a 16-byte pack, widened to float.
template <typename T>
__device__ __forceinline__ float elem(const uint4& w, int k) {
  const uint32_t word = (&w.x)[k >> 1];
  const uint32_t h = (k & 1) ? (word >> 16) : (word & 0xffffu);
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(h << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__ldg(p));
  else return __half2float(__ldg(p));
}

template <typename T>
__device__ __forceinline__ uint16_t to_bits(float v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  else return __half_as_ushort(__float2half_rn(v));
}

// Two floats rounded to the 16-bit dtype and packed (lo = a, hi = b): the
// rounding is the one T(x) applies, done two at a time.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
template <typename T>
__device__ __forceinline__ float lo(uint32_t u) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(u << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(u & 0xffffu)));
}
template <typename T>
__device__ __forceinline__ float hi(uint32_t u) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(u & 0xffff0000u);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(u >> 16)));
}

// max(|lo|, |hi|) of a packed pair, as a packed pair (exact: 16-bit values).
template <typename T>
__device__ __forceinline__ uint32_t absmax2(uint32_t a, uint32_t b) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 r = __hmax2(__habs2(*reinterpret_cast<const __nv_bfloat162*>(&a)),
                                     __habs2(*reinterpret_cast<const __nv_bfloat162*>(&b)));
    return *reinterpret_cast<const uint32_t*>(&r);
  } else {
    const __half2 r = __hmax2(__habs2(*reinterpret_cast<const __half2*>(&a)),
                              __habs2(*reinterpret_cast<const __half2*>(&b)));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
}

// INT8 code of v * inv: clamp(rint(RN(v * inv)), -127, 127).  |RN(v * inv)|
// <= 127 * (1 + 2^-23) because |v| <= amax and inv = RN(127 / amax), so only
// NaN needs the clamp (fmaxf maps it to -127, as the reference's
// fminf(127, fmaxf(-127, NaN)) does); adding 1.5 * 2^23 rounds to the nearest
// integer, ties to even, and leaves it two's-complement in the low byte.
__device__ __forceinline__ uint32_t code_bits(float v, float inv) {
  return __float_as_uint(__fadd_rn(fmaxf(__fmul_rn(v, inv), -127.0f), 12582912.0f));
}
__device__ __forceinline__ uint32_t pack_codes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

struct QkRopeArgs {
  const void* in[2];        // Q, K
  int8_t* out[2];
  float* scale[2];
  const void* norm[2];      // [D] (head scope) or [heads * D] (row scope)
  float* rrms[2];           // row scope: [B, L] per token, else null
  const void* freqs;        // [fb, fs, 1, rot_dim/2, 2, 2] or null
  int heads[2], length[2], blocks[2];
  int64_t s_b[2], s_h[2], s_l[2];     // input strides (elements)
  int64_t o_b[2], o_h[2], o_l[2];     // output strides
  int64_t sc_b[2], sc_h[2];           // scale strides
  int64_t f_b, f_s, f_p, f_r, f_c;    // freqs strides
  int f_batches, f_seq;
  int rot_dim;
  int fast_freqs;           // interleaved, f_p == 4, f_r == 2, f_c == 1, 16-byte rows
  float eps;
  int row_scope;
  int rrms_given;           // row scope with the RRMS supplied by the caller
  int sum_only;             // row pass: write the sum of squares, not the RRMS
  void* proc[2];            // processed mode: T outputs (strides o_*), no codes
  int processed;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  // Zero-fill when !valid (source size 0; the address is still a valid one).
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

constexpr int kQkStages = 2;      // heads in flight per CTA (cp.async ring)

template <int D>
struct QkGeom {
  static constexpr int P = D / 8;                        // packs per token
  static constexpr int kTokPerIter = kQkThreads / P;     // 16 (D 128) or 32 (D 64)
  static constexpr int kIters = kQkBlock / kTokPerIter;  // 4 or 2
  static constexpr int kStageBytes = kIters * kQkThreads * 16;
  static constexpr int kFreqBytes = kIters * 2 * kQkThreads * 16;   // fast-path rotations
  static constexpr int kSmemBytes = kQkStages * kStageBytes + kFreqBytes;
};

// One 64-token block of Q (which = 0) or K (which = 1) for the heads
// [h0, h1): the tokens' rotations and row RRMS are loaded once, and each
// thread streams its own 16-byte packs of the next heads into a private
// cp.async ring while it works on the current head.
// PROC: write the normalized + rotated values (a.proc) instead of codes.
template <typename T, int D, bool SPLIT, bool PROC>
__device__ __forceinline__ void qk_block(const QkRopeArgs& a, int which, int blk, int h0, int h1,
                                         int batch, uint8_t* ring) {
  using G = QkGeom<D>;
  constexpr int P = G::P, kTokPerIter = G::kTokPerIter, kIters = G::kIters;
  constexpr int kWarps = kQkThreads / 32;
  __shared__ __align__(16) uint16_t nsm[SPLIT ? kQkBlock * D : 8];
  __shared__ float red[2][kWarps][kIters];
  __shared__ float inv_sm[2][4];

  const int tid = threadIdx.x, warp = tid >> 5;
  const int p = tid % P, tin = tid / P;
  const int L = a.length[which];
  const int tok0 = blk * kQkBlock;
  const T* in = static_cast<const T*>(a.in[which]) + static_cast<int64_t>(batch) * a.s_b[which] + p * 8;
  const uint32_t ring_s = smem_u32(ring) + tid * 16;

  // Per-token data shared by all heads: the row RRMS in registers, the
  // interleaved rotations (fast path) in a private shared-memory area filled
  // with the first ring group.
  const int rot = a.rot_dim;
  const T* freqs = static_cast<const T*>(a.freqs);
  const int64_t fbb = rot > 0 ? static_cast<int64_t>(a.f_batches == 1 ? 0 : batch) * a.f_b : 0;
  const bool fast = !SPLIT && a.fast_freqs && p * 8 + 8 <= rot;
  const uint32_t fr_s = smem_u32(ring) + kQkStages * G::kStageBytes + tid * 16;
  if (fast) {
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int tok = tok0 + it * kTokPerIter + tin;
      const T* f_tok = freqs + fbb + static_cast<int64_t>(a.f_seq == 1 ? 0 : tok) * a.f_s + p * 16;
      cp_async16(fr_s + (it * 2) * kQkThreads * 16, tok < L ? f_tok : freqs, tok < L);
      cp_async16(fr_s + (it * 2 + 1) * kQkThreads * 16, tok < L ? f_tok + 8 : freqs, tok < L);
    }
  }
  float rrms_row[kIters];
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int tok = tok0 + it * kTokPerIter + tin;
    rrms_row[it] = a.row_scope && tok < L ? __ldg(a.rrms[which] + static_cast<int64_t>(batch) * L + tok) : 0.0f;
  }

  auto issue = [&](int head, int stage) {
    if (head < h1) {
      const T* src = in + static_cast<int64_t>(head) * a.s_h[which];
#pragma unroll
      for (int it = 0; it < kIters; ++it) {
        const int tok = tok0 + it * kTokPerIter + tin;
        const bool ok = tok < L;
        cp_async16(ring_s + stage * G::kStageBytes + it * kQkThreads * 16,
                   ok ? static_cast<const void*>(src + static_cast<int64_t>(tok) * a.s_l[which])
                      : static_cast<const void*>(in),
                   ok);
      }
    }
    cp_async_commit();  // one group per slot, empty past the last head
  };
#pragma unroll
  for (int st = 0; st < kQkStages - 1; ++st) issue(h0 + st, st);

  const T* norm = static_cast<const T*>(a.norm[which]);
  uint4 wv_next = __ldg(reinterpret_cast<const uint4*>(norm + (a.row_scope ? h0 * D : 0) + p * 8));
  for (int head = h0; head < h1; ++head) {
    const int slot = (head - h0) % kQkStages;
    const int rb = (head - h0) & 1;  // red / inv_sm buffer: alternates by head
    issue(head + kQkStages - 1, (head - h0 + kQkStages - 1) % kQkStages);
    cp_async_wait<kQkStages - 1>();
    const uint4 wv = wv_next;
    if (a.row_scope && head + 1 < h1)  // the next head's weights, one head ahead
      wv_next = __ldg(reinterpret_cast<const uint4*>(norm + (head + 1) * D + p * 8));
    float w[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) w[c] = elem<T>(wv, c);

    // Normalize (once per element); v holds the T-rounded values as packed pairs.
    uint32_t v[kIters][4];
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int tok = tok0 + it * kTokPerIter + tin;
      const uint4 raw = *reinterpret_cast<const uint4*>(ring + (slot * G::kStageBytes + it * kQkThreads * 16 + tid * 16));
      float x[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) x[c] = elem<T>(raw, c);
      float rrms = rrms_row[it];
      if (!a.row_scope) {
        // 8-channel FMA chain, then the XOR tree over the token's P lanes
        // (every lane takes part, valid or not).
        float sum = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) sum = fmaf(x[c], x[c], sum);
#pragma unroll
        for (int o = P / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o, P);
        rrms = __frsqrt_rn(sum / static_cast<float>(D) + a.eps);
      }
      if (tok >= L) rrms = 0.0f;  // tokens past the end quantize zeros
#pragma unroll
      for (int c = 0; c < 8; c += 2)
        v[it][c >> 1] = pack2<T>(x[c] * rrms * w[c], x[c + 1] * rrms * w[c + 1]);
    }

    // RoPE.
    if (rot > 0) {
      if constexpr (SPLIT) {
        const int half = rot / 2;
        __syncthreads();  // the previous head's partners have been read
#pragma unroll
        for (int it = 0; it < kIters; ++it)
          *reinterpret_cast<uint4*>(nsm + (it * kTokPerIter + tin) * D + p * 8) =
              make_uint4(v[it][0], v[it][1], v[it][2], v[it][3]);
        __syncthreads();
        if (p * 8 < rot) {
#pragma unroll
          for (int it = 0; it < kIters; ++it) {
            const int tl = it * kTokPerIter + tin;
            const int tok = tok0 + tl;
            if (tok >= L) continue;
            const T* f_tok = freqs + fbb + static_cast<int64_t>(a.f_seq == 1 ? 0 : tok) * a.f_s;
            const uint16_t* row = nsm + tl * D;
            float r[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int ch = p * 8 + c;
              r[c] = (c & 1) ? hi<T>(v[it][c >> 1]) : lo<T>(v[it][c >> 1]);
              if (ch < rot) {
                const int comp = ch >= half;
                const int pair = comp ? ch - half : ch;
                const float x0 = lo<T>(row[pair]);
                const float x1 = lo<T>(row[pair + half]);
                const T* f = f_tok + pair * a.f_p + comp * a.f_r;
                r[c] = fmaf(ldf(f + a.f_c), x1, ldf(f) * x0);
              }
            }
#pragma unroll
            for (int c = 0; c < 8; c += 2) v[it][c >> 1] = pack2<T>(r[c], r[c + 1]);
          }
        }
      } else if (p * 8 < rot) {
#pragma unroll
        for (int it = 0; it < kIters; ++it) {
          const int tok = tok0 + it * kTokPerIter + tin;
          if (tok >= L) continue;
          const T* f_tok = freqs + fbb + static_cast<int64_t>(a.f_seq == 1 ? 0 : tok) * a.f_s;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // Pair q of the pack: (x0, x1) -> (f[0][0] x0 + f[0][1] x1, f[1][0] x0 + f[1][1] x1).
            const float x0 = lo<T>(v[it][q]), x1 = hi<T>(v[it][q]);
            float f00, f01, f10, f11;
            if (fast) {
              // [r0c0, r0c1, r1c0, r1c1] of four pairs, loaded once per block.
              const uint4 fq = *reinterpret_cast<const uint4*>(
                  ring + (kQkStages * G::kStageBytes + (it * 2 + (q >> 1)) * kQkThreads * 16 + tid * 16));
              const int b = (q & 1) * 4;
              f00 = elem<T>(fq, b); f01 = elem<T>(fq, b + 1);
              f10 = elem<T>(fq, b + 2); f11 = elem<T>(fq, b + 3);
            } else {
              const int pair = p * 4 + q;
              if (2 * pair >= rot) break;
              const T* f = f_tok + pair * a.f_p;
              f00 = ldf(f); f01 = ldf(f + a.f_c);
              f10 = ldf(f + a.f_r); f11 = ldf(f + a.f_r + a.f_c);
            }
            v[it][q] = pack2<T>(fmaf(f01, x1, f00 * x0), fmaf(f11, x1, f10 * x0));
          }
        }
      }
    }

    if constexpr (PROC) {
      // The normalized + rotated values themselves (already rounded to T).
      T* dst = static_cast<T*>(a.proc[which]) + static_cast<int64_t>(batch) * a.o_b[which] +
               static_cast<int64_t>(head) * a.o_h[which] + p * 8;
#pragma unroll
      for (int it = 0; it < kIters; ++it) {
        const int tok = tok0 + it * kTokPerIter + tin;
        if (tok < L)
          *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(tok) * a.o_l[which]) =
              make_uint4(v[it][0], v[it][1], v[it][2], v[it][3]);
      }
    } else {
      // Max |v| per iteration and warp, then per Q warp tile (16 tokens) or the K block.
#pragma unroll
      for (int it = 0; it < kIters; ++it) {
        const uint32_t m2 = absmax2<T>(absmax2<T>(v[it][0], v[it][1]), absmax2<T>(v[it][2], v[it][3]));
        float m = fmaxf(1e-7f, fmaxf(lo<T>(m2), hi<T>(m2)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((tid & 31) == 0) red[rb][warp][it] = m;
      }
      __syncthreads();
      const int n_tiles = which == 0 ? 4 : 1;
      if (tid < n_tiles) {
        // Warp w of iteration it covers tokens it*kTokPerIter + w*(32/P) .. + 32/P - 1.
        float m = 1e-7f;
#pragma unroll
        for (int it = 0; it < kIters; ++it)
#pragma unroll
          for (int wp = 0; wp < kWarps; ++wp) {
            const int t16 = (it * kTokPerIter + wp * (32 / P)) / 16;
            if (which == 1 || t16 == tid) m = fmaxf(m, red[rb][wp][it]);
          }
        a.scale[which][static_cast<int64_t>(batch) * a.sc_b[which] +
                       static_cast<int64_t>(head) * a.sc_h[which] + blk * n_tiles + tid] =
            __fdiv_rn(m, 127.0f);
        inv_sm[rb][tid] = __fdiv_rn(127.0f, m);
      }
      __syncthreads();
      float inv[kIters];
#pragma unroll
      for (int it = 0; it < kIters; ++it) inv[it] = inv_sm[rb][which == 0 ? (it * kTokPerIter + tin) / 16 : 0];
      // red / inv_sm alternate between two buffers: the next head writes the
      // other one, and the head after it passes two barriers first.

      int8_t* out = a.out[which] + static_cast<int64_t>(batch) * a.o_b[which] +
                    static_cast<int64_t>(head) * a.o_h[which] + p * 8;
#pragma unroll
      for (int it = 0; it < kIters; ++it) {
        const int tok = tok0 + it * kTokPerIter + tin;
        if (tok >= L) continue;
        uint32_t cb[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
          cb[c] = code_bits((c & 1) ? hi<T>(v[it][c >> 1]) : lo<T>(v[it][c >> 1]), inv[it]);
        const uint32_t wq[2] = {pack_codes(cb[0], cb[1], cb[2], cb[3]), pack_codes(cb[4], cb[5], cb[6], cb[7])};
        *reinterpret_cast<uint2*>(out + static_cast<int64_t>(tok) * a.o_l[which]) = make_uint2(wq[0], wq[1]);
      }
    }
  }
  cp_async_wait<0>();
}

// grid (Q tasks + K tasks, batch); a task is one 64-token block and one group
// of head_group consecutive heads.
template <typename T, int D, bool SPLIT, bool PROC>
__global__ void __launch_bounds__(kQkThreads, 3) qk_rms_rope_kernel(const QkRopeArgs a, int head_group) {
  extern __shared__ __align__(16) uint8_t ring[];
  const int task = blockIdx.x;
  const int batch = blockIdx.y;
  const int q_groups = (a.heads[0] + head_group - 1) / head_group;
  const int k_groups = (a.heads[1] + head_group - 1) / head_group;
  const int q_tasks = q_groups * a.blocks[0];
  const int which = task < q_tasks ? 0 : 1;
  const int local = which == 0 ? task : task - q_tasks;
  const int groups = which == 0 ? q_groups : k_groups;
  const int blk = local / groups, grp = local - blk * groups;
  const int h0 = grp * head_group;
  const int h1 = min(a.heads[which], h0 + head_group);
  qk_block<T, D, SPLIT, PROC>(a, which, blk, h0, h1, batch, ring);
}

// Row scope: RRMS of every token over all heads (qk_preprocess.cu:203-251).
// The reference gives thread t (of 256) the elements i = t, t + 256, ... of
// the token's H*D row, i = h*D + c: the channel c = t mod D and the heads
// h = t/D, t/D + 256/D, ...; each thread here owns one residue r = t/D and one
// 8-channel pack and keeps those 8 chains in the same head order.  The 256
// chains are then summed as the reference's block reduction does: an XOR
// butterfly over each warp's 32 consecutive t, then over the 8 warp sums
// padded with zeros to 32 lanes.
template <typename T, int D>
__global__ void __launch_bounds__(kQkThreads) row_rrms_kernel(const QkRopeArgs a, int q_groups) {
  constexpr int P = D / 8;
  constexpr int R = kQkThreads / D;           // head residues (2 or 4)
  constexpr int kItems = kRowTokens * R * P;  // 512
  __shared__ float chains[kRowTokens][kQkThreads];
  const int batch = blockIdx.y;
  const int which = static_cast<int>(blockIdx.x) < q_groups ? 0 : 1;
  const int grp = which == 0 ? blockIdx.x : blockIdx.x - q_groups;
  const int L = a.length[which], H = a.heads[which];
  const T* in = static_cast<const T*>(a.in[which]) + static_cast<int64_t>(batch) * a.s_b[which];
  const int tid = threadIdx.x;
#pragma unroll
  for (int k = 0; k < kItems / kQkThreads; ++k) {
    const int item = tid + k * kQkThreads;
    const int p = item % P, r = (item / P) % R, tl = item / (P * R);
    const int tok = grp * kRowTokens + tl;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    if (tok < L) {
      const T* base = in + static_cast<int64_t>(tok) * a.s_l[which] + p * 8;
      int h = r;
      for (; h + 3 * R < H; h += 4 * R) {
        uint4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          x[u] = __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(h + u * R) * a.s_h[which]));
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float e = elem<T>(x[u], c);
            acc[c] = fmaf(e, e, acc[c]);
          }
      }
      for (; h < H; h += R) {
        const uint4 x = __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(h) * a.s_h[which]));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float e = elem<T>(x, c);
          acc[c] = fmaf(e, e, acc[c]);
        }
      }
    }
    float4* dst = reinterpret_cast<float4*>(&chains[tl][r * D + p * 8]);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
  const int lane = tid & 31, warp = tid >> 5;
  const float n = static_cast<float>(H * D);
  for (int tl = warp; tl < kRowTokens; tl += kQkThreads / 32) {
    const int tok = grp * kRowTokens + tl;
    float ws[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float t = chains[tl][w * 32 + lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      ws[w] = t;
    }
    const float total = ((ws[0] + ws[4]) + (ws[2] + ws[6])) + ((ws[1] + ws[5]) + (ws[3] + ws[7]));
    if (lane == 0 && tok < L)
      a.rrms[which][static_cast<int64_t>(batch) * L + tok] =
          a.sum_only ? total : __frsqrt_rn(total / n + a.eps);
  }
}

}  // namespace

void row_rrms_launch(QkRopeArgs& a, int batch, int head_dim, int dtype, cudaStream_t stream) {
  const int q_groups = (a.length[0] + kRowTokens - 1) / kRowTokens;
  const int k_groups = (a.length[1] + kRowTokens - 1) / kRowTokens;
  const dim3 grid(static_cast<unsigned>(q_groups + k_groups), static_cast<unsigned>(batch));
#define TB_RR_LAUNCH(T, D) row_rrms_kernel<T, D><<<grid, kQkThreads, 0, stream>>>(a, q_groups)
  if (dtype == TB_DTYPE_BF16) {
    if (head_dim == 128) TB_RR_LAUNCH(__nv_bfloat16, 128); else TB_RR_LAUNCH(__nv_bfloat16, 64);
  } else {
    if (head_dim == 128) TB_RR_LAUNCH(__half, 128); else TB_RR_LAUNCH(__half, 64);
  }
#undef TB_RR_LAUNCH
  TB_CUDA_CHECK(cudaGetLastError());
}

void qk_rms_rope_launch(QkRopeArgs& a, int batch, int head_dim, int split_half, int dtype,
                        cudaStream_t stream) {
  if (a.row_scope && !a.rrms_given) row_rrms_launch(a, batch, head_dim, dtype, stream);
  // Heads per task: about 8, balanced over the head count, so the per-token
  // rotations and row RRMS are loaded once per 8 heads and the ring has a few
  // heads to run ahead on.
  const int max_heads = a.heads[0] > a.heads[1] ? a.heads[0] : a.heads[1];
  const int n_groups = (max_heads + 7) / 8;
  const int head_group = (max_heads + n_groups - 1) / n_groups;
  const int tasks = ((a.heads[0] + head_group - 1) / head_group) * a.blocks[0] +
                    ((a.heads[1] + head_group - 1) / head_group) * a.blocks[1];
  const dim3 grid(static_cast<unsigned>(tasks), static_cast<unsigned>(batch));
#define TB_QK_LAUNCH1(T, D, S, PR)                                                                \
  do {                                                                                            \
    static bool attr_set = false;                                                                 \
    if (!attr_set) {                                                                              \
      TB_CUDA_CHECK(cudaFuncSetAttribute(qk_rms_rope_kernel<T, D, S, PR>,                         \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,             \
                                         QkGeom<D>::kSmemBytes));                                 \
      attr_set = true;                                                                            \
    }                                                                                             \
    qk_rms_rope_kernel<T, D, S, PR><<<grid, kQkThreads, QkGeom<D>::kSmemBytes, stream>>>(a, head_group); \
  } while (0)
#define TB_QK_LAUNCH(T, D, S)                          \
  do {                                                 \
    if (a.processed) TB_QK_LAUNCH1(T, D, S, true);     \
    else TB_QK_LAUNCH1(T, D, S, false);                \
  } while (0)
  if (dtype == TB_DTYPE_BF16) {
    using T = __nv_bfloat16;
    if (head_dim == 128) { if (split_half) TB_QK_LAUNCH(T, 128, true); else TB_QK_LAUNCH(T, 128, false); }
    else { if (split_half) TB_QK_LAUNCH(T, 64, true); else TB_QK_LAUNCH(T, 64, false); }
  } else {
    using T = __half;
    if (head_dim == 128) { if (split_half) TB_QK_LAUNCH(T, 128, true); else TB_QK_LAUNCH(T, 128, false); }
    else { if (split_half) TB_QK_LAUNCH(T, 64, true); else TB_QK_LAUNCH(T, 64, false); }
  }
#undef TB_QK_LAUNCH
#undef TB_QK_LAUNCH1
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tb

using tb::guarded;

namespace {

// Checks and kernel arguments shared by the quantizing and the processed-value
// entries (outputs: INT8 codes + scales, or 16-bit values).
tb::QkRopeArgs prologue_args(const void* query, const void* key, void* query_out, void* key_out,
                             float* query_scale, float* key_scale, const void* query_norm,
                             const void* key_norm, const void* freqs, float* query_rrms,
                             float* key_rrms, int64_t batch, int64_t query_heads,
                             int64_t key_heads, int64_t query_length, int64_t key_length,
                             int64_t head_dim, const int64_t* strides, const int64_t* freq_strides,
                             int64_t freq_batches, int64_t freq_sequence, int64_t rot_dim,
                             int norm_scope, int split_half, int dtype, float epsilon,
                             bool processed) {
  TB_REQUIRE(query && key && query_out && key_out && query_norm && key_norm && strides,
             "Q/K, outputs and norm weights must be CUDA tensors");
  TB_REQUIRE(processed || (query_scale && key_scale), "scales must be CUDA tensors");
  TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16, "Q/K must be float16 or bfloat16");
  TB_REQUIRE(head_dim == 64 || head_dim == 128,
             "fused Q/K preprocessing requires head_dim 64 or 128");
  TB_REQUIRE(norm_scope >= 0 && norm_scope <= 2,
             "norm_scope must be 0 (per head), 1 (whole row) or 2 (whole row, RRMS given)");
  TB_REQUIRE(rot_dim >= 0 && rot_dim <= head_dim && rot_dim % 2 == 0,
             "rot_dim must be even and within head_dim");
  TB_REQUIRE(rot_dim == 0 || (freqs && freq_strides),
             "RoPE frequencies are required when rot_dim > 0");
  TB_REQUIRE(norm_scope == 0 || (query_rrms && key_rrms), "row RRMS scratch must be provided");
  TB_REQUIRE(batch > 0 && query_heads > 0 && key_heads > 0 && query_length > 0 && key_length > 0,
             "Q/K dimensions must be positive");
  TB_REQUIRE(batch <= 65535 && query_heads <= INT32_MAX && query_length <= INT32_MAX &&
                 key_length <= INT32_MAX,
             "Q/K dimensions exceed the CUDA kernel range");
  for (int i = 0; i < 12; ++i)
    TB_REQUIRE(strides[i] % 8 == 0,
               "Q/K and output strides must be multiples of 8 elements (16-byte packs)");
  TB_REQUIRE((reinterpret_cast<uintptr_t>(query) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(key) & 15u) == 0,
             "Q/K must be 16-byte aligned");
  const uintptr_t out_align = processed ? 15u : 7u;
  TB_REQUIRE((reinterpret_cast<uintptr_t>(query_out) & out_align) == 0 &&
                 (reinterpret_cast<uintptr_t>(key_out) & out_align) == 0,
             processed ? "the processed Q/K outputs must be 16-byte aligned"
                       : "the INT8 Q/K outputs must be 8-byte aligned");
  TB_REQUIRE((reinterpret_cast<uintptr_t>(query_norm) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(key_norm) & 15u) == 0,
             "Q/K norm weights must be 16-byte aligned");
  tb::QkRopeArgs a{};
  a.in[0] = query; a.in[1] = key;
  a.processed = processed ? 1 : 0;
  if (processed) {
    a.proc[0] = query_out; a.proc[1] = key_out;
  } else {
    a.out[0] = static_cast<int8_t*>(query_out); a.out[1] = static_cast<int8_t*>(key_out);
    a.scale[0] = query_scale; a.scale[1] = key_scale;
  }
  a.norm[0] = query_norm; a.norm[1] = key_norm;
  a.freqs = freqs;
  a.heads[0] = static_cast<int>(query_heads); a.heads[1] = static_cast<int>(key_heads);
  a.length[0] = static_cast<int>(query_length); a.length[1] = static_cast<int>(key_length);
  a.blocks[0] = static_cast<int>((query_length + 63) / 64);
  a.blocks[1] = static_cast<int>((key_length + 63) / 64);
  // strides: q (b, h, l), k (b, h, l), q_out (b, h, l), k_out (b, h, l) and,
  // quantizing, q_scale (b, h), k_scale (b, h).
  for (int w = 0; w < 2; ++w) {
    a.s_b[w] = strides[3 * w + 0]; a.s_h[w] = strides[3 * w + 1]; a.s_l[w] = strides[3 * w + 2];
    a.o_b[w] = strides[6 + 3 * w + 0]; a.o_h[w] = strides[6 + 3 * w + 1]; a.o_l[w] = strides[6 + 3 * w + 2];
    if (!processed) {
      a.sc_b[w] = strides[12 + 2 * w + 0]; a.sc_h[w] = strides[12 + 2 * w + 1];
    }
  }
  if (rot_dim > 0) {
    a.f_b = freq_strides[0]; a.f_s = freq_strides[1]; a.f_p = freq_strides[2];
    a.f_r = freq_strides[3]; a.f_c = freq_strides[4];
    a.f_batches = static_cast<int>(freq_batches);
    a.f_seq = static_cast<int>(freq_sequence);
    a.fast_freqs = !split_half && a.f_p == 4 && a.f_r == 2 && a.f_c == 1 && a.f_s % 8 == 0 &&
                   a.f_b % 8 == 0 && (reinterpret_cast<uintptr_t>(freqs) & 15u) == 0;
  } else {
    a.f_batches = a.f_seq = 1;
  }
  a.rot_dim = static_cast<int>(rot_dim);
  a.eps = epsilon;
  a.row_scope = norm_scope ? 1 : 0;
  a.rrms_given = norm_scope == 2;
  // Loads that the kernel skips at run time (no RoPE, head-scope norm) must
  // still name readable memory: the compiler may issue a guarded load ahead
  // of its guard (for example when hoisting it out of the per-head loop), so
  // the unused pointers name the inputs themselves, with zero strides for
  // the rotations.
  a.rrms[0] = norm_scope ? query_rrms : static_cast<float*>(const_cast<void*>(query));
  a.rrms[1] = norm_scope ? key_rrms : static_cast<float*>(const_cast<void*>(key));
  if (rot_dim == 0) {
    a.freqs = query;
    a.f_b = a.f_s = a.f_p = a.f_r = a.f_c = 0;
  }
  return a;
}

}  // namespace

extern "C" int tb_quant_qk_rms_rope_int8(
    const void* query, const void* key, int8_t* query_out, int8_t* key_out, float* query_scale,
    float* key_scale, const void* query_norm, const void* key_norm, const void* freqs,
    float* query_rrms, float* key_rrms, int64_t batch, int64_t query_heads, int64_t key_heads,
    int64_t query_length, int64_t key_length, int64_t head_dim, const int64_t* strides,
    const int64_t* freq_strides, int64_t freq_batches, int64_t freq_sequence, int64_t rot_dim,
    int norm_scope, int split_half, int dtype, float epsilon, tb_stream_t stream) {
  return guarded([&] {
    tb::QkRopeArgs a = prologue_args(query, key, query_out, key_out, query_scale, key_scale,
                                     query_norm, key_norm, freqs, query_rrms, key_rrms, batch,
                                     query_heads, key_heads, query_length, key_length, head_dim,
                                     strides, freq_strides, freq_batches, freq_sequence, rot_dim,
                                     norm_scope, split_half, dtype, epsilon, false);
    tb::require_sm100();
    tb::qk_rms_rope_launch(a, static_cast<int>(batch), static_cast<int>(head_dim), split_half,
                           dtype, static_cast<cudaStream_t>(stream));
  });
}

extern "C" int tb_qk_rms_rope_apply(
    const void* query, const void* key, void* query_out, void* key_out, const void* query_norm,
    const void* key_norm, const void* freqs, float* query_rrms, float* key_rrms, int64_t batch,
    int64_t query_heads, int64_t key_heads, int64_t query_length, int64_t key_length,
    int64_t head_dim, const int64_t* strides, const int64_t* freq_strides, int64_t freq_batches,
    int64_t freq_sequence, int64_t rot_dim, int norm_scope, int split_half, int dtype,
    float epsilon, tb_stream_t stream) {
  return guarded([&] {
    tb::QkRopeArgs a = prologue_args(query, key, query_out, key_out, nullptr, nullptr, query_norm,
                                     key_norm, freqs, query_rrms, key_rrms, batch, query_heads,
                                     key_heads, query_length, key_length, head_dim, strides,
                                     freq_strides, freq_batches, freq_sequence, rot_dim,
                                     norm_scope, split_half, dtype, epsilon, true);
    tb::require_sm100();
    tb::qk_rms_rope_launch(a, static_cast<int>(batch), static_cast<int>(head_dim), split_half,
                           dtype, static_cast<cudaStream_t>(stream));
  });
}

extern "C" int tb_row_sum_squares(const void* input, float* sums, int64_t batch, int64_t heads,
                                  int64_t length, int64_t head_dim, const int64_t* strides,
                                  int dtype, tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(input && sums && strides, "input, sums and strides must be given");
    TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16, "input must be float16 or bfloat16");
    TB_REQUIRE(head_dim == 64 || head_dim == 128, "head_dim must be 64 or 128");
    TB_REQUIRE(batch > 0 && heads > 0 && length > 0 && batch <= 65535 && length <= INT32_MAX &&
                   heads <= INT32_MAX,
               "dimensions must be positive and within the CUDA kernel range");
    for (int i = 0; i < 3; ++i)
      TB_REQUIRE(strides[i] % 8 == 0, "strides must be multiples of 8 elements (16-byte packs)");
    TB_REQUIRE((reinterpret_cast<uintptr_t>(input) & 15u) == 0, "input must be 16-byte aligned");
    tb::require_sm100();
    tb::QkRopeArgs a{};
    a.in[0] = a.in[1] = input;
    a.heads[0] = a.heads[1] = static_cast<int>(heads);
    a.length[0] = static_cast<int>(length);
    a.length[1] = 0;  // one tensor: the second half of the grid is empty
    a.s_b[0] = strides[0]; a.s_h[0] = strides[1]; a.s_l[0] = strides[2];
    a.rrms[0] = a.rrms[1] = sums;
    a.row_scope = 1;
    a.sum_only = 1;
    tb::row_rrms_launch(a, static_cast<int>(batch), static_cast<int>(head_dim), dtype,
                        static_cast<cudaStream_t>(stream));
  });
}

