// Sage INT8 attention for sm_100a (tcgen05 + TMA + TMEM).
//
// Semantics (kernel/csrc/turing/sage/qk_int_sv_f16_cuda_sm75.cu:48-830,
// attn_utils.cuh:465-585, 923-965): for each query row,
//   S_int = Q8 . K8^T                       (exact INT32, tensor core kind::i8)
//   s     = S_int * (sm_scale * log2 e * q_scale[row/16] * k_scale[key/64])
//   online softmax in base 2: m = running max, p = exp2(s - m),
//   d = sum p, O = sum p * V (fp32 accumulation), out = O / d.
// P and V enter the second contraction as 16-bit floats of V's dtype (bf16
// for bf16 V: the north-star "bf16 PV"; fp16 for fp16 V, as the reference).
// Keys >= Lk (and, when causal, keys after the query) are masked.  The
// running max is refreshed lazily: O and d are rescaled only when the row max
// grows by more than 2^8 over the reference point (p stays <= 256), which
// changes no result beyond rounding.
//
// CTA = 2 query tiles of 128 rows (256 rows of one head), keys in blocks of
// 64 (one k_scale block), 12 warps:
//   warps 0-7   softmax: warp w serves query tile w / 4 and TMEM lane
//               quadrant w % 4, one query row per thread;
//   warp 8      TMA producer: Q (once), then K (int8) and V (16-bit) blocks
//               of 64 keys into a 6-stage ring (128B swizzle);
//   warps 9-10  MMA issuers, one per query tile (warp 9 also owns TMEM):
//               S_t = Q_t K_j^T (kind::i8, M=128, N=64) and
//               O_t += P_t V_j (kind::f16, A = P read from TMEM, B = V
//               MN-major from shared memory);
//   warp 11     idle (it completes the control warpgroup).
// Each query tile has two S buffers: while the softmax turns S_t(j) into P,
// the tensor core already computes S_t(j+1), so the softmax warps of both
// tiles run back to back and never wait on the tensor core.  An issuing
// thread's barrier wait drains the tensor pipe (it is ordered after the
// shared-memory operand reads of the MMAs before it), so each tile has its
// own issuer and one issuer's waits overlap the other's MMAs.
// For a full block with an established reference point the Sage softmax
// takes the exponentials first and the row max in the same pass (the lazy
// reference rarely moves); a block whose max does move is read again from
// TMEM and redone after the rescale.  W8A8, whose exact running max moves
// often, always takes the row max first.
// TMEM columns: O0 [0,128) O1 [128,256) and S(t, b) at 256 + 128 t + 64 b;
// P_t(j) is written as packed 16-bit pairs over the first 32 columns of its
// S buffer.
//
// W8A8 variant (dense W8A8-PV, kernel/csrc/turing/sage/sol_sparse_cuda_sm75.cu:
// 1197-1320, attn_utils.cuh:465-625, 793-841): the reference point is the
// exact running max m = max_j fma(max_t s_t, c_j, -log2 255), so that
// p = 2^fma(s, c, -m) lies in (0, 255]; P enters PV as its u8 code rni(p)
// and V as its per-channel INT8 code, both carried as exact fp16 integers;
// d sums the unrounded p and the epilogue multiplies by the V channel scale.
// Every product and every 16-key partial sum of PV is an integer below 2^24,
// so the fp16 tensor path computes the reference's u8 x s8 products exactly;
// the fp32 accumulator in TMEM takes the rescale that an INT32 one could not.
// Every wait is bounded (tb_common.cuh).  Here the barrier probes carry no
// suspend-time hint: the waiting warps (softmax, issuers, producer) resume as
// soon as the phase completes, which measured 16.26 vs 16.99 ms (Sage) and
// 20.02 vs 20.32 ms (W8A8) at configs[1] on one B200 with identical outputs.
#define TB_TRY_WAIT_NO_HINT 1
#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

constexpr int kBlockM = 128;   // rows per query tile
constexpr int kQTiles = 2;     // query tiles per CTA
constexpr int kBlockN = 64;    // keys per KV block (= one k_scale block)
constexpr int kStages = 6;
constexpr int kThreads = 384;
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;    // warps 9 and 10: MMA issuers of tiles 0 and 1
constexpr uint32_t kOCols = 128;
constexpr uint32_t kSBase = 256;
// Pairs (bit i: pair i mod 16 of a block) whose exp2 runs on the FMA pipe.
#ifndef TB_ATTN_POLY_MASK
#define TB_ATTN_POLY_MASK 0x0000u
#endif
constexpr uint32_t kPolyPairMask = TB_ATTN_POLY_MASK;
// 1: a block's second 32 score columns load from TMEM while the first 32 are
// exponentiated.
#ifndef TB_ATTN_SPLIT_LD
#define TB_ATTN_SPLIT_LD 1
#endif
constexpr bool kSplitLd = TB_ATTN_SPLIT_LD != 0;


struct AttnParams {
  int B, Hq, Hk, Lq, Lk, groups;  // groups = Hq / Hk
  int q_tiles_scale;              // entries per (b, h) in q_scale
  int k_tiles_scale;              // entries per (b, h) in k_scale
  const float* q_scale;
  const float* k_scale;
  void* out;
  int64_t o_sb, o_sh, o_sl;       // output strides (elements)
  float* lse;                     // [B, Hq, Lq] base-2 or null
  float sm_scale_log2;            // sm_scale * log2(e)
  int causal;
  const float* v_scale;           // W8A8: [B, Hk, D] channel scales of the V codes
};

template <int D>
struct AttnSmem {
  static constexpr int kQBytes = kBlockM * D;          // int8
  static constexpr int kKBytes = kBlockN * D;          // int8
  static constexpr int kVBytes = kBlockN * D * 2;      // 16-bit
  static constexpr int kStageBytes = kKBytes + kVBytes;
  static constexpr int kDataBytes = kQTiles * kQBytes + kStages * kStageBytes;
};

struct __align__(8) AttnBarriers {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];          // one commit per issuer
  uint64_t s_full[kQTiles][2];         // S buffer b of tile t computed
  uint64_t p_full[kQTiles][2];         // the tile's 4 softmax warps stored P in buffer b
  uint64_t o_done[kQTiles];            // after each of the tile's last two PVs
  uint64_t o_final[kQTiles];           // after the tile's last PV
  uint64_t drain[kQTiles];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > TB_WAIT_TIMEOUT_NS) {
      record_device_error(kDevWaitTimeoutDrain);
      return;
    }
  }
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exact int32 -> float for |v| < 2^22 (|S| <= 127 * 127 * 128 < 2^21).
__device__ __forceinline__ float i2f_exact(int32_t v) {
  return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) {
  return __uint_as_float(static_cast<uint32_t>(v >> 32));
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// The helpers below keep each key pair in one 64-bit register pair built
// inside a single asm block (mov.b64 {lo, hi}), so the packed f32x2
// arithmetic needs no moves to assemble its operands.

// Float bits of 1.5 * 2^23 + s for a pair of int32 scores (exact for
// |s| < 2^22).
__device__ __forceinline__ uint64_t magic_pair(uint32_t s0, uint32_t s1) {
  uint64_t r;
  asm("{\n\t.reg .b32 a, b;\n\t"
      "add.s32 a, %1, 0x4B400000;\n\t"
      "add.s32 b, %2, 0x4B400000;\n\t"
      "mov.b64 %0, {a, b};\n\t}"
      : "=l"(r)
      : "r"(s0), "r"(s1));
  return r;
}

// 2^x of both halves on the MUFU unit.
__device__ __forceinline__ uint64_t ex2_pair(uint64_t x2) {
  uint64_t r;
  asm("{\n\t.reg .f32 a, b;\n\t"
      "mov.b64 {a, b}, %1;\n\t"
      "ex2.approx.ftz.f32 a, a;\n\t"
      "ex2.approx.ftz.f32 b, b;\n\t"
      "mov.b64 %0, {a, b};\n\t}"
      : "=l"(r)
      : "l"(x2));
  return r;
}

// 2^x of both halves on the FMA pipe.  x = n + f with n = rint(x) (the
// 1.5 * 2^23 rounding constant leaves n in the low mantissa bits of r) and f
// in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients are a
// minimax fit of the relative error on [-0.5, 0.5] (Remez exchange; max
// relative error 7.5e-5, far below the 2^-9 rounding of the 16-bit P); 2^n is
// added to the exponent field: bits(r) << 23 == n << 23 (mod 2^32).  x is
// clamped at -120 first (2^-120 is 0 for every later use) so the exponent
// stays in range; x < 128 holds because scores never exceed the reference by
// 2^8.
__device__ __forceinline__ uint64_t exp2_poly_pair(uint64_t x2) {
  asm("{\n\t.reg .f32 a, b;\n\t"
      "mov.b64 {a, b}, %0;\n\t"
      "max.f32 a, a, 0fC2F00000;\n\t"
      "max.f32 b, b, 0fC2F00000;\n\t"
      "mov.b64 %0, {a, b};\n\t}"
      : "+l"(x2));
  const uint64_t rnd = f2_pack(12582912.0f, 12582912.0f);
  const uint64_t r2 = f2_add(x2, rnd);
  const uint64_t fr = f2_sub(x2, f2_sub(r2, rnd));
  uint64_t q = f2_fma(fr, f2_pack(0.0551716685295105f, 0.0551716685295105f),
                      f2_pack(0.2426111251115799f, 0.2426111251115799f));
  q = f2_fma(q, fr, f2_pack(0.6932609677314758f, 0.6932609677314758f));
  q = f2_fma(q, fr, f2_pack(0.9999280571937561f, 0.9999280571937561f));
  uint64_t out;
  asm("{\n\t.reg .b32 q0, q1, r0, r1;\n\t"
      "mov.b64 {q0, q1}, %1;\n\t"
      "mov.b64 {r0, r1}, %2;\n\t"
      "shl.b32 r0, r0, 23;\n\t"
      "shl.b32 r1, r1, 23;\n\t"
      "add.s32 q0, q0, r0;\n\t"
      "add.s32 q1, q1, r1;\n\t"
      "mov.b64 %0, {q0, q1};\n\t}"
      : "=l"(out)
      : "l"(q), "l"(r2));
  return out;
}

template <typename TV>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<TV, __nv_bfloat16>::value) return pack_bf16x2(lo, hi);
  else return pack_f16x2(lo, hi);
}

// Both halves of a pair rounded to TV and packed (low half = even key).
template <typename TV>
__device__ __forceinline__ uint32_t pack_pair(uint64_t p2) {
  uint32_t r;
  if constexpr (std::is_same<TV, __nv_bfloat16>::value) {
    asm("{\n\t.reg .f32 a, b;\n\tmov.b64 {a, b}, %1;\n\tcvt.rn.bf16x2.f32 %0, b, a;\n\t}"
        : "=r"(r)
        : "l"(p2));
  } else {
    asm("{\n\t.reg .f32 a, b;\n\tmov.b64 {a, b}, %1;\n\tcvt.rn.f16x2.f32 %0, b, a;\n\t}"
        : "=r"(r)
        : "l"(p2));
  }
  return r;
}

// W8A8 P code of a pair: rni_sat_u8(p) as exact fp16 values.  Adding and
// subtracting 1.5 * 2^23 rounds p to the nearest integer (ties to even, as
// rni); the saturation at 255 (p reaches 255.5 only when |m| >= 2^16) is one
// packed fp16 min after the exact conversion of the integers <= 256.
__device__ __forceinline__ uint32_t u8_code_pair(uint64_t p2) {
  const uint64_t rnd2 = f2_pack(12582912.0f, 12582912.0f);
  uint32_t r = pack_pair<__half>(f2_sub(f2_add(p2, rnd2), rnd2));
  asm("min.f16x2 %0, %0, %1;" : "+r"(r) : "r"(0x5BF85BF8u));  // 255 in both halves
  return r;
}

// Exact floats of a pair of int32 scores (W8A8's fma(s, c, -m) needs s itself).
__device__ __forceinline__ uint64_t score_pair_f32(uint32_t s0, uint32_t s1) {
  uint64_t r;
  asm("{\n\t.reg .f32 a, b;\n\t"
      "cvt.rn.f32.s32 a, %1;\n\t"
      "cvt.rn.f32.s32 b, %2;\n\t"
      "mov.b64 %0, {a, b};\n\t}"
      : "=l"(r)
      : "r"(s0), "r"(s1));
  return r;
}

// The fast path of a full block: p = exp2(s * c - m_ref) against the current
// reference, in place as exp_block, with the integer row max of the raw
// scores accumulated in the same loop (the ALU work of the max hides under
// the exponentials).  Returns that max.  W8A8 as in exp_block.
template <typename TV, bool WAIT_HI, bool W8A8>
__device__ __forceinline__ int exp_block_max(uint32_t (&v)[kBlockN], uint64_t cx2, uint64_t bx2,
                                             uint64_t (&sum2)[2]) {
  int m[4] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};
#pragma unroll
  for (int i = 0; i < kBlockN / 2; ++i) {
    // Pairs 0..15 read columns 0..31 and write v[0..15]; the load of columns
    // 32..63 (still in flight when WAIT_HI) is waited for before pair 16.
    if (WAIT_HI && i == kBlockN / 4) tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(v + 32));
    m[i & 3] = __vimax3_s32(m[i & 3], static_cast<int>(v[2 * i]), static_cast<int>(v[2 * i + 1]));
    uint64_t x2;
    if constexpr (W8A8) x2 = f2_fma(score_pair_f32(v[2 * i], v[2 * i + 1]), cx2, bx2);
    else x2 = f2_fma(magic_pair(v[2 * i], v[2 * i + 1]), cx2, bx2);
    const uint64_t p2 =
        (!W8A8 && ((kPolyPairMask >> (i & 15)) & 1u)) ? exp2_poly_pair(x2) : ex2_pair(x2);
    sum2[i & 1] = f2_add(sum2[i & 1], p2);
    if constexpr (W8A8) v[i] = u8_code_pair(p2);
    else v[i] = pack_pair<TV>(p2);
  }
  return max(max(m[0], m[1]), max(m[2], m[3]));
}

// p = exp2(s * c - m_ref) for the 64 scores of a block, in place: packed pair
// i (16-bit P) overwrites v[i], whose score was consumed by pair i / 2.  The
// row sum of p accumulates in sum2.  MASKED zeroes keys >= valid; it is
// instantiated separately so full blocks carry no per-key selects.  (The
// reference scores masked keys -5e6, attn_utils.cuh:407-461, which gives them
// 2^(-5e6 c - m): exactly 0 in fp32 unless c < ~2.6e-5, i.e. unless Q/K scales
// are degenerate; there the reference's output carries the padding's mass and
// this kernel's does not.)
//
// W8A8: x = fma(s, c, -m) with s the exact float of the score (bx2 = -m) and
// P = the fp16 of rni_sat_u8(p) (the sum takes the unrounded p).
template <typename TV, bool MASKED, bool W8A8>
__device__ __forceinline__ void exp_block(uint32_t (&v)[kBlockN], uint64_t cx2, uint64_t bx2,
                                          int valid, uint64_t (&sum2)[2]) {
#pragma unroll
  for (int i = 0; i < kBlockN / 2; ++i) {
    uint64_t x2;
    if constexpr (W8A8) x2 = f2_fma(score_pair_f32(v[2 * i], v[2 * i + 1]), cx2, bx2);
    else x2 = f2_fma(magic_pair(v[2 * i], v[2 * i + 1]), cx2, bx2);
    uint64_t p2 = (!W8A8 && ((kPolyPairMask >> (i & 15)) & 1u)) ? exp2_poly_pair(x2) : ex2_pair(x2);
    if constexpr (MASKED) {
      p2 = f2_pack(2 * i < valid ? f2_lo(p2) : 0.0f, 2 * i + 1 < valid ? f2_hi(p2) : 0.0f);
    }
    sum2[i & 1] = f2_add(sum2[i & 1], p2);
    if constexpr (W8A8) v[i] = u8_code_pair(p2);
    else v[i] = pack_pair<TV>(p2);
  }
}

// TV: 16-bit type of P and V in the PV contraction; TO: output type.
template <int D, typename TV, typename TO, bool CAUSAL, bool W8A8>
__global__ void __launch_bounds__(kThreads, 1)
    sage_attn_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  using SM = AttnSmem<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* q_smem = smem;
  unsigned char* kv_smem = smem + kQTiles * SM::kQBytes;
  AttnBarriers* bar = reinterpret_cast<AttnBarriers*>(smem + SM::kDataBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qblk = blockIdx.x;          // 256-row block
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / p.groups;
  const int q0 = qblk * kBlockM * kQTiles;

  // KV blocks this CTA visits (causal: up to the last row of the block).
  int kv_len = p.Lk;
  if (CAUSAL) kv_len = min(p.Lk, q0 + kBlockM * kQTiles);
  const int n_kv = (kv_len + kBlockN - 1) / kBlockN;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar->kv_full[s], 1);
      mbar_init(&bar->kv_empty[s], kQTiles);
    }
    for (int t = 0; t < kQTiles; ++t) {
      for (int bb = 0; bb < 2; ++bb) {
        mbar_init(&bar->s_full[t][bb], 1);
        mbar_init(&bar->p_full[t][bb], 4);
      }
      mbar_init(&bar->o_done[t], 1);
      mbar_init(&bar->o_final[t], 1);
      mbar_init(&bar->drain[t], 1);
    }
    bar->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort_flag = &bar->abort_flag;
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_kv > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&bar->q_full, kQTiles * SM::kQBytes);
      for (int t = 0; t < kQTiles; ++t)
        tma_load_4d(q_smem + t * SM::kQBytes, &tm_q, &bar->q_full, 0, q0 + t * kBlockM, h, b);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        if (!mbar_wait(&bar->kv_empty[stage], phase ^ 1u, abort_flag, kDevWaitTimeoutProducer))
          break;
        unsigned char* k_dst = kv_smem + stage * SM::kStageBytes;
        unsigned char* v_dst = k_dst + SM::kKBytes;
        mbar_arrive_expect_tx(&bar->kv_full[stage], SM::kStageBytes);
        tma_load_4d(k_dst, &tm_k, &bar->kv_full[stage], 0, j * kBlockN, hk, b);
#pragma unroll
        for (int dh = 0; dh < D / 64; ++dh)
          tma_load_4d(v_dst + dh * (kBlockN * 128), &tm_v, &bar->kv_full[stage], dh * 64,
                      j * kBlockN, hk, b);
        ++issued;
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Drain: every copy issued by this CTA lands before it exits.
      drain_wait(&bar->q_full, 0);
      const int outstanding = issued < kStages ? issued : kStages;
      int s = stage;
      uint32_t ph = phase;
      for (int i = 0; i < outstanding; ++i) {
        if (--s < 0) {
          s = kStages - 1;
          ph ^= 1u;
        }
        drain_wait(&bar->kv_full[s], ph);
      }
    }
  } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
    // ------------------------------------------------------------ MMA issuers
    const int t = warp - kMmaWarp;  // query tile this thread serves
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_qk = idesc_i8(kBlockM, kBlockN);
      constexpr uint32_t idesc_pv =
          idesc_f16(kBlockM, D, std::is_same<TV, __nv_bfloat16>::value, /*b_mn_major=*/true);
      const uint32_t kv_addr = smem_u32(kv_smem);
      const uint32_t o_tmem = tmem + static_cast<uint32_t>(t) * kOCols;
      const uint32_t s_tmem0 = tmem + kSBase + static_cast<uint32_t>(t) * 2u * kBlockN;
      const uint64_t q_desc = umma_desc_sw128(smem_u32(q_smem) + t * SM::kQBytes);
      // S_t(j) = Q_t K_j^T into S buffer j % 2.
      auto issue_s = [&](int j) {
        const int stage = j % kStages;
        const uint32_t d_tmem = s_tmem0 + static_cast<uint32_t>(j & 1) * kBlockN;
        const uint64_t bk = umma_desc_sw128(kv_addr + stage * SM::kStageBytes);
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk)
          mma_i8_ss(d_tmem, q_desc + 2u * kk, bk + 2u * kk, idesc_qk, kk > 0 ? 1u : 0u);
      };
      auto wait_kv = [&](int j) {
        return mbar_wait(&bar->kv_full[j % kStages], static_cast<uint32_t>(j / kStages) & 1u,
                         abort_flag, kDevWaitTimeoutMma);
      };
      bool ok = mbar_wait(&bar->q_full, 0, abort_flag, kDevWaitTimeoutMma);
      for (int j = 0; j < 2 && j < n_kv && ok; ++j) {
        ok = wait_kv(j);
        if (ok) {
          tc_fence_after();
          issue_s(j);
          mma_commit(&bar->s_full[t][j & 1]);
        }
      }
      // Per block: both waits first (a barrier wait issued after an MMA would
      // wait for that MMA's shared-memory reads), then PV(j) and QK^T(j + 2)
      // back to back, then the commits.  The s_full commit of S_t(j + 2) also
      // tells the softmax that PV(j) is done; o_done marks the last two PVs,
      // which no S commit follows.
      for (int j = 0; j < n_kv && ok; ++j) {
        const bool next_s = j + 2 < n_kv;
        if (!mbar_wait(&bar->p_full[t][j & 1], static_cast<uint32_t>(j >> 1) & 1u, abort_flag,
                       kDevWaitTimeoutMma)) {
          ok = false;
          break;
        }
        if (next_s && !wait_kv(j + 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // O_t += P_t(j) V_j: 16 keys per MMA = two 8-row swizzle atoms of V
        // (2 x 1024 B); the D halves are separate TMA boxes kBlockN * 128 B
        // apart (LBO).
        const int stage = j % kStages;
        const uint32_t v_addr = kv_addr + stage * SM::kStageBytes + SM::kKBytes;
        const uint32_t p_tmem = s_tmem0 + static_cast<uint32_t>(j & 1) * kBlockN;
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          const uint64_t bv = umma_desc_sw128_mn(v_addr + kk * 2048, kBlockN * 128, 1024);
          mma_f16_ts(o_tmem, p_tmem + static_cast<uint32_t>(kk * 8), bv, idesc_pv,
                     (j > 0 || kk > 0) ? 1u : 0u);
        }
        // S buffer j % 2 is free once PV(j) has read P_t(j): S_t(j + 2).
        if (next_s) {
          issue_s(j + 2);
          mma_commit(&bar->s_full[t][j & 1]);
        } else {
          mma_commit(&bar->o_done[t]);
        }
        mma_commit(&bar->kv_empty[stage]);
        if (j + 1 == n_kv) mma_commit(&bar->o_final[t]);
      }
      mma_commit(&bar->drain[t]);
      drain_wait(&bar->drain[t], 0);
    }
  } else if (warp < kSoftmaxWarps) {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;              // query tile
    const int quad = warp & 3;            // TMEM lane quadrant
    const int r = quad * 32 + lane;       // row within the query tile
    const int row = q0 + t * kBlockM + r; // query row
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_tmem0 = tmem + lane_off + kSBase + static_cast<uint32_t>(t) * 2u * kBlockN;
    const uint32_t o_tmem = tmem + lane_off + static_cast<uint32_t>(t) * kOCols;
    const int bh = b * p.Hq + h;
    const float* ks_row = p.k_scale + static_cast<int64_t>(b * p.Hk + hk) * p.k_tiles_scale;
    const float qs = row < p.Lq
        ? __ldg(p.q_scale + static_cast<int64_t>(bh) * p.q_tiles_scale + row / 16) : 0.0f;
    const float cq = p.sm_scale_log2 * qs;
    float ks = n_kv > 0 ? __ldg(ks_row) : 0.0f;  // k_scale of block j, loaded one ahead
    float m_ref = -INFINITY;  // exponent reference point
    float dsum = 0.0f;        // row sum of p
    bool ok = n_kv > 0;
    // Control flow stays warp-uniform: tcgen05.ld / st are .sync.aligned
    // warp-collective instructions, so every decision that guards one is
    // taken by a warp vote.
    for (int j = 0; j < n_kv && ok; ++j) {
      const float c = cq * ks;
      if (j + 1 < n_kv) ks = __ldg(ks_row + j + 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&bar->s_full[t][j & 1],
                                             static_cast<uint32_t>(j >> 1) & 1u, abort_flag,
                                             kDevWaitTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      const uint32_t s_tmem = s_tmem0 + static_cast<uint32_t>(j & 1) * kBlockN;
      // Keys of this block visible to this row: [key0, key_end).
      const int key0 = j * kBlockN;
      int key_end = min(p.Lk, key0 + kBlockN);
      if (CAUSAL) key_end = min(key_end, row + 1);
      const int valid = key_end - key0;  // may be <= 0 (fully masked)
      uint32_t v[kBlockN];
      tmem_ld32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(v));
      if (kSplitLd) tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      if (!kSplitLd) tmem_wait_ld();
      bool hi_pending = kSplitLd;  // columns 32..63 still loading
      // Warp-uniform: full blocks take the paths without per-key selects.
      const bool all_full = __all_sync(0xffffffffu, valid >= kBlockN);
      const uint64_t cx2 = f2_pack(c, c);
      uint64_t sum2[2] = {0ull, 0ull};
      // x = s * c - m_ref = fma(t, c, b) with t = 1.5 * 2^23 + s (exact, by
      // integer addition to the float bits) and b = -(1.5 * 2^23 * c) - m_ref:
      // one packed FMA per key pair.
      bool done = false;
      bool need_rescale = false;  // some row of the warp moved its reference point
      float f = 1.0f;             // this row's rescale factor 2^(m_old - m_new)
      // Sage only: W8A8's exact running max moves in about a quarter of the
      // warp-blocks (any of 32 rows finding a new maximum), and redoing those
      // blocks costs more than taking the row max first every time
      // (configs[1]: 20.7 against 23.4 ms).
      if (!W8A8 && all_full && __all_sync(0xffffffffu, m_ref != -INFINITY)) {
        // Usual case: the reference point stands, so the exponentials need
        // not wait for the row max.  If any row's max moved past it, the
        // scores are read again and the block takes the general path.
        const float bb = W8A8 ? -m_ref : fmaf(-12582912.0f, c, -m_ref);
        const int mx = exp_block_max<TV, kSplitLd, W8A8>(v, cx2, f2_pack(bb, bb), sum2);
        hi_pending = false;
        done = !__any_sync(0xffffffffu, W8A8 ? fmaf(i2f_exact(mx), c, -7.9943534f) > m_ref
                                             : i2f_exact(mx) * c > m_ref + 8.0f);
        if (!done) {
          sum2[0] = sum2[1] = 0ull;
          tmem_ld32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(v));
          tmem_ld32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
          tmem_wait_ld();
        }
      }
      if (!done) {
        // Row max (integer max, then one multiply), over 16 columns at a
        // time; on a full block the first 32 columns while the last 32 load.
        auto max16 = [&](int q) {
          const uint32_t* w = v + 16 * q;
          int m = static_cast<int>(w[0]);
#pragma unroll
          for (int i = 1; i < 15; i += 2)
            m = __vimax3_s32(m, static_cast<int>(w[i]), static_cast<int>(w[i + 1]));
          return max(m, static_cast<int>(w[15]));
        };
        int a[4];
        if (all_full) {
          a[0] = max16(0);
          a[1] = max16(1);
          if (hi_pending) tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(v + 32));
          a[2] = max16(2);
          a[3] = max16(3);
        } else {
          if (hi_pending) tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(v + 32));
          // Ragged last block or causal diagonal: masked keys never win the
          // max and get p = 0 below.
#pragma unroll
          for (int i = 0; i < kBlockN; ++i)
            if (i >= valid) v[i] = static_cast<uint32_t>(INT32_MIN);
#pragma unroll
          for (int q = 0; q < 4; ++q) a[q] = max16(q);
        }
        const int mx = max(__vimax3_s32(a[0], a[1], a[2]), a[3]);
        // W8A8 keeps the reference's offset point fma(max, c, -log2 255).
        const float m_blk = mx == INT32_MIN ? -INFINITY
                            : W8A8          ? fmaf(i2f_exact(mx), c, -7.9943534f)
                                            : i2f_exact(mx) * c;
        // New reference point when the row max grew by more than 2^8 (W8A8:
        // at all); rows that already had one scale d now and O below, after
        // P(j) is stored, so the exponentials overlap the wait for PV(j - 1).
        const bool move = W8A8 ? m_blk > m_ref : m_blk > m_ref + 8.0f;
        const bool rescale = move && j > 0 && m_ref != -INFINITY;
        need_rescale = __any_sync(0xffffffffu, rescale);
        f = rescale ? ex2(m_ref - m_blk) : 1.0f;
        dsum *= f;
        if (move) m_ref = m_blk;
        const float nm = (m_ref == -INFINITY) ? 0.0f : -m_ref;
        const float bb = W8A8 ? nm : fmaf(-12582912.0f, c, nm);
        const uint64_t bx2 = f2_pack(bb, bb);
        if (all_full) exp_block<TV, false, W8A8>(v, cx2, bx2, valid, sum2);
        else exp_block<TV, true, W8A8>(v, cx2, bx2, valid, sum2);
      }
      tmem_st32(s_tmem, *reinterpret_cast<const uint32_t(*)[32]>(v));
      const uint64_t s01 = f2_add(sum2[0], sum2[1]);
      dsum += f2_lo(s01) + f2_hi(s01);
      if (need_rescale) {
        // O holds PV(0..j-1) once PV(j - 1) is done: the commit of
        // S_t(j + 1), issued right after PV(j - 1), marks it, and o_done
        // (phase 0) marks PV(n_kv - 2) when no S_t(j + 1) exists.  PV(j)
        // waits for this warp's p_full arrival below.
        const bool waited =
            j + 1 < n_kv
                ? mbar_wait(&bar->s_full[t][(j + 1) & 1], static_cast<uint32_t>((j + 1) >> 1) & 1u,
                            abort_flag, kDevWaitTimeoutSoftmax)
                : mbar_wait(&bar->o_done[t], 0u, abort_flag, kDevWaitTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, waited);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < D / 16; ++cc) {
          uint32_t o[16];
          tmem_ld16(o_tmem + cc * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st16(o_tmem + cc * 16, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full[t][j & 1]);
    }
    // Epilogue: O / d -> out (16-bit), optional base-2 LSE.
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar->o_final[t], 0u, abort_flag,
                                                   kDevWaitTimeoutSoftmax));
    if (ok) {
      tc_fence_after();
      const float inv = dsum > 0.0f ? 1.0f / dsum : 0.0f;
      TO* orow = static_cast<TO*>(p.out) + b * p.o_sb + h * p.o_sh +
                 static_cast<int64_t>(row) * p.o_sl;
      const float* vs = W8A8 ? p.v_scale + static_cast<int64_t>(b * p.Hk + hk) * D : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < D / 16; ++cc) {
        uint32_t o[16];
        tmem_ld16(o_tmem + cc * 16, o);
        tmem_wait_ld();
        float f[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(o[i]) * inv;
        if constexpr (W8A8) {
          // (O / d) * v_scale[c] (attn_utils.cuh:923-965 order).
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 s4 = __ldg(reinterpret_cast<const float4*>(vs + cc * 16 + i));
            f[i] *= s4.x;
            f[i + 1] *= s4.y;
            f[i + 2] *= s4.z;
            f[i + 3] *= s4.w;
          }
        }
        if (row < p.Lq) {
          uint4 w0 = make_uint4(pack2<TO>(f[0], f[1]), pack2<TO>(f[2], f[3]),
                                pack2<TO>(f[4], f[5]), pack2<TO>(f[6], f[7]));
          uint4 w1 = make_uint4(pack2<TO>(f[8], f[9]), pack2<TO>(f[10], f[11]),
                                pack2<TO>(f[12], f[13]), pack2<TO>(f[14], f[15]));
          *reinterpret_cast<uint4*>(orow + cc * 16) = w0;
          *reinterpret_cast<uint4*>(orow + cc * 16 + 8) = w1;
        }
      }
      if (p.lse != nullptr && row < p.Lq) {
        float l2;
        asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(l2) : "f"(dsum));
        p.lse[static_cast<int64_t>(bh) * p.Lq + row] = m_ref + l2;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

void make_map_4d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int64_t d_elems,
                 int64_t L, int64_t H, int64_t B, int64_t sl, int64_t sh, int64_t sb,
                 int elem_bytes, uint32_t box_inner, uint32_t box_rows) {
  const uint64_t dims[4] = {static_cast<uint64_t>(d_elems), static_cast<uint64_t>(L),
                            static_cast<uint64_t>(H), static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(sl * elem_bytes),
                               static_cast<uint64_t>(sh * elem_bytes),
                               static_cast<uint64_t>(sb * elem_bytes)};
  const uint32_t box[4] = {box_inner, box_rows, 1, 1};
  encode_tensor_map(map, dt, 4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

void sage_attn_launch(const AttnArgs& a, cudaStream_t stream) {
  const bool w8a8 = a.v_scale != nullptr;
  TB_REQUIRE(a.D == 128, "the sm_100a Sage attention kernel takes head_dim 128 (pad 64 < D < 128)");
  if (w8a8) {
    TB_REQUIRE(a.v_dtype == TB_DTYPE_F16, "W8A8 V codes must be the fp16 codes of the V quantizer");
    TB_REQUIRE(a.out_dtype == TB_DTYPE_BF16 || a.out_dtype == TB_DTYPE_F16,
               "output must be float16 or bfloat16");
    TB_REQUIRE(a.lse == nullptr, "the W8A8 attention returns no log-sum-exp");
    TB_REQUIRE((reinterpret_cast<uintptr_t>(a.v_scale) & 15u) == 0,
               "V scale must be 16-byte aligned");
  } else {
    TB_REQUIRE(a.v_dtype == a.out_dtype, "value and output dtypes must match");
    TB_REQUIRE(a.v_dtype == TB_DTYPE_BF16 || a.v_dtype == TB_DTYPE_F16,
               "value must be float16 or bfloat16");
  }
  TB_REQUIRE(a.Hq % a.Hk == 0, "num_qo_heads must be divisible by num_kv_heads");
  TB_REQUIRE(a.B <= 65535 && a.Hq <= 65535, "batch/head count exceeds the grid range");
  TB_REQUIRE(a.q_sl % 16 == 0 && a.q_sh % 16 == 0 && a.q_sb % 16 == 0 && a.k_sl % 16 == 0 &&
                 a.k_sh % 16 == 0 && a.k_sb % 16 == 0,
             "Q/K strides must be multiples of 16 bytes");
  TB_REQUIRE(a.v_sl % 8 == 0 && a.v_sh % 8 == 0 && a.v_sb % 8 == 0 && a.o_sl % 8 == 0,
             "V/O strides must be multiples of 16 bytes");
  TB_REQUIRE((reinterpret_cast<uintptr_t>(a.q) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(a.k) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(a.v) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0,
             "Q/K/V/O must be 16-byte aligned");
  constexpr int D = 128;
  CUtensorMap tq, tk, tv;
  make_map_4d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.q, D, a.Lq, a.Hq, a.B, a.q_sl, a.q_sh, a.q_sb,
              1, D, kBlockM);
  make_map_4d(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.k, D, a.Lk, a.Hk, a.B, a.k_sl, a.k_sh, a.k_sb,
              1, D, kBlockN);
  make_map_4d(&tv,
              a.v_dtype == TB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
              a.v, D, a.Lk, a.Hk, a.B, a.v_sl, a.v_sh, a.v_sb, 2, 64, kBlockN);
  AttnParams p{};
  p.B = static_cast<int>(a.B);
  p.Hq = static_cast<int>(a.Hq);
  p.Hk = static_cast<int>(a.Hk);
  p.Lq = static_cast<int>(a.Lq);
  p.Lk = static_cast<int>(a.Lk);
  p.groups = static_cast<int>(a.Hq / a.Hk);
  p.q_tiles_scale = static_cast<int>(a.q_tiles_scale);
  p.k_tiles_scale = static_cast<int>(a.k_tiles_scale);
  p.q_scale = a.q_scale;
  p.k_scale = a.k_scale;
  p.out = a.out;
  p.o_sb = a.o_sb;
  p.o_sh = a.o_sh;
  p.o_sl = a.o_sl;
  p.lse = a.lse;
  p.sm_scale_log2 = a.sm_scale * 1.4426950408889634f;
  p.causal = a.causal;
  p.v_scale = a.v_scale;
  const size_t smem = AttnSmem<D>::kDataBytes + sizeof(AttnBarriers) + 1024;
  dim3 grid(static_cast<unsigned>((a.Lq + kBlockM * kQTiles - 1) / (kBlockM * kQTiles)),
            static_cast<unsigned>(a.Hq), static_cast<unsigned>(a.B));
#define TB_ATTN_LAUNCH(TV, TO, CAUSAL, W8A8)                                            \
  {                                                                                     \
    auto kern = sage_attn_kernel<D, TV, TO, CAUSAL, W8A8>;                              \
    TB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                       static_cast<int>(smem)));                        \
    kern<<<grid, kThreads, smem, stream>>>(tq, tk, tv, p);                              \
  }
  if (w8a8) {
    if (a.out_dtype == TB_DTYPE_BF16) {
      if (a.causal) TB_ATTN_LAUNCH(__half, __nv_bfloat16, true, true)
      else TB_ATTN_LAUNCH(__half, __nv_bfloat16, false, true)
    } else {
      if (a.causal) TB_ATTN_LAUNCH(__half, __half, true, true)
      else TB_ATTN_LAUNCH(__half, __half, false, true)
    }
  } else if (a.v_dtype == TB_DTYPE_BF16) {
    if (a.causal) TB_ATTN_LAUNCH(__nv_bfloat16, __nv_bfloat16, true, false)
    else TB_ATTN_LAUNCH(__nv_bfloat16, __nv_bfloat16, false, false)
  } else {
    if (a.causal) TB_ATTN_LAUNCH(__half, __half, true, false)
    else TB_ATTN_LAUNCH(__half, __half, false, false)
  }
#undef TB_ATTN_LAUNCH
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tb
