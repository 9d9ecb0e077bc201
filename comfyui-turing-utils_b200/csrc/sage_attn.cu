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
// CTA = 2 query tiles of 128 rows (256 rows of one head), 20 warps:
//   warps 0-15  softmax: warp w serves query tile w / 8, key half (w / 4) % 2
//               (keys 0-63 or 64-127 of each 128-key tile, and the matching
//               64 O columns) and TMEM lane quadrant w % 4 (one query row per
//               thread).  Four softmax warps per SM sub-partition keep the
//               exp (MUFU) and integer/float pipes fed; the two query tiles
//               run independently, so one tile's exponentials overlap the
//               tensor work of the other.
//   warp 16     TMA producer: Q (once), then K (int8) and V (16-bit) tiles of
//               128 keys into a 3-stage ring (128B swizzle);
//   warp 17     TMEM owner + MMA issuer, alternating the two query tiles:
//               S_t = Q_t K_j^T (kind::i8, M=N=128) into TMEM, then
//               O_t += P_t V_j (kind::f16, A = P read from TMEM, B = V
//               MN-major from shared memory);
//   warps 18-19 idle (they complete the control warpgroup).
// A softmax thread reads its 64 scores with one TMEM wait, takes their max
// with 3-input integer max, combines it with the other half's through shared
// memory and an mbarrier, and forms p with packed f32x2 arithmetic (exact
// int->float by the 2^23 magic constant, then scale and exponent offset) and
// one ex2 per element.  Row sums are kept per half and added in the epilogue.
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512); P_t is
// written as packed 16-bit pairs over the first 64 columns of S_t.
// Every wait is bounded (tb_common.cuh).
#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

constexpr int kBlockM = 128;   // rows per query tile
constexpr int kQTiles = 2;     // query tiles per CTA
constexpr int kBlockN = 128;   // keys per KV tile
constexpr int kStages = 3;
constexpr int kThreads = 640;
constexpr int kSoftmaxWarps = 16;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;

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
  uint64_t kv_empty[kStages];
  uint64_t s_full[kQTiles];
  uint64_t p_full[kQTiles];
  uint64_t o_done[kQTiles];
  uint64_t drain;
  uint64_t max_ready[kQTiles];  // both halves posted their partial row max
  uint64_t sum_ready[kQTiles];  // both halves posted their row sums
  float row_max[kQTiles][2][kBlockM];  // per-half partial max of each row
  float row_sum[kQTiles][2][kBlockM];  // epilogue: per-half row sums
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

template <typename TV>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<TV, __nv_bfloat16>::value) return pack_bf16x2(lo, hi);
  else return pack_f16x2(lo, hi);
}

template <int D, typename TV, bool CAUSAL>
// Launched at <= 96 registers per thread (640 threads, 61,440 registers);
// after set-up the control warpgroup (warps 16-19) gives registers back
// (setmaxnreg.dec to 40) and the four softmax warpgroups take them
// (setmaxnreg.inc to 104): 128 x 40 + 512 x 104 = 58,368 <= 61,440, and per
// SM sub-partition 4 x 32 x 104 + 32 x 40 = 14,592 <= 16,384.
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

  // KV tiles this CTA visits (causal: up to the last row of the block).
  int kv_len = p.Lk;
  if (CAUSAL) kv_len = min(p.Lk, q0 + kBlockM * kQTiles);
  const int n_kv = (kv_len + kBlockN - 1) / kBlockN;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar->kv_full[s], 1);
      mbar_init(&bar->kv_empty[s], 1);
    }
    for (int t = 0; t < kQTiles; ++t) {
      mbar_init(&bar->s_full[t], 1);
      mbar_init(&bar->p_full[t], 8);
      mbar_init(&bar->o_done[t], 1);
      mbar_init(&bar->max_ready[t], 8);
      mbar_init(&bar->sum_ready[t], 8);
    }
    mbar_init(&bar->drain, 1);
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
  if (warp >= kSoftmaxWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
  }
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
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_qk = idesc_i8(kBlockM, kBlockN);
      constexpr uint32_t idesc_pv =
          idesc_f16(kBlockM, D, std::is_same<TV, __nv_bfloat16>::value, /*b_mn_major=*/true);
      const uint32_t q_addr = smem_u32(q_smem);
      const uint32_t kv_addr = smem_u32(kv_smem);
      bool ok = mbar_wait(&bar->q_full, 0, abort_flag, kDevWaitTimeoutMma);
      // S_t(j) = Q_t K_j^T
      auto issue_s = [&](int t, int stage) {
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(t * 128);
        const uint64_t a = umma_desc_sw128(q_addr + t * SM::kQBytes);
        const uint64_t bk = umma_desc_sw128(kv_addr + stage * SM::kStageBytes);
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk)
          mma_i8_ss(d_tmem, a + 2u * kk, bk + 2u * kk, idesc_qk, kk > 0 ? 1u : 0u);
        mma_commit(&bar->s_full[t]);
      };
      // O_t += P_t V_j
      auto issue_pv = [&](int t, int stage, int j) {
        const uint32_t d_tmem = tmem + 256u + static_cast<uint32_t>(t * 128);
        const uint32_t p_tmem = tmem + static_cast<uint32_t>(t * 128);
        const uint32_t v_addr = kv_addr + stage * SM::kStageBytes + SM::kKBytes;
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          // 16 keys per MMA = two 8-row swizzle atoms (2 x 1024 B); the D
          // halves are separate TMA boxes kBlockN * 128 B apart (LBO).
          const uint64_t bv = umma_desc_sw128_mn(v_addr + kk * 2048, kBlockN * 128, 1024);
          mma_f16_ts(d_tmem, p_tmem + static_cast<uint32_t>(kk * 8), bv, idesc_pv,
                     (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bar->o_done[t]);
      };
      if (ok) ok = mbar_wait(&bar->kv_full[0], 0, abort_flag, kDevWaitTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      int stage = 0;
      uint32_t phase = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int next_stage = stage + 1 == kStages ? 0 : stage + 1;
        const uint32_t next_phase = next_stage == 0 ? phase ^ 1u : phase;
        for (int t = 0; t < kQTiles; ++t) {
          if (!mbar_wait(&bar->p_full[t], static_cast<uint32_t>(j) & 1u, abort_flag,
                         kDevWaitTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, stage, j);
          if (t == kQTiles - 1) mma_commit(&bar->kv_empty[stage]);
          if (j + 1 < n_kv) {
            if (t == 0 && !mbar_wait(&bar->kv_full[next_stage], next_phase, abort_flag,
                                     kDevWaitTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(t, next_stage);
          }
        }
        stage = next_stage;
        phase = next_phase;
      }
      mma_commit(&bar->drain);
      drain_wait(&bar->drain, 0);
    }
  } else if (warp < kSoftmaxWarps) {
    // ------------------------------------------------------------ softmax
    asm volatile("setmaxnreg.inc.sync.aligned.u32 104;\n" ::: "memory");
    const int t = warp >> 3;              // query tile
    const int half = (warp >> 2) & 1;     // key half of each tile / O column half
    const int quad = warp & 3;            // TMEM lane quadrant
    const int r = quad * 32 + lane;       // row within the query tile
    const int row = q0 + t * kBlockM + r; // query row
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_tmem = tmem + lane_off + static_cast<uint32_t>(t * 128 + half * 64);
    const uint32_t p_tmem = tmem + lane_off + static_cast<uint32_t>(t * 128 + half * 32);
    const uint32_t o_tmem = tmem + lane_off + 256u + static_cast<uint32_t>(t * 128 + half * 64);
    const int bh = b * p.Hq + h;
    const float* ks_row = p.k_scale + static_cast<int64_t>(b * p.Hk + hk) * p.k_tiles_scale;
    const float qs = row < p.Lq
        ? __ldg(p.q_scale + static_cast<int64_t>(bh) * p.q_tiles_scale + row / 16) : 0.0f;
    const float cq = p.sm_scale_log2 * qs;
    float m_ref = -INFINITY;  // exponent reference point
    float dsum = 0.0f;        // this half's row sum
    bool ok = n_kv > 0;
    // Control flow stays warp-uniform: tcgen05.ld / st are .sync.aligned
    // warp-collective instructions, so every decision that guards one is
    // taken by a warp vote.
    for (int j = 0; j < n_kv && ok; ++j) {
      const int key0 = j * kBlockN + half * 64;
      const float c = key0 < p.Lk ? cq * __ldg(ks_row + 2 * j + half) : 0.0f;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar->s_full[t], static_cast<uint32_t>(j) & 1u,
                                             abort_flag, kDevWaitTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      // Keys of this half visible to this row: [key0, key_end).
      int key_end = min(p.Lk, key0 + 64);
      if (CAUSAL) key_end = min(key_end, row + 1);
      const int valid = key_end - key0;  // may be <= 0 (fully masked)
      uint32_t v[64];
      tmem_ld32(s_tmem + 0, *reinterpret_cast<uint32_t(*)[32]>(v + 0));
      tmem_ld32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_wait_ld();
      const bool full = valid >= 64;
      if (!full) {
        // Ragged last tile or causal diagonal: masked keys never win the max
        // and get p = 0 below.
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= valid) v[i] = static_cast<uint32_t>(INT32_MIN);
      }
      int mx;
      {
        int a[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          int m = static_cast<int>(v[16 * q]);
#pragma unroll
          for (int i = 1; i < 15; i += 2)
            m = __vimax3_s32(m, static_cast<int>(v[16 * q + i]), static_cast<int>(v[16 * q + i + 1]));
          a[q] = max(m, static_cast<int>(v[16 * q + 15]));
        }
        mx = max(__vimax3_s32(a[0], a[1], a[2]), a[3]);
      }
      // Row max over both halves: partial maxima meet in shared memory.
      bar->row_max[t][half][r] = mx != INT32_MIN ? i2f_exact(mx) * c : -INFINITY;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->max_ready[t]);
      ok = __all_sync(0xffffffffu, mbar_wait(&bar->max_ready[t], static_cast<uint32_t>(j) & 1u,
                                             abort_flag, kDevWaitTimeoutSoftmax));
      if (!ok) break;
      const float m_tile = fmaxf(bar->row_max[t][0][r], bar->row_max[t][1][r]);
      // New reference point when the row max grew by more than 2^8; rows that
      // already had one rescale O and d (O is complete up to tile j-1).
      const bool move = m_tile > m_ref + 8.0f;
      const bool rescale = move && j > 0 && m_ref != -INFINITY;
      if (__any_sync(0xffffffffu, rescale)) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&bar->o_done[t], static_cast<uint32_t>(j - 1) & 1u, abort_flag,
                                  kDevWaitTimeoutSoftmax));
        if (!ok) break;
        tc_fence_after();
        const float f = rescale ? ex2(m_ref - m_tile) : 1.0f;
        dsum *= f;
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[16];
          tmem_ld16(o_tmem + cc * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st16(o_tmem + cc * 16, o);
        }
        tmem_wait_st();
      }
      if (move) m_ref = m_tile;
      // p = exp2(s * c - m_ref) on packed pairs; partial row sum; 16-bit P
      // packed in place over the consumed scores, then into TMEM (this
      // half's 32 packed columns of the first 64 of S_t).
      const float nm = (m_ref == -INFINITY) ? 0.0f : -m_ref;
      const uint64_t magic2 = f2_pack(12582912.0f, 12582912.0f);
      const uint64_t cx2 = f2_pack(c, c), nmx2 = f2_pack(nm, nm);
      uint64_t sum2[2] = {0ull, 0ull};
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const uint64_t t2 = f2_pack(__int_as_float(static_cast<int>(v[i]) + 0x4B400000),
                                    __int_as_float(static_cast<int>(v[i + 1]) + 0x4B400000));
        const uint64_t x2 = f2_fma(f2_sub(t2, magic2), cx2, nmx2);
        float p0 = ex2(f2_lo(x2)), p1 = ex2(f2_hi(x2));
        if (!full) {
          p0 = i < valid ? p0 : 0.0f;
          p1 = i + 1 < valid ? p1 : 0.0f;
        }
        sum2[(i >> 1) & 1] = f2_add(sum2[(i >> 1) & 1], f2_pack(p0, p1));
        v[i >> 1] = pack2<TV>(p0, p1);
      }
      tmem_st32(p_tmem, *reinterpret_cast<uint32_t(*)[32]>(v + 0));
      const uint64_t s01 = f2_add(sum2[0], sum2[1]);
      dsum += f2_lo(s01) + f2_hi(s01);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full[t]);
    }
    // Epilogue: O / d -> out (16-bit), optional base-2 LSE.  Each half owns
    // 64 O columns; the row sum is the sum of the two halves' partial sums.
    bar->row_sum[t][half][r] = dsum;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar->sum_ready[t]);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar->sum_ready[t], 0, abort_flag,
                                                   kDevWaitTimeoutSoftmax));
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar->o_done[t],
                                                   static_cast<uint32_t>(n_kv - 1) & 1u,
                                                   abort_flag, kDevWaitTimeoutSoftmax));
    if (ok) {
      tc_fence_after();
      const float d = bar->row_sum[t][0][r] + bar->row_sum[t][1][r];
      const float inv = d > 0.0f ? 1.0f / d : 0.0f;
      TV* orow = static_cast<TV*>(p.out) + b * p.o_sb + h * p.o_sh +
                 static_cast<int64_t>(row) * p.o_sl + half * 64;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[16];
        tmem_ld16(o_tmem + cc * 16, o);
        tmem_wait_ld();
        if (row < p.Lq) {
          uint4 w0 = make_uint4(pack2<TV>(__uint_as_float(o[0]) * inv, __uint_as_float(o[1]) * inv),
                                pack2<TV>(__uint_as_float(o[2]) * inv, __uint_as_float(o[3]) * inv),
                                pack2<TV>(__uint_as_float(o[4]) * inv, __uint_as_float(o[5]) * inv),
                                pack2<TV>(__uint_as_float(o[6]) * inv, __uint_as_float(o[7]) * inv));
          uint4 w1 = make_uint4(pack2<TV>(__uint_as_float(o[8]) * inv, __uint_as_float(o[9]) * inv),
                                pack2<TV>(__uint_as_float(o[10]) * inv, __uint_as_float(o[11]) * inv),
                                pack2<TV>(__uint_as_float(o[12]) * inv, __uint_as_float(o[13]) * inv),
                                pack2<TV>(__uint_as_float(o[14]) * inv, __uint_as_float(o[15]) * inv));
          *reinterpret_cast<uint4*>(orow + cc * 16) = w0;
          *reinterpret_cast<uint4*>(orow + cc * 16 + 8) = w1;
        }
      }
      if (p.lse != nullptr && row < p.Lq && half == 0) {
        float l2;
        asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(l2) : "f"(d));
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
};

void sage_attn_launch(const AttnArgs& a, cudaStream_t stream) {
  TB_REQUIRE(a.D == 128, "the sm_100a Sage attention kernel takes head_dim 128 (pad 64 < D < 128)");
  TB_REQUIRE(a.v_dtype == a.out_dtype, "value and output dtypes must match");
  TB_REQUIRE(a.v_dtype == TB_DTYPE_BF16 || a.v_dtype == TB_DTYPE_F16,
             "value must be float16 or bfloat16");
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
  const size_t smem = AttnSmem<D>::kDataBytes + sizeof(AttnBarriers) + 1024;
  dim3 grid(static_cast<unsigned>((a.Lq + kBlockM * kQTiles - 1) / (kBlockM * kQTiles)),
            static_cast<unsigned>(a.Hq), static_cast<unsigned>(a.B));
#define TB_ATTN_LAUNCH(TV, CAUSAL)                                                      \
  {                                                                                     \
    auto kern = sage_attn_kernel<D, TV, CAUSAL>;                                        \
    TB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                       static_cast<int>(smem)));                        \
    kern<<<grid, kThreads, smem, stream>>>(tq, tk, tv, p);                              \
  }
  if (a.v_dtype == TB_DTYPE_BF16) {
    if (a.causal) TB_ATTN_LAUNCH(__nv_bfloat16, true) else TB_ATTN_LAUNCH(__nv_bfloat16, false)
  } else {
    if (a.causal) TB_ATTN_LAUNCH(__half, true) else TB_ATTN_LAUNCH(__half, false)
  }
#undef TB_ATTN_LAUNCH
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tb
