// INT8 x INT8 -> INT32 GEMM on sm_100a tensor cores (tcgen05.mma kind::i8)
// with the W8A8 dequant epilogue of the reference fused on the TMEM read-out:
//   out[m, n] = bf16_rn(((float)acc[m, n] * a_s[m]) * w_s[n] + bias[n])
// (kernel/csrc/turing/w4a8.cu:474-525 EVT tree; one rounding at the bf16
// store), or the raw INT32 accumulators (acc mode, bit-exact test hook and
// the input of turing_dequantize_int8_bf16).
//
// Two forms with the same results bit for bit.  The default runs clusters of
// two CTAs whose tensor cores act as one (tcgen05 .cta_group::2) on 256 x 256
// tiles (gemm_i8_pair_kernel below: each SM loads 32 KB per K-block instead
// of 48 KB; 2430 vs 2270 TOPS at configs[0], 2910 vs 2550 TOPS at the DiT
// block's Q/K/V GEMM on one B200).  TB_GEMM_PAIR=0 selects the single-CTA
// form, whose structure (one CTA per SM, persistent over 128 x 256 output
// tiles) is:
//   warp 0      TMA producer: A [128 x 128 B] and B [256 x 128 B] K-blocks,
//               128-byte swizzle, into a 4-stage shared-memory ring;
//   warp 1      TMEM allocator + MMA issuer: 4 x tcgen05.mma (M=128, N=256,
//               K=32) per K-block into one of two 256-column TMEM
//               accumulators, tcgen05.commit to release ring stages;
//   warps 2..5  epilogue: tcgen05.ld of the accumulator rows (one row per
//               thread), scale/bias/cast, 16-byte global stores; releases the
//               accumulator so the next tile's MMAs overlap this epilogue.
// A and B are both K-major (act [M, K] row-major, weight [N, K] row-major),
// matching the reference's RowMajor A / ColumnMajor B (w4a8.cu:388-391).
// Partial tiles rely on TMA zero fill (K tail, M tail, N tail); the epilogue
// masks rows >= M and columns >= N.
#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 128;  // bytes = int8 elements per K-block (one 128B swizzle row)
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK;
constexpr int kBBytes = kBN * kBK;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;

enum EpiMode { kEpiBf16 = 0, kEpiS32 = 1 };

struct GemmParams {
  int m, n, k;
  int num_m_blocks, num_n_blocks, num_k_blocks;
  int num_tiles;
  int group_m;   // M-blocks per tile group (tile_coords)
  const float* a_scale;  // [m]
  const float* w_scale;  // [n]
  const float* bias;     // [n] or null
  void* out;             // bf16 [m, ldo] or int32 [m, ldo]
  int64_t ldo;
};

constexpr int kStages2 = 6;  // ring depth of the CTA-pair form

struct __align__(8) GemmShared2 {
  uint64_t full[kStages2];
  uint64_t empty[kStages2];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct __align__(8) GemmShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// Tiles run in groups of group_m M-blocks; inside a group the M-block varies
// fastest, then the N-block.  The group's A rows (group_m * 128 * K bytes,
// sized to stay in L2) are then reused across every N-block instead of
// streaming all of A from HBM once per N-block, which is what an M-fastest
// order does once A outgrows L2.  The last group may hold fewer M-blocks.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& m0, int& n0) {
  const int per_group = p.group_m * p.num_n_blocks;
  const int g = tile / per_group;
  const int first_m = g * p.group_m;
  const int rows = min(p.group_m, p.num_m_blocks - first_m);
  const int local = tile - g * per_group;
  m0 = (first_m + local % rows) * kBM;
  n0 = (local / rows) * kBN;
}

// Waits without honouring the abort flag: used on the exit path to drain
// copies / MMAs this CTA issued before it deallocates TMEM and returns.
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

// Epilogue of one row's 32 accumulator columns [col0, col0 + 32): bf16 of
// ((float(acc) * a_s) * w_s + bias) (two roundings, no FMA: the reference's
// EVT order), or the raw INT32 values; columns >= N are skipped.
template <int EPI>
__device__ __forceinline__ void store_row_chunk(const GemmParams& p, int row, int col0, float a_s,
                                                const uint32_t (&r)[32]) {
  if constexpr (EPI == kEpiBf16) {
    __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int cb = col0 + g * 8;
      if (cb >= p.n) break;  // n % 8 == 0: an 8-column group is all in or all out
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int n = cb + j;
        float t = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(r[g * 8 + j])), a_s),
                            __ldg(p.w_scale + n));
        if (p.bias != nullptr) t = __fadd_rn(t, __ldg(p.bias + n));
        v[j] = t;
      }
      uint4 packed = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
      *reinterpret_cast<uint4*>(orow + cb) = packed;
    }
  } else {
    int32_t* orow = static_cast<int32_t*>(p.out) + static_cast<int64_t>(row) * p.ldo;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const int cb = col0 + g * 4;
      if (cb >= p.n) break;
      *reinterpret_cast<uint4*>(orow + cb) =
          make_uint4(r[g * 4], r[g * 4 + 1], r[g * 4 + 2], r[g * 4 + 3]);
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, const GemmParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // Stage buffers must be 1024-byte aligned for the 128B swizzle atoms.
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  GemmShared* sh = reinterpret_cast<GemmShared*>(smem + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh->acc_full[a], 1);
      mbar_init(&sh->acc_empty[a], 4);
    }
    mbar_init(&sh->drain, 1);
    sh->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = sh->tmem_base;
  volatile int* abort_flag = &sh->abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int m0, n0;
        tile_coords(p, tile, m0, n0);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&sh->empty[stage], phase ^ 1u, abort_flag, kDevWaitTimeoutProducer)) {
            ok = false;
            break;
          }
          unsigned char* a_dst = smem + stage * kStageBytes;
          unsigned char* b_dst = a_dst + kABytes;
          mbar_arrive_expect_tx(&sh->full[stage], kStageBytes);
          tma_load_2d(a_dst, &tmap_a, &sh->full[stage], kb * kBK, m0);
          tma_load_2d(b_dst, &tmap_b, &sh->full[stage], kb * kBK, n0);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every load this CTA issued has landed before it may exit.
      const int outstanding = issued < kStages ? static_cast<int>(issued) : kStages;
      int s = stage;
      uint32_t ph = phase;
      for (int j = 0; j < outstanding; ++j) {
        if (--s < 0) {
          s = kStages - 1;
          ph ^= 1u;
        }
        drain_wait(&sh->full[s], ph);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kBM, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>(local >> 1) & 1u;
        if (!mbar_wait(&sh->acc_empty[acc], acc_phase ^ 1u, abort_flag, kDevWaitTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&sh->full[stage], phase, abort_flag, kDevWaitTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * kStageBytes);
          const uint32_t b_addr = a_addr + kABytes;
          const uint64_t a_desc = umma_desc_sw128(a_addr);
          const uint64_t b_desc = umma_desc_sw128(b_addr);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {
            // +32 bytes along K inside the 128-byte swizzle row = +2 in the
            // descriptor's 16-byte address field.
            mma_i8_ss(d_tmem, a_desc + 2u * kk, b_desc + 2u * kk, idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&sh->empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&sh->acc_full[acc]);
      }
      // Drain: all MMAs issued by this thread complete before TMEM is freed.
      mma_commit(&sh->drain);
      drain_wait(&sh->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(local >> 1) & 1u;
      // Warp vote: the tcgen05.ld below is warp-collective.
      if (!__all_sync(0xffffffffu, mbar_wait(&sh->acc_full[acc], acc_phase, abort_flag,
                                             kDevWaitTimeoutEpilogue)))
        break;
      tc_fence_after();
      int m0, n0;
      tile_coords(p, tile, m0, n0);
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.m;
      const float a_s = (EPI == kEpiBf16 && row_ok) ? __ldg(p.a_scale + row) : 0.0f;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * kBN);
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_wait_ld();
        const int col0 = n0 + c * 32;
        if (!row_ok || col0 >= p.n) continue;
        store_row_chunk<EPI>(p, row, col0, a_s, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

constexpr size_t kGemmSmem = kStages * kStageBytes + sizeof(GemmShared) + 1024;

// ------------------------------------------------------------ CTA-pair form
// The same GEMM on 256 x 256 output tiles computed by a cluster of two CTAs
// whose tensor cores act as one (tcgen05 .cta_group::2, M = 256, N = 256,
// K = 32 per MMA).  CTA rank r of the pair loads its own 128 rows of A
// (tile rows 128 r ..) and half of the tile's B rows (n0 + 128 r ..) into its
// shared memory, so each SM brings in 32 KB per 128-deep K-block instead of
// 48 KB; rank 0 (the leader) issues the MMAs, which read A and B from both
// CTAs and write each CTA's 128 accumulator rows into its own TMEM.
//   full[s]      leader only: both CTAs' loads of stage s (the peer's TMA
//                counts its bytes on the leader's barrier);
//   empty[s]     both CTAs: stage s consumed (one commit, multicast);
//   acc_full[a]  both CTAs: accumulator a complete (one commit, multicast);
//   acc_empty[a] leader only: the 4 epilogue warps of both CTAs read it.
// No TMA multicast: every load reads global memory into its own CTA.
constexpr int kBM2 = 256;            // tile rows per pair (128 per CTA)
constexpr int kHalf = 128;           // A rows / B rows per CTA
constexpr int kAHalfBytes = kHalf * kBK;
constexpr int kBHalfBytes = kHalf * kBK;
constexpr int kStageBytes2 = kAHalfBytes + kBHalfBytes;

__device__ __forceinline__ void tile_coords2(const GemmParams& p, int tile, int& m0, int& n0) {
  const int per_group = p.group_m * p.num_n_blocks;
  const int g = tile / per_group;
  const int first_m = g * p.group_m;
  const int rows = min(p.group_m, p.num_m_blocks - first_m);
  const int local = tile - g * per_group;
  m0 = (first_m + local % rows) * kBM2;
  n0 = (local / rows) * kBN;
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b, const GemmParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  GemmShared2* sh = reinterpret_cast<GemmShared2*>(smem + kStages2 * kStageBytes2);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh->acc_full[a], 1);
      mbar_init(&sh->acc_empty[a], 8);
    }
    mbar_init(&sh->drain, 1);
    sh->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&sh->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers exist before either CTA signals the other's.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = sh->tmem_base;
  volatile int* abort_flag = &sh->abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ producers
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += pairs) {
        int m0, n0;
        tile_coords2(p, tile, m0, n0);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&sh->empty[stage], phase ^ 1u, abort_flag, kDevWaitTimeoutProducer)) {
            ok = false;
            break;
          }
          unsigned char* a_dst = smem + stage * kStageBytes2;
          unsigned char* b_dst = a_dst + kAHalfBytes;
          const uint32_t full_leader = mapa_shared(smem_u32(&sh->full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&sh->full[stage], 2 * kStageBytes2);
          tma_load_2d_pair(a_dst, &tmap_a, full_leader, kb * kBK, m0 + kHalf * static_cast<int>(rank));
          tma_load_2d_pair(b_dst, &tmap_b, full_leader, kb * kBK, n0 + kHalf * static_cast<int>(rank));
          ++issued;
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain (leader): the full barriers count both CTAs' loads, so every
      // load of the pair has landed before the final cluster barrier lets
      // either CTA exit.  (After a normal run the MMAs consumed them all.)
      if (leader) {
        const int outstanding = issued < kStages2 ? static_cast<int>(issued) : kStages2;
        int s = stage;
        uint32_t ph = phase;
        for (int j = 0; j < outstanding; ++j) {
          if (--s < 0) {
            s = kStages2 - 1;
            ph ^= 1u;
          }
          drain_wait(&sh->full[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kBM2, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>(local >> 1) & 1u;
        if (!mbar_wait(&sh->acc_empty[acc], acc_phase ^ 1u, abort_flag, kDevWaitTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(&sh->full[stage], phase, abort_flag, kDevWaitTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * kStageBytes2);
          const uint64_t a_desc = umma_desc_sw128(a_addr);
          const uint64_t b_desc = umma_desc_sw128(a_addr + kAHalfBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            mma_i8_ss_pair(d_tmem, a_desc + 2u * kk, b_desc + 2u * kk, idesc,
                           (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit_pair(&sh->empty[stage], 0x3);
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(&sh->acc_full[acc], 0x3);
      }
      // Drain: all MMAs of the pair complete before either CTA frees TMEM.
      mma_commit_pair(&sh->drain, 0x3);
      drain_wait(&sh->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int row_in_tile = kHalf * static_cast<int>(rank) + quad * 32 + lane;
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&sh->acc_empty[0]), 0);
    int local = 0;
    for (int tile = pair; tile < p.num_tiles; tile += pairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(local >> 1) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&sh->acc_full[acc], acc_phase, abort_flag,
                                             kDevWaitTimeoutEpilogue)))
        break;
      tc_fence_after();
      int m0, n0;
      tile_coords2(p, tile, m0, n0);
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.m;
      const float a_s = (EPI == kEpiBf16 && row_ok) ? __ldg(p.a_scale + row) : 0.0f;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * kBN);
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_wait_ld();
        const int col0 = n0 + c * 32;
        if (!row_ok || col0 >= p.n) continue;
        store_row_chunk<EPI>(p, row, col0, a_s, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + static_cast<uint32_t>(acc) * 8u);
    }
  }

  tc_fence_before();
  // Neither CTA leaves (or frees TMEM) while the other may still signal it.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

constexpr size_t kGemmSmem2 = kStages2 * kStageBytes2 + sizeof(GemmShared2) + 1024;

void make_kmajor_i8_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k,
                        int box_rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(k)};
  const uint32_t box[2] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(box_rows)};
  encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

// The CTA-pair kernel is used unless TB_GEMM_PAIR=0 is set in the
// environment (read at every launch, so a process can compare the two forms).
bool use_pair_kernel() {
  const char* v = getenv("TB_GEMM_PAIR");
  return v == nullptr || v[0] != '0';
}

// Largest number of CTA pairs the device holds at once (one CTA per SM; a
// pair occupies two SMs of one cluster slot).  Sets the kernels' shared
// memory limit on first use; cached per device.
int pair_kernel_max_clusters(int epi) {
  static int cached[64][2] = {};
  int dev = 0;
  TB_CUDA_CHECK(cudaGetDevice(&dev));
  const int e = epi == kEpiS32 ? 1 : 0;
  if (dev < 64 && cached[dev][e] > 0) return cached[dev][e];
  const void* fn = epi == kEpiS32 ? reinterpret_cast<const void*>(gemm_i8_pair_kernel<kEpiS32>)
                                  : reinterpret_cast<const void*>(gemm_i8_pair_kernel<kEpiBf16>);
  TB_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kGemmSmem2)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(device_sm_count() / 2 * 2), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kGemmSmem2;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  TB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg));
  TB_REQUIRE(clusters > 0, "the CTA-pair GEMM does not fit on this device");
  if (dev < 64) cached[dev][e] = clusters;
  return clusters;
}

}  // namespace

// Launches the tcgen05 GEMM.  `out` is bf16 (epi = 0) or int32 (epi = 1).
void gemm_i8_launch(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                    const float* a_scale, const float* w_scale, const float* bias, void* out,
                    int64_t ldo, int epi, cudaStream_t stream) {
  TB_REQUIRE(m > 0 && n > 0 && k > 0, "GEMM dimensions must be positive");
  TB_REQUIRE(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX,
             "GEMM dimensions exceed the CUDA kernel range");
  TB_REQUIRE(k % 16 == 0, "K must be a multiple of 16 (16-byte TMA row pitch)");
  TB_REQUIRE(epi == kEpiS32 ? (n % 4 == 0) : (n % 8 == 0), "N must be a multiple of 8");
  TB_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0,
             "activation and weight must be 16-byte aligned");
  TB_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15u) == 0 && ldo >= n &&
                 (ldo * (epi == kEpiS32 ? 4 : 2)) % 16 == 0,
             "output must be 16-byte aligned with a 16-byte row pitch");
  CUtensorMap tmap_a, tmap_b;
  make_kmajor_i8_map(&tmap_a, a, m, k, kBM);
  make_kmajor_i8_map(&tmap_b, w, n, k, kBN);
  GemmParams p{};
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.num_m_blocks = static_cast<int>((m + kBM - 1) / kBM);
  p.num_n_blocks = static_cast<int>((n + kBN - 1) / kBN);
  p.num_k_blocks = static_cast<int>((k + kBK - 1) / kBK);
  p.num_tiles = p.num_m_blocks * p.num_n_blocks;
  // About 24 MB of A rows per group: with the weight (B) that the group
  // sweeps, it fits the 126 MB L2.
  constexpr int64_t kGroupABytes = 24ll << 20;
  const int64_t gm = kGroupABytes / (static_cast<int64_t>(kBM) * k);
  p.group_m = static_cast<int>(gm < 1 ? 1 : (gm > p.num_m_blocks ? p.num_m_blocks : gm));
  p.a_scale = a_scale;
  p.w_scale = w_scale;
  p.bias = bias;
  p.out = out;
  p.ldo = ldo;
  if (use_pair_kernel()) {
    // CTA pairs over 256 x 256 tiles; B is loaded in 128-row halves.
    make_kmajor_i8_map(&tmap_b, w, n, k, kHalf);
    p.num_m_blocks = static_cast<int>((m + kBM2 - 1) / kBM2);
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    const int64_t gm2 = kGroupABytes / (static_cast<int64_t>(kBM2) * k);
    p.group_m = static_cast<int>(gm2 < 1 ? 1 : (gm2 > p.num_m_blocks ? p.num_m_blocks : gm2));
    const int max_pairs = pair_kernel_max_clusters(epi);
    const int pairs = p.num_tiles < max_pairs ? p.num_tiles : max_pairs;
    if (epi == kEpiS32) {
      gemm_i8_pair_kernel<kEpiS32><<<2 * pairs, kThreads, kGemmSmem2, stream>>>(tmap_a, tmap_b, p);
    } else {
      gemm_i8_pair_kernel<kEpiBf16><<<2 * pairs, kThreads, kGemmSmem2, stream>>>(tmap_a, tmap_b, p);
    }
    TB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int sms = device_sm_count();
  const int grid = p.num_tiles < sms ? p.num_tiles : sms;
  if (epi == kEpiS32) {
    auto kern = gemm_i8_kernel<kEpiS32>;
    TB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kGemmSmem)));
    kern<<<grid, kThreads, kGemmSmem, stream>>>(tmap_a, tmap_b, p);
  } else {
    auto kern = gemm_i8_kernel<kEpiBf16>;
    TB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kGemmSmem)));
    kern<<<grid, kThreads, kGemmSmem, stream>>>(tmap_a, tmap_b, p);
  }
  TB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tb
