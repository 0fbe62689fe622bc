// Dense BF16 GEMM on CTA pairs: one 256 x 256 output tile per pair of SMs.
//
// tcgen05.mma.cta_group::2 lets two CTAs of a cluster share one MMA: each CTA holds 128
// of the 256 A rows and 128 of the 256 B rows of the tile in its own shared memory and
// receives its 128 accumulator rows in its own TMEM.  Per MMA of 2 * 256 * 256 * 16 FLOP a
// CTA therefore stages 16 KB of A and 16 KB of B instead of 16 KB + 32 KB, which cuts
// the L2 -> shared-memory traffic of the main loop by a third.  Every load is a plain
// cp.async.bulk.tensor (no cluster multicast); the peer's loads signal the leader's
// "full" barrier, the leader's single MMA thread issues for the pair and its commits
// arrive on the barriers of both CTAs.
//
// Roles per CTA as in gemm_bf16.cuh: warp 0 TMA producer, warp 1 TMEM allocator (+ MMA
// issuer in the leader), warps 2..5 epilogue of this CTA's 128 rows.
#pragma once

#include "gemm_bf16.cuh"

namespace b200 {

constexpr int kPairTileM = 256;
// per CTA and stage: 128 rows of A (16 KB) + BN/2 rows of B
template <int BN>
__host__ __device__ constexpr int pair_stage_bytes() {
  return kBlockP * kBlockK * 2 + (BN / 2) * kBlockK * 2;
}

template <int STAGES>
struct PairSmemTail {
  uint64_t full[STAGES];      // leader's copy is the one in use (expects both CTAs' bytes)
  uint64_t empty[STAGES];     // each CTA waits on its own copy
  uint64_t tmem_full[2];      // each CTA waits on its own copy
  uint64_t tmem_empty[2];     // leader's copy: 8 arrivals = 4 epilogue warps x 2 CTAs
  uint32_t tmem_slot;
  int abort_flag;
};

template <int STAGES, int BN>
constexpr size_t gemm_pair_smem_bytes() {
  return 1024 + size_t(STAGES) * pair_stage_bytes<BN>() + sizeof(PairSmemTail<STAGES>);
}

// status code: the two CTAs of a pair were given different TMEM base columns
enum PairCode { kPairTmemMismatch = 9 };

struct PairUnit {
  int m0, n0;
};

template <int BN>
__device__ __forceinline__ PairUnit pair_decode(int u, int tiles_m, int tiles_n) {
  // groups of 8 row tiles (2048 rows) sweep the column tiles together
  constexpr int kGroup = 8;
  const int per_group = kGroup * tiles_n;
  const int g = u / per_group;
  const int r = u - g * per_group;
  const int gsz = min(kGroup, tiles_m - g * kGroup);
  const int nt = r / gsz;
  const int mt = g * kGroup + (r - nt * gsz);
  return PairUnit{mt * kPairTileM, nt * BN};
}

// BN = 256 or 128 output columns per tile (the narrower tile halves the unit of work, which
// matters when the tile count is a small non-multiple of the 74 CTA pairs).
template <int STAGES, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                          const __grid_constant__ CUtensorMap map_b, const GemmArgs args) {
  using Tail = PairSmemTail<STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_aligned = smem_raw + (smem_base - smem_u32(smem_raw));
  constexpr int kStageBytes = pair_stage_bytes<BN>();
  constexpr int kTmemCols = 2 * BN;  // two accumulator buffers (256 or 512 columns)
  Tail* tail = reinterpret_cast<Tail*>(smem_aligned + size_t(STAGES) * kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();  // 0 = leader
  const AbortCtx ctx{&tail->abort_flag, args.status};

  if (threadIdx.x == 0) {
    tail->abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&tail->full[s]), 1);
      mbar_init(smem_u32(&tail->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tail->tmem_full[b]), 1);
      mbar_init(smem_u32(&tail->tmem_empty[b]), 8);
    }
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) tmem_alloc(smem_u32(&tail->tmem_slot), kTmemCols);
  // nothing above reads or writes global memory: it may overlap the previous kernel's tail
  griddep_wait();
  griddep_launch_dependents();
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // barriers of both CTAs are initialised before any remote arrival
  tc_fence_after_sync();

  const uint32_t tmem_base = tail->tmem_slot;
  // The leader's MMA addresses the accumulators of both CTAs by the leader's TMEM base, while
  // each CTA's epilogue reads at its own: the two allocations must have landed on the same
  // columns.  (They do when no other kernel holds tensor memory on either SM; a mismatch is
  // reported through the status word and the pair does no work.)
  if (threadIdx.x == 0 && rank == 1) {
    const uint32_t leader_base = ld_shared_cluster_u32(map_to_cta(smem_u32(&tail->tmem_slot), 0));
    if (leader_base != tmem_base) {
      tail->abort_flag = 1;
      atomicCAS(args.status, 0, (kPairTmemMismatch << 16) | static_cast<int>(blockIdx.x & 0xffffu));
    }
  }
  const int tiles_m = ceil_div(args.M, kPairTileM);
  const int tiles_n = ceil_div(args.N, BN);
  const int total_units = tiles_m * tiles_n;
  const int k_blocks = ceil_div(args.K, kBlockK);
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (warp == 0) {
    // ======================= TMA producer (both CTAs) ======================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair_id; u < total_units && ok; u += num_pairs) {
        const PairUnit t = pair_decode<BN>(u, tiles_m, tiles_n);
        const int a_row = t.m0 + int(rank) * kBlockP;
        const int b_row = t.n0 + int(rank) * (BN / 2);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, ctx, kWaitEmptyStage)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = map_to_cta(smem_u32(&tail->full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(smem_u32(&tail->full[stage]), 2 * kStageBytes);
          const uint32_t sa = smem_base + stage * kStageBytes;
          const uint32_t sb = sa + kBlockP * kBlockK * 2;
          tma_load_2d_pair(sa, &map_a, leader_full, kb * kBlockK, a_row);
          tma_load_2d_pair(sb, &map_b, leader_full, kb * kBlockK, b_row);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer (leader only) ======================
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kPairTileM, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = pair_id; u < total_units && ok; u += num_pairs, ++it) {
        const int buf = it & 1;
        const uint32_t buf_phase = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&tail->tmem_empty[buf]), buf_phase ^ 1u, ctx, kWaitTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&tail->full[stage]), phase, ctx, kWaitFullStage)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sa = smem_base + stage * kStageBytes;
          const uint32_t sb = sa + kBlockP * kBlockK * 2;
#pragma unroll
          for (int k = 0; k < kBlockK / kUmmaK; ++k) {
            umma_bf16_ss_pair(d_tmem, make_smem_desc_sw128(sa + k * kUmmaK * 2, 0, 1024),
                              make_smem_desc_sw128(sb + k * kUmmaK * 2, 0, 1024), idesc,
                              (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&tail->empty[stage]), 3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_pair(smem_u32(&tail->tmem_full[buf]), 3);
      }
    }
  } else {
    // ======================= epilogue (both CTAs) ==========================
    const int quad = warp & 3;
    const int p = quad * 32 + lane;
    const bool vec_ok = (args.ldo % 8 == 0) && ((reinterpret_cast<uintptr_t>(args.out) & 15) == 0);
    int it = 0;
    bool ok = true;
    for (int u = pair_id; u < total_units && ok; u += num_pairs, ++it) {
      const PairUnit t = pair_decode<BN>(u, tiles_m, tiles_n);
      const int buf = it & 1;
      const uint32_t buf_phase = (it >> 1) & 1;
      if (!mbar_wait(smem_u32(&tail->tmem_full[buf]), buf_phase, ctx, kWaitTmemFull)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after_sync();
      const uint32_t t_acc = tmem_base + (uint32_t(quad * 32) << 16) + buf * BN;
      const int row = t.m0 + int(rank) * kBlockP + p;
      const bool row_ok = row < args.M;
      const int cols_valid = min(BN, args.N - t.n0);
      __nv_bfloat16* orow = args.out + size_t(row) * args.ldo + t.n0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_acc + c * 32, v);
        tmem_ld_wait();
        if (row_ok) {
          const int col0 = c * 32;
          if (vec_ok && col0 + 32 <= cols_valid) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 q;
              q.x = pack_bf16x2(__uint_as_float(v[j + 0]), __uint_as_float(v[j + 1]));
              q.y = pack_bf16x2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
              q.z = pack_bf16x2(__uint_as_float(v[j + 4]), __uint_as_float(v[j + 5]));
              q.w = pack_bf16x2(__uint_as_float(v[j + 6]), __uint_as_float(v[j + 7]));
              *reinterpret_cast<uint4*>(orow + col0 + j) = q;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < cols_valid) orow[col0 + j] = __float2bfloat16_rn(__uint_as_float(v[j]));
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(smem_u32(&tail->tmem_empty[buf]), 0);
    }
  }

  // ---- teardown: neither CTA may exit while the other can still touch its memory ----
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after_sync();
  if (tail->abort_flag) {
    for (int i = 0; i < 200; ++i) __nanosleep(1000);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace b200
