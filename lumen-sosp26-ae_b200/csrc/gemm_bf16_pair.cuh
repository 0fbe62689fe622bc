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
// Tail of the last wave.  A launch runs its tiles round-robin over the CTA pairs, so the last
// round keeps only (tiles mod pairs) of them busy.  When that remainder R is at most half
// of the pairs, each of the last R tiles is cut into s = pairs / R slices along K (at least
// 8 K blocks each; s = 2, 4 or 8), one slice per pair: the last round then takes 1 / s of a full
// one.  The slices of a tile exchange fp32 partial sums through the workspace like a
// reduce-scatter (each finishes 1 / s of the columns, adding in slice order, so the result is the
// same from run to run).  Without a workspace the launcher does not split.
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

template <int STAGES, bool GROUPED = false>
struct PairSmemTail {
  uint64_t full[STAGES];      // leader's copy is the one in use (expects both CTAs' bytes)
  uint64_t empty[STAGES];     // each CTA waits on its own copy
  uint64_t tmem_full[2];      // each CTA waits on its own copy
  uint64_t tmem_empty[2];     // leader's copy: 8 arrivals = 4 epilogue warps x 2 CTAs
  uint32_t tmem_slot;
  int abort_flag;
  int unit_start[GROUPED ? kMaxExperts + 1 : 1];  // grouped: first unit of each expert
};

template <int STAGES, int BN, bool GROUPED = false>
constexpr size_t gemm_pair_smem_bytes() {
  return 1024 + size_t(STAGES) * pair_stage_bytes<BN>() + sizeof(PairSmemTail<STAGES, GROUPED>);
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

// One piece of work of a pair: an output tile over K blocks [kb0, kb1).
struct PairWork {
  int m0, n0;         // first A row of the tile; first output column
  int b_row;          // first B (weight) row of the tile (grouped: inside the expert's block)
  int rows_valid;     // output rows of the tile that exist, counted from m0
  int kb0, kb1;
  int slice, slices;  // slices == 1: the whole K range, stored directly
  int tail_idx;       // index of the tile among the split ones
};

// Grouped (expert by expert) work of the pair kernel, tokens on the 256 accumulator rows: the
// units of expert e are [unit_start[e], unit_start[e + 1]), 256-row token tile fastest so that
// pairs running together share a weight tile in L2.  A gated tile holds 64 gate + 64 up weight
// rows per CTA and produces BN / 2 output columns.
template <int BN, bool GATED>
struct PairGroupedDecoder {
  static constexpr int kOutCols = GATED ? BN / 2 : BN;
  const GemmArgs& a;
  const int* unit_start;
  int cursor = 0;
  __device__ PairGroupedDecoder(const GemmArgs& args, const int* us) : a(args), unit_start(us) {}
  __device__ PairWork decode(int u, int k_blocks) {
    int e = cursor;
    while (u >= unit_start[e + 1]) ++e;
    cursor = e;
    const int local = u - unit_start[e];
    const int cnt = a.expert_counts[e];
    const int act_tiles = ceil_div(cnt, kPairTileM);
    const int w_tile = local / act_tiles;
    const int at = local - w_tile * act_tiles;
    PairWork r;
    r.m0 = a.expert_offsets[e] + at * kPairTileM;
    r.rows_valid = cnt - at * kPairTileM;
    r.n0 = w_tile * kOutCols;
    r.b_row = e * a.w_rows_per_expert + r.n0;
    r.kb0 = 0;
    r.kb1 = k_blocks;
    r.slice = 0;
    r.slices = 1;
    r.tail_idx = 0;
    return r;
  }
};

template <int BN>
__device__ __forceinline__ PairWork pair_work(int w, int tiles_m, int tiles_n, int k_blocks, int tail_first,
                                              int slices) {
  PairWork r;
  int u = w;
  r.kb0 = 0;
  r.kb1 = k_blocks;
  r.slice = 0;
  r.slices = 1;
  r.tail_idx = 0;
  if (w >= tail_first) {
    const int x = w - tail_first;
    r.tail_idx = x / slices;
    r.slice = x - r.tail_idx * slices;
    r.slices = slices;
    u = tail_first + r.tail_idx;
    r.kb0 = (k_blocks * r.slice) / slices;
    r.kb1 = (k_blocks * (r.slice + 1)) / slices;
  }
  const PairUnit t = pair_decode<BN>(u, tiles_m, tiles_n);
  r.m0 = t.m0;
  r.n0 = t.n0;
  r.b_row = t.n0;
  r.rows_valid = 1 << 30;  // dense: rows are bounded by args.M
  return r;
}

// BN = 256 or 128 output columns per tile (the narrower tile halves the unit of work, which
// matters when the tile count is a small non-multiple of the 74 CTA pairs).
// GROUPED: A = the routed rows of all experts, B = the stacked expert weights, units from the
// expert counts on the device (GATED: SiLU(gate) * up in the epilogue); the map of B then has
// boxes of BN / 4 rows.
template <int STAGES, int BN, bool GROUPED = false, bool GATED = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                          const __grid_constant__ CUtensorMap map_b, const GemmArgs args) {
  static_assert(!GATED || GROUPED, "the gated epilogue belongs to the expert GEMM");
  using Tail = PairSmemTail<STAGES, GROUPED>;
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
  if constexpr (GROUPED) {
    // unit_start[e] = units of the experts before e; warp 0 scans the counts
    if (warp == 0) {
      const int w_tiles = ceil_div(args.N, PairGroupedDecoder<BN, GATED>::kOutCols);
      int carry = 0;
      for (int base = 0; base < args.num_experts; base += 32) {
        const int e = base + lane;
        const int v = (e < args.num_experts) ? ceil_div(args.expert_counts[e], kPairTileM) * w_tiles : 0;
        int incl = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int o = __shfl_up_sync(0xffffffffu, incl, d);
          if (lane >= d) incl += o;
        }
        if (e < args.num_experts) tail->unit_start[e] = carry + incl - v;
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) tail->unit_start[args.num_experts] = carry;
    }
  }
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
  const int tiles_m = GROUPED ? 0 : ceil_div(args.M, kPairTileM);
  const int tiles_n = GROUPED ? 0 : ceil_div(args.N, BN);
  const int total_units = GROUPED ? tail->unit_start[args.num_experts] : tiles_m * tiles_n;
  const int k_blocks = ceil_div(args.K, kBlockK);
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  // pieces of work: whole tiles [0, tail_first), then `slices` K slices of each later tile
  const int slices = (!GROUPED && args.splits > 1) ? args.splits : 1;
  const int tail_first = slices > 1 ? args.tail_first : total_units;
  const int total_work = tail_first + (total_units - tail_first) * slices;
  // each role walks the work list with its own decoder (the grouped one keeps a cursor)
  auto make_decoder = [&]() { return PairGroupedDecoder<BN, GATED>(args, tail->unit_start); };
  auto decode = [&](PairGroupedDecoder<BN, GATED>& dec, int w) {
    if constexpr (GROUPED) {
      return dec.decode(w, k_blocks);
    } else {
      return pair_work<BN>(w, tiles_m, tiles_n, k_blocks, tail_first, slices);
    }
  };

  if (warp == 0) {
    // ======================= TMA producer (both CTAs) ======================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      auto dec = make_decoder();
      for (int w = pair_id; w < total_work && ok; w += num_pairs) {
        const PairWork t = decode(dec, w);
        const int a_row = t.m0 + int(rank) * kBlockP;
        // B rows of this CTA: BN / 2 consecutive ones, or for a gated tile BN / 4 gate rows and the
        // BN / 4 up rows that belong to them
        const int b_row = t.b_row + int(rank) * (GATED ? BN / 4 : BN / 2);
        for (int kb = t.kb0; kb < t.kb1; ++kb) {
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
          if constexpr (GATED)
            tma_load_2d_pair(sb + (BN / 4) * kBlockK * 2, &map_b, leader_full, kb * kBlockK,
                             b_row + args.up_row_offset);
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
      auto dec = make_decoder();
      for (int w = pair_id; w < total_work && ok; w += num_pairs, ++it) {
        const PairWork t = decode(dec, w);
        const int buf = it & 1;
        const uint32_t buf_phase = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&tail->tmem_empty[buf]), buf_phase ^ 1u, ctx, kWaitTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = t.kb0; kb < t.kb1; ++kb) {
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
                              (kb > t.kb0 || k > 0) ? 1u : 0u);
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
    auto dec = make_decoder();
    for (int w = pair_id; w < total_work && ok; w += num_pairs, ++it) {
      const PairWork t = decode(dec, w);
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
      const bool row_ok = GROUPED ? (int(rank) * kBlockP + p < t.rows_valid) : (row < args.M);
      const int cols_valid = min(GATED ? BN / 2 : BN, args.N - t.n0);
      __nv_bfloat16* orow = args.out + size_t(row) * args.ldo + t.n0;
      // 32 fp32 values of this thread's row, columns [c * 32, c * 32 + 32) of the tile -> bf16 -> C
      auto store_chunk = [&](const uint32_t (&v)[32], int c) {
        if (!row_ok) return;
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
      };
      if (t.slices == 1) {
        if constexpr (GATED) {
          // accumulator columns of this CTA's rows: [gate of CTA 0 | up of CTA 0 | gate of CTA 1 |
          // up of CTA 1], BN / 4 each; output chunk c = columns [c * 32, c * 32 + 32) of the tile
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            const int half = (c * 32) / (BN / 4);
            const int within = c * 32 - half * (BN / 4);
            uint32_t g[32], u[32];
            tmem_ld_32x32b_x32(t_acc + half * (BN / 2) + within, g);
            tmem_ld_32x32b_x32(t_acc + half * (BN / 2) + BN / 4 + within, u);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              g[j] = __float_as_uint(silu_mul(__uint_as_float(g[j]), __uint_as_float(u[j])));
            store_chunk(g, c);
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_acc + c * 32, v);
            tmem_ld_wait();
            store_chunk(v, c);
          }
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(smem_u32(&tail->tmem_empty[buf]), 0);
        continue;
      }
      // ---- one K slice of a split tile ----
      // The `slices` pairs that share the tile exchange partial sums through the workspace like
      // a reduce-scatter: slice i finishes the 32-column chunks [i * own, (i + 1) * own) of every
      // row, so it stores its other chunks, waits until the warps of the other slices that hold
      // the same 32 rows have stored theirs, and adds what they left for its chunks, in slice
      // order.  All pairs of a launch are resident together, so the wait is on running CTAs; it
      // is bounded like every other wait.
      // workspace: [tile][writing slice][CTA of the pair][128 rows][BN] fp32
      constexpr int kChunks = BN / 32;
      constexpr size_t kHalfTile = size_t(kBlockP) * BN;
      const int own = kChunks / t.slices;
      const int own_first = t.slice * own;
      float* tile_ws = args.ws + size_t(t.tail_idx) * t.slices * 2 * kHalfTile;
      float* mine = tile_ws + (size_t(t.slice) * 2 + rank) * kHalfTile + size_t(p) * BN;
#pragma unroll 1
      for (int c = 0; c < kChunks; ++c) {
        if (c >= own_first && c < own_first + own) continue;
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_acc + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          __stcg(reinterpret_cast<uint4*>(mine + c * 32 + j), make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]));
      }
      __threadfence();
      __syncwarp();
      int* arrivals = args.counters + ((t.tail_idx * 2 + int(rank)) * 4 + quad) * 2;
      int* departures = arrivals + 1;
      int seen = 1;
      if (lane == 0) {
        atomicAdd(arrivals, 1);
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (ld_acquire_gpu(arrivals) < t.slices) {
          if ((++spins & 0xffu) == 0u) {
            if (*ctx.cta_abort) {
              seen = 0;
              break;
            }
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              *ctx.cta_abort = 1;
              atomicCAS(ctx.status, 0, (kWaitSlices << 16) | static_cast<int>(blockIdx.x & 0xffffu));
              seen = 0;
              break;
            }
          }
        }
      }
      seen = __shfl_sync(0xffffffffu, seen, 0);
      if (!seen) {
        ok = false;
        break;
      }
      __threadfence();
      const float* rows = tile_ws + size_t(rank) * kHalfTile + size_t(p) * BN;
#pragma unroll 1
      for (int c = own_first; c < own_first + own; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_acc + c * 32, v);
        tmem_ld_wait();
        for (int sl = 0; sl < t.slices; ++sl) {
          if (sl == t.slice) continue;
          const float* src = rows + size_t(sl) * 2 * kHalfTile + c * 32;
          uint4 x[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) x[j] = __ldcg(reinterpret_cast<const uint4*>(src) + j);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[4 * j + 0] = __float_as_uint(__uint_as_float(v[4 * j + 0]) + __uint_as_float(x[j].x));
            v[4 * j + 1] = __float_as_uint(__uint_as_float(v[4 * j + 1]) + __uint_as_float(x[j].y));
            v[4 * j + 2] = __float_as_uint(__uint_as_float(v[4 * j + 2]) + __uint_as_float(x[j].z));
            v[4 * j + 3] = __float_as_uint(__uint_as_float(v[4 * j + 3]) + __uint_as_float(x[j].w));
          }
        }
        store_chunk(v, c);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_cluster(smem_u32(&tail->tmem_empty[buf]), 0);
        // the last of the slices to have read resets both counters for the next launch
        if (atomicAdd(departures, 1) == t.slices - 1) {
          *departures = 0;
          *arrivals = 0;
        }
      }
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
