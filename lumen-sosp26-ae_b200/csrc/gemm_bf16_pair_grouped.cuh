// Per-expert (grouped) BF16 GEMM on CTA pairs, weights on the accumulator rows.
//
// One unit of work = one expert x one weight tile x up to 320 of the expert's token rows,
// computed by a pair of SMs with tcgen05.mma.cta_group::2 (M = 256, K = 16).  The tokens are
// the MMA's N, which is set per unit at run time, so a ragged expert pays for its own rows
// (rounded up to 16) and not for whole row tiles:
//
//   A operand (M side)  weight rows, 128 per CTA.  Plain units: CTA r stages rows
//                        [w0 + 128 r, +128) and the pair produces 256 output columns.  Gated
//                        units: CTA r stages the 64 gate rows [w0 + 64 r, +64) and the 64 up
//                        rows that belong to them, so one accumulator holds gate values in
//                        lanes 0..63 and up values in lanes 64..127 of the same output
//                        columns; the pair produces 128 output columns of silu(gate) * up.
//   B operand (N side)  token rows.  The first 256 tokens of the unit are one MMA (each CTA
//                        stages half of them in a 128-row box); tokens 257..320, if any, are a
//                        second MMA on the same weight stage (32-row box per CTA), so that an
//                        expert a little over 256 rows does not stream its weights twice.
//   D                   TMEM columns = tokens.  TMEM is handled as two halves of 256 columns:
//                        a unit of at most 256 tokens takes one half (alternating, so its
//                        epilogue overlaps the next unit's main loop), a larger unit takes both.
//
// Per MMA each CTA stages half the bytes a single CTA would (the other half comes from its
// peer): 32 KB per 256 x 256 x 64 block, the ratio of the dense pair kernel.
//
// Epilogue: thread p of a CTA owns accumulator row p; TMEM column j is token t0 + j.  Plain
// units: thread p stores output column w0 + 128 r + p; a warp stores 32 consecutive columns
// (64 bytes) of one token per instruction.  Gated units: the gate lanes and the up lanes of a
// column sit in different warps, so for every group of 32 tokens one side hands its values to
// the other through shared memory (the sides alternate, which splits the SiLU work evenly).
// All loads are plain cp.async.bulk.tensor (no cluster multicast) from this GPU's memory.
#pragma once

#include "gemm_bf16_pair.cuh"

namespace b200 {

constexpr int kPgMainTokens = 256;  // tokens of the first MMA of a unit (the largest UMMA N)
constexpr int kPgTailTokens = 64;   // tokens of the second MMA
constexpr int kPgUnitTokens = kPgMainTokens + kPgTailTokens;
constexpr int kPgTailBox = kPgTailTokens / 2;  // token rows each CTA stages for the second MMA
constexpr int kPgBoxBytes = kBlockP * kBlockK * 2;          // 128 rows x 64 bf16
constexpr int kPgTailBytes = kPgTailBox * kBlockK * 2;      // 32 rows x 64 bf16
constexpr int kPgStageBytes = 2 * kPgBoxBytes + kPgTailBytes;  // weights + tokens + tail tokens

template <int STAGES, bool GATED>
struct PgSmemTail {
  uint64_t full[STAGES];   // leader's copy is the one in use (expects both CTAs' bytes)
  uint64_t empty[STAGES];  // each CTA waits on its own copy
  uint64_t tmem_full[2];   // per TMEM half; each CTA waits on its own copy
  uint64_t tmem_empty[2];  // per TMEM half; leader's copy: 8 arrivals = 4 epilogue warps x 2 CTAs
  uint32_t tmem_slot;
  int abort_flag;
  int total_units;
  int unit_start[kMaxExperts + 1];  // first unit of each expert
  // gated: values one side of the lanes hands to the other, [buffer][token of the group][column]
  float handoff[GATED ? 2 * 32 * 64 : 1];
};

template <int STAGES, bool GATED>
constexpr size_t gemm_pg_smem_bytes() {
  return 1024 + size_t(STAGES) * kPgStageBytes + sizeof(PgSmemTail<STAGES, GATED>);
}

struct PgUnit {
  int w_row;    // gated: first gate row of the pair's 128; plain: first weight row of the pair's 256
  int out_col;  // first output column of the pair
  int tok_row;  // first activation row
  int n_tok;    // token rows of this unit (1..320)
};

// Which TMEM half (or both) consecutive units use, and the barrier phases that go with them.
// The MMA issuer and the epilogue warps run the same sequence over the same units.
struct PgTmemSeq {
  int uses[2] = {0, 0};
  int next_small = 0;
  struct Slot {
    bool both;
    int half;          // the half of a small unit
    uint32_t phase[2]; // parity of this use of each half taken
    int col;           // first TMEM column of the unit
  };
  __device__ Slot take(int n_tok) {
    Slot s;
    s.both = n_tok > kPgMainTokens;
    if (s.both) {
      s.half = 0;
      s.phase[0] = uses[0]++ & 1;
      s.phase[1] = uses[1]++ & 1;
      s.col = 0;
    } else {
      s.half = next_small;
      next_small ^= 1;
      s.phase[s.half] = uses[s.half]++ & 1;
      s.phase[s.half ^ 1] = 0;
      s.col = s.half * kPgMainTokens;
    }
    return s;
  }
};

template <int STAGES, bool GATED>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_pair_grouped_kernel(const __grid_constant__ CUtensorMap map_w,
                                  const __grid_constant__ CUtensorMap map_x,
                                  const __grid_constant__ CUtensorMap map_x_tail, const GemmArgs args) {
  using Tail = PgSmemTail<STAGES, GATED>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_aligned = smem_raw + (smem_base - smem_u32(smem_raw));
  constexpr int kOutCols = GATED ? kBlockP : 2 * kBlockP;  // output columns per unit
  Tail* tail = reinterpret_cast<Tail*>(smem_aligned + size_t(STAGES) * kPgStageBytes);

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
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_x_tail);
  }
  if (warp == 1) tmem_alloc(smem_u32(&tail->tmem_slot), 512);
  // nothing above reads or writes global memory: it may overlap the previous kernel's tail
  griddep_wait();
  griddep_launch_dependents();
  // units of expert e: (weight tiles) x (token tiles of at most 320 rows); warp 0 scans
  const int w_tiles = ceil_div(args.N, kOutCols);
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < args.num_experts; base += 32) {
      const int e = base + lane;
      const int v = (e < args.num_experts) ? ceil_div(args.expert_counts[e], args.unit_tokens) * w_tiles : 0;
      int incl = v;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += o;
      }
      if (e < args.num_experts) tail->unit_start[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      tail->unit_start[args.num_experts] = carry;
      tail->total_units = carry;
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // barriers of both CTAs are initialised before any remote arrival
  tc_fence_after_sync();

  const uint32_t tmem_base = tail->tmem_slot;
  // The leader's MMA addresses the accumulator of both CTAs by the leader's TMEM base: each CTA
  // allocated all 512 columns, so both bases are column 0; verify instead of assuming.
  if (threadIdx.x == 0 && rank == 1) {
    const uint32_t leader_base = ld_shared_cluster_u32(map_to_cta(smem_u32(&tail->tmem_slot), 0));
    if (leader_base != tmem_base) {
      tail->abort_flag = 1;
      atomicCAS(args.status, 0, (kPairTmemMismatch << 16) | static_cast<int>(blockIdx.x & 0xffffu));
    }
  }
  const int total_units = tail->total_units;
  const int k_blocks = ceil_div(args.K, kBlockK);
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  int cursor = 0;  // expert of the previous unit (units come in increasing order)
  auto decode = [&](int u) {
    int e = cursor;
    while (u >= tail->unit_start[e + 1]) ++e;
    cursor = e;
    const int local = u - tail->unit_start[e];
    const int cnt = args.expert_counts[e];
    const int tok_tiles = ceil_div(cnt, args.unit_tokens);
    // token tile fastest: units that run together share a weight tile in L2
    const int wt = local / tok_tiles;
    const int tt = local - wt * tok_tiles;
    // the expert's rows are dealt out evenly over its token tiles
    const int base = cnt / tok_tiles, extra = cnt - base * tok_tiles;
    PgUnit t;
    t.out_col = wt * kOutCols;
    t.w_row = e * args.w_rows_per_expert + t.out_col;
    t.tok_row = args.expert_offsets[e] + tt * base + min(tt, extra);
    t.n_tok = base + (tt < extra ? 1 : 0);
    return t;
  };

  if (warp == 0) {
    // ======================= TMA producer (both CTAs) ======================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair_id; u < total_units && ok; u += num_pairs) {
        const PgUnit t = decode(u);
        const int n1 = min(t.n_tok, kPgMainTokens);
        const int n1_mma = (n1 + 15) & ~15;
        const int n2 = t.n_tok - n1;
        const int n2_mma = (n2 + 15) & ~15;
        const int x_row = t.tok_row + int(rank) * (n1_mma / 2);
        const int x_row2 = t.tok_row + kPgMainTokens + int(rank) * (n2_mma / 2);
        const uint32_t bytes = 2 * kPgBoxBytes + (n2 > 0 ? kPgTailBytes : 0);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, ctx, kWaitEmptyStage)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = map_to_cta(smem_u32(&tail->full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(smem_u32(&tail->full[stage]), 2 * bytes);
          const uint32_t sw = smem_base + stage * kPgStageBytes;
          const uint32_t sx = sw + kPgBoxBytes;
          const int kx = kb * kBlockK;
          if constexpr (GATED) {
            // 64 gate rows, then the 64 up rows of the same output columns (64-row boxes)
            const int g_row = t.w_row + int(rank) * (kBlockP / 2);
            tma_load_2d_pair(sw, &map_w, leader_full, kx, g_row);
            tma_load_2d_pair(sw + kPgBoxBytes / 2, &map_w, leader_full, kx, g_row + args.up_row_offset);
          } else {
            tma_load_2d_pair(sw, &map_w, leader_full, kx, t.w_row + int(rank) * kBlockP);
          }
          tma_load_2d_pair(sx, &map_x, leader_full, kx, x_row);
          if (n2 > 0) tma_load_2d_pair(sx + kPgBoxBytes, &map_x_tail, leader_full, kx, x_row2);
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
      int stage = 0;
      uint32_t phase = 0;
      PgTmemSeq seq;
      bool ok = true;
      for (int u = pair_id; u < total_units && ok; u += num_pairs) {
        const PgUnit t = decode(u);
        const int n1 = min(t.n_tok, kPgMainTokens);
        const int n2 = t.n_tok - n1;
        const uint32_t idesc1 = make_idesc_bf16(2 * kBlockP, (n1 + 15) & ~15, 0, 0);
        const uint32_t idesc2 = make_idesc_bf16(2 * kBlockP, n2 > 0 ? (n2 + 15) & ~15 : 16, 0, 0);
        const PgTmemSeq::Slot slot = seq.take(t.n_tok);
        for (int h = 0; h < 2 && ok; ++h) {
          if (!slot.both && h != slot.half) continue;
          if (!mbar_wait(smem_u32(&tail->tmem_empty[h]), slot.phase[h] ^ 1u, ctx, kWaitTmemEmpty)) ok = false;
        }
        if (!ok) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + slot.col;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&tail->full[stage]), phase, ctx, kWaitFullStage)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sw = smem_base + stage * kPgStageBytes;
          const uint32_t sx = sw + kPgBoxBytes;
#pragma unroll
          for (int k = 0; k < kBlockK / kUmmaK; ++k) {
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            const uint64_t dw = make_smem_desc_sw128(sw + k * kUmmaK * 2, 0, 1024);
            umma_bf16_ss_pair(d_tmem, dw, make_smem_desc_sw128(sx + k * kUmmaK * 2, 0, 1024), idesc1, acc);
            if (n2 > 0)
              umma_bf16_ss_pair(d_tmem + kPgMainTokens, dw,
                                make_smem_desc_sw128(sx + kPgBoxBytes + k * kUmmaK * 2, 0, 1024), idesc2, acc);
          }
          umma_commit_pair(smem_u32(&tail->empty[stage]), 3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          if (slot.both || slot.half == 0) umma_commit_pair(smem_u32(&tail->tmem_full[0]), 3);
          if (slot.both || slot.half == 1) umma_commit_pair(smem_u32(&tail->tmem_full[1]), 3);
        }
      }
    }
  } else {
    // ======================= epilogue (both CTAs) ==========================
    const int quad = warp & 3;
    const int p = quad * 32 + lane;  // accumulator row
    PgTmemSeq seq;
    bool ok = true;
    for (int u = pair_id; u < total_units; u += num_pairs) {
      const PgUnit t = decode(u);
      const PgTmemSeq::Slot slot = seq.take(t.n_tok);
      for (int h = 0; h < 2 && ok; ++h) {
        if (!slot.both && h != slot.half) continue;
        if (!mbar_wait(smem_u32(&tail->tmem_full[h]), slot.phase[h], ctx, kWaitTmemFull)) ok = false;
      }
      // the four epilogue warps go on together or stop together (they meet at barriers below)
      {
        int all_ok;
        asm volatile(
            "{\n"
            ".reg .pred pi, po;\n"
            "setp.ne.b32 pi, %1, 0;\n"
            "bar.red.and.pred po, 1, 128, pi;\n"
            "selp.b32 %0, 1, 0, po;\n"
            "}\n"
            : "=r"(all_ok)
            : "r"(ok ? 1 : 0)
            : "memory");
        ok = all_ok != 0;
      }
      if (!ok) break;
      tc_fence_after_sync();
      const uint32_t t_acc = tmem_base + (uint32_t(quad * 32) << 16) + slot.col;
      const int chunks = (t.n_tok + 31) / 32;  // 32-token groups the MMAs wrote

      if constexpr (!GATED) {
        const int col = t.out_col + int(rank) * kBlockP + p;
        const bool col_ok = col < args.N;
#pragma unroll 1
        for (int c = 0; c < chunks; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_acc + c * 32, v);
          tmem_ld_wait();
          if (col_ok) {
            const int rows_here = min(32, t.n_tok - c * 32);
            if (args.out_row_ptrs) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (j < rows_here) {
                  __nv_bfloat16* base = args.out_row_ptrs[t.tok_row + c * 32 + j];
                  if (base) base[col] = __float2bfloat16_rn(__uint_as_float(v[j]));
                }
              }
            } else {
              __nv_bfloat16* o = args.out + size_t(t.tok_row + c * 32) * args.ldo + col;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < rows_here) o[size_t(j) * args.ldo] = __float2bfloat16_rn(__uint_as_float(v[j]));
            }
          }
        }
      } else {
        // lanes 0..63 hold gate values, lanes 64..127 the up values of the same 64 columns
        const bool gate_side = p < kBlockP / 2;
        const int pc = p & (kBlockP / 2 - 1);  // column of this CTA's 64
        const int col = t.out_col + int(rank) * (kBlockP / 2) + pc;
        const bool col_ok = col < args.N;
#pragma unroll 1
        for (int c = 0; c < chunks; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_acc + c * 32, v);
          tmem_ld_wait();
          // even groups: the up side hands over, the gate side finishes; odd groups: the reverse
          const bool finisher = gate_side == ((c & 1) == 0);
          float* hand = tail->handoff + (c & 1) * (32 * 64);
          if (!finisher) {
#pragma unroll
            for (int j = 0; j < 32; ++j) hand[j * 64 + pc] = __uint_as_float(v[j]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (finisher) {
            float f[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float other = hand[j * 64 + pc];
              const float g = gate_side ? __uint_as_float(v[j]) : other;
              const float up = gate_side ? other : __uint_as_float(v[j]);
              f[j] = silu_mul(g, up);
            }
            if (col_ok) {
              const int rows_here = min(32, t.n_tok - c * 32);
              if (args.out_row_ptrs) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  if (j < rows_here) {
                    __nv_bfloat16* base = args.out_row_ptrs[t.tok_row + c * 32 + j];
                    if (base) base[col] = __float2bfloat16_rn(f[j]);
                  }
                }
              } else {
                __nv_bfloat16* o = args.out + size_t(t.tok_row + c * 32) * args.ldo + col;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < rows_here) o[size_t(j) * args.ldo] = __float2bfloat16_rn(f[j]);
              }
            }
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (slot.both || slot.half == 0) mbar_arrive_cluster(smem_u32(&tail->tmem_empty[0]), 0);
        if (slot.both || slot.half == 1) mbar_arrive_cluster(smem_u32(&tail->tmem_empty[1]), 0);
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
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace b200
