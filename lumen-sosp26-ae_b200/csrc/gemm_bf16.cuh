// BF16 contraction core for sm_100a:  D = P * Q^T with fp32 accumulation in TMEM.
//
// One persistent, warp-specialised kernel template, one CTA per tile.  It serves the
// weight-streaming form of the dense GEMM C = A * B^T (few activation rows, split-K), the
// grouped (per-expert) GEMMs of the MoE, and a 128 x 256 dense tiling; large dense
// problems use the CTA-pair kernel of gemm_bf16_pair.cuh instead.
//
//   warp 0      TMA producer: global -> 128B-swizzled shared-memory ring (plain
//               cp.async.bulk.tensor loads, one mbarrier per stage)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: tcgen05.ld -> fp32 registers -> bf16 -> global
//
// "P" is the operand that feeds the 128 TMEM lanes (UMMA M = 128), "Q" the operand
// that feeds the TMEM columns (UMMA N = BN).  In the normal orientation P is the
// activation matrix and Q the weight matrix; in the swapped orientation (few
// activation rows, HBM-bound weight streaming) P is the weight matrix so that a
// 16 KB stage buffer holds nothing but weights, and the epilogue stores D^T.
//
// The accumulator is double-buffered in TMEM so that the epilogue of unit i
// overlaps the main loop of unit i+1.
#pragma once

#include "lumen_b200_internal.h"

namespace b200 {

constexpr int kBlockP = 128;       // rows of P per unit = TMEM lanes
constexpr int kBlockK = 64;        // K elements per stage = one 128-byte swizzle row
constexpr int kUmmaK = 16;         // K per tcgen05.mma for 16-bit inputs
constexpr int kGemmThreads = 192;  // 6 warps

// wait-site codes reported in the status word
enum GemmWaitCode {
  kWaitEmptyStage = 1,
  kWaitFullStage = 2,
  kWaitTmemEmpty = 3,
  kWaitTmemFull = 4,
  kWaitSlices = 5,  // the other K slices of a split tile did not arrive
};

// split-K counters: arrivals of tile i at counters[i], departures at counters[kSplitTileSlots + i]
constexpr int kSplitTileSlots = 2048;

struct GemmArgs {
  __nv_bfloat16* out;  // [rows_out, N] row-major, leading dimension ldo
  int ldo;
  int M;  // activation rows (dense) / unused (grouped)
  int N;  // output columns = weight rows per expert that produce outputs
  int K;
  int splits;     // split-K factor: K slices per tile (swapped dense) or per tile of the last, partial wave (CTA pairs); 1 = none
  int tail_first; // CTA pairs: first output tile that is split over K (tiles before it run whole)
  float* ws;      // split-K partial tiles
  int* counters;  // split-K arrival counters, zero between launches
  // grouped
  const int* expert_offsets;  // [E+1] first activation row of each expert
  const int* expert_counts;   // [E] valid rows of each expert
  int num_experts;
  int w_rows_per_expert;  // rows of the stacked weight tensor per expert
  int up_row_offset;      // gated: distance from a gate row to its up row
  // grouped, optional: where each output row lives.  out_row_ptrs[r] is the address of the
  // first element of output row r (possibly in a peer GPU's memory: the epilogue then is the
  // send of the expert-parallel return trip) or nullptr for a row that must not be stored.
  __nv_bfloat16* const* out_row_ptrs;
  int unit_tokens;  // pair kernel: most token rows one unit takes (256: one MMA; up to 320: two)
  int* status;
};

// One unit of work: a [128 x BN] accumulator tile over a K range.
struct Unit {
  int p_row;       // row coordinate of the P box
  int q_row;       // row coordinate of the Q box
  int p_row2;      // second P box (swapped gated)
  int q_row2;      // second Q box (normal gated)
  int out_row;     // first output row
  int out_col;     // first output column
  int rows_valid;  // output rows to store
  int cols_valid;  // output columns to store
  int kb_begin;    // K range in units of kBlockK
  int kb_end;
  int tile_id;  // split-K: output tile index
  int split;    // split-K: which slice
};

template <int BN, bool SWAP, bool GATED, bool GROUPED>
struct GemmCfg {
  // rows of Q (normal) covered by one box; a gated normal tile loads two boxes
  // (gate rows, up rows) of BN/2 rows each into one BN-row operand.
  static constexpr int kQBoxRows = (!SWAP && GATED) ? BN / 2 : BN;
  static constexpr int kQBoxes = (!SWAP && GATED) ? 2 : 1;
  static constexpr int kPBoxes = (SWAP && GATED) ? 2 : 1;
  static constexpr int kPBytes = kPBoxes * kBlockP * kBlockK * 2;
  static constexpr int kQBytes = BN * kBlockK * 2;
  // keep every operand buffer 1024-byte aligned (swizzle atom = 8 rows x 128 B)
  static constexpr int kQBytesPadded = (kQBytes + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kPBytes + kQBytesPadded;
  // accumulator columns per buffer
  static constexpr int kAccCols = (SWAP && GATED) ? 2 * BN : BN;
  static constexpr int kTmemColsRaw = 2 * kAccCols;
  static constexpr int kTmemCols = kTmemColsRaw <= 32    ? 32
                                   : kTmemColsRaw <= 64  ? 64
                                   : kTmemColsRaw <= 128 ? 128
                                   : kTmemColsRaw <= 256 ? 256
                                                         : 512;
  // output columns (normal) produced per unit
  static constexpr int kOutCols = SWAP ? kBlockP : (GATED ? BN / 2 : BN);
  // activation rows per unit
  static constexpr int kActRows = SWAP ? BN : kBlockP;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M = 128");
  static_assert(kTmemColsRaw <= 512, "TMEM has 512 columns");
};

// Shared-memory bookkeeping placed after the stage ring.
template <int STAGES, bool GROUPED>
struct GemmSmemTail {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_slot;
  int abort_flag;
  int total_units;
  int last_flag;
  int unit_start[GROUPED ? kMaxExperts + 1 : 1];  // grouped: first unit of each expert
};

template <int BN, int STAGES, bool SWAP, bool GATED, bool GROUPED>
constexpr size_t gemm_smem_bytes() {
  return 1024 /*alignment slack*/ + size_t(STAGES) * GemmCfg<BN, SWAP, GATED, GROUPED>::kStageBytes +
         sizeof(GemmSmemTail<STAGES, GROUPED>);
}

__device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// unit decode
// ---------------------------------------------------------------------------
template <int BN, bool SWAP, bool GATED, bool GROUPED>
struct UnitDecoder {
  using Cfg = GemmCfg<BN, SWAP, GATED, GROUPED>;
  const GemmArgs& a;
  const int* unit_start;  // shared memory (grouped)
  int cursor = 0;         // grouped: expert of the previous unit (units come in increasing order)
  int k_blocks;
  int w_tiles;  // tiles along the weight-row dimension

  __device__ UnitDecoder(const GemmArgs& args, const int* us) : a(args), unit_start(us) {
    k_blocks = ceil_div(a.K, kBlockK);
    w_tiles = ceil_div(a.N, Cfg::kOutCols);
  }

  __device__ int dense_total() const {
    const int act_tiles = ceil_div(a.M, Cfg::kActRows);
    return act_tiles * w_tiles * a.splits;
  }

  __device__ Unit decode(int u) {
    Unit t;
    t.kb_begin = 0;
    t.kb_end = k_blocks;
    t.tile_id = 0;
    t.split = 0;
    int act_row, act_valid, w_tile, w_base;
    if constexpr (GROUPED) {
      int e = cursor;
      while (u >= unit_start[e + 1]) ++e;
      cursor = e;
      const int local = u - unit_start[e];
      const int cnt = a.expert_counts[e];
      const int act_tiles = ceil_div(cnt, Cfg::kActRows);
      // activation tile fastest: neighbouring units share one weight tile in L2
      w_tile = local / act_tiles;
      const int at = local - w_tile * act_tiles;
      act_row = a.expert_offsets[e] + at * Cfg::kActRows;
      act_valid = min(Cfg::kActRows, cnt - at * Cfg::kActRows);
      w_base = e * a.w_rows_per_expert;
    } else {
      const int act_tiles = ceil_div(a.M, Cfg::kActRows);
      int at;
      if constexpr (SWAP) {
        const int tile = u / a.splits;
        t.split = u - tile * a.splits;
        t.tile_id = tile;
        w_tile = tile / act_tiles;
        at = tile - w_tile * act_tiles;
        // even partition of the K blocks over the splits
        t.kb_begin = static_cast<int>((static_cast<long long>(k_blocks) * t.split) / a.splits);
        t.kb_end = static_cast<int>((static_cast<long long>(k_blocks) * (t.split + 1)) / a.splits);
      } else {
        // groups of 16 activation tiles sweep the weight tiles together so that
        // the CTAs running at one time share few distinct operand panels
        constexpr int kGroup = 16;
        const int per_group = kGroup * w_tiles;
        const int g = u / per_group;
        const int r = u - g * per_group;
        const int gsz = min(kGroup, act_tiles - g * kGroup);
        w_tile = r / gsz;
        at = g * kGroup + (r - w_tile * gsz);
      }
      act_row = at * Cfg::kActRows;
      act_valid = min(Cfg::kActRows, a.M - act_row);
      w_base = 0;
    }
    const int w_row = w_base + w_tile * Cfg::kOutCols;
    t.out_row = act_row;
    t.rows_valid = act_valid;
    t.out_col = w_tile * Cfg::kOutCols;
    t.cols_valid = min(Cfg::kOutCols, a.N - t.out_col);
    if constexpr (SWAP) {
      t.p_row = w_row;
      t.p_row2 = w_row + a.up_row_offset;
      t.q_row = act_row;
      t.q_row2 = 0;
    } else {
      t.p_row = act_row;
      t.p_row2 = 0;
      t.q_row = w_row;
      t.q_row2 = w_row + a.up_row_offset;
    }
    return t;
  }
};

__device__ __forceinline__ float silu_mul(float g, float u) {
  // silu(g) * u with g / (1 + 2^(-g*log2e))
  const float e = fast_exp2(-g * 1.4426950408889634f);
  return __fdividef(g, 1.0f + e) * u;
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
template <int BN, int STAGES, bool SWAP, bool GATED, bool GROUPED>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_p,
                     const __grid_constant__ CUtensorMap map_q, const GemmArgs args) {
  using Cfg = GemmCfg<BN, SWAP, GATED, GROUPED>;
  using Tail = GemmSmemTail<STAGES, GROUPED>;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_aligned = smem_raw + (smem_base - smem_u32(smem_raw));
  Tail* tail = reinterpret_cast<Tail*>(smem_aligned + size_t(STAGES) * Cfg::kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const AbortCtx ctx{&tail->abort_flag, args.status};

  // ---- one-time setup ------------------------------------------------------
  if (threadIdx.x == 0) {
    tail->abort_flag = 0;
    tail->last_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&tail->full[s]), 1);
      mbar_init(smem_u32(&tail->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tail->tmem_full[b]), 1);
      mbar_init(smem_u32(&tail->tmem_empty[b]), 4);  // one arrival per epilogue warp
    }
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&map_p);
    tma_prefetch_desc(&map_q);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tail->tmem_slot), Cfg::kTmemCols);
  }
  // nothing above reads or writes global memory: it may overlap the previous kernel's tail
  griddep_wait();
  griddep_launch_dependents();
  if constexpr (GROUPED) {
    // unit_start[e] = (weight tiles) * (activation tiles of experts before e); warp 0 scans
    if (warp == 0) {
      const int w_tiles = ceil_div(args.N, Cfg::kOutCols);
      int carry = 0;
      for (int base = 0; base < args.num_experts; base += 32) {
        const int e = base + lane;
        const int v =
            (e < args.num_experts) ? ceil_div(args.expert_counts[e], Cfg::kActRows) * w_tiles : 0;
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
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();

  const uint32_t tmem_base = tail->tmem_slot;
  UnitDecoder<BN, SWAP, GATED, GROUPED> dec(args, tail->unit_start);
  const int total_units = GROUPED ? tail->total_units : dec.dense_total();

  if (warp == 0) {
    // ======================= TMA producer =================================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const Unit t = dec.decode(u);
        for (int kb = t.kb_begin; kb < t.kb_end; ++kb) {
          if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, ctx, kWaitEmptyStage)) {
            ok = false;
            break;
          }
          const uint32_t bar = smem_u32(&tail->full[stage]);
          const uint32_t sp = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sq = sp + Cfg::kPBytes;
          mbar_arrive_expect_tx(bar, Cfg::kPBytes + Cfg::kQBytes);
          const int kx = kb * kBlockK;
          tma_load_2d(sp, &map_p, bar, kx, t.p_row);
          if constexpr (Cfg::kPBoxes == 2)
            tma_load_2d(sp + kBlockP * kBlockK * 2, &map_p, bar, kx, t.p_row2);
          tma_load_2d(sq, &map_q, bar, kx, t.q_row);
          if constexpr (Cfg::kQBoxes == 2)
            tma_load_2d(sq + Cfg::kQBoxRows * kBlockK * 2, &map_q, bar, kx, t.q_row2);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer ===================================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++it) {
        const Unit t = dec.decode(u);
        // swapped orientation: the activation rows are the MMA's N, so a ragged unit
        // only pays for its own rows (rounded up to the instruction granularity of 16)
        const uint32_t idesc =
            make_idesc_bf16(kBlockP, SWAP ? min(BN, (t.rows_valid + 15) & ~15) : BN, 0, 0);
        const int buf = it & 1;
        const uint32_t buf_phase = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&tail->tmem_empty[buf]), buf_phase ^ 1u, ctx, kWaitTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * Cfg::kAccCols;
        for (int kb = t.kb_begin; kb < t.kb_end; ++kb) {
          if (!mbar_wait(smem_u32(&tail->full[stage]), phase, ctx, kWaitFullStage)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sp = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sq = sp + Cfg::kPBytes;
#pragma unroll
          for (int k = 0; k < kBlockK / kUmmaK; ++k) {
            const uint32_t acc = (kb > t.kb_begin || k > 0) ? 1u : 0u;
            const uint64_t dq = make_smem_desc_sw128(sq + k * kUmmaK * 2, 0, 1024);
            const uint64_t dp = make_smem_desc_sw128(sp + k * kUmmaK * 2, 0, 1024);
            umma_bf16_ss(d_tmem, dp, dq, idesc, acc);
            if constexpr (Cfg::kPBoxes == 2) {
              const uint64_t dp2 =
                  make_smem_desc_sw128(sp + kBlockP * kBlockK * 2 + k * kUmmaK * 2, 0, 1024);
              umma_bf16_ss(d_tmem + BN, dp2, dq, idesc, acc);
            }
          }
          umma_commit(smem_u32(&tail->empty[stage]));  // stage reusable once these MMAs retire
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(smem_u32(&tail->tmem_full[buf]));
      }
    }
  } else {
    // ======================= epilogue (warps 2..5) ========================
    const int quad = warp & 3;        // TMEM lane quadrant this warp may read
    const int p = quad * 32 + lane;   // accumulator row owned by this thread
    const int epi_tid = threadIdx.x - 64;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++it) {
      const Unit t = dec.decode(u);
      const int buf = it & 1;
      const uint32_t buf_phase = (it >> 1) & 1;
      if (!mbar_wait(smem_u32(&tail->tmem_full[buf]), buf_phase, ctx, kWaitTmemFull)) {
        ok = false;
        break;
      }
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the spin
      tc_fence_after_sync();
      const uint32_t t_acc = tmem_base + (uint32_t(quad * 32) << 16) + buf * Cfg::kAccCols;

      if constexpr (!SWAP) {
        // thread p owns output row out_row + p; 32-column chunks
        bool row_ok = p < t.rows_valid;
        __nv_bfloat16* orow;
        bool vec_ok;
        if (GROUPED && args.out_row_ptrs) {
          __nv_bfloat16* base = row_ok ? args.out_row_ptrs[t.out_row + p] : nullptr;
          row_ok = base != nullptr;
          orow = base + t.out_col;
          vec_ok = (reinterpret_cast<uintptr_t>(base) & 15) == 0;
        } else {
          orow = args.out + size_t(t.out_row + p) * args.ldo + t.out_col;
          vec_ok = (args.ldo % 8 == 0) && ((reinterpret_cast<uintptr_t>(args.out) & 15) == 0);
        }
        constexpr int kChunks = Cfg::kOutCols / 32;
#pragma unroll 1
        for (int c = 0; c < kChunks; ++c) {
          uint32_t v[32];
          float f[32];
          tmem_ld_32x32b_x32(t_acc + c * 32, v);
          if constexpr (GATED) {
            uint32_t w[32];
            tmem_ld_32x32b_x32(t_acc + BN / 2 + c * 32, w);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = silu_mul(__uint_as_float(v[j]), __uint_as_float(w[j]));
          } else {
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
          }
          if (row_ok) {
            const int col0 = c * 32;
            if (vec_ok && col0 + 32 <= t.cols_valid) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 q;
                q.x = pack_bf16x2(f[j + 0], f[j + 1]);
                q.y = pack_bf16x2(f[j + 2], f[j + 3]);
                q.z = pack_bf16x2(f[j + 4], f[j + 5]);
                q.w = pack_bf16x2(f[j + 6], f[j + 7]);
                *reinterpret_cast<uint4*>(orow + col0 + j) = q;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < t.cols_valid) orow[col0 + j] = __float2bfloat16_rn(f[j]);
            }
          }
        }
      } else {
        // swapped: thread p owns output column out_col + p; TMEM column j is
        // activation row out_row + j.  A warp stores 32 consecutive columns per row.
        const bool col_ok = p < t.cols_valid;
        constexpr int kChunks = (BN + 31) / 32;
        constexpr int kChunkCols = BN < 32 ? BN : 32;
        const bool split_k = (!GROUPED) && args.splits > 1;
        float* ws_tile = nullptr;
        if (split_k)
          ws_tile = args.ws + (size_t(t.tile_id) * args.splits + t.split) * (size_t(BN) * kBlockP);
        const int chunks_used = min(kChunks, (t.rows_valid + 31) / 32);  // columns the MMA wrote
#pragma unroll 1
        for (int c = 0; c < chunks_used; ++c) {
          float f[kChunkCols];
          if constexpr (kChunkCols == 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_acc + c * 32, v);
            if constexpr (GATED) {
              uint32_t w[32];
              tmem_ld_32x32b_x32(t_acc + BN + c * 32, w);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j)
                f[j] = silu_mul(__uint_as_float(v[j]), __uint_as_float(w[j]));
            } else {
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
            }
          } else {
            uint32_t v[16];
            tmem_ld_32x32b_x16(t_acc, v);
            if constexpr (GATED) {
              uint32_t w[16];
              tmem_ld_32x32b_x16(t_acc + BN, w);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j)
                f[j] = silu_mul(__uint_as_float(v[j]), __uint_as_float(w[j]));
            } else {
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(v[j]);
            }
          }
          if (split_k) {
#pragma unroll
            for (int j = 0; j < kChunkCols; ++j) ws_tile[(c * 32 + j) * kBlockP + p] = f[j];
          } else if (col_ok) {
#pragma unroll
            for (int j = 0; j < kChunkCols; ++j) {
              const int r = c * 32 + j;
              if (r < t.rows_valid) {
                if (GROUPED && args.out_row_ptrs) {
                  __nv_bfloat16* base = args.out_row_ptrs[t.out_row + r];
                  if (base) base[t.out_col + p] = __float2bfloat16_rn(f[j]);
                } else {
                  args.out[size_t(t.out_row + r) * args.ldo + t.out_col + p] = __float2bfloat16_rn(f[j]);
                }
              }
            }
          }
        }
        if (split_k) {
          // The slices of a tile add their partial tiles like a reduce-scatter: each waits until
          // all have stored theirs, then sums 1 / splits of the tile's elements over the slices
          // in slice order (so the result is the same from run to run) and stores them.  A launch
          // has one unit per CTA and no more units than SMs, so every slice is running; the wait is
          // bounded like the others.
          __threadfence();
          asm volatile("bar.sync 1, 128;" ::: "memory");
          int* arrivals = args.counters + t.tile_id;
          int* departures = args.counters + kSplitTileSlots + t.tile_id;
          if (epi_tid == 0) {
            atomicAdd(arrivals, 1);
            int seen = 1;
            const uint64_t t0 = globaltimer_ns();
            uint32_t spins = 0;
            while (ld_acquire_gpu(arrivals) < args.splits) {
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
            tail->last_flag = seen;
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          const bool seen = tail->last_flag != 0;
          if (seen) {
            __threadfence();
            // the valid rows of the tile as float4 elements, [row][32]; this slice's share of them
            const float* base = args.ws + size_t(t.tile_id) * args.splits * (size_t(BN) * kBlockP);
            const int total4 = t.rows_valid * (kBlockP / 4);
            const int share = (total4 + args.splits - 1) / args.splits;
            const int first = t.split * share;
            const int end = min(first + share, total4);
            constexpr int kInFlight = 4;
            const bool vec_store = (args.ldo % 4 == 0) &&
                                   ((reinterpret_cast<uintptr_t>(args.out) & 7) == 0);
            for (int i0 = first + epi_tid; i0 < end; i0 += 128 * kInFlight) {
              float4 acc[kInFlight];
#pragma unroll
              for (int i = 0; i < kInFlight; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
              for (int s = 0; s < args.splits; ++s) {
                const float4* slice = reinterpret_cast<const float4*>(base + size_t(s) * (size_t(BN) * kBlockP));
                float4 v[kInFlight];
#pragma unroll
                for (int i = 0; i < kInFlight; ++i) v[i] = __ldcg(slice + min(i0 + 128 * i, end - 1));
#pragma unroll
                for (int i = 0; i < kInFlight; ++i) {
                  acc[i].x += v[i].x;
                  acc[i].y += v[i].y;
                  acc[i].z += v[i].z;
                  acc[i].w += v[i].w;
                }
              }
#pragma unroll
              for (int i = 0; i < kInFlight; ++i) {
                const int idx = i0 + 128 * i;
                if (idx >= end) continue;
                const int r = idx / (kBlockP / 4);
                const int c4 = (idx % (kBlockP / 4)) * 4;
                __nv_bfloat16* o = args.out + size_t(t.out_row + r) * args.ldo + t.out_col + c4;
                if (vec_store && c4 + 4 <= t.cols_valid) {
                  uint2 q;
                  q.x = pack_bf16x2(acc[i].x, acc[i].y);
                  q.y = pack_bf16x2(acc[i].z, acc[i].w);
                  *reinterpret_cast<uint2*>(o) = q;
                } else {
                  if (c4 + 0 < t.cols_valid) o[0] = __float2bfloat16_rn(acc[i].x);
                  if (c4 + 1 < t.cols_valid) o[1] = __float2bfloat16_rn(acc[i].y);
                  if (c4 + 2 < t.cols_valid) o[2] = __float2bfloat16_rn(acc[i].z);
                  if (c4 + 3 < t.cols_valid) o[3] = __float2bfloat16_rn(acc[i].w);
                }
              }
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");  // all reads done; last_flag is reused by the next unit
          if (epi_tid == 0 && seen) {
            // the last slice to have read resets both counters for the next launch
            if (atomicAdd(departures, 1) == args.splits - 1) {
              *departures = 0;
              *arrivals = 0;
            }
          }
          if (!seen) ok = false;
        }
      }
      // hand the accumulator buffer back to the MMA issuer
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tail->tmem_empty[buf]));
    }
  }

  // ---- teardown ------------------------------------------------------------
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (tail->abort_flag) {
    // a wait gave up: let copies and MMAs that may still be in flight land
    for (int i = 0; i < 200; ++i) __nanosleep(1000);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace b200
