// FP8 (e4m3) block-scale expert GEMMs of the MoE on the 5th-generation tensor cores.
//
// The reference's MoE stores activations and weights as fp8 codes with fp32 scales per
// 1 x 128 (activations) and 128 x 128 (weights) block, multiplies the codes and folds the
// scales into every 128-wide K block (datasets/inference/moe/lumen/fused_moe.py:400-443), and
// re-quantises the gated intermediate per row before the second GEMM (:684-788).  Here:
//
//   * one pipeline stage = one 128-wide K block = one scale block: 128 weight rows x 128
//     bytes (two such boxes for gated units: gate rows and up rows) and BN token rows x 128
//     bytes, loaded by TMA into 128-byte-swizzled shared memory;
//   * the stage's product is four tcgen05.mma.kind::f8f6f4 (K = 32) into a TMEM partial buffer
//     (weights on the 128 lanes, the unit's tokens on the columns; N is the unit's token count
//     rounded up to 16);
//   * four promotion warps read the partial out of TMEM, multiply it by
//     act_scale[token, kb] * w_scale[expert, row block, kb] and add it to fp32 accumulators
//     in registers, while the MMA warp fills the other partial buffer;
//   * the epilogue applies silu(gate) * up (gated units) and either stores bf16, or quantises:
//     per token the 128 output columns of the unit are exactly one scale block, so the block
//     maximum is a reduction over the 128 lanes, the scale is max / 448, and codes and scales
//     are stored in the layout the second GEMM reads.
//
// Activation scales are kept K-block-major ([K/128][rows], the transposed layout the
// reference's kernel uses too, datasets/inference/moe/lumen/model.py:259), so the BN scales a
// stage needs are contiguous.  Codes are OCP e4m3 ("e4m3fn"); codes in the e4m3fnuz encoding
// represent exactly half the value of the same bits (for every finite code that both
// encodings have), which callers fold into `scale_mul`.
#include "gemm_bf16.cuh"

namespace b200 {

constexpr int kF8BlockK = 128;  // K elements (bytes) per stage = one scale block
constexpr int kF8BoxBytes = kBlockP * kF8BlockK;

enum F8WaitCode { kF8WaitPartEmpty = 40, kF8WaitPartFull = 41 };

struct F8Args {
  void* out;                 // QUANT: uint8 codes [max_rows, N]; else bf16 [max_rows, N]
  float* out_scale_t;        // QUANT: [N / 128][max_rows]
  const float* act_scale_t;  // [K / 128][max_rows]
  const float* w_scale;      // [E][w_rows / 128][K / 128]
  const int* expert_offsets;
  const int* expert_counts;
  int num_experts;
  int max_rows;
  int N, K;
  int w_rows_per_expert;
  int up_row_offset;
  float scale_mul;
  int* status;
};

template <int BN, bool GATED>
struct F8Cfg {
  static constexpr int kWBoxes = GATED ? 2 : 1;
  static constexpr int kXBytes = BN * kF8BlockK;
  static constexpr int kStageBytes = kWBoxes * kF8BoxBytes + (kXBytes + 1023) / 1024 * 1024;
  static constexpr int kAccCols = GATED ? 2 * BN : BN;  // TMEM columns of one partial buffer
  static constexpr int kTmemCols = 2 * kAccCols <= 32 ? 32 : 2 * kAccCols <= 64 ? 64 : 2 * kAccCols <= 128 ? 128 : 256;
  static_assert(2 * kAccCols <= 256 && BN % 32 == 0, "partial buffers");
};

template <int BN, int STAGES>
struct F8Tail {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t part_full[2];
  uint64_t part_empty[2];
  uint32_t tmem_slot;
  int abort_flag;
  int total_units;
  int unit_start[kMaxExperts + 1];
  float warp_max[4][BN];  // quantising epilogue: per-warp maxima of |h| per token
  float col_max[BN];
  // per promotion warp: this K block's combined scales (token scale x weight-block scale) of the
  // BN tokens, for the gate rows and for the up rows, read back as broadcasts
  alignas(16) float scale_g[4][BN];
  alignas(16) float scale_u[4][BN];
};

template <int BN, int STAGES, bool GATED>
constexpr size_t f8_smem_bytes() {
  return 1024 + size_t(STAGES) * F8Cfg<BN, GATED>::kStageBytes + sizeof(F8Tail<BN, STAGES>);
}

// two fp32 -> two e4m3 codes (round to nearest even, saturating): low byte = lo
__device__ __forceinline__ uint32_t pack_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int BN, int STAGES, bool GATED, bool QUANT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_fp8_grouped_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                           const F8Args args) {
  using Cfg = F8Cfg<BN, GATED>;
  using Tail = F8Tail<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_aligned = smem_raw + (smem_base - smem_u32(smem_raw));
  Tail* tail = reinterpret_cast<Tail*>(smem_aligned + size_t(STAGES) * Cfg::kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const AbortCtx ctx{&tail->abort_flag, args.status};

  if (threadIdx.x == 0) {
    tail->abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&tail->full[s]), 1);
      mbar_init(smem_u32(&tail->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tail->part_full[b]), 1);
      mbar_init(smem_u32(&tail->part_empty[b]), 4);  // one arrival per promotion warp
    }
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
  }
  if (warp == 1) tmem_alloc(smem_u32(&tail->tmem_slot), Cfg::kTmemCols);
  // nothing above reads or writes global memory: it may overlap the previous kernel's tail
  griddep_wait();
  griddep_launch_dependents();
  // units of expert e: (128-row weight tiles) x (BN-row token tiles); warp 0 scans
  const int w_tiles = args.N / kBlockP;
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < args.num_experts; base += 32) {
      const int e = base + lane;
      const int v = (e < args.num_experts) ? ceil_div(args.expert_counts[e], BN) * w_tiles : 0;
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
  tc_fence_after_sync();

  const uint32_t tmem_base = tail->tmem_slot;
  const int total_units = tail->total_units;
  const int k_blocks = args.K / kF8BlockK;

  struct U {
    int expert, out_col, w_row, tok_row, rows;
  };
  int cursor = 0;
  auto decode = [&](int u) {
    int e = cursor;
    while (u >= tail->unit_start[e + 1]) ++e;
    cursor = e;
    const int local = u - tail->unit_start[e];
    const int cnt = args.expert_counts[e];
    const int tok_tiles = ceil_div(cnt, BN);
    const int wt = local / tok_tiles;  // token tile fastest: neighbours share a weight tile in L2
    const int tt = local - wt * tok_tiles;
    U t;
    t.expert = e;
    t.out_col = wt * kBlockP;
    t.w_row = e * args.w_rows_per_expert + t.out_col;
    t.tok_row = args.expert_offsets[e] + tt * BN;
    t.rows = min(BN, cnt - tt * BN);
    return t;
  };

  if (warp == 0) {
    // ======================= TMA producer =================================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const U t = decode(u);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, ctx, kWaitEmptyStage)) {
            ok = false;
            break;
          }
          const uint32_t bar = smem_u32(&tail->full[stage]);
          const uint32_t sw = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sx = sw + Cfg::kWBoxes * kF8BoxBytes;
          mbar_arrive_expect_tx(bar, Cfg::kWBoxes * kF8BoxBytes + Cfg::kXBytes);
          const int kx = kb * kF8BlockK;
          tma_load_2d(sw, &map_w, bar, kx, t.w_row);
          if constexpr (GATED) tma_load_2d(sw + kF8BoxBytes, &map_w, bar, kx, t.w_row + args.up_row_offset);
          tma_load_2d(sx, &map_x, bar, kx, t.tok_row);
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
      uint32_t it = 0;  // partial buffers alternate over all stages of all units
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const U t = decode(u);
        const uint32_t idesc = make_idesc_e4m3(kBlockP, (t.rows + 15) & ~15);
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const uint32_t b = it & 1u;
          if (!mbar_wait(smem_u32(&tail->full[stage]), phase, ctx, kWaitFullStage) ||
              !mbar_wait(smem_u32(&tail->part_empty[b]), ((it >> 1) & 1u) ^ 1u, ctx, kF8WaitPartEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sw = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sx = sw + Cfg::kWBoxes * kF8BoxBytes;
          const uint32_t d_tmem = tmem_base + b * Cfg::kAccCols;
#pragma unroll
          for (int k = 0; k < kF8BlockK / 32; ++k) {
            const uint64_t dx = make_smem_desc_sw128(sx + k * 32, 0, 1024);
            umma_f8_ss(d_tmem, make_smem_desc_sw128(sw + k * 32, 0, 1024), dx, idesc, k > 0 ? 1u : 0u);
            if constexpr (GATED)
              umma_f8_ss(d_tmem + BN, make_smem_desc_sw128(sw + kF8BoxBytes + k * 32, 0, 1024), dx, idesc,
                         k > 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&tail->empty[stage]));
          umma_commit(smem_u32(&tail->part_full[b]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else {
    // ======================= promotion + epilogue (warps 2..5) =============
    const int quad = warp & 3;
    const int p = quad * 32 + lane;  // accumulator row = weight row of the tile
    const int kb_total = k_blocks;
    const int w_blocks = args.w_rows_per_expert / kBlockP;
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      const U t = decode(u);
      const int chunks = (t.rows + 31) / 32;  // 32-token groups the MMAs wrote
      float acc[Cfg::kAccCols];
#pragma unroll
      for (int j = 0; j < Cfg::kAccCols; ++j) acc[j] = 0.f;
      const float* ws_g = args.w_scale + (size_t(t.expert) * w_blocks + t.out_col / kBlockP) * kb_total;
      const float* ws_u = ws_g + size_t(args.up_row_offset / kBlockP) * kb_total;
      // this lane's share of the tokens' scales of K block kb: token tok_row + 32 * i + lane
      auto load_act_scales = [&](int kb, float (&as)[BN / 32]) {
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) {
          const int row = min(t.tok_row + 32 * i + lane, args.max_rows - 1);
          as[i] = __ldg(args.act_scale_t + size_t(kb) * args.max_rows + row);
        }
      };
      // The scales of a K block are requested three blocks ahead and handed down by register
      // copies, so that a stage never waits for them (a load issued in the stage that uses it
      // costs a trip to L2 or HBM per stage, more than the stage's own work).
      struct Scales {
        float as[BN / 32];
        float wg, wu;
      };
      auto load_scales = [&](int kb, Scales& sc) {
        if (kb >= kb_total) return;
        load_act_scales(kb, sc.as);
        sc.wg = __ldg(ws_g + kb);
        sc.wu = GATED ? __ldg(ws_u + kb) : 0.f;
      };
      Scales s0{}, s1{}, s2{};
      load_scales(0, s0);
      load_scales(1, s1);
      load_scales(2, s2);
      for (int kb = 0; kb < kb_total; ++kb, ++it) {
        const uint32_t b = it & 1u;
        float as[BN / 32];
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) as[i] = s0.as[i];
        const float wg = s0.wg * args.scale_mul;
        const float wu = s0.wu * args.scale_mul;
        s0 = s1;
        s1 = s2;
        load_scales(kb + 3, s2);
        // lane l knows the scale of token 32 c + l; every lane needs all of them: through shared
        // memory, as 16-byte broadcast reads (a shuffle and two multiplies per token cost more
        // than the two multiply-adds they feed)
        float* sg = tail->scale_g[quad];
        float* su = tail->scale_u[quad];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          sg[c * 32 + lane] = as[c] * wg;
          if constexpr (GATED) su[c * 32 + lane] = as[c] * wu;
        }
        __syncwarp();
        if (!mbar_wait(smem_u32(&tail->part_full[b]), (it >> 1) & 1u, ctx, kF8WaitPartFull)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after_sync();
        const uint32_t t_part = tmem_base + (uint32_t(quad * 32) << 16) + b * Cfg::kAccCols;
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          if (c < chunks) {  // warp-uniform
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_part + c * 32, v);
            if constexpr (GATED) {
              uint32_t w[32];
              tmem_ld_32x32b_x32(t_part + BN + c * 32, w);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 g4 = *reinterpret_cast<const float4*>(sg + c * 32 + j);
                const float4 u4 = *reinterpret_cast<const float4*>(su + c * 32 + j);
                acc[c * 32 + j + 0] = fmaf(__uint_as_float(v[j + 0]), g4.x, acc[c * 32 + j + 0]);
                acc[c * 32 + j + 1] = fmaf(__uint_as_float(v[j + 1]), g4.y, acc[c * 32 + j + 1]);
                acc[c * 32 + j + 2] = fmaf(__uint_as_float(v[j + 2]), g4.z, acc[c * 32 + j + 2]);
                acc[c * 32 + j + 3] = fmaf(__uint_as_float(v[j + 3]), g4.w, acc[c * 32 + j + 3]);
                acc[BN + c * 32 + j + 0] = fmaf(__uint_as_float(w[j + 0]), u4.x, acc[BN + c * 32 + j + 0]);
                acc[BN + c * 32 + j + 1] = fmaf(__uint_as_float(w[j + 1]), u4.y, acc[BN + c * 32 + j + 1]);
                acc[BN + c * 32 + j + 2] = fmaf(__uint_as_float(w[j + 2]), u4.z, acc[BN + c * 32 + j + 2]);
                acc[BN + c * 32 + j + 3] = fmaf(__uint_as_float(w[j + 3]), u4.w, acc[BN + c * 32 + j + 3]);
              }
            } else {
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 g4 = *reinterpret_cast<const float4*>(sg + c * 32 + j);
                acc[c * 32 + j + 0] = fmaf(__uint_as_float(v[j + 0]), g4.x, acc[c * 32 + j + 0]);
                acc[c * 32 + j + 1] = fmaf(__uint_as_float(v[j + 1]), g4.y, acc[c * 32 + j + 1]);
                acc[c * 32 + j + 2] = fmaf(__uint_as_float(v[j + 2]), g4.z, acc[c * 32 + j + 2]);
                acc[c * 32 + j + 3] = fmaf(__uint_as_float(v[j + 3]), g4.w, acc[c * 32 + j + 3]);
              }
            }
          }
        }
        __syncwarp();  // every lane has read the scales before the next K block overwrites them
        // the partial is in registers: hand its buffer back to the MMA issuer
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tail->part_empty[b]));
      }
      // the four warps go on together or stop together (the quantising epilogue meets at
      // barriers, which a warp that gave up would never reach)
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

      // ---- epilogue of the unit ------------------------------------------------------
      const int col = t.out_col + p;
      if constexpr (GATED) {
#pragma unroll
        for (int j = 0; j < BN; ++j) acc[j] = silu_mul(acc[j], acc[BN + j]);
      }
      if constexpr (!QUANT) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(args.out);
#pragma unroll
        for (int j = 0; j < BN; ++j)
          if (j < t.rows) out[size_t(t.tok_row + j) * args.N + col] = __float2bfloat16_rn(acc[j]);
      } else {
        // per token: maximum of |h| over the unit's 128 columns = over the 128 lanes
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(acc[j])));
          if (lane == (j & 31)) tail->warp_max[quad][j] = __uint_as_float(m);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        for (int j = p; j < BN; j += 128)
          tail->col_max[j] = fmaxf(fmaxf(tail->warp_max[0][j], tail->warp_max[1][j]),
                                   fmaxf(tail->warp_max[2][j], tail->warp_max[3][j]));
        asm volatile("bar.sync 1, 128;" ::: "memory");
        uint8_t* out = static_cast<uint8_t*>(args.out);
#pragma unroll
        for (int j = 0; j < BN; j += 2) {
          const float m0 = tail->col_max[j], m1 = tail->col_max[j + 1];
          const float q0 = m0 > 0.f ? 448.0f / m0 : 0.f, q1 = m1 > 0.f ? 448.0f / m1 : 0.f;
          const uint32_t codes = pack_e4m3x2(acc[j] * q0, acc[j + 1] * q1);
          if (j < t.rows) out[size_t(t.tok_row + j) * args.N + col] = static_cast<uint8_t>(codes & 0xffu);
          if (j + 1 < t.rows) out[size_t(t.tok_row + j + 1) * args.N + col] = static_cast<uint8_t>(codes >> 8);
        }
        // one thread per token writes the block's scale (K-block-major for the next GEMM)
        for (int j = p; j < t.rows; j += 128) {
          const float m = tail->col_max[j];
          args.out_scale_t[size_t(t.out_col / kBlockP) * args.max_rows + t.tok_row + j] = m > 0.f ? m / 448.0f : 1.0f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // col_max is reused by the next unit
      }
    }
  }

  // ---- teardown ------------------------------------------------------------
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (tail->abort_flag) {
    for (int i = 0; i < 200; ++i) __nanosleep(1000);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// scale_t[kb][pos] = scale[token(sorted_token_ids[pos])][kb] for pos < num_valid_ids[0], 1 for
// pad rows and beyond: the activation scales gathered into expert order, K-block-major.
__global__ void __launch_bounds__(256)
    moe_gather_scales_t_kernel(const float* __restrict__ scale, const int* __restrict__ sorted_token_ids,
                               const int* __restrict__ num_valid_ids, float* __restrict__ out_t, int T, int KB,
                               int max_rows) {
  const int valid = num_valid_ids[0];
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       i < static_cast<long long>(KB) * max_rows; i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int kb = static_cast<int>(i / max_rows);
    const int pos = static_cast<int>(i - static_cast<long long>(kb) * max_rows);
    float v = 1.0f;
    if (pos < valid) {
      const int token = sorted_token_ids[pos] & 0xffffff;
      if (token < T) v = __ldg(scale + size_t(token) * KB + kb);
    }
    out_t[i] = v;
  }
}

namespace {

template <int BN, int STAGES, bool GATED, bool QUANT>
int launch_f8(const CUtensorMap& mw, const CUtensorMap& mx, const F8Args& args, int grid, cudaStream_t st) {
  auto kern = moe_fp8_grouped_kernel<BN, STAGES, GATED, QUANT>;
  constexpr size_t smem = f8_smem_bytes<BN, STAGES, GATED>();
  static_assert(smem <= 227 * 1024, "stage ring does not fit shared memory");
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LUMEN_B200_ECUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return LUMEN_B200_ECUDA;
    configured[dev] = true;
  }
  kern<<<grid, kGemmThreads, smem, st>>>(mw, mx, args);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int lumen_b200_moe_grouped_gemm_fp8(const void* acts_q, const void* act_scale_t,
                                                const void* weights_q, const void* w_scale, void* out,
                                                void* out_scale_t, const void* expert_offsets,
                                                const void* expert_counts, int max_rows, int E, int N, int K,
                                                int gated, int quantize_out, float scale_mul, int rows_hint,
                                                void* stream) {
  if (!acts_q || !act_scale_t || !weights_q || !w_scale || !out || !expert_offsets || !expert_counts)
    return LUMEN_B200_EINVAL;
  if (quantize_out && !out_scale_t) return LUMEN_B200_EINVAL;
  if (max_rows <= 0 || E <= 0 || E > kMaxExperts || N <= 0 || K <= 0 || !(scale_mul > 0.f)) return LUMEN_B200_EINVAL;
  if (N % kBlockP != 0 || K % kF8BlockK != 0) return LUMEN_B200_EUNSUPPORTED;  // whole 128 x 128 scale blocks
  if (quantize_out && !gated) return LUMEN_B200_EUNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(acts_q) & 15) || (reinterpret_cast<uintptr_t>(weights_q) & 15))
    return LUMEN_B200_EINVAL;
  const int sms = device_sm_count();
  int* status = device_status_word();
  if (sms <= 0 || !status) return LUMEN_B200_ECUDA;

  const int w_rows = gated ? 2 * N : N;
  F8Args args{};
  args.out = out;
  args.out_scale_t = static_cast<float*>(out_scale_t);
  args.act_scale_t = static_cast<const float*>(act_scale_t);
  args.w_scale = static_cast<const float*>(w_scale);
  args.expert_offsets = static_cast<const int*>(expert_offsets);
  args.expert_counts = static_cast<const int*>(expert_counts);
  args.num_experts = E;
  args.max_rows = max_rows;
  args.N = N;
  args.K = K;
  args.w_rows_per_expert = w_rows;
  args.up_row_offset = N;
  args.scale_mul = scale_mul;
  args.status = status;

  CUtensorMap mw, mx;
  if (encode_tmap_u8_2d(&mw, weights_q, uint64_t(E) * w_rows, K, K, kBlockP) != 0) return LUMEN_B200_ECUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Token rows per unit.  With few rows per expert the GEMM streams weights: a narrow token box
  // leaves shared memory for a deeper ring, i.e. more weight bytes in flight per SM.
  const bool narrow = rows_hint > 0 && rows_hint <= 32;
  if (gated) {
    if (encode_tmap_u8_2d(&mx, acts_q, max_rows, K, K, narrow ? 32 : 64) != 0) return LUMEN_B200_ECUDA;
    if (narrow)
      return quantize_out ? launch_f8<32, 5, true, true>(mw, mx, args, sms, st)
                          : launch_f8<32, 5, true, false>(mw, mx, args, sms, st);
    return quantize_out ? launch_f8<64, 4, true, true>(mw, mx, args, sms, st)
                        : launch_f8<64, 4, true, false>(mw, mx, args, sms, st);
  }
  if (encode_tmap_u8_2d(&mx, acts_q, max_rows, K, K, narrow ? 32 : 128) != 0) return LUMEN_B200_ECUDA;
  return narrow ? launch_f8<32, 10, false, false>(mw, mx, args, sms, st)
                : launch_f8<128, 5, false, false>(mw, mx, args, sms, st);
}

extern "C" int lumen_b200_moe_gather_scales_t(const void* scale, const void* sorted_token_ids,
                                               const void* num_valid_ids, void* out_t, int T, int KB,
                                               int max_rows, void* stream) {
  if (!scale || !sorted_token_ids || !num_valid_ids || !out_t || T <= 0 || KB <= 0 || max_rows <= 0)
    return LUMEN_B200_EINVAL;
  const int sms = device_sm_count();
  if (sms <= 0) return LUMEN_B200_ECUDA;
  const long long total = static_cast<long long>(KB) * max_rows;
  long long grid = (total + 255) / 256;
  if (grid > sms * 16) grid = sms * 16;
  moe_gather_scales_t_kernel<<<static_cast<unsigned>(grid), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(scale), static_cast<const int*>(sorted_token_ids),
      static_cast<const int*>(num_valid_ids), static_cast<float*>(out_t), T, KB, max_rows);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}
