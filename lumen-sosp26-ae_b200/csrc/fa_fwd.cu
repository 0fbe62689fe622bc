// Flash-attention forward for sm_100a: O = softmax(scale * Q K^T [+ causal mask]) V,
// bf16 in/out, head dimension 128, grouped-query heads, fp32 softmax state.
//
// One CTA owns a pair of query tiles (2 x 128 rows of one head) and streams the K and
// V tiles of its KV head once for both.  Warp roles:
//
//   warp 0        TMA producer: Q tiles once, then K_0, V_0, K_1, V_1, ... through a ring
//   warp 1        single-thread tcgen05.mma issuer: S_t = Q_t K_j^T (operands in shared
//                 memory) and O_t += P_t V_j (P read from TMEM, V as an MN-major operand)
//   warp 2        TMEM allocator
//   warps 4..7    softmax of query tile 0: one thread per row
//   warps 8..11   softmax of query tile 1
//
// TMEM (512 columns): S_0 [0,128)  S_1 [128,256)  O_0 [256,384)  O_1 [384,512); the bf16
// probabilities P_t overwrite the first 64 columns of S_t.  The two query tiles run half
// a step apart, so the tensor core works on one tile while the other is in its softmax.
//
// Online softmax: a thread keeps the running maximum m and sum l of its row in
// registers.  The maximum is only raised (and O rescaled in TMEM) when the new maximum
// exceeds it by more than 2^8 in the exp2 domain, the lazy-rescale rule of the
// reference kernel (datasets/inference/attention/lumen/attn_06_inst_scheduling.py:694-716);
// probabilities are exp2(s * scale * log2e - m * scale * log2e), rounded to bf16 for the
// P V product as in the reference (:626,631), and summed in fp32.
#include "lumen_b200_internal.h"

namespace b200 {

constexpr int kFaThreads = 384;      // 4 copy/MMA warps + one softmax warpgroup per query tile
constexpr int kFaRegsCopy = 72;      // registers per thread kept by the copy/MMA warpgroup
constexpr int kFaRegsSoftmax = 216;  // registers per thread taken by the softmax warpgroups
static_assert(128 * kFaRegsCopy + 256 * kFaRegsSoftmax <= 384 * 168, "register file budget");
constexpr int kFaTile = 128;     // query rows per tile and keys per KV tile
constexpr int kFaD = 128;        // head dimension
constexpr int kFaHalfBytes = kFaTile * 64 * 2;   // one [128][64] bf16 swizzled panel
constexpr int kFaTileBytes = 2 * kFaHalfBytes;   // one [128][128] tile = two panels
constexpr float kLazyRescaleLog2 = 8.0f;

enum FaWaitCode {
  kFaWaitQ = 16,
  kFaWaitKvEmpty = 17,
  kFaWaitKvFull = 18,
  kFaWaitS = 19,
  kFaWaitP = 20,
  kFaWaitO = 21,
};

struct FaParams {
  __nv_bfloat16* O;
  const int* seq_ptr;  // [B + 1] first packed row of each sequence, or nullptr: B sequences of S rows
  int B, S, Hq, Hkv;
  int causal;
  float scale_log2;  // scale * log2(e)
  int q_blocks;      // ceil(longest sequence / 256)
  int* status;
};

template <int SLOTS>
struct FaSmemTail {
  uint64_t q_full;
  uint64_t kv_full[SLOTS];
  uint64_t kv_empty[SLOTS];
  uint64_t s_ready[2];
  uint64_t p_ready[2];
  uint64_t o_done[2];
  uint32_t tmem_slot;
  int abort_flag;
};

template <int SLOTS>
constexpr size_t fa_smem_bytes() {
  return 1024 + size_t(2 + SLOTS) * kFaTileBytes + sizeof(FaSmemTail<SLOTS>);
}

template <int SLOTS>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                  const __grid_constant__ CUtensorMap map_v, const FaParams prm) {
  using Tail = FaSmemTail<SLOTS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_aligned = smem_raw + (smem_base - smem_u32(smem_raw));
  Tail* tail = reinterpret_cast<Tail*>(smem_aligned + size_t(2 + SLOTS) * kFaTileBytes);
  const uint32_t smem_q = smem_base;                     // two query tiles
  const uint32_t smem_kv = smem_base + 2 * kFaTileBytes;  // ring of K/V tiles

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const AbortCtx ctx{&tail->abort_flag, prm.status};

  // ---- work decode: heavy (late) query blocks first ---------------------------------
  const int hq = blockIdx.x % prm.Hq;
  const int b = (blockIdx.x / prm.Hq) % prm.B;
  const int qb = prm.q_blocks - 1 - blockIdx.x / (prm.Hq * prm.B);
  const int hk = hq / (prm.Hq / prm.Hkv);
  const int q0 = qb * 2 * kFaTile;  // first query row of tile 0 (within its sequence)
  // Q, K, V, O are addressed as packed rows [sum of lengths, H, D]; sequence b owns rows
  // [row_base, row_base + seq_len).  Keys past the end of a sequence are the next sequence's
  // rows (or TMA zero fill at the very end): they are masked like any key beyond kv_lim.
  const int row_base = prm.seq_ptr ? prm.seq_ptr[b] : b * prm.S;
  const int seq_len = prm.seq_ptr ? prm.seq_ptr[b + 1] - row_base : prm.S;
  const int kv_tiles_all = (seq_len + kFaTile - 1) / kFaTile;
  int n_tiles[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int row0 = q0 + t * kFaTile;
    if (row0 >= seq_len) {
      n_tiles[t] = 0;
    } else if (prm.causal) {
      const int last_row = min(row0 + kFaTile, seq_len) - 1;
      n_tiles[t] = min(kv_tiles_all, last_row / kFaTile + 1);
    } else {
      n_tiles[t] = kv_tiles_all;
    }
  }
  const int n_max = max(n_tiles[0], n_tiles[1]);

  // ---- setup ---------------------------------------------------------------------------
  if (threadIdx.x == 0) {
    tail->abort_flag = 0;
    mbar_init(smem_u32(&tail->q_full), 1);
    for (int s = 0; s < SLOTS; ++s) {
      mbar_init(smem_u32(&tail->kv_full[s]), 1);
      mbar_init(smem_u32(&tail->kv_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&tail->s_ready[t]), 1);
      mbar_init(smem_u32(&tail->p_ready[t]), 4);  // one elected lane per softmax warp
      mbar_init(smem_u32(&tail->o_done[t]), 1);
    }
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
  }
  if (warp == 2) tmem_alloc(smem_u32(&tail->tmem_slot), 512);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = tail->tmem_slot;

  // Registers: the copy/MMA warpgroup gives most of its launch allocation back, the softmax
  // warpgroups take it (each role branch below starts with its own setmaxnreg so that the
  // register bound of a branch is visible to the compiler).
  constexpr int kRegsCopy = kFaRegsCopy;
  constexpr int kRegsSoftmax = kFaRegsSoftmax;
  if (warp == 0) {
    // ================================ TMA producer ======================================
    reg_dealloc<kRegsCopy>();
    if (lane == 0) {
      const uint32_t qbar = smem_u32(&tail->q_full);
      const int active = (n_tiles[0] > 0 ? 1 : 0) + (n_tiles[1] > 0 ? 1 : 0);
      mbar_arrive_expect_tx(qbar, active * kFaTileBytes);
      for (int t = 0; t < 2; ++t) {
        if (n_tiles[t] == 0) continue;
        const uint32_t dst = smem_q + t * kFaTileBytes;
        tma_load_3d(dst, &map_q, qbar, 0, hq, row_base + q0 + t * kFaTile);
        tma_load_3d(dst + kFaHalfBytes, &map_q, qbar, 64, hq, row_base + q0 + t * kFaTile);
      }
      bool ok = true;
      for (int seq = 0; seq < 2 * n_max && ok; ++seq) {
        const int slot = seq % SLOTS;
        const uint32_t phase = (seq / SLOTS) & 1;
        if (!mbar_wait(smem_u32(&tail->kv_empty[slot]), phase ^ 1u, ctx, kFaWaitKvEmpty)) {
          ok = false;
          break;
        }
        const uint32_t bar = smem_u32(&tail->kv_full[slot]);
        const uint32_t dst = smem_kv + slot * kFaTileBytes;
        const CUtensorMap* map = (seq & 1) ? &map_v : &map_k;
        const int row = row_base + (seq >> 1) * kFaTile;
        mbar_arrive_expect_tx(bar, kFaTileBytes);
        tma_load_3d(dst, map, bar, 0, hk, row);
        tma_load_3d(dst + kFaHalfBytes, map, bar, 64, hk, row);
      }
    }
  } else if (warp == 1) {
    // ================================ MMA issuer ========================================
    reg_dealloc<kRegsCopy>();
    if (lane == 0) {
      // S = Q K^T: both operands K-major (rows of 128 d-elements as two 64-wide panels)
      constexpr uint32_t idesc_qk = make_idesc_bf16(128, 128, 0, 0);
      // O += P V: A = P from TMEM, B = V with N (= d) contiguous: MN-major
      constexpr uint32_t idesc_pv = make_idesc_bf16(128, 128, 0, 1);
      bool ok = mbar_wait(smem_u32(&tail->q_full), 0, ctx, kFaWaitQ);

      auto issue_qk = [&](int t, uint32_t k_smem) {
        const uint32_t q_smem = smem_q + t * kFaTileBytes;
        const uint32_t d_tmem = tmem_base + t * 128;
#pragma unroll
        for (int kk = 0; kk < kFaD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kFaHalfBytes + (kk & 3) * 32;
          umma_bf16_ss(d_tmem, make_smem_desc_sw128(q_smem + off, 0, 1024),
                       make_smem_desc_sw128(k_smem + off, 0, 1024), idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, uint32_t v_smem, bool accumulate) {
        const uint32_t d_tmem = tmem_base + 256 + t * 128;
        const uint32_t p_tmem = tmem_base + t * 128;
#pragma unroll
        for (int kk = 0; kk < kFaTile / 16; ++kk) {
          // 16 keys per MMA: 16 rows of the V panels (2048 B), 8 TMEM columns of packed P
          const uint64_t vdesc = make_smem_desc_sw128(v_smem + kk * 2048, kFaHalfBytes, 1024);
          umma_bf16_ts(d_tmem, p_tmem + kk * 8, vdesc, idesc_pv, (accumulate || kk > 0) ? 1u : 0u);
        }
      };
      auto slot_addr = [&](int seq) { return smem_kv + (seq % SLOTS) * kFaTileBytes; };
      auto wait_full = [&](int seq) {
        const bool r = mbar_wait(smem_u32(&tail->kv_full[seq % SLOTS]), (seq / SLOTS) & 1, ctx,
                                 kFaWaitKvFull);
        tc_fence_after_sync();
        return r;
      };

      if (ok && n_max > 0) {
        ok = wait_full(0);
        if (ok) {
          for (int t = 0; t < 2; ++t) {
            if (n_tiles[t] > 0) {
              issue_qk(t, slot_addr(0));
              umma_commit(smem_u32(&tail->s_ready[t]));
            }
          }
          umma_commit(smem_u32(&tail->kv_empty[0]));
        }
      }
      for (int j = 0; j < n_max && ok; ++j) {
        const int vseq = 2 * j + 1;
        const int kseq = 2 * j + 2;
        // V_j and K_{j+1} were requested steps ago (the ring is four tiles deep): confirm them
        // now, while the softmax is still working, not between "P is ready" and the first P V MMA
        ok = wait_full(vseq);
        if (ok && j + 1 < n_max) ok = wait_full(kseq);
        if (!ok) break;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= n_tiles[t]) continue;
          if (!mbar_wait(smem_u32(&tail->p_ready[t]), j & 1, ctx, kFaWaitP)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_pv(t, slot_addr(vseq), j > 0);
          umma_commit(smem_u32(&tail->o_done[t]));
          if (j + 1 < n_tiles[t]) {
            issue_qk(t, slot_addr(kseq));
            umma_commit(smem_u32(&tail->s_ready[t]));
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tail->kv_empty[vseq % SLOTS]));
        if (j + 1 < n_max) umma_commit(smem_u32(&tail->kv_empty[kseq % SLOTS]));
      }
    }
  } else if (warp < 4) {
    reg_dealloc<kRegsCopy>();
  } else {
    // ================================ softmax + epilogue ================================
    reg_alloc<kRegsSoftmax>();
    const int t = (warp - 4) >> 2;          // query tile of this warpgroup
    const int quad = warp & 3;              // TMEM lane quadrant
    const int r = quad * 32 + lane;         // row of the tile
    const int q = q0 + t * kFaTile + r;     // query position
    const int n = n_tiles[t];
    const uint32_t lane_sel = uint32_t(quad * 32) << 16;
    const uint32_t s_tmem = tmem_base + lane_sel + t * 128;        // scores; packed P overwrites columns 0..63
    const uint32_t o_tmem = tmem_base + lane_sel + 256 + t * 128;  // output accumulator
    const float sl2 = prm.scale_log2;
    // last key this row may see
    const int kv_lim = prm.causal ? min(q, seq_len - 1) : seq_len - 1;

    float m = -INFINITY;  // maximum the probabilities are taken against (raw score units)
    float l = 0.f;        // running sum of probabilities
    bool ok = true;

    // raise m to m_new: O and l shrink by 2^((m - m_new) * sl2).  O of step j - 1 must be complete.
    auto raise_max = [&](float m_new, int j) {
      const float factor = fast_exp2((m - m_new) * sl2);  // 0 on the first tile
      m = m_new;
      l *= factor;
      if (j > 0) {
        if (!mbar_wait(smem_u32(&tail->o_done[t]), (j - 1) & 1, ctx, kFaWaitO)) return false;
        __syncwarp();
        tc_fence_after_sync();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(o_tmem + c * 32, ov);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * factor);
          tmem_st_32x32b_x32(o_tmem + c * 32, ov);
        }
        tmem_st_wait();
      }
      return true;
    };
    // maximum of 32 scores: independent chains of three-input max
    auto chunk_max = [](const uint32_t (&s)[32]) {
      float a = max3(__uint_as_float(s[0]), __uint_as_float(s[1]), __uint_as_float(s[2]));
      float b2 = max3(__uint_as_float(s[3]), __uint_as_float(s[4]), __uint_as_float(s[5]));
#pragma unroll
      for (int i = 6; i + 3 < 32; i += 4) {
        a = max3(a, __uint_as_float(s[i]), __uint_as_float(s[i + 1]));
        b2 = max3(b2, __uint_as_float(s[i + 2]), __uint_as_float(s[i + 3]));
      }
      return max3(a, b2, fmaxf(__uint_as_float(s[30]), __uint_as_float(s[31])));
    };
    // 32 scores -> probabilities 2^(s * sl2 + neg_m), packed to 16 bf16x2 columns at P group c
    auto emit_chunk = [&](const uint32_t (&s)[32], int c, float neg_m, float (&sum4)[4]) {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float p0 = fast_exp2(fmaf(__uint_as_float(s[i + 0]), sl2, neg_m));
        const float p1 = fast_exp2(fmaf(__uint_as_float(s[i + 1]), sl2, neg_m));
        const float p2 = fast_exp2(fmaf(__uint_as_float(s[i + 2]), sl2, neg_m));
        const float p3 = fast_exp2(fmaf(__uint_as_float(s[i + 3]), sl2, neg_m));
        sum4[0] += p0;
        sum4[1] += p1;
        sum4[2] += p2;
        sum4[3] += p3;
        pk[i / 2] = pack_bf16x2(p0, p1);
        pk[i / 2 + 1] = pack_bf16x2(p2, p3);
      }
      tmem_st_32x32b_x16(s_tmem + c * 16, pk);
    };
    auto mask_chunk = [](uint32_t (&s)[32], int first_col, int cmax) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (first_col + i > cmax) s[i] = __float_as_uint(-INFINITY);
    };

    for (int j = 0; j < n && ok; ++j) {
      if (!mbar_wait(smem_u32(&tail->s_ready[t]), j & 1, ctx, kFaWaitS)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after_sync();
      uint32_t sv[4][32];
      const int cmax = kv_lim - j * kFaTile;  // columns [0, cmax] are visible
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};

      // whole row first: maximum, lazy rescale, then the probabilities
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(s_tmem + c * 32, sv[c]);
      tmem_ld_wait();
      if (cmax < kFaTile - 1) {
#pragma unroll
        for (int c = 0; c < 4; ++c) mask_chunk(sv[c], c * 32, cmax);
      }
      const float mx = fmaxf(fmaxf(chunk_max(sv[0]), chunk_max(sv[1])), fmaxf(chunk_max(sv[2]), chunk_max(sv[3])));
      // lazy rescale: raise m only when the tile maximum is far above it (warp-uniform,
      // because the O update is a warp-collective TMEM access)
      if (__any_sync(0xffffffffu, (mx - m) * sl2 > kLazyRescaleLog2)) {
        if (!raise_max(fmaxf(m, mx), j)) {
          ok = false;
          break;
        }
      }
      const float neg_m = -m * sl2;
#pragma unroll
      for (int c = 0; c < 4; ++c) emit_chunk(sv[c], c, neg_m, sum4);
      l += (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      // P is complete in TMEM: one elected lane per warp tells the MMA thread
      tmem_st_wait();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tail->p_ready[t]));
    }

    // ---- epilogue: O / l -> bf16 -> global -------------------------------------------
    if (ok && n > 0) {
      if (mbar_wait(smem_u32(&tail->o_done[t]), (n - 1) & 1, ctx, kFaWaitO)) {
        __syncwarp();
        tc_fence_after_sync();
        const float inv_l = 1.0f / l;
        __nv_bfloat16* orow = prm.O + ((size_t(row_base) + q) * prm.Hq + hq) * kFaD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(o_tmem + c * 32, ov);
          tmem_ld_wait();
          if (q < seq_len) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(ov[i + 0]) * inv_l, __uint_as_float(ov[i + 1]) * inv_l);
              o.y = pack_bf16x2(__uint_as_float(ov[i + 2]) * inv_l, __uint_as_float(ov[i + 3]) * inv_l);
              o.z = pack_bf16x2(__uint_as_float(ov[i + 4]) * inv_l, __uint_as_float(ov[i + 5]) * inv_l);
              o.w = pack_bf16x2(__uint_as_float(ov[i + 6]) * inv_l, __uint_as_float(ov[i + 7]) * inv_l);
              *reinterpret_cast<uint4*>(orow + c * 32 + i) = o;
            }
          }
        }
      }
    }
  }

  // ---- teardown ------------------------------------------------------------------------
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (tail->abort_flag) {
    for (int i = 0; i < 200; ++i) __nanosleep(1000);
  }
  if (warp == 2) {
    __syncwarp();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace b200

using namespace b200;

namespace {

int launch_fa_kernel(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FaParams& prm,
                     long long grid, cudaStream_t st) {
  constexpr int kSlots = 4;
  auto kern = fa_fwd_kernel<kSlots>;
  constexpr size_t smem = fa_smem_bytes<kSlots>();
  static_assert(smem <= 227 * 1024, "K/V ring does not fit shared memory");
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LUMEN_B200_ECUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return LUMEN_B200_ECUDA;
    configured[dev] = true;
  }
  kern<<<static_cast<unsigned>(grid), kFaThreads, smem, st>>>(mq, mk, mv, prm);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

// rows = packed tokens; S_max = longest sequence (sizes the grid)
int launch_fa(const void* Q, const void* K, const void* V, void* O, const int* seq_ptr, int B, int S_uniform,
              long long rows, int S_max, int Hq, int Hkv, float scale, int causal, cudaStream_t st) {
  int* status = device_status_word();
  if (!status) return LUMEN_B200_ECUDA;
  auto make_map = [&](CUtensorMap* map, const void* base, int heads) {
    // [rows, H, D] contiguous, innermost first: D, H, rows; box = 64 x 1 x 128
    const uint64_t dims[3] = {uint64_t(kFaD), uint64_t(heads), uint64_t(rows)};
    const uint64_t strides[2] = {uint64_t(kFaD) * 2, uint64_t(heads) * kFaD * 2};
    const uint32_t box[3] = {64, 1, uint32_t(kFaTile)};
    return encode_tmap_bf16(map, base, 3, dims, strides, box);
  };
  CUtensorMap mq, mk, mv;
  if (make_map(&mq, Q, Hq) != 0 || make_map(&mk, K, Hkv) != 0 || make_map(&mv, V, Hkv) != 0)
    return LUMEN_B200_ECUDA;

  FaParams prm{};
  prm.O = static_cast<__nv_bfloat16*>(O);
  prm.seq_ptr = seq_ptr;
  prm.B = B;
  prm.S = S_uniform;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.causal = causal ? 1 : 0;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.q_blocks = (S_max + 2 * kFaTile - 1) / (2 * kFaTile);
  prm.status = status;

  const long long grid = static_cast<long long>(prm.q_blocks) * B * Hq;
  if (grid <= 0 || grid > 0x7fffffffLL) return LUMEN_B200_EUNSUPPORTED;
  return launch_fa_kernel(mq, mk, mv, prm, grid, st);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" int lumen_b200_fa_fwd_bf16(const void* Q, const void* K, const void* V, void* O, int B,
                                       int S, int Hq, int Hkv, int D, float scale, int causal,
                                       void* stream) {
  if (!Q || !K || !V || !O || B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0) return LUMEN_B200_EINVAL;
  if (D != kFaD) return LUMEN_B200_EUNSUPPORTED;
  if (Hq % Hkv != 0 || !(scale > 0.f)) return LUMEN_B200_EINVAL;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return LUMEN_B200_EINVAL;
  return launch_fa(Q, K, V, O, nullptr, B, S, static_cast<long long>(B) * S, S, Hq, Hkv, scale, causal,
                   static_cast<cudaStream_t>(stream));
}

extern "C" int lumen_b200_fa_fwd_varlen_bf16(const void* Q, const void* K, const void* V, void* O,
                                              const void* seq_ptr, int num_seqs, int total_tokens,
                                              int max_seq_len, int Hq, int Hkv, int D, float scale,
                                              int causal, void* stream) {
  if (!Q || !K || !V || !O || !seq_ptr || num_seqs <= 0 || total_tokens <= 0 || max_seq_len <= 0 ||
      Hq <= 0 || Hkv <= 0)
    return LUMEN_B200_EINVAL;
  if (D != kFaD) return LUMEN_B200_EUNSUPPORTED;
  if (Hq % Hkv != 0 || !(scale > 0.f) || max_seq_len > total_tokens) return LUMEN_B200_EINVAL;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return LUMEN_B200_EINVAL;
  return launch_fa(Q, K, V, O, static_cast<const int*>(seq_ptr), num_seqs, 0, total_tokens, max_seq_len, Hq,
                   Hkv, scale, causal, static_cast<cudaStream_t>(stream));
}
