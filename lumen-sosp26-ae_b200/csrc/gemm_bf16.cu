// Host launchers and C-ABI entry points of the BF16 contraction core: the dense
// GEMM C = A * B^T and the per-expert (grouped) GEMMs of the MoE.
#include "gemm_bf16.cuh"
#include "gemm_bf16_pair.cuh"
#include "gemm_bf16_pair_grouped.cuh"
#include <cstdlib>
#include <string>
#include "lumen_b200_internal.h"

namespace b200 {
namespace {

// Launch with programmatic stream serialization: the kernel may begin (up to its
// griddep_wait()) before the previous kernel of the stream has finished.  Every kernel
// launched through here waits before it touches global memory.  LUMEN_B200_PDL=0 turns the
// attribute off (measurement aid).
template <typename Kern, typename... Args>
int launch_overlapped(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  static int pdl = -1;
  if (pdl < 0) {
    const char* v = std::getenv("LUMEN_B200_PDL");
    pdl = (v && v[0] == '0') ? 0 : 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

template <int BN, int STAGES, bool SWAP, bool GATED, bool GROUPED>
int launch_gemm(const CUtensorMap& mp, const CUtensorMap& mq, const GemmArgs& args, int grid,
                cudaStream_t st) {
  auto kern = gemm_bf16_kernel<BN, STAGES, SWAP, GATED, GROUPED>;
  constexpr size_t smem = gemm_smem_bytes<BN, STAGES, SWAP, GATED, GROUPED>();
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
  return launch_overlapped(kern, dim3(grid), dim3(kGemmThreads), smem, st, mp, mq, args);
}

constexpr int kSplitCounterSlots = 2 * kSplitTileSlots;  // split-K counters at the head of a workspace

// Split of the last, partial wave of a CTA-pair launch: the `units % pairs` tiles left over
// after the full rounds are cut into `slices` K slices each, one slice per pair.
struct PairTailPlan {
  int slices;      // 1 = no split
  int tail_first;  // first split tile
  size_t bytes;    // fp32 partial tiles
};

PairTailPlan plan_pair_tail(int units, int pairs, int K, int bn) {
  PairTailPlan p{1, units, 0};
  static const bool enabled = [] {
    const char* v = std::getenv("LUMEN_B200_GEMM_TAIL");  // "0" switches the split off
    return !(v && v[0] == '0');
  }();
  if (!enabled || pairs <= 0 || units <= 0) return p;
  const int rem = units % pairs;
  if (rem == 0) return p;
  const int k_blocks = (K + kBlockK - 1) / kBlockK;
  int slices = pairs / rem;
  if (slices > k_blocks / 8) slices = k_blocks / 8;  // at least 8 K blocks per slice
  slices = slices >= 8 ? 8 : slices >= 4 ? 4 : slices >= 2 ? 2 : 1;  // a divisor of the tile's 32-column chunks
  if (slices < 2) return p;
  p.slices = slices;
  p.tail_first = units - rem;
  p.bytes = size_t(rem) * slices * kPairTileM * bn * sizeof(float);
  return p;
}

// dense GEMM on CTA pairs (clusters of 2); grid = 2 CTAs per co-resident cluster.  With a
// workspace that is large enough, the last partial wave is split along K.
template <int STAGES, int BN, bool GROUPED = false, bool GATED = false>
int launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& args_in, int units,
                     void* workspace, size_t workspace_bytes, cudaStream_t st) {
  auto kern = gemm_bf16_pair_kernel<STAGES, BN, GROUPED, GATED>;
  constexpr size_t smem = gemm_pair_smem_bytes<STAGES, BN, GROUPED>();
  static_assert(smem <= 227 * 1024, "stage ring does not fit shared memory");
  static bool configured[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LUMEN_B200_ECUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return LUMEN_B200_ECUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = device_sm_count() / 2;
    }
    max_clusters[dev] = n;
    configured[dev] = true;
  }
  GemmArgs args = args_in;
  args.splits = 1;
  args.tail_first = units;
  if (GROUPED)  // the unit count is on the device: one resident pair per two SMs
    return launch_overlapped(kern, dim3(2 * max_clusters[dev]), dim3(kGemmThreads), smem, st, ma, mb, args);
  int work = units;
  const PairTailPlan plan = plan_pair_tail(units, max_clusters[dev], args.K, BN);
  constexpr size_t counter_bytes = size_t(kSplitCounterSlots) * sizeof(int);
  if (plan.slices > 1 && workspace && workspace_bytes >= counter_bytes + plan.bytes) {
    // the arrival counters at the head of the workspace are zero on entry (the caller zero-fills
    // a new workspace once) and the kernel leaves them zero
    args.splits = plan.slices;
    args.tail_first = plan.tail_first;
    args.counters = static_cast<int*>(workspace);
    args.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + counter_bytes);
    work = plan.tail_first + (units - plan.tail_first) * plan.slices;
  }
  const int clusters = work < max_clusters[dev] ? work : max_clusters[dev];
  return launch_overlapped(kern, dim3(2 * clusters), dim3(kGemmThreads), smem, st, ma, mb, args);
}

// grouped GEMM on CTA pairs (weights on the accumulator rows, tokens on the MMA's N)
template <int STAGES, bool GATED>
int launch_gemm_pair_grouped(const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& mx_tail,
                             const GemmArgs& args, cudaStream_t st) {
  auto kern = gemm_bf16_pair_grouped_kernel<STAGES, GATED>;
  constexpr size_t smem = gemm_pg_smem_bytes<STAGES, GATED>();
  static_assert(smem <= 227 * 1024, "stage ring does not fit shared memory");
  static bool configured[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LUMEN_B200_ECUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return LUMEN_B200_ECUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = device_sm_count() / 2;
    }
    max_clusters[dev] = n;
    configured[dev] = true;
  }
  return launch_overlapped(kern, dim3(2 * max_clusters[dev]), dim3(kGemmThreads), smem, st, mw, mx, mx_tail, args);
}

// Grouped GEMMs with many rows per expert: the one-CTA 128 x 256 token-major tiling, or,
// when the environment variable LUMEN_B200_MOE_TILE says "pair", the CTA-pair kernel with
// the tokens on the MMA's N.
bool use_pair_grouped() {
  static int cached = -1;
  if (cached < 0) {
    const char* v = std::getenv("LUMEN_B200_MOE_TILE");
    cached = (v && v[0] == 'p') ? 1 : 0;
  }
  return cached == 1;
}

// Rows per expert (the caller's hint) from which the expert GEMMs run on CTA pairs with the tokens
// on the 256 accumulator rows; LUMEN_B200_MOE_PAIR_ROWS overrides (0 = never).
int token_pair_min_rows() {
  static const int rows = [] {
    const char* v = std::getenv("LUMEN_B200_MOE_PAIR_ROWS");
    if (!v) return 768;
    const int r = std::atoi(v);
    return r > 0 ? r : (1 << 30);
  }();
  return rows;
}

// Width of the pair tile.  128-column tiles would cut the idle tail of the last wave in
// half, but a 256 x 128 pair MMA runs at about two thirds of the 256 x 256 rate (measured:
// 1035 against 1515 TFLOP/s on 8192 x 4096 x 4096), so the wide tile always wins; the narrow
// instance stays selectable with LUMEN_B200_GEMM_TILE=pair128 for measurement.
int pick_pair_tile_n(int, int, int) { return 256; }

// Tile choice for the dense path: "pair" (256 x 256 per CTA pair) unless the environment
// variable LUMEN_B200_GEMM_TILE says "single" (128 x 256 per CTA).
bool use_pair_tiles() {
  static int cached = -1;
  if (cached < 0) {
    const char* v = std::getenv("LUMEN_B200_GEMM_TILE");
    cached = (v && v[0] == 's') ? 0 : 1;
  }
  return cached == 1;
}

// LUMEN_B200_GEMM_TILE=pair128 / pair256 pins the pair tile width (0 = choose per shape)
int forced_pair_tile_n() {
  static int cached = -1;
  if (cached < 0) {
    const char* v = std::getenv("LUMEN_B200_GEMM_TILE");
    cached = 0;
    if (v && std::string(v) == "pair128") cached = 128;
    if (v && std::string(v) == "pair256") cached = 256;
  }
  return cached;
}

inline int ceil_div_h(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }


// swapped dense path: tile geometry and split-K plan for M <= 128
struct SwapPlan {
  int bn;       // activation rows per tile (UMMA N)
  int tiles;    // output tiles
  int splits;   // K slices per tile
  size_t counter_bytes;
  size_t partial_bytes;
};

SwapPlan plan_swap(int M, int N, int K, int sms) {
  SwapPlan p;
  p.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  p.tiles = ceil_div_h(N, kBlockP) * ceil_div_h(M, p.bn);
  const int k_blocks = ceil_div_h(K, kBlockK);
  // one unit per CTA: as many K slices as fit the SMs, at least 4 K blocks per slice.  Every
  // slice adds 1 / splits of the tile, so the reduction does not grow with the slice count; the
  // cap bounds the partial-sum traffic (splits x the tile in fp32, written and read once).
  int splits = sms / p.tiles;
  const int max_splits = k_blocks / 4 > 0 ? k_blocks / 4 : 1;
  if (splits > max_splits) splits = max_splits;
  static const int cap = [] {
    const char* v = std::getenv("LUMEN_B200_SPLIT_CAP");  // measurement aid
    const int c = v ? std::atoi(v) : 0;
    return c > 0 ? c : 16;
  }();
  if (splits > cap) splits = cap;
  if (splits < 1 || p.tiles > kSplitTileSlots) splits = 1;
  p.splits = splits;
  // the counters own a fixed region at the head of the scratch buffer, so that partial
  // sums of one shape never land where another shape keeps its counters
  p.counter_bytes = size_t(kSplitCounterSlots) * sizeof(int);
  p.partial_bytes = splits > 1 ? size_t(p.tiles) * splits * p.bn * kBlockP * sizeof(float) : 0;
  return p;
}

}  // namespace
}  // namespace b200

using namespace b200;

// The dense GEMM streams weights (swapped orientation, split-K) when there are few
// activation rows, and also when the problem is so small that 256 x 256 tiles would
// leave most CTA pairs idle (e.g. one GPU's column shard of a modest GEMM).
static bool takes_streaming_path(int M, int N, int K, int sms) {
  if (M <= 128) return true;
  static const int forced = [] {
    const char* v = std::getenv("LUMEN_B200_GEMM_SMALL");  // measurement aid: "pair" / "stream"
    return (v && v[0] == 'p') ? 1 : (v && v[0] == 's') ? 2 : 0;
  }();
  if (forced == 1) return false;
  const long long pair_units =
      static_cast<long long>((M + kPairTileM - 1) / kPairTileM) * ((N + 255) / 256);
  const long long swap_tiles = static_cast<long long>((N + kBlockP - 1) / kBlockP) * ((M + 127) / 128);
  return pair_units * 5 < static_cast<long long>(sms / 2) * 2 && swap_tiles <= sms && K >= 512;
}

extern "C" size_t lumen_b200_gemm_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int sms = device_sm_count();
  if (sms <= 0) return 0;
  if (!takes_streaming_path(M, N, K, sms)) {
    if (!use_pair_tiles()) return 0;
    // CTA pairs: room for the K slices of the last partial wave, if this shape has one to split
    const int bn = forced_pair_tile_n() ? forced_pair_tile_n() : pick_pair_tile_n(M, N, sms / 2);
    const int units = ((M + kPairTileM - 1) / kPairTileM) * ((N + bn - 1) / bn);
    const PairTailPlan tail = plan_pair_tail(units, sms / 2, K, bn);
    return tail.slices > 1 ? size_t(kSplitCounterSlots) * sizeof(int) + tail.bytes : 0;
  }
  const SwapPlan p = plan_swap(M, N, K, sms);
  return p.splits > 1 ? p.counter_bytes + p.partial_bytes : 0;
}

extern "C" int lumen_b200_gemm_bf16_nt(const void* A, const void* B, void* C, int M, int N, int K,
                                        int lda, int ldb, int ldc, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0) return LUMEN_B200_EINVAL;
  if (lda < K || ldb < K || ldc < N) return LUMEN_B200_EINVAL;
  if (lda % 8 != 0 || ldb % 8 != 0) return LUMEN_B200_EINVAL;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
    return LUMEN_B200_EINVAL;
  const int sms = device_sm_count();
  int* status = device_status_word();
  if (sms <= 0 || !status) return LUMEN_B200_ECUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  GemmArgs args{};
  args.out = static_cast<__nv_bfloat16*>(C);
  args.ldo = ldc;
  args.M = M;
  args.N = N;
  args.K = K;
  args.splits = 1;
  args.status = status;

  CUtensorMap mp, mq;
  const bool streaming = takes_streaming_path(M, N, K, sms);
  if (!streaming && use_pair_tiles()) {
    // CTA pairs: each CTA loads 128-row boxes of A and of B
    const int bn = forced_pair_tile_n() ? forced_pair_tile_n() : pick_pair_tile_n(M, N, sms / 2);
    if (encode_tmap_bf16_2d(&mp, A, M, K, lda, kBlockP) != 0) return LUMEN_B200_ECUDA;
    if (encode_tmap_bf16_2d(&mq, B, N, K, ldb, bn / 2) != 0) return LUMEN_B200_ECUDA;
    const int units = ((M + kPairTileM - 1) / kPairTileM) * ((N + bn - 1) / bn);
    return bn == 128 ? launch_gemm_pair<8, 128>(mp, mq, args, units, workspace, workspace_bytes, st)
                     : launch_gemm_pair<6, 256>(mp, mq, args, units, workspace, workspace_bytes, st);
  }
  if (!streaming) {
    // P = A (128-row boxes), Q = B (256-row boxes)
    if (encode_tmap_bf16_2d(&mp, A, M, K, lda, kBlockP) != 0) return LUMEN_B200_ECUDA;
    if (encode_tmap_bf16_2d(&mq, B, N, K, ldb, 256) != 0) return LUMEN_B200_ECUDA;
    const int units = ceil_div_h(M, kBlockP) * ceil_div_h(N, 256);
    const int grid = units < sms ? units : sms;
    return launch_gemm<256, 4, false, false, false>(mp, mq, args, grid, st);
  }

  // weight-streaming path: P = B (weights on the TMEM lanes), Q = A
  SwapPlan plan = plan_swap(M, N, K, sms);
  if (plan.splits > 1) {
    if (!workspace || workspace_bytes < plan.counter_bytes + plan.partial_bytes) {
      if (workspace) return LUMEN_B200_EWORKSPACE;
      plan.splits = 1;
    }
  }
  if (plan.splits > 1) {
    args.splits = plan.splits;
    args.counters = static_cast<int*>(workspace);
    args.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + plan.counter_bytes);
    // the arrival counters at the head of the workspace are zero on entry (the caller
    // zero-fills a new workspace once) and the kernel leaves them zero
  }
  if (encode_tmap_bf16_2d(&mp, B, N, K, ldb, kBlockP) != 0) return LUMEN_B200_ECUDA;
  if (encode_tmap_bf16_2d(&mq, A, M, K, lda, plan.bn) != 0) return LUMEN_B200_ECUDA;
  const int units = plan.tiles * plan.splits;
  const int grid = units < sms ? units : sms;
  switch (plan.bn) {
    case 16:
      return launch_gemm<16, 10, true, false, false>(mp, mq, args, grid, st);
    case 32:
      return launch_gemm<32, 10, true, false, false>(mp, mq, args, grid, st);
    case 64:
      return launch_gemm<64, 8, true, false, false>(mp, mq, args, grid, st);
    default:
      return launch_gemm<128, 6, true, false, false>(mp, mq, args, grid, st);
  }
}

static int grouped_gemm_impl(const void* acts, const void* weights, void* out, const void* const* out_row_ptrs,
                             const void* expert_offsets, const void* expert_counts, int max_rows, int E,
                             int N, int K, int gated, int rows_hint, void* stream);

extern "C" int lumen_b200_moe_grouped_gemm(const void* acts, const void* weights, void* out,
                                            const void* expert_offsets, const void* expert_counts,
                                            int max_rows, int E, int N, int K, int gated,
                                            int rows_hint, void* stream) {
  if (!out) return LUMEN_B200_EINVAL;
  return grouped_gemm_impl(acts, weights, out, nullptr, expert_offsets, expert_counts, max_rows, E, N, K,
                           gated, rows_hint, stream);
}

extern "C" int lumen_b200_moe_grouped_gemm_to_rows(const void* acts, const void* weights,
                                                    const void* const* out_row_ptrs,
                                                    const void* expert_offsets,
                                                    const void* expert_counts, int max_rows, int E,
                                                    int N, int K, int gated, int rows_hint,
                                                    void* stream) {
  if (!out_row_ptrs) return LUMEN_B200_EINVAL;
  return grouped_gemm_impl(acts, weights, nullptr, out_row_ptrs, expert_offsets, expert_counts, max_rows, E,
                           N, K, gated, rows_hint, stream);
}

static int grouped_gemm_impl(const void* acts, const void* weights, void* out, const void* const* out_row_ptrs,
                             const void* expert_offsets, const void* expert_counts, int max_rows, int E,
                             int N, int K, int gated, int rows_hint, void* stream) {
  if (!acts || !weights || !expert_offsets || !expert_counts) return LUMEN_B200_EINVAL;
  if (max_rows <= 0 || E <= 0 || E > kMaxExperts || N <= 0 || K <= 0 || K % 8 != 0)
    return LUMEN_B200_EINVAL;
  if ((reinterpret_cast<uintptr_t>(acts) & 15) || (reinterpret_cast<uintptr_t>(weights) & 15))
    return LUMEN_B200_EINVAL;
  const int sms = device_sm_count();
  int* status = device_status_word();
  if (sms <= 0 || !status) return LUMEN_B200_ECUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  const int w_rows = gated ? 2 * N : N;
  GemmArgs args{};
  args.out = static_cast<__nv_bfloat16*>(out);
  args.ldo = N;
  args.M = 0;
  args.N = N;
  args.K = K;
  args.splits = 1;
  args.expert_offsets = static_cast<const int*>(expert_offsets);
  args.expert_counts = static_cast<const int*>(expert_counts);
  args.num_experts = E;
  args.w_rows_per_expert = w_rows;
  args.up_row_offset = N;
  args.out_row_ptrs = reinterpret_cast<__nv_bfloat16* const*>(const_cast<void* const*>(out_row_ptrs));
  args.status = status;

  const uint64_t w_total_rows = uint64_t(E) * w_rows;
  CUtensorMap mp, mq;
  const int grid = sms;
  if (rows_hint > 128 && use_pair_grouped()) {
    // CTA pairs: one weight tile x up to 320 token rows per unit, the token count is the MMA's N.
    // Weight boxes: 128 rows, or for gated units 64 gate rows + 64 up rows; token boxes: 128
    // rows for the first 256 tokens of a unit and 32 rows for the rest.
    CUtensorMap mq_tail;
    {
      static int unit = 0;  // LUMEN_B200_PG_UNIT=256 keeps every unit to one MMA (measurement aid)
      if (unit == 0) {
        const char* v = std::getenv("LUMEN_B200_PG_UNIT");
        unit = (v && std::atoi(v) >= 16 && std::atoi(v) <= kPgUnitTokens) ? std::atoi(v) : kPgUnitTokens;
      }
      args.unit_tokens = unit;
    }
    if (encode_tmap_bf16_2d(&mp, weights, w_total_rows, K, K, gated ? kBlockP / 2 : kBlockP) != 0)
      return LUMEN_B200_ECUDA;
    if (encode_tmap_bf16_2d(&mq, acts, max_rows, K, K, kBlockP) != 0) return LUMEN_B200_ECUDA;
    if (encode_tmap_bf16_2d(&mq_tail, acts, max_rows, K, K, kPgTailBox) != 0) return LUMEN_B200_ECUDA;
    return gated ? launch_gemm_pair_grouped<5, true>(mp, mq, mq_tail, args, st)
                 : launch_gemm_pair_grouped<6, false>(mp, mq, mq_tail, args, st);
  }
  // (and only with at least three rounds of 256 x 256 tiles over the CTA pairs: with one or two
  // experts per GPU the coarser tiles leave the last round mostly empty)
  const long long pair_units = static_cast<long long>(E) * ((rows_hint + kPairTileM - 1) / kPairTileM) *
                               ((N + (gated ? 127 : 255)) / (gated ? 128 : 256));
  if (rows_hint >= token_pair_min_rows() && !out_row_ptrs && pair_units >= 3LL * (sms / 2)) {
    // many rows per expert: CTA pairs, 256 token rows x 256 weight rows per unit (gated: 64 gate +
    // 64 up rows per CTA), the tile shape that feeds the tensor core at full rate
    if (encode_tmap_bf16_2d(&mp, acts, max_rows, K, K, kBlockP) != 0) return LUMEN_B200_ECUDA;
    if (encode_tmap_bf16_2d(&mq, weights, w_total_rows, K, K, gated ? 64 : 128) != 0) return LUMEN_B200_ECUDA;
    return gated ? launch_gemm_pair<6, 256, true, true>(mp, mq, args, 0, nullptr, 0, st)
                 : launch_gemm_pair<6, 256, true, false>(mp, mq, args, 0, nullptr, 0, st);
  }
  if (rows_hint > 128) {
    // tokens on the TMEM lanes, 128 rows per unit
    if (encode_tmap_bf16_2d(&mp, acts, max_rows, K, K, kBlockP) != 0) return LUMEN_B200_ECUDA;
    if (encode_tmap_bf16_2d(&mq, weights, w_total_rows, K, K, gated ? 128 : 256) != 0)
      return LUMEN_B200_ECUDA;
    return gated ? launch_gemm<256, 4, false, true, true>(mp, mq, args, grid, st)
                 : launch_gemm<256, 4, false, false, true>(mp, mq, args, grid, st);
  }
  // up to ~128 rows per expert: weights on the TMEM lanes, the expert's rows are the MMA's
  // N dimension (sized per unit, so ragged expert loads waste little).  Beyond that the
  // 128 x 256 token-major tile wins: a 128 x 128 MMA with both operands in shared memory is
  // bound by shared-memory bandwidth (measured: 4.18 ms against 3.98 ms for the gated GEMM
  // of the 256-expert configuration at 8192 tokens).
  const int bn = rows_hint <= 16 ? 16 : rows_hint <= 32 ? 32 : rows_hint <= 64 ? 64 : (gated ? 128 : 256);
  if (encode_tmap_bf16_2d(&mp, weights, w_total_rows, K, K, kBlockP) != 0) return LUMEN_B200_ECUDA;
  if (encode_tmap_bf16_2d(&mq, acts, max_rows, K, K, bn) != 0) return LUMEN_B200_ECUDA;
  if (gated) {
    switch (bn) {
      case 16:
        return launch_gemm<16, 6, true, true, true>(mp, mq, args, grid, st);
      case 32:
        return launch_gemm<32, 6, true, true, true>(mp, mq, args, grid, st);
      case 64:
        return launch_gemm<64, 5, true, true, true>(mp, mq, args, grid, st);
      default:
        return launch_gemm<128, 4, true, true, true>(mp, mq, args, grid, st);
    }
  }
  switch (bn) {
    case 16:
      return launch_gemm<16, 10, true, false, true>(mp, mq, args, grid, st);
    case 32:
      return launch_gemm<32, 10, true, false, true>(mp, mq, args, grid, st);
    case 64:
      return launch_gemm<64, 8, true, false, true>(mp, mq, args, grid, st);
    default:
      return launch_gemm<256, 4, true, false, true>(mp, mq, args, grid, st);
  }
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the weight-streaming (M <= 128) GEMM.
//
// Some callers cannot hand this library a scratch buffer because they may not call
// cudaMalloc at all: code running inside a stream capture, plugins whose host hands
// them only their input and output tensors, and processes whose memory pool was sized
// up front and is closed to later requests.  For them the split-K scratch of the
// M <= 128 path lives in the library image itself, as a fixed array in device memory
// that every GPU loading the library keeps until the process exits.
// ---------------------------------------------------------------------------
namespace b200 {
namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per GPU

// Device storage.  In host code this name is only a handle for the runtime: it is not
// a device address, so it is never passed to a kernel; the address is looked up below.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device, looked up once per device
// with that device current.  Returns nullptr if the runtime refuses.
unsigned char* static_scratch_ptr() {
  static unsigned char* ptrs[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    unsigned char* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_static_scratch) != cudaSuccess)
      return nullptr;
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace
}  // namespace b200

extern "C" size_t lumen_b200_gemm_static_scratch_limit(void) { return kStaticScratchBytes; }

extern "C" int lumen_b200_gemm_bf16_nt_static(const void* A, const void* B, void* C, int M, int N,
                                               int K, int lda, int ldb, int ldc, void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0) return LUMEN_B200_EINVAL;
  if (M > 128) return LUMEN_B200_EUNSUPPORTED;  // larger M uses no scratch: call the plain entry point
  if (lda < K || ldb < K || ldc < N) return LUMEN_B200_EINVAL;
  if (lda % 8 != 0 || ldb % 8 != 0) return LUMEN_B200_EINVAL;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
    return LUMEN_B200_EINVAL;
  const int sms = device_sm_count();
  int* status = device_status_word();
  if (sms <= 0 || !status) return LUMEN_B200_ECUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  const SwapPlan plan = plan_swap(M, N, K, sms);
  const size_t need = plan.splits > 1 ? plan.counter_bytes + plan.partial_bytes : 0;
  if (need > kStaticScratchBytes) return LUMEN_B200_ESCRATCH_LIMIT;

  GemmArgs args{};
  args.out = static_cast<__nv_bfloat16*>(C);
  args.ldo = ldc;
  args.M = M;
  args.N = N;
  args.K = K;
  args.splits = plan.splits;
  args.status = status;
  if (plan.splits > 1) {
    unsigned char* scratch = static_scratch_ptr();
    if (!scratch) return LUMEN_B200_ECUDA;
    args.counters = reinterpret_cast<int*>(scratch);
    args.ws = reinterpret_cast<float*>(scratch + plan.counter_bytes);
    // the arrival counters must start at zero; the partial tiles are fully rewritten
    if (cudaMemsetAsync(args.counters, 0, plan.counter_bytes, st) != cudaSuccess)
      return LUMEN_B200_ECUDA;
  }
  CUtensorMap mp, mq;
  if (encode_tmap_bf16_2d(&mp, B, N, K, ldb, kBlockP) != 0) return LUMEN_B200_ECUDA;
  if (encode_tmap_bf16_2d(&mq, A, M, K, lda, plan.bn) != 0) return LUMEN_B200_ECUDA;
  const int units = plan.tiles * plan.splits;
  const int grid = units < sms ? units : sms;
  switch (plan.bn) {
    case 16:
      return launch_gemm<16, 10, true, false, false>(mp, mq, args, grid, st);
    case 32:
      return launch_gemm<32, 10, true, false, false>(mp, mq, args, grid, st);
    case 64:
      return launch_gemm<64, 8, true, false, false>(mp, mq, args, grid, st);
    default:
      return launch_gemm<128, 6, true, false, false>(mp, mq, args, grid, st);
  }
}
