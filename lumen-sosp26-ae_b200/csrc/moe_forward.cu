// The MoE forward as one C call: the launch sequence of the routing, grouped-GEMM and
// combine entry points on one stream, with every intermediate carved out of a single
// caller-owned scratch buffer.  Host code only; the kernels live in moe_routing.cu and
// gemm_bf16.cu.
#include "lumen_b200_internal.h"

namespace {

constexpr size_t kCarveAlign = 256;

size_t round_up(size_t v) { return (v + kCarveAlign - 1) / kCarveAlign * kCarveAlign; }

// Offsets (from a 256-byte aligned base) of the intermediates of one forward.
struct MoeForwardLayout {
  size_t sorted_token_ids, sorted_weights, sorted_expert_ids, num_valid_ids, expert_offsets,
      expert_counts, route_pos, topk_ids, topk_weights, sort_scratch, xs, h, y, total;
  size_t sort_scratch_bytes;
  int max_rows;
};

MoeForwardLayout moe_forward_layout(int T, int H, int I, int E, int k) {
  MoeForwardLayout L{};
  const size_t routes = size_t(T) * k;
  const size_t P = routes + size_t(E) * 32 - k;  // padded routes, the bound of the reference layout
  const size_t blocks = (P + 31) / 32;
  L.max_rows = static_cast<int>(P);
  L.sort_scratch_bytes = lumen_b200_moe_sort_scratch_bytes(T, E, k);
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t here = at;
    at += round_up(bytes);
    return here;
  };
  L.sorted_token_ids = take(P * 4);
  L.sorted_weights = take(P * 4);
  L.sorted_expert_ids = take(blocks * 4);
  L.num_valid_ids = take(2 * 4);
  L.expert_offsets = take((size_t(E) + 1) * 4);
  L.expert_counts = take(size_t(E) * 4);
  L.route_pos = take(routes * 4);
  L.topk_ids = take(routes * 4);
  L.topk_weights = take(routes * 4);
  L.sort_scratch = take(L.sort_scratch_bytes > 4 ? L.sort_scratch_bytes : 4);
  L.xs = take(P * size_t(H) * 2);
  L.h = take(P * size_t(I) * 2);
  L.y = take(P * size_t(H) * 2);
  L.total = at;
  return L;
}

bool shape_ok(int T, int H, int I, int E, int k) {
  return T > 0 && H > 0 && I > 0 && E > 0 && k > 0 && k <= E && E <= b200::kMaxExperts &&
         H % 8 == 0 && I % 8 == 0 && size_t(T) * k + size_t(E) * 32 < (size_t(1) << 31);
}

}  // namespace

extern "C" size_t lumen_b200_moe_forward_scratch_bytes(int T, int H, int I, int E, int k) {
  if (!shape_ok(T, H, I, E, k)) return 0;
  return moe_forward_layout(T, H, I, E, k).total + kCarveAlign;  // room to align the base
}

extern "C" int lumen_b200_moe_forward(const void* x, const void* w13, const void* w2,
                                       const void* logits, const void* topk_ids,
                                       const void* topk_weights, void* out, void* scratch,
                                       size_t scratch_bytes, int T, int H, int I, int E, int k,
                                       void* stream) {
  if (!x || !w13 || !w2 || !out || !scratch) return LUMEN_B200_EINVAL;
  if (!shape_ok(T, H, I, E, k)) return LUMEN_B200_EINVAL;
  // exactly one of: logits, or both routing arrays
  if (logits ? (topk_ids || topk_weights) : !(topk_ids && topk_weights)) return LUMEN_B200_EINVAL;
  const MoeForwardLayout L = moe_forward_layout(T, H, I, E, k);
  const uintptr_t raw = reinterpret_cast<uintptr_t>(scratch);
  const uintptr_t base_addr = (raw + kCarveAlign - 1) / kCarveAlign * kCarveAlign;
  if (scratch_bytes < (base_addr - raw) + L.total) return LUMEN_B200_EWORKSPACE;
  char* base = reinterpret_cast<char*>(base_addr);

  int rc;
  if (logits) {
    rc = lumen_b200_moe_route_topk(logits, base + L.topk_ids, base + L.topk_weights, T, E, k, stream);
    if (rc != LUMEN_B200_OK) return rc;
    topk_ids = base + L.topk_ids;
    topk_weights = base + L.topk_weights;
  }
  rc = lumen_b200_moe_sort_routes(topk_ids, topk_weights, base + L.sorted_token_ids,
                                  base + L.sorted_weights, base + L.sorted_expert_ids,
                                  base + L.num_valid_ids, base + L.expert_offsets,
                                  base + L.expert_counts, base + L.route_pos, base + L.sort_scratch,
                                  L.sort_scratch_bytes > 4 ? L.sort_scratch_bytes : 4, T, E, k, 32, stream);
  if (rc != LUMEN_B200_OK) return rc;
  rc = lumen_b200_moe_permute_rows(x, base + L.sorted_token_ids, base + L.num_valid_ids, base + L.xs, T,
                                   H, L.max_rows, stream);
  if (rc != LUMEN_B200_OK) return rc;
  const int rows_hint = static_cast<int>((size_t(T) * k + E - 1) / E);
  rc = lumen_b200_moe_grouped_gemm(base + L.xs, w13, base + L.h, base + L.expert_offsets,
                                   base + L.expert_counts, L.max_rows, E, I, H, 1, rows_hint, stream);
  if (rc != LUMEN_B200_OK) return rc;
  rc = lumen_b200_moe_grouped_gemm(base + L.h, w2, base + L.y, base + L.expert_offsets,
                                   base + L.expert_counts, L.max_rows, E, H, I, 0, rows_hint, stream);
  if (rc != LUMEN_B200_OK) return rc;
  return lumen_b200_moe_combine(base + L.y, base + L.route_pos, topk_weights, out, T, H, k, stream);
}
