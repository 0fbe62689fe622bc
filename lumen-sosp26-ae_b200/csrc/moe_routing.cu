// Memory-bound kernels of the fused MoE forward: router logits, top-k softmax
// routing, the stable expert-major sort of the T*k routes (the permutation that
// _build_sorted_routes in datasets/inference/moe/lumen/model.py:34-98 of the
// reference defines), the row gather into expert order and the weighted combine.
//
// All of them are HBM-bound integer / byte movers: vectorised 16-byte accesses,
// one warp or one CTA per row, no tensor cores.
#include "lumen_b200_internal.h"

namespace b200 {

constexpr int kRouteChunk = 1024;  // routes ranked by one CTA

// ---------------------------------------------------------------------------
// router logits: logits[t][e] = sum_h x[t][h] * wr[e][h]   (bf16 in, fp32 out)
// One warp per pair of tokens; the router matrix is staged once per CTA in
// shared memory.  Mirrors `logits = x.float() @ Wr.float().T`.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    moe_router_logits_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wr,
                             float* __restrict__ logits, int T, int H, int E) {
  extern __shared__ uint4 s_wr[];  // [E][H/8] 16-byte chunks
  const int chunks = H / 8;
  for (int i = threadIdx.x; i < E * chunks; i += blockDim.x)
    s_wr[i] = reinterpret_cast<const uint4*>(wr)[i];
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int warps_per_cta = blockDim.x >> 5;
  const int gwarp = blockIdx.x * warps_per_cta + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * warps_per_cta;

  for (int t0 = gwarp * 2; t0 < T; t0 += nwarps * 2) {
    const bool has1 = (t0 + 1) < T;
    const uint4* x0 = reinterpret_cast<const uint4*>(x + size_t(t0) * H);
    const uint4* x1 = reinterpret_cast<const uint4*>(x + size_t(has1 ? t0 + 1 : t0) * H);
    for (int e0 = 0; e0 < E; e0 += 8) {
      float acc0[8], acc1[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc0[e] = acc1[e] = 0.f;
      for (int c = lane; c < chunks; c += 32) {
        const uint4 a = __ldg(x0 + c);
        const uint4 b = __ldg(x1 + c);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
        float af[8], bf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fa = __bfloat1622float2(a2[j]);
          const float2 fb = __bfloat1622float2(b2[j]);
          af[2 * j] = fa.x;
          af[2 * j + 1] = fa.y;
          bf[2 * j] = fb.x;
          bf[2 * j + 1] = fb.y;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e0 + e < E) {
            const uint4 w = s_wr[(e0 + e) * chunks + c];
            const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 fw = __bfloat1622float2(w2[j]);
              acc0[e] = fmaf(af[2 * j], fw.x, acc0[e]);
              acc0[e] = fmaf(af[2 * j + 1], fw.y, acc0[e]);
              acc1[e] = fmaf(bf[2 * j], fw.x, acc1[e]);
              acc1[e] = fmaf(bf[2 * j + 1], fw.y, acc1[e]);
            }
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
          acc0[e] += __shfl_xor_sync(0xffffffffu, acc0[e], d);
          acc1[e] += __shfl_xor_sync(0xffffffffu, acc1[e], d);
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e0 + e < E) {
            logits[size_t(t0) * E + e0 + e] = acc0[e];
            if (has1) logits[size_t(t0 + 1) * E + e0 + e] = acc1[e];
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// top-k + softmax over the selected logits.  One warp per token.
//   ids[t][j]     = index of the j-th largest logit (ties: lowest index first)
//   weights[t][j] = softmax over the k selected logits
// Mirrors torch.topk(sorted=True) followed by softmax(topk_val)
// (scripts/benchmark/backend_moe.py:131-139 of the reference).
// VPL = logits held per lane; supports E <= 32 * VPL.
// ---------------------------------------------------------------------------
template <int VPL>
__global__ void __launch_bounds__(256)
    moe_topk_softmax_kernel(const float* __restrict__ logits, int* __restrict__ ids,
                            float* __restrict__ weights, int T, int E, int k) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const float* row = logits + size_t(t) * E;
  float v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = (e < E) ? row[e] : -INFINITY;
  }
  uint32_t taken = 0;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if (i * 32 + lane >= E) taken |= (1u << i);

  float my_val = 0.f;
  int my_idx = 0;
  float top_val = 0.f;
  for (int j = 0; j < k; ++j) {
    // lane-local best among values not yet taken
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const bool free_slot = !((taken >> i) & 1u);
      const int e = i * 32 + lane;
      if (free_slot && (bi == 0x7fffffff || v[i] > bv)) {
        bv = v[i];
        bi = e;
      }
    }
    // warp argmax, ties to the lower index
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, d);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
      const bool take = (oi != 0x7fffffff) && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi));
      if (take) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (j == 0) top_val = bv;
    if (lane == j) {
      my_val = bv;
      my_idx = bi;
    }
  }
  const float ex = (lane < k) ? expf(my_val - top_val) : 0.f;
  float sum = ex;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
  if (lane < k) {
    ids[size_t(t) * k + lane] = my_idx;
    weights[size_t(t) * k + lane] = ex / sum;
  }
}

// ---------------------------------------------------------------------------
// stable expert-major sort of the routes, in three small kernels
// ---------------------------------------------------------------------------
// (1) per-chunk histogram: block_hist[b][e] = routes of chunk b that go to expert e
__global__ void __launch_bounds__(kRouteChunk)
    moe_block_hist_kernel(const int* __restrict__ ids, int* __restrict__ block_hist, int routes,
                          int E) {
  extern __shared__ int s_hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist[e] = 0;
  __syncthreads();
  const int r = blockIdx.x * kRouteChunk + threadIdx.x;
  if (r < routes) {
    const int e = ids[r];
    if (e >= 0 && e < E) atomicAdd(&s_hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_hist[size_t(blockIdx.x) * E + e] = s_hist[e];
}

// (2) one CTA: per-expert scan over chunks, padded exclusive scan over experts,
//     block -> expert map, and the pad fill of the sorted arrays.
__global__ void __launch_bounds__(1024)
    moe_scan_kernel(int* __restrict__ block_hist /* in: counts, out: chunk bases */,
                    int* __restrict__ expert_offsets, int* __restrict__ expert_counts,
                    int* __restrict__ sorted_token_ids, float* __restrict__ sorted_weights,
                    int* __restrict__ sorted_expert_ids, int* __restrict__ num_valid_ids, int T, int k,
                    int E, int nchunks, int group) {
  __shared__ int s_warp[32];
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  // `group`: every expert's routes are padded to a multiple of it (32 = the reference
  // layout with its per-block expert map; 1 = compact, no padding, no block map)
  const int max_padded = T * k + E * group - k;
  const int max_blocks = (max_padded + group - 1) / group;
  const int sentinel = (k << 24) | T;
  for (int i = tid; i < max_padded; i += blockDim.x) {
    sorted_token_ids[i] = sentinel;
    sorted_weights[i] = 0.f;
  }
  if (sorted_expert_ids)
    for (int i = tid; i < max_blocks; i += blockDim.x) sorted_expert_ids[i] = -1;

  int carry_all = 0;  // padded routes of the experts handled in earlier rounds
  for (int e0 = 0; e0 < E; e0 += blockDim.x) {
    const int e = e0 + tid;
    int cnt = 0;
    if (e < E) {
      for (int b = 0; b < nchunks; ++b) {
        const int v = block_hist[size_t(b) * E + e];
        block_hist[size_t(b) * E + e] = cnt;
        cnt += v;
      }
    }
    const int padded = (cnt + group - 1) / group * group;
    // block-wide exclusive scan of `padded`
    int incl = padded;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = s_warp[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += o;
      }
      s_warp[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int warp_base = (warp == 0) ? 0 : s_warp[warp - 1];
    const int off = carry_all + warp_base + incl - padded;
    const int round_total = s_warp[31];
    if (e < E) {
      expert_offsets[e] = off;
      expert_counts[e] = cnt;
    }
    __syncthreads();  // the pad fill above is complete before any block id is written
    if (e < E && sorted_expert_ids) {
      for (int b = off / group; b < (off + padded) / group; ++b) sorted_expert_ids[b] = e;
    }
    carry_all += round_total;
    __syncthreads();
  }
  if (tid == 0) {
    expert_offsets[E] = carry_all;
    num_valid_ids[0] = carry_all;
    num_valid_ids[1] = T;
  }
}

// (3) stable rank inside the chunk + scatter.  Route r = t*k + slot keeps the
//     (token ascending, slot ascending) order inside its expert.
__global__ void __launch_bounds__(kRouteChunk)
    moe_rank_scatter_kernel(const int* __restrict__ ids, const float* __restrict__ weights,
                            const int* __restrict__ chunk_base, const int* __restrict__ expert_offsets,
                            int* __restrict__ sorted_token_ids, float* __restrict__ sorted_weights,
                            int* __restrict__ route_pos, int routes, int k, int E) {
  __shared__ int s_e[kRouteChunk];
  const int i = threadIdx.x;
  const int r = blockIdx.x * kRouteChunk + i;
  int e = -1;
  if (r < routes) {
    e = ids[r];
    if (e < 0 || e >= E) e = -1;
  }
  s_e[i] = e;
  __syncthreads();
  // rank = number of earlier routes of this chunk with the same expert
  const int warp_last = (i | 31);
  int rank = 0;
  for (int j = 0; j < warp_last; ++j) rank += (j < i && s_e[j] == e) ? 1 : 0;
  if (e >= 0) {
    const int pos = expert_offsets[e] + chunk_base[size_t(blockIdx.x) * E + e] + rank;
    const int token = r / k;
    const int slot = r - token * k;
    sorted_token_ids[pos] = (slot << 24) | token;
    sorted_weights[pos] = weights[r];
    route_pos[r] = pos;
  } else if (r < routes) {
    route_pos[r] = -1;
  }
}

// The same sort in one launch for up to 1024 routes (one CTA): histogram in shared memory,
// padded scan over the experts, pad fill, stable rank, scatter.  Keeps the latency of the
// small-batch (weight-streaming) MoE down: one launch instead of three.
__global__ void __launch_bounds__(kRouteChunk)
    moe_sort_one_cta_kernel(const int* __restrict__ ids, const float* __restrict__ weights,
                            int* __restrict__ expert_offsets, int* __restrict__ expert_counts,
                            int* __restrict__ sorted_token_ids, float* __restrict__ sorted_weights,
                            int* __restrict__ sorted_expert_ids, int* __restrict__ num_valid_ids,
                            int* __restrict__ route_pos, int T, int k, int E, int group) {
  __shared__ int s_e[kRouteChunk];
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_off[kMaxExperts];
  __shared__ int s_warp[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int routes = T * k;

  int e = -1;
  if (tid < routes) {
    e = ids[tid];
    if (e < 0 || e >= E) e = -1;
  }
  s_e[tid] = e;
  if (tid < E) s_cnt[tid] = 0;
  const int max_padded = routes + E * group - k;
  const int max_blocks = (max_padded + group - 1) / group;
  const int sentinel = (k << 24) | T;
  for (int i = tid; i < max_padded; i += blockDim.x) {
    sorted_token_ids[i] = sentinel;
    sorted_weights[i] = 0.f;
  }
  if (sorted_expert_ids)
    for (int i = tid; i < max_blocks; i += blockDim.x) sorted_expert_ids[i] = -1;
  __syncthreads();
  if (e >= 0) atomicAdd(&s_cnt[e], 1);
  __syncthreads();

  // padded exclusive scan over the experts (E <= 1024 = one value per thread)
  const int cnt = tid < E ? s_cnt[tid] : 0;
  const int padded = (cnt + group - 1) / group * group;
  int incl = padded;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += o;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += o;
    }
    s_warp[lane] = w;
  }
  __syncthreads();
  const int off = (warp == 0 ? 0 : s_warp[warp - 1]) + incl - padded;
  if (tid < E) {
    s_off[tid] = off;
    expert_offsets[tid] = off;
    expert_counts[tid] = cnt;
    if (sorted_expert_ids)
      for (int b = off / group; b < (off + padded) / group; ++b) sorted_expert_ids[b] = tid;
  }
  if (tid == 0) {
    const int total = s_warp[31];
    expert_offsets[E] = total;
    num_valid_ids[0] = total;
    num_valid_ids[1] = T;
  }
  __syncthreads();

  // stable rank among the routes of the same expert, then scatter (threads past the last
  // route have nothing to rank: with a handful of routes the loop is a handful of steps)
  int rank = 0;
  if (e >= 0)
    for (int j = 0; j < tid; ++j) rank += (s_e[j] == e) ? 1 : 0;
  if (e >= 0) {
    const int pos = s_off[e] + rank;
    const int token = tid / k;
    sorted_token_ids[pos] = ((tid - token * k) << 24) | token;
    sorted_weights[pos] = weights[tid];
    route_pos[tid] = pos;
  } else if (tid < routes) {
    route_pos[tid] = -1;
  }
}

// ---------------------------------------------------------------------------
// gather rows into expert order: xs[pos][:] = x[token(pos)][:], pad rows = 0.
// One CTA per sorted position; 16-byte accesses.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    moe_permute_rows_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ sorted_token_ids,
                            const int* __restrict__ num_valid_ids, __nv_bfloat16* __restrict__ xs, int T,
                            int H) {
  const int total = num_valid_ids[0];
  const int chunks = H / 8;
  for (int pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const int token = sorted_token_ids[pos] & 0xffffff;
    uint4* dst = reinterpret_cast<uint4*>(xs + size_t(pos) * H);
    if (token < T) {
      const uint4* src = reinterpret_cast<const uint4*>(x + size_t(token) * H);
      for (int c = threadIdx.x; c < chunks; c += blockDim.x) dst[c] = __ldg(src + c);
    } else {
      for (int c = threadIdx.x; c < chunks; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    }
  }
}

// ---------------------------------------------------------------------------
// weighted combine: out[t][:] = sum_slot w[t][slot] * y[route_pos[t*k+slot]][:]
// fp32 accumulation in slot order (deterministic), bf16 round-to-nearest-even out.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ route_pos,
                       const float* __restrict__ weights, __nv_bfloat16* __restrict__ out, int T, int H,
                       int k) {
  const int chunks = H / 8;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int s = 0; s < k; ++s) {
        const int pos = route_pos[size_t(t) * k + s];
        if (pos < 0) continue;
        const float w = weights[size_t(t) * k + s];
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(y + size_t(pos) * H) + c);
        const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(q2[j]);
          acc[2 * j] = fmaf(w, f.x, acc[2 * j]);
          acc[2 * j + 1] = fmaf(w, f.y, acc[2 * j + 1]);
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out + size_t(t) * H)[c] = o;
    }
  }
}

}  // namespace b200

using namespace b200;

// ===========================================================================
// C-ABI
// ===========================================================================
extern "C" int lumen_b200_moe_router_logits(const void* x, const void* wr, void* logits, int T, int H,
                                             int E, void* stream) {
  if (!x || !wr || !logits || T <= 0 || H <= 0 || E <= 0 || H % 8 != 0) return LUMEN_B200_EINVAL;
  const size_t smem = size_t(E) * H * 2;
  if (smem > 200 * 1024) return LUMEN_B200_EUNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(moe_router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024) != cudaSuccess)
      return LUMEN_B200_ECUDA;
    attr_set[dev] = true;
  }
  const int sms = device_sm_count();
  const int warps = 8;
  int grid = (T + warps * 2 - 1) / (warps * 2);
  if (grid > sms) grid = sms;
  moe_router_logits_kernel<<<grid, warps * 32, smem, st>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(wr),
      static_cast<float*>(logits), T, H, E);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_moe_route_topk(const void* logits, void* topk_ids, void* topk_weights, int T,
                                          int E, int k, void* stream) {
  if (!logits || !topk_ids || !topk_weights || T <= 0 || E <= 0 || k <= 0 || k > E || k > 32 ||
      E > 1024)
    return LUMEN_B200_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int warps = 8;
  const int grid = (T + warps - 1) / warps;
  const float* lg = static_cast<const float*>(logits);
  int* ids = static_cast<int*>(topk_ids);
  float* w = static_cast<float*>(topk_weights);
  if (E <= 32)
    moe_topk_softmax_kernel<1><<<grid, warps * 32, 0, st>>>(lg, ids, w, T, E, k);
  else if (E <= 256)
    moe_topk_softmax_kernel<8><<<grid, warps * 32, 0, st>>>(lg, ids, w, T, E, k);
  else
    moe_topk_softmax_kernel<32><<<grid, warps * 32, 0, st>>>(lg, ids, w, T, E, k);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" size_t lumen_b200_moe_sort_scratch_bytes(int T, int E, int k) {
  if (T <= 0 || E <= 0 || k <= 0) return 0;
  const size_t routes = size_t(T) * k;
  const size_t nchunks = (routes + kRouteChunk - 1) / kRouteChunk;
  return nchunks * E * sizeof(int);
}

extern "C" int lumen_b200_moe_sort_routes(const void* topk_ids, const void* topk_weights,
                                           void* sorted_token_ids, void* sorted_weights,
                                           void* sorted_expert_ids, void* num_valid_ids,
                                           void* expert_offsets, void* expert_counts, void* route_pos,
                                           void* scratch, size_t scratch_bytes, int T, int E, int k,
                                           int route_group, void* stream) {
  if (!topk_ids || !topk_weights || !sorted_token_ids || !sorted_weights || !num_valid_ids ||
      !expert_offsets || !expert_counts || !route_pos || !scratch)
    return LUMEN_B200_EINVAL;
  if (route_group < 1 || (route_group > 1 && !sorted_expert_ids)) return LUMEN_B200_EINVAL;
  // token index must fit the 24-bit field of the packed route id
  if (T <= 0 || E <= 0 || k <= 0 || E > kMaxExperts || T >= (1 << 24) || k > 127)
    return LUMEN_B200_EINVAL;
  if (scratch_bytes < lumen_b200_moe_sort_scratch_bytes(T, E, k)) return LUMEN_B200_EWORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int routes = T * k;
  const int nchunks = (routes + kRouteChunk - 1) / kRouteChunk;
  if (routes <= kRouteChunk) {
    moe_sort_one_cta_kernel<<<1, kRouteChunk, 0, st>>>(
        static_cast<const int*>(topk_ids), static_cast<const float*>(topk_weights),
        static_cast<int*>(expert_offsets), static_cast<int*>(expert_counts),
        static_cast<int*>(sorted_token_ids), static_cast<float*>(sorted_weights),
        static_cast<int*>(sorted_expert_ids), static_cast<int*>(num_valid_ids), static_cast<int*>(route_pos),
        T, k, E, route_group);
    return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
  }
  int* hist = static_cast<int*>(scratch);
  moe_block_hist_kernel<<<nchunks, kRouteChunk, E * sizeof(int), st>>>(
      static_cast<const int*>(topk_ids), hist, routes, E);
  moe_scan_kernel<<<1, 1024, 0, st>>>(hist, static_cast<int*>(expert_offsets),
                                      static_cast<int*>(expert_counts),
                                      static_cast<int*>(sorted_token_ids),
                                      static_cast<float*>(sorted_weights),
                                      static_cast<int*>(sorted_expert_ids),
                                      static_cast<int*>(num_valid_ids), T, k, E, nchunks, route_group);
  moe_rank_scatter_kernel<<<nchunks, kRouteChunk, 0, st>>>(
      static_cast<const int*>(topk_ids), static_cast<const float*>(topk_weights), hist,
      static_cast<const int*>(expert_offsets), static_cast<int*>(sorted_token_ids),
      static_cast<float*>(sorted_weights), static_cast<int*>(route_pos), routes, k, E);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_moe_permute_rows(const void* x, const void* sorted_token_ids,
                                            const void* num_valid_ids, void* xs, int T, int H,
                                            int max_rows, void* stream) {
  if (!x || !sorted_token_ids || !num_valid_ids || !xs || T <= 0 || H <= 0 || H % 8 != 0 ||
      max_rows <= 0)
    return LUMEN_B200_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = device_sm_count();
  int grid = max_rows < sms * 16 ? max_rows : sms * 16;
  moe_permute_rows_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                static_cast<const int*>(sorted_token_ids),
                                                static_cast<const int*>(num_valid_ids),
                                                static_cast<__nv_bfloat16*>(xs), T, H);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_moe_combine(const void* y, const void* route_pos, const void* topk_weights,
                                       void* out, int T, int H, int k, void* stream) {
  if (!y || !route_pos || !topk_weights || !out || T <= 0 || H <= 0 || H % 8 != 0 || k <= 0)
    return LUMEN_B200_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = device_sm_count();
  int grid = T < sms * 16 ? T : sms * 16;
  moe_combine_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(y),
                                           static_cast<const int*>(route_pos),
                                           static_cast<const float*>(topk_weights),
                                           static_cast<__nv_bfloat16*>(out), T, H, k);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

// ---------------------------------------------------------------------------
// fp8 activations with per-128-element scales -> bf16 (the harness' default storage
// format, scripts/benchmark/backend_moe.py:86-147 of the reference).  The 256-entry
// table holds the float value of every fp8 code, so e4m3fn and e4m3fnuz are both covered.
// out[t][h] = lut[q[t][h]] * scale[t][h / 128]; 16 elements per thread.
// ---------------------------------------------------------------------------
namespace b200 {
__global__ void __launch_bounds__(256)
    moe_dequant_fp8_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scale,
                           const float* __restrict__ lut, __nv_bfloat16* __restrict__ out, int T, int H) {
  __shared__ float s_lut[256];
  s_lut[threadIdx.x] = lut[threadIdx.x];
  __syncthreads();
  const int chunks_per_row = H / 16;
  const long long total = static_cast<long long>(T) * chunks_per_row;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / chunks_per_row);
    const int c = static_cast<int>(i - static_cast<long long>(t) * chunks_per_row);
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(q + static_cast<size_t>(t) * H) + c);
    const float sc = __ldg(scale + static_cast<size_t>(t) * (H / 128) + (c * 16) / 128);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
    uint32_t packed[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      packed[j] = pack_bf16x2(s_lut[b[2 * j]] * sc, s_lut[b[2 * j + 1]] * sc);
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + c * 16);
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  }
}
}  // namespace b200

extern "C" int lumen_b200_moe_dequant_fp8(const void* q, const void* scale, const void* lut, void* out, int T,
                                           int H, void* stream) {
  if (!q || !scale || !lut || !out || T <= 0 || H <= 0 || H % 128 != 0) return LUMEN_B200_EINVAL;
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return LUMEN_B200_EINVAL;
  const int sms = b200::device_sm_count();
  if (sms <= 0) return LUMEN_B200_ECUDA;
  const long long total = static_cast<long long>(T) * (H / 16);
  long long grid = (total + 255) / 256;
  if (grid > sms * 16) grid = sms * 16;
  b200::moe_dequant_fp8_kernel<<<static_cast<unsigned>(grid), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(q), static_cast<const float*>(scale), static_cast<const float*>(lut),
      static_cast<__nv_bfloat16*>(out), T, H);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

// ===========================================================================
// Expert-parallel dispatch and return over peer memory (NVLink / NVSwitch).
//
// Tokens are sharded over the G GPUs, experts too (expert e lives on GPU e / El).  Instead
// of packing a send buffer and calling a collective, the row gather of the dispatch
// writes each row straight into its final place in the owning GPU's expert-grouped
// buffer with peer stores, and after the expert GEMMs the owner writes every output row
// straight back into the source GPU's buffer.  Every GPU derives all offsets from the
// same G x E count matrix, so no sizes travel and the host reads nothing.
// ===========================================================================
namespace b200 {

constexpr int kMaxEpRanks = 16;

struct PeerPtrs {
  void* p[kMaxEpRanks];
};

// One CTA.  counts[s][e] = routes of GPU s for global expert e.
//   send_dst_start[e]          row in the owner's grouped buffer where this GPU's rows of expert e start
//   local_offsets[le], local_counts[le]   grouped layout of this GPU's own experts (El + 1 / El entries)
//   seg_start[le * G + s]      first grouped row of the rows that GPU s sent for local expert le (El*G + 1)
//   seg_home_row[le * G + s]   row in GPU s's compact sorted order where those rows came from
__global__ void __launch_bounds__(1024)
    moe_ep_plan_kernel(const int* __restrict__ counts, int G, int E, int rank, int* __restrict__ send_dst_start,
                       int* __restrict__ local_offsets, int* __restrict__ local_counts,
                       int* __restrict__ seg_start, int* __restrict__ seg_home_row,
                       const int* __restrict__ status) {
  // after a wait that gave up (a barrier that ran out) the count matrix may be incomplete:
  // keep the previous plan, whose offsets are in bounds, and let the host see the status
  if (*status != 0) return;
  __shared__ int s_prefix[kMaxExperts + 1];  // exclusive prefix over experts of the column totals
  __shared__ int s_warp[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int El = E / G;

  // block-wide exclusive scan over e of value(e); result in s_prefix[0..E]
  auto block_scan = [&](int v) {
    int incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += o;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = s_warp[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += o;
      }
      s_warp[lane] = w;
    }
    __syncthreads();
    const int base = warp == 0 ? 0 : s_warp[warp - 1];
    if (tid < E) s_prefix[tid] = base + incl - v;
    if (tid == E - 1) s_prefix[E] = base + incl;
    __syncthreads();
  };

  const int e = tid;
  int total = 0, before_me = 0;
  if (e < E) {
    for (int s = 0; s < G; ++s) {
      const int c = counts[s * E + e];
      if (s < rank) before_me += c;
      total += c;
    }
  }
  block_scan(e < E ? total : 0);
  if (e < E) {
    const int owner = e / El;
    send_dst_start[e] = s_prefix[e] - s_prefix[owner * El] + before_me;
    if (owner == rank) {
      const int le = e - rank * El;
      const int off = s_prefix[e] - s_prefix[rank * El];
      local_offsets[le] = off;
      local_counts[le] = total;
      int run = off;
      for (int s = 0; s < G; ++s) {
        seg_start[le * G + s] = run;
        run += counts[s * E + e];
      }
      if (le == El - 1) {
        local_offsets[El] = run;
        seg_start[El * G] = run;
      }
    }
  }
  __syncthreads();
  // home rows: exclusive prefix over ALL experts of each source GPU's own counts
  for (int s = 0; s < G; ++s) {
    block_scan(e < E ? counts[s * E + e] : 0);
    if (e < E && e / El == rank) seg_home_row[(e - rank * El) * G + s] = s_prefix[e];
    __syncthreads();
  }
}

// One row of `chunks` 16-byte pieces by a whole CTA: four loads in flight per thread before the
// (possibly remote) stores, so that a row does not cost a load latency per piece.
__device__ __forceinline__ void copy_row_16b(uint4* __restrict__ dst, const uint4* __restrict__ src, int chunks) {
  for (int c0 = threadIdx.x; c0 < chunks; c0 += 4 * blockDim.x) {
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + i * blockDim.x;
      if (c < chunks) v[i] = __ldg(src + c);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + i * blockDim.x;
      if (c < chunks) dst[c] = v[i];
    }
  }
}

// Dispatch: for every compactly sorted route of this GPU, copy the token's row into the
// owner GPU's grouped buffer.  One CTA per route (grid-stride), 16-byte copies.
__global__ void __launch_bounds__(256)
    moe_ep_dispatch_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ sorted_token_ids,
                           const int* __restrict__ row_expert, const int* __restrict__ expert_offsets,
                           const int* __restrict__ send_dst_start, const int* __restrict__ num_valid_ids,
                           PeerPtrs peers, int T, int H, int El, int capacity_rows, int* status) {
  if (*status != 0) return;  // an earlier wait gave up: move nothing across GPUs
  const int total = num_valid_ids[0];
  const int chunks = H / 8;
  for (int pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const int token = sorted_token_ids[pos] & 0xffffff;
    const int e = row_expert[pos];
    if (token >= T || e < 0) continue;
    const int dst_row = send_dst_start[e] + (pos - expert_offsets[e]);
    if (dst_row < 0 || dst_row >= capacity_rows) {  // never write outside the peer's buffer
      if (threadIdx.x == 0) atomicCAS(status, 0, (32 << 16) | (blockIdx.x & 0xffff));
      continue;
    }
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(peers.p[e / El]) + size_t(dst_row) * H);
    const uint4* src = reinterpret_cast<const uint4*>(x + size_t(token) * H);
    copy_row_16b(dst, src, chunks);
  }
  __threadfence_system();
}

// Return: every grouped output row goes back to the GPU it came from, at the row of that
// GPU's compact sorted order, ready for its weighted combine.
__global__ void __launch_bounds__(256)
    moe_ep_return_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ seg_start,
                         const int* __restrict__ seg_home_row, PeerPtrs peers, int H, int G, int nseg,
                         int home_capacity_rows, int* status) {
  if (*status != 0) return;  // an earlier wait gave up: move nothing across GPUs
  const int total = seg_start[nseg];
  const int chunks = H / 8;
  for (int g = blockIdx.x; g < total; g += gridDim.x) {
    // segment k with seg_start[k] <= g < seg_start[k + 1] (empty segments are skipped)
    int lo = 0, hi = nseg;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (seg_start[mid] <= g) lo = mid; else hi = mid;
    }
    const int k = lo;
    const int src_gpu = k % G;
    const int dst_row = seg_home_row[k] + (g - seg_start[k]);
    if (dst_row < 0 || dst_row >= home_capacity_rows) {
      if (threadIdx.x == 0) atomicCAS(status, 0, (33 << 16) | (blockIdx.x & 0xffff));
      continue;
    }
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(peers.p[src_gpu]) + size_t(dst_row) * H);
    const uint4* src = reinterpret_cast<const uint4*>(y + size_t(g) * H);
    copy_row_16b(dst, src, chunks);
  }
  __threadfence_system();
}

// ---------------------------------------------------------------------------
// Cross-GPU synchronisation over peer memory (no collective library on the data path).
// Every GPU owns a signal array in symmetric memory: sig[slot * 16 + r] holds the last
// epoch GPU r announced on that slot.  A barrier = bump this GPU's epoch of the slot, store
// it into every peer's array (release, system scope), then wait until every peer's entry in
// the local array has reached it (acquire).  Epochs only grow and every GPU runs the same
// sequence of barriers, so ">=" is the completion test.  The wait is bounded like every
// other wait in this library.
// ---------------------------------------------------------------------------
constexpr int kSigStride = 16;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// called by one whole CTA; threads 0..G-1 do the signalling and the waiting
__device__ void peer_barrier(const PeerPtrs& sigs, int* epochs, int slot, int rank, int G, int* status,
                             uint64_t limit_ns) {
  __shared__ int s_epoch;
  __threadfence_system();  // this GPU's earlier peer stores are visible before the signal
  __syncthreads();
  if (threadIdx.x == 0) s_epoch = ++epochs[slot];
  __syncthreads();
  const int epoch = s_epoch;
  if (threadIdx.x < G) {
    const int peer = threadIdx.x;
    st_release_sys(static_cast<int*>(sigs.p[peer]) + slot * kSigStride + rank, epoch);
    const int* mine = static_cast<const int*>(sigs.p[rank]) + slot * kSigStride + peer;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys(mine) < epoch) {
      if ((++spins & 0x3ffu) == 0u && globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(status, 0, (35 << 16) | (slot << 8) | peer);
        break;
      }
    }
  }
  __syncthreads();
  __threadfence_system();
}

// all-gather of the per-expert counts by peer stores, then a barrier: on return row s of
// the local count matrix holds GPU s's counts
__global__ void __launch_bounds__(1024)
    moe_ep_exchange_counts_kernel(const int* __restrict__ counts, int E, int rank, int G, PeerPtrs matrices,
                                  PeerPtrs sigs, int* epochs, int slot, int* status, uint64_t limit_ns) {
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int c = counts[e];
    for (int p = 0; p < G; ++p) static_cast<int*>(matrices.p[p])[rank * E + e] = c;
  }
  peer_barrier(sigs, epochs, slot, rank, G, status, limit_ns);
}

__global__ void __launch_bounds__(32)
    moe_ep_barrier_kernel(PeerPtrs sigs, int* epochs, int slot, int rank, int G, int* status,
                          uint64_t limit_ns) {
  peer_barrier(sigs, epochs, slot, rank, G, status, limit_ns);
}

// How long a GPU waits for its peers in the barriers above; host-side setting of this process.
static uint64_t g_ep_wait_limit_ns = kWaitLimitNs;

// Address of every grouped output row on its way home: row g of segment k goes to GPU
// k % G, row seg_home_row[k] + (g - seg_start[k]).  Rows past the last segment get nullptr.
__global__ void __launch_bounds__(256)
    moe_ep_row_ptrs_kernel(const int* __restrict__ seg_start, const int* __restrict__ seg_home_row,
                           PeerPtrs peers, int H, int G, int nseg, int home_capacity_rows, int max_rows,
                           __nv_bfloat16** __restrict__ row_ptrs, int* status) {
  const int total = seg_start[nseg];
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < max_rows; g += gridDim.x * blockDim.x) {
    __nv_bfloat16* ptr = nullptr;
    if (g < total) {
      int lo = 0, hi = nseg;
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (seg_start[mid] <= g) lo = mid; else hi = mid;
      }
      const int dst_row = seg_home_row[lo] + (g - seg_start[lo]);
      if (dst_row >= 0 && dst_row < home_capacity_rows)
        ptr = static_cast<__nv_bfloat16*>(peers.p[lo % G]) + size_t(dst_row) * H;
      else
        atomicCAS(status, 0, (34 << 16) | (blockIdx.x & 0xffff));
    }
    row_ptrs[g] = ptr;
  }
}

}  // namespace b200

extern "C" int lumen_b200_moe_ep_row_ptrs(const void* seg_start, const void* seg_home_row,
                                           const void* const* peer_buffers, int G, int El, int H,
                                           int max_rows, int home_capacity_rows, void* row_ptrs,
                                           void* stream) {
  if (!seg_start || !seg_home_row || !peer_buffers || !row_ptrs) return LUMEN_B200_EINVAL;
  if (G <= 0 || G > kMaxEpRanks || El <= 0 || H <= 0 || H % 8 != 0 || max_rows <= 0 ||
      home_capacity_rows <= 0)
    return LUMEN_B200_EINVAL;
  PeerPtrs peers{};
  for (int g = 0; g < G; ++g) {
    if (!peer_buffers[g] || (reinterpret_cast<uintptr_t>(peer_buffers[g]) & 15)) return LUMEN_B200_EINVAL;
    peers.p[g] = const_cast<void*>(peer_buffers[g]);
  }
  int* status = device_status_word();
  if (!status) return LUMEN_B200_ECUDA;
  const int grid = (max_rows + 255) / 256;
  moe_ep_row_ptrs_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const int*>(seg_start), static_cast<const int*>(seg_home_row), peers, H, G, El * G,
      home_capacity_rows, max_rows, static_cast<__nv_bfloat16**>(row_ptrs), status);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

static bool fill_peers(PeerPtrs& peers, const void* const* ptrs, int G, uintptr_t align_mask) {
  for (int g = 0; g < G; ++g) {
    if (!ptrs[g] || (reinterpret_cast<uintptr_t>(ptrs[g]) & align_mask)) return false;
    peers.p[g] = const_cast<void*>(ptrs[g]);
  }
  return true;
}

extern "C" int lumen_b200_moe_ep_exchange_counts(const void* counts, int E, int rank, int G,
                                                  const void* const* peer_count_matrices,
                                                  const void* const* peer_signals, void* epochs, int slot,
                                                  void* stream) {
  if (!counts || !peer_count_matrices || !peer_signals || !epochs) return LUMEN_B200_EINVAL;
  if (G <= 0 || G > kMaxEpRanks || E <= 0 || E > kMaxExperts || rank < 0 || rank >= G || slot < 0 || slot >= 4)
    return LUMEN_B200_EINVAL;
  PeerPtrs mats{}, sigs{};
  if (!fill_peers(mats, peer_count_matrices, G, 3) || !fill_peers(sigs, peer_signals, G, 3))
    return LUMEN_B200_EINVAL;
  int* status = device_status_word();
  if (!status) return LUMEN_B200_ECUDA;
  moe_ep_exchange_counts_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const int*>(counts), E, rank, G, mats, sigs, static_cast<int*>(epochs), slot, status,
      g_ep_wait_limit_ns);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_moe_ep_set_wait_limit_ns(unsigned long long limit_ns) {
  g_ep_wait_limit_ns = limit_ns ? static_cast<uint64_t>(limit_ns) : kWaitLimitNs;
  return LUMEN_B200_OK;
}

extern "C" int lumen_b200_moe_ep_barrier(int rank, int G, const void* const* peer_signals, void* epochs,
                                          int slot, void* stream) {
  if (!peer_signals || !epochs || G <= 0 || G > kMaxEpRanks || rank < 0 || rank >= G || slot < 0 || slot >= 4)
    return LUMEN_B200_EINVAL;
  PeerPtrs sigs{};
  if (!fill_peers(sigs, peer_signals, G, 3)) return LUMEN_B200_EINVAL;
  int* status = device_status_word();
  if (!status) return LUMEN_B200_ECUDA;
  moe_ep_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(sigs, static_cast<int*>(epochs), slot,
                                                                          rank, G, status, g_ep_wait_limit_ns);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_moe_ep_plan(const void* counts, int G, int E, int rank, void* send_dst_start,
                                       void* local_offsets, void* local_counts, void* seg_start,
                                       void* seg_home_row, void* stream) {
  if (!counts || !send_dst_start || !local_offsets || !local_counts || !seg_start || !seg_home_row)
    return LUMEN_B200_EINVAL;
  if (G <= 0 || G > kMaxEpRanks || E <= 0 || E > kMaxExperts || E % G != 0 || rank < 0 || rank >= G)
    return LUMEN_B200_EINVAL;
  const int* status = device_status_word();
  if (!status) return LUMEN_B200_ECUDA;
  moe_ep_plan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const int*>(counts), G, E, rank, static_cast<int*>(send_dst_start),
      static_cast<int*>(local_offsets), static_cast<int*>(local_counts), static_cast<int*>(seg_start),
      static_cast<int*>(seg_home_row), status);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_moe_ep_dispatch(const void* x, const void* sorted_token_ids, const void* row_expert,
                                           const void* expert_offsets, const void* send_dst_start,
                                           const void* num_valid_ids, const void* const* peer_buffers,
                                           int G, int T, int H, int E, int max_rows, int capacity_rows,
                                           void* stream) {
  if (!x || !sorted_token_ids || !row_expert || !expert_offsets || !send_dst_start || !num_valid_ids ||
      !peer_buffers)
    return LUMEN_B200_EINVAL;
  if (G <= 0 || G > kMaxEpRanks || E % G != 0 || T <= 0 || H <= 0 || H % 8 != 0 || max_rows <= 0 ||
      capacity_rows <= 0)
    return LUMEN_B200_EINVAL;
  PeerPtrs peers{};
  for (int g = 0; g < G; ++g) {
    if (!peer_buffers[g] || (reinterpret_cast<uintptr_t>(peer_buffers[g]) & 15)) return LUMEN_B200_EINVAL;
    peers.p[g] = const_cast<void*>(peer_buffers[g]);
  }
  int* status = device_status_word();
  const int sms = device_sm_count();
  if (!status || sms <= 0) return LUMEN_B200_ECUDA;
  const int grid = max_rows < sms * 16 ? max_rows : sms * 16;
  moe_ep_dispatch_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const int*>(sorted_token_ids),
      static_cast<const int*>(row_expert), static_cast<const int*>(expert_offsets),
      static_cast<const int*>(send_dst_start), static_cast<const int*>(num_valid_ids), peers, T, H, E / G,
      capacity_rows, status);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}

extern "C" int lumen_b200_moe_ep_return(const void* y, const void* seg_start, const void* seg_home_row,
                                         const void* const* peer_buffers, int G, int El, int H, int max_rows,
                                         int home_capacity_rows, void* stream) {
  if (!y || !seg_start || !seg_home_row || !peer_buffers) return LUMEN_B200_EINVAL;
  if (G <= 0 || G > kMaxEpRanks || El <= 0 || H <= 0 || H % 8 != 0 || max_rows <= 0 ||
      home_capacity_rows <= 0)
    return LUMEN_B200_EINVAL;
  PeerPtrs peers{};
  for (int g = 0; g < G; ++g) {
    if (!peer_buffers[g] || (reinterpret_cast<uintptr_t>(peer_buffers[g]) & 15)) return LUMEN_B200_EINVAL;
    peers.p[g] = const_cast<void*>(peer_buffers[g]);
  }
  int* status = device_status_word();
  const int sms = device_sm_count();
  if (!status || sms <= 0) return LUMEN_B200_ECUDA;
  const int grid = max_rows < sms * 16 ? max_rows : sms * 16;
  moe_ep_return_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), static_cast<const int*>(seg_start),
      static_cast<const int*>(seg_home_row), peers, H, G, El * G, home_capacity_rows, status);
  return cudaGetLastError() == cudaSuccess ? LUMEN_B200_OK : LUMEN_B200_ECUDA;
}
