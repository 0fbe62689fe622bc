/* liblumen_b200.so -- C-ABI of the B200 (sm_100a) inference-kernel path:
 * BF16 GEMM, flash-attention forward and fused MoE forward.
 *
 * Conventions shared by every entry point
 *   - plain pointers and sizes only; every pointer is a DEVICE pointer on the
 *     current CUDA device unless a comment says "host";
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued on it and the
 *     call returns without synchronising, so it can be captured in a CUDA graph;
 *   - no entry point allocates or frees device memory; scratch is caller-owned
 *     and sized with the matching *_bytes() helper;
 *   - inputs are borrowed and never written;
 *   - return value: LUMEN_B200_OK or a negative LUMEN_B200_E* code.  Errors found
 *     by a running kernel (a bounded wait that gave up) are reported later by
 *     lumen_b200_device_status().
 *
 * Each declaration names the interface of the reference (haohui/lumen-sosp26-ae,
 * path relative to the reference tree) that it stands in for.
 */
#ifndef LUMEN_B200_H_
#define LUMEN_B200_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LUMEN_B200_OK 0
#define LUMEN_B200_EINVAL (-1)       /* null pointer, non-positive size, misaligned pitch */
#define LUMEN_B200_EWORKSPACE (-2)   /* scratch buffer smaller than *_bytes() asks for */
#define LUMEN_B200_ECUDA (-3)        /* the CUDA runtime or driver refused a call */
#define LUMEN_B200_EUNSUPPORTED (-4) /* shape outside what the kernels cover */
#define LUMEN_B200_EDEVICE (-5)      /* a kernel recorded a wait that gave up */
#define LUMEN_B200_ESCRATCH_LIMIT (-6) /* shape needs more than the built-in scratch array holds */

/* Library identification, e.g. "lumen_b200 0.1 sm_100a".  Host pointer, static storage. */
const char* lumen_b200_version(void);

/* Number of SMs of the current device, or a negative error code. */
int lumen_b200_sm_count(void);

/* Synchronises the current device, then stores the device status word in *status
 * (host pointer): 0, or (wait site << 16 | CTA index) of the first kernel wait that
 * gave up.  Returns LUMEN_B200_OK, LUMEN_B200_EDEVICE when *status != 0, or ECUDA.
 * Stands in for the hipError_t that the reference's launch wrappers return
 * (datasets/inference/gemm/ksearch/kernel.h:7-17) and that its bindings turn into
 * a RuntimeError (datasets/inference/gemm/ksearch/best_binding.cpp:41-43). */
int lumen_b200_device_status(int* status);

/* Resets the device status word to 0 (synchronises). */
int lumen_b200_clear_status(void);

/* Enqueues on `stream` a copy of the device status word into *host_dst (page-locked host
 * memory, so that the copy is asynchronous and can be captured in a CUDA graph).  Does not
 * synchronise: the value is there once the work queued before it has run.  Lets a host loop
 * notice a wait that gave up without stalling on lumen_b200_device_status() every step --
 * the role the returned hipError_t plays for the reference's synchronous launch wrappers
 * (datasets/inference/gemm/ksearch/kernel.h:7-17). */
int lumen_b200_status_snapshot(int* host_dst, void* stream);

/* ------------------------------------------------------------------ GEMM -- */

/* C[M,N] = A[M,K] * B[N,K]^T, bf16 inputs, fp32 accumulation, bf16 output rounded
 * to nearest even.  Row-major with pitches lda, ldb, ldc in elements; lda and ldb
 * must be multiples of 8 and A, B 16-byte aligned.  M <= 128 (and problems too small
 * to fill the GPU with 256 x 256 tiles) take the weight-streaming split-K path, which
 * uses `workspace`; with workspace == NULL that path runs unsplit.  Larger problems use the
 * workspace only to split the tiles of their last, partial wave over the idle SMs: with
 * workspace == NULL, or one smaller than lumen_b200_gemm_workspace_bytes(), they run
 * unsplit with the same result up to fp32 summation order.  A new workspace must be
 * zero-filled once by the caller;
 * every call leaves its first lumen_b200_gemm_workspace_bytes() bytes reusable by the
 * next call on the same stream (calls that overlap on the GPU need separate workspaces).
 * Replaces gemm_pipeline_transposed_b(A, B, out)
 * (datasets/inference/gemm/lumen/amdgpu_gemm.py:872-923), the ksearch launch
 * wrapper (datasets/inference/gemm/ksearch/kernel.h:7-17) and
 * hipblaslt_bf16_mm_out(a, b, d)
 * (datasets/inference/gemm/hipblaslt/hipblaslt_internal_ext.cpp:124-158). */
int lumen_b200_gemm_bf16_nt(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                            int ldb, int ldc, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Scratch bytes lumen_b200_gemm_bf16_nt wants for this shape on the current device
 * (0 when the shape does not split).  Counterpart of the 32 MiB plan workspace at
 * datasets/inference/gemm/hipblaslt/hipblaslt_internal_ext.cpp:12,110. */
size_t lumen_b200_gemm_workspace_bytes(int M, int N, int K);

/* Same result as lumen_b200_gemm_bf16_nt for M <= 128, for callers that cannot give the
 * library a scratch buffer because they are not allowed to allocate device memory: code
 * that runs while a stream is being captured, plugins whose host passes them nothing
 * but their input and output tensors, processes whose memory was carved up at start-up.
 * The split-K scratch is a 16 MiB array inside the library image (see
 * lumen_b200_gemm_static_scratch_limit); each GPU that loads the library holds it until
 * the process exits.  The call allocates and frees nothing.
 *   - A shape whose split-K plan needs more than the array holds is refused with
 *     LUMEN_B200_ESCRATCH_LIMIT; M > 128 is refused with LUMEN_B200_EUNSUPPORTED (that
 *     path needs no scratch: use lumen_b200_gemm_bf16_nt with workspace == NULL).
 *   - The first call on a device looks up the array's device address and sets kernel
 *     attributes; make that first call before any stream capture begins.
 *   - All calls on one device share the one array, and it keeps whatever the previous
 *     call left there; the part that must start at zero is cleared on `stream` by the
 *     call itself.  Two calls whose kernels can overlap on the GPU (different streams)
 *     race on the array: serialise them.
 * This entry point has no counterpart in the reference. */
int lumen_b200_gemm_bf16_nt_static(const void* A, const void* B, void* C, int M, int N, int K,
                                   int lda, int ldb, int ldc, void* stream);

/* Size in bytes of the built-in scratch array used by lumen_b200_gemm_bf16_nt_static.
 * No counterpart in the reference. */
size_t lumen_b200_gemm_static_scratch_limit(void);

/* ------------------------------------------------------------- attention -- */

/* O = softmax(scale * Q K^T [+ causal mask]) V for Q,O [B,S,Hq,D] and K,V
 * [B,S,Hkv,D], bf16, contiguous; query head h reads KV head h / (Hq / Hkv).
 * D must be 128.  fp32 scores and softmax, bf16 output.
 * Replaces flash_attn(q, k, v, seq_ptr, max_seq_len, out=)
 * (datasets/inference/attention/lumen/attn_06_inst_scheduling.py:2144-2193) and
 * run(q, k, v, sm_scale) (datasets/inference/attention/ksearch/best_binding.cpp:7-68). */
int lumen_b200_fa_fwd_bf16(const void* Q, const void* K, const void* V, void* O, int B, int S,
                           int Hq, int Hkv, int D, float scale, int causal, void* stream);

/* The same forward over variable-length sequences packed along the token dimension:
 * Q,O [total_tokens,Hq,D], K,V [total_tokens,Hkv,D], seq_ptr int32 [num_seqs+1] prefix
 * sums of the lengths (device pointer), max_seq_len = the longest sequence (sizes the
 * grid).  This is the native calling convention of the reference kernel:
 * flash_attn(q, k, v, seq_ptr, max_seq_len, out=)
 * (datasets/inference/attention/lumen/attn_06_inst_scheduling.py:2144-2193), with
 * seq_ptr built as at datasets/inference/attention/lumen/model.py:75-79. */
int lumen_b200_fa_fwd_varlen_bf16(const void* Q, const void* K, const void* V, void* O,
                                  const void* seq_ptr, int num_seqs, int total_tokens,
                                  int max_seq_len, int Hq, int Hkv, int D, float scale, int causal,
                                  void* stream);

/* ------------------------------------------------------------------- MoE -- */

/* logits[T,E] (fp32) = x[T,H] * wr[E,H]^T, bf16 inputs.  E * H * 2 bytes must fit
 * 200 KiB of shared memory.  The reference draws router scores directly
 * (scripts/benchmark/backend_moe.py:125-130); this is the in-op router that
 * precedes them for a model with a router matrix. */
int lumen_b200_moe_router_logits(const void* x, const void* wr, void* logits, int T, int H, int E,
                                 void* stream);

/* topk_ids[T,k] (int32) and topk_weights[T,k] (fp32): the k largest logits of each
 * row in descending order (ties: lower index first) and the softmax over those k.
 * Replaces torch.topk(sorted=True) + softmax(topk_val)
 * (scripts/benchmark/backend_moe.py:131-139). */
int lumen_b200_moe_route_topk(const void* logits, void* topk_ids, void* topk_weights, int T, int E,
                              int k, void* stream);

size_t lumen_b200_moe_sort_scratch_bytes(int T, int E, int k);

/* Stable expert-major sort of the T*k routes.  route_group = 32 gives the reference
 * layout below; route_group = 1 gives the compact layout (no padding between experts,
 * sorted_expert_ids may be NULL) that the expert-parallel dispatch sends.  With
 * P = T*k + E*32 - k and NB = ceil(P / 32):
 *   sorted_token_ids[P]  int32  (slot << 24) | token, pads (k << 24) | T
 *   sorted_weights[P]    fp32   route weight, pads 0
 *   sorted_expert_ids[NB] int32 expert of each block of 32 sorted routes, unused -1
 *   num_valid_ids[2]     int32  {padded route count, T}
 * exactly as _build_sorted_routes (datasets/inference/moe/lumen/model.py:34-98)
 * returns them, plus what the grouped GEMM and the combine read:
 *   expert_offsets[E+1] int32  first sorted position of each expert (padded to 32)
 *   expert_counts[E]    int32  routes of each expert
 *   route_pos[T*k]      int32  sorted position of route t*k+slot */
int lumen_b200_moe_sort_routes(const void* topk_ids, const void* topk_weights,
                               void* sorted_token_ids, void* sorted_weights,
                               void* sorted_expert_ids, void* num_valid_ids, void* expert_offsets,
                               void* expert_counts, void* route_pos, void* scratch,
                               size_t scratch_bytes, int T, int E, int k, int route_group,
                               void* stream);

/* xs[pos,:] = x[token(sorted_token_ids[pos]),:] for pos < num_valid_ids[0]; pad rows
 * become 0.  max_rows = T*k + E*32 - k bounds the launch.  Replaces the gather in
 * _input_fetch_async (datasets/inference/moe/lumen/fused_moe.py:246-271). */
int lumen_b200_moe_permute_rows(const void* x, const void* sorted_token_ids,
                                const void* num_valid_ids, void* xs, int T, int H, int max_rows,
                                void* stream);

/* Per-expert GEMM over rows in expert order:
 *   gated == 0:  out[r, 0:N] = acts[r, 0:K] * W_e[0:N, 0:K]^T
 *   gated != 0:  out[r, 0:N] = silu(acts[r] * W_e[0:N]^T) * (acts[r] * W_e[N:2N]^T)
 * for every row r of expert e (expert_offsets[e] <= r < expert_offsets[e] +
 * expert_counts[e]); `weights` is [E, w_rows, K] bf16 with w_rows = N (plain) or 2N
 * (gate rows first, up rows second, the w1_q layout of
 * scripts/benchmark/backend_moe.py:162-171).  acts is [max_rows, K], out
 * [max_rows, N].  rows_hint = expected rows per expert, picks the tile orientation.
 * Replaces stage 1 + SiLU (gated) and stage 2 (plain) of
 * _fused_moe_blockscale_fp8_kernel (datasets/inference/moe/lumen/fused_moe.py:1100-1335). */
int lumen_b200_moe_grouped_gemm(const void* acts, const void* weights, void* out,
                                const void* expert_offsets, const void* expert_counts,
                                int max_rows, int E, int N, int K, int gated, int rows_hint,
                                void* stream);

/* The same per-expert GEMM with its output rows scattered: row r is written at
 * out_row_ptrs[r] (device array of max_rows device pointers; nullptr = do not store),
 * which may point into a peer GPU's memory.  With the table of
 * lumen_b200_moe_ep_row_ptrs the epilogue of the second expert GEMM is the return trip of
 * the expert-parallel exchange: each tile's rows leave for their home GPU as soon as the
 * tile is done.  Fuses what the reference's single-GPU kernel does with atomics in
 * _stage2_write_back (datasets/inference/moe/lumen/fused_moe.py:864-888). */
int lumen_b200_moe_grouped_gemm_to_rows(const void* acts, const void* weights,
                                        const void* const* out_row_ptrs,
                                        const void* expert_offsets, const void* expert_counts,
                                        int max_rows, int E, int N, int K, int gated,
                                        int rows_hint, void* stream);

/* out[t,:] = sum_slot topk_weights[t,slot] * y[route_pos[t*k+slot],:], fp32 sum in
 * slot order, bf16 out.  Replaces the atomic write-back of _stage2_write_back
 * (datasets/inference/moe/lumen/fused_moe.py:864-888) with a deterministic gather. */
int lumen_b200_moe_combine(const void* y, const void* route_pos, const void* topk_weights,
                           void* out, int T, int H, int k, void* stream);

/* The whole MoE forward in one call: top-k softmax of `logits` (skipped when the routing
 * is given), stable sort of the routes, row gather, gated expert GEMM, second expert GEMM,
 * weighted combine -- the entry points above launched in that order on `stream`, their
 * intermediates carved out of `scratch` (at least lumen_b200_moe_forward_scratch_bytes(),
 * no initial contents required).  x [T,H] bf16; w13 [E,2I,H] bf16, gate rows first; w2
 * [E,H,I] bf16; out [T,H] bf16.  Give either logits [T,E] fp32 (topk_ids = topk_weights =
 * NULL) or topk_ids [T,k] int32 + topk_weights [T,k] fp32 (logits = NULL), the routing the
 * harness precomputes (scripts/benchmark/backend_moe.py:131-139).  H % 8 == 0, I % 8 == 0.
 * Stands where the reference has one host call for the operator:
 * fused_moe_fp8_blockscale_g1u1 (datasets/inference/moe/lumen/fused_moe.py:1439-1526) and
 * run(8 tensors) of the native system (datasets/inference/moe/ksearch/main.cpp:113-245). */
size_t lumen_b200_moe_forward_scratch_bytes(int T, int H, int I, int E, int k);
int lumen_b200_moe_forward(const void* x, const void* w13, const void* w2, const void* logits,
                           const void* topk_ids, const void* topk_weights, void* out,
                           void* scratch, size_t scratch_bytes, int T, int H, int I, int E, int k,
                           void* stream);

/* out[T,H] (bf16) = lut[q[t,h]] * scale[t, h/128]: fp8 activations (one byte each) with
 * per-128-element fp32 scales to bf16.  lut = 256 floats, the value of every fp8 code
 * (covers e4m3fn and e4m3fnuz).  H % 128 == 0.  Stands in for the activation dequantisation
 * the reference folds into its MFMA loop (datasets/inference/moe/lumen/fused_moe.py:400-443). */
int lumen_b200_moe_dequant_fp8(const void* q, const void* scale, const void* lut, void* out, int T,
                               int H, void* stream);

/* ------------------------------------------------ MoE, fp8 block-scale -- */
/* The reference's own data format: fp8 e4m3 codes with fp32 scales per 1 x 128 block of an
 * activation row and per 128 x 128 block of a weight matrix
 * (scripts/benchmark/backend_moe.py:86-210).  The products run on the tensor cores in fp8
 * (tcgen05.mma.kind::f8f6f4); each 128-wide K block's partial sum is multiplied by
 * act_scale * w_scale while it is added to an fp32 accumulator, as the reference kernel does
 * (datasets/inference/moe/lumen/fused_moe.py:400-443). */

/* scale_t[kb, pos] (fp32, [KB, max_rows]) = scale[token(sorted_token_ids[pos]), kb] for
 * pos < num_valid_ids[0], 1 elsewhere: the activation scales [T, KB] gathered into expert
 * order and stored K-block-major, the layout the reference kernel reads too
 * (datasets/inference/moe/lumen/model.py:259).  The codes themselves are gathered with
 * lumen_b200_moe_permute_rows (a row of H codes = H / 2 two-byte elements). */
int lumen_b200_moe_gather_scales_t(const void* scale, const void* sorted_token_ids,
                                   const void* num_valid_ids, void* out_t, int T, int KB, int max_rows,
                                   void* stream);

/* Per-expert GEMM over fp8 rows in expert order:
 *   acts_q [max_rows, K] codes, act_scale_t [K/128, max_rows] fp32;
 *   weights_q [E, w_rows, K] codes (w_rows = N, or 2N gate rows first for gated != 0),
 *   w_scale [E, w_rows/128, K/128] fp32 (the fc1_scale / fc2_scale layout of the harness).
 *   gated == 0:                     out bf16 [max_rows, N]
 *   gated != 0, quantize_out == 0:  out bf16 [max_rows, N] = silu(gate) * up
 *   gated != 0, quantize_out != 0:  out = fp8 codes [max_rows, N] of silu(gate) * up, re-quantised
 *                                   per row and 128-column block (scale = block maximum / 448,
 *                                   out_scale_t [N/128, max_rows]) for the second GEMM -- the
 *                                   per-row re-quantisation of the reference kernel
 *                                   (datasets/inference/moe/lumen/fused_moe.py:684-788).
 * N % 128 == 0 and K % 128 == 0 (whole scale blocks, as scripts/benchmark/backend_moe.py:77-83
 * requires).  Codes are OCP e4m3; every product is also multiplied by scale_mul, which is how
 * e4m3fnuz inputs are taken: the same bits mean half the value, so pass 0.5 per fnuz operand.
 * rows_hint = expected rows per expert (0 = unknown), picks the token tile. */
int lumen_b200_moe_grouped_gemm_fp8(const void* acts_q, const void* act_scale_t, const void* weights_q,
                                    const void* w_scale, void* out, void* out_scale_t,
                                    const void* expert_offsets, const void* expert_counts, int max_rows,
                                    int E, int N, int K, int gated, int quantize_out, float scale_mul,
                                    int rows_hint, void* stream);

/* ---------------------------------------------- MoE, expert parallel (G GPUs) -- */
/* Tokens and experts are sharded over G GPUs (expert e on GPU e / (E/G)); each GPU sorts
 * its own routes compactly (route_group = 1).  `counts` is the G x E matrix of every
 * GPU's expert_counts (all-gathered by the caller).  The reference has no multi-GPU
 * path; these stand where its single-GPU gather (_input_fetch_async,
 * datasets/inference/moe/lumen/fused_moe.py:246-271) and write-back
 * (_stage2_write_back, :864-888) stand, across GPUs. */

/* From `counts` [G,E] int32 derive, for GPU `rank`:
 *   send_dst_start[E]     row in the owner's grouped buffer where this GPU's rows of expert e start
 *   local_offsets[E/G+1], local_counts[E/G]   grouped layout of this GPU's experts
 *   seg_start[E/G*G+1]    first grouped row of the rows GPU s sent for local expert le (index le*G+s)
 *   seg_home_row[E/G*G]   row of GPU s's compact sorted order those rows came from */
int lumen_b200_moe_ep_plan(const void* counts, int G, int E, int rank, void* send_dst_start,
                           void* local_offsets, void* local_counts, void* seg_start,
                           void* seg_home_row, void* stream);

/* Dispatch: copy x[token] of every compactly sorted route of this GPU straight into the
 * owner GPU's grouped buffer.  peer_buffers (host array of G device pointers, each
 * [capacity_rows, H] bf16, 16-byte aligned, peer-accessible; entry `rank` is this GPU's
 * own buffer).  row_expert[pos] = expert of sorted position pos (the sorted_expert_ids of
 * a route_group = 1 sort).  Rows that would fall outside capacity_rows are dropped and
 * flagged in the device status word.  Callers synchronise the GPUs before reading. */
int lumen_b200_moe_ep_dispatch(const void* x, const void* sorted_token_ids, const void* row_expert,
                               const void* expert_offsets, const void* send_dst_start,
                               const void* num_valid_ids, const void* const* peer_buffers, int G,
                               int T, int H, int E, int max_rows, int capacity_rows, void* stream);

/* Return: copy every grouped output row y[g] back to the GPU it came from, at its row in
 * that GPU's compact sorted order (peer_buffers: G pointers to [home_capacity_rows, H]). */
int lumen_b200_moe_ep_return(const void* y, const void* seg_start, const void* seg_home_row,
                             const void* const* peer_buffers, int G, int El, int H, int max_rows,
                             int home_capacity_rows, void* stream);

/* Synchronisation of the G GPUs over peer memory, without a collective library.
 * peer_signals: host array of G device pointers to each GPU's signal array (int32[64] in
 * peer-accessible memory, zero before first use); epochs: this GPU's private int32[4],
 * zero before first use; slot 0..3 selects an independent barrier.  The kernel announces
 * this GPU's next epoch of the slot to every peer and waits (bounded: a wait that gives up
 * is reported in the device status word) until every peer has announced it too.  All GPUs
 * must issue the same sequence of calls per slot. */
int lumen_b200_moe_ep_barrier(int rank, int G, const void* const* peer_signals, void* epochs,
                              int slot, void* stream);

/* How long (nanoseconds) the two entry points around this comment wait for a peer before
 * they give up, record (35 << 16 | slot << 8 | peer) in the device status word and return;
 * 0 restores the default of 2 s.  A process-wide host setting read at launch.  It bounds the
 * skew between the GPUs' launches: a peer that is later than this (first-call module load, a
 * stalled host thread) makes the forward fail -- the expert-parallel kernels that follow skip
 * their work while the status word is non-zero -- instead of hanging the GPU.  The reference
 * has no multi-GPU path and no counterpart. */
int lumen_b200_moe_ep_set_wait_limit_ns(unsigned long long limit_ns);

/* All-gather of expert_counts[E] by peer stores followed by such a barrier: on completion
 * row s of this GPU's count matrix (peer_count_matrices[rank], int32 [G,E]) holds GPU s's
 * counts.  Input of lumen_b200_moe_ep_plan. */
int lumen_b200_moe_ep_exchange_counts(const void* counts, int E, int rank, int G,
                                      const void* const* peer_count_matrices,
                                      const void* const* peer_signals, void* epochs, int slot,
                                      void* stream);

/* row_ptrs[g] (max_rows device pointers) = home address of grouped output row g: GPU
 * k % G, row seg_home_row[k] + (g - seg_start[k]) for the segment k that holds g; nullptr
 * past the last segment.  Input of lumen_b200_moe_grouped_gemm_to_rows. */
int lumen_b200_moe_ep_row_ptrs(const void* seg_start, const void* seg_home_row,
                               const void* const* peer_buffers, int G, int El, int H, int max_rows,
                               int home_capacity_rows, void* row_ptrs, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LUMEN_B200_H_ */
