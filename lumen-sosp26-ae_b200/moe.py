"""Host side of the fused MoE forward (bf16, in-op router).

Pipeline, all on the current CUDA stream and with no host read of device data, so
the whole forward can be captured in a CUDA graph:

    router logits -> top-k softmax -> stable expert-major sort -> row gather
    -> grouped GEMM (w1|w3, SiLU gate fused) -> grouped GEMM (w2) -> weighted combine

The sorted-route arrays are the ones the reference builds on the host with
_build_sorted_routes (datasets/inference/moe/lumen/model.py:34-98); here they are
produced on the device and are what the grouped GEMMs actually consume.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _cabi

ROUTE_GROUP_SIZE = 32


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("MoE operators need CUDA tensors: there is no CPU path.")
        if t.device != dev:
            raise ValueError(f"all tensors must be on {dev}, got {t.device}.")
        if not t.is_contiguous():
            raise ValueError("MoE operators need contiguous tensors.")
    return dev


def router_logits(x: torch.Tensor, w_router: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """logits[T,E] fp32 = x[T,H] @ w_router[E,H]^T (bf16 inputs)."""
    dev = _need_cuda(x, w_router)
    if x.dtype != torch.bfloat16 or w_router.dtype != torch.bfloat16:
        raise ValueError("router_logits expects bf16 x and w_router.")
    T, H = x.shape
    E = w_router.shape[0]
    if w_router.shape[1] != H:
        raise ValueError(f"w_router must be [E,{H}], got {tuple(w_router.shape)}.")
    if out is None:
        out = torch.empty((T, E), dtype=torch.float32, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_router_logits(
            x.data_ptr(), w_router.data_ptr(), out.data_ptr(), T, H, E, _stream(dev))
    _cabi.check("lumen_b200_moe_router_logits", rc)
    return out


def route_topk(logits: torch.Tensor, topk: int,
               ids_out: torch.Tensor | None = None,
               weights_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(topk_ids int32 [T,k], topk_weights fp32 [T,k]) = topk(sorted) + softmax(topk values)."""
    dev = _need_cuda(logits)
    if logits.dtype != torch.float32 or logits.ndim != 2:
        raise ValueError("route_topk expects fp32 logits [T,E].")
    T, E = logits.shape
    if topk > E:
        raise ValueError(f"topk ({topk}) must be <= experts ({E})")
    ids = ids_out if ids_out is not None else torch.empty((T, topk), dtype=torch.int32, device=dev)
    w = weights_out if weights_out is not None else torch.empty((T, topk), dtype=torch.float32, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_route_topk(
            logits.data_ptr(), ids.data_ptr(), w.data_ptr(), T, E, topk, _stream(dev))
    _cabi.check("lumen_b200_moe_route_topk", rc)
    return ids, w


@dataclass
class SortedRoutes:
    """Device-side result of the route sort; first four fields are the reference's tuple."""

    sorted_token_ids: torch.Tensor
    sorted_weights: torch.Tensor
    sorted_expert_ids: torch.Tensor
    num_valid_ids: torch.Tensor
    expert_offsets: torch.Tensor
    expert_counts: torch.Tensor
    route_pos: torch.Tensor

    def as_reference_tuple(self):
        return (self.sorted_token_ids, self.sorted_weights, self.sorted_expert_ids, self.num_valid_ids)


def max_padded_routes(tokens: int, topk: int, experts: int, group: int = ROUTE_GROUP_SIZE) -> int:
    return tokens * topk + experts * group - topk


def alloc_sorted_routes(tokens: int, topk: int, experts: int, device: torch.device,
                        group: int = ROUTE_GROUP_SIZE) -> SortedRoutes:
    P = max_padded_routes(tokens, topk, experts, group)
    nb = (P + group - 1) // group
    i32 = dict(dtype=torch.int32, device=device)
    return SortedRoutes(
        sorted_token_ids=torch.empty((P,), **i32),
        sorted_weights=torch.empty((P,), dtype=torch.float32, device=device),
        sorted_expert_ids=torch.empty((nb,), **i32),
        num_valid_ids=torch.empty((2,), **i32),
        expert_offsets=torch.empty((experts + 1,), **i32),
        expert_counts=torch.empty((experts,), **i32),
        route_pos=torch.empty((tokens * topk,), **i32),
    )


def build_sorted_routes(*, topk_ids: torch.Tensor, topk_weights: torch.Tensor, experts: int,
                        out: SortedRoutes | None = None, scratch: torch.Tensor | None = None,
                        group: int = ROUTE_GROUP_SIZE) -> SortedRoutes:
    """Device version of _build_sorted_routes (same keyword arguments).  group=32 is the
    reference layout; group=1 packs the experts back to back (expert-parallel dispatch)."""
    dev = _need_cuda(topk_ids, topk_weights)
    if topk_ids.dtype != torch.int32 or topk_weights.dtype != torch.float32:
        raise ValueError("topk_ids must be int32 and topk_weights float32.")
    tokens, topk = topk_ids.shape
    if tuple(topk_weights.shape) != (tokens, topk):
        raise ValueError("topk_weights shape mismatch.")
    lib = _cabi.load()
    need = int(lib.lumen_b200_moe_sort_scratch_bytes(tokens, experts, topk))
    if scratch is None:
        scratch = torch.empty((max(need, 4),), dtype=torch.uint8, device=dev)
    if out is None:
        out = alloc_sorted_routes(tokens, topk, experts, dev, group)
    with _cabi.on_device(dev):
        rc = lib.lumen_b200_moe_sort_routes(
            topk_ids.data_ptr(), topk_weights.data_ptr(), out.sorted_token_ids.data_ptr(),
            out.sorted_weights.data_ptr(), out.sorted_expert_ids.data_ptr(),
            out.num_valid_ids.data_ptr(), out.expert_offsets.data_ptr(),
            out.expert_counts.data_ptr(), out.route_pos.data_ptr(), scratch.data_ptr(),
            scratch.numel(), tokens, experts, topk, int(group), _stream(dev))
    _cabi.check("lumen_b200_moe_sort_routes", rc)
    return out


def permute_rows(x: torch.Tensor, routes: SortedRoutes, out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _need_cuda(x)
    T, H = x.shape
    P = routes.sorted_token_ids.numel()
    if out is None:
        out = torch.empty((P, H), dtype=torch.bfloat16, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_permute_rows(
            x.data_ptr(), routes.sorted_token_ids.data_ptr(), routes.num_valid_ids.data_ptr(),
            out.data_ptr(), T, H, P, _stream(dev))
    _cabi.check("lumen_b200_moe_permute_rows", rc)
    return out


_fp8_luts: dict = {}


def dequant_fp8_rows(q: torch.Tensor, scale: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [T,H] = value(q[t,h]) * scale[t, h // 128] for fp8 q (any torch float8 dtype)."""
    dev = _need_cuda(q, scale)
    if q.element_size() != 1 or not q.dtype.is_floating_point:
        raise ValueError(f"q must be a float8 tensor, got {q.dtype}")
    T, H = q.shape
    if H % 128 != 0 or tuple(scale.shape) != (T, H // 128) or scale.dtype != torch.float32:
        raise ValueError("scale must be fp32 [T, H/128] and H a multiple of 128")
    key = (dev.index, q.dtype)
    lut = _fp8_luts.get(key)
    if lut is None:  # the float value of each of the 256 codes of this fp8 flavour
        lut = torch.arange(256, dtype=torch.uint8, device=dev).view(q.dtype).to(torch.float32)
        lut = torch.nan_to_num(lut, nan=0.0, posinf=0.0, neginf=0.0).contiguous()
        _fp8_luts[key] = lut
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_dequant_fp8(q.data_ptr(), scale.data_ptr(), lut.data_ptr(),
                                                     out.data_ptr(), T, H, _stream(dev))
    _cabi.check("lumen_b200_moe_dequant_fp8", rc)
    return out


_row_counts: dict = {}


def _row_count(dev: torch.device, n: int) -> torch.Tensor:
    """Device-resident int32 [n, 0] (the num_valid_ids form the row gather reads), cached."""
    key = (dev.index, n)
    t = _row_counts.get(key)
    if t is None:
        if len(_row_counts) > 4096:
            _row_counts.clear()
        t = torch.tensor([n, 0], dtype=torch.int32, device=dev)
        _row_counts[key] = t
    return t


def gather_rows(rows: torch.Tensor, index: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[i,:] = rows[index[i],:] (an index >= len(rows) gives a zero row); bf16 rows, int32 index."""
    dev = _need_cuda(rows, index)
    if index.dtype != torch.int32 or index.ndim != 1:
        raise ValueError("index must be a 1-D int32 tensor")
    R, H = rows.shape
    n = index.numel()
    if out is None:
        out = torch.empty((n, H), dtype=torch.bfloat16, device=dev)
    if n == 0:
        return out
    count = _row_count(dev, n)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_permute_rows(
            rows.data_ptr(), index.data_ptr(), count.data_ptr(), out.data_ptr(), R, H, n, _stream(dev))
    _cabi.check("lumen_b200_moe_permute_rows", rc)
    return out


def grouped_gemm(acts: torch.Tensor, weights: torch.Tensor, routes: SortedRoutes, *, gated: bool,
                 rows_hint: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-expert GEMM over rows in expert order; `weights` is [E, (2)N, K]."""
    dev = _need_cuda(acts, weights)
    P, K = acts.shape
    E, w_rows, K2 = weights.shape
    if K2 != K:
        raise ValueError(f"weights K ({K2}) must equal activations K ({K}).")
    N = w_rows // 2 if gated else w_rows
    if out is None:
        out = torch.empty((P, N), dtype=torch.bfloat16, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_grouped_gemm(
            acts.data_ptr(), weights.data_ptr(), out.data_ptr(), routes.expert_offsets.data_ptr(),
            routes.expert_counts.data_ptr(), P, E, N, K, 1 if gated else 0, int(rows_hint),
            _stream(dev))
    _cabi.check("lumen_b200_moe_grouped_gemm", rc)
    return out


def grouped_gemm_to_rows(acts: torch.Tensor, weights: torch.Tensor, row_ptrs: torch.Tensor, routes, *,
                         gated: bool, rows_hint: int) -> None:
    """grouped_gemm whose output row r is written at the address row_ptrs[r] (int64 device
    tensor of addresses, 0 = skip); the addresses may lie in a peer GPU's memory."""
    dev = _need_cuda(acts, weights, row_ptrs)
    if row_ptrs.dtype != torch.int64:
        raise ValueError("row_ptrs must be an int64 tensor of device addresses")
    P, K = acts.shape
    E, w_rows, K2 = weights.shape
    if K2 != K:
        raise ValueError(f"weights K ({K2}) must equal activations K ({K}).")
    if row_ptrs.numel() < P:
        raise ValueError("row_ptrs must have one entry per activation row")
    N = w_rows // 2 if gated else w_rows
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_grouped_gemm_to_rows(
            acts.data_ptr(), weights.data_ptr(), row_ptrs.data_ptr(), routes.expert_offsets.data_ptr(),
            routes.expert_counts.data_ptr(), P, E, N, K, 1 if gated else 0, int(rows_hint), _stream(dev))
    _cabi.check("lumen_b200_moe_grouped_gemm_to_rows", rc)


def combine(y: torch.Tensor, routes: SortedRoutes, topk_weights: torch.Tensor, tokens: int,
            out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _need_cuda(y, topk_weights)
    H = y.shape[1]
    k = topk_weights.shape[1]
    if out is None:
        out = torch.empty((tokens, H), dtype=torch.bfloat16, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_combine(
            y.data_ptr(), routes.route_pos.data_ptr(), topk_weights.data_ptr(), out.data_ptr(),
            tokens, H, k, _stream(dev))
    _cabi.check("lumen_b200_moe_combine", rc)
    return out


def moe_forward(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, *, topk: int,
                logits: torch.Tensor | None = None, topk_ids: torch.Tensor | None = None,
                topk_weights: torch.Tensor | None = None, out: torch.Tensor | None = None,
                scratch: torch.Tensor | None = None) -> torch.Tensor:
    """The whole forward through the single C entry point lumen_b200_moe_forward: give either
    `logits` [T,E] fp32 (the top-k softmax runs first) or precomputed `topk_ids` / `topk_weights`.
    `scratch` (uint8, at least moe_forward_scratch_bytes(...)) holds every intermediate."""
    dev = _need_cuda(x, w13, w2)
    T, H = x.shape
    E, two_i, H2 = w13.shape
    inter = two_i // 2
    if H2 != H or tuple(w2.shape) != (E, H, inter):
        raise ValueError("w13 must be [E, 2I, H] and w2 [E, H, I].")
    if (logits is None) == (topk_ids is None) or (topk_ids is None) != (topk_weights is None):
        raise ValueError("give exactly one of logits or (topk_ids, topk_weights)")
    if logits is not None and (logits.dtype != torch.float32 or tuple(logits.shape) != (T, E)):
        raise ValueError("logits must be float32 [T, E].")
    if topk_ids is not None and (topk_ids.dtype != torch.int32 or topk_weights.dtype != torch.float32 or
                                 tuple(topk_ids.shape) != (T, topk) or tuple(topk_weights.shape) != (T, topk)):
        raise ValueError("topk_ids must be int32 [T, k] and topk_weights float32 [T, k].")
    lib = _cabi.load()
    need = moe_forward_scratch_bytes(T, H, inter, E, topk)
    if scratch is None:
        scratch = torch.empty((need,), dtype=torch.uint8, device=dev)
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    ptr = lambda t: 0 if t is None else t.data_ptr()  # noqa: E731
    with _cabi.on_device(dev):
        rc = lib.lumen_b200_moe_forward(
            x.data_ptr(), w13.data_ptr(), w2.data_ptr(), ptr(logits), ptr(topk_ids), ptr(topk_weights),
            out.data_ptr(), scratch.data_ptr(), scratch.numel(), T, H, inter, E, int(topk), _stream(dev))
    _cabi.check("lumen_b200_moe_forward", rc)
    return out


def moe_forward_scratch_bytes(tokens: int, hidden: int, inter: int, experts: int, topk: int) -> int:
    need = int(_cabi.load().lumen_b200_moe_forward_scratch_bytes(tokens, hidden, inter, experts, topk))
    if need == 0:
        raise ValueError("shape outside what lumen_b200_moe_forward covers")
    return need


class FusedMoE:
    """Pre-allocated buffers + the launch sequence of one MoE forward shape.

    forward_routed(x, topk_ids, topk_weights) takes precomputed routing (the reference
    harness contract); forward(x, logits=...) / forward(x, w_router=...) runs the in-op
    router first.  w13 is [E, 2I, H] (gate rows first, up rows second: the w1_q layout of
    scripts/benchmark/backend_moe.py:162-171), w2 is [E, H, I].
    """

    def __init__(self, *, tokens: int, hidden: int, inter: int, experts: int, topk: int,
                 device: torch.device):
        self.T, self.H, self.I, self.E, self.k = tokens, hidden, inter, experts, topk
        self.device = device
        P = max_padded_routes(tokens, topk, experts)
        self.routes = alloc_sorted_routes(tokens, topk, experts, device)
        need = int(_cabi.load().lumen_b200_moe_sort_scratch_bytes(tokens, experts, topk))
        self.scratch = torch.empty((max(need, 4),), dtype=torch.uint8, device=device)
        self.logits = torch.empty((tokens, experts), dtype=torch.float32, device=device)
        self.topk_ids = torch.empty((tokens, topk), dtype=torch.int32, device=device)
        self.topk_weights = torch.empty((tokens, topk), dtype=torch.float32, device=device)
        self.xs = torch.empty((P, hidden), dtype=torch.bfloat16, device=device)
        self.h = torch.empty((P, inter), dtype=torch.bfloat16, device=device)
        self.y = torch.empty((P, hidden), dtype=torch.bfloat16, device=device)
        self.out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=device)
        self.rows_hint = max(1, (tokens * topk + experts - 1) // experts)

    def forward_routed(self, x, topk_ids, topk_weights, w13, w2):
        build_sorted_routes(topk_ids=topk_ids, topk_weights=topk_weights, experts=self.E,
                            out=self.routes, scratch=self.scratch)
        permute_rows(x, self.routes, out=self.xs)
        grouped_gemm(self.xs, w13, self.routes, gated=True, rows_hint=self.rows_hint, out=self.h)
        grouped_gemm(self.h, w2, self.routes, gated=False, rows_hint=self.rows_hint, out=self.y)
        return combine(self.y, self.routes, topk_weights, self.T, out=self.out)

    def forward(self, x, w13, w2, *, w_router=None, logits=None):
        if (w_router is None) == (logits is None):
            raise ValueError("give exactly one of w_router (in-op router) or logits")
        if w_router is not None:
            logits = router_logits(x, w_router, out=self.logits)
        route_topk(logits, self.k, ids_out=self.topk_ids, weights_out=self.topk_weights)
        return self.forward_routed(x, self.topk_ids, self.topk_weights, w13, w2)

    def stage_times(self, x, w13, w2, *, w_router=None, logits=None, repeats: int = 5) -> dict:
        """Median device time (ms) of each launch group of one forward, from CUDA events
        on the current stream.  Measurement helper; not used by forward()."""
        import statistics

        def timed(fn):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            return (e0, e1)

        samples: dict[str, list] = {}
        for _ in range(repeats):
            ev = {}
            if w_router is not None:
                ev["router_logits"] = timed(lambda: router_logits(x, w_router, out=self.logits))
                lg = self.logits
            else:
                lg = logits
            ev["topk_softmax"] = timed(lambda: route_topk(lg, self.k, ids_out=self.topk_ids,
                                                          weights_out=self.topk_weights))
            ev["sort_routes"] = timed(lambda: build_sorted_routes(
                topk_ids=self.topk_ids, topk_weights=self.topk_weights, experts=self.E,
                out=self.routes, scratch=self.scratch))
            ev["permute_rows"] = timed(lambda: permute_rows(x, self.routes, out=self.xs))
            ev["gemm_w13_silu"] = timed(lambda: grouped_gemm(self.xs, w13, self.routes, gated=True,
                                                             rows_hint=self.rows_hint, out=self.h))
            ev["gemm_w2"] = timed(lambda: grouped_gemm(self.h, w2, self.routes, gated=False,
                                                       rows_hint=self.rows_hint, out=self.y))
            ev["combine"] = timed(lambda: combine(self.y, self.routes, self.topk_weights, self.T,
                                                  out=self.out))
            torch.cuda.synchronize()
            for name, (e0, e1) in ev.items():
                samples.setdefault(name, []).append(e0.elapsed_time(e1))
        return {name: statistics.median(v) for name, v in samples.items()}


# --------------------------------------------------------------------------- fp8 block scale
FP8_BLOCK = 128


def fp8_code_factor(dtype: torch.dtype) -> float:
    """What one unit of an fp8 code of `dtype` is worth relative to the same bits read as OCP
    e4m3 (the tensor cores' format): 1 for float8_e4m3fn, 0.5 for float8_e4m3fnuz (exponent
    bias 8 instead of 7; every finite code of one is a finite code of the other except the
    fnuz values +-240, bit patterns 0x7F / 0xFF, which e4m3fn reads as NaN)."""
    if dtype == torch.float8_e4m3fn:
        return 1.0
    if dtype == getattr(torch, "float8_e4m3fnuz", None):
        return 0.5
    raise ValueError(f"fp8 MoE takes float8_e4m3fn or float8_e4m3fnuz codes, got {dtype}")


def gather_scales_t(scale: torch.Tensor, routes: SortedRoutes, out: torch.Tensor | None = None) -> torch.Tensor:
    """[T, KB] per-token block scales -> [KB, P] in expert order (1 for pad rows)."""
    dev = _need_cuda(scale)
    if scale.dtype != torch.float32 or scale.ndim != 2:
        raise ValueError("scale must be a float32 [T, KB] tensor")
    T, KB = scale.shape
    P = routes.sorted_token_ids.numel()
    if out is None:
        out = torch.empty((KB, P), dtype=torch.float32, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_gather_scales_t(
            scale.data_ptr(), routes.sorted_token_ids.data_ptr(), routes.num_valid_ids.data_ptr(),
            out.data_ptr(), T, KB, P, _stream(dev))
    _cabi.check("lumen_b200_moe_gather_scales_t", rc)
    return out


def grouped_gemm_fp8(acts_q: torch.Tensor, act_scale_t: torch.Tensor, weights_q: torch.Tensor,
                     w_scale: torch.Tensor, routes, *, gated: bool, quantize_out: bool = False,
                     scale_mul: float = 1.0, rows_hint: int = 0, out: torch.Tensor | None = None,
                     out_scale_t: torch.Tensor | None = None):
    """Per-expert fp8 block-scale GEMM (see lumen_b200_moe_grouped_gemm_fp8).  Returns `out`, or
    (`out` codes as uint8, `out_scale_t`) when quantize_out."""
    dev = _need_cuda(acts_q, act_scale_t, weights_q, w_scale)
    if acts_q.element_size() != 1 or weights_q.element_size() != 1:
        raise ValueError("acts_q and weights_q hold one-byte fp8 codes")
    P, K = acts_q.shape
    E, w_rows, K2 = weights_q.shape
    N = w_rows // 2 if gated else w_rows
    if K2 != K or K % FP8_BLOCK or N % FP8_BLOCK:
        raise ValueError(f"K ({K}, {K2}) and N ({N}) must agree and be multiples of {FP8_BLOCK}")
    if tuple(act_scale_t.shape) != (K // FP8_BLOCK, P) or act_scale_t.dtype != torch.float32:
        raise ValueError(f"act_scale_t must be float32 [{K // FP8_BLOCK}, {P}]")
    if w_scale.dtype != torch.float32 or w_scale.numel() != E * (w_rows // FP8_BLOCK) * (K // FP8_BLOCK):
        raise ValueError("w_scale must be float32 [E, w_rows/128, K/128]")
    if out is None:
        out = torch.empty((P, N), dtype=torch.uint8 if quantize_out else torch.bfloat16, device=dev)
    if quantize_out and out_scale_t is None:
        out_scale_t = torch.ones((N // FP8_BLOCK, P), dtype=torch.float32, device=dev)
    with _cabi.on_device(dev):
        rc = _cabi.load().lumen_b200_moe_grouped_gemm_fp8(
            acts_q.data_ptr(), act_scale_t.data_ptr(), weights_q.data_ptr(), w_scale.data_ptr(), out.data_ptr(),
            out_scale_t.data_ptr() if quantize_out else None, routes.expert_offsets.data_ptr(),
            routes.expert_counts.data_ptr(), P, E, N, K, 1 if gated else 0, 1 if quantize_out else 0,
            float(scale_mul), int(rows_hint), _stream(dev))
    _cabi.check("lumen_b200_moe_grouped_gemm_fp8", rc)
    return (out, out_scale_t) if quantize_out else out


class FusedMoEFp8:
    """The MoE forward on fp8 codes and block scales, the reference harness' own format
    (scripts/benchmark/backend_moe.py:86-210): sort -> gather codes and scales -> gated expert
    GEMM in fp8 with the intermediate re-quantised per row and 128-column block -> second expert
    GEMM in fp8 -> weighted combine.  No tensor is dequantised to bf16 on the way in."""

    def __init__(self, *, tokens: int, hidden: int, inter: int, experts: int, topk: int, device: torch.device):
        if hidden % FP8_BLOCK or inter % FP8_BLOCK:
            raise ValueError(f"hidden ({hidden}) and inter ({inter}) must be multiples of {FP8_BLOCK}")
        self.T, self.H, self.I, self.E, self.k = tokens, hidden, inter, experts, topk
        self.device = device
        P = max_padded_routes(tokens, topk, experts)
        self.routes = alloc_sorted_routes(tokens, topk, experts, device)
        need = int(_cabi.load().lumen_b200_moe_sort_scratch_bytes(tokens, experts, topk))
        self.scratch = torch.empty((max(need, 4),), dtype=torch.uint8, device=device)
        self.xs_q = torch.zeros((P, hidden), dtype=torch.uint8, device=device)
        self.xs_scale_t = torch.ones((hidden // FP8_BLOCK, P), dtype=torch.float32, device=device)
        self.h_q = torch.zeros((P, inter), dtype=torch.uint8, device=device)
        self.h_scale_t = torch.ones((inter // FP8_BLOCK, P), dtype=torch.float32, device=device)
        self.y = torch.empty((P, hidden), dtype=torch.bfloat16, device=device)
        self.out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=device)
        self.rows_hint = max(1, (tokens * topk + experts - 1) // experts)

    def forward_routed(self, x_q, x_scale, topk_ids, topk_weights, w13_q, w13_scale, w2_q, w2_scale):
        fx, f1, f2 = fp8_code_factor(x_q.dtype), fp8_code_factor(w13_q.dtype), fp8_code_factor(w2_q.dtype)
        build_sorted_routes(topk_ids=topk_ids, topk_weights=topk_weights, experts=self.E,
                            out=self.routes, scratch=self.scratch)
        # a row of H one-byte codes moves as H / 2 two-byte elements
        permute_rows(x_q.view(torch.uint8).view(torch.bfloat16), self.routes, out=self.xs_q.view(torch.bfloat16))
        gather_scales_t(x_scale, self.routes, out=self.xs_scale_t)
        grouped_gemm_fp8(self.xs_q, self.xs_scale_t, w13_q.view(torch.uint8), w13_scale, self.routes, gated=True,
                         quantize_out=True, scale_mul=fx * f1, rows_hint=self.rows_hint, out=self.h_q,
                         out_scale_t=self.h_scale_t)
        grouped_gemm_fp8(self.h_q, self.h_scale_t, w2_q.view(torch.uint8), w2_scale, self.routes, gated=False,
                         scale_mul=f2, rows_hint=self.rows_hint, out=self.y)
        return combine(self.y, self.routes, topk_weights, self.T, out=self.out)
