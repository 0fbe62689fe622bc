"""Oracle for the fused MoE forward (bf16, SiLU-gated experts, top-k softmax router).

Restates, for unit scales and bf16 storage,
  * routing: scripts/benchmark/backend_moe.py:131-139 (topk sorted, softmax of the k values);
  * the token permutation: `_build_sorted_routes`
    (datasets/inference/moe/lumen/model.py:34-98), here in numpy integer arithmetic;
  * expert compute and combine: `_moe_reference` (scripts/benchmark/backend_moe.py:469-504),
    i.e. per expert  silu(x W1^T) * (x W3^T) W2^T  in fp32, weighted index_add, bf16 out,
    with w1_q = [gate rows; up rows] stacked along dim 1.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

ROUTE_GROUP_SIZE = 32  # datasets/inference/moe/lumen/model.py:14


def router_logits(x: torch.Tensor, w_router: torch.Tensor) -> torch.Tensor:
    """fp32 logits = x.float() @ Wr.float().T"""
    return x.to(torch.float32) @ w_router.to(torch.float32).transpose(0, 1)


def route_topk(logits: torch.Tensor, topk: int):
    """ids int32 [T,k] (descending value, ties to the lower index), weights fp32 [T,k]."""
    order = torch.sort(logits.to(torch.float32), dim=-1, descending=True, stable=True)
    ids = order.indices[:, :topk].to(torch.int32).contiguous()
    vals = order.values[:, :topk]
    weights = torch.softmax(vals, dim=-1).to(torch.float32).contiguous()
    return ids, weights


def min_topk_gap(logits: torch.Tensor, topk: int) -> float:
    """Smallest gap between neighbouring values among the top (k+1) of any row: the
    margin by which a perturbation of the logits could change ids or their order."""
    vals = torch.sort(logits.to(torch.float32), dim=-1, descending=True).values
    upto = min(topk + 1, vals.shape[1])
    gaps = vals[:, : upto - 1] - vals[:, 1:upto]
    return float(gaps.min())


def build_sorted_routes(topk_ids: np.ndarray, topk_weights: np.ndarray, experts: int,
                        group: int = ROUTE_GROUP_SIZE):
    """numpy restatement of _build_sorted_routes (`group` = its ROUTE_GROUP_SIZE; 1 gives
    the compact layout without padding between experts).  Returns
    (sorted_token_ids i32 [P], sorted_weights f32 [P], sorted_expert_ids i32 [NB],
     num_valid_ids i32 [2], expert_offsets i32 [E+1], expert_counts i32 [E], route_pos i32 [T*k]);
    the first four are the reference's tuple, the last three are the derived tables the
    device pipeline also emits."""
    topk_ids = np.asarray(topk_ids, dtype=np.int32)
    topk_weights = np.asarray(topk_weights, dtype=np.float32)
    tokens, topk = topk_ids.shape
    P = tokens * topk + experts * group - topk
    NB = (P + group - 1) // group
    sorted_token_ids = np.full((P,), (topk << 24) | tokens, dtype=np.int32)
    sorted_weights = np.zeros((P,), dtype=np.float32)
    sorted_expert_ids = np.full((NB,), -1, dtype=np.int32)
    expert_offsets = np.zeros((experts + 1,), dtype=np.int32)
    expert_counts = np.zeros((experts,), dtype=np.int32)
    route_pos = np.full((tokens * topk,), -1, dtype=np.int32)
    begin = 0
    blk = 0
    for e in range(experts):
        expert_offsets[e] = begin
        tok, slot = np.nonzero(topk_ids == e)  # row-major: token ascending, slot ascending
        n = int(tok.size)
        expert_counts[e] = n
        if n == 0:
            continue
        sorted_token_ids[begin:begin + n] = (slot.astype(np.int32) << 24) | tok.astype(np.int32)
        sorted_weights[begin:begin + n] = topk_weights[tok, slot]
        route_pos[tok * topk + slot] = begin + np.arange(n, dtype=np.int32)
        nblk = (n + group - 1) // group
        sorted_expert_ids[blk:blk + nblk] = e
        begin += nblk * group
        blk += nblk
    expert_offsets[experts] = begin
    num_valid_ids = np.array([begin, tokens], dtype=np.int32)
    return (sorted_token_ids, sorted_weights, sorted_expert_ids, num_valid_ids,
            expert_offsets, expert_counts, route_pos)


def moe_reference(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, topk_ids: torch.Tensor,
                  topk_weights: torch.Tensor) -> torch.Tensor:
    """x [T,H] bf16, w13 [E,2I,H] bf16 (gate rows then up rows), w2 [E,H,I] bf16 -> bf16 [T,H]."""
    T, H = x.shape
    E, two_i, _ = w13.shape
    inter = two_i // 2
    xf = x.to(torch.float32)
    out = torch.zeros((T, H), dtype=torch.float32)
    for e in range(E):
        tok, slot = torch.nonzero(topk_ids == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        w1 = w13[e].to(torch.float32)
        stage1 = xf[tok] @ w1.transpose(0, 1)
        gate, up = stage1.split(inter, dim=-1)
        expert_out = (F.silu(gate) * up) @ w2[e].to(torch.float32).transpose(0, 1)
        out.index_add_(0, tok, expert_out * topk_weights[tok, slot].unsqueeze(1))
    return out.to(torch.bfloat16)


def moe_inputs(tokens: int, hidden: int, inter: int, experts: int, seed: int, *,
               with_router: bool):
    """Seeded stand-in inputs with the configurations' distributions: x ~ N(0,1);
    weights ~ N(0, 0.02) from seed+17 (the reference's weight seed offset,
    scripts/benchmark/backend_moe.py:160); router matrix ~ N(0, 0.02) or logits ~ N(0,1)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn((tokens, hidden), generator=g, dtype=torch.float32).to(torch.bfloat16)
    logits = None if with_router else torch.randn((tokens, experts), generator=g, dtype=torch.float32)
    gw = torch.Generator(device="cpu")
    gw.manual_seed(seed + 17)
    w_router = None
    if with_router:
        w_router = (torch.randn((experts, hidden), generator=gw, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    w1 = torch.randn((experts, inter, hidden), generator=gw, dtype=torch.float32) * 0.02
    w3 = torch.randn((experts, inter, hidden), generator=gw, dtype=torch.float32) * 0.02
    w2 = (torch.randn((experts, hidden, inter), generator=gw, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    w13 = torch.cat([w1, w3], dim=1).to(torch.bfloat16)
    return dict(x=x, logits=logits, w_router=w_router, w13=w13, w2=w2)


BLOCK = 128  # scale block edge (scripts/benchmark/backend_moe.py:19-20)


def block_dequant(codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """codes [rows, cols] (any dtype, read by value) times scale [(rows/128) * (cols/128)] ->
    fp32: `_dequantize_weight` (scripts/benchmark/backend_moe.py:507-525)."""
    rows, cols = codes.shape
    s = scale.to(torch.float32).reshape(rows // BLOCK, 1, cols // BLOCK, 1)
    return (codes.to(torch.float32).reshape(rows // BLOCK, BLOCK, cols // BLOCK, BLOCK) * s).reshape(rows, cols)


def quantize_rows_e4m3(h: torch.Tensor):
    """Per row and 128-column block: scale = max|h| / 448 (1 for an all-zero block), codes =
    e4m3fn(h / scale).  Returns (dequantised h, scales [rows, cols/128]).  Models the per-row
    re-quantisation of the intermediate (datasets/inference/moe/lumen/fused_moe.py:684-788) with
    the OCP e4m3 range of the target hardware."""
    rows, cols = h.shape
    hb = h.to(torch.float32).reshape(rows, cols // BLOCK, BLOCK)
    amax = hb.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (hb / scale).to(torch.float8_e4m3fn).to(torch.float32)
    return (q * scale).reshape(rows, cols), scale.squeeze(-1)


def moe_reference_blockscale(x_q, x_scale, w13_q, w13_scale, w2_q, w2_scale, topk_ids, topk_weights, *,
                             quantize_h: bool = False) -> torch.Tensor:
    """`_moe_reference` (scripts/benchmark/backend_moe.py:469-504) with its block scales: x_q [T,H]
    and the weights are fp8 (or bf16) codes read by value, x_scale [T,H/128], w13_scale
    [E,(2I/128)*(H/128)], w2_scale [E,(H/128)*(I/128)].  fp32 throughout, bf16 out.
    quantize_h=True re-quantises the intermediate like the fp8 kernels do."""
    T, H = x_q.shape
    E, two_i, _ = w13_q.shape
    inter = two_i // 2
    xf = (x_q.to(torch.float32).reshape(T, H // BLOCK, BLOCK) * x_scale.to(torch.float32).unsqueeze(-1)).reshape(T, H)
    out = torch.zeros((T, H), dtype=torch.float32)
    for e in range(E):
        tok, slot = torch.nonzero(topk_ids == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        stage1 = xf[tok] @ block_dequant(w13_q[e], w13_scale[e]).transpose(0, 1)
        gate, up = stage1.split(inter, dim=-1)
        h = F.silu(gate) * up
        if quantize_h:
            h, _ = quantize_rows_e4m3(h)
        expert_out = h @ block_dequant(w2_q[e], w2_scale[e]).transpose(0, 1)
        out.index_add_(0, tok, expert_out * topk_weights[tok, slot].unsqueeze(1))
    return out.to(torch.bfloat16)


def moe_fp8_inputs(tokens: int, hidden: int, inter: int, experts: int, topk: int, seed: int,
                   dtype=torch.float8_e4m3fn, w_scale: float = 1e-2):
    """Seeded stand-ins with the distributions of the harness' fp8 mode
    (scripts/benchmark/backend_moe.py:86-210): x = randn + 0.1 and weights = randn * 8 cast to fp8,
    positive block scales around 0.1 (activations) and `w_scale` (weights; the harness uses 0.01,
    the parity tests a larger value so that outputs are of order 1), routing from N(0,1) scores."""
    g = torch.Generator().manual_seed(seed)
    x_q = (torch.randn((tokens, hidden), generator=g) + 0.1).to(dtype)
    x_scale = (torch.randn((tokens, hidden // BLOCK), generator=g) * 2e-2 + 1e-1).clamp_min(1e-8)
    ids, weights = route_topk(torch.randn((tokens, experts), generator=g), topk)
    gw = torch.Generator().manual_seed(seed + 17)
    w13_q = (torch.randn((experts, 2 * inter, hidden), generator=gw) * 8.0).to(dtype)
    w2_q = (torch.randn((experts, hidden, inter), generator=gw) * 8.0).to(dtype)
    w13_scale = (torch.randn((experts, (2 * inter // BLOCK) * (hidden // BLOCK)), generator=gw) * 0.2 * w_scale + w_scale).clamp_min(1e-8)
    w2_scale = (torch.randn((experts, (hidden // BLOCK) * (inter // BLOCK)), generator=gw) * 0.2 * w_scale + w_scale).clamp_min(1e-8)
    return dict(x_q=x_q, x_scale=x_scale, topk_ids=ids, topk_weights=weights, w13_q=w13_q, w13_scale=w13_scale,
                w2_q=w2_q, w2_scale=w2_scale)
