"""How each operator is split over the GPUs of one node (one process per GPU).

GEMM and attention shard into independent pieces: no collective on the data path.
  * GEMM  C = A * B^T : rank g owns rows [g*N/G, (g+1)*N/G) of B and produces that column
    slice of C; A is replicated.
  * attention          : the B * Hkv (batch, KV-head) units are dealt out in contiguous
    runs; a KV head always travels with its Hq/Hkv query heads.
The MoE is expert-parallel and has one real exchange step each way (moe_ep.py).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def even_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-even split of range(total): the first total % world ranks get one more."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gemm_column_range(n: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Rows of B (= columns of C) owned by `rank`; boundaries are multiples of `align`
    so that every shard keeps 16-byte aligned rows and vector stores."""
    if n % align != 0:
        return even_range(n, world, rank)
    lo, hi = even_range(n // align, world, rank)
    return lo * align, hi * align


class ColumnShardedGemm:
    """C[:, n0:n1] = A * B[n0:n1, :]^T on this rank; the shard of B is held contiguously."""

    def __init__(self, b_full_or_shard: torch.Tensor, n_total: int, world: int, rank: int,
                 *, is_shard: bool = False):
        from .gemm import gemm_pipeline_transposed_b

        self._gemm = gemm_pipeline_transposed_b
        self.n0, self.n1 = gemm_column_range(n_total, world, rank)
        if is_shard:
            if b_full_or_shard.shape[0] != self.n1 - self.n0:
                raise ValueError("shard has the wrong number of rows")
            self.b = b_full_or_shard.contiguous()
        else:
            self.b = b_full_or_shard[self.n0:self.n1].contiguous()

    def forward(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return self._gemm(a, self.b, out)

    __call__ = forward


@dataclass(frozen=True)
class AttentionShard:
    """Half-open ranges of the batch and of the KV heads that one rank computes."""

    b0: int
    b1: int
    hk0: int
    hk1: int

    def units(self) -> int:
        return (self.b1 - self.b0) * (self.hk1 - self.hk0)


def attention_shard(batch: int, kv_heads: int, world: int, rank: int) -> AttentionShard:
    """Deal the batch * kv_heads units out contiguously.  With world <= batch (and batch
    divisible) whole batch entries go to a rank; otherwise each batch entry's KV heads are
    split over world / batch ranks.  Every rank's shard is a rectangle, so it can be held
    as one contiguous [B_l, S, H_l, D] tensor."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    if world <= batch:
        if batch % world != 0:
            raise ValueError(f"batch {batch} does not split over {world} ranks")
        per = batch // world
        return AttentionShard(rank * per, (rank + 1) * per, 0, kv_heads)
    if world % batch != 0:
        raise ValueError(f"{world} ranks do not split into {batch} batch entries")
    per_batch = world // batch
    if kv_heads % per_batch != 0:
        raise ValueError(f"{kv_heads} KV heads do not split over {per_batch} ranks per batch entry")
    hpr = kv_heads // per_batch
    b = rank // per_batch
    j = rank % per_batch
    return AttentionShard(b, b + 1, j * hpr, (j + 1) * hpr)


def slice_attention_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, shard: AttentionShard):
    """Contiguous copies of this rank's part of q [B,S,Hq,D], k, v [B,S,Hkv,D]."""
    groups = q.shape[2] // k.shape[2]
    qs = q[shard.b0:shard.b1, :, shard.hk0 * groups:shard.hk1 * groups].contiguous()
    ks = k[shard.b0:shard.b1, :, shard.hk0:shard.hk1].contiguous()
    vs = v[shard.b0:shard.b1, :, shard.hk0:shard.hk1].contiguous()
    return qs, ks, vs
