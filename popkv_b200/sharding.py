"""KV-head sharding of the retrieval path across the GPUs of one node.

The reference is single-GPU.  KV heads are independent through scoring,
selection and attention (GQA groups never cross KV heads), so rank r of N owns
KV heads [r*KVH/N, (r+1)*KVH/N) -- their K/V cache and bit-plane metadata --
and the query heads that read them, [r*QH/N, (r+1)*QH/N).  Each rank runs the
whole decode step on its heads; one all-gather of the per-head attention
outputs per layer gives every rank the full [B, QH, D] input of the replicated
output projection.  The all-gather is the only collective on the path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_start: int
    kv_end: int
    q_start: int
    q_end: int

    @property
    def kv_slice(self) -> slice:
        return slice(self.kv_start, self.kv_end)

    @property
    def q_slice(self) -> slice:
        return slice(self.q_start, self.q_end)

    @property
    def kv_heads(self) -> int:
        return self.kv_end - self.kv_start

    @property
    def q_heads(self) -> int:
        return self.q_end - self.q_start

    def local_head_to_kv(self, device=None) -> torch.Tensor:
        group = self.q_heads // self.kv_heads
        return torch.arange(self.q_heads, device=device, dtype=torch.int64) // group


def head_shard(q_heads: int, kv_heads: int, world: int, rank: int) -> HeadShard:
    """The heads rank ``rank`` of ``world`` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads cannot be split evenly over {world} ranks")
    if q_heads % kv_heads:
        raise ValueError("query heads must be a multiple of KV heads")
    kv_local = kv_heads // world
    q_local = q_heads // world
    return HeadShard(rank, world, rank * kv_local, (rank + 1) * kv_local,
                     rank * q_local, (rank + 1) * q_local)


def gather_heads(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-rank head outputs [B, QH/N, D] into [B, QH, D] (rank order).

    One ``all_gather_into_tensor`` (NCCL over NVLink on GPUs, gloo on CPU).
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local
    batch, q_local, dim = (int(x) for x in local.shape)
    flat = torch.empty((world * batch * q_local * dim,), device=local.device, dtype=local.dtype)
    dist.all_gather_into_tensor(flat, local.contiguous().view(-1), group=group)
    return flat.view(world, batch, q_local, dim).permute(1, 0, 2, 3).reshape(batch, world * q_local, dim)
