"""(batch x head) sharding of the path across the GPUs of one node.

Every (batch, head) pair -- a *unit* -- is independent: pooling, scoring,
selection and the fine stage never mix heads.  Rank r of a world of size W
takes the contiguous unit range ``unit_range(B*H, W, r)`` (ceil split, so the
last ranks may get fewer units or none), computes it with no communication,
and -- only when the caller wants the whole output on every rank -- the ranks
exchange results with one ``all_gather_into_tensor`` over NCCL (NVLink /
NVSwitch on a B200 node), padded to equal shards.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist


def unit_range(num_units: int, world_size: int, rank: int):
    """[start, stop) of the units rank ``rank`` owns (contiguous ceil split)."""
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError(f"rank {rank} outside world of size {world_size}")
    per = math.ceil(num_units / world_size)
    start = min(num_units, rank * per)
    return start, min(num_units, start + per)


def local_units(x: torch.Tensor, world_size: int, rank: int) -> torch.Tensor:
    """This rank's units of a (B, H, N, D) tensor as a (1, n, N, D) view."""
    B, H, N, D = x.shape
    a, b = unit_range(B * H, world_size, rank)
    return x.reshape(B * H, N, D)[a:b].unsqueeze(0)


def gather_units(local: torch.Tensor, num_units: int, group=None) -> torch.Tensor:
    """All-gather per-rank unit outputs (1, n_r, N, D) into (num_units, N, D)."""
    world = dist.get_world_size(group)
    per = math.ceil(num_units / world)
    _, n, N, D = local.shape
    send = local.new_zeros(per, N, D)
    if n:
        send[:n] = local[0]
    out = local.new_empty(per * world, N, D)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, send, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), send, group=group)
    return out[:num_units]


def sharded_attention(Q, K, V, causal=False, block_size=64, top_k=16, *, group=None,
                      gather=True, attn_fn=None):
    """Head-sharded forward.  Q, K, V: full (B, H, N, D) tensors on every rank.

    Returns the full (B, H, N, D) output on every rank when ``gather``, else
    this rank's (1, n, N, D) slice.  ``attn_fn`` defaults to the B200 kernel
    path (``block_indexer_b200.attention``).
    """
    if attn_fn is None:
        from .block_indexer_b200 import attention as attn_fn
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, H, N, D = Q.shape
    q, k, v = (local_units(t, world, rank) for t in (Q, K, V))
    if q.shape[1]:
        out = attn_fn(q, k, v, causal=causal, block_size=block_size, top_k=top_k)
    else:
        out = q.new_empty(q.shape)
    if not gather:
        return out
    return gather_units(out, B * H, group).reshape(B, H, N, D)
