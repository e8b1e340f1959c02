"""Multi-GPU plumbing for the DiT block: token-row sharding and Ulysses all-to-all.

The reference is single-GPU (model/layers.py:4-6); this is the B200 scale-out:
every linear / quantizer / norm is row-local, so token rows are split across
ranks with no communication, and attention exchanges tokens for heads once
each way (NCCL all_to_all over NVLink; gloo in the CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s contiguous token slice; total must divide."""
    if world <= 0 or total % world:
        raise ValueError(f"{total} rows do not split evenly over {world} ranks")
    per = total // world
    return rank * per, per


def tokens_to_heads(qkv: torch.Tensor, heads: int, head_dim: int, group=None) -> torch.Tensor:
    """[L/P, 3*H*D] (own tokens, all heads; q|k|v blocks of H*D) ->
    [L, 3*(H/P)*D] (all tokens in rank order, own head group; q|k|v blocks of (H/P)*D)."""
    P = dist.get_world_size(group)
    if heads % P:
        raise ValueError(f"{heads} heads do not split over {P} ranks")
    Lp = qkv.shape[0]
    hd = heads // P * head_dim
    send = qkv.reshape(Lp, 3, P, hd).permute(2, 0, 1, 3).contiguous()   # [P, Lp, 3, hd]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(P * Lp, 3 * hd)


def heads_to_tokens(o: torch.Tensor, local_rows: int, group=None) -> torch.Tensor:
    """[L, (H/P)*D] (all tokens, own head group) -> [L/P, H*D] (own tokens, all heads)."""
    P = dist.get_world_size(group)
    send = o.contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    hd = o.shape[1]
    return recv.view(P, local_rows, hd).permute(1, 0, 2).reshape(local_rows, P * hd)
