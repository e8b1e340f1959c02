"""Multi-GPU plumbing for the DiT block: token-row sharding and Ulysses all-to-all.

The reference is single-GPU (model/layers.py:4-6); this is the B200 scale-out:
every linear / quantizer / norm is row-local, so token rows are split across
ranks with no communication, and attention exchanges tokens for heads once
each way (NCCL all_to_all over NVLink; gloo in the CPU tests).

The token -> head exchange is split into three collectives, K first, then V, then
Q, issued asynchronously: the K preparation (mean, pooling, INT8) runs while V and
Q are still in flight, and the V preparation while Q is.  A head order (a
permutation of the heads, rank p taking entries [p*H/P, (p+1)*H/P)) lets the
caller balance the per-rank attention work; every rank's result is the same
whatever the order, because each head's attention is computed whole on one rank.
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


def _check_order(order: torch.Tensor | None, heads: int) -> None:
    if order is not None and (order.numel() != heads or not torch.equal(order.sort().values,
                                                                        torch.arange(heads, device=order.device))):
        raise ValueError("head order must be a permutation of the heads")


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


def _pack(src: torch.Tensor, rows: int, heads: int, head_dim: int, P: int, order: torch.Tensor | None) -> torch.Tensor:
    """[rows, heads, D] view (unit stride in the last two dims) -> send buffer [P, rows, H/P * D].
    CUDA tensors take the native kernel (h3b_ulysses_pack: one read, one write); CPU
    tensors (gloo process groups, the host-side tests of the exchange) take the same
    layout in torch."""
    hpr = heads // P
    if not src.is_cuda:
        if order is not None:
            src = src.index_select(1, order)
        return src.reshape(rows, P, hpr * head_dim).permute(1, 0, 2).contiguous()
    from ._lib import check, lib
    from .ops import _p, _stream

    if head_dim != 128 or src.dtype != torch.bfloat16 or src.stride(2) != 1 or src.stride(1) != 128:
        raise ValueError("the Ulysses pack kernel takes bf16 heads of 128 contiguous channels")
    dst = torch.empty((P, rows, hpr * head_dim), device=src.device, dtype=src.dtype)
    o = None if order is None else order.to(device=src.device, dtype=torch.int64).contiguous()
    check(lib().h3b_ulysses_pack(_p(src), rows, heads, src.stride(0), _p(o), P, _p(dst), _stream(src)),
          "ulysses_pack")
    return dst


def _unpack(recv: torch.Tensor, rows: int, P: int, hd: int, order: torch.Tensor | None) -> torch.Tensor:
    """[P, rows, hd] received chunks -> token rows [rows, P*hd] in head index order."""
    if not recv.is_cuda:
        tokens = recv.view(P, rows, hd).permute(1, 0, 2).reshape(rows, P * hd)
        if order is None:
            return tokens
        heads = order.numel()
        D = P * hd // heads
        out = torch.empty_like(tokens)
        out.view(rows, heads, D).index_copy_(1, order, tokens.view(rows, heads, D))
        return out
    from ._lib import check, lib
    from .ops import _p, _stream

    heads = P * hd // 128
    out = torch.empty((rows, P * hd), device=recv.device, dtype=recv.dtype)
    o = None if order is None else order.to(device=recv.device, dtype=torch.int64).contiguous()
    check(lib().h3b_ulysses_unpack(_p(recv), rows, heads, _p(o), P, _p(out), out.stride(0), _stream(recv)),
          "ulysses_unpack")
    return out


def exchange_qkv_async(qkv: torch.Tensor, heads: int, head_dim: int, group=None,
                       order: torch.Tensor | None = None) -> dict[str, tuple[torch.Tensor, object]]:
    """Start the token -> head exchange of K, V and Q (in that order) from the QKV
    projection rows [L/P, 3*H*D].  Returns {"k" | "v" | "q": (tensor [L, H/P, D], work)}:
    a tensor holds all tokens (in rank order) of this rank's heads, valid on the
    current stream after `work.wait()`.  `order` (int64 [H], a permutation) assigns
    heads order[p*H/P:(p+1)*H/P] to rank p; None keeps heads in order."""
    P = dist.get_world_size(group)
    if heads % P:
        raise ValueError(f"{heads} heads do not split over {P} ranks")
    _check_order(order, heads)
    Lp = qkv.shape[0]
    hpr = heads // P
    view = qkv.view(Lp, 3, heads, head_dim)
    out = {}
    for name, slot in (("k", 1), ("v", 2), ("q", 0)):
        send = _pack(view[:, slot], Lp, heads, head_dim, P, order)   # [P, Lp, hd]
        recv = torch.empty((P * Lp, hpr, head_dim), device=qkv.device, dtype=qkv.dtype)
        work = dist.all_to_all_single(recv.view(P, Lp, hpr * head_dim), send, group=group, async_op=True)
        out[name] = (recv, work)
    return out


def heads_to_tokens(o: torch.Tensor, local_rows: int, group=None, order: torch.Tensor | None = None) -> torch.Tensor:
    """[L, (H/P)*D] (all tokens, own head group) -> [L/P, H*D] (own tokens, all heads, in
    head index order even when `order` assigned the heads to ranks out of order)."""
    P = dist.get_world_size(group)
    send = o.contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return _unpack(recv, local_rows, P, o.shape[1], order)


def balanced_head_order(kept: torch.Tensor, world: int) -> torch.Tensor:
    """A head order giving every rank H/P heads with nearly equal total work:
    heads by descending kept-tile count, each to the least-loaded rank that still
    has room (ties to the lower rank).  kept: per-head work [H] (any device);
    returns int64 [H] on kept's device, identical on every rank for identical input."""
    H = kept.numel()
    if H % world:
        raise ValueError(f"{H} heads do not split over {world} ranks")
    cap = H // world
    counts = [int(c) for c in kept.reshape(-1).cpu().tolist()]
    load = [0] * world
    members: list[list[int]] = [[] for _ in range(world)]
    for h in sorted(range(H), key=lambda i: (-counts[i], i)):
        r = min((r for r in range(world) if len(members[r]) < cap), key=lambda r: (load[r], r))
        members[r].append(h)
        load[r] += counts[h]
    order = [h for r in range(world) for h in sorted(members[r])]
    return torch.tensor(order, dtype=torch.int64, device=kept.device)


def gather_head_counts(local: torch.Tensor, order: torch.Tensor | None, heads: int, group=None) -> torch.Tensor:
    """Per-head counts [H] in head index order from each rank's counts of its own
    heads (local: [H/P], in the rank's assignment order)."""
    P = dist.get_world_size(group)
    parts = [torch.empty_like(local) for _ in range(P)]
    dist.all_gather(parts, local.contiguous(), group=group)
    flat = torch.cat(parts)
    if order is None:
        return flat
    full = torch.empty_like(flat)
    full[order.to(flat.device)] = flat
    return full
