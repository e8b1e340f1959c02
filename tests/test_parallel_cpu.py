"""The Ulysses exchange and the failure path on world-size-2 gloo ranks (CPU).

The all-to-all pair must hand each rank exactly its head group of every token
and restore the token-sharded layout; a rank that dies before a collective must
surface as an error on the other rank within the process-group timeout, not as
a hang.
"""

import multiprocessing as mp
import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "x-minimaxh3_b200"))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn, q):
    try:
        sys.path.insert(0, os.path.join(ROOT, "x-minimaxh3_b200"))
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        q.put((rank, "ok", fn(rank, world)))
    except Exception as e:  # reported to the parent, never re-raised into a hang
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run(fn, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=timeout)
        out[r] = (status, payload)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def _full_qkv(L, H, D):
    g = torch.Generator().manual_seed(0)
    return torch.randn(L, 3 * H * D, generator=g)


def exchange_roundtrip(rank, world):
    from h3b import parallel as P
    L, H, D = 12, 4, 8
    full = _full_qkv(L, H, D)
    r0, n = P.shard_rows(L, world, rank)
    local = full[r0:r0 + n].clone()
    heads = P.tokens_to_heads(local, H, D)
    hd = H // world * D
    expect = full.view(L, 3, world, hd)[:, :, rank, :].reshape(L, 3 * hd)
    assert torch.equal(heads, expect)
    o = heads.view(L, 3, hd)[:, 0, :]                 # pretend attention output = this rank's q heads
    back = P.heads_to_tokens(o, n)
    assert torch.equal(back, full[r0:r0 + n, :H * D])
    return True


def async_exchange_with_order(rank, world):
    """K, V, Q exchanged separately with a head order that sends heads out of order:
    each rank receives exactly its assigned heads of every token, the output exchange
    restores head index order, and the balanced assignment is identical on both ranks."""
    from h3b import parallel as P
    L, H, D = 12, 4, 8
    full = _full_qkv(L, H, D)
    r0, n = P.shard_rows(L, world, rank)
    local = full[r0:r0 + n].clone()
    order = torch.tensor([3, 0, 2, 1])
    ex = P.exchange_qkv_async(local, H, D, order=order)
    mine = order[rank * 2:(rank + 1) * 2]
    view = full.view(L, 3, H, D)
    for name, slot in (("k", 1), ("v", 2), ("q", 0)):
        t, work = ex[name]
        work.wait()
        assert torch.equal(t, view[:, slot][:, mine]), name
    q, _ = ex["q"]
    back = P.heads_to_tokens(q.reshape(L, 2 * D), n, order=order)
    assert torch.equal(back, full[r0:r0 + n, :H * D])
    counts = P.gather_head_counts(torch.tensor([10.0 * rank + 1, 10.0 * rank + 2]), order, H)
    expect = torch.empty(4)
    expect[order] = torch.tensor([1.0, 2.0, 11.0, 12.0])
    assert torch.equal(counts, expect)
    return P.balanced_head_order(counts, world).tolist()


def dead_peer(rank, world):
    import torch.distributed as dist
    from h3b import parallel as P
    if rank == 1:
        os._exit(3)                                   # host-side failure between steps
    local = torch.zeros(4, 3 * 4 * 8)
    P.tokens_to_heads(local, 4, 8)                    # must raise, not hang
    return "collective unexpectedly completed"


def test_shard_rows():
    from h3b import parallel as P
    assert P.shard_rows(111600, 8, 3) == (3 * 13950, 13950)
    with pytest.raises(ValueError):
        P.shard_rows(10, 3, 0)


def test_ulysses_exchange_roundtrip_gloo():
    out = _run(exchange_roundtrip)
    assert out[0] == ("ok", True) and out[1] == ("ok", True), out


def test_async_exchange_with_head_order_gloo():
    out = _run(async_exchange_with_order)
    assert out[0][0] == "ok" and out[1][0] == "ok", out
    assert out[0][1] == out[1][1]                     # both ranks choose the same assignment


def test_balanced_head_order():
    from h3b import parallel as P
    kept = torch.tensor([900, 100, 120, 880, 500, 510, 300, 290, 50, 60, 700, 650, 410, 420, 330, 340])
    for world in (2, 4, 8):
        order = P.balanced_head_order(kept, world)
        assert sorted(order.tolist()) == list(range(16))
        load = kept[order].view(world, -1).sum(1).double()
        naive = kept.view(world, -1).sum(1).double()
        assert load.max() / load.mean() <= naive.max() / naive.mean()
        # the heaviest head (900) needs a partner of at least 50 when each rank takes two
        best = {2: 3280, 4: 1640, 8: 950}[world]
        assert load.max() <= best * 1.02


def test_dead_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, dead_peer, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, status, payload = q.get(timeout=90)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert rank == 0 and status == "error", (rank, status, payload)
