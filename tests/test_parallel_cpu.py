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
