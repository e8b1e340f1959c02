"""The long-sequence attention seam, driven by the reference's own caller.

FusedQKVAttention.stream_gated_residual_ of the reference (model/layers.py:302-897)
runs one memory-bounded attention layer through a backend's long-sequence
protocol: prepare V, check its metadata tuple, prepare K, stream the protected
prefix queries and then the video queries in chunks with their token indices,
optionally building K/V slab by slab (begin_compact_long_sequence_kv).  These
tests import that caller from an X-MinimaxH3 checkout -- the directory named by
REFERENCE_ROOT, else a `reference` directory beside this repository -- and let it
drive SpargeLongSequenceB200 / DenseLongSequenceB200 on CPU tensors.  The
backends' device stages are swapped for the CPU oracle, which the GPU tests hold
bit-identical to the kernels, so what is tested here is the protocol itself.
Skipped when no reference checkout is importable.
"""

from __future__ import annotations

import math
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "x-minimaxh3_b200"))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def _reference_root() -> str | None:
    for cand in (os.environ.get("REFERENCE_ROOT", ""), os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "h3serve", "native_engine", "model")):
            return cand
    return None


REF = _reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="no X-MinimaxH3 checkout (set REFERENCE_ROOT)")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, REF)
    import h3serve.native_engine.model.kernels as K
    import h3serve.native_engine.model.layers as Lyr

    return Lyr, K


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def _pad(n: int) -> int:
    return (n + 127) // 128 * 128


class OracleStages:
    """The stage functions of h3b.attention, computed by the CPU oracle, with a call log."""

    def __init__(self, A):
        self.A = A
        self.log: list[tuple] = []

    def prepare_values(self, v):
        L, H = v.shape[:2]
        vt, vs = O.value_fp8(_bits(v))
        self.log.append(("values", L))
        return self.A.PreparedValues(torch.from_numpy(vt), torch.from_numpy(vs), L, vt.shape[-1])

    def prepare_blocks(self, x, block, threshold=-0.1, mean=None, padded=None):
        L, H = x.shape[:2]
        thr = np.full(H, float(threshold), np.float32)
        pooled, sim, q, sc = O.pool_sim_quant(_bits(x), block, thr, None if mean is None else _bits(mean))
        Lpad = padded or _pad(L)
        qp = np.zeros((H, Lpad, 128), np.int8)
        qp[:, :q.shape[1]] = q
        self.log.append(("blocks", L, block))
        return self.A.PreparedBlocks(_bf16(pooled), torch.from_numpy(sim), torch.from_numpy(qp),
                                     torch.from_numpy(sc), L, block, Lpad)

    def key_mean(self, k, workspace=None):
        return _bf16(O.key_mean(_bits(k)))

    def block_mask(self, pq, pk, cfg, *, query_indices=None, protected_query_tokens=0):
        H = pq.pooled.shape[0]
        frames, ftok = cfg.video_layout or (0, 0)
        flags = int(cfg.keep_first_column) | (2 * int(cfg.keep_diagonal))
        bm = O.block_mask(_bits(pq.pooled), pq.similar.numpy(), _bits(pk.pooled), pk.similar.numpy(),
                          mode=0 if cfg.mode == "topk" else 1, budget=np.full(H, cfg.budget, np.float32),
                          protected_kb=(cfg.protected_tokens + 63) // 64, flags=flags,
                          temporal_radius=cfg.temporal_radius, temporal_spatial_radius=cfg.temporal_spatial_radius,
                          frames=frames, frame_tokens=ftok, protected_tokens=cfg.protected_tokens,
                          q_tokens=pq.tokens, q_index=None if query_indices is None else query_indices.numpy(),
                          protected_qb=(protected_query_tokens + 127) // 128)
        self.log.append(("mask", pq.tokens, cfg.protected_tokens, cfg.temporal_radius,
                         None if query_indices is None else query_indices.clone(), bm, pq, pk))
        return torch.from_numpy(bm.view(np.int32))

    def attention(self, pq, pk, pv, bitmap=None, sm_scale=None, out=None):
        bm = None if bitmap is None else bitmap.numpy().view(np.uint32)
        o = O.attention(pq.qi8.numpy(), pq.scale.numpy(), pq.block, pq.tokens, pk.qi8.numpy(), pk.scale.numpy(),
                        pk.tokens, pv.vt.numpy(), pv.scale.numpy(), bitmap=bm)
        self.log.append(("attention", pq.tokens, pq.block, bitmap is not None))
        return _bf16(o)

    def install(self, monkeypatch):
        for name in ("prepare_values", "prepare_blocks", "key_mean", "block_mask", "attention"):
            monkeypatch.setattr(self.A, name, getattr(self, name))
        monkeypatch.setattr(self.A, "_cuda", lambda *a, **k: None)


def _layer(Lyr, backend, hidden=256, heads=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    W = heads * 128
    qkv = torch.nn.Linear(hidden, 3 * W, dtype=torch.bfloat16)
    out = torch.nn.Linear(W, hidden, dtype=torch.bfloat16)
    with torch.no_grad():
        qkv.weight.copy_(torch.randn(3 * W, hidden, generator=g) * hidden ** -0.5)
        qkv.bias.copy_(torch.randn(3 * W, generator=g) * 0.1)
        out.weight.copy_(torch.randn(hidden, W, generator=g) * W ** -0.5)
        out.bias.zero_()
    layer = Lyr.FusedQKVAttention(qkv, out, num_heads=heads, head_dim=128, backend=backend, dtype=torch.bfloat16)
    with torch.no_grad():
        layer.q_norm.weight.fill_(1.0)
        layer.k_norm.weight.fill_(1.0)
    return layer


PREFIX, FRAMES, FRAME_TOKENS = 256, 4, 192
SEQ = PREFIX + FRAMES * FRAME_TOKENS


def _inputs(hidden=256, seed=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(SEQ, hidden, generator=g).to(torch.bfloat16)
    res = torch.randn(SEQ, hidden, generator=g).to(torch.bfloat16)
    gate = (torch.rand(2, hidden, generator=g) + 0.5).to(torch.bfloat16)
    segments = ((0, PREFIX, 0), (PREFIX, SEQ, 1))
    return x, res, gate, segments


def _stream(layer, x, res, gate, segments, chunk=256):
    r = res.clone()
    handled = layer.stream_gated_residual_(r, x, None, gate, segments, query_chunk_tokens=chunk,
                                           projection_chunk_tokens=128)
    assert handled, "the reference caller refused the B200 backend's long-sequence protocol"
    return r


def _unstreamed(Lyr, layer, x, res, gate, segments):
    """The reference's whole-sequence path with exact attention (torch_sdpa)."""
    layer.backend, saved = Lyr.torch_sdpa, layer.backend
    try:
        with torch.no_grad():
            proj = layer(x, None)
    finally:
        layer.backend = saved
    r = res.clone()
    Lyr._gated_residual_slice_(r, proj, gate, segments, start=0, stop=SEQ)
    return r


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm()))


def test_contract_selects_nhd(ref):
    from h3b.attention import SpargeLongSequenceB200

    from h3serve.native_engine.model.long_sequence_contract import resolve_physical_long_sequence_contract

    c = resolve_physical_long_sequence_contract(SpargeLongSequenceB200(), compact_kv=False,
                                                direct_nhd_kv_requested=False, fused_qknorm_hnd_requested=True,
                                                direct_hnd_fp8_value_requested=True)
    assert c.kv_layout == "NHD" and not c.fused_qknorm_hnd_layout and not c.direct_hnd_fp8_value


def test_sparge_stream_through_reference_caller(ref, monkeypatch):
    Lyr, K = ref
    import h3b.attention as A

    stages = OracleStages(A)
    stages.install(monkeypatch)
    backend = A.SpargeLongSequenceB200(A.MaskConfig("topk", 1.0), context=K)
    layer = _layer(Lyr, backend)
    x, res, gate, segments = _inputs()
    with torch.no_grad():
        got = _stream(layer, x, res, gate, segments)
        want = _unstreamed(Lyr, layer, x, res, gate, segments)
    # the prepared V tuple was accepted (heads / key_tokens / head_dim), K prepared once,
    # the prefix [0, 256) ran dense, the video ran as three chunks of at most 256 rows
    kinds = [e[0] for e in stages.log]
    assert kinds.count("values") == 1
    attn = [e for e in stages.log if e[0] == "attention"]
    assert [e[1] for e in attn] == [256, 256, 256, 256]
    assert attn[0][2] == 32 and not attn[0][3]          # prefix: per-warp Q, dense
    assert all(e[2] == 128 and e[3] for e in attn[1:])  # video: Sparge mask
    masks = [e for e in stages.log if e[0] == "mask"]
    assert all(m[2] == PREFIX for m in masks)
    # with a Top-K budget of 1.0 every tile is kept: the stream equals the reference's
    # own whole-sequence layer up to the INT8 / FP8 attention quantization
    d_got, d_want = (got.float() - res.float()), (want.float() - res.float())
    assert _cos(d_got, d_want) > 0.995, _cos(d_got, d_want)


def test_temporal_rail_uses_chunk_indices(ref, monkeypatch):
    Lyr, K = ref
    import h3b.attention as A

    stages = OracleStages(A)
    stages.install(monkeypatch)
    cfg = A.MaskConfig("topk", 0.25, temporal_radius=1, temporal_spatial_radius=0)
    backend = A.SpargeLongSequenceB200(cfg, context=K)
    layer = _layer(Lyr, backend)
    x, res, gate, segments = _inputs()
    with torch.no_grad(), K.attention_video_layout(FRAMES, FRAME_TOKENS):
        _stream(layer, x, res, gate, segments)
    masks = [e for e in stages.log if e[0] == "mask"]
    assert len(masks) == 3
    starts = [0, 256, 512]
    added = 0
    for (_, lq, prot, radius, idx, bm, pq, pk), s in zip(masks, starts):
        assert radius == 1 and prot == PREFIX
        assert idx is not None and torch.equal(idx, torch.arange(s, s + lq))
        # the rail centred on the chunk's own positions in the video, not on rows 0..lq
        for i in range(math.ceil(lq / 128)):
            qc = int(idx[min(i * 128 + 64, lq - 1)])
            qf, qsp = divmod(qc, FRAME_TOKENS)
            for j in range((SEQ + 63) // 64):
                kc = j * 64 + 32 - PREFIX
                if not 0 <= kc < FRAMES * FRAME_TOKENS:
                    continue
                kf, ksp = divmod(kc, FRAME_TOKENS)
                if abs(qf - kf) <= 1 and abs(qsp - ksp) <= 96:
                    assert np.all((bm[:, i, j // 32] >> (j % 32)) & 1 == 1)
        no_rail = stages.block_mask(pq, pk, A.MaskConfig("topk", 0.25, protected_tokens=PREFIX)).numpy()
        added += int((np.unpackbits(bm.view(np.uint8)) != np.unpackbits(no_rail.view(np.uint8))).sum())
    assert added > 0, "the temporal rail kept no block beyond the Top-K selection: the test would not see it"


def test_compact_kv_through_reference_caller(ref, monkeypatch):
    Lyr, K = ref
    import h3b.attention as A

    stages = OracleStages(A)
    stages.install(monkeypatch)
    built = {}

    class OracleCompactBuilder:
        """The product builder's protocol, with the slabs quantized by the oracle at finish()."""

        def __init__(self, *, key_tokens, heads, head_dim, key_mean, value_absmax, device, similarity_threshold=-0.1):
            self.L, self.H = key_tokens, heads
            self.mean = key_mean.to(torch.bfloat16).reshape(heads, 128)
            self.absmax = value_absmax.float().reshape(heads, 128)
            self.k = torch.empty(key_tokens, heads, 128, dtype=torch.bfloat16)
            self.v = torch.empty(key_tokens, heads, 128, dtype=torch.bfloat16)
            self.starts = []
            built["builder"] = self

        def add(self, start, key, value):
            assert start % 128 == 0
            self.starts.append(start)
            self.k[start:start + key.shape[0]] = key
            self.v[start:start + value.shape[0]] = value.to(torch.bfloat16)

        def finish(self):
            pk = stages.prepare_blocks(self.k, 64, -0.1, self.mean)
            pv = stages.prepare_values(self.v)
            return A.PreparedLongSequenceKVB200(pk, self.mean, pv, self.H, self.L)

    monkeypatch.setattr(A, "CompactLongSequenceKVBuilderB200", OracleCompactBuilder)
    backend = A.SpargeLongSequenceB200(A.MaskConfig("topk", 1.0), context=K)
    layer = _layer(Lyr, backend)

    # the compact build needs output-sliced projections (model/layers.py:430-434)
    def forward_output_slice(value, start, stop):
        w, b = layer.qkv_proj.weight[start:stop], layer.qkv_proj.bias[start:stop]
        return torch.nn.functional.linear(value, w, b)

    layer.qkv_proj.forward_output_slice = forward_output_slice
    x, res, gate, segments = _inputs()
    with torch.no_grad():
        tokens = [K._LONG_SEQUENCE_COMPACT_KV.set(True), K._LONG_SEQUENCE_SPLIT_QKV_OUTPUTS.set(True)]
        try:
            got = _stream(layer, x, res, gate, segments)
        finally:
            K._LONG_SEQUENCE_SPLIT_QKV_OUTPUTS.reset(tokens[1])
            K._LONG_SEQUENCE_COMPACT_KV.reset(tokens[0])
        want = _unstreamed(Lyr, layer, x, res, gate, segments)
    b = built["builder"]
    assert b.starts == list(range(0, SEQ, 128))
    d_got, d_want = (got.float() - res.float()), (want.float() - res.float())
    assert _cos(d_got, d_want) > 0.995, _cos(d_got, d_want)


def test_dense_stream_through_reference_caller(ref, monkeypatch):
    Lyr, K = ref
    import h3b.attention as A

    stages = OracleStages(A)
    stages.install(monkeypatch)
    layer = _layer(Lyr, A.DenseLongSequenceB200())
    x, res, gate, segments = _inputs()
    with torch.no_grad():
        got = _stream(layer, x, res, gate, segments)
        want = _unstreamed(Lyr, layer, x, res, gate, segments)
    attn = [e for e in stages.log if e[0] == "attention"]
    # long_sequence_all_queries: the whole packed sequence in chunks from its origin
    assert [e[1] for e in attn] == [256] * (SEQ // 256) and all(e[2] == 32 and not e[3] for e in attn)
    d_got, d_want = (got.float() - res.float()), (want.float() - res.float())
    assert _cos(d_got, d_want) > 0.995, _cos(d_got, d_want)
