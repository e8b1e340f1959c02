"""Quantized attention backends over libh3b.so.

Both backends are `AttentionBackend` callables of the native engine
(model/layers.py:20, 276-300): (q, k, v) bf16 [L, H, 128] -> bf16 [L, H, 128].

* SageAttentionB200    dense: per-block INT8 Q (128 rows) and K (64 rows, K
                       mean-smoothed), per-channel FP8 V, INT8 QK^T and FP8 PV
                       on tcgen05 (replaces sage_attention_sm89,
                       model/kernels.py:7645-7661)
* SpargeAttentionB200  the same kernel driven by the Sparge block mask: pooled
                       similarity, fixed Top-K or top-CDF selection and the
                       mandatory rails (replaces the Sparge backends,
                       model/kernels.py:2360-2441, 3668-3997)

The stage functions (prepare_queries / prepare_keys / prepare_values /
block_mask / attention) are public so a caller can stream K/V preparation
and query chunks the way the long-sequence protocol does (model/layers.py:341-356).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from ._lib import MaskParams, check, lib
from .ops import _cuda, _p, _stream

HEAD_DIM = 128


def _pad(n: int, m: int = 128) -> int:
    return (n + m - 1) // m * m


def _nhd_rows(x: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    """[L, H, 128] (unit stride in the last two dims) -> (tensor, L, H, row stride)."""
    if x.ndim != 3 or x.shape[-1] != HEAD_DIM:
        raise ValueError("attention inputs must be [L, H, 128]")
    if x.dtype != torch.bfloat16:
        raise ValueError("attention inputs must be bfloat16")
    if x.stride(2) != 1 or x.stride(1) != HEAD_DIM or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    return x, x.shape[0], x.shape[1], x.stride(0)


@dataclass
class PreparedBlocks:
    """Per-block INT8 tokens with Sparge pooled metadata."""

    pooled: torch.Tensor    # bf16 [H, nb, 128]
    similar: torch.Tensor   # u8 [H, nb]
    qi8: torch.Tensor       # int8 [H, Lpad, 128]
    scale: torch.Tensor     # f32 [H, nb]
    tokens: int
    block: int
    padded: int


@dataclass
class PreparedValues:
    vt: torch.Tensor        # e4m3 bytes [H, 128, Lpad]
    scale: torch.Tensor     # f32 [H, 128]
    tokens: int
    padded: int


def _thr(threshold, H: int, device) -> torch.Tensor:
    if isinstance(threshold, torch.Tensor):
        t = threshold.to(device=device, dtype=torch.float32).reshape(-1)
        if t.numel() == 1:
            t = t.expand(H)
        return t.contiguous()
    return torch.full((H,), float(threshold), device=device, dtype=torch.float32)


def key_mean(k: torch.Tensor, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Per-(head, channel) mean of K over the sequence, bf16 [H, 128]."""
    _cuda("key_mean", k)
    k, L, H, stride = _nhd_rows(k)
    need = int(lib().h3b_key_mean_workspace_bytes(L, H))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=k.device, dtype=torch.uint8)
    mean = torch.empty((H, HEAD_DIM), device=k.device, dtype=torch.bfloat16)
    check(lib().h3b_key_mean(_p(k), L, H, stride, _p(mean), _p(workspace), need, _stream(k)), "key_mean")
    return mean


def prepare_blocks(x: torch.Tensor, block: int, threshold=-0.1, mean: torch.Tensor | None = None,
                   padded: int | None = None) -> PreparedBlocks:
    """Sparge pool / similarity / per-block INT8 (model/sparge_nhd.py:163-227)."""
    _cuda("prepare_blocks", x, mean)
    x, L, H, stride = _nhd_rows(x)
    nb = (L + block - 1) // block
    Lpad = padded if padded is not None else _pad(L)
    dev = x.device
    pooled = torch.empty((H, nb, HEAD_DIM), device=dev, dtype=torch.bfloat16)
    similar = torch.empty((H, nb), device=dev, dtype=torch.uint8)
    qi8 = torch.empty((H, Lpad, HEAD_DIM), device=dev, dtype=torch.int8)
    if Lpad > nb * block:
        qi8[:, nb * block:].zero_()
    scale = torch.empty((H, nb), device=dev, dtype=torch.float32)
    thr = _thr(threshold, H, dev)
    m = None if mean is None else mean.to(torch.bfloat16).contiguous()
    check(lib().h3b_pool_sim_quant(_p(x), L, H, stride, _p(m), block, _p(thr), _p(pooled), _p(similar), _p(qi8),
                                   _p(scale), Lpad, _stream(x)), "pool_sim_quant")
    return PreparedBlocks(pooled, similar, qi8, scale, L, block, Lpad)


def prepare_queries(q: torch.Tensor, block: int = 128, threshold=-0.1) -> PreparedBlocks:
    return prepare_blocks(q, block, threshold)


def prepare_keys(k: torch.Tensor, threshold=-0.1, smooth: bool = True) -> tuple[PreparedBlocks, torch.Tensor | None]:
    mean = key_mean(k) if smooth else None
    return prepare_blocks(k, 64, threshold, mean), mean


def prepare_values(v: torch.Tensor) -> PreparedValues:
    """V -> per-channel FP8 E4M3 in [H, 128, Lpad] (model/compact_fp8.py:253-300)."""
    _cuda("prepare_values", v)
    v, L, H, stride = _nhd_rows(v)
    Lpad = _pad(L)
    vt = torch.empty((H, HEAD_DIM, Lpad), device=v.device, dtype=torch.uint8)
    vs = torch.empty((H, HEAD_DIM), device=v.device, dtype=torch.float32)
    check(lib().h3b_value_fp8(_p(v), L, H, stride, Lpad, _p(vt), _p(vs), _stream(v)), "value_fp8")
    return PreparedValues(vt, vs, L, Lpad)


@dataclass
class MaskConfig:
    """Selector and rails (model/kernels.py:3668-3941, 5206-5294)."""

    mode: str = "topk"            # "topk" (fixed Top-K) or "cdf" (top-CDF)
    budget: float | tuple = 0.5   # Top-K fraction, or CDF threshold
    protected_tokens: int = 0     # dense prefix keys (text / audio)
    keep_first_column: bool = False
    keep_diagonal: bool = False
    temporal_radius: int = -1
    temporal_spatial_radius: int = 0
    video_layout: tuple[int, int] | None = None  # (latent frames, tokens per frame)


def block_mask(pq: PreparedBlocks, pk: PreparedBlocks, cfg: MaskConfig) -> torch.Tensor:
    """uint32 bitmap [H, Qb, ceil(Kb/32)] of kept (Q block, K block) tiles."""
    H, Qb, _ = pq.pooled.shape
    Kb = pk.pooled.shape[1]
    dev = pq.pooled.device
    budget = cfg.budget if isinstance(cfg.budget, (tuple, list)) else (cfg.budget,) * H
    if len(budget) != H:
        raise ValueError(f"head-wise budget has {len(budget)} values for {H} heads")
    bud = torch.tensor(budget, dtype=torch.float32).to(dev)
    words = (Kb + 31) // 32
    bitmap = torch.empty((H, Qb, words), device=dev, dtype=torch.int32)
    frames, ftok = cfg.video_layout or (0, 0)
    p = MaskParams(0 if cfg.mode == "topk" else 1, ctypes.c_void_p(bud.data_ptr()),
                   (cfg.protected_tokens + 63) // 64, int(cfg.keep_first_column), int(cfg.keep_diagonal),
                   int(cfg.temporal_radius), int(cfg.temporal_spatial_radius), frames, ftok, cfg.protected_tokens,
                   pq.tokens)
    if cfg.mode not in ("topk", "cdf"):
        raise ValueError("mask mode must be 'topk' or 'cdf'")
    check(lib().h3b_block_mask(_p(pq.pooled), _p(pq.similar), Qb, _p(pk.pooled), _p(pk.similar), Kb, H,
                               ctypes.byref(p), _p(bitmap), _stream(bitmap)), "block_mask")
    # `bud` may be freed on return: the caching allocator hands its memory only to
    # later work on this stream, which runs after the kernel has read it.
    return bitmap


def bitmap_to_lut(bitmap: torch.Tensor, key_blocks: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Bitmap -> Sparge delta LUT [.., Kb] int32 and valid counts (model/sparse_lut.py:144-192)."""
    rows = bitmap.numel() // bitmap.shape[-1]
    lut = torch.empty(bitmap.shape[:-1] + (key_blocks,), device=bitmap.device, dtype=torch.int32)
    valid = torch.empty(bitmap.shape[:-1], device=bitmap.device, dtype=torch.int32)
    check(lib().h3b_bitmap_to_lut(_p(bitmap), rows, key_blocks, _p(lut), _p(valid), _stream(bitmap)),
          "bitmap_to_lut")
    return lut, valid


def attention(pq: PreparedBlocks, pk: PreparedBlocks, pv: PreparedValues, bitmap: torch.Tensor | None = None,
              sm_scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Quantized attention over prepared Q/K/V; bf16 [Lq, H, 128] (or into `out`, any row stride)."""
    H = pq.qi8.shape[0]
    Lq, Lk = pq.tokens, pk.tokens
    dev = pq.qi8.device
    if out is None:
        out = torch.empty((Lq, H, HEAD_DIM), device=dev, dtype=torch.bfloat16)
    if out.stride(2) != 1 or out.stride(1) != HEAD_DIM:
        raise ValueError("output must be [Lq, H, 128] with contiguous heads")
    scale = (1.0 / math.sqrt(HEAD_DIM)) if sm_scale is None else float(sm_scale)
    check(lib().h3b_attention(_p(pq.qi8), _p(pq.scale), pq.block, Lq, pq.padded, _p(pk.qi8), _p(pk.scale), Lk,
                              pk.padded, _p(pv.vt), _p(pv.scale), H, _p(bitmap), scale, _p(out), out.stride(0),
                              _stream(out)), "attention")
    return out


class SageAttentionB200:
    """Dense quantized attention backend (q, k, v: bf16 [L, H, 128])."""

    approximate = True

    def __init__(self, q_block: int = 128, smooth_k: bool = True) -> None:
        if q_block not in (64, 128):
            raise ValueError("q_block must be 64 or 128")
        self.q_block = q_block
        self.smooth_k = smooth_k

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        pv = prepare_values(v)
        pk, _ = prepare_keys(k, smooth=self.smooth_k)
        pq = prepare_queries(q, self.q_block)
        return attention(pq, pk, pv)


class SpargeAttentionB200:
    """Block-sparse quantized attention backend driven by the Sparge mask."""

    approximate = True

    def __init__(self, mask: MaskConfig | None = None, similarity_threshold: float = -0.1) -> None:
        self.mask = mask or MaskConfig()
        self.similarity_threshold = similarity_threshold
        self.last_density: float | None = None

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        pv = prepare_values(v)
        pk, _ = prepare_keys(k, self.similarity_threshold)
        pq = prepare_queries(q, 128, self.similarity_threshold)
        bitmap = block_mask(pq, pk, self.mask)
        return attention(pq, pk, pv, bitmap)


# ----------------------------------------------------------------------------- long-sequence protocol


@dataclass
class PreparedLongSequenceKVB200:
    """Reusable quantized K/V of one layer for query-streamed attention
    (the role of PreparedLongSequenceKV, model/kernels.py:2452-2476)."""

    keys: PreparedBlocks
    key_mean: torch.Tensor | None
    values: PreparedValues
    heads: int
    key_tokens: int
    head_dim: int = HEAD_DIM
    tensor_layout: str = "NHD"


def _as_lhd(x: torch.Tensor) -> torch.Tensor:
    if x.ndim == 4:
        if x.shape[0] != 1:
            raise ValueError("long-sequence tensors must have batch one")
        x = x[0]
    return x


class _LongSequenceMixin:
    """Duck-typed long-sequence protocol of the native engine
    (model/layers.py:341-356; model/kernels.py:3357-4000, 5441-5619): K/V are
    prepared once, query chunks are evaluated against them."""

    long_sequence_kv_layout = "NHD"
    long_sequence_value_dtype = torch.bfloat16
    supports_direct_nhd_kv = True

    def resolve_long_sequence_backend(self, query_tokens: int):
        return self

    def prepare_long_sequence_values(self, value: torch.Tensor):
        pv = prepare_values(_as_lhd(value))
        return pv.vt, pv.scale, pv.tokens, pv.padded, pv.vt.shape[0]

    def prepare_long_sequence_keys(self, key: torch.Tensor, value_fp8: torch.Tensor, value_scale: torch.Tensor,
                                   ) -> PreparedLongSequenceKVB200:
        key = _as_lhd(key)
        pk, mean = prepare_keys(key, getattr(self, "similarity_threshold", -0.1),
                                smooth=getattr(self, "smooth_k", True))
        L = key.shape[0]
        pv = PreparedValues(value_fp8, value_scale, L, value_fp8.shape[-1])
        return PreparedLongSequenceKVB200(pk, mean, pv, key.shape[1], L)

    def long_sequence_prefix_queries(self, query: torch.Tensor, prepared: PreparedLongSequenceKVB200) -> torch.Tensor:
        """Protected prefix queries (text / audio): dense over every key."""
        pq = prepare_queries(_as_lhd(query), 128, getattr(self, "similarity_threshold", -0.1))
        return attention(pq, prepared.keys, prepared.values)

    def long_sequence_all_queries(self, query: torch.Tensor, prepared: PreparedLongSequenceKVB200) -> torch.Tensor:
        return self.long_sequence_video_queries(query, prepared, protected_tokens=0, query_token_indices=None)


class DenseLongSequenceB200(_LongSequenceMixin, SageAttentionB200):
    """Dense backend with the long-sequence protocol (role of
    DenseLongSequenceAttentionBackend, model/kernels.py:5441-5619)."""

    def long_sequence_video_queries(self, query, prepared, *, protected_tokens=0, query_token_indices=None):
        pq = prepare_queries(_as_lhd(query), self.q_block)
        return attention(pq, prepared.keys, prepared.values)


class SpargeLongSequenceB200(_LongSequenceMixin, SpargeAttentionB200):
    """Sparge backend with the long-sequence protocol (role of
    SplitModalityProtectedSpargeAttentionBackend.long_sequence_video_queries,
    model/kernels.py:3668-3997): the chunk's queries are pooled and selected
    against the prepared keys; the protected prefix keys stay dense."""

    smooth_k = True

    def long_sequence_video_queries(self, query, prepared, *, protected_tokens=0, query_token_indices=None):
        q = _as_lhd(query)
        if query_token_indices is not None and query_token_indices.numel() != q.shape[0]:
            raise ValueError("long-sequence Query indices must align with the chunk")
        pq = prepare_queries(q, 128, self.similarity_threshold)
        cfg = MaskConfig(**{**self.mask.__dict__, "protected_tokens": int(protected_tokens)})
        if query_token_indices is not None and cfg.temporal_radius >= 0:
            # the temporal rail assumes the whole video sequence as queries
            cfg.temporal_radius = -1
        bitmap = block_mask(pq, prepared.keys, cfg)
        return attention(pq, prepared.keys, prepared.values, bitmap)
