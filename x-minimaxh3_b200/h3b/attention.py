"""Quantized attention backends over libh3b.so.

Both backends are `AttentionBackend` callables of the native engine
(model/layers.py:20, 276-300): (q, k, v) bf16 [L, H, 128] -> bf16 [L, H, 128].

* SageAttentionB200    dense: INT8 Q and K (K mean-smoothed) in Sage's per_thread,
                       per_warp or per-block scale groups, per-channel FP8 V,
                       INT8 QK^T and FP8 PV on tcgen05 (replaces
                       sage_attention_sm89, model/kernels.py:7645-7746)
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
from dataclasses import dataclass, replace

import torch

from . import context as _context
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


GRAN_BLOCK, GRAN_PER_THREAD = 0, 1


@dataclass
class PreparedBlocks:
    """INT8 tokens with their scales (and, for Sparge, pooled metadata).

    gran GRAN_BLOCK: one scale per `block` rows (Sparge per-block, Sage per_warp);
    gran GRAN_PER_THREAD: Sage per_thread groups (Q: 32 per 128 rows, K: 4 per 64)."""

    pooled: torch.Tensor | None    # bf16 [H, nb, 128] (None: not pooled)
    similar: torch.Tensor | None   # u8 [H, nb]
    qi8: torch.Tensor              # int8 [H, Lpad, 128]
    scale: torch.Tensor            # f32 [H, nb] (per_thread: [H, nb * groups])
    tokens: int
    block: int
    padded: int
    gran: int = GRAN_BLOCK


@dataclass
class PreparedValues:
    vt: torch.Tensor        # e4m3 bytes [H, 128, Lpad]
    scale: torch.Tensor     # f32 [H, 128]
    tokens: int
    padded: int


_THRESHOLDS: dict[tuple, torch.Tensor] = {}


def _thr(threshold, H: int, device) -> torch.Tensor:
    if isinstance(threshold, torch.Tensor):
        t = threshold.to(device=device, dtype=torch.float32).reshape(-1)
        if t.numel() == 1:
            t = t.expand(H)
        return t.contiguous()
    # a scalar threshold: its [H] device copy is made once per (value, H, device)
    key = (float(threshold), H, str(device))
    t = _THRESHOLDS.get(key)
    if t is None:
        t = torch.full((H,), float(threshold), device=device, dtype=torch.float32)
        _THRESHOLDS[key] = t
    return t


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


def quantize_per_thread(x: torch.Tensor, kind: str, mean: torch.Tensor | None = None) -> PreparedBlocks:
    """Sage per_thread INT8 (qk_quant_gran 3) of Q (kind "q": 32 scale groups per
    128 rows) or K (kind "k": 4 groups per 64 rows, values bf16(k - mean)); the
    grouping of sageattention's per_thread_int8 (model/sage_fused_quant.py:20-283)."""
    _cuda("quantize_per_thread", x, mean)
    x, L, H, stride = _nhd_rows(x)
    blk, ng = (128, 32) if kind == "q" else (64, 4)
    if kind not in ("q", "k"):
        raise ValueError("kind must be 'q' or 'k'")
    nb = (L + blk - 1) // blk
    Lpad = _pad(L)
    dev = x.device
    qi8 = torch.empty((H, Lpad, HEAD_DIM), device=dev, dtype=torch.int8)
    if Lpad > nb * blk:
        qi8[:, nb * blk:].zero_()
    scale = torch.empty((H, nb * ng), device=dev, dtype=torch.float32)
    m = None if mean is None else mean.to(torch.bfloat16).contiguous()
    check(lib().h3b_quantize_per_thread_int8(_p(x), L, H, stride, _p(m), 0 if kind == "q" else 1, _p(qi8), _p(scale),
                                             Lpad, _stream(x)), "quantize_per_thread_int8")
    return PreparedBlocks(None, None, qi8, scale, L, blk, Lpad, GRAN_PER_THREAD)


def prepare_queries(q: torch.Tensor, block: int = 128, threshold=-0.1) -> PreparedBlocks:
    """Q in `block`-row scale groups: 128 (Sparge per-block), 64, or 32 (Sage per_warp)."""
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


_BUDGETS: dict[tuple, torch.Tensor] = {}


def _budget_tensor(budget: tuple[float, ...], device) -> torch.Tensor:
    """The head-wise budgets on the device, uploaded once per (values, device)."""
    key = (budget, str(device))
    t = _BUDGETS.get(key)
    if t is None:
        t = torch.tensor(budget, dtype=torch.float32).to(device)
        _BUDGETS[key] = t
    return t


def block_mask(pq: PreparedBlocks, pk: PreparedBlocks, cfg: MaskConfig, *,
               query_indices: torch.Tensor | None = None, protected_query_tokens: int = 0) -> torch.Tensor:
    """uint32 bitmap [H, Qb, ceil(Kb/32)] of kept (Q block, K block) tiles.

    query_indices: int64 [Lq] video positions of a chunk of selected queries; the
    temporal rail then centres query block i at query_indices[min(128 i + 64, Lq - 1)]
    (model/kernels.py:5247-5254).  protected_query_tokens: the first
    ceil(p / 128) query blocks keep every key block (model/kernels.py:2423-2426)."""
    H, Qb, _ = pq.pooled.shape
    Kb = pk.pooled.shape[1]
    dev = pq.pooled.device
    if cfg.mode not in ("topk", "cdf"):
        raise ValueError("mask mode must be 'topk' or 'cdf'")
    budget = tuple(cfg.budget) if isinstance(cfg.budget, (tuple, list)) else (cfg.budget,) * H
    if len(budget) != H:
        raise ValueError(f"head-wise budget has {len(budget)} values for {H} heads")
    bud = _budget_tensor(tuple(float(b) for b in budget), dev)
    idx = None
    if query_indices is not None:
        if query_indices.ndim != 1 or query_indices.numel() != pq.tokens or query_indices.device != dev:
            raise ValueError("query indices must be one device index per query row")
        idx = query_indices.to(torch.int64).contiguous()
    words = (Kb + 31) // 32
    bitmap = torch.empty((H, Qb, words), device=dev, dtype=torch.int32)
    frames, ftok = cfg.video_layout or (0, 0)
    p = MaskParams(0 if cfg.mode == "topk" else 1, ctypes.c_void_p(bud.data_ptr()),
                   (cfg.protected_tokens + 63) // 64, int(cfg.keep_first_column), int(cfg.keep_diagonal),
                   int(cfg.temporal_radius), int(cfg.temporal_spatial_radius), frames, ftok, cfg.protected_tokens,
                   pq.tokens, _p(idx), (int(protected_query_tokens) + 127) // 128)
    check(lib().h3b_block_mask(_p(pq.pooled), _p(pq.similar), Qb, _p(pk.pooled), _p(pk.similar), Kb, H,
                               ctypes.byref(p), _p(bitmap), _stream(bitmap)), "block_mask")
    # `idx` may be freed on return: the caching allocator hands its memory only to
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
    if bitmap is not None and (pq.gran != GRAN_BLOCK or pq.block != 128):
        raise ValueError("the block mask is defined over 128-row per-block query tiles")
    check(lib().h3b_attention(_p(pq.qi8), _p(pq.scale), pq.gran, pq.block, Lq, pq.padded, _p(pk.qi8), _p(pk.scale),
                              pk.gran, Lk, pk.padded, _p(pv.vt), _p(pv.scale), H, _p(bitmap), scale, _p(out),
                              out.stride(0), _stream(out)), "attention")
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


QK_QUANT_GRANS = ("per_thread", "per_warp", "per_block")


class SageAttentionB200:
    """Dense quantized attention backend (q, k, v: bf16 [L, H, 128]), the role of
    sage_attention_sm89 (model/kernels.py:7645-7661) with its qk_quant_gran:

    * "per_thread" (the reference's default, kernels.py:118-120): Q scale groups of 4
      rows, K groups of 16 keys per 64-key block (quantize_per_thread);
    * "per_warp": Q groups of 32 rows, K per 64-key block (kernels.py:4142-4151);
    * "per_block": Q groups of `q_block` rows (128, or 64 for per-64-token blocks),
      K per 64-key block -- Sparge's per-block quantization.

    K is mean-smoothed (bf16(k - mean_L(k))) unless smooth_k is False; V is per-channel
    FP8 with scale absmax / 2.25."""

    approximate = True

    def __init__(self, q_block: int = 128, smooth_k: bool = True, qk_quant_gran: str | None = None) -> None:
        if qk_quant_gran is None:
            qk_quant_gran = "per_warp" if q_block == 32 else "per_block"
        if qk_quant_gran not in QK_QUANT_GRANS:
            raise ValueError(f"qk_quant_gran must be one of {QK_QUANT_GRANS}")
        if qk_quant_gran == "per_warp":
            q_block = 32
        if q_block not in (32, 64, 128):
            raise ValueError("q_block must be 32, 64 or 128")
        self.q_block = q_block
        self.qk_quant_gran = qk_quant_gran
        self.smooth_k = smooth_k

    def quantize_queries(self, q: torch.Tensor) -> PreparedBlocks:
        if self.qk_quant_gran == "per_thread":
            return quantize_per_thread(q, "q")
        return prepare_queries(q, self.q_block)

    def quantize_keys(self, k: torch.Tensor) -> PreparedBlocks:
        if self.qk_quant_gran == "per_thread":
            return quantize_per_thread(k, "k", key_mean(k) if self.smooth_k else None)
        return prepare_keys(k, smooth=self.smooth_k)[0]

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        pv = prepare_values(v)
        pk = self.quantize_keys(k)
        pq = self.quantize_queries(q)
        return attention(pq, pk, pv)


class SpargeAttentionB200:
    """Block-sparse quantized attention backend driven by the Sparge mask.

    The request's protected prefix (read from the context source, see h3b.context)
    keeps its query rows and key columns dense, as ModalityProtectedSpargeAttentionBackend
    does (model/kernels.py:2381-2427); a video layout in the context enables the
    temporal rail when `mask.temporal_radius >= 0` and the mask names no layout."""

    approximate = True

    def __init__(self, mask: MaskConfig | None = None, similarity_threshold: float = -0.1, context=None) -> None:
        self.mask = mask or MaskConfig()
        self.similarity_threshold = similarity_threshold
        self.context = _context if context is None else context
        self.last_density: float | None = None

    def request_protected_prefix(self) -> int:
        return int(_context.source_getter(self.context, "current_attention_protected_prefix", 0) or 0)

    def request_video_layout(self) -> tuple[int, int] | None:
        layout = _context.source_getter(self.context, "current_attention_video_layout", None)
        return None if layout is None else (int(layout[0]), int(layout[1]))

    def _temporal(self, cfg: MaskConfig, key_tokens: int, protected_tokens: int, query_tokens: int,
                  selected: bool) -> MaskConfig:
        """cfg with the temporal rail's layout filled in, or switched off where the
        reference leaves the map unchanged (model/kernels.py:5226-5245)."""
        layout = cfg.video_layout or self.request_video_layout()
        if cfg.temporal_radius < 0 or layout is None:
            return replace(cfg, temporal_radius=-1)
        frames, ftok = layout
        video = frames * ftok
        if key_tokens - protected_tokens != video or (not selected and query_tokens != video):
            return replace(cfg, temporal_radius=-1)
        return replace(cfg, video_layout=(frames, ftok), protected_tokens=protected_tokens)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        pv = prepare_values(v)
        pk, _ = prepare_keys(k, self.similarity_threshold)
        pq = prepare_queries(q, 128, self.similarity_threshold)
        prefix = self.request_protected_prefix()
        prefix = prefix if 0 < prefix < pq.tokens else 0
        cfg = self.mask
        if prefix:
            cfg = replace(cfg, protected_tokens=max(cfg.protected_tokens, prefix))
        if cfg.temporal_radius >= 0 and cfg.video_layout is None:
            cfg = self._temporal(cfg, pk.tokens, cfg.protected_tokens, pq.tokens, False)
        bitmap = block_mask(pq, pk, cfg, protected_query_tokens=prefix)
        return attention(pq, pk, pv, bitmap)


# ----------------------------------------------------------------------------- long-sequence protocol


@dataclass
class PreparedLongSequenceKVB200:
    """Reusable quantized K/V of one layer for query-streamed attention
    (the role of PreparedLongSequenceKV, model/kernels.py:2452-2476).  Holds no
    sequence-long bf16 K or V: INT8 K with its per-64-row scales and Sparge pooled
    metadata, FP8 V with its per-channel scales."""

    keys: PreparedBlocks
    key_mean: torch.Tensor | None
    values: PreparedValues
    heads: int
    key_tokens: int
    head_dim: int = HEAD_DIM
    tensor_layout: str = "NHD"


def _as_lhd(x: torch.Tensor, what: str) -> torch.Tensor:
    """[1, L, H, 128] or [L, H, 128] (NHD, the layout this backend declares) -> [L, H, 128]."""
    if x.ndim == 4:
        if x.shape[0] != 1:
            raise ValueError(f"long-sequence {what} must have batch one")
        x = x[0]
    if x.ndim != 3 or x.shape[-1] != HEAD_DIM:
        raise ValueError(f"long-sequence {what} must use [1,L,H,128] layout")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"long-sequence {what} must be bfloat16")
    return x


def _values_from_protocol(value_fp8: torch.Tensor, value_scale: torch.Tensor, heads: int,
                          key_tokens: int) -> PreparedValues:
    """The (value_fp8 [1, H, 128, Lpad], value_scale [1, H, 128]) pair of
    prepare_long_sequence_values back to the kernel's arrays, shape-checked
    against K as the reference checks it (model/kernels.py:3548-3557)."""
    Lpad = _pad(key_tokens)
    if tuple(value_fp8.shape) != (1, heads, HEAD_DIM, Lpad):
        raise ValueError("prepared long-sequence V shape does not match K")
    if tuple(value_scale.shape) != (1, heads, HEAD_DIM):
        raise ValueError("prepared long-sequence V scale does not match K")
    vt = value_fp8.view(torch.uint8).reshape(heads, HEAD_DIM, Lpad)
    return PreparedValues(vt, value_scale.reshape(heads, HEAD_DIM), key_tokens, Lpad)


class CompactLongSequenceKVBuilderB200:
    """Builds a layer's prepared K/V slab by slab, so no sequence-long bf16 K or V
    ever exists (the role of _CompactSparseKVBuilder / _CompactDenseKVBuilder,
    model/kernels.py:2586-2772).  The caller gathers the K mean and the V absmax
    over the whole sequence first (model/layers.py:531-555), then hands each
    projected slab to add(); finish() returns the prepared K/V.

    Per slab: K - mean -> bf16 -> Sparge pool / similarity / per-64-row INT8
    (h3b_pool_sim_quant_slab) and V * 2.25/absmax -> E4M3 (h3b_value_fp8_given_absmax),
    both written in place into the sequence's arrays."""

    def __init__(self, *, key_tokens: int, heads: int, head_dim: int, key_mean: torch.Tensor,
                 value_absmax: torch.Tensor, device, similarity_threshold: float = -0.1) -> None:
        if head_dim != HEAD_DIM:
            raise ValueError("the B200 attention requires head dimension 128")
        if key_tokens <= 0 or heads <= 0:
            raise ValueError("key tokens and heads must be positive")
        if tuple(key_mean.shape[-2:]) != (heads, head_dim) or key_mean.numel() != heads * head_dim:
            raise ValueError("compact K mean must be [heads, head_dim]")
        if tuple(value_absmax.shape) != (heads, head_dim):
            raise ValueError("compact V absmax must use [heads,head_dim]")
        dev = torch.device(device)
        _cuda("begin_compact_long_sequence_kv", key_mean.to(dev))
        self.key_tokens, self.heads, self.head_dim = int(key_tokens), int(heads), int(head_dim)
        L, H = self.key_tokens, self.heads
        Kb, Lpad = (L + 63) // 64, _pad(L)
        self.mean = key_mean.to(device=dev, dtype=torch.bfloat16).reshape(H, HEAD_DIM).contiguous()
        self.absmax = value_absmax.to(device=dev, dtype=torch.float32).contiguous()
        self.thr = _thr(similarity_threshold, H, dev)
        self.pooled = torch.empty((H, Kb, HEAD_DIM), device=dev, dtype=torch.bfloat16)
        self.similar = torch.empty((H, Kb), device=dev, dtype=torch.uint8)
        self.qi8 = torch.empty((H, Lpad, HEAD_DIM), device=dev, dtype=torch.int8)
        if Lpad > Kb * 64:
            self.qi8[:, Kb * 64:].zero_()
        self.kscale = torch.empty((H, Kb), device=dev, dtype=torch.float32)
        self.vt = torch.empty((H, HEAD_DIM, Lpad), device=dev, dtype=torch.uint8)
        self.vscale = torch.empty((H, HEAD_DIM), device=dev, dtype=torch.float32)
        self._covered = 0

    def add(self, start: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Quantize the slab of rows [start, start + rows) (start a multiple of 128,
        slabs in order); key / value: bf16 [rows, H, 128], any row stride."""
        if key.shape != value.shape or tuple(key.shape[1:]) != (self.heads, self.head_dim):
            raise ValueError("compact Sparse K/V slab shape mismatch")
        rows = int(key.shape[0])
        if start % 128 or start + rows > self.key_tokens or rows <= 0:
            raise ValueError("compact Sparse K/V slab boundary is invalid")
        if start != self._covered:
            raise ValueError("compact K/V slabs must arrive in order without gaps")
        k, _, H, kst = _nhd_rows(key)
        v, _, _, vst = _nhd_rows(value.to(torch.bfloat16))
        _cuda("compact_kv_add", k, v)
        b0 = start // 64
        check(lib().h3b_pool_sim_quant_slab(_p(k), rows, H, kst, _p(self.mean), 64, _p(self.thr),
                                            _p(self.pooled[:, b0:]), _p(self.similar[:, b0:]),
                                            _p(self.qi8[:, start:]), _p(self.kscale[:, b0:]),
                                            self.pooled.shape[1], self.qi8.shape[1], _stream(k)),
              "pool_sim_quant_slab")
        check(lib().h3b_value_fp8_given_absmax(_p(v), rows, H, vst, _p(self.absmax), _p(self.vt[:, :, start:]),
                                               self.vt.shape[2], _p(self.vscale), _stream(v)),
              "value_fp8_given_absmax")
        self._covered = start + rows

    def finish(self) -> PreparedLongSequenceKVB200:
        if self._covered != self.key_tokens:
            raise ValueError(f"compact K/V covers {self._covered} of {self.key_tokens} tokens")
        keys = PreparedBlocks(self.pooled, self.similar, self.qi8, self.kscale, self.key_tokens, 64,
                              self.qi8.shape[1])
        values = PreparedValues(self.vt, self.vscale, self.key_tokens, self.vt.shape[2])
        return PreparedLongSequenceKVB200(keys, self.mean, values, self.heads, self.key_tokens)


class _LongSequenceMixin:
    """Duck-typed long-sequence protocol of the native engine
    (model/layers.py:341-356, 424-897; model/kernels.py:3357-4000, 5441-5619): K/V
    are prepared once per layer -- whole (prepare_long_sequence_values, then _keys)
    or slab by slab (begin_compact_long_sequence_kv) -- and query chunks are
    evaluated against them.  K/V travel in NHD ([1, L, H, 128]), the layout this
    backend declares (long_sequence_kv_layout), which
    model/long_sequence_contract.py:35-47 then selects for every request."""

    long_sequence_kv_layout = "NHD"
    long_sequence_value_dtype = torch.bfloat16
    supports_direct_nhd_kv = True
    minimum_long_sequence_tokens = 128

    def resolve_long_sequence_backend(self, query_tokens: int):
        return self if int(query_tokens) >= self.minimum_long_sequence_tokens else None

    def prepare_long_sequence_values(self, value: torch.Tensor):
        """V [1, L, H, 128] -> (value_fp8 e4m3 [1, H, 128, Lpad], value_scale f32 [1, H, 128],
        heads, key_tokens, head_dim), the tuple model/layers.py:668-680 unpacks."""
        v = _as_lhd(value, "V")
        pv = prepare_values(v)
        H = v.shape[1]
        return (pv.vt.view(torch.float8_e4m3fn).unsqueeze(0), pv.scale.unsqueeze(0), H, pv.tokens, HEAD_DIM)

    def prepare_long_sequence_keys(self, key: torch.Tensor, value_fp8: torch.Tensor, value_scale: torch.Tensor,
                                   ) -> PreparedLongSequenceKVB200:
        k = _as_lhd(key, "K")
        L, H = k.shape[0], k.shape[1]
        pv = _values_from_protocol(value_fp8, value_scale, H, L)
        pk, mean = prepare_keys(k, getattr(self, "similarity_threshold", -0.1), smooth=getattr(self, "smooth_k", True))
        return PreparedLongSequenceKVB200(pk, mean, pv, H, L)

    def begin_compact_long_sequence_kv(self, *, key_tokens: int, heads: int, head_dim: int, key_mean: torch.Tensor,
                                       value_absmax: torch.Tensor, device) -> CompactLongSequenceKVBuilderB200:
        return CompactLongSequenceKVBuilderB200(key_tokens=key_tokens, heads=heads, head_dim=head_dim,
                                                key_mean=key_mean, value_absmax=value_absmax, device=device,
                                                similarity_threshold=getattr(self, "similarity_threshold", -0.1))

    @staticmethod
    def _check_query(q: torch.Tensor, prepared: PreparedLongSequenceKVB200) -> None:
        if q.ndim != 3 or q.shape[0] <= 0 or q.shape[1] != prepared.heads or q.shape[2] != prepared.head_dim:
            raise ValueError("long-sequence Query chunk does not match prepared K/V")

    def long_sequence_prefix_queries(self, query: torch.Tensor, prepared: PreparedLongSequenceKVB200) -> torch.Tensor:
        """Protected prefix queries (text / audio): dense over every key, per-warp
        (32-row) Q scales over the prepared per-64-row K, the formulation of the
        reference's compact prefix path (model/kernels.py:3628-3666)."""
        q = _as_lhd(query, "Query")
        self._check_query(q, prepared)
        pq = prepare_queries(q, 32)
        return attention(pq, prepared.keys, prepared.values)


class DenseLongSequenceB200(_LongSequenceMixin, SageAttentionB200):
    """Dense backend with the long-sequence protocol (role of
    DenseLongSequenceAttentionBackend, model/kernels.py:5441-5619): every query
    chunk, prefix or video, runs with per-warp Q scales over all keys."""

    def __init__(self, smooth_k: bool = True) -> None:
        super().__init__(smooth_k=smooth_k, qk_quant_gran="per_warp")

    def long_sequence_all_queries(self, query: torch.Tensor, prepared: PreparedLongSequenceKVB200) -> torch.Tensor:
        """Every query of the packed sequence, in chunks from its origin (model/layers.py:852-860)."""
        return self.long_sequence_prefix_queries(query, prepared)

    def long_sequence_video_queries(self, query, prepared, *, protected_tokens=0, query_token_indices=None):
        return self.long_sequence_prefix_queries(query, prepared)


class SpargeLongSequenceB200(_LongSequenceMixin, SpargeAttentionB200):
    """Sparge backend with the long-sequence protocol (role of
    SplitModalityProtectedSpargeAttentionBackend, model/kernels.py:2775-4000):
    prefix queries run dense; each chunk of video queries is pooled and selected
    against the prepared keys, the protected prefix keys stay dense, and the
    temporal rail (when configured and the request's video layout covers the key
    sequence after the prefix) centres each query block on its position in the
    video, recovered from the chunk's token indices."""

    smooth_k = True

    def long_sequence_video_queries(self, query, prepared, *, protected_tokens=0, query_token_indices=None):
        q = _as_lhd(query, "Query")
        self._check_query(q, prepared)
        if query_token_indices is not None and (
                query_token_indices.ndim != 1 or query_token_indices.numel() != q.shape[0]
                or query_token_indices.device != q.device):
            raise ValueError("long-sequence Query indices must align with the chunk")
        pq = prepare_queries(q, 128, self.similarity_threshold)
        cfg = replace(self.mask, protected_tokens=int(protected_tokens))
        cfg = self._temporal(cfg, prepared.key_tokens, int(protected_tokens), q.shape[0],
                             query_token_indices is not None)
        idx = query_token_indices if cfg.temporal_radius >= 0 else None
        bitmap = block_mask(pq, prepared.keys, cfg, query_indices=idx)
        return attention(pq, prepared.keys, prepared.values, bitmap)
