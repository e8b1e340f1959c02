"""An H3-shaped DiT block on the B200 kernels (the benchmark's unit of work).

Per block (model/layers.py:1074-1298, fused_mlp.py:269-426):
  adaln(t) -> shift/scale/gate x 2           h3b_adaln_projection (one GEMV per step)
  xq = rms_adaln + ConvRot + INT8(x)          h3b_rms_adaln_quantize_int8
  qkv = INT8 GEMM(xq, W_qkv) + bias, with    h3b_int8_gemm_dequant_qk_rope (one kernel;
    q, k <- per-head RMSNorm + 3-D RoPE       h3b_int8_gemm_dequant + h3b_qk_rmsnorm_rope
    in the epilogue                           for shapes the fused epilogue does not take)
  [Ulysses all-to-all tokens -> heads]        NCCL, only when world > 1: K, V, Q as
                                              three async exchanges overlapping the K / V prep
  attention (Sparge-masked quantized)         prep / mask / h3b_attention
  [all-to-all heads -> tokens]
  x += gate_a * INT8 GEMM(ConvRot INT8(o))    h3b_quantize_int8_rowwise_convrot + gated-residual GEMM
  xq = rms_adaln + ConvRot + INT8(x)
  h = W4A8 GEMM(xq, W_fc1) + bias,            h3b_dequant_int4_grouped_to_int8 +
    gelu + ConvRot in the epilogue            h3b_int8_gemm_gelu_convrot, then
  hq = INT8(h)                                h3b_quantize_rotated_int8 (swiglu, or
                                              shapes the fused epilogue does not take:
                                              GEMM + h3b_quantize_int8_rowwise_convrot)
  x += gate_m * W4A8 GEMM(hq, W_fc2)          gated-residual GEMM

Weights are random-initialised with the checkpoint formats the reference loads
(per-output-channel INT8, grouped packed INT4 with fp32 s_rel and s_channel).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import attention as A
from . import ops
from . import parallel as P
from . import quantization as Q


@dataclass
class BlockConfig:
    hidden: int = 4096
    heads: int = 32
    head_dim: int = 128
    ffn: int = 16384
    mlp_act: str = "gelu_tanh"       # "gelu_tanh" (the benchmark block) or "swiglu" (real H3: fc1 out = 2*ffn)
    w4_group: int = 128
    convrot: int = 256
    eps: float = 1e-5
    qk_eps: float = 1e-6
    rope_splits: tuple[int, int, int] = (44, 42, 42)
    t_dim: int = 4096
    mask: A.MaskConfig | None = field(
        default_factory=lambda: A.MaskConfig("cdf", 0.6, keep_first_column=True, keep_diagonal=True))


def _int8_per_channel(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    amax = w.abs().amax(dim=1).clamp_min(1e-12)
    scale = amax / 127.0
    q = torch.clamp(torch.round(w / scale[:, None]), -127, 127).to(torch.int8)
    return q, scale.float()


def _int4_grouped(w: torch.Tensor, group: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Symmetric int4 groups -> (packed [N, K/2] int8, s_rel f32 [N, K/G], s_channel f32 [N])."""
    N, K = w.shape
    wg = w.view(N, K // group, group)
    gscale = (wg.abs().amax(-1) / 7.0).clamp_min(1e-12)
    cscale = gscale.amax(-1) / 127.0
    codes = torch.clamp(torch.round(wg / gscale.unsqueeze(-1)), -8, 7).to(torch.int32) + 8
    codes = codes.view(N, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)
    return packed.contiguous(), (gscale / cscale.unsqueeze(-1)).float().contiguous(), cscale.float().contiguous()


def _runs(segments, rows: int, table_rows: int):
    """Validated AdaLN runs ((start, stop, row), ...) or None for row 0 everywhere."""
    if segments is None:
        return None
    runs, prev = [], 0
    for start, stop, row in segments:
        start, stop, row = int(start), int(stop), int(row)
        if start != prev or stop <= start:
            raise ValueError("modulation segments must be an ordered partition")
        if not 0 <= row < table_rows:
            raise ValueError(f"modulation row {row} outside the {table_rows} AdaLN rows")
        runs.append((start, stop, row))
        prev = stop
    if prev != rows:
        raise ValueError("modulation segments do not cover the packed sequence")
    return runs


def _chunk_segments(segments, r0: int, r1: int):
    """AdaLN runs restricted to rows [r0, r1), in chunk-relative rows (None stays None)."""
    if segments is None:
        return None
    out = []
    for start, stop, row in segments:
        a, b = max(int(start), r0), min(int(stop), r1)
        if a < b:
            out.append((a - r0, b - r0, int(row)))
    return tuple(out)


def rope_tables_from_frequencies(frequencies: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) bf16 [L, rot/2] tables from the engine's RoPE input: split-half angles
    [L, rot] (model/layers.py:51-57) or the packed rotation table [1, L, 1, rot/2, 2, 2]
    (model/layers.py:60-69).  The angle form takes cos/sin in fp32 and rounds to bf16,
    as the engine's unfused path does (model/layers.py:137-140)."""
    if frequencies.dim() == 6:
        table = frequencies[0, :, 0]
        return table[..., 0, 0].to(torch.bfloat16).contiguous(), table[..., 1, 0].to(torch.bfloat16).contiguous()
    if frequencies.dim() != 2 or frequencies.shape[1] % 2:
        raise ValueError("frequencies must be angles [L, rot] or a rotation table [1, L, 1, rot/2, 2, 2]")
    half = frequencies.shape[1] // 2
    active = frequencies[:, :half].float()
    return torch.cos(active).to(torch.bfloat16).contiguous(), torch.sin(active).to(torch.bfloat16).contiguous()


def rope_tables(grid: tuple[int, int, int], splits=(44, 42, 42), theta: float = 10000.0, start: int = 0,
                count: int | None = None, device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """Split-half 3-D RoPE tables (cos, sin) bf16 [L, sum(splits)/2] for a (t, h, w)
    token grid (model/layers.py:51-70)."""
    T, Hh, W = grid
    L = T * Hh * W
    count = L - start if count is None else count
    idx = torch.arange(start, start + count, device=device)
    pos = torch.stack((idx // (Hh * W), (idx // W) % Hh, idx % W), dim=1).float()
    halves = []
    for axis, width in enumerate(splits):
        inv = 1.0 / (theta ** (torch.arange(0, width, 2, device=device).float() / width))
        halves.append(pos[:, axis:axis + 1] * inv[None, :])
    ang = torch.cat(halves, dim=1)
    return ang.cos().to(torch.bfloat16).contiguous(), ang.sin().to(torch.bfloat16).contiguous()


class DiTBlockB200:
    """One DiT block on one GPU (or one Ulysses rank).

    The four projections are `h3b.quantization` layers (INT8 or packed W4A8, chosen per
    layer as the checkpoint records); `DiTBlockB200(cfg)` random-initialises them in the
    benchmark block's formats (INT8 attention projections, W4A8 MLP) and
    `h3b.checkpoint.load_block` assembles them from a checkpoint."""

    def __init__(self, cfg: BlockConfig, device="cuda", seed: int = 0, group=None):
        self._setup(cfg, device, group)
        g = torch.Generator(device=self.device).manual_seed(seed)
        D, F, W = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim

        def randn(*shape, std=1.0):
            return torch.randn(*shape, generator=g, device=self.device) * std

        # AdaLN projection t -> 6 * hidden (shift/scale/gate for attention and MLP)
        self.ada_w = randn(6 * D, cfg.t_dim, std=0.02).to(torch.bfloat16)
        self.ada_b = randn(6 * D, std=0.02).to(torch.bfloat16)
        self.norm1 = (1 + randn(D, std=0.05)).to(torch.bfloat16)
        self.norm2 = (1 + randn(D, std=0.05)).to(torch.bfloat16)
        self.q_norm = (1 + randn(cfg.head_dim, std=0.05)).to(torch.bfloat16)
        self.k_norm = (1 + randn(cfg.head_dim, std=0.05)).to(torch.bfloat16)
        # INT8 linears (ConvRot weights are stored rotated; random weights stand in)
        int8 = Q.ComfyQuantSpec("int8_tensorwise", convrot=bool(cfg.convrot), convrot_groupsize=256)
        w, s = _int8_per_channel(randn(3 * W, D, std=0.02))
        self.qkv = Q.Int8Linear(w, s, randn(3 * W, std=0.01).to(torch.bfloat16), spec=int8)
        w, s = _int8_per_channel(randn(D, W, std=0.02))
        self.out = Q.Int8Linear(w, s, randn(D, std=0.01).to(torch.bfloat16), spec=int8)
        w4 = Q.W4A8QuantSpec("asym_w4a8_int8", group_size=cfg.w4_group)
        fc1_out = 2 * F if cfg.mlp_act == "swiglu" else F
        qd, sr, sc = _int4_grouped(randn(fc1_out, D, std=0.02), cfg.w4_group)
        self.fc1 = Q.W4A8Linear(qd, sr, sc, bias=randn(fc1_out, std=0.01).to(torch.bfloat16), spec=w4)
        qd, sr, sc = _int4_grouped(randn(D, F, std=0.02), cfg.w4_group)
        self.fc2 = Q.W4A8Linear(qd, sr, sc, bias=randn(D, std=0.01).to(torch.bfloat16), spec=w4)

    def _setup(self, cfg: BlockConfig, device, group) -> None:
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        self.world = torch.distributed.get_world_size(group) if group is not None else 1
        if cfg.heads % self.world:
            raise ValueError(f"{cfg.heads} heads do not split over {self.world} ranks")
        self.last_mask_density: float | None = None
        self.head_order: torch.Tensor | None = None   # Ulysses head -> rank assignment (None: in order)

    @classmethod
    def from_parts(cls, cfg: BlockConfig, *, ada_w, ada_b, norm1, norm2, q_norm, k_norm, qkv, out, fc1, fc2,
                   device="cuda", group=None) -> "DiTBlockB200":
        """A block over given weights (bf16 vectors / AdaLN projection, quantization layers)."""
        blk = cls.__new__(cls)
        blk._setup(cfg, device, group)
        blk.ada_w = ada_w.to(torch.bfloat16).contiguous()
        blk.ada_b = None if ada_b is None else ada_b.to(torch.bfloat16).contiguous()
        blk.norm1, blk.norm2, blk.q_norm, blk.k_norm = norm1, norm2, q_norm, k_norm
        blk.qkv, blk.out, blk.fc1, blk.fc2 = qkv, out, fc1, fc2
        W = cfg.heads * cfg.head_dim
        fc1_out = 2 * cfg.ffn if cfg.mlp_act == "swiglu" else cfg.ffn
        shapes = {"qkv": (qkv, 3 * W, cfg.hidden), "out": (out, cfg.hidden, W), "fc1": (fc1, fc1_out, cfg.hidden),
                  "fc2": (fc2, cfg.hidden, cfg.ffn)}
        for name, (lin, n, k) in shapes.items():
            if (lin.out_features, lin.in_features) != (n, k):
                raise ValueError(f"{name} is [{lin.out_features}, {lin.in_features}], the config needs [{n}, {k}]")
        if ada_w.shape[0] % (6 * cfg.hidden) or ada_w.shape[1] != cfg.t_dim:
            raise ValueError("the AdaLN projection must map t_dim to a multiple of 6 * hidden")
        if fc2.convrot_group_size == 0 and cfg.mlp_act:
            raise ValueError("the FC2 input activation is fused only into the ConvRot quantizer")
        return blk

    # ------------------------------------------------------------------ stages
    def modulation(self, t: torch.Tensor) -> torch.Tensor:
        """AdaLN parameters [R, 6, hidden] (shift_a, scale_a, gate_a, shift_m, scale_m, gate_m)
        from the projection input t [t_dim] or [rows, t_dim].  A projection to 18 * hidden
        (the H3 checkpoints) gives three modulation rows per input row, selected by
        `segments` (model/layers.py:910-913)."""
        out = ops.adaln_projection(self.ada_w, self.ada_b, t.to(self.device))
        return out.reshape(-1, 6, self.cfg.hidden)

    def attention(self, qkv_heads: torch.Tensor) -> torch.Tensor:
        """qkv_heads: [L, 3*h*128] -> o [L, h, 128] (h heads of this rank)."""
        cfg = self.cfg
        L = qkv_heads.shape[0]
        h = qkv_heads.shape[1] // (3 * cfg.head_dim)
        view = qkv_heads.view(L, 3, h, cfg.head_dim)
        q, k, v = view[:, 0], view[:, 1], view[:, 2]
        # the three preparations are independent and none fills the GPU alone: V and Q
        # run on side streams while K (mean, pooling, INT8) runs on the current stream
        main = torch.cuda.current_stream(self.device)
        side = self._side_streams()
        for st in side:
            st.wait_stream(main)
        with torch.cuda.stream(side[0]):
            pv = A.prepare_values(v)
        with torch.cuda.stream(side[1]):
            pq = A.prepare_queries(q)
        pk, _ = A.prepare_keys(k)
        main.wait_stream(side[1])
        _used_on(main, pq.pooled, pq.similar, pq.qi8, pq.scale)
        bitmap = A.block_mask(pq, pk, cfg.mask) if cfg.mask is not None else None
        main.wait_stream(side[0])
        _used_on(main, pv.vt, pv.scale)
        self._last_attn = (pq, pk, pv, bitmap)
        return A.attention(pq, pk, pv, bitmap)

    def _side_streams(self) -> tuple[torch.cuda.Stream, torch.cuda.Stream]:
        streams = getattr(self, "_streams", None)
        if streams is None:
            streams = (torch.cuda.Stream(device=self.device), torch.cuda.Stream(device=self.device))
            self._streams = streams
        return streams

    def attention_ulysses(self, qkv: torch.Tensor) -> torch.Tensor:
        """qkv: this rank's token rows [L/P, 3*H*128] -> o [L, H/P, 128] for this rank's
        heads.  K, V and Q cross NVLink as three asynchronous all-to-alls; the K
        preparation starts when K has arrived, while V and Q are still in flight."""
        cfg = self.cfg
        ex = P.exchange_qkv_async(qkv, cfg.heads, cfg.head_dim, self.group, self.head_order)
        k, work = ex["k"]
        work.wait()
        pk, _ = A.prepare_keys(k)
        v, work = ex["v"]
        work.wait()
        pv = A.prepare_values(v)
        q, work = ex["q"]
        work.wait()
        pq = A.prepare_queries(q)
        bitmap = A.block_mask(pq, pk, cfg.mask) if cfg.mask is not None else None
        self._last_attn = (pq, pk, pv, bitmap)
        return A.attention(pq, pk, pv, bitmap)

    def rebalance_heads(self) -> torch.Tensor | None:
        """Reassign heads to ranks so each rank's Sparge work (kept tiles of the last
        forward) is nearly equal; every rank computes the same order.  Collective:
        call on all ranks between forwards.  The block's output does not depend on
        the assignment."""
        if self.world == 1 or getattr(self, "_last_attn", None) is None:
            return self.head_order
        pq, pk, _, bitmap = self._last_attn
        hl = pq.qi8.shape[0]
        if bitmap is None:
            local = torch.full((hl,), float(pq.qi8.shape[1] // 128), device=self.device)
        else:
            local = kept_tiles_per_head(bitmap).to(torch.float64)
        counts = P.gather_head_counts(local, self.head_order, self.cfg.heads, self.group)
        self.head_order = P.balanced_head_order(counts, self.world)
        return self.head_order

    @staticmethod
    def _gated(lin, x, gate, q, s, runs) -> None:
        if runs is None:
            lin.gated_residual_(x, gate[0], q, s)
            return
        for start, stop, row in runs:
            lin.gated_residual_(x[start:stop], gate[row], q[start:stop], s[start:stop])

    def forward(self, x: torch.Tensor, t: torch.Tensor, rope: tuple[torch.Tensor, torch.Tensor],
                segments=None, *, chunks=None, rows_ready=None, rows_done=None) -> torch.Tensor:
        """x: bf16 [L_local, hidden] (updated in place and returned); rope: tables for these
        tokens; segments: AdaLN runs ((start, stop, row), ...) over x's rows, or None for
        modulation row 0 everywhere (model/layers.py:916-960).

        chunks: row boundaries [0, b1, ..., L_local] for the row-local phases (RMSNorm +
        AdaLN + QKV + q/k RoPE before the attention; RMSNorm + AdaLN + MLP + gated residual
        after it), which then run chunk by chunk.  rows_ready(i) is called before chunk i's
        rows are first read, rows_done(i) once its final values are enqueued; a host pipeline
        uses them to overlap row copies with the neighbouring chunks' work.  Every operation
        of these phases is row-local, so the result does not depend on the chunking."""
        cfg = self.cfg
        mod = self.modulation(t)
        shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = mod.unbind(1)
        Lp = x.shape[0]
        runs = _runs(segments, Lp, mod.shape[0])
        bounds = [0, Lp] if chunks is None else [int(b) for b in chunks]
        if bounds[0] != 0 or bounds[-1] != Lp or any(b1 <= b0 for b0, b1 in zip(bounds, bounds[1:])):
            raise ValueError("chunks must be increasing row boundaries from 0 to the row count")
        W = cfg.heads * cfg.head_dim
        qkv = torch.empty((Lp, 3 * W), device=x.device, dtype=torch.bfloat16)
        for i, (r0, r1) in enumerate(zip(bounds, bounds[1:])):
            if rows_ready is not None:
                rows_ready(i)
            seg_i = _chunk_segments(segments, r0, r1)
            xq, xs = ops.rms_adaln_quantize_int8(x[r0:r1], self.norm1, scale_a, shift_a, seg_i, cfg.eps,
                                                 self.qkv.convrot_group_size)
            self.qkv.forward_prequantized_qk_rope(xq, xs, qkv[r0:r1], cfg.heads, 0, W, self.q_norm, self.k_norm,
                                                  rope[0][r0:r1], rope[1][r0:r1], cfg.qk_eps)
        if self.world > 1:
            o = self.attention_ulysses(qkv)
            o2 = P.heads_to_tokens(o.view(o.shape[0], -1), Lp, self.group, self.head_order)
        else:
            o2 = self.attention(qkv).view(Lp, W)
        del qkv
        oq, os_ = self.out.quantize(o2)
        self._gated(self.out, x, gate_a, oq, os_, runs)
        del oq, os_, o2
        for i, (r0, r1) in enumerate(zip(bounds, bounds[1:])):
            seg_i = _chunk_segments(segments, r0, r1)
            xq, xs = ops.rms_adaln_quantize_int8(x[r0:r1], self.norm2, scale_m, shift_m, seg_i, cfg.eps,
                                                 self.fc1.convrot_group_size)
            hq, hs = self.fc1.forward_prequantized_for(self.fc2, xq, xs, cfg.mlp_act)
            self._gated(self.fc2, x[r0:r1], gate_m, hq, hs, _runs(seg_i, r1 - r0, mod.shape[0]))
            if rows_done is not None:
                rows_done(i)
        return x

    # ------------------------------------------------------------------ accounting
    def linear_ops(self, tokens: int) -> float:
        cfg = self.cfg
        W = cfg.heads * cfg.head_dim
        fc1_out = 2 * cfg.ffn if cfg.mlp_act == "swiglu" else cfg.ffn
        return 2.0 * tokens * (cfg.hidden * (3 * W + fc1_out) + W * cfg.hidden + cfg.ffn * cfg.hidden)


class HostPipeline:
    """Runs a block over a series of host-resident inputs with the copies hidden.

    Each step copies its hidden states (and timestep vector) from pinned host
    memory to the GPU, runs the block and copies the result back.  The copies run
    on their own streams: the host->device copy of step k + 1 and the
    device->host copy of step k - 1 overlap the block of step k (two device
    buffers; a buffer is refilled only after the result it held has been read
    out).  The first step's input arrives in `chunks` row chunks, and its block
    starts on the first chunk while the rest copy; the last step's output leaves in
    row chunks as the block finishes each one (the block's row-local phases run
    chunk by chunk there).  All ordering is by CUDA events; nothing waits on the host.
    """

    def __init__(self, block: DiTBlockB200, rope: tuple[torch.Tensor, torch.Tensor], tokens: int, chunks: int = 8):
        dev = block.device
        self.block, self.rope = block, rope
        self.x = [torch.empty((tokens, block.cfg.hidden), device=dev, dtype=torch.bfloat16) for _ in range(2)]
        self.t = [torch.empty((block.cfg.t_dim,), device=dev, dtype=torch.bfloat16) for _ in range(2)]
        self.s_in = torch.cuda.Stream(device=dev)
        self.s_out = torch.cuda.Stream(device=dev)
        n = max(1, min(int(chunks), tokens))
        self.bounds = [tokens * i // n for i in range(n + 1)]

    def run(self, xs_host: list[torch.Tensor], ts_host: list[torch.Tensor], outs_host: list[torch.Tensor]) -> None:
        """xs_host[k] / ts_host[k] (pinned, bf16) -> outs_host[k] (pinned, bf16), for every k.

        Enqueued on the current stream's timeline: the copies start after the work
        already on the current stream, and the current stream waits for the last
        device->host copy, so synchronizing it (or an event recorded on it after
        this call) makes every output available on the host."""
        n = len(xs_host)
        if not (len(ts_host) == n == len(outs_host)):
            raise ValueError("xs_host, ts_host and outs_host must have the same length")
        comp = torch.cuda.current_stream(self.block.device)
        self.s_in.wait_stream(comp)
        self.s_out.wait_stream(comp)
        whole = [0, self.bounds[-1]]
        loaded: list[list[torch.cuda.Event] | None] = [None] * n   # [t copied, row chunk 0, 1, ...]
        read_out: list[torch.cuda.Event | None] = [None, None]

        def record(stream) -> torch.cuda.Event:
            ev = torch.cuda.Event()
            ev.record(stream)
            return ev

        def load(k: int) -> None:
            b = k % 2
            bounds = self.bounds if k == 0 else whole
            with torch.cuda.stream(self.s_in):
                if read_out[b] is not None:
                    self.s_in.wait_event(read_out[b])
                self.t[b].copy_(ts_host[k], non_blocking=True)
                evs = [record(self.s_in)]
                for r0, r1 in zip(bounds, bounds[1:]):
                    self.x[b][r0:r1].copy_(xs_host[k][r0:r1], non_blocking=True)
                    evs.append(record(self.s_in))
                loaded[k] = evs

        def store(k: int, r0: int, r1: int) -> torch.cuda.Event:
            done = record(comp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(done)
                outs_host[k][r0:r1].copy_(self.x[k % 2][r0:r1], non_blocking=True)
                return record(self.s_out)

        if n:
            load(0)
        for k in range(n):
            if k + 1 < n:
                load(k + 1)
            b = k % 2
            comp.wait_event(loaded[k][0])
            first, last = k == 0, k == n - 1
            if not (first or last):
                comp.wait_event(loaded[k][1])
                self.block.forward(self.x[b], self.t[b], self.rope)
                read_out[b] = store(k, 0, whole[1])
                continue
            bounds = self.bounds
            in_evs = loaded[k][1:]
            outs: list[torch.cuda.Event] = []

            def ready(i: int, k=k, in_evs=in_evs, bounds=bounds) -> None:
                # chunk i of this step's rows: the copy that holds them has landed
                if len(in_evs) == 1:
                    if i == 0:
                        comp.wait_event(in_evs[0])
                else:
                    comp.wait_event(in_evs[i])

            def done(i: int, k=k, bounds=bounds) -> None:
                if last:
                    outs.append(store(k, bounds[i], bounds[i + 1]))

            self.block.forward(self.x[b], self.t[b], self.rope, chunks=bounds, rows_ready=ready, rows_done=done)
            if last:
                read_out[b] = outs[-1]
            else:
                read_out[b] = store(k, 0, whole[1])
        comp.wait_stream(self.s_out)


def _used_on(stream: torch.cuda.Stream, *tensors: torch.Tensor | None) -> None:
    """Tensors made on a side stream and consumed on `stream`: their memory is not
    reused before `stream`'s work up to this point is done."""
    for t in tensors:
        if t is not None:
            t.record_stream(stream)


def kept_tiles_per_head(bitmap: torch.Tensor) -> torch.Tensor:
    """Kept (Q block, K block) tiles of each head, int64 [H] on the bitmap's device."""
    v = bitmap.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    cnt = torch.zeros(v.shape[0], dtype=torch.int64, device=v.device)
    for _ in range(32):
        cnt += (v & 1).sum(dim=(1, 2))
        v = v >> 1
    return cnt


def kept_tiles(bitmap: torch.Tensor, key_tokens: int) -> int:
    """Number of kept (Q block, K block) tiles in a bitmap (bits beyond Kb are zero)."""
    b = bitmap.view(torch.int32)
    cnt = torch.zeros_like(b)
    v = b.clone()
    for _ in range(32):
        cnt += v & 1
        v = v >> 1
        v &= 0x7FFFFFFF
    return int(cnt.sum().item())


def attention_ops(bitmap: torch.Tensor | None, Lq: int, Lk: int, heads: int) -> float:
    """Executed tensor ops of the attention: 4 * 128 * 64 * 128 per kept 128x64 tile
    (QK^T and PV); dense when bitmap is None (exactly 4*Lq*Lk*H*D over the padded tiles)."""
    per_tile = 4.0 * 128 * 64 * 128
    if bitmap is None:
        return per_tile * math.ceil(Lq / 128) * math.ceil(Lk / 64) * heads
    return per_tile * kept_tiles(bitmap, Lk)
