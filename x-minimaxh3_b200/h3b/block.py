"""An H3-shaped DiT block on the B200 kernels (the benchmark's unit of work).

Per block (model/layers.py:1074-1298, fused_mlp.py:269-426):
  adaln(t) -> shift/scale/gate x 2           (torch matmul; one GEMV per step)
  xq = rms_adaln + ConvRot + INT8(x)          h3b_rms_adaln_quantize_int8
  qkv = INT8 GEMM(xq, W_qkv) + bias           h3b_int8_gemm_dequant
  q, k <- per-head RMSNorm + 3-D RoPE         h3b_qk_rmsnorm_rope
  [Ulysses all-to-all tokens -> heads]        NCCL, only when world > 1
  attention (Sparge-masked quantized)         prep / mask / h3b_attention
  [all-to-all heads -> tokens]
  x += gate_a * INT8 GEMM(ConvRot INT8(o))    h3b_quantize_int8_rowwise_convrot + gated-residual GEMM
  xq = rms_adaln + ConvRot + INT8(x)
  h = W4A8 GEMM(xq, W_fc1) + bias             h3b_dequant_int4_grouped_to_int8 + GEMM
  x += gate_m * W4A8 GEMM(gelu/swiglu + ConvRot INT8(h), W_fc2)

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


@dataclass
class BlockConfig:
    hidden: int = 4096
    heads: int = 32
    head_dim: int = 128
    ffn: int = 16384
    mlp_act: str = "gelu_tanh"       # "gelu_tanh" (BASELINE) or "swiglu" (real H3: fc1 out = 2*ffn)
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
    """One DiT block with random-init H3-format weights on one GPU (or one Ulysses rank)."""

    def __init__(self, cfg: BlockConfig, device="cuda", seed: int = 0, group=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        self.world = torch.distributed.get_world_size(group) if group is not None else 1
        if cfg.heads % self.world:
            raise ValueError(f"{cfg.heads} heads do not split over {self.world} ranks")
        g = torch.Generator(device=self.device).manual_seed(seed)
        D, F = cfg.hidden, cfg.ffn

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
        self.w_qkv, self.s_qkv = _int8_per_channel(randn(3 * D, D, std=0.02))
        self.b_qkv = randn(3 * D, std=0.01).to(torch.bfloat16)
        self.w_o, self.s_o = _int8_per_channel(randn(D, D, std=0.02))
        self.b_o = randn(D, std=0.01).to(torch.bfloat16)
        fc1_out = 2 * F if cfg.mlp_act == "swiglu" else F
        self.fc1 = _int4_grouped(randn(fc1_out, D, std=0.02), cfg.w4_group)
        self.b_fc1 = randn(fc1_out, std=0.01).to(torch.bfloat16)
        self.fc2 = _int4_grouped(randn(D, F, std=0.02), cfg.w4_group)
        self.b_fc2 = randn(D, std=0.01).to(torch.bfloat16)
        self.last_mask_density: float | None = None

    # ------------------------------------------------------------------ stages
    def modulation(self, t: torch.Tensor) -> torch.Tensor:
        tv = t.float().reshape(-1).to(self.device)
        return (torch.mv(self.ada_w.float(), tv) + self.ada_b.float()).reshape(6, -1).to(torch.bfloat16)

    def attention(self, qkv_heads: torch.Tensor) -> torch.Tensor:
        """qkv_heads: [L, 3*h*128] -> o [L, h, 128] (h heads of this rank)."""
        cfg = self.cfg
        L = qkv_heads.shape[0]
        h = qkv_heads.shape[1] // (3 * cfg.head_dim)
        view = qkv_heads.view(L, 3, h, cfg.head_dim)
        q, k, v = view[:, 0], view[:, 1], view[:, 2]
        pv = A.prepare_values(v)
        pk, _ = A.prepare_keys(k)
        pq = A.prepare_queries(q)
        bitmap = A.block_mask(pq, pk, cfg.mask) if cfg.mask is not None else None
        self._last_attn = (pq, pk, pv, bitmap)
        return A.attention(pq, pk, pv, bitmap)

    def forward(self, x: torch.Tensor, t: torch.Tensor, rope: tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
        """x: bf16 [L_local, hidden] (updated in place and returned); rope: tables for these tokens."""
        cfg = self.cfg
        D = cfg.hidden
        mod = self.modulation(t)
        shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = mod.unbind(0)
        xq, xs = ops.rms_adaln_quantize_int8(x, self.norm1, scale_a, shift_a, None, cfg.eps, cfg.convrot)
        qkv = ops.int8_linear_prequantized(xq, xs, self.w_qkv, self.s_qkv, self.b_qkv)
        ops.qk_rmsnorm_rope_(qkv, cfg.heads, 0, D, self.q_norm, self.k_norm, rope[0], rope[1], cfg.qk_eps)
        Lp = x.shape[0]
        if self.world > 1:
            o = self.attention(P.tokens_to_heads(qkv, cfg.heads, cfg.head_dim, self.group))
            o2 = P.heads_to_tokens(o.view(o.shape[0], -1), Lp, self.group)
        else:
            o2 = self.attention(qkv).view(Lp, D)
        oq, os_ = ops.quantize_int8_rowwise_convrot64(o2, cfg.convrot)
        ops.int8_linear_gated_residual_(x, gate_a, oq, os_, self.w_o, self.s_o, self.b_o)
        xq, xs = ops.rms_adaln_quantize_int8(x, self.norm2, scale_m, shift_m, None, cfg.eps, cfg.convrot)
        w1 = ops.dequant_int4_grouped_to_int8(self.fc1[0], self.fc1[1], None, cfg.w4_group)
        h = ops.int8_linear_prequantized(xq, xs, w1, self.fc1[2], self.b_fc1)
        hq, hs = ops.quantize_int8_rowwise_convrot64(h, cfg.convrot, cfg.mlp_act)
        w2 = ops.dequant_int4_grouped_to_int8(self.fc2[0], self.fc2[1], None, cfg.w4_group)
        ops.int8_linear_gated_residual_(x, gate_m, hq, hs, w2, self.fc2[2], self.b_fc2)
        return x

    # ------------------------------------------------------------------ accounting
    def linear_ops(self, tokens: int) -> float:
        cfg = self.cfg
        fc1_out = 2 * cfg.ffn if cfg.mlp_act == "swiglu" else cfg.ffn
        return 2.0 * tokens * cfg.hidden * (3 * cfg.hidden + cfg.hidden + fc1_out + cfg.ffn)


class HostPipeline:
    """Runs a block over a series of host-resident inputs with the copies hidden.

    Each step copies its hidden states (and timestep vector) from pinned host
    memory to the GPU, runs the block and copies the result back.  The copies run
    on their own streams: the host->device copy of step k + 1 and the
    device->host copy of step k - 1 overlap the block of step k (two device
    buffers; a buffer is refilled only after the result it held has been read
    out).  All ordering is by CUDA events; nothing waits on the host.
    """

    def __init__(self, block: DiTBlockB200, rope: tuple[torch.Tensor, torch.Tensor], tokens: int):
        dev = block.device
        self.block, self.rope = block, rope
        self.x = [torch.empty((tokens, block.cfg.hidden), device=dev, dtype=torch.bfloat16) for _ in range(2)]
        self.t = [torch.empty((block.cfg.t_dim,), device=dev, dtype=torch.bfloat16) for _ in range(2)]
        self.s_in = torch.cuda.Stream(device=dev)
        self.s_out = torch.cuda.Stream(device=dev)

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
        loaded: list[torch.cuda.Event | None] = [None] * n
        read_out: list[torch.cuda.Event | None] = [None, None]

        def load(k: int) -> None:
            b = k % 2
            with torch.cuda.stream(self.s_in):
                if read_out[b] is not None:
                    self.s_in.wait_event(read_out[b])
                self.x[b].copy_(xs_host[k], non_blocking=True)
                self.t[b].copy_(ts_host[k], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.s_in)
                loaded[k] = ev

        if n:
            load(0)
        for k in range(n):
            if k + 1 < n:
                load(k + 1)
            b = k % 2
            comp.wait_event(loaded[k])
            self.block.forward(self.x[b], self.t[b], self.rope)
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(done)
                outs_host[k].copy_(self.x[b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.s_out)
                read_out[b] = ev
        comp.wait_stream(self.s_out)


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
