"""CPU port of the reference's own CPU path for one DiT block (test infrastructure).

Used only by bench.py (its cpu_baseline leg and `--impl reference`).  It
restates, with torch CPU ops and all host threads, the computations the
X-MinimaxH3 modules run when no CUDA kernel is injected:

  ConvRotInt8Linear CPU path    groupwise_hadamard(x.float()) then F.linear with
                                qweight.float() * scale           (model/quantization.py:190-207, 295-304)
  ConvRotW4A8Linear CPU path    _reference_weight decode + F.linear (quantization.py:486-516, 557-586)
  rms_adaln (eager order)       F.rms_norm, * bf16(1+scale), + shift (layers.py:33-48, 916-941)
  attention                     torch_sdpa (layers.py:245-250)
  gated residual                residual.addcmul_(update, gate) (layers.py:944-960)

A full block at 720p/5 s is hours of CPU time, so each measurement runs a
bounded sample (the weight dequantizations, a slice of token rows through every
linear, and a slice of query rows of one head against all keys) and
extrapolates linearly to the whole block; results are labelled as extrapolated.
The reference's CPU attention is dense; the B200 arm's is Sparge-masked.
"""

from __future__ import annotations

import math
import os
import time

import torch
import torch.nn.functional as F


def hadamard256(device="cpu") -> torch.Tensor:
    h4 = torch.tensor(((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1)), dtype=torch.float32)
    m = h4
    while m.shape[0] < 256:
        m = torch.kron(m, h4)
    return (m / 16.0).to(device)


def groupwise_hadamard(x: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    g = h.shape[0]
    return torch.matmul(x.reshape(-1, x.shape[-1] // g, g), h).reshape_as(x)


class ReferenceBlockCPU:
    """Random-init weights kept in the reference's stored formats (INT8 + scale, packed
    W4 codes + s_rel + s_channel) and dequantized on every call, as the reference's CPU
    fallbacks do (model/quantization.py:295-304, 486-516)."""

    def __init__(self, hidden=4096, heads=32, ffn=16384, group=128, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.hidden, self.heads, self.ffn, self.group = hidden, heads, ffn, group
        self.h = hadamard256()

        def int8w(n, k):
            q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8)
            return q, torch.rand(n, generator=g) * 2e-4

        def w4(n, k):
            return (torch.randint(0, 16, (n, k), generator=g, dtype=torch.int16).to(torch.int8),
                    torch.rand(n, k // group, generator=g) * 20 + 1, torch.rand(n, generator=g) * 1e-4)

        self.w_qkv = int8w(3 * hidden, hidden)
        self.w_o = int8w(hidden, hidden)
        self.w_fc1 = w4(ffn, hidden)
        self.w_fc2 = w4(hidden, ffn)
        self.b_qkv = torch.randn(3 * hidden, generator=g) * 0.01
        self.b_o = torch.randn(hidden, generator=g) * 0.01
        self.b_fc1 = torch.randn(ffn, generator=g) * 0.01
        self.b_fc2 = torch.randn(hidden, generator=g) * 0.01
        self.norm = torch.ones(hidden, dtype=torch.bfloat16)
        self.mod = (torch.randn(6, hidden, generator=g) * 0.1).to(torch.bfloat16)

    def dequant_int8(self, w):
        q, s = w
        return q.float() * s.reshape(-1, 1)

    def dequant_w4(self, w):
        codes, s_rel, s_ch = w
        n, k = codes.shape
        grid = ((codes.float() - 8.0).view(n, k // self.group, self.group) * s_rel.unsqueeze(-1)).round().clamp_(-127, 127)
        return (grid * s_ch.view(-1, 1, 1)).reshape(n, k)

    def dequant_all(self):
        return (self.dequant_int8(self.w_qkv), self.dequant_int8(self.w_o), self.dequant_w4(self.w_fc1),
                self.dequant_w4(self.w_fc2))

    def _rms_adaln(self, x, shift, scale):
        h = F.rms_norm(x, (x.shape[-1],), weight=self.norm, eps=1e-5)
        return h.mul_(1.0 + scale).add_(shift)

    def _linear(self, x, w, b):
        return F.linear(groupwise_hadamard(x.float(), self.h), w, b).to(torch.bfloat16)

    def linear_rows(self, x: torch.Tensor, weights) -> torch.Tensor:
        """Every linear of the block (plus norms / residuals) over a slice of token rows,
        with the dequantized weights of this call."""
        w_qkv, w_o, w_fc1, w_fc2 = weights
        shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = self.mod.unbind(0)
        h = self._rms_adaln(x, shift_a, scale_a)
        self._linear(h, w_qkv, self.b_qkv)
        x = x.addcmul(self._linear(h, w_o, self.b_o), gate_a)
        h = self._rms_adaln(x, shift_m, scale_m)
        u = F.gelu(self._linear(h, w_fc1, self.b_fc1), approximate="tanh")
        return x.addcmul(self._linear(u, w_fc2, self.b_fc2), gate_m)

    @staticmethod
    def attention_rows(q, k, v):
        return F.scaled_dot_product_attention(q, k, v)


def measure(L: int = 111600, heads: int = 32, row_sample: int = 256, query_sample: int = 256,
            block: ReferenceBlockCPU | None = None, seed: int = 0) -> dict:
    """One bounded sample of the reference's CPU path: the four weight dequantizations
    (once per block call, as the CPU fallbacks dequantize per call), `row_sample` token
    rows through every linear, and `query_sample` queries of one head against all L keys
    (dense torch SDPA, the reference's CPU attention).  Returns the wall time of the
    sample and the seconds for a whole block extrapolated from it: dequantization once,
    the linears x L / row_sample, the attention x (L / query_sample) x heads."""
    torch.manual_seed(seed)
    block = block or ReferenceBlockCPU()
    x = torch.randn(row_sample, block.hidden).to(torch.bfloat16)
    q = torch.randn(1, 1, query_sample, 128).to(torch.bfloat16)
    k = torch.randn(1, 1, L, 128).to(torch.bfloat16)
    v = torch.randn(1, 1, L, 128).to(torch.bfloat16)
    t0 = time.perf_counter()
    weights = block.dequant_all()
    t1 = time.perf_counter()
    block.linear_rows(x, weights)
    t2 = time.perf_counter()
    block.attention_rows(q, k, v)
    t3 = time.perf_counter()
    t_deq, t_lin, t_att = t1 - t0, t2 - t1, t3 - t2
    full = t_deq + t_lin * (L / row_sample) + t_att * (L / query_sample) * heads
    return {"seconds_per_block": full, "sample_seconds": t3 - t0, "t_dequant": t_deq, "t_linear_sample": t_lin,
            "t_attention_sample": t_att, "threads": torch.get_num_threads(), "cores": os.cpu_count(),
            "sample": f"weight dequantization of all four linears (per call, as the reference's CPU "
                      f"fallbacks do) + {row_sample} token rows through all four linears + {query_sample} "
                      f"queries x 1 head against all {L} keys (dense torch SDPA); the whole-block time is "
                      f"extrapolated linearly to {L} tokens x {heads} heads"}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


if __name__ == "__main__":
    r = measure()
    print(r, "tokens/s", 111600 / r["seconds_per_block"], math.nan)
