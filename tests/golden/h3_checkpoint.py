"""A seeded synthetic block checkpoint in the pruned H3 tensor contract (test infrastructure).

`synthetic_block(seed)` returns (state, quantization_metadata, inputs) for block 0 of a
small H3-shaped model whose layers mix the checkpoint formats the engine's
`_quant_linear` distinguishes by tensor names (model/assembly.py:166-228):

  attn.qkv_proj   ConvRot INT8, per-output-row weight_scale            (no bias: the
                  engine passes only weight / weight_scale / comfy_quant)
  attn.out_proj   packed W4A8, group 16, e4m3 s_rel, 16-entry codebook, bias;
                  spec taken from the H3 default (no file metadata for this layer)
  mlp.fc1         packed W4A8, group 32, fp32 s_rel, uniform levels, correction, bias;
                  spec recorded in the file metadata
  mlp.fc2         ConvRot INT8, scalar weight_scale

hidden 256, 4 heads of 128 (attention width 512, unlike hidden, as in H3), SwiGLU MLP
(fc1 256 -> 2 x 512, fc2 512 -> 256), AdaLN projection 8 -> 18 x hidden (three
modulation rows per timestep row).  Inputs: 384 tokens on a 3 x 8 x 16 grid, two
timestep rows, three modulation segments, split-half RoPE angles from 16 inverse
frequencies per axis (rotary width 96; model/layers.py:51-57).

Both the fixture generator (which runs the engine's own block on these tensors) and the
tests build the checkpoint from here; `state_digest` pins the bytes so a change in the
generator cannot go unnoticed.
"""

from __future__ import annotations

import hashlib
import json

import torch

HIDDEN, HEADS, HEAD_DIM, FFN, CURVE_DIM = 256, 4, 128, 512, 8
GRID = (3, 8, 16)
SEGMENTS = ((0, 64, 0), (64, 128, 4), (128, 384, 5))
PREFIX = "blocks.0"
FC1_SPEC = {"format": "asym_w4a8_int8", "group_size": 32, "convrot": True, "convrot_groupsize": 256}


def _int8_rows(w: torch.Tensor, per_row: bool) -> tuple[torch.Tensor, torch.Tensor]:
    amax = w.abs().amax(dim=1, keepdim=True) if per_row else w.abs().amax().reshape(1, 1)
    scale = amax / 127.0
    q = torch.clamp(torch.round(w / scale), -127, 127).to(torch.int8)
    return q, scale.reshape(-1).float()


def _comfy_quant(convrot: bool) -> torch.Tensor:
    body = json.dumps({"format": "int8_tensorwise", "params": {"convrot": convrot, "convrot_groupsize": 256}})
    return torch.tensor(list(body.encode("utf-8")), dtype=torch.uint8)


def _w4(g, n: int, k: int, group: int, *, e4m3: bool, codebook: bool, correction: bool, bias: bool) -> dict:
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)
    s_rel = torch.rand(n, k // group, generator=g) * 10.0 + 5.0
    t = {"weight": packed.contiguous(),
         "weight_s_rel": s_rel.to(torch.float8_e4m3fn) if e4m3 else s_rel,
         "weight_s_channel": (torch.rand(n, generator=g) * 1e-3 + 1e-3).float()}
    if codebook:
        t["weight_codebook"] = (torch.linspace(-7.5, 7.5, 16) + 0.2 * torch.rand(16, generator=g) - 0.1).float()
    if correction:
        t["weight_correction"] = (torch.randn(k // group, n, generator=g) * 1e-2).to(torch.bfloat16)
    if bias:
        t["bias"] = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    return t


def synthetic_block(seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    W = HEADS * HEAD_DIM
    state: dict[str, torch.Tensor] = {}

    def put(prefix: str, tensors: dict) -> None:
        for name, value in tensors.items():
            state[f"{PREFIX}.{prefix}.{name}"] = value

    q, s = _int8_rows(torch.randn(3 * W, HIDDEN, generator=g) * 0.08, per_row=True)
    put("attn.qkv_proj", {"weight": q, "weight_scale": s, "comfy_quant": _comfy_quant(True)})
    put("attn.out_proj", _w4(g, HIDDEN, W, 16, e4m3=True, codebook=True, correction=False, bias=True))
    put("mlp.fc1", _w4(g, 2 * FFN, HIDDEN, 32, e4m3=False, codebook=False, correction=True, bias=True))
    q, s = _int8_rows(torch.randn(HIDDEN, FFN, generator=g) * 0.06, per_row=False)
    put("mlp.fc2", {"weight": q, "weight_scale": s, "comfy_quant": _comfy_quant(True)})
    for name, n in (("attn.q_norm.weight", HEAD_DIM), ("attn.k_norm.weight", HEAD_DIM),
                    ("norm1.weight", HIDDEN), ("norm2.weight", HIDDEN)):
        state[f"{PREFIX}.{name}"] = (1 + 0.05 * torch.randn(n, generator=g)).to(torch.bfloat16)
    state[f"{PREFIX}.adaln_proj.linear.weight"] = (torch.randn(18 * HIDDEN, CURVE_DIM, generator=g) * 0.2).to(
        torch.bfloat16)
    state[f"{PREFIX}.adaln_proj.linear.bias"] = (torch.randn(18 * HIDDEN, generator=g) * 0.05).to(torch.bfloat16)
    metadata = {f"{PREFIX}.mlp.fc1": dict(FC1_SPEC)}

    L = GRID[0] * GRID[1] * GRID[2]
    x = (torch.randn(L, HIDDEN, generator=g) * 0.25).to(torch.bfloat16)
    curve_rows = (torch.randn(2, CURVE_DIM, generator=g)).to(torch.bfloat16)
    idx = torch.arange(L)
    positions = torch.stack((idx // (GRID[1] * GRID[2]), (idx // GRID[2]) % GRID[1], idx % GRID[2]), dim=1)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, 32, 2).float() / 32))
    per_axis = positions.float().unsqueeze(-1) * inv_freq.reshape(1, 1, -1)
    half = torch.cat(per_axis.unbind(dim=1), dim=-1)
    frequencies = torch.cat((half, half), dim=-1)
    inputs = {"x": x, "curve_rows": curve_rows, "frequencies": frequencies, "segments": SEGMENTS}
    return state, metadata, inputs


def state_digest(state: dict[str, torch.Tensor]) -> str:
    h = hashlib.sha256()
    for key in sorted(state):
        t = state[key].contiguous()
        h.update(key.encode())
        h.update(str(t.dtype).encode())
        h.update(str(tuple(t.shape)).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return h.hexdigest()
