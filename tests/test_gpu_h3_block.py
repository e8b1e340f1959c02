"""The block at the real H3 dimensions (model/config.py:12-17), loaded through the
checkpoint path, against an fp32 torch restatement of the same block.

hidden 5376, 56 heads of 128 (attention width 7168 != hidden), SwiGLU MLP
5376 -> 2 x 14336 -> 5376, layers mixed as a `*_pruned_w4a8_mixed` file mixes them:
QKV ConvRot INT8 (per-row scales), out-proj and FC1 packed W4A8 (group 16, e4m3 s_rel,
16-entry codebook, bias), FC2 ConvRot INT8 (scalar scale); AdaLN projection to
18 x hidden (three modulation rows per timestep row) with three segments; RoPE of width
96 (16 inverse frequencies per axis) from the engine's angle form.  Dense attention,
so the comparison does not depend on block selection.

The quantized path (per-token INT8, W4/W8 weights, INT8 QK / FP8 PV) is compared on the
residual update x_out - x_in with the tolerance of the benchmark-shaped block test
(test_gpu_block.py).
"""

import math

import pytest
import torch
import torch.nn.functional as F

from gpu_util import cosine, rel_l2

pytestmark = pytest.mark.gpu

HIDDEN, HEADS, HD, FFN, CURVE = 5376, 56, 128, 14336, 8
GRID = (2, 16, 32)                       # 1024 tokens
SEGMENTS = ((0, 100, 0), (100, 300, 4), (300, 1024, 5))


def _comfy_quant():
    import json
    body = json.dumps({"format": "int8_tensorwise", "params": {"convrot": True, "convrot_groupsize": 256}})
    return torch.tensor(list(body.encode("utf-8")), dtype=torch.uint8)


def _int8(g, n, k, std, per_row):
    w = torch.randn(n, k, generator=g, device="cuda") * std
    amax = w.abs().amax(dim=1, keepdim=True) if per_row else w.abs().amax().reshape(1, 1)
    scale = amax / 127.0
    return torch.clamp(torch.round(w / scale), -127, 127).to(torch.int8), scale.reshape(-1).float()


def _w4(g, n, k, group):
    codes = torch.randint(0, 16, (n, k), generator=g, device="cuda", dtype=torch.int32)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8).view(torch.int8).contiguous()
    s_rel = (torch.rand(n, k // group, generator=g, device="cuda") * 10.0 + 5.0).to(torch.float8_e4m3fn)
    s_ch = (torch.rand(n, generator=g, device="cuda") * 2e-4 + 2e-4).float()
    cb = (torch.linspace(-7.5, 7.5, 16, device="cuda") + 0.2 * torch.rand(16, generator=g, device="cuda") - 0.1)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.01).to(torch.bfloat16)
    return {"weight": packed, "weight_s_rel": s_rel, "weight_s_channel": s_ch, "weight_codebook": cb.float(),
            "bias": bias}


def h3_state(seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = HEADS * HD
    st = {}

    def put(prefix, tensors):
        for k, v in tensors.items():
            st[f"blocks.0.{prefix}.{k}"] = v

    q, s = _int8(g, 3 * W, HIDDEN, 0.04, per_row=True)
    put("attn.qkv_proj", {"weight": q, "weight_scale": s, "comfy_quant": _comfy_quant()})
    put("attn.out_proj", _w4(g, HIDDEN, W, 16))
    put("mlp.fc1", _w4(g, 2 * FFN, HIDDEN, 16))
    q, s = _int8(g, HIDDEN, FFN, 0.02, per_row=False)
    put("mlp.fc2", {"weight": q, "weight_scale": s, "comfy_quant": _comfy_quant()})
    for name, n in (("attn.q_norm.weight", HD), ("attn.k_norm.weight", HD), ("norm1.weight", HIDDEN),
                    ("norm2.weight", HIDDEN)):
        st[f"blocks.0.{name}"] = (1 + 0.05 * torch.randn(n, generator=g, device="cuda")).to(torch.bfloat16)
    st["blocks.0.adaln_proj.linear.weight"] = (torch.randn(18 * HIDDEN, CURVE, generator=g, device="cuda")
                                               * 0.2).to(torch.bfloat16)
    st["blocks.0.adaln_proj.linear.bias"] = (torch.randn(18 * HIDDEN, generator=g, device="cuda")
                                             * 0.05).to(torch.bfloat16)
    return st, g


def _had(device):
    h4 = torch.tensor(((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1)), dtype=torch.float32)
    m = h4
    while m.shape[0] < 256:
        m = torch.kron(m, h4)
    return (m / 16.0).to(device)


def _rot(x, h):
    return torch.matmul(x.reshape(-1, x.shape[-1] // 256, 256), h).reshape_as(x)


def reference_block(blk, x, curve_rows, cos, sin, segments):
    """fp32 block over the dequantized weights: exact Hadamard rotation, exact softmax."""
    cfg = blk.cfg
    hm = _had(x.device)
    mod = blk.modulation(curve_rows).float()                 # [R, 6, hidden]
    rows = torch.empty(x.shape[0], dtype=torch.long, device=x.device)
    for start, stop, r in segments:
        rows[start:stop] = r
    sa, ca, ga, sm, cm, gm = (mod[rows, i] for i in range(6))

    def rms_adaln(v, w, scale, shift):
        n = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + cfg.eps) * w.float()
        return n * (1 + scale) + shift

    def lin(layer, v):
        b = None if layer.bias is None else layer.bias.float()
        return F.linear(_rot(v, hm), layer.dense_weight(), b)

    L = x.shape[0]
    xf = x.float()
    qkv = lin(blk.qkv, rms_adaln(xf, blk.norm1, ca, sa))
    q, k, v = qkv.view(L, 3, HEADS, HD).unbind(1)
    rot = 2 * cos.shape[1]
    c, s = cos.float()[:, None, :], sin.float()[:, None, :]

    def norm_rope(z, w):
        z = z * torch.rsqrt(z.pow(2).mean(-1, keepdim=True) + cfg.qk_eps) * w.float()
        a, b, rest = z[..., :rot // 2], z[..., rot // 2:rot], z[..., rot:]
        return torch.cat((a * c - b * s, a * s + b * c, rest), -1)

    q, k = norm_rope(q, blk.q_norm), norm_rope(k, blk.k_norm)
    p = torch.softmax(torch.einsum("lhd,mhd->hlm", q, k) / math.sqrt(HD), -1)
    o = torch.einsum("hlm,mhd->lhd", p, v).reshape(L, HEADS * HD)
    xf = xf + lin(blk.out, o) * ga
    h = lin(blk.fc1, rms_adaln(xf, blk.norm2, cm, sm))
    gate, up = h[:, :FFN], h[:, FFN:]
    return xf + lin(blk.fc2, F.silu(gate) * up) * gm


def test_h3_dimension_block_from_checkpoint_tracks_fp32():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import h3b
    from h3b import checkpoint as C
    from h3b.block import rope_tables_from_frequencies

    state, g = h3_state(0)
    meta = {"blocks.0.attn.out_proj": {"format": "asym_w4a8_int8", "group_size": 16},
            "blocks.0.mlp.fc1": {"format": "asym_w4a8_int8", "group_size": 16}}
    blk = C.load_block(0, C.MappingTensorSource(state, quantization_metadata=meta), device="cuda")
    assert (blk.cfg.hidden, blk.cfg.heads, blk.cfg.ffn, blk.cfg.mlp_act) == (HIDDEN, HEADS, FFN, "swiglu")
    assert type(blk.qkv).__name__ == "Int8Linear" and type(blk.fc1).__name__ == "W4A8Linear"

    L = GRID[0] * GRID[1] * GRID[2]
    x = (torch.randn(L, HIDDEN, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    curve_rows = torch.randn(2, CURVE, generator=g, device="cuda").to(torch.bfloat16)
    idx = torch.arange(L, device="cuda")
    pos = torch.stack((idx // (GRID[1] * GRID[2]), (idx // GRID[2]) % GRID[1], idx % GRID[2]), 1).float()
    inv = 1.0 / (10000.0 ** (torch.arange(0, 32, 2, device="cuda").float() / 32))
    half = torch.cat((pos[:, 0:1] * inv, pos[:, 1:2] * inv, pos[:, 2:3] * inv), -1)
    frequencies = torch.cat((half, half), -1)                 # [L, 96]
    cos, sin = rope_tables_from_frequencies(frequencies)

    ref = reference_block(blk, x, curve_rows, cos, sin, SEGMENTS)
    out = blk.forward(x.clone(), curve_rows, (cos, sin), segments=SEGMENTS).float()
    upd, upd_ref = out - x.float(), ref - x.float()
    assert upd_ref.pow(2).mean().sqrt() > 8 * 2.0 ** -9 * x.float().abs().mean()   # update well above bf16 steps of x
    assert cosine(upd, upd_ref) > 0.995
    assert rel_l2(upd, upd_ref) < 0.1
    for start, stop, _ in SEGMENTS:
        assert cosine(upd[start:stop], upd_ref[start:stop]) > 0.99, (start, stop)
    assert h3b.device_status(0) == 0
