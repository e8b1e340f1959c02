"""End-to-end check of the B200 DiT block against an fp32 torch restatement of
the same block (dequantized weights, exact Hadamard rotation, exact softmax).

The quantized path (per-token INT8, W4, INT8 QK / FP8 PV) is compared on the
residual update x_out - x_in, where quantization error shows; a mask-free
(dense) block keeps the comparison independent of block selection.
"""

import math

import pytest
import torch
import torch.nn.functional as F

from gpu_util import cosine, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def blockmod():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import block as B
    return B


def _had(device):
    h4 = torch.tensor(((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1)), dtype=torch.float32)
    m = h4
    while m.shape[0] < 256:
        m = torch.kron(m, h4)
    return (m / 16.0).to(device)


def _rot(x, h):
    return torch.matmul(x.reshape(-1, x.shape[-1] // 256, 256), h).reshape_as(x)


def reference_block(blk, x, t, rope):
    cfg = blk.cfg
    H, D = cfg.heads, cfg.head_dim
    hm = _had(x.device)
    mod = blk.modulation(t).float()[0]
    sa, ca, ga, sm, cm, gm = mod.unbind(0)

    def rms_adaln(v, w, scale, shift):
        n = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + cfg.eps) * w.float()
        return n * (1 + scale) + shift

    xf = x.float()
    h = rms_adaln(xf, blk.norm1, ca, sa)
    qkv = F.linear(_rot(h, hm), blk.qkv.dense_weight(), blk.qkv.bias.float())
    L = x.shape[0]
    q, k, v = qkv.view(L, 3, H, D).unbind(1)
    cos, sin = rope[0].float(), rope[1].float()

    def norm_rope(z, w):
        z = z * torch.rsqrt(z.pow(2).mean(-1, keepdim=True) + cfg.qk_eps) * w.float()
        a, b = z[..., :64], z[..., 64:]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.cat((a * c - b * s, a * s + b * c), -1)

    q, k = norm_rope(q, blk.q_norm), norm_rope(k, blk.k_norm)
    o = torch.softmax(torch.einsum("lhd,mhd->hlm", q, k) / math.sqrt(D), -1)
    o = torch.einsum("hlm,mhd->lhd", o, v).reshape(L, H * D)
    xf = xf + F.linear(_rot(o, hm), blk.out.dense_weight(), blk.out.bias.float()) * ga
    h = rms_adaln(xf, blk.norm2, cm, sm)
    u = F.gelu(F.linear(_rot(h, hm), blk.fc1.dense_weight(), blk.fc1.bias.float()), approximate="tanh")
    return xf + F.linear(_rot(u, hm), blk.fc2.dense_weight(), blk.fc2.bias.float()) * gm


@pytest.mark.parametrize("L", [1536, 2000])
def test_dense_block_matches_fp32_reference(blockmod, L):
    B = blockmod
    cfg = B.BlockConfig(hidden=1024, heads=8, ffn=4096, t_dim=256, mask=None)
    blk = B.DiTBlockB200(cfg, device="cuda", seed=3)
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(L, cfg.hidden, generator=g, device="cuda").to(torch.bfloat16)
    t = torch.randn(cfg.t_dim, generator=g, device="cuda").to(torch.bfloat16)
    rope = B.rope_tables((1, L // 16, 16) if L % 16 == 0 else (1, 1, L), cfg.rope_splits, device="cuda")
    ref = reference_block(blk, x, t, rope)
    out = blk.forward(x.clone(), t, rope).float()
    upd, upd_ref = out - x.float(), ref - x.float()
    assert cosine(upd, upd_ref) > 0.995
    assert rel_l2(upd, upd_ref) < 0.1


def test_sparse_block_runs_and_tracks_dense(blockmod):
    B = blockmod
    from h3b import attention as A
    cfg_d = B.BlockConfig(hidden=1024, heads=8, ffn=4096, t_dim=256, mask=None)
    cfg_s = B.BlockConfig(hidden=1024, heads=8, ffn=4096, t_dim=256, mask=A.MaskConfig("topk", 1.0))
    L = 1024
    bd = B.DiTBlockB200(cfg_d, device="cuda", seed=1)
    bs = B.DiTBlockB200(cfg_s, device="cuda", seed=1)
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(L, 1024, generator=g, device="cuda").to(torch.bfloat16)
    t = torch.randn(256, generator=g, device="cuda").to(torch.bfloat16)
    rope = B.rope_tables((4, 16, 16), cfg_d.rope_splits, device="cuda")
    yd = bd.forward(x.clone(), t, rope)
    ys = bs.forward(x.clone(), t, rope)
    # a Top-K budget of 1.0 keeps every block: the sparse kernel must equal the dense one
    assert torch.equal(yd, ys)


def test_host_pipeline_matches_sequential_forwards(blockmod):
    """The overlapped host->device / block / device->host runner gives, step for
    step, the bits of plain forwards on the same inputs."""
    B = blockmod
    cfg = B.BlockConfig(hidden=1024, heads=8, ffn=4096, t_dim=256)
    blk = B.DiTBlockB200(cfg, device="cuda", seed=4)
    L, steps = 1024, 4
    g = torch.Generator().manual_seed(6)
    xs = [torch.randn(L, cfg.hidden, generator=g).to(torch.bfloat16).pin_memory() for _ in range(steps)]
    ts = [torch.randn(cfg.t_dim, generator=g).to(torch.bfloat16).pin_memory() for _ in range(steps)]
    outs = [torch.empty(L, cfg.hidden, dtype=torch.bfloat16).pin_memory() for _ in range(steps)]
    rope = B.rope_tables((4, 16, 16), cfg.rope_splits, device="cuda")
    pipe = B.HostPipeline(blk, rope, L)
    pipe.run(xs, ts, outs)
    torch.cuda.synchronize()
    for k in range(steps):
        ref = blk.forward(xs[k].cuda(), ts[k].cuda(), rope).cpu()
        assert torch.equal(outs[k], ref), k


def test_chunked_forward_matches_single_chunk(blockmod):
    """The row-local phases run chunk by chunk give the bits of the whole-row run,
    with AdaLN segments that cross the chunk boundaries."""
    B = blockmod
    cfg = B.BlockConfig(hidden=1024, heads=8, ffn=4096, t_dim=256)
    blk = B.DiTBlockB200(cfg, device="cuda", seed=7)
    L = 1024
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(L, cfg.hidden, generator=g, device="cuda").to(torch.bfloat16)
    t = torch.randn(3, cfg.t_dim, generator=g, device="cuda").to(torch.bfloat16)
    rope = B.rope_tables((4, 16, 16), cfg.rope_splits, device="cuda")
    segments = ((0, 300, 0), (300, 700, 1), (700, 1024, 2))
    whole = blk.forward(x.clone(), t, rope, segments=segments)
    seen = []
    chunked = blk.forward(x.clone(), t, rope, segments=segments, chunks=[0, 100, 517, 1000, 1024],
                          rows_ready=lambda i: seen.append(("in", i)), rows_done=lambda i: seen.append(("out", i)))
    assert torch.equal(whole, chunked)
    assert seen == [("in", 0), ("in", 1), ("in", 2), ("in", 3), ("out", 0), ("out", 1), ("out", 2), ("out", 3)]
