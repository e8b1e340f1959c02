"""Helpers shared by the GPU parity tests (torch <-> oracle numpy formats)."""

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns (numpy, CPU)."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def rel_l2(a, b) -> float:
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def cosine(a, b) -> float:
    a = torch.as_tensor(a).double().cpu().reshape(-1)
    b = torch.as_tensor(b).double().cpu().reshape(-1)
    return float(a @ b / (a.norm() * b.norm()).clamp_min(1e-30))


def outlier_activations(g, m, k, frac=0.01, mult=20.0):
    """Activations with outlier channels, as the INT8 GEMM benchmark uses: N(0,1) with 1% of
    channels scaled by 20."""
    x = torch.randn(m, k, generator=g)
    nout = max(1, int(round(k * frac)))
    cols = torch.randperm(k, generator=g)[:nout]
    x[:, cols] *= mult
    return x


def scale_of_rows(pb, rows: torch.Tensor) -> torch.Tensor:
    """[H, len(rows)] scale of each row of a PreparedBlocks (any granularity)."""
    if pb.gran == 1:
        idx = (rows // 32) * 8 + rows % 8 if pb.block == 128 else (rows // 64) * 4 + (rows % 8) // 2
    else:
        idx = rows // pb.block
    return pb.scale[:, idx]


def tile_rows(Lq: int, tiles) -> torch.Tensor:
    return torch.cat([torch.arange(t * 128, min(Lq, t * 128 + 128)) for t in tiles])


def kernel_order_reference(pq, pk, pv, bitmap=None, tiles=None, heads=None):
    """The CPU oracle in the kernel's own arithmetic (P -> E4M3 under the lazy running
    max) for the query rows of `tiles` (128-row tiles, default all) and `heads`
    (default all): float32 [rows, heads, 128] and the row indices."""
    from oracle import oracle as O

    H = pq.qi8.shape[0]
    heads = list(range(H)) if heads is None else list(heads)
    Lq, Lk = pq.tokens, pk.tokens
    tiles = list(range((Lq + 127) // 128)) if tiles is None else list(tiles)
    hsel = torch.tensor(heads)
    k = pk.qi8[hsel].cpu().numpy()
    ks = pk.scale[hsel].cpu().numpy()
    vt = pv.vt[hsel].cpu().numpy()
    vs = pv.scale[hsel].cpu().numpy()
    qall = pq.qi8[hsel].cpu().numpy()
    qsall = pq.scale[hsel].cpu().numpy()
    bm = None if bitmap is None else bitmap.view(torch.int32)[hsel].cpu().numpy().view(np.uint32)
    outs = []
    for t in tiles:
        n = min(128, Lq - t * 128)
        q = np.zeros((len(heads), 128, 128), np.int8)
        q[:, :n] = qall[:, t * 128:t * 128 + n]
        if pq.gran == 1:
            qs = qsall[:, t * 32:(t + 1) * 32]
        else:
            per = 128 // pq.block
            qs = qsall[:, t * per:(t + 1) * per]
        o = O.attention_kernel(q, qs, n, k, ks, Lk, vt, vs, None if bm is None else bm[:, t:t + 1],
                               q_gran=pq.gran, q_block=pq.block, k_gran=pk.gran)
        outs.append(O.bf16_bits_to_f32(o))
    return np.concatenate(outs, 0), tile_rows(Lq, tiles)


def exact_reference(pq, pk, pv, bitmap=None, rows=None, heads=None):
    """fp32 softmax attention (torch, on the device) over the same dequantized INT8 Q / K
    and E4M3 V, restricted to the bitmap's blocks: float32 [rows, heads, 128]."""
    import math

    from oracle import oracle as O

    H = pq.qi8.shape[0]
    dev = pq.qi8.device
    hsel = torch.arange(H, device=dev) if heads is None else torch.tensor(list(heads), device=dev)
    Lq, Lk = pq.tokens, pk.tokens
    rows = torch.arange(Lq) if rows is None else rows
    rows = rows.to(dev)
    keys = torch.arange(Lk, device=dev)
    q = pq.qi8[hsel][:, rows].float() * scale_of_rows(pq, rows)[hsel][..., None]
    k = pk.qi8[hsel][:, :Lk].float() * scale_of_rows(pk, keys)[hsel][..., None]
    lut = torch.tensor([O.lib().h3bo_e4m3_to_f32(i) for i in range(256)], device=dev)
    v = lut[pv.vt[hsel][:, :, :Lk].long()].transpose(1, 2) * pv.scale[hsel][:, None, :]
    s = q @ k.transpose(1, 2) / math.sqrt(128)
    if bitmap is not None:
        words = bitmap.view(torch.int32)[hsel][:, rows // 128]
        Kb = (Lk + 63) // 64
        keep = ((words[..., :, None] >> torch.arange(32, device=dev)) & 1).reshape(len(hsel), len(rows), -1)[..., :Kb]
        s = s.masked_fill(~keep.bool().repeat_interleave(64, 2)[..., :Lk], float("-inf"))
    return (s.softmax(-1) @ v).permute(1, 0, 2).cpu()


# Attention tolerances.  Against the kernel-order oracle (the same P -> E4M3 rounding,
# lazy max and fp32 row sums) the kernel differs only by ex2.approx's last bits and the
# tensor core's fp32 accumulation order; against exact softmax over the same operands
# the E4M3 rounding of P (3 mantissa bits) adds about 2.5 % rel-L2, which the
# north_star cosine bound (>= 0.999) covers.
KERNEL_ORDER_REL_L2 = 5e-3
KERNEL_ORDER_COS = 0.9999
EXACT_COS = 0.999


def assert_attention_parity(out, pq, pk, pv, bitmap=None, tiles=None, heads=None):
    """out: the kernel's bf16 [Lq, H, 128]; checks sampled tiles / heads (default all)."""
    H = pq.qi8.shape[0]
    hs = list(range(H)) if heads is None else list(heads)
    ko, rows = kernel_order_reference(pq, pk, pv, bitmap, tiles, hs)
    got = out[rows.to(out.device)][:, hs].float().cpu()
    r, c = rel_l2(got, ko), cosine(got, ko)
    assert r <= KERNEL_ORDER_REL_L2 and c >= KERNEL_ORDER_COS, f"vs kernel-order oracle: rel-L2 {r:.2e} cos {c:.6f}"
    ex = exact_reference(pq, pk, pv, bitmap, rows, hs)
    ce = cosine(got, ex)
    assert ce >= EXACT_COS, f"vs exact softmax: cos {ce:.6f}"
    return r, c, ce
