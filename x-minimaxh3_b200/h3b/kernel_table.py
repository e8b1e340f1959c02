"""Every kernel of one DiT block step at the benchmark's shape, against its roofline.

    python x-minimaxh3_b200/h3b/kernel_table.py [--tokens 111600] [--reps 10]

Each call of the block (720p/5 s: 111,600 tokens, hidden 4096, 32 heads, MLP 16384 with
W4A8 G=128 weights and the tanh-GELU FC2 quantizer, Sparge cdf 0.6) is timed alone with
CUDA events over `--reps` launches after warm-up, on inputs larger than L2.  Each row
gives the algorithmic work of one call -- bytes that must cross HBM once (read + write) for
the memory-bound kernels, 2 x multiply-adds for the tensor-core ones (the attention counts
the tiles the block bitmap keeps; fp32 multiply-adds for the mask's scores) -- and the
fraction of the measured peak it reaches:
HBM copy bandwidth, or twice the sustained bf16 GEMM rate for INT8/FP8 (MEASURED_PEAKS.json
next to bench.py; the fallback figures when it is absent).  Prints a markdown table.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from h3b import attention as A  # noqa: E402
from h3b import block as B  # noqa: E402
from h3b import ops  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), 2.0 * float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 2.0 * 1400.0, "fallback"


def timed(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=111600)
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    hbm, tensor, src = peaks()
    L = args.tokens
    cfg = B.BlockConfig()
    blk = B.DiTBlockB200(cfg, device="cuda", seed=0)
    D, F, H = cfg.hidden, cfg.ffn, cfg.heads
    W = H * cfg.head_dim
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(L, D, device="cuda", generator=g).to(torch.bfloat16)
    t = torch.randn(cfg.t_dim, device="cuda", generator=g).to(torch.bfloat16)
    grid = (31, 45, 80) if L == 111600 else (1, 1, L)
    rope = B.rope_tables(grid, cfg.rope_splits, device="cuda")
    mod = blk.modulation(t)
    sh_a, sc_a, ga, sh_m, sc_m, gm = mod.unbind(1)
    rows = []

    def row(name, ms, work, kind):
        if kind == "hbm":
            achieved = work / ms / 1e6
            rows.append((name, ms, f"{work / 1e9:.2f} GB", f"{achieved:,.0f} GB/s", achieved / hbm))
        elif kind == "fma":
            rows.append((name, ms, f"{work / 1e9:.1f} GFLOP", f"{work / ms / 1e9:,.1f} TFLOP/s fp32", None))
        else:
            achieved = work / ms / 1e9
            rows.append((name, ms, f"{work / 1e12:.1f} Tops", f"{achieved:,.0f} TOPS", achieved / tensor))

    # RMSNorm + AdaLN + ConvRot + INT8 (norm1; norm2 is the same call)
    ms = timed(lambda: ops.rms_adaln_quantize_int8(x, blk.norm1, sc_a, sh_a, None, cfg.eps, 256), args.reps)
    row("rms_adaln + ConvRot INT8 quantizer (K 4096) x2", ms, L * D * 3 + L * 4, "hbm")
    xq, xs = ops.rms_adaln_quantize_int8(x, blk.norm1, sc_a, sh_a, None, cfg.eps, 256)
    qkv = torch.empty(L, 3 * W, device="cuda", dtype=torch.bfloat16)
    ms = timed(lambda: blk.qkv.forward_prequantized_qk_rope(xq, xs, qkv, H, 0, W, blk.q_norm, blk.k_norm, rope[0],
                                                            rope[1], cfg.qk_eps), args.reps)
    row("QKV INT8 GEMM + dequant + q/k RMSNorm/RoPE epilogue (N 12288, K 4096)", ms, 2.0 * L * 3 * W * D,
        "tensor")
    view = qkv.view(L, 3, H, cfg.head_dim)
    q, k, v = view[:, 0], view[:, 1], view[:, 2]
    ms = timed(lambda: A.prepare_values(v), args.reps)
    row("V -> FP8 (absmax, scale, transpose)", ms, L * W * 2 + L * W, "hbm")
    ms = timed(lambda: A.prepare_keys(k), args.reps)
    row("K mean + pool / similarity / INT8", ms, 2 * L * W * 2 + L * W, "hbm")
    ms = timed(lambda: A.prepare_queries(q), args.reps)
    row("Q pool / similarity / INT8", ms, L * W * 2 + L * W, "hbm")
    pv = A.prepare_values(v)
    pk, _ = A.prepare_keys(k)
    pq = A.prepare_queries(q)
    ms = timed(lambda: A.block_mask(pq, pk, cfg.mask), args.reps)
    qb, kb = math.ceil(L / 128), math.ceil(L / 64)
    row("Sparge block mask (fp32 scores + selection)", ms, 2.0 * qb * kb * H * 128, "fma")
    bitmap = A.block_mask(pq, pk, cfg.mask)
    ms = timed(lambda: A.attention(pq, pk, pv, bitmap), args.reps)
    row(f"attention (INT8 QK, FP8 PV; kept tiles {B.kept_tiles(bitmap, L) / (qb * kb * H):.3f})", ms,
        B.attention_ops(bitmap, L, L, H), "tensor")
    o2 = A.attention(pq, pk, pv, bitmap).view(L, W)
    ms = timed(lambda: blk.out.quantize(o2), args.reps)
    row("ConvRot INT8 quantizer (out-proj input, K 4096)", ms, L * W * 3 + L * 4, "hbm")
    oq, os_ = blk.out.quantize(o2)
    xr = x.clone()
    ms = timed(lambda: blk.out.gated_residual_(xr, ga[0], oq, os_), args.reps)
    row("out-proj INT8 GEMM + gated residual (N 4096, K 4096)", ms, 2.0 * L * D * W, "tensor")
    ms = timed(lambda: blk.fc1.int8_weight(), args.reps)
    row("W4 -> INT8 decode, FC1 weight (16384 x 4096)", ms, F * D / 2 + F * (D // cfg.w4_group) * 4 + F * D, "hbm")
    xq2, xs2 = ops.rms_adaln_quantize_int8(x, blk.norm2, sc_m, sh_m, None, cfg.eps, 256)
    ms = timed(lambda: blk.fc1.forward_prequantized(xq2, xs2), args.reps)
    row("FC1 W4A8 (decode + INT8 GEMM, N 16384, K 4096)", ms, 2.0 * L * F * D, "tensor")
    h = blk.fc1.forward_prequantized(xq2, xs2)
    ms = timed(lambda: blk.fc2.quantize(h, cfg.mlp_act), args.reps)
    row("tanh-GELU + ConvRot INT8 quantizer (K 16384)", ms, L * F * 3 + L * 4, "hbm")
    hq, hs = blk.fc2.quantize(h, cfg.mlp_act)
    del h
    ms = timed(lambda: blk.fc2.gated_residual_(xr, gm[0], hq, hs), args.reps)
    row("FC2 W4A8 + gated residual (N 4096, K 16384)", ms, 2.0 * L * D * F, "tensor")

    step = timed(lambda: blk.forward(x.clone(), t, rope), 3)
    print(f"L = {L}, {torch.cuda.get_device_name()}; peaks ({src}): HBM {hbm:,.0f} GB/s, "
          f"INT8/FP8 {tensor:,.0f} TOPS (2 x bf16 sustained)\n")
    print("| kernel (one call) | ms | work | achieved | of peak |")
    print("|---|---:|---:|---:|---:|")
    for name, ms, work, ach, frac in rows:
        print(f"| {name} | {ms:.3f} | {work} | {ach} | {'-' if frac is None else f'{frac:.2f}'} |")
    print(f"\nblock forward (all of the above, norm quantizer twice, x.clone() included): {step:.2f} ms")


if __name__ == "__main__":
    main()
