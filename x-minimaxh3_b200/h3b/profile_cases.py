"""Single-kernel cases for profiling the hot path (ncu captures, CUDA-event timing).

    python -m h3b.profile_cases <case> [--reps N] [--time]

Each case builds seeded inputs at a size that keeps an `ncu --set full` capture short
(inputs larger than L2, a few GB on the device at most), then launches the kernel
`--reps` times.  With `--time` it prints the mean CUDA-event time of the launches.

Cases:
    attn_dense / attn_sparse   h3b_attention, L = 65,536, 8 heads (sparse: cdf 0.6 mask)
    gemm                       h3b_int8_gemm_dequant, 16,384 x 4,096 x 4,096
    quant_convrot              h3b_quantize_int8_rowwise_convrot, 65,536 x 4,096
    quant_gelu                 the same with the tanh-GELU input activation, 16,384 x 16,384
    rms_adaln                  h3b_rms_adaln_quantize_int8 (ConvRot), 65,536 x 4,096
    pool_q                     h3b_pool_sim_quant on the queries, L = 65,536, 32 heads, 128-row blocks
    mask                       h3b_block_mask (cdf 0.6 + first column + diagonal), L = 65,536, 32 heads
    qk_rope                    h3b_qk_rmsnorm_rope on QKV rows [65,536, 3 x 4,096], rotary width 128
    keys                       K mean + pool / similarity / INT8 (prepare_keys), L = 65,536, 32 heads
    values                     V absmax + FP8 transpose (prepare_values), L = 65,536, 32 heads
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from h3b import attention as A  # noqa: E402
from h3b import ops  # noqa: E402


def _case(name: str, g: torch.Generator):
    dev = "cuda"
    if name in ("attn_dense", "attn_sparse"):
        L, H = 65536, 8
        q, k, v = (torch.randn(L, H, 128, device=dev, generator=g).bfloat16() for _ in range(3))
        pk, _ = A.prepare_keys(k)
        pq, pv = A.prepare_queries(q), A.prepare_values(v)
        bm = (A.block_mask(pq, pk, A.MaskConfig("cdf", 0.6, keep_first_column=True, keep_diagonal=True))
              if name == "attn_sparse" else None)
        return lambda: A.attention(pq, pk, pv, bm)
    if name == "gemm":
        M, N, K = 16384, 4096, 4096
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        xs = torch.rand(M, device=dev, generator=g)
        ws = torch.rand(N, device=dev, generator=g)
        return lambda: ops.int8_linear_prequantized(a, xs, b, ws)
    if name == "quant_convrot":
        x = torch.randn(65536, 4096, device=dev, generator=g).bfloat16()
        return lambda: ops.quantize_int8_rowwise_convrot64(x, 256)
    if name == "quant_gelu":
        x = torch.randn(16384, 16384, device=dev, generator=g).bfloat16()
        return lambda: ops.quantize_int8_rowwise_convrot64(x, 256, "gelu_tanh")
    if name == "rms_adaln":
        x = torch.randn(65536, 4096, device=dev, generator=g).bfloat16()
        w = (1 + 0.05 * torch.randn(4096, device=dev, generator=g)).bfloat16()
        sc = (0.1 * torch.randn(4096, device=dev, generator=g)).bfloat16()
        sh = (0.1 * torch.randn(4096, device=dev, generator=g)).bfloat16()
        return lambda: ops.rms_adaln_quantize_int8(x, w, sc, sh, None, 1e-5, 256)
    if name in ("keys", "values"):
        x = torch.randn(65536, 32, 128, device=dev, generator=g).bfloat16()
        return (lambda: A.prepare_keys(x)) if name == "keys" else (lambda: A.prepare_values(x))
    if name in ("pool_q", "mask"):
        L, H = 65536, 32
        q, k = (torch.randn(L, H, 128, device=dev, generator=g).bfloat16() for _ in range(2))
        if name == "pool_q":
            return lambda: A.prepare_queries(q)
        pq = A.prepare_queries(q)
        pk, _ = A.prepare_keys(k)
        cfg = A.MaskConfig("cdf", 0.6, keep_first_column=True, keep_diagonal=True)
        return lambda: A.block_mask(pq, pk, cfg)
    if name == "qk_rope":
        L, H = 65536, 32
        qkv = torch.randn(L, 3 * H * 128, device=dev, generator=g).bfloat16()
        w = (1 + 0.05 * torch.randn(128, device=dev, generator=g)).bfloat16()
        ang = torch.rand(L, 64, device=dev, generator=g) * 6.0
        cos, sin = ang.cos().bfloat16(), ang.sin().bfloat16()
        return lambda: ops.qk_rmsnorm_rope_(qkv, H, 0, H * 128, w, w, cos, sin, 1e-6)
    raise SystemExit(f"unknown case {name!r}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--time", action="store_true")
    args = ap.parse_args()
    g = torch.Generator(device="cuda").manual_seed(0)
    fn = _case(args.case, g)
    if args.time:
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        print(f"{args.case}: {s.elapsed_time(e) / args.reps:.3f} ms per launch")
    else:
        for _ in range(args.reps):
            fn()
        torch.cuda.synchronize()
        print(f"{args.case}: ok")


if __name__ == "__main__":
    main()
