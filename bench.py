"""Benchmark: H3-shaped DiT block tokens/s at 720p/5 s (L = 111,600) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl h3b|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1: Ulysses)

A step is one forward of one DiT block (--layers blocks) over the whole 720p/5 s sequence:
rms_adaln + ConvRot INT8 quant, INT8 QKV GEMM, q/k RMSNorm + 3-D RoPE, Sparge
mask (top-CDF 0.6 + first column + diagonal) and quantized attention, INT8
out-projection with gated residual, W4A8 FC1 (G=128) -> GELU-tanh + ConvRot INT8
quant -> W4A8 FC2 with gated residual.  Random-init weights, synthetic N(0,1)
hidden states from one seed.  With N GPUs the sequence is split into N token
slices (strong scaling: total work fixed, every N times identical inputs and
masks), GEMMs run on local rows with no communication and attention uses NCCL
all-to-alls (tokens -> heads as three async exchanges of K, V, Q; heads ->
tokens), with heads assigned to ranks by the first warm-up step's kept tiles.

Prints ONE JSON line on rank 0 (see the keys below).  `value` is device-timed
with inputs resident in HBM; `e2e` adds the pinned host->device copy of each
step's hidden states and the device->host read of the result, through
h3b.block.HostPipeline (the copies of neighbouring steps overlap the block).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "x-minimaxh3_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "H3 DiT block tokens/s @720p5s INT8/W4A8; GEMM & attn % of B200 tensor peak"
GRID = (31, 45, 80)  # latent frames x patch rows x patch cols = 111,600 tokens


def workload_name(grid) -> str:
    names = {(31, 45, 80): "720p/5 s", (91, 68, 120): "1080p/15 s"}
    return "H3-shaped DiT block, " + names.get(tuple(grid), "grid %dx%dx%d" % tuple(grid))


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("h3b", "reference"), default="h3b")
    ap.add_argument("--tokens", type=int, default=0, help="override L (must divide by the GPU count)")
    ap.add_argument("--grid", type=str, default="", help="latent video grid T,H,W (default 31,45,80 = 720p/5 s; "
                    "91,68,120 = 1080p/15 s); L is its product unless --tokens is given")
    ap.add_argument("--layers", type=int, default=1, help="DiT blocks per step (BASELINE config 5: 4)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", type=str, default="",
                    help="run one kernel case instead of the block (for ncu captures and CUDA-event timing); "
                         "see KERNEL_CASES")
    ap.add_argument("--reps", type=int, default=2, help="launches of --case")
    ap.add_argument("--time", action="store_true", help="print the mean CUDA-event time of the --case launches")
    ap.add_argument("--kernel-table", action="store_true",
                    help="time every kernel of one block step alone at the bench shape (markdown table)")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ----------------------------------------------------------------------------- reference arm


def run_reference(args, L):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch

    from oracle import reference_cpu as R

    torch.set_num_threads(os.cpu_count() or 1)
    block = R.ReferenceBlockCPU()
    vals, walls = [], []
    info = None
    for i in range(args.warmup + args.steps):
        info = R.measure(L=L, row_sample=512, query_sample=512, block=block, seed=i)
        if i >= args.warmup:
            vals.append(info["seconds_per_block"] * args.layers)
            walls.append(info["sample_seconds"])
    sec = sorted(vals)[len(vals) // 2]
    wall = sorted(walls)[len(walls) // 2]
    value = L / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        # what each timed step actually ran: one bounded sample (see cpu_baseline.sample)
        "ms_per_step": wall * 1000.0,
        "extrapolated": {"ms_per_block_step": sec * 1000.0,
                         "how": "value = tokens / (the sample's time extrapolated to the whole block)"},
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 (dequantized weights, torch CPU)", "data": "synthetic",
        "config": {"workload": workload_name(args.grid_t), "tokens": L, "layers": args.layers, "hidden": 4096,
                   "heads": 32, "ffn": 16384,
                   "attention": "dense torch SDPA (the reference's CPU attention; the B200 arm runs Sparge)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": info["threads"], "kind": "port",
                         "sample": info["sample"] + f"; median of {args.steps} timed samples ({R.cpu_model()})"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- single-kernel cases

KERNEL_CASES = """
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
    w4_decode                  h3b_dequant_int4_grouped_to_int8, 16,384 x 4,096, G = 128
    gemm_gelu                  h3b_int8_gemm_gelu_convrot (GELU + ConvRot epilogue), 16,384 x 16,384 x 4,096
    quant_rotated              h3b_quantize_rotated_int8 on its output, 16,384 x 16,384
    adaln                      h3b_adaln_projection, weight 24,576 x 4,096 (6 x hidden), one timestep row
"""


def _kernel_case(name: str, g):
    """Seeded inputs for one kernel at a size that keeps an `ncu --set full` capture short
    (inputs larger than L2, a few GB on the device at most); returns the launch."""
    import torch

    from h3b import attention as A
    from h3b import ops

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
    if name == "w4_decode":
        N, K, G = 16384, 4096, 128
        qd = torch.randint(-128, 128, (N, K // 2), dtype=torch.int8, device=dev, generator=g)
        srel = torch.rand(N, K // G, device=dev, generator=g) * 20 + 1
        return lambda: ops.dequant_int4_grouped_to_int8(qd, srel, None, G)
    if name in ("gemm_gelu", "quant_rotated"):
        M, N, K = 16384, 16384, 4096
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        xs = torch.rand(M, device=dev, generator=g) * 1e-2
        ws = torch.rand(N, device=dev, generator=g) * 1e-2
        bias = torch.randn(N, device=dev, generator=g)
        rot = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        amax = torch.empty(M, N // 128, device=dev, dtype=torch.float32)
        from h3b._lib import check, lib
        stream = torch.cuda.current_stream().cuda_stream

        def fused():
            check(lib().h3b_int8_gemm_gelu_convrot(a.data_ptr(), b.data_ptr(), xs.data_ptr(), ws.data_ptr(), N,
                                                   bias.data_ptr(), rot.data_ptr(), M, N, K, N, amax.data_ptr(),
                                                   N // 128, stream), "gemm_gelu")
        if name == "gemm_gelu":
            return fused
        fused()
        return lambda: ops.quantize_rotated_int8(rot, amax)
    if name == "adaln":
        w = (torch.randn(6 * 4096, 4096, device=dev, generator=g) * 0.02).bfloat16()
        b = (torch.randn(6 * 4096, device=dev, generator=g) * 0.02).bfloat16()
        t = torch.randn(4096, device=dev, generator=g).bfloat16()
        return lambda: ops.adaln_projection(w, b, t)
    raise SystemExit(f"unknown case {name!r}; cases:{KERNEL_CASES}")


def run_case(args) -> int:
    import torch

    g = torch.Generator(device="cuda").manual_seed(0)
    fn = _kernel_case(args.case, g)
    if args.time:
        for _ in range(3):
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
    return 0


def _timed(fn, reps: int) -> float:
    import torch

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


def run_kernel_table(args, L) -> int:
    """Every kernel of one block step at the bench shape, each call timed alone with CUDA
    events over --reps launches after warm-up on inputs larger than L2, against its roofline:
    bytes that must cross HBM once (read + write) for the memory-bound kernels, 2 x
    multiply-adds for the tensor-core ones (the attention counts the tiles the bitmap keeps;
    fp32 multiply-adds for the mask's scores).  Peaks: HBM copy bandwidth, and twice the
    burst bf16 GEMM rate for INT8/FP8, from MEASURED_PEAKS.json (fallback figures if absent)."""
    import torch

    from h3b import attention as A
    from h3b import block as B
    from h3b import ops

    pk_, src = measured_peaks()
    hbm, tensor = float(pk_["hbm_gbs"]), 2.0 * float(pk_["bf16_tflops"])
    reps = max(args.reps, 3)
    cfg = B.BlockConfig()
    blk = B.DiTBlockB200(cfg, device="cuda", seed=0)
    D, F, H = cfg.hidden, cfg.ffn, cfg.heads
    W = H * cfg.head_dim
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(L, D, device="cuda", generator=g).to(torch.bfloat16)
    t = torch.randn(cfg.t_dim, device="cuda", generator=g).to(torch.bfloat16)
    rope = B.rope_tables(args.grid_t, cfg.rope_splits, device="cuda")
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

    ms = _timed(lambda: ops.rms_adaln_quantize_int8(x, blk.norm1, sc_a, sh_a, None, cfg.eps, 256), reps)
    row("rms_adaln + ConvRot INT8 quantizer (K 4096) x2", ms, L * D * 3 + L * 4, "hbm")
    xq, xs = ops.rms_adaln_quantize_int8(x, blk.norm1, sc_a, sh_a, None, cfg.eps, 256)
    qkv = torch.empty(L, 3 * W, device="cuda", dtype=torch.bfloat16)
    ms = _timed(lambda: blk.qkv.forward_prequantized_qk_rope(xq, xs, qkv, H, 0, W, blk.q_norm, blk.k_norm, rope[0],
                                                             rope[1], cfg.qk_eps), reps)
    row("QKV INT8 GEMM + dequant + q/k RMSNorm/RoPE epilogue (N 12288, K 4096)", ms, 2.0 * L * 3 * W * D, "tensor")
    view = qkv.view(L, 3, H, cfg.head_dim)
    q, k, v = view[:, 0], view[:, 1], view[:, 2]
    ms = _timed(lambda: A.prepare_values(v), reps)
    row("V -> FP8 (absmax, scale, transpose)", ms, L * W * 2 + L * W, "hbm")
    ms = _timed(lambda: A.prepare_keys(k), reps)
    row("K mean + pool / similarity / INT8", ms, 2 * L * W * 2 + L * W, "hbm")
    ms = _timed(lambda: A.prepare_queries(q), reps)
    row("Q pool / similarity / INT8", ms, L * W * 2 + L * W, "hbm")
    pv = A.prepare_values(v)
    pk, _ = A.prepare_keys(k)
    pq = A.prepare_queries(q)
    ms = _timed(lambda: A.block_mask(pq, pk, cfg.mask), reps)
    qb, kb = math.ceil(L / 128), math.ceil(L / 64)
    row("Sparge block mask (fp32 scores + selection)", ms, 2.0 * qb * kb * H * 128, "fma")
    bitmap = A.block_mask(pq, pk, cfg.mask)
    ms = _timed(lambda: A.attention(pq, pk, pv, bitmap), reps)
    row(f"attention (INT8 QK, FP8 PV; kept tiles {B.kept_tiles(bitmap, L) / (qb * kb * H):.3f})", ms,
        B.attention_ops(bitmap, L, L, H), "tensor")
    o2 = A.attention(pq, pk, pv, bitmap).view(L, W)
    ms = _timed(lambda: blk.out.quantize(o2), reps)
    row("ConvRot INT8 quantizer (out-proj input, K 4096)", ms, L * W * 3 + L * 4, "hbm")
    oq, os_ = blk.out.quantize(o2)
    xr = x.clone()
    ms = _timed(lambda: blk.out.gated_residual_(xr, ga[0], oq, os_), reps)
    row("out-proj INT8 GEMM + gated residual (N 4096, K 4096)", ms, 2.0 * L * D * W, "tensor")
    ms = _timed(lambda: blk.fc1.int8_weight(), reps)
    row("W4 -> INT8 decode, FC1 weight (16384 x 4096)", ms, F * D / 2 + F * (D // cfg.w4_group) * 4 + F * D, "hbm")
    xq2, xs2 = ops.rms_adaln_quantize_int8(x, blk.norm2, sc_m, sh_m, None, cfg.eps, 256)
    ms = _timed(lambda: blk.fc1.forward_prequantized(xq2, xs2), reps)
    row("FC1 W4A8 (decode + INT8 GEMM, N 16384, K 4096)", ms, 2.0 * L * F * D, "tensor")
    h = blk.fc1.forward_prequantized(xq2, xs2)
    ms = _timed(lambda: blk.fc2.quantize(h, cfg.mlp_act), reps)
    row("tanh-GELU + ConvRot INT8 quantizer (K 16384)", ms, L * F * 3 + L * 4, "hbm")
    hq, hs = blk.fc2.quantize(h, cfg.mlp_act)
    del h
    ms = _timed(lambda: blk.fc1.forward_prequantized_for(blk.fc2, xq2, xs2, cfg.mlp_act), reps)
    row("FC1 W4A8 with tanh-GELU + ConvRot epilogue, then codes (the block's path)", ms, 2.0 * L * F * D, "tensor")
    w8, ws8 = blk.fc1.int8_weight()
    rot = torch.empty(L, F, device="cuda", dtype=torch.bfloat16)
    amax = torch.empty(L, F // 128, device="cuda", dtype=torch.float32)
    b32 = blk.fc1.bias.float()
    from h3b._lib import lib as _lib
    stream = torch.cuda.current_stream().cuda_stream

    def fused_gemm():
        _lib().h3b_int8_gemm_gelu_convrot(xq2.data_ptr(), w8.data_ptr(), xs2.data_ptr(), ws8.data_ptr(),
                                          ws8.numel(), b32.data_ptr(), rot.data_ptr(), L, F, D, F,
                                          amax.data_ptr(), F // 128, stream)
    ms = _timed(fused_gemm, reps)
    row("  of which: INT8 GEMM + GELU + ConvRot epilogue (N 16384, K 4096)", ms, 2.0 * L * F * D, "tensor")
    ms = _timed(lambda: ops.quantize_rotated_int8(rot, amax), reps)
    row("  of which: rotated rows -> INT8 codes (K 16384)", ms, L * F * 3 + L * F // 128 * 4 + L * 4, "hbm")
    del rot, amax
    ms = _timed(lambda: blk.fc2.gated_residual_(xr, gm[0], hq, hs), reps)
    row("FC2 W4A8 + gated residual (N 4096, K 16384)", ms, 2.0 * L * D * F, "tensor")
    step = _timed(lambda: blk.forward(x.clone(), t, rope), 3)
    print(f"L = {L}, {torch.cuda.get_device_name()}; peaks ({src}): HBM {hbm:,.0f} GB/s, "
          f"INT8/FP8 {tensor:,.0f} TOPS (2 x bf16 burst)\n")
    print("| kernel (one call) | ms | work | achieved | of peak |")
    print("|---|---:|---:|---:|---:|")
    for name, ms, work, ach, frac in rows:
        print(f"| {name} | {ms:.3f} | {work} | {ach} | {'-' if frac is None else f'{frac:.2f}'} |")
    print(f"\nblock forward (all of the above, norm quantizer twice, x.clone() included): {step:.2f} ms")
    return 0


# ----------------------------------------------------------------------------- host placement


def _bind_near_gpu(local: int) -> bool:
    """Restrict this process to the host cores NVML reports as nearest GPU `local` (best
    effort: returns False and changes nothing when NVML or the affinity call is unavailable)."""
    try:
        import pynvml
        import torch

        p = torch.cuda.get_device_properties(local)
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0")
        words = (os.cpu_count() + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(handle, words)
        cpus = {64 * w + b for w, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return False
        os.sched_setaffinity(0, cpus)
        return True
    except Exception:
        return False


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"h3b_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        try:
            for line in open(self.path):
                f = [c.strip() for c in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = max(mx, float(f[2]))
                except ValueError:
                    continue
                for name, val in zip(names, f[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        except OSError:
            return None
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- B200 arm


def run_h3b(args, L):
    import torch
    import torch.distributed as dist

    import h3b
    from h3b import _lib
    from h3b.block import BlockConfig, DiTBlockB200, attention_ops, rope_tables

    world = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    bound = False
    if world > 1:
        # each rank copies its own rows to and from pinned host memory every step (e2e):
        # keep the process, and so that memory, on the host cores nearest its GPU
        bound = _bind_near_gpu(local)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD
        if dist.get_world_size() != world:
            raise SystemExit("--gpus does not match the launched world size")
    if L % world:
        raise SystemExit(f"{L} tokens do not split over {world} ranks")
    Lp = L // world
    cfg = BlockConfig()
    blocks = [DiTBlockB200(cfg, device=dev, seed=layer, group=group) for layer in range(args.layers)]
    # one global input from one seed, each rank taking its own token rows: every N times
    # the same work and the same masks
    g = torch.Generator(device=dev).manual_seed(1234)
    x_full = torch.randn(L, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    t = torch.randn(cfg.t_dim, generator=g, device=dev).to(torch.bfloat16)
    x0 = x_full[rank * Lp:(rank + 1) * Lp].clone()
    del x_full
    rope = rope_tables(args.grid_t, cfg.rope_splits, start=rank * Lp, count=Lp, device=dev)
    x = torch.empty_like(x0)

    # instrument the dominant kernel (the quantized attention) with CUDA events
    # on the stream it is launched on
    from h3b import attention as A
    attn_events = []
    orig_attention = A.attention

    def timed_attention(*a, **kw):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        out = orig_attention(*a, **kw)
        e.record()
        attn_events.append((s, e))
        return out

    import h3b.block as B
    B.A.attention = timed_attention

    def step():
        x.copy_(x0)
        for blk in blocks:
            blk.forward(x, t, rope)

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        step()
        if i == 0 and world > 1:
            # assign heads to ranks by the kept tiles the first step measured (the
            # blocks' outputs do not depend on the assignment)
            for blk in blocks:
                blk.rebalance_heads()
    torch.cuda.synchronize()
    barrier()
    attn_events.clear()
    _lib.reset_launch_count()
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    s_ev = torch.cuda.Event(enable_timing=True)
    e_ev = torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(args.steps):
        step()
    e_ev.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks else None
    launches = _lib.launch_count()
    ms = s_ev.elapsed_time(e_ev) / args.steps
    attn_ms = sum(a.elapsed_time(b) for a, b in attn_events) / max(1, len(attn_events))
    # executed tensor ops of one attention launch (this rank's heads), averaged over layers
    attn_ops_launch = sum(attention_ops(b._last_attn[3], b._last_attn[0].tokens, b._last_attn[1].tokens,
                                        b._last_attn[0].qi8.shape[0]) for b in blocks) / len(blocks)
    pq0, pk0 = blocks[0]._last_attn[0], blocks[0]._last_attn[1]
    rank_attn = None
    if world > 1:
        tmax = torch.tensor([ms, attn_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        per = [torch.zeros(2, device=dev, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(per, torch.tensor([attn_ms, attn_ops_launch], device=dev, dtype=torch.float64))
        rank_attn = [(float(p[0]), float(p[1])) for p in per]
        ms = float(tmax[0])
    status = h3b.device_status(local)

    # end-to-end through the public host-side runner (h3b.block.HostPipeline):
    # every step copies its hidden states from pinned host memory to the GPU,
    # runs the block and copies the result back; the copies of neighbouring
    # steps overlap the block on their own streams
    e2e = None
    if not args.no_e2e and args.layers == 1:
        from h3b.block import HostPipeline
        xh = x0.cpu().pin_memory()
        th = t.cpu().pin_memory()
        outs = [torch.empty_like(xh).pin_memory() for _ in range(2)]
        pipe = HostPipeline(blocks[0], rope, Lp)
        pipe.run([xh] * 2, [th] * 2, outs)                      # warm-up
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        s2 = torch.cuda.Event(enable_timing=True)
        e2 = torch.cuda.Event(enable_timing=True)
        s2.record()
        pipe.run([xh] * args.steps, [th] * args.steps, [outs[k % 2] for k in range(args.steps)])
        e2.record()
        torch.cuda.synchronize()
        out_h = outs[0]
        e2e_ms = s2.elapsed_time(e2) / args.steps
        if world > 1:
            tm = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            e2e_ms = float(tm[0])
        e2e = {"value": L / (e2e_ms / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": xh.numel() * xh.element_size() + th.numel() * th.element_size(),
               "d2h_bytes_per_step": out_h.numel() * out_h.element_size(), "ms_per_step": e2e_ms}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import reference_cpu as R

        torch.set_num_threads(os.cpu_count() or 1)
        rb = R.ReferenceBlockCPU()
        samples = []
        t_end = time.time() + 15.0
        info = None
        while time.time() < t_end or not samples:
            info = R.measure(L=L, row_sample=512, query_sample=512, block=rb, seed=len(samples))
            samples.append(info["seconds_per_block"] * args.layers)
        sec = sorted(samples)[len(samples) // 2]
        cpu = {"value": L / sec, "unit": "tokens/s", "cores": info["threads"], "kind": "port",
               "sample": info["sample"] + f"; median of {len(samples)} samples ({R.cpu_model()})"}

    if rank == 0:
        peaks, src = measured_peaks()
        peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
        achieved = attn_ops_launch / (attn_ms / 1000.0) / 1e12
        traffic = None
        prof = os.path.join(ROOT, "profiles", "attn_traffic.json")
        if os.path.exists(prof):
            try:
                prof_d = json.load(open(prof))
                # the capture is scaled to the default workload's launch only
                if L == GRID[0] * GRID[1] * GRID[2] and world == 1:
                    traffic = prof_d.get("bytes_per_launch_scaled")
            except (OSError, ValueError):
                traffic = None
        heads_local = pq0.qi8.shape[0]
        dense_ops = 4.0 * 128 * 64 * 128 * math.ceil(pq0.tokens / 128) * math.ceil(pk0.tokens / 64) * heads_local
        density = attn_ops_launch / dense_ops
        line = {
            "metric": METRIC, "value": L / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 (W8A8 / W4A8 GEMMs), int8-QK / fp8-PV attention",
            "data": "synthetic (N(0,1) hidden states from one seed, each rank its token rows; random-init "
                    "H3-format weights)",
            "config": {"workload": workload_name(args.grid_t) + " (BASELINE configs 1-4 combined in one block)",
                       "tokens": L, "layers": args.layers, "grid": list(args.grid_t), "hidden": cfg.hidden,
                       "heads": cfg.heads, "ffn": cfg.ffn, "mlp": f"W4A8 G={cfg.w4_group} {cfg.mlp_act}",
                       "attention": f"Sparge {cfg.mask.mode} {cfg.mask.budget} + first column + diagonal",
                       "kept_tile_fraction": round(density, 4),
                       "parallelism": f"ulysses{world}" if world > 1 else "single",
                       "host_cores": "nearest the GPU (NVML affinity)" if bound else "all",
                       "l2": "inputs larger than L2 (hidden 914 MB, weights 33-100 MB per layer)"},
            "roofline": {"bound": "tensor", "kernel": "h3b attn_kernel (tcgen05 int8 QK + fp8 PV)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"2 x bf16_tflops (burst) of {src} (int8/fp8 dense rate is twice bf16)",
                         "traffic": traffic, "attn_ms_per_launch": attn_ms, "ops_per_launch": attn_ops_launch},
            "gpu_launches": launches,
            "device_status": status,
        }
        if rank_attn:
            times = [a for a, _ in rank_attn]
            line["ranks"] = {"attn_ms_per_launch": [round(a, 3) for a in times],
                             "attn_ops_per_launch": [o for _, o in rank_attn],
                             "attn_max_over_mean": max(times) / (sum(times) / len(times)),
                             "head_assignment": "balanced by the kept tiles of the first warm-up step"}
        if e2e:
            line["e2e"] = e2e
        if cpu:
            line["cpu_baseline"] = cpu
        if clk:
            line["clocks"] = clk
        print(json.dumps(line), flush=True)
    B.A.attention = orig_attention
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    args.grid_t = tuple(int(v) for v in args.grid.split(",")) if args.grid else GRID
    if len(args.grid_t) != 3 or min(args.grid_t) <= 0:
        raise SystemExit("--grid takes three positive integers T,H,W")
    L = args.tokens or args.grid_t[0] * args.grid_t[1] * args.grid_t[2]
    if args.case:
        return run_case(args)
    if args.kernel_table:
        return run_kernel_table(args, L)
    if args.impl == "reference":
        return run_reference(args, L)
    return run_h3b(args, L)


if __name__ == "__main__":
    sys.exit(main())
