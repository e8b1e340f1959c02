"""Benchmark: H3-shaped DiT block tokens/s at 720p/5 s (L = 111,600) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl h3b|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1: Ulysses)

A step is one forward of one DiT block over the whole 720p/5 s sequence:
rms_adaln + ConvRot INT8 quant, INT8 QKV GEMM, q/k RMSNorm + 3-D RoPE, Sparge
mask (top-CDF 0.6 + first column + diagonal) and quantized attention, INT8
out-projection with gated residual, W4A8 FC1 (G=128) -> GELU-tanh + ConvRot INT8
quant -> W4A8 FC2 with gated residual.  Random-init weights, synthetic N(0,1)
hidden states.  With N GPUs the sequence is split into N token slices (strong
scaling: total work fixed), GEMMs run on local rows with no communication and
attention uses a NCCL all-to-all (tokens -> heads and back).

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
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    vals = []
    info = None
    for i in range(args.warmup + args.steps):
        info = R.measure(L=L, row_sample=512, query_sample=512, block=block, seed=i)
        if i >= args.warmup:
            vals.append(info["seconds_per_block"])
    sec = sorted(vals)[len(vals) // 2]
    value = L / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1000.0, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 (dequantized weights, torch CPU)",
        "data": "synthetic", "config": {"workload": workload_name(args.grid_t), "tokens": L,
                                         "hidden": 4096, "heads": 32, "ffn": 16384, "attention": "dense SDPA (CPU)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": info["threads"], "kind": "port",
                         "sample": info["sample"] + "; median of the timed steps"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


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
    block = DiTBlockB200(cfg, device=dev, seed=0, group=group)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    x0 = torch.randn(Lp, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    t = torch.randn(cfg.t_dim, generator=g, device=dev).to(torch.bfloat16)
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
        block.forward(x, t, rope)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
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
    pq, pk, pv, bitmap = block._last_attn
    attn_ops_launch = attention_ops(bitmap, pq.tokens, pk.tokens, pq.qi8.shape[0])
    if world > 1:
        tmax = torch.tensor([ms, attn_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        ms, attn_ms = float(tmax[0]), float(tmax[1])
    status = h3b.device_status(local)

    # end-to-end through the public host-side runner (h3b.block.HostPipeline):
    # every step copies its hidden states from pinned host memory to the GPU,
    # runs the block and copies the result back; the copies of neighbouring
    # steps overlap the block on their own streams
    e2e = None
    if not args.no_e2e:
        from h3b.block import HostPipeline
        xh = x0.cpu().pin_memory()
        th = t.cpu().pin_memory()
        outs = [torch.empty_like(xh).pin_memory() for _ in range(2)]
        pipe = HostPipeline(block, rope, Lp)
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
            samples.append(info["seconds_per_block"])
        sec = sorted(samples)[len(samples) // 2]
        cpu = {"value": L / sec, "unit": "tokens/s", "cores": info["threads"], "kind": "port",
               "sample": info["sample"] + f"; median of {len(samples)} samples ({R.cpu_model()})"}

    if rank == 0:
        peaks, src = measured_peaks()
        peak = 2.0 * float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1400.0)))
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
        density = attn_ops_launch / (4.0 * 128 * 64 * 128 * math.ceil(pq.tokens / 128) * math.ceil(pk.tokens / 64)
                                     * pq.qi8.shape[0])
        line = {
            "metric": METRIC, "value": L / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 (W8A8 / W4A8 GEMMs), int8-QK / fp8-PV attention",
            "data": "synthetic (N(0,1) hidden states, random-init H3-format weights)",
            "config": {"workload": workload_name(args.grid_t) + " (BASELINE configs 1-4 combined in one block)",
                       "tokens": L, "grid": list(args.grid_t), "hidden": cfg.hidden, "heads": cfg.heads,
                       "ffn": cfg.ffn, "mlp": f"W4A8 G={cfg.w4_group} {cfg.mlp_act}",
                       "attention": f"Sparge {cfg.mask.mode} {cfg.mask.budget} + first column + diagonal",
                       "kept_tile_fraction": round(density, 4),
                       "parallelism": f"ulysses{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (hidden 914 MB, weights 33-100 MB per layer)"},
            "roofline": {"bound": "tensor", "kernel": "h3b attn_kernel (tcgen05 int8 QK + fp8 PV)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"2 x bf16_tflops_sustained of {src} (int8/fp8 dense rate is twice bf16)",
                         "traffic": traffic, "attn_ms_per_launch": attn_ms,
                         "ops_per_launch": attn_ops_launch},
            "gpu_launches": launches,
            "device_status": status,
        }
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
    if args.impl == "reference":
        return run_reference(args, L)
    return run_h3b(args, L)


if __name__ == "__main__":
    sys.exit(main())
