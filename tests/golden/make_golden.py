"""Generate golden vectors from the reference's own importable Python code.

Run once in a container that has the X-MinimaxH3 sources (read-only), passing
their location as the first argument or in REFERENCE_ROOT; the resulting *.npz fixtures are
committed and are the only thing the tests read.  Every fixture records the
reference function that produced it:

  quant_rowwise.npz   comfy_kitchen eager quantize_int8_rowwise
                      (backends/eager/quantization.py:857-875)
  convrot.npz         comfy_kitchen eager _rotate_activation / quantize_and_rotate_rowwise
                      (tensor/int8_utils.py:11-74, eager/quantization.py:878-895)
  input_act.npz       comfy_kitchen apply_input_act (backends/_activations.py:41-53)
  w4_decode.npz       comfy_kitchen eager _dequant_int4_grouped_to_int8 (eager/w4a8_int8.py:344-363)
  linear.npz          eager int8_linear (eager/quantization.py:971-1062), ConvRotInt8Linear
                      and ConvRotW4A8Linear CPU fallbacks (model/quantization.py:278-304, 557-586)
  sparge_pool.npz     sparge_nhd.pool_sim_quant_nhd + hnd_compatible_key_mean_nhd under
                      TRITON_INTERPRET=1 (model/sparge_nhd.py:26-227)
  lut.npz             sparse_lut block_map_to_absolute_lut / absolute_lut_to_delta under
                      TRITON_INTERPRET=1 (model/sparse_lut.py:25-74)
  block_ckpt.npz      assemble_pruned_block + H3TransformerBlock.forward on CPU (no kernels
                      injected: the ConvRotInt8Linear / ConvRotW4A8Linear float fallbacks,
                      torch_sdpa attention; model/assembly.py:259-333, layers.py:996-1298) over
                      the synthetic checkpoint of tests/golden/h3_checkpoint.py, plus each
                      layer's output on a seeded input and the layer class / spec chosen
  rms_adaln.npz       RMSNorm module (F.rms_norm) + kernels.rms_adaln's eager segmented
                      modulation on CPU bf16 rows (model/layers.py:33-49, kernels.py:7594-7642),
                      hidden 5376 and 4096, three modulation segments
  qk_rope.npz         apply_qknorm_rope on CPU bf16 tensors with the engine's packed split-half
                      rotation table (model/layers.py:60-118: rope_rotation_table, F.rms_norm,
                      rotate_table), rotary widths 128 and 96
  sage_k_per_thread.npz  sage_fused_quant.quantize_key_sub_mean_per_thread_int8 under
                      TRITON_INTERPRET=1 (model/sage_fused_quant.py:20-162), Lk 197 / 64 / 1000
  mask_topk.npz       SplitModalityProtectedSpargeAttentionBackend.long_sequence_video_queries
                      (model/kernels.py:3668-3997) with the two absent Sparge helpers replaced
                      by recorders (fill: set the first `count` sorted indices; LUT: capture
                      the final block map), the same injection the reference tests use
                      (tests/native_engine/test_model_optimizations.py:532-569)

Usage:  python tests/golden/make_golden.py [REFERENCE_ROOT [gen_name ...]]
"""

from __future__ import annotations

import os
import sys
import types

import numpy as np

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", "")
if not REF or not os.path.isdir(REF):
    raise SystemExit("usage: make_golden.py <X-MinimaxH3 checkout> (or set REFERENCE_ROOT)")
os.environ["TRITON_INTERPRET"] = "1"
sys.path[:0] = [os.path.join(REF, "backends/turbo/vendor"), REF]

import torch  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def save(name, **arrays):
    np.savez_compressed(os.path.join(OUT, name), **arrays)
    print("wrote", name, {k: getattr(v, "shape", v) for k, v in arrays.items()})


def outlier_activations(g, m, k, frac=0.01, mult=20.0):
    x = torch.randn(m, k, generator=g)
    nout = max(1, int(round(k * frac)))
    cols = torch.randperm(k, generator=g)[:nout]
    x[:, cols] *= mult
    return x


def gen_quant():
    from comfy_kitchen.backends.eager.quantization import quantize_int8_rowwise

    g = torch.Generator().manual_seed(0)
    x = outlier_activations(g, 61, 512).to(torch.bfloat16)
    x[0] = 0.0                      # all-zero row: scale clamps to 1e-30
    x[1, :] = 1e-30                 # tiny row
    x[2, 7] = 3.0e38                # near the bf16 finite maximum
    x[3] = torch.linspace(-127, 127, 512).to(torch.bfloat16)  # exact ties after division
    q, s = quantize_int8_rowwise(x)
    save("quant_rowwise.npz", x=bits(x), q=q.numpy(), scale=s.reshape(-1).numpy())


def gen_convrot():
    from comfy_kitchen.tensor.int8_utils import _build_hadamard, _rotate_activation
    from comfy_kitchen.backends.eager.quantization import quantize_and_rotate_rowwise

    g = torch.Generator().manual_seed(1)
    x = outlier_activations(g, 24, 1024).to(torch.bfloat16)
    h32 = _build_hadamard(256, device="cpu", dtype=torch.float32)
    rot32 = _rotate_activation(x.float(), h32, 256)
    hb = _build_hadamard(256, device="cpu", dtype=torch.bfloat16)
    q, s = quantize_and_rotate_rowwise(x, hb, 256)
    save("convrot.npz", x=bits(x), rot_f32=rot32.numpy(), q_eager=q.numpy(), scale_eager=s.reshape(-1).numpy())


def gen_act():
    from comfy_kitchen.backends._activations import apply_input_act

    g = torch.Generator().manual_seed(2)
    x = (torch.randn(16, 512, generator=g) * 3).to(torch.bfloat16)
    gelu = apply_input_act(x.float(), "gelu_tanh")
    sw = apply_input_act(x.float(), "swiglu")
    save("input_act.npz", x=bits(x), gelu_f32=gelu.numpy(), swiglu_f32=sw.numpy())


def gen_w4():
    from comfy_kitchen.backends.eager.w4a8_int8 import _dequant_int4_grouped_to_int8

    g = torch.Generator().manual_seed(3)
    cases = {}
    for tag, n, k, G, cb, e4m3 in (
        ("g4_codebook_e4m3", 48, 256, 4, True, True),
        ("g16_uniform_f32", 40, 512, 16, False, False),
        ("g128_uniform_f32", 32, 1024, 128, False, False),
        ("g16_codebook_e4m3", 24, 512, 16, True, True),
    ):
        qdata = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int16).to(torch.int8)
        srel = torch.rand(n, k // G, generator=g) * 30 + 0.5
        if e4m3:
            srel_t = srel.to(torch.float8_e4m3fn)
            srel_store = srel_t.view(torch.uint8).numpy()
        else:
            srel_t = srel
            srel_store = srel.numpy()
        codebook = torch.linspace(-7.5, 7.5, 16) if cb else None
        out = _dequant_int4_grouped_to_int8(qdata, srel_t, codebook, G)
        cases[tag + "_qdata"] = qdata.numpy()
        cases[tag + "_srel"] = srel_store
        cases[tag + "_codebook"] = codebook.numpy() if cb else np.zeros(0, np.float32)
        cases[tag + "_G"] = np.array(G)
        cases[tag + "_out"] = out.numpy()
    save("w4_decode.npz", **cases)


def gen_linear():
    from comfy_kitchen.backends.eager.quantization import int8_linear, quantize_int8_rowwise
    from comfy_kitchen.backends.eager.w4a8_int8 import w4a8_int8_linear
    from h3serve.native_engine.model.quantization import (
        ComfyQuantSpec, ConvRotInt8Linear, ConvRotW4A8Linear, W4A8QuantSpec)

    g = torch.Generator().manual_seed(0)
    M, K, N = 96, 512, 160
    x = outlier_activations(g, M, K).to(torch.bfloat16)
    w = torch.randn(N, K, generator=g) * 0.02
    wq, ws = quantize_int8_rowwise(w)
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    ws = ws.reshape(-1)
    out_eager = int8_linear(x, wq, ws, bias, torch.bfloat16, convrot=False)
    out_eager_rot = int8_linear(x, wq, ws, bias, torch.bfloat16, convrot=True, convrot_groupsize=256)
    mod = ConvRotInt8Linear(wq, ws, bias, spec=ComfyQuantSpec("int8_tensorwise", True, 256))
    out_module_rot = mod(x)
    # W4A8: symmetric int4 groups of 128 (the benchmark format), s_rel = group/channel scale in fp32
    G = 128
    wg = (torch.randn(N, K, generator=g) * 0.02).view(N, K // G, G)
    gscale = wg.abs().amax(-1) / 7.0
    cscale = gscale.amax(-1) / 127.0
    codes = torch.clamp(torch.round(wg / gscale.unsqueeze(-1)), -8, 7).to(torch.int32) + 8
    codes = codes.view(N, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)
    s_rel = (gscale / cscale.unsqueeze(-1)).float()
    s_ch = cscale.float()
    out_w4_eager = w4a8_int8_linear(x, packed, s_rel, s_ch, None, None, bias, G, 256, torch.bfloat16)
    w4mod = ConvRotW4A8Linear(packed, s_rel, s_ch, bias=bias, spec=W4A8QuantSpec("asym_w4a8_int8", G, True, 256))
    out_w4_module = w4mod(x)
    save("linear.npz", x=bits(x), wq=wq.numpy(), ws=ws.numpy(), bias=bits(bias),
         out_eager=bits(out_eager), out_eager_rot=bits(out_eager_rot),
         out_module_rot=bits(out_module_rot), w4_qdata=packed.numpy(), w4_srel=s_rel.numpy(),
         w4_sch=s_ch.numpy(), w4_G=np.array(G), out_w4_eager=bits(out_w4_eager),
         out_w4_module=bits(out_w4_module))


def gen_sparge():
    from h3serve.native_engine.model.sparge_nhd import hnd_compatible_key_mean_nhd, pool_sim_quant_nhd

    # Shapes and distribution of tests/native_engine/test_sage_fused_quant.py (seed 82736,
    # Lq=131, Lk=197, H=4, D=128, K = N(0,1)*0.125 + 5).
    g = torch.Generator().manual_seed(82736)
    H, D, Lq, Lk = 4, 128, 131, 197
    q = torch.randn(1, Lq, H, D, generator=g).to(torch.bfloat16)
    k = (torch.randn(1, Lk, H, D, generator=g) * 0.125 + 5).to(torch.bfloat16)
    thr = torch.full((H,), -0.1)
    pq, sq, qq, qs = pool_sim_quant_nhd(q, None, 128, thr)
    kmean = hnd_compatible_key_mean_nhd(k)
    # The fused-mean branch of the kernel does not run correctly under the Triton
    # interpreter (NaN pools); its first step is the bf16 store boundary
    # value = bf16(k - mean), so the smoothed K is formed here with the same bf16
    # subtraction and fed through the kernel's mean-free branch.
    k_smoothed = k - kmean
    pk, sk, kq, ks = pool_sim_quant_nhd(k_smoothed, None, 64, thr)
    # a block-structured case whose similarity decisions are far from the threshold
    kb = torch.randn(1, 8, H, D, generator=g).repeat_interleave(32, dim=1)
    kb = (kb + 0.01 * torch.randn(kb.shape, generator=g)).to(torch.bfloat16)
    thr2 = torch.tensor([0.5, 0.9, 0.99, -0.1])
    pb, sb, qb, sbs = pool_sim_quant_nhd(kb, None, 64, thr2)
    save("sparge_pool.npz", q=bits(q[0]), k=bits(k[0]), kmean=bits(kmean[0, 0]),
         pq=bits(pq[0]), sq=sq[0].numpy().astype(np.uint8), qq=qq[0].numpy(), qs=qs[0].numpy(),
         pk=bits(pk[0]), sk=sk[0].numpy().astype(np.uint8), kq=kq[0].numpy(), ks=ks[0].numpy(),
         kb=bits(kb[0]), thr2=thr2.numpy(), pb=bits(pb[0]), sb=sb[0].numpy().astype(np.uint8),
         qb=qb[0].numpy(), sbs=sbs[0].numpy())


def gen_sage_k():
    """Sage per_thread K quantization with mean smoothing: the in-tree Triton kernel
    (model/sage_fused_quant.py:20-162) under the interpreter, on the reference test's
    ragged non-zero-mean inputs (tests/native_engine/test_sage_fused_quant.py:14-38)."""
    from h3serve.native_engine.model.sage_fused_quant import quantize_key_sub_mean_per_thread_int8

    g = torch.Generator().manual_seed(82736)
    H, D = 4, 128
    out = {}
    for Lk in (197, 64, 1000):
        k = (torch.randn(1, Lk, H, D, generator=g) * 0.125 + 5.0).to(torch.bfloat16)
        kmean = k.mean(dim=1, keepdim=True)
        q8 = torch.empty_like(k, dtype=torch.int8)
        sc = torch.empty((1, H, (Lk + 63) // 64 * 4), dtype=torch.float32)
        # The interpreter keeps bf16 as raw uint16 and subtracts the bit patterns;
        # fp32 copies of the same bf16 values reproduce the kernel's arithmetic
        # exactly: the fp32 difference of two bf16 numbers of this range is exact,
        # and the kernel's own .to(bf16) then rounds it as on the GPU.
        quantize_key_sub_mean_per_thread_int8(k.float(), kmean.float(), q8, sc)
        out[f"k{Lk}"] = bits(k[0])
        out[f"kmean{Lk}"] = bits(kmean[0, 0])
        out[f"kq{Lk}"] = q8[0].numpy()
        out[f"ks{Lk}"] = sc[0].numpy()
    save("sage_k_per_thread.npz", **out)


def gen_rms_adaln():
    from h3serve.native_engine.model.kernels import rms_adaln
    from h3serve.native_engine.model.layers import RMSNorm

    g = torch.Generator().manual_seed(94)
    arrays = {}
    for K in (5376, 4096):
        rows = 16
        x = (torch.randn(rows, K, generator=g) * 2).to(torch.bfloat16)
        x[5] *= 40.0                                            # a row far from unit scale
        norm = RMSNorm(K, eps=1e-5, dtype=torch.bfloat16)
        with torch.no_grad():
            norm.weight.copy_((1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16))
        scale = (0.2 * torch.randn(3, K, generator=g)).to(torch.bfloat16)
        shift = (0.2 * torch.randn(3, K, generator=g)).to(torch.bfloat16)
        segments = ((0, 4, 2), (4, 9, 0), (9, rows, 1))
        with torch.no_grad():
            out = rms_adaln(x.clone(), norm, shift, scale, segments)
        arrays.update({f"k{K}_x": bits(x), f"k{K}_w": bits(norm.weight.detach()), f"k{K}_scale": bits(scale),
                       f"k{K}_shift": bits(shift), f"k{K}_segments": np.array(segments, np.int64),
                       f"k{K}_out": bits(out)})
    save("rms_adaln.npz", **arrays)


def gen_qk_rope():
    from h3serve.native_engine.model.layers import apply_qknorm_rope, rope_rotation_table

    g = torch.Generator().manual_seed(72)
    L, H = 67, 3
    arrays = {}
    for rot in (128, 96):
        q = (torch.randn(L, H, 128, generator=g) * 2).to(torch.bfloat16)
        k = (torch.randn(L, H, 128, generator=g) * 2 + 0.5).to(torch.bfloat16)
        qw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
        kw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
        angles = torch.rand(L, rot, generator=g) * 6        # split-half: the first rot/2 are used
        table = rope_rotation_table(angles, torch.bfloat16)
        qo, ko = apply_qknorm_rope(q, k, q_weight=qw, k_weight=kw, frequencies=table, eps=1e-6)
        half = rot // 2
        arrays.update({f"r{rot}_q": bits(q), f"r{rot}_k": bits(k), f"r{rot}_qw": bits(qw), f"r{rot}_kw": bits(kw),
                       f"r{rot}_cos": bits(table[0, :, 0, :, 0, 0].contiguous()),
                       f"r{rot}_sin": bits(table[0, :, 0, :, 1, 0].contiguous()),
                       f"r{rot}_qo": bits(qo), f"r{rot}_ko": bits(ko),
                       f"r{rot}_angles": angles.numpy(), f"r{rot}_table": bits(table)})
        assert table.shape[3] == half
    save("qk_rope.npz", **arrays)


def gen_lut():
    from h3serve.native_engine.model.sparse_lut import _parallel_lut_kernels

    g = torch.Generator().manual_seed(5)
    B, H, Qb, Kb = 1, 3, 5, 77
    bm = torch.rand(B, H, Qb, Kb, generator=g) < 0.3
    bm[0, 0, 0] = False
    bm[0, 1, 2] = True
    triton, compact, delta = _parallel_lut_kernels()
    block = triton.next_power_of_2(Kb)
    rows = B * H * Qb
    absl = torch.zeros(bm.shape, dtype=torch.int32)
    lut = torch.zeros(bm.shape, dtype=torch.int32)
    valid = torch.zeros((B, H, Qb), dtype=torch.int32)
    compact[(rows,)](bm, absl, valid, key_blocks=Kb, BLOCK=block)
    delta[(rows,)](absl, lut, valid, key_blocks=Kb, BLOCK=block)
    save("lut.npz", block_map=bm[0].numpy(), lut=lut[0].numpy(), valid=valid[0].numpy())


def gen_mask():
    from h3serve.native_engine.model import kernels as K
    from h3serve.native_engine.model.kernels import (
        PreparedLongSequenceKV, SplitModalityProtectedSpargeAttentionBackend)

    captured = {}

    def fill_block_map_triton(block_map, num_to_select, sorted_indices):
        rows = block_map.view(-1, block_map.shape[-1])
        counts = num_to_select.reshape(-1)
        idx = sorted_indices.reshape(-1, sorted_indices.shape[-1])
        for r in range(rows.shape[0]):
            rows[r, idx[r, : int(counts[r])]] = True
        return block_map

    def block_map_lut_triton(block_map):
        captured["block_map"] = block_map.clone()
        return torch.zeros(1), torch.zeros(1)

    def hyperparameter_check(value, heads, device):
        return torch.full((heads,), float(value), device=device)

    def core_fn(*args, **kwargs):
        captured["core_args"] = True

    utils = types.SimpleNamespace(
        block_map_lut_triton=block_map_lut_triton, fill_block_map_triton=fill_block_map_triton,
        get_pool_sim_triton_simmean_fuse_quant=None, hyperparameter_check=hyperparameter_check)
    core = types.SimpleNamespace(
        qk_int8_sv_f8_accum_f16_block_sparse_attn_inst_buf_fuse_v_scale_with_pv_threshold=core_fn)
    pkg = types.ModuleType("spas_sage_attn")
    pkg.core = core
    pkg.utils = utils
    sys.modules["spas_sage_attn"] = pkg
    sys.modules["spas_sage_attn.core"] = core
    sys.modules["spas_sage_attn.utils"] = utils

    # Block-constant integer-valued Q and K rows: pooled vectors are exact, every
    # pooled score is an exact small integer, and the scores are distinct, so
    # the selection has no ties and no summation-order sensitivity.
    g = torch.Generator().manual_seed(7)
    H, D = 2, 128
    Lq, Lk = 128 * 6 + 40, 64 * 23 + 17          # ragged tails on both sides
    Qb, Kb = (Lq + 127) // 128, (Lk + 63) // 64
    basis = torch.zeros(Kb, D)
    for j in range(Kb):
        basis[j, j % D] = 1.0
    qvec = torch.zeros(H, Qb, D)
    kvec = torch.zeros(H, Kb, D)
    for h in range(H):
        for i in range(Qb):
            perm = torch.randperm(Kb, generator=g)
            qvec[h, i, :Kb] = (perm.float() * 2.0 - Kb) / 8.0
        kvec[h] = basis * 8.0
    q = torch.zeros(Lq, H, D)
    k = torch.zeros(Lk, H, D)
    for h in range(H):
        for i in range(Qb):
            q[i * 128:(i + 1) * 128, h] = qvec[h, i]
        for j in range(Kb):
            k[j * 64:(j + 1) * 64, h] = kvec[h, j]
    q = q.to(torch.bfloat16)
    k = k.to(torch.bfloat16)
    from h3serve.native_engine.model.sparge_nhd import pool_sim_quant_nhd

    thr = torch.full((H,), -0.1)
    pk, sk, kq, ks = pool_sim_quant_nhd(k.unsqueeze(0), None, 64, thr)
    results = {"q": bits(q), "k": bits(k)}
    for topk in (0.5, 0.75):
        for protected in (0, 100):
            backend = SplitModalityProtectedSpargeAttentionBackend(topk)
            prepared = PreparedLongSequenceKV(
                key=None, key_mean=torch.zeros(1, 1, H, D), pooled_key=pk, similar_key_blocks=sk,
                key_int8=kq, key_scale=ks, prefix_key_int8=None, prefix_key_scale=None,
                value_fp8=torch.zeros(1), value_scale=torch.zeros(1), heads=H, key_tokens=Lk,
                head_dim=D, tensor_layout="NHD")
            captured.clear()
            backend.long_sequence_video_queries(
                q, prepared, protected_tokens=protected, query_token_indices=torch.arange(Lq))
            tag = f"topk{int(topk * 100)}_prot{protected}"
            results[tag] = captured["block_map"][0].numpy()
    results["pk"] = bits(pk[0])
    results["sk"] = sk[0].numpy().astype(np.uint8)
    save("mask_topk.npz", **results)
    del K


def gen_block_ckpt():
    import json

    sys.path.insert(0, OUT)
    import h3_checkpoint as HC
    from h3serve.native_engine.model.assembly import MappingTensorSource, assemble_pruned_block
    from h3serve.native_engine.model.config import H3CoreConfig
    from h3serve.native_engine.model.layers import torch_sdpa
    from h3serve.native_engine.model.lora import AdaLNCurveRows

    state, metadata, inputs = HC.synthetic_block(0)
    cfg = H3CoreConfig(hidden_size=HC.HIDDEN, num_heads=HC.HEADS, head_dim=HC.HEAD_DIM, ffn_size=HC.FFN,
                       num_layers=1)
    source = MappingTensorSource(state, quantization_metadata=metadata)
    block = assemble_pruned_block(0, source, config=cfg, device="cpu", compute_dtype=torch.bfloat16,
                                  attention_backend=torch_sdpa)
    names = {"qkv": "attn.qkv_proj", "out": "attn.out_proj", "fc1": "mlp.fc1", "fc2": "mlp.fc2"}
    modules = {"qkv": block.attention.qkv_proj, "out": block.attention.out_proj, "fc1": block.mlp.fc1,
               "fc2": block.mlp.fc2}
    g = torch.Generator().manual_seed(11)
    arrays, chosen = {}, {}
    with torch.no_grad():
        for tag, mod in modules.items():
            xin = torch.randn(32, mod.in_features, generator=g).to(torch.bfloat16)
            arrays[f"layer_{tag}_x"] = bits(xin)
            arrays[f"layer_{tag}_out"] = bits(mod(xin))
            spec = mod.spec
            chosen[names[tag]] = {"class": type(mod).__name__,
                                  "spec": {k: getattr(spec, k) for k in spec.__slots__}}
        rows = AdaLNCurveRows(compressed=inputs["curve_rows"], full_silu=None)
        out = block(inputs["x"].clone(), timestep_rows=rows, modulation_segments=inputs["segments"],
                    frequencies=inputs["frequencies"])
    save("block_ckpt.npz", out=bits(out), x=bits(inputs["x"]), digest=np.array(HC.state_digest(state)),
         chosen=np.array(json.dumps(chosen, sort_keys=True)), **arrays)


if __name__ == "__main__":
    torch.manual_seed(0)
    only = sys.argv[2:]
    for fn in (gen_quant, gen_convrot, gen_act, gen_w4, gen_linear, gen_sparge, gen_lut, gen_mask, gen_block_ckpt,
               gen_qk_rope, gen_rms_adaln, gen_sage_k):
        if not only or fn.__name__ in only:
            fn()
