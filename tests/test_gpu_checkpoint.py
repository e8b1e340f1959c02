"""A pruned-H3-format checkpoint through the B200 loader (tests/golden/h3_checkpoint.py,
fixture tests/golden/block_ckpt.npz from the engine's own assemble_pruned_block).

  * each layer (ConvRot INT8 per-row / scalar scale; W4A8 with e4m3 s_rel + codebook,
    and with fp32 s_rel + correction) equals the oracle bit for bit where the output is
    the oracle's quant + GEMM + epilogue, and is within 2e-2 relative L2 of the
    engine's float layer;
  * the whole block, loaded from a safetensors file with `_quantization_metadata`, run
    with the engine's modulation segments and RoPE angles, tracks the engine's CPU block
    on the residual update (cos >= 0.99, relative L2 <= 0.1): the engine keeps
    activations and attention in bf16, this path quantizes them (INT8 rows, INT8 QK,
    FP8 PV), the same gap the block test against the fp32 restatement allows.
"""

import json
import os
import sys

import numpy as np
import pytest
import torch

from gpu_util import bits, cosine, rel_l2
from oracle import oracle as O

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")
sys.path.insert(0, G)
import h3_checkpoint as HC  # noqa: E402


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import checkpoint as C
    return C, np.load(os.path.join(G, "block_ckpt.npz")), HC.synthetic_block(0)


def from_bits(a):
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).cuda()


def test_layers_match_oracle_and_engine(env):
    from h3b import ops

    C, z, (state, metadata, _) = env
    source = C.MappingTensorSource(state, quantization_metadata=metadata)
    for tag, name in (("qkv", "attn.qkv_proj"), ("out", "attn.out_proj"), ("fc1", "mlp.fc1"), ("fc2", "mlp.fc2")):
        lin = C.quant_linear(source, f"{HC.PREFIX}.{name}", device="cuda")
        x = from_bits(z[f"layer_{tag}_x"])
        out = lin(x)
        assert rel_l2(out.float(), from_bits(z[f"layer_{tag}_out"]).float()) < 2e-2, tag
        xq, xs = lin.quantize(x)
        w8, ws = lin.int8_weight()
        bias = None if lin.bias is None else lin.bias.float().cpu().numpy()
        ref = O.int8_linear(z[f"layer_{tag}_x"], w8.cpu().numpy(), ws.cpu().numpy(), bias, convrot=256)
        if getattr(lin, "correction", None) is None:
            np.testing.assert_array_equal(bits(out), ref, err_msg=tag)
        else:
            # the GEMM part alone, before the group correction is added
            plain = ops.int8_linear_prequantized(xq, xs, w8, ws, lin.bias)
            np.testing.assert_array_equal(bits(plain), ref, err_msg=tag)
            corr = plain.clone()
            ops.w4a8_group_correction_(corr, xq, xs, lin.correction, lin.spec.group_size)
            assert torch.equal(corr, out), tag
            # the native correction against the oracle's: within one bf16 ulp
            exp = O.w4a8_correction(xq.cpu().numpy(), xs.cpu().numpy(), lin.spec.group_size,
                                    bits(lin.correction.to(torch.bfloat16)), bits(plain))
            diff = np.abs(bits(out).astype(np.int32) - exp.astype(np.int32))
            assert diff.max() <= 1, tag


def test_block_from_safetensors_tracks_engine_block(env, tmp_path):
    from safetensors.torch import save_file
    from h3b.block import rope_tables_from_frequencies
    import h3b

    C, z, (state, metadata, inputs) = env
    path = str(tmp_path / "h3_block.safetensors")
    save_file(state, path, metadata={"_quantization_metadata": json.dumps({"layers": metadata})})
    with C.SafeTensorSource(path) as src:
        blk = C.load_block(0, src, num_layers=1, device="cuda")
    rope = rope_tables_from_frequencies(inputs["frequencies"].cuda())
    x = inputs["x"].cuda()
    out = blk.forward(x.clone(), inputs["curve_rows"].cuda(), rope, segments=inputs["segments"]).float()
    ref = from_bits(z["out"]).float()
    upd, upd_ref = out - x.float(), ref - x.float()
    assert cosine(upd, upd_ref) >= 0.99
    assert rel_l2(upd, upd_ref) <= 0.1
    # each modulation segment on its own (a wrong row selection shows here first)
    for start, stop, _ in inputs["segments"]:
        assert cosine(upd[start:stop], upd_ref[start:stop]) >= 0.98, (start, stop)
    assert h3b.device_status(0) == 0
