"""Host side of the checkpoint contract (no GPU): which layer class and spec each
tensor-name set selects, the safetensors source and its `_quantization_metadata`, the
constructor checks, and the oracle against the engine's own layer outputs on the
synthetic checkpoint (tests/golden/block_ckpt.npz, made by tests/golden/make_golden.py)."""

import json
import os
import sys

import numpy as np
import pytest
import torch

from oracle import oracle as O

G = os.path.join(os.path.dirname(__file__), "golden")
sys.path.insert(0, G)
import h3_checkpoint as HC  # noqa: E402

from h3b import checkpoint as C  # noqa: E402
from h3b import quantization as Q  # noqa: E402
from h3b.block import rope_tables_from_frequencies  # noqa: E402


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(G, "block_ckpt.npz"))


@pytest.fixture(scope="module")
def ckpt():
    return HC.synthetic_block(0)


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_synthetic_checkpoint_is_the_one_the_fixture_was_made_from(ckpt, golden):
    state, _, inputs = ckpt
    assert HC.state_digest(state) == str(golden["digest"])
    np.testing.assert_array_equal(inputs["x"].view(torch.int16).numpy().view(np.uint16), golden["x"])


def test_layer_choice_matches_the_engine(ckpt, golden):
    state, metadata, _ = ckpt
    source = C.MappingTensorSource(state, quantization_metadata=metadata)
    want = json.loads(str(golden["chosen"]))
    kinds = {"ConvRotInt8Linear": Q.Int8Linear, "ConvRotW4A8Linear": Q.W4A8Linear}
    for name, ref in want.items():
        lin = C.quant_linear(source, f"{HC.PREFIX}.{name}", device="cpu")
        assert type(lin) is kinds[ref["class"]], name
        got = {k: getattr(lin.spec, k) for k in ref["spec"]}
        assert got == ref["spec"], name


def test_int8_layer_has_no_bias_even_if_stored(ckpt):
    state, metadata, _ = ckpt
    s = dict(state)
    s[f"{HC.PREFIX}.attn.qkv_proj.bias"] = torch.zeros(3 * HC.HEADS * HC.HEAD_DIM, dtype=torch.bfloat16)
    lin = C.quant_linear(C.MappingTensorSource(s), f"{HC.PREFIX}.attn.qkv_proj", device="cpu")
    assert lin.bias is None


def test_load_block_reads_dimensions_from_the_tensors(ckpt):
    state, metadata, _ = ckpt
    blk = C.load_block(0, C.MappingTensorSource(state, quantization_metadata=metadata), num_layers=1, device="cpu")
    cfg = blk.cfg
    assert (cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.mlp_act, cfg.t_dim) == (256, 4, 128, 512, "swiglu", 8)
    assert cfg.mask is None and cfg.qk_eps == 1e-5
    assert blk.ada_w.shape == (18 * 256, 8)
    with pytest.raises(IndexError):
        C.load_block(1, C.MappingTensorSource(state), num_layers=1, device="cpu")


def test_missing_or_unknown_layer_is_a_key_error(ckpt):
    state, _, _ = ckpt
    s = {k: v for k, v in state.items() if not k.startswith(f"{HC.PREFIX}.mlp.fc1.weight_s")}
    with pytest.raises(KeyError, match="neither ConvRot INT8 nor W4A8"):
        C.quant_linear(C.MappingTensorSource(s), f"{HC.PREFIX}.mlp.fc1", device="cpu")
    s = {k: v for k, v in state.items() if k != f"{HC.PREFIX}.attn.qkv_proj.comfy_quant"}
    with pytest.raises(KeyError, match="qkv_proj.comfy_quant"):
        C.quant_linear(C.MappingTensorSource(s), f"{HC.PREFIX}.attn.qkv_proj", device="cpu")
    with pytest.raises(KeyError, match="incomplete quantized layer"):
        Q.Int8Linear.from_state_dict(s, f"{HC.PREFIX}.attn.qkv_proj")


def test_safetensors_source_round_trip(ckpt, tmp_path):
    from safetensors.torch import save_file

    state, metadata, _ = ckpt
    path = str(tmp_path / "block.safetensors")
    save_file(state, path, metadata={"_quantization_metadata": json.dumps({"layers": metadata})})
    src = C.SafeTensorSource(path)
    with pytest.raises(RuntimeError, match="context manager"):
        src.tensor(f"{HC.PREFIX}.norm1.weight")
    with src:
        assert src.quantization_spec(f"{HC.PREFIX}.mlp.fc1") == HC.FC1_SPEC
        assert src.quantization_spec(f"{HC.PREFIX}.attn.out_proj") is None
        for key, value in state.items():
            assert src.has_tensor(key)
            assert torch.equal(src.tensor(key).view(torch.uint8), value.contiguous().view(torch.uint8)), key
        fc1 = C.quant_linear(src, f"{HC.PREFIX}.mlp.fc1", device="cpu")
        assert fc1.spec.group_size == 32
    bad = str(tmp_path / "bad.safetensors")
    save_file({"a": torch.zeros(1)}, bad, metadata={"_quantization_metadata": "{not json"})
    with pytest.raises(ValueError, match="_quantization_metadata"):
        with C.SafeTensorSource(bad):
            pass
    assert C.parse_quantization_metadata({"_quantization_metadata": json.dumps({"layers": {"x": {"group_size": 8},
                                                                                          "y": 3}})}) == \
        {"x": {"group_size": 8}}


def test_spec_decoding_and_checks():
    spec = Q.ComfyQuantSpec("int8_tensorwise", True, 256)
    for raw in (spec.encode(), bytes(spec.encode().tolist()), bytes(spec.encode().tolist()).decode(),
                {"format": "int8_tensorwise", "convrot": True}):
        assert Q.ComfyQuantSpec.decode(raw) == spec
    with pytest.raises(TypeError):
        Q.ComfyQuantSpec.decode(3.0)
    w = torch.zeros(8, 256, dtype=torch.int8)
    with pytest.raises(ValueError, match="int8_tensorwise"):
        Q.Int8Linear(w, torch.ones(8), spec=Q.ComfyQuantSpec("fp8"))
    with pytest.raises(ValueError, match="power of four"):
        Q.Int8Linear(w, torch.ones(8), spec=Q.ComfyQuantSpec("int8_tensorwise", True, 128))
    with pytest.raises(ValueError, match="ConvRot group 256"):
        Q.Int8Linear(w, torch.ones(8), spec=Q.ComfyQuantSpec("int8_tensorwise", True, 64))
    with pytest.raises(ValueError, match="scalar or one value per output row"):
        Q.Int8Linear(w, torch.ones(3), spec=spec)
    qd = torch.zeros(8, 128, dtype=torch.int8)
    with pytest.raises(ValueError, match="s_rel must be"):
        Q.W4A8Linear(qd, torch.ones(8, 8), torch.ones(8))
    with pytest.raises(ValueError, match="requires ConvRot"):
        Q.W4A8Linear(qd, torch.ones(8, 16), torch.ones(8), spec=Q.W4A8QuantSpec(convrot=False))
    with pytest.raises(ValueError, match="group size"):
        Q.W4A8Linear(qd, torch.ones(8, 16), torch.ones(8), spec=Q.W4A8QuantSpec(group_size=24))
    with pytest.raises(ValueError, match="correction"):
        Q.W4A8Linear(qd, torch.ones(8, 16), torch.ones(8), correction=torch.ones(8, 16))
    with pytest.raises(ValueError, match="16 entries"):
        Q.W4A8Linear(qd, torch.ones(8, 16), torch.ones(8), codebook=torch.ones(15))


def test_rope_tables_from_both_frequency_forms(ckpt):
    _, _, inputs = ckpt
    f = inputs["frequencies"]
    c, s = rope_tables_from_frequencies(f)
    assert c.shape == (f.shape[0], 48) and c.dtype == torch.bfloat16
    half = f[:, :48]
    packed = torch.stack((torch.cos(half), -torch.sin(half), torch.sin(half), torch.cos(half)), -1)
    packed = packed.reshape(1, f.shape[0], 1, 48, 2, 2).to(torch.bfloat16)
    c2, s2 = rope_tables_from_frequencies(packed)
    assert torch.equal(c, c2) and torch.equal(s, s2)


@pytest.mark.parametrize("rot", [128, 96])
def test_rope_tables_equal_reference_rotation_table(rot):
    """The cos / sin tables the kernels read, built from the engine's split-half angles and
    from its packed table, equal the reference's rope_rotation_table entries
    (model/layers.py:60-69) bit for bit (fixture tests/golden/qk_rope.npz)."""
    z = np.load(os.path.join(G, "qk_rope.npz"))
    table = torch.from_numpy(z[f"r{rot}_table"].astype(np.int16)).view(torch.bfloat16)
    for freq in (torch.from_numpy(z[f"r{rot}_angles"]), table):
        c, s = rope_tables_from_frequencies(freq)
        assert c.shape == (table.shape[1], rot // 2)
        np.testing.assert_array_equal(c.view(torch.int16).numpy().view(np.uint16), z[f"r{rot}_cos"])
        np.testing.assert_array_equal(s.view(torch.int16).numpy().view(np.uint16), z[f"r{rot}_sin"])


def _layer_tensors(state, name):
    p = f"{HC.PREFIX}.{name}."
    return {k[len(p):]: v for k, v in state.items() if k.startswith(p)}


def test_oracle_layers_against_engine_layer_outputs(ckpt, golden):
    """The oracle's decode + ConvRot INT8 linear against the engine's float fallback
    (activations unquantized) on every layer of the checkpoint: bf16 output within 2e-2
    relative L2, the tolerance of the single-layer module fixtures."""
    state, metadata, _ = ckpt
    for tag, name in (("qkv", "attn.qkv_proj"), ("out", "attn.out_proj"), ("fc1", "mlp.fc1"), ("fc2", "mlp.fc2")):
        t = _layer_tensors(state, name)
        x = golden[f"layer_{tag}_x"]
        bias = None if "bias" not in t or "weight_scale" in t else O.bf16_bits_to_f32(
            t["bias"].view(torch.int16).numpy().view(np.uint16))
        if "weight_scale" in t:
            wq, ws = t["weight"].numpy(), t["weight_scale"].numpy()
        else:
            group = metadata.get(f"{HC.PREFIX}.{name}", {}).get("group_size", 16)
            sr = t["weight_s_rel"]
            sr = sr.view(torch.uint8).numpy() if sr.dtype == torch.float8_e4m3fn else sr.numpy()
            cb = t["weight_codebook"].numpy() if "weight_codebook" in t else None
            wq, ws = O.w4_decode(t["weight"].numpy(), sr, cb, group), t["weight_s_channel"].numpy()
        out = O.bf16_bits_to_f32(O.int8_linear(x, wq, ws, bias, convrot=256))
        if "weight_correction" in t:
            q, s = O.quant_rowwise_convrot(x, 0)
            group = metadata[f"{HC.PREFIX}.{name}"]["group_size"]
            sx = q.reshape(q.shape[0], -1, group).astype(np.int64).sum(-1) * s.reshape(-1, 1)
            out = out + sx @ t["weight_correction"].float().numpy()
        assert rel_l2(out, O.bf16_bits_to_f32(golden[f"layer_{tag}_out"])) < 2e-2, tag


def test_chunk_segments_restrict_and_shift():
    from h3b.block import _chunk_segments, _runs
    segs = ((0, 300, 0), (300, 700, 4), (700, 1024, 5))
    assert _chunk_segments(None, 0, 10) is None
    assert _chunk_segments(segs, 0, 100) == ((0, 100, 0),)
    assert _chunk_segments(segs, 100, 517) == ((0, 200, 0), (200, 417, 4))
    assert _chunk_segments(segs, 517, 1024) == ((0, 183, 4), (183, 507, 5))
    for r0, r1 in ((0, 100), (100, 517), (517, 1000), (1000, 1024)):
        runs = _runs(_chunk_segments(segs, r0, r1), r1 - r0, 6)
        assert runs[0][0] == 0 and runs[-1][1] == r1 - r0
    with pytest.raises(ValueError):
        _runs(((0, 5, 0), (6, 10, 1)), 10, 6)
