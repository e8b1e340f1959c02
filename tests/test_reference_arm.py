"""The bench's CPU reference arm, held to the reference's own CPU code.

`bench.py --impl reference` and the bench line's `cpu_baseline` time
oracle/reference_cpu.py, a torch restatement of the reference's CPU path.  These
tests import the reference's modules from an X-MinimaxH3 checkout (REFERENCE_ROOT,
else a `reference` directory beside this repository) and check that the restated
pieces compute what the reference computes, bit for bit on the same inputs:

  ConvRotInt8Linear  CPU fallback (model/quantization.py:278-309)
  ConvRotW4A8Linear  CPU fallback through _reference_weight (quantization.py:486-560)
  rms_adaln          eager segmented order (model/kernels.py:7594-7642) over RMSNorm
                     (model/layers.py:33-48)

Skipped when no reference checkout is importable.
"""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle import reference_cpu as R  # noqa: E402


def _reference_root() -> str | None:
    for cand in (os.environ.get("REFERENCE_ROOT", ""), os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "h3serve", "native_engine", "model")):
            return cand
    return None


REF = _reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="no X-MinimaxH3 checkout (set REFERENCE_ROOT)")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, REF)
    import h3serve.native_engine.model.kernels as K
    import h3serve.native_engine.model.layers as Lyr
    import h3serve.native_engine.model.quantization as Q

    return Q, K, Lyr


@pytest.fixture(scope="module")
def block():
    # the reference arm's block at small widths (same code as the bench's 4096 / 16384)
    return R.ReferenceBlockCPU(hidden=512, heads=4, ffn=1024, group=128, seed=3)


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int16)


def test_int8_linear_matches_reference_cpu_fallback(ref, block):
    Q, _, _ = ref
    g = torch.Generator().manual_seed(11)
    q, s = block.w_qkv
    x = torch.randn(37, block.hidden, generator=g).to(torch.bfloat16)
    layer = Q.ConvRotInt8Linear(q, s, block.b_qkv, spec=Q.ComfyQuantSpec("int8_tensorwise", True, 256))
    expected = layer(x)
    got = block._linear(x, block.dequant_int8(block.w_qkv), block.b_qkv)
    assert got.dtype == expected.dtype == torch.bfloat16
    assert torch.equal(_bits(got), _bits(expected))


def test_w4a8_linear_matches_reference_cpu_fallback(ref, block):
    Q, _, _ = ref
    g = torch.Generator().manual_seed(12)
    codes, s_rel, s_ch = block.w_fc1
    # the reference stores two 4-bit codes per byte, the even column in the low nibble
    c = codes.to(torch.int32)
    qdata = (c[:, 0::2] | (c[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)
    layer = Q.ConvRotW4A8Linear(qdata, s_rel, s_ch, bias=block.b_fc1,
                                spec=Q.W4A8QuantSpec(group_size=block.group))
    x = torch.randn(29, block.hidden, generator=g).to(torch.bfloat16)
    expected = layer(x)
    got = block._linear(x, block.dequant_w4(block.w_fc1), block.b_fc1)
    assert torch.equal(_bits(got), _bits(expected))
    # the decoded weight itself
    assert torch.equal(block.dequant_w4(block.w_fc1),
                       layer._reference_weight(qdata, s_rel, s_ch, None, None))


def test_rms_adaln_matches_reference_eager_order(ref, block):
    _, K, Lyr = ref
    g = torch.Generator().manual_seed(13)
    x = torch.randn(50, block.hidden, generator=g).to(torch.bfloat16)
    norm = Lyr.RMSNorm(block.hidden, eps=1e-5, dtype=torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(block.norm)
    shift_a, scale_a = block.mod[0], block.mod[1]
    expected = K.rms_adaln(x, norm, shift_a.unsqueeze(0), scale_a.unsqueeze(0), ((0, x.shape[0], 0),))
    got = block._rms_adaln(x, shift_a, scale_a)
    assert torch.equal(_bits(got), _bits(expected))
