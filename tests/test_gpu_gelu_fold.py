"""FC1 with tanh-GELU + ConvRot in the GEMM epilogue, then the codes pass.

The fused path (h3b_int8_gemm_gelu_convrot + h3b_quantize_rotated_int8) must give the
codes and scales of the unfused one (FC1 store epilogue, then the GELU + ConvRot
quantizer) bit for bit, and the oracle's on sampled rows (GEMM, epilogue and
quantizer restated on the CPU).  Shapes cover tail rows (M not a multiple of 256),
bias present or absent, scalar and per-channel weight scales, and the fallback for a
shape that does not run the 2-SM kernel.
"""

import numpy as np
import pytest
import torch

from gpu_util import bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import ops as _ops
    return _ops


def _operands(m, n, k, seed, bias=True, scalar_ws=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20.0
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8)
    ws = torch.rand(1 if scalar_ws else n, generator=g) * 2e-3 + 1e-4
    b = (torch.randn(n, generator=g) * 0.5).to(torch.bfloat16) if bias else None
    return x.to(torch.bfloat16), w, ws, b


@pytest.mark.parametrize("m,n,k,bias,scalar_ws", [
    (4096, 4096, 1024, True, False),
    (4133, 4096, 512, False, False),    # tail rows
    (2560, 16384, 1024, True, True),    # FC1's width; scalar weight scale
    (300, 1024, 512, True, False),      # 1-SM shape: the unfused fallback
])
def test_fused_equals_unfused_and_oracle(ops, m, n, k, bias, scalar_ws):
    x, w, ws, b = _operands(m, n, k, m + n + k, bias, scalar_ws)
    xq, xs = ops.quantize_int8_rowwise_convrot64(x.cuda(), 256)
    wc, wsc = w.cuda(), ws.cuda()
    bc = None if b is None else b.cuda()
    hq, hs = ops.int8_linear_gelu_convrot_quantize(xq, xs, wc, wsc, bc)
    h = ops.int8_linear_prequantized(xq, xs, wc, wsc, bc)
    rq, rs = ops.quantize_int8_rowwise_convrot64(h, 256, "gelu_tanh")
    assert torch.equal(hq, rq)
    assert torch.equal(hs, rs)
    rows = np.unique(np.array([0, 1, 255, 256, m // 2, m - 2, m - 1]))
    acc = O.gemm_i8(xq.cpu().numpy()[rows], w.numpy())
    hb = O.epilogue(acc, xs.cpu().numpy().reshape(-1)[rows], ws.numpy(),
                    None if b is None else b.float().numpy())
    q_o, s_o = O.quant_rowwise_convrot(hb, 1)
    np.testing.assert_array_equal(hq.cpu().numpy()[rows], q_o)
    np.testing.assert_array_equal(hs.cpu().numpy().reshape(-1)[rows], s_o)


def test_rotated_values_and_absmax(ops):
    """The epilogue's stored values are the bf16 rotation of GELU(h) (close to a
    double-precision GELU followed by the oracle's fp32 transform), and each absmax entry
    is the max of |rotated| over its 128 columns (four 32-column runs of one tile; taken on
    the fp32 values, so the bf16 maximum is that value rounded: within half a bf16 ulp)."""
    from h3b._lib import lib
    m, n, k = 4096, 4096, 512
    x, w, ws, b = _operands(m, n, k, 7)
    xq, xs = ops.quantize_int8_rowwise_convrot64(x.cuda(), 256)
    wc, wsc, bc = w.cuda(), ws.cuda(), b.cuda()
    rot = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    amax = torch.empty(m, n // 128, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    b32 = bc.float()
    st = lib().h3b_int8_gemm_gelu_convrot(xq.data_ptr(), wc.data_ptr(), xs.reshape(-1).data_ptr(), wsc.data_ptr(),
                                          n, b32.data_ptr(), rot.data_ptr(), m, n, k, n, amax.data_ptr(), n // 128,
                                          stream)
    assert st == 0
    h = ops.int8_linear_prequantized(xq, xs, wc, wsc, bc)
    rows = np.array([0, 77, 2048, 4095])
    hb = bits(h)[rows]
    gelu = O.bf16_bits_to_f32(hb).astype(np.float64)
    # the rotation of the oracle's GELU values (fp32 transform), rounded to bf16
    g32 = np.array([[_gelu_ref(v) for v in row] for row in gelu], dtype=np.float32)
    r32 = O.fht256(g32).reshape(len(rows), n)
    got = rot[torch.from_numpy(rows).cuda()].float().cpu().numpy()
    # bf16 storage: relative L2 error per row near 2^-9; double-precision GELU differs by ulps
    err = np.linalg.norm(got - r32, axis=1) / np.linalg.norm(r32, axis=1)
    assert np.all(err < 4e-3), err
    am = amax[torch.from_numpy(rows).cuda()].cpu().numpy()
    # entry 2 t + h: columns 64 j + 32 h + [0, 32) of 256-column tile t, j = 0..3
    blk = np.abs(got).reshape(len(rows), n // 256, 4, 2, 32).max(axis=(2, 4)).reshape(len(rows), n // 128)
    assert np.all(am <= blk * (1 + 2 ** -8)) and np.all(blk <= am * (1 + 2 ** -8))


def _gelu_ref(v: float) -> float:
    import math
    return 0.5 * v * (1.0 + math.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))


def test_unsupported_shape_is_reported(ops):
    """The C entry refuses (H3B_ERR_UNSUPPORTED, nothing launched) a width that is not
    a multiple of 256; the Python wrapper then takes the unfused path."""
    from h3b._lib import lib, H3B_ERR_UNSUPPORTED
    m, n, k = 8192, 4160, 512
    x, w, ws, b = _operands(m, n, k, 3)
    xq, xs = ops.quantize_int8_rowwise_convrot64(x.cuda(), 256)
    rot = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    amax = torch.empty(m, n // 128 + 1, device="cuda", dtype=torch.float32)
    st = lib().h3b_int8_gemm_gelu_convrot(xq.data_ptr(), w.cuda().data_ptr(), xs.reshape(-1).data_ptr(),
                                          ws.cuda().data_ptr(), n, None, rot.data_ptr(), m, n, k, n,
                                          amax.data_ptr(), amax.shape[1], torch.cuda.current_stream().cuda_stream)
    assert st == H3B_ERR_UNSUPPORTED


def test_block_mlp_uses_fold_and_matches_unfused(ops):
    """A block whose MLP runs the fused FC1 path gives the bits of the same block with
    the unfused FC1 -> quantizer composition."""
    from h3b import block as B
    from h3b import quantization as Q
    cfg = B.BlockConfig(hidden=1024, heads=8, ffn=4096, t_dim=256)
    blk = B.DiTBlockB200(cfg, device="cuda", seed=5)
    L = 4096
    g = torch.Generator(device="cuda").manual_seed(6)
    x0 = torch.randn(L, cfg.hidden, generator=g, device="cuda").to(torch.bfloat16)
    t = torch.randn(cfg.t_dim, generator=g, device="cuda").to(torch.bfloat16)
    rope = B.rope_tables((16, 16, 16), cfg.rope_splits, device="cuda")
    calls = []
    orig = ops.int8_linear_gelu_convrot_quantize

    def spy(*a, **kw):
        calls.append(1)
        return orig(*a, **kw)

    ops.int8_linear_gelu_convrot_quantize = spy
    try:
        fused = blk.forward(x0.clone(), t, rope)
    finally:
        ops.int8_linear_gelu_convrot_quantize = orig
    assert calls, "the block did not take the fused FC1 path"

    def unfused(self, next_layer, xq, xs, input_act):
        h = self.forward_prequantized(xq, xs)
        return next_layer.quantize(h, input_act)

    saved = Q._QuantLinear.forward_prequantized_for
    Q._QuantLinear.forward_prequantized_for = unfused
    try:
        ref = blk.forward(x0.clone(), t, rope)
    finally:
        Q._QuantLinear.forward_prequantized_for = saved
    assert torch.equal(fused, ref)
