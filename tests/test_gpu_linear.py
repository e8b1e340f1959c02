"""GPU parity of the quantizers, the tcgen05 INT8 GEMM and W4A8 against the CPU oracle.

Bit-exact wherever the computation is integer or has a fixed IEEE order
(codes, scales, int32 accumulators, bf16 epilogue outputs); bf16 linear outputs
against the reference's own eager / module outputs within 1e-2 relative L2.
"""

import os

import numpy as np
import pytest
import torch

from gpu_util import bits, from_bits, outlier_activations, rel_l2
from oracle import oracle as O

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import ops as _ops
    return _ops


def _x(m, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    return outlier_activations(g, m, k).to(torch.bfloat16)


@pytest.mark.parametrize("m,k", [(1, 256), (77, 512), (300, 4096), (5, 5376), (3, 16384), (2, 14336), (9, 48)])
def test_quant_rowwise_bit_exact(ops, m, k):
    x = _x(m, k, seed=m + k)
    q, s = ops.quantize_int8_rowwise(x.cuda())
    qo, so = O.quant_rowwise(bits(x))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), so)


def test_quant_rowwise_golden_edge_rows(ops):
    z = np.load(os.path.join(G, "quant_rowwise.npz"))
    q, s = ops.quantize_int8_rowwise(from_bits(z["x"]))
    np.testing.assert_array_equal(q.cpu().numpy(), z["q"])
    np.testing.assert_allclose(s.cpu().numpy().reshape(-1), z["scale"], rtol=2.5e-7)


@pytest.mark.parametrize("act", [None, "gelu_tanh", "swiglu"])
@pytest.mark.parametrize("m,k", [(1, 256), (130, 4096), (7, 5376), (4, 14336), (3, 16384), (1000, 8192)])
def test_quant_convrot_bit_exact(ops, act, m, k):
    width = 2 * k if act == "swiglu" else k
    x = _x(m, width, seed=3 * m + k)
    q, s = ops.quantize_int8_rowwise_convrot64(x.cuda(), 256, act)
    qo, so = O.quant_rowwise_convrot(bits(x), {None: 0, "gelu_tanh": 1, "swiglu": 2}[act])
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), so)


def test_quant_act_range_edges_bit_exact(ops):
    """Input activations at the exponential's range edges: gate values on both sides of
    the overflow (exp(-g) > FLT_MAX) and underflow bounds, huge, infinite and subnormal
    values, for the SwiGLU and tanh-GELU quantizers, bit for bit against the oracle."""
    edges = [-88.0, -88.5, -89.0, -90.0, -100.0, -103.5, -104.0, -119.0, -121.0, -200.0, -3.0e38,
             88.0, 88.5, 89.0, 103.5, 104.0, 105.0, 120.0, 121.0, 200.0, 3.0e38, float("inf"), float("-inf"),
             0.0, -0.0, 1e-40, -1e-40, 9.0, 10.0, 11.0, -9.5, -10.5, 0.5, -0.5]
    k = 256
    g = torch.Generator().manual_seed(5)
    rows = []
    for i in range(0, len(edges), 8):
        gate = torch.randn(k, generator=g)
        vals = torch.tensor(edges[i:i + 8])
        gate[:len(vals)] = vals
        up = torch.randn(k, generator=g)
        rows.append(torch.cat([gate, up]))
    x = torch.stack(rows).to(torch.bfloat16)
    for act, code, xin in (("swiglu", 2, x), ("gelu_tanh", 1, x[:, :k].contiguous())):
        q, s = ops.quantize_int8_rowwise_convrot64(xin.cuda(), 256, act)
        qo, so = O.quant_rowwise_convrot(bits(xin), code)
        np.testing.assert_array_equal(q.cpu().numpy(), qo, err_msg=act)
        np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), so, err_msg=act)


def test_quant_convrot_strided_rows(ops):
    x = _x(64, 3 * 1024, seed=11)
    xs = x.cuda()[:, 1024:2048]
    q, s = ops.quantize_int8_rowwise_convrot64(xs, 256)
    qo, so = O.quant_rowwise_convrot(bits(x[:, 1024:2048]), 0)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), so)


@pytest.mark.parametrize("convrot", [0, 256])
@pytest.mark.parametrize("m,k", [(64, 4096), (5, 5376), (3, 16384)])
def test_rms_adaln_quant_bit_exact(ops, convrot, m, k):
    g = torch.Generator().manual_seed(m * 7 + k)
    x = (torch.randn(m, k, generator=g) * 2).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    sc = (0.2 * torch.randn(3, k, generator=g)).to(torch.bfloat16)
    sh = (0.2 * torch.randn(3, k, generator=g)).to(torch.bfloat16)
    segs = ((0, m // 4, 2), (m // 4, m // 2, 0), (m // 2, m, 1)) if m >= 8 else ((0, m, 1),)
    q, s = ops.rms_adaln_quantize_int8(x.cuda(), w.cuda(), sc.cuda(), sh.cuda(), segs, 1e-5, convrot)
    seg_row = ops.segment_rows(segs, m, "cpu")
    qo, so = O.rms_adaln_quant(bits(x), bits(w), bits(sc), bits(sh),
                               None if seg_row is None else seg_row.numpy(), 1e-5, convrot)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), so)


@pytest.mark.parametrize("m,n,k", [(1, 16, 16), (100, 72, 256), (300, 520, 4096), (129, 257, 1040), (512, 384, 16384)])
def test_gemm_i32_bit_exact(ops, m, n, k):
    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int16).to(torch.int8)
    b = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8)
    acc = ops.int8_mm_i32(a.cuda(), b.cuda())
    np.testing.assert_array_equal(acc.cpu().numpy(), O.gemm_i8(a.numpy(), b.numpy()))


def test_gemm_i32_full_size_vs_cublas(ops):
    """The INT8 GEMM benchmark shape 4096^3: int32 accumulators equal cuBLASLt's (torch._int_mm)."""
    g = torch.Generator().manual_seed(0)
    a = torch.randint(-127, 128, (4096, 4096), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    b = torch.randint(-127, 128, (4096, 4096), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    acc = ops.int8_mm_i32(a, b)
    ref = torch._int_mm(a, b.t())
    assert torch.equal(acc, ref)


@pytest.mark.parametrize("m,n,k", [(2222, 4160, 2048), (4100, 4096, 4224)])
def test_gemm_pair_kernel_bit_exact(ops, m, n, k):
    """Shapes with at least one 256-row pair tile per SM run the 2-SM kernel
    (tcgen05.mma.cta_group::2): its int32 accumulators equal cuBLAS's, and its
    dequant epilogue equals the oracle's epilogue on those accumulators."""
    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    ref = torch._int_mm(a, b.t())
    assert torch.equal(ops.int8_mm_i32(a, b), ref)
    xs = torch.rand(m, generator=g) * 1e-2 + 1e-4
    ws = torch.rand(n, generator=g) * 1e-3 + 1e-5
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    out = ops.int8_linear_prequantized(a, xs.cuda(), b, ws.cuda(), bias.cuda())
    exp = O.epilogue(ref.cpu().numpy(), xs.numpy(), ws.numpy(), bias.float().numpy())
    np.testing.assert_array_equal(bits(out), exp)


@pytest.mark.parametrize("m,n,ws_kind,with_bias", [(2222, 4104, "channel", True), (4100, 4096, "scalar", False),
                                                   (3001, 4160, "channel", False)])
def test_gemm_pair_kernel_gated_residual_bit_exact(ops, m, n, ws_kind, with_bias):
    """The 2-SM kernel's in-place gated residual (vector 32-column chunks, and the
    per-element tail when N is not a multiple of 32) against the oracle epilogue on
    cuBLAS's accumulators; ragged rows, scalar and per-channel weight scales."""
    k = 1024
    g = torch.Generator().manual_seed(m + n)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    xs = torch.rand(m, generator=g) * 1e-2 + 1e-4
    ws = torch.rand(n if ws_kind == "channel" else 1, generator=g) * 1e-3 + 1e-5
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16) if with_bias else None
    res = torch.randn(m, n, generator=g).to(torch.bfloat16)
    gate = (torch.randn(n, generator=g) * 0.5).to(torch.bfloat16)
    r = res.cuda()
    ops.int8_linear_gated_residual_(r, gate.cuda(), a, xs.cuda(), b, ws.cuda(),
                                    None if bias is None else bias.cuda())
    acc = torch._int_mm(a, b.t()).cpu().numpy()
    exp = O.epilogue(acc, xs.numpy(), ws.numpy(), None if bias is None else bias.float().numpy(),
                     residual=bits(res), gate=bits(gate))
    np.testing.assert_array_equal(bits(r), exp)


@pytest.mark.parametrize("m,heads,rot,ws_kind,with_bias", [
    (4100, 8, 128, "channel", True),     # 2-SM kernel, ragged last row tile
    (3100, 8, 96, "scalar", False),      # 2-SM kernel, the real-H3 rotary width
    (5000, 5, 128, "channel", True),     # 2-SM kernel, a tile holding a Q head and a K head
    (1000, 8, 128, "channel", True),     # 1-SM shape: the op runs the two kernels instead
    (3100, 8, 64, "channel", False),     # rotary width the epilogue does not take: two kernels
])
def test_qkv_epilogue_qk_rope_bit_exact(ops, m, heads, rot, ws_kind, with_bias):
    """The QKV GEMM with the q/k RMSNorm + RoPE in its epilogue equals the GEMM
    followed by the standalone q/k kernel bit for bit, and the oracle on a row sample."""
    k, W = 1024, heads * 128
    n = 3 * W
    g = torch.Generator().manual_seed(m + rot)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8).cuda()
    xs = (torch.rand(m, generator=g) * 1e-2 + 1e-4).cuda()
    ws = (torch.rand(n if ws_kind == "channel" else 1, generator=g) * 1e-3 + 1e-5).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda() if with_bias else None
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).cuda()
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).cuda()
    ang = torch.rand(m, rot // 2, generator=g) * 6
    ct, st = ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda()
    ref = ops.int8_linear_prequantized(a, xs, b, ws, bias)
    ops.qk_rmsnorm_rope_(ref, heads, 0, W, qw, kw, ct, st, 1e-6)
    got = torch.full((m, n), 7.0, device="cuda", dtype=torch.bfloat16)
    ops.int8_linear_prequantized_qk_rope(a, xs, b, ws, bias, got, heads, 0, W, qw, kw, ct, st, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    rows = torch.tensor([0, 1, m // 2, m - 2, m - 1])
    acc = torch._int_mm(a, b.t()).cpu().numpy()[rows.numpy()]
    y = O.epilogue(acc, xs.cpu().numpy()[rows.numpy()], ws.cpu().numpy(),
                   None if bias is None else bias.float().cpu().numpy())
    exp = O.qk_rmsnorm_rope(y, heads, 0, W, bits(qw), bits(kw), bits(ct[rows.cuda()]), bits(st[rows.cuda()]), rot,
                            1e-6)
    np.testing.assert_array_equal(bits(got[rows.cuda()]), exp)


@pytest.mark.parametrize("ws_kind", ["channel", "scalar"])
@pytest.mark.parametrize("with_bias", [True, False])
def test_linear_epilogue_bit_exact(ops, ws_kind, with_bias):
    m, n, k = 200, 264, 1024
    x = _x(m, k, seed=5)
    g = torch.Generator().manual_seed(9)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8)
    ws = (torch.rand(n if ws_kind == "channel" else 1, generator=g) * 1e-3 + 1e-4).float()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16) if with_bias else None
    out = ops.int8_linear(x.cuda(), w.cuda(), ws.cuda(), None if bias is None else bias.cuda(), convrot=True)
    ref = O.int8_linear(bits(x), w.numpy(), ws.numpy(), None if bias is None else bias.float().numpy(), convrot=256)
    np.testing.assert_array_equal(bits(out), ref)


def test_gated_residual_bit_exact(ops):
    m, n, k = 150, 4096, 512
    x = _x(m, k, seed=6)
    g = torch.Generator().manual_seed(10)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8)
    ws = (torch.rand(n, generator=g) * 1e-3).float()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16)
    gate = (torch.randn(n, generator=g) * 0.5).to(torch.bfloat16)
    xq, xs = ops.quantize_int8_rowwise_convrot64(x.cuda(), 256)
    r = res.cuda().clone()
    ops.int8_linear_gated_residual_(r, gate.cuda(), xq, xs, w.cuda(), ws.cuda(), bias.cuda())
    qo, so = O.quant_rowwise_convrot(bits(x), 0)
    ref = O.epilogue(O.gemm_i8(qo, w.numpy()), so, ws.numpy(), bias.float().numpy(), residual=bits(res),
                     gate=bits(gate))
    np.testing.assert_array_equal(bits(r), ref)


@pytest.mark.parametrize("tag", ["g4_codebook_e4m3", "g16_uniform_f32", "g128_uniform_f32", "g16_codebook_e4m3"])
def test_w4_decode_matches_reference_golden(ops, tag):
    z = np.load(os.path.join(G, "w4_decode.npz"))
    qd = torch.from_numpy(z[tag + "_qdata"]).cuda()
    sr = z[tag + "_srel"]
    srt = (torch.from_numpy(sr).view(torch.float8_e4m3fn) if sr.dtype == np.uint8 else torch.from_numpy(sr)).cuda()
    cb = z[tag + "_codebook"]
    out = ops.dequant_int4_grouped_to_int8(qd, srt, torch.from_numpy(cb).cuda() if cb.size else None,
                                           int(z[tag + "_G"]))
    np.testing.assert_array_equal(out.cpu().numpy(), z[tag + "_out"])


def test_linear_vs_reference_outputs(ops):
    """Reference eager int8_linear / ConvRotInt8Linear / W4A8 outputs (golden) within 1e-2 rel-L2."""
    z = np.load(os.path.join(G, "linear.npz"))
    x = from_bits(z["x"])
    wq = torch.from_numpy(z["wq"]).cuda()
    ws = torch.from_numpy(z["ws"]).cuda()
    bias = from_bits(z["bias"])
    out = ops.int8_linear(x, wq, ws, bias, convrot=False)
    assert rel_l2(out.float(), from_bits(z["out_eager"]).float()) < 1e-2
    out_r = ops.int8_linear(x, wq, ws, bias, convrot=True)
    assert rel_l2(out_r.float(), from_bits(z["out_eager_rot"]).float()) < 1e-2
    assert rel_l2(out_r.float(), from_bits(z["out_module_rot"]).float()) < 2e-2
    w4 = ops.w4a8_int8_linear(x, torch.from_numpy(z["w4_qdata"]).cuda(), torch.from_numpy(z["w4_srel"]).cuda(),
                              torch.from_numpy(z["w4_sch"]).cuda(), None, None, bias, int(z["w4_G"]), 256)
    assert rel_l2(w4.float(), from_bits(z["out_w4_eager"]).float()) < 1e-2
    assert rel_l2(w4.float(), from_bits(z["out_w4_module"]).float()) < 2e-2


def test_int8_kernel_callable_matches_oracle(ops):
    """h3b_int8_kernel, the callable the engine's Int8Kernel slot takes, reproduces the
    oracle bit for bit (same quant + GEMM + epilogue)."""
    from h3b import h3b_int8_kernel
    z = np.load(os.path.join(G, "linear.npz"))
    x = from_bits(z["x"])
    out = h3b_int8_kernel(x, torch.from_numpy(z["wq"]).cuda(), torch.from_numpy(z["ws"]).cuda(),
                          from_bits(z["bias"]), 256)
    ref = O.int8_linear(z["x"], z["wq"], z["ws"], O.bf16_bits_to_f32(z["bias"]), convrot=256)
    np.testing.assert_array_equal(bits(out), ref)


@pytest.mark.parametrize("rows,n,k", [(1, 24576, 4096), (3, 18 * 256, 8), (8, 1000, 264), (5, 96, 4096)])
def test_adaln_projection(ops, rows, n, k):
    """The AdaLN projection GEMV against torch's fp32 product of the same bf16 operands:
    the fp32 sums differ only in order, so after bf16 rounding at most one bf16 ulp
    apart, and nearly all equal."""
    g = torch.Generator().manual_seed(rows * 7 + k)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    t = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    out = ops.adaln_projection(w.cuda(), b.cuda(), t.cuda())
    ref = (t.double() @ w.double().T + b.double()).float().to(torch.bfloat16)
    ulps = _bf16_ulps(bits(out), bits(ref))
    assert ulps.max() <= 1
    assert (ulps == 0).mean() > 0.98
    one = ops.adaln_projection(w.cuda(), None, t[0].cuda())
    ref1 = (t[:1].double() @ w.double().T).float().to(torch.bfloat16)
    assert _bf16_ulps(bits(one), bits(ref1)).max() <= 1


def test_no_device_timeouts_recorded(ops):
    from h3b import device_status
    assert device_status(0) == 0


def _bf16_ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in bf16 units in the last place (bit patterns, sign-magnitude)."""
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x & 0x7FFF)
    return np.abs(key(a) - key(b))


@pytest.mark.parametrize("m,k,g,n", [(300, 5376, 16, 1000), (4096, 14336, 16, 5376), (129, 2048, 4, 520),
                                     (64, 4096, 128, 4096)])
def test_w4a8_group_correction_native(ops, m, k, g, n):
    """The W4A8 group correction (comfy_kitchen backends/cuda/__init__.py:2294-2297) as two
    native kernels (group sums, then a tcgen05 bf16 GEMM accumulating into the output):
    bit-equal to the oracle (which sums the exact bf16 products in double) on at least 99 %
    of the elements, every element inside the rounding bound of an fp32 accumulation, and
    close to the reference's own formula (torch addmm on the GPU)."""
    gen = torch.Generator().manual_seed(m + k + n)
    xq = torch.randint(-127, 128, (m, k), generator=gen, dtype=torch.int16).to(torch.int8)
    xs = torch.rand(m, generator=gen) * 1e-2 + 1e-4
    corr = (torch.randn(k // g, n, generator=gen) * 0.02).to(torch.bfloat16)
    out0 = torch.randn(m, n, generator=gen).to(torch.bfloat16)
    out = out0.cuda()
    ops.w4a8_group_correction_(out, xq.cuda(), xs.cuda(), corr.cuda(), g)
    exp = O.w4a8_correction(xq.numpy(), xs.numpy(), g, bits(corr), bits(out0))
    ulps = _bf16_ulps(bits(out), exp)
    assert (ulps == 0).mean() >= 0.99, (ulps.max(), (ulps == 0).mean())
    # every element within the error bound of an fp32-accumulated sum of the exact products
    # (groups terms; near cancellation a few bf16 ulps of a small result are that bound)
    sx64 = (xq.view(m, k // g, g).sum(-1, dtype=torch.int32).to(torch.bfloat16)
            * xs.reshape(m, 1).to(torch.bfloat16)).double()
    corr64 = corr.double()
    exact = out0.double() + sx64 @ corr64
    got64 = out.double().cpu()
    ulp = torch.ldexp(torch.ones_like(exact), torch.frexp(exact.abs().float())[1].double().long() - 8)
    bound = ulp + (k // g) * 2.0 ** -23 * (sx64.abs() @ corr64.abs())
    assert bool(((got64 - exact).abs() <= bound).all()), float(((got64 - exact).abs() / bound).max())
    # the reference's eager formula, on the GPU (cuBLAS)
    sx = xq.cuda().view(m, k // g, g).sum(-1, dtype=torch.int32).to(torch.bfloat16)
    sx = sx * xs.cuda().reshape(m, 1).to(torch.bfloat16)
    ref = out0.cuda().addmm_(sx, corr.cuda()).float().cpu()
    got = out.float().cpu()
    # cuBLAS may round the product before the add: one bf16 ulp of the larger of the
    # result and the correction term (the term can cancel against out0)
    term = (sx.float() @ corr.cuda().float()).abs().cpu()
    assert bool(((got - ref).abs() <= (ref.abs() + term) * 2.0 ** -7 + 2e-4).all())
    assert rel_l2(got, ref) <= 4e-3   # two bf16 roundings apart at most
