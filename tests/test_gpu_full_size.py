"""The BASELINE.json configurations the benchmark times, checked at full size.

C1  INT8 W8A8 linear, M = N = K = 4096, activations N(0, 1) with 1 % of channels x20,
    per-output-channel INT8 weights from N(0, 0.02), bf16 bias N(0, 0.01): every row's
    codes and scale, and the bf16 output of sampled rows, bit-exact vs the CPU oracle;
    the whole output within 1e-2 rel-L2 of the dequantized-matmul formula of the
    reference's eager int8_linear (comfy_kitchen backends/eager/quantization.py:971-1062).
C2  W4A8 MLP pair at the 720p/5 s token count, M = 111,600, 4096 -> 16384 (GELU-tanh)
    -> 4096, symmetric int4 weights in groups of 128 (fp32 s_rel), ConvRot INT8
    activations, gated residual into a bf16 N(0, 1) stream: the FC1 output, the
    GELU + ConvRot FC2-input codes and the updated residual of sampled rows bit-exact
    vs the oracle.
C3  dense quantized attention, H = 32, L = 111,600, K with a per-channel N(0, 3) offset,
    with per-64-token Q / K blocks (the config's scales) and with Sage per_thread
    groups (the reference's default): sampled query tiles against all keys within
    rel-L2 <= 5e-3 of the oracle in the kernel's arithmetic and cos >= 0.999 of exact
    softmax over the same operands.
"""

import numpy as np
import pytest
import torch

from gpu_util import assert_attention_parity, bits, outlier_activations, rel_l2
from oracle import oracle as O

pytestmark = pytest.mark.gpu

M_720P5S = 31 * 45 * 80


@pytest.fixture(scope="module")
def h3b_mods():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import attention, block, ops, quantization
    return ops, block, quantization, attention


def _sample_rows(m: int, n: int, seed: int) -> np.ndarray:
    g = np.random.default_rng(seed)
    fixed = np.array([0, 1, m // 2, m - 1])
    return np.unique(np.concatenate([fixed, g.choice(m, n, replace=False)]))


def test_config1_int8_linear_full_size(h3b_mods):
    ops, block, _, _ = h3b_mods
    g = torch.Generator().manual_seed(0)
    x = outlier_activations(g, 4096, 4096).to(torch.bfloat16)
    wq, ws = block._int8_per_channel(torch.randn(4096, 4096, generator=g) * 0.02)
    bias = (torch.randn(4096, generator=g) * 0.01).to(torch.bfloat16)
    xc, wc, wsc, bc = x.cuda(), wq.cuda(), ws.cuda(), bias.cuda()
    q, s = ops.quantize_int8_rowwise(xc)
    qo, so = O.quant_rowwise(bits(x))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), so)
    out = ops.int8_linear(xc, wc, wsc, bc)
    rows = _sample_rows(4096, 60, 1)
    exp = O.int8_linear(bits(x)[rows], wq.numpy(), ws.numpy(), bias.float().numpy())
    np.testing.assert_array_equal(bits(out)[rows], exp)
    ref = torch._int_mm(q, wc.t()).float() * s.reshape(-1, 1) * wsc.reshape(1, -1) + bc.float()
    assert rel_l2(out.float(), ref) <= 1e-2


def test_config2_w4a8_mlp_full_size(h3b_mods):
    ops, block, Q, _ = h3b_mods
    M, D, F, G = M_720P5S, 4096, 16384, 128
    g = torch.Generator().manual_seed(2)
    spec = Q.W4A8QuantSpec("asym_w4a8_int8", group_size=G)
    qd1, sr1, sc1 = block._int4_grouped(torch.randn(F, D, generator=g) * 0.02, G)
    qd2, sr2, sc2 = block._int4_grouped(torch.randn(D, F, generator=g) * 0.02, G)
    b1 = (torch.randn(F, generator=g) * 0.01).to(torch.bfloat16)
    b2 = (torch.randn(D, generator=g) * 0.01).to(torch.bfloat16)
    fc1 = Q.W4A8Linear(qd1.cuda(), sr1.cuda(), sc1.cuda(), bias=b1.cuda(), spec=spec)
    fc2 = Q.W4A8Linear(qd2.cuda(), sr2.cuda(), sc2.cuda(), bias=b2.cuda(), spec=spec)
    gd = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, D, device="cuda", generator=gd).to(torch.bfloat16)
    res0 = torch.randn(M, D, device="cuda", generator=gd).to(torch.bfloat16)
    gate = (torch.rand(D, generator=g) + 0.5).to(torch.bfloat16)
    xq, xs = fc1.quantize(x)
    h = fc1.forward_prequantized(xq, xs)
    hq, hs = fc2.quantize(h, "gelu_tanh")
    # the block's path: tanh-GELU + ConvRot in FC1's GEMM epilogue, then the codes pass;
    # every row's codes and scale equal the unfused FC1 + GELU quantizer's
    hq_f, hs_f = fc1.forward_prequantized_for(fc2, xq, xs, "gelu_tanh")
    assert torch.equal(hq_f, hq) and torch.equal(hs_f.reshape(-1), hs.reshape(-1))
    del hq_f, hs_f
    res = res0.clone()
    fc2.gated_residual_(res, gate.cuda(), hq, hs)
    torch.cuda.synchronize()

    rows = _sample_rows(M, 12, 4)
    r = torch.from_numpy(rows).cuda()
    xq_o, xs_o = O.quant_rowwise_convrot(bits(x[r]))
    np.testing.assert_array_equal(xq[r].cpu().numpy(), xq_o)
    h_o = O.epilogue(O.gemm_i8(xq_o, O.w4_decode(qd1.numpy(), sr1.numpy(), None, G)), xs_o, sc1.numpy(),
                     b1.float().numpy())
    np.testing.assert_array_equal(bits(h[r]), h_o)
    hq_o, hs_o = O.quant_rowwise_convrot(h_o, 1)
    np.testing.assert_array_equal(hq[r].cpu().numpy(), hq_o)
    np.testing.assert_array_equal(hs[r].cpu().numpy().reshape(-1), hs_o)
    res_o = O.epilogue(O.gemm_i8(hq_o, O.w4_decode(qd2.numpy(), sr2.numpy(), None, G)), hs_o, sc2.numpy(),
                       b2.float().numpy(), residual=bits(res0[r]), gate=bits(gate))
    np.testing.assert_array_equal(bits(res[r]), res_o)


@pytest.mark.parametrize("gran", ["per_block_64", "per_thread"])
def test_config3_dense_attention_full_size(h3b_mods, gran):
    _, _, _, A = h3b_mods
    L, H = M_720P5S, 32
    gd = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(L, H, 128, device="cuda", generator=gd).to(torch.bfloat16)
    k = (torch.randn(L, H, 128, device="cuda", generator=gd)
         + torch.randn(1, H, 128, device="cuda", generator=gd) * 3.0).to(torch.bfloat16)
    v = torch.randn(L, H, 128, device="cuda", generator=gd).to(torch.bfloat16)
    if gran == "per_thread":
        sage = A.SageAttentionB200(qk_quant_gran="per_thread")
        pq, pk = sage.quantize_queries(q), sage.quantize_keys(k)
    else:
        pq = A.prepare_queries(q, 64)
        pk, _ = A.prepare_keys(k)
    pv = A.prepare_values(v)
    out = A.attention(pq, pk, pv)
    qt = (L + 127) // 128
    assert_attention_parity(out, pq, pk, pv, tiles=(0, 1, qt // 2, qt - 1), heads=(0, 31))
