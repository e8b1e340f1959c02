"""The DiT block checked stage by stage against the CPU oracle.

Each stage's GPU output is compared with the oracle applied to the GPU's own output of
the previous stage, so a wrong head, row or segment shows at the stage that makes it:
RMSNorm + AdaLN + ConvRot INT8 codes, the QKV projection with its q/k RMSNorm + RoPE
epilogue, the attention preparation and block mask (bit-exact), the attention output
(the kernel-order oracle's tolerance), the out-projection's quantizer and gated residual,
the MLP's quantizer, W4A8 FC1, GELU + ConvRot quantizer and FC2 gated residual
(bit-exact; GEMM outputs on sampled rows).  Finally `forward` must give the bits of the
staged composition.
"""

import numpy as np
import pytest
import torch

from gpu_util import assert_attention_parity, bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import attention as A
    from h3b import block as B
    from h3b import ops
    return A, B, ops


def _linear_rows(lin, xq, xs, rows, residual=None, gate=None):
    """The oracle's output rows of a quantized layer from the GPU's codes and scales."""
    w8, ws = lin.int8_weight()
    acc = O.gemm_i8(xq[rows].cpu().numpy(), w8.cpu().numpy())
    bias = None if lin.bias is None else lin.bias.float().cpu().numpy()
    return O.epilogue(acc, xs.reshape(-1)[rows].cpu().numpy(), ws.cpu().numpy(), bias, residual=residual, gate=gate)


@pytest.mark.parametrize("sparse", [False, True])
def test_block_stage_by_stage(mods, sparse):
    A, B, ops = mods
    mask = A.MaskConfig("cdf", 0.6, keep_first_column=True, keep_diagonal=True) if sparse else None
    cfg = B.BlockConfig(hidden=1024, heads=8, ffn=4096, t_dim=256, mask=mask)
    blk = B.DiTBlockB200(cfg, device="cuda", seed=11)
    L, H, D, W = 1536, cfg.heads, cfg.head_dim, cfg.heads * cfg.head_dim
    g = torch.Generator(device="cuda").manual_seed(12)
    x0 = torch.randn(L, cfg.hidden, generator=g, device="cuda").to(torch.bfloat16)
    t = torch.randn(cfg.t_dim, generator=g, device="cuda").to(torch.bfloat16)
    rope = B.rope_tables((6, 16, 16), cfg.rope_splits, device="cuda")
    rows = torch.tensor([0, 1, 127, 128, 700, 1023, 1500, L - 1], device="cuda")
    r_np = rows.cpu().numpy()
    sh_a, sc_a, ga, sh_m, sc_m, gm = blk.modulation(t).unbind(1)

    # RMSNorm + AdaLN + ConvRot INT8
    x = x0.clone()
    xq, xs = ops.rms_adaln_quantize_int8(x, blk.norm1, sc_a, sh_a, None, cfg.eps, 256)
    q_o, s_o = O.rms_adaln_quant(bits(x), bits(blk.norm1), bits(sc_a), bits(sh_a), None, cfg.eps, True)
    np.testing.assert_array_equal(xq.cpu().numpy(), q_o)
    np.testing.assert_array_equal(xs.cpu().numpy().reshape(-1), s_o)

    # QKV projection + q/k RMSNorm + RoPE epilogue
    qkv = torch.empty(L, 3 * W, device="cuda", dtype=torch.bfloat16)
    blk.qkv.forward_prequantized_qk_rope(xq, xs, qkv, H, 0, W, blk.q_norm, blk.k_norm, rope[0], rope[1], cfg.qk_eps)
    y = _linear_rows(blk.qkv, xq, xs, rows)
    exp = O.qk_rmsnorm_rope(y, H, 0, W, bits(blk.q_norm), bits(blk.k_norm), bits(rope[0])[r_np],
                            bits(rope[1])[r_np], 128, cfg.qk_eps)
    np.testing.assert_array_equal(bits(qkv)[r_np], exp)

    # attention preparation and mask (from the GPU's QKV rows)
    view = qkv.view(L, 3, H, D)
    q, k, v = view[:, 0], view[:, 1], view[:, 2]
    pv = A.prepare_values(v)
    pk, mean = A.prepare_keys(k)
    pq = A.prepare_queries(q)
    vt_o, vs_o = O.value_fp8(bits(v))
    np.testing.assert_array_equal(pv.vt.cpu().numpy(), vt_o)
    np.testing.assert_array_equal(bits(mean), O.key_mean(bits(k)))
    thr = np.full(H, -0.1, np.float32)
    _, _, kq_o, ks_o = O.pool_sim_quant(bits(k), 64, thr, bits(mean))
    np.testing.assert_array_equal(pk.qi8[:, :L].cpu().numpy(), kq_o[:, :L])
    np.testing.assert_array_equal(pk.scale.cpu().numpy(), ks_o)
    _, _, qq_o, _ = O.pool_sim_quant(bits(q), 128, thr)
    np.testing.assert_array_equal(pq.qi8[:, :L].cpu().numpy(), qq_o[:, :L])
    bitmap = None
    if sparse:
        bitmap = A.block_mask(pq, pk, mask)
        bm_o = O.block_mask(bits(pq.pooled), pq.similar.cpu().numpy(), bits(pk.pooled), pk.similar.cpu().numpy(),
                            mode=1, budget=0.6, flags=3)
        np.testing.assert_array_equal(bitmap.cpu().numpy().view(np.uint32), bm_o)

    # attention (every head, first / middle / last tiles)
    o = A.attention(pq, pk, pv, bitmap)
    assert_attention_parity(o, pq, pk, pv, bitmap, tiles=(0, 5, 11))
    o2 = o.view(L, W)

    # out-projection: ConvRot quantizer, gated residual
    oq, os_ = blk.out.quantize(o2)
    oq_o, os_o = O.quant_rowwise_convrot(bits(o2))
    np.testing.assert_array_equal(oq.cpu().numpy(), oq_o)
    np.testing.assert_array_equal(os_.cpu().numpy().reshape(-1), os_o)
    x_before = bits(x)[r_np]
    blk.out.gated_residual_(x, ga[0], oq, os_)
    exp = _linear_rows(blk.out, oq, os_, rows, residual=x_before, gate=bits(ga[0]))
    np.testing.assert_array_equal(bits(x)[r_np], exp)

    # MLP: RMSNorm + AdaLN quantizer, W4A8 FC1, GELU + ConvRot quantizer, FC2 gated residual
    xq2, xs2 = ops.rms_adaln_quantize_int8(x, blk.norm2, sc_m, sh_m, None, cfg.eps, 256)
    q_o, s_o = O.rms_adaln_quant(bits(x), bits(blk.norm2), bits(sc_m), bits(sh_m), None, cfg.eps, True)
    np.testing.assert_array_equal(xq2.cpu().numpy(), q_o)
    h = blk.fc1.forward_prequantized(xq2, xs2)
    np.testing.assert_array_equal(bits(h)[r_np], _linear_rows(blk.fc1, xq2, xs2, rows))
    hq, hs = blk.fc2.quantize(h, cfg.mlp_act)
    hq_o, hs_o = O.quant_rowwise_convrot(bits(h), 1)
    np.testing.assert_array_equal(hq.cpu().numpy(), hq_o)
    np.testing.assert_array_equal(hs.cpu().numpy().reshape(-1), hs_o)
    x_before = bits(x)[r_np]
    blk.fc2.gated_residual_(x, gm[0], hq, hs)
    exp = _linear_rows(blk.fc2, hq, hs, rows, residual=x_before, gate=bits(gm[0]))
    np.testing.assert_array_equal(bits(x)[r_np], exp)

    # the block's forward is exactly this composition
    assert torch.equal(blk.forward(x0.clone(), t, rope), x)
