"""GPU parity of the attention preparation, the Sparge mask and the tcgen05
quantized attention kernel.

Preparation (K mean, pool / similarity / INT8, Sage per_thread INT8, V FP8), the
block mask and the LUT are bit-exact against the CPU oracle.  The attention output
is compared with the oracle in the kernel's own arithmetic -- P = 2^x * 112 rounded
to E4M3 under the lazy running max, fp32 row sums in the kernel's order -- at
rel-L2 <= 5e-3 and cos >= 0.9999 (what is left is ex2.approx's last bits and the
tensor core's fp32 accumulation order), and with exact softmax over the same
quantized Q / K / V at cos >= 0.999.  (The E4M3 rounding of P, 3 mantissa bits, is
the P format of the reference's sm89 kernel too and alone puts about 2.5 % rel-L2
between any such kernel and exact softmax.)
"""

import math
import os

import numpy as np
import pytest
import torch

from gpu_util import assert_attention_parity, bits, cosine, from_bits, rel_l2
from oracle import oracle as O

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def attn():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import attention as _attn
    return _attn


def qkv(L, H, seed, k_offset=True, Lk=None):
    g = torch.Generator().manual_seed(seed)
    Lk = Lk or L
    q = torch.randn(L, H, 128, generator=g)
    k = torch.randn(Lk, H, 128, generator=g)
    if k_offset:
        k = k + torch.randn(1, H, 128, generator=g) * 3.0   # per-channel offset: the K-smoothing case
    v = torch.randn(Lk, H, 128, generator=g)
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


@pytest.mark.parametrize("rot", [128, 64, 96])
def test_qk_rmsnorm_rope_bit_exact(attn, rot):
    from h3b import ops
    g = torch.Generator().manual_seed(rot)
    L, H = 300, 3
    qkv = (torch.randn(L, 3 * H * 128 + 8, generator=g) * 2).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    ang = torch.rand(L, rot // 2, generator=g) * 6
    ct, st = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    got = ops.qk_rmsnorm_rope_(qkv.cuda(), H, 0, H * 128, qw.cuda(), kw.cuda(), ct.cuda(), st.cuda(), 1e-6)
    ref = O.qk_rmsnorm_rope(bits(qkv), H, 0, H * 128, bits(qw), bits(kw), bits(ct), bits(st), rot, 1e-6)
    np.testing.assert_array_equal(bits(got), ref)


@pytest.mark.parametrize("L,H", [(197, 4), (1000, 2), (4096, 1)])
def test_key_mean_bit_exact(attn, L, H):
    _, k, _ = qkv(L, H, seed=L)
    m = attn.key_mean(k.cuda())
    np.testing.assert_array_equal(bits(m), O.key_mean(bits(k)))


@pytest.mark.parametrize("block", [64, 128])
@pytest.mark.parametrize("L,H,smooth", [(131, 4, False), (197, 4, True), (1000, 3, True), (64, 1, False)])
def test_pool_sim_quant_bit_exact(attn, block, L, H, smooth):
    _, k, _ = qkv(L, H, seed=L + block)
    kc = k.cuda()
    mean = attn.key_mean(kc) if smooth else None
    pb = attn.prepare_blocks(kc, block, -0.1, mean)
    po, so, qo, sco = O.pool_sim_quant(bits(k), block, np.full(H, -0.1, np.float32),
                                       None if mean is None else bits(mean))
    np.testing.assert_array_equal(bits(pb.pooled), po)
    np.testing.assert_array_equal(pb.similar.cpu().numpy(), so)
    np.testing.assert_array_equal(pb.scale.cpu().numpy(), sco)
    nb = po.shape[1]
    np.testing.assert_array_equal(pb.qi8[:, :nb * block].cpu().numpy(), qo)


def test_pool_sim_quant_reference_golden(attn):
    """The reference's pool_sim_quant_nhd fixture (seed 82736, Lq=131, Lk=197, H=4)."""
    z = np.load(os.path.join(G, "sparge_pool.npz"))
    q = from_bits(z["q"])
    pq = attn.prepare_blocks(q, 128, -0.1)
    np.testing.assert_array_equal(pq.similar.cpu().numpy(), z["sq"])
    np.testing.assert_array_equal(pq.qi8[:, :131].permute(1, 0, 2).cpu().numpy(), z["qq"])
    k = from_bits(z["k"])
    mean = attn.key_mean(k)
    np.testing.assert_array_equal(bits(mean), z["kmean"])
    pk = attn.prepare_blocks(k, 64, -0.1, mean)
    np.testing.assert_array_equal(pk.similar.cpu().numpy(), z["sk"])
    np.testing.assert_array_equal(pk.qi8[:, :197].permute(1, 0, 2).cpu().numpy(), z["kq"])


@pytest.mark.parametrize("L,H", [(997, 4), (128, 2), (1, 1)])
def test_value_fp8_bit_exact(attn, L, H):
    _, _, v = qkv(L, H, seed=L * 3)
    pv = attn.prepare_values(v.cuda())
    vt, vs = O.value_fp8(bits(v), pv.padded)
    np.testing.assert_array_equal(pv.vt.cpu().numpy(), vt)
    np.testing.assert_array_equal(pv.scale.cpu().numpy(), vs)


def _prepared_pair(attn, L, H, seed, Lk=None):
    q, k, v = qkv(L, H, seed, Lk=Lk)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    pk, mean = attn.prepare_keys(kc)
    pq = attn.prepare_queries(qc)
    pv = attn.prepare_values(vc)
    return (q, k, v), pq, pk, pv, mean


@pytest.mark.parametrize("cfg", [
    dict(mode="topk", budget=0.5),
    dict(mode="topk", budget=0.25, protected_tokens=200),
    dict(mode="cdf", budget=0.6, keep_first_column=True, keep_diagonal=True),
    dict(mode="cdf", budget=0.3),
    dict(mode="topk", budget=0.1, temporal_radius=1, temporal_spatial_radius=1, video_layout=(4, 250)),
])
def test_block_mask_bit_exact(attn, cfg):
    _, pq, pk, _, _ = _prepared_pair(attn, 1000, 3, seed=21)
    mc = attn.MaskConfig(**cfg)
    bm = attn.block_mask(pq, pk, mc)
    frames, ftok = mc.video_layout or (0, 0)
    ref = O.block_mask(bits(pq.pooled), pq.similar.cpu().numpy(), bits(pk.pooled), pk.similar.cpu().numpy(),
                       mode=0 if mc.mode == "topk" else 1, budget=mc.budget,
                       protected_kb=(mc.protected_tokens + 63) // 64,
                       flags=int(mc.keep_first_column) | 2 * int(mc.keep_diagonal),
                       temporal_radius=mc.temporal_radius, temporal_spatial_radius=mc.temporal_spatial_radius,
                       frames=frames, frame_tokens=ftok, protected_tokens=mc.protected_tokens, q_tokens=pq.tokens)
    np.testing.assert_array_equal(bm.cpu().numpy().view(np.uint32), ref)


def test_block_mask_bit_exact_beyond_8192_key_blocks(attn):
    """8208 key blocks (525,295 keys, the 4-rows-per-CTA kernel): bit-exact."""
    _, pq, pk, _, _ = _prepared_pair(attn, 1000, 1, seed=31, Lk=8208 * 64 - 17)
    assert pk.scale.shape[1] == 8208
    mc = attn.MaskConfig("cdf", 0.6, keep_first_column=True, keep_diagonal=True)
    bm = attn.block_mask(pq, pk, mc)
    ref = O.block_mask(bits(pq.pooled), pq.similar.cpu().numpy(), bits(pk.pooled), pk.similar.cpu().numpy(),
                       mode=1, budget=mc.budget, protected_kb=0, flags=3, temporal_radius=mc.temporal_radius,
                       temporal_spatial_radius=mc.temporal_spatial_radius, frames=0, frame_tokens=0,
                       protected_tokens=0, q_tokens=pq.tokens)
    np.testing.assert_array_equal(bm.cpu().numpy().view(np.uint32), ref)


def test_block_mask_reference_selector_golden(attn):
    """Reference fixed-TopK selector (kernels.py:3668-3941) on tie-free inputs."""
    z = np.load(os.path.join(G, "mask_topk.npz"))
    q, k = from_bits(z["q"]), from_bits(z["k"])
    pq = attn.prepare_queries(q)
    pk, _ = attn.prepare_keys(k, smooth=False)
    Kb = pk.pooled.shape[1]
    for topk in (50, 75):
        for prot in (0, 100):
            bm = attn.block_mask(pq, pk, attn.MaskConfig("topk", topk / 100.0, protected_tokens=prot))
            got = O.bitmap_to_bool(bm.cpu().numpy().view(np.uint32), Kb)
            np.testing.assert_array_equal(got, z[f"topk{topk}_prot{prot}"])


def test_bitmap_to_lut_bit_exact(attn):
    z = np.load(os.path.join(G, "lut.npz"))
    bm = z["block_map"]
    H, Qb, Kb = bm.shape
    words = (Kb + 31) // 32
    packed = np.zeros((H, Qb, words * 32), np.uint8)
    packed[..., :Kb] = bm
    bitmap = np.packbits(packed, axis=-1, bitorder="little").view(np.int32)
    lut, valid = attn.bitmap_to_lut(torch.from_numpy(bitmap).cuda(), Kb)
    lo, vo = O.bitmap_to_lut(bitmap.view(np.uint32), Kb)
    np.testing.assert_array_equal(valid.cpu().numpy(), z["valid"])
    np.testing.assert_array_equal(lut.cpu().numpy(), lo)


@pytest.mark.parametrize("L,H,Lk", [(1000, 2, None), (128, 1, None), (300, 2, 77), (2048, 1, None), (64, 1, 1)])
def test_dense_attention_parity(attn, L, H, Lk):
    _, pq, pk, pv, _ = _prepared_pair(attn, L, H, seed=L + H, Lk=Lk)
    out = attn.attention(pq, pk, pv)
    assert_attention_parity(out, pq, pk, pv)


@pytest.mark.parametrize("sparse", [False, True])
def test_long_sequence_attention_parity(attn, sparse):
    """L = 8192: sampled tiles (first pair, a middle pair, the last) on both heads."""
    _, pq, pk, pv, _ = _prepared_pair(attn, 8192, 2, seed=77)
    bm = attn.block_mask(pq, pk, attn.MaskConfig("cdf", 0.6, keep_first_column=True, keep_diagonal=True)) \
        if sparse else None
    out = attn.attention(pq, pk, pv, bm)
    assert_attention_parity(out, pq, pk, pv, bm, tiles=(0, 1, 30, 31, 63))


@pytest.mark.parametrize("block", [64, 32])
def test_dense_attention_q_groups(attn, block):
    """Per-64-token Q blocks and Sage per_warp 32-row groups."""
    q, k, v = qkv(700, 2, seed=5 + block)
    pv = attn.prepare_values(v.cuda())
    pk, _ = attn.prepare_keys(k.cuda())
    pq = attn.prepare_queries(q.cuda(), block=block)
    out = attn.attention(pq, pk, pv)
    assert_attention_parity(out, pq, pk, pv)


@pytest.mark.parametrize("cfg", [dict(mode="topk", budget=0.3), dict(mode="cdf", budget=0.6, keep_first_column=True,
                                                                     keep_diagonal=True)])
def test_sparse_attention_parity(attn, cfg):
    _, pq, pk, pv, _ = _prepared_pair(attn, 1500, 2, seed=99)
    bm = attn.block_mask(pq, pk, attn.MaskConfig(**cfg))
    out = attn.attention(pq, pk, pv, bm)
    assert_attention_parity(out, pq, pk, pv, bm)


@pytest.mark.parametrize("L", [197, 64, 1000])
def test_sage_k_per_thread_golden(attn, L):
    """Sage per_thread K quantization on the GPU equals the reference's in-tree kernel
    (model/sage_fused_quant.py:20-162; fixture made by tests/golden/make_golden.py)."""
    z = np.load(os.path.join(G, "sage_k_per_thread.npz"))
    pk = attn.quantize_per_thread(from_bits(z[f"k{L}"]), "k", from_bits(z[f"kmean{L}"]))
    np.testing.assert_array_equal(pk.qi8[:, :L].cpu().numpy().transpose(1, 0, 2), z[f"kq{L}"])
    np.testing.assert_array_equal(pk.scale.cpu().numpy(), z[f"ks{L}"])


@pytest.mark.parametrize("L,H", [(1000, 3), (131, 2), (4100, 1)])
def test_quant_per_thread_bit_exact(attn, L, H):
    q, k, _ = qkv(L, H, seed=L)
    mean = attn.key_mean(k.cuda())
    pq = attn.quantize_per_thread(q.cuda(), "q")
    pk = attn.quantize_per_thread(k.cuda(), "k", mean)
    for pb, x, kind, m in ((pq, q, 0, None), (pk, k, 1, bits(mean))):
        rq, rs = O.quant_per_thread(bits(x), kind, m)
        np.testing.assert_array_equal(pb.qi8.cpu().numpy(), rq)
        np.testing.assert_array_equal(pb.scale.cpu().numpy(), rs)


@pytest.mark.parametrize("L,H,Lk", [(1000, 2, None), (300, 2, 77), (4096, 1, None)])
def test_dense_attention_per_thread(attn, L, H, Lk):
    """Sage per_thread granularity (the reference's dense default, qk_quant_gran 3):
    4-row Q scale groups, 16-key K groups per 64-key block."""
    q, k, v = qkv(L, H, seed=3 * L, Lk=Lk)
    backend = attn.SageAttentionB200(qk_quant_gran="per_thread")
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = backend(qc, kc, vc)
    pq, pk, pv = backend.quantize_queries(qc), backend.quantize_keys(kc), attn.prepare_values(vc)
    assert pq.gran == 1 and pk.gran == 1
    assert torch.equal(out, attn.attention(pq, pk, pv))
    assert_attention_parity(out, pq, pk, pv)


def _sdpa(q, k, v):
    qf, kf, vf = (t.float().permute(1, 0, 2) for t in (q, k, v))
    s = qf @ kf.transpose(1, 2) / math.sqrt(128)
    return (s.softmax(-1) @ vf).permute(1, 0, 2)


def test_backends_are_attention_callables(attn):
    """The backends against fp32 attention on the unquantized inputs: INT8 Q / K, FP8 P
    and V together stay within cos 0.99 (the per-stage bounds are in the tests above)."""
    q, k, v = qkv(513, 2, seed=3)
    dense = attn.SageAttentionB200()(q.cuda(), k.cuda(), v.cuda())
    assert dense.shape == (513, 2, 128) and dense.dtype == torch.bfloat16
    assert cosine(dense.float().cpu(), _sdpa(q, k, v)) >= 0.99
    for gran in ("per_thread", "per_warp"):
        o = attn.SageAttentionB200(qk_quant_gran=gran)(q.cuda(), k.cuda(), v.cuda())
        assert cosine(o.float().cpu(), _sdpa(q, k, v)) >= 0.99
    sparse = attn.SpargeAttentionB200(attn.MaskConfig("topk", 1.0))(q.cuda(), k.cuda(), v.cuda())
    assert cosine(sparse.float().cpu(), dense.float().cpu()) >= 0.9999


def test_no_device_timeouts_recorded(attn):
    from h3b import device_status
    assert device_status(0) == 0


def test_long_sequence_protocol_matches_whole_sequence(attn):
    """Prepared K/V + query chunks reproduce the one-shot backend (same kernels,
    same blocks) -- the streamed protocol of model/layers.py:341-356, with the
    prepared-V tuple the reference caller unpacks (model/layers.py:668-680)."""
    q, k, v = qkv(1024 + 256, 2, seed=17)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    backend = attn.SpargeLongSequenceB200(attn.MaskConfig("topk", 0.5))
    vt, vs, heads, key_tokens, head_dim = backend.prepare_long_sequence_values(vc.unsqueeze(0))
    assert (heads, key_tokens, head_dim) == (2, 1280, 128)
    assert vt.shape == (1, 2, 128, 1280) and vt.dtype == torch.float8_e4m3fn and vs.shape == (1, 2, 128)
    prepared = backend.prepare_long_sequence_keys(kc.unsqueeze(0), vt, vs)
    whole = backend.long_sequence_video_queries(qc, prepared, protected_tokens=0, query_token_indices=None)
    one_shot = attn.SpargeAttentionB200(attn.MaskConfig("topk", 0.5))(qc, kc, vc)
    assert torch.equal(whole, one_shot)
    # a 128-aligned chunk sees the same pooled query blocks -> same rows
    chunk = backend.long_sequence_video_queries(qc[512:1024], prepared, protected_tokens=0,
                                                query_token_indices=torch.arange(512, 1024, device="cuda"))
    assert torch.equal(chunk, whole[512:1024])
    with pytest.raises(ValueError):
        backend.prepare_long_sequence_keys(kc[:1000].unsqueeze(0), vt, vs)
    dense = attn.DenseLongSequenceB200()
    prep_d = dense.prepare_long_sequence_keys(kc.unsqueeze(0), vt, vs)
    assert torch.equal(dense.long_sequence_prefix_queries(qc[:256], prep_d),
                       attn.SageAttentionB200(q_block=32)(qc, kc, vc)[:256])
    assert torch.equal(dense.long_sequence_all_queries(qc, prep_d), attn.SageAttentionB200(q_block=32)(qc, kc, vc))


@pytest.mark.parametrize("selected", ["offset", "gathered"])
def test_block_mask_query_indices_and_protected_rows_bit_exact(attn, selected):
    """Temporal rail centred through a chunk's token indices (model/kernels.py:5247-5254)
    and protected query rows (kernels.py:2423-2426): bit-exact vs the oracle."""
    g = torch.Generator().manual_seed(5)
    frames, ftok, prefix = 6, 300, 192
    Lk = prefix + frames * ftok
    q = torch.randn(640, 3, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(Lk, 3, 128, generator=g).to(torch.bfloat16)
    pq = attn.prepare_queries(q.cuda())
    pk, _ = attn.prepare_keys(k.cuda())
    if selected == "offset":
        idx = torch.arange(900, 900 + 640)
    else:  # calibration-style: whole 128-row blocks gathered from across the video
        starts = torch.tensor([0, 1280, 384, 1536, 768])
        idx = (starts[:, None] + torch.arange(128)[None, :]).reshape(-1)
    mc = attn.MaskConfig("topk", 0.2, protected_tokens=prefix, temporal_radius=1, temporal_spatial_radius=1,
                         video_layout=(frames, ftok))
    bm = attn.block_mask(pq, pk, mc, query_indices=idx.cuda(), protected_query_tokens=130)
    ref = O.block_mask(bits(pq.pooled), pq.similar.cpu().numpy(), bits(pk.pooled), pk.similar.cpu().numpy(),
                       mode=0, budget=0.2, protected_kb=(prefix + 63) // 64, flags=0, temporal_radius=1,
                       temporal_spatial_radius=1, frames=frames, frame_tokens=ftok, protected_tokens=prefix,
                       q_tokens=640, q_index=idx.numpy(), protected_qb=2)
    np.testing.assert_array_equal(bm.cpu().numpy().view(np.uint32), ref)
    no_idx = attn.block_mask(pq, pk, mc, protected_query_tokens=130)
    assert not torch.equal(no_idx, bm), "the indices should move the rail"


def test_compact_kv_builder_matches_whole_build(attn):
    """Slab-by-slab K/V (begin_compact_long_sequence_kv, model/kernels.py:2677-2772) equals
    the whole-sequence preparation byte for byte when given the same K mean and V absmax."""
    L, H = 1000, 3
    _, k, v = qkv(L, H, seed=41)
    kc, vc = k.cuda(), v.cuda()
    pk, mean = attn.prepare_keys(kc)
    pv = attn.prepare_values(vc)
    absmax = vc.float().abs().amax(0)
    backend = attn.SpargeLongSequenceB200()
    b = backend.begin_compact_long_sequence_kv(key_tokens=L, heads=H, head_dim=128, key_mean=mean.float(),
                                               value_absmax=absmax, device=kc.device)
    for s0 in range(0, L, 256):
        b.add(s0, kc[s0:s0 + 256], vc[s0:s0 + 256])
    prep = b.finish()
    for a_, b_ in ((prep.keys.qi8, pk.qi8), (prep.keys.scale, pk.scale), (prep.keys.pooled, pk.pooled),
                   (prep.keys.similar, pk.similar), (prep.values.vt, pv.vt), (prep.values.scale, pv.scale)):
        assert a_.shape == b_.shape
        assert torch.equal(a_.view(torch.uint8) if a_.dtype != torch.uint8 else a_,
                           b_.view(torch.uint8) if b_.dtype != torch.uint8 else b_)
    with pytest.raises(ValueError):
        b2 = backend.begin_compact_long_sequence_kv(key_tokens=L, heads=H, head_dim=128, key_mean=mean.float(),
                                                    value_absmax=absmax, device=kc.device)
        b2.add(64, kc[64:128], vc[64:128])


def test_dense_attention_per_warp_q(attn):
    """Per-warp (32-row) Q scales, Sage's per_warp granularity (model/kernels.py:5571-5573)."""
    q, k, v = qkv(700, 2, seed=6)
    pv = attn.prepare_values(v.cuda())
    pk, _ = attn.prepare_keys(k.cuda())
    pq = attn.prepare_queries(q.cuda(), block=32)
    assert pq.scale.shape == (2, 22)
    out = attn.attention(pq, pk, pv)
    assert_attention_parity(out, pq, pk, pv)
