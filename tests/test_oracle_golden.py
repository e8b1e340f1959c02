"""Pin the CPU oracle against golden vectors from the reference's own code.

The fixtures were produced by tests/golden/make_golden.py from the X-MinimaxH3
sources; each test names the reference function behind its fixture.
"""

import os

import numpy as np
import pytest

from oracle import oracle as O

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(G, name))


def bf(b):
    return O.bf16_bits_to_f32(b)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_quant_rowwise_matches_eager_codes():
    """comfy_kitchen eager quantize_int8_rowwise (eager/quantization.py:857-875)."""
    z = load("quant_rowwise.npz")
    q, s = O.quant_rowwise(z["x"])
    np.testing.assert_array_equal(q, z["q"])
    # CUDA kernel form absmax*(1/127) vs eager absmax/127: equal to within one fp32 ulp
    np.testing.assert_allclose(s, z["scale"], rtol=2.5e-7, atol=0)


def test_fht_matches_eager_rotation():
    """ConvRot rotation vs eager _rotate_activation in fp32 (tensor/int8_utils.py:11-74)."""
    z = load("convrot.npz")
    rot = O.fht256(bf(z["x"]))
    assert rel_l2(rot, z["rot_f32"]) < 1e-6
    np.testing.assert_allclose(rot, z["rot_f32"], rtol=0, atol=2e-5 * np.abs(z["rot_f32"]).max())


def test_convrot_codes_within_one_of_eager():
    """Fused ConvRot quant vs eager quantize_and_rotate_rowwise (bf16 matmul rotation):
    codes may differ by one (rarely two, where the eager bf16 scale moves) because
    the eager rotation is a bf16 matmul while the CUDA kernel rotates in fp32."""
    z = load("convrot.npz")
    q, s = O.quant_rowwise_convrot(z["x"], 0)
    diff = np.abs(q.astype(np.int32) - z["q_eager"].astype(np.int32))
    assert diff.max() <= 2
    assert (diff <= 1).mean() > 0.999
    assert (diff == 0).mean() > 0.97
    np.testing.assert_allclose(s, z["scale_eager"], rtol=1e-2)


def test_input_activations_match_torch():
    """gelu_tanh / swiglu (backends/_activations.py:41-53) to a few fp32 ulp."""
    z = load("input_act.npz")
    x = bf(z["x"])
    # act applied inside the quantizer; check through the exported scalar functions
    lib = O.lib()
    gelu = np.vectorize(lambda v: 0.5 * v * (1.0 + lib.h3bo_tanhf(np.float32(0.7978845608028654 * (v + 0.044715 * v * v * v)))))(x.astype(np.float64))
    np.testing.assert_allclose(gelu, z["gelu_f32"], rtol=2e-6, atol=2e-7)
    K = x.shape[1] // 2
    gate, up = x[:, :K].astype(np.float64), x[:, K:].astype(np.float64)
    e = np.vectorize(lambda v: lib.h3bo_expf(np.float32(-v)))(gate)
    sw = gate / (1.0 + e) * up
    np.testing.assert_allclose(sw, z["swiglu_f32"], rtol=2e-6, atol=2e-7)


def test_expf_accuracy():
    lib = O.lib()
    xs = np.concatenate([np.linspace(-100, 88, 20001), np.linspace(-1, 1, 5001)]).astype(np.float32)
    ours = np.array([lib.h3bo_expf(float(v)) for v in xs], np.float64)
    ref = np.exp(xs.astype(np.float64))
    ok = ref > 1.2e-38
    rel = np.abs(ours[ok] - ref[ok]) / ref[ok]
    assert rel.max() < 2.5e-7  # about two fp32 ulp


@pytest.mark.parametrize("tag", ["g4_codebook_e4m3", "g16_uniform_f32", "g128_uniform_f32", "g16_codebook_e4m3"])
def test_w4_decode_bit_exact(tag):
    """eager _dequant_int4_grouped_to_int8 (eager/w4a8_int8.py:344-363)."""
    z = load("w4_decode.npz")
    cb = z[tag + "_codebook"]
    out = O.w4_decode(z[tag + "_qdata"], z[tag + "_srel"], cb if cb.size else None, int(z[tag + "_G"]))
    np.testing.assert_array_equal(out, z[tag + "_out"])


def test_int8_linear_vs_eager_and_module():
    """int8_linear: eager (eager/quantization.py:971-1062) and the ConvRotInt8Linear CPU
    fallback (model/quantization.py:278-304), bf16 output within 1e-2 relative L2."""
    z = load("linear.npz")
    bias = bf(z["bias"])
    out = O.int8_linear(z["x"], z["wq"], z["ws"], bias, convrot=0)
    assert rel_l2(bf(out), bf(z["out_eager"])) < 1e-2
    out_r = O.int8_linear(z["x"], z["wq"], z["ws"], bias, convrot=256)
    assert rel_l2(bf(out_r), bf(z["out_eager_rot"])) < 1e-2
    assert rel_l2(bf(out_r), bf(z["out_module_rot"])) < 2e-2


def test_w4a8_linear_vs_eager_and_module():
    """w4a8_int8_linear eager (eager/w4a8_int8.py:457-508) and ConvRotW4A8Linear CPU path."""
    z = load("linear.npz")
    wq = O.w4_decode(z["w4_qdata"], z["w4_srel"], None, int(z["w4_G"]))
    out = O.int8_linear(z["x"], wq, z["w4_sch"], bf(z["bias"]), convrot=256)
    assert rel_l2(bf(out), bf(z["out_w4_eager"])) < 1e-2
    assert rel_l2(bf(out), bf(z["out_w4_module"])) < 2e-2


def assert_pooled_equal(ours, ref):
    """Pooled means are stored to bf16.  The Triton interpreter that produced the
    fixture narrows fp32 to bf16 by truncation, where the GPU (and the oracle)
    round to nearest even; so a fixture value may sit one bf16 step closer to
    zero than ours, never anywhere else."""
    a = O.bf16_bits_to_f32(ours).astype(np.float64)
    b = O.bf16_bits_to_f32(ref).astype(np.float64)
    d = np.abs(ours.astype(np.int64) - ref.astype(np.int64))
    assert d.max() <= 1
    m = d != 0
    assert np.all(np.abs(b[m]) < np.abs(a[m]))
    assert np.all(np.sign(a[m]) == np.sign(b[m]))


def test_sparge_pool_sim_quant_reference_shapes():
    """sparge_nhd.pool_sim_quant_nhd + hnd_compatible_key_mean_nhd (TRITON_INTERPRET)."""
    z = load("sparge_pool.npz")
    thr = np.full(4, -0.1, np.float32)
    pq, sq, qq, qs = O.pool_sim_quant(z["q"], 128, thr)
    assert_pooled_equal(pq, z["pq"])
    np.testing.assert_array_equal(sq, z["sq"])
    np.testing.assert_allclose(qs, z["qs"], rtol=1e-7)
    L = z["q"].shape[0]
    np.testing.assert_array_equal(qq[:, :L].transpose(1, 0, 2), z["qq"])
    kmean = O.key_mean(z["k"])
    np.testing.assert_array_equal(kmean, z["kmean"])
    pk, sk, kq, ks = O.pool_sim_quant(z["k"], 64, thr, mean=kmean)
    assert_pooled_equal(pk, z["pk"])
    np.testing.assert_array_equal(sk, z["sk"])
    np.testing.assert_allclose(ks, z["ks"], rtol=1e-7)
    Lk = z["k"].shape[0]
    np.testing.assert_array_equal(kq[:, :Lk].transpose(1, 0, 2), z["kq"])


def test_sparge_similarity_thresholds():
    z = load("sparge_pool.npz")
    pb, sb, qb, sbs = O.pool_sim_quant(z["kb"], 64, z["thr2"])
    np.testing.assert_array_equal(sb, z["sb"])
    assert_pooled_equal(pb, z["pb"])
    np.testing.assert_array_equal(qb.transpose(1, 0, 2), z["qb"])


def test_lut_matches_reference_kernels():
    """sparse_lut block_map_to_absolute_lut + absolute_lut_to_delta (TRITON_INTERPRET)."""
    z = load("lut.npz")
    bm = z["block_map"]
    H, Qb, Kb = bm.shape
    words = (Kb + 31) // 32
    packed = np.zeros((H, Qb, words * 32), np.uint8)
    packed[..., :Kb] = bm
    bitmap = np.packbits(packed, axis=-1, bitorder="little").view(np.uint32)
    lut, valid = O.bitmap_to_lut(bitmap, Kb)
    np.testing.assert_array_equal(valid, z["valid"])
    for h in range(H):
        for i in range(Qb):
            n = valid[h, i]
            np.testing.assert_array_equal(lut[h, i, :n], z["lut"][h, i, :n])


def test_fixed_topk_mask_matches_reference_selector():
    """SplitModalityProtectedSpargeAttentionBackend.long_sequence_video_queries
    (model/kernels.py:3668-3941) on tie-free integer inputs: block maps identical."""
    z = load("mask_topk.npz")
    thr = np.full(2, -0.1, np.float32)
    pq, sq, _, _ = O.pool_sim_quant(z["q"], 128, thr)
    pk, sk, _, _ = O.pool_sim_quant(z["k"], 64, thr)
    np.testing.assert_array_equal(pk, z["pk"])
    np.testing.assert_array_equal(sk, z["sk"])
    Kb = pk.shape[1]
    for topk in (50, 75):
        for prot in (0, 100):
            bm = O.block_mask(pq, sq, pk, sk, mode=0, budget=topk / 100.0, protected_kb=(prot + 63) // 64)
            got = O.bitmap_to_bool(bm, Kb)
            np.testing.assert_array_equal(got, z[f"topk{topk}_prot{prot}"], err_msg=f"topk{topk} prot{prot}")


@pytest.mark.parametrize("rot", [128, 96])
def test_qk_rmsnorm_rope_vs_reference_cpu_path(rot):
    """apply_qknorm_rope on CPU bf16 tensors with the engine's packed rotation table
    (model/layers.py:60-118).  The per-head RMSNorm agrees bit for bit (the channels past
    the rotary width).  The rotated channels differ by rounding only: the reference's CPU
    path rounds each product to bf16 before the bf16 sum, while the oracle (like the
    reference's fused CUDA kernel, rms_rope.cu) keeps fp32 until one final rounding.  So
    each rotated output stays within 2^-6 of |n_d| |cos| + |n_e| |sin|, the magnitudes of
    its two products (measured at most 2^-7)."""
    z = load("qk_rope.npz")
    q, k = z[f"r{rot}_q"], z[f"r{rot}_k"]
    L, H, D = q.shape
    half = rot // 2
    qkv = np.zeros((L, 3 * H * D), np.uint16)
    qkv[:, :H * D] = q.reshape(L, -1)
    qkv[:, H * D:2 * H * D] = k.reshape(L, -1)
    out = O.qk_rmsnorm_rope(qkv, H, 0, H * D, z[f"r{rot}_qw"], z[f"r{rot}_kw"], z[f"r{rot}_cos"],
                            z[f"r{rot}_sin"], rot, 1e-6)
    c = bf(z[f"r{rot}_cos"])[:, None, :].astype(np.float64)
    s = bf(z[f"r{rot}_sin"])[:, None, :].astype(np.float64)
    for x, w, cols, ref in ((q, z[f"r{rot}_qw"], slice(0, H * D), z[f"r{rot}_qo"]),
                            (k, z[f"r{rot}_kw"], slice(H * D, 2 * H * D), z[f"r{rot}_ko"])):
        got = out[:, cols].reshape(L, H, D)
        np.testing.assert_array_equal(got[..., rot:], ref[..., rot:])
        xf = bf(x).astype(np.float64)
        n = xf / np.sqrt((xf ** 2).mean(-1, keepdims=True) + 1e-6) * bf(w)
        first, second = n[..., :half], n[..., half:rot]
        scale = np.concatenate((np.abs(first * c) + np.abs(second * s), np.abs(first * s) + np.abs(second * c)), -1)
        err = np.abs(bf(got[..., :rot]).astype(np.float64) - bf(ref[..., :rot]))
        assert (err <= 2.0 ** -6 * scale).all(), float((err / scale).max())


@pytest.mark.parametrize("K", [4096, 5376])
def test_rms_adaln_rows_vs_reference_eager(K):
    """RMSNorm module (F.rms_norm) + kernels.rms_adaln's eager segmented modulation on CPU
    bf16 rows, three segments (model/layers.py:33-49, kernels.py:7594-7642): the modulated
    rows the fused quantizer rotates, bit-exact on this fixture, and the fused oracle
    quantizer's codes and scales equal its ConvRot quantizer applied to the reference's rows.
    The fp32 sum of squares depends on the summation order (torch's reduction against the
    kernel's fixed tree): on other rows 1 / rms can move by an ulp and leave a value up to
    2 bf16 steps apart (a 48-row sample at K = 5376 showed 5 such values of 258,048)."""
    z = load("rms_adaln.npz")
    x = z[f"k{K}_x"]
    seg_row = np.zeros(x.shape[0], np.int32)
    for start, stop, r in z[f"k{K}_segments"]:
        seg_row[start:stop] = r
    rows = O.rms_adaln_rows(x, z[f"k{K}_w"], z[f"k{K}_scale"], z[f"k{K}_shift"], seg_row, 1e-5)
    assert not (rows.view(np.uint32) & 0xFFFF).any(), "modulated rows must be bf16 values"
    ref = z[f"k{K}_out"]
    np.testing.assert_array_equal((rows.view(np.uint32) >> 16).astype(np.uint16), ref)
    q1, s1 = O.rms_adaln_quant(x, z[f"k{K}_w"], z[f"k{K}_scale"], z[f"k{K}_shift"], seg_row, 1e-5, True)
    q2, s2 = O.quant_rowwise_convrot(ref, 0)
    np.testing.assert_array_equal(q1, q2)
    np.testing.assert_array_equal(s1, s2)


def test_value_fp8_vs_reference_formula_in_torch():
    """V -> FP8 (model/compact_fp8.py:253-300 host part, 13-97 kernel math): per (head,
    channel) absmax by aminmax, scaled = float(v) * (2.25 / absmax) in fp32, then E4M3 with
    round-to-nearest (the kernel's cvt.rn.satfinite; |scaled| <= 2.25, so torch's
    float8_e4m3fn cast rounds identically), scale = absmax / 2.25.  The factor is the IEEE
    quotient, as everywhere in this build (torch's scalar `2.25 / t` multiplies by a rounded
    reciprocal and the reference's Triton `/` is not correctly rounded either; either can
    move a near-tie to the neighbouring code).  The oracle's bytes, transposed to
    [H, 128, Lpad] without the sm89 16-row permutation, equal torch's.  An all-zero channel
    gets zeros and scale 0 (the reference would divide by zero)."""
    import torch

    g = torch.Generator().manual_seed(31)
    L, H = 300, 3
    v = (torch.randn(L, H, 128, generator=g) * torch.rand(1, H, 128, generator=g) * 4).to(torch.bfloat16)
    v[:, 1, 7] = 0                                          # an all-zero channel
    vt, vs = O.value_fp8(v.contiguous().view(torch.int16).numpy().view(np.uint16))
    hnd = v.permute(1, 0, 2).float()                        # [H, L, 128]
    mn, mx = torch.aminmax(hnd, dim=1)
    absmax = torch.maximum(mn.abs(), mx.abs())
    factor = torch.full_like(absmax, 2.25) / absmax        # IEEE quotient (tensor / tensor)
    scaled = hnd * factor[:, None, :]
    ref = scaled.to(torch.float8_e4m3fn).view(torch.uint8).permute(0, 2, 1).numpy()   # [H, 128, L]
    live = absmax.numpy() > 0
    for h in range(H):
        for d in range(128):
            if live[h, d]:
                np.testing.assert_array_equal(vt[h, d, :L], ref[h, d])
            else:
                assert not vt[h, d].any() and vs[h, d] == 0
    np.testing.assert_array_equal(vs[live], (absmax / 2.25).numpy()[live])
    assert not vt[:, :, L:].any()


def test_sage_k_per_thread_golden():
    """Sage per_thread K quantization with mean smoothing: the oracle equals the
    reference's in-tree kernel (model/sage_fused_quant.py:20-162) code for code and
    scale for scale, on the reference test's ragged non-zero-mean inputs."""
    z = np.load(os.path.join(G, "sage_k_per_thread.npz"))
    for L in (197, 64, 1000):
        q, sc = O.quant_per_thread(z[f"k{L}"], 1, z[f"kmean{L}"])
        np.testing.assert_array_equal(q[:, :L].transpose(1, 0, 2), z[f"kq{L}"])
        np.testing.assert_array_equal(sc, z[f"ks{L}"])
        assert not q[:, L:].any()


def test_kernel_order_attention_models_the_p_format():
    """The kernel-order oracle (P -> E4M3 under the lazy running max) sits at the
    E4M3 format error from exact softmax over the same operands (rel-L2 about 2.5 %,
    cos >= 0.999), for per-block and per_thread scale groups alike."""
    g = np.random.default_rng(0)
    L, H = 300, 2
    q = O.f32_to_bf16_bits(g.standard_normal((L, H, 128)).astype(np.float32))
    k = O.f32_to_bf16_bits((g.standard_normal((L, H, 128)) + 3 * g.standard_normal((1, H, 128))).astype(np.float32))
    v = O.f32_to_bf16_bits(g.standard_normal((L, H, 128)).astype(np.float32))
    mean = O.key_mean(k)
    vt, vs = O.value_fp8(v)
    thr = np.full(H, -0.1, np.float32)
    _, _, qb, qbs = O.pool_sim_quant(q, 128, thr)
    _, _, kb, kbs = O.pool_sim_quant(k, 64, thr, mean)
    pad = lambda a: np.concatenate([a, np.zeros((H, (-a.shape[1]) % 128, 128), np.int8)], 1)
    qb, kb = pad(qb), pad(kb)
    exact = O.bf16_bits_to_f32(O.attention(qb, qbs, 128, L, kb, kbs, L, vt, vs))
    fmt = O.bf16_bits_to_f32(O.attention_kernel(qb, qbs, L, kb, kbs, L, vt, vs))
    rel = np.linalg.norm(fmt - exact) / np.linalg.norm(exact)
    cos = float((fmt * exact).sum() / np.linalg.norm(fmt) / np.linalg.norm(exact))
    assert 0.01 < rel < 0.04 and cos >= 0.999
    qt, qts = O.quant_per_thread(q, 0)
    kt, kts = O.quant_per_thread(k, 1, mean)
    fmt_t = O.bf16_bits_to_f32(O.attention_kernel(qt, qts, L, kt, kts, L, vt, vs, q_gran=1, k_gran=1))
    cos_t = float((fmt_t * exact).sum() / np.linalg.norm(fmt_t) / np.linalg.norm(exact))
    assert cos_t >= 0.999
