"""The Ulysses layout kernels (h3b_ulysses_pack / _unpack) against the torch layout
expressions they replace: for P = 1, 2, 4, 8 ranks, in head order and with a shuffled
head order, every element lands where the exchange expects it (bit-identical copies)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("P", [1, 2, 4, 8])
@pytest.mark.parametrize("shuffled", [False, True])
def test_pack_unpack_match_torch_layout(P, shuffled):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import parallel as Pm

    g = torch.Generator(device="cuda").manual_seed(P)
    rows, H, D = 1000, 32, 128
    qkv = torch.randn(rows, 3 * H * D + 16, device="cuda", generator=g).to(torch.bfloat16)
    view = qkv[:, :3 * H * D].view(rows, 3, H, D)
    order = torch.randperm(H, device="cuda", generator=g) if shuffled else None
    hpr = H // P
    for slot in range(3):
        src = view[:, slot]
        got = Pm._pack(src, rows, H, D, P, order)
        ref = (src if order is None else src.index_select(1, order)).reshape(rows, P, hpr * D).permute(1, 0, 2)
        assert torch.equal(got, ref.contiguous())
        back = Pm._unpack(got, rows, P, hpr * D, order)
        assert torch.equal(back, src.reshape(rows, H * D))
