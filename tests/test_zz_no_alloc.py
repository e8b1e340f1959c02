"""The allocation-free K-mean entry point, h3b_key_mean_no_alloc.

Some hosts cannot give this library a device workspace: a serving process that
has handed all GPU memory to its own pool, or code running where a device
allocation is not allowed.  For them the library keeps a fixed scratch array
inside libh3b.so.  These tests call that entry point through the C ABI and
require the same bytes as h3b_key_mean (which takes a caller workspace), twice
in a row so that the scratch left by the first call cannot leak into the
second.  This file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b._lib import lib as _lib
    return _lib()


def _keys(L, H, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(L, H * 128, generator=g) * 0.5 + torch.randn(1, H * 128, generator=g) * 3
    return k.to(torch.bfloat16).cuda()


def _with_workspace(lib, k, L, H):
    need = lib.h3b_key_mean_workspace_bytes(L, H)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    mean = torch.empty(H, 128, dtype=torch.bfloat16, device="cuda")
    st = lib.h3b_key_mean(ctypes.c_void_p(k.data_ptr()), L, H, k.stride(0), ctypes.c_void_p(mean.data_ptr()),
                          ctypes.c_void_p(ws.data_ptr()), need, None)
    assert st == 0, lib.h3b_last_error()
    return mean


def _no_alloc(lib, k, L, H):
    mean = torch.empty(H, 128, dtype=torch.bfloat16, device="cuda")
    st = lib.h3b_key_mean_no_alloc(ctypes.c_void_p(k.data_ptr()), L, H, k.stride(0),
                                   ctypes.c_void_p(mean.data_ptr()), None)
    assert st == 0, lib.h3b_last_error()
    return mean


def test_no_alloc_key_mean_matches_workspace_entry_twice(lib):
    # two different shapes in a row: the second call reuses the scratch the first one filled
    for L, H, seed in ((111600 // 8, 32, 1), (5000, 4, 2)):
        k = _keys(L, H, seed)
        got = _no_alloc(lib, k, L, H)
        ref = _with_workspace(lib, k, L, H)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_no_alloc_key_mean_rejects_sizes_beyond_its_scratch(lib):
    # ceil(L/1024) * H * 128 > 2^20 partial sums: refused before any launch (k is
    # allocated at full size anyway, so nothing could read out of bounds)
    k = torch.zeros(262144 + 1024, 32 * 128, dtype=torch.bfloat16, device="cuda")
    mean = torch.empty(32, 128, dtype=torch.bfloat16, device="cuda")
    st = lib.h3b_key_mean_no_alloc(ctypes.c_void_p(k.data_ptr()), 262144 + 1024, 32, 32 * 128,
                                   ctypes.c_void_p(mean.data_ptr()), None)
    assert st == -2
    assert b"exceed the fixed scratch" in lib.h3b_last_error()
    from h3b import device_status
    assert device_status(0) == 0
