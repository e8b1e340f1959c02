"""The kernels' bounded-wait failure path, exercised on the GPU without a fault.

Every wait of the GEMM and attention kernels on a hardware barrier gives up after a
bounded time, records a code in the per-device status word and returns.  Here a
self-test kernel runs that same wait routine on a barrier nothing will release, with
a 2 ms limit: the launch must finish, h3b_device_status must report the code (and
clear it on reset), and the context must still run kernels correctly afterwards.
"""

import time

import numpy as np
import pytest
import torch

from gpu_util import bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_reports_and_leaves_the_context_usable():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from h3b import _lib, device_status, ops

    assert device_status(0) == 0
    t0 = time.monotonic()
    _lib.check(_lib.lib().h3b_selftest_bounded_wait(2_000_000, None), "selftest_bounded_wait")
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 5.0
    assert device_status(0, reset=False) == -103      # H3B_STATUS_SELFTEST_TIMEOUT, still set
    assert device_status(0) == -103                   # read and cleared
    assert device_status(0) == 0
    g = torch.Generator().manual_seed(9)
    x = torch.randn(64, 512, generator=g).to(torch.bfloat16)
    q, s = ops.quantize_int8_rowwise(x.cuda())
    qo, so = O.quant_rowwise(bits(x))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    assert device_status(0) == 0
