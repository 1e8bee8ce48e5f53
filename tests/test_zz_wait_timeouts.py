"""Runs after the other GPU tests: no bounded shared-memory wait gave up.

The streaming qmv and the fused decode attention wait on mbarriers with an
iteration limit instead of spinning forever; a wait that gives up is counted on
the device. After the whole GPU suite the count must still be zero.
"""
import ctypes

import pytest

from tests.conftest import has_gpu

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]


def test_no_wait_gave_up(built_lib):
    import torch
    from hyperion_b200 import check, lib
    torch.zeros(1, device="cuda")
    torch.cuda.synchronize()
    n = ctypes.c_int64(-1)
    check(lib().hyb_wait_timeouts(ctypes.byref(n)))
    assert n.value == 0
