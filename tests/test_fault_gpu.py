"""Failure detection on the GPU without faulting it: a bounded device wait that
nothing completes must give up, leave DAK_ERR_TIMEOUT in the device error word
and leave the CUDA context usable for the next launch."""
import numpy as np
import pytest
import torch

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_stays_usable():
    from directaccesskernel_b200 import _lib, runtime

    assert runtime.device_status() == 0
    _lib.check(_lib.LIB.dak_selftest_wait_timeout(20000, torch.cuda.current_stream().cuda_stream), "selftest")
    assert runtime.device_status(clear=True) == _lib.DAK_ERR_TIMEOUT
    assert runtime.device_status() == 0  # cleared
    # The context still runs kernels correctly.
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(256, 512, generator=g) * 0.02).half()
    x = torch.randn(2, 512, generator=g).half()
    y = torch.empty(2, 256, dtype=torch.float16, device="cuda")
    runtime.linear_split(x.cuda(), y, None, w.t().contiguous().cuda())
    assert rel_err(y.float().cpu().numpy(), oracle.linear(x.numpy(), w.numpy())) < 1e-2
    assert runtime.device_status() == 0


def test_selftest_rejects_bad_timeouts():
    from directaccesskernel_b200 import _lib

    assert _lib.LIB.dak_selftest_wait_timeout(0, None) == _lib.DAK_ERR_INVALID_ARG
