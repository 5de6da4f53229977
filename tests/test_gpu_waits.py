"""Failure detection without a GPU fault: a kernel waits on an mbarrier that
nothing completes; its bounded wait must give up after the limit, record
MB_ERR_DEVICE_TIMEOUT in the device status word and return, leaving the context
usable (no trap, no hang)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives():
    import metalblas_b200 as mb
    mb.kernels.device_status_clear()
    assert mb.kernels.device_status() == 0
    mb.kernels.debug_wait_timeout(2000)          # 2 ms limit
    assert mb.kernels.device_status() == 4       # MB_ERR_DEVICE_TIMEOUT
    mb.kernels.device_status_clear()
    assert mb.kernels.device_status() == 0
    a = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    b = torch.randn(512, 384, device="cuda").to(torch.bfloat16)
    c = mb.matmul(a, b)
    ref = a.float() @ b.float()
    assert torch.allclose(c.float(), ref, rtol=2e-2, atol=2e-1)
    assert mb.kernels.device_status() == 0


def test_limit_is_validated():
    import metalblas_b200 as mb
    with pytest.raises(ValueError):
        mb.kernels.debug_wait_timeout(0)
