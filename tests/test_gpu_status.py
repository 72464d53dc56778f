"""Failure detection without a GPU fault: a kernel whose mbarrier wait can
never complete gives up after its limit, records the status bit, and returns;
the context stays usable for the next launch."""

from __future__ import annotations

import pytest
import torch

from transformer_opt import attention_forward
from transformer_opt.kernels import _native

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports():
    _native.device_status(0, clear=True)
    _native.selftest_wait_timeout(0, timeout_us=2000)
    status = _native.device_status(0, clear=True)
    assert status & _native.STATUS_SELFTEST_TIMEOUT
    assert not status & _native.STATUS_PIPELINE_TIMEOUT
    # the context is intact: a real kernel still runs and the word stays clean
    q = torch.randn(1, 64, 2, 64, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        out, decision = attention_forward(q, q, q, backend="b200")
    torch.cuda.synchronize()
    assert decision.selected == "b200" and torch.isfinite(out).all()
    assert _native.device_status(0) == 0
