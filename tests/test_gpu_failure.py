"""Failure detection on the GPU without a fault: the bounded mbarrier wait
every pipeline role uses runs out on a barrier nothing arrives at, reports
FRN_DEVERR_WAIT_TIMEOUT through the device error word, and the context stays
usable for the next fused call."""
import time

import pytest
import torch

from oracle import rmsnorm_linear as orc
from src import capi

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_survives():
    capi.device_error(0, clear=True)
    t0 = time.perf_counter()
    capi.selftest_wait_timeout(100)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert 0.09 <= dt < 5.0, f"wait lasted {dt:.3f} s"
    flags = capi.device_error(0, clear=True)
    assert flags & 0x1, f"device error word {flags:#x}"
    assert capi.device_error(0) == 0
    # the next fused launch on the same context is correct
    x, gamma, W = orc.make_inputs(300, 512, 1024, seed=2)
    Wn = orc.fold_gamma(W, gamma)
    out = capi.fused_rmsnorm_linear(x.cuda(), Wn.cuda(), None, orc.EPS)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), orc.unfused_reference(x, gamma, W, None,
                                                                        orc.EPS).float(),
                               atol=2e-2, rtol=2e-2)
    assert capi.device_error(0) == 0


def test_selftest_rejects_unbounded_limits():
    with pytest.raises(capi.FrnError, match="timeout_ms"):
        capi.selftest_wait_timeout(0)
    with pytest.raises(capi.FrnError, match="timeout_ms"):
        capi.selftest_wait_timeout(60000)
