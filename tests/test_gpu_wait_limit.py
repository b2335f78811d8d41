"""Bounded device waits run out, report CE_ERR_TIMEOUT, and leave the GPU
usable. The reference's stream-K consumer spins on its flag without a limit
(applications/loom_private/decoder/decoder_optimized.cu:391-394); every
wait of this library gives up after the limit set by ce_set_wait_limit.

1 GPU: a row-shard exchange opened as rank 0 of 2 and never connected, so
no peer ever writes its flag; its wait kernel must give up after the short
limit, ce_device_status must say so (and clear), and a GEMM run afterwards
must still be right."""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_exchange_wait_runs_out_and_reports(ce, dev):
    x = ce.RowExchange(4, 64, 2, 0)
    try:
        ce.set_wait_limit(0.05)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        x.wait()
        with pytest.raises(ce.CeError) as err:
            ce.device_status()
        elapsed = time.perf_counter() - t0
        assert err.value.status == ce.ERR_TIMEOUT
        assert "row-shard exchange wait" in str(err.value)
        assert 0.04 <= elapsed < 1.5, elapsed
        ce.device_status()  # the report was cleared
    finally:
        ce.set_wait_limit(2.0)
        x.close()
    # the context still works: a bf16 GEMM after the timeout is exact against
    # a float64 product of the same bf16 operands (within the gamma_K rule)
    a = torch.randn(64, 256, device=dev).to(torch.bfloat16)
    b = torch.randn(96, 256, device=dev).to(torch.bfloat16)
    d = torch.full((64, 96), float("nan"), device=dev)
    ce.gemm_bf16(d, a, b)
    ce.device_status()
    ref = a.double() @ b.double().T
    k = 256
    gamma = k * 2.0 ** -24 / (1 - k * 2.0 ** -24)
    bound = gamma * (a.double().abs() @ b.double().abs().T)
    assert bool(((d.double() - ref).abs() <= bound + 1e-30).all())


def test_unconnected_exchange_rejects_the_gemm(ce, dev):
    x = ce.RowExchange(8, 64, 2, 1)
    plan = ce.Plan(8, 128, 32, ce.PREC_BF16)
    try:
        plan.set_weights(torch.randn(32, 128, device=dev))
        with pytest.raises(ce.CeError) as err:
            plan.gemm_rowx(x)
        assert err.value.status == ce.ERR_USAGE
        assert "not connected" in str(err.value)
    finally:
        plan.close()
        x.close()


def test_wait_limit_range(ce):
    for bad in (0.0, -1.0, 1e6):
        with pytest.raises(ce.CeError) as err:
            ce.set_wait_limit(bad)
        assert err.value.status == ce.ERR_USAGE
