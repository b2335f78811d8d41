"""The no-allocation rmsnorm -> bf16 GEMM (ce_rmsnorm_gemm_bf16_noalloc),
called through the C ABI, against the plan entry point that keeps its
operand in cudaMalloc'd workspace.

Callers of this entry point cannot allocate device memory (graph capture in
progress, a framework allocator owning the device, no implicit sync allowed),
so its operand lives in a fixed array inside the library. This file is named
to be collected last: if it fails, a run that stops at the first failure has
already run every other test. It passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

_vp, _i, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def _noalloc(ce):
    fn = ce.lib().ce_rmsnorm_gemm_bf16_noalloc
    fn.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp]
    fn.restype = ctypes.c_int
    return fn


def test_noalloc_matches_plan_two_calls(ce, O, dev):
    fn = _noalloc(ce)
    b, s, r = 96, 1000, 700  # ragged size: padded operand rows of 1024
    stream = torch.cuda.current_stream().cuda_stream
    ld_w = ((s + 63) // 64) * 64
    for call, seed in enumerate((1, 2)):  # two calls in a row, different inputs
        x, w, _, W = O.trio_inputs(seed, b, s, r)
        dx, dw, dW = (torch.from_numpy(a).to(dev) for a in (x, w, W))
        wb = torch.empty((r, ld_w), dtype=torch.int16, device=dev)
        ce.convert_bf16(wb, dW)

        plan = ce.Plan(b, s, r, ce.PREC_BF16)
        plan.set_weights(dW)
        want = torch.full((b, r), float("nan"), device=dev)
        want_norm = torch.full((b, s), float("nan"), device=dev)
        plan.rmsnorm_gemm(want, dx, dw, normalized=want_norm)

        got = torch.full((b, r), float("nan"), device=dev)
        got_norm = torch.full((b, s), float("nan"), device=dev)
        rc = fn(got.data_ptr(), got_norm.data_ptr(), dx.data_ptr(), dw.data_ptr(), wb.data_ptr(),
                ld_w, b, s, r, ce.RMS_EPS, stream)
        assert rc == ce.OK, ce.last_error()
        ce.device_status()
        plan.close()

        g, wnt = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}"
        # the bf16 GEMM tolerance of the other tests: relative L2 <= 1e-2,
        # here against the existing entry point's output
        assert O.rel_l2(g, wnt) <= 1e-2, f"call {call}"
        gn, wn = got_norm.cpu().numpy(), want_norm.cpu().numpy()
        assert np.all(np.abs(gn - wn) <= 1e-5 * np.abs(wn) + 1e-30), f"call {call}"
        # and the oracle: the double GEMM of the fp32 normalized rows
        ref, _ = O.gemm_ref(O.rmsnorm_ref(x, w), W)
        assert O.rel_l2(g, ref) <= 1e-2, f"call {call}"


def test_noalloc_without_normalized_output_fits_after_rounding(ce, O, dev):
    """normalized_dev = NULL (only the product is wanted), at the largest
    batch whose rounded-up operand still fits: 1024 x roundup(4033, 64) =
    4,194,304 values, exactly the operand."""
    fn = _noalloc(ce)
    b, s, r = 1024, 4033, 96
    stream = torch.cuda.current_stream().cuda_stream
    ld_w = ((s + 7) // 8) * 8
    x, w, _, W = O.trio_inputs(3, b, s, r)
    dx, dw, dW = (torch.from_numpy(a).to(dev) for a in (x, w, W))
    wb = torch.empty((r, ld_w), dtype=torch.int16, device=dev)
    ce.convert_bf16(wb, dW)
    plan = ce.Plan(b, s, r, ce.PREC_BF16)
    plan.set_weights(dW)
    want = torch.full((b, r), float("nan"), device=dev)
    plan.rmsnorm_gemm(want, dx, dw)
    got = torch.full((b, r), float("nan"), device=dev)
    rc = fn(got.data_ptr(), None, dx.data_ptr(), dw.data_ptr(), wb.data_ptr(), ld_w, b, s, r, ce.RMS_EPS,
            stream)
    assert rc == ce.OK, ce.last_error()
    ce.device_status()
    plan.close()
    g = got.cpu().numpy()
    assert np.isfinite(g).all()
    assert O.rel_l2(g, want.cpu().numpy()) <= 1e-2


@pytest.mark.parametrize("batch,size,ld_w,words", [
    (1025, 4096, 4096, ("exceeds", "4194304")),  # too many values
    (1025, 4033, 4040, ("exceeds", "4198400")),  # fits unrounded (4,133,825), not rounded up to 64
    (64, 512, 511, ("leading dimension",)),      # ld_w < size
    (64, 512, 513, ("multiple of 8",)),          # ld_w not a multiple of 8
])
def test_noalloc_rejects_bad_shapes(ce, dev, batch, size, ld_w, words):
    fn = _noalloc(ce)
    # rejected before any device work, so dummy non-null pointers are never touched
    dummy = 256
    rc = fn(dummy, None, dummy, dummy, dummy, ld_w, batch, size, 64, 1e-5, None)
    assert rc == ce.ERR_USAGE
    code, msg = ce.last_error()
    assert all(w in msg for w in words), msg
