"""GPU parity of the row kernels (rmsnorm, softmax, GEMV and their one-launch
fusion) against the oracle, through the C ABI. Shapes follow the reference's
own check matrix (llama2c/Makefile:25-28, 44-56: 64x1000x300, 33x1001x77 for
the generic path, 1024x16384x8192) plus config 1 (8x288x768), the minimum
shape and a row too long for the register path."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(8, 288, 768), (64, 1000, 300), (33, 1001, 77), (3, 2, 2), (1, 4100, 300),
          (16, 40000, 64), (64, 256, 512)]


def _poisoned(shape, dev):
    return torch.full(shape, float("nan"), device=dev)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("random,seed", [(0, 0), (1, 1), (1, 2)])
def test_iteration_matches_reference_oracle(ce, O, dev, shape, random, seed):
    b, s, r = shape
    x, p, w, m = O.llama2c_inputs(random, seed, b, s, r)
    dx, dp, dw, dm = (torch.from_numpy(a).to(dev) for a in (x, p, w, m))
    norm, soft, prod = _poisoned((b, s), dev), _poisoned((b, s), dev), _poisoned((r,), dev)
    ce.llama2c_iteration(norm, soft, prod, dx, dw, dp, dm)
    torch.cuda.synchronize()
    hn, hs, hp = norm.cpu().numpy(), soft.cpu().numpy(), prod.cpu().numpy()
    valid, tol, refv = O.validate_llama2c(random, x, p, w, m, hn, hs, hp)
    assert valid
    # 1e-5 relative for the fp32 norm and softmax
    en = O.rmsnorm_ref(x, w)
    assert np.all(np.abs(hn - en) <= 1e-5 * np.abs(en) + 1e-30)
    es = O.softmax_ref(p)
    assert np.all(np.abs(hs - es) <= 1e-5 * es + 1e-12)


@pytest.mark.parametrize("shape", [(8, 288, 768), (33, 1001, 77), (64, 16384, 256)])
def test_single_ops_equal_fused_launch(ce, O, dev, shape):
    """ce_rmsnorm / ce_softmax / ce_gemv give bitwise the fused iteration's values."""
    b, s, r = shape
    x, p, w, m = O.llama2c_inputs(1, 4, b, s, r)
    dx, dp, dw, dm = (torch.from_numpy(a).to(dev) for a in (x, p, w, m))
    n1, s1, p1 = _poisoned((b, s), dev), _poisoned((b, s), dev), _poisoned((r,), dev)
    ce.llama2c_iteration(n1, s1, p1, dx, dw, dp, dm)
    n2, s2, p2 = _poisoned((b, s), dev), _poisoned((b, s), dev), _poisoned((r,), dev)
    ce.rmsnorm(n2, dx, dw)
    ce.softmax(s2, dp)
    ce.gemv(p2, dm, dx.reshape(-1)[:s])
    torch.cuda.synchronize()
    assert torch.equal(n1, n2) and torch.equal(s1, s2) and torch.equal(p1, p2)


@pytest.mark.parametrize("shape", [(8, 288, 768), (33, 1001, 77)])
def test_partial_launches_equal_fused_launch(ce, O, dev, shape):
    """The copy-mode split (rmsnorm rows alone, then softmax + GEMV rows in a
    second launch on another stream) gives bitwise the fused iteration's
    values and leaves the other outputs untouched."""
    b, s, r = shape
    x, p, w, m = O.llama2c_inputs(1, 5, b, s, r)
    dx, dp, dw, dm = (torch.from_numpy(a).to(dev) for a in (x, p, w, m))
    n1, s1, p1 = _poisoned((b, s), dev), _poisoned((b, s), dev), _poisoned((r,), dev)
    ce.llama2c_iteration(n1, s1, p1, dx, dw, dp, dm)
    n2, s2, p2 = _poisoned((b, s), dev), _poisoned((b, s), dev), _poisoned((r,), dev)
    ce.llama2c_rows(n2, None, None, dx, dw, None, None, b, 0, 0)
    torch.cuda.synchronize()
    assert torch.equal(n1, n2)
    assert torch.isnan(s2).all() and torch.isnan(p2).all()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        ce.llama2c_rows(None, s2, p2, dx, None, dp, dm, 0, b, r, stream=side)
    torch.cuda.synchronize()
    assert torch.equal(s1, s2) and torch.equal(p1, p2)
    # partial row counts: only the first rows are written
    n3 = _poisoned((b, s), dev)
    ce.llama2c_rows(n3, None, None, dx, dw, None, None, b // 2, 0, 0)
    torch.cuda.synchronize()
    assert torch.equal(n3[: b // 2], n1[: b // 2]) and torch.isnan(n3[b // 2:]).all()


def test_deterministic_identity_gemv(ce, O, dev):
    """Known answer (llama2c_common.h:195-196): with the shifted-identity
    matrix the GEMV is a gather, product[r] == input[r % size] exactly."""
    b, s, r = 4, 512, 1500
    x, p, w, m = O.llama2c_inputs(0, 0, b, s, r)
    dx, dm = torch.from_numpy(x).to(dev), torch.from_numpy(m).to(dev)
    prod = _poisoned((r,), dev)
    ce.gemv(prod, dm, dx.reshape(-1)[:s])
    assert np.array_equal(prod.cpu().numpy(), x.ravel()[np.arange(r) % s])


def test_rmsnorm_bf16_operand(ce, O, dev):
    """The fused GEMM-operand output is the RNE bf16 of the fp32 output, with
    zero padding columns."""
    b, s, ld = 37, 1000, 1024
    x, w, _, _ = O.trio_inputs(3, b, s, 4)
    dx, dw = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
    out = _poisoned((b, s), dev)
    ob = torch.full((b, ld), -1, dtype=torch.int16, device=dev)
    ce.rmsnorm_bf16(out, ob, dx, dw)
    torch.cuda.synchronize()
    hb = ob.cpu().numpy().view(np.uint16)
    assert np.array_equal(hb[:, :s], O.bf16_bits(out.cpu().numpy()))
    assert np.all(hb[:, s:] == 0)


def test_sheet_shape(ce, O, dev):
    """BASELINE config 2 (1024 x 16384, 8192 rows), reference random inputs:
    the reference's full validate_all plus the 1e-5 relative bound."""
    b, s, r = 1024, 16384, 8192
    x, p, w, m = ce.fill_llama2c_host(1, 1, b, s, r)
    dx, dp, dw, dm = (torch.from_numpy(a).to(dev) for a in (x, p, w, m))
    norm, soft, prod = _poisoned((b, s), dev), _poisoned((b, s), dev), _poisoned((r,), dev)
    ce.llama2c_iteration(norm, soft, prod, dx, dw, dp, dm)
    torch.cuda.synchronize()
    hn, hs, hp = norm.cpu().numpy(), soft.cpu().numpy(), prod.cpu().numpy()
    valid, _, _ = O.validate_llama2c(1, x, p, w, m, hn, hs, hp)
    assert valid
    en = O.rmsnorm_ref(x, w)
    assert np.all(np.abs(hn - en) <= 1e-5 * np.abs(en) + 1e-30)
    es = O.softmax_ref(p)
    assert np.all(np.abs(hs - es) <= 1e-5 * es + 1e-12)


@pytest.mark.parametrize("batch,size", [(1024, 16384), (300, 8192), (7, 12288)])
def test_streaming_rows_kernel_equals_register_kernel(ce, O, dev, batch, size):
    """The trio's rows stage on long rows (32-64 KiB) runs the persistent
    streaming kernel (bulk copies two rows ahead); the llama2c iteration with
    its GEMV rows still runs the one-row-per-CTA register kernel. Both give
    the same bits for the normalized and softmax rows, and the streaming
    kernel's bf16 operand is the rounding of its fp32 output."""
    x, w, logits, _ = O.trio_inputs(5, batch, size, 8)
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    mat = torch.zeros((8, size), device=dev)
    n_reg, s_reg = torch.full_like(dx, float("nan")), torch.full_like(dl, float("nan"))
    prod = torch.empty(8, device=dev)
    ce.llama2c_iteration(n_reg, s_reg, prod, dx, dw, dl, mat)
    plan = ce.Plan(batch, size, 8, ce.PREC_BF16)
    n_str, s_str = torch.full_like(dx, float("nan")), torch.full_like(dl, float("nan"))
    plan.rows(n_str, s_str, dx, dw, dl)
    a = torch.empty((batch, size), device=dev)
    plan.operands(a=a)
    ce.device_status()
    plan.close()
    assert torch.equal(n_reg, n_str)
    assert torch.equal(s_reg, s_str)
    assert torch.equal(a, n_str.to(torch.bfloat16).float())
