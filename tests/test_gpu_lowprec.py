"""GPU parity of the FP8-E4M3 per-row path (BASELINE config 3's first case):
device codes and scales bit-exact against the oracle's quantizer, the fused
rmsnorm -> E4M3 operand, the kind::f8f6f4 GEMM against the double GEMM of
the dequantized operands (the implementation-check bound of
experiments/blackwell/lowprec/decoder_lowprec.cu:981-1052 and <= 1e-2
relative L2, north star), and the FP8 plan."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ld16(k):
    return ((k + 15) // 16) * 16


def test_weight_quantizer_bit_exact(ce, O, dev):
    rows, cols = 67, 1000
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((rows, cols)) * rng.uniform(0.01, 50, (rows, 1))).astype(np.float32)
    x[3] = 0.0
    x[5, 7] = 1e30
    ld = _ld16(cols)
    codes = torch.full((rows, ld), 0x55, dtype=torch.uint8, device=dev)
    scales = torch.full((rows,), float("nan"), device=dev)
    ce.quantize_e4m3_rows(codes, scales, torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    want_c, want_s = O.quantize_e4m3_rows(x)
    hc = codes.cpu().numpy()
    assert np.array_equal(hc[:, :cols], want_c)
    assert np.all(hc[:, cols:] == 0)
    assert np.array_equal(scales.cpu().numpy(), want_s)


@pytest.mark.parametrize("shape", [(8, 288), (64, 16384), (33, 1024)])
def test_rmsnorm_e4m3_operand(ce, O, dev, shape):
    rows, cols = shape
    x, w, _, _ = O.trio_inputs(2, rows, cols, 1)
    dx, dw = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
    ld = ((cols + 63) // 64) * 64
    out = torch.full((rows, cols), float("nan"), device=dev)
    codes = torch.full((rows, ld), 0x55, dtype=torch.uint8, device=dev)
    scales = torch.full((rows,), float("nan"), device=dev)
    ce.rmsnorm_e4m3(out, codes, scales, dx, dw)
    ref_out = torch.full((rows, cols), float("nan"), device=dev)
    ce.rmsnorm(ref_out, dx, dw)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    want_c, want_s = O.quantize_e4m3_rows(out.cpu().numpy())
    hc = codes.cpu().numpy()
    assert np.array_equal(hc[:, :cols], want_c)
    assert np.all(hc[:, cols:] == 0)
    assert np.array_equal(scales.cpu().numpy(), want_s)


def _check_e4m3_gemm(O, d, ca, sa, cb, sb):
    a = O.dequantize_e4m3_rows(ca, sa)
    b = O.dequantize_e4m3_rows(cb, sb)
    ref, mag = O.gemm_ref(a, b)
    k = ca.shape[1]
    bound = O.gamma_worst(k) * mag + 2.0 ** -22 * np.abs(ref) + 1e-30
    err = np.abs(d.astype(np.float64) - ref)
    assert np.all(err <= bound), float((err / bound).max())
    assert O.rel_l2(d, ref) <= 1e-2


@pytest.mark.parametrize("shape", [(8, 768, 288), (300, 1000, 512), (1024, 1000, 1040), (1, 1, 16)])
def test_gemm_e4m3(ce, O, dev, shape):
    M, N, K = shape
    rng = np.random.default_rng(M + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    ca, sa = O.quantize_e4m3_rows(A)
    cb, sb = O.quantize_e4m3_rows(B)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_e4m3(d, torch.from_numpy(ca).to(dev), torch.from_numpy(sa).to(dev),
                 torch.from_numpy(cb).to(dev), torch.from_numpy(sb).to(dev))
    ce.device_status()
    _check_e4m3_gemm(O, d.cpu().numpy(), ca, sa, cb, sb)


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("tile_n", [128, 224, 256])
def test_forced_kernel_e4m3(ce, O, dev, cta_group, tile_n):
    M, N, K = 300, 1000, 528
    rng = np.random.default_rng(tile_n + cta_group)
    ca = rng.integers(0, 256, (M, K), dtype=np.uint8)
    cb = rng.integers(0, 256, (N, K), dtype=np.uint8)
    ca[(ca & 0x7F) == 0x7F] = 0  # no NaN codes
    cb[(cb & 0x7F) == 0x7F] = 0
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_config(ce.PREC_FP8_E4M3, d, torch.from_numpy(ca).to(dev), torch.from_numpy(cb).to(dev),
                   cta_group=cta_group, tile_n=tile_n)
    ce.device_status()
    _check_e4m3_gemm(O, d.cpu().numpy(), ca, np.ones(M, np.float32), cb, np.ones(N, np.float32))


@pytest.mark.parametrize("shape", [(8, 288, 768), (64, 1024, 512), (1024, 16384, 8192)])
def test_plan_fp8_trio(ce, O, dev, shape):
    b, s, r = shape
    x, w, logits, W = (O.trio_inputs if b < 1024 else ce.trio_inputs_host)(0, b, s, r)
    plan = ce.Plan(b, s, r, ce.PREC_FP8_E4M3)
    plan.set_weights(torch.from_numpy(W).to(dev))
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    norm = torch.empty((b, s), device=dev)
    soft = torch.empty((b, s), device=dev)
    out = torch.full((b, r), float("nan"), device=dev)
    plan.trio(norm, soft, out, dx, dw, dl)
    ce.device_status()
    hn = norm.cpu().numpy()
    rows = np.arange(b) if b <= 64 else np.random.default_rng(0).choice(b, 24, replace=False)
    ca, sa = O.quantize_e4m3_rows(hn[rows])
    cb, sb = O.quantize_e4m3_rows(W)
    a = O.dequantize_e4m3_rows(ca, sa)
    bq = O.dequantize_e4m3_rows(cb, sb)
    ref, _ = O.gemm_ref(a, bq)
    ho = out.cpu().numpy()[rows]
    assert O.rel_l2(ho, ref) <= 1e-2       # against the dequantized operands
    ref32, _ = O.gemm_ref(O.rmsnorm_ref(x[rows], w), W)
    assert O.rel_l2(ho, ref32) <= 0.08     # quantization error of both operands (e4m3)
    plan.close()


def _crafted_rows(O, width, rows, seed):
    x = O.normals(seed, 1, rows * width).reshape(rows, width).copy()
    x[1, :32] = 0.0                               # zero block
    x[2, 32:64] = 28.0 * 2.0 ** -3                 # exact largest-code block
    x[3, :16] = np.float32(1e-30)                  # tiny block
    x[4, 64:96] = np.linspace(-40, 40, 32)         # saturation
    x[5, :] *= 1e-20
    x[6, 96:128] = (np.arange(32) % 4) * 0.125     # ties
    return np.ascontiguousarray(x.astype(np.float32))


@pytest.mark.parametrize("shape", [(130, 1024), (7, 1000), (64, 16384)])
def test_mxfp6_quantizer_bit_exact(ce, O, dev, shape):
    rows, width = shape
    x = _crafted_rows(O, width, rows, 2)
    nb = (width + 31) // 32
    codes = torch.full((rows, width), 0x55, dtype=torch.uint8, device=dev)
    scales = torch.full((rows, nb), 0x55, dtype=torch.uint8, device=dev)
    ce.quantize_mxfp6(codes, scales, torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    L = O.orc()
    wc = np.empty((rows, nb * 32), np.uint8)
    ws = np.empty((rows, nb), np.uint8)
    for r in range(rows):
        row = np.zeros(nb * 32, np.float32)
        row[:width] = x[r]
        L.orc_quantize_mxfp6(row, width, wc[r], ws[r])
    assert np.array_equal(codes.cpu().numpy(), wc[:, :width])
    assert np.array_equal(scales.cpu().numpy(), ws)


@pytest.mark.parametrize("shape", [(130, 1024), (7, 1000), (64, 16384)])
def test_nvfp4_quantizer_bit_exact(ce, O, dev, shape):
    rows, width = shape
    x = _crafted_rows(O, width, rows, 3)
    nb = (width + 15) // 16
    ldb = (width + 1) // 2
    codes = torch.full((rows, ldb), 0x55, dtype=torch.uint8, device=dev)
    scales = torch.full((rows, nb), 0x55, dtype=torch.uint8, device=dev)
    ts = torch.full((2,), float("nan"), device=dev)
    scratch = torch.zeros(1, dtype=torch.int32, device=dev)
    ce.quantize_nvfp4(codes, scales, ts, scratch, torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    L = O.orc()
    s = L.orc_nvfp4_encode_scale(float(np.abs(x).max()))
    assert ts.cpu().numpy()[0] == np.float32(s)
    assert ts.cpu().numpy()[1] == np.float32(1.0) / np.float32(s)
    wc = np.empty((rows, nb * 16), np.uint8)
    ws = np.empty((rows, nb), np.uint8)
    for r in range(rows):
        row = np.zeros(nb * 16, np.float32)
        row[:width] = x[r]
        L.orc_quantize_nvfp4(row, width, s, wc[r], ws[r])
    packed = (wc[:, 0::2] | (wc[:, 1::2] << 4)).astype(np.uint8)[:, :ldb]
    assert np.array_equal(scales.cpu().numpy(), ws)
    assert np.array_equal(codes.cpu().numpy(), packed)
