"""GPU parity of the op-trio plan (rmsnorm -> GEMM on the normalized batch,
softmax) for every available precision, and CUDA-graph replay equality."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PRECS = {"fp32": 0, "tf32": 1, "bf16": 2}
# relative L2 against the double reference on fp32 operands
REL_L2 = {"fp32": 1e-5, "tf32": 1e-2, "bf16": 1e-2}


def _run(ce, O, dev, prec, b, s, r, seed=0):
    x, w, logits, W = O.trio_inputs(seed, b, s, r)
    plan = ce.Plan(b, s, r, PRECS[prec])
    plan.set_weights(torch.from_numpy(W).to(dev))
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    norm = torch.full((b, s), float("nan"), device=dev)
    soft = torch.full((b, s), float("nan"), device=dev)
    out = torch.full((b, r), float("nan"), device=dev)
    plan.trio(norm, soft, out, dx, dw, dl)
    ce.device_status()
    return plan, (x, w, logits, W), (dx, dw, dl), (norm, soft, out)


@pytest.mark.parametrize("prec", list(PRECS))
@pytest.mark.parametrize("shape", [(8, 288, 768), (64, 1024, 128), (33, 1000, 77)])
def test_trio(ce, O, dev, prec, shape):
    b, s, r = shape
    plan, (x, w, logits, W), _, (norm, soft, out) = _run(ce, O, dev, prec, b, s, r)
    en = O.rmsnorm_ref(x, w)
    hn = norm.cpu().numpy()
    assert np.all(np.abs(hn - en) <= 1e-5 * np.abs(en) + 1e-30)
    es = O.softmax_ref(logits)
    assert np.all(np.abs(soft.cpu().numpy() - es) <= 1e-5 * es + 1e-12)
    ref, _ = O.gemm_ref(en, W)
    assert O.rel_l2(out.cpu().numpy(), ref) <= REL_L2[prec]
    plan.close()


def test_trio_graph_replay_is_bitwise(ce, O, dev):
    b, s, r = 64, 1024, 512
    plan, _, (dx, dw, dl), (norm, soft, out) = _run(ce, O, dev, "bf16", b, s, r)
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            plan.trio(norm, soft, out, dx, dw, dl)
    out.fill_(float("nan"))
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    ce.device_status()
    assert torch.equal(out, first)
    plan.close()


def test_trio_sheet_shape_bf16(ce, O, dev):
    """BASELINE config 2 with the bf16 GEMM: 1024 x 16384 x 8192."""
    b, s, r = 1024, 16384, 8192
    x, w, logits, W = ce.trio_inputs_host(0, b, s, r)
    plan = ce.Plan(b, s, r, ce.PREC_BF16)
    plan.set_weights(torch.from_numpy(W).to(dev))
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    norm = torch.empty((b, s), device=dev)
    soft = torch.empty((b, s), device=dev)
    out = torch.empty((b, r), device=dev)
    plan.trio(norm, soft, out, dx, dw, dl)
    ce.device_status()
    rows = np.random.default_rng(1).choice(b, 32, replace=False)
    en = O.rmsnorm_ref(x[rows], w)
    ref, _ = O.gemm_ref(en, W)
    assert O.rel_l2(out.cpu().numpy()[rows], ref) <= 1e-2
    hn = norm.cpu().numpy()[rows]
    assert np.all(np.abs(hn - en) <= 1e-5 * np.abs(en) + 1e-30)
    plan.close()


ALL_PRECS = ["fp32", "tf32", "bf16", "fp8", "mxfp6", "nvfp4"]


def _reconstruct(ce, O, dev, prec, X):
    """The GEMM operand the plan forms from fp32 rows X (device), rebuilt
    from the standalone quantizers / conversions and dequantized in the
    oracle, rounded to fp32 once as the device does."""
    n, s = X.shape
    h = X.cpu().numpy()
    if prec in ("fp32", "tf32"):
        return h
    if prec == "bf16":
        return O.bf16_value(O.bf16_bits(h)).astype(np.float32)
    if prec == "fp8":
        codes, scales = O.quantize_e4m3_rows(h)
        return O.dequantize_e4m3_rows(codes, scales).astype(np.float32)
    if prec == "mxfp6":
        c = torch.empty((n, s), dtype=torch.uint8, device=dev)
        sc = torch.empty((n, s // 32), dtype=torch.uint8, device=dev)
        ce.quantize_mxfp6(c, sc, X)
        return O.dequantize_mxfp6(c.cpu().numpy(), sc.cpu().numpy()).astype(np.float32)
    c = torch.empty((n, s // 2), dtype=torch.uint8, device=dev)
    sc = torch.empty((n, s // 16), dtype=torch.uint8, device=dev)
    ts = torch.empty(2, device=dev)
    scratch = torch.zeros(1, dtype=torch.int32, device=dev)
    ce.quantize_nvfp4(c, sc, ts, scratch, X)
    return O.dequantize_nvfp4(c.cpu().numpy(), sc.cpu().numpy(), s,
                              float(ts.cpu()[1])).astype(np.float32)


@pytest.mark.parametrize("prec", ALL_PRECS)
@pytest.mark.parametrize("shape", [(8, 384, 300), (130, 1024, 250)])
def test_plan_operands_are_the_quantized_operands(ce, O, dev, prec, shape):
    """ce_plan_operands returns, bit for bit, the operands the plan's GEMM
    multiplies (the standalone quantizers are bit-exact against the
    reference's host quantizer), and the GEMM output is within the
    implementation-check bound of their double product."""
    b, s, r = shape
    pval = {"fp32": ce.PREC_FP32, "tf32": ce.PREC_TF32, "bf16": ce.PREC_BF16,
            "fp8": ce.PREC_FP8_E4M3, "mxfp6": ce.PREC_MXFP6_E3M2, "nvfp4": ce.PREC_NVFP4_E2M1}[prec]
    x, w, logits, W = O.trio_inputs(2, b, s, r)
    plan = ce.Plan(b, s, r, pval)
    dW = torch.from_numpy(W).to(dev)
    plan.set_weights(dW)
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    norm = torch.empty((b, s), device=dev)
    soft = torch.empty((b, s), device=dev)
    out = torch.empty((b, r), device=dev)
    plan.trio(norm, soft, out, dx, dw, dl)
    a = torch.full((b, s), float("nan"), device=dev)
    wq = torch.full((r, s), float("nan"), device=dev)
    plan.operands(a, wq)
    torch.cuda.synchronize()
    ce.device_status()
    ha, hw = a.cpu().numpy(), wq.cpu().numpy()
    assert np.array_equal(ha.view(np.uint32), _reconstruct(ce, O, dev, prec, norm).view(np.uint32))
    assert np.array_equal(hw.view(np.uint32), _reconstruct(ce, O, dev, prec, dW).view(np.uint32))
    ref, mag = O.gemm_ref(ha, hw)
    extra = 2.0 ** -9 if prec == "tf32" else 0.0
    bound = (O.gamma_worst(s) + extra) * mag + 2.0 ** -22 * np.abs(ref) + 1e-30
    assert np.all(np.abs(out.cpu().numpy().astype(np.float64) - ref) <= bound)
    plan.close()
