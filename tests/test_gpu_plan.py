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
