"""GPU parity of the loom_private llama2c decoder (applications/loom_private/
decoder/) through the C ABI: the reference's test shapes
(decoder/tests/run_tests.sh:36-50), its check protocol (poison -> run twice
per launch mode -> oracle check -> digest, all digests equal,
lp_harness.cuh:512-556), its injected faults, and the large shape's golden
digest 4fcc3e102976547b (decoder/README.md:183-185)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = {"wraparound": (40, 96, 16, 5), "minimum": (3, 2, 2, 2), "square": (1030, 1000, 1000, 3),
          "wide": (1, 4100, 300, 2), "graph-only": (70, 200, 33, 4)}


def _run(ce, dec, mode, stream):
    dec.poison_outputs(stream=stream)
    if mode == "direct":
        with torch.cuda.stream(stream):
            dec.enqueue_application(stream=stream)
    else:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                dec.enqueue_application(stream=stream)
        g.replay()
    torch.cuda.synchronize()
    ce.device_status()
    return dec.outputs()


def _digest(O, outs):
    return O.fnv1a64(list(outs))


@pytest.mark.parametrize("name", list(SHAPES))
def test_decoder_fp32_contract(ce, O, dev, name):
    B, W, V, S = SHAPES[name]
    ref = O.decoder_reference(B, W, V, S)
    dec = ce.Decoder(B, W, V, S, ce.PREC_FP32)
    stream = torch.cuda.Stream()
    modes = ["graph", "graph"] if name == "graph-only" else ["direct", "direct", "graph", "graph"]
    digests = []
    for mode in modes:
        outs = _run(ce, dec, mode, stream)
        ok, report = O.decoder_check(ref, *outs)
        assert ok, (mode, report)
        digests.append(_digest(O, outs))
    assert len(set(digests)) == 1
    dec.close()


@pytest.mark.parametrize("fault,kind", [(1, "token"), (2, "invariant"), (3, "dense")])
def test_decoder_injected_faults_are_caught(ce, O, dev, fault, kind):
    """fault 1: last generated token of the last sequence; 2: final-step
    activation of the middle sequence; 3: one final-step probability of
    sequence 0 (decoder.cu:346-358)."""
    B, W, V, S = SHAPES["wraparound"]
    ref = O.decoder_reference(B, W, V, S)
    dec = ce.Decoder(B, W, V, S, ce.PREC_FP32)
    stream = torch.cuda.Stream()
    dec.poison_outputs(stream=stream)
    with torch.cuda.stream(stream):
        dec.enqueue_application(stream=stream)
    torch.cuda.synchronize()
    dec.inject_fault(fault)
    g, n, lg, p = dec.outputs()
    if fault == 2:
        n[S - 1, B // 2, 0] *= 2.0
    if fault == 3:
        p[S - 1, 0, V // 2] *= np.float32(1.001)
    ok, report = O.decoder_check(ref, g, n, lg, p)
    assert not ok
    assert report[kind], report
    if fault == 1:
        assert report["token"][0] == "token mismatch sequence 39 step 4: expected 12, actual 13"
    if fault == 2:
        assert report["invariant"][0] == "invariant failure sequence 20 step 4"
    if fault == 3:
        assert report["dense"][0].startswith("probability mismatch sequence 0 step 4 index 8: expected")
    dec.close()


def test_decoder_skipped_prompt_upload_fails(ce, O, dev):
    """Poisoned prompts: a compute-scope run without the upload starts from
    token -1 and must fail the check (contract.json "outputs.poison")."""
    B, W, V, S = SHAPES["wraparound"]
    ref = O.decoder_reference(B, W, V, S)
    dec = ce.Decoder(B, W, V, S, ce.PREC_FP32)
    dec.poison_outputs()
    dec.enqueue_compute()
    torch.cuda.synchronize()
    g, n, lg, p = dec.outputs(from_device=True)
    ok, _ = O.decoder_check(ref, g, n, lg, p)
    assert not ok
    dec.close()


@pytest.mark.parametrize("prec", ["bf16", "tf32"])
@pytest.mark.parametrize("name", ["wraparound", "square", "graph-only"])
def test_decoder_tensor_core(ce, O, dev, prec, name):
    """Tensor-core classifiers: greedy tokens equal the analytic progression
    (the north star asks >= 99.9 %; the synthetic model gives all), the fp32
    rmsnorm is the contract's, and each logit is within the fp32-accumulation
    bound of the double dot product of the GPU's own rounded operands."""
    B, W, V, S = SHAPES[name]
    if prec == "tf32" and W % 4:
        pytest.skip("tf32 needs width % 4 == 0")
    p_ = {"bf16": ce.PREC_BF16, "tf32": ce.PREC_TF32}[prec]
    ref = O.decoder_reference(B, W, V, S)
    dec = ce.Decoder(B, W, V, S, p_)
    outs = _run(ce, dec, "direct", torch.cuda.Stream())
    g, n, lg, p = outs
    assert np.array_equal(g, ref["tokens"])
    for i, b in enumerate(ref["sampled"]):
        for s in range(S):
            e = ref["normalized"][i, s]
            assert np.all(np.abs(n[s, b] - e) <= 2e-6 * np.abs(e) + 1e-12)
    # logits: one nonzero product per row; bf16 / tf32 rounding of o
    if prec == "bf16":
        a = O.bf16_value(O.bf16_bits(n))
    else:
        a = (n.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)  # tf32 truncation bound
    perm = (np.arange(V) + V - 1) % V
    exp = a[:, :, perm].astype(np.float64)
    tol = (2.0 ** -10 if prec == "tf32" else 0.0) * np.abs(exp) + O.gamma_worst(W) * np.abs(exp) + 1e-30
    assert np.all(np.abs(lg - exp) <= tol)
    # probabilities sum to 1 and the token is the first argmax of them
    assert np.all(np.abs(p.astype(np.float64).sum(axis=2) - 1.0) <= 1e-6 + 1.2e-7 * V)
    first = np.argmax(p, axis=2)                       # [S][B]
    assert np.array_equal(first.T, g)
    dec.close()


def test_decoder_large_golden_digest(ce, O, dev):
    """The contract's large shape, 1024 x 16384 x 8192 x 4 steps, FP32 mode:
    passes the oracle check and reproduces the reference's digest."""
    B, W, V, S = 1024, 16384, 8192, 4
    ref = O.decoder_reference(B, W, V, S)
    dec = ce.Decoder(B, W, V, S, ce.PREC_FP32)
    outs = _run(ce, dec, "direct", torch.cuda.Stream())
    ok, report = O.decoder_check(ref, *outs)
    assert ok, report
    assert f"{_digest(O, outs):016x}" == "4fcc3e102976547b"
    dec.close()
