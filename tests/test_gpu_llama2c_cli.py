"""The llama2c drop-in executable (cuda-elastic_b200/llama2c_b200) on the
reference's own check matrix (llama2c/Makefile:44-56, check-sota: shapes
64x1000x300, 33x1001x77 and the sheet 1024x16384x8192; deterministic,
random=1, random=2; graph and direct; nocopy and copy), its dump, and the
op-trio mode (trio=PRECISION) with its L2CDUMP2 dump."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "cuda-elastic_b200", "llama2c_b200")


def run(args, env=None):
    r = subprocess.run([EXE] + args, capture_output=True, text=True, timeout=600, env=env)
    fields = dict(kv.split("=", 1) for kv in r.stdout.split()) if r.stdout.strip() else {}
    return r, fields


@pytest.mark.parametrize("shape", [(64, 1000, 300), (33, 1001, 77), (64, 256, 512)])
@pytest.mark.parametrize("inputs", ["deterministic", "random=1", "random=2"])
@pytest.mark.parametrize("mode", ["graph", "direct"])
@pytest.mark.parametrize("copy", ["nocopy", "copy"])
@pytest.mark.parametrize("layout", ["fused", "streams"])
def test_check_matrix(shape, inputs, mode, copy, layout):
    b, s, r = shape
    res, f = run([mode, "3", str(b), str(s), str(r), "1", "1", copy, "coalesced", inputs, layout])
    assert res.returncode == 0, res.stderr
    assert f["valid"] == "1" and f["batch"] == str(b) and f["rows"] == str(r)
    assert f["mode"] == mode and f["copies"] == ("1" if copy == "copy" else "0")


@pytest.mark.parametrize("inputs", ["deterministic", "random=1"])
def test_sheet_shape_auto(inputs):
    res, f = run(["graph", "auto", "1024", "16384", "8192", "1", "20", "nocopy", "coalesced", inputs])
    assert res.returncode == 0, res.stderr
    assert f["valid"] == "1"
    assert float(f["min_bytes_per_iter"]) == 805470208.0
    assert 20 <= int(f["launches"]) <= 5000


@pytest.mark.parametrize("layout", ["fused", "streams"])
@pytest.mark.parametrize("mode", ["graph", "direct"])
def test_copy_mode_split_equals_nocopy(O, tmp_path, layout, mode):
    """Copy mode (the last repeat's outputs copied to the host inside every
    iteration; the fused layout splits that repeat into an rmsnorm launch
    and a softmax + GEMV launch on a second stream) dumps bitwise the
    outputs of nocopy mode, and reports the reference's launch count."""
    b, s, r, repeats = 64, 1000, 300, 3
    out = {}
    for copy in ("copy", "nocopy"):
        path = str(tmp_path / f"{copy}.bin")
        res, f = run([mode, "4", str(b), str(s), str(r), str(repeats), "1", copy, "random=6",
                      layout, f"--dump={path}"])
        assert res.returncode == 0, res.stderr
        assert f["valid"] == "1" and f["layout"] == layout
        want = (repeats + (copy == "copy")) if layout == "fused" else 3 * repeats
        assert int(f["kernels_per_iter"]) == want
        out[copy] = O.read_l2cdump1(path)
    for key in ("normalized", "softmax", "product"):
        assert np.array_equal(out["copy"][key].view(np.uint32), out["nocopy"][key].view(np.uint32))


def test_dump_matches_oracle(O, tmp_path):
    """--dump writes L2CDUMP1 whose outputs pass the oracle and whose
    per-row tolerance and double reference equal the oracle's."""
    path = str(tmp_path / "d.bin")
    b, s, r = 33, 1001, 77
    res, f = run(["direct", "2", str(b), str(s), str(r), "1", "1", "nocopy", "random=3",
                  f"--dump={path}"])
    assert res.returncode == 0, res.stderr
    d = O.read_l2cdump1(path)
    assert (d["batch"], d["size"], d["rows"], d["random"], d["seed"]) == (b, s, r, 1, 3)
    x, p, w, m = O.llama2c_inputs(1, 3, b, s, r)
    valid, tol, ref = O.validate_llama2c(1, x, p, w, m, d["normalized"], d["softmax"], d["product"])
    assert valid
    assert np.allclose(d["product_tolerance"], tol, rtol=1e-6, atol=0)
    assert np.allclose(d["product_reference"], ref, rtol=1e-12, atol=1e-300)


def test_dump_from_environment(O, tmp_path):
    path = str(tmp_path / "env.bin")
    env = dict(os.environ, LLAMA2C_DUMP=path)
    res, _ = run(["direct", "2", "8", "64", "16", "1", "1", "deterministic"], env=env)
    assert res.returncode == 0, res.stderr
    d = O.read_l2cdump1(path)
    x, p, w, m = O.llama2c_inputs(0, 0, 8, 64, 16)
    assert np.array_equal(d["product"], x.ravel()[np.arange(16) % 64])


TRIO_PRECS = ["fp32", "tf32", "bf16", "fp8", "mxfp6", "nvfp4"]


@pytest.mark.parametrize("prec", TRIO_PRECS)
def test_trio_mode_dump(ce, O, dev, tmp_path, prec):
    """trio=PREC runs the op trio through the plan, passes its own check and
    dumps L2CDUMP2: rows against the oracle, the carried double reference
    equal to the oracle's GEMM of the operands rebuilt from the standalone
    quantizers, out within the carried tolerance."""
    import torch
    from test_gpu_plan import _reconstruct

    b, s, r, seed = 70, 256, 96, 4
    path = str(tmp_path / "t.bin")
    res, f = run(["direct", "3", str(b), str(s), str(r), "1", "1", "nocopy", f"random={seed}",
                  f"trio={prec}", f"--dump={path}"])
    assert res.returncode == 0, res.stderr
    assert f["valid"] == "1" and f["layout"] == "trio" and f["precision"] == prec
    assert int(f["checked_rows"]) == 64 and float(f["out_rel_l2"]) <= 1e-2
    d = O.read_l2cdump2(path)
    pval = {"fp32": 0, "tf32": 1, "bf16": 2, "fp8": 3, "mxfp6": 4, "nvfp4": 5}[prec]
    assert (d["batch"], d["size"], d["rows"], d["inputs"], d["seed"], d["precision"]) == \
        (b, s, r, 2, seed, pval)
    x, w, logits, W = O.trio_inputs(seed, b, s, r)
    en = O.rmsnorm_ref(x, w)
    assert np.all(np.abs(d["normalized"] - en) <= 1e-5 * np.abs(en) + 1e-30)
    es = O.softmax_ref(logits)
    assert np.all(np.abs(d["softmax"] - es) <= 1e-5 * es + 1e-12)
    rows = d["checked_rows"]
    assert np.array_equal(rows, (np.arange(64) * b) // 64)
    a = _reconstruct(ce, O, dev, prec, torch.from_numpy(d["normalized"]).to(dev))
    wq = _reconstruct(ce, O, dev, prec, torch.from_numpy(W).to(dev))
    ref, mag = O.gemm_ref(a[rows], wq)
    assert np.allclose(d["out_reference"], ref, rtol=1e-12, atol=1e-300)
    err = np.abs(d["out"][rows].astype(np.float64) - d["out_reference"])
    assert np.all(err <= d["out_tolerance"])


def test_trio_graph_direct_copy_dumps_compare(tmp_path):
    """graph / direct and copy / nocopy runs of the trio give bitwise the same
    outputs; the package's compare_dumps passes them (exit 0) and fails a
    different precision's dump (header mismatch, exit 1)."""
    b, s, r = 64, 1024, 512
    paths = []
    for mode, copy in (("graph", "copy"), ("direct", "nocopy"), ("graph", "nocopy")):
        p = str(tmp_path / f"{mode}_{copy}.bin")
        res, f = run([mode, "5", str(b), str(s), str(r), "2", "1", copy, "random=9", "trio=bf16",
                      f"--dump={p}"])
        assert res.returncode == 0, res.stderr
        assert f["valid"] == "1" and f["copies"] == ("1" if copy == "copy" else "0")
        paths.append(p)
    cmp = [sys.executable, os.path.join(ROOT, "cuda-elastic_b200", "compare_dumps.py")]
    r1 = subprocess.run(cmp + paths, capture_output=True, text=True, timeout=120)
    assert r1.returncode == 0, r1.stdout + r1.stderr
    assert r1.stdout.count("PASS (bitwise identical)") == 2
    p8 = str(tmp_path / "fp8.bin")
    res, _ = run(["direct", "2", str(b), str(s), str(r), "1", "1", "nocopy", "random=9", "trio=fp8",
                  f"--dump={p8}"])
    assert res.returncode == 0, res.stderr
    r2 = subprocess.run(cmp + [paths[0], p8], capture_output=True, text=True, timeout=120)
    assert r2.returncode == 1
