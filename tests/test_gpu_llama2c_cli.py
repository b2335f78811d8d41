"""The llama2c drop-in executable (cuda-elastic_b200/llama2c_b200) on the
reference's own check matrix (llama2c/Makefile:44-56, check-sota: shapes
64x1000x300, 33x1001x77 and the sheet 1024x16384x8192; deterministic,
random=1, random=2; graph and direct; nocopy and copy), and its dump."""
import os
import subprocess

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
