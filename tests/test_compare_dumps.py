"""The dump comparison tool (cuda-elastic_b200/compare_dumps.py): on dumps
written by the reference's own writer it gives the reference
compare_dumps.py's exit status and tolerance ratios (tests/golden/compare.npz,
made by tests/golden/make_compare_golden.py), and it applies the same rules
to the op-trio dump L2CDUMP2."""
import contextlib
import importlib.util
import io
import os
import struct

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = np.load(os.path.join(ROOT, "tests", "golden", "compare.npz"))


@pytest.fixture(scope="module")
def tool():
    path = os.path.join(ROOT, "cuda-elastic_b200", "compare_dumps.py")
    spec = importlib.util.spec_from_file_location("ce_compare_dumps", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _run(tool, *paths):
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf), contextlib.redirect_stderr(io.StringIO()):
        status = tool.main(["compare_dumps.py", *paths])
    return status, buf.getvalue()


def _write(tmp_path, name, data):
    path = str(tmp_path / name)
    with open(path, "wb") as f:
        f.write(bytes(data))
    return path


@pytest.mark.parametrize("name", [str(n) for n in GOLDEN["names"]])
def test_reference_verdicts(tool, tmp_path, name):
    base = _write(tmp_path, "base.bin", GOLDEN["base"])
    other = _write(tmp_path, name + ".bin", GOLDEN[f"dump_{name}"])
    status, text = _run(tool, base, other)
    assert status == int(GOLDEN[f"status_{name}"]), text
    if f"ratios_{name}" in GOLDEN.files:
        _, ref = tool.load(base)
        _, oth = tool.load(other)
        stats = tool.compare(ref, oth)
        got = np.array([stats[k][0] for k in ("normalized", "softmax", "product")])
        exp = GOLDEN[f"ratios_{name}"]
        assert np.array_equal(np.isinf(got), np.isinf(exp))
        fin = np.isfinite(exp)
        assert np.allclose(got[fin], exp[fin], rtol=1e-12, atol=0)
    if name == "identical":
        assert "bitwise identical" in text


def test_reader_matches_oracle(tool, O, tmp_path):
    base = _write(tmp_path, "base.bin", GOLDEN["base"])
    h, sec = tool.load(base)
    d = O.read_l2cdump1(base)
    assert (h["batch"], h["size"], h["rows"], h["inputs"], h["seed"]) == \
        (d["batch"], d["size"], d["rows"], d["random"], d["seed"])
    for k in ("normalized", "softmax", "product", "product_tolerance", "product_reference"):
        assert np.array_equal(sec[k].ravel(), d[k].ravel())


def test_usage_and_unreadable(tool, tmp_path):
    assert _run(tool, "only_one.bin")[0] == 2
    base = _write(tmp_path, "base.bin", GOLDEN["base"])
    assert _run(tool, base, _write(tmp_path, "short.bin", GOLDEN["base"][:-5]))[0] == 1
    assert _run(tool, base, _write(tmp_path, "junk.bin", b"NOTADUMP" + bytes(40)))[0] == 1
    assert _run(tool, base, str(tmp_path / "missing.bin"))[0] == 1


def _v2(b, s, r, checked, norm, soft, out, tol, ref, seed=3, precision=2):
    head = b"L2CDUMP2" + struct.pack("<4iQ2i", b, s, r, 2, seed, precision, len(checked))
    return (head + norm.astype("<f4").tobytes() + soft.astype("<f4").tobytes() +
            out.astype("<f4").tobytes() + np.asarray(checked, "<i4").tobytes() +
            tol.astype("<f4").tobytes() + ref.astype("<f8").tobytes())


@pytest.fixture()
def v2case():
    rng = np.random.default_rng(5)
    b, s, r = 6, 32, 20
    norm = rng.standard_normal((b, s)).astype(np.float32)
    soft = rng.random((b, s)).astype(np.float32)
    soft /= soft.sum(axis=1, keepdims=True)
    ref = rng.standard_normal((b, r))
    out = ref.astype(np.float32)
    checked = [0, 2, 4]
    tol = np.full((3, r), 1e-3, np.float32)
    return b, s, r, checked, norm, soft, out, tol, ref[checked]


def test_v2_round_trip_and_oracle_reader(tool, O, tmp_path, v2case):
    b, s, r, checked, norm, soft, out, tol, ref = v2case
    path = _write(tmp_path, "a.bin", _v2(*v2case))
    h, sec = tool.load(path)
    assert h == dict(version=2, batch=b, size=s, rows=r, inputs=2, seed=3, precision=2, checked=3)
    d = O.read_l2cdump2(path)
    assert np.array_equal(sec["out"], d["out"]) and np.array_equal(sec["checked_rows"], d["checked_rows"])
    assert np.array_equal(d["out_reference"], ref) and d["precision"] == 2
    ratio, _ = tool.own_error(sec)
    assert ratio < 1e-3


def test_v2_rules(tool, tmp_path, v2case):
    b, s, r, checked, norm, soft, out, tol, ref = v2case
    base = _write(tmp_path, "base.bin", _v2(*v2case))

    def status(**change):
        o = out.copy()
        n = norm.copy()
        for (row, col), delta in change.get("out", {}).items():
            o[row, col] += delta
        for (row, col), delta in change.get("norm", {}).items():
            n[row, col] += delta
        other = _write(tmp_path, "o.bin", _v2(b, s, r, checked, n, soft, o, tol, ref,
                                               seed=change.get("seed", 3),
                                               precision=change.get("precision", 2)))
        return _run(tool, base, other)[0]

    assert status() == 0
    assert status(out={(2, 5): 5e-4}) == 0          # checked row, inside its tolerance
    assert status(out={(2, 5): 2e-3}) == 1          # checked row, outside
    assert status(out={(1, 5): 2e-3}) == 0          # unchecked row: only relative L2 applies
    assert status(out={(1, 5): 10.0}) == 1          # relative L2 over all of out > 1e-2
    assert status(out={(1, 5): np.nan}) == 1
    assert status(norm={(0, 0): 4e-4}) == 1
    assert status(seed=4) == 1                      # header mismatch
    assert status(precision=5) == 1
    # the reference dump's own error does not fail the comparison; an OTHER's does
    bad = _write(tmp_path, "bad.bin", _v2(b, s, r, checked, norm, soft, out, tol, ref + 1.0))
    assert _run(tool, bad, base)[0] == 0
    assert _run(tool, base, bad)[0] == 1
