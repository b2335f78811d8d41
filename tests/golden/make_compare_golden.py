"""Writes tests/golden/compare.npz: L2CDUMP1 dumps written by the REFERENCE's
own writer (write_dump, llama2c/llama2c_common.h:321-345, through
oracle/_ref/libref.so) and the verdicts of the REFERENCE's own
llama2c/compare_dumps.py on them, so the package's compare_dumps tool is
pinned to both without the reference tree. Run in a container that has it:

    make -C oracle && python tests/golden/make_compare_golden.py

Cases (one base dump from seeded random inputs, 6 x 40 x 24, and variants of
its outputs): identical; normalized off by 2e-4 (inside 3e-4) and 4e-4
(outside); softmax off by 0.5e-3 and 2e-3 relative; product off by 0.5 and
2 of its tolerance; a NaN product; another seed in the header. For each: the
reference's exit status of `compare_dumps.py base variant` and its
compare() ratios.
"""
import contextlib
import ctypes
import importlib.util
import io
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

# the reference tree's root, as oracle/Makefile's REF: $CE_REFERENCE, else a
# checkout named `reference` beside this repository
REF_TREE = os.environ.get("CE_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
REF_COMPARE = os.path.join(REF_TREE, "llama2c", "compare_dumps.py")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")


def main():
    R = O.ref()
    if R is None or not os.path.exists(REF_COMPARE):
        raise SystemExit("needs oracle/_ref/libref.so and the reference tree")
    R.ref_write_dump.restype = ctypes.c_int
    R.ref_write_dump.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p, _f32p, _f64p]
    spec = importlib.util.spec_from_file_location("ref_compare_dumps", REF_COMPARE)
    C = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(C)

    b, s, r, seed = 6, 40, 24, 7
    x, p, w, m = (np.empty(n, np.float32) for n in (b * s, b * s, s, r * s))
    R.ref_fill_inputs(1, seed, b, s, r, x, p, w, m)
    x2, p2 = x.reshape(b, s), p.reshape(b, s)
    norm = O.rmsnorm_ref(x2, w).astype(np.float32).ravel()
    soft = O.softmax_ref(p2).astype(np.float32).ravel()
    prod = (m.reshape(r, s).astype(np.float64) @ x[:s].astype(np.float64)).astype(np.float32)
    tol, refv = np.empty(r, np.float32), np.empty(r, np.float64)
    assert R.ref_validate_all(1, seed, x, p, w, m, norm, soft, prod, b, s, r, tol, refv) == 1

    def variant(name):
        n, sm, pr, sd = norm.copy(), soft.copy(), prod.copy(), seed
        if name == "norm_inside":
            n[5] += 2e-4
        elif name == "norm_outside":
            n[5] += 4e-4
        elif name == "softmax_inside":
            sm[17] *= 1 + 0.5e-3
        elif name == "softmax_outside":
            sm[17] *= 1 + 2e-3
        elif name == "product_inside":
            pr[3] += np.float32(0.5 * tol[3])
        elif name == "product_outside":
            pr[3] += np.float32(2.0 * tol[3])
        elif name == "product_nan":
            pr[3] = np.nan
        elif name == "other_seed":
            sd = seed + 1
        return n, sm, pr, sd

    names = ["identical", "norm_inside", "norm_outside", "softmax_inside", "softmax_outside",
             "product_inside", "product_outside", "product_nan", "other_seed"]
    out = {"names": np.array(names)}
    with tempfile.TemporaryDirectory() as tmp:
        base = os.path.join(tmp, "base.bin")
        assert R.ref_write_dump(base.encode(), 1, seed, b, s, r, norm, soft, prod, tol, refv) == 1
        out["base"] = np.frombuffer(open(base, "rb").read(), np.uint8)
        for name in names:
            n, sm, pr, sd = variant(name)
            path = os.path.join(tmp, name + ".bin")
            assert R.ref_write_dump(path.encode(), 1, sd, b, s, r, n, sm, pr, tol, refv) == 1
            out[f"dump_{name}"] = np.frombuffer(open(path, "rb").read(), np.uint8)
            with contextlib.redirect_stdout(io.StringIO()):
                out[f"status_{name}"] = np.array(C.main(["compare_dumps.py", base, path]))
            _, hr = C.load(base)
            ho, so = C.load(path)
            if ho == C.load(base)[0]:
                stats = C.compare(hr, so)
                out[f"ratios_{name}"] = np.array([stats[k][0] for k in ("normalized", "softmax", "product")])
    np.savez_compressed(os.path.join(HERE, "compare.npz"), **out)


if __name__ == "__main__":
    main()
