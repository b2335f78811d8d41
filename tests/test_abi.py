"""The C ABI library loads, exports every symbol include/ce_b200.h declares,
its host-side generators match the oracle bit for bit, and argument errors
come back as CE_ERR_USAGE before any device work. No GPU needed."""
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(ce_\w+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(ce):
    L = ce.lib()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert ce.lib().ce_version().decode().startswith("ce_b200")


@pytest.mark.parametrize("random,seed", [(0, 0), (1, 1), (1, 99)])
def test_llama2c_generator_matches_oracle(ce, O, random, seed):
    shape = (7, 130, 33)
    got = ce.fill_llama2c_host(random, seed, *shape)
    want = O.llama2c_inputs(random, seed, *shape)
    for g, w in zip(got, want):
        assert np.array_equal(g, w)


def test_llama2c_generator_large_is_parallel_and_exact(ce, O):
    # big enough to take the multithreaded path of the library
    got = ce.fill_llama2c_host(1, 3, 64, 4096, 4)
    want = O.llama2c_inputs(1, 3, 64, 4096, 4)
    for g, w in zip(got, want):
        assert np.array_equal(g, w)


@pytest.mark.parametrize("first,count", [(0, 1), (0, 1001), (1, 1000), (12345, 70001)])
def test_normal_and_uniform_generators_match_oracle(ce, O, first, count):
    full = O.normals(5, 2, first + count, 0.125)
    assert np.array_equal(ce.fill_normal_host(5, 2, count, 0.125, first=first), full[first:])
    fu = O.uniforms(5, 4, first + count, 0.5, 1.5)
    assert np.array_equal(ce.fill_uniform_host(5, 4, count, 0.5, 1.5, first=first), fu[first:])


def test_trio_inputs_match_oracle(ce, O):
    for a, b in zip(ce.trio_inputs_host(0, 8, 288, 768), O.trio_inputs(0, 8, 288, 768)):
        assert np.array_equal(a, b)


def test_usage_errors_before_device_work(ce):
    L = ce.lib()
    assert L.ce_rmsnorm(None, None, None, 0, 16, 1e-5, None) == ce.ERR_USAGE
    code, msg = ce.last_error()
    assert code == ce.ERR_USAGE and "rows" in msg
    assert L.ce_softmax(None, None, 4, 0, None) == ce.ERR_USAGE
    assert L.ce_gemv(None, None, None, -1, 4, None) == ce.ERR_USAGE
    h = __import__("ctypes").c_void_p()
    assert L.ce_plan_create(__import__("ctypes").byref(h), 8, 288, 768, 9) == ce.ERR_USAGE
    assert L.ce_plan_create(__import__("ctypes").byref(h), 0, 288, 768, 2) == ce.ERR_USAGE
    assert L.ce_fill_llama2c_host(1, 1, 0, 4, 4, None, None, None, None) == ce.ERR_USAGE
    assert L.ce_llama2c_rows(None, None, None, None, None, None, None, 16, 0, 0, 0, 1e-5,
                             None) == ce.ERR_USAGE
    assert "no rows" in ce.last_error()[1]
    assert L.ce_llama2c_rows(None, None, None, None, None, None, None, 16, 4, 0, 0, 1e-5,
                             None) == ce.ERR_USAGE
    assert "rmsnorm needs" in ce.last_error()[1]
    with pytest.raises(ce.CeError) as e:
        ce.check(L.ce_rmsnorm(None, None, None, 1, 0, 1e-5, None))
    assert e.value.status == ce.ERR_USAGE


# The reference's invalid-dimension cases (decoder/tests/run_tests.sh:52-62):
# rejected with CE_ERR_USAGE (its exit code 2) and the same message, before
# any device work.
@pytest.mark.parametrize("dims,pattern", [
    ((1024, 8, 1, 4), "vocab must satisfy"),
    ((1024, 16, 17, 4), "vocab must satisfy"),
    ((1024, 32, 8, 1), "steps must be"),
    ((0, 16384, 8192, 4), "batch must be"),
    ((1024, 0, 8192, 4), "width must be"),
    ((1, 16777201, 2, 2), "width must be"),
    ((1048576, 16384, 8192, 4), "GiB"),
    ((1024, 16384, 8192, 1025), "steps must be"),
])
def test_decoder_invalid_dimensions(ce, dims, pattern):
    import ctypes
    h = ctypes.c_void_p()
    rc = ce.lib().ce_decoder_create(ctypes.byref(h), *dims, ce.PREC_FP32, None)
    assert rc == ce.ERR_USAGE
    assert pattern in ce.last_error()[1]
    assert not h.value


def _llama2c_exe():
    return os.path.join(ROOT, "cuda-elastic_b200", "llama2c_b200")


@pytest.mark.parametrize("args,pattern", [(["bogus"], "Usage:"), (["0"], "Usage:"),
                                          (["1", "2", "3", "4", "5", "6", "7"], "Usage:"),
                                          (["random=x1"], "bad seed")])
def test_llama2c_cli_usage_errors(args, pattern):
    """Command-line errors exit with EXIT_FAILURE before any device work, with
    the reference's messages (llama2c_cuda_graph.cu:195-258)."""
    import subprocess
    r = subprocess.run([_llama2c_exe()] + args, capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    assert pattern in r.stderr
