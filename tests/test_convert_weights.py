"""The offline weight tools (cuda-elastic_b200/convert_weights.py) on the
CPU: the llama2.c checkpoint reader against its writer (shared and separate
classifier), the library's global row order of the fused matrices, and the
NVFP4 weight file's writer / reader."""
import importlib.util
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def cw():
    spec = importlib.util.spec_from_file_location(
        "ce_convert_weights", os.path.join(ROOT, "cuda-elastic_b200", "convert_weights.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


CFG = dict(dim=64, hidden_dim=96, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=50, seq_len=16)


def random_tensors(cfg, seed=0):
    rng = np.random.default_rng(seed)
    D, H, L, V = cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["vocab_size"]
    kvd = D // cfg["n_heads"] * cfg["n_kv_heads"]
    shapes = dict(tok_emb=(V, D), rms_att=(L, D), wq=(L, D, D), wk=(L, kvd, D), wv=(L, kvd, D), wo=(L, D, D),
                  rms_ffn=(L, D), w1=(L, H, D), w2=(L, D, H), w3=(L, H, D), rms_final=(D,), wcls=(V, D))
    return {k: rng.standard_normal(s).astype(np.float32) for k, s in shapes.items()}


@pytest.mark.parametrize("shared", [True, False])
def test_llama2c_round_trip(cw, tmp_path, shared):
    t = random_tensors(CFG)
    if shared:
        t["wcls"] = t["tok_emb"]
    path = str(tmp_path / "m.bin")
    cw.write_llama2c(path, CFG, t, shared=shared)
    cfg, r, sh = cw.read_llama2c(path)
    assert cfg == CFG and sh == shared
    for k in t:
        assert np.array_equal(np.asarray(r[k]), t[k]), k
    hs = CFG["dim"] // CFG["n_heads"]
    assert r["rope_real"].shape == (CFG["seq_len"], hs // 2)


def test_llama2c_errors(cw, tmp_path):
    t = random_tensors(CFG)
    path = str(tmp_path / "m.bin")
    cw.write_llama2c(path, CFG, t, shared=False)
    raw = open(path, "rb").read()
    short = str(tmp_path / "short.bin")
    open(short, "wb").write(raw[:-8])
    with pytest.raises(ValueError, match="truncated"):
        cw.read_llama2c(short)
    long = str(tmp_path / "long.bin")
    open(long, "wb").write(raw + bytes(8))
    with pytest.raises(ValueError, match="trailing"):
        cw.read_llama2c(long)


def test_model_row_order(cw):
    t = random_tensors(CFG)
    kvd = CFG["dim"] // CFG["n_heads"] * CFG["n_kv_heads"]
    qkv = cw.model_matrix(t, "wqkv", 1)
    assert np.array_equal(qkv[:64], t["wq"][1]) and np.array_equal(qkv[64:64 + kvd], t["wk"][1])
    assert np.array_equal(qkv[64 + kvd:], t["wv"][1])
    w13 = cw.model_matrix(t, "w13", 0)
    assert np.array_equal(w13[0::2], t["w1"][0]) and np.array_equal(w13[1::2], t["w3"][0])
    assert [m[:2] for m in cw.matrix_shapes(CFG)][:5] == [("wqkv", 0), ("wo", 0), ("w13", 0), ("w2", 0),
                                                         ("wqkv", 1)]


def test_nvfp4_file_round_trip(cw, tmp_path):
    rng = np.random.default_rng(2)
    D, L, V = CFG["dim"], CFG["n_layers"], CFG["vocab_size"]
    emb = rng.integers(0, 65535, (V, D), dtype=np.uint16)
    norms = (rng.random((L, D), np.float32), rng.random((L, D), np.float32), rng.random(D, np.float32))
    mats = []
    for _, _, rows, cols in cw.matrix_shapes(CFG):
        mats.append((rng.random(2, np.float32), rng.integers(0, 255, (rows, cols // 2), dtype=np.uint8),
                     rng.integers(0, 127, (rows, cols // 16), dtype=np.uint8)))
    path = str(tmp_path / "w.nvfp4")
    cw.write_nvfp4_file(path, CFG, emb, norms, mats)
    cfg, e, n, m = cw.read_nvfp4_file(path)
    assert cfg == CFG and np.array_equal(e, emb)
    for a, b in zip(n, norms):
        assert np.array_equal(a, b)
    for (name, layer, alpha, codes, scales), (a2, c2, s2), shape in zip(m, mats, cw.matrix_shapes(CFG)):
        assert (name, layer) == shape[:2]
        assert np.array_equal(alpha, a2) and np.array_equal(codes, c2) and np.array_equal(scales, s2)
    open(path, "ab").write(b"x")
    with pytest.raises(ValueError, match="trailing"):
        cw.read_nvfp4_file(path)
