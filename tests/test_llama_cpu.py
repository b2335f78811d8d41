"""CPU side of the Llama-2 decoder step: the C ABI's shape checks (no CUDA
call), and the float64 oracle (oracle/llama_ref.py) cross-checked against a
second, loop-by-loop restatement of one decode step on a tiny model, with
grouped-query heads, a non-zero position and a partly filled cache."""
import ctypes
import math

import numpy as np
import pytest

from oracle import llama_ref
from oracle.oracle import bf16_bits


@pytest.mark.parametrize("change,pattern", [
    (dict(dim=100), "dim must be a multiple of 8"),
    (dict(hidden_dim=12), "hidden_dim must be a positive multiple of 8"),
    (dict(n_heads=5), "n_heads must divide dim"),
    (dict(n_kv_heads=5), "n_kv_heads must divide n_heads"),
    (dict(n_heads=4), "head size dim / n_heads must be 64 or 128"),
    (dict(vocab_size=1001), "vocab_size must be a multiple of 4"),
    (dict(seq_len=0), "seq_len must be in"),
    (dict(seq_len=1 << 20, n_layers=64), "GiB of device memory per GPU"),
])
def test_validate_rejects_bad_shapes(ce, change, pattern):
    cfg = dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, vocab_size=32000, seq_len=1024)
    cfg.update(change)
    c = ce.llama_config(**cfg)
    rc = ce.lib().ce_llama_validate(ctypes.byref(c), 256, 64, ce.PREC_BF16)
    assert rc == ce.ERR_USAGE
    assert pattern in ce.last_error()[1]


def test_validate_accepts_the_baseline_shapes(ce):
    for cfg, batch in ((dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, vocab_size=32000,
                             seq_len=1024), 256),
                       (dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, vocab_size=32000,
                             seq_len=2048), 32)):
        c = ce.llama_config(**cfg)
        assert ce.lib().ce_llama_validate(ctypes.byref(c), batch, 64, ce.PREC_BF16) == ce.OK, ce.last_error()


def test_rope_known_answer():
    hs = 8
    v = np.zeros(hs)
    v[0] = 1.0  # pair 0 has frequency 1: rotation by pos radians
    out = llama_ref.rope(v, 3, hs)
    assert np.allclose(out[:2], [math.cos(3), math.sin(3)])
    w = np.arange(2 * hs, dtype=np.float64)
    r = llama_ref.rope(w, 17, hs).reshape(-1, 2)
    assert np.allclose((r * r).sum(1), (w.reshape(-1, 2) ** 2).sum(1))  # rotations keep pair norms
    assert np.array_equal(llama_ref.rope(w, 0, hs), w)


def _loop_step(c, W, tok, pos, kc, vc):
    """One token of one sequence, written as plain loops."""
    D, Hd, H, KH, L = c["dim"], c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"]
    hs = D // H
    kvd = hs * KH
    rnd = llama_ref.bf16_round
    emb = llama_ref.to64(W["tok_emb"])

    def norm(x, w):
        ss = sum(t * t for t in x) / len(x)
        return [w[i] * (x[i] / math.sqrt(ss + 1e-5)) for i in range(len(x))]

    def matvec(m, x):
        return [sum(m[r][j] * x[j] for j in range(len(x))) for r in range(len(m))]

    x = list(emb[tok])
    for l in range(L):
        xb = list(rnd(norm(x, W["rms_att"][l])))
        qkv = matvec(llama_ref.to64(W["wqkv"][l]), xb)
        q, k, v = qkv[:D], qkv[D:D + kvd], qkv[D + kvd:]
        for vec in (q, k):
            for i in range(0, len(vec), 2):
                j = i % hs
                a = pos * 10000.0 ** (-j / hs)
                e, o = vec[i], vec[i + 1]
                vec[i], vec[i + 1] = e * math.cos(a) - o * math.sin(a), e * math.sin(a) + o * math.cos(a)
        for kh in range(KH):
            kc[l][kh][pos] = rnd(k[kh * hs:(kh + 1) * hs])
            vc[l][kh][pos] = rnd(v[kh * hs:(kh + 1) * hs])
        att = []
        for h in range(H):
            kh = h // (H // KH)
            qh = q[h * hs:(h + 1) * hs]
            s = [sum(qh[d] * kc[l][kh][t][d] for d in range(hs)) / math.sqrt(hs) for t in range(pos + 1)]
            mx = max(s)
            e = [math.exp(t - mx) for t in s]
            tot = sum(e)
            att += [sum(e[t] / tot * vc[l][kh][t][d] for t in range(pos + 1)) for d in range(hs)]
        o = matvec(llama_ref.to64(W["wo"][l]), list(rnd(att)))
        x = [x[i] + o[i] for i in range(D)]
        xb = list(rnd(norm(x, W["rms_ffn"][l])))
        hh = matvec(llama_ref.to64(W["w13"][l]), xb)
        sw = [hh[2 * i] / (1 + math.exp(-hh[2 * i])) * hh[2 * i + 1] for i in range(Hd)]
        o = matvec(llama_ref.to64(W["w2"][l]), list(rnd(sw)))
        x = [x[i] + o[i] for i in range(D)]
    return matvec(llama_ref.to64(W["wcls"]), list(rnd(norm(x, W["rms_final"]))))


def test_oracle_matches_loop_restatement():
    c = dict(dim=16, hidden_dim=24, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=20, seq_len=6)
    hs = c["dim"] // c["n_heads"]
    kvd = hs * c["n_kv_heads"]
    rng = np.random.default_rng(5)

    def mat(r, k):
        return bf16_bits((rng.standard_normal((r, k)) * 0.3).astype(np.float32))

    W = {"tok_emb": mat(c["vocab_size"], c["dim"]), "wcls": mat(c["vocab_size"], c["dim"]),
         "rms_final": (1 + 0.1 * rng.standard_normal(c["dim"])).astype(np.float32),
         "wqkv": [mat(c["dim"] + 2 * kvd, c["dim"]) for _ in range(2)],
         "wo": [mat(c["dim"], c["dim"]) for _ in range(2)],
         "w13": [mat(2 * c["hidden_dim"], c["dim"]) for _ in range(2)],
         "w2": [mat(c["dim"], c["hidden_dim"]) for _ in range(2)],
         "rms_att": [(1 + 0.1 * rng.standard_normal(c["dim"])).astype(np.float32) for _ in range(2)],
         "rms_ffn": [(1 + 0.1 * rng.standard_normal(c["dim"])).astype(np.float32) for _ in range(2)]}
    pos = 3
    cache = llama_ref.bf16_round(rng.standard_normal((2, 2, c["n_kv_heads"], c["seq_len"], hs)))
    cache[:, :, :, pos:, :] = 0.0
    orc = llama_ref.LlamaOracle(c, W)
    kc = [cache[0, l][None].copy() for l in range(2)]
    vc = [cache[1, l][None].copy() for l in range(2)]
    got = orc.step(np.array([7]), pos, kc, vc)[0]
    kl = [[list(map(list, cache[0, l, kh])) for kh in range(c["n_kv_heads"])] for l in range(2)]
    vl = [[list(map(list, cache[1, l, kh])) for kh in range(c["n_kv_heads"])] for l in range(2)]
    want = np.array(_loop_step(c, W, 7, pos, kl, vl))
    assert np.allclose(got, want, rtol=1e-9, atol=1e-9)
    assert np.allclose(kc[1][0], np.array(kl[1]), rtol=0, atol=0)  # appended keys agree


def test_layerwise_oracle_matches_step_oracle():
    """The layer-major teacher-forced oracle (every (sequence, step) row of a
    layer at once) gives the step-major LlamaOracle.decode logits: 3
    sequences x 4 steps, grouped-query heads, a partly filled cache, bf16
    and fp16 operand rounding."""
    c = dict(dim=32, hidden_dim=48, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=40, seq_len=12)
    hs = c["dim"] // c["n_heads"]
    kvd = hs * c["n_kv_heads"]
    rng = np.random.default_rng(9)

    def mat(r, k):
        return bf16_bits((rng.standard_normal((r, k)) * 0.3).astype(np.float32))

    W = {"tok_emb": mat(c["vocab_size"], c["dim"]), "wcls": mat(c["vocab_size"], c["dim"]),
         "rms_final": (1 + 0.1 * rng.standard_normal(c["dim"])).astype(np.float32),
         "wqkv": [mat(c["dim"] + 2 * kvd, c["dim"]) for _ in range(2)],
         "wo": [mat(c["dim"], c["dim"]) for _ in range(2)],
         "w13": [mat(2 * c["hidden_dim"], c["dim"]) for _ in range(2)],
         "w2": [mat(c["dim"], c["hidden_dim"]) for _ in range(2)],
         "rms_att": [(1 + 0.1 * rng.standard_normal(c["dim"])).astype(np.float32) for _ in range(2)],
         "rms_ffn": [(1 + 0.1 * rng.standard_normal(c["dim"])).astype(np.float32) for _ in range(2)]}
    n, S, pos0 = 3, 4, 5
    cache = llama_ref.bf16_round(rng.standard_normal((2, 2, n, c["n_kv_heads"], c["seq_len"], hs)))
    cache[..., pos0:, :] = 0.0
    tokens0 = np.array([3, 17, 39])
    forced = rng.integers(0, c["vocab_size"], (n, S))
    for operand in ("bf16", "f16"):
        orc = llama_ref.LlamaOracle(c, W, operand=operand)
        kc = [cache[0, l].copy() for l in range(2)]
        vc = [cache[1, l].copy() for l in range(2)]
        want, _, _ = orc.decode(tokens0, pos0, forced, kc, vc)
        tokens_in = np.concatenate([tokens0[:, None], forced[:, :S - 1]], axis=1)
        kc2 = [cache[0, l].copy() for l in range(2)]
        vc2 = [cache[1, l].copy() for l in range(2)]
        lw = lambda l: {"wqkv": orc.wqkv[l], "wo": orc.wo[l], "w13": orc.w13[l], "w2": orc.w2[l],
                        "rms_att": orc.rms_att[l], "rms_ffn": orc.rms_ffn[l]}
        got = llama_ref.teacher_forced_layerwise(c, lw, orc.emb, orc.rms_final, orc.wcls, tokens_in, pos0,
                                                 lambda l: (kc2[l], vc2[l]), operand=operand)
        assert got.shape == want.shape
        assert np.allclose(got, want, rtol=1e-9, atol=1e-9), np.abs(got - want).max()
        for l in range(2):  # the appended keys and values agree
            assert np.array_equal(kc[l], kc2[l]) and np.array_equal(vc[l], vc2[l])


@pytest.mark.parametrize("cfg,world", [
    (dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, vocab_size=32000, seq_len=2048), 8),
    (dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, vocab_size=32000, seq_len=2048), 2),
    (dict(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4, vocab_size=1024, seq_len=64), 4),
])
def test_shard_rows_partition_every_weight(ce, cfg, world):
    """Every rank's rows of every sharded weight, concatenated in rank order,
    are each global row exactly once; QKV rows are q, k, v of the rank's
    heads; the w1|w3 pairs stay whole."""
    c = ce.llama_config(**cfg)
    hs = c.dim // c.n_heads
    kvd = hs * c.n_kv_heads
    total = {ce.LLAMA_WQKV: c.dim + 2 * kvd, ce.LLAMA_WO: c.dim, ce.LLAMA_W13: 2 * c.hidden_dim,
             ce.LLAMA_W2: c.dim, ce.LLAMA_WCLS: c.vocab_size}
    for which, n in total.items():
        parts = [ce.llama_shard_rows(c, r, world, which) for r in range(world)]
        allr = np.concatenate(parts)
        assert sorted(allr.tolist()) == list(range(n))
        if which == ce.LLAMA_W13:
            assert all(len(p) % 2 == 0 and p[0] % 2 == 0 for p in parts)
    q = ce.llama_shard_rows(c, 1, world, ce.LLAMA_WQKV)
    lq, lkv = c.dim // world, kvd // world
    assert q[0] == lq and q[lq] == c.dim + lkv and q[lq + lkv] == c.dim + kvd + lkv


@pytest.mark.parametrize("change,world,pattern", [
    (dict(n_heads=4), 8, "heads"),
    (dict(hidden_dim=40), 2, "hidden_dim / world"),
    (dict(vocab_size=1004), 8, "vocab_size / world"),
])
def test_validate_shard_rejects_uneven_splits(ce, change, world, pattern):
    cfg = dict(dim=1024, hidden_dim=2048, n_layers=2, n_heads=8, vocab_size=32000, seq_len=64)
    cfg.update(change)
    c = ce.llama_config(**cfg)
    rc = ce.lib().ce_llama_validate_shard(ctypes.byref(c), 8, 4, ce.PREC_BF16, 0, world)
    assert rc == ce.ERR_USAGE
    assert pattern in ce.last_error()[1]


def test_shard_memory_is_per_rank(ce):
    """BASELINE config 5 at batch 512 (a 512 GiB KV cache) fits 8 ranks (their
    heads' share each) but not one GPU."""
    c = ce.llama_config(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, vocab_size=32000, seq_len=2048)
    assert ce.lib().ce_llama_validate_shard(ctypes.byref(c), 512, 32, ce.PREC_NVFP4_E2M1, 3, 8) == ce.OK, ce.last_error()
    assert ce.lib().ce_llama_validate_shard(ctypes.byref(c), 512, 32, ce.PREC_NVFP4_E2M1, 0, 1) == ce.ERR_USAGE
    assert "GiB of device memory per GPU" in ce.last_error()[1]
    assert ce.lib().ce_llama_validate_shard(ctypes.byref(c), 64, 32, ce.PREC_NVFP4_E2M1, 0, 1) == ce.OK


def test_sampler_restatement_properties():
    """The oracle sampler: a near-zero temperature gives the argmax, a tiny
    top-p gives the most probable token, the coin is reproducible, and the
    multinomial draw follows the probabilities."""
    rng = np.random.default_rng(11)
    lg = rng.standard_normal(300) * 2.0
    for step in range(5):
        u = llama_ref.sample_coin(7, step, 3)
        assert u == llama_ref.sample_coin(7, step, 3) and 0.0 <= u < 1.0
        assert llama_ref.sample_row(lg, 1e-3, 0.0, u)[0] == int(np.argmax(lg))
        assert llama_ref.sample_row(lg, 1.0, 1e-6, u)[0] == int(np.argmax(lg))
    small = np.log(np.array([0.5, 0.3, 0.2]))
    counts = np.zeros(3)
    for row in range(3000):
        counts[llama_ref.sample_row(small, 1.0, 0.0, llama_ref.sample_coin(1, 0, row))[0]] += 1
    assert np.allclose(counts / 3000, [0.5, 0.3, 0.2], atol=0.03)
    # top-p 0.7 keeps only the two most probable tokens of (0.5, 0.3, 0.2)
    kept = {llama_ref.sample_row(small, 1.0, 0.7, llama_ref.sample_coin(2, 0, row))[0] for row in range(500)}
    assert kept == {0, 1}
