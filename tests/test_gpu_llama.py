"""The Llama-2 decoder step (ce_llama_*) against the float64 oracle
(oracle/llama_ref.py, teacher-forced with the device's own tokens): logits
within relative L2 tolerance at every step, greedy tokens equal wherever the
oracle's top-2 logits are not a near tie, on small configurations
(multi-head, grouped-query, head size 128, attention spanning several
position chunks) and on sampled sequences of the 110M-shaped configuration;
the greedy-token agreement counted over every sequence of the 110M-shaped
model (2048 tokens) and over the 32-layer 7B-shaped NVFP4 model (see
_agreement: the head stage >= 99.9%; the whole model against the ceiling an
fp32-exact implementation reaches on these random-init models). Also: a captured step graph replays bit for bit like direct
steps, and a step past the end of the KV cache reports an error instead of
writing out of bounds."""
import numpy as np
import pytest
import torch

from oracle.llama_ref import LlamaOracle, cache_from_device

pytestmark = pytest.mark.gpu

# bf16 operands, fp32 accumulation: observed relative L2 of the logits is
# ~1e-4; the north star's bound for a bf16 GEMM is 1e-2.
LOGIT_REL_L2 = 1e-2
NEAR_TIE = 2e-3  # top-2 logit gap below which a token difference is a tie


def run_and_check(ce, O, cfg, batch, kv_fill, steps, seqs=None, seed=1, precision=None):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    m = ce.Llama(cfg, batch, steps, precision=ce.PREC_BF16 if precision is None else precision)
    try:
        m.init_random(seed=seed, weight_std=0.02, kv_fill=kv_fill)
        rng = np.random.default_rng(seed)
        tokens0 = rng.integers(0, m.cfg.vocab_size, batch).astype(np.int32)
        m.start(tokens0, kv_fill)
        seqs = list(range(batch)) if seqs is None else seqs
        kc, vc = cache_from_device(m, seqs, kv_fill)
        orc = LlamaOracle(m.cfg.as_dict(), m.weights(),
                          operand="f16" if m.precision == ce.PREC_NVFP4_E2M1 else "bf16")
        dev_logits = []
        for _ in range(steps):
            m.step()
            torch.cuda.synchronize()
            dev_logits.append(m.logits()[seqs].astype(np.float64))
        ce.llama_status()
        gen = m.generated()[seqs]
        assert (gen >= 0).all() and (gen < m.cfg.vocab_size).all()
        lg, best, gap = orc.decode(tokens0[seqs], kv_fill, gen, kc, vc)
        for s in range(steps):
            assert O.rel_l2(dev_logits[s], lg[s]) <= LOGIT_REL_L2, (s, O.rel_l2(dev_logits[s], lg[s]))
        # A greedy token may differ from the oracle's only where the device's
        # own logit error on that row could account for it: the oracle logit
        # of the device's token is within twice the row's largest logit error
        # (and NEAR_TIE) of the oracle's maximum.
        for s in range(steps):
            for i in range(len(seqs)):
                if gen[i, s] == best[s, i]:
                    continue
                err = np.abs(dev_logits[s][i] - lg[s, i]).max()
                short = lg[s, i].max() - lg[s, i, gen[i, s]]
                assert short <= max(2 * err, NEAR_TIE), (
                    f"step {s} seq {seqs[i]}: device token {gen[i, s]} is {short:.3g} below the oracle "
                    f"maximum (token {best[s, i]}); largest logit error {err:.3g}")
        return m, gen, dev_logits
    finally:
        m.close()


@pytest.mark.parametrize("cfg,batch,kv_fill,steps", [
    (dict(dim=128, hidden_dim=256, n_layers=2, n_heads=2, vocab_size=512, seq_len=64), 5, 10, 6),
    (dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=1000, seq_len=48), 3, 0, 5),
    (dict(dim=256, hidden_dim=384, n_layers=3, n_heads=2, vocab_size=260, seq_len=40), 4, 7, 4),
    (dict(dim=128, hidden_dim=256, n_layers=1, n_heads=2, vocab_size=128, seq_len=640), 2, 300, 3),
    # K = 1024 over few output tiles: the w1|w3 GEMM runs split and SwiGLU runs as its own kernel
    (dict(dim=1024, hidden_dim=256, n_layers=1, n_heads=8, vocab_size=256, seq_len=32), 4, 5, 3),
    # 2 x hidden = 400: the SwiGLU epilogue's last tile is ragged
    (dict(dim=128, hidden_dim=200, n_layers=2, n_heads=2, vocab_size=64, seq_len=32), 3, 4, 3),
])
def test_small_configs_match_oracle(ce, O, cfg, batch, kv_fill, steps):
    run_and_check(ce, O, cfg, batch, kv_fill, steps)


@pytest.mark.parametrize("cfg,batch,kv_fill,steps", [
    (dict(dim=128, hidden_dim=256, n_layers=2, n_heads=2, vocab_size=512, seq_len=64), 5, 10, 5),
    (dict(dim=256, hidden_dim=320, n_layers=2, n_heads=2, n_kv_heads=1, vocab_size=1000, seq_len=48), 3, 7, 4),
    (dict(dim=1024, hidden_dim=256, n_layers=1, n_heads=8, vocab_size=256, seq_len=32), 4, 5, 3),
])
def test_nvfp4_weights_match_oracle(ce, O, cfg, batch, kv_fill, steps):
    """Every GEMM weight NVFP4 (the device quantizer's codes, scales and
    decode scale), expanded inside the W4A16 GEMM: against the oracle run on
    the dequantized weights."""
    run_and_check(ce, O, cfg, batch, kv_fill, steps, precision=ce.PREC_NVFP4_E2M1)


def test_7b_layer_shape_nvfp4(ce, O):
    """One layer at the 7B shape of BASELINE config 5 (dim 4096, 32 heads,
    SwiGLU 11008, vocab 32000, seq_len 2048) with NVFP4 weights, batch 64,
    the cache filled to position 1023: 3 steps, 2 sampled sequences."""
    cfg = dict(dim=4096, hidden_dim=11008, n_layers=1, n_heads=32, vocab_size=32000, seq_len=2048)
    run_and_check(ce, O, cfg, 64, 1024, 3, seqs=[5, 63], precision=ce.PREC_NVFP4_E2M1)


def test_graph_replay_equals_direct(ce):
    cfg = dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, vocab_size=1024, seq_len=64)
    outs = []
    for graph in (False, True):
        m = ce.Llama(cfg, 6, 8)
        try:
            m.init_random(seed=7, kv_fill=5)
            m.start(np.arange(6, dtype=np.int32) * 17, 5)
            if graph:
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    m.step(stream=s)  # first step direct (configures every kernel)
                torch.cuda.current_stream().wait_stream(s)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    m.step()
                for _ in range(7):
                    g.replay()
                torch.cuda.synchronize()
                del g
            else:
                for _ in range(8):
                    m.step()
                torch.cuda.synchronize()
            ce.llama_status()
            outs.append((m.generated().copy(), m.logits().copy(),
                         m.read(ce.LLAMA_POS, dtype=np.int32)[0]))
        finally:
            m.close()
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])
    assert outs[0][2] == outs[1][2] == 13


def test_programmatic_launch_changes_no_bits(ce):
    """Programmatic dependent launch only overlaps prologues: the same bits
    with it on and off, in direct steps and in a replayed graph."""
    cfg = dict(dim=512, hidden_dim=1024, n_layers=3, n_heads=8, n_kv_heads=4, vocab_size=2048, seq_len=300)
    outs = []
    for pdl in (False, True):
        m = ce.Llama(cfg, 40, 6)
        try:
            m.set_pdl(pdl)
            m.init_random(seed=11, kv_fill=200)
            m.start(np.arange(40, dtype=np.int32) * 31, 200)
            m.step()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                m.step()
            for _ in range(5):
                g.replay()
            torch.cuda.synchronize()
            del g
            ce.llama_status()
            outs.append((m.generated().copy(), m.logits().copy(), m.read(ce.LLAMA_RESIDUAL, dtype=np.float32)))
        finally:
            m.close()
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a, b)


def test_110m_shape_sampled_sequences(ce, O):
    """BASELINE config 4 shape (dim 768, 12 layers, 12 heads, SwiGLU 2048,
    vocab 32000, seq_len 1024), batch 256 with the cache filled to position
    511: 6 steps, 4 sampled sequences checked against the oracle."""
    cfg = dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, vocab_size=32000, seq_len=1024)
    run_and_check(ce, O, cfg, 256, 512, 6, seqs=[0, 77, 200, 255])


# fp32-level noise put on every matrix product of a second copy of the
# oracle's rows: how far such noise alone moves this random-init model
PERTURB_REL = 1e-7


def _agreement(ce, m, tokens0, kv_fill, steps, seqs, residuals):
    """Greedy-token agreement of a model that has just run `steps` device
    steps (`residuals[s]`: the device's residual stream after step s),
    counted over every (sequence, step) the way the reference's accuracy
    mode counts tokens (experiments/blackwell/lowprec/decoder_lowprec.cu:
    1285-1302):

    head  the head stage on the device's own hidden state -- final RMSNorm,
          16-bit operand, classifier, first maximum -- in float64, against
          the device's token (the stage the reference's loom_private decoder
          is: rmsnorm -> classifier -> argmax);
    full  the whole model teacher-forced with the device's tokens in float64
          (layer-major oracle, each layer's weights and cache read from the
          device once), against the device's token;
    ceiling the same oracle against a second copy of itself whose every
          matrix product carries PERTURB_REL relative noise: the agreement
          an exact-to-fp32 implementation can expect on this model, whose
          16-bit operand roundings amplify any fp32-level difference.
    Returns a dict of counts, the worst per-step logit relative L2 and the
    oracle logits."""
    from oracle import llama_ref
    c = m.cfg
    nv = m.precision == ce.PREC_NVFP4_E2M1
    op = llama_ref.f16_round if nv else llama_ref.bf16_round
    n = len(seqs)
    gen = m.generated()[seqs]
    tokens_in = np.concatenate([np.asarray(tokens0)[seqs][:, None], gen[:, :steps - 1]], axis=1)

    def mat(which, l=0):
        if nv:
            return llama_ref.to64(m.nvfp4_weight(which, l))
        return llama_ref.to64(m.read(which, l).reshape(m._shape(which)))

    def layer_weights(l):
        return {"wqkv": mat(ce.LLAMA_WQKV, l), "wo": mat(ce.LLAMA_WO, l), "w13": mat(ce.LLAMA_W13, l),
                "w2": mat(ce.LLAMA_W2, l),
                "rms_att": m.read(ce.LLAMA_RMS_ATT, l, np.float32).astype(np.float64),
                "rms_ffn": m.read(ce.LLAMA_RMS_FFN, l, np.float32).astype(np.float64)}

    span = kv_fill + steps
    all_seqs = n == m.batch

    def layer_cache(l):  # the sequences' cache twice: the clean and the noisy oracle copy
        out = []
        for which in (ce.LLAMA_KCACHE, ce.LLAMA_VCACHE):
            if all_seqs:  # one read of the layer's whole cache
                full = m.read(which, l).reshape(m.batch, c.n_kv_heads, c.seq_len, m.hs)[:, :, :span]
            else:
                full = np.stack([m.cache_rows(l, b, which, span) for b in seqs])
            v = llama_ref.to64(full.reshape(-1, m.hs)).reshape(n, c.n_kv_heads, span, m.hs)
            out.append(np.concatenate([v, v]))
        return out

    rng = np.random.default_rng(2024)

    def perturb(y):  # noise on the second copy's rows only
        y[n * steps:] *= 1.0 + PERTURB_REL * rng.standard_normal(y[n * steps:].shape)
        return y

    emb = llama_ref.to64(m.read(ce.LLAMA_TOK_EMB).reshape(c.vocab_size, c.dim))
    rms_final = m.read(ce.LLAMA_RMS_FINAL, dtype=np.float32).astype(np.float64)
    wcls = mat(ce.LLAMA_WCLS)
    lg2 = llama_ref.teacher_forced_layerwise(
        c.as_dict(), layer_weights, emb, rms_final, wcls, np.concatenate([tokens_in, tokens_in]), kv_fill,
        layer_cache, operand="f16" if nv else "bf16", perturb=perturb)
    lg, noisy = lg2[:, :n], lg2[:, n:]
    best, best_noisy = lg.argmax(axis=2), noisy.argmax(axis=2)  # first maxima, [steps][n]
    head = np.stack([(op(llama_ref.rmsnorm(residuals[s][seqs].astype(np.float64), rms_final)) @ wcls.T)
                     .argmax(axis=1) for s in range(steps)])
    top2 = np.sort(lg, axis=2)[:, :, -2:]
    gap = top2[:, :, 1] - top2[:, :, 0]
    band = np.abs(lg - noisy).max(axis=2)
    decisive = gap > 4 * band
    return {"total": n * steps, "head": int((head == gen[:, :steps].T).sum()),
            "full": int((best == gen[:, :steps].T).sum()), "ceiling": int((best == best_noisy).sum()),
            "decisive": int(decisive.sum()), "decisive_agree": int(((best == gen[:, :steps].T) & decisive).sum()),
            "noisy_rel_l2": max(float(np.linalg.norm(lg[s] - noisy[s]) / np.linalg.norm(lg[s]))
                                for s in range(steps))}, lg


def _run_device(ce, cfg, batch, kv_fill, steps, precision, seed=1):
    m = ce.Llama(cfg, batch, steps, precision=precision)
    m.init_random(seed=seed, weight_std=0.02, kv_fill=kv_fill)
    tokens0 = np.random.default_rng(seed).integers(0, m.cfg.vocab_size, batch).astype(np.int32)
    m.start(tokens0, kv_fill)
    logits, residuals = [], []
    for _ in range(steps):
        m.step()
        torch.cuda.synchronize()
        logits.append(m.logits().astype(np.float64))
        residuals.append(m.read(ce.LLAMA_RESIDUAL, dtype=np.float32).reshape(batch, m.cfg.dim))
    ce.llama_status()
    return m, tokens0, logits, residuals


def _check_agreement(ce, O, m, tokens0, kv_fill, steps, seqs, dev_logits, residuals):
    r, lg = _agreement(ce, m, tokens0, kv_fill, steps, seqs, residuals)
    worst = max(O.rel_l2(dev_logits[s][seqs], lg[s]) for s in range(steps))
    t = r["total"]
    print(f"greedy-token agreement over {t} tokens: head stage {r['head']}/{t}, full model "
          f"{r['full']}/{t} (ceiling: oracle vs itself with {PERTURB_REL:g} noise per product "
          f"{r['ceiling']}/{t}, its logits moved {r['noisy_rel_l2']:.3g}), decisive tokens "
          f"{r['decisive_agree']}/{r['decisive']}; worst device logit rel L2 {worst:.3g}")
    # the head stage on the device's own hidden state: the north star's bar
    assert r["head"] / t >= 0.999, r
    # the whole model: within the bf16 bound, and as close to the oracle as
    # fp32-level noise alone lets the oracle stay to itself (1.5 points of
    # slack for the count's statistics)
    assert worst <= LOGIT_REL_L2
    assert r["full"] / t >= r["ceiling"] / t - 0.015, r
    return r


def test_110m_token_agreement_all_sequences(ce, O):
    """BASELINE config 4 (110M shape, bf16, batch 256, cache to 511): all 256
    sequences x 8 greedy steps (2048 tokens)."""
    cfg = dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, vocab_size=32000, seq_len=1024)
    steps = 8
    m, tokens0, dev_logits, res = _run_device(ce, cfg, 256, 512, steps, ce.PREC_BF16)
    try:
        _check_agreement(ce, O, m, tokens0, 512, steps, list(range(256)), dev_logits, res)
    finally:
        m.close()


def test_7b_nvfp4_all_layers_token_agreement(ce, O):
    """BASELINE config 5 (7B shape, all 32 layers, NVFP4 weights, batch 64,
    cache to 1023 of 2048): 4 sequences x 8 greedy steps against the oracle
    on the dequantized weights."""
    cfg = dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, vocab_size=32000, seq_len=2048)
    steps, seqs = 8, [0, 21, 42, 63]
    m, tokens0, dev_logits, res = _run_device(ce, cfg, 64, 1024, steps, ce.PREC_NVFP4_E2M1)
    try:
        _check_agreement(ce, O, m, tokens0, 1024, steps, seqs, dev_logits, res)
    finally:
        m.close()


def test_step_past_cache_end_reports(ce):
    cfg = dict(dim=128, hidden_dim=256, n_layers=1, n_heads=2, vocab_size=64, seq_len=8)
    m = ce.Llama(cfg, 2, 4)
    try:
        m.init_random(seed=3, kv_fill=7)
        m.start(np.array([1, 2], np.int32), 7)
        m.step()                       # position 7: the last cache slot
        torch.cuda.synchronize()
        ce.llama_status()
        m.step()                       # position 8: past the end
        with pytest.raises(ce.CeError) as err:
            ce.llama_status()
        assert "end of the KV cache" in str(err.value)
        ce.llama_status()              # the status word was cleared
    finally:
        m.close()


@pytest.mark.parametrize("vocab,temperature,top_p", [(1000, 0.8, 0.0), (1000, 1.2, 0.9), (4096, 0.7, 0.8),
                                                     (4096, 1.0, 0.95), (4096, 0.05, 0.5)])
def test_sampling_matches_oracle_sampler(ce, vocab, temperature, top_p):
    """On-device sampling (ce_llama_set_sampling): every step's drawn token
    equals the oracle sampler's on the device's own logits with the same
    coin, except where the coin's target sits within 1e-4 of a cumulative
    boundary (fp32 against float64 arithmetic); vocabularies below and above
    the 1024-candidate cap of the top-p path."""
    from oracle import llama_ref
    cfg = dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, vocab_size=vocab, seq_len=64)
    batch, steps, seed = 48, 4, 1234
    m = ce.Llama(cfg, batch, steps)
    try:
        m.init_random(seed=5, weight_std=0.08, kv_fill=10)
        m.set_sampling(temperature, top_p, seed)
        m.start(np.arange(batch, dtype=np.int32) * 13 % vocab, 10)
        agree = total = 0
        for s in range(steps):
            m.step()
            torch.cuda.synchronize()
            lg = m.logits().astype(np.float64)
            tok = m.generated()[:, s]
            for b in range(batch):
                want, margin = llama_ref.sample_row(lg[b], temperature, top_p, llama_ref.sample_coin(seed, s, b))
                total += 1
                if tok[b] == want:
                    agree += 1
                else:
                    assert margin < 1e-4, (s, b, int(tok[b]), want, margin)
        ce.llama_status()
        assert agree >= 0.99 * total, (agree, total)
    finally:
        m.close()


@pytest.mark.parametrize("cfg,batch,pos0,plen,rows,prec", [
    # chunks of 16 positions over a cache filled to 5
    (dict(dim=128, hidden_dim=256, n_layers=2, n_heads=2, vocab_size=512, seq_len=128), 3, 5, 37, 48, "bf16"),
    # grouped-query, one chunk of 130 positions (three key tiles)
    (dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=1000, seq_len=200),
     2, 0, 130, 512, "bf16"),
    # head size 128, chunks of 33 positions (ragged query tiles) after 70 cached positions
    (dict(dim=256, hidden_dim=384, n_layers=2, n_heads=2, vocab_size=260, seq_len=300), 4, 70, 100, 132, "bf16"),
    # NVFP4 weights, fp16 operands
    (dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, vocab_size=512, seq_len=128), 3, 9, 40, 60, "nvfp4"),
    # two full 128-position query tiles per chunk, keys over three tiles
    (dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, vocab_size=512, seq_len=400), 2, 100, 290, 512, "bf16"),
])
@pytest.mark.parametrize("simt", [False, True], ids=["tensor-cores", "simt"])
def test_prefill_matches_oracle(ce, O, cfg, batch, pos0, plen, rows, prec, simt):
    """ce_llama_enqueue_prefill, with the tensor-core and the SIMT prefill
    attention: the last prompt position's logits and the prompt's K/V rows
    against the oracle's teacher-forced decode of the prompt, the first
    token by the near-tie rule, the position advanced by the prompt length;
    then decode steps continue from it against the oracle."""
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    steps = 3
    m = ce.Llama(cfg, batch, 1 + steps,
                 precision=ce.PREC_NVFP4_E2M1 if prec == "nvfp4" else ce.PREC_BF16)
    try:
        m.init_random(seed=4, weight_std=0.05, kv_fill=pos0)
        m.prefill_reserve(rows)
        m.set_prefill_attention(simt)
        rng = np.random.default_rng(7)
        prompt = rng.integers(0, m.cfg.vocab_size, (batch, plen)).astype(np.int32)
        m.start(prompt[:, 0].copy(), pos0)
        seqs = list(range(batch))
        kc, vc = cache_from_device(m, seqs, pos0)
        m.prefill(torch.from_numpy(prompt).to(dev))
        torch.cuda.synchronize()
        ce.llama_status()
        assert m.read(ce.LLAMA_POS, dtype=np.int32)[0] == pos0 + plen
        dev_logits = m.logits().astype(np.float64)
        orc = LlamaOracle(m.cfg.as_dict(), m.weights(), operand="f16" if prec == "nvfp4" else "bf16")
        forced = np.concatenate([prompt[:, 1:], prompt[:, :1]], axis=1)
        lg, best, _ = orc.decode(prompt[:, 0], pos0, forced, kc, vc)
        assert O.rel_l2(dev_logits, lg[-1]) <= LOGIT_REL_L2
        gen = m.generated()
        for i in seqs:
            if gen[i, 0] != best[-1, i]:
                err = np.abs(dev_logits[i] - lg[-1, i]).max()
                assert lg[-1, i].max() - lg[-1, i, gen[i, 0]] <= max(2 * err, NEAR_TIE)
        # the prompt's K / V rows of the device cache against the oracle's
        dk, dv = cache_from_device(m, seqs, pos0 + plen)
        for l in range(m.cfg.n_layers):
            sl = slice(pos0, pos0 + plen)
            assert O.rel_l2(dk[l][:, :, sl], kc[l][:, :, sl]) <= LOGIT_REL_L2
            assert O.rel_l2(dv[l][:, :, sl], vc[l][:, :, sl]) <= LOGIT_REL_L2
        # decoding continues from the prefill's token and position
        step_logits = []
        for _ in range(steps):
            m.step()
            torch.cuda.synchronize()
            step_logits.append(m.logits().astype(np.float64))
        ce.llama_status()
        gen = m.generated()
        lg2, _, _ = orc.decode(gen[:, 0], pos0 + plen, gen[:, 1:], kc, vc)
        for s in range(steps):
            assert O.rel_l2(step_logits[s], lg2[s]) <= LOGIT_REL_L2
    finally:
        m.close()


def test_prefill_past_cache_end_reports(ce):
    cfg = dict(dim=128, hidden_dim=256, n_layers=1, n_heads=2, vocab_size=64, seq_len=16)
    m = ce.Llama(cfg, 2, 2)
    try:
        m.init_random(seed=3, kv_fill=10)
        with pytest.raises(ce.CeError):
            m.prefill(torch.zeros((2, 4), dtype=torch.int32, device="cuda"))  # no workspace yet
        m.prefill_reserve(16)
        m.start(np.array([1, 2], np.int32), 10)
        m.prefill(torch.ones((2, 6), dtype=torch.int32, device="cuda"))  # positions 10 .. 15: fits
        torch.cuda.synchronize()
        ce.llama_status()
        m.start(np.array([1, 2], np.int32), 12)
        m.prefill(torch.ones((2, 6), dtype=torch.int32, device="cuda"))  # positions 12 .. 17: past the end
        with pytest.raises(ce.CeError) as err:
            ce.llama_status()
        assert "end of the KV cache" in str(err.value)
        ce.llama_status()
    finally:
        m.close()


def test_prefill_110m_shape_sampled(ce, O):
    """BASELINE config 4 shape, batch 16, a 300-token prompt after 20 cached
    positions, chunks of 128 positions: two sequences checked against the
    oracle's teacher-forced decode of their prompts."""
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, vocab_size=32000, seq_len=1024)
    batch, pos0, plen = 16, 20, 300
    m = ce.Llama(cfg, batch, 2)
    try:
        m.init_random(seed=8, weight_std=0.02, kv_fill=pos0)
        m.prefill_reserve(batch * 128)
        prompt = np.random.default_rng(3).integers(0, 32000, (batch, plen)).astype(np.int32)
        m.start(prompt[:, 0].copy(), pos0)
        seqs = [3, 14]
        kc, vc = cache_from_device(m, seqs, pos0)
        m.prefill(torch.from_numpy(prompt).to(dev))
        torch.cuda.synchronize()
        ce.llama_status()
        dev_logits = m.logits()[seqs].astype(np.float64)
        orc = LlamaOracle(m.cfg.as_dict(), m.weights(), operand="bf16")
        forced = np.concatenate([prompt[seqs, 1:], prompt[seqs, :1]], axis=1)
        lg, _, _ = orc.decode(prompt[seqs, 0], pos0, forced, kc, vc)
        assert O.rel_l2(dev_logits, lg[-1]) <= LOGIT_REL_L2
    finally:
        m.close()


def _checkpoint(tmp_path, cfg, shared, seed=5):
    from test_convert_weights import random_tensors
    import cuda_elastic_b200.convert_weights as cw
    t = random_tensors(cfg, seed)
    for k in t:
        if k.startswith("rms"):
            t[k] = (0.5 + np.abs(t[k]) % 1.0).astype(np.float32)
        else:
            t[k] *= np.float32(0.05)
    if shared:
        t["wcls"] = t["tok_emb"]
    path = str(tmp_path / "model.bin")
    cw.write_llama2c(path, cfg, t, shared=shared)
    return path, t, cw


LOAD_CFG = dict(dim=256, hidden_dim=384, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=300, seq_len=64)


@pytest.mark.parametrize("shared", [True, False])
def test_load_llama2c_bf16(ce, O, tmp_path, shared):
    """ce_llama_load from a llama2.c checkpoint: every weight equals the bf16
    rounding of the checkpoint's matrix in the library's row order (q|k|v,
    w1/w3 interleaved), norms exact; decode steps against the oracle."""
    path, t, cw = _checkpoint(tmp_path, LOAD_CFG, shared)
    m = ce.Llama(LOAD_CFG, 3, 3)
    try:
        m.init_random(seed=1, kv_fill=4)   # cache; the weights are replaced below
        m.load_llama2c(path)
        w = m.weights()
        for l in range(LOAD_CFG["n_layers"]):
            for name in ("wqkv", "wo", "w13", "w2"):
                assert np.array_equal(w[name][l], O.bf16_bits(cw.model_matrix(t, name, l))), (name, l)
            assert np.array_equal(w["rms_att"][l], t["rms_att"][l])
            assert np.array_equal(w["rms_ffn"][l], t["rms_ffn"][l])
        assert np.array_equal(w["wcls"], O.bf16_bits(t["wcls"]))
        assert np.array_equal(w["tok_emb"], O.bf16_bits(t["tok_emb"]))
        assert np.array_equal(w["rms_final"], t["rms_final"])
        tokens0 = np.array([1, 77, 299], np.int32)
        m.start(tokens0, 4)
        kc, vc = cache_from_device(m, [0, 1, 2], 4)
        logits = []
        for _ in range(3):
            m.step()
            torch.cuda.synchronize()
            logits.append(m.logits().astype(np.float64))
        ce.llama_status()
        orc = LlamaOracle(m.cfg.as_dict(), w, operand="bf16")
        lg, _, _ = orc.decode(tokens0, 4, m.generated(), kc, vc)
        for s in range(3):
            assert O.rel_l2(logits[s], lg[s]) <= LOGIT_REL_L2
    finally:
        m.close()


def test_offline_nvfp4_equals_quantization_at_load(ce, O, tmp_path):
    """convert_weights (offline NVFP4 file) + ce_llama_load_nvfp4 gives bit
    for bit the weights ce_llama_load quantizes at load, and the same decode;
    the loaded NVFP4 weights are the quantizer's codes of the checkpoint."""
    path, t, cw = _checkpoint(tmp_path, LOAD_CFG, False)
    out = str(tmp_path / "model.nvfp4")
    cw.convert(path, out)
    models = [ce.Llama(LOAD_CFG, 3, 3, precision=ce.PREC_NVFP4_E2M1) for _ in range(2)]
    try:
        for m in models:
            m.init_random(seed=1, kv_fill=4)
        models[0].load_llama2c(path)
        models[1].load_nvfp4_file(out)
        w0, w1 = models[0].weights(), models[1].weights()
        for name in ("wqkv", "wo", "w13", "w2"):
            for l in range(LOAD_CFG["n_layers"]):
                for a, b in zip(w0[name][l], w1[name][l]):
                    assert np.array_equal(np.asarray(a), np.asarray(b)), (name, l)
        for a, b in zip(w0["wcls"], w1["wcls"]):
            assert np.array_equal(np.asarray(a), np.asarray(b))
        assert np.array_equal(w0["tok_emb"], w1["tok_emb"])
        # the codes dequantize to within the NVFP4 step of the checkpoint
        codes, scales, decode = w0["w13"][1]
        deq = O.dequantize_nvfp4(codes, scales, LOAD_CFG["dim"], decode)
        ref = cw.model_matrix(t, "w13", 1)
        assert O.rel_l2(deq, ref) <= 0.15
        outs = []
        for m in models:
            m.start(np.array([5, 6, 7], np.int32), 4)
            for _ in range(3):
                m.step()
            torch.cuda.synchronize()
            outs.append((m.generated().copy(), m.logits().copy()))
        ce.llama_status()
        assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    finally:
        for m in models:
            m.close()
