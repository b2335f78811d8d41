"""CPU oracle of the Llama-2 decoder step -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module, and only as the checker (or the timed CPU baseline).

Parity unpinned: the reference has no transformer (its loom_private decoder
runs only the final rmsnorm -> classifier -> argmax stage,
applications/loom_private/decoder/decoder.cu:267-296, and llama2.c's run.c,
whose forward() the reference cites by hash only, is not in the reference
tree). This is a restatement of the standard Llama-2 decoder mathematics in
float64 numpy:

  x = embedding[token]
  per layer: xb = rmsnorm(x, w_att); q, k, v = xb Wq^T, xb Wk^T, xb Wv^T;
             RoPE rotates each (even, odd) pair at head-dimension index j by
             pos * 10000^(-j / head_size); k, v appended to the cache;
             per head: softmax(q k^T / sqrt(head_size)) over positions 0..pos, times v;
             x += att Wo^T; xb = rmsnorm(x, w_ffn);
             x += (silu(xb W1^T) * (xb W3^T)) W2^T,  silu(g) = g / (1 + e^-g)
  logits = rmsnorm(x, w_final) Wcls^T; next token = first argmax
  rmsnorm(x, w) = w * x / sqrt(mean(x^2) + 1e-5)

It rounds where the device path stores 16-bit values (the GEMM operands:
normalized rows, attention output, SwiGLU product, in bf16 or, for the NVFP4
model, fp16; the appended k and v in bf16), so the comparison measures the
device's arithmetic, not the format. Weights and the initial KV cache are inputs copied from the device.
"""
import numpy as np

from .oracle import bf16_bits, bf16_value, decode_array

EPS = 1e-5


def bf16_round(x):
    """Values rounded to bf16 (through float32, as the device rounds its fp32
    values), returned as float64."""
    return bf16_value(bf16_bits(np.asarray(x, np.float32))).astype(np.float64)


def f16_round(x):
    """Values rounded to fp16 (through float32), returned as float64."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float64)


def to64(w):
    """A weight as float64 values: bf16 bits (uint16 array), or an NVFP4
    (codes two per byte with the even index in the low nibble, UE4M3 scales per
    16 values, decode scale) tuple dequantized as e2m1(code) * ue4m3(scale) *
    decode scale (the ce_quantize_nvfp4 format)."""
    if isinstance(w, tuple):
        codes, scales, alpha = w
        rows = codes.shape[0]
        # byte -> (low-nibble value, high-nibble value), then one scale per 16
        pair = np.stack([decode_array(0, np.arange(256) & 0x0F), decode_array(0, np.arange(256) >> 4)],
                        axis=1).astype(np.float64)
        sf = decode_array(2, np.arange(256)).astype(np.float64)
        vals = pair[codes].reshape(rows, -1, 16)
        vals *= sf[scales][:, :, None]
        vals *= alpha
        return vals.reshape(rows, -1)
    return bf16_value(w).astype(np.float64)


def rmsnorm(x, w):
    return w * (x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + EPS))


def rope_angles(pos, hs):
    """(cos, sin) of pos * 10000^(-2i / hs), i < hs / 2."""
    i = np.arange(hs // 2, dtype=np.float64)
    a = pos * np.power(10000.0, -2.0 * i / hs)
    return np.cos(a), np.sin(a)


def rope(v, pos, hs):
    """Rotates the (even, odd) pairs of v [..., n * hs] head by head."""
    c, s = rope_angles(pos, hs)
    shp = v.shape
    w = v.reshape(shp[:-1] + (shp[-1] // hs, hs // 2, 2))
    e, o = w[..., 0], w[..., 1]
    out = np.empty_like(w)
    out[..., 0] = e * c - o * s
    out[..., 1] = e * s + o * c
    return out.reshape(shp)


class LlamaOracle:
    """Teacher-forced greedy decoding of a few sequences.

    cfg: dict with dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size,
    seq_len. weights: the device weights as host arrays (bf16 bits for the
    matrices, fp32 RMSNorm weights), as Llama.weights() returns them; the
    w13 rows interleave w1 and w3 (w1_0, w3_0, w1_1, ...).
    """

    def __init__(self, cfg, weights, operand="bf16"):
        self.c = dict(cfg)
        # rounding of the GEMM operands: bf16, or fp16 (the NVFP4 model)
        self.op = f16_round if operand == "f16" else bf16_round
        self.hs = self.c["dim"] // self.c["n_heads"]
        self.kv_dim = self.hs * self.c["n_kv_heads"]
        self.emb = to64(weights["tok_emb"])
        self.wcls = to64(weights["wcls"])
        self.rms_final = np.asarray(weights["rms_final"], np.float64)
        self.wqkv = [to64(w) for w in weights["wqkv"]]
        self.wo = [to64(w) for w in weights["wo"]]
        self.w13 = [to64(w) for w in weights["w13"]]
        self.w2 = [to64(w) for w in weights["w2"]]
        self.rms_att = [np.asarray(w, np.float64) for w in weights["rms_att"]]
        self.rms_ffn = [np.asarray(w, np.float64) for w in weights["rms_ffn"]]

    def step(self, tokens, pos, kcache, vcache):
        """One decode step of the sequences whose current tokens are given.

        kcache, vcache: per layer float64 [n][kv_heads][seq_len][hs] (bf16
        values), updated in place at pos. Returns logits [n][vocab]."""
        c, hs = self.c, self.hs
        D, Hd, H, KH = c["dim"], c["hidden_dim"], c["n_heads"], c["n_kv_heads"]
        x = self.emb[np.asarray(tokens)]
        group = H // KH
        for l in range(c["n_layers"]):
            xb = self.op(rmsnorm(x, self.rms_att[l]))
            qkv = xb @ self.wqkv[l].T
            q = rope(qkv[:, :D], pos, hs)
            k = rope(qkv[:, D:D + self.kv_dim], pos, hs)
            v = qkv[:, D + self.kv_dim:]
            n = x.shape[0]
            kcache[l][:, :, pos, :] = bf16_round(k).reshape(n, KH, hs)
            vcache[l][:, :, pos, :] = bf16_round(v).reshape(n, KH, hs)
            qh = q.reshape(n, H, hs)
            att = np.empty((n, H, hs))
            for h in range(H):
                kh = h // group
                keys = kcache[l][:, kh, :pos + 1, :]          # [n][pos+1][hs]
                vals = vcache[l][:, kh, :pos + 1, :]
                s = np.einsum("nd,ntd->nt", qh[:, h, :], keys) / np.sqrt(hs)
                p = np.exp(s - s.max(axis=1, keepdims=True))
                p /= p.sum(axis=1, keepdims=True)
                att[:, h, :] = np.einsum("nt,ntd->nd", p, vals)
            x = x + self.op(att.reshape(n, D)) @ self.wo[l].T
            xb = self.op(rmsnorm(x, self.rms_ffn[l]))
            hh = xb @ self.w13[l].T          # rows interleave w1 and w3
            g, u = hh[:, 0::2], hh[:, 1::2]
            x = x + self.op(g / (1.0 + np.exp(-g)) * u) @ self.w2[l].T
        return self.op(rmsnorm(x, self.rms_final)) @ self.wcls.T

    def decode(self, tokens0, pos0, forced, kcache, vcache):
        """Teacher-forced decode: step s feeds tokens0 (s = 0) or forced[:, s-1].
        Returns (logits [S][n][vocab], argmax [S][n], top-2 gap [S][n])."""
        forced = np.asarray(forced)
        S = forced.shape[1]
        logits, best, gap = [], [], []
        tok = np.asarray(tokens0)
        for s in range(S):
            lg = self.step(tok, pos0 + s, kcache, vcache)
            top2 = np.sort(lg, axis=1)[:, -2:]
            logits.append(lg)
            best.append(np.argmax(lg, axis=1))  # first maximum
            gap.append(top2[:, 1] - top2[:, 0])
            tok = forced[:, s]
        return np.stack(logits), np.stack(best), np.stack(gap)


def teacher_forced_layerwise(cfg, layer_weights, emb, rms_final, wcls, tokens_in, pos0, layer_cache,
                             operand="bf16", x0=None, perturb=None):
    """Teacher-forced logits of n sequences over S steps computed one layer
    at a time, as a prefill of the forced tokens: the arithmetic of
    LlamaOracle.step applied to every (sequence, step) row at once, so each
    layer's weights and cache are needed once (a 7B-shaped model never has
    to sit in host memory as float64).

    layer_weights(l): dict of float64 wqkv, wo, w13, w2 and rms_att, rms_ffn;
    layer_cache(l): float64 K, V [n][kv_heads][seq_len][hs] with positions
    < pos0 filled (updated in place); emb, wcls float64 [vocab][dim];
    tokens_in [n][S]: the token fed at step s (step 0: the start token);
    x0: optional float64 [n * S][dim] residual rows to start from instead of
    the embedding rows (row b * S + s); perturb: optional function applied to
    every matrix product's result rows (used to measure how far fp32-level
    noise moves this model). Returns logits [S][n][vocab]."""
    c = dict(cfg)
    op = f16_round if operand == "f16" else bf16_round
    D, H = c["dim"], c["n_heads"]
    KH = c.get("n_kv_heads", H)
    hs = D // H
    kv_dim = hs * KH
    group = H // KH
    tokens_in = np.asarray(tokens_in)
    n, S = tokens_in.shape
    x = emb[tokens_in.reshape(-1)] if x0 is None else np.asarray(x0, np.float64)  # row b * S + s
    mm = (lambda a, w: a @ w.T) if perturb is None else (lambda a, w: perturb(a @ w.T))
    for l in range(c["n_layers"]):
        W = layer_weights(l)
        kc, vc = layer_cache(l)
        xb = op(rmsnorm(x, W["rms_att"]))
        qkv = mm(xb, W["wqkv"])
        q = np.empty((n * S, D))
        for s in range(S):
            rows = np.arange(n) * S + s
            q[rows] = rope(qkv[rows, :D], pos0 + s, hs)
            k = rope(qkv[rows, D:D + kv_dim], pos0 + s, hs)
            kc[:, :, pos0 + s, :] = bf16_round(k).reshape(n, KH, hs)
            vc[:, :, pos0 + s, :] = bf16_round(qkv[rows, D + kv_dim:]).reshape(n, KH, hs)
        att = np.empty((n * S, H, hs))
        for s in range(S):
            rows = np.arange(n) * S + s
            qh = q[rows].reshape(n, H, hs)
            for h in range(H):
                keys = kc[:, h // group, :pos0 + s + 1, :]
                vals = vc[:, h // group, :pos0 + s + 1, :]
                sc = np.einsum("nd,ntd->nt", qh[:, h, :], keys) / np.sqrt(hs)
                p = np.exp(sc - sc.max(axis=1, keepdims=True))
                p /= p.sum(axis=1, keepdims=True)
                att[rows, h, :] = np.einsum("nt,ntd->nd", p, vals)
        x = x + mm(op(att.reshape(n * S, D)), W["wo"])
        xb = op(rmsnorm(x, W["rms_ffn"]))
        hh = mm(xb, W["w13"])
        g, u = hh[:, 0::2], hh[:, 1::2]
        x = x + mm(op(g / (1.0 + np.exp(-g)) * u), W["w2"])
    lg = mm(op(rmsnorm(x, rms_final)), wcls)
    return lg.reshape(n, S, -1).transpose(1, 0, 2)


def cache_from_device(model, seqs, positions):
    """Per layer float64 [n][kv_heads][seq_len][hs] K and V caches of the given
    sequences, with device positions [0, positions) copied in."""
    import importlib
    ce = importlib.import_module("cuda_elastic_b200")
    c = model.cfg
    kc, vc = [], []
    for l in range(c.n_layers):
        k = np.zeros((len(seqs), c.n_kv_heads, c.seq_len, model.hs))
        v = np.zeros_like(k)
        for i, b in enumerate(seqs):
            if positions > 0:
                k[i, :, :positions] = to64(model.cache_rows(l, b, ce.LLAMA_KCACHE, positions))
                v[i, :, :positions] = to64(model.cache_rows(l, b, ce.LLAMA_VCACHE, positions))
        kc.append(k)
        vc.append(v)
    return kc, vc


# --- sampling (the decoder's ce_llama_set_sampling) -------------------------
# Restates the device sampler: coin from splitmix64, softmax(logits / T),
# inverse CDF in vocabulary order, or nucleus (top-p) over the 1024 most
# probable tokens in descending order (llama2.c's sample_mult / sample_topp).
_M64 = (1 << 64) - 1
SAMPLE_CANDIDATES = 1024


def mix64(z):
    """splitmix64 finalizer of a 64-bit integer (the device's mix64)."""
    z = (z + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def sample_coin(seed, step, row):
    """u in [0, 1): (mix64(seed ^ mix64(step * 0x9E3779B97F4A7C15 + row + 1)) >> 40) / 2^24."""
    r = mix64((seed & _M64) ^ mix64((step * 0x9E3779B97F4A7C15 + row + 1) & _M64))
    return float(np.float32((r >> 40) * (1.0 / 16777216.0)))


def sample_row(logits, temperature, top_p, u):
    """(token, margin) for one row: margin is how far the coin's target lies
    from the nearest cumulative-probability boundary of the walk (small
    margins are where fp32 and float64 arithmetic may choose differently)."""
    lg = np.asarray(logits, np.float64)
    e = np.exp((lg - lg.max()) / temperature)
    total = e.sum()
    if not (0.0 < top_p < 1.0):
        cdf = np.cumsum(e)
        target = u * total
        idx = np.nonzero(cdf > target)[0]
        tok = int(idx[0]) if len(idx) else len(lg) - 1
        margin = min(abs(cdf[tok] - target), abs(cdf[tok - 1] - target) if tok > 0 else np.inf) / total
        return tok, margin
    order = np.lexsort((np.arange(len(e)), -e))[:SAMPLE_CANDIDATES]  # descending probability, lower index first
    p = e[order] / total
    cum = np.cumsum(p)
    over = np.nonzero(cum > top_p)[0]
    end = int(over[0]) if len(over) else len(p) - 1
    r = u * cum[end]
    pick = np.nonzero(cum[:end + 1] > r)[0]
    j = int(pick[0]) if len(pick) else end
    margin = min(abs(cum[j] - r), abs(cum[j - 1] - r) if j > 0 else np.inf,
                 abs(cum[end] - top_p), abs(cum[end - 1] - top_p) if end > 0 else np.inf)
    return int(order[j]), margin
