#!/usr/bin/env python3
"""Offline weight conversion for the Llama decoder (ce_llama_*).

Usage: convert_weights.py MODEL.bin OUT.nvfp4

Reads a llama2.c checkpoint (fp32) and writes its GEMM weights quantized to
NVFP4 ahead of time, so that serving loads them with ce_llama_load_nvfp4
instead of converting at set-up (the reference converts its classifier at
set-up, experiments/blackwell/lowprec/decoder_lowprec.cu:573-579). The
quantizer is the library's own device quantizer (ce_quantize_nvfp4: tensor
scale from the matrix amax, UE4M3 per 16 values, E2M1 codes), so a model
loaded from the file holds bit for bit the weights that ce_llama_load would
have quantized at load. Needs a GPU.

llama2.c checkpoint: int32 dim, hidden_dim, n_layers, n_heads, n_kv_heads,
vocab_size (negative: a separate classifier follows), seq_len; then fp32
token embedding [vocab][dim], rms_att [L][dim], wq [L][dim][dim], wk
[L][kv_dim][dim], wv [L][kv_dim][dim], wo [L][dim][dim], rms_ffn [L][dim],
w1 [L][hidden][dim], w2 [L][dim][hidden], w3 [L][hidden][dim], rms_final
[dim], two RoPE tables [seq_len][head_size / 2] (unused: the library
computes its own), and the classifier [vocab][dim] when not shared.

NVFP4 file: "CENVFP41", int32 dim, hidden_dim, n_layers, n_heads,
n_kv_heads, vocab_size, seq_len, int32 0; the embedding as bf16 bits
[vocab][dim]; rms_att [L][dim], rms_ffn [L][dim], rms_final [dim] fp32; then
per layer the matrices wqkv (q, k, v rows), wo, w13 (w1 and w3 rows
interleaved), w2, and last the classifier, each as float32 alpha[2]
(encode, decode), uint8 codes [rows][cols / 2], uint8 scales [rows][cols /
16].
"""
import os
import sys

import numpy as np

MAGIC = b"CENVFP41"
CONFIG_KEYS = ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "seq_len")
MATRICES = ("wqkv", "wo", "w13", "w2")


def read_llama2c(path):
    """(config dict, tensors dict of fp32 arrays, shared classifier flag) of
    a llama2.c checkpoint; the arrays are read-only views of a memory map."""
    head = np.fromfile(path, dtype="<i4", count=7)
    if head.size != 7:
        raise ValueError(f"{path}: too short for a llama2.c header")
    cfg = dict(zip(CONFIG_KEYS, (int(v) for v in head)))
    shared = cfg["vocab_size"] > 0
    cfg["vocab_size"] = abs(cfg["vocab_size"])
    D, H, L, V = cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["vocab_size"]
    if D <= 0 or H <= 0 or L <= 0 or cfg["n_heads"] <= 0 or cfg["n_kv_heads"] <= 0 or cfg["seq_len"] <= 0:
        raise ValueError(f"{path}: invalid llama2.c config {cfg}")
    hs = D // cfg["n_heads"]
    kvd = hs * cfg["n_kv_heads"]
    data = np.memmap(path, dtype="<f4", mode="r", offset=28)
    layout = [("tok_emb", (V, D)), ("rms_att", (L, D)), ("wq", (L, D, D)), ("wk", (L, kvd, D)),
              ("wv", (L, kvd, D)), ("wo", (L, D, D)), ("rms_ffn", (L, D)), ("w1", (L, H, D)),
              ("w2", (L, D, H)), ("w3", (L, H, D)), ("rms_final", (D,)),
              ("rope_real", (cfg["seq_len"], hs // 2)), ("rope_imag", (cfg["seq_len"], hs // 2))]
    if not shared:
        layout.append(("wcls", (V, D)))
    out, off = {}, 0
    for name, shape in layout:
        n = int(np.prod(shape))
        if off + n > data.size:
            raise ValueError(f"{path}: truncated in {name}")
        out[name] = data[off:off + n].reshape(shape)
        off += n
    if off != data.size:
        raise ValueError(f"{path}: {4 * (data.size - off)} trailing bytes")
    if shared:
        out["wcls"] = out["tok_emb"]
    return cfg, out, shared


def write_llama2c(path, cfg, t, shared=True):
    """Writes a llama2.c checkpoint (the inverse of read_llama2c; RoPE tables
    as llama2.c's export writes them)."""
    hs = cfg["dim"] // cfg["n_heads"]
    pos = np.arange(cfg["seq_len"])[:, None]
    freqs = 1.0 / (10000.0 ** (np.arange(0, hs, 2)[None, :] / hs))
    with open(path, "wb") as f:
        head = [cfg[k] for k in CONFIG_KEYS]
        if not shared:
            head[5] = -head[5]
        f.write(np.asarray(head, "<i4").tobytes())
        for name in ("tok_emb", "rms_att", "wq", "wk", "wv", "wo", "rms_ffn", "w1", "w2", "w3", "rms_final"):
            f.write(np.ascontiguousarray(t[name], "<f4").tobytes())
        f.write(np.cos(pos * freqs).astype("<f4").tobytes())
        f.write(np.sin(pos * freqs).astype("<f4").tobytes())
        if not shared:
            f.write(np.ascontiguousarray(t["wcls"], "<f4").tobytes())


def model_matrix(t, name, layer):
    """A GEMM weight of the checkpoint in the library's global row order:
    wqkv = the q, k, v rows; w13 = w1 and w3 rows interleaved."""
    if name == "wqkv":
        return np.concatenate([t["wq"][layer], t["wk"][layer], t["wv"][layer]], axis=0)
    if name == "w13":
        w1, w3 = t["w1"][layer], t["w3"][layer]
        out = np.empty((2 * w1.shape[0], w1.shape[1]), np.float32)
        out[0::2], out[1::2] = w1, w3
        return out
    if name == "wcls":
        return np.asarray(t["wcls"])
    return np.asarray(t[name][layer])


def write_nvfp4_file(path, cfg, emb_bf16, norms, mats):
    """norms: (rms_att [L][dim], rms_ffn [L][dim], rms_final [dim]); mats: a
    list, in file order, of (alpha[2] f32, codes, scales)."""
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(np.asarray([cfg[k] for k in CONFIG_KEYS] + [0], "<i4").tobytes())
        f.write(np.ascontiguousarray(emb_bf16, "<u2").tobytes())
        for a in norms:
            f.write(np.ascontiguousarray(a, "<f4").tobytes())
        for alpha, codes, scales in mats:
            f.write(np.asarray(alpha, "<f4").tobytes())
            f.write(np.ascontiguousarray(codes, np.uint8).tobytes())
            f.write(np.ascontiguousarray(scales, np.uint8).tobytes())


def matrix_shapes(cfg):
    """(name, layer, rows, cols) of every GEMM weight in file order."""
    D, H, L, V = cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["vocab_size"]
    kvd = D // cfg["n_heads"] * cfg["n_kv_heads"]
    rows = {"wqkv": (D + 2 * kvd, D), "wo": (D, D), "w13": (2 * H, D), "w2": (D, H)}
    out = [(name, l) + rows[name] for l in range(L) for name in MATRICES]
    out.append(("wcls", 0, V, D))
    return out


def read_nvfp4_file(path):
    """(config dict, embedding bf16 bits, (rms_att, rms_ffn, rms_final),
    [(name, layer, alpha, codes, scales)]) of an NVFP4 file; arrays are views
    of a memory map."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    if bytes(raw[:8]) != MAGIC:
        raise ValueError(f"{path}: not an NVFP4 weight file")
    head = np.frombuffer(raw[8:40].tobytes(), "<i4")
    cfg = dict(zip(CONFIG_KEYS, (int(v) for v in head[:7])))
    D, L, V = cfg["dim"], cfg["n_layers"], cfg["vocab_size"]
    off = 40

    def take(dtype, shape):
        nonlocal off
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        if off + n > raw.size:
            raise ValueError(f"{path}: truncated")
        a = raw[off:off + n].view(dtype).reshape(shape)
        off += n
        return a

    emb = take("<u2", (V, D))
    norms = (take("<f4", (L, D)), take("<f4", (L, D)), take("<f4", (D,)))
    mats = []
    for name, layer, rows, cols in matrix_shapes(cfg):
        alpha = take("<f4", (2,))
        mats.append((name, layer, alpha, take(np.uint8, (rows, cols // 2)), take(np.uint8, (rows, cols // 16))))
    if off != raw.size:
        raise ValueError(f"{path}: {raw.size - off} trailing bytes")
    return cfg, emb, norms, mats


def convert(src, dst):
    """llama2.c checkpoint -> NVFP4 file, quantized on the GPU by the library."""
    import importlib
    import torch
    ce = importlib.import_module(__package__) if __package__ else _load_package()
    cfg, t, _ = read_llama2c(src)
    dev = torch.device("cuda", torch.cuda.current_device())
    emb = torch.from_numpy(np.array(t["tok_emb"], dtype=np.float32)).to(dev)
    emb_bits = torch.empty(emb.shape, dtype=torch.int16, device=dev)
    ce.convert_bf16(emb_bits, emb)
    mats = []
    scratch = torch.zeros(1, dtype=torch.int32, device=dev)
    for name, layer, rows, cols in matrix_shapes(cfg):
        w = torch.from_numpy(np.array(model_matrix(t, name, layer), dtype=np.float32)).to(dev)
        codes = torch.empty((rows, cols // 2), dtype=torch.uint8, device=dev)
        scales = torch.empty((rows, cols // 16), dtype=torch.uint8, device=dev)
        ts = torch.empty(2, device=dev)
        ce.quantize_nvfp4(codes, scales, ts, scratch, w)
        mats.append((ts.cpu().numpy(), codes.cpu().numpy(), scales.cpu().numpy()))
    torch.cuda.synchronize()
    write_nvfp4_file(dst, cfg, emb_bits.cpu().numpy().view(np.uint16),
                     (np.asarray(t["rms_att"]), np.asarray(t["rms_ffn"]), np.asarray(t["rms_final"])), mats)
    return cfg


def _load_package():
    import importlib.util
    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("cuda_elastic_b200", os.path.join(here, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["cuda_elastic_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def main(argv):
    if len(argv) != 3:
        print(__doc__, file=sys.stderr)
        return 2
    cfg = convert(argv[1], argv[2])
    print(f"wrote {argv[2]}: " + " ".join(f"{k}={cfg[k]}" for k in CONFIG_KEYS))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
