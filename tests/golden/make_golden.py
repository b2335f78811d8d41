"""Writes the golden vectors under tests/golden/ from the REFERENCE's own
host code (oracle/_ref/libref.so, compiled from the reference sources by
oracle/Makefile). Run in a container that has the reference tree:

    make -C oracle && python tests/golden/make_golden.py

Fixtures (small, seeded):
  llama2c.npz    fill_inputs (deterministic 8x64x48; random=5 6x40x24) and
                 validate_all's per-row product tolerance and double reference
                 (llama2c/llama2c_common.h:105-132, 237-319)
  formats.npz    decode tables of E2M1/E3M2/UE4M3/UE8M0, encodings of probe
                 values (ties, saturation), bf16 conversions
                 (experiments/blackwell/lowprec/reference.cpp:13-103)
  quantized.npz  MXFP6 / NVFP4 codes and scales of fixture rows
                 (reference.cpp:105-150)
  fixture.npz    make_fixture normals (reference.cpp:172-211)
  decoder.npz    the decoder oracle's token progression
                 (applications/loom_private/decoder/oracle.cpp:84-123)
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402


def main():
    R = O.ref()
    if R is None:
        raise SystemExit("oracle/_ref/libref.so missing: build it with `make -C oracle`")
    out = {}
    for tag, random, seed, (b, s, r) in (("det", 0, 0, (8, 64, 48)), ("rand", 1, 5, (6, 40, 24))):
        x, p = np.empty(b * s, np.float32), np.empty(b * s, np.float32)
        w, m = np.empty(s, np.float32), np.empty(r * s, np.float32)
        R.ref_fill_inputs(random, seed, b, s, r, x, p, w, m)
        # the reference oracle needs outputs to check; its tolerance and double
        # reference do not depend on them
        norm = np.zeros(b * s, np.float32)
        soft = np.zeros(b * s, np.float32)
        prod = np.zeros(r, np.float32)
        tol, refv = np.empty(r, np.float32), np.empty(r, np.float64)
        R.ref_validate_all(random, seed, x, p, w, m, norm, soft, prod, b, s, r, tol, refv)
        out.update({f"{tag}_shape": np.array([b, s, r]), f"{tag}_random": np.array(random),
                    f"{tag}_seed": np.array(seed), f"{tag}_input": x, f"{tag}_probabilities": p,
                    f"{tag}_weight": w, f"{tag}_matrix": m, f"{tag}_product_tolerance": tol,
                    f"{tag}_product_reference": refv})
    np.savez_compressed(os.path.join(HERE, "llama2c.npz"), **out)

    tables = {name: np.array([R.ref_decode(f, c) for c in range(n)])
              for f, (name, n) in enumerate((("e2m1", 16), ("e3m2", 64), ("ue4m3", 127), ("ue8m0", 255)))}
    rng = np.random.default_rng(11)
    probes = np.concatenate([[0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 100.0, 1e-30, 448.0,
                              464.0, 0.0625, 0.1875, 28.0, 30.0],
                             rng.standard_normal(200) * 8, -rng.random(50) * 6])
    enc = {}
    for f, name in enumerate(("enc_e2m1", "enc_e3m2", "enc_ue4m3", "enc_ue8m0")):
        enc[name] = np.array([R.ref_encode(f, v if f < 2 else abs(v)) for v in probes], np.uint32)
    bf_in = np.concatenate([rng.standard_normal(500).astype(np.float32),
                            (np.arange(64, dtype=np.uint32) << 16 | 0x8000).view(np.float32)])
    bf_out = np.array([R.ref_to_bf16(float(v)) for v in bf_in], np.uint16)
    np.savez_compressed(os.path.join(HERE, "formats.npz"), probes=probes, bf16_in=bf_in,
                        bf16_out=bf_out, **tables, **enc)

    width, vocab = 256, 5
    emb, cls = np.empty(width * vocab, np.float32), np.empty(width * vocab, np.float32)
    R.ref_make_fixture(1, width, vocab, emb, cls)
    np.savez_compressed(os.path.join(HERE, "fixture.npz"), shape_seed=np.array([width, vocab, 1]),
                        embedding=emb, classifier=cls)

    rows = emb.reshape(vocab, width).copy()
    rows[1, :32] = 0.0
    rows[2, :16] = np.float32(1e-30)
    s_enc = R.ref_nvfp4_encode_scale(float(np.abs(rows).max()))
    mxc = np.empty((vocab, width), np.uint8); mxs = np.empty((vocab, width // 32), np.uint8)
    nvc = np.empty((vocab, width), np.uint8); nvs = np.empty((vocab, width // 16), np.uint8)
    for i in range(vocab):
        R.ref_quantize_mxfp6(np.ascontiguousarray(rows[i]), width, mxc[i], mxs[i])
        R.ref_quantize_nvfp4(np.ascontiguousarray(rows[i]), width, s_enc, nvc[i], nvs[i])
    np.savez_compressed(os.path.join(HERE, "quantized.npz"), rows=rows, mx_codes=mxc,
                        mx_scales=mxs, nv_codes=nvc, nv_scales=nvs,
                        nv_encode_scale=np.array(s_enc, np.float32))

    B, W, V, S = 40, 96, 16, 5
    tokens = np.empty(B * S, np.int32)
    sampled = np.empty(8, np.int64)
    n = ctypes.c_int()
    nd = np.empty(8 * S * W); lg = np.empty(8 * S * V); pr = np.empty(8 * S * V)
    assert R.ref_decoder_compute(B, W, V, S, tokens, sampled, ctypes.byref(n), nd, lg, pr) == 1
    np.savez_compressed(os.path.join(HERE, "decoder.npz"), shape=np.array([B, W, V, S]),
                        tokens=tokens, sampled=sampled[:n.value],
                        normalized=nd[:n.value * S * W], logits=lg[:n.value * S * V],
                        probabilities=pr[:n.value * S * V])
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
