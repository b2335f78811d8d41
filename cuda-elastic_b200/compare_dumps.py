#!/usr/bin/env python3
"""Compare llama2c_b200 output dumps (--dump=FILE).

Usage: compare_dumps.py REFERENCE.bin OTHER.bin [OTHER.bin ...]

The command line, rules and exit status of the reference harness's
llama2c/compare_dumps.py: every OTHER dump must come from the same inputs (the
same header) and match REFERENCE within the oracle tolerances of
llama2c/llama2c_common.h --

  normalized  |a - b| <= 3e-4
  softmax     |a - b| <= 1e-9 + 1e-3 |reference|
  product     |a - b| <= product_tolerance[row] of REFERENCE     (L2CDUMP1)
  out         |a - b| <= out_tolerance of REFERENCE on its checked rows,
              and relative L2 over all of out <= 1e-2             (L2CDUMP2)

-- and its own GEMV / GEMM output within its own tolerance of the double
reference it carries. Prints one line per dump; exit status 0 when every
OTHER dump passes, 1 on any mismatch or unreadable dump, 2 on usage errors.

L2CDUMP1 (llama2c_common.h:16-32): "L2CDUMP1", int32 batch, size, rows,
inputs, uint64 seed, then normalized[B*S] f32, softmax[B*S] f32,
product[R] f32, product_tolerance[R] f32, product_reference[R] f64.
L2CDUMP2 (the op-trio mode): "L2CDUMP2", int32 batch, size, rows, inputs
(2 = the op-trio generator), uint64 seed, int32 precision, int32 checked
count C, then normalized[B*S] f32, softmax[B*S] f32, out[B*R] f32,
checked_rows[C] i32, out_tolerance[C*R] f32, out_reference[C*R] f64.
"""
import os
import sys

import numpy as np

RMS_TOLERANCE = 3.0e-4
SOFTMAX_RELATIVE = 1.0e-3
SOFTMAX_ABSOLUTE = 1.0e-9
OUT_REL_L2 = 1.0e-2
PRECISIONS = {0: "fp32", 1: "tf32", 2: "bf16", 3: "fp8", 4: "mxfp6", 5: "nvfp4"}


class DumpError(Exception):
    pass


def _take(raw, offset, dtype, count, path, name):
    width = np.dtype(dtype).itemsize
    end = offset + count * width
    if end > len(raw):
        raise DumpError(f"{path}: truncated in {name}")
    return np.frombuffer(raw, dtype, count, offset), end


def load(path):
    """(header dict, sections dict) of an L2CDUMP1 or L2CDUMP2 file."""
    with open(path, "rb") as f:
        raw = f.read()
    magic = raw[:8]
    if magic not in (b"L2CDUMP1", b"L2CDUMP2"):
        raise DumpError(f"{path}: not a llama2c dump")
    version = 1 if magic == b"L2CDUMP1" else 2
    if len(raw) < (32 if version == 1 else 40):
        raise DumpError(f"{path}: truncated header")
    batch, size, rows, inputs = (int(v) for v in np.frombuffer(raw, "<i4", 4, 8))
    seed = int(np.frombuffer(raw, "<u8", 1, 24)[0])
    header = dict(version=version, batch=batch, size=size, rows=rows, inputs=inputs, seed=seed)
    vec = batch * size
    sec = {}
    if version == 1:
        layout = (("normalized", "<f4", vec), ("softmax", "<f4", vec), ("product", "<f4", rows),
                  ("product_tolerance", "<f4", rows), ("product_reference", "<f8", rows))
        offset = 32
    else:
        precision, checked = (int(v) for v in np.frombuffer(raw, "<i4", 2, 32))
        header.update(precision=precision, checked=checked)
        layout = (("normalized", "<f4", vec), ("softmax", "<f4", vec), ("out", "<f4", batch * rows),
                  ("checked_rows", "<i4", checked), ("out_tolerance", "<f4", checked * rows),
                  ("out_reference", "<f8", checked * rows))
        offset = 40
    for name, dtype, count in layout:
        sec[name], offset = _take(raw, offset, dtype, count, path, name)
    if offset != len(raw):
        raise DumpError(f"{path}: {len(raw) - offset} trailing bytes")
    if version == 2:
        sec["out"] = sec["out"].reshape(batch, rows)
        sec["out_tolerance"] = sec["out_tolerance"].reshape(checked, rows)
        sec["out_reference"] = sec["out_reference"].reshape(checked, rows)
        if checked and (sec["checked_rows"].min() < 0 or sec["checked_rows"].max() >= batch):
            raise DumpError(f"{path}: checked row out of range")
    return header, sec


def _stat(actual, expected, tolerance):
    """(max |a - e| / tolerance, max |a - e|); inf when any difference is not finite."""
    d = np.abs(np.asarray(actual, np.float64) - np.asarray(expected, np.float64))
    if d.size == 0:
        return 0.0, 0.0
    if not np.all(np.isfinite(d)):
        return float("inf"), float("inf")
    return float(np.max(d / tolerance)), float(np.max(d))


def compare(ref, other):
    """{output: (max |diff| / tolerance, max |diff|)} of OTHER against REFERENCE."""
    out = {
        "normalized": _stat(other["normalized"], ref["normalized"], RMS_TOLERANCE),
        "softmax": _stat(other["softmax"], ref["softmax"],
                         SOFTMAX_ABSOLUTE + SOFTMAX_RELATIVE * np.abs(ref["softmax"].astype(np.float64))),
    }
    if "product" in ref:
        out["product"] = _stat(other["product"], ref["product"],
                               ref["product_tolerance"].astype(np.float64))
    else:
        rows = ref["checked_rows"]
        out["out"] = _stat(other["out"][rows], ref["out"][rows],
                           ref["out_tolerance"].astype(np.float64))
        a = other["out"].astype(np.float64)
        e = ref["out"].astype(np.float64)
        err = float(np.sqrt(((a - e) ** 2).sum() / max((e * e).sum(), 1e-300)))
        if not np.isfinite(err):
            err = float("inf")
        out["out_rel_l2"] = (err / OUT_REL_L2, err)
    return out


def own_error(sec):
    """A dump's GEMV / GEMM output against the double reference it carries:
    (max |diff| / tolerance, max |diff|)."""
    if "product" in sec:
        return _stat(sec["product"], sec["product_reference"], sec["product_tolerance"].astype(np.float64))
    return _stat(sec["out"][sec["checked_rows"]], sec["out_reference"],
                 sec["out_tolerance"].astype(np.float64))


def identical(a, b):
    keys = ("normalized", "softmax", "product") if "product" in a else ("normalized", "softmax", "out")
    return all(np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)) for k in keys)


def _describe(h):
    text = (f"batch={h['batch']} size={h['size']} rows={h['rows']} "
            f"inputs={ {0: 'deterministic', 1: 'random', 2: 'trio'}.get(h['inputs'], h['inputs']) } "
            f"seed={h['seed']}")
    if h["version"] == 2:
        text += f" precision={PRECISIONS.get(h['precision'], h['precision'])} checked_rows={h['checked']}"
    return text


def main(argv):
    if len(argv) < 3:
        print(__doc__, file=sys.stderr)
        return 2
    try:
        ref_header, ref = load(argv[1])
    except (OSError, DumpError) as e:
        print(f"  {e}", file=sys.stderr)
        return 1
    name = "product" if ref_header["version"] == 1 else "out"
    print(f"  shape {_describe(ref_header)} (numpy)")
    ratio, err = own_error(ref)
    print(f"  {os.path.basename(argv[1])}: reference; {name} error vs double reference "
          f"{err:.3e} ({ratio:.2e} of tolerance)")
    ok = True
    for path in argv[2:]:
        base = os.path.basename(path)
        try:
            header, other = load(path)
        except (OSError, DumpError) as e:
            print(f"  {e}", file=sys.stderr)
            return 1
        if header != ref_header:
            print(f"  {base}: header {_describe(header)} != {_describe(ref_header)}")
            ok = False
            continue
        stats = compare(ref, other)
        ratio, err = own_error(other)
        passed = all(r <= 1.0 for r, _ in stats.values()) and ratio <= 1.0
        ok = ok and passed
        details = " ".join(f"{k}: max|diff|={a:.3e} ({r:.2e} of tol)" for k, (r, a) in stats.items())
        print(f"  {base}: {'PASS' if passed else 'FAIL'}"
              f"{' (bitwise identical)' if identical(ref, other) else ''}; {details}; "
              f"{name} error vs double reference {err:.3e} ({ratio:.2e} of tolerance)")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main(sys.argv))
