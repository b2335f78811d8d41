"""CPU oracle of the llama2c hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module, and only as the checker (or the timed CPU baseline).

Byte/integer work (generators, quantizers, token progression) is in orc.c
(liborc.so); the double-precision references and the tolerance rules are
restated here with numpy. Each function cites the reference file:line it
follows (paths relative to the reference project root).

Parity is pinned: tests/test_oracle_pin.py compares this oracle with the
reference's own host code (oracle/_ref/libref.so, compiled from the
reference sources by oracle/Makefile) and with the committed golden vectors
under tests/golden/ that the reference produced.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBORC = os.path.join(HERE, "liborc.so")
LIBREF = os.path.join(HERE, "_ref", "libref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")

_orc = None
_ref = None


def build():
    """Compiles liborc.so (and _ref/libref.so when the reference is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def orc():
    global _orc
    if _orc is None:
        if not os.path.exists(LIBORC):
            build()
        L = ctypes.CDLL(LIBORC)
        L.orc_llama2c_uniform.restype = ctypes.c_float
        L.orc_llama2c_uniform.argtypes = [ctypes.c_uint64] * 3
        L.orc_fill_llama2c.restype = None
        L.orc_fill_llama2c.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, _f32p, _f32p, _f32p, _f32p]
        L.orc_normals.restype = None
        L.orc_normals.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float, _f32p]
        L.orc_uniforms.restype = None
        L.orc_uniforms.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float,
                                   ctypes.c_float, _f32p]
        L.orc_decode.restype = ctypes.c_double
        L.orc_decode.argtypes = [ctypes.c_int, ctypes.c_uint]
        L.orc_encode.restype = ctypes.c_uint
        L.orc_encode.argtypes = [ctypes.c_int, ctypes.c_double]
        L.orc_bf16.restype = ctypes.c_uint16
        L.orc_bf16.argtypes = [ctypes.c_float]
        L.orc_quantize_mxfp6.restype = None
        L.orc_quantize_mxfp6.argtypes = [_f32p, ctypes.c_int64, _u8p, _u8p]
        L.orc_quantize_nvfp4.restype = None
        L.orc_quantize_nvfp4.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float, _u8p, _u8p]
        L.orc_nvfp4_encode_scale.restype = ctypes.c_float
        L.orc_nvfp4_encode_scale.argtypes = [ctypes.c_float]
        L.orc_decoder_tokens.restype = None
        L.orc_decoder_tokens.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _i32p]
        L.orc_fnv1a64.restype = ctypes.c_uint64
        L.orc_fnv1a64.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint64]
        L.orc_cpu_threads.restype = ctypes.c_int
        L.orc_trio_fp32.restype = ctypes.c_int
        L.orc_trio_fp32.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int]
        _orc = L
    return _orc


def ref():
    """The reference's own host code (oracle/_ref/libref.so), or None."""
    global _ref
    if _ref is None:
        if not os.path.exists(LIBREF):
            return None
        L = ctypes.CDLL(LIBREF)
        L.ref_fill_inputs.restype = None
        L.ref_fill_inputs.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, _f32p, _f32p, _f32p, _f32p]
        L.ref_validate_all.restype = ctypes.c_int
        L.ref_validate_all.argtypes = [ctypes.c_int, ctypes.c_uint64, _f32p, _f32p, _f32p, _f32p,
                                       _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       _f32p, _f64p]
        L.ref_time_validate_all.restype = ctypes.c_double
        L.ref_time_validate_all.argtypes = [ctypes.c_int, ctypes.c_uint64, _f32p, _f32p, _f32p, _f32p, _f32p,
                                            _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        L.ref_gamma_probabilistic.restype = ctypes.c_double
        L.ref_gamma_probabilistic.argtypes = [ctypes.c_int]
        L.ref_decoder_compute.restype = ctypes.c_int
        L.ref_decoder_compute.argtypes = [ctypes.c_longlong] * 4 + [_i32p, _i64p,
                                          ctypes.POINTER(ctypes.c_int), _f64p, _f64p, _f64p]
        L.ref_decoder_check.restype = ctypes.c_int
        L.ref_decoder_check.argtypes = [ctypes.c_longlong] * 4 + [_i32p, _f32p, _f32p, _f32p]
        L.ref_decode.restype = ctypes.c_double
        L.ref_decode.argtypes = [ctypes.c_int, ctypes.c_uint]
        L.ref_encode.restype = ctypes.c_uint
        L.ref_encode.argtypes = [ctypes.c_int, ctypes.c_double]
        L.ref_to_bf16.restype = ctypes.c_uint16
        L.ref_to_bf16.argtypes = [ctypes.c_float]
        L.ref_quantize_mxfp6.restype = None
        L.ref_quantize_mxfp6.argtypes = [_f32p, ctypes.c_longlong, _u8p, _u8p]
        L.ref_quantize_nvfp4.restype = None
        L.ref_quantize_nvfp4.argtypes = [_f32p, ctypes.c_longlong, ctypes.c_float, _u8p, _u8p]
        L.ref_nvfp4_encode_scale.restype = ctypes.c_float
        L.ref_nvfp4_encode_scale.argtypes = [ctypes.c_float]
        L.ref_make_fixture.restype = None
        L.ref_make_fixture.argtypes = [ctypes.c_int, ctypes.c_longlong, ctypes.c_longlong, _f32p, _f32p]
        L.ref_rmsnorm_float.restype = None
        L.ref_rmsnorm_float.argtypes = [_f32p, ctypes.c_longlong, _f32p]
        _ref = L
    return _ref


def ref_time_validate_all(x, probs, w, matrix, normalized, softmax, product, random=1, seed=0, reps=1):
    """Mean seconds of the reference's own validate_all (its CPU path of the
    llama2c iteration, compiled unmodified into _ref/libref.so) on the given
    inputs and outputs, and its verdict; None when libref.so is absent."""
    R = ref()
    if R is None:
        return None
    b, s = x.shape
    rows = matrix.shape[0]
    valid = ctypes.c_int(0)
    c = lambda a: np.ascontiguousarray(a, np.float32)
    sec = R.ref_time_validate_all(random, seed, c(x), c(probs), c(w), c(matrix), c(normalized), c(softmax),
                                  c(product), b, s, rows, reps, ctypes.byref(valid))
    return sec, bool(valid.value)


# ---------------------------------------------------------------------------
# Inputs

def llama2c_inputs(random, seed, batch, size, rows):
    """fill_inputs, llama2c/llama2c_common.h:105-132."""
    x = np.empty(batch * size, np.float32)
    p = np.empty(batch * size, np.float32)
    w = np.empty(size, np.float32)
    m = np.empty(rows * size, np.float32)
    orc().orc_fill_llama2c(int(random), seed, batch, size, rows, x, p, w, m)
    return x.reshape(batch, size), p.reshape(batch, size), w, m.reshape(rows, size)


def normals(seed, stream, count, scale=1.0):
    """Fixture normals, experiments/blackwell/lowprec/reference.cpp:183-209."""
    out = np.empty(count, np.float32)
    orc().orc_normals(seed, stream, count, scale, out)
    return out


def uniforms(seed, stream, count, lo, hi):
    out = np.empty(count, np.float32)
    orc().orc_uniforms(seed, stream, count, lo, hi, out)
    return out


def trio_inputs(seed, batch, size, rows):
    """BASELINE op-trio inputs (configs 1-2): x ~ N(0,1) stream 1, the matrix
    W ~ N(0,1)/sqrt(size) stream 2 (float product, as the reference's fixture
    classifier, reference.cpp:203-209), softmax logits ~ N(0,1) stream 3 and
    the rmsnorm weight ~ U(0.5,1.5) stream 4 of the fixture generator."""
    x = normals(seed, 1, batch * size).reshape(batch, size)
    W = normals(seed, 2, rows * size, float(np.float32(1.0 / np.sqrt(size)))).reshape(rows, size)
    logits = normals(seed, 3, batch * size).reshape(batch, size)
    w = uniforms(seed, 4, size, 0.5, 1.5)
    return x, w, logits, W


# ---------------------------------------------------------------------------
# Double references and tolerance rules

RMS_EPS = np.float32(1.0e-5)  # kRmsEpsilon, llama2c_common.h:44


def rmsnorm_ref(x, w, eps=RMS_EPS):
    """validate_outputs_reference's rmsnorm, llama2c_common.h:251-256, 265:
    x * (1 / sqrt(sum x^2 / size + eps)) * w in double."""
    x64 = np.asarray(x, np.float64)
    scale = 1.0 / np.sqrt((x64 * x64).sum(axis=1) / x.shape[1] + float(eps))
    return x64 * scale[:, None] * np.asarray(w, np.float64)[None, :]


def softmax_ref(logits):
    """llama2c_common.h:257-267: exp(p - max) / sum in double."""
    l64 = np.asarray(logits, np.float64)
    e = np.exp(l64 - l64.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


def gamma_probabilistic(n):
    """llama2c_gamma_probabilistic, llama2c_common.h:231-235."""
    u = 2.0 ** -24
    lam = 9.0
    return np.expm1(lam * np.sqrt(n) * u + n * u * u / (1.0 - u))


def gemv_ref(matrix, x):
    """llama2c_common.h:279-292: double dot products and the per-row
    tolerance gamma~_n(9) * sum|M x| + FLT_MIN."""
    m64 = np.asarray(matrix, np.float64)
    x64 = np.asarray(x, np.float64)
    ref = m64 @ x64
    mag = np.abs(m64) @ np.abs(x64)
    tol = gamma_probabilistic(matrix.shape[1]) * mag + np.finfo(np.float32).tiny
    return ref, tol


def validate_llama2c(random, x, probs, w, matrix, normalized, softmax, product):
    """validate_all, llama2c_common.h:150-198, 237-319. Returns (valid,
    product_tolerance float32, product_reference float64)."""
    batch, size = x.shape
    rows = matrix.shape[0]
    valid = True
    exp_norm = rmsnorm_ref(x, w)
    if not np.all(np.abs(normalized.astype(np.float64) - exp_norm) <= 3.0e-4):
        valid = False
    exp_p = softmax_ref(probs)
    act = softmax.astype(np.float64)
    if not np.all(np.abs(act - exp_p) <= 1.0e-9 + 1.0e-3 * exp_p):
        valid = False
    if not np.all(np.isfinite(act)) or np.any(act < 0):
        valid = False
    psum = act.sum(axis=1)
    if not np.all(np.isfinite(psum) & (np.abs(psum - 1.0) <= 3.0e-4)):
        valid = False
    ref, tol = gemv_ref(matrix, x.reshape(-1)[:size])
    tol32 = tol.astype(np.float32)
    if not np.all(np.abs(product.astype(np.float64) - ref) <= tol):
        valid = False
    if not random:
        # validate_outputs (the deterministic oracle), llama2c_common.h:150-198
        xf = x.astype(np.float32)
        ss = (x.astype(np.float64) ** 2).sum(axis=1)
        scale = (np.float32(1.0) / np.sqrt((ss / size).astype(np.float32) + RMS_EPS)).astype(np.float32)
        expected = xf * scale[:, None] * w[None, :]
        if not np.all(np.abs(normalized - expected) <= np.float32(3.0e-4)):
            valid = False
        mx = xf.max(axis=1, keepdims=True)
        e = np.exp((xf - mx).astype(np.float64))
        ep = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
        if not np.all(np.abs(softmax - ep) <= np.float32(1e-9) + np.float32(1e-3) * np.abs(ep)):
            valid = False
        if not np.all(np.abs(product - xf.reshape(-1)[np.arange(rows) % size]) <= np.float32(1e-4)):
            valid = False
        tol32 = np.minimum(tol32, np.float32(1.0e-4))
    return valid, tol32, ref


def gemm_ref(a, b):
    """out[m][n] = sum_k a[m][k] * b[n][k] in double, and sum |a||b| (the
    scale of the rounding-error bounds)."""
    a64 = np.asarray(a, np.float64)
    b64 = np.asarray(b, np.float64)
    return a64 @ b64.T, np.abs(a64) @ np.abs(b64).T


def gamma_worst(k, u=2.0 ** -23):
    """gamma_K = K u / (1 - K u), the worst-case fp32 accumulation bound of the
    lowprec implementation check (decoder_lowprec.cu:981-1052, spec.json
    "implementation_check.logits")."""
    return k * u / (1.0 - k * u)


def rel_l2(actual, expected):
    """Relative L2 error ||a - e|| / ||e|| (the north-star GEMM metric)."""
    e = np.asarray(expected, np.float64)
    d = np.asarray(actual, np.float64) - e
    return float(np.sqrt((d * d).sum() / max((e * e).sum(), 1e-300)))


# ---------------------------------------------------------------------------
# bf16 / low-precision codes

def bf16_bits(x):
    """Round-to-nearest-even bf16 bits of float32 values (reference.cpp:84-96)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_value(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def encode(fmt, v):
    return orc().orc_encode(fmt, float(v))


def decode(fmt, code):
    return orc().orc_decode(fmt, int(code))


# ---------------------------------------------------------------------------
# Decoder (applications/loom_private/decoder)

def decoder_tokens(batch, vocab, steps):
    """oracle.cpp:84-95: [batch][steps] analytic token progression."""
    t = np.empty(batch * steps, np.int32)
    orc().orc_decoder_tokens(batch, vocab, steps, t)
    return t.reshape(batch, steps)


# lp::fnv1a64's initial state is the literal 1469598103934665603
# (applications/loom_private/common/lp_harness.cuh:108), one decimal digit
# short of the published FNV-1a 64 offset basis 14695981039346656037; the
# reference's digests (e.g. the decoder's 4fcc3e102976547b) are defined with
# it, so the oracle uses the same state.
LP_FNV_STATE = 1469598103934665603


def fnv1a64(arrays, h=LP_FNV_STATE):
    """lp::fnv1a64 chained over the byte images of arrays
    (applications/loom_private/common/lp_harness.cuh:107-115)."""
    for a in arrays:
        a = np.ascontiguousarray(a)
        h = orc().orc_fnv1a64(a.ctypes.data, a.nbytes, h)
    return h


# ---------------------------------------------------------------------------
# Timed CPU baseline

def cpu_threads():
    return orc().orc_cpu_threads()


def trio_fp32(x, w, logits, W, eps=RMS_EPS, threads=0):
    """Multithreaded fp32 op-trio step on the CPU (rmsnorm, softmax, GEMM of
    the normalized rows). Returns (normalized, softmax, out, threads)."""
    b, k = x.shape
    n = W.shape[0]
    norm = np.empty((b, k), np.float32)
    soft = np.empty((b, k), np.float32)
    out = np.empty((b, n), np.float32)
    used = orc().orc_trio_fp32(np.ascontiguousarray(x), np.ascontiguousarray(w),
                               np.ascontiguousarray(logits), np.ascontiguousarray(W),
                               norm, soft, out, b, k, n, float(eps), threads)
    return norm, soft, out, used


def decoder_sampled(batch):
    """Up to 8 sequences spread evenly over the batch, both ends included
    (applications/loom_private/decoder/oracle.cpp:97-102)."""
    count = min(8, batch)
    out = []
    for i in range(count):
        b = 0 if count == 1 else i * (batch - 1) // (count - 1)
        if not out or out[-1] != b:
            out.append(b)
    return out


def decoder_reference(batch, width, vocab, steps):
    """decoder_oracle::compute (oracle.cpp:31-123) for the synthetic model:
    analytic tokens, and the double-precision rmsnorm -> classifier ->
    softmax -> argmax of the sampled sequences. The classifier row r has a
    single 1 at column (r + vocab - 1) mod vocab, so its dense double sum is
    that one product (every other term is an exact zero)."""
    tokens = decoder_tokens(batch, vocab, steps)
    sampled = decoder_sampled(batch)
    n = len(sampled)
    normalized = np.empty((n, steps, width))
    logits = np.empty((n, steps, vocab))
    probs = np.empty((n, steps, vocab))
    consistent = True
    perm = (np.arange(vocab) + vocab - 1) % vocab
    for i, b in enumerate(sampled):
        token = b % vocab
        for s in range(steps):
            act = np.ones(width)
            act[token] = 4.0
            ss = float((act * act).sum())
            scale = 1.0 / np.sqrt(ss / width + 1.0e-5)
            o = 1.0 * (scale * act)
            lg = o[perm]
            p = np.exp(lg - lg.max())
            p = p / p.sum()
            best = int(np.argmax(p))  # first maximum
            if best != (token + 1) % vocab:
                consistent = False
            normalized[i, s], logits[i, s], probs[i, s] = o, lg, p
            token = best
    return {"tokens": tokens, "sampled": sampled, "normalized": normalized, "logits": logits,
            "probabilities": probs, "self_consistent": consistent}


def decoder_check(ref, generated, normalized, logits, probabilities):
    """decoder_oracle::check (oracle.cpp:125-229). generated [B][S] int32,
    normalized [S][B][W], logits / probabilities [S][B][V] float32. Returns
    (pass, report) where report lists the first mismatches of each kind."""
    tokens = ref["tokens"]
    B, S = tokens.shape
    W = normalized.shape[2]
    V = logits.shape[2]
    report = {"token": [], "invariant": [], "dense": []}
    bad = np.argwhere(generated != tokens)
    for b, s in bad[:8]:
        report["token"].append(f"token mismatch sequence {b} step {s}: expected {tokens[b, s]}, "
                               f"actual {generated[b, s]}")
    token_errors = len(bad)
    square_bound = np.float32(2.0e-5) + np.float32(1.2e-7) * np.float32(W)
    prob_bound = np.float32(1.0e-6) + np.float32(1.2e-7) * np.float32(V)
    sq = (normalized.astype(np.float64) ** 2).sum(axis=2)          # [S][B]
    square_mean = (sq / W).astype(np.float32)
    psum = probabilities.astype(np.float64).sum(axis=2).astype(np.float32)
    sq_err = np.abs(square_mean - np.float32(1.0))
    p_err = np.abs(psum - np.float32(1.0))
    inv_bad = ~((sq_err <= square_bound) & (p_err <= prob_bound))  # NaN fails
    for s, b in np.argwhere(inv_bad)[:8]:
        report["invariant"].append(f"invariant failure sequence {b} step {s}")
    invariant_errors = int(inv_bad.sum())
    dense_errors = 0
    for i, b in enumerate(ref["sampled"]):
        for s in range(S):
            for what, obs, exp, rel in (("normalized", normalized[s, b], ref["normalized"][i, s], 2.0e-6),
                                        ("logit", logits[s, b], ref["logits"][i, s], 2.0e-6),
                                        ("probability", probabilities[s, b], ref["probabilities"][i, s], 2.0e-5)):
                ok = np.abs(obs.astype(np.float64) - exp) <= rel * np.abs(exp) + 1.0e-12
                if not ok.all():
                    idx = np.argwhere(~ok).ravel()
                    dense_errors += len(idx)
                    if len(report["dense"]) < 8:
                        j = idx[0]
                        report["dense"].append(f"{what} mismatch sequence {b} step {s} index {j}: "
                                               f"expected {exp[j]:.9g}, actual {obs[j]:.9g}")
    passed = ref["self_consistent"] and token_errors == 0 and invariant_errors == 0 and dense_errors == 0
    report.update(token_errors=token_errors, invariant_errors=invariant_errors, dense_errors=dense_errors)
    return passed, report


def read_l2cdump1(path):
    """Reader of the L2CDUMP1 dump (llama2c/llama2c_common.h:16-32):
    header, normalized[B*S] f32, softmax[B*S] f32, product[R] f32,
    product_tolerance[R] f32, product_reference[R] f64."""
    with open(path, "rb") as f:
        raw = f.read()
    if raw[:8] != b"L2CDUMP1":
        raise ValueError(f"{path}: not an L2CDUMP1 dump")
    batch, size, rows, inputs = np.frombuffer(raw, np.int32, 4, 8)
    seed = int(np.frombuffer(raw, np.uint64, 1, 24)[0])
    off = 32
    vec = int(batch) * int(size)
    out = {"batch": int(batch), "size": int(size), "rows": int(rows), "random": int(inputs),
           "seed": seed}
    for name, dt, n in (("normalized", np.float32, vec), ("softmax", np.float32, vec),
                        ("product", np.float32, int(rows)), ("product_tolerance", np.float32, int(rows)),
                        ("product_reference", np.float64, int(rows))):
        out[name] = np.frombuffer(raw, dt, n, off).copy()
        off += n * np.dtype(dt).itemsize
    if off != len(raw):
        raise ValueError(f"{path}: {len(raw) - off} trailing bytes")
    out["normalized"] = out["normalized"].reshape(int(batch), int(size))
    out["softmax"] = out["softmax"].reshape(int(batch), int(size))
    return out


def read_l2cdump2(path):
    """Reader of the op-trio dump L2CDUMP2 of the llama2c_b200 harness (the
    L2CDUMP1 layout with the GEMM output out[B][R] in place of the GEMV
    product): "L2CDUMP2", int32 batch, size, rows, inputs, uint64 seed, int32
    precision, int32 checked C, normalized[B*S] f32, softmax[B*S] f32,
    out[B*R] f32, checked_rows[C] i32, out_tolerance[C*R] f32,
    out_reference[C*R] f64."""
    with open(path, "rb") as f:
        raw = f.read()
    if raw[:8] != b"L2CDUMP2":
        raise ValueError(f"{path}: not an L2CDUMP2 dump")
    batch, size, rows, inputs = (int(v) for v in np.frombuffer(raw, np.int32, 4, 8))
    seed = int(np.frombuffer(raw, np.uint64, 1, 24)[0])
    precision, checked = (int(v) for v in np.frombuffer(raw, np.int32, 2, 32))
    out = {"batch": batch, "size": size, "rows": rows, "inputs": inputs, "seed": seed,
           "precision": precision, "checked": checked}
    off = 40
    for name, dt, n, shape in (("normalized", np.float32, batch * size, (batch, size)),
                               ("softmax", np.float32, batch * size, (batch, size)),
                               ("out", np.float32, batch * rows, (batch, rows)),
                               ("checked_rows", np.int32, checked, (checked,)),
                               ("out_tolerance", np.float32, checked * rows, (checked, rows)),
                               ("out_reference", np.float64, checked * rows, (checked, rows))):
        out[name] = np.frombuffer(raw, dt, n, off).copy().reshape(shape)
        off += n * np.dtype(dt).itemsize
    if off != len(raw):
        raise ValueError(f"{path}: {len(raw) - off} trailing bytes")
    return out


_TABLES = {}
_NCODES = {0: 8, 1: 32, 2: 127, 3: 255, 4: 127}   # magnitude codes per format
_SIGN = {0: 8, 1: 32, 4: 128}


def magnitude_table(fmt):
    if fmt not in _TABLES:
        _TABLES[fmt] = np.array([decode(fmt, c) for c in range(_NCODES[fmt])])
    return _TABLES[fmt]


def encode_array(fmt, v):
    """Vectorised orc_encode (experiments/blackwell/lowprec/reference.cpp:67-82
    rules): nearest code, ties to the code whose last magnitude bit is 0,
    saturation at the largest magnitude, +0 for a zero magnitude. fmt 4 is
    the signed OCP E4M3 of the FP8 mode (UE4M3's magnitudes plus a sign bit)."""
    v = np.asarray(v, np.float64)
    t = np.abs(v)
    tab = magnitude_table(fmt)
    top = len(tab) - 1
    below = np.clip(np.searchsorted(tab, t, side="right") - 1, 0, top)
    nxt = np.minimum(below + 1, top)
    down = t - tab[below]
    up = tab[nxt] - t
    go_up = (below < top) & (tab[below] < t) & ((up < down) | ((up == down) & ((below & 1) == 1)))
    best = np.where(go_up, below + 1, below).astype(np.uint32)
    sign = _SIGN.get(fmt, 0)
    if sign:
        best = np.where((v < 0) & (best != 0), best | sign, best)
    return best


def decode_array(fmt, codes):
    codes = np.asarray(codes, np.uint32)
    sign = _SIGN.get(fmt, 0)
    mag = codes & (sign - 1) if sign else codes
    vals = magnitude_table(fmt)[np.minimum(mag, _NCODES[fmt] - 1)]
    return np.where(sign and (codes & sign) != 0, -vals, vals) if sign else vals


def quantize_e4m3_rows(x):
    """FP8 per-row mode: amax = max|x| of the row, inv = 448 / amax, scale =
    amax / 448 (fp32; 0 for a zero row), code = E4M3(x * inv) with the
    rounding above. Returns (codes uint8 [rows][cols], scales float32)."""
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=1)
    with np.errstate(divide="ignore"):
        inv = np.where(amax > 0, np.float32(448.0) / amax, np.float32(0.0)).astype(np.float32)
    scale = (amax / np.float32(448.0)).astype(np.float32)
    q = (x * inv[:, None]).astype(np.float32)
    return encode_array(4, q).astype(np.uint8), scale


def dequantize_e4m3_rows(codes, scales):
    return decode_array(4, codes) * np.asarray(scales, np.float64)[:, None]


def dequantize_mxfp6(codes, scales):
    """E3M2 codes [rows][cols] (one per byte) times 2^(UE8M0 - 127) of their
    32-value block (decoder_lowprec.cu's MXFP6 mode), in double."""
    vals = decode_array(1, codes)
    exps = np.repeat(np.asarray(scales, np.float64) - 127.0, 32, axis=1)[:, :vals.shape[1]]
    return vals * np.exp2(exps)


def dequantize_nvfp4(packed, scales, cols, decode=1.0):
    """E2M1 codes packed two per byte (even column in the low nibble) times
    the UE4M3 scale of their 16-value block times the fp32 decode tensor
    scale, in double."""
    packed = np.asarray(packed, np.uint8)
    codes = np.empty((packed.shape[0], packed.shape[1] * 2), np.uint8)
    codes[:, 0::2], codes[:, 1::2] = packed & 0x0F, packed >> 4
    vals = decode_array(0, codes[:, :cols])
    return vals * np.repeat(decode_array(2, scales), 16, axis=1)[:, :cols] * float(decode)
