"""GPU parity of the block-scaled GEMMs (tcgen05 kind::mxf8f6f4 and
kind::mxf4nvf4 with block scales applied by the tensor core) against the
double GEMM of the dequantized operands: the implementation-check bound of
experiments/blackwell/lowprec/decoder_lowprec.cu:981-1052 (gamma_K sum|a b|
+ 2^-23 |expected|) and <= 1e-2 relative L2 (north star). Operands come from
the device quantizers, which are bit-exact against the reference's host
quantizer (tests/test_gpu_lowprec.py)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _operands(O, M, N, K, seed):
    A = O.normals(seed, 1, M * K).reshape(M, K)
    B = O.normals(seed, 2, N * K, float(np.float32(1.0 / np.sqrt(K)))).reshape(N, K)
    return np.ascontiguousarray(A), np.ascontiguousarray(B)


def _check(O, d, a, b, alpha=1.0):
    ref, mag = O.gemm_ref(a, b)
    ref *= alpha
    mag *= abs(alpha)
    k = a.shape[1]
    bound = O.gamma_worst(k) * mag + 2.0 ** -22 * np.abs(ref) + 1e-30
    err = np.abs(d.astype(np.float64) - ref)
    assert np.all(err <= bound), float((err / bound).max())
    assert O.rel_l2(d, ref) <= 1e-2


def test_pack_mxfp6_layout(ce, O, dev):
    """16 codes -> 12 bytes of 6-bit fields (value i at bits 6i..6i+5) + 4
    zero bytes; ragged last group zero-filled."""
    rng = np.random.default_rng(3)
    rows, cols = 5, 40
    codes = rng.integers(0, 64, (rows, cols)).astype(np.uint8)
    op = ce.pack_mxfp6(torch.from_numpy(codes).to(dev)).cpu().numpy()
    assert op.shape == (rows, 48)
    for r in range(rows):
        for g in range(3):
            grp = np.zeros(16, np.int64)
            n = min(16, cols - 16 * g)
            grp[:n] = codes[r, 16 * g:16 * g + n]
            bits = sum(int(v) << (6 * i) for i, v in enumerate(grp))
            want = bits.to_bytes(12, "little") + bytes(4)
            assert bytes(op[r, 16 * g:16 * g + 16]) == want


def _mx_dequant(O, codes, scales):
    vals = O.decode_array(1, codes)
    return vals * np.exp2(np.repeat(scales.astype(np.float64) - 127.0, 32, axis=1)[:, :codes.shape[1]])


def _nv_dequant(O, packed, scales, K):
    lo = packed & 0x0F
    hi = packed >> 4
    codes = np.empty((packed.shape[0], packed.shape[1] * 2), np.uint8)
    codes[:, 0::2], codes[:, 1::2] = lo, hi
    vals = O.decode_array(0, codes[:, :K])
    return vals * np.repeat(O.decode_array(2, scales), 16, axis=1)[:, :K]


SHAPES = [(128, 224, 128), (300, 1000, 1024), (130, 450, 256), (1, 8, 384)]


@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_mxfp6(ce, O, dev, shape):
    M, N, K = shape
    A, B = _operands(O, M, N, K, 4)
    out = []
    for X in (A, B):
        rows = X.shape[0]
        codes = torch.empty((rows, K), dtype=torch.uint8, device=dev)
        sc = torch.empty((rows, K // 32), dtype=torch.uint8, device=dev)
        ce.quantize_mxfp6(codes, sc, torch.from_numpy(X).to(dev))
        out.append((codes, sc))
    (ca, sa), (cb, sb) = out
    atoms_a = ce.sf_atoms(0, sa, M, K, 128)
    atoms_b = ce.sf_atoms(0, sb, N, K, ce.BS_TILE_N)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_mxfp6(d, ce.pack_mxfp6(ca), atoms_a, ce.pack_mxfp6(cb), atoms_b, k=K)
    ce.device_status()
    a = _mx_dequant(O, ca.cpu().numpy(), sa.cpu().numpy())
    b = _mx_dequant(O, cb.cpu().numpy(), sb.cpu().numpy())
    _check(O, d.cpu().numpy(), a, b)


@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_nvfp4(ce, O, dev, shape):
    M, N, K = shape
    A, B = _operands(O, M, N, K, 5)
    out = []
    for X in (A, B):
        rows = X.shape[0]
        codes = torch.empty((rows, K // 2), dtype=torch.uint8, device=dev)
        sc = torch.empty((rows, K // 16), dtype=torch.uint8, device=dev)
        ts = torch.empty(2, device=dev)
        scratch = torch.zeros(1, dtype=torch.int32, device=dev)
        ce.quantize_nvfp4(codes, sc, ts, scratch, torch.from_numpy(X).to(dev))
        out.append((codes, sc, ts))
    (ca, sa, ta), (cb, sb, tb) = out
    atoms_a = ce.sf_atoms(1, sa, M, K, 128)
    atoms_b = ce.sf_atoms(1, sb, N, K, ce.BS_TILE_N)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_nvfp4(d, ca, atoms_a, ta, cb, atoms_b, tb, K)
    ce.device_status()
    a = _nv_dequant(O, ca.cpu().numpy(), sa.cpu().numpy(), K)
    b = _nv_dequant(O, cb.cpu().numpy(), sb.cpu().numpy(), K)
    alpha = float(np.float32(ta.cpu().numpy()[1]) * np.float32(tb.cpu().numpy()[1]))
    _check(O, d.cpu().numpy(), a, b, alpha)


@pytest.mark.parametrize("prec", ["mxfp6", "nvfp4"])
@pytest.mark.parametrize("shape", [(8, 384, 768), (64, 1024, 512), (1024, 16384, 8192)])
def test_plan_block_scaled(ce, O, dev, prec, shape):
    """The op-trio plan in MXFP6 / NVFP4: weights quantized at setup,
    activations quantized every step after the rmsnorm; the output against
    the double GEMM of the dequantized operands (the spec's implementation
    check), <= 1e-2 relative L2 (north star)."""
    b, s, r = shape
    x, w, logits, W = (O.trio_inputs if b < 1024 else ce.trio_inputs_host)(0, b, s, r)
    pval = {"mxfp6": ce.PREC_MXFP6_E3M2, "nvfp4": ce.PREC_NVFP4_E2M1}[prec]
    plan = ce.Plan(b, s, r, pval)
    dW = torch.from_numpy(W).to(dev)
    plan.set_weights(dW)
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    norm = torch.empty((b, s), device=dev)
    soft = torch.empty((b, s), device=dev)
    out = torch.full((b, r), float("nan"), device=dev)
    plan.trio(norm, soft, out, dx, dw, dl)
    ce.device_status()
    rows = np.arange(b) if b <= 64 else np.random.default_rng(0).choice(b, 16, replace=False)
    # the plan's operands, reproduced by the (bit-exact) standalone quantizers
    ops = []
    for X in (norm, dW):
        n = X.shape[0]
        if prec == "mxfp6":
            c = torch.empty((n, s), dtype=torch.uint8, device=dev)
            sc = torch.empty((n, s // 32), dtype=torch.uint8, device=dev)
            ce.quantize_mxfp6(c, sc, X)
            ops.append((_mx_dequant(O, c.cpu().numpy(), sc.cpu().numpy()), 1.0))
        else:
            c = torch.empty((n, s // 2), dtype=torch.uint8, device=dev)
            sc = torch.empty((n, s // 16), dtype=torch.uint8, device=dev)
            ts = torch.empty(2, device=dev)
            scratch = torch.zeros(1, dtype=torch.int32, device=dev)
            ce.quantize_nvfp4(c, sc, ts, scratch, X)
            ops.append((_nv_dequant(O, c.cpu().numpy(), sc.cpu().numpy(), s), float(ts.cpu()[1])))
    (a, da), (bq, db) = ops
    alpha = float(np.float32(da) * np.float32(db))
    ref, _ = O.gemm_ref(a[rows], bq)
    ho = out.cpu().numpy()[rows]
    assert O.rel_l2(ho, ref * alpha) <= 1e-2
    ref32, _ = O.gemm_ref(O.rmsnorm_ref(x[rows], w), W)
    assert O.rel_l2(ho, ref32) <= (0.12 if prec == "mxfp6" else 0.25)
    plan.close()


W4_SHAPES = [(64, 4096, 1024), (256, 768, 2048), (130, 452, 320), (1, 8, 64), (300, 1000, 1024)]


@pytest.mark.parametrize("shape", W4_SHAPES)
def test_gemm_w4a16_nvfp4_weights_fp16_activations(ce, O, dev, shape):
    """NVFP4 weights expanded to fp16 inside the GEMM (the decode GEMM of the
    7B-shaped decoder): against the double GEMM of the fp16 activations and
    the dequantized weights, times the weight decode scale."""
    M, N, K = shape
    A, B = _operands(O, M, N, K, 6)
    codes = torch.empty((N, K // 2), dtype=torch.uint8, device=dev)
    sc = torch.empty((N, K // 16), dtype=torch.uint8, device=dev)
    ts = torch.empty(2, device=dev)
    scratch = torch.zeros(1, dtype=torch.int32, device=dev)
    ce.quantize_nvfp4(codes, sc, ts, scratch, torch.from_numpy(B).to(dev))
    ct = torch.empty((K // 64) * N * 32, dtype=torch.uint8, device=dev)
    st = torch.empty((K // 64) * N * 4, dtype=torch.uint8, device=dev)
    ce.w4_pack(ct, st, codes, sc, N, K)
    a16 = A.astype(np.float16)
    da = torch.from_numpy(a16.view(np.int16)).to(dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_w4a16(d, da, ct, st, ts[1:])
    ce.device_status()
    a = a16.astype(np.float64)
    b = _nv_dequant(O, codes.cpu().numpy(), sc.cpu().numpy(), K)
    _check(O, d.cpu().numpy(), a, b, float(ts.cpu().numpy()[1]))


def test_w4_pack_layout(ce, O, dev):
    N, K = 12, 192
    rng = np.random.default_rng(2)
    codes = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    sc = rng.integers(0, 120, (N, K // 16), dtype=np.uint8)
    ct = torch.empty((K // 64) * N * 32, dtype=torch.uint8, device=dev)
    st = torch.empty((K // 64) * N * 4, dtype=torch.uint8, device=dev)
    ce.w4_pack(ct, st, torch.from_numpy(codes).to(dev), torch.from_numpy(sc).to(dev), N, K)
    ct = ct.cpu().numpy().reshape(K // 64, N, 32)
    st = st.cpu().numpy().reshape(K // 64, N, 4)
    for kb in range(K // 64):
        assert np.array_equal(ct[kb], codes[:, kb * 32:(kb + 1) * 32])
        assert np.array_equal(st[kb], sc[:, kb * 4:(kb + 1) * 4])


# N % 4 == 0 writes fp32 outputs through the staged bulk-copy epilogue (N =
# 1001: direct stores); 40960 rows = 160 tiles, so some CTAs reuse the
# staging block for a second tile.
W4T_SHAPES = [(64, 4096, 1024, 1), (64, 4352, 4096, 4), (9, 2752, 4096, 3), (130, 452, 320, 1),
              (1, 8, 64, 1), (300, 1000, 1024, 2), (512, 512, 4096, 8), (100, 1000, 1216, 2), (256, 768, 2048, 1),
              (40, 1001, 512, 2), (64, 40960, 256, 1)]


@pytest.mark.parametrize("shape", W4T_SHAPES)
def test_gemm_w4t_decode_form(ce, O, dev, shape):
    """The decode-form W4A16 GEMM (weights the 128-row MMA operand, expanded
    to fp16 in tensor memory; batch the narrow operand): batches of 1 to 512
    (one and two 128-row halves per tile, several batch tiles), N not a
    multiple of 256, K not a multiple of 128, split-K partials summed in
    split order; against the double GEMM of the fp16 activations and the
    dequantized weights, times the decode scale."""
    M, N, K, splits = shape
    A, B = _operands(O, M, N, K, 7)
    codes = torch.empty((N, K // 2), dtype=torch.uint8, device=dev)
    sc = torch.empty((N, K // 16), dtype=torch.uint8, device=dev)
    ts = torch.empty(2, device=dev)
    scratch = torch.zeros(1, dtype=torch.int32, device=dev)
    ce.quantize_nvfp4(codes, sc, ts, scratch, torch.from_numpy(B).to(dev))
    packed = torch.full((ce.w4t_packed_bytes(N, K),), 0xAB, dtype=torch.uint8, device=dev)
    ce.w4t_pack(packed, codes, sc, N, K)
    a16 = A.astype(np.float16)
    da = torch.from_numpy(a16.view(np.int16)).to(dev)
    d = torch.full((splits, M, N), float("nan"), device=dev)
    ce.gemm_w4t(d, da, packed, ts[1:], splits=splits)
    ce.device_status()
    parts = d.cpu().numpy()
    out = parts[0].astype(np.float32)
    for s in range(1, splits):
        out = out + parts[s]
    a = a16.astype(np.float64)
    b = _nv_dequant(O, codes.cpu().numpy(), sc.cpu().numpy(), K)
    _check(O, out, a, b, float(ts.cpu().numpy()[1]))


def test_w4t_pack_layout(ce, O, dev):
    """ce_w4t_pack against a numpy restatement of its layout: per 128-wide k
    block and 128-row group, 8 KB of codes (four 32-row quarters, each four
    16-byte columns of 32 rows) then 1 KB of scales (32 rows of 8 bytes per
    quarter); zero past N and past K; and the host unpacking inverts it."""
    N, K = 40, 320
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    sc = rng.integers(0, 120, (N, K // 16), dtype=np.uint8)
    kb, npad = (K + 127) // 128, (N + 255) // 256 * 256
    nbytes = ce.w4t_packed_bytes(N, K)
    assert nbytes == kb * (npad // 128) * 9216
    packed = torch.full((nbytes,), 0xAB, dtype=torch.uint8, device=dev)
    ce.w4t_pack(packed, torch.from_numpy(codes).to(dev), torch.from_numpy(sc).to(dev), N, K)
    got = packed.cpu().numpy().reshape(kb, npad // 128, 9216)
    cpad = np.zeros((npad, kb * 64), np.uint8)
    cpad[:N, :K // 2] = codes
    spad = np.zeros((npad, kb * 8), np.uint8)
    spad[:N, :K // 16] = sc
    for k in range(kb):
        for hg in range(npad // 128):
            blk = got[k, hg]
            for q in range(4):
                rows = slice(hg * 128 + q * 32, hg * 128 + q * 32 + 32)
                for j in range(4):
                    piece = blk[(q * 4 + j) * 512:(q * 4 + j + 1) * 512].reshape(32, 16)
                    assert np.array_equal(piece, cpad[rows, k * 64 + j * 16:k * 64 + j * 16 + 16])
                srow = blk[8192 + q * 256:8192 + (q + 1) * 256].reshape(32, 8)
                assert np.array_equal(srow, spad[rows, k * 8:k * 8 + 8])
    c2, s2 = ce.w4t_unpack(got.ravel(), N, K)
    assert np.array_equal(c2, codes) and np.array_equal(s2, sc)


@pytest.mark.parametrize("shape", [(300, 512), (256, 256), (1000, 1216)])
def test_w4t_expand_f16(ce, O, dev, shape):
    """ce_w4t_expand_f16: every value e2m1(code) x ue4m3(scale) as fp16, bit
    for bit, from the W4T-packed layout."""
    n, k = shape
    W = torch.randn(n, k, device=dev) * 0.05
    codes = torch.empty((n, k // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((n, k // 16), dtype=torch.uint8, device=dev)
    ts = torch.empty(2, device=dev)
    scratch = torch.zeros(1, dtype=torch.int32, device=dev)
    ce.quantize_nvfp4(codes, scales, ts, scratch, W)
    packed = torch.empty(ce.w4t_packed_bytes(n, k), dtype=torch.uint8, device=dev)
    ce.w4t_pack(packed, codes, scales, n, k)
    out = torch.full((n, k), 0x7E00, dtype=torch.int16, device=dev)
    ce.w4t_expand_f16(out, packed, n, k)
    torch.cuda.synchronize()
    ref = O.dequantize_nvfp4(codes.cpu().numpy(), scales.cpu().numpy(), k).astype(np.float16)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("shape", [(60, 768, 256), (512, 1024, 512), (130, 200, 320)])
def test_gemm_f16(ce, O, dev, shape):
    """ce_gemm_f16 (kind::f16, fp16 operands, alpha from the device): within
    the implementation-check bound of the double product."""
    M, N, K = shape
    a = (torch.randn(M, K, device=dev) * 0.5).half()
    b = (torch.randn(N, K, device=dev) * 0.5).half()
    alpha = torch.tensor([0.37], device=dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_f16(d, a.view(torch.int16), b.view(torch.int16), alpha)
    torch.cuda.synchronize()
    ref, mag = O.gemm_ref(a.float().cpu().numpy(), b.float().cpu().numpy())
    ref *= float(np.float32(0.37))
    bound = O.gamma_worst(K) * mag * 0.37 + 2.0 ** -22 * np.abs(ref) + 1e-30
    assert np.all(np.abs(d.cpu().numpy().astype(np.float64) - ref) <= bound)
