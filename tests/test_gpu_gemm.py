"""GPU parity of the tensor-core GEMMs (tcgen05 bf16 / tf32) and the SIMT
fp32 control, through the C ABI, against the oracle.

Bounds: for bf16 the double reference is computed on the same bf16 operands
and every element must satisfy |d - ref| <= gamma_K * sum_k |a_k b_k| +
1e-30 (fp32 accumulation in any order; the implementation check of
experiments/blackwell/lowprec/decoder_lowprec.cu:981-1052). Against the fp32
operands the relative L2 error must be <= 1e-2 (north star)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bf16_dev(a, dev, ld=None):
    bits = a if a.dtype == np.uint16 else None
    rows, k = a.shape
    ld = ld or k
    buf = np.zeros((rows, ld), np.uint16)
    buf[:, :k] = bits if bits is not None else 0
    return torch.from_numpy(buf.view(np.int16)).to(dev)


def _check_bf16(O, d, A, B):
    ab, bb = O.bf16_value(O.bf16_bits(A)), O.bf16_value(O.bf16_bits(B))
    ref, mag = O.gemm_ref(ab, bb)
    k = A.shape[1]
    bound = O.gamma_worst(k) * mag + 1e-30
    err = np.abs(d.astype(np.float64) - ref)
    assert np.all(err <= bound), float((err / bound).max())
    ref32, _ = O.gemm_ref(A, B)
    assert O.rel_l2(d, ref32) <= 1e-2


SHAPES = [(8, 768, 288), (128, 256, 64), (200, 300, 1000), (1, 1, 8), (129, 257, 72),
          (256, 512, 4096), (1024, 1000, 320), (300, 4100, 64)]


@pytest.mark.parametrize("shape", SHAPES)
def test_bf16_gemm(ce, O, dev, shape):
    M, N, K = shape
    rng = np.random.default_rng(M * 7 + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    da, db = _bf16_dev(O.bf16_bits(A), dev), _bf16_dev(O.bf16_bits(B), dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_bf16(d, da, db)
    ce.device_status()
    _check_bf16(O, d.cpu().numpy(), A, B)


@pytest.mark.parametrize("tile_n", [64, 96, 128, 160, 192, 224, 256])
def test_bf16_gemm_every_tile_width(ce, O, dev, tile_n):
    M, N, K = 300, 1000, 520
    rng = np.random.default_rng(tile_n)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    da, db = _bf16_dev(O.bf16_bits(A), dev), _bf16_dev(O.bf16_bits(B), dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_bf16(d, da, db, tile_n=tile_n)
    ce.device_status()
    _check_bf16(O, d.cpu().numpy(), A, B)


@pytest.mark.parametrize("shape,splits", [((256, 768, 768), 3), ((300, 1000, 520), 9),
                                          ((64, 2304, 4096), 8), ((5, 96, 64), 1), ((130, 200, 1000), 16)])
def test_bf16_split_k_partials_sum_to_the_product(ce, O, dev, shape, splits):
    """Every split writes its own partial; their sum (in split order) meets
    the bf16 GEMM bound, and each partial is the product over its own
    balanced k-block range."""
    M, N, K = shape
    rng = np.random.default_rng(M + splits)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    da, db = _bf16_dev(O.bf16_bits(A), dev), _bf16_dev(O.bf16_bits(B), dev)
    d = torch.full((splits, M, N), float("nan"), device=dev)
    ce.gemm_bf16_split(d, da, db, splits)
    ce.device_status()
    parts = d.cpu().numpy().astype(np.float64)
    _check_bf16(O, parts.sum(axis=0).astype(np.float32), A, B)
    kb = (K + 63) // 64
    Ab, Bb = O.bf16_value(O.bf16_bits(A)).astype(np.float64), O.bf16_value(O.bf16_bits(B)).astype(np.float64)
    for sp in range(splits):
        k0, k1 = 64 * (sp * kb // splits), min(K, 64 * ((sp + 1) * kb // splits))
        ref = Ab[:, k0:k1] @ Bb[:, k0:k1].T
        assert np.allclose(parts[sp], ref, rtol=1e-5, atol=1e-4 * np.sqrt(k1 - k0))


def test_bf16_split_k_rejects_bad_splits(ce, dev):
    a = torch.zeros((8, 128), dtype=torch.int16, device=dev)
    b = torch.zeros((16, 128), dtype=torch.int16, device=dev)
    d = torch.zeros((3, 8, 16), device=dev)
    with pytest.raises(ce.CeError, match="split count"):
        ce.gemm_bf16_split(d, a, b, 3)  # K = 128 is 2 k-blocks


def test_bf16_gemm_ragged_k_with_padded_rows(ce, O, dev):
    """K = 77 inside rows padded to 80 (the columns past K hold garbage that
    the tensor map's extent must exclude)."""
    M, N, K, ld = 70, 90, 77, 80
    rng = np.random.default_rng(5)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    abuf = np.full((M, ld), 0x7fc0, np.uint16)  # NaN bf16 in the padding
    bbuf = np.full((N, ld), 0x7fc0, np.uint16)
    abuf[:, :K], bbuf[:, :K] = O.bf16_bits(A), O.bf16_bits(B)
    da = torch.from_numpy(abuf.view(np.int16)).to(dev)
    db = torch.from_numpy(bbuf.view(np.int16)).to(dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_bf16(d, da, db, k=K)
    ce.device_status()
    _check_bf16(O, d.cpu().numpy(), A, B)


@pytest.mark.parametrize("shape", [(8, 768, 288), (200, 300, 1000), (129, 257, 36)])
def test_tf32_gemm(ce, O, dev, shape):
    M, N, K = shape
    rng = np.random.default_rng(K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_tf32(d, torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev))
    ce.device_status()
    ref, mag = O.gemm_ref(A, B)
    dd = d.cpu().numpy().astype(np.float64)
    # each tf32 operand carries a relative error below 2^-10 (10 stored
    # mantissa bits, rounding or truncation), plus fp32 accumulation
    bound = (2.0 * 2.0 ** -10 + O.gamma_worst(K)) * mag + 1e-30
    assert np.all(np.abs(dd - ref) <= bound)
    assert O.rel_l2(dd, ref) <= 1e-2


@pytest.mark.parametrize("shape", [(8, 768, 288), (130, 70, 1001), (1, 1, 1), (300, 12600, 37),
                                   (1024, 8192, 20), (512, 8192, 24)])
def test_fp32_simt_gemm_is_sequential(ce, O, dev, shape):
    """Bitwise equal to sequential fp32 accumulation from 0 in increasing k
    with separate multiply and add (the decoder contract's order)."""
    M, N, K = shape
    rng = np.random.default_rng(3)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_fp32(d, torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev))
    torch.cuda.synchronize()
    acc = np.zeros((M, N), np.float32)
    for k in range(K):
        acc = acc + np.multiply.outer(A[:, k], B[:, k]).astype(np.float32)
    assert np.array_equal(d.cpu().numpy(), acc)


def test_bf16_gemm_sheet_shape(ce, O, dev):
    """1024 x 8192 x 16384 (the BASELINE GEMM), checked on 48 sampled rows of
    the output against the bound, and the relative L2 on them."""
    M, N, K = 1024, 8192, 16384
    x, w, _, W = ce.trio_inputs_host(0, M, K, N)
    da = torch.from_numpy(O.bf16_bits(x).view(np.int16)).to(dev)
    db = torch.from_numpy(O.bf16_bits(W).view(np.int16)).to(dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_bf16(d, da, db)
    ce.device_status()
    hd = d.cpu().numpy()
    assert np.isfinite(hd).all()
    rows = np.random.default_rng(0).choice(M, 48, replace=False)
    _check_bf16(O, hd[rows], x[rows], W)


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("tile_n", [64, 96, 128, 160, 192, 224, 256])
def test_forced_kernel_and_tile_bf16(ce, O, dev, cta_group, tile_n):
    """Both kernels (single CTA, CTA pair) at every tile width, on a shape
    that is ragged in M, N and K."""
    M, N, K = 300, 1000, 520
    rng = np.random.default_rng(tile_n + 7 * cta_group)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    da, db = _bf16_dev(O.bf16_bits(A), dev), _bf16_dev(O.bf16_bits(B), dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_config(ce.PREC_BF16, d, da, db, cta_group=cta_group, tile_n=tile_n)
    ce.device_status()
    _check_bf16(O, d.cpu().numpy(), A, B)


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("shape", [(520, 300, 100), (256, 224, 32), (1100, 700, 1028)])
def test_forced_kernel_tf32(ce, O, dev, cta_group, shape):
    M, N, K = shape
    rng = np.random.default_rng(M + cta_group)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_config(ce.PREC_TF32, d, torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev),
                   cta_group=cta_group)
    ce.device_status()
    ref, mag = O.gemm_ref(A, B)
    dd = d.cpu().numpy().astype(np.float64)
    bound = (2.0 * 2.0 ** -10 + O.gamma_worst(K)) * mag + 1e-30
    assert np.all(np.abs(dd - ref) <= bound)


@pytest.mark.parametrize("cta_group", [1, 2])
def test_kernels_agree_on_sheet_shape(ce, O, dev, cta_group):
    """Single-CTA and CTA-pair kernels on the BASELINE GEMM shape: the output
    within the bf16 bound on sampled rows."""
    M, N, K = 1024, 8192, 16384
    rng = np.random.default_rng(cta_group)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) / 128.0).astype(np.float32)
    da = torch.from_numpy(O.bf16_bits(A).view(np.int16)).to(dev)
    db = torch.from_numpy(O.bf16_bits(B).view(np.int16)).to(dev)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_config(ce.PREC_BF16, d, da, db, cta_group=cta_group)
    ce.device_status()
    hd = d.cpu().numpy()
    assert np.isfinite(hd).all()
    rows = np.random.default_rng(2).choice(M, 24, replace=False)
    _check_bf16(O, hd[rows], A[rows], B)


@pytest.mark.parametrize("tile_n", [224, 240, 256])
@pytest.mark.parametrize("shape", [(300, 1000, 520), (257, 481, 64), (1024, 2000, 1028)])
def test_two_piece_pair_tiles_bf16(ce, O, dev, tile_n, shape):
    """CTA-pair tiles of two N pieces (cta_group 3: 256 x 2 tile_n, one
    512-column accumulator), ragged in M, N and K, with several tiles per
    pair on the larger shape."""
    M, N, K = shape
    rng = np.random.default_rng(tile_n + M)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    ld = (K + 7) // 8 * 8  # 16-byte row strides
    da, db = _bf16_dev(O.bf16_bits(A), dev, ld), _bf16_dev(O.bf16_bits(B), dev, ld)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_config(ce.PREC_BF16, d, da, db, k=K, cta_group=3, tile_n=tile_n)
    ce.device_status()
    _check_bf16(O, d.cpu().numpy(), A, B)


def test_two_piece_pair_tiles_tf32(ce, O, dev):
    M, N, K = 520, 1000, 100
    rng = np.random.default_rng(5)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    d = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_config(ce.PREC_TF32, d, torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev), cta_group=3,
                   tile_n=240)
    ce.device_status()
    ref, mag = O.gemm_ref(A, B)
    bound = (2.0 * 2.0 ** -10 + O.gamma_worst(K)) * mag + 1e-30
    assert np.all(np.abs(d.cpu().numpy().astype(np.float64) - ref) <= bound)


def test_two_piece_tiles_equal_the_pair_kernel_on_sheet_shape(ce, O, dev):
    """The BASELINE GEMM (1024 x 8192 x 16384) in two-piece pair tiles (the
    automatic choice there) equals the one-piece pair kernel bit for bit:
    every output element accumulates the same products in the same k order."""
    M, N, K = 1024, 8192, 16384
    rng = np.random.default_rng(11)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) / 128.0).astype(np.float32)
    da = torch.from_numpy(O.bf16_bits(A).view(np.int16)).to(dev)
    db = torch.from_numpy(O.bf16_bits(B).view(np.int16)).to(dev)
    d2 = torch.full((M, N), float("nan"), device=dev)
    d3 = torch.full((M, N), float("nan"), device=dev)
    ce.gemm_config(ce.PREC_BF16, d2, da, db, cta_group=2, tile_n=224)
    ce.gemm_config(ce.PREC_BF16, d3, da, db, cta_group=3, tile_n=240)
    ce.device_status()
    assert torch.equal(d2, d3)
    rows = np.random.default_rng(3).choice(M, 16, replace=False)
    _check_bf16(O, d3.cpu().numpy()[rows], A[rows], B)
