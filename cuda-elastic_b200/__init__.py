"""cuda-elastic_b200: the B200-native llama2c hot path, host-side mirror.

The compute lives in libce_b200.so (hand-written sm_100a CUDA behind the C
ABI of include/ce_b200.h). This module binds that ABI with ctypes and
mirrors the reference's operator surface for the path:

  * the llama2c iteration (llama2c/llama2c_cuda_graph.cu): rmsnorm, softmax
    and the GEMV, with the same seeded inputs (llama2c_common.h:105-132);
  * the BASELINE op trio: rmsnorm -> tensor-core GEMM on the normalized
    batch, plus softmax, through a Plan (weights prepared once at setup).

PyTorch is used only for device memory and streams; tensors are passed to
the library as raw device pointers. There is no CPU fallback: if the
library is missing, importing or calling this module fails loudly.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libce_b200.so")

OK = 0
ERR_USAGE = 2
ERR_CUDA = 70
ERR_TIMEOUT = 71
ERR_NOMEM = 72

PREC_FP32 = 0
PREC_TF32 = 1
PREC_BF16 = 2
PREC_FP8_E4M3 = 3
PREC_MXFP6_E3M2 = 4
PREC_NVFP4_E2M1 = 5

RMS_EPS = 1.0e-5  # kRmsEpsilon, llama2c/llama2c_common.h:44
NCCL_ID_BYTES = 128  # CE_NCCL_ID_BYTES

_lib = None


class CeError(RuntimeError):
    """A non-zero status from libce_b200 (status in .status)."""

    def __init__(self, status, message):
        super().__init__(f"libce_b200 status {status}: {message}")
        self.status = status


def build(verbose=False):
    """Compiles libce_b200.so in place (nvcc, sm_100a)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_ce_b200_build", os.path.join(_HERE, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(verbose=verbose)


_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_u64 = ctypes.c_uint64
_i64 = ctypes.c_int64

# name -> argtypes (restype int unless listed in _RESTYPES)
_SIGNATURES = {
    "ce_version": [],
    "ce_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "ce_device_info": [ctypes.POINTER(_i), ctypes.POINTER(_i)],
    "ce_device_status": [],
    "ce_fill_llama2c_host": [_i, _u64, _i, _i, _i, _vp, _vp, _vp, _vp],
    "ce_fill_normal_host": [_u64, _u64, _i64, _i64, _f, _vp],
    "ce_fill_uniform_host": [_u64, _u64, _i64, _i64, _f, _f, _vp],
    "ce_rmsnorm": [_vp, _vp, _vp, _i, _i, _f, _vp],
    "ce_softmax": [_vp, _vp, _i, _i, _vp],
    "ce_gemv": [_vp, _vp, _vp, _i, _i, _vp],
    "ce_llama2c_iteration": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _vp],
    "ce_llama2c_rows": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp],
    "ce_gemm_bf16": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_gemm_bf16_tile": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp],
    "ce_gemm_tf32": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_gemm_tuning": [_i],
    "ce_gemm_wide_tiles": [_i],
    "ce_rows_tuning": [_i],
    "ce_gemm_config": [_i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp],
    "ce_gemm_fp32": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_convert_bf16": [_vp, _vp, _i, _i, _i, _vp],
    "ce_quantize_e4m3_rows": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ce_quantize_mxfp6": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ce_quantize_nvfp4": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp],
    "ce_sf_atom_bytes": [_i, _i, _i, _i, ctypes.POINTER(ctypes.c_size_t)],
    "ce_sf_to_atoms": [_i, _vp, _vp, _i, _i, _i, _vp],
    "ce_pack_mxfp6": [_vp, _vp, _i, _i, _i, _i, _vp],
    "ce_gemm_mxfp6": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_gemm_nvfp4": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_rmsnorm_e4m3": [_vp, _vp, _i, _vp, _vp, _vp, _i, _i, _f, _vp],
    "ce_gemm_e4m3": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_rmsnorm_bf16": [_vp, _vp, _i, _vp, _vp, _i, _i, _f, _vp],
    "ce_plan_create": [ctypes.POINTER(_vp), _i, _i, _i, _i],
    "ce_plan_destroy": [_vp],
    "ce_plan_set_weights": [_vp, _vp, _vp],
    "ce_plan_rmsnorm_gemm": [_vp, _vp, _vp, _vp, _vp, _f, _vp],
    "ce_plan_trio": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _vp],
    "ce_plan_rows": [_vp, _vp, _vp, _vp, _vp, _vp, _f, _vp],
    "ce_plan_gemm": [_vp, _vp, _vp],
    "ce_plan_operands": [_vp, _vp, _vp, _vp],
    "ce_decoder_validate": [_i64, _i64, _i64, _i64, _i],
    "ce_decoder_create": [ctypes.POINTER(_vp), _i64, _i64, _i64, _i64, _i, _vp],
    "ce_decoder_destroy": [_vp],
    "ce_decoder_set_model": [_vp, _vp, _vp, _vp, _vp],
    "ce_decoder_enqueue_compute": [_vp, _vp],
    "ce_decoder_enqueue_application": [_vp, _vp],
    "ce_decoder_poison": [_vp, _vp],
    "ce_decoder_copy_outputs": [_vp, _i, _vp, _vp, _vp, _vp],
    "ce_decoder_inject_fault": [_vp, _i],
    "ce_gemm_bf16_split": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i64, _vp],
    "ce_w4_pack": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "ce_gemm_w4a16": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp],
    "ce_w4t_packed_bytes": [_i, _i, ctypes.POINTER(ctypes.c_size_t)],
    "ce_w4t_pack": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "ce_gemm_w4t": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i64, _vp],
    "ce_llama_validate": [_vp, _i, _i, _i],
    "ce_llama_create": [ctypes.POINTER(_vp), _vp, _i, _i, _i, _vp],
    "ce_llama_destroy": [_vp],
    "ce_llama_init_random": [_vp, ctypes.c_uint64, _f, _i, _vp],
    "ce_llama_start": [_vp, _vp, _i, _vp],
    "ce_llama_enqueue_step": [_vp, _vp],
    "ce_llama_set_pdl": [_vp, _i],
    "ce_llama_read_nvfp4": [_vp, _i, _i, _vp, _vp, _vp],
    "ce_llama_validate_shard": [_vp, _i, _i, _i, _i, _i],
    "ce_llama_create_shard": [ctypes.POINTER(_vp), _vp, _i, _i, _i, _i, _i, _vp],
    "ce_llama_create_shard_ex": [ctypes.POINTER(_vp), _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_llama_bind_exchange": [_vp, _vp, _vp, _vp, _vp],
    "ce_llama_exchange_open": [_vp, _vp],
    "ce_llama_prefill_reserve": [_vp, _i],
    "ce_llama_set_prefill_attention": [_vp, _i],
    "ce_w4t_expand_f16": [_vp, _vp, _i, _i, _vp],
    "ce_gemm_f16": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ce_llama_load": [_vp, _i, _i, _vp],
    "ce_llama_load_nvfp4": [_vp, _i, _i, _vp, _vp, _vp],
    "ce_llama_enqueue_prefill": [_vp, _vp, _i, _vp],
    "ce_llama_set_sampling": [_vp, _f, _f, _u64],
    "ce_llama_exchange_connect": [_vp, ctypes.c_char_p],
    "ce_llama_enqueue_segment": [_vp, _i, _i, _vp],
    "ce_llama_shard_rows": [_vp, _i, _i, _i, _vp, _vp],
    "ce_llama_read": [_vp, _i, _i, _vp, _i64, _i64],
    "ce_llama_write": [_vp, _i, _i, _vp, _i64, _i64],
    "ce_llama_status": [],
    "ce_plan_gemm_ld": [_vp, _vp, _i, _vp],
    "ce_plan_rows_range": [_vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _vp],
    "ce_shard_bounds": [_i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)],
    "ce_set_wait_limit": [ctypes.c_double],
    "ce_nccl_version": [ctypes.POINTER(_i)],
    "ce_nccl_unique_id": [_vp],
    "ce_nccl_comm_init": [ctypes.POINTER(_vp), _i, _i, _vp],
    "ce_nccl_comm_destroy": [_vp],
    "ce_allgather_staging_floats": [_i, _i, _i, ctypes.POINTER(ctypes.c_size_t)],
    "ce_allgather_rows": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "ce_rowx_open": [ctypes.POINTER(_vp), _i, _i, _i, _i, _vp],
    "ce_rowx_connect": [_vp, ctypes.c_char_p],
    "ce_rowx_output": [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_i), ctypes.POINTER(_i)],
    "ce_plan_gemm_rowx": [_vp, _vp, _vp],
    "ce_rowx_wait": [_vp, _vp],
    "ce_rowx_put": [_vp, _vp],
    "ce_rowx_close": [_vp],
}
_RESTYPES = {"ce_version": ctypes.c_char_p}


def lib():
    """The loaded libce_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() "
                              "(the CUDA library is required; there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = L
    return _lib


def last_error():
    buf = ctypes.create_string_buffer(1024)
    code = lib().ce_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(status):
    if status != OK:
        raise CeError(status, last_error()[1])
    return status


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def device_status():
    """Synchronizes and raises CeError(ERR_TIMEOUT) if a device wait gave up."""
    return check(lib().ce_device_status())


def device_info():
    sms, sm100 = _i(), _i()
    check(lib().ce_device_info(ctypes.byref(sms), ctypes.byref(sm100)))
    return sms.value, bool(sm100.value)


# ---------------------------------------------------------------------------
# Host generators (the reference harness's fill_inputs and fixture normals)

def fill_llama2c_host(random, seed, batch, size, rows):
    """llama2c inputs (llama2c_common.h:105-132) as numpy float32 arrays:
    input [batch][size], probabilities [batch][size], weight [size],
    matrix [rows][size]."""
    x = np.empty((batch, size), np.float32)
    p = np.empty((batch, size), np.float32)
    w = np.empty(size, np.float32)
    m = np.empty((rows, size), np.float32)
    check(lib().ce_fill_llama2c_host(int(bool(random)), seed, batch, size, rows,
                                     _ptr(x), _ptr(p), _ptr(w), _ptr(m)))
    return x, p, w, m


def fill_normal_host(seed, stream, count, scale=1.0, first=0, out=None):
    out = np.empty(count, np.float32) if out is None else out
    check(lib().ce_fill_normal_host(seed, stream, first, count, scale, _ptr(out)))
    return out


def fill_uniform_host(seed, stream, count, lo, hi, first=0, out=None):
    out = np.empty(count, np.float32) if out is None else out
    check(lib().ce_fill_uniform_host(seed, stream, first, count, lo, hi, _ptr(out)))
    return out


def trio_inputs_host(seed, batch, size, rows):
    """BASELINE op-trio inputs: x ~ N(0,1) (stream 1), weight matrix
    W ~ N(0,1) * float(1/sqrt(size)) (stream 2), softmax logits ~ N(0,1)
    (stream 3), rmsnorm weight ~ U(0.5, 1.5) (stream 4), from the fixture
    generator of experiments/blackwell/lowprec/reference.cpp:172-209."""
    x = fill_normal_host(seed, 1, batch * size).reshape(batch, size)
    W = fill_normal_host(seed, 2, rows * size,
                         float(np.float32(1.0 / np.sqrt(size)))).reshape(rows, size)
    logits = fill_normal_host(seed, 3, batch * size).reshape(batch, size)
    w = fill_uniform_host(seed, 4, size, 0.5, 1.5)
    return x, w, logits, W


# ---------------------------------------------------------------------------
# Row operations (device tensors)

def rmsnorm(out, x, w, eps=RMS_EPS, stream=None):
    rows, cols = x.shape
    check(lib().ce_rmsnorm(_ptr(out), _ptr(x), _ptr(w), rows, cols, eps, _stream(stream)))
    return out


def rmsnorm_bf16(out, out_bf16, x, w, eps=RMS_EPS, stream=None):
    rows, cols = x.shape
    check(lib().ce_rmsnorm_bf16(_ptr(out), _ptr(out_bf16), out_bf16.shape[1], _ptr(x), _ptr(w),
                                rows, cols, eps, _stream(stream)))
    return out_bf16


def softmax(out, logits, stream=None):
    rows, cols = logits.shape
    check(lib().ce_softmax(_ptr(out), _ptr(logits), rows, cols, _stream(stream)))
    return out


def gemv(product, matrix, x, stream=None):
    rows, cols = matrix.shape
    check(lib().ce_gemv(_ptr(product), _ptr(matrix), _ptr(x), rows, cols, _stream(stream)))
    return product


def llama2c_iteration(normalized, softmax_out, product, inp, weight, probabilities, matrix,
                      eps=RMS_EPS, stream=None):
    """One llama2c iteration in one launch (rmsnorm + softmax + GEMV on the
    first `size` floats of the input)."""
    batch, size = inp.shape
    rows = matrix.shape[0]
    check(lib().ce_llama2c_iteration(_ptr(normalized), _ptr(softmax_out), _ptr(product), _ptr(inp),
                                     _ptr(weight), _ptr(probabilities), _ptr(matrix), batch, size,
                                     rows, eps, _stream(stream)))


def llama2c_rows(normalized, softmax_out, product, inp, weight, probabilities, matrix,
                 rms_rows, softmax_rows, matmul_rows, eps=RMS_EPS, stream=None):
    """Part of the llama2c iteration in one launch: rmsnorm of the first
    rms_rows input rows, softmax of the first softmax_rows probability rows,
    GEMV of the first matmul_rows matrix rows (any count may be 0; the
    SOTA harness's copy-mode split, llama2c_sota.cu:447-496)."""
    size = inp.shape[1]
    check(lib().ce_llama2c_rows(_ptr(normalized), _ptr(softmax_out), _ptr(product), _ptr(inp),
                                _ptr(weight), _ptr(probabilities), _ptr(matrix), size, rms_rows,
                                softmax_rows, matmul_rows, eps, _stream(stream)))


# ---------------------------------------------------------------------------
# GEMMs: d[m][n] = sum_k a[m][k] * b[n][k]

def gemm_bf16(d, a, b, k=None, tile_n=0, stream=None):
    """a, b: int16/uint16/bfloat16 tensors holding bf16 bits, K-contiguous."""
    M, lda = a.shape
    N, ldb = b.shape
    K = lda if k is None else k
    check(lib().ce_gemm_bf16_tile(_ptr(d), _ptr(a), _ptr(b), M, N, K, lda, ldb, d.shape[1], tile_n,
                                  _stream(stream)))
    return d


def gemm_bf16_split(d, a, b, splits, stream=None):
    """Split-K bf16 GEMM: d [splits][M][N] fp32 receives one partial per split
    (their sum is A B^T)."""
    M, lda = a.shape
    N, ldb = b.shape
    assert d.shape == (splits, M, N)
    check(lib().ce_gemm_bf16_split(_ptr(d), _ptr(a), _ptr(b), M, N, lda, lda, ldb, N, splits, M * N,
                                   _stream(stream)))
    return d


def w4_pack(codes_t, scales_t, codes, scales, n, k, stream=None):
    """NVFP4 weights (ce_quantize_nvfp4 layout) -> the W4A16 GEMM's k-block-major layout."""
    check(lib().ce_w4_pack(_ptr(codes_t), _ptr(scales_t), _ptr(codes), _ptr(scales), n, k,
                           codes.shape[1], scales.shape[1], _stream(stream)))


def gemm_w4a16(d, a, codes_t, scales_t, alpha=None, n=None, stream=None):
    """d [M][N] fp32 = alpha * A W^T, A fp16 bits [M][K], W packed by w4_pack."""
    M, K = a.shape
    N = d.shape[1] if n is None else n
    check(lib().ce_gemm_w4a16(_ptr(d), _ptr(a), _ptr(codes_t), _ptr(scales_t), _ptr(alpha), M, N, K, K,
                              d.shape[1], _stream(stream)))
    return d


def w4t_packed_bytes(n, k):
    """Bytes of ce_w4t_pack's layout for an n x k weight."""
    b = ctypes.c_size_t()
    check(lib().ce_w4t_packed_bytes(n, k, ctypes.byref(b)))
    return b.value


def w4t_pack(packed, codes, scales, n, k, stream=None):
    """NVFP4 weights (ce_quantize_nvfp4 layout) -> the decode-form W4A16 GEMM's packed layout."""
    check(lib().ce_w4t_pack(_ptr(packed), _ptr(codes), _ptr(scales), n, k, codes.shape[1], scales.shape[1],
                            _stream(stream)))


def w4t_unpack(packed, n, k):
    """The inverse of w4t_pack on the host: (codes uint8 [n][k/2], scales uint8 [n][k/16])."""
    kb, npad = (k + 127) // 128, (n + 255) // 256 * 256
    blocks = np.asarray(packed, np.uint8).reshape(kb, npad // 128, 9216)
    codes = blocks[:, :, :8192].reshape(kb, npad // 128, 4, 4, 32, 16)
    codes = codes.transpose(1, 2, 4, 0, 3, 5).reshape(npad, kb * 64)
    scales = blocks[:, :, 8192:].reshape(kb, npad // 128, 4, 32, 8).transpose(1, 2, 3, 0, 4).reshape(npad, kb * 8)
    return np.ascontiguousarray(codes[:n, :k // 2]), np.ascontiguousarray(scales[:n, :k // 16])


def gemm_w4t(d, a, packed, alpha=None, n=None, splits=1, stream=None):
    """d [M][N] fp32 = alpha * A W^T (decode form), A fp16 bits [M][K], W packed by w4t_pack;
    with splits > 1, d is [splits][M][N] partials."""
    M, K = a.shape
    N = d.shape[-1] if n is None else n
    check(lib().ce_gemm_w4t(_ptr(d), _ptr(a), _ptr(packed), _ptr(alpha), M, N, K, K, d.shape[-1], splits,
                            M * d.shape[-1], _stream(stream)))
    return d


def w4t_expand_f16(out, packed, n, k, stream=None):
    """W4T-packed weight [n][k] -> fp16 bits [n][k] (e2m1 x ue4m3, no decode scale)."""
    check(lib().ce_w4t_expand_f16(_ptr(out), _ptr(packed), n, k, _stream(stream)))
    return out


def gemm_f16(d, a, b, alpha=None, stream=None):
    """d [M][N] fp32 = alpha * A B^T, A [M][K] and B [N][K] fp16 bits (tensor cores)."""
    M, K = a.shape
    N = b.shape[0]
    check(lib().ce_gemm_f16(_ptr(d), _ptr(a), _ptr(b), _ptr(alpha), M, N, K, a.shape[1], b.shape[1], d.shape[1],
                            _stream(stream)))
    return d


def gemm_config(precision, d, a, b, k=None, cta_group=0, tile_n=0, stream=None):
    """Tensor-core GEMM with a forced kernel (cta_group 1 or 2) and tile width."""
    M, lda = a.shape
    N, ldb = b.shape
    K = lda if k is None else k
    check(lib().ce_gemm_config(precision, _ptr(d), _ptr(a), _ptr(b), M, N, K, lda, ldb, d.shape[1],
                               cta_group, tile_n, _stream(stream)))
    return d


def gemm_tf32(d, a, b, k=None, stream=None):
    M, lda = a.shape
    N, ldb = b.shape
    K = lda if k is None else k
    check(lib().ce_gemm_tf32(_ptr(d), _ptr(a), _ptr(b), M, N, K, lda, ldb, d.shape[1],
                             _stream(stream)))
    return d


def gemm_fp32(d, a, b, k=None, stream=None):
    M, lda = a.shape
    N, ldb = b.shape
    K = lda if k is None else k
    check(lib().ce_gemm_fp32(_ptr(d), _ptr(a), _ptr(b), M, N, K, lda, ldb, d.shape[1],
                             _stream(stream)))
    return d


def quantize_e4m3_rows(codes, scales, x, stream=None):
    """Per-row E4M3 quantization: codes uint8 [rows][ld], scales float32 [rows]."""
    rows, cols = x.shape
    check(lib().ce_quantize_e4m3_rows(_ptr(codes), _ptr(scales), _ptr(x), rows, cols, codes.shape[1],
                                      _stream(stream)))
    return codes, scales


def quantize_mxfp6(codes, scales, x, stream=None):
    """codes uint8 [rows][ld] (one per value), scales uint8 [rows][ceil(cols/32)]."""
    rows, cols = x.shape
    check(lib().ce_quantize_mxfp6(_ptr(codes), _ptr(scales), _ptr(x), rows, cols, codes.shape[1],
                                  _stream(stream)))
    return codes, scales


def quantize_nvfp4(codes, scales, tensor_scales, scratch, x, stream=None):
    """codes uint8 [rows][ld_bytes] (two per byte), scales uint8 [rows][ceil(cols/16)],
    tensor_scales float32 [2] (encode, decode), scratch int32 [1]."""
    rows, cols = x.shape
    check(lib().ce_quantize_nvfp4(_ptr(codes), _ptr(scales), _ptr(tensor_scales), _ptr(scratch),
                                  _ptr(x), rows, cols, codes.shape[1], _stream(stream)))
    return codes, scales


BS_TILE_N = 224


def sf_atoms(fmt, scales, rows, K, group_rows, stream=None):
    """Scale atoms (uint8 device tensor) of row-major scales [rows][K/vec]."""
    import torch
    n = ctypes.c_size_t()
    check(lib().ce_sf_atom_bytes(fmt, rows, K, group_rows, ctypes.byref(n)))
    atoms = torch.empty(n.value, dtype=torch.uint8, device=scales.device)
    check(lib().ce_sf_to_atoms(fmt, _ptr(atoms), _ptr(scales), rows, K, group_rows, _stream(stream)))
    return atoms


def pack_mxfp6(codes, stream=None):
    """GEMM operand layout of E3M2 codes [rows][cols] (uint8 device tensor)."""
    import torch
    rows, cols = codes.shape
    ld = ((cols + 15) // 16) * 16
    op = torch.empty((rows, ld), dtype=torch.uint8, device=codes.device)
    check(lib().ce_pack_mxfp6(_ptr(op), _ptr(codes), rows, cols, cols, ld, _stream(stream)))
    return op


def gemm_mxfp6(d, a, a_atoms, b, b_atoms, k=None, stream=None):
    M, lda = a.shape
    N, ldb = b.shape
    K = lda if k is None else k
    check(lib().ce_gemm_mxfp6(_ptr(d), _ptr(a), _ptr(a_atoms), _ptr(b), _ptr(b_atoms), M, N, K, lda,
                              ldb, d.shape[1], _stream(stream)))
    return d


def gemm_nvfp4(d, a, a_atoms, a_scales, b, b_atoms, b_scales, k, stream=None):
    M, lda = a.shape
    N, ldb = b.shape
    check(lib().ce_gemm_nvfp4(_ptr(d), _ptr(a), _ptr(a_atoms), _ptr(a_scales), _ptr(b), _ptr(b_atoms),
                              _ptr(b_scales), M, N, k, lda, ldb, d.shape[1], _stream(stream)))
    return d


def rmsnorm_e4m3(out, codes, scales, x, w, eps=RMS_EPS, stream=None):
    rows, cols = x.shape
    check(lib().ce_rmsnorm_e4m3(_ptr(out), _ptr(codes), codes.shape[1], _ptr(scales), _ptr(x),
                                _ptr(w), rows, cols, eps, _stream(stream)))
    return codes, scales


def gemm_e4m3(d, a, a_scale, b, b_scale, k=None, stream=None):
    M, lda = a.shape
    N, ldb = b.shape
    K = lda if k is None else k
    check(lib().ce_gemm_e4m3(_ptr(d), _ptr(a), _ptr(a_scale), _ptr(b), _ptr(b_scale), M, N, K, lda,
                             ldb, d.shape[1], _stream(stream)))
    return d


def convert_bf16(out, inp, stream=None):
    rows, cols = inp.shape
    check(lib().ce_convert_bf16(_ptr(out), _ptr(inp), rows, cols, out.shape[1], _stream(stream)))
    return out


class Plan:
    """Op-trio plan (rmsnorm -> GEMM on the normalized batch, + softmax) for
    one shape and precision. Weights are converted once by set_weights."""

    def __init__(self, batch, size, rows, precision=PREC_BF16):
        self.batch, self.size, self.n_rows, self.precision = batch, size, rows, precision
        h = ctypes.c_void_p()
        check(lib().ce_plan_create(ctypes.byref(h), batch, size, rows, precision))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().ce_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_weights(self, W, stream=None):
        check(lib().ce_plan_set_weights(self._h, _ptr(W), _stream(stream)))

    def rmsnorm_gemm(self, out, x, norm_w, normalized=None, eps=RMS_EPS, stream=None):
        check(lib().ce_plan_rmsnorm_gemm(self._h, _ptr(out), _ptr(normalized), _ptr(x),
                                         _ptr(norm_w), eps, _stream(stream)))
        return out

    def rows(self, normalized, softmax_out, x, norm_w, logits, eps=RMS_EPS, stream=None):
        check(lib().ce_plan_rows(self._h, _ptr(normalized), _ptr(softmax_out), _ptr(x),
                                 _ptr(norm_w), _ptr(logits), eps, _stream(stream)))

    def gemm(self, out, stream=None):
        check(lib().ce_plan_gemm(self._h, _ptr(out), _stream(stream)))
        return out

    def trio(self, normalized, softmax_out, out, x, norm_w, logits, eps=RMS_EPS, stream=None):
        check(lib().ce_plan_trio(self._h, _ptr(normalized), _ptr(softmax_out), _ptr(out), _ptr(x),
                                 _ptr(norm_w), _ptr(logits), eps, _stream(stream)))
        return out

    def operands(self, a=None, w=None, stream=None):
        """The GEMM operands as the tensor cores multiply them, as fp32:
        a [batch][size] (the latest rows stage), w [rows][size]."""
        check(lib().ce_plan_operands(self._h, _ptr(a), _ptr(w), _stream(stream)))
        return a, w

    def rows_range(self, normalized, softmax_out, x, norm_w, logits, row_lo, row_hi, eps=RMS_EPS,
                   stream=None):
        """Rows stage of one row-shard rank: the GEMM operand of every batch
        row, the fp32 normalized and softmax rows only for [row_lo, row_hi)."""
        check(lib().ce_plan_rows_range(self._h, _ptr(normalized), _ptr(softmax_out), _ptr(x), _ptr(norm_w),
                                       _ptr(logits), eps, row_lo, row_hi, _stream(stream)))

    def gemm_ld(self, out, ldd, stream=None):
        """The GEMM into out [batch][ldd] (ldd >= rows)."""
        check(lib().ce_plan_gemm_ld(self._h, _ptr(out), ldd, _stream(stream)))
        return out

    def gemm_rowx(self, rowx, stream=None):
        """This rank's slice GEMM, its tiles stored into every rank's
        exchange output (RowExchange)."""
        check(lib().ce_plan_gemm_rowx(self._h, rowx._h, _stream(stream)))


def set_wait_limit(seconds):
    """Limit of every bounded device wait launched afterwards on the
    current device (2 s by default)."""
    check(lib().ce_set_wait_limit(float(seconds)))


def shard_bounds(rows, world, rank):
    """[lo, hi) of rank's contiguous slice of `rows` (ce_shard_bounds)."""
    lo, hi = _i(), _i()
    check(lib().ce_shard_bounds(rows, world, rank, ctypes.byref(lo), ctypes.byref(hi)))
    return lo.value, hi.value


class _DeviceArray:
    """A library-owned device buffer as a CUDA array (for torch.as_tensor)."""

    def __init__(self, ptr, shape, typestr="<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class RowExchange:
    """Peer-memory join of the row-shard GEMM (ce_rowx_*): this rank's
    out [batch][rows] in device memory shared by CUDA IPC. open() returns the
    IPC handle; gather every rank's handle in rank order and call connect()."""

    def __init__(self, batch, rows, world, rank):
        self.batch, self.rows, self.world, self.rank = batch, rows, world, rank
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(lib().ce_rowx_open(ctypes.byref(h), batch, rows, world, rank, buf))
        self._h = h
        self.handle = buf.raw
        p, lo, hi = ctypes.c_void_p(), _i(), _i()
        check(lib().ce_rowx_output(h, ctypes.byref(p), ctypes.byref(lo), ctypes.byref(hi)))
        self.lo, self.hi = lo.value, hi.value
        import torch
        self.output = torch.as_tensor(_DeviceArray(p.value, (batch, rows)), device="cuda")

    def connect(self, handles):
        check(lib().ce_rowx_connect(self._h, b"".join(handles)))

    def wait(self, stream=None):
        check(lib().ce_rowx_wait(self._h, _stream(stream)))

    def put(self, stream=None):
        """Copies this rank's slice of output into every peer's (copy engines)."""
        check(lib().ce_rowx_put(self._h, _stream(stream)))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self.output = None
            lib().ce_rowx_close(self._h)
            self._h = None


class NcclComm:
    """An NCCL communicator made through the library (ce_nccl_*); `uid` is
    the CE_NCCL_ID_BYTES that rank 0 got from nccl_unique_id()."""

    def __init__(self, world, rank, uid):
        h = ctypes.c_void_p()
        check(lib().ce_nccl_comm_init(ctypes.byref(h), world, rank, uid))
        self._h, self.world, self.rank = h, world, rank

    @property
    def handle(self):
        return self._h.value

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().ce_nccl_comm_destroy(self._h)
            self._h = None


def nccl_unique_id():
    buf = ctypes.create_string_buffer(NCCL_ID_BYTES)
    check(lib().ce_nccl_unique_id(buf))
    return buf.raw


def nccl_version():
    v = _i()
    check(lib().ce_nccl_version(ctypes.byref(v)))
    return v.value


def allgather_staging_floats(batch, rows, world):
    n = ctypes.c_size_t()
    check(lib().ce_allgather_staging_floats(batch, rows, world, ctypes.byref(n)))
    return n.value


def allgather_rows(comm, out, staging, batch, rows, world, rank, stream=None):
    """NCCL join of the row-shard slices (ce_allgather_rows)."""
    check(lib().ce_allgather_rows(comm.handle if isinstance(comm, NcclComm) else comm, _ptr(out), _ptr(staging),
                                  batch, rows, world, rank, _stream(stream)))
    return out


class Decoder:
    """The loom_private llama2c decoder workload (B sequences x S greedy steps
    on the synthetic model, or on caller weights). Mirrors lp::Workload:
    setup at construction, enqueue_compute / enqueue_application (both
    capturable), poison_outputs, and outputs() as the check's diagnostics
    copy."""

    def __init__(self, batch, width, vocab, steps, precision=PREC_FP32, stream=None):
        self.batch, self.width, self.vocab, self.steps = batch, width, vocab, steps
        self.precision = precision
        h = ctypes.c_void_p()
        check(lib().ce_decoder_create(ctypes.byref(h), batch, width, vocab, steps, precision,
                                      _stream(stream)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().ce_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_model(self, embedding, classifier, norm_w, stream=None):
        check(lib().ce_decoder_set_model(self._h, _ptr(embedding), _ptr(classifier), _ptr(norm_w),
                                         _stream(stream)))

    def enqueue_compute(self, stream=None):
        check(lib().ce_decoder_enqueue_compute(self._h, _stream(stream)))

    def enqueue_application(self, stream=None):
        check(lib().ce_decoder_enqueue_application(self._h, _stream(stream)))

    def poison_outputs(self, stream=None):
        check(lib().ce_decoder_poison(self._h, _stream(stream)))

    def inject_fault(self, fault):
        check(lib().ce_decoder_inject_fault(self._h, fault))

    def outputs(self, from_device=False, which=("generated", "normalized", "logits", "probabilities")):
        """Host copies: generated [B][S] int32, normalized [S][B][W],
        logits and probabilities [S][B][V] float32."""
        B, W, V, S = self.batch, self.width, self.vocab, self.steps
        g = np.empty((B, S), np.int32) if "generated" in which else None
        n = np.empty((S, B, W), np.float32) if "normalized" in which else None
        lg = np.empty((S, B, V), np.float32) if "logits" in which else None
        p = np.empty((S, B, V), np.float32) if "probabilities" in which else None
        check(lib().ce_decoder_copy_outputs(self._h, int(bool(from_device)), _ptr(g), _ptr(n),
                                            _ptr(lg), _ptr(p)))
        return g, n, lg, p


# --------------------------------------------------------------------------
# Llama-2 decoder step (ce_llama_*)

LLAMA_TOK_EMB, LLAMA_WQKV, LLAMA_WO, LLAMA_W13, LLAMA_W2 = 0, 1, 2, 3, 4
LLAMA_RMS_ATT, LLAMA_RMS_FFN, LLAMA_RMS_FINAL, LLAMA_WCLS = 5, 6, 7, 8
LLAMA_KCACHE, LLAMA_VCACHE, LLAMA_LOGITS, LLAMA_TOKENS = 9, 10, 11, 12
LLAMA_GENERATED, LLAMA_POS, LLAMA_RESIDUAL = 13, 14, 15
IPC_HANDLE_BYTES = 64  # CE_IPC_HANDLE_BYTES
SEG_ATTN, SEG_OPROJ, SEG_FFN_IN, SEG_FFN_OUT, SEG_HEAD, SEG_PICK = 0, 1, 2, 3, 4, 5
LLAMA_REPRODUCIBLE_SPLITS = 1  # CE_LLAMA_REPRODUCIBLE_SPLITS


class LlamaConfig(ctypes.Structure):
    """llama2.c's Config (dim, hidden_dim, n_layers, n_heads, n_kv_heads,
    vocab_size, seq_len)."""
    _fields_ = [(n, ctypes.c_int32) for n in
                ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "seq_len")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


def llama_config(**kw):
    c = LlamaConfig()
    kw.setdefault("n_kv_heads", kw.get("n_heads"))
    for n, _ in LlamaConfig._fields_:
        setattr(c, n, int(kw[n]))
    return c


class Llama:
    """Batched greedy decoding of a Llama-2 transformer on one GPU: weights,
    KV cache and buffers live in the library; step() enqueues one decode step
    for every sequence (capturable; position and step counters are on the
    device, so a captured step replays for every token)."""

    def __init__(self, cfg, batch, max_steps, precision=PREC_BF16, stream=None, rank=0, world=1, flags=0):
        self.cfg = cfg if isinstance(cfg, LlamaConfig) else llama_config(**cfg)
        self.batch, self.max_steps, self.precision = batch, max_steps, precision
        self.rank, self.world = rank, world
        self.hs = self.cfg.dim // self.cfg.n_heads
        self.kv_dim = self.hs * self.cfg.n_kv_heads // world  # this shard's k (and v) rows
        h = ctypes.c_void_p()
        check(lib().ce_llama_create_shard_ex(ctypes.byref(h), ctypes.byref(self.cfg), batch, max_steps,
                                             precision, rank, world, flags, _stream(stream)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().ce_llama_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_random(self, seed=0, weight_std=0.02, kv_fill=0, stream=None):
        check(lib().ce_llama_init_random(self._h, seed, weight_std, kv_fill, _stream(stream)))

    def start(self, tokens, pos, stream=None):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        assert t.shape == (self.batch,)
        check(lib().ce_llama_start(self._h, t.ctypes.data, pos, _stream(stream)))

    def step(self, stream=None):
        check(lib().ce_llama_enqueue_step(self._h, _stream(stream)))

    def prefill_reserve(self, max_rows):
        """Allocates the prefill chunk workspace (max_rows = batch x positions per chunk)."""
        check(lib().ce_llama_prefill_reserve(self._h, max_rows))

    def set_prefill_attention(self, simt):
        """Prefill attention on the SIMT kernel (True) or the tensor cores (False, default)."""
        check(lib().ce_llama_set_prefill_attention(self._h, int(bool(simt))))

    def prefill(self, prompt, stream=None):
        """Enqueues the prefill of prompt (device int32 [batch][prompt_len])
        at the current position; the next token is chosen from the last
        prompt position, as a step would."""
        import torch
        assert prompt.dtype == torch.int32 and prompt.is_contiguous() and prompt.shape[0] == self.batch
        check(lib().ce_llama_enqueue_prefill(self._h, _ptr(prompt), prompt.shape[1], _stream(stream)))

    def set_pdl(self, enable):
        check(lib().ce_llama_set_pdl(self._h, int(bool(enable))))

    def load_llama2c(self, path):
        """Loads a llama2.c fp32 checkpoint whose config matches this model's:
        bf16 models convert on the device, NVFP4 models quantize every GEMM
        weight on the device at load (ce_llama_load)."""
        from . import convert_weights as cw
        cfg, t, _ = cw.read_llama2c(path)
        self._check_config(cfg)
        L = self.cfg.n_layers

        def load(which, layer, a):
            a = np.ascontiguousarray(a, dtype=np.float32)
            check(lib().ce_llama_load(self._h, which, layer, a.ctypes.data))

        load(LLAMA_TOK_EMB, 0, t["tok_emb"])
        for l in range(L):
            load(LLAMA_RMS_ATT, l, t["rms_att"][l])
            load(LLAMA_RMS_FFN, l, t["rms_ffn"][l])
            for name, which in (("wqkv", LLAMA_WQKV), ("wo", LLAMA_WO), ("w13", LLAMA_W13), ("w2", LLAMA_W2)):
                load(which, l, cw.model_matrix(t, name, l))
        load(LLAMA_RMS_FINAL, 0, t["rms_final"])
        load(LLAMA_WCLS, 0, cw.model_matrix(t, "wcls", 0))

    def load_nvfp4_file(self, path):
        """Loads the output of convert_weights (weights quantized ahead of
        time) into an NVFP4 model (ce_llama_load_nvfp4); no quantization at
        load."""
        from . import convert_weights as cw
        cfg, emb, norms, mats = cw.read_nvfp4_file(path)
        self._check_config(cfg)
        self.write(LLAMA_TOK_EMB, np.ascontiguousarray(emb))
        rms_att, rms_ffn, rms_final = norms
        for l in range(self.cfg.n_layers):
            self.write(LLAMA_RMS_ATT, np.ascontiguousarray(rms_att[l]), l)
            self.write(LLAMA_RMS_FFN, np.ascontiguousarray(rms_ffn[l]), l)
        self.write(LLAMA_RMS_FINAL, np.ascontiguousarray(rms_final))
        which = {"wqkv": LLAMA_WQKV, "wo": LLAMA_WO, "w13": LLAMA_W13, "w2": LLAMA_W2, "wcls": LLAMA_WCLS}
        for name, layer, alpha, codes, scales in mats:
            a, c, sc = (np.ascontiguousarray(x) for x in (alpha, codes, scales))
            check(lib().ce_llama_load_nvfp4(self._h, which[name], layer, c.ctypes.data, sc.ctypes.data,
                                            a.ctypes.data))

    def _check_config(self, cfg):
        mine = {k: getattr(self.cfg, k) for k in cfg}
        if mine != cfg:
            raise ValueError(f"checkpoint config {cfg} does not match the model's {mine}")

    def read(self, which, layer=0, dtype=np.uint16, count=None, offset=0):
        """Host copy of `count` elements of a tensor from element `offset`."""
        item = np.dtype(dtype).itemsize
        if count is None:
            count = self._size(which) // item - offset
        out = np.empty(count, dtype)
        check(lib().ce_llama_read(self._h, which, layer, out.ctypes.data, offset * item, count * item))
        return out

    def write(self, which, array, layer=0, offset=0):
        a = np.ascontiguousarray(array)
        check(lib().ce_llama_write(self._h, which, layer, a.ctypes.data, offset * a.itemsize, a.nbytes))

    def _size(self, which):
        c, B, n = self.cfg, self.batch, self.world
        kvh = c.n_kv_heads // n
        sizes = {LLAMA_TOK_EMB: c.vocab_size * c.dim * 2, LLAMA_RMS_ATT: c.dim * 4, LLAMA_RMS_FFN: c.dim * 4,
                 LLAMA_RMS_FINAL: c.dim * 4,
                 LLAMA_KCACHE: B * kvh * c.seq_len * self.hs * 2,
                 LLAMA_VCACHE: B * kvh * c.seq_len * self.hs * 2,
                 LLAMA_LOGITS: B * (c.vocab_size // n) * 4, LLAMA_TOKENS: B * 4,
                 LLAMA_GENERATED: B * self.max_steps * 4, LLAMA_POS: 4, LLAMA_RESIDUAL: B * c.dim * 4}
        if which in (LLAMA_WQKV, LLAMA_WO, LLAMA_W13, LLAMA_W2, LLAMA_WCLS):
            r, k = self._shape(which)
            return r * k * 2
        return sizes[which]

    def generated(self):
        return self.read(LLAMA_GENERATED, dtype=np.int32).reshape(self.batch, self.max_steps)

    def logits(self):
        """This shard's logits [batch][vocab_size / world]."""
        return self.read(LLAMA_LOGITS, dtype=np.float32).reshape(self.batch, self.cfg.vocab_size // self.world)

    def cache_rows(self, layer, seq, which=LLAMA_KCACHE, positions=None):
        """bf16 bits [kv_heads][positions][hs] of one sequence's cache (this shard's heads)."""
        c = self.cfg
        n = c.seq_len if positions is None else positions
        per_head = c.seq_len * self.hs
        kvh = c.n_kv_heads // self.world
        out = np.empty((kvh, n, self.hs), np.uint16)
        for kh in range(kvh):
            off = (seq * kvh + kh) * per_head
            out[kh] = self.read(which, layer, np.uint16, n * self.hs, off).reshape(n, self.hs)
        return out

    def nvfp4_weight(self, which, layer=0):
        """NVFP4 model: (codes uint8 [rows][cols / 2] two per byte, even index
        in the low nibble; UE4M3 scales uint8 [rows][cols / 16]; decode scale)
        of one weight matrix, un-packed from the decode-form W4A16 layout
        (ce_w4t_pack)."""
        rows, cols = self._shape(which)
        packed = np.empty(w4t_packed_bytes(rows, cols), np.uint8)
        alpha = np.empty(2, np.float32)
        check(lib().ce_llama_read_nvfp4(self._h, which, layer, packed.ctypes.data, None, alpha.ctypes.data))
        codes, scales = w4t_unpack(packed, rows, cols)
        return codes, scales, float(alpha[1])

    def _shape(self, which):
        c, n = self.cfg, self.world
        return {LLAMA_WQKV: (c.dim // n + 2 * self.kv_dim, c.dim), LLAMA_WO: (c.dim // n, c.dim),
                LLAMA_W13: (2 * c.hidden_dim // n, c.dim), LLAMA_W2: (c.dim // n, c.hidden_dim),
                LLAMA_WCLS: (c.vocab_size // n, c.dim)}[which]

    def segment(self, seg, layer=0, stream=None):
        check(lib().ce_llama_enqueue_segment(self._h, seg, layer, _stream(stream)))

    def bind_exchange(self, att, delta, hb, top):
        check(lib().ce_llama_bind_exchange(self._h, _ptr(att), _ptr(delta), _ptr(hb), _ptr(top)))

    def set_sampling(self, temperature=0.0, top_p=0.0, seed=0):
        """Greedy (temperature 0) or sampled token choice for later steps (ce_llama_set_sampling)."""
        check(lib().ce_llama_set_sampling(self._h, float(temperature), float(top_p), int(seed)))

    def exchange_open(self):
        """Allocates this rank's peer-exchange block; returns its CUDA IPC handle (bytes)."""
        h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(lib().ce_llama_exchange_open(self._h, h))
        return h.raw

    def exchange_connect(self, handles):
        """Maps every rank's exchange block (handles: all ranks' handles concatenated in rank order)."""
        if len(handles) != IPC_HANDLE_BYTES * self.world:
            raise ValueError("need one IPC handle per rank")
        check(lib().ce_llama_exchange_connect(self._h, handles))

    def weights(self):
        """Every weight as host arrays: bf16 bits (uint16) for a bf16 model,
        (codes, scales, decode scale) tuples from nvfp4_weight for the GEMM
        weights of an NVFP4 model; the embedding is bf16 bits and the RMSNorm
        weights fp32 either way."""
        c = self.cfg
        nv = self.precision == PREC_NVFP4_E2M1
        w = {"tok_emb": self.read(LLAMA_TOK_EMB).reshape(c.vocab_size, c.dim),
             "wcls": self.nvfp4_weight(LLAMA_WCLS) if nv else self.read(LLAMA_WCLS).reshape(c.vocab_size, c.dim),
             "rms_final": self.read(LLAMA_RMS_FINAL, dtype=np.float32)}
        for key, which in (("wqkv", LLAMA_WQKV), ("wo", LLAMA_WO), ("w13", LLAMA_W13), ("w2", LLAMA_W2)):
            shape = self._shape(which)
            w[key] = [self.nvfp4_weight(which, l) if nv else self.read(which, l).reshape(shape)
                      for l in range(c.n_layers)]
        w["rms_att"] = [self.read(LLAMA_RMS_ATT, l, np.float32) for l in range(c.n_layers)]
        w["rms_ffn"] = [self.read(LLAMA_RMS_FFN, l, np.float32) for l in range(c.n_layers)]
        return w


def llama_status():
    """Reads and clears the decode kernels' status (raises on a failure)."""
    check(lib().ce_llama_status())


def llama_shard_rows(cfg, rank, world, which):
    """Global rows of rank's rows of a sharded weight (no CUDA call)."""
    c = cfg if isinstance(cfg, LlamaConfig) else llama_config(**cfg)
    n = ctypes.c_int()
    check(lib().ce_llama_shard_rows(ctypes.byref(c), rank, world, which, None, ctypes.byref(n)))
    out = np.empty(n.value, np.int32)
    check(lib().ce_llama_shard_rows(ctypes.byref(c), rank, world, which, out.ctypes.data, ctypes.byref(n)))
    return out
