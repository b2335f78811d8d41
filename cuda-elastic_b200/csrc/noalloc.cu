// rmsnorm -> bf16 tensor-core GEMM that allocates no device memory.
//
// The plan entry points (ce_plan_*) keep the GEMM's bf16 activation operand
// in a workspace that ce_plan_create allocates with cudaMalloc. Some callers
// cannot allocate: code that runs while a CUDA graph is being captured
// (cudaMalloc is not a stream operation, so a capture cannot record it),
// processes whose framework allocator has already reserved the device
// memory, and latency-critical loops that cannot afford cudaMalloc's
// implicit device synchronization. ce_rmsnorm_gemm_bf16_noalloc serves them:
// its operand lives in the file-scope array below, which the module holds on
// every GPU that loads the library until the process exits.
#include <mutex>

#include "common.cuh"

namespace ce {

int rows_iteration(float *normalized, uint16_t *normalized_bf16, int ld_bf16, const float *input,
                   const float *weight, float *softmax, const float *logits, float *product,
                   const float *matrix, const float *gemv_x, int batch_rms, int batch_softmax,
                   int cols, int gemv_rows, float eps, cudaStream_t s,
                   uint8_t *normalized_e4m3 = nullptr, int ld_e4m3 = 0, float *e4m3_scale = nullptr,
                   int norm_lo = 0, int norm_hi = 0x7fffffff, const RowsExtras *extras = nullptr);
int gemm_bf16(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
              int ldb, int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group = 0);

// 4,194,304 bf16 values (8 MiB): batch x roundup(size, 64) must fit, e.g.
// 256 x 16384 or 1024 x 4096.
constexpr size_t kNoAllocOperandElems = (size_t)4 << 20;
static __device__ __align__(256) uint16_t g_noalloc_operand[kNoAllocOperandElems];

namespace {

// In host code g_noalloc_operand names a host-side stand-in, not device
// memory; the device address is looked up once per device, with that device
// current, and cached for the life of the process (a cudaDeviceReset frees
// the array and leaves the cached address stale: the entry point must not be
// called on a device after it was reset).
int operand_address(uint16_t **out) {
  static std::mutex mu;
  static uint16_t *cached[64] = {};
  int dev = 0;
  CE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(CE_ERR_USAGE, format("device ordinal %d is out of range", dev));
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == nullptr) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_operand);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_operand)");
    cached[dev] = static_cast<uint16_t *>(p);
  }
  *out = cached[dev];
  return CE_OK;
}

}  // namespace
}  // namespace ce

using namespace ce;

extern "C" int ce_rmsnorm_gemm_bf16_noalloc(float *out, float *normalized, const float *x,
                                            const float *norm_w, const uint16_t *w_bf16, int ld_w,
                                            int batch, int size, int rows, float eps,
                                            ce_stream_t stream) {
  CE_REQUIRE(out && x && norm_w && w_bf16, "null argument");
  CE_REQUIRE(batch >= 1 && size >= 1 && rows >= 1, "batch, size and rows must be >= 1");
  CE_REQUIRE(ld_w >= size && ld_w % 8 == 0,
             "weight leading dimension must be >= size and a multiple of 8 (got %d)", ld_w);
  const int ld = ((size + 63) / 64) * 64;
  CE_REQUIRE((size_t)batch * (size_t)ld <= kNoAllocOperandElems,
             "batch x roundup(size, 64) = %zu bf16 values exceeds the fixed no-allocation "
             "operand of %zu values (8 MiB); use the ce_plan_* entry points",
             (size_t)batch * (size_t)ld, kNoAllocOperandElems);
  uint16_t *operand = nullptr;
  int rc = operand_address(&operand);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  // The GEMM reads only columns [0, size) of each operand row (its tensor
  // map's inner extent is size; TMA fills the rest of the last k-block with
  // zeros) and this rows launch rewrites all of them first, so nothing an
  // earlier call left in the array is read.
  rc = rows_iteration(normalized, operand, ld, x, norm_w, nullptr, nullptr, nullptr, nullptr,
                      nullptr, batch, 0, size, 0, eps, s);
  if (rc) return rc;
  return gemm_bf16(out, operand, w_bf16, batch, rows, size, ld, ld_w, rows, nullptr, nullptr, 0, s);
}
