// extern "C" entry points of libce_b200.so (declared in include/ce_b200.h),
// the host-side seeded input generators, and the op-trio plan.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace ce {

// ---- kernels defined in the other translation units ----
int rows_iteration(float *normalized, uint16_t *normalized_bf16, int ld_bf16, const float *input,
                   const float *weight, float *softmax, const float *logits, float *product,
                   const float *matrix, const float *gemv_x, int batch_rms, int batch_softmax,
                   int cols, int gemv_rows, float eps, cudaStream_t s,
                   uint8_t *normalized_e4m3 = nullptr, int ld_e4m3 = 0, float *e4m3_scale = nullptr,
                   int norm_lo = 0, int norm_hi = 0x7fffffff, const RowsExtras *extras = nullptr);
int convert_bf16(uint16_t *out, const float *in, int rows, int cols, int ld, cudaStream_t s);
size_t w4t_packed_bytes(int N, int K);
int w4t_expand_f16(uint16_t *out, const uint8_t *packed, int N, int K, cudaStream_t s);
int gemm_f16(float *d, const uint16_t *a, const uint16_t *b, const float *alpha, int M, int N, int K, int lda,
             int ldb, int ldd, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl);
int w4t_pack(uint8_t *packed, const uint8_t *codes, const uint8_t *scales, int N, int K, int ld_bytes, int nsf,
             cudaStream_t s, const int *row_map);
int gemm_w4t(float *d, const uint16_t *a, const uint8_t *packed, const float *alpha, int M, int N, int K, int lda,
             int ldd, int splits, long long split_stride, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl,
             const ExchangeWait *xw = nullptr);
int gemm_bf16(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
              int ldb, int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group = 0);
int gemm_tf32(float *d, const float *a, const float *b, int M, int N, int K, int lda, int ldb,
              int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group = 0);
int gemm_simt_fp32(float *d, const float *a, const float *b, int M, int N, int K, int lda,
                   int ldb, int ldd, cudaStream_t s);
int gemm_bf16_split(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
                    int ldb, int ldd, int splits, long long split_stride, cudaStream_t s, bool pdl);
int gemm_w4a16(float *d, const uint16_t *a, const uint8_t *codes_t, const uint8_t *scales_t,
               const float *alpha, int M, int N, int K, int lda, int ldd, int splits,
               long long split_stride, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl);
int w4_pack(uint8_t *codes_t, uint8_t *scales_t, const uint8_t *codes, const uint8_t *scales, int N, int K,
            int ld_bytes, int nsf, cudaStream_t s, const int *row_map = nullptr);
int gemm_status();
int gemm_bs_status();
int rowx_status();
int rows_status();
int rows_set_wait_limit(unsigned long long ns);
int rows_set_streaming(int on);
int gemm_set_wait_limit(unsigned long long ns);
int gemm_bs_set_wait_limit(unsigned long long ns);
int llama_set_wait_limit(unsigned long long ns);
int rowx_set_wait_limit(unsigned long long ns);
int rowx_sync(const ce_rowx *x, RowxSync *rx, float **out, int *lo, int *hi, int *batch, int *rows);
int x_device_of(const ce_rowx *x);
int gemm_rowx(int kind, float *d, const void *a, const void *b, int M, int N, int K, int lda, int ldb,
              int ldd, const float *row_scale, const float *col_scale, const RowxSync &rx, cudaStream_t s);
int pack_mxfp6(uint8_t *operand, const uint8_t *codes, int rows, int cols, int ld_codes,
               int ld_operand, cudaStream_t s);
int sf_katoms(int fmt, int K);
int sf_row_atoms(int rows, int group_rows);
int sf_to_atoms(uint8_t *atoms, const uint8_t *scales, int rows, int nsf, int katoms,
                int group_rows, cudaStream_t s);
int gemm_mxfp6(float *d, const uint8_t *a, const uint8_t *sfa, const uint8_t *b,
               const uint8_t *sfb, int M, int N, int K, int lda, int ldb, int ldd, cudaStream_t s);
int gemm_nvfp4(float *d, const uint8_t *a, const uint8_t *sfa, const float *alpha_a,
               const uint8_t *b, const uint8_t *sfb, const float *alpha_b, int M, int N, int K,
               int lda_bytes, int ldb_bytes, int ldd, cudaStream_t s);
int gemm_e4m3(float *d, const uint8_t *a, const uint8_t *b, int M, int N, int K, int lda,
              int ldb, int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group = 0);
int quantize_rows_e4m3(uint8_t *codes, float *scales, const float *x, int rows, int cols, int ld,
                       cudaStream_t s);
int quantize_mxfp6(uint8_t *codes, uint8_t *scales, const float *x, int rows, int cols,
                   int ld_codes, cudaStream_t s);
int quantize_nvfp4(uint8_t *codes, uint8_t *scales, float *encode_decode, unsigned int *amax_bits,
                   const float *x, int rows, int cols, int ld_bytes, cudaStream_t s);
int gemm_set_prefetch(int kblocks);
int quantize_nvfp4_atoms(uint8_t *codes, uint8_t *atoms, float *encode_decode, const unsigned int *amax_bits,
                         const float *x, int rows, int cols, int ld_bytes, int katoms, cudaStream_t s);
int gemm_set_wide_tiles(int on);

// ---------------------------------------------------------------------------
// Status

namespace {
thread_local int t_last_code = CE_OK;
thread_local std::string t_last_msg;
}  // namespace

int set_error(int code, const std::string &msg) {
  t_last_code = code;
  t_last_msg = msg;
  return code;
}

int cuda_error(cudaError_t err, const char *what) {
  return set_error(err == cudaErrorMemoryAllocation ? CE_ERR_NOMEM : CE_ERR_CUDA,
                   format("%s failed: %s", what, cudaGetErrorString(err)));
}

std::string format(const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return std::string(buf);
}

namespace {
struct DeviceProps {
  int sms = 0;
  int major = 0;
};
DeviceProps props_of_current() {
  static std::mutex mu;
  static DeviceProps cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return {};
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].sms == 0) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
  }
  return cache[dev];
}
}  // namespace

int sm_count() {
  const int n = props_of_current().sms;
  return n > 0 ? n : 148;
}
bool is_sm100() { return props_of_current().major == 10; }

// ---------------------------------------------------------------------------
// Seeded generators (host)

namespace {

inline uint64_t splitmix_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
// llama2c counter generator: mix(x) = splitmix64 finaliser of x + golden.
inline uint64_t llama2c_mix(uint64_t x) { return splitmix_mix(x + 0x9e3779b97f4a7c15ull); }
inline float llama2c_uniform(uint64_t seed, uint64_t stream, uint64_t index) {
  const uint64_t bits = llama2c_mix(llama2c_mix(seed * 4 + stream) ^ index);
  return (float)(int64_t)(bits >> 40) * (1.0f / 8388608.0f) - 1.0f;
}
// Output number k (1-based) of the sequential splitmix64 generator seeded
// with `state`: the state advances by the golden increment per call, so any
// output can be computed directly.
inline uint64_t splitmix_nth(uint64_t state, uint64_t k) {
  return splitmix_mix(state + k * 0x9e3779b97f4a7c15ull);
}
inline double unit_of(uint64_t x) { return (double)(x >> 11) * 0x1.0p-53; }

template <class F>
void parallel_for(int64_t n, F &&body) {
  unsigned hw = std::thread::hardware_concurrency();
  int64_t threads = hw == 0 ? 1 : (int64_t)hw;
  if (n < (1 << 16)) threads = 1;
  if (threads > n) threads = n > 0 ? n : 1;
  if (threads <= 1) {
    body(0, n);
    return;
  }
  std::vector<std::thread> pool;
  const int64_t chunk = (n + threads - 1) / threads;
  for (int64_t t = 0; t < threads; ++t) {
    const int64_t lo = t * chunk, hi = std::min<int64_t>(n, lo + chunk);
    if (lo >= hi) break;
    pool.emplace_back([&body, lo, hi] { body(lo, hi); });
  }
  for (auto &th : pool) th.join();
}

}  // namespace
}  // namespace ce

using namespace ce;

// ---------------------------------------------------------------------------
// C ABI

extern "C" {

const char *ce_version(void) { return "ce_b200 0.1"; }

int ce_last_error(char *buf, size_t len) {
  if (buf != nullptr && len > 0) {
    std::strncpy(buf, t_last_msg.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return t_last_code;
}

int ce_device_info(int *sms, int *sm100) {
  int dev = 0;
  CE_CUDA_TRY(cudaGetDevice(&dev));
  if (sms) *sms = sm_count();
  if (sm100) *sm100 = is_sm100() ? 1 : 0;
  return CE_OK;
}

// Synchronizes the device and returns CE_ERR_TIMEOUT if a bounded device
// wait of a tensor-core kernel gave up since the last call (clearing it).
int ce_device_status(void) {
  const int a = gemm_status();
  const int b = gemm_bs_status();
  const int c = rowx_status();
  const int d = rows_status();
  return a != CE_OK ? a : b != CE_OK ? b : c != CE_OK ? c : d;
}

int ce_set_wait_limit(double seconds) {
  CE_REQUIRE(seconds >= 1e-3 && seconds <= 3600.0, "wait limit must be in [0.001, 3600] s (got %g)", seconds);
  const unsigned long long ns = (unsigned long long)(seconds * 1e9);
  for (int (*set)(unsigned long long) :
       {gemm_set_wait_limit, gemm_bs_set_wait_limit, llama_set_wait_limit, rowx_set_wait_limit,
        rows_set_wait_limit}) {
    const int rc = set(ns);
    if (rc != CE_OK) return set_error(rc, "cudaMemcpyToSymbol(wait limit) failed");
  }
  return CE_OK;
}

int ce_fill_llama2c_host(int random, uint64_t seed, int batch, int size, int rows, float *input,
                         float *probabilities, float *weight, float *matrix) {
  CE_REQUIRE(batch >= 1 && size >= 1 && rows >= 1, "batch, size and rows must be >= 1");
  const int64_t vec = (int64_t)batch * size, mat = (int64_t)rows * size;
  if (!random) {
    parallel_for(vec, [&](int64_t lo, int64_t hi) {
      for (int64_t i = lo; i < hi; ++i) {
        const float v = 1.0f + (float)(i % 4);
        if (input) input[i] = v;
        if (probabilities) probabilities[i] = v;
      }
    });
    if (weight)
      for (int i = 0; i < size; ++i) weight[i] = 1.0f;
    if (matrix)
      parallel_for(mat, [&](int64_t lo, int64_t hi) {
        for (int64_t i = lo; i < hi; ++i) {
          const int64_t r = i / size, c = i % size;
          matrix[i] = c == (r % size) ? 1.0f : 0.0f;
        }
      });
    return CE_OK;
  }
  parallel_for(vec, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      if (input) input[i] = llama2c_uniform(seed, 0, (uint64_t)i);
      if (probabilities) probabilities[i] = llama2c_uniform(seed, 1, (uint64_t)i);
    }
  });
  if (weight)
    for (int i = 0; i < size; ++i) weight[i] = llama2c_uniform(seed, 2, (uint64_t)i);
  if (matrix)
    parallel_for(mat, [&](int64_t lo, int64_t hi) {
      for (int64_t i = lo; i < hi; ++i) matrix[i] = llama2c_uniform(seed, 3, (uint64_t)i);
    });
  return CE_OK;
}

int ce_fill_normal_host(uint64_t seed, uint64_t stream, int64_t first, int64_t count, float scale,
                        float *out) {
  CE_REQUIRE(first >= 0 && count >= 0 && out != nullptr, "bad normal fill range");
  const uint64_t state = seed * 0x100000001b3ull + stream;
  const double two_pi = 6.283185307179586476925286766559;
  parallel_for(count, [&](int64_t lo, int64_t hi) {
    for (int64_t j = lo; j < hi; ++j) {
      const int64_t i = first + j, pair = i / 2;
      const double u1 = unit_of(splitmix_nth(state, (uint64_t)(2 * pair + 1)));
      const double u2 = unit_of(splitmix_nth(state, (uint64_t)(2 * pair + 2)));
      const double radius = std::sqrt(-2.0 * std::log(1.0 - u1));
      const double v = (i & 1) ? radius * std::sin(two_pi * u2) : radius * std::cos(two_pi * u2);
      out[j] = (float)v * scale;
    }
  });
  return CE_OK;
}

int ce_fill_uniform_host(uint64_t seed, uint64_t stream, int64_t first, int64_t count, float lo_v,
                         float hi_v, float *out) {
  CE_REQUIRE(first >= 0 && count >= 0 && out != nullptr, "bad uniform fill range");
  const uint64_t state = seed * 0x100000001b3ull + stream;
  parallel_for(count, [&](int64_t lo, int64_t hi) {
    for (int64_t j = lo; j < hi; ++j) {
      const double u = unit_of(splitmix_nth(state, (uint64_t)(first + j + 1)));
      out[j] = (float)((double)lo_v + ((double)hi_v - (double)lo_v) * u);
    }
  });
  return CE_OK;
}

int ce_rmsnorm(float *out, const float *x, const float *w, int rows, int cols, float eps,
               ce_stream_t stream) {
  CE_REQUIRE(rows >= 1 && cols >= 1, "rows and cols must be >= 1 (got %d, %d)", rows, cols);
  return rows_iteration(out, nullptr, 0, x, w, nullptr, nullptr, nullptr, nullptr, nullptr, rows,
                        0, cols, 0, eps, (cudaStream_t)stream);
}

int ce_rmsnorm_bf16(float *out, uint16_t *out_bf16, int ld_bf16, const float *x, const float *w,
                    int rows, int cols, float eps, ce_stream_t stream) {
  CE_REQUIRE(rows >= 1 && cols >= 1, "rows and cols must be >= 1 (got %d, %d)", rows, cols);
  CE_REQUIRE(out_bf16 != nullptr, "null bf16 output");
  return rows_iteration(out, out_bf16, ld_bf16, x, w, nullptr, nullptr, nullptr, nullptr, nullptr,
                        rows, 0, cols, 0, eps, (cudaStream_t)stream);
}

int ce_softmax(float *out, const float *logits, int rows, int cols, ce_stream_t stream) {
  CE_REQUIRE(rows >= 1 && cols >= 1, "rows and cols must be >= 1 (got %d, %d)", rows, cols);
  return rows_iteration(nullptr, nullptr, 0, nullptr, nullptr, out, logits, nullptr, nullptr,
                        nullptr, 0, rows, cols, 0, 0.f, (cudaStream_t)stream);
}

int ce_gemv(float *product, const float *matrix, const float *x, int rows, int cols,
            ce_stream_t stream) {
  CE_REQUIRE(rows >= 1 && cols >= 1, "rows and cols must be >= 1 (got %d, %d)", rows, cols);
  return rows_iteration(nullptr, nullptr, 0, nullptr, nullptr, nullptr, nullptr, product, matrix,
                        x, 0, 0, cols, rows, 0.f, (cudaStream_t)stream);
}

int ce_llama2c_iteration(float *normalized, float *softmax, float *product, const float *input,
                         const float *weight, const float *probabilities, const float *matrix,
                         int batch, int size, int rows, float eps, ce_stream_t stream) {
  CE_REQUIRE(batch >= 1 && size >= 1 && rows >= 1, "batch, size and rows must be >= 1");
  return rows_iteration(normalized, nullptr, 0, input, weight, softmax, probabilities, product,
                        matrix, input, batch, batch, size, rows, eps, (cudaStream_t)stream);
}

int ce_llama2c_rows(float *normalized, float *softmax, float *product, const float *input,
                    const float *weight, const float *probabilities, const float *matrix, int size,
                    int rms_rows, int softmax_rows, int matmul_rows, float eps, ce_stream_t stream) {
  CE_REQUIRE(size >= 1, "size must be >= 1 (got %d)", size);
  CE_REQUIRE(rms_rows >= 0 && softmax_rows >= 0 && matmul_rows >= 0,
             "row counts must be >= 0 (got %d, %d, %d)", rms_rows, softmax_rows, matmul_rows);
  CE_REQUIRE(rms_rows + softmax_rows + matmul_rows > 0, "no rows to compute");
  return rows_iteration(rms_rows ? normalized : nullptr, nullptr, 0, rms_rows ? input : nullptr,
                        rms_rows ? weight : nullptr, softmax_rows ? softmax : nullptr,
                        softmax_rows ? probabilities : nullptr, matmul_rows ? product : nullptr,
                        matmul_rows ? matrix : nullptr, matmul_rows ? input : nullptr, rms_rows,
                        softmax_rows, size, matmul_rows, eps, (cudaStream_t)stream);
}

int ce_gemm_bf16(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
                 int ldb, int ldd, ce_stream_t stream) {
  return gemm_bf16(d, a, b, M, N, K, lda, ldb, ldd, nullptr, nullptr, 0, (cudaStream_t)stream);
}

int ce_gemm_bf16_tile(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
                      int ldb, int ldd, int tile_n, ce_stream_t stream) {
  return gemm_bf16(d, a, b, M, N, K, lda, ldb, ldd, nullptr, nullptr, tile_n,
                   (cudaStream_t)stream, 1);
}

int ce_gemm_tuning(int l2_prefetch_kblocks) { return gemm_set_prefetch(l2_prefetch_kblocks); }

int ce_gemm_wide_tiles(int on) { return gemm_set_wide_tiles(on); }

int ce_rows_tuning(int streaming) { return rows_set_streaming(streaming); }

int ce_gemm_config(int precision, float *d, const void *a, const void *b, int M, int N, int K,
                   int lda, int ldb, int ldd, int cta_group, int tile_n, ce_stream_t stream) {
  if (precision == CE_PREC_BF16)
    return gemm_bf16(d, static_cast<const uint16_t *>(a), static_cast<const uint16_t *>(b), M, N,
                     K, lda, ldb, ldd, nullptr, nullptr, tile_n, (cudaStream_t)stream, cta_group);
  if (precision == CE_PREC_TF32)
    return gemm_tf32(d, static_cast<const float *>(a), static_cast<const float *>(b), M, N, K, lda,
                     ldb, ldd, nullptr, nullptr, tile_n, (cudaStream_t)stream, cta_group);
  if (precision == CE_PREC_FP8_E4M3)
    return gemm_e4m3(d, static_cast<const uint8_t *>(a), static_cast<const uint8_t *>(b), M, N, K,
                     lda, ldb, ldd, nullptr, nullptr, tile_n, (cudaStream_t)stream, cta_group);
  return set_error(CE_ERR_USAGE, format("ce_gemm_config: precision %d has no tensor-core kernel", precision));
}

int ce_gemm_bf16_split(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
                       int ldb, int ldd, int splits, int64_t split_stride, ce_stream_t stream) {
  return gemm_bf16_split(d, a, b, M, N, K, lda, ldb, ldd, splits, (long long)split_stride,
                         (cudaStream_t)stream, false);
}

int ce_w4_pack(uint8_t *codes_t, uint8_t *scales_t, const uint8_t *codes, const uint8_t *scales, int N,
               int K, int ld_bytes, int nsf, ce_stream_t stream) {
  return w4_pack(codes_t, scales_t, codes, scales, N, K, ld_bytes, nsf, (cudaStream_t)stream);
}

int ce_gemm_w4a16(float *d, const uint16_t *a, const uint8_t *codes_t, const uint8_t *scales_t,
                  const float *alpha, int M, int N, int K, int lda, int ldd, ce_stream_t stream) {
  return gemm_w4a16(d, a, codes_t, scales_t, alpha, M, N, K, lda, ldd, 1, 0, nullptr, 0,
                    (cudaStream_t)stream, false);
}

int ce_w4t_packed_bytes(int N, int K, size_t *bytes) {
  CE_REQUIRE(N >= 1 && K >= 64 && K % 64 == 0, "bad NVFP4 weight shape %dx%d", N, K);
  CE_REQUIRE(bytes != nullptr, "null argument");
  *bytes = w4t_packed_bytes(N, K);
  return CE_OK;
}

int ce_w4t_pack(uint8_t *packed, const uint8_t *codes, const uint8_t *scales, int N, int K, int ld_bytes, int nsf,
                ce_stream_t stream) {
  return w4t_pack(packed, codes, scales, N, K, ld_bytes, nsf, (cudaStream_t)stream, nullptr);
}

int ce_gemm_w4t(float *d, const uint16_t *a, const uint8_t *packed, const float *alpha, int M, int N, int K, int lda,
                int ldd, int splits, int64_t split_stride, ce_stream_t stream) {
  return gemm_w4t(d, a, packed, alpha, M, N, K, lda, ldd, splits, (long long)split_stride, nullptr, 0,
                  (cudaStream_t)stream, false);
}

int ce_w4t_expand_f16(uint16_t *out, const uint8_t *packed, int N, int K, ce_stream_t stream) {
  return w4t_expand_f16(out, packed, N, K, (cudaStream_t)stream);
}

int ce_gemm_f16(float *d, const uint16_t *a, const uint16_t *b, const float *alpha, int M, int N, int K, int lda,
                int ldb, int ldd, ce_stream_t stream) {
  return gemm_f16(d, a, b, alpha, M, N, K, lda, ldb, ldd, nullptr, 0, (cudaStream_t)stream, false);
}

int ce_gemm_tf32(float *d, const float *a, const float *b, int M, int N, int K, int lda, int ldb,
                 int ldd, ce_stream_t stream) {
  return gemm_tf32(d, a, b, M, N, K, lda, ldb, ldd, nullptr, nullptr, 0, (cudaStream_t)stream);
}

int ce_gemm_fp32(float *d, const float *a, const float *b, int M, int N, int K, int lda, int ldb,
                 int ldd, ce_stream_t stream) {
  return gemm_simt_fp32(d, a, b, M, N, K, lda, ldb, ldd, (cudaStream_t)stream);
}

int ce_quantize_e4m3_rows(uint8_t *codes, float *scales, const float *x, int rows, int cols,
                          int ld, ce_stream_t stream) {
  return quantize_rows_e4m3(codes, scales, x, rows, cols, ld, (cudaStream_t)stream);
}

int ce_quantize_mxfp6(uint8_t *codes, uint8_t *scales, const float *x, int rows, int cols,
                      int ld_codes, ce_stream_t stream) {
  return quantize_mxfp6(codes, scales, x, rows, cols, ld_codes, (cudaStream_t)stream);
}

int ce_quantize_nvfp4(uint8_t *codes, uint8_t *scales, float *tensor_scales, uint32_t *scratch,
                      const float *x, int rows, int cols, int ld_bytes, ce_stream_t stream) {
  return quantize_nvfp4(codes, scales, tensor_scales, scratch, x, rows, cols, ld_bytes,
                        (cudaStream_t)stream);
}

// Bytes of the scale-atom buffer: format 0 = MXFP6 (32 values per scale),
// 1 = NVFP4 (16); rows grouped by group_rows (128 for the A operand,
// CE_BS_TILE_N for the B operand).
int ce_sf_atom_bytes(int format, int rows, int K, int group_rows, size_t *bytes) {
  CE_REQUIRE(format == 0 || format == 1, "format must be 0 (MXFP6) or 1 (NVFP4)");
  CE_REQUIRE(rows >= 1 && K >= 1 && group_rows >= 1 && bytes, "bad arguments");
  *bytes = (size_t)sf_row_atoms(rows, group_rows) * sf_katoms(format, K) * 512;
  return CE_OK;
}

int ce_sf_to_atoms(int format, uint8_t *atoms, const uint8_t *scales, int rows, int K,
                   int group_rows, ce_stream_t stream) {
  CE_REQUIRE(format == 0 || format == 1, "format must be 0 (MXFP6) or 1 (NVFP4)");
  const int vec = format == 0 ? 32 : 16;
  return sf_to_atoms(atoms, scales, rows, (K + vec - 1) / vec, sf_katoms(format, K), group_rows,
                     (cudaStream_t)stream);
}

int ce_pack_mxfp6(uint8_t *operand, const uint8_t *codes, int rows, int cols, int ld_codes,
                  int ld_operand, ce_stream_t stream) {
  return pack_mxfp6(operand, codes, rows, cols, ld_codes, ld_operand, (cudaStream_t)stream);
}

int ce_gemm_mxfp6(float *d, const uint8_t *a, const uint8_t *a_sf, const uint8_t *b,
                  const uint8_t *b_sf, int M, int N, int K, int lda, int ldb, int ldd,
                  ce_stream_t stream) {
  return gemm_mxfp6(d, a, a_sf, b, b_sf, M, N, K, lda, ldb, ldd, (cudaStream_t)stream);
}

int ce_gemm_nvfp4(float *d, const uint8_t *a, const uint8_t *a_sf, const float *a_scales,
                  const uint8_t *b, const uint8_t *b_sf, const float *b_scales, int M, int N, int K,
                  int lda_bytes, int ldb_bytes, int ldd, ce_stream_t stream) {
  return gemm_nvfp4(d, a, a_sf, a_scales ? a_scales + 1 : nullptr, b, b_sf,
                    b_scales ? b_scales + 1 : nullptr, M, N, K, lda_bytes, ldb_bytes, ldd,
                    (cudaStream_t)stream);
}

int ce_rmsnorm_e4m3(float *out, uint8_t *codes, int ld, float *scales, const float *x,
                    const float *w, int rows, int cols, float eps, ce_stream_t stream) {
  CE_REQUIRE(rows >= 1 && cols >= 1, "rows and cols must be >= 1 (got %d, %d)", rows, cols);
  CE_REQUIRE(codes && scales && x && w, "null argument");
  return rows_iteration(out, nullptr, 0, x, w, nullptr, nullptr, nullptr, nullptr, nullptr, rows, 0,
                        cols, 0, eps, (cudaStream_t)stream, codes, ld, scales);
}

int ce_gemm_e4m3(float *d, const uint8_t *a, const float *a_scale, const uint8_t *b,
                 const float *b_scale, int M, int N, int K, int lda, int ldb, int ldd,
                 ce_stream_t stream) {
  return gemm_e4m3(d, a, b, M, N, K, lda, ldb, ldd, a_scale, b_scale, 0, (cudaStream_t)stream);
}

int ce_convert_bf16(uint16_t *out, const float *in, int rows, int cols, int ld_out,
                    ce_stream_t stream) {
  CE_REQUIRE(out && in, "null pointer");
  return convert_bf16(out, in, rows, cols, ld_out, (cudaStream_t)stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Op-trio plan

struct ce_plan {
  int batch = 0, size = 0, rows = 0, precision = 0, device = 0;
  int ld = 0;                    // padded K of the prepared operands
  void *weights = nullptr;       // bf16 / fp32 / e4m3 [rows][ld], or fp32 [rows][size] (FP32)
  void *activations = nullptr;   // bf16 / fp32 / e4m3 [batch][ld]
  float *w_scale = nullptr;      // e4m3: per weight row
  float *a_scale = nullptr;      // e4m3: per activation row
  // block-scaled (MXFP6 / NVFP4): scale atoms, tensor scales, staging
  uint8_t *w_atoms = nullptr;    // B scale atoms, grouped by CE_BS_TILE_N rows
  uint8_t *a_atoms = nullptr;    // A scale atoms, grouped by 128 rows
  float *a_f32 = nullptr;        // NVFP4: normalized rows when the caller passes none
  float *a_ts = nullptr;         // NVFP4 tensor scales of A (encode, decode)
  float *w_ts = nullptr;         // NVFP4 tensor scales of W
  uint32_t *scratch = nullptr;   // NVFP4 amax reduction word
  bool has_weights = false;
};

extern "C" int ce_plan_destroy(ce_plan *p);

static bool block_scaled(int precision) {
  return precision == CE_PREC_MXFP6_E3M2 || precision == CE_PREC_NVFP4_E2M1;
}

extern "C" {

int ce_plan_create(ce_plan **out, int batch, int size, int rows, int precision) {
  CE_REQUIRE(out != nullptr, "null plan pointer");
  *out = nullptr;
  CE_REQUIRE(batch >= 1 && size >= 1 && rows >= 1, "batch, size and rows must be >= 1");
  CE_REQUIRE(precision == CE_PREC_FP32 || precision == CE_PREC_TF32 || precision == CE_PREC_BF16 ||
                 precision == CE_PREC_FP8_E4M3 || block_scaled(precision),
             "precision %d is not available in this build", precision);
  CE_REQUIRE(!block_scaled(precision) || size % 128 == 0,
             "block-scaled plans need size %% 128 == 0 (got %d)", size);
  CE_REQUIRE(precision != CE_PREC_FP8_E4M3 || (size % 4 == 0 && size <= 32768),
             "the e4m3 plan needs size %% 4 == 0 and size <= 32768 (got %d)", size);
  ce_plan *p = new ce_plan();
  p->batch = batch;
  p->size = size;
  p->rows = rows;
  p->precision = precision;
  CE_CUDA_TRY(cudaGetDevice(&p->device));
  p->ld = precision == CE_PREC_FP32 ? size : ((size + 63) / 64) * 64;
  const size_t elem = precision == CE_PREC_BF16 ? 2 : precision == CE_PREC_FP8_E4M3 ? 1 : 4;
  if (block_scaled(precision)) {
    const int fmt = precision == CE_PREC_MXFP6_E3M2 ? 0 : 1;
    const int vec = fmt == 0 ? 32 : 16;
    p->ld = fmt == 0 ? size : size / 2;  // operand bytes per row
    (void)vec;
    // the rows launch writes the A operand and its scale atoms itself (MXFP6),
    // or max |normalized| for a quantizer pass (NVFP4); the atoms' padding
    // bytes are zeroed once here and never written again
    const size_t atom_bytes = (size_t)sf_row_atoms(batch, 128) * sf_katoms(fmt, size) * 512;
    cudaError_t e2 = cudaMalloc(&p->activations, (size_t)batch * p->ld);
    if (e2 == cudaSuccess) e2 = cudaMalloc(&p->a_atoms, atom_bytes);
    if (e2 == cudaSuccess) e2 = cudaMemset(p->a_atoms, 0, atom_bytes);
    if (e2 == cudaSuccess && fmt == 1) e2 = cudaMalloc(&p->a_f32, (size_t)batch * size * 4);
    if (e2 == cudaSuccess && fmt == 1) e2 = cudaMalloc(&p->a_ts, 2 * sizeof(float));
    if (e2 == cudaSuccess && fmt == 1) e2 = cudaMalloc(&p->w_ts, 2 * sizeof(float));
    if (e2 == cudaSuccess && fmt == 1) e2 = cudaMalloc(&p->scratch, sizeof(uint32_t));
    if (e2 != cudaSuccess) {
      ce_plan_destroy(p);
      return cuda_error(e2, "cudaMalloc(block-scaled plan)");
    }
    *out = p;
    return CE_OK;
  }
  cudaError_t e = cudaMalloc(&p->activations, (size_t)batch * p->ld * elem);
  if (e == cudaSuccess && precision == CE_PREC_FP8_E4M3) {
    e = cudaMalloc(&p->a_scale, (size_t)batch * 4);
    if (e == cudaSuccess) e = cudaMalloc(&p->w_scale, (size_t)rows * 4);
  }
  if (e != cudaSuccess) {
    if (p->activations) cudaFree(p->activations);
    if (p->a_scale) cudaFree(p->a_scale);
    delete p;
    return cuda_error(e, "cudaMalloc(activations)");
  }
  *out = p;
  return CE_OK;
}

int ce_plan_destroy(ce_plan *p) {
  if (p == nullptr) return CE_OK;
  if (p->weights) cudaFree(p->weights);
  if (p->activations) cudaFree(p->activations);
  for (void *q : {(void *)p->a_scale, (void *)p->w_scale, (void *)p->w_atoms, (void *)p->a_atoms,
                  (void *)p->a_f32, (void *)p->a_ts, (void *)p->w_ts, (void *)p->scratch})
    if (q) cudaFree(q);
  delete p;
  return CE_OK;
}

int ce_plan_set_weights(ce_plan *p, const float *w, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && w != nullptr, "null plan or weights");
  cudaStream_t s = (cudaStream_t)stream;
  if (block_scaled(p->precision)) {
    const int fmt = p->precision == CE_PREC_MXFP6_E3M2 ? 0 : 1;
    const int vec = fmt == 0 ? 32 : 16;
    const size_t w_bytes = (size_t)p->rows * (fmt == 0 ? p->size : p->size / 2);
    if (p->weights == nullptr) CE_CUDA_TRY(cudaMalloc(&p->weights, w_bytes));
    if (p->w_atoms == nullptr)
      CE_CUDA_TRY(cudaMalloc(&p->w_atoms, (size_t)sf_row_atoms(p->rows, CE_BS_TILE_N) *
                                              sf_katoms(fmt, p->size) * 512));
    uint8_t *sf = nullptr, *codes = nullptr;
    CE_CUDA_TRY(cudaMalloc(&sf, (size_t)p->rows * (p->size / vec)));
    int rc;
    if (fmt == 0) {
      cudaError_t e = cudaMalloc(&codes, (size_t)p->rows * p->size);
      if (e != cudaSuccess) {
        cudaFree(sf);
        return cuda_error(e, "cudaMalloc(weight codes)");
      }
      rc = quantize_mxfp6(codes, sf, w, p->rows, p->size, p->size, s);
      if (rc == CE_OK)
        rc = pack_mxfp6(static_cast<uint8_t *>(p->weights), codes, p->rows, p->size, p->size,
                        p->size, s);
    } else {
      rc = quantize_nvfp4(static_cast<uint8_t *>(p->weights), sf, p->w_ts, p->scratch, w, p->rows,
                          p->size, p->size / 2, s);
    }
    if (rc == CE_OK)
      rc = sf_to_atoms(p->w_atoms, sf, p->rows, p->size / vec, sf_katoms(fmt, p->size),
                       CE_BS_TILE_N, s);
    cudaError_t e = cudaStreamSynchronize(s);
    cudaFree(sf);
    if (codes) cudaFree(codes);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_error(e, "cudaStreamSynchronize");
    p->has_weights = true;
    return CE_OK;
  }
  const size_t elem = p->precision == CE_PREC_BF16 ? 2 : p->precision == CE_PREC_FP8_E4M3 ? 1 : 4;
  if (p->weights == nullptr) CE_CUDA_TRY(cudaMalloc(&p->weights, (size_t)p->rows * p->ld * elem));
  if (p->precision == CE_PREC_FP8_E4M3) {
    int rc = quantize_rows_e4m3(static_cast<uint8_t *>(p->weights), p->w_scale, w, p->rows, p->size,
                                p->ld, s);
    if (rc) return rc;
  } else if (p->precision == CE_PREC_BF16) {
    int rc = convert_bf16(static_cast<uint16_t *>(p->weights), w, p->rows, p->size, p->ld, s);
    if (rc) return rc;
  } else {
    CE_CUDA_TRY(cudaMemset2DAsync(p->weights, (size_t)p->ld * 4, 0, (size_t)p->ld * 4, p->rows, s));
    CE_CUDA_TRY(cudaMemcpy2DAsync(p->weights, (size_t)p->ld * 4, w, (size_t)p->size * 4,
                                  (size_t)p->size * 4, p->rows, cudaMemcpyDeviceToDevice, s));
  }
  CE_CUDA_TRY(cudaStreamSynchronize(s));
  p->has_weights = true;
  return CE_OK;
}

static int plan_gemm(ce_plan *p, float *out, cudaStream_t s, int ldd = 0) {
  if (ldd == 0) ldd = p->rows;
  switch (p->precision) {
    case CE_PREC_MXFP6_E3M2:
      return gemm_mxfp6(out, static_cast<const uint8_t *>(p->activations), p->a_atoms,
                        static_cast<const uint8_t *>(p->weights), p->w_atoms, p->batch, p->rows,
                        p->size, p->size, p->size, ldd, s);
    case CE_PREC_NVFP4_E2M1:
      return gemm_nvfp4(out, static_cast<const uint8_t *>(p->activations), p->a_atoms, p->a_ts + 1,
                        static_cast<const uint8_t *>(p->weights), p->w_atoms, p->w_ts + 1, p->batch,
                        p->rows, p->size, p->size / 2, p->size / 2, ldd, s);
    case CE_PREC_BF16:
      return gemm_bf16(out, static_cast<const uint16_t *>(p->activations),
                       static_cast<const uint16_t *>(p->weights), p->batch, p->rows, p->size,
                       p->ld, p->ld, ldd, nullptr, nullptr, 0, s);
    case CE_PREC_FP8_E4M3:
      return gemm_e4m3(out, static_cast<const uint8_t *>(p->activations),
                       static_cast<const uint8_t *>(p->weights), p->batch, p->rows, p->size, p->ld,
                       p->ld, ldd, p->a_scale, p->w_scale, 0, s);
    case CE_PREC_TF32:
      return gemm_tf32(out, static_cast<const float *>(p->activations),
                       static_cast<const float *>(p->weights), p->batch, p->rows, p->size, p->ld,
                       p->ld, ldd, nullptr, nullptr, 0, s);
    default:
      return gemm_simt_fp32(out, static_cast<const float *>(p->activations),
                            static_cast<const float *>(p->weights), p->batch, p->rows, p->size,
                            p->ld, p->ld, ldd, s);
  }
}

// Rows stage of the trio: rmsnorm (fp32 output plus the GEMM operand in the
// plan's layout) and, if logits != NULL, the softmax rows in the same launch.
static int plan_rows(ce_plan *p, float *normalized, float *softmax, const float *x,
                     const float *norm_w, const float *logits, float eps, cudaStream_t s) {
  const int nsoft = logits ? p->batch : 0;
  if (block_scaled(p->precision)) {
    // The activation quantizer of the format (the reference converts with
    // separate launches per step, decoder_lowprec.cu:202-340, 469-482) fused
    // into the rows launch: MXFP6's block scales need only each 32-value
    // block, so the rows launch writes the packed codes and scale atoms from
    // the normalized values in registers; NVFP4's tensor scale needs max
    // |normalized| over the whole batch first, so the rows launch reduces it
    // (keeping the fp32 rows L2-resident) and one pass writes codes and atoms.
    const int fmt = p->precision == CE_PREC_MXFP6_E3M2 ? 0 : 1;
    const int katoms = sf_katoms(fmt, p->size);
    RowsExtras ex;
    ex.katoms = katoms;
    if (fmt == 0) {
      ex.mx_operand = static_cast<uint8_t *>(p->activations);
      ex.mx_ld = p->size;
      ex.mx_atoms = p->a_atoms;
      return rows_iteration(normalized, nullptr, 0, x, norm_w, softmax, logits, nullptr, nullptr, nullptr,
                            p->batch, nsoft, p->size, 0, eps, s, nullptr, 0, nullptr, 0, 0x7fffffff, &ex);
    }
    float *xn = normalized ? normalized : p->a_f32;
    ex.amax_bits = p->scratch;
    ex.keep_normalized = 1;
    CE_CUDA_TRY(cudaMemsetAsync(p->scratch, 0, sizeof(uint32_t), s));
    int rc = rows_iteration(xn, nullptr, 0, x, norm_w, softmax, logits, nullptr, nullptr, nullptr, p->batch, nsoft,
                            p->size, 0, eps, s, nullptr, 0, nullptr, 0, 0x7fffffff, &ex);
    if (rc) return rc;
    return quantize_nvfp4_atoms(static_cast<uint8_t *>(p->activations), p->a_atoms, p->a_ts, p->scratch, xn,
                                p->batch, p->size, p->size / 2, katoms, s);
  }
  if (p->precision == CE_PREC_FP8_E4M3)
    return rows_iteration(normalized, nullptr, 0, x, norm_w, softmax, logits, nullptr, nullptr,
                          nullptr, p->batch, nsoft, p->size, 0, eps, s,
                          static_cast<uint8_t *>(p->activations), p->ld, p->a_scale);
  if (p->precision == CE_PREC_BF16)
    return rows_iteration(normalized, static_cast<uint16_t *>(p->activations), p->ld, x, norm_w,
                          softmax, logits, nullptr, nullptr, nullptr, p->batch, nsoft, p->size, 0,
                          eps, s);
  // fp32 operand: the normalized rows themselves, written into the padded
  // workspace (ld == size for FP32; for TF32 the padding columns stay 0 from
  // the memset at the first call of this plan's stream work).
  float *work = static_cast<float *>(p->activations);
  int rc;
  if (p->ld == p->size) {
    rc = rows_iteration(work, nullptr, 0, x, norm_w, softmax, logits, nullptr, nullptr, nullptr,
                        p->batch, nsoft, p->size, 0, eps, s);
    if (rc) return rc;
    if (normalized)
      CE_CUDA_TRY(cudaMemcpyAsync(normalized, work, (size_t)p->batch * p->size * 4,
                                  cudaMemcpyDeviceToDevice, s));
    return CE_OK;
  }
  float *dst = normalized ? normalized : work;
  rc = rows_iteration(dst, nullptr, 0, x, norm_w, softmax, logits, nullptr, nullptr, nullptr,
                      p->batch, nsoft, p->size, 0, eps, s);
  if (rc) return rc;
  CE_CUDA_TRY(cudaMemset2DAsync(work, (size_t)p->ld * 4, 0, (size_t)p->ld * 4, p->batch, s));
  CE_CUDA_TRY(cudaMemcpy2DAsync(work, (size_t)p->ld * 4, dst, (size_t)p->size * 4,
                                (size_t)p->size * 4, p->batch, cudaMemcpyDeviceToDevice, s));
  return CE_OK;
}

int ce_plan_operands(ce_plan *p, float *a, float *w, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr, "null plan");
  CE_REQUIRE(w == nullptr || p->has_weights, "ce_plan_set_weights has not been called");
  cudaStream_t s = (cudaStream_t)stream;
  for (int which = 0; which < 2; ++which) {
    float *out = which == 0 ? a : w;
    if (out == nullptr) continue;
    DequantOperand d;
    d.rows = which == 0 ? p->batch : p->rows;
    d.cols = p->size;
    d.out = out;
    d.out_ld = p->size;
    d.data = which == 0 ? p->activations : p->weights;
    d.ld = p->ld;
    switch (p->precision) {
      case CE_PREC_BF16: d.format = kOperandBF16; break;
      case CE_PREC_FP8_E4M3:
        d.format = kOperandE4M3;
        d.row_scale = which == 0 ? p->a_scale : p->w_scale;
        break;
      case CE_PREC_MXFP6_E3M2:
      case CE_PREC_NVFP4_E2M1: {
        const int fmt = p->precision == CE_PREC_MXFP6_E3M2 ? 0 : 1;
        d.format = fmt == 0 ? kOperandMXFP6 : kOperandNVFP4;
        d.ld = fmt == 0 ? p->size : p->size / 2;
        d.nsf = p->size / (fmt == 0 ? 32 : 16);
        // both as the GEMM reads them: scale atoms, A grouped by 128 rows,
        // W by the GEMM's B tile rows
        d.atoms = true;
        d.sf = which == 0 ? p->a_atoms : p->w_atoms;
        d.katoms = sf_katoms(fmt, p->size);
        d.group_rows = which == 0 ? 128 : CE_BS_TILE_N;
        if (fmt == 1) d.tensor_decode = (which == 0 ? p->a_ts : p->w_ts) + 1;
        break;
      }
      default: d.format = kOperandF32;
    }
    const int rc = dequant_operand(d, s);
    if (rc) return rc;
  }
  return CE_OK;
}

int ce_plan_rows(ce_plan *p, float *normalized, float *softmax, const float *x,
                 const float *norm_w, const float *logits, float eps, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && x && norm_w, "null argument");
  CE_REQUIRE((logits == nullptr) == (softmax == nullptr), "logits and softmax go together");
  return plan_rows(p, normalized, softmax, x, norm_w, logits, eps, (cudaStream_t)stream);
}

int ce_plan_rows_range(ce_plan *p, float *normalized, float *softmax, const float *x, const float *norm_w,
                       const float *logits, float eps, int row_lo, int row_hi, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && x && norm_w, "null argument");
  CE_REQUIRE((logits == nullptr) == (softmax == nullptr), "logits and softmax go together");
  CE_REQUIRE(0 <= row_lo && row_lo <= row_hi && row_hi <= p->batch, "row range [%d, %d) is outside the batch of %d",
             row_lo, row_hi, p->batch);
  CE_REQUIRE(p->precision == CE_PREC_BF16 || p->precision == CE_PREC_FP8_E4M3,
             "a row range of the rows stage needs a bf16 or fp8 plan (precision %d)", p->precision);
  cudaStream_t s = (cudaStream_t)stream;
  const int nsoft = logits ? row_hi - row_lo : 0;
  const size_t off = (size_t)row_lo * p->size;
  float *sm = softmax ? softmax + off : nullptr;
  const float *lg = logits ? logits + off : nullptr;
  if (p->precision == CE_PREC_FP8_E4M3)
    return rows_iteration(normalized, nullptr, 0, x, norm_w, sm, lg, nullptr, nullptr, nullptr, p->batch, nsoft,
                          p->size, 0, eps, s, static_cast<uint8_t *>(p->activations), p->ld, p->a_scale, row_lo,
                          row_hi);
  return rows_iteration(normalized, static_cast<uint16_t *>(p->activations), p->ld, x, norm_w, sm, lg, nullptr,
                        nullptr, nullptr, p->batch, nsoft, p->size, 0, eps, s, nullptr, 0, nullptr, row_lo, row_hi);
}

int ce_plan_gemm(ce_plan *p, float *out, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && out != nullptr, "null argument");
  CE_REQUIRE(p->has_weights, "ce_plan_set_weights has not been called");
  return plan_gemm(p, out, (cudaStream_t)stream);
}

int ce_plan_gemm_ld(ce_plan *p, float *out, int ldd, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && out != nullptr, "null argument");
  CE_REQUIRE(p->has_weights, "ce_plan_set_weights has not been called");
  CE_REQUIRE(ldd >= p->rows, "output row stride %d is below the plan's %d rows", ldd, p->rows);
  return plan_gemm(p, out, (cudaStream_t)stream, ldd);
}

int ce_plan_gemm_rowx(ce_plan *p, ce_rowx *x, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && x != nullptr, "null argument");
  CE_REQUIRE(p->has_weights, "ce_plan_set_weights has not been called");
  RowxSync rx;
  float *out = nullptr;
  int lo = 0, hi = 0, batch = 0, rows = 0;
  int rc = rowx_sync(x, &rx, &out, &lo, &hi, &batch, &rows);
  if (rc) return rc;
  CE_REQUIRE(p->batch == batch && p->rows == hi - lo,
             "the plan (batch %d, rows %d) is not this rank's slice of the exchange (batch %d, rows %d..%d)",
             p->batch, p->rows, batch, lo, hi);
  CE_REQUIRE(p->device == x_device_of(x), "plan and exchange are on different devices");
  cudaStream_t s = (cudaStream_t)stream;
  switch (p->precision) {
    case CE_PREC_BF16:
      return gemm_rowx(0, out + lo, p->activations, p->weights, p->batch, p->rows, p->size, p->ld, p->ld, rows,
                       nullptr, nullptr, rx, s);
    case CE_PREC_TF32:
      return gemm_rowx(1, out + lo, p->activations, p->weights, p->batch, p->rows, p->size, p->ld, p->ld, rows,
                       nullptr, nullptr, rx, s);
    case CE_PREC_FP8_E4M3:
      return gemm_rowx(2, out + lo, p->activations, p->weights, p->batch, p->rows, p->size, p->ld, p->ld, rows,
                       p->a_scale, p->w_scale, rx, s);
    default:
      return set_error(CE_ERR_USAGE, format("the row-shard fan-out GEMM supports bf16, tf32 and fp8 plans "
                                            "(precision %d)", p->precision));
  }
}

int ce_plan_rmsnorm_gemm(ce_plan *p, float *out, float *normalized, const float *x,
                         const float *norm_w, float eps, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && out && x && norm_w, "null argument");
  CE_REQUIRE(p->has_weights, "ce_plan_set_weights has not been called");
  cudaStream_t s = (cudaStream_t)stream;
  int rc = plan_rows(p, normalized, nullptr, x, norm_w, nullptr, eps, s);
  if (rc) return rc;
  return plan_gemm(p, out, s);
}

int ce_plan_trio(ce_plan *p, float *normalized, float *softmax, float *out, const float *x,
                 const float *norm_w, const float *logits, float eps, ce_stream_t stream) {
  CE_REQUIRE(p != nullptr && out && x && norm_w && logits && softmax, "null argument");
  CE_REQUIRE(p->has_weights, "ce_plan_set_weights has not been called");
  cudaStream_t s = (cudaStream_t)stream;
  int rc = plan_rows(p, normalized, softmax, x, norm_w, logits, eps, s);
  if (rc) return rc;
  return plan_gemm(p, out, s);
}

}  // extern "C"
