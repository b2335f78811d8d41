// Weight quantizers (setup-time conversions, as the reference quantizes its
// classifier once in setup, experiments/blackwell/lowprec/decoder_lowprec.cu:
// 444-458, 573-579).
//
// E4M3 with one fp32 scale per row: amax = max |w| of the row, inv = 448 /
// amax, scale = amax / 448 (IEEE fp32; 0 for an all-zero row), code =
// E4M3(w * inv) rounded to nearest even and saturated to +-448. Rows are
// written into a [rows][ld] code buffer whose columns past `cols` are 0.
#include "row_ops.cuh"

namespace ce {
namespace {

using namespace rowops;

__global__ void __launch_bounds__(256)
quantize_rows_e4m3_kernel(uint8_t *codes, float *scales, const float *x, int cols, int ld) {
  __shared__ float scratch[32];
  const size_t row = blockIdx.x;
  const float *xr = x + row * (size_t)cols;
  float amax = 0.f;
  for (int k = threadIdx.x; k < cols; k += blockDim.x) amax = fmaxf(amax, fabsf(xr[k]));
  amax = block_max(amax, scratch);
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
  if (threadIdx.x == 0) scales[row] = amax / 448.0f;
  uint8_t *cr = codes + row * (size_t)ld;
  for (int k = threadIdx.x; k < ld; k += blockDim.x)
    cr[k] = k < cols ? (uint8_t)(e4m3x2(xr[k] * inv, 0.f) & 0xFFu) : (uint8_t)0;
}

}  // namespace

int quantize_rows_e4m3(uint8_t *codes, float *scales, const float *x, int rows, int cols, int ld,
                       cudaStream_t s) {
  CE_REQUIRE(codes && scales && x, "null argument");
  CE_REQUIRE(rows >= 1 && cols >= 1 && ld >= cols, "bad quantization shape %dx%d ld %d", rows, cols, ld);
  quantize_rows_e4m3_kernel<<<rows, 256, 0, s>>>(codes, scales, x, cols, ld);
  CE_LAUNCH_CHECK("quantize_rows_e4m3_kernel");
  return CE_OK;
}

}  // namespace ce
