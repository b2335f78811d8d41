// SIMT fp32 GEMM with the reference's bitwise contract: every output
// D[m][n] = sum over k = 0..K-1 of A[m][k] * B[n][k], accumulated by one
// thread from 0.0f in increasing k with a separate multiply and add. This
// file is compiled with --fmad=false so no multiply-add is contracted.
// It restates the arithmetic order of the reference's classifier
// (applications/loom_private/decoder/decoder.cu:79-125 and the optimized
// stream-K variant, decoder_optimized.cu:343-439): the llama2.c matmul order
// that the decoder contract pins (contract.json "operation_order").
// It is the control path (CE_PREC_FP32); the tensor-core paths are gemm.cu.
#include "common.cuh"

namespace ce {
namespace {

constexpr int kTile = 128;   // 128 x 128 outputs per block
constexpr int kTileK = 16;   // k columns per shared-memory stage
constexpr int kThreadsXY = 16;

__global__ void __launch_bounds__(kThreadsXY * kThreadsXY)
simt_gemm_kernel(float *d, const float *a, const float *b, int M, int N, int K, int lda,
                 int ldb, int ldd) {
  __shared__ float as[kTileK][kTile + 4];  // [k][m]
  __shared__ float bs[kTileK][kTile + 4];  // [k][n]
  const int tx = threadIdx.x % kThreadsXY, ty = threadIdx.x / kThreadsXY;
  const int n0 = blockIdx.x * kTile, m0 = blockIdx.y * kTile;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += kTileK) {
    for (int e = threadIdx.x; e < kTile * kTileK; e += blockDim.x) {
      const int line = e / kTileK, kk = e % kTileK, k = k0 + kk;
      const int m = m0 + line, n = n0 + line;
      as[kk][line] = (m < M && k < K) ? a[(size_t)m * lda + k] : 0.0f;
      bs[kk][line] = (n < N && k < K) ? b[(size_t)n * ldb + k] : 0.0f;
    }
    __syncthreads();
    const int count = min(kTileK, K - k0);
    for (int kk = 0; kk < count; ++kk) {
      float av[8], bv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) av[i] = as[kk][ty + kThreadsXY * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) bv[j] = bs[kk][tx + kThreadsXY * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float product = bv[j] * av[i];
          acc[i][j] = acc[i][j] + product;
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + ty + kThreadsXY * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + tx + kThreadsXY * j;
      if (n < N) d[(size_t)m * ldd + n] = acc[i][j];
    }
  }
}

}  // namespace

int gemm_simt_fp32(float *d, const float *a, const float *b, int M, int N, int K, int lda,
                   int ldb, int ldd, cudaStream_t s) {
  CE_REQUIRE(M >= 1 && N >= 1 && K >= 1, "GEMM dims must be >= 1 (M=%d N=%d K=%d)", M, N, K);
  CE_REQUIRE(lda >= K && ldb >= K && ldd >= N, "leading dimensions too small");
  CE_REQUIRE(d && a && b, "null operand");
  dim3 grid((N + kTile - 1) / kTile, (M + kTile - 1) / kTile);
  simt_gemm_kernel<<<grid, kThreadsXY * kThreadsXY, 0, s>>>(d, a, b, M, N, K, lda, ldb, ldd);
  CE_LAUNCH_CHECK("simt_gemm_kernel");
  return CE_OK;
}

}  // namespace ce
