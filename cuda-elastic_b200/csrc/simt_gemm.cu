// SIMT fp32 GEMM with the reference's bitwise contract: every output
// D[m][n] = sum over k = 0..K-1 of A[m][k] * B[n][k], accumulated by one
// thread from 0.0f in increasing k with a separate multiply and add. This
// file is compiled with --fmad=false so no multiply-add is contracted.
// It restates the arithmetic order of the reference's classifier
// (applications/loom_private/decoder/decoder.cu:79-125 and the optimized
// stream-K variant, decoder_optimized.cu:343-439): the llama2.c matmul order
// that the decoder contract pins (contract.json "operation_order").
// It is the control path (CE_PREC_FP32); the tensor-core paths are gemm.cu.
//
// Design. Without FMA every multiply-add is two FP32 instructions, so the
// kernel is bound by instruction issue (one warp instruction per SM
// sub-partition per clock): the B200 ceiling is 148 SMs x 64 multiply-adds
// per clock. Each thread owns an 8 x 8 block of outputs (8 x 6 or 8 x 4 in
// the narrow tiles below) and per k reads its 8 A values and 8 B values as
// float4 shared loads, 4 loads for 128 arithmetic instructions. Operands
// reach shared memory through a 3-stage cp.async pipeline of 4-byte copies
// that transpose the K-major global rows into [k][row] shared rows (row
// stride 136 floats, so a warp's 8 rows x 4 k copy hits 32 distinct banks).
// Two 256-thread blocks are resident per SM. When the 128 x 128 tiles would
// leave a partly empty last wave, the columns are split into two regions:
// the first holds whole waves of 128-wide tiles, the second is cut into
// 96- or 64-wide tiles sized so the last wave fills the SMs (chosen by a
// small list-scheduling estimate on the host).
#include <algorithm>
#include <queue>
#include <vector>

#include "common.cuh"

namespace ce {
namespace {

constexpr int kBM = 128;      // rows of A per tile
constexpr int kBK = 16;       // k per pipeline stage
constexpr int kStages = 3;
constexpr int kThreads = 256;
constexpr int kLd = 136;      // floats per shared row (== 8 mod 32)

struct SimtSmem {
  float a[kStages][kBK][kLd];
  float b[kStages][kBK][kLd];
};

__device__ __forceinline__ void cp_async4(float *dst, const float *src, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Copies rows [row0, row0 + ROWS) x k [k0, k0 + 16) of a K-major matrix into
// dst[k][row], zero-filling outside [0, nrows) x [0, K). Warp w copies rows
// (w % 2) * ROWS/2 + [0, ROWS/2) at k (w / 2) * 4 + [0, 4): ROWS / 16 copies of
// 8 rows x 4 consecutive k, lane (l % 8, l / 8), one 4-byte copy each.
template <int ROWS>
struct StageLoader {
  const float *src;    // matrix base (source of the zero-filled copies)
  const float *base;   // this thread's first row at its k offset
  size_t step;         // 8 rows
  int rbase, kq;       // this thread's first shared row and k offset
  unsigned rows_ok;    // bit j: row rbase + 8j is inside the matrix

  __device__ __forceinline__ StageLoader(const float *m, int ld, int row0, int nrows) : src(m) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    rbase = (warp % 2) * (ROWS / 2) + lane % 8;
    kq = (warp / 2) * 4 + lane / 8;
    base = m + (size_t)(row0 + rbase) * ld + kq;
    step = (size_t)8 * ld;
    rows_ok = 0;
#pragma unroll
    for (int j = 0; j < ROWS / 16; ++j) rows_ok |= (row0 + rbase + 8 * j < nrows ? 1u : 0u) << j;
  }
  __device__ __forceinline__ void load(float (*dst)[kLd], int k0, int K) const {
    constexpr unsigned kAllRows = (1u << (ROWS / 16)) - 1;
    if (rows_ok == kAllRows && k0 + kBK <= K) {  // interior: no predicates
      const float *p = base + k0;
#pragma unroll
      for (int j = 0; j < ROWS / 16; ++j) cp_async4(&dst[kq][rbase + 8 * j], p + j * step, true);
      return;
    }
    const bool k_ok = k0 + kq < K;
#pragma unroll
    for (int j = 0; j < ROWS / 16; ++j) {
      const bool valid = k_ok && ((rows_ok >> j) & 1u);
      cp_async4(&dst[kq][rbase + 8 * j], valid ? base + j * step + k0 : src, valid);
    }
  }
};

// One tile of kBM x (64 + 16 * TN2) outputs. Thread (tx, ty) of 16 x 16 owns
// rows ty*4 + {0..3} and 64 + ty*4 + {0..3}, columns tx*4 + {0..3} and
// 64 + tx*TN2 + {0..TN2-1}.
template <int TN2>
__device__ __forceinline__ void simt_tile(SimtSmem &sm, float *d, const float *a, const float *b,
                                          int M, int N, int K, int lda, int ldb, int ldd, int m0,
                                          int n0) {
  constexpr int BN = 64 + 16 * TN2, TN = 4 + TN2;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[8][TN];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  const int tiles = (K + kBK - 1) / kBK;
  const StageLoader<kBM> load_a(a, lda, m0, M);
  const StageLoader<BN> load_b(b, ldb, n0, N);
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < tiles) {
      load_a.load(sm.a[s], s * kBK, K);
      load_b.load(sm.b[s], s * kBK, K);
    }
    cp_async_commit();
  }

  auto step = [&](const float (*as)[kLd], const float (*bs)[kLd], int kk) {
    const float4 a0 = *reinterpret_cast<const float4 *>(&as[kk][ty * 4]);
    const float4 a1 = *reinterpret_cast<const float4 *>(&as[kk][64 + ty * 4]);
    const float4 b0 = *reinterpret_cast<const float4 *>(&bs[kk][tx * 4]);
    float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float bv[TN];
    bv[0] = b0.x, bv[1] = b0.y, bv[2] = b0.z, bv[3] = b0.w;
    if constexpr (TN2 == 4) {
      const float4 b1 = *reinterpret_cast<const float4 *>(&bs[kk][64 + tx * 4]);
      bv[4] = b1.x, bv[5] = b1.y, bv[6] = b1.z, bv[7] = b1.w;
    } else if constexpr (TN2 == 2) {
      const float2 b1 = *reinterpret_cast<const float2 *>(&bs[kk][64 + tx * 2]);
      bv[4] = b1.x, bv[5] = b1.y;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const float product = bv[j] * av[i];
        acc[i][j] = acc[i][j] + product;
      }
  };

  for (int t = 0; t < tiles; ++t) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    // refill the stage consumed in the previous iteration
    const int next = t + kStages - 1;
    if (next < tiles) {
      load_a.load(sm.a[next % kStages], next * kBK, K);
      load_b.load(sm.b[next % kStages], next * kBK, K);
    }
    cp_async_commit();
    const float(*as)[kLd] = sm.a[t % kStages];
    const float(*bs)[kLd] = sm.b[t % kStages];
    const int count = min(kBK, K - t * kBK);
    if (count == kBK) {
      // a partial unroll keeps the loop body within the instruction cache
#pragma unroll 4
      for (int kk = 0; kk < kBK; ++kk) step(as, bs, kk);
    } else {
      for (int kk = 0; kk < count; ++kk) step(as, bs, kk);
    }
  }
  cp_async_wait<0>();

  const bool vec = (ldd % 4 == 0) && ((reinterpret_cast<uintptr_t>(d) & 15) == 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= M) continue;
    float *row = d + (size_t)m * ldd;
    const int nA = n0 + tx * 4;
    if (vec && nA + 3 < N) {
      *reinterpret_cast<float4 *>(row + nA) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (nA + j < N) row[nA + j] = acc[i][j];
    }
    if constexpr (TN2 > 0) {
      const int nB = n0 + 64 + tx * TN2;
#pragma unroll
      for (int j = 0; j < TN2; ++j)
        if (nB + j < N) row[nB + j] = acc[i][4 + j];
    }
  }
}

// Blocks [0, tiles1) are 128 x 128 tiles over columns [0, n_split), the rest
// are 128 x (64 + 16 * TN2B) tiles over [n_split, N); both m-fastest, so the
// blocks that share a B tile run together and read it from HBM once.
template <int TN2B>
__global__ void __launch_bounds__(kThreads, 2)
simt_gemm_kernel(float *d, const float *a, const float *b, int M, int N, int K, int lda, int ldb,
                 int ldd, int mt, int tiles1, int n_split) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SimtSmem &sm = *reinterpret_cast<SimtSmem *>(smem_raw);
  const int id = blockIdx.x;
  if constexpr (TN2B == 4) {
    simt_tile<4>(sm, d, a, b, M, N, K, lda, ldb, ldd, (id % mt) * kBM, (id / mt) * 128);
  } else if (id < tiles1) {
    simt_tile<4>(sm, d, a, b, M, N, K, lda, ldb, ldd, (id % mt) * kBM, (id / mt) * 128);
  } else {
    const int r = id - tiles1;
    simt_tile<TN2B>(sm, d, a, b, M, N, K, lda, ldb, ldd, (r % mt) * kBM,
                    n_split + (r / mt) * (64 + 16 * TN2B));
  }
}

struct SimtPlan {
  int width2 = 128;  // second-region tile width (128: no second region)
  int tiles1 = 0, tiles2 = 0, n_split = 0;
};

// Makespan (in 128 x 128 tile times) of `first` unit blocks followed by
// `second` blocks of duration `w` on `slots` greedy slots.
double makespan(int first, int second, double w, int slots) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> q;
  for (int i = 0; i < slots; ++i) q.push(0.0);
  double end = 0.0;
  for (int i = 0; i < first + second; ++i) {
    const double t = q.top() + (i < first ? 1.0 : w);
    q.pop();
    q.push(t);
    end = std::max(end, t);
  }
  return end;
}

SimtPlan plan_tiles(int M, int N, int slots) {
  const int mt = (M + kBM - 1) / kBM, ct = (N + 127) / 128;
  SimtPlan best;
  best.tiles1 = mt * ct;
  best.n_split = N;
  const int total = mt * ct;
  if (total <= slots || total % slots == 0 || total > 64 * slots) return best;
  double best_time = makespan(total, 0, 0.0, slots);
  for (int q = 1; q <= total / slots; ++q) {
    const int c1 = q * slots / mt;
    if (c1 <= 0 || c1 >= ct) continue;
    const int rest = N - c1 * 128;
    for (int w : {96, 64}) {
      const int c2 = (rest + w - 1) / w;
      const double t = makespan(mt * c1, mt * c2, w / 128.0, slots);
      if (t < best_time - 1e-9) {
        best_time = t;
        best.width2 = w;
        best.tiles1 = mt * c1;
        best.tiles2 = mt * c2;
        best.n_split = c1 * 128;
      }
    }
  }
  return best;
}

template <int TN2B>
int launch(const SimtPlan &p, float *d, const float *a, const float *b, int M, int N, int K,
           int lda, int ldb, int ldd, cudaStream_t s) {
  const int mt = (M + kBM - 1) / kBM;
  simt_gemm_kernel<TN2B><<<p.tiles1 + p.tiles2, kThreads, sizeof(SimtSmem), s>>>(
      d, a, b, M, N, K, lda, ldb, ldd, mt, p.tiles1, p.n_split);
  CE_LAUNCH_CHECK("simt_gemm_kernel");
  return CE_OK;
}

// Resident 256-thread blocks on the whole device, once per device.
int g_slots[64];

int device_slots() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (g_slots[dev]) return g_slots[dev];
  int sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  const int bytes = (int)sizeof(SimtSmem);
  for (auto kernel : {simt_gemm_kernel<4>, simt_gemm_kernel<2>, simt_gemm_kernel<0>})
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
      return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, simt_gemm_kernel<4>, kThreads, bytes) !=
      cudaSuccess)
    return 0;
  g_slots[dev] = std::max(1, sms * per_sm);
  return g_slots[dev];
}

}  // namespace

int gemm_simt_fp32(float *d, const float *a, const float *b, int M, int N, int K, int lda,
                   int ldb, int ldd, cudaStream_t s) {
  CE_REQUIRE(M >= 1 && N >= 1 && K >= 1, "GEMM dims must be >= 1 (M=%d N=%d K=%d)", M, N, K);
  CE_REQUIRE(lda >= K && ldb >= K && ldd >= N, "leading dimensions too small");
  CE_REQUIRE(d && a && b, "null operand");
  const int slots = device_slots();
  if (slots <= 0) return cuda_error(cudaGetLastError(), "simt_gemm set-up");
  const SimtPlan p = plan_tiles(M, N, slots);
  if (p.width2 == 96) return launch<2>(p, d, a, b, M, N, K, lda, ldb, ldd, s);
  if (p.width2 == 64) return launch<0>(p, d, a, b, M, N, K, lda, ldb, ldd, s);
  return launch<4>(p, d, a, b, M, N, K, lda, ldb, ldd, s);
}

}  // namespace ce
