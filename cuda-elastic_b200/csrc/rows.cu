// Row kernels of the llama2c iteration: RMSNorm, softmax, GEMV and their
// one-launch fusion. All four are HBM streams (each input read once, each
// output written once), so they are written for bandwidth:
//   * one CTA per 64 KiB row, the row held in registers as float4s loaded
//     with 16-byte streaming loads (ld.global.cs), reduced with warp
//     shuffles plus one shared-memory step, written back from the same
//     registers with streaming stores -- one read and one write per element;
//   * GEMV: one warp per matrix row, 16-byte streaming loads unrolled so each
//     warp keeps 4 KiB in flight, the x vector served from L1/L2;
//   * shapes whose rows do not fit the register budget, or whose rows are
//     not 16-byte aligned, take a generic two-pass path in the same files.
// Reference kernels replaced: llama2c/llama2c_cuda_graph.cu:58-162 and the
// fused llama2c/llama2c_sota.cu:263-298.
#include "row_ops.cuh"

namespace ce {
namespace {

using namespace rowops;

constexpr int kRowThreads = 512;      // register path: threads per row
constexpr int kGenericThreads = 512;  // generic path
constexpr int kGemvUnroll = 8;        // float4 loads in flight per lane

// GEMV rows: warp w of the block computes product[row0 + w].
__device__ __forceinline__ void gemv_rows_vec(const float4 *matrix, const float4 *x, float *product,
                                              int row0, int rows, int cols4) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int row = row0 + warp; row < rows && row < row0 + nwarps; row += nwarps) {
    const float4 *m = matrix + (size_t)row * cols4;
    float acc[kGemvUnroll];
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) acc[u] = 0.f;
    int i = lane;
    for (; i + 32 * (kGemvUnroll - 1) < cols4; i += 32 * kGemvUnroll) {
      float4 a[kGemvUnroll];
#pragma unroll
      for (int u = 0; u < kGemvUnroll; ++u) a[u] = __ldcs(m + i + 32 * u);
#pragma unroll
      for (int u = 0; u < kGemvUnroll; ++u) {
        const float4 b = __ldg(x + i + 32 * u);
        acc[u] += a[u].x * b.x + a[u].y * b.y + a[u].z * b.z + a[u].w * b.w;
      }
    }
    for (; i < cols4; i += 32) {
      const float4 a = __ldcs(m + i);
      const float4 b = __ldg(x + i);
      acc[0] += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
    }
    float sum = 0.f;
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) sum += acc[u];
    sum = warp_sum(sum);
    if (lane == 0) product[row] = sum;
  }
}

// ---------------------------------------------------------------------------
// Kernels

// Work of one fused launch. Blocks [0, 2*min(nr,ns)) alternate rmsnorm and
// softmax rows, then the leftover rows of the longer list, then GEMV blocks
// of kGemvWarps rows each.
struct IterationWork {
  float *normalized;
  uint2 *normalized_bf16;
  int ld_bf16_4;  // bf16 row stride in units of 4 elements
  uint32_t *normalized_e4m3;  // E4M3 operand (4 codes per word) or nullptr
  int ld_e4m3_4;              // its row stride in units of 4 codes
  float *e4m3_scale;          // per-row dequantization scale
  const float *input;
  const float *weight;
  float *softmax;
  const float *logits;
  float *product;
  const float *matrix;
  const float *gemv_x;
  int cols;
  int rms_rows;
  int softmax_rows;
  int gemv_rows;
  float eps;
  int norm_lo, norm_hi;  // the fp32 normalized output covers rmsnorm rows [norm_lo, norm_hi)
  // block-scaled GEMM operands from the normalized rows (RowsExtras)
  uint8_t *mx_operand;   // MXFP6 packed operand [rms_rows][mx_ld bytes], or nullptr
  int mx_ld;
  uint8_t *mx_atoms;     // its UE8M0 scale atoms
  int katoms;
  unsigned int *amax_bits;  // max |normalized| over the launch (NVFP4 pass 1), or nullptr
  int keep_normalized;      // fp32 normalized with L2-resident stores (read again next)
};

// The rmsnorm row's extra outputs, from its normalized values in registers.
template <int NV>
__device__ __forceinline__ void rms_extras(const IterationWork &w, const float4 (&o)[NV], int row, int cols4,
                                           float *scratch) {
  if (w.mx_operand != nullptr)
    mxfp6_row<NV>(o, w.mx_operand + (size_t)row * w.mx_ld, w.mx_atoms, row, w.katoms, cols4);
  if (w.amax_bits != nullptr) {
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      if (i < cols4) m = fmaxf(m, fmaxf(fmaxf(fabsf(o[j].x), fabsf(o[j].y)), fmaxf(fabsf(o[j].z), fabsf(o[j].w))));
    }
    m = block_max(m, scratch);
    if (threadIdx.x == 0) atomicMax(w.amax_bits, __float_as_uint(m));  // m >= 0: bits order as values
  }
}

// rmsnorm_row (row_ops.cuh) with the normalized values kept in registers for
// rms_extras; the same arithmetic, so the same bits.
template <int NV>
__device__ __forceinline__ void rmsnorm_row_extras(const IterationWork &w, int row, float *scratch) {
  const int cols4 = w.cols >> 2;
  float4 v[NV];
  load_row<NV>(v, reinterpret_cast<const float4 *>(w.input) + (size_t)row * cols4, cols4);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  ss = block_sum(ss, scratch);
  const float scale = 1.0f / sqrtf(ss / (float)w.cols + w.eps);
  float4 *out = (w.normalized != nullptr && row >= w.norm_lo && row < w.norm_hi)
                    ? reinterpret_cast<float4 *>(w.normalized) + (size_t)row * cols4 : nullptr;
  const float4 *wt = reinterpret_cast<const float4 *>(w.weight);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4) {
      const float4 g = __ldg(wt + i);
      v[j].x = g.x * (scale * v[j].x);
      v[j].y = g.y * (scale * v[j].y);
      v[j].z = g.z * (scale * v[j].z);
      v[j].w = g.w * (scale * v[j].w);
      if (out != nullptr) {
        if (w.keep_normalized) out[i] = v[j];
        else __stcs(out + i, v[j]);
      }
    }
  }
  rms_extras<NV>(w, v, row, cols4, scratch);
}

template <int NV>
__global__ void __launch_bounds__(kRowThreads, (NV <= 8 ? 2 : 1))
iteration_kernel(IterationWork w) {
  __shared__ float scratch[32];
  const int cols4 = w.cols >> 2;
  int b = blockIdx.x;
  const int both = min(w.rms_rows, w.softmax_rows);
  int rms_row = -1, soft_row = -1;
  if (b < 2 * both) {
    if (b & 1) soft_row = b >> 1; else rms_row = b >> 1;
  } else {
    b -= 2 * both;
    const int extra_rms = w.rms_rows - both, extra_soft = w.softmax_rows - both;
    if (b < extra_rms) {
      rms_row = both + b;
    } else if (b < extra_rms + extra_soft) {
      soft_row = both + (b - extra_rms);
    } else {
      b -= extra_rms + extra_soft;
      gemv_rows_vec(reinterpret_cast<const float4 *>(w.matrix),
                    reinterpret_cast<const float4 *>(w.gemv_x), w.product,
                    b * (int)(blockDim.x >> 5), w.gemv_rows, cols4);
      return;
    }
  }
  float *const normalized = rms_row >= w.norm_lo && rms_row < w.norm_hi ? w.normalized : nullptr;
  if (rms_row >= 0 && w.normalized_e4m3 != nullptr) {
    const size_t off = (size_t)rms_row * cols4;
    rmsnorm_row_e4m3<NV>(reinterpret_cast<const float4 *>(w.input) + off,
                         reinterpret_cast<const float4 *>(w.weight),
                         normalized ? reinterpret_cast<float4 *>(normalized) + off : nullptr,
                         w.normalized_e4m3 + (size_t)rms_row * w.ld_e4m3_4, w.e4m3_scale + rms_row,
                         cols4, w.cols, w.eps, scratch);
  } else if (rms_row >= 0 && (w.mx_operand != nullptr || w.amax_bits != nullptr)) {
    rmsnorm_row_extras<NV>(w, rms_row, scratch);
  } else if (rms_row >= 0) {
    const size_t off = (size_t)rms_row * cols4;
    rmsnorm_row<NV>(reinterpret_cast<const float4 *>(w.input) + off,
                    reinterpret_cast<const float4 *>(w.weight),
                    normalized ? reinterpret_cast<float4 *>(normalized) + off : nullptr,
                    w.normalized_bf16 ? w.normalized_bf16 + (size_t)rms_row * w.ld_bf16_4 : nullptr,
                    cols4, w.cols, w.eps, scratch);
  } else {
    const size_t off = (size_t)soft_row * cols4;
    softmax_row<NV>(reinterpret_cast<const float4 *>(w.logits) + off,
                    reinterpret_cast<float4 *>(w.softmax) + off, cols4, scratch);
  }
}

// ---------------------------------------------------------------------------
// Streaming rows kernel for long rows (the trio's rows stage at the sheet
// shape: 64 KiB per row). A persistent grid, one 512-thread CTA per SM, walks
// the launch's row list (rmsnorm and softmax rows interleaved as in
// iteration_kernel) with a stride of the grid. Rows arrive in a ring of
// kRingRows shared-memory buffers filled by bulk copies issued two rows
// ahead, so each SM always has loads in flight while it reduces the current
// row from registers and streams its results out. Each thread owns the same
// float4 slots as in iteration_kernel and does the same arithmetic in the
// same order, so the results are the same bits. The RMSNorm weight stays in
// registers for the whole launch.
constexpr int kRingRows = 3;
static __device__ DeviceStatus g_rows_status;

__device__ __forceinline__ void bulk_row(void *smem_dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_arrive_expect_tx(bar, bytes);
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int NV>
__global__ void __launch_bounds__(kRowThreads, 1)
rows_stream_kernel(IterationWork w) {
  extern __shared__ __align__(128) uint8_t ring_raw[];
  __shared__ float scratch[32];
  __shared__ uint64_t full[kRingRows];
  const int cols4 = w.cols >> 2;
  const uint32_t row_bytes = (uint32_t)w.cols * 4u;
  const int both = min(w.rms_rows, w.softmax_rows);
  const int items = w.rms_rows + w.softmax_rows;
  // item k of the row list -> (is rmsnorm, row)
  auto item_of = [&](int k, int *row) -> bool {
    if (k < 2 * both) {
      *row = k >> 1;
      return (k & 1) == 0;
    }
    k -= 2 * both;
    if (k < w.rms_rows - both) {
      *row = both + k;
      return true;
    }
    *row = both + (k - (w.rms_rows - both));
    return false;
  };
  auto src_of = [&](int k) -> const float4 * {
    int row = 0;
    const bool rms = item_of(k, &row);
    return reinterpret_cast<const float4 *>(rms ? w.input : w.logits) + (size_t)row * cols4;
  };
  float4 *ring = reinterpret_cast<float4 *>(ring_raw);
  if (threadIdx.x == 0) {
    for (int b = 0; b < kRingRows; ++b) mbar_init(&full[b], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int first = blockIdx.x, step = gridDim.x;
  if (threadIdx.x == 0)
    for (int j = 0; j < kRingRows - 1; ++j) {
      const int k = first + j * step;
      if (k < items) bulk_row(ring + (size_t)j * cols4, src_of(k), row_bytes, &full[j]);
    }
  // the RMSNorm weight of this thread's slots, for every rmsnorm row
  float4 g[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    g[j] = (i < cols4 && w.rms_rows > 0) ? __ldg(reinterpret_cast<const float4 *>(w.weight) + i)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int n = 0;
  for (int k = first; k < items; k += step, ++n) {
    const int buf = n % kRingRows;
    // the buffer of two rows ahead was read by every thread before the last
    // row's block reductions, so it is free
    if (threadIdx.x == 0) {
      const int ahead = k + (kRingRows - 1) * step;
      if (ahead < items)
        bulk_row(ring + (size_t)((n + kRingRows - 1) % kRingRows) * cols4, src_of(ahead), row_bytes,
                 &full[(n + kRingRows - 1) % kRingRows]);
    }
    const bool landed = mbar_wait(&full[buf], (uint32_t)((n / kRingRows) & 1), &g_rows_status, 1u);
    if (!__syncthreads_and(landed)) break;  // a wait that gave up ends the CTA as a whole
    const float4 *sv = ring + (size_t)buf * cols4;
    float4 v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      v[j] = i < cols4 ? sv[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    int row = 0;
    if (item_of(k, &row)) {
      // rmsnorm_row's arithmetic
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      ss = block_sum(ss, scratch);
      const float scale = 1.0f / sqrtf(ss / (float)w.cols + w.eps);
      float4 *out = (w.normalized != nullptr && row >= w.norm_lo && row < w.norm_hi)
                        ? reinterpret_cast<float4 *>(w.normalized) + (size_t)row * cols4 : nullptr;
      uint2 *ob = w.normalized_bf16 != nullptr ? w.normalized_bf16 + (size_t)row * w.ld_bf16_4 : nullptr;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols4) {
          float4 o;
          o.x = g[j].x * (scale * v[j].x);
          o.y = g[j].y * (scale * v[j].y);
          o.z = g[j].z * (scale * v[j].z);
          o.w = g[j].w * (scale * v[j].w);
          v[j] = o;
          if (out != nullptr) {
            if (w.keep_normalized) out[i] = o;
            else __stcs(out + i, o);
          }
          if (ob != nullptr) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(o.x, o.y);
            __nv_bfloat162 hi = __floats2bfloat162_rn(o.z, o.w);
            uint2 packed;
            packed.x = *reinterpret_cast<uint32_t *>(&lo);
            packed.y = *reinterpret_cast<uint32_t *>(&hi);
            ob[i] = packed;
          }
        }
      }
      if (w.mx_operand != nullptr || w.amax_bits != nullptr) rms_extras<NV>(w, v, row, cols4, scratch);
    } else {
      // softmax_row's arithmetic
      float m = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols4) m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
      }
      m = block_max(m, scratch);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols4) {
          v[j].x = expf(v[j].x - m);
          v[j].y = expf(v[j].y - m);
          v[j].z = expf(v[j].z - m);
          v[j].w = expf(v[j].w - m);
          sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        }
      }
      sum = block_sum(sum, scratch);
      float4 *out = reinterpret_cast<float4 *>(w.softmax) + (size_t)row * cols4;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < cols4) {
          float4 o;
          o.x = v[j].x / sum;
          o.y = v[j].y / sum;
          o.z = v[j].z / sum;
          o.w = v[j].w / sum;
          __stcs(out + i, o);
        }
      }
    }
  }
  // every bulk copy this CTA issued has landed before it exits
  for (int j = n; j < n + kRingRows; ++j) {
    const int k = first + j * step;
    if (k < items) mbar_wait(&full[j % kRingRows], (uint32_t)((j / kRingRows) & 1), &g_rows_status, 2u);
  }
}

// Generic path: any cols, any alignment, rows longer than the register
// budget. One 512-thread block per row; RMSNorm reads its row twice
// (sum of squares, then scale), softmax runs an online max/sum pass then a
// write pass. GEMV: warp per row, scalar loads.
__global__ void __launch_bounds__(kGenericThreads)
generic_rmsnorm_kernel(float *out, __nv_bfloat16 *out_bf16, int ld_bf16, const float *x,
                       const float *w, int rows, int cols, float eps, int norm_lo, int norm_hi) {
  __shared__ float scratch[32];
  const int row = blockIdx.x;
  if (row >= rows) return;
  if (row < norm_lo || row >= norm_hi) out = nullptr;
  const float *xr = x + (size_t)row * cols;
  float ss = 0.f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    const float v = xr[i];
    ss += v * v;
  }
  ss = block_sum(ss, scratch);
  const float scale = 1.0f / sqrtf(ss / (float)cols + eps);
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    const float o = w[i] * (scale * xr[i]);
    if (out) out[(size_t)row * cols + i] = o;
    if (out_bf16) out_bf16[(size_t)row * ld_bf16 + i] = __float2bfloat16_rn(o);
  }
}

__global__ void __launch_bounds__(kGenericThreads)
generic_softmax_kernel(float *out, const float *logits, int rows, int cols) {
  __shared__ float sm[32], ss[32];
  const int row = blockIdx.x;
  if (row >= rows) return;
  const float *l = logits + (size_t)row * cols;
  // Online pass: running maximum m and sum s of exp(l - m).
  float m = -FLT_MAX, s = 0.f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    const float v = l[i];
    if (v > m) {
      s = s * expf(m - v) + 1.0f;
      m = v;
    } else {
      s += expf(v - m);
    }
  }
  // Combine (m, s) pairs across the block.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = s * expf(m - mm) + s2 * expf(m2 - mm);
    m = mm;
  }
  if (lane == 0) { sm[warp] = m; ss[warp] = s; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -FLT_MAX;
    s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = s * expf(m - mm) + s2 * expf(m2 - mm);
      m = mm;
    }
    if (lane == 0) { sm[0] = m; ss[0] = s; }
  }
  __syncthreads();
  m = sm[0];
  s = ss[0];
  float *o = out + (size_t)row * cols;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) o[i] = expf(l[i] - m) / s;
}

__global__ void __launch_bounds__(kGenericThreads)
generic_gemv_kernel(float *product, const float *matrix, const float *x, int rows, int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= rows) return;
  const float *m = matrix + (size_t)row * cols;
  float acc = 0.f;
  for (int i = lane; i < cols; i += 32) acc += __ldcs(m + i) * __ldg(x + i);
  acc = warp_sum(acc);
  if (lane == 0) product[row] = acc;
}

// Pads columns [cols, ld) of a bf16 matrix with zeros.
__global__ void pad_bf16_kernel(__nv_bfloat16 *out, int rows, int cols, int ld) {
  const int pad = ld - cols;
  const size_t total = (size_t)rows * pad;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / pad, c = cols + i % pad;
    out[r * ld + c] = __float2bfloat16_rn(0.f);
  }
}

__global__ void convert_bf16_kernel(__nv_bfloat16 *out, const float *in, int rows, int cols,
                                    int ld) {
  const size_t total = (size_t)rows * ld;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / ld, c = i % ld;
    out[i] = __float2bfloat16_rn(c < (size_t)cols ? in[r * cols + c] : 0.f);
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Picks float4 slots per thread (NV) and threads per row for the register
// path; returns 0 if the row is too long (generic path).
int pick_nv(int cols4, int *threads) {
  static const int kNv[] = {1, 2, 4, 8, 16};
  for (int nv : kNv) {
    const int need = (cols4 + nv - 1) / nv;
    if (need <= kRowThreads) {
      *threads = ((need + 31) / 32) * 32;
      if (*threads < 32) *threads = 32;
      return nv;
    }
  }
  return 0;
}

// The streaming kernel for launches of long rmsnorm / softmax rows only
// (32 to 64 KiB), with the thread count and slots iteration_kernel would use
// (hence the same bits).
int g_stream_rows = 1;  // ce_rows_tuning

bool stream_rows_apply(const IterationWork &w, int nv, int threads) {
  const int cols4 = w.cols >> 2;
  return g_stream_rows && w.gemv_rows == 0 && w.normalized_e4m3 == nullptr && threads >= 256 && threads <= kRowThreads &&
         nv <= 8 && cols4 >= 2048 && w.rms_rows + w.softmax_rows > 0;
}

template <int NV>
int launch_stream_nv(const IterationWork &w, int threads, cudaStream_t s) {
  const size_t smem = (size_t)kRingRows * w.cols * 4;
  static bool configured[64] = {};
  int dev = 0;
  CE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    CE_CUDA_TRY(cudaFuncSetAttribute(rows_stream_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)((size_t)kRingRows * 16384 * 4)));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int items = w.rms_rows + w.softmax_rows;
  const int grid = items < sm_count() ? items : sm_count();
  rows_stream_kernel<NV><<<grid, threads, smem, s>>>(w);
  CE_LAUNCH_CHECK("rows_stream_kernel");
  return CE_OK;
}

int launch_stream(const IterationWork &w, int nv, int threads, cudaStream_t s) {
  switch (nv) {
    case 4: return launch_stream_nv<4>(w, threads, s);
    case 8: return launch_stream_nv<8>(w, threads, s);
  }
  return set_error(CE_ERR_USAGE, std::string("internal: bad vector count for the streaming rows kernel"));
}

int launch_iteration(const IterationWork &w, int nv, int threads, cudaStream_t s) {
  if (stream_rows_apply(w, nv, threads)) return launch_stream(w, nv, threads, s);
  const int both = w.rms_rows < w.softmax_rows ? w.rms_rows : w.softmax_rows;
  const int row_blocks = 2 * both + (w.rms_rows - both) + (w.softmax_rows - both);
  const int warps = threads / 32;
  const int gemv_blocks = w.gemv_rows > 0 ? (w.gemv_rows + warps - 1) / warps : 0;
  const int grid = row_blocks + gemv_blocks;
  if (grid == 0) return CE_OK;
  switch (nv) {
    case 1: iteration_kernel<1><<<grid, threads, 0, s>>>(w); break;
    case 2: iteration_kernel<2><<<grid, threads, 0, s>>>(w); break;
    case 4: iteration_kernel<4><<<grid, threads, 0, s>>>(w); break;
    case 8: iteration_kernel<8><<<grid, threads, 0, s>>>(w); break;
    case 16: iteration_kernel<16><<<grid, threads, 0, s>>>(w); break;
    default: return set_error(CE_ERR_USAGE, std::string("internal: bad vector count"));
  }
  CE_LAUNCH_CHECK("iteration_kernel");
  return CE_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Entry points used by capi.cu

int rows_iteration(float *normalized, uint16_t *normalized_bf16, int ld_bf16, const float *input,
                   const float *weight, float *softmax, const float *logits, float *product,
                   const float *matrix, const float *gemv_x, int batch_rms, int batch_softmax,
                   int cols, int gemv_rows, float eps, cudaStream_t s, uint8_t *normalized_e4m3,
                   int ld_e4m3, float *e4m3_scale, int norm_lo, int norm_hi, const RowsExtras *extras) {
  CE_REQUIRE(cols >= 1, "cols must be >= 1 (got %d)", cols);
  CE_REQUIRE(batch_rms >= 0 && batch_softmax >= 0 && gemv_rows >= 0, "negative row count");
  const bool ex_out = extras != nullptr && (extras->mx_operand != nullptr || extras->amax_bits != nullptr);
  if (batch_rms > 0)
    CE_REQUIRE(input && weight && (normalized || normalized_bf16 || normalized_e4m3 || ex_out),
               "rmsnorm needs input, weight and an output");
  if (extras != nullptr && extras->mx_operand != nullptr)
    CE_REQUIRE(extras->mx_atoms != nullptr && cols % 32 == 0 && extras->mx_ld >= cols && extras->mx_ld % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(extras->mx_operand) & 15u) == 0,
               "the fused MXFP6 operand needs its scale atoms, cols %% 32 == 0 and 16-byte rows");
  if (batch_softmax > 0) CE_REQUIRE(logits && softmax, "softmax needs logits and an output");
  if (gemv_rows > 0) CE_REQUIRE(matrix && gemv_x && product, "gemv needs matrix, x and product");
  if (normalized_bf16) CE_REQUIRE(ld_bf16 >= cols && ld_bf16 % 8 == 0, "bf16 leading dimension must be >= cols and a multiple of 8 (got %d)", ld_bf16);
  if (normalized_e4m3) {
    CE_REQUIRE(ld_e4m3 >= cols && ld_e4m3 % 16 == 0, "e4m3 leading dimension must be >= cols and a multiple of 16 (got %d)", ld_e4m3);
    CE_REQUIRE(e4m3_scale != nullptr && normalized_bf16 == nullptr, "e4m3 operand needs a scale buffer and excludes the bf16 operand");
    CE_REQUIRE(cols % 4 == 0 && cols / 4 <= 16 * kRowThreads, "the e4m3 operand needs cols %% 4 == 0 and cols <= 32768 (got %d)", cols);
  }
  int threads = 0;
  const int nv = (cols % 4 == 0) ? pick_nv(cols / 4, &threads) : 0;
  const bool vec = nv > 0 && aligned16(normalized) && aligned16(input) && aligned16(weight) &&
                   aligned16(softmax) && aligned16(logits) && aligned16(matrix) &&
                   aligned16(gemv_x) && aligned16(normalized_bf16) && aligned16(normalized_e4m3);
  if (normalized_e4m3 != nullptr && !vec)
    return set_error(CE_ERR_USAGE, std::string("the e4m3 operand needs 16-byte aligned rows"));
  if (ex_out && !vec)
    return set_error(CE_ERR_USAGE, std::string("the fused block-scaled operands need 16-byte aligned rows"));
  if (vec) {
    IterationWork w;
    w.normalized = normalized;
    w.normalized_bf16 = reinterpret_cast<uint2 *>(normalized_bf16);
    w.ld_bf16_4 = ld_bf16 / 4;
    w.normalized_e4m3 = reinterpret_cast<uint32_t *>(normalized_e4m3);
    w.ld_e4m3_4 = ld_e4m3 / 4;
    w.e4m3_scale = e4m3_scale;
    w.input = input;
    w.weight = weight;
    w.softmax = softmax;
    w.logits = logits;
    w.product = product;
    w.matrix = matrix;
    w.gemv_x = gemv_x;
    w.cols = cols;
    w.rms_rows = batch_rms;
    w.softmax_rows = batch_softmax;
    w.gemv_rows = gemv_rows;
    w.eps = eps;
    w.norm_lo = norm_lo;
    w.norm_hi = norm_hi;
    const RowsExtras none;
    const RowsExtras &ex = extras != nullptr ? *extras : none;
    w.mx_operand = ex.mx_operand;
    w.mx_ld = ex.mx_ld;
    w.mx_atoms = ex.mx_atoms;
    w.katoms = ex.katoms;
    w.amax_bits = ex.amax_bits;
    w.keep_normalized = ex.keep_normalized;
    // At least 256 threads per block whatever the launch contains, so the
    // reduction order of a row (and so its bits) does not depend on whether
    // GEMV blocks share the launch; the GEMV blocks use the same size.
    if (threads < 256) threads = 256;
    int rc = launch_iteration(w, nv, threads, s);
    if (rc != CE_OK) return rc;
  } else {
    if (batch_rms > 0) {
      generic_rmsnorm_kernel<<<batch_rms, kGenericThreads, 0, s>>>(
          normalized, reinterpret_cast<__nv_bfloat16 *>(normalized_bf16), ld_bf16, input, weight,
          batch_rms, cols, eps, norm_lo, norm_hi);
      CE_LAUNCH_CHECK("generic_rmsnorm_kernel");
    }
    if (batch_softmax > 0) {
      generic_softmax_kernel<<<batch_softmax, kGenericThreads, 0, s>>>(softmax, logits,
                                                                      batch_softmax, cols);
      CE_LAUNCH_CHECK("generic_softmax_kernel");
    }
    if (gemv_rows > 0) {
      const int warps = kGenericThreads / 32;
      generic_gemv_kernel<<<(gemv_rows + warps - 1) / warps, kGenericThreads, 0, s>>>(
          product, matrix, gemv_x, gemv_rows, cols);
      CE_LAUNCH_CHECK("generic_gemv_kernel");
    }
  }
  if (normalized_e4m3 && ld_e4m3 > cols && batch_rms > 0) {
    CE_CUDA_TRY(cudaMemset2DAsync(normalized_e4m3 + cols, (size_t)ld_e4m3, 0, (size_t)(ld_e4m3 - cols),
                                  batch_rms, s));
  }
  if (normalized_bf16 && ld_bf16 > cols && batch_rms > 0) {
    pad_bf16_kernel<<<256, 256, 0, s>>>(reinterpret_cast<__nv_bfloat16 *>(normalized_bf16),
                                        batch_rms, cols, ld_bf16);
    CE_LAUNCH_CHECK("pad_bf16_kernel");
  }
  return CE_OK;
}

// Synchronizes the device, reads and clears the status word of the
// streaming rows kernel (a bulk-copy wait that gave up).
int rows_status() {
  CE_CUDA_TRY(cudaDeviceSynchronize());
  DeviceStatus h{};
  CE_CUDA_TRY(cudaMemcpyFromSymbol(&h, g_rows_status, sizeof(h)));
  if (h.code == 0) return CE_OK;
  const DeviceStatus zero{};
  CE_CUDA_TRY(cudaMemcpyToSymbol(g_rows_status, &zero, sizeof(zero)));
  return set_error(CE_ERR_TIMEOUT, format("rows kernel bulk-copy wait %u gave up in block %u", h.where, h.block));
}

int rows_set_wait_limit(unsigned long long ns) { return set_wait_limit_here(ns); }

int rows_set_streaming(int on) {
  g_stream_rows = on != 0;
  return CE_OK;
}

int convert_bf16(uint16_t *out, const float *in, int rows, int cols, int ld, cudaStream_t s) {
  CE_REQUIRE(rows >= 1 && cols >= 1 && ld >= cols, "bad conversion shape %dx%d ld %d", rows, cols, ld);
  const size_t total = (size_t)rows * ld;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  convert_bf16_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<__nv_bfloat16 *>(out), in, rows,
                                             cols, ld);
  CE_LAUNCH_CHECK("convert_bf16_kernel");
  return CE_OK;
}

}  // namespace ce
