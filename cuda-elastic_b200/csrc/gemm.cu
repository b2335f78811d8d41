// Tensor-core GEMM for sm_100a: D[m][n] = sum_k A[m][k] * B[n][k].
//
// This is the B200 engine behind the reference's classifier / matmul GEMMs
// (applications/loom_private/decoder/decoder_optimized.cu:343-439, SIMT
// SGEMM with stream-K; experiments/blackwell/lowprec/decoder_lowprec.cu:85-127,
// CUTLASS mma.sync / SM120 GEMMs). Design:
//   * persistent kernel, one CTA per SM, static round-robin tile schedule
//     (tile t -> m block t % tiles_m, n block t / tiles_m, so the CTAs that
//     run together share B tiles through L2);
//   * warp specialisation, 192 threads: warp 0 = TMA producer, warp 1 = TMEM
//     allocator + tcgen05.mma issuer, warps 2-5 = epilogue (tcgen05.ld ->
//     registers -> global);
//   * operands staged by TMA (cp.async.bulk.tensor, no multicast) into a
//     kStages ring of 128-byte-swizzled K-major tiles, 128 bytes of K per
//     stage whatever the element type;
//   * accumulators in TMEM, two buffers of BN fp32 columns, so the epilogue
//     of tile i overlaps the main loop of tile i + 1;
//   * every mbarrier wait is bounded (common.cuh); a wait that gives up
//     records CE_ERR_TIMEOUT in g_gemm_status, the CTA drains its own TMA
//     copies and MMAs (bounded), frees its TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace ce {

static __device__ DeviceStatus g_gemm_status;

namespace {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr int kRowBytes = 128;  // K bytes per stage (one swizzle row)

// Operand kinds: 0 = bf16 (kind::f16), 1 = fp32 as tf32 (kind::tf32),
// 2 = fp8 e4m3 (kind::f8f6f4).
template <int kKind>
struct Kind;
template <>
struct Kind<0> {
  static constexpr int elem = 2;
  static constexpr uint32_t fmt = 1;  // BF16
};
template <>
struct Kind<1> {
  static constexpr int elem = 4;
  static constexpr uint32_t fmt = 2;  // TF32
};
template <>
struct Kind<2> {
  static constexpr int elem = 1;
  static constexpr uint32_t fmt = 0;  // E4M3
};
template <>
struct Kind<3> {
  static constexpr int elem = 2;
  static constexpr uint32_t fmt = 0;  // F16 (kind::f16 with fp16 operands)
};

// Shared memory of the row-shard fan-out epilogue: one padded 32 x 33 fp32
// transpose tile per epilogue warp.
constexpr int kFanTile = 32 * 33;
constexpr int kFanBytes = 4 * kFanTile * 4;

template <int BN, int FAN = 0>
struct Smem {
  static constexpr int a_bytes = BM * kRowBytes;
  static constexpr int b_bytes = BN * kRowBytes;
  static constexpr int stage_bytes = a_bytes + b_bytes;
  static constexpr int max_stages = (232448 - 2048 - FAN * kFanBytes) / stage_bytes;
  static constexpr int stages = max_stages > 8 ? 8 : max_stages;
  static constexpr int bar_offset = stages * stage_bytes;
  // full[kStages], empty[kStages], tmem_full[2], tmem_empty[2], drain, tmem holder
  static constexpr int fan_offset = bar_offset + 256;
  static constexpr int total = fan_offset + FAN * kFanBytes + 1024;  // + alignment slack
};

// Instruction descriptor (kind::f16 / tf32 / f8f6f4): D fp32 (bits 4-5 = 1),
// A and B format (bits 7-9, 10-12), both K-major (bits 15, 16 = 0),
// N >> 3 (bits 17-22), M >> 4 (bits 24-28).
template <int kKind, int BN>
__host__ __device__ constexpr uint32_t instr_desc() {
  return (1u << 4) | (Kind<kKind>::fmt << 7) | (Kind<kKind>::fmt << 10) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

struct GemmArgs {
  float *d;
  const float *row_scale;  // optional per-m scale (nullptr = 1)
  const float *col_scale;  // optional per-n scale (nullptr = 1)
  const float *alpha;      // optional scalar scale on the device (nullptr = 1)
  int M, N, K, ldd;
  int tiles_m, tiles_n, k_blocks;
  int prefetch;  // L2 prefetch distance in k-blocks (0 = none)
  int splits;    // k ranges per tile (split-K); split s writes d + s * split_stride
  long long split_stride;
  // Epilogue 1 (SwiGLU): the B rows interleave w1 and w3, so output columns
  // (2i, 2i+1) are (g_i, u_i); the epilogue writes bf16(silu(g_i) * u_i) to
  // column i of out_bf16 (row stride ld_out) instead of the fp32 d.
  int epilogue;
  uint16_t *out_bf16;  // bf16, or fp16 when out_f16
  int ld_out;
  int out_f16;
  // Row-shard fan-out (ce_plan_gemm_rowx): d points into this rank's block
  // of the exchange, and every output row piece is also stored at the same
  // offset of each peer's block (rx.world <= 1: none).
  RowxSync rx;
};

// 32 consecutive fp32 outputs of one row (n_valid of them inside the matrix).
__device__ __forceinline__ void store_row32(float *dst, const float (&v)[32], int n_valid, bool vec) {
  if (vec && n_valid >= 32) {
    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n_valid) dst[j] = v[j];
  }
}

// The epilogue's plain output: this rank's d, then (row-shard fan-out) the
// same offset of every peer's block.
__device__ __forceinline__ void store_out32(const GemmArgs &args, float *dst, const float (&v)[32], int n_valid,
                                            bool vec, bool peers) {
  store_row32(dst, v, n_valid, vec);
  if (peers) {
    const ptrdiff_t off = dst - reinterpret_cast<float *>(args.rx.blocks[args.rx.rank]);
    for (int q = 0; q < args.rx.world; ++q)
      if (q != args.rx.rank) store_row32(reinterpret_cast<float *>(args.rx.blocks[q]) + off, v, n_valid, vec);
  }
}

// Row-shard fan-out through shared memory: the warp's 32 rows x 32 columns
// (lane = row, v = its 32 columns starting at col0) are transposed through a
// padded 32 x 33 tile, then written one row per instruction with lanes on
// consecutive columns -- a full 128-byte segment per destination (this rank
// and every peer), which NVLink carries far better than the lane-per-row
// 16-byte pieces of store_out32. row0: the warp's first row.
__device__ __forceinline__ void store_fan32(const GemmArgs &args, float *tile, float *d, int row0, int col0,
                                            const float (&v)[32], bool peers) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 32; ++j) tile[lane * 33 + j] = v[j];
  __syncwarp();
  float *const own = reinterpret_cast<float *>(args.rx.blocks[args.rx.rank]);
  const bool col_ok = col0 + lane < args.N;
#pragma unroll 4
  for (int r = 0; r < 32; ++r) {
    const int row = row0 + r;
    if (row < args.M && col_ok) {
      const float x = tile[r * 33 + lane];
      float *dst = d + (size_t)row * args.ldd + col0 + lane;
      *dst = x;
      if (peers) {
        const ptrdiff_t off = dst - own;
        for (int q = 0; q < args.rx.world; ++q)
          if (q != args.rx.rank) reinterpret_cast<float *>(args.rx.blocks[q])[off] = x;
      }
    }
  }
  __syncwarp();
}

// SwiGLU epilogue of one row's 32 accumulator columns starting at col0 (even).
__device__ __forceinline__ void store_swiglu(const GemmArgs &args, int row, int col0, const float (&v)[32]) {
  uint16_t *orow = args.out_bf16 + (size_t)row * args.ld_out;
  uint32_t packed[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float g0 = v[4 * k], u0 = v[4 * k + 1], g1 = v[4 * k + 2], u1 = v[4 * k + 3];
    const float h0 = g0 / (1.0f + expf(-g0)) * u0, h1 = g1 / (1.0f + expf(-g1)) * u1;
    if (args.out_f16) {
      __half2 h = __floats2half2_rn(h0, h1);
      packed[k] = *reinterpret_cast<uint32_t *>(&h);
    } else {
      __nv_bfloat162 h = __floats2bfloat162_rn(h0, h1);
      packed[k] = *reinterpret_cast<uint32_t *>(&h);
    }
  }
  const int oc = col0 / 2;
  if (col0 + 32 <= args.N && (args.ld_out & 7) == 0 && (reinterpret_cast<uintptr_t>(orow) & 15u) == 0) {
    uint4 *dst = reinterpret_cast<uint4 *>(orow + oc);
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (col0 + 2 * k + 1 < args.N) orow[oc + k] = (uint16_t)(packed[k / 2] >> (16 * (k & 1)));
  }
}

// Work unit u of a launch: output tile u % tiles, k-block range of split
// u / tiles (balanced, never empty: splits <= k_blocks).
struct Unit {
  int tile, kb0, kb1;
  float *d;
};

__device__ __forceinline__ Unit unit_of(const GemmArgs &args, int u) {
  const int tiles = args.tiles_m * args.tiles_n;
  const int split = u / tiles;
  Unit w;
  w.tile = u - split * tiles;
  w.kb0 = (int)((long long)split * args.k_blocks / args.splits);
  w.kb1 = (int)((long long)(split + 1) * args.k_blocks / args.splits);
  w.d = args.d + (size_t)split * (size_t)args.split_stride;
  return w;
}

template <int kKind, int BN, int FAN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            GemmArgs args) {
  using S = Smem<BN, FAN>;
  constexpr int kElemsPerRow = kRowBytes / Kind<kKind>::elem;  // K elements per stage
  constexpr int kUmmaK = 32 / Kind<kKind>::elem;               // K elements per MMA
  constexpr int kMmasPerStage = kElemsPerRow / kUmmaK;         // = 4
  constexpr uint32_t kIdesc = instr_desc<kKind, BN>();
  constexpr uint32_t kAccStride = 256;                         // TMEM columns per buffer

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::bar_offset);
  uint64_t *empty = full + S::stages;
  uint64_t *tmem_full = empty + S::stages;
  uint64_t *tmem_empty = tmem_full + 2;
  uint64_t *drain = tmem_empty + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

  DeviceStatus *st = &g_gemm_status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = args.tiles_m * args.tiles_n * args.splits;  // work units

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // Programmatic launch: warm L2 with this CTA's first B k-blocks (an L2
  // prefetch is safe whatever runs before), then wait for the predecessor.
  if (warp == 0 && lane == 0 && (int)blockIdx.x < num_tiles) {
    const Unit w = unit_of(args, blockIdx.x);
    const int n0 = (w.tile / args.tiles_m) * BN;
    for (int kb = w.kb0; kb < w.kb1 && kb < w.kb0 + S::stages; ++kb)
      tma_prefetch_2d(&tmB, kb * kElemsPerRow, n0);
  }
  pdl_launch_dependents();
  pdl_wait();
  if (args.rx.world > 1 && threadIdx.x == 0) rowx_signal_ready(args.rx);

  if (warp == 0) {
    // ---------------- TMA producer (lane 0 issues; the warp stays converged)
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_tiles && okay; t += gridDim.x) {
      const Unit w = unit_of(args, t);
      const int m0 = (w.tile % args.tiles_m) * BM;
      const int n0 = (w.tile / args.tiles_m) * BN;
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&empty[stage], phase ^ 1u, st, 1)) {
          okay = false;
          break;
        }
        if (lane == 0) {
          uint8_t *a_dst = smem + stage * S::stage_bytes;
          uint8_t *b_dst = a_dst + S::a_bytes;
          if (args.prefetch > 0 && kb + args.prefetch < w.kb1) {
            tma_prefetch_2d(&tmA, (kb + args.prefetch) * kElemsPerRow, m0);
            tma_prefetch_2d(&tmB, (kb + args.prefetch) * kElemsPerRow, n0);
          }
          mbar_arrive_expect_tx(&full[stage], S::stage_bytes);
          tma_load_2d(a_dst, &tmA, &full[stage], kb * kElemsPerRow, m0);
          tma_load_2d(b_dst, &tmB, &full[stage], kb * kElemsPerRow, n0);
        }
        __syncwarp();
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == S::stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Every copy this warp issued must land before the CTA can exit.
    for (int s = 0; s < S::stages; ++s)
      if (issued_mask & (1u << s)) warp_wait(&full[s], (issued_parity >> s) & 1u, st, 2);
  } else if (warp == 1) {
    // ---------------- MMA issuer (lane 0 issues)
    int stage = 0;
    uint32_t phase = 0;
    bool okay = true;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles && okay; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!warp_wait(&tmem_empty[acc], acc_phase ^ 1u, st, 3)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)acc * kAccStride;
      const Unit w = unit_of(args, t);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&full[stage], phase, st, 4)) {
          okay = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * S::stage_bytes);
          const uint32_t b_addr = a_addr + S::a_bytes;
#pragma unroll
          for (int k = 0; k < kMmasPerStage; ++k) {
            const uint64_t a_desc = smem_desc_sw128(a_addr + k * 32);
            const uint64_t b_desc = smem_desc_sw128(b_addr + k * 32);
            tc_mma<kKind>(d_tmem, a_desc, b_desc, kIdesc, ((kb - w.kb0) | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == S::stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (okay && lane == 0) tc_commit(&tmem_full[acc]);
      __syncwarp();
    }
    // All MMAs issued by this warp complete before TMEM is released.
    if (lane == 0) tc_commit(drain);
    __syncwarp();
    warp_wait(drain, 0, st, 5);
  } else {
    // ---------------- Epilogue (warps 2-5)
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    // row-shard fan-out: every peer accepts this exchange before any store
    const bool peers_ok = args.rx.world > 1 && rowx_wait_ready_warp(args.rx, st, 70);
    float *const fan_tile = reinterpret_cast<float *>(smem + S::fan_offset) + quarter * kFanTile;
    (void)fan_tile;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!warp_wait(&tmem_full[acc], acc_phase, st, 6)) break;
      tc_fence_after();
      const Unit w = unit_of(args, t);
      const int m0 = (w.tile % args.tiles_m) * BM;
      const int n0 = (w.tile / args.tiles_m) * BN;
      const int row = m0 + quarter * 32 + lane;
      const float rs = ((args.row_scale != nullptr && row < args.M) ? args.row_scale[row] : 1.0f) *
                       (args.alpha != nullptr ? *args.alpha : 1.0f);
      float *drow = w.d + (size_t)row * args.ldd;
      const bool vec_ok = ((args.ldd & 3) == 0) && ((reinterpret_cast<uintptr_t>(w.d) & 15u) == 0);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)acc * kAccStride + c, r);
        tmem_ld_wait();
        if constexpr (FAN != 0) {
          // every lane joins the transposed store, rows past M included
          const int col0 = n0 + c;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(r[j]) * rs;
            if (args.col_scale != nullptr && col0 + j < args.N) x *= args.col_scale[col0 + j];
            v[j] = x;
          }
          store_fan32(args, fan_tile, w.d, m0 + quarter * 32, col0, v, peers_ok);
        } else if (row < args.M) {
          const int col0 = n0 + c;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(r[j]) * rs;
            if (args.col_scale != nullptr && col0 + j < args.N) x *= args.col_scale[col0 + j];
            v[j] = x;
          }
          if (args.epilogue == 1) {
            store_swiglu(args, row, col0, v);
          } else {
            store_out32(args, drow + col0, v, args.N - col0, vec_ok, peers_ok);
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (args.rx.world > 1) rowx_signal_done(args.rx);
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (tcgen05 cta_group::2): a cluster of 2 CTAs on 2 SMs owns a
// 256 x (NSUB x BN) output tile. Each CTA stages its own 128 rows of A and,
// per N piece, its own BN/2 rows of B (plain TMA loads into its own shared
// memory, completion signalled on the even CTA's barrier); one thread of the
// even CTA issues M=256 MMAs that read both CTAs' shared memory and write
// both CTAs' TMEM (each holds its 128 rows x NSUB x BN fp32 accumulator). Per
// SM this halves the B bytes staged per multiply-add compared with the 1-CTA
// kernel; NSUB = 2 (two N=BN MMAs per k step on the same A tile, the whole
// 512-column TMEM as one accumulator) cuts the bytes per multiply-add by
// another ~30% for large GEMMs, at the price of an epilogue that no longer
// overlaps the next tile's main loop (one tile per pair there anyway).

template <int BN, int NSUB = 1, int FAN = 0>
struct SmemPair {
  static constexpr int a_bytes = BM * kRowBytes;
  static constexpr int b_bytes = NSUB * (BN / 2) * kRowBytes;  // NSUB pieces of BN / 2 rows
  static constexpr int stage_bytes = a_bytes + b_bytes;
  static constexpr int max_stages = (232448 - 2048 - FAN * kFanBytes) / stage_bytes;
  static constexpr int stages = max_stages > 8 ? 8 : max_stages;
  static constexpr int bar_offset = stages * stage_bytes;
  static constexpr int fan_offset = bar_offset + 256;
  static constexpr int total = fan_offset + FAN * kFanBytes + 1024;
};

template <int kKind, int BN>
__host__ __device__ constexpr uint32_t instr_desc_pair() {
  return (1u << 4) | (Kind<kKind>::fmt << 7) | (Kind<kKind>::fmt << 10) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

template <int kKind, int BN, int NSUB, int FAN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 GemmArgs args) {
  using S = SmemPair<BN, NSUB, FAN>;
  constexpr int kTileN = NSUB * BN;                  // output columns of a tile
  constexpr int kNumAcc = kTileN <= 256 ? 2 : 1;     // TMEM accumulator buffers
  constexpr uint32_t kPiece = (BN / 2) * kRowBytes;  // bytes of one N piece of B per CTA
  constexpr int kSt = S::stages;
  constexpr int kElemsPerRow = kRowBytes / Kind<kKind>::elem;
  constexpr int kUmmaK = 32 / Kind<kKind>::elem;
  constexpr int kMmasPerStage = kElemsPerRow / kUmmaK;
  constexpr uint32_t kIdesc = instr_desc_pair<kKind, BN>();
  constexpr uint32_t kAccStride = 256;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::bar_offset);
  uint64_t *empty = full + kSt;
  uint64_t *tmem_full = empty + kSt;
  uint64_t *tmem_empty = tmem_full + 2;
  uint64_t *drain = tmem_empty + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

  DeviceStatus *st = &g_gemm_status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 issues the MMAs
  const int num_tiles = args.tiles_m * args.tiles_n * args.splits;  // work units
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSt; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (warp == 0 && lane == 0 && pair < num_tiles) {  // see gemm_kernel
    const Unit w = unit_of(args, pair);
    const int n0 = (w.tile / args.tiles_m) * kTileN + (int)rank * (BN / 2);
    for (int kb = w.kb0; kb < w.kb1 && kb < w.kb0 + kSt; ++kb)
      tma_prefetch_2d(&tmB, kb * kElemsPerRow, n0);
  }
  pdl_launch_dependents();
  pdl_wait();
  if (args.rx.world > 1 && threadIdx.x == 0) rowx_signal_ready(args.rx);
  const uint32_t full0_leader = cluster_map(smem_u32(&full[0]), 0);
  const uint32_t tmem_empty0_leader = cluster_map(smem_u32(&tmem_empty[0]), 0);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool okay = true;
    for (int t = pair; t < num_tiles && okay; t += npairs) {
      const Unit w = unit_of(args, t);
      const int m0 = (w.tile % args.tiles_m) * (2 * BM) + (int)rank * BM;
      const int n0 = (w.tile / args.tiles_m) * kTileN + (int)rank * (BN / 2);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait_cluster(&empty[stage], phase ^ 1u, st, 11)) {
          okay = false;
          break;
        }
        if (lane == 0) {
          uint8_t *a_dst = smem + stage * S::stage_bytes;
          uint8_t *b_dst = a_dst + S::a_bytes;
          if (args.prefetch > 0 && kb + args.prefetch < w.kb1) {
            tma_prefetch_2d(&tmA, (kb + args.prefetch) * kElemsPerRow, m0);
            tma_prefetch_2d(&tmB, (kb + args.prefetch) * kElemsPerRow, n0);
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * S::stage_bytes);
          const uint32_t bar = full0_leader + 8u * (uint32_t)stage;
          tma_load_2d_pair(a_dst, &tmA, bar, kb * kElemsPerRow, m0);
#pragma unroll
          for (int p = 0; p < NSUB; ++p)
            tma_load_2d_pair(b_dst + p * kPiece, &tmB, bar, kb * kElemsPerRow, n0 + p * BN);
        }
        __syncwarp();
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kSt) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // The even CTA's MMAs consume every stage either CTA issued and then
    // arrive on both CTAs' empty barriers: waiting for that consumption of
    // each stage's last issue also waits for its copies to land.
    for (int s = 0; s < kSt; ++s)
      if (issued_mask & (1u << s)) warp_wait_cluster(&empty[s], (issued_parity >> s) & 1u, st, 12);
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------- MMA issuer (even CTA only)
      int stage = 0;
      uint32_t phase = 0;
      bool okay = true;
      int local = 0;
      for (int t = pair; t < num_tiles && okay; t += npairs, ++local) {
        const int acc = local % kNumAcc;
        const uint32_t acc_phase = (local / kNumAcc) & 1;
        if (!warp_wait_cluster(&tmem_empty[acc], acc_phase ^ 1u, st, 13)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)acc * kAccStride;
        const Unit w = unit_of(args, t);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!warp_wait_cluster(&full[stage], phase, st, 14)) {
            okay = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(smem + stage * S::stage_bytes);
            const uint32_t b_addr = a_addr + S::a_bytes;
#pragma unroll
            for (int k = 0; k < kMmasPerStage; ++k) {
              const uint64_t a_desc = smem_desc_sw128(a_addr + k * 32);
#pragma unroll
              for (int p = 0; p < NSUB; ++p) {
                const uint64_t b_desc = smem_desc_sw128(b_addr + p * kPiece + k * 32);
                tc_mma_pair<kKind>(d_tmem + (uint32_t)(p * BN), a_desc, b_desc, kIdesc,
                                   ((kb - w.kb0) | k) != 0 ? 1u : 0u);
              }
            }
            const uint32_t e = smem_u32(&empty[stage]);
            tc_commit_pair(cluster_map(e, 0));
            tc_commit_pair(cluster_map(e, 1));
          }
          __syncwarp();
          if (++stage == kSt) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (okay && lane == 0) {
          const uint32_t f = smem_u32(&tmem_full[acc]);
          tc_commit_pair(cluster_map(f, 0));
          tc_commit_pair(cluster_map(f, 1));
        }
        __syncwarp();
      }
      if (lane == 0) tc_commit_pair(cluster_map(smem_u32(drain), 0));
      __syncwarp();
      warp_wait_cluster(drain, 0, st, 15);
    }
  } else {
    // ---------------- Epilogue (warps 2-5 of both CTAs)
    const int quarter = warp & 3;
    const bool peers_ok = args.rx.world > 1 && rowx_wait_ready_warp(args.rx, st, 71);
    float *const fan_tile = reinterpret_cast<float *>(smem + S::fan_offset) + quarter * kFanTile;
    (void)fan_tile;
    int local = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++local) {
      const int acc = local % kNumAcc;
      const uint32_t acc_phase = (local / kNumAcc) & 1;
      if (!warp_wait_cluster(&tmem_full[acc], acc_phase, st, 16)) break;
      tc_fence_after();
      const Unit w = unit_of(args, t);
      const int m0 = (w.tile % args.tiles_m) * (2 * BM) + (int)rank * BM;
      const int n0 = (w.tile / args.tiles_m) * kTileN;
      const int row = m0 + quarter * 32 + lane;
      const float rs = ((args.row_scale != nullptr && row < args.M) ? args.row_scale[row] : 1.0f) *
                       (args.alpha != nullptr ? *args.alpha : 1.0f);
      float *drow = w.d + (size_t)row * args.ldd;
      const bool vec_ok = ((args.ldd & 3) == 0) && ((reinterpret_cast<uintptr_t>(w.d) & 15u) == 0);
#pragma unroll 1
      for (int c = 0; c < kTileN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)acc * kAccStride + c, r);
        tmem_ld_wait();
        if constexpr (FAN != 0) {
          // every lane joins the transposed store, rows past M included
          const int col0 = n0 + c;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(r[j]) * rs;
            if (args.col_scale != nullptr && col0 + j < args.N) x *= args.col_scale[col0 + j];
            v[j] = x;
          }
          store_fan32(args, fan_tile, w.d, m0 + quarter * 32, col0, v, peers_ok);
        } else if (row < args.M) {
          const int col0 = n0 + c;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(r[j]) * rs;
            if (args.col_scale != nullptr && col0 + j < args.N) x *= args.col_scale[col0 + j];
            v[j] = x;
          }
          if (args.epilogue == 1) {
            store_swiglu(args, row, col0, v);
          } else {
            store_out32(args, drow + col0, v, args.N - col0, vec_ok, peers_ok);
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      if (lane == 0) mbar_arrive_cluster(tmem_empty0_leader + 8u * (uint32_t)acc);
      __syncwarp();
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (args.rx.world > 1) rowx_signal_done(args.rx);
}

// ---------------------------------------------------------------------------
// W4A16 GEMM: NVFP4 weights (E2M1 codes, UE4M3 scale per 16 values, one fp32
// tensor decode scale alpha) against 16-bit activations, the dequantization
// fused into the GEMM. At decode sizes the weights are the only HBM stream,
// so they travel in their own deep ring, apart from the activation tiles:
//   warp 0     weight producer: bulk copies of one 64-wide k-block of the B
//              tile's codes ([kb][N][32 bytes]) and scales ([kb][N][4]), the
//              k-block-major layout of w4_pack, kW4WStages k-blocks ahead;
//   warp 10    activation producer: TMA for the fp16 A tile into the operand
//              ring (kW4OStages slots, each A plus the expanded B);
//   warps 6-9  converters: cvt.rn.f16x2.e2m1x2 and a half2 multiply by the
//              UE4M3 scale (cvt.rn.f16x2.e4m3x2) write the fp16 B operand in
//              the 128-byte-swizzled K-major layout (every product is exact:
//              at most 6 significant bits, magnitudes 2^-10 .. 2688), then a
//              proxy fence so the tensor cores see the stores;
//   warp 1     MMA issuer (kind::f16, fp16 x fp16) once A and B are in;
//   warps 2-5  epilogue: alpha x accumulator, with the split-K and SwiGLU
//              (fp16 out) modes of the bf16 GEMM.

constexpr int kW4ConvWarps = 8;
constexpr int kW4Threads = (7 + kW4ConvWarps) * 32;  // see the role list above
constexpr int kW4AProducerWarp = 6 + kW4ConvWarps;
constexpr int kW4WMaxStages = 16;  // raw weight k-blocks in flight (fewer for wide tiles)
constexpr int kW4BStages = 4;    // expanded fp16 weight tiles
constexpr int kW4AMaxStages = 16;
constexpr int kW4SmemBudget = 232448 - 1024;

template <int BN>
struct SmemW4 {
  static constexpr int b_bytes = BN * kRowBytes;        // expanded fp16 operand
  static constexpr int code_bytes = BN * 32;            // 64 E2M1 codes per row
  static constexpr int scale_bytes = BN * 4;            // 4 UE4M3 scales per row
  static constexpr int w_stage = code_bytes + scale_bytes;
  static constexpr int w_fit = 73728 / w_stage;           // about 72 KB of raw weights
  static constexpr int w_stages = w_fit > kW4WMaxStages ? kW4WMaxStages : w_fit;
  static constexpr int b_offset = 0;                    // B ring, 1 KB aligned slots
  static constexpr int w_offset = kW4BStages * b_bytes;
  static constexpr int a_offset = ((w_offset + w_stages * w_stage + 1023) / 1024) * 1024;
  static constexpr int bar_bytes = 1024;
  // A ring: slots of a_slot bytes (8 KB when M <= 64: a 64-row box; the
  // 128-row MMA then reads 8 KB past the slot, rows it never stores) up to
  // the budget, one full 16 KB tile of slack after the last slot.
  static int a_stages(int a_slot) {
    const int room = kW4SmemBudget - a_offset - bar_bytes - BM * kRowBytes;
    const int n = room / a_slot + 1;
    return n > kW4AMaxStages ? kW4AMaxStages : n;
  }
  static int total(int a_slot) { return a_offset + a_stages(a_slot) * a_slot + BM * kRowBytes - a_slot + bar_bytes + 1024; }
};

struct W4Args {
  GemmArgs g;
  const uint8_t *codes;   // [k_blocks][N][32]
  const uint8_t *scales;  // [k_blocks][N][4]
  const float *alpha;     // weight decode scale (device) or nullptr
  int a_slot;             // bytes per A ring slot (8192 or 16384)
  int a_stages;
};

__device__ __forceinline__ void bulk_g2s_gemm(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Two E2M1 codes (one byte, even index in the low nibble) to fp16x2.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t d;
  asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(d) : "r"(byte));
  return d;
}
// A UE4M3 scale byte to fp16, broadcast into both halves.
__device__ __forceinline__ uint32_t ue4m3_to_f16x2(uint32_t code) {
  uint32_t d;
  const unsigned short pair = (unsigned short)(code | (code << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(pair));
  return d;
}

template <int BN>
__global__ void __launch_bounds__(kW4Threads, 1)
gemm_w4a16_kernel(const __grid_constant__ CUtensorMap tmA, W4Args wargs) {
  using S = SmemW4<BN>;
  const GemmArgs &args = wargs.g;
  constexpr int kMmasPerStage = 4;                 // 64 fp16 of K per stage, 16 per MMA
  constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);  // fp16 x fp16 -> fp32
  constexpr uint32_t kAccStride = 256;
  const int a_stages = wargs.a_stages, a_slot = wargs.a_slot;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t *wfull = reinterpret_cast<uint64_t *>(smem + S::a_offset + a_stages * a_slot + BM * kRowBytes - a_slot);
  uint64_t *wempty = wfull + kW4WMaxStages;
  uint64_t *bready = wempty + kW4WMaxStages;
  uint64_t *bempty = bready + kW4BStages;
  uint64_t *afull = bempty + kW4BStages;
  uint64_t *aempty = afull + kW4AMaxStages;
  uint64_t *tmem_full = aempty + kW4AMaxStages;
  uint64_t *tmem_empty = tmem_full + 2;
  uint64_t *drain = tmem_empty + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

  DeviceStatus *st = &g_gemm_status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_units = args.tiles_m * args.tiles_n * args.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::w_stages; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kW4ConvWarps);
    }
    for (int s = 0; s < kW4BStages; ++s) {
      mbar_init(&bready[s], kW4ConvWarps);
      mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < a_stages; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ---------------- weight producer
    int ws = 0;
    uint32_t wph = 0, issued_mask = 0, issued_parity = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x) {
      const Unit w = unit_of(args, t);
      const int n0 = (w.tile / args.tiles_m) * BN;
      const int rows = min(BN, args.N - n0);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&wempty[ws], wph ^ 1u, st, 41)) {
          okay = false;
          break;
        }
        if (lane == 0) {
          uint8_t *c_dst = smem + S::w_offset + ws * S::w_stage;
          const size_t rowbase = (size_t)kb * args.N + n0;
          mbar_arrive_expect_tx(&wfull[ws], rows * 36);
          bulk_g2s_gemm(c_dst, wargs.codes + rowbase * 32, rows * 32, &wfull[ws]);
          bulk_g2s_gemm(c_dst + S::code_bytes, wargs.scales + rowbase * 4, rows * 4, &wfull[ws]);
        }
        __syncwarp();
        issued_mask |= 1u << ws;
        issued_parity = (issued_parity & ~(1u << ws)) | (wph << ws);
        if (++ws == S::w_stages) {
          ws = 0;
          wph ^= 1u;
        }
      }
    }
    for (int s = 0; s < S::w_stages; ++s)
      if (issued_mask & (1u << s)) warp_wait(&wfull[s], (issued_parity >> s) & 1u, st, 42);
  } else if (warp == kW4AProducerWarp) {
    // ---------------- activation producer
    int as = 0;
    uint32_t aph = 0, issued_mask = 0, issued_parity = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x) {
      const Unit w = unit_of(args, t);
      const int m0 = (w.tile % args.tiles_m) * BM;
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&aempty[as], aph ^ 1u, st, 49)) {
          okay = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&afull[as], a_slot);
          tma_load_2d(smem + S::a_offset + as * a_slot, &tmA, &afull[as], kb * 64, m0);
        }
        __syncwarp();
        issued_mask |= 1u << as;
        issued_parity = (issued_parity & ~(1u << as)) | (aph << as);
        if (++as == a_stages) {
          as = 0;
          aph ^= 1u;
        }
      }
    }
    for (int s = 0; s < a_stages; ++s)
      if (issued_mask & (1u << s)) warp_wait(&afull[s], (issued_parity >> s) & 1u, st, 50);
  } else if (warp >= 6) {
    // ---------------- converters: E2M1 x UE4M3 -> swizzled fp16
    constexpr int kConvThreads = kW4ConvWarps * 32;
    const int ct = threadIdx.x - 192;
    int ws = 0, bs = 0;
    uint32_t wph = 0, bph = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x) {
      const Unit w = unit_of(args, t);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&wfull[ws], wph, st, 43) || !warp_wait(&bempty[bs], bph ^ 1u, st, 51)) {
          okay = false;
          break;
        }
        uint8_t *b_s = smem + S::b_offset + bs * S::b_bytes;
        const uint8_t *c_s = smem + S::w_offset + ws * S::w_stage;
        const uint8_t *s_s = c_s + S::code_bytes;
#pragma unroll 2
        for (int u = ct; u < BN * 8; u += kConvThreads) {
          const int r = u >> 3, c = u & 7;  // row, 16-byte chunk (8 values) of the row
          const uint32_t q = *reinterpret_cast<const uint32_t *>(c_s + r * 32 + c * 4);
          const uint32_t sc = ue4m3_to_f16x2(s_s[r * 4 + (c >> 1)]);
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t v = e2m1x2_to_f16x2((q >> (8 * j)) & 0xFFu);
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[j]) : "r"(v), "r"(sc));
          }
          *reinterpret_cast<uint4 *>(b_s + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bready[bs]);
          mbar_arrive(&wempty[ws]);
        }
        if (++ws == S::w_stages) {
          ws = 0;
          wph ^= 1u;
        }
        if (++bs == kW4BStages) {
          bs = 0;
          bph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    int as = 0, bs = 0;
    uint32_t aph = 0, bph = 0;
    bool okay = true;
    int local = 0;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!warp_wait(&tmem_empty[acc], acc_phase ^ 1u, st, 44)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)acc * kAccStride;
      const Unit w = unit_of(args, t);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&afull[as], aph, st, 45) || !warp_wait(&bready[bs], bph, st, 46)) {
          okay = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + S::a_offset + as * a_slot);
          const uint32_t b_addr = smem_u32(smem + S::b_offset + bs * S::b_bytes);
#pragma unroll
          for (int k = 0; k < kMmasPerStage; ++k) {
            const uint64_t a_desc = smem_desc_sw128(a_addr + k * 32);
            const uint64_t b_desc = smem_desc_sw128(b_addr + k * 32);
            tc_mma<0>(d_tmem, a_desc, b_desc, kIdesc, ((kb - w.kb0) | k) != 0 ? 1u : 0u);
          }
          tc_commit(&aempty[as]);
          tc_commit(&bempty[bs]);
        }
        __syncwarp();
        if (++as == a_stages) {
          as = 0;
          aph ^= 1u;
        }
        if (++bs == kW4BStages) {
          bs = 0;
          bph ^= 1u;
        }
      }
      if (okay && lane == 0) tc_commit(&tmem_full[acc]);
      __syncwarp();
    }
    if (lane == 0) tc_commit(drain);
    __syncwarp();
    warp_wait(drain, 0, st, 47);
  } else if (warp >= 2 && warp <= 5) {
    // ---------------- epilogue (warps 2-5)
    const int quarter = warp & 3;
    const float alpha = wargs.alpha != nullptr ? *wargs.alpha : 1.0f;
    int local = 0;
    for (int t = blockIdx.x; t < num_units; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!warp_wait(&tmem_full[acc], acc_phase, st, 48)) break;
      tc_fence_after();
      const Unit w = unit_of(args, t);
      const int m0 = (w.tile % args.tiles_m) * BM;
      const int n0 = (w.tile / args.tiles_m) * BN;
      const int row = m0 + quarter * 32 + lane;
      float *drow = w.d + (size_t)row * args.ldd;
      const bool vec_ok = ((args.ldd & 3) == 0) && ((reinterpret_cast<uintptr_t>(w.d) & 15u) == 0);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)acc * kAccStride + c, r);
        tmem_ld_wait();
        if (row < args.M) {
          const int col0 = n0 + c;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * alpha;
          if (args.epilogue == 1) {
            store_swiglu(args, row, col0, v);
          } else {
            store_out32(args, drow + col0, v, args.N - col0, vec_ok, false);
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// k-block-major copy of row-major NVFP4 weights: codes [N][ld_bytes] (two
// per byte) and scales [N][nsf] -> codes_t [K/64][N][32], scales_t [K/64][N][4].
__global__ void w4_pack_kernel(uint8_t *codes_t, uint8_t *scales_t, const uint8_t *codes,
                               const uint8_t *scales, int N, int K, int ld_bytes, int nsf,
                               const int *row_map) {
  const int kbs = K / 64;
  const size_t words = (size_t)kbs * N * 8;  // 4-byte words of codes_t
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += step) {
    const size_t kb = i / ((size_t)N * 8), rem = i % ((size_t)N * 8);
    const size_t n = rem / 8, j = rem % 8;
    const size_t sr = row_map ? (size_t)row_map[n] : n;  // source row
    const uint8_t *src = codes + sr * ld_bytes + kb * 32 + j * 4;
    uint32_t v = (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16) | ((uint32_t)src[3] << 24);
    reinterpret_cast<uint32_t *>(codes_t)[i] = v;
    if (j == 0) {
      const uint8_t *ss = scales + sr * nsf + kb * 4;
      reinterpret_cast<uint32_t *>(scales_t)[kb * N + n] =
          (uint32_t)ss[0] | ((uint32_t)ss[1] << 8) | ((uint32_t)ss[2] << 16) | ((uint32_t)ss[3] << 24);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// K-major operand [outer][ld] with `inner` valid K elements; box = 128 bytes
// of K by box_outer rows, 128-byte swizzle, zero fill out of bounds.
int make_operand_map(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem,
                     int inner, int outer, int ld, int box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(CE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * (cuuint64_t)elem};
  cuuint32_t box[2] = {(cuuint32_t)(kRowBytes / elem), (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(CE_ERR_CUDA, format("cuTensorMapEncodeTiled failed (%d) for %dx%d ld %d", (int)r, outer, inner, ld));
  return CE_OK;
}

// Opts a kernel into its dynamic shared memory size. The attribute is per
// kernel and device, so the flag is per instantiation (template on the
// kernel itself) and per device.
template <auto kernel>
int configure_smem(int bytes) {
  static bool configured[64] = {};
  int dev = 0;
  CE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    CE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  return CE_OK;
}

template <int kKind, int BN, int FAN = 0>
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &args, int grid,
                cudaStream_t s, bool pdl) {
  using S = Smem<BN, FAN>;
  int rc = configure_smem<gemm_kernel<kKind, BN, FAN>>(S::total);
  if (rc) return rc;
  return launch_kernel(gemm_kernel<kKind, BN, FAN>, dim3(grid), dim3(kThreads), S::total, s, pdl,
                       "gemm_kernel", ta, tb, args);
}

template <int kKind, int BN, int NSUB = 1, int FAN = 0>
int launch_gemm_pair(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &args,
                     int grid, cudaStream_t s, bool pdl) {
  using S = SmemPair<BN, NSUB, FAN>;
  int rc = configure_smem<gemm_pair_kernel<kKind, BN, NSUB, FAN>>(S::total);
  if (rc) return rc;
  return launch_kernel(gemm_pair_kernel<kKind, BN, NSUB, FAN>, dim3(grid), dim3(kThreads), S::total, s, pdl,
                       "gemm_pair_kernel", ta, tb, args);
}

struct GemmChoice {
  int pair;  // 1: CTA-pair kernel (256-row tiles), 0: single-CTA kernel (128-row tiles)
  int bn;    // N of one MMA
  int nsub = 1;  // N pieces per tile (CTA pair only): tile width nsub x bn
};

// Kernel and tile width: minimise (waves x BN) / efficiency, where a wave is
// one tile per SM (single-CTA) or per SM pair, and the CTA-pair kernel is
// credited with its lower staging cost per multiply-add (measured: about
// 0.67 of peak tensor throughput for the single-CTA kernel).
int g_prefetch_kblocks = 0;  // set by ce_gemm_tuning (setup time)
int g_wide_tiles = 1;        // two-piece pair tiles allowed (ce_gemm_tuning)

GemmChoice choose_tiles(int M, int N, int sms, bool allow_wide = true) {
  // 96- and 64-wide tiles only enter when 128-wide tiles cannot give every
  // SM (or SM pair) a tile: decode-sized GEMMs (few rows, narrow N), where
  // more CTAs streaming the weights beat fewer wide tiles. Two-piece pair
  // tiles (2 x bn wide) enter for GEMMs whose tiles fit one wave: their
  // single accumulator buffer cannot overlap a next tile's main loop.
  static const int kCandidates[] = {256, 224, 192, 160, 128, 96, 64};
  static const int kWide[] = {256, 240, 224};
  GemmChoice best{0, 256};
  double best_cost = -1;
  auto consider = [&](int pair, int bn, int nsub, double eff) {
    const int rows = pair ? 2 * BM : BM;
    const int units = pair ? sms / 2 : sms;
    const long long tiles_m = (M + rows - 1) / rows;
    const long long tiles = tiles_m * ((N + nsub * bn - 1) / (nsub * bn));
    const long long waves = (tiles + units - 1) / units;
    if (nsub > 1 && waves > 1) return;
    const double cost = (double)(waves * nsub * bn) / eff;
    if (best_cost < 0 || cost < best_cost - 1e-9) {
      best_cost = cost;
      best = GemmChoice{pair, bn, nsub};
    }
  };
  for (int pair = 0; pair < 2; ++pair) {
    const int rows = pair ? 2 * BM : BM;
    const int units = pair ? sms / 2 : sms;
    if (pair && M <= BM) continue;
    const long long tiles_m = (M + rows - 1) / rows;
    const bool narrow_ok = tiles_m * ((N + 127) / 128) < units;
    for (int bn : kCandidates) {
      if (bn < 128 && !narrow_ok) continue;
      consider(pair, bn, 1, pair ? 0.85 : 0.67);
    }
  }
  if (M > BM && g_wide_tiles && allow_wide)
    for (int bn : kWide) consider(1, bn, 2, 0.95);
  return best;
}

template <int kKind>
int gemm_dispatch(float *d, const void *a, const void *b, int M, int N, int K, int lda, int ldb,
                  int ldd, const float *row_scale, const float *col_scale, int force_bn,
                  int force_group, cudaStream_t s, int splits = 1, long long split_stride = 0,
                  bool pdl = false, uint16_t *swiglu_out = nullptr, int swiglu_ld = 0,
                  const float *alpha = nullptr, const RowxSync *rx = nullptr) {
  constexpr int elem = Kind<kKind>::elem;
  const CUtensorMapDataType dt = kKind == 0 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : kKind == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : kKind == 3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CE_REQUIRE(M >= 1 && N >= 1 && K >= 1, "GEMM dims must be >= 1 (M=%d N=%d K=%d)", M, N, K);
  CE_REQUIRE(lda >= K && ldb >= K && ldd >= N, "leading dimensions too small");
  CE_REQUIRE((lda * elem) % 16 == 0 && (ldb * elem) % 16 == 0,
             "operand row strides must be multiples of 16 bytes (lda=%d ldb=%d)", lda, ldb);
  CE_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15u) == 0 && (reinterpret_cast<uintptr_t>(b) & 15u) == 0,
             "operand base pointers must be 16-byte aligned");
  CE_REQUIRE(d != nullptr || swiglu_out != nullptr, "null output");
  CE_REQUIRE(swiglu_out == nullptr || (splits == 1 && N % 2 == 0 && swiglu_ld >= N / 2),
             "the SwiGLU epilogue needs one split, an even N and ld_out >= N / 2");
  CE_REQUIRE(force_group >= 0 && force_group <= 3,
             "cta group must be 0 (automatic), 1, 2 or 3 (CTA pair, two N pieces per tile) (got %d)",
             force_group);
  CE_REQUIRE(force_bn == 0 || force_bn == 64 || force_bn == 96 || force_bn == 128 || force_bn == 160 ||
                 force_bn == 192 || force_bn == 224 || force_bn == 256 || (force_bn == 240 && force_group == 3),
             "tile width must be 0, 64, 96, 128, 160, 192, 224 or 256 (or 240 with two-piece tiles) (got %d)",
             force_bn);
  const int k_blocks_all = (K + (kRowBytes / elem) - 1) / (kRowBytes / elem);
  CE_REQUIRE(splits >= 1 && splits <= k_blocks_all,
             "split count must be in [1, %d] for K = %d (got %d)", k_blocks_all, K, splits);
  CE_REQUIRE(splits == 1 || split_stride >= (long long)(M - 1) * ldd + N,
             "split stride %lld is smaller than one output", split_stride);
  if (!is_sm100()) return set_error(CE_ERR_USAGE, "tcgen05 GEMM needs an sm_100 device");
  const int sms = sm_count();
  // a forced one-piece kernel takes the widths chosen among one-piece tiles
  const bool fan = rx != nullptr && rx->world > 1;
  GemmChoice c = choose_tiles(M, N, sms, (force_group == 0 || force_group == 3) && !fan);
  if (force_group != 0) {
    c.pair = force_group >= 2;
    c.nsub = force_group == 3 ? 2 : 1;
    if (c.nsub == 2 && force_bn == 0 && c.bn != 256 && c.bn != 240 && c.bn != 224) c.bn = 256;
  }
  if (force_bn != 0) c.bn = force_bn;
  if (c.nsub == 2) {
    CE_REQUIRE(c.bn == 256 || c.bn == 240 || c.bn == 224,
               "two-piece tiles take an MMA width of 224, 240 or 256 (got %d)", c.bn);
    CE_REQUIRE(M > BM, "two-piece tiles need more than %d rows (M = %d)", BM, M);
  }
  const int rows_per_tile = c.pair ? 2 * BM : BM;
  CUtensorMap ta, tb;
  int rc = make_operand_map(&ta, a, dt, elem, K, M, lda, BM);
  if (rc) return rc;
  rc = make_operand_map(&tb, b, dt, elem, K, N, ldb, c.pair ? c.bn / 2 : c.bn);
  if (rc) return rc;
  GemmArgs args;
  args.d = d;
  args.row_scale = row_scale;
  args.col_scale = col_scale;
  args.alpha = alpha;
  args.M = M;
  args.N = N;
  args.K = K;
  args.ldd = ldd;
  args.tiles_m = (M + rows_per_tile - 1) / rows_per_tile;
  args.tiles_n = (N + c.nsub * c.bn - 1) / (c.nsub * c.bn);
  args.k_blocks = (K + (kRowBytes / elem) - 1) / (kRowBytes / elem);
  args.prefetch = g_prefetch_kblocks;
  args.splits = splits;
  args.split_stride = splits > 1 ? split_stride : 0;
  args.epilogue = swiglu_out != nullptr ? 1 : 0;
  args.out_bf16 = swiglu_out;
  args.ld_out = swiglu_ld;
  args.out_f16 = kKind == 3 ? 1 : 0;
  if (rx != nullptr && rx->world > 1) {
    CE_REQUIRE(splits == 1 && swiglu_out == nullptr, "the row-shard fan-out needs one split and the plain epilogue");
    CE_REQUIRE(rx->world <= kRowxMaxRanks && rx->rank >= 0 && rx->rank < rx->world,
               "row-shard rank %d of %d is out of range", rx->rank, rx->world);
    args.rx = *rx;
  }
  const int tiles = args.tiles_m * args.tiles_n * splits;
  if constexpr (kKind == 0) {
    // bf16 fan-out: the epilogue stages its stores through shared memory
    if (fan && c.nsub == 1) {
      if (c.pair) {
        const int grid = 2 * (tiles < sms / 2 ? tiles : sms / 2);
        switch (c.bn) {
          case 256: return launch_gemm_pair<kKind, 256, 1, 1>(ta, tb, args, grid, s, pdl);
          case 224: return launch_gemm_pair<kKind, 224, 1, 1>(ta, tb, args, grid, s, pdl);
          case 192: return launch_gemm_pair<kKind, 192, 1, 1>(ta, tb, args, grid, s, pdl);
          case 160: return launch_gemm_pair<kKind, 160, 1, 1>(ta, tb, args, grid, s, pdl);
          case 128: return launch_gemm_pair<kKind, 128, 1, 1>(ta, tb, args, grid, s, pdl);
          case 96: return launch_gemm_pair<kKind, 96, 1, 1>(ta, tb, args, grid, s, pdl);
          case 64: return launch_gemm_pair<kKind, 64, 1, 1>(ta, tb, args, grid, s, pdl);
        }
      } else {
        const int grid = tiles < sms ? tiles : sms;
        switch (c.bn) {
          case 256: return launch_gemm<kKind, 256, 1>(ta, tb, args, grid, s, pdl);
          case 224: return launch_gemm<kKind, 224, 1>(ta, tb, args, grid, s, pdl);
          case 192: return launch_gemm<kKind, 192, 1>(ta, tb, args, grid, s, pdl);
          case 160: return launch_gemm<kKind, 160, 1>(ta, tb, args, grid, s, pdl);
          case 128: return launch_gemm<kKind, 128, 1>(ta, tb, args, grid, s, pdl);
          case 96: return launch_gemm<kKind, 96, 1>(ta, tb, args, grid, s, pdl);
          case 64: return launch_gemm<kKind, 64, 1>(ta, tb, args, grid, s, pdl);
        }
      }
      return set_error(CE_ERR_USAGE, format("unsupported tile width %d", c.bn));
    }
  }
  if (c.pair && c.nsub == 2) {
    const int pairs = tiles < sms / 2 ? tiles : sms / 2;
    const int grid = 2 * pairs;
    switch (c.bn) {
      case 256: return launch_gemm_pair<kKind, 256, 2>(ta, tb, args, grid, s, pdl);
      case 240: return launch_gemm_pair<kKind, 240, 2>(ta, tb, args, grid, s, pdl);
      case 224: return launch_gemm_pair<kKind, 224, 2>(ta, tb, args, grid, s, pdl);
    }
  } else if (c.pair) {
    const int pairs = tiles < sms / 2 ? tiles : sms / 2;
    const int grid = 2 * pairs;
    switch (c.bn) {
      case 256: return launch_gemm_pair<kKind, 256>(ta, tb, args, grid, s, pdl);
      case 224: return launch_gemm_pair<kKind, 224>(ta, tb, args, grid, s, pdl);
      case 192: return launch_gemm_pair<kKind, 192>(ta, tb, args, grid, s, pdl);
      case 160: return launch_gemm_pair<kKind, 160>(ta, tb, args, grid, s, pdl);
      case 128: return launch_gemm_pair<kKind, 128>(ta, tb, args, grid, s, pdl);
      case 96: return launch_gemm_pair<kKind, 96>(ta, tb, args, grid, s, pdl);
      case 64: return launch_gemm_pair<kKind, 64>(ta, tb, args, grid, s, pdl);
    }
  } else {
    const int grid = tiles < sms ? tiles : sms;
    switch (c.bn) {
      case 256: return launch_gemm<kKind, 256>(ta, tb, args, grid, s, pdl);
      case 224: return launch_gemm<kKind, 224>(ta, tb, args, grid, s, pdl);
      case 192: return launch_gemm<kKind, 192>(ta, tb, args, grid, s, pdl);
      case 160: return launch_gemm<kKind, 160>(ta, tb, args, grid, s, pdl);
      case 128: return launch_gemm<kKind, 128>(ta, tb, args, grid, s, pdl);
      case 96: return launch_gemm<kKind, 96>(ta, tb, args, grid, s, pdl);
      case 64: return launch_gemm<kKind, 64>(ta, tb, args, grid, s, pdl);
    }
  }
  return set_error(CE_ERR_USAGE, format("unsupported tile width %d", c.bn));
}


// ---------------------------------------------------------------------------
// W4A16 GEMM, decode form (gemm_w4t): d[b][n] = alpha * sum_k x[b][k] w[n][k]
// with the NVFP4 weights as the M operand of the MMA, expanded straight into
// tensor memory. At decode sizes the batch is small, so the weights are the
// 128-row operand and the batch is the N dimension (no padded rows); the
// expanded fp16 weights go registers -> TMEM (tcgen05.st) -> tensor core
// (the A operand of tcgen05.mma may live in TMEM), so shared memory only
// carries the packed weights and the activation tiles. One stage covers 128
// of K for a tile of TR weight rows (one or two M=128 halves).
//   warp 0     weight producer: one bulk copy per stage of the tile's codes
//              and scales (TR x 72 bytes, contiguous in the layout of
//              w4t_pack: a separate small copy for the scales costs the
//              SM's bulk-copy path as much as a large one); weights are
//              constant, so this starts before the programmatic-launch wait;
//   warps 1-4  MMA issuers (kind::f16, A from TMEM), each with its own
//              accumulator: one per (128-row half, 64-wide k chunk) when the
//              batch fits 64 columns, one per half up to 128, one in all
//              for 128-row tiles. A tcgen05.mma costs its issuing thread
//              ~120 cycles whatever its size at these shapes (clock-timed on
//              B200), so several issuers multiply the rate and overlap each
//              other's barrier waits; warp 1 also owns the TMEM allocation;
//   warp 5     activation producer: two TMA boxes of 64 x NB per stage
//              (first, when the activations come from the peers' exchange
//              puts, a bounded wait on their flags);
//   warps 8-11 epilogue (TMEM lane quarter = warp % 4): the chunk
//              accumulators summed in order, alpha x sum, split-K partials
//              or the SwiGLU product;
//   warps 12-27 converters, four per lane quarter, one (half, chunk) piece
//              of 64 values per row each: cvt.rn.f16x2.e2m1x2 and a half2
//              multiply by the UE4M3 scale, then tcgen05.st of 32 columns.
// The activation slot and the TMEM stage of a stage are filled under one
// barrier (TMA bytes + the converters' arrivals) and freed together by one
// tcgen05.commit per issuer.
constexpr int kW4tWarps = 28;         // roles: see gemm_w4t_kernel
constexpr int kW4tThreads = kW4tWarps * 32;
constexpr int kW4tConvWarps = 16;     // four per TMEM lane quarter
constexpr int kW4tFirstConv = 12;
constexpr int kW4tFirstEpi = 8;
constexpr int kW4tMaxStages = 4;   // activation slots = TMEM weight stages
constexpr int kW4tMaxWStages = 8;  // packed weight stages in shared memory
// Warps per TMEM lane quarter that store the CTA's last unit: the epilogue
// warp, the four converter warps and two of warps 0-7 (done by then).
constexpr int kW4tLastWorkers = 7;
constexpr int kW4tSmemBudget = 232448 - 1024;

struct W4tArgs {
  float *d;
  uint16_t *swiglu_out;  // fp16 SwiGLU product [M][ld_out], or nullptr
  const uint8_t *packed; // per 128-wide k block and 128-row group: 8 KB codes + 1 KB scales (w4t_pack)
  const float *alpha;
  int M, N, K, ldd, ld_out;
  int npad;              // packed rows (multiple of 256)
  int kb_total;          // 128-wide k blocks
  int nb;                // batch columns per tile (multiple of 16)
  int tiles_n, tiles_b, splits;
  long long split_stride;
  int stages, w_stages;
  int act_stage_bytes;   // 2 x nb x 128
  int acc_cols;          // TMEM columns before the weight stages
  int issuers;           // MMA-issuing warps, each with its own accumulator (1, 2 or 4)
  ExchangeWait xw;       // activations delivered by peers' exchange puts (flags null: local)
};

struct W4tUnit {
  int tile_n, tile_b, kb0, kb1;
  float *d;
};

__device__ __forceinline__ W4tUnit w4t_unit(const W4tArgs &a, int u) {
  W4tUnit w;
  w.tile_b = u % a.tiles_b;
  const int rest = u / a.tiles_b;
  const int split = rest % a.splits;
  w.tile_n = rest / a.splits;
  w.kb0 = (int)((long long)split * a.kb_total / a.splits);
  w.kb1 = (int)((long long)(split + 1) * a.kb_total / a.splits);
  w.d = a.d != nullptr ? a.d + (size_t)split * a.split_stride : nullptr;
  return w;
}

// Epilogue of one unit for the calling warp (TMEM lane quarter `quarter`):
// the (128-row half, 16 batch columns) chunks ci with ci % nworkers ==
// worker. The chunk accumulators are summed in order, times alpha; then the
// SwiGLU product (fp16) or the fp32 outputs / split-K partials.
template <int TR>
__device__ __forceinline__ void w4t_store_chunks(const W4tArgs &args, const W4tUnit &w, uint32_t tmem_base,
                                                 int quarter, int lane, float alpha, int worker, int nworkers) {
  constexpr int kHalves = TR / 128;
  const int NB = args.nb, per_half = args.issuers == 4 ? 2 : 1;  // accumulators per half (k chunks)
  const int b0 = w.tile_b * NB, chunks = NB / 16;
  const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
  for (int ci = worker; ci < kHalves * chunks; ci += nworkers) {
    const int h = ci / chunks, c0 = (ci % chunks) * 16;
    const int n = w.tile_n * TR + h * 128 + quarter * 32 + lane;
    uint32_t r[16], r2[16];
    float v[16];
    tmem_ld_32x32b_x16(lane_base + (uint32_t)(h * per_half * NB + c0), r);
    if (per_half == 2)  // the second k chunk's accumulator, added in order
      tmem_ld_32x32b_x16(lane_base + (uint32_t)((h * 2 + 1) * NB + c0), r2);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
    if (per_half == 2) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += __uint_as_float(r2[j]);
    }
    if (args.swiglu_out != nullptr) {
      // rows (2i, 2i+1) = (g_i, u_i) sit in adjacent lanes
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float x = v[j] * alpha;
        const float u = __shfl_xor_sync(0xffffffffu, x, 1);
        const int b = b0 + c0 + j;
        if ((lane & 1) == 0 && n < args.N && b < args.M) {
          const __half hv = __float2half_rn(x / (1.0f + expf(-x)) * u);
          args.swiglu_out[(size_t)b * args.ld_out + n / 2] = *reinterpret_cast<const uint16_t *>(&hv);
        }
      }
    } else if (n < args.N) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = b0 + c0 + j;
        if (b < args.M) w.d[(size_t)b * args.ldd + n] = v[j] * alpha;
      }
    }
  }
}

template <int TR>
__global__ void __launch_bounds__(kW4tThreads, 1)
gemm_w4t_kernel(const __grid_constant__ CUtensorMap tmA, W4tArgs args) {
  constexpr int kHalves = TR / 128;
  constexpr int kGroupBytes = 9216;                // 128 rows: 8 KB codes + 1 KB scales
  constexpr int kStageBytes = kHalves * kGroupBytes;
  constexpr int kStageCols = kHalves * 64;         // TMEM columns of a stage's weights
  constexpr int kPieces = kHalves * 2;             // (half, 64-wide k chunk) pieces per stage
  const int S = args.stages, SW = args.w_stages, NB = args.nb;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t *act = smem;                                         // [S][2][NB][128]
  uint8_t *wring = smem + (size_t)S * args.act_stage_bytes;    // [SW][codes | scales]
  uint64_t *bars = reinterpret_cast<uint64_t *>(wring + (size_t)SW * kStageBytes);
  uint64_t *wfull = bars, *wempty = bars + kW4tMaxWStages;
  uint64_t *afull = wempty + kW4tMaxWStages, *tready = afull + kW4tMaxStages;
  uint64_t *sempty = tready + kW4tMaxStages;
  uint64_t *accfull = sempty + kW4tMaxStages, *accempty = accfull + 1, *drain = accempty + 1;
  uint64_t *acc_last = drain + 1;  // the CTA's last unit accumulated (one phase per launch)
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_last + 1);

  DeviceStatus *st = &g_gemm_status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_units = args.tiles_n * args.tiles_b * args.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kW4tConvWarps);
    }
    for (int s = 0; s < S; ++s) {
      // stage ready: the activation producer (with the TMA bytes) and every
      // converter arrive; the MMA issuers wait on this one barrier
      mbar_init(&afull[s], 1 + kW4tConvWarps);
      mbar_init(&sempty[s], args.issuers);  // one commit per MMA issuer
    }
    mbar_init(accfull, args.issuers);
    mbar_init(accempty, 4);
    mbar_init(drain, args.issuers);
    mbar_init(acc_last, args.issuers);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- weight producer (constant data: no launch wait)
    int ws = 0;
    uint32_t wph = 0, issued_mask = 0, issued_parity = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x) {
      const W4tUnit w = w4t_unit(args, t);
      const size_t row0 = (size_t)w.tile_n * TR;
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&wempty[ws], wph ^ 1u, st, 61)) {
          okay = false;
          break;
        }
        if (lane == 0) {  // the tile's groups are contiguous: one copy per stage
          uint8_t *dst = wring + (size_t)ws * kStageBytes;
          const size_t group = (size_t)kb * (args.npad / 128) + row0 / 128;
          mbar_arrive_expect_tx(&wfull[ws], kStageBytes);
          bulk_g2s_gemm(dst, args.packed + group * kGroupBytes, kStageBytes, &wfull[ws]);
        }
        __syncwarp();
        issued_mask |= 1u << ws;
        issued_parity = (issued_parity & ~(1u << ws)) | (wph << ws);
        if (++ws == SW) {
          ws = 0;
          wph ^= 1u;
        }
      }
    }
    for (int s = 0; s < SW; ++s)
      if (issued_mask & (1u << s)) warp_wait(&wfull[s], (issued_parity >> s) & 1u, st, 62);
  } else if (warp == 5) {
    // ---------------- activation producer
    pdl_wait();
    if (args.xw.flags != nullptr) {
      // the activations are the peers' slices, written over NVLink: wait for
      // their flags (the weight producer and converters run meanwhile), then
      // order the TMA reads after the acquire
      exchange_wait_warp(args.xw, st, 72);
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    int as = 0;
    uint32_t aph = 0, issued_mask = 0, issued_parity = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x) {
      const W4tUnit w = w4t_unit(args, t);
      const int b0 = w.tile_b * NB;
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&sempty[as], aph ^ 1u, st, 63)) {
          okay = false;
          break;
        }
        if (lane == 0) {
          uint8_t *dst = act + (size_t)as * args.act_stage_bytes;
          mbar_arrive_expect_tx(&afull[as], (uint32_t)args.act_stage_bytes);
          tma_load_2d(dst, &tmA, &afull[as], kb * 128, b0);
          tma_load_2d(dst + args.act_stage_bytes / 2, &tmA, &afull[as], kb * 128 + 64, b0);
        }
        __syncwarp();
        issued_mask |= 1u << as;
        issued_parity = (issued_parity & ~(1u << as)) | (aph << as);
        if (++as == S) {
          as = 0;
          aph ^= 1u;
        }
      }
    }
    for (int s = 0; s < S; ++s)
      if (issued_mask & (1u << s)) warp_wait(&afull[s], (issued_parity >> s) & 1u, st, 64);
  } else if (warp >= kW4tFirstConv) {
    // ---------------- converters: E2M1 x UE4M3 -> fp16 pairs -> TMEM
    const int quarter = warp & 3, slot = (warp - kW4tFirstConv) >> 2;  // piece `slot` of each stage
    const bool has = slot < kPieces;
    const int h = slot >> 1, c = slot & 1;
    int ws = 0, ts = 0;
    uint32_t wph = 0, tph = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x) {
      const W4tUnit w = w4t_unit(args, t);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&wfull[ws], wph, st, 65)) {
          okay = false;
          break;
        }
        const uint8_t *wsm = wring + (size_t)ws * kStageBytes;
        uint32_t r[32];
        if (has) {
          const uint8_t *grp = wsm + (size_t)h * kGroupBytes;  // this half's 128 rows
          const uint4 *src = reinterpret_cast<const uint4 *>(grp + (size_t)(quarter * 4 + c * 2) * 512) + lane;
          const uint4 cq0 = src[0], cq1 = src[32];
          const uint32_t sq = *reinterpret_cast<const uint32_t *>(grp + 8192 + (size_t)(quarter * 32 + lane) * 8 + c * 4);
          __syncwarp();
          if (lane == 0) mbar_arrive(&wempty[ws]);
          // convert in registers while the MMAs of earlier stages still
          // hold this stage's TMEM columns
          const uint32_t words[8] = {cq0.x, cq0.y, cq0.z, cq0.w, cq1.x, cq1.y, cq1.z, cq1.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // 16 values (8 bytes of codes) per scale
            const uint32_t sc = ue4m3_to_f16x2((sq >> (8 * q)) & 0xFFu);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t byte = (words[q * 2 + j / 4] >> (8 * (j & 3))) & 0xFFu;
              const uint32_t v = e2m1x2_to_f16x2(byte);
              asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r[q * 8 + j]) : "r"(v), "r"(sc));
            }
          }
        } else {
          __syncwarp();
          if (lane == 0) mbar_arrive(&wempty[ws]);
        }
        if (!warp_wait(&sempty[ts], tph ^ 1u, st, 66)) {
          okay = false;
          break;
        }
        tc_fence_after();
        if (has) {
          const uint32_t col = (uint32_t)args.acc_cols + (uint32_t)ts * kStageCols + h * 64 + c * 32;
          tmem_st_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + col, r);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[ts]);
        if (++ws == SW) {
          ws = 0;
          wph ^= 1u;
        }
        if (++ts == S) {
          ts = 0;
          tph ^= 1u;
        }
      }
    }
  } else if (warp >= 1 && warp <= args.issuers) {
    // ---------------- MMA issuers (see the role list)
    const int i = warp - 1, nis = args.issuers;
    const uint32_t idesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    // issuer i: its half, its chunks [c_lo, c_hi), its accumulator
    const int h = nis == 4 ? i >> 1 : (nis == 2 ? i : 0);
    const int c_lo = nis == 4 ? (i & 1) : 0, c_hi = nis == 4 ? c_lo + 1 : 2;
    const uint32_t d_tmem = tmem_base + (uint32_t)(i * NB);
    int s = 0;
    uint32_t ph = 0;
    bool okay = true;
    int local = 0;
    for (int t = blockIdx.x; t < num_units && okay; t += gridDim.x, ++local) {
      if (!warp_wait(accempty, (uint32_t)(local & 1) ^ 1u, st, 67)) break;
      tc_fence_after();
      const W4tUnit w = w4t_unit(args, t);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!warp_wait(&afull[s], ph, st, 68)) {
          okay = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(act + (size_t)s * args.act_stage_bytes);
          const uint32_t t_col = (uint32_t)args.acc_cols + (uint32_t)s * kStageCols + h * 64;
          for (int c = c_lo; c < c_hi; ++c)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t b_desc = smem_desc_sw128(a_addr + (uint32_t)c * (args.act_stage_bytes / 2) + k * 32);
              tc_mma_ts(d_tmem, tmem_base + t_col + c * 32 + k * 8, b_desc, idesc,
                        (kb > w.kb0 || c > c_lo || k > 0) ? 1u : 0u);
            }
          tc_commit(&sempty[s]);
        }
        __syncwarp();
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (okay && lane == 0) {
        tc_commit(accfull);
        if (t + (int)gridDim.x >= num_units) tc_commit(acc_last);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(drain);
    __syncwarp();
    warp_wait(drain, 0, st, 70);
  } else if (warp >= kW4tFirstEpi && warp < kW4tFirstEpi + 4) {
    // ---------------- epilogue
    pdl_wait();
    const int quarter = warp & 3;
    const float alpha = args.alpha != nullptr ? *args.alpha : 1.0f;
    int local = 0;
    for (int t = blockIdx.x; t < num_units; t += gridDim.x, ++local) {
      if (!warp_wait(accfull, (uint32_t)(local & 1), st, 71)) break;
      tc_fence_after();
      // the CTA's last unit is shared with the (then idle) converter warps
      const bool last = t + (int)gridDim.x >= num_units;
      w4t_store_chunks<TR>(args, w4t_unit(args, t), tmem_base, quarter, lane, alpha, 0,
                           last ? kW4tLastWorkers : 1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty);
    }
  }

  // The stores of the CTA's last unit (four epilogue warps alone wrote ~25
  // GB/s per SM: the per-warp store rate bounds them): every warp whose role
  // has ended takes a share of its lane quarter's chunks.
  if (warp < kW4tFirstEpi || warp >= kW4tFirstConv) {
    const int worker = warp >= kW4tFirstConv ? 1 + ((warp - kW4tFirstConv) >> 2) : 5 + (warp >> 2);
    if (blockIdx.x < num_units) {
      pdl_wait();  // outputs may be buffers the previous kernel reads
      if (warp_wait(acc_last, 0, st, 75)) {
        tc_fence_after();
        const float alpha = args.alpha != nullptr ? *args.alpha : 1.0f;
        const int t_last = blockIdx.x + (num_units - 1 - (int)blockIdx.x) / (int)gridDim.x * (int)gridDim.x;
        w4t_store_chunks<TR>(args, w4t_unit(args, t_last), tmem_base, warp & 3, lane, alpha, worker,
                             kW4tLastWorkers);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Packs NVFP4 weights (codes [N][ld_bytes] two per byte, even index in the
// low nibble; UE4M3 scales [N][nsf], one per 16 values) into the layout of
// gemm_w4t_kernel: per 128-wide k block kb and 128-row group hg a block of
// 9216 bytes at (kb * npad / 128 + hg) * 9216: the codes of its four 32-row
// quarters as four 16-byte columns of 32 rows ([4][4][32][16], 8 KB) and
// then their scales as 32 rows of 8 bytes ([4][32][8], 1 KB); rows past N
// and k past K are zero. Output row n takes source row map[n] when map is given.
__global__ void w4t_pack_kernel(uint8_t *packed, const uint8_t *codes, const uint8_t *scales, int N, int K,
                                int ld_bytes, int nsf, int npad, int kb_total, const int *map) {
  const size_t total = (size_t)kb_total * npad * 4;  // one thread per 16-byte code piece
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
    const int r = (int)(i % 32);
    const int j = (int)((i / 32) % 4);
    const size_t gk = i / 128;                 // kb * (npad / 32) + 32-row group
    const int g = (int)(gk % (npad / 32));
    const int kb = (int)(gk / (npad / 32));
    const int hg = g / 4, q = g % 4;
    uint8_t *blk = packed + ((size_t)kb * (npad / 128) + hg) * 9216;
    const int n = g * 32 + r;
    const int src_row = n < N ? (map != nullptr ? map[n] : n) : -1;
    const int byte0 = kb * 64 + j * 16;        // code bytes of the piece in the source row
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (src_row >= 0 && byte0 + 16 <= K / 2) {
      const uint8_t *p = codes + (size_t)src_row * ld_bytes + byte0;
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        w[e] = (uint32_t)p[4 * e] | ((uint32_t)p[4 * e + 1] << 8) | ((uint32_t)p[4 * e + 2] << 16) |
               ((uint32_t)p[4 * e + 3] << 24);
      v = make_uint4(w[0], w[1], w[2], w[3]);
    }
    *reinterpret_cast<uint4 *>(blk + (size_t)(q * 4 + j) * 512 + r * 16) = v;
    if (j == 0) {
      uint32_t lo = 0, hi = 0;
      if (src_row >= 0) {
        const uint8_t *s8 = scales + (size_t)src_row * nsf + kb * 8;
        for (int e = 0; e < 8; ++e) {
          const uint32_t b = kb * 8 + e < K / 16 ? s8[e] : 0u;
          if (e < 4) lo |= b << (8 * e);
          else hi |= b << (8 * (e - 4));
        }
      }
      *reinterpret_cast<uint2 *>(blk + 8192 + (size_t)(q * 32 + r) * 8) = make_uint2(lo, hi);
    }
  }
}

}  // namespace

// 2-D bf16 tensor map of rows of `inner` elements (`ld` apart) with a
// [box_outer rows][64 elements] box and the 128-byte swizzle, for kernels
// outside this file (the prefill attention's K and V tiles).
int make_bf16_rows_map(CUtensorMap *map, const void *base, unsigned long long inner,
                       unsigned long long outer, unsigned long long ld, int box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(CE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(CE_ERR_CUDA, format("cuTensorMapEncodeTiled failed (%d) for %llu rows of %llu", (int)r, outer,
                                         inner));
  return CE_OK;
}

int gemm_bf16(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
              int ldb, int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group) {
  return gemm_dispatch<0>(d, a, b, M, N, K, lda, ldb, ldd, row_scale, col_scale, force_bn,
                          force_group, s);
}

int gemm_tf32(float *d, const float *a, const float *b, int M, int N, int K, int lda, int ldb,
              int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group) {
  return gemm_dispatch<1>(d, a, b, M, N, K, lda, ldb, ldd, row_scale, col_scale, force_bn,
                          force_group, s);
}

int gemm_e4m3(float *d, const uint8_t *a, const uint8_t *b, int M, int N, int K, int lda,
              int ldb, int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group) {
  return gemm_dispatch<2>(d, a, b, M, N, K, lda, ldb, ldd, row_scale, col_scale, force_bn,
                          force_group, s);
}

// Row-shard GEMM (ce_plan_gemm_rowx): the plain GEMM of one rank's slice of
// W's rows whose epilogue also stores every output piece into each peer's
// exchange block, ordered by the ready / done flags of rx (common.cuh).
// kind: 0 bf16, 1 tf32, 2 e4m3 (row_scale / col_scale as for gemm_e4m3).
int gemm_rowx(int kind, float *d, const void *a, const void *b, int M, int N, int K, int lda, int ldb,
              int ldd, const float *row_scale, const float *col_scale, const RowxSync &rx, cudaStream_t s) {
  switch (kind) {
    case 0:
      return gemm_dispatch<0>(d, a, b, M, N, K, lda, ldb, ldd, nullptr, nullptr, 0, 0, s, 1, 0, false,
                              nullptr, 0, nullptr, &rx);
    case 1:
      return gemm_dispatch<1>(d, a, b, M, N, K, lda, ldb, ldd, nullptr, nullptr, 0, 0, s, 1, 0, false,
                              nullptr, 0, nullptr, &rx);
    case 2:
      return gemm_dispatch<2>(d, a, b, M, N, K, lda, ldb, ldd, row_scale, col_scale, 0, 0, s, 1, 0, false,
                              nullptr, 0, nullptr, &rx);
  }
  return set_error(CE_ERR_USAGE, format("no row-shard GEMM for operand kind %d", kind));
}

// Split-K bf16 GEMM: split s of `splits` accumulates its balanced range of
// k-blocks and writes its fp32 partial at d + s * split_stride; the caller
// sums the partials (in split order, so the result is deterministic). pdl:
// launch with programmatic stream serialization (the kernel waits for its
// predecessor before reading A or writing D).
int gemm_bf16_split(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
                    int ldb, int ldd, int splits, long long split_stride, cudaStream_t s, bool pdl) {
  return gemm_dispatch<0>(d, a, b, M, N, K, lda, ldb, ldd, nullptr, nullptr, 0, 0, s, splits,
                          split_stride, pdl);
}

// Split count that fills the SMs for a bf16 GEMM of this shape: the tiles
// of the automatic choice, times splits, up to one wave, with at least
// min_kblocks k-blocks per split; at most max_splits.
int gemm_bf16_auto_splits(int M, int N, int K, int max_splits, int min_kblocks) {
  const int sms = sm_count();
  if (sms <= 0) return 1;
  const GemmChoice c = choose_tiles(M, N, sms);
  const int rows = c.pair ? 2 * BM : BM;
  const int units = c.pair ? sms / 2 : sms;
  const long long tiles = (long long)((M + rows - 1) / rows) * ((N + c.bn - 1) / c.bn);
  const int k_blocks = (K + 63) / 64;
  long long sp = units / (tiles > 0 ? tiles : 1);
  sp = sp < (long long)max_splits ? sp : (long long)max_splits;
  const long long by_k = k_blocks / (min_kblocks > 0 ? min_kblocks : 1);
  sp = sp < by_k ? sp : by_k;
  return sp < 1 ? 1 : (int)sp;
}

// bf16 GEMM whose epilogue applies SwiGLU to interleaved (w1, w3) output
// column pairs: out[m][i] = bf16(silu(D[m][2i]) * D[m][2i+1]), D = A B^T, no
// fp32 output. N = 2 x hidden.
int gemm_bf16_swiglu(uint16_t *out, int ld_out, const uint16_t *a, const uint16_t *b, int M, int N,
                     int K, int lda, int ldb, cudaStream_t s, bool pdl) {
  return gemm_dispatch<0>(nullptr, a, b, M, N, K, lda, ldb, N, nullptr, nullptr, 0, 0, s, 1, 0, pdl,
                          out, ld_out);
}

// fp16 GEMM (kind::f16 with fp16 operands): d = alpha x A B^T, alpha a
// scalar on the device (nullptr = 1); with swiglu_out, B's rows interleave
// w1 and w3 and fp16(silu(g) * u) goes to swiglu_out [M][swiglu_ld].
int gemm_f16(float *d, const uint16_t *a, const uint16_t *b, const float *alpha, int M, int N, int K, int lda,
             int ldb, int ldd, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl) {
  return gemm_dispatch<3>(d, a, b, M, N, K, lda, ldb, swiglu_out != nullptr ? N : ldd, nullptr, nullptr, 0, 0, s,
                          1, 0, pdl, swiglu_out, swiglu_ld, alpha);
}

// Time of the busiest CTA of a W4A16 launch, in units of one weight row of
// one k-block: waves x (k-blocks per split + kW4UnitKb) x (kW4StepRows +
// width). Each
// k-block also costs a fixed pipeline round (measured about 0.4 us, worth
// some 400 rows of conversion and MMA), so wide tiles and few waves win.
// A work unit also pays its pipeline fill and epilogue (its fp32 partial
// written and summed again), about kW4UnitKb k-blocks' worth.
constexpr long long kW4StepRows = 400;
constexpr long long kW4UnitKb = 6;

long long w4_cost(int M, int N, int K, int splits, int width, int sms) {
  const long long units = (long long)((M + BM - 1) / BM) * ((N + width - 1) / width) * splits;
  const long long kb = (K / 64 + splits - 1) / splits;
  return ((units + sms - 1) / sms) * (kb + kW4UnitKb) * (kW4StepRows + width);
}

// Tile width of a W4A16 GEMM with `splits` k ranges: the one in
// {64, ..., 224} with the smallest w4_cost.
int w4_tile_width(int M, int N, int K, int splits, int sms) {
  static const int kWidths[] = {64, 96, 128, 160, 192, 224};
  int best = 128;
  long long best_cost = -1;
  for (int w : kWidths) {
    const long long cost = w4_cost(M, N, K, splits, w, sms);
    if (best_cost < 0 || cost < best_cost) best = w, best_cost = cost;
  }
  return best;
}

// W4A16 GEMM (see gemm_w4a16_kernel): d = alpha x A W^T with W in the
// k-block-major NVFP4 layout of w4_pack; split-K partials and the SwiGLU
// epilogue as in gemm_bf16_split / gemm_bf16_swiglu.
int gemm_w4a16(float *d, const uint16_t *a, const uint8_t *codes_t, const uint8_t *scales_t,
               const float *alpha, int M, int N, int K, int lda, int ldd, int splits,
               long long split_stride, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl) {
  CE_REQUIRE(M >= 1 && N >= 1 && K >= 64, "W4A16 GEMM dims (M=%d N=%d K=%d)", M, N, K);
  CE_REQUIRE(K % 64 == 0 && N % 4 == 0, "W4A16 GEMM needs K %% 64 == 0 and N %% 4 == 0 (K=%d N=%d)", K, N);
  CE_REQUIRE(lda >= K && (lda * 2) % 16 == 0, "lda must be >= K and a multiple of 8 (got %d)", lda);
  CE_REQUIRE(a && codes_t && scales_t && (d || swiglu_out), "null operand");
  CE_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15u) == 0 && (reinterpret_cast<uintptr_t>(codes_t) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_t) & 15u) == 0,
             "operands must be 16-byte aligned");
  const int k_blocks = K / 64;
  CE_REQUIRE(splits >= 1 && splits <= k_blocks, "split count must be in [1, %d] (got %d)", k_blocks, splits);
  CE_REQUIRE(swiglu_out == nullptr || (splits == 1 && N % 2 == 0 && swiglu_ld >= N / 2),
             "the SwiGLU epilogue needs one split, an even N and ld_out >= N / 2");
  CE_REQUIRE(swiglu_out != nullptr || ldd >= N, "ldd must be >= N");
  if (!is_sm100()) return set_error(CE_ERR_USAGE, "tcgen05 GEMM needs an sm_100 device");
  const int sms = sm_count();
  const int tiles_m = (M + BM - 1) / BM;
  const int bn = w4_tile_width(M, N, K, splits, sms);
  // A tiles: a 64-row box (8 KB slots, a deeper ring) when the rows fit
  const int a_rows = M <= 64 ? 64 : BM;
  CUtensorMap ta;
  int rc = make_operand_map(&ta, a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, M, lda, a_rows);
  if (rc) return rc;
  W4Args w{};
  w.a_slot = a_rows * kRowBytes;
  w.g.d = d;
  w.g.M = M;
  w.g.N = N;
  w.g.K = K;
  w.g.ldd = ldd;
  w.g.tiles_m = tiles_m;
  w.g.tiles_n = (N + bn - 1) / bn;
  w.g.k_blocks = k_blocks;
  w.g.splits = splits;
  w.g.split_stride = splits > 1 ? split_stride : 0;
  w.g.epilogue = swiglu_out != nullptr ? 1 : 0;
  w.g.out_bf16 = swiglu_out;
  w.g.ld_out = swiglu_ld;
  w.g.out_f16 = 1;
  w.codes = codes_t;
  w.scales = scales_t;
  w.alpha = alpha;
  const int units = w.g.tiles_m * w.g.tiles_n * splits;
  const int grid = units < sms ? units : sms;
  switch (bn) {
#define CE_W4_LAUNCH(W)                                                                          \
  case W:                                                                                        \
    w.a_stages = SmemW4<W>::a_stages(w.a_slot);                                                  \
    if (w.a_stages < 2 || SmemW4<W>::total(w.a_slot) > kW4SmemBudget)                            \
      return set_error(CE_ERR_USAGE, format("W4A16 tile width %d does not fit shared memory", W)); \
    rc = configure_smem<gemm_w4a16_kernel<W>>(kW4SmemBudget);                                    \
    if (rc) return rc;                                                                           \
    return launch_kernel(gemm_w4a16_kernel<W>, dim3(grid), dim3(kW4Threads), SmemW4<W>::total(w.a_slot), s, \
                         pdl, "gemm_w4a16_kernel", ta, w);
    CE_W4_LAUNCH(64)
    CE_W4_LAUNCH(96)
    CE_W4_LAUNCH(128)
    CE_W4_LAUNCH(160)
    CE_W4_LAUNCH(192)
    CE_W4_LAUNCH(224)
#undef CE_W4_LAUNCH
  }
  return set_error(CE_ERR_USAGE, format("unsupported W4A16 tile width %d", bn));
}

// Split count that fills the SMs for a W4A16 GEMM of this shape (tiles of
// the width gemm_w4a16 picks, times splits, up to one CTA per SM), with at
// least min_kblocks 64-wide k-blocks per split; at most max_splits.
int gemm_w4a16_auto_splits(int M, int N, int K, int max_splits, int min_kblocks) {
  const int sms = sm_count();
  if (sms <= 0) return 1;
  const long long kb = K / 64;
  const long long by_k = kb / (min_kblocks > 0 ? min_kblocks : 1);
  int best = 1;
  long long best_cost = -1;
  for (int sp = 1; sp <= max_splits && sp <= by_k; ++sp) {
    const long long cost = w4_cost(M, N, K, sp, w4_tile_width(M, N, K, sp, sms), sms);
    if (best_cost < 0 || cost < best_cost) best = sp, best_cost = cost;
  }
  return best;
}

// row_map (device, N entries; nullptr = identity): packed row n comes from
// source row row_map[n] (a shard's rows of a whole quantized matrix).
int w4_pack(uint8_t *codes_t, uint8_t *scales_t, const uint8_t *codes, const uint8_t *scales, int N, int K,
            int ld_bytes, int nsf, cudaStream_t s, const int *row_map) {
  CE_REQUIRE(codes_t && scales_t && codes && scales, "null argument");
  CE_REQUIRE(N >= 1 && K >= 64 && K % 64 == 0 && ld_bytes * 2 >= K && nsf * 16 >= K,
             "bad NVFP4 weight shape %dx%d (ld_bytes %d, scales per row %d)", N, K, ld_bytes, nsf);
  const size_t words = (size_t)(K / 64) * N * 8;
  int blocks = (int)((words + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  w4_pack_kernel<<<blocks, 256, 0, s>>>(codes_t, scales_t, codes, scales, N, K, ld_bytes, nsf, row_map);
  CE_LAUNCH_CHECK("w4_pack_kernel");
  return CE_OK;
}

// Tile plan of gemm_w4t for a batch of M rows: 256 weight rows per tile
// (two M=128 halves) while the batch fits 128 TMEM columns, else 128; batch
// columns per tile (a multiple of 16, at most 256); TMEM weight stages =
// activation slots (what TMEM and shared memory hold), packed weight stages.
struct W4tPlan {
  int tr, nb, tiles_b, stages, w_stages, act_stage, acc_cols, issuers;
  int smem;
};

W4tPlan w4t_plan(int M) {
  W4tPlan p{};
  const int m16 = (M + 15) / 16 * 16;
  p.tr = m16 <= 128 ? 256 : 128;
  p.nb = m16 <= 256 ? m16 : 256;
  p.tiles_b = (M + p.nb - 1) / p.nb;
  const int halves = p.tr / 128;
  p.issuers = p.tr == 256 ? (p.nb <= 64 ? 4 : 2) : 1;  // one accumulator each
  p.acc_cols = (p.issuers * p.nb + 63) / 64 * 64;
  int tstages = ((int)kTmemCols - p.acc_cols) / (halves * 64);
  if (tstages > kW4tMaxStages) tstages = kW4tMaxStages;
  p.act_stage = 2 * p.nb * kRowBytes;
  const int w_stage = p.tr * 72, fixed = 2048;  // barriers + alignment slack
  int S = tstages;
  while (S > 2 && S * p.act_stage + 3 * w_stage + fixed > kW4tSmemBudget) --S;
  p.stages = S;
  int SW = (kW4tSmemBudget - S * p.act_stage - fixed) / w_stage;
  p.w_stages = SW > kW4tMaxWStages ? kW4tMaxWStages : SW;
  p.smem = S * p.act_stage + p.w_stages * w_stage + fixed;
  return p;
}

// Split count for gemm_w4t: units of (weight tile, batch tile, k range) are
// spread over the SMs; a unit costs its 128-wide k blocks plus about three
// blocks of fill and epilogue.
int gemm_w4t_auto_splits(int M, int N, int K, int max_splits) {
  const int sms = sm_count();
  if (sms <= 0) return 1;
  const W4tPlan p = w4t_plan(M);
  const long long kb = (K + 127) / 128;
  const long long tiles = (long long)((N + p.tr - 1) / p.tr) * p.tiles_b;
  int best = 1;
  long long best_cost = -1;
  for (int sp = 1; sp <= max_splits && sp <= kb; ++sp) {
    const long long units = tiles * sp;
    const long long cost = ((units + sms - 1) / sms) * ((kb + sp - 1) / sp + 3);
    if (best_cost < 0 || cost < best_cost) best = sp, best_cost = cost;
  }
  return best;
}

// Bytes of the packed NVFP4 weights of gemm_w4t for N x K.
size_t w4t_packed_bytes(int N, int K) {
  const size_t kb = (size_t)(K + 127) / 128, npad = (size_t)(N + 255) / 256 * 256;
  return kb * (npad / 128) * 9216;
}

namespace {

// One 32-value piece of a W4T-packed weight row to fp16: e2m1(code) x
// ue4m3(scale), exact in fp16 (at most 6 significant bits, magnitudes in
// [2^-10, 2688]); the tensor decode scale stays with the GEMM's alpha.
__global__ void w4t_expand_f16_kernel(uint16_t *out, const uint8_t *packed, int N, int K, int npad) {
  const int pieces = K / 32;
  const size_t total = (size_t)N * pieces;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(i / pieces), p = (int)(i % pieces);
    const int kb = p / 4, j = p % 4;
    const int g = n / 32, r = n % 32, hg = g / 4, q = g % 4;
    const uint8_t *blk = packed + ((size_t)kb * (npad / 128) + hg) * 9216;
    const uint4 c = *reinterpret_cast<const uint4 *>(blk + (size_t)(q * 4 + j) * 512 + r * 16);
    const uint8_t *sc = blk + 8192 + (size_t)(q * 32 + r) * 8 + 2 * j;
    float scale[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t u = sc[h];
      const int e = (u >> 3) & 15, mm = u & 7;
      scale[h] = e == 0 ? ldexpf((float)mm, -9) : ldexpf((float)(8 + mm), e - 10);
    }
    const uint32_t words[4] = {c.x, c.y, c.z, c.w};
    uint32_t o[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      const uint32_t byte = (words[b / 4] >> (8 * (b % 4))) & 0xFFu;
      float v[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t code = h ? byte >> 4 : byte & 15u;
        const uint32_t mag = code & 7u;
        const float m = mag < 4 ? 0.5f * (float)mag : (float)(mag == 4 ? 2 : mag == 5 ? 3 : mag == 6 ? 4 : 6);
        v[h] = ((code & 8u) ? -m : m) * scale[b / 8];
      }
      __half2 hv = __floats2half2_rn(v[0], v[1]);
      o[b] = *reinterpret_cast<uint32_t *>(&hv);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)n * K + (size_t)p * 32);
#pragma unroll
    for (int w = 0; w < 4; ++w) dst[w] = make_uint4(o[4 * w], o[4 * w + 1], o[4 * w + 2], o[4 * w + 3]);
  }
}

}  // namespace

// W4T-packed weight [N][K] (w4t_pack's layout) expanded to fp16 [N][K]
// without the tensor decode scale (the GEMM applies it as alpha).
int w4t_expand_f16(uint16_t *out, const uint8_t *packed, int N, int K, cudaStream_t s) {
  CE_REQUIRE(out && packed && N >= 1 && K >= 64 && K % 64 == 0, "bad W4T expansion (N=%d K=%d)", N, K);
  const int npad = (N + 255) / 256 * 256;
  const size_t total = (size_t)N * (K / 32);
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  w4t_expand_f16_kernel<<<blocks, 256, 0, s>>>(out, packed, N, K, npad);
  CE_LAUNCH_CHECK("w4t_expand_f16_kernel");
  return CE_OK;
}

int w4t_pack(uint8_t *packed, const uint8_t *codes, const uint8_t *scales, int N, int K, int ld_bytes, int nsf,
             cudaStream_t s, const int *row_map) {
  CE_REQUIRE(packed && codes && scales, "null argument");
  CE_REQUIRE(N >= 1 && K >= 64 && K % 64 == 0 && ld_bytes * 2 >= K && nsf * 16 >= K,
             "bad NVFP4 weight shape %dx%d (ld_bytes %d, scales per row %d)", N, K, ld_bytes, nsf);
  CE_REQUIRE((reinterpret_cast<uintptr_t>(packed) & 15u) == 0, "the packed buffer must be 16-byte aligned");
  const int kb_total = (K + 127) / 128, npad = (N + 255) / 256 * 256;
  const size_t pieces = (size_t)kb_total * npad * 4;
  int blocks = (int)((pieces + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  w4t_pack_kernel<<<blocks, 256, 0, s>>>(packed, codes, scales, N, K, ld_bytes, nsf, npad, kb_total, row_map);
  CE_LAUNCH_CHECK("w4t_pack_kernel");
  return CE_OK;
}

// W4A16 GEMM, decode form (gemm_w4t_kernel): d = alpha x A W^T with A fp16
// [M][lda] and W packed by w4t_pack; split s of `splits` k ranges writes
// d + s * split_stride; with swiglu_out the rows of W interleave w1 and w3
// and the fp16 SwiGLU product goes to swiglu_out [M][swiglu_ld] instead.
int gemm_w4t(float *d, const uint16_t *a, const uint8_t *packed, const float *alpha, int M, int N, int K, int lda,
             int ldd, int splits, long long split_stride, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl,
             const ExchangeWait *xw) {
  CE_REQUIRE(M >= 1 && N >= 1 && K >= 64 && K % 64 == 0, "W4A16 GEMM dims (M=%d N=%d K=%d; K %% 64 == 0)", M, N,
             K);
  CE_REQUIRE(lda >= K && (lda * 2) % 16 == 0, "lda must be >= K and a multiple of 8 (got %d)", lda);
  CE_REQUIRE(a && packed && (d || swiglu_out), "null operand");
  CE_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15u) == 0 && (reinterpret_cast<uintptr_t>(packed) & 15u) == 0,
             "operands must be 16-byte aligned");
  const int kb_total = (K + 127) / 128;
  CE_REQUIRE(splits >= 1 && splits <= kb_total, "split count must be in [1, %d] (got %d)", kb_total, splits);
  CE_REQUIRE(swiglu_out == nullptr || (splits == 1 && N % 2 == 0 && swiglu_ld >= N / 2),
             "the SwiGLU epilogue needs one split, an even N and ld_out >= N / 2");
  CE_REQUIRE(swiglu_out != nullptr || ldd >= N, "ldd must be >= N");
  if (!is_sm100()) return set_error(CE_ERR_USAGE, "tcgen05 GEMM needs an sm_100 device");
  const W4tPlan p = w4t_plan(M);
  if (p.stages < 2 || p.w_stages < 2 || p.smem > kW4tSmemBudget)
    return set_error(CE_ERR_USAGE, format("W4A16 plan for M=%d does not fit shared memory", M));
  CUtensorMap ta;
  int rc = make_operand_map(&ta, a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, M, lda, p.nb);
  if (rc) return rc;
  W4tArgs w{};
  w.d = d;
  w.swiglu_out = swiglu_out;
  w.packed = packed;
  w.alpha = alpha;
  w.M = M;
  w.N = N;
  w.K = K;
  w.ldd = ldd;
  w.ld_out = swiglu_ld;
  w.npad = (N + 255) / 256 * 256;
  w.kb_total = kb_total;
  w.nb = p.nb;
  w.tiles_n = (N + p.tr - 1) / p.tr;
  w.tiles_b = p.tiles_b;
  w.splits = splits;
  w.split_stride = splits > 1 ? split_stride : 0;
  w.stages = p.stages;
  w.w_stages = p.w_stages;
  w.act_stage_bytes = p.act_stage;
  w.acc_cols = p.acc_cols;
  w.issuers = p.issuers;
  if (xw != nullptr) w.xw = *xw;
  const int sms = sm_count();
  const int units = w.tiles_n * w.tiles_b * splits;
  const int grid = units < sms ? units : sms;
  if (p.tr == 256) {
    rc = configure_smem<gemm_w4t_kernel<256>>(kW4tSmemBudget);
    if (rc) return rc;
    return launch_kernel(gemm_w4t_kernel<256>, dim3(grid), dim3(kW4tThreads), (size_t)p.smem, s, pdl,
                         "gemm_w4t_kernel", ta, w);
  }
  rc = configure_smem<gemm_w4t_kernel<128>>(kW4tSmemBudget);
  if (rc) return rc;
  return launch_kernel(gemm_w4t_kernel<128>, dim3(grid), dim3(kW4tThreads), (size_t)p.smem, s, pdl,
                       "gemm_w4t_kernel", ta, w);
}

int gemm_set_prefetch(int kblocks) {
  CE_REQUIRE(kblocks >= 0 && kblocks <= 64, "prefetch distance must be in [0, 64] (got %d)", kblocks);
  g_prefetch_kblocks = kblocks;
  return CE_OK;
}

int gemm_set_wide_tiles(int on) {
  g_wide_tiles = on != 0;
  return CE_OK;
}

int gemm_set_wait_limit(unsigned long long ns) { return set_wait_limit_here(ns); }

// Synchronizes the device, reads and clears the GEMM status word.
int gemm_status() {
  CE_CUDA_TRY(cudaDeviceSynchronize());
  DeviceStatus h{};
  CE_CUDA_TRY(cudaMemcpyFromSymbol(&h, g_gemm_status, sizeof(h)));
  if (h.code != 0) {
    DeviceStatus zero{};
    CE_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(zero)));
    return set_error(CE_ERR_TIMEOUT, format("tensor-core GEMM wait %u gave up in block %u", h.where, h.block));
  }
  return CE_OK;
}

}  // namespace ce
