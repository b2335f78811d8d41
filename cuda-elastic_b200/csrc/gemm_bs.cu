// Block-scaled tensor-core GEMM for sm_100a: the MXFP6-E3M2 and NVFP4-E2M1
// classifier GEMMs of experiments/blackwell/lowprec/decoder_lowprec.cu:93-127
// (there CUTLASS SM120 block-scaled GEMMs), here hand-written with
// tcgen05.mma ... .block_scale: the tensor core applies the per-block scales
// itself, so the GEMM runs at the FP6 / FP4 rates with dequantization fused.
//
//   D[m][n] = alpha * sum_k (a[m][k] * sfa[m][k / V]) * (b[n][k] * sfb[n][k / V])
//
// MXFP6: codes in groups of 16 packed 6-bit fields padded to 16 bytes
//        (ce_pack_mxfp6: one byte per value on average, the shared-memory
//        form kind::mxf8f6f4 reads for E3M2), V = 32, UE8M0 scales,
//        kind::mxf8f6f4 (K = 32 per MMA, scale_vec::1X), alpha = 1.
// NVFP4: codes two per byte (even index in the low nibble), V = 16, UE4M3
//        scales, kind::mxf4nvf4 scale_vec::4X (K = 64 per MMA), alpha =
//        decode_a * decode_b read from device memory.
//
// Scale factors live in HBM in 512-byte atoms covering 128 rows x 4 scale
// columns: byte (r % 32) * 16 + (r / 32 % 4) * 4 + c of an atom, atoms
// ordered with the scale-column index fastest (ce_sf_to_atoms). A's rows
// are grouped by 128 (one atom row per 128-row tile); B's by 224, the GEMM's
// tile width (two atom rows per tile, the second padded), so every tile's
// scales start on an atom boundary. Per stage the atoms are staged into
// shared memory by bulk copies and moved to TMEM with tcgen05.cp
// .32x128b.warpx4, which gives TMEM lane l the 16 bytes of atom row l % 32
// (4 columns): the MMA reads lane l's scales from column base + l / 32,
// byte sf_id.
//
// Structure otherwise follows gemm.cu's single-CTA kernel: persistent CTAs,
// warp 0 TMA + bulk-copy producer, warp 1 TMEM allocator / copy + MMA
// issuer, warps 2-5 epilogue, two TMEM accumulators of BN columns, bounded
// waits. BN = 224 so accumulators (448 columns) and scale factors (up to 64
// columns) share the 512 TMEM columns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace ce {

static __device__ DeviceStatus g_gemm_bs_status;

namespace {

constexpr int BM = 128;
constexpr int BN = 224;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr int kRowBytes = 128;
constexpr int kSfAtom = 512;
// B's scale atoms are grouped per BN-row tile (rows of tile t start a new
// atom row), so a tile's scales never start inside an atom: 2 atom rows.
constexpr int kSfbRowAtoms = 2;

// kFmt 0: MXFP6 (kind::mxf8f6f4, 1X), 1: NVFP4 (kind::mxf4nvf4, 4X)
template <int kFmt>
struct Fmt;
template <>
struct Fmt<0> {
  static constexpr int k_per_stage = 128;   // elements per 128-byte row
  static constexpr int k_atoms = 1;         // scale atoms along K per stage
  static constexpr uint32_t ab_format = 4;  // E3M2
  static constexpr uint32_t sf_format = 1;  // UE8M0
};
template <>
struct Fmt<1> {
  static constexpr int k_per_stage = 256;
  static constexpr int k_atoms = 4;
  static constexpr uint32_t ab_format = 1;  // E2M1 (mxf4nvf4 encoding)
  static constexpr uint32_t sf_format = 0;  // UE4M3
};

template <int kFmt>
struct BsSmem {
  static constexpr int a_bytes = BM * kRowBytes;
  static constexpr int b_bytes = BN * kRowBytes;
  static constexpr int sfa_bytes = Fmt<kFmt>::k_atoms * kSfAtom;
  static constexpr int sfb_bytes = kSfbRowAtoms * Fmt<kFmt>::k_atoms * kSfAtom;
  static constexpr int stage_bytes = a_bytes + b_bytes + sfa_bytes + sfb_bytes;
  static constexpr int max_stages = (232448 - 2048) / stage_bytes;
  static constexpr int stages = max_stages > 6 ? 6 : max_stages;
  static constexpr int bar_offset = stages * stage_bytes;
  static constexpr int total = bar_offset + 256 + 1024;
};

// TMEM columns: accumulators [0, 448), A scales then B scales after them.
constexpr uint32_t kAccStride = BN;
constexpr uint32_t kSfaCol = 2 * BN;

// Instruction descriptor of the block-scaled kinds: B scale id bits 4-5,
// A / B formats bits 7-9 / 10-12, K-major both, N >> 3 bits 17-22, scale
// format bit 23, M >> 4 bits 24-28, A scale id bits 29-30.
template <int kFmt>
__device__ __forceinline__ uint32_t bs_idesc(uint32_t sf_id) {
  return (sf_id << 4) | (Fmt<kFmt>::ab_format << 7) | (Fmt<kFmt>::ab_format << 10) |
         ((uint32_t)(BN >> 3) << 17) | (Fmt<kFmt>::sf_format << 23) |
         ((uint32_t)(BM >> 4) << 24) | (sf_id << 29);
}

template <int kFmt>
__device__ __forceinline__ void bs_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                       uint32_t accumulate) {
  if constexpr (kFmt == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem),
          "r"(sfb_tmem));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem),
          "r"(sfb_tmem));
  }
}

// Shared-memory descriptor of one 512-byte scale atom as the source of
// tcgen05.cp .32x128b: no swizzle, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t sf_atom_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;            // leading byte offset (one 16-byte column)
  d |= (uint64_t)(128u >> 4) << 32;   // stride byte offset between 8-row groups
  d |= (uint64_t)1u << 46;            // descriptor version
  return d;                           // layout type 0: no swizzle
}

__device__ __forceinline__ void tmem_cp_atom(uint32_t taddr, uint64_t src_desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc));
}

// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses and size), completion on bar.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

struct BsArgs {
  float *d;
  const uint8_t *sfa;       // atoms of A's scales
  const uint8_t *sfb;       // atoms of B's scales
  const float *alpha_a;     // NVFP4 decode scale of A (device) or nullptr
  const float *alpha_b;     // NVFP4 decode scale of B (device) or nullptr
  int M, N, K, ldd;
  int tiles_m, tiles_n, k_stages;
  int sf_katoms_a;          // atoms along K per atom row of A (row stride in atoms)
  int sf_katoms_b;
};

template <int kFmt>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               BsArgs args) {
  using S = BsSmem<kFmt>;
  using F = Fmt<kFmt>;
  constexpr int kSt = S::stages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::bar_offset);
  uint64_t *empty = full + kSt;
  uint64_t *tmem_full = empty + kSt;
  uint64_t *tmem_empty = tmem_full + 2;
  uint64_t *drain = tmem_empty + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

  DeviceStatus *st = &g_gemm_bs_status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = args.tiles_m * args.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSt; ++s) {
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

  if (warp == 0) {
    // ---------------- producer: codes by TMA, scale atoms by bulk copies
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool okay = true;
    for (int t = blockIdx.x; t < num_tiles && okay; t += gridDim.x) {
      const int m0 = (t % args.tiles_m) * BM;
      const int tn = t / args.tiles_m;
      const int n0 = tn * BN;
      const int rb0 = tn * kSfbRowAtoms;
      constexpr int rb_count = kSfbRowAtoms;
      const uint32_t bytes = (uint32_t)(S::a_bytes + S::b_bytes + S::sfa_bytes + S::sfb_bytes);
      for (int kb = 0; kb < args.k_stages; ++kb) {
        if (!warp_wait(&empty[stage], phase ^ 1u, st, 21)) {
          okay = false;
          break;
        }
        if (lane == 0) {
          uint8_t *a_dst = smem + stage * S::stage_bytes;
          uint8_t *b_dst = a_dst + S::a_bytes;
          uint8_t *sfa_dst = b_dst + S::b_bytes;
          uint8_t *sfb_dst = sfa_dst + S::sfa_bytes;
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(a_dst, &tmA, &full[stage], kb * kRowBytes, m0);
          tma_load_2d(b_dst, &tmB, &full[stage], kb * kRowBytes, n0);
          const size_t katom0 = (size_t)kb * F::k_atoms;
          bulk_load(sfa_dst, args.sfa + ((size_t)(m0 / 128) * args.sf_katoms_a + katom0) * kSfAtom,
                    (uint32_t)S::sfa_bytes, &full[stage]);
          for (int j = 0; j < rb_count; ++j)
            bulk_load(sfb_dst + j * F::k_atoms * kSfAtom,
                      args.sfb + ((size_t)(rb0 + j) * args.sf_katoms_b + katom0) * kSfAtom,
                      (uint32_t)(F::k_atoms * kSfAtom), &full[stage]);
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
    for (int s = 0; s < kSt; ++s)
      if (issued_mask & (1u << s)) warp_wait(&full[s], (issued_parity >> s) & 1u, st, 22);
  } else if (warp == 1) {
    // ---------------- scale copies + MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    bool okay = true;
    int local = 0;
    const uint32_t sfa_tmem = tmem_base + kSfaCol;
    const uint32_t sfb_tmem = sfa_tmem + 4u * F::k_atoms;
    for (int t = blockIdx.x; t < num_tiles && okay; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      constexpr int rb_count = kSfbRowAtoms;
      if (!warp_wait(&tmem_empty[acc], acc_phase ^ 1u, st, 23)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)acc * kAccStride;
      for (int kb = 0; kb < args.k_stages; ++kb) {
        if (!warp_wait(&full[stage], phase, st, 24)) {
          okay = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * S::stage_bytes);
          const uint32_t b_addr = a_addr + S::a_bytes;
          const uint32_t sfa_addr = b_addr + S::b_bytes;
          const uint32_t sfb_addr = sfa_addr + S::sfa_bytes;
          // scales of this stage into TMEM: A atoms k = 0..k_atoms-1 at
          // 4 columns each; B atoms grouped per k: [k][row atom j]
#pragma unroll
          for (int k = 0; k < F::k_atoms; ++k) {
            tmem_cp_atom(sfa_tmem + 4u * k, sf_atom_desc(sfa_addr + k * kSfAtom));
            for (int j = 0; j < rb_count; ++j)
              tmem_cp_atom(sfb_tmem + 4u * (kSfbRowAtoms * k + j),
                           sf_atom_desc(sfb_addr + (j * F::k_atoms + k) * kSfAtom));
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t a_desc = smem_desc_sw128(a_addr + k * 32);
            const uint64_t b_desc = smem_desc_sw128(b_addr + k * 32);
            const uint32_t ka = kFmt == 0 ? 0u : (uint32_t)k;        // atom of this k-step
            const uint32_t sf_id = kFmt == 0 ? (uint32_t)k : 0u;     // byte of the scale word
            bs_mma<kFmt>(d_tmem, a_desc, b_desc, bs_idesc<kFmt>(sf_id), sfa_tmem + 4u * ka,
                         sfb_tmem + 4u * kSfbRowAtoms * ka, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == kSt) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (okay && lane == 0) tc_commit(&tmem_full[acc]);
      __syncwarp();
    }
    if (lane == 0) tc_commit(drain);
    __syncwarp();
    warp_wait(drain, 0, st, 25);
  } else {
    // ---------------- epilogue
    const int quarter = warp & 3;
    const float alpha = (args.alpha_a && args.alpha_b) ? (*args.alpha_a) * (*args.alpha_b) : 1.0f;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!warp_wait(&tmem_full[acc], acc_phase, st, 26)) break;
      tc_fence_after();
      const int m0 = (t % args.tiles_m) * BM;
      const int n0 = (t / args.tiles_m) * BN;
      const int row = m0 + quarter * 32 + lane;
      float *drow = args.d + (size_t)row * args.ldd;
      const bool vec_ok = ((args.ldd & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.d) & 15u) == 0);
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
          if (vec_ok && col0 + 32 <= args.N) {
            float4 *dst = reinterpret_cast<float4 *>(drow + col0);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < args.N) drow[col0 + j] = v[j];
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

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_bs() {
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

// Byte-addressed K-major map: inner = bytes of K per row, box 128 x rows.
int make_byte_map(CUtensorMap *map, const void *base, int inner_bytes, int outer, int ld_bytes,
                  int box_outer) {
  auto fn = encode_fn_bs();
  if (fn == nullptr) return set_error(CE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner_bytes, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {(cuuint32_t)kRowBytes, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(CE_ERR_CUDA, format("cuTensorMapEncodeTiled failed (%d)", (int)r));
  return CE_OK;
}

template <int kFmt>
int launch_bs(float *d, const uint8_t *a, const uint8_t *sfa, const float *alpha_a,
              const uint8_t *b, const uint8_t *sfb, const float *alpha_b, int M, int N, int K,
              int lda_bytes, int ldb_bytes, int ldd, cudaStream_t s) {
  using S = BsSmem<kFmt>;
  using F = Fmt<kFmt>;
  const int vec = kFmt == 0 ? 32 : 16;
  CE_REQUIRE(M >= 1 && N >= 1 && K >= 1, "GEMM dims must be >= 1");
  CE_REQUIRE(K % 128 == 0, "block-scaled GEMMs need K %% 128 == 0 (got %d)", K);
  CE_REQUIRE(ldd >= N && d && a && b && sfa && sfb, "bad output or null operand");
  const int k_bytes = kFmt == 0 ? K : K / 2;
  CE_REQUIRE(lda_bytes >= k_bytes && ldb_bytes >= k_bytes && lda_bytes % 16 == 0 && ldb_bytes % 16 == 0,
             "operand row strides must cover K and be multiples of 16 bytes");
  CE_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15u) == 0 && (reinterpret_cast<uintptr_t>(b) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(sfa) & 15u) == 0 && (reinterpret_cast<uintptr_t>(sfb) & 15u) == 0,
             "operands and scale atoms must be 16-byte aligned");
  if (!is_sm100()) return set_error(CE_ERR_USAGE, "tcgen05 GEMM needs an sm_100 device");
  CUtensorMap ta, tb;
  int rc = make_byte_map(&ta, a, k_bytes, M, lda_bytes, BM);
  if (rc) return rc;
  rc = make_byte_map(&tb, b, k_bytes, N, ldb_bytes, BN);
  if (rc) return rc;
  BsArgs args;
  args.d = d;
  args.sfa = sfa;
  args.sfb = sfb;
  args.alpha_a = alpha_a;
  args.alpha_b = alpha_b;
  args.M = M;
  args.N = N;
  args.K = K;
  args.ldd = ldd;
  args.tiles_m = (M + BM - 1) / BM;
  args.tiles_n = (N + BN - 1) / BN;
  args.k_stages = (K + F::k_per_stage - 1) / F::k_per_stage;
  // atoms along K are padded to whole stages by the atom layout
  const int nsf = K / vec;
  const int katoms = ((nsf + 3) / 4 + F::k_atoms - 1) / F::k_atoms * F::k_atoms;
  args.sf_katoms_a = katoms;
  args.sf_katoms_b = katoms;
  static bool configured[64] = {};
  int dev = 0;
  CE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    CE_CUDA_TRY(cudaFuncSetAttribute(gemm_bs_kernel<kFmt>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     S::total));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int tiles = args.tiles_m * args.tiles_n;
  const int sms = sm_count();
  gemm_bs_kernel<kFmt><<<tiles < sms ? tiles : sms, kThreads, S::total, s>>>(ta, tb, args);
  CE_LAUNCH_CHECK("gemm_bs_kernel");
  return CE_OK;
}

}  // namespace

// Scale atoms along K per atom row (padded to whole stages of the format).
int sf_katoms(int fmt, int K) {
  const int vec = fmt == 0 ? 32 : 16;
  const int k_atoms = fmt == 0 ? 1 : 4;
  const int nsf = (K + vec - 1) / vec;
  return ((nsf + 3) / 4 + k_atoms - 1) / k_atoms * k_atoms;
}

// Atom rows for `rows` rows grouped by `group_rows` (each group padded to a
// multiple of 128 rows).
int sf_row_atoms(int rows, int group_rows) {
  const int groups = (rows + group_rows - 1) / group_rows;
  return groups * ((group_rows + 127) / 128);
}

int gemm_mxfp6(float *d, const uint8_t *a, const uint8_t *sfa, const uint8_t *b,
               const uint8_t *sfb, int M, int N, int K, int lda, int ldb, int ldd, cudaStream_t s) {
  return launch_bs<0>(d, a, sfa, nullptr, b, sfb, nullptr, M, N, K, lda, ldb, ldd, s);
}

int gemm_nvfp4(float *d, const uint8_t *a, const uint8_t *sfa, const float *alpha_a,
               const uint8_t *b, const uint8_t *sfb, const float *alpha_b, int M, int N, int K,
               int lda_bytes, int ldb_bytes, int ldd, cudaStream_t s) {
  return launch_bs<1>(d, a, sfa, alpha_a, b, sfb, alpha_b, M, N, K, lda_bytes, ldb_bytes, ldd, s);
}

int gemm_bs_set_wait_limit(unsigned long long ns) { return set_wait_limit_here(ns); }

int gemm_bs_status() {
  CE_CUDA_TRY(cudaDeviceSynchronize());
  DeviceStatus h{};
  CE_CUDA_TRY(cudaMemcpyFromSymbol(&h, g_gemm_bs_status, sizeof(h)));
  if (h.code != 0) {
    DeviceStatus zero{};
    CE_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_bs_status, &zero, sizeof(zero)));
    return set_error(CE_ERR_TIMEOUT, format("block-scaled GEMM wait %u gave up in block %u", h.where, h.block));
  }
  return CE_OK;
}

}  // namespace ce
