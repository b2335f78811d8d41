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

// ---------------------------------------------------------------------------
// MXFP6 E3M2 and NVFP4 E2M1 (experiments/blackwell/lowprec/spec.json
// "mxfp6", "nvfp4"; host restatement reference.cpp:105-150). Codes must
// equal the spec's host quantizer bit for bit, so every step keeps the
// spec's order: the hardware conversions round to nearest even and saturate
// (E3M2 to 28, E2M1 to 6, E4M3 to 448), and a zero result is written as +0.

namespace ce {
namespace {

__device__ __forceinline__ uint32_t e3m2x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e3m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  uint32_t c = r;
  if ((c & 0xFFu) == 0x20u) c &= ~0xFFu;        // -0 -> +0
  if ((c & 0xFF00u) == 0x2000u) c &= ~0xFF00u;
  return c;
}

// Two fp32 values to two E2M1 codes in one byte (lo in the low nibble).
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}"
      : "=h"(r) : "f"(hi), "f"(lo));
  uint32_t c = r & 0xFFu;
  if ((c & 0x0Fu) == 0x08u) c &= ~0x0Fu;         // -0 -> +0
  if ((c & 0xF0u) == 0x80u) c &= ~0xF0u;
  return c;
}

__device__ __forceinline__ float ue4m3_value(uint32_t code) {
  const int e = (code >> 3) & 15, m = code & 7;
  return e == 0 ? ldexpf((float)m / 8.0f, -6) : ldexpf(1.0f + (float)m / 8.0f, e - 7);
}

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per 32-value block: codes one byte per value (6 used),
// scales one UE8M0 byte per block, row-major [rows][nblocks].
__global__ void quantize_mxfp6_kernel(uint8_t *codes, uint8_t *scales, const float *x, int rows,
                                      int cols, int ld_codes, int nblocks) {
  const int lane = threadIdx.x & 31;
  const long long warp = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long total = (long long)rows * nblocks;
  if (warp >= total) return;
  const int row = (int)(warp / nblocks), blk = (int)(warp % nblocks);
  const int col = blk * 32 + lane;
  const float v = col < cols ? x[(size_t)row * cols + col] : 0.f;
  const float amax = warp_max_f(fabsf(v));
  int shared = 0;
  uint32_t scale_code = 0;
  if (amax != 0.f) {
    shared = ilogbf(amax) - 4;   // floor(log2 amax) - (largest E3M2 exponent)
    shared = max(-127, min(127, shared));
    scale_code = (uint32_t)(shared + 127);
  }
  // v * 2^-shared is exact for every value that can round to a nonzero code
  const float scaled = amax != 0.f ? v * ldexpf(1.0f, -shared) : 0.f;
  // both lanes of a pair convert (even, odd) together and keep their byte
  const float other = __shfl_xor_sync(0xffffffffu, scaled, 1);
  const uint32_t pair = (lane & 1) ? e3m2x2(other, scaled) : e3m2x2(scaled, other);
  const uint32_t mine = (lane & 1) ? (pair >> 8) & 0xFFu : pair & 0xFFu;
  if (col < ld_codes) codes[(size_t)row * ld_codes + col] = col < cols ? (uint8_t)mine : (uint8_t)0;
  if (lane == 0) scales[(size_t)row * nblocks + blk] = (uint8_t)scale_code;
}

// Tensor amax of |x| (x >= 0 compares as its bit pattern).
__global__ void amax_kernel(unsigned int *amax_bits, const float *x, size_t n) {
  float m = 0.f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
  m = warp_max_f(m);
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));
}

// NVFP4: encode scale s = 2688 / a_t (1 when a_t = 0), decode scale 1 / s.
__global__ void nvfp4_tensor_scale_kernel(float *encode_decode, const unsigned int *amax_bits) {
  const float a = __uint_as_float(*amax_bits);
  const float s = a > 0.f ? 2688.0f / a : 1.0f;
  encode_decode[0] = s;
  encode_decode[1] = 1.0f / s;
}

// One 16-value block per half warp: codes packed two per byte (even index in
// the low nibble) [rows][ld_bytes], scales one UE4M3 byte per block.
__global__ void quantize_nvfp4_kernel(uint8_t *codes, uint8_t *scales, const float *x,
                                      const float *encode_decode, int rows, int cols,
                                      int ld_bytes, int nblocks) {
  const int lane = threadIdx.x & 31;
  const long long half = ((long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2 + (lane >> 4);
  const long long total = (long long)rows * nblocks;
  const bool live = half < total;
  const int row = live ? (int)(half / nblocks) : 0, blk = live ? (int)(half % nblocks) : 0;
  const int i = lane & 15, col = blk * 16 + i;
  const float v = (live && col < cols) ? x[(size_t)row * cols + col] : 0.f;
  float amax = fabsf(v);
#pragma unroll
  for (int o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = encode_decode[0];
  float target = amax / 6.0f;
  target = target * s;
  const uint32_t sc = e4m3x2(target, 0.f) & 0x7Fu;
  const float f = ue4m3_value(sc);
  float r = 0.f;
  if (sc != 0) {
    r = v * s;
    r = r / f;
  }
  const float other = __shfl_xor_sync(0xffffffffu, r, 1);
  if (live && (i & 1) == 0) {
    const uint32_t byte = sc != 0 ? e2m1x2(r, other) : 0u;
    if (col / 2 < ld_bytes) codes[(size_t)row * ld_bytes + col / 2] = col < cols ? (uint8_t)byte : (uint8_t)0;
  }
  if (live && i == 0) scales[(size_t)row * nblocks + blk] = (uint8_t)sc;
}

// NVFP4 activation operand after a rows launch that reduced max |x| into
// amax_bits: the tensor scales (thread 0 of block 0 publishes them for the
// GEMM's alpha) and the codes with quantize_nvfp4_kernel's arithmetic, four
// consecutive values per thread (one float4 load, two code bytes), the four
// threads of a 16-value block sharing its amax by shuffles; the UE4M3 scales
// go straight into the A operand's 512-byte atoms. cols % 16 == 0.
__global__ void quantize_nvfp4_atoms_kernel(uint8_t *codes, uint8_t *atoms, float *encode_decode,
                                            const unsigned int *amax_bits, const float4 *x, int rows, int cols,
                                            int ld_bytes, int katoms) {
  const float a = __uint_as_float(*amax_bits);
  const float s = a > 0.f ? 2688.0f / a : 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    encode_decode[0] = s;
    encode_decode[1] = 1.0f / s;
  }
  const int cols4 = cols / 4;
  const long long total = (long long)rows * cols4;
  const int lane = threadIdx.x & 31;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t - lane < total;
       t += (long long)gridDim.x * blockDim.x) {
    const bool live = t < total;
    const int row = live ? (int)(t / cols4) : 0, q = live ? (int)(t % cols4) : 0;  // columns 4q .. 4q + 3
    const float4 v = live ? x[t] : make_float4(0.f, 0.f, 0.f, 0.f);
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    float target = amax / 6.0f;
    target = target * s;
    const uint32_t sc = e4m3x2(target, 0.f) & 0x7Fu;
    const float f = ue4m3_value(sc);
    float r[4] = {0.f, 0.f, 0.f, 0.f};
    if (sc != 0) {
      r[0] = v.x * s; r[0] = r[0] / f;
      r[1] = v.y * s; r[1] = r[1] / f;
      r[2] = v.z * s; r[2] = r[2] / f;
      r[3] = v.w * s; r[3] = r[3] / f;
    }
    if (live) {
      const uint32_t lo = sc != 0 ? e2m1x2(r[0], r[1]) : 0u, hi = sc != 0 ? e2m1x2(r[2], r[3]) : 0u;
      *reinterpret_cast<uint16_t *>(codes + (size_t)row * ld_bytes + 2 * q) = (uint16_t)(lo | (hi << 8));
      if ((q & 3) == 0) {
        const int blk = q / 4, mm = row % 128;
        atoms[((size_t)(row / 128) * katoms + blk / 4) * 512 + (mm % 32) * 16 + (mm / 32) * 4 + (blk % 4)] =
            (uint8_t)sc;
      }
    }
  }
}

// Row-major scales [rows][nsf] -> 512-byte atoms (see gemm_bs.cu): rows are
// taken in groups of group_rows, each group padded to whole 128-row atom
// rows; scale columns padded to katoms * 4. Padding bytes are 0.
__global__ void sf_to_atoms_kernel(uint8_t *atoms, const uint8_t *scales, int rows, int nsf,
                                   int katoms, int group_rows, size_t total) {
  const int atoms_per_group = (group_rows + 127) / 128;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t atom = i / 512;
    const int o = (int)(i % 512);
    const int kb = (int)(atom % katoms);
    const int ra = (int)(atom / katoms);
    const int group = ra / atoms_per_group, sub = ra % atoms_per_group;
    const int m = sub * 128 + ((o % 16) / 4) * 32 + o / 16;  // row within the group
    const int c = kb * 4 + (o % 4);
    const int row = group * group_rows + m;
    atoms[i] = (m < group_rows && row < rows && c < nsf) ? scales[(size_t)row * nsf + c] : (uint8_t)0;
  }
}

// MXFP6 GEMM operand: each group of 16 E3M2 codes (one byte each, low 6
// bits) becomes 12 bytes of little-endian 6-bit fields (value i at bits
// 6i..6i+5, the spec's packed order) followed by 4 zero bytes, so 16 values
// occupy 16 bytes and a 32-value MMA step is 16-byte aligned in shared
// memory, where the tensor core reads packed 6-bit fields.
__global__ void pack_mxfp6_kernel(uint8_t *operand, const uint8_t *codes, int rows, int cols,
                                  int ld_codes, int ld_operand, size_t groups_total) {
  const int groups = ld_operand / 16;
  for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < groups_total;
       g += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(g / groups), grp = (int)(g % groups);
    unsigned long long lo = 0, hi = 0;  // bits 0-63, 64-127 of the group
    for (int i = 0; i < 16; ++i) {
      const int col = grp * 16 + i;
      const unsigned long long v = col < cols ? (codes[(size_t)row * ld_codes + col] & 63u) : 0u;
      const int bit = 6 * i;
      if (bit < 64) {
        lo |= v << bit;
        if (bit > 58) hi |= v >> (64 - bit);
      } else {
        hi |= v << (bit - 64);
      }
    }
    uint4 out;
    out.x = (uint32_t)lo;
    out.y = (uint32_t)(lo >> 32);
    out.z = (uint32_t)hi;
    out.w = 0u;
    *reinterpret_cast<uint4 *>(operand + (size_t)row * ld_operand + (size_t)grp * 16) = out;
  }
}

// Element values of the operand formats, from their definitions (sign,
// exponent bias, subnormals at exponent field 0): E4M3 bias 7, E3M2 bias 3,
// E2M1 bias 1; UE8M0 = 2^(e - 127).
__device__ __forceinline__ float e4m3_value(uint32_t c) {
  const int e = (c >> 3) & 15, m = c & 7;
  const float v = e == 0 ? ldexpf((float)m, -9) : ldexpf((float)(8 + m), e - 10);
  return (c & 0x80u) ? -v : v;
}
__device__ __forceinline__ float e3m2_value(uint32_t c) {
  const int e = (c >> 2) & 7, m = c & 3;
  const float v = e == 0 ? ldexpf((float)m, -4) : ldexpf((float)(4 + m), e - 5);
  return (c & 0x20u) ? -v : v;
}
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const int e = (c >> 1) & 3, m = c & 1;
  const float v = e == 0 ? 0.5f * (float)m : ldexpf((float)(2 + m), e - 2);
  return (c & 0x8u) ? -v : v;
}

// Index of scale (row, column c) in the 512-byte atom layout written by
// sf_to_atoms_kernel: the inverse of its (o -> row, column) map.
__device__ __forceinline__ size_t atom_index(int row, int c, int katoms, int group_rows) {
  const int atoms_per_group = (group_rows + 127) / 128;
  const int group = row / group_rows, m = row % group_rows;
  const int ra = group * atoms_per_group + m / 128, mm = m % 128;
  return ((size_t)ra * katoms + c / 4) * 512 + (mm % 32) * 16 + (mm / 32) * 4 + (c % 4);
}

// One GEMM operand [rows][cols] back to fp32, value by value, as the tensor
// cores multiply it (codes x block scale x tensor scale; bf16 widened; fp32
// and the E4M3 row scale as stored).
__global__ void dequant_operand_kernel(DequantOperand d) {
  const size_t total = (size_t)d.rows * d.cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / d.cols), col = (int)(i % d.cols);
    const uint8_t *base = static_cast<const uint8_t *>(d.data);
    float v = 0.f;
    switch (d.format) {
      case kOperandF32:
        v = static_cast<const float *>(d.data)[(size_t)row * d.ld + col];
        break;
      case kOperandBF16:
        v = __uint_as_float((uint32_t)static_cast<const uint16_t *>(d.data)[(size_t)row * d.ld + col] << 16);
        break;
      case kOperandE4M3:
        v = e4m3_value(base[(size_t)row * d.ld + col]) * d.row_scale[row];
        break;
      case kOperandMXFP6: {
        const uint8_t *g = base + (size_t)row * d.ld + (size_t)(col / 16) * 16;
        const int bit = 6 * (col % 16);
        const uint32_t pair = (uint32_t)g[bit / 8] | ((uint32_t)g[bit / 8 + 1] << 8);
        const int c = col / 32;
        const uint32_t sf = d.atoms ? d.sf[atom_index(row, c, d.katoms, d.group_rows)]
                                    : d.sf[(size_t)row * d.nsf + c];
        v = e3m2_value((pair >> (bit % 8)) & 63u) * ldexpf(1.0f, (int)sf - 127);
        break;
      }
      default: {  // kOperandNVFP4
        const uint32_t byte = base[(size_t)row * d.ld + col / 2];
        const int c = col / 16;
        const uint32_t sf = d.atoms ? d.sf[atom_index(row, c, d.katoms, d.group_rows)]
                                    : d.sf[(size_t)row * d.nsf + c];
        v = e2m1_value((col & 1) ? byte >> 4 : byte & 15u) * ue4m3_value(sf) * d.tensor_decode[0];
      }
    }
    d.out[(size_t)row * d.out_ld + col] = v;
  }
}

}  // namespace

int pack_mxfp6(uint8_t *operand, const uint8_t *codes, int rows, int cols, int ld_codes,
               int ld_operand, cudaStream_t s) {
  CE_REQUIRE(operand && codes, "null argument");
  CE_REQUIRE(rows >= 1 && cols >= 1 && ld_codes >= cols && ld_operand >= ((cols + 15) / 16) * 16 &&
                 ld_operand % 16 == 0,
             "bad mxfp6 operand shape %dx%d ld %d/%d", rows, cols, ld_codes, ld_operand);
  CE_REQUIRE((reinterpret_cast<uintptr_t>(operand) & 15u) == 0, "operand must be 16-byte aligned");
  const size_t total = (size_t)rows * (ld_operand / 16);
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  pack_mxfp6_kernel<<<blocks, 256, 0, s>>>(operand, codes, rows, cols, ld_codes, ld_operand, total);
  CE_LAUNCH_CHECK("pack_mxfp6_kernel");
  return CE_OK;
}

int sf_to_atoms(uint8_t *atoms, const uint8_t *scales, int rows, int nsf, int katoms,
                int group_rows, cudaStream_t s) {
  CE_REQUIRE(atoms && scales, "null argument");
  CE_REQUIRE(rows >= 1 && nsf >= 1 && katoms * 4 >= nsf && group_rows >= 1, "bad scale layout");
  const int groups = (rows + group_rows - 1) / group_rows;
  const size_t total = (size_t)groups * ((group_rows + 127) / 128) * katoms * 512;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  sf_to_atoms_kernel<<<blocks, 256, 0, s>>>(atoms, scales, rows, nsf, katoms, group_rows, total);
  CE_LAUNCH_CHECK("sf_to_atoms_kernel");
  return CE_OK;
}

int quantize_mxfp6(uint8_t *codes, uint8_t *scales, const float *x, int rows, int cols,
                   int ld_codes, cudaStream_t s) {
  CE_REQUIRE(codes && scales && x, "null argument");
  CE_REQUIRE(rows >= 1 && cols >= 1 && ld_codes >= cols, "bad mxfp6 shape %dx%d ld %d", rows, cols, ld_codes);
  const int nblocks = (cols + 31) / 32;
  const long long warps = (long long)rows * nblocks;
  quantize_mxfp6_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(codes, scales, x, rows, cols,
                                                                    ld_codes, nblocks);
  CE_LAUNCH_CHECK("quantize_mxfp6_kernel");
  return CE_OK;
}

// encode_decode (device, 2 floats) receives the tensor scales; amax_bits
// (device, 1 word) is the reduction scratch.
int quantize_nvfp4(uint8_t *codes, uint8_t *scales, float *encode_decode, unsigned int *amax_bits,
                   const float *x, int rows, int cols, int ld_bytes, cudaStream_t s) {
  CE_REQUIRE(codes && scales && encode_decode && amax_bits && x, "null argument");
  CE_REQUIRE(rows >= 1 && cols >= 1 && ld_bytes * 2 >= cols, "bad nvfp4 shape %dx%d ld %d bytes", rows, cols, ld_bytes);
  CE_CUDA_TRY(cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), s));
  const size_t n = (size_t)rows * cols;
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  amax_kernel<<<blocks, 256, 0, s>>>(amax_bits, x, n);
  CE_LAUNCH_CHECK("amax_kernel");
  nvfp4_tensor_scale_kernel<<<1, 1, 0, s>>>(encode_decode, amax_bits);
  CE_LAUNCH_CHECK("nvfp4_tensor_scale_kernel");
  const int nblocks = (cols + 15) / 16;
  const long long halves = (long long)rows * nblocks;
  quantize_nvfp4_kernel<<<(unsigned)((halves + 15) / 16), 256, 0, s>>>(
      codes, scales, x, encode_decode, rows, cols, ld_bytes, nblocks);
  CE_LAUNCH_CHECK("quantize_nvfp4_kernel");
  return CE_OK;
}

// Pass 2 of the fused NVFP4 activation quantizer (pass 1: the rows launch
// with RowsExtras::amax_bits). Padding atom bytes must already be zero.
int quantize_nvfp4_atoms(uint8_t *codes, uint8_t *atoms, float *encode_decode, const unsigned int *amax_bits,
                         const float *x, int rows, int cols, int ld_bytes, int katoms, cudaStream_t s) {
  CE_REQUIRE(codes && atoms && encode_decode && amax_bits && x, "null argument");
  CE_REQUIRE(rows >= 1 && cols >= 16 && cols % 16 == 0 && ld_bytes * 2 >= cols && ld_bytes % 2 == 0 &&
                 katoms * 64 >= cols && (reinterpret_cast<uintptr_t>(x) & 15u) == 0,
             "bad nvfp4 shape %dx%d (cols %% 16 == 0, 16-byte aligned rows)", rows, cols);
  const long long total = (long long)rows * (cols / 4);
  const long long want = (total + 255) / 256;
  const int blocks = (int)(want < (long long)sm_count() * 16 ? want : (long long)sm_count() * 16);
  quantize_nvfp4_atoms_kernel<<<blocks, 256, 0, s>>>(codes, atoms, encode_decode, amax_bits,
                                                     reinterpret_cast<const float4 *>(x), rows, cols, ld_bytes,
                                                     katoms);
  CE_LAUNCH_CHECK("quantize_nvfp4_atoms_kernel");
  return CE_OK;
}

int dequant_operand(const DequantOperand &d, cudaStream_t s) {
  CE_REQUIRE(d.data && d.out && d.rows >= 1 && d.cols >= 1 && d.out_ld >= d.cols, "bad operand");
  CE_REQUIRE(d.format != kOperandE4M3 || d.row_scale, "the E4M3 operand needs its row scales");
  CE_REQUIRE(d.format < kOperandMXFP6 || d.sf, "a block-scaled operand needs its scales");
  CE_REQUIRE(d.format != kOperandNVFP4 || d.tensor_decode, "the NVFP4 operand needs its tensor scale");
  const size_t total = (size_t)d.rows * d.cols;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  dequant_operand_kernel<<<blocks, 256, 0, s>>>(d);
  CE_LAUNCH_CHECK("dequant_operand_kernel");
  return CE_OK;
}

}  // namespace ce
