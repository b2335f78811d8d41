// Device building blocks shared by the row kernels (rows.cu) and the
// decoder kernels (decoder.cu): warp / block reductions and the
// register-resident RMSNorm and softmax row bodies. Keeping one copy means
// the decoder's gathered RMSNorm produces the same bits as ce_rmsnorm.
#pragma once

#include <cuda_bf16.h>
#include <float.h>

#include "common.cuh"

namespace ce {
namespace rowops {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum / max, result broadcast to every thread. `scratch` holds 32
// floats; the trailing barrier lets the caller reuse it immediately.
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? scratch[lane] : 0.0f;
  v = warp_sum(v);
  __syncthreads();
  return v;
}
__device__ __forceinline__ float block_max(float v, float *scratch) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? scratch[lane] : -FLT_MAX;
  v = warp_max(v);
  __syncthreads();
  return v;
}

// ---------------------------------------------------------------------------
// Register-resident row bodies. Each thread owns float4 slots
// threadIdx.x + j * blockDim.x, j < NV, of a row of cols4 float4s.

template <int NV>
__device__ __forceinline__ void load_row(float4 (&v)[NV], const float4 *row, int cols4) {
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    v[j] = i < cols4 ? __ldcs(row + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// RMSNorm of one row: out = x * scale * w, scale = 1 / sqrtf(ss / cols + eps)
// (IEEE division and square root, the llama2.c order of run.c's rmsnorm as
// restated in applications/loom_private/decoder/decoder.cu:71-76).
template <int NV>
__device__ __forceinline__ void rmsnorm_row(const float4 *x, const float4 *w, float4 *out,
                                            uint2 *out_bf16, int cols4, int cols,
                                            float eps, float *scratch) {
  float4 v[NV];
  load_row<NV>(v, x, cols4);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  ss = block_sum(ss, scratch);
  const float scale = 1.0f / sqrtf(ss / (float)cols + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4) {
      const float4 g = __ldg(w + i);
      float4 o;
      o.x = g.x * (scale * v[j].x);
      o.y = g.y * (scale * v[j].y);
      o.z = g.z * (scale * v[j].z);
      o.w = g.w * (scale * v[j].w);
      if (out != nullptr) __stcs(out + i, o);
      if (out_bf16 != nullptr) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(o.x, o.y);
        __nv_bfloat162 hi = __floats2bfloat162_rn(o.z, o.w);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t *>(&lo);
        packed.y = *reinterpret_cast<uint32_t *>(&hi);
        out_bf16[i] = packed;
      }
    }
  }
}

// Softmax of one row held in registers: max, then e = expf(l - max) kept in
// registers, their sum, then e / sum. One read, one write.
template <int NV>
__device__ __forceinline__ void softmax_row(const float4 *logits, float4 *out, int cols4,
                                            float *scratch) {
  float4 v[NV];
  load_row<NV>(v, logits, cols4);
  float m = -FLT_MAX;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4) m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
  }
  m = block_max(m, scratch);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4) {
      v[j].x = expf(v[j].x - m);
      v[j].y = expf(v[j].y - m);
      v[j].z = expf(v[j].z - m);
      v[j].w = expf(v[j].w - m);
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
  }
  s = block_sum(s, scratch);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4) {
      float4 o;
      o.x = v[j].x / s;
      o.y = v[j].y / s;
      o.z = v[j].z / s;
      o.w = v[j].w / s;
      __stcs(out + i, o);
    }
  }
}

// Clears the sign of every byte equal to 0x80 (E4M3 -0): the spec's
// rounding rule encodes a magnitude that rounds to zero as +0 (code 0),
// whereas the hardware conversion keeps the sign. Exact zero-byte test:
// bytes of t that are 0 get 0x80 in z.
__device__ __forceinline__ uint32_t e4m3_positive_zero(uint32_t codes) {
  const uint32_t t = codes ^ 0x80808080u;
  const uint32_t z = ~(((t & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | t | 0x7F7F7F7Fu);
  return codes & ~z;
}

// Two fp32 values to two OCP E4M3 codes (round to nearest even, saturating
// to +-448; NaN stays NaN; a zero result is +0): lo in the low byte, hi in
// the high byte.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return e4m3_positive_zero((uint32_t)r);
}

// Per-row E4M3 quantization of values held in registers: amax over the row,
// inv = 448 / amax and scale = amax / 448 (both IEEE fp32; 0 for an all-zero
// row), code = E4M3(v * inv). codes holds 4 codes per float4 slot.
template <int NV>
__device__ __forceinline__ void quantize_row_e4m3(const float4 (&v)[NV], uint32_t *codes,
                                                  float *scale_out, int cols4, float *scratch) {
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4)
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
  }
  amax = block_max(amax, scratch);
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
  if (threadIdx.x == 0) *scale_out = amax / 448.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4)
      codes[i] = e4m3x2(v[j].x * inv, v[j].y * inv) | (e4m3x2(v[j].z * inv, v[j].w * inv) << 16);
  }
}

// RMSNorm of one row (as rmsnorm_row) whose GEMM operand is E4M3 with a
// per-row scale instead of bf16.
template <int NV>
__device__ __forceinline__ void rmsnorm_row_e4m3(const float4 *x, const float4 *w, float4 *out,
                                                 uint32_t *codes, float *scale_out, int cols4,
                                                 int cols, float eps, float *scratch) {
  float4 v[NV];
  load_row<NV>(v, x, cols4);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  ss = block_sum(ss, scratch);
  const float scale = 1.0f / sqrtf(ss / (float)cols + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < cols4) {
      const float4 g = __ldg(w + i);
      v[j].x = g.x * (scale * v[j].x);
      v[j].y = g.y * (scale * v[j].y);
      v[j].z = g.z * (scale * v[j].z);
      v[j].w = g.w * (scale * v[j].w);
      if (out != nullptr) __stcs(out + i, v[j]);
    }
  }
  quantize_row_e4m3<NV>(v, codes, scale_out, cols4, scratch);
}

// --- block-scaled GEMM operands written from normalized rows -------------
// (the MXFP6 and NVFP4 activation quantizers fused into the rows launch)

// Two fp32 values to two E3M2 codes (round to nearest even, saturating to
// +-28; a zero result is +0): lo in bits 0-7, hi in bits 8-15.
__device__ __forceinline__ uint32_t e3m2x2_codes(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e3m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  uint32_t c = r;
  if ((c & 0xFFu) == 0x20u) c &= ~0xFFu;  // -0 -> +0
  if ((c & 0xFF00u) == 0x2000u) c &= ~0xFF00u;
  return c;
}

// Byte offset of scale (row, scale column c) in the 512-byte atom layout of
// the block-scaled GEMM's A operand (rows in groups of 128, 4 scale columns
// per atom; the layout sf_to_atoms writes).
__device__ __forceinline__ size_t a_atom_offset(int row, int c, int katoms) {
  const int mm = row % 128;
  return ((size_t)(row / 128) * katoms + c / 4) * 512 + (mm % 32) * 16 + (mm / 32) * 4 + (c % 4);
}

// MXFP6 (E3M2, UE8M0 per 32 values) operand of one normalized row held as
// float4 slots tid + j * blockDim.x: the 8 lanes of a 32-value block share
// its amax by shuffles, 4 lanes of a 16-value group gather their 6-bit codes
// into the packed 16-byte group (12 bytes of fields, 4 zero bytes), and the
// block's first lane writes the scale atom byte. The arithmetic is the
// standalone quantizer's: shared = ilogb(amax) - 4, v * 2^-shared, E3M2.
// blockDim.x must be a multiple of 8 (it is a multiple of 32).
template <int NV>
__device__ __forceinline__ void mxfp6_row(const float4 (&o)[NV], uint8_t *operand_row, uint8_t *atoms, int row,
                                          int katoms, int cols4) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * blockDim.x;  // float4 slot: columns 4i .. 4i + 3
    const bool live = i < cols4;
    float amax = live ? fmaxf(fmaxf(fabsf(o[j].x), fabsf(o[j].y)), fmaxf(fabsf(o[j].z), fabsf(o[j].w))) : 0.f;
#pragma unroll
    for (int m = 1; m < 8; m <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    int shared = 0;
    uint32_t scale_code = 0;
    if (amax != 0.f) {
      shared = ilogbf(amax) - 4;
      shared = max(-127, min(127, shared));
      scale_code = (uint32_t)(shared + 127);
    }
    const float f = amax != 0.f ? ldexpf(1.0f, -shared) : 0.f;
    const uint32_t a = e3m2x2_codes(o[j].x * f, o[j].y * f), b = e3m2x2_codes(o[j].z * f, o[j].w * f);
    const uint32_t c24 = (a & 63u) | (((a >> 8) & 63u) << 6) | ((b & 63u) << 12) | (((b >> 8) & 63u) << 18);
    const uint32_t c1 = __shfl_down_sync(0xffffffffu, c24, 1);
    const uint32_t c2 = __shfl_down_sync(0xffffffffu, c24, 2);
    const uint32_t c3 = __shfl_down_sync(0xffffffffu, c24, 3);
    if (live && (lane & 3) == 0)
      *reinterpret_cast<uint4 *>(operand_row + (size_t)(i / 4) * 16) =
          make_uint4(c24 | (c1 << 24), (c1 >> 8) | (c2 << 16), (c2 >> 16) | (c3 << 8), 0u);
    if (live && (lane & 7) == 0) atoms[a_atom_offset(row, i / 8, katoms)] = (uint8_t)scale_code;
  }
}

}  // namespace rowops
}  // namespace ce
