// Batched greedy decode step of a Llama-2 transformer (the llama2.c model:
// token embedding, n_layers x [RMSNorm -> QKV -> RoPE -> causal attention
// over the KV cache -> output projection -> residual, RMSNorm -> SwiGLU FFN
// -> residual], final RMSNorm, classifier, greedy argmax), the full decoder
// step that the llama2c decoder workload of the reference
// (applications/loom_private/decoder/decoder.cu:267-296) runs only the last
// stage of. The arithmetic is the standard Llama-2 decoder, restated from the
// mathematics: rmsnorm o = w * x / sqrt(mean(x^2) + 1e-5); RoPE rotates each
// (even, odd) pair of q and k at head-dimension index j by pos * 10000^(-j/hs);
// attention softmax(q k^T / sqrt(hs)) v per head over positions 0..pos;
// SwiGLU w2(silu(w1 x) * w3 x) with silu(g) = g / (1 + e^-g).
//
// B200 layout. The residual stream x is fp32 [batch][dim]; every GEMM operand
// is bf16 (the normalized rows, the attention output, the SwiGLU product) and
// every GEMM accumulates and writes fp32 through the tcgen05 engine of
// gemm.cu. Weights are bf16 [out][in] (K-major), the per-layer QKV rows
// stacked [q; k; v] and the FFN's w1 and w3 rows interleaved (w1_0, w3_0,
// w1_1, ...) so each is one GEMM and the SwiGLU pairs meet in one tile of
// the w1|w3 GEMM, whose epilogue writes the w2 operand directly. The KV
// cache is bf16 [layer][batch][kv_head][seq_len][head_size]: the keys of one
// (sequence, head) are one contiguous run that bulk copies move into shared
// memory. Decode attention streams each (sequence, head), or a balanced
// share of its positions, through one single-warp CTA with an online softmax
// (attn_decode_kernel). The current position and step live
// in device memory, advanced by the last launch of the step, so one captured
// step graph replays for every token.
//
// Row-sharded tensor parallelism (world > 1): rank r of n holds the rows of
// every weight that produce its slice of each output (its n_heads / n query
// heads and n_kv_heads / n KV heads of the QKV rows and of the cache, dim / n
// rows of wo and w2, hidden / n interleaved w1|w3 pairs, vocab / n classifier
// rows) and computes them on the full, replicated activations; the host joins
// the slices with all-gathers between the segments of ce_llama_enqueue_segment
// (attention output, o-projection output, SwiGLU product, w2 output, and the
// per-rank greedy candidates). The residual stream is replicated: every rank
// adds the same gathered outputs. Each rank generates exactly its rows of
// the same global random model, so the sharded and unsharded models agree.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "row_ops.cuh"

namespace ce {

int gemm_bf16(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
              int ldb, int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group = 0);
int gemm_bf16_split(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
                    int ldb, int ldd, int splits, long long split_stride, cudaStream_t s, bool pdl);
int gemm_bf16_auto_splits(int M, int N, int K, int max_splits, int min_kblocks);
int gemm_bf16_swiglu(uint16_t *out, int ld_out, const uint16_t *a, const uint16_t *b, int M, int N,
                     int K, int lda, int ldb, cudaStream_t s, bool pdl);
int gemm_w4a16(float *d, const uint16_t *a, const uint8_t *codes_t, const uint8_t *scales_t,
               const float *alpha, int M, int N, int K, int lda, int ldd, int splits,
               long long split_stride, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl);
int gemm_w4a16_auto_splits(int M, int N, int K, int max_splits, int min_kblocks);
int gemm_w4t(float *d, const uint16_t *a, const uint8_t *packed, const float *alpha, int M, int N, int K, int lda,
             int ldd, int splits, long long split_stride, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl,
             const ExchangeWait *xw = nullptr);
int gemm_w4t_auto_splits(int M, int N, int K, int max_splits);
size_t w4t_packed_bytes(int N, int K);
int w4t_pack(uint8_t *packed, const uint8_t *codes, const uint8_t *scales, int N, int K, int ld_bytes, int nsf,
             cudaStream_t s, const int *row_map);
int w4_pack(uint8_t *codes_t, uint8_t *scales_t, const uint8_t *codes, const uint8_t *scales, int N, int K,
            int ld_bytes, int nsf, cudaStream_t s, const int *row_map = nullptr);
int quantize_nvfp4(uint8_t *codes, uint8_t *scales, float *encode_decode, unsigned int *amax_bits,
                   const float *x, int rows, int cols, int ld_bytes, cudaStream_t s);
int make_bf16_rows_map(CUtensorMap *map, const void *base, unsigned long long inner, unsigned long long outer,
                       unsigned long long ld, int box_outer);
int convert_bf16(uint16_t *out, const float *in, int rows, int cols, int ld, cudaStream_t s);
int gemm_f16(float *d, const uint16_t *a, const uint16_t *b, const float *alpha, int M, int N, int K, int lda,
             int ldb, int ldd, uint16_t *swiglu_out, int swiglu_ld, cudaStream_t s, bool pdl);
int w4t_expand_f16(uint16_t *out, const uint8_t *packed, int N, int K, cudaStream_t s);

static __device__ DeviceStatus g_llama_status;

int llama_set_wait_limit(unsigned long long ns) { return set_wait_limit_here(ns); }

namespace {

using rowops::block_max;
using rowops::block_sum;

constexpr int kRowThreads = 256;
constexpr int kAttnChunk = 32;  // positions of one attention chunk: one per lane
// chunks of K and V in flight per attention CTA (one warp); measured on the
// 110M and 7B shapes: 2 beats 3, 4 and 6 (more resident CTAs per SM hide
// more latency than a deeper ring per CTA)
constexpr int attn_stages(int) { return 2; }


__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// A GEMM operand pair: bf16, or fp16 for the NVFP4 model (whose W4A16 GEMM
// multiplies fp16 x fp16).
__device__ __forceinline__ uint32_t pack_operand(float lo, float hi, int f16) {
  if (f16) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
  return pack_bf16x2(lo, hi);
}

// splitmix64 of a counter: the deterministic source of the random init.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// N(0, std) bf16 values (Box-Muller on two 24-bit uniforms of one counter)
// into the first `filled` elements of each of the n / filled runs of `run`
// elements at out (filled == run: one contiguous fill of n elements). The
// value at element e is a function of (seed, stream, e) only.
__global__ void init_normal_bf16_kernel(uint16_t *out, size_t n, uint64_t seed, uint64_t stream,
                                        float std, size_t run, size_t filled, size_t group_runs = 1,
                                        size_t global_group_runs = 1, size_t group_offset = 0) {
  // local run r of a group of group_runs is global run (r / group_runs) *
  // global_group_runs + group_offset + r % group_runs (the KV heads of a shard)
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += step) {
    const size_t run_local = k / filled;
    const size_t rg = (run_local / group_runs) * global_group_runs + group_offset + run_local % group_runs;
    const size_t i = rg * run + k % filled;
    const uint64_t r = mix64(seed ^ mix64(stream * 0x632BE59BD9B4E019ull + i));
    const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((r >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    __nv_bfloat16 h = __float2bfloat16_rn(z * std);
    out[k / filled * run + k % filled] = *reinterpret_cast<uint16_t *>(&h);
  }
}

// Rows of stacked per-layer bf16 matrices: local element (l, i, c) of
// [layers][rows][cols] takes the value of global element (l, map[i], c) of
// [layers][global_rows][cols] (stream `stream` of seed).
__global__ void init_rows_bf16_kernel(uint16_t *out, int layers, int rows, int cols, int global_rows,
                                      const int *map, uint64_t seed, uint64_t stream, float std) {
  const size_t n = (size_t)layers * rows * cols;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += step) {
    const size_t c = k % cols, li = k / cols;
    const size_t l = li / rows, i = li % rows;
    const size_t g = ((size_t)l * global_rows + map[i]) * cols + c;
    const uint64_t r = mix64(seed ^ mix64(stream * 0x632BE59BD9B4E019ull + g));
    const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((r >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    __nv_bfloat16 h = __float2bfloat16_rn(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2) * std);
    out[k] = *reinterpret_cast<uint16_t *>(&h);
  }
}

// As init_normal_bf16_kernel, fp32 values (the source of quantized weights).
__global__ void init_normal_f32_kernel(float *out, size_t n, uint64_t seed, uint64_t stream, float std) {
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const uint64_t r = mix64(seed ^ mix64(stream * 0x632BE59BD9B4E019ull + i));
    const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((r >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    out[i] = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2) * std;
  }
}

__global__ void fill_f32_kernel(float *out, size_t n, float v) {
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) out[i] = v;
}

// One row of the residual stream per block of THREADS: x = embedding[token]
// (first layer), or x += delta (after a sublayer; delta is the sum of nsplit
// split-K partials split_stride floats apart), then xb = bf16(w * (x *
// scale)), scale = 1 / sqrtf(sum(x^2) / dim + eps). An out-of-range token
// makes the row NaN so the failure shows in every output. A decode step has
// one block per sequence (64 for the 7B bench), so each thread issues all of
// its split partials' loads before the first add (the sum stays in split
// order): with one load in flight per thread the kernel waited on L2 latency
// nsplit times over.
template <int NV, int THREADS>
__global__ void __launch_bounds__(THREADS)
residual_rmsnorm_kernel(float *x, const float *delta, int nsplit, size_t split_stride,
                        const uint16_t *emb, const int *tokens, int vocab, const float *w,
                        uint16_t *xb, int dim, float eps, int f16, int shard_cols, ExchangeWait xw) {
  constexpr int kMaxLoads = 8;  // split partials loaded together
  __shared__ float scratch[32];
  pdl_launch_dependents();
  pdl_wait();
  if (xw.flags != nullptr) {  // delta from the peers' exchange puts
    if (threadIdx.x < 32) exchange_wait_warp(xw, &g_llama_status, 920u);
    __syncthreads();
  }
  const int b = blockIdx.x, cols4 = dim / 4;
  float4 *xr = reinterpret_cast<float4 *>(x + (size_t)b * dim);
  float4 v[NV];
  if (emb != nullptr) {
    const int tok = tokens[b];
    const bool ok = tok >= 0 && tok < vocab;
    const uint2 *er = reinterpret_cast<const uint2 *>(emb + (size_t)(ok ? tok : 0) * dim);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * THREADS;
      if (i < cols4) {
        const uint2 e = er[i];
        v[j] = make_float4(__uint_as_float(e.x << 16), __uint_as_float(e.x & 0xFFFF0000u),
                           __uint_as_float(e.y << 16), __uint_as_float(e.y & 0xFFFF0000u));
        if (!ok) v[j] = make_float4(NAN, NAN, NAN, NAN);
        xr[i] = v[j];
      }
    }
  } else {
    const float4 *dr = delta ? reinterpret_cast<const float4 *>(delta + (size_t)b * dim) : nullptr;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * THREADS;
      if (i < cols4) {
        v[j] = xr[i];
        if (dr) {
          float4 d;
          if (shard_cols > 0) {
            // gathered shards: [shard][batch][shard_cols], shard_cols * batch apart
            const int col = 4 * i, sh = col / shard_cols;
            d = *reinterpret_cast<const float4 *>(delta + (size_t)sh * split_stride +
                                                  (size_t)b * shard_cols + (col - sh * shard_cols));
          } else {
            // the sublayer's output: its split-K partials summed in split order
            float4 e[kMaxLoads];
#pragma unroll
            for (int sp = 0; sp < kMaxLoads; ++sp)
              if (sp < nsplit) e[sp] = dr[i + sp * (split_stride / 4)];
            d = e[0];
#pragma unroll
            for (int sp = 1; sp < kMaxLoads; ++sp)
              if (sp < nsplit) d.x += e[sp].x, d.y += e[sp].y, d.z += e[sp].z, d.w += e[sp].w;
            for (int sp = kMaxLoads; sp < nsplit; ++sp) {
              const float4 f = dr[i + sp * (split_stride / 4)];
              d.x += f.x, d.y += f.y, d.z += f.z, d.w += f.w;
            }
          }
          v[j].x += d.x, v[j].y += d.y, v[j].z += d.z, v[j].w += d.w;
          xr[i] = v[j];
        }
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (threadIdx.x + j * THREADS < cols4)
      ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  ss = block_sum(ss, scratch);
  const float scale = 1.0f / sqrtf(ss / (float)dim + eps);
  uint2 *out = reinterpret_cast<uint2 *>(xb + (size_t)b * dim);
  const float4 *wr = reinterpret_cast<const float4 *>(w);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * THREADS;
    if (i < cols4) {
      const float4 g = wr[i];
      uint2 o;
      o.x = pack_operand(g.x * (v[j].x * scale), g.y * (v[j].y * scale), f16);
      o.y = pack_operand(g.z * (v[j].z * scale), g.w * (v[j].w * scale), f16);
      out[i] = o;
    }
  }
}

// RoPE on q and k (in place in the fp32 QKV rows), then k and v to the bf16
// cache: one thread per (row, pair), the q pairs of a row first, then its
// k/v pairs; grid (pair blocks, rows). Row r belongs to sequence r / per_seq
// at position *pos + off + r % per_seq (a decode step: per_seq 1, off 0; a
// prefill chunk: per_seq positions of every sequence). rope holds (cos, sin)
// of pos * 10000^(-2i/hs) for every position and pair index i.
__global__ void __launch_bounds__(256)
rope_append_kernel(float *qkv, int ld_qkv, int nsplit, size_t split_stride, uint16_t *kcache,
                   uint16_t *vcache, const float2 *rope, const int *pos_ptr, int dim, int kv_dim, int hs,
                   int kv_heads, int seq_len, int per_seq, int off) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y / per_seq;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  const int pos = *pos_ptr + off + (int)(blockIdx.y % per_seq);
  if (pos < 0 || pos >= seq_len) {
    if (threadIdx.x == 0) report_timeout(&g_llama_status, 900u);  // position out of the cache
    return;
  }
  const int qpairs = dim / 2;
  if (p >= qpairs + kv_dim / 2) return;
  float *row = qkv + (size_t)blockIdx.y * ld_qkv;
  // pair i of the QKV row: its split-K partials summed in split order
  auto pair_at = [&](int i) {
    float2 v = *reinterpret_cast<const float2 *>(row + i);
    for (int sp = 1; sp < nsplit; ++sp) {
      const float2 e = *reinterpret_cast<const float2 *>(row + sp * split_stride + i);
      v.x += e.x, v.y += e.y;
    }
    return v;
  };
  const float2 *rp = rope + (size_t)pos * (hs / 2);
  if (p < qpairs) {
    const int i = 2 * p;
    const float2 cs = rp[(i % hs) / 2];
    const float2 q = pair_at(i);
    // rotated q, read by the attention from partial 0
    *reinterpret_cast<float2 *>(row + i) = make_float2(q.x * cs.x - q.y * cs.y, q.x * cs.y + q.y * cs.x);
    return;
  }
  const int i = 2 * (p - qpairs), kh = i / hs, d = i % hs;
  const float2 cs = rp[d / 2];
  const float2 k = pair_at(dim + i), v = pair_at(dim + kv_dim + i);
  const size_t at = ((size_t)b * kv_heads + kh) * seq_len * hs + (size_t)pos * hs + d;
  *reinterpret_cast<uint32_t *>(kcache + at) = pack_bf16x2(k.x * cs.x - k.y * cs.y, k.x * cs.y + k.y * cs.x);
  *reinterpret_cast<uint32_t *>(vcache + at) = pack_bf16x2(v.x, v.y);
}

__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xFFFF0000u); }

// o[0 .. VPL) += w * the VPL bf16 values at v (8- or 4-byte aligned)
template <int VPL>
__device__ __forceinline__ void attn_accumulate(float *o, const uint16_t *v, float w) {
  if constexpr (VPL == 4) {
    const uint2 x = *reinterpret_cast<const uint2 *>(v);
    o[0] += w * bf16_lo(x.x), o[1] += w * bf16_hi(x.x), o[2] += w * bf16_lo(x.y), o[3] += w * bf16_hi(x.y);
  } else {
    const uint32_t x = *reinterpret_cast<const uint32_t *>(v);
    o[0] += w * bf16_lo(x), o[1] += w * bf16_hi(x);
  }
}

// Decode attention of one (sequence, head), or of one of `splits` balanced
// ranges of its position chunks, by one warp: the warp streams its chunks of
// 32 K and V rows through a ring of attn_stages(HS) bulk copies (separate K
// and V barriers, so the scores of a chunk run while its V rows land) and
// keeps an online softmax: running max m, per-lane sums and the
// unnormalized output o, rescaled by e^(m_old - m_new) per chunk, s = q . k_t
// / sqrt(hs). Lane t scores position t of the chunk: its K row is read in
// 16-byte pieces rotated by the lane (lanes of one shared-memory phase hit 8
// different bank groups) against q held in registers in the same rotation.
// For the output each lane owns hs / 32 consecutive dimensions of every V
// row (coalesced) with the chunk's weights broadcast from shared memory. No
// block barrier anywhere: small CTAs, many per SM, hide each other's
// latencies. With one split the CTA writes att = bf16(o / l) itself; with
// several, each writes its (m, l, o) to part and the last of the (sequence,
// head)'s CTAs to arrive (an arrival counter that it resets) merges them in
// split order.
template <int HS>
__global__ void __launch_bounds__(32)
attn_decode_kernel(const float *qkv, int ld_qkv, const uint16_t *kcache, const uint16_t *vcache,
                   const int *pos_ptr, int n_heads, int kv_heads, int seq_len, int splits,
                   float *part, int *arrivals, uint16_t *att, int dim, int f16) {
  constexpr int ST = attn_stages(HS);
  constexpr int R = HS / 8;                        // 16-byte pieces per K row
  constexpr int VPL = HS / 32;                     // output dimensions per lane
  constexpr size_t kStage = (size_t)kAttnChunk * HS;  // elements of one K (or V) chunk
  static_assert(VPL == 2 || VPL == 4, "head size 64 or 128");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar[ST][2];      // [stage][K, V]
  uint16_t *ring = reinterpret_cast<uint16_t *>(smem);               // [stage][K | V][32][HS]
  float *es = reinterpret_cast<float *>(ring + 2 * ST * kStage);      // [32] weights of a chunk

  pdl_launch_dependents();
  pdl_wait();
  const int sp = blockIdx.x, h = blockIdx.y, b = blockIdx.z, lane = threadIdx.x;
  const int bh = b * n_heads + h;
  const int n = *pos_ptr + 1;
  const bool valid = n >= 1 && n <= seq_len;
  const int nch = valid ? (n + kAttnChunk - 1) / kAttnChunk : 0;
  const int c0 = (int)((long long)sp * nch / splits), c1 = (int)((long long)(sp + 1) * nch / splits);
  const int kh = h / (n_heads / kv_heads);
  const size_t base = ((size_t)b * kv_heads + kh) * seq_len * HS;

  if (lane == 0) {
    for (int st = 0; st < ST; ++st) {
      mbar_init(&bar[st][0], 1);
      mbar_init(&bar[st][1], 1);
    }
    fence_barrier_init();
  }
  __syncwarp();
  auto issue = [&](int c, int st) {  // lane 0: K and V rows of chunk c into stage st
    const int t0 = c * kAttnChunk;
    const uint32_t bytes = (uint32_t)min(kAttnChunk, n - t0) * HS * 2;
    uint16_t *kd = ring + (size_t)st * 2 * kStage;
    mbar_arrive_expect_tx(&bar[st][0], bytes);
    bulk_g2s(kd, kcache + base + (size_t)t0 * HS, bytes, &bar[st][0]);
    mbar_arrive_expect_tx(&bar[st][1], bytes);
    bulk_g2s(kd + kStage, vcache + base + (size_t)t0 * HS, bytes, &bar[st][1]);
  };
  if (lane == 0)
    for (int c = c0; c < c1 && c < c0 + ST; ++c) issue(c, c - c0);

  // q / sqrt(hs) in registers, piece jj holding q[8j .. 8j+7] for the piece
  // j = (jj + lane) mod R that this lane reads of its K row at step jj
  const float qscale = rsqrtf((float)HS);
  const float *qg = qkv + (size_t)b * ld_qkv + (size_t)h * HS;
  float qr[R][8];
#pragma unroll
  for (int jj = 0; jj < R; ++jj) {
    const int j = (jj + lane) & (R - 1);
    const float4 x0 = *reinterpret_cast<const float4 *>(qg + j * 8);
    const float4 x1 = *reinterpret_cast<const float4 *>(qg + j * 8 + 4);
    qr[jj][0] = x0.x * qscale, qr[jj][1] = x0.y * qscale, qr[jj][2] = x0.z * qscale, qr[jj][3] = x0.w * qscale;
    qr[jj][4] = x1.x * qscale, qr[jj][5] = x1.y * qscale, qr[jj][6] = x1.z * qscale, qr[jj][7] = x1.w * qscale;
  }

  float m = -INFINITY, lsum = 0.f, o[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) o[v] = 0.f;
  bool ok = valid;
  int c = c0;
  for (; ok && c < c1; ++c) {
    const int i = c - c0, st = i % ST;
    const uint32_t parity = (uint32_t)(i / ST) & 1u;
    const int cnt = min(kAttnChunk, n - c * kAttnChunk);
    const uint16_t *ks = ring + (size_t)st * 2 * kStage, *vs = ks + kStage;
    if (!warp_wait(&bar[st][0], parity, &g_llama_status, 901u)) {
      ok = false;
      break;
    }
    float sc = -INFINITY;
    if (lane < cnt) {
      const uint4 *kr = reinterpret_cast<const uint4 *>(ks + (size_t)lane * HS);
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int jj = 0; jj < R; ++jj) {
        const uint4 kv = kr[(jj + lane) & (R - 1)];
        a0 += qr[jj][0] * bf16_lo(kv.x) + qr[jj][1] * bf16_hi(kv.x);
        a1 += qr[jj][2] * bf16_lo(kv.y) + qr[jj][3] * bf16_hi(kv.y);
        a0 += qr[jj][4] * bf16_lo(kv.z) + qr[jj][5] * bf16_hi(kv.z);
        a1 += qr[jj][6] * bf16_lo(kv.w) + qr[jj][7] * bf16_hi(kv.w);
      }
      sc = a0 + a1;
    }
    float cmax = sc;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
    const float m_new = fmaxf(m, cmax);
    const float rescale = expf(m - m_new);  // 0 for the first chunk (m = -inf)
    const float e = lane < cnt ? expf(sc - m_new) : 0.f;
    lsum = lsum * rescale + e;
    m = m_new;
    es[lane] = e;
    __syncwarp();
    if (!warp_wait(&bar[st][1], parity, &g_llama_status, 902u)) {
      ok = false;
      break;
    }
#pragma unroll
    for (int v = 0; v < VPL; ++v) o[v] *= rescale;
    const uint16_t *vr = vs + lane * VPL;
    if (cnt == kAttnChunk) {
#pragma unroll 8
      for (int t = 0; t < kAttnChunk; ++t) attn_accumulate<VPL>(o, vr + (size_t)t * HS, es[t]);
    } else {
      for (int t = 0; t < cnt; ++t) attn_accumulate<VPL>(o, vr + (size_t)t * HS, es[t]);
    }
    __syncwarp();  // stage st and es are free
    if (lane == 0 && c + ST < c1) issue(c + ST, st);
  }
  if (!ok) {
    // a staging wait gave up: let this CTA's copies still in flight land
    // (bounded waits) before it exits, and leave NaN outputs
    for (int cc = c; cc < c1 && cc < c + ST; ++cc) {
      const int i = cc - c0;
      mbar_wait(&bar[i % ST][0], (uint32_t)(i / ST) & 1u, &g_llama_status, 903u);
      mbar_wait(&bar[i % ST][1], (uint32_t)(i / ST) & 1u, &g_llama_status, 903u);
    }
    m = NAN;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
  if (splits == 1) {
    const float inv = (ok && lsum > 0.f) ? 1.0f / lsum : NAN;
    uint16_t *dst = att + (size_t)b * dim + (size_t)h * HS + lane * VPL;
    if constexpr (VPL == 4) {
      uint2 w;
      w.x = pack_operand(o[0] * inv, o[1] * inv, f16);
      w.y = pack_operand(o[2] * inv, o[3] * inv, f16);
      *reinterpret_cast<uint2 *>(dst) = w;
    } else {
      *reinterpret_cast<uint32_t *>(dst) = pack_operand(o[0] * inv, o[1] * inv, f16);
    }
    return;
  }
  float *out = part + ((size_t)bh * splits + sp) * (HS + 2);
#pragma unroll
  for (int v = 0; v < VPL; ++v) out[2 + lane * VPL + v] = o[v];
  if (lane == 0) {
    out[0] = (c1 > c0 || !ok) ? m : -INFINITY;
    out[1] = lsum;
  }
  __threadfence();
  __syncwarp();  // this CTA's partial is written
  int last = 0;
  if (lane == 0) {
    const int before = atomicAdd(&arrivals[bh], 1);
    last = before == splits - 1;
    if (last) arrivals[bh] = 0;
  }
  if (!__shfl_sync(0xffffffffu, last, 0)) return;
  __threadfence();
  const float *pp = part + (size_t)bh * splits * (HS + 2);
  for (int d = lane; d < HS; d += 32) {
    float M = -INFINITY;
    for (int k = 0; k < splits; ++k) M = fmaxf(M, __ldcg(pp + k * (HS + 2)));
    float L = 0.f, acc = 0.f;
    for (int k = 0; k < splits; ++k) {
      const float mk = __ldcg(pp + k * (HS + 2));
      if (mk == -INFINITY) continue;
      const float f = expf(mk - M);
      L += __ldcg(pp + k * (HS + 2) + 1) * f;
      acc += __ldcg(pp + k * (HS + 2) + 2 + d) * f;
    }
    const uint32_t r = pack_operand(acc / L, 0.f, f16);
    att[(size_t)b * dim + (size_t)h * HS + d] = (uint16_t)(r & 0xFFFFu);
  }
}

// Prefill attention: causal attention of a chunk of per_seq query positions
// of every sequence (chunk row r = sequence r / per_seq, position *pos + off
// + r % per_seq) over its cache, positions 0 .. the query's own (appended by
// rope_append_kernel before this launch). One CTA per (tile of kPfQ queries,
// head, sequence), kPfThreads threads: thread t serves query t / 8 of the
// tile, with the keys t % 8 + 8 j of each key tile for the scores and the
// output dimensions 4 (t % 8) + 32 i. K and V tiles of kPfK positions are
// staged in shared memory as fp32, rows padded by 4 floats so the 16-byte
// reads of 8 threads fall in 8 different bank groups; an online softmax per
// query (max and sum over its 8 threads by shuffles) rescales the output
// after each tile, s = q . k / sqrt(hs) as in the decode attention.
constexpr int kPfQ = 16, kPfK = 64, kPfThreads = 128;
constexpr size_t pf_smem_bytes(int hs) {
  return ((size_t)(kPfQ + 2 * kPfK) * (hs + 4) + (size_t)kPfQ * (kPfK + 4)) * sizeof(float);
}

template <int HS>
__global__ void __launch_bounds__(kPfThreads)
attn_prefill_kernel(const float *qkv, int ld_qkv, const uint16_t *kcache, const uint16_t *vcache,
                    const int *pos_ptr, int off, int per_seq, int n_heads, int kv_heads, int seq_len,
                    uint16_t *att, int dim, int f16) {
  extern __shared__ __align__(16) float pf_smem[];
  constexpr int LD = HS + 4, PLD = kPfK + 4, NI = HS / 32;
  float *qs = pf_smem;         // [kPfQ][LD]
  float *ks = qs + kPfQ * LD;  // [kPfK][LD]
  float *vs = ks + kPfK * LD;  // [kPfK][LD]
  float *ps = vs + kPfK * LD;  // [kPfQ][PLD]
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.z, h = blockIdx.y, c0 = blockIdx.x * kPfQ;
  const int kvh = h / (n_heads / kv_heads);
  const int t = threadIdx.x, qi = t >> 3, g = t & 7;
  const int base = *pos_ptr + off;         // position of the chunk's first row
  const int nq = min(kPfQ, per_seq - c0);  // live queries of the tile
  const int last = base + c0 + nq - 1;     // position of its last one
  if (base < 0 || last >= seq_len) {
    if (t == 0) report_timeout(&g_llama_status, 901u);  // position out of the cache
    return;
  }
  const float qscale = rsqrtf((float)HS);
  for (int i = t; i < kPfQ * HS / 4; i += kPfThreads) {
    const int r = i / (HS / 4), d4 = i % (HS / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nq) {
      v = *reinterpret_cast<const float4 *>(qkv + (size_t)(b * per_seq + c0 + r) * ld_qkv + h * HS + 4 * d4);
      v.x *= qscale, v.y *= qscale, v.z *= qscale, v.w *= qscale;
    }
    *reinterpret_cast<float4 *>(qs + r * LD + 4 * d4) = v;
  }
  const int my_pos = base + c0 + qi;
  const size_t head_off = ((size_t)b * kv_heads + kvh) * seq_len * HS;
  const uint16_t *kh = kcache + head_off, *vh = vcache + head_off;
  float m = -INFINITY, l = 0.f;
  float o[NI][4];
#pragma unroll
  for (int i = 0; i < NI; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int k0 = 0; k0 <= last; k0 += kPfK) {
    const int nk = min(kPfK, last + 1 - k0);
    __syncthreads();  // the previous tile's readers are done (first time: q staged)
    for (int i = t; i < kPfK * HS / 8; i += kPfThreads) {
      const int r = i / (HS / 8), d8 = i % (HS / 8);
      uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
      if (r < nk) {
        kv = *reinterpret_cast<const uint4 *>(kh + (size_t)(k0 + r) * HS + 8 * d8);
        vv = *reinterpret_cast<const uint4 *>(vh + (size_t)(k0 + r) * HS + 8 * d8);
      }
      float4 *kd = reinterpret_cast<float4 *>(ks + r * LD + 8 * d8);
      float4 *vd = reinterpret_cast<float4 *>(vs + r * LD + 8 * d8);
      kd[0] = make_float4(bf16_lo(kv.x), bf16_hi(kv.x), bf16_lo(kv.y), bf16_hi(kv.y));
      kd[1] = make_float4(bf16_lo(kv.z), bf16_hi(kv.z), bf16_lo(kv.w), bf16_hi(kv.w));
      vd[0] = make_float4(bf16_lo(vv.x), bf16_hi(vv.x), bf16_lo(vv.y), bf16_hi(vv.y));
      vd[1] = make_float4(bf16_lo(vv.z), bf16_hi(vv.z), bf16_lo(vv.w), bf16_hi(vv.w));
    }
    __syncthreads();
    float sc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HS; d += 4) {
      const float4 q = *reinterpret_cast<const float4 *>(qs + qi * LD + d);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 k = *reinterpret_cast<const float4 *>(ks + (g + 8 * j) * LD + d);
        sc[j] = fmaf(q.x, k.x, sc[j]);
        sc[j] = fmaf(q.y, k.y, sc[j]);
        sc[j] = fmaf(q.z, k.z, sc[j]);
        sc[j] = fmaf(q.w, k.w, sc[j]);
      }
    }
    float tmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int kj = g + 8 * j;
      if (kj >= nk || k0 + kj > my_pos) sc[j] = -INFINITY;
      tmax = fmaxf(tmax, sc[j]);
    }
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
    const float m_new = fmaxf(m, tmax);
    const float rescale = m_new == -INFINITY ? 1.f : expf(m - m_new);  // 0 on the first tile
    float psum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e = sc[j] == -INFINITY ? 0.f : expf(sc[j] - m_new);
      ps[qi * PLD + g + 8 * j] = e;
      psum += e;
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    psum += __shfl_xor_sync(0xffffffffu, psum, 4);
    l = l * rescale + psum;
    m = m_new;
#pragma unroll
    for (int i = 0; i < NI; ++i) o[i][0] *= rescale, o[i][1] *= rescale, o[i][2] *= rescale, o[i][3] *= rescale;
    __syncwarp();  // a query's weights are written and read by the 8 lanes of one warp
    for (int k = 0; k < nk; ++k) {
      const float pk = ps[qi * PLD + k];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const float4 v = *reinterpret_cast<const float4 *>(vs + k * LD + 4 * g + 32 * i);
        o[i][0] = fmaf(pk, v.x, o[i][0]);
        o[i][1] = fmaf(pk, v.y, o[i][1]);
        o[i][2] = fmaf(pk, v.z, o[i][2]);
        o[i][3] = fmaf(pk, v.w, o[i][3]);
      }
    }
  }
  if (qi < nq) {
    const float inv = 1.f / l;
    uint16_t *dst = att + (size_t)(b * per_seq + c0 + qi) * dim + h * HS;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      uint2 w;
      w.x = pack_operand(o[i][0] * inv, o[i][1] * inv, f16);
      w.y = pack_operand(o[i][2] * inv, o[i][3] * inv, f16);
      *reinterpret_cast<uint2 *>(dst + 4 * g + 32 * i) = w;
    }
  }
}

// Prefill attention on the tensor cores (the kernel the prefill runs; the
// SIMT kernel above states the same arithmetic plainly). One CTA per (tile of
// kFaM = 128 query positions, head, sequence), six warps:
//   warps 0-7  one query row and one column half per thread (warps w and
//              w + 4 share the TMEM lanes of row quarter w): stage q log2(e)
//              / sqrt(hs) as bf16 into shared memory (128-byte swizzled,
//              K-major), so scores come in base-2 units; per key tile read
//              the half's scores from TMEM, mask keys past the query, swap
//              the half-row maxima with the partner warp (shared memory,
//              bounded wait), online softmax with weights 2^(s - m) (running
//              max m, the half's sum of the bf16-rounded weights), rescale
//              the half's output columns in TMEM when m grows, write the
//              half's weights P as bf16 into TMEM; at the end the two sums
//              are added and O / l goes to att;
//   warp 8     one thread: TMA loads of the K and V tiles (kFaN = 128
//              positions, two stages each) from the bf16 cache;
//   warp 9     one thread issues S = Q K^T (A, B from shared memory) and
//              O += P V (A = P from TMEM, B = V as an MN-major operand straight
//              from its [positions][hs] cache layout); the warp zeroes the V
//              rows past the tile's last key (uninitialized cache rows must
//              not meet a zero weight: 0 x NaN).
// TMEM: S fp32 [128 x 128] at column 0, P bf16 pairs at 128, O fp32 [128 x
// hs] at kColO. Every wait is bounded; a timeout records its site and the
// CTA drains its copies and MMAs before freeing TMEM.
// 2^x by the ex2.approx instruction (relative error ~2^-22, far below the
// bf16 rounding of the weights it feeds); 2^-inf = +0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr int kFaM = 128, kFaN = 128, kFaThreads = 320;
template <int HS>
struct FaLayout {
  static constexpr int q_bytes = kFaM * HS * 2;   // HS / 64 blocks of [128 rows][128 B]
  static constexpr int kv_bytes = kFaN * HS * 2;  // one K or V tile, HS / 64 boxes of [128 rows][128 B]
  static constexpr int k_off = q_bytes;
  static constexpr int v_off = k_off + 2 * kv_bytes;
  static constexpr int bar_off = v_off + 2 * kv_bytes;
  static constexpr int total = bar_off + 256 + 1024;  // barriers + TMEM holder, 1024-byte alignment slack
  static constexpr uint32_t tmem_cols = HS == 64 ? 256 : 512;
  static constexpr uint32_t col_o = HS == 64 ? 192 : 256;
};

template <int HS>
__global__ void __launch_bounds__(kFaThreads, 1)
attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const float *qkv, int ld_qkv, const int *pos_ptr, int off, int per_seq, int n_heads,
                       int kv_heads, int seq_len, long long layer_row, uint16_t *att, int dim, int f16) {
  using Lay = FaLayout<HS>;
  constexpr int KB = HS / 64;
  constexpr uint32_t kColS = 0, kColP = 128, kColO = Lay::col_o;
  extern __shared__ uint8_t fa_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *qs = sm, *ks = sm + Lay::k_off, *vs = sm + Lay::v_off;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + Lay::bar_off);
  uint64_t *kfull = bars, *vfull = bars + 2, *kempty = bars + 4, *vempty = bars + 6;
  uint64_t *q_ready = bars + 8, *s_full = bars + 9, *s_free = bars + 10, *p_full = bars + 11,
           *o_ready = bars + 12, *done = bars + 13;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 16);
  __shared__ int abort_flag;
  __shared__ float pair_max[2][2][kFaM];  // [tile parity][column half][row]: the halves' row maxima
  __shared__ float pair_l[2][kFaM];       // [column half][row]: the halves' weight sums
  __shared__ unsigned pair_count[4];      // postings per row quarter (both halves)
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y, c0 = blockIdx.x * kFaM;
  const int kvh = h / (n_heads / kv_heads);
  const int base = *pos_ptr + off;
  const int nq = min(kFaM, per_seq - c0);
  const int first = base + c0, last = first + nq - 1;
  if (base < 0 || last >= seq_len) {
    if (threadIdx.x == 0) report_timeout(&g_llama_status, 901u);  // position out of the cache
    return;
  }
  const int ntiles = last / kFaN + 1;
  const int nk_last = last + 1 - (ntiles - 1) * kFaN;  // keys of the last tile
  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) mbar_init(bars + i, 1);
    mbar_init(q_ready, 8);
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(p_full, 8);
    mbar_init(o_ready, 1);
    mbar_init(done, 1);
    abort_flag = 0;
    for (int i = 0; i < 4; ++i) pair_count[i] = 0u;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_holder, Lay::tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  volatile int *abort_v = &abort_flag;
  // warp-uniform: every lane of the warp takes the same branch
  auto aborted = [&]() { return __any_sync(0xffffffffu, *abort_v != 0) != 0; };

  if (warp < 8) {
    // thread: row r (its TMEM lane), column half hh of S, P and O; the two
    // warps of a row quarter (w, w + 4) exchange row maxima through shared
    // memory with a bounded wait and add their weight sums at the end
    const int r = (warp & 3) * 32 + lane, hh = warp >> 2;
    {  // Q tile: this half's 16-byte chunks of row r
      // scores in base-2 units: q / sqrt(hs) * log2(e), weights 2^(s - m)
      const float qscale = rsqrtf((float)HS) * 1.4426950408889634f;
      const float *qrow = qkv + (size_t)(b * per_seq + c0 + r) * ld_qkv + h * HS;
#pragma unroll
      for (int t = hh * KB * 4; t < (hh + 1) * KB * 4; ++t) {
        const int kb = t / 8, c = t % 8;
        float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
        if (r < nq) {
          x0 = *reinterpret_cast<const float4 *>(qrow + kb * 64 + c * 8);
          x1 = *reinterpret_cast<const float4 *>(qrow + kb * 64 + c * 8 + 4);
        }
        uint4 v;
        v.x = pack_bf16x2(x0.x * qscale, x0.y * qscale);
        v.y = pack_bf16x2(x0.z * qscale, x0.w * qscale);
        v.z = pack_bf16x2(x1.x * qscale, x1.y * qscale);
        v.w = pack_bf16x2(x1.z * qscale, x1.w * qscale);
        *reinterpret_cast<uint4 *>(qs + kb * (kFaM * 128) + r * 128 + ((c ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    constexpr int kHalfS = kFaN / 2, kHalfO = HS / 2;
    const int qpos = first + r;
    const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t colS = kColS + hh * kHalfS, colP = kColP + hh * (kHalfS / 2), colO = kColO + hh * kHalfO;
    unsigned *cnt = &pair_count[warp & 3];
    // posts this warp's value for row r, then waits (bounded) until the
    // partner warp has posted `target` times in all; returns its value
    auto exchange = [&](float *mine, float *theirs, float v, unsigned target, unsigned where, float *out) {
      *mine = v;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) atomicAdd(cnt, 1u);
      bool done_ok = true;
      if (lane == 0) {
        const unsigned long long t0 = globaltimer();
        while (*reinterpret_cast<volatile unsigned *>(cnt) < target) {
          if (globaltimer() - t0 > wait_limit_ns()) {
            report_timeout(&g_llama_status, where);
            done_ok = false;
            break;
          }
        }
      }
      done_ok = __shfl_sync(0xffffffffu, done_ok ? 1 : 0, 0) != 0;
      __syncwarp();  // orders lane 0's observation before every lane's read
      __threadfence_block();
      *out = *reinterpret_cast<volatile float *>(theirs);
      return done_ok;
    };
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      ok = warp_wait(s_full, j & 1, &g_llama_status, 910u) && !aborted();
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[kHalfS];
#pragma unroll
      for (int q = 0; q < kHalfS / 32; ++q)
        tmem_ld_32x32b_x32(tbase + lanes + colS + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(sv + 32 * q));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      const int kmax = min(qpos, last) - j * kFaN - hh * kHalfS;  // last valid column of this half
      float tmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < kHalfS; ++i) {
        const float sc = i <= kmax ? __uint_as_float(sv[i]) : -INFINITY;
        sv[i] = __float_as_uint(sc);
        tmax = fmaxf(tmax, sc);
      }
      float other;
      ok = exchange(&pair_max[j & 1][hh][r], &pair_max[j & 1][hh ^ 1][r], tmax, 2u * (j + 1), 921u, &other);
      ok = __all_sync(0xffffffffu, ok) && !aborted();
      if (!ok) break;
      const float m_new = fmaxf(m, fmaxf(tmax, other));  // finite: key 0 is valid for every row
      const float alpha = ex2_approx(m - m_new);  // 2^-inf = 0 on the first tile
      float rs = 0.f;
      uint32_t pk[kHalfS / 2];
#pragma unroll
      for (int i = 0; i < kHalfS / 2; ++i) {
        // masked scores are -inf: 2^-inf = 0
        pk[i] = pack_bf16x2(ex2_approx(__uint_as_float(sv[2 * i]) - m_new),
                            ex2_approx(__uint_as_float(sv[2 * i + 1]) - m_new));
        rs += bf16_lo(pk[i]) + bf16_hi(pk[i]);
      }
      l = l * alpha + rs;  // this half's sum; the halves share m and alpha
      m = m_new;
      if (j > 0) {  // O and P are free once the previous tile's O += P V is done
        ok = warp_wait(o_ready, (j - 1) & 1, &g_llama_status, 911u) && !aborted();
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int q = 0; q < kHalfO / 32; ++q) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(tbase + lanes + colO + 32 * q, ov);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st_32x32b_x32(tbase + lanes + colO + 32 * q, ov);
          }
        }
      }
      tmem_st_32x32b_x32(tbase + lanes + colP, *reinterpret_cast<const uint32_t(*)[32]>(pk));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    float l_other = 0.f;
    if (ok) {
      ok = exchange(&pair_l[hh][r], &pair_l[hh ^ 1][r], l, 2u * (ntiles + 1), 922u, &l_other);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok && warp_wait(o_ready, (ntiles - 1) & 1, &g_llama_status, 912u)) {
      tc_fence_after();
      const float inv = 1.f / (l + l_other);
      uint16_t *dst = att + (size_t)(b * per_seq + c0 + r) * dim + h * HS + hh * kHalfO;
#pragma unroll
      for (int q = 0; q < kHalfO / 32; ++q) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(tbase + lanes + colO + 32 * q, ov);
        tmem_ld_wait();
        if (r < nq) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_operand(__uint_as_float(ov[i]) * inv, __uint_as_float(ov[i + 1]) * inv, f16);
            w.y = pack_operand(__uint_as_float(ov[i + 2]) * inv, __uint_as_float(ov[i + 3]) * inv, f16);
            w.z = pack_operand(__uint_as_float(ov[i + 4]) * inv, __uint_as_float(ov[i + 5]) * inv, f16);
            w.w = pack_operand(__uint_as_float(ov[i + 6]) * inv, __uint_as_float(ov[i + 7]) * inv, f16);
            *reinterpret_cast<uint4 *>(dst + 32 * q + i) = w;
          }
        }
      }
    } else {
      *abort_v = 1;
    }
  } else if (warp == 8) {
    if (lane == 0) {
      const long long head_row = layer_row + ((long long)b * kv_heads + kvh) * seq_len;
      int k_issued = 0, v_issued = 0;  // tiles whose K / V copies were started
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (j >= 2 && (!mbar_wait(kempty + st, ph ^ 1, &g_llama_status, 913u) || *abort_v)) break;
        mbar_arrive_expect_tx(kfull + st, Lay::kv_bytes);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          tma_load_2d(ks + st * Lay::kv_bytes + kb * (kFaN * 128), &tmK, kfull + st, kb * 64,
                      (int)(head_row + (long long)j * kFaN));
        k_issued = j + 1;
        if (j >= 2 && (!mbar_wait(vempty + st, ph ^ 1, &g_llama_status, 913u) || *abort_v)) break;
        mbar_arrive_expect_tx(vfull + st, Lay::kv_bytes);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          tma_load_2d(vs + st * Lay::kv_bytes + kb * (kFaN * 128), &tmV, vfull + st, kb * 64,
                      (int)(head_row + (long long)j * kFaN));
        v_issued = j + 1;
      }
      if (k_issued < ntiles || v_issued < ntiles) *abort_v = 1;
      // the last copies of each stage land before the CTA may exit (they are
      // complete already unless the loop ended early)
      for (int j = k_issued - 2 < 0 ? 0 : k_issued - 2; j < k_issued; ++j)
        mbar_wait(kfull + (j & 1), (j >> 1) & 1, &g_llama_status, 914u);
      for (int j = v_issued - 2 < 0 ? 0 : v_issued - 2; j < v_issued; ++j)
        mbar_wait(vfull + (j & 1), (j >> 1) & 1, &g_llama_status, 914u);
    }
  } else {
    constexpr uint32_t idesc_qk = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kFaN >> 3) << 17) |
                                  ((uint32_t)(kFaM >> 4) << 24);
    constexpr uint32_t idesc_pv = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(HS >> 3) << 17) |
                                  ((uint32_t)(kFaM >> 4) << 24);
    bool ok = warp_wait(q_ready, 0, &g_llama_status, 915u);
    bool issued_any = false;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      ok = warp_wait(kfull + st, ph, &g_llama_status, 916u) &&
           (j == 0 || warp_wait(s_free, (j - 1) & 1, &g_llama_status, 917u)) && !aborted();
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kbase = smem_u32(ks + st * Lay::kv_bytes), qbase = smem_u32(qs);
#pragma unroll
        for (int k = 0; k < HS / 16; ++k) {
          const uint64_t a = smem_desc_sw128(qbase + (k / 4) * (kFaM * 128) + (k % 4) * 32);
          const uint64_t bd = smem_desc_sw128(kbase + (k / 4) * (kFaN * 128) + (k % 4) * 32);
          tc_mma<0>(tbase + kColS, a, bd, idesc_qk, k > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        tc_commit(kempty + st);
        issued_any = true;
      }
      __syncwarp();
      ok = warp_wait(vfull + st, ph, &g_llama_status, 918u) && !aborted();
      if (!ok) break;
      if (j == ntiles - 1 && nk_last < kFaN) {
        // zero the V rows past the last key (both 64-wide chunks)
        uint8_t *vt = vs + st * Lay::kv_bytes;
        for (int i = lane; i < KB * (kFaN - nk_last) * 8; i += 32) {
          const int kb = i / ((kFaN - nk_last) * 8), rem = i % ((kFaN - nk_last) * 8);
          const int row = nk_last + rem / 8, piece = rem % 8;
          *reinterpret_cast<uint4 *>(vt + kb * (kFaN * 128) + row * 128 + piece * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      ok = warp_wait(p_full, j & 1, &g_llama_status, 919u) && !aborted();
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t vbase = smem_u32(vs + st * Lay::kv_bytes);
#pragma unroll
        for (int k = 0; k < kFaN / 16; ++k) {
          const uint64_t bd = smem_desc_sw128_mn(vbase + k * 2048, kFaN * 128);
          tc_mma_ts(tbase + kColO, tbase + kColP + k * 8, bd, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(o_ready);
        tc_commit(vempty + st);
      }
      __syncwarp();
    }
    if (!ok) *abort_v = 1;
    if (issued_any && lane == 0) {  // every MMA of this CTA complete before TMEM is freed
      tc_commit(done);
      mbar_wait(done, 0, &g_llama_status, 920u);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tbase, Lay::tmem_cols);
}

// Prefill helpers: the chunk's prompt tokens in row order (row b * per_seq + c
// takes prompt[b][off + c]); the final-norm rows of every sequence's last
// prompt position into the decode step's operand rows; the position and step
// advance after a prefill.
__global__ void prefill_tokens_kernel(int *rows_tokens, const int *prompt, int prompt_len, int off, int per_seq,
                                      int batch) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= batch * per_seq) return;
  rows_tokens[i] = prompt[(size_t)(i / per_seq) * prompt_len + off + i % per_seq];
}

__global__ void gather_rows16_kernel(uint16_t *dst, const uint16_t *src, int per_seq, int pick, int cols,
                                     int batch) {
  pdl_launch_dependents();
  pdl_wait();
  const int v8 = cols / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < batch * v8; i += gridDim.x * blockDim.x) {
    const int b = i / v8, c = i % v8;
    reinterpret_cast<uint4 *>(dst)[(size_t)b * v8 + c] =
        reinterpret_cast<const uint4 *>(src)[((size_t)b * per_seq + pick) * v8 + c];
  }
}

__global__ void advance_by_kernel(int *pos, int *step, int positions) {
  pdl_launch_dependents();
  pdl_wait();
  *pos += positions;
  *step += 1;
}


// hb = bf16(silu(g) * u), h = interleaved (g_i, u_i) pairs per row (the sum
// of nsplit split-K partials split_stride floats apart), silu(g) = g / (1 + e^-g).
// Used when the w1|w3 GEMM runs split; otherwise its epilogue does this.
__global__ void swiglu_kernel(const float *h, int nsplit, size_t split_stride, uint16_t *hb, int rows,
                              int hidden, int f16) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t n = (size_t)rows * hidden / 2;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const size_t r = (2 * i) / hidden, c = (2 * i) % hidden;
    float4 gu = *reinterpret_cast<const float4 *>(h + r * 2 * hidden + 2 * c);  // g_c, u_c, g_c+1, u_c+1
    for (int sp = 1; sp < nsplit; ++sp) {
      const float4 e = *reinterpret_cast<const float4 *>(h + sp * split_stride + r * 2 * hidden + 2 * c);
      gu.x += e.x, gu.y += e.y, gu.z += e.z, gu.w += e.w;
    }
    const float a = gu.x / (1.0f + expf(-gu.x)) * gu.y;
    const float bb = gu.z / (1.0f + expf(-gu.z)) * gu.w;
    *reinterpret_cast<uint32_t *>(hb + r * hidden + c) = pack_operand(a, bb, f16);
  }
}

// Greedy token of each row: index of the first maximum logit (NaN never
// wins); written to tokens[b] and generated[b][step] while step < cap.
__global__ void __launch_bounds__(kRowThreads)
argmax_kernel(const float *logits, int vocab, int *tokens, int *generated, int cap, const int *step_ptr) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const float *row = logits + (size_t)b * vocab;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < vocab; i += kRowThreads) {
    const float v = row[i];
    if (v > best) best = v, idx = i;  // strided order: first max of this thread
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, best, off);
    const int oi = __shfl_down_sync(0xffffffffu, idx, off);
    if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sv[w] = best, si[w] = idx;
  __syncthreads();
  if (w == 0) {
    best = lane < kRowThreads / 32 ? sv[lane] : -INFINITY;
    idx = lane < kRowThreads / 32 ? si[lane] : 0x7fffffff;
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, best, off);
      const int oi = __shfl_down_sync(0xffffffffu, idx, off);
      if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
    }
    if (lane == 0) {
      if (idx == 0x7fffffff) idx = 0;  // every logit NaN
      tokens[b] = idx;
      const int step = *step_ptr;
      if (step >= 0 && step < cap) generated[(size_t)b * cap + step] = idx;
    }
  }
}

__global__ void advance_kernel(int *pos, int *step) {
  pdl_launch_dependents();
  pdl_wait();
  *pos += 1;
  *step += 1;
}

// [shards][batch][cols] 16-bit slices to [batch][shards * cols] rows (cols % 8 == 0).
__global__ void join_shards_kernel(const uint16_t *src, uint16_t *dst, int shards, int batch, int cols) {
  pdl_launch_dependents();
  pdl_wait();
  const int v8 = cols / 8;
  const size_t n = (size_t)shards * batch * v8;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const size_t sh = i / ((size_t)batch * v8), rem = i % ((size_t)batch * v8);
    const size_t b = rem / v8, c = rem % v8;
    reinterpret_cast<uint4 *>(dst)[b * (size_t)shards * v8 + sh * v8 + c] = reinterpret_cast<const uint4 *>(src)[i];
  }
}

// dst[b][j] = sum over s (in split order) of src[s][b][j], fp32, n4 float4s per split.
__global__ void sum_splits_kernel(const float *src, float *dst, int splits, size_t n4) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += step) {
    float4 a = reinterpret_cast<const float4 *>(src)[i];
    for (int sp = 1; sp < splits; ++sp) {
      const float4 e = reinterpret_cast<const float4 *>(src)[i + sp * n4];
      a.x += e.x, a.y += e.y, a.z += e.z, a.w += e.w;
    }
    reinterpret_cast<float4 *>(dst)[i] = a;
  }
}

// This rank's delta slice: the split-K partials src [splits][rows][cols]
// (cols % 4 == 0) summed in split order and written at byte offset off
// (row stride ld floats) of every rank's delta exchange, then the peers
// are signalled.
__global__ void sum_splits_put_kernel(const float *src, int splits, int rows, int cols, ExchangePut xp, size_t off,
                                      int ld) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t n4 = (size_t)rows * cols / 4, plane = (size_t)rows * cols;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += step) {
    float4 a = reinterpret_cast<const float4 *>(src)[i];
    for (int sp = 1; sp < splits; ++sp) {
      const float4 e = reinterpret_cast<const float4 *>(src + sp * plane)[i];
      a.x += e.x, a.y += e.y, a.z += e.z, a.w += e.w;
    }
    const size_t r = 4 * i / cols, c = 4 * i % cols;
    const size_t at = off + (r * ld + c) * 4;
    for (int q = 0; q < xp.world; ++q) *reinterpret_cast<float4 *>(xp.blocks[q] + at) = a;
  }
  exchange_signal(xp);
}

// This rank's SwiGLU product (as swiglu_kernel: h interleaves (g_i, u_i),
// the sum of nsplit split-K partials) written at byte offset off (row stride
// ld values) of every rank's product exchange, then the peers are signalled.
__global__ void swiglu_put_kernel(const float *h, int nsplit, size_t split_stride, int rows, int hidden, int f16,
                                  ExchangePut xp, size_t off, int ld) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t n = (size_t)rows * hidden / 2;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const size_t r = (2 * i) / hidden, c = (2 * i) % hidden;
    float4 gu = *reinterpret_cast<const float4 *>(h + r * 2 * hidden + 2 * c);
    for (int sp = 1; sp < nsplit; ++sp) {
      const float4 e = *reinterpret_cast<const float4 *>(h + sp * split_stride + r * 2 * hidden + 2 * c);
      gu.x += e.x, gu.y += e.y, gu.z += e.z, gu.w += e.w;
    }
    const float a = gu.x / (1.0f + expf(-gu.x)) * gu.y;
    const float bb = gu.z / (1.0f + expf(-gu.z)) * gu.w;
    const uint32_t v = pack_operand(a, bb, f16);
    const size_t at = off + (r * ld + c) * 2;
    for (int q = 0; q < xp.world; ++q) *reinterpret_cast<uint32_t *>(xp.blocks[q] + at) = v;
  }
  exchange_signal(xp);
}

// --- on-device sampling --------------------------------------------------
// The token of each row drawn from softmax(logits / temperature) with the
// coin u = (mix64(seed ^ mix64(step * 0x9E3779B97F4A7C15 + row + 1)) >> 40)
// / 2^24, the sampler of llama2.c restated: without top-p, the first index
// (vocabulary order) whose cumulative probability exceeds u; with top-p in
// (0, 1), over the 1024 most probable tokens (ties to the lower index)
// sorted by descending probability, the nucleus is the shortest prefix
// whose cumulative probability exceeds top_p, and the token is the first of
// it whose cumulative probability exceeds u times the nucleus' mass. One
// 1024-thread block per row; all reductions in a fixed order.
constexpr int kSampleThreads = 1024;
constexpr int kSampleCands = 1024;

__device__ __forceinline__ float sample_coin(uint64_t seed, int step, int row) {
  const uint64_t r = mix64(seed ^ mix64((uint64_t)step * 0x9E3779B97F4A7C15ull + (uint64_t)row + 1));
  return (float)(r >> 40) * (1.0f / 16777216.0f);
}

// Block-wide sum (or max) of one value per thread, the same order every time.
template <bool kMax>
__device__ __forceinline__ float sample_reduce(float v, float *red) {
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, v, off);
    v = kMax ? fmaxf(v, o) : v + o;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = red[lane];
    for (int off = 16; off > 0; off >>= 1) {
      const float o = __shfl_xor_sync(0xffffffffu, v, off);
      v = kMax ? fmaxf(v, o) : v + o;
    }
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

// Exclusive block scan of one value per thread (thread order); returns this
// thread's prefix, and the total in *total.
__device__ __forceinline__ float sample_scan(float v, float *red, float *total) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float incl = v;
  for (int off = 1; off < 32; off <<= 1) {
    const float o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  __syncthreads();
  if (lane == 31) red[w] = incl;
  __syncthreads();
  if (w == 0) {
    float x = red[lane], xi = x;
    for (int off = 1; off < 32; off <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, xi, off);
      if (lane >= off) xi += o;
    }
    red[lane] = xi - x;  // exclusive prefix of the warp sums
    if (lane == 31) red[32] = xi;
  }
  __syncthreads();
  *total = red[32];
  return red[w] + incl - v;
}

// Block count of a predicate over the row, one chunk per thread.
__device__ __forceinline__ int sample_count(int v, int *ired) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) ired[w] = v;
  __syncthreads();
  if (w == 0) {
    v = ired[lane];
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) ired[32] = v;
  }
  __syncthreads();
  return ired[32];
}

__global__ void __launch_bounds__(kSampleThreads)
sample_kernel(const float *logits, int vocab, float temperature, float top_p, uint64_t seed, int *tokens,
              int *generated, int cap, const int *step_ptr) {
  __shared__ float red[33];
  __shared__ int ired[33];
  __shared__ unsigned long long cand[kSampleCands];
  __shared__ float cprob[kSampleCands];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  const float *row = logits + (size_t)b * vocab;
  const int chunk = (vocab + kSampleThreads - 1) / kSampleThreads;
  const int i0 = min(vocab, tid * chunk), i1 = min(vocab, i0 + chunk);
  const int step = *step_ptr;
  const float u = sample_coin(seed, step, b);
  // softmax numerators e_i = exp((l_i - max) / T)
  float mx = -INFINITY;
  for (int i = i0; i < i1; ++i) mx = fmaxf(mx, row[i]);
  mx = sample_reduce<true>(mx, red);
  const float inv_t = 1.0f / temperature;
  float part = 0.f;
  for (int i = i0; i < i1; ++i) part += expf((row[i] - mx) * inv_t);
  float total = 0.f;
  const float before = sample_scan(part, red, &total);  // prefix of the chunks in vocabulary order
  int token = vocab - 1;
  if (!(top_p > 0.f && top_p < 1.f)) {
    // inverse CDF in vocabulary order: the first i with prefix_i > u * total
    const float target = u * total;
    int found = 0x7fffffff;
    if (before <= target && before + part > target) {
      float acc = before;
      for (int i = i0; i < i1; ++i) {
        acc += expf((row[i] - mx) * inv_t);
        if (acc > target) {
          found = i;
          break;
        }
      }
      if (found == 0x7fffffff) found = i1 - 1;  // the chunk's own order of additions fell short: its end
    }
    const int f = sample_count(found == 0x7fffffff ? 0 : found + 1, ired);  // at most one thread contributes
    if (f > 0) token = f - 1;
  } else {
    // the kSampleCands largest e_i: bisection on the float bits (e_i >= 0
    // orders like its bits) for the largest threshold with enough entries
    const int want = min(vocab, kSampleCands);
    uint32_t lo = 0u, hi = 0x7F800000u;  // count(bits >= lo) >= want always
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo + 1) / 2;
      int c = 0;
      for (int i = i0; i < i1; ++i) c += __float_as_uint(expf((row[i] - mx) * inv_t)) >= mid;
      if (sample_count(c, ired) >= want) lo = mid;
      else hi = mid - 1;
    }
    // above the threshold: all; at it: the lowest indices up to `want`
    int above = 0, at = 0;
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = __float_as_uint(expf((row[i] - mx) * inv_t));
      above += k > lo;
      at += k == lo;
    }
    const int n_above = sample_count(above, ired);
    float at_total = 0.f;
    const int at_before = (int)sample_scan((float)at, red, &at_total);
    if (tid == 0) ired[32] = 0;
    __syncthreads();
    int taken_at = 0;
    for (int i = i0; i < i1; ++i) {
      const float e = expf((row[i] - mx) * inv_t);
      const uint32_t k = __float_as_uint(e);
      bool take = k > lo;
      if (k == lo) take = at_before + taken_at++ < want - n_above;
      if (take) {
        const int slot = atomicAdd(&ired[32], 1);
        if (slot < kSampleCands)
          cand[slot] = ((unsigned long long)k << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
      }
    }
    __syncthreads();
    const int n = min(ired[32], kSampleCands);
    for (int j = n + tid; j < kSampleCands; j += kSampleThreads) cand[j] = 0ull;  // pad below every entry
    __syncthreads();
    // bitonic sort, descending: probability, then lower index first
    for (int size = 2; size <= kSampleCands; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const int j = tid ^ stride;
        if (j > tid) {
          const unsigned long long a = cand[tid], c = cand[j];
          const bool desc = (tid & size) == 0;
          if (desc ? a < c : a > c) cand[tid] = c, cand[j] = a;
        }
        __syncthreads();
      }
    }
    const float p = tid < n ? __uint_as_float((uint32_t)(cand[tid] >> 32)) / total : 0.f;
    float ptot = 0.f;
    const float cum_before = sample_scan(p, red, &ptot);
    cprob[tid] = cum_before + p;  // inclusive cumulative probability
    __syncthreads();
    // nucleus: the first j whose cumulative probability exceeds top_p
    const int last = sample_count((tid < n && cum_before <= top_p && cprob[tid] > top_p) ? tid + 1 : 0, ired);
    const int end = last > 0 ? last - 1 : n - 1;
    const float r = u * cprob[end];
    const int pick = sample_count((tid <= end && cum_before <= r && cprob[tid] > r) ? tid + 1 : 0, ired);
    const int j = pick > 0 ? pick - 1 : end;
    token = (int)(0xFFFFFFFFu - (uint32_t)(cand[j] & 0xFFFFFFFFull));
  }
  if (tid == 0) {
    tokens[b] = token;
    if (step >= 0 && step < cap) generated[(size_t)b * cap + step] = token;
  }
}

// First maximum of each row of this shard's logits [batch][cols]: (value,
// global index first + idx) as a float2 whose second lane holds the index
// bits (NaN never wins; an all-NaN row gives (-inf, first)).
__global__ void __launch_bounds__(kRowThreads)
shard_top1_kernel(const float *logits, int cols, int first, float2 *top, ExchangePut xp, size_t top_off) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const float *row = logits + (size_t)b * cols;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < cols; i += kRowThreads) {
    const float v = row[i];
    if (v > best) best = v, idx = i;
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, best, off);
    const int oi = __shfl_down_sync(0xffffffffu, idx, off);
    if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sv[w] = best, si[w] = idx;
  __syncthreads();
  if (w == 0) {
    best = lane < kRowThreads / 32 ? sv[lane] : -INFINITY;
    idx = lane < kRowThreads / 32 ? si[lane] : 0x7fffffff;
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, best, off);
      const int oi = __shfl_down_sync(0xffffffffu, idx, off);
      if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
    }
    if (lane == 0) {
      const float2 t = make_float2(best, __int_as_float(first + (idx == 0x7fffffff ? 0 : idx)));
      if (xp.blocks == nullptr) {
        top[b] = t;
      } else {  // into every rank's candidate exchange
        for (int q = 0; q < xp.world; ++q) *reinterpret_cast<float2 *>(xp.blocks[q] + top_off + (size_t)b * 8) = t;
      }
    }
  }
  if (xp.blocks != nullptr) exchange_signal(xp);
}

// The global greedy token of each row from the shards' candidates
// top[shards][batch]: largest value, lowest index on ties (the first maximum
// over the whole vocabulary).
__global__ void pick_top_kernel(const float2 *top, int shards, int batch, int *tokens, int *generated,
                                int cap, const int *step_ptr, ExchangeWait xw) {
  pdl_launch_dependents();
  pdl_wait();
  if (xw.flags != nullptr) {  // candidates from the peers' exchange puts
    if (threadIdx.x < 32) exchange_wait_warp(xw, &g_llama_status, 923u);
    __syncthreads();
  }
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int s = 0; s < shards; ++s) {
    const float2 t = top[(size_t)s * batch + b];
    const int ti = __float_as_int(t.y);
    if (t.x > best || (t.x == best && ti < idx)) best = t.x, idx = ti;
  }
  if (idx == 0x7fffffff) idx = 0;
  tokens[b] = idx;
  const int step = *step_ptr;
  if (step >= 0 && step < cap) generated[(size_t)b * cap + step] = idx;
}

// --- peer-memory exchange of the row-sharded step ---------------------------
// Each rank's exchange block (CUDA IPC shared) holds, per exchange kind (0
// attention output, 1 delta, 2 SwiGLU product, 3 classifier candidates), the
// slots [rank][batch][cols] and a flag per sending rank. A put copies this
// rank's slot into every peer's block, and the last of its CTAs to finish
// (an arrival counter it resets) fences at system scope and stores the
// exchange's epoch into each peer's flag for this rank; a wait spins (bounded)
// until every peer's flag for the kind has reached the epoch. Epoch =
// generation << 32 | (step * per_step + index + 1), from the device step
// counter, so one captured step graph serves every token; a buffer is
// reused two exchanges later at the earliest, by when every rank has
// consumed it (producing exchange k needs every rank's exchange k - 1, which
// each rank produced after consuming k - 2).
// Copies rows x row_bytes (16-byte multiple) at byte offset off, row stride
// `stride`, of this rank's exchange block into every peer's block, then
// signals the peers (the attention output, which many CTAs write).
__global__ void __launch_bounds__(256)
exchange_put_kernel(ExchangePut xp, size_t off, int rows, size_t row_bytes, size_t stride) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t per_row = row_bytes / 16, n16 = (size_t)rows * per_row;
  const size_t step = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += step) {
    const size_t at = off + (i / per_row) * stride + (i % per_row) * 16;
    const uint4 v = *reinterpret_cast<const uint4 *>(xp.blocks[xp.rank] + at);
    for (int q = 0; q < xp.world; ++q)
      if (q != xp.rank) *reinterpret_cast<uint4 *>(xp.blocks[q] + at) = v;
  }
  exchange_signal(xp);
}

// A consumer-side wait as its own launch (before a bf16 GEMM, which reads
// its operand with TMA and has no wait of its own).
__global__ void exchange_wait_kernel(ExchangeWait xw, unsigned where) {
  pdl_launch_dependents();
  pdl_wait();
  exchange_wait_warp(xw, &g_llama_status, where);
}

template <typename F>
int launch_rows(int nv, F &&f) {
  switch (nv) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 8: f(std::integral_constant<int, 8>{}); break;
    default: return set_error(CE_ERR_USAGE, "dim too large for the row kernels");
  }
  return CE_OK;
}

int pow2_at_least(int v);

// Launches residual_rmsnorm_kernel with one block per row: 1024 threads for
// rows of 4096 values or more, else 256; NV float4 per thread.
template <typename... Args>
int launch_norm(int dim, dim3 grid, cudaStream_t s, bool pdl, Args... args) {
  const int cols4 = dim / 4, threads = cols4 >= 1024 ? 1024 : 256;
  const int nv = pow2_at_least((cols4 + threads - 1) / threads);
  int lrc = CE_OK;
  const int rc = launch_rows(nv, [&](auto nvt) {
    constexpr int NV = decltype(nvt)::value;
    lrc = threads == 1024
              ? launch_kernel(residual_rmsnorm_kernel<NV, 1024>, grid, dim3(1024), 0, s, pdl,
                              "residual_rmsnorm_kernel", args...)
              : launch_kernel(residual_rmsnorm_kernel<NV, 256>, grid, dim3(256), 0, s, pdl,
                              "residual_rmsnorm_kernel", args...);
  });
  return rc ? rc : lrc;
}

// Grid of rope_append_kernel: blocks of 256 (sequence, pair) threads over the
// dim / 2 q pairs and kv_dim / 2 k/v pairs of each of the batch rows.
dim3 rope_grid(int dim, int kv_dim, int batch) {
  return dim3((unsigned)((dim / 2 + kv_dim / 2 + 255) / 256), (unsigned)batch);
}

// Dynamic shared memory of one attention CTA: its ring of K and V chunks and
// the chunk's weights.
constexpr size_t attn_smem_bytes(int hs) {
  return (size_t)attn_stages(hs) * 2 * kAttnChunk * hs * 2 + kAttnChunk * 4;
}

// Opts the attention kernels into their dynamic shared memory, once per device.
int configure_attention() {
  static bool done[64] = {};
  int dev = 0;
  CE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && done[dev]) return CE_OK;
  CE_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_bytes(64)));
  CE_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_bytes(128)));
  CE_CUDA_TRY(cudaFuncSetAttribute(attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)pf_smem_bytes(64)));
  CE_CUDA_TRY(cudaFuncSetAttribute(attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)pf_smem_bytes(128)));
  CE_CUDA_TRY(cudaFuncSetAttribute(attn_prefill_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   FaLayout<64>::total));
  CE_CUDA_TRY(cudaFuncSetAttribute(attn_prefill_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   FaLayout<128>::total));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return CE_OK;
}

// Splits of each (sequence, head)'s positions among attention CTAs: the
// count whose CTAs fill the resident slots' last wave best (every CTA costs
// the same, the positions being common to all sequences), each split keeping
// at least 8 chunks of the full cache; a little is charged per split for the
// merge.
int attn_choose_splits(int hs, long long pairs, int seq_len) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &per_sm, hs == 64 ? attn_decode_kernel<64> : attn_decode_kernel<128>, 32, attn_smem_bytes(hs)) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const double slots = (double)per_sm * sm_count();
  const int max_splits = std::max(1, std::min(16, (seq_len + kAttnChunk - 1) / kAttnChunk / 8));
  int best = 1;
  double best_score = -1.0;
  for (int sp = 1; sp <= max_splits; ++sp) {
    const double x = (double)pairs * sp / slots;
    const double score = x / std::ceil(x) - 0.01 * (sp - 1);
    if (score > best_score + 1e-9) best = sp, best_score = score;
  }
  return best;
}

int pow2_at_least(int v) {
  int p = 1;
  while (p < v) p *= 2;
  return p;
}

}  // namespace
}  // namespace ce

using namespace ce;

// One NVFP4 weight matrix in the decode-form W4A16 GEMM's layout (w4t_pack:
// per 128-wide k block and 128-row group, 8 KB of codes then 1 KB of scales).
struct QMat {
  uint8_t *packed;
  size_t bytes;
  float *alpha;     // (encode, decode) tensor scales; the GEMM uses alpha[1]
  int rows, cols;
};

struct ce_llama {
  ce_llama_config c{};
  int B = 0, cap = 0, precision = 0;
  // shard: rank of world; local heads, KV heads, attention width (heads x hs),
  // hidden slice and vocabulary slice (all global when world == 1)
  int rank = 0, world = 1, lH = 0, lKH = 0, lD = 0, lHd = 0, lV = 0;
  // exchange buffers of the sharded segments (caller-owned device memory):
  // [world][batch][lD] 16-bit, [world][batch][lD] fp32, [world][batch][lHd]
  // 16-bit, [world][batch] float2
  uint16_t *x_att = nullptr, *x_hb = nullptr;
  float *x_delta = nullptr;
  float2 *x_top = nullptr;
  // peer-memory exchange (ce_llama_exchange_open / _connect): this rank's
  // block [att | delta | hb | top | flags], shared with the peers by CUDA IPC;
  // x_att .. x_top then point into it
  uint8_t *x_block = nullptr;
  size_t x_off[5] = {};                   // byte offsets: att, delta, hb, top, flags
  size_t x_block_bytes = 0;
  std::vector<uint8_t *> peer_block;      // every rank's block as mapped here (own = x_block)
  uint8_t **d_blocks = nullptr;           // device copy of peer_block
  int *x_counter = nullptr;               // last-CTA counter of the put kernel
  unsigned *x_gen = nullptr;              // run generation (advanced by ce_llama_start)
  unsigned host_gen = 0;
  bool p2p = false;
  // token choice: greedy (temperature 0) or sampled (ce_llama_set_sampling)
  float temperature = 0.f, top_p = 0.f;
  uint64_t seed = 0;
  int hs = 0, kv_dim = 0, qkv_rows = 0, nv = 0;
  int sp_qkv = 1, sp_o = 1, sp_13 = 1, sp_2 = 1;  // split-K counts of the layer GEMMs
  bool pdl = true;  // programmatic dependent launch between the step's kernels
  int attn_splits = 1;  // CTAs per (sequence, head) in the attention
  size_t layer_kv = 0;  // cache elements of one layer (batch x kv_heads x seq_len x hs)
  // weights
  uint16_t *tok_emb = nullptr, *wqkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr,
           *wcls = nullptr;
  float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr;
  float2 *rope = nullptr;
  // cache and activations
  uint16_t *kcache = nullptr, *vcache = nullptr, *xb = nullptr, *att = nullptr, *hb = nullptr;
  float *x = nullptr, *delta = nullptr, *qkv = nullptr, *h = nullptr, *logits = nullptr,
        *part = nullptr;
  int *tokens = nullptr, *generated = nullptr, *pos = nullptr, *step = nullptr;
  int *arrivals = nullptr;  // per (sequence, head) chunk arrivals of the attention merge
  // NVFP4 weights (precision CE_PREC_NVFP4_E2M1): matrix 4 l + k of layer l
  // is k = 0 wqkv, 1 wo, 2 w13, 3 w2; matrix 4 n_layers is the classifier
  uint8_t *q_codes = nullptr, *q_scales = nullptr;
  float *q_alpha = nullptr;
  std::vector<QMat> qm;
  // prefill workspace (ce_llama_prefill_reserve): pf_rows chunk rows
  int pf_rows = 0;
  bool pf_simt = false;           // prefill attention on the SIMT kernel instead of the tensor cores
  CUtensorMap pf_tmk{}, pf_tmv{};  // K / V cache rows for the tensor-core prefill attention
  float *pf_x = nullptr, *pf_qkv = nullptr, *pf_delta = nullptr;
  uint16_t *pf_xb = nullptr, *pf_att = nullptr, *pf_hb = nullptr;
  uint16_t *pf_w16 = nullptr;  // NVFP4 model: one layer's weights expanded to fp16 (wqkv | wo | w13 | w2)
  int *pf_tokens = nullptr;
};

namespace {

void free_prefill(ce_llama *m) {
  for (void *p : {(void *)m->pf_x, (void *)m->pf_qkv, (void *)m->pf_delta, (void *)m->pf_xb, (void *)m->pf_att,
                  (void *)m->pf_hb, (void *)m->pf_tokens, (void *)m->pf_w16})
    if (p) cudaFree(p);
  m->pf_x = m->pf_qkv = m->pf_delta = nullptr;
  m->pf_xb = m->pf_att = m->pf_hb = m->pf_w16 = nullptr;
  m->pf_tokens = nullptr;
  m->pf_rows = 0;
}

void free_llama(ce_llama *m) {
  free_prefill(m);
  for (size_t q = 0; q < m->peer_block.size(); ++q)
    if (m->peer_block[q] != nullptr && (int)q != m->rank) cudaIpcCloseMemHandle(m->peer_block[q]);
  for (void *p : {(void *)m->x_block, (void *)m->d_blocks, (void *)m->x_counter, (void *)m->x_gen})
    if (p) cudaFree(p);
  for (void *p : {(void *)m->tok_emb, (void *)m->wqkv, (void *)m->wo, (void *)m->w13, (void *)m->w2,
                  (void *)m->wcls, (void *)m->rms_att, (void *)m->rms_ffn, (void *)m->rms_final,
                  (void *)m->rope, (void *)m->kcache, (void *)m->vcache, (void *)m->xb, (void *)m->att,
                  (void *)m->hb, (void *)m->x, (void *)m->delta, (void *)m->qkv, (void *)m->h,
                  (void *)m->logits, (void *)m->part, (void *)m->tokens, (void *)m->generated,
                  (void *)m->pos, (void *)m->step, (void *)m->arrivals, (void *)m->q_codes,
                  (void *)m->q_scales, (void *)m->q_alpha})
    if (p) cudaFree(p);
  delete m;
}

size_t wqkv_elems(const ce_llama *m) { return (size_t)m->qkv_rows * m->c.dim; }
size_t wo_elems(const ce_llama *m) { return (size_t)m->lD * m->c.dim; }
size_t w13_elems(const ce_llama *m) { return (size_t)2 * m->lHd * m->c.dim; }
size_t w2_elems(const ce_llama *m) { return (size_t)m->lD * m->c.hidden_dim; }

// (rows, cols) of this shard's weight kind k: 0 wqkv, 1 wo, 2 w13, 3 w2,
// 4 classifier.
void mat_shape(const ce_llama *m, int k, int *rows, int *cols) {
  const ce_llama_config &c = m->c;
  const int r[5] = {m->qkv_rows, m->lD, 2 * m->lHd, m->lD, m->lV};
  const int q[5] = {c.dim, c.dim, c.dim, c.hidden_dim, c.dim};
  *rows = r[k];
  *cols = q[k];
}

// Global row of each of this shard's rows of weight kind k (see mat_shape),
// for a model of config c split over world ranks.
void shard_rows(const ce_llama_config &c, int rank, int world, int k, std::vector<int> *rows) {
  const int hs = c.dim / c.n_heads, kvd = hs * c.n_kv_heads;
  const int lD = c.dim / world, lKV = kvd / world, lHd = c.hidden_dim / world, lV = c.vocab_size / world;
  rows->clear();
  auto add = [&](int g0, int n) {
    for (int i = 0; i < n; ++i) rows->push_back(g0 + i);
  };
  switch (k) {
    case 0:  // q rows of this rank's heads, then its k and v rows
      add(rank * lD, lD);
      add(c.dim + rank * lKV, lKV);
      add(c.dim + kvd + rank * lKV, lKV);
      break;
    case 1: add(rank * lD, lD); break;
    case 2: add(rank * 2 * lHd, 2 * lHd); break;  // interleaved (w1, w3) pairs
    case 3: add(rank * lD, lD); break;
    default: add(rank * lV, lV); break;
  }
}

int global_rows(const ce_llama_config &c, int k) {
  const int kvd = c.dim / c.n_heads * c.n_kv_heads;
  const int r[5] = {c.dim + 2 * kvd, c.dim, 2 * c.hidden_dim, c.dim, c.vocab_size};
  return r[k];
}

struct TensorView {
  void *ptr;
  size_t bytes;
};

// Device tensor `which` of layer `layer` (layer ignored for global tensors).
int tensor_of(ce_llama *m, int which, int layer, TensorView *v) {
  const ce_llama_config &c = m->c;
  const bool per_layer = which == CE_LLAMA_WQKV || which == CE_LLAMA_WO || which == CE_LLAMA_W13 ||
                         which == CE_LLAMA_W2 || which == CE_LLAMA_RMS_ATT || which == CE_LLAMA_RMS_FFN ||
                         which == CE_LLAMA_KCACHE || which == CE_LLAMA_VCACHE;
  CE_REQUIRE(!per_layer || (layer >= 0 && layer < c.n_layers), "layer %d out of range", layer);
  const bool bf16_weight = which == CE_LLAMA_WQKV || which == CE_LLAMA_WO || which == CE_LLAMA_W13 ||
                           which == CE_LLAMA_W2 || which == CE_LLAMA_WCLS;
  CE_REQUIRE(!bf16_weight || m->precision == CE_PREC_BF16,
             "tensor %d is not stored in this precision (see ce_llama_read_nvfp4)", which);
  const size_t L = (size_t)layer;
  switch (which) {
    case CE_LLAMA_TOK_EMB: *v = {m->tok_emb, (size_t)c.vocab_size * c.dim * 2}; break;
    case CE_LLAMA_WQKV: *v = {m->wqkv + L * wqkv_elems(m), wqkv_elems(m) * 2}; break;
    case CE_LLAMA_WO: *v = {m->wo + L * wo_elems(m), wo_elems(m) * 2}; break;
    case CE_LLAMA_W13: *v = {m->w13 + L * w13_elems(m), w13_elems(m) * 2}; break;
    case CE_LLAMA_W2: *v = {m->w2 + L * w2_elems(m), w2_elems(m) * 2}; break;
    case CE_LLAMA_RMS_ATT: *v = {m->rms_att + L * c.dim, (size_t)c.dim * 4}; break;
    case CE_LLAMA_RMS_FFN: *v = {m->rms_ffn + L * c.dim, (size_t)c.dim * 4}; break;
    case CE_LLAMA_RMS_FINAL: *v = {m->rms_final, (size_t)c.dim * 4}; break;
    case CE_LLAMA_WCLS: *v = {m->wcls, (size_t)m->lV * c.dim * 2}; break;
    case CE_LLAMA_KCACHE: *v = {m->kcache + L * m->layer_kv, m->layer_kv * 2}; break;
    case CE_LLAMA_VCACHE: *v = {m->vcache + L * m->layer_kv, m->layer_kv * 2}; break;
    case CE_LLAMA_LOGITS: *v = {m->logits, (size_t)m->B * m->lV * 4}; break;
    case CE_LLAMA_TOKENS: *v = {m->tokens, (size_t)m->B * 4}; break;
    case CE_LLAMA_GENERATED: *v = {m->generated, (size_t)m->B * m->cap * 4}; break;
    case CE_LLAMA_POS: *v = {m->pos, 4}; break;
    case CE_LLAMA_RESIDUAL: *v = {m->x, (size_t)m->B * c.dim * 4}; break;
    default: return set_error(CE_ERR_USAGE, format("unknown llama tensor %d", which));
  }
  return CE_OK;
}

}  // namespace

extern "C" {

// Device memory of one rank's share of the model (its heads' KV cache, its
// rows of every GEMM weight; the bf16 embedding on every rank) against the
// 180 GB of a B200, with room for activations.
int llama_memory_check(const ce_llama_config *c, int batch, int precision, int world) {
  const int hs = c->dim / c->n_heads;
  const double kv = 2.0 * c->n_layers * (double)batch * hs * c->n_kv_heads * c->seq_len * 2 / world;
  const double per_value = precision == CE_PREC_NVFP4_E2M1 ? 0.5625 : 2.0;
  const double w = per_value * ((double)c->n_layers * ((double)(c->dim + 2 * hs * c->n_kv_heads) * c->dim +
                                                       (double)c->dim * c->dim + 3.0 * c->hidden_dim * c->dim) +
                                (double)c->vocab_size * c->dim) / world +
                   2.0 * (double)c->vocab_size * c->dim;
  CE_REQUIRE(kv + w <= 170.0 * (1LL << 30),
             "model and KV cache need %.1f GiB of device memory per GPU (limit 170 GiB)", (kv + w) / (1LL << 30));
  return CE_OK;
}

int llama_shape_check(const ce_llama_config *c, int batch, int max_steps, int precision) {
  CE_REQUIRE(c != nullptr, "null config");
  CE_REQUIRE(c->dim >= 8 && c->dim % 8 == 0 && c->dim <= 8192, "dim must be a multiple of 8 in [8, 8192] (got %d)", c->dim);
  CE_REQUIRE(c->hidden_dim >= 8 && c->hidden_dim % 8 == 0, "hidden_dim must be a positive multiple of 8 (got %d)", c->hidden_dim);
  CE_REQUIRE(c->n_layers >= 1 && c->n_layers <= 1024, "n_layers must be in [1, 1024] (got %d)", c->n_layers);
  CE_REQUIRE(c->n_heads >= 1 && c->dim % c->n_heads == 0, "n_heads must divide dim (dim %d, n_heads %d)", c->dim, c->n_heads);
  CE_REQUIRE(c->n_kv_heads >= 1 && c->n_heads % c->n_kv_heads == 0, "n_kv_heads must divide n_heads (got %d, %d)", c->n_kv_heads, c->n_heads);
  const int hs = c->dim / c->n_heads;
  CE_REQUIRE(hs == 64 || hs == 128, "head size dim / n_heads must be 64 or 128 (got %d)", hs);
  CE_REQUIRE(c->vocab_size >= 2, "vocab_size must be >= 2 (got %d)", c->vocab_size);
  CE_REQUIRE(c->vocab_size % 4 == 0, "vocab_size must be a multiple of 4 (got %d)", c->vocab_size);
  CE_REQUIRE(c->seq_len >= 1 && c->seq_len <= (1 << 20), "seq_len must be in [1, 2^20] (got %d)", c->seq_len);
  CE_REQUIRE(batch >= 1 && batch <= 65535, "batch must be in [1, 65535] (got %d)", batch);
  CE_REQUIRE(max_steps >= 1, "max_steps must be >= 1 (got %d)", max_steps);
  CE_REQUIRE(precision == CE_PREC_BF16 || precision == CE_PREC_NVFP4_E2M1,
             "llama weight precision %d is not available (bf16 or NVFP4)", precision);
  CE_REQUIRE(precision != CE_PREC_NVFP4_E2M1 || (c->dim % 64 == 0 && c->hidden_dim % 64 == 0),
             "NVFP4 weights need dim and hidden_dim multiples of 64 (got %d, %d)", c->dim, c->hidden_dim);
  return CE_OK;
}

int ce_llama_validate(const ce_llama_config *c, int batch, int max_steps, int precision) {
  if (int rc = llama_shape_check(c, batch, max_steps, precision)) return rc;
  return llama_memory_check(c, batch, precision, 1);
}

int ce_llama_validate_shard(const ce_llama_config *c, int batch, int max_steps, int precision, int rank,
                            int world) {
  if (int rc = llama_shape_check(c, batch, max_steps, precision)) return rc;
  CE_REQUIRE(world >= 1 && rank >= 0 && rank < world, "rank %d of world %d", rank, world);
  if (world == 1) return llama_memory_check(c, batch, precision, 1);
  CE_REQUIRE(c->n_heads % world == 0 && c->n_kv_heads % world == 0,
             "the heads (%d query, %d key/value) must split evenly over %d ranks", c->n_heads, c->n_kv_heads, world);
  CE_REQUIRE(c->hidden_dim % (8 * world) == 0, "hidden_dim / world must be a multiple of 8 (hidden %d, world %d)",
             c->hidden_dim, world);
  CE_REQUIRE(c->vocab_size % (4 * world) == 0, "vocab_size / world must be a multiple of 4 (vocab %d, world %d)",
             c->vocab_size, world);
  CE_REQUIRE((c->dim / world) % 8 == 0, "dim / world must be a multiple of 8 (dim %d, world %d)", c->dim, world);
  return llama_memory_check(c, batch, precision, world);
}

int ce_llama_create_shard_ex(ce_llama **out, const ce_llama_config *cfg, int batch, int max_steps,
                             int precision, int rank, int world, int flags, ce_stream_t stream) {
  CE_REQUIRE(out != nullptr, "null model pointer");
  CE_REQUIRE((flags & ~CE_LLAMA_REPRODUCIBLE_SPLITS) == 0, "unknown shard flags 0x%x", flags);
  *out = nullptr;
  if (int rc = ce_llama_validate_shard(cfg, batch, max_steps, precision, rank, world)) return rc;
  if (int rc = configure_attention()) return rc;
  ce_llama *m = new ce_llama();
  m->c = *cfg;
  m->B = batch;
  m->cap = max_steps;
  m->precision = precision;
  m->rank = rank;
  m->world = world;
  m->hs = cfg->dim / cfg->n_heads;
  m->lH = cfg->n_heads / world;
  m->lKH = cfg->n_kv_heads / world;
  m->lD = m->lH * m->hs;
  m->lHd = cfg->hidden_dim / world;
  m->lV = cfg->vocab_size / world;
  m->kv_dim = m->hs * m->lKH;  // this shard's k (and v) rows
  m->qkv_rows = m->lD + 2 * m->kv_dim;
  m->nv = pow2_at_least((cfg->dim / 4 + kRowThreads - 1) / kRowThreads);
  // CE_LLAMA_REPRODUCIBLE_SPLITS: the attention and split-K GEMM splits of
  // the unsharded model, so every value this rank computes is summed in the
  // unsharded model's order (the same bits, at the cost of fewer CTAs)
  const bool repro = (flags & CE_LLAMA_REPRODUCIBLE_SPLITS) != 0;
  m->attn_splits = attn_choose_splits(m->hs, (long long)batch * (repro ? cfg->n_heads : m->lH), cfg->seq_len);
  m->layer_kv = (size_t)batch * m->lKH * cfg->seq_len * m->hs;
  // split-K for the GEMMs whose tiles alone leave SMs idle at decode sizes;
  // at least 4 k-blocks (256 of K) per split
  auto splits = [&](int N, int K) {
    return precision == CE_PREC_NVFP4_E2M1 ? gemm_w4t_auto_splits(batch, N, K, 8)
                                           : gemm_bf16_auto_splits(batch, N, K, 8, 4);
  };
  m->sp_qkv = splits(repro ? cfg->dim + 2 * m->hs * cfg->n_kv_heads : m->qkv_rows, cfg->dim);
  m->sp_o = splits(repro ? cfg->dim : m->lD, cfg->dim);
  m->sp_13 = splits(repro ? 2 * cfg->hidden_dim : 2 * m->lHd, cfg->dim);
  m->sp_2 = splits(repro ? cfg->dim : m->lD, cfg->hidden_dim);
  const int sp_delta = m->sp_o > m->sp_2 ? m->sp_o : m->sp_2;
  const ce_llama_config &c = *cfg;
  const size_t L = c.n_layers;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaSuccess;
#define CE_ALLOC(ptr, bytes)                           \
  do {                                                 \
    e = cudaMalloc(&(ptr), (bytes));                   \
    if (e != cudaSuccess) {                            \
      free_llama(m);                                   \
      return cuda_error(e, "cudaMalloc(" #ptr ")");    \
    }                                                  \
  } while (0)
  CE_ALLOC(m->tok_emb, (size_t)c.vocab_size * c.dim * 2);
  if (precision == CE_PREC_NVFP4_E2M1) {
    size_t codes = 0;  // bytes of every packed weight
    const int nmat = 4 * c.n_layers + 1;
    for (int i = 0; i < nmat; ++i) {
      int r, q;
      mat_shape(m, i == 4 * c.n_layers ? 4 : i % 4, &r, &q);
      codes += w4t_packed_bytes(r, q);
    }
    CE_ALLOC(m->q_codes, codes);
    CE_ALLOC(m->q_alpha, (size_t)nmat * 2 * 4);
    codes = 0;
    for (int i = 0; i < nmat; ++i) {
      QMat q{};
      mat_shape(m, i == 4 * c.n_layers ? 4 : i % 4, &q.rows, &q.cols);
      q.bytes = w4t_packed_bytes(q.rows, q.cols);
      q.packed = m->q_codes + codes;
      q.alpha = m->q_alpha + 2 * i;
      codes += q.bytes;
      m->qm.push_back(q);
    }
  } else {
    CE_ALLOC(m->wqkv, L * wqkv_elems(m) * 2);
    CE_ALLOC(m->wo, L * wo_elems(m) * 2);
    CE_ALLOC(m->w13, L * w13_elems(m) * 2);
    CE_ALLOC(m->w2, L * w2_elems(m) * 2);
    CE_ALLOC(m->wcls, (size_t)m->lV * c.dim * 2);
  }
  CE_ALLOC(m->rms_att, L * c.dim * 4);
  CE_ALLOC(m->rms_ffn, L * c.dim * 4);
  CE_ALLOC(m->rms_final, (size_t)c.dim * 4);
  CE_ALLOC(m->rope, (size_t)c.seq_len * (m->hs / 2) * sizeof(float2));
  CE_ALLOC(m->kcache, L * m->layer_kv * 2);
  CE_ALLOC(m->vcache, L * m->layer_kv * 2);
  CE_ALLOC(m->xb, (size_t)batch * c.dim * 2);
  CE_ALLOC(m->att, (size_t)batch * c.dim * 2);
  CE_ALLOC(m->hb, (size_t)batch * c.hidden_dim * 2);
  CE_ALLOC(m->x, (size_t)batch * c.dim * 4);
  CE_ALLOC(m->delta, (size_t)sp_delta * batch * c.dim * 4);
  CE_ALLOC(m->qkv, (size_t)m->sp_qkv * batch * m->qkv_rows * 4);
  CE_ALLOC(m->h, (size_t)m->sp_13 * batch * 2 * m->lHd * 4);
  CE_ALLOC(m->logits, (size_t)batch * m->lV * 4);
  CE_ALLOC(m->part, (size_t)batch * m->lH * m->attn_splits * (m->hs + 2) * 4);
  CE_ALLOC(m->tokens, (size_t)batch * 4);
  CE_ALLOC(m->generated, (size_t)batch * max_steps * 4);
  CE_ALLOC(m->pos, 4);
  CE_ALLOC(m->step, 4);
  CE_ALLOC(m->arrivals, (size_t)batch * m->lH * 4);
#undef CE_ALLOC
  // RoPE table: (cos, sin) of pos * 10000^(-2i/hs), computed in double once
  std::vector<float2> table((size_t)c.seq_len * (m->hs / 2));
  for (int p = 0; p < c.seq_len; ++p)
    for (int i = 0; i < m->hs / 2; ++i) {
      const double freq = std::pow(10000.0, -(2.0 * i) / (double)m->hs);
      const double a = (double)p * freq;
      table[(size_t)p * (m->hs / 2) + i] = make_float2((float)std::cos(a), (float)std::sin(a));
    }
  e = cudaMemcpyAsync(m->rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->pos, 0, 4, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->step, 0, 4, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->arrivals, 0, (size_t)batch * m->lH * 4, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->generated, 0xFF, (size_t)batch * max_steps * 4, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the host table goes out of scope
  if (e != cudaSuccess) {
    free_llama(m);
    return cuda_error(e, "llama set-up");
  }
  *out = m;
  return CE_OK;
}

int ce_llama_create_shard(ce_llama **out, const ce_llama_config *cfg, int batch, int max_steps,
                          int precision, int rank, int world, ce_stream_t stream) {
  return ce_llama_create_shard_ex(out, cfg, batch, max_steps, precision, rank, world, 0, stream);
}

int ce_llama_create(ce_llama **out, const ce_llama_config *cfg, int batch, int max_steps,
                    int precision, ce_stream_t stream) {
  return ce_llama_create_shard_ex(out, cfg, batch, max_steps, precision, 0, 1, 0, stream);
}

int ce_llama_destroy(ce_llama *m) {
  if (m) free_llama(m);
  return CE_OK;
}

int ce_llama_init_random(ce_llama *m, uint64_t seed, float weight_std, int kv_fill, ce_stream_t stream) {
  CE_REQUIRE(m != nullptr, "null model");
  CE_REQUIRE(kv_fill >= 0 && kv_fill <= m->c.seq_len, "kv_fill must be in [0, seq_len] (got %d)", kv_fill);
  cudaStream_t s = (cudaStream_t)stream;
  const ce_llama_config &c = m->c;
  const size_t L = c.n_layers;
  const int grid = 4 * sm_count(), threads = 256;
  // Streams of the random model: 1 embedding, 2 wqkv, 3 wo, 4 w13, 5 w2,
  // 6 classifier (bf16 weights; values indexed by the global element, so a
  // shard generates exactly its rows), 1000 + i NVFP4 matrix i, 100 / 101
  // the K / V cache.
  init_normal_bf16_kernel<<<grid, threads, 0, s>>>(m->tok_emb, (size_t)c.vocab_size * c.dim, seed, 1, weight_std,
                                                   (size_t)c.vocab_size * c.dim, (size_t)c.vocab_size * c.dim);
  CE_LAUNCH_CHECK("init_normal_bf16_kernel");
  // row maps of this shard, kinds 0..4
  std::vector<int> rows[5];
  size_t most = 1;
  for (int k = 0; k < 5; ++k) {
    shard_rows(c, m->rank, m->world, k, &rows[k]);
    most = std::max(most, rows[k].size());
  }
  int *d_map = nullptr;
  CE_CUDA_TRY(cudaMalloc(&d_map, 5 * most * sizeof(int)));
  int rc = CE_OK;
  for (int k = 0; k < 5 && rc == CE_OK; ++k) {
    const cudaError_t e = cudaMemcpy(d_map + k * most, rows[k].data(), rows[k].size() * sizeof(int),
                                     cudaMemcpyHostToDevice);
    if (e != cudaSuccess) rc = cuda_error(e, "cudaMemcpy(row map)");
  }
  if (rc == CE_OK && m->precision == CE_PREC_BF16) {
    uint16_t *w[5] = {m->wqkv, m->wo, m->w13, m->w2, m->wcls};
    for (int k = 0; k < 5 && rc == CE_OK; ++k) {
      int r, q;
      mat_shape(m, k, &r, &q);
      init_rows_bf16_kernel<<<grid, threads, 0, s>>>(w[k], k == 4 ? 1 : c.n_layers, r, q, global_rows(c, k),
                                                     d_map + k * most, seed, 2 + k, weight_std);
      const cudaError_t e = cudaPeekAtLastError();
      if (e != cudaSuccess) rc = cuda_error(e, "init_rows_bf16_kernel");
    }
  }
  if (rc == CE_OK && m->precision == CE_PREC_NVFP4_E2M1) {
    // every matrix: the global matrix in fp32 N(0, std), the NVFP4 quantizer
    // over all of it (tensor amax, UE4M3 per 16 values, E2M1 codes), then
    // this shard's rows in the W4A16 GEMM's layout
    size_t biggest = 0;
    for (int k = 0; k < 5; ++k) {
      int r, q;
      mat_shape(m, k, &r, &q);
      biggest = std::max(biggest, (size_t)global_rows(c, k) * q);
    }
    float *tmp = nullptr;
    uint8_t *tcodes = nullptr, *tscales = nullptr;
    unsigned int *amax = nullptr;
    cudaError_t e = cudaMalloc(&tmp, biggest * 4);
    if (e == cudaSuccess) e = cudaMalloc(&tcodes, biggest / 2);
    if (e == cudaSuccess) e = cudaMalloc(&tscales, biggest / 16);
    if (e == cudaSuccess) e = cudaMalloc(&amax, 4);
    rc = e == cudaSuccess ? CE_OK : cuda_error(e, "cudaMalloc(quantization scratch)");
    for (size_t i = 0; i < m->qm.size() && rc == CE_OK; ++i) {
      const QMat &q = m->qm[i];
      const int k = i == m->qm.size() - 1 ? 4 : (int)(i % 4);
      const int grows = global_rows(c, k);
      init_normal_f32_kernel<<<grid, threads, 0, s>>>(tmp, (size_t)grows * q.cols, seed, 1000 + i, weight_std);
      e = cudaPeekAtLastError();
      if (e != cudaSuccess) rc = cuda_error(e, "init_normal_f32_kernel");
      if (rc == CE_OK) rc = quantize_nvfp4(tcodes, tscales, q.alpha, amax, tmp, grows, q.cols, q.cols / 2, s);
      if (rc == CE_OK)
        rc = w4t_pack(q.packed, tcodes, tscales, q.rows, q.cols, q.cols / 2, q.cols / 16, s,
                      d_map + k * most);
    }
    e = cudaStreamSynchronize(s);
    if (rc == CE_OK && e != cudaSuccess) rc = cuda_error(e, "NVFP4 weight set-up");
    for (void *p : {(void *)tmp, (void *)tcodes, (void *)tscales, (void *)amax})
      if (p) cudaFree(p);
  }
  const cudaError_t se = cudaStreamSynchronize(s);
  if (rc == CE_OK && se != cudaSuccess) rc = cuda_error(se, "weight set-up");
  cudaFree(d_map);
  if (rc) return rc;
  fill_f32_kernel<<<grid, threads, 0, s>>>(m->rms_att, L * c.dim, 1.0f);
  fill_f32_kernel<<<grid, threads, 0, s>>>(m->rms_ffn, L * c.dim, 1.0f);
  fill_f32_kernel<<<grid, threads, 0, s>>>(m->rms_final, (size_t)c.dim, 1.0f);
  CE_LAUNCH_CHECK("fill_f32_kernel");
  // KV cache: positions [0, kv_fill) of every (layer, sequence, head) N(0, 1)
  CE_CUDA_TRY(cudaMemsetAsync(m->kcache, 0, L * m->layer_kv * 2, s));
  CE_CUDA_TRY(cudaMemsetAsync(m->vcache, 0, L * m->layer_kv * 2, s));
  if (kv_fill > 0) {
    const size_t runs = L * m->B * m->lKH;  // contiguous [seq_len][hs] runs of this shard's KV heads
    const size_t run = (size_t)c.seq_len * m->hs, filled = (size_t)kv_fill * m->hs;
    for (int which = 0; which < 2; ++which) {
      init_normal_bf16_kernel<<<grid, threads, 0, s>>>(which ? m->vcache : m->kcache, runs * filled, seed,
                                                       100 + which, 1.0f, run, filled, (size_t)m->lKH,
                                                       (size_t)c.n_kv_heads, (size_t)m->rank * m->lKH);
      CE_LAUNCH_CHECK("init_normal_bf16_kernel");
    }
  }
  CE_CUDA_TRY(cudaStreamSynchronize(s));
  return CE_OK;
}

int ce_llama_start(ce_llama *m, const int32_t *tokens_host, int pos, ce_stream_t stream) {
  CE_REQUIRE(m != nullptr && tokens_host != nullptr, "null argument");
  CE_REQUIRE(pos >= 0 && pos < m->c.seq_len, "pos must be in [0, seq_len) (got %d)", pos);
  cudaStream_t s = (cudaStream_t)stream;
  const int zero = 0;
  CE_CUDA_TRY(cudaMemcpyAsync(m->tokens, tokens_host, (size_t)m->B * 4, cudaMemcpyHostToDevice, s));
  CE_CUDA_TRY(cudaMemcpyAsync(m->pos, &pos, 4, cudaMemcpyHostToDevice, s));
  CE_CUDA_TRY(cudaMemcpyAsync(m->step, &zero, 4, cudaMemcpyHostToDevice, s));
  CE_CUDA_TRY(cudaMemsetAsync(m->generated, 0xFF, (size_t)m->B * m->cap * 4, s));
  if (m->x_gen != nullptr) {
    // a new run: exchange epochs carry the generation, so flags left by an
    // earlier run never satisfy this run's waits (every rank starts the same
    // number of runs)
    ++m->host_gen;
    CE_CUDA_TRY(cudaMemcpyAsync(m->x_gen, &m->host_gen, 4, cudaMemcpyHostToDevice, s));
  }
  CE_CUDA_TRY(cudaStreamSynchronize(s));
  return CE_OK;
}

int ce_llama_enqueue_step(ce_llama *m, ce_stream_t stream) {
  CE_REQUIRE(m != nullptr, "null model");
  CE_REQUIRE(m->world == 1, "a sharded model steps through ce_llama_enqueue_segment");
  cudaStream_t s = (cudaStream_t)stream;
  const ce_llama_config &c = m->c;
  const int B = m->B, D = c.dim, Hd = c.hidden_dim;
  const float eps = 1e-5f;
  const size_t delta_stride = (size_t)B * D, qkv_stride = (size_t)B * m->qkv_rows,
               h_stride = (size_t)B * 2 * Hd;
  const bool pdl = m->pdl;
  const bool w4 = m->precision == CE_PREC_NVFP4_E2M1;
  // y = a W^T of weight kind k (0 wqkv, 1 wo, 2 w13, 3 w2, 4 classifier) of
  // layer l; sw_out set: the SwiGLU epilogue writes the w2 operand (bf16, or
  // fp16 for the NVFP4 model)
  auto gemm = [&](int k, int l, float *d, const uint16_t *a, int ldd, int splits, long long stride,
                  uint16_t *sw_out) -> int {
    int N, K;
    mat_shape(m, k, &N, &K);
    if (w4) {
      const QMat &q = m->qm[k == 4 ? 4 * c.n_layers : 4 * l + k];
      return gemm_w4t(d, a, q.packed, q.alpha + 1, B, N, K, K, ldd, splits, stride, sw_out,
                      sw_out ? N / 2 : 0, s, pdl);
    }
    const uint16_t *w = k == 0 ? m->wqkv + l * wqkv_elems(m) : k == 1 ? m->wo + l * wo_elems(m)
                        : k == 2 ? m->w13 + l * w13_elems(m) : k == 3 ? m->w2 + l * w2_elems(m) : m->wcls;
    if (sw_out) return gemm_bf16_swiglu(sw_out, N / 2, a, w, B, N, K, K, K, s, pdl);
    return gemm_bf16_split(d, a, w, B, N, K, K, K, ldd, splits, stride, s, pdl);
  };
  auto norm = [&](const float *delta, int nsplit, const uint16_t *emb, const float *w) {
    return launch_norm(D, dim3(B), s, pdl, m->x, delta, nsplit, delta_stride, emb, (const int *)m->tokens,
                       c.vocab_size, w, m->xb, D, eps, (int)w4, 0, ExchangeWait{});
  };
  const size_t attn_smem = attn_smem_bytes(m->hs);
  for (int l = 0; l < c.n_layers; ++l) {
    int rc = norm(l == 0 ? nullptr : m->delta, m->sp_2, l == 0 ? m->tok_emb : nullptr,
                  m->rms_att + (size_t)l * D);
    if (rc) return rc;
    CE_LAUNCH_CHECK("residual_rmsnorm_kernel");
    rc = gemm(0, l, m->qkv, m->xb, m->qkv_rows, m->sp_qkv, (long long)qkv_stride, nullptr);
    if (rc) return rc;
    uint16_t *kc = m->kcache + l * m->layer_kv, *vc = m->vcache + l * m->layer_kv;
    rc = launch_kernel(rope_append_kernel, rope_grid(D, m->kv_dim, B), dim3(256), 0, s, pdl, "rope_append_kernel", m->qkv,
                       m->qkv_rows, m->sp_qkv, qkv_stride, kc, vc, (const float2 *)m->rope,
                       (const int *)m->pos, D, m->kv_dim, m->hs, c.n_kv_heads, c.seq_len, 1, 0);
    if (rc) return rc;
    const dim3 agrid(m->attn_splits, c.n_heads, B);
    auto attention = [&](auto hs_tag) {
      constexpr int HS = decltype(hs_tag)::value;
      return launch_kernel(attn_decode_kernel<HS>, agrid, dim3(32), attn_smem, s, pdl,
                           "attn_decode_kernel", (const float *)m->qkv, m->qkv_rows,
                           (const uint16_t *)kc, (const uint16_t *)vc, (const int *)m->pos, c.n_heads,
                           c.n_kv_heads, c.seq_len, m->attn_splits, m->part, m->arrivals,
                           m->att, D, (int)w4);
    };
    rc = m->hs == 64 ? attention(std::integral_constant<int, 64>{}) : attention(std::integral_constant<int, 128>{});
    if (rc) return rc;
    rc = gemm(1, l, m->delta, m->att, D, m->sp_o, (long long)delta_stride, nullptr);
    if (rc) return rc;
    rc = norm(m->delta, m->sp_o, nullptr, m->rms_ffn + (size_t)l * D);
    if (rc) return rc;
    CE_LAUNCH_CHECK("residual_rmsnorm_kernel");
    if (m->sp_13 == 1) {  // SwiGLU in the GEMM epilogue, straight to the bf16 operand
      rc = gemm(2, l, nullptr, m->xb, 2 * Hd, 1, 0, m->hb);
      if (rc) return rc;
    } else {
      rc = gemm(2, l, m->h, m->xb, 2 * Hd, m->sp_13, (long long)h_stride, nullptr);
      if (rc) return rc;
      rc = launch_kernel(swiglu_kernel, dim3(4 * sm_count()), dim3(256), 0, s, pdl, "swiglu_kernel",
                         (const float *)m->h, m->sp_13, h_stride, m->hb, B, Hd, (int)w4);
      if (rc) return rc;
    }
    rc = gemm(3, l, m->delta, m->hb, D, m->sp_2, (long long)delta_stride, nullptr);
    if (rc) return rc;
  }
  int rc = norm(m->delta, m->sp_2, nullptr, m->rms_final);
  if (rc) return rc;
  CE_LAUNCH_CHECK("residual_rmsnorm_kernel");
  rc = gemm(4, 0, m->logits, m->xb, c.vocab_size, 1, 0, nullptr);
  if (rc) return rc;
  rc = m->temperature > 0.f
           ? launch_kernel(sample_kernel, dim3(B), dim3(kSampleThreads), 0, s, pdl, "sample_kernel",
                           (const float *)m->logits, c.vocab_size, m->temperature, m->top_p, m->seed, m->tokens,
                           m->generated, m->cap, (const int *)m->step)
           : launch_kernel(argmax_kernel, dim3(B), dim3(kRowThreads), 0, s, pdl, "argmax_kernel",
                     (const float *)m->logits, c.vocab_size, m->tokens, m->generated, m->cap,
                     (const int *)m->step);
  if (rc) return rc;
  return launch_kernel(advance_kernel, dim3(1), dim3(1), 0, s, pdl, "advance_kernel", m->pos, m->step);
}

}  // extern "C"

namespace {

// Elements of one layer's four GEMM weights (wqkv, wo, w13, w2), and the
// offset of weight kind k among them.
size_t layer_w16_offset(const ce_llama *m, int k) {
  size_t off = 0;
  for (int i = 0; i < k; ++i) {
    int r, c;
    mat_shape(m, i, &r, &c);
    off += (size_t)r * c;
  }
  return off;
}
size_t layer_w16_elems(const ce_llama *m) { return layer_w16_offset(m, 4); }

}  // namespace

extern "C" {

int ce_llama_prefill_reserve(ce_llama *m, int max_rows) {
  CE_REQUIRE(m != nullptr, "null model");
  CE_REQUIRE(m->world == 1, "prefill runs on an unsharded model");
  CE_REQUIRE(max_rows >= m->B && max_rows <= 65535, "max_rows must be in [batch (%d), 65535] (got %d)", m->B,
             max_rows);
  const ce_llama_config &c = m->c;
  const size_t R = (size_t)max_rows;
  free_prefill(m);
  cudaError_t e = cudaSuccess;
  for (auto [ptr, bytes] : {std::pair<void **, size_t>{(void **)&m->pf_x, R * c.dim * 4},
                            {(void **)&m->pf_qkv, R * m->qkv_rows * 4},
                            {(void **)&m->pf_delta, R * c.dim * 4},
                            {(void **)&m->pf_xb, R * c.dim * 2},
                            {(void **)&m->pf_att, R * c.dim * 2},
                            {(void **)&m->pf_hb, R * c.hidden_dim * 2},
                            {(void **)&m->pf_tokens, R * 4},
                            {(void **)&m->pf_w16, m->precision == CE_PREC_NVFP4_E2M1 ? layer_w16_elems(m) * 2 : 0}}) {
    if (bytes == 0) continue;
    e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) {
      free_prefill(m);
      return cuda_error(e, "cudaMalloc(prefill workspace)");
    }
  }
  // the whole K / V cache as rows of head_size elements (one row per
  // layer, sequence, KV head and position)
  const unsigned long long cache_rows = (unsigned long long)c.n_layers * (m->layer_kv / m->hs);
  int rc = make_bf16_rows_map(&m->pf_tmk, m->kcache, m->hs, cache_rows, m->hs, kFaN);
  if (rc == CE_OK) rc = make_bf16_rows_map(&m->pf_tmv, m->vcache, m->hs, cache_rows, m->hs, kFaN);
  if (rc != CE_OK) {
    free_prefill(m);
    return rc;
  }
  m->pf_rows = max_rows;
  return CE_OK;
}

int ce_llama_set_prefill_attention(ce_llama *m, int simt) {
  CE_REQUIRE(m != nullptr, "null model");
  m->pf_simt = simt != 0;
  return CE_OK;
}

int ce_llama_enqueue_prefill(ce_llama *m, const int32_t *prompt, int prompt_len, ce_stream_t stream) {
  CE_REQUIRE(m != nullptr && prompt != nullptr, "null argument");
  CE_REQUIRE(m->world == 1, "prefill runs on an unsharded model");
  CE_REQUIRE(m->pf_rows >= m->B, "ce_llama_prefill_reserve has not been called");
  CE_REQUIRE(prompt_len >= 1 && prompt_len <= m->c.seq_len, "prompt_len must be in [1, seq_len] (got %d)",
             prompt_len);
  cudaStream_t s = (cudaStream_t)stream;
  const ce_llama_config &c = m->c;
  const int B = m->B, D = c.dim, Hd = c.hidden_dim;
  const float eps = 1e-5f;
  const bool pdl = m->pdl;
  const bool w4 = m->precision == CE_PREC_NVFP4_E2M1;
  const int per = std::min(prompt_len, m->pf_rows / B);  // positions per chunk
  // y = a W^T of weight kind k for M chunk rows, one split (M is large). The
  // NVFP4 model multiplies the layer's weights expanded to fp16 (by the
  // chunk, before its first GEMM) with the fp16 tensor-core GEMM and the
  // decode scale as alpha: at M in the thousands that beats expanding the
  // weights inside the W4T GEMM once per 256-row batch tile.
  auto gemm = [&](int k, int l, int M, float *d, const uint16_t *a, int ldd, uint16_t *sw_out) -> int {
    int N, K;
    mat_shape(m, k, &N, &K);
    if (w4) {
      const QMat &q = m->qm[4 * l + k];
      return gemm_f16(d, a, m->pf_w16 + layer_w16_offset(m, k), q.alpha + 1, M, N, K, K, K, ldd, sw_out,
                      sw_out ? N / 2 : 0, s, pdl);
    }
    const uint16_t *w = k == 0 ? m->wqkv + l * wqkv_elems(m) : k == 1 ? m->wo + l * wo_elems(m)
                        : k == 2 ? m->w13 + l * w13_elems(m) : k == 3 ? m->w2 + l * w2_elems(m) : m->wcls;
    if (sw_out) return gemm_bf16_swiglu(sw_out, N / 2, a, w, M, N, K, K, K, s, pdl);
    return gemm_bf16_split(d, a, w, M, N, K, K, K, ldd, 1, 0, s, pdl);
  };
  auto norm = [&](int rows, float *x, const float *delta, size_t stride, const uint16_t *emb, const int *toks,
                  const float *w, uint16_t *out) {
    return launch_norm(D, dim3(rows), s, pdl, x, delta, 1, stride, emb, toks, c.vocab_size, w, out, D, eps,
                       (int)w4, 0, ExchangeWait{});
  };
  for (int off = 0; off < prompt_len; off += per) {
    const int n = std::min(per, prompt_len - off), rows = B * n;
    int rc = launch_kernel(prefill_tokens_kernel, dim3((rows + 255) / 256), dim3(256), 0, s, pdl,
                           "prefill_tokens_kernel", m->pf_tokens, (const int *)prompt, prompt_len, off, n, B);
    if (rc) return rc;
    for (int l = 0; l < c.n_layers; ++l) {
      if (w4) {
        for (int k = 0; k < 4 && rc == CE_OK; ++k) {
          const QMat &q = m->qm[4 * l + k];
          rc = w4t_expand_f16(m->pf_w16 + layer_w16_offset(m, k), q.packed, q.rows, q.cols, s);
        }
        if (rc) return rc;
      }
      rc = norm(rows, m->pf_x, l == 0 ? nullptr : m->pf_delta, (size_t)rows * D, l == 0 ? m->tok_emb : nullptr,
                m->pf_tokens, m->rms_att + (size_t)l * D, m->pf_xb);
      if (rc) return rc;
      rc = gemm(0, l, rows, m->pf_qkv, m->pf_xb, m->qkv_rows, nullptr);
      if (rc) return rc;
      uint16_t *kc = m->kcache + l * m->layer_kv, *vc = m->vcache + l * m->layer_kv;
      rc = launch_kernel(rope_append_kernel, rope_grid(D, m->kv_dim, rows), dim3(256), 0, s, pdl,
                         "rope_append_kernel", m->pf_qkv, m->qkv_rows, 1, (size_t)0, kc, vc,
                         (const float2 *)m->rope, (const int *)m->pos, D, m->kv_dim, m->hs, c.n_kv_heads,
                         c.seq_len, n, off);
      if (rc) return rc;
      auto attention = [&](auto hs_tag) {
        constexpr int HS = decltype(hs_tag)::value;
        if (m->pf_simt) {
          const dim3 grid((unsigned)((n + kPfQ - 1) / kPfQ), (unsigned)c.n_heads, (unsigned)B);
          return launch_kernel(attn_prefill_kernel<HS>, grid, dim3(kPfThreads), pf_smem_bytes(HS), s, pdl,
                               "attn_prefill_kernel", (const float *)m->pf_qkv, m->qkv_rows,
                               (const uint16_t *)kc, (const uint16_t *)vc, (const int *)m->pos, off, n, c.n_heads,
                               c.n_kv_heads, c.seq_len, m->pf_att, D, (int)w4);
        }
        const dim3 grid((unsigned)((n + kFaM - 1) / kFaM), (unsigned)c.n_heads, (unsigned)B);
        const long long layer_row = (long long)l * (long long)(m->layer_kv / m->hs);
        return launch_kernel(attn_prefill_tc_kernel<HS>, grid, dim3(kFaThreads), (size_t)FaLayout<HS>::total, s,
                             pdl, "attn_prefill_tc_kernel", m->pf_tmk, m->pf_tmv, (const float *)m->pf_qkv,
                             m->qkv_rows, (const int *)m->pos, off, n, c.n_heads, c.n_kv_heads, c.seq_len,
                             layer_row, m->pf_att, D, (int)w4);
      };
      rc = m->hs == 64 ? attention(std::integral_constant<int, 64>{})
                       : attention(std::integral_constant<int, 128>{});
      if (rc) return rc;
      rc = gemm(1, l, rows, m->pf_delta, m->pf_att, D, nullptr);
      if (rc) return rc;
      rc = norm(rows, m->pf_x, m->pf_delta, (size_t)rows * D, nullptr, nullptr, m->rms_ffn + (size_t)l * D,
                m->pf_xb);
      if (rc) return rc;
      rc = gemm(2, l, rows, nullptr, m->pf_xb, 2 * Hd, m->pf_hb);  // SwiGLU epilogue
      if (rc) return rc;
      rc = gemm(3, l, rows, m->pf_delta, m->pf_hb, D, nullptr);
      if (rc) return rc;
    }
    if (off + n < prompt_len) continue;
    // last chunk: final norm, then the decode step's tail on each
    // sequence's last prompt position
    rc = norm(rows, m->pf_x, m->pf_delta, (size_t)rows * D, nullptr, nullptr, m->rms_final, m->pf_xb);
    if (rc) return rc;
    rc = launch_kernel(gather_rows16_kernel, dim3(2 * sm_count()), dim3(256), 0, s, pdl, "gather_rows16_kernel",
                       m->xb, (const uint16_t *)m->pf_xb, n, n - 1, D, B);
    if (rc) return rc;
  }
  int rc;
  {
    int N, K;
    mat_shape(m, 4, &N, &K);
    if (w4) {
      const QMat &q = m->qm[4 * c.n_layers];
      rc = gemm_w4t(m->logits, m->xb, q.packed, q.alpha + 1, B, N, K, K, c.vocab_size, 1, 0, nullptr, 0, s, pdl);
    } else {
      rc = gemm_bf16_split(m->logits, m->xb, m->wcls, B, N, K, K, K, c.vocab_size, 1, 0, s, pdl);
    }
    if (rc) return rc;
  }
  rc = m->temperature > 0.f
           ? launch_kernel(sample_kernel, dim3(B), dim3(kSampleThreads), 0, s, pdl, "sample_kernel",
                           (const float *)m->logits, c.vocab_size, m->temperature, m->top_p, m->seed, m->tokens,
                           m->generated, m->cap, (const int *)m->step)
           : launch_kernel(argmax_kernel, dim3(B), dim3(kRowThreads), 0, s, pdl, "argmax_kernel",
                           (const float *)m->logits, c.vocab_size, m->tokens, m->generated, m->cap,
                           (const int *)m->step);
  if (rc) return rc;
  return launch_kernel(advance_by_kernel, dim3(1), dim3(1), 0, s, pdl, "advance_by_kernel", m->pos, m->step,
                       prompt_len);
}

int ce_llama_bind_exchange(ce_llama *m, uint16_t *att, float *delta, uint16_t *hb, float *top) {
  CE_REQUIRE(m != nullptr, "null model");
  CE_REQUIRE(att && delta && hb && top, "null exchange buffer");
  CE_REQUIRE(((reinterpret_cast<uintptr_t>(att) | reinterpret_cast<uintptr_t>(delta) |
               reinterpret_cast<uintptr_t>(hb) | reinterpret_cast<uintptr_t>(top)) & 15u) == 0,
             "exchange buffers must be 16-byte aligned");
  m->x_att = att;
  m->x_delta = delta;
  m->x_hb = hb;
  m->x_top = reinterpret_cast<float2 *>(top);
  return CE_OK;
}

int ce_llama_exchange_open(ce_llama *m, void *handle_out) {
  CE_REQUIRE(m != nullptr && handle_out != nullptr, "null argument");
  CE_REQUIRE(m->world > 1, "peer exchange needs a sharded model (world > 1)");
  CE_REQUIRE(m->world <= 32, "peer exchange supports at most 32 ranks (world %d)", m->world);
  if (m->x_block == nullptr) {
    const size_t n = m->world, B = m->B;
    const size_t sizes[5] = {n * B * m->lD * 2, n * B * m->lD * 4, n * B * m->lHd * 2, n * B * 8, 4 * n * 8};
    size_t off = 0;
    for (int i = 0; i < 5; ++i) {
      m->x_off[i] = off;
      off += (sizes[i] + 255) / 256 * 256;
    }
    m->x_block_bytes = off;
    CE_CUDA_TRY(cudaMalloc(&m->x_block, off));
    CE_CUDA_TRY(cudaMemset(m->x_block, 0, off));
    CE_CUDA_TRY(cudaMalloc(&m->x_counter, 4));
    CE_CUDA_TRY(cudaMemset(m->x_counter, 0, 4));
    CE_CUDA_TRY(cudaMalloc(&m->x_gen, 4));
    CE_CUDA_TRY(cudaMemcpy(m->x_gen, &m->host_gen, 4, cudaMemcpyHostToDevice));
    CE_CUDA_TRY(cudaMalloc(&m->d_blocks, n * sizeof(uint8_t *)));
    m->x_att = reinterpret_cast<uint16_t *>(m->x_block + m->x_off[0]);
    m->x_delta = reinterpret_cast<float *>(m->x_block + m->x_off[1]);
    m->x_hb = reinterpret_cast<uint16_t *>(m->x_block + m->x_off[2]);
    m->x_top = reinterpret_cast<float2 *>(m->x_block + m->x_off[3]);
  }
  cudaIpcMemHandle_t h;
  CE_CUDA_TRY(cudaIpcGetMemHandle(&h, m->x_block));
  static_assert(sizeof(cudaIpcMemHandle_t) <= CE_IPC_HANDLE_BYTES, "IPC handle size");
  std::memset(handle_out, 0, CE_IPC_HANDLE_BYTES);
  std::memcpy(handle_out, &h, sizeof(h));
  return CE_OK;
}

int ce_llama_exchange_connect(ce_llama *m, const void *handles) {
  CE_REQUIRE(m != nullptr && handles != nullptr, "null argument");
  CE_REQUIRE(m->x_block != nullptr, "call ce_llama_exchange_open first");
  CE_REQUIRE(!m->p2p, "the exchange is already connected");
  const int n = m->world;
  m->peer_block.assign(n, nullptr);
  for (int q = 0; q < n; ++q) {
    if (q == m->rank) {
      m->peer_block[q] = m->x_block;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)q * CE_IPC_HANDLE_BYTES, sizeof(h));
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_error(e, format("cudaIpcOpenMemHandle(rank %d)", q).c_str());
    m->peer_block[q] = static_cast<uint8_t *>(p);
  }
  CE_CUDA_TRY(cudaMemcpy(m->d_blocks, m->peer_block.data(), n * sizeof(uint8_t *), cudaMemcpyHostToDevice));
  m->p2p = true;
  return CE_OK;
}

// One segment of the row-sharded step with the peer-memory exchange: the
// exchange buffers are the consumers' operands ([batch][full width], this
// rank's columns at rank x slice), producers write their slice into every
// rank's buffer and signal, consumers wait on the flags (the W4A16 GEMM in
// its activation producer, so the wait overlaps its weight streaming).
int enqueue_segment_p2p(ce_llama *m, int segment, int l, cudaStream_t s) {
  const ce_llama_config &c = m->c;
  const int B = m->B, D = c.dim, Hd = c.hidden_dim, n = m->world, r = m->rank, L = c.n_layers;
  const int lD = m->lD, lHd = m->lHd;
  const bool pdl = m->pdl, w4 = m->precision == CE_PREC_NVFP4_E2M1;
  const float eps = 1e-5f;
  auto wait_of = [&](int kind, int per_step, int index) {
    ExchangeWait w{};
    w.flags = reinterpret_cast<const unsigned long long *>(m->x_block + m->x_off[4]) + (size_t)kind * n;
    w.gen = m->x_gen;
    w.step = m->step;
    w.world = n;
    w.rank = r;
    w.per_step = per_step;
    w.index = index;
    return w;
  };
  auto put_of = [&](int kind, int per_step, int index) {
    ExchangePut p{};
    p.blocks = m->d_blocks;
    p.flag_off = m->x_off[4] + ((size_t)kind * n + r) * 8;
    p.counter = m->x_counter;
    p.gen = m->x_gen;
    p.step = m->step;
    p.world = n;
    p.rank = r;
    p.per_step = per_step;
    p.index = index;
    return p;
  };
  const unsigned grid_put = (unsigned)(2 * sm_count());
  // y = a W^T of weight kind k of layer l into split-K partials; xw: the
  // operand a is an exchange buffer delivered by the peers
  auto gemm = [&](int k, int l, float *d, const uint16_t *a, int lda, int ldd, int splits, long long stride,
                  const ExchangeWait *xw) -> int {
    int N, K;
    mat_shape(m, k, &N, &K);
    if (w4) {
      const QMat &q = m->qm[k == 4 ? 4 * L : 4 * l + k];
      return gemm_w4t(d, a, q.packed, q.alpha + 1, B, N, K, lda, ldd, splits, stride, nullptr, 0, s, pdl,
                      xw);
    }
    if (xw != nullptr) {
      const int rc = launch_kernel(exchange_wait_kernel, dim3(1), dim3(32), 0, s, pdl, "exchange_wait_kernel", *xw,
                                   930u + (unsigned)k);
      if (rc) return rc;
    }
    const uint16_t *w = k == 0 ? m->wqkv + l * wqkv_elems(m) : k == 1 ? m->wo + l * wo_elems(m)
                        : k == 2 ? m->w13 + l * w13_elems(m) : k == 3 ? m->w2 + l * w2_elems(m) : m->wcls;
    return gemm_bf16_split(d, a, w, B, N, K, lda, K, ldd, splits, stride, s, pdl);
  };
  // residual add of the exchanged delta [batch][dim] (after its wait) or the
  // embedding, then RMSNorm into xb
  auto norm = [&](bool embed, const float *w, ExchangeWait xw) {
    return launch_norm(D, dim3(B), s, pdl, m->x, embed ? (const float *)nullptr : (const float *)m->x_delta, 1,
                       (size_t)0, embed ? (const uint16_t *)m->tok_emb : (const uint16_t *)nullptr,
                       (const int *)m->tokens, c.vocab_size, w, m->xb, D, eps, (int)w4, 0, xw);
  };
  // the o-projection / w2 output: split-K partials summed into this rank's
  // columns of every rank's delta exchange
  auto to_delta = [&](int k, int l, const uint16_t *a, int lda, const ExchangeWait &xw, int splits, int index) {
    int rc = gemm(k, l, m->delta, a, lda, lD, splits, (long long)B * lD, &xw);
    if (rc) return rc;
    return launch_kernel(sum_splits_put_kernel, dim3(grid_put), dim3(256), 0, s, pdl, "sum_splits_put_kernel",
                         (const float *)m->delta, splits, B, lD, put_of(1, 2 * L, index),
                         m->x_off[1] + (size_t)r * lD * 4, D);
  };
  int rc = CE_OK;
  switch (segment) {
    case CE_LLAMA_SEG_ATTN: {
      rc = norm(l == 0, m->rms_att + (size_t)l * D, l == 0 ? ExchangeWait{} : wait_of(1, 2 * L, 2 * (l - 1) + 1));
      if (rc) return rc;
      const size_t qkv_stride = (size_t)B * m->qkv_rows;
      rc = gemm(0, l, m->qkv, m->xb, D, m->qkv_rows, m->sp_qkv, (long long)qkv_stride, nullptr);
      if (rc) return rc;
      uint16_t *kc = m->kcache + l * m->layer_kv, *vc = m->vcache + l * m->layer_kv;
      rc = launch_kernel(rope_append_kernel, rope_grid(lD, m->kv_dim, B), dim3(256), 0, s, pdl, "rope_append_kernel",
                         m->qkv, m->qkv_rows, m->sp_qkv, qkv_stride, kc, vc, (const float2 *)m->rope,
                         (const int *)m->pos, lD, m->kv_dim, m->hs, m->lKH, c.seq_len, 1, 0);
      if (rc) return rc;
      const dim3 agrid(m->attn_splits, m->lH, B);
      const size_t smem = attn_smem_bytes(m->hs);
      uint16_t *out = m->x_att + (size_t)r * lD;  // this rank's columns of [batch][dim]
      auto attention = [&](auto hs_tag) {
        constexpr int HS = decltype(hs_tag)::value;
        return launch_kernel(attn_decode_kernel<HS>, agrid, dim3(32), smem, s, pdl, "attn_decode_kernel",
                             (const float *)m->qkv, m->qkv_rows, (const uint16_t *)kc, (const uint16_t *)vc,
                             (const int *)m->pos, m->lH, m->lKH, c.seq_len, m->attn_splits, m->part, m->arrivals,
                             out, D, (int)w4);
      };
      rc = m->hs == 64 ? attention(std::integral_constant<int, 64>{}) : attention(std::integral_constant<int, 128>{});
      if (rc) return rc;
      return launch_kernel(exchange_put_kernel, dim3(grid_put), dim3(256), 0, s, pdl, "exchange_put_kernel",
                           put_of(0, L, l), m->x_off[0] + (size_t)r * lD * 2, B, (size_t)lD * 2, (size_t)D * 2);
    }
    case CE_LLAMA_SEG_OPROJ:
      return to_delta(1, l, m->x_att, D, wait_of(0, L, l), m->sp_o, 2 * l);
    case CE_LLAMA_SEG_FFN_IN: {
      rc = norm(false, m->rms_ffn + (size_t)l * D, wait_of(1, 2 * L, 2 * l));
      if (rc) return rc;
      const size_t h_stride = (size_t)B * 2 * lHd;
      rc = gemm(2, l, m->h, m->xb, D, 2 * lHd, m->sp_13, (long long)h_stride, nullptr);
      if (rc) return rc;
      return launch_kernel(swiglu_put_kernel, dim3(grid_put), dim3(256), 0, s, pdl, "swiglu_put_kernel",
                           (const float *)m->h, m->sp_13, h_stride, B, lHd, (int)w4, put_of(2, L, l),
                           m->x_off[2] + (size_t)r * lHd * 2, Hd);
    }
    case CE_LLAMA_SEG_FFN_OUT:
      return to_delta(3, l, m->x_hb, Hd, wait_of(2, L, l), m->sp_2, 2 * l + 1);
    case CE_LLAMA_SEG_HEAD:
      rc = norm(false, m->rms_final, wait_of(1, 2 * L, 2 * (L - 1) + 1));
      if (rc) return rc;
      rc = gemm(4, 0, m->logits, m->xb, D, m->lV, 1, 0, nullptr);
      if (rc) return rc;
      return launch_kernel(shard_top1_kernel, dim3(B), dim3(kRowThreads), 0, s, pdl, "shard_top1_kernel",
                           (const float *)m->logits, m->lV, r * m->lV, (float2 *)nullptr, put_of(3, 1, 0),
                           m->x_off[3] + (size_t)r * B * 8);
    case CE_LLAMA_SEG_PICK:
      rc = launch_kernel(pick_top_kernel, dim3((B + 127) / 128), dim3(128), 0, s, pdl, "pick_top_kernel",
                         (const float2 *)m->x_top, n, B, m->tokens, m->generated, m->cap, (const int *)m->step,
                         wait_of(3, 1, 0));
      if (rc) return rc;
      return launch_kernel(advance_kernel, dim3(1), dim3(1), 0, s, pdl, "advance_kernel", m->pos, m->step);
    default:
      return set_error(CE_ERR_USAGE, format("unknown segment %d", segment));
  }
}

int ce_llama_enqueue_segment(ce_llama *m, int segment, int layer, ce_stream_t stream) {
  CE_REQUIRE(m != nullptr, "null model");
  CE_REQUIRE(m->p2p || (m->x_att && m->x_delta && m->x_hb && m->x_top),
             "exchange buffers are not bound (ce_llama_bind_exchange or ce_llama_exchange_connect)");
  const ce_llama_config &c = m->c;
  CE_REQUIRE(segment == CE_LLAMA_SEG_HEAD || segment == CE_LLAMA_SEG_PICK || (layer >= 0 && layer < c.n_layers),
             "layer %d out of range", layer);
  cudaStream_t s = (cudaStream_t)stream;
  if (m->p2p) return enqueue_segment_p2p(m, segment, layer, s);
  const int B = m->B, D = c.dim, n = m->world, r = m->rank;
  const int lD = m->lD, lHd = m->lHd;
  const bool pdl = m->pdl, w4 = m->precision == CE_PREC_NVFP4_E2M1;
  const size_t slot_d = (size_t)B * lD;  // one rank's slot of the delta / attention exchange
  const float eps = 1e-5f;
  auto gemm = [&](int k, int l, float *d, const uint16_t *a, int ldd, int splits, long long stride,
                  uint16_t *sw_out, int sw_ld) -> int {
    int N, K;
    mat_shape(m, k, &N, &K);
    if (w4) {
      const QMat &q = m->qm[k == 4 ? 4 * c.n_layers : 4 * l + k];
      return gemm_w4t(d, a, q.packed, q.alpha + 1, B, N, K, K, ldd, splits, stride, sw_out, sw_ld, s,
                      pdl);
    }
    const uint16_t *w = k == 0 ? m->wqkv + l * wqkv_elems(m) : k == 1 ? m->wo + l * wo_elems(m)
                        : k == 2 ? m->w13 + l * w13_elems(m) : k == 3 ? m->w2 + l * w2_elems(m) : m->wcls;
    if (sw_out) return gemm_bf16_swiglu(sw_out, sw_ld, a, w, B, N, K, K, K, s, pdl);
    return gemm_bf16_split(d, a, w, B, N, K, K, K, ldd, splits, stride, s, pdl);
  };
  // residual add of the gathered delta ([rank][batch][lD]) or the embedding,
  // then RMSNorm into xb
  auto norm = [&](bool embed, const float *w) {
    return launch_norm(D, dim3(B), s, pdl, m->x, embed ? (const float *)nullptr : (const float *)m->x_delta, 1,
                       slot_d, embed ? (const uint16_t *)m->tok_emb : (const uint16_t *)nullptr,
                       (const int *)m->tokens, c.vocab_size, w, m->xb, D, eps, (int)w4, lD, ExchangeWait{});
  };
  // the o-projection / w2 output: GEMM into the split partials, summed into
  // this rank's slot of the delta exchange
  auto to_delta_slot = [&](int k, int l, const uint16_t *a, int splits) -> int {
    const long long stride = (long long)B * lD;
    int rc = gemm(k, l, m->delta, a, lD, splits, stride, nullptr, 0);
    if (rc) return rc;
    const size_t n4 = slot_d / 4;
    return launch_kernel(sum_splits_kernel, dim3((unsigned)std::min<size_t>((n4 + 255) / 256, 4 * sm_count())),
                         dim3(256), 0, s, pdl, "sum_splits_kernel", (const float *)m->delta,
                         m->x_delta + (size_t)r * slot_d, splits, n4);
  };
  const int join_grid = 2 * sm_count();
  const int l = layer;
  int rc = CE_OK;
  switch (segment) {
    case CE_LLAMA_SEG_ATTN: {
      rc = norm(l == 0, m->rms_att + (size_t)l * D);
      if (rc) return rc;
      const size_t qkv_stride = (size_t)B * m->qkv_rows;
      rc = gemm(0, l, m->qkv, m->xb, m->qkv_rows, m->sp_qkv, (long long)qkv_stride, nullptr, 0);
      if (rc) return rc;
      uint16_t *kc = m->kcache + l * m->layer_kv, *vc = m->vcache + l * m->layer_kv;
      rc = launch_kernel(rope_append_kernel, rope_grid(lD, m->kv_dim, B), dim3(256), 0, s, pdl, "rope_append_kernel",
                         m->qkv, m->qkv_rows, m->sp_qkv, qkv_stride, kc, vc, (const float2 *)m->rope,
                         (const int *)m->pos, lD, m->kv_dim, m->hs, m->lKH, c.seq_len, 1, 0);
      if (rc) return rc;
      const dim3 agrid(m->attn_splits, m->lH, B);
      const size_t smem = attn_smem_bytes(m->hs);
      uint16_t *slot = m->x_att + (size_t)r * slot_d;
      auto attention = [&](auto hs_tag) {
        constexpr int HS = decltype(hs_tag)::value;
        return launch_kernel(attn_decode_kernel<HS>, agrid, dim3(32), smem, s, pdl, "attn_decode_kernel",
                             (const float *)m->qkv, m->qkv_rows, (const uint16_t *)kc, (const uint16_t *)vc,
                             (const int *)m->pos, m->lH, m->lKH, c.seq_len, m->attn_splits, m->part, m->arrivals,
                             slot, lD, (int)w4);
      };
      return m->hs == 64 ? attention(std::integral_constant<int, 64>{})
                         : attention(std::integral_constant<int, 128>{});
    }
    case CE_LLAMA_SEG_OPROJ:
      rc = launch_kernel(join_shards_kernel, dim3(join_grid), dim3(256), 0, s, pdl, "join_shards_kernel",
                         (const uint16_t *)m->x_att, m->att, n, B, lD);
      if (rc) return rc;
      return to_delta_slot(1, l, m->att, m->sp_o);
    case CE_LLAMA_SEG_FFN_IN: {
      rc = norm(false, m->rms_ffn + (size_t)l * D);
      if (rc) return rc;
      uint16_t *slot = m->x_hb + (size_t)r * B * lHd;
      if (m->sp_13 == 1) return gemm(2, l, nullptr, m->xb, 2 * lHd, 1, 0, slot, lHd);
      const size_t h_stride = (size_t)B * 2 * lHd;
      rc = gemm(2, l, m->h, m->xb, 2 * lHd, m->sp_13, (long long)h_stride, nullptr, 0);
      if (rc) return rc;
      return launch_kernel(swiglu_kernel, dim3(4 * sm_count()), dim3(256), 0, s, pdl, "swiglu_kernel",
                           (const float *)m->h, m->sp_13, h_stride, slot, B, lHd, (int)w4);
    }
    case CE_LLAMA_SEG_FFN_OUT:
      rc = launch_kernel(join_shards_kernel, dim3(join_grid), dim3(256), 0, s, pdl, "join_shards_kernel",
                         (const uint16_t *)m->x_hb, m->hb, n, B, lHd);
      if (rc) return rc;
      return to_delta_slot(3, l, m->hb, m->sp_2);
    case CE_LLAMA_SEG_HEAD:
      rc = norm(false, m->rms_final);
      if (rc) return rc;
      rc = gemm(4, 0, m->logits, m->xb, m->lV, 1, 0, nullptr, 0);
      if (rc) return rc;
      return launch_kernel(shard_top1_kernel, dim3(B), dim3(kRowThreads), 0, s, pdl, "shard_top1_kernel",
                           (const float *)m->logits, m->lV, r * m->lV, m->x_top + (size_t)r * B, ExchangePut{},
                           (size_t)0);
    case CE_LLAMA_SEG_PICK:
      rc = launch_kernel(pick_top_kernel, dim3((B + 127) / 128), dim3(128), 0, s, pdl, "pick_top_kernel",
                         (const float2 *)m->x_top, n, B, m->tokens, m->generated, m->cap, (const int *)m->step,
                         ExchangeWait{});
      if (rc) return rc;
      return launch_kernel(advance_kernel, dim3(1), dim3(1), 0, s, pdl, "advance_kernel", m->pos, m->step);
    default:
      return set_error(CE_ERR_USAGE, format("unknown segment %d", segment));
  }
}

int ce_llama_shard_rows(const ce_llama_config *cfg, int rank, int world, int which, int32_t *rows_out,
                        int *count) {
  CE_REQUIRE(cfg != nullptr && count != nullptr, "null argument");
  const int k = which == CE_LLAMA_WQKV ? 0 : which == CE_LLAMA_WO ? 1 : which == CE_LLAMA_W13 ? 2
                : which == CE_LLAMA_W2 ? 3 : which == CE_LLAMA_WCLS ? 4 : -1;
  CE_REQUIRE(k >= 0, "tensor %d is not a sharded weight", which);
  if (int rc = ce_llama_validate_shard(cfg, 1, 1, CE_PREC_BF16, rank, world)) return rc;
  std::vector<int> rows;
  shard_rows(*cfg, rank, world, k, &rows);
  if (rows_out) std::copy(rows.begin(), rows.end(), rows_out);
  *count = (int)rows.size();
  return CE_OK;
}

int ce_llama_set_sampling(ce_llama *m, float temperature, float top_p, uint64_t seed) {
  CE_REQUIRE(m != nullptr, "null model");
  CE_REQUIRE(temperature >= 0.f && temperature < 1e30f, "temperature must be >= 0 (got %g)", (double)temperature);
  CE_REQUIRE(top_p >= 0.f && top_p <= 1.f, "top_p must be in [0, 1] (got %g)", (double)top_p);
  CE_REQUIRE(temperature == 0.f || m->world == 1,
             "sampling needs the whole vocabulary on one GPU (a sharded model picks greedily)");
  m->temperature = temperature;
  m->top_p = top_p;
  m->seed = seed;
  return CE_OK;
}

int ce_llama_set_pdl(ce_llama *m, int enable) {
  CE_REQUIRE(m != nullptr, "null model");
  m->pdl = enable != 0;
  return CE_OK;
}

int ce_llama_read(ce_llama *m, int which, int layer, void *host, int64_t offset, int64_t bytes) {
  CE_REQUIRE(m != nullptr && host != nullptr, "null argument");
  TensorView v;
  if (int rc = tensor_of(m, which, layer, &v)) return rc;
  CE_REQUIRE(offset >= 0 && bytes >= 0 && (size_t)(offset + bytes) <= v.bytes,
             "range [%lld, %lld) outside the tensor (%zu bytes)", (long long)offset, (long long)(offset + bytes), v.bytes);
  CE_CUDA_TRY(cudaDeviceSynchronize());
  CE_CUDA_TRY(cudaMemcpy(host, (uint8_t *)v.ptr + offset, (size_t)bytes, cudaMemcpyDeviceToHost));
  return CE_OK;
}

int ce_llama_read_nvfp4(ce_llama *m, int which, int layer, uint8_t *packed_host, uint8_t *unused_host,
                        float *alpha_host) {
  CE_REQUIRE(m != nullptr, "null model");
  CE_REQUIRE(m->precision == CE_PREC_NVFP4_E2M1, "the model's weights are not NVFP4");
  const int k = which == CE_LLAMA_WQKV ? 0 : which == CE_LLAMA_WO ? 1 : which == CE_LLAMA_W13 ? 2
                : which == CE_LLAMA_W2 ? 3 : which == CE_LLAMA_WCLS ? 4 : -1;
  CE_REQUIRE(k >= 0, "tensor %d is not an NVFP4 weight", which);
  CE_REQUIRE(k == 4 || (layer >= 0 && layer < m->c.n_layers), "layer %d out of range", layer);
  const QMat &q = m->qm[k == 4 ? 4 * m->c.n_layers : 4 * layer + k];
  CE_CUDA_TRY(cudaDeviceSynchronize());
  (void)unused_host;
  if (packed_host) CE_CUDA_TRY(cudaMemcpy(packed_host, q.packed, q.bytes, cudaMemcpyDeviceToHost));
  if (alpha_host) CE_CUDA_TRY(cudaMemcpy(alpha_host, q.alpha, 8, cudaMemcpyDeviceToHost));
  return CE_OK;
}

int ce_llama_write(ce_llama *m, int which, int layer, const void *host, int64_t offset, int64_t bytes) {
  CE_REQUIRE(m != nullptr && host != nullptr, "null argument");
  TensorView v;
  if (int rc = tensor_of(m, which, layer, &v)) return rc;
  CE_REQUIRE(offset >= 0 && bytes >= 0 && (size_t)(offset + bytes) <= v.bytes,
             "range [%lld, %lld) outside the tensor (%zu bytes)", (long long)offset, (long long)(offset + bytes), v.bytes);
  CE_CUDA_TRY(cudaDeviceSynchronize());
  CE_CUDA_TRY(cudaMemcpy((uint8_t *)v.ptr + offset, host, (size_t)bytes, cudaMemcpyHostToDevice));
  return CE_OK;
}

}  // extern "C"

namespace {

// Weight kind (0 wqkv, 1 wo, 2 w13, 3 w2, 4 classifier) of a CE_LLAMA_*
// matrix, or -1.
int weight_kind(int which) {
  switch (which) {
    case CE_LLAMA_WQKV: return 0;
    case CE_LLAMA_WO: return 1;
    case CE_LLAMA_W13: return 2;
    case CE_LLAMA_W2: return 3;
    case CE_LLAMA_WCLS: return 4;
    default: return -1;
  }
}

// Scratch of a load call, freed on every path.
struct LoadScratch {
  std::vector<void *> ptrs;
  template <class T>
  int alloc(T **p, size_t bytes) {
    void *q = nullptr;
    const cudaError_t e = cudaMalloc(&q, bytes);
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(load scratch)");
    ptrs.push_back(q);
    *p = static_cast<T *>(q);
    return CE_OK;
  }
  ~LoadScratch() {
    for (void *q : ptrs) cudaFree(q);
  }
};

}  // namespace

extern "C" {

int ce_llama_load(ce_llama *m, int which, int layer, const float *host) {
  CE_REQUIRE(m != nullptr && host != nullptr, "null argument");
  const ce_llama_config &c = m->c;
  const int k = weight_kind(which);
  cudaStream_t s = nullptr;
  CE_CUDA_TRY(cudaDeviceSynchronize());
  if (k < 0) {
    switch (which) {
      case CE_LLAMA_RMS_ATT:
      case CE_LLAMA_RMS_FFN:
      case CE_LLAMA_RMS_FINAL: {
        TensorView v;
        if (int rc = tensor_of(m, which, layer, &v)) return rc;
        CE_CUDA_TRY(cudaMemcpy(v.ptr, host, v.bytes, cudaMemcpyHostToDevice));
        return CE_OK;
      }
      case CE_LLAMA_TOK_EMB: {
        LoadScratch sc;
        float *tmp = nullptr;
        const size_t n = (size_t)c.vocab_size * c.dim;
        if (int rc = sc.alloc(&tmp, n * 4)) return rc;
        CE_CUDA_TRY(cudaMemcpy(tmp, host, n * 4, cudaMemcpyHostToDevice));
        if (int rc = convert_bf16(m->tok_emb, tmp, c.vocab_size, c.dim, c.dim, s)) return rc;
        CE_CUDA_TRY(cudaStreamSynchronize(s));
        return CE_OK;
      }
      default:
        return set_error(CE_ERR_USAGE, format("tensor %d is not a loadable weight", which));
    }
  }
  CE_REQUIRE(k == 4 || (layer >= 0 && layer < c.n_layers), "layer %d out of range", layer);
  int rows, cols;
  mat_shape(m, k, &rows, &cols);
  std::vector<int> map;
  shard_rows(c, m->rank, m->world, k, &map);
  LoadScratch sc;
  if (m->precision == CE_PREC_BF16) {
    // this shard's rows, gathered on the host, converted on the device
    std::vector<float> mine((size_t)rows * cols);
    for (int r = 0; r < rows; ++r)
      std::memcpy(mine.data() + (size_t)r * cols, host + (size_t)map[r] * cols, (size_t)cols * 4);
    float *tmp = nullptr;
    if (int rc = sc.alloc(&tmp, mine.size() * 4)) return rc;
    CE_CUDA_TRY(cudaMemcpy(tmp, mine.data(), mine.size() * 4, cudaMemcpyHostToDevice));
    TensorView v;
    if (int rc = tensor_of(m, which, layer, &v)) return rc;
    if (int rc = convert_bf16(static_cast<uint16_t *>(v.ptr), tmp, rows, cols, cols, s)) return rc;
    CE_CUDA_TRY(cudaStreamSynchronize(s));
    return CE_OK;
  }
  // NVFP4: the whole global matrix quantized (tensor amax over all of it),
  // then this shard's rows packed
  const int grows = global_rows(c, k);
  const size_t n = (size_t)grows * cols;
  float *tmp = nullptr;
  uint8_t *codes = nullptr, *scales = nullptr;
  unsigned int *amax = nullptr;
  int *d_map = nullptr;
  int rc = sc.alloc(&tmp, n * 4);
  if (rc == CE_OK) rc = sc.alloc(&codes, n / 2);
  if (rc == CE_OK) rc = sc.alloc(&scales, n / 16);
  if (rc == CE_OK) rc = sc.alloc(&amax, 4);
  if (rc == CE_OK) rc = sc.alloc(&d_map, map.size() * sizeof(int));
  if (rc) return rc;
  CE_CUDA_TRY(cudaMemcpy(tmp, host, n * 4, cudaMemcpyHostToDevice));
  CE_CUDA_TRY(cudaMemcpy(d_map, map.data(), map.size() * sizeof(int), cudaMemcpyHostToDevice));
  const QMat &q = m->qm[k == 4 ? 4 * c.n_layers : 4 * layer + k];
  rc = quantize_nvfp4(codes, scales, q.alpha, amax, tmp, grows, cols, cols / 2, s);
  if (rc == CE_OK) rc = w4t_pack(q.packed, codes, scales, rows, cols, cols / 2, cols / 16, s, d_map);
  if (rc) return rc;
  CE_CUDA_TRY(cudaStreamSynchronize(s));
  return CE_OK;
}

int ce_llama_load_nvfp4(ce_llama *m, int which, int layer, const uint8_t *codes_host, const uint8_t *scales_host,
                        const float *alpha_host) {
  CE_REQUIRE(m != nullptr && codes_host && scales_host && alpha_host, "null argument");
  CE_REQUIRE(m->precision == CE_PREC_NVFP4_E2M1, "ce_llama_load_nvfp4 needs an NVFP4 model");
  const ce_llama_config &c = m->c;
  const int k = weight_kind(which);
  CE_REQUIRE(k >= 0, "tensor %d is not a weight matrix", which);
  CE_REQUIRE(k == 4 || (layer >= 0 && layer < c.n_layers), "layer %d out of range", layer);
  int rows, cols;
  mat_shape(m, k, &rows, &cols);
  std::vector<int> map;
  shard_rows(c, m->rank, m->world, k, &map);
  const size_t n = (size_t)global_rows(c, k) * cols;
  LoadScratch sc;
  uint8_t *codes = nullptr, *scales = nullptr;
  int *d_map = nullptr;
  int rc = sc.alloc(&codes, n / 2);
  if (rc == CE_OK) rc = sc.alloc(&scales, n / 16);
  if (rc == CE_OK) rc = sc.alloc(&d_map, map.size() * sizeof(int));
  if (rc) return rc;
  CE_CUDA_TRY(cudaDeviceSynchronize());
  CE_CUDA_TRY(cudaMemcpy(codes, codes_host, n / 2, cudaMemcpyHostToDevice));
  CE_CUDA_TRY(cudaMemcpy(scales, scales_host, n / 16, cudaMemcpyHostToDevice));
  CE_CUDA_TRY(cudaMemcpy(d_map, map.data(), map.size() * sizeof(int), cudaMemcpyHostToDevice));
  const QMat &q = m->qm[k == 4 ? 4 * c.n_layers : 4 * layer + k];
  CE_CUDA_TRY(cudaMemcpy(q.alpha, alpha_host, 2 * sizeof(float), cudaMemcpyHostToDevice));
  rc = w4t_pack(q.packed, codes, scales, rows, cols, cols / 2, cols / 16, nullptr, d_map);
  if (rc) return rc;
  CE_CUDA_TRY(cudaStreamSynchronize(nullptr));
  return CE_OK;
}

// Reads and clears the status word of the decode kernels (position out of
// the cache, or a staging wait that gave up); synchronizes the device.
int ce_llama_status(void) {
  CE_CUDA_TRY(cudaDeviceSynchronize());
  DeviceStatus h{};
  CE_CUDA_TRY(cudaMemcpyFromSymbol(&h, g_llama_status, sizeof(h)));
  if (h.code == 0) return CE_OK;
  const DeviceStatus zero{};
  CE_CUDA_TRY(cudaMemcpyToSymbol(g_llama_status, &zero, sizeof(zero)));
  if (h.where == 900u) return set_error(CE_ERR_USAGE, "decode position reached the end of the KV cache");
  if (h.where == 901u) return set_error(CE_ERR_USAGE, "prefill positions reached the end of the KV cache");
  if (h.where == 920u || h.where == 923u || (h.where >= 930u && h.where <= 934u))  // peer flag waits
    return set_error(CE_ERR_TIMEOUT, format("peer exchange wait gave up (site %u, block %u)", h.where, h.block));
  return set_error(CE_ERR_TIMEOUT, format("attention staging wait gave up (site %u, block %u)", h.where, h.block));
}

}  // extern "C"
