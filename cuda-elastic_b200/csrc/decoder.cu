// The loom_private llama2c decoder step (applications/loom_private/decoder/):
// for B sequences, every step gathers the embedding row of each sequence's
// current token, RMSNorms it (llama2.c order), multiplies the batch by the
// classifier (logits[b][r] = sum_k C[r][k] * o[b][k]), and turns each logit
// row into probabilities and its first argmax, which becomes the sequence's
// next token on the device. S dependent steps per invocation, no host sync.
//
// Classifier precisions: CE_PREC_FP32 runs the SIMT kernel whose sums follow
// the contract's order (sequential k, separate multiply and add), so the
// synthetic model's outputs are bitwise the reference's; CE_PREC_TF32 and
// CE_PREC_BF16 run the tcgen05 GEMM (gemm.cu), checked by bounds.
#include <stdlib.h>
#include <string.h>

#include <climits>

#include "row_ops.cuh"

namespace ce {

int gemm_bf16(float *d, const uint16_t *a, const uint16_t *b, int M, int N, int K, int lda,
              int ldb, int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group = 0);
int gemm_tf32(float *d, const float *a, const float *b, int M, int N, int K, int lda, int ldb,
              int ldd, const float *row_scale, const float *col_scale, int force_bn,
              cudaStream_t s, int force_group = 0);
int gemm_simt_fp32(float *d, const float *a, const float *b, int M, int N, int K, int lda,
                   int ldb, int ldd, cudaStream_t s);
int convert_bf16(uint16_t *out, const float *in, int rows, int cols, int ld, cudaStream_t s);

namespace {

using namespace rowops;

constexpr int kNormThreads = 512;
constexpr int kSoftmaxThreads = 256;

// Synthetic model (contract.json "data_generation", decoder.cu:28-43):
// embedding row t is 1 everywhere except 4 at column t; classifier row r is
// 0 except 1 at column (r + vocab - 1) mod vocab; the RMSNorm weight is 1.
__global__ void init_synthetic_model_kernel(float *embedding, float *classifier, float *norm_w,
                                            int width, int vocab) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t first = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)vocab * width;
  for (size_t i = first; i < total; i += stride) {
    const int row = (int)(i / (size_t)width);
    const int col = (int)(i % (size_t)width);
    embedding[i] = col == row ? 4.0f : 1.0f;
    classifier[i] = col == (row + vocab - 1) % vocab ? 1.0f : 0.0f;
  }
  for (size_t j = first; j < (size_t)width; j += stride) norm_w[j] = 1.0f;
}

// RMSNorm of the embedding row of each sequence's token (one block per
// sequence). Register path when the row is 16-byte vectorisable, else a
// scalar two-pass path. A token outside [0, vocab) marks the row NaN so the
// check fails (decoder.cu:58-61).
template <int NV>
__global__ void __launch_bounds__(kNormThreads)
gather_rmsnorm_kernel(float *normalized, uint16_t *operand_bf16, int ld_bf16, const int *tokens,
                      const float *embedding, const float *w, int width, int vocab, float eps) {
  __shared__ float scratch[32];
  const int b = blockIdx.x;
  const int token = tokens[b];
  float *o = normalized + (size_t)b * width;
  uint16_t *ob = operand_bf16 ? operand_bf16 + (size_t)b * ld_bf16 : nullptr;
  if (token < 0 || token >= vocab) {
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      o[j] = __int_as_float(0x7fffffff);
      if (ob) ob[j] = 0x7fff;
    }
    return;
  }
  const float *x = embedding + (size_t)token * width;
  if constexpr (NV > 0) {
    rmsnorm_row<(NV > 0 ? NV : 1)>(reinterpret_cast<const float4 *>(x),
                                   reinterpret_cast<const float4 *>(w), reinterpret_cast<float4 *>(o),
                                   reinterpret_cast<uint2 *>(ob), width >> 2, width, eps, scratch);
  } else {
    float ss = 0.f;
    for (int j = threadIdx.x; j < width; j += blockDim.x) ss += x[j] * x[j];
    ss = block_sum(ss, scratch);
    const float scale = 1.0f / sqrtf(ss / (float)width + eps);
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      const float v = w[j] * (scale * x[j]);
      o[j] = v;
      if (ob) ob[j] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
  }
  if (ob)  // zero padding columns of the GEMM operand
    for (int j = width + threadIdx.x; j < ld_bf16; j += blockDim.x) ob[j] = 0;
}

// Softmax + first argmax of one logit row per block, with the contract's
// fixed reduction order (contract.json "operation_order"; the order of
// decoder.cu:131-198): thread t of 256 visits r = t, t + 256, ... in
// increasing r, the 256 partials are combined by a halving tree
// (stride 128, 64, ..., 1), the maximum the same way; probabilities are
// e / sum; ties of the argmax go to the lower index. Keeping this order keeps
// the probability bits (and the output digest) of the reference's contract.
__global__ void __launch_bounds__(kSoftmaxThreads)
softmax_argmax_kernel(float *probabilities, const float *logits, int *tokens, int *generated,
                      int vocab, int steps, int step) {
  __shared__ float value[kSoftmaxThreads];
  __shared__ int index[kSoftmaxThreads];
  const int t = threadIdx.x;
  const size_t row = blockIdx.x;
  const float *x = logits + row * (size_t)vocab;
  float *p = probabilities + row * (size_t)vocab;

  float m = -INFINITY;
  for (int r = t; r < vocab; r += kSoftmaxThreads) m = fmaxf(m, x[r]);
  value[t] = m;
  __syncthreads();
  for (int stride = kSoftmaxThreads / 2; stride > 0; stride >>= 1) {
    if (t < stride) value[t] = fmaxf(value[t], value[t + stride]);
    __syncthreads();
  }
  m = value[0];
  __syncthreads();

  float s = 0.f;
  for (int r = t; r < vocab; r += kSoftmaxThreads) {
    const float e = expf(x[r] - m);
    p[r] = e;
    s += e;
  }
  value[t] = s;
  __syncthreads();
  for (int stride = kSoftmaxThreads / 2; stride > 0; stride >>= 1) {
    if (t < stride) value[t] += value[t + stride];
    __syncthreads();
  }
  s = value[0];
  __syncthreads();

  float best = -INFINITY;
  int best_index = INT_MAX;
  for (int r = t; r < vocab; r += kSoftmaxThreads) {
    const float q = p[r] / s;
    p[r] = q;
    if (q > best) {
      best = q;
      best_index = r;
    }
  }
  value[t] = best;
  index[t] = best_index;
  __syncthreads();
  for (int stride = kSoftmaxThreads / 2; stride > 0; stride >>= 1) {
    if (t < stride) {
      const float ov = value[t + stride];
      const int oi = index[t + stride];
      if (ov > value[t] || (ov == value[t] && oi < index[t])) {
        value[t] = ov;
        index[t] = oi;
      }
    }
    __syncthreads();
  }
  if (t == 0) {
    const int next = index[0] == INT_MAX ? -1 : index[0];
    tokens[row] = next;
    generated[row * (size_t)steps + step] = next;
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace ce

using namespace ce;

struct ce_decoder {
  int64_t B = 0, W = 0, V = 0, S = 0;
  int precision = 0;
  int ld = 0;  // bf16 operand / classifier leading dimension
  float *embedding = nullptr, *classifier = nullptr, *norm_w = nullptr;
  uint16_t *classifier_bf16 = nullptr, *operand_bf16 = nullptr;
  int32_t *d_prompts = nullptr, *d_tokens = nullptr, *d_generated = nullptr;
  float *d_normalized = nullptr, *d_logits = nullptr, *d_probabilities = nullptr;
  int32_t *h_prompts = nullptr, *h_generated = nullptr;
  float eps = 1e-5f;
};

namespace {

void free_decoder(ce_decoder *d) {
  void *dev[] = {d->embedding, d->classifier, d->norm_w, d->classifier_bf16, d->operand_bf16,
                 d->d_prompts, d->d_tokens, d->d_generated, d->d_normalized, d->d_logits,
                 d->d_probabilities};
  for (void *p : dev)
    if (p) cudaFree(p);
  if (d->h_prompts) cudaFreeHost(d->h_prompts);
  if (d->h_generated) cudaFreeHost(d->h_generated);
  delete d;
}

int convert_classifier(ce_decoder *d, cudaStream_t s) {
  if (d->precision != CE_PREC_BF16) return CE_OK;
  return convert_bf16(d->classifier_bf16, d->classifier, (int)d->V, (int)d->W, d->ld, s);
}

}  // namespace

extern "C" {

// Validation and allocation of applications/loom_private/decoder/decoder.cu:
// 369-408 (make_decoder, with its limits and messages) and setup (:241-265).
int ce_decoder_validate(int64_t batch, int64_t width, int64_t vocab, int64_t steps, int precision) {
  CE_REQUIRE(batch >= 1 && batch <= (1LL << 20), "batch must be in [1, 1048576] (got %lld)",
             (long long)batch);
  CE_REQUIRE(width >= 2 && width <= (1LL << 24) - 16,
             "width must be in [2, 16777200] so the rmsnorm square sum (width + 15) stays an "
             "exact float integer (got %lld)",
             (long long)width);
  CE_REQUIRE(vocab >= 2 && vocab <= width,
             "vocab must satisfy 2 <= vocab <= width: every token owns one embedding position "
             "(got vocab=%lld, width=%lld)",
             (long long)vocab, (long long)width);
  CE_REQUIRE(steps >= 2 && steps <= 1024,
             "steps must be in [2, 1024]: generation repeats the per-token kernels (got %lld)",
             (long long)steps);
  CE_REQUIRE(precision == CE_PREC_FP32 || precision == CE_PREC_TF32 || precision == CE_PREC_BF16,
             "decoder precision %d is not available", precision);
  CE_REQUIRE(precision != CE_PREC_TF32 || width % 4 == 0,
             "the tf32 classifier needs width %% 4 == 0 (got %lld)", (long long)width);
  const double diagnostics = 4.0 * (double)steps * (double)batch * ((double)width + 2.0 * (double)vocab);
  const double device = 4.0 * (2.0 * (double)vocab * (double)width) + diagnostics;
  CE_REQUIRE(device <= 160.0 * (1LL << 30) && diagnostics <= 64.0 * (1LL << 30),
             "dimensions need %.1f GiB of device memory and %.1f GiB of host diagnostics "
             "(limits 160 and 64 GiB)",
             device / (1LL << 30), diagnostics / (1LL << 30));
  return CE_OK;
}

int ce_decoder_create(ce_decoder **out, int64_t batch, int64_t width, int64_t vocab, int64_t steps,
                      int precision, ce_stream_t stream) {
  CE_REQUIRE(out != nullptr, "null decoder pointer");
  *out = nullptr;
  if (int rc = ce_decoder_validate(batch, width, vocab, steps, precision)) return rc;
  ce_decoder *d = new ce_decoder();
  d->B = batch;
  d->W = width;
  d->V = vocab;
  d->S = steps;
  d->precision = precision;
  d->ld = (int)(((width + 63) / 64) * 64);
  const size_t model = (size_t)vocab * width;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaSuccess;
#define CE_ALLOC(ptr, bytes)                                   \
  do {                                                         \
    e = cudaMalloc(&(ptr), (bytes));                           \
    if (e != cudaSuccess) {                                    \
      free_decoder(d);                                         \
      return cuda_error(e, "cudaMalloc(" #ptr ")");            \
    }                                                          \
  } while (0)
  CE_ALLOC(d->embedding, model * 4);
  CE_ALLOC(d->classifier, model * 4);
  CE_ALLOC(d->norm_w, (size_t)width * 4);
  CE_ALLOC(d->d_prompts, (size_t)batch * 4);
  CE_ALLOC(d->d_tokens, (size_t)batch * 4);
  CE_ALLOC(d->d_generated, (size_t)batch * steps * 4);
  CE_ALLOC(d->d_normalized, (size_t)steps * batch * width * 4);
  CE_ALLOC(d->d_logits, (size_t)steps * batch * vocab * 4);
  CE_ALLOC(d->d_probabilities, (size_t)steps * batch * vocab * 4);
  if (precision == CE_PREC_BF16) {
    CE_ALLOC(d->classifier_bf16, (size_t)vocab * d->ld * 2);
    CE_ALLOC(d->operand_bf16, (size_t)batch * d->ld * 2);
  }
#undef CE_ALLOC
  e = cudaMallocHost(&d->h_prompts, (size_t)batch * 4);
  if (e == cudaSuccess) e = cudaMallocHost(&d->h_generated, (size_t)batch * steps * 4);
  if (e != cudaSuccess) {
    free_decoder(d);
    return cuda_error(e, "cudaMallocHost");
  }
  for (int64_t b = 0; b < batch; ++b) d->h_prompts[b] = (int32_t)(b % vocab);
  init_synthetic_model_kernel<<<1024, 256, 0, s>>>(d->embedding, d->classifier, d->norm_w,
                                                   (int)width, (int)vocab);
  e = cudaPeekAtLastError();
  int rc = e == cudaSuccess ? convert_classifier(d, s) : cuda_error(e, "init_synthetic_model_kernel");
  if (rc == CE_OK) {
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) rc = cuda_error(e, "cudaStreamSynchronize");
  }
  if (rc != CE_OK) {
    free_decoder(d);
    return rc;
  }
  *out = d;
  return CE_OK;
}

int ce_decoder_destroy(ce_decoder *d) {
  if (d) free_decoder(d);
  return CE_OK;
}

// Replaces the synthetic model by caller weights (device, fp32):
// embedding and classifier [vocab][width], norm weight [width]. Setup call.
int ce_decoder_set_model(ce_decoder *d, const float *embedding, const float *classifier,
                         const float *norm_w, ce_stream_t stream) {
  CE_REQUIRE(d && embedding && classifier && norm_w, "null argument");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t model = (size_t)d->V * d->W * 4;
  CE_CUDA_TRY(cudaMemcpyAsync(d->embedding, embedding, model, cudaMemcpyDeviceToDevice, s));
  CE_CUDA_TRY(cudaMemcpyAsync(d->classifier, classifier, model, cudaMemcpyDeviceToDevice, s));
  CE_CUDA_TRY(cudaMemcpyAsync(d->norm_w, norm_w, (size_t)d->W * 4, cudaMemcpyDeviceToDevice, s));
  int rc = convert_classifier(d, s);
  if (rc) return rc;
  CE_CUDA_TRY(cudaStreamSynchronize(s));
  return CE_OK;
}

// Token reset from the resident prompts and every step (decoder.cu:276-296).
int ce_decoder_enqueue_compute(ce_decoder *d, ce_stream_t stream) {
  CE_REQUIRE(d != nullptr, "null decoder");
  cudaStream_t s = (cudaStream_t)stream;
  const int B = (int)d->B, W = (int)d->W, V = (int)d->V;
  CE_CUDA_TRY(cudaMemcpyAsync(d->d_tokens, d->d_prompts, (size_t)B * 4, cudaMemcpyDeviceToDevice, s));
  const bool vec = W % 4 == 0 && W / 4 <= 16 * kNormThreads && aligned16(d->embedding);
  int nv = 0;
  if (vec) nv = W / 4 <= kNormThreads ? 1 : W / 4 <= 2 * kNormThreads ? 2 : W / 4 <= 4 * kNormThreads ? 4 : W / 4 <= 8 * kNormThreads ? 8 : 16;
  for (int64_t step = 0; step < d->S; ++step) {
    float *normalized = d->d_normalized + (size_t)step * d->B * d->W;
    float *logits = d->d_logits + (size_t)step * d->B * d->V;
    float *probs = d->d_probabilities + (size_t)step * d->B * d->V;
    uint16_t *opb = d->precision == CE_PREC_BF16 ? d->operand_bf16 : nullptr;
    switch (nv) {
#define CE_NORM(NVv)                                                                          \
  case NVv:                                                                                   \
    gather_rmsnorm_kernel<NVv><<<B, kNormThreads, 0, s>>>(normalized, opb, d->ld, d->d_tokens, \
                                                          d->embedding, d->norm_w, W, V, d->eps); \
    break;
      CE_NORM(0)
      CE_NORM(1)
      CE_NORM(2)
      CE_NORM(4)
      CE_NORM(8)
      CE_NORM(16)
#undef CE_NORM
    }
    CE_LAUNCH_CHECK("gather_rmsnorm_kernel");
    int rc;
    if (d->precision == CE_PREC_BF16)
      rc = gemm_bf16(logits, opb, d->classifier_bf16, B, V, W, d->ld, d->ld, V, nullptr, nullptr, 0, s);
    else if (d->precision == CE_PREC_TF32)
      rc = gemm_tf32(logits, normalized, d->classifier, B, V, W, W, W, V, nullptr, nullptr, 0, s);
    else
      rc = gemm_simt_fp32(logits, normalized, d->classifier, B, V, W, W, W, V, s);
    if (rc) return rc;
    softmax_argmax_kernel<<<B, kSoftmaxThreads, 0, s>>>(probs, logits, d->d_tokens, d->d_generated,
                                                        V, (int)d->S, (int)step);
    CE_LAUNCH_CHECK("softmax_argmax_kernel");
  }
  return CE_OK;
}

// Prompt upload (pinned H2D), compute, generated download (pinned D2H),
// decoder.cu:267-274.
int ce_decoder_enqueue_application(ce_decoder *d, ce_stream_t stream) {
  CE_REQUIRE(d != nullptr, "null decoder");
  cudaStream_t s = (cudaStream_t)stream;
  CE_CUDA_TRY(cudaMemcpyAsync(d->d_prompts, d->h_prompts, (size_t)d->B * 4, cudaMemcpyHostToDevice, s));
  int rc = ce_decoder_enqueue_compute(d, stream);
  if (rc) return rc;
  CE_CUDA_TRY(cudaMemcpyAsync(d->h_generated, d->d_generated, (size_t)d->B * d->S * 4,
                              cudaMemcpyDeviceToHost, s));
  return CE_OK;
}

// 0xFF bytes into every output and into the device prompts and tokens
// (token -1, float NaN), device and host (decoder.cu:298-312).
int ce_decoder_poison(ce_decoder *d, ce_stream_t stream) {
  CE_REQUIRE(d != nullptr, "null decoder");
  cudaStream_t s = (cudaStream_t)stream;
  CE_CUDA_TRY(cudaMemsetAsync(d->d_prompts, 0xFF, (size_t)d->B * 4, s));
  CE_CUDA_TRY(cudaMemsetAsync(d->d_tokens, 0xFF, (size_t)d->B * 4, s));
  CE_CUDA_TRY(cudaMemsetAsync(d->d_generated, 0xFF, (size_t)d->B * d->S * 4, s));
  CE_CUDA_TRY(cudaMemsetAsync(d->d_normalized, 0xFF, (size_t)d->S * d->B * d->W * 4, s));
  CE_CUDA_TRY(cudaMemsetAsync(d->d_logits, 0xFF, (size_t)d->S * d->B * d->V * 4, s));
  CE_CUDA_TRY(cudaMemsetAsync(d->d_probabilities, 0xFF, (size_t)d->S * d->B * d->V * 4, s));
  CE_CUDA_TRY(cudaStreamSynchronize(s));
  memset(d->h_generated, 0xFF, (size_t)d->B * d->S * 4);
  return CE_OK;
}

// Synchronous diagnostics copy (decoder.cu:318-331): any pointer may be NULL.
// generated [batch][steps] comes from the pinned buffer the application scope
// downloads into, or (from_device != 0) from the device.
int ce_decoder_copy_outputs(ce_decoder *d, int from_device, int32_t *generated, float *normalized,
                            float *logits, float *probabilities) {
  CE_REQUIRE(d != nullptr, "null decoder");
  CE_CUDA_TRY(cudaDeviceSynchronize());
  const size_t g = (size_t)d->B * d->S * 4;
  if (generated) {
    if (from_device) CE_CUDA_TRY(cudaMemcpy(generated, d->d_generated, g, cudaMemcpyDeviceToHost));
    else memcpy(generated, d->h_generated, g);
  }
  if (normalized)
    CE_CUDA_TRY(cudaMemcpy(normalized, d->d_normalized, (size_t)d->S * d->B * d->W * 4, cudaMemcpyDeviceToHost));
  if (logits)
    CE_CUDA_TRY(cudaMemcpy(logits, d->d_logits, (size_t)d->S * d->B * d->V * 4, cudaMemcpyDeviceToHost));
  if (probabilities)
    CE_CUDA_TRY(cudaMemcpy(probabilities, d->d_probabilities, (size_t)d->S * d->B * d->V * 4,
                           cudaMemcpyDeviceToHost));
  return CE_OK;
}

// Host-side overwrite of one output after the download, the reference's
// test hook (decoder.cu:346-358, --set fault=1|2|3): 1 flips the last
// generated token's low bit in the pinned buffer. Faults 2 and 3 corrupt
// diagnostics the caller holds on the host (see the Python mirror).
int ce_decoder_inject_fault(ce_decoder *d, int fault) {
  CE_REQUIRE(d != nullptr, "null decoder");
  CE_REQUIRE(fault >= 0 && fault <= 3, "fault must be 0, 1, 2 or 3 (got %d)", fault);
  if (fault == 1) d->h_generated[d->B * d->S - 1] ^= 1;
  return CE_OK;
}

}  // extern "C"
