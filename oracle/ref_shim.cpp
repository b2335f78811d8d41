// ref_shim.cpp -- extern "C" wrappers that expose the reference's own host
// code, compiled unmodified from its source tree, to the tests. TEST
// INFRASTRUCTURE ONLY: built into oracle/_ref/libref.so by oracle/Makefile
// when the reference tree is present, and used to pin the oracle.
//
// Wrapped reference code (paths relative to the reference project root):
//   llama2c/llama2c_common.h                     fill_inputs, validate_all
//   applications/loom_private/decoder/oracle.cpp  decoder_oracle::compute/check
//   experiments/blackwell/lowprec/reference.cpp   lowprec_ref::*
#include <cstdint>
#include <chrono>
#include <cstring>
#include <vector>

#include "llama2c_common.h"
#include "oracle.h"
#include "reference.h"

extern "C" {

void ref_fill_inputs(int random, uint64_t seed, int batch, int size, int rows, float *input,
                     float *probabilities, float *weight, float *matrix) {
  InputOptions o;
  o.random = random != 0;
  o.seed = seed;
  std::vector<float> in, pr, w, m;
  fill_inputs(o, batch, size, rows, &in, &pr, &w, &m);
  std::memcpy(input, in.data(), in.size() * 4);
  std::memcpy(probabilities, pr.data(), pr.size() * 4);
  std::memcpy(weight, w.data(), w.size() * 4);
  std::memcpy(matrix, m.data(), m.size() * 4);
}

// validate_all on given inputs/outputs; fills the per-row tolerance and
// double reference of the product. Returns 1 when valid.
int ref_validate_all(int random, uint64_t seed, const float *input, const float *probabilities,
                     const float *weight, const float *matrix, const float *normalized,
                     const float *softmax, const float *product, int batch, int size, int rows,
                     float *tolerance, double *reference) {
  InputOptions o;
  o.random = random != 0;
  o.seed = seed;
  const size_t vec = (size_t)batch * size, mat = (size_t)rows * size;
  std::vector<float> tol;
  std::vector<double> ref;
  const bool ok = validate_all(
      o, std::vector<float>(input, input + vec), std::vector<float>(probabilities, probabilities + vec),
      std::vector<float>(weight, weight + size), std::vector<float>(matrix, matrix + mat),
      std::vector<float>(normalized, normalized + vec), std::vector<float>(softmax, softmax + vec),
      std::vector<float>(product, product + rows), batch, size, rows, &tol, &ref);
  if (tolerance) std::memcpy(tolerance, tol.data(), rows * 4);
  if (reference) std::memcpy(reference, ref.data(), rows * 8);
  return ok ? 1 : 0;
}

// validate_all timed: the input and output vectors are built once, then
// validate_all runs `reps` times; returns the mean wall seconds per call and
// sets *valid. This is the reference's own CPU path of the llama2c iteration
// (validate_outputs_reference: double rmsnorm, softmax and GEMV with its
// checks, llama2c/llama2c_common.h:237-319), single-threaded as shipped.
double ref_time_validate_all(int random, uint64_t seed, const float *input, const float *probabilities,
                             const float *weight, const float *matrix, const float *normalized,
                             const float *softmax, const float *product, int batch, int size, int rows,
                             int reps, int *valid) {
  InputOptions o;
  o.random = random != 0;
  o.seed = seed;
  const size_t vec = (size_t)batch * size, mat = (size_t)rows * size;
  const std::vector<float> in(input, input + vec), pr(probabilities, probabilities + vec),
      w(weight, weight + size), m(matrix, matrix + mat), nz(normalized, normalized + vec),
      sm(softmax, softmax + vec), pd(product, product + rows);
  std::vector<float> tol;
  std::vector<double> ref;
  bool ok = true;
  const auto t0 = std::chrono::steady_clock::now();
  for (int r = 0; r < reps; ++r) ok = validate_all(o, in, pr, w, m, nz, sm, pd, batch, size, rows, &tol, &ref) && ok;
  const auto t1 = std::chrono::steady_clock::now();
  if (valid) *valid = ok ? 1 : 0;
  return std::chrono::duration<double>(t1 - t0).count() / (reps > 0 ? reps : 1);
}

double ref_gamma_probabilistic(int n) { return llama2c_gamma_probabilistic(n); }

int ref_write_dump(const char *path, int random, uint64_t seed, int batch, int size, int rows,
                   const float *normalized, const float *softmax, const float *product,
                   const float *tolerance, const double *reference) {
  InputOptions o;
  o.random = random != 0;
  o.seed = seed;
  return write_dump(path, o, batch, size, rows, normalized, softmax, product,
                    std::vector<float>(tolerance, tolerance + rows),
                    std::vector<double>(reference, reference + rows)) ? 1 : 0;
}

// Decoder oracle: tokens [batch][steps] and the sampled dense references.
int ref_decoder_compute(long long batch, long long width, long long vocab, long long steps,
                        int32_t *tokens, long long *sampled, int *n_sampled, double *normalized,
                        double *logits, double *probabilities) {
  const decoder_oracle::Shape shape{batch, width, vocab, steps};
  const decoder_oracle::Reference r = decoder_oracle::compute(shape);
  std::memcpy(tokens, r.tokens.data(), r.tokens.size() * 4);
  *n_sampled = (int)r.sampled.size();
  for (size_t i = 0; i < r.sampled.size(); ++i) sampled[i] = r.sampled[i];
  if (normalized) std::memcpy(normalized, r.normalized.data(), r.normalized.size() * 8);
  if (logits) std::memcpy(logits, r.logits.data(), r.logits.size() * 8);
  if (probabilities) std::memcpy(probabilities, r.probabilities.data(), r.probabilities.size() * 8);
  return r.self_consistent ? 1 : 0;
}

int ref_decoder_check(long long batch, long long width, long long vocab, long long steps,
                      const int32_t *tokens, const float *normalized, const float *logits,
                      const float *probabilities) {
  const decoder_oracle::Shape shape{batch, width, vocab, steps};
  const decoder_oracle::Reference r = decoder_oracle::compute(shape);
  const decoder_oracle::Observed obs{tokens, normalized, logits, probabilities};
  return decoder_oracle::check(shape, r, obs) ? 1 : 0;
}

// lowprec formats: 0 E2M1, 1 E3M2, 2 UE4M3, 3 UE8M0 (lowprec_ref::Format).
double ref_decode(int format, unsigned code) {
  return lowprec_ref::decode((lowprec_ref::Format)format, code);
}
unsigned ref_encode(int format, double v) {
  return lowprec_ref::encode((lowprec_ref::Format)format, v);
}
uint16_t ref_to_bf16(float v) { return lowprec_ref::to_bf16(v); }
void ref_quantize_mxfp6(const float *row, long long width, uint8_t *codes, uint8_t *scales) {
  lowprec_ref::quantize_mxfp6(row, width, codes, scales);
}
void ref_quantize_nvfp4(const float *row, long long width, float s, uint8_t *codes,
                        uint8_t *scales) {
  lowprec_ref::quantize_nvfp4(row, width, s, codes, scales);
}
float ref_nvfp4_encode_scale(float amax) { return lowprec_ref::nvfp4_encode_scale(amax); }
void ref_make_fixture(int seed, long long width, long long vocab, float *embedding,
                      float *classifier) {
  const lowprec_ref::Fixture f = lowprec_ref::make_fixture(seed, width, vocab);
  std::memcpy(embedding, f.embedding.data(), f.embedding.size() * 4);
  std::memcpy(classifier, f.classifier.data(), f.classifier.size() * 4);
}
void ref_rmsnorm_float(const float *x, long long width, float *out) {
  lowprec_ref::rmsnorm_float(x, width, out);
}

}  // extern "C"
