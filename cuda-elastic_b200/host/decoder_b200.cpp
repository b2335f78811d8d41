// decoder_b200: drop-in for the reference's loom_private decoder executable
// (applications/loom_private/decoder/decoder.cu:200-412 on the harness of
// common/lp_harness.cuh): batched greedy decoding of the synthetic llama2c
// model, rmsnorm -> dense fp32 classifier -> softmax + argmax with the token
// fed back on the device, computed by libce_b200's decoder (ce_decoder_*,
// include/ce_b200.h) under the fp32 arithmetic contract, so its digest is
// bitwise the reference's.
//
//   decoder_b200 [--preset large] [--launch direct|graph|both]
//                [--action check|bench|profile] [--iterations N] [--warmup W]
//                [--set batch|width|vocab|steps|fault=N]... [--json-out PATH]
//
// Exit codes: 0 pass, 1 output mismatch, 2 usage or invalid dimensions,
// 70 CUDA error. --set fault=1|2|3 (check only) corrupts one host output after
// the download (decoder.cu:346-358) so a test can confirm the check rejects it.
#include <cstring>
#include <vector>

#include "ce_b200.h"
#include "decoder_check.h"
#include "lp_front.h"

namespace {

using lp_front::ce_or_die;
using lp_front::Fields;
using lp_front::json_int;

// The large preset (contract.json "large").
constexpr long long kBatch = 1024, kWidth = 16384, kVocab = 8192, kSteps = 4;

// sha256 of applications/loom_private/decoder/contract.json, the contract this
// executable implements (the reference records the same in its result).
constexpr const char *kContractSha256 = "847d3367d564ef22250df7f929c1871067c0ac048f92429d03a7e4f15165340d";

class DecoderApp final : public lp_front::App {
 public:
  DecoderApp(long long b, long long w, long long v, long long s, int fault)
      : sh_{b, w, v, s}, fault_(fault) {}
  ~DecoderApp() override { ce_decoder_destroy(dec_); }

  std::string identity() const override { return "loom-private/llama2c-decoder"; }
  Fields dimensions() const override {
    return {{"batch", json_int(sh_.batch)},
            {"width", json_int(sh_.width)},
            {"vocab", json_int(sh_.vocab)},
            {"steps", json_int(sh_.steps)},
            {"generated_tokens", json_int(sh_.batch * sh_.steps)},
            {"classifier_macs_per_step", json_int(sh_.batch * sh_.vocab * sh_.width)},
            {"model_bytes", json_int((2 * sh_.vocab * sh_.width + sh_.width) * 4)}};
  }
  std::string application_scope() const override {
    return "pinned prompt upload (batch int32), device token reset, every step (gathered rmsnorm, "
           "fp32 contract classifier GEMM, softmax + first argmax feeding the next token), pinned "
           "download of the generated tokens (batch x steps int32); model and buffers resident";
  }
  std::string compute_scope() const override {
    return "device token reset from the resident prompts and every step (gathered rmsnorm, fp32 "
           "contract classifier GEMM, softmax + first argmax)";
  }

  void setup(void *stream) override {
    ce_or_die(ce_decoder_create(&dec_, sh_.batch, sh_.width, sh_.vocab, sh_.steps, CE_PREC_FP32, (ce_stream_t)stream),
              "ce_decoder_create");
    generated_.resize((size_t)(sh_.batch * sh_.steps));
    normalized_.resize((size_t)(sh_.steps * sh_.batch * sh_.width));
    logits_.resize((size_t)(sh_.steps * sh_.batch * sh_.vocab));
    probabilities_.resize(logits_.size());
  }
  void enqueue(void *stream, bool compute_only) override {
    if (compute_only) ce_or_die(ce_decoder_enqueue_compute(dec_, (ce_stream_t)stream), "ce_decoder_enqueue_compute");
    else ce_or_die(ce_decoder_enqueue_application(dec_, (ce_stream_t)stream), "ce_decoder_enqueue_application");
  }
  void poison(void *stream) override {
    ce_or_die(ce_decoder_poison(dec_, (ce_stream_t)stream), "ce_decoder_poison");
    std::memset(generated_.data(), 0xFF, generated_.size() * 4);
    std::memset(normalized_.data(), 0xFF, normalized_.size() * 4);
    std::memset(logits_.data(), 0xFF, logits_.size() * 4);
    std::memset(probabilities_.data(), 0xFF, probabilities_.size() * 4);
  }
  void reference() override { expect_ = ce_host::decoder_expect(sh_); }
  bool check() override {
    ce_or_die(ce_decoder_copy_outputs(dec_, 0, nullptr, normalized_.data(), logits_.data(),
                                      probabilities_.data()),
              "ce_decoder_copy_outputs");
    ce_or_die(ce_decoder_inject_fault(dec_, fault_ == 1 ? 1 : 0), "ce_decoder_inject_fault");
    pull_generated();
    const long long last = sh_.steps - 1;
    if (fault_ == 2) normalized_[(size_t)((last * sh_.batch + sh_.batch / 2) * sh_.width)] *= 2.0f;
    if (fault_ == 3) probabilities_[(size_t)(last * sh_.batch * sh_.vocab + sh_.vocab / 2)] *= 1.001f;
    return ce_host::decoder_check(sh_, expect_, generated_.data(), normalized_.data(), logits_.data(),
                                  probabilities_.data());
  }
  uint64_t digest() override {
    pull_generated();
    uint64_t h = lp_front::fnv1a64(generated_.data(), generated_.size() * 4);
    h = lp_front::fnv1a64(normalized_.data(), normalized_.size() * 4, h);
    h = lp_front::fnv1a64(logits_.data(), logits_.size() * 4, h);
    return lp_front::fnv1a64(probabilities_.data(), probabilities_.size() * 4, h);
  }

 private:
  // generated as the last application scope downloaded it (pinned buffer)
  void pull_generated() {
    ce_or_die(ce_decoder_copy_outputs(dec_, 0, generated_.data(), nullptr, nullptr, nullptr),
              "ce_decoder_copy_outputs");
  }

  ce_host::DecoderShape sh_;
  int fault_;
  ce_decoder *dec_ = nullptr;
  std::vector<int32_t> generated_;
  std::vector<float> normalized_, logits_, probabilities_;
  ce_host::DecoderExpect expect_;
};

lp_front::App *make_decoder(lp_front::Options &o) {
  const long long batch = o.integer("batch", kBatch);
  const long long width = o.integer("width", kWidth);
  const long long vocab = o.integer("vocab", kVocab);
  const long long steps = o.integer("steps", kSteps);
  const long long fault = o.integer("fault", 0);
  if (o.preset != "large") return nullptr;
  ce_or_die(ce_decoder_validate(batch, width, vocab, steps, CE_PREC_FP32), "ce_decoder_validate");
  if (fault < 0 || fault > 3) lp_front::die(lp_front::kUsage, "fault must be 0, 1, 2 or 3 (got %lld)", fault);
  return new DecoderApp(batch, width, vocab, steps, (int)fault);
}

}  // namespace

int main(int argc, char **argv) {
  return lp_front::run(argc, argv, {"decoder", "b200", kContractSha256}, make_decoder);
}
