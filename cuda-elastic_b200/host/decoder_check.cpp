// See decoder_check.h. Tolerances (contract.json "tolerances", oracle.cpp:23-29):
// normalized and logits within 2e-6 relative, probabilities within 2e-5
// relative, each plus 1e-12 absolute, of the double results; mean square of
// the normalized row within 2e-5 + 1.2e-7 * width of 1 and probability sum
// within 1e-6 + 1.2e-7 * vocab of 1 (float, summed in double); NaN fails.
#include "decoder_check.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <thread>

namespace ce_host {
namespace {

constexpr double kRelNormalized = 2.0e-6, kRelLogit = 2.0e-6, kRelProbability = 2.0e-5;
constexpr double kFloor = 1.0e-12;
constexpr long long kReported = 8;

// Runs body(i) for i in [0, n) on the host's threads, in chunks.
template <class F>
void parallel(long long n, F body) {
  unsigned hw = std::thread::hardware_concurrency();
  const long long threads = std::max<long long>(1, std::min<long long>({hw ? hw : 1, 64, n}));
  std::atomic<long long> next{0};
  const long long chunk = std::max<long long>(1, n / (threads * 8));
  std::vector<std::thread> pool;
  for (long long t = 0; t < threads; ++t)
    pool.emplace_back([&] {
      for (long long lo; (lo = next.fetch_add(chunk)) < n;)
        for (long long i = lo; i < std::min(n, lo + chunk); ++i) body(i);
    });
  for (auto &th : pool) th.join();
}

// The synthetic model (contract.json "data_generation").
inline double embedding_at(long long token, long long column) { return column == token ? 4.0 : 1.0; }
inline double classifier_at(long long row, long long column, long long vocab) {
  return column == (row + vocab - 1) % vocab ? 1.0 : 0.0;
}

bool near(double observed, double expected, double rel) {
  return std::fabs(observed - expected) <= rel * std::fabs(expected) + kFloor;  // NaN fails
}

}  // namespace

DecoderExpect decoder_expect(const DecoderShape &sh) {
  const long long B = sh.batch, W = sh.width, V = sh.vocab, S = sh.steps;
  DecoderExpect ex;
  ex.tokens.resize((size_t)(B * S));
  for (long long b = 0; b < B; ++b)
    for (long long s = 0, t = b % V; s < S; ++s) {
      t = (t + 1) % V;
      ex.tokens[(size_t)(b * S + s)] = (int32_t)t;
    }
  const long long n = std::min<long long>(8, B);
  for (long long i = 0; i < n; ++i) {
    const long long b = n == 1 ? 0 : i * (B - 1) / (n - 1);
    if (ex.sampled.empty() || ex.sampled.back() != b) ex.sampled.push_back(b);
  }
  const size_t m = ex.sampled.size();
  ex.normalized.resize(m * S * W);
  ex.logits.resize(m * S * V);
  ex.probabilities.resize(m * S * V);
  for (size_t i = 0; i < m; ++i) {
    long long token = ex.sampled[i] % V;
    for (long long s = 0; s < S; ++s) {
      double *o = &ex.normalized[(i * S + s) * W];
      double *l = &ex.logits[(i * S + s) * V];
      double *p = &ex.probabilities[(i * S + s) * V];
      double ss = 0.0;
      for (long long j = 0; j < W; ++j) ss += embedding_at(token, j) * embedding_at(token, j);
      const double scale = 1.0 / std::sqrt(ss / (double)W + 1.0e-5);
      for (long long j = 0; j < W; ++j) o[j] = 1.0 * (scale * embedding_at(token, j));
      // every classifier row against every column
      parallel(V, [&](long long r) {
        double acc = 0.0;
        for (long long j = 0; j < W; ++j) acc += classifier_at(r, j, V) * o[j];
        l[r] = acc;
      });
      const double mx = *std::max_element(l, l + V);
      double total = 0.0;
      for (long long r = 0; r < V; ++r) total += (p[r] = std::exp(l[r] - mx));
      long long best = 0;
      for (long long r = 0; r < V; ++r) {
        p[r] /= total;
        if (p[r] > p[best]) best = r;
      }
      if (best != (token + 1) % V) ex.consistent = false;
      token = best;
    }
  }
  if (!ex.consistent)
    std::fprintf(stderr, "decoder oracle: dense evaluation disagrees with the analytic token progression\n");
  return ex;
}

bool decoder_check(const DecoderShape &sh, const DecoderExpect &ex, const int32_t *generated,
                   const float *normalized, const float *logits, const float *probabilities) {
  const long long B = sh.batch, W = sh.width, V = sh.vocab, S = sh.steps;

  long long token_bad = 0;
  for (long long b = 0; b < B; ++b)
    for (long long s = 0; s < S; ++s) {
      const size_t k = (size_t)(b * S + s);
      if (generated[k] == ex.tokens[k]) continue;
      if (token_bad++ < kReported)
        std::fprintf(stderr, "decoder: token mismatch sequence %lld step %lld: expected %d, actual %d\n", b,
                     s, ex.tokens[k], generated[k]);
    }

  // per (step, sequence): float mean square and float probability sum
  const float sq_bound = 2.0e-5f + 1.2e-7f * (float)W;
  const float p_bound = 1.0e-6f + 1.2e-7f * (float)V;
  std::vector<float> sq_mean((size_t)(S * B)), p_sum((size_t)(S * B));
  parallel(S * B, [&](long long row) {
    const float *o = normalized + (size_t)row * W;
    const float *p = probabilities + (size_t)row * V;
    double q = 0.0, t = 0.0;
    for (long long j = 0; j < W; ++j) q += (double)o[j] * (double)o[j];
    for (long long r = 0; r < V; ++r) t += (double)p[r];
    sq_mean[(size_t)row] = (float)(q / (double)W);
    p_sum[(size_t)row] = (float)t;
  });
  long long inv_bad = 0;
  float worst_sq = 0.0f, worst_p = 0.0f;
  for (long long s = 0; s < S; ++s)
    for (long long b = 0; b < B; ++b) {
      const size_t row = (size_t)(s * B + b);
      const float e_sq = std::fabs(sq_mean[row] - 1.0f), e_p = std::fabs(p_sum[row] - 1.0f);
      const bool ok_sq = e_sq <= sq_bound, ok_p = e_p <= p_bound;
      if (ok_sq) worst_sq = std::max(worst_sq, e_sq);
      if (ok_p) worst_p = std::max(worst_p, e_p);
      if (ok_sq && ok_p) continue;
      if (inv_bad++ < kReported)
        std::fprintf(stderr,
                     "decoder: invariant failure sequence %lld step %lld: mean square expected 1 +- %.3g, "
                     "actual %.9g; probability sum expected 1 +- %.3g, actual %.9g\n",
                     b, s, sq_bound, sq_mean[row], p_bound, p_sum[row]);
    }

  long long dense_bad = 0;
  double worst[3] = {0.0, 0.0, 0.0};
  auto compare = [&](const char *what, int kind, long long b, long long s, long long idx, float got,
                     double want, double rel) {
    if (near(got, want, rel)) {
      worst[kind] = std::max(worst[kind], std::fabs(got - want) / std::max(std::fabs(want), kFloor));
      return;
    }
    if (dense_bad++ < kReported)
      std::fprintf(stderr, "decoder: %s mismatch sequence %lld step %lld index %lld: expected %.9g, actual %.9g\n",
                   what, b, s, idx, want, (double)got);
  };
  for (size_t i = 0; i < ex.sampled.size(); ++i) {
    const long long b = ex.sampled[i];
    for (long long s = 0; s < S; ++s) {
      const size_t at = (size_t)(s * B + b);
      const double *eo = &ex.normalized[(i * S + s) * W];
      const double *el = &ex.logits[(i * S + s) * V];
      const double *ep = &ex.probabilities[(i * S + s) * V];
      for (long long j = 0; j < W; ++j)
        compare("normalized", 0, b, s, j, normalized[at * W + j], eo[j], kRelNormalized);
      for (long long r = 0; r < V; ++r) {
        compare("logit", 1, b, s, r, logits[at * V + r], el[r], kRelLogit);
        compare("probability", 2, b, s, r, probabilities[at * V + r], ep[r], kRelProbability);
      }
    }
  }

  const bool pass = ex.consistent && token_bad == 0 && inv_bad == 0 && dense_bad == 0;
  std::fprintf(stderr,
               "decoder: %s: %lld/%lld tokens wrong; %lld/%lld (sequence, step) invariant failures "
               "(worst passing |mean square - 1| %.3g, |probability sum - 1| %.3g); dense check of %zu "
               "sequences x %lld steps: %lld mismatches (worst passing relative error normalized %.3g, "
               "logits %.3g, probabilities %.3g)\n",
               pass ? "PASS" : "FAIL", token_bad, B * S, inv_bad, B * S, (double)worst_sq, (double)worst_p,
               ex.sampled.size(), S, dense_bad, worst[0], worst[1], worst[2]);
  return pass;
}

}  // namespace ce_host
