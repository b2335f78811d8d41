// llama2c_b200: drop-in for the reference's llama2c_cuda_graph / llama2c_sota
// executables (llama2c/llama2c_cuda_graph.cu:178-540, llama2c_sota.cu), with
// the same command line, the same key=value result line and the same dump,
// computing through libce_b200 (include/ce_b200.h).
//
//   llama2c_b200 [graph|direct] [launches|auto] [batch] [size] [rows] [repeats]
//                [warmup_ms] [copy|nocopy] [naive|coalesced] [fused|streams]
//                [deterministic|random[=SEED]] [--dump=FILE]
//
// Tokens are order-free; the integers are positional, as in the reference
// (parse_options, llama2c_cuda_graph.cu:211-258); LLAMA2C_DUMP names the dump
// when --dump is absent. "fused" (default) runs the iteration as one launch
// (ce_llama2c_iteration, the SOTA layout); "streams" runs ce_rmsnorm,
// ce_softmax and ce_gemv on three forked streams (the baseline's layout).
// naive|coalesced are accepted for compatibility; both select the library's
// GEMV. Exit status 0 iff the outputs pass the reference's validation.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "ce_b200.h"
#include "llama2c_check.h"

namespace {

#define CUDA_CHECK(call)                                                              \
  do {                                                                                \
    cudaError_t e__ = (call);                                                         \
    if (e__ != cudaSuccess) {                                                         \
      std::fprintf(stderr, "%s failed: %s\n", #call, cudaGetErrorString(e__));        \
      std::exit(EXIT_FAILURE);                                                        \
    }                                                                                 \
  } while (0)

#define CE_CHECK(call)                                                                \
  do {                                                                                \
    int rc__ = (call);                                                                \
    if (rc__ != CE_OK) {                                                              \
      char msg__[512];                                                                \
      ce_last_error(msg__, sizeof msg__);                                             \
      std::fprintf(stderr, "%s failed (%d): %s\n", #call, rc__, msg__);               \
      std::exit(EXIT_FAILURE);                                                        \
    }                                                                                 \
  } while (0)

constexpr float kRmsEpsilon = 1.0e-5f;
constexpr double kAutoTargetMs = 50.0;
constexpr int kAutoMinLaunches = 20, kAutoMaxLaunches = 5000, kSingleIterations = 20;

struct Options {
  bool graph = true;
  int launches = 180;
  int batch = 512, size = 16384, rows = 8192, repeats = 1, warmup_ms = 100;
  bool copy_outputs = true;
  bool coalesced = false;
  bool fused = true;
  bool auto_launches = false;
  bool random = false;
  uint64_t seed = 0;
  std::string dump_path;
};

void usage(const char *prog) {
  std::fprintf(stderr,
               "Usage: %s [graph|direct] [launches|auto] [batch] [size] [rows] [repeats] [warmup_ms]"
               " [copy|nocopy] [naive|coalesced] [fused|streams] [deterministic|random[=SEED]]"
               " [--dump=FILE]\n",
               prog);
}

bool positive_int(const char *text, int *value) {
  char *end = nullptr;
  const long v = std::strtol(text, &end, 10);
  if (*text == '\0' || *end != '\0' || v <= 0 || v > INT_MAX) return false;
  *value = (int)v;
  return true;
}

bool parse(int argc, char **argv, Options *o) {
  int positional = 0;
  for (int i = 1; i < argc; ++i) {
    const char *a = argv[i];
    if (!std::strcmp(a, "deterministic")) { o->random = false; o->seed = 0; continue; }
    if (!std::strcmp(a, "random")) { o->random = true; o->seed = 1; continue; }
    if (!std::strncmp(a, "random=", 7)) {
      char *end = nullptr;
      const unsigned long long s = std::strtoull(a + 7, &end, 10);
      if (a[7] == '\0' || *end != '\0') {
        std::fprintf(stderr, "bad seed in '%s'\n", a);
        std::exit(EXIT_FAILURE);
      }
      o->random = true;
      o->seed = s;
      continue;
    }
    if (!std::strncmp(a, "--dump=", 7)) { o->dump_path = a + 7; continue; }
    if (!std::strcmp(a, "graph")) { o->graph = true; continue; }
    if (!std::strcmp(a, "direct")) { o->graph = false; continue; }
    if (!std::strcmp(a, "nocopy")) { o->copy_outputs = false; continue; }
    if (!std::strcmp(a, "copy")) { o->copy_outputs = true; continue; }
    if (!std::strcmp(a, "naive")) { o->coalesced = false; continue; }
    if (!std::strcmp(a, "coalesced")) { o->coalesced = true; continue; }
    if (!std::strcmp(a, "fused")) { o->fused = true; continue; }
    if (!std::strcmp(a, "streams")) { o->fused = false; continue; }
    if (positional == 0 && !std::strcmp(a, "auto")) {
      o->auto_launches = true;
      ++positional;
      continue;
    }
    int *dst = nullptr;
    if (positional == 0) dst = &o->launches;
    if (positional == 1) dst = &o->batch;
    if (positional == 2) dst = &o->size;
    if (positional == 3) dst = &o->rows;
    if (positional == 4) dst = &o->repeats;
    if (positional == 5) dst = &o->warmup_ms;
    if (dst == nullptr || !positive_int(a, dst)) return false;
    ++positional;
  }
  const char *env = std::getenv("LLAMA2C_DUMP");
  if (env && *env && o->dump_path.empty()) o->dump_path = env;
  return true;
}

double ms_since(std::chrono::steady_clock::time_point t) {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t).count();
}

}  // namespace

int main(int argc, char **argv) {
  Options o;
  if (!parse(argc, argv, &o)) {
    usage(argv[0]);
    return EXIT_FAILURE;
  }
  const size_t vec = (size_t)o.batch * o.size, mat = (size_t)o.rows * o.size;
  std::vector<float> h_input(vec), h_prob(vec), h_weight(o.size), h_matrix(mat);
  CE_CHECK(ce_fill_llama2c_host(o.random ? 1 : 0, o.seed, o.batch, o.size, o.rows, h_input.data(),
                                h_prob.data(), h_weight.data(), h_matrix.data()));
  float *d_input, *d_weight, *d_prob, *d_softmax, *d_matrix, *d_norm, *d_product;
  CUDA_CHECK(cudaMalloc(&d_input, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_weight, (size_t)o.size * 4));
  CUDA_CHECK(cudaMalloc(&d_prob, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_softmax, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_matrix, mat * 4));
  CUDA_CHECK(cudaMalloc(&d_norm, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_product, (size_t)o.rows * 4));
  CUDA_CHECK(cudaMemcpy(d_input, h_input.data(), vec * 4, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_weight, h_weight.data(), (size_t)o.size * 4, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_prob, h_prob.data(), vec * 4, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_matrix, h_matrix.data(), mat * 4, cudaMemcpyHostToDevice));
  float *h_norm, *h_softmax, *h_product;
  CUDA_CHECK(cudaMallocHost(&h_norm, vec * 4));
  CUDA_CHECK(cudaMallocHost(&h_softmax, vec * 4));
  CUDA_CHECK(cudaMallocHost(&h_product, (size_t)o.rows * 4));

  cudaStream_t s0, s1, s2;
  CUDA_CHECK(cudaStreamCreateWithFlags(&s0, cudaStreamNonBlocking));
  CUDA_CHECK(cudaStreamCreateWithFlags(&s1, cudaStreamNonBlocking));
  CUDA_CHECK(cudaStreamCreateWithFlags(&s2, cudaStreamNonBlocking));
  cudaEvent_t fork, join1, join2;
  CUDA_CHECK(cudaEventCreateWithFlags(&fork, cudaEventDisableTiming));
  CUDA_CHECK(cudaEventCreateWithFlags(&join1, cudaEventDisableTiming));
  CUDA_CHECK(cudaEventCreateWithFlags(&join2, cudaEventDisableTiming));
  const ce_stream_t c0 = (ce_stream_t)s0, c1 = (ce_stream_t)s1, c2 = (ce_stream_t)s2;

  // Minimum device traffic per iteration (llama2c_cuda_graph.cu:340-345).
  const double vector_bytes = (double)vec * 4;
  const double min_bytes = o.repeats * (2.0 * vector_bytes + o.size * 4.0 + 2.0 * vector_bytes +
                                        (double)mat * 4 + ((double)o.size + o.rows) * 4);

  // Fused layout: one launch per repeat. In copy mode the last repeat is
  // split (llama2c_sota.cu:477-496): the rmsnorm rows run alone on s0 and
  // their copy to the host starts at once, while softmax + GEMV run as a
  // second launch on s1 followed by their copies; s0 joins s1 before the
  // iteration ends. Streams layout: three forked streams, one op each.
  auto enqueue_iteration = [&]() {
    if (!o.fused) {
      CUDA_CHECK(cudaEventRecord(fork, s0));
      CUDA_CHECK(cudaStreamWaitEvent(s1, fork, 0));
      CUDA_CHECK(cudaStreamWaitEvent(s2, fork, 0));
    }
    for (int r = 0; r < o.repeats; ++r) {
      const bool last_copy = r + 1 == o.repeats && o.copy_outputs;
      if (o.fused && !last_copy) {
        CE_CHECK(ce_llama2c_iteration(d_norm, d_softmax, d_product, d_input, d_weight, d_prob,
                                      d_matrix, o.batch, o.size, o.rows, kRmsEpsilon, c0));
      } else if (o.fused) {
        CUDA_CHECK(cudaEventRecord(fork, s0));
        CUDA_CHECK(cudaStreamWaitEvent(s1, fork, 0));
        CE_CHECK(ce_llama2c_rows(d_norm, nullptr, nullptr, d_input, d_weight, nullptr, nullptr,
                                 o.size, o.batch, 0, 0, kRmsEpsilon, c0));
        CUDA_CHECK(cudaMemcpyAsync(h_norm, d_norm, vec * 4, cudaMemcpyDeviceToHost, s0));
        CE_CHECK(ce_llama2c_rows(nullptr, d_softmax, d_product, d_input, nullptr, d_prob,
                                 d_matrix, o.size, 0, o.batch, o.rows, kRmsEpsilon, c1));
        CUDA_CHECK(cudaMemcpyAsync(h_softmax, d_softmax, vec * 4, cudaMemcpyDeviceToHost, s1));
        CUDA_CHECK(cudaMemcpyAsync(h_product, d_product, (size_t)o.rows * 4,
                                   cudaMemcpyDeviceToHost, s1));
        CUDA_CHECK(cudaEventRecord(join1, s1));
        CUDA_CHECK(cudaStreamWaitEvent(s0, join1, 0));
      } else {
        CE_CHECK(ce_rmsnorm(d_norm, d_input, d_weight, o.batch, o.size, kRmsEpsilon, c0));
        CE_CHECK(ce_softmax(d_softmax, d_prob, o.batch, o.size, c1));
        CE_CHECK(ce_gemv(d_product, d_matrix, d_input, o.rows, o.size, c2));
        if (last_copy) {
          CUDA_CHECK(cudaMemcpyAsync(h_norm, d_norm, vec * 4, cudaMemcpyDeviceToHost, s0));
          CUDA_CHECK(cudaMemcpyAsync(h_softmax, d_softmax, vec * 4, cudaMemcpyDeviceToHost, s1));
          CUDA_CHECK(cudaMemcpyAsync(h_product, d_product, (size_t)o.rows * 4,
                                     cudaMemcpyDeviceToHost, s2));
        }
      }
    }
    if (!o.fused) {
      CUDA_CHECK(cudaEventRecord(join1, s1));
      CUDA_CHECK(cudaEventRecord(join2, s2));
      CUDA_CHECK(cudaStreamWaitEvent(s0, join1, 0));
      CUDA_CHECK(cudaStreamWaitEvent(s0, join2, 0));
    }
  };
  // Kernel launches per iteration (llama2c_sota.cu:475-476 for the fused
  // layout; three per repeat for the streams layout).
  const int kernels_per_iter =
      o.fused ? o.repeats + (o.copy_outputs ? 1 : 0) : 3 * o.repeats;

  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  double capture_ms = 0, instantiate_ms = 0, upload_ms = 0;
  if (o.graph) {
    auto t = std::chrono::steady_clock::now();
    CUDA_CHECK(cudaStreamBeginCapture(s0, cudaStreamCaptureModeGlobal));
    enqueue_iteration();
    CUDA_CHECK(cudaStreamEndCapture(s0, &graph));
    capture_ms = ms_since(t);
    t = std::chrono::steady_clock::now();
    CUDA_CHECK(cudaGraphInstantiate(&exec, graph, nullptr, nullptr, 0));
    instantiate_ms = ms_since(t);
    t = std::chrono::steady_clock::now();
    CUDA_CHECK(cudaGraphUpload(exec, s0));
    CUDA_CHECK(cudaStreamSynchronize(s0));
    upload_ms = ms_since(t);
  }
  auto launch = [&]() {
    if (o.graph) CUDA_CHECK(cudaGraphLaunch(exec, s0));
    else enqueue_iteration();
  };
  auto sync_all = [&]() {
    CUDA_CHECK(cudaStreamSynchronize(s0));
    CUDA_CHECK(cudaStreamSynchronize(s1));
    CUDA_CHECK(cudaStreamSynchronize(s2));
  };

  const auto warm_start = std::chrono::steady_clock::now();
  int warmup_iterations = 0;
  do {
    launch();
    sync_all();
    ++warmup_iterations;
  } while (ms_since(warm_start) < o.warmup_ms);
  if (o.auto_launches) {
    const double per = ms_since(warm_start) / warmup_iterations;
    o.launches = (int)std::fmin(kAutoMaxLaunches, std::fmax(kAutoMinLaunches, kAutoTargetMs / per));
  }

  cudaEvent_t t0, t1;
  CUDA_CHECK(cudaEventCreate(&t0));
  CUDA_CHECK(cudaEventCreate(&t1));
  CUDA_CHECK(cudaEventRecord(t0, s0));
  const auto wall_start = std::chrono::steady_clock::now();
  for (int i = 0; i < o.launches; ++i) launch();
  const double submit_us = ms_since(wall_start) * 1000.0;
  CUDA_CHECK(cudaEventRecord(t1, s0));
  sync_all();
  const double wall_ms = ms_since(wall_start);
  float gpu_ms = 0;
  CUDA_CHECK(cudaEventElapsedTime(&gpu_ms, t0, t1));
  std::vector<double> singles;
  for (int i = 0; i < kSingleIterations; ++i) {
    sync_all();
    CUDA_CHECK(cudaEventRecord(t0, s0));
    launch();
    CUDA_CHECK(cudaEventRecord(t1, s0));
    CUDA_CHECK(cudaEventSynchronize(t1));
    float ms = 0;
    CUDA_CHECK(cudaEventElapsedTime(&ms, t0, t1));
    singles.push_back(1000.0 * ms);
  }
  sync_all();
  std::sort(singles.begin(), singles.end());
  const double single_us = (singles[(kSingleIterations - 1) / 2] + singles[kSingleIterations / 2]) / 2.0;
  if (!o.copy_outputs) {
    CUDA_CHECK(cudaMemcpy(h_norm, d_norm, vec * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(h_softmax, d_softmax, vec * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(h_product, d_product, (size_t)o.rows * 4, cudaMemcpyDeviceToHost));
  }
  const int status = ce_device_status();
  ce_host::Llama2cCheck check = ce_host::validate_llama2c(
      o.random, h_input.data(), h_prob.data(), h_weight.data(), h_matrix.data(), h_norm, h_softmax,
      h_product, o.batch, o.size, o.rows);
  bool valid = check.valid && status == CE_OK;
  if (!valid) std::fprintf(stderr, "Output validation failed\n");
  if (!o.dump_path.empty() &&
      !ce_host::write_l2cdump1(o.dump_path, o.random, o.seed, o.batch, o.size, o.rows, h_norm,
                               h_softmax, h_product, check.product_tolerance, check.product_reference))
    valid = false;
  const double per_iter = gpu_ms / o.launches;
  // Waves = blocks / (resident blocks per SM x SMs), as the reference reports
  // them (llama2c_cuda_graph.cu:318-336), for this build's launch shapes: a
  // 64 KiB row per 512-thread block (two resident per SM), a GEMV block per
  // 16 matrix rows.
  int sms = 148, sm100 = 0;
  CE_CHECK(ce_device_info(&sms, &sm100));
  const double resident = 2.0 * sms;
  const double rms_waves = o.batch / resident, softmax_waves = o.batch / resident;
  const double matmul_waves = std::ceil(o.rows / 16.0) / resident;
  const double min_waves = std::fmin(rms_waves, std::fmin(softmax_waves, matmul_waves));
  std::printf(
      "mode=%s matmul=%s launches=%d batch=%d size=%d rows=%d repeats=%d copies=%d warmup_ms=%d "
      "warmup_iterations=%d gpu_ms=%.6f gpu_ms_per_iter=%.6f single_iterations=%d single_us=%.3f "
      "wall_ms=%.6f wall_ms_per_iter=%.6f submit_us=%.3f submit_us_per_iter=%.3f "
      "graph_capture_ms=%.6f graph_instantiate_ms=%.6f graph_upload_ms=%.6f rms_waves=%.3f "
      "softmax_waves=%.3f matmul_waves=%.3f min_waves=%.3f "
      "min_bytes_per_iter=%.0f achieved_gbps=%.1f valid=%d inputs=%s seed=%llu "
      "implementation=ce_b200 layout=%s kernels_per_iter=%d\n",
      o.graph ? "graph" : "direct", o.coalesced ? "coalesced" : "naive", o.launches, o.batch,
      o.size, o.rows, o.repeats, o.copy_outputs ? 1 : 0, o.warmup_ms, warmup_iterations, gpu_ms,
      per_iter, kSingleIterations, single_us, wall_ms, wall_ms / o.launches, submit_us,
      submit_us / o.launches, capture_ms, instantiate_ms, upload_ms, rms_waves, softmax_waves,
      matmul_waves, min_waves, min_bytes,
      min_bytes / (per_iter * 1.0e6), valid ? 1 : 0, o.random ? "random" : "deterministic",
      (unsigned long long)o.seed, o.fused ? "fused" : "streams", kernels_per_iter);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  cudaFreeHost(h_norm);
  cudaFreeHost(h_softmax);
  cudaFreeHost(h_product);
  for (void *p : {(void *)d_input, (void *)d_weight, (void *)d_prob, (void *)d_softmax,
                  (void *)d_matrix, (void *)d_norm, (void *)d_product})
    cudaFree(p);
  return valid ? EXIT_SUCCESS : EXIT_FAILURE;
}
