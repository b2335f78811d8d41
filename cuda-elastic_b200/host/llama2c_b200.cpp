// llama2c_b200: drop-in for the reference's llama2c_cuda_graph / llama2c_sota
// executables (llama2c/llama2c_cuda_graph.cu:178-540, llama2c_sota.cu), with
// the same command line, the same key=value result line and the same dump,
// computing through libce_b200 (include/ce_b200.h).
//
//   llama2c_b200 [graph|direct] [launches|auto] [batch] [size] [rows] [repeats]
//                [warmup_ms] [copy|nocopy] [naive|coalesced] [fused|streams]
//                [deterministic|random[=SEED]] [trio[=PRECISION]] [--dump=FILE]
//
// Tokens are order-free; the integers are positional, as in the reference
// (parse_options, llama2c_cuda_graph.cu:211-258); LLAMA2C_DUMP names the dump
// when --dump is absent. "fused" (default) runs the iteration as one launch
// (ce_llama2c_iteration, the SOTA layout); "streams" runs ce_rmsnorm,
// ce_softmax and ce_gemv on three forked streams (the baseline's layout).
// naive|coalesced are accepted for compatibility; both select the library's
// GEMV. "trio[=fp32|tf32|bf16|fp8|mxfp6|nvfp4]" (bf16 by default) runs the
// op trio instead -- rmsnorm -> GEMM of the normalized batch by W
// [rows][size] in that precision, plus a softmax -- through the op-trio
// plan (ce_plan_*), checked against the double product of the GEMM's own
// dequantized operands; its --dump writes L2CDUMP2 (llama2c_check.h).
// Exit status 0 iff the outputs pass the validation.
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
// op-trio rows whose GEMM outputs are checked value by value (spread evenly)
constexpr int kTrioCheckedRows = 64;

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
  bool trio = false;              // op-trio mode: rmsnorm -> GEMM + softmax
  int precision = CE_PREC_BF16;   // its GEMM precision
};

// trio=NAME precisions (CE_PREC_*).
struct PrecisionName {
  const char *name;
  int precision;
};
constexpr PrecisionName kPrecisions[] = {
    {"fp32", CE_PREC_FP32},      {"tf32", CE_PREC_TF32},          {"bf16", CE_PREC_BF16},
    {"fp8", CE_PREC_FP8_E4M3},   {"mxfp6", CE_PREC_MXFP6_E3M2},   {"nvfp4", CE_PREC_NVFP4_E2M1}};

const char *precision_name(int precision) {
  for (const auto &p : kPrecisions)
    if (p.precision == precision) return p.name;
  return "?";
}

void usage(const char *prog) {
  std::fprintf(stderr,
               "Usage: %s [graph|direct] [launches|auto] [batch] [size] [rows] [repeats] [warmup_ms]"
               " [copy|nocopy] [naive|coalesced] [fused|streams] [deterministic|random[=SEED]]"
               " [trio[=fp32|tf32|bf16|fp8|mxfp6|nvfp4]] [--dump=FILE]\n",
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
    if (!std::strcmp(a, "trio")) { o->trio = true; continue; }
    if (!std::strncmp(a, "trio=", 5)) {
      o->trio = true;
      bool known = false;
      for (const auto &p : kPrecisions)
        if (!std::strcmp(a + 5, p.name)) {
          o->precision = p.precision;
          known = true;
        }
      if (!known) {
        std::fprintf(stderr, "unknown precision in '%s' (fp32, tf32, bf16, fp8, mxfp6, nvfp4)\n", a);
        std::exit(EXIT_FAILURE);
      }
      continue;
    }
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

// The harness's streams: s0 carries every iteration (its start and end),
// s1 / s2 the forked work.
struct Streams {
  cudaStream_t s0, s1, s2;
  cudaEvent_t fork, join1, join2;
  Streams() {
    CUDA_CHECK(cudaStreamCreateWithFlags(&s0, cudaStreamNonBlocking));
    CUDA_CHECK(cudaStreamCreateWithFlags(&s1, cudaStreamNonBlocking));
    CUDA_CHECK(cudaStreamCreateWithFlags(&s2, cudaStreamNonBlocking));
    CUDA_CHECK(cudaEventCreateWithFlags(&fork, cudaEventDisableTiming));
    CUDA_CHECK(cudaEventCreateWithFlags(&join1, cudaEventDisableTiming));
    CUDA_CHECK(cudaEventCreateWithFlags(&join2, cudaEventDisableTiming));
  }
  void sync_all() const {
    CUDA_CHECK(cudaStreamSynchronize(s0));
    CUDA_CHECK(cudaStreamSynchronize(s1));
    CUDA_CHECK(cudaStreamSynchronize(s2));
  }
};

struct Timing {
  double capture_ms = 0, instantiate_ms = 0, upload_ms = 0;
  int warmup_iterations = 0;
  float gpu_ms = 0;
  double wall_ms = 0, submit_us = 0, single_us = 0;
};

// The reference's measurement protocol (llama2c_cuda_graph.cu:385-470): the
// iteration captured once into a graph (graph mode) or enqueued each time
// (direct), warm-up for warmup_ms (auto picks the launch count from it),
// `launches` back-to-back iterations between two events on s0, then the
// median of single timed iterations.
template <class Enqueue>
Timing run_iterations(Options &o, const Streams &st, Enqueue enqueue_iteration) {
  Timing t;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  if (o.graph) {
    auto c = std::chrono::steady_clock::now();
    CUDA_CHECK(cudaStreamBeginCapture(st.s0, cudaStreamCaptureModeGlobal));
    enqueue_iteration();
    CUDA_CHECK(cudaStreamEndCapture(st.s0, &graph));
    t.capture_ms = ms_since(c);
    c = std::chrono::steady_clock::now();
    CUDA_CHECK(cudaGraphInstantiate(&exec, graph, nullptr, nullptr, 0));
    t.instantiate_ms = ms_since(c);
    c = std::chrono::steady_clock::now();
    CUDA_CHECK(cudaGraphUpload(exec, st.s0));
    CUDA_CHECK(cudaStreamSynchronize(st.s0));
    t.upload_ms = ms_since(c);
  }
  auto launch = [&]() {
    if (o.graph) CUDA_CHECK(cudaGraphLaunch(exec, st.s0));
    else enqueue_iteration();
  };
  const auto warm_start = std::chrono::steady_clock::now();
  do {
    launch();
    st.sync_all();
    ++t.warmup_iterations;
  } while (ms_since(warm_start) < o.warmup_ms);
  if (o.auto_launches) {
    const double per = ms_since(warm_start) / t.warmup_iterations;
    o.launches = (int)std::fmin(kAutoMaxLaunches, std::fmax(kAutoMinLaunches, kAutoTargetMs / per));
  }
  cudaEvent_t t0, t1;
  CUDA_CHECK(cudaEventCreate(&t0));
  CUDA_CHECK(cudaEventCreate(&t1));
  CUDA_CHECK(cudaEventRecord(t0, st.s0));
  const auto wall_start = std::chrono::steady_clock::now();
  for (int i = 0; i < o.launches; ++i) launch();
  t.submit_us = ms_since(wall_start) * 1000.0;
  CUDA_CHECK(cudaEventRecord(t1, st.s0));
  st.sync_all();
  t.wall_ms = ms_since(wall_start);
  CUDA_CHECK(cudaEventElapsedTime(&t.gpu_ms, t0, t1));
  std::vector<double> singles;
  for (int i = 0; i < kSingleIterations; ++i) {
    st.sync_all();
    CUDA_CHECK(cudaEventRecord(t0, st.s0));
    launch();
    CUDA_CHECK(cudaEventRecord(t1, st.s0));
    CUDA_CHECK(cudaEventSynchronize(t1));
    float ms = 0;
    CUDA_CHECK(cudaEventElapsedTime(&ms, t0, t1));
    singles.push_back(1000.0 * ms);
  }
  st.sync_all();
  std::sort(singles.begin(), singles.end());
  t.single_us = (singles[(kSingleIterations - 1) / 2] + singles[kSingleIterations / 2]) / 2.0;
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  return t;
}

// The key=value fields every mode prints first, in the reference's order.
void print_common(const Options &o, const Timing &t) {
  std::printf(
      "mode=%s matmul=%s launches=%d batch=%d size=%d rows=%d repeats=%d copies=%d warmup_ms=%d "
      "warmup_iterations=%d gpu_ms=%.6f gpu_ms_per_iter=%.6f single_iterations=%d single_us=%.3f "
      "wall_ms=%.6f wall_ms_per_iter=%.6f submit_us=%.3f submit_us_per_iter=%.3f "
      "graph_capture_ms=%.6f graph_instantiate_ms=%.6f graph_upload_ms=%.6f ",
      o.graph ? "graph" : "direct", o.coalesced ? "coalesced" : "naive", o.launches, o.batch,
      o.size, o.rows, o.repeats, o.copy_outputs ? 1 : 0, o.warmup_ms, t.warmup_iterations,
      t.gpu_ms, t.gpu_ms / o.launches, kSingleIterations, t.single_us, t.wall_ms,
      t.wall_ms / o.launches, t.submit_us, t.submit_us / o.launches, t.capture_ms,
      t.instantiate_ms, t.upload_ms);
}

// The llama2c iteration (the reference harness's workload).
int run_llama2c(Options &o) {
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

  const Streams st;
  const cudaStream_t s0 = st.s0, s1 = st.s1, s2 = st.s2;
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
      CUDA_CHECK(cudaEventRecord(st.fork, s0));
      CUDA_CHECK(cudaStreamWaitEvent(s1, st.fork, 0));
      CUDA_CHECK(cudaStreamWaitEvent(s2, st.fork, 0));
    }
    for (int r = 0; r < o.repeats; ++r) {
      const bool last_copy = r + 1 == o.repeats && o.copy_outputs;
      if (o.fused && !last_copy) {
        CE_CHECK(ce_llama2c_iteration(d_norm, d_softmax, d_product, d_input, d_weight, d_prob,
                                      d_matrix, o.batch, o.size, o.rows, kRmsEpsilon, c0));
      } else if (o.fused) {
        CUDA_CHECK(cudaEventRecord(st.fork, s0));
        CUDA_CHECK(cudaStreamWaitEvent(s1, st.fork, 0));
        CE_CHECK(ce_llama2c_rows(d_norm, nullptr, nullptr, d_input, d_weight, nullptr, nullptr,
                                 o.size, o.batch, 0, 0, kRmsEpsilon, c0));
        CUDA_CHECK(cudaMemcpyAsync(h_norm, d_norm, vec * 4, cudaMemcpyDeviceToHost, s0));
        CE_CHECK(ce_llama2c_rows(nullptr, d_softmax, d_product, d_input, nullptr, d_prob,
                                 d_matrix, o.size, 0, o.batch, o.rows, kRmsEpsilon, c1));
        CUDA_CHECK(cudaMemcpyAsync(h_softmax, d_softmax, vec * 4, cudaMemcpyDeviceToHost, s1));
        CUDA_CHECK(cudaMemcpyAsync(h_product, d_product, (size_t)o.rows * 4,
                                   cudaMemcpyDeviceToHost, s1));
        CUDA_CHECK(cudaEventRecord(st.join1, s1));
        CUDA_CHECK(cudaStreamWaitEvent(s0, st.join1, 0));
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
      CUDA_CHECK(cudaEventRecord(st.join1, s1));
      CUDA_CHECK(cudaEventRecord(st.join2, s2));
      CUDA_CHECK(cudaStreamWaitEvent(s0, st.join1, 0));
      CUDA_CHECK(cudaStreamWaitEvent(s0, st.join2, 0));
    }
  };
  // Kernel launches per iteration (llama2c_sota.cu:475-476 for the fused
  // layout; three per repeat for the streams layout).
  const int kernels_per_iter =
      o.fused ? o.repeats + (o.copy_outputs ? 1 : 0) : 3 * o.repeats;

  const Timing t = run_iterations(o, st, enqueue_iteration);
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
  const double per_iter = t.gpu_ms / o.launches;
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
  print_common(o, t);
  std::printf(
      "rms_waves=%.3f softmax_waves=%.3f matmul_waves=%.3f min_waves=%.3f "
      "min_bytes_per_iter=%.0f achieved_gbps=%.1f valid=%d inputs=%s seed=%llu "
      "implementation=ce_b200 layout=%s kernels_per_iter=%d\n",
      rms_waves, softmax_waves, matmul_waves, min_waves, min_bytes,
      min_bytes / (per_iter * 1.0e6), valid ? 1 : 0, o.random ? "random" : "deterministic",
      (unsigned long long)o.seed, o.fused ? "fused" : "streams", kernels_per_iter);
  cudaFreeHost(h_norm);
  cudaFreeHost(h_softmax);
  cudaFreeHost(h_product);
  for (void *p : {(void *)d_input, (void *)d_weight, (void *)d_prob, (void *)d_softmax,
                  (void *)d_matrix, (void *)d_norm, (void *)d_product})
    cudaFree(p);
  return valid ? EXIT_SUCCESS : EXIT_FAILURE;
}

// The BASELINE op trio at the harness's shapes: normalized = rmsnorm(x),
// softmax of an independent logits batch, out [batch][rows] = the GEMM of the
// normalized batch with W [rows][size] in the chosen precision (ce_plan_*).
// Inputs from the op-trio generator (x, logits ~ N(0,1), W ~ N(0,1)/sqrt(size),
// rmsnorm weight ~ U(0.5,1.5); seed 0 unless random=SEED). In copy mode the
// last repeat runs the rows launch, starts the normalized and softmax copies
// on s1, and runs the GEMM on s0 meanwhile, then copies out.
int run_trio(Options &o) {
  const size_t vec = (size_t)o.batch * o.size, mat = (size_t)o.rows * o.size;
  const size_t outs = (size_t)o.batch * o.rows;
  const uint64_t seed = o.random ? o.seed : 0;
  std::vector<float> h_x(vec), h_logits(vec), h_w(o.size), h_W(mat);
  CE_CHECK(ce_fill_normal_host(seed, 1, 0, (int64_t)vec, 1.0f, h_x.data()));
  CE_CHECK(ce_fill_normal_host(seed, 2, 0, (int64_t)mat, (float)(1.0 / std::sqrt((double)o.size)),
                               h_W.data()));
  CE_CHECK(ce_fill_normal_host(seed, 3, 0, (int64_t)vec, 1.0f, h_logits.data()));
  CE_CHECK(ce_fill_uniform_host(seed, 4, 0, o.size, 0.5f, 1.5f, h_w.data()));
  float *d_x, *d_logits, *d_w, *d_W, *d_norm, *d_soft, *d_out;
  CUDA_CHECK(cudaMalloc(&d_x, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_logits, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_w, (size_t)o.size * 4));
  CUDA_CHECK(cudaMalloc(&d_W, mat * 4));
  CUDA_CHECK(cudaMalloc(&d_norm, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_soft, vec * 4));
  CUDA_CHECK(cudaMalloc(&d_out, outs * 4));
  CUDA_CHECK(cudaMemcpy(d_x, h_x.data(), vec * 4, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_logits, h_logits.data(), vec * 4, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_w, h_w.data(), (size_t)o.size * 4, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_W, h_W.data(), mat * 4, cudaMemcpyHostToDevice));
  float *h_norm, *h_soft, *h_out;
  CUDA_CHECK(cudaMallocHost(&h_norm, vec * 4));
  CUDA_CHECK(cudaMallocHost(&h_soft, vec * 4));
  CUDA_CHECK(cudaMallocHost(&h_out, outs * 4));

  const Streams st;
  const cudaStream_t s0 = st.s0, s1 = st.s1;
  const ce_stream_t c0 = (ce_stream_t)s0;
  ce_plan *plan = nullptr;
  CE_CHECK(ce_plan_create(&plan, o.batch, o.size, o.rows, o.precision));
  CE_CHECK(ce_plan_set_weights(plan, d_W, c0));
  CUDA_CHECK(cudaStreamSynchronize(s0));

  auto enqueue_iteration = [&]() {
    for (int r = 0; r < o.repeats; ++r) {
      if (!(o.copy_outputs && r + 1 == o.repeats)) {
        CE_CHECK(ce_plan_trio(plan, d_norm, d_soft, d_out, d_x, d_w, d_logits, kRmsEpsilon, c0));
        continue;
      }
      CE_CHECK(ce_plan_rows(plan, d_norm, d_soft, d_x, d_w, d_logits, kRmsEpsilon, c0));
      CUDA_CHECK(cudaEventRecord(st.fork, s0));
      CUDA_CHECK(cudaStreamWaitEvent(s1, st.fork, 0));
      CUDA_CHECK(cudaMemcpyAsync(h_norm, d_norm, vec * 4, cudaMemcpyDeviceToHost, s1));
      CUDA_CHECK(cudaMemcpyAsync(h_soft, d_soft, vec * 4, cudaMemcpyDeviceToHost, s1));
      CE_CHECK(ce_plan_gemm(plan, d_out, c0));
      CUDA_CHECK(cudaMemcpyAsync(h_out, d_out, outs * 4, cudaMemcpyDeviceToHost, s0));
      CUDA_CHECK(cudaEventRecord(st.join1, s1));
      CUDA_CHECK(cudaStreamWaitEvent(s0, st.join1, 0));
    }
  };
  const Timing t = run_iterations(o, st, enqueue_iteration);
  if (!o.copy_outputs) {
    CUDA_CHECK(cudaMemcpy(h_norm, d_norm, vec * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(h_soft, d_soft, vec * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(h_out, d_out, outs * 4, cudaMemcpyDeviceToHost));
  }
  // the GEMM's own operands, dequantized on the device (W reuses d_W)
  float *d_a = nullptr;
  CUDA_CHECK(cudaMalloc(&d_a, vec * 4));
  CE_CHECK(ce_plan_operands(plan, d_a, d_W, c0));
  CUDA_CHECK(cudaStreamSynchronize(s0));
  std::vector<float> a_op(vec), w_op(mat);
  CUDA_CHECK(cudaMemcpy(a_op.data(), d_a, vec * 4, cudaMemcpyDeviceToHost));
  CUDA_CHECK(cudaMemcpy(w_op.data(), d_W, mat * 4, cudaMemcpyDeviceToHost));
  const int status = ce_device_status();
  const double operand_u = o.precision == CE_PREC_TF32 ? std::ldexp(1.0, -9) : 0.0;
  const ce_host::TrioCheck check = ce_host::validate_trio(
      h_x.data(), h_logits.data(), h_w.data(), h_W.data(), h_norm, h_soft, h_out, a_op.data(),
      w_op.data(), operand_u, o.batch, o.size, o.rows, kTrioCheckedRows);
  bool valid = check.valid && status == CE_OK;
  if (!valid) std::fprintf(stderr, "Output validation failed\n");
  if (!o.dump_path.empty() &&
      !ce_host::write_l2cdump2(o.dump_path, seed, o.precision, o.batch, o.size, o.rows, h_norm,
                               h_soft, h_out, check))
    valid = false;
  const double per_iter = t.gpu_ms / o.launches;
  // Algorithmic traffic per repeat: x, logits read and normalized, softmax
  // written (fp32), the rmsnorm weight, W once in the plan's format, out
  // written; FLOPs 2 * batch * rows * size.
  const double w_bytes_per = o.precision == CE_PREC_BF16 ? 2.0
                           : o.precision == CE_PREC_FP8_E4M3 ? 1.0
                           : o.precision == CE_PREC_MXFP6_E3M2 ? 0.75 + 1.0 / 32
                           : o.precision == CE_PREC_NVFP4_E2M1 ? 0.5 + 1.0 / 16 : 4.0;
  const double min_bytes = o.repeats * (4.0 * vec * 4 + o.size * 4.0 + mat * w_bytes_per +
                                        (double)outs * 4);
  const double flops = o.repeats * 2.0 * o.batch * (double)o.rows * o.size;
  print_common(o, t);
  std::printf(
      "min_bytes_per_iter=%.0f achieved_gbps=%.1f tflops=%.1f valid=%d inputs=trio seed=%llu "
      "implementation=ce_b200 layout=trio precision=%s checked_rows=%zu out_rel_l2=%.3e "
      "out_worst_of_bound=%.3e out_rel_l2_exact=%.3e\n",
      min_bytes, min_bytes / (per_iter * 1.0e6), flops / (per_iter * 1.0e9), valid ? 1 : 0,
      (unsigned long long)seed, precision_name(o.precision), check.checked_rows.size(),
      check.rel_l2, check.worst_ratio, check.rel_l2_exact);
  ce_plan_destroy(plan);
  cudaFreeHost(h_norm);
  cudaFreeHost(h_soft);
  cudaFreeHost(h_out);
  for (void *p : {(void *)d_x, (void *)d_logits, (void *)d_w, (void *)d_W, (void *)d_norm,
                  (void *)d_soft, (void *)d_out, (void *)d_a})
    cudaFree(p);
  return valid ? EXIT_SUCCESS : EXIT_FAILURE;
}

}  // namespace

int main(int argc, char **argv) {
  Options o;
  if (!parse(argc, argv, &o)) {
    usage(argv[0]);
    return EXIT_FAILURE;
  }
  return o.trio ? run_trio(o) : run_llama2c(o);
}
