// See lp_front.h. Protocols (lp_harness.cuh:14-40):
//   check   setup, the host oracle once, then per selected launch mode two
//           invocations, each after poisoning the outputs, each checked and
//           digested; all digests must agree (Direct against Graph bitwise).
//   bench   setup, W warm-ups, a batch of I back-to-back invocations between
//           two events, then I single invocations each between two events;
//           application scope first, then compute scope.
//   profile one warm-up invocation, then one between cudaProfilerStart/Stop.
#include "lp_front.h"

#include <cuda_profiler_api.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>

#include "ce_b200.h"

namespace lp_front {
namespace {

const char *g_app = "lp";

const char *launch_name(Launch l) {
  return l == Launch::Direct ? "direct" : l == Launch::Graph ? "graph" : "both";
}

const char *action_name(Action a) {
  return a == Action::Check ? "check" : a == Action::Bench ? "bench" : "profile";
}

double since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

[[noreturn]] void usage(int code) {
  std::fprintf(code ? stderr : stdout,
               "usage: %s [--preset large] [--launch direct|graph|both]\n"
               "          [--action check|bench|profile] [--iterations N] [--warmup W]\n"
               "          [--set key=value]... [--asset name=path]... [--json-out PATH]\n"
               "Defaults: --preset large --action check --launch both.\n"
               "bench and profile need an explicit --launch direct or --launch graph.\n",
               g_app);
  std::exit(code);
}

std::pair<std::string, std::string> key_value(const char *flag, const std::string &text) {
  const size_t eq = text.find('=');
  if (eq == std::string::npos || eq == 0) die(kUsage, "%s expects key=value, got '%s'", flag, text.c_str());
  return {text.substr(0, eq), text.substr(eq + 1)};
}

int count_arg(const char *flag, const std::string &text, int minimum) {
  char *end = nullptr;
  const long v = std::strtol(text.c_str(), &end, 10);
  if (end == text.c_str() || *end || v < minimum || v > 1000000)
    die(kUsage, "%s expects an integer >= %d, got '%s'", flag, minimum, text.c_str());
  return (int)v;
}

Options parse(int argc, char **argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string flag = argv[i];
    if (flag == "--help" || flag == "-h") usage(0);
    if (i + 1 >= argc) die(kUsage, "%s needs a value", flag.c_str());
    const std::string v = argv[++i];
    if (flag == "--preset") {
      o.preset = v;
    } else if (flag == "--launch") {
      o.launch_given = true;
      if (v == "direct") o.launch = Launch::Direct;
      else if (v == "graph") o.launch = Launch::Graph;
      else if (v == "both") o.launch = Launch::Both;
      else die(kUsage, "--launch must be direct, graph or both");
    } else if (flag == "--action") {
      if (v == "check") o.action = Action::Check;
      else if (v == "bench") o.action = Action::Bench;
      else if (v == "profile") o.action = Action::Profile;
      else die(kUsage, "--action must be check, bench or profile");
    } else if (flag == "--iterations") {
      o.iterations = count_arg("--iterations", v, 1);
    } else if (flag == "--warmup") {
      o.warmup = count_arg("--warmup", v, 0);
    } else if (flag == "--set") {
      const auto kv = key_value("--set", v);
      o.sets[kv.first] = kv.second;
    } else if (flag == "--asset") {
      const auto kv = key_value("--asset", v);
      o.assets[kv.first] = kv.second;
    } else if (flag == "--json-out") {
      o.json_out = v;
    } else {
      die(kUsage, "unknown option %s (see --help)", flag.c_str());
    }
  }
  if (o.action != Action::Check) {
    if (!o.launch_given || o.launch == Launch::Both)
      die(kUsage, "%s needs --launch direct or --launch graph", action_name(o.action));
    if (!o.sets.empty()) die(kUsage, "--set is only valid with --action check");
  }
  return o;
}

// Direct: enqueue on every launch. Graph: enqueue captured once into an
// instantiated, uploaded graph that every launch replays.
class Runner {
 public:
  Runner(Launch mode, cudaStream_t s, App &app, bool compute_only)
      : mode_(mode), s_(s), app_(app), compute_only_(compute_only) {
    if (mode_ != Launch::Graph) return;
    cudaGraph_t g = nullptr;
    cuda_or_die(cudaStreamBeginCapture(s_, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    app_.enqueue(s_, compute_only_);
    cuda_or_die(cudaStreamEndCapture(s_, &g), "cudaStreamEndCapture");
    cuda_or_die(cudaGraphInstantiate(&exec_, g, 0), "cudaGraphInstantiate");
    cuda_or_die(cudaGraphDestroy(g), "cudaGraphDestroy");
    cuda_or_die(cudaGraphUpload(exec_, s_), "cudaGraphUpload");
    cuda_or_die(cudaStreamSynchronize(s_), "cudaStreamSynchronize");
  }
  ~Runner() {
    if (exec_) cudaGraphExecDestroy(exec_);
  }
  Runner(const Runner &) = delete;
  Runner &operator=(const Runner &) = delete;
  void go() {
    if (exec_) cuda_or_die(cudaGraphLaunch(exec_, s_), "cudaGraphLaunch");
    else app_.enqueue(s_, compute_only_);
  }

 private:
  Launch mode_;
  cudaStream_t s_;
  App &app_;
  bool compute_only_;
  cudaGraphExec_t exec_ = nullptr;
};

double median_of(std::vector<double> v) {
  if (v.empty()) return 0.0;
  std::sort(v.begin(), v.end());
  const size_t n = v.size();
  return n % 2 ? v[n / 2] : 0.5 * (v[n / 2 - 1] + v[n / 2]);
}

std::string time_scope(Launch mode, cudaStream_t s, App &app, bool compute_only, const Options &o,
                       const std::string &scope) {
  Runner runner(mode, s, app, compute_only);
  for (int i = 0; i < o.warmup; ++i) runner.go();
  cuda_or_die(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  cudaEvent_t t0, t1;
  cuda_or_die(cudaEventCreate(&t0), "cudaEventCreate");
  cuda_or_die(cudaEventCreate(&t1), "cudaEventCreate");
  float ms = 0.0f;
  cuda_or_die(cudaEventRecord(t0, s), "cudaEventRecord");
  for (int i = 0; i < o.iterations; ++i) runner.go();
  cuda_or_die(cudaEventRecord(t1, s), "cudaEventRecord");
  cuda_or_die(cudaEventSynchronize(t1), "cudaEventSynchronize");
  cuda_or_die(cudaEventElapsedTime(&ms, t0, t1), "cudaEventElapsedTime");
  const double batch_ms = ms;
  std::vector<double> singles;
  for (int i = 0; i < o.iterations; ++i) {
    cuda_or_die(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    cuda_or_die(cudaEventRecord(t0, s), "cudaEventRecord");
    runner.go();
    cuda_or_die(cudaEventRecord(t1, s), "cudaEventRecord");
    cuda_or_die(cudaEventSynchronize(t1), "cudaEventSynchronize");
    cuda_or_die(cudaEventElapsedTime(&ms, t0, t1), "cudaEventElapsedTime");
    singles.push_back(1000.0 * ms);
  }
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  std::string list = "[";
  for (size_t i = 0; i < singles.size(); ++i) list += (i ? ", " : "") + json_number(singles[i]);
  list += "]";
  return json_object({{"scope", json_string(scope)},
                      {"batch_total_ms", json_number(batch_ms)},
                      {"batch_per_iteration_us", json_number(1000.0 * batch_ms / o.iterations)},
                      {"single_median_us", json_number(median_of(singles))},
                      {"single_us", list}});
}

}  // namespace

void die(int code, const char *format, ...) {
  std::fprintf(stderr, "%s: ", g_app);
  va_list args;
  va_start(args, format);
  std::vfprintf(stderr, format, args);
  va_end(args);
  std::fprintf(stderr, "\n");
  std::exit(code);
}

void ce_or_die(int status, const char *what) {
  if (status == CE_OK) return;
  char msg[1024];
  ce_last_error(msg, sizeof msg);
  if (status == CE_ERR_USAGE) die(kUsage, "%s", msg);
  die(kCuda, "%s failed (%d): %s", what, status, msg);
}

void cuda_or_die(int status, const char *what) {
  if (status == (int)cudaSuccess) return;
  die(kCuda, "%s failed: %s", what, cudaGetErrorString((cudaError_t)status));
}

uint64_t fnv1a64(const void *data, size_t bytes, uint64_t state) {
  const unsigned char *p = static_cast<const unsigned char *>(data);
  for (size_t i = 0; i < bytes; ++i) state = (state ^ p[i]) * 1099511628211ull;
  return state;
}

std::string hex64(uint64_t value) {
  char text[17];
  std::snprintf(text, sizeof text, "%016llx", (unsigned long long)value);
  return text;
}

std::string json_string(const std::string &text) {
  std::string out = "\"";
  for (unsigned char c : text) {
    if (c == '"') out += "\\\"";
    else if (c == '\\') out += "\\\\";
    else if (c == '\n') out += "\\n";
    else if (c == '\t') out += "\\t";
    else if (c < 0x20) {
      char esc[8];
      std::snprintf(esc, sizeof esc, "\\u%04x", c);
      out += esc;
    } else {
      out += (char)c;
    }
  }
  return out + "\"";
}

std::string json_number(double value) {
  char text[64];
  std::snprintf(text, sizeof text, "%.9g", value);
  return text;
}

std::string json_int(long long value) { return std::to_string(value); }

std::string json_object(const Fields &fields) {
  std::string out = "{";
  for (size_t i = 0; i < fields.size(); ++i)
    out += (i ? ", " : "") + json_string(fields[i].first) + ": " + fields[i].second;
  return out + "}";
}

long long Options::integer(const std::string &key, long long fallback) {
  auto it = sets.find(key);
  if (it == sets.end()) return fallback;
  char *end = nullptr;
  errno = 0;
  const long long v = std::strtoll(it->second.c_str(), &end, 0);
  if (errno || end == it->second.c_str() || *end)
    die(kUsage, "--set %s=%s is not an integer", key.c_str(), it->second.c_str());
  sets.erase(it);
  consumed.push_back({key, v});
  return v;
}

int run(int argc, char **argv, const Identity &id, App *(*make)(Options &)) {
  g_app = id.app;
  Options o = parse(argc, argv);
  std::unique_ptr<App> app(make(o));
  if (!app) die(kUsage, "unknown preset '%s' (available: large)", o.preset.c_str());
  if (!o.sets.empty()) die(kUsage, "unsupported --set key '%s'", o.sets.begin()->first.c_str());
  if (!o.assets.empty()) die(kUsage, "unsupported --asset name '%s'", o.assets.begin()->first.c_str());

  int device = 0, runtime = 0, driver = 0;
  cudaDeviceProp prop{};
  cuda_or_die(cudaGetDevice(&device), "cudaGetDevice");
  cuda_or_die(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  cuda_or_die(cudaRuntimeGetVersion(&runtime), "cudaRuntimeGetVersion");
  cuda_or_die(cudaDriverGetVersion(&driver), "cudaDriverGetVersion");
  cudaStream_t s;
  cuda_or_die(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
  auto t0 = std::chrono::steady_clock::now();
  app->setup(s);
  cuda_or_die(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  std::fprintf(stderr, "%s: setup %.2f s\n", g_app, since(t0));

  Fields overrides;
  for (const auto &kv : o.consumed) overrides.push_back({kv.first, json_int(kv.second)});
  Fields record = {
      {"schema", json_string("loom_private.result/1")},
      {"suite_version", json_string("v1")},
      {"identity", json_string(app->identity())},
      {"variant", json_string(id.variant)},
      {"loom_commit", json_string("4a75f8d743ef7fe755822bab0ea0fb78009c145b")},
      {"contract_sha256", json_string(id.contract_sha256)},
      {"preset", json_string(o.preset)},
      {"overrides", json_object(overrides)},
      {"dimensions", json_object(app->dimensions())},
      {"asset_sha256", "{}"},
      {"action", json_string(action_name(o.action))},
      {"launch", json_string(launch_name(o.launch))},
      {"device", json_object({{"name", json_string(prop.name)},
                              {"cc", json_string(std::to_string(prop.major) + "." +
                                                 std::to_string(prop.minor))},
                              {"cuda_runtime", json_int(runtime)},
                              {"cuda_driver", json_int(driver)}})},
      {"timing_scope", json_object({{"application", json_string(app->application_scope())},
                                    {"compute", json_string(app->compute_scope())}})},
  };

  int code = kPass;
  if (o.action == Action::Check) {
    t0 = std::chrono::steady_clock::now();
    app->reference();
    std::fprintf(stderr, "%s: CPU oracle %.2f s\n", g_app, since(t0));
    std::vector<Launch> modes;
    if (o.launch != Launch::Graph) modes.push_back(Launch::Direct);
    if (o.launch != Launch::Direct) modes.push_back(Launch::Graph);
    std::string checks = "[";
    std::vector<uint64_t> digests;
    bool pass = true;
    for (Launch mode : modes) {
      Runner runner(mode, s, *app, false);
      for (int rep = 1; rep <= 2; ++rep) {
        app->poison(s);
        cuda_or_die(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        t0 = std::chrono::steady_clock::now();
        runner.go();
        cuda_or_die(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        cuda_or_die(cudaGetLastError(), "kernel launch");
        const double secs = since(t0);
        const bool ok = app->check();
        const uint64_t dg = app->digest();
        digests.push_back(dg);
        pass = pass && ok;
        std::fprintf(stderr, "%s: %s invocation %d: %s, digest %s (%.2f s, untimed)\n", g_app,
                     launch_name(mode), rep, ok ? "PASS" : "FAIL", hex64(dg).c_str(), secs);
        if (checks.size() > 1) checks += ", ";
        checks += json_object({{"launch", json_string(launch_name(mode))},
                               {"invocation", json_int(rep)},
                               {"pass", ok ? "true" : "false"},
                               {"digest", json_string(hex64(dg))}});
      }
    }
    checks += "]";
    const bool agree = std::all_of(digests.begin(), digests.end(),
                                   [&](uint64_t d) { return d == digests[0]; });
    if (!agree) std::fprintf(stderr, "%s: FAIL: invocations or launch modes disagree\n", g_app);
    pass = pass && agree;
    record.push_back({"checks", checks});
    record.push_back({"outputs_agree", agree ? "true" : "false"});
    record.push_back({"timing", "null"});
    record.push_back({"status", json_string(pass ? "pass" : "fail")});
    code = pass ? kPass : kMismatch;
  } else if (o.action == Action::Profile) {
    Runner runner(o.launch, s, *app, false);
    runner.go();
    cuda_or_die(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    cuda_or_die(cudaProfilerStart(), "cudaProfilerStart");
    runner.go();
    cuda_or_die(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    cuda_or_die(cudaProfilerStop(), "cudaProfilerStop");
    record.push_back({"profiled", json_string("one application-scope invocation after one warmup invocation")});
    record.push_back({"timing", "null"});
    record.push_back({"output_digest", json_string(hex64(app->digest()))});
    record.push_back({"status", json_string("profile")});
  } else {
    const std::string application = time_scope(o.launch, s, *app, false, o, app->application_scope());
    const std::string compute = time_scope(o.launch, s, *app, true, o, app->compute_scope());
    cuda_or_die(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    record.push_back({"iterations", json_int(o.iterations)});
    record.push_back({"warmup", json_int(o.warmup)});
    record.push_back({"timing", json_object({{"application", application}, {"compute", compute}})});
    record.push_back({"output_digest", json_string(hex64(app->digest()))});
    record.push_back({"status", json_string("unvalidated_bench")});
  }

  const std::string line = json_object(record);
  std::printf("RESULT %s\n", line.c_str());
  std::fflush(stdout);
  if (!o.json_out.empty()) {
    std::FILE *f = std::fopen(o.json_out.c_str(), "w");
    const bool ok = f && std::fprintf(f, "%s\n", line.c_str()) >= 0;
    if (!f || std::fclose(f) != 0 || !ok) die(kUsage, "cannot write %s", o.json_out.c_str());
  }
  app.reset();
  cudaStreamDestroy(s);
  return code;
}

}  // namespace lp_front
