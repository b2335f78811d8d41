// Command-line front end shared by the loom_private drop-in executables.
//
// It reproduces the interface of the reference harness
// (applications/loom_private/common/lp_harness.cuh:1-40 and :426-596): the
// same flags (--preset, --launch, --action, --iterations, --warmup, --set,
// --asset, --json-out), the same exit codes (0 pass, 1 mismatch, 2 usage,
// 3 asset, 70 CUDA), the same check / bench / profile protocols and the same
// "RESULT {...}" record (schema loom_private.result/1), so scripts written
// for the reference binaries run unchanged. The workload behind it computes
// through libce_b200 (include/ce_b200.h).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

namespace lp_front {

enum Exit { kPass = 0, kMismatch = 1, kUsage = 2, kAsset = 3, kCuda = 70 };

// Prints "<app>: <message>" to stderr and exits with code.
[[noreturn]] void die(int code, const char *format, ...) __attribute__((format(printf, 2, 3)));
// Exits through die() when a libce_b200 call failed: CE_ERR_USAGE maps to
// exit 2, every other failure to exit 70.
void ce_or_die(int status, const char *what);
// Exits 70 when a CUDA runtime call failed.
void cuda_or_die(int status, const char *what);

uint64_t fnv1a64(const void *data, size_t bytes, uint64_t state = 1469598103934665603ull);
std::string hex64(uint64_t value);

// Ordered JSON object: key -> already rendered JSON text.
using Fields = std::vector<std::pair<std::string, std::string>>;
std::string json_string(const std::string &text);
std::string json_number(double value);
std::string json_int(long long value);
std::string json_object(const Fields &fields);

enum class Launch { Direct, Graph, Both };
enum class Action { Check, Bench, Profile };

struct Options {
  std::string preset = "large";
  Launch launch = Launch::Both;
  bool launch_given = false;
  Action action = Action::Check;
  int iterations = 20, warmup = 3;
  std::map<std::string, std::string> sets, assets;
  std::string json_out;

  // Integer --set key (consumed), or fallback when absent; exit 2 when the
  // value is not an integer.
  long long integer(const std::string &key, long long fallback);
  std::vector<std::pair<std::string, long long>> consumed;
};

// One workload. enqueue() must be capturable into a CUDA graph (no host
// synchronization, allocation or device-result-dependent host logic).
class App {
 public:
  virtual ~App() = default;
  virtual std::string identity() const = 0;
  virtual Fields dimensions() const = 0;
  virtual std::string application_scope() const = 0;
  virtual std::string compute_scope() const = 0;
  virtual void setup(void *stream) = 0;
  virtual void enqueue(void *stream, bool compute_only) = 0;
  virtual void poison(void *stream) = 0;
  virtual void reference() = 0;  // host oracle of the check, run once
  virtual bool check() = 0;      // copies the outputs and compares
  virtual uint64_t digest() = 0;      // FNV-1a of the host copies of the outputs
};

struct Identity {
  const char *app;              // stderr prefix (the reference's LP_APP)
  const char *variant;          // "b200"
  const char *contract_sha256;  // sha256 of the contract implemented
};

// Parses argv, builds the App with make(options) (nullptr: unknown preset),
// runs the selected action and prints the RESULT record. Returns the exit code.
int run(int argc, char **argv, const Identity &id, App *(*make)(Options &));

}  // namespace lp_front
