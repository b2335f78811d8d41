// Host-side validation and dump of the llama2c harness (product code of the
// drop-in executable, not the test oracle): the double-precision acceptance
// rules of llama2c/llama2c_common.h:150-319 (validate_outputs,
// validate_outputs_reference, validate_all) and the L2CDUMP1 writer
// (llama2c_common.h:16-32, 321-345). Multithreaded over rows.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace ce_host {

// gamma~_n(9) of the reference's GEMV tolerance: exp(9 sqrt(n) u + n u^2 /
// (1 - u)) - 1 with u = 2^-24 (llama2c_common.h:231-235).
double gamma_probabilistic(int n);

struct Llama2cCheck {
  bool valid = false;
  std::vector<float> product_tolerance;    // per row
  std::vector<double> product_reference;   // per row
};

// random == false applies the deterministic-input rules in addition.
Llama2cCheck validate_llama2c(bool random, const float *input, const float *probabilities,
                              const float *weight, const float *matrix, const float *normalized,
                              const float *softmax, const float *product, int batch, int size,
                              int rows);

bool write_l2cdump1(const std::string &path, bool random, uint64_t seed, int batch, int size,
                    int rows, const float *normalized, const float *softmax, const float *product,
                    const std::vector<float> &product_tolerance,
                    const std::vector<double> &product_reference);

}  // namespace ce_host
