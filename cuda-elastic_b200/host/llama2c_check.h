// Host-side validation and dumps of the llama2c harness (product code of the
// drop-in executable, not the test oracle): the double-precision acceptance
// rules of llama2c/llama2c_common.h:150-319 (validate_outputs,
// validate_outputs_reference, validate_all), the L2CDUMP1 writer
// (llama2c_common.h:16-32, 321-345), and for the op-trio mode (rmsnorm ->
// GEMM of the normalized batch, softmax) its check and the L2CDUMP2 writer.
// Multithreaded over rows.
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

// Op-trio check. Rows: the general rmsnorm / softmax rules above. GEMM:
// out[b][n] on the checked rows against the double product of the GEMM's own
// dequantized operands a [batch][size], w [rows][size] (as the reference's
// implementation check, decoder_lowprec.cu:947-1102), per value within its
// bound (gamma_K + operand_u) * sum_k |a w| + 2^-22 |ref| + FLT_MIN, gamma_K
// = K u / (1 - K u), u = 2^-23 (operand_u covers operands the tensor cores
// round further, 2^-9 for TF32, else 0), and in relative L2 within 1e-2. rel_l2_exact compares with the double product of
// the double rmsnorm and the fp32 weight matrix (the precision's own error;
// reported, not checked).
struct TrioCheck {
  bool valid = false;
  std::vector<int32_t> checked_rows;
  std::vector<float> out_tolerance;    // [checked][rows]
  std::vector<double> out_reference;   // [checked][rows]
  double rel_l2 = 0.0, rel_l2_exact = 0.0, worst_ratio = 0.0;
};

TrioCheck validate_trio(const float *input, const float *logits, const float *weight,
                        const float *matrix, const float *normalized, const float *softmax,
                        const float *out, const float *a_operand, const float *w_operand,
                        double operand_u, int batch, int size, int rows, int max_checked);

// L2CDUMP2: "L2CDUMP2", int32 batch, size, rows, inputs (2 = the op-trio
// generator), uint64 seed, int32 precision (CE_PREC_*), int32 checked count
// C, then normalized[B*S] f32, softmax[B*S] f32, out[B*N] f32,
// checked_rows[C] i32, out_tolerance[C*N] f32, out_reference[C*N] f64.
bool write_l2cdump2(const std::string &path, uint64_t seed, int precision, int batch, int size,
                    int rows, const float *normalized, const float *softmax, const float *out,
                    const TrioCheck &check);

}  // namespace ce_host
