/*
 * orc.c -- CPU oracle of the llama2c hot path. TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker or the timed CPU baseline; the
 * product path (libce_b200.so and the package) never calls it.
 *
 * It restates, in plain C, the integer / byte-level parts of the
 * reference's algorithm (file:line in the reference project):
 *   - the llama2c counter generator and fill_inputs
 *       (llama2c/llama2c_common.h:92-132);
 *   - the sequential splitmix64 + Box-Muller fixture normals
 *       (experiments/blackwell/lowprec/reference.cpp:172-209);
 *   - the low-precision format tables and nearest-code quantizers
 *       (experiments/blackwell/lowprec/reference.cpp:13-157, spec.json
 *       "formats", "mxfp6", "nvfp4");
 *   - the decoder's analytic token progression
 *       (applications/loom_private/decoder/oracle.cpp:84-95);
 * and a multithreaded fp32 CPU implementation of the op-trio step (rmsnorm,
 * softmax, GEMM on the normalized batch), used as the timed CPU baseline.
 * The double-precision references live in oracle.py (numpy).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------ */
/* Generators                                                          */

/* splitmix64 finaliser of x + golden (llama2c/llama2c_common.h:92-97). */
static uint64_t mix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

/* Uniform in [-1, 1) on a 2^-23 grid (llama2c_common.h:100-103). */
float orc_llama2c_uniform(uint64_t seed, uint64_t stream, uint64_t index) {
  const uint64_t bits = mix64(mix64(seed * 4 + stream) ^ index);
  return (float)(int64_t)(bits >> 40) * (1.0f / 8388608.0f) - 1.0f;
}

/* fill_inputs (llama2c_common.h:105-132). */
void orc_fill_llama2c(int random, uint64_t seed, int batch, int size, int rows, float *input,
                      float *probabilities, float *weight, float *matrix) {
  const size_t vec = (size_t)batch * size, mat = (size_t)rows * size;
  if (!random) {
    for (size_t i = 0; i < vec; ++i) {
      if (input) input[i] = 1.0f + (float)(i % 4);
      if (probabilities) probabilities[i] = 1.0f + (float)(i % 4);
    }
    if (weight)
      for (int i = 0; i < size; ++i) weight[i] = 1.0f;
    if (matrix)
      for (int r = 0; r < rows; ++r)
        for (int c = 0; c < size; ++c) matrix[(size_t)r * size + c] = (c == r % size) ? 1.0f : 0.0f;
    return;
  }
  for (size_t i = 0; i < vec; ++i) {
    if (input) input[i] = orc_llama2c_uniform(seed, 0, i);
    if (probabilities) probabilities[i] = orc_llama2c_uniform(seed, 1, i);
  }
  if (weight)
    for (int i = 0; i < size; ++i) weight[i] = orc_llama2c_uniform(seed, 2, (uint64_t)i);
  if (matrix)
    for (size_t i = 0; i < mat; ++i) matrix[i] = orc_llama2c_uniform(seed, 3, i);
}

/* Sequential splitmix64 (reference.cpp:172-181): next() adds the golden
 * increment to the state and returns the finaliser of the new state. */
typedef struct { uint64_t state; } orc_splitmix;
static uint64_t sm_next(orc_splitmix *g) {
  uint64_t z = (g->state += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
static double sm_uniform(orc_splitmix *g) { return (double)(sm_next(g) >> 11) * 0x1.0p-53; }

/* Standard normals of stream `stream` (reference.cpp:183-194), elements
 * [0, count), each times `scale` as a float product (reference.cpp:203-209).
 * Generated sequentially, as the reference does. */
void orc_normals(uint64_t seed, uint64_t stream, int64_t count, float scale, float *out) {
  orc_splitmix g = {seed * 0x100000001b3ull + stream};
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t i = 0; i < count; i += 2) {
    const double u1 = sm_uniform(&g), u2 = sm_uniform(&g);
    const double radius = sqrt(-2.0 * log(1.0 - u1));
    out[i] = (float)(radius * cos(two_pi * u2)) * scale;
    if (i + 1 < count) out[i + 1] = (float)(radius * sin(two_pi * u2)) * scale;
  }
}

/* Uniform lo + (hi - lo) u of the same sequential stream, one call each. */
void orc_uniforms(uint64_t seed, uint64_t stream, int64_t count, float lo, float hi, float *out) {
  orc_splitmix g = {seed * 0x100000001b3ull + stream};
  for (int64_t i = 0; i < count; ++i)
    out[i] = (float)((double)lo + ((double)hi - (double)lo) * sm_uniform(&g));
}

/* ------------------------------------------------------------------ */
/* Low-precision formats (reference.cpp:13-82, spec.json "formats").  */
/* format: 0 E2M1, 1 E3M2, 2 UE4M3, 3 UE8M0, 4 E4M3 (signed OCP FP8,   */
/* largest 448, used by the FP8 per-row mode of this build).          */

static unsigned max_code(int f) {
  switch (f) {
    case 0: return 7;
    case 1: return 31;
    case 2: return 126;
    case 3: return 254;
    case 4: return 126;
  }
  abort();
}
static unsigned sign_bit(int f) { return f == 0 ? 8 : f == 1 ? 32 : f == 4 ? 128 : 0; }

static double magnitude(int f, unsigned code) {
  switch (f) {
    case 0: {
      static const double v[8] = {0, 0.5, 1, 1.5, 2, 3, 4, 6};
      return v[code & 7];
    }
    case 1: {
      const int e = (code >> 2) & 7, m = code & 3;
      return e == 0 ? ldexp(m / 4.0, -2) : ldexp(1.0 + m / 4.0, e - 3);
    }
    case 2:
    case 4: {
      const int e = (code >> 3) & 15, m = code & 7;
      return e == 0 ? ldexp(m / 8.0, -6) : ldexp(1.0 + m / 8.0, e - 7);
    }
    case 3: return ldexp(1.0, (int)code - 127);
  }
  abort();
}

double orc_decode(int f, unsigned code) {
  const unsigned s = sign_bit(f);
  const double v = magnitude(f, s ? (code & (s - 1)) : code);
  return (s && (code & s)) ? -v : v;
}

/* Nearest code, ties to the code with an even last magnitude bit,
 * saturation at the largest magnitude, +0 for a zero magnitude. */
unsigned orc_encode(int f, double v) {
  const double target = fabs(v);
  const unsigned top = max_code(f);
  /* last code whose magnitude is <= target (magnitudes increase with code) */
  unsigned lo = 0, hi = top;
  if (magnitude(f, top) <= target) {
    lo = top;
  } else {
    while (hi - lo > 1) {
      const unsigned mid = (lo + hi) / 2;
      if (magnitude(f, mid) <= target) lo = mid; else hi = mid;
    }
  }
  unsigned best = lo;
  if (lo < top && magnitude(f, lo) < target) {
    const double down = target - magnitude(f, lo), up = magnitude(f, lo + 1) - target;
    if (up < down || (up == down && (lo & 1))) best = lo + 1;
  }
  if (best == 0) return 0;
  return (v < 0 && sign_bit(f)) ? (best | sign_bit(f)) : best;
}

/* bf16 bits, round to nearest even (reference.cpp:84-96). */
uint16_t orc_bf16(float v) {
  uint32_t bits;
  memcpy(&bits, &v, 4);
  const uint32_t lsb = (bits >> 16) & 1u;
  return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}
float orc_bf16_value(uint16_t b) {
  const uint32_t w = (uint32_t)b << 16;
  float v;
  memcpy(&v, &w, 4);
  return v;
}

/* MXFP6 E3M2 with UE8M0 per 32 (reference.cpp:105-122, spec.json "mxfp6").
 * codes: one byte per value (unpacked); scales: one byte per block. */
void orc_quantize_mxfp6(const float *row, int64_t width, uint8_t *codes, uint8_t *scales) {
  for (int64_t b = 0; b * 32 < width; ++b) {
    const float *x = row + b * 32;
    const int n = (int)((width - b * 32) < 32 ? (width - b * 32) : 32);
    float amax = 0.f;
    for (int i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(x[i]));
    if (amax == 0.f) {
      scales[b] = 0;
      for (int i = 0; i < n; ++i) codes[b * 32 + i] = 0;
      continue;
    }
    int e;
    frexp((double)amax, &e);
    int shared = (e - 1) - 4;
    if (shared > 127) shared = 127;
    if (shared < -127) shared = -127;
    scales[b] = (uint8_t)(shared + 127);
    for (int i = 0; i < n; ++i) codes[b * 32 + i] = (uint8_t)orc_encode(1, ldexp((double)x[i], -shared));
  }
}

/* NVFP4 tensor scale (reference.cpp:124-127). */
float orc_nvfp4_encode_scale(float amax) { return amax > 0.0f ? 2688.0f / amax : 1.0f; }

/* NVFP4 E2M1 with UE4M3 per 16 (reference.cpp:129-150). */
void orc_quantize_nvfp4(const float *row, int64_t width, float s, uint8_t *codes, uint8_t *scales) {
  for (int64_t b = 0; b * 16 < width; ++b) {
    const float *x = row + b * 16;
    const int n = (int)((width - b * 16) < 16 ? (width - b * 16) : 16);
    float amax = 0.f;
    for (int i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(x[i]));
    float target = amax / 6.0f;
    target = target * s;
    const unsigned sc = orc_encode(2, target);
    scales[b] = (uint8_t)sc;
    const float f = (float)orc_decode(2, sc);
    for (int i = 0; i < n; ++i) {
      if (sc == 0) {
        codes[b * 16 + i] = 0;
        continue;
      }
      float r = x[i] * s;
      r = r / f;
      codes[b * 16 + i] = (uint8_t)orc_encode(0, r);
    }
  }
}

/* ------------------------------------------------------------------ */
/* Decoder analytic tokens (applications/loom_private/decoder/oracle.cpp:84-95,
 * contract.json "tolerances.generated"): token after step s of sequence b is
 * (b mod V + s + 1) mod V. tokens is [batch][steps].                   */
void orc_decoder_tokens(int64_t batch, int64_t vocab, int64_t steps, int32_t *tokens) {
  for (int64_t b = 0; b < batch; ++b) {
    int64_t t = b % vocab;
    for (int64_t s = 0; s < steps; ++s) {
      t = (t + 1) % vocab;
      tokens[b * steps + s] = (int32_t)t;
    }
  }
}

/* FNV-1a 64 (applications/loom_private/common/lp_harness.cuh:107-115). */
uint64_t orc_fnv1a64(const void *data, size_t n, uint64_t h) {
  const unsigned char *p = (const unsigned char *)data;
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 0x100000001b3ull;
  }
  return h;
}

/* ------------------------------------------------------------------ */
/* Multithreaded fp32 op-trio step on the CPU (the timed CPU baseline). */

typedef struct {
  const float *x, *w, *logits, *W;
  float *normalized, *softmax, *out;
  int rows_b, K, N;   /* sampled batch rows, width, output rows */
  float eps;
  int t, nthreads;
} trio_job;

static float dot8(const float *a, const float *b, int n) {
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int k = 0;
  for (; k + 8 <= n; k += 8)
    for (int j = 0; j < 8; ++j) s[j] += a[k + j] * b[k + j];
  float r = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
  for (; k < n; ++k) r += a[k] * b[k];
  return r;
}

static void *trio_worker(void *arg) {
  trio_job *j = (trio_job *)arg;
  const int K = j->K;
  /* rows stage: batch rows split over threads */
  for (int b = j->t; b < j->rows_b; b += j->nthreads) {
    const float *x = j->x + (size_t)b * K;
    float ss = 0.f;
    for (int k = 0; k < K; ++k) ss += x[k] * x[k];
    const float scale = 1.0f / sqrtf(ss / (float)K + j->eps);
    for (int k = 0; k < K; ++k) j->normalized[(size_t)b * K + k] = j->w[k] * (scale * x[k]);
    const float *l = j->logits + (size_t)b * K;
    float m = -INFINITY, s = 0.f;
    for (int k = 0; k < K; ++k) m = fmaxf(m, l[k]);
    float *p = j->softmax + (size_t)b * K;
    for (int k = 0; k < K; ++k) s += (p[k] = expf(l[k] - m));
    for (int k = 0; k < K; ++k) p[k] /= s;
  }
  return NULL;
}

static void *gemm_worker(void *arg) {
  trio_job *j = (trio_job *)arg;
  const int K = j->K;
  /* GEMM stage: output rows (W rows) split over threads, each W row read
   * once for all sampled batch rows. */
  for (int r = j->t; r < j->N; r += j->nthreads) {
    const float *wr = j->W + (size_t)r * K;
    for (int b = 0; b < j->rows_b; ++b) j->out[(size_t)b * j->N + r] = dot8(wr, j->normalized + (size_t)b * K, K);
  }
  return NULL;
}

int orc_cpu_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

/* normalized, softmax [rows_b][K]; out [rows_b][N]. Returns threads used. */
int orc_trio_fp32(const float *x, const float *w, const float *logits, const float *W,
                  float *normalized, float *softmax, float *out, int rows_b, int K, int N,
                  float eps, int nthreads) {
  if (nthreads <= 0) nthreads = orc_cpu_threads();
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * nthreads);
  trio_job *jobs = (trio_job *)malloc(sizeof(trio_job) * nthreads);
  for (int stage = 0; stage < 2; ++stage) {
    for (int t = 0; t < nthreads; ++t) {
      trio_job j = {x, w, logits, W, normalized, softmax, out, rows_b, K, N, eps, t, nthreads};
      jobs[t] = j;
      pthread_create(&th[t], NULL, stage == 0 ? trio_worker : gemm_worker, &jobs[t]);
    }
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
  }
  free(th);
  free(jobs);
  return nthreads;
}
