/*
 * ce_b200.h -- C ABI of the B200-native llama2c hot path (libce_b200.so).
 *
 * The reference (ankaijin/cuda-elastic) exposes this path only as CUDA
 * kernels with raw-pointer signatures, launched on a caller's stream by a
 * per-workload harness. Every entry point below replaces one of those
 * kernels or harness steps; the comment above each names the reference
 * symbol (file:line, paths relative to the reference project root).
 *
 * Conventions
 *   - Every function returns an int status: CE_OK (0) or one of CE_ERR_*.
 *     The status values follow the loom_private harness exit codes
 *     (applications/loom_private/common/lp_harness.cuh:88-92): usage errors
 *     are 2, CUDA errors 70. ce_last_error() returns the message of the last
 *     failure on the calling host thread.
 *   - Pointers named *_dev are device pointers allocated by the caller; host
 *     pointers are named *_host. Matrices are row-major, rows contiguous.
 *   - Enqueue functions (everything that takes a ce_stream_t except the
 *     *_create / *_set_* setup calls) allocate nothing, never synchronize the
 *     host and read no environment variable, so they can be captured in a
 *     CUDA graph (the reference's lp::Workload::enqueue_compute contract,
 *     lp_harness.cuh:236-239).
 *   - ce_stream_t is binary-identical to cudaStream_t / CUstream; NULL is the
 *     legacy default stream.
 */
#ifndef CE_B200_H
#define CE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ce_stream_t;

/* Status codes. */
#define CE_OK 0
#define CE_ERR_USAGE 2        /* invalid argument or unsupported shape */
#define CE_ERR_CUDA 70        /* a CUDA runtime / driver call failed */
#define CE_ERR_TIMEOUT 71     /* a bounded device-side wait ran out */
#define CE_ERR_NOMEM 72       /* device or pinned allocation failed */

/* Arithmetic of the matmul (the classifier / GEMM operand precision). */
#define CE_PREC_FP32 0        /* SIMT fp32, sequential k, separate mul+add */
#define CE_PREC_TF32 1        /* tcgen05 kind::tf32 on fp32 operands */
#define CE_PREC_BF16 2        /* tcgen05 kind::f16, bf16 operands */
#define CE_PREC_FP8_E4M3 3    /* tcgen05 kind::f8f6f4, E4M3 with per-row fp32 scales */
#define CE_PREC_MXFP6_E3M2 4  /* tcgen05 kind::mxf8f6f4 block-scaled E3M2, UE8M0 / 32 */
#define CE_PREC_NVFP4_E2M1 5  /* tcgen05 kind::mxf4nvf4 block-scaled E2M1, UE4M3 / 16 */

/* Output-tile width of the block-scaled GEMMs; the B operand's scale atoms
 * are grouped by this many rows. */
#define CE_BS_TILE_N 224

/* ------------------------------------------------------------------ */
/* Library                                                             */

/* Version string of the library ("ce_b200 <major>.<minor>"). */
const char *ce_version(void);

/* Copies the last error message of the calling thread into buf (always
 * NUL-terminated when len > 0) and returns the last status. */
int ce_last_error(char *buf, size_t len);

/* Number of SMs of the current device and whether it is an sm_100 part
 * (tcgen05 paths need it). */
int ce_device_info(int *sm_count, int *is_sm100);

/* Synchronizes the current device and reports whether a bounded device-side
 * wait of a tensor-core kernel gave up since the last call (CE_ERR_TIMEOUT,
 * then cleared). The reference's stream-K consumer waits without a limit
 * (applications/loom_private/decoder/decoder_optimized.cu:391-394); every
 * wait of this library is bounded and reported here instead. */
int ce_device_status(void);

/* ------------------------------------------------------------------ */
/* Seeded inputs (host side, multithreaded).                           */

/* llama2c input generator: llama2c/llama2c_common.h:105-132 (fill_inputs).
 * random == 0: deterministic inputs (1,2,3,4 repeating; weight 1; shifted
 * identity matrix). random != 0: uniform in [-1,1) from the counter-based
 * splitmix64 stream (seed, stream 0 input, 1 probabilities, 2 weight,
 * 3 matrix). Any output pointer may be NULL to skip it. */
int ce_fill_llama2c_host(int random, uint64_t seed, int batch, int size, int rows,
                         float *input_host, float *probabilities_host,
                         float *weight_host, float *matrix_host);

/* Standard normals of the reference's fixture generator
 * (experiments/blackwell/lowprec/reference.cpp:172-194): splitmix64 seeded
 * with seed * 0x100000001b3 + stream, Box-Muller pairs in double, each
 * value times `scale` (float product, reference.cpp:203-209), rounded to
 * float. Writes elements [first, first + count) of the stream. */
int ce_fill_normal_host(uint64_t seed, uint64_t stream, int64_t first, int64_t count,
                        float scale, float *out_host);

/* Uniform values lo + (hi - lo) * u, u = (splitmix64 >> 11) * 2^-53, of the
 * same seeded stream layout as ce_fill_normal_host (one value per call of
 * the generator). */
int ce_fill_uniform_host(uint64_t seed, uint64_t stream, int64_t first, int64_t count,
                         float lo, float hi, float *out_host);

/* ------------------------------------------------------------------ */
/* Row operations (HBM-bound).                                         */

/* RMSNorm: out[b,i] = x[b,i] * rsqrt(sum_i x[b,i]^2 / cols + eps) * w[i].
 * Replaces rmsnorm_kernel, llama2c/llama2c_cuda_graph.cu:58-78. */
int ce_rmsnorm(float *out_dev, const float *x_dev, const float *w_dev, int rows, int cols,
               float eps, ce_stream_t stream);

/* Row softmax: out[b,i] = exp(l[b,i] - max_b) / sum_i exp(l[b,i] - max_b).
 * Replaces softmax_kernel, llama2c/llama2c_cuda_graph.cu:82-115. */
int ce_softmax(float *out_dev, const float *logits_dev, int rows, int cols,
               ce_stream_t stream);

/* GEMV: product[r] = sum_c matrix[r,c] * x[c] (x = the first `cols` floats
 * of the raw input). Replaces matmul_kernel / matmul_coalesced_kernel,
 * llama2c/llama2c_cuda_graph.cu:119-162. */
int ce_gemv(float *product_dev, const float *matrix_dev, const float *x_dev, int rows,
            int cols, ce_stream_t stream);

/* The llama2c iteration in one launch: rmsnorm of input [batch][size],
 * softmax of probabilities [batch][size], GEMV of matrix [rows][size] with
 * input row 0. Replaces llama2c_sota_kernel, llama2c/llama2c_sota.cu:263-298
 * (and the three-stream enqueue_iteration, llama2c_cuda_graph.cu:347-381). */
int ce_llama2c_iteration(float *normalized_dev, float *softmax_dev, float *product_dev,
                         const float *input_dev, const float *weight_dev,
                         const float *probabilities_dev, const float *matrix_dev,
                         int batch, int size, int rows, float eps, ce_stream_t stream);

/* Part of the llama2c iteration in one launch: rmsnorm of the first
 * rms_rows rows of input, softmax of the first softmax_rows rows of
 * probabilities, GEMV of the first matmul_rows rows of matrix with input row
 * 0; any count may be 0 (its pointers are then unused), not all three. The
 * copy mode of the SOTA harness splits its last repeat into an rmsnorm-only
 * launch and a softmax + GEMV launch on a second stream so the normalized
 * copy to the host overlaps the rest. Replaces the Work split (rms_work /
 * rest_work), llama2c/llama2c_sota.cu:82-94 and :447-496. */
int ce_llama2c_rows(float *normalized_dev, float *softmax_dev, float *product_dev,
                    const float *input_dev, const float *weight_dev,
                    const float *probabilities_dev, const float *matrix_dev, int size,
                    int rms_rows, int softmax_rows, int matmul_rows, float eps,
                    ce_stream_t stream);

/* ------------------------------------------------------------------ */
/* Tensor-core GEMM (tcgen05 + TMEM, operands by TMA).                 */

/* D[m][n] = sum_k A[m][k] * B[n][k] (both operands K-contiguous, D fp32
 * row-major with leading dimension ldd). A and B are bf16 bit patterns
 * (uint16). Requirements: lda, ldb multiples of 8 elements, 16-byte aligned
 * base pointers; M, N, K >= 1. Ragged M, N, K are handled (zero fill).
 * This is the engine behind the classifier GEMM of
 * applications/loom_private/decoder/decoder_optimized.cu:343-439 and the
 * BF16 CUTLASS GEMM of experiments/blackwell/lowprec/decoder_lowprec.cu:85-92. */
int ce_gemm_bf16(float *d_dev, const uint16_t *a_dev, const uint16_t *b_dev, int M, int N,
                 int K, int lda, int ldb, int ldd, ce_stream_t stream);

/* ce_gemm_bf16 on the single-CTA kernel (128-row tiles) with a forced
 * output-tile width (128, 160, 192, 224 or 256 columns; 0 = automatic). */
int ce_gemm_bf16_tile(float *d_dev, const uint16_t *a_dev, const uint16_t *b_dev, int M, int N,
                      int K, int lda, int ldb, int ldd, int tile_n, ce_stream_t stream);

/* Tensor-core GEMM with a forced kernel: precision CE_PREC_BF16 (a, b bf16
 * bits), CE_PREC_TF32 (a, b fp32) or CE_PREC_FP8_E4M3 (a, b E4M3 codes, no
 * scales); cta_group 1 = single-CTA kernel
 * (128 x tile_n tiles), 2 = CTA-pair kernel (256 x tile_n tiles on two SMs,
 * tcgen05 cta_group::2), 3 = CTA-pair kernel with two N pieces per tile
 * (256 x 2 tile_n tiles: two N = tile_n MMAs per k step on the same A tile,
 * one 512-column TMEM accumulator; tile_n 224, 240 or 256, M > 128),
 * 0 = automatic; tile_n 64/96/128/160/192/224/256 or 0.
 * Test hook in the spirit of the reference's forced tiles and schedules
 * (decoder_optimized.cu:543-557, DECODER_OPT_TILE / _SCHEDULE). */
int ce_gemm_config(int precision, float *d_dev, const void *a_dev, const void *b_dev, int M, int N,
                   int K, int lda, int ldb, int ldd, int cta_group, int tile_n,
                   ce_stream_t stream);

/* Split-K bf16 GEMM for decode-sized shapes (few rows, so the output tiles
 * alone leave SMs idle): split s of `splits` (1 <= splits <= ceil(K / 64))
 * accumulates its balanced share of K and writes its fp32 partial
 * D_s = A[:, K_s] B[:, K_s]^T at d_dev + s * split_stride (elements, at
 * least (M - 1) * ldd + N); the caller sums the partials, in split order for
 * a deterministic result. No counterpart in the reference (its GEMMs are
 * whole-K tiles, decoder_lowprec.cu:85-127). */
int ce_gemm_bf16_split(float *d_dev, const uint16_t *a_dev, const uint16_t *b_dev, int M, int N,
                       int K, int lda, int ldb, int ldd, int splits, int64_t split_stride,
                       ce_stream_t stream);

/* Repacks NVFP4 weights from the ce_quantize_nvfp4 layout (codes [N][ld_bytes],
 * two per byte; UE4M3 scales [N][nsf], nsf = K / 16) into the k-block-major
 * layout the W4A16 GEMM streams: codes_t [K/64][N][32], scales_t [K/64][N][4].
 * K % 64 == 0. Setup-time. */
int ce_w4_pack(uint8_t *codes_t_dev, uint8_t *scales_t_dev, const uint8_t *codes_dev,
               const uint8_t *scales_dev, int N, int K, int ld_bytes, int nsf, ce_stream_t stream);

/* W4A16 GEMM with the dequantization fused: D[m][n] = alpha * sum_k
 * A[m][k] * W[n][k], A fp16 [M][lda], W NVFP4 in the ce_w4_pack layout
 * (E2M1 code x UE4M3 scale, expanded to fp16 in shared memory right before
 * the tensor cores read it; every such product is exact in fp16), alpha =
 * the weight's decode scale (device fp32, element 1 of ce_quantize_nvfp4's
 * tensor scales; NULL = 1), fp32 accumulation and output. K % 64 == 0,
 * N % 4 == 0. The reference's NVFP4 GEMM quantizes the activations too
 * (decoder_lowprec.cu:111-127); this one keeps them 16-bit. */
int ce_gemm_w4a16(float *d_dev, const uint16_t *a_dev, const uint8_t *codes_t_dev,
                  const uint8_t *scales_t_dev, const float *alpha_dev, int M, int N, int K, int lda,
                  int ldd, ce_stream_t stream);

/* Bytes of the decode-form packed NVFP4 weights (ce_w4t_pack) of an N x K
 * weight: ceil(K/128) * roundup(N, 256) / 128 * 9216. Host-only. */
int ce_w4t_packed_bytes(int N, int K, size_t *bytes);

/* Packs NVFP4 weights (the ce_quantize_nvfp4 layout, as ce_w4_pack takes
 * them) into the decode-form layout of ce_gemm_w4t: per 128-wide k block kb
 * and 128-row group hg, a block of 9216 bytes at (kb * roundup(N, 256) / 128
 * + hg) * 9216 holding the E2M1 codes of its four 32-row quarters as four
 * 16-byte columns of 32 rows ([4][4][32][16]) and then their UE4M3 scales
 * as 32 rows of 8 bytes ([4][32][8]); zero past N and past K. A 256-row
 * tile's stage is one contiguous 18 KB copy. K % 64 == 0. Setup-time. */
int ce_w4t_pack(uint8_t *packed_dev, const uint8_t *codes_dev, const uint8_t *scales_dev, int N, int K,
                int ld_bytes, int nsf, ce_stream_t stream);

/* W4A16 GEMM, decode form: the same product as ce_gemm_w4a16 (D[m][n] =
 * alpha * sum_k A[m][k] W[n][k], A fp16 [M][lda], fp32 accumulation) with
 * the weights as the 128-row operand of the tensor cores, expanded to fp16
 * in tensor memory, and the batch (M) as the narrow operand, for the small
 * batches of a decode step. W in the ce_w4t_pack layout; K % 64 == 0. Split
 * s of `splits` (1 <= splits <= ceil(K / 128)) writes its fp32 partial at
 * d_dev + s * split_stride; the caller sums the partials in split order.
 * Replaces the NVFP4 classifier GEMM of the reference's low-precision
 * decoder (decoder_lowprec.cu:111-127), keeping the activations 16-bit. */
int ce_gemm_w4t(float *d_dev, const uint16_t *a_dev, const uint8_t *packed_dev, const float *alpha_dev,
                int M, int N, int K, int lda, int ldd, int splits, int64_t split_stride, ce_stream_t stream);

/* A ce_w4t_pack-layout weight [N][K] expanded to fp16 [N][K]: e2m1(code) x
 * ue4m3(scale), exact in fp16; the tensor decode scale is left for the GEMM
 * (alpha below). The NVFP4 prefill multiplies its layer weights this way. */
int ce_w4t_expand_f16(uint16_t *out_dev, const uint8_t *packed_dev, int N, int K, ce_stream_t stream);

/* fp16 tensor-core GEMM (tcgen05 kind::f16 with fp16 operands):
 * d[m][n] = alpha x sum_k A[m][k] B[n][k], A and B fp16 bit patterns,
 * K-contiguous (lda, ldb multiples of 8, 16-byte aligned bases); alpha_dev a
 * scalar on the device or NULL (1). */
int ce_gemm_f16(float *d_dev, const uint16_t *a_dev, const uint16_t *b_dev, const float *alpha_dev,
                int M, int N, int K, int lda, int ldb, int ldd, ce_stream_t stream);

/* Library-wide GEMM tuning, set at setup time (not during a capture): the
 * TMA producer prefetches operand tiles this many k-blocks ahead into L2
 * (0 = off, at most 64). */
int ce_gemm_tuning(int l2_prefetch_kblocks);

/* Library-wide, set at setup time: whether the automatic tile choice may
 * take two-piece CTA-pair tiles (cta_group 3 of ce_gemm_config) for GEMMs
 * whose tiles then fit one wave (1, the default) or not (0). */
int ce_gemm_wide_tiles(int on);

/* Library-wide, set at setup time: launches of long rmsnorm / softmax rows
 * (32 to 64 KiB, no GEMV rows) run the persistent streaming kernel (one CTA
 * per SM, rows arriving by bulk copies two rows ahead; 1, the default) or
 * one register-resident CTA per row (0). Both give the same bits. */
int ce_rows_tuning(int streaming);

/* Same contraction on fp32 operands with tcgen05 kind::tf32 (the tensor
 * core reads the upper 19 bits of each fp32 value). lda, ldb multiples of 4
 * elements, 16-byte aligned base pointers. */
int ce_gemm_tf32(float *d_dev, const float *a_dev, const float *b_dev, int M, int N, int K,
                 int lda, int ldb, int ldd, ce_stream_t stream);

/* Same contraction on the SIMT cores with the reference's bitwise contract:
 * each output accumulated from 0.0f in increasing k with separate multiply
 * and add (applications/loom_private/decoder/decoder.cu:79-125). Any
 * alignment; the control path of CE_PREC_FP32. */
int ce_gemm_fp32(float *d_dev, const float *a_dev, const float *b_dev, int M, int N, int K,
                 int lda, int ldb, int ldd, ce_stream_t stream);

/* E4M3 (OCP FP8, largest 448) quantization of a [rows][cols] fp32 matrix
 * with one fp32 scale per row: amax = max |x| of the row, inv = 448 / amax,
 * scale = amax / 448 (IEEE fp32; 0 for an all-zero row), code = E4M3(x * inv),
 * round to nearest even, saturating. codes [rows][ld], columns past cols are
 * 0. The FP8-E4M3 per-row mode of the op trio has no reference counterpart
 * (BASELINE config 3); the conversion follows the spec's rounding rules
 * (experiments/blackwell/lowprec/spec.json "rounding"). */
int ce_quantize_e4m3_rows(uint8_t *codes_dev, float *scales_dev, const float *x_dev, int rows,
                          int cols, int ld, ce_stream_t stream);

/* MXFP6 E3M2 quantization with one UE8M0 scale per 32 values along each
 * row (experiments/blackwell/lowprec/decoder_lowprec.cu:243-286,
 * quantize_mxfp6_kernel; rules of spec.json "mxfp6"): codes one byte per
 * value (6 bits used) [rows][ld_codes], columns past cols 0; scales
 * [rows][ceil(cols / 32)] row-major. Bit-exact with the spec's host
 * quantizer (reference.cpp:105-122). */
int ce_quantize_mxfp6(uint8_t *codes_dev, uint8_t *scales_dev, const float *x_dev, int rows,
                      int cols, int ld_codes, ce_stream_t stream);

/* NVFP4 E2M1 quantization (decoder_lowprec.cu:202-219, 294-340,
 * tensor_amax_kernel and quantize_nvfp4_kernel; spec.json "nvfp4"): the
 * tensor amax of x gives the encode scale s = 2688 / amax (1 when 0) and
 * decode scale 1 / s, written to tensor_scales_dev[0..1]; each 16-value
 * block gets the UE4M3 scale code of (amax_block / 6) * s and codes
 * E2M1((v * s) / f), two per byte, even index in the low nibble
 * [rows][ld_bytes]. scratch_dev is one device word used for the amax
 * reduction. Bit-exact with reference.cpp:124-150. */
int ce_quantize_nvfp4(uint8_t *codes_dev, uint8_t *scales_dev, float *tensor_scales_dev,
                      uint32_t *scratch_dev, const float *x_dev, int rows, int cols, int ld_bytes,
                      ce_stream_t stream);

/* Block-scaled GEMM operands keep their scales in 512-byte atoms of 128
 * rows x 4 scale columns (byte (r % 32) * 16 + (r / 32) * 4 + c), atoms
 * along K fastest, rows taken in groups of group_rows (128 for A, and
 * CE_BS_TILE_N for B so that every output tile's scales start on an atom
 * boundary), each group padded to whole atoms; padding bytes 0. This
 * replaces the reference's CUTLASS Sm1xxBlkScaledConfig layout
 * (experiments/blackwell/lowprec/spec.json "layout.scale_factors") with one
 * shaped for this library's tiles. format: 0 = MXFP6 (one scale per 32
 * values), 1 = NVFP4 (per 16). */
int ce_sf_atom_bytes(int format, int rows, int K, int group_rows, size_t *bytes);
int ce_sf_to_atoms(int format, uint8_t *atoms_dev, const uint8_t *scales_dev, int rows, int K,
                   int group_rows, ce_stream_t stream);

/* MXFP6 GEMM operand layout: every 16 E3M2 codes of a row (one byte each,
 * as ce_quantize_mxfp6 writes them) become 12 bytes of little-endian 6-bit
 * fields (value i at bits 6i..6i+5, the spec's packed bit order) followed by
 * 4 zero bytes: the form in which the tensor core reads E3M2 from shared
 * memory. ld_operand is a multiple of 16 bytes covering roundup(cols, 16). */
int ce_pack_mxfp6(uint8_t *operand_dev, const uint8_t *codes_dev, int rows, int cols, int ld_codes,
                  int ld_operand, ce_stream_t stream);

/* MXFP6 GEMM (decoder_lowprec.cu:93-110): D[m][n] = sum_k a[m][k] b[n][k]
 * with a, b E3M2 operands in the ce_pack_mxfp6 layout scaled per
 * 32 values by their UE8M0 scales (atoms: A grouped by 128 rows, B by
 * CE_BS_TILE_N), fp32 accumulation and output. K % 128 == 0; lda, ldb
 * multiples of 16. */
int ce_gemm_mxfp6(float *d_dev, const uint8_t *a_dev, const uint8_t *a_sf_dev,
                  const uint8_t *b_dev, const uint8_t *b_sf_dev, int M, int N, int K, int lda,
                  int ldb, int ldd, ce_stream_t stream);

/* NVFP4 GEMM (decoder_lowprec.cu:111-127): E2M1 codes two per byte
 * (ce_quantize_nvfp4 layout), UE4M3 scales per 16 values (atoms as above),
 * times alpha = a_scales[1] * b_scales[1] (the tensors' decode scales,
 * device memory, as written by ce_quantize_nvfp4; NULL = 1). K % 128 == 0;
 * lda_bytes, ldb_bytes multiples of 16. */
int ce_gemm_nvfp4(float *d_dev, const uint8_t *a_dev, const uint8_t *a_sf_dev,
                  const float *a_scales_dev, const uint8_t *b_dev, const uint8_t *b_sf_dev,
                  const float *b_scales_dev, int M, int N, int K, int lda_bytes, int ldb_bytes,
                  int ldd, ce_stream_t stream);

/* RMSNorm whose GEMM operand is written as E4M3 codes [rows][ld] with one
 * scale per row (the quantizer above applied to the normalized row, fused in
 * the same launch). out_dev (fp32 [rows][cols]) may be NULL. Needs cols % 4
 * == 0, cols <= 32768, ld % 16 == 0. */
int ce_rmsnorm_e4m3(float *out_dev, uint8_t *codes_dev, int ld, float *scales_dev,
                    const float *x_dev, const float *w_dev, int rows, int cols, float eps,
                    ce_stream_t stream);

/* D[m][n] = a_scale[m] * b_scale[n] * sum_k A[m][k] * B[n][k] with E4M3
 * operands (tcgen05 kind::f8f6f4, fp32 accumulation). lda, ldb multiples of
 * 16; a_scale / b_scale may be NULL (scale 1). */
int ce_gemm_e4m3(float *d_dev, const uint8_t *a_dev, const float *a_scale_dev,
                 const uint8_t *b_dev, const float *b_scale_dev, int M, int N, int K, int lda,
                 int ldb, int ldd, ce_stream_t stream);

/* Round-to-nearest-even conversion fp32 -> bf16 of a [rows][cols] matrix
 * into a [rows][ld_out] buffer; columns cols..ld_out-1 are written as 0.
 * (experiments/blackwell/lowprec/decoder_lowprec.cu:222-238, to_bf16_kernel.) */
int ce_convert_bf16(uint16_t *out_dev, const float *in_dev, int rows, int cols, int ld_out,
                    ce_stream_t stream);

/* RMSNorm that also writes the normalized rows as bf16 into a [rows][ld_bf16]
 * buffer (padding columns 0), the fused producer of the GEMM A operand.
 * out_dev may be NULL (bf16 only). */
int ce_rmsnorm_bf16(float *out_dev, uint16_t *out_bf16_dev, int ld_bf16, const float *x_dev,
                    const float *w_dev, int rows, int cols, float eps, ce_stream_t stream);

/* ------------------------------------------------------------------ */
/* Op-trio plan: rmsnorm -> GEMM on the normalized batch, plus softmax. */

/* A plan owns the prepared weights (converted once, like the reference's
 * setup-time weight conversion, decoder_lowprec.cu:573-579) and the
 * activation workspace for one shape and precision. Create and set_weights
 * allocate and may synchronize; everything else is enqueue-only. */
typedef struct ce_plan ce_plan;

int ce_plan_create(ce_plan **plan, int batch, int size, int rows, int precision);
int ce_plan_destroy(ce_plan *plan);

/* Converts the fp32 weight matrix [rows][size] (device) into the plan's
 * layout for its precision. Setup only (allocates on first call). */
int ce_plan_set_weights(ce_plan *plan, const float *w_dev, ce_stream_t stream);

/* out[b][r] = sum_k W[r][k] * xnorm[b][k], xnorm = rmsnorm(x, norm_w, eps).
 * normalized_dev (fp32 [batch][size]) may be NULL. */
int ce_plan_rmsnorm_gemm(ce_plan *plan, float *out_dev, float *normalized_dev,
                         const float *x_dev, const float *norm_w_dev, float eps,
                         ce_stream_t stream);

/* The two halves of ce_plan_trio, for callers that time or overlap them:
 * ce_plan_rows writes normalized (may be NULL), the plan's GEMM operand and,
 * when logits != NULL, softmax, in one launch; ce_plan_gemm multiplies the
 * plan's current operand by the prepared weights into out [batch][rows]. */
int ce_plan_rows(ce_plan *plan, float *normalized_dev, float *softmax_dev, const float *x_dev,
                 const float *norm_w_dev, const float *logits_dev, float eps,
                 ce_stream_t stream);
int ce_plan_gemm(ce_plan *plan, float *out_dev, ce_stream_t stream);

/* The rows stage of one rank of the row-shard layer (bf16 and fp8 plans):
 * the GEMM operand of every batch row (the rank's slice GEMM multiplies
 * the whole batch), but the fp32 normalized rows (normalized_dev may be
 * NULL) and, when logits != NULL, the softmax rows only for batch rows
 * [row_lo, row_hi) -- this rank's share of those row-independent outputs,
 * which nothing downstream exchanges. Pointers index the full batch. */
int ce_plan_rows_range(ce_plan *plan, float *normalized_dev, float *softmax_dev, const float *x_dev,
                       const float *norm_w_dev, const float *logits_dev, float eps, int row_lo, int row_hi,
                       ce_stream_t stream);

/* The plan's two GEMM operands as the tensor cores multiply them, written
 * back as fp32: a_dev [batch][size] from the operand of the latest
 * ce_plan_rows / ce_plan_trio / ce_plan_rmsnorm_gemm on this plan, w_dev
 * [rows][size] from the prepared weights. Each is codes x block scale x
 * tensor scale (MXFP6: UE8M0 per 32; NVFP4: UE4M3 per 16 and the fp32
 * decode scale), E4M3 code x row scale, bf16 widened, or the fp32 value
 * (TF32 plans: as stored; the tensor cores read 10 of its mantissa bits).
 * Either pointer may be NULL. The reference's implementation check computes
 * its CPU product on the dequantized operands the same way
 * (decoder_lowprec.cu:947-1102). Enqueue-only. */
int ce_plan_operands(ce_plan *plan, float *a_dev, float *w_dev, ce_stream_t stream);

/* rmsnorm -> bf16 tensor-core GEMM that allocates no device memory, for
 * callers that cannot call cudaMalloc: code running while a CUDA graph is
 * captured, processes whose allocator already owns the device memory, and
 * loops that cannot take cudaMalloc's implicit synchronization. No
 * counterpart in the reference (its harnesses allocate everything in setup).
 *   out[b][r] = sum_k W[r][k] * xnorm[b][k], xnorm = rmsnorm(x, norm_w, eps);
 *   normalized_dev (fp32 [batch][size]) may be NULL; w_bf16_dev holds W as
 *   bf16 [rows][ld_w] (ld_w >= size, a multiple of 8; ce_convert_bf16 makes
 *   it). The caller passes inputs and outputs; the bf16 normalized operand
 *   lives in one fixed 8 MiB device array of the library (4,194,304 bf16
 *   values), which every GPU that loads the library holds until exit.
 *   batch x roundup(size, 64) above that limit returns CE_ERR_USAGE.
 * The first call on a device looks up that array's device address (once per
 * device, with the device current) and keeps it for the life of the
 * process; make that first call before any stream capture. A device reset
 * (cudaDeviceReset) frees the array, so do not call this entry point on a
 * device after resetting it. All calls share the array: calls that overlap
 * on the GPU (two streams, two host threads) race on it and must be
 * serialized by the caller. The GEMM reads only the first `size` columns of
 * each operand row, which the same call writes first, so no clearing is
 * needed. */
int ce_rmsnorm_gemm_bf16_noalloc(float *out_dev, float *normalized_dev, const float *x_dev,
                                 const float *norm_w_dev, const uint16_t *w_bf16_dev, int ld_w,
                                 int batch, int size, int rows, float eps, ce_stream_t stream);

/* One step of the BASELINE op trio: normalized = rmsnorm(x), softmax of an
 * independent logits buffer, out = GEMM of the normalized batch. */
int ce_plan_trio(ce_plan *plan, float *normalized_dev, float *softmax_dev, float *out_dev,
                 const float *x_dev, const float *norm_w_dev, const float *logits_dev,
                 float eps, ce_stream_t stream);

/* The plan's GEMM with the output row stride given: out_dev [batch][ldd],
 * ldd >= the plan's rows, e.g. a column block of a wider output or one
 * rank's slot of the row-shard staging buffer (ce_allgather_rows). */
int ce_plan_gemm_ld(ce_plan *plan, float *out_dev, int ldd, ce_stream_t stream);

/* ------------------------------------------------------------------ */
/* Row-shard (tensor-parallel) layer of the op-trio GEMM.               */
/* The reference runs this GEMM (the classifier, decoder.cu:83-125 and    */
/* decoder_lowprec.cu:85-127) on one GPU and has no multi-GPU code. Here  */
/* W's rows are split into contiguous slices over the ranks of one node   */
/* (rank r of n holds rows [lo_r, hi_r): the first rows % n ranks take    */
/* one extra row), every rank multiplies the full normalized batch by its */
/* slice with a plan of hi_r - lo_r rows, and the slices are joined into  */
/* every rank's out [batch][rows].                                        */

/* [lo, hi) of rank's slice of `rows`. */
int ce_shard_bounds(int rows, int world, int rank, int *lo, int *hi);

/* Bounded device waits (2 s by default) give up after `seconds` instead,
 * for kernels launched afterwards on the current device; a wait that gives
 * up is reported as CE_ERR_TIMEOUT by ce_device_status / ce_llama_status.
 * The reference's stream-K consumer spins without a limit
 * (applications/loom_private/decoder/decoder_optimized.cu:391-394).
 * Setup call. */
int ce_set_wait_limit(double seconds);

/* NCCL join. The library binds at run time to the libnccl.so.2 the process
 * has already loaded (the caller's: PyTorch's, or the one a C++ host links
 * with -lnccl) and never loads a second copy; until one is loaded these
 * return CE_ERR_USAGE. A caller without a communicator makes one: rank 0 calls
 * ce_nccl_unique_id, sends the CE_NCCL_ID_BYTES to the other ranks, and
 * every rank calls ce_nccl_comm_init (setup calls). */
#define CE_NCCL_ID_BYTES 128
int ce_nccl_version(int *version);
int ce_nccl_unique_id(void *id_out);
int ce_nccl_comm_init(void **comm_out, int world, int rank, const void *id);
int ce_nccl_comm_destroy(void *comm);

/* Floats of the staging buffer of ce_allgather_rows: world x batch x
 * ceil(rows / world). */
int ce_allgather_staging_floats(int batch, int rows, int world, size_t *floats);

/* Joins the ranks' slices: staging_dev [world][batch][ceil(rows/world)]
 * holds this rank's slice [batch][hi - lo] in slot `rank` (written there by
 * ce_plan_gemm_ld with ldd = ceil(rows / world)); an in-place ncclAllGather
 * on `comm` (the caller's ncclComm_t of these ranks, rank `rank` of `world`)
 * fills every slot, then a kernel scatters the slots into out_dev
 * [batch][rows]. Enqueue-only (graph capturable: NCCL collectives are). */
int ce_allgather_rows(void *comm, float *out_dev, float *staging_dev, int batch, int rows, int world, int rank,
                      ce_stream_t stream);

/* Peer-memory join fused into the GEMM. Each rank opens an exchange that
 * holds its out [batch][rows] (device memory shared by CUDA IPC) and writes
 * its IPC handle (CE_IPC_HANDLE_BYTES) to handle_out; the caller gathers the
 * handles of all ranks in rank order and passes them to ce_rowx_connect,
 * which maps the peers' exchanges (plain NVLink loads and stores; no
 * multicast object). ce_plan_gemm_rowx then runs this rank's slice GEMM
 * (a plan of hi - lo rows: bf16, tf32 or fp8) whose epilogue stores every
 * output tile into all ranks' outputs as it leaves tensor memory, and
 * ce_rowx_wait waits (bounded) until every peer's slice of the same call
 * has landed here; after it, ce_rowx_output's buffer holds the full
 * product. Ordering: a rank's GEMM stores into a peer only after that
 * peer's GEMM of the same call has started, i.e. after every consumer the
 * peer enqueued before it has read the previous product. Every rank makes
 * the same sequence of calls. 2 <= world <= 8. open / connect / close are
 * setup calls; ce_plan_gemm_rowx and ce_rowx_wait are enqueue-only (the
 * exchange count lives in device memory). */
/* ce_rowx_put is the same join with the copies on the copy engines instead
 * of the GEMM's epilogue: the caller writes this rank's slice into its own
 * output (ce_plan_gemm_ld into ce_rowx_output's buffer + lo, ldd = rows),
 * then ce_rowx_put enqueues a readiness handshake with the peers (bounded
 * wait), one strided cudaMemcpy2DAsync of the slice into each peer's output
 * over NVLink -- each on an internal stream of the exchange, forked from and
 * joined back to `stream` by events, so several copy engines run at once --
 * and a kernel that signals the peers; ce_rowx_wait as above. Enqueue-only;
 * one host thread at a time per exchange. */
typedef struct ce_rowx ce_rowx;
int ce_rowx_open(ce_rowx **x, int batch, int rows, int world, int rank, void *handle_out);
int ce_rowx_connect(ce_rowx *x, const void *handles);
int ce_rowx_output(ce_rowx *x, float **out_dev, int *lo, int *hi);
int ce_plan_gemm_rowx(ce_plan *plan, ce_rowx *x, ce_stream_t stream);
int ce_rowx_wait(ce_rowx *x, ce_stream_t stream);
int ce_rowx_put(ce_rowx *x, ce_stream_t stream);
int ce_rowx_close(ce_rowx *x);

/* ------------------------------------------------------------------ */
/* loom_private llama2c decoder (applications/loom_private/decoder/).   */

/* A decoder workload: B sequences decoded greedily for S dependent steps
 * through rmsnorm -> classifier -> softmax + first argmax, the token fed back
 * on the device. Mirrors the reference's lp::Workload
 * (applications/loom_private/common/lp_harness.cuh:240-267) as implemented by
 * decoder.cu:200-367. */
typedef struct ce_decoder ce_decoder;

/* The dimension and precision checks of ce_decoder_create alone, with the
 * limits and messages of make_decoder (decoder.cu:369-408; device limit 160
 * GiB): CE_OK or CE_ERR_USAGE with the message in ce_last_error. Makes no
 * CUDA call, so a front end can reject a shape before it touches the device. */
int ce_decoder_validate(int64_t batch, int64_t width, int64_t vocab, int64_t steps, int precision);

/* Validates the dimensions with the limits and messages of make_decoder
 * (decoder.cu:369-408; the device limit is raised to B200 memory: 160 GiB),
 * allocates every buffer, generates the synthetic model on the device
 * (init_model_kernel, decoder.cu:31-43) and writes the prompts b mod vocab
 * into the decoder's pinned buffer. precision: CE_PREC_FP32 (the contract's
 * bitwise order), CE_PREC_TF32 (width % 4 == 0) or CE_PREC_BF16. Setup call:
 * allocates and synchronizes the stream. */
int ce_decoder_create(ce_decoder **dec, int64_t batch, int64_t width, int64_t vocab, int64_t steps,
                      int precision, ce_stream_t stream);
int ce_decoder_destroy(ce_decoder *dec);

/* Replaces the synthetic model by caller weights (device fp32: embedding and
 * classifier [vocab][width], norm weight [width]); setup call. */
int ce_decoder_set_model(ce_decoder *dec, const float *embedding_dev, const float *classifier_dev,
                         const float *norm_w_dev, ce_stream_t stream);

/* Token reset from the resident prompts, then every step (decoder.cu:276-296).
 * Capturable. */
int ce_decoder_enqueue_compute(ce_decoder *dec, ce_stream_t stream);

/* Prompt upload (pinned H2D), compute, generated-token download (pinned D2H)
 * (decoder.cu:267-274). Capturable. */
int ce_decoder_enqueue_application(ce_decoder *dec, ce_stream_t stream);

/* 0xFF into every output, the device prompts and tokens, and the pinned
 * generated buffer (decoder.cu:298-312); synchronizes the stream. */
int ce_decoder_poison(ce_decoder *dec, ce_stream_t stream);

/* Synchronous diagnostics copy of the outputs into host memory (any pointer
 * may be NULL): generated [batch][steps] (from the pinned buffer of the last
 * application scope, or from the device when from_device != 0), normalized
 * [steps][batch][width], logits and probabilities [steps][batch][vocab]
 * (decoder.cu:318-331). */
int ce_decoder_copy_outputs(ce_decoder *dec, int from_device, int32_t *generated_host,
                            float *normalized_host, float *logits_host,
                            float *probabilities_host);

/* The reference's host-side fault hook (decoder.cu:346-358): fault 1 flips
 * the low bit of the last generated token in the pinned buffer; 0 does
 * nothing; 2 and 3 are applied by the caller to its diagnostics copy. */
int ce_decoder_inject_fault(ce_decoder *dec, int fault);

/* ---------------------------------------------------------------------------
 * Llama-2 decoder step (the full transformer of the north star's "loom_private
 * llama2c decoder step": attention over the KV cache, SwiGLU FFN, classifier;
 * the reference runs only its final rmsnorm -> classifier -> argmax stage,
 * applications/loom_private/decoder/decoder.cu:267-296). Batched greedy decode:
 * every sequence of the batch is at the same position. Weights bf16
 * [out][in], residual stream fp32, KV cache bf16 [layer][batch][kv_head]
 * [seq_len][head_size]. Field names follow llama2.c's Config.
 */
typedef struct ce_llama ce_llama;

typedef struct ce_llama_config {
  int32_t dim;        /* model width; multiple of 8 */
  int32_t hidden_dim; /* SwiGLU width; multiple of 8 */
  int32_t n_layers;
  int32_t n_heads;    /* head size dim / n_heads must be 64 or 128 */
  int32_t n_kv_heads; /* divides n_heads (grouped-query attention) */
  int32_t vocab_size; /* multiple of 4 */
  int32_t seq_len;    /* KV cache positions */
} ce_llama_config;

/* Tensors readable / writable through ce_llama_read / ce_llama_write. */
#define CE_LLAMA_TOK_EMB 0    /* bf16 [vocab][dim] */
#define CE_LLAMA_WQKV 1       /* bf16 [dim + 2 kv_dim][dim] of a layer: rows q, k, v */
#define CE_LLAMA_WO 2         /* bf16 [dim][dim] of a layer */
#define CE_LLAMA_W13 3        /* bf16 [2 hidden][dim] of a layer: rows w1_0, w3_0, w1_1, w3_1, ... */
#define CE_LLAMA_W2 4         /* bf16 [dim][hidden] of a layer */
#define CE_LLAMA_RMS_ATT 5    /* fp32 [dim] of a layer */
#define CE_LLAMA_RMS_FFN 6    /* fp32 [dim] of a layer */
#define CE_LLAMA_RMS_FINAL 7  /* fp32 [dim] */
#define CE_LLAMA_WCLS 8       /* bf16 [vocab][dim] */
#define CE_LLAMA_KCACHE 9     /* bf16 [batch][kv_heads][seq_len][head_size] of a layer */
#define CE_LLAMA_VCACHE 10    /* same */
#define CE_LLAMA_LOGITS 11    /* fp32 [batch][vocab] of the last step */
#define CE_LLAMA_TOKENS 12    /* int32 [batch]: current token of each sequence */
#define CE_LLAMA_GENERATED 13 /* int32 [batch][max_steps]: token of each step (-1 unset) */
#define CE_LLAMA_POS 14       /* int32: position of the next step */
#define CE_LLAMA_RESIDUAL 15  /* fp32 [batch][dim]: residual stream after the last layer */

/* Segments of one decode step of a row-sharded model (ce_llama_enqueue_segment). */
#define CE_LLAMA_SEG_ATTN 0    /* residual + RMSNorm, this rank's QKV rows, RoPE, KV append,
                                  attention of its heads into its slot of the att exchange */
#define CE_LLAMA_SEG_OPROJ 1   /* gathered att -> this rank's wo rows -> its slot of the delta exchange */
#define CE_LLAMA_SEG_FFN_IN 2  /* residual + RMSNorm, this rank's w1|w3 pairs, SwiGLU -> its hb slot */
#define CE_LLAMA_SEG_FFN_OUT 3 /* gathered hb -> this rank's w2 rows -> its delta slot */
#define CE_LLAMA_SEG_HEAD 4    /* residual + final RMSNorm, this rank's classifier rows, its
                                  greedy candidate -> its top slot */
#define CE_LLAMA_SEG_PICK 5    /* gathered candidates -> tokens and generated; advance */

/* Shape and memory checks of ce_llama_create alone (no CUDA call). */
int ce_llama_validate(const ce_llama_config *cfg, int batch, int max_steps, int precision);

/* Allocates weights, KV cache and buffers for `batch` sequences and up to
 * max_steps generated tokens per start. precision CE_PREC_BF16 (bf16
 * weights, bf16 GEMM operands) or CE_PREC_NVFP4_E2M1 (every GEMM weight
 * NVFP4, expanded to fp16 inside the W4A16 GEMM, fp16 GEMM operands; the
 * token embedding stays bf16; dim and hidden_dim multiples of 64). */
int ce_llama_create(ce_llama **model, const ce_llama_config *cfg, int batch, int max_steps,
                    int precision, ce_stream_t stream);
int ce_llama_destroy(ce_llama *model);

/* Random model on the device: every matrix N(0, weight_std) (bf16, or fp32
 * quantized to NVFP4 by the ce_quantize_nvfp4 rule per matrix), RMSNorm
 * weights 1, and KV positions [0, kv_fill) of every layer, sequence and head
 * N(0, 1) (bf16), the rest of the cache 0. Deterministic in seed. */
int ce_llama_init_random(ce_llama *model, uint64_t seed, float weight_std, int kv_fill,
                         ce_stream_t stream);

/* Sets the current token of every sequence (host int32 [batch]) and the
 * position of the next step, and clears the generated tokens. Synchronous. */
int ce_llama_start(ce_llama *model, const int32_t *tokens_host, int pos, ce_stream_t stream);

/* One decode step for the whole batch: reads each sequence's current token
 * and the device position, appends k and v at that position, writes the
 * logits, the greedy next token (first maximum) into the current tokens and
 * generated[b][step], and advances position and step on the device.
 * Capturable: a captured step replays for every token. */
int ce_llama_enqueue_step(ce_llama *model, ce_stream_t stream);

/* Row-sharded tensor parallelism over `world` ranks (one process per GPU):
 * rank `rank` holds the rows of every weight that produce its slice of each
 * output (n_heads / world query heads and n_kv_heads / world KV heads, dim /
 * world rows of wo and w2, hidden_dim / world interleaved w1|w3 pairs,
 * vocab_size / world classifier rows) and the KV cache of its heads, and
 * generates exactly those rows of the same global random model as an
 * unsharded one (NVFP4: quantized over the whole matrix). world 1 is
 * ce_llama_create. The north star's "sharded by output rows ... joined by an
 * all-gather"; the reference has no multi-GPU code. */
int ce_llama_validate_shard(const ce_llama_config *cfg, int batch, int max_steps, int precision,
                            int rank, int world);
int ce_llama_create_shard(ce_llama **model, const ce_llama_config *cfg, int batch, int max_steps,
                          int precision, int rank, int world, ce_stream_t stream);

/* ce_llama_create_shard with flags. CE_LLAMA_REPRODUCIBLE_SPLITS: the shard
 * splits its attention and its split-K GEMMs as the unsharded model does
 * (the counts of world 1), so every value it computes is summed in the
 * unsharded order and the sharded step gives the unsharded model's bits
 * (logits, tokens, residual stream). Without it each shard picks the splits
 * that fill the GPU for its own slice, which reassociates those fp32 sums. */
#define CE_LLAMA_REPRODUCIBLE_SPLITS 1
int ce_llama_create_shard_ex(ce_llama **model, const ce_llama_config *cfg, int batch, int max_steps,
                             int precision, int rank, int world, int flags, ce_stream_t stream);

/* Peer-memory exchange for a sharded model, instead of caller-bound buffers
 * joined by all-gathers: ce_llama_exchange_open allocates this rank's
 * exchange block (the four slot arrays and one flag per kind and sending
 * rank) and writes its CUDA IPC handle (CE_IPC_HANDLE_BYTES) to handle_out;
 * after every rank has opened, each passes all ranks' handles (rank order,
 * world x CE_IPC_HANDLE_BYTES) to ce_llama_exchange_connect, which maps the
 * peers' blocks. From then on the segments exchange by themselves: after
 * each producer a put copies this rank's slot into every peer's block over
 * NVLink and stores the exchange's epoch into the peers' flags; before each
 * consumer a wait spins (bounded; ce_llama_status reports a timeout) until
 * every peer's flag is current. No NCCL call, so a captured step graph holds
 * only kernels. Every rank must call ce_llama_start the same number of times
 * (the epoch carries a run generation). Replaces the ncclAllGather joins of
 * the row-sharded step (output-row sharding of the classifier GEMM,
 * decoder.cu:83-125, extended to every layer of the step). */
#define CE_IPC_HANDLE_BYTES 64
int ce_llama_exchange_open(ce_llama *model, void *handle_out);
int ce_llama_exchange_connect(ce_llama *model, const void *handles);

/* Caller-owned device exchange buffers of a sharded step, all-gathered by
 * the caller between segments (each rank writes its own slot r):
 * att   16-bit [world][batch][dim / world]         (after SEG_ATTN)
 * delta fp32   [world][batch][dim / world]         (after SEG_OPROJ, SEG_FFN_OUT)
 * hb    16-bit [world][batch][hidden_dim / world]  (after SEG_FFN_IN)
 * top   fp32   [world][batch][2] (value, index bits) (after SEG_HEAD).
 * A step: for each layer ATTN, gather att, OPROJ, gather delta, FFN_IN,
 * gather hb, FFN_OUT, gather delta; then HEAD, gather top, PICK. */
int ce_llama_bind_exchange(ce_llama *model, uint16_t *att_dev, float *delta_dev, uint16_t *hb_dev,
                           float *top_dev);
int ce_llama_enqueue_segment(ce_llama *model, int segment, int layer, ce_stream_t stream);

/* Prompt prefill, the step before decoding (the reference's decoder takes a
 * one-token prompt per sequence and resets its tokens from it,
 * decoder.cu:264-277; a longer prompt would otherwise take one decode step
 * per token). ce_llama_enqueue_prefill runs every sequence's prompt
 * prompt_dev int32 [batch][prompt_len] (device) at positions pos ..
 * pos + prompt_len - 1 (pos: the device position, ce_llama_start's or after
 * earlier steps) in chunks of max_rows / batch positions: the layer GEMMs
 * with M = batch x chunk positions, RoPE and KV append of every row, causal
 * attention of each position over the cache up to itself; then the final
 * RMSNorm, classifier and token choice (greedy, or the sampler) of each
 * sequence's last prompt position, as a decode step would make it: the
 * chosen token goes to the tokens and to generated[step], the position
 * advances by prompt_len and the step by 1, so decoding continues with
 * ce_llama_enqueue_step. Capturable; allocates nothing (the chunk
 * workspace comes from ce_llama_prefill_reserve, max_rows in
 * [batch, 65535], a setup call that allocates). Unsharded models only.
 * After a prefill the RESIDUAL tensor is not the last position's. A prompt
 * running past the cache is reported by ce_llama_status, as for a step. */
int ce_llama_prefill_reserve(ce_llama *model, int max_rows);
/* Prefill attention kernel: 0 (default) the tensor-core kernel (tcgen05,
 * scores and weights in tensor memory), 1 the SIMT kernel (the same
 * arithmetic in fp32 FMAs; a cross-check). */
int ce_llama_set_prefill_attention(ce_llama *model, int simt);
int ce_llama_enqueue_prefill(ce_llama *model, const int32_t *prompt_dev, int prompt_len,
                             ce_stream_t stream);

/* Global rows of rank's rows of weight `which` (CE_LLAMA_WQKV, _WO, _W13,
 * _W2, _WCLS) in local order; rows_out may be NULL to get the count. No CUDA call. */
int ce_llama_shard_rows(const ce_llama_config *cfg, int rank, int world, int which,
                        int32_t *rows_out, int *count);

/* Token choice of each step: temperature 0 (the default) picks the first
 * maximum logit; temperature > 0 samples from softmax(logits / temperature)
 * with the coin u = (mix64(seed ^ mix64(step * 0x9E3779B97F4A7C15 + row +
 * 1)) >> 40) / 2^24 (splitmix64 finalizer mix64): without top-p (0 or 1) the
 * first token in vocabulary order whose cumulative probability exceeds u;
 * with top_p in (0, 1), among the 1024 most probable tokens (ties to the
 * lower index) in descending order, the shortest prefix whose cumulative
 * probability exceeds top_p, and in it the first token whose cumulative
 * probability exceeds u times the prefix's mass (the nucleus sampler of
 * llama2.c, which the reference's decoder names but does not carry). Takes
 * effect for steps enqueued afterwards (a captured graph keeps the values it
 * was captured with). Single-GPU models only. */
int ce_llama_set_sampling(ce_llama *model, float temperature, float top_p, uint64_t seed);

/* Programmatic dependent launch between the kernels of a step (default on):
 * each kernel's prologue, and the GEMMs' L2 prefetch of their first weight
 * blocks, overlap the previous kernel's tail. 0 turns it off (plain stream
 * order); results are the same bits either way. */
int ce_llama_set_pdl(ce_llama *model, int enable);

/* Synchronous copies of a byte range of a tensor (CE_LLAMA_*; layer for the
 * per-layer ones) to and from host memory. */
int ce_llama_read(ce_llama *model, int which, int layer, void *host, int64_t offset, int64_t bytes);
int ce_llama_write(ce_llama *model, int which, int layer, const void *host, int64_t offset,
                   int64_t bytes);

/* Weight loading (setup calls: they allocate scratch and synchronize).
 * ce_llama_load takes one tensor as a global fp32 host array in the model's
 * global layout: the embedding [vocab][dim]; a norm; or a weight matrix in
 * the row orders above (WQKV = the q, k, v rows; W13 = w1 and w3 rows
 * interleaved; a sharded model takes its rows, ce_llama_shard_rows). The
 * bf16 model converts to bf16 on the device; the NVFP4 model quantizes the
 * whole global matrix on the device (tensor scale from its amax, UE4M3 per
 * 16 values, E2M1 codes: the reference's setup-time convert_weights,
 * decoder_lowprec.cu:573-579) and packs its rows.
 * ce_llama_load_nvfp4 (NVFP4 model) takes one matrix quantized ahead of
 * time, the offline conversion's output: codes_host [global rows][cols / 2]
 * (two E2M1 codes per byte, even column in the low nibble), scales_host
 * [global rows][cols / 16] (UE4M3) and alpha_host (encode, decode) tensor
 * scales; the weight is e2m1(code) * ue4m3(scale) * alpha[1]. */
int ce_llama_load(ce_llama *model, int which, int layer, const float *host);
int ce_llama_load_nvfp4(ce_llama *model, int which, int layer, const uint8_t *codes_host,
                        const uint8_t *scales_host, const float *alpha_host);

/* NVFP4 model only: host copies of one weight matrix (CE_LLAMA_WQKV, _WO,
 * _W13, _W2 of a layer, or _WCLS; this shard's rows): packed_host receives
 * it in the ce_w4t_pack layout (ce_w4t_packed_bytes(rows, cols) bytes; codes
 * and scales together), unused_host is not written; alpha = (encode,
 * decode) tensor scales; the weight is e2m1(code) * ue4m3(scale) *
 * alpha[1]. Any pointer may be NULL. */
int ce_llama_read_nvfp4(ce_llama *model, int which, int layer, uint8_t *packed_host,
                        uint8_t *unused_host, float *alpha_host);

/* Reads and clears the decode kernels' status word: CE_OK, CE_ERR_USAGE when
 * a step ran past the end of the KV cache, CE_ERR_TIMEOUT when a staging wait
 * gave up. Synchronizes the device. */
int ce_llama_status(void);

#ifdef __cplusplus
}
#endif

#endif /* CE_B200_H */
