/*
 * sdc_b200 — C ABI of the B200 (sm_100a) ABFT GEMM hot path.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream, enqueues its kernels on that stream and returns an SDC_* status.
 * Nothing here synchronises the host or allocates device memory: buffers and
 * scratch ("workspace") are owned by the caller, whose allocator orders their
 * reuse on the stream. On a non-zero status, sdc_last_error() returns a
 * thread-local message naming the violated contract.
 *
 * Each function names the reference operator it replaces (meiyou666/SDC,
 * paths relative to that project). The torch extension in sdc_b200/csrc
 * registers the reference's `sdc_cutlass::*` schemas on top of this ABI.
 *
 * Layout conventions (identical to the reference operators):
 *   FP8 operands   a: e4m3 [M,K] row-major, b_rows: e4m3 [N,K] row-major.
 *   NVFP4 operands a_packed: u8 [M,K/2], b_packed: u8 [N,K/2]; two e2m1 codes
 *                  per byte, even K index in the low nibble; sfa/sfb: ue4m3
 *                  block-16 scales in the 128x4 interleaved atom layout
 *                  (see sdc_nvfp4_scale_offset).
 *   Checksums      C = 2 channels for algorithm 0 (Classic), 1 for algorithm 1
 *                  (Sum). weights: fp32 [C,M]. Partials: fp32 [C, Tm, Np] with
 *                  Tm = ceil(M/128) and Np = ceil(N/64)*64 (FP8) or
 *                  ceil(N/128)*128 (NVFP4).
 */
#ifndef SDC_B200_H
#define SDC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* sdc_stream_t; /* == cudaStream_t */

enum sdc_status {
  SDC_OK = 0,
  SDC_ERR_INVALID = 1,            /* argument contract violated (message in sdc_last_error) */
  SDC_ERR_UNSUPPORTED_DEVICE = 2, /* current device is not sm_100 */
  SDC_ERR_CUDA = 3,               /* a CUDA runtime/driver call failed */
  SDC_ERR_WORKSPACE = 4,          /* workspace missing or too small */
  SDC_ERR_UNKNOWN_ALGORITHM = 5   /* algorithm id is not a compiled policy */
};

/* Checksum partial layouts for the input-fused ABFT GEMMs. */
enum sdc_reference_layout {
  /* predicted/magnitude[c, t, col] = contribution of M-tile t (rows
   * 128t..128t+127), exactly the reference operator's layout. */
  SDC_LAYOUT_TILE = 0,
  /* predicted/magnitude[c, t, col] = contribution of the 64-wide K slices s
   * with s % Tm == t, summed over ALL rows. The sum over t equals the TILE
   * layout's sum over t (up to fp32 rounding); finalize is unchanged. The
   * projection w^T A and the propagation run inside the GEMM launch (one extra read of A and of B, overlapped with the tensor-core
   * mainloop) instead of ~C/32 of the GEMM on CUDA cores; that launch
   * synchronises its CTAs twice, so two such launches must not run
   * concurrently on one GPU (different streams): one of them would wait until
   * its watchdog gives up and reports the call as detected. Short-M shapes
   * take the projection out of the GEMM instead (no such restriction), with
   * bit-identical results: at M <= 2048 with K >= 4 N (FP8, NVFP4) or NVFP4
   * with N >= 16 M, two kernels compute it before the GEMM; NVFP4 with
   * 2048 < M <= 4096 and N >= 16 M runs the projection and the prediction as
   * kernels before an observed-only GEMM. */
  SDC_LAYOUT_KSLICE = 1
};

/* Operand kinds of the generic (kind-dispatched) entry points. */
enum sdc_kind {
  SDC_KIND_FP8 = 0,       /* e4m3 tensorwise: scales unused, alpha device scalar */
  SDC_KIND_NVFP4 = 1,     /* packed e2m1 + ue4m3 scale atoms, alpha device scalar */
  SDC_KIND_FP8_BLOCK = 2  /* e4m3 + fp32 1x128 (A) / 128x128 (B) block scales, no alpha */
};

/* ---- library / device ------------------------------------------------- */

const char* sdc_last_error(void);
/* Returns SDC_OK when `device` is an sm_100 GPU this library was built for. */
int sdc_device_check(int device);
/* Reads and clears the device watchdog word of the current device: 0 when no
 * kernel gave up a bounded wait since the last call, otherwise the code of the
 * first wait that expired. Synchronises `stream`. */
int sdc_read_device_error(sdc_stream_t stream, int32_t* code);
/* Test hook (no counterpart in the reference): wait_limit_ns != 0 replaces the
 * 2 s limit of every bounded wait in later GEMM launches; pace_extra > 0 is
 * added to the prediction warps' pacing targets, which makes their wait
 * unreachable so that it expires. (0, 0) restores normal operation. Lets a
 * test check that an expired wait is reported in-band (hit bit 1, detected)
 * without hanging or faulting the GPU. */
int sdc_test_set_watchdog(uint64_t wait_limit_ns, int32_t pace_extra);
/* Test hook (no counterpart in the reference): how later K-slice launches
 * compute their prediction. 0 (default) chooses by shape; 1 forces the
 * in-GEMM path (projection and prediction inside the GEMM), 2 the standalone
 * kernels before an observed-only GEMM, 3 the projection by the standalone
 * kernels and the prediction inside the GEMM. All give bit-identical
 * partials; the hook lets a test check it. */
int sdc_test_set_kslice_path(int mode);

/* ---- quantisation (src/cutlass_gemm/quantization.py:99-162) ------------ */

/* Scratch bytes sdc_quantize_* needs for a [rows, cols] input. */
size_t sdc_quantize_workspace_bytes(int64_t rows, int64_t cols);

/* FP8 tensorwise quantize: replaces quantize(matrix, "fp8", global_scale)
 * (src/cutlass_gemm/quantization.py:114-140). x is fp32 (dtype 0) or bf16
 * (dtype 1) [rows, cols]. st = 448/amax(|x|) (1 when amax == 0) if use_amax,
 * else global_scale. codes = e4m3_rn_satfinite(x*st); *multiplier = st. */
int sdc_quantize_fp8(const void* x, int dtype, int64_t rows, int64_t cols,
                     int use_amax, float global_scale, uint8_t* codes,
                     float* multiplier, void* workspace, size_t workspace_bytes,
                     sdc_stream_t stream);

/* NVFP4 quantize: replaces quantize(matrix, "nvfp4", global_scale)
 * (src/cutlass_gemm/quantization.py:141-162) fused with the scale scatter of
 * _pack_scales (src/cutlass_gemm/backend.py:124-127). st = 2688/amax;
 * per 16-block: s = e4m3(amax16 * (st * (1/6))); codes =
 * e2m1_rn_satfinite(x * min(st/s, FLT_MAX)). Writes codes [rows, cols/2],
 * natural scales [rows, cols/16] (nullable) and MMA-layout scales (nullable,
 * sdc_nvfp4_scale_size(rows, cols) bytes, padding zeroed). */
int sdc_quantize_nvfp4(const void* x, int dtype, int64_t rows, int64_t cols,
                       int use_amax, float global_scale, uint8_t* codes,
                       uint8_t* scales, uint8_t* scales_mma, float* multiplier,
                       void* workspace, size_t workspace_bytes,
                       sdc_stream_t stream);

/* Row-sharded quantisation (extension; no counterpart in the reference): the
 * same casts as sdc_quantize_fp8 / sdc_quantize_nvfp4 with the "amax"
 * multiplier of the WHOLE matrix, taken from a device fp32 scalar `amax`
 * (max |x| over all shards, e.g. a MAX all-reduce of the shards' maxima), so
 * a shard's codes equal the unsharded matrix's rows bit for bit with no host
 * read of the maximum. No workspace. */
int sdc_quantize_fp8_global_amax(const void* x, int dtype, int64_t rows,
                                 int64_t cols, const float* amax,
                                 uint8_t* codes, float* multiplier,
                                 sdc_stream_t stream);
int sdc_quantize_nvfp4_global_amax(const void* x, int dtype, int64_t rows,
                                   int64_t cols, const float* amax,
                                   uint8_t* codes, uint8_t* scales,
                                   uint8_t* scales_mma, float* multiplier,
                                   sdc_stream_t stream);

/* ---- NVFP4 scale-factor layout (src/cutlass_gemm/csrc/gemm/nvfp4.cu:122-147)
 * Byte offset of natural scale (row, block) in the 128x4 atom layout, and the
 * layout's byte size for a [rows, k] operand. Host functions. */
int64_t sdc_nvfp4_scale_offset(int64_t row, int64_t block, int64_t k);
int64_t sdc_nvfp4_scale_size(int64_t rows, int64_t k);
/* Replaces sdc_cutlass_nvfp4_scale_layout: fills indices[rows*(k/16)]. */
int sdc_nvfp4_scale_layout(int64_t rows, int64_t k, int64_t* indices);
/* Device scatter of natural scales into the atom layout (zero padding);
 * replaces _pack_scales (src/cutlass_gemm/backend.py:124-127). */
int sdc_nvfp4_pack_scales(const uint8_t* scales, int64_t rows, int64_t k,
                          uint8_t* packed, sdc_stream_t stream);

/* ---- GEMMs -------------------------------------------------------------- */

/* Replaces sdc_cutlass_fp8_mm (src/cutlass_gemm/csrc/gemm/fp8.cu:96-139):
 * d = alpha * a . b_rows^T, fp32 column-major [M,N] (element (r,c) at
 * d[c*M + r]). alpha: device fp32 scalar. K % 16 == 0. */
int sdc_fp8_gemm(const uint8_t* a, const uint8_t* b_rows, int64_t m, int64_t n,
                 int64_t k, const float* alpha, float* d, sdc_stream_t stream);

/* Replaces sdc_cutlass_nvfp4_mm (src/cutlass_gemm/csrc/gemm/nvfp4.cu:150-200):
 * d = alpha * sum_k (a*sfa)(b*sfb), bf16 row-major [M,N]. K % 32 == 0. */
int sdc_nvfp4_gemm(const uint8_t* a_packed, const uint8_t* b_packed,
                   const uint8_t* sfa, const uint8_t* sfb, int64_t m, int64_t n,
                   int64_t k, const float* alpha, uint16_t* d,
                   sdc_stream_t stream);

/* ---- ABFT GEMMs --------------------------------------------------------
 * Common arguments:
 *   algorithm  0 = Classic (2 channels), 1 = Sum (1 channel); other values
 *              return SDC_ERR_UNKNOWN_ALGORITHM.
 *   weights    fp32 [C, M] row weights of the column checksums.
 *   row,col,bit  accumulator fault: all -1, or 0<=row<M, 0<=col<N, 0<=bit<32.
 *              The epilogue XORs bit `bit` of the post-alpha fp32 value at
 *              (row, col) before the checksum and the output cast.
 *   nonfinite  nullable int32[1]; zeroed, then set to 1 when a converted
 *              in-bounds output element is not finite.
 *   observed   fp32 [C,Tm,Np]: sum over the tile's rows of w_c[row]*value.
 *   hit        int32[1]: bit 0 set when the fault was applied; bit 1 set when
 *              the launch gave up a bounded wait (its outputs and partials
 *              are incomplete; finalize then reports detected and
 *              nonfinite, and `nonfinite`, when given, is set to 1).
 * Input-fused variants also write predicted = alpha * w^T A B and
 * magnitude = |alpha| * |w|^T |A| |B| partials in `reference_layout`.
 */

/* Workspace bytes of the input-fused ABFT GEMMs. */
size_t sdc_abft_workspace_bytes(int algorithm, int64_t m, int64_t n, int64_t k,
                                int reference_layout);

/* Replaces sdc_cutlass_abft_fp8_mm (src/cutlass_gemm/csrc/abft/fp8/fp8_observe.cu:113-190). */
int sdc_abft_fp8_gemm(const uint8_t* a, const uint8_t* b_rows, int64_t m,
                      int64_t n, int64_t k, const float* alpha, int algorithm,
                      const float* weights, int64_t row, int64_t col,
                      int64_t bit, int32_t* nonfinite, float* d,
                      float* observed, int32_t* hit, sdc_stream_t stream);

/* Replaces sdc_cutlass_abft_fp8_reference_mm
 * (src/cutlass_gemm/csrc/abft/fp8/fp8_reference.cu:123-216). */
int sdc_abft_fp8_reference_gemm(
    const uint8_t* a, const uint8_t* b_rows, int64_t m, int64_t n, int64_t k,
    const float* alpha, int algorithm, const float* weights, int64_t row,
    int64_t col, int64_t bit, int32_t* nonfinite, float* d, float* observed,
    int32_t* hit, float* predicted, float* magnitude, int reference_layout,
    void* workspace, size_t workspace_bytes, sdc_stream_t stream);

/* Replaces sdc_cutlass_abft_nvfp4_mm (src/cutlass_gemm/csrc/abft/nvfp4/nvfp4_observe.cu:159-245). */
int sdc_abft_nvfp4_gemm(const uint8_t* a_packed, const uint8_t* b_packed,
                        const uint8_t* sfa, const uint8_t* sfb, int64_t m,
                        int64_t n, int64_t k, const float* alpha,
                        int algorithm, const float* weights, int64_t row,
                        int64_t col, int64_t bit, int32_t* nonfinite,
                        uint16_t* d, float* observed, int32_t* hit,
                        sdc_stream_t stream);

/* Replaces sdc_cutlass_abft_nvfp4_reference_mm
 * (src/cutlass_gemm/csrc/abft/nvfp4/nvfp4_reference.cu:165-267). */
int sdc_abft_nvfp4_reference_gemm(
    const uint8_t* a_packed, const uint8_t* b_packed, const uint8_t* sfa,
    const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* alpha,
    int algorithm, const float* weights, int64_t row, int64_t col, int64_t bit,
    int32_t* nonfinite, uint16_t* d, float* observed, int32_t* hit,
    float* predicted, float* magnitude, int reference_layout, void* workspace,
    size_t workspace_bytes, sdc_stream_t stream);

/* ---- block-scaled FP8 (extension; the reference has no such operator) ----
 * e4m3 codes with one fp32 dequantisation scale per 128-wide K block of
 * `block_rows` rows: 1 x 128 for activations (A), 128 x 128 for weights (B,
 * stored as rows [N, K]). d = amax(|x|) / 448 (1 when amax == 0),
 * code = e4m3_rn_satfinite(x / d). cols (K) must be a multiple of 128.
 * scales: float [ceil(rows / block_rows)][cols / 128]. */
int sdc_quantize_fp8_block(const void* x, int dtype, int64_t rows,
                           int64_t cols, int block_rows, uint8_t* codes,
                           float* scales, sdc_stream_t stream);

/* D (bf16 row-major [M,N]) = sum over 128-wide K blocks kb of
 * scale_a[m][kb] * scale_b[n / 128][kb] * (A_kb . B_kb^T), each block
 * accumulated in fp32 on the tensor cores and the scaled sum kept in fp32. */
int sdc_fp8_block_gemm(const uint8_t* a, const uint8_t* b_rows,
                       const float* scale_a, const float* scale_b, int64_t m,
                       int64_t n, int64_t k, uint16_t* d, sdc_stream_t stream);

/* Block-scaled FP8 with the ABFT epilogue (observed checksums of the fp32
 * values before the bf16 cast; Np = ceil(N/128)*128), same fault and
 * nonfinite semantics as sdc_abft_fp8_gemm. */
int sdc_abft_fp8_block_gemm(const uint8_t* a, const uint8_t* b_rows,
                            const float* scale_a, const float* scale_b,
                            int64_t m, int64_t n, int64_t k, int algorithm,
                            const float* weights, int64_t row, int64_t col,
                            int64_t bit, int32_t* nonfinite, uint16_t* d,
                            float* observed, int32_t* hit, sdc_stream_t stream);

/* Block-scaled FP8 with the input-fused prediction in the K-slice layout
 * (the only layout offered; the projection uses the dequantised operands
 * code * scale). Workspace: sdc_abft_workspace_bytes(..., SDC_LAYOUT_KSLICE). */
int sdc_abft_fp8_block_reference_gemm(
    const uint8_t* a, const uint8_t* b_rows, const float* scale_a,
    const float* scale_b, int64_t m, int64_t n, int64_t k, int algorithm,
    const float* weights, int64_t row, int64_t col, int64_t bit,
    int32_t* nonfinite, uint16_t* d, float* observed, int32_t* hit,
    float* predicted, float* magnitude, void* workspace,
    size_t workspace_bytes, sdc_stream_t stream);

/* ---- BF16 GEMM and augmented BF16 ABFT ------------------------------------
 * bf16 operands (a [M,K] row-major, b_rows [N,K] row-major, K % 8 == 0),
 * fp32 accumulation on the tensor cores, d = a . b_rows^T as bf16 [M,N]
 * row-major. */

/* Replaces sdc_cutlass_mm for bf16 operands
 * (src/cutlass_gemm/csrc/gemm/fp32_bf16.cu:34-125; the reference's fp32
 * variant stays outside this library). */
int sdc_bf16_gemm(const uint16_t* a, const uint16_t* b_rows, int64_t m,
                  int64_t n, int64_t k, uint16_t* d, sdc_stream_t stream);

/* The encoding step of sdc_abft_bf16_augmented_gemm on its own (the
 * reference forms these rows inside its augmented mainloop,
 * src/cutlass_gemm/csrc/abft/fp32_bf16/bf16_augmented.h:200-320): for each
 * 128-row M-tile t and channel c, q[t*C + c][k] = bf16 (round to nearest
 * even) of the sum, in ascending order, of eight fp32 fma chains of
 * w_c[row] * A[row][k], each over a 16-row segment of the tile (rows
 * ascending, rows >= M absent). a: bf16 [M, K] row-major, K % 8 == 0; weights: bf16
 * [C, M]; q: bf16 [C * ceil(M/128), K]; a and q 16-byte aligned. */
int sdc_abft_augment_encode(const uint16_t* a, int64_t m, int64_t k,
                            int algorithm, const uint16_t* weights,
                            uint16_t* q, sdc_stream_t stream);

/* Workspace bytes of sdc_abft_bf16_augmented_gemm (256-byte aligned). */
size_t sdc_abft_augmented_workspace_bytes(int algorithm, int64_t m,
                                          int64_t k);

/* Replaces sdc_cutlass_abft_augmented_mm and _compact
 * (src/cutlass_gemm/csrc/abft/fp32_bf16/bf16_augmented.cu:12-162). The
 * checksum rows of every 128-row M-tile t, q[t*C + c] = bf16(w_c^T A_t)
 * (the order of sdc_abft_augment_encode), run as extra M-tiles of the
 * same GEMM; their fp32 results are predicted[c, t, :]. The data tiles'
 * epilogue applies the fault (XOR of bit `bit` of the fp32 value at
 * (row, col)) and writes observed = sum_rows w_c v and the output-side
 * magnitude sum_rows |w_c v|. weights: bf16 [C, M]. observed, predicted,
 * magnitude: fp32 [C, Tm, Np], Np = ceil(N/128)*128 (padding zero). hit:
 * nullable int32[1], zeroed, bit 0 = fault applied, bit 1 = a bounded wait
 * expired. tile_flags: nullable int32 [Tm, ceil(N/128)], zeroed, ORed with
 * bit 0 = fault applied and bit 1 = non-finite output in that block (the
 * packed finalize's status input). */
int sdc_abft_bf16_augmented_gemm(
    const uint16_t* a, const uint16_t* b_rows, int64_t m, int64_t n, int64_t k,
    int algorithm, const uint16_t* weights, int64_t row, int64_t col,
    int64_t bit, uint16_t* d, float* observed, float* predicted,
    float* magnitude, int32_t* hit, int32_t* tile_flags, void* workspace,
    size_t workspace_bytes, sdc_stream_t stream);

/* ---- row checksums and two-dimensional localisation (extension) ---------
 * The reference checks column sums only; these add C.e against A.(B^T e):
 * the GEMM epilogue also writes row_observed[b][m] = sum of row m's fp32
 * values (after the fault) over the 64 columns of block b, ascending, from
 * +0; sdc_abft_row_reference forms predicted_rows = alpha * A . u and
 * magnitude_rows = |alpha| * |A| . u_abs with u = e^T B, u_abs = e^T |B| (the
 * K-slice projection of B with unit weights); sdc_abft_locate2d decides the
 * rows like finalize decides the columns (threshold atol + rtol * magnitude,
 * no FMA, strict >, non-finite fails) and locates (row, col) when exactly one
 * row and one column fail and nothing is non-finite. */

/* The input-fused GEMM of `kind` (a_scales/b_scales as the kind's entry point
 * takes them) plus row_observed fp32 [ceil(N/64)][M]. Other arguments as
 * sdc_abft_{fp8,nvfp4,fp8_block}_reference_gemm. */
int sdc_abft_reference_gemm_rows(
    int kind, const uint8_t* a, const void* a_scales, const uint8_t* b_rows,
    const void* b_scales, int64_t m, int64_t n, int64_t k, const float* alpha,
    int algorithm, const float* weights, int64_t row, int64_t col, int64_t bit,
    int32_t* nonfinite, void* d, float* observed, int32_t* hit,
    float* predicted, float* magnitude, int reference_layout,
    float* row_observed, void* workspace, size_t workspace_bytes,
    sdc_stream_t stream);

/* Workspace of sdc_abft_row_reference: u, u_abs for K rounded up to 64,
 * and the projection's partials of each 128-row band of B. */
size_t sdc_abft_row_workspace_bytes(int64_t n, int64_t k);
/* predicted_rows / magnitude_rows fp32 [M] of `kind`; alpha null for
 * SDC_KIND_FP8_BLOCK. */
int sdc_abft_row_reference(int kind, const uint8_t* a, const void* a_scales,
                           const uint8_t* b_rows, const void* b_scales,
                           int64_t m, int64_t n, int64_t k, const float* alpha,
                           float* predicted_rows, float* magnitude_rows,
                           void* workspace, size_t workspace_bytes,
                           sdc_stream_t stream);

/* Workspace of sdc_abft_locate2d. */
size_t sdc_abft_locate2d_workspace_bytes(void);
/* col_residual / col_threshold / col_flags: finalize's diagnostics outputs
 * ([C, N] and u8[5]). Writes row_residual / row_threshold [M] (nullable),
 * location int64[2] and located u8[1] (the element when exactly one row and
 * one column fail, else -1 / 0), row_flags u8[2] (a row failed, a row was
 * non-finite). */
int sdc_abft_locate2d(const float* row_observed, int64_t row_blocks,
                      const float* predicted_rows, const float* magnitude_rows,
                      int64_t m, float atol, float rtol,
                      const float* col_residual, const float* col_threshold,
                      int algorithm, int64_t n, const uint8_t* col_flags,
                      float* row_residual, float* row_threshold,
                      int64_t* location, uint8_t* located, uint8_t* row_flags,
                      void* workspace, size_t workspace_bytes,
                      sdc_stream_t stream);

/* ---- finalize (src/cutlass_gemm/csrc/abft/common/finalize.cu:55-319) ------
 * Sums the per-tile partials of each (channel, column) in ascending tile
 * order with IEEE round-to-nearest adds, then applies the policy
 *   res = obs - pred;  thr = override ? t : atol + (rtol * mag)  (no FMA)
 *   nonfinite = !finite(obs, pred, mag, res, thr)
 *   detected  = nonfinite || thr < 0 || |res| > thr
 * observed/predicted/magnitude: fp32 [C, m_tiles, padded_n] each (padding
 * columns are never read). reference: fp32 [2, C, n]; written when
 * use_reference == 0, read (first-call evidence) otherwise. residual and
 * threshold: fp32 [C, n], written when diagnostics != 0. thresholds: nullable
 * fp32 override, [1] (scalar_threshold=1) or [C, n]. Status inputs: either
 * tile_flags int32[flag_count] (bit0 hit, bit1 nonfinite; packed entry) or
 * hit_in/nonfinite_in int32[1] (input-fused entry). Outputs: flags u8[5] =
 * {detected, nonfinite, 0, 0, 0}, hit_out int32[1], location int64[2] = -1.
 */
size_t sdc_abft_finalize_workspace_bytes(int algorithm, int64_t n,
                                         int64_t m_tiles);
int sdc_abft_finalize(int algorithm, const float* observed,
                      const float* predicted, const float* magnitude,
                      int64_t m_tiles, int64_t padded_n, int64_t n,
                      const int32_t* tile_flags, int64_t flag_count,
                      const int32_t* hit_in, const int32_t* nonfinite_in,
                      float atol, float rtol, float* reference,
                      int use_reference, int diagnostics, float* residual,
                      float* threshold, const float* thresholds,
                      int scalar_threshold, uint8_t* flags, int32_t* hit_out,
                      int64_t* location, void* workspace,
                      size_t workspace_bytes, sdc_stream_t stream);

/* Allocation-free variant of sdc_abft_finalize (no counterpart in the
 * reference). For hosts that cannot allocate device memory when they run the
 * check, e.g. a plain C/FFI caller with no device allocator of its own: the
 * per-block scratch comes from a fixed 64 KiB device array inside this
 * library (allocated once per GPU that loads it, kept until process exit).
 * Same arguments and results as sdc_abft_finalize minus the workspace.
 * Limit: channels * ceil(n / 64) <= 16384 (n <= 524288 for Classic); larger
 * n returns SDC_ERR_INVALID without launching. The first call on a device
 * looks the array's address up with that device current; make that first
 * call before any stream capture. Every call shares the one array, so calls
 * that may overlap on the GPU (different streams, concurrent hosts) race:
 * serialise them. The entry point itself allocates nothing. */
int sdc_abft_finalize_noalloc(int algorithm, const float* observed,
                              const float* predicted, const float* magnitude,
                              int64_t m_tiles, int64_t padded_n, int64_t n,
                              const int32_t* tile_flags, int64_t flag_count,
                              const int32_t* hit_in,
                              const int32_t* nonfinite_in, float atol,
                              float rtol, float* reference, int use_reference,
                              int diagnostics, float* residual,
                              float* threshold, const float* thresholds,
                              int scalar_threshold, uint8_t* flags,
                              int32_t* hit_out, int64_t* location,
                              sdc_stream_t stream);

/* ---- localisation and single-error correction (extension) ---------------
 * Device restatement of the Classic ratio locator (src/abft/methods.py:
 * 201-237 of the reference; no reference operator exists for it). Inputs are
 * finalize's residual/threshold fp32 [2, n] and flags u8[5]; writes
 * location int64[2] ((row, col) or (-1, -1)) and located u8[1]. Only
 * meaningful for algorithm 0 (two channels: ones and row+1 weights). */
int sdc_abft_locate(const float* residual, const float* threshold,
                    const uint8_t* flags, int64_t m, int64_t n,
                    int64_t* location, uint8_t* located, sdc_stream_t stream);

/* Single-error correction: when *located != 0, recomputes output element
 * location = (row, col) as alpha * sum_k a[row,k] * b[col,k] in fp32 on CUDA
 * cores and overwrites it in d; sets corrected u8[1]. Replaces the
 * reference's full-GEMM recompute for a located single error. */
int sdc_abft_correct_fp8(const uint8_t* a, const uint8_t* b_rows, int64_t m,
                         int64_t n, int64_t k, const float* alpha,
                         const int64_t* location, const uint8_t* located,
                         float* d_colmajor, uint8_t* corrected,
                         sdc_stream_t stream);
int sdc_abft_correct_nvfp4(const uint8_t* a_packed, const uint8_t* b_packed,
                           const uint8_t* sfa, const uint8_t* sfb, int64_t m,
                           int64_t n, int64_t k, const float* alpha,
                           const int64_t* location, const uint8_t* located,
                           uint16_t* d_rowmajor, uint8_t* corrected,
                           sdc_stream_t stream);
/* Block-scaled FP8: sum_k (a * scale_a) * (b * scale_b), bf16 row-major d. */
int sdc_abft_correct_fp8_block(const uint8_t* a, const uint8_t* b_rows,
                               const float* scale_a, const float* scale_b,
                               int64_t m, int64_t n, int64_t k,
                               const int64_t* location, const uint8_t* located,
                               uint16_t* d_rowmajor, uint8_t* corrected,
                               sdc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SDC_B200_H */
