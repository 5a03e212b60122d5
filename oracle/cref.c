/*
 * CPU oracle (test infrastructure only; never linked into the product).
 *
 * Plain-C restatement of the order-sensitive fp32 arithmetic of the
 * reference's input-fused checksum ("mainloop reference"):
 *   src/cutlass_gemm/csrc/abft/fp8/fp8_reference.cuh:31-83
 *   src/cutlass_gemm/csrc/abft/nvfp4/nvfp4_reference.cuh:31-84
 * Per 128-row M-tile t and checksum channel c:
 *   q[c][k]     = fmaf(w[c][row], A[row][k], q)   over rows ascending
 *   q_abs[c][k] = fmaf(|w|, |A|, q_abs)
 *   r[c][n]     = fmaf(q[c][k], B[n][k], r)       over k ascending
 *   a[c][n]     = fmaf(q_abs[c][k], |B[n][k]|, a)
 *   predicted = alpha * r, magnitude = |alpha| * a  (columns < padded_n;
 *   columns >= n stay alpha * 0)
 * C99 fmaf is correctly rounded, and this file is compiled with
 * -ffp-contract=off so every other operation is a single IEEE fp32 op.
 *
 * kind 2 is block-scaled FP8 (an sdc_b200 extension; 1 x 128 A and
 * 128 x 128 B fp32 scales): the operands are the dequantised values
 * code * scale and alpha is 1.
 *
 * The KSLICE entry restates the sdc_b200 fast layout (an extension with no
 * reference counterpart): q summed over tiles ascending, then per slot
 * t = s % Tm over its 64-wide K slices s (slices ascending, k ascending).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float decode_e4m3(uint8_t b) {
  const int sign = b & 0x80;
  const int exp = (b >> 3) & 0xF;
  const int man = b & 7;
  float v;
  if (exp == 0xF && man == 7) return NAN;
  if (exp == 0) v = ldexpf((float)man, -9);
  else v = ldexpf(1.0f + (float)man / 8.0f, exp - 7);
  return sign ? -v : v;
}

static float decode_e2m1(int nib) {
  static const float table[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = table[nib & 7];
  return (nib & 8) ? -v : v;
}

static int64_t sf_offset(int64_t row, int64_t block, int64_t k) {
  const int64_t k_atoms = (k + 63) / 64;
  return ((row >> 7) * k_atoms + (block >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (block & 3);
}

/* kind 0: e4m3 [rows, k]; kind 1: packed e2m1 [rows, k/2] with scale atoms;
 * kind 2 / 3: block-scaled e4m3 with fp32 scales [rows / r, k / 128] for
 * r = 1 (kind 2, the A operand) / 128 (kind 3, B rows): code * scale, one
 * fp32 rounding. */
static float value_at(int kind, const uint8_t* x, const uint8_t* sf, int64_t row, int64_t kk, int64_t k) {
  if (kind == 0) return decode_e4m3(x[row * k + kk]);
  if (kind >= 2) {
    const float* scales = (const float*)sf;
    const int64_t r = kind == 2 ? row : row / 128;
    return decode_e4m3(x[row * k + kk]) * scales[r * (k / 128) + kk / 128];
  }
  const uint8_t byte = x[row * (k / 2) + kk / 2];
  const float code = decode_e2m1((kk & 1) ? (byte >> 4) : (byte & 15));
  return code * decode_e4m3(sf[sf_offset(row, kk / 16, k)]);
}

/* All k values of one operand row (same values as value_at, one row at a time). */
static void decode_row(int kind, const uint8_t* x, const uint8_t* sf, int64_t row, int64_t k, float* out) {
  static float lut[256];
  static int lut_ready = 0;
  if (!lut_ready) {
    for (int i = 0; i < 256; ++i) lut[i] = decode_e4m3((uint8_t)i);
    lut_ready = 1;
  }
  if (kind == 0) {
    const uint8_t* r = x + row * k;
    for (int64_t kk = 0; kk < k; ++kk) out[kk] = lut[r[kk]];
  } else if (kind >= 2) {
    const float* scales = (const float*)sf;
    const int64_t srow = kind == 2 ? row : row / 128;
    const uint8_t* r = x + row * k;
    for (int64_t kk = 0; kk < k; ++kk) out[kk] = lut[r[kk]] * scales[srow * (k / 128) + kk / 128];
  } else {
    const uint8_t* r = x + row * (k / 2);
    for (int64_t kk = 0; kk < k; ++kk) {
      const uint8_t byte = r[kk / 2];
      const float code = decode_e2m1((kk & 1) ? (byte >> 4) : (byte & 15));
      out[kk] = code * lut[sf[sf_offset(row, kk / 16, k)]];
    }
  }
}

/* q layout: [(c*2 + h) * tiles * k + t * k + kk]. */
static void encode_tiles(int kind, const uint8_t* a, const uint8_t* sfa, int64_t m, int64_t k,
                         const float* w, int channels, float* q) {
  const int64_t tiles = (m + 127) / 128;
  for (int64_t t = 0; t < tiles; ++t) {
    for (int64_t kk = 0; kk < k; ++kk) {
      for (int c = 0; c < channels; ++c) {
        float enc = 0.f, mag = 0.f;
        for (int64_t r = 0; r < 128 && t * 128 + r < m; ++r) {
          const int64_t row = t * 128 + r;
          const float v = value_at(kind, a, sfa, row, kk, k);
          const float wt = w[c * m + row];
          enc = fmaf(wt, v, enc);
          mag = fmaf(fabsf(wt), fabsf(v), mag);
        }
        q[((c * 2 + 0) * tiles + t) * k + kk] = enc;
        q[((c * 2 + 1) * tiles + t) * k + kk] = mag;
      }
    }
  }
}

int oracle_tile_reference(int kind, const uint8_t* a, const uint8_t* sfa, const uint8_t* b,
                          const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* w,
                          int channels, float alpha, float* pred, float* mag, int64_t padded_n) {
  const int64_t tiles = (m + 127) / 128;
  float* q = (float*)malloc(sizeof(float) * channels * 2 * tiles * k);
  if (!q) return 1;
  encode_tiles(kind, a, sfa, m, k, w, channels, q);
  for (int c = 0; c < channels; ++c) {
    for (int64_t t = 0; t < tiles; ++t) {
      const float* qe = q + ((c * 2 + 0) * tiles + t) * k;
      const float* qa = q + ((c * 2 + 1) * tiles + t) * k;
      for (int64_t col = 0; col < padded_n; ++col) {
        float r = 0.f, s = 0.f;
        if (col < n) {
          for (int64_t kk = 0; kk < k; ++kk) {
            const float v = value_at(kind == 2 ? 3 : kind, b, sfb, col, kk, k);
            r = fmaf(qe[kk], v, r);
            s = fmaf(qa[kk], fabsf(v), s);
          }
        }
        pred[(c * tiles + t) * padded_n + col] = alpha * r;
        mag[(c * tiles + t) * padded_n + col] = fabsf(alpha) * s;
      }
    }
  }
  free(q);
  return 0;
}

int oracle_kslice_reference(int kind, const uint8_t* a, const uint8_t* sfa, const uint8_t* b,
                            const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* w,
                            int channels, float alpha, float* pred, float* mag, int64_t padded_n) {
  const int64_t tiles = (m + 127) / 128;
  const int64_t slices = (k + 63) / 64;
  float* qf = (float*)calloc((size_t)channels * 2 * k, sizeof(float));
  float* lanes = (float*)malloc(sizeof(float) * channels * 2 * 8 * k); /* [c][h][lane][k] */
  float* row_v = (float*)malloc(sizeof(float) * k);
  if (!qf || !lanes || !row_v) {
    free(qf);
    free(lanes);
    free(row_v);
    return 1;
  }
  /* q over all rows in the projection kernel's order: bands of 128 rows; in a
   * band, 8 row lanes l each run an fma chain over rows band_start + l, + 8,
   * ... (ascending), combined as ((p0 + p1) + (p2 + p3)) + ((p4 + p5) +
   * (p6 + p7)); q = ((band_0 + band_1) + ...) + band_last. Rows are walked in
   * order (each fma chain keeps its own accumulator), which is the same
   * arithmetic as walking each chain separately. */
  const int64_t bands = (m + 127) / 128;
  for (int64_t bnd = 0; bnd < bands; ++bnd) {
    const int64_t begin = bnd * 128, end = begin + 128 < m ? begin + 128 : m;
    memset(lanes, 0, sizeof(float) * channels * 2 * 8 * k);
    for (int64_t row = begin; row < end; ++row) {
      const int l = (int)((row - begin) & 7);
      decode_row(kind, a, sfa, row, k, row_v);
      for (int c = 0; c < channels; ++c) {
        const float wv = w[c * m + row], wa = fabsf(wv);
        float* e = lanes + ((c * 2 + 0) * 8 + l) * k;
        float* g = lanes + ((c * 2 + 1) * 8 + l) * k;
        for (int64_t kk = 0; kk < k; ++kk) {
          e[kk] = fmaf(wv, row_v[kk], e[kk]);
          g[kk] = fmaf(wa, fabsf(row_v[kk]), g[kk]);
        }
      }
    }
    for (int c = 0; c < channels; ++c) {
      for (int h = 0; h < 2; ++h) {
        const float* p = lanes + (c * 2 + h) * 8 * k;
        float* q = qf + (c * 2 + h) * k;
        for (int64_t kk = 0; kk < k; ++kk) {
          const float band = ((p[0 * k + kk] + p[1 * k + kk]) + (p[2 * k + kk] + p[3 * k + kk])) +
                             ((p[4 * k + kk] + p[5 * k + kk]) + (p[6 * k + kk] + p[7 * k + kk]));
          q[kk] = bnd == 0 ? band : q[kk] + band;
        }
      }
    }
  }
  for (int64_t col = 0; col < padded_n; ++col) {
    if (col < n) decode_row(kind == 2 ? 3 : kind, b, sfb, col, k, row_v);
    for (int c = 0; c < channels; ++c) {
      const float* qe = qf + (c * 2 + 0) * k;
      const float* qa = qf + (c * 2 + 1) * k;
      for (int64_t slot = 0; slot < tiles; ++slot) {
        float r = 0.f, s = 0.f;
        if (col < n) {
          for (int64_t sl = slot; sl < slices; sl += tiles) {
            for (int64_t kk = sl * 64; kk < sl * 64 + 64 && kk < k; ++kk) {
              r = fmaf(qe[kk], row_v[kk], r);
              s = fmaf(qa[kk], fabsf(row_v[kk]), s);
            }
          }
        }
        pred[(c * tiles + slot) * padded_n + col] = alpha * r;
        mag[(c * tiles + slot) * padded_n + col] = fabsf(alpha) * s;
      }
    }
  }
  free(qf);
  free(lanes);
  free(row_v);
  return 0;
}

/* TILE layout for a subset of M-tiles: pred/mag [C][ntiles][padded_n], entry
 * (c, i, col) equal to oracle_tile_reference's (c, tiles[i], col). Makes the
 * per-tile parity check affordable at the benchmark sizes. */
int oracle_tile_reference_subset(int kind, const uint8_t* a, const uint8_t* sfa, const uint8_t* b,
                                 const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* w,
                                 int channels, float alpha, const int64_t* tiles, int64_t ntiles, float* pred,
                                 float* mag, int64_t padded_n) {
  float* q = (float*)calloc((size_t)ntiles * channels * 2 * k, sizeof(float)); /* [i][c][h][k] */
  float* bv = (float*)malloc(sizeof(float) * k);
  if (!q || !bv) {
    free(q);
    free(bv);
    return 1;
  }
  for (int64_t i = 0; i < ntiles; ++i) {
    const int64_t t = tiles[i];
    for (int64_t r = 0; r < 128 && t * 128 + r < m; ++r) {
      const int64_t row = t * 128 + r;
      decode_row(kind, a, sfa, row, k, bv);
      for (int c = 0; c < channels; ++c) {
        const float wt = w[c * m + row], wa = fabsf(wt);
        float* qe = q + ((i * channels + c) * 2 + 0) * k;
        float* qa = q + ((i * channels + c) * 2 + 1) * k;
        for (int64_t kk = 0; kk < k; ++kk) {
          qe[kk] = fmaf(wt, bv[kk], qe[kk]);
          qa[kk] = fmaf(wa, fabsf(bv[kk]), qa[kk]);
        }
      }
    }
  }
  for (int64_t col = 0; col < padded_n; ++col) {
    if (col < n) decode_row(kind == 2 ? 3 : kind, b, sfb, col, k, bv);
    for (int64_t i = 0; i < ntiles; ++i) {
      for (int c = 0; c < channels; ++c) {
        const float* qe = q + ((i * channels + c) * 2 + 0) * k;
        const float* qa = q + ((i * channels + c) * 2 + 1) * k;
        float r = 0.f, s = 0.f;
        if (col < n) {
          for (int64_t kk = 0; kk < k; ++kk) {
            r = fmaf(qe[kk], bv[kk], r);
            s = fmaf(qa[kk], fabsf(bv[kk]), s);
          }
        }
        pred[(c * ntiles + i) * padded_n + col] = alpha * r;
        mag[(c * ntiles + i) * padded_n + col] = fabsf(alpha) * s;
      }
    }
  }
  free(q);
  free(bv);
  return 0;
}

/* Observed column checksums in the sm_100a epilogue's reduction order (an
 * sdc_b200 extension; the reference's in-tile order, CUTLASS's
 * Sm90RowReduction, is unpinned). v: the fp32 values the epilogue checksums
 * (alpha * accumulator, after the fault XOR), row-major [m, n]. Per 128-row
 * tile, 32-row quarter q (rows 32q..32q+31, lane L = row % 32) and 32-column
 * chunk (columns 32j..32j+31, column index i within it):
 *   level 16: lane L with bit 4 equal to bit 4 of i holds
 *             fmaf(w[L], v[L][i], fl(w[L^16] * v[L^16][i]));
 *   levels 8, 4, 2, 1: lane L keeps the columns whose bit matches its own and
 *             adds the partner lane's (L ^ width) value: fl(own + partner);
 *   lane i ends with column i's quarter sum S_q;
 * observed[c][t][col] = (((0 + S_0) + S_1) + S_2) + S_3, columns < padded_n
 * (columns >= n contribute zeros; rows >= m have weight 0). */
int oracle_observed_epilogue(const float* v, int64_t m, int64_t n, const float* w, int channels,
                             float* observed, int64_t padded_n) {
  const int64_t tiles = (m + 127) / 128;
  for (int c = 0; c < channels; ++c) {
    for (int64_t t = 0; t < tiles; ++t) {
      for (int64_t col = 0; col < padded_n; ++col) {
        const int i = (int)(col & 31);
        float sum = 0.f;
        for (int q = 0; q < 4; ++q) {
          float lane_val[32];
          float wl[32], vl[32];
          for (int L = 0; L < 32; ++L) {
            const int64_t row = t * 128 + q * 32 + L;
            const int in = row < m && col < n;
            wl[L] = row < m ? w[c * m + row] : 0.f;
            vl[L] = in ? v[row * n + col] : 0.f;
          }
          for (int L = 0; L < 32; ++L) {
            const float partner = wl[L ^ 16] * vl[L ^ 16];
            lane_val[L] = fmaf(wl[L], vl[L], partner);
          }
          for (int width = 8; width >= 1; width >>= 1) {
            float next[32];
            for (int L = 0; L < 32; ++L) next[L] = lane_val[L] + lane_val[L ^ width];
            memcpy(lane_val, next, sizeof(next));
          }
          sum = sum + lane_val[i];
        }
        observed[(c * tiles + t) * padded_n + col] = sum;
      }
    }
  }
  return 0;
}

/* Exact dot products in double for the GEMM output reference: every product
 * of two decoded operands is exact in double and K <= 2^20 terms of at most
 * 2^-20..2^18 magnitude keep the double sum within 1 ulp of fp32 output. */
int oracle_gemm_f64(int kind, const uint8_t* a, const uint8_t* sfa, const uint8_t* b,
                    const uint8_t* sfb, int64_t m, int64_t n, int64_t k, double* out) {
  float* bv = (float*)malloc(sizeof(float) * k);
  float* av = (float*)malloc(sizeof(float) * k * m);
  if (!bv || !av) return 1;
  for (int64_t row = 0; row < m; ++row)
    for (int64_t kk = 0; kk < k; ++kk) av[row * k + kk] = value_at(kind, a, sfa, row, kk, k);
  for (int64_t col = 0; col < n; ++col) {
    for (int64_t kk = 0; kk < k; ++kk) bv[kk] = value_at(kind == 2 ? 3 : kind, b, sfb, col, kk, k);
    for (int64_t row = 0; row < m; ++row) {
      double s = 0.0;
      const float* ar = av + row * k;
      for (int64_t kk = 0; kk < k; ++kk) s += (double)ar[kk] * (double)bv[kk];
      out[row * n + col] = s;
    }
  }
  free(bv);
  free(av);
  return 0;
}

/* Augmented BF16 encoding, the fixed order of the sdc_b200 augmented GEMM's
 * encode kernel (the reference forms the same rows with tensor-core MMAs,
 * src/cutlass_gemm/csrc/abft/fp32_bf16/bf16_augmented.h:216-320, whose
 * internal summation order is unspecified): for each 128-row M-tile t,
 * channel c and column kk,
 *   s_j = fmaf(w_c[row], A[row][kk], s_j) over rows [16 j, 16 j + 16) of
 *         the tile that are < m, ascending, from s_j = +0 (j = 0..7);
 *   q[t * C + c][kk] = bf16(((s_0 + s_1) + s_2) + ... + s_7), nearest even.
 * a: bf16 bits [m, k]; w: bf16 bits [C, m]; q: bf16 bits [C * tiles, k]. */
static float bf16_value(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t bf16_round(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFF; /* canonical NaN */
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

int oracle_augment_encode(const uint16_t* a, int64_t m, int64_t k, const uint16_t* w, int channels,
                          uint16_t* q) {
  const int64_t tiles = (m + 127) / 128;
  float* seg = (float*)malloc(sizeof(float) * k * 8);
  if (!seg) return 1;
  for (int64_t t = 0; t < tiles; ++t) {
    for (int c = 0; c < channels; ++c) {
      for (int64_t i = 0; i < k * 8; ++i) seg[i] = 0.f;
      for (int j = 0; j < 8; ++j) {
        for (int64_t row = t * 128 + 16 * j; row < t * 128 + 16 * j + 16 && row < m; ++row) {
          const float wv = bf16_value(w[c * m + row]);
          const uint16_t* ar = a + row * k;
          for (int64_t kk = 0; kk < k; ++kk) seg[j * k + kk] = fmaf(wv, bf16_value(ar[kk]), seg[j * k + kk]);
        }
      }
      uint16_t* out = q + (t * channels + c) * k;
      for (int64_t kk = 0; kk < k; ++kk) {
        float sum = seg[kk];
        for (int j = 1; j < 8; ++j) sum = sum + seg[j * k + kk];
        out[kk] = bf16_round(sum);
      }
    }
  }
  free(seg);
  return 0;
}

/* Row checksums (the sdc_b200 extension; the reference checks columns only).
 *
 * oracle_row_observed: out[b][row] = sum of v[row][col] over the 64 columns
 * col of block b that are < n, ascending, from +0 (the GEMM epilogue's order).
 * v: fp32 [m][n] row-major; out: [ceil(n/64)][m]. */
int oracle_row_observed(const float* v, int64_t m, int64_t n, float* out) {
  const int64_t blocks = (n + 63) / 64;
  for (int64_t b = 0; b < blocks; ++b) {
    for (int64_t row = 0; row < m; ++row) {
      float s = 0.f;
      for (int64_t col = b * 64; col < b * 64 + 64 && col < n; ++col) s = s + v[row * n + col];
      out[b * m + row] = s;
    }
  }
  return 0;
}

/* oracle_row_reference: u[k] = e^T B, u_abs[k] = e^T |B| over the n rows of
 * B in the K-slice projection's order (bands of 128 rows; in a band, 8 row
 * lanes l each run an fma chain over rows begin + l, + 8, ...; combined as
 * ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)); bands ascending) with
 * unit weights; then for each row m of A, 32 lane chains: lane j runs
 * acc_j = fmaf(A[m][k], u[k], acc_j) (and the |A| u_abs chain) over the
 * 16-element groups g = j, j + 32, ... (k ascending), combined by a butterfly
 * (p[j] = p[j] + p[j ^ w] for w = 16, 8, 4, 2, 1; the result is p[0]);
 * pred[m] = alpha * acc, mag[m] = |alpha| * acc_abs. kind: 0 FP8, 1 NVFP4,
 * 2 block-scaled FP8 (B's scales per 128 x 128 block). */
int oracle_row_reference(int kind, const uint8_t* a, const uint8_t* sfa, const uint8_t* b, const uint8_t* sfb,
                         int64_t m, int64_t n, int64_t k, float alpha, float* pred, float* mag) {
  float* u = (float*)calloc((size_t)k, sizeof(float));
  float* ua = (float*)calloc((size_t)k, sizeof(float));
  float* lanes = (float*)malloc(sizeof(float) * 2 * 8 * k);
  float* row_v = (float*)malloc(sizeof(float) * k);
  if (!u || !ua || !lanes || !row_v) {
    free(u);
    free(ua);
    free(lanes);
    free(row_v);
    return 1;
  }
  const int bkind = kind == 2 ? 3 : kind;
  const int64_t bands = (n + 127) / 128;
  for (int64_t bnd = 0; bnd < bands; ++bnd) {
    const int64_t begin = bnd * 128, end = begin + 128 < n ? begin + 128 : n;
    memset(lanes, 0, sizeof(float) * 2 * 8 * k);
    for (int64_t row = begin; row < end; ++row) {
      const int l = (int)((row - begin) & 7);
      decode_row(bkind, b, sfb, row, k, row_v);
      float* e = lanes + (0 * 8 + l) * k;
      float* g = lanes + (1 * 8 + l) * k;
      for (int64_t kk = 0; kk < k; ++kk) {
        e[kk] = fmaf(1.f, row_v[kk], e[kk]);
        g[kk] = fmaf(1.f, fabsf(row_v[kk]), g[kk]);
      }
    }
    for (int h = 0; h < 2; ++h) {
      const float* p = lanes + h * 8 * k;
      float* q = h == 0 ? u : ua;
      for (int64_t kk = 0; kk < k; ++kk) {
        const float band = ((p[0 * k + kk] + p[1 * k + kk]) + (p[2 * k + kk] + p[3 * k + kk])) +
                           ((p[4 * k + kk] + p[5 * k + kk]) + (p[6 * k + kk] + p[7 * k + kk]));
        q[kk] = bnd == 0 ? band : q[kk] + band;
      }
    }
  }
  const int64_t groups = k / 16;
  for (int64_t row = 0; row < m; ++row) {
    decode_row(kind, a, sfa, row, k, row_v);
    float p[32], pa[32];
    for (int j = 0; j < 32; ++j) {
      float acc = 0.f, acc_a = 0.f;
      for (int64_t g = j; g < groups; g += 32) {
        for (int64_t kk = g * 16; kk < g * 16 + 16; ++kk) {
          acc = fmaf(row_v[kk], u[kk], acc);
          acc_a = fmaf(fabsf(row_v[kk]), ua[kk], acc_a);
        }
      }
      p[j] = acc;
      pa[j] = acc_a;
    }
    for (int w = 16; w >= 1; w >>= 1) {
      float np[32], npa[32];
      for (int j = 0; j < 32; ++j) {
        np[j] = p[j] + p[j ^ w];
        npa[j] = pa[j] + pa[j ^ w];
      }
      memcpy(p, np, sizeof(p));
      memcpy(pa, npa, sizeof(pa));
    }
    pred[row] = alpha * p[0];
    mag[row] = fabsf(alpha) * pa[0];
  }
  free(u);
  free(ua);
  free(lanes);
  free(row_v);
  return 0;
}
