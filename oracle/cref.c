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
  float* qf = (float*)malloc(sizeof(float) * channels * 2 * k);
  if (!qf) return 1;
  /* q over all rows in the GEMM prediction warps' order: bands of 512 rows;
   * in a band, 8 row lanes l each run an fma chain over rows
   * band_start + l, + 8, ... (ascending), combined as
   * ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)); q = ((band_0 + band_1)
   * + ...) + band_last. */
  const int64_t bands = (m + 511) / 512;
  for (int c = 0; c < channels; ++c) {
    for (int64_t kk = 0; kk < k; ++kk) {
      float q[2] = {0.f, 0.f};
      for (int64_t b = 0; b < bands; ++b) {
        const int64_t begin = b * 512, end = begin + 512 < m ? begin + 512 : m;
        float lanes[2][8];
        for (int l = 0; l < 8; ++l) {
          float e = 0.f, g = 0.f;
          for (int64_t row = begin + l; row < end; row += 8) {
            const float v = value_at(kind, a, sfa, row, kk, k);
            const float wv = w[c * m + row];
            e = fmaf(wv, v, e);
            g = fmaf(fabsf(wv), fabsf(v), g);
          }
          lanes[0][l] = e;
          lanes[1][l] = g;
        }
        for (int h = 0; h < 2; ++h) {
          const float* p = lanes[h];
          const float band = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
          q[h] = b == 0 ? band : q[h] + band;
        }
      }
      qf[(c * 2 + 0) * k + kk] = q[0];
      qf[(c * 2 + 1) * k + kk] = q[1];
    }
  }
  for (int c = 0; c < channels; ++c) {
    for (int64_t slot = 0; slot < tiles; ++slot) {
      for (int64_t col = 0; col < padded_n; ++col) {
        float r = 0.f, s = 0.f;
        if (col < n) {
          for (int64_t sl = slot; sl < slices; sl += tiles) {
            for (int64_t kk = sl * 64; kk < sl * 64 + 64 && kk < k; ++kk) {
              const float v = value_at(kind == 2 ? 3 : kind, b, sfb, col, kk, k);
              r = fmaf(qf[(c * 2 + 0) * k + kk], v, r);
              s = fmaf(qf[(c * 2 + 1) * k + kk], fabsf(v), s);
            }
          }
        }
        pred[(c * tiles + slot) * padded_n + col] = alpha * r;
        mag[(c * tiles + slot) * padded_n + col] = fabsf(alpha) * s;
      }
    }
  }
  free(qf);
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
