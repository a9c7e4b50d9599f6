/*
 * CPU restatement of the reference's NVFP4 quantise / swizzle / dequantise path.
 *
 * TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the cpu_baseline leg of
 * bench.py as the checker. Nothing in the gemm3_b200 package links or calls it.
 *
 * Follows nvfp4_gemm_cute/quant.py (the reference package, version 0.1.0):
 *   oracle_e2m1_code    quant.py:15-28  (_round_e2m1: clamp to 6, |mag - table| + 1e-6 on odd
 *                                        codes, first argmin, sign bit from q < 0)
 *   oracle_swizzle      quant.py:31-38  (swizzle_sf: pad to 128 rows x 4 columns, [32][4][4])
 *   oracle_quantize     quant.py:41-59  (quantize_nvfp4)
 *   oracle_dequantize   quant.py:62-70  (dequantize_nvfp4)
 * The E4M3 conversion is PyTorch's float -> float8_e4m3fn cast (round to nearest even, overflow
 * to NaN), restated here from the format definition. The formulation deliberately differs from
 * the CUDA kernels (full 8-entry argmin, frexp-based rounding) so the two cross-check each other.
 *
 * div_mode: 0 = "/ scalar" rounds like PyTorch on CUDA (x * fl(1/s)); 1 = like PyTorch on CPU
 * (correctly rounded x / s). Build with -ffp-contract=off so every float operation rounds once.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

uint8_t oracle_e4m3_encode(float f) {
  const uint8_t sign = signbit(f) ? 0x80 : 0x00;
  if (isnan(f)) return sign | 0x7F;
  const float a = fabsf(f);
  if (a > 464.0f) return sign | 0x7F; /* rounds past 448 (or is infinite): NaN */
  if (a == 0.0f) return sign;
  int ex;
  (void)frexpf(a, &ex); /* a = m * 2^ex, m in [0.5, 1) */
  int e = ex - 1;       /* a in [2^e, 2^(e+1)) */
  if (e < -6) e = -6;   /* subnormal: fixed quantum 2^-9 */
  double scaled = ldexp((double)a, 3 - e); /* exact; quantum becomes 1 */
  double r = nearbyint(scaled);            /* round half to even (default rounding mode) */
  if (r >= 16.0) {
    e += 1;
    r = 8.0;
  }
  int bits;
  if (r < 8.0) {
    bits = (int)r; /* subnormal (only reachable with e == -6) */
  } else {
    bits = ((e + 7) << 3) | ((int)r - 8);
  }
  if (bits >= 0x7F) return sign | 0x7F;
  return sign | (uint8_t)bits;
}

float oracle_e4m3_decode(uint8_t b) {
  const int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
  float v;
  if (e == 15 && m == 7) return s ? -NAN : NAN;
  if (e == 0)
    v = ldexpf((float)m, -9);
  else
    v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

uint8_t oracle_e2m1_code(float q) {
  float mag = fabsf(q);
  if (mag > 6.0f) mag = 6.0f;
  const float pen = (float)1e-6;
  int best = 0;
  float best_d = fabsf(mag - kE2M1[0]) + 0.0f;
  for (int i = 1; i < 8; ++i) {
    const float d = fabsf(mag - kE2M1[i]) + ((i & 1) ? pen : 0.0f);
    if (d < best_d) {
      best_d = d;
      best = i;
    }
  }
  return (uint8_t)(best | (q < 0.0f ? 8 : 0));
}

/* x: [rows, k] float32 (inputs of lower precision are passed widened, as x.float() does).
 * packed: [rows, k/2]; sf_lin: [rows, k/16]. */
void oracle_quantize(const float* x, int64_t rows, int64_t k, float gs, int div_mode, uint8_t* packed,
                     uint8_t* sf_lin) {
  const int64_t cols = k / 16;
  const float inv6 = 1.0f / 6.0f;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c) {
      const float* src = x + r * k + c * 16;
      float xb[16];
      float amax = 0.0f;
      int has_nan = 0;
      for (int i = 0; i < 16; ++i) {
        xb[i] = src[i] * gs;
        const float a = fabsf(xb[i]);
        if (isnan(a))
          has_nan = 1;
        else if (a > amax)
          amax = a;
      }
      const float s = div_mode == 0 ? amax * inv6 : amax / 6.0f;
      const uint8_t sf = has_nan ? 0x7F : oracle_e4m3_encode(s);
      const float denom = oracle_e4m3_decode(sf);
      uint8_t codes[16];
      for (int i = 0; i < 16; ++i) {
        const float q = (denom > 0.0f) ? xb[i] / denom : 0.0f;
        codes[i] = oracle_e2m1_code(q);
      }
      for (int j = 0; j < 8; ++j) packed[r * (k / 2) + c * 8 + j] = (uint8_t)(codes[2 * j] | (codes[2 * j + 1] << 4));
      sf_lin[r * cols + c] = sf;
    }
  }
}

/* sf_lin: [rows, cols] -> out: ceil(rows/128)*128 * ceil(cols/4)*4 bytes. */
void oracle_swizzle(const uint8_t* sf_lin, int64_t rows, int64_t cols, uint8_t* out) {
  const int64_t rp = (rows + 127) / 128 * 128, cp = (cols + 3) / 4 * 4;
  memset(out, 0, (size_t)(rp * cp));
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c) {
      /* pad.view(rp/128, 4, 32, cp/4, 4).permute(0, 3, 2, 1, 4): dims (rb, c4, r32, r4, c%4) */
      const int64_t rb = r / 128, r4 = (r % 128) / 32, r32 = r % 32, c4 = c / 4, cc = c % 4;
      const int64_t off = (((rb * (cp / 4) + c4) * 32 + r32) * 4 + r4) * 4 + cc;
      out[off] = sf_lin[r * cols + c];
    }
  }
}

/* out: [rows, k] float32 = table[code & 7] * (+-1) * e4m3(sf) / gs. */
void oracle_dequantize(const uint8_t* packed, const uint8_t* sf_lin, int64_t rows, int64_t k, float gs,
                       int div_mode, float* out) {
  const int64_t cols = k / 16;
  const float inv_gs = 1.0f / gs;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t e = 0; e < k; ++e) {
      const uint8_t byte = packed[r * (k / 2) + e / 2];
      const uint8_t code = (e & 1) ? (byte >> 4) : (byte & 15);
      const float val = kE2M1[code & 7] * ((code & 8) ? -1.0f : 1.0f);
      const float scale = oracle_e4m3_decode(sf_lin[r * cols + e / 16]);
      const float vs = val * scale;
      out[r * k + e] = div_mode == 0 ? vs * inv_gs : vs / gs;
    }
  }
}

/* Vector helpers for tests. */
void oracle_e4m3_encode_n(const float* x, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_e4m3_encode(x[i]);
}
void oracle_e2m1_code_n(const float* x, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_e2m1_code(x[i]);
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  extern int omp_get_max_threads(void);
  return omp_get_max_threads();
#else
  return 1;
#endif
}
