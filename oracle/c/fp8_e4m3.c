/* e4m3 ("fn": no infinities, max finite 448, NaN = S.1111.111) quantisation, restated from
 * the format definition (OCP FP8 spec): sign, 4 exponent bits with bias 7, 3 mantissa bits;
 * subnormals are m * 2^-9.  Rounding is round-to-nearest-even on the exact binary value; values
 * whose magnitude rounds above 448 saturate to 448 (the clamp(x/scale, -448, 448) of the FP8
 * store restatement).  TEST ORACLE ONLY. */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_to_float(uint16_t v) {
  uint32_t u = ((uint32_t)v) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint8_t oracle_float_to_e4m3(float x) {
  if (isnan(x)) return 0x7F;
  uint8_t sign = signbit(x) ? 0x80 : 0x00;
  double a = fabs((double)x);
  if (a >= 448.0) return sign | 0x7E;
  if (a < ldexp(1.0, -6)) {
    /* subnormal range: integer multiple of 2^-9, round half to even */
    double q = nearbyint(a * 512.0);
    if (q >= 8.0) return sign | 0x08; /* rounds up to the smallest normal */
    return sign | (uint8_t)q;
  }
  int e;
  double fr = frexp(a, &e); /* a = fr * 2^e, fr in [0.5, 1) */
  int exp2 = e - 1;          /* a = (2*fr) * 2^exp2, 2*fr in [1, 2) */
  double q = nearbyint(ldexp(a, 3 - exp2)); /* in [8, 16] */
  if (q >= 16.0) {
    q = 8.0;
    exp2 += 1;
  }
  int field = exp2 + 7;
  int mant = (int)q - 8;
  if (field > 15 || (field == 15 && mant == 7)) return sign | 0x7E;
  return sign | (uint8_t)((field << 3) | mant);
}

float oracle_e4m3_to_float(uint8_t v) {
  int s = v >> 7, field = (v >> 3) & 0xF, mant = v & 7;
  if (field == 15 && mant == 7) return NAN;
  double mag = field == 0 ? ldexp((double)mant, -9) : ldexp(1.0 + mant / 8.0, field - 7);
  return (float)(s ? -mag : mag);
}

/* out[i] = e4m3(bf16[i] / scale[(i / head_dim) % num_heads]) for a [n_rows, num_heads*head_dim]
 * bf16 matrix: the per-KV-head FP8 store of one or more token rows. */
void oracle_quantize_rows(const uint16_t* bf16, int64_t n_rows, int num_heads, int head_dim,
                          const float* scale, uint8_t* out) {
  const int64_t row = (int64_t)num_heads * head_dim;
  for (int64_t r = 0; r < n_rows; ++r)
    for (int64_t i = 0; i < row; ++i) {
      float s = scale ? scale[i / head_dim] : 1.0f;
      volatile float y = bf16_to_float(bf16[r * row + i]) / s; /* IEEE single division */
      out[r * row + i] = oracle_float_to_e4m3(y);
    }
}
