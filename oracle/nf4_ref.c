/*
 * NF4 dequantiser on the CPU, in C. TEST INFRASTRUCTURE ONLY (the timed CPU baseline of the NF4
 * row and a second check of the numpy oracle in oracle/nf4.py).
 *
 * Arithmetic of the reference kernel, solution/nf4.py:27-45: nested absmax
 * fp32(code2[u8] * absmax2[b / qblock2]) + offset, then fp16(nf4[nibble] * absmax), high nibble
 * first; every operation rounded on its own (built with -ffp-contract=off), the fp16 conversion
 * is round-to-nearest-even (_Float16). OpenMP over rows of bytes.
 */
#include <stdint.h>

typedef _Float16 half_t;

static inline uint16_t to_half_bits(float f) {
  half_t h = (half_t)f;
  uint16_t bits;
  __builtin_memcpy(&bits, &h, sizeof(bits));
  return bits;
}

int oracle_nf4_unpack_nested(const uint8_t *packed, const uint8_t *absmax_u8, const float *code2,
                             const float *absmax2, float offset, const float *table,
                             uint16_t *out, int64_t n_bytes, int32_t qblock, int32_t qblock2) {
  if (qblock <= 0 || qblock % 2 || qblock2 <= 0) return -1;
  const int64_t half = qblock / 2;
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n_bytes; ++j) {
    const int64_t b = j / half;
    const float prod = code2[absmax_u8[b]] * absmax2[b / qblock2];
    const float scale = prod + offset;
    const uint8_t byte = packed[j];
    out[2 * j] = to_half_bits(table[byte >> 4] * scale);
    out[2 * j + 1] = to_half_bits(table[byte & 15] * scale);
  }
  return 0;
}

int oracle_nf4_unpack_plain(const uint8_t *packed, const float *absmax, const float *table,
                            uint16_t *out, int64_t n_bytes, int32_t qblock) {
  if (qblock <= 0 || qblock % 2) return -1;
  const int64_t half = qblock / 2;
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n_bytes; ++j) {
    const float scale = absmax[j / half];
    const uint8_t byte = packed[j];
    out[2 * j] = to_half_bits(table[byte >> 4] * scale);
    out[2 * j + 1] = to_half_bits(table[byte & 15] * scale);
  }
  return 0;
}
