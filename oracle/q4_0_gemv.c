/* Oracle (test infrastructure only): the Metal shader flash_dequant_gemv_q4
 * (mlx_flash_compress/kernels/flash_dequant.metal:19-49) restated in C.
 *
 * One output row at a time, codes in storage order: for every group g and
 * byte i of the group, low nibble (even column) then high nibble (odd
 * column), value (code - 8) * scale, accumulated in fp32 as
 *     acc += (v * scale) * x[col]
 * with every product and sum rounded separately (built with
 * -ffp-contract=off).  fp16 scales are widened exactly in software. */
#include <stdint.h>
#include <string.h>

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      exp = 127 - 15 + 1;
      while (!(man & 0x400)) {
        man <<= 1;
        exp--;
      }
      man &= 0x3ff;
      bits = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

/* weights uint8 [M, N/2], scales fp16 bits [M, N/gs], x fp32 [N], y fp32 [M] */
void q4_0_gemv(const uint8_t* weights, const uint16_t* scales, const float* x, float* y, uint32_t M, uint32_t N,
               uint32_t group_size) {
  const uint32_t n_groups = N / group_size;
  const uint32_t bytes_per_group = group_size / 2;
  for (uint32_t row = 0; row < M; ++row) {
    float acc = 0.0f;
    for (uint32_t g = 0; g < n_groups; ++g) {
      const float scale = half_to_float(scales[row * n_groups + g]);
      const uint64_t base_byte = (uint64_t)row * (N / 2) + (uint64_t)g * bytes_per_group;
      const uint32_t base_x = g * group_size;
      for (uint32_t i = 0; i < bytes_per_group; ++i) {
        const uint8_t packed = weights[base_byte + i];
        const float v0 = (float)(packed & 0x0F) - 8.0f;
        const float v1 = (float)(packed >> 4) - 8.0f;
        const float p0 = v0 * scale;
        const float t0 = p0 * x[base_x + 2 * i];
        acc = acc + t0;
        const float p1 = v1 * scale;
        const float t1 = p1 * x[base_x + 2 * i + 1];
        acc = acc + t1;
      }
    }
    y[row] = acc;
  }
}
