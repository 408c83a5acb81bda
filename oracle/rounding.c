/*
 * rounding.c — C restatement of the reference shaders' fp32 -> bf16 / fp16 rounding and of the
 * int8 dequant loop. TEST INFRASTRUCTURE ONLY (the oracle); built by oracle/Makefile into
 * oracle/liboracle.so and loaded by tests/test_oracle.py.
 *
 *   f2bf: vkrt/shaders/types.glsl:45-50   round-to-nearest-even on the upper 16 bits, NaN -> 0x7FC0
 *   f2h:  vkrt/shaders/types.glsl:18-41   round-to-nearest-even incl. subnormals, overflow -> inf
 *   dq8:  vkrt/shaders/dq8.comp.in:27-62  out = round(float(q) * float(scale[r, c/64]))
 */
#include <stdint.h>
#include <string.h>

static uint32_t bits_of(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static float float_of(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t oracle_f2bf(float x) {
  uint32_t u = bits_of(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float oracle_bf2f(uint16_t h) { return float_of((uint32_t)h << 16); }

uint16_t oracle_f2h(float f) {
  uint32_t u = bits_of(f);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t e = (u >> 23) & 0xFFu;
  uint32_t m = u & 0x7FFFFFu;
  if (e == 0xFFu) return (uint16_t)(sign | 0x7C00u | (m ? (0x200u | (m >> 13)) : 0u));
  int ne = (int)e - 127 + 15;
  if (ne >= 31) return (uint16_t)(sign | 0x7C00u);
  if (ne <= 0) {
    if (ne < -10) return (uint16_t)sign;
    m |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - ne);
    uint32_t hm = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (hm & 1u))) hm++;
    return (uint16_t)(sign | hm);
  }
  uint32_t hm = m >> 13;
  uint32_t rem = m & 0x1FFFu;
  uint32_t h = sign | ((uint32_t)ne << 10) | hm;
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h++;
  return (uint16_t)h;
}

void oracle_f2bf_array(const float* x, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f2bf(x[i]);
}
void oracle_f2h_array(const float* x, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f2h(x[i]);
}

/* kind: 0 = f32 out, 1 = bf16 out, 2 = f16 out; scale bf16 [rows, ceil(cols/64)] */
void oracle_dequant_int8(const int8_t* q, const uint16_t* scale, void* out, int64_t rows, int64_t cols, int kind) {
  int64_t nb = (cols + 63) / 64;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      float v = (float)q[r * cols + c] * oracle_bf2f(scale[r * nb + c / 64]);
      int64_t i = r * cols + c;
      if (kind == 0) ((float*)out)[i] = v;
      else if (kind == 1) ((uint16_t*)out)[i] = oracle_f2bf(v);
      else ((uint16_t*)out)[i] = oracle_f2h(v);
    }
}
