// Host-side IEEE binary16 conversions (round to nearest even), shared by the synthetic
// generator and the runtime's loader helpers.
#pragma once
#include <cstdint>
#include <cstring>

namespace qasr {

inline uint16_t f32_to_f16_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) {  // inf / nan: keep a quiet nan payload bit
    return static_cast<uint16_t>(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  }
  if (ax < 0x38800000u) {  // below the smallest f16 normal (2^-14): subnormal or zero
    if (ax < 0x33000000u) return static_cast<uint16_t>(sign);  // < 2^-25: rounds to 0
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;  // value = m * 2^(e-150); units of 2^-24
    uint32_t k = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1u);
    if (rem > halfway || (rem == halfway && (k & 1u))) ++k;
    return static_cast<uint16_t>(sign | k);
  }
  const uint32_t r = ax - 0x38000000u;  // rebias exponent 127 -> 15
  uint32_t h = r >> 13;
  const uint32_t rem = r & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  if (h >= 0x7c00u) h = 0x7c00u;  // overflow rounds to infinity
  return static_cast<uint16_t>(sign | h);
}

inline float f16_bits_to_f32(uint16_t h) {
  const uint32_t sign = (static_cast<uint32_t>(h) & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  const uint32_t m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {  // subnormal: m * 2^-24
      float v = static_cast<float>(m) * 5.9604644775390625e-08f;
      std::memcpy(&x, &v, 4);
      x |= sign;
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

}  // namespace qasr
