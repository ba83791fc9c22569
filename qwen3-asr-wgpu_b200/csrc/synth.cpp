// Seeded synthetic tensors for the Qwen3-ASR decoder (see include/qasr_synth.h).
#include "qasr_synth.h"

#include <cmath>
#include <cstdlib>

#include "f16_host.h"

namespace {

inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

}  // namespace

extern "C" {

uint64_t qasr_synth_key(uint64_t seed, uint64_t tensor_id) {
  return mix64(seed ^ mix64(tensor_id * 0x2545f4914f6cdd1dull + 0x1234567ull));
}

void qasr_synth_normal_f16(uint16_t* out, size_t n, uint64_t seed, uint64_t tensor_id, float mean,
                           float std_) {
  const uint64_t key = qasr_synth_key(seed, tensor_id);
  const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < static_cast<long long>(n); ++i) {
    const uint64_t r = mix64(key + static_cast<uint64_t>(i));
    // two 24-bit uniforms: u1 in (0, 1], u2 in [0, 1)
    const double u1 = (static_cast<double>(r >> 40) + 1.0) * (1.0 / 16777216.0);
    const double u2 = static_cast<double>((r >> 8) & 0xffffffull) * (1.0 / 16777216.0);
    const double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2);
    out[i] = qasr::f32_to_f16_bits(static_cast<float>(z * static_cast<double>(std_) +
                                                       static_cast<double>(mean)));
  }
}

void qasr_synth_uniform_ids(int32_t* out, size_t n, uint64_t seed, uint64_t tensor_id, int32_t lo,
                            int32_t hi) {
  const uint64_t key = qasr_synth_key(seed, tensor_id);
  const uint64_t span = static_cast<uint64_t>(static_cast<int64_t>(hi) - lo);
  for (size_t i = 0; i < n; ++i) {
    const uint64_t r = mix64(key + i);
    out[i] = lo + static_cast<int32_t>(span ? (r >> 11) % span : 0);
  }
}

void qasr_synth_quantize_rows(const uint16_t* w, int rows, int cols, int8_t* q, uint16_t* scale) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint16_t* row = w + static_cast<size_t>(r) * cols;
    float amax = 0.0f;
    for (int c = 0; c < cols; ++c) {
      const float v = std::fabs(qasr::f16_bits_to_f32(row[c]));
      if (v > amax) amax = v;
    }
    uint16_t sh = qasr::f32_to_f16_bits(amax / 127.0f);
    float s = qasr::f16_bits_to_f32(sh);
    if (!(s > 0.0f)) {  // all-zero row: any positive scale dequantises to zeros
      sh = qasr::f32_to_f16_bits(1.0f);
      s = 1.0f;
    }
    scale[r] = sh;
    int8_t* qr = q + static_cast<size_t>(r) * cols;
    for (int c = 0; c < cols; ++c) {
      float v = std::nearbyint(qasr::f16_bits_to_f32(row[c]) / s);
      if (v > 127.0f) v = 127.0f;
      if (v < -127.0f) v = -127.0f;
      qr[c] = static_cast<int8_t>(v);
    }
  }
}

uint16_t qasr_f32_to_f16(float f) { return qasr::f32_to_f16_bits(f); }
float qasr_f16_to_f32(uint16_t h) { return qasr::f16_bits_to_f32(h); }

void qasr_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < static_cast<long long>(n); ++i) out[i] = qasr::f32_to_f16_bits(in[i]);
}

void qasr_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < static_cast<long long>(n); ++i) out[i] = qasr::f16_bits_to_f32(in[i]);
}

}  // extern "C"
