// Host helpers of the reference's loader that feed the decoder: the MRoPE tables
// (src/mrope.rs:5-80, rounded to f16 as src/inference.rs:1037-1047 does) and the INT8
// dequantisation rule (src/weights.rs:372-385).
#include <cmath>
#include <cstdint>
#include <vector>

#include "f16_host.h"
#include "qasr_b200.h"

extern "C" {

qasr_status qasr_build_dim_map(const int* section, int nsection, int half, int interleaved,
                               int* out) {
  if (!section || nsection <= 0 || half <= 0 || !out) return QASR_ERR_INVALID_ARG;
  for (int d = 0; d < nsection; ++d)
    if (section[d] < 0) return QASR_ERR_INVALID_ARG;
  int len = 0;
  if (interleaved) {
    // Qwen2-VL order: 0,1,2,0,1,2,... while each axis has quota left
    std::vector<int> used(nsection, 0);
    bool progress = true;
    while (len < half && progress) {
      progress = false;
      for (int d = 0; d < nsection && len < half; ++d) {
        if (used[d] < section[d]) {
          out[len++] = d;
          ++used[d];
          progress = true;
        }
      }
    }
  } else {
    for (int d = 0; d < nsection && len < half; ++d)
      for (int i = 0; i < section[d] && len < half; ++i) out[len++] = d;
    while (len < half) out[len++] = nsection - 1;
  }
  for (int i = len; i < half; ++i) out[i] = -1;  // quotas ran out before `half`
  return QASR_OK;
}

qasr_status qasr_build_rope_tables(uint16_t* cos_out, uint16_t* sin_out, int positions,
                                   int head_dim, double rope_theta, const int* section,
                                   int nsection, int interleaved) {
  if (!cos_out || !sin_out || positions <= 0 || head_dim <= 0 || head_dim % 2 || rope_theta <= 0)
    return QASR_ERR_INVALID_ARG;
  const int half = head_dim / 2;
  std::vector<int> dm(half);
  qasr_status s = qasr_build_dim_map(section, nsection, half, interleaved, dm.data());
  if (s != QASR_OK) return s;
  std::vector<double> inv(half);
  for (int i = 0; i < half; ++i)
    inv[i] = 1.0 / std::pow(rope_theta, 2.0 * i / static_cast<double>(head_dim));
  // Text positions: every axis carries 0..positions, so the axis map (dm) selects the
  // same position for every frequency; it still decides nothing numerically here, but
  // the map is validated the way the reference builds it.
#pragma omp parallel for schedule(static)
  for (int t = 0; t < positions; ++t) {
    for (int j = 0; j < half; ++j) {
      const double angle = static_cast<double>(t) * inv[j];
      const uint16_t c = qasr::f32_to_f16_bits(static_cast<float>(std::cos(angle)));
      const uint16_t sn = qasr::f32_to_f16_bits(static_cast<float>(std::sin(angle)));
      const size_t b = static_cast<size_t>(t) * head_dim;
      cos_out[b + j] = c;
      cos_out[b + j + half] = c;
      sin_out[b + j] = sn;
      sin_out[b + j + half] = sn;
    }
  }
  return QASR_OK;
}

qasr_status qasr_dequant_i8(const int8_t* q, const float* scale_f32, int rows, int cols,
                            uint16_t* out) {
  if (!q || !scale_f32 || !out || rows < 0 || cols < 0) return QASR_ERR_INVALID_ARG;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float s = scale_f32[r];
    for (int c = 0; c < cols; ++c) {
      const size_t i = static_cast<size_t>(r) * cols + c;
      out[i] = qasr::f32_to_f16_bits(static_cast<float>(q[i]) * s);
    }
  }
  return QASR_OK;
}

}  // extern "C"
