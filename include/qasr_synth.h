/*
 * qasr_synth.h — seeded synthetic weights and prefixes for the Qwen3-ASR decoder.
 *
 * The reference is measured on real checkpoints and audio (src/inference.rs:939-1047,
 * scripts/bench.ps1); neither exists on the build or GPU machines, so every benchmark
 * and parity run uses synthetic tensors of the checkpoint's shapes.  This generator
 * is the one source of those bytes: the CPU oracle and the B200 library consume the
 * identical host buffers it fills.
 *
 * RNG: counter-based.  key = mix(seed, tensor_id); element i draws r = mix(key + i)
 * with mix = splitmix64 finaliser; two 24-bit uniforms from r feed Box–Muller
 * (z = sqrt(-2 ln u1) * cos(2 pi u2), f64), the value f32(z * std + mean) is rounded
 * to f16 by IEEE round-to-nearest-even.  Results do not depend on thread count.
 *
 * INT8: per-row symmetric quantisation of an f16 matrix:
 *   s = f16(max_c |w[r, c]| / 127), q = clamp(rint(w / s), -127, 127)  (s widened to f32)
 * which is the layout `PackedInt8` carries (src/weights.rs:309-356) with the scale
 * stored as f16 instead of the reference's F32 (the f16 value widens exactly).
 */
#ifndef QASR_SYNTH_H
#define QASR_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Tensor ids of the synthetic model (layer tensors: layer * 32 + kind). */
enum {
  QASR_T_Q = 0, QASR_T_K = 1, QASR_T_V = 2, QASR_T_O = 3,
  QASR_T_GATE = 4, QASR_T_UP = 5, QASR_T_DOWN = 6,
  QASR_T_ILN = 7, QASR_T_PLN = 8, QASR_T_QN = 9, QASR_T_KN = 10
};
#define QASR_T_EMBED (1u << 20)
#define QASR_T_FINAL_NORM ((1u << 20) + 1u)
#define QASR_T_PREFIX_AUDIO (1ull << 32)   /* + slot * 65536 + refill index */
#define QASR_T_PREFIX_IDS ((1ull << 33))   /* + slot * 65536 + refill index */

uint64_t qasr_synth_key(uint64_t seed, uint64_t tensor_id);
/* n values ~ N(mean, std) rounded to f16. */
void qasr_synth_normal_f16(uint16_t* out, size_t n, uint64_t seed, uint64_t tensor_id,
                           float mean, float std_);
/* n ids uniform in [lo, hi). */
void qasr_synth_uniform_ids(int32_t* out, size_t n, uint64_t seed, uint64_t tensor_id,
                            int32_t lo, int32_t hi);
/* Per-row symmetric int8 quantisation (see header comment). */
void qasr_synth_quantize_rows(const uint16_t* w, int rows, int cols, int8_t* q,
                              uint16_t* scale);
/* IEEE binary16 <-> binary32, round to nearest even (matches half::f16::from_f32). */
uint16_t qasr_f32_to_f16(float f);
float qasr_f16_to_f32(uint16_t h);
void qasr_f32_to_f16_array(const float* in, uint16_t* out, size_t n);
void qasr_f16_to_f32_array(const uint16_t* in, float* out, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* QASR_SYNTH_H */
