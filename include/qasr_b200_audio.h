/*
 * qasr_b200_audio.h — C ABI of the B200 (sm_100a) audio tower: log-mel spectrogram in,
 * audio embedding rows out (the rows the text decoder's prefill takes as its audio
 * prefix, src/inference.rs:2263-2273).
 *
 * It replaces the reference's encoder pair: `GpuAudioEncoder::{load, encode,
 * encode_batch}` (src/audio_encoder_gpu.rs:599, 905-915, 971) and its CPU twin
 * `CpuAudioEncoder::{load, forward}` (src/audio_encoder.rs:676-770), whose arithmetic is
 * the one restated here: conv2d1..3 (3x3, stride 2, pad 1) + bias + GELU, conv_out +
 * sinusoidal positions, `encoder_layers` pre-LayerNorm transformer layers with attention
 * inside windows of tpc * (n_window_infer / (2 n_window)) tokens, ln_post, proj1 + GELU,
 * proj2.  The conventions of qasr_b200.h apply (plain C types, borrowed host buffers,
 * qasr_status results, one host thread per context, f16 as uint16_t bit patterns).
 */
#ifndef QASR_B200_AUDIO_H
#define QASR_B200_AUDIO_H

#include <stdint.h>

#include "qasr_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Hyper-parameters; mirrors `AudioEncoderConfig` (src/config.rs:26-64) with its
 * defaults (0.6B) in the comments.  The 1.7B tower: d_model 1024, 24 layers, 16 heads,
 * ffn 4096, output_dim 2048. */
typedef struct {
  int32_t d_model;                 /* 896 */
  int32_t encoder_layers;          /* 18 */
  int32_t encoder_attention_heads; /* 14 */
  int32_t encoder_ffn_dim;         /* 3584 */
  int32_t num_mel_bins;            /* 128 */
  int32_t downsample_hidden_size;  /* 480: conv channel count */
  int32_t max_source_positions;    /* 1500: rows of the sinusoidal table */
  int32_t n_window;                /* 50: a conv chunk is 2 * n_window mel frames */
  int32_t n_window_infer;          /* 800: attention window = tpc * (n_window_infer / chunk) */
  int32_t output_dim;              /* 1024: the text decoder's hidden size */
} qasr_audio_config;

/* Device weights, host pointers (copied).  f16 matrices are row-major [out][in] as the
 * checkpoint stores them (conv weights [out][in][3][3]); biases and LayerNorm parameters
 * are f32 (the CPU tower widens them, src/audio_encoder.rs:106-113, 141-149).  A NULL
 * bias means "no bias" (CpuAudioLinear's optional bias). */
typedef struct {
  const uint16_t* q_w; const float* q_b;       /* self_attn.q_proj [d][d] */
  const uint16_t* k_w; const float* k_b;       /* self_attn.k_proj */
  const uint16_t* v_w; const float* v_b;       /* self_attn.v_proj */
  const uint16_t* o_w; const float* o_b;       /* self_attn.out_proj */
  const float* ln1_w; const float* ln1_b;      /* self_attn_layer_norm */
  const float* ln2_w; const float* ln2_b;      /* final_layer_norm */
  const uint16_t* fc1_w; const float* fc1_b;   /* fc1 [ffn][d] */
  const uint16_t* fc2_w; const float* fc2_b;   /* fc2 [d][ffn] */
} qasr_audio_layer_weights;

typedef struct {
  const uint16_t* conv1_w; const float* conv1_b;        /* conv2d1 [C][1][3][3] */
  const uint16_t* conv2_w; const float* conv2_b;        /* conv2d2 [C][C][3][3] */
  const uint16_t* conv3_w; const float* conv3_b;        /* conv2d3 [C][C][3][3] */
  const uint16_t* conv_out_w; const float* conv_out_b;  /* conv_out [d][C * F3] */
  const qasr_audio_layer_weights* layers;               /* encoder_layers entries */
  const float* ln_post_w; const float* ln_post_b;
  const uint16_t* proj1_w; const float* proj1_b;        /* [d][d] */
  const uint16_t* proj2_w; const float* proj2_b;        /* [output_dim][d] */
} qasr_audio_weights;

typedef struct qasr_audio_ctx qasr_audio_ctx;

/* AsrConfig::from_file for the tower (src/config.rs:142-173): `{model_dir}/config.json`'s
 * thinker_config.audio_config (or the HF layout's top-level audio_config), absent fields
 * taking AudioEncoderConfig's defaults (src/config.rs:54-64).  err (optional) receives a
 * message on failure. */
qasr_status qasr_read_audio_config(const char* model_dir, qasr_audio_config* out, char* err, int errlen);

/* Token rows a mel of n_frames frames produces: full chunks give feo(2 n_window) rows,
 * the tail chunk feo(tail) (feo = three (l - 1) / 2 + 1 halvings, src/audio_encoder.rs:634-637). */
int32_t qasr_audio_token_count(const qasr_audio_config* cfg, int32_t n_frames);

/* Create a tower on `device` (GpuAudioEncoder::load's geometry checks,
 * src/audio_encoder_gpu.rs:599-760).  err (optional) receives a message on failure. */
qasr_status qasr_audio_create(const qasr_audio_config* cfg, int device, qasr_audio_ctx** out, char* err,
                              int errlen);
void qasr_audio_destroy(qasr_audio_ctx* ctx);
const char* qasr_audio_last_error(const qasr_audio_ctx* ctx);

/* Upload weights (GpuAudioEncoder::load / CpuAudioEncoder::load). */
qasr_status qasr_audio_load_weights(qasr_audio_ctx* ctx, const qasr_audio_weights* w);
/* The same from a checkpoint opened with qasr_checkpoint_open; prefix NULL =
 * "thinker.audio_tower" (HF "model.audio_tower." / "model.multi_modal_projector." names are
 * remapped, src/weights.rs:173-200). */
qasr_status qasr_audio_load_checkpoint(qasr_audio_ctx* ctx, qasr_checkpoint* ck, const char* prefix);

/* Encode one utterance (GpuAudioEncoder::encode): mel f32 [n_mels][n_frames] (mel-bin
 * major) -> out f16 [n_tokens][output_dim].  out_rows = capacity of `out` in rows; the
 * call fails with QASR_ERR_CAPACITY when the mel needs more. */
qasr_status qasr_audio_encode(qasr_audio_ctx* ctx, const float* mel, int32_t n_mels, int32_t n_frames,
                              uint16_t* out, int32_t out_rows, int32_t* n_tokens);

/* Encode several utterances with one transformer pass (GpuAudioEncoder::encode_batch,
 * src/audio_encoder_gpu.rs:956-1080): the utterances' token rows sit back to back and
 * every attention window stays inside its utterance, so each result equals a lone
 * encode.  outs[i] receives qasr_audio_token_count(n_frames[i]) rows. */
qasr_status qasr_audio_encode_batch(qasr_audio_ctx* ctx, int32_t n, const float* const* mels,
                                    const int32_t* n_frames, int32_t n_mels, uint16_t* const* outs);

/* Device-resident variant for a caller that keeps its buffers on the GPU: mel_dev f32
 * [n_mels][n_frames] and out_dev f16 [n_tokens][output_dim] are device pointers on the
 * context's device.  The work is enqueued on the context's stream (qasr_audio_stream)
 * and the call returns without waiting; qasr_audio_sync waits and reports device-side
 * failures. */
qasr_status qasr_audio_encode_device(qasr_audio_ctx* ctx, const float* mel_dev, int32_t n_mels,
                                     int32_t n_frames, uint16_t* out_dev, int32_t* n_tokens);
/* encode_batch for device-resident mels: mels_dev[i] f32 [n_mels][n_frames[i]] on the
 * context's device; out_dev f16 receives every utterance's rows back to back (utterance i
 * starts after the rows of 0..i-1); n_tokens (optional, host) receives each utterance's
 * row count.  Enqueued on the context's stream like qasr_audio_encode_device. */
qasr_status qasr_audio_encode_batch_device(qasr_audio_ctx* ctx, int32_t n, const float* const* mels_dev,
                                           const int32_t* n_frames, int32_t n_mels, uint16_t* out_dev,
                                           int32_t* n_tokens);
qasr_status qasr_audio_sync(qasr_audio_ctx* ctx);
void* qasr_audio_stream(qasr_audio_ctx* ctx);
/* Kernel launches issued by the audio tower so far (all of them this library's own). */
uint64_t qasr_audio_launch_count(const qasr_audio_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* QASR_B200_AUDIO_H */
