// Device kernels of the audio tower: the encoder that turns a log-mel spectrogram into the
// audio rows of the text decoder's prefill prefix.  It restates the reference's
// CpuAudioEncoder (src/audio_encoder.rs:669-770) / GpuAudioEncoder (src/audio_encoder_gpu.rs)
// for sm_100a.  The projections — conv2d2 / conv2d3 as GEMMs over an im2col operand,
// conv_out, the fused q|k|v, out_proj, fc1, fc2, proj1, proj2 — run on gemm_tc_kernel
// (tcgen05, weights as UMMA M) with the EPI_BIAS_* epilogues; this file holds the rest:
//
//   audio_conv1_kernel      conv2d1 (1 input channel, 9 taps) + bias + GELU, f32 CUDA cores
//   audio_im2col_kernel     3x3 / stride 2 / pad 1 operand of conv2d2 and conv2d3
//   audio_pack_kernel       conv3 output -> conv_out operand rows (valid tokens only) and the
//                           sinusoidal position rows the conv_out epilogue adds onto
//   audio_layernorm_kernel  LayerNorm (mean, variance, eps 1e-5) f32 -> f16 GEMM operand
//   audio_window_attention_kernel  bidirectional attention inside token windows
//
// Layouts in HBM (one round of conv chunks at a time; tokens of every chunk packed):
//   mel       f32 [n_mels][n_frames] per utterance (the reference's mel-bin-major input)
//   conv act  f16 [chunk][h][w][ldc] channel-last (ldc = channel count rounded up to 128)
//   im2col    f16 [chunk * ho * wo][kpad], k = (kh * 3 + kw) * C + c, zero-padded to kpad
//   h         f32 [tokens][d_model] residual stream (the CPU keeps f32 activations)
//   q|k|v     f32 [tokens][3 d_model]
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace qasr {

// gelu as the reference: 0.5 x (1 + erf(x / sqrt 2)) in f32 (src/audio_encoder.rs:177-179)
__device__ __forceinline__ float audio_gelu(float y) {
  return __fmul_rn(__fmul_rn(0.5f, y), __fadd_rn(1.0f, erff(__fmul_rn(y, 0.70710678118654752f))));
}

// One conv chunk: n_window * 2 mel frames of one utterance (the tail chunk zero-padded),
// src/audio_encoder.rs:702-735.
struct AudioChunk {
  int mel_off;   // element offset of the utterance's mel [n_mels][n_frames] in the mel buffer
  int n_frames;  // the utterance's frame count (row length of its mel)
  int frame0;    // first frame of the chunk
  int valid;     // frames of the chunk that exist (cs, or the tail)
  int tok0;      // first token row of the chunk in the packed token rows
  int ntok;      // tokens the chunk contributes (feo(valid))
};

// conv2d1 + bias + GELU over the chunks [0, n) of the current round: out[chunk][ho][wo][c].
// One thread computes 8 channels of one output position; the 9 taps are summed in
// (kh, kw) order in f32.  x beyond the chunk's valid frames or outside the mel bins is 0
// (the chunk buffer's zero fill and the conv padding, src/audio_encoder.rs:185-225).
__global__ void __launch_bounds__(256) audio_conv1_kernel(const float* __restrict__ mel,
                                                          const AudioChunk* __restrict__ chunks, int n,
                                                          int n_mels, int h1, int w1,
                                                          const float* __restrict__ w /*[C][9]*/,
                                                          const float* __restrict__ bias, int C,
                                                          __half* __restrict__ out, int ldc) {
  extern __shared__ float c1_smem[];
  float* sw = c1_smem;           // [C][9]
  float* sb = c1_smem + C * 9;   // [C]
  for (int i = threadIdx.x; i < C * 9; i += blockDim.x) sw[i] = w[i];
  for (int i = threadIdx.x; i < C; i += blockDim.x) sb[i] = bias[i];
  __syncthreads();
  const int groups = C >> 3;
  const long long total = static_cast<long long>(n) * h1 * w1 * groups;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    const long long pos = i / groups;
    const int wo = static_cast<int>(pos % w1);
    const int ho = static_cast<int>((pos / w1) % h1);
    const int ch = static_cast<int>(pos / (static_cast<long long>(w1) * h1));
    const AudioChunk k = chunks[ch];
    float x[9];
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
#pragma unroll
      for (int kw = 0; kw < 3; ++kw) {
        const int mb = ho * 2 + kh - 1, fr = wo * 2 + kw - 1;
        x[kh * 3 + kw] = (mb >= 0 && mb < n_mels && fr >= 0 && fr < k.valid)
                             ? mel[k.mel_off + static_cast<long long>(mb) * k.n_frames + k.frame0 + fr]
                             : 0.0f;
      }
    }
    alignas(16) __half o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = g * 8 + j;
      float acc = 0.0f;
#pragma unroll
      for (int t = 0; t < 9; ++t) acc = __fadd_rn(acc, __fmul_rn(sw[c * 9 + t], x[t]));
      o[j] = __float2half_rn(audio_gelu(__fadd_rn(acc, sb[c])));
    }
    *reinterpret_cast<uint4*>(out + pos * ldc + g * 8) = *reinterpret_cast<const uint4*>(o);
  }
}

// im2col of a 3x3 / stride 2 / pad 1 conv over channel-last activations
// act[chunk][h][w][ldc] (C channels used): X[(chunk * ho_n + ho) * wo_n + wo][k], k = tap * C + c,
// zero outside the plane and for k >= 9 C (up to kpad).  One thread = one 16-byte vector.
__global__ void __launch_bounds__(256) audio_im2col_kernel(const __half* __restrict__ act, int n, int h, int w,
                                                           int C, int ldc, int ho_n, int wo_n,
                                                           __half* __restrict__ X, int kpad) {
  const int vrow = kpad >> 3;
  const long long total = static_cast<long long>(n) * ho_n * wo_n * vrow;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % vrow);
    const long long pos = i / vrow;
    const int wo = static_cast<int>(pos % wo_n);
    const int ho = static_cast<int>((pos / wo_n) % ho_n);
    const int ch = static_cast<int>(pos / (static_cast<long long>(wo_n) * ho_n));
    const int k0 = v * 8;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (k0 < 9 * C) {
      const int tap = k0 / C, c0 = k0 - tap * C;
      const int ih = ho * 2 + tap / 3 - 1, iw = wo * 2 + tap % 3 - 1;
      if (ih >= 0 && ih < h && iw >= 0 && iw < w)
        val = *reinterpret_cast<const uint4*>(act + ((static_cast<long long>(ch) * h + ih) * w + iw) * ldc + c0);
    }
    *reinterpret_cast<uint4*>(X + pos * kpad + k0) = val;
  }
}

// conv3 output act[chunk][f][t][ldc] -> the conv_out operand rows of the chunk's valid tokens,
// packed[tok][c * F + f] (the permute of src/audio_encoder.rs:290-305, and the packing of
// :736-744), and h[tok][:] = pe[t][:] (the conv_out epilogue then adds the projection:
// pe + (acc + bias) == (acc + bias) + pe, as the reference orders it).
__global__ void __launch_bounds__(256) audio_pack_kernel(const __half* __restrict__ act, const AudioChunk* __restrict__ chunks,
                                                         int n, int F, int T, int C, int ldc,
                                                         __half* __restrict__ packed, float* __restrict__ h,
                                                         const float* __restrict__ pe, int dm) {
  const int ch = blockIdx.y;
  if (ch >= n) return;
  const AudioChunk k = chunks[ch];
  const int per_tok = C;  // one thread per (token, channel): F contiguous outputs
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < k.ntok * per_tok; i += gridDim.x * blockDim.x) {
    const int t = i / per_tok, c = i - t * per_tok;
    __half* dst = packed + static_cast<long long>(k.tok0 + t) * (C * F) + c * F;
    for (int f = 0; f < F; ++f)
      dst[f] = act[((static_cast<long long>(ch) * F + f) * T + t) * ldc + c];
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < k.ntok * dm; i += gridDim.x * blockDim.x) {
    const int t = i / dm, j = i - t * dm;
    h[static_cast<long long>(k.tok0 + t) * dm + j] = pe[t * dm + j];
  }
}

// LayerNorm over d (src/audio_encoder.rs:152-172): mean, then the mean of squared
// deviations, inv_std = 1 / sqrt(var + eps); o = (x - mean) * inv_std * w + b.  One warp per
// row; f32 math with IEEE-rounded steps, the output rounded once to f16 (a GEMM operand).
__global__ void __launch_bounds__(256) audio_layernorm_kernel(const float* __restrict__ x, int rows, int d,
                                                              const float* __restrict__ w,
                                                              const float* __restrict__ b, float eps,
                                                              __half* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* xr = x + static_cast<long long>(warp) * d;
  float s = 0.0f;
  for (int j = lane; j < d; j += 32) s = __fadd_rn(s, xr[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  const float mean = __fdiv_rn(s, static_cast<float>(d));
  float v = 0.0f;
  for (int j = lane; j < d; j += 32) {
    const float dv = __fsub_rn(xr[j], mean);
    v = __fadd_rn(v, __fmul_rn(dv, dv));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, static_cast<float>(d)), eps)));
  __half* orow = out + static_cast<long long>(warp) * d;
  for (int j = lane; j < d; j += 32)
    orow[j] = __float2half_rn(__fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[j], mean), inv), w[j]), b[j]));
}

// Attention inside token windows (attention_window, src/audio_encoder.rs:519-566): window
// `blockIdx.x` = rows [win[2i], win[2i] + win[2i+1]), head `blockIdx.y`.  q|k|v come from
// qkv [tokens][3 dm] f32 (head h at columns h*hd, dm + h*hd, 2 dm + h*hd).  Per query row:
// s_j = (q . k_j) * scale (the dot summed over dims in order, one rounding per step, like
// the reference), softmax with the row max, p_j = exp(s_j - max), inv = 1 / sum p,
// out = sum_j (p_j * inv) v_j summed over keys in order; out is rounded to f16 (the
// out_proj operand).  K and V of the window sit in shared memory (row stride hd + 1:
// conflict-free column reads) when they fit, else they are read from global memory.
constexpr int AUDIO_ATTN_THREADS = 256;
constexpr int AUDIO_ATTN_WARPS = AUDIO_ATTN_THREADS / 32;
constexpr int AUDIO_ATTN_MAX_HD = 128;

__host__ __device__ constexpr size_t audio_attn_smem_floats(int wlen, int hd, bool kv_in_smem) {
  return (kv_in_smem ? static_cast<size_t>(2) * wlen * (hd + 1) : 0) +
         static_cast<size_t>(AUDIO_ATTN_WARPS) * (wlen + hd);
}

template <bool KV_SMEM>
__global__ void __launch_bounds__(AUDIO_ATTN_THREADS) audio_window_attention_kernel(
    const float* __restrict__ qkv, const int* __restrict__ win, int dm, int hd, float scale,
    int wmax, __half* __restrict__ out) {
  extern __shared__ float at_smem[];
  const int start = win[2 * blockIdx.x], len = win[2 * blockIdx.x + 1];
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long ld = 3LL * dm;
  const int ks = KV_SMEM ? hd + 1 : static_cast<int>(ld);  // row stride of K / V
  const float* K;
  const float* V;
  float* pbase = at_smem + (KV_SMEM ? static_cast<size_t>(2) * wmax * (hd + 1) : 0);
  if constexpr (KV_SMEM) {
    float* sk = at_smem;
    float* sv = at_smem + static_cast<size_t>(wmax) * (hd + 1);
    for (int i = threadIdx.x; i < len * hd; i += blockDim.x) {
      const int r = i / hd, d = i - r * hd;
      const float* row = qkv + (start + r) * ld + h * hd + d;
      sk[r * (hd + 1) + d] = row[dm];
      sv[r * (hd + 1) + d] = row[2 * dm];
    }
    __syncthreads();
    K = sk;
    V = sv;
  } else {
    K = qkv + start * ld + dm + h * hd;
    V = qkv + start * ld + 2 * dm + h * hd;
  }
  float* p = pbase + static_cast<size_t>(warp) * (wmax + hd);  // [len] probabilities
  float* qs = p + wmax;                                         // [hd] this row's q
  for (int r = warp; r < len; r += AUDIO_ATTN_WARPS) {
    const float* qrow = qkv + (start + r) * ld + h * hd;
    for (int d = lane; d < hd; d += 32) qs[d] = qrow[d];
    __syncwarp();
    float mx = -INFINITY;
    for (int j = lane; j < len; j += 32) {
      const float* kr = K + static_cast<long long>(j) * ks;
      float dot = 0.0f;
      for (int d = 0; d < hd; ++d) dot = __fadd_rn(dot, __fmul_rn(qs[d], kr[d]));
      const float sc = __fmul_rn(dot, scale);
      p[j] = sc;
      mx = fmaxf(mx, sc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int j = lane; j < len; j += 32) {
      const float e = expf(__fsub_rn(p[j], mx));
      p[j] = e;
      sum = __fadd_rn(sum, e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float inv = __fdiv_rn(1.0f, sum);
    __syncwarp();
    float acc[AUDIO_ATTN_MAX_HD / 32];
#pragma unroll
    for (int i = 0; i < AUDIO_ATTN_MAX_HD / 32; ++i) acc[i] = 0.0f;
    for (int j = 0; j < len; ++j) {
      const float wj = __fmul_rn(p[j], inv);
      const float* vr = V + static_cast<long long>(j) * ks;
#pragma unroll
      for (int i = 0; i < AUDIO_ATTN_MAX_HD / 32; ++i)
        if (lane + 32 * i < hd) acc[i] = __fadd_rn(acc[i], __fmul_rn(wj, vr[lane + 32 * i]));
    }
    __half* orow = out + static_cast<long long>(start + r) * dm + h * hd;
#pragma unroll
    for (int i = 0; i < AUDIO_ATTN_MAX_HD / 32; ++i)
      if (lane + 32 * i < hd) orow[lane + 32 * i] = __float2half_rn(acc[i]);
    __syncwarp();
  }
}

}  // namespace qasr
