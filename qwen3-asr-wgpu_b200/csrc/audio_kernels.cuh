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
//                           sinusoidal position rows the conv_out output is added onto
//   audio_residual_layernorm_kernel  h += delta (a block's output), then LayerNorm
//                           (mean, variance, eps 1e-5) f32 -> f16 GEMM operand
//   audio_window_attention_tc_kernel  bidirectional attention inside token windows on the
//                           tensor cores (mma.sync, TF32); audio_window_attention_kernel, the
//                           CUDA-core f32 form, for windows longer than 128 tokens
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

#include "device_common.cuh"
#include "gemm_tc.cuh"  // griddep_wait / griddep_launch_dependents

namespace qasr {

// Every kernel here is launched as a programmatic dependent of the kernel before it: it may
// become resident while that kernel drains, waits (griddepcontrol.wait) before reading
// anything, and then lets the next launch (a GEMM that streams its weights before its own
// wait) be scheduled.  The dependent grid starts only after every CTA of this one has
// issued the trigger, i.e. is resident, so no kernel ever waits for resources held by a
// kernel that waits on it.
__device__ __forceinline__ void audio_pdl_entry() {
  griddep_wait();
  griddep_launch_dependents();
}

// 16-byte global -> shared copy that bypasses the registers (cp.async, L2 only): a thread
// issues all of its copies before waiting for any.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// gelu as the reference: 0.5 x (1 + erf(x / sqrt 2)) in f32 (src/audio_encoder.rs:177-179)
__device__ __forceinline__ float audio_gelu(float y) {
  return __fmul_rn(__fmul_rn(0.5f, y), __fadd_rn(1.0f, erff(__fmul_rn(y, 0.70710678118654752f))));
}

// One conv chunk: n_window * 2 mel frames of one utterance (the tail chunk zero-padded),
// src/audio_encoder.rs:702-735.
struct AudioChunk {
  const float* mel;  // the utterance's mel [n_mels][n_frames]
  int n_frames;  // the utterance's frame count (row length of its mel)
  int frame0;    // first frame of the chunk
  int valid;     // frames of the chunk that exist (cs, or the tail)
  int tok0;      // first token row of the chunk in the packed token rows
  int ntok;      // tokens the chunk contributes (feo(valid))
};

// conv2d1 + bias + GELU over the chunks [0, n) of the current round: out[chunk][ho][wo][c].
// A thread owns one group of 8 channels for its whole grid-stride loop (the block is a
// multiple of the group count, so the group is fixed per thread) and holds those 8 x 9
// weights in registers, loaded once; each item is AUDIO_C1_POS consecutive output columns of
// one output row.  The 9 taps are summed in (kh, kw) order in f32.  x beyond the chunk's
// valid frames or outside the mel bins is 0 (the chunk buffer's zero fill and the conv
// padding, src/audio_encoder.rs:185-225).  Index arithmetic is 32-bit (a round holds
// < 2^31 outputs; the host checks): a 64-bit division is a long software sequence.
constexpr int AUDIO_C1_POS = 2;
__host__ __device__ constexpr int audio_conv1_block(int groups) { return groups * (256 / groups); }
__global__ void __launch_bounds__(256, 2) audio_conv1_kernel(const AudioChunk* __restrict__ chunks, int n,
                                                             int n_mels, int h1, int w1,
                                                             const float* __restrict__ w /*[C][9]*/,
                                                             const float* __restrict__ bias, int C,
                                                             __half* __restrict__ out, int ldc) {
  audio_pdl_entry();
  const unsigned groups = static_cast<unsigned>(C) >> 3;
  const unsigned per_block = blockDim.x / groups;  // items of one group in flight per block
  if (threadIdx.x >= per_block * groups) return;
  const int g = static_cast<int>(threadIdx.x % groups);
  float wr[8][9], br[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int t = 0; t < 9; ++t) wr[j][t] = __ldg(w + (g * 8 + j) * 9 + t);
    br[j] = __ldg(bias + g * 8 + j);
  }
  const unsigned wq = (static_cast<unsigned>(w1) + AUDIO_C1_POS - 1) / AUDIO_C1_POS;  // column groups per row
  const unsigned items = static_cast<unsigned>(n) * h1 * wq;
  for (unsigned it = blockIdx.x * per_block + threadIdx.x / groups; it < items; it += gridDim.x * per_block) {
    const int wo0 = static_cast<int>(it % wq) * AUDIO_C1_POS;
    const unsigned row = it / wq;  // chunk * h1 + ho
    const int ho = static_cast<int>(row % static_cast<unsigned>(h1));
    const int ch = static_cast<int>(row / static_cast<unsigned>(h1));
    const AudioChunk k = chunks[ch];
    // the 3 mel rows x (2 * AUDIO_C1_POS + 1) frames this item reads
    float x[3][2 * AUDIO_C1_POS + 1];
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
      const int mb = ho * 2 + kh - 1;
#pragma unroll
      for (int f = 0; f < 2 * AUDIO_C1_POS + 1; ++f) {
        const int fr = wo0 * 2 - 1 + f;
        x[kh][f] = (mb >= 0 && mb < n_mels && fr >= 0 && fr < k.valid)
                       ? __ldg(k.mel + static_cast<size_t>(mb) * k.n_frames + k.frame0 + fr)
                       : 0.0f;
      }
    }
#pragma unroll
    for (int q = 0; q < AUDIO_C1_POS; ++q) {
      const int wo = wo0 + q;
      if (wo < w1) {
        alignas(16) __half o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float acc = 0.0f;
#pragma unroll
          for (int kh = 0; kh < 3; ++kh)
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) acc = __fadd_rn(acc, __fmul_rn(wr[j][kh * 3 + kw], x[kh][2 * q + kw]));
          o[j] = __float2half_rn(audio_gelu(__fadd_rn(acc, br[j])));
        }
        *reinterpret_cast<uint4*>(out + (static_cast<size_t>(row) * w1 + wo) * ldc + g * 8) =
            *reinterpret_cast<const uint4*>(o);
      }
    }
  }
}

// im2col of a 3x3 / stride 2 / pad 1 conv over channel-last activations
// act[chunk][h][w][ldc] (C channels used): X[(chunk * ho_n + ho) * wo_n + wo][k], k = tap * C + c,
// zero outside the plane and for k >= 9 C (up to kpad).  One thread = one 16-byte vector.
__global__ void __launch_bounds__(256) audio_im2col_kernel(const __half* __restrict__ act, int n, int h, int w,
                                                           int C, int ldc, int ho_n, int wo_n,
                                                           __half* __restrict__ X, int kpad) {
  audio_pdl_entry();
  const unsigned vrow = static_cast<unsigned>(kpad) >> 3;
  const unsigned total = static_cast<unsigned>(n) * ho_n * wo_n * vrow;  // < 2^31 (host-checked)
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int v = static_cast<int>(i % vrow);
    const unsigned pos = i / vrow;
    const int wo = static_cast<int>(pos % static_cast<unsigned>(wo_n));
    const int ho = static_cast<int>((pos / static_cast<unsigned>(wo_n)) % static_cast<unsigned>(ho_n));
    const int ch = static_cast<int>(pos / (static_cast<unsigned>(wo_n) * ho_n));
    const int k0 = v * 8;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (k0 < 9 * C) {
      const int tap = k0 / C, c0 = k0 - tap * C;
      const int ih = ho * 2 + tap / 3 - 1, iw = wo * 2 + tap % 3 - 1;
      if (ih >= 0 && ih < h && iw >= 0 && iw < w)
        val = *reinterpret_cast<const uint4*>(act + ((static_cast<long long>(ch) * h + ih) * w + iw) * ldc + c0);
    }
    *reinterpret_cast<uint4*>(X + static_cast<size_t>(pos) * kpad + k0) = val;
  }
}

// conv3 output act[chunk][f][t][ldc] -> the conv_out operand rows of the chunk's valid tokens,
// packed[tok][c * F + f] (the permute of src/audio_encoder.rs:290-305, and the packing of
// :736-744), and h[tok][:] = pe[t][:] (the first residual add then adds the conv_out
// projection: pe + (acc + bias) == (acc + bias) + pe, as the reference orders it).
__global__ void __launch_bounds__(256) audio_pack_kernel(const __half* __restrict__ act, const AudioChunk* __restrict__ chunks,
                                                         int n, int F, int T, int C, int ldc,
                                                         __half* __restrict__ packed, float* __restrict__ h,
                                                         const float* __restrict__ pe, int dm) {
  audio_pdl_entry();
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

// Residual add + LayerNorm (CpuAudioLayer::forward's `x += block(x)` then the next
// CpuAudioLayerNorm::forward, src/audio_encoder.rs:614-630, 152-172): when `delta` is given
// the row becomes h = h + delta (stored back: the f32 residual stream); then mean, the mean
// of squared deviations, inv_std = 1 / sqrt(var + eps), o = (h - mean) * inv_std * w + b.
// One warp per row, the row held in registers (lane l: float4 vectors l, l + 32, ...; every
// load in flight at once); f32 math with IEEE-rounded steps, the output rounded once to f16
// (a GEMM operand).  d is a multiple of 4 and at most 128 * AUDIO_LN_MAXV.
constexpr int AUDIO_LN_MAXV = 10;
__global__ void __launch_bounds__(256) audio_residual_layernorm_kernel(float* __restrict__ x,
                                                                       const float* __restrict__ delta, int rows,
                                                                       int d, const float* __restrict__ w,
                                                                       const float* __restrict__ b, float eps,
                                                                       __half* __restrict__ out) {
  audio_pdl_entry();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int nv = d >> 2;
  float4* xr = reinterpret_cast<float4*>(x + static_cast<size_t>(warp) * d);
  float4 v[AUDIO_LN_MAXV];
#pragma unroll
  for (int k = 0; k < AUDIO_LN_MAXV; ++k)
    v[k] = lane + 32 * k < nv ? xr[lane + 32 * k] : make_float4(0.f, 0.f, 0.f, 0.f);
  if (delta != nullptr) {
    const float4* dr = reinterpret_cast<const float4*>(delta + static_cast<size_t>(warp) * d);
    float4 dv[AUDIO_LN_MAXV];
#pragma unroll
    for (int k = 0; k < AUDIO_LN_MAXV; ++k)
      dv[k] = lane + 32 * k < nv ? dr[lane + 32 * k] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < AUDIO_LN_MAXV; ++k) {
      if (lane + 32 * k < nv) {
        v[k] = make_float4(__fadd_rn(v[k].x, dv[k].x), __fadd_rn(v[k].y, dv[k].y), __fadd_rn(v[k].z, dv[k].z),
                           __fadd_rn(v[k].w, dv[k].w));
        xr[lane + 32 * k] = v[k];
      }
    }
  }
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < AUDIO_LN_MAXV; ++k)
    s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[k].x), v[k].y), v[k].z), v[k].w);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  const float mean = __fdiv_rn(s, static_cast<float>(d));
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < AUDIO_LN_MAXV; ++k) {
    if (lane + 32 * k < nv) {
      const float a0 = __fsub_rn(v[k].x, mean), a1 = __fsub_rn(v[k].y, mean), a2 = __fsub_rn(v[k].z, mean),
                  a3 = __fsub_rn(v[k].w, mean);
      q = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(q, __fmul_rn(a0, a0)), __fmul_rn(a1, a1)), __fmul_rn(a2, a2)),
                    __fmul_rn(a3, a3));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, o));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, static_cast<float>(d)), eps)));
  __half2* orow = reinterpret_cast<__half2*>(out + static_cast<size_t>(warp) * d);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
  for (int k = 0; k < AUDIO_LN_MAXV; ++k) {
    const int c = lane + 32 * k;
    if (c < nv) {
      const float4 ww = w4[c], bb = b4[c];
      auto f = [&](float xv, float wv, float bv) {
        return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv, mean), inv), wv), bv);
      };
      orow[2 * c] = __floats2half2_rn(f(v[k].x, ww.x, bb.x), f(v[k].y, ww.y, bb.y));
      orow[2 * c + 1] = __floats2half2_rn(f(v[k].z, ww.z, bb.z), f(v[k].w, ww.w, bb.w));
    }
  }
}

// Attention inside token windows (attention_window, src/audio_encoder.rs:519-566): window
// `blockIdx.x` = rows [win[2i], win[2i] + win[2i+1]), head `blockIdx.y`, query rows
// [AUDIO_ATTN_QB * blockIdx.z, +AUDIO_ATTN_QB) of the window.  q|k|v come from qkv
// [tokens][3 dm] f32 (head h at columns h*hd, dm + h*hd, 2 dm + h*hd).  Per query row:
// s_j = (q . k_j) * scale (the dot summed over dims in order, like
// the reference, but each step a fused multiply-add, so a dot can differ from the
// reference's in the last bit), softmax with the row max, p_j = exp(s_j - max),
// inv = 1 / sum p, out = sum_j (p_j * inv) v_j summed over keys in order (fused
// multiply-adds); out is rounded to f16 (the out_proj operand).  The CTA's q rows and, when they fit, the window's K (rows padded to
// hd + 4 floats: lane j reads key j's 16-byte vectors without bank conflicts) and V come
// into shared memory with cp.async, every copy in flight at once; otherwise K and V are
// read from global memory.  A warp takes two query rows at a time and a lane four keys at
// a time, so each K / V read feeds several independent accumulation chains.
constexpr int AUDIO_ATTN_THREADS = 256;
constexpr int AUDIO_ATTN_WARPS = AUDIO_ATTN_THREADS / 32;
constexpr int AUDIO_ATTN_MAX_HD = 128;
constexpr int AUDIO_ATTN_QB = 16;  // query rows per CTA (two per warp)

__host__ __device__ constexpr size_t audio_attn_smem_floats(int wlen, int hd, bool kv_in_smem) {
  return (kv_in_smem ? static_cast<size_t>(wlen) * (2 * hd + 4) : 0) + static_cast<size_t>(AUDIO_ATTN_QB) * hd +
         static_cast<size_t>(AUDIO_ATTN_WARPS) * 2 * wlen;
}

template <bool KV_SMEM>
__global__ void __launch_bounds__(AUDIO_ATTN_THREADS) audio_window_attention_kernel(
    const float* __restrict__ qkv, const int* __restrict__ win, int dm, int hd, float scale,
    int wmax, __half* __restrict__ out) {
  audio_pdl_entry();
  extern __shared__ __align__(16) float at_smem[];
  const int start = win[2 * blockIdx.x], len = win[2 * blockIdx.x + 1];
  const int r0 = blockIdx.z * AUDIO_ATTN_QB;
  if (r0 >= len) return;
  const int r1 = min(len, r0 + AUDIO_ATTN_QB);
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t ld = 3 * static_cast<size_t>(dm);
  const int v4 = hd >> 2;  // 16-byte vectors per head row
  const float* qkv_rows = qkv + static_cast<size_t>(start) * ld + h * hd;  // row r of the window: + r * ld
  float* sk = at_smem;                                                      // [wmax][hd + 4]
  float* sv = sk + (KV_SMEM ? static_cast<size_t>(wmax) * (hd + 4) : 0);   // [wmax][hd]
  float* sq = sv + (KV_SMEM ? static_cast<size_t>(wmax) * hd : 0);         // [QB][hd]
  float* p0 = sq + AUDIO_ATTN_QB * hd + static_cast<size_t>(warp) * 2 * wmax;  // [len] probabilities, row a
  float* p1 = p0 + wmax;                                                        // row b
  if constexpr (KV_SMEM) {
    for (int i = threadIdx.x; i < len * v4; i += blockDim.x) {
      const int r = i / v4, c = (i - r * v4) * 4;
      const float* row = qkv_rows + r * ld + c;
      cp_async16(sk + r * (hd + 4) + c, row + dm);
      cp_async16(sv + r * hd + c, row + 2 * dm);
    }
  }
  for (int i = threadIdx.x; i < (r1 - r0) * v4; i += blockDim.x) {
    const int r = i / v4, c = (i - r * v4) * 4;
    cp_async16(sq + r * hd + c, qkv_rows + (r0 + r) * ld + c);
  }
  cp_async_wait_all();
  __syncthreads();
  const float* K = KV_SMEM ? sk : qkv_rows + dm;
  const float* V = KV_SMEM ? sv : qkv_rows + 2 * dm;
  const size_t ks = KV_SMEM ? static_cast<size_t>(hd + 4) : ld;
  const size_t vs = KV_SMEM ? static_cast<size_t>(hd) : ld;
  for (int ra = r0 + 2 * warp; ra < r1; ra += 2 * AUDIO_ATTN_WARPS) {
    const bool two = ra + 1 < r1;  // row b = ra + 1 (or a repeat of row a, discarded)
    const float4* qa = reinterpret_cast<const float4*>(sq + (ra - r0) * hd);
    const float4* qb = two ? qa + v4 : qa;
    float mxa = -INFINITY, mxb = -INFINITY;
    for (int j0 = 0; j0 < len; j0 += 128) {
      const float4* kp[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int j = j0 + lane + 32 * t;
        kp[t] = reinterpret_cast<const float4*>(K + static_cast<size_t>(j < len ? j : 0) * ks);
      }
      float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = 0; c < v4; ++c) {
        const float4 x = qa[c], y = qb[c];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float4 kv = kp[t][c];
          da[t] = __fmaf_rn(x.x, kv.x, da[t]);
          db[t] = __fmaf_rn(y.x, kv.x, db[t]);
          da[t] = __fmaf_rn(x.y, kv.y, da[t]);
          db[t] = __fmaf_rn(y.y, kv.y, db[t]);
          da[t] = __fmaf_rn(x.z, kv.z, da[t]);
          db[t] = __fmaf_rn(y.z, kv.z, db[t]);
          da[t] = __fmaf_rn(x.w, kv.w, da[t]);
          db[t] = __fmaf_rn(y.w, kv.w, db[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int j = j0 + lane + 32 * t;
        if (j < len) {
          const float sa = __fmul_rn(da[t], scale), sb = __fmul_rn(db[t], scale);
          p0[j] = sa;
          p1[j] = sb;
          mxa = fmaxf(mxa, sa);
          mxb = fmaxf(mxb, sb);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, o));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, o));
    }
    float suma = 0.0f, sumb = 0.0f;
    for (int j = lane; j < len; j += 32) {
      const float ea = expf(__fsub_rn(p0[j], mxa)), eb = expf(__fsub_rn(p1[j], mxb));
      p0[j] = ea;
      p1[j] = eb;
      suma = __fadd_rn(suma, ea);
      sumb = __fadd_rn(sumb, eb);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      suma = __fadd_rn(suma, __shfl_xor_sync(0xffffffffu, suma, o));
      sumb = __fadd_rn(sumb, __shfl_xor_sync(0xffffffffu, sumb, o));
    }
    const float inva = __fdiv_rn(1.0f, suma), invb = __fdiv_rn(1.0f, sumb);
    __syncwarp();
    // lane owns dims 2 lane + 64 i, +1 (hd is a multiple of 32: a lane's pair exists or not)
    float2 acca[AUDIO_ATTN_MAX_HD / 64], accb[AUDIO_ATTN_MAX_HD / 64];
#pragma unroll
    for (int i = 0; i < AUDIO_ATTN_MAX_HD / 64; ++i) acca[i] = accb[i] = make_float2(0.f, 0.f);
    for (int j = 0; j < len; ++j) {
      const float wa = __fmul_rn(p0[j], inva), wb = __fmul_rn(p1[j], invb);
      const float* vr = V + j * vs;
#pragma unroll
      for (int i = 0; i < AUDIO_ATTN_MAX_HD / 64; ++i) {
        const int d = 2 * lane + 64 * i;
        if (d < hd) {
          const float2 vv = *reinterpret_cast<const float2*>(vr + d);
          acca[i].x = __fmaf_rn(wa, vv.x, acca[i].x);
          acca[i].y = __fmaf_rn(wa, vv.y, acca[i].y);
          accb[i].x = __fmaf_rn(wb, vv.x, accb[i].x);
          accb[i].y = __fmaf_rn(wb, vv.y, accb[i].y);
        }
      }
    }
    __half* oa = out + static_cast<size_t>(start + ra) * dm + h * hd;
#pragma unroll
    for (int i = 0; i < AUDIO_ATTN_MAX_HD / 64; ++i) {
      const int d = 2 * lane + 64 * i;
      if (d < hd) {
        *reinterpret_cast<__half2*>(oa + d) = __floats2half2_rn(acca[i].x, acca[i].y);
        if (two) *reinterpret_cast<__half2*>(oa + dm + d) = __floats2half2_rn(accb[i].x, accb[i].y);
      }
    }
    __syncwarp();
  }
}

// Attention inside a window on the tensor cores (mma.sync m16n8k8, TF32 operands, f32
// accumulate) for windows of at most AUDIO_TCATT_MAXW tokens: CTA = (window, head); q, K and
// V of the window come into shared memory by cp.async (rows past the window zero-filled);
// CTA z of a (window, head) takes query rows [64 z, 64 z + 64), a warp 16 of them: S = Q K^T (16 x len, registers), scaled, exact
// softmax per row in f32 (row max, exp(s - max), sum, inv = 1 / sum, p * inv — the
// reference's steps, src/audio_encoder.rs:519-566), P through shared memory, O = P V; O is
// rounded to f16 (the out_proj operand).  q, k, p and v are rounded to TF32 (10-bit
// mantissa) for the products: a numpy emulation puts the tower's output within 7.2e-4 of
// the f32 oracle either way.  Row strides (hd + 4 for q / K / P, hd + 8 for V) make every
// fragment read conflict-free.
constexpr int AUDIO_TCATT_MAXW = 128;
constexpr int AUDIO_TCATT_WARPS = 4;
constexpr int AUDIO_TCATT_QROWS = 16 * AUDIO_TCATT_WARPS;  // query rows per CTA

__host__ __device__ constexpr size_t audio_tcatt_smem_floats(int wlen, int hd) {
  return static_cast<size_t>(((wlen + 15) / 16) * 16) * (2 * hd + 12) +
         static_cast<size_t>(AUDIO_TCATT_QROWS) * (hd + 4) +
         static_cast<size_t>(AUDIO_TCATT_WARPS) * 16 * (((wlen + 7) / 8) * 8 + 4);
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int HD>
__global__ void __launch_bounds__(AUDIO_TCATT_WARPS * 32) audio_window_attention_tc_kernel(
    const float* __restrict__ qkv, const int* __restrict__ win, int dm, float scale, int wmax,
    __half* __restrict__ out) {
  audio_pdl_entry();
  extern __shared__ __align__(16) float tc_smem[];
  constexpr int QS = HD + 4, KS = HD + 4, VS = HD + 8;
  const int start = win[2 * blockIdx.x], len = win[2 * blockIdx.x + 1];
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = blockIdx.z * AUDIO_TCATT_QROWS;  // this CTA's first query row
  if (q0 >= len) return;
  const int rows16 = ((wmax + 15) / 16) * 16;  // padded window rows in shared memory
  const int ntiles = (len + 7) >> 3;           // key tiles of 8
  const int ps = ((wmax + 7) / 8) * 8 + 4;     // P row stride
  float* sk = tc_smem;                         // [rows16][KS]
  float* sv = sk + static_cast<size_t>(rows16) * KS;                  // [rows16][VS]
  float* sq = sv + static_cast<size_t>(rows16) * VS;                  // [QROWS][QS]
  float* sp = sq + static_cast<size_t>(AUDIO_TCATT_QROWS) * QS + static_cast<size_t>(warp) * 16 * ps;  // [16][ps]
  const size_t ld = 3 * static_cast<size_t>(dm);
  const float* base = qkv + static_cast<size_t>(start) * ld + h * HD;
  constexpr int V4 = HD / 4;
  const int lpad = ((len + 7) / 8) * 8;  // key rows that fragments touch
  for (int i = threadIdx.x; i < lpad * V4; i += blockDim.x) {
    const int r = i / V4, c = (i - r * V4) * 4;
    if (r < len) {
      const float* row = base + r * ld + c;
      cp_async16(sk + r * KS + c, row + dm);
      cp_async16(sv + r * VS + c, row + 2 * dm);
    } else {  // padding rows: zeros (a zero V row times a zero probability stays 0)
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(sk + r * KS + c) = z;
      *reinterpret_cast<float4*>(sv + r * VS + c) = z;
    }
  }
  for (int i = threadIdx.x; i < AUDIO_TCATT_QROWS * V4; i += blockDim.x) {
    const int r = i / V4, c = (i - r * V4) * 4;
    if (q0 + r < len)
      cp_async16(sq + r * QS + c, base + (q0 + r) * ld + c);
    else
      *reinterpret_cast<float4*>(sq + r * QS + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  cp_async_wait_all();
  __syncthreads();
  {
    const int mt = warp;  // query rows q0 + 16 mt ...
    if (q0 + mt * 16 >= len) return;
    const float* qa = sq + (mt * 16 + g) * QS;
    float sacc[AUDIO_TCATT_MAXW / 8][4];
#pragma unroll
    for (int nt = 0; nt < AUDIO_TCATT_MAXW / 8; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 8; ++kk) {
      const uint32_t a0 = to_tf32(qa[kk * 8 + t]), a1 = to_tf32(qa[8 * QS + kk * 8 + t]);
      const uint32_t a2 = to_tf32(qa[kk * 8 + t + 4]), a3 = to_tf32(qa[8 * QS + kk * 8 + t + 4]);
#pragma unroll
      for (int nt = 0; nt < AUDIO_TCATT_MAXW / 8; ++nt) {
        if (nt < ntiles) {
          const float* kb = sk + (nt * 8 + g) * KS + kk * 8;
          mma_tf32(sacc[nt], a0, a1, a2, a3, to_tf32(kb[t]), to_tf32(kb[t + 4]));
        }
      }
    }
    // exact softmax of rows g (elements 0, 1) and g + 8 (2, 3); columns >= len masked
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < AUDIO_TCATT_MAXW / 8; ++nt) {
      if (nt < ntiles) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = nt * 8 + 2 * t + (e & 1);
          sacc[nt][e] = col < len ? __fmul_rn(sacc[nt][e], scale) : -INFINITY;
        }
        mx0 = fmaxf(mx0, fmaxf(sacc[nt][0], sacc[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(sacc[nt][2], sacc[nt][3]));
      }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < AUDIO_TCATT_MAXW / 8; ++nt) {
      if (nt < ntiles) {
        sacc[nt][0] = expf(__fsub_rn(sacc[nt][0], mx0));
        sacc[nt][1] = expf(__fsub_rn(sacc[nt][1], mx0));
        sacc[nt][2] = expf(__fsub_rn(sacc[nt][2], mx1));
        sacc[nt][3] = expf(__fsub_rn(sacc[nt][3], mx1));
        sum0 = __fadd_rn(__fadd_rn(sum0, sacc[nt][0]), sacc[nt][1]);
        sum1 = __fadd_rn(__fadd_rn(sum1, sacc[nt][2]), sacc[nt][3]);
      }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      sum0 = __fadd_rn(sum0, __shfl_xor_sync(0xffffffffu, sum0, o));
      sum1 = __fadd_rn(sum1, __shfl_xor_sync(0xffffffffu, sum1, o));
    }
    const float inv0 = __fdiv_rn(1.0f, sum0), inv1 = __fdiv_rn(1.0f, sum1);
#pragma unroll
    for (int nt = 0; nt < AUDIO_TCATT_MAXW / 8; ++nt) {
      if (nt < ntiles) {
        float* p0 = sp + g * ps + nt * 8 + 2 * t;
        p0[0] = __fmul_rn(sacc[nt][0], inv0);
        p0[1] = __fmul_rn(sacc[nt][1], inv0);
        p0[8 * ps] = __fmul_rn(sacc[nt][2], inv1);
        p0[8 * ps + 1] = __fmul_rn(sacc[nt][3], inv1);
      }
    }
    __syncwarp();
    float oacc[HD / 8][4];
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) oacc[nd][0] = oacc[nd][1] = oacc[nd][2] = oacc[nd][3] = 0.f;
    for (int kk = 0; kk < ntiles; ++kk) {
      const float* pa = sp + g * ps + kk * 8;
      const uint32_t a0 = to_tf32(pa[t]), a1 = to_tf32(pa[8 * ps + t]);
      const uint32_t a2 = to_tf32(pa[t + 4]), a3 = to_tf32(pa[8 * ps + t + 4]);
      const float* vb = sv + (kk * 8 + t) * VS + g;
#pragma unroll
      for (int nd = 0; nd < HD / 8; ++nd)
        mma_tf32(oacc[nd], a0, a1, a2, a3, to_tf32(vb[nd * 8]), to_tf32(vb[4 * VS + nd * 8]));
    }
    const int r0 = q0 + mt * 16 + g;
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) {
      const int col = h * HD + nd * 8 + 2 * t;
      if (r0 < len)
        *reinterpret_cast<__half2*>(out + static_cast<size_t>(start + r0) * dm + col) =
            __floats2half2_rn(oacc[nd][0], oacc[nd][1]);
      if (r0 + 8 < len)
        *reinterpret_cast<__half2*>(out + static_cast<size_t>(start + r0 + 8) * dm + col) =
            __floats2half2_rn(oacc[nd][2], oacc[nd][3]);
    }
  }
}

}  // namespace qasr
