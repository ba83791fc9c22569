// Host runtime of the B200 audio tower: the C ABI of include/qasr_b200_audio.h.
//
// One context = one device, one stream, one copy of the tower's weights and a set of
// activation buffers grown to the largest request seen.  An encode is one stream of
// launches (no host round trip inside): per round of up to AUDIO_ROUND_CHUNKS conv chunks
// conv2d1 (CUDA cores) -> im2col -> conv2d2 GEMM -> im2col -> conv2d3 GEMM -> token packing;
// then conv_out over all tokens, the transformer layers, ln_post and the projector.  GEMM
// epilogues only store (bias, GELU); each residual add is fused into the LayerNorm kernel
// that follows it (h += delta, then normalise), so no GEMM reads the residual stream.  The
// GEMMs are gemm_tc_kernel (tcgen05, weights as UMMA M, stream-K over (tile, k-block)
// units) launched as programmatic dependents so each streams its weights while the
// previous kernel drains.
//
// Reference: GpuAudioEncoder (src/audio_encoder_gpu.rs:599-1301) for the structure and the
// geometry checks, CpuAudioEncoder (src/audio_encoder.rs:669-770) for the arithmetic.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <string>
#include <vector>

#include "abi_guard.h"
#include "audio_kernels.cuh"
#include "f16_host.h"
#include "gemm_tc.cuh"
#include "host_gemm.cuh"
#include "qasr_b200.h"
#include "qasr_b200_audio.h"

namespace {

using namespace qasr;

constexpr int AUDIO_ROUND_CHUNKS = 32;  // conv chunks per round (bounds the im2col buffers)
constexpr float AUDIO_LN_EPS = 1e-5f;   // CpuAudioLayerNorm eps (src/audio_encoder.rs:603-606)

int feo(int l) {  // src/audio_encoder.rs:634-637
  auto f = [](int x) { return (x - 1) / 2 + 1; };
  return f(f(f(l)));
}
int conv_len(int l) { return (l + 2 - 3) / 2 + 1; }  // src/audio_encoder_gpu.rs:2252-2254
int round_up(int x, int m) { return (x + m - 1) / m * m; }

struct ALin {
  void* w = nullptr;      // tiled f16 [n_out][k] (weight_tile_offset layout)
  float* bias = nullptr;  // f32 [n_out] or null
  int n_out = 0, k = 0;
};

struct ALayer {
  ALin qkv, o, fc1, fc2;
  float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
};

struct Buf {
  void* p = nullptr;
  size_t bytes = 0;
};

}  // namespace

struct qasr_audio_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  qasr_audio_config cfg{};
  std::string err;
  // geometry (GpuAudioEncoder::load, src/audio_encoder_gpu.rs:606-700)
  int cs = 0, tpc = 0, h1 = 0, w1 = 0, h2 = 0, w2 = 0, h3 = 0, w3 = 0;
  int C = 0, ldc = 0, kconv = 0, cf = 0, dm = 0, hd = 0, nh = 0, ffn = 0, out_dim = 0, wlen = 0;
  bool attn_kv_smem = false;
  size_t attn_smem = 0;
  bool attn_tc = false;  // tensor-core attention (windows <= 128 tokens, head dim 64 or 128)
  size_t attn_tc_smem = 0;
  // weights
  std::vector<void*> wallocs;
  float *c1_w = nullptr, *c1_b = nullptr, *pe = nullptr;
  ALin c2, c3, co, p1, p2;
  std::vector<ALayer> layers;
  float *lnp_w = nullptr, *lnp_b = nullptr;
  bool loaded = false;
  // activations (grown on demand)
  Buf mel, chunks, win, act1, x2, act2, x3, act3, packed, h32, delta, xn, qkv32, attn16, ffn16, p116, out16, ws, cnt;
  uint32_t* status = nullptr;
  // host copies of the launch tables (they outlive an asynchronous encode's copies)
  std::vector<AudioChunk> h_chunks;
  std::vector<int> h_win;
  uint64_t launches = 0;
};

namespace {

qasr_status afail(qasr_audio_ctx* c, qasr_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return s;
}

qasr_status acuda(qasr_audio_ctx* c, cudaError_t e, const char* what) {
  return afail(c, e == cudaErrorMemoryAllocation ? QASR_ERR_OOM : QASR_ERR_DEVICE, "%s: %s", what,
               cudaGetErrorString(e));
}

#define ACK(call, what)                                \
  do {                                                 \
    cudaError_t _e = (call);                           \
    if (_e != cudaSuccess) return acuda(c, _e, what);  \
  } while (0)

qasr_status walloc(qasr_audio_ctx* c, void** p, size_t bytes, const char* what) {
  ACK(cudaMalloc(p, std::max<size_t>(bytes, 256)), what);
  c->wallocs.push_back(*p);
  return QASR_OK;
}

// Grow an activation buffer (the stream is drained first: an earlier launch may still read it).
qasr_status grow(qasr_audio_ctx* c, Buf& b, size_t bytes, const char* what, bool zero = false) {
  if (bytes <= b.bytes) return QASR_OK;
  ACK(cudaStreamSynchronize(c->stream), "stream sync");
  if (b.p) cudaFree(b.p);
  b.p = nullptr;
  b.bytes = 0;
  ACK(cudaMalloc(&b.p, bytes), what);
  if (zero) ACK(cudaMemsetAsync(b.p, 0, bytes, c->stream), what);
  b.bytes = bytes;
  return QASR_OK;
}

template <class T>
T* P(const Buf& b) {
  return static_cast<T*>(b.p);
}

template <class T>
qasr_status upload(qasr_audio_ctx* c, T** dst, const T* src, size_t n, const char* what) {
  void* p = nullptr;
  qasr_status s = walloc(c, &p, n * sizeof(T), what);
  if (s) return s;
  ACK(cudaMemcpy(p, src, n * sizeof(T), cudaMemcpyHostToDevice), what);
  *dst = static_cast<T*>(p);
  return QASR_OK;
}

// f16 row-major [n_out][k] (host) -> the tiled layout gemm_tc_kernel streams.
qasr_status upload_linear(qasr_audio_ctx* c, ALin* L, const uint16_t* w, int n_out, int k, const float* bias,
                          const char* what) {
  if (n_out % 128 != 0 || k % 64 != 0)
    return afail(c, QASR_ERR_INVALID_ARG, "%s: [%d x %d] is not a multiple of 128 x 64", what, n_out, k);
  const size_t bytes = static_cast<size_t>(n_out) * k * 2;
  void* staging = nullptr;
  ACK(cudaMalloc(&staging, bytes), what);
  cudaError_t e = cudaMemcpy(staging, w, bytes, cudaMemcpyHostToDevice);
  qasr_status s = QASR_OK;
  if (e == cudaSuccess) s = walloc(c, &L->w, bytes, what);
  if (e == cudaSuccess && s == QASR_OK) {
    pack_weight_tiles_kernel<<<1024, 256, 0, c->stream>>>(static_cast<const uint4*>(staging),
                                                           static_cast<uint4*>(L->w), n_out, k * 2);
    c->launches++;
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  }
  cudaFree(staging);
  if (e != cudaSuccess) return acuda(c, e, what);
  if (s) return s;
  L->n_out = n_out;
  L->k = k;
  L->bias = nullptr;
  if (bias) return upload(c, &L->bias, bias, static_cast<size_t>(n_out), what);
  return QASR_OK;
}

bool check_config(const qasr_audio_config& g, std::string* why) {
  char b[256];
  auto bad = [&](const char* m) {
    *why = m;
    return false;
  };
  if (g.d_model <= 0 || g.encoder_layers < 0 || g.encoder_attention_heads <= 0 || g.encoder_ffn_dim <= 0 ||
      g.num_mel_bins <= 0 || g.downsample_hidden_size <= 0 || g.max_source_positions <= 0 || g.n_window <= 0 ||
      g.n_window_infer <= 0 || g.output_dim <= 0)
    return bad("audio config: every field must be positive (encoder_layers may be 0)");
  if (g.d_model % g.encoder_attention_heads != 0) {
    snprintf(b, sizeof b, "d_model %d not divisible by %d heads", g.d_model, g.encoder_attention_heads);
    return bad(b);
  }
  const int hd = g.d_model / g.encoder_attention_heads;
  if (hd % 32 != 0 || hd > AUDIO_ATTN_MAX_HD) {
    snprintf(b, sizeof b, "head dim %d: this tower supports multiples of 32 up to %d", hd, AUDIO_ATTN_MAX_HD);
    return bad(b);
  }
  if (g.d_model % 128 || g.encoder_ffn_dim % 128 || g.output_dim % 128) {
    snprintf(b, sizeof b, "d_model %d, ffn %d and output_dim %d must be multiples of 128", g.d_model,
             g.encoder_ffn_dim, g.output_dim);
    return bad(b);
  }
  if (g.d_model > 128 * AUDIO_LN_MAXV) {
    snprintf(b, sizeof b, "d_model %d: this tower's LayerNorm holds rows of at most %d", g.d_model,
             128 * AUDIO_LN_MAXV);
    return bad(b);
  }
  if (g.downsample_hidden_size % 8 || g.downsample_hidden_size > 2048)
    return bad("downsample_hidden_size must be a multiple of 8, at most 2048");
  const int h3 = conv_len(conv_len(conv_len(g.num_mel_bins)));
  if ((g.downsample_hidden_size * h3) % 64) {
    snprintf(b, sizeof b, "conv_out width %d x %d is not a multiple of 64", g.downsample_hidden_size, h3);
    return bad(b);
  }
  if (g.max_source_positions < feo(2 * g.n_window)) return bad("max_source_positions below tokens per chunk");
  {  // the conv kernels index a round with 32-bit arithmetic
    const long long C = g.downsample_hidden_size, w1 = conv_len(2 * g.n_window), h1 = conv_len(g.num_mel_bins);
    const long long kv = (9 * C + 63) / 64 * 64 / 8;
    if (AUDIO_ROUND_CHUNKS * h1 * w1 * std::max(C / 8, kv) >= (1LL << 31)) return bad("conv chunk too large");
  }
  return true;
}

qasr_status check_device_status(qasr_audio_ctx* c) {
  uint32_t st[2] = {0, 0};
  ACK(cudaMemcpyAsync(st, c->status, sizeof st, cudaMemcpyDeviceToHost, c->stream), "status read");
  ACK(cudaStreamSynchronize(c->stream), "stream sync");
  if (st[0] != 0) {
    const uint32_t zero[2] = {0, 0};
    cudaMemcpy(c->status, zero, sizeof zero, cudaMemcpyHostToDevice);
    if (st[0] == DEVERR_TIMEOUT)
      return afail(c, QASR_ERR_DEVICE_TIMEOUT, "a device-side wait timed out (site 0x%x)", st[1]);
    return afail(c, QASR_ERR_DEVICE, "device-side check failed (code %u, site 0x%x)", st[0], st[1]);
  }
  return QASR_OK;
}

template <int EPI>
cudaError_t set_gemm_attr() {
  return cudaFuncSetAttribute(gemm_tc_kernel<false, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              g_dyn_smem_max);
}

// Plan of an audio GEMM: CTA count and activation-tile width.  With fewer tiles than SMs,
// each tile is cut into s k-segments (grid = tiles * s): s = 1 needs no split fixup, a
// larger s streams fewer units per CTA but adds the last CTA's pass over s partials.
// Measured per CTA (B200, f16, 128-row tiles): ~4 us of set-up and first loads, ~0.6 us per
// (16 KB W + 16 KB X) unit (the SM's load rate; a unit of narrower tiles costs in
// proportion to its bytes), ~2.5 us per partial of a split tile (in proportion to its
// size).  64-row tiles double the tile count of a GEMM over a few hundred rows.  With at
// least as many tiles as SMs the default stream-K split applies.  The cheapest plan wins.
struct AudioPlan {
  int grid = 0;    // 0: the default stream-K grid
  int n_tile = 0;  // 0: the default width
};

AudioPlan audio_plan(int n_out, int k, int rows, int sms) {
  static const bool narrow_ok = !(std::getenv("QASR_B200_AUDIO_NT64") && std::getenv("QASR_B200_AUDIO_NT64")[0] == '0');
  AudioPlan best;
  double best_t = 1e30;
  for (int nt : {0, 64}) {
    if (nt == 64 && (!narrow_ok || rows <= 64)) continue;
    const GemmShape d = gemm_shape(n_out, k, false, rows, sms, 0, true, nt);
    if (nt == 64 && d.n_tile != 64) continue;
    const double unit = 0.6 * (16384.0 + 128.0 * d.n_tile) / 32768.0;
    const double part = 2.5 * d.n_tile / 128.0;
    if (d.tiles >= sms) {
      const double t = 4.0 + unit * std::ceil(static_cast<double>(d.units) / sms) + part;
      if (t < best_t) {
        best_t = t;
        best = AudioPlan{0, nt};
      }
      continue;
    }
    for (int sp = 1; sp <= 8 && d.tiles * sp <= sms; ++sp) {
      const double t = 4.0 + unit * static_cast<double>(d.kblocks) / sp + (sp > 1 ? part * sp : 0.0);
      if (t < best_t) {
        best_t = t;
        best = AudioPlan{d.tiles * sp, nt};
      }
    }
  }
  return best;
}

// One GEMM: out = epilogue(X [rows, L.k] . W^T + bias).  The split workspace must already
// hold the plan (reserve_gemm).
qasr_status gemm(qasr_audio_ctx* c, const ALin& L, const __half* X, int rows, int epi, __half* out16, int ldo,
                 float* out32, int ldo32) {
  const AudioPlan pl = audio_plan(L.n_out, L.k, rows, c->num_sms);
  const GemmShape s = gemm_shape(L.n_out, L.k, false, rows, c->num_sms, pl.grid, true, pl.n_tile);
  if (2ull * static_cast<unsigned long long>(s.units) * static_cast<unsigned long long>(s.grid) >= (1ull << 32))
    return afail(c, QASR_ERR_CAPACITY, "GEMM %d x %d over %d rows: too many units", L.n_out, L.k, rows);
  if (s.ws_floats * sizeof(float) > c->ws.bytes || static_cast<size_t>(s.tiles) * sizeof(int) > c->cnt.bytes)
    return afail(c, QASR_ERR_CAPACITY, "GEMM workspace not reserved for %d x %d over %d rows", L.n_out, L.k,
                 rows);
  CUtensorMap tmx{};
  if (!make_tmap(&tmx, X, false, static_cast<uint64_t>(L.k), static_cast<uint64_t>(rows),
                 static_cast<uint64_t>(L.k) * 2, 64, static_cast<uint32_t>(s.n_tile), &c->err))
    return QASR_ERR_DEVICE;
  GemmArgs a{};
  a.n_out = L.n_out;
  a.k = L.k;
  a.rows = rows;
  a.n_tile = s.n_tile;
  a.n_tiles = s.n_tiles;
  a.kblocks = s.kblocks;
  a.units = s.units;
  a.grid = s.grid;
  a.stages = s.stages;
  a.max_seg = s.max_seg;
  a.w_tiles = static_cast<const uint8_t*>(L.w);
  a.epi = epi;
  a.out = out16;
  a.ldo = ldo;
  a.bias = L.bias;
  a.out32 = out32;
  a.ldo32 = ldo32;
  a.ws = P<float>(c->ws);
  a.counters = P<int>(c->cnt);
  a.status = c->status;
  cudaError_t e = cudaErrorInvalidValue;
  const dim3 grid(s.grid), block(gemm_threads(false));
  switch (epi) {
    case EPI_BIAS_F16:
      e = launch_k(gemm_tc_kernel<false, EPI_BIAS_F16>, grid, block, s.smem, c->stream, true, tmx, a);
      break;
    case EPI_BIAS_GELU:
      e = launch_k(gemm_tc_kernel<false, EPI_BIAS_GELU>, grid, block, s.smem, c->stream, true, tmx, a);
      break;
    case EPI_BIAS_F32:
      e = launch_k(gemm_tc_kernel<false, EPI_BIAS_F32>, grid, block, s.smem, c->stream, true, tmx, a);
      break;
    default:
      break;
  }
  c->launches++;
  ACK(e, "audio GEMM launch");
  return QASR_OK;
}

// Split workspace and tile counters for every GEMM of an encode of `tokens` rows whose
// conv rounds have `round_rows2` / `round_rows3` positions (and the last round's).
qasr_status reserve_gemm(qasr_audio_ctx* c, const std::vector<std::pair<const ALin*, int>>& plan) {
  size_t wsf = 64, tiles = 1;
  for (auto& pr : plan) {
    const AudioPlan pl = audio_plan(pr.first->n_out, pr.first->k, pr.second, c->num_sms);
    const GemmShape s =
        gemm_shape(pr.first->n_out, pr.first->k, false, pr.second, c->num_sms, pl.grid, true, pl.n_tile);
    wsf = std::max(wsf, s.ws_floats);
    tiles = std::max(tiles, static_cast<size_t>(s.tiles));
  }
  qasr_status s = grow(c, c->ws, wsf * sizeof(float), "GEMM workspace");
  if (s) return s;
  return grow(c, c->cnt, tiles * sizeof(int), "GEMM tile counters", true);
}

struct Utt {
  const float* mel;  // the caller's (host or device) mel
  int n_frames;
  const float* mel_dev;  // the same mel on the device
  int tok0, ntok;
};

// The whole tower over `utts` (each mel already on the device at `mel_dev`) into
// out [tokens][out_dim] f16 on the device, the utterances' rows back to back.  Enqueue only.
qasr_status run_tower(qasr_audio_ctx* c, std::vector<Utt>& utts, __half* out) {
  const qasr_audio_config& g = c->cfg;
  c->h_chunks.clear();
  c->h_win.clear();
  int tokens = 0;
  for (Utt& u : utts) {
    const int nfull = u.n_frames / c->cs, tail = u.n_frames % c->cs;
    const int n_chunks = nfull + (tail > 0 ? 1 : 0);
    u.tok0 = tokens;
    for (int i = 0; i < n_chunks; ++i) {
      AudioChunk k{};
      k.mel = u.mel_dev;
      k.n_frames = u.n_frames;
      k.frame0 = i * c->cs;
      k.valid = i < nfull ? c->cs : tail;
      k.ntok = i < nfull ? c->tpc : feo(tail);
      k.tok0 = tokens;
      tokens += k.ntok;
      c->h_chunks.push_back(k);
    }
    u.ntok = tokens - u.tok0;
    for (int st = 0; st < u.ntok; st += c->wlen) {  // windows never cross an utterance
      c->h_win.push_back(u.tok0 + st);
      c->h_win.push_back(std::min(c->wlen, u.ntok - st));
    }
  }
  const int n_chunks = static_cast<int>(c->h_chunks.size());
  const int n_win = static_cast<int>(c->h_win.size() / 2);
  const int R = std::min(AUDIO_ROUND_CHUNKS, n_chunks);
  const int dm = c->dm, T = tokens;
  const size_t p1 = static_cast<size_t>(c->h1) * c->w1, p2 = static_cast<size_t>(c->h2) * c->w2,
               p3 = static_cast<size_t>(c->h3) * c->w3;
  qasr_status s;
  if ((s = grow(c, c->chunks, sizeof(AudioChunk) * n_chunks, "chunk table")) ||
      (s = grow(c, c->win, sizeof(int) * 2 * n_win, "window table")) ||
      (s = grow(c, c->act1, 2 * R * p1 * c->ldc, "conv1 activations")) ||
      (s = grow(c, c->x2, 2 * R * p2 * c->kconv, "conv2 operand")) ||
      (s = grow(c, c->act2, 2 * R * p2 * c->ldc, "conv2 activations")) ||
      (s = grow(c, c->x3, 2 * R * p3 * c->kconv, "conv3 operand")) ||
      (s = grow(c, c->act3, 2 * R * p3 * c->ldc, "conv3 activations")) ||
      (s = grow(c, c->packed, 2ull * T * c->cf, "conv_out operand")) ||
      (s = grow(c, c->h32, 4ull * T * dm, "residual stream")) ||
      (s = grow(c, c->delta, 4ull * T * dm, "block outputs")) ||
      (s = grow(c, c->xn, 2ull * T * dm, "normed rows")) ||
      (s = grow(c, c->qkv32, 4ull * T * 3 * dm, "q|k|v")) ||
      (s = grow(c, c->attn16, 2ull * T * dm, "attention rows")) ||
      (s = grow(c, c->ffn16, 2ull * T * c->ffn, "fc1 rows")) ||
      (s = grow(c, c->p116, 2ull * T * dm, "proj1 rows")))
    return s;
  std::vector<std::pair<const ALin*, int>> plan;
  for (int r0 = 0; r0 < n_chunks; r0 += R) {
    const int n = std::min(R, n_chunks - r0);
    plan.push_back({&c->c2, static_cast<int>(n * p2)});
    plan.push_back({&c->c3, static_cast<int>(n * p3)});
  }
  plan.push_back({&c->co, T});
  if (!c->layers.empty()) {
    const ALayer& L = c->layers[0];
    for (const ALin* l : {&L.qkv, &L.o, &L.fc1, &L.fc2}) plan.push_back({l, T});
  }
  plan.push_back({&c->p1, T});
  plan.push_back({&c->p2, T});
  if ((s = reserve_gemm(c, plan))) return s;
  ACK(cudaMemcpyAsync(c->chunks.p, c->h_chunks.data(), sizeof(AudioChunk) * n_chunks, cudaMemcpyHostToDevice,
                      c->stream),
      "chunk table upload");
  ACK(cudaMemcpyAsync(c->win.p, c->h_win.data(), sizeof(int) * 2 * n_win, cudaMemcpyHostToDevice, c->stream),
      "window table upload");

  const int sms = c->num_sms;
  auto grid_for = [&](long long work) {
    return static_cast<int>(std::min<long long>(std::max<long long>(1, (work + 255) / 256), 16LL * sms));
  };
  // ---- conv stem, one round of chunks at a time (CpuConvStem::forward_stages, :267-336)
  for (int r0 = 0; r0 < n_chunks; r0 += R) {
    const int n = std::min(R, n_chunks - r0);
    const AudioChunk* ch = P<AudioChunk>(c->chunks) + r0;
    const int c1_block = audio_conv1_block(c->C / 8);
    const long long c1_items = static_cast<long long>(n) * c->h1 * ((c->w1 + AUDIO_C1_POS - 1) / AUDIO_C1_POS);
    ACK(launch_k(audio_conv1_kernel,
                 dim3(static_cast<unsigned>(std::min<long long>(
                     std::max<long long>(1, c1_items / (c1_block / (c->C / 8)) + 1), 8LL * sms))),
                 dim3(c1_block), 0, c->stream, true, ch, n, g.num_mel_bins, c->h1, c->w1,
                 static_cast<const float*>(c->c1_w), static_cast<const float*>(c->c1_b), c->C, P<__half>(c->act1),
                 c->ldc),
        "conv1 launch");
    ACK(launch_k(audio_im2col_kernel, dim3(grid_for(static_cast<long long>(n) * p2 * (c->kconv / 8))), dim3(256), 0,
                 c->stream, true, static_cast<const __half*>(P<__half>(c->act1)), n, c->h1, c->w1, c->C, c->ldc,
                 c->h2, c->w2, P<__half>(c->x2), c->kconv),
        "im2col launch");
    c->launches += 2;
    if ((s = gemm(c, c->c2, P<__half>(c->x2), static_cast<int>(n * p2), EPI_BIAS_GELU, P<__half>(c->act2), c->ldc,
                  nullptr, 0)))
      return s;
    ACK(launch_k(audio_im2col_kernel, dim3(grid_for(static_cast<long long>(n) * p3 * (c->kconv / 8))), dim3(256), 0,
                 c->stream, true, static_cast<const __half*>(P<__half>(c->act2)), n, c->h2, c->w2, c->C, c->ldc,
                 c->h3, c->w3, P<__half>(c->x3), c->kconv),
        "im2col launch");
    c->launches++;
    if ((s = gemm(c, c->c3, P<__half>(c->x3), static_cast<int>(n * p3), EPI_BIAS_GELU, P<__half>(c->act3), c->ldc,
                  nullptr, 0)))
      return s;
    ACK(launch_k(audio_pack_kernel, dim3(std::max(1, (c->tpc * std::max(c->C, dm) + 255) / 256), n), dim3(256), 0,
                 c->stream, true, static_cast<const __half*>(P<__half>(c->act3)), ch, n, c->h3, c->w3, c->C, c->ldc,
                 P<__half>(c->packed), P<float>(c->h32), static_cast<const float*>(c->pe), dm),
        "pack launch");
    c->launches++;
  }
  // conv_out: delta = packed . W^T + b; the first residual add makes h = pe + delta
  if ((s = gemm(c, c->co, P<__half>(c->packed), T, EPI_BIAS_F32, nullptr, 0, P<float>(c->delta), dm))) return s;

  // ---- transformer layers (CpuAudioLayer::forward, src/audio_encoder.rs:614-630)
  const int ln_grid = (T * 32 + 255) / 256;
  const float scale = 1.0f / std::sqrt(static_cast<float>(c->hd));
  const int qblocks = (c->wlen + AUDIO_ATTN_QB - 1) / AUDIO_ATTN_QB;
  for (const ALayer& L : c->layers) {
    ACK(launch_k(audio_residual_layernorm_kernel, dim3(ln_grid), dim3(256), 0, c->stream, true, P<float>(c->h32),
                 static_cast<const float*>(P<float>(c->delta)), T, dm, static_cast<const float*>(L.ln1_w),
                 static_cast<const float*>(L.ln1_b), AUDIO_LN_EPS, P<__half>(c->xn)),
        "layernorm launch");
    c->launches++;
    if ((s = gemm(c, L.qkv, P<__half>(c->xn), T, EPI_BIAS_F32, nullptr, 0, P<float>(c->qkv32), 3 * dm))) return s;
    if (c->attn_tc)
      ACK(launch_k(c->hd == 64 ? audio_window_attention_tc_kernel<64> : audio_window_attention_tc_kernel<128>,
                   dim3(n_win, c->nh, (c->wlen + AUDIO_TCATT_QROWS - 1) / AUDIO_TCATT_QROWS),
                   dim3(AUDIO_TCATT_WARPS * 32), c->attn_tc_smem, c->stream, true,
                   static_cast<const float*>(P<float>(c->qkv32)), static_cast<const int*>(P<int>(c->win)), dm, scale,
                   c->wlen, P<__half>(c->attn16)),
          "window attention launch");
    else
      ACK(launch_k(c->attn_kv_smem ? audio_window_attention_kernel<true> : audio_window_attention_kernel<false>,
                   dim3(n_win, c->nh, qblocks), dim3(AUDIO_ATTN_THREADS), c->attn_smem, c->stream, true,
                   static_cast<const float*>(P<float>(c->qkv32)), static_cast<const int*>(P<int>(c->win)), dm,
                   c->hd, scale, c->wlen, P<__half>(c->attn16)),
          "window attention launch");
    c->launches++;
    if ((s = gemm(c, L.o, P<__half>(c->attn16), T, EPI_BIAS_F32, nullptr, 0, P<float>(c->delta), dm))) return s;
    ACK(launch_k(audio_residual_layernorm_kernel, dim3(ln_grid), dim3(256), 0, c->stream, true, P<float>(c->h32),
                 static_cast<const float*>(P<float>(c->delta)), T, dm, static_cast<const float*>(L.ln2_w),
                 static_cast<const float*>(L.ln2_b), AUDIO_LN_EPS, P<__half>(c->xn)),
        "layernorm launch");
    c->launches++;
    if ((s = gemm(c, L.fc1, P<__half>(c->xn), T, EPI_BIAS_GELU, P<__half>(c->ffn16), c->ffn, nullptr, 0))) return s;
    if ((s = gemm(c, L.fc2, P<__half>(c->ffn16), T, EPI_BIAS_F32, nullptr, 0, P<float>(c->delta), dm))) return s;
  }
  // ---- ln_post, proj1 + GELU, proj2 (src/audio_encoder.rs:750-755)
  ACK(launch_k(audio_residual_layernorm_kernel, dim3(ln_grid), dim3(256), 0, c->stream, true, P<float>(c->h32),
               static_cast<const float*>(P<float>(c->delta)), T, dm, static_cast<const float*>(c->lnp_w),
               static_cast<const float*>(c->lnp_b), AUDIO_LN_EPS, P<__half>(c->xn)),
      "layernorm launch");
  c->launches++;
  if ((s = gemm(c, c->p1, P<__half>(c->xn), T, EPI_BIAS_GELU, P<__half>(c->p116), dm, nullptr, 0))) return s;
  return gemm(c, c->p2, P<__half>(c->p116), T, EPI_BIAS_F16, out, c->out_dim, nullptr, 0);
}

qasr_status begin(qasr_audio_ctx* c) {
  if (!c->loaded) return afail(c, QASR_ERR_STATE, "audio tower weights not loaded");
  ACK(cudaSetDevice(c->device), "cudaSetDevice");
  return QASR_OK;
}

}  // namespace

extern "C" {

int32_t qasr_audio_token_count(const qasr_audio_config* cfg, int32_t n_frames) {
  if (!cfg || cfg->n_window <= 0 || n_frames <= 0) return 0;
  const int cs = 2 * cfg->n_window;
  const int nfull = n_frames / cs, tail = n_frames % cs;
  return nfull * feo(cs) + (tail > 0 ? feo(tail) : 0);
}

qasr_status qasr_audio_create(const qasr_audio_config* cfg, int device, qasr_audio_ctx** out, char* err,
                              int errlen) {
  auto fail_out = [&](qasr_status s, const std::string& m) {
    if (err && errlen > 0) snprintf(err, static_cast<size_t>(errlen), "%s", m.c_str());
    return s;
  };
  if (!cfg || !out) return fail_out(QASR_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  std::string why;
  if (!check_config(*cfg, &why)) return fail_out(QASR_ERR_INVALID_ARG, why);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail_out(QASR_ERR_DEVICE, "no CUDA device " + std::to_string(device));
  if (cudaSetDevice(device) != cudaSuccess) return fail_out(QASR_ERR_DEVICE, "cudaSetDevice failed");
  cudaDeviceProp prop{};
  cudaGetDeviceProperties(&prop, device);
  if (prop.major != 10) return fail_out(QASR_ERR_DEVICE, "the audio tower is built for sm_100a (B200)");
  std::string e;
  if (init_kernel_attrs(&e) != cudaSuccess) return fail_out(QASR_ERR_DEVICE, e);
  cudaError_t ce = set_gemm_attr<EPI_BIAS_F16>();
  if (ce == cudaSuccess) ce = set_gemm_attr<EPI_BIAS_GELU>();
  if (ce == cudaSuccess) ce = set_gemm_attr<EPI_BIAS_F32>();
  if (ce != cudaSuccess) return fail_out(QASR_ERR_DEVICE, std::string("GEMM attributes: ") + cudaGetErrorString(ce));

  auto* c = new qasr_audio_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  c->cfg = *cfg;
  const qasr_audio_config& g = *cfg;
  c->cs = 2 * g.n_window;
  c->tpc = feo(c->cs);
  c->h1 = conv_len(g.num_mel_bins);
  c->w1 = conv_len(c->cs);
  c->h2 = conv_len(c->h1);
  c->w2 = conv_len(c->w1);
  c->h3 = conv_len(c->h2);
  c->w3 = conv_len(c->w2);
  c->C = g.downsample_hidden_size;
  c->ldc = round_up(c->C, 128);
  c->kconv = round_up(9 * c->C, 64);
  c->cf = c->C * c->h3;
  c->dm = g.d_model;
  c->nh = g.encoder_attention_heads;
  c->hd = g.d_model / g.encoder_attention_heads;
  c->ffn = g.encoder_ffn_dim;
  c->out_dim = g.output_dim;
  // window = tpc * (window_infer / chunk), window_infer = max(n_window_infer, chunk)
  // (src/inference.rs:982, src/audio_encoder_gpu.rs:736)
  c->wlen = c->tpc * (std::max(g.n_window_infer, c->cs) / c->cs);
  const size_t smem_kv = audio_attn_smem_floats(c->wlen, c->hd, true) * sizeof(float);
  c->attn_kv_smem = smem_kv <= 200 * 1024;
  c->attn_smem = audio_attn_smem_floats(c->wlen, c->hd, c->attn_kv_smem) * sizeof(float);
  c->attn_tc_smem = audio_tcatt_smem_floats(c->wlen, c->hd) * sizeof(float);
  c->attn_tc = c->wlen <= AUDIO_TCATT_MAXW && (c->hd == 64 || c->hd == 128) && c->attn_tc_smem <= 200 * 1024 &&
               !(std::getenv("QASR_B200_AUDIO_F32_ATTN") && std::getenv("QASR_B200_AUDIO_F32_ATTN")[0] == '1');
  if (c->attn_smem > 200 * 1024) {
    delete c;
    return fail_out(QASR_ERR_INVALID_ARG, "attention window of " + std::to_string(g.n_window_infer) +
                                              " frames is too long for this tower");
  }
  if (c->w3 != c->tpc) {  // GpuAudioEncoder::load's conv chain check (src/audio_encoder_gpu.rs:665)
    delete c;
    return fail_out(QASR_ERR_INVALID_ARG, "conv chain: t3 != tokens per chunk");
  }
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaFuncSetAttribute(audio_window_attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(c->attn_smem)) != cudaSuccess ||
      cudaFuncSetAttribute(audio_window_attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(c->attn_smem)) != cudaSuccess ||
      (c->attn_tc && cudaFuncSetAttribute(c->hd == 64 ? audio_window_attention_tc_kernel<64>
                                                      : audio_window_attention_tc_kernel<128>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(c->attn_tc_smem)) != cudaSuccess) ||
      cudaMalloc(&c->status, 2 * sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(c->status, 0, 2 * sizeof(uint32_t)) != cudaSuccess) {
    qasr_audio_destroy(c);
    return fail_out(QASR_ERR_DEVICE, "audio tower stream / status setup failed");
  }
  *out = c;
  return QASR_OK;
}

void qasr_audio_destroy(qasr_audio_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  for (void* p : c->wallocs) cudaFree(p);
  for (Buf* b : {&c->mel, &c->chunks, &c->win, &c->act1, &c->x2, &c->act2, &c->x3, &c->act3, &c->packed, &c->h32, &c->delta,
                 &c->xn, &c->qkv32, &c->attn16, &c->ffn16, &c->p116, &c->out16, &c->ws, &c->cnt})
    if (b->p) cudaFree(b->p);
  if (c->status) cudaFree(c->status);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

const char* qasr_audio_last_error(const qasr_audio_ctx* c) { return c ? c->err.c_str() : "null context"; }

void* qasr_audio_stream(qasr_audio_ctx* c) { return c ? static_cast<void*>(c->stream) : nullptr; }

uint64_t qasr_audio_launch_count(const qasr_audio_ctx* c) { return c ? c->launches : 0; }

qasr_status qasr_audio_load_weights(qasr_audio_ctx* c, const qasr_audio_weights* w) {
  if (!c || !w) return QASR_ERR_INVALID_ARG;
  const qasr_audio_config& g = c->cfg;
  if (!w->conv1_w || !w->conv1_b || !w->conv2_w || !w->conv2_b || !w->conv3_w || !w->conv3_b || !w->conv_out_w ||
      (g.encoder_layers > 0 && !w->layers) || !w->ln_post_w || !w->ln_post_b || !w->proj1_w || !w->proj2_w)
    return afail(c, QASR_ERR_INVALID_ARG, "audio weights: a required tensor is null");
  for (int l = 0; l < g.encoder_layers; ++l) {
    const qasr_audio_layer_weights& L = w->layers[l];
    if (!L.q_w || !L.k_w || !L.v_w || !L.o_w || !L.ln1_w || !L.ln1_b || !L.ln2_w || !L.ln2_b || !L.fc1_w ||
        !L.fc2_w)
      return afail(c, QASR_ERR_INVALID_ARG, "audio weights: layer %d is missing a tensor", l);
  }
  ACK(cudaSetDevice(c->device), "cudaSetDevice");
  ACK(cudaStreamSynchronize(c->stream), "stream sync");
  for (void* p : c->wallocs) cudaFree(p);
  c->wallocs.clear();
  c->layers.clear();
  c->loaded = false;
  const int C = c->C, dm = c->dm;
  qasr_status s;
  // conv2d1: [C][1][3][3] f16 -> f32 [C][9] (exact); the CUDA-core kernel reads it
  {
    std::vector<float> w1(static_cast<size_t>(C) * 9);
    for (size_t i = 0; i < w1.size(); ++i) w1[i] = f16_bits_to_f32(w->conv1_w[i]);
    if ((s = upload(c, &c->c1_w, w1.data(), w1.size(), "conv2d1 weight")) ||
        (s = upload(c, &c->c1_b, w->conv1_b, static_cast<size_t>(C), "conv2d1 bias")))
      return s;
  }
  // conv2d2 / conv2d3: [C][C][3][3] -> GEMM rows [ldc][kconv] with k = tap * C + c (the
  // im2col operand's order), zero rows beyond C and zero columns beyond 9 C
  auto conv_gemm = [&](ALin* L, const uint16_t* src, const float* bias, const char* what) {
    std::vector<uint16_t> m(static_cast<size_t>(c->ldc) * c->kconv, 0);
    for (int o = 0; o < C; ++o)
      for (int ci = 0; ci < C; ++ci)
        for (int tap = 0; tap < 9; ++tap)
          m[static_cast<size_t>(o) * c->kconv + tap * C + ci] = src[(static_cast<size_t>(o) * C + ci) * 9 + tap];
    std::vector<float> b(static_cast<size_t>(c->ldc), 0.0f);
    std::copy(bias, bias + C, b.begin());
    return upload_linear(c, L, m.data(), c->ldc, c->kconv, b.data(), what);
  };
  if ((s = conv_gemm(&c->c2, w->conv2_w, w->conv2_b, "conv2d2")) ||
      (s = conv_gemm(&c->c3, w->conv3_w, w->conv3_b, "conv2d3")) ||
      (s = upload_linear(c, &c->co, w->conv_out_w, dm, c->cf, w->conv_out_b, "conv_out")))
    return s;
  // sinusoidal positions (CpuConvStem::load, src/audio_encoder.rs:241-250): f64 angles,
  // sin / cos narrowed to f32; the tokens of a chunk use rows 0 .. tpc-1
  {
    const int half = dm / 2;
    const double lt = std::log(10000.0) / (static_cast<double>(half) - 1.0);
    std::vector<float> pe(static_cast<size_t>(c->tpc) * dm);
    for (int p = 0; p < c->tpc; ++p)
      for (int i = 0; i < half; ++i) {
        const double a = static_cast<double>(p) * std::exp(-static_cast<double>(i) * lt);
        pe[static_cast<size_t>(p) * dm + i] = static_cast<float>(std::sin(a));
        pe[static_cast<size_t>(p) * dm + half + i] = static_cast<float>(std::cos(a));
      }
    if ((s = upload(c, &c->pe, pe.data(), pe.size(), "position table"))) return s;
  }
  c->layers.resize(static_cast<size_t>(g.encoder_layers));
  const size_t dd = static_cast<size_t>(dm) * dm;
  for (int l = 0; l < g.encoder_layers; ++l) {
    const qasr_audio_layer_weights& W = w->layers[l];
    ALayer& L = c->layers[static_cast<size_t>(l)];
    // q|k|v fused rows (GpuLinear::load_fused, src/audio_encoder_gpu.rs:256-330)
    std::vector<uint16_t> qkv(3 * dd);
    std::copy(W.q_w, W.q_w + dd, qkv.begin());
    std::copy(W.k_w, W.k_w + dd, qkv.begin() + static_cast<std::ptrdiff_t>(dd));
    std::copy(W.v_w, W.v_w + dd, qkv.begin() + static_cast<std::ptrdiff_t>(2 * dd));
    std::vector<float> qb(static_cast<size_t>(3 * dm), 0.0f);
    const bool any_b = W.q_b || W.k_b || W.v_b;
    if (W.q_b) std::copy(W.q_b, W.q_b + dm, qb.begin());
    if (W.k_b) std::copy(W.k_b, W.k_b + dm, qb.begin() + dm);
    if (W.v_b) std::copy(W.v_b, W.v_b + dm, qb.begin() + 2 * dm);
    if ((s = upload_linear(c, &L.qkv, qkv.data(), 3 * dm, dm, any_b ? qb.data() : nullptr, "q|k|v")) ||
        (s = upload_linear(c, &L.o, W.o_w, dm, dm, W.o_b, "out_proj")) ||
        (s = upload_linear(c, &L.fc1, W.fc1_w, c->ffn, dm, W.fc1_b, "fc1")) ||
        (s = upload_linear(c, &L.fc2, W.fc2_w, dm, c->ffn, W.fc2_b, "fc2")) ||
        (s = upload(c, &L.ln1_w, W.ln1_w, static_cast<size_t>(dm), "self_attn_layer_norm")) ||
        (s = upload(c, &L.ln1_b, W.ln1_b, static_cast<size_t>(dm), "self_attn_layer_norm")) ||
        (s = upload(c, &L.ln2_w, W.ln2_w, static_cast<size_t>(dm), "final_layer_norm")) ||
        (s = upload(c, &L.ln2_b, W.ln2_b, static_cast<size_t>(dm), "final_layer_norm")))
      return s;
  }
  if ((s = upload(c, &c->lnp_w, w->ln_post_w, static_cast<size_t>(dm), "ln_post")) ||
      (s = upload(c, &c->lnp_b, w->ln_post_b, static_cast<size_t>(dm), "ln_post")) ||
      (s = upload_linear(c, &c->p1, w->proj1_w, dm, dm, w->proj1_b, "proj1")) ||
      (s = upload_linear(c, &c->p2, w->proj2_w, c->out_dim, dm, w->proj2_b, "proj2")))
    return s;
  c->loaded = true;
  return QASR_OK;
}

static qasr_status audio_load_checkpoint_body(qasr_audio_ctx* c, qasr_checkpoint* ck, const char* prefix_c) {
  if (!c || !ck) return QASR_ERR_INVALID_ARG;
  const std::string pre = std::string(prefix_c ? prefix_c : "thinker.audio_tower") + ".";
  const qasr_audio_config& g = c->cfg;
  std::deque<std::vector<uint16_t>> h16;
  std::deque<std::vector<float>> h32;
  auto from_ck = [&](qasr_status st) {
    return afail(c, st, "%s", qasr_checkpoint_last_error(ck));
  };
  // f16 matrix (get_f16 narrowing, src/weights.rs:394-417) of `count` elements
  auto m16 = [&](const std::string& name, int64_t count, const uint16_t** out) -> qasr_status {
    h16.emplace_back(static_cast<size_t>(count));
    const qasr_status st = qasr_checkpoint_read_f16(ck, (pre + name).c_str(), h16.back().data(), count);
    if (st) return from_ck(st);
    *out = h16.back().data();
    return QASR_OK;
  };
  // f32 vector (RawTensor::as_f32); optional ones may be absent (CpuAudioLinear's bias)
  auto v32 = [&](const std::string& name, int64_t count, const float** out, bool optional) -> qasr_status {
    *out = nullptr;
    int nd = 0;
    if (optional && qasr_checkpoint_tensor_info(ck, (pre + name).c_str(), nullptr, 0, nullptr, 0, &nd) != QASR_OK)
      return QASR_OK;
    h32.emplace_back(static_cast<size_t>(count));
    const qasr_status st = qasr_checkpoint_read_f32(ck, (pre + name).c_str(), h32.back().data(), count);
    if (st) return from_ck(st);
    *out = h32.back().data();
    return QASR_OK;
  };
  const int64_t C = c->C, d = c->dm, ffn = c->ffn, od = c->out_dim;
  qasr_audio_weights w{};
  std::vector<qasr_audio_layer_weights> lw(static_cast<size_t>(g.encoder_layers));
  qasr_status s;
  if ((s = m16("conv2d1.weight", C * 9, &w.conv1_w)) || (s = v32("conv2d1.bias", C, &w.conv1_b, false)) ||
      (s = m16("conv2d2.weight", C * C * 9, &w.conv2_w)) || (s = v32("conv2d2.bias", C, &w.conv2_b, false)) ||
      (s = m16("conv2d3.weight", C * C * 9, &w.conv3_w)) || (s = v32("conv2d3.bias", C, &w.conv3_b, false)) ||
      (s = m16("conv_out.weight", d * c->cf, &w.conv_out_w)) || (s = v32("conv_out.bias", d, &w.conv_out_b, true)))
    return s;
  for (int l = 0; l < g.encoder_layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    qasr_audio_layer_weights& L = lw[static_cast<size_t>(l)];
    if ((s = m16(p + "self_attn.q_proj.weight", d * d, &L.q_w)) ||
        (s = v32(p + "self_attn.q_proj.bias", d, &L.q_b, true)) ||
        (s = m16(p + "self_attn.k_proj.weight", d * d, &L.k_w)) ||
        (s = v32(p + "self_attn.k_proj.bias", d, &L.k_b, true)) ||
        (s = m16(p + "self_attn.v_proj.weight", d * d, &L.v_w)) ||
        (s = v32(p + "self_attn.v_proj.bias", d, &L.v_b, true)) ||
        (s = m16(p + "self_attn.out_proj.weight", d * d, &L.o_w)) ||
        (s = v32(p + "self_attn.out_proj.bias", d, &L.o_b, true)) ||
        (s = v32(p + "self_attn_layer_norm.weight", d, &L.ln1_w, false)) ||
        (s = v32(p + "self_attn_layer_norm.bias", d, &L.ln1_b, false)) ||
        (s = v32(p + "final_layer_norm.weight", d, &L.ln2_w, false)) ||
        (s = v32(p + "final_layer_norm.bias", d, &L.ln2_b, false)) ||
        (s = m16(p + "fc1.weight", ffn * d, &L.fc1_w)) || (s = v32(p + "fc1.bias", ffn, &L.fc1_b, true)) ||
        (s = m16(p + "fc2.weight", d * ffn, &L.fc2_w)) || (s = v32(p + "fc2.bias", d, &L.fc2_b, true)))
      return s;
  }
  w.layers = lw.data();
  if ((s = v32("ln_post.weight", d, &w.ln_post_w, false)) || (s = v32("ln_post.bias", d, &w.ln_post_b, false)) ||
      (s = m16("proj1.weight", d * d, &w.proj1_w)) || (s = v32("proj1.bias", d, &w.proj1_b, true)) ||
      (s = m16("proj2.weight", od * d, &w.proj2_w)) || (s = v32("proj2.bias", od, &w.proj2_b, true)))
    return s;
  return qasr_audio_load_weights(c, &w);
}

qasr_status qasr_audio_encode_device(qasr_audio_ctx* c, const float* mel_dev, int32_t n_mels, int32_t n_frames,
                                     uint16_t* out_dev, int32_t* n_tokens) {
  if (!c || !mel_dev || !out_dev) return QASR_ERR_INVALID_ARG;
  qasr_status s = begin(c);
  if (s) return s;
  if (n_mels != c->cfg.num_mel_bins)
    return afail(c, QASR_ERR_INVALID_ARG, "mel bins %d != %d", n_mels, c->cfg.num_mel_bins);
  if (n_frames <= 0) return afail(c, QASR_ERR_INVALID_ARG, "empty mel");
  std::vector<Utt> utts{{mel_dev, n_frames, mel_dev, 0, 0}};
  if ((s = run_tower(c, utts, reinterpret_cast<__half*>(out_dev)))) return s;
  if (n_tokens) *n_tokens = utts[0].ntok;
  return QASR_OK;
}

qasr_status qasr_audio_encode_batch_device(qasr_audio_ctx* c, int32_t n, const float* const* mels_dev,
                                           const int32_t* n_frames, int32_t n_mels, uint16_t* out_dev,
                                           int32_t* n_tokens) {
  if (!c || n <= 0 || !mels_dev || !n_frames || !out_dev) return QASR_ERR_INVALID_ARG;
  qasr_status s = begin(c);
  if (s) return s;
  if (n_mels != c->cfg.num_mel_bins)
    return afail(c, QASR_ERR_INVALID_ARG, "mel bins %d != %d", n_mels, c->cfg.num_mel_bins);
  std::vector<Utt> utts(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) {
    if (!mels_dev[i]) return afail(c, QASR_ERR_INVALID_ARG, "utterance %d: null buffer", i);
    if (n_frames[i] <= 0) return afail(c, QASR_ERR_INVALID_ARG, "utterance %d: empty mel", i);
    utts[static_cast<size_t>(i)] = Utt{mels_dev[i], n_frames[i], mels_dev[i], 0, 0};
  }
  if ((s = run_tower(c, utts, reinterpret_cast<__half*>(out_dev)))) return s;
  if (n_tokens)
    for (int i = 0; i < n; ++i) n_tokens[i] = utts[static_cast<size_t>(i)].ntok;
  return QASR_OK;
}

qasr_status qasr_audio_sync(qasr_audio_ctx* c) {
  if (!c) return QASR_ERR_INVALID_ARG;
  ACK(cudaSetDevice(c->device), "cudaSetDevice");
  ACK(cudaStreamSynchronize(c->stream), "stream sync");
  return check_device_status(c);
}

static qasr_status audio_encode_batch_body(qasr_audio_ctx* c, int32_t n, const float* const* mels,
                                          const int32_t* n_frames, int32_t n_mels, uint16_t* const* outs) {
  if (!c || n <= 0 || !mels || !n_frames || !outs) return QASR_ERR_INVALID_ARG;
  qasr_status s = begin(c);
  if (s) return s;
  if (n_mels != c->cfg.num_mel_bins)
    return afail(c, QASR_ERR_INVALID_ARG, "mel bins %d != %d", n_mels, c->cfg.num_mel_bins);
  std::vector<Utt> utts(static_cast<size_t>(n));
  size_t off = 0;
  int tokens = 0;
  for (int i = 0; i < n; ++i) {
    if (!mels[i] || !outs[i]) return afail(c, QASR_ERR_INVALID_ARG, "utterance %d: null buffer", i);
    if (n_frames[i] <= 0) return afail(c, QASR_ERR_INVALID_ARG, "utterance %d: empty mel", i);
    utts[static_cast<size_t>(i)] = Utt{mels[i], n_frames[i], nullptr, 0, 0};
    off += static_cast<size_t>(n_mels) * n_frames[i];
    tokens += qasr_audio_token_count(&c->cfg, n_frames[i]);
  }
  if ((s = grow(c, c->mel, off * sizeof(float), "mel input")) ||
      (s = grow(c, c->out16, 2ull * tokens * c->out_dim, "embeddings")))
    return s;
  off = 0;
  for (Utt& u : utts) {
    u.mel_dev = P<float>(c->mel) + off;
    ACK(cudaMemcpyAsync(P<float>(c->mel) + off, u.mel, sizeof(float) * n_mels * u.n_frames, cudaMemcpyHostToDevice,
                        c->stream),
        "mel upload");
    off += static_cast<size_t>(n_mels) * u.n_frames;
  }
  if ((s = run_tower(c, utts, P<__half>(c->out16)))) return s;
  for (int i = 0; i < n; ++i) {
    const Utt& u = utts[static_cast<size_t>(i)];
    ACK(cudaMemcpyAsync(outs[i], P<uint16_t>(c->out16) + static_cast<size_t>(u.tok0) * c->out_dim,
                        2ull * u.ntok * c->out_dim, cudaMemcpyDeviceToHost, c->stream),
        "embedding read");
  }
  return check_device_status(c);
}

// Behind the guard that keeps C++ exceptions (a failed host allocation, most of all)
// inside the library: the two entry points whose host buffers follow the input.
qasr_status qasr_audio_load_checkpoint(qasr_audio_ctx* c, qasr_checkpoint* ck, const char* prefix_c) {
  return qasr::guard([&] { return audio_load_checkpoint_body(c, ck, prefix_c); },
                     [&](qasr_status s, const std::string& m) { return c ? afail(c, s, "%s", m.c_str()) : s; });
}

qasr_status qasr_audio_encode_batch(qasr_audio_ctx* c, int32_t n, const float* const* mels,
                                    const int32_t* n_frames, int32_t n_mels, uint16_t* const* outs) {
  return qasr::guard([&] { return audio_encode_batch_body(c, n, mels, n_frames, n_mels, outs); },
                     [&](qasr_status s, const std::string& m) { return c ? afail(c, s, "%s", m.c_str()) : s; });
}

qasr_status qasr_audio_encode(qasr_audio_ctx* c, const float* mel, int32_t n_mels, int32_t n_frames, uint16_t* out,
                              int32_t out_rows, int32_t* n_tokens) {
  if (!c || !mel || !out) return QASR_ERR_INVALID_ARG;
  const int32_t need = qasr_audio_token_count(&c->cfg, n_frames);
  if (n_frames > 0 && need > out_rows)
    return afail(c, QASR_ERR_CAPACITY, "mel of %d frames gives %d rows, out holds %d", n_frames, need, out_rows);
  uint16_t* outs[1] = {out};
  const float* mels[1] = {mel};
  const qasr_status s = qasr_audio_encode_batch(c, 1, mels, &n_frames, n_mels, outs);
  if (s == QASR_OK && n_tokens) *n_tokens = need;
  return s;
}

}  // extern "C"
