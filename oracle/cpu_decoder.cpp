// CPU oracle: restatement of CpuTextDecoder (src/cpu_decoder.rs) — TEST INFRASTRUCTURE.
// Built with -ffp-contract=off -fno-fast-math: Rust neither contracts a*b+c into an FMA
// nor reassociates, so every f32 expression below is evaluated in source order.
#include "oracle.h"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace {

// half::f16::from_f32 (IEEE binary16, round to nearest even).
uint16_t to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return static_cast<uint16_t>(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax < 0x38800000u) {
    if (ax < 0x33000000u) return static_cast<uint16_t>(sign);
    const uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u, sh = 126u - e;
    uint32_t k = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u), hw = 1u << (sh - 1u);
    if (rem > hw || (rem == hw && (k & 1u))) ++k;
    return static_cast<uint16_t>(sign | k);
  }
  const uint32_t r = ax - 0x38000000u;
  uint32_t h = r >> 13;
  const uint32_t rem = r & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  if (h >= 0x7c00u) h = 0x7c00u;
  return static_cast<uint16_t>(sign | h);
}

float to_f32(uint16_t h) {
  const uint32_t sign = (static_cast<uint32_t>(h) & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {
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

// f16 -> f16 rounding of an f32 value, returned as f32 (what the reference's f16
// buffers hold once read back with to_f32()).
inline float r16(float v) { return to_f32(to_f16(v)); }

// Summation order of every f32 dot product: 0 = the reference's (below), 1 = each
// accumulator walks k backwards.  The second is an equally valid evaluation of the same
// sums; tests run the oracle both ways to measure the model's own sensitivity to the
// order of f32 additions (the floor under any GPU-vs-CPU logit difference).
int g_sum_order = 0;

// `Mat` (src/cpu_decoder.rs:11-102): row-major f32 copy of the f16 (or dequantised
// int8) weight.
struct Mat {
  std::vector<float> data;
  int rows = 0, cols = 0;

  // dot_transposed (src/cpu_decoder.rs:64-101) for one input row: 4 strided f32
  // accumulators, (a0+a1)+(a2+a3), then the tail.
  float dot4(int o, const float* x) const {
    const float* w = &data[static_cast<size_t>(o) * cols];
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    const int quads = cols / 4;
    for (int qq = 0; qq < quads; ++qq) {
      const int k = (g_sum_order ? quads - 1 - qq : qq) * 4;
      a0 += w[k] * x[k];
      a1 += w[k + 1] * x[k + 1];
      a2 += w[k + 2] * x[k + 2];
      a3 += w[k + 3] * x[k + 3];
    }
    float s = (a0 + a1) + (a2 + a3);
    for (int k = quads * 4; k < cols; ++k) s += w[k] * x[k];
    return s;
  }

  // The rows >= 2 path calls the `gemm` crate (src/cpu_decoder.rs:558-585) whose
  // summation order is not restated here: a fixed 16-way strided order stands in.
  float dot16(int o, const float* x) const {
    const float* w = &data[static_cast<size_t>(o) * cols];
    float a[16] = {0};
    const int blocks = cols / 16;
    for (int bb = 0; bb < blocks; ++bb) {
      const int b = g_sum_order ? blocks - 1 - bb : bb;
      for (int j = 0; j < 16; ++j) a[j] += w[b * 16 + j] * x[b * 16 + j];
    }
    for (int j = 8; j > 0; j >>= 1)
      for (int i = 0; i < j; ++i) a[i] = a[i] + a[i + j];
    float s = a[0];
    for (int k = blocks * 16; k < cols; ++k) s += w[k] * x[k];
    return s;
  }

  // acc[r * rows_out + o] = W[o] . x[r]
  void matmul(const std::vector<float>& xs, int nrows, std::vector<float>& acc) const {
    acc.assign(static_cast<size_t>(nrows) * rows, 0.f);
    if (nrows == 1) {
#pragma omp parallel for schedule(static, 64)
      for (int o = 0; o < rows; ++o) acc[o] = dot4(o, xs.data());
    } else {
#pragma omp parallel for collapse(2) schedule(static)
      for (int r = 0; r < nrows; ++r)
        for (int o = 0; o < rows; ++o)
          acc[static_cast<size_t>(r) * rows + o] = dot16(o, &xs[static_cast<size_t>(r) * cols]);
    }
  }

  // batch_dot (src/cpu_decoder.rs:28-43): out = f16(acc)
  void batch_dot(const std::vector<uint16_t>& x, int nrows, std::vector<uint16_t>& out) const {
    std::vector<float> xs(x.size()), acc;
    for (size_t i = 0; i < x.size(); ++i) xs[i] = to_f32(x[i]);
    matmul(xs, nrows, acc);
    out.resize(acc.size());
    for (size_t i = 0; i < acc.size(); ++i) out[i] = to_f16(acc[i]);
  }

  // batch_dot_acc (src/cpu_decoder.rs:45-62): h = f16(f32(h) + acc), one rounding
  void batch_dot_acc(const std::vector<uint16_t>& x, int nrows, std::vector<uint16_t>& h) const {
    std::vector<float> xs(x.size()), acc;
    for (size_t i = 0; i < x.size(); ++i) xs[i] = to_f32(x[i]);
    matmul(xs, nrows, acc);
    for (size_t i = 0; i < acc.size(); ++i) h[i] = to_f16(to_f32(h[i]) + acc[i]);
  }
};

// dequant_i8 (src/weights.rs:372-385): f16(f32(q) * scale[row]) per value.
void dequant_rows(const int8_t* q, const float* scale, int rows, int cols, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float s = scale[r];
    for (int c = 0; c < cols; ++c) {
      const size_t i = static_cast<size_t>(r) * cols + c;
      out[i] = to_f16(static_cast<float>(q[i]) * s);
    }
  }
}

struct Layer {
  std::vector<float> iln, pln, qn, kn;
  Mat q, k, v, o, gate, up, down;
};

}  // namespace

struct oracle_model {
  oracle_cfg cfg;
  std::vector<uint16_t> embed;
  std::vector<float> norm_w;
  std::vector<Layer> layers;
  std::vector<float> cos, sin;
  int rope_positions = 0;
};

struct oracle_seq {
  oracle_model* m;
  int max_seq;
  int cap;
  int pos = 0;
  uint32_t last_token = 0;
  std::vector<float> k_cache, v_cache;  // [layer][kvh][cap][hd]
  std::vector<uint16_t> last_x;         // hidden rows of the last forward
  int last_rows = 0;
};

namespace {

void rms_norm_row(const uint16_t* x, const float* w, int n, float eps, uint16_t* out) {
  // src/cpu_decoder.rs:261-272
  float sum2 = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float f = to_f32(x[i]);
    sum2 += f * f;
  }
  const float inv = 1.0f / std::sqrt(sum2 / static_cast<float>(n) + eps);
  for (int i = 0; i < n; ++i) out[i] = to_f16(to_f32(x[i]) * inv * w[i]);
}

void norm_rope_head(const uint16_t* raw, const float* nw, int hd, float eps, const float* c,
                    const float* s, uint16_t* out) {
  // src/cpu_decoder.rs:274-290
  const int half = hd / 2;
  float sum2 = 0.0f;
  for (int j = 0; j < hd; ++j) {
    const float f = to_f32(raw[j]);
    sum2 += f * f;
  }
  const float inv = 1.0f / std::sqrt(sum2 / static_cast<float>(hd) + eps);
  for (int j = 0; j < hd; ++j) {
    const float xj = to_f32(raw[j]) * inv * nw[j];
    const int pj = j < half ? j + half : j - half;
    const float sign = j < half ? -1.0f : 1.0f;
    const float xp = to_f32(raw[pj]) * inv * nw[pj];
    out[j] = to_f16(xj * c[j] + sign * xp * s[j]);
  }
}

void attention_head(const float* qrow, const float* krow_all, const float* vrow_all, int valid,
                    int hd, float scale, float* scores, float* acc, uint16_t* out) {
  // src/cpu_decoder.rs:315-361
  float best = -INFINITY;
  const int quads = hd / 4;
  for (int t = 0; t < valid; ++t) {
    const float* krow = krow_all + static_cast<size_t>(t) * hd;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int q = 0; q < quads; ++q) {
      const int j = q * 4;
      a0 += qrow[j] * krow[j];
      a1 += qrow[j + 1] * krow[j + 1];
      a2 += qrow[j + 2] * krow[j + 2];
      a3 += qrow[j + 3] * krow[j + 3];
    }
    const float dot = (a0 + a1) + (a2 + a3);
    const float sc = dot * scale;
    scores[t] = sc;
    if (sc > best) best = sc;
  }
  float sum = 0.0f;
  for (int t = 0; t < valid; ++t) {
    scores[t] = std::exp(scores[t] - best);
    sum += scores[t];
  }
  const float inv = 1.0f / sum;
  for (int j = 0; j < hd; ++j) acc[j] = 0.0f;
  for (int t = 0; t < valid; ++t) {
    const float w = scores[t] * inv;
    const float* vrow = vrow_all + static_cast<size_t>(t) * hd;
    for (int j = 0; j < hd; ++j) acc[j] += w * vrow[j];
  }
  for (int j = 0; j < hd; ++j) out[j] = to_f16(acc[j]);
}

// forward (src/cpu_decoder.rs:367-456): x is [rows][hs] f16, positions q0..q0+rows.
void forward(oracle_seq* s, std::vector<uint16_t>& x, int q0, int rows) {
  oracle_model* m = s->m;
  const oracle_cfg& c = m->cfg;
  const int hs = c.hidden_size, nqh = c.num_attention_heads, nkvh = c.num_key_value_heads,
            hd = c.head_dim, inter = c.intermediate_size;
  const int q_dim = nqh * hd, kv_dim = nkvh * hd;
  const size_t kv_stride = static_cast<size_t>(s->cap) * hd;
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  const int rep = nqh / nkvh;

  std::vector<uint16_t> normed(static_cast<size_t>(rows) * hs), q, k, v,
      attn(static_cast<size_t>(rows) * q_dim), norm2(static_cast<size_t>(rows) * hs), gate, up;
  for (size_t li = 0; li < m->layers.size(); ++li) {
    const Layer& L = m->layers[li];
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
      rms_norm_row(&x[static_cast<size_t>(r) * hs], L.iln.data(), hs, c.rms_norm_eps,
                   &normed[static_cast<size_t>(r) * hs]);
    L.q.batch_dot(normed, rows, q);
    L.k.batch_dot(normed, rows, k);
    L.v.batch_dot(normed, rows, v);

    const size_t layer_off = li * nkvh * kv_stride;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
      const int pos = q0 + r;
      std::vector<uint16_t> raw(hd), tmp(hd);
      const float* cr = &m->cos[static_cast<size_t>(pos) * hd];
      const float* sr = &m->sin[static_cast<size_t>(pos) * hd];
      for (int h = 0; h < nqh; ++h) {
        const size_t off = static_cast<size_t>(r) * q_dim + static_cast<size_t>(h) * hd;
        std::memcpy(raw.data(), &q[off], hd * 2);
        norm_rope_head(raw.data(), L.qn.data(), hd, c.rms_norm_eps, cr, sr, tmp.data());
        std::memcpy(&q[off], tmp.data(), hd * 2);
      }
      for (int h = 0; h < nkvh; ++h) {
        const size_t off = static_cast<size_t>(r) * kv_dim + static_cast<size_t>(h) * hd;
        std::memcpy(raw.data(), &k[off], hd * 2);
        norm_rope_head(raw.data(), L.kn.data(), hd, c.rms_norm_eps, cr, sr, tmp.data());
        const size_t dst = layer_off + h * kv_stride + static_cast<size_t>(pos) * hd;
        for (int j = 0; j < hd; ++j) s->k_cache[dst + j] = to_f32(tmp[j]);
        for (int j = 0; j < hd; ++j) s->v_cache[dst + j] = to_f32(v[off + j]);
      }
    }

    // attention (src/cpu_decoder.rs:292-365), parallel over (row, head)
#pragma omp parallel
    {
      std::vector<float> scores(s->cap), acc(hd), qrow(hd);
#pragma omp for schedule(dynamic, 4)
      for (int hi = 0; hi < rows * nqh; ++hi) {
        const int r = hi / nqh, h = hi % nqh;
        const int pos = q0 + r;
        const int valid = std::min(pos + 1, s->cap);
        const uint16_t* qh = &q[static_cast<size_t>(r) * q_dim + static_cast<size_t>(h) * hd];
        for (int d = 0; d < hd; ++d) qrow[d] = to_f32(qh[d]);
        const size_t kb = layer_off + static_cast<size_t>(h / rep) * kv_stride;
        attention_head(qrow.data(), &s->k_cache[kb], &s->v_cache[kb], valid, hd, scale,
                       scores.data(), acc.data(),
                       &attn[static_cast<size_t>(r) * q_dim + static_cast<size_t>(h) * hd]);
      }
    }

    L.o.batch_dot_acc(attn, rows, x);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
      rms_norm_row(&x[static_cast<size_t>(r) * hs], L.pln.data(), hs, c.rms_norm_eps,
                   &norm2[static_cast<size_t>(r) * hs]);
    L.gate.batch_dot(norm2, rows, gate);
    L.up.batch_dot(norm2, rows, up);
    // SiLU * up (src/cpu_decoder.rs:442-448)
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < static_cast<long long>(rows) * inter; ++i) {
      const float g = to_f32(gate[i]);
      const float silu = g / (1.0f + std::exp(-g));
      gate[i] = to_f16(silu * to_f32(up[i]));
    }
    L.down.batch_dot_acc(gate, rows, x);
  }
}

// final_norm_logits + argmax (src/cpu_decoder.rs:458-482)
int32_t logits_argmax(oracle_seq* s, const std::vector<uint16_t>& x, int rows, float* logits_out) {
  oracle_model* m = s->m;
  const int hs = m->cfg.hidden_size, vocab = m->cfg.vocab_size;
  std::vector<uint16_t> normed(hs);
  rms_norm_row(&x[static_cast<size_t>(rows - 1) * hs], m->norm_w.data(), hs, m->cfg.rms_norm_eps,
               normed.data());
  std::vector<float> nx(hs);
  for (int i = 0; i < hs; ++i) nx[i] = to_f32(normed[i]);
  std::vector<float> logits(vocab);
#pragma omp parallel for schedule(static, 256)
  for (int t = 0; t < vocab; ++t) {
    const uint16_t* row = &m->embed[static_cast<size_t>(t) * hs];
    float acc = 0.0f;
    for (int ii = 0; ii < hs; ++ii) {
      const int i = g_sum_order ? hs - 1 - ii : ii;
      acc += to_f32(row[i]) * nx[i];
    }
    logits[t] = acc;
  }
  int best = 0;
  for (int i = 0; i < vocab; ++i)
    if (logits[i] > logits[best]) best = i;
  if (logits_out) std::memcpy(logits_out, logits.data(), sizeof(float) * vocab);
  return best;
}

}  // namespace

extern "C" {

oracle_model* oracle_model_create(const oracle_cfg* cfg) {
  if (!cfg || cfg->num_key_value_heads <= 0 ||
      cfg->num_attention_heads % cfg->num_key_value_heads != 0)
    return nullptr;
  auto* m = new oracle_model();
  m->cfg = *cfg;
  m->layers.resize(cfg->num_hidden_layers);
  return m;
}

void oracle_model_destroy(oracle_model* m) { delete m; }

int oracle_load_embed(oracle_model* m, const uint16_t* embed, const uint16_t* final_norm) {
  const size_t n = static_cast<size_t>(m->cfg.vocab_size) * m->cfg.hidden_size;
  m->embed.assign(embed, embed + n);
  m->norm_w.resize(m->cfg.hidden_size);
  for (int i = 0; i < m->cfg.hidden_size; ++i) m->norm_w[i] = to_f32(final_norm[i]);
  return 0;
}

int oracle_load_layer(oracle_model* m, int layer, int weight_format, const void* const lin[7],
                      const float* const scales[7], const uint16_t* iln, const uint16_t* pln,
                      const uint16_t* qn, const uint16_t* kn) {
  if (layer < 0 || layer >= m->cfg.num_hidden_layers) return 1;
  const oracle_cfg& c = m->cfg;
  const int hs = c.hidden_size, qd = c.num_attention_heads * c.head_dim,
            kvd = c.num_key_value_heads * c.head_dim, I = c.intermediate_size;
  const int shapes[7][2] = {{qd, hs}, {kvd, hs}, {kvd, hs}, {hs, qd}, {I, hs}, {I, hs}, {hs, I}};
  Layer& L = m->layers[layer];
  Mat* mats[7] = {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down};
  for (int i = 0; i < 7; ++i) {
    const int rows = shapes[i][0], cols = shapes[i][1];
    const size_t n = static_cast<size_t>(rows) * cols;
    std::vector<uint16_t> h(n);
    if (weight_format == 1) {
      dequant_rows(static_cast<const int8_t*>(lin[i]), scales[i], rows, cols, h.data());
    } else {
      std::memcpy(h.data(), lin[i], n * 2);
    }
    mats[i]->rows = rows;
    mats[i]->cols = cols;
    mats[i]->data.resize(n);
#pragma omp parallel for schedule(static)
    for (long long j = 0; j < static_cast<long long>(n); ++j) mats[i]->data[j] = to_f32(h[j]);
  }
  auto vec = [&](const uint16_t* p, int n, std::vector<float>& out) {
    out.resize(n);
    for (int i = 0; i < n; ++i) out[i] = to_f32(p[i]);
  };
  vec(iln, hs, L.iln);
  vec(pln, hs, L.pln);
  vec(qn, c.head_dim, L.qn);
  vec(kn, c.head_dim, L.kn);
  return 0;
}

int oracle_set_rope_tables(oracle_model* m, const uint16_t* cos, const uint16_t* sin,
                           int positions) {
  const size_t n = static_cast<size_t>(positions) * m->cfg.head_dim;
  m->cos.resize(n);
  m->sin.resize(n);
  for (size_t i = 0; i < n; ++i) {
    m->cos[i] = to_f32(cos[i]);
    m->sin[i] = to_f32(sin[i]);
  }
  m->rope_positions = positions;
  return 0;
}

oracle_seq* oracle_seq_create(oracle_model* m, int max_seq) {
  auto* s = new oracle_seq();
  s->m = m;
  s->max_seq = max_seq;
  // The reference grows its CPU cache in KV_STEP steps and *discards* the contents
  // on growth (src/cpu_decoder.rs:227-249); the oracle sizes it once, up front.
  s->cap = max_seq;
  const size_t n = static_cast<size_t>(m->cfg.num_hidden_layers) * m->cfg.num_key_value_heads *
                   max_seq * m->cfg.head_dim;
  s->k_cache.assign(n, 0.0f);
  s->v_cache.assign(n, 0.0f);
  return s;
}

void oracle_seq_destroy(oracle_seq* s) { delete s; }

int oracle_prefill(oracle_seq* s, const uint16_t* hidden, int rows, int kv_start, int32_t* token,
                   float* logits) {
  // src/cpu_decoder.rs:487-515
  const int hs = s->m->cfg.hidden_size;
  if (rows <= 0 || kv_start < 0 || kv_start + rows > s->max_seq ||
      kv_start + rows > s->m->rope_positions)
    return 1;
  std::vector<uint16_t> x(hidden, hidden + static_cast<size_t>(rows) * hs);
  forward(s, x, kv_start, rows);
  s->pos = kv_start + rows;
  const int32_t tok = logits_argmax(s, x, rows, logits);
  s->last_token = static_cast<uint32_t>(tok);
  s->last_x = x;
  s->last_rows = rows;
  if (token) *token = tok;
  return 0;
}

int oracle_step(oracle_seq* s, int32_t* token, float* logits) {
  // src/cpu_decoder.rs:518-530
  const int hs = s->m->cfg.hidden_size;
  if (s->pos >= s->max_seq || s->pos >= s->m->rope_positions) return 1;
  std::vector<uint16_t> x(hs);
  std::memcpy(x.data(), &s->m->embed[static_cast<size_t>(s->last_token) * hs], hs * 2);
  forward(s, x, s->pos, 1);
  s->pos += 1;
  const int32_t tok = logits_argmax(s, x, 1, logits);
  s->last_token = static_cast<uint32_t>(tok);
  s->last_x = x;
  s->last_rows = 1;
  if (token) *token = tok;
  return 0;
}

void oracle_set_last_token(oracle_seq* s, int32_t tok) { s->last_token = static_cast<uint32_t>(tok); }
int oracle_pos(const oracle_seq* s) { return s->pos; }
void oracle_set_sum_order(int order) { g_sum_order = order ? 1 : 0; }

void oracle_set_pos(oracle_seq* s, int pos) {
  if (pos >= 0 && pos <= s->max_seq) s->pos = pos;  // out-of-range positions are ignored
}

int oracle_last_hidden(const oracle_seq* s, uint16_t* out, int rows) {
  if (rows > s->last_rows) return 1;
  std::memcpy(out, s->last_x.data(), static_cast<size_t>(rows) * s->m->cfg.hidden_size * 2);
  return 0;
}

int oracle_kv_rows(const oracle_seq* s, int layer, int kv_head, int pos0, int n, float* k,
                   float* v) {
  const oracle_cfg& c = s->m->cfg;
  if (layer < 0 || layer >= c.num_hidden_layers || kv_head < 0 ||
      kv_head >= c.num_key_value_heads || pos0 < 0 || pos0 + n > s->cap)
    return 1;
  const size_t base = (static_cast<size_t>(layer) * c.num_key_value_heads + kv_head) *
                          static_cast<size_t>(s->cap) * c.head_dim +
                      static_cast<size_t>(pos0) * c.head_dim;
  std::memcpy(k, &s->k_cache[base], sizeof(float) * n * c.head_dim);
  std::memcpy(v, &s->v_cache[base], sizeof(float) * n * c.head_dim);
  return 0;
}

uint16_t oracle_f32_to_f16(float f) { return to_f16(f); }
float oracle_f16_to_f32(uint16_t h) { return to_f32(h); }

void oracle_dequant_i8(const int8_t* q, const float* scale, int rows, int cols, uint16_t* out) {
  dequant_rows(q, scale, rows, cols, out);
}

void oracle_gemv_f16(const uint16_t* w, int n_out, int cols, const uint16_t* x, uint16_t* y) {
  Mat m;
  m.rows = n_out;
  m.cols = cols;
  m.data.resize(static_cast<size_t>(n_out) * cols);
  for (size_t i = 0; i < m.data.size(); ++i) m.data[i] = to_f32(w[i]);
  std::vector<uint16_t> xv(x, x + cols), out;
  m.batch_dot(xv, 1, out);
  std::memcpy(y, out.data(), sizeof(uint16_t) * n_out);
}

void oracle_gemv_acc_f16(const uint16_t* w, int n_out, int cols, const uint16_t* x, uint16_t* h) {
  Mat m;
  m.rows = n_out;
  m.cols = cols;
  m.data.resize(static_cast<size_t>(n_out) * cols);
  for (size_t i = 0; i < m.data.size(); ++i) m.data[i] = to_f32(w[i]);
  std::vector<uint16_t> xv(x, x + cols), hv(h, h + n_out);
  m.batch_dot_acc(xv, 1, hv);
  std::memcpy(h, hv.data(), sizeof(uint16_t) * n_out);
}

void oracle_matmul_rows(const float* x, const float* w, int m, int n, int k, float* out) {
  // the rows >= 2 path of Mat::batch_dot (stands in for the `gemm` crate call)
  Mat mat;
  mat.rows = n;
  mat.cols = k;
  mat.data.assign(w, w + static_cast<size_t>(n) * k);
  std::vector<float> xs(x, x + static_cast<size_t>(m) * k), acc;
  mat.matmul(xs, m, acc);
  std::memcpy(out, acc.data(), sizeof(float) * acc.size());
}

void oracle_gemm_naive(float* out, const float* x, const float* w, int m, int n, int k) {
  // the reference test's naive loop (src/cpu_decoder.rs:606-613)
  for (int r = 0; r < m; ++r)
    for (int o = 0; o < n; ++o) {
      float s = 0.0f;
      for (int p = 0; p < k; ++p) s += x[static_cast<size_t>(r) * k + p] * w[static_cast<size_t>(o) * k + p];
      out[static_cast<size_t>(r) * n + o] = s;
    }
}

void oracle_rms_norm_row(const uint16_t* x, const float* w, int n, float eps, uint16_t* out) {
  rms_norm_row(x, w, n, eps, out);
}

void oracle_norm_rope_head(const uint16_t* raw, const float* nw, int hd, float eps,
                           const float* cos_row, const float* sin_row, uint16_t* out) {
  norm_rope_head(raw, nw, hd, eps, cos_row, sin_row, out);
}

void oracle_attention_head(const uint16_t* q, const float* k, const float* v, int valid, int hd,
                           uint16_t* out) {
  std::vector<float> qrow(hd), scores(valid > 0 ? valid : 1), acc(hd);
  for (int d = 0; d < hd; ++d) qrow[d] = to_f32(q[d]);
  attention_head(qrow.data(), k, v, valid, hd, 1.0f / std::sqrt(static_cast<float>(hd)),
                 scores.data(), acc.data(), out);
}

int oracle_argmax(const float* logits, int n) {
  int best = 0;
  for (int i = 0; i < n; ++i)
    if (logits[i] > logits[best]) best = i;
  return best;
}

void oracle_build_dim_map(const int* section, int nsection, int half, int interleaved, int* out) {
  // src/mrope.rs:5-41
  int len = 0;
  if (interleaved) {
    std::vector<int> used(nsection, 0);
    while (len < half) {
      const int before = len;
      for (int d = 0; d < nsection; ++d) {
        if (len >= half) break;
        if (used[d] < section[d]) {
          out[len++] = d;
          used[d] += 1;
        }
      }
      if (len == before) break;
    }
  } else {
    for (int d = 0; d < nsection; ++d)
      for (int i = 0; i < section[d]; ++i) {
        if (len >= half) break;
        out[len++] = d;
      }
    while (len < half) out[len++] = nsection - 1;
  }
  for (int i = len; i < half; ++i) out[i] = -1;  // quotas exhausted before `half`
}

void oracle_mrope_cos_sin_f32(int positions, int head_dim, double theta, const int* section,
                              int nsection, int interleaved, float* cos_out, float* sin_out) {
  // compute_mrope_cos_sin over text_positions (src/mrope.rs:46-80): every axis holds
  // 0..positions, so the per-frequency axis map selects the same position.
  const int half = head_dim / 2;
  std::vector<double> inv(half);
  for (int i = 0; i < half; ++i)
    inv[i] = 1.0 / std::pow(theta, 2.0 * static_cast<double>(i) / static_cast<double>(head_dim));
  std::vector<int> dm(half);
  oracle_build_dim_map(section, nsection, half, interleaved, dm.data());
  for (int t = 0; t < positions; ++t)
    for (int j = 0; j < half; ++j) {
      const double angle = static_cast<double>(t) * inv[j];
      const float c = static_cast<float>(std::cos(angle));
      const float s = static_cast<float>(std::sin(angle));
      const size_t b = static_cast<size_t>(t) * head_dim;
      cos_out[b + j] = c;
      sin_out[b + j] = s;
      cos_out[b + j + half] = c;
      sin_out[b + j + half] = s;
    }
}

}  // extern "C"
