// One decode round of a streaming session: the part of the reference's streaming loop
// that drives the decoder (src/stream.rs:338-403).  Each round the caller hands over the
// full prefill rows of the round (prompt embeddings, audio rows, rolled-back text); the
// session prefills only the rows after the longest prefix unchanged since the previous
// round (the cached KV rows of that prefix are exactly what a re-prefill would recompute),
// then decodes greedily until an end id or the round's budget, and drops same-token runs
// longer than the cap from what it returns.  Text assembly, rollback and the tokenizer
// stay with the caller.
#include <algorithm>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "abi_guard.h"
#include "ctx_internal.h"
#include "qasr_b200.h"

struct qasr_session {
  qasr_ctx* ctx;
  int slot;
  int kv_reuse;
  int hidden_size;
  std::vector<uint16_t> prev;  // the previous round's prefill rows (kv_reuse only)
};

extern "C" {

// common_rows (src/stream.rs:666-676): whole `row_bytes` rows equal at the start of both.
size_t qasr_common_rows(const void* a, size_t a_bytes, const void* b, size_t b_bytes, size_t row_bytes) {
  if (row_bytes == 0 || a == nullptr || b == nullptr) return 0;
  const size_t n = std::min(a_bytes / row_bytes, b_bytes / row_bytes);
  const unsigned char* pa = static_cast<const unsigned char*>(a);
  const unsigned char* pb = static_cast<const unsigned char*>(b);
  size_t i = 0;
  while (i < n && std::memcmp(pa + i * row_bytes, pb + i * row_bytes, row_bytes) == 0) ++i;
  return i;
}

// suppress_runs (src/stream.rs:702-737): the run of the last token of `prev` (counted
// back, capped at max_run) continues into `next`; a token that extends a run past max_run
// is dropped.  Writes the kept tokens to `out` (room for n_next) and returns the number
// dropped, or -1 on a bad argument.
int qasr_suppress_runs(const uint32_t* prev, int n_prev, const uint32_t* next, int n_next, int max_run,
                       uint32_t* out, int* n_out) {
  if (n_prev < 0 || n_next < 0 || (n_prev > 0 && !prev) || (n_next > 0 && (!next || !out)) || !n_out) return -1;
  bool have = false;
  uint32_t tok = 0;
  int run = 0;
  if (n_prev > 0) {
    have = true;
    tok = prev[n_prev - 1];
    run = 1;
    for (int i = n_prev - 2; i >= 0; --i) {
      if (prev[i] != tok) break;
      ++run;
      if (run >= max_run) break;
    }
  }
  int kept = 0, dropped = 0;
  for (int i = 0; i < n_next; ++i) {
    bool drop = false;
    if (have && next[i] == tok) {
      ++run;
      drop = run > max_run;
    } else {
      have = true;
      tok = next[i];
      run = 1;
    }
    if (drop) ++dropped;
    else out[kept++] = next[i];
  }
  *n_out = kept;
  return dropped;
}

qasr_status qasr_session_create(qasr_ctx* ctx, int slot, int kv_reuse, qasr_session** out) {
  if (!ctx || !out) return QASR_ERR_INVALID_ARG;
  *out = nullptr;
  qasr_text_config cfg{};
  int fmt = 0;
  if (!qasr::ctx_shape(ctx, &cfg, &fmt)) return QASR_ERR_INVALID_ARG;
  int pos = 0;
  if (qasr_status s = qasr_slot_pos(ctx, slot, &pos)) return s;  // the slot must be allocated
  qasr_session* s = new (std::nothrow) qasr_session{ctx, slot, kv_reuse ? 1 : 0, cfg.hidden_size, {}};
  if (!s) return QASR_ERR_OOM;
  *out = s;
  return QASR_OK;
}

void qasr_session_destroy(qasr_session* s) { delete s; }

// The stream's recovery step forgets the previous round's rows (src/stream.rs:605), so
// the next round prefills all of its rows.
void qasr_session_reset(qasr_session* s) {
  if (s) s->prev.clear();
}

static qasr_status session_round_body(qasr_session* s, const uint16_t* hidden, int rows, int budget,
                                      const int32_t* eos, int n_eos, const uint32_t* prev_tokens, int n_prev,
                                      int max_run, int32_t* tokens, int* n_tokens, int* dropped, int* hit_eos,
                                      int* reused_rows) {
  if (!s || !hidden || rows <= 0 || budget <= 0 || (n_eos > 0 && !eos) || n_eos < 0 || max_run <= 0 || !tokens ||
      !n_tokens || !dropped || !hit_eos || !reused_rows || n_prev < 0 || (n_prev > 0 && !prev_tokens))
    return QASR_ERR_INVALID_ARG;
  *n_tokens = *dropped = *hit_eos = *reused_rows = 0;
  const size_t row_bytes = static_cast<size_t>(s->hidden_size) * sizeof(uint16_t);
  // the round must fit the decoder (src/stream.rs:343-348), then the slot grows to it
  if (static_cast<long long>(rows) + budget + 8 > qasr_max_seq(s->ctx))
    return qasr::ctx_fail(s->ctx, QASR_ERR_CAPACITY,
                          "live seq " + std::to_string(rows) + " + max_new " + std::to_string(budget) +
                              " exceeds decoder max_seq " + std::to_string(qasr_max_seq(s->ctx)));
  int cap = 0;
  if (qasr_status st = qasr_ensure_capacity(s->ctx, s->slot, rows + budget + 8, &cap)) return st;
  // the longest unchanged prefix, at most rows - 1 (one row is always prefilled for the
  // first token's logits), src/stream.rs:369-373
  size_t reuse = 0;
  if (s->kv_reuse)
    reuse = std::min(qasr_common_rows(s->prev.data(), s->prev.size() * sizeof(uint16_t), hidden,
                                      static_cast<size_t>(rows) * row_bytes, row_bytes),
                     static_cast<size_t>(rows - 1));
  // from here on the slot's rows past `reuse` are rewritten: until this round's prefill
  // has succeeded, only the first `reuse` rows of `prev` still describe its cache (a round
  // that fails part-way cannot leave a longer reusable prefix behind)
  if (s->kv_reuse) s->prev.resize(reuse * static_cast<size_t>(s->hidden_size));
  int32_t tok = 0;
  const int r = static_cast<int>(reuse);
  if (qasr_status st = qasr_prefill(s->ctx, s->slot, hidden + reuse * s->hidden_size, rows - r, r, &tok)) return st;
  if (s->kv_reuse) s->prev.assign(hidden, hidden + static_cast<size_t>(rows) * s->hidden_size);
  *reused_rows = r;
  // greedy decode until an end id or the budget (src/stream.rs:380-395)
  std::vector<uint32_t> fresh;
  fresh.reserve(static_cast<size_t>(budget));
  while (true) {
    if (std::find(eos, eos + n_eos, tok) != eos + n_eos) {
      *hit_eos = 1;
      break;
    }
    fresh.push_back(static_cast<uint32_t>(tok));
    if (static_cast<int>(fresh.size()) >= budget) break;
    if (qasr_status st = qasr_step(s->ctx, s->slot, &tok)) return st;
  }
  // same-token runs past max_run are dropped (src/stream.rs:403); the run may continue one
  // that ends the text fed back into this round's rows (`prev_tokens`)
  int kept = 0;
  std::vector<uint32_t> out(fresh.size());
  *dropped = qasr_suppress_runs(prev_tokens, n_prev, fresh.data(), static_cast<int>(fresh.size()), max_run,
                                out.data(), &kept);
  for (int i = 0; i < kept; ++i) tokens[i] = static_cast<int32_t>(out[i]);
  *n_tokens = kept;
  return QASR_OK;
}

qasr_status qasr_session_round(qasr_session* s, const uint16_t* hidden, int rows, int budget, const int32_t* eos,
                               int n_eos, const uint32_t* prev_tokens, int n_prev, int max_run, int32_t* tokens,
                               int* n_tokens, int* dropped, int* hit_eos, int* reused_rows) {
  return qasr::guard(
      [&] {
        return session_round_body(s, hidden, rows, budget, eos, n_eos, prev_tokens, n_prev, max_run, tokens,
                                  n_tokens, dropped, hit_eos, reused_rows);
      },
      [&](qasr_status st, const std::string& m) {
        if (s && s->kv_reuse) s->prev.clear();  // a round cut short leaves no reusable prefix
        return s ? qasr::ctx_fail(s->ctx, st, m) : st;
      });
}

}  // extern "C"
