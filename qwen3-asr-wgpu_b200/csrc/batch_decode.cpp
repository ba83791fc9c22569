// Many segments through a few decode slots: the reference's batch driver
// (decode_batch_embeds / run_batch_attempt, src/inference.rs:1944-2227; fill_slots
// :699-756; Outcomes :866-915; the single-sequence loop of generate_from_embeds
// :2229-2376) over the operations of a qasr_decode_backend.  Host code only: the
// device work is the backend's (a qasr_ctx, or a test's fake).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <vector>

#include "abi_guard.h"
#include "ctx_internal.h"
#include "qasr_b200.h"

namespace {

long long round_up(long long x, int m) { return (x + m - 1) / m * m; }

struct Run {
  const qasr_decode_backend* be;
  const qasr_segment* segs;
  const qasr_batch_options* o;
  const qasr_batch_events* ev;
  qasr_item_result* res;
  std::vector<char> emitted;

  bool is_eos(int32_t t) const { return t == o->eos[0] || t == o->eos[1]; }
  bool should_stop() const { return ev && ev->should_stop && ev->should_stop(ev->user) != 0; }
  // KV positions a segment needs, in 64-bit (len + max_new near INT_MAX must not wrap)
  long long cap_of(int i) const {
    return round_up(static_cast<long long>(segs[i].len) + segs[i].max_new_tokens + 8, o->kv_step);
  }

  // Outcomes::done: the first result of an item is final and reported at once
  void done(int i, int status, int stop, const std::vector<int32_t>& toks) {
    if (emitted[static_cast<size_t>(i)]) return;
    emitted[static_cast<size_t>(i)] = 1;
    qasr_item_result& r = res[i];
    r.status = status;
    r.stop_reason = stop;
    r.n_tokens = status == QASR_OK ? static_cast<int32_t>(std::min<size_t>(toks.size(), segs[i].max_new_tokens)) : 0;
    if (r.n_tokens > 0) std::memcpy(r.tokens, toks.data(), static_cast<size_t>(r.n_tokens) * sizeof(int32_t));
    if (ev && ev->on_item) ev->on_item(ev->user, i, &r);
  }

  // generate_from_embeds' loop (src/inference.rs:2300-2376): first token from the
  // prefill; EOS there ends with nothing; then at most max_new - 1 steps.
  int decode_one(int i, std::vector<int32_t>* toks, int* stop) {
    const qasr_segment& g = segs[i];
    int slot = -1;
    // a cap past INT32_MAX is asked as INT32_MAX: the backend clamps it to its max_seq
    // and the prefill or a step then reports the shortfall
    int st = be->fork_capped(be->user, static_cast<int>(std::min<long long>(cap_of(i), INT32_MAX)), &slot);
    if (st) return st;
    int32_t tok = 0;
    st = be->prefill_batch(be->user, &slot, 1, g.hidden, &g.len, &tok);
    *stop = QASR_STOP_MAX_TOKENS;
    if (!st) {
      if (is_eos(tok)) {
        *stop = QASR_STOP_EOS;
      } else {
        toks->push_back(tok);
        for (int k = 1; k < g.max_new_tokens; ++k) {
          if ((st = be->step_batch(be->user, &slot, 1, &tok))) break;
          if (is_eos(tok)) {
            *stop = QASR_STOP_EOS;
            break;
          }
          toks->push_back(tok);
        }
      }
    }
    be->slot_free(be->user, slot);
    return st;
  }

  void decode_one_reported(int i) {
    if (should_stop()) {
      done(i, QASR_ERR_CANCELLED, QASR_STOP_MAX_TOKENS, {});
      return;
    }
    std::vector<int32_t> toks;
    int stop = QASR_STOP_MAX_TOKENS;
    const int st = decode_one(i, &toks, &stop);
    done(i, st, stop, toks);
  }

  enum Attempt { kAll, kStopped, kFailed };

  // run_batch_attempt (src/inference.rs:2110-2227)
  Attempt attempt(const std::vector<int>& run, int width) {
    const int nslots = std::min<int>(width, static_cast<int>(run.size()));
    int cap = o->kv_step;  // the run's segments all fit batch_seq_cap, an int
    for (int i : run) cap = std::max(cap, static_cast<int>(cap_of(i)));
    std::vector<int> slot_id;
    auto release = [&]() {
      for (int s : slot_id) be->slot_free(be->user, s);
    };
    for (int k = 0; k < nslots; ++k) {
      int s = -1;
      if (be->fork_capped(be->user, cap, &s)) {
        release();
        return kFailed;
      }
      slot_id.push_back(s);
    }
    const size_t nseg = static_cast<size_t>(emitted.size());
    std::vector<std::vector<int32_t>> gen(nseg);
    std::vector<int> stop(nseg, QASR_STOP_MAX_TOKENS);
    std::vector<int> active(static_cast<size_t>(nslots), -1);  // segment per slot
    size_t frontier = 0;
    // longest prompt first (a stable sort, like sort_by_key)
    std::vector<int> order = run;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return segs[a].len > segs[b].len; });
    const size_t hs = static_cast<size_t>(be->hidden_size);

    // fill_slots (src/inference.rs:699-756): every free slot from the frontier, in one
    // batched prefill; a segment whose first token is an eos id frees its slot again
    // (and, as in the reference, is not reported here)
    auto fill = [&]() -> bool {
      while (true) {
        std::vector<int> free;
        for (int s = 0; s < nslots; ++s)
          if (active[static_cast<size_t>(s)] < 0) free.push_back(s);
        const size_t take = std::min(free.size(), order.size() - frontier);
        if (take == 0) return true;
        std::vector<int> ids, lens;
        std::vector<uint16_t> hidden;
        for (size_t k = 0; k < take; ++k) {
          const qasr_segment& g = segs[order[frontier + k]];
          ids.push_back(slot_id[static_cast<size_t>(free[k])]);
          lens.push_back(g.len);
          hidden.insert(hidden.end(), g.hidden, g.hidden + static_cast<size_t>(g.len) * hs);
        }
        std::vector<int32_t> firsts(take);
        if (be->prefill_batch(be->user, ids.data(), static_cast<int>(take), hidden.data(), lens.data(),
                              firsts.data()))
          return false;
        for (size_t k = 0; k < take; ++k) {
          const int g = order[frontier + k];
          if (is_eos(firsts[k])) {
            stop[static_cast<size_t>(g)] = QASR_STOP_EOS;
          } else {
            gen[static_cast<size_t>(g)].push_back(firsts[k]);
            active[static_cast<size_t>(free[k])] = g;
          }
        }
        frontier += take;
      }
    };

    if (!fill()) {
      release();
      return kFailed;
    }
    std::vector<int> step_ids;
    std::vector<int> step_slots;
    std::vector<int32_t> toks;
    while (std::any_of(active.begin(), active.end(), [](int a) { return a >= 0; })) {
      if (should_stop()) {
        release();
        return kStopped;
      }
      step_ids.clear();
      step_slots.clear();
      for (int s = 0; s < nslots; ++s)
        if (active[static_cast<size_t>(s)] >= 0) {
          step_ids.push_back(slot_id[static_cast<size_t>(s)]);
          step_slots.push_back(s);
        }
      toks.assign(step_ids.size(), 0);
      if (be->step_batch(be->user, step_ids.data(), static_cast<int>(step_ids.size()), toks.data())) {
        release();
        return kFailed;
      }
      for (size_t k = 0; k < step_slots.size(); ++k) {
        const int s = step_slots[k];
        const int seg = active[static_cast<size_t>(s)];
        if (seg < 0) continue;
        const int32_t tok = toks[k];
        std::vector<int32_t>& gs = gen[static_cast<size_t>(seg)];
        if (is_eos(tok)) {
          stop[static_cast<size_t>(seg)] = QASR_STOP_EOS;
          active[static_cast<size_t>(s)] = -1;
        } else if (static_cast<int>(gs.size()) >= segs[seg].max_new_tokens) {
          stop[static_cast<size_t>(seg)] = QASR_STOP_MAX_TOKENS;
          active[static_cast<size_t>(s)] = -1;
        } else {
          gs.push_back(tok);
        }
        if (active[static_cast<size_t>(s)] < 0) {
          done(seg, QASR_OK, stop[static_cast<size_t>(seg)], gs);
          if (!fill()) {
            release();
            return kFailed;
          }
        }
      }
    }
    release();
    return kAll;
  }
};

struct CtxBackend {
  qasr_ctx* ctx;
  static int fork(void* u, int cap, int* slot) { return qasr_fork_capped(static_cast<CtxBackend*>(u)->ctx, cap, slot); }
  static int slot_free(void* u, int slot) { return qasr_slot_free(static_cast<CtxBackend*>(u)->ctx, slot); }
  static int prefill(void* u, const int* slots, int n, const uint16_t* hidden, const int* lens, int32_t* first) {
    return qasr_prefill_batch(static_cast<CtxBackend*>(u)->ctx, slots, n, hidden, lens, nullptr, first);
  }
  static int step(void* u, const int* slots, int n, int32_t* out) {
    return qasr_step_batch(static_cast<CtxBackend*>(u)->ctx, slots, n, out);
  }
};

}  // namespace

extern "C" {

static qasr_status batch_decode_body(const qasr_decode_backend* be, const qasr_segment* segs, int n,
                                     const qasr_batch_options* opts, const qasr_batch_events* events,
                                     qasr_item_result* results) {
  if (!be || !be->fork_capped || !be->slot_free || !be->prefill_batch || !be->step_batch || be->hidden_size <= 0 ||
      !opts || n < 0 || (n > 0 && (!segs || !results)) || opts->kv_step <= 0 || opts->batch_seq_cap <= 0)
    return QASR_ERR_INVALID_ARG;
  for (int i = 0; i < n; ++i)
    if (!segs[i].hidden || segs[i].len <= 0 || segs[i].max_new_tokens <= 0 || !results[i].tokens)
      return QASR_ERR_INVALID_ARG;
  Run r{be, segs, opts, events, results, std::vector<char>(static_cast<size_t>(n), 0)};
  for (int i = 0; i < n; ++i) {
    results[i].status = QASR_ERR_NOT_DECODED;
    results[i].stop_reason = QASR_STOP_MAX_TOKENS;
    results[i].n_tokens = 0;
  }
  // segments beyond the batched attention's reach: the single-sequence path, first
  std::vector<int> pending;
  for (int i = 0; i < n; ++i) {
    if (r.cap_of(i) > opts->batch_seq_cap) r.decode_one_reported(i);
    else pending.push_back(i);
  }
  int width = std::max(1, opts->width);
  while (!pending.empty()) {
    if (width < 2) {  // nothing to share a weight read with: one segment at a time
      for (int i : pending) r.decode_one_reported(i);
      break;
    }
    const Run::Attempt a = r.attempt(pending, width);
    if (a == Run::kAll) {
      pending.clear();
    } else if (a == Run::kStopped) {
      for (int i : pending) r.done(i, QASR_ERR_CANCELLED, QASR_STOP_MAX_TOKENS, {});
      pending.clear();
    } else {  // the slots could not hold this group: keep the finished, retry narrower
      width = std::max(1, width / 2);
      pending.erase(std::remove_if(pending.begin(), pending.end(),
                                   [&](int i) { return r.emitted[static_cast<size_t>(i)] != 0; }),
                    pending.end());
    }
  }
  for (int i = 0; i < n; ++i)  // Outcomes::finish: the rest were not decoded
    if (!r.emitted[static_cast<size_t>(i)]) r.done(i, QASR_ERR_NOT_DECODED, QASR_STOP_MAX_TOKENS, {});
  return QASR_OK;
}

qasr_status qasr_batch_decode_backend(const qasr_decode_backend* be, const qasr_segment* segs, int n,
                                      const qasr_batch_options* opts, const qasr_batch_events* events,
                                      qasr_item_result* results) {
  // no context to hold a message here: the status alone reports a host failure
  return qasr::guard([&] { return batch_decode_body(be, segs, n, opts, events, results); },
                     [](qasr_status s, const std::string&) { return s; });
}

qasr_status qasr_batch_decode(qasr_ctx* ctx, const qasr_segment* segs, int n, const qasr_batch_options* opts,
                              const qasr_batch_events* events, qasr_item_result* results) {
  qasr_text_config cfg{};
  if (!qasr::ctx_shape(ctx, &cfg, nullptr)) return QASR_ERR_INVALID_ARG;
  CtxBackend cb{ctx};
  qasr_decode_backend be{};
  be.user = &cb;
  be.hidden_size = cfg.hidden_size;
  be.fork_capped = &CtxBackend::fork;
  be.slot_free = &CtxBackend::slot_free;
  be.prefill_batch = &CtxBackend::prefill;
  be.step_batch = &CtxBackend::step;
  return qasr_batch_decode_backend(&be, segs, n, opts, events, results);
}

}  // extern "C"
