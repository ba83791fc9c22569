/*
 * qasr_b200.h — C ABI of the B200 (sm_100a) Qwen3-ASR text-decoder backend.
 *
 * This is the drop-in boundary for the reference crate's text-decoder hot path
 * (eclipse005/qwen3-asr-wgpu v0.3.0).  The reference binds that path through the
 * `TextBackend` enum (src/inference.rs:213-269) and, for batched decode, through
 * `WgpuTextDecoder::{fork_capped, set_input_token, pos}` (src/decoder.rs:2453, 1670,
 * 929), `prefill_batch` (src/decoder.rs:3599) and `BatchProjections::{new, step}`
 * (src/decoder.rs:2945, 3339).  Every entry point below names the reference call it
 * replaces.  A Rust `TextBackend::B200` variant binds these through `extern "C"`.
 *
 * Conventions
 *  - Plain C types only.  Host buffers are borrowed for the duration of the call and
 *    copied; the library owns all device memory.
 *  - f16 values travel as IEEE binary16 bit patterns in uint16_t (little endian), the
 *    same bytes the reference hands its kernels ("hidden_words", src/inference.rs:219).
 *  - Every call returns a qasr_status.  A failing call never aborts or traps; the
 *    message is available from qasr_last_error() until the next call on the context.
 *  - A context is bound to one CUDA device and must be used from one host thread at a
 *    time (the reference's decoder is likewise single-threaded behind a Mutex,
 *    src/inference.rs:303-316).  Eight GPUs = eight contexts.
 */
#ifndef QASR_B200_H
#define QASR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference maps failures to anyhow::Result / AsrError
 * (src/error.rs:1-25, src/decoder.rs:4458-4486); these are their C equivalents. */
typedef enum {
  QASR_OK = 0,
  QASR_ERR_INVALID_ARG = 1,    /* bad pointer, size, slot id or token (ensure!/bail!) */
  QASR_ERR_OOM = 2,            /* device or host allocation failed                  */
  QASR_ERR_CAPACITY = 3,       /* KV or slot capacity exceeded (max_seq, pages)     */
  QASR_ERR_DEVICE = 4,         /* CUDA runtime/driver error                          */
  QASR_ERR_DEVICE_TIMEOUT = 5, /* a bounded device-side wait gave up                 */
  QASR_ERR_CANCELLED = 6,      /* the caller asked to stop (BatchEvents::should_stop) */
  QASR_ERR_STATE = 7,          /* call order violated (e.g. step before load)        */
  QASR_ERR_NOT_DECODED = 8     /* a batch ended without a result for the item
                                  (Outcomes::finish / not_decoded, src/inference.rs:894-915) */
} qasr_status;

/* Weight storage formats of the decoder linears. */
enum {
  QASR_WEIGHTS_F16 = 0,     /* f16 [out, in] row-major, as the reference's f16 kernels read */
  QASR_WEIGHTS_INT8 = 1,    /* int8 [out, in] + f16 per-row scale: value = f16(f32(q) * s)  */
  QASR_WEIGHTS_INT8_F32 = 2 /* int8 [out, in] + f32 per-row scale, the INT8 export's own
                               `.weight_scale` (PackedInt8, src/weights.rs:309-356):
                               value = f16(f32(q) * s), the f32 product rounded to f16 */
};

/* Text decoder hyper-parameters; mirrors `TextConfig` (src/decoder.rs:166-175) with
 * the defaults of `TextDecoderConfig` (src/config.rs:102-110). */
typedef struct {
  int32_t vocab_size;          /* 151936 */
  int32_t hidden_size;         /* 1024 (0.6B) / 2048 (1.7B) */
  int32_t intermediate_size;   /* 3072 / 6144 */
  int32_t num_hidden_layers;   /* 28 */
  int32_t num_attention_heads; /* 16 */
  int32_t num_key_value_heads; /* 8 */
  int32_t head_dim;            /* 128 */
  float rms_norm_eps;          /* 1e-6, narrowed f64 -> f32 as src/decoder.rs:191 does */
} qasr_text_config;

/* Capacity plan of a context (replaces the reference's per-fork buffers,
 * src/decoder.rs:2457-2778, with one paged pool). */
typedef struct {
  int32_t weight_format;     /* QASR_WEIGHTS_F16 or QASR_WEIGHTS_INT8 */
  int32_t max_slots;         /* slot table size (reference MAX_BATCH = 32 is lifted) */
  int32_t max_seq;           /* per-slot position ceiling (rope table rows needed)   */
  int32_t kv_pages;          /* pool pages of QASR_PAGE_POSITIONS positions; 0 = max_slots*ceil(max_seq/page) */
  int32_t max_prefill_rows;  /* rows per prefill launch chunk; 0 = 4096             */
  int32_t flags;             /* QASR_FLAG_* */
} qasr_options;

#define QASR_PAGE_POSITIONS 64
/* Keep the f32 logits of the last prefill/step rows so qasr_read_logits can return
 * them (the reference's CPU decoder exposes f32 logits, src/cpu_decoder.rs:458-472). */
#define QASR_FLAG_KEEP_LOGITS 1u
/* Replay batched decode steps through a CUDA graph (default on). */
#define QASR_FLAG_NO_GRAPH 2u
/* Record per-CTA %globaltimer stamps inside the decode-chain launches of each step
 * (read with qasr_read_trace; a diagnostic like the reference's QWEN3_ASR_PROFILE
 * timings, src/decoder.rs:84-96). */
#define QASR_FLAG_TRACE 4u
#define QASR_TRACE_SLOTS 128

/* Weights of one decoder layer (HF names, src/cpu_decoder.rs:126-138).  Linear
 * weights are [out, in] row-major: q [nqh*hd, hs], k/v [nkv*hd, hs], o [hs, nqh*hd],
 * gate/up [I, hs], down [hs, I].  With QASR_WEIGHTS_INT8 each linear points at int8
 * data and its *_scale at `out` f16 scales, with QASR_WEIGHTS_INT8_F32 at `out` f32
 * scales; with QASR_WEIGHTS_F16 the *_scale fields are ignored.  Norm gains are f16
 * vectors. */
typedef struct {
  const void *q_proj, *k_proj, *v_proj, *o_proj, *gate_proj, *up_proj, *down_proj;
  const void *q_scale, *k_scale, *v_scale, *o_scale, *gate_scale, *up_scale, *down_scale;
  const uint16_t *input_layernorm, *post_attention_layernorm, *q_norm, *k_norm;
} qasr_layer_weights;

typedef struct qasr_ctx qasr_ctx;

/* --- lifetime (WgpuTextDecoder::load, src/decoder.rs:977-1573) ------------------ */
qasr_status qasr_create(const qasr_text_config* cfg, const qasr_options* opts, int device,
                        qasr_ctx** out);
void qasr_destroy(qasr_ctx* ctx);
const char* qasr_last_error(const qasr_ctx* ctx);
/* Version string of the library build. */
const char* qasr_version(void);

/* Run all device work of this context on `stream` (a cudaStream_t); NULL restores
 * the context's own stream.  Lets a caller time the hot path with its own events. */
qasr_status qasr_set_stream(qasr_ctx* ctx, void* stream);
qasr_status qasr_synchronize(qasr_ctx* ctx);

/* Tied embedding / lm_head table f16 [vocab, hidden] and the final norm gain f16
 * [hidden] (src/cpu_decoder.rs:182-192, 458-472). */
qasr_status qasr_load_embed(qasr_ctx* ctx, const uint16_t* embed, const uint16_t* final_norm);
/* One layer's weights (Layer::load src/cpu_decoder.rs:118-139; fused layout of
 * convert_layer src/decoder.rs:4366-4417).  The library fuses q|k|v and gate|up. */
qasr_status qasr_load_layer(qasr_ctx* ctx, int layer, const qasr_layer_weights* w);

/* TextBackend::set_rope_tables (src/inference.rs:263-268): f16 cos/sin, each
 * [positions, head_dim] row-major, as computed by qasr_build_rope_tables. */
qasr_status qasr_set_rope_tables(qasr_ctx* ctx, const uint16_t* cos, const uint16_t* sin,
                                 int positions);
/* TextBackend::max_seq (src/inference.rs:233-238). */
int32_t qasr_max_seq(const qasr_ctx* ctx);

/* --- slots (WgpuTextDecoder::fork_capped / pos / set_input_token) -------------- */
/* fork_capped (src/decoder.rs:2453): a new decode slot sharing the weights, with a
 * private KV of `cap` positions (rounded up to whole pages). */
qasr_status qasr_fork_capped(qasr_ctx* ctx, int cap, int* slot);
qasr_status qasr_slot_free(qasr_ctx* ctx, int slot);
/* TextBackend::ensure_capacity (src/inference.rs:242-247): grow-only; keeps the KV
 * contents (the GPU decoder's contract, src/decoder.rs:1604-1661).  Returns the new
 * capacity in *cap. */
qasr_status qasr_ensure_capacity(qasr_ctx* ctx, int slot, int need, int* cap);
/* WgpuTextDecoder::pos (src/decoder.rs:929): positions already in the slot's KV. */
qasr_status qasr_slot_pos(qasr_ctx* ctx, int slot, int* pos);
/* Set a slot's position (fill_slots sets d.pos = len, src/inference.rs:745). */
qasr_status qasr_set_slot_pos(qasr_ctx* ctx, int slot, int pos);
/* WgpuTextDecoder::set_input_token (src/decoder.rs:1670-1672): the token the next
 * step embeds.  Without it the next step embeds the slot's own last argmax. */
qasr_status qasr_set_input_token(qasr_ctx* ctx, int slot, int32_t token);

/* set_input_token for several slots at once, without a host sync: the tokens are
 * staged in pinned memory and scattered on the device ahead of the next step (the
 * per-step host->device input of a caller that feeds tokens itself). */
qasr_status qasr_set_input_tokens(qasr_ctx* ctx, const int* slots, int n, const int32_t* tokens);

/* --- the hot path ---------------------------------------------------------------- */
/* TextBackend::prefill (src/inference.rs:219-224): run `s` f16 hidden rows
 * ([s, hidden]) at positions kv_start.. through every layer into the slot's KV, then
 * return the argmax of the last row in *token. */
qasr_status qasr_prefill(qasr_ctx* ctx, int slot, const uint16_t* hidden, int s, int kv_start,
                         int32_t* token);
/* TextBackend::step (src/inference.rs:226-231): embed the slot's input token, run
 * one position, return the argmax. */
qasr_status qasr_step(qasr_ctx* ctx, int slot, int32_t* token);
/* prefill_batch (src/decoder.rs:3599-3637): several slots in one launch sequence.
 * `hidden` holds the segments' rows back to back (Σ lens rows); kv_starts may be
 * NULL (all zero).  first_tokens[i] receives segment i's argmax. */
qasr_status qasr_prefill_batch(qasr_ctx* ctx, const int* slots, int n, const uint16_t* hidden,
                               const int* lens, const int* kv_starts, int32_t* first_tokens);
/* BatchProjections::step (src/decoder.rs:3339-3510): one decode position for each
 * listed slot.  Input tokens come from qasr_set_input_token or, by default, from the
 * slot's previous argmax, read on the device (on-device feedback, src/decoder.rs:
 * 2125-2126).  If out_tokens is non-NULL the step's argmax ids are copied to it (a
 * host sync); with NULL the step is enqueued and returns at once. */
qasr_status qasr_step_batch(qasr_ctx* ctx, const int* slots, int n, int32_t* out_tokens);
/* Copy the f32 logits [rows, vocab] of the last prefill (one row per segment) or step
 * (one row per slot) — only with QASR_FLAG_KEEP_LOGITS. */
qasr_status qasr_read_logits(qasr_ctx* ctx, float* out, int rows);
/* Copy the stamps of the last decode step (QASR_FLAG_TRACE): [launch][cta][slot] uint64
 * nanoseconds, launch = chain launch index of the step (layers + 1 of them), slot 0 =
 * CTA entry, 1 + 2 i = operation i done by this CTA, 2 + 2 i = the barrier after it
 * passed (i < 12), 25 + g = GEMM g's input seen ready, 29 + g = its first MMA issued,
 * 33 + g = its last MMA issued, 37 / 38 / 39 = barriers initialised / set-up done /
 * producer ready, 64 / 65 = the first unit's weights seen / A slot free by the builders,
 * 66 = the epilogue's wait for the previous launch returned,
 * 72 + j = unit j's A operand published, 40 + j / 104 + j = the CTA's j-th unit of the launch
 * seen complete (A built, X landed) / its MMAs issued (j < 24),
 * QASR_TRACE_SLOTS - 1 = exit; 0 where nothing happened.
 * *count receives launches * ctas * slots; at most `cap` values are written. */
qasr_status qasr_read_trace(qasr_ctx* ctx, uint64_t* out, int cap, int* count);
/* Copy the attention launches' stamps of the last decode step (QASR_FLAG_TRACE):
 * [layer][cta][QASR_ATTN_TRACE_SLOTS] uint64 nanoseconds, slot 0 = CTA entry, 1 = unit
 * table ready, 2 = first stage landed, 3 = first unit merged, 4 = last stage consumed,
 * 5 = last unit merged, 6 = last page copy issued, 7 = units processed (a count).
 * *count receives layers * ctas * slots; at most `cap` values are written. */
#define QASR_ATTN_TRACE_SLOTS 8
qasr_status qasr_read_attn_trace(qasr_ctx* ctx, uint64_t* out, int cap, int* count);
/* Switch the stamps of a QASR_FLAG_TRACE context off (0) or back on (default on): the
 * steps recorded afterwards carry no trace stores, so a caller can time untraced steps
 * and take a traced pass apart.  QASR_ERR_STATE without the trace buffers. */
qasr_status qasr_set_trace(qasr_ctx* ctx, int enabled);

/* Diagnostic of the device-side error path (the reference maps device failures to an
 * Err, src/decoder.rs:4458-4486): launches one kernel on the context's stream whose two
 * bounded waits — on an mbarrier nothing arrives at, and on a device word nothing sets,
 * the wait forms the kernels use inside a CTA and across CTAs — give up after `wait_us`
 * (1..2,000,000) microseconds, exactly as a stalled kernel's waits do after 2 s.  Returns
 * what any call then returns, QASR_ERR_DEVICE_TIMEOUT with the site in
 * qasr_last_error, and clears the status so the context stays usable.  Faults nothing. */
qasr_status qasr_check_wait_timeout(qasr_ctx* ctx, uint32_t wait_us);

/* --- checkpoints (src/weights.rs, src/config.rs) -------------------------------- */
/* The decode path's part of a model directory's config.json (AsrConfig::from_file,
 * src/config.rs:142-173): `thinker_config.text_config`, or the HF-native top-level
 * `text_config`; absent fields take the reference's defaults (src/config.rs:102-124,
 * 137); `rope_parameters.rope_theta` overrides `rope_theta`; rms_norm_eps is narrowed
 * f64 -> f32 (src/decoder.rs:191).  mrope_section / mrope_interleaved follow
 * TextDecoderConfig::mrope_section / mrope_interleaved (src/config.rs:175-189). */
typedef struct {
  qasr_text_config text;
  double rope_theta;
  int32_t mrope_section[4];  /* the first n_mrope_section entries are set */
  int32_t n_mrope_section;
  int32_t mrope_interleaved;
} qasr_model_config;
qasr_status qasr_read_model_config(const char* model_dir, qasr_model_config* out, char* err, int errlen);

/* An opened checkpoint: every safetensors shard of `model_dir` memory-mapped
 * (load_tensors, src/weights.rs:150-171: model.safetensors.index.json's shards, else
 * model.safetensors), HF-native names remapped (src/weights.rs:173-201:
 * model.language_model.* -> thinker.model.*, model.audio_tower.* ->
 * thinker.audio_tower.*, model.multi_modal_projector.linear_{1,2}* ->
 * thinker.audio_tower.proj{1,2}*).  Host-only: needs no GPU. */
typedef struct qasr_checkpoint qasr_checkpoint;
qasr_status qasr_checkpoint_open(const char* model_dir, qasr_checkpoint** out, char* err, int errlen);
void qasr_checkpoint_close(qasr_checkpoint* ck);
const char* qasr_checkpoint_last_error(const qasr_checkpoint* ck);
/* Tensors in the checkpoint (after remapping). */
int64_t qasr_checkpoint_tensor_count(const qasr_checkpoint* ck);
/* dtype (safetensors name, e.g. "BF16", "I8") and shape of `name`; ndim receives the
 * rank, at most `cap` dims are written.  QASR_ERR_INVALID_ARG if absent. */
qasr_status qasr_checkpoint_tensor_info(qasr_checkpoint* ck, const char* name, char* dtype, int dtype_cap,
                                        int64_t* shape, int cap, int* ndim);
/* The weight format a context needs for `{prefix}.layers.0.self_attn.q_proj.weight`
 * (prefix NULL = "thinker.model"): QASR_WEIGHTS_INT8_F32 when it is I8 (the INT8
 * export, src/weights.rs:300-308), else QASR_WEIGHTS_F16. */
qasr_status qasr_checkpoint_weight_format(qasr_checkpoint* ck, const char* prefix, int* weight_format);
/* get_f16 (src/weights.rs:394-417): `name` as f16 (bf16 / f32 narrowed with
 * round-to-nearest-even, src/weights.rs:55-80; I8 dequantised with its
 * `<name without .weight>.weight_scale`, f16(f32(q) * s)); `count` = elements. */
qasr_status qasr_checkpoint_read_f16(qasr_checkpoint* ck, const char* name, uint16_t* out, int64_t count);
/* RawTensor::as_f32 (src/weights.rs:109-111): `name` (F16 / BF16 / F32) widened to f32
 * exactly — biases and LayerNorm parameters of the audio tower; `count` = elements. */
qasr_status qasr_checkpoint_read_f32(qasr_checkpoint* ck, const char* name, float* out, int64_t count);
/* append_f16_row_le (src/weights.rs:121-146): rows `rows[0..n)` of a 2-D `name` as f16
 * into out [n][cols] (the token-embedding lookup that builds a prefill's hidden rows). */
qasr_status qasr_checkpoint_rows_f16(qasr_checkpoint* ck, const char* name, const int32_t* rows, int n,
                                     uint16_t* out, int64_t count);
/* WgpuTextDecoder::load's weight intake (src/decoder.rs:1253-1262, 4366-4417;
 * get_matrix / get_int8 src/weights.rs:459-489): `{prefix}.embed_tokens.weight`,
 * `{prefix}.norm.weight` and every layer's norms and linears into `ctx` (prefix NULL
 * = "thinker.model").  A QASR_WEIGHTS_F16 context takes float linears narrowed to f16
 * and I8 linears dequantised; a QASR_WEIGHTS_INT8_F32 context takes I8 + F32
 * `.weight_scale` verbatim (PackedInt8 src/weights.rs:309-356: cols % 4 == 0, scale F32
 * [rows]); a QASR_WEIGHTS_INT8 context takes I8 whose scales are all f16 values.
 * Shapes are checked against the context's config. */
qasr_status qasr_load_checkpoint(qasr_ctx* ctx, qasr_checkpoint* ck, const char* prefix);

/* --- many segments through a few slots (decode_batch_embeds / run_batch_attempt,
 *     src/inference.rs:1944-2227; fill_slots :699-756; BatchEvents :823-836) -------- */
enum { QASR_STOP_EOS = 0, QASR_STOP_MAX_TOKENS = 1 }; /* StopReason, src/prompt.rs:6-12 */
#define QASR_ENDOFTEXT_TOKEN_ID 151643 /* src/prompt.rs:25 */
#define QASR_IM_END_TOKEN_ID 151645    /* src/prompt.rs:24 */

/* One segment: its prompt rows (f16 [len][hidden], e.g. built with
 * qasr_checkpoint_rows_f16 around the audio rows) and its max_new_tokens. */
typedef struct {
  const uint16_t* hidden;
  int32_t len;
  int32_t max_new_tokens;
} qasr_segment;
/* A segment's outcome.  tokens (caller-allocated, max_new_tokens entries) receives the
 * generated ids; status is QASR_OK or the error that belongs to this segment alone. */
typedef struct {
  int32_t status;
  int32_t stop_reason; /* QASR_STOP_* (status QASR_OK) */
  int32_t n_tokens;
  int32_t* tokens;
} qasr_item_result;
/* BatchEvents: on_item once per segment in completion order (longest prompt first, so
 * not input order); should_stop polled between decode steps (true: unfinished
 * segments end QASR_ERR_CANCELLED).  Either may be NULL. */
typedef struct {
  void* user;
  void (*on_item)(void* user, int index, const qasr_item_result* result);
  int (*should_stop)(void* user);
} qasr_batch_events;
typedef struct {
  int32_t width;         /* slots per attempt (--batch); halved after a failed attempt */
  int32_t eos[2];        /* {QASR_ENDOFTEXT_TOKEN_ID, QASR_IM_END_TOKEN_ID} */
  int32_t kv_step;       /* KV capacity granule (KV_STEP = 256, src/decoder.rs:725) */
  int32_t batch_seq_cap; /* segments needing more positions take the single-sequence
                            path (BATCH_SEQ_CAP = 4096, src/decoder.rs:684) */
} qasr_batch_options;
/* The decoder operations the scheduler drives (a qasr_ctx supplies them; tests supply
 * fakes).  step_batch embeds each slot's previous argmax (on-device feedback); every
 * function returns a qasr_status. */
typedef struct {
  void* user;
  int32_t hidden_size;
  int (*fork_capped)(void* user, int cap, int* slot);
  int (*slot_free)(void* user, int slot);
  int (*prefill_batch)(void* user, const int* slots, int n, const uint16_t* hidden, const int* lens,
                       int32_t* first_tokens);
  int (*step_batch)(void* user, const int* slots, int n, int32_t* out_tokens);
} qasr_decode_backend;
/* Decode every segment the way decode_batch_embeds does: segments whose
 * round_up(len + max_new + 8, kv_step) exceeds batch_seq_cap first, one at a time on
 * the single-sequence path (generate_from_embeds, src/inference.rs:2229-2376); the rest
 * in attempts of `width` slots — longest prompt first, free slots refilled from the
 * frontier in one batched prefill, a slot finishing at an eos id or when max_new_tokens
 * are generated — and, when an attempt fails, again at half the width for the segments
 * not yet finished (width < 2: the single-sequence path).  As in the reference, a
 * batched segment whose first token is an eos id ends without a result
 * (QASR_ERR_NOT_DECODED).  Returns QASR_OK once every segment has its result, or an
 * argument error. */
qasr_status qasr_batch_decode(qasr_ctx* ctx, const qasr_segment* segs, int n, const qasr_batch_options* opts,
                              const qasr_batch_events* events, qasr_item_result* results);
qasr_status qasr_batch_decode_backend(const qasr_decode_backend* backend, const qasr_segment* segs, int n,
                                      const qasr_batch_options* opts, const qasr_batch_events* events,
                                      qasr_item_result* results);

/* --- streaming session rounds (src/stream.rs:338-403) --------------------------- */
/* The decoder-facing part of one round of the reference's streaming loop.  A session
 * wraps one allocated slot.  Each round the caller passes the round's full prefill rows
 * (f16 [rows, hidden_size]: prompt embeddings, audio rows, fed-back text); with kv_reuse
 * the session prefills only the rows after the longest prefix unchanged since the
 * previous round (common_rows, src/stream.rs:366-376: those cached KV rows are what a
 * re-prefill would recompute; at most rows - 1 are reused), grows the slot to rows +
 * budget + 8 (src/stream.rs:343-349, QASR_ERR_CAPACITY past max_seq), then decodes greedily
 * until one of `eos` or `budget` tokens (src/stream.rs:380-395), and returns the tokens with
 * same-token runs longer than max_run dropped (suppress_runs, src/stream.rs:403; the run
 * may continue the fed-back text `prev_tokens`).  The reference's constants: budget 32
 * (CHUNK_MAX_NEW) on a non-final round, max_run 12 (MAX_REPEAT_RUN), eos {151643, 151645}.
 * Text assembly, rollback and the tokenizer stay with the caller.  Between rounds the
 * slot belongs to the session: prefilling, stepping, rolling back or freeing it through
 * other calls voids the reuse, which assumes its cached rows are the previous round's.
 * A session borrows its context: destroy it before the context. */
typedef struct qasr_session qasr_session;
qasr_status qasr_session_create(qasr_ctx* ctx, int slot, int kv_reuse, qasr_session** out);
void qasr_session_destroy(qasr_session* session);
/* Forget the previous round's rows, so the next round prefills all of its rows: the
 * stream's recovery step (reanchor, src/stream.rs:593-607) clears them the same way. */
void qasr_session_reset(qasr_session* session);
/* tokens: room for `budget`; reused_rows: rows taken from the previous round's KV. */
qasr_status qasr_session_round(qasr_session* session, const uint16_t* hidden, int rows, int budget,
                               const int32_t* eos, int n_eos, const uint32_t* prev_tokens, int n_prev,
                               int max_run, int32_t* tokens, int* n_tokens, int* dropped, int* hit_eos,
                               int* reused_rows);
/* common_rows (src/stream.rs:666-676): how many whole row_bytes rows a and b share at
 * their start. */
size_t qasr_common_rows(const void* a, size_t a_bytes, const void* b, size_t b_bytes, size_t row_bytes);
/* suppress_runs (src/stream.rs:702-737): kept tokens into out (room for n_next), count in
 * *n_out; returns the number dropped, -1 on a bad argument.  Host only. */
int qasr_suppress_runs(const uint32_t* prev, int n_prev, const uint32_t* next, int n_next, int max_run,
                       uint32_t* out, int* n_out);

/* --- host helpers of the reference's loader ------------------------------------ */
/* compute_mrope_cos_sin + text_positions (src/mrope.rs:46-80) rounded to f16 the
 * way src/inference.rs:1037-1047 does: angles in f64, cos/sin -> f32 -> f16.
 * `section`/`nsection` is the mrope quota ([24,20,20]); interleaved != 0 picks the
 * Qwen2-VL interleaved map (build_dim_map, src/mrope.rs:5-41). */
qasr_status qasr_build_rope_tables(uint16_t* cos, uint16_t* sin, int positions, int head_dim,
                                   double rope_theta, const int* section, int nsection,
                                   int interleaved);
/* build_dim_map (src/mrope.rs:5-41): writes `half` axis indices into out. */
qasr_status qasr_build_dim_map(const int* section, int nsection, int half, int interleaved,
                               int* out);
/* dequant_i8 (src/weights.rs:372-385): out[r, c] = f16(f32(q[r, c]) * scale_f32[r]). */
qasr_status qasr_dequant_i8(const int8_t* q, const float* scale_f32, int rows, int cols,
                            uint16_t* out);

#ifdef __cplusplus
}
#endif
#endif /* QASR_B200_H */
