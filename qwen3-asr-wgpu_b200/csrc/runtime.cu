// Host runtime of the B200 text-decoder backend: the C ABI of include/qasr_b200.h.
//
// One context = one device, one stream, one replica of the weights, one paged KV pool
// and a slot table.  The batched decode step (BatchProjections::step,
// src/decoder.rs:3339-3510) is recorded once per slot list into a CUDA graph and
// replayed; per-step state (input tokens, positions) lives in device memory, so a
// step needs no host->device traffic (on-device token feedback,
// src/decoder.rs:2125-2126).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "attention.cuh"
#include "decode_chain.cuh"
#include "f16_host.h"
#include "gemm_tc.cuh"
#include "host_gemm.cuh"
#include "qasr_b200.h"
#include "abi_guard.h"
#include "ctx_internal.h"
#include "qasr_b200_kernels.h"
#include "rows.cuh"

namespace qasr {

std::atomic<uint64_t> g_launches{0};


template <bool I8, int EPI>
static cudaError_t gemm_set_attr(int dyn) {
  return cudaFuncSetAttribute(gemm_tc_kernel<I8, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              dyn);
}

// cudaFuncSetAttribute applies to the device current when it is called, so the set-up
// runs once for every device a context or probe uses (with that device current).
cudaError_t init_kernel_attrs(std::string* err) {
  constexpr int kMaxDev = 64;
  static std::once_flag once[kMaxDev];
  static cudaError_t results[kMaxDev] = {};
  int dev = 0;
  cudaError_t de = cudaGetDevice(&dev);
  if (de == cudaSuccess && (dev < 0 || dev >= kMaxDev)) de = cudaErrorInvalidDevice;
  if (de != cudaSuccess) {
    if (err) *err = std::string("kernel attribute setup: ") + cudaGetErrorString(de);
    return de;
  }
  cudaError_t& result = results[dev];
  std::call_once(once[dev], [&result, dev] {
    cudaFuncAttributes fa{};
    result = cudaFuncGetAttributes(&fa, gemm_tc_kernel<true, EPI_QKV>);
    if (result != cudaSuccess) return;
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    g_dyn_smem_max = optin - static_cast<int>(fa.sharedSizeBytes) - 256;
    const int d = g_dyn_smem_max;
    cudaError_t e = cudaSuccess;
    e = e ? e : gemm_set_attr<false, EPI_STORE>(d);
    e = e ? e : gemm_set_attr<false, EPI_RESID>(d);
    e = e ? e : gemm_set_attr<false, EPI_SILU>(d);
    e = e ? e : gemm_set_attr<false, EPI_QKV>(d);
    e = e ? e : gemm_set_attr<false, EPI_LOGITS>(d);
    e = e ? e : gemm_set_attr<true, EPI_STORE>(d);
    e = e ? e : gemm_set_attr<true, EPI_RESID>(d);
    e = e ? e : gemm_set_attr<true, EPI_SILU>(d);
    e = e ? e : gemm_set_attr<true, EPI_QKV>(d);
    e = e ? e : cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(attn_smem_bytes(ATTN_MAX_ROWS)));
    cudaFuncAttributes fc{};
    e = e ? e : cudaFuncGetAttributes(&fc, decode_chain_kernel<CHAIN_PROG_MIDDLE, false>);
    if (e == cudaSuccess) {
      g_chain_dyn_max = optin - static_cast<int>(fc.sharedSizeBytes) - 256;
      const int cd = g_chain_dyn_max;
      const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
      e = cudaFuncSetAttribute(decode_chain_kernel<CHAIN_PROG_FIRST, false>, attr, cd);
      e = e ? e : cudaFuncSetAttribute(decode_chain_kernel<CHAIN_PROG_MIDDLE, false>, attr, cd);
      e = e ? e : cudaFuncSetAttribute(decode_chain_kernel<CHAIN_PROG_LAST, false>, attr, cd);
      e = e ? e : cudaFuncSetAttribute(decode_chain_kernel<CHAIN_PROG_FIRST, true>, attr, cd);
      e = e ? e : cudaFuncSetAttribute(decode_chain_kernel<CHAIN_PROG_MIDDLE, true>, attr, cd);
      e = e ? e : cudaFuncSetAttribute(decode_chain_kernel<CHAIN_PROG_LAST, true>, attr, cd);
    }
    result = e;
  });
  if (result != cudaSuccess && err) *err = std::string("kernel attribute setup: ") + cudaGetErrorString(result);
  return result;
}


// ----------------------------------------------------------------------------- decode chain
static_assert(CHAIN_TRACE_SLOTS == QASR_TRACE_SLOTS, "trace layout of the C ABI");
static_assert(ATTN_TRACE_SLOTS == QASR_ATTN_TRACE_SLOTS, "attention trace layout of the C ABI");
struct ChainShape {
  int n_tile, w_stages, a_stages, n_acc;
  size_t smem;
};

static ChainShape chain_shape(int rows) {
  ChainShape s{};
  s.n_tile = std::max(16, (rows + 15) / 16 * 16);
  const int dstr = (s.n_tile + 31) / 32 * 32;  // TMEM columns of one accumulator
  // MMA issuer warps (one accumulator each): a thread issues a tcgen05 instruction only
  // every ~120-230 cycles, so small-N units need several issuers
  s.n_acc = dstr <= 32 ? 3 : (dstr <= 64 ? 2 : 1);
  const int dcols = dstr * s.n_acc;
  // unit slots: one 64-column A stage in TMEM and one X tile in shared memory each
  s.a_stages = std::min(CHAIN_MAX_A_STAGES, (static_cast<int>(GEMM_TMEM_COLS) - 2 * dcols) / 64);
  // the accumulators (2 x n_acc x dstr) and at least one A stage must fit the 512 TMEM
  // columns the CTA allocates: n_acc falls as the tile widens (at most 128 rows: 2 x 128 +
  // 4 x 64 = 512)
  static_assert(2 * CHAIN_MAX_ROWS + 64 <= static_cast<int>(GEMM_TMEM_COLS), "chain TMEM budget");
  const int xstage = 2 * s.n_tile * 128;
  const int dyn = g_chain_dyn_max > 0 ? g_chain_dyn_max : 200 * 1024;
  s.w_stages = std::min(CHAIN_MAX_W_STAGES, (dyn - 1024 - s.a_stages * xstage) / 16384);
  s.smem = 1024 + static_cast<size_t>(s.w_stages) * 16384 + static_cast<size_t>(s.a_stages) * xstage;
  return s;
}

// bound on segments per tile for the chain GEMM kinds (QKV, o_proj, gate|up, down): the
// reader of each adds that many partial slots with all loads in flight
static int chain_seg_cap(int kind) {
  return kind == 0 ? CHAIN_QKV_SEG : (kind == 2 ? CHAIN_SILU_SEG : CHAIN_MAX_SEG);
}

// GEMM of the chain (units of 128 rows x 128 k; int8 or f16): at least two units per
// taking-part CTA, and few enough taking-part CTAs that no tile is cut into more than
// `max_seg_cap` segments (the bound of the operation that adds the partials).
static ChainGemm chain_gemm_plan(const uint8_t* w, const void* scale, bool scale32, int n_out, int k, int xmap,
                                 int sms, int max_seg_cap) {
  ChainGemm g{};
  g.w = w;
  g.scale = scale;
  g.scale32 = scale32 ? 1 : 0;
  g.kblocks = k / 128;
  g.units = (n_out / 128) * g.kblocks;
  for (g.grid = std::max(1, std::min(sms, g.units / 2));; --g.grid) {
    int ms = 1;
    for (int t = 0; t < n_out / 128; ++t) {
      const long long a = static_cast<long long>(t) * g.kblocks;
      ms = std::max(ms, cta_of_unit_host(a + g.kblocks - 1, g.units, g.grid) - cta_of_unit_host(a, g.units, g.grid) + 1);
    }
    g.max_seg = ms;
    if (ms <= max_seg_cap || g.grid == 1) break;
  }
  g.xmap = xmap;
  return g;
}

static cudaError_t launch_gemm(const GemmLaunch& L, cudaStream_t st, bool pdl) {
  dim3 grid(L.grid), block(gemm_threads(L.int8));
#define QASR_GEMM_CASE(I8, EPI)                                                          \
  if (L.int8 == I8 && L.epi == EPI)                                                      \
    return launch_k(gemm_tc_kernel<I8, EPI>, grid, block, L.smem, st, pdl, L.tmx, L.args);
  QASR_GEMM_CASE(false, EPI_STORE)
  QASR_GEMM_CASE(false, EPI_RESID)
  QASR_GEMM_CASE(false, EPI_SILU)
  QASR_GEMM_CASE(false, EPI_QKV)
  QASR_GEMM_CASE(false, EPI_LOGITS)
  QASR_GEMM_CASE(true, EPI_STORE)
  QASR_GEMM_CASE(true, EPI_RESID)
  QASR_GEMM_CASE(true, EPI_SILU)
  QASR_GEMM_CASE(true, EPI_QKV)
#undef QASR_GEMM_CASE
  return cudaErrorInvalidValue;
}

// Per-device workspaces shared by the probe entry points (grow-only).
struct ProbeWs {
  float* ws = nullptr;
  size_t ws_floats = 0;
  int* cnt = nullptr;
  size_t cnt_n = 0;
};

}  // namespace qasr

using namespace qasr;

// ============================================================================ context
struct LayerDev {
  Linear qkv, o, gu, down;
  float *iln = nullptr, *pln = nullptr, *qn = nullptr, *kn = nullptr;
  bool loaded = false;
};

struct SlotState {
  bool used = false;
  int cap = 0;
  int pos = 0;
  std::vector<int> pages;
};

struct qasr_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  qasr_text_config cfg{};
  qasr_options opts{};
  std::string err;
  std::vector<void*> allocs;

  std::vector<LayerDev> layers;
  Linear lm;  // tied embedding as an f16 [vocab, hs] weight (tiled, for the lm_head GEMM)
  __half* embed = nullptr;  // the same table row-major, for the token embedding gather
  float* final_norm = nullptr;
  bool embed_loaded = false;
  __half *rope_cos = nullptr, *rope_sin = nullptr;
  int rope_positions = 0;

  __half* kv_pool = nullptr;
  int kv_pages = 0, max_pages = 0;
  int* page_table = nullptr;
  std::vector<int> free_pages;
  std::vector<SlotState> slots;
  int* pos_dev = nullptr;
  int* next_tok_dev = nullptr;

  int rows_max = 0;
  __half *h = nullptr, *x = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *xf = nullptr;
  int *drow_slot = nullptr, *drow_pos = nullptr;  // decode rows (read by the step graph)
  int *prow_slot = nullptr, *prow_pos = nullptr;  // prefill rows
  int *fin_slot = nullptr, *fin_pos = nullptr, *fin_src = nullptr, *out_tok = nullptr;
  int* tok_in = nullptr;
  unsigned long long* best = nullptr;
  float* logits = nullptr;
  int logits_rows = 0;
  int last_logit_rows = 0;
  float* gemm_ws = nullptr;
  size_t gemm_ws_floats = 0;
  int* gemm_cnt = nullptr;
  size_t gemm_cnt_n = 0;
  float* attn_ws = nullptr;
  unsigned long long* attn_trace = nullptr;  // QASR_FLAG_TRACE: [L][sms][ATTN_TRACE_SLOTS]
  // decode chain (int8 weights, <= CHAIN_MAX_ROWS rows): partial sums and barrier counters
  bool chain_ok = false;
  bool chain_f16 = false;  // the chain runs the f16-weight kernels
  bool chain_pdl = false;  // per-layer chain launches start while the attention drains (PDL)
  int chain_wcap = 3;      // weight copies in flight per chain CTA (QASR_B200_CHAIN_WCAP overrides)
  uint64_t* chain_ws[4] = {};  // flagged partial sums of the chain's QKV, o_proj, gate|up, down GEMMs
  size_t chain_ws_n[4] = {};
  int chain_ws_rows = 0;
  unsigned int* chain_bar = nullptr;        // grid barrier counters, one per launch of a step
  uint64_t* chain_ss[CHAIN_CHANNELS] = {};  // flagged per-tile sums of squares [CHAIN_MAX_ROWS][CHAIN_MAX_HS / 128]
  unsigned int* step_epoch = nullptr;       // step counter of the chain's flags (finalize increments)
  int* chain_row_page = nullptr;        // [CHAIN_MAX_ROWS]
  __half* chain_row_rope = nullptr;     // [CHAIN_MAX_ROWS][256]
  unsigned long long* chain_trace = nullptr;  // QASR_FLAG_TRACE: [L + 1][sms][slots]
  bool trace_on = false;  // stamps written by the next recorded steps (qasr_set_trace)
  uint32_t* status = nullptr;
  int* pinned_tok = nullptr;  // synchronous staging
  int* pinned_in = nullptr;   // input-token staging, reusable once ev_in completed
  cudaEvent_t ev_in = nullptr;

  std::vector<int> chain_flags_for;  // slot list the chain's flagged words were last cleared for

  cudaGraphExec_t graph = nullptr;
  std::vector<int> graph_slots;
  uint64_t graph_kernels = 0;
};

namespace {

qasr_status fail(qasr_ctx* c, qasr_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return s;
}

qasr_status cuda_fail(qasr_ctx* c, cudaError_t e, const char* what) {
  return fail(c, e == cudaErrorMemoryAllocation ? QASR_ERR_OOM : QASR_ERR_DEVICE, "%s: %s", what,
              cudaGetErrorString(e));
}

#define CK(call, what)                                 \
  do {                                                 \
    cudaError_t _e = (call);                           \
    if (_e != cudaSuccess) return cuda_fail(c, _e, what); \
  } while (0)

template <class T>
qasr_status dalloc(qasr_ctx* c, T** p, size_t count, const char* what) {
  void* v = nullptr;
  const size_t bytes = std::max<size_t>(count * sizeof(T), 256);
  cudaError_t e = cudaMalloc(&v, bytes);
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  e = cudaMemset(v, 0, bytes);
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  c->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return QASR_OK;
}

void drop_graph(qasr_ctx* c) {
  if (c->graph) cudaGraphExecDestroy(c->graph);
  c->graph = nullptr;
  c->graph_slots.clear();
}

qasr_status check_device_status(qasr_ctx* c) {
  uint32_t st[2] = {0, 0};
  CK(cudaMemcpyAsync(st, c->status, sizeof st, cudaMemcpyDeviceToHost, c->stream), "status read");
  CK(cudaStreamSynchronize(c->stream), "stream sync");
  if (st[0] != 0) {
    const uint32_t zero[2] = {0, 0};
    cudaMemcpy(c->status, zero, sizeof zero, cudaMemcpyHostToDevice);
    if (st[0] == DEVERR_TIMEOUT)
      return fail(c, QASR_ERR_DEVICE_TIMEOUT, "a device-side wait timed out (site 0x%x)", st[1]);
    return fail(c, QASR_ERR_INVALID_ARG, "device-side bounds check failed (code %u, site 0x%x)",
                st[0], st[1]);
  }
  return QASR_OK;
}

// Build a launch of `lin` over activations X [rows, lin.k] (row stride ldx elements).
qasr_status plan_gemm(qasr_ctx* c, const Linear& lin, const __half* X, int ldx, int rows, int epi,
                      GemmLaunch* L) {
  const GemmShape s = gemm_shape(lin.n_out, lin.k, lin.int8, rows, c->num_sms);
  if (2ull * static_cast<unsigned long long>(s.units) * static_cast<unsigned long long>(s.grid) >= (1ull << 32))
    return fail(c, QASR_ERR_CAPACITY, "GEMM %d x %d over %d rows: too many units for 32-bit unit maps",
                lin.n_out, lin.k, rows);
  if (s.ws_floats > c->gemm_ws_floats || static_cast<size_t>(s.tiles) > c->gemm_cnt_n)
    return fail(c, QASR_ERR_CAPACITY, "GEMM workspace too small for %d x %d over %d rows",
                lin.n_out, lin.k, rows);
  if (!gemm_tmem_fits(s, lin.int8))
    return fail(c, QASR_ERR_CAPACITY, "GEMM %d x %d over %d rows: %d-column tiles need more TMEM than a CTA holds",
                lin.n_out, lin.k, rows, s.n_tile);
  if (!make_tmap(&L->tmx, X, false, static_cast<uint64_t>(lin.k), static_cast<uint64_t>(rows),
                 static_cast<uint64_t>(ldx) * 2, 64, static_cast<uint32_t>(s.n_tile), &c->err))
    return QASR_ERR_DEVICE;
  L->int8 = lin.int8;
  L->epi = epi;
  L->grid = s.grid;
  L->smem = s.smem;
  GemmArgs& a = L->args;
  a = GemmArgs{};
  a.n_out = lin.n_out;
  a.k = lin.k;
  a.rows = rows;
  a.n_tile = s.n_tile;
  a.n_tiles = s.n_tiles;
  a.kblocks = s.kblocks;
  a.units = s.units;
  a.grid = s.grid;
  a.stages = s.stages;
  a.max_seg = s.max_seg;
  a.w_tiles = static_cast<const uint8_t*>(lin.w);
  a.scale = lin.scale;
  a.scale32 = lin.scale32 ? 1 : 0;
  a.epi = epi;
  a.ws = c->gemm_ws;
  a.counters = c->gemm_cnt;
  a.status = c->status;
  a.eps = c->cfg.rms_norm_eps;
  a.kv.pool = c->kv_pool;
  a.kv.page_table = c->page_table;
  a.kv.max_pages = c->max_pages;
  a.kv.layers = c->cfg.num_hidden_layers;
  a.kv.nkv = c->cfg.num_key_value_heads;
  a.q_ld = c->cfg.num_attention_heads * c->cfg.head_dim;
  a.rope_cos = c->rope_cos;
  a.rope_sin = c->rope_sin;
  return QASR_OK;
}

qasr_status run_gemm(qasr_ctx* c, const GemmLaunch& L) {
  CK(launch_gemm(L, c->stream, true), "GEMM launch");
  return QASR_OK;
}

// attention_kernel and, behind it, attention_merge_kernel (rows cut into several chunks).
// merge_pdl: the merge launch may start while the attention drains (its CTAs then hold
// SMs until the attention completes); without, it starts once the attention is done,
// which leaves every SM the attention frees to a PDL-launched successor.
cudaError_t launch_attention_pair(const AttnArgs& a, int sms, cudaStream_t st, bool pdl, bool merge_pdl = true) {
  cudaError_t e = launch_k(attention_kernel, dim3(sms), dim3(ATTN_THREADS), attn_smem_bytes(a.rows), st, pdl, a);
  if (e != cudaSuccess) return e;
  return launch_k(attention_merge_kernel, dim3(a.rows * a.kv.nkv), dim3(256), 0, st, pdl && merge_pdl, a);
}

// `early` > 0 only where the previous launch appended exactly that many positions per
// row and wrote q, and everything else the attention reads predates it.
qasr_status launch_attention(qasr_ctx* c, int layer, int rows, const int* rs, const int* rp, int early = 0,
                             bool merge_pdl = true) {
  AttnArgs a{};
  a.q = c->q;
  a.q_ld = c->cfg.num_attention_heads * c->cfg.head_dim;
  a.out = c->attn;
  a.row_slot = rs;
  a.row_pos = rp;
  a.kv.pool = c->kv_pool;
  a.kv.page_table = c->page_table;
  a.kv.max_pages = c->max_pages;
  a.kv.layers = c->cfg.num_hidden_layers;
  a.kv.nkv = c->cfg.num_key_value_heads;
  a.layer = layer;
  a.rows = rows;
  a.scale = 1.0f / std::sqrt(static_cast<float>(c->cfg.head_dim));
  a.ws = c->attn_ws;
  a.early = early;
  a.status = c->status;
  if (c->attn_trace && c->trace_on)
    a.trace = c->attn_trace + static_cast<size_t>(layer) * c->num_sms * ATTN_TRACE_SLOTS;
  CK(launch_attention_pair(a, c->num_sms, c->stream, true, merge_pdl), "attention launch");
  return QASR_OK;
}

// All layers over `rows` rows already in c->h with row_slot/row_pos set.
qasr_status enqueue_layers(qasr_ctx* c, int rows, const int* rs, const int* rp, uint64_t* nk) {
  const int hs = c->cfg.hidden_size;
  const int qd = c->cfg.num_attention_heads * c->cfg.head_dim;
  const int I = c->cfg.intermediate_size;
  for (int l = 0; l < c->cfg.num_hidden_layers; ++l) {
    LayerDev& L = c->layers[l];
    CK(launch_k(rmsnorm_rows_kernel, dim3(rows), dim3(256), 0, c->stream, true, c->x,
                (const __half*)c->h, (const int*)nullptr, (const float*)L.iln, hs, c->cfg.rms_norm_eps),
       "rmsnorm launch");
    GemmLaunch g;
    qasr_status s = plan_gemm(c, L.qkv, c->x, hs, rows, EPI_QKV, &g);
    if (s) return s;
    g.args.qn_w = L.qn;
    g.args.kn_w = L.kn;
    g.args.q_out = c->q;
    g.args.layer = l;
    g.args.row_slot = rs;
    g.args.row_pos = rp;
    if ((s = run_gemm(c, g))) return s;
    if ((s = launch_attention(c, l, rows, rs, rp))) return s;
    if ((s = plan_gemm(c, L.o, c->attn, qd, rows, EPI_RESID, &g))) return s;
    g.args.out = c->h;
    g.args.ldo = hs;
    if ((s = run_gemm(c, g))) return s;
    CK(launch_k(rmsnorm_rows_kernel, dim3(rows), dim3(256), 0, c->stream, true, c->x,
                (const __half*)c->h, (const int*)nullptr, (const float*)L.pln, hs, c->cfg.rms_norm_eps),
       "rmsnorm launch");
    if ((s = plan_gemm(c, L.gu, c->x, hs, rows, EPI_SILU, &g))) return s;
    g.args.out = c->act;
    g.args.ldo = I;
    if ((s = run_gemm(c, g))) return s;
    if ((s = plan_gemm(c, L.down, c->act, I, rows, EPI_RESID, &g))) return s;
    g.args.out = c->h;
    g.args.ldo = hs;
    if ((s = run_gemm(c, g))) return s;
    *nk += 8;
  }
  return QASR_OK;
}

// final norm + lm_head + argmax for `n` rows: xf[i] = norm(h[src_rows[i]]).
qasr_status enqueue_head(qasr_ctx* c, int n, const int* src_rows, const int* slot_of,
                         const int* pos_of, int* out_tok, int logit_row0, uint64_t* nk,
                         bool norm = true, unsigned int* epoch = nullptr) {
  const int hs = c->cfg.hidden_size;
  if (norm) {
    CK(launch_k(rmsnorm_rows_kernel, dim3(n), dim3(256), 0, c->stream, true, c->xf, (const __half*)c->h,
                src_rows, (const float*)c->final_norm, hs, c->cfg.rms_norm_eps),
       "final norm launch");
    *nk += 1;
  }
  GemmLaunch g;
  qasr_status s = plan_gemm(c, c->lm, c->xf, hs, n, EPI_LOGITS, &g);
  if (s) return s;
  g.args.logits = (c->opts.flags & QASR_FLAG_KEEP_LOGITS)
                      ? c->logits + static_cast<size_t>(logit_row0) * c->cfg.vocab_size
                      : nullptr;
  g.args.ld_logits = c->cfg.vocab_size;
  g.args.best = c->best;
  if ((s = run_gemm(c, g))) return s;
  CK(launch_k(finalize_rows_kernel, dim3((n + 127) / 128), dim3(128), 0, c->stream, true, c->best, n,
              slot_of, pos_of, out_tok, c->next_tok_dev, c->pos_dev, epoch),
     "finalize launch");
  *nk += 2;
  return QASR_OK;
}

qasr_status enqueue_decode_chain(qasr_ctx* c, int n, uint64_t* nk);

qasr_status enqueue_decode(qasr_ctx* c, int n, uint64_t* nk) {
  if (c->chain_ok && n <= CHAIN_MAX_ROWS) return enqueue_decode_chain(c, n, nk);
  CK(launch_k(embed_rows_kernel, dim3(n), dim3(128), 0, c->stream, true, c->h, (const __half*)c->embed,
              c->cfg.hidden_size, c->cfg.vocab_size, (const int*)c->drow_slot, (const int*)c->next_tok_dev,
              (const int*)c->pos_dev, c->drow_pos, c->status),
     "embed launch");
  *nk += 1;
  qasr_status s = enqueue_layers(c, n, c->drow_slot, c->drow_pos, nk);
  if (s) return s;
  return enqueue_head(c, n, nullptr, c->drow_slot, c->drow_pos, c->out_tok, 0, nk);
}

// One cooperative launch of decode_chain_kernel (one CTA per SM).
// Whether every SM holds exactly one chain CTA with `smem` bytes (the PDL launch relies
// on it instead of the cooperative attribute's check).
static bool chain_one_cta_per_sm(size_t smem) {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, decode_chain_kernel<CHAIN_PROG_MIDDLE, false>, CHAIN_THREADS,
                                                    smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return blocks == 1;
}

// `pdl`: the previous launch is the attention merge, which this chain reads only after
// griddepcontrol.wait, so it may start while the merge drains (see decode_chain_kernel).
qasr_status launch_chain(qasr_ctx* c, const ChainArgs& a, const ChainShape& sh, int n, int prog, bool pdl = false) {
  const int hs = c->cfg.hidden_size, qd = c->cfg.num_attention_heads * c->cfg.head_dim;
  const int I = c->cfg.intermediate_size;
  CUtensorMap tx, ta, tact;
  const uint32_t box = static_cast<uint32_t>(sh.n_tile);
  const uint32_t nch = 2;  // 64-column tiles per unit (128 k)
  if (!make_tmap_chunks(&tx, c->x, hs, n, static_cast<uint64_t>(hs) * 2, box, nch, &c->err) ||
      !make_tmap_chunks(&ta, c->attn, qd, n, static_cast<uint64_t>(qd) * 2, box, nch, &c->err) ||
      !make_tmap_chunks(&tact, c->act, I, n, static_cast<uint64_t>(I) * 2, box, nch, &c->err))
    return QASR_ERR_DEVICE;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(c->num_sms);
  cfg.blockDim = dim3(CHAIN_THREADS);
  cfg.dynamicSmemBytes = sh.smem;
  cfg.stream = c->stream;
  // A cooperative launch is placed as a whole, so under PDL it could not start before
  // every SM is free.  The PDL launch is therefore a plain one: one CTA per SM (its shared
  // memory admits no second, checked at context creation), every CTA resident once the
  // attention's CTAs have exited (they never wait on this grid), and every wait on another
  // CTA (grid barriers, flagged words) is bounded in any case.
  cudaLaunchAttribute attr[1];
  const bool use_pdl = pdl && c->chain_pdl;
  if (use_pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  } else {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaErrorInvalidValue;
#define QASR_CHAIN_LAUNCH(P)                                                                    \
  (c->chain_f16 ? cudaLaunchKernelEx(&cfg, decode_chain_kernel<P, true>, tx, ta, tact, a)       \
                : cudaLaunchKernelEx(&cfg, decode_chain_kernel<P, false>, tx, ta, tact, a))
  if (prog == CHAIN_PROG_FIRST) e = QASR_CHAIN_LAUNCH(CHAIN_PROG_FIRST);
  else if (prog == CHAIN_PROG_MIDDLE)
    e = QASR_CHAIN_LAUNCH(CHAIN_PROG_MIDDLE);
  else if (prog == CHAIN_PROG_LAST) e = QASR_CHAIN_LAUNCH(CHAIN_PROG_LAST);
#undef QASR_CHAIN_LAUNCH
  CK(e, "decode chain launch");
  return QASR_OK;
}

// The decode step (int8 or f16 weights) as 1 + 3 L + 2 launches: chain (embed, norm, QKV 0), then per
// layer attention + merge + chain (o_proj ... next layer's QKV, or the final norm),
// then lm_head + argmax.
qasr_status enqueue_decode_chain(qasr_ctx* c, int n, uint64_t* nk) {
  const ChainShape sh = chain_shape(n);
  const int L = c->cfg.num_hidden_layers, hs = c->cfg.hidden_size, I = c->cfg.intermediate_size;
  const int nq = c->cfg.num_attention_heads, nkv = c->cfg.num_key_value_heads;
  const int qd = nq * c->cfg.head_dim, qkv_out = qd + 2 * nkv * 128;
  const int sms = c->num_sms;
  CK(cudaMemsetAsync(c->chain_bar, 0, static_cast<size_t>(L + 1) * sizeof(unsigned int), c->stream),
     "chain barrier reset");
  ChainArgs base{};
  base.rows = n;
  base.n_tile = sh.n_tile;
  base.w_stages = sh.w_stages;
  base.n_acc = sh.n_acc;
  base.a_stages = sh.a_stages;
  base.hs = hs;
  base.inter = I;
  base.nq = nq;
  base.nkv = nkv;
  base.eps = c->cfg.rms_norm_eps;
  base.h = c->h;
  base.q = c->q;
  base.act = c->act;
  base.embed = c->embed;
  base.vocab = c->cfg.vocab_size;
  base.row_slot = c->drow_slot;
  base.row_pos = c->drow_pos;
  base.next_tok = c->next_tok_dev;
  base.pos = c->pos_dev;
  base.rope_cos = c->rope_cos;
  base.rope_sin = c->rope_sin;
  base.row_page = c->chain_row_page;
  base.row_rope = c->chain_row_rope;
  base.kv.pool = c->kv_pool;
  base.kv.page_table = c->page_table;
  base.kv.max_pages = c->max_pages;
  base.kv.layers = L;
  base.kv.nkv = nkv;
  base.ws_rows = c->chain_ws_rows;
  for (int ch = 0; ch < CHAIN_CHANNELS; ++ch) base.ss[ch] = c->chain_ss[ch];
  base.epoch = c->step_epoch;
  base.w_inflight = c->chain_wcap;
  base.status = c->status;
  auto gemm = [&](const Linear& lin, int xmap, int kind) {
    ChainGemm g = chain_gemm_plan(static_cast<const uint8_t*>(lin.w), lin.scale, lin.scale32, lin.n_out, lin.k, xmap, sms,
                                  chain_seg_cap(kind));
    g.ws = c->chain_ws[kind];
    return g;
  };
  auto op = [](int kind, int g) {
    ChainOp o{};
    o.kind = kind;
    o.gemm = g;
    return o;
  };
  // chain 0: embed + input norm of layer 0, QKV GEMM, q/k norm + RoPE + K/V append
  {
    ChainArgs a = base;
    a.barrier = c->chain_bar;
    a.launch_idx = 0;
    a.trace = c->trace_on ? c->chain_trace : nullptr;
    const LayerDev& L0 = c->layers[0];
    a.gemms[0] = gemm(L0.qkv, 0, 0);
    a.next_first = gemm(L0.o, 1, 1);
    a.ops[0] = op(CH_EMBED_NORM, 0);
    a.ops[0].norm_w = L0.iln;
    a.ops[0].norm_out = c->x;
    a.ops[1] = op(CH_GEMM, 0);
    a.ops[2] = op(CH_QKV, 0);
    a.ops[2].qn_w = L0.qn;
    a.ops[2].kn_w = L0.kn;
    a.ops[2].layer = 0;
    a.n_ops = 3;
    qasr_status s = launch_chain(c, a, sh, n, CHAIN_PROG_FIRST);
    if (s) return s;
  }
  for (int l = 0; l < L; ++l) {
    // layer 0's row_pos comes from chain 0 (the launch just before it): no early start
    // with a programmatic chain the merge launch is not programmatic, so no merge CTA holds
    // an SM during the attention and the chain's CTAs start on the SMs the merge leaves —
    // unless the merge grid (rows x kv heads) fits beside it in one CTA per SM: then it is
    // programmatic too, and its launch latency hides under the attention (measured at one
    // row: 0.8 us less per layer)
    qasr_status s = launch_attention(c, l, n, c->drow_slot, c->drow_pos, l > 0 ? 1 : 0,
                                     !c->chain_pdl || n * c->cfg.num_key_value_heads <= c->num_sms);
    if (s) return s;
    const LayerDev& Ld = c->layers[l];
    ChainArgs a = base;
    a.barrier = c->chain_bar + l + 1;
    a.launch_idx = l + 1;
    if (c->chain_trace && c->trace_on) a.trace = c->chain_trace + static_cast<size_t>(l + 1) * sms * CHAIN_TRACE_SLOTS;
    a.gemms[0] = gemm(Ld.o, 1, 1);
    if (l + 1 < L) a.next_first = gemm(c->layers[l + 1].o, 1, 1);
    a.gemms[1] = gemm(Ld.gu, 0, 2);
    a.gemms[2] = gemm(Ld.down, 2, 3);
    int k = 0;
    a.ops[k++] = op(CH_GEMM, 0);
    a.ops[k] = op(CH_RESID, 0);
    a.ops[k++].ch = 0;
    a.ops[k] = op(CH_NORM, 0);
    a.ops[k].ch = 0;
    a.ops[k].norm_w = Ld.pln;
    a.ops[k++].norm_out = c->x;
    a.ops[k++] = op(CH_GEMM, 1);
    a.ops[k++] = op(CH_SILU, 1);
    a.ops[k++] = op(CH_GEMM, 2);
    a.ops[k] = op(CH_RESID, 2);
    a.ops[k++].ch = 1;
    a.ops[k] = op(CH_NORM, 2);
    a.ops[k].ch = 1;
    if (l + 1 < L) {
      const LayerDev& Ln = c->layers[l + 1];
      a.ops[k].norm_w = Ln.iln;
      a.ops[k++].norm_out = c->x;
      a.gemms[3] = gemm(Ln.qkv, 0, 0);
      a.ops[k++] = op(CH_GEMM, 3);
      a.ops[k] = op(CH_QKV, 3);
      a.ops[k].qn_w = Ln.qn;
      a.ops[k].kn_w = Ln.kn;
      a.ops[k++].layer = l + 1;
    } else {
      a.ops[k].norm_w = c->final_norm;
      a.ops[k++].norm_out = c->xf;
    }
    a.n_ops = k;
    if ((s = launch_chain(c, a, sh, n, l + 1 < L ? CHAIN_PROG_MIDDLE : CHAIN_PROG_LAST, true))) return s;
  }
  (void)qkv_out;
  *nk += 1 + 3 * static_cast<uint64_t>(L);  // chain 0, then per layer attention + merge + chain
  return enqueue_head(c, n, nullptr, c->drow_slot, c->drow_pos, c->out_tok, 0, nk, false, c->step_epoch);
}

qasr_status ready(qasr_ctx* c) {
  if (!c->embed_loaded) return fail(c, QASR_ERR_STATE, "embedding not loaded");
  for (size_t l = 0; l < c->layers.size(); ++l)
    if (!c->layers[l].loaded) return fail(c, QASR_ERR_STATE, "layer %zu not loaded", l);
  if (c->rope_positions <= 0) return fail(c, QASR_ERR_STATE, "rope tables not set");
  return QASR_OK;
}

qasr_status check_slot(qasr_ctx* c, int slot) {
  if (slot < 0 || slot >= static_cast<int>(c->slots.size()) || !c->slots[slot].used)
    return fail(c, QASR_ERR_INVALID_ARG, "slot %d is not allocated", slot);
  return QASR_OK;
}

qasr_status grow_slot(qasr_ctx* c, int slot, int need) {
  SlotState& S = c->slots[slot];
  if (need <= S.cap) return QASR_OK;
  if (need > c->opts.max_seq)
    return fail(c, QASR_ERR_CAPACITY, "slot %d needs %d positions, max_seq is %d", slot, need,
                c->opts.max_seq);
  const int want_pages = (need + QASR_PAGE_POSITIONS - 1) / QASR_PAGE_POSITIONS;
  const int add = want_pages - static_cast<int>(S.pages.size());
  if (add > static_cast<int>(c->free_pages.size()))
    return fail(c, QASR_ERR_CAPACITY, "KV pool exhausted: slot %d needs %d more pages, %zu free",
                slot, add, c->free_pages.size());
  for (int i = 0; i < add; ++i) {
    S.pages.push_back(c->free_pages.back());
    c->free_pages.pop_back();
  }
  S.cap = static_cast<int>(S.pages.size()) * QASR_PAGE_POSITIONS;
  CK(cudaMemcpyAsync(c->page_table + static_cast<size_t>(slot) * c->max_pages, S.pages.data(),
                     S.pages.size() * sizeof(int), cudaMemcpyHostToDevice, c->stream),
     "page table upload");
  CK(cudaStreamSynchronize(c->stream), "page table sync");
  return QASR_OK;
}

qasr_status upload_linear(qasr_ctx* c, Linear* lin, int n_out, int k, bool int8, bool scale32,
                          const std::vector<const void*>& parts, const std::vector<int>& part_rows,
                          const std::vector<const void*>& scales,
                          const std::vector<int>& row_order /* fused row -> (part,row) flat */) {
  // Fuse the parts along the output dim in `row_order` (scales in the same order) and upload.
  const size_t elem = int8 ? 1 : 2;
  const size_t selem = scale32 ? 4 : 2;
  std::vector<uint8_t> host(static_cast<size_t>(n_out) * k * elem);
  std::vector<uint8_t> host_s(int8 ? static_cast<size_t>(n_out) * selem : 0);
  std::vector<int> part_base(parts.size(), 0);
  for (size_t p = 1; p < parts.size(); ++p) part_base[p] = part_base[p - 1] + part_rows[p - 1];
  for (int r = 0; r < n_out; ++r) {
    const int src = row_order.empty() ? r : row_order[r];
    size_t p = 0;
    while (p + 1 < parts.size() && src >= part_base[p + 1]) ++p;
    const int pr = src - part_base[p];
    std::memcpy(&host[static_cast<size_t>(r) * k * elem],
                static_cast<const uint8_t*>(parts[p]) + static_cast<size_t>(pr) * k * elem, k * elem);
    if (int8) std::memcpy(&host_s[static_cast<size_t>(r) * selem], static_cast<const uint8_t*>(scales[p]) + pr * selem, selem);
  }
  if (!lin->w) {
    qasr_status s = dalloc(c, reinterpret_cast<uint8_t**>(&lin->w), host.size(), "weight alloc");
    if (s) return s;
    if (int8 && (s = dalloc(c, reinterpret_cast<uint8_t**>(&lin->scale), host_s.size(), "scale alloc"))) return s;
  } else if (int8 && lin->scale32 != scale32) {
    return fail(c, QASR_ERR_INVALID_ARG, "scale width differs from the first load of this linear");
  }
  // row-major staging copy, then the tiled HBM layout the GEMM streams
  void* staging = nullptr;
  CK(cudaMalloc(&staging, host.size()), "weight staging");
  cudaError_t e = cudaMemcpy(staging, host.data(), host.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    pack_weight_tiles_kernel<<<1024, 256>>>(static_cast<const uint4*>(staging), static_cast<uint4*>(lin->w),
                                           n_out, static_cast<int>(k * elem));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(staging);
  if (e != cudaSuccess) return cuda_fail(c, e, "weight upload");
  if (int8) CK(cudaMemcpy(lin->scale, host_s.data(), host_s.size(), cudaMemcpyHostToDevice), "scale upload");
  lin->n_out = n_out;
  lin->k = k;
  lin->int8 = int8;
  lin->scale32 = scale32;
  return QASR_OK;
}

qasr_status upload_f32_vec(qasr_ctx* c, float** dst, const uint16_t* src, int n) {
  if (!src) return fail(c, QASR_ERR_INVALID_ARG, "missing norm vector");
  std::vector<float> f(n);
  for (int i = 0; i < n; ++i) f[i] = f16_bits_to_f32(src[i]);
  if (!*dst) {
    qasr_status s = dalloc(c, dst, n, "norm alloc");
    if (s) return s;
  }
  CK(cudaMemcpy(*dst, f.data(), n * sizeof(float), cudaMemcpyHostToDevice), "norm upload");
  return QASR_OK;
}

}  // namespace

namespace qasr {
bool ctx_shape(const qasr_ctx* c, qasr_text_config* cfg, int* weight_format) {
  if (!c) return false;
  if (cfg) *cfg = c->cfg;
  if (weight_format) *weight_format = c->opts.weight_format;
  return true;
}
qasr_status ctx_fail(qasr_ctx* c, qasr_status s, const std::string& msg) {
  if (c) c->err = msg;
  return s;
}
}  // namespace qasr

// ============================================================================ C ABI
extern "C" {

const char* qasr_version(void) { return "qasr_b200 0.1.0 (sm_100a, tcgen05)"; }

const char* qasr_last_error(const qasr_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

uint64_t qasr_kernel_launch_count(void) { return g_launches.load(); }

static qasr_status create_body(const qasr_text_config* cfg, const qasr_options* opts, int device,
                               qasr_ctx** out) {
  if (!cfg || !opts || !out) return QASR_ERR_INVALID_ARG;
  *out = nullptr;
  auto* c = new qasr_ctx();
  c->cfg = *cfg;
  c->opts = *opts;
  c->device = device;
  const qasr_text_config& t = *cfg;
  auto bad = [&](const char* m) {
    fail(c, QASR_ERR_INVALID_ARG, "%s", m);
    *out = c;  // the caller reads the message, then destroys
    return QASR_ERR_INVALID_ARG;
  };
  if (t.head_dim != 128) return bad("head_dim must be 128");
  if (t.num_key_value_heads <= 0 || t.num_attention_heads != 2 * t.num_key_value_heads)
    return bad("the B200 kernels need 2 query heads per kv head (GQA rep 2)");
  if (t.hidden_size % 128 || t.intermediate_size % 128 || t.vocab_size % 128 ||
      t.hidden_size < 128 || t.vocab_size <= 0 || t.num_hidden_layers <= 0)
    return bad("hidden, intermediate and vocab sizes must be positive multiples of 128");
  if (opts->weight_format != QASR_WEIGHTS_F16 && opts->weight_format != QASR_WEIGHTS_INT8 &&
      opts->weight_format != QASR_WEIGHTS_INT8_F32)
    return bad("weight_format must be QASR_WEIGHTS_F16, QASR_WEIGHTS_INT8 or QASR_WEIGHTS_INT8_F32");
  if (opts->max_slots <= 0 || opts->max_slots > 4096 || opts->max_seq <= 0)
    return bad("max_slots must be 1..4096 and max_seq positive");
  {  // page-table entries and page ids are 32-bit: their counts, in 64-bit, must fit
    const long long mp = (static_cast<long long>(opts->max_seq) + QASR_PAGE_POSITIONS - 1) / QASR_PAGE_POSITIONS;
    const long long table = static_cast<long long>(opts->max_slots) * mp;
    if (opts->kv_pages < 0 || table > INT32_MAX)
      return bad("max_slots x max_seq / 64 pages must fit 32-bit page indices; kv_pages must not be negative");
  }
  if (c->opts.max_prefill_rows <= 0) c->opts.max_prefill_rows = 2048;
  c->opts.max_prefill_rows = std::min(c->opts.max_prefill_rows, ATTN_MAX_ROWS);
  *out = c;

  CK(cudaSetDevice(device), "cudaSetDevice");
  CK(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device), "SM count");
  int major = 0;
  CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "cc");
  if (major != 10) return fail(c, QASR_ERR_DEVICE, "device %d is not an sm_100 (B200) GPU", device);
  if (init_kernel_attrs(&c->err) != cudaSuccess) return QASR_ERR_DEVICE;
  CK(cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking), "stream create");
  c->stream = c->own_stream;

  const int L = t.num_hidden_layers, hs = t.hidden_size, I = t.intermediate_size;
  const int qd = t.num_attention_heads * t.head_dim;
  c->layers.resize(L);
  c->max_pages = (opts->max_seq + QASR_PAGE_POSITIONS - 1) / QASR_PAGE_POSITIONS;
  c->kv_pages = opts->kv_pages > 0 ? opts->kv_pages : opts->max_slots * c->max_pages;
  const size_t page_elems = static_cast<size_t>(L) * 2 * t.num_key_value_heads * 64 * 128;
  qasr_status s;
  if ((s = dalloc(c, &c->kv_pool, page_elems * c->kv_pages, "KV pool"))) return s;
  if ((s = dalloc(c, &c->page_table, static_cast<size_t>(opts->max_slots) * c->max_pages, "page table")))
    return s;
  c->free_pages.resize(c->kv_pages);
  for (int i = 0; i < c->kv_pages; ++i) c->free_pages[i] = c->kv_pages - 1 - i;
  c->slots.resize(opts->max_slots);
  if ((s = dalloc(c, &c->pos_dev, opts->max_slots, "pos"))) return s;
  if ((s = dalloc(c, &c->next_tok_dev, opts->max_slots, "tokens"))) return s;

  c->rows_max = std::max(opts->max_slots, c->opts.max_prefill_rows);
  const size_t R = c->rows_max;
  if ((s = dalloc(c, &c->h, R * hs, "h")) || (s = dalloc(c, &c->x, R * hs, "x")) ||
      (s = dalloc(c, &c->q, R * qd, "q")) || (s = dalloc(c, &c->attn, R * qd, "attn")) ||
      (s = dalloc(c, &c->act, R * I, "act")) ||
      (s = dalloc(c, &c->xf, static_cast<size_t>(opts->max_slots) * hs, "xf")) ||
      (s = dalloc(c, &c->drow_slot, opts->max_slots, "drow_slot")) ||
      (s = dalloc(c, &c->drow_pos, opts->max_slots, "drow_pos")) ||
      (s = dalloc(c, &c->prow_slot, R, "prow_slot")) || (s = dalloc(c, &c->prow_pos, R, "prow_pos")) ||
      (s = dalloc(c, &c->fin_slot, opts->max_slots, "fin_slot")) ||
      (s = dalloc(c, &c->fin_pos, opts->max_slots, "fin_pos")) ||
      (s = dalloc(c, &c->fin_src, opts->max_slots, "fin_src")) ||
      (s = dalloc(c, &c->out_tok, opts->max_slots, "out_tok")) ||
      (s = dalloc(c, &c->tok_in, 2 * static_cast<size_t>(opts->max_slots), "tok_in")) ||
      (s = dalloc(c, &c->best, opts->max_slots, "argmax keys")) ||
      (s = dalloc(c, &c->status, 4, "status")))
    return s;
  if (opts->flags & QASR_FLAG_KEEP_LOGITS) {
    c->logits_rows = opts->max_slots;
    if ((s = dalloc(c, &c->logits, static_cast<size_t>(opts->max_slots) * t.vocab_size, "logits")))
      return s;
  }
  // GEMM split workspace: worst case over every GEMM shape and row count used.
  const bool i8 = opts->weight_format != QASR_WEIGHTS_F16;
  size_t wsf = 0, cnt = 0;
  const int shapes[4][2] = {{qd + 2 * t.num_key_value_heads * 128, hs}, {hs, qd}, {2 * I, hs}, {hs, I}};
  for (int rows = 1; rows <= c->rows_max; rows = rows < 128 ? rows + 1 : rows + 128) {
    for (auto& sh : shapes) {
      const GemmShape g = gemm_shape(sh[0], sh[1], i8, rows, c->num_sms);
      wsf = std::max(wsf, g.ws_floats);
      cnt = std::max(cnt, static_cast<size_t>(g.tiles));
    }
    if (rows <= opts->max_slots) {
      const GemmShape g = gemm_shape(t.vocab_size, hs, false, rows, c->num_sms);
      wsf = std::max(wsf, g.ws_floats);
      cnt = std::max(cnt, static_cast<size_t>(g.tiles));
    }
  }
  c->gemm_ws_floats = wsf;
  c->gemm_cnt_n = cnt;
  if ((s = dalloc(c, &c->gemm_ws, std::max<size_t>(wsf, 64), "GEMM workspace")) ||
      (s = dalloc(c, &c->gemm_cnt, cnt, "GEMM counters")))
    return s;
  const size_t apart = R * t.num_key_value_heads * ATTN_ROW_CHUNKS * ATTN_PART_FLOATS;
  if ((s = dalloc(c, &c->attn_ws, apart, "attention workspace")))
    return s;
  // The decode step runs as persistent chain launches when its shapes fit them (int8 or
  // f16 weights).
  const char* no_chain = std::getenv("QASR_B200_NO_CHAIN");
  c->chain_f16 = !i8;
  c->chain_ok = hs <= CHAIN_MAX_HS && hs % (2 * CHAIN_EPI_THREADS) == 0 && I % 128 == 0 &&
                !(no_chain && no_chain[0] == '1');
  if (c->chain_ok) {
    if (const char* wc = std::getenv("QASR_B200_CHAIN_WCAP")) c->chain_wcap = std::max(1, std::atoi(wc));
    const char* no_cpdl = std::getenv("QASR_B200_NO_CHAIN_PDL");
    c->chain_pdl = pdl_enabled() && !(no_cpdl && no_cpdl[0] == '1') &&
                   chain_one_cta_per_sm(chain_shape(std::min(opts->max_slots, CHAIN_MAX_ROWS)).smem);
    c->chain_ws_rows = chain_shape(std::min(opts->max_slots, CHAIN_MAX_ROWS)).n_tile;
    for (int i = 0; i < 4; ++i) {  // shapes[] order: QKV, o_proj, gate|up, down
      const ChainGemm g = chain_gemm_plan(nullptr, nullptr, false, shapes[i][0], shapes[i][1], 0, c->num_sms,
                                          chain_seg_cap(i));
      if (2ull * static_cast<unsigned long long>(g.units) * static_cast<unsigned long long>(g.grid) >= (1ull << 32))
        return fail(c, QASR_ERR_CAPACITY, "decode chain GEMM: too many units for 32-bit unit maps");
      c->chain_ws_n[i] = static_cast<size_t>(shapes[i][0] / 128) * g.max_seg * chain_slot_words(c->chain_ws_rows);
      if ((s = dalloc(c, &c->chain_ws[i], c->chain_ws_n[i], "chain workspace"))) return s;
    }
    for (int ch = 0; ch < CHAIN_CHANNELS; ++ch)
      if ((s = dalloc(c, &c->chain_ss[ch], static_cast<size_t>(CHAIN_MAX_ROWS) * CHAIN_MAX_HS / 128, "chain norms")))
        return s;
    if ((s = dalloc(c, &c->chain_bar, static_cast<size_t>(L + 1), "chain barriers")) ||
        (s = dalloc(c, &c->step_epoch, 1, "step counter")) ||
        (s = dalloc(c, &c->chain_row_page, static_cast<size_t>(CHAIN_MAX_ROWS), "chain row pages")) ||
        (s = dalloc(c, &c->chain_row_rope, static_cast<size_t>(CHAIN_MAX_ROWS) * 256, "chain row rope")))
      return s;
    if ((opts->flags & QASR_FLAG_TRACE) &&
        ((s = dalloc(c, &c->chain_trace, static_cast<size_t>(L + 1) * c->num_sms * CHAIN_TRACE_SLOTS,
                     "chain trace")) ||
         (s = dalloc(c, &c->attn_trace, static_cast<size_t>(L) * c->num_sms * ATTN_TRACE_SLOTS,
                     "attention trace"))))
      return s;
    c->trace_on = c->chain_trace != nullptr;
  }
  CK(cudaMallocHost(&c->pinned_tok, sizeof(int) * opts->max_slots * 2), "pinned alloc");
  CK(cudaMallocHost(&c->pinned_in, sizeof(int) * opts->max_slots * 2), "pinned alloc");
  CK(cudaEventCreateWithFlags(&c->ev_in, cudaEventDisableTiming), "event create");
  return QASR_OK;
}

qasr_status qasr_create(const qasr_text_config* cfg, const qasr_options* opts, int device,
                        qasr_ctx** out) {
  // a failure after the context exists is reported on it (the caller reads, then destroys)
  return qasr::guard([&] { return create_body(cfg, opts, device, out); },
                     [&](qasr_status s, const std::string& m) { return out && *out ? qasr::ctx_fail(*out, s, m) : s; });
}

void qasr_destroy(qasr_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  drop_graph(c);
  for (void* p : c->allocs) cudaFree(p);
  if (c->pinned_tok) cudaFreeHost(c->pinned_tok);
  if (c->pinned_in) cudaFreeHost(c->pinned_in);
  if (c->ev_in) cudaEventDestroy(c->ev_in);
  if (c->own_stream) cudaStreamDestroy(c->own_stream);
  delete c;
}

qasr_status qasr_set_stream(qasr_ctx* c, void* stream) {
  if (!c) return QASR_ERR_INVALID_ARG;
  drop_graph(c);
  c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
  return QASR_OK;
}

qasr_status qasr_synchronize(qasr_ctx* c) {
  if (!c) return QASR_ERR_INVALID_ARG;
  cudaSetDevice(c->device);
  return check_device_status(c);
}

qasr_status qasr_load_embed(qasr_ctx* c, const uint16_t* embed, const uint16_t* final_norm) {
  if (!c || !embed || !final_norm) return fail(c, QASR_ERR_INVALID_ARG, "null embed/final_norm");
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  drop_graph(c);
  const int V = c->cfg.vocab_size, hs = c->cfg.hidden_size;
  qasr_status s = upload_linear(c, &c->lm, V, hs, false, false, {embed}, {V}, {}, {});
  if (s) return s;
  if (!c->embed && (s = dalloc(c, &c->embed, static_cast<size_t>(V) * hs, "embed alloc"))) return s;
  CK(cudaMemcpy(c->embed, embed, static_cast<size_t>(V) * hs * 2, cudaMemcpyHostToDevice), "embed upload");
  if ((s = upload_f32_vec(c, &c->final_norm, final_norm, hs))) return s;
  c->embed_loaded = true;
  return QASR_OK;
}

qasr_status qasr_load_layer(qasr_ctx* c, int layer, const qasr_layer_weights* w) {
  if (!c || !w) return fail(c, QASR_ERR_INVALID_ARG, "null layer weights");
  if (layer < 0 || layer >= c->cfg.num_hidden_layers)
    return fail(c, QASR_ERR_INVALID_ARG, "layer %d out of range", layer);
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  drop_graph(c);
  const bool i8 = c->opts.weight_format != QASR_WEIGHTS_F16;
  const bool s32 = c->opts.weight_format == QASR_WEIGHTS_INT8_F32;
  const int hs = c->cfg.hidden_size, I = c->cfg.intermediate_size;
  const int qd = c->cfg.num_attention_heads * c->cfg.head_dim;
  const int kvd = c->cfg.num_key_value_heads * c->cfg.head_dim;
  const void* lin[7] = {w->q_proj, w->k_proj, w->v_proj, w->o_proj, w->gate_proj, w->up_proj, w->down_proj};
  const void* sc[7] = {w->q_scale, w->k_scale, w->v_scale, w->o_scale, w->gate_scale, w->up_scale, w->down_scale};
  for (int i = 0; i < 7; ++i) {
    if (!lin[i]) return fail(c, QASR_ERR_INVALID_ARG, "layer %d: missing linear %d", layer, i);
    if (i8 && !sc[i]) return fail(c, QASR_ERR_INVALID_ARG, "layer %d: missing int8 scale %d", layer, i);
  }
  LayerDev& L = c->layers[layer];
  qasr_status s;
  // fused [q|k|v] rows (fused_pieces / fused_i8_pieces, src/decoder.rs:4243-4314)
  if ((s = upload_linear(c, &L.qkv, qd + 2 * kvd, hs, i8, s32, {lin[0], lin[1], lin[2]}, {qd, kvd, kvd},
                         {sc[0], sc[1], sc[2]}, {})))
    return s;
  if ((s = upload_linear(c, &L.o, hs, qd, i8, s32, {lin[3]}, {hs}, {sc[3]}, {}))) return s;
  // gate|up interleaved in 64-row blocks so one 128-row tile holds gate[j..j+64) and
  // up[j..j+64): the SiLU product is formed in the GEMM epilogue.
  std::vector<int> order(2 * I);
  for (int r = 0; r < 2 * I; ++r) {
    const int blk = r / 128, within = r % 128;
    order[r] = within < 64 ? blk * 64 + within : I + blk * 64 + (within - 64);
  }
  if ((s = upload_linear(c, &L.gu, 2 * I, hs, i8, s32, {lin[4], lin[5]}, {I, I}, {sc[4], sc[5]}, order)))
    return s;
  if ((s = upload_linear(c, &L.down, hs, I, i8, s32, {lin[6]}, {hs}, {sc[6]}, {}))) return s;
  if ((s = upload_f32_vec(c, &L.iln, w->input_layernorm, hs)) ||
      (s = upload_f32_vec(c, &L.pln, w->post_attention_layernorm, hs)) ||
      (s = upload_f32_vec(c, &L.qn, w->q_norm, c->cfg.head_dim)) ||
      (s = upload_f32_vec(c, &L.kn, w->k_norm, c->cfg.head_dim)))
    return s;
  L.loaded = true;
  return QASR_OK;
}

qasr_status qasr_set_rope_tables(qasr_ctx* c, const uint16_t* cos, const uint16_t* sin, int positions) {
  if (!c || !cos || !sin || positions <= 0) return fail(c, QASR_ERR_INVALID_ARG, "bad rope tables");
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  drop_graph(c);
  const size_t n = static_cast<size_t>(positions) * c->cfg.head_dim;
  if (positions > c->rope_positions) {
    qasr_status s;
    if ((s = dalloc(c, &c->rope_cos, n, "rope cos")) || (s = dalloc(c, &c->rope_sin, n, "rope sin")))
      return s;
  }
  CK(cudaMemcpy(c->rope_cos, cos, n * 2, cudaMemcpyHostToDevice), "rope upload");
  CK(cudaMemcpy(c->rope_sin, sin, n * 2, cudaMemcpyHostToDevice), "rope upload");
  c->rope_positions = positions;
  return QASR_OK;
}

int32_t qasr_max_seq(const qasr_ctx* c) { return c ? c->opts.max_seq : 0; }

qasr_status qasr_fork_capped(qasr_ctx* c, int cap, int* slot) {
  if (!c || !slot || cap <= 0) return fail(c, QASR_ERR_INVALID_ARG, "bad fork_capped arguments");
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  int id = -1;
  for (size_t i = 0; i < c->slots.size(); ++i)
    if (!c->slots[i].used) {
      id = static_cast<int>(i);
      break;
    }
  if (id < 0) return fail(c, QASR_ERR_CAPACITY, "all %zu slots are in use", c->slots.size());
  c->slots[id] = SlotState{};
  c->slots[id].used = true;
  qasr_status s = grow_slot(c, id, std::min(cap, c->opts.max_seq));
  if (s) {
    c->slots[id].used = false;
    return s;
  }
  CK(cudaMemsetAsync(c->pos_dev + id, 0, 4, c->stream), "pos reset");
  CK(cudaMemsetAsync(c->next_tok_dev + id, 0, 4, c->stream), "token reset");
  CK(cudaStreamSynchronize(c->stream), "sync");
  *slot = id;
  return QASR_OK;
}

qasr_status qasr_slot_free(qasr_ctx* c, int slot) {
  if (!c) return QASR_ERR_INVALID_ARG;
  qasr_status s = check_slot(c, slot);
  if (s) return s;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  SlotState& S = c->slots[slot];
  for (int p : S.pages) c->free_pages.push_back(p);
  S = SlotState{};
  return QASR_OK;
}

qasr_status qasr_ensure_capacity(qasr_ctx* c, int slot, int need, int* cap) {
  if (!c) return QASR_ERR_INVALID_ARG;
  qasr_status s = check_slot(c, slot);
  if (s) return s;
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  // grow-only and stepped like KV_STEP (src/decoder.rs:1604-1661); contents are kept
  const long long stepped = (static_cast<long long>(need) + 255) / 256 * 256;  // no int wrap near INT_MAX
  const int target = static_cast<int>(std::min<long long>(c->opts.max_seq, stepped));
  if ((s = grow_slot(c, slot, std::max(target, need)))) return s;
  if (cap) *cap = c->slots[slot].cap;
  return QASR_OK;
}

qasr_status qasr_slot_pos(qasr_ctx* c, int slot, int* pos) {
  if (!c || !pos) return QASR_ERR_INVALID_ARG;
  qasr_status s = check_slot(c, slot);
  if (s) return s;
  *pos = c->slots[slot].pos;
  return QASR_OK;
}

qasr_status qasr_set_slot_pos(qasr_ctx* c, int slot, int pos) {
  if (!c) return QASR_ERR_INVALID_ARG;
  qasr_status s = check_slot(c, slot);
  if (s) return s;
  if (pos < 0 || pos > c->slots[slot].cap)
    return fail(c, QASR_ERR_INVALID_ARG, "position %d outside slot capacity %d", pos, c->slots[slot].cap);
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  c->pinned_tok[0] = pos;
  CK(cudaMemcpyAsync(c->pos_dev + slot, c->pinned_tok, 4, cudaMemcpyHostToDevice, c->stream), "pos upload");
  CK(cudaStreamSynchronize(c->stream), "sync");
  c->slots[slot].pos = pos;
  return QASR_OK;
}

qasr_status qasr_set_input_token(qasr_ctx* c, int slot, int32_t token) {
  if (!c) return QASR_ERR_INVALID_ARG;
  qasr_status s = check_slot(c, slot);
  if (s) return s;
  if (token < 0 || token >= c->cfg.vocab_size)
    return fail(c, QASR_ERR_INVALID_ARG, "token %d outside the vocabulary", token);
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  c->pinned_tok[0] = token;
  CK(cudaMemcpyAsync(c->next_tok_dev + slot, c->pinned_tok, 4, cudaMemcpyHostToDevice, c->stream),
     "token upload");
  CK(cudaStreamSynchronize(c->stream), "sync");
  return QASR_OK;
}

qasr_status qasr_set_input_tokens(qasr_ctx* c, const int* slots, int n, const int32_t* tokens) {
  if (!c || n < 0 || (n > 0 && (!slots || !tokens))) return fail(c, QASR_ERR_INVALID_ARG, "bad arguments");
  if (n == 0) return QASR_OK;
  if (n > static_cast<int>(c->slots.size())) return fail(c, QASR_ERR_INVALID_ARG, "too many slots");
  for (int i = 0; i < n; ++i) {
    qasr_status s = check_slot(c, slots[i]);
    if (s) return s;
    if (tokens[i] < 0 || tokens[i] >= c->cfg.vocab_size)
      return fail(c, QASR_ERR_INVALID_ARG, "token %d outside the vocabulary", tokens[i]);
  }
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  CK(cudaEventSynchronize(c->ev_in), "staging reuse");
  std::memcpy(c->pinned_in, slots, n * sizeof(int));
  std::memcpy(c->pinned_in + c->slots.size(), tokens, n * sizeof(int));
  CK(cudaMemcpyAsync(c->tok_in, c->pinned_in + c->slots.size(), n * sizeof(int), cudaMemcpyHostToDevice,
                     c->stream),
     "token upload");
  int* slots_dev = c->tok_in + c->slots.size();
  CK(cudaMemcpyAsync(slots_dev, c->pinned_in, n * sizeof(int), cudaMemcpyHostToDevice, c->stream),
     "slot upload");
  CK(cudaEventRecord(c->ev_in, c->stream), "event record");
  scatter_tokens_kernel<<<(n + 127) / 128, 128, 0, c->stream>>>(c->next_tok_dev, slots_dev, c->tok_in, n);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  CK(cudaGetLastError(), "scatter launch");
  return QASR_OK;
}

qasr_status qasr_step_batch(qasr_ctx* c, const int* slots, int n, int32_t* out_tokens) {
  if (!c || (!slots && n > 0) || n < 0) return fail(c, QASR_ERR_INVALID_ARG, "bad step arguments");
  if (n == 0) return QASR_OK;
  qasr_status s = ready(c);
  if (s) return s;
  if (n > static_cast<int>(c->slots.size()))
    return fail(c, QASR_ERR_INVALID_ARG, "%d rows exceed max_slots", n);
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  std::vector<int> list(slots, slots + n);
  {
    std::vector<int> sorted = list;
    std::sort(sorted.begin(), sorted.end());
    if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end())
      return fail(c, QASR_ERR_INVALID_ARG, "a slot is listed twice");
  }
  for (int sl : list) {
    if ((s = check_slot(c, sl))) return s;
    const SlotState& S = c->slots[sl];
    if (S.pos >= S.cap)
      return fail(c, QASR_ERR_CAPACITY, "slot %d is full (%d positions); ensure_capacity first", sl, S.cap);
    if (S.pos >= c->rope_positions)
      return fail(c, QASR_ERR_CAPACITY, "slot %d position %d beyond the rope tables", sl, S.pos);
  }
  const bool use_graph = !(c->opts.flags & QASR_FLAG_NO_GRAPH);
  if (c->chain_ok && n <= CHAIN_MAX_ROWS && c->chain_flags_for != list) {
    // A new row set splits the GEMMs differently, so a word the new launches read may
    // have last been written long ago: start every flag from zero (never a live flag).
    for (int i = 0; i < 4; ++i)
      CK(cudaMemsetAsync(c->chain_ws[i], 0, c->chain_ws_n[i] * sizeof(uint64_t), c->stream), "flag reset");
    for (int ch = 0; ch < CHAIN_CHANNELS; ++ch)
      CK(cudaMemsetAsync(c->chain_ss[ch], 0, static_cast<size_t>(CHAIN_MAX_ROWS) * CHAIN_MAX_HS / 128 * 8, c->stream),
         "flag reset");
    c->chain_flags_for = list;
  }
  if (!use_graph || !c->graph || c->graph_slots != list) {
    drop_graph(c);
    CK(cudaMemcpyAsync(c->drow_slot, list.data(), n * sizeof(int), cudaMemcpyHostToDevice, c->stream),
       "row upload");
    if (use_graph) {
      uint64_t nk = 0;
      const uint64_t before = g_launches.load();
      CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "graph capture");
      s = enqueue_decode(c, n, &nk);
      cudaGraph_t g = nullptr;
      const cudaError_t e = cudaStreamEndCapture(c->stream, &g);
      g_launches.store(before);  // recorded, not launched
      if (s) {
        if (g) cudaGraphDestroy(g);
        return s;
      }
      if (e != cudaSuccess) return cuda_fail(c, e, "graph capture");
      const cudaError_t ie = cudaGraphInstantiate(&c->graph, g, 0);
      cudaGraphDestroy(g);
      if (ie != cudaSuccess) return cuda_fail(c, ie, "graph instantiate");
      c->graph_slots = list;
      c->graph_kernels = nk;
    }
  }
  if (use_graph) {
    CK(cudaGraphLaunch(c->graph, c->stream), "graph launch");
    g_launches.fetch_add(c->graph_kernels, std::memory_order_relaxed);
  } else {
    uint64_t nk = 0;
    if ((s = enqueue_decode(c, n, &nk))) return s;
  }
  for (int sl : list) c->slots[sl].pos += 1;
  c->last_logit_rows = n;
  if (out_tokens) {
    CK(cudaMemcpyAsync(c->pinned_tok, c->out_tok, n * sizeof(int), cudaMemcpyDeviceToHost, c->stream),
       "token readback");
    if ((s = check_device_status(c))) return s;
    std::memcpy(out_tokens, c->pinned_tok, n * sizeof(int));
  }
  return QASR_OK;
}

qasr_status qasr_step(qasr_ctx* c, int slot, int32_t* token) {
  return qasr_step_batch(c, &slot, 1, token);
}

static qasr_status prefill_batch_body(qasr_ctx* c, const int* slots, int n, const uint16_t* hidden,
                                      const int* lens, const int* kv_starts, int32_t* first_tokens) {
  if (!c || !slots || !hidden || !lens || n <= 0 || !first_tokens)
    return fail(c, QASR_ERR_INVALID_ARG, "bad prefill arguments");
  qasr_status s = ready(c);
  if (s) return s;
  if (n > static_cast<int>(c->slots.size())) return fail(c, QASR_ERR_INVALID_ARG, "too many segments");
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  std::vector<int> seen;
  long long total = 0;
  for (int i = 0; i < n; ++i) {
    if ((s = check_slot(c, slots[i]))) return s;
    const int ks = kv_starts ? kv_starts[i] : 0;
    if (lens[i] <= 0 || ks < 0) return fail(c, QASR_ERR_INVALID_ARG, "segment %d: bad length/start", i);
    const long long end = static_cast<long long>(ks) + lens[i];  // no int wrap past max_seq
    if (end > c->opts.max_seq)
      return fail(c, QASR_ERR_CAPACITY, "prefill needs %lld positions, max_seq is %d", end, c->opts.max_seq);
    if (end > c->rope_positions)
      return fail(c, QASR_ERR_CAPACITY, "prefill beyond the rope tables");
    if ((s = grow_slot(c, slots[i], ks + lens[i]))) return s;
    seen.push_back(slots[i]);
    total += lens[i];
  }
  std::sort(seen.begin(), seen.end());
  if (std::adjacent_find(seen.begin(), seen.end()) != seen.end())
    return fail(c, QASR_ERR_INVALID_ARG, "a slot is listed twice");
  const int hs = c->cfg.hidden_size;
  const int chunk = c->rows_max;
  std::vector<int> rs, rp;
  std::vector<int> seg_end;  // global row index of each segment's last row
  rs.reserve(total);
  rp.reserve(total);
  for (int i = 0; i < n; ++i) {
    const int ks = kv_starts ? kv_starts[i] : 0;
    for (int j = 0; j < lens[i]; ++j) {
      rs.push_back(slots[i]);
      rp.push_back(ks + j);
    }
    seg_end.push_back(static_cast<int>(rs.size()) - 1);
  }
  int next_seg = 0;
  for (long long r0 = 0; r0 < total; r0 += chunk) {
    const int rows = static_cast<int>(std::min<long long>(chunk, total - r0));
    CK(cudaMemcpyAsync(c->h, hidden + static_cast<size_t>(r0) * hs, static_cast<size_t>(rows) * hs * 2,
                       cudaMemcpyHostToDevice, c->stream),
       "hidden upload");
    CK(cudaMemcpyAsync(c->prow_slot, rs.data() + r0, rows * sizeof(int), cudaMemcpyHostToDevice, c->stream),
       "row upload");
    CK(cudaMemcpyAsync(c->prow_pos, rp.data() + r0, rows * sizeof(int), cudaMemcpyHostToDevice, c->stream),
       "row upload");
    uint64_t nk = 0;
    if ((s = enqueue_layers(c, rows, c->prow_slot, c->prow_pos, &nk))) return s;
    std::vector<int> fsrc, fslot, fpos;
    const int seg0 = next_seg;
    while (next_seg < n && seg_end[next_seg] < r0 + rows) {
      fsrc.push_back(static_cast<int>(seg_end[next_seg] - r0));
      fslot.push_back(slots[next_seg]);
      fpos.push_back(rp[seg_end[next_seg]]);
      ++next_seg;
    }
    if (!fsrc.empty()) {
      const int nf = static_cast<int>(fsrc.size());
      CK(cudaMemcpyAsync(c->fin_src, fsrc.data(), nf * sizeof(int), cudaMemcpyHostToDevice, c->stream), "fin upload");
      CK(cudaMemcpyAsync(c->fin_slot, fslot.data(), nf * sizeof(int), cudaMemcpyHostToDevice, c->stream), "fin upload");
      CK(cudaMemcpyAsync(c->fin_pos, fpos.data(), nf * sizeof(int), cudaMemcpyHostToDevice, c->stream), "fin upload");
      // segment i's token and logits land at row i (prefill chunks append segments)
      if ((s = enqueue_head(c, nf, c->fin_src, c->fin_slot, c->fin_pos, c->out_tok + seg0, seg0, &nk))) return s;
    }
    // the next chunk overwrites the row buffers: finish this one first
    CK(cudaStreamSynchronize(c->stream), "prefill chunk sync");
  }
  CK(cudaMemcpyAsync(c->pinned_tok, c->out_tok, n * sizeof(int), cudaMemcpyDeviceToHost, c->stream),
     "token readback");
  if ((s = check_device_status(c))) return s;
  std::memcpy(first_tokens, c->pinned_tok, n * sizeof(int));
  for (int i = 0; i < n; ++i) c->slots[slots[i]].pos = (kv_starts ? kv_starts[i] : 0) + lens[i];
  c->last_logit_rows = n;
  return QASR_OK;
}

qasr_status qasr_prefill_batch(qasr_ctx* c, const int* slots, int n, const uint16_t* hidden,
                               const int* lens, const int* kv_starts, int32_t* first_tokens) {
  return qasr::guard([&] { return prefill_batch_body(c, slots, n, hidden, lens, kv_starts, first_tokens); },
                     [&](qasr_status s, const std::string& m) { return qasr::ctx_fail(c, s, m); });
}

qasr_status qasr_prefill(qasr_ctx* c, int slot, const uint16_t* hidden, int s, int kv_start,
                         int32_t* token) {
  return qasr_prefill_batch(c, &slot, 1, hidden, &s, &kv_start, token);
}

qasr_status qasr_read_logits(qasr_ctx* c, float* out, int rows) {
  if (!c || !out) return QASR_ERR_INVALID_ARG;
  if (!(c->opts.flags & QASR_FLAG_KEEP_LOGITS) || !c->logits)
    return fail(c, QASR_ERR_STATE, "context created without QASR_FLAG_KEEP_LOGITS");
  if (rows <= 0 || rows > c->last_logit_rows)
    return fail(c, QASR_ERR_INVALID_ARG, "asked for %d logit rows, last call produced %d", rows,
                c->last_logit_rows);
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  CK(cudaMemcpyAsync(out, c->logits, static_cast<size_t>(rows) * c->cfg.vocab_size * sizeof(float),
                     cudaMemcpyDeviceToHost, c->stream),
     "logits readback");
  return check_device_status(c);
}

qasr_status qasr_read_trace(qasr_ctx* c, uint64_t* out, int cap, int* count) {
  if (!c || !out || !count || cap < 0) return QASR_ERR_INVALID_ARG;
  if (!c->chain_trace) return fail(c, QASR_ERR_STATE, "no trace: create the context with QASR_FLAG_TRACE (decode-chain steps)");
  const size_t n = static_cast<size_t>(c->cfg.num_hidden_layers + 1) * c->num_sms * CHAIN_TRACE_SLOTS;
  *count = static_cast<int>(n);
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  CK(cudaMemcpyAsync(out, c->chain_trace, std::min(n, static_cast<size_t>(cap)) * sizeof(uint64_t),
                     cudaMemcpyDeviceToHost, c->stream),
     "trace readback");
  return check_device_status(c);
}

qasr_status qasr_set_trace(qasr_ctx* c, int enabled) {
  if (!c) return QASR_ERR_INVALID_ARG;
  if (enabled && !c->chain_trace)
    return fail(c, QASR_ERR_STATE, "no trace buffers: create the context with QASR_FLAG_TRACE (decode-chain steps)");
  if (c->trace_on != (enabled != 0)) drop_graph(c);  // the recorded launches carry the trace pointers
  c->trace_on = enabled != 0;
  return QASR_OK;
}

qasr_status qasr_check_wait_timeout(qasr_ctx* c, uint32_t wait_us) {
  if (!c) return QASR_ERR_INVALID_ARG;
  if (wait_us == 0 || wait_us > 2000000u) return fail(c, QASR_ERR_INVALID_ARG, "wait_us must be 1..2000000");
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  // status[2] is never written by any kernel: the "flag that nothing sets"
  wait_timeout_probe_kernel<<<1, 32, 0, c->stream>>>(c->status + 2, static_cast<uint64_t>(wait_us) * 1000ull,
                                                      c->status);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  CK(cudaGetLastError(), "wait probe launch");
  return check_device_status(c);
}

qasr_status qasr_read_attn_trace(qasr_ctx* c, uint64_t* out, int cap, int* count) {
  if (!c || !out || !count || cap < 0) return QASR_ERR_INVALID_ARG;
  if (!c->attn_trace) return fail(c, QASR_ERR_STATE, "no trace: create the context with QASR_FLAG_TRACE (decode-chain steps)");
  const size_t n = static_cast<size_t>(c->cfg.num_hidden_layers) * c->num_sms * ATTN_TRACE_SLOTS;
  *count = static_cast<int>(n);
  CK(cudaSetDevice(c->device), "cudaSetDevice");
  CK(cudaMemcpyAsync(out, c->attn_trace, std::min(n, static_cast<size_t>(cap)) * sizeof(uint64_t),
                     cudaMemcpyDeviceToHost, c->stream),
     "trace readback");
  return check_device_status(c);
}

// ============================================================================ probes
static qasr_status probe_err(char* err, int errlen, qasr_status s, const std::string& m) {
  if (err && errlen > 0) {
    std::snprintf(err, errlen, "%s", m.c_str());
  }
  return s;
}

qasr_status qasr_kernel_gemm(int device, void* stream, int weight_format, const void* w,
                             const void* scale, int n_out, int k, const uint16_t* x, int ldx,
                             int rows, uint16_t* out, int ldo, int accumulate, char* err, int errlen) {
  return qasr_kernel_gemm_traced(device, stream, weight_format, w, scale, n_out, k, x, ldx, rows, out, ldo,
                                 accumulate, nullptr, nullptr, err, errlen);
}

qasr_status qasr_kernel_gemm_traced(int device, void* stream, int weight_format, const void* w,
                                    const void* scale, int n_out, int k, const uint16_t* x, int ldx,
                                    int rows, uint16_t* out, int ldo, int accumulate,
                                    unsigned long long* trace, int* grid_out, char* err, int errlen) {
  static std::mutex mu;
  static ProbeWs pws[16];
  std::lock_guard<std::mutex> lock(mu);
  std::string e;
  if (device < 0 || device >= 16 || !w || !x || !out || rows <= 0 || n_out <= 0 || k <= 0 || n_out % 128 ||
      k % 128 || ldx < k || ldo < n_out ||
      (weight_format != QASR_WEIGHTS_F16 && weight_format != QASR_WEIGHTS_INT8 &&
       weight_format != QASR_WEIGHTS_INT8_F32) ||
      (weight_format != QASR_WEIGHTS_F16 && !scale))
    return probe_err(err, errlen, QASR_ERR_INVALID_ARG, "bad gemm probe arguments");
  if (cudaSetDevice(device) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, "cudaSetDevice");
  if (init_kernel_attrs(&e) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, e);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const bool i8 = weight_format != QASR_WEIGHTS_F16;
  const GemmShape s = gemm_shape(n_out, k, i8, rows, sms);
  ProbeWs& P = pws[device];
  if (s.ws_floats > P.ws_floats) {
    if (P.ws) cudaFree(P.ws);
    P.ws = nullptr;
    if (cudaMalloc(&P.ws, s.ws_floats * sizeof(float)) != cudaSuccess)
      return probe_err(err, errlen, QASR_ERR_OOM, "workspace");
    P.ws_floats = s.ws_floats;
  }
  if (static_cast<size_t>(s.tiles) > P.cnt_n) {
    if (P.cnt) cudaFree(P.cnt);
    P.cnt = nullptr;
    if (cudaMalloc(&P.cnt, s.tiles * sizeof(int)) != cudaSuccess ||
        cudaMemset(P.cnt, 0, s.tiles * sizeof(int)) != cudaSuccess)
      return probe_err(err, errlen, QASR_ERR_OOM, "counters");
    P.cnt_n = s.tiles;
  }
  GemmLaunch L;
  if (!make_tmap(&L.tmx, x, false, k, rows, static_cast<uint64_t>(ldx) * 2, 64, s.n_tile, &e))
    return probe_err(err, errlen, QASR_ERR_DEVICE, e);
  L.int8 = i8;
  L.epi = accumulate ? EPI_RESID : EPI_STORE;
  L.grid = s.grid;
  L.smem = s.smem;
  GemmArgs& a = L.args;
  a.n_out = n_out;
  a.k = k;
  a.rows = rows;
  a.n_tile = s.n_tile;
  a.n_tiles = s.n_tiles;
  a.kblocks = s.kblocks;
  a.units = s.units;
  a.grid = s.grid;
  a.stages = s.stages;
  a.max_seg = s.max_seg;
  a.w_tiles = static_cast<const uint8_t*>(w);
  a.scale = scale;
  a.scale32 = weight_format == QASR_WEIGHTS_INT8_F32 ? 1 : 0;
  a.epi = L.epi;
  a.out = reinterpret_cast<__half*>(out);
  a.ldo = ldo;
  a.ws = P.ws;
  a.counters = P.cnt;
  a.trace = trace;
  if (grid_out) *grid_out = s.grid;
  const cudaError_t ce = launch_gemm(L, static_cast<cudaStream_t>(stream), false);
  if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  return QASR_OK;
}

}  // extern "C"

// The attention probes.  `check`: wait for the launches and report a device-side
// timeout or bounds error recorded in the probe's status word (the traced diagnostic);
// without it the call only enqueues (the timed probe).
static qasr_status attention_probe(int device, void* stream, const uint16_t* q, int q_ld, uint16_t* out,
                                   const uint16_t* kv_pool, const int* page_table, int max_pages, int layers,
                                   int nkv, int layer, const int* row_slot, const int* row_pos, int rows,
                                   unsigned long long* trace, bool check, char* err, int errlen) {
  static std::mutex mu;
  static ProbeWs pws[16];
  static uint32_t* status_words[16] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 16 || !q || !out || !kv_pool || !page_table || !row_slot || !row_pos ||
      rows <= 0 || nkv <= 0 || q_ld != 2 * nkv * 128 || layer < 0 || layer >= layers || max_pages <= 0)
    return probe_err(err, errlen, QASR_ERR_INVALID_ARG, "bad attention probe arguments");
  if (cudaSetDevice(device) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, "cudaSetDevice");
  const int max_chunks = ATTN_ROW_CHUNKS;
  ProbeWs& P = pws[device];
  const size_t need = static_cast<size_t>(std::min(rows, ATTN_MAX_ROWS)) * nkv * max_chunks * ATTN_PART_FLOATS;
  if (need > P.ws_floats) {
    if (P.ws) cudaFree(P.ws);
    P.ws = nullptr;
    if (cudaMalloc(&P.ws, need * sizeof(float)) != cudaSuccess)
      return probe_err(err, errlen, QASR_ERR_OOM, "attention workspace");
    P.ws_floats = need;
  }

  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  AttnArgs a{};
  a.q = reinterpret_cast<const __half*>(q);
  a.q_ld = q_ld;
  a.out = reinterpret_cast<__half*>(out);
  a.row_slot = row_slot;
  a.row_pos = row_pos;
  a.kv.pool = const_cast<__half*>(reinterpret_cast<const __half*>(kv_pool));
  a.kv.page_table = page_table;
  a.kv.max_pages = max_pages;
  a.kv.layers = layers;
  a.kv.nkv = nkv;
  a.layer = layer;
  a.rows = rows;
  a.scale = 1.0f / std::sqrt(128.0f);
  a.ws = P.ws;
  a.trace = trace;
  std::string e;
  if (init_kernel_attrs(&e) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, e);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (status_words[device] == nullptr) {
    void* p = nullptr;
    if (cudaMalloc(&p, 2 * sizeof(uint32_t)) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_OOM, "status word");
    status_words[device] = static_cast<uint32_t*>(p);
  }
  a.status = status_words[device];
  cudaError_t ce = cudaMemsetAsync(a.status, 0, 2 * sizeof(uint32_t), st);
  if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  // one launch per ATTN_MAX_ROWS rows (the unit table of a launch lives in shared memory)
  for (int r0 = 0; r0 < rows; r0 += ATTN_MAX_ROWS) {
    AttnArgs b = a;
    b.rows = std::min(ATTN_MAX_ROWS, rows - r0);
    b.q = a.q + static_cast<size_t>(r0) * q_ld;
    b.out = a.out + static_cast<size_t>(r0) * q_ld;
    b.row_slot = row_slot + r0;
    b.row_pos = row_pos + r0;
    ce = launch_attention_pair(b, sms, st, false);
    if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  }
  if (!check) return QASR_OK;
  uint32_t dev_status[2] = {0, 0};
  ce = cudaStreamSynchronize(st);
  if (ce == cudaSuccess) ce = cudaMemcpy(dev_status, a.status, sizeof dev_status, cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  if (dev_status[0] != 0) {
    char m[96];
    std::snprintf(m, sizeof m, "device-side %s (code %u, site 0x%x)",
                  dev_status[0] == DEVERR_TIMEOUT ? "wait timed out" : "check failed", dev_status[0], dev_status[1]);
    return probe_err(err, errlen, dev_status[0] == DEVERR_TIMEOUT ? QASR_ERR_DEVICE_TIMEOUT : QASR_ERR_DEVICE, m);
  }
  return QASR_OK;
}

extern "C" {

qasr_status qasr_kernel_attention(int device, void* stream, const uint16_t* q, int q_ld,
                                  uint16_t* out, const uint16_t* kv_pool, const int* page_table,
                                  int max_pages, int layers, int nkv, int layer,
                                  const int* row_slot, const int* row_pos, int rows, char* err,
                                  int errlen) {
  return attention_probe(device, stream, q, q_ld, out, kv_pool, page_table, max_pages, layers, nkv, layer,
                         row_slot, row_pos, rows, nullptr, false, err, errlen);
}

qasr_status qasr_kernel_attention_traced(int device, void* stream, const uint16_t* q, int q_ld,
                                         uint16_t* out, const uint16_t* kv_pool, const int* page_table,
                                         int max_pages, int layers, int nkv, int layer,
                                         const int* row_slot, const int* row_pos, int rows,
                                         unsigned long long* trace, char* err, int errlen) {
  return attention_probe(device, stream, q, q_ld, out, kv_pool, page_table, max_pages, layers, nkv, layer,
                         row_slot, row_pos, rows, trace, true, err, errlen);
}

}  // extern "C"

// ============================================================================ no-alloc variant
// Attention for callers that must not allocate device memory (see
// qasr_kernel_attention_noalloc in include/qasr_b200_kernels.h).  Its scratch — the
// chunk partials of the split-row merge — is this file-scope array, sized for
// NOALLOC_MAX_ROWS rows x NOALLOC_MAX_KV kv heads; the partials need no clearing between
// calls (every partial a merge reads is written by the same call).  Beside it, a status
// word (first device-side error code + site) that every call clears before its launch
// and reads back after it, so a bounded wait that gave up inside the kernels turns into
// QASR_ERR_DEVICE_TIMEOUT instead of a silent partial result.  Every GPU that loads the
// library holds both until the process exits.  In host code the array names are
// host-side stand-ins for the symbols; the device addresses come from
// cudaGetSymbolAddress, once per device.
namespace qasr {
constexpr int NOALLOC_MAX_ROWS = 64;
constexpr int NOALLOC_MAX_KV = 8;
constexpr size_t NOALLOC_SCRATCH_BYTES = static_cast<size_t>(NOALLOC_MAX_ROWS) * NOALLOC_MAX_KV *
                                         ATTN_ROW_CHUNKS * ATTN_PART_FLOATS * sizeof(float);  // ~2 MiB
}  // namespace qasr

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[qasr::NOALLOC_SCRATCH_BYTES];
static __device__ __align__(8) uint32_t g_attn_noalloc_status[2];

namespace {
constexpr int kMaxDevices = 16;
std::once_flag g_noalloc_once[kMaxDevices];
void* g_noalloc_addr[kMaxDevices] = {};
void* g_noalloc_status_addr[kMaxDevices] = {};
cudaError_t g_noalloc_setup[kMaxDevices] = {};
}  // namespace

extern "C" qasr_status qasr_kernel_attention_noalloc(int device, void* stream, const uint16_t* q,
                                                     int q_ld, uint16_t* out, const uint16_t* kv_pool,
                                                     const int* page_table, int max_pages, int layers,
                                                     int nkv, int layer, const int* row_slot,
                                                     const int* row_pos, int rows, char* err,
                                                     int errlen) {
  if (device < 0 || device >= kMaxDevices || !q || !out || !kv_pool || !page_table || !row_slot ||
      !row_pos || rows <= 0 || nkv <= 0 || q_ld != 2 * nkv * 128 || layer < 0 || layer >= layers ||
      max_pages <= 0)
    return probe_err(err, errlen, QASR_ERR_INVALID_ARG, "bad attention arguments");
  if (rows > NOALLOC_MAX_ROWS || nkv > NOALLOC_MAX_KV)
    return probe_err(err, errlen, QASR_ERR_CAPACITY,
                     "qasr_kernel_attention_noalloc handles at most 64 query rows and 8 kv heads per "
                     "call (its scratch is a fixed static array); split the rows or use "
                     "qasr_kernel_attention");
  if (cudaSetDevice(device) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, "cudaSetDevice");
  // set-up, once per device, with that device current: the array's device address
  std::call_once(g_noalloc_once[device], [device] {
    cudaError_t e = cudaGetSymbolAddress(&g_noalloc_addr[device], g_attn_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&g_noalloc_status_addr[device], g_attn_noalloc_status);
    g_noalloc_setup[device] = e;
  });
  if (g_noalloc_setup[device] != cudaSuccess || g_noalloc_addr[device] == nullptr ||
      g_noalloc_status_addr[device] == nullptr)
    return probe_err(err, errlen, QASR_ERR_DEVICE,
                     std::string("cudaGetSymbolAddress of the static attention scratch failed: ") +
                         cudaGetErrorString(g_noalloc_setup[device]));
  std::string e;
  if (init_kernel_attrs(&e) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, e);
  float* partials = static_cast<float*>(g_noalloc_addr[device]);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  AttnArgs a{};
  a.q = reinterpret_cast<const __half*>(q);
  a.q_ld = q_ld;
  a.out = reinterpret_cast<__half*>(out);
  a.row_slot = row_slot;
  a.row_pos = row_pos;
  a.kv.pool = const_cast<__half*>(reinterpret_cast<const __half*>(kv_pool));
  a.kv.page_table = page_table;
  a.kv.max_pages = max_pages;
  a.kv.layers = layers;
  a.kv.nkv = nkv;
  a.layer = layer;
  a.rows = rows;
  a.scale = 1.0f / std::sqrt(128.0f);
  a.ws = partials;
  uint32_t* status = static_cast<uint32_t*>(g_noalloc_status_addr[device]);
  a.status = status;
  cudaError_t ce = cudaMemsetAsync(status, 0, 2 * sizeof(uint32_t), st);
  if (ce == cudaSuccess) ce = launch_attention_pair(a, sms, st, false);
  if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  // the call completes before it returns, so its result code covers what happened on the
  // device: a bounded wait that gave up is reported, never an OK with partial output
  uint32_t dev_status[2] = {0, 0};
  ce = cudaStreamSynchronize(st);
  if (ce == cudaSuccess) ce = cudaMemcpy(dev_status, status, sizeof dev_status, cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  if (dev_status[0] == DEVERR_TIMEOUT) {
    char m[96];
    std::snprintf(m, sizeof m, "a device-side wait timed out (site 0x%x)", dev_status[1]);
    return probe_err(err, errlen, QASR_ERR_DEVICE_TIMEOUT, m);
  }
  if (dev_status[0] != 0) {
    char m[96];
    std::snprintf(m, sizeof m, "device-side check failed (code %u, site 0x%x)", dev_status[0], dev_status[1]);
    return probe_err(err, errlen, QASR_ERR_DEVICE, m);
  }
  return QASR_OK;
}

namespace qasr {
__global__ void kv_append_kernel(const __half* __restrict__ k, const __half* __restrict__ v,
                                 KvLayout kv, int layer, const int* __restrict__ row_slot,
                                 const int* __restrict__ row_pos) {
  const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int ld = kv.nkv * 128;
  const size_t ko = kv_elem_offset(kv, row_slot[r], row_pos[r], layer, 0, h);
  const size_t vo = kv_elem_offset(kv, row_slot[r], row_pos[r], layer, 1, h);
  const int sd = kv_dim_swizzle(row_pos[r], d);
  kv.pool[ko + sd] = k[static_cast<size_t>(r) * ld + h * 128 + d];
  kv.pool[vo + sd] = v[static_cast<size_t>(r) * ld + h * 128 + d];
}
}  // namespace qasr

extern "C" qasr_status qasr_kernel_pack_weights(int device, void* stream, int weight_format,
                                                const void* w_rowmajor, int n_out, int k, void* w_tiled,
                                                char* err, int errlen) {
  if (!w_rowmajor || !w_tiled || n_out <= 0 || n_out % 128 || k <= 0 || k % 128)
    return probe_err(err, errlen, QASR_ERR_INVALID_ARG, "bad pack arguments");
  if (cudaSetDevice(device) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, "cudaSetDevice");
  const int row_bytes = k * (weight_format != QASR_WEIGHTS_F16 ? 1 : 2);
  pack_weight_tiles_kernel<<<1024, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(w_rowmajor), static_cast<uint4*>(w_tiled), n_out, row_bytes);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  return QASR_OK;
}

extern "C" qasr_status qasr_kernel_kv_append(int device, void* stream, const uint16_t* k,
                                             const uint16_t* v, uint16_t* kv_pool,
                                             const int* page_table, int max_pages, int layers,
                                             int nkv, int layer, const int* row_slot,
                                             const int* row_pos, int rows, char* err, int errlen) {
  if (!k || !v || !kv_pool || !page_table || !row_slot || !row_pos || rows <= 0 || nkv <= 0 ||
      layer < 0 || layer >= layers || max_pages <= 0)
    return probe_err(err, errlen, QASR_ERR_INVALID_ARG, "bad kv append arguments");
  if (cudaSetDevice(device) != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, "cudaSetDevice");
  KvLayout kv{reinterpret_cast<__half*>(kv_pool), page_table, max_pages, layers, nkv};
  kv_append_kernel<<<dim3(rows, nkv), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __half*>(k), reinterpret_cast<const __half*>(v), kv, layer, row_slot, row_pos);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return probe_err(err, errlen, QASR_ERR_DEVICE, cudaGetErrorString(ce));
  return QASR_OK;
}
