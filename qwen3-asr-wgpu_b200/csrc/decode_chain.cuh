// The decode step between two attention launches as ONE persistent kernel.
//
// One launch runs a short program of operations over the step's decode rows, e.g.
//   o_proj GEMM -> residual + post-attention RMSNorm -> gate|up GEMM -> SiLU ->
//   down GEMM -> residual + next layer's input RMSNorm -> next layer's QKV GEMM ->
//   q/k RMSNorm + RoPE + paged K/V append
// which is what CpuTextDecoder::forward_layer (src/cpu_decoder.rs:367-455) does between
// two attention calls; the per-kernel path of this library launches those as 7 kernels.
// One CTA per SM (all CTAs resident: a cooperative launch, or a plain launch of one CTA
// per SM whose residency the host checks).
//
// GEMM operations are the tcgen05 weight-streaming GEMM of gemm_tc.cuh in stream-K form,
// but every (tile, CTA) segment stores its f32 partial sums to a workspace and the NEXT
// operation adds the partials in segment order while it builds its own input (residual
// add, SiLU, q/k norm): no CTA finishes another's tile, so no tile fix-up sits on the
// critical path.  The weights of later GEMMs do not depend on anything computed in the
// launch, so the weight producer and the int8 dequantising builders run ahead into the
// next GEMM's units as far as their rings allow.
//
// Hand-offs between CTAs.  The partial sums and the per-tile sums of squares of the
// residual stream travel as 8-byte words {32-bit value, 32-bit flag} written with one store
// (the layout of NCCL's LL protocol): the flag is this launch's epoch, so the reader polls
// exactly the words it needs and no barrier or fence stands between a GEMM and the
// operation that consumes its partials, or between a residual add and its RMSNorm.  (A
// gpu-scope release, the heart of a grid barrier, waits for this SM's weight copies in
// flight: ~0.3 us idle, ~1.5 us with 12 x 16 KB in flight, measured.)  The epoch is
// (step counter << 6) | (launch index + 1); the step counter is a device word the step's
// last kernel increments.  The activation tile of a GEMM (its MMA B operand) is copied by
// TMA from global memory, which every CTA reads at once; a grid barrier still precedes
// those copies (three per launch instead of nine): TMA-fed tiles measured far faster than
// tiles built from flagged words with ordinary loads (every CTA reading the same freshly
// written rows with 16-byte loads took ~10 us per batch of three tiles).
//
// Roles (512 threads):
//   warp 0      producer: 16 KB bulk copy per weight unit into the W ring, and the TMA of
//               each unit's X tile once its GEMM's input is ready
//   warps 1-3   UMMA issuers (int8 weights: A from TMEM; f16 weights: A straight from the
//               W ring), B = X from shared memory, units dealt round-robin over them;
//               warp 2 also allocates the TMEM
//   warps 4-7   int8 A builders: f16(q * s) into TMEM (idle with f16 weights)
//
// Weight formats (template parameter F16): a unit is 128 output rows x 128 k, its weights
// one 16 KB tile of the tiled layout (weight_tile_offset) in int8, two consecutive tiles
// (64 k each) in f16; either way its activation tile is 128 k.
//   warps 8-15  epilogue (two warps per TMEM lane quadrant, splitting the accumulator
//               columns) and row operations; they also run the grid barriers
#pragma once
#include "device_common.cuh"
#include "gemm_tc.cuh"

namespace qasr {

constexpr int CHAIN_MAX_OPS = 12;
constexpr int CHAIN_MAX_GEMMS = 4;
constexpr int CHAIN_THREADS = 512;
constexpr int CHAIN_MAX_W_STAGES = 12;
constexpr int CHAIN_MAX_A_STAGES = 8;
constexpr int CHAIN_MAX_ROWS = 128;  // one N tile
constexpr int CHAIN_TRACE_SLOTS = 128;  // == QASR_TRACE_SLOTS
constexpr int CHAIN_MAX_HS = 2048;   // hidden size the row operations hold in registers
// warps 8-15 run the epilogue and the row operations (two per TMEM lane quadrant), warps
// 4-7 dequantise: one builder warpgroup keeps pace with the MMA issuers
constexpr int CHAIN_EPI_WARPS = 8;
constexpr int CHAIN_EPI_THREADS = CHAIN_EPI_WARPS * 32;
// most segments a tile of a chain GEMM may be cut into, per reader (all loads of a read are
// issued at once): residual adds (o_proj, down), SiLU (gate|up), q/k/v (QKV)
constexpr int CHAIN_MAX_SEG = 12;
constexpr int CHAIN_SILU_SEG = 4;
constexpr int CHAIN_QKV_SEG = 8;
constexpr int CHAIN_CHANNELS = 2;  // flagged sums of squares: one per residual add of a launch
// padding (in 8-byte words) of each partial-sum slot, so that the segments of a tile are
// not a power of two apart
constexpr int CHAIN_ROW_PAD = 16;
// words of one partial-sum slot (one (tile, segment) of a chain GEMM: ws_rows rows x 128)
__host__ __device__ constexpr size_t chain_slot_words(int ws_rows) {
  return static_cast<size_t>(ws_rows) * 128 + CHAIN_ROW_PAD;
}
// the launch programs (the op lists the host fills ChainArgs::ops with, in this order)
enum ChainProgram : int {
  CHAIN_PROG_FIRST = 0,   // EMBED_NORM | GEMM (QKV of layer 0) | QKV
  CHAIN_PROG_MIDDLE = 1,  // GEMM (o) | RESID | NORM | GEMM (gate|up) | SILU | GEMM (down) | RESID |
                          // NORM | GEMM (next QKV) | QKV
  CHAIN_PROG_LAST = 2,    // as MIDDLE up to the second NORM (the final norm)
};

enum ChainOpKind : int {
  CH_GEMM = 0,        // partial sums of W x over this CTA's (tile, k-block) range
  CH_EMBED_NORM = 1,  // h[r] = embed[next_tok[slot_r]], row_pos[r] = pos[slot_r]; x = rmsnorm(h)
  CH_RESID = 2,       // h = f16(h + sum of the GEMM's partials); per-tile sums of squares (channel ch)
  CH_NORM = 3,        // x = rmsnorm(h) from those sums (channel ch)
  CH_SILU = 4,        // act = f16(silu(f16 gate) * f16 up) from the gate|up GEMM's partials
  CH_QKV = 5,         // q/k RMSNorm + RoPE -> q and paged K; raw V -> paged V
};

struct ChainGemm {
  const uint8_t* w;     // int8 weights in the tiled layout (weight_tile_offset)
  const void* scale;    // per-row scales: f16, or f32 when scale32
  int scale32;
  int kblocks;          // K / 128
  int units;            // (n_out / 128) * kblocks
  int grid;             // CTAs that take part: the first `grid` of the launch
  int max_seg;          // most segments (CTAs) any tile is cut into
  int xmap;             // X source: 0 = normalised rows, 1 = attention output, 2 = act
  uint64_t* ws;         // this GEMM's flagged partial sums: [tile][max_seg] slots of
                        // chain_slot_words(ws_rows) words, [ws_rows][128] {f32, flag} each
};

struct ChainOp {
  int kind;
  int gemm;             // CH_GEMM: index into gemms; row ops: the GEMM whose partials they add
  const float* norm_w;  // *_NORM: RMSNorm gain
  __half* norm_out;     // *_NORM: normalised rows [rows][hs]
  const float* qn_w;    // CH_QKV: q / k RMSNorm gains
  const float* kn_w;
  int layer;            // CH_QKV: KV-cache layer
  int ch;               // CH_RESID / CH_NORM: channel of the flagged sums of squares
};

struct ChainArgs {
  ChainOp ops[CHAIN_MAX_OPS];
  ChainGemm gemms[CHAIN_MAX_GEMMS];
  int n_ops;
  int rows, n_tile;
  int w_stages, a_stages;  // weight stages; unit slots (A stage in TMEM + X tile in smem)
  int w_inflight;          // most weight copies in flight at once (0: the W ring's depth)
  int n_acc;  // MMA issuer warps = accumulators per segment buffer (1 to 3)
  ChainGemm next_first;  // the next chain launch's first GEMM (w == nullptr: none): its
                         // units of this CTA are prefetched into L2 once this launch's
                         // weights are all issued, so they are resident when it starts
  int hs, inter, nq, nkv;
  float eps;
  __half* h;    // [rows][hs] residual stream
  __half* q;    // [rows][nq * 128]
  __half* act;  // [rows][inter]
  const __half* embed;
  int vocab;
  const int* row_slot;
  int* row_pos;
  const int* next_tok;
  const int* pos;
  const __half* rope_cos;
  const __half* rope_sin;
  // per decode row, filled by CH_EMBED_NORM so CH_QKV's loads do not chain: the KV page of
  // the row's position, and its RoPE cos | sin rows [rows][256]
  int* row_page;
  __half* row_rope;
  KvLayout kv;
  int ws_rows;               // rows per partial slot (fixed for the context, >= n_tile)
  uint64_t* ss[CHAIN_CHANNELS];  // flagged per-tile sums of squares of h [rows][CHAIN_MAX_HS / 128]
  const unsigned int* epoch;     // the step counter (incremented by the step's last kernel)
  int launch_idx;                // this launch's index in the step (< 63)
  unsigned int* barrier;     // grid barrier counter, zero at launch
  uint32_t* status;
  unsigned long long* trace;  // optional: per CTA CHAIN_TRACE_SLOTS %globaltimer stamps: 0 entry,
                              // 1 + 2 i op i done, 2 + 2 i barrier after op i passed (i < 12),
                              // 25 + g GEMM g's input seen ready, 29 + g its first MMA issued,
                              // 33 + g its last MMA issued, 37 / 38 / 39 barriers initialised /
                              // set-up done / producer ready, 64 / 65 the first unit's W seen /
                              // A slot free (builder warp 4), 66 the epilogue's wait for the
                              // previous launch returned, 72 + j unit j's A published,
                              // 40 + j / 104 + j the CTA's j-th
                              // unit of the launch seen complete / its MMAs issued (j < 24),
                              // 127 exit
};

__device__ __forceinline__ void chain_unit_range(const ChainGemm& g, int cta, int& ub, int& ue) {
  if (cta >= g.grid) {
    ub = ue = 0;
    return;
  }
  // 32-bit unsigned arithmetic (cta * units < 2^32: chain_gemm_plan bounds units); a
  // 64-bit division here is a software routine that delayed every CTA's first copy
  const unsigned int u = static_cast<unsigned int>(g.units), gr = static_cast<unsigned int>(g.grid);
  ub = static_cast<int>(static_cast<unsigned int>(cta) * u / gr);
  ue = static_cast<int>(static_cast<unsigned int>(cta + 1) * u / gr);
}

// non-blocking test of an mbarrier phase
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ unsigned int ld_relaxed_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_cta_shared(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta_shared(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// ---------------------------------------------------------------- flagged words
// {data, flag} pairs, two per 16 bytes; each 8-byte half is written by one store and read
// by one load, so a reader that sees its flag sees the data written with it.
__device__ __forceinline__ uint4 ll_ld16(const uint64_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint2 ll_ld8(const uint64_t* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ll_st16(uint64_t* p, uint32_t d0, uint32_t d1, uint32_t flag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(d0), "r"(flag), "r"(d1), "r"(flag)
               : "memory");
}
__device__ __forceinline__ void ll_st8(uint64_t* p, uint32_t d, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(d), "r"(flag) : "memory");
}

// Bounded polls of flagged words (the data's producer is another CTA of this launch).
// They return the last word read; on a timeout the error is recorded and the CTA's abort
// flag set (a caller tells success by the flags of the returned word).
struct LLWait {
  volatile int* abort_flag;
  uint32_t* status;
  uint32_t flag;
};
__device__ __forceinline__ uint2 ll_spin8(const uint64_t* p, LLWait w, uint32_t site) {
  const uint64_t t0 = globaltimer();
  while (true) {
    const uint2 v = ll_ld8(p);
    if (v.y == w.flag || *w.abort_flag) return v;
    if (globaltimer() - t0 > QASR_WAIT_NS) {
      report_error(w.status, DEVERR_TIMEOUT, site);
      *w.abort_flag = 1;
      return v;
    }
  }
}
// N 16-byte words at p + s * stride + h * 2 (s < n, h < H): loaded until every one carries
// the flag.  Every round re-issues the loads of all the words not yet ready, so they are in
// flight together: a round costs one L2 round trip however many producers are late.
template <int N, int H>
__device__ __forceinline__ bool ll_poll(const uint64_t* p, size_t stride, int n, uint4 (&v)[N * H], const LLWait& w,
                                        uint32_t site) {
  auto ready = [&](const uint4& x) { return x.y == w.flag && x.w == w.flag; };
#pragma unroll
  for (int k = 0; k < N * H; ++k)
    if (k / H < n) v[k] = ll_ld16(p + (k / H) * stride + (k % H) * 2);
  uint64_t t0 = 0;
  while (true) {
    bool all = true;
#pragma unroll
    for (int k = 0; k < N * H; ++k)
      if (k / H < n) all = all && ready(v[k]);
    if (all) return true;
    if (*w.abort_flag) return false;
    const uint64_t now = globaltimer();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > QASR_WAIT_NS) {
      report_error(w.status, DEVERR_TIMEOUT, site);
      *w.abort_flag = 1;
      return false;
    }
#pragma unroll
    for (int k = 0; k < N * H; ++k)
      if (k / H < n && !ready(v[k])) v[k] = ll_ld16(p + (k / H) * stride + (k % H) * 2);
  }
}

// Partials of (tile t, row n, columns m, m + 1): segment s at chain_partial(...) + s * chain_slot_words.
__device__ __forceinline__ const uint64_t* chain_partial(const ChainArgs& a, const ChainGemm& g, int t, int n,
                                                         int m) {
  return g.ws + static_cast<size_t>(t) * g.max_seg * chain_slot_words(a.ws_rows) + static_cast<size_t>(n) * 128 + m;
}
// Segments tile t of g is cut into (CTAs that own some of its units).
__device__ __forceinline__ int chain_tile_segs(const ChainGemm& g, int t) {
  const long long a0 = static_cast<long long>(t) * g.kblocks;
  return cta_of_unit(a0 + g.kblocks - 1, g.units, g.grid) - cta_of_unit(a0, g.units, g.grid) + 1;
}
// Sum, in segment order, of the flagged partials of 4 consecutive columns of one row:
// `nseg` segments (at most MAXSEG), two 16-byte words each.  SPLIT: the words of the first
// two columns, then those of the last two (at most MAXSEG words in flight, half the
// registers, one more round trip); otherwise all 2 * nseg words at once.
template <int MAXSEG, bool SPLIT = (MAXSEG > 4)>
__device__ __forceinline__ bool chain_sum4(const uint64_t* p, size_t stride, int nseg, float4& acc, const LLWait& w,
                                          uint32_t site) {
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
  bool ok;
  if constexpr (SPLIT) {
    uint4 v[MAXSEG];
    ok = ll_poll<MAXSEG, 1>(p, stride, nseg, v, w, site);
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s)
      if (s < nseg) {
        acc.x += __uint_as_float(v[s].x);
        acc.y += __uint_as_float(v[s].z);
      }
    ok = ll_poll<MAXSEG, 1>(p + 2, stride, nseg, v, w, site) && ok;
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s)
      if (s < nseg) {
        acc.z += __uint_as_float(v[s].x);
        acc.w += __uint_as_float(v[s].z);
      }
  } else {
    uint4 v[2 * MAXSEG];  // segment s: v[2 s] columns 0-1, v[2 s + 1] columns 2-3
    ok = ll_poll<MAXSEG, 2>(p, stride, nseg, v, w, site);
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s)
      if (s < nseg) {
        acc.x += __uint_as_float(v[2 * s].x);
        acc.y += __uint_as_float(v[2 * s].z);
        acc.z += __uint_as_float(v[2 * s + 1].x);
        acc.w += __uint_as_float(v[2 * s + 1].z);
      }
  }
  return ok;
}

// SiLU's read of a gate|up tile: the gate partials of 4 columns (two words at p) and the
// up partials (two words at p + 64) of `nseg` segments, every word polled together.
__device__ __forceinline__ bool chain_sum_gate_up(const uint64_t* p, size_t stride, int nseg, float4& gs, float4& us,
                                                  const LLWait& w, uint32_t site) {
  constexpr int S = CHAIN_SILU_SEG;
  uint4 v[4 * S];  // segment s: v[4 s + 0..1] gate, v[4 s + 2..3] up
  auto addr = [&](int k) { return p + (k >> 2) * stride + ((k & 2) ? 64 : 0) + (k & 1) * 2; };
  auto ready = [&](const uint4& x) { return x.y == w.flag && x.w == w.flag; };
#pragma unroll
  for (int k = 0; k < 4 * S; ++k)
    if ((k >> 2) < nseg) v[k] = ll_ld16(addr(k));
  uint64_t t0 = 0;
  bool ok = true;
  while (true) {
    bool all = true;
#pragma unroll
    for (int k = 0; k < 4 * S; ++k)
      if ((k >> 2) < nseg) all = all && ready(v[k]);
    if (all) break;
    if (*w.abort_flag) {
      ok = false;
      break;
    }
    const uint64_t now = globaltimer();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > QASR_WAIT_NS) {
      report_error(w.status, DEVERR_TIMEOUT, site);
      *w.abort_flag = 1;
      ok = false;
      break;
    }
#pragma unroll
    for (int k = 0; k < 4 * S; ++k)
      if ((k >> 2) < nseg && !ready(v[k])) v[k] = ll_ld16(addr(k));
  }
  gs = make_float4(0.f, 0.f, 0.f, 0.f);
  us = gs;
#pragma unroll
  for (int s = 0; s < S; ++s)
    if (s < nseg) {
      gs.x += __uint_as_float(v[4 * s].x);
      gs.y += __uint_as_float(v[4 * s].z);
      gs.z += __uint_as_float(v[4 * s + 1].x);
      gs.w += __uint_as_float(v[4 * s + 1].z);
      us.x += __uint_as_float(v[4 * s + 2].x);
      us.y += __uint_as_float(v[4 * s + 2].z);
      us.z += __uint_as_float(v[4 * s + 3].x);
      us.w += __uint_as_float(v[4 * s + 3].z);
    }
  return ok;
}

// Sum over the epilogue group (CHAIN_EPI_WARPS warps), the same value in every thread.
__device__ __forceinline__ float chain_group_sum(float v, float* red, int e) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  named_bar_sync(1, CHAIN_EPI_THREADS);
  if ((e & 31) == 0) red[e >> 5] = v;
  named_bar_sync(1, CHAIN_EPI_THREADS);
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < CHAIN_EPI_WARPS; ++w) t += red[w];
  return t;
}

template <int PROG, bool F16>
__global__ void __launch_bounds__(CHAIN_THREADS, 1)
    decode_chain_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_attn,
                        const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ ChainArgs a) {
  constexpr int KSTEPS = 8;            // 128 k elements per unit, UMMA K = 16
  constexpr int WPU = F16 ? 2 : 1;     // 16 KB weight tiles (W stages) per unit
  constexpr int EPI_WARP0 = 16 - CHAIN_EPI_WARPS;
  extern __shared__ __align__(1024) uint8_t chain_dsmem[];
  __shared__ __align__(8) uint64_t wfull_bar[CHAIN_MAX_W_STAGES], wfree_bar[CHAIN_MAX_W_STAGES];
  // unit slots: A stage (TMEM) + X tile (shared memory) of one unit.  ufull completes when
  // the four builder warps published A and the X tile landed; ufree when its MMAs retired.
  __shared__ __align__(8) uint64_t ufull_bar[CHAIN_MAX_A_STAGES], ufree_bar[CHAIN_MAX_A_STAGES];
  __shared__ __align__(8) uint64_t dfull_bar[2], dfree_bar[2], done_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ int xready;  // GEMMs whose X input is complete (written by the epilogue leader)
  __shared__ int prev_done;  // the previous launch is complete (epilogue leader, after its wait)
  __shared__ int seg_ok, bar_ok;
  __shared__ float red[CHAIN_EPI_WARPS];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(chain_dsmem) + 1023) & ~uintptr_t(1023));
  const int SW = a.w_stages, SU = a.a_stages;  // W stages, unit slots
  const uint32_t x_tile_bytes = static_cast<uint32_t>(a.n_tile) * 128u;
  const uint32_t x_stage_bytes = 2u * x_tile_bytes;
  uint8_t* xring = smem + static_cast<size_t>(SW) * 16384;
  // TMEM columns: two accumulator buffers (double-buffered segments), each split into
  // NACC accumulators (one per MMA issuer warp) that the epilogue adds in index order;
  // then the A stages.
  const int NACC = a.n_acc;
  const uint32_t DSTR = (static_cast<uint32_t>(a.n_tile) + 31u) & ~31u;  // one accumulator
  const uint32_t DCOLS = DSTR * static_cast<uint32_t>(NACC);
  const uint32_t A_COLS0 = 2u * DCOLS;
  int n_gemm_ops = 0;
  for (int i = 0; i < a.n_ops; ++i) n_gemm_ops += a.ops[i].kind == CH_GEMM ? 1 : 0;

  if (threadIdx.x == 0) {
    if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS] = globaltimer();
    for (int i = 0; i < SW; ++i) {
      mbar_init(&wfull_bar[i], 1);
      mbar_init(&wfree_bar[i], F16 ? 1 : 4);  // the unit's MMA commit, or the 4 builder warps
    }
    for (int i = 0; i < SU; ++i) {
      // 4 builder warps + the X copy's expect_tx arrival (f16: the X copy alone)
      mbar_init(&ufull_bar[i], F16 ? 1 : 5);
      mbar_init(&ufree_bar[i], 1);  // the commit of the issuer that took the unit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull_bar[i], NACC);
      mbar_init(&dfree_bar[i], CHAIN_EPI_WARPS);
    }
    mbar_init(&done_bar, NACC);
    abort_flag = 0;
    xready = (a.n_ops > 0 && a.ops[0].kind == CH_GEMM) ? 1 : 0;
    prev_done = 0;
    fence_mbar_init();
    if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 37] = globaltimer();
  }
  if (warp == 2) {
    tmem_alloc(&tmem_base_sh, GEMM_TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 3 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_attn);
    tma_prefetch_desc(&tm_act);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  // Programmatic dependent launch: the previous launch (the attention merge) may still be
  // running.  Weights, scales, shared memory and TMEM never depend on it, so the producer,
  // the A builders and the MMA issuers start at once; the epilogue / row-operation warps
  // wait (in their own branch), then open the first GEMM's X copies (prev_done); every
  // later X gate follows a grid barrier they pass after that.
  if (threadIdx.x == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 38] = globaltimer();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One thread feeds both rings: weight units (16 KB bulk copies, run ahead across the
    // GEMMs as far as the W ring allows) and X tiles (TMA, once the GEMM's input is
    // complete on every CTA).  Non-blocking polls, so neither stream waits on the other.
    if (lane == 0) {
      int wg = -1, wu = 0, wue = 0, wst = 0, wissued = 0;
      int xg = -1, xu = 0, xue = 0, xst = 0, xissued = 0;
      uint32_t wph = 0, xph = 0;
      bool xgate = false;
      auto w_advance = [&]() {  // wu, wue count weight tiles (WPU per unit)
        while (wu >= wue && wg + 1 < n_gemm_ops) {
          ++wg;
          chain_unit_range(a.gemms[wg], blockIdx.x, wu, wue);
          wu *= WPU;
          wue *= WPU;
        }
      };
      auto x_advance = [&]() {
        while (xu >= xue && xg + 1 < n_gemm_ops) {
          ++xg;
          chain_unit_range(a.gemms[xg], blockIdx.x, xu, xue);
          xgate = false;
        }
      };
      w_advance();
      x_advance();
      if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 39] = globaltimer();
      uint64_t t_idle = globaltimer();
      int wlanded = 0;  // weight copies seen complete, in issue order
      // at most SW in flight: a copy's landing is checked before its stage is re-armed (a
      // barrier two phases on would read as not landed)
      const int cap = a.w_inflight > 0 ? min(a.w_inflight, SW) : SW;
      while (wu < wue || xu < xue) {
        bool prog = false;
        while (wissued - wlanded >= cap &&
               mbar_test(&wfull_bar[wlanded % SW], static_cast<uint32_t>((wlanded / SW) & 1)))
          ++wlanded;
        if (wu < wue && wissued - wlanded < cap && mbar_test(&wfree_bar[wst], wph ^ 1u)) {
          mbar_arrive_expect_tx(&wfull_bar[wst], 16384u);
          bulk_load(smem + static_cast<size_t>(wst) * 16384, a.gemms[wg].w + static_cast<size_t>(wu) * 16384, 16384u,
                    &wfull_bar[wst]);
          ++wissued;
          if (++wst == SW) {
            wst = 0;
            wph ^= 1u;
          }
          ++wu;
          w_advance();
          prog = true;
        }
        if (xu < xue) {
          // the first GEMM's X is the previous launch's output: also wait for its completion
          if (!xgate && ld_acquire_cta_shared(&xready) > xg && (xg > 0 || ld_acquire_cta_shared(&prev_done) != 0)) {
            fence_proxy_async_global();  // X was written by other CTAs with ordinary stores
            xgate = true;
            if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 25 + xg] = globaltimer();
          }
          if (xgate && mbar_test(&ufree_bar[xst], xph ^ 1u)) {
            const ChainGemm& g = a.gemms[xg];
            const CUtensorMap* tm = g.xmap == 0 ? &tm_x : (g.xmap == 1 ? &tm_attn : &tm_act);
            const int kb = xu % g.kblocks;
            uint8_t* dst = xring + static_cast<size_t>(xst) * x_stage_bytes;
            mbar_arrive_expect_tx(&ufull_bar[xst], x_stage_bytes);
            // both 64-column halves in one copy (the map views X as {64, rows, K / 64}):
            // the producer's copies queue behind the weight copies, so each one counts
            tma_load_3d(dst, tm, &ufull_bar[xst], 0, 0, 2 * kb);
            ++xissued;
            if (++xst == SU) {
              xst = 0;
              xph ^= 1u;
            }
            ++xu;
            x_advance();
            prog = true;
          }
        }
        if (prog) {
          t_idle = globaltimer();
        } else if (abort_flag) {
          break;
        } else if (globaltimer() - t_idle > QASR_WAIT_NS) {
          report_error(a.status, DEVERR_TIMEOUT, 0x701);
          abort_flag = 1;
          break;
        } else {
          __nanosleep(32);  // leave the issue slots to this SM sub-partition's other warps
        }
      }
      // the next launch's first weights and their row scales: into L2 while this launch
      // and the attention run
      if (a.next_first.w != nullptr && !abort_flag) {
        const ChainGemm& nf = a.next_first;
        int nu, nue;
        chain_unit_range(nf, blockIdx.x, nu, nue);
        for (int u = nu; u < nue; ++u) {
          bulk_prefetch_l2(nf.w + static_cast<size_t>(u) * 16384, 16384u);
          if (u == nu || u % nf.kblocks == 0) {  // a new 128-row tile: its 128 scales
            const uint32_t sb = nf.scale32 ? 4u : 2u;
            bulk_prefetch_l2(static_cast<const uint8_t*>(nf.scale) + static_cast<size_t>(u / nf.kblocks) * 128 * sb,
                             128u * sb);
          }
        }
      }
      // every issued copy lands before exit
      for (int j = 0; j < SW && j < wissued; ++j) {
        const int il = wissued - 1 - ((wissued - 1 - j) % SW);
        mbar_wait(&wfull_bar[j], static_cast<uint32_t>((il / SW) & 1), nullptr, a.status, 0x702);
      }
      if (abort_flag) {  // X copies complete on barriers the builders also arrive on: give them time
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 100000ull) __nanosleep(1000);
      } else {
        for (int j = 0; j < SU && j < xissued; ++j) {
          const int il = xissued - 1 - ((xissued - 1 - j) % SU);
          mbar_wait(&ufull_bar[j], static_cast<uint32_t>((il / SU) & 1), nullptr, a.status, 0x713);
        }
      }
    }
  } else if (warp <= 3) {
    // ------------------------------------------------------------ UMMA issuers
    // A thread can issue a tcgen05 instruction (mma, commit) or an mbarrier wait only every
    // ~120-230 cycles, whatever the MMA's size, so NACC warps issue in parallel: within a
    // segment, unit r goes to issuer r % NACC, which accumulates it into its own
    // accumulator; the epilogue adds the accumulators of the issuers that had units.  Every
    // issuer passes every segment's dfree wait and commits its dfull (count NACC), so
    // arrivals for a segment never run ahead into an earlier segment's phase.
    const int j = warp - 1;
    if (lane == 0 && j < NACC) {
      const uint32_t idesc = umma_idesc_f16_m128(static_cast<uint32_t>(a.n_tile));
      int us = 0, seg = -1, d = 0, i = 0, seg_i0 = 0;
      uint32_t uph = 0;
      bool ok = true, started = false;
      for (int gi = 0; gi < n_gemm_ops && ok; ++gi) {
        const ChainGemm& g = a.gemms[gi];
        int ub, ue;
        chain_unit_range(g, blockIdx.x, ub, ue);
        for (int u = ub; u < ue; ++u, ++i) {
          const int my_us = us;
          const uint32_t my_uph = uph;
          if (++us == SU) {
            us = 0;
            uph ^= 1u;
          }
          // f16: the unit's two W stages (the producer fills the ring tile by tile in unit order)
          const int wt0 = 2 * i, wt1 = 2 * i + 1;
          const int ws0 = wt0 % SW, ws1 = wt1 % SW;
          const uint32_t wp0 = static_cast<uint32_t>((wt0 / SW) & 1), wp1 = static_cast<uint32_t>((wt1 / SW) & 1);
          const int kb = u % g.kblocks;
          const bool first = (u == ub) || (kb == 0);
          const bool last = (u == ue - 1) || (kb == g.kblocks - 1);
          if (first) {
            ++seg;
            d = seg & 1;
            seg_i0 = i;
            started = false;
            if (!mbar_wait(&dfree_bar[d], static_cast<uint32_t>(((seg >> 1) & 1) ^ 1), &abort_flag, a.status,
                           0x721)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if ((i - seg_i0) % NACC == j) {
            if (!mbar_wait(&ufull_bar[my_us], my_uph, &abort_flag, a.status, 0x722) ||
                (F16 && (!mbar_wait(&wfull_bar[ws0], wp0, &abort_flag, a.status, 0x726) ||
                         !mbar_wait(&wfull_bar[ws1], wp1, &abort_flag, a.status, 0x727)))) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (a.trace != nullptr && i < 24) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 40 + i] = globaltimer();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(d) * DCOLS + static_cast<uint32_t>(j) * DSTR;
            const uint32_t x_base = smem_u32(xring + static_cast<size_t>(my_us) * x_stage_bytes);
            if constexpr (F16) {
              // A = the weight tiles themselves (128 rows x 64 k each, 128-byte swizzled rows)
              const uint32_t w0 = smem_u32(smem + static_cast<size_t>(ws0) * 16384);
              const uint32_t w1 = smem_u32(smem + static_cast<size_t>(ws1) * 16384);
#pragma unroll
              for (int kk = 0; kk < KSTEPS; ++kk) {
                const uint32_t b_addr = x_base + static_cast<uint32_t>(kk >> 2) * x_tile_bytes +
                                        static_cast<uint32_t>(kk & 3) * 32u;
                umma_f16_ss(d_tmem, smem_desc_sw128((kk < 4 ? w0 : w1) + static_cast<uint32_t>(kk & 3) * 32u),
                            smem_desc_sw128(b_addr), idesc, (!started && kk == 0) ? 0u : 1u);
              }
            } else {
              const uint32_t a_tmem = tmem_base + A_COLS0 + static_cast<uint32_t>(my_us) * 64u;
#pragma unroll
              for (int kk = 0; kk < KSTEPS; ++kk) {
                const uint32_t b_addr = x_base + static_cast<uint32_t>(kk >> 2) * x_tile_bytes +
                                        static_cast<uint32_t>(kk & 3) * 32u;
                umma_f16_ts(d_tmem, a_tmem + static_cast<uint32_t>(kk) * 8u, smem_desc_sw128(b_addr), idesc,
                            (!started && kk == 0) ? 0u : 1u);
              }
            }
            started = true;
            umma_commit(&ufree_bar[my_us]);
            if constexpr (F16) {  // the W stages are read
              umma_commit(&wfree_bar[ws0]);
              umma_commit(&wfree_bar[ws1]);
            }
            if (a.trace != nullptr) {
              const unsigned long long now = globaltimer();
              if (u == ub) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 29 + gi] = now;
              if (u == ue - 1) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 33 + gi] = now;
              if (i < 24) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 104 + i] = now;
            }
          }
          if (last) umma_commit(&dfull_bar[d]);
        }
      }
      // all MMAs retire before the TMEM is released (a commit with none pending arrives at once)
      umma_commit(&done_bar);
      mbar_wait(&done_bar, 0, nullptr, a.status, 0x724);
    }
  } else if (!F16 && warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ int8 A builders
    // Each unit is published as soon as its TMEM stores land (tcgen05.wait::st is cheap).
    const int t = (threadIdx.x - 128) & 127;  // row of the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int st = 0, ast = 0, i = 0;  // W stage, unit slot
    uint32_t ph = 0, aph = 0;
    bool ok = true;
    for (int gi = 0; gi < n_gemm_ops && ok; ++gi) {
      const ChainGemm& g = a.gemms[gi];
      int ub, ue;
      chain_unit_range(g, blockIdx.x, ub, ue);
      const bool f32s = g.scale32 != 0;
      // the rows' scales of a tile: loaded one unit ahead of the tile's first unit, so the
      // load's latency never stands between two units
      auto load_scale = [&](int tile, __half& s16, float& s32) {
        const int srow = tile * 128 + t;
        s32 = f32s ? static_cast<const float*>(g.scale)[srow] : 1.0f;
        s16 = f32s ? __float2half_rn(1.0f) : static_cast<const __half*>(g.scale)[srow];
      };
      __half sc = __float2half_rn(1.0f), nsc = sc;
      float sc32 = 1.0f, nsc32 = 1.0f;
      if (ub < ue) load_scale(ub / g.kblocks, sc, sc32);
      for (int u = ub; u < ue; ++u, ++i) {
        const int my_st = st, my_ast = ast;
        const uint32_t my_ph = ph, my_aph = aph;
        if (++st == SW) {
          st = 0;
          ph ^= 1u;
        }
        if (++ast == SU) {
          ast = 0;
          aph ^= 1u;
        }
        const bool next_tile = u + 1 < ue && (u + 1) % g.kblocks == 0;
        if (next_tile) load_scale((u + 1) / g.kblocks, nsc, nsc32);
        if (!mbar_wait_warp(&wfull_bar[my_st], my_ph, &abort_flag, a.status, 0x731)) {
          ok = false;
          break;
        }
        if (i == 0 && warp == 4 && lane == 0 && a.trace != nullptr)
          a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 64] = globaltimer();
        if (!mbar_wait_warp(&ufree_bar[my_ast], my_aph ^ 1u, &abort_flag, a.status, 0x732)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const __half2 sc2 = __halves2half2(sc, sc);
        if (i == 0 && warp == 4 && lane == 0 && a.trace != nullptr)
          a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 65] = globaltimer();
        const uint8_t* row = smem + static_cast<size_t>(my_st) * 16384 + t * 128;
        uint4 chunk[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) chunk[c] = *reinterpret_cast<const uint4*>(row + ((c ^ (t & 7)) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfree_bar[my_st]);  // the W stage is read: refill it
        const uint32_t taddr = tmem_base + lane_base + A_COLS0 + static_cast<uint32_t>(my_ast) * 64u;
        // one body per scale width: the choice is made once per unit, not per word.  Two
        // 32-column stores per row: a tcgen05 instruction costs its warp ~130 cycles to
        // issue whatever its width (measured on B200)
        auto build_row = [&](auto f32tag) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t outw[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 ch = chunk[4 * h + c];
              const uint32_t w4[4] = {ch.x, ch.y, ch.z, ch.w};
#pragma unroll
              for (int q = 0; q < 4; ++q)
                dequant_i8x4<decltype(f32tag)::value>(w4[q], sc2, sc32, outw[8 * c + 2 * q], outw[8 * c + 2 * q + 1]);
            }
            tmem_st_x32(taddr + static_cast<uint32_t>(h) * 32u, outw);
          }
        };
        if (f32s) build_row(std::true_type{});
        else build_row(std::false_type{});
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ufull_bar[my_ast]);
        if (i < 24 && warp == 4 && lane == 0 && a.trace != nullptr)
          a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 72 + i] = globaltimer();
        if (next_tile) {
          sc = nsc;
          sc32 = nsc32;
        }
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ------------------------------------------------------------ epilogue + row operations
    const int e = threadIdx.x - EPI_WARP0 * 32;  // 0 .. CHAIN_EPI_THREADS - 1
    const int we = warp - EPI_WARP0;
    const int row = (warp & 3) * 32 + lane;       // TMEM lane quadrant of this warp = tile row
    const int half = we >> 2;                     // two warps per quadrant split the columns
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const size_t slot_u64 = chain_slot_words(a.ws_rows);
    const int ss_ld = CHAIN_MAX_HS / 128;
    int seg = -1, nbar = 0;
    bool ok = true;
    griddep_wait();
    // this launch's flag: the step counter was written by an earlier step's last kernel
    const uint32_t flag = (*reinterpret_cast<const volatile unsigned int*>(a.epoch) << 6) |
                          static_cast<uint32_t>(a.launch_idx + 1);
    const LLWait llw{&abort_flag, a.status, flag};
    if (e == 0) {
      st_release_cta_shared(&prev_done, 1);  // opens the first GEMM's X copies
      if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 66] = globaltimer();
    }
    const int wid = blockIdx.x * CHAIN_EPI_WARPS + we, nwarps = gridDim.x * CHAIN_EPI_WARPS;

    // GEMM gi: this CTA's accumulators -> flagged partial sums (one slot per (tile, CTA))
    auto op_gemm = [&](int gi) {
      const ChainGemm& g = a.gemms[gi];
      int ub, ue;
      chain_unit_range(g, blockIdx.x, ub, ue);
      int u = ub;
      while (u < ue) {
        const int T = u / g.kblocks;
        const int seg_end = min(ue, (T + 1) * g.kblocks);
        ++seg;
        const int d = seg & 1;
        if (e == 0)
          seg_ok = mbar_wait(&dfull_bar[d], static_cast<uint32_t>((seg >> 1) & 1), &abort_flag, a.status, 0x741)
                       ? 1
                       : 0;
        named_bar_sync(1, CHAIN_EPI_THREADS);
        const int got = seg_ok;
        named_bar_sync(1, CHAIN_EPI_THREADS);
        if (!got) {
          ok = false;
          return;
        }
        mbar_try_wait(&dfull_bar[d], static_cast<uint32_t>((seg >> 1) & 1));
        tc_fence_after();
        const int segidx = static_cast<int>(blockIdx.x) - cta_of_unit(static_cast<long long>(T) * g.kblocks,
                                                                       g.units, g.grid);
        uint64_t* dst = g.ws + (static_cast<size_t>(T) * g.max_seg + segidx) * slot_u64 + row;
        const uint32_t dt = tmem_base + lane_base + static_cast<uint32_t>(d) * DCOLS;
        const int n_used = min(NACC, seg_end - u);  // issuers that had units in the segment
        for (int c0 = 16 * half; c0 < a.n_tile; c0 += 32) {
          float v[16];
          for (int q = 0; q < n_used; ++q) {
            uint32_t r[16];
            tmem_ld_x16(dt + static_cast<uint32_t>(q) * DSTR + static_cast<uint32_t>(c0), r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = q == 0 ? __uint_as_float(r[j]) : v[j] + __uint_as_float(r[j]);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < a.rows) ll_st8(dst + static_cast<size_t>(c0 + j) * 128, __float_as_uint(v[j]), flag);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfree_bar[d]);
        u = seg_end;
      }
    };

    // grid barrier after operation oi (before a GEMM whose X tiles the producer copies with
    // TMA): release this CTA's writes (the group's, ordered by the named barrier), arrive,
    // poll with acquire loads, then open GEMM next_gemm's X copies.  (Measured on B200: a
    // release, or a fence.acq_rel, waits until every bulk copy the SM has in flight has
    // landed, ~1.3 us while the weight ring streams; an acquire load costs what a relaxed
    // load does, so the poll carries the acquire and no fence follows it.)
    auto grid_barrier = [&](int oi, int next_gemm) {
      named_bar_sync(1, CHAIN_EPI_THREADS);
      if (e == 0) {
        if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * oi] = globaltimer();
        ++nbar;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.barrier) : "memory");
        const unsigned int target = static_cast<unsigned int>(nbar) * gridDim.x;
        if (ld_acquire_gpu(a.barrier) < target) {
          const uint64_t t0 = globaltimer();
          while (ld_acquire_gpu(a.barrier) < target) {
            if (abort_flag || globaltimer() - t0 > QASR_WAIT_NS) {
              if (!abort_flag) report_error(a.status, DEVERR_TIMEOUT, 0x761);
              abort_flag = 1;
              break;
            }
          }
        }
        bar_ok = abort_flag ? 0 : 1;
        if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 2 + 2 * oi] = globaltimer();
        st_release_cta_shared(&xready, next_gemm + 1);
      }
      named_bar_sync(1, CHAIN_EPI_THREADS);
      if (!bar_ok) ok = false;
    };
    // between two operations without a barrier: the next one waits for exactly the flagged
    // words it reads; only a CTA-wide verdict (and the trace stamp)
    auto next_op = [&](int oi) {
      named_bar_sync(1, CHAIN_EPI_THREADS);
      if (e == 0) {
        if (a.trace != nullptr) {
          const unsigned long long now = globaltimer();
          a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * oi] = now;
          a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 2 + 2 * oi] = now;
        }
        bar_ok = abort_flag ? 0 : 1;
      }
      named_bar_sync(1, CHAIN_EPI_THREADS);
      if (!bar_ok) ok = false;
    };

    // h[r] = embed row of the slot's input token, x[r] = rmsnorm(h[r]); one row per CTA,
    // thread e holds the column pairs 2e + 256 j
    auto op_embed_norm = [&](const ChainOp& op) {
      const int np = a.hs / (2 * CHAIN_EPI_THREADS);
      for (int r = blockIdx.x; r < a.rows; r += gridDim.x) {
        __half* hr = a.h + static_cast<size_t>(r) * a.hs;
        const int slot = a.row_slot[r];
        int tok = a.next_tok[slot];
        if (tok < 0 || tok >= a.vocab) {
          if (e == 0) report_error(a.status, DEVERR_BOUNDS, 0x751);
          tok = 0;
        }
        const __half* src = a.embed + static_cast<size_t>(tok) * a.hs;
        const int pos = a.pos[slot];
        if (e == 0) {
          a.row_pos[r] = pos;
          a.row_page[r] = a.kv.page_table[static_cast<size_t>(slot) * a.kv.max_pages + (pos >> 6)];
        }
        if (e < 32) {  // cos | sin rows of the position, 16 bytes per thread
          const __half* rs = (e < 16 ? a.rope_cos : a.rope_sin) + static_cast<size_t>(pos) * 128 + (e & 15) * 8;
          __stcg(reinterpret_cast<uint4*>(a.row_rope + static_cast<size_t>(r) * 256 + e * 8),
                 *reinterpret_cast<const uint4*>(rs));
        }
        float2 v[CHAIN_MAX_HS / (2 * CHAIN_EPI_THREADS)];
        float sq = 0.f;
#pragma unroll
        for (int j = 0; j < CHAIN_MAX_HS / (2 * CHAIN_EPI_THREADS); ++j) {
          if (j < np) {
            const int i = 2 * e + 2 * CHAIN_EPI_THREADS * j;
            v[j] = __half22float2(*reinterpret_cast<const __half2*>(src + i));
            __stcg(reinterpret_cast<__half2*>(hr + i), __floats2half2_rn(v[j].x, v[j].y));
            sq = __fadd_rn(sq, __fmul_rn(v[j].x, v[j].x));
            sq = __fadd_rn(sq, __fmul_rn(v[j].y, v[j].y));
          }
        }
        const float tot = chain_group_sum(sq, red, e);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(a.hs)), a.eps)));
        __half* y = op.norm_out + static_cast<size_t>(r) * a.hs;
#pragma unroll
        for (int j = 0; j < CHAIN_MAX_HS / (2 * CHAIN_EPI_THREADS); ++j) {
          if (j < np) {
            const int i = 2 * e + 2 * CHAIN_EPI_THREADS * j;
            const float x0 = __fmul_rn(__fmul_rn(v[j].x, inv), op.norm_w[i]);
            const float x1 = __fmul_rn(__fmul_rn(v[j].y, inv), op.norm_w[i + 1]);
            __stcg(reinterpret_cast<__half2*>(y + i), __floats2half2_rn(x0, x1));
          }
        }
        named_bar_sync(1, CHAIN_EPI_THREADS);  // `red` is reused by the next row
      }
    };

    // h[r, 128 T + c] = f16(h + sum of the GEMM's flagged partials), and the tile's sum of
    // squares of the new f16 values, flagged, into ss[ch][r][T]; one warp per (row, tile),
    // lane = 4 columns
    auto op_resid = [&](const ChainOp& op) {
      const ChainGemm& g = a.gemms[op.gemm];
      const int tiles = a.hs / 128;
      for (int it = wid; it < a.rows * tiles; it += nwarps) {
        const int r = it / tiles, T = it - r * tiles;
        // the residual's load is issued before the poll, so its round trip overlaps it
        __half* hp = a.h + static_cast<size_t>(r) * a.hs + T * 128 + 4 * lane;
        const uint2 hw = __ldcg(reinterpret_cast<const uint2*>(hp));
        float4 acc;
        const bool lok = chain_sum4<CHAIN_MAX_SEG>(chain_partial(a, g, T, r, 4 * lane), slot_u64,
                                                   chain_tile_segs(g, T), acc, llw, 0x752);
        if (!__all_sync(0xffffffffu, lok)) break;
        const float2 h01 = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
        const float2 h23 = __half22float2(*reinterpret_cast<const __half2*>(&hw.y));
        const __half2 n01 = __floats2half2_rn(__fadd_rn(h01.x, acc.x), __fadd_rn(h01.y, acc.y));
        const __half2 n23 = __floats2half2_rn(__fadd_rn(h23.x, acc.z), __fadd_rn(h23.y, acc.w));
        uint2 nw;
        nw.x = *reinterpret_cast<const uint32_t*>(&n01);
        nw.y = *reinterpret_cast<const uint32_t*>(&n23);
        __stcg(reinterpret_cast<uint2*>(hp), nw);
        const float2 f01 = __half22float2(n01), f23 = __half22float2(n23);
        float sq = __fmul_rn(f01.x, f01.x);
        sq = __fadd_rn(sq, __fmul_rn(f01.y, f01.y));
        sq = __fadd_rn(sq, __fmul_rn(f23.x, f23.x));
        sq = __fadd_rn(sq, __fmul_rn(f23.y, f23.y));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) ll_st8(a.ss[op.ch] + static_cast<size_t>(r) * ss_ld + T, __float_as_uint(sq), flag);
      }
    };

    // norm_out[r] = f16(h * inv * w), inv = 1 / sqrt(sum_T ss[ch][r][T] / hs + eps)
    // (rms_norm_row, src/cpu_decoder.rs:261-272); one warp per (row, tile), the same warp
    // that wrote the tile's h in the residual add before it
    auto op_norm = [&](const ChainOp& op) {
      const int tiles = a.hs / 128;
      for (int it = wid; it < a.rows * tiles; it += nwarps) {
        const int r = it / tiles, T = it - r * tiles;
        // this warp's h tile (it wrote it in the residual add) and the gains, loaded before
        // the poll so their round trips overlap it
        const int c = T * 128 + 4 * lane;
        const uint2 hw = __ldcg(reinterpret_cast<const uint2*>(a.h + static_cast<size_t>(r) * a.hs + c));
        const float4 w = *reinterpret_cast<const float4*>(op.norm_w + c);
        bool lok = true;
        float t = 0.f;
        if (lane < tiles) {
          const uint64_t* src = a.ss[op.ch] + static_cast<size_t>(r) * ss_ld + lane;
          uint2 w = ll_ld8(src);
          if (w.y != flag) {
            w = ll_spin8(src, llw, 0x753);
            lok = w.y == flag;
          }
          t = __uint_as_float(w.x);
        }
        if (!__all_sync(0xffffffffu, lok)) break;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        t = __shfl_sync(0xffffffffu, t, 0);  // lane 0's order, the same value everywhere
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(a.hs)), a.eps)));
        const float2 h01 = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
        const float2 h23 = __half22float2(*reinterpret_cast<const __half2*>(&hw.y));
        const __half2 x01 = __floats2half2_rn(__fmul_rn(__fmul_rn(h01.x, inv), w.x), __fmul_rn(__fmul_rn(h01.y, inv), w.y));
        const __half2 x23 = __floats2half2_rn(__fmul_rn(__fmul_rn(h23.x, inv), w.z), __fmul_rn(__fmul_rn(h23.y, inv), w.w));
        uint2 xw;
        xw.x = *reinterpret_cast<const uint32_t*>(&x01);
        xw.y = *reinterpret_cast<const uint32_t*>(&x23);
        __stcg(reinterpret_cast<uint2*>(op.norm_out + static_cast<size_t>(r) * a.hs + c), xw);
      }
    };

    // gate|up tile t: rows [0, 64) gate[64 t + i], rows [64, 128) up[64 t + i].  Work unit:
    // 4 outputs (row r, tile t, quad c); each thread takes every (G * 256)-th one
    auto op_silu = [&](const ChainOp& op) {
      const ChainGemm& g = a.gemms[op.gemm];
      const int tiles = g.units / g.kblocks;
      const int total = a.rows * tiles * 16;
      const int stride = gridDim.x * CHAIN_EPI_THREADS;
      for (int q = blockIdx.x * CHAIN_EPI_THREADS + e; q < total; q += stride) {
        const int c = q & 15, rt = q >> 4;
        const int r = rt / tiles, t = rt - r * tiles;
        const int nseg = chain_tile_segs(g, t);
        const uint64_t* p = chain_partial(a, g, t, r, 4 * c);
        // per segment: the gate words (at p) and the up words (at p + 64), all polled together
        float4 gs, us;
        if (!chain_sum_gate_up(p, slot_u64, nseg, gs, us, llw, 0x755)) break;
        const float gv[4] = {gs.x, gs.y, gs.z, gs.w}, uv[4] = {us.x, us.y, us.z, us.w};
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float gt = f16_round(gv[j]);
          const float silu = __fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt)));
          o[j] = __fmul_rn(silu, f16_round(uv[j]));
        }
        const __half2 o01 = __floats2half2_rn(o[0], o[1]), o23 = __floats2half2_rn(o[2], o[3]);
        uint2 ow;
        ow.x = *reinterpret_cast<const uint32_t*>(&o01);
        ow.y = *reinterpret_cast<const uint32_t*>(&o23);
        __stcg(reinterpret_cast<uint2*>(a.act + static_cast<size_t>(r) * a.inter + t * 64 + 4 * c), ow);
      }
    };

    // q/k RMSNorm + RoPE -> q and paged K; raw V -> paged V.  One warp per (row, head),
    // lane = dims 4 lane .. +3; the rotate-half partner of dim d (d ^ 64) sits in lane ^ 16
    auto op_qkv = [&](const ChainOp& op) {
      const ChainGemm& g = a.gemms[op.gemm];
      const int heads = a.nq + 2 * a.nkv;
      for (int it = wid; it < a.rows * heads; it += nwarps) {
        const int r = it / heads, t = it - r * heads;
        const int d0 = 4 * lane;
        const int pos = __ldcg(a.row_pos + r);
        const int page = __ldcg(a.row_page + r);
        const uint2 cw = __ldcg(reinterpret_cast<const uint2*>(a.row_rope + static_cast<size_t>(r) * 256 + d0));
        const uint2 sw = __ldcg(reinterpret_cast<const uint2*>(a.row_rope + static_cast<size_t>(r) * 256 + 128 + d0));
        const float4 w = t < a.nq + a.nkv ? *reinterpret_cast<const float4*>((t < a.nq ? op.qn_w : op.kn_w) + d0)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 acc;
        const bool lok = chain_sum4<CHAIN_QKV_SEG>(chain_partial(a, g, t, r, 4 * lane), slot_u64,
                                                   chain_tile_segs(g, t), acc, llw, 0x757);
        if (!__all_sync(0xffffffffu, lok)) break;
        // offset of the (page, layer, K|V, head) row of `pos` (the layout of kv_elem_offset)
        auto kv_off = [&](int which, int head) {
          return ((((static_cast<size_t>(page) * a.kv.layers + op.layer) * 2 + which) * a.kv.nkv + head) * 64 +
                  (pos & 63)) *
                 128;
        };
        if (t >= a.nq + a.nkv) {  // V: raw f16 projection into the cache
          const size_t off = kv_off(1, t - a.nq - a.nkv);
          const __half2 v01 = __floats2half2_rn(acc.x, acc.y), v23 = __floats2half2_rn(acc.z, acc.w);
          uint2 vw;
          vw.x = *reinterpret_cast<const uint32_t*>(&v01);
          vw.y = *reinterpret_cast<const uint32_t*>(&v23);
          *reinterpret_cast<uint2*>(a.kv.pool + off + kv_dim_swizzle(pos, d0)) = vw;
          continue;
        }
        const float x[4] = {f16_round(acc.x), f16_round(acc.y), f16_round(acc.z), f16_round(acc.w)};
        float ss = __fmul_rn(x[0], x[0]);
        ss = __fadd_rn(ss, __fmul_rn(x[1], x[1]));
        ss = __fadd_rn(ss, __fmul_rn(x[2], x[2]));
        ss = __fadd_rn(ss, __fmul_rn(x[3], x[3]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        ss = __shfl_sync(0xffffffffu, ss, 0);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps)));
        const float wv[4] = {w.x, w.y, w.z, w.w};
        float xn[4], xp[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xn[j] = __fmul_rn(__fmul_rn(x[j], inv), wv[j]);
#pragma unroll
        for (int j = 0; j < 4; ++j) xp[j] = __shfl_xor_sync(0xffffffffu, xn[j], 16);
        const float2 c01 = __half22float2(*reinterpret_cast<const __half2*>(&cw.x));
        const float2 c23 = __half22float2(*reinterpret_cast<const __half2*>(&cw.y));
        const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&sw.x));
        const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&sw.y));
        const float cv[4] = {c01.x, c01.y, c23.x, c23.y}, sv[4] = {s01.x, s01.y, s23.x, s23.y};
        const float sign = lane < 16 ? -1.0f : 1.0f;
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = __fadd_rn(__fmul_rn(xn[j], cv[j]), __fmul_rn(__fmul_rn(sign, xp[j]), sv[j]));
        const __half2 o01 = __floats2half2_rn(o[0], o[1]), o23 = __floats2half2_rn(o[2], o[3]);
        uint2 ow;
        ow.x = *reinterpret_cast<const uint32_t*>(&o01);
        ow.y = *reinterpret_cast<const uint32_t*>(&o23);
        if (t < a.nq) {
          *reinterpret_cast<uint2*>(a.q + static_cast<size_t>(r) * a.nq * 128 + t * 128 + d0) = ow;
        } else {
          const size_t off = kv_off(0, t - a.nq);
          *reinterpret_cast<uint2*>(a.kv.pool + off + kv_dim_swizzle(pos, d0)) = ow;
        }
      }
    };

    // the launch's program as straight-line code: each operation's set-up lives only while
    // it runs (a loop over a list of operations kept all of them live and spilled)
    auto done = [&](int oi) {
      if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * oi] = globaltimer();
    };
    if constexpr (PROG == CHAIN_PROG_FIRST) {
      // embed + layer 0's input norm | QKV GEMM | q/k norm + RoPE + K/V append
      op_embed_norm(a.ops[0]);
      grid_barrier(0, 0);
      if (ok) op_gemm(0);
      if (ok) next_op(1);
      if (ok) op_qkv(a.ops[2]);
      done(2);
    } else {
      // o_proj | residual | post-attention norm || gate|up | SiLU || down | residual |
      // next input norm (or the final norm) || QKV GEMM | q/k norm + RoPE + K/V append
      op_gemm(0);
      if (ok) next_op(0);
      if (ok) op_resid(a.ops[1]);
      if (ok) next_op(1);
      if (ok) op_norm(a.ops[2]);
      if (ok) grid_barrier(2, 1);
      if (ok) op_gemm(1);
      if (ok) next_op(3);
      if (ok) op_silu(a.ops[4]);
      if (ok) grid_barrier(4, 2);
      if (ok) op_gemm(2);
      if (ok) next_op(5);
      if (ok) op_resid(a.ops[6]);
      if (ok) next_op(6);
      if (ok) op_norm(a.ops[7]);
      if constexpr (PROG == CHAIN_PROG_MIDDLE) {
        if (ok) grid_barrier(7, 3);
        if (ok) op_gemm(3);
        if (ok) next_op(8);
        if (ok) op_qkv(a.ops[9]);
        done(9);
      } else {
        done(7);
      }
    }
  }

  griddep_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, GEMM_TMEM_COLS);
  if (threadIdx.x == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + CHAIN_TRACE_SLOTS - 1] = globaltimer();
}

}  // namespace qasr
