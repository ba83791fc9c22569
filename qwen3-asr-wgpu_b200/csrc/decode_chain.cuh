// The decode step between two attention launches as ONE persistent kernel.
//
// One launch runs a short program of operations over the step's decode rows, e.g.
//   o_proj GEMM -> residual add -> gate|up GEMM (input: post-attention RMSNorm) -> SiLU ->
//   down GEMM -> residual add -> next layer's QKV GEMM (input: its input RMSNorm) ->
//   q/k RMSNorm + RoPE + paged K/V append
// which is what CpuTextDecoder::forward_layer (src/cpu_decoder.rs:367-455) does between
// two attention calls; the per-kernel path of this library launches those as 7 kernels.
// One CTA per SM, all CTAs resident (cooperative launch, or a plain launch of one CTA per
// SM whose residency the host checks).
//
// No grid barrier.  Every value one CTA hands to another travels as an 8-byte word
// {32-bit data, 32-bit flag} written with one store (the layout of NCCL's LL protocol):
// the flag is this launch's epoch, so a reader polls the words it needs until their
// flags match and then uses the data — no fence, no counter.  (A gpu-scope release would
// also wait for this SM's weight copies in flight, ~1-4 us per barrier.)  The epoch is
// (step counter << 6) | (launch index + 1); the step counter is a device word the step's
// last kernel increments, so every launch of every step writes flags no earlier write to
// the same word carried.
//
// GEMM operations are the tcgen05 weight-streaming GEMM of gemm_tc.cuh in stream-K form:
// every (tile, CTA) segment stores its f32 partial sums (flagged) to a per-GEMM workspace,
// and the NEXT operation adds a tile's partials in segment order while it builds its own
// result (residual add, SiLU, q/k norm): no CTA finishes another's tile.  The weights of
// later GEMMs do not depend on anything computed in the launch, so the weight producer
// and the int8 dequantising builders run ahead into the next GEMMs' units as far as their
// rings allow.  The activation tile (X, the MMA's B operand) of each unit is built by the
// epilogue warps straight into shared memory from flagged words: an RMSNorm is folded into
// that build (x = f16(h * inv * w), inv from the per-tile sums of squares the residual add
// left), SiLU output and attention output are copied.
//
// Roles (512 threads):
//   warp 0      producer: 16 KB bulk copy per weight unit into the W ring
//   warps 1-3   UMMA issuers (A from TMEM, B = X from shared memory), units dealt
//               round-robin within a segment; warp 2 also allocates the TMEM
//   warps 4-7   int8 A builders: f16(q * s) into TMEM
//   warps 8-15  epilogue (two warps per TMEM lane quadrant, splitting the accumulator
//               columns), X-tile builds and row operations
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
constexpr int CHAIN_MAX_HS = 2048;   // hidden size the row operations and flagged rows hold
// warps 8-15 run the epilogue, the X builds and the row operations (two per TMEM lane
// quadrant), warps 4-7 dequantise: one builder warpgroup keeps pace with the MMA issuers
constexpr int CHAIN_EPI_WARPS = 8;
constexpr int CHAIN_EPI_THREADS = CHAIN_EPI_WARPS * 32;
// most segments a tile of a chain GEMM may be cut into, per reader (all loads of a read are
// issued at once): residual adds (o_proj, down), SiLU (gate|up), q/k/v (QKV)
constexpr int CHAIN_MAX_SEG = 12;
constexpr int CHAIN_SILU_SEG = 4;
constexpr int CHAIN_QKV_SEG = 8;
constexpr int CHAIN_CHANNELS = 2;  // flagged residual rows + sums of squares: two per launch
constexpr int CHAIN_X_BATCH = 3;   // X tiles whose loads are in flight together
// the launch programs (the op lists the host fills ChainArgs::ops with)
enum ChainProgram : int {
  CHAIN_PROG_FIRST = 0,   // embed, QKV GEMM (X: input norm of layer 0), QKV op
  CHAIN_PROG_MIDDLE = 1,  // o_proj, resid, gate|up (X: post-attention norm), SiLU, down, resid,
                          // next layer's QKV GEMM (X: its input norm), QKV op
  CHAIN_PROG_LAST = 2,    // as MIDDLE up to the second resid, then the final norm
};

enum ChainOpKind : int {
  CH_GEMM = 0,   // partial sums of W x over this CTA's (tile, k-block) range
  CH_EMBED = 1,  // h[r] = embed[next_tok[slot_r]] (+ flagged copy and per-tile sums of
                 // squares in channel `ch`); row_pos / row_page / row_rope for the step
  CH_RESID = 2,  // h = f16(h + sum of the GEMM's partials), flagged copy + sums of squares
  CH_NORM = 3,   // norm_out = rmsnorm(h) from channel `ch` (the final norm -> lm_head input)
  CH_SILU = 4,   // act = f16(silu(f16 gate) * f16 up) from the gate|up GEMM's partials
  CH_QKV = 5,    // q/k RMSNorm + RoPE -> q and paged K; raw V -> paged V
};

enum ChainXSrc : int {
  XS_ATTN = 0,  // the attention output [rows][nq * 128] (written by the previous launches)
  XS_NORM = 1,  // rmsnorm of the flagged residual rows of channel xch, gain xnorm_w
  XS_ACT = 2,   // the flagged SiLU output [rows][inter]
};

struct ChainGemm {
  const uint8_t* w;     // int8 weights in the tiled layout (weight_tile_offset)
  const void* scale;    // per-row scales: f16, or f32 when scale32
  int scale32;
  int kblocks;          // K / 128
  int units;            // (n_out / 128) * kblocks
  int grid;             // CTAs that take part: the first `grid` of the launch
  int max_seg;          // most segments (CTAs) any tile is cut into
  int xsrc;             // ChainXSrc of the B operand
  int xch;              // XS_NORM: channel
  const float* xnorm_w; // XS_NORM: RMSNorm gain
  uint64_t* ws;         // flagged partial sums [tile][max_seg][ws_rows][128] {f32, flag}
};

struct ChainOp {
  int kind;
  int gemm;             // CH_GEMM: index into gemms; row ops: the GEMM whose partials they add
  int ch;               // CH_EMBED / CH_RESID: channel written; CH_NORM: channel read
  const float* norm_w;  // CH_NORM: RMSNorm gain
  __half* norm_out;     // CH_NORM: normalised rows [rows][hs]
  const float* qn_w;    // CH_QKV: q / k RMSNorm gains
  const float* kn_w;
  int layer;            // CH_QKV: KV-cache layer
  int direct_meta;      // CH_QKV: read the rows' position / page / rope rows from the tables
                        // (the launch that also runs CH_EMBED, which fills the per-row copies)
};

struct ChainArgs {
  ChainOp ops[CHAIN_MAX_OPS];
  ChainGemm gemms[CHAIN_MAX_GEMMS];
  int n_ops;
  int rows, n_tile;
  int w_stages, a_stages;  // weight stages; unit slots (A stage in TMEM + X tile in smem)
  int w_inflight;          // most weight copies in flight at once: an SM's loads queue behind
                           // its bulk copies, so a deep burst would delay every X and flag read
  int n_acc;  // MMA issuer warps = accumulators per segment buffer (1 to 3)
  ChainGemm next_first;  // the next chain launch's first GEMM (w == nullptr: none): its
                         // units of this CTA are prefetched into L2 once this launch's
                         // weights are all issued, so they are resident when it starts
  int hs, inter, nq, nkv;
  float eps;
  __half* h;           // [rows][hs] residual stream (read by the next launches)
  __half* q;           // [rows][nq * 128]
  const __half* attn;  // [rows][nq * 128] attention output (XS_ATTN)
  const __half* embed;
  int vocab;
  const int* row_slot;
  int* row_pos;
  const int* next_tok;
  const int* pos;
  const __half* rope_cos;
  const __half* rope_sin;
  // per decode row, filled by CH_EMBED for the later launches of the step: the KV page of
  // the row's position and its RoPE cos | sin rows [rows][256]
  int* row_page;
  __half* row_rope;
  KvLayout kv;
  int ws_rows;                   // rows per partial slot (fixed for the context, >= n_tile)
  uint64_t* hf[CHAIN_CHANNELS];  // flagged residual rows [CHAIN_MAX_ROWS][CHAIN_MAX_HS / 2] {half2, flag}
  uint64_t* ss[CHAIN_CHANNELS];  // flagged per-tile sums of squares [CHAIN_MAX_ROWS][CHAIN_MAX_HS / 128]
  uint64_t* actf;                // flagged SiLU output [CHAIN_MAX_ROWS][inter / 2] {half2, flag}
  const unsigned int* epoch;     // the step counter (incremented by the step's last kernel)
  int launch_idx;                // this launch's index in the step (< 63)
  uint32_t* status;
  unsigned long long* trace;  // optional: per CTA CHAIN_TRACE_SLOTS %globaltimer stamps: 0 entry,
                              // 1 + 2 i op i done, 2 + 2 i the next op's inputs seen (i < 12),
                              // 25 + g GEMM g's first X tile built, 29 + g its first MMA issued,
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
__device__ __forceinline__ uint4 ll_spin16(const uint64_t* p, LLWait w, uint32_t site) {
  const uint64_t t0 = globaltimer();
  while (true) {
    const uint4 v = ll_ld16(p);
    if ((v.y == w.flag && v.w == w.flag) || *w.abort_flag) return v;
    if (globaltimer() - t0 > QASR_WAIT_NS) {
      report_error(w.status, DEVERR_TIMEOUT, site);
      *w.abort_flag = 1;
      return v;
    }
  }
}
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
// N 16-byte words at p, p + stride, ...: all first loads in flight at once, then a poll of
// whichever were not ready.  True when every word carries the flag.
template <int N>
__device__ __forceinline__ bool ll_get16(const uint64_t* p, size_t stride, int n, uint4 (&v)[N], const LLWait& w,
                                         uint32_t site) {
  bool ok = true;
#pragma unroll
  for (int s = 0; s < N; ++s)
    if (s < n) v[s] = ll_ld16(p + s * stride);
#pragma unroll
  for (int s = 0; s < N; ++s) {
    if (s < n && !(v[s].y == w.flag && v[s].w == w.flag)) {
      v[s] = ll_spin16(p + s * stride, w, site);
      ok = ok && v[s].y == w.flag && v[s].w == w.flag;
    }
  }
  return ok;
}

// Partials of (tile t, row n, columns m, m + 1): segment s at chain_partial(...) + s * ws_rows * 128.
__device__ __forceinline__ const uint64_t* chain_partial(const ChainArgs& a, const ChainGemm& g, int t, int n,
                                                         int m) {
  return g.ws + (static_cast<size_t>(t) * g.max_seg * a.ws_rows + n) * 128 + m;
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
template <int MAXSEG, bool SPLIT>
__device__ __forceinline__ bool chain_sum4(const uint64_t* p, size_t stride, int nseg, float4& acc, const LLWait& w,
                                          uint32_t site) {
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
  bool ok;
  if constexpr (SPLIT) {
    uint4 v[MAXSEG];
    ok = ll_get16<MAXSEG>(p, stride, nseg, v, w, site);
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s)
      if (s < nseg) {
        acc.x += __uint_as_float(v[s].x);
        acc.y += __uint_as_float(v[s].z);
      }
    ok = ll_get16<MAXSEG>(p + 2, stride, nseg, v, w, site) && ok;
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s)
      if (s < nseg) {
        acc.z += __uint_as_float(v[s].x);
        acc.w += __uint_as_float(v[s].z);
      }
  } else {
    uint4 lo[MAXSEG], hi[MAXSEG];
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s)
      if (s < nseg) {
        lo[s] = ll_ld16(p + s * stride);
        hi[s] = ll_ld16(p + 2 + s * stride);
      }
    ok = true;
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s) {
      if (s < nseg && !(lo[s].y == w.flag && lo[s].w == w.flag)) {
        lo[s] = ll_spin16(p + s * stride, w, site);
        ok = ok && lo[s].y == w.flag && lo[s].w == w.flag;
      }
      if (s < nseg && !(hi[s].y == w.flag && hi[s].w == w.flag)) {
        hi[s] = ll_spin16(p + 2 + s * stride, w, site);
        ok = ok && hi[s].y == w.flag && hi[s].w == w.flag;
      }
    }
#pragma unroll
    for (int s = 0; s < MAXSEG; ++s)
      if (s < nseg) {
        acc.x += __uint_as_float(lo[s].x);
        acc.y += __uint_as_float(lo[s].z);
        acc.z += __uint_as_float(hi[s].x);
        acc.w += __uint_as_float(hi[s].z);
      }
  }
  return ok;
}

// Register split among the warpgroups (setmaxnreg; the launch gives every thread 128):
// the weight producer + MMA issuers (warps 0-3) and the int8 A builders (warps 4-7) need
// few, the epilogue / row-operation warps (8-15) hold up to CHAIN_MAX_SEG 16-byte words in
// flight per thread.  A spilled register would live in L2 here (the shared-memory carve-out
// leaves the L1 almost nothing) behind the SM's weight copies, so none may spill.  Each
// role sets its share on entry and returns to 128 before the roles rejoin; the builders'
// and the producer's return waits for the epilogue's, which waits on nothing they do after
// their main loops.
constexpr int CHAIN_REGS_PRODUCER = 56, CHAIN_REGS_BUILDER = 96, CHAIN_REGS_EPI = 176;
static_assert(128 * CHAIN_REGS_PRODUCER + 128 * CHAIN_REGS_BUILDER + CHAIN_EPI_THREADS * CHAIN_REGS_EPI <=
                  CHAIN_THREADS * 128,
              "the warpgroups' registers must fit in what the launch allocates (512 threads x 128)");
static_assert(CHAIN_EPI_WARPS == 8 && CHAIN_THREADS == 512, "warpgroups 0 / 1 / 2-3 = producer+MMA / builders / epilogue");
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// CH_RESID over this warp's (row, tile) items: h = f16(h + the GEMM's partials), the flagged
// copy and the tile's sum of squares of the new f16 values into channel op.ch.
__device__ __forceinline__ void chain_resid(const ChainArgs& a, const ChainOp& op, int warp_id, int warps,
                                         LLWait llw) {
  const int lane = threadIdx.x & 31;
  const size_t slot_u64 = static_cast<size_t>(a.ws_rows) * 128;
  const int hf_ld = CHAIN_MAX_HS / 2, ss_ld = CHAIN_MAX_HS / 128;
  const uint32_t flag = llw.flag;
  // h[r, 128 T + c] = f16(h + sum of partials), and the tile's sum of squares of the
  // new f16 values; one warp per (row, tile), lane = 4 columns
  const ChainGemm& g = a.gemms[op.gemm];
  const int tiles = a.hs / 128;
  for (int it = warp_id; it < a.rows * tiles; it += warps) {
    const int r = it / tiles, T = it - r * tiles;
    float4 acc;
    const bool lok = chain_sum4<CHAIN_MAX_SEG, true>(chain_partial(a, g, T, r, 4 * lane), slot_u64,
                                               chain_tile_segs(g, T), acc, llw, 0x752);
    if (!__all_sync(0xffffffffu, lok)) break;
    __half* hp = a.h + static_cast<size_t>(r) * a.hs + T * 128 + 4 * lane;
    const uint2 hw = __ldcg(reinterpret_cast<const uint2*>(hp));
    const float2 h01 = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
    const float2 h23 = __half22float2(*reinterpret_cast<const __half2*>(&hw.y));
    const __half2 n01 = __floats2half2_rn(__fadd_rn(h01.x, acc.x), __fadd_rn(h01.y, acc.y));
    const __half2 n23 = __floats2half2_rn(__fadd_rn(h23.x, acc.z), __fadd_rn(h23.y, acc.w));
    uint2 nw;
    nw.x = *reinterpret_cast<const uint32_t*>(&n01);
    nw.y = *reinterpret_cast<const uint32_t*>(&n23);
    __stcg(reinterpret_cast<uint2*>(hp), nw);
    ll_st16(a.hf[op.ch] + static_cast<size_t>(r) * hf_ld + (T * 128 + 4 * lane) / 2, nw.x, nw.y, flag);
    const float2 f01 = __half22float2(n01), f23 = __half22float2(n23);
    float sq = __fmul_rn(f01.x, f01.x);
    sq = __fadd_rn(sq, __fmul_rn(f01.y, f01.y));
    sq = __fadd_rn(sq, __fmul_rn(f23.x, f23.x));
    sq = __fadd_rn(sq, __fmul_rn(f23.y, f23.y));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0) ll_st8(a.ss[op.ch] + static_cast<size_t>(r) * ss_ld + T, __float_as_uint(sq), flag);
  }
}

// CH_QKV over this warp's (row, head) items (see the operation list above).
__device__ __forceinline__ void chain_qkv(const ChainArgs& a, const ChainOp& op, int warp_id, int warps, LLWait llw) {
  const int lane = threadIdx.x & 31;
  const size_t slot_u64 = static_cast<size_t>(a.ws_rows) * 128;
  // one warp per (row, head), lane = dims 4 lane .. +3; the rotate-half partner of
  // dim d (d ^ 64) sits in lane ^ 16
  const ChainGemm& g = a.gemms[op.gemm];
  const int heads = a.nq + 2 * a.nkv;
  for (int it = warp_id; it < a.rows * heads; it += warps) {
    const int r = it / heads, t = it - r * heads;
    const int d0 = 4 * lane;
    int pos, page;
    uint2 cw, sw;
    if (op.direct_meta) {  // the launch that fills the per-row copies: from the tables
      const int slot = a.row_slot[r];
      pos = a.pos[slot];
      page = a.kv.page_table[static_cast<size_t>(slot) * a.kv.max_pages + (pos >> 6)];
      cw = *reinterpret_cast<const uint2*>(a.rope_cos + static_cast<size_t>(pos) * 128 + d0);
      sw = *reinterpret_cast<const uint2*>(a.rope_sin + static_cast<size_t>(pos) * 128 + d0);
    } else {
      pos = __ldcg(a.row_pos + r);
      page = __ldcg(a.row_page + r);
      cw = __ldcg(reinterpret_cast<const uint2*>(a.row_rope + static_cast<size_t>(r) * 256 + d0));
      sw = __ldcg(reinterpret_cast<const uint2*>(a.row_rope + static_cast<size_t>(r) * 256 + 128 + d0));
    }
    float4 acc;
    const bool lok = chain_sum4<CHAIN_QKV_SEG, true>(chain_partial(a, g, t, r, 4 * lane), slot_u64,
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
      uint2 vw;
      vw.x = pack_half2(acc.x, acc.y);
      vw.y = pack_half2(acc.z, acc.w);
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
    const float4 w = *reinterpret_cast<const float4*>((t < a.nq ? op.qn_w : op.kn_w) + d0);
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
    uint2 ow;
    ow.x = pack_half2(o[0], o[1]);
    ow.y = pack_half2(o[2], o[3]);
    if (t < a.nq) {
      *reinterpret_cast<uint2*>(a.q + static_cast<size_t>(r) * a.nq * 128 + t * 128 + d0) = ow;
    } else {
      const size_t off = kv_off(0, t - a.nq);
      *reinterpret_cast<uint2*>(a.kv.pool + off + kv_dim_swizzle(pos, d0)) = ow;
    }
  }
}

template <int PROG>
__global__ void __launch_bounds__(CHAIN_THREADS, 1) decode_chain_kernel(const __grid_constant__ ChainArgs a) {
  constexpr int KSTEPS = 8;  // 128 k elements per unit, UMMA K = 16
  constexpr int EPI_WARP0 = 16 - CHAIN_EPI_WARPS;
  extern __shared__ __align__(1024) uint8_t chain_dsmem[];
  __shared__ __align__(8) uint64_t wfull_bar[CHAIN_MAX_W_STAGES], wfree_bar[CHAIN_MAX_W_STAGES];
  // unit slots: A stage (TMEM) + X tile (shared memory) of one unit.  ufull completes when
  // the four builder warps published A and the eight epilogue warps built X; ufree when
  // its MMAs retired.
  __shared__ __align__(8) uint64_t ufull_bar[CHAIN_MAX_A_STAGES], ufree_bar[CHAIN_MAX_A_STAGES];
  __shared__ __align__(8) uint64_t dfull_bar[2], dfree_bar[2], done_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ int seg_ok, bar_ok;
  __shared__ float inv_sh[CHAIN_MAX_ROWS];  // XS_NORM: 1 / rms of each row, per GEMM

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
      mbar_init(&wfree_bar[i], 4);
    }
    for (int i = 0; i < SU; ++i) {
      mbar_init(&ufull_bar[i], 4 + CHAIN_EPI_WARPS);  // 4 builder warps + 8 X-building warps
      mbar_init(&ufree_bar[i], 1);  // the commit of the issuer that took the unit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull_bar[i], NACC);
      mbar_init(&dfree_bar[i], CHAIN_EPI_WARPS);
    }
    mbar_init(&done_bar, NACC);
    abort_flag = 0;
    fence_mbar_init();
    if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 37] = globaltimer();
  }
  if (warp == 2) {
    tmem_alloc(&tmem_base_sh, GEMM_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  // Programmatic dependent launch: the previous launch (the attention merge) may still be
  // running.  Weights, scales, shared memory and TMEM never depend on it, so the producer,
  // the A builders and the MMA issuers start at once; the epilogue / row-operation warps
  // wait (griddepcontrol.wait in their own branch) before they read any activation.
  if (threadIdx.x == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 38] = globaltimer();

  if (warp < 4) {
  regs_dec<CHAIN_REGS_PRODUCER>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One thread streams the weight units of all the launch's GEMMs (16 KB bulk copies)
    // through the W ring, running ahead across GEMMs as far as the ring allows.
    if (lane == 0) {
      int wg = -1, wu = 0, wue = 0, wst = 0, wissued = 0;
      uint32_t wph = 0;
      auto w_advance = [&]() {
        while (wu >= wue && wg + 1 < n_gemm_ops) {
          ++wg;
          chain_unit_range(a.gemms[wg], blockIdx.x, wu, wue);
        }
      };
      w_advance();
      if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 39] = globaltimer();
      uint64_t t_idle = globaltimer();
      int wlanded = 0;  // copies seen complete, in issue order
      const int cap = a.w_inflight > 0 ? a.w_inflight : SW;
      while (wu < wue) {
        while (wissued - wlanded >= cap &&
               mbar_test(&wfull_bar[wlanded % SW], static_cast<uint32_t>((wlanded / SW) & 1)))
          ++wlanded;
        if (wissued - wlanded < cap && mbar_test(&wfree_bar[wst], wph ^ 1u)) {
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
            if (!mbar_wait(&ufull_bar[my_us], my_uph, &abort_flag, a.status, 0x722)) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (a.trace != nullptr && i < 24) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 40 + i] = globaltimer();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(d) * DCOLS + static_cast<uint32_t>(j) * DSTR;
            const uint32_t a_tmem = tmem_base + A_COLS0 + static_cast<uint32_t>(my_us) * 64u;
            const uint32_t x_base = smem_u32(xring + static_cast<size_t>(my_us) * x_stage_bytes);
#pragma unroll
            for (int kk = 0; kk < KSTEPS; ++kk) {
              const uint32_t b_addr = x_base + static_cast<uint32_t>(kk >> 2) * x_tile_bytes +
                                      static_cast<uint32_t>(kk & 3) * 32u;
              umma_f16_ts(d_tmem, a_tmem + static_cast<uint32_t>(kk) * 8u, smem_desc_sw128(b_addr), idesc,
                          (!started && kk == 0) ? 0u : 1u);
            }
            started = true;
            umma_commit(&ufree_bar[my_us]);
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
  }
  regs_inc<128>();  // back to the launch's count before the roles rejoin
  } else if (warp < 8) {
    regs_dec<CHAIN_REGS_BUILDER>();
    // ------------------------------------------------------------ int8 A builders
    // Each unit is published as soon as its TMEM stores land (tcgen05.wait::st is cheap);
    // the row scale of the unit's tile is loaded before the unit's barrier waits so its
    // latency overlaps them.
    const int t = (threadIdx.x - 128) & 127;  // row of the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int st = 0, ast = 0, i = 0;  // W stage, unit slot
    uint32_t ph = 0, aph = 0;
    bool ok = true;
    for (int gi = 0; gi < n_gemm_ops && ok; ++gi) {
      const ChainGemm& g = a.gemms[gi];
      int ub, ue;
      chain_unit_range(g, blockIdx.x, ub, ue);
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
        const bool f32s = g.scale32 != 0;
        const int srow = (u / g.kblocks) * 128 + t;
        const float sc32 = f32s ? static_cast<const float*>(g.scale)[srow] : 1.0f;
        const __half sc = f32s ? __float2half_rn(1.0f) : static_cast<const __half*>(g.scale)[srow];
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
        // one body per scale width: the choice is made once per unit, not per word
        auto build_row = [&](auto f32tag) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t w4[4] = {chunk[c].x, chunk[c].y, chunk[c].z, chunk[c].w};
            uint32_t outw[8];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dequant_i8x4<decltype(f32tag)::value>(w4[q], sc2, sc32, outw[2 * q], outw[2 * q + 1]);
            tmem_st_x8(taddr + static_cast<uint32_t>(c) * 8u, reinterpret_cast<const uint32_t(&)[8]>(outw));
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
      }
    }
    regs_inc<128>();
  } else {
    regs_inc<CHAIN_REGS_EPI>();
    // ------------------------------------------------------------ epilogue, X builds, row operations
    const int e = threadIdx.x - EPI_WARP0 * 32;  // 0 .. CHAIN_EPI_THREADS - 1
    const int we = warp - EPI_WARP0;
    const int row = (warp & 3) * 32 + lane;       // TMEM lane quadrant of this warp = tile row
    const int half = we >> 2;                     // two warps per quadrant split the columns
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const size_t slot_u64 = static_cast<size_t>(a.ws_rows) * 128;
    const int hf_ld = CHAIN_MAX_HS / 2, ss_ld = CHAIN_MAX_HS / 128;
    int seg = -1;
    int xs = 0;  // unit-slot cursor of the X builds (the builders and issuers walk the same units)
    uint32_t xph = 0;
    bool ok = true;
    griddep_wait();
    // this launch's flag: the step counter was written by an earlier step's last kernel
    const uint32_t flag = (*reinterpret_cast<const volatile unsigned int*>(a.epoch) << 6) |
                          static_cast<uint32_t>(a.launch_idx + 1);
    const LLWait llw{&abort_flag, a.status, flag};
    if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 66] = globaltimer();

    // CTA-wide verdict among the epilogue warps (also orders their shared-memory use)
    auto uniform_ok = [&]() -> bool {
      named_bar_sync(1, CHAIN_EPI_THREADS);
      if (e == 0) bar_ok = abort_flag ? 0 : 1;
      named_bar_sync(1, CHAIN_EPI_THREADS);
      return bar_ok != 0;
    };

    // 1 / rms of every row from the flagged per-tile sums of squares of channel ch
    // (rms_norm_row, src/cpu_decoder.rs:261-272): two rows per warp pass, lanes 16 j + t
    // hold tile t of the pass's row j; the tile sums are added in the butterfly order of
    // the group's first lane
    auto compute_inv = [&](int ch) {
      const int tiles = a.hs / 128;
      bool lok = true;
      for (int p = we; 2 * p < a.rows; p += CHAIN_EPI_WARPS) {
        const int r = 2 * p + (lane >> 4), t = lane & 15;
        float v = 0.f;
        if (r < a.rows && t < tiles && lok) {
          const uint64_t* src = a.ss[ch] + static_cast<size_t>(r) * ss_ld + t;
          uint2 w = ll_ld8(src);
          if (w.y != flag) {
            w = ll_spin8(src, llw, 0x747);
            lok = w.y == flag;
          }
          v = __uint_as_float(w.x);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((lane & 15) == 0 && r < a.rows)
          inv_sh[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, static_cast<float>(a.hs)), a.eps)));
      }
    };

    // X tiles of units u0 .. u0 + cnt - 1 (cnt <= CHAIN_X_BATCH) of GEMM g into the next
    // unit slots: rows n < rows from the source, zeros in the tiles' padding rows; the
    // 128-byte swizzle of the K-major UMMA operand (16-byte chunk c of row n at chunk
    // c ^ (n % 8), two 64-column halves).  All the batch's loads are issued before any is
    // used, so the batch costs one round trip, not one per unit.
    auto build_x = [&](const ChainGemm& g, int u0, int cnt) {
      const int items = a.n_tile * 16;
      // per unit, this thread's items (n, c) = (it >> 4, it & 15), it = j0 + e + 256 j, two at a time
      uint4 raw[CHAIN_X_BATCH][2][2];  // [unit][item][word]
      const bool flagged = g.xsrc != XS_ATTN;
      auto src_of = [&](int n, int k0) -> const uint64_t* {
        return g.xsrc == XS_NORM ? a.hf[g.xch] + static_cast<size_t>(n) * hf_ld + k0 / 2
                                 : a.actf + static_cast<size_t>(n) * (a.inter / 2) + k0 / 2;
      };
      for (int j0 = 0; j0 < items; j0 += 2 * CHAIN_EPI_THREADS) {
#pragma unroll
        for (int b = 0; b < CHAIN_X_BATCH; ++b) {
          const int kb = (u0 + b) % g.kblocks;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int it = j0 + e + j * CHAIN_EPI_THREADS;
            const int n = it >> 4, c = it & 15;
            const int k0 = kb * 128 + c * 8;
            if (b < cnt && it < items && n < a.rows) {
              if (flagged) {
                const uint64_t* src = src_of(n, k0);
                raw[b][j][0] = ll_ld16(src);
                raw[b][j][1] = ll_ld16(src + 2);
              } else {
                raw[b][j][0] = __ldcg(reinterpret_cast<const uint4*>(a.attn + static_cast<size_t>(n) * a.nq * 128 + k0));
              }
            }
          }
        }
#pragma unroll
        for (int b = 0; b < CHAIN_X_BATCH; ++b) {
          if (b >= cnt) continue;
          const int my = (xs + b) % a.a_stages;
          const uint32_t myph = xph ^ ((xs + b) >= a.a_stages ? 1u : 0u);
          if (j0 == 0 && !mbar_wait_warp(&ufree_bar[my], myph ^ 1u, &abort_flag, a.status, 0x745)) continue;
          const int kb = (u0 + b) % g.kblocks;
          const uint32_t dst = smem_u32(xring + static_cast<size_t>(my) * x_stage_bytes);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int it = j0 + e + j * CHAIN_EPI_THREADS;
            if (it >= items) continue;
            const int n = it >> 4, c = it & 15;
            const int k0 = kb * 128 + c * 8;
            uint4 out = make_uint4(0u, 0u, 0u, 0u);
            if (n < a.rows) {
              if (!flagged) {
                out = raw[b][j][0];
              } else {
                const uint64_t* src = src_of(n, k0);
                uint4 w0 = raw[b][j][0], w1 = raw[b][j][1];
                if (!(w0.y == flag && w0.w == flag)) w0 = ll_spin16(src, llw, 0x746);
                if (!(w1.y == flag && w1.w == flag)) w1 = ll_spin16(src + 2, llw, 0x746);
                if (g.xsrc == XS_ACT) {
                  out = make_uint4(w0.x, w0.z, w1.x, w1.z);
                } else {
                  const float inv = inv_sh[n];
                  const float4 wa = *reinterpret_cast<const float4*>(g.xnorm_w + k0);
                  const float4 wb = *reinterpret_cast<const float4*>(g.xnorm_w + k0 + 4);
                  const uint32_t hw[4] = {w0.x, w0.z, w1.x, w1.z};
                  const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                  uint32_t o[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const float2 hv = __half22float2(*reinterpret_cast<const __half2*>(&hw[q]));
                    o[q] = pack_half2(__fmul_rn(__fmul_rn(hv.x, inv), wv[2 * q]),
                                      __fmul_rn(__fmul_rn(hv.y, inv), wv[2 * q + 1]));
                  }
                  out = make_uint4(o[0], o[1], o[2], o[3]);
                }
              }
            }
            st_shared_v4(dst + static_cast<uint32_t>(c >> 3) * x_tile_bytes + static_cast<uint32_t>(n) * 128u +
                             (static_cast<uint32_t>((c & 7) ^ (n & 7)) << 4),
                         out);
          }
        }
      }
#pragma unroll
      for (int b = 0; b < CHAIN_X_BATCH; ++b) {
        if (b >= cnt) continue;
        const int my = (xs + b) % a.a_stages;
        fence_proxy_async_shared();  // the MMA reads the tile through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(&ufull_bar[my]);
      }
      xs += cnt;
      if (xs >= a.a_stages) {
        xs -= a.a_stages;
        xph ^= 1u;
      }
    };
    // all units [x0, x1) of GEMM g, in batches
    auto build_xs = [&](const ChainGemm& g, int x0, int x1) {
      for (int u = x0; u < x1; u += CHAIN_X_BATCH) build_x(g, u, min(CHAIN_X_BATCH, x1 - u));
    };

    // The launch's operations as straight-line code (the program is a template parameter):
    // each operation's set-up then lives only while it runs, and nothing is hoisted into
    // state held across all of them.
    auto op_gemm = [&](const ChainOp& op, int gi) {
      (void)op;
      const ChainGemm& g = a.gemms[gi];
      int ub, ue;
      chain_unit_range(g, blockIdx.x, ub, ue);
      auto seg_end_of = [&](int uu) { return min(ue, (uu / g.kblocks + 1) * g.kblocks); };
      if (ub < ue && g.xsrc == XS_NORM) {
        compute_inv(g.xch);
        named_bar_sync(1, CHAIN_EPI_THREADS);  // inv_sh complete
      }
      // X tiles of the first segment, then per segment: the next segment's X tiles, then
      // this segment's accumulators (so the issuers always have work queued)
      int xu = ub;
      if (ub < ue) {
        build_xs(g, xu, seg_end_of(ub));
        xu = seg_end_of(ub);
        if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 25 + gi] = globaltimer();
      }
      int u = ub;
      while (u < ue) {
        const int T = u / g.kblocks;
        const int seg_end = seg_end_of(u);
        if (xu < ue) {
          const int ne = seg_end_of(xu);
          build_xs(g, xu, ne);
          xu = ne;
        }
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
          break;
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
    auto op_embed = [&](const ChainOp& op) {
      // h[r] = embed row of the slot's input token: one warp per (row, 128-column tile),
      // lane = 4 columns; the plain copy for the later launches, the flagged copy and the
      // tile's sum of squares for this launch's norm
      const int tiles = a.hs / 128;
      for (int it = blockIdx.x * CHAIN_EPI_WARPS + we; it < a.rows * tiles; it += gridDim.x * CHAIN_EPI_WARPS) {
        const int r = it / tiles, T = it - r * tiles;
        const int slot = a.row_slot[r];
        int tok = a.next_tok[slot];
        if (tok < 0 || tok >= a.vocab) {
          if (T == 0 && lane == 0) report_error(a.status, DEVERR_BOUNDS, 0x751);
          tok = 0;
        }
        const int pos = a.pos[slot];
        if (T == 0) {
          if (lane == 0) {
            a.row_pos[r] = pos;
            a.row_page[r] = a.kv.page_table[static_cast<size_t>(slot) * a.kv.max_pages + (pos >> 6)];
          }
          // cos | sin rows of the position, 16 bytes per lane
          const __half* rs = (lane < 16 ? a.rope_cos : a.rope_sin) + static_cast<size_t>(pos) * 128 + (lane & 15) * 8;
          __stcg(reinterpret_cast<uint4*>(a.row_rope + static_cast<size_t>(r) * 256 + lane * 8),
                 *reinterpret_cast<const uint4*>(rs));
        }
        const int c = T * 128 + 4 * lane;
        const uint2 hw = *reinterpret_cast<const uint2*>(a.embed + static_cast<size_t>(tok) * a.hs + c);
        __stcg(reinterpret_cast<uint2*>(a.h + static_cast<size_t>(r) * a.hs + c), hw);
        ll_st16(a.hf[op.ch] + static_cast<size_t>(r) * hf_ld + c / 2, hw.x, hw.y, flag);
        const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
        const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&hw.y));
        float sq = __fmul_rn(f01.x, f01.x);
        sq = __fadd_rn(sq, __fmul_rn(f01.y, f01.y));
        sq = __fadd_rn(sq, __fmul_rn(f23.x, f23.x));
        sq = __fadd_rn(sq, __fmul_rn(f23.y, f23.y));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) ll_st8(a.ss[op.ch] + static_cast<size_t>(r) * ss_ld + T, __float_as_uint(sq), flag);
      }
    };
    auto op_norm = [&](const ChainOp& op) {
      // norm_out[r] = f16(h * inv * w) from channel ch (rms_norm_row,
      // src/cpu_decoder.rs:261-272); one warp per (row, tile)
      const int tiles = a.hs / 128;
      for (int it = blockIdx.x * CHAIN_EPI_WARPS + we; it < a.rows * tiles; it += gridDim.x * CHAIN_EPI_WARPS) {
        const int r = it / tiles, T = it - r * tiles;
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
        const int c = T * 128 + 4 * lane;
        uint4 hv[1];
        lok = ll_get16<1>(a.hf[op.ch] + static_cast<size_t>(r) * hf_ld + c / 2, 2, 1, hv, llw, 0x754) && lok;
        if (!__all_sync(0xffffffffu, lok)) break;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        t = __shfl_sync(0xffffffffu, t, 0);  // lane 0's order, the same value everywhere
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(a.hs)), a.eps)));
        const float2 h01 = __half22float2(*reinterpret_cast<const __half2*>(&hv[0].x));
        const float2 h23 = __half22float2(*reinterpret_cast<const __half2*>(&hv[0].z));
        const float4 w = *reinterpret_cast<const float4*>(op.norm_w + c);
        uint2 xw;
        xw.x = pack_half2(__fmul_rn(__fmul_rn(h01.x, inv), w.x), __fmul_rn(__fmul_rn(h01.y, inv), w.y));
        xw.y = pack_half2(__fmul_rn(__fmul_rn(h23.x, inv), w.z), __fmul_rn(__fmul_rn(h23.y, inv), w.w));
        __stcg(reinterpret_cast<uint2*>(op.norm_out + static_cast<size_t>(r) * a.hs + c), xw);
      }
    };
    auto op_silu = [&](const ChainOp& op) {
      // gate|up tile t: rows [0, 64) gate[64 t + i], rows [64, 128) up[64 t + i].  Work
      // unit: 4 outputs (row r, tile t, quad c); each thread takes every (G * 256)-th one.
      const ChainGemm& g = a.gemms[op.gemm];
      const int tiles = g.units / g.kblocks;
      const int total = a.rows * tiles * 16;
      const int stride = gridDim.x * CHAIN_EPI_THREADS;
      for (int q = blockIdx.x * CHAIN_EPI_THREADS + e; q < total; q += stride) {
        const int c = q & 15, rt = q >> 4;
        const int r = rt / tiles, t = rt - r * tiles;
        const int nseg = chain_tile_segs(g, t);
        const uint64_t* p = chain_partial(a, g, t, r, 4 * c);
        float4 gs, us;
        bool lok = chain_sum4<CHAIN_SILU_SEG, false>(p, slot_u64, nseg, gs, llw, 0x755);
        lok = chain_sum4<CHAIN_SILU_SEG, false>(p + 64, slot_u64, nseg, us, llw, 0x756) && lok;
        if (!lok) break;
        const float gv[4] = {gs.x, gs.y, gs.z, gs.w}, uv[4] = {us.x, us.y, us.z, us.w};
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float gt = f16_round(gv[j]);
          const float silu = __fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt)));
          o[j] = __fmul_rn(silu, f16_round(uv[j]));
        }
        ll_st16(a.actf + static_cast<size_t>(r) * (a.inter / 2) + (t * 64 + 4 * c) / 2, pack_half2(o[0], o[1]),
                pack_half2(o[2], o[3]), flag);
      }
    };
    // after operation oi: a CTA-wide verdict of the epilogue warps (no grid barrier: the
    // next operation waits for exactly the flagged words it reads)
    auto next = [&](int oi) {
      if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * oi] = globaltimer();
      if (!uniform_ok()) ok = false;
      if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 2 + 2 * oi] = globaltimer();
      return ok;
    };
    const int wid = blockIdx.x * CHAIN_EPI_WARPS + we, nwarps = gridDim.x * CHAIN_EPI_WARPS;
    if constexpr (PROG == CHAIN_PROG_FIRST) {
      // embed + layer 0's input norm -> QKV GEMM -> q/k norm + RoPE + K/V append
      op_embed(a.ops[0]);
      if (next(0)) op_gemm(a.ops[1], 0);
      if (next(1)) chain_qkv(a, a.ops[2], wid, nwarps, llw);
      if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * 2] = globaltimer();
    } else {
      // o_proj -> residual -> gate|up -> SiLU -> down -> residual -> (QKV + q/k norm, RoPE,
      // K/V append | the final norm)
      op_gemm(a.ops[0], 0);
      if (next(0)) chain_resid(a, a.ops[1], wid, nwarps, llw);
      if (next(1)) op_gemm(a.ops[2], 1);
      if (next(2)) op_silu(a.ops[3]);
      if (next(3)) op_gemm(a.ops[4], 2);
      if (next(4)) chain_resid(a, a.ops[5], wid, nwarps, llw);
      if constexpr (PROG == CHAIN_PROG_MIDDLE) {
        if (next(5)) op_gemm(a.ops[6], 3);
        if (next(6)) chain_qkv(a, a.ops[7], wid, nwarps, llw);
        if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * 7] = globaltimer();
      } else {
        if (next(5)) op_norm(a.ops[6]);
        if (e == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * 6] = globaltimer();
      }
    }
    regs_dec<128>();
  }

  griddep_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, GEMM_TMEM_COLS);
  if (threadIdx.x == 0 && a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + CHAIN_TRACE_SLOTS - 1] = globaltimer();
}

}  // namespace qasr
