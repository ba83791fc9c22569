// Weight-streaming GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   out[r, m] = epilogue( sum_k  W[m, k] * X[r, k] )      W: [n_out, K] f16 or int8
//                                                          X: [rows, K] f16 (activations)
//
// This replaces the reference's decoder GEMVs/GEMMs: gemv / gemv_w8 / gemv_norm /
// gemv_batch_slots / prefill_gemm(_w8) (src/shaders.rs:273-1132, 2995-3082).  It is
// "swap-AB": the weight rows are the UMMA M dimension (tiles of 128 rows) and the
// activation rows (decode slots or prefill rows) are N (16..128 per tile), so a decode
// step with B slots reads every weight byte once, whatever B is.
//
// Roles of the CTA (one persistent CTA per SM):
//   warp 0      producer: one 16 KB bulk copy per weight unit (128 rows x 128 B, stored
//               pre-tiled and pre-swizzled in HBM) + TMA of the activation tile(s)
//   warp 1      UMMA issuer: tcgen05.mma kind::f16, f32 accumulators in TMEM
//   warp 2      TMEM allocator (512 columns)
//   f16 weights: the weight tile in shared memory already is the canonical K-major
//               128-byte-swizzled operand, so A is read straight from shared memory.
//   int8 weights: two warpgroups of "A builders" (warps 4-11) take alternate units:
//               each thread reads one W row from the swizzled tile, dequantises it to
//               f16(f32(q) * scale) (the value dequant_i8 produces, src/weights.rs:372-385;
//               see dequant_i8x4) and stores the row into TMEM, which the MMA then reads as
//               its A operand.
//   last 4 warps  epilogue: TMEM accumulators -> fused epilogue (see EpiKind)
//
// Work split: the (tile, k-block) units are cut into equal contiguous ranges, one per
// CTA ("stream-K").  A tile split across CTAs is finished by the CTA that arrives last
// on the tile's counter; it adds the f32 partials in segment order, so results do not
// depend on arrival order.  No CTA ever waits on another.
#pragma once
#include <type_traits>
#include "device_common.cuh"

namespace qasr {

enum EpiKind : int {
  EPI_STORE = 0,   // out[r, m] = f16(acc)
  EPI_RESID = 1,   // h[r, m] = f16(f32(h[r, m]) + acc)  (batch_dot_acc, src/cpu_decoder.rs:45-62)
  EPI_SILU = 2,    // interleaved gate|up tiles -> f16(silu(f16 g) * f16 u) (src/cpu_decoder.rs:442-448)
  EPI_QKV = 3,     // per-head q/k RMSNorm + rotate-half RoPE; Q -> q_out, K and raw V -> paged KV
  EPI_LOGITS = 4,  // f32 logits (optional) + per-row argmax via 64-bit atomicMax keys
  // audio tower (CpuAudioLinear::forward + the ops that follow it, src/audio_encoder.rs:117-131);
  // `bias` may be null (no bias add)
  EPI_BIAS_F16 = 5,      // out[r, m] = f16(acc + bias[m])
  EPI_BIAS_GELU = 6,     // out[r, m] = f16(gelu(acc + bias[m])), gelu = 0.5 x (1 + erf(x / sqrt 2))
  EPI_BIAS_F32 = 7,      // out32[r, m] = acc + bias[m]
};

constexpr int GEMM_BUILD_GROUPS = 2;  // int8 A-builder warpgroups
__host__ __device__ constexpr int gemm_threads(bool int8) {
  return 128 + (int8 ? GEMM_BUILD_GROUPS * 128 : 0) + 128;
}
constexpr int GEMM_MAX_STAGES = 12;
constexpr int GEMM_A_STAGES = 8;  // upper bound; the kernel fits what TMEM allows
constexpr int GEMM_MAX_NTILE = 128;
constexpr int GEMM_WIDE_NTILE = 256;  // f16 only: 2 x 256 accumulator columns fill the TMEM
constexpr uint32_t GEMM_TMEM_COLS = 512;

struct KvLayout {
  __half* pool;             // [pages][layers][2][nkv][64][head_dim]
  const int* page_table;    // [slots][max_pages]
  int max_pages;
  int layers;
  int nkv;
};

// Within a page, position p's 128 dims are one 256-byte row whose 16-byte chunk c is
// stored at chunk c ^ (p & 7): eight consecutive positions of one chunk then sit in eight
// different bank groups, which makes the attention kernel's ldmatrix reads conflict-free.
__host__ __device__ __forceinline__ int kv_dim_swizzle(int pos, int d) {
  return ((((d >> 3) ^ (pos & 7)) << 3) | (d & 7));
}

// Offset of the 128-dim row of (slot, pos) in the pool; add kv_dim_swizzle(pos, d).
__device__ __forceinline__ size_t kv_elem_offset(const KvLayout& kv, int slot, int pos, int layer,
                                                 int which, int kvh) {
  const int page = kv.page_table[static_cast<size_t>(slot) * kv.max_pages + (pos >> 6)];
  return ((((static_cast<size_t>(page) * kv.layers + layer) * 2 + which) * kv.nkv + kvh) * 64 +
          (pos & 63)) *
         128;
}

struct GemmArgs {
  int n_out, k, rows, n_tile, n_tiles, kblocks, units, grid, stages, max_seg;
  const uint8_t* w_tiles;  // weights in the tiled layout (weight_tile_offset)
  const void* scale;       // int8: per-row scale, f16 or (scale32) f32
  int scale32;
  // epilogue
  int epi;
  __half* out;
  int ldo;
  // EPI_QKV
  const float* qn_w;
  const float* kn_w;
  const __half* rope_cos;
  const __half* rope_sin;
  const int* row_slot;
  const int* row_pos;
  KvLayout kv;
  int layer;
  __half* q_out;
  int q_ld;
  float eps;
  // EPI_LOGITS
  float* logits;
  int ld_logits;
  unsigned long long* best;
  // EPI_BIAS_*
  const float* bias;
  float* out32;
  int ldo32;
  // split tiles
  float* ws;
  int* counters;
  uint32_t* status;
  // optional latency trace: per CTA GEMM_TRACE_SLOTS %globaltimer stamps (diagnostics)
  unsigned long long* trace;
};

constexpr int GEMM_TRACE_SLOTS = 12;
// trace slots: 0 entry, 1 setup done, 2 first W issued, 3 first X issued, 4 first W seen by
// the A builders, 5 first A stage built, 6 first MMA issued, 7 last MMA issued, 8 first
// accumulator seen by the epilogue, 9 last tile stored / partial written, 10 split fixup done,
// 11 exit
__device__ __forceinline__ void trace_stamp(const GemmArgs& a, int slot) {
  if (a.trace != nullptr) a.trace[blockIdx.x * GEMM_TRACE_SLOTS + slot] = globaltimer();
}

__device__ __forceinline__ int cta_of_unit(long long x, long long units, long long grid) {
  // CTA c owns units [c*U/G, (c+1)*U/G); the owner of x is the largest c with c*U/G <= x.
  // Unsigned 32-bit arithmetic ((x + 1) * G + U <= 2 U G < 2^32 for every GEMM of these
  // models: U <= 19K units, G <= the SM count); a 64-bit division is a slow software routine.
  const unsigned int xu = static_cast<unsigned int>(x), U = static_cast<unsigned int>(units),
                     G = static_cast<unsigned int>(grid);
  return static_cast<int>(((xu + 1u) * G + U - 1u) / U) - 1;
}

// Four int8 weights (one little-endian word, byte j = value j) -> f16(f32(q) * s) as two
// packed f16 pairs (values 0,1 and 2,3).  q + 1152 is built exactly as an f16 by byte
// placement and the bias subtracted exactly.  An f16 scale: q * s is exact in f32
// (8 x 11 significant bits), so one f16 multiply rounds it once, as f16(f32(q) * s).  An
// f32 scale (the INT8 export's `.weight_scale`, PackedInt8 src/weights.rs:309-356): the
// f32 product, then the f16 rounding — both of the reference's roundings.
template <bool F32S>
__device__ __forceinline__ void dequant_i8x4(uint32_t w, __half2 s16, float s32, uint32_t& o01, uint32_t& o23) {
  const __half2 bias = __floats2half2_rn(1152.0f, 1152.0f);
  const uint32_t ub8 = w ^ 0x80808080u;  // q + 128 as unsigned bytes
  uint32_t lo = __byte_perm(ub8, 0x64646464u, 0x4140);
  uint32_t hi = __byte_perm(ub8, 0x64646464u, 0x4342);
  __half2 hl = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);  // exact q
  __half2 hh = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
  if constexpr (F32S) {
    const float2 fl = __half22float2(hl), fh = __half22float2(hh);
    hl = __floats2half2_rn(__fmul_rn(fl.x, s32), __fmul_rn(fl.y, s32));
    hh = __floats2half2_rn(__fmul_rn(fh.x, s32), __fmul_rn(fh.y, s32));
  } else {
    hl = __hmul2_rn(hl, s16);
    hh = __hmul2_rn(hh, s16);
  }
  o01 = *reinterpret_cast<uint32_t*>(&hl);
  o23 = *reinterpret_cast<uint32_t*>(&hh);
}

// ------------------------------------------------------------------ epilogues
struct EpiSmem {
  float red[4][16];
  float xs[16][128];
  int last_flag;
};

__device__ __forceinline__ void warp_sum16(float (&s)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, EpiSmem& es, int mt, int nt,
                                               int c0, int e, const float (&v)[16]) {
  const int warp_e = e >> 5;
  const int lane = e & 31;
  const int nbase = nt * a.n_tile + c0;
  if constexpr (EPI == EPI_STORE) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = nbase + j;
      if (n < a.rows) a.out[static_cast<size_t>(n) * a.ldo + mt * 128 + e] = __float2half_rn(v[j]);
    }
  } else if constexpr (EPI == EPI_RESID) {
    // all 16 residual reads in flight before the first write (a read after a write to the
    // same array would otherwise wait for it)
    __half old[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = nbase + j;
      old[j] = n < a.rows ? a.out[static_cast<size_t>(n) * a.ldo + mt * 128 + e] : __float2half_rn(0.0f);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = nbase + j;
      if (n < a.rows)
        a.out[static_cast<size_t>(n) * a.ldo + mt * 128 + e] = __float2half_rn(__fadd_rn(__half2float(old[j]), v[j]));
    }
  } else if constexpr (EPI == EPI_SILU) {
    // tile mt: rows [0,64) = gate[mt*64 + i], rows [64,128) = up[mt*64 + i]
    if (e >= 64) {
#pragma unroll
      for (int j = 0; j < 16; ++j) es.xs[j][e - 64] = f16_round(v[j]);
    }
    named_bar_sync(1, 128);
    if (e < 64) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = nbase + j;
        if (n < a.rows) {
          const float g = f16_round(v[j]);
          const float u = es.xs[j][e];
          const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
          a.out[static_cast<size_t>(n) * a.ldo + mt * 64 + e] = __float2half_rn(__fmul_rn(silu, u));
        }
      }
    }
    named_bar_sync(1, 128);
  } else if constexpr (EPI == EPI_QKV) {
    // tile mt = one head: 0..15 q, 16..23 k, 24..31 v (fused [q|k|v] rows)
    const int nq = a.q_ld / 128;
    if (mt >= nq + a.kv.nkv) {  // V: raw f16 projection into the cache
      const int kvh = mt - nq - a.kv.nkv;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = nbase + j;
        if (n < a.rows) {
          const size_t off = kv_elem_offset(a.kv, a.row_slot[n], a.row_pos[n], a.layer, 1, kvh);
          a.kv.pool[off + kv_dim_swizzle(a.row_pos[n], e)] = __float2half_rn(v[j]);
        }
      }
      return;
    }
    float x[16], s[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      x[j] = f16_round(v[j]);
      s[j] = __fmul_rn(x[j], x[j]);
    }
    warp_sum16(s);
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < 16; ++j) es.red[warp_e][j] = s[j];
    }
    named_bar_sync(1, 128);
    const float w = (mt < nq ? a.qn_w : a.kn_w)[e];
    float xn[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float sum2 = (es.red[0][j] + es.red[1][j]) + (es.red[2][j] + es.red[3][j]);
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum2, 128.0f), a.eps)));
      xn[j] = __fmul_rn(__fmul_rn(x[j], inv), w);
      es.xs[j][e] = xn[j];
    }
    named_bar_sync(1, 128);
    const float sign = e < 64 ? -1.0f : 1.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = nbase + j;
      if (n < a.rows) {
        const int pos = a.row_pos[n];
        const float c = __half2float(a.rope_cos[static_cast<size_t>(pos) * 128 + e]);
        const float sn = __half2float(a.rope_sin[static_cast<size_t>(pos) * 128 + e]);
        const float xp = es.xs[j][e ^ 64];
        const float o = __fadd_rn(__fmul_rn(xn[j], c), __fmul_rn(__fmul_rn(sign, xp), sn));
        const __half oh = __float2half_rn(o);
        if (mt < nq) {
          a.q_out[static_cast<size_t>(n) * a.q_ld + mt * 128 + e] = oh;
        } else {
          const size_t off = kv_elem_offset(a.kv, a.row_slot[n], pos, a.layer, 0, mt - nq);
          a.kv.pool[off + kv_dim_swizzle(pos, e)] = oh;
        }
      }
    }
    named_bar_sync(1, 128);
  } else if constexpr (EPI == EPI_BIAS_F16 || EPI == EPI_BIAS_GELU || EPI == EPI_BIAS_F32) {
    const int m = mt * 128 + e;
    const float b = a.bias != nullptr ? a.bias[m] : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = nbase + j;  // warp-uniform
      if (n < a.rows) {
        const float y = a.bias != nullptr ? __fadd_rn(v[j], b) : v[j];
        if constexpr (EPI == EPI_BIAS_F16) {
          a.out[static_cast<size_t>(n) * a.ldo + m] = __float2half_rn(y);
        } else if constexpr (EPI == EPI_BIAS_GELU) {
          const float g = __fmul_rn(__fmul_rn(0.5f, y), __fadd_rn(1.0f, erff(__fmul_rn(y, 0.70710678118654752f))));
          a.out[static_cast<size_t>(n) * a.ldo + m] = __float2half_rn(g);
        } else {
          a.out32[static_cast<size_t>(n) * a.ldo32 + m] = y;
        }
      }
    }
  } else if constexpr (EPI == EPI_LOGITS) {
    const uint32_t vocab_row = static_cast<uint32_t>(mt * 128 + e);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = nbase + j;  // warp-uniform
      if (n < a.rows) {
        if (a.logits != nullptr) a.logits[static_cast<size_t>(n) * a.ld_logits + vocab_row] = v[j];
        unsigned long long key = argmax_key(v[j], vocab_row);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
          key = other > key ? other : key;
        }
        if (lane == 0) atomicMax(a.best + n, key);
      }
    }
  }
}

// ------------------------------------------------------------------ weight tiles
// HBM layout of a weight matrix [n_out, K] (1-byte int8 or 2-byte f16): unit (mt, kb) =
// rows [128 mt, +128) x bytes [128 kb, +128) of each row, stored as one contiguous
// 16 KB block at ((mt * KB + kb) * 16384), row r at r * 128, and 16-byte chunk c of the
// row at chunk position c ^ (r & 7) — the 128-byte swizzle the shared-memory tile uses,
// so one cp.async.bulk lands it ready for the A builders (no strided 128-row gather).
__device__ __forceinline__ size_t weight_tile_offset(int row, int chunk16, int kb_per_row) {
  const int mt = row >> 7, r = row & 127;
  const int kb = chunk16 >> 3, c = chunk16 & 7;
  return (static_cast<size_t>(mt) * kb_per_row + kb) * 16384 + static_cast<size_t>(r) * 128 +
         static_cast<size_t>((c ^ (r & 7)) << 4);
}

static __global__ void pack_weight_tiles_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                         int n_out, int row_bytes) {
  const int chunks = row_bytes >> 4;
  const long long total = static_cast<long long>(n_out) * chunks;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / chunks), ch = static_cast<int>(i % chunks);
    dst[weight_tile_offset(row, ch, row_bytes >> 7) >> 4] = src[i];
  }
}

// ------------------------------------------------------------------ PDL
// Programmatic dependent launch: a kernel may start while its predecessor drains; it
// must execute griddep_wait() before touching anything the predecessor produces or
// consumes.  Weights, scales and tables are constant during a step and may be read
// before it.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ kernel
// Position in the (tile, k-block) unit order, advanced without divisions (the
// single-thread producer / MMA loops must not spend hundreds of cycles per unit).
struct UnitCursor {
  int kb, mt, nt, KB, NT;
  __device__ __forceinline__ UnitCursor(int u, int KB_, int NT_) : KB(KB_), NT(NT_) {
    const int T = u / KB_;
    kb = u - T * KB_;
    mt = T / NT_;
    nt = T - mt * NT_;
  }
  __device__ __forceinline__ void advance() {
    if (++kb == KB) {
      kb = 0;
      if (++nt == NT) {
        nt = 0;
        ++mt;
      }
    }
  }
};

template <bool INT8, int EPI>
__global__ void __launch_bounds__(gemm_threads(INT8), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ GemmArgs a) {
  constexpr int NBG = INT8 ? GEMM_BUILD_GROUPS : 0;  // builder warpgroups
  constexpr int EPI_WARP0 = 4 + 4 * NBG;
  constexpr int KE = INT8 ? 128 : 64;        // k elements per unit (128 bytes of W row)
  constexpr int ATOMS = INT8 ? 2 : 1;        // 64-element (128-byte) X atoms per unit
  constexpr uint32_t ACOLS = KE / 2;         // TMEM columns of one A stage (2 f16 / column)
  constexpr int KSTEPS = KE / 16;            // UMMA K = 16 per instruction

  extern __shared__ __align__(1024) uint8_t dsmem[];
  __shared__ __align__(8) uint64_t wfull_bar[GEMM_MAX_STAGES], xfull_bar[GEMM_MAX_STAGES],
      sfree_bar[GEMM_MAX_STAGES];
  __shared__ __align__(8) uint64_t afull_bar[GEMM_A_STAGES], afree_bar[GEMM_A_STAGES];
  __shared__ __align__(8) uint64_t dfull_bar[2], dfree_bar[2], done_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ EpiSmem es;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const uint32_t x_tile_bytes = static_cast<uint32_t>(a.n_tile) * 128u;
  const uint32_t stage_bytes = 16384u + ATOMS * x_tile_bytes;
  // TMEM: two accumulator buffers of DCOLS columns, then SA dequantised A stages
  const uint32_t DCOLS = (static_cast<uint32_t>(a.n_tile) + 31u) & ~31u;
  const uint32_t A_COLS0 = 2u * DCOLS;
  int SA = static_cast<int>((GEMM_TMEM_COLS - A_COLS0) / ACOLS);
  SA = SA > GEMM_A_STAGES ? GEMM_A_STAGES : SA;
  if (!INT8) SA = 1;  // unused: A comes from shared memory

  const long long U = a.units, G = a.grid;
  const long long ub = static_cast<long long>(blockIdx.x) * U / G;
  const long long ue = static_cast<long long>(blockIdx.x + 1) * U / G;
  const int KB = a.kblocks;

  if (threadIdx.x == 0) {
    trace_stamp(a, 0);
    for (int i = 0; i < S; ++i) {
      mbar_init(&wfull_bar[i], 1);
      mbar_init(&xfull_bar[i], 1);
      mbar_init(&sfree_bar[i], 1);
    }
    for (int i = 0; i < SA; ++i) {
      mbar_init(&afull_bar[i], 4);
      mbar_init(&afree_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull_bar[i], 1);
      mbar_init(&dfree_bar[i], 4);
    }
    mbar_init(&done_bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&tmem_base_sh, GEMM_TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm_x);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch_dependents();
  const uint32_t tmem_base = tmem_base_sh;
  if (threadIdx.x == 0) trace_stamp(a, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int n = static_cast<int>(ue - ub);
      const int pre = n < S ? n : S;
      UnitCursor cw(static_cast<int>(ub), KB, a.n_tiles), cx = cw;
      auto issue_w = [&](int st, const UnitCursor& c) {
        uint64_t* bar = &wfull_bar[st];
        mbar_arrive_expect_tx(bar, 16384u);
        bulk_load(smem + static_cast<size_t>(st) * stage_bytes,
                  a.w_tiles + (static_cast<size_t>(c.mt) * KB + c.kb) * 16384, 16384u, bar);
      };
      auto issue_x = [&](int st, const UnitCursor& c) {
        uint64_t* bar = &xfull_bar[st];
        uint8_t* dst = smem + static_cast<size_t>(st) * stage_bytes + 16384;
        mbar_arrive_expect_tx(bar, ATOMS * x_tile_bytes);
#pragma unroll
        for (int at = 0; at < ATOMS; ++at)
          tma_load_2d(dst + at * x_tile_bytes, &tm_x, bar, c.kb * KE + at * 64, c.nt * a.n_tile);
      };
      // weights do not depend on the previous kernel: stream the first stages at once
      for (int i = 0; i < pre; ++i) {
        issue_w(i, cw);
        cw.advance();
      }
      trace_stamp(a, 2);
      griddep_wait();
      for (int i = 0; i < pre; ++i) {
        issue_x(i, cx);
        cx.advance();
      }
      trace_stamp(a, 3);
      int st = pre == S ? 0 : pre;
      uint32_t ph = pre == S ? 1u : 0u;  // phase index parity of unit i = i / S
      int i = pre;
      for (; i < n; ++i) {
        if (!mbar_wait(&sfree_bar[st], ph ^ 1u, &abort_flag, a.status, 0x101)) break;
        issue_w(st, cw);
        issue_x(st, cx);
        cw.advance();
        cx.advance();
        if (++st == S) {
          st = 0;
          ph ^= 1u;
        }
      }
      // drain: every issued copy lands before the CTA may exit (slot j last held unit
      // i_j = the largest issued unit index congruent to j)
      const int issued = i;
      for (int j = 0; j < S && j < issued; ++j) {
        const int il = issued - 1 - ((issued - 1 - j) % S);
        const uint32_t pj = static_cast<uint32_t>((il / S) & 1);
        mbar_wait(&wfull_bar[j], pj, nullptr, a.status, 0x102);
        mbar_wait(&xfull_bar[j], pj, nullptr, a.status, 0x103);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16_m128(static_cast<uint32_t>(a.n_tile));
      const int n = static_cast<int>(ue - ub);
      UnitCursor c(static_cast<int>(ub), KB, a.n_tiles);
      int st = 0, ast = 0, seg = -1, d = 0;
      uint32_t ph = 0, aph = 0;
      bool issued_any = false;
      for (int i = 0; i < n; ++i) {
        const bool first = (i == 0) || (c.kb == 0);
        const bool last = (i == n - 1) || (c.kb == KB - 1);
        if (first) {
          ++seg;
          d = seg & 1;
          if (!mbar_wait(&dfree_bar[d], static_cast<uint32_t>(((seg >> 1) & 1) ^ 1), &abort_flag,
                         a.status, 0x201))
            break;
          tc_fence_after();
        }
        if (INT8) {
          if (!mbar_wait(&afull_bar[ast], aph, &abort_flag, a.status, 0x202)) break;
        } else {
          if (!mbar_wait(&wfull_bar[st], ph, &abort_flag, a.status, 0x205)) break;
        }
        if (!mbar_wait(&xfull_bar[st], ph, &abort_flag, a.status, 0x203)) break;
        tc_fence_after();
        if (i == 0) trace_stamp(a, 6);
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(d) * DCOLS;
        const uint32_t w_base = smem_u32(smem + static_cast<size_t>(st) * stage_bytes);
        const uint32_t x_base = w_base + 16384u;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          const uint32_t b_addr = x_base + static_cast<uint32_t>(kk >> 2) * x_tile_bytes +
                                  static_cast<uint32_t>(kk & 3) * 32u;
          const uint32_t acc = (first && kk == 0) ? 0u : 1u;
          if constexpr (INT8) {
            const uint32_t a_tmem = tmem_base + A_COLS0 + static_cast<uint32_t>(ast) * ACOLS;
            umma_f16_ts(d_tmem, a_tmem + static_cast<uint32_t>(kk) * 8u, smem_desc_sw128(b_addr), idesc, acc);
          } else {
            umma_f16_ss(d_tmem, smem_desc_sw128(w_base + static_cast<uint32_t>(kk) * 32u),
                        smem_desc_sw128(b_addr), idesc, acc);
          }
        }
        umma_commit(&sfree_bar[st]);
        if (INT8) umma_commit(&afree_bar[ast]);
        if (last) umma_commit(&dfull_bar[d]);
        issued_any = true;
        c.advance();
        if (++st == S) {
          st = 0;
          ph ^= 1u;
        }
        if (++ast == SA) {
          ast = 0;
          aph ^= 1u;
        }
      }
      if (issued_any) {  // all MMAs must retire before the TMEM is released
        trace_stamp(a, 7);
        umma_commit(&done_bar);
        mbar_wait(&done_bar, 0, nullptr, a.status, 0x204);
      }
    }
  } else if (INT8 && warp >= 4 && warp < EPI_WARP0) {
    // ------------------------------------------------------------ A builders
    const int grp = (warp - 4) >> 2;                // this warpgroup builds units grp, grp+NBG, ...
    const int t = (threadIdx.x - 128) & 127;        // row of the 128-row tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int n = static_cast<int>(ue - ub);
    UnitCursor cur(static_cast<int>(ub) + grp, KB, a.n_tiles);
    int st = grp % S, ast = grp % SA;
    uint32_t ph = static_cast<uint32_t>((grp / S) & 1), aph = static_cast<uint32_t>((grp / SA) & 1);
    int cur_mt = -1, pend_ast = -1;
    __half2 sc2 = __floats2half2_rn(1.0f, 1.0f);
    float sc32 = 1.0f;
    const bool f32s = a.scale32 != 0;
    for (int i = grp; i < n; i += NBG) {
      if (!mbar_wait_warp(&wfull_bar[st], ph, &abort_flag, a.status, 0x301)) break;
      if (!mbar_wait_warp(&afree_bar[ast], aph ^ 1u, &abort_flag, a.status, 0x302)) break;
      tc_fence_after();
      if (i == 0 && t == 0) trace_stamp(a, 4);
      const int mt = cur.mt;
      if (INT8 && mt != cur_mt) {
        if (f32s) {
          sc32 = static_cast<const float*>(a.scale)[mt * 128 + t];
        } else {
          const __half sc = static_cast<const __half*>(a.scale)[mt * 128 + t];
          sc2 = __halves2half2(sc, sc);
        }
        cur_mt = mt;
      }
      const uint8_t* row = smem + static_cast<size_t>(st) * stage_bytes + t * 128;
      const uint32_t taddr = tmem_base + lane_base + A_COLS0 + static_cast<uint32_t>(ast) * ACOLS;
      // one body per scale width: the choice is made once per unit, not per word
      auto build_row = [&](auto f32tag) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 chunk = *reinterpret_cast<const uint4*>(row + ((c ^ (t & 7)) << 4));
          if constexpr (INT8) {
            const uint32_t w4[4] = {chunk.x, chunk.y, chunk.z, chunk.w};
            uint32_t outw[8];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dequant_i8x4<decltype(f32tag)::value>(w4[q], sc2, sc32, outw[2 * q], outw[2 * q + 1]);
            tmem_st_x8(taddr + static_cast<uint32_t>(c) * 8u, reinterpret_cast<const uint32_t(&)[8]>(outw));
          } else {
            const uint32_t w4[4] = {chunk.x, chunk.y, chunk.z, chunk.w};
            tmem_st_x4(taddr + static_cast<uint32_t>(c) * 4u, w4);
          }
        }
      };
      if (INT8 && f32s) build_row(std::true_type{});
      else build_row(std::false_type{});
      // Publish two built units per wait: the TMEM store round trip is paid once for both.
      // (Needs S >= NBG + 1 and SA >= NBG + 1 so the unit built next never waits on the
      // pending one; the host guarantees both.)
      if (pend_ast >= 0 || i + NBG >= n) {
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (pend_ast >= 0) mbar_arrive(&afull_bar[pend_ast]);
          mbar_arrive(&afull_bar[ast]);
        }
        pend_ast = -1;
      } else {
        pend_ast = ast;
      }
      if (i == 0 && t == 0) trace_stamp(a, 5);
#pragma unroll
      for (int q = 0; q < NBG; ++q) cur.advance();
      st += NBG;
      if (st >= S) {
        st -= S;
        ph ^= 1u;
      }
      ast += NBG;
      if (ast >= SA) {
        ast -= SA;
        aph ^= 1u;
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ------------------------------------------------------------ epilogue
    griddep_wait();  // outputs, residual inputs and split workspaces belong to the stream order
    const int e = threadIdx.x - EPI_WARP0 * 32;
    const uint32_t lane_base = static_cast<uint32_t>((warp - EPI_WARP0) * 32) << 16;
    int seg = -1;
    int u = static_cast<int>(ub);
    const int uend = static_cast<int>(ue);
    while (u < uend) {
      const int T = u / KB;
      const int tile_end = (T + 1) * KB;
      const int seg_end = uend < tile_end ? uend : tile_end;
      const int kb0 = u - T * KB;
      const int kb1 = seg_end - T * KB;
      ++seg;
      const int d = seg & 1;
      if (e == 0)
        es.last_flag = mbar_wait(&dfull_bar[d], static_cast<uint32_t>((seg >> 1) & 1), &abort_flag,
                                 a.status, 0x401)
                           ? 1
                           : 0;
      named_bar_sync(1, 128);
      const int got = es.last_flag;
      named_bar_sync(1, 128);
      if (!got) break;
      mbar_try_wait(&dfull_bar[d], static_cast<uint32_t>((seg >> 1) & 1));
      tc_fence_after();
      if (seg == 0 && e == 0) trace_stamp(a, 8);
      const int mt = T / a.n_tiles, nt = T % a.n_tiles;
      const uint32_t dt = tmem_base + lane_base + static_cast<uint32_t>(d) * DCOLS;
      if (kb0 == 0 && kb1 == KB) {
        for (int c0 = 0; c0 < a.n_tile; c0 += 16) {
          uint32_t r[16];
          tmem_ld_x16(dt + static_cast<uint32_t>(c0), r);
          tmem_wait_ld();
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
          epilogue_chunk<EPI>(a, es, mt, nt, c0, e, v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfree_bar[d]);
        if (e == 0) trace_stamp(a, 9);
      } else {
        // split tile: partial [seg][row][n_tile] f32; the last CTA adds them in seg order
        const int first_cta = cta_of_unit(static_cast<long long>(T) * KB, U, G);
        const int last_cta = cta_of_unit(static_cast<long long>(T) * KB + KB - 1, U, G);
        const int nseg = last_cta - first_cta + 1;
        const int segidx = static_cast<int>(blockIdx.x) - first_cta;
        const size_t tile_elems = static_cast<size_t>(a.n_tile) * 128;
        float* wsT = a.ws + static_cast<size_t>(T) * a.max_seg * tile_elems;
        float* mine = wsT + segidx * tile_elems + static_cast<size_t>(e) * a.n_tile;
        for (int c0 = 0; c0 < a.n_tile; c0 += 16) {
          uint32_t r[16];
          tmem_ld_x16(dt + static_cast<uint32_t>(c0), r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            __stcg(reinterpret_cast<float4*>(mine + c0 + j),
                   make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                               __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfree_bar[d]);
        if (e == 0) trace_stamp(a, 9);
        __threadfence();
        named_bar_sync(1, 128);
        if (e == 0) {
          const int old = atomicAdd(a.counters + T, 1);
          es.last_flag = (old == nseg - 1) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (es.last_flag) {
          __threadfence();
          const float* rowp = wsT + static_cast<size_t>(e) * a.n_tile;
          for (int c0 = 0; c0 < a.n_tile; c0 += 16) {
            float4 acc[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            // SEGU segments per round, SEGU * 4 independent 16-byte loads in flight (a short
            // last round loads only its segments); partials are added in segment order
            constexpr int SEGU = INT8 ? 2 : 4;  // the int8 CTA has more threads: fewer registers
            for (int sg = 0; sg < nseg; sg += SEGU) {
              float4 p[SEGU][4];
#pragma unroll
              for (int q = 0; q < SEGU; ++q)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  p[q][j] = sg + q < nseg
                                ? __ldcg(reinterpret_cast<const float4*>(rowp + (sg + q) * tile_elems + c0 + 4 * j))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
              for (int q = 0; q < SEGU; ++q) {
                if (sg + q < nseg) {
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    acc[j].x += p[q][j].x;
                    acc[j].y += p[q][j].y;
                    acc[j].z += p[q][j].z;
                    acc[j].w += p[q][j].w;
                  }
                }
              }
            }
            float v[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[4 * j] = acc[j].x;
              v[4 * j + 1] = acc[j].y;
              v[4 * j + 2] = acc[j].z;
              v[4 * j + 3] = acc[j].w;
            }
            epilogue_chunk<EPI>(a, es, mt, nt, c0, e, v);
          }
          if (e == 0) {
            a.counters[T] = 0;
            trace_stamp(a, 10);
          }
        }
        named_bar_sync(1, 128);
      }
      u = seg_end;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, GEMM_TMEM_COLS);
  if (threadIdx.x == 0) trace_stamp(a, 11);
}

}  // namespace qasr
