// The decode step between two attention launches as ONE persistent cooperative kernel.
//
// One launch runs a short program of operations over the step's decode rows, e.g.
//   o_proj GEMM -> residual + post-attention RMSNorm -> gate|up GEMM -> SiLU ->
//   down GEMM -> residual + next layer's input RMSNorm -> next layer's QKV GEMM ->
//   q/k RMSNorm + RoPE + paged K/V append
// which is what CpuTextDecoder::forward_layer (src/cpu_decoder.rs:367-455) does between
// two attention calls; the per-kernel path of this library launches those as 7 kernels.
// One CTA per SM (cooperative launch: all CTAs are resident), grid-wide barriers
// between dependent operations.
//
// GEMM operations are the tcgen05 weight-streaming GEMM of gemm_tc.cuh in stream-K form,
// but every (tile, CTA) segment stores its f32 partial sum to a workspace and the NEXT
// operation adds the partials in segment order while it builds its own input (residual
// add, SiLU, q/k norm): no CTA finishes another's tile, so no tile fix-up sits on the
// critical path.  The weights of later GEMMs do not depend on anything computed in the
// launch, so the weight producer and the int8 dequantising builders run ahead across
// the barriers into the next GEMM's units as far as their rings allow; only the
// activation (X) loads wait for the barrier before their GEMM.
//
// Roles (512 threads):
//   warp 0      producer: 16 KB bulk copy per weight unit into the W ring, and the TMA of
//               each unit's X tile once its GEMM's input is ready
//   warps 1-3   UMMA issuers (A from TMEM, B = X from shared memory), k-steps split
//               round-robin over them; warp 2 also allocates the TMEM
//   warps 4-7   int8 A builders: f16(q * s) into TMEM
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

enum ChainOpKind : int {
  CH_GEMM = 0,        // partial sums of W x over this CTA's (tile, k-block) range
  CH_EMBED_NORM = 1,  // h[r] = embed[next_tok[slot_r]], row_pos[r] = pos[slot_r]; x = rmsnorm(h)
  CH_RESID = 2,       // h = f16(h + sum of the GEMM's partials); per-tile sums of squares
  CH_NORM = 3,        // x = rmsnorm(h) from those sums
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
  float* ws;            // this GEMM's partial sums: [tile][max_seg][ws_rows][128] f32, zeroed
                        // once; a (tile, segment) slot is either written by every step or
                        // by none, so readers add all max_seg slots without knowing which
};

struct ChainOp {
  int kind;
  int gemm;             // CH_GEMM: index into gemms; row ops: the GEMM whose partials they add
  const float* norm_w;  // *_NORM: RMSNorm gain
  __half* norm_out;     // *_NORM: normalised rows [rows][hs]
  const float* qn_w;    // CH_QKV: q / k RMSNorm gains
  const float* kn_w;
  int layer;            // CH_QKV: KV-cache layer
};

struct ChainArgs {
  ChainOp ops[CHAIN_MAX_OPS];
  ChainGemm gemms[CHAIN_MAX_GEMMS];
  int n_ops;
  int rows, n_tile;
  int w_stages, a_stages;  // weight stages; unit slots (A stage in TMEM + X tile in smem)
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
  float* ss;                 // [rows][CHAIN_MAX_HS / 128] per-tile sums of squares of h
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
__device__ __forceinline__ int ld_acquire_cta_shared(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta_shared(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// Partials of (tile t, row n, column m): segment s at chain_partial(...) + s * ws_rows * 128.
__device__ __forceinline__ const float* chain_partial(const ChainArgs& a, const ChainGemm& g, int t, int n,
                                                      int m) {
  return g.ws + (static_cast<size_t>(t) * g.max_seg * a.ws_rows + n) * 128 + m;
}

// Sum of the `nseg` float4 partial slots at p, p + stride, ... in slot order, all loads in
// flight at once (unused slots hold zeros, which leave the sum unchanged).
template <int MAXSEG>
__device__ __forceinline__ float4 chain_sum_slots4(const float* p, size_t stride, int nseg) {
  float4 v[MAXSEG];
#pragma unroll
  for (int s = 0; s < MAXSEG; ++s)
    v[s] = s < nseg ? __ldcg(reinterpret_cast<const float4*>(p + s * stride)) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int s = 0; s < MAXSEG; ++s) {
    acc.x += v[s].x;
    acc.y += v[s].y;
    acc.z += v[s].z;
    acc.w += v[s].w;
  }
  return acc;
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

__global__ void __launch_bounds__(CHAIN_THREADS, 1)
    decode_chain_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_attn,
                        const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ ChainArgs a) {
  constexpr int KSTEPS = 8;  // 128 k elements per unit, UMMA K = 16
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
      mbar_init(&wfree_bar[i], 4);
    }
    for (int i = 0; i < SU; ++i) {
      mbar_init(&ufull_bar[i], 5);  // 4 builder warps + the X copy's expect_tx arrival
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
      auto w_advance = [&]() {
        while (wu >= wue && wg + 1 < n_gemm_ops) {
          ++wg;
          chain_unit_range(a.gemms[wg], blockIdx.x, wu, wue);
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
      while (wu < wue || xu < xue) {
        bool prog = false;
        if (wu < wue && mbar_test(&wfree_bar[wst], wph ^ 1u)) {
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
            tma_load_2d(dst, tm, &ufull_bar[xst], kb * 128, 0);
            tma_load_2d(dst + x_tile_bytes, tm, &ufull_bar[xst], kb * 128 + 64, 0);
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
  } else if (warp >= 4 && warp < 8) {
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
  } else if (warp >= EPI_WARP0) {
    // ------------------------------------------------------------ epilogue + row operations
    const int e = threadIdx.x - EPI_WARP0 * 32;  // 0 .. CHAIN_EPI_THREADS - 1
    const int we = warp - EPI_WARP0;
    const int row = (warp & 3) * 32 + lane;       // TMEM lane quadrant of this warp = tile row
    const int half = we >> 2;                     // two warps per quadrant split the columns
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const size_t slot_floats = static_cast<size_t>(a.ws_rows) * 128;
    int seg = -1, nbar = 0, gi = 0;
    bool ok = true;
    griddep_wait();
    if (e == 0) {
      st_release_cta_shared(&prev_done, 1);  // opens the first GEMM's X copies
      if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 66] = globaltimer();
    }
    for (int oi = 0; oi < a.n_ops && ok; ++oi) {
      const ChainOp& op = a.ops[oi];
      if (op.kind == CH_GEMM) {
        const ChainGemm& g = a.gemms[gi++];
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
            break;
          }
          mbar_try_wait(&dfull_bar[d], static_cast<uint32_t>((seg >> 1) & 1));
          tc_fence_after();
          const int segidx = static_cast<int>(blockIdx.x) - cta_of_unit(static_cast<long long>(T) * g.kblocks,
                                                                         g.units, g.grid);
          float* dst = g.ws + (static_cast<size_t>(T) * g.max_seg + segidx) * slot_floats + row;
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
            for (int j = 0; j < 16; ++j) __stcg(dst + static_cast<size_t>(c0 + j) * 128, v[j]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dfree_bar[d]);
          u = seg_end;
        }
        if (!ok) break;
      } else if (op.kind == CH_EMBED_NORM) {
        // h[r] = embed row of the slot's input token, x[r] = rmsnorm(h[r]); one row per CTA,
        // thread e holds the column pairs 2e + 256 j
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
      } else if (op.kind == CH_RESID) {
        // h[r, 128 T + c] = f16(h + sum of partials), and the tile's sum of squares of the
        // new f16 values into ss[r][T]; one warp per (row, tile), lane = 4 columns
        const ChainGemm& g = a.gemms[op.gemm];
        const int tiles = a.hs / 128;
        for (int it = blockIdx.x * CHAIN_EPI_WARPS + we; it < a.rows * tiles; it += gridDim.x * CHAIN_EPI_WARPS) {
          const int r = it / tiles, T = it - r * tiles;
          const float4 acc = chain_sum_slots4<CHAIN_MAX_SEG>(chain_partial(a, g, T, r, 4 * lane), slot_floats,
                                                             g.max_seg);
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
          const float2 f01 = __half22float2(n01), f23 = __half22float2(n23);
          float sq = __fmul_rn(f01.x, f01.x);
          sq = __fadd_rn(sq, __fmul_rn(f01.y, f01.y));
          sq = __fadd_rn(sq, __fmul_rn(f23.x, f23.x));
          sq = __fadd_rn(sq, __fmul_rn(f23.y, f23.y));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
          if (lane == 0) __stcg(a.ss + r * CHAIN_MAX_HS / 128 + T, sq);
        }
      } else if (op.kind == CH_NORM) {
        // x[r] = f16(h * inv * w), inv = 1 / sqrt(sum_T ss[r][T] / hs + eps) (rms_norm_row,
        // src/cpu_decoder.rs:261-272); one warp per (row, tile)
        const int tiles = a.hs / 128;
        for (int it = blockIdx.x * CHAIN_EPI_WARPS + we; it < a.rows * tiles; it += gridDim.x * CHAIN_EPI_WARPS) {
          const int r = it / tiles, T = it - r * tiles;
          float t = lane < tiles ? __ldcg(a.ss + r * CHAIN_MAX_HS / 128 + lane) : 0.f;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
          t = __shfl_sync(0xffffffffu, t, 0);  // lane 0's order, the same value everywhere
          const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(a.hs)), a.eps)));
          const int c = T * 128 + 4 * lane;
          const uint2 hw = __ldcg(reinterpret_cast<const uint2*>(a.h + static_cast<size_t>(r) * a.hs + c));
          const float2 h01 = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
          const float2 h23 = __half22float2(*reinterpret_cast<const __half2*>(&hw.y));
          const float4 w = *reinterpret_cast<const float4*>(op.norm_w + c);
          const __half2 x01 = __floats2half2_rn(__fmul_rn(__fmul_rn(h01.x, inv), w.x), __fmul_rn(__fmul_rn(h01.y, inv), w.y));
          const __half2 x23 = __floats2half2_rn(__fmul_rn(__fmul_rn(h23.x, inv), w.z), __fmul_rn(__fmul_rn(h23.y, inv), w.w));
          uint2 xw;
          xw.x = *reinterpret_cast<const uint32_t*>(&x01);
          xw.y = *reinterpret_cast<const uint32_t*>(&x23);
          __stcg(reinterpret_cast<uint2*>(op.norm_out + static_cast<size_t>(r) * a.hs + c), xw);
        }
      } else if (op.kind == CH_SILU) {
        // gate|up tile t: rows [0, 64) gate[64 t + i], rows [64, 128) up[64 t + i].  Work
        // unit: 4 outputs (row r, tile t, quad c); each thread takes every (G * 128)-th one,
        // two at a time so that all their partial loads are in flight together.
        const ChainGemm& g = a.gemms[op.gemm];
        const int tiles = g.units / g.kblocks;
        const int total = a.rows * tiles * 16;
        const int stride = gridDim.x * CHAIN_EPI_THREADS;
        for (int q0 = blockIdx.x * CHAIN_EPI_THREADS + e; q0 < total; q0 += 2 * stride) {
          float4 gs[2], us[2];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int q = q0 + k * stride;
            if (q < total) {
              const int c = q & 15, rt = q >> 4;
              const int r = rt / tiles, t = rt - r * tiles;
              const float* p = chain_partial(a, g, t, r, 4 * c);
              gs[k] = chain_sum_slots4<CHAIN_SILU_SEG>(p, slot_floats, g.max_seg);
              us[k] = chain_sum_slots4<CHAIN_SILU_SEG>(p + 64, slot_floats, g.max_seg);
            }
          }
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int q = q0 + k * stride;
            if (q >= total) continue;
            const int c = q & 15, rt = q >> 4;
            const int r = rt / tiles, t = rt - r * tiles;
            const float gv[4] = {gs[k].x, gs[k].y, gs[k].z, gs[k].w}, uv[4] = {us[k].x, us[k].y, us[k].z, us[k].w};
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
        }
      } else if (op.kind == CH_QKV) {
        // one warp per (row, head), lane = dims 4 lane .. +3; the rotate-half partner of
        // dim d (d ^ 64) sits in lane ^ 16
        const ChainGemm& g = a.gemms[op.gemm];
        const int heads = a.nq + 2 * a.nkv;
        for (int it = blockIdx.x * CHAIN_EPI_WARPS + we; it < a.rows * heads; it += gridDim.x * CHAIN_EPI_WARPS) {
          const int r = it / heads, t = it - r * heads;
          const int d0 = 4 * lane;
          const int pos = __ldcg(a.row_pos + r);
          const int page = __ldcg(a.row_page + r);
          const uint2 cw = __ldcg(reinterpret_cast<const uint2*>(a.row_rope + static_cast<size_t>(r) * 256 + d0));
          const uint2 sw = __ldcg(reinterpret_cast<const uint2*>(a.row_rope + static_cast<size_t>(r) * 256 + 128 + d0));
          const float4 acc = chain_sum_slots4<CHAIN_QKV_SEG>(chain_partial(a, g, t, r, 4 * lane), slot_floats,
                                                             g.max_seg);
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
      }
      // ---- grid barrier between dependent operations
      if (oi + 1 < a.n_ops) {
        named_bar_sync(1, CHAIN_EPI_THREADS);
        if (e == 0) {
          if (a.trace != nullptr && oi < 12) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * oi] = globaltimer();
          ++nbar;
          // release this CTA's writes (the group's, ordered by the named barrier), arrive,
          // poll with relaxed loads, then one acquire fence
          asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.barrier) : "memory");
          const unsigned int target = static_cast<unsigned int>(nbar) * gridDim.x;
          if (ld_relaxed_gpu(a.barrier) < target) {
            const uint64_t t0 = globaltimer();
            while (ld_relaxed_gpu(a.barrier) < target) {
              if (abort_flag || globaltimer() - t0 > QASR_WAIT_NS) {
                if (!abort_flag) report_error(a.status, DEVERR_TIMEOUT, 0x761);
                abort_flag = 1;
                break;
              }
            }
          }
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          bar_ok = abort_flag ? 0 : 1;
          if (a.trace != nullptr && oi < 12) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 2 + 2 * oi] = globaltimer();
          if (a.ops[oi + 1].kind == CH_GEMM) st_release_cta_shared(&xready, gi + 1);
        }
        named_bar_sync(1, CHAIN_EPI_THREADS);
        if (!bar_ok) ok = false;
      } else if (e == 0 && a.trace != nullptr && oi < 12) {
        a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + 1 + 2 * oi] = globaltimer();
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
