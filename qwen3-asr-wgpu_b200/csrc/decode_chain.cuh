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
//   warp 0      weight producer: 16 KB bulk copy per unit into the W ring
//   warp 1      UMMA issuer (A from TMEM, B = X from shared memory)
//   warp 2      TMEM allocator
//   warp 3      activation producer: TMA of the unit's X tile once its GEMM's input is ready
//   warps 4-11  int8 A builders (two warpgroups, alternate units): f16(q * s) into TMEM
//   warps 12-15 epilogue and row operations; they also run the grid barriers
#pragma once
#include "device_common.cuh"
#include "gemm_tc.cuh"

namespace qasr {

constexpr int CHAIN_MAX_OPS = 8;
constexpr int CHAIN_MAX_GEMMS = 4;
constexpr int CHAIN_THREADS = 512;
constexpr int CHAIN_MAX_W_STAGES = 12;
constexpr int CHAIN_X_STAGES = 4;
constexpr int CHAIN_MAX_A_STAGES = 8;
constexpr int CHAIN_MAX_ROWS = 128;  // one N tile
constexpr int CHAIN_TRACE_SLOTS = 16;
constexpr int CHAIN_MAX_HS = 2048;   // hidden size the row operations hold in registers

enum ChainOpKind : int {
  CH_GEMM = 0,        // partial sums of W x over this CTA's (tile, k-block) range
  CH_EMBED_NORM = 1,  // h[r] = embed[next_tok[slot_r]], row_pos[r] = pos[slot_r]; x = rmsnorm(h)
  CH_RESID_NORM = 2,  // h = f16(h + sum of the GEMM's partials); x = rmsnorm(h)
  CH_SILU = 3,        // act = f16(silu(f16 gate) * f16 up) from the gate|up GEMM's partials
  CH_QKV = 4,         // q/k RMSNorm + RoPE -> q and paged K; raw V -> paged V
};

struct ChainGemm {
  const uint8_t* w;     // int8 weights in the tiled layout (weight_tile_offset)
  const __half* scale;  // f16 per-row scales
  int kblocks;          // K / 128
  int units;            // (n_out / 128) * kblocks
  int grid;             // CTAs that take part: the first `grid` of the launch
  int max_seg;          // most segments (CTAs) any tile is cut into
  int xmap;             // X source: 0 = normalised rows, 1 = attention output, 2 = act
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
  int w_stages, a_stages;
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
  KvLayout kv;
  float* ws;                 // partials: [(tile * max_seg + seg)][n_tile][128] f32
  unsigned int* barrier;     // grid barrier counter, zero at launch
  uint32_t* status;
  unsigned long long* trace;  // optional: per CTA CHAIN_TRACE_SLOTS %globaltimer stamps
};

__device__ __forceinline__ void chain_unit_range(const ChainGemm& g, int cta, int& ub, int& ue) {
  if (cta >= g.grid) {
    ub = ue = 0;
    return;
  }
  ub = static_cast<int>(static_cast<long long>(cta) * g.units / g.grid);
  ue = static_cast<int>(static_cast<long long>(cta + 1) * g.units / g.grid);
}

// CTA owning unit x (the largest c with c * units / grid <= x), 32-bit: units * grid < 2^31
__device__ __forceinline__ int chain_cta_of_unit(int x, const ChainGemm& g) {
  return static_cast<int>((static_cast<unsigned>(x + 1) * g.grid + g.units - 1) / static_cast<unsigned>(g.units)) - 1;
}
// segments of tile t (the CTAs its k-blocks are spread over)
__device__ __forceinline__ int chain_tile_segments(const ChainGemm& g, int t) {
  const int a = t * g.kblocks;
  return chain_cta_of_unit(a + g.kblocks - 1, g) - chain_cta_of_unit(a, g) + 1;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
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

// Partials of (tile t, row n, column m): segment s at chain_partial(...) + s * tile_floats.
// Callers add them in segment order with the segment loop outermost, so each round's
// loads (over all of the thread's outputs) are in flight together.
__device__ __forceinline__ const float* chain_partial(const ChainArgs& a, const ChainGemm& g, int t, int n,
                                                      int m) {
  const size_t tile_floats = static_cast<size_t>(a.n_tile) * 128;
  return a.ws + static_cast<size_t>(t) * g.max_seg * tile_floats + static_cast<size_t>(n) * 128 + m;
}

// Block-of-128 sum (the four epilogue warps), the same value in every thread.
__device__ __forceinline__ float chain_sum128(float v, float* red, int e) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  named_bar_sync(1, 128);
  if ((e & 31) == 0) red[e >> 5] = v;
  named_bar_sync(1, 128);
  return (red[0] + red[1]) + (red[2] + red[3]);
}

__global__ void __launch_bounds__(CHAIN_THREADS, 1)
    decode_chain_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_attn,
                        const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ ChainArgs a) {
  constexpr int KSTEPS = 8;  // 128 k elements per unit, UMMA K = 16
  constexpr int EPI_WARP0 = 12;
  extern __shared__ __align__(1024) uint8_t chain_dsmem[];
  __shared__ __align__(8) uint64_t wfull_bar[CHAIN_MAX_W_STAGES], wfree_bar[CHAIN_MAX_W_STAGES];
  __shared__ __align__(8) uint64_t xfull_bar[CHAIN_X_STAGES], xfree_bar[CHAIN_X_STAGES];
  __shared__ __align__(8) uint64_t afull_bar[CHAIN_MAX_A_STAGES], afree_bar[CHAIN_MAX_A_STAGES];
  __shared__ __align__(8) uint64_t dfull_bar[2], dfree_bar[2], done_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ int xready;  // GEMMs whose X input is complete (written by the epilogue leader)
  __shared__ int seg_ok, bar_ok;
  __shared__ float red[4];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(chain_dsmem) + 1023) & ~uintptr_t(1023));
  const int SW = a.w_stages, SA = a.a_stages;
  const uint32_t x_tile_bytes = static_cast<uint32_t>(a.n_tile) * 128u;
  const uint32_t x_stage_bytes = 2u * x_tile_bytes;
  uint8_t* xring = smem + static_cast<size_t>(SW) * 16384;
  const uint32_t DCOLS = (static_cast<uint32_t>(a.n_tile) + 31u) & ~31u;
  const uint32_t A_COLS0 = 2u * DCOLS;
  int n_gemm_ops = 0;
  for (int i = 0; i < a.n_ops; ++i) n_gemm_ops += a.ops[i].kind == CH_GEMM ? 1 : 0;

  if (threadIdx.x == 0) {
    if (a.trace != nullptr) a.trace[blockIdx.x * CHAIN_TRACE_SLOTS] = globaltimer();
    for (int i = 0; i < SW; ++i) {
      mbar_init(&wfull_bar[i], 1);
      mbar_init(&wfree_bar[i], 4);
    }
    for (int i = 0; i < CHAIN_X_STAGES; ++i) {
      mbar_init(&xfull_bar[i], 1);
      mbar_init(&xfree_bar[i], 1);
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
    xready = (a.n_ops > 0 && a.ops[0].kind == CH_GEMM) ? 1 : 0;
    fence_mbar_init();
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
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      int st = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int gi = 0; gi < CHAIN_MAX_GEMMS && gi < n_gemm_ops && ok; ++gi) {
        const ChainGemm& g = a.gemms[gi];
        int ub, ue;
        chain_unit_range(g, blockIdx.x, ub, ue);
        for (int u = ub; u < ue; ++u) {
          if (!mbar_wait(&wfree_bar[st], ph ^ 1u, &abort_flag, a.status, 0x701)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&wfull_bar[st], 16384u);
          bulk_load(smem + static_cast<size_t>(st) * 16384, g.w + static_cast<size_t>(u) * 16384, 16384u,
                    &wfull_bar[st]);
          ++issued;
          if (++st == SW) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      for (int j = 0; j < SW && j < issued; ++j) {  // every issued copy lands before exit
        const int il = issued - 1 - ((issued - 1 - j) % SW);
        mbar_wait(&wfull_bar[j], static_cast<uint32_t>((il / SW) & 1), nullptr, a.status, 0x702);
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ activation producer
    if (lane == 0) {
      int st = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int gi = 0; gi < n_gemm_ops && ok; ++gi) {
        const ChainGemm& g = a.gemms[gi];
        // wait until the operation before this GEMM completed on every CTA
        const uint64_t t0 = globaltimer();
        while (ld_acquire_cta_shared(&xready) <= gi) {
          if (abort_flag || globaltimer() - t0 > QASR_WAIT_NS) {
            if (!abort_flag) report_error(a.status, DEVERR_TIMEOUT, 0x711);
            abort_flag = 1;
            ok = false;
            break;
          }
        }
        if (!ok) break;
        fence_proxy_async_global();  // X was written by other CTAs with ordinary stores
        const CUtensorMap* tm = g.xmap == 0 ? &tm_x : (g.xmap == 1 ? &tm_attn : &tm_act);
        int ub, ue;
        chain_unit_range(g, blockIdx.x, ub, ue);
        for (int u = ub; u < ue; ++u) {
          if (!mbar_wait(&xfree_bar[st], ph ^ 1u, &abort_flag, a.status, 0x712)) {
            ok = false;
            break;
          }
          const int kb = u % g.kblocks;
          uint8_t* dst = xring + static_cast<size_t>(st) * x_stage_bytes;
          mbar_arrive_expect_tx(&xfull_bar[st], x_stage_bytes);
          tma_load_2d(dst, tm, &xfull_bar[st], kb * 128, 0);
          tma_load_2d(dst + x_tile_bytes, tm, &xfull_bar[st], kb * 128 + 64, 0);
          ++issued;
          if (++st == CHAIN_X_STAGES) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      for (int j = 0; j < CHAIN_X_STAGES && j < issued; ++j) {
        const int il = issued - 1 - ((issued - 1 - j) % CHAIN_X_STAGES);
        mbar_wait(&xfull_bar[j], static_cast<uint32_t>((il / CHAIN_X_STAGES) & 1), nullptr, a.status, 0x713);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16_m128(static_cast<uint32_t>(a.n_tile));
      int xs = 0, ast = 0, seg = -1, d = 0;
      uint32_t xph = 0, aph = 0;
      bool ok = true, issued_any = false;
      for (int gi = 0; gi < n_gemm_ops && ok; ++gi) {
        const ChainGemm& g = a.gemms[gi];
        int ub, ue;
        chain_unit_range(g, blockIdx.x, ub, ue);
        for (int u = ub; u < ue; ++u) {
          const int kb = u % g.kblocks;
          const bool first = (u == ub) || (kb == 0);
          const bool last = (u == ue - 1) || (kb == g.kblocks - 1);
          if (first) {
            ++seg;
            d = seg & 1;
            if (!mbar_wait(&dfree_bar[d], static_cast<uint32_t>(((seg >> 1) & 1) ^ 1), &abort_flag, a.status,
                           0x721)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (!mbar_wait(&afull_bar[ast], aph, &abort_flag, a.status, 0x722) ||
              !mbar_wait(&xfull_bar[xs], xph, &abort_flag, a.status, 0x723)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(d) * DCOLS;
          const uint32_t a_tmem = tmem_base + A_COLS0 + static_cast<uint32_t>(ast) * 64u;
          const uint32_t x_base = smem_u32(xring + static_cast<size_t>(xs) * x_stage_bytes);
#pragma unroll
          for (int kk = 0; kk < KSTEPS; ++kk) {
            const uint32_t b_addr = x_base + static_cast<uint32_t>(kk >> 2) * x_tile_bytes +
                                    static_cast<uint32_t>(kk & 3) * 32u;
            umma_f16_ts(d_tmem, a_tmem + static_cast<uint32_t>(kk) * 8u, smem_desc_sw128(b_addr), idesc,
                        (first && kk == 0) ? 0u : 1u);
          }
          umma_commit(&xfree_bar[xs]);
          umma_commit(&afree_bar[ast]);
          if (last) umma_commit(&dfull_bar[d]);
          issued_any = true;
          if (++xs == CHAIN_X_STAGES) {
            xs = 0;
            xph ^= 1u;
          }
          if (++ast == SA) {
            ast = 0;
            aph ^= 1u;
          }
        }
      }
      if (issued_any) {  // all MMAs retire before the TMEM is released
        umma_commit(&done_bar);
        mbar_wait(&done_bar, 0, nullptr, a.status, 0x724);
      }
    }
  } else if (warp >= 4 && warp < EPI_WARP0) {
    // ------------------------------------------------------------ int8 A builders
    const int grp = (warp - 4) >> 2;
    const int t = (threadIdx.x - 128) & 127;  // row of the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int st = 0, ast = 0, i = 0, pend_ast = -1;
    uint32_t ph = 0, aph = 0;
    bool ok = true;
    for (int gi = 0; gi < n_gemm_ops && ok; ++gi) {
      const ChainGemm& g = a.gemms[gi];
      int ub, ue;
      chain_unit_range(g, blockIdx.x, ub, ue);
      int cur_mt = -1;
      __half2 sc2 = __floats2half2_rn(1.0f, 1.0f);
      for (int u = ub; u < ue; ++u, ++i) {
        const int my_st = st, my_ast = ast;
        const uint32_t my_ph = ph, my_aph = aph;
        if (++st == SW) {
          st = 0;
          ph ^= 1u;
        }
        if (++ast == SA) {
          ast = 0;
          aph ^= 1u;
        }
        if ((i & 1) != grp) continue;
        if (!mbar_wait_warp(&wfull_bar[my_st], my_ph, &abort_flag, a.status, 0x731) ||
            !mbar_wait_warp(&afree_bar[my_ast], my_aph ^ 1u, &abort_flag, a.status, 0x732)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int mt = u / g.kblocks;
        if (mt != cur_mt) {
          const __half sc = g.scale[mt * 128 + t];
          sc2 = __halves2half2(sc, sc);
          cur_mt = mt;
        }
        const uint8_t* row = smem + static_cast<size_t>(my_st) * 16384 + t * 128;
        uint4 chunk[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) chunk[c] = *reinterpret_cast<const uint4*>(row + ((c ^ (t & 7)) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfree_bar[my_st]);  // the W stage is read: refill it
        const uint32_t taddr = tmem_base + lane_base + A_COLS0 + static_cast<uint32_t>(my_ast) * 64u;
        const __half2 bias = __floats2half2_rn(1152.0f, 1152.0f);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t w4[4] = {chunk[c].x, chunk[c].y, chunk[c].z, chunk[c].w};
          uint32_t outw[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t ub8 = w4[q] ^ 0x80808080u;  // q + 128 as unsigned bytes
            uint32_t lo = __byte_perm(ub8, 0x64646464u, 0x4140);
            uint32_t hi = __byte_perm(ub8, 0x64646464u, 0x4342);
            __half2 hl = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);  // exact q
            __half2 hh = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
            hl = __hmul2_rn(hl, sc2);  // f16(q * s), one IEEE rounding
            hh = __hmul2_rn(hh, sc2);
            outw[2 * q] = *reinterpret_cast<uint32_t*>(&hl);
            outw[2 * q + 1] = *reinterpret_cast<uint32_t*>(&hh);
          }
          tmem_st_x8(taddr + static_cast<uint32_t>(c) * 8u, reinterpret_cast<const uint32_t(&)[8]>(outw));
        }
        // publish two of this group's units per TMEM store wait, except at the end of a GEMM
        const bool group_last_in_gemm = (u + 2 >= ue);
        if (pend_ast >= 0 || group_last_in_gemm) {
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (pend_ast >= 0) mbar_arrive(&afull_bar[pend_ast]);
            mbar_arrive(&afull_bar[my_ast]);
          }
          pend_ast = -1;
        } else {
          pend_ast = my_ast;
        }
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ------------------------------------------------------------ epilogue + row operations
    const int e = threadIdx.x - EPI_WARP0 * 32;
    const int we = warp - EPI_WARP0;
    const uint32_t lane_base = static_cast<uint32_t>(we * 32) << 16;
    const size_t tile_floats = static_cast<size_t>(a.n_tile) * 128;
    int seg = -1, nbar = 0, gi = 0;
    bool ok = true;
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
          named_bar_sync(1, 128);
          const int got = seg_ok;
          named_bar_sync(1, 128);
          if (!got) {
            ok = false;
            break;
          }
          mbar_try_wait(&dfull_bar[d], static_cast<uint32_t>((seg >> 1) & 1));
          tc_fence_after();
          const int segidx = static_cast<int>(blockIdx.x) - cta_of_unit(static_cast<long long>(T) * g.kblocks,
                                                                         g.units, g.grid);
          float* dst = a.ws + (static_cast<size_t>(T) * g.max_seg + segidx) * tile_floats + e;
          const uint32_t dt = tmem_base + lane_base + static_cast<uint32_t>(d) * DCOLS;
          for (int c0 = 0; c0 < a.n_tile; c0 += 16) {
            uint32_t r[16];
            tmem_ld_x16(dt + static_cast<uint32_t>(c0), r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) __stcg(dst + static_cast<size_t>(c0 + j) * 128, __uint_as_float(r[j]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dfree_bar[d]);
          u = seg_end;
        }
        if (!ok) break;
      } else if (op.kind == CH_EMBED_NORM || op.kind == CH_RESID_NORM) {
        // one row per CTA; thread e holds the column pairs 2e + 256 j (j < hs / 256)
        const ChainGemm& g = a.gemms[op.gemm];
        const int np = a.hs / 256;
        for (int r = blockIdx.x; r < a.rows; r += gridDim.x) {
          __half* hr = a.h + static_cast<size_t>(r) * a.hs;
          float2 v[CHAIN_MAX_HS / 256];
          if (op.kind == CH_EMBED_NORM) {
            const int slot = a.row_slot[r];
            int tok = a.next_tok[slot];
            if (tok < 0 || tok >= a.vocab) {
              if (e == 0) report_error(a.status, DEVERR_BOUNDS, 0x751);
              tok = 0;
            }
            const __half* src = a.embed + static_cast<size_t>(tok) * a.hs;
            if (e == 0) a.row_pos[r] = a.pos[slot];
#pragma unroll
            for (int j = 0; j < CHAIN_MAX_HS / 256; ++j)
              if (j < np) v[j] = __half22float2(*reinterpret_cast<const __half2*>(src + 2 * e + 256 * j));
          } else {
            float2 acc[CHAIN_MAX_HS / 256];
            int nseg[CHAIN_MAX_HS / 256];
            int smax = 0;
#pragma unroll
            for (int j = 0; j < CHAIN_MAX_HS / 256; ++j) {
              acc[j] = make_float2(0.f, 0.f);
              nseg[j] = j < np ? chain_tile_segments(g, (2 * e + 256 * j) >> 7) : 0;
              smax = max(smax, nseg[j]);
              if (j < np) v[j] = __half22float2(__ldcg(reinterpret_cast<const __half2*>(hr + 2 * e + 256 * j)));
            }
            const size_t tile_floats = static_cast<size_t>(a.n_tile) * 128;
            for (int sg = 0; sg < smax; ++sg) {
#pragma unroll
              for (int j = 0; j < CHAIN_MAX_HS / 256; ++j) {
                if (sg < nseg[j]) {
                  const int i = 2 * e + 256 * j;
                  const float2 p = __ldcg(reinterpret_cast<const float2*>(
                      chain_partial(a, g, i >> 7, r, i & 127) + sg * tile_floats));
                  acc[j].x += p.x;
                  acc[j].y += p.y;
                }
              }
            }
#pragma unroll
            for (int j = 0; j < CHAIN_MAX_HS / 256; ++j) {
              v[j].x = f16_round(__fadd_rn(v[j].x, acc[j].x));  // batch_dot_acc: f16(h + acc)
              v[j].y = f16_round(__fadd_rn(v[j].y, acc[j].y));
            }
          }
          float sq = 0.f;
#pragma unroll
          for (int j = 0; j < CHAIN_MAX_HS / 256; ++j) {
            if (j < np) {
              __stcg(reinterpret_cast<__half2*>(hr + 2 * e + 256 * j), __floats2half2_rn(v[j].x, v[j].y));
              sq = __fadd_rn(sq, __fmul_rn(v[j].x, v[j].x));
              sq = __fadd_rn(sq, __fmul_rn(v[j].y, v[j].y));
            }
          }
          const float tot = chain_sum128(sq, red, e);
          const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(a.hs)), a.eps)));
          __half* y = op.norm_out + static_cast<size_t>(r) * a.hs;
#pragma unroll
          for (int j = 0; j < CHAIN_MAX_HS / 256; ++j) {
            if (j < np) {
              const int i = 2 * e + 256 * j;
              const float x0 = __fmul_rn(__fmul_rn(v[j].x, inv), op.norm_w[i]);
              const float x1 = __fmul_rn(__fmul_rn(v[j].y, inv), op.norm_w[i + 1]);
              __stcg(reinterpret_cast<__half2*>(y + i), __floats2half2_rn(x0, x1));
            }
          }
          named_bar_sync(1, 128);  // `red` is reused by the next row
        }
      } else if (op.kind == CH_SILU) {
        // gate|up tile t: rows [0, 64) gate[64 t + i], rows [64, 128) up[64 t + i]; thread e
        // takes column i = e % 64 of rows e / 64, + 2, + 4, ... in batches of 8 rows
        const ChainGemm& g = a.gemms[op.gemm];
        const int tiles = g.units / g.kblocks;
        const int i = e & 63;
        const size_t tile_floats = static_cast<size_t>(a.n_tile) * 128;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
          const int nseg = chain_tile_segments(g, t);
          for (int r0 = e >> 6; r0 < a.rows; r0 += 16) {
            float ga[8], ua[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) ga[k] = ua[k] = 0.f;
            for (int sg = 0; sg < nseg; ++sg) {
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const int r = r0 + 2 * k;
                if (r < a.rows) {
                  const float* p = chain_partial(a, g, t, r, i) + sg * tile_floats;
                  ga[k] += __ldcg(p);
                  ua[k] += __ldcg(p + 64);
                }
              }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int r = r0 + 2 * k;
              if (r < a.rows) {
                const float gt = f16_round(ga[k]);
                const float up = f16_round(ua[k]);
                const float silu = __fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt)));
                __stcg(a.act + static_cast<size_t>(r) * a.inter + t * 64 + i, __float2half_rn(__fmul_rn(silu, up)));
              }
            }
          }
        }
      } else if (op.kind == CH_QKV) {
        // one warp per (row, head); lane l holds dims l + 32 j, so the rotate-half
        // partner of dim d (d ^ 64) is the same lane's j ^ 2
        const ChainGemm& g = a.gemms[op.gemm];
        const int heads = a.nq + 2 * a.nkv;
        for (int item = blockIdx.x * 4 + we; item < a.rows * heads; item += gridDim.x * 4) {
          const int r = item / heads, t = item - r * heads;
          const int nseg = chain_tile_segments(g, t);
          const size_t tile_floats = static_cast<size_t>(a.n_tile) * 128;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          const float* p = chain_partial(a, g, t, r, lane);
          for (int sg = 0; sg < nseg; ++sg) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] += __ldcg(p + sg * tile_floats + 32 * j);
          }
          const int slot = a.row_slot[r];
          const int pos = __ldcg(a.row_pos + r);
          if (t >= a.nq + a.nkv) {
            const size_t off = kv_elem_offset(a.kv, slot, pos, op.layer, 1, t - a.nq - a.nkv);
#pragma unroll
            for (int j = 0; j < 4; ++j) a.kv.pool[off + kv_dim_swizzle(pos, lane + 32 * j)] = __float2half_rn(v[j]);
            continue;
          }
          float x[4], ss = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            x[j] = f16_round(v[j]);
            ss = __fadd_rn(ss, __fmul_rn(x[j], x[j]));
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps)));
          const float* w = t < a.nq ? op.qn_w : op.kn_w;
          float xn[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) xn[j] = __fmul_rn(__fmul_rn(x[j], inv), w[lane + 32 * j]);
          size_t koff = 0;
          if (t >= a.nq) koff = kv_elem_offset(a.kv, slot, pos, op.layer, 0, t - a.nq);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int dd = lane + 32 * j;
            const float c = __half2float(a.rope_cos[static_cast<size_t>(pos) * 128 + dd]);
            const float sn = __half2float(a.rope_sin[static_cast<size_t>(pos) * 128 + dd]);
            const float sign = j < 2 ? -1.0f : 1.0f;
            const float o = __fadd_rn(__fmul_rn(xn[j], c), __fmul_rn(__fmul_rn(sign, xn[j ^ 2]), sn));
            if (t < a.nq)
              a.q[static_cast<size_t>(r) * a.nq * 128 + t * 128 + dd] = __float2half_rn(o);
            else
              a.kv.pool[koff + kv_dim_swizzle(pos, dd)] = __float2half_rn(o);
          }
        }
      }
      // ---- grid barrier between dependent operations
      if (oi + 1 < a.n_ops) {
        named_bar_sync(1, 128);
        if (e == 0) {
          ++nbar;
          __threadfence();
          fence_proxy_async_global();
          atomicAdd(a.barrier, 1u);
          const unsigned int target = static_cast<unsigned int>(nbar) * gridDim.x;
          const uint64_t t0 = globaltimer();
          while (ld_acquire_gpu(a.barrier) < target) {
            if (abort_flag || globaltimer() - t0 > QASR_WAIT_NS) {
              if (!abort_flag) report_error(a.status, DEVERR_TIMEOUT, 0x761);
              abort_flag = 1;
              break;
            }
          }
          __threadfence();
          bar_ok = abort_flag ? 0 : 1;
          if (a.trace != nullptr && oi + 1 < CHAIN_TRACE_SLOTS)
            a.trace[blockIdx.x * CHAIN_TRACE_SLOTS + oi + 1] = globaltimer();
          if (a.ops[oi + 1].kind == CH_GEMM) st_release_cta_shared(&xready, gi + 1);
        }
        named_bar_sync(1, 128);
        if (!bar_ok) ok = false;
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
