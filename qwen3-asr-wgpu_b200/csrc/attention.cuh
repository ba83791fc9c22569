// GQA attention of query rows over their slot's paged KV (decode and prefill).
//
// Replaces gqa_decode_single(_slots), gqa_decode_split_p1(_pair) and gqa_split_merge
// (src/shaders.rs:1881-2182, 2270-2905); the math follows CpuTextDecoder::attention
// (src/cpu_decoder.rs:292-365): s_t = (q . k_t) * 1/sqrt(hd), softmax over t <= pos,
// o = f16(sum_t p_t v_t / sum_t p_t).
//
// Each query row r (slot s_r, position p_r) attends to positions [0, p_r] of its slot,
// so one kernel serves a decode step (one row per slot) and a prefill chunk
// (consecutive positions of a slot; causal by construction).
//
// Layout: a KV page holds 64 positions; the K (or V) rows of one (page, layer, kv head)
// are one contiguous 16 KB block.  Work unit = (row, kv head, chunk of stages); a
// stage is two pages (128 positions).  Both q heads of the kv head are done together
// so K/V are read once (the reference's "pair" kernel idea).  A row is cut into at
// most ATTN_ROW_CHUNKS chunks as a function of its own length, so a slot's result does
// not depend on the other rows of the launch.
//
// Persistent CTA per SM: warp 8 streams the pages of the CTA's units (and each unit's q
// rows, with its first stage), stage after stage, into a 3-deep shared-memory ring with
// cp.async.bulk (completion counted on mbarriers, no multicast); warps 0-7 each take 16
// positions of a stage and compute S^T = K Q^T and O^T += V^T P^T on the tensor cores
// (mma.sync: with two real query rows per kv head the work is too thin for tcgen05) with
// an online softmax per head and warp.  At a unit's end the consumer warps drop their
// state into a double-buffered shared slot and move on; warp 9 merges the 8 warps and
// stores the output or, for a row cut into several chunks, the chunk's partial, which
// attention_merge_kernel combines in chunk order.
//
// Programmatic dependent launch: with `early` > 0 (the decode step, where the launch
// before this one appended exactly `early` new positions per row and wrote q), the page
// producer streams stages made only of older positions before griddepcontrol.wait, so
// the first KV bytes are in flight while the previous kernel drains; q and the stages
// holding new positions are fetched after the wait.
#pragma once
#include "device_common.cuh"
#include "gemm_tc.cuh"  // KvLayout, kv_elem_offset, griddep_*

namespace qasr {

constexpr int ATTN_CONSUMER_WARPS = 8;
constexpr int ATTN_THREADS = (ATTN_CONSUMER_WARPS + 2) * 32;  // + page producer + merger
constexpr int ATTN_STAGES = 3;
constexpr int ATTN_PAGE_BYTES = 64 * 128 * 2;            // K or V rows of one page / head
constexpr int ATTN_STAGE_BYTES = 4 * ATTN_PAGE_BYTES;    // 2 pages x (K + V)
constexpr int ATTN_PART_FLOATS = 4 + 2 * 128;            // m0, m1, l0, l1, o0[128], o1[128]
constexpr int ATTN_ROW_CHUNKS = 4;                       // chunks per row (upper bound)
constexpr int ATTN_MAX_ROWS = 2048;

__host__ __device__ __forceinline__ int attn_row_stages(int len) { return (len + 127) / 128; }
__host__ __device__ __forceinline__ int attn_chunk_stages(int len) {
  const int st = attn_row_stages(len);
  return (st + ATTN_ROW_CHUNKS - 1) / ATTN_ROW_CHUNKS;
}
__host__ __device__ __forceinline__ int attn_row_chunks(int len) {
  const int cs = attn_chunk_stages(len);
  return (attn_row_stages(len) + cs - 1) / cs;
}
// dynamic shared memory of one CTA for `rows` query rows
__host__ __device__ __forceinline__ size_t attn_smem_bytes(int rows) {
  return 1024 + static_cast<size_t>(ATTN_STAGES) * ATTN_STAGE_BYTES +
         static_cast<size_t>(rows + 1) * sizeof(int);
}

struct AttnArgs {
  const __half* q;  // [rows][q_ld], heads 2g and 2g+1 use kv head g
  int q_ld;
  __half* out;      // [rows][q_ld]
  const int* row_slot;
  const int* row_pos;
  KvLayout kv;
  int layer;
  int rows;
  float scale;
  float* ws;        // [rows * nkv * ATTN_ROW_CHUNKS][ATTN_PART_FLOATS]: chunk partials
  int early;        // > 0: positions >= len - early are new (see above); 0: wait first
  uint32_t* status;
  unsigned long long* trace;  // optional: per CTA ATTN_TRACE_SLOTS %globaltimer stamps
};

constexpr int ATTN_TRACE_SLOTS = 8;
// slots: 0 entry, 1 unit table ready, 2 first stage landed (consumer warp 0), 3 first
// unit handed to the merger, 4 last stage consumed, 5 last unit merged, 6 producer done,
// 7 units processed by this CTA
__device__ __forceinline__ void attn_stamp(const AttnArgs& a, int slot) {
  if (a.trace != nullptr) a.trace[blockIdx.x * ATTN_TRACE_SLOTS + slot] = globaltimer();
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D += A B, m16n8k16, f16 operands, f32 accumulators
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct AttnUnit {
  int r, g, c, nch, len, s0, s1;  // row, kv head, chunk, chunks of the row, row length, stages [s0, s1)
};

__device__ __forceinline__ AttnUnit attn_unit(const AttnArgs& a, const int* prefix, int u) {
  int lo = 0, hi = a.rows - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= u) lo = mid; else hi = mid - 1;
  }
  AttnUnit t;
  t.r = lo;
  t.len = a.row_pos[lo] + 1;
  t.nch = attn_row_chunks(t.len);
  const int rem = u - prefix[lo];
  t.g = rem / t.nch;
  t.c = rem % t.nch;
  const int cs = attn_chunk_stages(t.len);
  t.s0 = t.c * cs;
  const int st = attn_row_stages(t.len);
  t.s1 = min(t.s0 + cs, st);
  return t;
}

__global__ void __launch_bounds__(ATTN_THREADS, 1)
    attention_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t attn_dsmem[];
  __shared__ __align__(8) uint64_t full_bar[ATTN_STAGES], empty_bar[ATTN_STAGES];
  __shared__ __align__(8) uint64_t mfull_bar[2], mfree_bar[2];
  __shared__ __align__(16) __half sm_q[ATTN_STAGES][256];             // q of heads 2g, 2g+1
  __shared__ float sm_m[2][ATTN_CONSUMER_WARPS][2], sm_l[2][ATTN_CONSUMER_WARPS][2];
  __shared__ __align__(16) float sm_acc[2][ATTN_CONSUMER_WARPS][2][128];
  __shared__ int sh_units, sh_scan[ATTN_THREADS / 32];
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_dsmem) + 1023) & ~uintptr_t(1023));
  int* prefix = reinterpret_cast<int*>(smem + ATTN_STAGES * ATTN_STAGE_BYTES);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkv = a.kv.nkv;

  if (tid == 0) {
    attn_stamp(a, 0);
    for (int i = 0; i < ATTN_STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], ATTN_CONSUMER_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&mfull_bar[i], ATTN_CONSUMER_WARPS);
      mbar_init(&mfree_bar[i], 1);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  // row_slot / row_pos / page tables and the older KV positions predate the previous
  // launch; q, the new positions and the outputs' readers belong to it.
  if (a.early <= 0) griddep_wait();
  griddep_launch_dependents();

  // ---- unit table: prefix[r] = first unit of row r (block-wide scan)
  {
    const int per = (a.rows + ATTN_THREADS - 1) / ATTN_THREADS;
    const int r0 = tid * per, r1 = min(r0 + per, a.rows);
    int local = 0;
    for (int r = r0; r < r1; ++r) local += attn_row_chunks(a.row_pos[r] + 1) * nkv;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) sh_scan[warp] = incl;
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int w = 0; w < ATTN_THREADS / 32; ++w) {
        const int v = sh_scan[w];
        sh_scan[w] = acc;
        acc += v;
      }
      sh_units = acc;
    }
    __syncthreads();
    int run = sh_scan[warp] + incl - local;
    for (int r = r0; r < r1; ++r) {
      prefix[r] = run;
      run += attn_row_chunks(a.row_pos[r] + 1) * nkv;
    }
    if (tid == 0) prefix[a.rows] = sh_units;
    __syncthreads();
  }
  const int U = sh_units;
  if (tid == 0) attn_stamp(a, 1);

  if (warp == ATTN_CONSUMER_WARPS) {
    // ------------------------------------------------------------ page producer
    // The whole warp fetches a unit's page ids at once (lane i: pages i and 32 + i of
    // the unit) and prefetches the next unit's while the current one streams, so issuing a
    // stage never waits on a row_slot -> page_table pointer chase.
    int sl = 0, gs = 0;
    uint32_t ph = 0;  // (gs / ATTN_STAGES) & 1, kept incrementally
    // Each KV byte is read once per launch: evict-first, so the stream leaves L2's other
    // contents (weights prefetched for the next launch, activations) in place.
    const uint64_t kv_pol = l2_policy_evict_first();
    bool ok = true;
    const size_t head_stride = static_cast<size_t>(64) * 128;  // elements per (page, layer, which, head)
    auto page_base = [&](int page, int which, int g) {
      return a.kv.pool + ((((static_cast<size_t>(page) * a.kv.layers + a.layer) * 2 + which) * a.kv.nkv + g) *
                          head_stride);
    };
    auto fetch = [&](int u, AttnUnit& t, int& slot, int& pg0, int& pg1) {
      t = attn_unit(a, prefix, u);
      slot = a.row_slot[t.r];
      const int pages = (t.len + 63) >> 6;
      const int p0 = t.s0 * 2;
      const int* row = a.kv.page_table + static_cast<size_t>(slot) * a.kv.max_pages;
      pg0 = (p0 + lane < pages) ? row[p0 + lane] : 0;
      pg1 = (p0 + 32 + lane < pages) ? row[p0 + 32 + lane] : 0;
    };
    AttnUnit t{}, tn{};
    int slot = 0, pg0 = 0, pg1 = 0, slotn = 0, pn0 = 0, pn1 = 0;
    // Stages issued before griddepcontrol.wait (at most the ring's depth) that start a
    // unit still owe their q rows: the pending q source per ring slot, loaded after the wait.
    bool waited = a.early <= 0;
    const __half* q_owed[ATTN_STAGES] = {};
    auto wait_prev = [&]() {
      griddep_wait();
      waited = true;
      if (lane == 0)
        for (int j = 0; j < ATTN_STAGES; ++j)
          if (q_owed[j] != nullptr) bulk_load(&sm_q[j][0], q_owed[j], 512u, &full_bar[j]);
    };
    int u = blockIdx.x;
    if (u < U) fetch(u, t, slot, pg0, pg1);
    for (; u < U && ok; u += gridDim.x) {
      const int un = u + gridDim.x;
      if (un < U) fetch(un, tn, slotn, pn0, pn1);  // in flight while this unit streams
      const int pages = (t.len + 63) >> 6;
      const int* row = a.kv.page_table + static_cast<size_t>(slot) * a.kv.max_pages;
      for (int st = t.s0; st < t.s1; ++st) {
        // before the wait: only the first ring pass, and only stages of older positions
        if (!waited && (gs >= ATTN_STAGES || (st + 1) * 128 > t.len - a.early)) wait_prev();
        int w = 1;
        if (lane == 0) w = mbar_wait(&empty_bar[sl], ph ^ 1u, &abort_flag, a.status, 0x601) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, w, 0)) {
          ok = false;
          break;
        }
        const int p0 = st * 2;
        const int np = min(2, pages - p0);
        int pid[2];
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          const int ui = p0 + pp - t.s0 * 2;  // page index within the unit
          const int v0 = __shfl_sync(0xffffffffu, pg0, ui & 31);
          const int v1 = __shfl_sync(0xffffffffu, pg1, ui & 31);
          pid[pp] = ui < 32 ? v0 : v1;
        }
        if (lane == 0) {
          uint8_t* buf = smem + static_cast<size_t>(sl) * ATTN_STAGE_BYTES;
          const bool first = st == t.s0;
          mbar_arrive_expect_tx(&full_bar[sl],
                                static_cast<uint32_t>(np) * 2u * ATTN_PAGE_BYTES + (first ? 512u : 0u));
          if (first) {  // the unit's q rows (heads 2g, 2g+1: 512 contiguous bytes) ride along
            const __half* qs = a.q + static_cast<size_t>(t.r) * a.q_ld + 2 * t.g * 128;
            if (waited) bulk_load(&sm_q[sl][0], qs, 512u, &full_bar[sl]);
            else q_owed[sl] = qs;
          }
          for (int pp = 0; pp < np; ++pp) {
            const int ui = p0 + pp - t.s0 * 2;
            const int page = ui < 64 ? pid[pp] : row[p0 + pp];  // units longer than 64 pages: direct
            bulk_load_hint(buf + pp * ATTN_PAGE_BYTES, page_base(page, 0, t.g), ATTN_PAGE_BYTES, &full_bar[sl], kv_pol);
            bulk_load_hint(buf + (2 + pp) * ATTN_PAGE_BYTES, page_base(page, 1, t.g), ATTN_PAGE_BYTES, &full_bar[sl],
                           kv_pol);
          }
        }
        ++gs;
        if (++sl == ATTN_STAGES) {
          sl = 0;
          ph ^= 1u;
        }
      }
      t = tn;
      slot = slotn;
      pg0 = pn0;
      pg1 = pn1;
    }
    if (!waited) wait_prev();
    if (lane == 0) {
      attn_stamp(a, 6);
      for (int j = gs > ATTN_STAGES ? gs - ATTN_STAGES : 0; j < gs; ++j)  // drain
        mbar_wait(&full_bar[j % ATTN_STAGES], static_cast<uint32_t>((j / ATTN_STAGES) & 1), nullptr,
                  a.status, 0x602);
    }
  } else if (warp == ATTN_CONSUMER_WARPS + 1) {
    // ------------------------------------------------------------ merger
    // Combines the 8 warps of a unit; stores the output (one-chunk rows) or the chunk's
    // partial (m, l, o) for attention_merge_kernel.  No fence or atomic on this path: a
    // gpu-scope fence here would also wait for the CTA's page copies in flight.
    if (a.early > 0) griddep_wait();
    int k = 0;
    for (int u = blockIdx.x; u < U; u += gridDim.x, ++k) {
      const AttnUnit t = attn_unit(a, prefix, u);
      const int b = k & 1;
      if (!mbar_wait_warp(&mfull_bar[b], static_cast<uint32_t>((k >> 1) & 1), &abort_flag, a.status, 0x604))
        break;
      // lane covers dims [4 lane, +4) of both heads
      float M[2], Ls[2], O[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < ATTN_CONSUMER_WARPS; ++w) mx = fmaxf(mx, sm_m[b][w][h]);
        float ls = 0.f;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < ATTN_CONSUMER_WARPS; ++w) {
          const float mw = sm_m[b][w][h];
          if (mw == -INFINITY) continue;
          const float f = expf(mw - mx);
          ls += sm_l[b][w][h] * f;
          const float4 v = *reinterpret_cast<const float4*>(&sm_acc[b][w][h][4 * lane]);
          o[0] += v.x * f;
          o[1] += v.y * f;
          o[2] += v.z * f;
          o[3] += v.w * f;
        }
        M[h] = mx;
        Ls[h] = ls;
#pragma unroll
        for (int d = 0; d < 4; ++d) O[h][d] = o[d];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&mfree_bar[b]);  // state read: the consumers may reuse the buffer
      if (lane == 0 && k == 0) attn_stamp(a, 3);
      if (t.nch == 1) {
        __half* outp = a.out + static_cast<size_t>(t.r) * a.q_ld + (2 * t.g) * 128 + 4 * lane;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          __half2 v01 = __floats2half2_rn(O[h][0] / Ls[h], O[h][1] / Ls[h]);
          __half2 v23 = __floats2half2_rn(O[h][2] / Ls[h], O[h][3] / Ls[h]);
          uint2 pk;
          pk.x = *reinterpret_cast<uint32_t*>(&v01);
          pk.y = *reinterpret_cast<uint32_t*>(&v23);
          *reinterpret_cast<uint2*>(outp + h * 128) = pk;
        }
      } else {
        float* part = a.ws + ((static_cast<size_t>(t.r) * nkv + t.g) * ATTN_ROW_CHUNKS + t.c) * ATTN_PART_FLOATS;
        if (lane == 0) *reinterpret_cast<float4*>(part) = make_float4(M[0], M[1], Ls[0], Ls[1]);
#pragma unroll
        for (int h = 0; h < 2; ++h)
          *reinterpret_cast<float4*>(part + 4 + h * 128 + 4 * lane) = make_float4(O[h][0], O[h][1], O[h][2], O[h][3]);
      }
    }
    if (lane == 0) attn_stamp(a, 5);
  } else {
    // ------------------------------------------------------------ consumers (tensor cores)
    // Per stage a warp owns 16 positions and computes, transposed so that positions and
    // dims take the 16-wide M side of mma.sync m16n8k16 and the two GQA heads the N side:
    //   S^T [16 pos x 8] = K [16 pos x 128] . Q^T [128 x 8]      (8 MMAs, K via ldmatrix)
    //   O^T [128 x 8]   += V^T [128 x 16 pos] . P^T [16 pos x 8] (8 m-tiles x hi/lo = 16 MMAs)
    // Q columns 2..7 are zero.  Lane (g4 = lane / 4, tig = lane % 4) holds S^T / O^T
    // columns 2 tig, 2 tig + 1, so the real heads 0 and 1 live in the tig == 0 lanes: scores
    // of positions g4 and g4 + 8, and O^T rows 16 mt + g4 and 16 mt + g4 + 8.  P (f32) is
    // split into f16 hi + lo terms so the softmax weights keep ~22 bits.
    const int g4 = lane >> 2, tig = lane & 3;
    const int lrow = lane & 7, lmat = lane >> 3;
    if (a.early > 0) griddep_wait();
    int sl = 0, k = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < U && ok; u += gridDim.x, ++k) {
      const AttnUnit t = attn_unit(a, prefix, u);
      uint32_t qb[8][2];
      float o[8][4];
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
      for (int st = t.s0; st < t.s1; ++st) {
        if (!mbar_wait_warp(&full_bar[sl], ph, &abort_flag, a.status, 0x603)) {
          ok = false;
          break;
        }
        if (k == 0 && st == t.s0 && tid == 0) attn_stamp(a, 2);
        if (st == t.s0) {  // Q^T B fragments: head g4 (g4 < 2), dims 16 ks + 2 tig (+8)
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            qb[ks][0] = g4 < 2 ? *reinterpret_cast<const uint32_t*>(&sm_q[sl][g4 * 128 + 16 * ks + 2 * tig]) : 0u;
            qb[ks][1] = g4 < 2 ? *reinterpret_cast<const uint32_t*>(&sm_q[sl][g4 * 128 + 16 * ks + 8 + 2 * tig]) : 0u;
          }
        }
        const int tw = st * 128 + warp * 16;  // first position of this warp's 16
        if (tw < t.len) {
          const uint8_t* buf = smem + static_cast<size_t>(sl) * ATTN_STAGE_BYTES;
          const uint32_t kb = smem_u32(buf) + warp * 16 * 256;
          const uint32_t vb = smem_u32(buf + 2 * ATTN_PAGE_BYTES) + warp * 16 * 256;
          float sacc[4] = {0.f, 0.f, 0.f, 0.f};
          {
            const int pl = (lmat & 1) * 8 + lrow;  // position this lane addresses
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const int chunk = 2 * ks + (lmat >> 1);
              uint32_t a0, a1, a2, a3;
              ldmatrix_x4(kb + pl * 256 + ((chunk ^ lrow) << 4), a0, a1, a2, a3);
              mma_16816(sacc, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
            }
          }
          // sacc: [pos g4][head 2tig], [pos g4][2tig+1], [pos g4+8][2tig], [pos g4+8][2tig+1]
          const bool v0 = tw + g4 < t.len, v1 = tw + g4 + 8 < t.len;
          float sc[4] = {v0 ? sacc[0] * a.scale : -INFINITY, v0 ? sacc[1] * a.scale : -INFINITY,
                         v1 ? sacc[2] * a.scale : -INFINITY, v1 ? sacc[3] * a.scale : -INFINITY};
          float p[4], corr[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(sc[h], sc[2 + h]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(m[h], mx);  // finite: position tw is always valid
            corr[h] = (m[h] == mn) ? 1.0f : expf(m[h] - mn);
            p[h] = v0 ? expf(sc[h] - mn) : 0.f;
            p[2 + h] = v1 ? expf(sc[2 + h] - mn) : 0.f;
            l[h] = l[h] * corr[h] + (p[h] + p[2 + h]);
            m[h] = mn;
          }
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[mt][0] *= corr[0];
            o[mt][1] *= corr[1];
            o[mt][2] *= corr[0];
            o[mt][3] *= corr[1];
          }
          // P^T B fragments for column (head) g4: positions 2 tig, 2 tig + 1 (b0) and
          // 8 + 2 tig, 9 + 2 tig (b1), held by lanes 8 tig and 8 tig + 4 (tig == 0 there)
          const int s0l = 8 * tig, s1l = 8 * tig + 4;
          const float x00 = __shfl_sync(0xffffffffu, p[0], s0l), x01 = __shfl_sync(0xffffffffu, p[1], s0l);
          const float y00 = __shfl_sync(0xffffffffu, p[0], s1l), y01 = __shfl_sync(0xffffffffu, p[1], s1l);
          const float x20 = __shfl_sync(0xffffffffu, p[2], s0l), x21 = __shfl_sync(0xffffffffu, p[3], s0l);
          const float y20 = __shfl_sync(0xffffffffu, p[2], s1l), y21 = __shfl_sync(0xffffffffu, p[3], s1l);
          const bool real = g4 < 2;
          const float pa = real ? (g4 == 0 ? x00 : x01) : 0.f, pb = real ? (g4 == 0 ? y00 : y01) : 0.f;
          const float pc = real ? (g4 == 0 ? x20 : x21) : 0.f, pd = real ? (g4 == 0 ? y20 : y21) : 0.f;
          const __half2 h0 = __floats2half2_rn(pa, pb), h1 = __floats2half2_rn(pc, pd);
          const float2 r0 = __half22float2(h0), r1 = __half22float2(h1);
          const __half2 l0 = __floats2half2_rn(pa - r0.x, pb - r0.y), l1 = __floats2half2_rn(pc - r1.x, pd - r1.y);
          const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&h0), bh1 = *reinterpret_cast<const uint32_t*>(&h1);
          const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&l0), bl1 = *reinterpret_cast<const uint32_t*>(&l1);
          {
            const int pl = (lmat >> 1) * 8 + lrow;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              const int chunk = 2 * mt + (lmat & 1);
              uint32_t a0, a1, a2, a3;
              ldmatrix_x4_trans(vb + pl * 256 + ((chunk ^ lrow) << 4), a0, a1, a2, a3);
              mma_16816(o[mt], a0, a1, a2, a3, bh0, bh1);
              mma_16816(o[mt], a0, a1, a2, a3, bl0, bl1);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[sl]);
        if (++sl == ATTN_STAGES) {
          sl = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
      // ---- hand this warp's state to the merger (double-buffered by unit parity)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 4);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 8);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 16);
      }
      const int b = k & 1;
      if (!mbar_wait_warp(&mfree_bar[b], static_cast<uint32_t>(((k >> 1) & 1) ^ 1), &abort_flag, a.status,
                          0x605))
        break;
      if (tig == 0) {
        if (g4 == 0) {
          sm_m[b][warp][0] = m[0];
          sm_m[b][warp][1] = m[1];
          sm_l[b][warp][0] = l[0];
          sm_l[b][warp][1] = l[1];
        }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          sm_acc[b][warp][0][16 * mt + g4] = o[mt][0];
          sm_acc[b][warp][1][16 * mt + g4] = o[mt][1];
          sm_acc[b][warp][0][16 * mt + g4 + 8] = o[mt][2];
          sm_acc[b][warp][1][16 * mt + g4 + 8] = o[mt][3];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&mfull_bar[b]);
    }
    if (tid == 0) {
      attn_stamp(a, 4);
      if (a.trace != nullptr) a.trace[blockIdx.x * ATTN_TRACE_SLOTS + 7] = static_cast<unsigned long long>(k);
    }
  }
}

// Rows cut into several chunks: merge the chunks' (m, l, o) in index order and store
// the f16 output.  One CTA of 256 threads per (row, kv head); one-chunk rows exit.
__global__ void __launch_bounds__(256) attention_merge_kernel(const __grid_constant__ AttnArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int nkv = a.kv.nkv;
  const int r = blockIdx.x / nkv, g = blockIdx.x % nkv;
  if (r >= a.rows) return;
  const int len = a.row_pos[r] + 1;
  const int nch = attn_row_chunks(len);
  if (nch == 1) return;
  const int h = threadIdx.x >> 7, d = threadIdx.x & 127;
  const float* parts = a.ws + (static_cast<size_t>(r) * nkv + g) * ATTN_ROW_CHUNKS * ATTN_PART_FLOATS;
  float mc[ATTN_ROW_CHUNKS], lc[ATTN_ROW_CHUNKS], oc[ATTN_ROW_CHUNKS];
#pragma unroll
  for (int c = 0; c < ATTN_ROW_CHUNKS; ++c) {  // independent loads, all in flight
    const bool have = c < nch;
    mc[c] = have ? parts[c * ATTN_PART_FLOATS + h] : -INFINITY;
    lc[c] = have ? parts[c * ATTN_PART_FLOATS + 2 + h] : 0.f;
    oc[c] = have ? parts[c * ATTN_PART_FLOATS + 4 + h * 128 + d] : 0.f;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int c = 0; c < ATTN_ROW_CHUNKS; ++c) mx = fmaxf(mx, mc[c]);
  float ls = 0.f, os = 0.f;
#pragma unroll
  for (int c = 0; c < ATTN_ROW_CHUNKS; ++c) {
    if (mc[c] == -INFINITY) continue;
    const float f = expf(mc[c] - mx);
    ls += lc[c] * f;
    os += oc[c] * f;
  }
  a.out[static_cast<size_t>(r) * a.q_ld + (2 * g + h) * 128 + d] = __float2half_rn(os / ls);
}

}  // namespace qasr
