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
// positions of a stage, lane l holding dims [4l, 4l+4): 32 partial dot products
// (16 positions x 2 heads) are finished by one 5-round transposing butterfly and the
// softmax is online per head and warp.  At a unit's end the consumer warps drop their
// state into a double-buffered shared slot and move on; warp 9 merges the 8 warps,
// stores the output (or the chunk's partial), and the CTA that finishes a row's last
// chunk merges the chunks in index order (atomic counter, no waiting).
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
  float* ws;        // [rows * nkv * ATTN_ROW_CHUNKS][ATTN_PART_FLOATS]
  int* counters;    // [rows * nkv], zero between launches
  int max_chunks;
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
  __shared__ __align__(16) float sm_p[ATTN_CONSUMER_WARPS][32];
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
  griddep_wait();
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
    int u = blockIdx.x;
    if (u < U) fetch(u, t, slot, pg0, pg1);
    for (; u < U && ok; u += gridDim.x) {
      const int un = u + gridDim.x;
      if (un < U) fetch(un, tn, slotn, pn0, pn1);  // in flight while this unit streams
      const int pages = (t.len + 63) >> 6;
      const int* row = a.kv.page_table + static_cast<size_t>(slot) * a.kv.max_pages;
      for (int st = t.s0; st < t.s1; ++st) {
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
          if (first)  // the unit's q rows (heads 2g, 2g+1: 512 contiguous bytes) ride along
            bulk_load(&sm_q[sl][0], a.q + static_cast<size_t>(t.r) * a.q_ld + 2 * t.g * 128, 512u, &full_bar[sl]);
          for (int pp = 0; pp < np; ++pp) {
            const int ui = p0 + pp - t.s0 * 2;
            const int page = ui < 64 ? pid[pp] : row[p0 + pp];  // units longer than 64 pages: direct
            bulk_load(buf + pp * ATTN_PAGE_BYTES, page_base(page, 0, t.g), ATTN_PAGE_BYTES, &full_bar[sl]);
            bulk_load(buf + (2 + pp) * ATTN_PAGE_BYTES, page_base(page, 1, t.g), ATTN_PAGE_BYTES, &full_bar[sl]);
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
    if (lane == 0) {
      attn_stamp(a, 6);
      for (int j = gs > ATTN_STAGES ? gs - ATTN_STAGES : 0; j < gs; ++j)  // drain
        mbar_wait(&full_bar[j % ATTN_STAGES], static_cast<uint32_t>((j / ATTN_STAGES) & 1), nullptr,
                  a.status, 0x602);
    }
  } else if (warp == ATTN_CONSUMER_WARPS + 1) {
    // ------------------------------------------------------------ merger
    int k = 0;
    for (int u = blockIdx.x; u < U; u += gridDim.x, ++k) {
      const AttnUnit t = attn_unit(a, prefix, u);
      const int b = k & 1;
      if (!mbar_wait_warp(&mfull_bar[b], static_cast<uint32_t>((k >> 1) & 1), &abort_flag, a.status, 0x604))
        break;
      // lane covers dims [4 lane, +4) of both heads; combine the 8 warps
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
      __half* outp = a.out + static_cast<size_t>(t.r) * a.q_ld + (2 * t.g) * 128 + 4 * lane;
      if (t.nch == 1) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float inv = 1.0f / Ls[h];
          __half2 v01 = __floats2half2_rn(O[h][0] / Ls[h], O[h][1] / Ls[h]);
          __half2 v23 = __floats2half2_rn(O[h][2] / Ls[h], O[h][3] / Ls[h]);
          (void)inv;
          uint2 pk;
          pk.x = *reinterpret_cast<uint32_t*>(&v01);
          pk.y = *reinterpret_cast<uint32_t*>(&v23);
          *reinterpret_cast<uint2*>(outp + h * 128) = pk;
        }
      } else {
        const size_t pidx = (static_cast<size_t>(t.r) * nkv + t.g) * ATTN_ROW_CHUNKS;
        float* part = a.ws + (pidx + t.c) * ATTN_PART_FLOATS;
        if (lane == 0) {
          part[0] = M[0];
          part[1] = M[1];
          part[2] = Ls[0];
          part[3] = Ls[1];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
          __stcg(reinterpret_cast<float4*>(part + 4 + h * 128 + 4 * lane),
                 make_float4(O[h][0], O[h][1], O[h][2], O[h][3]));
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = (atomicAdd(a.counters + t.r * nkv + t.g, 1) == t.nch - 1) ? 1 : 0;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          const float* parts = a.ws + pidx * ATTN_PART_FLOATS;
          float mc[ATTN_ROW_CHUNKS][2], lc[ATTN_ROW_CHUNKS][2];
          float4 oc[ATTN_ROW_CHUNKS][2];
#pragma unroll
          for (int cc = 0; cc < ATTN_ROW_CHUNKS; ++cc) {  // independent loads, all in flight
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (cc < t.nch) {
                mc[cc][h] = __ldcg(parts + cc * ATTN_PART_FLOATS + h);
                lc[cc][h] = __ldcg(parts + cc * ATTN_PART_FLOATS + 2 + h);
                oc[cc][h] = __ldcg(reinterpret_cast<const float4*>(parts + cc * ATTN_PART_FLOATS + 4 + h * 128 + 4 * lane));
              } else {
                mc[cc][h] = -INFINITY;
                lc[cc][h] = 0.f;
                oc[cc][h] = make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float mx = -INFINITY;
#pragma unroll
            for (int cc = 0; cc < ATTN_ROW_CHUNKS; ++cc) mx = fmaxf(mx, mc[cc][h]);
            float ls = 0.f;
            float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int cc = 0; cc < ATTN_ROW_CHUNKS; ++cc) {
              if (mc[cc][h] == -INFINITY) continue;
              const float f = expf(mc[cc][h] - mx);
              ls += lc[cc][h] * f;
              o[0] += oc[cc][h].x * f;
              o[1] += oc[cc][h].y * f;
              o[2] += oc[cc][h].z * f;
              o[3] += oc[cc][h].w * f;
            }
            __half2 v01 = __floats2half2_rn(o[0] / ls, o[1] / ls);
            __half2 v23 = __floats2half2_rn(o[2] / ls, o[3] / ls);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&v01);
            pk.y = *reinterpret_cast<uint32_t*>(&v23);
            *reinterpret_cast<uint2*>(outp + h * 128) = pk;
          }
          if (lane == 0) a.counters[t.r * nkv + t.g] = 0;
        }
      }
    }
    if (lane == 0) attn_stamp(a, 5);
  } else {
    // ------------------------------------------------------------ consumers
    int sl = 0, k = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < U && ok; u += gridDim.x, ++k) {
      const AttnUnit t = attn_unit(a, prefix, u);
      float qa[4], qb[4];
      // lanes 0-15 carry head 2g's running max / partial sum, lanes 16-31 head 2g+1's
      float m = -INFINITY, l = 0.f;
      float acc_a[4] = {0.f, 0.f, 0.f, 0.f}, acc_b[4] = {0.f, 0.f, 0.f, 0.f};
      for (int st = t.s0; st < t.s1; ++st) {
        if (!mbar_wait_warp(&full_bar[sl], ph, &abort_flag, a.status, 0x603)) {
          ok = false;
          break;
        }
        if (k == 0 && st == t.s0 && tid == 0) attn_stamp(a, 2);
        if (st == t.s0) {
          const uint2 qa2 = *reinterpret_cast<const uint2*>(&sm_q[sl][4 * lane]);
          const uint2 qb2 = *reinterpret_cast<const uint2*>(&sm_q[sl][128 + 4 * lane]);
          const float2 a01 = __half22float2(*reinterpret_cast<const __half2*>(&qa2.x));
          const float2 a23 = __half22float2(*reinterpret_cast<const __half2*>(&qa2.y));
          const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&qb2.x));
          const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&qb2.y));
          qa[0] = a01.x; qa[1] = a01.y; qa[2] = a23.x; qa[3] = a23.y;
          qb[0] = b01.x; qb[1] = b01.y; qb[2] = b23.x; qb[3] = b23.y;
        }
        const int tw = st * 128 + warp * 16;  // first position of this warp's 16
        if (tw < t.len) {
          const uint8_t* buf = smem + static_cast<size_t>(sl) * ATTN_STAGE_BYTES;
          const __half* kbuf = reinterpret_cast<const __half*>(buf) + warp * 16 * 128;
          const __half* vbuf = reinterpret_cast<const __half*>(buf + 2 * ATTN_PAGE_BYTES) + warp * 16 * 128;
          float v[32];
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            const uint2 kr = *reinterpret_cast<const uint2*>(kbuf + p * 128 + 4 * lane);
            const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kr.x));
            const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kr.y));
            v[p] = fmaf(qa[3], k23.y, fmaf(qa[2], k23.x, fmaf(qa[1], k01.y, qa[0] * k01.x)));
            v[16 + p] = fmaf(qb[3], k23.y, fmaf(qb[2], k23.x, fmaf(qb[1], k01.y, qb[0] * k01.x)));
          }
          // transposing butterfly: lane j ends with the full dot product of value j
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < o; ++j) {
              const float send = upper ? v[j] : v[j + o];
              const float keep = upper ? v[j + o] : v[j];
              v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
          }
          const bool valid = tw + (lane & 15) < t.len;
          const float s = valid ? v[0] * a.scale : -INFINITY;
          float bm = s;
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
          const float mn = fmaxf(m, bm);
          const float corr = (m == mn) ? 1.0f : expf(m - mn);
          const float p = valid ? expf(s - mn) : 0.0f;
          l = l * corr + p;
          m = mn;
          sm_p[warp][lane] = p;
          const float ca = __shfl_sync(0xffffffffu, corr, 0);
          const float cb = __shfl_sync(0xffffffffu, corr, 16);
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            acc_a[d] *= ca;
            acc_b[d] *= cb;
          }
          __syncwarp();
          const int nvalid = min(16, t.len - tw);
#pragma unroll
          for (int p4 = 0; p4 < 4; ++p4) {
            const float4 pa4 = *reinterpret_cast<const float4*>(&sm_p[warp][4 * p4]);
            const float4 pb4 = *reinterpret_cast<const float4*>(&sm_p[warp][16 + 4 * p4]);
            const float pa[4] = {pa4.x, pa4.y, pa4.z, pa4.w};
            const float pb[4] = {pb4.x, pb4.y, pb4.z, pb4.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int pp = 4 * p4 + q;
              if (pp < nvalid) {
                const uint2 vr = *reinterpret_cast<const uint2*>(vbuf + pp * 128 + 4 * lane);
                const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vr.x));
                const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vr.y));
                acc_a[0] = fmaf(pa[q], v01.x, acc_a[0]);
                acc_a[1] = fmaf(pa[q], v01.y, acc_a[1]);
                acc_a[2] = fmaf(pa[q], v23.x, acc_a[2]);
                acc_a[3] = fmaf(pa[q], v23.y, acc_a[3]);
                acc_b[0] = fmaf(pb[q], v01.x, acc_b[0]);
                acc_b[1] = fmaf(pb[q], v01.y, acc_b[1]);
                acc_b[2] = fmaf(pb[q], v23.x, acc_b[2]);
                acc_b[3] = fmaf(pb[q], v23.y, acc_b[3]);
              }
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
      for (int o = 8; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      const int b = k & 1;
      if (!mbar_wait_warp(&mfree_bar[b], static_cast<uint32_t>(((k >> 1) & 1) ^ 1), &abort_flag, a.status,
                          0x605))
        break;
      if (lane == 0 || lane == 16) {
        sm_m[b][warp][lane >> 4] = m;
        sm_l[b][warp][lane >> 4] = l;
      }
      *reinterpret_cast<float4*>(&sm_acc[b][warp][0][4 * lane]) = make_float4(acc_a[0], acc_a[1], acc_a[2], acc_a[3]);
      *reinterpret_cast<float4*>(&sm_acc[b][warp][1][4 * lane]) = make_float4(acc_b[0], acc_b[1], acc_b[2], acc_b[3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&mfull_bar[b]);
    }
    if (tid == 0) {
      attn_stamp(a, 4);
      if (a.trace != nullptr) a.trace[blockIdx.x * ATTN_TRACE_SLOTS + 7] = static_cast<unsigned long long>(k);
    }
  }
}

}  // namespace qasr
