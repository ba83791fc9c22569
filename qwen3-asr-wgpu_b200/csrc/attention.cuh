// GQA attention of query rows over their slot's paged KV (decode and prefill).
//
// Replaces gqa_decode_single(_slots), gqa_decode_split_p1(_pair) and gqa_split_merge
// (src/shaders.rs:1881-2182, 2270-2905); the math follows CpuTextDecoder::attention
// (src/cpu_decoder.rs:292-365): s_t = (q . k_t) * 1/sqrt(hd), softmax over t <= pos,
// o = f16(sum_t p_t v_t / sum_t p_t).
//
// Each query row r (slot s_r, position p_r) attends to positions [0, p_r] of its slot,
// which makes one kernel serve a decode step (one row per slot) and a prefill chunk
// (consecutive positions of a slot; causal by construction).
//
// Work unit = (row, kv head, chunk); both q heads of the kv head are done together so
// K/V are read once (the reference's "pair" kernel idea).  A row of length len is cut
// into chunks of CH = max(64, roundup64(len / ATTN_ROW_CHUNKS)) positions — a function
// of the row alone, so a slot's result does not depend on the other slots of the
// batch.  A row with several chunks is merged by the CTA that finishes its last chunk
// (atomic counter, no waiting), chunks in index order.
//
// Inside a unit each warp takes 32-position batches: lane L covers dims
// [8*(L%16), +8) of the positions p0 + 2*i + L/16 (i < 16), i.e. 16-byte loads that
// read a whole 256-byte K or V row per half-warp; the dot products are finished by a
// 4-round transposing butterfly, the softmax is online per warp, the warps merge in
// shared memory.
#pragma once
#include "device_common.cuh"
#include "gemm_tc.cuh"  // KvLayout, kv_elem_offset

namespace qasr {

constexpr int ATTN_THREADS = 128;
constexpr int ATTN_PART_FLOATS = 4 + 2 * 128;  // m_a, m_b, l_a, l_b, o_a[128], o_b[128]
constexpr int ATTN_ROW_CHUNKS = 8;             // chunks per row (upper bound)

__host__ __device__ __forceinline__ int attn_chunk_len(int len) {
  const int c = (len + ATTN_ROW_CHUNKS - 1) / ATTN_ROW_CHUNKS;
  const int r = (c + 63) / 64 * 64;
  return r < 64 ? 64 : r;
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
  float* ws;        // [rows * nkv * max_chunks][ATTN_PART_FLOATS]
  int* counters;    // [rows * nkv], zero between launches
  int max_chunks;
  uint32_t* status;
};

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__global__ void __launch_bounds__(ATTN_THREADS)
    attention_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ int prefix[];  // rows + 1 entries
  __shared__ int sh_units;
  __shared__ float sm_m[4][2], sm_l[4][2];
  __shared__ float sm_acc[4][2][128];
  __shared__ int sh_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkv = a.kv.nkv;
  griddep_wait();
  griddep_launch_dependents();

  // ---- unit decomposition (identical in every CTA) ----
  if (tid == 0) {
    int acc = 0;
    for (int r = 0; r < a.rows; ++r) {
      prefix[r] = acc;
      const int len = a.row_pos[r] + 1;
      const int ch = attn_chunk_len(len);
      acc += ((len + ch - 1) / ch) * nkv;
    }
    prefix[a.rows] = acc;
    sh_units = acc;
  }
  __syncthreads();
  const int U = sh_units;

  for (int u = blockIdx.x; u < U; u += gridDim.x) {
    // find row r with prefix[r] <= u < prefix[r+1]
    int lo = 0, hi = a.rows - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    const int r = lo;
    const int len = a.row_pos[r] + 1;
    const int CH = attn_chunk_len(len);
    const int nch = (len + CH - 1) / CH;
    const int rem = u - prefix[r];
    const int g = rem / nch, c = rem % nch;
    const int slot = a.row_slot[r];
    const int t0 = c * CH;
    const int t1 = min(t0 + CH, len);

    // q of heads 2g, 2g+1 for this lane's 8 dims
    const int d0 = 8 * (lane & 15);
    const int hw = lane >> 4;
    float qa[8], qb[8];
    unpack8(*reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(r) * a.q_ld + (2 * g) * 128 + d0), qa);
    unpack8(*reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(r) * a.q_ld + (2 * g + 1) * 128 + d0), qb);

    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    float acc_a[8], acc_b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc_a[i] = acc_b[i] = 0.f;

    for (int p0 = t0 + warp * 32; p0 < t1; p0 += 4 * 32) {
      const size_t kbase = kv_elem_offset(a.kv, slot, p0, a.layer, 0, g);
      const size_t vbase = kv_elem_offset(a.kv, slot, p0, a.layer, 1, g);
      const __half* kp = a.kv.pool + kbase + d0;
      const __half* vp = a.kv.pool + vbase + d0;
      float da[16], db[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint4 kr = __ldg(reinterpret_cast<const uint4*>(kp + (2 * i + hw) * 128));
        float kf[8];
        unpack8(kr, kf);
        float sa = 0.f, sb = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          sa = fmaf(qa[d], kf[d], sa);
          sb = fmaf(qb[d], kf[d], sb);
        }
        da[i] = sa;
        db[i] = sb;
      }
      // transposing butterfly over the 16 lanes of each half-warp: lane j ends up with
      // the full dot product of position index j
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < o; ++j) {
          const float send_a = upper ? da[j] : da[j + o];
          const float keep_a = upper ? da[j + o] : da[j];
          const float send_b = upper ? db[j] : db[j + o];
          const float keep_b = upper ? db[j + o] : db[j];
          da[j] = keep_a + __shfl_xor_sync(0xffffffffu, send_a, o);
          db[j] = keep_b + __shfl_xor_sync(0xffffffffu, send_b, o);
        }
      }
      const int my_pos = p0 + 2 * (lane & 15) + hw;
      const bool valid = my_pos < t1;
      const float s_a = valid ? da[0] * a.scale : -INFINITY;
      const float s_b = valid ? db[0] * a.scale : -INFINITY;
      float bm_a = s_a, bm_b = s_b;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        bm_a = fmaxf(bm_a, __shfl_xor_sync(0xffffffffu, bm_a, o));
        bm_b = fmaxf(bm_b, __shfl_xor_sync(0xffffffffu, bm_b, o));
      }
      const float mn_a = fmaxf(m_a, bm_a), mn_b = fmaxf(m_b, bm_b);
      const float corr_a = expf(m_a - mn_a), corr_b = expf(m_b - mn_b);
      const float p_a = valid ? expf(s_a - mn_a) : 0.f;
      const float p_b = valid ? expf(s_b - mn_b) : 0.f;
      l_a = l_a * corr_a + p_a;
      l_b = l_b * corr_b + p_b;
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        acc_a[d] *= corr_a;
        acc_b[d] *= corr_b;
      }
      m_a = mn_a;
      m_b = mn_b;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float pa = __shfl_sync(0xffffffffu, p_a, (lane & 16) | i);
        const float pb = __shfl_sync(0xffffffffu, p_b, (lane & 16) | i);
        if (p0 + 2 * i + hw < t1) {
          const uint4 vr = __ldg(reinterpret_cast<const uint4*>(vp + (2 * i + hw) * 128));
          float vf[8];
          unpack8(vr, vf);
#pragma unroll
          for (int d = 0; d < 8; ++d) {
            acc_a[d] = fmaf(pa, vf[d], acc_a[d]);
            acc_b[d] = fmaf(pb, vf[d], acc_b[d]);
          }
        }
      }
    }
    // combine the two half-warps (same running max) and the lanes' partial sums
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      acc_a[d] += __shfl_xor_sync(0xffffffffu, acc_a[d], 16);
      acc_b[d] += __shfl_xor_sync(0xffffffffu, acc_b[d], 16);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      l_a += __shfl_xor_sync(0xffffffffu, l_a, o);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, o);
    }
    if (lane == 0) {
      sm_m[warp][0] = m_a;
      sm_m[warp][1] = m_b;
      sm_l[warp][0] = l_a;
      sm_l[warp][1] = l_b;
    }
    if (lane < 16) {
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        sm_acc[warp][0][d0 + d] = acc_a[d];
        sm_acc[warp][1][d0 + d] = acc_b[d];
      }
    }
    __syncthreads();
    // merge the 4 warps: thread tid owns dim tid of both heads
    float M[2], L[2], O[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
      for (int w = 0; w < 4; ++w) mx = fmaxf(mx, sm_m[w][h]);
      float ls = 0.f, os = 0.f;
      for (int w = 0; w < 4; ++w) {
        if (sm_m[w][h] == -INFINITY) continue;
        const float f = expf(sm_m[w][h] - mx);
        ls += sm_l[w][h] * f;
        os += sm_acc[w][h][tid] * f;
      }
      M[h] = mx;
      L[h] = ls;
      O[h] = os;
    }
    const size_t obase = static_cast<size_t>(r) * a.q_ld + (2 * g) * 128 + tid;
    if (nch == 1) {
      a.out[obase] = __float2half_rn(O[0] / L[0]);
      a.out[obase + 128] = __float2half_rn(O[1] / L[1]);
    } else {
      const size_t pidx = (static_cast<size_t>(r) * nkv + g) * a.max_chunks;
      float* part = a.ws + (pidx + c) * ATTN_PART_FLOATS;
      if (tid == 0) {
        part[0] = M[0];
        part[1] = M[1];
        part[2] = L[0];
        part[3] = L[1];
      }
      part[4 + tid] = O[0];
      part[4 + 128 + tid] = O[1];
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const int old = atomicAdd(a.counters + r * nkv + g, 1);
        sh_last = (old == nch - 1) ? 1 : 0;
      }
      __syncthreads();
      if (sh_last) {
        __threadfence();
        const float* parts = a.ws + pidx * ATTN_PART_FLOATS;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float mx = -INFINITY;
          for (int cc = 0; cc < nch; ++cc) mx = fmaxf(mx, __ldcg(parts + cc * ATTN_PART_FLOATS + h));
          float ls = 0.f, os = 0.f;
          for (int cc = 0; cc < nch; ++cc) {
            const float mc = __ldcg(parts + cc * ATTN_PART_FLOATS + h);
            if (mc == -INFINITY) continue;
            const float f = expf(mc - mx);
            ls += __ldcg(parts + cc * ATTN_PART_FLOATS + 2 + h) * f;
            os += __ldcg(parts + cc * ATTN_PART_FLOATS + 4 + h * 128 + tid) * f;
          }
          a.out[obase + h * 128] = __float2half_rn(os / ls);
        }
        if (tid == 0) a.counters[r * nkv + g] = 0;
      }
    }
    __syncthreads();
  }
}

}  // namespace qasr
