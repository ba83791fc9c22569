// Row kernels around the GEMMs: embedding gather (+ decode row metadata), RMSNorm,
// argmax finalisation with on-device token feedback, token scatter.
#pragma once
#include "device_common.cuh"
#include "gemm_tc.cuh"  // griddep_wait / griddep_launch_dependents

namespace qasr {

// embed_lookup_single (src/shaders.rs:2956-2979) / embed_row (src/cpu_decoder.rs:256-259)
// for every decode row: h[r] = embed[next_tok[slot_r]], row_pos[r] = pos[slot_r].
__global__ void embed_rows_kernel(__half* __restrict__ h, const __half* __restrict__ embed, int hs,
                                  int vocab, const int* __restrict__ row_slot,
                                  const int* __restrict__ next_tok, const int* __restrict__ pos,
                                  int* __restrict__ row_pos, uint32_t* status) {
  griddep_wait();
  griddep_launch_dependents();
  const int r = blockIdx.x;
  const int slot = row_slot[r];
  int tok = next_tok[slot];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) report_error(status, DEVERR_BOUNDS, 0x501);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(embed + static_cast<size_t>(tok) * hs);
  uint4* dst = reinterpret_cast<uint4*>(h + static_cast<size_t>(r) * hs);
  for (int i = threadIdx.x; i < hs / 8; i += blockDim.x) dst[i] = src[i];
  if (threadIdx.x == 0) row_pos[r] = pos[slot];
}

// rms_norm_row (src/cpu_decoder.rs:261-272): out = f16(x * inv * w),
// inv = 1 / sqrt(sum(x^2) / n + eps).  `src_rows` (optional) picks the input row.
__global__ void rmsnorm_rows_kernel(__half* __restrict__ out, const __half* __restrict__ in,
                                    const int* __restrict__ src_rows, const float* __restrict__ w,
                                    int hs, float eps) {
  __shared__ float red[32];
  griddep_wait();
  griddep_launch_dependents();
  const int r = blockIdx.x;
  const int src = src_rows ? src_rows[r] : r;
  const __half* x = in + static_cast<size_t>(src) * hs;
  float s = 0.f;
  for (int i = threadIdx.x * 2; i < hs; i += blockDim.x * 2) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(x + i));
    s = __fadd_rn(s, __fmul_rn(v.x, v.x));
    s = __fadd_rn(s, __fmul_rn(v.y, v.y));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv =
      __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], static_cast<float>(hs)), eps)));
  __half* y = out + static_cast<size_t>(r) * hs;
  for (int i = threadIdx.x * 2; i < hs; i += blockDim.x * 2) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(x + i));
    const float a = __fmul_rn(__fmul_rn(v.x, inv), w[i]);
    const float b = __fmul_rn(__fmul_rn(v.y, inv), w[i + 1]);
    *reinterpret_cast<__half2*>(y + i) = __floats2half2_rn(a, b);
  }
}

// argmax_into_slot (src/shaders.rs:2907-2954) tail: decode the 64-bit max keys, reset
// them, hand each token to its slot (next step's input, read on device) and advance
// the slot's position past the row.  `epoch` (optional): the decode step's counter, one
// increment per step (the decode chain derives its flags from it).
__global__ void finalize_rows_kernel(unsigned long long* __restrict__ best, int rows,
                                     const int* __restrict__ row_slot,
                                     const int* __restrict__ row_pos, int* __restrict__ out_tok,
                                     int* __restrict__ next_tok, int* __restrict__ pos,
                                     unsigned int* __restrict__ epoch) {
  griddep_wait();
  griddep_launch_dependents();
  if (epoch != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *epoch += 1u;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const unsigned long long key = best[r];
  const int tok = static_cast<int>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
  best[r] = 0ull;
  out_tok[r] = tok;
  const int slot = row_slot[r];
  next_tok[slot] = tok;
  pos[slot] = row_pos[r] + 1;
}

// The bounded-wait error path, exercised without a fault: one thread waits on an
// mbarrier that nothing arrives on, then polls a word that nothing sets (the two wait
// forms the kernels use: within a CTA, and on another CTA's data), each giving up after
// `limit_ns` and recording DEVERR_TIMEOUT (first site wins) in the status word.
__global__ void wait_timeout_probe_kernel(const unsigned int* never_set, uint64_t limit_ns, uint32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  mbar_wait(&bar, 0, nullptr, status, 0x7f1, limit_ns);
  const uint64_t t0 = globaltimer();
  while (*reinterpret_cast<const volatile unsigned int*>(never_set) == 0u) {
    if (globaltimer() - t0 > limit_ns) {
      report_error(status, DEVERR_TIMEOUT, 0x7f2);
      break;
    }
    __nanosleep(256);
  }
}

__global__ void scatter_tokens_kernel(int* __restrict__ next_tok, const int* __restrict__ slots,
                                      const int* __restrict__ toks, int n) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) next_tok[slots[i]] = toks[i];
}

}  // namespace qasr
