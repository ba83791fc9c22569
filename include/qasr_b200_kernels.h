/*
 * qasr_b200_kernels.h — device-pointer entry points of the individual B200 kernels.
 *
 * The reference checks and measures its kernels one by one with dedicated probes:
 * src/bin/w8_probe.rs (W8 GEMV/GEMM vs an f64 reference), src/bin/batch_gemv_bench.rs
 * (batched GEMV bandwidth), src/bin/attn_bench.rs and src/bin/attn_slots_probe.rs
 * (decode attention).  These calls are the same seams for the B200 kernels: all
 * pointers are device pointers, `stream` is a cudaStream_t (NULL = legacy default
 * stream), nothing is synchronised.  Workspaces are cached per device inside the
 * library and only grow.  Errors are written to `err` (if non-NULL, `errlen` bytes).
 */
#ifndef QASR_B200_KERNELS_H
#define QASR_B200_KERNELS_H

#include <stdint.h>

#include "qasr_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Re-lay a row-major weight [n_out, k] (f16 or int8) into the tiled HBM layout the
 * GEMM streams: 16 KB blocks of 128 rows x 128 bytes, one per (row tile, k block),
 * 128-byte swizzle applied.  w_tiled must hold n_out * k * element-size bytes.
 * (The reference uploads the file bytes verbatim, src/weights.rs:300-308; the B200
 * loader re-lays them once at load.) */
qasr_status qasr_kernel_pack_weights(int device, void* stream, int weight_format,
                                     const void* w_rowmajor, int n_out, int k, void* w_tiled,
                                     char* err, int errlen);

/* out[r, m] = f16(sum_k W[m, k] x[r, k])            (accumulate == 0)
 * out[r, m] = f16(f32(out[r, m]) + sum_k ...)         (accumulate != 0)
 * W: [n_out, k] f16 (weight_format QASR_WEIGHTS_F16) or int8 + a per-row scale, f16
 * (QASR_WEIGHTS_INT8) or f32 (QASR_WEIGHTS_INT8_F32), value f16(f32(q) * s), in the
 * layout qasr_kernel_pack_weights produces.  n_out % 128 == 0; k % 128 == 0; x is
 * [rows, ldx] and out [rows, ldo] f16 with ldx >= k, ldo >= n_out (ldx * 2 a multiple of
 * 16 bytes, the activation copy's stride).
 * Replaces gemv / gemv_w8 / gemv_batch_slots / prefill_gemm(_w8)
 * (src/shaders.rs:273-889, 2995-3082). */
qasr_status qasr_kernel_gemm(int device, void* stream, int weight_format, const void* w,
                             const void* scale, int n_out, int k, const uint16_t* x, int ldx,
                             int rows, uint16_t* out, int ldo, int accumulate, char* err,
                             int errlen);

/* qasr_kernel_gemm with a latency trace: if `trace` (device, grid * 12 uint64) is
 * non-NULL each CTA records %globaltimer stamps of its pipeline milestones (entry, setup,
 * first weight/activation copies issued, first stage seen/built, first/last MMA, first
 * accumulator, last store, split fixup, exit); *grid_out receives the CTA count. */
qasr_status qasr_kernel_gemm_traced(int device, void* stream, int weight_format, const void* w,
                                    const void* scale, int n_out, int k, const uint16_t* x,
                                    int ldx, int rows, uint16_t* out, int ldo, int accumulate,
                                    unsigned long long* trace, int* grid_out, char* err,
                                    int errlen);

/* GQA attention of `rows` query rows over their slot's paged KV (gqa_decode_* /
 * gqa_split_merge, src/shaders.rs:1881-2905).  q/out: [rows, q_ld] f16 (q heads 2g and
 * 2g+1 read kv head g); kv_pool: [pages][layers][2][nkv][64][128] f16 with each
 * 128-dim row stored swizzled: dim d of position p sits at column
 * ((d/8) ^ (p%8))*8 + d%8 (16-byte chunks permuted by the position's low 3 bits, so
 * tensor-core fragment loads from shared memory are bank-conflict free); page_table:
 * [slots][max_pages] int32; row r attends positions 0..row_pos[r] of slot row_slot[r].
 * The device arrays are taken as given (the call checks only its scalar arguments):
 * row_pos[r] < max_pages * 64, and every page id the rows reach lies in kv_pool.
 * Only enqueues (for timing with the caller's events): a bounded device-side wait that
 * gives up is not reported by this call; the traced and no-alloc variants report it. */
qasr_status qasr_kernel_attention(int device, void* stream, const uint16_t* q, int q_ld,
                                  uint16_t* out, const uint16_t* kv_pool, const int* page_table,
                                  int max_pages, int layers, int nkv, int layer,
                                  const int* row_slot, const int* row_pos, int rows, char* err,
                                  int errlen);

/* qasr_kernel_attention with a latency trace: if `trace` (device, SM count x 8 uint64) is
 * non-NULL each CTA records %globaltimer stamps (entry, unit table ready, first stage
 * landed, first unit merged, last stage consumed, last unit merged, producer done) and
 * the number of units it processed.  Waits for its launches and returns
 * QASR_ERR_DEVICE_TIMEOUT if a bounded device-side wait gave up. */
qasr_status qasr_kernel_attention_traced(int device, void* stream, const uint16_t* q, int q_ld,
                                         uint16_t* out, const uint16_t* kv_pool,
                                         const int* page_table, int max_pages, int layers,
                                         int nkv, int layer, const int* row_slot,
                                         const int* row_pos, int rows, unsigned long long* trace,
                                         char* err, int errlen);

/* qasr_kernel_attention without any device allocation — for callers that may not call
 * cudaMalloc: hosts that hand the library a fixed memory budget up front (an embedding
 * application that owns all device memory), and real-time audio paths that must not
 * touch the allocator between frames (an allocation can block on the driver for
 * milliseconds).  No counterpart in the reference (its wgpu decoder owns all buffers).
 * The scratch is one static device array inside the library (about 2 MiB) plus an
 * 8-byte status word, held by every GPU that loads the library until the process exits, so:
 *   - at most 64 query rows and 8 kv heads per call; larger calls fail with
 *     QASR_ERR_CAPACITY (use qasr_kernel_attention);
 *   - the first call on a device looks the array's address up
 *     (cudaGetSymbolAddress): make that first call before any stream capture;
 *   - all calls share the array and the status word: calls that overlap on the GPU
 *     (other streams, other threads) race and must be serialised by the caller;
 *   - the call waits for its kernels on `stream` and reads the status word back, so a
 *     bounded device-side wait that gave up returns QASR_ERR_DEVICE_TIMEOUT.
 * Same inputs, outputs and results as qasr_kernel_attention. */
qasr_status qasr_kernel_attention_noalloc(int device, void* stream, const uint16_t* q, int q_ld,
                                          uint16_t* out, const uint16_t* kv_pool,
                                          const int* page_table, int max_pages, int layers,
                                          int nkv, int layer, const int* row_slot,
                                          const int* row_pos, int rows, char* err, int errlen);

/* Append K and V rows ([rows, nkv*128] f16 each) at (row_slot[r], row_pos[r]) of
 * layer `layer`, in the swizzled row layout qasr_kernel_attention reads — the cache
 * writes of qkv_extract(_slots) (src/shaders.rs:1376-1635). */
qasr_status qasr_kernel_kv_append(int device, void* stream, const uint16_t* k, const uint16_t* v,
                                  uint16_t* kv_pool, const int* page_table, int max_pages,
                                  int layers, int nkv, int layer, const int* row_slot,
                                  const int* row_pos, int rows, char* err, int errlen);

/* Number of kernels this library launched since load (all contexts and probes). */
uint64_t qasr_kernel_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* QASR_B200_KERNELS_H */
