// Host-side helpers shared by the translation units that launch gemm_tc_kernel: TMA
// descriptors (through the driver entry point), the launch wrapper with programmatic
// stream serialization, and the stream-K GEMM plan.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>

#include "gemm_tc.cuh"

namespace qasr {

extern std::atomic<uint64_t> g_launches;

// ----------------------------------------------------------------------------- TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn(std::string* err) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn && err) *err = "cuTensorMapEncodeTiled is not available from the driver";
  return fn;
}

// 2-D row-major tensor [outer, inner] with 128-byte swizzled boxes {box_inner, box_outer}.
inline bool make_tmap(CUtensorMap* m, const void* base, bool bytes1, uint64_t inner,
                      uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                      std::string* err) {
  EncodeTiledFn fn = encode_fn(err);
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, bytes1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")";
    return false;
  }
  return true;
}

// 2-D row-major tensor [outer, inner] viewed as 3-D {64, outer, inner / 64}: one box of
// {64, box_outer, box_chunks} lands as box_chunks consecutive 128-byte swizzled [box_outer][64]
// tiles, the layout two 2-D boxes at consecutive 64-column offsets would give.
inline bool make_tmap_chunks(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                             uint32_t box_outer, uint32_t box_chunks, std::string* err) {
  EncodeTiledFn fn = encode_fn(err);
  if (!fn) return false;
  const cuuint64_t dims[3] = {64, outer, inner / 64};
  const cuuint64_t strides[2] = {row_bytes, 128};
  const cuuint32_t box[3] = {64, box_outer, box_chunks};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled (chunked view) failed (code " + std::to_string(static_cast<int>(r)) + ")";
    return false;
  }
  return true;
}

// ----------------------------------------------------------------------------- GEMM plan
struct Linear {
  void* w = nullptr;        // device, tiled layout (weight_tile_offset)
  void* scale = nullptr;    // device [n_out] (int8): f16, or f32 when scale32
  int n_out = 0, k = 0;
  bool int8 = false;
  bool scale32 = false;
};

// Launch with programmatic stream serialization (PDL) unless disabled by
// QASR_B200_NO_PDL=1: the kernel may start while its predecessor drains and orders
// itself with griddepcontrol.wait.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("QASR_B200_NO_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

struct GemmLaunch {
  CUtensorMap tmx{};
  GemmArgs args{};
  int grid = 0;
  size_t smem = 0;
  bool int8 = false;
  int epi = 0;
};

inline int g_dyn_smem_max = 0;
inline int g_chain_dyn_max = 0;

inline int cta_of_unit_host(long long x, long long units, long long grid) {
  return static_cast<int>(((x + 1) * grid + units - 1) / units - 1);
}

struct GemmShape {
  int n_tile, n_tiles, kblocks, tiles, units, grid, stages, max_seg;
  size_t smem, ws_floats;
};

// grid_override > 0 fixes the CTA count (at most num_sms); otherwise at least 4 units per CTA.
// wide: f16 weights over many rows may take 256-row activation tiles (UMMA N = 256): a
// unit then moves 16 KB of weights + 32 KB of activations for 4 MFLOP instead of 16 + 16 KB
// for 2 MFLOP, which raises the per-SM load ceiling; used only when the 256-row tiles still
// give every SM a tile (otherwise the narrower tiles spread the work better).
// n_tile_override > 0 (a multiple of 16, at most 128, below the default) narrows the
// activation tiles: more tiles for a GEMM over few rows.
inline GemmShape gemm_shape(int n_out, int k, bool int8, int rows, int num_sms, int grid_override = 0,
                            bool wide = false, int n_tile_override = 0) {
  GemmShape s{};
  s.n_tile = rows <= GEMM_MAX_NTILE ? std::max(16, (rows + 15) / 16 * 16) : GEMM_MAX_NTILE;
  if (n_tile_override > 0 && n_tile_override < s.n_tile) s.n_tile = n_tile_override;
  if (wide && !int8 && n_tile_override <= 0 && rows >= GEMM_WIDE_NTILE &&
      (n_out / 128) * ((rows + GEMM_WIDE_NTILE - 1) / GEMM_WIDE_NTILE) >= num_sms)
    s.n_tile = GEMM_WIDE_NTILE;
  s.n_tiles = (rows + s.n_tile - 1) / s.n_tile;
  const int ke = int8 ? 128 : 64;
  s.kblocks = k / ke;
  s.tiles = (n_out / 128) * s.n_tiles;
  s.units = s.tiles * s.kblocks;
  // at least 4 units per CTA: a CTA that streams less than ~64 KB of weights spends
  // more on its pipeline fill and split fixup than on the bytes
  s.grid = grid_override > 0 ? std::min(grid_override, std::min(num_sms, s.units))
                              : std::max(1, std::min(num_sms, s.units / 4));
  const int atoms = int8 ? 2 : 1;
  const int stage = 16384 + atoms * s.n_tile * 128;
  const int dyn = g_dyn_smem_max > 0 ? g_dyn_smem_max : 200 * 1024;
  // >= 3 stages: the int8 A builders publish units in pairs (see the kernel)
  s.stages = std::max(3, std::min(GEMM_MAX_STAGES, (dyn - 1024) / stage));
  s.smem = static_cast<size_t>(s.stages) * stage + 1024;
  int max_seg = 1;
  for (int t = 0; t < s.tiles; ++t) {
    const long long a = static_cast<long long>(t) * s.kblocks;
    const int f = cta_of_unit_host(a, s.units, s.grid);
    const int l = cta_of_unit_host(a + s.kblocks - 1, s.units, s.grid);
    max_seg = std::max(max_seg, l - f + 1);
  }
  s.max_seg = max_seg;
  s.ws_floats = max_seg > 1 ? static_cast<size_t>(s.tiles) * max_seg * s.n_tile * 128 : 0;
  return s;
}

// TMEM columns one gemm_tc_kernel CTA addresses: two accumulator buffers of the tile's
// width rounded to 32, and for int8 weights at least one 64-column dequantised A stage.
// Every tcgen05 access must stay inside the GEMM_TMEM_COLS the CTA allocates; a plan
// that would not is refused on the host (plan_gemm) rather than run.
inline bool gemm_tmem_fits(const GemmShape& s, bool int8) {
  const int dcols = (s.n_tile + 31) / 32 * 32;
  const int a_cols = int8 ? 64 : 0;  // at least one A stage
  return 2 * dcols + a_cols <= static_cast<int>(GEMM_TMEM_COLS);
}

// Dynamic shared memory limits and kernel attributes (once per device, on the current one).
cudaError_t init_kernel_attrs(std::string* err);

}  // namespace qasr
