// C ABI of the B200 fused MoE expert-MLP library: argument checking, TMA
// tensor-map setup, operand pre-split for the 3xTF32 path, and dispatch to
// the sm_100a kernels.  Declarations: include/moe_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/moe_b200.h"
#include "ep_exchange.cuh"
#include "router.cuh"
#include "fused_pair.cuh"
#include "grouped_gemm.cuh"
#include "grouped_gemm_swap.cuh"
#include "grouped_gemm_bwd.cuh"

namespace moe {
__device__ int g_status = 0;

// ------------------------------------------------------------------ errors
static thread_local char t_err[512] = {0};

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

#define MOE_CUDA_TRY(expr)                                                                   \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    if (_e != cudaSuccess) return fail(MOE_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

// ------------------------------------------------------------------ tuning
static int64_t g_tune_splits = 0;
static int64_t g_tune_ctas = 0;
static int64_t g_tune_trace = 0;  // device address of a trace buffer (MOE_TRACE builds)
static int64_t g_tune_pair = 0;   // 0 auto, 1 single-CTA kernel, 2 CTA-pair kernel
static int64_t g_tune_group_m = 0;  // grouped GEMMs: rasterisation group in 256-row blocks (0 = 8)
static int64_t g_tune_l2 = 0;       // grouped GEMMs: L2 hint mode of the A / B loads (GemmParams::l2_mode)
static int64_t g_tune_fp8 = 0;      // e4m3 weights: 0 automatic, 1 row-tiled pair kernel, 2 expert super-tiles
static int64_t g_tune_wide = 0;     // bf16 down GEMM: 0 automatic, 1 256-column tiles, 2 512-column tiles
static int64_t g_tune_tail = 0;     // fused small-D kernel: 0 automatic (half units in a short last wave), 1 off

// bf16 down GEMM (f32 Y): 256-column tiles unless 512 are asked for.  At C4
// the 512-column tiles cut the down GEMM's DRAM reads by a third (fewer
// waves re-read H and W_down) but take 3% more cycles (no double-buffered
// accumulator), and the clock under the power cap did not rise measurably.
static bool down_wide() { return g_tune_wide == 2; }

// e4m3-weight GELU experts: the super-tile (swap) kernel when the experts are
// small -- at most one super-tile (384 rows) on average -- else the row-tiled
// pair kernel.  Host-side only: the group sizes stay on the device.
static bool fp8_use_swap(int64_t M, int E) {
  if (g_tune_fp8 == 1) return false;
  if (g_tune_fp8 == 2) return true;
  return M <= (int64_t)SwapCfg<0>::TOKENS * E;
}

// ------------------------------------------------------------------ driver entry point
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// The current context of the calling thread (driver API through the runtime's
// entry-point query, so the library links no libcuda).  Per-device caches
// below remember the context they were filled in: after cudaDeviceReset the
// primary context is rebuilt, modules reload (device symbols may move) and
// function attributes are gone, so a cache from the old context is refilled.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
static CUcontext current_ctx() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

// Encoded maps of recent calls, per host thread: a map is a pure function of
// (base, type, shape, box), so a hit skips the driver call.  Weights,
// workspaces and reused activation buffers hit on repeated calls.
struct MapKey {
  const void* base;
  uint64_t rows, cols;
  uint32_t box_cols, box_rows;
  int dt;
  uint64_t depth;  // 3-D maps: the outer extent (experts); 0 for 2-D maps
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && box_cols == o.box_cols &&
           box_rows == o.box_rows && dt == o.dt && depth == o.depth;
  }
};
struct MapCacheEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapCacheSlots = 64;
static thread_local MapCacheEntry t_maps[kMapCacheSlots];

// 2-D row-major tensor [rows, cols] with a {box_cols, box_rows} box and the
// 128-byte swizzle; out-of-range elements read as zero.
static int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int esz, uint64_t rows,
                       uint64_t cols, uint32_t box_cols, uint32_t box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(MOE_ERR_MISALIGNED, "operand base %p is not 16-byte aligned", base);
  const MapKey key{base, rows, cols, box_cols, box_rows, (int)dt, 0};
  const uint64_t h = (reinterpret_cast<uintptr_t>(base) >> 8) * 0x9E3779B97F4A7C15ull ^ rows * 0xC2B2AE3D27D4EB4Full ^
                     cols * 0x165667B19E3779F9ull ^ ((uint64_t)box_cols << 20 | (uint64_t)box_rows << 8 | (uint64_t)dt);
  MapCacheEntry& slot = t_maps[(h >> 40) % kMapCacheSlots];
  if (slot.valid && slot.key == key) {
    *map = slot.map;
    return 0;
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)esz};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu box=%ux%u", (int)r,
                (unsigned long long)rows, (unsigned long long)cols, box_cols, box_rows);
  slot.key = key;
  slot.map = *map;
  slot.valid = true;
  return 0;
}

// 3-D row-major tensor [depth][rows][cols] (per-expert weights) with a
// {box_cols, box_rows, 1} box and the 128-byte swizzle; a box never crosses
// from one expert into the next, and out-of-range elements read as zero.
static int make_map_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int esz, uint64_t depth,
                       uint64_t rows, uint64_t cols, uint32_t box_cols, uint32_t box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(MOE_ERR_MISALIGNED, "operand base %p is not 16-byte aligned", base);
  if ((cols * (uint64_t)esz) % 16 != 0)
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "row of %llu elements x %d bytes is not a multiple of 16 bytes",
                (unsigned long long)cols, esz);
  const MapKey key{base, rows, cols, box_cols, box_rows, (int)dt, depth};
  const uint64_t h = (reinterpret_cast<uintptr_t>(base) >> 8) * 0x9E3779B97F4A7C15ull ^ rows * 0xC2B2AE3D27D4EB4Full ^
                     cols * 0x165667B19E3779F9ull ^ depth * 0xD6E8FEB86659FD93ull ^
                     ((uint64_t)box_cols << 20 | (uint64_t)box_rows << 8 | (uint64_t)dt);
  MapCacheEntry& slot = t_maps[(h >> 40) % kMapCacheSlots];
  if (slot.valid && slot.key == key) {
    *map = slot.map;
    return 0;
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {cols, rows, depth};
  cuuint64_t strides[2] = {cols * (uint64_t)esz, rows * cols * (uint64_t)esz};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d) depth=%llu rows=%llu cols=%llu box=%ux%u",
                (int)r, (unsigned long long)depth, (unsigned long long)rows, (unsigned long long)cols, box_cols,
                box_rows);
  slot.key = key;
  slot.map = *map;
  slot.valid = true;
  return 0;
}

// ------------------------------------------------------------------ device info
struct DevInfo {
  CUcontext ctx = nullptr;  // context the entries below belong to
  int sms = 0;
  int* status = nullptr;  // device address of g_status on this device
  bool attr_set[46] = {};
  int pairs[30] = {};  // co-resident CTA pairs per pair-kernel variant (0 = not queried)
};
static DevInfo g_dev[64];
static std::mutex g_dev_mu;

static int device_info(int* dev_out, DevInfo** info) {
  int dev = 0;
  MOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MOE_ERR_CUDA, "device ordinal %d out of range", dev);
  // cudaGetDevice above made the device's primary context current (or kept
  // the caller's), so the context read here is the one kernels launch in.
  const CUcontext ctx = current_ctx();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_dev[dev].sms == 0 || g_dev[dev].ctx != ctx) {
    g_dev[dev] = DevInfo();
    int sms = 0;
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    int major = 0, minor = 0;
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0)
      return fail(MOE_ERR_CUDA, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major,
                  minor);
    int* status = nullptr;
    MOE_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_status));
    g_dev[dev].status = status;
    g_dev[dev].sms = sms;
    g_dev[dev].ctx = ctx;
  }
  *dev_out = dev;
  *info = &g_dev[dev];
  return 0;
}

// The tf32 split reads raw f32 weights in 16-byte vectors.
static int check_weights_aligned(const void* w_up, const void* w_down) {
  if ((reinterpret_cast<uintptr_t>(w_up) | reinterpret_cast<uintptr_t>(w_down)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "f32 weights must be 16-byte aligned");
  return 0;
}

// ------------------------------------------------------------------ operand pre-split (3xTF32)
// W (E, R, C) f32 -> hi/lo planes of W^T (E, C, R): hi = W rounded to the
// nearest tf32 value (tf32_hi_bits), lo = W - hi.  One 32x32 tile (rows r0..,
// columns c0.. of expert e) per 256 threads through a padded shared tile, in
// 16-byte vectors both ways: thread t loads row t / 8, columns 4 (t % 8) ..
// +3, and stores column t / 8, rows 4 (t % 8) .. +3 of both planes.  R and C
// are multiples of 4 and W and the planes 16-byte aligned (the callers check).
// The transposed read of the tile is conflict-free: rows 4 (t % 8) + j and
// column t / 8 fall in 32 distinct banks with the 33-float row pitch.
__device__ __forceinline__ void split_transpose_tile(const float* __restrict__ w, float* __restrict__ hi,
                                                     float* __restrict__ lo, int R, int C, int e, int c0, int r0,
                                                     int tx, int ty, float (*tile)[33]) {
  const int t = ty * 32 + tx;
  const float* src = w + (size_t)e * R * C;
  {
    const int i = t >> 3, c4 = (t & 7) * 4;
    const int r = r0 + i, c = c0 + c4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < R && c < C) v = __ldg(reinterpret_cast<const float4*>(src + (size_t)r * C + c));
    tile[i][c4] = v.x;
    tile[i][c4 + 1] = v.y;
    tile[i][c4 + 2] = v.z;
    tile[i][c4 + 3] = v.w;
  }
  __syncthreads();
  const int cc = t >> 3, r4 = (t & 7) * 4;
  const int c = c0 + cc, r = r0 + r4;
  if (r < R && c < C) {
    float v[4], h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = tile[r4 + j][cc];
      h[j] = __uint_as_float(tf32_hi_bits(__float_as_uint(v[j])));
    }
    const size_t o = (size_t)e * R * C + (size_t)c * R + r;
    *reinterpret_cast<float4*>(hi + o) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + o) = make_float4(v[0] - h[0], v[1] - h[1], v[2] - h[2], v[3] - h[3]);
  }
}

__global__ void __launch_bounds__(256) split_transpose_kernel(const float* __restrict__ w, float* __restrict__ hi,
                                                              float* __restrict__ lo, int R, int C) {
  __shared__ float tile[32][33];
  split_transpose_tile(w, hi, lo, R, C, blockIdx.z, blockIdx.x * 32, blockIdx.y * 32, threadIdx.x, threadIdx.y,
                       tile);
}

__device__ __forceinline__ float4 tf32_hi4(float4 v) {
  return make_float4(__uint_as_float(tf32_hi_bits(__float_as_uint(v.x))),
                     __uint_as_float(tf32_hi_bits(__float_as_uint(v.y))),
                     __uint_as_float(tf32_hi_bits(__float_as_uint(v.z))),
                     __uint_as_float(tf32_hi_bits(__float_as_uint(v.w))));
}

// Everything a small-D call does before the fused kernel, in one launch:
// blocks [0, 2 w_blocks) split W_up and W_down into their tf32 planes (one
// 32x32 tile each), the next x_blocks split X, the last y_blocks zero Y (for
// the F-split grid, whose CTAs add into Y).  Unused segments have 0 blocks.
struct PrepArgs {
  const float* wu;
  float *wu_hi, *wu_lo;  // W_up (E, D, F) -> planes (E, F, D)
  const float* wd;
  float *wd_hi, *wd_lo;  // W_down (E, F, D) -> planes (E, D, F)
  int D, F, E;
  int w_blocks;          // tiles per weight matrix
  const int32_t* w_gs;   // group sizes: experts with no rows keep unsplit planes (no kernel reads them); null = all
  const float4* x;
  float4 *x_hi, *x_lo;
  size_t x_n4;
  int x_blocks;
  float4* y;
  size_t y_n4;
  int y_blocks;
  // Zero only the rows of the fused kernel's half units (one F-split): the
  // launch's unit plan is recomputed here from the group sizes.
  const int32_t* gs;
  int y_tail, M, nch, grid;
};

__global__ void __launch_bounds__(256) small_prep_kernel(const PrepArgs a) {
  __shared__ float tile[32][33];
  int b = (int)blockIdx.x;
  const int t = (int)threadIdx.x;
  if (b < 2 * a.w_blocks) {
    const bool down = b >= a.w_blocks;
    if (down) b -= a.w_blocks;
    const int R = down ? a.F : a.D, C = down ? a.D : a.F;
    const int tc = (C + 31) / 32, tr = (R + 31) / 32;
    const int e = b / (tr * tc), rem = b % (tr * tc);
    if (a.w_gs && __ldg(a.w_gs + e) <= 0) return;
    split_transpose_tile(down ? a.wd : a.wu, down ? a.wd_hi : a.wu_hi, down ? a.wd_lo : a.wu_lo, R, C, e,
                         (rem % tc) * 32, (rem / tc) * 32, t & 31, t >> 5, tile);
    return;
  }
  b -= 2 * a.w_blocks;
  if (b < a.x_blocks) {
    for (size_t i = (size_t)b * 256 + t; i < a.x_n4; i += (size_t)a.x_blocks * 256) {
      const float4 v = a.x[i];
      const float4 h = tf32_hi4(v);
      a.x_hi[i] = h;
      a.x_lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    }
    return;
  }
  b -= a.x_blocks;
  size_t n0 = 0, n1 = a.y_n4;
  if (a.y_tail) {
    // One thread computes the plan's row range for the block (the branch is
    // block-uniform, so the barrier is reached by every thread).
    __shared__ unsigned long long range[2];
    if (t == 0) {
      const SmallUnits su = small_units(a.gs, a.E, a.M, 1, a.nch, a.grid, 1);
      range[0] = su.halves == 1 ? 0 : (size_t)small_block_row(a.gs, a.E, a.M, su.full) * (size_t)a.D / 4;
      range[1] = su.halves == 1 ? 0 : (size_t)small_block_row(a.gs, a.E, a.M, 1 << 30) * (size_t)a.D / 4;
    }
    __syncthreads();
    n0 = range[0];
    n1 = range[1];
  }
  for (size_t i = n0 + (size_t)b * 256 + t; i < n1; i += (size_t)a.y_blocks * 256)
    a.y[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// ------------------------------------------------------------------ large-D dispatch (two grouped GEMMs)
// Any D and F whose rows start on 16-byte boundaries in every operand (the
// TMA rule): the grouped GEMMs mask partial column tiles and read zeros past
// K.  Shapes the fused small-D kernel covers are routed there first.
static bool large_supported(int D, int F, int dtype) {
  if (dtype == MOE_DTYPE_BF16) return D % 8 == 0 && F % 8 == 0;
  if (dtype == MOE_DTYPE_FP8_E4M3_BLK128) return D % 16 == 0 && F % 16 == 0;
  if (dtype == MOE_DTYPE_F32) return D % 4 == 0 && F % 4 == 0;
  return false;
}
static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Large-D workspace.  bf16: H (M, F) bf16; e4m3 weights: H (M, F) f16.  f32 (3xTF32):
// the tf32 hi/lo planes of W_up^T (E, F, D) and
// W_down^T (E, D, F) -- the layout moe_prepare_weights writes -- then X hi/lo
// (M, D) and H hi/lo (M, F), all f32.
struct Tf32LargeLayout {
  size_t wu_hi, wu_lo, wd_hi, wd_lo, x_hi, x_lo, h_hi, h_lo, total;  // byte offsets
};
static Tf32LargeLayout tf32_large_layout(int64_t M, int D, int F, int E) {
  Tf32LargeLayout l{};
  const size_t w = (size_t)E * D * F * sizeof(float);
  size_t o = 0;
  l.wu_hi = o;  // the first four match the small-D path's (and moe_prepare_weights') planes
  l.wu_lo = o += w;
  l.wd_hi = o += w;
  l.wd_lo = o += w;
  o = align256(o + w);
  l.x_hi = o;
  l.x_lo = o = align256(o + (size_t)M * D * sizeof(float));
  l.h_hi = o = align256(o + (size_t)M * D * sizeof(float));
  l.h_lo = o = align256(o + (size_t)M * F * sizeof(float));
  l.total = align256(o + (size_t)M * F * sizeof(float));
  return l;
}
static size_t large_ws_bytes(int64_t M, int D, int F, int E, int dtype) {
  if (dtype == MOE_DTYPE_F32) return tf32_large_layout(M, D, F, E).total;
  return align256((size_t)M * F * 2);  // H (bf16; f16 with e4m3 weights)
}

template <int EPI, bool BFP8, bool TF32 = false, int WIDE = 1>
static int launch_gemm(const GemmMaps& maps, const GemmParams& prm_in, DevInfo* di, cudaStream_t st, int ctas_req) {
  GemmParams prm = prm_in;
  if (g_tune_group_m > 0) prm.group_m = (int)g_tune_group_m;
  prm.l2_mode = (int)g_tune_l2;
  using Cfg = GemmCfg<EPI, BFP8, TF32, WIDE>;
  auto kern = grouped_gemm_pair_kernel<EPI, BFP8, TF32, WIDE>;
  constexpr int slot = WIDE == 2 ? 44 : (TF32 ? 40 + EPI : 24 + 2 * EPI + (BFP8 ? 1 : 0));
  constexpr int pslot = WIDE == 2 ? 28 : (TF32 ? 24 + EPI : 8 + 2 * EPI + (BFP8 ? 1 : 0));
  static_assert(slot < 46 && pslot < 30 && (TF32 ? EPI < 2 : true), "attribute slot");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!di->attr_set[slot]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    cfg.gridDim = dim3(2 * (di->sms / 2));
    int clusters = 0;
    MOE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
    if (clusters < 1) return fail(MOE_ERR_CUDA, "no CTA pair fits on this device");
    di->pairs[pslot] = clusters;
    di->attr_set[slot] = true;
  }
  int pairs = di->pairs[pslot];
  if (ctas_req > 0 && ctas_req / 2 < pairs) pairs = ctas_req / 2 > 0 ? ctas_req / 2 : 1;
  cfg.gridDim = dim3(2 * pairs);
  MOE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, maps, prm));
  return 0;
}

template <int EPI>
static int launch_swap(const SwapMaps& maps, const GemmParams& prm, DevInfo* di, cudaStream_t st, int ctas_req) {
  using Cfg = SwapCfg<EPI>;
  auto kern = grouped_gemm_swap_kernel<EPI>;
  constexpr int slot = 42 + EPI;
  constexpr int pslot = 26 + EPI;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!di->attr_set[slot]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    cfg.gridDim = dim3(2 * (di->sms / 2));
    int clusters = 0;
    MOE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
    if (clusters < 1) return fail(MOE_ERR_CUDA, "no CTA pair fits on this device");
    di->pairs[pslot] = clusters;
    di->attr_set[slot] = true;
  }
  int pairs = di->pairs[pslot];
  if (ctas_req > 0 && ctas_req / 2 < pairs) pairs = ctas_req / 2 > 0 ? ctas_req / 2 : 1;
  cfg.gridDim = dim3(2 * pairs);
  MOE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, maps, prm));
  return 0;
}

// Launch options shared by the single-GPU entry points (defaults) and the
// expert-parallel engine: `ctas` > 0 caps the persistent grid (leaving SMs to
// concurrent exchange kernels), `skip_tail` leaves Y rows past
// sum(group_sizes) unwritten (a landing region whose tail nobody reads).
struct RunOpts {
  int ctas = 0;
  bool skip_tail = false;
  const EpScatter* scatter = nullptr;  // large-D path: rows of Y go to their source ranks
  const EpDispatch* dispatch = nullptr;  // large-D bf16 path: the token dispatch runs inside the up GEMM
};

// f32 inputs with D outside the fused small-D kernels: the two grouped GEMMs
// in 3xTF32.  One preparation launch splits X (and, unless the weights were
// prepared, W_up and W_down, transposed) into tf32 hi/lo planes; the up GEMM
// writes H as hi/lo planes; the down GEMM writes Y.
static int run_large_tf32(const float* x, const float* w_up, const float* w_down, const int32_t* gs, float* y,
                          int64_t M, int D, int F, int E, void* ws, size_t ws_bytes, cudaStream_t st, RunOpts opt,
                          bool split_weights, DevInfo* di) {
  const Tf32LargeLayout L = tf32_large_layout(M, D, F, E);
  if (ws_bytes < L.total) return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, L.total);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  if (reinterpret_cast<uintptr_t>(x) & 15u) return fail(MOE_ERR_MISALIGNED, "x must be 16-byte aligned");
  if (split_weights)
    if (int r = check_weights_aligned(w_up, w_down)) return r;
  uint8_t* b = static_cast<uint8_t*>(ws);
  float* wu_hi = reinterpret_cast<float*>(b + L.wu_hi);
  float* wu_lo = reinterpret_cast<float*>(b + L.wu_lo);
  float* wd_hi = reinterpret_cast<float*>(b + L.wd_hi);
  float* wd_lo = reinterpret_cast<float*>(b + L.wd_lo);
  float* x_hi = reinterpret_cast<float*>(b + L.x_hi);
  float* x_lo = reinterpret_cast<float*>(b + L.x_lo);
  float* h_hi = reinterpret_cast<float*>(b + L.h_hi);
  float* h_lo = reinterpret_cast<float*>(b + L.h_lo);
  const int ctas = opt.ctas > 0 ? opt.ctas : (int)g_tune_ctas;
  {
    PrepArgs pa{};
    const int cap = di->sms * 4;
    if (split_weights) {
      pa.wu = w_up;
      pa.wd = w_down;
      pa.wu_hi = wu_hi;
      pa.wu_lo = wu_lo;
      pa.wd_hi = wd_hi;
      pa.wd_lo = wd_lo;
      pa.D = D;
      pa.F = F;
      pa.E = E;
      pa.w_blocks = E * ((D + 31) / 32) * ((F + 31) / 32);
      pa.w_gs = gs;
    }
    pa.x = reinterpret_cast<const float4*>(x);
    pa.x_hi = reinterpret_cast<float4*>(x_hi);
    pa.x_lo = reinterpret_cast<float4*>(x_lo);
    pa.x_n4 = (size_t)M * D / 4;
    pa.x_blocks = (int)std::min<size_t>((pa.x_n4 + 255) / 256, (size_t)cap);
    small_prep_kernel<<<2 * pa.w_blocks + pa.x_blocks, 256, 0, st>>>(pa);
    MOE_CUDA_TRY(cudaGetLastError());
  }
  const auto F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  // up: H = GELU(X @ W_up[e]); B = W_up^T planes [E][F][D] (K-major)
  GemmMaps m1;
  memset(&m1, 0, sizeof(m1));
  if (int r = make_map_2d(&m1.a, x_hi, F32, 4, (uint64_t)M, D, 32, 128)) return r;
  if (int r = make_map_2d(&m1.a_lo, x_lo, F32, 4, (uint64_t)M, D, 32, 128)) return r;
  if (int r = make_map_3d(&m1.b, wu_hi, F32, 4, (uint64_t)E, F, D, 32, 128)) return r;
  if (int r = make_map_3d(&m1.b_lo, wu_lo, F32, 4, (uint64_t)E, F, D, 32, 128)) return r;
  GemmParams p1{gs, h_hi, (int)M, E, F, D, 8, di->status, nullptr, 0};
  p1.out2 = h_lo;
  if (int r = launch_gemm<0, false, true>(m1, p1, di, st, ctas)) return r;
  // down: Y = H @ W_down[e]; B = W_down^T planes [E][D][F]
  GemmMaps m2;
  memset(&m2, 0, sizeof(m2));
  if (int r = make_map_2d(&m2.a, h_hi, F32, 4, (uint64_t)M, F, 32, 128)) return r;
  if (int r = make_map_2d(&m2.a_lo, h_lo, F32, 4, (uint64_t)M, F, 32, 128)) return r;
  if (int r = make_map_3d(&m2.b, wd_hi, F32, 4, (uint64_t)E, D, F, 32, 128)) return r;
  if (int r = make_map_3d(&m2.b_lo, wd_lo, F32, 4, (uint64_t)E, D, F, 32, 128)) return r;
  GemmParams p2{gs, y, (int)M, E, D, F, 8, di->status, nullptr, opt.skip_tail ? 1 : 0};
  if (opt.scatter) p2.scatter = *opt.scatter;
  return launch_gemm<1, false, true>(m2, p2, di, st, ctas);
}

static int run_large(const void* x, const void* w_up, const void* w_down, const int32_t* gs,
                     const float* w_up_scale, const float* w_down_scale, float* y, int64_t M, int D, int F, int E,
                     int dtype, void* ws, size_t ws_bytes, cudaStream_t st, RunOpts opt = RunOpts(),
                     bool split_weights = true) {
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  if (dtype == MOE_DTYPE_F32)
    return run_large_tf32(static_cast<const float*>(x), static_cast<const float*>(w_up),
                          static_cast<const float*>(w_down), gs, y, M, D, F, E, ws, ws_bytes, st, opt, split_weights,
                          di);
  const int ctas = opt.ctas > 0 ? opt.ctas : (int)g_tune_ctas;
  const size_t need = large_ws_bytes(M, D, F, E, dtype);
  if (ws_bytes < need) return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, need);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  const bool fp8 = dtype == MOE_DTYPE_FP8_E4M3_BLK128;
  if (fp8 && (!w_up_scale || !w_down_scale))
    return fail(MOE_ERR_INVALID_ARG, "FP8 weights need w_up_scale and w_down_scale");
  int* status = di->status;
  const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  // e4m3 weights: the up GEMM runs on bf16 operands (X as given, weights
  // decoded to bf16 in shared memory) and stores H in f16, the down GEMM's
  // 16-bit type (weights decoded to f16).
  const auto A16 = BF16;
  const auto H16 = fp8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : BF16;
  const void* xa = x;
  // Small experts with e4m3 weights: expert super-tiles (grouped_gemm_swap.cuh),
  // unless the down GEMM must store Y rows into their source ranks.
  const bool swap = fp8 && !opt.scatter && fp8_use_swap(M, E);
  if (swap) {
    // Token rows in 32-, 64- and 128-row boxes; e4m3 weights {128, 64, 1}.
    auto swap_maps = [&](SwapMaps* m, const void* rows, CUtensorMapDataType rt, int K, const void* w,
                         int N) -> int {
      memset(m, 0, sizeof(*m));
      if (int r = make_map_2d(&m->x32, rows, rt, 2, (uint64_t)M, K, 64, 32)) return r;
      if (int r = make_map_2d(&m->x64, rows, rt, 2, (uint64_t)M, K, 64, 64)) return r;
      if (int r = make_map_2d(&m->x128, rows, rt, 2, (uint64_t)M, K, 64, 128)) return r;
      return make_map_3d(&m->w, w, U8, 1, (uint64_t)E, K, N, 128, 64);
    };
    SwapMaps s1, s2;
    if (int r = swap_maps(&s1, xa, BF16, D, w_up, F)) return r;
    GemmParams p1{gs, ws, (int)M, E, F, D, 8, status, w_up_scale, 0};
    if (int r = launch_swap<0>(s1, p1, di, st, ctas)) return r;
    if (int r = swap_maps(&s2, ws, H16, F, w_down, D)) return r;
    GemmParams p2{gs, y, (int)M, E, D, F, 8, status, w_down_scale, opt.skip_tail ? 1 : 0};
    return launch_swap<1>(s2, p2, di, st, ctas);
  }
  // up: H = GELU(X @ W_up[e])
  GemmMaps m1;
  memset(&m1, 0, sizeof(m1));
  if (int r = make_map_2d(&m1.a, xa, A16, 2, (uint64_t)M, D, 64, 128)) return r;
  if (fp8) {
    if (int r = make_map_3d(&m1.b, w_up, U8, 1, (uint64_t)E, D, F, 128, 64)) return r;
  } else {
    if (int r = make_map_3d(&m1.b, w_up, BF16, 2, (uint64_t)E, D, F, 64, 64)) return r;
  }
  GemmParams p1{gs, ws, (int)M, E, F, D, 8, status, w_up_scale, 0};
  if (opt.dispatch && !fp8) p1.dispatch = *opt.dispatch;  // (f32 took run_large_tf32 above)
  if (int r = fp8 ? launch_gemm<0, true>(m1, p1, di, st, ctas) : launch_gemm<0, false>(m1, p1, di, st, ctas))
    return r;
  // down: Y = H @ W_down[e]
  GemmMaps m2;
  memset(&m2, 0, sizeof(m2));
  if (int r = make_map_2d(&m2.a, ws, H16, 2, (uint64_t)M, F, 64, 128)) return r;
  if (fp8) {
    if (int r = make_map_3d(&m2.b, w_down, U8, 1, (uint64_t)E, F, D, 128, 64)) return r;
  } else {
    if (int r = make_map_3d(&m2.b, w_down, BF16, 2, (uint64_t)E, F, D, 64, 64)) return r;
  }
  GemmParams p2{gs, y, (int)M, E, D, F, 8, status, w_down_scale, opt.skip_tail ? 1 : 0};
  if (opt.scatter) p2.scatter = *opt.scatter;
  if (fp8) return launch_gemm<1, true>(m2, p2, di, st, ctas);
  return down_wide() ? launch_gemm<1, false, false, 2>(m2, p2, di, st, ctas)
                     : launch_gemm<1, false, false>(m2, p2, di, st, ctas);
}

// ------------------------------------------------------------------ training: forward with saved pre-activation, backward
template <int MODE>
static int launch_bwd(const GemmMaps& maps, const BwdParams& prm, DevInfo* di, cudaStream_t st, int ctas_req) {
  using Cfg = BwdCfg<MODE>;
  auto kern = grouped_bwd_pair_kernel<MODE>;
  constexpr int slot = 36 + MODE;
  constexpr int pslot = 18 + MODE;
  static_assert(slot < 40 && pslot < 24, "attribute slot");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!di->attr_set[slot]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    cfg.gridDim = dim3(2 * (di->sms / 2));
    int clusters = 0;
    MOE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
    if (clusters < 1) return fail(MOE_ERR_CUDA, "no CTA pair fits on this device");
    di->pairs[pslot] = clusters;
    di->attr_set[slot] = true;
  }
  int pairs = di->pairs[pslot];
  if (ctas_req > 0 && ctas_req / 2 < pairs) pairs = ctas_req / 2 > 0 ? ctas_req / 2 : 1;
  cfg.gridDim = dim3(2 * pairs);
  MOE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, maps, prm));
  return 0;
}

static bool train_supported(int D, int F) { return D >= 256 && D % 256 == 0 && F >= 256 && F % 256 == 0; }

// Padded rows of the backward's row-layout buffers: every expert's rows
// rounded up to 64, at most 63 extra rows per expert.
static int64_t bwd_padded_rows(int64_t M, int E) { return M + 64 * (int64_t)E; }

static size_t bwd_ws_bytes(int64_t M, int D, int F, int E) {
  const int64_t mp = bwd_padded_rows(M, E);
  return 2 * align256((size_t)mp * D * 2) + 2 * align256((size_t)mp * F * 2);
}

// Forward of the bf16 expert MLP on the grouped GEMMs, saving A = X W_up.
static int run_train_forward(const void* x, const void* w_up, const void* w_down, const int32_t* gs, float* y,
                             void* a_save, int64_t M, int D, int F, int E, void* ws, size_t ws_bytes,
                             cudaStream_t st) {
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const size_t need = large_ws_bytes(M, D, F, E, MOE_DTYPE_BF16);
  if (ws_bytes < need) return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, need);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int* status = di->status;
  const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int ctas = (int)g_tune_ctas;
  GemmMaps m1;
  memset(&m1, 0, sizeof(m1));
  if (int r = make_map_2d(&m1.a, x, BF16, 2, (uint64_t)M, D, 64, 128)) return r;
  if (int r = make_map_3d(&m1.b, w_up, BF16, 2, (uint64_t)E, D, F, 64, 64)) return r;
  GemmParams p1{gs, ws, (int)M, E, F, D, 8, status, nullptr, 0};
  p1.out2 = a_save;
  if (int r = launch_gemm<3, false>(m1, p1, di, st, ctas)) return r;
  GemmMaps m2;
  memset(&m2, 0, sizeof(m2));
  if (int r = make_map_2d(&m2.a, ws, BF16, 2, (uint64_t)M, F, 64, 128)) return r;
  if (int r = make_map_3d(&m2.b, w_down, BF16, 2, (uint64_t)E, F, D, 64, 64)) return r;
  GemmParams p2{gs, y, (int)M, E, D, F, 8, status, nullptr, 0};
  return launch_gemm<1, false>(m2, p2, di, st, ctas);
}

static int run_backward(const void* x, const void* w_up, const void* w_down, const int32_t* gs, const void* a_saved,
                        const void* dy, int dy_dtype, float* dx, float* dw_up, float* dw_down, int64_t M, int D,
                        int F, int E, void* ws, size_t ws_bytes, cudaStream_t st) {
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const size_t need = bwd_ws_bytes(M, D, F, E);
  if (ws_bytes < need) return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, need);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int* status = di->status;
  const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int ctas = (int)g_tune_ctas;
  const int64_t mp = bwd_padded_rows(M, E);
  uint8_t* w = static_cast<uint8_t*>(ws);
  uint16_t* x_pad = reinterpret_cast<uint16_t*>(w);
  uint16_t* dy_pad = reinterpret_cast<uint16_t*>(w + align256((size_t)mp * D * 2));
  uint16_t* da_pad = reinterpret_cast<uint16_t*>(w + 2 * align256((size_t)mp * D * 2));
  uint16_t* h_pad = reinterpret_cast<uint16_t*>(w + 2 * align256((size_t)mp * D * 2) + align256((size_t)mp * F * 2));
  // 1. X and dY in the padded row layout.
  {
    const int blocks = (int)std::min<int64_t>((mp + 7) / 8, (int64_t)di->sms * 8);
    bwd_pad_rows_kernel<<<blocks, 256, 8 * (E + 1), st>>>(static_cast<const uint16_t*>(x), dy,
                                                           dy_dtype == MOE_DTYPE_F32 ? 1 : 0, gs, E, (int)M, D,
                                                           x_pad, dy_pad);
    MOE_CUDA_TRY(cudaGetLastError());
  }
  GemmMaps m;
  // 2. dH = dY W_down^T -> dA = dH GELU'(A), H = GELU(A) (padded rows).
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, dy_pad, BF16, 2, (uint64_t)mp, D, 64, 128)) return r;
  if (int r = make_map_2d(&m.b, w_down, BF16, 2, (uint64_t)E * F, D, 64, 128)) return r;
  BwdParams p{gs, (int)M, E, F, D, 0, 8, status, static_cast<const uint16_t*>(a_saved), da_pad, h_pad};
  if (int r = launch_bwd<kBwdDH>(m, p, di, st, ctas)) return r;
  // 3. dX = dA W_up^T (natural rows).
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, da_pad, BF16, 2, (uint64_t)mp, F, 64, 128)) return r;
  if (int r = make_map_2d(&m.b, w_up, BF16, 2, (uint64_t)E * D, F, 64, 128)) return r;
  p = BwdParams{gs, (int)M, E, D, F, 0, 8, status, nullptr, dx, nullptr};
  if (int r = launch_bwd<kBwdDX>(m, p, di, st, ctas)) return r;
  // 4. dW_up[e] = X_e^T dA_e  (E, D, F).
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, x_pad, BF16, 2, (uint64_t)mp, D, 64, 64)) return r;
  if (int r = make_map_2d(&m.b, da_pad, BF16, 2, (uint64_t)mp, F, 64, 64)) return r;
  p = BwdParams{gs, (int)M, E, F, 0, D, 8, status, nullptr, dw_up, nullptr};
  if (int r = launch_bwd<kBwdDW>(m, p, di, st, ctas)) return r;
  // 5. dW_down[e] = H_e^T dY_e  (E, F, D).
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, h_pad, BF16, 2, (uint64_t)mp, F, 64, 64)) return r;
  if (int r = make_map_2d(&m.b, dy_pad, BF16, 2, (uint64_t)mp, D, 64, 64)) return r;
  p = BwdParams{gs, (int)M, E, D, 0, F, 8, status, nullptr, dw_down, nullptr};
  return launch_bwd<kBwdDW>(m, p, di, st, ctas);
}

// SwiGLU training: forward saving the raw gate/up columns, and its backward.
static size_t swiglu_bwd_ws_bytes(int64_t M, int D, int F, int E) {
  const int64_t mp = bwd_padded_rows(M, E);
  return 2 * align256((size_t)mp * D * 2) + align256((size_t)mp * 2 * F * 2) + align256((size_t)mp * F * 2);
}

static int run_swiglu_train_forward(const void* x, const void* w_gu, const void* w_down, const int32_t* gs, float* y,
                                    void* gu_save, int64_t M, int D, int F, int E, void* ws, size_t ws_bytes,
                                    cudaStream_t st) {
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const size_t need = align256((size_t)M * F * 2);
  if (ws_bytes < need) return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, need);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int* status = di->status;
  const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int ctas = (int)g_tune_ctas;
  GemmMaps m1;
  memset(&m1, 0, sizeof(m1));
  if (int r = make_map_2d(&m1.a, x, BF16, 2, (uint64_t)M, D, 64, 128)) return r;
  if (int r = make_map_3d(&m1.b, w_gu, BF16, 2, (uint64_t)E, D, 2 * F, 64, 64)) return r;
  GemmParams p1{gs, ws, (int)M, E, 2 * F, D, 8, status, nullptr, 0};
  p1.out2 = gu_save;
  if (int r = launch_gemm<4, false>(m1, p1, di, st, ctas)) return r;
  GemmMaps m2;
  memset(&m2, 0, sizeof(m2));
  if (int r = make_map_2d(&m2.a, ws, BF16, 2, (uint64_t)M, F, 64, 128)) return r;
  if (int r = make_map_3d(&m2.b, w_down, BF16, 2, (uint64_t)E, F, D, 64, 64)) return r;
  GemmParams p2{gs, y, (int)M, E, D, F, 8, status, nullptr, 0};
  return launch_gemm<1, false>(m2, p2, di, st, ctas);
}

static int run_swiglu_backward(const void* x, const void* w_gu, const void* w_down, const int32_t* gs,
                               const void* gu_saved, const void* dy, int dy_dtype, float* dx, float* dw_gu,
                               float* dw_down, int64_t M, int D, int F, int E, void* ws, size_t ws_bytes,
                               cudaStream_t st) {
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const size_t need = swiglu_bwd_ws_bytes(M, D, F, E);
  if (ws_bytes < need) return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, need);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int* status = di->status;
  const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int ctas = (int)g_tune_ctas;
  const int64_t mp = bwd_padded_rows(M, E);
  const size_t sx = align256((size_t)mp * D * 2);
  uint8_t* w = static_cast<uint8_t*>(ws);
  uint16_t* x_pad = reinterpret_cast<uint16_t*>(w);
  uint16_t* dy_pad = reinterpret_cast<uint16_t*>(w + sx);
  uint16_t* dgu_pad = reinterpret_cast<uint16_t*>(w + 2 * sx);
  uint16_t* h_pad = reinterpret_cast<uint16_t*>(w + 2 * sx + align256((size_t)mp * 2 * F * 2));
  {
    const int blocks = (int)std::min<int64_t>((mp + 7) / 8, (int64_t)di->sms * 8);
    bwd_pad_rows_kernel<<<blocks, 256, 8 * (E + 1), st>>>(static_cast<const uint16_t*>(x), dy,
                                                           dy_dtype == MOE_DTYPE_F32 ? 1 : 0, gs, E, (int)M, D,
                                                           x_pad, dy_pad);
    MOE_CUDA_TRY(cudaGetLastError());
  }
  GemmMaps m;
  // dH = dY W_down^T -> dGate, dUp (interleaved like the weights), H (padded rows).
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, dy_pad, BF16, 2, (uint64_t)mp, D, 64, 128)) return r;
  if (int r = make_map_2d(&m.b, w_down, BF16, 2, (uint64_t)E * F, D, 64, 128)) return r;
  BwdParams p{gs, (int)M, E, F, D, 0, 8, status, static_cast<const uint16_t*>(gu_saved), dgu_pad, h_pad};
  if (int r = launch_bwd<kBwdDHSwiGLU>(m, p, di, st, ctas)) return r;
  // dX = [dGate | dUp] W_gate_up^T (K = 2F).
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, dgu_pad, BF16, 2, (uint64_t)mp, 2 * F, 64, 128)) return r;
  if (int r = make_map_2d(&m.b, w_gu, BF16, 2, (uint64_t)E * D, 2 * F, 64, 128)) return r;
  p = BwdParams{gs, (int)M, E, D, 2 * F, 0, 8, status, nullptr, dx, nullptr};
  if (int r = launch_bwd<kBwdDX>(m, p, di, st, ctas)) return r;
  // dW_gate_up[e] = X_e^T [dGate | dUp]_e  (E, D, 2F), interleaved like the weights.
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, x_pad, BF16, 2, (uint64_t)mp, D, 64, 64)) return r;
  if (int r = make_map_2d(&m.b, dgu_pad, BF16, 2, (uint64_t)mp, 2 * F, 64, 64)) return r;
  p = BwdParams{gs, (int)M, E, 2 * F, 0, D, 8, status, nullptr, dw_gu, nullptr};
  if (int r = launch_bwd<kBwdDW>(m, p, di, st, ctas)) return r;
  // dW_down[e] = H_e^T dY_e  (E, F, D).
  memset(&m, 0, sizeof(m));
  if (int r = make_map_2d(&m.a, h_pad, BF16, 2, (uint64_t)mp, F, 64, 64)) return r;
  if (int r = make_map_2d(&m.b, dy_pad, BF16, 2, (uint64_t)mp, D, 64, 64)) return r;
  p = BwdParams{gs, (int)M, E, D, 0, F, 8, status, nullptr, dw_down, nullptr};
  return launch_bwd<kBwdDW>(m, p, di, st, ctas);
}

// ------------------------------------------------------------------ SwiGLU experts
// (E, D, F) gate and up weights -> (E, D, 2F) with columns interleaved every
// 128: [gate 0..127 | up 0..127 | gate 128..255 | up 128..255 | ...], so that
// every 256-column tile of the up GEMM holds matching gate and up columns.
// One thread per 16-byte vector (8 bf16).
// `vin` vectors per input row, `vblk` vectors per 128-column block (16 for
// bf16, 8 for e4m3): output period = one gate block then one up block.
__global__ void swiglu_interleave_kernel(const uint4* __restrict__ gate, const uint4* __restrict__ up,
                                         uint4* __restrict__ out, size_t rows, int vin, int vblk) {
  const int vout = 2 * vin;
  const size_t n = rows * (size_t)vout;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / vout;
    const int v = (int)(i - r * vout);
    const int j = v / (2 * vblk), w = v % (2 * vblk);
    const uint4* src = w < vblk ? gate : up;
    out[i] = src[r * vin + (size_t)j * vblk + (w % vblk)];
  }
}

// 128 x 128 block scales of e4m3 gate and up weights, (rows, nb) each ->
// (rows, 2 nb): one gate block, then the up block of the same columns.
__global__ void swiglu_interleave_scales_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                                float* __restrict__ out, size_t rows, int nb) {
  const size_t n = rows * (size_t)(2 * nb);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / (2 * nb);
    const int c = (int)(i - r * (2 * nb));
    out[i] = ((c & 1) ? up : gate)[r * nb + (c >> 1)];
  }
}

static bool swiglu_supported(int D, int F) { return D >= 256 && D % 256 == 0 && F % 128 == 0; }

static size_t swiglu_ws_bytes(int64_t M, int D, int F, bool fp8) {
  (void)D;
  (void)fp8;
  return align256((size_t)M * F * 2);  // H (bf16; f16 with e4m3 weights)
}

// SwiGLU experts on the two grouped GEMMs.  e4m3 weights (fp8): block
// scales s_gu (E, D/128, 2F/128) interleaved like the weights and s_down
// (E, F/128, D/128); the up GEMM runs on bf16 operands, the down GEMM on f16 (H f16).
static int run_swiglu(const void* x, const void* w_gu, const void* w_down, const float* s_gu, const float* s_down,
                      const int32_t* gs, float* y, int64_t M, int D, int F, int E, bool fp8, void* ws,
                      size_t ws_bytes, cudaStream_t st) {
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const size_t need = swiglu_ws_bytes(M, D, F, fp8);
  if (ws_bytes < need) return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, need);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int* status = di->status;
  const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto A16 = BF16;  // e4m3 weights: bf16 up GEMM on X as given; f16 H for the down GEMM
  const auto H16 = fp8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : BF16;
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const int ctas = (int)g_tune_ctas;
  const void* xa = x;
  // up: H = SiLU(X @ W_gate[e]) * (X @ W_up[e]) over the interleaved (E*D, 2F) weights
  GemmMaps m1;
  memset(&m1, 0, sizeof(m1));
  if (int r = make_map_2d(&m1.a, xa, A16, 2, (uint64_t)M, D, 64, 128)) return r;
  if (fp8) {
    if (int r = make_map_3d(&m1.b, w_gu, U8, 1, (uint64_t)E, D, 2 * F, 128, 64)) return r;
  } else {
    if (int r = make_map_3d(&m1.b, w_gu, BF16, 2, (uint64_t)E, D, 2 * F, 64, 64)) return r;
  }
  GemmParams p1{gs, ws, (int)M, E, 2 * F, D, 8, status, s_gu, 0};
  if (int r = fp8 ? launch_gemm<2, true>(m1, p1, di, st, ctas) : launch_gemm<2, false>(m1, p1, di, st, ctas))
    return r;
  // down: Y = H @ W_down[e]
  GemmMaps m2;
  memset(&m2, 0, sizeof(m2));
  if (int r = make_map_2d(&m2.a, ws, H16, 2, (uint64_t)M, F, 64, 128)) return r;
  if (fp8) {
    if (int r = make_map_3d(&m2.b, w_down, U8, 1, (uint64_t)E, F, D, 128, 64)) return r;
  } else {
    if (int r = make_map_3d(&m2.b, w_down, BF16, 2, (uint64_t)E, F, D, 64, 64)) return r;
  }
  GemmParams p2{gs, y, (int)M, E, D, F, 8, status, s_down, 0};
  return fp8 ? launch_gemm<1, true>(m2, p2, di, st, ctas) : launch_gemm<1, false>(m2, p2, di, st, ctas);
}

// ------------------------------------------------------------------ small-D dispatch
struct SmallPlan {
  int bf;
  bool x_res;
  size_t ws_bytes;
};

static bool small_supported(int D, int F, int dtype) {
  if (!(D == 64 || D == 128 || D == 256)) return false;
  if (dtype == MOE_DTYPE_F32) return F % 64 == 0;
  if (dtype == MOE_DTYPE_BF16) return F % 128 == 0;
  return false;
}

static SmallPlan small_plan(int64_t M, int D, int F, int E, int dtype) {
  SmallPlan s{};
  if (dtype == MOE_DTYPE_F32) {
    s.bf = 64;
    s.x_res = D <= 128;
    const size_t w = (size_t)E * D * F * sizeof(float);
    s.ws_bytes = 4 * w + (s.x_res ? 0 : 2 * (size_t)M * D * sizeof(float));
  } else {
    s.bf = 128;
    s.x_res = true;
    s.ws_bytes = 0;
  }
  return s;
}


template <int MODE, int D, int BF, bool XR>
static int launch_small(const FusedMaps& maps, const FusedParams& prm, int ctas, DevInfo* di, cudaStream_t st) {
  using Cfg = FusedCfg<MODE, D, BF, XR>;
  auto kern = fused_mlp_small_kernel<MODE, D, BF, XR>;
  constexpr int slot = (MODE * 3 + (D == 64 ? 0 : D == 128 ? 1 : 2)) * 2 + (XR ? 1 : 0);
  static_assert(slot < 16, "attribute slot");
  if (!di->attr_set[slot]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    di->attr_set[slot] = true;
  }
  kern<<<ctas, Cfg::THREADS, Cfg::SMEM, st>>>(maps, prm);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

static int check_workspace(const SmallPlan& plan, const void* ws, size_t ws_bytes) {
  if (ws_bytes < plan.ws_bytes)
    return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, plan.ws_bytes);
  if (plan.ws_bytes && (reinterpret_cast<uintptr_t>(ws) & 255u))
    return fail(MOE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  return 0;
}

// Weight preparation: for the 3xTF32 paths (fused small-D and grouped
// large-D), split W_up / W_down into K-major tf32 hi/lo planes at the start
// of the workspace.  Nothing for bf16 or e4m3.
static int prepare_small(const void* w_up, const void* w_down, int D, int F, int E, int dtype, void* ws,
                         size_t ws_bytes, cudaStream_t st) {
  const SmallPlan plan = small_plan(0, D, F, E, dtype);
  if (dtype != MOE_DTYPE_F32) return 0;
  if (int r = check_workspace(plan, ws, ws_bytes)) return r;
  if (int r = check_weights_aligned(w_up, w_down)) return r;
  const size_t wsz = (size_t)E * D * F;
  float* wu_hi = static_cast<float*>(ws);
  float* wu_lo = wu_hi + wsz;
  float* wd_hi = wu_lo + wsz;
  float* wd_lo = wd_hi + wsz;
  dim3 blk(32, 8);
  dim3 g_up((F + 31) / 32, (D + 31) / 32, E);  // W_up (E, D, F) -> planes (E, F, D)
  split_transpose_kernel<<<g_up, blk, 0, st>>>(static_cast<const float*>(w_up), wu_hi, wu_lo, D, F);
  MOE_CUDA_TRY(cudaGetLastError());
  dim3 g_dn((D + 31) / 32, (F + 31) / 32, E);  // W_down (E, F, D) -> planes (E, D, F)
  split_transpose_kernel<<<g_dn, blk, 0, st>>>(static_cast<const float*>(w_down), wd_hi, wd_lo, F, D);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

// Main fused launch; for 3xTF32 the weight planes must already be in `ws`.
static bool pair_supported(int D, int dtype) {
  if (dtype == MOE_DTYPE_F32) return D == 64 || D == 128;
  if (dtype == MOE_DTYPE_BF16) return D == 128 || D == 256;
  return false;
}

template <int MODE, int D, int BF>
static int launch_pair(const FusedMaps& maps, const FusedParams& prm, int pairs_req, DevInfo* di, cudaStream_t st) {
  using Cfg = PairCfg<MODE, D, BF>;
  auto kern = fused_mlp_pair_kernel<MODE, D, BF>;
  constexpr int slot = 16 + MODE * 3 + (D == 64 ? 0 : D == 128 ? 1 : 2);
  constexpr int pslot = MODE * 3 + (D == 64 ? 0 : D == 128 ? 1 : 2);
  static_assert(slot < 32 && pslot < 8, "attribute slot");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!di->attr_set[slot]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    cfg.gridDim = dim3(2 * (di->sms / 2));
    int clusters = 0;
    MOE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
    if (clusters < 1) return fail(MOE_ERR_CUDA, "no CTA pair fits on this device");
    di->pairs[pslot] = clusters;
    di->attr_set[slot] = true;
  }
  int pairs = di->pairs[pslot];
  if (pairs_req > 0 && pairs_req < pairs) pairs = pairs_req;
  cfg.gridDim = dim3(2 * pairs);
  MOE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, maps, prm));
  return 0;
}

// F-splits of a small-D call: the tuning value if set, else the most splits
// that still fit the (expert, row-block) units in one wave of SMs (or SM
// pairs) -- a second wave of shorter units costs more than it balances
// (measured on B200 over M = 128 ... 131072, D = 64 ... 256, E = 4 ... 16,
// f32 and bf16).  Row blocks are estimated from M; at small M every expert is
// taken to hold a partial block of its own.
static int small_splits(int64_t M, int E, int nch_total, bool pair, int sms) {
  if (g_tune_splits > 0) return (int)g_tune_splits;
  const int rows_per_unit = pair ? 256 : 128;
  const int64_t workers = pair ? sms / 2 : sms;
  const int64_t blocks_est =
      std::max<int64_t>((M + rows_per_unit - 1) / rows_per_unit, std::min<int64_t>(E, (M + 15) / 16));
  int splits = 1;
  while (blocks_est * splits * 2 <= workers && nch_total % (splits * 2) == 0 && splits * 2 <= nch_total) splits *= 2;
  return splits;
}

// `split_weights`: the 3xTF32 weight planes are built by this call's
// preparation launch (raw f32 weights); otherwise they are already in `ws`.
static int run_small(const void* x, const void* w_up, const void* w_down, const int32_t* gs, float* y, int64_t M,
                     int D, int F, int E, int dtype, void* ws, size_t ws_bytes, cudaStream_t st,
                     RunOpts opt = RunOpts(), bool split_weights = false) {
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const SmallPlan plan = small_plan(M, D, F, E, dtype);
  if (int r = check_workspace(plan, ws, ws_bytes)) return r;

  const int nch_total = F / plan.bf;
  // The single-CTA family is the automatic choice: measured faster on B200
  // for D <= 256 (the pair family trades half the weight bytes per SM for a
  // wider X_lo pass and cross-SM hand-offs).  Pairs stay selectable.
  const bool pair = g_tune_pair == 2;
  if (pair && !pair_supported(D, dtype))
    return fail(MOE_ERR_INVALID_ARG, "CTA-pair kernel not available for D=%d dtype=%d", D, dtype);
  if (g_tune_splits > 0 && nch_total % g_tune_splits != 0)
    return fail(MOE_ERR_INVALID_ARG, "tuning splits=%d does not divide %d chunks", (int)g_tune_splits, nch_total);
  const int splits = small_splits(M, E, nch_total, pair, di->sms);
  const int ctas_req = opt.ctas > 0 ? opt.ctas : (int)g_tune_ctas;
  int ctas = ctas_req > 0 && ctas_req < di->sms ? ctas_req : di->sms;

  int* status = di->status;

  FusedParams prm{};
  prm.group_sizes = gs;
  prm.y = y;
  prm.M = (int)M;
  prm.E = E;
  prm.F = F;
  prm.splits = splits;
  prm.chunks_per_split = nch_total / splits;
  prm.atomic_out = splits > 1 ? 1 : 0;
  prm.status = status;
  prm.trace = reinterpret_cast<unsigned long long*>(g_tune_trace);
  prm.skip_tail = opt.skip_tail ? 1 : 0;
  // Half units in a short last wave need their Y rows zeroed up front: only
  // when the preparation launch runs anyway (F-splits zero all of Y; f32
  // calls that split raw weights or X), so no launch is added for them.
  const bool f32_prep = dtype == MOE_DTYPE_F32 && (split_weights || !plan.x_res);
  prm.tail_halves = (!pair && g_tune_tail == 0 && (splits > 1 || f32_prep)) ? 1 : 0;

  FusedMaps maps;
  memset(&maps, 0, sizeof(maps));
  const size_t wsz = (size_t)E * D * F;
  float* wu_hi = static_cast<float*>(ws);
  float* wu_lo = wu_hi + wsz;
  float* wd_hi = wu_lo + wsz;
  float* wd_lo = wd_hi + wsz;
  float* x_hi = wd_lo + wsz;
  float* x_lo = x_hi + (size_t)M * D;
  const bool f32 = dtype == MOE_DTYPE_F32;
  if (f32 && split_weights)
    if (int r = check_weights_aligned(w_up, w_down)) return r;
  {
    // One preparation launch for what this call needs before the fused kernel.
    PrepArgs pa{};
    const int cap = di->sms * 4;
    if (f32 && split_weights) {
      pa.wu = static_cast<const float*>(w_up);
      pa.wd = static_cast<const float*>(w_down);
      pa.wu_hi = wu_hi;
      pa.wu_lo = wu_lo;
      pa.wd_hi = wd_hi;
      pa.wd_lo = wd_lo;
      pa.D = D;
      pa.F = F;
      pa.E = E;
      pa.w_blocks = E * ((D + 31) / 32) * ((F + 31) / 32);
      pa.w_gs = gs;
    }
    if (f32 && !pair && !plan.x_res) {
      pa.x = static_cast<const float4*>(x);
      pa.x_hi = reinterpret_cast<float4*>(x_hi);
      pa.x_lo = reinterpret_cast<float4*>(x_lo);
      pa.x_n4 = (size_t)M * D / 4;
      pa.x_blocks = (int)std::min<size_t>((pa.x_n4 + 255) / 256, (size_t)cap);
    }
    if (splits > 1) {
      pa.y = reinterpret_cast<float4*>(y);
      pa.y_n4 = (size_t)M * D / 4;
      pa.y_blocks = (int)std::min<size_t>((pa.y_n4 + 255) / 256, (size_t)cap);
    } else if (prm.tail_halves && M > 0) {
      // Half units (at most ctas / 2 blocks of 128 rows) reduce-add into
      // rows zeroed here; the kernel recomputes the same plan.
      pa.y = reinterpret_cast<float4*>(y);
      pa.y_tail = 1;
      pa.gs = gs;
      pa.M = (int)M;
      pa.D = D;
      pa.E = E;
      pa.nch = prm.chunks_per_split;
      pa.grid = ctas;
      const size_t max4 = (size_t)(ctas / 2) * 128 * D / 4;
      pa.y_blocks = (int)std::min<size_t>((max4 + 2047) / 2048, (size_t)di->sms);  // ~8 float4 per thread
    }
    const int blocks = 2 * pa.w_blocks + pa.x_blocks + pa.y_blocks;
    if (blocks > 0) {
      small_prep_kernel<<<blocks, 256, 0, st>>>(pa);
      MOE_CUDA_TRY(cudaGetLastError());
    }
  }

  if (dtype == MOE_DTYPE_BF16) {
    const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (int r = make_map_2d(&maps.x[0], x, BF16, 2, (uint64_t)M, D, 64, 128)) return r;
    if (int r = make_map_2d(&maps.wu[0], w_up, BF16, 2, (uint64_t)E * D, F, 64, 64)) return r;
    if (int r = make_map_2d(&maps.wd[0], w_down, BF16, 2, (uint64_t)E * F, D, 64, 64)) return r;
    if (pair) {
      const int pairs_req = ctas_req > 0 ? ctas_req / 2 : 0;
      if (D == 128) return launch_pair<kModeBF16, 128, 128>(maps, prm, pairs_req, di, st);
      return launch_pair<kModeBF16, 256, 128>(maps, prm, pairs_req, di, st);
    }
    switch (D) {
      case 64: return launch_small<kModeBF16, 64, 128, true>(maps, prm, ctas, di, st);
      case 128: return launch_small<kModeBF16, 128, 128, true>(maps, prm, ctas, di, st);
      case 256: return launch_small<kModeBF16, 256, 128, true>(maps, prm, ctas, di, st);
    }
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "D=%d", D);
  }

  const auto F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (int r = make_map_2d(&maps.wu[0], wu_hi, F32, 4, (uint64_t)E * F, D, 32, plan.bf)) return r;
  if (int r = make_map_2d(&maps.wu[1], wu_lo, F32, 4, (uint64_t)E * F, D, 32, plan.bf)) return r;
  const uint32_t wd_box_rows = pair ? D / 2 : D;
  if (int r = make_map_2d(&maps.wd[0], wd_hi, F32, 4, (uint64_t)E * D, F, 32, wd_box_rows)) return r;
  if (int r = make_map_2d(&maps.wd[1], wd_lo, F32, 4, (uint64_t)E * D, F, 32, wd_box_rows)) return r;
  if (pair) {
    if (int r = make_map_2d(&maps.x[0], x, F32, 4, (uint64_t)M, D, 32, 128)) return r;
    const int pairs_req = ctas_req > 0 ? ctas_req / 2 : 0;
    if (D == 64) return launch_pair<kModeTF32x3, 64, 64>(maps, prm, pairs_req, di, st);
    return launch_pair<kModeTF32x3, 128, 64>(maps, prm, pairs_req, di, st);
  }
  if (plan.x_res) {
    if (int r = make_map_2d(&maps.x[0], x, F32, 4, (uint64_t)M, D, 32, 128)) return r;
  } else {
    if (int r = make_map_2d(&maps.x[0], x_hi, F32, 4, (uint64_t)M, D, 32, 128)) return r;
    if (int r = make_map_2d(&maps.x[1], x_lo, F32, 4, (uint64_t)M, D, 32, 128)) return r;
  }
  switch (D) {
    case 64: return launch_small<kModeTF32x3, 64, 64, true>(maps, prm, ctas, di, st);
    case 128: return launch_small<kModeTF32x3, 128, 64, true>(maps, prm, ctas, di, st);
    case 256: return launch_small<kModeTF32x3, 256, 64, false>(maps, prm, ctas, di, st);
  }
  return fail(MOE_ERR_UNSUPPORTED_SHAPE, "D=%d", D);
}


// ------------------------------------------------------------------ allocation-free entry point
// Scratch of moe_fused_mlp_noalloc: a file-scope device array that every GPU
// loading this library holds until the process exits.  16 MiB fits the 3xTF32
// weight planes of E*D*F <= 1,048,576 weight elements per projection (e.g.
// E=16, D=128, F=512 or E=8, D=128, F=1024).
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// In host code `g_noalloc_scratch` only names a host-side stand-in, so its
// device address is looked up per device (with that device current) and
// cached here together with the context it was resolved in; a new context
// (after cudaDeviceReset) resolves it again.
static void* g_noalloc_ptr[64] = {};
static CUcontext g_noalloc_ctx[64] = {};
static std::mutex g_noalloc_mu;

static int noalloc_scratch(void** out) {
  int dev = 0;
  MOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MOE_ERR_CUDA, "device ordinal %d out of range", dev);
  const CUcontext ctx = current_ctx();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev] || g_noalloc_ctx[dev] != ctx) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(MOE_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}


// ------------------------------------------------------------------ expert-parallel engine
// What one rank publishes to the others (fits MOE_EP_HANDLE_BYTES): the IPC
// handle of its symmetric buffer plus everything the peers must agree on.
struct EpHandleBlob {
  char magic[8];
  int32_t rank, world, el, D, F, dtype, waves, pad;
  int64_t region_cap;
  uint64_t buffer_bytes;
  unsigned char uuid[16];
  cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(EpHandleBlob) <= MOE_EP_HANDLE_BYTES, "handle blob");
static const char kEpMagic[8] = {'m', 'o', 'e', 'e', 'p', '0', '0', '1'};

}  // namespace moe

struct moe_ep_s {
  int dev = -1;
  int rank = 0, world = 1, el = 1, E = 1, D = 0, F = 0, dtype = 0, waves = 1;
  int comm_ctas = 16, mlp_ctas = 0;
  bool scatter = false;  // large-D: combine fused into the down GEMM's epilogue
  size_t off_yl = 0;     // scatter mode: Y landing area (max_tokens rows, f32)
  int4* recv = nullptr;  // scatter mode: [el][world] receive table
  int64_t max_tokens = 0;
  int region_cap = 0;
  size_t off_gs = 0, off_x = 0, off_y = 0, region_x_bytes = 0, region_y_bytes = 0, buf_bytes = 0;
  uint8_t* buf = nullptr;
  uint8_t* peer[moe::kEpMaxWorld] = {};
  bool opened[moe::kEpMaxWorld] = {};
  bool connected = false;
  uint8_t* tables = nullptr;
  moe::EpSlice* slices = nullptr;
  int* wave_rows = nullptr;
  int* local_gs = nullptr;
  int* routed = nullptr;
  unsigned* push_ctr = nullptr;
  int* abort_word = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  const void* w_up = nullptr;
  const void* w_down = nullptr;
  const float* w_up_scale = nullptr;
  const float* w_down_scale = nullptr;
  bool weights_set = false;
  cudaStream_t comm = nullptr;
  cudaEvent_t ev_start = nullptr, ev_end = nullptr;
  cudaEvent_t ev_push[moe::kEpMaxWaves] = {}, ev_mlp[moe::kEpMaxWaves] = {};
  uint32_t epoch = 0;
  int* status = nullptr;
};

namespace moe {

static void ep_release(moe_ep_s* ep) {
  if (!ep) return;
  int prev = -1;
  cudaGetDevice(&prev);
  if (ep->dev >= 0) cudaSetDevice(ep->dev);
  if (ep->comm) cudaStreamSynchronize(ep->comm);
  for (int s = 0; s < kEpMaxWorld; ++s)
    if (ep->opened[s]) cudaIpcCloseMemHandle(ep->peer[s]);
  for (int v = 0; v < kEpMaxWaves; ++v) {
    if (ep->ev_push[v]) cudaEventDestroy(ep->ev_push[v]);
    if (ep->ev_mlp[v]) cudaEventDestroy(ep->ev_mlp[v]);
  }
  if (ep->ev_start) cudaEventDestroy(ep->ev_start);
  if (ep->ev_end) cudaEventDestroy(ep->ev_end);
  if (ep->comm) cudaStreamDestroy(ep->comm);
  if (ep->ws) cudaFree(ep->ws);
  if (ep->tables) cudaFree(ep->tables);
  if (ep->buf) cudaFree(ep->buf);
  if (prev >= 0) cudaSetDevice(prev);
  delete ep;
}

static_assert(kEpMaxWorld == 8, "EpScatter holds 8 peer buffers");

static int ep_mlp_launches(const moe_ep_s* ep) {
  if (!small_supported(ep->D, ep->F, ep->dtype))                   // up + down grouped GEMMs
    return 2;
  return (ep->dtype == MOE_DTYPE_F32 && ep->D == 256) ? 2 : 1;   // (+ X split) fused kernel
}

static int ep_check_device(const moe_ep_s* ep) {
  int dev = -1;
  MOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != ep->dev) return fail(MOE_ERR_INVALID_ARG, "engine lives on device %d, current device is %d", ep->dev, dev);
  return 0;
}

}  // namespace moe

using namespace moe;

namespace moe {
// One sample per block: {SM id, SM cycle counter, global ns timer}.
__global__ void sm_clock_sample_kernel(uint64_t* out) {
  uint32_t smid;
  uint64_t ns;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ns));
  const uint64_t cyc = clock64();
  out[3 * blockIdx.x] = smid;
  out[3 * blockIdx.x + 1] = cyc;
  out[3 * blockIdx.x + 2] = ns;
}
}  // namespace moe

extern "C" {

const char* moe_last_error(void) { return t_err; }

int moe_sm_clock_sample(uint64_t* out, int32_t blocks, void* stream) {
  t_err[0] = 0;
  if (!out || blocks < 1 || blocks > 1024) return fail(MOE_ERR_INVALID_ARG, "out=%p blocks=%d", out, blocks);
  sm_clock_sample_kernel<<<blocks, 1, 0, static_cast<cudaStream_t>(stream)>>>(out);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

int moe_version(void) { return 100; }

int moe_set_tuning(int32_t key, int64_t value) {
  if (value < 0) return fail(MOE_ERR_INVALID_ARG, "negative tuning value");
  switch (key) {
    case 1:
      if (value & (value - 1)) return fail(MOE_ERR_INVALID_ARG, "splits must be a power of two");
      g_tune_splits = value;
      return 0;
    case 2:
      g_tune_ctas = value;
      return 0;
    case 3:
      g_tune_trace = value;
      return 0;
    case 4:
      if (value > 2) return fail(MOE_ERR_INVALID_ARG, "pair mode must be 0, 1 or 2");
      g_tune_pair = value;
      return 0;
    case 5:
      if (value > 64) return fail(MOE_ERR_INVALID_ARG, "rasterisation group must be 0 .. 64 row blocks");
      g_tune_group_m = value;
      return 0;
    case 6:
      if (value > 3) return fail(MOE_ERR_INVALID_ARG, "L2 hint mode must be 0 .. 3");
      g_tune_l2 = value;
      return 0;
    case 7:
      if (value > 2) return fail(MOE_ERR_INVALID_ARG, "e4m3 kernel choice must be 0, 1 or 2");
      g_tune_fp8 = value;
      return 0;
    case 8:
      if (value > 2) return fail(MOE_ERR_INVALID_ARG, "down-GEMM tile width choice must be 0, 1 or 2");
      g_tune_wide = value;
      return 0;
    case 10:
      if (value > 1) return fail(MOE_ERR_INVALID_ARG, "tail-unit choice must be 0 or 1");
      g_tune_tail = value;
      return 0;
  }
  return fail(MOE_ERR_INVALID_ARG, "unknown tuning key %d", key);
}

int moe_device_status(int reset) {
  int v = 0;
  MOE_CUDA_TRY(cudaDeviceSynchronize());
  MOE_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_status, sizeof(int)));
  if (reset) {
    int z = 0;
    MOE_CUDA_TRY(cudaMemcpyToSymbol(g_status, &z, sizeof(int)));
  }
  return v;
}

size_t moe_fused_mlp_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E, int32_t dtype) {
  if (M < 0 || D <= 0 || F <= 0 || E <= 0) return 0;
  if (small_supported(D, F, dtype)) return align256(small_plan(M, D, F, E, dtype).ws_bytes);
  if (large_supported(D, F, dtype)) return align256(large_ws_bytes(M, D, F, E, dtype));
  return 0;
}

static int check_args(const void* x, const void* w_up, const void* w_down, const int32_t* gs, const float* y,
                      int64_t M, int32_t D, int32_t F, int32_t E, int32_t dtype) {
  if (M < 0 || D <= 0 || F <= 0 || E <= 0)
    return fail(MOE_ERR_INVALID_ARG, "bad sizes M=%lld D=%d F=%d E=%d", (long long)M, D, F, E);
  if (M > (int64_t)0x7fffffff) return fail(MOE_ERR_UNSUPPORTED_SHAPE, "M=%lld exceeds 2^31-1", (long long)M);
  if (dtype != MOE_DTYPE_F32 && dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP8_E4M3_BLK128)
    return fail(MOE_ERR_UNSUPPORTED_DTYPE, "dtype %d", dtype);
  if (M == 0) return 0;
  if (!x || !w_up || !w_down || !gs || !y) return fail(MOE_ERR_INVALID_ARG, "null operand pointer");
  if (reinterpret_cast<uintptr_t>(y) & 15u) return fail(MOE_ERR_MISALIGNED, "y must be 16-byte aligned");
  if (!small_supported(D, F, dtype) && !large_supported(D, F, dtype))
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "no kernel for D=%d F=%d dtype=%d", D, F, dtype);
  return 0;
}

int moe_prepare_weights(const void* w_up, const void* w_down, const float* w_up_scale, const float* w_down_scale,
                        int32_t D, int32_t F, int32_t E, int32_t dtype, void* workspace, size_t workspace_bytes,
                        void* stream) {
  t_err[0] = 0;
  (void)w_up_scale;
  (void)w_down_scale;
  if (D <= 0 || F <= 0 || E <= 0) return fail(MOE_ERR_INVALID_ARG, "bad sizes D=%d F=%d E=%d", D, F, E);
  if (dtype != MOE_DTYPE_F32 && dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP8_E4M3_BLK128)
    return fail(MOE_ERR_UNSUPPORTED_DTYPE, "dtype %d", dtype);
  if (!w_up || !w_down) return fail(MOE_ERR_INVALID_ARG, "null weight pointer");
  if (!small_supported(D, F, dtype) && !large_supported(D, F, dtype))
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "no kernel for D=%d F=%d dtype=%d", D, F, dtype);
  // 16-bit and e4m3 weights are used as given; f32 weights (either path)
  // become the four tf32 planes at the start of the workspace.
  return prepare_small(w_up, w_down, D, F, E, dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int moe_fused_mlp_prepared(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                           const float* w_up_scale, const float* w_down_scale, float* y, int64_t M, int32_t D,
                           int32_t F, int32_t E, int32_t dtype, void* workspace, size_t workspace_bytes,
                           void* stream) {
  t_err[0] = 0;
  if (int r = check_args(x, w_up, w_down, group_sizes, y, M, D, F, E, dtype)) return r;
  if (M == 0) return 0;
  if (!small_supported(D, F, dtype))
    return run_large(x, w_up, w_down, group_sizes, w_up_scale, w_down_scale, y, M, D, F, E, dtype, workspace,
                     workspace_bytes, static_cast<cudaStream_t>(stream), RunOpts(), /*split_weights=*/false);
  return run_small(x, w_up, w_down, group_sizes, y, M, D, F, E, dtype, workspace, workspace_bytes,
                   static_cast<cudaStream_t>(stream));
}

int moe_fused_mlp(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                  const float* w_up_scale, const float* w_down_scale, float* y, int64_t M, int32_t D, int32_t F,
                  int32_t E, int32_t dtype, void* workspace, size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (int r = check_args(x, w_up, w_down, group_sizes, y, M, D, F, E, dtype)) return r;
  if (M == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!small_supported(D, F, dtype))
    return run_large(x, w_up, w_down, group_sizes, w_up_scale, w_down_scale, y, M, D, F, E, dtype, workspace,
                     workspace_bytes, st);
  return run_small(x, w_up, w_down, group_sizes, y, M, D, F, E, dtype, workspace, workspace_bytes, st, RunOpts(),
                   true);
}

int moe_fused_mlp_noalloc(const float* x, const float* w_up, const float* w_down, const int32_t* group_sizes,
                          float* y, int64_t M, int32_t D, int32_t F, int32_t E, void* stream) {
  t_err[0] = 0;
  if (int r = check_args(x, w_up, w_down, group_sizes, y, M, D, F, E, MOE_DTYPE_F32)) return r;
  if (M == 0) return 0;
  if (!(D == 64 || D == 128) || F % 64 != 0)
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "moe_fused_mlp_noalloc supports D in {64, 128} and F %% 64 == 0");
  const size_t need = small_plan(M, D, F, E, MOE_DTYPE_F32).ws_bytes;
  if (need > kNoAllocScratchBytes)
    return fail(MOE_ERR_WORKSPACE_TOO_SMALL,
                "moe_fused_mlp_noalloc: E*D*F = %lld needs %zu scratch bytes, above the %zu-byte static buffer "
                "(limit E*D*F <= %zu); use moe_fused_mlp with a caller workspace",
                (long long)E * D * F, need, kNoAllocScratchBytes, kNoAllocScratchBytes / 16);
  void* scratch = nullptr;
  if (int r = noalloc_scratch(&scratch)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Every scratch byte the fused kernel reads is written by the weight split
  // earlier in this same call, so nothing needs clearing between calls.
  return run_small(x, w_up, w_down, group_sizes, y, M, D, F, E, MOE_DTYPE_F32, scratch, kNoAllocScratchBytes, st,
                   RunOpts(), true);
}

// ------------------------------------------------------------------ expert-parallel engine
int moe_ep_create(int32_t rank, int32_t world, int32_t num_local_experts, int64_t max_tokens, int32_t D, int32_t F,
                  int32_t dtype, int32_t waves, int32_t comm_ctas, moe_ep_t* out) {
  t_err[0] = 0;
  if (!out) return fail(MOE_ERR_INVALID_ARG, "null output handle");
  *out = nullptr;
  if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world)
    return fail(MOE_ERR_INVALID_ARG, "rank %d / world %d (world must be 1..%d)", rank, world, kEpMaxWorld);
  if (num_local_experts < 1 || (int64_t)num_local_experts * world > kEpMaxExperts)
    return fail(MOE_ERR_INVALID_ARG, "%d experts per rank x %d ranks (at most %d experts)", num_local_experts,
                world, kEpMaxExperts);
  if (waves < 1 || waves > kEpMaxWaves) return fail(MOE_ERR_INVALID_ARG, "waves %d (1..%d)", waves, kEpMaxWaves);
  if (max_tokens < 1) return fail(MOE_ERR_INVALID_ARG, "max_tokens %lld", (long long)max_tokens);
  if (comm_ctas < 0 || comm_ctas > 64) return fail(MOE_ERR_INVALID_ARG, "comm_ctas %d (0..64)", comm_ctas);
  if (dtype != MOE_DTYPE_F32 && dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_FP8_E4M3_BLK128)
    return fail(MOE_ERR_UNSUPPORTED_DTYPE, "dtype %d", dtype);
  if (D <= 0 || F <= 0 || (!small_supported(D, F, dtype) && !large_supported(D, F, dtype)))
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "no kernel for D=%d F=%d dtype=%d", D, F, dtype);
  // The engine's two-GEMM experts are the 16-bit / e4m3 grouped GEMMs on
  // whole 256-column tiles; f32 runs through the fused small-D kernels only.
  if (!small_supported(D, F, dtype) && (dtype == MOE_DTYPE_F32 || D % 256 != 0 || F % 256 != 0))
    return fail(MOE_ERR_UNSUPPORTED_SHAPE,
                "expert-parallel engine: two-GEMM experts need bf16 or e4m3 with D and F multiples of 256 "
                "(got D=%d F=%d dtype=%d)", D, F, dtype);
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;

  // Large-D experts (two grouped GEMMs) take the combine into the down GEMM's
  // epilogue: one wave on every SM, rows stored straight back to their
  // sources.  Small-D experts pull their results back in `waves` slices.
  const bool scatter = !small_supported(D, F, dtype);
  if (scatter) waves = 1;
  // Rows per landing region: wave v of a group of c rows holds at most
  // ceil(c / waves) <= c / waves + 1 rows, over world sources and el experts.
  const int64_t cap64 = ((int64_t)world * max_tokens + waves - 1) / waves + (int64_t)world * num_local_experts;
  const int64_t cap = (cap64 + 255) / 256 * 256;
  if (cap > (int64_t)1 << 30 || max_tokens > (int64_t)1 << 30)
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "landing region of %lld rows", (long long)cap);

  moe_ep_s* ep = new moe_ep_s();
  ep->dev = dev;
  ep->rank = rank;
  ep->world = world;
  ep->el = num_local_experts;
  ep->E = world * num_local_experts;
  ep->D = D;
  ep->F = F;
  ep->dtype = dtype;
  ep->waves = waves;
  ep->comm_ctas = comm_ctas > 0 ? comm_ctas : 16;
  ep->max_tokens = max_tokens;
  ep->region_cap = (int)cap;
  const int sx = dtype == MOE_DTYPE_F32 ? 4 : 2;
  ep->off_gs = 4096;
  ep->off_x = align256(ep->off_gs + (size_t)2 * world * ep->E * sizeof(int32_t));
  ep->region_x_bytes = align256((size_t)cap * D * sx);
  ep->scatter = scatter;
  ep->off_y = ep->off_x + (size_t)waves * ep->region_x_bytes;
  ep->region_y_bytes = scatter ? 0 : align256((size_t)cap * D * sizeof(float));
  ep->off_yl = ep->off_y + (size_t)waves * ep->region_y_bytes;
  ep->buf_bytes = ep->off_yl + (scatter ? align256((size_t)max_tokens * D * sizeof(float)) : 0);
  // Exchange kernels that run beside the experts take the SMs the expert
  // kernels leave free (pairs: even); in scatter mode nothing runs beside them.
  ep->mlp_ctas = world > 1 && !scatter ? ((di->sms - ep->comm_ctas) & ~1) : 0;
  if (world > 1 && !scatter && ep->mlp_ctas < 2) {
    ep_release(ep);
    return fail(MOE_ERR_INVALID_ARG, "comm_ctas %d leaves no SMs for the experts", comm_ctas);
  }

  auto cuda_fail = [&](cudaError_t e, const char* what) {
    ep_release(ep);
    return fail(MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  };
  cudaError_t e;
  if ((e = cudaMalloc(&ep->buf, ep->buf_bytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(symmetric buffer)");
  if ((e = cudaMemset(ep->buf, 0, ep->off_x)) != cudaSuccess) return cuda_fail(e, "cudaMemset(flags)");
  const size_t t_slices = align256((size_t)waves * ep->E * sizeof(EpSlice));
  const size_t t_rows = align256((size_t)waves * (ep->E + 1) * sizeof(int));
  const size_t t_gs = align256((size_t)waves * ep->el * sizeof(int));
  const size_t t_misc = 256 + (size_t)kEpMaxWaves * sizeof(unsigned) + 256;
  const size_t t_recv = scatter ? align256((size_t)ep->el * world * sizeof(int4)) : 0;
  const size_t t_all = t_slices + t_rows + t_gs + t_misc + t_recv;
  if ((e = cudaMalloc(&ep->tables, t_all)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(tables)");
  if ((e = cudaMemset(ep->tables, 0, t_all)) != cudaSuccess) return cuda_fail(e, "cudaMemset(tables)");
  ep->slices = reinterpret_cast<EpSlice*>(ep->tables);
  ep->wave_rows = reinterpret_cast<int*>(ep->tables + t_slices);
  ep->local_gs = reinterpret_cast<int*>(ep->tables + t_slices + t_rows);
  ep->routed = reinterpret_cast<int*>(ep->tables + t_slices + t_rows + t_gs);
  ep->push_ctr = reinterpret_cast<unsigned*>(ep->tables + t_slices + t_rows + t_gs + 256);
  ep->abort_word = reinterpret_cast<int*>(ep->tables + t_slices + t_rows + t_gs + 256 + 256);
  if (scatter) ep->recv = reinterpret_cast<int4*>(ep->tables + t_slices + t_rows + t_gs + t_misc);
  ep->ws_bytes = small_supported(D, F, dtype) ? align256(small_plan(cap, D, F, ep->el, dtype).ws_bytes)
                                              : align256(large_ws_bytes(cap, D, F, ep->el, dtype));
  if (ep->ws_bytes && (e = cudaMalloc(&ep->ws, ep->ws_bytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(workspace)");
  if ((e = cudaStreamCreateWithFlags(&ep->comm, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_fail(e, "cudaStreamCreate");
  if ((e = cudaEventCreateWithFlags(&ep->ev_start, cudaEventDisableTiming)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&ep->ev_end, cudaEventDisableTiming)) != cudaSuccess)
    return cuda_fail(e, "cudaEventCreate");
  for (int v = 0; v < waves; ++v)
    if ((e = cudaEventCreateWithFlags(&ep->ev_push[v], cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&ep->ev_mlp[v], cudaEventDisableTiming)) != cudaSuccess)
      return cuda_fail(e, "cudaEventCreate");
  if ((e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ep->status), g_status)) != cudaSuccess)
    return cuda_fail(e, "cudaGetSymbolAddress(status)");
  // The largest engine's need, so that engines of different sizes coexist.
  const size_t smem = ep_counts_smem(kEpMaxWorld, kEpMaxExperts, kEpMaxWaves);
  if ((e = cudaFuncSetAttribute(ep_counts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
      cudaSuccess)
    return cuda_fail(e, "cudaFuncSetAttribute(ep_counts_kernel)");
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  ep->peer[rank] = ep->buf;
  *out = ep;
  return 0;
}

int moe_ep_export(moe_ep_t ep, void* handle) {
  t_err[0] = 0;
  if (!ep || !handle) return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (int r = ep_check_device(ep)) return r;
  EpHandleBlob b;
  memset(&b, 0, sizeof(b));
  memcpy(b.magic, kEpMagic, sizeof(b.magic));
  b.rank = ep->rank;
  b.world = ep->world;
  b.el = ep->el;
  b.D = ep->D;
  b.F = ep->F;
  b.dtype = ep->dtype;
  b.waves = ep->waves;
  b.region_cap = ep->region_cap;
  b.buffer_bytes = ep->buf_bytes;
  cudaDeviceProp prop;
  MOE_CUDA_TRY(cudaGetDeviceProperties(&prop, ep->dev));
  memcpy(b.uuid, &prop.uuid, sizeof(b.uuid));
  MOE_CUDA_TRY(cudaIpcGetMemHandle(&b.ipc, ep->buf));
  memset(handle, 0, MOE_EP_HANDLE_BYTES);
  memcpy(handle, &b, sizeof(b));
  return 0;
}

int moe_ep_connect(moe_ep_t ep, const void* handles) {
  t_err[0] = 0;
  if (!ep || !handles) return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (ep->connected) return fail(MOE_ERR_INVALID_ARG, "engine already connected");
  if (int r = ep_check_device(ep)) return r;
  const unsigned char* hb = static_cast<const unsigned char*>(handles);
  EpHandleBlob mine;
  memcpy(&mine, hb + (size_t)ep->rank * MOE_EP_HANDLE_BYTES, sizeof(mine));
  cudaDeviceProp prop;
  MOE_CUDA_TRY(cudaGetDeviceProperties(&prop, ep->dev));
  for (int s = 0; s < ep->world; ++s) {
    EpHandleBlob b;
    memcpy(&b, hb + (size_t)s * MOE_EP_HANDLE_BYTES, sizeof(b));
    if (memcmp(b.magic, kEpMagic, sizeof(b.magic)) != 0)
      return fail(MOE_ERR_INVALID_ARG, "handle %d is not an expert-parallel handle", s);
    if (b.rank != s || b.world != ep->world || b.el != ep->el || b.D != ep->D || b.F != ep->F ||
        b.dtype != ep->dtype || b.waves != ep->waves || b.region_cap != ep->region_cap ||
        b.buffer_bytes != ep->buf_bytes)
      return fail(MOE_ERR_INVALID_ARG,
                  "handle %d (rank %d of %d, %d experts, D=%d F=%d dtype=%d waves=%d) does not match this engine",
                  s, b.rank, b.world, b.el, b.D, b.F, b.dtype, b.waves);
    if (s == ep->rank) continue;
    // Exchange kernels of two ranks on one GPU would wait on one another
    // with no guarantee of running at the same time: refuse.
    if (memcmp(b.uuid, &prop.uuid, sizeof(b.uuid)) == 0)
      return fail(MOE_ERR_INVALID_ARG, "ranks %d and %d share one GPU; every rank needs its own", s, ep->rank);
  }
  for (int s = 0; s < ep->world; ++s) {
    if (s == ep->rank) continue;
    EpHandleBlob b;
    memcpy(&b, hb + (size_t)s * MOE_EP_HANDLE_BYTES, sizeof(b));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, b.ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < s; ++q)
        if (ep->opened[q]) {
          cudaIpcCloseMemHandle(ep->peer[q]);
          ep->opened[q] = false;
          ep->peer[q] = nullptr;
        }
      return fail(MOE_ERR_CUDA, "cudaIpcOpenMemHandle(rank %d): %s", s, cudaGetErrorString(e));
    }
    ep->peer[s] = static_cast<uint8_t*>(p);
    ep->opened[s] = true;
  }
  ep->connected = true;
  return 0;
}

int moe_ep_set_weights(moe_ep_t ep, const void* w_up_local, const void* w_down_local, const float* w_up_scale,
                       const float* w_down_scale, void* stream) {
  t_err[0] = 0;
  if (!ep || !w_up_local || !w_down_local) return fail(MOE_ERR_INVALID_ARG, "null argument");
  if (int r = ep_check_device(ep)) return r;
  if (ep->dtype == MOE_DTYPE_FP8_E4M3_BLK128 && (!w_up_scale || !w_down_scale))
    return fail(MOE_ERR_INVALID_ARG, "FP8 weights need w_up_scale and w_down_scale");
  ep->w_up = w_up_local;
  ep->w_down = w_down_local;
  ep->w_up_scale = w_up_scale;
  ep->w_down_scale = w_down_scale;
  if (small_supported(ep->D, ep->F, ep->dtype))
    if (int r = prepare_small(w_up_local, w_down_local, ep->D, ep->F, ep->el, ep->dtype, ep->ws, ep->ws_bytes,
                              static_cast<cudaStream_t>(stream)))
      return r;
  ep->weights_set = true;
  return 0;
}

int moe_ep_forward(moe_ep_t ep, const void* x, const int32_t* group_sizes, float* y, int64_t M, void* stream) {
  t_err[0] = 0;
  if (!ep) return fail(MOE_ERR_INVALID_ARG, "null engine");
  if (!ep->connected) return fail(MOE_ERR_INVALID_ARG, "engine not connected (moe_ep_connect)");
  if (!ep->weights_set) return fail(MOE_ERR_INVALID_ARG, "no expert weights (moe_ep_set_weights)");
  if (int r = ep_check_device(ep)) return r;
  if (M < 0 || M > ep->max_tokens)
    return fail(MOE_ERR_INVALID_ARG, "M=%lld outside [0, max_tokens=%lld]", (long long)M, (long long)ep->max_tokens);
  if (!group_sizes) return fail(MOE_ERR_INVALID_ARG, "null group_sizes");
  if (M > 0 && (!x || (!y && !ep->scatter))) return fail(MOE_ERR_INVALID_ARG, "null x or y");
  if (!y && ep->scatter) y = reinterpret_cast<float*>(ep->buf + ep->off_yl);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "x and y must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  EpArgs a;
  memset(&a, 0, sizeof(a));
  for (int s = 0; s < ep->world; ++s) a.base[s] = ep->peer[s];
  a.rank = ep->rank;
  a.world = ep->world;
  a.el = ep->el;
  a.E = ep->E;
  a.waves = ep->waves;
  a.region_cap = ep->region_cap;
  a.max_rows = (int)ep->max_tokens;
  a.M = (int)M;
  a.epoch = ++ep->epoch;
  a.off_gs = ep->off_gs;
  a.off_x = ep->off_x;
  a.off_y = ep->off_y;
  a.region_x_bytes = ep->region_x_bytes;
  a.region_y_bytes = ep->region_y_bytes;
  a.row_bytes_x = ep->D * (ep->dtype == MOE_DTYPE_F32 ? 4 : 2);
  a.row_bytes_y = ep->D * 4;
  a.gs = group_sizes;
  a.x = static_cast<const uint8_t*>(x);
  a.y = y;
  a.slices = ep->slices;
  a.wave_rows = ep->wave_rows;
  a.local_gs = ep->local_gs;
  a.recv = ep->recv;
  a.off_yl = ep->off_yl;
  a.routed = ep->routed;
  a.push_ctr = ep->push_ctr;
  a.abort_word = ep->abort_word;
  a.status = ep->status;

  MOE_CUDA_TRY(cudaEventRecord(ep->ev_start, st));
  MOE_CUDA_TRY(cudaStreamWaitEvent(ep->comm, ep->ev_start, 0));
  ep_counts_kernel<<<1, 1024, ep_counts_smem(ep->world, ep->E, ep->waves), ep->comm>>>(a);
  MOE_CUDA_TRY(cudaGetLastError());
  RunOpts opt;
  opt.ctas = ep->mlp_ctas;
  opt.skip_tail = true;
  if (ep->scatter && ep->dtype == MOE_DTYPE_BF16) {
    // bf16 two-GEMM experts: the owner's own rows are copied into its landing
    // region first (they lead every expert's rows), then the up GEMM starts at
    // once: its dispatch warps push this rank's rows to the other owners while
    // its producer waits, tile by tile, only for the peers whose rows the tile
    // reads.  The down GEMM stores each Y row into its source's landing area.
    int dev;
    DevInfo* di;
    if (int r = device_info(&dev, &di)) return r;
    MOE_CUDA_TRY(cudaEventRecord(ep->ev_push[0], ep->comm));
    MOE_CUDA_TRY(cudaStreamWaitEvent(st, ep->ev_push[0], 0));
    ep_push_kernel<<<di->sms, 1024, 0, st>>>(a, 0, 1);
    MOE_CUDA_TRY(cudaGetLastError());
    EpDispatch dp;
    memset(&dp, 0, sizeof(dp));
    for (int s2 = 0; s2 < ep->world; ++s2) dp.base[s2] = ep->peer[s2];
    dp.x = static_cast<const uint8_t*>(x);
    dp.off_x = ep->off_x;
    dp.slices = ep->slices;
    dp.wave_rows = ep->wave_rows;
    dp.recv = ep->recv;
    dp.data_flags = reinterpret_cast<EpFlags*>(ep->buf)->data[0];
    dp.push_ctr = ep->push_ctr;
    dp.abort_word = ep->abort_word;
    dp.E = ep->E;
    dp.rank = ep->rank;
    dp.world = ep->world;
    dp.row_bytes = a.row_bytes_x;
    dp.epoch = a.epoch;
    dp.on = 1;
    opt.dispatch = &dp;
    EpScatter sc;
    memset(&sc, 0, sizeof(sc));
    for (int s2 = 0; s2 < ep->world; ++s2) sc.base[s2] = ep->peer[s2];
    sc.off = ep->off_yl;
    sc.recv = ep->recv;
    sc.world = ep->world;
    sc.on = 1;
    opt.scatter = &sc;
    float* yl = reinterpret_cast<float*>(ep->buf + ep->off_yl);
    if (int r = run_large(ep->buf + ep->off_x, ep->w_up, ep->w_down, ep->local_gs, ep->w_up_scale, ep->w_down_scale,
                          yl, ep->region_cap, ep->D, ep->F, ep->el, ep->dtype, ep->ws, ep->ws_bytes, st, opt))
      return r;
    ep_ydone_kernel<<<1, 32, 0, st>>>(a);
    MOE_CUDA_TRY(cudaGetLastError());
    ep_finish_kernel<<<di->sms, 1024, 0, st>>>(a);
    MOE_CUDA_TRY(cudaGetLastError());
    return 0;
  }
  // In scatter mode the push runs before the experts, alone: it gets every SM.
  int push_ctas = ep->comm_ctas;
  if (ep->scatter) {
    int dev;
    DevInfo* di;
    if (int r = device_info(&dev, &di)) return r;
    push_ctas = di->sms;
  }
  for (int v = 0; v < ep->waves; ++v) {
    ep_push_kernel<<<push_ctas, 1024, 0, ep->comm>>>(a, v, 0);
    MOE_CUDA_TRY(cudaGetLastError());
    MOE_CUDA_TRY(cudaEventRecord(ep->ev_push[v], ep->comm));
  }
  if (ep->scatter) {
    // One wave: land every row, run both GEMMs on every SM with the down
    // GEMM storing each Y row straight into its source's landing area, tell
    // the sources, and finish this rank's Y once every owner has told it.
    EpScatter sc;
    memset(&sc, 0, sizeof(sc));
    for (int s2 = 0; s2 < ep->world; ++s2) sc.base[s2] = ep->peer[s2];
    sc.off = ep->off_yl;
    sc.recv = ep->recv;
    sc.world = ep->world;
    sc.on = 1;
    opt.scatter = &sc;
    MOE_CUDA_TRY(cudaStreamWaitEvent(st, ep->ev_push[0], 0));
    ep_wait_kernel<<<1, 32, 0, st>>>(a, 0);
    MOE_CUDA_TRY(cudaGetLastError());
    float* yl = reinterpret_cast<float*>(ep->buf + ep->off_yl);
    if (int r = run_large(ep->buf + ep->off_x, ep->w_up, ep->w_down, ep->local_gs, ep->w_up_scale, ep->w_down_scale,
                          yl, ep->region_cap, ep->D, ep->F, ep->el, ep->dtype, ep->ws, ep->ws_bytes, st, opt))
      return r;
    ep_ydone_kernel<<<1, 32, 0, st>>>(a);
    MOE_CUDA_TRY(cudaGetLastError());
    int dev;
    DevInfo* di;
    if (int r = device_info(&dev, &di)) return r;
    ep_finish_kernel<<<di->sms, 1024, 0, st>>>(a);
    MOE_CUDA_TRY(cudaGetLastError());
    return 0;
  }
  for (int v = 0; v < ep->waves; ++v) {
    MOE_CUDA_TRY(cudaStreamWaitEvent(st, ep->ev_push[v], 0));
    ep_wait_kernel<<<1, 32, 0, st>>>(a, v);
    MOE_CUDA_TRY(cudaGetLastError());
    const void* xr = ep->buf + ep->off_x + (size_t)v * ep->region_x_bytes;
    float* yr = reinterpret_cast<float*>(ep->buf + ep->off_y + (size_t)v * ep->region_y_bytes);
    const int32_t* gs_v = ep->local_gs + (size_t)v * ep->el;
    int r;
    if (small_supported(ep->D, ep->F, ep->dtype))
      r = run_small(xr, ep->w_up, ep->w_down, gs_v, yr, ep->region_cap, ep->D, ep->F, ep->el, ep->dtype, ep->ws,
                    ep->ws_bytes, st, opt);
    else
      r = run_large(xr, ep->w_up, ep->w_down, gs_v, ep->w_up_scale, ep->w_down_scale, yr, ep->region_cap, ep->D,
                    ep->F, ep->el, ep->dtype, ep->ws, ep->ws_bytes, st, opt);
    if (r) return r;
    MOE_CUDA_TRY(cudaEventRecord(ep->ev_mlp[v], st));
    MOE_CUDA_TRY(cudaStreamWaitEvent(ep->comm, ep->ev_mlp[v], 0));
    ep_pull_kernel<<<ep->comm_ctas, 1024, 0, ep->comm>>>(a, v);
    MOE_CUDA_TRY(cudaGetLastError());
  }
  MOE_CUDA_TRY(cudaEventRecord(ep->ev_end, ep->comm));
  MOE_CUDA_TRY(cudaStreamWaitEvent(st, ep->ev_end, 0));
  return 0;
}

int moe_ep_launches_per_forward(moe_ep_t ep) {
  if (!ep) return fail(MOE_ERR_INVALID_ARG, "null engine");
  if (ep->scatter && ep->dtype == MOE_DTYPE_BF16)
    return 2 + ep_mlp_launches(ep) + 2;  // counts, local copy, GEMMs (dispatch inside the up GEMM), ydone, finish
  if (ep->scatter) return 3 + ep_mlp_launches(ep) + 2;  // counts, push, wait, GEMMs, ydone, finish
  return 1 + ep->waves * (3 + ep_mlp_launches(ep));
}

void* moe_ep_output(moe_ep_t ep) {
  if (!ep || !ep->scatter) return nullptr;
  return ep->buf + ep->off_yl;
}

int moe_ep_destroy(moe_ep_t ep) {
  t_err[0] = 0;
  ep_release(ep);
  return 0;
}

// ------------------------------------------------------------------ routing and permutation
int moe_route_topk(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* topk_ids, float* topk_weights,
                   void* stream) {
  t_err[0] = 0;
  if (T < 0 || E < 1 || E > kRouteMaxExperts || k < 1 || k > kRouteMaxK || k > E)
    return fail(MOE_ERR_INVALID_ARG, "T=%lld E=%d k=%d (1 <= k <= min(%d, E), E <= %d)", (long long)T, E, k,
                kRouteMaxK, kRouteMaxExperts);
  if (T == 0) return 0;
  if (!logits || !topk_ids || !topk_weights) return fail(MOE_ERR_INVALID_ARG, "null pointer");
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const int blocks = (int)std::min<int64_t>((T + 7) / 8, (int64_t)di->sms * 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int pl = (E + 31) / 32;
  if (pl <= 1) launch_topk<1>(logits, T, E, k, topk_ids, topk_weights, blocks, st);
  else if (pl <= 2) launch_topk<2>(logits, T, E, k, topk_ids, topk_weights, blocks, st);
  else if (pl <= 4) launch_topk<4>(logits, T, E, k, topk_ids, topk_weights, blocks, st);
  else if (pl <= 8) launch_topk<8>(logits, T, E, k, topk_ids, topk_weights, blocks, st);
  else if (pl <= 16) launch_topk<16>(logits, T, E, k, topk_ids, topk_weights, blocks, st);
  else launch_topk<32>(logits, T, E, k, topk_ids, topk_weights, blocks, st);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

size_t moe_permute_workspace_size(int64_t N, int32_t E) {
  if (N < 0 || E < 1) return 0;
  return align256((size_t)((N + kPermBlock - 1) / kPermBlock) * (size_t)E * sizeof(int32_t));
}

int moe_permute(const int32_t* expert_ids, int64_t N, int32_t E, int32_t* group_sizes, int32_t* sorted_src,
                int32_t* inverse, void* workspace, size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (N < 0 || N > 0x7fffffff || E < 1 || E > kRouteMaxExperts)
    return fail(MOE_ERR_INVALID_ARG, "N=%lld E=%d (N < 2^31, 1 <= E <= %d)", (long long)N, E, kRouteMaxExperts);
  if (!group_sizes) return fail(MOE_ERR_INVALID_ARG, "null group_sizes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N == 0) {
    MOE_CUDA_TRY(cudaMemsetAsync(group_sizes, 0, (size_t)E * sizeof(int32_t), st));
    return 0;
  }
  if (!expert_ids || !sorted_src || !inverse) return fail(MOE_ERR_INVALID_ARG, "null pointer");
  const size_t need = moe_permute_workspace_size(N, E);
  if (workspace_bytes < need || !workspace)
    return fail(MOE_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", workspace_bytes, need);
  static bool attr_done[64] = {};
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  int* status = di->status;
  const size_t smem_scatter = (size_t)(kPermBlock / 32) * E * sizeof(int);
  if (!attr_done[dev]) {
    MOE_CUDA_TRY(cudaFuncSetAttribute(perm_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)((kPermBlock / 32) * kRouteMaxExperts * sizeof(int))));
    attr_done[dev] = true;
  }
  const int64_t nb = (N + kPermBlock - 1) / kPermBlock;
  int32_t* hist = static_cast<int32_t*>(workspace);
  perm_hist_kernel<<<(unsigned)nb, kPermBlock, E * sizeof(int), st>>>(expert_ids, N, E, hist, status);
  MOE_CUDA_TRY(cudaGetLastError());
  perm_scan_kernel<<<1, 1024, 0, st>>>(hist, nb, E, group_sizes);
  MOE_CUDA_TRY(cudaGetLastError());
  perm_scatter_kernel<<<(unsigned)nb, kPermBlock, smem_scatter, st>>>(expert_ids, N, E, hist, sorted_src, inverse);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

int moe_gather_rows(const void* x, const int32_t* sorted_src, int64_t rows, int32_t k, int32_t row_bytes, void* out,
                    void* stream) {
  t_err[0] = 0;
  if (rows < 0 || k < 1 || row_bytes <= 0 || (row_bytes & 15))
    return fail(MOE_ERR_INVALID_ARG, "rows=%lld k=%d row_bytes=%d (a positive multiple of 16)", (long long)rows, k,
                row_bytes);
  if (rows == 0) return 0;
  if (!x || !sorted_src || !out) return fail(MOE_ERR_INVALID_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "x and out must be 16-byte aligned");
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const int blocks = (int)std::min<int64_t>((rows + 15) / 16, (int64_t)di->sms * 4);
  gather_rows_kernel<<<blocks, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(x), sorted_src, rows, k, row_bytes, static_cast<uint8_t*>(out));
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

int moe_combine_rows(const float* y_sorted, const int32_t* inverse, const float* weights, int64_t T, int32_t k,
                     int32_t D, float* y, void* stream) {
  t_err[0] = 0;
  if (T < 0 || k < 1 || D <= 0 || (D & 3))
    return fail(MOE_ERR_INVALID_ARG, "T=%lld k=%d D=%d (D a positive multiple of 4)", (long long)T, k, D);
  if (T == 0) return 0;
  if (!y_sorted || !inverse || !weights || !y) return fail(MOE_ERR_INVALID_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(y_sorted) | reinterpret_cast<uintptr_t>(y)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "y_sorted and y must be 16-byte aligned");
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const int blocks = (int)std::min<int64_t>((T + 15) / 16, (int64_t)di->sms * 4);
  combine_rows_kernel<<<blocks, 512, 0, static_cast<cudaStream_t>(stream)>>>(y_sorted, inverse, weights, T, k, D, y);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

// ------------------------------------------------------------------ SwiGLU experts
int moe_swiglu_interleave(const void* w_gate, const void* w_up, void* w_gate_up, int32_t E, int32_t D, int32_t F,
                          void* stream) {
  t_err[0] = 0;
  if (E <= 0 || D <= 0 || F <= 0 || F % 128) return fail(MOE_ERR_INVALID_ARG, "E=%d D=%d F=%d (F %% 128 == 0)", E, D, F);
  if (!w_gate || !w_up || !w_gate_up) return fail(MOE_ERR_INVALID_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(w_gate) | reinterpret_cast<uintptr_t>(w_up) |
       reinterpret_cast<uintptr_t>(w_gate_up)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "weights must be 16-byte aligned");
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const size_t rows = (size_t)E * D, n = rows * (size_t)(F / 4);
  const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)di->sms * 8);
  swiglu_interleave_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(w_gate), static_cast<const uint4*>(w_up), static_cast<uint4*>(w_gate_up), rows, F / 8,
      16);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

size_t moe_fused_mlp_swiglu_workspace_size(int64_t M, int32_t D, int32_t F) {
  if (M < 0 || !swiglu_supported(D, F)) return 0;
  return align256((size_t)M * F * 2);
}

int moe_fused_mlp_swiglu(const void* x, const void* w_gate_up, const void* w_down, const int32_t* group_sizes,
                         float* y, int64_t M, int32_t D, int32_t F, int32_t E, void* workspace,
                         size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (M < 0 || D <= 0 || F <= 0 || E <= 0)
    return fail(MOE_ERR_INVALID_ARG, "bad sizes M=%lld D=%d F=%d E=%d", (long long)M, D, F, E);
  if (M > (int64_t)0x7fffffff) return fail(MOE_ERR_UNSUPPORTED_SHAPE, "M=%lld exceeds 2^31-1", (long long)M);
  if (!swiglu_supported(D, F))
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "SwiGLU experts need D %% 256 == 0 (D >= 256) and F %% 128 == 0");
  if (M == 0) return 0;
  if (!x || !w_gate_up || !w_down || !group_sizes || !y) return fail(MOE_ERR_INVALID_ARG, "null operand pointer");
  if (reinterpret_cast<uintptr_t>(y) & 15u) return fail(MOE_ERR_MISALIGNED, "y must be 16-byte aligned");
  return run_swiglu(x, w_gate_up, w_down, nullptr, nullptr, group_sizes, y, M, D, F, E, false, workspace,
                    workspace_bytes, static_cast<cudaStream_t>(stream));
}

int moe_fused_mlp_launch_count(int64_t M, int32_t D, int32_t F, int32_t E, int32_t dtype) {
  t_err[0] = 0;
  if (M < 0 || D <= 0 || F <= 0 || E <= 0 || dtype < 0 || dtype > 2)
    return fail(MOE_ERR_INVALID_ARG, "bad arguments M=%lld D=%d F=%d E=%d dtype=%d", (long long)M, D, F, E, dtype);
  if (M == 0) return 0;
  if (!small_supported(D, F, dtype)) {
    if (!large_supported(D, F, dtype)) return fail(MOE_ERR_UNSUPPORTED_SHAPE, "D=%d F=%d dtype=%d", D, F, dtype);
    // bf16 and e4m3 weights: up GEMM, down GEMM; f32: the tf32 split first
    return dtype == MOE_DTYPE_F32 ? 3 : 2;
  }
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  const SmallPlan plan = small_plan(M, D, F, E, dtype);
  const int splits = small_splits(M, E, F / plan.bf, g_tune_pair == 2, di->sms);
  // One preparation launch (weight planes, X planes, Y zeroing) when any of
  // them is needed, then the fused kernel.
  return (dtype == MOE_DTYPE_F32 || splits > 1 ? 1 : 0) + 1;
}

}  // extern "C"

namespace moe {
static void desc_set(moe_launch_desc* d, const char* name, int grid, int threads, int smem, int tmem, int cluster,
                     int tm, int tn, int sk, int stages, int kind, int n, int k, int splits, int accs) {
  memset(d, 0, sizeof(*d));
  snprintf(d->kernel, sizeof(d->kernel), "%s", name);
  d->grid = grid;
  d->threads = threads;
  d->smem_bytes = smem;
  d->tmem_cols = tmem;
  d->cluster = cluster;
  d->tile_m = tm;
  d->tile_n = tn;
  d->stage_k = sk;
  d->stages = stages;
  d->mma_kind = kind;
  d->gemm_n = n;
  d->gemm_k = k;
  d->f_splits = splits;
  d->accumulators = accs;
}
template <int EPI, bool BFP8, bool TF32, int WIDE = 1>
static void desc_gemm(moe_launch_desc* d, const char* name, int pairs, int N, int K) {
  using C = GemmCfg<EPI, BFP8, TF32, WIDE>;
  desc_set(d, name, 2 * pairs, C::THREADS, C::SMEM, C::TMEM_COLS, 2, 2 * C::BM, C::TILE_N, C::BK, C::NS,
           TF32 ? MOE_MMA_TF32X3 : (BFP8 ? (EPI == 1 ? MOE_MMA_F16_E4M3 : MOE_MMA_BF16_E4M3) : MOE_MMA_BF16), N, K, 1,
           (int)C::NACC);
}
// Super-tile kernel: tile_m = tokens per super-tile, tile_n = features per tile.
template <int EPI>
static void desc_swap(moe_launch_desc* d, const char* name, int pairs, int N, int K) {
  using C = SwapCfg<EPI>;
  desc_set(d, name, 2 * pairs, C::THREADS, C::SMEM, C::TMEM_COLS, 2, C::TOKENS, 2 * C::FM, C::BK, C::NS,
           EPI == 1 ? MOE_MMA_F16_E4M3 : MOE_MMA_BF16_E4M3, N, K, 1, 2);
}
template <int MODE, int D, int BF, bool XR>
static void desc_small(moe_launch_desc* d, int ctas, int F, int splits) {
  using C = FusedCfg<MODE, D, BF, XR>;
  desc_set(d, "fused_mlp_small_kernel", ctas, C::THREADS, C::SMEM, C::TMEM_COLS, 1, C::BM, BF, C::SK1, C::NS,
           MODE == kModeTF32x3 ? MOE_MMA_TF32X3 : MOE_MMA_BF16, D, F, splits, 2);
}
}  // namespace moe

extern "C" {

int moe_ep_build_tables(const int32_t* counts, int32_t world, int32_t rank, int32_t num_local_experts,
                        int32_t waves, int32_t region_cap, int32_t max_rows, int64_t M, int32_t* slices,
                        int32_t* wave_rows, int32_t* local_gs, int32_t* recv) {
  t_err[0] = 0;
  const int W = world, EL = num_local_experts, V = waves;
  if (W < 1 || W > kEpMaxWorld || rank < 0 || rank >= W || EL < 1 || (int64_t)EL * W > kEpMaxExperts || V < 1 ||
      V > kEpMaxWaves || region_cap < 0 || max_rows < 0 || M < 0 || M > 0x7fffffff || !counts || !slices ||
      !wave_rows || !local_gs)
    return fail(MOE_ERR_INVALID_ARG, "moe_ep_build_tables: bad arguments");
  const int E = W * EL;
  int status = 0;
  std::vector<int> cnt((size_t)W * E), own_off(E), src_off((size_t)W * E), T((size_t)V * E);
  // This rank's sizes as the count kernel clamps them.
  std::vector<int> gs(E);
  int64_t total = 0;
  for (int g = 0; g < E; ++g) {
    int c = counts[(size_t)rank * E + g];
    if (c < 0) {
      status |= kStatusBadGroupSize;
      c = 0;
    }
    c = (int64_t)c > M ? (int)M : c;
    gs[g] = c;
  }
  for (int g = 0; g < E; ++g) {  // exclusive prefix saturating at M, sizes cut to the room left
    own_off[g] = (int)std::min<int64_t>(total, M);
    total = std::min<int64_t>(total + gs[g], M);
    const int room = (int)(M - own_off[g]);
    if (gs[g] > room) {
      gs[g] = room;
      status |= kStatusRowsClamped;
    }
  }
  for (int s2 = 0; s2 < W; ++s2)
    for (int g = 0; g < E; ++g) {
      int c = s2 == rank ? gs[g] : counts[(size_t)s2 * E + g];
      cnt[(size_t)s2 * E + g] = c < 0 ? 0 : (c > max_rows ? max_rows : c);
    }
  for (int s2 = 0; s2 < W; ++s2) {
    int64_t run = 0;
    for (int g = 0; g < E; ++g) {
      src_off[(size_t)s2 * E + g] = (int)std::min<int64_t>(run, 0x7fffffff);
      run += cnt[(size_t)s2 * E + g];
    }
  }
  for (int v = 0; v < V; ++v)
    for (int g = 0; g < E; ++g) T[(size_t)v * E + g] = ep_wave_total(cnt.data(), W, E, V, v, g);
  for (int v = 0; v < V; ++v)
    for (int p2 = 0; p2 < W; ++p2)
      ep_owner_region(T.data() + (size_t)v * E, p2, EL, region_cap, p2 == rank ? local_gs + (size_t)v * EL : nullptr);
  for (int v = 0; v < V; ++v) {
    int64_t run = 0;
    for (int g = 0; g < E; ++g) {
      bool clamped;
      const EpSlice sl = ep_slice(cnt.data(), own_off.data(), T[(size_t)v * E + g], W, E, EL, V, rank, region_cap,
                                  v, g, &clamped);
      if (clamped) status |= kStatusRowsClamped;
      int32_t* o = slices + ((size_t)v * E + g) * 4;
      o[0] = sl.src_row;
      o[1] = sl.n;
      o[2] = sl.dst_row;
      o[3] = sl.owner;
      wave_rows[(size_t)v * (E + 1) + g] = (int)std::min<int64_t>(run, 0x7fffffff);
      run += sl.n;
    }
    wave_rows[(size_t)v * (E + 1) + E] = (int)std::min<int64_t>(run, 0x7fffffff);
  }
  if (recv)
    for (int e = 0; e < EL; ++e)
      for (int sr = 0; sr < W; ++sr) {
        const int4 r = ep_recv_entry(cnt.data(), local_gs, src_off.data(), W, E, EL, rank, region_cap, e, sr);
        int32_t* o = recv + ((size_t)e * W + sr) * 4;
        o[0] = r.x;
        o[1] = r.y;
        o[2] = r.z;
        o[3] = r.w;
      }
  return status;
}

int moe_describe_plan(int64_t M, int32_t D, int32_t F, int32_t E, int32_t dtype, int32_t sms, moe_launch_desc* out,
                      int32_t max_out) {
  t_err[0] = 0;
  if (M < 0 || D <= 0 || F <= 0 || E <= 0 || dtype < 0 || dtype > 2 || max_out < 0 || (max_out > 0 && !out))
    return fail(MOE_ERR_INVALID_ARG, "bad arguments M=%lld D=%d F=%d E=%d dtype=%d", (long long)M, D, F, E, dtype);
  if (sms <= 0) {
    int dev;
    DevInfo* di;
    if (int r = device_info(&dev, &di)) return r;
    sms = di->sms;
  }
  if (M == 0) return 0;
  moe_launch_desc d[4];
  int n = 0;
  const int prep_cap = sms * 4;
  const int ctas_req = (int)g_tune_ctas;
  if (!small_supported(D, F, dtype)) {
    if (!large_supported(D, F, dtype)) return fail(MOE_ERR_UNSUPPORTED_SHAPE, "D=%d F=%d dtype=%d", D, F, dtype);
    int pairs = sms / 2;
    if (ctas_req > 0 && ctas_req / 2 < pairs) pairs = ctas_req / 2 > 0 ? ctas_req / 2 : 1;
    if (dtype == MOE_DTYPE_F32) {
      const int wb = E * ((D + 31) / 32) * ((F + 31) / 32);
      const int xb = (int)std::min<int64_t>(((int64_t)M * D / 4 + 255) / 256, prep_cap);
      desc_set(&d[n++], "small_prep_kernel", 2 * wb + xb, 256, 32 * 33 * 4, 0, 1, 0, 0, 0, 0, MOE_MMA_NONE, 0, 0, 1, 0);
      desc_gemm<0, false, true>(&d[n++], "grouped_gemm_pair_kernel (up)", pairs, F, D);
      desc_gemm<1, false, true>(&d[n++], "grouped_gemm_pair_kernel (down)", pairs, D, F);
    } else if (dtype == MOE_DTYPE_FP8_E4M3_BLK128) {
      if (fp8_use_swap(M, E)) {
        desc_swap<0>(&d[n++], "grouped_gemm_swap_kernel (up)", pairs, F, D);
        desc_swap<1>(&d[n++], "grouped_gemm_swap_kernel (down)", pairs, D, F);
      } else {
        desc_gemm<0, true, false>(&d[n++], "grouped_gemm_pair_kernel (up)", pairs, F, D);
        desc_gemm<1, true, false>(&d[n++], "grouped_gemm_pair_kernel (down)", pairs, D, F);
      }
    } else {
      desc_gemm<0, false, false>(&d[n++], "grouped_gemm_pair_kernel (up)", pairs, F, D);
      if (down_wide()) desc_gemm<1, false, false, 2>(&d[n++], "grouped_gemm_pair_kernel (down)", pairs, D, F);
      else desc_gemm<1, false, false>(&d[n++], "grouped_gemm_pair_kernel (down)", pairs, D, F);
    }
  } else {
    const SmallPlan plan = small_plan(M, D, F, E, dtype);
    const int splits = small_splits(M, E, F / plan.bf, false, sms);
    const int ctas = ctas_req > 0 && ctas_req < sms ? ctas_req : sms;
    const bool f32 = dtype == MOE_DTYPE_F32;
    const int wb = f32 ? E * ((D + 31) / 32) * ((F + 31) / 32) : 0;
    const int xb = (f32 && !plan.x_res) ? (int)std::min<int64_t>(((int64_t)M * D / 4 + 255) / 256, prep_cap) : 0;
    const int yb = splits > 1 ? (int)std::min<int64_t>(((int64_t)M * D / 4 + 255) / 256, prep_cap) : 0;
    if (2 * wb + xb + yb > 0)
      desc_set(&d[n++], "small_prep_kernel", 2 * wb + xb + yb, 256, 32 * 33 * 4, 0, 1, 0, 0, 0, 0, MOE_MMA_NONE, 0,
               0, 1, 0);
    if (f32) {
      if (D == 64) desc_small<kModeTF32x3, 64, 64, true>(&d[n++], ctas, F, splits);
      else if (D == 128) desc_small<kModeTF32x3, 128, 64, true>(&d[n++], ctas, F, splits);
      else desc_small<kModeTF32x3, 256, 64, false>(&d[n++], ctas, F, splits);
    } else {
      if (D == 64) desc_small<kModeBF16, 64, 128, true>(&d[n++], ctas, F, splits);
      else if (D == 128) desc_small<kModeBF16, 128, 128, true>(&d[n++], ctas, F, splits);
      else desc_small<kModeBF16, 256, 128, true>(&d[n++], ctas, F, splits);
    }
  }
  for (int i = 0; i < n && i < max_out; ++i) out[i] = d[i];
  return n;
}

// ------------------------------------------------------------------ training
static int check_train_args(int64_t M, int32_t D, int32_t F, int32_t E) {
  if (M < 0 || D <= 0 || F <= 0 || E <= 0)
    return fail(MOE_ERR_INVALID_ARG, "bad sizes M=%lld D=%d F=%d E=%d", (long long)M, D, F, E);
  if (E > 4096) return fail(MOE_ERR_UNSUPPORTED_SHAPE, "E=%d exceeds 4096", E);
  if (M + 64LL * E > (int64_t)0x7fffffff) return fail(MOE_ERR_UNSUPPORTED_SHAPE, "M=%lld too large", (long long)M);
  if (!train_supported(D, F))
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "training entry points need D and F multiples of 256 (got D=%d F=%d)", D, F);
  return 0;
}

size_t moe_fused_mlp_forward_train_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E) {
  if (M < 0 || E <= 0 || !train_supported(D, F)) return 0;
  return large_ws_bytes(M, D, F, E, MOE_DTYPE_BF16);
}

int moe_fused_mlp_forward_train(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                                float* y, void* a_save, int64_t M, int32_t D, int32_t F, int32_t E, void* workspace,
                                size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (int r = check_train_args(M, D, F, E)) return r;
  if (M == 0) return 0;
  if (!x || !w_up || !w_down || !group_sizes || !y || !a_save) return fail(MOE_ERR_INVALID_ARG, "null operand pointer");
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(a_save)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "y and a_save must be 16-byte aligned");
  return run_train_forward(x, w_up, w_down, group_sizes, y, a_save, M, D, F, E, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream));
}

size_t moe_fused_mlp_backward_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E) {
  if (M < 0 || E <= 0 || E > 4096 || !train_supported(D, F)) return 0;
  return bwd_ws_bytes(M, D, F, E);
}

int moe_fused_mlp_backward(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                           const void* a_saved, const void* dy, int32_t dy_dtype, float* dx, float* dw_up,
                           float* dw_down, int64_t M, int32_t D, int32_t F, int32_t E, void* workspace,
                           size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (int r = check_train_args(M, D, F, E)) return r;
  if (dy_dtype != MOE_DTYPE_F32 && dy_dtype != MOE_DTYPE_BF16)
    return fail(MOE_ERR_UNSUPPORTED_DTYPE, "dy_dtype %d (f32 or bf16)", dy_dtype);
  if (!x || !w_up || !w_down || !group_sizes || !a_saved || !dy || !dx || !dw_up || !dw_down)
    return fail(MOE_ERR_INVALID_ARG, "null operand pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(a_saved) | reinterpret_cast<uintptr_t>(dy) |
       reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dw_up) | reinterpret_cast<uintptr_t>(dw_down)) &
      15u)
    return fail(MOE_ERR_MISALIGNED, "operands must be 16-byte aligned");
  return run_backward(x, w_up, w_down, group_sizes, a_saved, dy, dy_dtype, dx, dw_up, dw_down, M, D, F, E, workspace,
                      workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t moe_fused_mlp_swiglu_forward_train_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E) {
  if (M < 0 || E <= 0 || !train_supported(D, F)) return 0;
  return align256((size_t)M * F * 2);
}

int moe_fused_mlp_swiglu_forward_train(const void* x, const void* w_gate_up, const void* w_down,
                                       const int32_t* group_sizes, float* y, void* gu_save, int64_t M, int32_t D,
                                       int32_t F, int32_t E, void* workspace, size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (int r = check_train_args(M, D, F, E)) return r;
  if (M == 0) return 0;
  if (!x || !w_gate_up || !w_down || !group_sizes || !y || !gu_save)
    return fail(MOE_ERR_INVALID_ARG, "null operand pointer");
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(gu_save)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "y and gu_save must be 16-byte aligned");
  return run_swiglu_train_forward(x, w_gate_up, w_down, group_sizes, y, gu_save, M, D, F, E, workspace,
                                  workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t moe_fused_mlp_swiglu_backward_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E) {
  if (M < 0 || E <= 0 || E > 4096 || !train_supported(D, F)) return 0;
  return swiglu_bwd_ws_bytes(M, D, F, E);
}

int moe_fused_mlp_swiglu_backward(const void* x, const void* w_gate_up, const void* w_down,
                                  const int32_t* group_sizes, const void* gu_saved, const void* dy, int32_t dy_dtype,
                                  float* dx, float* dw_gate_up, float* dw_down, int64_t M, int32_t D, int32_t F,
                                  int32_t E, void* workspace, size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (int r = check_train_args(M, D, F, E)) return r;
  if (dy_dtype != MOE_DTYPE_F32 && dy_dtype != MOE_DTYPE_BF16)
    return fail(MOE_ERR_UNSUPPORTED_DTYPE, "dy_dtype %d (f32 or bf16)", dy_dtype);
  if (!x || !w_gate_up || !w_down || !group_sizes || !gu_saved || !dy || !dx || !dw_gate_up || !dw_down)
    return fail(MOE_ERR_INVALID_ARG, "null operand pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gu_saved) | reinterpret_cast<uintptr_t>(dy) |
       reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dw_gate_up) |
       reinterpret_cast<uintptr_t>(dw_down)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "operands must be 16-byte aligned");
  return run_swiglu_backward(x, w_gate_up, w_down, group_sizes, gu_saved, dy, dy_dtype, dx, dw_gate_up, dw_down, M, D,
                             F, E, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int moe_swiglu_interleave_fp8(const void* w_gate, const void* w_up, const float* s_gate, const float* s_up,
                              void* w_gate_up, float* s_gate_up, int32_t E, int32_t D, int32_t F, void* stream) {
  t_err[0] = 0;
  if (E <= 0 || D <= 0 || F <= 0 || D % 128 || F % 128)
    return fail(MOE_ERR_INVALID_ARG, "E=%d D=%d F=%d (D and F multiples of 128)", E, D, F);
  if (!w_gate || !w_up || !s_gate || !s_up || !w_gate_up || !s_gate_up) return fail(MOE_ERR_INVALID_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(w_gate) | reinterpret_cast<uintptr_t>(w_up) |
       reinterpret_cast<uintptr_t>(w_gate_up)) & 15u)
    return fail(MOE_ERR_MISALIGNED, "weights must be 16-byte aligned");
  int dev;
  DevInfo* di;
  if (int r = device_info(&dev, &di)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t rows = (size_t)E * D, n = rows * (size_t)(F / 8);
  const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)di->sms * 8);
  swiglu_interleave_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(w_gate), static_cast<const uint4*>(w_up),
                                                   static_cast<uint4*>(w_gate_up), rows, F / 16, 8);
  MOE_CUDA_TRY(cudaGetLastError());
  const size_t srows = (size_t)E * (D / 128);
  const int sblocks = (int)std::min<size_t>((srows * (2 * F / 128) + 255) / 256, (size_t)di->sms * 4);
  swiglu_interleave_scales_kernel<<<sblocks, 256, 0, st>>>(s_gate, s_up, s_gate_up, srows, F / 128);
  MOE_CUDA_TRY(cudaGetLastError());
  return 0;
}

size_t moe_fused_mlp_swiglu_fp8_workspace_size(int64_t M, int32_t D, int32_t F) {
  if (M < 0 || !swiglu_supported(D, F)) return 0;
  return swiglu_ws_bytes(M, D, F, true);
}

int moe_fused_mlp_swiglu_fp8(const void* x, const void* w_gate_up, const void* w_down, const float* s_gate_up,
                             const float* s_down, const int32_t* group_sizes, float* y, int64_t M, int32_t D,
                             int32_t F, int32_t E, void* workspace, size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (M < 0 || D <= 0 || F <= 0 || E <= 0)
    return fail(MOE_ERR_INVALID_ARG, "bad sizes M=%lld D=%d F=%d E=%d", (long long)M, D, F, E);
  if (M > (int64_t)0x7fffffff) return fail(MOE_ERR_UNSUPPORTED_SHAPE, "M=%lld exceeds 2^31-1", (long long)M);
  if (!swiglu_supported(D, F))
    return fail(MOE_ERR_UNSUPPORTED_SHAPE, "SwiGLU experts need D %% 256 == 0 (D >= 256) and F %% 128 == 0");
  if (M == 0) return 0;
  if (!x || !w_gate_up || !w_down || !s_gate_up || !s_down || !group_sizes || !y)
    return fail(MOE_ERR_INVALID_ARG, "null operand pointer");
  if (reinterpret_cast<uintptr_t>(y) & 15u) return fail(MOE_ERR_MISALIGNED, "y must be 16-byte aligned");
  return run_swiglu(x, w_gate_up, w_down, s_gate_up, s_down, group_sizes, y, M, D, F, E, true, workspace,
                    workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
