// Fused expert MLP for small model dimension (D <= 256), sm_100a.
//
// One CTA per SM walks a static round-robin share of the real work units
// (expert e, 128-row block b, F-split s) -- there is no padded grid: units
// are enumerated from the device-resident group sizes, so an expert with
// zero tokens costs nothing and the last block of an expert is row-masked
// (reference kernel src/kernel.py:9-82, grid src/kernel.py:104-107).
//
// Per unit and per BF-wide chunk j of the hidden dimension F:
//   MMA1 (tcgen05, A = X tile in smem, B = W_up chunk in smem)
//        H_acc[j % 2] (TMEM, f32)  = X(128 x D) @ W_up[e][:, chunk j]
//   GELU warps: TMEM -> registers -> tanh-GELU -> TMEM operand
//        (bf16 pairs, or tf32 hi + lo planes for the 3xTF32 path)
//   MMA2 (tcgen05 with A read from TMEM, B = W_down chunk in smem)
//        Y_acc (TMEM, f32) += H(128 x BF) @ W_down[e][chunk j, :]
// The (128, BF) hidden block never leaves the SM.  MMA1 of chunk j+1 is
// issued before MMA2 of chunk j so the GELU of one chunk overlaps the tensor
// core work of the next.  After the last chunk the epilogue warps drain Y_acc
// to global memory with a row mask (or reduce-add it when F is split across
// CTAs).
//
// Precision modes:
//   kModeBF16  : bf16 X / W, f32 accumulate, bf16 hidden operand.
//   kModeTF32x3: f32 X / W.  Every product a*b is evaluated as
//                a_hi*b_hi + a_hi*b_lo + a_lo*b_hi with a_hi = a rounded
//                to the nearest tf32 value and a_lo = a - a_hi, which
//                keeps the result within ~1e-6 relative of f32 math.
//                Weights arrive pre-split (hi/lo planes, transposed to
//                K-major).  With a resident X tile (D <= 128) the GELU warps
//                split X in place: X_hi stays in shared memory and X_lo goes
//                to TMEM, where MMA1 reads it as an A operand; this keeps
//                shared memory for a deeper weight ring.  For D = 256 X is
//                pre-split and streamed with the weights.
//
// Warp roles (320 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2..9 GELU / epilogue (two warps per TMEM lane quadrant, each
// taking half of the columns).
#pragma once
#include "ptx.cuh"

namespace moe {

enum : int { kModeBF16 = 0, kModeTF32x3 = 1 };

constexpr int kMaxSmemPerBlock = 232448;  // 227 KB opt-in limit on sm_100

struct FusedParams {
  const int32_t* group_sizes;  // (E,) device, int32
  float* y;                    // (M, D) f32
  int M;
  int E;
  int F;
  int splits;                 // F-splits per 128-row block
  int chunks_per_split;       // BF-wide chunks handled by one unit
  int atomic_out;             // 1: Y was zeroed, units reduce-add into it
  int* status;                // device status word (kStatus* bits)
  unsigned long long* trace;  // MOE_TRACE builds: per-CTA event timeline (else unused)
  int skip_tail;              // 1: leave rows at or past sum(group_sizes) unwritten
  int tail_halves;            // 1: a last partial wave of at most half the grid runs as half units
};

// Work units of the fused kernel.  Unit u of the persistent grid (CTA c takes
// u = c, c + G, ...) is normally (128-row block u / S, F-split u % S) with NCH
// hidden chunks.  When the units do not fill the last wave and that wave
// would hold at most G / 2 of them, each of those last units is split into
// two halves of NCH / 2 chunks that run on two CTAs and reduce-add into Y
// (rows zeroed up front).  Two partial sums added onto zero give the same
// bits in either order, so results stay deterministic.
struct SmallUnits {
  int full;    // units [0, full) are whole
  int halves;  // 2: units from `full` on are halves; 1: none
};
// Block count of the routing (the same clamping as BlockCursorT).
__device__ __forceinline__ int small_block_count(const int32_t* gs, int E, int M, int shift = 7) {
  int nb = 0, row = 0;
  for (int e = 0; e < E; ++e) {
    int g = __ldg(gs + e);
    g = g < 0 ? 0 : g;
    const int rem = M - row;
    g = g > rem ? (rem > 0 ? rem : 0) : g;
    row += g;
    nb += (g + (1 << shift) - 1) >> shift;
  }
  return nb;
}
// The same count by a whole warp: 32 group sizes per load, the running total
// (clamped at M) from a warp scan -- one memory round trip per 32 experts
// instead of one per expert.  Every lane returns the count.
__device__ __forceinline__ int small_block_count_warp(const int32_t* gs, int E, int M, uint32_t lane) {
  int nb = 0;
  long long row = 0;  // unclamped running total of the earlier experts
  for (int e0 = 0; e0 < E; e0 += 32) {
    int g = e0 + (int)lane < E ? __ldg(gs + e0 + lane) : 0;
    g = g < 0 ? 0 : (g > M ? M : g);
    long long incl = g;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long t = __shfl_up_sync(0xffffffffu, incl, o);
      if ((int)lane >= o) incl += t;
    }
    // clamping the running total at M (as BlockCursorT does) leaves M - prefix
    // rows for this expert, at least 0
    const long long rem = (long long)M - (row + incl - g);
    const int gc = (long long)g > rem ? (rem > 0 ? (int)rem : 0) : g;
    int n = (gc + 127) >> 7;
#pragma unroll
    for (int o = 16; o; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
    nb += n;
    row += __shfl_sync(0xffffffffu, incl, 31);
  }
  return nb;
}
__device__ __forceinline__ SmallUnits small_units_from(int nb, int splits, int nch, int grid, int tail_halves) {
  const int u0 = nb * splits;
  const int full = (u0 / grid) * grid;
  const int tail = u0 - full;
  if (tail_halves && tail > 0 && 2 * tail <= grid && nch % 2 == 0) return {full, 2};
  return {u0, 1};
}
__device__ __forceinline__ SmallUnits small_units(const int32_t* gs, int E, int M, int splits, int nch, int grid,
                                                  int tail_halves) {
  return small_units_from(small_block_count(gs, E, M), splits, nch, grid, tail_halves);
}
// First row of global 128-row block `block`; the routed row count when the
// block is past the last one.
__device__ __forceinline__ int small_block_row(const int32_t* gs, int E, int M, int block) {
  int nb = 0, row = 0;
  for (int e = 0; e < E; ++e) {
    int g = __ldg(gs + e);
    g = g < 0 ? 0 : g;
    const int rem = M - row;
    g = g > rem ? (rem > 0 ? rem : 0) : g;
    const int n = (g + 127) >> 7;
    if (block < nb + n) return row + (block - nb) * 128;
    nb += n;
    row += g;
  }
  return row;
}
struct UnitWork {
  int gb;      // global 128-row block
  int fch0;    // first hidden chunk
  int nch;     // hidden chunks
  bool atomic; // reduce-add into Y
};
__device__ __forceinline__ UnitWork unit_work(int u, SmallUnits su, int S, int NCH, bool atomic_out) {
  if (u < su.full) return {u / S, (u % S) * NCH, NCH, atomic_out};
  const int v = u - su.full;
  const int w = su.full + v / su.halves;
  const int n = NCH / su.halves;
  return {w / S, (w % S) * NCH + (v % su.halves) * n, n, atomic_out || su.halves > 1};
}

// Optional timeline of pipeline events (clock64 per event) for CTA-level
// analysis; compiled in only with -DMOE_TRACE.  Layout per CTA: 4 rows
// (producer, MMA stage waits, GELU warp, MMA hidden waits) of kTraceLen.
constexpr int kTraceLen = 256;
#ifdef MOE_TRACE
#define MOE_TRACE_EV(row, idx)                                                    \
  do {                                                                            \
    if (p.trace && (idx) < kTraceLen)                                             \
      p.trace[((size_t)blockIdx.x * 4 + (row)) * kTraceLen + (idx)] = clock64(); \
  } while (0)
#else
#define MOE_TRACE_EV(row, idx) \
  do {                         \
  } while (0)
#endif

template <int MODE, int D, int BF, bool X_RES>
struct FusedCfg {
  static constexpr bool kTF32 = MODE == kModeTF32x3;
  static constexpr int ESZ = kTF32 ? 4 : 2;
  static constexpr int ATOM = 128 / ESZ;  // elements in one 128-byte swizzle row
  static constexpr int KI = 32 / ESZ;     // K of one MMA instruction
  static constexpr int PL = kTF32 ? 2 : 1;
  static constexpr bool XLO_TMEM = kTF32 && X_RES;  // X_lo lives in TMEM
  static constexpr int BM = 128;
  static constexpr int XBOX = BM * 128;                        // one X k-box: 128 rows x 128 B
  static constexpr int X_PLANE = (D / ATOM) * XBOX;            // one full X plane
  static constexpr int X_BYTES = X_RES ? X_PLANE : 0;          // resident X (bf16, or tf32 hi)
  // MMA1 stage: KB1 k-boxes, each [streamed X planes][W_up planes].
  static constexpr int KB1 = (kTF32 && X_RES) ? 2 : 1;
  static constexpr int S1_X = X_RES ? 0 : PL * XBOX;
  static constexpr int S1_WPLANE = BF * 128;  // one W_up plane of one k-box
  static constexpr int S1_SUB = S1_X + PL * S1_WPLANE;
  static constexpr int S1_BYTES = KB1 * S1_SUB;
  static constexpr int SK1 = KB1 * ATOM;      // K rows per MMA1 stage
  // MMA2 stage: one k-box of W_down planes.
  static constexpr int S2_WPLANE = D * 128;
  static constexpr int S2_BYTES = PL * S2_WPLANE;
  static constexpr int SK2 = ATOM;
  static constexpr int STAGE = S1_BYTES > S2_BYTES ? S1_BYTES : S2_BYTES;
  static constexpr int N1 = D / SK1;   // ring stages per MMA1 chunk
  static constexpr int N2 = BF / SK2;  // ring stages per MMA2 chunk
  static constexpr int BAR_BYTES = 256;
  static constexpr int Y_STAGE = 8 * 32 * 32 * 4;  // 4 KB per epilogue warp for coalesced Y stores
  static constexpr int NS_FIT = (kMaxSmemPerBlock - 1024 - BAR_BYTES - X_BYTES - Y_STAGE) / STAGE;
  static constexpr int NS = NS_FIT > 8 ? 8 : NS_FIT;
  static constexpr int SMEM = 1024 + X_BYTES + NS * STAGE + Y_STAGE + BAR_BYTES;
  static_assert((2 * NS + 9) * 8 + 4 * 4 <= BAR_BYTES, "barriers, TMEM slot, abort flag and unit plan");
  // TMEM columns: Y accumulator [0, D); hidden buffer b at D + b * HCOLS
  // (accumulator / hi plane first, lo plane after it); X_lo after both.
  static constexpr int HCOLS = PL * BF;
  static constexpr int XLO_COL = D + 2 * HCOLS;
  static constexpr int TMEM_USED = XLO_COL + (XLO_TMEM ? D : 0);
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t FMT = kTF32 ? kFmtTF32 : kFmtBF16;
  static constexpr uint32_t B_MN = kTF32 ? 0u : 1u;  // bf16 weights are read MN-major
  // 3xTF32 MMA1 reads the hi and lo W_up planes (adjacent in the stage) as
  // one N = 2*BF operand: D[:, 0:BF] += Xhi*Whi, D[:, BF:2BF] += Xhi*Wlo,
  // then D[:, 0:BF] += Xlo*Whi; the GELU warps add the two halves.
  static constexpr uint32_t IDESC1 = make_idesc(FMT, 128, kTF32 ? 2 * BF : BF, 0, B_MN);
  static constexpr uint32_t IDESC1_LO = make_idesc(FMT, 128, BF, 0, B_MN);
  static constexpr uint32_t IDESC2 = make_idesc(FMT, 128, D, 0, B_MN);
  static constexpr int EPI_WARPS = 8;  // two per TMEM lane quadrant
  static constexpr int EPI_THREADS = EPI_WARPS * 32;
  static constexpr int THREADS = 64 + EPI_THREADS;
  static constexpr uint32_t TX1 = S1_BYTES;
  static constexpr uint32_t TX2 = S2_BYTES;

  static_assert(NS >= 2, "shared memory too small for two ring stages");
  static_assert(D % SK1 == 0 && BF % SK2 == 0, "tile shape");
  static_assert(TMEM_USED <= TMEM_COLS, "TMEM budget");
  static_assert(!kTF32 || 2 * BF <= 256, "concatenated MMA1 N");
  static_assert(D % 16 == 0 && D <= 256 && BF % 16 == 0 && BF <= 256, "UMMA N range");
  static_assert(SMEM <= kMaxSmemPerBlock, "shared memory budget");
};

// Monotone walk over (expert, block) pairs built from group sizes; a block
// is 2^SHIFT rows (128 for one CTA, 256 for a CTA pair).
template <int SHIFT>
struct BlockCursorT {
  int e = -1;
  int blk_begin = 0;
  int nblk = 0;
  int row_begin = 0;
  int rows = 0;

  // Moves to the expert that owns global block `gb`; false when past the end.
  __device__ __forceinline__ bool seek(int gb, const int32_t* gs, int E, int M) {
    while (gb >= blk_begin + nblk) {
      blk_begin += nblk;
      row_begin += rows;
      if (++e >= E) return false;
      int g = __ldg(gs + e);
      g = g < 0 ? 0 : g;
      const int rem = M - row_begin;
      g = g > rem ? (rem > 0 ? rem : 0) : g;
      rows = g;
      nblk = (g + (1 << SHIFT) - 1) >> SHIFT;
    }
    return true;
  }
};
using BlockCursor = BlockCursorT<7>;

// Drains a 32-row x 32-column block of Y (this warp's TMEM lanes) to global
// memory.  tcgen05.ld gives each thread one row; the block goes through a
// per-warp 4 KB shared-memory tile (16-byte chunks XOR-swizzled by row, so
// both the writes and the reads are bank-conflict free) and leaves as
// row-contiguous 128-byte stores, masked per row at the expert's end.
template <int D>
// Columns at or past `col_end` (relative to `y`, like c0) are not stored.
__device__ __forceinline__ void store_y_block(uint32_t taddr, float4* stage, float* y, int row_base, int row_end,
                                              int c0, uint32_t lane, bool atomic, int ld = D, int col_end = 1 << 30) {
  uint32_t v[32];
  tmem_ld32(taddr, v);
  tmem_ld_wait();
#pragma unroll
  for (int k = 0; k < 8; ++k)
    stage[lane * 8 + (k ^ (lane & 7))] = make_float4(__uint_as_float(v[4 * k]), __uint_as_float(v[4 * k + 1]),
                                                     __uint_as_float(v[4 * k + 2]), __uint_as_float(v[4 * k + 3]));
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (int)(lane >> 3);
    const int k = (int)(lane & 7);
    const float4 val = stage[r * 8 + (k ^ (r & 7))];
    const int row = row_base + r;
    if (row < row_end && c0 + 4 * k < col_end) {
      float* dst = y + (size_t)row * ld + c0 + 4 * k;
      if (atomic)
        red_add_v4(dst, val.x, val.y, val.z, val.w);
      else
        *reinterpret_cast<float4*>(dst) = val;
    }
  }
  __syncwarp();
}

struct FusedMaps {
  CUtensorMap x[2];   // X (raw, or pre-split hi / lo planes when streamed)
  CUtensorMap wu[2];  // W_up operand planes
  CUtensorMap wd[2];  // W_down operand planes
};

template <int MODE, int D, int BF, bool X_RES>
__global__ void __launch_bounds__(64 + 256, 1)
    fused_mlp_small_kernel(const __grid_constant__ FusedMaps maps, const FusedParams p) {
  using C = FusedCfg<MODE, D, BF, X_RES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* xbuf = smem;
  uint8_t* ring = smem + C::X_BYTES;
  float4* ystage = reinterpret_cast<float4*>(ring + C::NS * C::STAGE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + C::NS * C::STAGE + C::Y_STAGE);
  uint64_t* full = bars;                // [NS]
  uint64_t* empty = bars + C::NS;       // [NS]
  uint64_t* x_full = bars + 2 * C::NS;  // raw X landed
  uint64_t* x_ready = x_full + 1;       // X operand (split) ready for MMA
  uint64_t* x_empty = x_full + 2;       // last MMA1 of the unit finished
  uint64_t* h_full = x_full + 3;        // [2] MMA1 done -> GELU
  uint64_t* h_ready = x_full + 5;       // [2] GELU operand written -> MMA2
  uint64_t* y_full = x_full + 7;        // last MMA2 done -> epilogue
  uint64_t* y_empty = x_full + 8;       // epilogue drained Y_acc
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_full + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* plan_smem = reinterpret_cast<int*>(tmem_slot + 2);  // SmallUnits of this launch

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (warp == 0) {
    const int nb = small_block_count_warp(p.group_sizes, p.E, p.M, lane);
    if (lane == 0) {
      const SmallUnits su0 = small_units_from(nb, p.splits, p.chunks_per_split, (int)gridDim.x, p.tail_halves);
      plan_smem[0] = su0.full;
      plan_smem[1] = su0.halves;
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_ready, C::EPI_THREADS);
    mbar_init(x_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(h_full + i, 1);
      mbar_init(h_ready + i, C::EPI_THREADS);
    }
    mbar_init(y_full, 1);
    mbar_init(y_empty, C::EPI_THREADS);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.x[0]);
    tma_prefetch_desc(&maps.wu[0]);
    tma_prefetch_desc(&maps.wd[0]);
    if (C::kTF32) {
      tma_prefetch_desc(&maps.wu[1]);
      tma_prefetch_desc(&maps.wd[1]);
      if (!X_RES) tma_prefetch_desc(&maps.x[1]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int S = p.splits;
  const int NCH = p.chunks_per_split;
  const SmallUnits su{plan_smem[0], plan_smem[1]};
  const bool atomic_all = p.atomic_out != 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      BlockCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ui = 0;
      bool ok = true;
      const uint64_t pol_w = l2_policy_evict_last();
      int tp = 0;
      auto next_stage = [&]() -> bool {
        if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, p.status)) return false;
        MOE_TRACE_EV(0, tp);
        ++tp;
        return true;
      };
      auto advance = [&]() {
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int u = blockIdx.x; ok; u += gridDim.x, ++ui) {
        const UnitWork uw = unit_work(u, su, S, NCH, atomic_all);
        const int gb = uw.gb;
        if (!cur.seek(gb, p.group_sizes, p.E, p.M)) break;
        const int e = cur.e;
        const int row0 = cur.row_begin + (gb - cur.blk_begin) * C::BM;
        const int fch0 = uw.fch0;
        const int nch = uw.nch;
        if constexpr (X_RES) {
          if (!mbar_wait(x_empty, (ui & 1u) ^ 1u, abort_flag, p.status)) break;
          // Raw X (the bf16 operand, or f32 split in place by the GELU warps).
          mbar_arrive_expect_tx(x_full, C::X_PLANE);
          for (int s = 0; s < D / C::ATOM; ++s)
            tma_load_2d(xbuf + s * C::XBOX, &maps.x[0], x_full, s * C::ATOM, row0);
        }
        auto load_s1 = [&](int j, int s) -> bool {
          if (!next_stage()) return false;
          uint8_t* st = ring + stage * C::STAGE;
          mbar_arrive_expect_tx(full + stage, C::TX1);
          const int f0 = (fch0 + j) * BF;
          for (int kb = 0; kb < C::KB1; ++kb) {
            const int k0 = s * C::SK1 + kb * C::ATOM;  // first d of this k-box
            uint8_t* sub = st + kb * C::S1_SUB;
            if constexpr (!X_RES) {
              for (int pl = 0; pl < C::PL; ++pl)
                tma_load_2d(sub + pl * C::XBOX, &maps.x[pl], full + stage, k0, row0);
            }
            uint8_t* w = sub + C::S1_X;
            if constexpr (C::kTF32) {
              // W_up^T planes: rows (e, f), K = d contiguous; box {32, BF}.
              for (int pl = 0; pl < C::PL; ++pl)
                tma_load_2d_hint(w + pl * C::S1_WPLANE, &maps.wu[pl], full + stage, k0, e * p.F + f0, pol_w);
            } else {
              // W_up rows (e, d), N = f contiguous; box {64, 64} per 64-wide f block.
              for (int nb = 0; nb < BF / C::ATOM; ++nb)
                tma_load_2d_hint(w + nb * C::ATOM * 128, &maps.wu[0], full + stage, f0 + nb * C::ATOM, e * D + k0,
                                 pol_w);
            }
          }
          advance();
          return true;
        };
        auto load_s2 = [&](int j, int t) -> bool {
          if (!next_stage()) return false;
          uint8_t* st = ring + stage * C::STAGE;
          mbar_arrive_expect_tx(full + stage, C::TX2);
          const int f0 = (fch0 + j) * BF + t * C::SK2;
          if constexpr (C::kTF32) {
            // W_down^T planes: rows (e, d), K = f contiguous; box {32, D}.
            for (int pl = 0; pl < C::PL; ++pl)
              tma_load_2d_hint(st + pl * C::S2_WPLANE, &maps.wd[pl], full + stage, f0, e * D, pol_w);
          } else {
            // W_down rows (e, f), N = d contiguous; box {64, 64} per 64-wide d block.
            for (int nb = 0; nb < D / C::ATOM; ++nb)
              tma_load_2d_hint(st + nb * C::SK2 * 128, &maps.wd[0], full + stage, nb * C::ATOM, e * p.F + f0,
                               pol_w);
          }
          advance();
          return true;
        };
        for (int j = 0; j < nch && ok; ++j) {
          for (int s = 0; s < C::N1 && ok; ++s) ok = load_s1(j, s);
          if (j > 0)
            for (int t = 0; t < C::N2 && ok; ++t) ok = load_s2(j - 1, t);
          if constexpr (X_RES) {
            // Warm L2 with the next unit's X tile so that its load at the end
            // of this unit does not wait on HBM.  Issued after the unit's
            // first stages: finding the next unit walks the group sizes.
            if (j == 0 && ok) {
              BlockCursor nxt = cur;
              const int gb_next = unit_work(u + (int)gridDim.x, su, S, NCH, atomic_all).gb;
              if (nxt.seek(gb_next, p.group_sizes, p.E, p.M)) {
                const int nrow0 = nxt.row_begin + (gb_next - nxt.blk_begin) * C::BM;
                for (int s = 0; s < D / C::ATOM; ++s) tma_prefetch_l2_2d(&maps.x[0], s * C::ATOM, nrow0);
              }
            }
          }
        }
        for (int t = 0; t < C::N2 && ok; ++t) ok = load_s2(nch - 1, t);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp)
    {
      BlockCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ui = 0;
      uint32_t hcount = 0;  // hidden chunks issued (selects the TMEM buffer)
      bool ok = true;
      const uint32_t t_y = tmem_base;
      int tm = 0;
      auto wait_full = [&]() -> bool {
        MOE_TRACE_EV(1, 2 * tm);
        if (!mbar_wait_warp(full + stage, phase, abort_flag, p.status)) return false;
        tc_fence_after();
        MOE_TRACE_EV(1, 2 * tm + 1);
        ++tm;
        return true;
      };
      auto release = [&]() {
        umma_commit(empty + stage);
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int u = blockIdx.x; ok; u += gridDim.x, ++ui) {
        const UnitWork uw = unit_work(u, su, S, NCH, atomic_all);
        const int nch = uw.nch;
        if (!cur.seek(uw.gb, p.group_sizes, p.E, p.M)) break;
        if constexpr (X_RES) {
          if (!mbar_wait_warp(x_ready, ui & 1u, abort_flag, p.status)) break;
          tc_fence_after();
        }
        // Descriptor start addresses advance in 16-byte units: adding
        // (bytes >> 4) to a descriptor moves its operand within the 14-bit
        // address field (all offsets here stay inside one stage / X tile).
        const uint64_t x_desc0 = make_sdesc(smem_u32(xbuf), 16, 1024);
        auto mma1 = [&](int j) -> bool {
          const uint32_t hb = (hcount + j) & 1u;
          const uint32_t d_tmem = tmem_base + D + hb * C::HCOLS;
          for (int s = 0; s < C::N1; ++s) {
            if (!wait_full()) return false;
            const uint32_t st = smem_u32(ring + stage * C::STAGE);
            const uint64_t st_desc = C::kTF32 ? make_sdesc(st, 16, 1024) : make_sdesc(st, C::ATOM * 128, 1024);
#pragma unroll
            for (int kb = 0; kb < C::KB1; ++kb) {
              const int kbox = s * C::KB1 + kb;  // k-box index along D
#pragma unroll
              for (int ki = 0; ki < C::ATOM / C::KI; ++ki) {
                const uint64_t a0 = X_RES ? x_desc0 + (uint64_t)((kbox * C::XBOX + ki * 32) >> 4)
                                          : st_desc + (uint64_t)((kb * C::S1_SUB + ki * 32) >> 4);
                const uint64_t b0 =
                    C::kTF32 ? st_desc + (uint64_t)((kb * C::S1_SUB + C::S1_X + ki * 32) >> 4)
                             : st_desc + (uint64_t)((kb * C::S1_SUB + C::S1_X + ki * (C::KI * 128)) >> 4);
                const uint32_t acc0 = (kbox > 0 || ki > 0) ? 1u : 0u;
                umma_ss<C::kTF32 ? Kind::TF32 : Kind::F16>(d_tmem, a0, b0, C::IDESC1, acc0);
                if constexpr (C::XLO_TMEM) {
                  const uint32_t xlo = tmem_base + C::XLO_COL + kbox * C::ATOM + ki * C::KI;
                  umma_ts<Kind::TF32>(d_tmem, xlo, b0, C::IDESC1_LO, 1u);
                } else if constexpr (C::kTF32) {
                  const uint64_t a1 = st_desc + (uint64_t)((kb * C::S1_SUB + C::XBOX + ki * 32) >> 4);
                  umma_ss<Kind::TF32>(d_tmem, a1, b0, C::IDESC1_LO, 1u);
                }
              }
            }
            release();
          }
          umma_commit(h_full + hb);
          return true;
        };
        auto mma2 = [&](int j) -> bool {
          const uint32_t hb = (hcount + j) & 1u;
          const uint32_t use = (hcount + j) >> 1;  // uses of this buffer so far
          MOE_TRACE_EV(3, (int)(2 * (hcount + j)));
          if (!mbar_wait_warp(h_ready + hb, use & 1u, abort_flag, p.status)) return false;
          tc_fence_after();
          MOE_TRACE_EV(3, (int)(2 * (hcount + j) + 1));
          if (j == 0) {
            if (!mbar_wait_warp(y_empty, (ui & 1u) ^ 1u, abort_flag, p.status)) return false;
            tc_fence_after();
          }
          const uint32_t h_tmem = tmem_base + D + hb * C::HCOLS;
          for (int t = 0; t < C::N2; ++t) {
            if (!wait_full()) return false;
            const uint32_t st = smem_u32(ring + stage * C::STAGE);
            const uint64_t st_desc = C::kTF32 ? make_sdesc(st, 16, 1024) : make_sdesc(st, C::SK2 * 128, 1024);
#pragma unroll
            for (int ki = 0; ki < C::SK2 / C::KI; ++ki) {
              const uint32_t kcol = (t * C::SK2 + ki * C::KI) * C::ESZ / 4;
              const uint64_t b0 = C::kTF32 ? st_desc + (uint64_t)((ki * 32) >> 4)
                                           : st_desc + (uint64_t)((ki * (C::KI * 128)) >> 4);
              const uint32_t acc0 = (j > 0 || t > 0 || ki > 0) ? 1u : 0u;
              umma_ts<C::kTF32 ? Kind::TF32 : Kind::F16>(t_y, h_tmem + kcol, b0, C::IDESC2, acc0);
              if constexpr (C::kTF32) {
                const uint64_t b1 = st_desc + (uint64_t)((C::S2_WPLANE + ki * 32) >> 4);
                umma_ts<Kind::TF32>(t_y, h_tmem + kcol, b1, C::IDESC2, 1u);
                umma_ts<Kind::TF32>(t_y, h_tmem + BF + kcol, b0, C::IDESC2, 1u);
              }
            }
            release();
          }
          return true;
        };
        for (int j = 0; j < nch && ok; ++j) {
          ok = mma1(j);
          if (ok && X_RES && j == nch - 1) umma_commit(x_empty);
          if (ok && j > 0) ok = mma2(j - 1);
        }
        if (ok) ok = mma2(nch - 1);
        if (ok) umma_commit(y_full);
        hcount += nch;
      }
    }
  } else {
    // ------------------------------------------------------------ GELU / epilogue warps
    const uint32_t q = warp & 3u;            // TMEM lane quadrant this warp may access
    const uint32_t half = (warp - 2u) >> 2;  // which half of the columns
    const uint32_t lane_base = tmem_base + ((q * 32u) << 16);
    const int erow = (int)(q * 32u + lane);  // row inside the 128-row block
    const int etid = (int)threadIdx.x - 64;  // 0..EPI_THREADS-1
    constexpr int NT = C::EPI_THREADS;

    if (etid == 0 && blockIdx.x == 0) {
      for (int e = 0; e < p.E; ++e)
        if (__ldg(p.group_sizes + e) < 0) atomicOr(p.status, kStatusBadGroupSize);
    }
    // Rows at or past sum(group_sizes) are zero in ragged_dot; write them
    // here unless Y was zeroed up front (reduce-add mode).
    if (!p.atomic_out && !p.skip_tail) {
      int total = 0;
      for (int e = 0; e < p.E; ++e) {
        int g = __ldg(p.group_sizes + e);
        total += g < 0 ? 0 : g;
        if (total >= p.M) {
          total = p.M;
          break;
        }
      }
      const size_t n4 = (size_t)(p.M - total) * D / 4;
      float4* base = reinterpret_cast<float4*>(p.y + (size_t)total * D);
      for (size_t i = (size_t)blockIdx.x * NT + etid; i < n4; i += (size_t)gridDim.x * NT)
        base[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    BlockCursor cur;
    uint32_t hcount = 0;
    uint32_t ui = 0;
    bool ok = true;
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
      bool r = mbar_wait(bar, parity, abort_flag, p.status);
      r = __all_sync(0xffffffffu, r);
      return r;
    };
    // Split of the resident f32 X tile: hi = x rounded to tf32 (tf32_hi_bits),
    // written back in place (shared memory, swizzled K-major layout); lo =
    // x - hi, written to this thread's TMEM lane as MMA1's second A operand.
    // Each thread owns one row and half of its D columns.
    auto split_x = [&](uint32_t uidx) -> bool {
      if (!warp_wait(x_full, uidx & 1u)) return false;
      const uint32_t rsw = (uint32_t)erow & 7u;
#pragma unroll 1
      for (int k0 = half * (D / 2); k0 < (int)(half + 1) * (D / 2); k0 += 32) {
        uint8_t* rowp = xbuf + (k0 / C::ATOM) * C::XBOX + erow * 128;
        uint32_t lo[32];
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          float4* ptr = reinterpret_cast<float4*>(rowp + ((g ^ rsw) << 4));
          float4 v = *ptr;
          float4 h;
          h.x = __uint_as_float(tf32_hi_bits(__float_as_uint(v.x)));
          h.y = __uint_as_float(tf32_hi_bits(__float_as_uint(v.y)));
          h.z = __uint_as_float(tf32_hi_bits(__float_as_uint(v.z)));
          h.w = __uint_as_float(tf32_hi_bits(__float_as_uint(v.w)));
          lo[4 * g + 0] = __float_as_uint(v.x - h.x);
          lo[4 * g + 1] = __float_as_uint(v.y - h.y);
          lo[4 * g + 2] = __float_as_uint(v.z - h.z);
          lo[4 * g + 3] = __float_as_uint(v.w - h.w);
          *ptr = h;
        }
        tmem_st32(lane_base + C::XLO_COL + k0, lo);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(x_ready);
      return true;
    };
    auto pass_x = [&](uint32_t uidx) -> bool {  // bf16: raw X is the operand
      if (!warp_wait(x_full, uidx & 1u)) return false;
      mbar_arrive(x_ready);
      return true;
    };

    int u = blockIdx.x;
    UnitWork uw = unit_work(u, su, S, NCH, atomic_all);
    bool have = cur.seek(uw.gb, p.group_sizes, p.E, p.M);
    if (have && X_RES) ok = C::kTF32 ? split_x(0) : pass_x(0);
    while (have && ok) {
      const int gb = uw.gb;
      const int nch = uw.nch;
      const int row0 = cur.row_begin + (gb - cur.blk_begin) * C::BM;
      const int row_end = cur.row_begin + cur.rows;
      // Hidden chunks: TMEM accumulator -> GELU -> MMA2 operand.
      for (int j = 0; j < nch && ok; ++j) {
        const uint32_t hb = (hcount + j) & 1u;
        const uint32_t use = (hcount + j) >> 1;
        if (!warp_wait(h_full + hb, use & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (warp == 2 && lane == 0) MOE_TRACE_EV(2, (int)(2 * (hcount + j)));
        const uint32_t hcol = D + hb * C::HCOLS;
        if constexpr (C::kTF32) {
          // Columns [half*BF/2, +BF/2): sum the two MMA1 halves, GELU, split.
#pragma unroll 1
          for (int c0 = half * (BF / 2); c0 < (int)(half + 1) * (BF / 2); c0 += 32) {
            uint32_t a[32], b[32];
            tmem_ld32(lane_base + hcol + c0, a);
            tmem_ld32(lane_base + hcol + BF + c0, b);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i += 2) gelu_split_tf32x2(a[i], a[i + 1], b[i], b[i + 1]);
            tmem_st32(lane_base + hcol + c0, a);
            tmem_st32(lane_base + hcol + BF + c0, b);
          }
        } else {
          // The packed bf16 operand overwrites the accumulator columns, so
          // both warps of a quadrant finish reading before either writes.
          constexpr int CW = BF / 2;  // accumulator columns per warp
          uint32_t v[CW];
#pragma unroll
          for (int c = 0; c < CW; c += 32)
            tmem_ld32(lane_base + hcol + half * CW + c, *reinterpret_cast<uint32_t(*)[32]>(v + c));
          tmem_ld_wait();
          asm volatile("bar.sync %0, 64;" ::"r"(1 + (int)q) : "memory");
#pragma unroll
          for (int c = 0; c < CW; c += 32) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = pack_bf16x2(gelu_tanh_fast(__uint_as_float(v[c + 2 * i])),
                                  gelu_tanh_fast(__uint_as_float(v[c + 2 * i + 1])));
            tmem_st16(lane_base + hcol + (half * CW + c) / 2, pk);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(h_ready + hb);
        if (warp == 2 && lane == 0) MOE_TRACE_EV(2, (int)(2 * (hcount + j) + 1));
      }
      if (!ok) break;
      hcount += nch;

      // Look ahead: prepare the next unit's X operand before draining Y so
      // the tensor core can start the next unit's MMA1 meanwhile.
      const int u_next = u + gridDim.x;
      const UnitWork uw_next = unit_work(u_next, su, S, NCH, atomic_all);
      BlockCursor nxt = cur;
      const bool have_next = nxt.seek(uw_next.gb, p.group_sizes, p.E, p.M);
      if (have_next && X_RES) {
        ok = C::kTF32 ? split_x(ui + 1) : pass_x(ui + 1);
        if (!ok) break;
      }

      // Y epilogue: this warp drains columns [half*D/2, +D/2) of its rows.
      if (!warp_wait(y_full, ui & 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float4* wstage = ystage + (warp - 2u) * 256u;
#pragma unroll 1
      for (int c0 = half * (D / 2); c0 < (int)(half + 1) * (D / 2); c0 += 32)
        store_y_block<D>(lane_base + c0, wstage, p.y, row0 + (int)(q * 32u), row_end, c0, lane, uw.atomic);
      tc_fence_before();
      mbar_arrive(y_empty);

      u = u_next;
      uw = uw_next;
      cur = nxt;
      have = have_next;
      ++ui;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace moe
