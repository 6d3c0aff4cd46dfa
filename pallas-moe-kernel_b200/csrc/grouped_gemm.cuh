// Persistent grouped GEMM over ragged expert row blocks on CTA pairs
// (2-SM tcgen05 MMA), sm_100a.  The large-D expert MLP runs as two launches:
//
//   up   : H[rows of e, :] = GELU_tanh(X[rows of e, :] @ W_up[e])   (bf16 H; f16 with e4m3 weights)
//   down : Y[rows of e, :] = H[rows of e, :] @ W_down[e]            (f32 Y)
//
// A (X or H, row-major, K-major) tiles of 128 rows come from each CTA of the
// pair; B (W_up[e] (D, F) or W_down[e] (F, D), N contiguous: MN-major) tiles
// are split along N between the two CTAs, so each SM streams half of every
// weight tile.  The leader CTA issues tcgen05.mma.cta_group::2 with
// M = 256, N = 256, K = 16 into TMEM; accumulators are double-buffered (2 x
// 256 columns) so the epilogue of one tile overlaps the MMAs of the next.
//
// f32 inputs (TF32 = true) run as 3xTF32 on kind::tf32: A and B come as tf32
// hi/lo planes (value = hi + lo, hi = the value rounded to tf32), B
// transposed to K-major (W^T (N, K) per expert), and every K step
// issues hi*hi + hi*lo + lo*hi.  The up GEMM's epilogue writes H as hi/lo f32
// planes for the down GEMM.
//
// Weights are read through 3-D tensor maps [E][K][N] (K-major planes:
// [E][N][K]), so a box never reaches into the next expert: columns past N
// and rows past K read as zero, and N and K need not be multiples of the
// tile (N, K multiples of 8 for 16-bit data, 4 for f32, 16 for e4m3, so that
// rows start on 16-byte boundaries); stores mask the columns past N.
//
// Tiles are (expert, 256-row block, 256-column block), enumerated on the
// device from the group sizes (no padded grid; the last row block of an
// expert is row-masked at the store), walked by every pair with a static
// stride and rasterised in groups of GM row blocks so that the pairs running
// at the same time share A and B tiles in L2.
//
// Warp roles: warp 0 TMA producer (both CTAs), warp 1 TMEM owner + MMA
// issuer (leader), warps 2..5 epilogue (one TMEM lane quadrant each; both
// CTAs), and for e4m3 weights warp 10 streams raw B tiles into a deep ring
// of their own while warps 6..9 dequantise each raw B tile
// (e4m3 x 128x128 block scale -> bf16; X and H are bf16 too) into the MMA's
// operand layout.
#pragma once
#include "ep_exchange.cuh"
#include "fused_small.cuh"

namespace moe {

// Expert-parallel combine fused into the f32 epilogue: each output row goes
// straight to its source rank's Y landing area (peer stores over NVLink)
// instead of this rank's Y.  `recv` lists, per local expert and source rank,
// {first row of the expert's rows that came from that source, rows, first row
// in the source's Y, source rank}.
struct EpScatter {
  uint8_t* base[8];    // every rank's symmetric buffer, in this process's address space
  size_t off;          // byte offset of the Y landing area inside those buffers
  const int4* recv;    // [E][world]
  int world;
  int on;
};

struct GemmParams {
  const int32_t* group_sizes;
  void* out;          // H (bf16 or, for e4m3 weights, f16; [M, N]) or Y (f32, [M, N])
  int M;              // rows of A / out
  int E;
  int N;              // output columns (F for up, D for down)
  int K;              // reduction (D for up, F for down)
  int group_m;        // tile rasterisation group (row blocks)
  int* status;
  const float* b_scale;  // FP8 weights: (E, ceil(K/128), ceil(N/128)) f32 block scales, else null
  int skip_tail;         // 1: leave rows at or past sum(group_sizes) unwritten (Y only)
  EpScatter scatter;     // Y only: rows go to their source ranks (expert parallelism)
  void* out2;            // EPI 3: the pre-activation X W_up (bf16, [M, N]) saved for the backward;
                         // TF32 EPI 0: the lo plane of H (f32, [M, N]; `out` holds the hi plane)
  EpDispatch dispatch;   // EPI 0, bf16: expert-parallel dispatch fused into the up GEMM
  int l2_mode;           // L2 hints of the A / B loads: 0 evict_last / evict_last, 1 evict_normal / evict_normal,
                         // 2 evict_first / evict_last, 3 evict_last / evict_first
};

__device__ __forceinline__ uint64_t gemm_l2_policy(int mode, bool b_operand) {
  switch (mode) {
    case 1: return l2_policy_evict_normal();
    case 2: return b_operand ? l2_policy_evict_last() : l2_policy_evict_first();
    case 3: return b_operand ? l2_policy_evict_first() : l2_policy_evict_last();
    default: return l2_policy_evict_last();
  }
}

// store_y_block with one destination row pointer per row: lane l of the warp
// holds the pointer of row l of the 32-row block (null = not stored); columns
// at or past `col_end` are not stored.
__device__ __forceinline__ void store_y_rows(uint32_t taddr, float4* stage, uint8_t* row_ptr, int col0,
                                             uint32_t lane, float mul, int col_end) {
  uint32_t v[32];
  tmem_ld32(taddr, v);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * mul);
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
    uint8_t* dst = reinterpret_cast<uint8_t*>(
        __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(row_ptr), r));
    if (dst && col0 + 4 * k < col_end) *reinterpret_cast<float4*>(dst + (size_t)(col0 + 4 * k) * 4) = val;
  }
  __syncwarp();
}

// EPI 0: GELU -> H, 1: f32 Y, 2: SwiGLU -> H (B holds gate and up weights
// interleaved every 128 columns, and for e4m3 their block scales one
// block per period; H has half the columns), 3: GELU -> H plus
// the pre-activation (bf16) to out2, 4: SwiGLU plus the raw gate/up columns
// (bf16) to out2; BFP8: e4m3 B dequantised in smem, f16 operands; TF32: f32
// operands as tf32 hi/lo planes (3xTF32), EPI 0 or 1 only.
//
// WIDE = 2 (bf16 Y only): a tile is 256 rows x 512 columns, two 256-column
// MMAs per K step sharing the A tile, one 512-column accumulator (no
// double-buffering).  Half as many tiles run the whole reduction, so half as
// many waves stream distinct operands through L2 -- for a long reduction
// (the down GEMM's K = F) most DRAM re-reads of H and W_down go away -- and
// each A byte staged feeds twice the MMA work.
template <int EPI, bool BFP8, bool TF32 = false, int WIDE = 1>
struct GemmCfg {
  static_assert(!(TF32 && (BFP8 || EPI > 1)), "3xTF32 runs the GELU and Y epilogues on f32 planes");
  static_assert(WIDE == 1 || (WIDE == 2 && EPI == 1 && !BFP8 && !TF32), "wide tiles: bf16 operands, f32 Y");
  static constexpr int BM = 128;   // rows per CTA (256 per pair)
  static constexpr int BN = 256;   // output columns per MMA (128 per CTA of B)
  static constexpr int TILE_N = BN * WIDE;  // output columns per tile
  static constexpr int BK = TF32 ? 32 : 64;  // elements of one 128-byte swizzle row
  static constexpr int A_BYTES = BM * 128;             // 16 KB (one plane)
  static constexpr int B_BYTES = (BN / 2) * 128;       // 16 KB (one plane of this CTA's B half)
  static constexpr int B8_BYTES = BFP8 ? (BN / 2) * BK : 0;  // 8 KB raw e4m3 tile
  static constexpr int PLANES = TF32 ? 2 : 1;          // hi and lo planes of A and of B
  static constexpr int STAGE = PLANES * (A_BYTES + WIDE * B_BYTES);  // operand stage
  static constexpr int NS = TF32 ? 3 : ((BFP8 || WIDE == 2) ? 4 : 6); // operand stages
  static constexpr int NR = BFP8 ? 10 : 0;             // raw e4m3 stages (HBM stream runs ahead)
  // 3xTF32 tiles hold all 512 TMEM columns (no overlap with the next tile's
  // MMAs), so their epilogue runs on eight warps: two per TMEM lane quadrant,
  // each draining half of the tile's columns.
  static constexpr int EPI_WARPS = TF32 ? 8 : 4;
  static constexpr int CVT_WARPS = BFP8 ? 8 : 0;  // two per SM sub-partition
  static constexpr int OUT_STAGE = EPI_WARPS * 32 * 128;  // 4 KB per warp: 32 rows x 128 B
  static constexpr int BAR_BYTES = BFP8 ? 512 : 256;
  // bf16 up GEMM: four warps that run the expert-parallel dispatch (idle
  // otherwise), with the slice row prefix in shared memory.
  static constexpr int PUSH_WARPS = (EPI == 0 && !BFP8 && !TF32) ? 4 : 0;
  static constexpr int PUSH_SMEM = PUSH_WARPS ? (kEpMaxExperts + 1) * 4 : 0;
  static constexpr int SMEM = 1024 + NS * STAGE + NR * B8_BYTES + OUT_STAGE + BAR_BYTES + PUSH_SMEM;
  static constexpr int TMEM_COLS = 512;                 // 2 accumulators x 256 columns
  // Accumulator buffers per tile: 16-bit operands double-buffer one
  // 256-column accumulator (the epilogue of tile t overlaps the MMAs of
  // t + 1).  3xTF32 keeps two accumulators per tile instead -- hi*hi in one,
  // the small cross terms hi*lo + lo*hi in the other, summed in the epilogue
  // with f32 rounding -- so that the large one takes K/8 accumulate steps
  // rather than 3K/8 (each accumulate step into TMEM truncates, an error that
  // grows with the number of steps), at the cost of that overlap.
  static constexpr uint32_t NACC = (TF32 || WIDE == 2) ? 1 : 2;
  // e4m3 weights: the up GEMM runs on bf16 operands (the caller's X, weights
  // decoded to bf16) and stores H in f16; the down GEMM runs on f16 operands
  // (H, weights decoded to f16 with a shorter decode).
  static constexpr bool DEC_F16 = BFP8 && EPI == 1;
  // 16-bit B is read MN-major (the weights' own layout); tf32 B is K-major.
  static constexpr uint32_t IDESC = TF32 ? make_idesc(kFmtTF32, 256, BN, 0, 0)
                                         : make_idesc(DEC_F16 ? kFmtF16 : kFmtBF16, 256, BN, 0, 1);
  static constexpr uint32_t TX = 2 * STAGE;                // both CTAs (bf16 or tf32 B)
  static constexpr uint32_t TX_A = 2 * A_BYTES;            // both CTAs' A (FP8 B arrives converted)
  static constexpr int RAW_WARP = 2 + EPI_WARPS + CVT_WARPS;  // FP8: producer of the raw ring
  static constexpr int THREADS = 64 + (EPI_WARPS + CVT_WARPS + PUSH_WARPS) * 32 + (BFP8 ? 32 : 0);
  // Register cap: that of a 320-thread block at least (the bf16 epilogue
  // was scheduled under it), or of the FP8 block with its extra warps.
  static constexpr int LAUNCH_BOUND = THREADS > 320 ? THREADS : 320;
  static_assert(SMEM <= kMaxSmemPerBlock, "shared memory budget");
  // Even ring depths: each raw stage is then always used by the same one of
  // the two alternating converter groups, which consumed its previous use, so
  // a parity wait cannot take a phase two uses old for the awaited one.
  static_assert(!BFP8 || (NS % 2 == 0 && NR % 2 == 0), "converter groups need even ring depths (mbarrier parity aliasing)");
};

struct GemmMaps {
  CUtensorMap a;     // X or H: [M, K] bf16 (f16 with e4m3 weights), box {64, 128}; TF32: hi plane, box {32, 128}
  CUtensorMap b;     // W_up / W_down as [E][K][N]: bf16 box {64, 64, 1}, or e4m3 bytes box {128, 64, 1};
                     // TF32: hi plane of W^T as [E][N][K], box {32, 128, 1}
  CUtensorMap a_lo;  // TF32 only: lo planes
  CUtensorMap b_lo;
};

// Four e4m3 values (one 32-bit word, lowest byte first) -> four bf16 (two
// bf16x2 words) times the block scale s.  e4m3 -> f16 (cvt.rn.f16x2.e4m3x2)
// and f16 -> f32 are exact; the f32 product is rounded to bf16 (with the
// f32 multiply's own rounding first).  bf16 keeps f32's exponent range, so
// X and H need no conversion or saturation.  (A shorter form -- the f16 bit
// pattern shifted into a bf16 one and one mul.rn.bf16x2 by the scale --
// measured 7-8% more cycles in the row-tiled kernel than this one.)
__device__ __forceinline__ uint2 e4m3x4_to_bf16x4(uint32_t v, float s) {
  uint32_t h01, h23;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h01), "=r"(h23)
      : "r"(v));
  float a0, a1, a2, a3;
  asm("{\n\t.reg .f16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
      : "=f"(a0), "=f"(a1)
      : "r"(h01));
  asm("{\n\t.reg .f16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
      : "=f"(a2), "=f"(a3)
      : "r"(h23));
  return make_uint2(pack_bf16x2(a0 * s, a1 * s), pack_bf16x2(a2 * s, a3 * s));
}

// Four e4m3 values -> four f16 (two f16x2 words) times the block scale s2
// (an f16x2 pair).  e4m3 values are exact in f16, so the multiply's rounding
// is the only one; decode and multiply are one instruction per pair each.
__device__ __forceinline__ uint2 e4m3x4_to_f16x4(uint32_t v, uint32_t s2) {
  uint32_t h01, h23;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h01), "=r"(h23)
      : "r"(v));
  asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h01) : "r"(s2));
  asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h23) : "r"(s2));
  return make_uint2(h01, h23);
}

// Block scale of one K step in the form the decoder of the GEMM takes, and
// the decode of four e4m3 values with it: f16 operands (the down GEMM: its A
// operand is H, which the up GEMM stores in f16) or bf16 operands (the up
// GEMM, whose A operand is the caller's bf16 X).
template <bool F16>
struct E4m3Decoder {
  uint32_t s2;
  float sf;
  __device__ __forceinline__ explicit E4m3Decoder(float scale) {
    if constexpr (F16) s2 = pack_f16x2_sat(scale, scale);
    else sf = scale;
  }
  __device__ __forceinline__ uint2 operator()(uint32_t v) const {
    if constexpr (F16) return e4m3x4_to_f16x4(v, s2);
    else return e4m3x4_to_bf16x4(v, sf);
  }
};

// Power-of-two exponent k of an FP8 tile: 2^k brings the largest block scale
// of the tile's two 128-column blocks (over all of K) into [1, 2), so the
// decoded weights sit in a fixed range whatever the scales' magnitude.  The
// converters multiply the weights by scale * 2^k; the epilogue multiplies the
// accumulator by 2^-k (exact).  Every lane of the calling warp returns the
// same k, in [-100, 100].
__device__ __forceinline__ int fp8_tile_shift(const float* b_scale, int K, int N, int e, int nb, uint32_t lane) {
  const int nkb = (K + 127) / 128, nnb = (N + 127) / 128;
  const float* sc = b_scale + (size_t)e * nkb * nnb + (size_t)nb * 2;
  const int ncb = nnb - 2 * nb < 2 ? nnb - 2 * nb : 2;  // scale blocks of this tile inside N (1 or 2)
  float m = 0.f;
  for (int i = (int)lane; i < 2 * nkb; i += 32)
    if ((i & 1) < ncb) m = fmaxf(m, __ldg(sc + (size_t)(i >> 1) * nnb + (i & 1)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int ex = (int)((__float_as_uint(m) >> 23) & 0xFFu);
  const int k = 127 - ex;
  return k < -100 ? -100 : (k > 100 ? 100 : k);
}
__device__ __forceinline__ float exp2i(int k) { return __uint_as_float((uint32_t)(127 + k) << 23); }

// Tile walk: global tile index -> (expert, row block, column block) with
// grouped rasterisation inside each expert; monotone in the tile index.
struct TileCursor {
  int e = -1;
  int t_begin = 0;   // first global tile of expert e
  int ntiles = 0;    // tiles of expert e
  int row_begin = 0;
  int rows = 0;
  int mt = 0;        // 256-row blocks of expert e

  __device__ __forceinline__ bool seek(int t, const int32_t* gs, int E, int M, int nt) {
    while (t >= t_begin + ntiles) {
      t_begin += ntiles;
      row_begin += rows;
      if (++e >= E) return false;
      int g = __ldg(gs + e);
      g = g < 0 ? 0 : g;
      const int rem = M - row_begin;
      g = g > rem ? (rem > 0 ? rem : 0) : g;
      rows = g;
      mt = (g + 255) >> 8;
      ntiles = mt * nt;
    }
    return true;
  }
  // (row block, column block) of global tile t (after seek).
  __device__ __forceinline__ void coords(int t, int nt, int gm_max, int& m, int& n) const {
    const int l = t - t_begin;
    const int per_group = gm_max * nt;
    const int g = l / per_group;
    const int r = l - g * per_group;
    int gm = mt - g * gm_max;
    gm = gm < gm_max ? gm : gm_max;
    m = g * gm_max + r % gm;
    n = r / gm;
  }
};

template <int EPI, bool BFP8, bool TF32 = false, int WIDE = 1>
__global__ void __launch_bounds__(GemmCfg<EPI, BFP8, TF32, WIDE>::LAUNCH_BOUND, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
  using C = GemmCfg<EPI, BFP8, TF32, WIDE>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* ring = smem;
  uint8_t* rawring = ring + C::NS * C::STAGE;   // FP8: [NR] raw e4m3 B tiles
  uint8_t* ostage = rawring + C::NR * C::B8_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ostage + C::OUT_STAGE);
  uint64_t* full = bars;                // [NS] leader
  uint64_t* empty = bars + C::NS;       // [NS] both (multicast commit)
  uint64_t* acc_full = bars + 2 * C::NS;  // [2] both (multicast commit)
  uint64_t* acc_empty = acc_full + 2;     // [2] leader (epilogue warps of both CTAs)
  uint64_t* raw_full = acc_full + 4;      // [NR] local: raw e4m3 B landed (FP8 only)
  uint64_t* raw_empty = raw_full + C::NR; // [NR] local: converters done with the raw tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(raw_empty + C::NR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* push_wr = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);  // PUSH_WARPS only

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1);
  const int npairs = (int)(gridDim.x >> 1);
  constexpr uint16_t kBoth = 0x3;
  const int nt = (p.N + C::TILE_N - 1) / C::TILE_N;
  const int nk = (p.K + C::BK - 1) / C::BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      // The leader producer's arrive + both CTAs' TMA bytes; e4m3 B adds one
      // arrival per warp of the stage's converter group in both CTAs.
      mbar_init(full + i, BFP8 ? 1 + 2 * (C::CVT_WARPS / 2) : 1);
      mbar_init(empty + i, 1);
    }
    for (int i = 0; i < C::NR; ++i) {
      mbar_init(raw_full + i, 1);
      mbar_init(raw_empty + i, C::CVT_WARPS / 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 2 * C::EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.a);
    tma_prefetch_desc(&maps.b);
    if constexpr (TF32) {
      tma_prefetch_desc(&maps.a_lo);
      tma_prefetch_desc(&maps.b_lo);
    }
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_l0 = mapa_shared(smem_u32(full), 0);
  const uint32_t acc_empty_l = mapa_shared(smem_u32(acc_empty), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      TileCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol_a = gemm_l2_policy(p.l2_mode, false);
      const uint64_t pol_b = gemm_l2_policy(p.l2_mode, true);
      uint32_t arrived = 0;  // dispatch: sources whose rows have landed here
      for (int t = pair;; t += npairs) {
        if (!cur.seek(t, p.group_sizes, p.E, p.M, nt)) break;
        int mb, nb;
        cur.coords(t, nt, p.group_m, mb, nb);
        const int row0 = cur.row_begin + mb * 256 + (int)rank * C::BM;
        const int n0 = nb * C::TILE_N + (int)rank * (C::BN / 2);
        bool ok = true;
        if (C::PUSH_WARPS > 0 && p.dispatch.on) {
          // Wait for every peer whose rows of this expert meet this CTA's 128
          // rows (a peer's flag covers all its rows of this step), then order
          // the TMA reads after the peer's stores.
          // The A box still spans all 128 rows, so in the expert's last row
          // block it also reads rows past the expert's end: the next expert's
          // rows, possibly from sources not waited for here and still being
          // written over NVLink.  That is correct only because each output
          // row depends on its own A row alone and the epilogue never stores
          // rows past the expert's end; an epilogue that mixes rows (or a
          // split-K sum) would have to wait for those sources as well.
          const EpDispatch& d = p.dispatch;
          for (int s = 0; s < d.world && ok; ++s) {
            if (s == d.rank || (arrived >> s) & 1u) continue;
            const int4 rc = d.recv[cur.e * d.world + s];
            if (rc.y <= 0 || rc.x >= row0 + C::BM || rc.x + rc.y <= row0) continue;
            const uint64_t t0 = global_timer_ns();
            while (!epoch_reached(ld_acquire_sys(d.data_flags + s), d.epoch)) {
              if (*reinterpret_cast<volatile int*>(d.abort_word) || *abort_flag) {
                ok = false;
                break;
              }
              if (global_timer_ns() - t0 > kEpWaitLimitNs) {
                atomicOr(p.status, kStatusPeerTimeout);
                atomicExch(d.abort_word, 1);
                *abort_flag = 1;
                ok = false;
                break;
              }
            }
            arrived |= 1u << s;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");
          if (!ok) break;
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + stage * C::STAGE;
          if constexpr (BFP8) {
            // A of both CTAs lands on the leader's barrier; the bf16 B half
            // of each CTA comes from its converter warps (raw ring below).
            const uint32_t bar = full_l0 + stage * 8;
            if (rank == 0) mbar_arrive_expect_tx(full + stage, C::TX_A);
            tma_load_2d_pair(st, &maps.a, bar, kb * C::BK, row0, pol_a);
          } else if constexpr (TF32) {
            // Stage layout: A hi | A lo | B hi | B lo (K-major, 128 rows x 128 B each).
            const uint32_t bar = full_l0 + stage * 8;
            if (rank == 0) mbar_arrive_expect_tx(full + stage, C::TX);
            tma_load_2d_pair(st, &maps.a, bar, kb * C::BK, row0, pol_a);
            tma_load_2d_pair(st + C::A_BYTES, &maps.a_lo, bar, kb * C::BK, row0, pol_a);
            tma_load_3d_pair(st + 2 * C::A_BYTES, &maps.b, bar, kb * C::BK, n0, cur.e, pol_b);
            tma_load_3d_pair(st + 2 * C::A_BYTES + C::B_BYTES, &maps.b_lo, bar, kb * C::BK, n0, cur.e, pol_b);
          } else {
            const uint32_t bar = full_l0 + stage * 8;
            if (rank == 0) mbar_arrive_expect_tx(full + stage, C::TX);
            tma_load_2d_pair(st, &maps.a, bar, kb * C::BK, row0, pol_a);
#pragma unroll
            for (int h = 0; h < WIDE; ++h) {  // this CTA's 128 columns of each 256-column MMA
              uint8_t* bd = st + C::A_BYTES + h * C::B_BYTES;
              tma_load_3d_pair(bd, &maps.b, bar, n0 + h * C::BN, kb * C::BK, cur.e, pol_b);
              tma_load_3d_pair(bd + 64 * 128, &maps.b, bar, n0 + h * C::BN + 64, kb * C::BK, cur.e, pol_b);
            }
          }
          if (++stage == C::NS) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader, whole warp)
    if (rank == 0) {
      TileCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t tcount = 0;
      for (int t = pair;; t += npairs, ++tcount) {
        if (!cur.seek(t, p.group_sizes, p.E, p.M, nt)) break;
        const uint32_t ab = tcount % C::NACC;
        const uint32_t use = tcount / C::NACC;
        if (!mbar_wait_warp(acc_empty + ab, (use & 1u) ^ 1u, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * C::BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait_warp(full + stage, phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(ring + stage * C::STAGE);
          if constexpr (TF32) {
            // K = 8 per instruction (32 bytes along the 128-byte row); the
            // small cross terms first, then hi * hi.
            const uint64_t ah = make_sdesc(st, 16, 1024), al = make_sdesc(st + C::A_BYTES, 16, 1024);
            const uint64_t bh = make_sdesc(st + 2 * C::A_BYTES, 16, 1024);
            const uint64_t bl = make_sdesc(st + 2 * C::A_BYTES + C::B_BYTES, 16, 1024);
#pragma unroll
            for (int ki = 0; ki < C::BK / 8; ++ki) {
              const uint64_t o = (uint64_t)((ki * 32) >> 4);
              const uint32_t acc = (kb > 0 || ki > 0) ? 1u : 0u;
              umma_ss_pair<Kind::TF32>(d_tmem + C::BN, ah + o, bl + o, C::IDESC, acc);  // cross terms
              umma_ss_pair<Kind::TF32>(d_tmem + C::BN, al + o, bh + o, C::IDESC, 1u);
              umma_ss_pair<Kind::TF32>(d_tmem, ah + o, bh + o, C::IDESC, acc);          // hi * hi
            }
          } else {
            const uint64_t a_desc = make_sdesc(st, 16, 1024);
            const uint64_t b_desc = make_sdesc(st + C::A_BYTES, 64 * 128, 1024);
#pragma unroll
            for (int ki = 0; ki < C::BK / 16; ++ki)
#pragma unroll
              for (int h = 0; h < WIDE; ++h)
                umma_ss_pair<Kind::F16>(d_tmem + h * C::BN, a_desc + (uint64_t)((ki * 32) >> 4),
                                        b_desc + (uint64_t)((h * C::B_BYTES + ki * 16 * 128) >> 4), C::IDESC,
                                        (kb > 0 || ki > 0) ? 1u : 0u);
          }
          umma_commit_pair(empty + stage, kBoth);
          if (++stage == C::NS) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(acc_full + ab, kBoth);
      }
    }
  } else if (BFP8 && warp == (uint32_t)C::RAW_WARP) {
    // ------------------------------------------------------------ raw e4m3 B producer (both CTAs)
    // Streams this CTA's half of every B tile from HBM into a ring of NR raw
    // stages that runs ahead of the operand ring by up to NR tiles.
    if (lane == 0) {
      TileCursor cur;
      int rs = 0;
      uint32_t rph = 0;
      const uint64_t pol_b = gemm_l2_policy(p.l2_mode, true);
      bool ok = true;
      for (int t = pair; ok; t += npairs) {
        if (!cur.seek(t, p.group_sizes, p.E, p.M, nt)) break;
        int mb, nb;
        cur.coords(t, nt, p.group_m, mb, nb);
        const int n0 = nb * C::BN + (int)rank * (C::BN / 2);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(raw_empty + rs, rph ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(raw_full + rs, C::B8_BYTES);
          tma_load_3d_hint(rawring + rs * C::B8_BYTES, &maps.b, raw_full + rs, n0, kb * C::BK, cur.e, pol_b);
          if (++rs == C::NR) {
            rs = 0;
            rph ^= 1u;
          }
        }
      }
    }
  } else if (BFP8 && warp >= 2u + C::EPI_WARPS) {
    // ------------------------------------------------------------ e4m3 -> bf16 B converters (both CTAs)
    // Two groups of four warps take alternate K steps of each tile: each
    // group has two stage times for its stage, and the fixed costs of a stage
    // (barrier checks, fence, hand-off) of the two groups overlap.  Every K
    // step goes to exactly one group and every barrier counts the arrivals of
    // one group, so an odd number of K steps per tile (K % 128 != 0) only
    // gives one group two steps in a row at the tile boundary.  In a group, thread t handles
    // k-row r = t % 64 of the 64 x 128 raw tile and half h = t / 64 of its
    // 128 columns (= one 64-column f16 atom row, 128 bytes): the 8 threads of
    // a quarter-warp own 8 consecutive rows, so their swizzled 16-byte
    // accesses fall in 8 distinct bank groups.  A raw tile is converted as
    // soon as it has landed and its operand stage is free.
    const int ct = (int)threadIdx.x - 64 - C::EPI_WARPS * 32;  // 0..255
    const int grp = ct >> 7;
    const int r = ct & 63, h = (ct >> 6) & 1;
    const int nkb_scale = (p.K + 127) / 128, nnb_scale = (p.N + 127) / 128;
    TileCursor cur;
    uint32_t gk = 0;  // K steps of this CTA's earlier tiles
    bool ok = true;
    for (int t = pair; ok; t += npairs) {
      if (!cur.seek(t, p.group_sizes, p.E, p.M, nt)) break;
      int mb, nb;
      cur.coords(t, nt, p.group_m, mb, nb);
      const int n0 = nb * C::BN + (int)rank * (C::BN / 2);
      // A half that starts at or past N holds only zero-filled columns: its
      // scales are never read (0 is used).
      const bool col_in = n0 / 128 < nnb_scale;
      const float* srow = p.b_scale + ((size_t)cur.e * nkb_scale) * nnb_scale + (col_in ? n0 / 128 : 0);
      // The tile's block scales along K (one per 128 rows of B), fetched once
      // per tile -- lane l holds k-blocks l and l + 32 -- and broadcast per
      // stage, so no stage waits on a global load.
      const float s_lo = col_in && (int)lane < nkb_scale ? __ldg(srow + (size_t)lane * nnb_scale) : 0.f;
      const float s_hi = col_in && (int)lane + 32 < nkb_scale ? __ldg(srow + (size_t)(lane + 32) * nnb_scale) : 0.f;
      const float up = exp2i(fp8_tile_shift(p.b_scale, p.K, p.N, cur.e, nb, lane));
      for (int kb = grp; kb < nk; kb += 2) {
        const uint32_t g = gk + (uint32_t)kb;
        constexpr uint32_t kNR = C::NR > 0 ? C::NR : 1;  // this branch only runs with e4m3 weights
        const int stage = (int)(g % C::NS), rs = (int)(g % kNR);
        const uint32_t phase = (g / C::NS) & 1u, rph = (g / kNR) & 1u;
        if (!mbar_wait_warp(raw_full + rs, rph, abort_flag, p.status) ||
            !mbar_wait_warp(empty + stage, phase ^ 1u, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const int kblk = (kb * C::BK) / 128;
        const float s_reg = __shfl_sync(0xffffffffu, kblk < 32 ? s_lo : s_hi, kblk & 31);
        const float sc = kblk < 64 ? s_reg : (col_in ? __ldg(srow + (size_t)kblk * nnb_scale) : 0.f);
        const E4m3Decoder<C::DEC_F16> dec(sc * up);
        const uint8_t* src = rawring + rs * C::B8_BYTES + r * 128;             // 128-byte swizzled raw row
        uint8_t* dst = ring + stage * C::STAGE + C::A_BYTES + h * (64 * 128) + r * 128;  // atom h, row r
        const int rsw = r & 7;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int chunk = 4 * h + c;  // 16 raw bytes = columns 16*chunk .. +15
          const uint4 v = *reinterpret_cast<const uint4*>(src + ((chunk ^ rsw) << 4));
          const uint2 b0 = dec(v.x), b1 = dec(v.y);
          const uint2 b2 = dec(v.z), b3 = dec(v.w);
          const int j0 = 2 * c, j1 = 2 * c + 1;  // output 16-byte chunks in the atom row
          *reinterpret_cast<uint4*>(dst + ((j0 ^ rsw) << 4)) = make_uint4(b0.x, b0.y, b1.x, b1.y);
          *reinterpret_cast<uint4*>(dst + ((j1 ^ rsw) << 4)) = make_uint4(b2.x, b2.y, b3.x, b3.y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(raw_empty + rs);
          mbar_arrive_cluster_cta(full_l0 + stage * 8);
        }
      }
      gk += (uint32_t)nk;
    }
  } else if (C::PUSH_WARPS > 0 && warp >= 2u + C::EPI_WARPS) {
    // ------------------------------------------------------------ expert-parallel dispatch (both CTAs)
    // This rank's rows of the other owners' experts go straight into their
    // X landing regions while the tensor cores work on the rows already here.
    if (p.dispatch.on) {
      const EpDispatch& d = p.dispatch;
      const int pt = (int)threadIdx.x - 64 - C::EPI_WARPS * 32;  // 0 .. 32 * PUSH_WARPS - 1
      constexpr int kPushThreads = C::PUSH_WARPS * 32;
      for (int g = pt; g <= d.E; g += kPushThreads) push_wr[g] = d.wave_rows[g];
      asm volatile("bar.sync 1, %0;" ::"n"(kPushThreads) : "memory");
      const int gw = (int)blockIdx.x * C::PUSH_WARPS + (pt >> 5);
      const int nw = (int)gridDim.x * C::PUSH_WARPS;
      const int rows = push_wr[d.E];
      if (*reinterpret_cast<volatile int*>(d.abort_word) == 0) {
        for (int row = gw; row < rows; row += nw) {
          const int g = ep_find_slice(push_wr, d.E, row);
          const EpSlice sl = d.slices[g];
          if (sl.owner == d.rank) continue;
          const int r = row - push_wr[g];
          warp_copy_row(d.base[sl.owner] + d.off_x + (size_t)(sl.dst_row + r) * d.row_bytes,
                        d.x + (size_t)(sl.src_row + r) * d.row_bytes, d.row_bytes, (int)lane);
        }
      }
      __threadfence_system();
      asm volatile("bar.sync 1, %0;" ::"n"(kPushThreads) : "memory");
      if (pt == 0) {
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(d.push_ctr) : "memory");
        if (prev == gridDim.x - 1) {
          // Last CTA: every row of this rank has left; tell the owners (an
          // aborted engine tells nobody, so its peers time out instead).
          *d.push_ctr = 0;
          __threadfence_system();
          if (*reinterpret_cast<volatile int*>(d.abort_word) == 0)
            for (int s = 0; s < d.world; ++s)
              if (s != d.rank)
                st_release_sys(reinterpret_cast<uint32_t*>(d.base[s]) +
                                   (d.data_flags - reinterpret_cast<const uint32_t*>(d.base[d.rank])) + d.rank,
                               d.epoch);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const uint32_t q = warp & 3u;
    const uint32_t lane_base = tmem_base + ((q * 32u) << 16);
    uint8_t* wst = ostage + (warp - 2u) * 4096u;
    if (EPI == 1 && !p.skip_tail) {
      // Rows at or past sum(group_sizes) are zero in ragged_dot.
      int total = 0;
      for (int e = 0; e < p.E; ++e) {
        const int g = __ldg(p.group_sizes + e);
        total += g < 0 ? 0 : g;
        if (total >= p.M) {
          total = p.M;
          break;
        }
      }
      const size_t n4 = (size_t)(p.M - total) * p.N / 4;
      float4* base = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)total * p.N);
      const int etid = (int)threadIdx.x - 64;  // epilogue threads are 64 .. 64 + 32 EPI_WARPS - 1
      for (size_t i = (size_t)blockIdx.x * (C::EPI_WARPS * 32) + etid; i < n4;
           i += (size_t)gridDim.x * (C::EPI_WARPS * 32))
        base[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    TileCursor cur;
    uint32_t tcount = 0;
    for (int t = pair;; t += npairs, ++tcount) {
      if (!cur.seek(t, p.group_sizes, p.E, p.M, nt)) break;
      int mb, nb;
      cur.coords(t, nt, p.group_m, mb, nb);
      const int row_end = cur.row_begin + cur.rows;
      const int wrow0 = cur.row_begin + mb * 256 + (int)rank * C::BM + (int)q * 32;
      const uint32_t ab = tcount % C::NACC;
      const uint32_t use = tcount / C::NACC;
      if (!mbar_wait_warp(acc_full + ab, use & 1u, abort_flag, p.status)) break;
      tc_fence_after();
      const uint32_t acc = lane_base + ab * C::BN;
      // FP8 tiles were accumulated with weights scaled by 2^k.
      const float mul = BFP8 ? exp2i(-fp8_tile_shift(p.b_scale, p.K, p.N, cur.e, nb, lane)) : 1.f;
      // Columns of this tile inside N (the last column tile may be partial).
      const int ncol = p.N - nb * C::TILE_N < C::TILE_N ? p.N - nb * C::TILE_N : C::TILE_N;
      // 3xTF32: this warp's half of the columns, [cb, ce).
      const int cb = TF32 ? (int)((warp - 2u) >> 2) * (C::BN / 2) : 0;
      const int ce = TF32 ? (ncol < cb + C::BN / 2 ? ncol : cb + C::BN / 2) : ncol;
      if constexpr (TF32 && EPI == 0) {
        // 32 columns per step: GELU (f32 accuracy), then the tf32 split
        // g = hi + lo (tf32_hi_bits); each plane goes out through the 32-row
        // x 128-byte staging as full-line row stores.
        float4* wst4 = reinterpret_cast<float4*>(wst);
#pragma unroll 1
        for (int c0 = cb; c0 < ce; c0 += 32) {
          uint32_t v[32], w[32];
          tmem_ld32(acc + c0, v);
          tmem_ld32(acc + C::BN + c0, w);  // cross terms
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = __float_as_uint(gelu_tanh_exp(__uint_as_float(v[i]) + __uint_as_float(w[i])));
          const int gcol = nb * C::BN + c0;
#pragma unroll 1
          for (int pl = 0; pl < 2; ++pl) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              float q[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float g = __uint_as_float(v[4 * k + j]);
                const float h = __uint_as_float(tf32_hi_bits(v[4 * k + j]));
                q[j] = pl == 0 ? h : g - h;
              }
              wst4[lane * 8 + (k ^ (lane & 7))] = make_float4(q[0], q[1], q[2], q[3]);
            }
            __syncwarp();
            float* P = reinterpret_cast<float*>(pl == 0 ? p.out : p.out2);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 4 * i + (int)(lane >> 3);
              const int k = (int)(lane & 7);
              const float4 val = wst4[r * 8 + (k ^ (r & 7))];
              const int row = wrow0 + r;
              if (row < row_end && c0 + 4 * k < ncol)
                *reinterpret_cast<float4*>(P + (size_t)row * p.N + gcol + 4 * k) = val;
            }
            __syncwarp();
          }
        }
      } else if constexpr (EPI == 0 || EPI == 3) {
        // 64 columns per step: GELU, pack to bf16 (f16 for FP8 weights),
        // stage 32 rows x 128 B, store rows as full 128-byte lines.
        uint16_t* H = reinterpret_cast<uint16_t*>(p.out);  // bf16 / f16 bits
#pragma unroll 1
        for (int c0 = 0; c0 < ncol; c0 += 64) {
          uint32_t v[64];
          uint4* srow = reinterpret_cast<uint4*>(wst) + lane * 8;
          if constexpr (BFP8) {
            // Two 32-column halves (fewer live registers: this block has the
            // converter warps' registers to share).
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
              tmem_ld32(acc + c0 + 32 * hh, *reinterpret_cast<uint32_t(*)[32]>(v));
              tmem_ld_wait();
              auto g = [&](int i) { return gelu_tanh_fast(__uint_as_float(v[i]) * mul); };
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                uint4 w;
                w.x = pack_f16x2_sat(g(8 * k + 0), g(8 * k + 1));
                w.y = pack_f16x2_sat(g(8 * k + 2), g(8 * k + 3));
                w.z = pack_f16x2_sat(g(8 * k + 4), g(8 * k + 5));
                w.w = pack_f16x2_sat(g(8 * k + 6), g(8 * k + 7));
                srow[(4 * hh + k) ^ (lane & 7)] = w;
              }
            }
          } else {
            tmem_ld32(acc + c0, *reinterpret_cast<uint32_t(*)[32]>(v));
            tmem_ld32(acc + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              uint4 w;
              w.x = pack_bf16x2(gelu_tanh_fast(__uint_as_float(v[8 * k + 0])), gelu_tanh_fast(__uint_as_float(v[8 * k + 1])));
              w.y = pack_bf16x2(gelu_tanh_fast(__uint_as_float(v[8 * k + 2])), gelu_tanh_fast(__uint_as_float(v[8 * k + 3])));
              w.z = pack_bf16x2(gelu_tanh_fast(__uint_as_float(v[8 * k + 4])), gelu_tanh_fast(__uint_as_float(v[8 * k + 5])));
              w.w = pack_bf16x2(gelu_tanh_fast(__uint_as_float(v[8 * k + 6])), gelu_tanh_fast(__uint_as_float(v[8 * k + 7])));
              srow[k ^ (lane & 7)] = w;
            }
          }
          __syncwarp();
          const int gcol = nb * C::BN + c0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (int)(lane >> 3);
            const int k = (int)(lane & 7);
            const uint4 val = reinterpret_cast<const uint4*>(wst)[r * 8 + (k ^ (r & 7))];
            const int row = wrow0 + r;
            if (row < row_end && c0 + 8 * k < ncol)
              *reinterpret_cast<uint4*>(H + (size_t)row * p.N + gcol + 8 * k) = val;
          }
          __syncwarp();
          if constexpr (EPI == 3 && !BFP8) {
            // The same 64 columns before the activation, for the backward.
            uint16_t* A = reinterpret_cast<uint16_t*>(p.out2);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(v[8 * k + 0]), __uint_as_float(v[8 * k + 1]));
              w.y = pack_bf16x2(__uint_as_float(v[8 * k + 2]), __uint_as_float(v[8 * k + 3]));
              w.z = pack_bf16x2(__uint_as_float(v[8 * k + 4]), __uint_as_float(v[8 * k + 5]));
              w.w = pack_bf16x2(__uint_as_float(v[8 * k + 6]), __uint_as_float(v[8 * k + 7]));
              srow[k ^ (lane & 7)] = w;
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 4 * i + (int)(lane >> 3);
              const int k = (int)(lane & 7);
              const uint4 val = reinterpret_cast<const uint4*>(wst)[r * 8 + (k ^ (r & 7))];
              const int row = wrow0 + r;
              if (row < row_end && c0 + 8 * k < ncol)
                *reinterpret_cast<uint4*>(A + (size_t)row * p.N + gcol + 8 * k) = val;
            }
            __syncwarp();
          }
        }
      } else if constexpr (EPI == 2 || EPI == 4) {
        // SwiGLU: columns [0, 128) of the tile are gate, [128, 256) up;
        // H[:, 128 nb + c] = SiLU(gate_c) * up_c, 64 columns per step through
        // the same 32-row x 128-byte staging as the GELU epilogue.
        uint16_t* H = reinterpret_cast<uint16_t*>(p.out);  // bf16 bits
        const int ldh = p.N / 2;
#pragma unroll 1
        for (int c0 = 0; c0 < C::BN / 2; c0 += 64) {
          uint4* srow = reinterpret_cast<uint4*>(wst) + lane * 8;
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t g[32], u[32];
            tmem_ld32(acc + c0 + 32 * hh, g);
            tmem_ld32(acc + C::BN / 2 + c0 + 32 * hh, u);
            tmem_ld_wait();
            // e4m3 weights: the tile was accumulated with weights scaled by
            // 2^k (mul = 2^-k); H is the f16 operand of the down GEMM.
            auto h = [&](int i) {
              return silu_fast(__uint_as_float(g[i]) * mul) * (__uint_as_float(u[i]) * mul);
            };
            auto pk = [&](float a, float b) { return BFP8 ? pack_f16x2_sat(a, b) : pack_bf16x2(a, b); };
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint4 w;
              w.x = pk(h(8 * k + 0), h(8 * k + 1));
              w.y = pk(h(8 * k + 2), h(8 * k + 3));
              w.z = pk(h(8 * k + 4), h(8 * k + 5));
              w.w = pk(h(8 * k + 6), h(8 * k + 7));
              srow[(4 * hh + k) ^ (lane & 7)] = w;
            }
          }
          __syncwarp();
          const int gcol = nb * (C::BN / 2) + c0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (int)(lane >> 3);
            const int k = (int)(lane & 7);
            const uint4 val = reinterpret_cast<const uint4*>(wst)[r * 8 + (k ^ (r & 7))];
            const int row = wrow0 + r;
            if (row < row_end)
              *reinterpret_cast<uint4*>(H + (size_t)row * ldh + gcol + 8 * k) = val;
          }
          __syncwarp();
        }
        if constexpr (EPI == 4) {
          // The tile's raw gate and up columns (bf16, same interleave as the
          // weights), saved for the backward.
          uint16_t* GU = reinterpret_cast<uint16_t*>(p.out2);
#pragma unroll 1
          for (int c0 = 0; c0 < C::BN; c0 += 64) {
            uint4* srow = reinterpret_cast<uint4*>(wst) + lane * 8;
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t v[32];
              tmem_ld32(acc + c0 + 32 * hh, v);
              tmem_ld_wait();
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                uint4 w;
                w.x = pack_bf16x2(__uint_as_float(v[8 * k + 0]), __uint_as_float(v[8 * k + 1]));
                w.y = pack_bf16x2(__uint_as_float(v[8 * k + 2]), __uint_as_float(v[8 * k + 3]));
                w.z = pack_bf16x2(__uint_as_float(v[8 * k + 4]), __uint_as_float(v[8 * k + 5]));
                w.w = pack_bf16x2(__uint_as_float(v[8 * k + 6]), __uint_as_float(v[8 * k + 7]));
                srow[(4 * hh + k) ^ (lane & 7)] = w;
              }
            }
            __syncwarp();
            const int gcol = nb * C::BN + c0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 4 * i + (int)(lane >> 3);
              const int k = (int)(lane & 7);
              const uint4 val = reinterpret_cast<const uint4*>(wst)[r * 8 + (k ^ (r & 7))];
              const int row = wrow0 + r;
              if (row < row_end)
                *reinterpret_cast<uint4*>(GU + (size_t)row * p.N + gcol + 8 * k) = val;
            }
            __syncwarp();
          }
        }
      } else if constexpr (TF32) {
        // f32 Y = hi*hi accumulator + cross-term accumulator, 32 columns per
        // step through the same staging as store_y_block.
        float* Y = reinterpret_cast<float*>(p.out) + (size_t)nb * C::BN;
        float4* wst4 = reinterpret_cast<float4*>(wst);
#pragma unroll 1
        for (int c0 = cb; c0 < ce; c0 += 32) {
          uint32_t v[32], w[32];
          tmem_ld32(acc + c0, v);
          tmem_ld32(acc + C::BN + c0, w);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 8; ++k)
            wst4[lane * 8 + (k ^ (lane & 7))] = make_float4(
                __uint_as_float(v[4 * k]) + __uint_as_float(w[4 * k]),
                __uint_as_float(v[4 * k + 1]) + __uint_as_float(w[4 * k + 1]),
                __uint_as_float(v[4 * k + 2]) + __uint_as_float(w[4 * k + 2]),
                __uint_as_float(v[4 * k + 3]) + __uint_as_float(w[4 * k + 3]));
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (int)(lane >> 3);
            const int k = (int)(lane & 7);
            const float4 val = wst4[r * 8 + (k ^ (r & 7))];
            const int row = wrow0 + r;
            if (row < row_end && c0 + 4 * k < ncol)
              *reinterpret_cast<float4*>(Y + (size_t)row * p.N + c0 + 4 * k) = val;
          }
          __syncwarp();
        }
      } else if (p.scatter.on) {
        // Destination of row wrow0 + lane: the source rank whose rows of
        // this expert cover it, at the row it came from.
        const int R = wrow0 + (int)lane;
        uint8_t* row_ptr = nullptr;
        if (R < row_end) {
          const int4* rc = p.scatter.recv + (size_t)cur.e * p.scatter.world;
          for (int sr = 0; sr < p.scatter.world; ++sr) {
            const int4 q = rc[sr];
            if (R >= q.x && R < q.x + q.y) {
              row_ptr = p.scatter.base[q.w] + p.scatter.off + (size_t)(q.z + (R - q.x)) * (size_t)p.N * 4;
              break;
            }
          }
        }
        float4* wst4 = reinterpret_cast<float4*>(wst);
#pragma unroll 1
        for (int c0 = 0; c0 < ncol; c0 += 32)
          store_y_rows(acc + c0, wst4, row_ptr, nb * C::TILE_N + c0, lane, mul, p.N);
      } else if (BFP8) {
        // f32 Y rows scaled back by 2^-k, through the same staging as below.
        float* Y = reinterpret_cast<float*>(p.out);
        float4* wst4 = reinterpret_cast<float4*>(wst);
        const int R = wrow0 + (int)lane;
        uint8_t* row_ptr = R < row_end ? reinterpret_cast<uint8_t*>(Y + (size_t)R * p.N) : nullptr;
#pragma unroll 1
        for (int c0 = 0; c0 < ncol; c0 += 32)
          store_y_rows(acc + c0, wst4, row_ptr, nb * C::BN + c0, lane, mul, p.N);
      } else {
        float* Y = reinterpret_cast<float*>(p.out);
        float4* wst4 = reinterpret_cast<float4*>(wst);
#pragma unroll 1
        for (int c0 = 0; c0 < ncol; c0 += 32)
          store_y_block<0>(acc + c0, wst4, Y + (size_t)nb * C::TILE_N, wrow0, row_end, c0, lane, false, p.N, ncol);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_cta(acc_empty_l + ab * 8);
    }
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

}  // namespace moe
