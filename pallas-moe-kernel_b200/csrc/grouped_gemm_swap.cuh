// Grouped GEMM with e4m3 block-scaled weights for small experts (a few
// hundred rows each, e.g. 256 experts x top-8 of 8192 tokens), sm_100a.
//
// The row-tiled kernel (grouped_gemm.cuh) runs 256-row pair tiles, so an
// expert of 270 rows costs two tiles: about a third of its MMA rows are
// padding, and each tile decodes the expert's weights again.  Here the roles
// are swapped: per (expert, 256-feature block) one "super-tile" computes
//
//   out^T[features, tokens] = W^T[features, K] . X^T[K, tokens]
//
// with the decoded weights as the MMA's A operand (M = 256 features over the
// CTA pair, MN-major: the weights' own layout, the same 16-bit tile the
// converters already produce) and the expert's tokens as B (K-major rows of X
// or H), N = the token count rounded up to 32.  A super-tile holds up to 384
// tokens in two chunks (N <= 256 and N <= 128): each decoded weight stage
// feeds both chunks' MMAs.  Padding drops to < 32 rows per chunk and the
// weights are decoded once per 384 tokens.
//
// TMEM: two 256-column accumulator buffers, handed out in order -- a
// one-chunk super-tile takes the next buffer (so consecutive tiles
// double-buffer), a two-chunk one takes the next two.  The accumulator's lanes
// are features and its columns tokens, so the epilogue writes every token row
// with the warp's 32 consecutive features (coalesced).
//
// Warp roles as in grouped_gemm_pair_kernel with e4m3 weights: warp 0 TMA
// producer of X rows (both CTAs), warp 1 TMEM owner + MMA issuer (leader),
// warps 2..5 epilogue, warps 6..13 converters (e4m3 -> bf16 / f16, two groups on
// alternate K steps), warp 14 producer of the raw e4m3 ring.
//
// Token rows arrive in as few TMA boxes as possible (one 128-row box for a
// full chunk-0 half, else a 64-row box plus 32-row boxes): the issue of the
// row loads, not their bytes, limited the K step with 32-row boxes only
// (four box loads per K step: 870 cycles per step against 760 with one, at
// uniform 256-token experts).
#pragma once
#include "grouped_gemm.cuh"

namespace moe {

// Tensor maps of the super-tile kernel: the token rows (X, or H for the down
// GEMM) as [M, K] 16-bit rows (bf16 X, f16 H) with 32-, 64- and 128-row boxes of one 128-byte swizzle
// row each, and the e4m3 weights as [E][K][N] bytes, box {128, 64, 1}.
struct SwapMaps {
  CUtensorMap x32, x64, x128;
  CUtensorMap w;
};

template <int EPI>
struct SwapCfg {
  static_assert(EPI == 0 || EPI == 1, "GELU -> H or f32 Y");
  static constexpr int FM = 128;                     // features per CTA (MMA M = 256 per pair)
  static constexpr int BK = 64;                      // K per stage (one 128-byte row of 16-bit values)
  static constexpr int N0 = 256, N1 = 128;           // tokens of chunk 0 / chunk 1 (MMA N)
  static constexpr int TOKENS = N0 + N1;             // tokens per super-tile
  static constexpr int A_BYTES = FM * BK * 2;        // 16 KB decoded weights (MN-major)
  static constexpr int B0_BYTES = (N0 / 2) * BK * 2; // 16 KB: 128 token rows per CTA (K-major)
  static constexpr int B1_BYTES = (N1 / 2) * BK * 2; // 8 KB: 64 token rows per CTA
  static constexpr int STAGE = A_BYTES + B0_BYTES + B1_BYTES;  // 40 KB
  static constexpr int NS = 4;
  static constexpr int B8_BYTES = FM * BK;           // 8 KB raw e4m3 tile
  static constexpr int NR = 8;
  static constexpr int XBOX = 32;                    // token rows of the smallest TMA box (4 KB)
  static_assert(N0 / 2 == 4 * XBOX && N1 / 2 == 2 * XBOX, "chunk halves of 4 and 2 small boxes");
  static constexpr int EPI_WARPS = 4;
  static constexpr int CVT_WARPS = 8;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = 1024 + NS * STAGE + NR * B8_BYTES + BAR_BYTES;
  static constexpr int TMEM_COLS = 512;              // two 256-column accumulator buffers
  static constexpr int RAW_WARP = 2 + EPI_WARPS + CVT_WARPS;
  static constexpr int THREADS = 64 + (EPI_WARPS + CVT_WARPS) * 32 + 32;
  static_assert(SMEM <= kMaxSmemPerBlock, "shared memory budget");
  // The two converter groups take alternate K steps (g even / odd).  With an
  // even ring depth every use of a raw stage falls to the same group, which
  // consumed the previous use, so its parity wait on raw_full can never see a
  // phase two uses old as complete.  With an odd depth the groups share the
  // stages and a group can run two phases ahead (a build with NR = 3 decoded
  // stale tiles).
  static_assert(NS % 2 == 0 && NR % 2 == 0, "converter groups need even ring depths (mbarrier parity aliasing)");
};

// Super-tile walk: global tile index -> (expert, token super-tile, feature
// block), feature block fastest (the pairs running at once share the
// expert's X rows in L2); monotone in the tile index.
struct SwapCursor {
  int e = -1;
  int t_begin = 0;   // first global tile of expert e
  int ntiles = 0;    // tiles of expert e
  int row_begin = 0;
  int rows = 0;

  __device__ __forceinline__ bool seek(int t, const int32_t* gs, int E, int M, int nfb, int per_tile) {
    while (t >= t_begin + ntiles) {
      t_begin += ntiles;
      row_begin += rows;
      if (++e >= E) return false;
      int g = __ldg(gs + e);
      g = g < 0 ? 0 : g;
      const int rem = M - row_begin;
      g = g > rem ? (rem > 0 ? rem : 0) : g;
      rows = g;
      ntiles = ((g + per_tile - 1) / per_tile) * nfb;
    }
    return true;
  }
};

struct SwapTile {
  int fb;        // feature block (256 features)
  int tok0;      // first token row of the super-tile
  int n[2];      // real tokens of chunk 0 / 1
  int nr[2];     // MMA N of chunk 0 / 1 (n rounded up to 32; 0 = no chunk)
  int chunks;
};
template <class C>
__device__ __forceinline__ SwapTile swap_tile(const SwapCursor& cur, int t, int nfb) {
  SwapTile s;
  const int l = t - cur.t_begin;
  const int st = l / nfb;
  s.fb = l - st * nfb;
  s.tok0 = cur.row_begin + st * C::TOKENS;
  const int rem = cur.rows - st * C::TOKENS;
  s.n[0] = rem < C::N0 ? rem : C::N0;
  s.n[1] = rem - s.n[0] < C::N1 ? rem - s.n[0] : C::N1;
  s.n[1] = s.n[1] < 0 ? 0 : s.n[1];
  // N in steps of 32 (16 token rows from each CTA of the pair): a shape
  // every 2-SM M = 256 kind::f16 MMA accepts.
  s.nr[0] = (s.n[0] + 31) & ~31;
  s.nr[1] = (s.n[1] + 31) & ~31;
  s.chunks = s.n[1] > 0 ? 2 : 1;
  return s;
}

template <int EPI>
__global__ void __launch_bounds__(SwapCfg<EPI>::THREADS, 1)
    grouped_gemm_swap_kernel(const __grid_constant__ SwapMaps maps, const GemmParams p) {
  using C = SwapCfg<EPI>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* ring = smem;                              // [NS] {A 16-bit | B chunk 0 | B chunk 1}
  uint8_t* rawring = ring + C::NS * C::STAGE;        // [NR] raw e4m3 weight tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(rawring + C::NR * C::B8_BYTES);
  uint64_t* full = bars;                  // [NS] leader: producer + converters of both CTAs
  uint64_t* empty = bars + C::NS;         // [NS] both (multicast commit)
  uint64_t* acc_full = bars + 2 * C::NS;  // [2] both (multicast commit)
  uint64_t* acc_empty = acc_full + 2;     // [2] leader (epilogue warps of both CTAs)
  uint64_t* raw_full = acc_full + 4;      // [NR] local
  uint64_t* raw_empty = raw_full + C::NR; // [NR] local
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(raw_empty + C::NR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1);
  const int npairs = (int)(gridDim.x >> 1);
  constexpr uint16_t kBoth = 0x3;
  const int nfb = (p.N + 255) / 256;
  const int nk = (p.K + C::BK - 1) / C::BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(full + i, 1 + 2 * (C::CVT_WARPS / 2));
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
    tma_prefetch_desc(&maps.x32);
    tma_prefetch_desc(&maps.x64);
    tma_prefetch_desc(&maps.x128);
    tma_prefetch_desc(&maps.w);
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_l0 = mapa_shared(smem_u32(full), 0);
  const uint32_t acc_empty_l = mapa_shared(smem_u32(acc_empty), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ token rows (B) producer (both CTAs)
    if (lane == 0) {
      SwapCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol = l2_policy_evict_last();
      bool ok = true;
      for (int t = pair; ok; t += npairs) {
        if (!cur.seek(t, p.group_sizes, p.E, p.M, nfb, C::TOKENS)) break;
        const SwapTile s = swap_tile<C>(cur, t, nfb);
        // This CTA supplies tokens [r nr/2, (r + 1) nr/2) of each chunk:
        // 32 nbox rows (nr/2 rounded up to 32, at most the chunk's region);
        // both CTAs' bytes land on the leader's barrier.
        int nbox[2], rowc[2];
        uint32_t tx = 0;
        for (int c = 0; c < 2; ++c) {
          const int half = s.nr[c] / 2;
          nbox[c] = (half + C::XBOX - 1) / C::XBOX;
          rowc[c] = s.tok0 + (c == 0 ? 0 : C::N0) + (int)rank * half;
          tx += 2u * (uint32_t)nbox[c] * (C::XBOX * 128);
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + stage * C::STAGE;
          const uint32_t bar = full_l0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(full + stage, tx);
          for (int c = 0; c < 2; ++c) {
            // 4 boxes of 32 rows -> one of 128; 2 or 3 -> one of 64 (+ one of 32).
            uint8_t* d = st + C::A_BYTES + (c == 0 ? 0 : C::B0_BYTES);
            int nb = nbox[c], row = rowc[c];
            if (nb == 4) {
              tma_load_2d_pair(d, &maps.x128, bar, kb * C::BK, row, pol);
              nb = 0;
            } else if (nb >= 2) {
              tma_load_2d_pair(d, &maps.x64, bar, kb * C::BK, row, pol);
              d += 2 * (C::XBOX * 128);
              row += 2 * C::XBOX;
              nb -= 2;
            }
            if (nb == 1) tma_load_2d_pair(d, &maps.x32, bar, kb * C::BK, row, pol);
          }
          if (++stage == C::NS) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader, whole warp)
    if (rank == 0) {
      SwapCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t u = 0;            // accumulator buffers handed out so far
      uint32_t use0 = 0, use1 = 0;  // uses of buffer 0 / 1 so far
      for (int t = pair;; t += npairs) {
        if (!cur.seek(t, p.group_sizes, p.E, p.M, nfb, C::TOKENS)) break;
        const SwapTile s = swap_tile<C>(cur, t, nfb);
        const uint32_t b0 = u & 1u, b1 = b0 ^ 1u;  // buffers of chunk 0 / chunk 1
        bool ok = mbar_wait_warp(acc_empty + b0, ((b0 ? use1 : use0) & 1u) ^ 1u, abort_flag, p.status);
        if (ok && s.chunks == 2)
          ok = mbar_wait_warp(acc_empty + b1, ((b1 ? use1 : use0) & 1u) ^ 1u, abort_flag, p.status);
        if (!ok) break;
        tc_fence_after();
        // up GEMM: bf16 operands (the caller's X); down GEMM: f16 (H as the up
        // GEMM stored it, weights decoded to f16).
        constexpr uint32_t fmt = EPI == 1 ? kFmtF16 : kFmtBF16;
        const uint32_t idesc0 = make_idesc(fmt, 256, (uint32_t)s.nr[0], 1, 0);
        const uint32_t idesc1 = make_idesc(fmt, 256, (uint32_t)(s.nr[1] ? s.nr[1] : 32), 1, 0);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait_warp(full + stage, phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(ring + stage * C::STAGE);
          const uint64_t a_desc = make_sdesc(st, 64 * 128, 1024);                  // MN-major weights
          const uint64_t b0_desc = make_sdesc(st + C::A_BYTES, 16, 1024);         // K-major tokens
          const uint64_t b1_desc = make_sdesc(st + C::A_BYTES + C::B0_BYTES, 16, 1024);
#pragma unroll
          for (int ki = 0; ki < C::BK / 16; ++ki) {
            const uint64_t ao = (uint64_t)((ki * 16 * 128) >> 4), bo = (uint64_t)((ki * 32) >> 4);
            const uint32_t acc = (kb > 0 || ki > 0) ? 1u : 0u;
            umma_ss_pair<Kind::F16>(tmem_base + b0 * 256u, a_desc + ao, b0_desc + bo, idesc0, acc);
            if (s.chunks == 2)
              umma_ss_pair<Kind::F16>(tmem_base + b1 * 256u, a_desc + ao, b1_desc + bo, idesc1, acc);
          }
          umma_commit_pair(empty + stage, kBoth);
          if (++stage == C::NS) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(acc_full + b0, kBoth);
        (b0 ? use1 : use0) += 1;
        if (s.chunks == 2) {
          umma_commit_pair(acc_full + b1, kBoth);
          (b1 ? use1 : use0) += 1;
        }
        u += (uint32_t)s.chunks;
      }
    }
  } else if (warp == (uint32_t)C::RAW_WARP) {
    // ------------------------------------------------------------ raw e4m3 weight producer (both CTAs)
    if (lane == 0) {
      SwapCursor cur;
      int rs = 0;
      uint32_t rph = 0;
      const uint64_t pol = l2_policy_evict_first();  // every weight tile is read once
      bool ok = true;
      for (int t = pair; ok; t += npairs) {
        if (!cur.seek(t, p.group_sizes, p.E, p.M, nfb, C::TOKENS)) break;
        const SwapTile s = swap_tile<C>(cur, t, nfb);
        const int f0 = s.fb * 256 + (int)rank * C::FM;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(raw_empty + rs, rph ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(raw_full + rs, C::B8_BYTES);
          tma_load_3d_hint(rawring + rs * C::B8_BYTES, &maps.w, raw_full + rs, f0, kb * C::BK, cur.e, pol);
          if (++rs == C::NR) {
            rs = 0;
            rph ^= 1u;
          }
        }
      }
    }
  } else if (warp >= 2u + C::EPI_WARPS) {
    // ------------------------------------------------------------ e4m3 -> bf16 (up) / f16 (down) converters (both CTAs)
    // As in grouped_gemm_pair_kernel: two groups of four warps on alternate K
    // steps; thread t of a group takes k-row t % 64 and half t / 64 of the
    // 128 features of this CTA, and writes the MN-major swizzled 16-bit tile
    // that is the MMA's A operand here.
    const int ct = (int)threadIdx.x - 64 - C::EPI_WARPS * 32;  // 0..255
    const int grp = ct >> 7;
    const int r = ct & 63, h = (ct >> 6) & 1;
    const int nkb_scale = (p.K + 127) / 128, nnb_scale = (p.N + 127) / 128;
    SwapCursor cur;
    uint32_t gk = 0;
    bool ok = true;
    for (int t = pair; ok; t += npairs) {
      if (!cur.seek(t, p.group_sizes, p.E, p.M, nfb, C::TOKENS)) break;
      const SwapTile s = swap_tile<C>(cur, t, nfb);
      const int f0 = s.fb * 256 + (int)rank * C::FM;
      const bool col_in = f0 / 128 < nnb_scale;
      const float* srow = p.b_scale + ((size_t)cur.e * nkb_scale) * nnb_scale + (col_in ? f0 / 128 : 0);
      const float s_lo = col_in && (int)lane < nkb_scale ? __ldg(srow + (size_t)lane * nnb_scale) : 0.f;
      const float s_hi = col_in && (int)lane + 32 < nkb_scale ? __ldg(srow + (size_t)(lane + 32) * nnb_scale) : 0.f;
      const float up = exp2i(fp8_tile_shift(p.b_scale, p.K, p.N, cur.e, s.fb, lane));
      for (int kb = grp; kb < nk; kb += 2) {
        const uint32_t g = gk + (uint32_t)kb;
        const int stage = (int)(g % C::NS), rs = (int)(g % C::NR);
        const uint32_t phase = (g / C::NS) & 1u, rph = (g / C::NR) & 1u;
        if (!mbar_wait_warp(raw_full + rs, rph, abort_flag, p.status) ||
            !mbar_wait_warp(empty + stage, phase ^ 1u, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const int kblk = (kb * C::BK) / 128;
        const float s_reg = __shfl_sync(0xffffffffu, kblk < 32 ? s_lo : s_hi, kblk & 31);
        const float sc = kblk < 64 ? s_reg : (col_in ? __ldg(srow + (size_t)kblk * nnb_scale) : 0.f);
        const E4m3Decoder<EPI == 1> dec(sc * up);
        const uint8_t* src = rawring + rs * C::B8_BYTES + r * 128;
        uint8_t* dst = ring + stage * C::STAGE + h * (64 * 128) + r * 128;
        const int rsw = r & 7;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int chunk = 4 * h + c;
          const uint4 v = *reinterpret_cast<const uint4*>(src + ((chunk ^ rsw) << 4));
          const uint2 b0 = dec(v.x), b1 = dec(v.y);
          const uint2 b2 = dec(v.z), b3 = dec(v.w);
          const int j0 = 2 * c, j1 = 2 * c + 1;
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
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Lane = feature (this warp's TMEM lane quadrant), column = token.
    const uint32_t q = warp & 3u;
    const uint32_t lane_base = tmem_base + ((q * 32u) << 16);
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
      const int etid = (int)threadIdx.x - 64;
      for (size_t i = (size_t)blockIdx.x * (C::EPI_WARPS * 32) + etid; i < n4;
           i += (size_t)gridDim.x * (C::EPI_WARPS * 32))
        base[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    SwapCursor cur;
    uint32_t u = 0;
    uint32_t use0 = 0, use1 = 0;
    for (int t = pair;; t += npairs) {
      if (!cur.seek(t, p.group_sizes, p.E, p.M, nfb, C::TOKENS)) break;
      const SwapTile s = swap_tile<C>(cur, t, nfb);
      const int f = s.fb * 256 + (int)rank * C::FM + (int)(q * 32u + lane);
      const bool f_in = f < p.N;
      const float mul = exp2i(-fp8_tile_shift(p.b_scale, p.K, p.N, cur.e, s.fb, lane));
      bool ok = true;
      for (int c = 0; c < s.chunks; ++c) {
        const uint32_t b = (u + (uint32_t)c) & 1u;
        if (!mbar_wait_warp(acc_full + b, (b ? use1 : use0) & 1u, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int tokc = s.tok0 + (c == 0 ? 0 : C::N0);
        const int nc = c == 0 ? s.n[0] : s.n[1];
        const uint32_t acc = lane_base + b * 256u;
#pragma unroll 1
        for (int j0 = 0; j0 < nc; j0 += 32) {
          uint32_t v[32];
          tmem_ld32(acc + (uint32_t)j0, v);
          tmem_ld_wait();
          const int jn = nc - j0 < 32 ? nc - j0 : 32;
          if constexpr (EPI == 1) {
            float* Y = reinterpret_cast<float*>(p.out) + (size_t)(tokc + j0) * p.N + f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < jn && f_in) Y[(size_t)j * p.N] = __uint_as_float(v[j]) * mul;
          } else {
            // H (f16, the down GEMM's operand): lanes 2i and 2i+1 hold features f, f+1; the even lane
            // stores both for token j, the odd lane both for token j+1.
            uint16_t* H = reinterpret_cast<uint16_t*>(p.out) + (size_t)(tokc + j0) * p.N + (f & ~1);
            const bool odd = lane & 1u;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float g0 = gelu_tanh_fast(__uint_as_float(v[j]) * mul);
              const float g1 = gelu_tanh_fast(__uint_as_float(v[j + 1]) * mul);
              const float o0 = __shfl_xor_sync(0xffffffffu, g0, 1);
              const float o1 = __shfl_xor_sync(0xffffffffu, g1, 1);
              const int jj = odd ? j + 1 : j;
              const uint32_t w = odd ? pack_f16x2_sat(o1, g1) : pack_f16x2_sat(g0, o0);
              if (jj < jn && f_in) *reinterpret_cast<uint32_t*>(H + (size_t)jj * p.N) = w;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_cta(acc_empty_l + b * 8);
        (b ? use1 : use0) += 1;
      }
      if (!ok) break;
      u += (uint32_t)s.chunks;
    }
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

}  // namespace moe
