// Fused expert MLP on CTA pairs (2-SM tcgen05 MMA, cluster of 2), sm_100a.
//
// Same dataflow as fused_mlp_small_kernel (MMA1 -> TMEM -> GELU -> TMEM ->
// MMA2, the hidden block never leaves the SMs), but a pair of CTAs on two SMs
// computes a 256-row tile: the leader CTA issues tcgen05.mma.cta_group::2
// with M = 256, each CTA supplies its own 128 rows of X (A operand) and HALF
// of every weight tile (B operand, split along N), and each CTA's TMEM holds
// the accumulators of its own rows.  Per SM this halves the weight bytes that
// stream from L2 for the same tensor work -- the limiter of the single-CTA
// kernel, which re-streams a whole expert's weights for every 128 rows.
//
//   3xTF32 (D <= 128): rank 0 holds the tf32 hi plane of the W_up chunk and
//     rank 1 the lo plane, so MMA1's concatenated N = 2*BF operand
//     [W_hi | W_lo] is read half from each SM; the X_lo pass uses the same
//     operand (it also adds the x_lo*w_lo term).  W_down: each CTA holds half
//     of the D rows of both planes.
//   bf16: W_up / W_down chunks split into 64-wide MN halves.
//
// Synchronisation: operand stages are counted on the leader's `full`
// barriers (the peer's TMA loads signal them across the pair); MMA
// completion is multicast to both CTAs (tcgen05.commit ... multicast);
// each GELU / epilogue warp of either CTA arrives once on the leader's
// h_ready / x_ready / y_empty barriers.  No TMA multicast is used: every CTA
// loads its own tiles.
#pragma once
#include "fused_small.cuh"

namespace moe {

template <int MODE, int D, int BF>
struct PairCfg {
  static constexpr bool kTF32 = MODE == kModeTF32x3;
  static constexpr int ESZ = kTF32 ? 4 : 2;
  static constexpr int ATOM = 128 / ESZ;
  static constexpr int KI = 32 / ESZ;
  static constexpr int PL = kTF32 ? 2 : 1;
  static constexpr int BM = 128;   // rows per CTA
  static constexpr int XBOX = BM * 128;
  static constexpr int X_PLANE = (D / ATOM) * XBOX;
  static constexpr int X_BYTES = X_PLANE;
  // MMA1 stage (per CTA): all of D in KB1 k-boxes.
  //   tf32: one plane, BF rows (K-major) per k-box.  bf16: 64 f-columns (one
  //   MN atom) x 64 d-rows per k-box.
  static constexpr int KB1 = D / ATOM;
  static constexpr int S1_BOX = kTF32 ? BF * 128 : ATOM * 128;
  static constexpr int S1_BYTES = KB1 * S1_BOX;
  // MMA2 stage (per CTA): all of BF in KB2 k-boxes.
  //   tf32: both planes, D/2 rows each per k-box.  bf16: D/2 d-columns (D/128
  //   MN atoms) x 64 f-rows per k-box.
  static constexpr int KB2 = BF / ATOM;
  static constexpr int S2_PLANE = (D / 2) * 128;  // tf32: one plane of one k-box
  static constexpr int S2_ATOMS = kTF32 ? 1 : (D / 2) / ATOM;
  static constexpr int S2_BOX = kTF32 ? PL * S2_PLANE : S2_ATOMS * ATOM * 128;
  static constexpr int S2_BYTES = KB2 * S2_BOX;
  static constexpr int STAGE = S1_BYTES > S2_BYTES ? S1_BYTES : S2_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int Y_STAGE = 8 * 32 * 32 * 4;  // 4 KB per epilogue warp for coalesced Y stores
  static constexpr int NS_FIT = (kMaxSmemPerBlock - 1024 - BAR_BYTES - X_BYTES - Y_STAGE) / STAGE;
  static constexpr int NS = NS_FIT > 8 ? 8 : NS_FIT;
  static constexpr int SMEM = 1024 + X_BYTES + NS * STAGE + Y_STAGE + BAR_BYTES;
  static constexpr int HCOLS = PL * BF;
  static constexpr int XLO_COL = D + 2 * HCOLS;
  static constexpr int TMEM_USED = XLO_COL + (kTF32 ? D : 0);
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t FMT = kTF32 ? kFmtTF32 : kFmtBF16;
  static constexpr uint32_t B_MN = kTF32 ? 0u : 1u;
  static constexpr uint32_t IDESC1 = make_idesc(FMT, 256, kTF32 ? 2 * BF : BF, 0, B_MN);
  static constexpr uint32_t IDESC2 = make_idesc(FMT, 256, D, 0, B_MN);
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + EPI_WARPS * 32;
  static constexpr int PAIR_ARRIVALS = 2 * EPI_WARPS;  // one per epilogue warp of each CTA
  static constexpr uint32_t TX1 = 2 * S1_BYTES;        // both CTAs' halves
  static constexpr uint32_t TX2 = 2 * S2_BYTES;

  static_assert(NS >= 2, "shared memory too small for two ring stages");
  static_assert(TMEM_USED <= TMEM_COLS, "TMEM budget");
  static_assert(!kTF32 || (2 * BF <= 256 && D <= 128), "tf32 pair tile");
  static_assert(kTF32 || (BF == 128 && D % 128 == 0 && D <= 256), "bf16 pair tile");
  static_assert(SMEM <= kMaxSmemPerBlock, "shared memory budget");
};

template <int MODE, int D, int BF>
__global__ void __launch_bounds__(64 + 256, 1)
    fused_mlp_pair_kernel(const __grid_constant__ FusedMaps maps, const FusedParams p) {
  using C = PairCfg<MODE, D, BF>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* xbuf = smem;
  uint8_t* ring = smem + C::X_BYTES;
  float4* ystage = reinterpret_cast<float4*>(ring + C::NS * C::STAGE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + C::NS * C::STAGE + C::Y_STAGE);
  uint64_t* full = bars;                // [NS]  leader: both halves landed
  uint64_t* empty = bars + C::NS;       // [NS]  both: stage consumed (multicast)
  uint64_t* x_full = bars + 2 * C::NS;  // local: raw X landed
  uint64_t* x_ready = x_full + 1;       // leader: both X tiles split
  uint64_t* x_empty = x_full + 2;       // both: last MMA1 of the unit done (multicast)
  uint64_t* h_full = x_full + 3;        // [2] both: MMA1 done (multicast)
  uint64_t* h_ready = x_full + 5;       // [2] leader: both GELU halves written
  uint64_t* y_full = x_full + 7;        // both: last MMA2 done (multicast)
  uint64_t* y_empty = x_full + 8;       // leader: both Y tiles drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_full + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();  // 0 = leader (issues the MMAs)
  const int pair = (int)(blockIdx.x >> 1);
  const int npairs = (int)(gridDim.x >> 1);
  constexpr uint16_t kBoth = 0x3;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_ready, C::PAIR_ARRIVALS);
    mbar_init(x_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(h_full + i, 1);
      mbar_init(h_ready + i, C::PAIR_ARRIVALS);
    }
    mbar_init(y_full, 1);
    mbar_init(y_empty, C::PAIR_ARRIVALS);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.x[0]);
    tma_prefetch_desc(&maps.wu[0]);
    tma_prefetch_desc(&maps.wd[0]);
    if (C::kTF32) {
      tma_prefetch_desc(&maps.wu[1]);
      tma_prefetch_desc(&maps.wd[1]);
    }
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int S = p.splits;
  const int NCH = p.chunks_per_split;
  // Leader-side barrier addresses in the cluster window.
  const uint32_t x_ready_l = mapa_shared(smem_u32(x_ready), 0);
  const uint32_t h_ready_l = mapa_shared(smem_u32(h_ready), 0);
  const uint32_t y_empty_l = mapa_shared(smem_u32(y_empty), 0);
  const uint32_t full_l0 = mapa_shared(smem_u32(full), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      BlockCursorT<8> cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ui = 0;
      bool ok = true;
      const uint64_t pol_w = l2_policy_evict_last();
      auto next_stage = [&]() -> bool {
        return mbar_wait(empty + stage, phase ^ 1u, abort_flag, p.status);
      };
      auto advance = [&]() {
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int u = pair; ok; u += npairs, ++ui) {
        const int gb = u / S;  // global 256-row pair-block
        if (!cur.seek(gb, p.group_sizes, p.E, p.M)) break;
        const int e = cur.e;
        const int row0 = cur.row_begin + (gb - cur.blk_begin) * 256 + (int)rank * C::BM;
        const int fch0 = (u % S) * NCH;
        if (!mbar_wait(x_empty, (ui & 1u) ^ 1u, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(x_full, C::X_PLANE);
        for (int s = 0; s < D / C::ATOM; ++s) tma_load_2d(xbuf + s * C::XBOX, &maps.x[0], x_full, s * C::ATOM, row0);
        {
          BlockCursorT<8> nxt = cur;
          const int u_next = u + npairs;
          if (nxt.seek(u_next / S, p.group_sizes, p.E, p.M)) {
            const int nrow0 = nxt.row_begin + (u_next / S - nxt.blk_begin) * 256 + (int)rank * C::BM;
            for (int s = 0; s < D / C::ATOM; ++s) tma_prefetch_l2_2d(&maps.x[0], s * C::ATOM, nrow0);
          }
        }
        auto load_s1 = [&](int j) -> bool {
          if (!next_stage()) return false;
          uint8_t* st = ring + stage * C::STAGE;
          const uint32_t bar = full_l0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(full + stage, C::TX1);
          const int f0 = (fch0 + j) * BF;
          for (int kb = 0; kb < C::KB1; ++kb) {
            if constexpr (C::kTF32) {
              // Plane `rank` of W_up^T (rows (e, f), K = d): box {32, BF}.
              tma_load_2d_pair(st + kb * C::S1_BOX, &maps.wu[rank], bar, kb * C::ATOM, e * p.F + f0, pol_w);
            } else {
              // f-columns [f0 + 64 rank, +64) of W_up (rows (e, d)): box {64, 64}.
              tma_load_2d_pair(st + kb * C::S1_BOX, &maps.wu[0], bar, f0 + (int)rank * C::ATOM,
                               e * D + kb * C::ATOM, pol_w);
            }
          }
          advance();
          return true;
        };
        auto load_s2 = [&](int j) -> bool {
          if (!next_stage()) return false;
          uint8_t* st = ring + stage * C::STAGE;
          const uint32_t bar = full_l0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(full + stage, C::TX2);
          const int f0 = (fch0 + j) * BF;
          for (int kb = 0; kb < C::KB2; ++kb) {
            if constexpr (C::kTF32) {
              // d-rows [D/2 rank, +D/2) of both W_down^T planes: box {32, D/2}.
              for (int pl = 0; pl < C::PL; ++pl)
                tma_load_2d_pair(st + kb * C::S2_BOX + pl * C::S2_PLANE, &maps.wd[pl], bar, f0 + kb * C::ATOM,
                                 e * D + (int)rank * (D / 2), pol_w);
            } else {
              // d-columns [D/2 rank, +D/2) of W_down (rows (e, f)): 64-wide boxes.
              for (int a = 0; a < C::S2_ATOMS; ++a)
                tma_load_2d_pair(st + kb * C::S2_BOX + a * C::ATOM * 128, &maps.wd[0], bar,
                                 (int)rank * (D / 2) + a * C::ATOM, e * p.F + f0 + kb * C::ATOM, pol_w);
            }
          }
          advance();
          return true;
        };
        for (int j = 0; j < NCH && ok; ++j) {
          ok = load_s1(j);
          if (ok && j > 0) ok = load_s2(j - 1);
        }
        if (ok) ok = load_s2(NCH - 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader, whole warp)
    if (rank == 0) {
      BlockCursorT<8> cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ui = 0;
      uint32_t hcount = 0;
      bool ok = true;
      const uint32_t t_y = tmem_base;
      const uint64_t x_desc0 = make_sdesc(smem_u32(xbuf), 16, 1024);
      auto wait_full = [&]() -> bool {
        if (!mbar_wait_warp(full + stage, phase, abort_flag, p.status)) return false;
        tc_fence_after();
        return true;
      };
      auto release = [&]() {
        umma_commit_pair(empty + stage, kBoth);
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int u = pair; ok; u += npairs, ++ui) {
        const int gb = u / S;
        if (!cur.seek(gb, p.group_sizes, p.E, p.M)) break;
        if (!mbar_wait_warp(x_ready, ui & 1u, abort_flag, p.status)) break;
        tc_fence_after();
        auto mma1 = [&](int j) -> bool {
          const uint32_t hb = (hcount + j) & 1u;
          const uint32_t d_tmem = tmem_base + D + hb * C::HCOLS;
          if (!wait_full()) return false;
          const uint32_t st = smem_u32(ring + stage * C::STAGE);
          const uint64_t st_desc = C::kTF32 ? make_sdesc(st, 16, 1024) : make_sdesc(st, C::ATOM * 128, 1024);
#pragma unroll
          for (int kb = 0; kb < C::KB1; ++kb) {
#pragma unroll
            for (int ki = 0; ki < C::ATOM / C::KI; ++ki) {
              const uint64_t a0 = x_desc0 + (uint64_t)((kb * C::XBOX + ki * 32) >> 4);
              const uint64_t b0 = C::kTF32 ? st_desc + (uint64_t)((kb * C::S1_BOX + ki * 32) >> 4)
                                           : st_desc + (uint64_t)((kb * C::S1_BOX + ki * (C::KI * 128)) >> 4);
              const uint32_t acc0 = (kb > 0 || ki > 0) ? 1u : 0u;
              umma_ss_pair<C::kTF32 ? Kind::TF32 : Kind::F16>(d_tmem, a0, b0, C::IDESC1, acc0);
              if constexpr (C::kTF32) {
                const uint32_t xlo = tmem_base + C::XLO_COL + kb * C::ATOM + ki * C::KI;
                umma_ts_pair<Kind::TF32>(d_tmem, xlo, b0, C::IDESC1, 1u);
              }
            }
          }
          release();
          umma_commit_pair(h_full + hb, kBoth);
          return true;
        };
        auto mma2 = [&](int j) -> bool {
          const uint32_t hb = (hcount + j) & 1u;
          const uint32_t use = (hcount + j) >> 1;
          if (!mbar_wait_warp(h_ready + hb, use & 1u, abort_flag, p.status)) return false;
          tc_fence_after();
          if (j == 0) {
            if (!mbar_wait_warp(y_empty, (ui & 1u) ^ 1u, abort_flag, p.status)) return false;
            tc_fence_after();
          }
          const uint32_t h_tmem = tmem_base + D + hb * C::HCOLS;
          if (!wait_full()) return false;
          const uint32_t st = smem_u32(ring + stage * C::STAGE);
          const uint64_t st_desc = C::kTF32 ? make_sdesc(st, 16, 1024) : make_sdesc(st, C::ATOM * 128, 1024);
#pragma unroll
          for (int kb = 0; kb < C::KB2; ++kb) {
#pragma unroll
            for (int ki = 0; ki < C::ATOM / C::KI; ++ki) {
              const uint32_t kcol = (kb * C::ATOM + ki * C::KI) * C::ESZ / 4;
              const uint32_t acc0 = (j > 0 || kb > 0 || ki > 0) ? 1u : 0u;
              if constexpr (C::kTF32) {
                const uint64_t bh = st_desc + (uint64_t)((kb * C::S2_BOX + ki * 32) >> 4);
                const uint64_t bl = st_desc + (uint64_t)((kb * C::S2_BOX + C::S2_PLANE + ki * 32) >> 4);
                umma_ts_pair<Kind::TF32>(t_y, h_tmem + kcol, bh, C::IDESC2, acc0);
                umma_ts_pair<Kind::TF32>(t_y, h_tmem + kcol, bl, C::IDESC2, 1u);
                umma_ts_pair<Kind::TF32>(t_y, h_tmem + BF + kcol, bh, C::IDESC2, 1u);
              } else {
                const uint64_t b0 = st_desc + (uint64_t)((kb * C::S2_BOX + ki * (C::KI * 128)) >> 4);
                umma_ts_pair<Kind::F16>(t_y, h_tmem + kcol, b0, C::IDESC2, acc0);
              }
            }
          }
          release();
          return true;
        };
        for (int j = 0; j < NCH && ok; ++j) {
          ok = mma1(j);
          if (ok && j == NCH - 1) umma_commit_pair(x_empty, kBoth);
          if (ok && j > 0) ok = mma2(j - 1);
        }
        if (ok) ok = mma2(NCH - 1);
        if (ok) umma_commit_pair(y_full, kBoth);
        hcount += NCH;
      }
    }
  } else {
    // ------------------------------------------------------------ GELU / epilogue warps (both CTAs)
    const uint32_t q = warp & 3u;
    const uint32_t half = (warp - 2u) >> 2;
    const uint32_t lane_base = tmem_base + ((q * 32u) << 16);
    const int erow = (int)(q * 32u + lane);
    const int etid = (int)threadIdx.x - 64;
    constexpr int NT = C::EPI_WARPS * 32;

    if (etid == 0 && blockIdx.x == 0) {
      for (int e = 0; e < p.E; ++e)
        if (__ldg(p.group_sizes + e) < 0) atomicOr(p.status, kStatusBadGroupSize);
    }
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

    BlockCursorT<8> cur;
    uint32_t hcount = 0;
    uint32_t ui = 0;
    bool ok = true;
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
      bool r = mbar_wait(bar, parity, abort_flag, p.status);
      return __all_sync(0xffffffffu, r);
    };
    // One arrival per warp on a leader barrier once every lane's prior
    // TMEM / shared-memory writes are complete.
    auto warp_arrive_leader = [&](uint32_t leader_bar) {
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_cta(leader_bar);
    };
    auto prep_x = [&](uint32_t uidx) -> bool {
      if (!warp_wait(x_full, uidx & 1u)) return false;
      if constexpr (C::kTF32) {
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
      }
      tc_fence_before();
      warp_arrive_leader(x_ready_l);
      return true;
    };

    int u = pair;
    bool have = cur.seek(u / S, p.group_sizes, p.E, p.M);
    if (have) ok = prep_x(0);
    while (have && ok) {
      const int gb = u / S;
      const int row0 = cur.row_begin + (gb - cur.blk_begin) * 256 + (int)rank * C::BM;
      const int row_end = cur.row_begin + cur.rows;
      for (int j = 0; j < NCH && ok; ++j) {
        const uint32_t hb = (hcount + j) & 1u;
        const uint32_t use = (hcount + j) >> 1;
        if (!warp_wait(h_full + hb, use & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t hcol = D + hb * C::HCOLS;
        if constexpr (C::kTF32) {
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
          constexpr int CW = BF / 2;
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
        warp_arrive_leader(h_ready_l + hb * 8);
      }
      if (!ok) break;
      hcount += NCH;

      const int u_next = u + npairs;
      BlockCursorT<8> nxt = cur;
      const bool have_next = nxt.seek(u_next / S, p.group_sizes, p.E, p.M);
      if (have_next) {
        ok = prep_x(ui + 1);
        if (!ok) break;
      }

      if (!warp_wait(y_full, ui & 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float4* wstage = ystage + (warp - 2u) * 256u;
#pragma unroll 1
      for (int c0 = half * (D / 2); c0 < (int)(half + 1) * (D / 2); c0 += 32)
        store_y_block<D>(lane_base + c0, wstage, p.y, row0 + (int)(q * 32u), row_end, c0, lane, p.atomic_out != 0);
      tc_fence_before();
      warp_arrive_leader(y_empty_l);

      u = u_next;
      cur = nxt;
      have = have_next;
      ++ui;
    }
  }

  tc_fence_before();
  cluster_sync();  // the leader's last MMAs touched both CTAs' TMEM / smem
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

}  // namespace moe
