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
//                toward zero to tf32 (19 bits) and a_lo = a - a_hi, which
//                keeps the result within ~1e-6 relative of f32 math.
//                Weights arrive pre-split (hi/lo planes, transposed to
//                K-major); X is split in shared memory by the GELU warps when
//                the tile is resident, else pre-split too.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2..5 GELU / epilogue (one TMEM lane quadrant each).
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
  int splits;            // F-splits per 128-row block
  int chunks_per_split;  // BF-wide chunks handled by one unit
  int atomic_out;        // 1: Y was zeroed, units reduce-add into it
  int* status;           // device status word (kStatus* bits)
};

template <int MODE, int D, int BF, bool X_RES>
struct FusedCfg {
  static constexpr bool kTF32 = MODE == kModeTF32x3;
  static constexpr int ESZ = kTF32 ? 4 : 2;
  static constexpr int ATOM = 128 / ESZ;  // elements in one 128-byte swizzle row
  static constexpr int KI = 32 / ESZ;     // K of one MMA instruction
  static constexpr int PL = kTF32 ? 2 : 1;
  static constexpr int BM = 128;
  static constexpr int SK = ATOM;                       // K rows per ring stage
  static constexpr int XBOX = BM * 128;                 // one X k-slice: 128 rows x 128 B
  static constexpr int X_PLANE = (D / ATOM) * XBOX;     // one full X plane
  static constexpr int X_BYTES = X_RES ? PL * X_PLANE : 0;
  static constexpr int S1_X = X_RES ? 0 : PL * XBOX;    // streamed X slice planes
  static constexpr int S1_WPLANE = BF * 128;            // one W_up slice plane
  static constexpr int S1_BYTES = S1_X + PL * S1_WPLANE;
  static constexpr int S2_WPLANE = D * 128;             // one W_down slice plane
  static constexpr int S2_BYTES = PL * S2_WPLANE;
  static constexpr int STAGE = S1_BYTES > S2_BYTES ? S1_BYTES : S2_BYTES;
  static constexpr int N1 = D / SK;   // ring stages per MMA1 chunk
  static constexpr int N2 = BF / SK;  // ring stages per MMA2 chunk
  static constexpr int BAR_BYTES = 256;
  static constexpr int NS_FIT = (kMaxSmemPerBlock - 1024 - BAR_BYTES - X_BYTES) / STAGE;
  static constexpr int NS = NS_FIT > 8 ? 8 : NS_FIT;
  static constexpr int SMEM = 1024 + X_BYTES + NS * STAGE + BAR_BYTES;
  // TMEM columns: Y accumulator [0, D); hidden buffer b at D + b * PL * BF
  // (accumulator / hi plane first, lo plane after it).
  static constexpr int HCOLS = PL * BF;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t FMT = kTF32 ? kFmtTF32 : kFmtBF16;
  static constexpr uint32_t B_MN = kTF32 ? 0u : 1u;  // bf16 weights are read MN-major
  static constexpr uint32_t IDESC1 = make_idesc(FMT, 128, BF, 0, B_MN);
  static constexpr uint32_t IDESC2 = make_idesc(FMT, 128, D, 0, B_MN);
  static constexpr uint32_t TX1 = S1_BYTES;
  static constexpr uint32_t TX2 = S2_BYTES;

  static_assert(NS >= 2, "shared memory too small for two ring stages");
  static_assert(D % SK == 0 && BF % SK == 0, "tile shape");
  static_assert(D + 2 * HCOLS <= TMEM_COLS, "TMEM budget");
  static_assert(D % 16 == 0 && D <= 256 && BF % 16 == 0 && BF <= 256, "UMMA N range");
  static_assert(SMEM <= kMaxSmemPerBlock, "shared memory budget");
};

// Monotone walk over (expert, 128-row block) pairs built from group sizes.
struct BlockCursor {
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
      nblk = (g + 127) >> 7;
    }
    return true;
  }
};

struct FusedMaps {
  CUtensorMap x[2];   // X planes (bf16: [0] only; tf32: hi, lo when pre-split)
  CUtensorMap wu[2];  // W_up operand planes
  CUtensorMap wd[2];  // W_down operand planes
};

template <int MODE, int D, int BF, bool X_RES>
__global__ void __launch_bounds__(192, 1)
    fused_mlp_small_kernel(const __grid_constant__ FusedMaps maps, const FusedParams p) {
  using C = FusedCfg<MODE, D, BF, X_RES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* xbuf = smem;
  uint8_t* ring = smem + C::X_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + C::NS * C::STAGE);
  uint64_t* full = bars;                 // [NS]
  uint64_t* empty = bars + C::NS;        // [NS]
  uint64_t* x_full = bars + 2 * C::NS;   // raw X landed
  uint64_t* x_ready = x_full + 1;        // X operand (split) ready for MMA
  uint64_t* x_empty = x_full + 2;        // last MMA1 of the unit finished
  uint64_t* h_full = x_full + 3;         // [2] MMA1 done -> GELU
  uint64_t* h_ready = x_full + 5;        // [2] GELU operand written -> MMA2
  uint64_t* y_full = x_full + 7;         // last MMA2 done -> epilogue
  uint64_t* y_empty = x_full + 8;        // epilogue drained Y_acc
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_full + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_ready, 128);
    mbar_init(x_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(h_full + i, 1);
      mbar_init(h_ready + i, 128);
    }
    mbar_init(y_full, 1);
    mbar_init(y_empty, 128);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      BlockCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ui = 0;
      bool ok = true;
      const uint64_t pol_w = l2_policy_evict_last();
      auto next_stage = [&]() -> bool {
        if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, p.status)) return false;
        return true;
      };
      auto advance = [&]() {
        if (++stage == C::NS) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int u = blockIdx.x; ok; u += gridDim.x, ++ui) {
        const int gb = u / S;
        if (!cur.seek(gb, p.group_sizes, p.E, p.M)) break;
        const int e = cur.e;
        const int row0 = cur.row_begin + (gb - cur.blk_begin) * C::BM;
        const int fch0 = (u % S) * NCH;
        if constexpr (X_RES) {
          if (!mbar_wait(x_empty, (ui & 1u) ^ 1u, abort_flag, p.status)) break;
          // Raw X (bf16 operand, or f32 to be split into hi/lo in place).
          mbar_arrive_expect_tx(x_full, C::X_PLANE);
          for (int s = 0; s < D / C::ATOM; ++s)
            tma_load_2d(xbuf + s * C::XBOX, &maps.x[0], x_full, s * C::ATOM, row0);
        }
        auto load_s1 = [&](int j, int s) -> bool {
          if (!next_stage()) return false;
          uint8_t* st = ring + stage * C::STAGE;
          mbar_arrive_expect_tx(full + stage, C::TX1);
          const int f0 = (fch0 + j) * BF;
          if constexpr (!X_RES) {
            for (int pl = 0; pl < C::PL; ++pl)
              tma_load_2d(st + pl * C::XBOX, &maps.x[pl], full + stage, s * C::ATOM, row0);
          }
          uint8_t* w = st + C::S1_X;
          if constexpr (C::kTF32) {
            // W_up^T planes: rows (e, f), K = d contiguous; box {32, BF}.
            for (int pl = 0; pl < C::PL; ++pl)
              tma_load_2d_hint(w + pl * C::S1_WPLANE, &maps.wu[pl], full + stage, s * C::ATOM, e * p.F + f0,
                               pol_w);
          } else {
            // W_up rows (e, d), N = f contiguous; box {64, 64} per 64-wide f block.
            for (int nb = 0; nb < BF / C::ATOM; ++nb)
              tma_load_2d_hint(w + nb * C::SK * 128, &maps.wu[0], full + stage, f0 + nb * C::ATOM,
                               e * D + s * C::SK, pol_w);
          }
          advance();
          return true;
        };
        auto load_s2 = [&](int j, int t) -> bool {
          if (!next_stage()) return false;
          uint8_t* st = ring + stage * C::STAGE;
          mbar_arrive_expect_tx(full + stage, C::TX2);
          const int f0 = (fch0 + j) * BF + t * C::SK;
          if constexpr (C::kTF32) {
            // W_down^T planes: rows (e, d), K = f contiguous; box {32, D}.
            for (int pl = 0; pl < C::PL; ++pl)
              tma_load_2d_hint(st + pl * C::S2_WPLANE, &maps.wd[pl], full + stage, f0, e * D, pol_w);
          } else {
            // W_down rows (e, f), N = d contiguous; box {64, 64} per 64-wide d block.
            for (int nb = 0; nb < D / C::ATOM; ++nb)
              tma_load_2d_hint(st + nb * C::SK * 128, &maps.wd[0], full + stage, nb * C::ATOM, e * p.F + f0,
                               pol_w);
          }
          advance();
          return true;
        };
        for (int j = 0; j < NCH && ok; ++j) {
          for (int s = 0; s < C::N1 && ok; ++s) ok = load_s1(j, s);
          if (j > 0)
            for (int t = 0; t < C::N2 && ok; ++t) ok = load_s2(j - 1, t);
        }
        for (int t = 0; t < C::N2 && ok; ++t) ok = load_s2(NCH - 1, t);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      BlockCursor cur;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ui = 0;
      uint32_t hcount = 0;  // hidden chunks issued (selects the TMEM buffer)
      bool ok = true;
      const uint32_t t_y = tmem_base;
      auto wait_full = [&]() -> bool {
        if (!mbar_wait(full + stage, phase, abort_flag, p.status)) return false;
        tc_fence_after();
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
        const int gb = u / S;
        if (!cur.seek(gb, p.group_sizes, p.E, p.M)) break;
        if constexpr (X_RES) {
          if (!mbar_wait(x_ready, ui & 1u, abort_flag, p.status)) break;
          tc_fence_after();
        }
        const uint32_t xbase = smem_u32(xbuf);
        auto mma1 = [&](int j) -> bool {
          const uint32_t hb = (hcount + j) & 1u;
          const uint32_t d_tmem = tmem_base + D + hb * C::HCOLS;
          for (int s = 0; s < C::N1; ++s) {
            if (!wait_full()) return false;
            const uint32_t st = smem_u32(ring + stage * C::STAGE);
            for (int ki = 0; ki < C::SK / C::KI; ++ki) {
              uint64_t a[2], b[2];
              for (int pl = 0; pl < C::PL; ++pl) {
                const uint32_t xa = X_RES ? xbase + pl * C::X_PLANE + s * C::XBOX + ki * 32
                                          : st + pl * C::XBOX + ki * 32;
                a[pl] = make_sdesc(xa, 16, 1024);
                if constexpr (C::kTF32) {
                  b[pl] = make_sdesc(st + C::S1_X + pl * C::S1_WPLANE + ki * 32, 16, 1024);
                } else {
                  b[pl] = make_sdesc(st + C::S1_X + ki * (C::KI * 128), C::SK * 128, 1024);
                }
              }
              const uint32_t acc0 = (s > 0 || ki > 0) ? 1u : 0u;
              umma_ss<C::kTF32 ? Kind::TF32 : Kind::F16>(d_tmem, a[0], b[0], C::IDESC1, acc0);
              if constexpr (C::kTF32) {
                umma_ss<Kind::TF32>(d_tmem, a[0], b[1], C::IDESC1, 1u);
                umma_ss<Kind::TF32>(d_tmem, a[1], b[0], C::IDESC1, 1u);
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
          if (!mbar_wait(h_ready + hb, use & 1u, abort_flag, p.status)) return false;
          tc_fence_after();
          if (j == 0) {
            if (!mbar_wait(y_empty, (ui & 1u) ^ 1u, abort_flag, p.status)) return false;
            tc_fence_after();
          }
          const uint32_t h_tmem = tmem_base + D + hb * C::HCOLS;
          for (int t = 0; t < C::N2; ++t) {
            if (!wait_full()) return false;
            const uint32_t st = smem_u32(ring + stage * C::STAGE);
            for (int ki = 0; ki < C::SK / C::KI; ++ki) {
              const uint32_t kcol = (t * C::SK + ki * C::KI) * C::ESZ / 4;
              uint64_t b[2];
              for (int pl = 0; pl < C::PL; ++pl) {
                if constexpr (C::kTF32) {
                  b[pl] = make_sdesc(st + pl * C::S2_WPLANE + ki * 32, 16, 1024);
                } else {
                  b[pl] = make_sdesc(st + ki * (C::KI * 128), C::SK * 128, 1024);
                }
              }
              const uint32_t acc0 = (j > 0 || t > 0 || ki > 0) ? 1u : 0u;
              umma_ts<C::kTF32 ? Kind::TF32 : Kind::F16>(t_y, h_tmem + kcol, b[0], C::IDESC2, acc0);
              if constexpr (C::kTF32) {
                umma_ts<Kind::TF32>(t_y, h_tmem + kcol, b[1], C::IDESC2, 1u);
                umma_ts<Kind::TF32>(t_y, h_tmem + BF + kcol, b[0], C::IDESC2, 1u);
              }
            }
            release();
          }
          return true;
        };
        for (int j = 0; j < NCH && ok; ++j) {
          ok = mma1(j);
          if (ok && X_RES && j == NCH - 1) umma_commit(x_empty);
          if (ok && j > 0) ok = mma2(j - 1);
        }
        if (ok) ok = mma2(NCH - 1);
        if (ok) umma_commit(y_full);
        hcount += NCH;
      }
    }
  } else {
    // ------------------------------------------------------------ GELU / epilogue warps
    const uint32_t q = warp & 3u;  // TMEM lane quadrant this warp may access
    const uint32_t lane_base = tmem_base + ((q * 32u) << 16);
    const int erow = (int)(q * 32u + lane);  // row inside the 128-row block
    const int etid = (int)threadIdx.x - 64;  // 0..127

    if (etid == 0 && blockIdx.x == 0) {
      for (int e = 0; e < p.E; ++e)
        if (__ldg(p.group_sizes + e) < 0) atomicOr(p.status, kStatusBadGroupSize);
    }
    // Rows at or past sum(group_sizes) are zero in ragged_dot; write them
    // here unless Y was zeroed up front (reduce-add mode).
    if (!p.atomic_out) {
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
      for (size_t i = (size_t)blockIdx.x * 128 + etid; i < n4; i += (size_t)gridDim.x * 128)
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
    // In-place split of the resident f32 X tile into tf32 hi (kept in plane 0)
    // and lo (written to plane 1); layout-agnostic because it is elementwise.
    auto split_x = [&](uint32_t uidx) -> bool {
      if (!warp_wait(x_full, uidx & 1u)) return false;
      float4* hi = reinterpret_cast<float4*>(xbuf);
      float4* lo = reinterpret_cast<float4*>(xbuf + C::X_PLANE);
      for (int i = etid; i < C::X_PLANE / 16; i += 128) {
        float4 v = hi[i];
        float4 h, l;
        h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
        h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
        h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
        h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
        l.x = v.x - h.x;
        l.y = v.y - h.y;
        l.z = v.z - h.z;
        l.w = v.w - h.w;
        hi[i] = h;
        lo[i] = l;
      }
      fence_proxy_async_smem();
      mbar_arrive(x_ready);
      return true;
    };
    auto pass_x = [&](uint32_t uidx) -> bool {  // bf16: raw X is the operand
      if (!warp_wait(x_full, uidx & 1u)) return false;
      mbar_arrive(x_ready);
      return true;
    };

    int u = blockIdx.x;
    bool have = cur.seek(u / S, p.group_sizes, p.E, p.M);
    if (have && X_RES) ok = C::kTF32 ? split_x(0) : pass_x(0);
    while (have && ok) {
      const int gb = u / S;
      const int row0 = cur.row_begin + (gb - cur.blk_begin) * C::BM;
      const int row_end = cur.row_begin + cur.rows;
      // Hidden chunks: TMEM accumulator -> GELU -> MMA2 operand.
      for (int j = 0; j < NCH && ok; ++j) {
        const uint32_t hb = (hcount + j) & 1u;
        const uint32_t use = (hcount + j) >> 1;
        if (!warp_wait(h_full + hb, use & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t hcol = D + hb * C::HCOLS;
#pragma unroll 1
        for (int c0 = 0; c0 < BF; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(lane_base + hcol + c0, v);
          tmem_ld_wait();
          if constexpr (C::kTF32) {
            uint32_t lo[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float g = gelu_tanh_accurate(__uint_as_float(v[i]));
              const uint32_t hbits = __float_as_uint(g) & 0xFFFFE000u;
              lo[i] = __float_as_uint(g - __uint_as_float(hbits));
              v[i] = hbits;
            }
            tmem_st32(lane_base + hcol + c0, v);
            tmem_st32(lane_base + hcol + BF + c0, lo);
          } else {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = pack_bf16x2(gelu_tanh_fast(__uint_as_float(v[2 * i])),
                                  gelu_tanh_fast(__uint_as_float(v[2 * i + 1])));
            tmem_st16(lane_base + hcol + c0 / 2, pk);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(h_ready + hb);
      }
      if (!ok) break;
      hcount += NCH;

      // Look ahead: prepare the next unit's X operand before draining Y so
      // the tensor core can start the next unit's MMA1 meanwhile.
      const int u_next = u + gridDim.x;
      BlockCursor nxt = cur;
      const bool have_next = nxt.seek(u_next / S, p.group_sizes, p.E, p.M);
      if (have_next && X_RES) {
        ok = C::kTF32 ? split_x(ui + 1) : pass_x(ui + 1);
        if (!ok) break;
      }

      // Y epilogue.
      if (!warp_wait(y_full, ui & 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int row = row0 + erow;
      const bool valid = row < row_end;
      float* yrow = p.y + (size_t)row * D;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(lane_base + c0, v);
        tmem_ld_wait();
        if (valid) {
          if (p.atomic_out) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              red_add_v4(yrow + c0 + i, __uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                         __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
          } else {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(yrow + c0 + i) =
                  make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]),
                              __uint_as_float(v[i + 3]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(y_empty);

      u = u_next;
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
