// Backward of the expert MLP  Y = GELU_tanh(X W_up[e]) W_down[e]  over
// expert-sorted rows (bf16 operands, f32 accumulation), sm_100a.
//
// Given the upstream gradient dY and the forward's saved pre-activation
// A = X W_up[e] (bf16, M x F):
//
//   dH  = dY W_down[e]^T              (rows of e; K = D)     mode DH
//   dA  = dH * GELU'(A),  H = GELU(A)                        (DH epilogue)
//   dX  = dA W_up[e]^T                (rows of e; K = F)     mode DX
//   dW_up[e]   = X_e^T dA_e           (K = rows of e)        mode DW
//   dW_down[e] = H_e^T dY_e           (K = rows of e)        mode DW
//
// Row layout.  The weight-gradient GEMMs reduce over an expert's rows, whose
// count and offset are arbitrary.  X and dY are first copied into a padded
// layout in which every expert's rows start at a multiple of 64 and the gap
// rows are zero (bwd_pad_rows_kernel); the DH epilogue writes dA and H in the
// same layout.  Every expert's K range is then whole 64-row TMA steps whose
// rows past the expert's end are zero, so no masking sits between TMA and the
// tensor cores.  DH and DX walk 256-row tiles in the padded layout (rows past
// an expert's end are masked at the store, as in the forward); DX writes dX
// back in the natural layout.
//
// All three modes run on CTA pairs (tcgen05.mma.cta_group::2, M = N = 256,
// K = 16 per instruction) with the forward kernel's warp roles: warp 0 TMA
// producer, warp 1 TMEM owner + MMA issuer (pair leader), warps 2..5
// epilogue; 2 x 256 TMEM accumulator columns so the epilogue of one tile
// overlaps the MMAs of the next.  Operand majorness per mode:
//   DH, DX: A (dY, dA) K-major; B = the weight viewed as [E*N, K] (K
//           contiguous): K-major, the transposed product without a transpose.
//   DW:     A = X^T or H^T and B = dA or dY, both read from row-major [rows,
//           cols] tiles: MN-major, 128-byte swizzle, two 64-column atoms per
//           CTA operand.
#pragma once
#include "grouped_gemm.cuh"

namespace moe {

enum : int { kBwdDH = 0, kBwdDX = 1, kBwdDW = 2, kBwdDHSwiGLU = 3 };

__host__ __device__ __forceinline__ int pad64(int g) { return (g + 63) & ~63; }

struct BwdParams {
  const int32_t* group_sizes;
  int M;              // natural rows (rows past sum(group_sizes) carry no gradient)
  int E;
  int N;              // output columns of the mode's GEMM
  int K;              // DH / DX: reduction length (D or F); DW: unused (the expert's padded rows)
  int m_out;          // DW: output rows per expert (D for dW_up, F for dW_down)
  int group_m;        // tile rasterisation group (row blocks)
  int* status;
  const uint16_t* a_saved;  // DH: pre-activation (M, N) bf16; DH SwiGLU: gate/up pre-activations
                            // (M, 2N) bf16 interleaved every 128 columns; natural rows
  void* out;          // DH: dA (Mp, N) bf16, padded rows; DH SwiGLU: dGate/dUp (Mp, 2N) interleaved;
                      // DX: dX (M, N) f32; DW: dW (E, m_out, N) f32
  void* out2;         // DH: H = GELU(A), DH SwiGLU: H = SiLU(gate) * up; (Mp, N) bf16, padded rows
};

template <int MODE>
struct BwdCfg {
  static constexpr int BM = 128;   // rows per CTA (256 per pair)
  static constexpr int BN = 256;   // output columns per tile (128 per CTA of B)
  static constexpr int BK = 64;    // 64 bf16 = one 128-byte swizzle row (K-major) / 64 K rows (MN-major)
  static constexpr int A_BYTES = BM * BK * 2;        // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KB
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NS = 6;
  static constexpr int EPI_WARPS = 4;
  static constexpr int OUT_STAGE = EPI_WARPS * 4096;  // 32 rows x 128 B per epilogue warp
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 + NS * STAGE + OUT_STAGE + BAR_BYTES;
  static constexpr int TMEM_COLS = 512;
  static constexpr bool MN = MODE == kBwdDW;  // A and B MN-major
  static constexpr uint32_t IDESC = make_idesc(kFmtBF16, 256, BN, MN ? 1 : 0, MN ? 1 : 0);
  static constexpr uint32_t TX = 2 * STAGE;
  static constexpr int THREADS = 64 + EPI_WARPS * 32;
  static_assert(SMEM <= kMaxSmemPerBlock, "shared memory budget");
};

// One tile of a backward GEMM as seen by every warp role.
struct BwdTile {
  int e, mb, nb;
  int nk;          // K steps of 64
  int row_begin;   // natural first row of expert e
  int prow_begin;  // padded first row of expert e
  int rows;        // rows of expert e (clamped to M)
};

// Tile walk, monotone in the global tile index t.  DH / DX: (expert,
// 256-row block, 256-column block) over each expert's rows, as in the
// forward.  DW: (expert, 256-row block of the expert's output, 256-column
// block); every expert has the same tiles, with K = its padded rows.
template <int MODE>
struct BwdWalk {
  int e = -1, t_begin = 0, ntiles = 0, row_begin = 0, prow_begin = 0, rows = 0, mt = 0;

  __device__ __forceinline__ bool next(int t, const BwdParams& p, int nt, int mtw, BwdTile& tl) {
    while (t >= t_begin + ntiles) {
      t_begin += ntiles;
      row_begin += rows;
      prow_begin += pad64(rows);
      if (++e >= p.E) return false;
      int g = __ldg(p.group_sizes + e);
      g = g < 0 ? 0 : g;
      const int rem = p.M - row_begin;
      g = g > rem ? (rem > 0 ? rem : 0) : g;
      rows = g;
      mt = MODE == kBwdDW ? mtw : (g + 255) >> 8;
      ntiles = mt * nt;
    }
    // Grouped rasterisation: GM row blocks share each column block.
    const int l = t - t_begin;
    const int per_group = p.group_m * nt;
    const int g = l / per_group;
    const int r = l - g * per_group;
    int gm = mt - g * p.group_m;
    gm = gm < p.group_m ? gm : p.group_m;
    tl.e = e;
    tl.mb = g * p.group_m + r % gm;
    tl.nb = r / gm;
    tl.nk = MODE == kBwdDW ? pad64(rows) / 64 : p.K / 64;
    tl.row_begin = row_begin;
    tl.prow_begin = prow_begin;
    tl.rows = rows;
    return true;
  }
};

// GELU_tanh(x) and its derivative.  tanh(u) and sech^2(u) = 1 - tanh^2(u)
// come from e = exp(-2|u|) (approximate exp2 and reciprocal), which keeps
// sech^2 accurate where tanh saturates and 1 - t*t would cancel:
//   tanh|u| = (1 - e) / (1 + e),  sech^2 u = 4e / (1 + e)^2,
//   GELU'(x) = 0.5 (1 + t) + 0.5 x sech^2(u) k0 (1 + 3 k1 x^2).
__device__ __forceinline__ void gelu_tanh_and_grad(float x, float& g, float& gp) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float x2 = x * x;
  const float u = k0 * fmaf(k1 * x2, x, x);
  const float e = ex2_approx(-2.8853900817779268f * fabsf(u));  // exp(-2|u|)
  const float r = rcp_approx(1.0f + e);
  const float t = copysignf((1.0f - e) * r, u);
  const float sech2 = 4.0f * e * r * r;
  const float hx = 0.5f * x;
  g = fmaf(hx, t, hx);
  gp = fmaf(0.5f, t, 0.5f) + hx * sech2 * k0 * fmaf(3.0f * k1, x2, 1.0f);
}

// SwiGLU backward of one element: from dH, gate g and up u,
//   s = sigmoid(g), H = g s u, dGate = dH u s (1 + g (1 - s)), dUp = dH g s.
// s = 1 / (1 + 2^(-g log2 e)) with the approximate exp2 and reciprocal.
__device__ __forceinline__ void swiglu_grad(float dh, float g, float u, float& dg, float& du, float& h) {
  const float s = rcp_approx(1.0f + ex2_approx(-1.4426950408889634f * g));
  const float silu = g * s;
  h = silu * u;
  du = dh * silu;
  dg = dh * u * s * fmaf(g, 1.0f - s, 1.0f);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// X (bf16) and dY (f32 or bf16) into the padded row layout (bf16): padded
// row pr of expert e holds natural row off_e + (pr - poff_e) while that is
// below off_e + rows_e, else zeros.  One warp per padded row; rows past the
// last expert's padded end are not written.
__global__ void __launch_bounds__(256) bwd_pad_rows_kernel(const uint16_t* __restrict__ x,
                                                           const void* __restrict__ dy, int dy_f32,
                                                           const int32_t* __restrict__ gs, int E, int M, int D,
                                                           uint16_t* __restrict__ x_pad,
                                                           uint16_t* __restrict__ dy_pad) {
  extern __shared__ int s_tab[];  // [E + 1] padded offsets, then [E + 1] natural offsets
  int* s_poff = s_tab;
  int* s_off = s_tab + E + 1;
  if (threadIdx.x == 0) {
    int off = 0, poff = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = off;
      s_poff[e] = poff;
      int g = gs[e];
      g = g < 0 ? 0 : g;
      g = g > M - off ? M - off : g;
      off += g;
      poff += pad64(g);
    }
    s_off[E] = off;
    s_poff[E] = poff;
  }
  __syncthreads();
  const int total = s_poff[E];
  const int wpb = (int)(blockDim.x >> 5);
  const int lane = (int)(threadIdx.x & 31);
  const int vec = D / 8;  // 16-byte vectors per bf16 row
  for (int pr = (int)blockIdx.x * wpb + (int)(threadIdx.x >> 5); pr < total; pr += (int)gridDim.x * wpb) {
    int lo = 0, hi = E - 1;  // last expert whose padded range starts at or before pr
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_poff[mid] <= pr) lo = mid;
      else hi = mid - 1;
    }
    const int lr = pr - s_poff[lo];
    uint4* xo = reinterpret_cast<uint4*>(x_pad + (size_t)pr * D);
    uint4* yo = reinterpret_cast<uint4*>(dy_pad + (size_t)pr * D);
    if (lr < s_off[lo + 1] - s_off[lo]) {
      const size_t src = (size_t)(s_off[lo] + lr) * D;
      const uint4* xi = reinterpret_cast<const uint4*>(x + src);
      for (int v = lane; v < vec; v += 32) xo[v] = __ldg(xi + v);
      if (dy_f32) {
        const float4* yi = reinterpret_cast<const float4*>(static_cast<const float*>(dy) + src);
        for (int v = lane; v < vec; v += 32) {
          const float4 a = __ldg(yi + 2 * v), b = __ldg(yi + 2 * v + 1);
          yo[v] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                             pack_bf16x2(b.z, b.w));
        }
      } else {
        const uint4* yi = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(dy) + src);
        for (int v = lane; v < vec; v += 32) yo[v] = __ldg(yi + v);
      }
    } else {
      for (int v = lane; v < vec; v += 32) {
        xo[v] = make_uint4(0u, 0u, 0u, 0u);
        yo[v] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(BwdCfg<MODE>::THREADS, 1)
    grouped_bwd_pair_kernel(const __grid_constant__ GemmMaps maps, const BwdParams p) {
  using C = BwdCfg<MODE>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* ring = smem;
  uint8_t* ostage = ring + C::NS * C::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ostage + C::OUT_STAGE);
  uint64_t* full = bars;                  // [NS] leader
  uint64_t* empty = bars + C::NS;         // [NS] both (multicast commit)
  uint64_t* acc_full = bars + 2 * C::NS;  // [2] both (multicast commit)
  uint64_t* acc_empty = acc_full + 2;     // [2] leader (epilogue warps of both CTAs)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1);
  const int npairs = (int)(gridDim.x >> 1);
  constexpr uint16_t kBoth = 0x3;
  const int nt = p.N / C::BN;
  const int mtw = MODE == kBwdDW ? p.m_out / C::BN : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
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
      BwdWalk<MODE> walk;
      BwdTile tl;
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol = l2_policy_evict_last();
      bool ok = true;
      for (int t = pair; ok && walk.next(t, p, nt, mtw, tl); t += npairs) {
        const int n0 = tl.nb * C::BN + (int)rank * (C::BN / 2);
        for (int kb = 0; kb < tl.nk; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + stage * C::STAGE;
          const uint32_t bar = full_l0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(full + stage, C::TX);
          if constexpr (MODE == kBwdDW) {
            // 64 rows of the expert's padded K range; this CTA's 128 output
            // rows of A^T and 128 output columns of B, 64 columns per box.
            const int krow = tl.prow_begin + kb * C::BK;
            const int m0 = tl.mb * 256 + (int)rank * C::BM;
            tma_load_2d_pair(st, &maps.a, bar, m0, krow, pol);
            tma_load_2d_pair(st + 64 * 128, &maps.a, bar, m0 + 64, krow, pol);
            tma_load_2d_pair(st + C::A_BYTES, &maps.b, bar, n0, krow, pol);
            tma_load_2d_pair(st + C::A_BYTES + 64 * 128, &maps.b, bar, n0 + 64, krow, pol);
          } else {
            const int row0 = tl.prow_begin + tl.mb * 256 + (int)rank * C::BM;
            tma_load_2d_pair(st, &maps.a, bar, kb * C::BK, row0, pol);
            tma_load_2d_pair(st + C::A_BYTES, &maps.b, bar, kb * C::BK, tl.e * p.N + n0, pol);
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
      BwdWalk<MODE> walk;
      BwdTile tl;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t tcount = 0;
      bool ok = true;
      for (int t = pair; ok && walk.next(t, p, nt, mtw, tl); t += npairs) {
        if (tl.nk == 0) continue;  // expert without rows: the epilogue writes zeros
        const uint32_t ab = tcount & 1u;
        const uint32_t use = tcount >> 1;
        ++tcount;
        if (!mbar_wait_warp(acc_empty + ab, (use & 1u) ^ 1u, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * C::BN;
        for (int kb = 0; kb < tl.nk; ++kb) {
          if (!mbar_wait_warp(full + stage, phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(ring + stage * C::STAGE);
          // K-major: 16 K = 32 bytes along the swizzled row; MN-major: 16 K
          // rows of 128 bytes.
          constexpr uint32_t kstep = C::MN ? 16 * 128 : 32;
          const uint64_t a_desc = make_sdesc(st, C::MN ? 64 * 128 : 16, 1024);
          const uint64_t b_desc = make_sdesc(st + C::A_BYTES, C::MN ? 64 * 128 : 16, 1024);
#pragma unroll
          for (int ki = 0; ki < C::BK / 16; ++ki)
            umma_ss_pair<Kind::F16>(d_tmem, a_desc + (uint64_t)((ki * kstep) >> 4),
                                    b_desc + (uint64_t)((ki * kstep) >> 4), C::IDESC, (kb > 0 || ki > 0) ? 1u : 0u);
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
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const uint32_t q = warp & 3u;
    const uint32_t lane_base = tmem_base + ((q * 32u) << 16);
    uint8_t* wst = ostage + (warp - 2u) * 4096u;
    float4* wst4 = reinterpret_cast<float4*>(wst);
    uint4* stg = reinterpret_cast<uint4*>(wst);
    if (MODE == kBwdDX) {
      // Rows at or past sum(group_sizes) have no gradient.
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
    BwdWalk<MODE> walk;
    BwdTile tl;
    uint32_t tcount = 0;
    for (int t = pair; walk.next(t, p, nt, mtw, tl); t += npairs) {
      if constexpr (MODE == kBwdDW) {
        if (tl.nk == 0) {
          // No rows routed to this expert: its weight gradients are zero.
          float* W = reinterpret_cast<float*>(p.out) + (size_t)tl.e * p.m_out * p.N;
          const int r0 = tl.mb * 256 + (int)rank * C::BM + (int)q * 32;
          for (int r = 0; r < 32; ++r) {
            float4* dst = reinterpret_cast<float4*>(W + (size_t)(r0 + r) * p.N + tl.nb * C::BN);
            dst[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
            dst[lane + 32] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
          continue;
        }
      }
      const uint32_t ab = tcount & 1u;
      const uint32_t use = tcount >> 1;
      ++tcount;
      if (!mbar_wait_warp(acc_full + ab, use & 1u, abort_flag, p.status)) break;
      tc_fence_after();
      const uint32_t acc = lane_base + ab * C::BN;
      // Expert-local row of this warp's first row.
      const int lr0 = tl.mb * 256 + (int)rank * C::BM + (int)q * 32;
      if constexpr (MODE == kBwdDW) {
        float* W = reinterpret_cast<float*>(p.out) + (size_t)tl.e * p.m_out * p.N + (size_t)tl.nb * C::BN;
#pragma unroll 1
        for (int c0 = 0; c0 < C::BN; c0 += 32) store_y_block<0>(acc + c0, wst4, W, lr0, p.m_out, c0, lane, false, p.N);
      } else if constexpr (MODE == kBwdDX) {
        float* Y = reinterpret_cast<float*>(p.out) + (size_t)tl.nb * C::BN;
#pragma unroll 1
        for (int c0 = 0; c0 < C::BN; c0 += 32)
          store_y_block<0>(acc + c0, wst4, Y, tl.row_begin + lr0, tl.row_begin + tl.rows, c0, lane, false, p.N);
      } else if constexpr (MODE == kBwdDHSwiGLU) {
        // 32 dH columns per step (inside one 128-column gate/up period): the
        // saved gate and up columns come in through the staging tile as one
        // 128-byte line per row (64 B gate | 64 B up); dGate|dUp leave the
        // same way, H as 64-byte row segments.
        uint16_t* dGU = reinterpret_cast<uint16_t*>(p.out);
        uint16_t* Hp = reinterpret_cast<uint16_t*>(p.out2);
        const int ld2 = 2 * p.N;
        const int prow_end = pad64(tl.rows);
#pragma unroll 1
        for (int c0 = 0; c0 < C::BN; c0 += 32) {
          const int fcol = tl.nb * C::BN + c0;              // first dH / H column
          const int gcol = 256 * (fcol >> 7) + (fcol & 127);  // its gate column; up is 128 further
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (int)(lane >> 3);
            const int k = (int)(lane & 7);
            const int lr = lr0 + r;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (lr < tl.rows)
              v = __ldg(reinterpret_cast<const uint4*>(p.a_saved + (size_t)(tl.row_begin + lr) * ld2 + gcol +
                                                       (k < 4 ? 8 * k : 128 + 8 * (k - 4))));
            stg[r * 8 + (k ^ (r & 7))] = v;
          }
          __syncwarp();
          uint32_t g[16], u[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 a = stg[lane * 8 + (j ^ (lane & 7))];
            const uint4 b = stg[lane * 8 + ((4 + j) ^ (lane & 7))];
            g[4 * j] = a.x;
            g[4 * j + 1] = a.y;
            g[4 * j + 2] = a.z;
            g[4 * j + 3] = a.w;
            u[4 * j] = b.x;
            u[4 * j + 1] = b.y;
            u[4 * j + 2] = b.z;
            u[4 * j + 3] = b.w;
          }
          __syncwarp();
          uint32_t v[32];
          tmem_ld32(acc + c0, v);
          tmem_ld_wait();
          uint32_t dg[16], du[16], hv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float dg0, du0, h0, dg1, du1, h1;
            swiglu_grad(__uint_as_float(v[2 * j]), bf16_lo(g[j]), bf16_lo(u[j]), dg0, du0, h0);
            swiglu_grad(__uint_as_float(v[2 * j + 1]), bf16_hi(g[j]), bf16_hi(u[j]), dg1, du1, h1);
            dg[j] = pack_bf16x2(dg0, dg1);
            du[j] = pack_bf16x2(du0, du1);
            hv[j] = pack_bf16x2(h0, h1);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            stg[lane * 8 + (j ^ (lane & 7))] = make_uint4(dg[4 * j], dg[4 * j + 1], dg[4 * j + 2], dg[4 * j + 3]);
            stg[lane * 8 + ((4 + j) ^ (lane & 7))] =
                make_uint4(du[4 * j], du[4 * j + 1], du[4 * j + 2], du[4 * j + 3]);
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (int)(lane >> 3);
            const int k = (int)(lane & 7);
            const int lr = lr0 + r;
            if (lr < prow_end)
              *reinterpret_cast<uint4*>(dGU + (size_t)(tl.prow_begin + lr) * ld2 + gcol +
                                        (k < 4 ? 8 * k : 128 + 8 * (k - 4))) = stg[r * 8 + (k ^ (r & 7))];
          }
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            stg[lane * 8 + (j ^ (lane & 7))] = make_uint4(hv[4 * j], hv[4 * j + 1], hv[4 * j + 2], hv[4 * j + 3]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (int)(lane >> 3);
            const int k = (int)(lane & 7);
            const int lr = lr0 + r;
            if (k < 4 && lr < prow_end)
              *reinterpret_cast<uint4*>(Hp + (size_t)(tl.prow_begin + lr) * p.N + fcol + 8 * k) =
                  stg[r * 8 + (k ^ (r & 7))];
          }
          __syncwarp();
        }
      } else {
        // dA = dH * GELU'(A) and H = GELU(A), 64 columns per step.  The saved
        // A rows come in through the staging tile (coalesced 128-byte row
        // reads, zeros for the expert's gap rows); dA and H leave through it
        // as 128-byte row stores over the expert's padded rows.
        uint16_t* dA = reinterpret_cast<uint16_t*>(p.out);
        uint16_t* Hp = reinterpret_cast<uint16_t*>(p.out2);
        const int prow_end = pad64(tl.rows);
#pragma unroll 1
        for (int c0 = 0; c0 < C::BN; c0 += 64) {
          const int gcol = tl.nb * C::BN + c0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (int)(lane >> 3);
            const int k = (int)(lane & 7);
            const int lr = lr0 + r;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (lr < tl.rows)
              v = __ldg(reinterpret_cast<const uint4*>(p.a_saved + (size_t)(tl.row_begin + lr) * p.N + gcol + 8 * k));
            stg[r * 8 + (k ^ (r & 7))] = v;
          }
          __syncwarp();
          uint32_t a[32];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 v = stg[lane * 8 + (j ^ (lane & 7))];
            a[4 * j] = v.x;
            a[4 * j + 1] = v.y;
            a[4 * j + 2] = v.z;
            a[4 * j + 3] = v.w;
          }
          __syncwarp();
          uint32_t da[32], hv[32];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t v[32];
            tmem_ld32(acc + c0 + 32 * hh, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float g0, gp0, g1, gp1;
              gelu_tanh_and_grad(bf16_lo(a[16 * hh + j]), g0, gp0);
              gelu_tanh_and_grad(bf16_hi(a[16 * hh + j]), g1, gp1);
              da[16 * hh + j] = pack_bf16x2(__uint_as_float(v[2 * j]) * gp0, __uint_as_float(v[2 * j + 1]) * gp1);
              hv[16 * hh + j] = pack_bf16x2(g0, g1);
            }
          }
#pragma unroll
          for (int out = 0; out < 2; ++out) {
            const uint32_t* src = out == 0 ? da : hv;
            uint16_t* dst = out == 0 ? dA : Hp;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              stg[lane * 8 + (j ^ (lane & 7))] = make_uint4(src[4 * j], src[4 * j + 1], src[4 * j + 2], src[4 * j + 3]);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 4 * i + (int)(lane >> 3);
              const int k = (int)(lane & 7);
              const int lr = lr0 + r;
              if (lr < prow_end)
                *reinterpret_cast<uint4*>(dst + (size_t)(tl.prow_begin + lr) * p.N + gcol + 8 * k) =
                    stg[r * 8 + (k ^ (r & 7))];
            }
            __syncwarp();
          }
        }
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
