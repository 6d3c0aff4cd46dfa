// Routing and permutation around the fused expert MLP (sm_100a): the steps
// before and after the reference's path, which takes rows already sorted by
// expert (its `fused_ragged_dot_caller` receives `x` and `group_sizes`).
//
//   route_topk_kernel   per token, the k largest router logits (ties: lower
//                       expert id first) and their softmax weights (= the
//                       full softmax renormalised over the selected experts).
//   perm_hist_kernel    per block of 512 (token, slot) entries, a histogram
//                       over experts.
//   perm_scan_kernel    group sizes, and each block's first row per expert in
//                       the expert-sorted order.
//   perm_scatter_kernel stable counting sort: entry i = t * k + j lands at
//                       row inverse[i]; sorted_src[row] = i.  Ranks inside a
//                       block come from per-warp expert histograms, so the
//                       order is deterministic (= a stable sort by expert).
//   gather_rows_kernel  X_sorted[row] = X[sorted_src[row] / k].
//   combine_rows_kernel Y[t] = sum_j w[t, j] * Y_sorted[inverse[t * k + j]],
//                       in slot order (deterministic).
//
// All are HBM-bound byte/integer work: coalesced 16-byte accesses, one warp
// per row or token, grids sized by the SM count.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace moe {

constexpr int kRouteMaxExperts = 1024;
constexpr int kRouteMaxK = 16;
constexpr int kPermBlock = 512;  // entries per histogram / scatter block (16 warps)
enum : int { kStatusBadExpertId = 16 };  // an expert id outside [0, E) was dropped

// ---------------------------------------------------------------- top-k
// One warp per token: lane l holds logits l, l + 32, ... in registers; k
// rounds of a warp arg-max (larger value, then lower expert id).
template <int PER_LANE>
__global__ void __launch_bounds__(256) route_topk_kernel(const float* __restrict__ logits, int64_t T, int E, int k,
                                                         int32_t* __restrict__ ids, float* __restrict__ w) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    float v[PER_LANE];
    const float* row = logits + t * E;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? __ldg(row + e) : -INFINITY;
    }
    uint32_t taken = 0;  // bit i: v[i] already selected
    float sel[kRouteMaxK];
    int sel_id[kRouteMaxK];
    for (int j = 0; j < k; ++j) {
      float bv = -INFINITY;
      int be = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !(taken >> i & 1u) && (v[i] > bv || (v[i] == bv && e < be))) {
          bv = v[i];
          be = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ov > bv || (ov == bv && oe < be)) {
          bv = ov;
          be = oe;
        }
      }
      // The owner lane marks the winner taken.
      if ((be & 31) == lane && be < E) taken |= 1u << (be >> 5);
      sel[j] = bv;
      sel_id[j] = be;
    }
    if (lane == 0) {
      // A slot with no finite winner (NaN logits) gets id -1 and weight 0;
      // the permutation drops it.
      float sum = 0.f;
      for (int j = 0; j < k; ++j)
        if (sel_id[j] < E) sum += __expf(sel[j] - sel[0]);
      const float inv = sum > 0.f ? 1.f / sum : 0.f;
      for (int j = 0; j < k; ++j) {
        const bool ok = sel_id[j] < E;
        ids[t * k + j] = ok ? sel_id[j] : -1;
        w[t * k + j] = ok ? __expf(sel[j] - sel[0]) * inv : 0.f;
      }
    }
  }
}

template <int PL>
static void launch_topk(const float* logits, int64_t T, int E, int k, int32_t* ids, float* w, int blocks,
                        cudaStream_t st) {
  route_topk_kernel<PL><<<blocks, 256, 0, st>>>(logits, T, E, k, ids, w);
}

// ---------------------------------------------------------------- permutation
__global__ void __launch_bounds__(kPermBlock) perm_hist_kernel(const int32_t* __restrict__ ids, int64_t N, int E,
                                                               int32_t* __restrict__ block_hist, int* status) {
  extern __shared__ int s_h[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_h[e] = 0;
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * kPermBlock + threadIdx.x;
  if (i < N) {
    const int e = __ldg(ids + i);
    if (e >= 0 && e < E)
      atomicAdd(&s_h[e], 1);
    else
      atomicOr(status, kStatusBadExpertId);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_hist[(int64_t)blockIdx.x * E + e] = s_h[e];
}

// One CTA of 32 warps; warp w owns experts w, w + 32, ...  block_hist[b][e]
// holds block b's entry count for expert e and becomes the block's first
// sorted row of expert e: the experts' exclusive offset plus the exclusive
// prefix over earlier blocks.  Pass 1 sums each expert's column (warp
// reduction), one warp scans the totals over experts, pass 2 scans each
// column in chunks of 32 blocks (warp-wide inclusive scan, carried across
// chunks), so every load of a chunk is in flight at once.
__device__ __forceinline__ int warp_inclusive_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}
__global__ void __launch_bounds__(1024) perm_scan_kernel(int32_t* __restrict__ block_hist, int64_t nblocks, int E,
                                                         int32_t* __restrict__ group_sizes) {
  __shared__ int s_base[kRouteMaxExperts];
  const int lane = (int)(threadIdx.x & 31u), warp = (int)(threadIdx.x >> 5), nw = (int)(blockDim.x >> 5);
  for (int e = warp; e < E; e += nw) {
    int sum = 0;
    for (int64_t b = lane; b < nblocks; b += 32) sum += block_hist[b * E + e];
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      s_base[e] = sum;
      group_sizes[e] = sum;
    }
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int v = e0 + lane < E ? s_base[e0 + lane] : 0;
      const int inc = warp_inclusive_scan(v, lane);
      if (e0 + lane < E) s_base[e0 + lane] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
  __syncthreads();
  for (int e = warp; e < E; e += nw) {
    int carry = s_base[e];
    for (int64_t b0 = 0; b0 < nblocks; b0 += 32) {
      const int64_t b = b0 + lane;
      const int v = b < nblocks ? block_hist[b * E + e] : 0;
      const int inc = warp_inclusive_scan(v, lane);
      if (b < nblocks) block_hist[b * E + e] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
}

__global__ void __launch_bounds__(kPermBlock) perm_scatter_kernel(const int32_t* __restrict__ ids, int64_t N, int E,
                                                                  const int32_t* __restrict__ block_off,
                                                                  int32_t* __restrict__ sorted_src,
                                                                  int32_t* __restrict__ inverse) {
  extern __shared__ int s_w[];  // [16 warps][E]: entries of expert e in warp w, then their exclusive prefix
  constexpr int kWarps = kPermBlock / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) s_w[i] = 0;
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * kPermBlock + threadIdx.x;
  int e = -1;
  if (i < N) {
    e = __ldg(ids + i);
    if (e < 0 || e >= E) e = -1;
  }
  const uint32_t peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) s_w[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int run = 0;
    for (int w2 = 0; w2 < kWarps; ++w2) {
      const int c = s_w[w2 * E + x];
      s_w[w2 * E + x] = run;
      run += c;
    }
  }
  __syncthreads();
  if (i < N) {
    if (e >= 0) {
      const int pos = block_off[(int64_t)blockIdx.x * E + e] + s_w[warp * E + e] + rank;
      sorted_src[pos] = (int32_t)i;
      inverse[i] = pos;
    } else {
      inverse[i] = -1;
    }
  }
}

// ---------------------------------------------------------------- rows
// Warp per destination row; rows of `row_bytes` (a multiple of 16).
__global__ void __launch_bounds__(512) gather_rows_kernel(const uint8_t* __restrict__ x,
                                                          const int32_t* __restrict__ sorted_src, int64_t rows,
                                                          int k, int row_bytes, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int n16 = row_bytes >> 4;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int64_t tok = __ldg(sorted_src + r) / k;
    const int4* s = reinterpret_cast<const int4*>(x + tok * row_bytes);
    int4* d = reinterpret_cast<int4*>(out + r * row_bytes);
    int c = lane;
    for (; c + 96 < n16; c += 128) {
      const int4 a0 = __ldg(s + c), a1 = __ldg(s + c + 32), a2 = __ldg(s + c + 64), a3 = __ldg(s + c + 96);
      d[c] = a0;
      d[c + 32] = a1;
      d[c + 64] = a2;
      d[c + 96] = a3;
    }
    for (; c < n16; c += 32) d[c] = __ldg(s + c);
  }
}

// Warp per token: f32 rows of D (a multiple of 4); slots accumulated in order.
__global__ void __launch_bounds__(512) combine_rows_kernel(const float* __restrict__ ys,
                                                           const int32_t* __restrict__ inverse,
                                                           const float* __restrict__ w, int64_t T, int k, int D,
                                                           float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int n4 = D >> 2;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    float4* yd = reinterpret_cast<float4*>(y + t * D);
    for (int c = lane; c < n4; c += 32) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < k; ++j) {
        const int p = __ldg(inverse + t * k + j);
        if (p < 0) continue;
        const float wj = __ldg(w + t * k + j);
        const float4 v = __ldg(reinterpret_cast<const float4*>(ys + (int64_t)p * D) + c);
        acc.x = fmaf(wj, v.x, acc.x);
        acc.y = fmaf(wj, v.y, acc.y);
        acc.z = fmaf(wj, v.z, acc.z);
        acc.w = fmaf(wj, v.w, acc.w);
      }
      yd[c] = acc;
    }
  }
}

}  // namespace moe
