// Expert-parallel token exchange over NVLink peer memory (sm_100a).
//
// Every rank of an expert-parallel group owns E_local = E / world experts and
// one "symmetric" device buffer with the same layout on every rank, mapped
// into every other rank's address space (CUDA IPC):
//
//   [flags 4 KB][group sizes 2 x world x E int32][X landing: waves regions]
//   [Y outbox: waves regions, f32]
//
// One forward step (epoch t = 1, 2, ...) of rank r:
//   ep_counts_kernel   r writes its clamped group sizes into every rank's
//                      buffer (slot parity t&1), raises cnt[r] = t on every
//                      peer and waits for cnt[s] = t from every peer; then
//                      derives, identically on every rank, where each
//                      (source, expert, wave) slice of rows lands.
//   ep_push_kernel(v)  r stores its rows of wave v straight into the owning
//                      rank's X landing region v (peer stores over NVLink);
//                      the last CTA raises data[v][r] = t on every peer.
//   ep_wait_kernel(v)  (on the compute stream) waits for data[v][s] = t from
//                      every peer; the fused expert MLP then runs over region
//                      v and writes the Y outbox region v.
//   ep_pull_kernel(v)  raises done[v][r] = t on every peer, waits for
//                      done[v][s] = t, and loads r's output rows of wave v
//                      from every owner's Y outbox into the caller's Y (peer
//                      loads); the last wave also zeroes Y's unrouted tail.
//
// Scatter mode (two-GEMM experts, one wave): there is no outbox; the down
// GEMM's epilogue stores each Y row into its source's Y landing area (peer
// stores), ep_ydone_kernel raises ydone[r] = t on every source, and
// ep_finish_kernel waits for every owner's ydone and copies the landing area
// into the caller's Y.
//
// Flags hold epochs, so they never need resetting.  Every wait targets flags
// raised by OTHER GPUs only (a rank's own slices are ordered by stream
// events), each is bounded in time, and a wait that runs out records
// kStatusPeerTimeout, raises the engine's abort word and stops all further
// data movement of that engine.  All row counts and offsets are clamped to
// the buffers they index, so stale or hostile group sizes cannot move a copy
// out of bounds.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace moe {

constexpr int kEpMaxWorld = 8;   // one NVSwitch domain of an HGX B200 node
constexpr int kEpMaxWaves = 8;
constexpr int kEpMaxExperts = 2048;
constexpr uint64_t kEpWaitLimitNs = 2000000000ull;  // 2 s: far above any skew between ranks of one step

enum : int {
  kStatusPeerTimeout = 4,   // a peer's flag did not arrive within kEpWaitLimitNs
  kStatusRowsClamped = 8,   // group sizes exceeded M or a landing region; rows were dropped
};

struct EpFlags {
  uint32_t cnt[kEpMaxWorld];                 // cnt[s] = t: source s published its group sizes of step t
  uint32_t data[kEpMaxWaves][kEpMaxWorld];   // data[v][s] = t: source s's rows of wave v have landed here
  uint32_t done[kEpMaxWaves][kEpMaxWorld];   // done[v][s] = t: owner s's outputs of wave v are ready
  uint32_t ydone[kEpMaxWorld];               // ydone[p] = t: owner p stored all of this rank's Y rows
};
static_assert(sizeof(EpFlags) <= 4096, "flag block");

// One routing slice: rows [src_row, src_row + n) of the source's X / Y,
// landing at rows [dst_row, dst_row + n) of the owner's region for its wave.
struct EpSlice {
  int src_row;
  int n;
  int dst_row;
  int owner;
};

struct EpArgs {
  uint8_t* base[kEpMaxWorld];  // every rank's symmetric buffer, in this process's address space
  int rank;
  int world;
  int el;            // experts per rank
  int E;             // experts in total (world * el)
  int waves;
  int region_cap;    // rows per landing region
  int max_rows;      // most rows any rank may hold in one step (max_tokens)
  int M;             // rows of this step's X / Y on this rank
  uint32_t epoch;
  size_t off_gs;     // byte offsets inside the symmetric buffer
  size_t off_x;
  size_t off_y;
  size_t region_x_bytes;
  size_t region_y_bytes;
  int row_bytes_x;   // D * sizeof(x element)
  int row_bytes_y;   // D * 4
  const int32_t* gs;     // (E,) this rank's group sizes (caller memory)
  const uint8_t* x;      // (M, D) caller X
  float* y;              // (M, D) caller Y
  // engine-local device tables
  EpSlice* slices;       // [waves][E]
  int* wave_rows;        // [waves][E + 1] prefix of slice rows (row -> slice search)
  int* local_gs;         // [waves][el] group sizes of each landing region
  int4* recv;            // scatter mode: [el][world] {first region row, rows, first source row, source}
  size_t off_yl;         // scatter mode: byte offset of the Y landing area (max_tokens rows)
  int* routed;           // rows of this rank's X that are routed (<= M)
  unsigned* push_ctr;    // [waves] CTAs finished with a push
  int* abort_word;
  int* status;
};

// Scatter mode with the dispatch fused into the up GEMM: the GEMM's dispatch
// warps store this rank's rows of the other owners' experts into their X
// landing regions (the owner's own rows are copied before the GEMM), and its
// TMA producer waits, per tile, for the sources whose rows the tile reads.
struct EpDispatch {
  uint8_t* base[kEpMaxWorld];  // every rank's symmetric buffer
  const uint8_t* x;            // this rank's X (rows sorted by global expert)
  size_t off_x;                // byte offset of the X landing region (wave 0)
  const EpSlice* slices;       // [E] this rank's slices (wave 0)
  const int* wave_rows;        // [E + 1] row prefix of the slices
  const int4* recv;            // [el][world] {first region row, rows, first source row, source}
  const uint32_t* data_flags;  // this rank's flags data[0][s]
  unsigned* push_ctr;          // CTAs of the GEMM done with their dispatch rows
  int* abort_word;
  int E, rank, world, row_bytes;
  uint32_t epoch;
  int on;
};

// ---------------------------------------------------------------- primitives
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ EpFlags* ep_flags(const EpArgs& a, int rank) {
  return reinterpret_cast<EpFlags*>(a.base[rank]);
}
// Epochs are compared modulo 2^32 so the counter may wrap.
__device__ __forceinline__ bool epoch_reached(uint32_t seen, uint32_t epoch) {
  return (int32_t)(seen - epoch) >= 0;
}

// Waits until *flag reaches `epoch`; false (and the abort word raised) after
// kEpWaitLimitNs or when another wait of this engine already gave up.
__device__ __forceinline__ bool ep_wait_flag(const uint32_t* flag, uint32_t epoch, const EpArgs& a) {
  const uint64_t t0 = global_timer_ns();
  while (!epoch_reached(ld_acquire_sys(flag), epoch)) {
    if (*reinterpret_cast<volatile int*>(a.abort_word)) return false;
    if (global_timer_ns() - t0 > kEpWaitLimitNs) {
      atomicOr(a.status, kStatusPeerTimeout);
      atomicExch(a.abort_word, 1);
      return false;
    }
    __nanosleep(200);
  }
  return true;
}

__host__ __device__ __forceinline__ int wave_cut(int c, int v, int waves) {
  return (int)(((int64_t)c * v) / waves);
}

// ---------------------------------------------------------------- slice tables
// The tables of one step are a pure function of the clamped count table
// cnt[W][E] (rows source s routes to global expert g), this rank's own row
// prefix own_off[E] and, in scatter mode, every source's row prefix
// src_off[W][E].  ep_counts_kernel evaluates the pieces below one entry per
// thread; moe_ep_build_tables evaluates them on the host, in order, so the
// same code is testable without a GPU.

// Rows of expert g in wave v over all sources.
__host__ __device__ __forceinline__ int ep_wave_total(const int* cnt, int W, int E, int V, int v, int g) {
  int n = 0;
  for (int s = 0; s < W; ++s) {
    const int c = cnt[s * E + g];
    n += wave_cut(c, v + 1, V) - wave_cut(c, v, V);
  }
  return n;
}

// Owner p's landing region of wave v: turns the wave totals of its experts
// (row[p * EL .. p * EL + EL)) into their first rows in the region, each cut
// to what the region still holds; the cut sizes are the owner's group sizes
// of that wave (written to local_gs when p is this rank).
__host__ __device__ __forceinline__ void ep_owner_region(int* row, int p, int EL, int region_cap, int* local_gs) {
  int run = 0;
  for (int e = 0; e < EL; ++e) {
    const int i = p * EL + e;
    int n = row[i];
    if (n > region_cap - run) n = region_cap - run;
    row[i] = run;
    if (local_gs) local_gs[e] = n;
    run += n;
  }
}

// This rank's slice of (wave v, expert g): inside the owner's region, sources
// in rank order starting at the owner itself (owner o: o, o + 1, ..., o - 1
// mod W), so that an owner's own rows lead each of its experts.  `start` is
// the expert's first region row (ep_owner_region).  *clamped is set when the
// slice had to be cut to the region.
__host__ __device__ __forceinline__ EpSlice ep_slice(const int* cnt, const int* own_off, int start, int W, int E,
                                                     int EL, int V, int rank, int region_cap, int v, int g,
                                                     bool* clamped) {
  const int o = g / EL;
  int before = 0;
  for (int s = o; s != rank; s = (s + 1 == W ? 0 : s + 1)) {
    const int c = cnt[s * E + g];
    before += wave_cut(c, v + 1, V) - wave_cut(c, v, V);
  }
  const int mine = cnt[rank * E + g];
  EpSlice sl;
  sl.src_row = own_off[g] + wave_cut(mine, v, V);
  sl.n = wave_cut(mine, v + 1, V) - wave_cut(mine, v, V);
  sl.dst_row = start + before;
  sl.owner = o;
  *clamped = false;
  if (sl.dst_row + sl.n > region_cap) {
    sl.n = sl.dst_row < region_cap ? region_cap - sl.dst_row : 0;
    *clamped = true;
  }
  return sl;
}

// Scatter mode (one wave): for this rank's local expert e and source sr, the
// region rows the source's rows landed on and where they go back to:
// {first region row, rows, first row in the source's X, source}.  The same
// arithmetic as the sources' side in ep_slice.
__host__ __device__ __forceinline__ int4 ep_recv_entry(const int* cnt, const int* local_gs, const int* src_off, int W,
                                                      int E, int EL, int rank, int region_cap, int e, int sr) {
  const int g = rank * EL + e;
  int start = 0;
  for (int e2 = 0; e2 < e; ++e2) start += local_gs[e2];
  for (int s2 = rank; s2 != sr; s2 = (s2 + 1 == W ? 0 : s2 + 1)) start += cnt[s2 * E + g];
  int n = cnt[sr * E + g];
  if (start + n > region_cap) n = start < region_cap ? region_cap - start : 0;
  int4 r;
  r.x = start;
  r.y = n;
  r.z = src_off[sr * E + g];
  r.w = sr;
  return r;
}

// Warp copy of one row of `bytes` (a multiple of 16) with 4 x 16 B in flight
// per lane.
__device__ __forceinline__ void warp_copy_row(uint8_t* dst, const uint8_t* src, int bytes, int lane) {
  const int n16 = bytes >> 4;
  const int4* s = reinterpret_cast<const int4*>(src);
  int4* d = reinterpret_cast<int4*>(dst);
  int i = lane;
  for (; i + 96 < n16; i += 128) {
    const int4 a0 = s[i], a1 = s[i + 32], a2 = s[i + 64], a3 = s[i + 96];
    d[i] = a0;
    d[i + 32] = a1;
    d[i + 64] = a2;
    d[i + 96] = a3;
  }
  for (; i < n16; i += 32) d[i] = s[i];
}

// In-place exclusive scan of n <= 2 * blockDim.x non-negative ints in shared
// memory, sums saturating at `cap`; returns the (saturated) total.  Every
// thread of the block must call it; blockDim.x is a multiple of 32.
__device__ __forceinline__ int block_exclusive_scan(int* data, int n, int cap) {
  __shared__ int s_warp[32];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, nw = blockDim.x >> 5;
  auto op = [cap](int a, int b) {
    const long long v = (long long)a + b;
    return v > cap ? cap : (int)v;
  };
  const int a0 = 2 * t < n ? data[2 * t] : 0;
  const int a1 = 2 * t + 1 < n ? data[2 * t + 1] : 0;
  int incl = op(a0, a1);
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl = op(u, incl);
  }
  int excl = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) excl = 0;
  if (lane == 31) s_warp[w] = incl;
  __syncthreads();
  if (w == 0) {
    int x = lane < nw ? s_warp[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x = op(u, x);
    }
    s_warp[lane] = x;  // inclusive over warps
  }
  __syncthreads();
  const int before = w > 0 ? s_warp[w - 1] : 0;
  const int total = s_warp[nw - 1];
  const int e0 = op(before, excl);
  if (2 * t < n) data[2 * t] = e0;
  if (2 * t + 1 < n) data[2 * t + 1] = op(e0, a0);
  __syncthreads();
  return total;
}

// Shared memory of ep_counts_kernel beyond its static arrays: the count
// table [world][E], the per-wave expert totals [waves][E] and the sources'
// row offsets [world][E].
__host__ __device__ constexpr size_t ep_counts_smem(int world, int E, int waves) {
  return (size_t)(2 * world + waves) * E * sizeof(int);
}

// ---------------------------------------------------------------- kernels
// One CTA of 1024 threads.  Publishes this rank's group sizes, meets every
// peer at the count barrier and builds the slice tables of this step.
__global__ void __launch_bounds__(1024) ep_counts_kernel(const __grid_constant__ EpArgs a) {
  __shared__ int s_gs[kEpMaxExperts];
  __shared__ int s_off[kEpMaxExperts];
  extern __shared__ int s_dyn[];
  const int tid = threadIdx.x;
  const int E = a.E, W = a.world, V = a.waves, EL = a.el;
  int* s_cnt = s_dyn;              // [W][E]
  int* s_T = s_dyn + W * E;        // [V][E]
  int* s_src = s_T + V * E;        // [W][E] first row of (source, expert) in the source's X
  const int par = (int)(a.epoch & 1u);

  // This rank's group sizes: negatives count as 0, the running total is cut at M.
  for (int g = tid; g < E; g += blockDim.x) {
    int c = __ldg(a.gs + g);
    if (c < 0) {
      atomicOr(a.status, kStatusBadGroupSize);
      c = 0;
    }
    c = c > a.M ? a.M : c;
    s_gs[g] = c;
    s_off[g] = c;
  }
  __syncthreads();
  const int routed = block_exclusive_scan(s_off, E, a.M);
  for (int g = tid; g < E; g += blockDim.x) {
    const int room = a.M - s_off[g];
    if (s_gs[g] > room) {
      s_gs[g] = room;
      atomicOr(a.status, kStatusRowsClamped);
    }
  }
  if (tid == 0) *a.routed = routed;
  __syncthreads();

  // Count barrier: publish, signal, wait (peers only).
  if (*reinterpret_cast<volatile int*>(a.abort_word) == 0) {
    for (int i = tid; i < W * E; i += blockDim.x) {
      const int s = i / E, g = i - s * E;
      int32_t* dst = reinterpret_cast<int32_t*>(a.base[s] + a.off_gs) + ((size_t)par * W + a.rank) * E;
      dst[g] = s_gs[g];
    }
    __threadfence_system();
    __syncthreads();
    if (tid < W && tid != a.rank) st_release_sys(&ep_flags(a, tid)->cnt[a.rank], a.epoch);
    if (tid < W && tid != a.rank) ep_wait_flag(&ep_flags(a, a.rank)->cnt[tid], a.epoch, a);
  }
  __syncthreads();
  const bool ok = *reinterpret_cast<volatile int*>(a.abort_word) == 0;

  // counts[s][g]: rows source s routes to global expert g in this step,
  // clamped to the rows one rank may hold, so that a wave of one expert over
  // all sources fits a landing region and no sum below can overflow.
  const int32_t* counts = reinterpret_cast<const int32_t*>(a.base[a.rank] + a.off_gs) + (size_t)par * W * E;
  for (int i = tid; i < W * E; i += blockDim.x) {
    const int s = i / E, g = i - s * E;
    int c = s == a.rank ? s_gs[g] : counts[i];
    c = c < 0 ? 0 : (c > a.max_rows ? a.max_rows : c);
    s_cnt[i] = ok ? c : 0;
  }
  __syncthreads();
  if (a.recv) {
    // Scatter mode: where each source's rows of each expert start in that
    // source's X (its own exclusive prefix over experts).
    for (int i = tid; i < W * E; i += blockDim.x) s_src[i] = s_cnt[i];
    __syncthreads();
    for (int sr = 0; sr < W; ++sr) block_exclusive_scan(s_src + sr * E, E, 0x7fffffff);
  }
  // T[v][g]: rows of expert g in wave v over all sources.
  for (int i = tid; i < V * E; i += blockDim.x) {
    const int v = i / E, g = i - v * E;
    s_T[i] = ep_wave_total(s_cnt, W, E, V, v, g);
  }
  __syncthreads();
  // Per (wave, owner): where each expert's rows start in the owner's landing
  // region; the owner's own region sizes are its group sizes for that wave.
  for (int vp = tid; vp < V * W; vp += blockDim.x) {
    const int v = vp / W, p = vp - v * W;
    ep_owner_region(s_T + v * E, p, EL, a.region_cap, p == a.rank ? a.local_gs + v * EL : nullptr);
  }
  __syncthreads();
  // This rank's slices (owner's own rows first in each expert: the up GEMM
  // can start on them before any peer's rows have landed).
  for (int i = tid; i < V * E; i += blockDim.x) {
    const int v = i / E, g = i - v * E;
    bool clamped;
    const EpSlice sl = ep_slice(s_cnt, s_off, s_T[i], W, E, EL, V, a.rank, a.region_cap, v, g, &clamped);
    if (clamped) atomicOr(a.status, kStatusRowsClamped);
    a.slices[i] = sl;
    s_T[i] = sl.n;
  }
  if (a.recv) {
    // Scatter mode (one wave): the receive table of this rank's experts.
    for (int i = tid; i < EL * W; i += blockDim.x) {
      const int e = i / W, sr = i - e * W;
      a.recv[i] = ep_recv_entry(s_cnt, a.local_gs, s_src, W, E, EL, a.rank, a.region_cap, e, sr);
    }
  }
  __syncthreads();
  // Row prefix of every wave's slices (for the row -> slice search).
  for (int v = 0; v < V; ++v) {
    int* row = s_T + v * E;
    const int total = block_exclusive_scan(row, E, 0x7fffffff);
    int* wr = a.wave_rows + (size_t)v * (E + 1);
    for (int g = tid; g < E; g += blockDim.x) wr[g] = row[g];
    if (tid == 0) wr[E] = total;
  }
}

// Row -> slice of wave v: the last g with wave_rows[g] <= row.
__device__ __forceinline__ int ep_find_slice(const int* wr, int E, int row) {
  int lo = 0, hi = E;  // wr[lo] <= row < wr[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (wr[mid] <= row) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Stores this rank's rows of wave v into the owners' X landing regions.
// `local_only`: copy only the slices this rank owns itself and raise no
// flags (the rest is pushed by the up GEMM's dispatch warps).
__global__ void __launch_bounds__(1024) ep_push_kernel(const __grid_constant__ EpArgs a, int v, int local_only) {
  __shared__ int s_wr[kEpMaxExperts + 1];
  __shared__ bool s_last;
  const int E = a.E;
  const int* wr = a.wave_rows + (size_t)v * (E + 1);
  for (int g = threadIdx.x; g <= E; g += blockDim.x) s_wr[g] = wr[g];
  __syncthreads();
  const bool ok = *reinterpret_cast<volatile int*>(a.abort_word) == 0;
  const int lane = threadIdx.x & 31;
  const int warps = (int)(blockDim.x >> 5) * gridDim.x;
  const int rows = s_wr[E];
  if (ok) {
    for (int row = (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); row < rows; row += warps) {
      const int g = ep_find_slice(s_wr, E, row);
      const EpSlice sl = a.slices[(size_t)v * E + g];
      if (local_only && sl.owner != a.rank) continue;
      const int r = row - s_wr[g];
      const uint8_t* src = a.x + (size_t)(sl.src_row + r) * a.row_bytes_x;
      uint8_t* dst = a.base[sl.owner] + a.off_x + (size_t)v * a.region_x_bytes + (size_t)(sl.dst_row + r) * a.row_bytes_x;
      warp_copy_row(dst, src, a.row_bytes_x, lane);
    }
  }
  if (local_only) return;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned prev;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.push_ctr + v) : "memory");
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    if (threadIdx.x == 0) a.push_ctr[v] = 0;
    __threadfence_system();
    const int p = threadIdx.x;
    // An aborted engine raises nothing, so its peers time out instead of
    // reading rows that never came.
    if (ok && p < a.world && p != a.rank) st_release_sys(&ep_flags(a, p)->data[v][a.rank], a.epoch);
  }
}

// Waits (one warp) until every peer's rows of wave v have landed here.
__global__ void ep_wait_kernel(const __grid_constant__ EpArgs a, int v) {
  const int p = threadIdx.x;
  if (p < a.world && p != a.rank && *reinterpret_cast<volatile int*>(a.abort_word) == 0)
    ep_wait_flag(&ep_flags(a, a.rank)->data[v][p], a.epoch, a);
}

// Announces this rank's outputs of wave v, waits for every owner's, and
// loads this rank's rows of wave v from the owners' Y outboxes into Y.
__global__ void __launch_bounds__(1024) ep_pull_kernel(const __grid_constant__ EpArgs a, int v) {
  __shared__ int s_wr[kEpMaxExperts + 1];
  const int E = a.E;
  if (blockIdx.x == 0 && threadIdx.x < a.world && (int)threadIdx.x != a.rank &&
      *reinterpret_cast<volatile int*>(a.abort_word) == 0) {
    __threadfence_system();
    st_release_sys(&ep_flags(a, threadIdx.x)->done[v][a.rank], a.epoch);
  }
  const int* wr = a.wave_rows + (size_t)v * (E + 1);
  for (int g = threadIdx.x; g <= E; g += blockDim.x) s_wr[g] = wr[g];
  if (threadIdx.x < a.world && (int)threadIdx.x != a.rank && *reinterpret_cast<volatile int*>(a.abort_word) == 0)
    ep_wait_flag(&ep_flags(a, a.rank)->done[v][threadIdx.x], a.epoch, a);
  __syncthreads();
  const bool ok = *reinterpret_cast<volatile int*>(a.abort_word) == 0;
  const int lane = threadIdx.x & 31;
  const int warps = (int)(blockDim.x >> 5) * gridDim.x;
  const int gwarp = (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5));
  if (ok) {
    const int rows = s_wr[E];
    for (int row = gwarp; row < rows; row += warps) {
      const int g = ep_find_slice(s_wr, E, row);
      const EpSlice sl = a.slices[(size_t)v * E + g];
      const int r = row - s_wr[g];
      const uint8_t* src =
          a.base[sl.owner] + a.off_y + (size_t)v * a.region_y_bytes + (size_t)(sl.dst_row + r) * a.row_bytes_y;
      uint8_t* dst = reinterpret_cast<uint8_t*>(a.y) + (size_t)(sl.src_row + r) * a.row_bytes_y;
      warp_copy_row(dst, src, a.row_bytes_y, lane);
    }
  }
  if (v == a.waves - 1) {  // rows at or past sum(group_sizes) are zero (ragged_dot)
    const int routed = *a.routed;
    const size_t n16 = (size_t)(a.M - routed) * (a.row_bytes_y >> 4);
    int4* t = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(a.y) + (size_t)routed * a.row_bytes_y);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
      t[i] = make_int4(0, 0, 0, 0);
  }
}

// Scatter mode: after this rank's down GEMM has stored every Y row it owns
// into the sources' landing areas, tell every source (one warp).
__global__ void ep_ydone_kernel(const __grid_constant__ EpArgs a) {
  const int p = threadIdx.x;
  if (*reinterpret_cast<volatile int*>(a.abort_word) != 0) return;
  __threadfence_system();
  if (p < a.world && p != a.rank) st_release_sys(&ep_flags(a, p)->ydone[a.rank], a.epoch);
}

// Scatter mode: waits until every owner has stored this rank's rows, then
// copies the landing area into the caller's Y (unless Y is the landing area)
// and zeroes Y's unrouted tail.
__global__ void __launch_bounds__(1024) ep_finish_kernel(const __grid_constant__ EpArgs a) {
  if (threadIdx.x < a.world && (int)threadIdx.x != a.rank && *reinterpret_cast<volatile int*>(a.abort_word) == 0)
    ep_wait_flag(&ep_flags(a, a.rank)->ydone[threadIdx.x], a.epoch, a);
  __syncthreads();
  const bool ok = *reinterpret_cast<volatile int*>(a.abort_word) == 0;
  const int routed = *a.routed;
  const int4* src = reinterpret_cast<const int4*>(a.base[a.rank] + a.off_yl);
  int4* y = reinterpret_cast<int4*>(a.y);
  const size_t n_routed = (size_t)routed * (a.row_bytes_y >> 4);
  const size_t n_all = (size_t)a.M * (a.row_bytes_y >> 4);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (ok && y != src)
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_routed; i += stride) y[i] = src[i];
  for (size_t i = n_routed + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_all; i += stride)
    y[i] = make_int4(0, 0, 0, 0);
}

}  // namespace moe
