/*
 * moe_b200 -- C ABI of the B200 (sm_100a) fused MoE expert-MLP library.
 *
 * Computes, over token rows pre-sorted by expert,
 *
 *     Y[rows of e] = GELU_tanh(X[rows of e] @ W_up[e]) @ W_down[e]
 *
 * with X (M, D), W_up (E, D, F), W_down (E, F, D), per-expert group sizes
 * (E,) int32 on the device, and Y (M, D) float32.  Rows at or past
 * sum(group_sizes) are written as zeros (jax.lax.ragged_dot semantics).
 *
 * All pointers are device pointers of the current CUDA device.  Calls are
 * stream-ordered on `stream` (a cudaStream_t; NULL = legacy default stream),
 * never synchronise the host, never allocate, and are safe to call from
 * several host threads on different streams as long as each call has its own
 * workspace.
 *
 * Return value: 0 on success, a negative MOE_ERR_* code otherwise; the text of
 * the last error of the calling thread is available from moe_last_error().
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Precision paths (argument `dtype`). */
enum {
  MOE_DTYPE_F32 = 0,            /* f32 X/W, 3xTF32 tensor-core products, f32 Y */
  MOE_DTYPE_BF16 = 1,           /* bf16 X/W, f32 accumulate, f32 Y              */
  MOE_DTYPE_FP8_E4M3_BLK128 = 2 /* bf16 X, e4m3 W + f32 128x128 block scales    */
};

/* Error codes. */
enum {
  MOE_OK = 0,
  MOE_ERR_INVALID_ARG = -1,
  MOE_ERR_UNSUPPORTED_SHAPE = -2,
  MOE_ERR_UNSUPPORTED_DTYPE = -3,
  MOE_ERR_WORKSPACE_TOO_SMALL = -4,
  MOE_ERR_CUDA = -5,
  MOE_ERR_DEVICE_TIMEOUT = -6,
  MOE_ERR_MISALIGNED = -7
};

/*
 * Fused expert MLP forward.
 *
 * Replaces the body of `fused_ragged_dot_caller(x, w_up, w_down, group_sizes,
 * *, BM, BF, max_group_size, interpret)` in the reference
 * (Krushna-B/pallas-moe-kernel src/kernel.py:85-123), i.e. the
 * `group_sizes_to_offsets` op (src/kernel.py:126-132) plus the
 * `pl.pallas_call` of `fused_mlp_one_expert` (src/kernel.py:9-82); the result
 * equals `ref_ragged_mlp` (src/kernel.py:152-175) within the precision of
 * `dtype`.  BM, BF and max_group_size are not arguments: the kernels walk the
 * real work units derived on the device from `group_sizes`.
 *
 * Kernels: D in {64, 128, 256} (f32: F % 64 == 0; bf16: F % 128 == 0) runs the
 * fused kernel with the hidden block on chip; every other shape runs two
 * grouped GEMMs with H through the workspace (f32 in 3xTF32; e4m3 weights
 * with small experts as expert super-tiles).  Any D and F whose rows start on
 * 16-byte boundaries are accepted: multiples of 4 (f32), 8 (bf16) or 16
 * (e4m3 weights); other shapes return MOE_ERR_UNSUPPORTED_SHAPE.
 *
 *   x            (M, D)   f32 (MOE_DTYPE_F32) or bf16 (other dtypes)
 *   w_up         (E, D, F) f32 / bf16 / e4m3 bytes
 *   w_down       (E, F, D) f32 / bf16 / e4m3 bytes
 *   group_sizes  (E,) int32, device memory; negative entries count as 0
 *   w_up_scale   (E, ceil(D/128), ceil(F/128)) f32 block scales (FP8 only, else NULL)
 *   w_down_scale (E, ceil(F/128), ceil(D/128)) f32 block scales (FP8 only, else NULL)
 *   y            (M, D) f32 output
 *   workspace    device scratch of at least moe_fused_mlp_workspace_size()
 *                bytes, 256-byte aligned (may be NULL when that size is 0)
 *   stream       cudaStream_t
 */
int moe_fused_mlp(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                  const float* w_up_scale, const float* w_down_scale, float* y, int64_t M, int32_t D, int32_t F,
                  int32_t E, int32_t dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes moe_fused_mlp needs for this problem (0 when none). */
size_t moe_fused_mlp_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E, int32_t dtype);
/* Number of kernel launches one moe_fused_mlp call with these arguments makes
 * on the current device under the current tuning (0 for M == 0), or a
 * negative MOE_ERR_* code.  Host-side: launches nothing. */
int moe_fused_mlp_launch_count(int64_t M, int32_t D, int32_t F, int32_t E, int32_t dtype);

/*
 * The launch plan of moe_fused_mlp for a problem, as the library would run it
 * on a device with `sms` SMs (<= 0: the current device).  No counterpart in
 * the reference; it feeds the analytic roofline model (src/analysis.py) with
 * the real tiling instead of a restatement of it.  No device work, no sync.
 * Fills out[0 .. min(count, max_out) - 1] in launch order and returns the
 * launch count (the value moe_fused_mlp_launch_count returns), or a negative
 * MOE_ERR_* code.  Grids are those of the automatic choices (persistent
 * kernels: one CTA per SM, or per SM pair) and of tuning keys 1 and 2 when
 * set; tuning key 4 (kernel family) is ignored.
 */
enum {
  MOE_MMA_NONE = 0,    /* no tensor-core work (conversion / split launches) */
  MOE_MMA_BF16 = 1,    /* tcgen05 kind::f16 on bf16 operands */
  MOE_MMA_BF16_E4M3 = 2, /* tcgen05 kind::f16 on bf16 operands, e4m3 weights decoded to bf16 in shared memory */
  MOE_MMA_TF32X3 = 3,  /* tcgen05 kind::tf32, three products per f32 product */
  MOE_MMA_F16_E4M3 = 4 /* tcgen05 kind::f16 on f16 operands, e4m3 weights decoded to f16 (down GEMM: f16 H) */
};
typedef struct moe_launch_desc {
  char kernel[48];       /* kernel family */
  int32_t grid;          /* CTAs launched */
  int32_t threads;       /* threads per CTA */
  int32_t smem_bytes;    /* shared memory per CTA (dynamic + static) */
  int32_t tmem_cols;     /* TMEM columns allocated per CTA (0: none) */
  int32_t cluster;       /* CTAs per cluster (2: CTA pair issuing cta_group::2 MMAs) */
  int32_t tile_m;        /* rows of one work unit (over the whole cluster) */
  int32_t tile_n;        /* grouped GEMM: output columns per tile; fused kernel: hidden columns per chunk */
  int32_t stage_k;       /* reduction elements per pipeline stage */
  int32_t stages;        /* operand ring stages */
  int32_t mma_kind;      /* MOE_MMA_* */
  int32_t gemm_n;        /* grouped GEMM: N; fused kernel: D */
  int32_t gemm_k;        /* grouped GEMM: K; fused kernel: F */
  int32_t f_splits;      /* fused kernel: F-splits per row block (1 elsewhere) */
  int32_t accumulators;  /* TMEM accumulator buffers in flight per CTA */
  int32_t reserved;
} moe_launch_desc;
int moe_describe_plan(int64_t M, int32_t D, int32_t F, int32_t E, int32_t dtype, int32_t sms, moe_launch_desc* out,
                      int32_t max_out);

/*
 * The expert-parallel engine's routing tables for one step, computed on the
 * host by the same code the engine's count kernel runs on the device (no
 * counterpart in the reference; it makes the tables testable without GPUs).
 * `counts` is the world x E table of rows each source routes to each global
 * expert in this step (host memory, row-major); row `rank` is this rank's own
 * group sizes, taken as moe_ep_forward takes them (negatives count as 0, the
 * running total is cut at M); the other rows are clamped to [0, max_rows].
 * Outputs (host memory): slices [waves][E][4] = {first source row, rows,
 * first row in the owner's landing region, owner} for this rank's rows;
 * wave_rows [waves][E + 1] = the slices' row prefix per wave; local_gs
 * [waves][num_local_experts] = this rank's landing-region group sizes;
 * recv [num_local_experts][world][4] = {first region row, rows, first source
 * row, source} (the scatter-mode receive table; may be null).  Returns the
 * status bits the device would raise (2 = a negative size was clamped, 8 =
 * rows were cut to M or a region) or a negative MOE_ERR_* code.
 */
int moe_ep_build_tables(const int32_t* counts, int32_t world, int32_t rank, int32_t num_local_experts,
                        int32_t waves, int32_t region_cap, int32_t max_rows, int64_t M, int32_t* slices,
                        int32_t* wave_rows, int32_t* local_gs, int32_t* recv);

/*
 * Two-stage form of moe_fused_mlp for weights that stay fixed across calls
 * (no counterpart in the reference, whose entry point re-reads the weights
 * every call; moe_fused_mlp == moe_prepare_weights + moe_fused_mlp_prepared).
 *
 * moe_prepare_weights writes the weight operands in the layout the kernel
 * reads (3xTF32: tf32 hi/lo planes, K-major) at the start of `workspace`;
 * for bf16 it does nothing.  moe_fused_mlp_prepared then runs the fused
 * kernel on a workspace prepared for the same (D, F, E, dtype) and the same
 * weights; its arguments mean what they mean for moe_fused_mlp.
 */
int moe_prepare_weights(const void* w_up, const void* w_down, const float* w_up_scale, const float* w_down_scale,
                        int32_t D, int32_t F, int32_t E, int32_t dtype, void* workspace, size_t workspace_bytes,
                        void* stream);
int moe_fused_mlp_prepared(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                           const float* w_up_scale, const float* w_down_scale, float* y, int64_t M, int32_t D,
                           int32_t F, int32_t E, int32_t dtype, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Allocation-free form of moe_fused_mlp for the f32 (3xTF32) path.  No
 * counterpart in the reference (its pallas_call always lets XLA allocate).
 *
 * For callers that hold only their input and output buffers and cannot
 * obtain device scratch: for example a host runtime that passes raw device
 * pointers through an FFI but exposes no device allocator, or a service that
 * reserves all device memory up front and forbids allocation on its request
 * path.  The scratch this path needs (the tf32 hi/lo weight planes) lives in
 * a 16 MiB array inside the library, resident on every GPU that loads the
 * library until the process exits; the call itself allocates and frees
 * nothing.
 *
 * Limits: D in {64, 128}, F % 64 == 0, E * D * F <= 1,048,576 (else
 * MOE_ERR_WORKSPACE_TOO_SMALL, and moe_fused_mlp with a workspace is the way).
 * The first call on a device looks up the scratch array's device address
 * (cudaGetSymbolAddress, a host-side runtime call); later calls reuse it.
 * After cudaDeviceReset the next call looks it up again (the array is a new
 * allocation of the new context and starts with undefined contents).
 * All calls share the one array: calls that can overlap on the GPU (other
 * streams, other host threads on the same device) race on it and must be
 * serialised by the caller.  Nothing in it has to start zeroed -- each call
 * writes every byte it later reads.  Arguments mean what they mean for
 * moe_fused_mlp with dtype = MOE_DTYPE_F32.
 */
int moe_fused_mlp_noalloc(const float* x, const float* w_up, const float* w_down, const int32_t* group_sizes,
                          float* y, int64_t M, int32_t D, int32_t F, int32_t E, void* stream);

/*
 * Expert-parallel engine: the fused expert MLP with its experts sharded over
 * `world` GPUs of one NVLink/NVSwitch node, one process (rank) per GPU.  No
 * counterpart in the reference, which runs on one device; this is the
 * dispatch -> experts -> combine exchange of an expert-parallel MoE layer
 * around the same kernels.
 *
 * Rank r owns global experts [r * num_local_experts, (r + 1) *
 * num_local_experts) and holds its own batch of rows sorted by global expert
 * (group_sizes has world * num_local_experts entries, as for moe_fused_mlp).
 * Each forward moves every row to its expert's rank, runs the fused MLP there
 * and brings the f32 result back to the row's original position, so that on
 * every rank Y equals moe_fused_mlp over all experts.  Transfers are our own
 * kernels over peer memory (CUDA IPC mappings of one buffer per rank): rows
 * are stored straight into the owner's landing buffer.  For D > 256 (the
 * two-GEMM experts: bf16 or e4m3 weights with D and F multiples of 256; other
 * two-GEMM shapes are refused) the combine is fused into the down GEMM: its epilogue
 * stores every Y row straight into the row's source rank (`waves` is then
 * 1).  For D <= 256 results are loaded back from the owner's outbox in
 * `waves` slices per step, so that the exchange of one slice overlaps the
 * experts of the next.  Group sizes are exchanged on the device: a forward
 * never synchronises the host.
 *
 * Set-up, on every rank with its own GPU current:
 *   moe_ep_create   allocates the engine (device memory proportional to
 *                   world * max_tokens rows; 0 comm_ctas = 16 SMs for the
 *                   exchange kernels, the experts run on the others);
 *   moe_ep_export   writes this rank's MOE_EP_HANDLE_BYTES-byte handle;
 *                   the caller gathers all ranks' handles in rank order by
 *                   any means (e.g. torch.distributed.all_gather) and then
 *                   calls
 *   moe_ep_connect  maps every peer's buffer (ranks must be distinct GPUs);
 *   moe_ep_set_weights  this rank's expert weights (E_local, D, F) /
 *                   (E_local, F, D) (+ FP8 block scales), kept by pointer
 *                   (prepared once for the f32 path).
 * Step:  moe_ep_forward on every rank, the same number of times on all
 *        ranks (it is a collective).  M <= max_tokens; x (M, D), y (M, D) f32.
 *        For D > 256, y may be NULL: Y is then left in the engine's own
 *        buffer (moe_ep_output; rows [0, M), valid until the next forward),
 *        which saves the final copy into the caller's array.
 * Exit:  moe_ep_destroy on every rank, after a host barrier that follows
 *        every rank's last forward having completed.
 *
 * Failure: every wait for a peer is bounded (2 s); a wait that runs out sets
 * status bit 4 (moe_device_status) and stops the engine's data movement for
 * good (that forward's and every later forward's routed rows of Y are
 * undefined; destroy the engine), so a dead peer never hangs a GPU.
 * Group sizes beyond M or beyond a landing region are cut (status bit 8).
 */
typedef struct moe_ep_s* moe_ep_t;
#define MOE_EP_HANDLE_BYTES 256

int moe_ep_create(int32_t rank, int32_t world, int32_t num_local_experts, int64_t max_tokens, int32_t D, int32_t F,
                  int32_t dtype, int32_t waves, int32_t comm_ctas, moe_ep_t* out);
int moe_ep_export(moe_ep_t ep, void* handle);
int moe_ep_connect(moe_ep_t ep, const void* handles);
int moe_ep_set_weights(moe_ep_t ep, const void* w_up_local, const void* w_down_local, const float* w_up_scale,
                       const float* w_down_scale, void* stream);
int moe_ep_forward(moe_ep_t ep, const void* x, const int32_t* group_sizes, float* y, int64_t M, void* stream);
/* Kernels one moe_ep_forward launches (exchange + expert kernels). */
int moe_ep_launches_per_forward(moe_ep_t ep);
/* Device address of the engine's own Y (D > 256 engines; NULL otherwise). */
void* moe_ep_output(moe_ep_t ep);
int moe_ep_destroy(moe_ep_t ep);

/*
 * Routing and permutation around the fused expert MLP.  No counterpart in the
 * reference, whose path starts from rows already sorted by expert (its
 * benchmarks build group_sizes directly, README.md:13); these produce that
 * input from router logits and fold the expert outputs back per token, so a
 * whole MoE layer runs as
 *     route_topk -> permute -> gather_rows -> moe_fused_mlp -> combine_rows.
 * Pointers are device pointers; calls are stream-ordered and allocate nothing.
 *
 * moe_route_topk   logits (T, E) f32 -> topk_ids (T, k) int32 (larger logit
 *                  first; ties to the lower expert id) and topk_weights
 *                  (T, k) f32 = softmax over the selected logits (the full
 *                  softmax renormalised to the top k).  E <= 1024, k <= 16.
 *                  A slot without a finite winner gets id -1, weight 0.
 * moe_permute      expert_ids (N = T * k entries, entry i = t * k + j) ->
 *                  group_sizes (E,), sorted_src (N,) = entry index of each
 *                  row in expert order (stable: entries of one expert keep
 *                  their order), inverse (N,) = row of each entry (-1 for an
 *                  id outside [0, E): dropped, status bit 16).  Needs
 *                  moe_permute_workspace_size(N, E) bytes of workspace.
 *                  Rows past sum(group_sizes) of sorted_src are untouched.
 * moe_gather_rows  out[r] = x[sorted_src[r] / k] for rows of row_bytes (a
 *                  multiple of 16) -- X in expert order for moe_fused_mlp.
 * moe_combine_rows y[t] = sum_j topk_weights[t, j] * y_sorted[inverse[t*k+j]]
 *                  (f32, D a multiple of 4, slots summed in order).
 */
int moe_route_topk(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* topk_ids, float* topk_weights,
                   void* stream);
size_t moe_permute_workspace_size(int64_t N, int32_t E);
int moe_permute(const int32_t* expert_ids, int64_t N, int32_t E, int32_t* group_sizes, int32_t* sorted_src,
                int32_t* inverse, void* workspace, size_t workspace_bytes, void* stream);
int moe_gather_rows(const void* x, const int32_t* sorted_src, int64_t rows, int32_t k, int32_t row_bytes, void* out,
                    void* stream);
int moe_combine_rows(const float* y_sorted, const int32_t* inverse, const float* topk_weights, int64_t T, int32_t k,
                     int32_t D, float* y, void* stream);

/*
 * SwiGLU experts: Y = ragged_dot(SiLU(ragged_dot(X, W_gate)) * ragged_dot(X,
 * W_up), W_down), the expert MLP of Mixtral / DeepSeek-style layers.  No
 * counterpart in the reference, whose expert MLP is GELU-tanh only
 * (src/kernel.py:46-63); the ragged layout, group_sizes semantics, rows past
 * sum(group_sizes) (zeros) and the error codes are those of moe_fused_mlp.
 * bf16 only; D a multiple of 256, F a multiple of 128.
 *
 * moe_swiglu_interleave  w_gate, w_up (E, D, F) bf16 -> w_gate_up (E, D, 2F):
 *                  columns interleaved every 128 (gate 0..127, up 0..127,
 *                  gate 128..255, ...), the operand layout of the up GEMM.
 *                  Run once per set of weights.
 * moe_fused_mlp_swiglu   x (M, D) bf16, w_gate_up (E, D, 2F) bf16 from
 *                  moe_swiglu_interleave, w_down (E, F, D) bf16 -> y (M, D)
 *                  f32.  H = SiLU(gate) * up goes through the workspace as
 *                  bf16 (M, F): moe_fused_mlp_swiglu_workspace_size bytes,
 *                  256-byte aligned.
 */
int moe_swiglu_interleave(const void* w_gate, const void* w_up, void* w_gate_up, int32_t E, int32_t D, int32_t F,
                          void* stream);
size_t moe_fused_mlp_swiglu_workspace_size(int64_t M, int32_t D, int32_t F);
int moe_fused_mlp_swiglu(const void* x, const void* w_gate_up, const void* w_down, const int32_t* group_sizes,
                         float* y, int64_t M, int32_t D, int32_t F, int32_t E, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * SwiGLU experts with e4m3 weights and 128 x 128 f32 block scales (the
 * DeepSeek-V3 weight format).  Dequantised weight = e4m3 value * its block's
 * scale, as for MOE_DTYPE_FP8_E4M3_BLK128; x is bf16; the GEMMs run on f16
 * operands with f32 accumulation.  D a multiple of 256, F of 128.
 *
 * moe_swiglu_interleave_fp8  w_gate, w_up (E, D, F) e4m3 with s_gate, s_up
 *                  (E, D/128, F/128) -> w_gate_up (E, D, 2F) interleaved every
 *                  128 columns and s_gate_up (E, D/128, 2F/128) (one gate
 *                  block, then the up block of the same columns).
 * moe_fused_mlp_swiglu_fp8   y (M, D) f32 from x, w_gate_up / s_gate_up and
 *                  w_down (E, F, D) e4m3 / s_down (E, F/128, D/128); workspace
 *                  moe_fused_mlp_swiglu_fp8_workspace_size bytes (H in f16),
 *                  256-byte aligned.
 */
int moe_swiglu_interleave_fp8(const void* w_gate, const void* w_up, const float* s_gate, const float* s_up,
                              void* w_gate_up, float* s_gate_up, int32_t E, int32_t D, int32_t F, void* stream);
size_t moe_fused_mlp_swiglu_fp8_workspace_size(int64_t M, int32_t D, int32_t F);
int moe_fused_mlp_swiglu_fp8(const void* x, const void* w_gate_up, const void* w_down, const float* s_gate_up,
                             const float* s_down, const int32_t* group_sizes, float* y, int64_t M, int32_t D,
                             int32_t F, int32_t E, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Training: forward with the pre-activation saved, and the backward.  No
 * counterpart in the reference, which has no backward pass (its kernel is
 * forward-only, src/kernel.py:9-123); the forward math, ragged layout and
 * group_sizes semantics are those of moe_fused_mlp.  bf16 operands, f32
 * accumulation; D and F multiples of 256; E <= 4096.
 *
 * moe_fused_mlp_forward_train  as moe_fused_mlp with MOE_DTYPE_BF16 (always
 *                  on the two grouped GEMMs), plus a_save (M, F) bf16 = the
 *                  pre-activation X W_up[e] of every routed row (rows past
 *                  sum(group_sizes) untouched).  Workspace:
 *                  moe_fused_mlp_forward_train_workspace_size bytes.
 * moe_fused_mlp_backward  given dy (M, D) (dy_dtype MOE_DTYPE_F32 or
 *                  MOE_DTYPE_BF16) and the forward's a_saved:
 *                    dx      (M, D) f32 = (dy W_down[e]^T * GELU'(A)) W_up[e]^T,
 *                            rows past sum(group_sizes) zero;
 *                    dw_up   (E, D, F) f32 = X_e^T (dy_e W_down[e]^T * GELU'(A_e));
 *                    dw_down (E, F, D) f32 = GELU(A_e)^T dy_e;
 *                  experts without rows get zero weight gradients.  dy and
 *                  the intermediate dA and GELU(A) are rounded to bf16 for
 *                  the tensor cores.  Workspace:
 *                  moe_fused_mlp_backward_workspace_size bytes (256-byte
 *                  aligned; padded copies of X, dy, dA and GELU(A)).
 */
size_t moe_fused_mlp_forward_train_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E);
int moe_fused_mlp_forward_train(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                                float* y, void* a_save, int64_t M, int32_t D, int32_t F, int32_t E, void* workspace,
                                size_t workspace_bytes, void* stream);
size_t moe_fused_mlp_backward_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E);
int moe_fused_mlp_backward(const void* x, const void* w_up, const void* w_down, const int32_t* group_sizes,
                           const void* a_saved, const void* dy, int32_t dy_dtype, float* dx, float* dw_up,
                           float* dw_down, int64_t M, int32_t D, int32_t F, int32_t E, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * SwiGLU training (bf16; D and F multiples of 256; E <= 4096).  Weights as for
 * moe_fused_mlp_swiglu: w_gate_up (E, D, 2F) interleaved every 128 columns.
 *
 * moe_fused_mlp_swiglu_forward_train  as moe_fused_mlp_swiglu, plus gu_save
 *                  (M, 2F) bf16 = the raw gate and up columns X W_gate_up[e]
 *                  of every routed row, in the weights' interleave.
 * moe_fused_mlp_swiglu_backward  given dy (f32 or bf16) and gu_saved:
 *                    dx         (M, D) f32, rows past sum(group_sizes) zero;
 *                    dw_gate_up (E, D, 2F) f32, interleaved like w_gate_up;
 *                    dw_down    (E, F, D) f32;
 *                  with s = sigmoid(gate): dGate = (dy W_down^T) up s (1 +
 *                  gate (1 - s)), dUp = (dy W_down^T) gate s, H = gate s up.
 */
size_t moe_fused_mlp_swiglu_forward_train_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E);
int moe_fused_mlp_swiglu_forward_train(const void* x, const void* w_gate_up, const void* w_down,
                                       const int32_t* group_sizes, float* y, void* gu_save, int64_t M, int32_t D,
                                       int32_t F, int32_t E, void* workspace, size_t workspace_bytes, void* stream);
size_t moe_fused_mlp_swiglu_backward_workspace_size(int64_t M, int32_t D, int32_t F, int32_t E);
int moe_fused_mlp_swiglu_backward(const void* x, const void* w_gate_up, const void* w_down,
                                  const int32_t* group_sizes, const void* gu_saved, const void* dy, int32_t dy_dtype,
                                  float* dx, float* dw_gate_up, float* dw_down, int64_t M, int32_t D, int32_t F,
                                  int32_t E, void* workspace, size_t workspace_bytes, void* stream);

/* Text of the calling thread's last error ("" when none). */
const char* moe_last_error(void);

/*
 * Reads the device status word of the current device (bits: 1 = a pipeline
 * wait timed out, 2 = a negative group size was clamped, 4 = an
 * expert-parallel wait for a peer timed out, 8 = group sizes were cut to fit
 * M or a landing region, 16 = an expert id outside [0, E) was dropped by
 * moe_permute).  Synchronises the device.  When `reset` is
 * non-zero the word is cleared afterwards.
 * Returns the bits (>= 0) or MOE_ERR_CUDA.
 */
int moe_device_status(int reset);

/* Library version: major * 10000 + minor * 100 + patch. */
int moe_version(void);

/*
 * Clock evidence for benchmarks (no counterpart in the reference).  Launches
 * `blocks` one-thread blocks on `stream`; block b writes out[3 b .. 3 b + 2]
 * = {SM id, the SM's cycle counter (clock64), the global nanosecond timer}.
 * Two samples taken around a region on the same stream give, for every SM
 * that appears in both, the SM clock averaged over the region:
 * cycles / nanoseconds.  `out` is device memory of 3 * blocks uint64 values;
 * blocks in 1 .. 1024.  Returns 0 or a negative MOE_ERR_* code.
 */
int moe_sm_clock_sample(uint64_t* out, int32_t blocks, void* stream);

/*
 * Tuning overrides for tests and benchmarks (0 restores the automatic
 * choice).  Keys: 1 = F-splits per 128-row block (power of two),
 * 2 = persistent CTAs per launch, 3 = device address of an event-trace
 * buffer (read only by builds compiled with -DMOE_TRACE), 4 = kernel family
 * (0 automatic, 1 one CTA per 128-row block, 2 CTA pairs per 256 rows),
 * 5 = grouped GEMMs' tile rasterisation group in 256-row blocks (1 .. 64;
 * 0 = 8), 6 = grouped GEMMs' L2 hints for the A / B tile loads (0 evict_last
 * for both, 1 evict_normal for both, 2 A evict_first, 3 B evict_first),
 * 7 = e4m3-weight GELU experts (0 automatic: expert super-tiles when M <=
 * 384 E, 1 row-tiled pair kernel, 2 expert super-tiles), 8 = bf16 down GEMM
 * tile width (0 automatic = 256 columns, 1 256 columns, 2 512 columns),
 * 10 = fused small-D kernel's last wave (0 automatic: a last wave of at most
 * half the grid runs as half units when the call's preparation launch runs
 * anyway, 1 whole units only).
 * Returns 0 or MOE_ERR_INVALID_ARG.
 */
int moe_set_tuning(int32_t key, int64_t value);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
