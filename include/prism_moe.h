/*
 * prism_moe.h — C ABI of the B200-native (sm_100a) Qwen3-MoE sparse block.
 *
 * Library: libprism_moe.so (built from prism_infer_b200/csrc by prism_infer_b200/build.py).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (``void*`` holding a
 * cudaStream_t; NULL = legacy default stream), launches asynchronously on that stream and
 * returns an ``int`` status (PRISM_MOE_OK = 0). Nothing here allocates device memory: the
 * caller owns every buffer, including the workspaces sized by the *_workspace_size helpers.
 * On a non-zero status, prism_moe_last_error() returns a message (thread-local).
 *
 * Kernels never trap. Waits inside kernels are bounded; a wait that runs out records
 * PRISM_MOE_ERR_TIMEOUT in a device error word that the host reads back with
 * prism_moe_read_device_error().
 *
 * Element types: PRISM_MOE_F32 (float) or PRISM_MOE_BF16 (bfloat16, IEEE bit layout, the
 * upper half of a float). Index outputs that the reference returns as torch.int64 are int64.
 *
 * The reference this ABI replaces is pure PyTorch; each function names the reference code
 * (path:line within SparkSnail/prism-infer) whose behaviour it reproduces.
 */
#ifndef PRISM_MOE_H_
#define PRISM_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PRISM_MOE_OK 0
#define PRISM_MOE_ERR_ARG 1          /* invalid argument (shape, dtype, null pointer, size)   */
#define PRISM_MOE_ERR_CUDA 2         /* a CUDA runtime / driver call failed                    */
#define PRISM_MOE_ERR_TIMEOUT 3      /* a bounded in-kernel wait ran out                       */
#define PRISM_MOE_ERR_UNSUPPORTED 4  /* shape or device outside what the kernels implement     */
#define PRISM_MOE_ERR_DEVICE 5       /* a kernel recorded an error in its device error word    */

#define PRISM_MOE_F32 0
#define PRISM_MOE_BF16 1

/* Expert GEMM engines (prism_moe_set_expert_engine). */
#define PRISM_MOE_ENGINE_AUTO 0    /* chosen per call from the rows per segment (default)     */
#define PRISM_MOE_ENGINE_FUSED 1   /* gate_up and down in one persistent launch, 128-row tiles */
#define PRISM_MOE_ENGINE_SINGLE 2  /* two launches, 128-row tiles                              */
#define PRISM_MOE_ENGINE_PAIR 3    /* two launches, 256-row tiles on CTA pairs (cta_group::2)  */

/* Library version (major*10000 + minor*100 + patch). */
int prism_moe_version(void);

/* Message describing the last non-zero status returned on this thread. */
const char* prism_moe_last_error(void);

/*
 * Router post-processing of one MoE block: fp32 softmax over the experts, top-k, optional
 * renormalisation of the k weights, cast of the weights to the logits' dtype.
 * Replaces prism_infer/layers/moe.py:77-81 (F.softmax(dtype=float) -> torch.topk -> /sum ->
 * .to(dtype)), reproducing torch's CUDA results bit for bit: the softmax sums in the order of
 * torch's warp softmax, top-k resolves ties as torch.topk on CUDA does (values equal to the
 * k-th are taken in ascending expert index, output order from torch's 32-wide bitonic sort),
 * and the renormalisation sum follows torch's reduction tree.
 *   logits        [T, E] row-major, dtype
 *   topk_ids      [T, k] int64 out
 *   topk_weights  [T, k] dtype out
 *   expert_counts [E] int32 out, or NULL (rows routed to each expert; zeroed first)
 * Limits: 1 <= E <= 1024, 1 <= k <= min(E, 32).
 */
int prism_moe_route_topk(const void* logits, int dtype, int64_t num_tokens, int32_t num_experts,
                         int32_t top_k, int32_t renorm, int64_t* topk_ids, void* topk_weights,
                         int32_t* expert_counts, void* stream);

/* Bytes of scratch prism_moe_build_dispatch_plan needs. */
size_t prism_moe_dispatch_workspace_size(int64_t num_tokens, int32_t top_k, int32_t num_experts,
                                         int32_t ep_size);

/*
 * Dispatch plan of the routed entries (flat index f = t*k + j), by a deterministic counting
 * sort. Replaces prism_infer/engine/parallel/expert_parallel.py:23-42 (build_dispatch_plan:
 * dst = id // E_l, perm = stable argsort(dst), input_splits = bincount(dst),
 * sorted_local_eid = (id % E_l)[perm]) and the per-expert grouping of
 * prism_infer/layers/moe.py:91-93. Outputs (each may be NULL if not wanted):
 *   perm             [T*k] int64  — identical to the reference's perm
 *   input_splits     [W]   int64  — rows sent to each EP rank
 *   sorted_local_eid [T*k] int64  — local expert id of perm's entries
 *   expert_counts    [E]   int32  — rows per expert
 *   expert_offsets   [E+1] int32  — exclusive scan of expert_counts
 *   entry_row        [T*k] int32  — row of entry f in expert-major order (experts ascending,
 *                                   flat order inside an expert); the layout the expert GEMMs
 *                                   and the EP send buffer use.
 * Requires num_experts % ep_size == 0 (the reference asserts the same,
 * expert_parallel.py:103). Expert ids must lie in [0, num_experts): the reference fails on
 * others (bincount of a negative destination, or an all_to_all split past the group). Here an
 * entry with an id outside that range is left out of every output (entry_row = -1; its perm and
 * sorted_local_eid slots, past the valid entries, are not written; the counts and splits do not
 * include it) and the kernel records PRISM_MOE_ERR_ARG in the workspace's first int32 word,
 * which prism_moe_read_device_error(workspace, stream) returns and clears. The workspace must
 * start zeroed.
 */
int prism_moe_build_dispatch_plan(const int64_t* topk_ids, int64_t num_tokens, int32_t top_k,
                                  int32_t num_experts, int32_t ep_size, int64_t* perm,
                                  int64_t* input_splits, int64_t* sorted_local_eid,
                                  int32_t* expert_counts, int32_t* expert_offsets,
                                  int32_t* entry_row, void* workspace, size_t workspace_bytes,
                                  void* stream);

/*
 * prism_moe_build_dispatch_plan without a workspace argument, for callers that cannot allocate
 * device memory (a plugin called from a host framework's execute/enqueue callback that only
 * hands over buffers it owns, or an embedded runtime whose device memory all belongs to its
 * own pool). This entry point has no counterpart in the reference. Its scratch is a fixed
 * 1 MiB __device__ array inside the library (held by every GPU that loads the library until
 * the process exits); outputs are those of prism_moe_build_dispatch_plan, bit for bit.
 * Limits: num_tokens * top_k <= 65536, num_experts <= 256, ep_size <= 64 — larger problems
 * return PRISM_MOE_ERR_ARG. The first call on a device looks up the array's address on that
 * device (make it before any stream capture starts). Calls share the array: calls whose
 * kernels may overlap on the GPU race and must be serialised. Allocates nothing.
 * Expert ids must lie in [0, num_experts); entries outside it are left out of the outputs as
 * in prism_moe_build_dispatch_plan, but the error word that records them lives in the shared
 * array and is not reported to the caller.
 */
int prism_moe_build_dispatch_plan_static(const int64_t* topk_ids, int64_t num_tokens,
                                         int32_t top_k, int32_t num_experts, int32_t ep_size,
                                         int64_t* perm, int64_t* input_splits,
                                         int64_t* sorted_local_eid, int32_t* expert_counts,
                                         int32_t* expert_offsets, int32_t* entry_row,
                                         void* stream);

/*
 * Gather token rows into expert-major order: x_sorted[entry_row[t*k + j]] = x[t].
 * Replaces prism_infer/engine/parallel/expert_parallel.py:154-156 (repeat_interleave + [perm])
 * and the per-expert x[token_idx] gathers of prism_infer/layers/moe.py:96. 16-byte vector
 * copies; rows must be 16-byte aligned (hidden * sizeof(dtype) % 16 == 0).
 */
int prism_moe_permute_rows(const void* x, int dtype, int64_t num_tokens, int64_t hidden,
                           int32_t top_k, const int32_t* entry_row, void* x_sorted, void* stream);

/* Bytes of scratch prism_moe_expert_swiglu needs for rows_capacity rows. */
size_t prism_moe_expert_workspace_size(int64_t rows_capacity, int64_t hidden, int64_t inter,
                                       int dtype);

/*
 * Grouped SwiGLU experts: for every segment s, rows [seg_offsets[s], seg_offsets[s+1]) of
 * x_sorted go through expert e = seg_expert[s] (or e = s when seg_expert is NULL):
 *   y = (silu(x Wg_e^T) * (x Wu_e^T)) Wd_e^T
 * with w_gate_up[e] = [Wg_e; Wu_e] of shape [2I, H] (gate rows first) and w_down[e] [H, I].
 * Replaces prism_infer/layers/moe.py:27-28 with activation.py:8-11, run per expert by the loops
 * of moe.py:92-96 and expert_parallel.py:165-169. bf16 runs on tcgen05 tensor cores (fp32
 * accumulation in TMEM, TMA-fed, SwiGLU fused into the first GEMM's epilogue); f32 runs on
 * CUDA cores in fp32. The intermediate gate/up values and the activation are rounded to
 * dtype where the reference materialises them.
 *   seg_offsets   [num_segments+1] int32, device, non-decreasing, last <= rows_capacity
 *   device_error  int32 device word, or NULL; a kernel that fails records its status there
 * Rows of x_sorted/y beyond the last segment are not touched. bf16 needs hidden % 8 == 0 and
 * inter % 8 == 0.
 */
int prism_moe_expert_swiglu(const void* x_sorted, int dtype, int64_t rows_capacity,
                            int64_t hidden, int64_t inter, const int32_t* seg_offsets,
                            const int32_t* seg_expert, int32_t num_segments,
                            int32_t num_local_experts, const void* w_gate_up, const void* w_down,
                            void* y, void* workspace, size_t workspace_bytes, int* device_error,
                            void* stream);

/*
 * Weighted combine: out[t] = sum_j w[t, j] * expert_out[row(t*k + j)], row = entry_row[f]
 * (identity when entry_row is NULL). Each product is rounded to dtype and the k products are
 * summed in fp32 in slot order, then rounded once: the numerics of the reference's
 * combine_weighted_sum. Replaces prism_infer/engine/parallel/expert_parallel.py:45-57 fused
 * with the un-permute of :173-174, and the index_add_ accumulation of
 * prism_infer/layers/moe.py:97-98.
 */
int prism_moe_combine(const void* expert_out, int dtype, const int32_t* entry_row,
                      const void* topk_weights, int64_t num_tokens, int32_t top_k, int64_t hidden,
                      void* out, void* stream);

/*
 * RMSNorm of [T, H] rows, optionally after adding the residual stream — the decoder layer's
 * norms, replacing prism_infer/layers/layernorm.py:16-40 (rms_forward when ``residual`` is NULL,
 * else add_rms_forward). Numerics as the reference: xf = float(x) (+ float(residual)),
 * residual_out = dtype(xf), out = dtype(dtype(xf * rsqrt(mean(xf^2) + eps)) * weight); the
 * reference compiles these with torch.compile, so sums of squares agree to rounding, not bits.
 *   x, residual, out, residual_out [T, H], weight [H]: dtype, 16-byte aligned rows.
 * ``out`` may be ``x`` or ``residual``; ``residual_out`` (required with a residual) may not.
 * One warp per row.
 */
int prism_moe_rmsnorm(const void* x, const void* residual, const void* weight, float eps,
                      int dtype, int64_t num_tokens, int64_t hidden, void* out,
                      void* residual_out, void* stream);

/*
 * The decoder layer's next residual add and RMSNorm, applied to the block output inside the
 * combine kernel (prism_infer/models/qwen3.py:179-186 runs them as the next layer's
 * input_layernorm(hidden, residual), layernorm.py:28-40): the *_norm entry points write
 *   residual_out = dtype(float(block output) + float(residual))
 *   out          = RMSNorm(that sum) with norm_weight and eps
 * instead of the block output, bit for bit what the plain entry point followed by
 * prism_moe_rmsnorm(out, residual, ...) gives, without the block output's round trip through
 * HBM. ``residual_out`` may alias neither ``residual`` nor ``out``.
 */
typedef struct prism_moe_norm_epilogue {
  const void* residual;      /* [T, H] dtype */
  const void* norm_weight;   /* [H] dtype    */
  float eps;
  void* residual_out;        /* [T, H] dtype */
} prism_moe_norm_epilogue;

/* Bytes of scratch prism_moe_block_forward needs. */
size_t prism_moe_block_workspace_size(int64_t num_tokens, int64_t hidden, int64_t inter,
                                      int32_t num_experts, int32_t top_k, int dtype);

/*
 * The whole single-GPU block after the router GEMM: route, plan, gather, grouped SwiGLU
 * experts, weighted combine. Replaces prism_infer/layers/moe.py:77-100 (the reference computes
 * router_logits = F.linear(x, W_gate) at moe.py:74 with its BLAS; the caller does the same and
 * passes the logits here, so routing sees the reference's exact logits).
 *   x [T, H], router_logits [T, E], w_gate_up [E, 2I, H], w_down [E, H, I], out [T, H]: dtype
 *   topk_ids [T, k] int64 and topk_weights [T, k] dtype: optional outputs (NULL = not wanted)
 * The workspace's first 4 bytes are the device error word read by
 * prism_moe_read_device_error().
 */
int prism_moe_block_forward(const void* x, const void* router_logits, int dtype,
                            int64_t num_tokens, int64_t hidden, int64_t inter,
                            int32_t num_experts, int32_t top_k, int32_t renorm,
                            const void* w_gate_up, const void* w_down, void* out,
                            int64_t* topk_ids, void* topk_weights, void* workspace,
                            size_t workspace_bytes, void* stream);

/* prism_moe_block_forward with the decoder layer's residual add + RMSNorm fused into the
 * combine (``epilogue`` NULL: identical to prism_moe_block_forward). */
int prism_moe_block_forward_norm(const void* x, const void* router_logits, int dtype,
                                 int64_t num_tokens, int64_t hidden, int64_t inter,
                                 int32_t num_experts, int32_t top_k, int32_t renorm,
                                 const void* w_gate_up, const void* w_down, void* out,
                                 int64_t* topk_ids, void* topk_weights, void* workspace,
                                 size_t workspace_bytes, void* stream,
                                 const prism_moe_norm_epilogue* epilogue);

/* ---------------------------------------------------------------------------------------------
 * Expert parallelism over NVLink peer memory (one process per GPU).
 *
 * Replaces the reference's NCCL exchange — counts all_to_all + host .tolist() and the three
 * variable all_to_all_single calls (prism_infer/engine/parallel/expert_parallel.py:113-136,
 * :157-162, :172) — with device-side exchange: every rank allocates one landing zone, shares it
 * through CUDA IPC, and each step writes rows straight into the owners' memory. Waits between
 * ranks are bounded (10 s) and record PRISM_MOE_ERR_TIMEOUT in the workspace's error word.
 * --------------------------------------------------------------------------------------------- */

/* Bytes of one rank's landing zone for up to ``max_tokens`` tokens per rank (identical on all
 * ranks: they must pass the same arguments). */
size_t prism_moe_ep_landing_bytes(int32_t ep_size, int64_t max_tokens, int32_t top_k,
                                  int64_t hidden, int32_t num_experts, int dtype);

/* Allocate (cudaMalloc) and zero the flag area of a landing zone on the current device, and
 * write its CUDA IPC handle (prism_moe_ep_ipc_handle_bytes() bytes) to ``ipc_handle``. These
 * setup calls are the only ones in the library that allocate. */
int prism_moe_ep_alloc_landing(size_t bytes, void** ptr, void* ipc_handle);
int prism_moe_ep_free_landing(void* ptr);
int prism_moe_ep_ipc_handle_bytes(void);

/* Map / unmap a peer rank's landing zone from its IPC handle. */
int prism_moe_ep_open_peer(const void* ipc_handle, void** ptr);
int prism_moe_ep_close_peer(void* ptr);

/* Bytes of the per-rank workspace prism_moe_ep_forward needs. Zero-fill it once before the
 * first step and pass the same workspace to every step (it carries completion counters). */
size_t prism_moe_ep_workspace_size(int64_t max_tokens, int64_t hidden, int64_t inter,
                                   int32_t num_experts, int32_t top_k, int32_t ep_size, int dtype);

/*
 * One expert-parallel MoE block step on this rank (bf16). Replaces
 * prism_infer/layers/moe.py:77-85 + ExpertParallelMoE.forward
 * (prism_infer/engine/parallel/expert_parallel.py:140-176). Collective: every rank of the EP
 * group calls it once per step. ``epoch`` numbers the step: either 0 on every call (the library
 * keeps the count in the workspace, so the arguments do not change from step to step and a
 * step can be captured in a CUDA graph and replayed; every rank must then make the same number
 * of calls) or the caller's count (1, 2, 3, ... increasing by one, the same on all ranks).
 *   x [T, H], out [T, H]; either router_logits [T, E] (routed here as prism_moe_route_topk) or
 *   topk_ids [T, k] int64 + topk_weights [T, k].
 *   w_gate_up [E/W, 2I, H], w_down [E/W, H, I]: this rank's experts e in [rank*E/W, (rank+1)*E/W)
 *   my_landing: this rank's landing zone; peer_landing: DEVICE array of W uint64 landing-zone
 *   addresses as mapped in this process (entry ep_rank = my_landing).
 * T <= max_tokens (the landing capacity). Kernels: route (when logits are given), dispatch plan,
 * a copy of x into the landing zone, counts all-gather, one fused expert launch (both GEMMs; its
 * copy warps fill this rank's receive buffer, pulling the rows other ranks routed here over
 * NVLink, one row per token and rank; its down epilogue writes the outputs back into the
 * sources' buffers), wait for the returned rows, combine.
 * Caller-given topk_ids outside [0, num_experts) are not sent anywhere (their slots add nothing
 * to ``out``) and record PRISM_MOE_ERR_ARG in the workspace's error word. When a wait for other
 * ranks runs out, PRISM_MOE_ERR_TIMEOUT is recorded there, the rest of that step does nothing
 * and ``out`` is undefined; the group should then be torn down.
 */
int prism_moe_ep_forward(const void* x, const void* router_logits, const int64_t* topk_ids,
                         const void* topk_weights, int dtype, int64_t num_tokens,
                         int64_t max_tokens, int64_t hidden, int64_t inter, int32_t num_experts,
                         int32_t top_k, int32_t renorm, int32_t ep_size, int32_t ep_rank,
                         const void* w_gate_up, const void* w_down, void* my_landing,
                         const uint64_t* peer_landing, uint64_t epoch, void* out,
                         void* workspace, size_t workspace_bytes, void* stream);

/* prism_moe_ep_forward with the decoder layer's residual add + RMSNorm fused into the final
 * combine (``epilogue`` NULL: identical to prism_moe_ep_forward). */
int prism_moe_ep_forward_norm(const void* x, const void* router_logits, const int64_t* topk_ids,
                              const void* topk_weights, int dtype, int64_t num_tokens,
                              int64_t max_tokens, int64_t hidden, int64_t inter,
                              int32_t num_experts, int32_t top_k, int32_t renorm,
                              int32_t ep_size, int32_t ep_rank, const void* w_gate_up,
                              const void* w_down, void* my_landing, const uint64_t* peer_landing,
                              uint64_t epoch, void* out, void* workspace, size_t workspace_bytes,
                              void* stream, const prism_moe_norm_epilogue* epilogue);

/*
 * Statistics of the last prism_moe_ep_forward step that used ``workspace`` (synchronises
 * ``stream``). ``stats`` receives 8 uint64 values: [0] the step's epoch, [1] the workspace's
 * epoch counter, [2] and [3] %globaltimer ns when the first dispatch chunk was claimed and when
 * the last one was stored, [4] and [5] when the fused expert launch's first CTA started and its
 * last CTA finished, [6] token rows this rank pulled from other ranks over NVLink (one per token
 * and rank, however many of this rank's experts the token chose), [7] rows this rank returned
 * to other ranks after the down GEMM (one per routed entry). Row bytes = hidden * 2. The
 * reference has no equivalent; this feeds the all-to-all bandwidth a benchmark reports.
 */
int prism_moe_ep_read_stats(const void* workspace, uint64_t* stats, void* stream);

/*
 * Process-wide controls, for tests and tuning (the defaults need no call).
 * prism_moe_set_expert_engine: the expert GEMM engine for calls without an expert-parallel
 * exchange (PRISM_MOE_ENGINE_*; AUTO picks by rows per segment; expert-parallel steps always use
 * the fused launch). prism_moe_set_wait_limits: the bound, in ns, of every in-kernel wait on this
 * GPU's own pipeline (default 2 s) and of every wait for other ranks (default 10 s); 0 restores a
 * default, values above 60 s are rejected. The limits are read when a kernel is launched.
 * Neither has a counterpart in the reference.
 */
int prism_moe_set_expert_engine(int engine);
int prism_moe_set_wait_limits(int64_t wait_ns, int64_t peer_wait_ns);

/*
 * Profiling hook: CUDA events (cudaEvent_t handles owned by the caller) that the following
 * calls on this thread record on their stream at stage boundaries — slot 0 route begin,
 * 1 dispatch-plan begin, 2 permute begin (EP: counts all-gather begin), 3 gate_up GEMM begin,
 * 4 down GEMM begin, 5 combine begin, 6 combine end (prism_moe_expert_swiglu records slots 3-5;
 * when both GEMMs run as one fused launch — always under expert parallelism — slot 4 is
 * recorded with slot 5, after the launch). ``count`` = 0 turns it off.
 * The reference has no equivalent (it times whole engine steps with host clocks,
 * prism_infer bench/bench.py:445-452); this exists so a benchmark can time each kernel on the
 * device inside its timed region.
 */
int prism_moe_profile_events(void* const* events, int32_t count);

/*
 * Synchronise ``stream`` and return the status recorded in a device error word
 * (PRISM_MOE_OK if none), clearing it. ``device_error`` is the int32 word passed to
 * prism_moe_expert_swiglu, or the start of a prism_moe_block_forward workspace.
 */
int prism_moe_read_device_error(int* device_error, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PRISM_MOE_H_ */
