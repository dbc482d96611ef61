// Host-side entry points of the kernels, shared by the extern "C" layer (capi.cu,
// dispatch_static.cu). Every function validates its own launch-specific limits and returns a
// PRISM_MOE_* status.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace prism {

// State of one expert-parallel step, kept at a fixed offset (kEpStepOffset) of the EP workspace.
// ep_counts_kernel fills it at the start of every step; the other kernels of the step read the
// epoch from here, so no kernel takes the epoch as a launch argument and a step can be replayed
// from a CUDA graph. The timing and row counts are statistics for the caller
// (prism_moe_ep_read_stats).
struct EpStepState {
  uint64_t epoch;               // this step's epoch (flag value; parity = epoch & 1)
  uint64_t counter;             // last epoch issued on this rank
  uint64_t disp_t0, disp_t1;    // %globaltimer ns: first dispatch chunk claimed, last one stored
  uint64_t fused_t0, fused_t1;  // %globaltimer ns: fused expert launch, first CTA in, last out
  uint64_t send_rows;           // token rows this rank pulled from other ranks (dispatch)
  uint64_t recv_rows;           // rows this rank returned to other ranks (down GEMM outputs)
};
constexpr size_t kEpStepOffset = 64;   // inside the workspace's first 256-byte block

// Where a grouped GEMM writes its output rows and how it announces completion. Default: dense
// rows ``out + r * ld``. With ``seg_base``, row r of segment s goes to the address
// seg_base[s] + (r - seg_offsets[s]) * ld * 2 (any GPU's memory reachable by peer access).
// With ``done_counter``, the last CTA to finish fences at system scope and stores the epoch
// (``*epoch_ptr``, or ``epoch`` when that is NULL) to each of the ``num_signal`` flag addresses.
struct GemmOutput {
  const uint64_t* seg_base = nullptr;
  uint64_t* const* signal_flags = nullptr;
  int num_signal = 0;
  uint64_t epoch = 0;
  const uint64_t* epoch_ptr = nullptr;
  unsigned int* done_counter = nullptr;
  EpStepState* step = nullptr;   // launch timing (fused_t0 / fused_t1), or NULL
  bool remote = false;           // rows or flags may live on other GPUs: system-scope fences
};

// Expert-parallel exchange carried out INSIDE the fused expert launch (ep.cu), by four extra
// copy warps per CTA that fill this rank's receive buffer. Its layout: W * El segments, segment
// (j, le), index j * El + le = rows of local expert le from source (me - j) mod W, in the
// source's expert-major order ("slot" j). Two kinds of work, claimed as one sequence of chunks:
//   * slot 0, this rank's own rows (chunks [0, chunk_base[1])): 32 expert-major rows per chunk,
//     copied from ``x``; after each run of one expert the run's length is added to arrival
//     counter le;
//   * slots j >= 1 (chunks [chunk_base[j], chunk_base[j+1])): the rows are PULLED from source s
//     over NVLink, ``32 / k`` tokens per chunk: the warp reads the tokens' expert ids and plan
//     rows from s's landing zone, and reads each token row once however many of this rank's
//     experts it chose, writing one copy per chosen expert (one NVLink row per token and rank:
//     the de-duplicated dispatch). After each chunk its token count is added to arrival counter
//     El + j.
// All arrival counters live in this GPU's memory and are written by this GPU's warps, so both
// the counts and the producer's acquire are GPU-scope. The GEMM's producer waits (bounded) until
// the counter of the segment a tile reads is complete: the segment's rows (slot 0) or the
// source's token count (slots j >= 1). Per-parity fields are indexed by ``*epoch_ptr & 1``.
struct GemmDispatch {
  const void* x = nullptr;              // [T, H] this rank's token rows (slot 0 source)
  int64_t vpr = 0;                      // 16-byte vectors per row
  int k = 1;
  int E = 1;                            // experts in total (W * El)
  const int64_t* ids = nullptr;         // [T*k] this rank's expert id of each flat entry
  const int32_t* row_entry = nullptr;   // [T*k] this rank's expert-major row -> flat entry
  const int32_t* expert_offsets = nullptr;   // [E+1] this rank's expert-major offsets
  const uint64_t* peers = nullptr;      // [W] landing-zone base addresses
  size_t src_x_off = 0;                 // every landing zone: [T_max, H] token rows
  size_t src_ids_off = 0;               //                     [T_max*k] int64 expert ids
  size_t src_row_off = 0;               //                     [T_max*k] int32 expert-major rows
  const int32_t* seg_offsets = nullptr; // [W*El+1] this rank's receive layout
  const int32_t* seg_src_row = nullptr; // [W*El] source-side expert-major row of a segment's row 0
  const int32_t* src_tokens = nullptr;  // [W] tokens of the source in slot j
  const int32_t* chunk_base = nullptr;  // [W+1] first chunk of slot j (chunk_base[W] = total)
  unsigned int* arrive = nullptr;       // [El+W] arrival counters (zeroed by ep_counts_kernel)
  const void* x_recv[2] = {nullptr, nullptr};   // this rank's receive buffers (GEMM A operand)
  const uint64_t* epoch_ptr = nullptr;  // the step's epoch (EpStepState::epoch)
  unsigned int* claim = nullptr;        // [0] next chunk to copy, [1] chunks stored
  EpStepState* step = nullptr;          // dispatch timing and rows pulled, or NULL
  const int* gate_err = nullptr;        // the launch does nothing when this holds ERR_TIMEOUT
  int W = 1, me = 0, El = 1;
};

// route.cu
int route_topk(const void* logits, int dtype, int64_t T, int E, int k, int renorm, int64_t* ids,
               void* w, int32_t* counts, cudaStream_t st);

// dispatch.cu — row_entry (row -> flat entry) is an internal output, NULL when not wanted.
// Entries whose expert id lies outside [0, E) are left out of every output (entry_row = -1)
// and record PRISM_MOE_ERR_ARG in ``err_out`` (NULL: the workspace's first word).
size_t dispatch_workspace_size(int64_t N, int E, int W);
int build_plan(const int64_t* ids, int64_t T, int k, int E, int W, int64_t* perm, int64_t* splits,
               int64_t* sorted_leid, int32_t* counts, int32_t* offsets, int32_t* entry_row,
               int32_t* row_entry, void* ws, size_t ws_bytes, cudaStream_t st,
               int* err_out = nullptr);
int permute_rows(const void* x, int64_t T, int64_t row_bytes, int k, const int32_t* entry_row,
                 void* xs, cudaStream_t st);

// Scratch of the expert GEMMs: h [rows_cap, I] (element size es), then (bf16) the fused
// launch's counters, which it zeroes itself before every launch.
size_t fused_sync_bytes(int64_t rows_cap);
inline size_t expert_scratch_bytes(int64_t rows_cap, int64_t I, int64_t es) {
  const size_t hb = (static_cast<size_t>(es * rows_cap * I) + 255) / 256 * 256;
  return hb + (fused_sync_bytes(rows_cap) + 255) / 256 * 256;
}
inline unsigned int* fused_sync(void* scratch, int64_t rows_cap, int64_t I) {
  return reinterpret_cast<unsigned int*>(static_cast<char*>(scratch) +
                                         (static_cast<size_t>(2 * rows_cap * I) + 255) / 256 * 256);
}

// expert_gemm_sm100.cu — records profiling stage slots 3, 4 (two-launch engines only), 5.
// ``h`` is the scratch above. ``down_out`` (optional) redirects the down GEMM's rows (y may
// then be NULL) and adds a completion signal. ``dispatch`` (optional) runs the expert-parallel
// dispatch inside the fused launch.
int expert_swiglu_bf16(const void* xs, int64_t rows_cap, int64_t H, int64_t I,
                       const int32_t* seg_offsets, const int32_t* seg_expert, int nseg, int El,
                       const void* wgu, const void* wd, void* y, void* h, int* err,
                       cudaStream_t st, const GemmOutput* down_out = nullptr,
                       const GemmDispatch* dispatch = nullptr);

// expert_fused_sm100.cu — both GEMMs in one persistent launch (single 128-row tiles).
int expert_swiglu_fused(const void* xs, int64_t rows_cap, int64_t H, int64_t I,
                        const int32_t* seg_offsets, const int32_t* seg_expert, int nseg, int El,
                        const void* wgu, const void* wd, void* y, void* h, unsigned int* sync,
                        int* err, cudaStream_t st, const GemmOutput* down_out,
                        const GemmDispatch* dispatch);

// expert_gemm_simt.cu
int expert_swiglu_f32(const float* x, int64_t rows_cap, int64_t H, int64_t I,
                      const int32_t* seg_offsets, const int32_t* seg_expert, int nseg, int El,
                      const float* wgu, const float* wd, float* y, float* h, cudaStream_t st);

// combine.cu
// With ``parity`` (EP steps): the rows are read from y + (*parity & 1) * parity_stride_bytes,
// and a launch whose ``gate_err`` word holds PRISM_MOE_ERR_TIMEOUT writes nothing.
// With ``norm_weight``: out = RMSNorm(residual + block output) and residual_out = the sum
// (norm.cuh), the decoder layer's next add_rms_forward fused into the combine.
struct CombineSource {
  const uint64_t* parity = nullptr;
  int64_t parity_stride_bytes = 0;
  const int* gate_err = nullptr;
  const void* residual = nullptr;      // [T, H]
  const void* norm_weight = nullptr;   // [H]
  void* residual_out = nullptr;        // [T, H]
  float eps = 1e-6f;
  int64_t hidden = 0;                  // set by combine()
};
int combine(const void* y, int dtype, const int32_t* entry_row, const void* w, int64_t T, int k,
            int64_t hidden, void* out, cudaStream_t st, const CombineSource* src = nullptr);

// norm.cu — RMSNorm (residual NULL) or residual add + RMSNorm of [T, H] rows.
int rmsnorm(const void* x, const void* residual, const void* weight, float eps, int dtype,
            int64_t T, int64_t hidden, void* out, void* residual_out, cudaStream_t st);

}  // namespace prism
