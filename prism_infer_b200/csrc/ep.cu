// Expert-parallel exchange over NVLink peer memory (one process per GPU, CUDA IPC mappings).
//
// Replaces the reference's NCCL all_to_all_single dispatch / combine and its host round trip
// for split sizes (prism_infer/engine/parallel/expert_parallel.py:113-136, 157-162, 172).
//
// Every rank owns one "landing zone" (cudaMalloc, mapped by all peers through CUDA IPC) with
// identical offsets on every rank:
//   flags   [2 phases][W] u64   phase A counts ready, C outputs landed; slot s is written
//                               (st.release) by source rank s with the step's epoch
//   counts  [2][W][E+1] i32     per-parity all-gathered expert histograms (row = source rank;
//                               element E = the source's token count)
//   src_x   [Tmax][H]           this rank's token rows of the step, which the owners pull
//   src_ids [Tmax*k] i64        this rank's expert ids of the step
//   src_row [Tmax*k] i32        this rank's plan: expert-major row of each routed entry
//   recv    [2][W*Tmax*k][H]    rows routed to this rank's experts, written by its own copy
//                               warps, W*El segments ordered by slot (ep_counts_kernel)
//   back    [2][Tmax*k][H]      this rank's expert outputs, written by the owners' down GEMM
// Parity = epoch & 1. The src_* buffers are single: an owner reads them during its expert launch
// of step i, and this rank writes them again only at step i+1, after it has seen every owner's C
// flag of step i (raised after that launch). recv/back double-buffering plus the per-step flag
// waits make their reuse safe: a rank can only reach step i+2's stores into a peer's
// parity-(i&1) back buffer after it has seen that peer's C flag of step i+1.
//
// Step (prism_moe_ep_forward): route (ids into src_ids) -> plan (rows into src_row) -> copy x
// into src_x -> counts all-gather (A) and tables -> one fused expert launch
// (expert_fused_sm100.cu) whose copy warps fill the receive buffer (own rows first, then each
// source's rows pulled over NVLink, one token row per token and rank) while its producer waits
// only for the counter of the segment each gate_up tile reads, and whose down epilogue stores
// every output row into its source rank's back buffer; its last CTA signals C -> wait C -> local
// combine. Every wait is bounded (prism_moe_set_wait_limits; 10 s by default); a wait that runs
// out records PRISM_MOE_ERR_TIMEOUT, and the later kernels of that step then do nothing (their
// tables may describe rows that never arrive).
//
// Epoch. The step's epoch (the flag value; its parity picks the buffers) lives in the workspace
// (EpStepState): ep_counts_kernel sets it — from the caller's ``epoch`` argument, or, when that is
// 0, by incrementing the workspace's counter — and every later kernel of the step reads it there.
// With the device counter no launch argument changes from step to step, so a step can be
// captured once in a CUDA graph and replayed.
//
// Scopes. A system-scope fence costs microseconds (more while host copies run); a GPU-scope one
// about half a microsecond. Only the flag exchange, the owners' first read of the sources' rows
// and the return of outputs use system scope; every arrival counter is this GPU's own.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace prism {
namespace {

constexpr int kMaxRanks = 64;
constexpr int kMaxExperts = 1024;
constexpr size_t kFlagBytes = 4096;   // 2 x 64 x 8 B flags, padded; zero at allocation
constexpr size_t kCountsMaxBytes = sizeof(int32_t) * 2 * kMaxRanks * (kMaxExperts + 1);

struct Landing {
  size_t flags, counts, src_x, src_ids, src_row, recv, back, total;
  int64_t rcap;       // rows of one recv parity
  int64_t bcap;       // rows of one back parity
};

Landing landing_layout(int W, int64_t max_tokens, int k, int64_t H, int E, int64_t es) {
  Landing L{};
  size_t o = 0;
  L.flags = o;
  o += kFlagBytes;
  L.counts = o;
  o += align_up(sizeof(int32_t) * 2 * W * (E + 1), 256);
  L.src_x = o;
  o += align_up(static_cast<size_t>(max_tokens * H * es), 256);
  L.src_ids = o;
  o += align_up(sizeof(int64_t) * max_tokens * k, 256);
  L.src_row = o;
  o += align_up(sizeof(int32_t) * max_tokens * k, 256);
  L.rcap = static_cast<int64_t>(W) * max_tokens * k;
  L.bcap = max_tokens * k;
  L.recv = o;
  o += align_up(static_cast<size_t>(2 * L.rcap * H * es), 256);
  L.back = o;
  o += align_up(static_cast<size_t>(2 * L.bcap * H * es), 256);
  L.total = o;
  return L;
}

struct EpWs {
  size_t err, w, plan, plan_bytes, counts, offsets, row_entry, seg_offsets, seg_expert, seg_base,
      seg_src_row, src_tokens, chunk_base, arrive, flag_c, done, h, total;
};

EpWs ep_ws_layout(int64_t max_tokens, int64_t H, int64_t I, int E, int k, int W, int64_t rcap,
                  int64_t es) {
  EpWs L{};
  const int64_t N = max_tokens * k;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align_up(bytes > 0 ? bytes : 1, 256);
    return at;
  };
  L.err = take(256);                                  // + EpStepState at kEpStepOffset
  L.w = take(es * N);
  L.plan_bytes = dispatch_workspace_size(N, E, 1);
  L.plan = take(L.plan_bytes);
  L.counts = take(sizeof(int32_t) * E);
  L.offsets = take(sizeof(int32_t) * (E + 1));
  L.row_entry = take(sizeof(int32_t) * N);
  L.seg_offsets = take(sizeof(int32_t) * (E + 1));   // W * El receive segments
  L.seg_expert = take(sizeof(int32_t) * E);
  L.seg_base = take(sizeof(uint64_t) * E);
  L.seg_src_row = take(sizeof(int32_t) * E);
  L.src_tokens = take(sizeof(int32_t) * W);
  L.chunk_base = take(sizeof(int32_t) * (W + 1));
  L.arrive = take(sizeof(uint32_t) * (E + W));       // El + W used
  L.flag_c = take(sizeof(uint64_t) * W);
  L.done = take(sizeof(unsigned int) * 4);   // chunk claim, chunks stored, CTAs done
  L.h = take(expert_scratch_bytes(rcap, I, es));
  L.total = o;
  return L;
}

__device__ __forceinline__ uint64_t* flag_addr(uint64_t base, size_t flags_off, int W, int phase,
                                               int slot) {
  return reinterpret_cast<uint64_t*>(base + flags_off) + phase * W + slot;
}

__device__ bool wait_flags(const uint64_t* local_flags, int W, uint64_t epoch, int* err,
                           uint64_t limit_ns) {
  const int s = threadIdx.x;
  bool ok = true;
  if (s < W) {
    const uint64_t t0 = global_timer_ns();
    while (load_relaxed_sys(local_flags + s) != epoch) {
      if (global_timer_ns() - t0 > limit_ns) {
        record_device_error(err, PRISM_MOE_ERR_TIMEOUT);
        ok = false;
        break;
      }
    }
    fence_acq_rel_scoped(W > 1);   // with the relaxed poll above: acquire of the flag stores
  }
  return ok;
}

// Block-wide exclusive scan of n <= 1024 values held one per thread (threadIdx.x < n).
__device__ int32_t block_excl_scan(int32_t v, int n, int32_t* tmp, int32_t* total) {
  const int i = threadIdx.x;
  tmp[i] = i < n ? v : 0;
  __syncthreads();
  for (int off = 1; off < blockDim.x; off <<= 1) {
    const int32_t y = i >= off ? tmp[i - off] : 0;
    __syncthreads();
    tmp[i] += y;
    __syncthreads();
  }
  const int32_t incl = tmp[i];
  if (total && i == blockDim.x - 1) *total = incl;
  __syncthreads();
  return incl - (i < n ? v : 0);
}

// Phase A: all-gather the expert histograms and token counts, then derive this step's tables.
//
// Receive layout on rank d: W * El segments in slot order. Segment (j, le), index j * El + le,
// holds the rows of local expert le of source (d - j) mod W, in the source's expert-major
// order. Slot 0 is d's own rows, copied first; the copy warps then pull slot 1, 2, ... in order,
// so d's GEMM reads the segments that are complete first.
struct CountsArgs {
  const int32_t* my_counts;   // [E] this rank's expert histogram
  int64_t my_tokens;          // this rank's token count
  const uint64_t* peers;      // [W] landing zones
  size_t flags_off, counts_off;
  size_t back_off, back_stride;       // parity-0 returned-rows buffer, bytes per parity
  int64_t row_bytes;
  int W, me, E, k;
  uint64_t host_epoch;        // 0: take the next value of the workspace's counter
  EpStepState* step;
  int32_t* seg_offsets;       // [W*El + 1]
  int32_t* seg_expert;        // [W*El]
  uint64_t* seg_base;         // [W*El] return address of each segment's first row
  int32_t* seg_src_row;       // [W*El] source-side expert-major row of each segment's first row
  int32_t* src_tokens;        // [W] token count of the source in slot j
  int32_t* chunk_base;        // [W+1] first copy chunk of slot j
  unsigned int* arrive;       // [El+W] arrival counters, zeroed here
  uint64_t* flag_c;           // [W]
  unsigned int* claim;        // [0] chunk claim, [1] chunks stored
  int* err;
  uint64_t peer_wait_ns;
};

__global__ void __launch_bounds__(1024) ep_counts_kernel(const CountsArgs a) {
  __shared__ int32_t tmp[1024];
  __shared__ int32_t total;
  __shared__ int32_t R[kMaxRanks * kMaxRanks];   // R[d * W + s]: rows source s sends to d
  __shared__ uint64_t s_epoch;
  const int32_t* __restrict__ my_counts = a.my_counts;
  const uint64_t* __restrict__ peers = a.peers;
  const size_t flags_off = a.flags_off, counts_off = a.counts_off;
  const int W = a.W, me = a.me, E = a.E;
  const int El = E / W;
  const int CE = E + 1;                            // counts row stride
  int* err = a.err;
  // 0. this step's epoch, and the step's statistics reset
  if (threadIdx.x == 0) {
    EpStepState* st = a.step;
    const uint64_t e = a.host_epoch ? a.host_epoch : st->counter + 1;
    st->counter = e;
    st->epoch = e;
    st->disp_t0 = 0;
    st->disp_t1 = 0;
    st->fused_t0 = ~0ull;
    st->fused_t1 = 0;
    st->send_rows = 0;
    s_epoch = e;
  }
  __syncthreads();
  const uint64_t epoch = s_epoch;
  const int par = static_cast<int>(epoch & 1);
  const size_t back_off = a.back_off + static_cast<size_t>(par) * a.back_stride;
  const int64_t row_bytes = a.row_bytes;
  // 1. my histogram and token count into row `me` of every rank's counts[par]
  for (int i = threadIdx.x; i < W * CE; i += blockDim.x) {
    const int d = i / CE, e = i % CE;
    int32_t* dst = reinterpret_cast<int32_t*>(peers[d] + counts_off) + (par * W + me) * CE;
    dst[e] = e < E ? my_counts[e] : static_cast<int32_t>(a.my_tokens);
  }
  threadfence_scoped(W > 1);   // also publishes src_x / src_ids / src_row written before this
  __syncthreads();
  if (threadIdx.x < W)
    store_release_scoped(flag_addr(peers[threadIdx.x], flags_off, W, 0, me), epoch, W > 1);
  // 2. wait for every source's histogram
  const uint64_t* my_flags = flag_addr(peers[me], flags_off, W, 0, 0);
  wait_flags(my_flags, W, epoch, err, a.peer_wait_ns);
  __syncthreads();
  __threadfence();
  const volatile int32_t* C =
      reinterpret_cast<const volatile int32_t*>(peers[me] + counts_off) + par * W * CE;
  const int i = threadIdx.x;
  // 3. my receive segments
  int32_t v = 0;
  if (i < E) {
    const int j = i / El, le = i % El;
    v = C[((me - j + W) % W) * CE + me * El + le];
  }
  const int32_t seg_ex = block_excl_scan(v, E, tmp, &total);
  if (i < E) {
    a.seg_offsets[i] = seg_ex;
    a.seg_expert[i] = i % El;
  }
  if (i == 0) a.seg_offsets[E] = total;
  // 4. rows per (destination, source) pair
  for (int p = i; p < W * W; p += blockDim.x) {
    const int d = p / W, s = p % W;
    int32_t r = 0;
    for (int le = 0; le < El; ++le) r += C[s * CE + d * El + le];
    R[p] = r;
  }
  __syncthreads();
  if (i == 0) {
    uint64_t back = 0;   // rows this rank's down GEMM returns to other ranks
    for (int s = 0; s < W; ++s)
      if (s != me) back += static_cast<uint64_t>(R[me * W + s]);
    a.step->recv_rows = back;
    // copy chunks: slot 0 in 32-row chunks of this rank's own rows, then slot j >= 1 in chunks
    // of 32 / k tokens of its source
    const int tpc = 32 / a.k;
    int32_t cb = 0;
    a.chunk_base[0] = 0;
    cb += (R[me * W + me] + 31) / 32;
    a.chunk_base[1] = cb;
    for (int j = 1; j < W; ++j) {
      cb += (C[((me - j + W) % W) * CE + E] + tpc - 1) / tpc;
      a.chunk_base[j + 1] = cb;
    }
  }
  if (i < W) a.src_tokens[i] = C[((me - i + W) % W) * CE + E];
  // 5. return address of each segment's first row (its source's back buffer, at the source's
  //    expert-major row of its first row for my expert le) and that row itself.
  //    One warp per source rank scans that source's histogram 32 experts at a time.
  {
    const int lane = i & 31;
    for (int s = i >> 5; s < W; s += blockDim.x >> 5) {
      const int j = (me - s + W) % W;
      int32_t carry = 0;
      for (int base = 0; base < (me + 1) * El; base += 32) {
        const int e = base + lane;
        const int32_t c = e < E ? C[s * CE + e] : 0;
        int32_t incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int32_t y = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += y;
        }
        if (e >= me * El && e < (me + 1) * El) {
          const int32_t first = carry + incl - c;
          a.seg_src_row[j * El + (e - me * El)] = first;
          a.seg_base[j * El + (e - me * El)] =
              peers[s] + back_off +
              static_cast<uint64_t>(first) * static_cast<uint64_t>(row_bytes);
        }
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
  }
  // 6. this step's copy counters start at zero; where this rank announces C (outputs landed)
  //    on each peer
  if (i < 2) a.claim[i] = 0u;
  for (int c = i; c < El + W; c += blockDim.x) a.arrive[c] = 0u;
  threadfence_scoped(W > 1);
  if (i < W) a.flag_c[i] = reinterpret_cast<uint64_t>(flag_addr(peers[i], flags_off, W, 1, me));
}

// Wait until every rank's flag of ``phase`` holds this step's epoch. Skipped when the step's
// exchange already failed (the flags would never come).
__global__ void ep_wait_kernel(const uint64_t* __restrict__ peers, int me, size_t flags_off,
                               int W, int phase, const EpStepState* __restrict__ step,
                               int* __restrict__ err, uint64_t limit_ns) {
  __shared__ int s_skip;
  if (threadIdx.x == 0)
    s_skip = *reinterpret_cast<const volatile int*>(err) == PRISM_MOE_ERR_TIMEOUT;
  __syncthreads();
  if (s_skip) return;
  wait_flags(flag_addr(peers[me], flags_off, W, phase, 0), W, step->epoch, err, limit_ns);
  __syncthreads();
  threadfence_scoped(W > 1);
}

}  // namespace
}  // namespace prism

using namespace prism;

extern "C" {

__attribute__((visibility("default"))) size_t prism_moe_ep_landing_bytes(
    int32_t ep_size, int64_t max_tokens, int32_t top_k, int64_t hidden, int32_t num_experts,
    int dtype) {
  if (ep_size < 1 || ep_size > kMaxRanks || max_tokens < 1 || top_k < 1 || hidden < 1 ||
      num_experts < 1 || num_experts > kMaxExperts)
    return 0;
  return landing_layout(ep_size, max_tokens, top_k, hidden, num_experts,
                        dtype == PRISM_MOE_BF16 ? 2 : 4)
      .total;
}

__attribute__((visibility("default"))) int prism_moe_ep_alloc_landing(size_t bytes, void** ptr,
                                                                      void* ipc_handle) {
  PRISM_CHECK_ARG(bytes > 0 && ptr && ipc_handle, "ep_alloc_landing: bad arguments");
  void* p = nullptr;
  PRISM_CUDA(cudaMalloc(&p, bytes));
  // flags at epoch 0 and the all-gathered histograms at 0 (so that a step whose counts exchange
  // timed out never derives tables from uninitialised memory)
  cudaError_t e = cudaMemset(p, 0, std::min(bytes, kFlagBytes + kCountsMaxBytes));
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) {
      std::memcpy(ipc_handle, &h, sizeof(h));
      *ptr = p;
      return PRISM_MOE_OK;
    }
  }
  cudaFree(p);
  return cuda_status(e, "ep_alloc_landing");
}

__attribute__((visibility("default"))) int prism_moe_ep_free_landing(void* ptr) {
  if (ptr) PRISM_CUDA(cudaFree(ptr));
  return PRISM_MOE_OK;
}

__attribute__((visibility("default"))) int prism_moe_ep_ipc_handle_bytes(void) {
  return static_cast<int>(sizeof(cudaIpcMemHandle_t));
}

__attribute__((visibility("default"))) int prism_moe_ep_open_peer(const void* ipc_handle,
                                                                  void** ptr) {
  PRISM_CHECK_ARG(ipc_handle && ptr, "ep_open_peer: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  PRISM_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return PRISM_MOE_OK;
}

__attribute__((visibility("default"))) int prism_moe_ep_close_peer(void* ptr) {
  if (ptr) PRISM_CUDA(cudaIpcCloseMemHandle(ptr));
  return PRISM_MOE_OK;
}

__attribute__((visibility("default"))) size_t prism_moe_ep_workspace_size(
    int64_t max_tokens, int64_t hidden, int64_t inter, int32_t num_experts, int32_t top_k,
    int32_t ep_size, int dtype) {
  if (max_tokens < 1 || hidden < 1 || inter < 1 || top_k < 1 || ep_size < 1 ||
      num_experts % ep_size != 0)
    return 0;
  const int64_t es = dtype == PRISM_MOE_BF16 ? 2 : 4;
  const Landing L = landing_layout(ep_size, max_tokens, top_k, hidden, num_experts, es);
  return ep_ws_layout(max_tokens, hidden, inter, num_experts, top_k, ep_size, L.rcap, es).total;
}

__attribute__((visibility("default"))) int prism_moe_ep_forward_norm(
    const void* x, const void* router_logits, const int64_t* topk_ids_in,
    const void* topk_weights_in, int dtype, int64_t num_tokens, int64_t max_tokens,
    int64_t hidden, int64_t inter, int32_t num_experts, int32_t top_k, int32_t renorm,
    int32_t ep_size, int32_t ep_rank, const void* w_gate_up, const void* w_down,
    void* my_landing, const uint64_t* peer_landing, uint64_t epoch, void* out, void* workspace,
    size_t workspace_bytes, void* stream, const prism_moe_norm_epilogue* epilogue) {
  PRISM_CHECK_ARG(dtype == PRISM_MOE_BF16, "ep_forward: bf16 only");
  PRISM_CHECK_ARG(ep_size >= 1 && ep_size <= kMaxRanks && ep_rank >= 0 && ep_rank < ep_size,
                  "ep_forward: bad ep_size/ep_rank");
  PRISM_CHECK_ARG(num_experts % ep_size == 0, "num_experts must be divisible by ep_size");
  PRISM_CHECK_ARG(num_experts <= 1024 && top_k >= 1 && top_k <= 32 && top_k <= num_experts,
                  "ep_forward: bad num_experts/top_k");
  PRISM_CHECK_ARG(num_tokens >= 0 && num_tokens <= max_tokens,
                  "ep_forward: num_tokens %lld exceeds the landing capacity %lld",
                  static_cast<long long>(num_tokens), static_cast<long long>(max_tokens));
  PRISM_CHECK_ARG(num_tokens == 0 || router_logits || (topk_ids_in && topk_weights_in),
                  "ep_forward: needs router_logits or topk ids and weights");
  PRISM_CHECK_ARG(my_landing && peer_landing && w_gate_up && w_down &&
                      (num_tokens == 0 || (x && out)),
                  "ep_forward: null pointer");
  PRISM_CHECK_ARG(hidden % 8 == 0 && inter % 8 == 0, "ep_forward: hidden, inter % 8 != 0");
  PRISM_CHECK_ARG(!epilogue || (epilogue->residual && epilogue->norm_weight &&
                                epilogue->residual_out && epilogue->eps >= 0.f),
                  "ep_forward: incomplete norm epilogue");
  const int64_t es = 2;
  const int W = ep_size, me = ep_rank, E = num_experts, El = E / W, k = top_k;
  const Landing LL = landing_layout(W, max_tokens, k, hidden, E, es);
  const EpWs L = ep_ws_layout(max_tokens, hidden, inter, E, k, W, LL.rcap, es);
  PRISM_CHECK_ARG(workspace && workspace_bytes >= L.total,
                  "ep_forward: workspace too small (%zu < %zu)", workspace_bytes, L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  char* land = static_cast<char*>(my_landing);
  int* err = reinterpret_cast<int*>(ws + L.err);
  EpStepState* step = reinterpret_cast<EpStepState*>(ws + kEpStepOffset);
  const int64_t T = num_tokens;
  // this step's ids and plan go straight into the landing zone, where the owners read them
  int64_t* ids = reinterpret_cast<int64_t*>(land + LL.src_ids);
  int32_t* entry_row = reinterpret_cast<int32_t*>(land + LL.src_row);
  record_stage(0, st);
  const void* w = topk_weights_in;
  if (router_logits) {
    w = ws + L.w;
    int r = route_topk(router_logits, dtype, T, E, k, renorm, ids, const_cast<void*>(w), nullptr,
                       st);
    if (r) return r;
  } else if (T > 0) {
    PRISM_CUDA(cudaMemcpyAsync(ids, topk_ids_in, sizeof(int64_t) * T * k,
                               cudaMemcpyDeviceToDevice, st));
  }
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* row_entry = reinterpret_cast<int32_t*>(ws + L.row_entry);
  record_stage(1, st);
  // ids outside [0, E) (caller-given) are left out of the plan and recorded as ERR_ARG in the
  // step's error word; no row is copied for them and their slots add nothing to the output
  int r = build_plan(ids, T, k, E, 1, nullptr, nullptr, nullptr, counts, offsets, entry_row,
                     row_entry, ws + L.plan, L.plan_bytes, st, err);
  if (r) return r;
  if (T > 0)   // this step's token rows, where the owners pull them from
    PRISM_CUDA(cudaMemcpyAsync(land + LL.src_x, x, static_cast<size_t>(T * hidden * es),
                               cudaMemcpyDeviceToDevice, st));
  record_stage(2, st);   // counts all-gather and the step's tables
  int32_t* seg_offsets = reinterpret_cast<int32_t*>(ws + L.seg_offsets);
  int32_t* seg_expert = reinterpret_cast<int32_t*>(ws + L.seg_expert);
  uint64_t* seg_base = reinterpret_cast<uint64_t*>(ws + L.seg_base);
  uint64_t* flag_c = reinterpret_cast<uint64_t*>(ws + L.flag_c);
  unsigned int* done = reinterpret_cast<unsigned int*>(ws + L.done);
  const size_t recv_stride = static_cast<size_t>(LL.rcap) * hidden * es;
  const size_t back_stride = static_cast<size_t>(LL.bcap) * hidden * es;

  CountsArgs ca{};
  ca.my_counts = counts;
  ca.my_tokens = T;
  ca.peers = peer_landing;
  ca.flags_off = LL.flags;
  ca.counts_off = LL.counts;
  ca.back_off = LL.back;
  ca.back_stride = back_stride;
  ca.row_bytes = hidden * es;
  ca.W = W;
  ca.me = me;
  ca.E = E;
  ca.k = k;
  ca.host_epoch = epoch;
  ca.step = step;
  ca.seg_offsets = seg_offsets;
  ca.seg_expert = seg_expert;
  ca.seg_base = seg_base;
  ca.seg_src_row = reinterpret_cast<int32_t*>(ws + L.seg_src_row);
  ca.src_tokens = reinterpret_cast<int32_t*>(ws + L.src_tokens);
  ca.chunk_base = reinterpret_cast<int32_t*>(ws + L.chunk_base);
  ca.arrive = reinterpret_cast<unsigned int*>(ws + L.arrive);
  ca.flag_c = flag_c;
  ca.claim = done;
  ca.err = err;
  ca.peer_wait_ns = peer_wait_limit_ns();
  ep_counts_kernel<<<1, 1024, 0, st>>>(ca);
  PRISM_LAUNCH_CHECK("ep_counts_kernel launch");
  // One launch per GPU for the rest of the exchange and the experts: its copy warps fill the
  // receive buffer (own rows, then every source's rows pulled over NVLink) while its producer
  // waits only for the counter of the segment the next gate_up tile reads; the down epilogue
  // stores every output row into its source rank's back buffer, and the last CTA signals C.
  GemmDispatch disp{};
  disp.x = x;
  disp.vpr = hidden * es / 16;
  disp.k = k;
  disp.E = E;
  disp.ids = ids;
  disp.row_entry = row_entry;
  disp.expert_offsets = offsets;
  disp.peers = peer_landing;
  disp.src_x_off = LL.src_x;
  disp.src_ids_off = LL.src_ids;
  disp.src_row_off = LL.src_row;
  disp.seg_offsets = seg_offsets;
  disp.seg_src_row = ca.seg_src_row;
  disp.src_tokens = ca.src_tokens;
  disp.chunk_base = ca.chunk_base;
  disp.arrive = ca.arrive;
  for (int p = 0; p < 2; ++p) disp.x_recv[p] = land + LL.recv + p * recv_stride;
  disp.epoch_ptr = &step->epoch;
  disp.claim = done;
  disp.step = step;
  disp.gate_err = err;
  disp.W = W;
  disp.me = me;
  disp.El = El;
  GemmOutput down{};
  down.seg_base = seg_base;
  down.signal_flags = reinterpret_cast<uint64_t* const*>(flag_c);
  down.num_signal = W;
  down.epoch_ptr = &step->epoch;
  down.done_counter = done + 2;
  down.step = step;
  down.remote = W > 1;
  r = expert_swiglu_bf16(land + LL.recv, LL.rcap, hidden, inter, seg_offsets, seg_expert, E, El,
                         w_gate_up, w_down, nullptr, ws + L.h, err, st, &down, &disp);
  if (r) return r;
  ep_wait_kernel<<<1, 64, 0, st>>>(peer_landing, me, LL.flags, W, 1, step, err,
                                   peer_wait_limit_ns());
  PRISM_LAUNCH_CHECK("ep_wait_kernel launch");
  CombineSource src{};
  src.parity = &step->epoch;
  src.parity_stride_bytes = static_cast<int64_t>(back_stride);
  src.gate_err = err;
  if (epilogue) {
    src.residual = epilogue->residual;
    src.norm_weight = epilogue->norm_weight;
    src.residual_out = epilogue->residual_out;
    src.eps = epilogue->eps;
  }
  r = combine(land + LL.back, dtype, entry_row, w, T, k, hidden, out, st, &src);
  record_stage(6, st);
  return r;
}

__attribute__((visibility("default"))) int prism_moe_ep_forward(
    const void* x, const void* router_logits, const int64_t* topk_ids_in,
    const void* topk_weights_in, int dtype, int64_t num_tokens, int64_t max_tokens,
    int64_t hidden, int64_t inter, int32_t num_experts, int32_t top_k, int32_t renorm,
    int32_t ep_size, int32_t ep_rank, const void* w_gate_up, const void* w_down,
    void* my_landing, const uint64_t* peer_landing, uint64_t epoch, void* out, void* workspace,
    size_t workspace_bytes, void* stream) {
  return prism_moe_ep_forward_norm(x, router_logits, topk_ids_in, topk_weights_in, dtype,
                                   num_tokens, max_tokens, hidden, inter, num_experts, top_k,
                                   renorm, ep_size, ep_rank, w_gate_up, w_down, my_landing,
                                   peer_landing, epoch, out, workspace, workspace_bytes, stream,
                                   nullptr);
}

__attribute__((visibility("default"))) int prism_moe_ep_read_stats(const void* workspace,
                                                                   uint64_t* stats,
                                                                   void* stream) {
  PRISM_CHECK_ARG(workspace && stats, "ep_read_stats: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  PRISM_CUDA(cudaMemcpyAsync(stats, static_cast<const char*>(workspace) + kEpStepOffset,
                             sizeof(EpStepState), cudaMemcpyDeviceToHost, st));
  PRISM_CUDA(cudaStreamSynchronize(st));
  return PRISM_MOE_OK;
}

}  // extern "C"
