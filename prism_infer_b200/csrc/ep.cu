// Expert-parallel exchange over NVLink peer memory (one process per GPU, CUDA IPC mappings).
//
// Replaces the reference's NCCL all_to_all_single dispatch / combine and its host round trip
// for split sizes (prism_infer/engine/parallel/expert_parallel.py:113-136, 157-162, 172).
//
// Every rank owns one "landing zone" (cudaMalloc, mapped by all peers through CUDA IPC) with
// identical offsets on every rank:
//   flags   [3 phases][W] u64   phase A counts ready, B rows landed, C outputs landed; slot s is
//                               written (st.release.sys) by source rank s with the step's epoch
//   counts  [2][W][E] i32       per-parity all-gathered expert histograms (row = source rank)
//   recv    [2][W*Tmax*k][H]    rows routed to this rank's experts, expert-major then source
//   back    [2][Tmax*k][H]      this rank's expert outputs, written by the owners' down GEMM
// Parity = epoch & 1. Double-buffering plus the per-step flag waits make reuse safe: a rank
// can only reach step i+2's writes into a peer's parity-(i&1) buffers after that peer has
// finished step i (see the flag chain in the design notes).
//
// Step (prism_moe_ep_forward): route -> plan -> counts all-gather (A) -> return addresses ->
// dispatch rows straight into the owners' recv buffers (B, last-block signal) -> wait B ->
// gate_up GEMM -> down GEMM whose epilogue stores every row into its source rank's back
// buffer and signals C from its last CTA -> wait C -> local weighted combine.
// Every wait is bounded (kPeerWaitNs); a wait that runs out records PRISM_MOE_ERR_TIMEOUT.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace prism {
namespace {

constexpr uint64_t kPeerWaitNs = 10000000000ull;  // 10 s: peers may start a step late
constexpr int kMaxRanks = 64;

struct Landing {
  size_t flags, counts, recv, back, total;
  int64_t rcap;       // rows of one recv parity
  int64_t bcap;       // rows of one back parity
};

Landing landing_layout(int W, int64_t max_tokens, int k, int64_t H, int E, int64_t es) {
  Landing L{};
  size_t o = 0;
  L.flags = o;
  o += 4096;
  L.counts = o;
  o += align_up(sizeof(int32_t) * 2 * W * E, 256);
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
  size_t err, ids, w, plan, plan_bytes, counts, offsets, entry_row, row_entry, seg_offsets,
      dst_base, recv_base, src_off, flag_b, flag_c, done, row_ptr, h, total;
};

EpWs ep_ws_layout(int64_t max_tokens, int64_t H, int64_t I, int E, int k, int W, int64_t rcap,
                  int64_t es) {
  EpWs L{};
  const int El = E / W;
  const int64_t N = max_tokens * k;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align_up(bytes > 0 ? bytes : 1, 256);
    return at;
  };
  L.err = take(256);
  L.ids = take(sizeof(int64_t) * N);
  L.w = take(es * N);
  L.plan_bytes = dispatch_workspace_size(N, E, 1);
  L.plan = take(L.plan_bytes);
  L.counts = take(sizeof(int32_t) * E);
  L.offsets = take(sizeof(int32_t) * (E + 1));
  L.entry_row = take(sizeof(int32_t) * N);
  L.row_entry = take(sizeof(int32_t) * N);
  L.seg_offsets = take(sizeof(int32_t) * (El + 1));
  L.dst_base = take(sizeof(int32_t) * E);
  L.recv_base = take(sizeof(int32_t) * El * W);
  L.src_off = take(sizeof(int32_t) * El * W);
  L.flag_b = take(sizeof(uint64_t) * W);
  L.flag_c = take(sizeof(uint64_t) * W);
  L.done = take(sizeof(unsigned int) * 4);
  L.row_ptr = take(sizeof(uint64_t) * rcap);
  L.h = take(static_cast<size_t>(es * rcap * I));
  L.total = o;
  return L;
}

__device__ __forceinline__ uint64_t* flag_addr(uint64_t base, size_t flags_off, int W, int phase,
                                               int slot) {
  return reinterpret_cast<uint64_t*>(base + flags_off) + phase * W + slot;
}

__device__ bool wait_flags(const uint64_t* local_flags, int W, uint64_t epoch, int* err) {
  const int s = threadIdx.x;
  bool ok = true;
  if (s < W) {
    const uint64_t t0 = global_timer_ns();
    while (load_acquire_sys(local_flags + s) != epoch) {
      if (global_timer_ns() - t0 > kPeerWaitNs) {
        record_device_error(err, PRISM_MOE_ERR_TIMEOUT);
        ok = false;
        break;
      }
    }
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

// Phase A: all-gather the expert histograms, then derive this step's tables.
__global__ void __launch_bounds__(1024)
    ep_counts_kernel(const int32_t* __restrict__ my_counts, const uint64_t* __restrict__ peers,
                     size_t flags_off, size_t counts_off, int W, int me, int E, uint64_t epoch,
                     int32_t* __restrict__ seg_offsets, int32_t* __restrict__ dst_base,
                     int32_t* __restrict__ recv_base, int32_t* __restrict__ src_off,
                     uint64_t* __restrict__ flag_b, uint64_t* __restrict__ flag_c,
                     int* __restrict__ err) {
  __shared__ int32_t tmp[1024];
  __shared__ int32_t total;
  const int El = E / W;
  const int par = static_cast<int>(epoch & 1);
  // 1. my histogram into row `me` of every rank's counts[par]
  for (int i = threadIdx.x; i < W * E; i += blockDim.x) {
    const int d = i / E, e = i % E;
    int32_t* dst = reinterpret_cast<int32_t*>(peers[d] + counts_off) + (par * W + me) * E;
    dst[e] = my_counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < W) store_release_sys(flag_addr(peers[threadIdx.x], flags_off, W, 0, me), epoch);
  // 2. wait for every source's histogram
  const uint64_t* my_flags = flag_addr(peers[me], flags_off, W, 0, 0);
  wait_flags(my_flags, W, epoch, err);
  __syncthreads();
  __threadfence();
  const volatile int32_t* C =
      reinterpret_cast<const volatile int32_t*>(peers[me] + counts_off) + par * W * E;
  // 3. totals per expert, and offsets of each expert inside its owner's receive layout
  const int e = threadIdx.x;
  int32_t tot = 0, before_me = 0;
  if (e < E)
    for (int s = 0; s < W; ++s) {
      const int32_t c = C[s * E + e];
      tot += c;
      if (s < me) before_me += c;
    }
  const int32_t ex = block_excl_scan(tot, E, tmp, &total);
  if (e < E) tmp[e] = ex;
  __syncthreads();
  if (e < E) {
    const int32_t within_owner = ex - tmp[(e / El) * El];   // offset inside owner's layout
    dst_base[e] = within_owner + before_me;
    if (e / El == me) {
      const int le = e - me * El;
      seg_offsets[le] = within_owner;
      int32_t b = within_owner;
      for (int s = 0; s < W; ++s) {
        recv_base[le * W + s] = b;
        b += C[s * E + e];
      }
    }
  }
  __syncthreads();
  if (e == 0) {
    int32_t r = 0;
    for (int le = 0; le < El; ++le)
      for (int s = 0; s < W; ++s) r += C[s * E + me * El + le];
    seg_offsets[El] = r;
  }
  // 4. each source's expert-major row offset of its first row for my expert le
  for (int s = 0; s < W; ++s) {
    const int32_t c = e < E ? C[s * E + e] : 0;
    const int32_t ex_s = block_excl_scan(c, E, tmp, nullptr);
    if (e < E && e / El == me) src_off[s * El + (e - me * El)] = ex_s;
  }
  // 5. where this rank announces B (rows landed) and C (outputs landed) on each peer
  if (threadIdx.x < W) {
    flag_b[threadIdx.x] = reinterpret_cast<uint64_t>(flag_addr(peers[threadIdx.x], flags_off, W, 1, me));
    flag_c[threadIdx.x] = reinterpret_cast<uint64_t>(flag_addr(peers[threadIdx.x], flags_off, W, 2, me));
  }
}

// Return address of every received row: its source rank's back buffer, at the source's
// expert-major row.
__global__ void ep_rowptr_kernel(const int32_t* __restrict__ seg_offsets,
                                 const int32_t* __restrict__ recv_base,
                                 const int32_t* __restrict__ src_off,
                                 const uint64_t* __restrict__ peers, size_t back_off, int W,
                                 int El, int64_t row_bytes, uint64_t* __restrict__ row_ptr) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int32_t R = seg_offsets[El];
  if (r >= R) return;
  int lo = 0, hi = El - 1;
  while (lo < hi) {   // largest le with seg_offsets[le] <= r
    const int mid = (lo + hi + 1) >> 1;
    if (seg_offsets[mid] <= r) lo = mid; else hi = mid - 1;
  }
  const int le = lo;
  int s = 0;
  for (int q = 1; q < W; ++q)
    if (recv_base[le * W + q] <= r) s = q;
  const int64_t src_row = src_off[s * El + le] + (r - recv_base[le * W + s]);
  row_ptr[r] = peers[s] + back_off + static_cast<uint64_t>(src_row * row_bytes);
}

// Dispatch: one warp per expert-major row of this rank, 16-byte stores into the owner's recv
// buffer; the last block to finish publishes phase B on every peer.
__global__ void __launch_bounds__(256)
    ep_dispatch_kernel(const uint4* __restrict__ x, int64_t N, int k, int64_t vpr,
                       const int64_t* __restrict__ ids, const int32_t* __restrict__ row_entry,
                       const int32_t* __restrict__ expert_offsets,
                       const int32_t* __restrict__ dst_base, int El,
                       const uint64_t* __restrict__ peers, size_t recv_off,
                       const uint64_t* __restrict__ flag_b, int W, int me, uint64_t epoch,
                       unsigned int* __restrict__ done) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  // Rows are destination-major; start at the next rank's block so that, at any moment, the
  // ranks write to different peers instead of all to the same one.
  const int64_t shift = N > 0 ? expert_offsets[((me + 1) % W) * El] : 0;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; i < N;
       i += warps) {
    const int64_t q = (i + shift) % N;
    const int32_t f = row_entry[q];
    const int64_t e = ids[f];
    const int64_t t = f / k;
    const int d = static_cast<int>(e / El);
    const int64_t dst_row = dst_base[e] + (q - expert_offsets[e]);
    uint4* dst = reinterpret_cast<uint4*>(peers[d] + recv_off) + dst_row * vpr;
    const uint4* src = x + t * vpr;
    for (int64_t v = lane; v < vpr; v += 32 * 4) {
      uint4 buf[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v + 32 * u < vpr) buf[u] = src[v + 32 * u];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v + 32 * u < vpr) dst[v + 32 * u] = buf[u];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      *done = 0u;
      __threadfence_system();
      for (int d = 0; d < W; ++d)
        store_release_sys(reinterpret_cast<uint64_t*>(flag_b[d]), epoch);
    }
  }
}

__global__ void ep_wait_kernel(const uint64_t* __restrict__ peers, int me, size_t flags_off,
                               int W, int phase, uint64_t epoch, int* __restrict__ err) {
  wait_flags(flag_addr(peers[me], flags_off, W, phase, 0), W, epoch, err);
  __syncthreads();
  __threadfence_system();
}

}  // namespace
}  // namespace prism

using namespace prism;

extern "C" {

__attribute__((visibility("default"))) size_t prism_moe_ep_landing_bytes(
    int32_t ep_size, int64_t max_tokens, int32_t top_k, int64_t hidden, int32_t num_experts,
    int dtype) {
  if (ep_size < 1 || max_tokens < 1 || top_k < 1 || hidden < 1 || num_experts < 1) return 0;
  return landing_layout(ep_size, max_tokens, top_k, hidden, num_experts,
                        dtype == PRISM_MOE_BF16 ? 2 : 4)
      .total;
}

__attribute__((visibility("default"))) int prism_moe_ep_alloc_landing(size_t bytes, void** ptr,
                                                                      void* ipc_handle) {
  PRISM_CHECK_ARG(bytes > 0 && ptr && ipc_handle, "ep_alloc_landing: bad arguments");
  void* p = nullptr;
  PRISM_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, 4096 + 256);   // flags start at epoch 0
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

__attribute__((visibility("default"))) int prism_moe_ep_forward(
    const void* x, const void* router_logits, const int64_t* topk_ids_in,
    const void* topk_weights_in, int dtype, int64_t num_tokens, int64_t max_tokens,
    int64_t hidden, int64_t inter, int32_t num_experts, int32_t top_k, int32_t renorm,
    int32_t ep_size, int32_t ep_rank, const void* w_gate_up, const void* w_down,
    void* my_landing, const uint64_t* peer_landing, uint64_t epoch, void* out, void* workspace,
    size_t workspace_bytes, void* stream) {
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
  PRISM_CHECK_ARG(epoch > 0, "ep_forward: epoch must be >= 1 and increase every step");
  PRISM_CHECK_ARG(my_landing && peer_landing && w_gate_up && w_down &&
                      (num_tokens == 0 || (x && out)),
                  "ep_forward: null pointer");
  PRISM_CHECK_ARG(hidden % 8 == 0 && inter % 8 == 0, "ep_forward: hidden, inter % 8 != 0");
  const int64_t es = 2;
  const int W = ep_size, me = ep_rank, E = num_experts, El = E / W, k = top_k;
  const Landing LL = landing_layout(W, max_tokens, k, hidden, E, es);
  const EpWs L = ep_ws_layout(max_tokens, hidden, inter, E, k, W, LL.rcap, es);
  PRISM_CHECK_ARG(workspace && workspace_bytes >= L.total,
                  "ep_forward: workspace too small (%zu < %zu)", workspace_bytes, L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws + L.err);
  const int par = static_cast<int>(epoch & 1);
  const int64_t T = num_tokens, N = T * k;
  record_stage(0, st);
  const int64_t* ids = topk_ids_in;
  const void* w = topk_weights_in;
  if (router_logits) {
    ids = reinterpret_cast<int64_t*>(ws + L.ids);
    w = ws + L.w;
    int r = route_topk(router_logits, dtype, T, E, k, renorm, const_cast<int64_t*>(ids),
                       const_cast<void*>(w), nullptr, st);
    if (r) return r;
  }
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* entry_row = reinterpret_cast<int32_t*>(ws + L.entry_row);
  int32_t* row_entry = reinterpret_cast<int32_t*>(ws + L.row_entry);
  record_stage(1, st);
  int r = build_plan(ids, T, k, E, 1, nullptr, nullptr, nullptr, counts, offsets, entry_row,
                     row_entry, ws + L.plan, L.plan_bytes, st);
  if (r) return r;
  record_stage(2, st);   // exchange: counts all-gather, dispatch, wait for every source
  int32_t* seg_offsets = reinterpret_cast<int32_t*>(ws + L.seg_offsets);
  int32_t* dst_base = reinterpret_cast<int32_t*>(ws + L.dst_base);
  int32_t* recv_base = reinterpret_cast<int32_t*>(ws + L.recv_base);
  int32_t* src_off = reinterpret_cast<int32_t*>(ws + L.src_off);
  uint64_t* flag_b = reinterpret_cast<uint64_t*>(ws + L.flag_b);
  uint64_t* flag_c = reinterpret_cast<uint64_t*>(ws + L.flag_c);
  unsigned int* done = reinterpret_cast<unsigned int*>(ws + L.done);
  uint64_t* row_ptr = reinterpret_cast<uint64_t*>(ws + L.row_ptr);
  const size_t counts_off = LL.counts;
  const size_t recv_off = LL.recv + static_cast<size_t>(par) * LL.rcap * hidden * es;
  const size_t back_off = LL.back + static_cast<size_t>(par) * LL.bcap * hidden * es;

  ep_counts_kernel<<<1, 1024, 0, st>>>(counts, peer_landing, LL.flags, counts_off, W, me, E,
                                       epoch, seg_offsets, dst_base, recv_base, src_off, flag_b,
                                       flag_c, err);
  PRISM_LAUNCH_CHECK("ep_counts_kernel launch");
  ep_rowptr_kernel<<<static_cast<unsigned>(ceil_div(LL.rcap, 256)), 256, 0, st>>>(
      seg_offsets, recv_base, src_off, peer_landing, back_off, W, El, hidden * es, row_ptr);
  PRISM_LAUNCH_CHECK("ep_rowptr_kernel launch");
  const unsigned dgrid = static_cast<unsigned>(std::max<int64_t>(
      1, std::min<int64_t>(ceil_div(N, 8), static_cast<int64_t>(num_sms()) * 8)));
  ep_dispatch_kernel<<<dgrid, 256, 0, st>>>(
      static_cast<const uint4*>(x), N, k, hidden * es / 16, ids, row_entry, offsets, dst_base,
      El, peer_landing, recv_off, flag_b, W, me, epoch, done);
  PRISM_LAUNCH_CHECK("ep_dispatch_kernel launch");
  ep_wait_kernel<<<1, 64, 0, st>>>(peer_landing, me, LL.flags, W, 1, epoch, err);
  PRISM_LAUNCH_CHECK("ep_wait_kernel launch");
  // expert GEMMs on the rows that landed here: gate_up locally, down with every row stored
  // into its source rank's back buffer and completion signal C from the last CTA
  char* land = static_cast<char*>(my_landing);
  GemmOutput down{};
  down.row_ptr = row_ptr;
  down.signal_flags = reinterpret_cast<uint64_t* const*>(flag_c);
  down.num_signal = W;
  down.epoch = epoch;
  down.done_counter = done + 1;
  r = expert_swiglu_bf16(land + recv_off, LL.rcap, hidden, inter, seg_offsets, nullptr, El, El,
                         w_gate_up, w_down, nullptr, ws + L.h, err, st, &down);
  if (r) return r;
  ep_wait_kernel<<<1, 64, 0, st>>>(peer_landing, me, LL.flags, W, 2, epoch, err);
  PRISM_LAUNCH_CHECK("ep_wait_kernel launch");
  r = combine(land + back_off, dtype, entry_row, w, T, k, hidden, out, st);
  record_stage(6, st);
  return r;
}

}  // extern "C"
