// Dispatch plan with its scratch in a fixed device array — for callers that cannot allocate.
//
// prism_moe_build_dispatch_plan takes a caller-allocated workspace. Some callers have no way to
// provide one: a plugin invoked from a host framework's execute/enqueue callback that only
// hands over the buffers it owns, or an embedded runtime whose memory is entirely owned by its
// own pool, where calling cudaMalloc would bypass that accounting or stall on a device-wide
// synchronisation. This variant keeps the plan's scratch in a file-scope __device__ array of
// fixed size, so the call allocates nothing.
//
// Limits (checked; larger problems get PRISM_MOE_ERR_ARG): num_tokens * top_k <= 65536
// routed entries, num_experts <= 256, ep_size <= 64. The array (1 MiB) is part of the module
// image: every GPU that loads the library holds it until the process exits.
//
// Set-up: the first call on a device looks up the array's device address with
// cudaGetSymbolAddress, with that device current, and caches it; make that first call before
// any stream capture begins. All calls on a device share the one array and it keeps the last
// call's contents; the plan's error word (its first bytes) is cleared at the start of every call
// and every other byte a call reads is written by that call first. Calls whose kernels overlap on
// the GPU (different streams, or different host threads) race on the array: serialise them.
//
// Expert ids must lie in [0, num_experts). Entries outside it are left out of the outputs, as in
// prism_moe_build_dispatch_plan; the kernel records that in the array's error word, which this
// entry point does not read back, so the caller is not told.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace prism {
namespace {

constexpr int64_t kStaticMaxEntries = 65536;
constexpr int kStaticMaxExperts = 256;
constexpr int kStaticMaxEpSize = 64;
constexpr size_t kStaticScratchBytes = 1024 * 1024;
constexpr int kMaxDevices = 64;

// Host code must not use this name as an address: on the host it is only a stand-in symbol.
static __device__ __align__(256) unsigned char g_plan_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("build_dispatch_plan_static: device ordinal %d outside [0, %d)", dev, kMaxDevices);
    return PRISM_MOE_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_plan_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_plan_scratch)");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return PRISM_MOE_OK;
}

}  // namespace
}  // namespace prism

using namespace prism;

extern "C" __attribute__((visibility("default"))) int prism_moe_build_dispatch_plan_static(
    const int64_t* topk_ids, int64_t num_tokens, int32_t top_k, int32_t num_experts,
    int32_t ep_size, int64_t* perm, int64_t* input_splits, int64_t* sorted_local_eid,
    int32_t* expert_counts, int32_t* expert_offsets, int32_t* entry_row, void* stream) {
  PRISM_CHECK_ARG(num_tokens >= 0 && top_k >= 1 && top_k <= 32,
                  "build_dispatch_plan_static: bad shape");
  PRISM_CHECK_ARG(num_tokens * top_k <= kStaticMaxEntries,
                  "build_dispatch_plan_static: %lld routed entries exceed the static limit of "
                  "%lld (use prism_moe_build_dispatch_plan with a workspace)",
                  static_cast<long long>(num_tokens * top_k),
                  static_cast<long long>(kStaticMaxEntries));
  PRISM_CHECK_ARG(num_experts >= 1 && num_experts <= kStaticMaxExperts,
                  "build_dispatch_plan_static: num_experts %d outside [1, %d]", num_experts,
                  kStaticMaxExperts);
  PRISM_CHECK_ARG(ep_size >= 1 && ep_size <= kStaticMaxEpSize && num_experts % ep_size == 0,
                  "build_dispatch_plan_static: ep_size %d must divide num_experts and be <= %d",
                  ep_size, kStaticMaxEpSize);
  PRISM_CHECK_ARG(num_tokens == 0 || topk_ids, "build_dispatch_plan_static: null topk_ids");
  const size_t need = dispatch_workspace_size(num_tokens * top_k, num_experts, ep_size);
  PRISM_CHECK_ARG(need <= kStaticScratchBytes,
                  "build_dispatch_plan_static: needs %zu scratch bytes, static array holds %zu",
                  need, kStaticScratchBytes);
  void* scratch = nullptr;
  if (int r = scratch_for_current_device(&scratch)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the plan's error word (first bytes of its scratch) must start at zero on every call
  PRISM_CUDA(cudaMemsetAsync(scratch, 0, 256, st));
  return build_plan(topk_ids, num_tokens, top_k, num_experts, ep_size, perm, input_splits,
                    sorted_local_eid, expert_counts, expert_offsets, entry_row, nullptr, scratch,
                    kStaticScratchBytes, st);
}
