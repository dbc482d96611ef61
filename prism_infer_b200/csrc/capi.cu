// extern "C" entry points of libprism_moe.so (declared in include/prism_moe.h).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "internal.h"

namespace prism {

namespace {
thread_local char g_err[512] = "";
thread_local cudaEvent_t g_stage_events[kNumStageEvents] = {};
thread_local int g_num_stage_events = 0;
}

void record_stage(int slot, cudaStream_t st) {
  if (slot < g_num_stage_events && g_stage_events[slot]) cudaEventRecord(g_stage_events[slot], st);
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return PRISM_MOE_ERR_CUDA;
}

namespace {
std::atomic<int> g_engine{PRISM_MOE_ENGINE_AUTO};
std::atomic<uint64_t> g_wait_ns{2000000000ull};        // 2 s: far above any legitimate wait
std::atomic<uint64_t> g_peer_wait_ns{10000000000ull};  // 10 s: peers may start a step late
std::mutex g_attr_mu;
std::set<std::pair<const void*, int>> g_attr_done;
}  // namespace

int expert_engine_setting() { return g_engine.load(std::memory_order_relaxed); }
uint64_t wait_limit_ns() { return g_wait_ns.load(std::memory_order_relaxed); }
uint64_t peer_wait_limit_ns() { return g_peer_wait_ns.load(std::memory_order_relaxed); }

int ensure_smem_attr(const void* func, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_attr_mu);
  if (g_attr_done.count({func, dev})) return PRISM_MOE_OK;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  g_attr_done.insert({func, dev});
  return PRISM_MOE_OK;
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 1;
  return n > 0 ? n : 1;
}

namespace {

int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    set_error("libprism_moe targets sm_100a (B200); device %d is sm_%d%d", dev, major, minor);
    return PRISM_MOE_ERR_UNSUPPORTED;
  }
  return PRISM_MOE_OK;
}

bool dtype_ok(int dtype) { return dtype == PRISM_MOE_F32 || dtype == PRISM_MOE_BF16; }
int64_t elem_size(int dtype) { return dtype == PRISM_MOE_BF16 ? 2 : 4; }

struct BlockLayout {
  size_t err, ids, w, plan, counts, offsets, entry_row, xs, h, y, total, plan_bytes;
};

BlockLayout block_layout(int64_t T, int64_t H, int64_t I, int E, int k, int dtype) {
  BlockLayout L{};
  const int64_t N = T * k;
  const size_t es = static_cast<size_t>(elem_size(dtype));
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
  L.xs = take(es * N * H);
  L.h = take(expert_scratch_bytes(N, I, static_cast<int64_t>(es)));
  L.y = take(es * N * H);
  L.total = o;
  return L;
}

}  // namespace
}  // namespace prism

using namespace prism;

extern "C" {

int prism_moe_version(void) { return 100; }

const char* prism_moe_last_error(void) { return g_err; }

int prism_moe_route_topk(const void* logits, int dtype, int64_t num_tokens, int32_t num_experts,
                         int32_t top_k, int32_t renorm, int64_t* topk_ids, void* topk_weights,
                         int32_t* expert_counts, void* stream) {
  PRISM_CHECK_ARG(dtype_ok(dtype), "route_topk: unknown dtype %d", dtype);
  PRISM_CHECK_ARG(num_tokens >= 0, "route_topk: negative num_tokens");
  PRISM_CHECK_ARG(num_experts >= 1 && num_experts <= 1024, "route_topk: num_experts %d outside [1, 1024]",
                  num_experts);
  PRISM_CHECK_ARG(top_k >= 1 && top_k <= 32 && top_k <= num_experts,
                  "route_topk: top_k %d outside [1, min(num_experts, 32)]", top_k);
  PRISM_CHECK_ARG(num_tokens == 0 || (logits && topk_ids && topk_weights),
                  "route_topk: null pointer");
  if (int r = check_device()) return r;
  return route_topk(logits, dtype, num_tokens, num_experts, top_k, renorm, topk_ids, topk_weights,
                    expert_counts, static_cast<cudaStream_t>(stream));
}

size_t prism_moe_dispatch_workspace_size(int64_t num_tokens, int32_t top_k, int32_t num_experts,
                                         int32_t ep_size) {
  if (num_tokens < 0 || top_k < 1 || num_experts < 1 || ep_size < 1) return 0;
  return dispatch_workspace_size(num_tokens * top_k, num_experts, ep_size);
}

int prism_moe_build_dispatch_plan(const int64_t* topk_ids, int64_t num_tokens, int32_t top_k,
                                  int32_t num_experts, int32_t ep_size, int64_t* perm,
                                  int64_t* input_splits, int64_t* sorted_local_eid,
                                  int32_t* expert_counts, int32_t* expert_offsets,
                                  int32_t* entry_row, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  PRISM_CHECK_ARG(num_tokens >= 0 && top_k >= 1 && top_k <= 32, "build_dispatch_plan: bad shape");
  PRISM_CHECK_ARG(ep_size >= 1 && num_experts >= 1 && num_experts % ep_size == 0,
                  "num_experts must be divisible by ep_size");
  PRISM_CHECK_ARG(num_tokens == 0 || (topk_ids && workspace), "build_dispatch_plan: null pointer");
  if (int r = check_device()) return r;
  return build_plan(topk_ids, num_tokens, top_k, num_experts, ep_size, perm, input_splits,
                    sorted_local_eid, expert_counts, expert_offsets, entry_row, nullptr,
                    workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int prism_moe_permute_rows(const void* x, int dtype, int64_t num_tokens, int64_t hidden,
                           int32_t top_k, const int32_t* entry_row, void* x_sorted, void* stream) {
  PRISM_CHECK_ARG(dtype_ok(dtype), "permute_rows: unknown dtype %d", dtype);
  PRISM_CHECK_ARG(num_tokens >= 0 && hidden >= 1, "permute_rows: bad shape");
  PRISM_CHECK_ARG(num_tokens == 0 || (x && entry_row && x_sorted), "permute_rows: null pointer");
  PRISM_CHECK_ARG((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(x_sorted)) % 16 == 0,
                  "permute_rows: buffers must be 16-byte aligned");
  if (int r = check_device()) return r;
  return permute_rows(x, num_tokens, hidden * elem_size(dtype), top_k, entry_row, x_sorted,
                      static_cast<cudaStream_t>(stream));
}

size_t prism_moe_expert_workspace_size(int64_t rows_capacity, int64_t hidden, int64_t inter,
                                       int dtype) {
  (void)hidden;
  if (rows_capacity < 0 || inter < 1 || !dtype_ok(dtype)) return 0;
  return expert_scratch_bytes(rows_capacity, inter, elem_size(dtype));
}

int prism_moe_expert_swiglu(const void* x_sorted, int dtype, int64_t rows_capacity,
                            int64_t hidden, int64_t inter, const int32_t* seg_offsets,
                            const int32_t* seg_expert, int32_t num_segments,
                            int32_t num_local_experts, const void* w_gate_up, const void* w_down,
                            void* y, void* workspace, size_t workspace_bytes, int* device_error,
                            void* stream) {
  PRISM_CHECK_ARG(dtype_ok(dtype), "expert_swiglu: unknown dtype %d", dtype);
  PRISM_CHECK_ARG(rows_capacity >= 0 && hidden >= 1 && inter >= 1, "expert_swiglu: bad shape");
  PRISM_CHECK_ARG(num_segments >= 1 && num_local_experts >= 1, "expert_swiglu: no segments");
  PRISM_CHECK_ARG(workspace_bytes >= prism_moe_expert_workspace_size(rows_capacity, hidden, inter, dtype),
                  "expert_swiglu: workspace too small");
  PRISM_CHECK_ARG(rows_capacity == 0 || (x_sorted && seg_offsets && w_gate_up && w_down && y && workspace),
                  "expert_swiglu: null pointer");
  if (int r = check_device()) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows_capacity == 0) return PRISM_MOE_OK;
  if (dtype == PRISM_MOE_BF16)
    return expert_swiglu_bf16(x_sorted, rows_capacity, hidden, inter, seg_offsets, seg_expert,
                              num_segments, num_local_experts, w_gate_up, w_down, y, workspace,
                              device_error, st);
  return expert_swiglu_f32(static_cast<const float*>(x_sorted), rows_capacity, hidden, inter,
                           seg_offsets, seg_expert, num_segments, num_local_experts,
                           static_cast<const float*>(w_gate_up), static_cast<const float*>(w_down),
                           static_cast<float*>(y), static_cast<float*>(workspace), st);
}

int prism_moe_combine(const void* expert_out, int dtype, const int32_t* entry_row,
                      const void* topk_weights, int64_t num_tokens, int32_t top_k, int64_t hidden,
                      void* out, void* stream) {
  PRISM_CHECK_ARG(dtype_ok(dtype), "combine: unknown dtype %d", dtype);
  PRISM_CHECK_ARG(num_tokens >= 0 && hidden >= 1, "combine: bad shape");
  PRISM_CHECK_ARG(num_tokens == 0 || (expert_out && topk_weights && out), "combine: null pointer");
  PRISM_CHECK_ARG((reinterpret_cast<uintptr_t>(expert_out) | reinterpret_cast<uintptr_t>(out)) % 16 == 0,
                  "combine: buffers must be 16-byte aligned");
  if (int r = check_device()) return r;
  return combine(expert_out, dtype, entry_row, topk_weights, num_tokens, top_k, hidden, out,
                 static_cast<cudaStream_t>(stream));
}

size_t prism_moe_block_workspace_size(int64_t num_tokens, int64_t hidden, int64_t inter,
                                      int32_t num_experts, int32_t top_k, int dtype) {
  if (num_tokens < 0 || hidden < 1 || inter < 1 || num_experts < 1 || top_k < 1 || !dtype_ok(dtype))
    return 0;
  return block_layout(num_tokens, hidden, inter, num_experts, top_k, dtype).total;
}

int prism_moe_block_forward_norm(const void* x, const void* router_logits, int dtype,
                                 int64_t num_tokens, int64_t hidden, int64_t inter,
                                 int32_t num_experts, int32_t top_k, int32_t renorm,
                                 const void* w_gate_up, const void* w_down, void* out,
                                 int64_t* topk_ids, void* topk_weights, void* workspace,
                                 size_t workspace_bytes, void* stream,
                                 const prism_moe_norm_epilogue* epilogue) {
  PRISM_CHECK_ARG(dtype_ok(dtype), "block_forward: unknown dtype %d", dtype);
  PRISM_CHECK_ARG(num_tokens >= 0 && hidden >= 1 && inter >= 1, "block_forward: bad shape");
  PRISM_CHECK_ARG(num_experts >= 1 && num_experts <= 1024, "block_forward: num_experts %d outside [1, 1024]",
                  num_experts);
  PRISM_CHECK_ARG(top_k >= 1 && top_k <= 32 && top_k <= num_experts,
                  "block_forward: top_k %d outside [1, min(num_experts, 32)]", top_k);
  const BlockLayout L = block_layout(num_tokens, hidden, inter, num_experts, top_k, dtype);
  PRISM_CHECK_ARG(workspace && workspace_bytes >= L.total,
                  "block_forward: workspace too small (%zu < %zu)", workspace_bytes, L.total);
  PRISM_CHECK_ARG(num_tokens == 0 || (x && router_logits && w_gate_up && w_down && out),
                  "block_forward: null pointer");
  PRISM_CHECK_ARG(!epilogue || (epilogue->residual && epilogue->norm_weight &&
                                epilogue->residual_out && epilogue->eps >= 0.f),
                  "block_forward: incomplete norm epilogue");
  if (int r = check_device()) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (num_tokens == 0) return PRISM_MOE_OK;
  char* ws = static_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws + L.err);
  int64_t* ids = topk_ids ? topk_ids : reinterpret_cast<int64_t*>(ws + L.ids);
  void* w = topk_weights ? topk_weights : static_cast<void*>(ws + L.w);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* entry_row = reinterpret_cast<int32_t*>(ws + L.entry_row);
  void* xs = ws + L.xs;
  void* h = ws + L.h;
  void* y = ws + L.y;
  const int64_t N = num_tokens * top_k;
  record_stage(0, st);
  int r = route_topk(router_logits, dtype, num_tokens, num_experts, top_k, renorm, ids, w, nullptr, st);
  if (r) return r;
  record_stage(1, st);
  r = build_plan(ids, num_tokens, top_k, num_experts, 1, nullptr, nullptr, nullptr, counts, offsets,
                 entry_row, nullptr, ws + L.plan, L.plan_bytes, st, err);
  if (r) return r;
  record_stage(2, st);
  r = permute_rows(x, num_tokens, hidden * elem_size(dtype), top_k, entry_row, xs, st);
  if (r) return r;
  if (dtype == PRISM_MOE_BF16)
    r = expert_swiglu_bf16(xs, N, hidden, inter, offsets, nullptr, num_experts, num_experts,
                           w_gate_up, w_down, y, h, err, st);
  else
    r = expert_swiglu_f32(static_cast<const float*>(xs), N, hidden, inter, offsets, nullptr,
                          num_experts, num_experts, static_cast<const float*>(w_gate_up),
                          static_cast<const float*>(w_down), static_cast<float*>(y),
                          static_cast<float*>(h), st);
  if (r) return r;
  CombineSource src{};
  if (epilogue) {
    src.residual = epilogue->residual;
    src.norm_weight = epilogue->norm_weight;
    src.residual_out = epilogue->residual_out;
    src.eps = epilogue->eps;
  }
  r = combine(y, dtype, entry_row, w, num_tokens, top_k, hidden, out, st, &src);
  record_stage(6, st);
  return r;
}

int prism_moe_block_forward(const void* x, const void* router_logits, int dtype,
                            int64_t num_tokens, int64_t hidden, int64_t inter,
                            int32_t num_experts, int32_t top_k, int32_t renorm,
                            const void* w_gate_up, const void* w_down, void* out,
                            int64_t* topk_ids, void* topk_weights, void* workspace,
                            size_t workspace_bytes, void* stream) {
  return prism_moe_block_forward_norm(x, router_logits, dtype, num_tokens, hidden, inter,
                                      num_experts, top_k, renorm, w_gate_up, w_down, out,
                                      topk_ids, topk_weights, workspace, workspace_bytes, stream,
                                      nullptr);
}

int prism_moe_rmsnorm(const void* x, const void* residual, const void* weight, float eps,
                      int dtype, int64_t num_tokens, int64_t hidden, void* out,
                      void* residual_out, void* stream) {
  PRISM_CHECK_ARG(dtype_ok(dtype), "rmsnorm: unknown dtype %d", dtype);
  PRISM_CHECK_ARG(num_tokens >= 0 && hidden >= 1, "rmsnorm: bad shape");
  PRISM_CHECK_ARG(eps >= 0.f, "rmsnorm: negative eps");
  PRISM_CHECK_ARG(num_tokens == 0 || (x && weight && out), "rmsnorm: null pointer");
  PRISM_CHECK_ARG((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(residual) |
                   reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(out) |
                   reinterpret_cast<uintptr_t>(residual_out)) % 16 == 0,
                  "rmsnorm: buffers must be 16-byte aligned");
  if (int r = check_device()) return r;
  return rmsnorm(x, residual, weight, eps, dtype, num_tokens, hidden, out, residual_out,
                 static_cast<cudaStream_t>(stream));
}

int prism_moe_profile_events(void* const* events, int32_t count) {
  PRISM_CHECK_ARG(count >= 0 && count <= kNumStageEvents, "profile_events: count %d outside [0, %d]",
                  count, kNumStageEvents);
  PRISM_CHECK_ARG(count == 0 || events != nullptr, "profile_events: null events");
  for (int i = 0; i < kNumStageEvents; ++i)
    g_stage_events[i] = i < count ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  g_num_stage_events = count;
  return PRISM_MOE_OK;
}

int prism_moe_set_expert_engine(int engine) {
  PRISM_CHECK_ARG(engine >= PRISM_MOE_ENGINE_AUTO && engine <= PRISM_MOE_ENGINE_PAIR,
                  "set_expert_engine: unknown engine %d", engine);
  g_engine.store(engine, std::memory_order_relaxed);
  return PRISM_MOE_OK;
}

int prism_moe_set_wait_limits(int64_t wait_ns, int64_t peer_wait_ns) {
  PRISM_CHECK_ARG(wait_ns >= 0 && peer_wait_ns >= 0, "set_wait_limits: negative limit");
  PRISM_CHECK_ARG(wait_ns <= 60000000000ll && peer_wait_ns <= 60000000000ll,
                  "set_wait_limits: limits above 60 s are not accepted");
  g_wait_ns.store(wait_ns > 0 ? static_cast<uint64_t>(wait_ns) : 2000000000ull,
                  std::memory_order_relaxed);
  g_peer_wait_ns.store(peer_wait_ns > 0 ? static_cast<uint64_t>(peer_wait_ns) : 10000000000ull,
                       std::memory_order_relaxed);
  return PRISM_MOE_OK;
}

int prism_moe_read_device_error(int* device_error, void* stream) {
  PRISM_CHECK_ARG(device_error != nullptr, "read_device_error: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  PRISM_CUDA(cudaMemcpyAsync(&v, device_error, sizeof(int), cudaMemcpyDeviceToHost, st));
  PRISM_CUDA(cudaStreamSynchronize(st));
  if (v != 0) {
    PRISM_CUDA(cudaMemsetAsync(device_error, 0, sizeof(int), st));
    PRISM_CUDA(cudaStreamSynchronize(st));
    set_error("a kernel recorded device status %d", v);
    return v;
  }
  return PRISM_MOE_OK;
}

}  // extern "C"
