// Kernel 2 — dispatch plan (deterministic counting sort) and the row permutation.
//
// Entries are the flat routing slots f = t*k + j. Two stable orders are produced:
//   * expert-major: experts ascending, flat order inside an expert (the GEMM / send layout);
//   * dst-rank-major: EP ranks ascending, flat order inside a rank — exactly the reference's
//     perm = argsort(id // E_l, stable=True) (expert_parallel.py:37-39).
// Three launches:
//   1. plan_chunk: per chunk of 256 entries (ids staged in shared memory), stable ranks inside
//      the chunk by expert (warp 0) and by destination rank (warp 1) with __match_any_sync,
//      and the chunk's histograms;
//   2. plan_scan: one CTA turns the [chunk][key] histograms into per-chunk bases (each key's
//      column split across up to 1024/keys threads, two passes) and the key offsets;
//   3. plan_scatter: every output (entry_row, row_entry, perm, sorted_local_eid).
#include "common.cuh"

namespace prism {
namespace {

constexpr int kChunk = 256;   // entries per chunk
constexpr int kMaxKeys = 1024;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__global__ void __launch_bounds__(64)
    plan_chunk_kernel(const int64_t* __restrict__ ids, int64_t N, int E, int El, int W,
                      int32_t* __restrict__ rank_e, int32_t* __restrict__ rank_d,
                      int32_t* __restrict__ hist_e, int32_t* __restrict__ hist_d,
                      int* __restrict__ err) {
  __shared__ int32_t cnt[2][kMaxKeys];
  __shared__ int32_t key_s[kChunk];
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kChunk;
  const int n = static_cast<int>(N - c0 < kChunk ? N - c0 : kChunk);
  for (int i = threadIdx.x; i < kMaxKeys; i += blockDim.x) {
    cnt[0][i] = 0;
    cnt[1][i] = 0;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t e = ids[c0 + i];
    const bool ok = e >= 0 && e < E;
    if (!ok) record_device_error(err, PRISM_MOE_ERR_ARG);
    key_s[i] = ok ? static_cast<int32_t>(e) : -1;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0 || rank_d != nullptr) {
    int32_t* my_cnt = cnt[warp];
    int32_t* my_rank = warp == 0 ? rank_e : rank_d;
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const bool in = i < n;
      int key = -1 - lane;  // unique non-matching key for idle lanes
      if (in && key_s[i] >= 0) key = warp == 0 ? key_s[i] : key_s[i] / El;
      const uint32_t peers = __match_any_sync(0xffffffffu, key);
      const int prior = key >= 0 ? my_cnt[key] : 0;
      __syncwarp();
      if (key >= 0) {
        my_rank[c0 + i] = prior + __popc(peers & lanemask_lt());
        if (lane == __ffs(peers) - 1) my_cnt[key] = prior + __popc(peers);
      } else if (in) {
        my_rank[c0 + i] = -1;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist_e[blockIdx.x * E + e] = cnt[0][e];
  if (hist_d)
    for (int d = threadIdx.x; d < W; d += blockDim.x) hist_d[blockIdx.x * W + d] = cnt[1][d];
}

// Exclusive block scan of ``vals`` (n <= blockDim.x == 1024) in shared memory.
__device__ void block_exclusive_scan(int32_t* vals, int n, int32_t* total) {
  __shared__ int32_t tmp[kMaxKeys];
  const int i = threadIdx.x;
  const int32_t x = i < n ? vals[i] : 0;
  tmp[i] = x;
  __syncthreads();
  for (int off = 1; off < blockDim.x; off <<= 1) {
    const int32_t y = i >= off ? tmp[i - off] : 0;
    __syncthreads();
    tmp[i] += y;
    __syncthreads();
  }
  if (i < n) vals[i] = tmp[i] - x;
  if (i == blockDim.x - 1 && total) *total = tmp[i];
  __syncthreads();
}

// hist[c][key] (nchunks x nkeys) -> per-chunk exclusive bases in place; totals[key].
// Thread (part, key): part p of P = 1024 / nkeys scans chunks [p*cpp, (p+1)*cpp).
__device__ void column_scan(int32_t* __restrict__ hist, int nchunks, int nkeys,
                            int32_t* totals, int32_t* part_sum) {
  const int P = kMaxKeys / nkeys;
  const int key = threadIdx.x % nkeys;
  const int part = threadIdx.x / nkeys;
  const int cpp = (nchunks + P - 1) / P;
  const int lo = part * cpp;
  const int hi = lo + cpp < nchunks ? lo + cpp : nchunks;
  int32_t s = 0;
  if (part < P) {
#pragma unroll 8
    for (int c = lo; c < hi; ++c) s += hist[c * nkeys + key];
    part_sum[part * nkeys + key] = s;
  }
  __syncthreads();
  if (part < P) {
    int32_t run = 0;
    for (int q = 0; q < part; ++q) run += part_sum[q * nkeys + key];
    if (part == 0) {
      int32_t tot = 0;
      for (int q = 0; q < P; ++q) tot += part_sum[q * nkeys + key];
      totals[key] = tot;
    }
#pragma unroll 8
    for (int c = lo; c < hi; ++c) {
      const int32_t h = hist[c * nkeys + key];
      hist[c * nkeys + key] = run;
      run += h;
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(1024)
    plan_scan_kernel(int nchunks, int E, int W, int32_t* __restrict__ hist_e,
                     int32_t* __restrict__ hist_d, int32_t* __restrict__ counts,
                     int32_t* __restrict__ offsets, int32_t* __restrict__ split_off,
                     int64_t* __restrict__ splits64) {
  __shared__ int32_t tot[kMaxKeys];
  __shared__ int32_t part_sum[kMaxKeys];
  __shared__ int32_t total;
  column_scan(hist_e, nchunks, E, tot, part_sum);
  if (threadIdx.x < E && counts) counts[threadIdx.x] = tot[threadIdx.x];
  block_exclusive_scan(tot, E, &total);
  if (threadIdx.x < E) offsets[threadIdx.x] = tot[threadIdx.x];
  if (threadIdx.x == 0) offsets[E] = total;
  __syncthreads();
  if (hist_d) {
    column_scan(hist_d, nchunks, W, tot, part_sum);
    if (threadIdx.x < W && splits64) splits64[threadIdx.x] = tot[threadIdx.x];
    block_exclusive_scan(tot, W, nullptr);
    if (threadIdx.x < W) split_off[threadIdx.x] = tot[threadIdx.x];
  }
}

__global__ void plan_scatter_kernel(const int64_t* __restrict__ ids, int64_t N, int E, int El,
                                    int W, const int32_t* __restrict__ rank_e,
                                    const int32_t* __restrict__ rank_d,
                                    const int32_t* __restrict__ base_e,
                                    const int32_t* __restrict__ base_d,
                                    const int32_t* __restrict__ offsets,
                                    const int32_t* __restrict__ split_off,
                                    int32_t* __restrict__ entry_row,
                                    int32_t* __restrict__ row_entry, int64_t* __restrict__ perm,
                                    int64_t* __restrict__ sorted_leid) {
  const int64_t f = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (f >= N) return;
  const int64_t e = ids[f];
  if (e < 0 || e >= E) {
    if (entry_row) entry_row[f] = -1;
    return;
  }
  const int c = static_cast<int>(f / kChunk);
  const int32_t row = offsets[e] + base_e[c * E + e] + rank_e[f];
  if (entry_row) entry_row[f] = row;
  if (row_entry) row_entry[row] = static_cast<int32_t>(f);
  if (perm || sorted_leid) {
    const int d = static_cast<int>(e / El);
    const int64_t p = split_off[d] + base_d[c * W + d] + rank_d[f];
    if (perm) perm[p] = f;
    if (sorted_leid) sorted_leid[p] = e % El;
  }
}

// One warp per token: read the row once, write it to its k expert-major rows.
template <int kVecPerLane>
__global__ void permute_rows_kernel(const uint4* __restrict__ x, int64_t T, int64_t vec_per_row,
                                    int k, const int32_t* __restrict__ entry_row,
                                    uint4* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  const int my_row = lane < k ? entry_row[t * k + lane] : -1;
  for (int64_t v0 = 0; v0 < vec_per_row; v0 += 32 * kVecPerLane) {
    uint4 buf[kVecPerLane];
#pragma unroll
    for (int q = 0; q < kVecPerLane; ++q) {
      const int64_t v = v0 + q * 32 + lane;
      if (v < vec_per_row) buf[q] = x[t * vec_per_row + v];
    }
    for (int j = 0; j < k; ++j) {
      const int r = __shfl_sync(0xffffffffu, my_row, j);
      if (r < 0) continue;
#pragma unroll
      for (int q = 0; q < kVecPerLane; ++q) {
        const int64_t v = v0 + q * 32 + lane;
        if (v < vec_per_row) xs[static_cast<int64_t>(r) * vec_per_row + v] = buf[q];
      }
    }
  }
}

}  // namespace

size_t dispatch_workspace_size(int64_t N, int E, int W) {
  const int64_t nchunks = ceil_div(N > 0 ? N : 1, kChunk);
  size_t b = 256;                                        // error word + scalars
  b += align_up(sizeof(int32_t) * N, 256) * 2;           // rank_e, rank_d
  b += align_up(sizeof(int32_t) * nchunks * E, 256);     // hist_e / base_e
  b += align_up(sizeof(int32_t) * nchunks * W, 256);     // hist_d / base_d
  b += align_up(sizeof(int32_t) * (E + 1), 256) * 2;     // counts, offsets (scratch copies)
  b += align_up(sizeof(int32_t) * (W + 1), 256);         // split_off
  return b;
}

int build_plan(const int64_t* ids, int64_t T, int k, int E, int W, int64_t* perm,
               int64_t* splits, int64_t* sorted_leid, int32_t* counts, int32_t* offsets,
               int32_t* entry_row, int32_t* row_entry, void* ws, size_t ws_bytes,
               cudaStream_t st, int* err_out) {
  const int64_t N = T * k;
  PRISM_CHECK_ARG(E >= 1 && E <= kMaxKeys, "num_experts %d outside [1, %d]", E, kMaxKeys);
  PRISM_CHECK_ARG(W >= 1 && E % W == 0, "num_experts %d not divisible by ep_size %d", E, W);
  PRISM_CHECK_ARG(ws_bytes >= dispatch_workspace_size(N, E, W),
                  "dispatch workspace too small (%zu < %zu)", ws_bytes,
                  dispatch_workspace_size(N, E, W));
  PRISM_CHECK_ARG(N <= (int64_t(1) << 31) - 1, "too many routed entries");
  const int El = E / W;
  const int64_t nchunks = ceil_div(N > 0 ? N : 1, kChunk);
  char* p = static_cast<char*>(ws);
  int* err = err_out ? err_out : reinterpret_cast<int*>(p);   // where ERR_ARG for ids goes
  p += 256;
  int32_t* rank_e = reinterpret_cast<int32_t*>(p);
  p += align_up(sizeof(int32_t) * N, 256);
  int32_t* rank_d = reinterpret_cast<int32_t*>(p);
  p += align_up(sizeof(int32_t) * N, 256);
  int32_t* hist_e = reinterpret_cast<int32_t*>(p);
  p += align_up(sizeof(int32_t) * nchunks * E, 256);
  int32_t* hist_d = reinterpret_cast<int32_t*>(p);
  p += align_up(sizeof(int32_t) * nchunks * W, 256);
  int32_t* counts_s = reinterpret_cast<int32_t*>(p);
  p += align_up(sizeof(int32_t) * (E + 1), 256);
  int32_t* offsets_s = reinterpret_cast<int32_t*>(p);
  p += align_up(sizeof(int32_t) * (E + 1), 256);
  int32_t* split_off = reinterpret_cast<int32_t*>(p);
  const bool want_d = perm || sorted_leid || splits;
  int32_t* cnt = counts ? counts : counts_s;
  int32_t* off = offsets ? offsets : offsets_s;
  if (N == 0) {
    PRISM_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int32_t) * E, st));
    PRISM_CUDA(cudaMemsetAsync(off, 0, sizeof(int32_t) * (E + 1), st));
    if (splits) PRISM_CUDA(cudaMemsetAsync(splits, 0, sizeof(int64_t) * W, st));
    return PRISM_MOE_OK;
  }
  plan_chunk_kernel<<<static_cast<unsigned>(nchunks), 64, 0, st>>>(
      ids, N, E, El, W, rank_e, want_d ? rank_d : nullptr, hist_e, want_d ? hist_d : nullptr,
      err);
  PRISM_LAUNCH_CHECK("plan_chunk_kernel launch");
  plan_scan_kernel<<<1, kMaxKeys, 0, st>>>(static_cast<int>(nchunks), E, W, hist_e,
                                           want_d ? hist_d : nullptr, cnt, off, split_off,
                                           splits);
  PRISM_LAUNCH_CHECK("plan_scan_kernel launch");
  plan_scatter_kernel<<<static_cast<unsigned>(ceil_div(N, 256)), 256, 0, st>>>(
      ids, N, E, El, W, rank_e, rank_d, hist_e, hist_d, off, split_off, entry_row, row_entry,
      perm, sorted_leid);
  PRISM_LAUNCH_CHECK("plan_scatter_kernel launch");
  return PRISM_MOE_OK;
}

int permute_rows(const void* x, int64_t T, int64_t row_bytes, int k, const int32_t* entry_row,
                 void* xs, cudaStream_t st) {
  PRISM_CHECK_ARG(row_bytes % 16 == 0, "row bytes %lld not a multiple of 16",
                  static_cast<long long>(row_bytes));
  PRISM_CHECK_ARG(k >= 1 && k <= 32, "top_k %d outside [1, 32]", k);
  if (T == 0) return PRISM_MOE_OK;
  const int64_t vpr = row_bytes / 16;
  const unsigned blocks = static_cast<unsigned>(ceil_div(T * 32, 256));
  if (vpr >= 256)
    permute_rows_kernel<8><<<blocks, 256, 0, st>>>(static_cast<const uint4*>(x), T, vpr, k,
                                                   entry_row, static_cast<uint4*>(xs));
  else
    permute_rows_kernel<2><<<blocks, 256, 0, st>>>(static_cast<const uint4*>(x), T, vpr, k,
                                                   entry_row, static_cast<uint4*>(xs));
  PRISM_LAUNCH_CHECK("permute_rows_kernel launch");
  return PRISM_MOE_OK;
}

}  // namespace prism
