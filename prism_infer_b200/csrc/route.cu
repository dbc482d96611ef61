// Kernel 1 — router post-processing: fp32 softmax, top-k, renormalisation, cast.
//
// One warp per token. The arithmetic reproduces what the reference's torch calls compute on
// CUDA (prism_infer/layers/moe.py:77-81), so that routing is bit-identical:
//   * softmax: lane l holds elements l + 32*it (it < next_pow2(E)/32; E <= 32 uses a
//     next_pow2(E)-wide lane group), sums them serially, then xor-butterfly sums; p = e / sum;
//   * top-k: all values greater than the k-th, then values equal to it in ascending expert index;
//     the k gathered pairs are ordered by the same 32-wide bitonic compare-exchange network
//     torch applies to top-k outputs, invalid slots sinking to the end;
//   * renorm: lane j of a last_pow2(k)-wide group sums w[j], w[j+width], ..., then lanes
//     combine by shuffle-down with offsets width/2, ..., 2, 1 (torch's intra-warp reduction
//     order on CUDA); w / sum; cast with round-to-nearest-even.
#include "common.cuh"

namespace prism {
namespace {

constexpr int kRouteWarps = 4;

__device__ __forceinline__ bool gt_nan(float a, float b) {
  return (isnan(a) && !isnan(b)) || a > b;
}

template <bool kBf16>
__device__ __forceinline__ float load_logit(const void* p, int64_t i) {
  if constexpr (kBf16) {
    return bf16_bits_to_float(reinterpret_cast<const uint16_t*>(p)[i]);
  } else {
    return reinterpret_cast<const float*>(p)[i];
  }
}

template <bool kBf16, int EPT>
__global__ void __launch_bounds__(32 * kRouteWarps)
    route_topk_kernel(const void* __restrict__ logits, int64_t num_tokens, int E, int k,
                      int renorm, int width, int64_t* __restrict__ ids_out,
                      void* __restrict__ w_out, int32_t* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kRouteWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  const float NEG_INF = -__int_as_float(0x7f800000);
  const bool lane_ok = lane < width;

  // ---- softmax (fp32) ----
  float v[EPT];
#pragma unroll
  for (int it = 0; it < EPT; ++it) {
    const int idx = lane + 32 * it;
    v[it] = (lane_ok && idx < E) ? load_logit<kBf16>(logits, t * E + idx) : NEG_INF;
  }
  float m = v[0];
#pragma unroll
  for (int it = 1; it < EPT; ++it) m = m > v[it] ? m : v[it];
  for (int off = width >> 1; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, m, off);
    m = m < o ? o : m;
  }
  float s = 0.f;
#pragma unroll
  for (int it = 0; it < EPT; ++it) {
    v[it] = expf(v[it] - m);
    s += v[it];
  }
  for (int off = width >> 1; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
#pragma unroll
  for (int it = 0; it < EPT; ++it) v[it] = v[it] / s;

  // ---- top-k selection: best value first, lowest index among equal values ----
  // Probabilities are >= 0, so their bit patterns order like their values; NaN maps above +inf
  // (torch.topk ranks NaN highest). Keys are offset by one so that 0 means "nothing left".
  uint32_t key_u[EPT];
#pragma unroll
  for (int it = 0; it < EPT; ++it) {
    const int idx = lane + 32 * it;
    key_u[it] = (lane_ok && idx < E) ? (isnan(v[it]) ? 0x7f800001u : __float_as_uint(v[it])) + 1u
                                     : 0u;
  }
  float my_v = 0.f;
  int my_i = 0;
  uint32_t my_key = 0;
  for (int j = 0; j < k; ++j) {
    uint32_t best = 0;
    uint32_t best_i = 0xffffffffu;
#pragma unroll
    for (int it = 0; it < EPT; ++it) {
      if (key_u[it] > best) {   // ascending it: the lowest index wins among equal keys
        best = key_u[it];
        best_i = lane + 32 * it;
      }
    }
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, best);
    const uint32_t widx = __reduce_min_sync(0xffffffffu, best == wmax ? best_i : 0xffffffffu);
    if ((widx & 31u) == static_cast<uint32_t>(lane)) {
#pragma unroll
      for (int it = 0; it < EPT; ++it)
        if (static_cast<uint32_t>(lane + 32 * it) == widx) key_u[it] = 0;
    }
    if (lane == j) {
      my_key = wmax;
      my_i = static_cast<int>(widx);
    }
  }
  // the selected probability itself, from the lane that holds it
  my_v = __shfl_sync(0xffffffffu, v[0], my_i & 31);
#pragma unroll
  for (int it = 1; it < EPT; ++it) {
    const float o = __shfl_sync(0xffffffffu, v[it], my_i & 31);
    if ((my_i >> 5) == it) my_v = o;
  }
  const bool valid = lane < k;
  float key = my_v;
  int val = my_i;

  // ---- torch's output order. Distinct values: descending, which the selection already is.
  // With ties, replay torch: gather (value > kth) by index, then (value == kth) by index, then
  // its 32-wide bitonic network (descending, invalid slots last).
  const uint32_t next_key = __shfl_down_sync(0xffffffffu, my_key, 1);
  const bool has_tie = __any_sync(0xffffffffu, lane < k - 1 && my_key == next_key);
  if (has_tie) {
    const float vk = __shfl_sync(0xffffffffu, my_v, k - 1);
    const bool is_gt = valid && gt_nan(my_v, vk);
    const int n_gt = __popc(__ballot_sync(0xffffffffu, is_gt));
    int gpos = lane;
    {
      int r = 0;
      for (int q = 0; q < n_gt; ++q) {
        const int oi = __shfl_sync(0xffffffffu, my_i, q);
        r += (oi < my_i) ? 1 : 0;
      }
      if (is_gt) gpos = r;
    }
    int src = lane;
    for (int q = 0; q < k; ++q) {
      const int g = __shfl_sync(0xffffffffu, gpos, q);
      if (g == lane) src = q;
    }
    key = __shfl_sync(0xffffffffu, my_v, src);
    val = __shfl_sync(0xffffffffu, my_i, src);
    int ok = valid ? 1 : 0;
    auto cmp_exchange = [&](int stride, bool flag) {
      const float pk = __shfl_xor_sync(0xffffffffu, key, stride);
      const int pv = __shfl_xor_sync(0xffffffffu, val, stride);
      const int pok = __shfl_xor_sync(0xffffffffu, ok, stride);
      const bool is_lo = (lane & stride) == 0;
      const float ak = is_lo ? key : pk;
      const float bk = is_lo ? pk : key;
      const int aok = is_lo ? ok : pok;
      const int bok = is_lo ? pok : ok;
      const bool swap = (gt_nan(ak, bk) && aok) || !bok;
      if (swap == flag) {
        key = pk;
        val = pv;
        ok = pok;
      }
    };
#pragma unroll
    for (int size = 2; size < 32; size <<= 1) {
#pragma unroll
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const int lo = lane & ~stride;
        cmp_exchange(stride, (lo & size) != 0);
      }
    }
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) cmp_exchange(stride, false);
  }

  // ---- renormalisation in torch's reduction order ----
  float w = key;
  if (renorm) {
    int rw = 1;
    while (rw * 2 <= k) rw *= 2;
    // lane l < rw holds w[l] (+ w[l+rw] when it exists: rw > k/2, so at most two elements)
    const float other = __shfl_down_sync(0xffffffffu, key, rw);
    float acc = 0.f;
    if (lane < rw) acc = (lane + rw < k) ? key + other : key;
    for (int off = rw >> 1; off > 0; off >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, off);
    const float sum = __shfl_sync(0xffffffffu, acc, 0);
    w = key / sum;
  }
  if (valid) {
    ids_out[t * k + lane] = static_cast<int64_t>(val);
    if constexpr (kBf16) {
      reinterpret_cast<uint16_t*>(w_out)[t * k + lane] = float_to_bf16_bits(w);
    } else {
      reinterpret_cast<float*>(w_out)[t * k + lane] = w;
    }
    if (counts) atomicAdd(counts + val, 1);
  }
}

template <bool kBf16>
int launch_route(const void* logits, int64_t T, int E, int k, int renorm, int64_t* ids, void* w,
                 int32_t* counts, cudaStream_t st) {
  int p2 = 1;
  while (p2 < E) p2 <<= 1;
  const int width = p2 < 32 ? p2 : 32;
  const int ept = p2 / width;
  const dim3 grid(static_cast<unsigned>(ceil_div(T, kRouteWarps)));
  const dim3 block(32 * kRouteWarps);
#define PRISM_ROUTE_CASE(N)                                                                   \
  case N:                                                                                     \
    route_topk_kernel<kBf16, N><<<grid, block, 0, st>>>(logits, T, E, k, renorm, width, ids, w, \
                                                       counts);                               \
    break;
  switch (ept) {
    PRISM_ROUTE_CASE(1)
    PRISM_ROUTE_CASE(2)
    PRISM_ROUTE_CASE(4)
    PRISM_ROUTE_CASE(8)
    PRISM_ROUTE_CASE(16)
    PRISM_ROUTE_CASE(32)
    default:
      set_error("route_topk: num_experts %d unsupported", E);
      return PRISM_MOE_ERR_UNSUPPORTED;
  }
#undef PRISM_ROUTE_CASE
  PRISM_LAUNCH_CHECK("route_topk_kernel launch");
  return PRISM_MOE_OK;
}

}  // namespace

int route_topk(const void* logits, int dtype, int64_t T, int E, int k, int renorm, int64_t* ids,
               void* w, int32_t* counts, cudaStream_t st) {
  if (counts) PRISM_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, st));
  if (T == 0) return PRISM_MOE_OK;
  return dtype == PRISM_MOE_BF16 ? launch_route<true>(logits, T, E, k, renorm, ids, w, counts, st)
                                 : launch_route<false>(logits, T, E, k, renorm, ids, w, counts, st);
}

}  // namespace prism
