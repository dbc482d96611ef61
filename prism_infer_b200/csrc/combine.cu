// Kernel 5 — weighted combine: out[t] = sum_j w[t, j] * y[row(t*k + j)].
//
// Numerics follow the reference's combine_weighted_sum (expert_parallel.py:45-57): each product
// w * y is materialised in the element type, the k products are accumulated in fp32 in slot
// order, and the sum is rounded once. One warp per token, 16-byte loads: each lane owns 8 bf16
// (or 4 fp32) columns per step, all k source rows are loaded before accumulating.
#include "common.cuh"

namespace prism {
namespace {

template <bool kBf16>
__global__ void __launch_bounds__(256)
    combine_kernel(const void* __restrict__ y, const int32_t* __restrict__ entry_row,
                   const void* __restrict__ w, int64_t T, int k, int64_t hidden,
                   void* __restrict__ out) {
  constexpr int kEl = kBf16 ? 8 : 4;  // elements per 16-byte vector
  const int lane = threadIdx.x & 31;
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  int64_t rows[32];
  float wt[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < k) {
      const int64_t f = t * k + j;
      rows[j] = entry_row ? static_cast<int64_t>(entry_row[f]) : f;
      if constexpr (kBf16)
        wt[j] = bf16_bits_to_float(reinterpret_cast<const uint16_t*>(w)[f]);
      else
        wt[j] = reinterpret_cast<const float*>(w)[f];
    }
  }
  const int64_t vpr = hidden / kEl;
  const uint4* yv = static_cast<const uint4*>(y);
  uint4* ov = static_cast<uint4*>(out);
  for (int64_t v = lane; v < vpr; v += 32) {
    float acc[kEl];
#pragma unroll
    for (int q = 0; q < kEl; ++q) acc[q] = 0.f;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
      if (j >= k) break;
      if (rows[j] < 0) continue;
      const uint4 u = yv[rows[j] * vpr + v];
      const uint32_t* uw = reinterpret_cast<const uint32_t*>(&u);
      if constexpr (kBf16) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = __uint_as_float(uw[q] << 16);
          const float hi = __uint_as_float(uw[q] & 0xffff0000u);
          acc[2 * q] += round_bf16(lo * wt[j]);
          acc[2 * q + 1] += round_bf16(hi * wt[j]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          acc[q] = __fadd_rn(acc[q], __fmul_rn(__uint_as_float(uw[q]), wt[j]));
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
    if constexpr (kBf16) {
#pragma unroll
      for (int q = 0; q < 4; ++q) ow[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) ow[q] = __float_as_uint(acc[q]);
    }
    ov[t * vpr + v] = o;
  }
}

}  // namespace

int combine(const void* y, int dtype, const int32_t* entry_row, const void* w, int64_t T, int k,
            int64_t hidden, void* out, cudaStream_t st) {
  const int64_t el = dtype == PRISM_MOE_BF16 ? 2 : 4;
  PRISM_CHECK_ARG((hidden * el) % 16 == 0, "combine: hidden*elem_size must be a multiple of 16");
  PRISM_CHECK_ARG(k >= 1 && k <= 32, "combine: top_k %d outside [1, 32]", k);
  if (T == 0) return PRISM_MOE_OK;
  const unsigned blocks = static_cast<unsigned>(ceil_div(T * 32, 256));
  if (dtype == PRISM_MOE_BF16)
    combine_kernel<true><<<blocks, 256, 0, st>>>(y, entry_row, w, T, k, hidden, out);
  else
    combine_kernel<false><<<blocks, 256, 0, st>>>(y, entry_row, w, T, k, hidden, out);
  PRISM_LAUNCH_CHECK("combine_kernel launch");
  return PRISM_MOE_OK;
}

}  // namespace prism
