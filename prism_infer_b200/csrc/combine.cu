// Kernel 5 — weighted combine: out[t] = sum_j w[t, j] * y[row(t*k + j)].
//
// Numerics follow the reference's combine_weighted_sum (expert_parallel.py:45-57): each product
// w * y is materialised in the element type, the k products are accumulated in fp32 in slot
// order, and the sum is rounded once. One warp per token, 16-byte loads: each lane owns 8 bf16
// (or 4 fp32) columns per step and issues all k row loads before accumulating. k is a template
// parameter for the common top-k values (rows and weights stay in registers); other k use a
// generic loop.
//
// Optional epilogue (CombineSource::norm_weight): the decoder layer's next residual add and
// RMSNorm on the block output, as prism_infer/models/qwen3.py:179-186 applies them in the next
// layer (add_rms_forward, layernorm.py:28-40): residual_out = dtype(float(moe_out) + residual),
// out = RMSNorm(that sum). The first pass writes moe_out into ``out`` and the residual, the
// second re-reads both (the same lane's own writes) and overwrites ``out`` with the normalised
// row — the arithmetic of norm.cuh, so it equals combine followed by prism_moe_rmsnorm.
#include "common.cuh"
#include "internal.h"
#include "norm.cuh"

namespace prism {
namespace {

template <bool kBf16>
__device__ __forceinline__ void accumulate(float* acc, const uint4& u, float w) {
  const uint32_t* uw = reinterpret_cast<const uint32_t*>(&u);
  if constexpr (kBf16) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[2 * q] += round_bf16(__uint_as_float(uw[q] << 16) * w);
      acc[2 * q + 1] += round_bf16(__uint_as_float(uw[q] & 0xffff0000u) * w);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(__uint_as_float(uw[q]), w));
  }
}

template <bool kBf16>
__device__ __forceinline__ uint4 pack(const float* acc) {   // round each sum once
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
  if constexpr (kBf16) {
#pragma unroll
    for (int q = 0; q < 4; ++q) ow[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) ow[q] = __float_as_uint(acc[q]);
  }
  return o;
}

template <bool kBf16>
__device__ __forceinline__ float load_w(const void* w, int64_t f) {
  if constexpr (kBf16)
    return bf16_bits_to_float(reinterpret_cast<const uint16_t*>(w)[f]);
  else
    return reinterpret_cast<const float*>(w)[f];
}

// kK > 0: compile-time top-k; kK == 0: runtime k (<= 32).
template <bool kBf16, int kK>
__global__ void __launch_bounds__(256)
    combine_kernel(const uint4* __restrict__ y, const int32_t* __restrict__ entry_row,
                   const void* __restrict__ w, int64_t T, int k_rt, int64_t vpr,
                   uint4* out, CombineSource src) {
  constexpr int kEl = kBf16 ? 8 : 4;
  const int lane = threadIdx.x & 31;
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  if (src.gate_err && *reinterpret_cast<const volatile int*>(src.gate_err) == PRISM_MOE_ERR_TIMEOUT)
    return;   // the step's exchange did not complete: its rows are not all there
  if (src.parity) y += static_cast<int64_t>(*src.parity & 1u) * (src.parity_stride_bytes / 16);
  const bool norm = src.norm_weight != nullptr;
  const uint4* res = static_cast<const uint4*>(src.residual);
  uint4* res_out = static_cast<uint4*>(src.residual_out);
  float ss = 0.f;
  // one output vector: plain, or the first pass of the norm epilogue
  auto emit = [&](int64_t v, const float* acc) {
    const uint4 a = pack<kBf16>(acc);
    out[t * vpr + v] = a;
    if (norm) {
      float xf[kEl];
      const uint4 rv = res[t * vpr + v];
      norm_sum<kBf16>(a, &rv, xf, ss);
      res_out[t * vpr + v] = pack_vec<kBf16>(xf);
    }
  };
  const int k = kK > 0 ? kK : k_rt;
  // lane j < k fetches slot j's row and weight once; broadcast by shuffle
  int64_t my_row = -1;
  float my_w = 0.f;
  if (lane < k) {
    const int64_t f = t * k + lane;
    my_row = entry_row ? static_cast<int64_t>(entry_row[f]) : f;
    my_w = load_w<kBf16>(w, f);
  }
  if constexpr (kK > 0) {
    int64_t rows[kK];
    float wt[kK];
#pragma unroll
    for (int j = 0; j < kK; ++j) {
      rows[j] = __shfl_sync(0xffffffffu, my_row, j);
      wt[j] = __shfl_sync(0xffffffffu, my_w, j);
    }
    for (int64_t v = lane; v < vpr; v += 32) {
      uint4 u[kK];
#pragma unroll
      for (int j = 0; j < kK; ++j) u[j] = rows[j] >= 0 ? y[rows[j] * vpr + v] : make_uint4(0, 0, 0, 0);
      float acc[kEl];
#pragma unroll
      for (int q = 0; q < kEl; ++q) acc[q] = 0.f;
#pragma unroll
      for (int j = 0; j < kK; ++j)
        if (rows[j] >= 0) accumulate<kBf16>(acc, u[j], wt[j]);
      emit(v, acc);
    }
  } else {
    for (int64_t v = lane; v < vpr; v += 32) {
      float acc[kEl];
#pragma unroll
      for (int q = 0; q < kEl; ++q) acc[q] = 0.f;
      for (int j = 0; j < k; ++j) {
        const int64_t r = __shfl_sync(0xffffffffu, my_row, j);
        const float wj = __shfl_sync(0xffffffffu, my_w, j);
        if (r >= 0) accumulate<kBf16>(acc, y[r * vpr + v], wj);
      }
      emit(v, acc);
    }
  }
  if (norm) {   // second pass: the normalised row
    const float rs = rms_scale(warp_sum(ss), src.hidden, src.eps);
    const uint4* wv = static_cast<const uint4*>(src.norm_weight);
    for (int64_t v = lane; v < vpr; v += 32) {
      float xf[kEl];
      const uint4 rv = res[t * vpr + v];
      float unused = 0.f;
      norm_sum<kBf16>(out[t * vpr + v], &rv, xf, unused);
      out[t * vpr + v] = norm_scale<kBf16>(xf, wv[v], rs);
    }
  }
}

template <bool kBf16>
void launch_combine(const void* y, const int32_t* entry_row, const void* w, int64_t T, int k,
                    int64_t vpr, void* out, const CombineSource& src, cudaStream_t st) {
  const unsigned blocks = static_cast<unsigned>(ceil_div(T * 32, 256));
  const uint4* yv = static_cast<const uint4*>(y);
  uint4* ov = static_cast<uint4*>(out);
  switch (k) {
    case 8: combine_kernel<kBf16, 8><<<blocks, 256, 0, st>>>(yv, entry_row, w, T, k, vpr, ov, src); break;
    case 4: combine_kernel<kBf16, 4><<<blocks, 256, 0, st>>>(yv, entry_row, w, T, k, vpr, ov, src); break;
    case 2: combine_kernel<kBf16, 2><<<blocks, 256, 0, st>>>(yv, entry_row, w, T, k, vpr, ov, src); break;
    case 1: combine_kernel<kBf16, 1><<<blocks, 256, 0, st>>>(yv, entry_row, w, T, k, vpr, ov, src); break;
    default: combine_kernel<kBf16, 0><<<blocks, 256, 0, st>>>(yv, entry_row, w, T, k, vpr, ov, src);
  }
}

}  // namespace

int combine(const void* y, int dtype, const int32_t* entry_row, const void* w, int64_t T, int k,
            int64_t hidden, void* out, cudaStream_t st, const CombineSource* src) {
  const int64_t el = dtype == PRISM_MOE_BF16 ? 2 : 4;
  PRISM_CHECK_ARG((hidden * el) % 16 == 0, "combine: hidden*elem_size must be a multiple of 16");
  PRISM_CHECK_ARG(k >= 1 && k <= 32, "combine: top_k %d outside [1, 32]", k);
  PRISM_CHECK_ARG(!src || src->parity_stride_bytes % 16 == 0, "combine: parity stride alignment");
  PRISM_CHECK_ARG(!src || !src->norm_weight || (src->residual && src->residual_out),
                  "combine: the norm epilogue needs residual and residual_out");
  PRISM_CHECK_ARG(!src || !src->norm_weight ||
                      (src->residual_out != src->residual && src->residual_out != out),
                  "combine: residual_out must not alias residual or out");
  if (T == 0) return PRISM_MOE_OK;
  const int64_t vpr = hidden * el / 16;
  CombineSource s = src ? *src : CombineSource{};
  s.hidden = hidden;
  if (dtype == PRISM_MOE_BF16)
    launch_combine<true>(y, entry_row, w, T, k, vpr, out, s, st);
  else
    launch_combine<false>(y, entry_row, w, T, k, vpr, out, s, st);
  PRISM_LAUNCH_CHECK("combine_kernel launch");
  return PRISM_MOE_OK;
}

}  // namespace prism
