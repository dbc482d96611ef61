// RMSNorm with the residual add of a decoder layer, as one warp per token row — shared by the
// standalone norm kernel (norm.cu) and the combine kernel's epilogue (combine.cu), which must
// produce the same bits for the same row.
//
// Numerics of prism_infer/layers/layernorm.py:16-40 (rms_forward / add_rms_forward):
//   xf = float(x) [+ float(residual)];  residual_out = dtype(xf)
//   var = mean(xf^2) over the row;       out = dtype(dtype(xf * rsqrt(var + eps)) * weight)
// Every lane owns the 16-byte vectors lane, lane + 32, ... of the row; the sum of squares is
// accumulated per lane in vector and element order and then reduced across the warp (xor
// butterfly), so two kernels that walk a row the same way agree bit for bit.
#pragma once
#include "common.cuh"

namespace prism {
namespace {

template <bool kBf16>
__device__ __forceinline__ void unpack_vec(const uint4& u, float* f) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
  if constexpr (kBf16) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      f[2 * q] = __uint_as_float(w[q] << 16);
      f[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) f[q] = __uint_as_float(w[q]);
  }
}

template <bool kBf16>
__device__ __forceinline__ uint4 pack_vec(const float* f) {
  uint4 o;
  uint32_t* w = reinterpret_cast<uint32_t*>(&o);
  if constexpr (kBf16) {
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = pack_bf16x2(f[2 * q], f[2 * q + 1]);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = __float_as_uint(f[q]);
  }
  return o;
}

// xf = a (+ r) in fp32 into ``xf``; adds xf^2 to ``ss`` in element order.
template <bool kBf16>
__device__ __forceinline__ void norm_sum(const uint4& a, const uint4* r, float* xf, float& ss) {
  constexpr int kEl = kBf16 ? 8 : 4;
  unpack_vec<kBf16>(a, xf);
  if (r) {
    float rf[kEl];
    unpack_vec<kBf16>(*r, rf);
#pragma unroll
    for (int q = 0; q < kEl; ++q) xf[q] = __fadd_rn(xf[q], rf[q]);
  }
#pragma unroll
  for (int q = 0; q < kEl; ++q) ss = __fmaf_rn(xf[q], xf[q], ss);
}

// out = dtype(dtype(xf * rs) * w) of one vector.
template <bool kBf16>
__device__ __forceinline__ uint4 norm_scale(const float* xf, const uint4& w, float rs) {
  constexpr int kEl = kBf16 ? 8 : 4;
  float wf[kEl], o[kEl];
  unpack_vec<kBf16>(w, wf);
#pragma unroll
  for (int q = 0; q < kEl; ++q) {
    const float n = __fmul_rn(xf[q], rs);
    o[q] = kBf16 ? __fmul_rn(round_bf16(n), wf[q]) : __fmul_rn(n, wf[q]);
  }
  return pack_vec<kBf16>(o);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float rms_scale(float ss, int64_t hidden, float eps) {
  return rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(hidden)), eps));
}

}  // namespace
}  // namespace prism
