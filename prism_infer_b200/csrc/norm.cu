// Kernel 6 — RMSNorm, optionally after the residual add (prism_infer/layers/layernorm.py:16-40):
// the decoder layer's post_attention_layernorm in front of the MoE router
// (prism_infer/models/qwen3.py:184). One warp per token row, two passes over the row: the
// first forms xf = x (+ residual), writes residual_out and the sum of squares, the second
// (re-reading the row, still in L1/L2) writes the scaled output. See norm.cuh for the
// numerics.
#include "internal.h"
#include "norm.cuh"

namespace prism {
namespace {

template <bool kBf16>
__global__ void __launch_bounds__(256)
    rmsnorm_kernel(const uint4* x, const uint4* residual,
                   const uint4* __restrict__ weight, int64_t T, int64_t vpr, int64_t hidden,
                   float eps, uint4* out, uint4* __restrict__ residual_out) {
  constexpr int kEl = kBf16 ? 8 : 4;
  const int lane = threadIdx.x & 31;
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  const uint4* xr = x + t * vpr;
  const uint4* rr = residual ? residual + t * vpr : nullptr;
  float ss = 0.f;
  for (int64_t v = lane; v < vpr; v += 32) {
    float xf[kEl];
    const uint4 rv = rr ? rr[v] : make_uint4(0, 0, 0, 0);
    norm_sum<kBf16>(xr[v], rr ? &rv : nullptr, xf, ss);
    if (residual_out) residual_out[t * vpr + v] = pack_vec<kBf16>(xf);
  }
  const float rs = rms_scale(warp_sum(ss), hidden, eps);
  for (int64_t v = lane; v < vpr; v += 32) {
    float xf[kEl];
    const uint4 rv = rr ? rr[v] : make_uint4(0, 0, 0, 0);
    float dummy = 0.f;
    norm_sum<kBf16>(xr[v], rr ? &rv : nullptr, xf, dummy);
    out[t * vpr + v] = norm_scale<kBf16>(xf, weight[v], rs);
  }
}

}  // namespace

int rmsnorm(const void* x, const void* residual, const void* weight, float eps, int dtype,
            int64_t T, int64_t hidden, void* out, void* residual_out, cudaStream_t st) {
  const int64_t el = dtype == PRISM_MOE_BF16 ? 2 : 4;
  PRISM_CHECK_ARG((hidden * el) % 16 == 0, "rmsnorm: hidden*elem_size must be a multiple of 16");
  PRISM_CHECK_ARG(!residual || residual_out, "rmsnorm: residual_out is required with residual");
  PRISM_CHECK_ARG(!residual_out || (residual_out != x && residual_out != residual),
                  "rmsnorm: residual_out must not alias x or residual");
  if (T == 0) return PRISM_MOE_OK;
  const int64_t vpr = hidden * el / 16;
  const unsigned blocks = static_cast<unsigned>(ceil_div(T * 32, 256));
  const uint4* xv = static_cast<const uint4*>(x);
  const uint4* rv = static_cast<const uint4*>(residual);
  const uint4* wv = static_cast<const uint4*>(weight);
  uint4* ov = static_cast<uint4*>(out);
  uint4* rov = residual ? static_cast<uint4*>(residual_out) : nullptr;
  if (dtype == PRISM_MOE_BF16)
    rmsnorm_kernel<true><<<blocks, 256, 0, st>>>(xv, rv, wv, T, vpr, hidden, eps, ov, rov);
  else
    rmsnorm_kernel<false><<<blocks, 256, 0, st>>>(xv, rv, wv, T, vpr, hidden, eps, ov, rov);
  PRISM_LAUNCH_CHECK("rmsnorm_kernel launch");
  return PRISM_MOE_OK;
}

}  // namespace prism
