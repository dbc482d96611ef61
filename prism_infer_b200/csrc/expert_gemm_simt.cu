// Grouped SwiGLU experts in fp32 on CUDA cores (the fp32 block; bf16 runs on tcgen05).
//
// GEMM-1: per segment, h = silu(x Wg^T) * (x Wu^T)  — 64 x 32 output tile, gate and up tiles
//         computed side by side so the activation is applied in registers.
// GEMM-2: y = h Wd^T                                — 64 x 64 output tile.
// fp32 throughout with the reference's operation order inside an element (separate rounding of
// the product and the sum is not modelled: fp32 parity is checked with a tolerance).
#include "segments.cuh"

namespace prism {
namespace {

constexpr int kBM = 64, kBK = 16;

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// GEMM-1 (SwiGLU): grid (m-tile slots, ceil(I/32)); 256 threads; each thread 2 rows x 4 cols.
__global__ void __launch_bounds__(256)
    simt_gate_up_kernel(const float* __restrict__ x, int64_t rows_cap, int64_t H, int64_t I,
                        const int32_t* __restrict__ seg_offsets,
                        const int32_t* __restrict__ seg_expert, int nseg, int El,
                        const float* __restrict__ wgu, float* __restrict__ h) {
  constexpr int BN = 32;
  __shared__ int32_t prefix[kMaxSegments + 1];
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bg[kBK][BN + 4];
  __shared__ float Bu[kBK][BN + 4];
  if (threadIdx.x < 32) build_tile_prefix(seg_offsets, nseg, kBM, prefix);
  __syncthreads();
  const int32_t total = prefix[nseg];
  const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * BN;
  for (int32_t mt = blockIdx.x; mt < total; mt += gridDim.x) {
    const int s = find_segment(prefix, nseg, mt);
    const int e = seg_expert ? seg_expert[s] : s;
    if (e < 0 || e >= El) continue;  // segment names no local expert: rows left untouched
    const int64_t r0 = seg_offsets[s] + static_cast<int64_t>(mt - prefix[s]) * kBM;
    const int64_t r_end = seg_offsets[s + 1] < rows_cap ? seg_offsets[s + 1] : rows_cap;
    const float* wg = wgu + static_cast<int64_t>(e) * 2 * I * H;
    const float* wu = wg + I * H;
    float ag[2][4] = {}, au[2][4] = {};
    for (int64_t k0 = 0; k0 < H; k0 += kBK) {
      for (int i = tid; i < kBM * kBK; i += 256) {
        const int r = i / kBK, c = i % kBK;
        const int64_t gr = r0 + r, gk = k0 + c;
        As[c][r] = (gr < r_end && gk < H) ? x[gr * H + gk] : 0.f;
      }
      for (int i = tid; i < BN * kBK; i += 256) {
        const int r = i / kBK, c = i % kBK;
        const int64_t gn = n0 + r, gk = k0 + c;
        const bool ok = gn < I && gk < H;
        Bg[c][r] = ok ? wg[gn * H + gk] : 0.f;
        Bu[c][r] = ok ? wu[gn * H + gk] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) {
        float a[2], bg[4], bu[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) a[i] = As[kk][ty * 2 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          bg[j] = Bg[kk][tx * 4 + j];
          bu[j] = Bu[kk][tx * 4 + j];
        }
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            ag[i][j] = fmaf(a[i], bg[j], ag[i][j]);
            au[i][j] = fmaf(a[i], bu[j], au[i][j]);
          }
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int64_t gr = r0 + ty * 2 + i;
      if (gr >= r_end) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + tx * 4 + j;
        if (gn < I) h[gr * I + gn] = silu_f(ag[i][j]) * au[i][j];
      }
    }
  }
}

// GEMM-2: grid (m-tile slots, ceil(H/64)); each thread 4 rows x 4 cols.
__global__ void __launch_bounds__(256)
    simt_down_kernel(const float* __restrict__ h, int64_t rows_cap, int64_t H, int64_t I,
                     const int32_t* __restrict__ seg_offsets,
                     const int32_t* __restrict__ seg_expert, int nseg, int El,
                     const float* __restrict__ wd, float* __restrict__ y) {
  constexpr int BN = 64;
  __shared__ int32_t prefix[kMaxSegments + 1];
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs[kBK][BN + 4];
  if (threadIdx.x < 32) build_tile_prefix(seg_offsets, nseg, kBM, prefix);
  __syncthreads();
  const int32_t total = prefix[nseg];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * BN;
  for (int32_t mt = blockIdx.x; mt < total; mt += gridDim.x) {
    const int s = find_segment(prefix, nseg, mt);
    const int e = seg_expert ? seg_expert[s] : s;
    if (e < 0 || e >= El) continue;  // segment names no local expert: rows left untouched
    const int64_t r0 = seg_offsets[s] + static_cast<int64_t>(mt - prefix[s]) * kBM;
    const int64_t r_end = seg_offsets[s + 1] < rows_cap ? seg_offsets[s + 1] : rows_cap;
    const float* w = wd + static_cast<int64_t>(e) * H * I;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < I; k0 += kBK) {
      for (int i = tid; i < kBM * kBK; i += 256) {
        const int r = i / kBK, c = i % kBK;
        const int64_t gr = r0 + r, gk = k0 + c;
        As[c][r] = (gr < r_end && gk < I) ? h[gr * I + gk] : 0.f;
      }
      for (int i = tid; i < BN * kBK; i += 256) {
        const int r = i / kBK, c = i % kBK;
        const int64_t gn = n0 + r, gk = k0 + c;
        Bs[c][r] = (gn < H && gk < I) ? w[gn * I + gk] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gr = r0 + ty * 4 + i;
      if (gr >= r_end) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + tx * 4 + j;
        if (gn < H) y[gr * H + gn] = acc[i][j];
      }
    }
  }
}

}  // namespace

int expert_swiglu_f32(const float* x, int64_t rows_cap, int64_t H, int64_t I,
                      const int32_t* seg_offsets, const int32_t* seg_expert, int nseg, int El,
                      const float* wgu, const float* wd, float* y, float* h, cudaStream_t st) {
  PRISM_CHECK_ARG(nseg >= 1 && nseg <= kMaxSegments, "segments %d outside [1, %d]", nseg,
                  kMaxSegments);
  const int64_t slots = std::min<int64_t>(ceil_div(rows_cap, kBM) + nseg, 65535);
  const dim3 g1(static_cast<unsigned>(slots), static_cast<unsigned>(ceil_div(I, 32)));
  simt_gate_up_kernel<<<g1, 256, 0, st>>>(x, rows_cap, H, I, seg_offsets, seg_expert, nseg, El, wgu, h);
  PRISM_LAUNCH_CHECK("simt_gate_up_kernel launch");
  const dim3 g2(static_cast<unsigned>(slots), static_cast<unsigned>(ceil_div(H, 64)));
  simt_down_kernel<<<g2, 256, 0, st>>>(h, rows_cap, H, I, seg_offsets, seg_expert, nseg, El, wd, y);
  PRISM_LAUNCH_CHECK("simt_down_kernel launch");
  return PRISM_MOE_OK;
}

}  // namespace prism
