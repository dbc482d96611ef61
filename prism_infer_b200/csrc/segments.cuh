// Segment -> tile mapping shared by the grouped expert GEMMs.
//
// A segment is a run of consecutive rows of the expert-major buffer that belongs to one expert
// (EP=1: one segment per expert; EP>1 receiver: one per (source rank, local expert)). The
// segment table lives on the device (it comes out of the dispatch plan), so the number of
// tiles is only known on the device: every CTA builds the prefix of m-tiles per segment in
// shared memory and maps its tile index back with a binary search.
#pragma once
#include "common.cuh"

namespace prism {

constexpr int kMaxSegments = 2048;

// Warp-cooperative: prefix[s] = first m-tile of segment s, prefix[nseg] = total m-tiles.
__device__ __forceinline__ void build_tile_prefix(const int32_t* __restrict__ seg_offsets,
                                                  int nseg, int bm, int32_t* prefix) {
  const int lane = threadIdx.x & 31;
  int32_t carry = 0;
  for (int base = 0; base < nseg; base += 32) {
    const int s = base + lane;
    int32_t n = 0;
    if (s < nseg) {
      const int32_t rows = seg_offsets[s + 1] - seg_offsets[s];
      n = rows > 0 ? (rows + bm - 1) / bm : 0;
    }
    int32_t incl = n;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += y;
    }
    if (s < nseg) prefix[s] = carry + incl - n;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) prefix[nseg] = carry;
}

// Largest s with prefix[s] <= mt (mt < prefix[nseg]).
__device__ __forceinline__ int find_segment(const int32_t* prefix, int nseg, int32_t mt) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= mt)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

}  // namespace prism
