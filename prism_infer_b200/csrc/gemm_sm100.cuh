// Shared pieces of the sm_100a expert GEMM kernels (expert_gemm_sm100.cu: one launch per GEMM;
// expert_fused_sm100.cu: gate_up and down in one persistent launch): tile constants, shared
// memory budget, SwiGLU and bf16 conversion, and the staged epilogue of one accumulator tile.
#pragma once
#include <cudaTypedefs.h>

#include "internal.h"
#include "segments.cuh"

namespace prism {

// Encode a bf16 tensor map with 128-byte swizzle (expert_gemm_sm100.cu).
int encode_bf16_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* stride_bytes, const uint32_t* box);

namespace {

constexpr int kBK = 64;   // 64 bf16 = 128 bytes = one swizzle row
constexpr int kBN = 256;  // MMA N
constexpr int kThreads = 192;          // producer, MMA, 4 epilogue warps
constexpr int kDispatchThreads = 320;  // + 4 copy warps when the EP dispatch runs in the launch
constexpr uint32_t kTmemCols = 512;
constexpr int kStageRowBytes = 64 * 2 + 16;   // epilogue staging: 64 bf16 + 16 B pad per row
constexpr size_t kPrefixBytes = ((kMaxSegments + 1) * 4 + 15) / 16 * 16;

template <bool kPair>
struct Cfg {
  static constexpr int kRows = kPair ? 256 : 128;           // rows per tile
  static constexpr int kABytes = 128 * kBK * 2;              // this CTA's A rows
  static constexpr int kBBytes = (kPair ? 128 : 256) * kBK * 2;   // this CTA's B rows
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kPair ? 6 : 4;
  static constexpr uint32_t kTxBytes = (kPair ? 2 : 1) * kStageBytes;   // per full barrier
  static constexpr uint32_t kIdesc = idesc_bf16_f32(kRows, kBN);
  static constexpr size_t kStageOutOffset =
      static_cast<size_t>(kStages) * kStageBytes + 256 + kPrefixBytes;
  static constexpr size_t kSmemBytes = 1024 + kStageOutOffset + 4 * 32 * kStageRowBytes;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum : int { kGateUp = 0, kDown = 1 };

// Half tiles. A segment's last m-tile that holds at most 64 valid rows runs M=64 MMAs (half the
// tensor-core time of M=128; the TMA copy still brings 128 rows, of which the MMA reads the
// first 64). The single-CTA M=64 accumulator uses the first 16 TMEM lanes of each 32-lane
// quarter: tile row 16 q + i lives in lane 32 q + i (i < 16), column n in column n — CUTLASS's
// "half subpartitions" layout (cute/atom/mma_traits_sm100.hpp, UMMA_1SM M=64). An epilogue warp
// of quarter q therefore drains rows 16 q .. 16 q + 15 from its lanes 0..15.
constexpr int32_t kHalfRows = 64;
__device__ __forceinline__ bool half_tile(int32_t rows_valid) { return rows_valid <= kHalfRows; }
__device__ __forceinline__ int tile_row_of_lane(bool half, int q, int lane) {
  return half ? (lane < 16 ? q * 16 + lane : 1 << 30) : q * 32 + lane;
}

// Two fp32 values -> packed bf16x2 (round to nearest even) in one instruction; lo in bits 0-15.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// SwiGLU of one (gate, up) pair of fp32 accumulators: both rounded to bf16 first (the reference
// materialises gate_up in bf16), then silu(g) * u = g*u / (1 + e^-g) in fp32 with the fast
// exponential and reciprocal — the result is rounded to bf16, far coarser than their error.
__device__ __forceinline__ uint32_t swiglu_pair(uint32_t g0b, uint32_t g1b, uint32_t u0b,
                                                uint32_t u1b) {
  const uint32_t gp = cvt_bf16x2(__uint_as_float(g0b), __uint_as_float(g1b));
  const uint32_t up = cvt_bf16x2(__uint_as_float(u0b), __uint_as_float(u1b));
  const float g0 = __uint_as_float(gp << 16), g1 = __uint_as_float(gp & 0xffff0000u);
  const float u0 = __uint_as_float(up << 16), u1 = __uint_as_float(up & 0xffff0000u);
  const float s0 = __fdividef(g0 * u0, 1.0f + __expf(-g0));
  const float s1 = __fdividef(g1 * u1, 1.0f + __expf(-g1));
  return cvt_bf16x2(s0, s1);
}

// Epilogue of one 128-row tile for one warp (TMEM lane quarter of the calling warp): read the
// accumulator columns, convert (SwiGLU for gate_up: gate in columns [0,128), up in [128,256) of
// the accumulator; plain bf16 for down), stage 32 rows x 64 columns per pass in shared memory
// and write 128-byte row segments (8 lanes per row, 4 rows per instruction) — full NVLink /
// DRAM bursts instead of 32 scattered 16-byte pieces. ``my_ptr`` is this lane's output row
// address (0 = no row) and ``col_base`` the tile's first output column.
template <bool kSwiGLU>
__device__ __forceinline__ void drain_tile(uint32_t taddr, uint64_t my_ptr, uint8_t* stage_out,
                                           int lane, int64_t col_base, int64_t n_out) {
  constexpr int kPassCols = 64;
  constexpr int kOutCols = kSwiGLU ? 128 : kBN;
#pragma unroll 1
  for (int cc = 0; cc < kOutCols; cc += kPassCols) {
#pragma unroll 1
    for (int c = 0; c < kPassCols; c += 32) {   // 32 columns per tcgen05.wait::ld
      __syncwarp();
      uint32_t packed[16];
      if constexpr (kSwiGLU) {
        uint32_t g[32], u[32];
        tmem_ld16(taddr + cc + c, *reinterpret_cast<uint32_t(*)[16]>(&g[0]));
        tmem_ld16(taddr + cc + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&g[16]));
        tmem_ld16(taddr + 128 + cc + c, *reinterpret_cast<uint32_t(*)[16]>(&u[0]));
        tmem_ld16(taddr + 128 + cc + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&u[16]));
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = swiglu_pair(g[2 * i], g[2 * i + 1], u[2 * i], u[2 * i + 1]);
      } else {
        uint32_t v[32];
        tmem_ld16(taddr + cc + c, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
        tmem_ld16(taddr + cc + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = cvt_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
      }
      uint4* srow = reinterpret_cast<uint4*>(stage_out + lane * kStageRowBytes + c * 2);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4)
        srow[q4] = make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2],
                              packed[4 * q4 + 3]);
    }
    __syncwarp();
    const int seg = lane & 7;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = (lane >> 3) + 4 * j;
      const uint64_t p = __shfl_sync(0xffffffffu, my_ptr, r);
      const int64_t col = col_base + cc + seg * 8;
      if (p != 0 && col + 8 <= n_out)
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p) + col) =
            *reinterpret_cast<const uint4*>(stage_out + r * kStageRowBytes + seg * 16);
    }
  }
}

}  // namespace
}  // namespace prism
