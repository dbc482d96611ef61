// Kernel 4 — grouped SwiGLU expert GEMMs on 5th-generation tensor cores (bf16, sm_100a).
//
// Two persistent launches over a device-side segment table (rows of one expert per segment):
//   GATE_UP: per tile, D[128 x 256] = X[128 rows, H] * [Wg(128 rows); Wu(128 rows)]^T — the gate
//            and up halves of one 128-column slice of the intermediate dimension side by side in
//            one N=256 MMA; the epilogue computes h = silu(bf16(g)) * bf16(u) and stores bf16.
//   DOWN:    per tile, D[128 x 256] = H[128 rows, I] * Wd(256 rows)^T, stored as bf16.
// Warp roles (192 threads, one CTA per SM):
//   warp 0      TMA producer (one lane): A and B tiles, 4-stage ring of 48 KB stages;
//   warp 1      TMEM owner + MMA issuer (one lane): tcgen05.mma kind::f16, M=128 N=256 K=16,
//               fp32 accumulators in TMEM, two 256-column accumulators (512 columns) so the
//               epilogue of tile i overlaps the MMAs of tile i+1;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 16 columns, convert, 16-byte global stores.
// Operands are K-major with the 128-byte swizzle TMA writes. No multicast anywhere. Every wait
// is bounded; a wait that runs out records PRISM_MOE_ERR_TIMEOUT and the CTA drains its
// in-flight copies and MMAs before releasing TMEM.
#include <cudaTypedefs.h>

#include <mutex>

#include "internal.h"
#include "segments.cuh"

namespace prism {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;   // 64 bf16 = 128 bytes = one swizzle row
constexpr int kBN = 256;  // MMA N
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitNs = 2000000000ull;    // 2 s: far above any legitimate wait
constexpr uint64_t kDrainNs = 100000000ull;    // 100 ms
constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, kBN);
constexpr int kStageRowBytes = 64 * 2 + 16;   // epilogue staging: 64 bf16 + 16 B pad per row
constexpr size_t kPrefixBytes = ((kMaxSegments + 1) * 4 + 15) / 16 * 16;
constexpr size_t kStageOutOffset = static_cast<size_t>(kStages) * kStageBytes + 256 + kPrefixBytes;
constexpr size_t kSmemBytes = 1024 + kStageOutOffset + 4 * 32 * kStageRowBytes;
static_assert(kSmemBytes <= 232448, "shared memory budget");

enum : int { kGateUp = 0, kDown = 1 };

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmap_a,
                              const __grid_constant__ CUtensorMap tmap_b,
                              const int32_t* __restrict__ seg_offsets,
                              const int32_t* __restrict__ seg_expert, int nseg, int num_kb,
                              int num_n_tiles, int64_t n_out, uint16_t* __restrict__ out,
                              int64_t out_ld, int32_t rows_cap, int* __restrict__ err,
                              GemmOutput tgt) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* prefix = reinterpret_cast<int32_t*>(smem + kStages * kStageBytes + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2) build_tile_prefix(seg_offsets, nseg, kBM, prefix);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int64_t total_tiles = static_cast<int64_t>(prefix[nseg]) * num_n_tiles;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0;           // bit s: stage s has a load issued
    uint32_t issued_parity = 0;    // bit s: full-barrier parity of that load
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
      const int32_t mt = static_cast<int32_t>(tile / num_n_tiles);
      const int nt = static_cast<int>(tile % num_n_tiles);
      const int s = find_segment(prefix, nseg, mt);
      const int e = seg_expert ? seg_expert[s] : s;
      const int32_t row0 = seg_offsets[s] + (mt - prefix[s]) * kBM;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort, kWaitNs)) {
          ok = false;
          break;
        }
        uint8_t* sa = stages + stage * kStageBytes;
        uint8_t* sb = sa + kABytes;
        mbar_arrive_expect_tx(&full[stage], kStageBytes);
        tma_load_2d(sa, &tmap_a, &full[stage], kb * kBK, row0);
        if constexpr (kMode == kGateUp) {
          tma_load_4d(sb, &tmap_b, &full[stage], kb * kBK, nt * 128, 0, e);
          tma_load_4d(sb + kBBytes / 2, &tmap_b, &full[stage], kb * kBK, nt * 128, 1, e);
        } else {
          tma_load_3d(sb, &tmap_b, &full[stage], kb * kBK, nt * kBN, e);
        }
        issued |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (!ok) {
      *abort = 1;
      record_device_error(err, PRISM_MOE_ERR_TIMEOUT);
    }
    if (*abort) {
      // let every copy this thread issued land before the CTA can exit
      for (int s = 0; s < kStages; ++s)
        if ((issued >> s) & 1u) {
          volatile int never = 0;
          mbar_wait_bounded(&full[s], (issued_parity >> s) & 1u, &never, kDrainNs);
        }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_bounded(&acc_empty[buf], acc_phase ^ 1, abort, kWaitNs)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * kBN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort, kWaitNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(stages + stage * kStageBytes);
        const uint32_t b0 = a0 + kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          tc_mma_bf16(d_tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                      kIdesc, (kb | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      tc_commit(&acc_full[buf]);
    }
    if (!ok) {
      *abort = 1;
      record_device_error(err, PRISM_MOE_ERR_TIMEOUT);
    }
    if (*abort) {
      tc_commit(drain);   // completes once every MMA issued above has finished
      volatile int never = 0;
      mbar_wait_bounded(drain, 0, &never, kDrainNs);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    uint8_t* stage_out = smem + kStageOutOffset + (warp - 2) * 32 * kStageRowBytes;
    int it = 0;
    for (int64_t tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int32_t mt = static_cast<int32_t>(tile / num_n_tiles);
      const int nt = static_cast<int>(tile % num_n_tiles);
      const int s = find_segment(prefix, nseg, mt);
      const int32_t row0 = seg_offsets[s] + (mt - prefix[s]) * kBM;
      const int32_t seg_end = seg_offsets[s + 1];
      const int32_t rows_valid = (seg_end < rows_cap ? seg_end : rows_cap) - row0;
      if (!mbar_wait_bounded(&acc_full[buf], acc_phase, abort, kWaitNs)) {
        *abort = 1;
        record_device_error(err, PRISM_MOE_ERR_TIMEOUT);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * kBN;
      // this lane's output row address (0 = no row): dense, or per-row (e.g. a peer GPU)
      uint64_t my_ptr = 0;
      if (row_in_tile < rows_valid)
        my_ptr = tgt.row_ptr ? tgt.row_ptr[row0 + row_in_tile]
                             : reinterpret_cast<uint64_t>(
                                   out + static_cast<int64_t>(row0 + row_in_tile) * out_ld);
      // Each pass stages 32 rows x 64 columns in shared memory, then the warp writes 128-byte
      // row segments (8 lanes per row, 4 rows per instruction) — full NVLink / DRAM bursts
      // instead of 32 scattered 16-byte pieces.
      constexpr int kPassCols = 64;
      constexpr int kOutCols = kMode == kGateUp ? 128 : kBN;
#pragma unroll 1
      for (int cc = 0; cc < kOutCols; cc += kPassCols) {
#pragma unroll 1
        for (int c = 0; c < kPassCols; c += 16) {
          __syncwarp();
          uint32_t packed[8];
          if constexpr (kMode == kGateUp) {
            uint32_t g[16], u[16];
            tmem_ld16(taddr + cc + c, g);
            tmem_ld16(taddr + 128 + cc + c, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float g0 = round_bf16(__uint_as_float(g[2 * i]));
              const float g1 = round_bf16(__uint_as_float(g[2 * i + 1]));
              const float u0 = round_bf16(__uint_as_float(u[2 * i]));
              const float u1 = round_bf16(__uint_as_float(u[2 * i + 1]));
              packed[i] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
            }
          } else {
            uint32_t v[16];
            tmem_ld16(taddr + cc + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i)
              packed[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          }
          uint4* srow = reinterpret_cast<uint4*>(stage_out + lane * kStageRowBytes + c * 2);
          srow[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          srow[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
        __syncwarp();
        const int64_t col_base = static_cast<int64_t>(nt) * kOutCols + cc;
        const int seg = lane & 7;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int r = (lane >> 3) + 4 * j;
          const uint64_t p = __shfl_sync(0xffffffffu, my_ptr, r);
          const int64_t col = col_base + seg * 8;
          if (p != 0 && col + 8 <= n_out)
            *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p) + col) =
                *reinterpret_cast<const uint4*>(stage_out + r * kStageRowBytes + seg * 16);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  if (tgt.done_counter != nullptr && warp >= 2) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  // completion signal: the last CTA to get here publishes `epoch` to every flag
  if (tgt.done_counter != nullptr && threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(tgt.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      *tgt.done_counter = 0u;  // ready for the next launch (stream-ordered)
      __threadfence_system();
      for (int i = 0; i < tgt.num_signal; ++i) store_release_sys(tgt.signal_flags[i], tgt.epoch);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_bf16_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* stride_bytes, const uint32_t* box) {
  auto enc = tensor_map_encoder();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return PRISM_MOE_ERR_CUDA;
  }
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = stride_bytes[i];
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d,
                         s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d, rank %d)", static_cast<int>(r), rank);
    return PRISM_MOE_ERR_CUDA;
  }
  return PRISM_MOE_OK;
}

template <int kMode>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const int32_t* seg_offsets,
                const int32_t* seg_expert, int nseg, int64_t rows_cap, int64_t K, int64_t n_out,
                uint16_t* out, int* err, const GemmOutput& tgt, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr_status = cudaSuccess;
  std::call_once(once, [] {
    attr_status = cudaFuncSetAttribute(grouped_gemm_sm100_kernel<kMode>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kSmemBytes));
  });
  PRISM_CUDA(attr_status);
  const int n_tile = kMode == kGateUp ? 128 : kBN;
  const int num_n_tiles = static_cast<int>(ceil_div(n_out, n_tile));
  const int num_kb = static_cast<int>(ceil_div(K, kBK));
  const int64_t max_tiles = (ceil_div(rows_cap, kBM) + nseg) * num_n_tiles;
  const int grid = static_cast<int>(std::min<int64_t>(num_sms(), std::max<int64_t>(max_tiles, 1)));
  grouped_gemm_sm100_kernel<kMode><<<grid, kThreads, kSmemBytes, st>>>(
      ma, mb, seg_offsets, seg_expert, nseg, num_kb, num_n_tiles, n_out, out, n_out,
      static_cast<int32_t>(rows_cap), err, tgt);
  PRISM_LAUNCH_CHECK("grouped_gemm_sm100_kernel launch");
  return PRISM_MOE_OK;
}

}  // namespace

int expert_swiglu_bf16(const void* xs, int64_t rows_cap, int64_t H, int64_t I,
                       const int32_t* seg_offsets, const int32_t* seg_expert, int nseg, int El,
                       const void* wgu, const void* wd, void* y, void* h, int* err,
                       cudaStream_t st, const GemmOutput* down_out) {
  const GemmOutput dense{};
  const GemmOutput& down_tgt = down_out ? *down_out : dense;
  PRISM_CHECK_ARG(H % 8 == 0 && I % 8 == 0, "bf16 experts need hidden %% 8 == 0 and inter %% 8 == 0");
  PRISM_CHECK_ARG(nseg >= 1 && nseg <= kMaxSegments, "segments %d outside [1, %d]", nseg,
                  kMaxSegments);
  PRISM_CHECK_ARG(rows_cap < (int64_t(1) << 31), "rows_capacity too large");
  PRISM_CHECK_ARG((reinterpret_cast<uintptr_t>(xs) | reinterpret_cast<uintptr_t>(wgu) |
                   reinterpret_cast<uintptr_t>(wd) | reinterpret_cast<uintptr_t>(y) |
                   reinterpret_cast<uintptr_t>(h)) % 16 == 0,
                  "bf16 expert operands must be 16-byte aligned");
  if (rows_cap == 0) return PRISM_MOE_OK;
  CUtensorMap a1, b1, a2, b2;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(H), static_cast<uint64_t>(rows_cap)};
    const uint64_t strides[1] = {static_cast<uint64_t>(H) * 2};
    const uint32_t box[2] = {kBK, kBM};
    int r = encode_bf16_map(&a1, xs, 2, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(H), static_cast<uint64_t>(I), 2,
                              static_cast<uint64_t>(El)};
    const uint64_t strides[3] = {static_cast<uint64_t>(H) * 2, static_cast<uint64_t>(I * H) * 2,
                                 static_cast<uint64_t>(2 * I * H) * 2};
    const uint32_t box[4] = {kBK, 128, 1, 1};
    int r = encode_bf16_map(&b1, wgu, 4, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(I), static_cast<uint64_t>(rows_cap)};
    const uint64_t strides[1] = {static_cast<uint64_t>(I) * 2};
    const uint32_t box[2] = {kBK, kBM};
    int r = encode_bf16_map(&a2, h, 2, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(I), static_cast<uint64_t>(H),
                              static_cast<uint64_t>(El)};
    const uint64_t strides[2] = {static_cast<uint64_t>(I) * 2, static_cast<uint64_t>(H * I) * 2};
    const uint32_t box[3] = {kBK, kBN, 1};
    int r = encode_bf16_map(&b2, wd, 3, dims, strides, box);
    if (r) return r;
  }
  record_stage(3, st);
  int r = launch_gemm<kGateUp>(a1, b1, seg_offsets, seg_expert, nseg, rows_cap, H, I,
                               static_cast<uint16_t*>(h), err, dense, st);
  if (r) return r;
  record_stage(4, st);
  r = launch_gemm<kDown>(a2, b2, seg_offsets, seg_expert, nseg, rows_cap, I, H,
                         static_cast<uint16_t*>(y), err, down_tgt, st);
  record_stage(5, st);
  return r;
}

}  // namespace prism
