// Kernel 4 — grouped SwiGLU expert GEMMs on 5th-generation tensor cores (bf16, sm_100a).
//
// Two persistent launches over a device-side segment table (rows of one expert per segment):
//   GATE_UP: per tile, D[rows x 256] = X[rows, H] * [Wg(128 rows); Wu(128 rows)]^T — the gate and
//            up halves of one 128-column slice of the intermediate dimension side by side in one
//            N=256 MMA; the epilogue computes h = silu(bf16(g)) * bf16(u) and stores bf16.
//   DOWN:    per tile, D[rows x 256] = H[rows, I] * Wd(256 rows)^T, stored as bf16.
// Two tile engines, same code:
//   single  (kPair=false): one CTA per tile of 128 rows; MMA M=128, N=256, K=16; stage =
//           A 16 KB + B 32 KB, 4 stages.
//   pair    (kPair=true):  a cluster of two CTAs on two SMs per tile of 256 rows; the even CTA
//           issues tcgen05.mma.cta_group::2 (M=256 across both SMs, N=256): each CTA stages its
//           own 128 A rows and HALF of B (GATE_UP: gate rows in CTA 0, up rows in CTA 1; DOWN:
//           output columns 0-127 / 128-255), 32 KB per stage, 6 stages — a third less shared
//           memory traffic per FLOP than the single engine. Both CTAs' TMA completions count on
//           the even CTA's barrier; MMA completions are committed to both CTAs' barriers; each CTA
//           drains its own 128 accumulator rows from its TMEM.
// Warp roles (192 threads, one CTA per SM):
//   warp 0      TMA producer (one lane);
//   warp 1      TMEM owner + MMA issuer (one lane; in a pair only the even CTA issues), fp32
//               accumulators in TMEM, two 256-column accumulators (512 columns) so the epilogue
//               of tile i overlaps the MMAs of tile i+1;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 16 columns, convert, stage 64 columns per row in
//               shared memory, store 128-byte row segments (dense, or per-row addresses that may
//               point into a peer GPU's memory).
// Operands are K-major with the 128-byte swizzle TMA writes; no TMA multicast. Every wait is
// bounded; a wait that runs out records PRISM_MOE_ERR_TIMEOUT and the CTA drains its in-flight
// copies and MMAs before releasing TMEM.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemm_sm100.cuh"

namespace prism {
namespace {

// Where a tile's operands start: n-tile, expert, first row of this CTA's 128 rows (before
// finish(): the segment's first row, and the tile's index within the segment).
struct TileLoc {
  int nt = 0;
  int e = 0;
  int32_t row0 = 0;
  int32_t mt_in_seg = 0;
};

template <int kMode, bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmap_a,
                              const __grid_constant__ CUtensorMap tmap_b,
                              const int32_t* __restrict__ seg_offsets,
                              const int32_t* __restrict__ seg_expert, int nseg, int num_kb,
                              int num_n_tiles, int64_t n_out, uint16_t* __restrict__ out,
                              int64_t out_ld, int32_t rows_cap, int* __restrict__ err,
                              GemmOutput tgt, uint64_t kWaitNs) {
  using C = Cfg<kPair>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* prefix = reinterpret_cast<int32_t*>(smem + C::kStages * C::kStageBytes + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;     // position in the CTA pair
  const bool leader = rank == 0;
  const int64_t unit = kPair ? blockIdx.x / 2 : blockIdx.x;   // tile-scheduling unit
  const int64_t num_units = kPair ? gridDim.x / 2 : gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kPair ? 256 : 128);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  if (warp == 2) build_tile_prefix(seg_offsets, nseg, C::kRows, prefix);
  tc_fence_before();
  if constexpr (kPair)
    cluster_sync();   // both CTAs' barriers initialised before any cross-CTA arrival
  else
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
    // A tile's first row and expert are looked up one tile ahead: the segment search and the
    // table loads are issued after the first k-block of the tile before it and their values
    // used only after that tile's last k-block, so the loads overlap copies in flight instead
    // of holding back the next tile's first copy.
    auto lookup = [&](int64_t tile) {
      TileLoc l;
      const int32_t mt = static_cast<int32_t>(tile / num_n_tiles);
      const int s = find_segment(prefix, nseg, mt);
      l.nt = static_cast<int>(tile % num_n_tiles);
      l.e = s;
      if (seg_expert) l.e = seg_expert[s];
      l.row0 = seg_offsets[s];                          // + the tile's offset, in finish()
      l.mt_in_seg = mt - prefix[s];
      return l;
    };
    auto finish = [&](TileLoc l) {
      l.row0 += l.mt_in_seg * C::kRows + 128 * static_cast<int32_t>(rank);
      return l;
    };
    TileLoc cur;
    if (unit < total_tiles) cur = finish(lookup(unit));
    for (int64_t tile = unit; ok && tile < total_tiles; tile += num_units) {
      const int nt = cur.nt, e = cur.e;
      const int32_t row0 = cur.row0;
      TileLoc nxt = cur;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort, kWaitNs)) {
          ok = false;
          break;
        }
        uint8_t* sa = stages + stage * C::kStageBytes;
        uint8_t* sb = sa + C::kABytes;
        if (leader) mbar_arrive_expect_tx(&full[stage], C::kTxBytes);
        if constexpr (kPair) {
          tma_load_2d_pair(sa, &tmap_a, &full[stage], kb * kBK, row0);
          if constexpr (kMode == kGateUp)
            tma_load_4d_pair(sb, &tmap_b, &full[stage], kb * kBK, nt * 128,
                             static_cast<int32_t>(rank), e);
          else
            tma_load_3d_pair(sb, &tmap_b, &full[stage], kb * kBK,
                             nt * kBN + 128 * static_cast<int32_t>(rank), e);
        } else {
          tma_load_2d(sa, &tmap_a, &full[stage], kb * kBK, row0);
          if constexpr (kMode == kGateUp) {
            // gate rows then up rows of n-tile nt in one copy (box spans both halves)
            tma_load_4d(sb, &tmap_b, &full[stage], kb * kBK, nt * 128, 0, e);
          } else {
            tma_load_3d(sb, &tmap_b, &full[stage], kb * kBK, nt * kBN, e);
          }
        }
        issued |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
        if (kb == 0 && tile + num_units < total_tiles) nxt = lookup(tile + num_units);
      }
      cur = finish(nxt);
    }
    if (!ok) {
      *abort = 1;
      record_device_error(err, PRISM_MOE_ERR_TIMEOUT);
    }
    if (*abort && leader) {
      // let every copy of the pair land before either CTA can exit (the even CTA's full
      // barriers count both CTAs' bytes)
      for (int s = 0; s < C::kStages; ++s)
        if ((issued >> s) & 1u) {
          volatile int never = 0;
          mbar_wait_bounded(&full[s], (issued_parity >> s) & 1u, &never, kDrainNs);
        }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ------------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    // A segment's last m-tile with <= 64 rows runs M=64 MMAs. The segment of the next tile is
    // looked up after the first k-block of this one and the decision taken after its last, so
    // the table loads do not delay a tile's first MMA. (x, y, z) = (segment start, segment
    // end, the tile's first row within the segment).
    auto lookup = [&](int64_t tile) -> int3 {
      const int32_t mt = static_cast<int32_t>(tile / num_n_tiles);
      const int s = find_segment(prefix, nseg, mt);
      return make_int3(seg_offsets[s], seg_offsets[s + 1], (mt - prefix[s]) * C::kRows);
    };
    auto tile_idesc = [&](int3 r) -> uint32_t {
      if constexpr (kPair) {
        return C::kIdesc;
      } else {
        return half_tile((r.y < rows_cap ? r.y : rows_cap) - (r.x + r.z))
                   ? idesc_bf16_f32(kHalfRows, kBN)
                   : C::kIdesc;
      }
    };
    uint32_t idesc = C::kIdesc;
    if (!kPair && unit < total_tiles) idesc = tile_idesc(lookup(unit));
    for (int64_t tile = unit; ok && tile < total_tiles; tile += num_units, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_bounded(&acc_empty[buf], acc_phase ^ 1, abort, kWaitNs)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * kBN;
      int3 next = make_int3(0, 0, 0);
      const bool has_next = !kPair && tile + num_units < total_tiles;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort, kWaitNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(stages + stage * C::kStageBytes);
        const uint32_t b0 = a0 + C::kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(a0 + kk * 32), bd = smem_desc_sw128(b0 + kk * 32);
          const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
          if constexpr (kPair)
            tc_mma_bf16_pair(d_tmem, ad, bd, C::kIdesc, acc);
          else
            tc_mma_bf16(d_tmem, ad, bd, idesc, acc);
        }
        if constexpr (kPair)
          tc_commit_pair(&empty[stage], 0x3);
        else
          tc_commit(&empty[stage]);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
        if (kb == 0 && has_next) next = lookup(tile + num_units);
      }
      if (!ok) break;
      if constexpr (kPair)
        tc_commit_pair(&acc_full[buf], 0x3);
      else
        tc_commit(&acc_full[buf]);
      if (has_next) idesc = tile_idesc(next);
    }
    if (!ok) {
      *abort = 1;
      record_device_error(err, PRISM_MOE_ERR_TIMEOUT);
    }
    if (*abort) {
      if constexpr (kPair)
        tc_commit_pair(drain, 0x1);
      else
        tc_commit(drain);   // completes once every MMA issued above has finished
      volatile int never = 0;
      mbar_wait_bounded(drain, 0, &never, kDrainNs);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    uint8_t* stage_out = smem + C::kStageOutOffset + (warp - 2) * 32 * kStageRowBytes;
    const uint32_t acc_empty_leader =
        kPair ? mapa_shared(smem_u32(&acc_empty[0]), 0) : smem_u32(&acc_empty[0]);
    int it = 0;
    for (int64_t tile = unit; tile < total_tiles; tile += num_units, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int32_t mt = static_cast<int32_t>(tile / num_n_tiles);
      const int nt = static_cast<int>(tile % num_n_tiles);
      const int s = find_segment(prefix, nseg, mt);
      const int32_t row0 = seg_offsets[s] + (mt - prefix[s]) * C::kRows + 128 * rank;
      const int32_t seg_end = seg_offsets[s + 1];
      const int32_t rows_valid = (seg_end < rows_cap ? seg_end : rows_cap) - row0;
      // row within this CTA's 128 rows held by this lane (half tiles: lanes 0-15 of a quarter)
      const int row_in_tile = tile_row_of_lane(!kPair && half_tile(rows_valid), q, lane);
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
        my_ptr = tgt.seg_base
                     ? tgt.seg_base[s] + static_cast<uint64_t>(
                                             (row0 + row_in_tile - seg_offsets[s]) * out_ld * 2)
                     : reinterpret_cast<uint64_t>(
                           out + static_cast<int64_t>(row0 + row_in_tile) * out_ld);
      drain_tile<kMode == kGateUp>(taddr, my_ptr, stage_out, lane,
                                   static_cast<int64_t>(nt) * (kMode == kGateUp ? 128 : kBN),
                                   n_out);
      tc_fence_before();
      if constexpr (kPair)
        mbar_arrive_cluster(acc_empty_leader + buf * 8);
      else
        mbar_arrive(&acc_empty[buf]);
    }
  }

  if (tgt.done_counter != nullptr && warp >= 2) threadfence_scoped(tgt.remote);
  tc_fence_before();
  if constexpr (kPair)
    cluster_sync();   // neither CTA leaves while its partner may still use its TMEM / smem
  else
    __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
  // completion signal: the last CTA to get here publishes `epoch` to every flag
  if (tgt.done_counter != nullptr && threadIdx.x == 0) {
    threadfence_scoped(tgt.remote);
    const unsigned int prev = atomicAdd(tgt.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      *tgt.done_counter = 0u;  // ready for the next launch (stream-ordered)
      threadfence_scoped(tgt.remote);
      const uint64_t ep = tgt.epoch_ptr ? *tgt.epoch_ptr : tgt.epoch;
      for (int i = 0; i < tgt.num_signal; ++i)
        store_release_scoped(tgt.signal_flags[i], ep, tgt.remote);
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

}  // namespace

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

namespace {

template <int kMode, bool kPair>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const int32_t* seg_offsets,
                const int32_t* seg_expert, int nseg, int64_t rows_cap, int64_t K, int64_t n_out,
                uint16_t* out, int* err, const GemmOutput& tgt, cudaStream_t st) {
  using C = Cfg<kPair>;
  auto kern = grouped_gemm_sm100_kernel<kMode, kPair>;
  constexpr int threads = kThreads;
  if (int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), static_cast<int>(C::kSmemBytes)))
    return r;
  // resident scheduling units (CTAs, or CTA pairs) per device, looked up once per device
  static std::mutex units_mu;
  static int units_of_dev[64] = {};
  int dev = 0;
  PRISM_CUDA(cudaGetDevice(&dev));
  int max_units = 0;
  {
    std::lock_guard<std::mutex> lock(units_mu);
    max_units = dev >= 0 && dev < 64 ? units_of_dev[dev] : 0;
  }
  if (max_units == 0) {
    max_units = num_sms();
    if (kPair) {
      // how many CTA pairs can be resident at once
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
      cfg.blockDim = dim3(threads, 1, 1);
      cfg.dynamicSmemBytes = C::kSmemBytes;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters > 0)
        max_units = clusters;
      else
        max_units = num_sms() / 2;
      cudaGetLastError();
    }
    std::lock_guard<std::mutex> lock(units_mu);
    if (dev >= 0 && dev < 64) units_of_dev[dev] = max_units;
  }
  const int n_tile = kMode == kGateUp ? 128 : kBN;
  const int num_n_tiles = static_cast<int>(ceil_div(n_out, n_tile));
  const int num_kb = static_cast<int>(ceil_div(K, kBK));
  const int64_t max_tiles = (ceil_div(rows_cap, C::kRows) + nseg) * num_n_tiles;
  const int units =
      static_cast<int>(std::min<int64_t>(max_units, std::max<int64_t>(max_tiles, 1)));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(static_cast<unsigned>(units * (kPair ? 2 : 1)), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  if (kPair) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  PRISM_CUDA(cudaLaunchKernelEx(&cfg, kern, ma, mb, seg_offsets, seg_expert, nseg, num_kb,
                                num_n_tiles, n_out, out, n_out, static_cast<int32_t>(rows_cap),
                                err, tgt, wait_limit_ns()));
  return PRISM_MOE_OK;
}

enum class Engine { kFused, kSingle, kPair };

// Pair tiles (256 rows) pay off once segments are long: tail tiles waste up to 255 rows per
// segment, single tiles up to 127. A dispatching step runs both GEMMs as one fused launch
// (expert_fused_sm100.cu), so that the dispatch and the down GEMM's stores into peers overlap
// tensor-core work; so does a step whose segments average under one m-tile (decode: the
// launch boundary between the GEMMs would idle the GPU while each weight stream runs once,
// measured 7% slower at 64 tokens). prism_moe_set_expert_engine overrides the choice for steps
// without a dispatch (single = two launches with 128-row tiles).
Engine pick_engine(int64_t rows_cap, int nseg, bool dispatch) {
  const int force = expert_engine_setting();
  if (dispatch || force == PRISM_MOE_ENGINE_FUSED) return Engine::kFused;
  if (force == PRISM_MOE_ENGINE_SINGLE) return Engine::kSingle;
  if (force == PRISM_MOE_ENGINE_PAIR) return Engine::kPair;
  const int64_t per_seg = rows_cap / std::max(nseg, 1);
  if (per_seg < 128) return Engine::kFused;
  return per_seg >= 2048 ? Engine::kPair : Engine::kSingle;
}

}  // namespace

int expert_swiglu_bf16(const void* xs, int64_t rows_cap, int64_t H, int64_t I,
                       const int32_t* seg_offsets, const int32_t* seg_expert, int nseg, int El,
                       const void* wgu, const void* wd, void* y, void* h, int* err,
                       cudaStream_t st, const GemmOutput* down_out,
                       const GemmDispatch* dispatch) {
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
  const Engine engine = pick_engine(rows_cap, nseg, dispatch != nullptr);
  if (engine == Engine::kFused) {
    record_stage(3, st);
    int r = expert_swiglu_fused(xs, rows_cap, H, I, seg_offsets, seg_expert, nseg, El, wgu, wd,
                                y, h, fused_sync(h, rows_cap, I), err, st, down_out, dispatch);
    record_stage(4, st);   // one launch: slot 3 -> 4 covers both GEMMs, 4 -> 5 is empty
    record_stage(5, st);
    return r;
  }
  const bool pair = engine == Engine::kPair;
  CUtensorMap a1, b1, a2, b2;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(H), static_cast<uint64_t>(rows_cap)};
    const uint64_t strides[1] = {static_cast<uint64_t>(H) * 2};
    const uint32_t box[2] = {kBK, 128};
    int r = encode_bf16_map(&a1, xs, 2, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(H), static_cast<uint64_t>(I), 2,
                              static_cast<uint64_t>(El)};
    const uint64_t strides[3] = {static_cast<uint64_t>(H) * 2, static_cast<uint64_t>(I * H) * 2,
                                 static_cast<uint64_t>(2 * I * H) * 2};
    // single tiles take both halves (gate, up) of an n-tile per copy; a pair CTA one half
    const uint32_t box[4] = {kBK, 128, pair ? 1u : 2u, 1};
    int r = encode_bf16_map(&b1, wgu, 4, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(I), static_cast<uint64_t>(rows_cap)};
    const uint64_t strides[1] = {static_cast<uint64_t>(I) * 2};
    const uint32_t box[2] = {kBK, 128};
    int r = encode_bf16_map(&a2, h, 2, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(I), static_cast<uint64_t>(H),
                              static_cast<uint64_t>(El)};
    const uint64_t strides[2] = {static_cast<uint64_t>(I) * 2, static_cast<uint64_t>(H * I) * 2};
    const uint32_t box[3] = {kBK, static_cast<uint32_t>(pair ? 128 : kBN), 1};
    int r = encode_bf16_map(&b2, wd, 3, dims, strides, box);
    if (r) return r;
  }
  record_stage(3, st);
  int r = pair ? launch_gemm<kGateUp, true>(a1, b1, seg_offsets, seg_expert, nseg, rows_cap,
                                                H, I, static_cast<uint16_t*>(h), err, dense, st)
                   : launch_gemm<kGateUp, false>(a1, b1, seg_offsets, seg_expert, nseg, rows_cap,
                                                 H, I, static_cast<uint16_t*>(h), err, dense, st);
  if (r) return r;
  record_stage(4, st);
  r = pair ? launch_gemm<kDown, true>(a2, b2, seg_offsets, seg_expert, nseg, rows_cap, I, H,
                                      static_cast<uint16_t*>(y), err, down_tgt, st)
           : launch_gemm<kDown, false>(a2, b2, seg_offsets, seg_expert, nseg, rows_cap, I, H,
                                       static_cast<uint16_t*>(y), err, down_tgt, st);
  record_stage(5, st);
  return r;
}

}  // namespace prism
