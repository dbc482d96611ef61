// Kernel 4b — both grouped SwiGLU expert GEMMs in ONE persistent launch (bf16, sm_100a).
//
// The gate_up and down GEMMs of expert_gemm_sm100.cu (same tiles: MMA M=128, N=256, K=16,
// 4 stages of A 16 KB + B 32 KB, two 256-column fp32 accumulators in TMEM) run as one tile
// stream that every CTA's producer claims from a global counter:
//   gate_up tile (mt, nt): h[rows of m-tile mt, 128 columns nt] = silu(x Wg^T) * (x Wu^T)
//   down tile    (mt, nt): y[rows of m-tile mt, 256 columns nt] = h Wd^T
// The stream interleaves the two kinds: after the gate_up tiles of the first L m-tiles, each
// step emits the gate_up tiles of m-tile r and the down tiles of m-tile r - L, so a down tile
// is claimed L steps (several hundred tiles) after the gate_up tiles it reads. Each gate_up
// epilogue warp publishes its stored h rows on a per-m-tile counter (release, GPU scope); the
// producer of a down tile waits (bounded) for that counter before its TMA reads h. Tiles are
// claimed in stream order by CTAs that are running and every dependency points to an earlier
// claim, so the launch makes progress even when the GPU holds fewer CTAs than the grid.
//
// With expert parallelism (``GemmDispatch``) four more warps per CTA fill this rank's receive
// buffer inside the same launch, in chunks claimed from a shared counter: first this rank's own
// rows (expert-major, published per expert segment), then, source by source, the rows other
// ranks routed here, PULLED over NVLink from the sources' landing zones one token row per
// (token, rank) however many of this rank's experts the token chose (the de-duplicated
// dispatch); every count lands on a counter in this GPU's memory at GPU scope, and the producer
// of a gate_up tile waits for the counter of its segment. The down epilogue stores every output
// row straight into its source rank's buffer (GemmOutput::seg_base, 128-byte segments over
// NVLink), so both transfers overlap tensor-core work. (Forwarding the outputs through the copy
// warps instead, staged in local memory, measured slower at 2 and 4 GPUs.)
//
// Warp roles: warp 0 lane 0 claims tiles, publishes each to a shared-memory ring (8 entries,
// full/empty mbarriers) and issues the TMA loads; warp 1 lane 0 issues the MMAs; warps 2..5
// drain the accumulators; warps 6..9 (expert parallelism only) copy rows. Every wait is bounded.
// The measured comparison with two launches (expert_gemm_sm100.cu): on one GPU the two
// launches are faster (every CTA works on one weight stream at a time), with an exchange the
// fused launch is.
#include <algorithm>

#include "gemm_sm100.cuh"

namespace prism {
namespace {

struct FusedCfg {
  static constexpr int kStages = 4;
  static constexpr int kABytes = 128 * kBK * 2;
  static constexpr int kBBytes = kBN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTxBytes = kStageBytes;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, kBN);
  static constexpr int kRing = 8;
  static constexpr size_t kBarOffset = static_cast<size_t>(kStages) * kStageBytes;
  static constexpr size_t kBarBytes = 512;
  static constexpr size_t kPrefixOffset = kBarOffset + kBarBytes;
  static constexpr size_t kStageOutOffset = kPrefixOffset + kPrefixBytes;
  static constexpr size_t kSmemBytes = 1024 + kStageOutOffset + 4 * 32 * kStageRowBytes;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  // full, empty, acc_full, acc_empty, ring_full, ring_empty, drain + ring, tmem slot, abort
  static_assert((2 * kStages + 4 + 2 * kRing + 1) * 8 + kRing * 4 + 8 <= kBarBytes,
                "barrier area");
};

struct FusedParams {
  const int32_t* seg_offsets = nullptr;
  const int32_t* seg_expert = nullptr;
  int nseg = 0;
  int32_t rows_cap = 0;
  int n_gu = 0;    // gate_up n-tiles: ceil(I / 128)
  int n_dn = 0;    // down n-tiles: ceil(H / 256)
  int kb_gu = 0;   // gate_up k-blocks: ceil(H / 64)
  int kb_dn = 0;   // down k-blocks: ceil(I / 64)
  int lag = 1;     // L, in m-tiles
  int64_t H = 0, I = 0;
  uint64_t wait_ns = 0;        // bound of every wait on this GPU's own pipeline
  uint64_t peer_wait_ns = 0;   // bound of a wait for rows from other ranks
  uint16_t* h = nullptr;               // [rows_cap, I]
  uint16_t* y = nullptr;               // [rows_cap, H] unless the output has seg_base
  unsigned int* claim = nullptr;       // tile claim counter, zero at launch
  unsigned int* h_ready = nullptr;     // per m-tile: gate_up epilogue warps done, zero at launch
  int* err = nullptr;
};

struct TileRef {
  int kind;     // 0 gate_up, 1 down
  int32_t mt;
  int nt;
};

// Position c of the interleaved tile stream over M m-tiles.
__device__ __forceinline__ TileRef tile_at(int32_t c, int32_t M, int nG, int nD, int L) {
  const int32_t A = M < L ? M : L;
  if (c < nG * A) return {0, c / nG, c % nG};
  c -= nG * A;
  const int per = nG + nD;
  const int32_t mid = M > L ? M - L : 0;
  if (c < per * mid) {
    const int32_t r = L + c / per;
    const int o = c % per;
    return o < nG ? TileRef{0, r, o} : TileRef{1, r - L, o - nG};
  }
  c -= per * mid;
  const int32_t first = M > L ? M - L : 0;
  return {1, first + c / nD, c % nD};
}

__device__ __forceinline__ uint32_t load_acquire_gpu(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void add_release_gpu(unsigned int* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---------------------------------------------------------------------------------------------
// copy warps (expert parallelism)
// ---------------------------------------------------------------------------------------------
// Rows per own-slot chunk (one lane looks up each row).
constexpr int kChunkRows = 32;

// Add ``n`` to this GPU's arrival counter ``ctr``: the warp barrier orders every lane's row stores
// before lane 0's release add (cumulative, GPU scope: writer and reader are both on this GPU).
__device__ __forceinline__ void arrival_add(const GemmDispatch& D, int ctr, unsigned int n,
                                            int lane) {
  __syncwarp();
  if (lane == 0) add_release_gpu_u32(D.arrive + ctr, n);
  __syncwarp();
}

// Copy one or two rows of ``vpr`` 16-byte vectors, 8 vectors per lane per row in flight.
__device__ __forceinline__ void copy_row_pair(const uint4* sa, uint4* da, const uint4* sb,
                                              uint4* db, bool two, int64_t vpr, int lane) {
  constexpr int kVec = 8;
  for (int64_t v0 = 0; v0 < vpr; v0 += 32 * kVec) {
    uint4 a[kVec], b[kVec];
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int64_t v = v0 + lane + 32 * u;
      if (v < vpr) a[u] = sa[v];
      if (two && v < vpr) b[u] = sb[v];
    }
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int64_t v = v0 + lane + 32 * u;
      if (v < vpr) da[v] = a[u];
      if (two && v < vpr) db[v] = b[u];
    }
  }
}

// Slot 0: chunk ``c`` of this rank's own expert-major rows for its own experts. Every row below
// the plan's count belongs to an entry with a valid expert id (the plan leaves the others out),
// so every store lands inside the receive buffer.
__device__ void own_chunk(const GemmDispatch& D, int64_t c, uint8_t* recv, int lane) {
  const int e0 = D.me * D.El;
  const int64_t base = D.expert_offsets[e0];
  const int64_t n = D.expert_offsets[e0 + D.El] - base;
  const int64_t i0 = c * kChunkRows;
  const int nr = static_cast<int>(n - i0 < kChunkRows ? n - i0 : kChunkRows);
  const uint4* x = static_cast<const uint4*>(D.x);
  int my_le = -1;
  int64_t my_src = 0;
  uint64_t my_dst = 0;
  if (lane < nr) {
    const int64_t q = base + i0 + lane;
    const int32_t f = D.row_entry[q];
    const int64_t e = D.ids[f];
    my_src = f / D.k;
    my_le = static_cast<int>(e - e0);
    const int64_t dst_row = D.seg_offsets[my_le] + (q - D.expert_offsets[e]);
    my_dst = reinterpret_cast<uint64_t>(recv) + static_cast<uint64_t>(dst_row * D.vpr * 16);
  }
  int c_run = -1;
  unsigned int n_run = 0;
  for (int r = 0; r < nr; r += 2) {
    const bool two = r + 1 < nr;
    const int rb = two ? r + 1 : r;
    copy_row_pair(x + __shfl_sync(0xffffffffu, my_src, r) * D.vpr,
                  reinterpret_cast<uint4*>(__shfl_sync(0xffffffffu, my_dst, r)),
                  x + __shfl_sync(0xffffffffu, my_src, rb) * D.vpr,
                  reinterpret_cast<uint4*>(__shfl_sync(0xffffffffu, my_dst, rb)), two, D.vpr,
                  lane);
    // runs of one expert; a run's rows are all stored before its count is published
    for (int t = r; t <= rb; ++t) {
      const int le = __shfl_sync(0xffffffffu, my_le, t);
      if (le != c_run) {
        if (n_run) arrival_add(D, c_run, n_run, lane);
        c_run = le;
        n_run = 0;
      }
      ++n_run;
    }
  }
  if (n_run) arrival_add(D, c_run, n_run, lane);
}

// Read one token row from a peer (over NVLink; L2-only loads, so nothing stale comes from L1)
// and write it to the receive rows of the lanes in ``mask`` (their addresses in ``my_dst``).
// (Two rows in flight per pass needed 64 more registers per thread and spilled; one row keeps
// 8 vectors per lane in flight.)
__device__ __forceinline__ void pull_row(const uint4* src, uint32_t mask, uint64_t my_dst,
                                         int64_t vpr, int lane) {
  constexpr int kVec = 8;
  for (int64_t v0 = 0; v0 < vpr; v0 += 32 * kVec) {
    uint4 a[kVec];
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int64_t v = v0 + lane + 32 * u;
      if (v < vpr) a[u] = __ldcg(src + v);
    }
    for (uint32_t m = mask; m; m &= m - 1) {
      uint4* dst = reinterpret_cast<uint4*>(__shfl_sync(0xffffffffu, my_dst, __ffs(m) - 1));
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        const int64_t v = v0 + lane + 32 * u;
        if (v < vpr) dst[v] = a[u];
      }
    }
  }
}

// Slots j >= 1: chunk ``c`` of source s = (me - j) mod W, tokens [t0, t0 + nt), one lane per
// routed entry (lane = token * k + slot). A lane whose entry chose one of this rank's experts
// reads the entry's expert-major row on s and derives its receive row; each token row then
// crosses NVLink once for all of this rank's experts it chose. Returns the rows read.
__device__ unsigned int pull_chunk(const GemmDispatch& D, int j, int64_t t0, int nt,
                                   uint8_t* recv, int lane) {
  const int s = (D.me - j + D.W) % D.W;
  const uint64_t base = D.peers[s];
  const int64_t* ids = reinterpret_cast<const int64_t*>(base + D.src_ids_off);
  const int32_t* rows = reinterpret_cast<const int32_t*>(base + D.src_row_off);
  const uint4* x = reinterpret_cast<const uint4*>(base + D.src_x_off);
  const int e0 = D.me * D.El;
  bool mine = false;
  uint64_t my_dst = 0;
  if (lane < nt * D.k) {
    const int64_t f = t0 * D.k + lane;
    const int64_t e = __ldcg(ids + f);
    mine = e >= e0 && e < e0 + D.El;   // ids outside [0, E) are never this rank's
    if (mine) {
      const int seg = j * D.El + static_cast<int>(e - e0);
      const int64_t q = __ldcg(rows + f);
      const int64_t dst_row = D.seg_offsets[seg] + (q - D.seg_src_row[seg]);
      my_dst = reinterpret_cast<uint64_t>(recv) + static_cast<uint64_t>(dst_row * D.vpr * 16);
    }
  }
  const uint32_t any = __ballot_sync(0xffffffffu, mine);
  const uint32_t tok_bits = D.k == 32 ? 0xffffffffu : ((1u << D.k) - 1u);
  unsigned int pulled = 0;
  for (int u = 0; u < nt; ++u) {
    const uint32_t mask = any & (tok_bits << (u * D.k));
    if (!mask) continue;
    pull_row(x + (t0 + u) * D.vpr, mask, my_dst, D.vpr, lane);
    ++pulled;
  }
  return pulled;
}

// Copy-warp loop: claim chunks (own slot first, then the sources in slot order) until none are
// left. The warp that claims the first chunk and the warp that stores the last one stamp the
// step's dispatch window; rows pulled over NVLink are counted into the step's statistics.
__device__ void copy_warp_loop(const GemmDispatch& D, int par, int lane) {
  uint8_t* recv = static_cast<uint8_t*>(const_cast<void*>(D.x_recv[par]));
  const int64_t total = D.chunk_base[D.W];
  const int64_t own = D.chunk_base[1];
  const int tpc = 32 / D.k;                       // tokens per pull chunk
  bool fenced = false;
  unsigned long long pulled = 0;
  for (;;) {
    unsigned int claimed = 0;
    if (lane == 0) claimed = atomicAdd(D.claim, 1u);
    const int64_t c = __shfl_sync(0xffffffffu, claimed, 0);
    if (c >= total) break;
    if (c == 0 && lane == 0 && D.step) D.step->disp_t0 = global_timer_ns();
    if (c < own) {
      own_chunk(D, c, recv, lane);
    } else {
      if (!fenced) {   // acquire (system scope) of the peers' rows, once per warp
        fence_acq_rel_sys();
        fenced = true;
      }
      int j = 1;
      while (j + 1 < D.W && D.chunk_base[j + 1] <= c) ++j;
      const int64_t t0 = (c - D.chunk_base[j]) * tpc;
      const int64_t Ts = D.src_tokens[j];
      const int nt = static_cast<int>(Ts - t0 < tpc ? Ts - t0 : tpc);
      pulled += pull_chunk(D, j, t0, nt, recv, lane);
      arrival_add(D, D.El + j, static_cast<unsigned int>(nt), lane);
    }
    if (lane == 0) {
      const unsigned int stored = atomicAdd(D.claim + 1, 1u);
      if (stored + 1 == static_cast<unsigned int>(total) && D.step)
        D.step->disp_t1 = global_timer_ns();
    }
  }
  if (lane == 0 && pulled && D.step)
    atomicAdd(reinterpret_cast<unsigned long long*>(&D.step->send_rows), pulled);
}

// ---------------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------------
template <bool kDispatch>
__global__ void __launch_bounds__(kDispatch ? kDispatchThreads : kThreads, 1)
    fused_experts_kernel(const __grid_constant__ CUtensorMap map_x,
                         const __grid_constant__ CUtensorMap map_x1,
                         const __grid_constant__ CUtensorMap map_wgu,
                         const __grid_constant__ CUtensorMap map_h,
                         const __grid_constant__ CUtensorMap map_wd, FusedParams P,
                         GemmOutput tgt, GemmDispatch disp) {
  using F = FusedCfg;
  extern __shared__ uint8_t smem_raw[];
  // An expert-parallel step whose exchange already failed (a peer wait ran out) runs nothing:
  // its tables may describe rows that never arrive.
  __shared__ int s_skip;
  if (threadIdx.x == 0) {
    s_skip = kDispatch && disp.gate_err &&
             *reinterpret_cast<const volatile int*>(disp.gate_err) == PRISM_MOE_ERR_TIMEOUT;
    if (!s_skip && tgt.step)
      atomicMin(reinterpret_cast<unsigned long long*>(&tgt.step->fused_t0),
                static_cast<unsigned long long>(global_timer_ns()));
  }
  __syncthreads();
  if (s_skip) return;
  // receive-buffer parity of this step (expert parallelism; always 0 otherwise)
  const int par = kDispatch ? static_cast<int>(*disp.epoch_ptr & 1u) : 0;
  const CUtensorMap* map_a = par ? &map_x1 : &map_x;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + F::kBarOffset);
  uint64_t* empty = full + F::kStages;
  uint64_t* acc_full = empty + F::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* ring_full = acc_empty + 2;
  uint64_t* ring_empty = ring_full + F::kRing;
  uint64_t* drain = ring_empty + F::kRing;
  int32_t* ring_tile = reinterpret_cast<int32_t*>(drain + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring_tile + F::kRing);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* prefix = reinterpret_cast<int32_t*>(smem + F::kPrefixOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < F::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    for (int i = 0; i < F::kRing; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 5);   // the MMA thread and the 4 epilogue warps
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(map_a);
    tma_prefetch_desc(&map_wgu);
    tma_prefetch_desc(&map_h);
    tma_prefetch_desc(&map_wd);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2) build_tile_prefix(P.seg_offsets, P.nseg, 128, prefix);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int32_t M = prefix[P.nseg];
  const int32_t total = M * (P.n_gu + P.n_dn);
  const uint32_t h_target = 4u * static_cast<uint32_t>(P.n_gu);

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ scheduler + TMA
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, issued_parity = 0;
    int rslot = 0;
    uint32_t rphase = 0;
    int ready_key = -1;      // dispatch: the last arrival counter seen complete
    int32_t ready_mt = -1;   // every h row of this m-tile is stored
    bool ok = true;
    for (;;) {
      int32_t t = -1;
      {
        const unsigned int c = atomicAdd(P.claim, 1u);
        if (c < static_cast<unsigned int>(total)) t = static_cast<int32_t>(c);
      }
      if (!mbar_wait_bounded(&ring_empty[rslot], rphase ^ 1, abort, P.wait_ns)) {
        ok = false;
        break;
      }
      ring_tile[rslot] = t;
      mbar_arrive(&ring_full[rslot]);
      if (++rslot == F::kRing) {
        rslot = 0;
        rphase ^= 1;
      }
      if (t < 0) break;
      const TileRef tr = tile_at(t, M, P.n_gu, P.n_dn, P.lag);
      const int s = find_segment(prefix, P.nseg, tr.mt);
      const int e = P.seg_expert ? P.seg_expert[s] : s;
      const int32_t row0 = P.seg_offsets[s] + (tr.mt - prefix[s]) * 128;
      const uint64_t t0 = global_timer_ns();
      if (tr.kind == 0) {
        // receive slot j of segment s (rows from source (me - j) mod W) and its counter: one per
        // segment in slot 0, one per slot after it. Counters only grow along the tile stream,
        // and this CTA claims stream positions in increasing order.
        const int j = kDispatch ? s / disp.El : 0;
        const int key = j == 0 ? s : disp.El + j;
        if (kDispatch && key > ready_key) {
          const uint32_t need =
              static_cast<uint32_t>(j == 0 ? P.seg_offsets[s + 1] - P.seg_offsets[s]
                                           : disp.src_tokens[j]);
          while (load_relaxed_sys(disp.arrive + key) != need) {
            if (*abort || global_timer_ns() - t0 > P.peer_wait_ns) {
              ok = false;
              break;
            }
          }
          fence_acq_rel_gpu();   // acquire: the copy warps' rows before the count they added
          // rows written through the generic proxy (peer stores), read next by TMA
          asm volatile("fence.proxy.async.global;" ::: "memory");
          ready_key = key;
        }
      } else if (tr.mt != ready_mt) {
        while (load_acquire_gpu(P.h_ready + tr.mt) != h_target) {
          if (*abort || global_timer_ns() - t0 > P.wait_ns) {
            ok = false;
            break;
          }
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");   // h: generic stores -> TMA
        ready_mt = tr.mt;
      }
      if (!ok) break;
      const int nkb = tr.kind == 0 ? P.kb_gu : P.kb_dn;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort, P.wait_ns)) {
          ok = false;
          break;
        }
        uint8_t* sa = stages + stage * F::kStageBytes;
        uint8_t* sb = sa + F::kABytes;
        mbar_arrive_expect_tx(&full[stage], F::kTxBytes);
        if (tr.kind == 0) {
          tma_load_2d(sa, map_a, &full[stage], kb * kBK, row0);
          // gate rows then up rows of n-tile nt in one copy (box spans both halves)
          tma_load_4d(sb, &map_wgu, &full[stage], kb * kBK, tr.nt * 128, 0, e);
        } else {
          tma_load_2d(sa, &map_h, &full[stage], kb * kBK, row0);
          tma_load_3d(sb, &map_wd, &full[stage], kb * kBK, tr.nt * kBN, e);
        }
        issued |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == F::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
    if (!ok) {
      *abort = 1;
      record_device_error(P.err, PRISM_MOE_ERR_TIMEOUT);
      for (int s = 0; s < F::kStages; ++s)   // every issued copy lands before the CTA exits
        if ((issued >> s) & 1u) {
          volatile int never = 0;
          mbar_wait_bounded(&full[s], (issued_parity >> s) & 1u, &never, kDrainNs);
        }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int rslot = 0;
    uint32_t rphase = 0;
    bool ok = true;
    for (int it = 0;; ++it) {
      if (!mbar_wait_bounded(&ring_full[rslot], rphase, abort, P.wait_ns)) {
        ok = false;
        break;
      }
      const int32_t t = ring_tile[rslot];
      mbar_arrive(&ring_empty[rslot]);
      if (++rslot == F::kRing) {
        rslot = 0;
        rphase ^= 1;
      }
      if (t < 0) break;
      const TileRef tr = tile_at(t, M, P.n_gu, P.n_dn, P.lag);
      const int nkb = tr.kind == 0 ? P.kb_gu : P.kb_dn;
      uint32_t idesc = F::kIdesc;
      {   // a segment's last m-tile with <= 64 rows: M=64 MMAs
        const int s = find_segment(prefix, P.nseg, tr.mt);
        const int32_t row0 = P.seg_offsets[s] + (tr.mt - prefix[s]) * 128;
        const int32_t seg_end = P.seg_offsets[s + 1];
        if (half_tile((seg_end < P.rows_cap ? seg_end : P.rows_cap) - row0))
          idesc = idesc_bf16_f32(kHalfRows, kBN);
      }
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_bounded(&acc_empty[buf], acc_phase ^ 1, abort, P.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * kBN;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort, P.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(stages + stage * F::kStageBytes);
        const uint32_t b0 = a0 + F::kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          tc_mma_bf16(d_tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                      idesc, (kb | kk) != 0 ? 1u : 0u);
        tc_commit(&empty[stage]);
        if (++stage == F::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      tc_commit(&acc_full[buf]);
    }
    if (!ok) {
      *abort = 1;
      record_device_error(P.err, PRISM_MOE_ERR_TIMEOUT);
    }
    if (*abort) {
      tc_commit(drain);   // completes once every MMA issued above has finished
      volatile int never = 0;
      mbar_wait_bounded(drain, 0, &never, kDrainNs);
    }
  } else if (kDispatch && warp >= 6) {
    // ------------------------------------------------------------------ copy warps
    copy_warp_loop(disp, par, lane);
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    uint8_t* stage_out = smem + F::kStageOutOffset + (warp - 2) * 32 * kStageRowBytes;
    int rslot = 0;
    uint32_t rphase = 0;
    for (int it = 0;; ++it) {
      if (!mbar_wait_bounded(&ring_full[rslot], rphase, abort, P.wait_ns)) {
        *abort = 1;
        record_device_error(P.err, PRISM_MOE_ERR_TIMEOUT);
        break;
      }
      const int32_t t = ring_tile[rslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&ring_empty[rslot]);
      if (++rslot == F::kRing) {
        rslot = 0;
        rphase ^= 1;
      }
      if (t < 0) break;
      const TileRef tr = tile_at(t, M, P.n_gu, P.n_dn, P.lag);
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int s = find_segment(prefix, P.nseg, tr.mt);
      const int32_t row0 = P.seg_offsets[s] + (tr.mt - prefix[s]) * 128;
      const int32_t seg_end = P.seg_offsets[s + 1];
      const int32_t rows_valid = (seg_end < P.rows_cap ? seg_end : P.rows_cap) - row0;
      if (!mbar_wait_bounded(&acc_full[buf], acc_phase, abort, P.wait_ns)) {
        *abort = 1;
        record_device_error(P.err, PRISM_MOE_ERR_TIMEOUT);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * kBN;
      // row within the tile held by this lane (half tiles: lanes 0-15 of a quarter)
      const int row_in_tile = tile_row_of_lane(half_tile(rows_valid), q, lane);
      const bool has_row = row_in_tile < rows_valid;
      const int64_t row = row0 + row_in_tile;
      if (tr.kind == 0) {
        const uint64_t my_ptr = has_row ? reinterpret_cast<uint64_t>(P.h + row * P.I) : 0;
        drain_tile<true>(taddr, my_ptr, stage_out, lane, static_cast<int64_t>(tr.nt) * 128,
                         P.I);
        // publish this warp's 32 h rows to the producers of the m-tile's down tiles
        __threadfence();
        __syncwarp();
        if (lane == 0) add_release_gpu(P.h_ready + tr.mt, 1u);
      } else {
        uint64_t my_ptr = 0;
        if (has_row)
          my_ptr = tgt.seg_base
                       ? tgt.seg_base[s] +
                             static_cast<uint64_t>((row - P.seg_offsets[s]) * P.H * 2)
                       : reinterpret_cast<uint64_t>(P.y + row * P.H);
        drain_tile<false>(taddr, my_ptr, stage_out, lane, static_cast<int64_t>(tr.nt) * kBN,
                          P.H);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  if (tgt.done_counter != nullptr && warp >= 2) threadfence_scoped(tgt.remote);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  // completion signal: the last CTA to get here publishes `epoch` to every flag
  if (tgt.done_counter != nullptr && threadIdx.x == 0) {
    threadfence_scoped(tgt.remote);
    const unsigned int prev = atomicAdd(tgt.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      *tgt.done_counter = 0u;  // ready for the next launch (stream-ordered)
      if (tgt.step) tgt.step->fused_t1 = global_timer_ns();
      threadfence_scoped(tgt.remote);
      const uint64_t ep = tgt.epoch_ptr ? *tgt.epoch_ptr : tgt.epoch;
      for (int i = 0; i < tgt.num_signal; ++i)
        store_release_scoped(tgt.signal_flags[i], ep, tgt.remote);
    }
  }
}

template <bool kDispatch>
int launch_fused(const CUtensorMap (&maps)[5], const FusedParams& P, const GemmOutput& tgt,
                 const GemmDispatch& disp, int grid, cudaStream_t st) {
  auto kern = fused_experts_kernel<kDispatch>;
  if (int r = ensure_smem_attr(reinterpret_cast<const void*>(kern),
                               static_cast<int>(FusedCfg::kSmemBytes)))
    return r;
  kern<<<grid, kDispatch ? kDispatchThreads : kThreads, FusedCfg::kSmemBytes, st>>>(
      maps[0], maps[4], maps[1], maps[2], maps[3], P, tgt, disp);
  PRISM_LAUNCH_CHECK("fused_experts_kernel launch");
  return PRISM_MOE_OK;
}

int64_t max_mtiles(int64_t rows_cap) { return ceil_div(rows_cap, 128) + kMaxSegments; }

}  // namespace

// [0] tile claim, [1] unused, h_ready[max m-tiles]
size_t fused_sync_bytes(int64_t rows_cap) {
  return sizeof(unsigned int) * static_cast<size_t>(2 + max_mtiles(rows_cap));
}

int expert_swiglu_fused(const void* xs, int64_t rows_cap, int64_t H, int64_t I,
                        const int32_t* seg_offsets, const int32_t* seg_expert, int nseg, int El,
                        const void* wgu, const void* wd, void* y, void* h, unsigned int* sync,
                        int* err, cudaStream_t st, const GemmOutput* down_out,
                        const GemmDispatch* dispatch) {
  // maps: [0] A rows (parity-0 receive buffer under expert parallelism), [1] gate/up weights,
  // [2] h, [3] down weights, [4] A rows of the parity-1 receive buffer (= [0] otherwise)
  CUtensorMap maps[5];
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(H), static_cast<uint64_t>(rows_cap)};
    const uint64_t strides[1] = {static_cast<uint64_t>(H) * 2};
    const uint32_t box[2] = {kBK, 128};
    const bool two = dispatch && dispatch->x_recv[0] && dispatch->x_recv[1];
    int r = encode_bf16_map(&maps[0], two ? dispatch->x_recv[0] : xs, 2, dims, strides, box);
    if (r) return r;
    if (two) {
      r = encode_bf16_map(&maps[4], dispatch->x_recv[1], 2, dims, strides, box);
      if (r) return r;
    } else {
      maps[4] = maps[0];
    }
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(H), static_cast<uint64_t>(I), 2,
                              static_cast<uint64_t>(El)};
    const uint64_t strides[3] = {static_cast<uint64_t>(H) * 2, static_cast<uint64_t>(I * H) * 2,
                                 static_cast<uint64_t>(2 * I * H) * 2};
    const uint32_t box[4] = {kBK, 128, 2, 1};   // gate and up halves of an n-tile
    int r = encode_bf16_map(&maps[1], wgu, 4, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(I), static_cast<uint64_t>(rows_cap)};
    const uint64_t strides[1] = {static_cast<uint64_t>(I) * 2};
    const uint32_t box[2] = {kBK, 128};
    int r = encode_bf16_map(&maps[2], h, 2, dims, strides, box);
    if (r) return r;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(I), static_cast<uint64_t>(H),
                              static_cast<uint64_t>(El)};
    const uint64_t strides[2] = {static_cast<uint64_t>(I) * 2, static_cast<uint64_t>(H * I) * 2};
    const uint32_t box[3] = {kBK, kBN, 1};
    int r = encode_bf16_map(&maps[3], wd, 3, dims, strides, box);
    if (r) return r;
  }
  const int grid = num_sms();
  FusedParams P;
  P.seg_offsets = seg_offsets;
  P.seg_expert = seg_expert;
  P.nseg = nseg;
  P.rows_cap = static_cast<int32_t>(rows_cap);
  P.n_gu = static_cast<int>(ceil_div(I, 128));
  P.n_dn = static_cast<int>(ceil_div(H, kBN));
  P.kb_gu = static_cast<int>(ceil_div(H, kBK));
  P.kb_dn = static_cast<int>(ceil_div(I, kBK));
  // A CTA holds up to about three tiles between claiming one and storing its output; a lag of
  // twice that keeps down tiles from waiting for h even when epilogues run slow.
  P.lag = static_cast<int>(std::max<int64_t>(1, ceil_div(6 * grid, P.n_gu + P.n_dn)));
  P.wait_ns = wait_limit_ns();
  P.peer_wait_ns = peer_wait_limit_ns();
  P.H = H;
  P.I = I;
  P.h = static_cast<uint16_t*>(h);
  P.y = static_cast<uint16_t*>(y);
  P.claim = sync;
  P.h_ready = sync + 2;
  P.err = err;
  PRISM_CUDA(cudaMemsetAsync(sync, 0, fused_sync_bytes(rows_cap), st));
  const GemmOutput dense{};
  const GemmOutput& tgt = down_out ? *down_out : dense;
  return dispatch ? launch_fused<true>(maps, P, tgt, *dispatch, grid, st)
                  : launch_fused<false>(maps, P, tgt, GemmDispatch{}, grid, st);
}

}  // namespace prism
