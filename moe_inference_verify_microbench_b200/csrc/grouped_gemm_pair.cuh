// CTA-pair variant of the grouped GEMM for large batches: one
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16) per K-step, issued by the
// even CTA of a (2,1,1) cluster.
//
// Work unit: one (pair tile, N-tile).  A pair tile is up to 256 consecutive
// rows of one expert (tile table built with 256-row blocks); CTA r of the pair
// owns rows row_begin + 128 r .. +127 of it and loads those A rows plus half of
// the B tile (the store GEMM: B rows n*256 + 128 r .. +127; the SwiGLU GEMM:
// gate rows n*128 + 64 r .. +63 followed by the up rows of the same indices,
// so that the accumulator holds [gate | up] of the same output columns in
// each 128-column half: [g 0..63 | u 0..63 | g 64..127 | u 64..127]).  Each
// CTA's tensor memory receives the 128 x 256 accumulator of its own rows.
// Per CTA and K-block the operands are 32 KB for 4.2 MFLOP, against 48 KB for
// the single-CTA 128 x 256 tile: the pair halves the B traffic from L2 and
// leaves room for six stages.
//
// Half tiles.  The last block of an expert often holds few rows (with ~1024
// rows per expert about half the experts end in a block of <= 64 rows); a
// tile of <= 128 rows runs M = 128 MMAs instead, with 64 A rows per CTA, at
// half the tensor work.  Their accumulator (the tcgen05 data-path layout of
// cta_group::2 at M = 128) keeps the CTA's 64 rows twice over: columns
// 0..127 of the tile in TMEM lanes 0..63 and columns 128..255 in lanes
// 64..127, both at TMEM columns 0..127; the epilogue maps lane quarters to
// rows and columns accordingly.  The gate/up column order above keeps gate
// and up of an output column in the same lane in both layouts.
//
// Roles per CTA (384 threads): warp 0 TMA producer (both CTAs; the copies of
// both count on the even CTA's stage barrier), warp 1 MMA issuer (even CTA
// only; its commits arrive on the stage and accumulator barriers of both
// CTAs), warp 2 tensor-memory allocator (.cta_group::2, both CTAs), warps
// 4..11 epilogue (both CTAs; they release an accumulator by arriving on the
// even CTA's barrier).  Every wait is bounded; a CTA leaves only after the
// final cluster barrier, so no copy, MMA or remote arrival can target a CTA
// that has exited.
//
// GATHER_A (512 threads): warps 12..15 of each CTA gather its 128 A rows from
// the source matrix through the index with 16-byte cp.async, as in the
// single-CTA kernel; the TMA producer then loads only B.  The loaders never
// wait for their copies: each thread arms a CTA-local barrier with
// cp.async.mbarrier.arrive.noinc, which completes once every loader thread's
// copies of the stage have landed, and lane 0 of warp 3 (the forwarder) waits
// for it, fences the generic->async proxy and publishes the stage on the even
// CTA's stage barrier.  (Publishing from the loaders themselves after
// cp.async.wait_group serialised them on their oldest copies: 3 % slower.)
// This fuses the permutation gather (C5/python/solution.py:137) into the
// gate/up GEMM and removes the gathered copy's round trip through HBM.
#pragma once

#include "grouped_gemm.cuh"

namespace moe {

constexpr int kPairBM = 2 * kBM;  // rows of a pair tile (M of the pair MMA)
constexpr int kPairBN = 256;
constexpr int kPairGatherWarp0 = 12;  // first of the four A-loader warps (GATHER_A)
constexpr int kPairForwardWarp = 3;   // publishes the loaders' stages (GATHER_A)

template <bool GATHER_A>
constexpr int pair_threads() {
  return GATHER_A ? 512 : 384;
}

template <int STAGES>
struct PairSmem {
  static constexpr int kABytes = kBM * kBK * 2;                // this CTA's 128 A rows
  static constexpr int kBBytes = (kPairBN / 2) * kBK * 2;      // this CTA's half of the B rows
  static constexpr int kStageBytes = kABytes + kBBytes;        // 32 KB
  static constexpr int kOutBytes = 8 * kEpiStageBytes;         // epilogue staging
  static constexpr int kTotal = 1024 + STAGES * kStageBytes + kOutBytes + 256;
};

template <int EPI, int STAGES, bool GATHER_A = false>
__global__ void __launch_bounds__(pair_threads<GATHER_A>(), 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB0,
                             const __grid_constant__ CUtensorMap tmB1, const GemmArgs args) {
  static_assert(EPI == kEpiSwiGLU || EPI == kEpiStore || EPI == kEpiAtomic,
                "pair kernel: SwiGLU, store or atomic epilogue");
  using L = PairSmem<STAGES>;
  constexpr int BN = kPairBN;
  constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  constexpr int kEpiWarps = 8;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kABytes;
  uint8_t* sOut = sB + STAGES * L::kBBytes;  // epilogue staging, kEpiStageBytes per warp
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + L::kOutBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* gat = drain + 1;  // GATHER_A: this CTA's loader copies of a stage have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gat + STAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: issues the pair's MMAs
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // The even CTA's producer (+ the bytes of both CTAs), and with GATHER_A
      // the forwarder of each CTA.
      mbar_init(&full[s], GATHER_A ? 1 + 2 : 1);
      mbar_init(&empty[s], 1);  // one MMA commit
      mbar_init(&gat[s], 4 * 32);  // the copies of every loader thread of this CTA
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);  // the epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    if (!GATHER_A) tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB0);
    if (EPI == kEpiSwiGLU) tma_prefetch_desc(&tmB1);
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  int num_tiles = args.num_tiles != nullptr ? *args.num_tiles : args.max_tiles;
  num_tiles = max(0, min(num_tiles, args.max_tiles));
  const int total = num_tiles * args.n_tiles;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const uint32_t stage_tx = static_cast<uint32_t>(GATHER_A ? L::kBBytes : L::kStageBytes);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int w = pair; ok && w < total; w += npairs) {
        const int mt = w / args.n_tiles;
        const int nt = w - mt * args.n_tiles;
        const int4 t = load_tile(args, mt);
        if (t.x < 0 || t.x >= args.num_experts || t.y < 0 || t.z > args.a_rows || t.y >= t.z ||
            t.z - t.y > kPairBM) {
          record_status(args.status, t.x < 0 || t.x >= args.num_experts ? kErrBadExpert : kErrBadRow);
          *abort_flag = 1;
          break;
        }
        // A rows of this CTA: 128 (64 in a half tile); the box always holds
        // 128 rows, of which a half tile's MMA reads the first 64.
        const int arow = t.y + (t.z - t.y <= kBM ? kBM / 2 : kBM) * static_cast<int>(rank);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, args.status, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * stage_tx);
          const uint32_t fb = cluster_addr(&full[s], 0);
          if (!GATHER_A) tma_load_2d_pair(sA + s * L::kABytes, &tmA, fb, kb * kBK, arow);
          uint8_t* b = sB + s * L::kBBytes;
          if (EPI == kEpiSwiGLU) {
            // gate rows nt*128 + 64 rank .. +63, then the up rows of the same indices
            const int brow = nt * (BN / 2) + (BN / 4) * static_cast<int>(rank);
            tma_load_3d_pair(b, &tmB0, fb, kb * kBK, brow, t.x);
            tma_load_3d_pair(b + L::kBBytes / 2, &tmB1, fb, kb * kBK, brow, t.x);
          } else {
            tma_load_3d_pair(b, &tmB0, fb, kb * kBK, nt * BN + (BN / 2) * static_cast<int>(rank),
                             t.x);
          }
          ++issued;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (*abort_flag && leader) {
        // Let every copy counted on this CTA's stage barriers land.
        const uint32_t first = issued > STAGES ? issued - STAGES : 0u;
        for (uint32_t i = first; i < issued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1u)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc_full = idesc_bf16_f32(kPairBM, BN);
      const uint32_t idesc_half = idesc_bf16_f32(kBM, BN);  // half tile: 64 rows per CTA
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      // Tile entries are read one work unit ahead, so the load is not waited on.
      int4 t_next = pair < total ? load_tile(args, pair / args.n_tiles) : make_int4(0, 0, 0, 0);
      for (int w = pair; ok && w < total; w += npairs, ++it) {
        const int4 t = t_next;
        if (w + npairs < total) t_next = load_tile(args, (w + npairs) / args.n_tiles);
        const uint32_t idesc = t.z - t.y <= kBM ? idesc_half : idesc_full;
        const int acc = it & 1;
        const uint32_t acc_ph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag, args.status,
                               kErrTimeoutAccEmpty))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, args.status, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * L::kABytes);
          const uint32_t b0 = smem_u32(sB + s * L::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            tc_mma_bf16_pair(d, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32),
                             idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit_pair(cluster_addr(&empty[s], 0));
          tc_commit_pair(cluster_addr(&empty[s], 1));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) {
          tc_commit_pair(cluster_addr(&acc_full[acc], 0));
          tc_commit_pair(cluster_addr(&acc_full[acc], 1));
        }
      }
      // Every MMA issued by this thread has finished once `drain` completes.
      tc_commit_pair(cluster_addr(drain, 0));
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
  } else if (GATHER_A && warp >= kPairGatherWarp0) {
    // ---------------------------------------------------------- A-row loaders
    // Thread g = 0..127 copies 16-byte chunk (g % 8) of this CTA's tile rows
    // (g / 8) + 16 j, j = 0..7, into the 128-byte-swizzled layout TMA would write.
    const int g = threadIdx.x - kPairGatherWarp0 * 32;
    const uint32_t chunk = static_cast<uint32_t>(g & 7);
    const int row0 = g >> 3;
    const int K = args.num_kb * kBK;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int w = pair; ok && w < total; w += npairs) {
      const int mt = w / args.n_tiles;
      const int4 t = load_tile(args, mt);
      const bool half_tile = t.z - t.y <= kBM;
      const int base = t.y + (half_tile ? kBM / 2 : kBM) * static_cast<int>(rank);
      const int nrows = half_tile ? 4 : 8;  // rows row0 + 16 j, j < nrows (64 or 128 rows)
      const __nv_bfloat16* src[8];
      uint32_t present = 0;  // bit j: row j of this thread exists
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int p = base + row0 + 16 * j;
        src[j] = args.a_src;  // any valid address when the row is absent (zero-filled)
        if (j < nrows && p < t.z) {
          const int i = args.a_index != nullptr ? args.a_index[p] / args.a_index_div : p;
          if (i >= 0 && i < args.a_src_rows) {
            src[j] = args.a_src + static_cast<size_t>(i) * K + chunk * 8;
            present |= 1u << j;
          } else {
            record_status(args.status, kErrBadRow);
          }
        }
      }
      for (int kb = 0; kb < args.num_kb; ++kb) {
        bool got = mbar_wait(&empty[s], ph ^ 1u, abort_flag, args.status, kErrTimeoutEmpty);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          ok = false;
          break;
        }
        const uint32_t sbase = smem_u32(sA + s * L::kABytes);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j >= nrows) break;  // a half tile's MMA reads rows 0..63 only
          const uint32_t r = static_cast<uint32_t>(row0 + 16 * j);
          const uint32_t dst = sbase + r * 128u + ((chunk ^ (r & 7u)) << 4);
          const bool have = (present >> j) & 1u;
          cp_async_16(dst, have ? src[j] + kb * kBK : src[j], have ? 16u : 0u);
        }
        cp_async_arrive_noinc(&gat[s]);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    cp_async_wait_all();  // every copy lands before the CTA can exit
  } else if (GATHER_A && warp == kPairForwardWarp) {
    if (lane == 0) {
      // -------------------------------------------------------- forwarder
      // A stage's A rows are complete once every loader thread's copies have
      // landed (gat); then the proxy fence makes them visible to the tensor
      // core's async proxy and the stage is published on the even CTA's barrier.
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int w = pair; ok && w < total; w += npairs) {
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&gat[s], ph, abort_flag, args.status, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();
          mbar_arrive_cluster(cluster_addr(&full[s], 0));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp >= 4 && warp < 4 + kEpiWarps) {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int part = (warp - 4) >> 2;       // which of the two column shares
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t release0 = cluster_addr(&acc_empty[0], 0);
    const uint32_t release1 = cluster_addr(&acc_empty[1], 0);
    int it = 0;
    for (int w = pair; w < total; w += npairs, ++it) {
      const int acc = it & 1;
      const uint32_t acc_ph = (it >> 1) & 1;
      const int mt = w / args.n_tiles;
      const int nt = w - mt * args.n_tiles;
      const int4 t = load_tile(args, mt);
      const bool half_tile = t.z - t.y <= kBM;
      const int row = half_tile ? t.y + (kBM / 2) * static_cast<int>(rank) + (q & 1) * 32 + lane
                                : t.y + kBM * static_cast<int>(rank) + q * 32 + lane;
      const bool valid = row < t.z;
      int orow_idx = row;
      float scale = 1.0f;
      bool st = valid;
      if constexpr (EPI == kEpiStore || EPI == kEpiAtomic) {
        if (st) {
          if (args.row_map != nullptr) orow_idx = args.row_map[row];
          if (orow_idx < 0 || orow_idx >= args.out_rows) {
            record_status(args.status, kErrBadRow);
            st = false;
          } else if (args.row_scale != nullptr) {
            scale = args.row_scale[orow_idx];
          }
        }
      } else {
        st = valid && row < args.out_rows;
      }
      bool ok = mbar_wait(&acc_full[acc], acc_ph, abort_flag, args.status,
                                  kErrTimeoutAccFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + static_cast<uint32_t>(acc * BN) + lane_off;
      uint8_t* const stage = sOut + (warp - 4) * kEpiStageBytes;
      // Columns of this warp.  Full tile: its share `part` of its lane quarter's
      // 256 columns.  Half tile: lane quarter q holds rows (q & 1) * 32 .. and
      // tile columns 128 (q >> 1) .. + 127 at TMEM columns 0..127.
      const int blk = q >> 1;
      if constexpr (EPI == kEpiSwiGLU) {
        // [g | u] pairs of 64 columns: output column nt*128 + 64 b + i has its
        // gate value at accumulator column 128 b + i and up at 128 b + 64 + i.
        if (!half_tile)
          epilogue_cols<kEpiSwiGLU, 64>(args, tb, st, row, 1.0f, 128 * part, 64,
                                        nt * (BN / 2) + 64 * part, 64, stage, lane);
        else
          epilogue_cols<kEpiSwiGLU, 32>(args, tb, st, row, 1.0f, 32 * part, 64,
                                        nt * (BN / 2) + 64 * blk + 32 * part, 32, stage, lane);
      } else if constexpr (EPI == kEpiStore) {
        if (!half_tile)
          epilogue_cols<kEpiStore, 64>(args, tb, st, orow_idx, scale, 128 * part, 0,
                                       nt * BN + 128 * part, 128, stage, lane);
        else
          epilogue_cols<kEpiStore, 64>(args, tb, st, orow_idx, scale, 64 * part, 0,
                                       nt * BN + 128 * blk + 64 * part, 64, stage, lane);
      } else {
        if (!half_tile)
          epilogue_cols_atomic(args, tb, st, orow_idx, scale, 128 * part, nt * BN + 128 * part,
                               128, stage, lane);
        else
          epilogue_cols_atomic(args, tb, st, orow_idx, scale, 64 * part,
                               nt * BN + 128 * blk + 64 * part, 64, stage, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? release1 : release0);
    }
  }

  tc_fence_before();
  cluster_sync_all();  // nothing targets either CTA after this point
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace moe
