// Persistent tcgen05 grouped GEMM over ragged per-expert row blocks.
//
// Replaces the reference's per-expert loop (C5/python/solution.py:142-157)
// and its Triton grouped_matmul_kernel (C9/python/solution.py:58-129).
//
// Work unit: one (M-tile, N-tile) pair.  An M-tile is 128 consecutive rows of
// the A operand that all belong to one expert (tile table entry
// {expert, row_begin, row_end}); rows past row_end inside the 128-row box are
// computed but never stored.  The tile table lives in device memory and its
// length is read on the device, so no host synchronisation is needed between
// the sort and the GEMM.
//
// CTA layout (256 threads, one CTA per SM, grid = min(#SMs, #work units)):
//   warp 0      TMA producer: A box [128 x 64] + B box [BN x 64] per stage
//   warp 1      MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per stage
//   warp 2      tensor-memory allocator (2 accumulators of BN fp32 columns)
//   warps 4..7  epilogue: tcgen05.ld of its 32 TMEM lanes -> registers -> HBM
// Shared-memory stages are released by tcgen05.commit; the two accumulators
// let the epilogue of tile i overlap the main loop of tile i+1.
//
// GATHER_A (384 threads): the A operand is not a pre-gathered matrix but rows
// of a source matrix picked through an index (row p of the tile reads source
// row index[p] / index_div: the token of routing record perm[p]).  Warps 8..11
// load them with 16-byte cp.async into the same 128-byte-swizzled layout TMA
// would write; eight consecutive lanes cover one row's 128 bytes, so every
// warp instruction moves four whole 128-byte lines.  The loaders do not wait
// for their copies: every loader thread arms the stage's gather barrier with
// cp.async.mbarrier.arrive.noinc, which completes once all of their copies of
// the stage have landed; lane 0 of warp 3 (the forwarder) waits for it,
// fences the generic->async proxy (the MMA reads shared memory through the
// async proxy) and arrives on the stage barrier.  Warp 0 then loads only B.
// This fuses the permutation gather (C5/python/solution.py:137) into the GEMM.
#pragma once

#include "ptx.cuh"

namespace moe {

enum EpiKind : int {
  kEpiSwiGLU = 0,  // out[row, nt*BN/2 + c] = silu(acc[c]) * acc[BN/2 + c]
  kEpiStore = 1,   // out[map(row), nt*BN + c] = scale(map(row)) * acc[c]
  kEpiRouter = 2,  // per row: bf16 logits -> top-k -> softmax
  kEpiAtomic = 3,  // out_f32[map(row) / red_div, nt*BN + c] += scale(map(row)) * acc[c]
};

struct GemmArgs {
  const int4* tiles;     // [max_tiles] {expert, row_begin, row_end, 0}; null = dense rows
  const int* num_tiles;  // device count of valid tile entries; null = max_tiles
  int max_tiles;         // host bound on the tile count (grid sizing / clamp)
  int n_tiles;           // N-tiles per M-tile
  int num_kb;            // K / 64
  int b_rows;            // rows of B per stage (BN, or E for the router)
  int a_rows;            // rows of the A operand (bounds check / dense tiling)
  int num_experts;       // experts addressed by the tile table (bounds check)
  // kEpiSwiGLU / kEpiStore
  __nv_bfloat16* out;
  int out_ld;            // elements between output rows
  int out_rows;          // output rows (bounds check)
  const int* row_map;    // kEpiStore: out row = row_map[row] (null = identity)
  const float* row_scale;  // kEpiStore: multiplier indexed by the mapped row (null = 1)
  // kEpiAtomic (with out_ld, out_rows, row_map, row_scale as for kEpiStore)
  float* out_f32;        // fp32 accumulation rows, added to with vector atomics
  int red_div;           // accumulation row = mapped row / red_div (top-k: slot -> token)
  // GATHER_A
  const __nv_bfloat16* a_src;  // source rows [a_src_rows, K]
  int a_src_rows;
  const int* a_index;          // A row p = a_src[a_index[p] / a_index_div] (null = p)
  int a_index_div;
  // kEpiRouter
  const float* bias;     // [E] fp32 added before bf16 rounding (null = none)
  int top_k;
  int norm_topk_prob;
  int* ids_out;          // [T, k] int32
  float* w_out;          // [T, k] fp32
  __nv_bfloat16* logits_out;  // [T, E] bf16 (null = not written)
  int* status;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kRouterMaxK = 8;

// Output staging: each epilogue warp owns 32 rows x 128 bytes of shared memory
// through which it turns its row-per-lane results into whole-line stores.
constexpr int kEpiStageBytes = 32 * 128;

template <int BN, int STAGES, int OUT_BYTES = 0>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOutBytes = OUT_BYTES;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kTotal = 1024 + STAGES * kStageBytes + kOutBytes + kBarrierBytes;
};

__device__ __forceinline__ int4 load_tile(const GemmArgs& a, int mt) {
  if (a.tiles != nullptr) return a.tiles[mt];
  const int r0 = mt * kBM;
  return make_int4(0, r0, min(a.a_rows, r0 + kBM), 0);
}

// silu(g) = g * sigmoid(g) with the fast exponential and division
// intrinsics; the result is rounded to bf16, far above their error.
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Router top-k keys.  A bf16 logit and its expert id pack into one 32-bit key
// whose unsigned order is "larger value first, lower expert id first among
// equal values" -- the reference's torch.topk with ties broken toward the lower
// id.  High half: the bf16 bits mapped to unsigned order (negative values
// flipped, positive ones offset by the sign bit); low half: 0xFFFF - id.
__device__ __forceinline__ uint32_t topk_key(float bf16_value, int id) {
  uint32_t b = __float_as_uint(bf16_value) >> 16;
  if (b == 0x8000u) b = 0u;  // -0 equals +0: let the id decide, as torch does
  const uint32_t ord = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(id));
}

__device__ __forceinline__ float topk_key_value(uint32_t key) {
  const uint32_t ord = key >> 16;
  const uint32_t b = (ord & 0x8000u) ? (ord & 0x7FFFu) : (~ord & 0xFFFFu);
  return __uint_as_float(b << 16);
}

__device__ __forceinline__ int topk_key_id(uint32_t key) {
  return static_cast<int>(0xFFFFu - (key & 0xFFFFu));
}

// Keep the kRouterMaxK largest keys in descending order: one max/min pair per
// slot, no data-dependent branches.
__device__ __forceinline__ void topk_insert(uint32_t (&top)[kRouterMaxK], uint32_t key) {
#pragma unroll
  for (int i = 0; i < kRouterMaxK; ++i) {
    const uint32_t hi = max(top[i], key);
    key = min(top[i], key);
    top[i] = hi;
  }
}

// 16-byte slot of row r's chunk j in a warp's staging rows of `row_bytes`:
// XOR-swizzled so that both the row-per-lane writes and the line-per-8-lanes
// reads are free of bank conflicts.
template <int ROW_BYTES>
__device__ __forceinline__ uint32_t stage_slot(int r, int j) {
  if constexpr (ROW_BYTES == 128) return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
  else return static_cast<uint32_t>(r * 64 + ((j ^ ((r >> 1) & 3)) << 4));
}

// Epilogue core: `ncols` output columns of this thread's row, in chunks of CW
// (32 or 64) columns: TMEM -> bf16 -> this warp's staging rows -> global.
// Output column ocol0 + c comes from TMEM column tcol0 + c of this warp's lane
// window `tb`; SwiGLU: out = silu(acc[tcol0 + c]) * acc[tcol0 + ucol + c];
// store: out = scale * acc[tcol0 + c].  Every lane stages its row, then each
// store instruction writes CW*2-byte row segments of 256/CW rows (whole
// 128-byte lines for CW = 64), with the row's destination and store flag
// taken from the lane that owns it.
template <int EPI, int CW>
__device__ __forceinline__ void epilogue_cols(const GemmArgs& args, uint32_t tb, bool st,
                                              int orow_idx, float scale, int tcol0, int ucol,
                                              int ocol0, int ncols, uint8_t* stage, int lane) {
  static_assert(CW == 32 || CW == 64, "epilogue chunks are 32 or 64 columns");
  constexpr int kRowBytes = 2 * CW;
  constexpr int kLanesPerRow = CW / 8;
  constexpr int kRowsPerStore = 32 / kLanesPerRow;
  const uint32_t my_stage = smem_u32(stage);
  const int j = lane % kLanesPerRow;
  const int rsub = lane / kLanesPerRow;
  __nv_bfloat16* const out_base = args.out + ocol0;
#pragma unroll 1
  for (int c0 = 0; c0 < ncols; c0 += CW) {
    uint32_t pk[CW / 2];
#pragma unroll
    for (int sub = 0; sub < CW / 32; ++sub) {
      if constexpr (EPI == kEpiSwiGLU) {
        uint32_t g[32], u[32];
        tmem_ld32(tb + tcol0 + c0 + 32 * sub, g);
        tmem_ld32(tb + tcol0 + ucol + c0 + 32 * sub, u);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float g0 = __uint_as_float(g[2 * i]), g1 = __uint_as_float(g[2 * i + 1]);
          const float u0 = __uint_as_float(u[2 * i]), u1 = __uint_as_float(u[2 * i + 1]);
          pk[16 * sub + i] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
        }
      } else {
        uint32_t r[32];
        tmem_ld32(tb + tcol0 + c0 + 32 * sub, r);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[16 * sub + i] = pack_bf16x2(__uint_as_float(r[2 * i]) * scale,
                                         __uint_as_float(r[2 * i + 1]) * scale);
      }
    }
#pragma unroll
    for (int q = 0; q < CW / 8; ++q) {
      const uint32_t a = my_stage + stage_slot<kRowBytes>(lane, q);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pk[4 * q]),
                   "r"(pk[4 * q + 1]), "r"(pk[4 * q + 2]), "r"(pk[4 * q + 3])
                   : "memory");
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32 / kRowsPerStore; ++i) {
      const int r = i * kRowsPerStore + rsub;
      const int o = __shfl_sync(0xffffffffu, orow_idx, r);
      const bool ok = __shfl_sync(0xffffffffu, st ? 1 : 0, r) != 0;
      uint4 v;
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                   : "r"(my_stage + stage_slot<kRowBytes>(r, j))
                   : "memory");
      if (ok)
        *reinterpret_cast<uint4*>(out_base + static_cast<size_t>(o) * args.out_ld + c0 + j * 8) = v;
    }
    __syncwarp();
  }
}

// Epilogue of one accumulator tile of the single-CTA kernel for this thread's
// row: the accumulator holds [gate BN/2 | up BN/2] (SwiGLU) or BN output
// columns (store); SwiGLU: out[row, nt*BN/2 + c] = silu(acc[c]) *
// acc[BN/2 + c]; store: out[orow, nt*BN + c] = scale * acc[c].  `half`
// selects this warp's share of the columns when kHalves warps serve one TMEM
// lane quarter.
template <int BN, int EPI, int kHalves>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& args, uint32_t tb, int row,
                                              bool valid, bool st, int orow_idx, float scale,
                                              int nt, int half, uint8_t* stage, int lane) {
  constexpr int kOut = EPI == kEpiSwiGLU ? BN / 2 : BN;  // output columns of the tile
  constexpr int kSplit = (kOut / kHalves >= 32) ? kHalves : 1;
  constexpr int kCols = kOut / kSplit;                   // this warp's output columns
  constexpr int CW = (kCols % 64 == 0) ? 64 : 32;
  static_assert(kCols % 32 == 0, "epilogue works in 32-column chunks");
  if (half >= kSplit) return;
  if constexpr (EPI == kEpiSwiGLU) {
    orow_idx = row;
    st = valid && row < args.out_rows;
  }
  epilogue_cols<EPI, CW>(args, tb, st, orow_idx, scale, half * kCols, BN / 2,
                         nt * kOut + half * kCols, kCols, stage, lane);
}

// Atomic-combine epilogue core (the reference's index_add_ on CUDA, C5:160):
// this row's scaled fp32 results of TMEM columns tcol0 .. tcol0 + ncols are
// added into its token's accumulation row at columns ocol0 .. with 16-byte
// fp32 vector atomics.  Rows are staged through this warp's shared memory so
// that eight lanes cover one 128-byte segment of a row and each instruction
// touches four whole segments.  The order in which the k records of a token
// land is not fixed, so the sums are not bitwise reproducible.
__device__ __forceinline__ void epilogue_cols_atomic(const GemmArgs& args, uint32_t tb, bool st,
                                                     int orow_idx, float scale, int tcol0,
                                                     int ocol0, int ncols, uint8_t* stage,
                                                     int lane) {
  const uint32_t my_stage = smem_u32(stage);
  const int j = lane & 7;
  const int rsub = lane >> 3;
  const int tok = st ? orow_idx / args.red_div : 0;
  float* const out_base = args.out_f32 + ocol0;
#pragma unroll 1
  for (int c0 = 0; c0 < ncols; c0 += 32) {
    uint32_t r[32];
    tmem_ld32(tb + tcol0 + c0, r);
    tc_wait_ld();
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t a = my_stage + stage_slot<128>(lane, q);
      asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                   "f"(__uint_as_float(r[4 * q]) * scale), "f"(__uint_as_float(r[4 * q + 1]) * scale),
                   "f"(__uint_as_float(r[4 * q + 2]) * scale),
                   "f"(__uint_as_float(r[4 * q + 3]) * scale)
                   : "memory");
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = i * 4 + rsub;
      const int t = __shfl_sync(0xffffffffu, tok, rr);
      const bool ok = __shfl_sync(0xffffffffu, st ? 1 : 0, rr) != 0;
      float4 v;
      asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                   : "r"(my_stage + stage_slot<128>(rr, j))
                   : "memory");
      if (ok)
        atomicAdd(reinterpret_cast<float4*>(out_base + static_cast<size_t>(t) * args.out_ld + c0 +
                                             j * 4),
                  v);
    }
    __syncwarp();
  }
}

template <int BN, int kHalves>
__device__ __forceinline__ void epilogue_tile_atomic(const GemmArgs& args, uint32_t tb, bool st,
                                                     int orow_idx, float scale, int nt, int half,
                                                     uint8_t* stage, int lane) {
  constexpr int kSplit = (BN / kHalves >= 32) ? kHalves : 1;
  constexpr int kCols = BN / kSplit;
  static_assert(kCols % 32 == 0, "epilogue works in 32-column chunks");
  if (half >= kSplit) return;
  epilogue_cols_atomic(args, tb, st, orow_idx, scale, half * kCols, nt * BN + half * kCols, kCols,
                       stage, lane);
}

constexpr int kGatherWarp0 = 8;    // first of the four A-loader warps
constexpr int kGatherWarps = 4;
constexpr int kForwardWarp = 3;    // publishes the loaders' stages

// Epilogue warps: 4..7 read TMEM lane quarters 0..3; without GATHER_A, warps
// 8..11 take the second half of the accumulator columns (two warps per lane
// quarter), so the epilogue keeps pace with short main loops (w2's K = I).
template <bool GATHER_A>
constexpr int epi_warps() {
  return GATHER_A ? 4 : 8;
}

template <int EPI, bool GATHER_A>
constexpr int gemm_out_bytes() {
  return EPI == kEpiRouter ? 0 : epi_warps<GATHER_A>() * kEpiStageBytes;
}

template <bool GATHER_A>
constexpr int gemm_threads() {
  return 384;
}

template <int BN, int EPI, int STAGES, bool GATHER_A = false>
__global__ void __launch_bounds__(gemm_threads<GATHER_A>(), 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB0,
                        const __grid_constant__ CUtensorMap tmB1, const GemmArgs args) {
  using L = GemmSmem<BN, STAGES, gemm_out_bytes<EPI, GATHER_A>()>;
  constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  static_assert(kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512,
                "TMEM allocation must be a power of 2 of at least 32 columns");

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
  uint64_t* gat = drain + 1;  // GATHER_A: the loaders' copies of a stage have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gat + STAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], GATHER_A ? 2 : 1);  // TMA (+ the forwarder)
      mbar_init(&empty[s], 1);
      mbar_init(&gat[s], kGatherWarps * 32);  // the copies of every loader thread
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], epi_warps<GATHER_A>());  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    if (!GATHER_A) tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB0);
    if (EPI == kEpiSwiGLU) tma_prefetch_desc(&tmB1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  int num_tiles = args.num_tiles != nullptr ? *args.num_tiles : args.max_tiles;
  num_tiles = max(0, min(num_tiles, args.max_tiles));
  const int total = num_tiles * args.n_tiles;
  const uint32_t stage_tx =
      static_cast<uint32_t>((GATHER_A ? 0 : L::kABytes) + args.b_rows * kBK * 2);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < total; w += gridDim.x) {
        const int mt = w / args.n_tiles;
        const int nt = w - mt * args.n_tiles;
        const int4 t = load_tile(args, mt);
        if (t.x < 0 || t.x >= args.num_experts || t.y < 0 || t.z > args.a_rows || t.y >= t.z ||
            t.z - t.y > kBM) {
          record_status(args.status, t.x < 0 || t.x >= args.num_experts ? kErrBadExpert : kErrBadRow);
          *abort_flag = 1;
          break;
        }
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, args.status, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], stage_tx);
          if (!GATHER_A) tma_load_2d(sA + s * L::kABytes, &tmA, &full[s], kb * kBK, t.y);
          uint8_t* b = sB + s * L::kBBytes;
          if (EPI == kEpiSwiGLU) {
            tma_load_3d(b, &tmB0, &full[s], kb * kBK, nt * (BN / 2), t.x);
            tma_load_3d(b + L::kBBytes / 2, &tmB1, &full[s], kb * kBK, nt * (BN / 2), t.x);
          } else {
            tma_load_3d(b, &tmB0, &full[s], kb * kBK, nt * BN, t.x);
          }
          ++issued;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (*abort_flag) {
        // Let every copy still in flight land before the CTA exits.
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
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(kBM, static_cast<uint32_t>(args.b_rows));
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < total; w += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_ph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag, args.status, kErrTimeoutAccEmpty))
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
            tc_mma_bf16(d, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(&acc_full[acc]);
      }
      // Every MMA issued by this thread has finished once `drain` completes.
      tc_commit(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
  } else if (GATHER_A && warp >= kGatherWarp0) {
    // ---------------------------------------------------------- A-row loaders
    // Thread g = 0..127 copies 16-byte chunk (g % 8) of tile rows (g / 8) + 16 j,
    // j = 0..7: lanes 8m..8m+7 of a warp read one row's 128 contiguous bytes.
    const int g = threadIdx.x - kGatherWarp0 * 32;
    const uint32_t chunk = static_cast<uint32_t>(g & 7);
    const int row0 = g >> 3;  // 0..15
    const int K = args.num_kb * kBK;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < total; w += gridDim.x) {
      const int mt = w / args.n_tiles;
      const int4 t = load_tile(args, mt);
      const __nv_bfloat16* src[8];
      uint32_t nbytes = 0;  // bit j set: row j present
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int p = t.y + row0 + 16 * j;
        src[j] = args.a_src;  // any valid address when the row is absent (zero-filled)
        if (p < t.z) {
          const int i = args.a_index != nullptr ? args.a_index[p] / args.a_index_div : p;
          if (i >= 0 && i < args.a_src_rows) {
            src[j] = args.a_src + static_cast<size_t>(i) * K + chunk * 8;
            nbytes |= 1u << j;
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
        const uint32_t base = smem_u32(sA + s * L::kABytes);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t r = static_cast<uint32_t>(row0 + 16 * j);
          const uint32_t dst = base + r * 128u + ((chunk ^ (r & 7u)) << 4);
          const bool have = (nbytes >> j) & 1u;
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
  } else if (GATHER_A && warp == kForwardWarp) {
    if (lane == 0) {
      // -------------------------------------------------------- forwarder
      // A stage's A rows are complete once every loader thread's copies have
      // landed (gat); the proxy fence then makes them visible to the tensor
      // core's async proxy and the stage barrier hears of it.
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < total; w += gridDim.x) {
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&gat[s], ph, abort_flag, args.status, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();
          mbar_arrive(&full[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp >= 4 && warp < 4 + epi_warps<GATHER_A>()) {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter owned by this warp
    constexpr int kHalves = epi_warps<GATHER_A>() / 4;
    const int half = (warp - 4) >> 2;       // which share of the columns (0 or 0/1)
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int it = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_ph = (it >> 1) & 1;
      const int mt = w / args.n_tiles;
      const int nt = w - mt * args.n_tiles;
      const int4 t = load_tile(args, mt);
      const int row = t.y + q * 32 + lane;
      const bool valid = row < t.z;
      // Store epilogue: the output row and its scale do not depend on the
      // accumulator, so their loads overlap the wait for it.
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
      }
      bool ok = mbar_wait(&acc_full[acc], acc_ph, abort_flag, args.status, kErrTimeoutAccFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + static_cast<uint32_t>(acc * BN) + lane_off;

      if constexpr (EPI == kEpiSwiGLU || EPI == kEpiStore) {
        epilogue_tile<BN, EPI, kHalves>(args, tb, row, valid, st, orow_idx, scale, nt, half,
                                        sOut + (warp - 4) * kEpiStageBytes, lane);
      } else if constexpr (EPI == kEpiAtomic) {
        epilogue_tile_atomic<BN, kHalves>(args, tb, st, orow_idx, scale, nt, half,
                                          sOut + (warp - 4) * kEpiStageBytes, lane);
      } else {
        if (half == 0) {  // one warp per lane quarter: rows are not split by columns
          // Router: the row's E logits -> bf16 -> top-k (value desc, id asc) -> softmax.
          const int E = args.b_rows;
          uint32_t top[kRouterMaxK];
  #pragma unroll
          for (int i = 0; i < kRouterMaxK; ++i) top[i] = 0u;  // below every real key
          float run_max = -INFINITY, run_sum = 0.0f;  // softmax over all E (norm_topk_prob=False)
  #pragma unroll 1
          for (int c0 = 0; c0 < E; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tb + c0, r);
            tc_wait_ld();
            float lv[16];
  #pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v = __uint_as_float(r[j]);
              if (args.bias != nullptr) v += args.bias[c0 + j];
              lv[j] = bf16_round_f(v);
            }
            if (valid && args.logits_out != nullptr) {
              uint4* dst = reinterpret_cast<uint4*>(args.logits_out + static_cast<size_t>(row) * E + c0);
              dst[0] = make_uint4(pack_bf16x2(lv[0], lv[1]), pack_bf16x2(lv[2], lv[3]),
                                  pack_bf16x2(lv[4], lv[5]), pack_bf16x2(lv[6], lv[7]));
              dst[1] = make_uint4(pack_bf16x2(lv[8], lv[9]), pack_bf16x2(lv[10], lv[11]),
                                  pack_bf16x2(lv[12], lv[13]), pack_bf16x2(lv[14], lv[15]));
            }
  #pragma unroll
            for (int j = 0; j < 16; ++j) {
              topk_insert(top, topk_key(lv[j], c0 + j));
              if (!args.norm_topk_prob) {
                const float m = fmaxf(run_max, lv[j]);
                run_sum = run_sum * expf(run_max - m) + expf(lv[j] - m);
                run_max = m;
              }
            }
          }
          if (valid) {
            const int k = args.top_k;
            float tv[kRouterMaxK];
            int ti[kRouterMaxK];
  #pragma unroll
            for (int i = 0; i < kRouterMaxK; ++i) {
              tv[i] = topk_key_value(top[i]);
              ti[i] = topk_key_id(top[i]);
            }
            float den = 0.0f, ref = tv[0];
            if (args.norm_topk_prob) {
  #pragma unroll
              for (int i = 0; i < kRouterMaxK; ++i)
                if (i < k) den += expf(tv[i] - ref);
            } else {
              den = run_sum;
              ref = run_max;
            }
            const float inv = 1.0f / den;
  #pragma unroll
            for (int i = 0; i < kRouterMaxK; ++i) {
              if (i < k) {
                args.ids_out[static_cast<size_t>(row) * k + i] = ti[i];
                args.w_out[static_cast<size_t>(row) * k + i] = expf(tv[i] - ref) * inv;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace moe
