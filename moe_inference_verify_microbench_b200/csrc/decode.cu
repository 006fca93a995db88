// Small-batch (decode) kernels of the MoE layer.  At a few routing records per
// expert the layer is a stream of the routed experts' weights; a 128-row
// tensor-core tile would idle there, so these kernels stream weight rows
// through shared memory with the bulk-copy engine and apply each row to all
// records of its expert on the CUDA cores.
//
//   router_sort_small  one 8-CTA cluster.  Each CTA stages the T tokens in shared
//                      memory; each warp holds one expert's router row in
//                      registers and dots it with every token; the logits meet in
//                      CTA 0's shared memory over distributed shared memory; CTA 0
//                      takes the top-k per token (one warp per token, same key
//                      order as the tensor-core router: value descending, lower
//                      expert id first) and, when asked, runs the one-CTA sort of
//                      sort_block.cuh on the fresh ids, so router + sort_align is
//                      one launch (C5/python/solution.py:124-136).
//   gemv_stream<true>  h[p] = silu(A[p] . Wg[e]) * (A[p] . Wu[e]), A[p] =
//                      src[index[p] / index_div] (C5/python/solution.py:79-80)
//   gemv_stream<false> out[row_map[p]] = row_scale[row_map[p]] * (h[p] . Wd[e])
//                      (C5/python/solution.py:80,158)
//
// gemv_stream is persistent, one CTA per SM.  Work item = (tile of the sort's
// tile table, block of output rows); every CTA takes a contiguous
// range of items, computed on the device from the tile count, so the host never
// synchronises.  One producer thread copies each item's weight rows (contiguous
// in memory: rows rb*B..rb*B+B-1 of expert e) into a ring of shared-memory
// stages; eight consumer warps own one output row each and dot it with the
// item's records (A rows read through L1).
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>

#include "grouped_gemm.cuh"
#include "internal.h"
#include "sort_block.cuh"

namespace cg = cooperative_groups;

namespace moe {

constexpr int kRouterCluster = 8;
constexpr int kRouterThreads = kSortThreads;  // CTA 0 also runs the one-CTA sort
constexpr int kRouterWarps = kRouterThreads / 32;
constexpr int kRouterSmallMaxT = 16;
constexpr int kRouterMaxVecPerLane = 16;      // H <= 32 * 16 * 8 = 4096
constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = 32 * (kGemvConsumerWarps + 1);  // + one producer warp
// Output rows per work item: one per consumer warp for the gate/up pair, four
// for the down projection (whose rows are short).
template <bool SWIGLU>
constexpr int gemv_rows_per_warp() {
  return SWIGLU ? 1 : 4;
}
template <bool SWIGLU>
constexpr int gemv_row_block() {
  return kGemvConsumerWarps * gemv_rows_per_warp<SWIGLU>();
}
constexpr int kGemvMaxRecs = 8;     // records sharing one pass over a weight row
constexpr int kGemvRingBytes = 192 * 1024;
constexpr int kGemvMaxStages = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Mixed-precision FMA: fma.rn.f32.bf16 multiplies two bf16 values exactly and
// adds them to an fp32 accumulator with one rounding, so weights and
// activations are used as stored, without conversion instructions.
__device__ __forceinline__ void fma_bf16x2(float& lo, float& hi, uint32_t w, uint32_t x) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %2;\n\t"
      "mov.b32 {xl, xh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.bf16 %1, wh, xh, %1;\n\t}"
      : "+f"(lo), "+f"(hi)
      : "r"(w), "r"(x));
}

// acc[0..3] += the 8-element dot product of w and x, over four dependency chains.
__device__ __forceinline__ void dot8_acc(const uint4& w, const uint4& x, float* acc) {
  fma_bf16x2(acc[0], acc[1], w.x, x.x);
  fma_bf16x2(acc[2], acc[3], w.y, x.y);
  fma_bf16x2(acc[0], acc[1], w.z, x.z);
  fma_bf16x2(acc[2], acc[3], w.w, x.w);
}

__device__ __forceinline__ float acc_sum(const float* acc) {
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// ------------------------------------------------------------------ router

__global__ void __cluster_dims__(kRouterCluster, 1, 1) __launch_bounds__(kRouterThreads, 1)
    router_sort_small(const uint4* __restrict__ x, const uint4* __restrict__ wr,
                      const float* __restrict__ bias, int T, int vec_per_row, int E, int k,
                      int norm_topk_prob, int* __restrict__ ids_out, float* __restrict__ w_out,
                      __nv_bfloat16* __restrict__ logits_out, int* counts, int* offsets,
                      int* perm, int4* tiles, int max_tiles, int* num_tiles, int* status) {
  __shared__ float logits[kRouterSmallMaxT * kSortThreads];  // [expert][token], rank 0 only
  __shared__ int sid[kRouterSmallMaxT * kRouterMaxK];
  extern __shared__ __align__(16) uint4 dyn[];
  uint4* xs = dyn;                                            // [T][vec_per_row]
  int* sort_sm = reinterpret_cast<int*>(dyn + static_cast<size_t>(T) * vec_per_row);
  cg::cluster_group cluster = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_cta = E / kRouterCluster;
  // The router rows are weights, not outputs of an earlier kernel: the first
  // expert row of each warp is loaded before waiting for the predecessor.
  uint4 wv[kRouterMaxVecPerLane];
  auto load_row = [&](int el) {
    const uint4* row =
        wr + (static_cast<size_t>(cluster.block_rank()) * per_cta + el) * vec_per_row;
#pragma unroll
    for (int j = 0; j < kRouterMaxVecPerLane; ++j) {
      const int v = lane + 32 * j;
      wv[j] = v < vec_per_row ? __ldg(row + v) : make_uint4(0, 0, 0, 0);
    }
  };
  if (warp < per_cta) load_row(warp);
  pdl_wait();
  pdl_trigger();
  {
    const int n = T * vec_per_row;
    int i = threadIdx.x;
    for (; i + 3 * kRouterThreads < n; i += 4 * kRouterThreads) {  // four loads in flight
      const uint4 v0 = __ldg(x + i), v1 = __ldg(x + i + kRouterThreads);
      const uint4 v2 = __ldg(x + i + 2 * kRouterThreads), v3 = __ldg(x + i + 3 * kRouterThreads);
      xs[i] = v0;
      xs[i + kRouterThreads] = v1;
      xs[i + 2 * kRouterThreads] = v2;
      xs[i + 3 * kRouterThreads] = v3;
    }
    for (; i < n; i += kRouterThreads) xs[i] = __ldg(x + i);
  }
  __syncthreads();

  // Warp = one expert row held in registers; tokens one by one.
  float* dst = cluster.map_shared_rank(logits, 0);
  for (int el = warp; el < per_cta; el += kRouterWarps) {
    const int e = static_cast<int>(cluster.block_rank()) * per_cta + el;
    if (el != warp) load_row(el);
    const float be = bias != nullptr ? bias[e] : 0.0f;
#pragma unroll 1
    for (int t = 0; t < T; ++t) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const uint4* xr = xs + t * vec_per_row;
#pragma unroll
      for (int j = 0; j < kRouterMaxVecPerLane; ++j) {
        const int v = lane + 32 * j;
        if (v < vec_per_row) dot8_acc(wv[j], xr[v], acc);
      }
      const float sum = warp_sum(acc_sum(acc));
      if (lane == 0) {
        const float b = bf16_round_f(sum + be);
        dst[e * T + t] = b;
        if (logits_out != nullptr) logits_out[static_cast<size_t>(t) * E + e] = __float2bfloat16_rn(b);
      }
    }
  }
  cluster.sync();  // every CTA's logits are in CTA 0's shared memory
  if (cluster.block_rank() != 0) return;

  for (int t = warp; t < T; t += kRouterWarps) {
    uint32_t top[kRouterMaxK];
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) top[i] = 0u;  // below every real key
    for (int c = lane; c < E; c += 32) topk_insert(top, topk_key(logits[c * T + t], c));
    uint32_t sel[kRouterMaxK];
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) {
      // Keys are unique (the id is part of the key): exactly one lane holds the max.
      const uint32_t m = __reduce_max_sync(0xffffffffu, top[0]);
      sel[i] = m;
      if (top[0] == m) {
#pragma unroll
        for (int j = 0; j + 1 < kRouterMaxK; ++j) top[j] = top[j + 1];
        top[kRouterMaxK - 1] = 0u;
      }
    }
    const float ref = topk_key_value(sel[0]);
    float den = 0.0f;
    if (norm_topk_prob) {
#pragma unroll
      for (int i = 0; i < kRouterMaxK; ++i)
        if (i < k) den += expf(topk_key_value(sel[i]) - ref);
    } else {
      for (int c = lane; c < E; c += 32) den += expf(logits[c * T + t] - ref);
      den = warp_sum(den);
    }
    const float inv = 1.0f / den;
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) {
      if (i < k && lane == i) {
        const int id = topk_key_id(sel[i]);
        ids_out[t * k + i] = id;
        w_out[t * k + i] = expf(topk_key_value(sel[i]) - ref) * inv;
        sid[t * k + i] = id;
      }
    }
  }
  if (perm == nullptr) return;  // block-uniform: router only
  __syncthreads();
  sort_small_block(sid, T * k, E, 0, E, kBM, counts, offsets, nullptr, perm, nullptr, tiles,
                   max_tiles, num_tiles, status, sort_sm);
}

// ------------------------------------------------------------------ streamed GEMV

struct StreamArgs {
  const uint4* act;      // A operand rows [act_rows][K]
  int act_rows;
  const int* index;      // A row of record p = act[index[p] / index_div] (null = p)
  int index_div;
  int M;                 // records
  const int4* tiles;
  const int* num_tiles;
  int max_tiles;
  const __nv_bfloat16* w0;  // [E][N][K]: gate (SwiGLU) or down weight
  const __nv_bfloat16* w1;  // [E][N][K]: up (SwiGLU only)
  int E, K, N;
  __nv_bfloat16* out;
  const int* row_map;       // down: out row of record p (null = p)
  const float* row_scale;   // down: scale indexed by the out row (null = 1)
  int out_rows;
  int stages;
  int* status;
  // Gate/up only: the down weights [E][next_N][next_K] of the same experts,
  // prefetched into L2 once this CTA has issued its own copies, when the
  // active experts' down weights fit comfortably in L2 (decode).
  const __nv_bfloat16* next_w;
  int next_N, next_K;
};

constexpr long long kPrefetchMaxBytes = 64ll << 20;  // half of the 126 MB L2
constexpr int kPrefetchRows = 32;                    // down rows per prefetch request

// One warp's pass over ROWS weight rows of a stage (row j at w + j * rstride,
// in uint4 units) for n <= NR records whose A rows are act[rows[r]], over CH
// dependency chains per (row, record).
// How the consumers read the A rows: the read-only path (inputs of the
// launch), through L2 (rows written earlier in the same launch by other
// CTAs), or a plain load (rows staged in this CTA's shared memory).
enum ActLoad : int { kActLdg = 0, kActL2 = 1, kActPlain = 2 };

template <int ROWS, int NR, int CH, int ACT = kActLdg>
__device__ __forceinline__ void stage_dots(const uint4* w, int rstride,
                                           const uint4* __restrict__ act, const int* rows, int n,
                                           int vec, int lane, float (&acc)[ROWS][NR][CH]) {
  static_assert(CH == 2 || CH == 4, "two or four chains");
#pragma unroll
  for (int j = 0; j < ROWS; ++j)
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int c = 0; c < CH; ++c) acc[j][r][c] = 0.0f;
#pragma unroll 2
  for (int v = lane; v < vec; v += 32) {
    uint4 wv[ROWS];
#pragma unroll
    for (int j = 0; j < ROWS; ++j) wv[j] = w[j * rstride + v];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      if (r < n) {
        const uint4* xp = act + static_cast<size_t>(rows[r]) * vec + v;
        const uint4 xv = ACT == kActLdg ? __ldg(xp) : ACT == kActL2 ? __ldcg(xp) : *xp;
#pragma unroll
        for (int j = 0; j < ROWS; ++j) {
          float* c = acc[j][r];
          fma_bf16x2(c[0], c[1], wv[j].x, xv.x);
          fma_bf16x2(c[CH - 2], c[CH - 1], wv[j].y, xv.y);
          fma_bf16x2(c[0], c[1], wv[j].z, xv.z);
          fma_bf16x2(c[CH - 2], c[CH - 1], wv[j].w, xv.w);
        }
      }
    }
  }
}

// Warp reduction of v[j][r] over the 32 lanes, scattered over records: after
// it, v[j][0] of lane L holds the full sum for record reduced_record<NR>(L),
// for every row j.  Halving steps exchange half of the remaining records with
// the lane `o` apart (ROWS * (NR - 1) shuffles in all), then plain butterfly
// steps finish the sums.
template <int NR>
__device__ __forceinline__ int reduced_record(int lane) {
  int r = 0;
#pragma unroll
  for (int k = 0; (NR >> k) > 1; ++k)
    if (lane & (16 >> k)) r += NR >> (k + 1);
  return r;
}

template <int ROWS, int NR>
__device__ __forceinline__ void reduce_records(float (&v)[ROWS][NR], int lane) {
#pragma unroll
  for (int k = 0; (NR >> k) > 1; ++k) {
    const int h = NR >> (k + 1);
    const int o = 16 >> k;
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < ROWS; ++j)
#pragma unroll
      for (int i = 0; i < NR / 2; ++i) {
        if (i < h) {
          const float keep = upper ? v[j][i + h] : v[j][i];
          const float send = upper ? v[j][i] : v[j][i + h];
          v[j][i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
  }
#pragma unroll
  for (int o = 16 / NR; o >= 1; o >>= 1)
#pragma unroll
    for (int j = 0; j < ROWS; ++j) v[j][0] += __shfl_xor_sync(0xffffffffu, v[j][0], o);
}

// Gate/up: rows 0 and 1 are the gate and up rows of output row `row`; down:
// rows j = 0..ROWS-1 are output rows row + j * kGemvConsumerWarps.  Both sit
// kGemvConsumerWarps rows apart in the stage.
template <bool SWIGLU, int NR, int ACT = kActLdg>
__device__ __forceinline__ void gemv_pass(const StreamArgs& a, const uint4* w, int p0, int n,
                                          int row, const int* rows, int my_out, float my_scale,
                                          int bad, int vec, int lane) {
  constexpr int ROWS = SWIGLU ? 2 : gemv_rows_per_warp<false>();
  constexpr int CH = ROWS * NR >= 16 ? 2 : 4;
  float acc[ROWS][NR][CH];
  stage_dots<ROWS, NR, CH, ACT>(w, kGemvConsumerWarps * vec, a.act, rows, n, vec, lane, acc);
  float v[ROWS][NR];
#pragma unroll
  for (int j = 0; j < ROWS; ++j)
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float t = acc[j][r][0] + acc[j][r][1];
      if (CH == 4) t += acc[j][r][CH - 2] + acc[j][r][CH - 1];
      v[j][r] = t;
    }
  reduce_records<ROWS, NR>(v, lane);
  const int r = reduced_record<NR>(lane);
  const int o = __shfl_sync(0xffffffffu, my_out, r);
  const float sc = __shfl_sync(0xffffffffu, my_scale, r);
  const int rbad = __shfl_sync(0xffffffffu, bad, r);
  const bool writer = (lane & (32 / NR - 1)) == 0 && r < n && !rbad;
  if (writer) {
    if (SWIGLU) {
      a.out[static_cast<size_t>(p0 + r) * a.N + row] = __float2bfloat16_rn(silu_f(v[0][0]) * v[1][0]);
    } else {
#pragma unroll
      for (int j = 0; j < ROWS; ++j)
        a.out[static_cast<size_t>(o) * a.N + row + j * kGemvConsumerWarps] =
            __float2bfloat16_rn(v[j][0] * sc);
    }
  }
}

// Cost of one work item of a tile, in units of one record's dot products: the
// weight rows stream at a fixed cost, each record of the tile adds one unit.
constexpr long long kItemCost0 = 4;

__device__ __forceinline__ long long item_cost(const StreamArgs& a, int i) {
  const int4 t = a.tiles[i];
  const int n = (t.z > t.y && t.y >= 0) ? min(t.z - t.y, a.M) : 0;  // bad tiles are reported later
  return kItemCost0 + n;
}

// Inclusive scan of v over the block (every thread calls it); *total gets the
// block's sum.
__device__ __forceinline__ long long block_scan_ll(long long v, long long* sh, long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    long long w = lane < nw ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) sh[lane] = w;
  }
  __syncthreads();
  const long long res = v + (warp > 0 ? sh[warp - 1] : 0);
  *total = sh[nw - 1];
  __syncthreads();
  return res;
}

// This CTA's contiguous item range [*lo, *hi): items are ordered (tile, row
// block) and the ranges split the summed item cost evenly over the grid, so a
// CTA that meets tiles with many records gets fewer items.
__device__ __forceinline__ void balanced_range(const StreamArgs& a, int nt, int blocks, long long* lo,
                               long long* hi) {
  __shared__ long long sh_scan[32];
  __shared__ long long sh_range[2];
  const long long total_items = static_cast<long long>(nt) * blocks;
  if (threadIdx.x == 0) sh_range[0] = sh_range[1] = total_items;
  const int nthr = blockDim.x;
  long long C = 0;
  long long my_cost = 0;  // item cost of this thread's tile when nt <= nthr
  if (nt <= nthr) {
    my_cost = static_cast<int>(threadIdx.x) < nt ? item_cost(a, threadIdx.x) : 0;
  } else {
    long long mine = 0;
    for (int i = threadIdx.x; i < nt; i += nthr) mine += item_cost(a, i) * blocks;
    block_scan_ll(mine, sh_scan, &C);
  }
  long long carry = 0;
  for (int base = 0; base < nt; base += nthr) {
    const int i = base + static_cast<int>(threadIdx.x);
    const long long ci = nt <= nthr ? my_cost : (i < nt ? item_cost(a, i) : 0);
    long long chunk = 0;
    const long long incl = block_scan_ll(ci * blocks, sh_scan, &chunk) + carry;
    if (nt <= nthr) C = chunk;  // one chunk: its total is the grand total
    const long long excl = incl - ci * blocks;
    const long long lo_c = C * blockIdx.x / gridDim.x;
    const long long hi_c = C * (blockIdx.x + 1) / gridDim.x;
    if (i < nt) {
      if (excl <= lo_c && lo_c < incl) sh_range[0] = static_cast<long long>(i) * blocks + (lo_c - excl + ci - 1) / ci;
      if (excl <= hi_c && hi_c < incl) sh_range[1] = static_cast<long long>(i) * blocks + (hi_c - excl + ci - 1) / ci;
    }
    carry += chunk;
  }
  __syncthreads();
  *lo = sh_range[0];
  *hi = sh_range[1];
}

// The work items [lo, hi) of a streamed GEMV on this CTA: the producer warp's
// lane 0 copies each item's weight rows into the ring `smem_raw` (a.stages
// stages, barriers full/empty, each used from phase 0), the consumer warps
// apply them.  Every thread of the CTA calls it; `nt` is the tile count.
// ACT: how the consumers read the A rows (ActLoad).
// The producer side of stream_items: lane 0 of the calling warp copies the
// weight rows of items [lo, hi) into the ring (a.stages stages, barriers
// full/empty, each used from phase 0) and, for the gate/up GEMV, prefetches
// the next GEMM's weights into L2 behind them.
template <bool SWIGLU>
__device__ __forceinline__ void produce_items(const StreamArgs& a, uint8_t* smem_raw,
                                              uint64_t* full, uint64_t* empty,
                                              volatile int* abort_flag, int nt, long long lo,
                                              long long hi) {
  const int lane = threadIdx.x & 31;
  constexpr int kRB = gemv_row_block<SWIGLU>();
  const uint32_t mat_bytes = static_cast<uint32_t>(kRB) * a.K * 2;  // one matrix's rows
  const uint32_t stage_bytes = (SWIGLU ? 2u : 1u) * mat_bytes;
  const int blocks = a.N / kRB;
  if (lane == 0) {
    int s = 0;
    uint32_t ph = 0, issued = 0;
    for (long long w = lo; w < hi; ++w) {
      const int ti = static_cast<int>(w / blocks);
      const int rb = static_cast<int>(w - static_cast<long long>(ti) * blocks);
      const int4 t = a.tiles[ti];
      if (t.x < 0 || t.x >= a.E || t.y < 0 || t.y > t.z || t.z > a.M) break;  // consumers report
      if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.status, kErrTimeoutEmpty)) break;
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      const size_t row0 = (static_cast<size_t>(t.x) * a.N + static_cast<size_t>(rb) * kRB) * a.K;
      uint8_t* dst = smem_raw + s * stage_bytes;
      bulk_load(dst, a.w0 + row0, mat_bytes, &full[s]);
      if (SWIGLU) bulk_load(dst + mat_bytes, a.w1 + row0, mat_bytes, &full[s]);
      ++issued;
      if (++s == a.stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    if (SWIGLU && a.next_w != nullptr && !*abort_flag) {
      // This CTA's share of the next GEMM's weights, in kPrefetchRows-row
      // requests, so the down projection streams from L2.  Issued after
      // this GEMM's own copies, which are on the critical path (issuing the
      // prefetch first measured slower at T=1 and 2).
      const int nblk = a.next_N / kPrefetchRows;
      const long long bytes_all =
          static_cast<long long>(nt) * a.next_N * a.next_K * static_cast<long long>(2);
      if (nblk > 0 && bytes_all <= kPrefetchMaxBytes) {
        const long long total2 = static_cast<long long>(nt) * nblk;
        const long long p_lo = total2 * blockIdx.x / gridDim.x;
        const long long p_hi = total2 * (blockIdx.x + 1) / gridDim.x;
        const uint32_t req = static_cast<uint32_t>(kPrefetchRows) * a.next_K * 2;
        for (long long q = p_lo; q < p_hi; ++q) {
          const int ti = static_cast<int>(q / nblk);
          const int rb = static_cast<int>(q - static_cast<long long>(ti) * nblk);
          const int e = a.tiles[ti].x;
          if (e < 0 || e >= a.E) continue;
          prefetch_l2_bulk(a.next_w + (static_cast<size_t>(e) * a.next_N +
                                       static_cast<size_t>(rb) * kPrefetchRows) * a.next_K,
                           req);
        }
      }
    }
    if (*abort_flag) {
      // Let every copy still in flight land before the CTA exits.
      const uint32_t first = issued > static_cast<uint32_t>(a.stages) ? issued - a.stages : 0u;
      for (uint32_t i = first; i < issued; ++i) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[i % a.stages], (i / a.stages) & 1u)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
  }
}

template <bool SWIGLU, int ACT = kActLdg>
__device__ __forceinline__ void stream_items(const StreamArgs& a, uint8_t* smem_raw, uint64_t* full,
                             uint64_t* empty, volatile int* abort_flag, int nt, long long lo,
                             long long hi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vec = a.K / 8;
  constexpr int kRB = gemv_row_block<SWIGLU>();
  const uint32_t mat_bytes = static_cast<uint32_t>(kRB) * a.K * 2;  // one matrix's rows
  const uint32_t stage_bytes = (SWIGLU ? 2u : 1u) * mat_bytes;
  const int blocks = a.N / kRB;

  if (warp == kGemvConsumerWarps) {
    produce_items<SWIGLU>(a, smem_raw, full, empty, abort_flag, nt, lo, hi);
    return;  // the producer warp has no consumer work
  }

  // -------------------------------------------------------------- consumers
  // Lane r < n holds record p0 + r's A row, out row and scale; a tile of at
  // most kGemvMaxRecs records keeps them across its items.
  int cached_ti = -1;
  int my_row = 0, my_out = 0, bad = 0;
  float my_scale = 1.0f;
  auto fetch = [&](int p0, int n) {
    my_row = my_out = bad = 0;
    my_scale = 1.0f;
    if (lane < n) {
      const int p = p0 + lane;
      if (SWIGLU) {
        my_row = a.index != nullptr ? a.index[p] / a.index_div : p;
        bad = my_row < 0 || my_row >= a.act_rows;
        if (bad) my_row = 0;
      } else {
        my_row = p;
        my_out = a.row_map != nullptr ? a.row_map[p] : p;
        bad = my_out < 0 || my_out >= a.out_rows;
        if (!bad && a.row_scale != nullptr) my_scale = a.row_scale[my_out];
      }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) record_status(a.status, kErrBadRow);
  };
  int s = 0;
  uint32_t ph = 0;
  for (long long w = lo; w < hi; ++w) {
    const int ti = static_cast<int>(w / blocks);
    const int rb = static_cast<int>(w - static_cast<long long>(ti) * blocks);
    const int4 t = a.tiles[ti];
    if (t.x < 0 || t.x >= a.E || t.y < 0 || t.y > t.z || t.z > a.M) {
      if (threadIdx.x == 0) record_status(a.status, t.x < 0 || t.x >= a.E ? kErrBadExpert : kErrBadRow);
      break;
    }
    const bool single = t.z - t.y <= kGemvMaxRecs;
    if (!single || ti != cached_ti) {
      fetch(t.y, min(kGemvMaxRecs, t.z - t.y));
      cached_ti = single ? ti : -1;
    }
    if (!mbar_wait(&full[s], ph, abort_flag, a.status, kErrTimeoutFull)) break;
    const uint4* w0 = reinterpret_cast<const uint4*>(smem_raw + s * stage_bytes) + warp * vec;
    const int row = rb * kRB + warp;  // this warp's (first) output row
    for (int p0 = t.y; p0 < t.z; p0 += kGemvMaxRecs) {
      const int n = min(kGemvMaxRecs, t.z - p0);
      if (p0 != t.y) fetch(p0, n);
      int rows[kGemvMaxRecs];
#pragma unroll
      for (int r = 0; r < kGemvMaxRecs; ++r) rows[r] = __shfl_sync(0xffffffffu, my_row, r);
      if (n == 1)
        gemv_pass<SWIGLU, 1, ACT>(a, w0, p0, n, row, rows, my_out, my_scale, bad, vec, lane);
      else if (n == 2)
        gemv_pass<SWIGLU, 2, ACT>(a, w0, p0, n, row, rows, my_out, my_scale, bad, vec, lane);
      else if (n <= 4)
        gemv_pass<SWIGLU, 4, ACT>(a, w0, p0, n, row, rows, my_out, my_scale, bad, vec, lane);
      else
        gemv_pass<SWIGLU, 8, ACT>(a, w0, p0, n, row, rows, my_out, my_scale, bad, vec, lane);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == a.stages) {
      s = 0;
      ph ^= 1u;
    }
  }
}

template <bool SWIGLU>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_stream(const StreamArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  constexpr int kRB = gemv_row_block<SWIGLU>();
  const uint32_t stage_bytes = (SWIGLU ? 2u : 1u) * static_cast<uint32_t>(kRB) * a.K * 2;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + a.stages * stage_bytes);
  uint64_t* empty = full + kGemvMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kGemvMaxStages);
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  const int nt = max(0, min(*a.num_tiles, a.max_tiles));
  long long lo, hi;
  balanced_range(a, nt, a.N / kRB, &lo, &hi);
  stream_items<SWIGLU>(a, smem_raw, full, empty, abort_flag, nt, lo, hi);
}

// ------------------------------------------------------------------ single-launch decode layer
//
// decode_layer_fused: the whole MoE layer for at most kFusedMaxRecs routing
// records (T * k <= 64: T <= 8 tokens at top-8) in one cooperative launch of
// one CTA per SM, the phases separated by grid-wide barriers:
//   1  router logits, one expert per CTA (the arithmetic of router_sort_small)
//   -  barrier
//   2  every CTA takes the top-k of every token from the logits and sorts the
//      records by expert (stable; one tile per expert) in its shared memory
//   3  gate/up + SwiGLU as gemv_stream<true>, the down weights of the routed
//      experts prefetched into L2 behind this CTA's own copies
//   -  barrier
//   4  down projection with the routing weights as gemv_stream<false>, to the
//      slot rows n*k + j
//   -  barrier
//   5  y[n] = sum_j slots[n*k + j] in fp32 in slot order (combine_rows)
// Four launches (router + sort, two GEMVs, combine) become one: no launch
// gaps, no kernel start-up or tail between the steps, the router spread over
// 128 SMs instead of one 8-CTA cluster.  Every phase does the arithmetic of
// the kernel it replaces, so the output is bitwise that of the four-launch
// path.  The grid barriers count arrivals on counters the launcher zeroes;
// every wait is bounded (kErrTimeoutGrid), and a CTA that gives up skips the
// rest of the layer.

constexpr int kFusedMaxRecs = 64;  // routing records of the single-launch layers (T*k)

struct DecodeArgs {
  const uint4* x;          // [T][H]
  const uint4* wr;         // [E][H]
  const float* bias;       // [E] or null
  int T, H, I, E, k, norm_topk_prob;
  const __nv_bfloat16* w_gate;
  const __nv_bfloat16* w_up;
  const __nv_bfloat16* w_down;
  float* logits;           // scratch [T][E]
  __nv_bfloat16* h;        // scratch [T*k][I]
  __nv_bfloat16* slots;    // scratch [T*k][H]
  unsigned int* bar;       // three counters, zero at launch
  uint4* y;                // [T][H]
  int stages3, stages4;
  int* status;
};

// All CTAs of the grid arrive on *ctr and wait until gridDim.x have arrived.
// False (and the CTA's abort flag raised) once the bounded wait gives up or
// the CTA has aborted before.
__device__ bool grid_barrier(unsigned int* ctr, volatile int* abort_flag, int* status) {
  __syncthreads();
  if (threadIdx.x == 0 && !*abort_flag) {
    __threadfence();
    atomicAdd(ctr, 1u);
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= gridDim.x) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(status, kErrTimeoutGrid);
        *abort_flag = 1;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
  }
  __syncthreads();
  return *abort_flag == 0;
}

// Phases 1 and 2 of the single-launch layers, run by every thread of every
// CTA: the router logits (one expert per CTA, the arithmetic of
// router_sort_small) to `logits`, a grid barrier on *bar, then in every CTA
// the top-k of every token and the stable sort of the T * k records by expert
// (one tile per expert) into rs.  False when the barrier gave up.
struct RouteSmem {
  int ids[kFusedMaxRecs];
  int first[kFusedMaxRecs];    // 1: the record opens its expert's tile
  float w[kFusedMaxRecs];      // routing weight of slot n*k + j
  int perm[kFusedMaxRecs];     // slot of the p-th record in expert order
  int pos[kFusedMaxRecs];      // position of slot s in expert order
  int tile_of[kFusedMaxRecs];  // tile of slot s
  int4 tiles[kFusedMaxRecs];
  int nt;
};

__device__ __forceinline__ bool route_and_sort(const uint4* __restrict__ x,
                                               const uint4* __restrict__ wr,
                                               const float* __restrict__ bias, int T, int H, int E,
                                               int k, int norm_topk_prob, float* logits,
                                               unsigned int* bar, volatile int* abort_flag,
                                               int* status, RouteSmem& rs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vec = H / 8, R = T * k;
  // ---------------------------------------------------------- 1: router logits
  if (warp == 0) {
    for (int e = blockIdx.x; e < E; e += gridDim.x) {
      const uint4* row = wr + static_cast<size_t>(e) * vec;
      const float be = bias != nullptr ? bias[e] : 0.0f;
      for (int t = 0; t < T; ++t) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint4* xr = x + static_cast<size_t>(t) * vec;
#pragma unroll
        for (int j = 0; j < kRouterMaxVecPerLane; ++j) {
          const int v = lane + 32 * j;
          if (v < vec) dot8_acc(__ldg(row + v), __ldg(xr + v), acc);
        }
        const float sum = warp_sum(acc_sum(acc));
        if (lane == 0) logits[t * E + e] = bf16_round_f(sum + be);
      }
    }
  }
  if (!grid_barrier(bar, abort_flag, status)) return false;

  // ------------------------------------------------- 2: top-k and the record sort
  for (int t = warp; t < T; t += static_cast<int>(blockDim.x >> 5)) {  // one warp per token
    const float* lg = logits + t * E;
    uint32_t top[kRouterMaxK];
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) top[i] = 0u;
    for (int c = lane; c < E; c += 32) topk_insert(top, topk_key(__ldcg(lg + c), c));
    uint32_t sel[kRouterMaxK];
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, top[0]);
      sel[i] = m;
      if (top[0] == m) {
#pragma unroll
        for (int j = 0; j + 1 < kRouterMaxK; ++j) top[j] = top[j + 1];
        top[kRouterMaxK - 1] = 0u;
      }
    }
    const float ref = topk_key_value(sel[0]);
    float den = 0.0f;
    if (norm_topk_prob) {
#pragma unroll
      for (int i = 0; i < kRouterMaxK; ++i)
        if (i < k) den += expf(topk_key_value(sel[i]) - ref);
    } else {
      for (int c = lane; c < E; c += 32) den += expf(__ldcg(lg + c) - ref);
      den = warp_sum(den);
    }
    const float inv = 1.0f / den;
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) {
      if (i < k && lane == i) {
        rs.ids[t * k + i] = topk_key_id(sel[i]);
        rs.w[t * k + i] = expf(topk_key_value(sel[i]) - ref) * inv;
      }
    }
  }
  __syncthreads();
  // Stable sort of the R <= kFusedMaxRecs records by expert, thread r =
  // slot r, over the ids in shared memory: a record's position counts the
  // records with a smaller id or the same id and a lower slot; one tile per
  // expert, ascending ids (the first record of an expert opens its tile).
  const int r = static_cast<int>(threadIdx.x);
  int my = 0x7fffffff, pos = 0, before = 0, same = 0;
  bool first = false;
  if (r < R) {
    my = rs.ids[r];
    first = true;
    for (int j = 0; j < R; ++j) {
      const int o = rs.ids[j];
      pos += (o < my || (o == my && j < r)) ? 1 : 0;
      before += o < my ? 1 : 0;
      same += o == my ? 1 : 0;
      if (o == my && j < r) first = false;
    }
    rs.first[r] = first ? 1 : 0;
  }
  __syncthreads();
  if (r < R) {
    int tile = 0, n_tiles = 0;
    for (int j = 0; j < R; ++j) {
      const bool f = rs.first[j] != 0;
      tile += (f && rs.ids[j] < my) ? 1 : 0;
      n_tiles += f ? 1 : 0;
    }
    rs.perm[pos] = r;
    rs.pos[r] = pos;
    rs.tile_of[r] = tile;
    if (first) rs.tiles[tile] = make_int4(my, before, before + same, 0);
    if (r == 0) rs.nt = n_tiles;
  }
  __syncthreads();
  return true;
}

__global__ void __launch_bounds__(kGemvThreads, 1) decode_layer_fused(const DecodeArgs d) {
  extern __shared__ __align__(128) uint8_t smem_raw[];  // ring, then both phases' barriers
  __shared__ RouteSmem rs;
  uint64_t* full3 = reinterpret_cast<uint64_t*>(smem_raw + kGemvRingBytes);
  uint64_t* empty3 = full3 + kGemvMaxStages;
  uint64_t* full4 = empty3 + kGemvMaxStages;
  uint64_t* empty4 = full4 + kGemvMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty4 + kGemvMaxStages);
  if (threadIdx.x == 0) {
    for (int s = 0; s < d.stages3; ++s) {
      mbar_init(&full3[s], 1);
      mbar_init(&empty3[s], kGemvConsumerWarps);
    }
    for (int s = 0; s < d.stages4; ++s) {
      mbar_init(&full4[s], 1);
      mbar_init(&empty4[s], kGemvConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int vec = d.H / 8, R = d.T * d.k;

  if (!route_and_sort(d.x, d.wr, d.bias, d.T, d.H, d.E, d.k, d.norm_topk_prob, d.logits, d.bar,
                      abort_flag, d.status, rs))
    return;
  const int nt = rs.nt;

  // ------------------------------------------------------------- 3: gate/up
  StreamArgs a{};
  a.act = d.x;
  a.act_rows = d.T;
  a.index = rs.perm;
  a.index_div = d.k;
  a.M = R;
  a.tiles = rs.tiles;
  a.num_tiles = &rs.nt;
  a.max_tiles = kFusedMaxRecs;
  a.w0 = d.w_gate;
  a.w1 = d.w_up;
  a.E = d.E;
  a.K = d.H;
  a.N = d.I;
  a.out = d.h;
  a.out_rows = R;
  a.stages = d.stages3;
  a.status = d.status;
  a.next_w = d.w_down;
  a.next_N = d.H;
  a.next_K = d.I;
  // Both phases' item ranges depend only on the tile table: computed here, so
  // the down phase starts streaming as soon as its barrier opens.
  const int hvec = d.I / 8;
  uint4* sh_h = reinterpret_cast<uint4*>(
      smem_raw + static_cast<size_t>(d.stages4) * gemv_row_block<false>() * d.I * 2);
  StreamArgs b{};
  b.act = sh_h;
  b.act_rows = R;
  b.index_div = 1;
  b.M = R;
  b.tiles = rs.tiles;
  b.num_tiles = &rs.nt;
  b.max_tiles = kFusedMaxRecs;
  b.w0 = d.w_down;
  b.E = d.E;
  b.K = d.I;
  b.N = d.H;
  b.out = d.slots;
  b.row_map = rs.perm;
  b.row_scale = rs.w;
  b.out_rows = R;
  b.stages = d.stages4;
  b.status = d.status;
  long long lo3, hi3, lo4, hi4;
  balanced_range(a, nt, d.I / gemv_row_block<true>(), &lo3, &hi3);
  __syncthreads();  // every thread has its range before the shared result is reused
  balanced_range(b, nt, d.H / gemv_row_block<false>(), &lo4, &hi4);
  stream_items<true>(a, smem_raw, full3, empty3, abort_flag, nt, lo3, hi3);
  if (!grid_barrier(d.bar + 1, abort_flag, d.status)) return;

  // ----------------------------------------------------- 4: down, to slot rows
  // The R rows of h (written by every CTA in phase 3) are staged in shared
  // memory behind the ring's stages, so the dot products read them at once
  // instead of waiting on L2 inside every pass.
  for (int i = threadIdx.x; i < R * hvec; i += blockDim.x)
    sh_h[i] = __ldcg(reinterpret_cast<const uint4*>(d.h) + i);
  __syncthreads();
  stream_items<false, kActPlain>(b, smem_raw, full4, empty4, abort_flag, nt, lo4, hi4);
  if (!grid_barrier(d.bar + 2, abort_flag, d.status)) return;

  // --------------------------------------------------------------- 5: combine
  const uint4* sl = reinterpret_cast<const uint4*>(d.slots);
  const long long total = static_cast<long long>(d.T) * vec;
  for (long long g = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(g / vec);
    const int v = static_cast<int>(g - static_cast<long long>(n) * vec);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < d.k; ++j)
      acc_bf16x8(acc, __ldcg(sl + static_cast<size_t>(n * d.k + j) * vec + v), 1.0f);
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    d.y[g] = o;
  }
}

// ------------------------------------------------------------------ split-I decode layer
//
// decode_layer_split: the single-launch layer with ONE pass over the routed
// experts' weights, for callers that keep the down weights also transposed,
// w_down_t [E][I][H] (row i of expert e = column i of Wd[e]).  Phases 1 and 2
// (router logits; top-k and the record sort in every CTA) are those of
// decode_layer_fused.  Phase 3 splits every routed expert along I: work item
// = (expert tile, 8 rows of I), each CTA a contiguous, cost-balanced item
// range.  One producer warp streams an item's 8 gate rows, 8 up rows and 8
// rows of w_down_t into a ring stage (contiguous bulk copies); each of the 8
// consumer warps forms h = bf16(silu(x . Wg) * (x . Wu)) for one of the rows,
// and every consumer thread then adds Wd[8t .. 8t+7, 8 cols] . h to fp32
// partials it keeps in registers for 8 output columns.  When the range leaves
// a tile, the partials go to scratch as one segment (CTA c, tile ti) at slot
// c + ti (unique: the ranges are contiguous and ascending).  After a grid
// barrier, phase 4 sums each slot's segments in CTA order, rounds the slot row
// bf16(w * D) and adds the k slots of a token in slot order (the rounding of
// the down GEMV and combine_rows).  Gate, up and down weights stream from HBM
// once, in contiguous copies, with no second pass over the down weights.  The
// output equals decode_layer_fused's up to fp32 summation order over I (a
// bf16 rounding flip on a few elements) and repeats bit for bit on a GPU.

constexpr int kFusedMaxT = 4;      // records of one expert tile <= T
constexpr int kSplitRows = gemv_row_block<true>();  // I rows per item
constexpr int kFusedConsumers = 32 * kGemvConsumerWarps;
constexpr int kSplitMaxH = 8 * kFusedConsumers;     // 8 output columns per consumer thread
constexpr int kFusedMaxGrid = 160;

struct SplitArgs {
  const uint4* x;          // [T][H]
  const uint4* wr;         // [E][H]
  const float* bias;       // [E] or null
  int T, H, I, E, k, norm_topk_prob;
  const __nv_bfloat16* w_gate;    // [E][I][H]
  const __nv_bfloat16* w_up;      // [E][I][H]
  const __nv_bfloat16* w_down_t;  // [E][I][H]
  float* logits;           // scratch [T][E]
  float* part;             // scratch [kFusedMaxGrid + kFusedMaxRecs][T][H]: segment partials
  int2* ranges;            // scratch [gridDim.x]: each CTA's item range
  unsigned int* bar;       // two counters, zero at launch
  uint2* y;                // [T][H / 4]
  int stages;
  int* status;
};

// One consumer warp's gate/up row of a stage for n <= NR records (rows[r] =
// token of record r): h_out[r] = bf16(silu(x . Wg) * (x . Wu)), the
// arithmetic of gemv_pass<true>.
template <int NR>
__device__ __forceinline__ void fused_gate_up(const uint4* w, int vec, const uint4* __restrict__ x,
                                              const int* rows, int n, int lane, float* h_out) {
  constexpr int CH = 2 * NR >= 16 ? 2 : 4;
  float acc[2][NR][CH];
  stage_dots<2, NR, CH, kActLdg>(w, kGemvConsumerWarps * vec, x, rows, n, vec, lane, acc);
  float v[2][NR];
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float t = acc[j][r][0] + acc[j][r][1];
      if (CH == 4) t += acc[j][r][CH - 2] + acc[j][r][CH - 1];
      v[j][r] = t;
    }
  reduce_records<2, NR>(v, lane);
  const int r = reduced_record<NR>(lane);
  if ((lane & (32 / NR - 1)) == 0 && r < n) h_out[r] = bf16_round_f(silu_f(v[0][0]) * v[1][0]);
}

__global__ void __launch_bounds__(kGemvThreads, 1) decode_layer_split(const SplitArgs d) {
  extern __shared__ __align__(128) uint8_t smem_raw[];  // ring, then its barriers
  __shared__ RouteSmem rs;
  __shared__ float s_h[2][kSplitRows][kFusedMaxT];  // h of an item, double-buffered
  __shared__ int2 s_rng[kFusedMaxGrid];
  __shared__ int s_first[kFusedMaxRecs], s_last[kFusedMaxRecs];  // CTAs holding a tile
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + kGemvRingBytes);
  uint64_t* empty = full + kGemvMaxStages;
  uint64_t* hbar = empty + kGemvMaxStages;  // [2]: every consumer warp wrote its h row
  volatile int* abort_flag = reinterpret_cast<volatile int*>(hbar + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < d.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumerWarps);
    }
    mbar_init(&hbar[0], kGemvConsumerWarps);
    mbar_init(&hbar[1], kGemvConsumerWarps);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (!route_and_sort(d.x, d.wr, d.bias, d.T, d.H, d.E, d.k, d.norm_topk_prob, d.logits, d.bar,
                      abort_flag, d.status, rs))
    return;
  const int nt = rs.nt, R = d.T * d.k, vec = d.H / 8;

  // ----------------------------------------- 3: gate/up and down in one pass
  const int ipt = d.I / kSplitRows;  // items per tile
  StreamArgs a{};
  a.M = R;
  a.tiles = rs.tiles;
  a.num_tiles = &rs.nt;
  a.max_tiles = kFusedMaxRecs;
  long long lo, hi;
  balanced_range(a, nt, ipt, &lo, &hi);
  if (threadIdx.x == 0) d.ranges[blockIdx.x] = make_int2(static_cast<int>(lo), static_cast<int>(hi));
  const uint32_t mat_bytes = static_cast<uint32_t>(kSplitRows) * d.H * 2;  // 8 rows of one matrix
  const uint32_t stage_bytes = 3u * mat_bytes;                            // gate, up, down^T
  if (warp == kGemvConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, issued = 0;
      for (long long w = lo; w < hi; ++w) {
        const int ti = static_cast<int>(w / ipt);
        const int rb = static_cast<int>(w - static_cast<long long>(ti) * ipt);
        const int e = rs.tiles[ti].x;
        if (e < 0 || e >= d.E) break;  // the consumers report it
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, d.status, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        const size_t row0 =
            (static_cast<size_t>(e) * d.I + static_cast<size_t>(rb) * kSplitRows) * d.H;
        uint8_t* dst = smem_raw + s * stage_bytes;
        bulk_load(dst, d.w_gate + row0, mat_bytes, &full[s]);
        bulk_load(dst + mat_bytes, d.w_up + row0, mat_bytes, &full[s]);
        bulk_load(dst + 2 * mat_bytes, d.w_down_t + row0, mat_bytes, &full[s]);
        ++issued;
        if (++s == d.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (*abort_flag) {
        // Let every copy still in flight land before the CTA exits.
        const uint32_t first = issued > static_cast<uint32_t>(d.stages) ? issued - d.stages : 0u;
        for (uint32_t i = first; i < issued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[i % d.stages], (i / d.stages) & 1u)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
          }
        }
      }
    }
  } else {
    // -------------------------------------------------------------- consumers
    // Thread ct owns output columns 8ct .. 8ct+7 of the down projection.
    const int ct = threadIdx.x;
    const bool owns = 8 * ct < d.H;
    float acc[8][kFusedMaxT];
    int rows[kFusedMaxT];
    int cur_ti = -1, n = 0, s = 0;
    uint32_t ph = 0, hph = 0;  // ring phase; bit b = phase of hbar[b]
    bool ok = true;
    auto flush = [&]() {
      if (!owns) return;
      float* dst = d.part + static_cast<size_t>(blockIdx.x + cur_ti) * d.T * d.H + 8 * ct;
#pragma unroll
      for (int r = 0; r < kFusedMaxT; ++r) {
        if (r < n) {
          float4* o = reinterpret_cast<float4*>(dst + static_cast<size_t>(r) * d.H);
          o[0] = make_float4(acc[0][r], acc[1][r], acc[2][r], acc[3][r]);
          o[1] = make_float4(acc[4][r], acc[5][r], acc[6][r], acc[7][r]);
        }
      }
    };
    int buf = 0;
    for (long long w = lo; w < hi; ++w, buf ^= 1) {
      const int ti = static_cast<int>(w / ipt);
      const int4 t = rs.tiles[ti];
      if (t.x < 0 || t.x >= d.E || t.y < 0 || t.z - t.y > kFusedMaxT || t.z - t.y > d.T ||
          t.z > R) {
        if (ct == 0) record_status(d.status, kErrBadRow);
        ok = false;
        break;
      }
      if (ti != cur_ti) {
        if (cur_ti >= 0) flush();
        cur_ti = ti;
        n = t.z - t.y;
#pragma unroll
        for (int r = 0; r < kFusedMaxT; ++r) {
          rows[r] = r < n ? rs.perm[t.y + r] / d.k : 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j][r] = 0.0f;
        }
      }
      if (!mbar_wait(&full[s], ph, abort_flag, d.status, kErrTimeoutFull)) {
        ok = false;
        break;
      }
      const uint8_t* stage = smem_raw + s * stage_bytes;
      const uint4* w0 = reinterpret_cast<const uint4*>(stage) + warp * vec;
      float* h_out = s_h[buf][warp];
      if (n == 1)
        fused_gate_up<1>(w0, vec, d.x, rows, n, lane, h_out);
      else if (n == 2)
        fused_gate_up<2>(w0, vec, d.x, rows, n, lane, h_out);
      else
        fused_gate_up<4>(w0, vec, d.x, rows, n, lane, h_out);
      __syncwarp();
      if (lane == 0) mbar_arrive(&hbar[buf]);
      if (!mbar_wait(&hbar[buf], (hph >> buf) & 1u, abort_flag, d.status, kErrTimeoutFull)) {
        ok = false;
        break;
      }
      hph ^= 1u << buf;
      if (owns) {
        // Row c of the stage's down^T block = column c of the item in Wd.
        const uint4* dt = reinterpret_cast<const uint4*>(stage + 2 * mat_bytes) + ct;
        const float(*hh)[kFusedMaxT] = s_h[buf];
#pragma unroll
        for (int c = 0; c < kSplitRows; ++c) {
          const uint4 wv = dt[c * vec];
          const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float wlo = __uint_as_float(w4[q] << 16);
            const float whi = __uint_as_float(w4[q] & 0xffff0000u);
#pragma unroll
            for (int r = 0; r < kFusedMaxT; ++r) {
              if (r < n) {
                acc[2 * q][r] = fmaf(wlo, hh[c][r], acc[2 * q][r]);
                acc[2 * q + 1][r] = fmaf(whi, hh[c][r], acc[2 * q + 1][r]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == d.stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    if (ok && cur_ti >= 0) flush();
  }
  if (!grid_barrier(d.bar + 1, abort_flag, d.status)) return;

  // ----------------------------------------------------- 4: segment sums, combine
  for (int c = threadIdx.x; c < static_cast<int>(gridDim.x); c += blockDim.x)
    s_rng[c] = __ldcg(d.ranges + c);
  __syncthreads();
  for (int c = threadIdx.x; c < static_cast<int>(gridDim.x); c += blockDim.x) {
    const int2 r = s_rng[c];
    if (r.x >= r.y) continue;
    for (int ti = (r.x + ipt - 1) / ipt; ti * ipt < r.y; ++ti) s_first[ti] = c;  // holds item ti*ipt
    for (int ti = r.x / ipt; (ti + 1) * ipt - 1 < r.y; ++ti)
      if ((ti + 1) * ipt - 1 >= r.x) s_last[ti] = c;  // holds the tile's last item
  }
  __syncthreads();
  // Work item = (token, group of 4 columns), one warp each: lane 4j + q sums
  // every fourth segment of slot t*k + j (q = 0..3), the four partial sums meet
  // over shuffles, and every lane adds the k slot values in slot order.
  const int groups = d.H / 4;
  const int jj = lane >> 2, q = lane & 3;
  constexpr int kWarps = kGemvThreads / 32;
  const int warps_all = static_cast<int>(gridDim.x) * kWarps;
  for (int item = blockIdx.x * kWarps + warp; item < d.T * groups; item += warps_all) {
    const int t = item / groups, col = (item - t * groups) * 4;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    float w = 0.0f;
    if (jj < d.k) {
      const int slot = t * d.k + jj;
      const int ti = rs.tile_of[slot];
      const int r = rs.pos[slot] - rs.tiles[ti].y;
      w = rs.w[slot];
      for (int c = s_first[ti] + q; c <= s_last[ti]; c += 4) {
        if (s_rng[c].x >= s_rng[c].y) continue;  // an empty range holds no segment
        const float4 p = __ldcg(reinterpret_cast<const float4*>(
            d.part + (static_cast<size_t>(c + ti) * d.T + r) * d.H + col));
        sum.x += p.x;
        sum.y += p.y;
        sum.z += p.z;
        sum.w += p.w;
      }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      sum.x += __shfl_xor_sync(0xffffffffu, sum.x, o);
      sum.y += __shfl_xor_sync(0xffffffffu, sum.y, o);
      sum.z += __shfl_xor_sync(0xffffffffu, sum.z, o);
      sum.w += __shfl_xor_sync(0xffffffffu, sum.w, o);
    }
    // slot value bf16(w * D), as the down GEMV writes its slot rows
    const float v0 = bf16_round_f(sum.x * w), v1 = bf16_round_f(sum.y * w);
    const float v2 = bf16_round_f(sum.z * w), v3 = bf16_round_f(sum.w * w);
    float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;
    for (int j = 0; j < d.k; ++j) {
      y0 += __shfl_sync(0xffffffffu, v0, 4 * j);
      y1 += __shfl_sync(0xffffffffu, v1, 4 * j);
      y2 += __shfl_sync(0xffffffffu, v2, 4 * j);
      y3 += __shfl_sync(0xffffffffu, v3, 4 * j);
    }
    if (lane == 0) d.y[item] = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
  }
}

// ------------------------------------------------------------------ launchers

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kRouterMaxDynSmem = 160 * 1024;
constexpr int kGemvMaxDynSmem = kGemvRingBytes + 2 * kGemvMaxStages * 8 + 16;

// Raise a kernel's dynamic shared memory limit to `bytes`, once per device.
template <class Kernel>
static bool allow_smem(Kernel* fn, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const uint64_t bit = 1ull << (dev & 63);
  if ((done.load(std::memory_order_acquire) & bit) != 0) return true;
  if (note_cuda_error(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           bytes)) != cudaSuccess)
    return false;
  done.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

static size_t router_dyn_smem(int T, int H, int E) {
  return static_cast<size_t>(T) * H * 2 + static_cast<size_t>(E) * (1 + kSortThreads / 32) * sizeof(int);
}

bool router_small_ok(int T, int H, int E, int k) {
  return T >= 1 && T <= kRouterSmallMaxT && (H % 8) == 0 && H <= 32 * 8 * kRouterMaxVecPerLane &&
         (E % kRouterCluster) == 0 && E <= kSortThreads && k >= 1 && k <= kRouterMaxK && k <= E &&
         router_dyn_smem(T, H, E) <= kRouterMaxDynSmem;
}

int launch_router_sort_small(const void* x, const void* wr, const float* bias, int T, int H, int E,
                             int k, int norm_topk_prob, int* ids_out, float* w_out,
                             void* logits_out, int* counts, int* offsets, int* perm, int4* tiles,
                             int max_tiles, int* num_tiles, int* status, cudaStream_t stream) {
  if (!router_small_ok(T, H, E, k) || !aligned16(x) || !aligned16(wr)) return kRcUnsupported;
  const size_t sh = router_dyn_smem(T, H, E);
  static std::atomic<uint64_t> attr{0};
  if (!allow_smem(router_sort_small, kRouterMaxDynSmem, attr)) return kRcCudaError;
  const cudaError_t e = launch_pdl(
      router_sort_small, dim3(kRouterCluster), dim3(kRouterThreads), sh, stream,
      static_cast<const uint4*>(x), static_cast<const uint4*>(wr), bias, T, H / 8, E, k,
      norm_topk_prob, ids_out, w_out, static_cast<__nv_bfloat16*>(logits_out), counts, offsets,
      perm, tiles, max_tiles, num_tiles, status);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

static int gemv_stages(int K, bool swiglu) {
  const long long rb = swiglu ? gemv_row_block<true>() : gemv_row_block<false>();
  const long long stage = (swiglu ? 2LL : 1LL) * rb * K * 2;
  return static_cast<int>(std::min<long long>(kGemvMaxStages, kGemvRingBytes / stage));
}

bool gemv_ok(int n_out, int K, bool swiglu) {
  const int rb = swiglu ? gemv_row_block<true>() : gemv_row_block<false>();
  return n_out > 0 && (n_out % rb) == 0 && K > 0 && (K % 8) == 0 &&
         gemv_stages(K, swiglu) >= 2;
}

template <bool SWIGLU>
static int launch_stream(StreamArgs a, cudaStream_t stream, int max_sms) {
  a.stages = gemv_stages(a.K, SWIGLU);
  const size_t stage = (SWIGLU ? 2u : 1u) * static_cast<size_t>(gemv_row_block<SWIGLU>()) * a.K * 2;
  const size_t sh = a.stages * stage + 2 * kGemvMaxStages * sizeof(uint64_t) + 16;
  static std::atomic<uint64_t> attr{0};
  if (!allow_smem(gemv_stream<SWIGLU>, kGemvMaxDynSmem, attr)) return kRcCudaError;
  const long long work = static_cast<long long>(a.max_tiles) * (a.N / gemv_row_block<SWIGLU>());
  const long long sms =
      max_sms > 0 ? std::min(max_sms, device_sm_count()) : device_sm_count();
  const int grid = static_cast<int>(std::min<long long>(work, sms));
  const cudaError_t e =
      launch_pdl(gemv_stream<SWIGLU>, dim3(grid), dim3(kGemvThreads), sh, stream, a);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

int launch_w13_gemv(const void* src, int src_rows, const int* index, int index_div, int M,
                    const int4* tiles, const int* num_tiles, int max_tiles, const void* w_gate,
                    const void* w_up, int E, int H, int I, void* h_out, int* status,
                    cudaStream_t stream, const void* w_down_prefetch, int max_sms) {
  if (!gemv_ok(I, H, true) || !aligned16(src) || !aligned16(w_gate) || !aligned16(w_up))
    return kRcUnsupported;
  if (M == 0 || max_tiles == 0) return kRcOk;
  StreamArgs a{};
  a.act = static_cast<const uint4*>(src);
  a.act_rows = src_rows;
  a.index = index;
  a.index_div = index_div;
  a.M = M;
  a.tiles = tiles;
  a.num_tiles = num_tiles;
  a.max_tiles = max_tiles;
  a.w0 = static_cast<const __nv_bfloat16*>(w_gate);
  a.w1 = static_cast<const __nv_bfloat16*>(w_up);
  a.E = E;
  a.K = H;
  a.N = I;
  a.out = static_cast<__nv_bfloat16*>(h_out);
  a.out_rows = M;
  a.status = status;
  if (w_down_prefetch != nullptr && aligned16(w_down_prefetch) && (I % 8) == 0) {
    a.next_w = static_cast<const __nv_bfloat16*>(w_down_prefetch);
    a.next_N = H;  // down weights are [E][H][I]
    a.next_K = I;
  }
  return launch_stream<true>(a, stream, max_sms);
}

int launch_w2_gemv(const void* h, int M, const int4* tiles, const int* num_tiles, int max_tiles,
                   const void* w_down, int E, int H, int I, const int* row_map,
                   const float* row_scale, void* out, int out_rows, int* status,
                   cudaStream_t stream, int max_sms) {
  if (!gemv_ok(H, I, false) || !aligned16(h) || !aligned16(w_down)) return kRcUnsupported;
  if (M == 0 || max_tiles == 0) return kRcOk;
  StreamArgs a{};
  a.act = static_cast<const uint4*>(h);
  a.act_rows = M;
  a.index_div = 1;
  a.M = M;
  a.tiles = tiles;
  a.num_tiles = num_tiles;
  a.max_tiles = max_tiles;
  a.w0 = static_cast<const __nv_bfloat16*>(w_down);
  a.E = E;
  a.K = I;
  a.N = H;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.row_map = row_map;
  a.row_scale = row_scale;
  a.out_rows = out_rows;
  a.status = status;
  return launch_stream<false>(a, stream, max_sms);
}

bool fused_decode_ok(int T, int H, int I, int E, int k) {
  const long long R = static_cast<long long>(T) * k;
  // the down phase keeps two ring stages and the R rows of h in shared memory
  const long long down_smem = 2LL * gemv_row_block<false>() * I * 2 + R * I * 2;
  return R >= 1 && R <= kFusedMaxRecs && router_small_ok(T, H, E, k) && gemv_ok(I, H, true) &&
         gemv_ok(H, I, false) && down_smem <= kGemvRingBytes;
}

size_t fused_decode_scratch_bytes(int T, int E) {
  return (static_cast<size_t>(T) * E * sizeof(float) + 255) / 256 * 256 + 256;
}

int launch_decode_fused(const void* x, const void* wr, const float* bias, int T, int H, int I,
                        int E, int k, int norm_topk_prob, const void* w_gate, const void* w_up,
                        const void* w_down, void* scratch, void* h, void* slots, void* y,
                        int* status, cudaStream_t stream) {
  if (!fused_decode_ok(T, H, I, E, k)) return kRcUnsupported;
  if (!aligned16(x) || !aligned16(wr) || !aligned16(w_gate) || !aligned16(w_up) ||
      !aligned16(w_down) || !aligned16(h) || !aligned16(slots) || !aligned16(y) ||
      scratch == nullptr)
    return kRcBadArgument;
  DecodeArgs d{};
  d.x = static_cast<const uint4*>(x);
  d.wr = static_cast<const uint4*>(wr);
  d.bias = bias;
  d.T = T;
  d.H = H;
  d.I = I;
  d.E = E;
  d.k = k;
  d.norm_topk_prob = norm_topk_prob;
  d.w_gate = static_cast<const __nv_bfloat16*>(w_gate);
  d.w_up = static_cast<const __nv_bfloat16*>(w_up);
  d.w_down = static_cast<const __nv_bfloat16*>(w_down);
  d.logits = static_cast<float*>(scratch);
  d.bar = reinterpret_cast<unsigned int*>(
      static_cast<uint8_t*>(scratch) + fused_decode_scratch_bytes(T, E) - 256);
  d.h = static_cast<__nv_bfloat16*>(h);
  d.slots = static_cast<__nv_bfloat16*>(slots);
  d.y = static_cast<uint4*>(y);
  d.stages3 = gemv_stages(H, true);
  // phase 4 leaves room behind its stages for the T*k rows of h
  const long long stage4 = static_cast<long long>(gemv_row_block<false>()) * I * 2;
  const long long h_bytes = static_cast<long long>(T) * k * I * 2;
  d.stages4 = static_cast<int>(
      std::min<long long>(gemv_stages(I, false), (kGemvRingBytes - h_bytes) / stage4));
  if (d.stages4 < 2) return kRcUnsupported;
  d.status = status;
  const size_t sh = kGemvRingBytes + 4 * kGemvMaxStages * sizeof(uint64_t) + 16;
  static std::atomic<uint64_t> attr{0};
  if (!allow_smem(decode_layer_fused, static_cast<int>(sh), attr)) return kRcCudaError;
  if (cudaMemsetAsync(d.bar, 0, 3 * sizeof(unsigned int), stream) != cudaSuccess)
    return kRcCudaError;
  // Cooperative: every CTA is resident at once, as the grid barriers need.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(device_sm_count());
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = sh;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_layer_fused, d) == cudaSuccess ? kRcOk : kRcCudaError;
}

// Ring stages of the split layer: an item is 8 rows each of gate, up and down^T.
static int split_stages(int H) {
  const long long stage = 3LL * kSplitRows * H * 2;
  return static_cast<int>(std::min<long long>(kGemvMaxStages, kGemvRingBytes / stage));
}

bool split_decode_ok(int T, int H, int I, int E, int k) {
  const long long R = static_cast<long long>(T) * k;
  return R >= 1 && R <= kFusedMaxRecs && T <= kFusedMaxT && router_small_ok(T, H, E, k) &&
         gemv_ok(I, H, true) && (I % kSplitRows) == 0 && (H % 8) == 0 && H <= kSplitMaxH &&
         split_stages(H) >= 2;
}

// Scratch of the split layer: logits [T][E] fp32, segment partials
// [kFusedMaxGrid + kFusedMaxRecs][T][H] fp32, the CTAs' item ranges and the
// barrier counters.
namespace {
struct SplitScratch {
  size_t logits, part, ranges, bar, total;
};
SplitScratch split_scratch(int T, int H, int E) {
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  SplitScratch f{};
  f.logits = 0;
  f.part = up(static_cast<size_t>(T) * E * sizeof(float));
  f.ranges = f.part + up(static_cast<size_t>(kFusedMaxGrid + kFusedMaxRecs) * T * H * sizeof(float));
  f.bar = f.ranges + up(kFusedMaxGrid * sizeof(int2));
  f.total = f.bar + 256;
  return f;
}
}  // namespace

size_t split_decode_scratch_bytes(int T, int H, int E) { return split_scratch(T, H, E).total; }

int launch_decode_split(const void* x, const void* wr, const float* bias, int T, int H, int I,
                        int E, int k, int norm_topk_prob, const void* w_gate, const void* w_up,
                        const void* w_down_t, void* scratch, void* y, int* status,
                        cudaStream_t stream) {
  if (!split_decode_ok(T, H, I, E, k)) return kRcUnsupported;
  if (!aligned16(x) || !aligned16(wr) || !aligned16(w_gate) || !aligned16(w_up) ||
      !aligned16(w_down_t) || !aligned16(y) || scratch == nullptr || !aligned16(scratch))
    return kRcBadArgument;
  const int grid = device_sm_count();
  if (grid < 1 || grid > kFusedMaxGrid) return kRcUnsupported;
  const SplitScratch f = split_scratch(T, H, E);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  SplitArgs d{};
  d.x = static_cast<const uint4*>(x);
  d.wr = static_cast<const uint4*>(wr);
  d.bias = bias;
  d.T = T;
  d.H = H;
  d.I = I;
  d.E = E;
  d.k = k;
  d.norm_topk_prob = norm_topk_prob;
  d.w_gate = static_cast<const __nv_bfloat16*>(w_gate);
  d.w_up = static_cast<const __nv_bfloat16*>(w_up);
  d.w_down_t = static_cast<const __nv_bfloat16*>(w_down_t);
  d.logits = reinterpret_cast<float*>(base + f.logits);
  d.part = reinterpret_cast<float*>(base + f.part);
  d.ranges = reinterpret_cast<int2*>(base + f.ranges);
  d.bar = reinterpret_cast<unsigned int*>(base + f.bar);
  d.y = static_cast<uint2*>(y);
  d.stages = split_stages(H);
  d.status = status;
  const size_t sh = kGemvRingBytes + (2 * kGemvMaxStages + 2) * sizeof(uint64_t) + 16;
  static std::atomic<uint64_t> attr{0};
  if (!allow_smem(decode_layer_split, static_cast<int>(sh), attr)) return kRcCudaError;
  // The grid barriers need every CTA resident: one per SM (checked once per device).
  static std::atomic<uint64_t> resident{0};
  int dev = 0;
  if (note_cuda_error(cudaGetDevice(&dev)) != cudaSuccess) return kRcCudaError;
  const uint64_t dev_bit = 1ull << (dev & 63);
  if ((resident.load(std::memory_order_acquire) & dev_bit) == 0) {
    int per_sm = 0;
    if (note_cuda_error(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, decode_layer_split, kGemvThreads, sh)) != cudaSuccess)
      return kRcCudaError;
    if (per_sm < 1) return kRcUnsupported;
    resident.fetch_or(dev_bit, std::memory_order_acq_rel);
  }
  if (note_cuda_error(cudaMemsetAsync(d.bar, 0, 2 * sizeof(unsigned int), stream)) != cudaSuccess)
    return kRcCudaError;
  // Cooperative: every CTA is resident at once, as the grid barriers need.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = sh;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  return note_cuda_error(cudaLaunchKernelEx(&cfg, decode_layer_split, d)) == cudaSuccess
             ? kRcOk
             : kRcCudaError;
}

}  // namespace moe
