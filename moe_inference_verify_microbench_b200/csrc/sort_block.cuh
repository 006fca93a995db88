// Block-level pieces of the token -> expert sort, shared by the sort kernels
// and the fused small-batch router (decode.cu).
#pragma once

#include "ptx.cuh"

namespace moe {

constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;  // records per thread per CTA chunk
constexpr int kSortChunk = kSortThreads * kSortItems;

__device__ __forceinline__ int local_expert(const int* ids, int r, int E, int e_begin, int E_local,
                                            int* status) {
  const int g = ids[r];
  if (g < 0 || g >= E) {
    record_status(status, kErrBadExpert);
    return -1;
  }
  const int e = g - e_begin;
  return (e >= 0 && e < E_local) ? e : -1;
}

// Exclusive scan of one value per thread over a block of up to 1024 threads.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) warp_sums[lane] = s;  // inclusive warp prefix
    if (lane == nw - 1) *total = s;
  }
  __syncthreads();
  const int before = warp > 0 ? warp_sums[warp - 1] : 0;
  const int res = before + x - v;
  __syncthreads();
  return res;
}

// Tile table from per-expert counts held by threads e < E (E <= blockDim.x).
__device__ __forceinline__ void write_tiles(int e, int E, int count, int offset, int block_m, int4* tiles,
                            int max_tiles, int* num_tiles, int* warp_sums, int* total) {
  const int nt = (e < E) ? (count + block_m - 1) / block_m : 0;
  const int first = block_exclusive_scan(nt, warp_sums, total);
  if (e < E) {
    for (int t = 0; t < nt; ++t) {
      const int slot = first + t;
      if (slot < max_tiles) {
        const int r0 = offset + t * block_m;
        tiles[slot] = make_int4(e, r0, min(offset + count, r0 + block_m), 0);
      }
    }
  }
  if (threadIdx.x == 0) *num_tiles = min(*total, max_tiles);
}

// One-CTA sort for R <= kSortChunk and E_local <= kSortThreads (decode
// batches), run by a block of exactly kSortThreads threads: histogram, scan,
// tile table and the stable scatter.  Same outputs, same stable order as
// sa_hist + sa_scan + sa_scatter.  `sm` holds (1 + kSortThreads / 32) *
// E_local ints of shared memory.  `ids` may point to shared or global memory.
__device__ __forceinline__ void sort_small_block(
    const int* ids, int R, int E, int e_begin, int E_local, int block_m, int* counts,
    int* offsets, long long* offsets64, int* perm, int* inv, int4* tiles, int max_tiles,
    int* num_tiles, int* status, int* sm) {
  int* base = sm;                 // [E_local]: counts, then next free position per expert
  int* wcnt = sm + E_local;       // [8][E_local]
  __shared__ int warp_sums[32];
  __shared__ int total;
  constexpr int kWarps = kSortThreads / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E_local; e += blockDim.x) {
    base[e] = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) wcnt[w * E_local + e] = 0;
  }
  __syncthreads();
  for (int r = tid; r < R; r += blockDim.x) {
    const int e = local_expert(ids, r, E, e_begin, E_local, status);
    if (e >= 0) atomicAdd(&base[e], 1);
  }
  __syncthreads();
  const int cnt = tid < E_local ? base[tid] : 0;
  const int off = block_exclusive_scan(cnt, warp_sums, &total);
  if (tid < E_local) {
    counts[tid] = cnt;
    offsets[tid] = off;
    if (offsets64 != nullptr) offsets64[tid] = off;
    base[tid] = off;
  }
  if (tid == 0) {
    offsets[E_local] = total;
    if (offsets64 != nullptr) offsets64[E_local] = total;
  }
  __syncthreads();
  write_tiles(tid, E_local, cnt, off, block_m, tiles, max_tiles, num_tiles, warp_sums, &total);
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int r0 = 0; r0 < R; r0 += kSortThreads) {
    const int r = r0 + tid;
    const int e = r < R ? local_expert(ids, r, E, e_begin, E_local, status) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    if (e >= 0 && rank == 0) wcnt[warp * E_local + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int p = base[e] + rank;
      for (int w = 0; w < warp; ++w) p += wcnt[w * E_local + e];
      perm[p] = r;
      if (inv != nullptr) inv[r] = p;
    } else if (r < R && inv != nullptr) {
      inv[r] = -1;
    }
    __syncthreads();
    for (int x = tid; x < E_local; x += blockDim.x) {
      int add = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        add += wcnt[w * E_local + x];
        wcnt[w * E_local + x] = 0;
      }
      base[x] += add;
    }
    __syncthreads();
  }
}


}  // namespace moe
