// Token -> expert sort and tile alignment, without any host synchronisation.
//
// Replaces the reference's argsort/bincount/offset construction
// (C5/python/solution.py:131-136, C6/python/solution.py:137-160,
// C7/python/solution.py:160-164,224-226) and the C9 tile metadata
// (C9/python/solution.py:142-159, which needs a host sync for its
// repeat_interleave).
//
// Three launches over R = T*k routing records (flat slot index s = n*k + j;
// one launch when E_local <= 256 and R <= 2048 (sa_small, one CTA) or
// R <= 32768 (sa_cluster, a cluster of up to 8 CTAs)):
//   1. sa_hist     per-CTA expert histograms of a contiguous record chunk
//   2. sa_scan     one CTA: per-expert counts, offsets[E+1], the per-CTA base of
//                  every expert, and the 128-row tile table
//   3. sa_scatter  per CTA, a stable rank of each record inside its expert
//                  (warp match + per-warp counts), giving perm[p] = s and inv[s] = p
// The permutation is stable: records of one expert keep increasing slot
// order, i.e. torch.sort(ids, stable=True) (C6:152, C8:181).
//
// Records whose expert lies outside [e_begin, e_begin + E_local) are left out
// (inv = -1): that is the local-expert filter of the replicated-input
// expert-parallel schedule (C6/python/solution.py:141-149).
#include "internal.h"
#include "sort_block.cuh"

#include <cooperative_groups.h>

namespace moe {

int sort_num_blocks(int R) { return (R + kSortChunk - 1) / kSortChunk; }

size_t sort_workspace_bytes(int R, int E_local) {
  return static_cast<size_t>(sort_num_blocks(R)) * static_cast<size_t>(E_local) * sizeof(int) + 256;
}

__global__ void __launch_bounds__(kSortThreads) sa_hist(const int* __restrict__ ids, int R, int E,
                                                        int e_begin, int E_local,
                                                        int* __restrict__ hist, int* status) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sh[];
  for (int e = threadIdx.x; e < E_local; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int base = blockIdx.x * kSortChunk;
  const int end = min(R, base + kSortChunk);
  for (int r = base + threadIdx.x; r < end; r += blockDim.x) {
    const int e = local_expert(ids, r, E, e_begin, E_local, status);
    if (e >= 0) atomicAdd(&sh[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E_local; e += blockDim.x)
    hist[static_cast<size_t>(blockIdx.x) * E_local + e] = sh[e];
}

__global__ void __launch_bounds__(1024) sa_scan(int* __restrict__ hist, int nblk, int E_local,
                                                int block_m, int* __restrict__ counts,
                                                int* __restrict__ offsets,
                                                long long* __restrict__ offsets64,
                                                int4* __restrict__ tiles, int max_tiles,
                                                int* __restrict__ num_tiles) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_sums[32];
  __shared__ int total;
  const int e = threadIdx.x;
  int run = 0;
  if (e < E_local) {
    // hist[b][e] becomes the records of expert e in chunks before b; eight
    // independent loads are in flight per batch.
    int b = 0;
    for (; b + 8 <= nblk; b += 8) {
      int c[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) c[u] = hist[static_cast<size_t>(b + u) * E_local + e];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        hist[static_cast<size_t>(b + u) * E_local + e] = run;
        run += c[u];
      }
    }
    for (; b < nblk; ++b) {
      int* h = hist + static_cast<size_t>(b) * E_local + e;
      const int c = *h;
      *h = run;
      run += c;
    }
  }
  const int off = block_exclusive_scan(e < E_local ? run : 0, warp_sums, &total);
  if (e < E_local) {
    counts[e] = run;
    offsets[e] = off;  // sa_scatter adds it to its chunk's base
    if (offsets64 != nullptr) offsets64[e] = off;
  }
  if (e == 0) {
    offsets[E_local] = total;
    if (offsets64 != nullptr) offsets64[E_local] = total;
  }
  __syncthreads();
  if (tiles != nullptr) write_tiles(e, E_local, run, off, block_m, tiles, max_tiles, num_tiles, warp_sums, &total);
}

__global__ void __launch_bounds__(kSortThreads) sa_scatter(const int* __restrict__ ids, int R, int E,
                                                           int e_begin, int E_local,
                                                           const int* __restrict__ hist,
                                                           const int* __restrict__ offsets,
                                                           int* __restrict__ perm,
                                                           int* __restrict__ inv, int* status) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sm[];
  int* base = sm;                       // [E_local] next free position per expert
  int* wcnt = sm + E_local;             // [8][E_local] per-warp counts of this round
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kSortThreads / 32;
  for (int e = threadIdx.x; e < E_local; e += blockDim.x) {
    base[e] = hist[static_cast<size_t>(blockIdx.x) * E_local + e] + offsets[e];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) wcnt[w * E_local + e] = 0;
  }
  __syncthreads();
  const int chunk0 = blockIdx.x * kSortChunk;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int round = 0; round < kSortItems; ++round) {
    const int r = chunk0 + round * kSortThreads + threadIdx.x;
    int e = -1;
    if (r < R) e = local_expert(ids, r, E, e_begin, E_local, status);
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
    for (int x = threadIdx.x; x < E_local; x += blockDim.x) {
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

__global__ void __launch_bounds__(kSortThreads) sa_small(
    const int* __restrict__ ids, int R, int E, int e_begin, int E_local, int block_m,
    int* __restrict__ counts, int* __restrict__ offsets, long long* __restrict__ offsets64,
    int* __restrict__ perm, int* __restrict__ inv, int4* __restrict__ tiles, int max_tiles,
    int* __restrict__ num_tiles, int* status) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sm[];
  sort_small_block(ids, R, E, e_begin, E_local, block_m, counts, offsets, offsets64, perm, inv,
                   tiles, max_tiles, num_tiles, status, sm);
}

// One-launch sort for mid-size batches: a cluster of up to kClusterSortMax
// CTAs, CTA c owning records [c*chunk, (c+1)*chunk), chunk = R / 8 rounded
// up to a multiple of the block (at most kClusterChunk records).  The
// per-CTA histograms meet over distributed shared memory, every CTA scans
// them (expert offsets and its own per-expert base), CTA 0 writes counts,
// offsets and the tile table, and each CTA scatters its chunk as sa_scatter
// does.  Same outputs, same stable order as the three-kernel path.
constexpr int kClusterSortMax = 8;
constexpr int kClusterChunk = 4096;

__global__ void __launch_bounds__(kSortThreads) sa_cluster(
    const int* __restrict__ ids, int R, int E, int e_begin, int E_local, int block_m,
    int* __restrict__ counts, int* __restrict__ offsets, long long* __restrict__ offsets64,
    int* __restrict__ perm, int* __restrict__ inv, int4* __restrict__ tiles, int max_tiles,
    int* __restrict__ num_tiles, int chunk, int* status) {
  namespace cg = cooperative_groups;
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sm[];
  int* hist = sm;                 // [E_local] this CTA's histogram (read by the others)
  int* base = sm + E_local;       // [E_local] next free position per expert
  int* wcnt = sm + 2 * E_local;   // [8][E_local] per-warp counts of a round
  __shared__ int warp_sums[32];
  __shared__ int total;
  constexpr int kWarps = kSortThreads / 32;
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int nc = static_cast<int>(cluster.num_blocks());
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E_local; e += blockDim.x) {
    hist[e] = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) wcnt[w * E_local + e] = 0;
  }
  __syncthreads();
  const int chunk0 = c * chunk;
  const int chunk1 = min(R, chunk0 + chunk);
  for (int r = chunk0 + tid; r < chunk1; r += blockDim.x) {
    const int e = local_expert(ids, r, E, e_begin, E_local, status);
    if (e >= 0) atomicAdd(&hist[e], 1);
  }
  cluster.sync();  // every CTA's histogram is complete
  int run = 0, before = 0;
  if (tid < E_local) {
    for (int q = 0; q < nc; ++q) {
      const int h = cluster.map_shared_rank(hist, q)[tid];
      if (q < c) before += h;
      run += h;
    }
  }
  const int off = block_exclusive_scan(tid < E_local ? run : 0, warp_sums, &total);
  if (tid < E_local) base[tid] = off + before;
  if (c == 0) {
    if (tid < E_local) {
      counts[tid] = run;
      offsets[tid] = off;
      if (offsets64 != nullptr) offsets64[tid] = off;
    }
    if (tid == 0) {
      offsets[E_local] = total;
      if (offsets64 != nullptr) offsets64[E_local] = total;
    }
    write_tiles(tid, E_local, run, off, block_m, tiles, max_tiles, num_tiles, warp_sums, &total);
  }
  cluster.sync();  // no CTA reads another's histogram after this point
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int r0 = chunk0; r0 < chunk1; r0 += kSortThreads) {
    const int r = r0 + tid;
    const int e = r < chunk1 ? local_expert(ids, r, E, e_begin, E_local, status) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    if (e >= 0 && rank == 0) wcnt[warp * E_local + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int p = base[e] + rank;
      for (int w = 0; w < warp; ++w) p += wcnt[w * E_local + e];
      perm[p] = r;
      if (inv != nullptr) inv[r] = p;
    } else if (r < chunk1 && inv != nullptr) {
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

__global__ void __launch_bounds__(1024) tiles_from_offsets(const long long* __restrict__ offsets,
                                                           int E, int block_m,
                                                           int4* __restrict__ tiles, int max_tiles,
                                                           int* __restrict__ num_tiles,
                                                           int* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_sums[32];
  __shared__ int total;
  const int e = threadIdx.x;
  int count = 0, off = 0;
  if (e < E) {
    const long long a = offsets[e], b = offsets[e + 1];
    if (a < 0 || b < a || b > 0x7fffffffLL) {
      record_status(status, kErrBadRow);
    } else {
      off = static_cast<int>(a);
      count = static_cast<int>(b - a);
    }
  }
  write_tiles(e, E, count, off, block_m, tiles, max_tiles, num_tiles, warp_sums, &total);
}

int launch_sort_align(const int* ids, int R, int E, int e_begin, int E_local, int block_m,
                      void* workspace, int* counts, int* offsets, long long* offsets64, int* perm,
                      int* inv, int4* tiles, int max_tiles, int* num_tiles, int* status,
                      cudaStream_t stream) {
  if (R < 0 || E <= 0 || E_local <= 0 || E_local > 1024 || e_begin < 0 || e_begin + E_local > E ||
      block_m <= 0)
    return kRcBadArgument;
  const int nblk = sort_num_blocks(R);
  if (nblk <= 1 && E_local <= kSortThreads) {
    const size_t sh = static_cast<size_t>(E_local) * (1 + kSortThreads / 32) * sizeof(int);
    const cudaError_t e = launch_pdl(sa_small, dim3(1), dim3(kSortThreads), sh, stream, ids, R, E,
                                     e_begin, E_local, block_m, counts, offsets, offsets64, perm,
                                     inv, tiles, max_tiles, num_tiles, status);
    return e == cudaSuccess ? kRcOk : kRcCudaError;
  }
  int chunk = (R + kClusterSortMax - 1) / kClusterSortMax;
  chunk = (chunk + kSortThreads - 1) / kSortThreads * kSortThreads;
  const int nclu = (R + chunk - 1) / chunk;
  if (chunk <= kClusterChunk && E_local <= kSortThreads) {
    const size_t sh = static_cast<size_t>(E_local) * (2 + kSortThreads / 32) * sizeof(int);
    const cudaError_t e = launch_pdl_cluster(
        sa_cluster, dim3(nclu), dim3(kSortThreads), sh, stream, static_cast<unsigned>(nclu), ids,
        R, E, e_begin, E_local, block_m, counts, offsets, offsets64, perm, inv, tiles, max_tiles,
        num_tiles, chunk, status);
    return e == cudaSuccess ? kRcOk : kRcCudaError;
  }
  int* hist = static_cast<int*>(workspace);
  const size_t sh_hist = static_cast<size_t>(E_local) * sizeof(int);
  const size_t sh_scatter = static_cast<size_t>(E_local) * (1 + kSortThreads / 32) * sizeof(int);
  // E_local <= 1024 keeps sh_scatter <= 36 KB, inside the default 48 KB limit.
  if (nblk > 0) {
    if (launch_pdl(sa_hist, dim3(nblk), dim3(kSortThreads), sh_hist, stream, ids, R, E, e_begin,
                   E_local, hist, status) != cudaSuccess)
      return kRcCudaError;
  }
  const int scan_threads = ((E_local + 31) / 32) * 32;
  if (launch_pdl(sa_scan, dim3(1), dim3(scan_threads), 0, stream, hist, nblk, E_local, block_m,
                 counts, offsets, offsets64, tiles, max_tiles, num_tiles) != cudaSuccess)
    return kRcCudaError;
  if (nblk > 0) {
    if (launch_pdl(sa_scatter, dim3(nblk), dim3(kSortThreads), sh_scatter, stream, ids, R, E,
                   e_begin, E_local, static_cast<const int*>(hist),
                   static_cast<const int*>(offsets), perm, inv, status) != cudaSuccess)
      return kRcCudaError;
  }
  return kRcOk;
}

int launch_tiles_from_offsets(const long long* offsets, int E, int block_m, int4* tiles,
                              int max_tiles, int* num_tiles, int* status, cudaStream_t stream) {
  if (E <= 0 || E > 1024 || block_m <= 0) return kRcBadArgument;
  const int threads = ((E + 31) / 32) * 32;
  const cudaError_t e = launch_pdl(tiles_from_offsets, dim3(1), dim3(threads), 0, stream, offsets,
                                   E, block_m, tiles, max_tiles, num_tiles, status);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

}  // namespace moe
