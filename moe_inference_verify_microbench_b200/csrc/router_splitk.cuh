// Router logits + top-k + softmax for mid-size batches, split along K.
//
// The tensor-core router (grouped_gemm_kernel<., kEpiRouter, .>) runs one CTA
// per 128-token tile, and each CTA streams the whole router weight and its
// tile's x rows: 1 MB per CTA for H=2048, E=128.  With a few tiles (T <= 1024)
// most SMs idle and the kernel is bound by one SM's copy rate.  Here a
// cluster of S CTAs shares a tile, CTA s multiplying the
// k-blocks [s*nkb/S, (s+1)*nkb/S) (C5/python/solution.py:124, self.gate(x)):
//
//   warp 0      one thread issues the TMA loads of x and of the router weight
//   warp 1      allocates 128 TMEM columns; one thread issues tcgen05.mma
//   warps 2..5  copy the fp32 partial accumulator (128 rows x E) from TMEM to
//               shared memory, padded rows
//   -           cluster barrier
//   all warps   rows [s*128/S, (s+1)*128/S) of the tile: a warp per row sums
//               the S partials over distributed shared memory in rank order,
//               adds the bias, rounds to bf16 (the logits), takes the top-k
//               (value descending, lower id first) and the softmax of
//               C5:125-129, and writes ids, weights and logits
//   -           cluster barrier (no CTA leaves while its partial is read)
//
// Every mbarrier wait is bounded; a CTA whose wait gave up still reaches both
// cluster barriers, so no CTA of the cluster waits forever.  No TMA load uses
// cluster multicast.
#pragma once

#include "grouped_gemm.cuh"

namespace moe {

constexpr int kRsThreads = 192;
constexpr int kRsStages = 4;
constexpr int kRsMaxE = 128;
constexpr int kRsMaxTiles = 8;  // the launcher splits K only up to this many tiles
constexpr int kRsPartStride = kRsMaxE + 4;  // floats per partial row (padded)
constexpr int kRsABytes = kBM * kBK * 2;
constexpr int kRsBBytes = kRsMaxE * kBK * 2;
constexpr size_t kRsSmemBytes = 1024 + kRsStages * (kRsABytes + kRsBBytes) +
                                static_cast<size_t>(kBM) * kRsPartStride * 4 +
                                (2 * kRsStages + 1) * 8 + 16;

struct RouterSplitArgs {
  int T, E, k, norm_topk_prob;
  int kb_per_split;  // k-blocks of kBK per cluster rank
  const float* bias;
  int* ids_out;
  float* w_out;
  __nv_bfloat16* logits_out;
  int* status;
};

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(kRsThreads, 1)
    router_splitk(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const RouterSplitArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kRsStages * kRsABytes;
  float* part = reinterpret_cast<float*>(sB + kRsStages * kRsBBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(part + kBM * kRsPartStride);
  uint64_t* empty = full + kRsStages;
  uint64_t* acc_full = empty + kRsStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  uint32_t nranks;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nranks));
  const int tile = static_cast<int>(blockIdx.x / nranks);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRsStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kRsMaxE);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  const int kb0 = static_cast<int>(rank) * a.kb_per_split;
  const uint32_t stage_tx = static_cast<uint32_t>(kRsABytes + a.E * kBK * 2);
  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      uint32_t issued = 0;
      for (int i = 0; i < a.kb_per_split; ++i) {
        const int s = i % kRsStages;
        const uint32_t ph = static_cast<uint32_t>(i / kRsStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.status, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[s], stage_tx);
        tma_load_2d(sA + s * kRsABytes, &tmA, &full[s], (kb0 + i) * kBK, tile * kBM);
        tma_load_3d(sB + s * kRsBBytes, &tmB, &full[s], (kb0 + i) * kBK, 0, 0);
        ++issued;
      }
      if (*abort_flag) {
        // Let every copy still in flight land before the CTA goes on.
        const uint32_t first = issued > kRsStages ? issued - kRsStages : 0u;
        for (uint32_t i = first; i < issued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[i % kRsStages], (i / kRsStages) & 1u)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(kBM, static_cast<uint32_t>(a.E));
      for (int i = 0; i < a.kb_per_split; ++i) {
        const int s = i % kRsStages;
        const uint32_t ph = static_cast<uint32_t>(i / kRsStages) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag, a.status, kErrTimeoutFull)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * kRsABytes);
        const uint32_t b0 = smem_u32(sB + s * kRsBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          tc_mma_bf16(tmem_base, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32),
                      idesc, (i | kk) != 0 ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      // acc_full completes once every MMA issued above has finished (also
      // after an abort, so the epilogue warps never wait on MMAs in flight).
      tc_commit(acc_full);
    }
  } else {
    // --------------------------------------------- partial accumulator to smem
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const bool got = mbar_wait(acc_full, 0, abort_flag, a.status, kErrTimeoutAccFull);
    if (__all_sync(0xffffffffu, got)) {
      tc_fence_after();
      float* prow = part + (q * 32 + lane) * kRsPartStride;
      for (int c0 = 0; c0 < a.E; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_base + lane_off + static_cast<uint32_t>(c0), r);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(prow + c0 + j) =
              make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                          __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync_all();  // every rank's partial is in its shared memory

  // -------------------------------- sum of the partials, top-k and softmax
  const int rows_per_rank = kBM / static_cast<int>(nranks);
  const int r_begin = static_cast<int>(rank) * rows_per_rank;
  const int c = 4 * lane;  // this lane's four expert columns
  constexpr int kWarps = kRsThreads / 32;
  for (int r = r_begin + warp; r < r_begin + rows_per_rank; r += kWarps) {
    const int token = tile * kBM + r;
    if (token >= a.T || *abort_flag) continue;  // warp-uniform
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < a.E) {
      const float* mine = part + r * kRsPartStride + c;
      for (uint32_t src = 0; src < nranks; ++src) {
        const float4 p = ld_dsmem_f4(cluster_addr(mine, src));
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
    }
    float lv[4] = {acc.x, acc.y, acc.z, acc.w};
    uint32_t top[kRouterMaxK];
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) top[i] = 0u;  // below every real key
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (c + j < a.E) {
        float v = lv[j];
        if (a.bias != nullptr) v += a.bias[c + j];
        lv[j] = bf16_round_f(v);
        topk_insert(top, topk_key(lv[j], c + j));
      }
    }
    if (a.logits_out != nullptr && c < a.E)
      *reinterpret_cast<uint2*>(a.logits_out + static_cast<size_t>(token) * a.E + c) =
          make_uint2(pack_bf16x2(lv[0], lv[1]), pack_bf16x2(lv[2], lv[3]));
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
    if (a.norm_topk_prob) {
#pragma unroll
      for (int i = 0; i < kRouterMaxK; ++i)
        if (i < a.k) den += expf(topk_key_value(sel[i]) - ref);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c + j < a.E) den += expf(lv[j] - ref);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    }
    const float inv = 1.0f / den;
#pragma unroll
    for (int i = 0; i < kRouterMaxK; ++i) {
      if (i < a.k && lane == i) {
        a.ids_out[static_cast<size_t>(token) * a.k + i] = topk_key_id(sel[i]);
        a.w_out[static_cast<size_t>(token) * a.k + i] = expf(topk_key_value(sel[i]) - ref) * inv;
      }
    }
  }
  cluster_sync_all();  // every rank has read the partials of every other
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kRsMaxE);
  }
}

}  // namespace moe
