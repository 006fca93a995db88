// Send-plan helpers of the all_to_all expert-parallel schedule
// (C7/python/solution.py:150-203 restated for one-row-per-owner dispatch):
//
//   ep_keys  keys[n, r] = r if one of token n's k experts lives on rank r,
//            else ep (a sentinel past the ranks): sorting the keys stably by
//            value gives the rank-major send order of (token, rank) pairs.
//   ep_meta  for every send row i (pair = perm[i] = n * ep + r, i below the
//            device count), the row's metadata for rank r: k local expert ids
//            (experts_per_rank marks "not on r") and k weights (0 when not on
//            r), as one int32 row of 2k entries (weights bit-cast), ready to
//            travel with the row.
#include "internal.h"

namespace moe {

constexpr int kPlanThreads = 256;

__global__ void __launch_bounds__(kPlanThreads) ep_keys(const int* __restrict__ ids, int N, int k,
                                                        int epr, int ep, int* __restrict__ keys,
                                                        int* status) {
  pdl_wait();
  pdl_trigger();
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
    unsigned mask = 0;
    for (int j = 0; j < k; ++j) {
      const int e = ids[static_cast<size_t>(n) * k + j];
      const int r = e / epr;
      if (e < 0 || r >= ep) {
        record_status(status, kErrBadExpert);
        continue;
      }
      mask |= 1u << r;
    }
    for (int r = 0; r < ep; ++r) keys[static_cast<size_t>(n) * ep + r] = (mask >> r) & 1u ? r : ep;
  }
}

__global__ void __launch_bounds__(kPlanThreads) ep_meta(const int* __restrict__ perm,
                                                        const int* __restrict__ count, int max_rows,
                                                        const int* __restrict__ ids,
                                                        const float* __restrict__ w, int N, int k,
                                                        int epr, int ep, int* __restrict__ meta,
                                                        int* status) {
  pdl_wait();
  pdl_trigger();
  const int rows = min(max_rows, *count);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
    const int pair = perm[i];
    const int n = pair / ep;
    const int r = pair - n * ep;
    int* out = meta + static_cast<size_t>(i) * 2 * k;
    if (pair < 0 || n >= N) {
      record_status(status, kErrBadRow);
      for (int j = 0; j < k; ++j) {
        out[j] = epr;
        out[k + j] = 0;
      }
      continue;
    }
    for (int j = 0; j < k; ++j) {
      const int e = ids[static_cast<size_t>(n) * k + j];
      const bool own = e >= 0 && e / epr == r;
      out[j] = own ? e - r * epr : epr;
      out[k + j] = own ? __float_as_int(w[static_cast<size_t>(n) * k + j]) : 0;
    }
  }
}

static int plan_grid(long long items) {
  const long long want = (items + kPlanThreads - 1) / kPlanThreads;
  const long long cap = static_cast<long long>(device_sm_count()) * 4;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

int launch_ep_keys(const int* ids, int N, int k, int epr, int ep, int* keys, int* status,
                   cudaStream_t stream) {
  if (N < 0 || k <= 0 || epr <= 0 || ep <= 0 || ep > 32) return kRcBadArgument;
  if (N == 0) return kRcOk;
  const cudaError_t e = launch_pdl(ep_keys, dim3(plan_grid(N)), dim3(kPlanThreads), 0, stream, ids,
                                   N, k, epr, ep, keys, status);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

int launch_ep_meta(const int* perm, const int* count, int max_rows, const int* ids, const float* w,
                   int N, int k, int epr, int ep, int* meta, int* status, cudaStream_t stream) {
  if (max_rows < 0 || N < 0 || k <= 0 || epr <= 0 || ep <= 0 || ep > 32) return kRcBadArgument;
  if (max_rows == 0) return kRcOk;
  const cudaError_t e = launch_pdl(ep_meta, dim3(plan_grid(max_rows)), dim3(kPlanThreads), 0,
                                   stream, perm, count, max_rows, ids, w, N, k, epr, ep, meta,
                                   status);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

}  // namespace moe
