// Row movement kernels: the permutation gather and the top-k combine.
//
// gather_rows   dst[p] = src[idx[p] / idx_div], p < min(R, *count)  (C5:135-137 gather
//               x_flat[token_ids_rep[perm]]; C7:167, C7:227 re-sort of received rows)
// combine_rows  y[n] = sum_j  w_j * rows[src_j]               (C5:158-160
//               weight scale + index_add_, C7:259-261, C8:221-224)
//               with src_j = slot_src ? slot_src[n*k+j] : n*k+j and w_j = slot_w ?
//               slot_w[n*k+j] : 1; a slot is skipped when src_j < 0 or when its
//               expert id (ids[n*k+j]) lies outside [e_begin, e_end).
//
// Both are HBM-bound copies with 16-byte vector accesses; the combine sums the
// k contributions in fp32 in slot order (deterministic, unlike the atomic
// index_add_ of the reference on CUDA).
#include "internal.h"

namespace moe {

constexpr int kRowsThreads = 256;
constexpr int kRowsWarps = kRowsThreads / 32;

__global__ void __launch_bounds__(kRowsThreads) gather_rows(const uint4* __restrict__ src,
                                                            int src_rows,
                                                            const int* __restrict__ idx, int R,
                                                            const int* __restrict__ count,
                                                            int idx_div, int vec_per_row,
                                                            uint4* __restrict__ dst, int* status) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = count != nullptr ? min(R, *count) : R;
  for (int p = blockIdx.x * kRowsWarps + warp; p < rows; p += gridDim.x * kRowsWarps) {
    const int s = idx[p] / idx_div;
    if (s < 0 || s >= src_rows) {
      if (lane == 0) record_status(status, kErrBadRow);
      continue;
    }
    const uint4* a = src + static_cast<size_t>(s) * vec_per_row;
    uint4* b = dst + static_cast<size_t>(p) * vec_per_row;
    // Eight loads in flight per lane before the stores; the gathered rows are
    // written with the streaming hint so the source rows (each read k times)
    // keep their place in L2.
    for (int v0 = 0; v0 < vec_per_row; v0 += 8 * 32) {
      uint4 buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v < vec_per_row) buf[u] = __ldg(a + v);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v < vec_per_row) __stcs(b + v, buf[u]);
      }
    }
  }
}

constexpr int kCombineMaxK = 8;  // the router selects at most 8 experts

// One thread per (token, 16-byte column vector): the k source rows' vectors are
// loaded independently (no dependent chain of round trips), summed in fp32 in
// slot order, and stored once.
__global__ void __launch_bounds__(kRowsThreads) combine_rows(
    const uint4* __restrict__ rows, int n_rows, const int* __restrict__ slot_src,
    const float* __restrict__ slot_w, const int* __restrict__ ids, int e_begin, int e_end, int T,
    int k, int vec_per_row, uint4* __restrict__ y, int* status) {
  pdl_wait();
  pdl_trigger();
  const long long total = static_cast<long long>(T) * vec_per_row;
  for (long long g = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(g / vec_per_row);
    const int v = static_cast<int>(g - static_cast<long long>(n) * vec_per_row);
    uint4 val[kCombineMaxK];
    float wt[kCombineMaxK];
#pragma unroll
    for (int j = 0; j < kCombineMaxK; ++j) {
      wt[j] = 0.0f;
      val[j] = make_uint4(0u, 0u, 0u, 0u);
      if (j < k) {
        const int s = n * k + j;
        int src = slot_src != nullptr ? __ldg(slot_src + s) : s;
        if (ids != nullptr) {
          const int e = __ldg(ids + s);
          if (e < e_begin || e >= e_end) src = -1;
        }
        if (src >= n_rows) {
          record_status(status, kErrBadRow);
          src = -1;
        }
        if (src >= 0) {
          wt[j] = slot_w != nullptr ? __ldg(slot_w + s) : 1.0f;
          val[j] = __ldg(rows + static_cast<size_t>(src) * vec_per_row + v);
        }
      }
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kCombineMaxK; ++j)
      if (j < k) acc_bf16x8(acc, val[j], wt[j]);
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    y[g] = o;
  }
}

// Large batches: one warp per token, each lane sums 16-byte vectors of the k
// rows.  All loads of COLS column vectors are issued before any is used
// (KMAX x COLS = 16 loads in flight per lane), so a small k (the per-owner
// partial rows of the expert-parallel combine) still keeps 16 in flight.
template <int KMAX, int COLS>
__global__ void __launch_bounds__(kRowsThreads) combine_rows_warp(
    const uint4* __restrict__ rows, int n_rows, const int* __restrict__ slot_src,
    const float* __restrict__ slot_w, const int* __restrict__ ids, int e_begin, int e_end, int T,
    int k, int vec_per_row, uint4* __restrict__ y, int* status) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int n = blockIdx.x * kRowsWarps + warp; n < T; n += gridDim.x * kRowsWarps) {
    int src = -1;
    float w = 0.0f;
    if (lane < k) {
      const int s = n * k + lane;
      src = slot_src != nullptr ? slot_src[s] : s;
      w = slot_w != nullptr ? slot_w[s] : 1.0f;
      if (ids != nullptr) {
        const int e = ids[s];
        if (e < e_begin || e >= e_end) src = -1;
      }
      if (src >= n_rows) {
        record_status(status, kErrBadRow);
        src = -1;
      }
    }
    // The k source rows and weights, shuffled out once per token.
    int sj[KMAX];
    float wj[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      sj[j] = __shfl_sync(0xffffffffu, src, j);
      wj[j] = __shfl_sync(0xffffffffu, w, j);
      if (j >= k) sj[j] = -1;
    }
    for (int v0 = 0; v0 < vec_per_row; v0 += 32 * COLS) {
      uint4 val[COLS][KMAX];
#pragma unroll
      for (int c = 0; c < COLS; ++c) {
        const int v = v0 + 32 * c + lane;
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
          val[c][j] = make_uint4(0, 0, 0, 0);
          if (sj[j] >= 0 && v < vec_per_row)
            val[c][j] = __ldg(rows + static_cast<size_t>(sj[j]) * vec_per_row + v);
        }
      }
#pragma unroll
      for (int c = 0; c < COLS; ++c) {
        const int v = v0 + 32 * c + lane;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < KMAX; ++j)  // slot order, as the reference sums
          if (sj[j] >= 0) acc_bf16x8(acc, val[c][j], wj[j]);
        if (v < vec_per_row) {
          uint4 o;
          o.x = pack_bf16x2(acc[0], acc[1]);
          o.y = pack_bf16x2(acc[2], acc[3]);
          o.z = pack_bf16x2(acc[4], acc[5]);
          o.w = pack_bf16x2(acc[6], acc[7]);
          y[static_cast<size_t>(n) * vec_per_row + v] = o;
        }
      }
    }
  }
}

// y = bf16(src), eight elements per thread (two 16-byte loads, one 16-byte
// store): the final rounding of the atomic combine's fp32 accumulation rows.
__global__ void __launch_bounds__(kRowsThreads) cast_f32_bf16(const float4* __restrict__ src,
                                                              long long n8, uint4* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = __ldcs(src + 2 * i), b = __ldcs(src + 2 * i + 1);
    y[i] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                      pack_bf16x2(b.z, b.w));
  }
}

// Pre-norm decoder block glue (the residual add and RMSNorm around the MoE of
// C8/python/solution.py:235-325, RMSNorm as the suite's harness defines it):
//   h = delta ? bf16(x + delta) : x
//   y = bf16((float(h) * rsqrt(mean_j float(h_j)^2 + eps)) * w)
// one warp per row, fp32 throughout, the row's sum of squares reduced across
// the warp; the second pass re-reads the row (L1/L2 hits).
__global__ void __launch_bounds__(kRowsThreads) add_rmsnorm_rows(
    const uint4* __restrict__ x, const uint4* __restrict__ delta, const float* __restrict__ w,
    int T, int vec, float eps, uint4* __restrict__ h_out, uint4* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float inv_h = 1.0f / static_cast<float>(vec * 8);
  for (int n = blockIdx.x * kRowsWarps + warp; n < T; n += gridDim.x * kRowsWarps) {
    const uint4* xr = x + static_cast<size_t>(n) * vec;
    const uint4* dr = delta != nullptr ? delta + static_cast<size_t>(n) * vec : nullptr;
    float ss = 0.0f;
    for (int v = lane; v < vec; v += 32) {
      uint4 a = __ldg(xr + v);
      if (dr != nullptr) {
        const uint4 b = __ldg(dr + v);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 fa = __bfloat1622float2(a2[q]), fb = __bfloat1622float2(b2[q]);
          o[q] = pack_bf16x2(fa.x + fb.x, fa.y + fb.y);
        }
        a = make_uint4(o[0], o[1], o[2], o[3]);
        h_out[static_cast<size_t>(n) * vec + v] = a;
      }
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h2[q]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss * inv_h + eps);
    // Each lane re-reads only the h_out vectors it stored itself.
    const uint4* hr = dr != nullptr ? h_out + static_cast<size_t>(n) * vec : xr;
    for (int v = lane; v < vec; v += 32) {
      const uint4 a = dr != nullptr ? hr[v] : __ldg(hr + v);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&a);
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * v);
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * v + 1);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h2[q]);
        o[q] = pack_bf16x2((f.x * r) * wv[2 * q], (f.y * r) * wv[2 * q + 1]);
      }
      y[static_cast<size_t>(n) * vec + v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

static int rows_grid(long long rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (rows + kRowsWarps - 1) / kRowsWarps;
  const long long cap = static_cast<long long>(sms) * 8;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

int launch_gather_rows(const void* src, int src_rows, const int* idx, int R, const int* count,
                       int idx_div, int H, void* dst, int* status, cudaStream_t stream) {
  if (R < 0 || H <= 0 || idx_div <= 0 || (H % 8) != 0) return kRcBadArgument;
  if (R == 0) return kRcOk;
  const cudaError_t e = launch_pdl(gather_rows, dim3(rows_grid(R)), dim3(kRowsThreads), 0, stream,
                                   static_cast<const uint4*>(src), src_rows, idx, R, count,
                                   idx_div, H / 8, static_cast<uint4*>(dst), status);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

int launch_combine(const void* rows, int n_rows, const int* slot_src, const float* slot_w,
                   const int* ids, int e_begin, int e_end, int T, int k, int H, void* y,
                   int* status, cudaStream_t stream) {
  if (T < 0 || k <= 0 || k > kCombineMaxK || H <= 0 || (H % 8) != 0) return kRcBadArgument;
  if (T == 0) return kRcOk;
  if (T >= 1024) {
    auto kern = k > 4 ? combine_rows_warp<8, 2> : k > 2 ? combine_rows_warp<4, 4>
                                                        : combine_rows_warp<2, 8>;
    const cudaError_t e = launch_pdl(kern, dim3(rows_grid(T)), dim3(kRowsThreads), 0, stream,
                                     static_cast<const uint4*>(rows), n_rows, slot_src, slot_w,
                                     ids, e_begin, e_end, T, k, H / 8, static_cast<uint4*>(y),
                                     status);
    return e == cudaSuccess ? kRcOk : kRcCudaError;
  }
  const long long threads = static_cast<long long>(T) * (H / 8);
  const long long blocks = (threads + kRowsThreads - 1) / kRowsThreads;
  const int grid = static_cast<int>(blocks < 148LL * 16 ? blocks : 148LL * 16);
  const cudaError_t e = launch_pdl(combine_rows, dim3(grid), dim3(kRowsThreads), 0, stream,
                                   static_cast<const uint4*>(rows), n_rows, slot_src, slot_w, ids,
                                   e_begin, e_end, T, k, H / 8, static_cast<uint4*>(y), status);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

int launch_add_rmsnorm(const void* x, const void* delta, const float* w, int T, int H, float eps,
                       void* h_out, void* y, cudaStream_t stream) {
  if (T < 0 || H <= 0 || (H % 8) != 0 || !(eps >= 0.0f) ||
      (T > 0 && (x == nullptr || w == nullptr || y == nullptr ||
                 (delta != nullptr && h_out == nullptr))))
    return kRcBadArgument;
  for (const void* p : {x, delta, static_cast<const void*>(w), static_cast<const void*>(h_out),
                        static_cast<const void*>(y)})
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return kRcBadArgument;
  if (T == 0) return kRcOk;
  const cudaError_t e = launch_pdl(add_rmsnorm_rows, dim3(rows_grid(T)), dim3(kRowsThreads), 0,
                                   stream, static_cast<const uint4*>(x),
                                   static_cast<const uint4*>(delta), w, T, H / 8, eps,
                                   static_cast<uint4*>(h_out), static_cast<uint4*>(y));
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

int launch_cast_f32_bf16(const float* src, long long n, void* y, cudaStream_t stream) {
  if (n < 0 || (n % 8) != 0 || (n > 0 && (src == nullptr || y == nullptr)) ||
      (reinterpret_cast<uintptr_t>(src) & 15u) != 0 || (reinterpret_cast<uintptr_t>(y) & 15u) != 0)
    return kRcBadArgument;
  if (n == 0) return kRcOk;
  const long long n8 = n / 8;
  const long long blocks = (n8 + kRowsThreads - 1) / kRowsThreads;
  const long long cap = static_cast<long long>(device_sm_count()) * 8;
  const int grid = static_cast<int>(blocks < cap ? blocks : cap);
  const cudaError_t e = launch_pdl(cast_f32_bf16, dim3(grid), dim3(kRowsThreads), 0, stream,
                                   reinterpret_cast<const float4*>(src), n8,
                                   static_cast<uint4*>(y));
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

}  // namespace moe
