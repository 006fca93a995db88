// Peer-store dispatch and combine of the all_to_all expert-parallel schedule
// (C7/python/solution.py:186-261, C8/python/solution.py:171-224) over NVLink,
// with the split sizes negotiated on the device: no host synchronisation and
// no NCCL call in the exchange, so a whole forward can be captured in a CUDA
// graph.
//
// Every rank of the expert-parallel group allocates one peer buffer of the
// same layout (PeerLayout), exports it with cudaIpcGetMemHandle, maps the
// other ranks' buffers with cudaIpcOpenMemHandle, and writes into them with
// plain stores (no peer loads anywhere).  One forward on rank `me`:
//
//   ep_publish     epoch e = state.epoch + 1 (the same on every rank: each
//                  forward advances it once); my per-destination send counts
//                  -> row `me` of every rank's count matrix, then
//                  count_flag[me] = e at every rank
//   ep_dispatch    wait for count_flag[s] >= e of every s; send row i (pair
//                  perm[i] = n*ep + d) -> x row n into rank d's receive block
//                  of source `me`, with the token's k expert ids localised to
//                  d (experts_per_rank where an expert is not on d) and its k
//                  weights; receive rows past my own total get the sentinel
//                  ids; the last CTA to finish sets disp_flag[me] = e at every
//                  rank
//   ep_recv_wait   wait for disp_flag[s] >= e of every s
//   ...            sort, gate/up and down GEMMs on the receive buffer
//   ep_return      per received row: the weighted fp32 sum of its records
//                  (record order) as bf16 into its source's return buffer at
//                  the row's send position; the last CTA sets
//                  ret_flag[me] = e at every rank
//   ep_ret_wait    wait for ret_flag[d] >= e of every d
//   ...            sum of the returned rows over owner ranks (moe_combine)
//
// Reuse across epochs follows from the order of these steps: a rank writes a
// peer's count row, receive block or flags for epoch e only after the peer
// published epoch e, which the peer does after its epoch e-1 return wait,
// i.e. after every rank finished reading epoch e-1 data; a rank writes a
// source's return buffer for epoch e only after the source dispatched epoch
// e, which it does after consuming its epoch e-1 returns.  Every wait is
// bounded (10 s unless set_peer_wait_limit changed it) and records
// kErrPeerTimeout; every store is bounds-checked against the layout and
// records kErrBadRow.
#include <cstring>

#include "internal.h"

namespace moe {

constexpr int kPeerThreads = 256;
constexpr int kPeerWarps = kPeerThreads / 32;
constexpr int kPeerMaxK = 8;
constexpr unsigned long long kPeerWaitLimitNs = 10000000000ull;  // 10 s (default)
static unsigned long long g_peer_wait_ns = kPeerWaitLimitNs;

// Rank-local bookkeeping at the start of every peer buffer (never written by
// a peer).
struct PeerState {
  unsigned long long epoch;
  unsigned long long disp_done;    // ep_dispatch CTAs finished in this epoch
  unsigned long long ret_done;     // ep_return CTAs finished in this epoch
  int n_recv;                      // rows received in this epoch
  int recv_base[kMaxEpRanks + 1];  // first receive row of every source
};
static_assert(sizeof(PeerState) <= 256, "peer state header");

struct PeerLayout {
  int ep, cap_rows, H, k;
  size_t flags, counts, recv_ids, recv_w, recv_rows, ret_rows, total;
};

static size_t peer_align(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static PeerLayout peer_layout(int ep, int cap_rows, int H, int k) {
  PeerLayout L{};
  L.ep = ep;
  L.cap_rows = cap_rows;
  L.H = H;
  L.k = k;
  size_t o = 256;  // PeerState
  L.flags = o;
  o = peer_align(o + 3 * static_cast<size_t>(ep) * sizeof(unsigned long long));
  L.counts = o;
  o = peer_align(o + static_cast<size_t>(ep) * ep * sizeof(int));
  L.recv_ids = o;
  o = peer_align(o + static_cast<size_t>(cap_rows) * k * sizeof(int));
  L.recv_w = o;
  o = peer_align(o + static_cast<size_t>(cap_rows) * k * sizeof(float));
  L.recv_rows = o;
  o = peer_align(o + static_cast<size_t>(cap_rows) * H * 2);
  L.ret_rows = o;
  o = peer_align(o + static_cast<size_t>(cap_rows) * H * 2);
  L.total = o;
  return L;
}

struct PeerArgs {
  unsigned char* base[kMaxEpRanks];  // every rank's peer buffer, mapped into this process
  PeerLayout L;
  int me;
  unsigned long long wait_ns;  // bound of every wait on a peer
  int* status;
};

enum FlagKind : int { kFlagCount = 0, kFlagDispatch = 1, kFlagReturn = 2 };

__device__ __forceinline__ PeerState* state_of(const PeerArgs& a) {
  return reinterpret_cast<PeerState*>(a.base[a.me]);
}

__device__ __forceinline__ unsigned long long* flag_ptr(const PeerArgs& a, int q, int kind,
                                                        int src) {
  return reinterpret_cast<unsigned long long*>(a.base[q] + a.L.flags) + kind * a.L.ep + src;
}

__device__ __forceinline__ int* counts_ptr(const PeerArgs& a, int q) {
  return reinterpret_cast<int*>(a.base[q] + a.L.counts);
}

__device__ __forceinline__ void store_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0 waits until this rank's flag `kind` of every source reaches `e`
// (bounded); the whole block then sees the result.  False on timeout.
__device__ bool wait_all_flags(const PeerArgs& a, int kind, unsigned long long e, int* ok_sm) {
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long t0 = globaltimer_ns();
    for (int s = 0; s < a.L.ep && ok; ++s) {
      const unsigned long long* f = flag_ptr(a, a.me, kind, s);
      while (load_acquire_sys(f) < e) {
        if (globaltimer_ns() - t0 > a.wait_ns) {
          record_status(a.status, kErrPeerTimeout);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    *ok_sm = ok;
  }
  __syncthreads();
  return *ok_sm != 0;
}

// Called by every thread after its last peer store: the last CTA of the grid
// to get here raises flag `kind`[me] = e at every rank.
__device__ void finish_and_signal(const PeerArgs& a, int kind, unsigned long long* done,
                                  unsigned long long e) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long old = atomicAdd(done, 1ull);
    if (old == gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q < a.L.ep; ++q) store_release_sys(flag_ptr(a, q, kind, a.me), e);
    }
  }
}

__device__ __forceinline__ unsigned long long current_epoch(const PeerArgs& a) {
  return *reinterpret_cast<volatile unsigned long long*>(&state_of(a)->epoch);
}

__global__ void __launch_bounds__(kPeerThreads) ep_publish(const PeerArgs a,
                                                           const int* __restrict__ send_counts) {
  __shared__ unsigned long long e_sm;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    PeerState* st = state_of(a);
    const unsigned long long e = st->epoch + 1;
    st->epoch = e;
    st->disp_done = 0;
    st->ret_done = 0;
    e_sm = e;
  }
  __syncthreads();
  const int ep = a.L.ep;
  for (int i = threadIdx.x; i < ep * ep; i += blockDim.x) {
    const int q = i / ep, d = i - q * ep;
    counts_ptr(a, q)[a.me * ep + d] = send_counts[d];
  }
  __threadfence_system();
  __syncthreads();
  if (static_cast<int>(threadIdx.x) < ep)
    store_release_sys(flag_ptr(a, threadIdx.x, kFlagCount, a.me), e_sm);
}

// Send row i (pair = perm[i] = n * ep + d, rank-major): x row n, its k expert
// ids localised to rank d and its k weights -> rank d's receive block.
__global__ void __launch_bounds__(kPeerThreads, 4) ep_dispatch(
    const PeerArgs a, const uint4* __restrict__ x, int N, const int* __restrict__ perm,
    const int* __restrict__ ids, const float* __restrict__ w, int epr) {
  __shared__ int ok_sm;
  __shared__ int base_in[kMaxEpRanks];  // my block's first row in rank d's receive buffer
  __shared__ int send_off[kMaxEpRanks + 1];
  __shared__ int n_recv_sm;
  pdl_wait();
  pdl_trigger();
  const int ep = a.L.ep, me = a.me, k = a.L.k, cap = a.L.cap_rows;
  const int vec = a.L.H / 8;
  const unsigned long long e = current_epoch(a);
  PeerState* st = state_of(a);
  if (wait_all_flags(a, kFlagCount, e, &ok_sm)) {
    if (threadIdx.x == 0) {
      const int* cnt = counts_ptr(a, me);
      int off = 0, nr = 0;
      for (int d = 0; d < ep; ++d) {
        int b = 0;
        for (int s = 0; s < me; ++s) b += __ldcv(cnt + s * ep + d);
        base_in[d] = b;
        send_off[d] = off;
        off += __ldcv(cnt + me * ep + d);
      }
      send_off[ep] = off;
      for (int s = 0; s < ep; ++s) {
        if (blockIdx.x == 0) st->recv_base[s] = min(nr, cap);
        nr += __ldcv(cnt + s * ep + me);
      }
      nr = min(nr, cap);
      n_recv_sm = nr;
      if (blockIdx.x == 0) {
        st->recv_base[ep] = nr;
        st->n_recv = nr;
      }
    }
    __syncthreads();
    const int total = min(send_off[ep], cap);
    int max_cnt = 0;
    for (int d = 0; d < ep; ++d) max_cnt = max(max_cnt, send_off[d + 1] - send_off[d]);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Warp task t serves destination (t + me) % ep: adjacent warps write to
    // different ranks, so every rank spreads its rows over all destinations
    // at once (no rank's ingress takes every sender's traffic while the
    // others idle) and the local copy runs beside the NVLink stores.
    const long long tasks = static_cast<long long>(ep) * max_cnt;
    for (long long t = blockIdx.x * kPeerWarps + warp; t < tasks;
         t += static_cast<long long>(gridDim.x) * kPeerWarps) {
      const int dd = static_cast<int>((t + me) % ep);
      const int j = static_cast<int>(t / ep);
      if (j >= send_off[dd + 1] - send_off[dd]) continue;
      const int i = send_off[dd] + j;
      if (i >= total) continue;
      const int pair = perm[i];
      const int n = pair / ep, d = pair - (pair / ep) * ep;
      const int pos = pair >= 0 ? base_in[d] + (i - send_off[d]) : -1;
      if (pair < 0 || n >= N || pos < 0 || pos >= cap) {
        if (lane == 0) record_status(a.status, kErrBadRow);
        continue;
      }
      const uint4* src = x + static_cast<size_t>(n) * vec;
      uint4* dst =
          reinterpret_cast<uint4*>(a.base[d] + a.L.recv_rows) + static_cast<size_t>(pos) * vec;
      for (int v0 = 0; v0 < vec; v0 += 8 * 32) {
        uint4 buf[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < vec) buf[u] = __ldg(src + v);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < vec) dst[v] = buf[u];
        }
      }
      if (lane < k) {
        const int ex = ids[static_cast<size_t>(n) * k + lane];
        const bool own = ex >= 0 && ex / epr == d;
        const size_t slot = static_cast<size_t>(pos) * k + lane;
        reinterpret_cast<int*>(a.base[d] + a.L.recv_ids)[slot] = own ? ex - d * epr : epr;
        reinterpret_cast<float*>(a.base[d] + a.L.recv_w)[slot] =
            own ? w[static_cast<size_t>(n) * k + lane] : 0.0f;
      }
    }
    // Receive rows no source fills this epoch: sentinel ids, so the sort
    // leaves them out of every expert's tiles.
    int* my_ids = reinterpret_cast<int*>(a.base[me] + a.L.recv_ids);
    const long long lo = static_cast<long long>(n_recv_sm) * k;
    const long long hi = static_cast<long long>(cap) * k;
    for (long long j = lo + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; j < hi;
         j += static_cast<long long>(gridDim.x) * blockDim.x)
      my_ids[j] = epr;
  } else if (blockIdx.x == 0 && threadIdx.x == 0) {
    st->n_recv = 0;
    for (int s = 0; s <= ep; ++s) st->recv_base[s] = 0;
  }
  finish_and_signal(a, kFlagDispatch, &st->disp_done, e);
}

__global__ void __launch_bounds__(32) ep_recv_wait(const PeerArgs a) {
  __shared__ int ok_sm;
  pdl_wait();
  pdl_trigger();
  wait_all_flags(a, kFlagDispatch, current_epoch(a), &ok_sm);
}

// Received row i < n_recv: sum_j w[i, j] * out[inv[i*k + j]] in fp32, record
// order (inv < 0: not one of this rank's experts), as bf16 into the source's
// return buffer at the row's position in the source's send order.
__global__ void __launch_bounds__(kPeerThreads, 2) ep_return(const PeerArgs a,
                                                          const uint4* __restrict__ out,
                                                          int out_rows,
                                                          const int* __restrict__ inv) {
  __shared__ int base[kMaxEpRanks + 1];
  __shared__ int src_off[kMaxEpRanks];  // my block's first row in source s's send order
  pdl_wait();
  pdl_trigger();
  const int ep = a.L.ep, k = a.L.k, vec = a.L.H / 8;
  PeerState* st = state_of(a);
  const unsigned long long e = current_epoch(a);
  if (threadIdx.x == 0) {
    const int* cnt = counts_ptr(a, a.me);
    for (int s = 0; s <= ep; ++s) base[s] = st->recv_base[s];
    for (int s = 0; s < ep; ++s) {
      int o = 0;
      for (int d = 0; d < a.me; ++d) o += __ldcv(cnt + s * ep + d);
      src_off[s] = o;
    }
  }
  __syncthreads();
  const int rows = min(st->n_recv, a.L.cap_rows);
  const float* wr = reinterpret_cast<const float*>(a.base[a.me] + a.L.recv_w);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int max_cnt = 0;
  for (int q = 0; q < ep; ++q) max_cnt = max(max_cnt, base[q + 1] - base[q]);
  // Warp task t serves source (t + me) % ep, as in ep_dispatch.
  const long long tasks = static_cast<long long>(ep) * max_cnt;
  for (long long t = blockIdx.x * kPeerWarps + warp; t < tasks;
       t += static_cast<long long>(gridDim.x) * kPeerWarps) {
    const int s = static_cast<int>((t + a.me) % ep);
    const int j = static_cast<int>(t / ep);
    if (j >= base[s + 1] - base[s]) continue;
    const int i = base[s] + j;
    if (i >= rows) continue;
    const int pos = src_off[s] + j;
    if (pos < 0 || pos >= a.L.cap_rows) {
      if (lane == 0) record_status(a.status, kErrBadRow);
      continue;
    }
    int slot[kPeerMaxK];
    float wt[kPeerMaxK];
#pragma unroll
    for (int j = 0; j < kPeerMaxK; ++j) {
      slot[j] = -1;
      wt[j] = 0.0f;
      if (j < k) {
        const int sl = inv[static_cast<size_t>(i) * k + j];
        if (sl >= out_rows) record_status(a.status, kErrBadRow);
        if (sl >= 0 && sl < out_rows) {
          slot[j] = sl;
          wt[j] = wr[static_cast<size_t>(i) * k + j];
        }
      }
    }
    uint4* dst =
        reinterpret_cast<uint4*>(a.base[s] + a.L.ret_rows) + static_cast<size_t>(pos) * vec;
    // Two column vectors per lane per pass: every record's loads of both are
    // in flight before any is summed.
    for (int v0 = 0; v0 < vec; v0 += 64) {
      uint4 val[2][kPeerMaxK];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int v = v0 + 32 * c + lane;
#pragma unroll
        for (int j = 0; j < kPeerMaxK; ++j)
          val[c][j] = slot[j] >= 0 && v < vec
                          ? __ldg(out + static_cast<size_t>(slot[j]) * vec + v)
                          : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int v = v0 + 32 * c + lane;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < kPeerMaxK; ++j) {  // record order
          if (slot[j] < 0) continue;
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&val[c][j]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __bfloat1622float2(h2[q]);
            acc[2 * q] = fmaf(wt[j], f.x, acc[2 * q]);
            acc[2 * q + 1] = fmaf(wt[j], f.y, acc[2 * q + 1]);
          }
        }
        if (v < vec)
          dst[v] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                              pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
      }
    }
  }
  finish_and_signal(a, kFlagReturn, &st->ret_done, e);
}

__global__ void __launch_bounds__(32) ep_ret_wait(const PeerArgs a) {
  __shared__ int ok_sm;
  pdl_wait();
  pdl_trigger();
  wait_all_flags(a, kFlagReturn, current_epoch(a), &ok_sm);
}

// ------------------------------------------------------------------ host side

static int make_args(PeerArgs* a, void* const* bases, int ep, int me, int cap_rows, int H, int k,
                     int* status) {
  if (ep < 1 || ep > kMaxEpRanks || me < 0 || me >= ep || cap_rows < 0 || H <= 0 ||
      (H % 8) != 0 || k < 1 || k > kPeerMaxK || bases == nullptr)
    return kRcBadArgument;
  *a = PeerArgs{};
  for (int q = 0; q < ep; ++q) {
    if (bases[q] == nullptr || (reinterpret_cast<uintptr_t>(bases[q]) & 255u) != 0)
      return kRcBadArgument;
    a->base[q] = static_cast<unsigned char*>(bases[q]);
  }
  a->L = peer_layout(ep, cap_rows, H, k);
  a->me = me;
  a->wait_ns = g_peer_wait_ns;
  a->status = status;
  return kRcOk;
}

static int peer_grid(long long rows, int ctas_per_sm) {
  const long long want = (rows + kPeerWarps - 1) / kPeerWarps;
  const long long cap = static_cast<long long>(device_sm_count()) * ctas_per_sm;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

void set_peer_wait_limit(unsigned long long ns) {
  g_peer_wait_ns = ns > 0 ? ns : kPeerWaitLimitNs;
}

size_t peer_buffer_bytes(int ep, int cap_rows, int H, int k) {
  return peer_layout(ep, cap_rows, H, k).total;
}

size_t peer_region_offset(int ep, int cap_rows, int H, int k, int region) {
  const PeerLayout L = peer_layout(ep, cap_rows, H, k);
  switch (region) {
    case 0: return L.recv_ids;
    case 1: return L.recv_w;
    case 2: return L.recv_rows;
    case 3: return L.ret_rows;
    case 4: return L.flags;
    case 5: return L.counts;
    default: return 0;  // PeerState
  }
}

int launch_ep_peer_dispatch(void* const* bases, int ep, int me, int cap_rows, int H, int k,
                            const int* send_counts, const void* x, int N, const int* perm,
                            const int* ids, const float* w, int experts_per_rank, int* status,
                            cudaStream_t stream) {
  PeerArgs a;
  const int rc = make_args(&a, bases, ep, me, cap_rows, H, k, status);
  if (rc != kRcOk) return rc;
  if (N < 0 || experts_per_rank <= 0 || send_counts == nullptr ||
      (N > 0 && (x == nullptr || perm == nullptr || ids == nullptr || w == nullptr)) ||
      (reinterpret_cast<uintptr_t>(x) & 15u) != 0)
    return kRcBadArgument;
  if (launch_pdl(ep_publish, dim3(1), dim3(kPeerThreads), 0, stream, a, send_counts) !=
      cudaSuccess)
    return kRcCudaError;
  if (launch_pdl(ep_dispatch, dim3(peer_grid(cap_rows, 4)), dim3(kPeerThreads), 0, stream, a,
                 static_cast<const uint4*>(x), N, perm, ids, w, experts_per_rank) != cudaSuccess)
    return kRcCudaError;
  if (launch_pdl(ep_recv_wait, dim3(1), dim3(32), 0, stream, a) != cudaSuccess)
    return kRcCudaError;
  return kRcOk;
}

int launch_ep_peer_return(void* const* bases, int ep, int me, int cap_rows, int H, int k,
                          const void* out, int out_rows, const int* inv, int* status,
                          cudaStream_t stream) {
  PeerArgs a;
  const int rc = make_args(&a, bases, ep, me, cap_rows, H, k, status);
  if (rc != kRcOk) return rc;
  if (out_rows < 0 || (out_rows > 0 && out == nullptr) || (cap_rows > 0 && inv == nullptr) ||
      (reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return kRcBadArgument;
  if (launch_pdl(ep_return, dim3(peer_grid(cap_rows, 2)), dim3(kPeerThreads), 0, stream, a,
                 static_cast<const uint4*>(out), out_rows, inv) != cudaSuccess)
    return kRcCudaError;
  if (launch_pdl(ep_ret_wait, dim3(1), dim3(32), 0, stream, a) != cudaSuccess)
    return kRcCudaError;
  return kRcOk;
}

int peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return kRcBadArgument;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return kRcCudaError;
  if (cudaMemset(p, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return kRcCudaError;
  }
  *ptr = p;
  return kRcOk;
}

int peer_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return kRcBadArgument;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? kRcOk
             : kRcCudaError;
}

int peer_close(void* ptr) {
  if (ptr == nullptr) return kRcBadArgument;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? kRcOk : kRcCudaError;
}

int peer_free(void* ptr) {
  if (ptr == nullptr) return kRcBadArgument;
  return cudaFree(ptr) == cudaSuccess ? kRcOk : kRcCudaError;
}

}  // namespace moe
