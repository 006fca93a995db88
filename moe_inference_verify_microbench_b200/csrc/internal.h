// Internal launchers shared by the C-ABI layer (capi.cu).  Nothing here
// crosses the library boundary.
#pragma once

#include <cstddef>
#include <cstdint>
#include <utility>

#include "ptx.cuh"

namespace moe {

// Host-side return codes of the C-ABI entry points.
enum ReturnCode : int {
  kRcOk = 0,
  kRcBadArgument = -1,    // null pointer, negative size, inconsistent sizes
  kRcUnsupported = -2,    // a shape this build's kernels do not handle
  kRcCudaError = -3,      // a CUDA runtime call or launch failed
  kRcTensorMap = -4,      // cuTensorMapEncodeTiled rejected a tensor map
  kRcWorkspace = -5,      // caller workspace smaller than required
};

// Launch with programmatic stream serialisation, so the kernel may be
// scheduled while its predecessor in the stream is finishing (see pdl_wait);
// `cluster_x` > 1 groups consecutive CTAs into clusters of that size.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  cfg.attrs = attr;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  return launch_pdl_cluster(kernel, grid, block, smem, stream, 1u, std::forward<Args>(args)...);
}

int sort_num_blocks(int R);
size_t sort_workspace_bytes(int R, int E_local);
int launch_sort_align(const int* ids, int R, int E, int e_begin, int E_local, int block_m,
                      void* workspace, int* counts, int* offsets, long long* offsets64, int* perm,
                      int* inv, int4* tiles, int max_tiles, int* num_tiles, int* status,
                      cudaStream_t stream);
int launch_tiles_from_offsets(const long long* offsets, int E, int block_m, int4* tiles,
                              int max_tiles, int* num_tiles, int* status, cudaStream_t stream);

int launch_gather_rows(const void* src, int src_rows, const int* idx, int R, const int* count,
                       int idx_div, int H, void* dst, int* status, cudaStream_t stream);
int launch_combine(const void* rows, int n_rows, const int* slot_src, const float* slot_w,
                   const int* ids, int e_begin, int e_end, int T, int k, int H, void* y,
                   int* status, cudaStream_t stream);

int launch_router(const void* x, const void* wr, const float* bias, int T, int H, int E, int k,
                  int norm_topk_prob, int* ids_out, float* w_out, void* logits_out, int* status,
                  cudaStream_t stream);
// max_sms (grouped GEMMs and GEMVs): at most this many SMs (<= 0: all), the
// others left to concurrent work on other streams.
// tile_rows: the height of the tile table's row blocks, 128 (MOE_BLOCK_M) or
// kPairTileRows (CTA-pair kernels, large batches).
constexpr int kPairTileRows = 256;
int launch_w13_swiglu(const void* a, int M, const int4* tiles, const int* num_tiles, int max_tiles,
                      const void* w_gate, const void* w_up, int E, int H, int I, void* h_out,
                      int* status, cudaStream_t stream, int tile_rows = 128);
int launch_w13_swiglu_gather(const void* src, int src_rows, const int* index, int index_div,
                             int M, const int4* tiles, const int* num_tiles, int max_tiles,
                             const void* w_gate, const void* w_up, int E, int H, int I,
                             void* h_out, int* status, cudaStream_t stream, int tile_rows = 128,
                             const void* w_down_prefetch = nullptr, int max_sms = 0);

int launch_w2(const void* h, int M, const int4* tiles, const int* num_tiles, int max_tiles,
              const void* w_down, int E, int H, int I, const int* row_map, const float* row_scale,
              void* out, int out_rows, int* status, cudaStream_t stream, int tile_rows = 128,
              int max_sms = 0);

// CTA-pair GEMMs pay off once the average expert has kPairMinRowsPerExpert
// rows: below that the padding of its last 256-row tile costs more tensor
// work than the halved B traffic saves (measured crossover on B200 between
// 512 and 1024 rows per expert).
constexpr int kPairMinRowsPerExpert = 1024;
// Whether the gate/up GEMM gathers the token rows itself (cp.async loader
// warps) instead of reading a gathered copy written by a separate kernel.
constexpr bool kFuseGatherPair = true;
constexpr bool kFuseGatherSingle = true;

inline bool use_pair_gemm(long long R, int E, int H, int I) {
  return R >= static_cast<long long>(kPairMinRowsPerExpert) * E && (I % 128) == 0 &&
         (H % 256) == 0 && (H % 64) == 0 && (I % 64) == 0;
}

int device_sm_count();

// The cudaError_t of the most recent failed CUDA call a launcher recorded on
// this thread (0 = none), and the recorder: returns `e` unchanged.
int last_cuda_error();
cudaError_t note_cuda_error(cudaError_t e);

// Small-batch kernels (decode.cu).  Below these sizes the layer streams the
// routed experts' weights through the CUDA cores instead of 128-row
// tensor-core tiles: the router for up to 16 tokens (router_small_ok), the
// gate/up GEMM for M <= kGemvW13MaxRows routing records and the down GEMM for
// M <= kGemvW2MaxRows (measured crossovers on B200, H=2048, I=768, E=128).
constexpr int kGemvW13MaxRows = 128;
constexpr int kGemvW2MaxRows = 64;

bool router_small_ok(int T, int H, int E, int k);
bool gemv_ok(int n_out, int K, bool swiglu);
inline bool use_router_small(int T, int H, int E, int k) { return router_small_ok(T, H, E, k); }
inline bool use_gemv_w13(long long M) { return M > 0 && M <= kGemvW13MaxRows; }
inline bool use_gemv_w2(long long M) { return M > 0 && M <= kGemvW2MaxRows; }

int launch_router_sort_small(const void* x, const void* wr, const float* bias, int T, int H, int E,
                             int k, int norm_topk_prob, int* ids_out, float* w_out,
                             void* logits_out, int* counts, int* offsets, int* perm, int4* tiles,
                             int max_tiles, int* num_tiles, int* status, cudaStream_t stream);
// w_down_prefetch (optional): the down weights [E][H][I] of the same experts,
// prefetched into L2 behind the gate/up stream when they fit.
int launch_w13_gemv(const void* src, int src_rows, const int* index, int index_div, int M,
                    const int4* tiles, const int* num_tiles, int max_tiles, const void* w_gate,
                    const void* w_up, int E, int H, int I, void* h_out, int* status,
                    cudaStream_t stream, const void* w_down_prefetch = nullptr, int max_sms = 0);
int launch_w2_gemv(const void* h, int M, const int4* tiles, const int* num_tiles, int max_tiles,
                   const void* w_down, int E, int H, int I, const int* row_map,
                   const float* row_scale, void* out, int out_rows, int* status,
                   cudaStream_t stream, int max_sms = 0);

// Whole decode layer in one cooperative launch (T * k <= 64 records):
// router, top-k, sort, gate/up and down GEMVs and the k-way combine, bitwise
// equal to the four-launch decode path.  `scratch` holds
// fused_decode_scratch_bytes(T, E) bytes; h [T*k, I] and slots [T*k, H] bf16.
bool fused_decode_ok(int T, int H, int I, int E, int k);
size_t fused_decode_scratch_bytes(int T, int E);
int launch_decode_fused(const void* x, const void* wr, const float* bias, int T, int H, int I,
                        int E, int k, int norm_topk_prob, const void* w_gate, const void* w_up,
                        const void* w_down, void* scratch, void* h, void* slots, void* y,
                        int* status, cudaStream_t stream);

// The single-launch layer with one pass over the weights (T <= 4 tokens,
// T * k <= 32 records), given the down weights transposed, w_down_t [E][I][H]:
// equal to the above up to fp32 summation order over I.  `scratch` holds
// split_decode_scratch_bytes(T, H, E) bytes.
bool split_decode_ok(int T, int H, int I, int E, int k);
size_t split_decode_scratch_bytes(int T, int H, int E);
int launch_decode_split(const void* x, const void* wr, const float* bias, int T, int H, int I,
                        int E, int k, int norm_topk_prob, const void* w_gate, const void* w_up,
                        const void* w_down_t, void* scratch, void* y, int* status,
                        cudaStream_t stream);

// Down GEMM with the atomic combine: out_f32[row_map[p] / red_div] +=
// row_scale[row_map[p]] * (h[p] @ w_down[e]^T) in fp32 (row_map[p] < n_slots).
int launch_w2_atomic(const void* h, int M, const int4* tiles, const int* num_tiles,
                     int max_tiles, const void* w_down, int E, int H, int I, const int* row_map,
                     const float* row_scale, int n_slots, int red_div, float* out_f32,
                     int* status, cudaStream_t stream, int tile_rows = 128);
// Block glue: h = delta ? bf16(x + delta) : x; y = bf16(h * rsqrt(mean(h^2) + eps) * w).
int launch_add_rmsnorm(const void* x, const void* delta, const float* w, int T, int H, float eps,
                       void* h_out, void* y, cudaStream_t stream);
// y[i] = bf16(src[i]) for n elements (n % 8 == 0).
int launch_cast_f32_bf16(const float* src, long long n, void* y, cudaStream_t stream);

// Expert-parallel send plan (ep_plan.cu).
int launch_ep_keys(const int* ids, int N, int k, int epr, int ep, int* keys, int* status,
                   cudaStream_t stream);
int launch_ep_meta(const int* perm, const int* count, int max_rows, const int* ids, const float* w,
                   int N, int k, int epr, int ep, int* meta, int* status, cudaStream_t stream);

// Peer-store expert-parallel exchange (ep_peer.cu).
constexpr int kMaxEpRanks = 8;
void set_peer_wait_limit(unsigned long long ns);
size_t peer_buffer_bytes(int ep, int cap_rows, int H, int k);
size_t peer_region_offset(int ep, int cap_rows, int H, int k, int region);
int launch_ep_peer_dispatch(void* const* bases, int ep, int me, int cap_rows, int H, int k,
                            const int* send_counts, const void* x, int N, const int* perm,
                            const int* ids, const float* w, int experts_per_rank, int* status,
                            cudaStream_t stream);
int launch_ep_peer_return(void* const* bases, int ep, int me, int cap_rows, int H, int k,
                          const void* out, int out_rows, const int* inv, int* status,
                          cudaStream_t stream);
int peer_alloc(size_t bytes, void** ptr, void* handle);
int peer_open(const void* handle, void** ptr);
int peer_close(void* ptr);
int peer_free(void* ptr);

inline int max_tiles_bound(long long R, int E, int block_m) {
  return static_cast<int>((R + block_m - 1) / block_m + E);
}

}  // namespace moe
