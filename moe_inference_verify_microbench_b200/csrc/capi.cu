// extern "C" entry points declared in include/moe_b200.h.
#include "../../include/moe_b200.h"
#include "internal.h"

using namespace moe;

namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

// Carves aligned sub-buffers out of the caller's workspace.
struct Carver {
  uint8_t* base;
  size_t used = 0;
  explicit Carver(void* p) : base(static_cast<uint8_t*>(p)) {}
  template <class T>
  T* take(size_t count) {
    T* p = reinterpret_cast<T*>(base + used);
    used = align_up(used + count * sizeof(T));
    return p;
  }
};

struct LayerPlan {
  long long R;
  int max_tiles;
  size_t sort_ws;
};

LayerPlan plan_layer(int T, int E, int k) {
  LayerPlan p;
  p.R = static_cast<long long>(T) * k;
  p.max_tiles = max_tiles_bound(p.R, E, MOE_BLOCK_M);
  p.sort_ws = sort_workspace_bytes(static_cast<int>(p.R), E);
  return p;
}

// How one layer call runs: decode kernels, tile height, whether the gate/up
// GEMM gathers its rows itself (then no gathered copy is allocated).
struct LayerPath {
  bool small;
  int tile_rows;
  bool fuse_gather;
};

LayerPath layer_path(long long R, int H, int I, int E) {
  LayerPath lp;
  lp.small = use_gemv_w13(R);
  lp.tile_rows = !lp.small && use_pair_gemm(R, E, H, I) ? kPairTileRows : MOE_BLOCK_M;
  lp.fuse_gather =
      lp.small || (lp.tile_rows == kPairTileRows ? kFuseGatherPair : kFuseGatherSingle);
  return lp;
}

// The atomic combine applies to the GEMM paths; decode-size batches keep the
// slot rows and the k-sum (one of the results the atomic order allows).
bool use_atomic_combine(int mode, const LayerPath& lp) {
  return mode == MOE_COMBINE_ATOMIC && !lp.small;
}

template <class Body>
size_t layer_layout(int T, int H, int I, int E, int k, int mode, void* ws, Body&& body) {
  const LayerPlan p = plan_layer(T, E, k);
  const LayerPath lp = layer_path(p.R, H, I, E);
  Carver c(ws);
  int* ids = c.take<int>(p.R);
  float* w = c.take<float>(p.R);
  void* sort_ws = c.take<uint8_t>(p.sort_ws);
  int* counts = c.take<int>(E);
  int* offsets = c.take<int>(E + 1);
  int* perm = c.take<int>(p.R);
  int4* tiles = c.take<int4>(p.max_tiles);
  int* num_tiles = c.take<int>(1);
  void* sorted_x = lp.fuse_gather ? nullptr : c.take<__nv_bfloat16>(p.R * H);
  void* h = c.take<__nv_bfloat16>(p.R * I);
  // slot rows [R, H] bf16, or with the atomic combine fp32 token rows [T, H]
  void* slots = use_atomic_combine(mode, lp)
                    ? static_cast<void*>(c.take<float>(static_cast<size_t>(T) * H))
                    : static_cast<void*>(c.take<__nv_bfloat16>(p.R * H));
  // single-launch decode layer: router logits and its grid-barrier counters
  void* fused = lp.small && fused_decode_ok(T, H, I, E, k)
                    ? static_cast<void*>(c.take<uint8_t>(fused_decode_scratch_bytes(T, E)))
                    : nullptr;
  body(p, ids, w, sort_ws, counts, offsets, perm, tiles, num_tiles, sorted_x, h, slots, fused);
  return c.used;
}

}  // namespace

extern "C" {

int moe_abi_version(void) { return MOE_B200_ABI_VERSION; }

const char* moe_error_string(int code) {
  switch (code) {
    case kRcOk: return "ok";
    case kRcBadArgument: return "bad argument (null pointer, negative or inconsistent size, misaligned buffer)";
    case kRcUnsupported: return "shape not supported by these kernels";
    case kRcCudaError: return "CUDA runtime error while launching";
    case kRcTensorMap: return "tensor map encoding failed";
    case kRcWorkspace: return "workspace smaller than required";
    case kErrTimeoutFull: return "device: MMA warp timed out waiting for a shared-memory stage";
    case kErrTimeoutEmpty: return "device: TMA producer timed out waiting for a free stage";
    case kErrTimeoutAccFull: return "device: epilogue timed out waiting for the accumulator";
    case kErrTimeoutAccEmpty: return "device: MMA warp timed out waiting for the epilogue";
    case kErrPeerTimeout: return "device: timed out waiting for a peer rank of the expert-parallel group";
    case kErrTimeoutGrid: return "device: timed out in a grid-wide barrier of the single-launch decode layer";
    case kErrBadExpert: return "device: expert id out of range";
    case kErrBadRow: return "device: row index out of range";
    default: return "unknown code";
  }
}

int moe_router_topk(const void* x, const void* router_weight, const float* router_bias, int T,
                    int H, int E, int top_k, int norm_topk_prob, int32_t* topk_ids,
                    float* topk_weights, void* logits, int32_t* status, cudaStream_t stream) {
  return launch_router(x, router_weight, router_bias, T, H, E, top_k, norm_topk_prob, topk_ids,
                       topk_weights, logits, status, stream);
}

size_t moe_sort_align_workspace_bytes(int R, int E_local) {
  if (R < 0 || E_local <= 0) return 0;
  return sort_workspace_bytes(R, E_local);
}

int moe_max_tiles(int R, int E_local) { return moe_max_tiles_rows(R, E_local, MOE_BLOCK_M); }

int moe_max_tiles_rows(int R, int E_local, int tile_rows) {
  if (R < 0 || E_local <= 0 || (tile_rows != MOE_BLOCK_M && tile_rows != MOE_PAIR_TILE_ROWS))
    return 0;
  return max_tiles_bound(R, E_local, tile_rows);
}

int moe_sort_align(const int32_t* topk_ids, int R, int E, int e_begin, int E_local,
                   void* workspace, size_t workspace_bytes, int32_t* counts, int32_t* offsets,
                   int64_t* offsets64, int32_t* perm, int32_t* inv, int32_t* tiles,
                   int max_tiles, int32_t* num_tiles, int32_t* status, cudaStream_t stream) {
  return moe_sort_align_rows(topk_ids, R, E, e_begin, E_local, workspace, workspace_bytes, counts,
                             offsets, offsets64, perm, inv, tiles, max_tiles, num_tiles,
                             MOE_BLOCK_M, status, stream);
}

int moe_sort_align_rows(const int32_t* topk_ids, int R, int E, int e_begin, int E_local,
                        void* workspace, size_t workspace_bytes, int32_t* counts,
                        int32_t* offsets, int64_t* offsets64, int32_t* perm, int32_t* inv,
                        int32_t* tiles, int max_tiles, int32_t* num_tiles, int tile_rows,
                        int32_t* status, cudaStream_t stream) {
  if ((R > 0 && (topk_ids == nullptr || perm == nullptr)) || counts == nullptr ||
      offsets == nullptr || workspace == nullptr || tiles == nullptr || num_tiles == nullptr)
    return kRcBadArgument;
  if (tile_rows != MOE_BLOCK_M && tile_rows != MOE_PAIR_TILE_ROWS) return kRcBadArgument;
  if (R < 0 || E_local <= 0 || max_tiles < moe_max_tiles_rows(R, E_local, tile_rows))
    return kRcBadArgument;
  if (workspace_bytes < sort_workspace_bytes(R, E_local)) return kRcWorkspace;
  return launch_sort_align(topk_ids, R, E, e_begin, E_local, tile_rows, workspace, counts,
                           offsets, reinterpret_cast<long long*>(offsets64), perm, inv,
                           reinterpret_cast<int4*>(tiles), max_tiles, num_tiles, status, stream);
}

int moe_tiles_from_offsets(const int64_t* offsets, int E, int32_t* tiles, int max_tiles,
                           int32_t* num_tiles, int32_t* status, cudaStream_t stream) {
  if (offsets == nullptr || tiles == nullptr || num_tiles == nullptr || max_tiles < 0)
    return kRcBadArgument;
  return launch_tiles_from_offsets(reinterpret_cast<const long long*>(offsets), E, MOE_BLOCK_M,
                                   reinterpret_cast<int4*>(tiles), max_tiles, num_tiles, status,
                                   stream);
}

int moe_gather_rows(const void* src, int src_rows, const int32_t* index, int R,
                    const int32_t* count, int index_div, int H, void* dst, int32_t* status,
                    cudaStream_t stream) {
  if (R > 0 && (src == nullptr || index == nullptr || dst == nullptr)) return kRcBadArgument;
  return launch_gather_rows(src, src_rows, index, R, count, index_div, H, dst, status, stream);
}

int moe_grouped_w13_swiglu(const void* sorted_x, int M, const int32_t* tiles,
                           const int32_t* num_tiles, int max_tiles, const void* w_gate,
                           const void* w_up, int E, int H, int I, void* h, int32_t* status,
                           cudaStream_t stream) {
  return moe_grouped_w13_swiglu_rows(sorted_x, M, tiles, num_tiles, max_tiles, w_gate, w_up, E, H,
                                     I, h, MOE_BLOCK_M, status, stream);
}

int moe_grouped_w13_swiglu_rows(const void* sorted_x, int M, const int32_t* tiles,
                                const int32_t* num_tiles, int max_tiles, const void* w_gate,
                                const void* w_up, int E, int H, int I, void* h, int tile_rows,
                                int32_t* status, cudaStream_t stream) {
  if (tile_rows != MOE_BLOCK_M && tile_rows != MOE_PAIR_TILE_ROWS) return kRcBadArgument;
  return launch_w13_swiglu(sorted_x, M, reinterpret_cast<const int4*>(tiles), num_tiles, max_tiles,
                           w_gate, w_up, E, H, I, h, status, stream, tile_rows);
}

int moe_grouped_w13_swiglu_gather(const void* src, int src_rows, const int32_t* index,
                                  int index_div, int M, const int32_t* tiles,
                                  const int32_t* num_tiles, int max_tiles, const void* w_gate,
                                  const void* w_up, int E, int H, int I, void* h,
                                  int32_t* status, cudaStream_t stream) {
  return moe_grouped_w13_swiglu_gather_rows(src, src_rows, index, index_div, M, tiles, num_tiles,
                                            max_tiles, w_gate, w_up, E, H, I, h, MOE_BLOCK_M,
                                            status, stream);
}

int moe_grouped_w13_swiglu_gather_rows(const void* src, int src_rows, const int32_t* index,
                                       int index_div, int M, const int32_t* tiles,
                                       const int32_t* num_tiles, int max_tiles,
                                       const void* w_gate, const void* w_up, int E, int H, int I,
                                       void* h, int tile_rows, int32_t* status,
                                       cudaStream_t stream) {
  if (tile_rows != MOE_BLOCK_M && tile_rows != MOE_PAIR_TILE_ROWS) return kRcBadArgument;
  return launch_w13_swiglu_gather(src, src_rows, index, index_div, M,
                                  reinterpret_cast<const int4*>(tiles), num_tiles, max_tiles,
                                  w_gate, w_up, E, H, I, h, status, stream, tile_rows);
}

int moe_device_sm_count(void) { return device_sm_count(); }

size_t moe_decode_layer_workspace_bytes(int T, int H, int E) {
  if (T <= 0 || H <= 0 || E <= 0) return 0;
  return split_decode_scratch_bytes(T, H, E);
}

int moe_decode_layer_split(const void* x, const void* router_weight, const float* router_bias,
                           const void* w_gate, const void* w_up, const void* w_down_t, int T,
                           int H, int I, int E, int top_k, int norm_topk_prob, void* workspace,
                           size_t workspace_bytes, void* y, int32_t* status, cudaStream_t stream) {
  if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || top_k <= 0 || w_down_t == nullptr)
    return kRcBadArgument;
  if (!split_decode_ok(T, H, I, E, top_k)) return kRcUnsupported;
  if (workspace == nullptr || workspace_bytes < split_decode_scratch_bytes(T, H, E))
    return kRcWorkspace;
  return launch_decode_split(x, router_weight, router_bias, T, H, I, E, top_k, norm_topk_prob,
                             w_gate, w_up, w_down_t, workspace, y, status, stream);
}

int moe_last_cuda_error(void) { return last_cuda_error(); }

int moe_grouped_w13_swiglu_gather_ex(const void* src, int src_rows, const int32_t* index,
                                     int index_div, int M, const int32_t* tiles,
                                     const int32_t* num_tiles, int max_tiles, const void* w_gate,
                                     const void* w_up, int E, int H, int I, void* h,
                                     int tile_rows, int max_sms, int32_t* status,
                                     cudaStream_t stream) {
  if (tile_rows != MOE_BLOCK_M && tile_rows != MOE_PAIR_TILE_ROWS) return kRcBadArgument;
  return launch_w13_swiglu_gather(src, src_rows, index, index_div, M,
                                  reinterpret_cast<const int4*>(tiles), num_tiles, max_tiles,
                                  w_gate, w_up, E, H, I, h, status, stream, tile_rows, nullptr,
                                  max_sms);
}

int moe_grouped_w2_ex(const void* h, int M, const int32_t* tiles, const int32_t* num_tiles,
                      int max_tiles, const void* w_down, int E, int H, int I,
                      const int32_t* row_map, const float* slot_scale, void* out, int out_rows,
                      int tile_rows, int max_sms, int32_t* status, cudaStream_t stream) {
  if (tile_rows != MOE_BLOCK_M && tile_rows != MOE_PAIR_TILE_ROWS) return kRcBadArgument;
  return launch_w2(h, M, reinterpret_cast<const int4*>(tiles), num_tiles, max_tiles, w_down, E, H,
                   I, row_map, slot_scale, out, out_rows, status, stream, tile_rows, max_sms);
}

int moe_grouped_w2(const void* h, int M, const int32_t* tiles, const int32_t* num_tiles,
                   int max_tiles, const void* w_down, int E, int H, int I,
                   const int32_t* row_map, const float* slot_scale, void* out, int out_rows,
                   int32_t* status, cudaStream_t stream) {
  return moe_grouped_w2_rows(h, M, tiles, num_tiles, max_tiles, w_down, E, H, I, row_map,
                             slot_scale, out, out_rows, MOE_BLOCK_M, status, stream);
}

int moe_grouped_w2_rows(const void* h, int M, const int32_t* tiles, const int32_t* num_tiles,
                        int max_tiles, const void* w_down, int E, int H, int I,
                        const int32_t* row_map, const float* slot_scale, void* out, int out_rows,
                        int tile_rows, int32_t* status, cudaStream_t stream) {
  if (tile_rows != MOE_BLOCK_M && tile_rows != MOE_PAIR_TILE_ROWS) return kRcBadArgument;
  return launch_w2(h, M, reinterpret_cast<const int4*>(tiles), num_tiles, max_tiles, w_down, E, H,
                   I, row_map, slot_scale, out, out_rows, status, stream, tile_rows);
}

int moe_combine(const void* rows, int n_rows, const int32_t* slot_src, const float* slot_w,
                const int32_t* ids, int e_begin, int e_end, int T, int k, int H, void* y,
                int32_t* status, cudaStream_t stream) {
  if (T > 0 && (rows == nullptr || y == nullptr)) return kRcBadArgument;
  return launch_combine(rows, n_rows, slot_src, slot_w, ids, e_begin, e_end, T, k, H, y, status,
                        stream);
}

size_t moe_layer_workspace_bytes(int T, int H, int I, int E, int top_k) {
  return moe_layer_workspace_bytes_ex(T, H, I, E, top_k, MOE_COMBINE_SLOTS);
}

size_t moe_layer_workspace_bytes_ex(int T, int H, int I, int E, int top_k, int combine_mode) {
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || top_k <= 0) return 0;
  if (combine_mode != MOE_COMBINE_SLOTS && combine_mode != MOE_COMBINE_ATOMIC) return 0;
  // The layer refuses more than 2^31 - 1 routing records; so does its size query.
  if (static_cast<long long>(T) * top_k > 0x7fffffffLL) return 0;
  return layer_layout(T, H, I, E, top_k, combine_mode, nullptr, [](auto&&...) {});
}

int moe_grouped_w2_atomic_rows(const void* h, int M, const int32_t* tiles,
                               const int32_t* num_tiles, int max_tiles, const void* w_down, int E,
                               int H, int I, const int32_t* row_map, const float* slot_scale,
                               int n_slots, int red_div, float* out_f32, int tile_rows,
                               int32_t* status, cudaStream_t stream) {
  return launch_w2_atomic(h, M, reinterpret_cast<const int4*>(tiles), num_tiles, max_tiles,
                          w_down, E, H, I, row_map, slot_scale, n_slots, red_div, out_f32, status,
                          stream, tile_rows);
}

int moe_add_rmsnorm(const void* x, const void* delta, const float* weight, int T, int H,
                    float eps, void* h_out, void* y, cudaStream_t stream) {
  return launch_add_rmsnorm(x, delta, weight, T, H, eps, h_out, y, stream);
}

int moe_cast_f32_to_bf16(const float* src, long long n, void* y, cudaStream_t stream) {
  return launch_cast_f32_bf16(src, n, y, stream);
}

int moe_ep_keys(const int32_t* ids, int N, int k, int experts_per_rank, int ep, int32_t* keys,
                int32_t* status, cudaStream_t stream) {
  if (N > 0 && (ids == nullptr || keys == nullptr)) return kRcBadArgument;
  return launch_ep_keys(ids, N, k, experts_per_rank, ep, keys, status, stream);
}

int moe_ep_meta(const int32_t* perm, const int32_t* count, int max_rows, const int32_t* ids,
                const float* weights, int N, int k, int experts_per_rank, int ep, int32_t* meta,
                int32_t* status, cudaStream_t stream) {
  if (max_rows > 0 && (perm == nullptr || count == nullptr || ids == nullptr ||
                       weights == nullptr || meta == nullptr))
    return kRcBadArgument;
  return launch_ep_meta(perm, count, max_rows, ids, weights, N, k, experts_per_rank, ep, meta,
                        status, stream);
}

size_t moe_ep_peer_buffer_bytes(int ep, int cap_rows, int H, int k) {
  if (ep < 1 || ep > kMaxEpRanks || cap_rows < 0 || H <= 0 || k < 1) return 0;
  return peer_buffer_bytes(ep, cap_rows, H, k);
}

size_t moe_ep_peer_region_offset(int ep, int cap_rows, int H, int k, int region) {
  if (ep < 1 || ep > kMaxEpRanks || cap_rows < 0 || H <= 0 || k < 1) return 0;
  return peer_region_offset(ep, cap_rows, H, k, region);
}

void moe_ep_peer_set_wait_limit_ms(int ms) {
  set_peer_wait_limit(ms > 0 ? static_cast<unsigned long long>(ms) * 1000000ull : 0ull);
}

int moe_ep_peer_alloc(size_t bytes, void** buffer, void* ipc_handle) {
  return peer_alloc(bytes, buffer, ipc_handle);
}

int moe_ep_peer_open(const void* ipc_handle, void** buffer) { return peer_open(ipc_handle, buffer); }

int moe_ep_peer_close(void* buffer) { return peer_close(buffer); }

int moe_ep_peer_free(void* buffer) { return peer_free(buffer); }

int moe_ep_peer_dispatch(void* const* buffers, int ep, int rank, int cap_rows, int H, int k,
                         const int32_t* send_counts, const void* x, int N, const int32_t* perm,
                         const int32_t* ids, const float* weights, int experts_per_rank,
                         int32_t* status, cudaStream_t stream) {
  return launch_ep_peer_dispatch(buffers, ep, rank, cap_rows, H, k, send_counts, x, N, perm, ids,
                                 weights, experts_per_rank, status, stream);
}

int moe_ep_peer_return(void* const* buffers, int ep, int rank, int cap_rows, int H, int k,
                       const void* out, int out_rows, const int32_t* inv, int32_t* status,
                       cudaStream_t stream) {
  return launch_ep_peer_return(buffers, ep, rank, cap_rows, H, k, out, out_rows, inv, status,
                               stream);
}

int moe_layer_tile_rows(int T, int H, int I, int E, int top_k) {
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || top_k <= 0) return 0;
  return layer_path(static_cast<long long>(T) * top_k, H, I, E).tile_rows;
}

int moe_layer_forward(const void* x, const void* router_weight, const float* router_bias,
                      const void* w_gate, const void* w_up, const void* w_down, int T, int H,
                      int I, int E, int top_k, int norm_topk_prob, void* workspace,
                      size_t workspace_bytes, void* y, int32_t* status, cudaStream_t stream) {
  return moe_layer_forward_ex(x, router_weight, router_bias, w_gate, w_up, w_down, T, H, I, E,
                              top_k, norm_topk_prob, MOE_COMBINE_SLOTS, workspace,
                              workspace_bytes, y, status, stream);
}

int moe_layer_forward_ex(const void* x, const void* router_weight, const float* router_bias,
                         const void* w_gate, const void* w_up, const void* w_down, int T, int H,
                         int I, int E, int top_k, int norm_topk_prob, int combine_mode,
                         void* workspace, size_t workspace_bytes, void* y, int32_t* status,
                         cudaStream_t stream) {
  if (combine_mode != MOE_COMBINE_SLOTS && combine_mode != MOE_COMBINE_ATOMIC)
    return kRcBadArgument;
  if (router_weight == nullptr || w_gate == nullptr || w_up == nullptr || w_down == nullptr ||
      T < 0 || H <= 0 || I <= 0 || E <= 0 || top_k <= 0 || top_k > E)
    return kRcBadArgument;
  if (T == 0) return kRcOk;  // empty batch: nothing to read or write, x and y may be NULL
  if (x == nullptr || y == nullptr || workspace == nullptr) return kRcBadArgument;
  if (static_cast<long long>(T) * top_k > 0x7fffffffLL) return kRcUnsupported;
  if (workspace_bytes < moe_layer_workspace_bytes_ex(T, H, I, E, top_k, combine_mode))
    return kRcWorkspace;
  int rc = kRcOk;
  layer_layout(T, H, I, E, top_k, combine_mode, workspace,
               [&](const LayerPlan& p, int* ids, float* w, void* sort_ws, int* counts,
                   int* offsets, int* perm, int4* tiles, int* num_tiles, void* sorted_x, void* h,
                   void* slots, void* fused) {
                 const int R = static_cast<int>(p.R);
                 if (fused != nullptr) {
                   // T * k <= 32 records: the whole layer in one launch (bitwise
                   // the result of the four-launch decode path below, which runs
                   // instead if the cooperative launch is refused).
                   rc = launch_decode_fused(x, router_weight, router_bias, T, H, I, E, top_k,
                                            norm_topk_prob, w_gate, w_up, w_down, fused, h,
                                            slots, y, status, stream);
                   if (rc == kRcOk) return;
                   (void)cudaGetLastError();  // a refused launch leaves no sticky error
                   rc = kRcOk;
                 }
                 const LayerPath lp = layer_path(R, H, I, E);
                 const bool small = lp.small;  // decode: weight-streaming kernels
                 const int tile_rows = lp.tile_rows;  // 256: CTA-pair GEMMs
                 const int max_tiles = max_tiles_bound(R, E, tile_rows);
                 if (small && use_router_small(T, H, E, top_k)) {
                   rc = launch_router_sort_small(x, router_weight, router_bias, T, H, E, top_k,
                                                 norm_topk_prob, ids, w, nullptr, counts, offsets,
                                                 perm, tiles, p.max_tiles, num_tiles, status,
                                                 stream);
                 } else {
                   rc = launch_router(x, router_weight, router_bias, T, H, E, top_k,
                                      norm_topk_prob, ids, w, nullptr, status, stream);
                   if (rc == kRcOk)
                     rc = launch_sort_align(ids, R, E, 0, E, tile_rows, sort_ws, counts, offsets,
                                            nullptr, perm, nullptr, tiles, max_tiles, num_tiles,
                                            status, stream);
                 }
                 // The gate/up kernel gathers the token rows itself (always for the
                 // decode GEMV), or a separate gather writes the copy TMA reads.
                 if (rc == kRcOk && lp.fuse_gather) {
                   rc = launch_w13_swiglu_gather(x, T, perm, top_k, R, tiles, num_tiles,
                                                 max_tiles, w_gate, w_up, E, H, I, h, status,
                                                 stream, tile_rows, small ? w_down : nullptr);
                 } else if (rc == kRcOk) {
                   rc = launch_gather_rows(x, T, perm, R, nullptr, top_k, H, sorted_x, status,
                                           stream);
                   if (rc == kRcOk)
                     rc = launch_w13_swiglu(sorted_x, R, tiles, num_tiles, max_tiles, w_gate,
                                            w_up, E, H, I, h, status, stream, tile_rows);
                 }
                 if (use_atomic_combine(combine_mode, lp)) {
                   // index_add_ semantics: every record adds its weighted row into
                   // its token's fp32 row, then one rounding to bf16.
                   float* acc = static_cast<float*>(slots);
                   if (rc == kRcOk &&
                       cudaMemsetAsync(acc, 0, static_cast<size_t>(T) * H * sizeof(float),
                                       stream) != cudaSuccess)
                     rc = kRcCudaError;
                   if (rc == kRcOk)
                     rc = launch_w2_atomic(h, R, tiles, num_tiles, max_tiles, w_down, E, H, I,
                                           perm, w, R, top_k, acc, status, stream, tile_rows);
                   if (rc == kRcOk)
                     rc = launch_cast_f32_bf16(acc, static_cast<long long>(T) * H, y, stream);
                   return;
                 }
                 if (rc == kRcOk)
                   rc = launch_w2(h, R, tiles, num_tiles, max_tiles, w_down, E, H, I, perm, w,
                                  slots, R, status, stream, tile_rows);
                 if (rc == kRcOk)
                   rc = launch_combine(slots, R, nullptr, nullptr, nullptr, 0, E, T, top_k, H, y,
                                       status, stream);
               });
  return rc;
}

}  // extern "C"
