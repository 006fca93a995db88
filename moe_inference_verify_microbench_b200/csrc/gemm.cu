// Host launchers for the tcgen05 kernels: tensor-map encoding, tile-width
// selection, grid sizing (one persistent CTA per SM at most).
#include <atomic>
#include <mutex>

#include "grouped_gemm.cuh"
#include "grouped_gemm_pair.cuh"
#include "internal.h"
#include "router_splitk.cuh"

namespace moe {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 tensor map with 128-byte swizzle.  dims[0] is the contiguous extent in
// elements; strides (bytes) are given for dims 1..rank-1.
int make_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
             const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return kRcTensorMap;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return kRcBadArgument;
  for (int i = 0; i < rank - 1; ++i)
    if ((strides[i] & 15u) != 0) return kRcBadArgument;
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                         const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kRcOk : kRcTensorMap;
}

// Row-major [rows, cols] operand, box [box_rows, 64].
int map_2d(CUtensorMap* m, const void* base, long long rows, int cols, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  return make_map(m, base, 2, dims, strides, box);
}

// Expert-stacked [E, rows, cols] weights, box [1, box_rows, 64].
int map_3d(CUtensorMap* m, const void* base, int E, int rows, int cols, int box_rows) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(E)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 2,
                                 static_cast<cuuint64_t>(rows) * static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows), 1u};
  return make_map(m, base, 3, dims, strides, box);
}

constexpr int kMaxDevices = 64;
constexpr int kMaxSmemPerBlock = 232448;  // sm_100 opt-in dynamic shared memory per block

int device_sms() {
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// Grid of a persistent GEMM: one CTA per SM, at most `max_sms` SMs when > 0
// (the caller leaves the others to concurrent work, e.g. an expert-parallel
// exchange on another stream).
long long sm_budget(int max_sms) {
  const long long sms = device_sms();
  return max_sms > 0 && max_sms < sms ? max_sms : sms;
}

// Raise a kernel's dynamic shared memory limit to `bytes`, once per device.
template <class Kernel>
bool allow_kernel_smem(Kernel* fn, int bytes, std::atomic<uint64_t>& done) {
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

template <int BN, int EPI, int STAGES, bool GATHER_A = false>
int launch_gemm(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                const GemmArgs& args, long long work_units, cudaStream_t stream,
                int max_sms = 0) {
  using L = GemmSmem<BN, STAGES, gemm_out_bytes<EPI, GATHER_A>()>;
  static_assert(L::kTotal <= kMaxSmemPerBlock, "shared memory budget");
  static std::atomic<uint64_t> attr_done{0};  // one bit per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kRcCudaError;
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_done.load(std::memory_order_acquire) & bit) == 0) {
    if (cudaFuncSetAttribute(grouped_gemm_kernel<BN, EPI, STAGES, GATHER_A>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) != cudaSuccess)
      return kRcCudaError;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  const long long sms = sm_budget(max_sms);
  const int grid = static_cast<int>(work_units < sms ? work_units : sms);
  if (grid <= 0) return kRcOk;
  const cudaError_t e = launch_pdl(grouped_gemm_kernel<BN, EPI, STAGES, GATHER_A>, dim3(grid),
                                   dim3(gemm_threads<GATHER_A>()), L::kTotal, stream, a, b0, b1,
                                   args);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

template <int EPI, int STAGES, bool GATHER_A = false>
int launch_gemm_pair(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                     const GemmArgs& args, long long work_units, cudaStream_t stream,
                     int max_sms = 0) {
  using L = PairSmem<STAGES>;
  static_assert(L::kTotal <= kMaxSmemPerBlock, "shared memory budget");
  static std::atomic<uint64_t> attr_done{0};  // one bit per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kRcCudaError;
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_done.load(std::memory_order_acquire) & bit) == 0) {
    if (cudaFuncSetAttribute(grouped_gemm_pair_kernel<EPI, STAGES, GATHER_A>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) != cudaSuccess)
      return kRcCudaError;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  const long long pairs = sm_budget(max_sms) / 2;
  const int grid = 2 * static_cast<int>(work_units < pairs ? work_units : pairs);
  if (grid <= 0) return kRcOk;
  const cudaError_t e =
      launch_pdl_cluster(grouped_gemm_pair_kernel<EPI, STAGES, GATHER_A>, dim3(grid),
                         dim3(pair_threads<GATHER_A>()), L::kTotal, stream, 2u, a, b0, b1, args);
  return e == cudaSuccess ? kRcOk : kRcCudaError;
}

constexpr int kPairStages = 6;

// Widest N-tile (of those the shape allows) that still gives every SM a work
// unit; narrow tiles only pay off for small batches (decode), where the
// weights of a handful of experts must be streamed by all SMs at once.
// `n_out` is the output width per expert, `out_per_bn` maps a tile width to
// the output columns it produces, `rows` bounds the number of non-empty tiles.
template <class OutPerBn>
int pick_bn(int n_out, long long rows, int max_tiles, int allowed_mask, OutPerBn out_per_bn) {
  const long long tiles = rows < max_tiles ? rows : max_tiles;
  const long long sms = device_sms();
  int best = 0;
  for (int bn : {256, 128, 64}) {
    const int bit = bn == 256 ? 1 : bn == 128 ? 2 : 4;
    if (!(allowed_mask & bit) || n_out % out_per_bn(bn) != 0) continue;
    best = bn;
    if (tiles * (n_out / out_per_bn(bn)) >= sms) return bn;
  }
  return best;
}

GemmArgs blank_args(int* status) {
  GemmArgs g{};
  g.status = status;
  g.top_k = 1;
  g.norm_topk_prob = 1;
  return g;
}

}  // namespace

int device_sm_count() { return device_sms(); }

namespace {
thread_local int t_last_cuda_error = 0;
}

int last_cuda_error() { return t_last_cuda_error; }

cudaError_t note_cuda_error(cudaError_t e) {
  if (e != cudaSuccess) t_last_cuda_error = static_cast<int>(e);
  return e;
}

int launch_router(const void* x, const void* wr, const float* bias, int T, int H, int E, int k,
                  int norm_topk_prob, int* ids_out, float* w_out, void* logits_out, int* status,
                  cudaStream_t stream) {
  if ((T > 0 && (x == nullptr || ids_out == nullptr || w_out == nullptr)) || wr == nullptr ||
      T < 0 || H <= 0)
    return kRcBadArgument;
  if ((H % kBK) != 0 || (E % 16) != 0 || E < 16 || E > 256 || k < 1 || k > kRouterMaxK || k > E)
    return kRcUnsupported;
  if (T == 0) return kRcOk;
  if (use_router_small(T, H, E, k))
    return launch_router_sort_small(x, wr, bias, T, H, E, k, norm_topk_prob, ids_out, w_out,
                                    logits_out, nullptr, nullptr, nullptr, nullptr, 0, nullptr,
                                    status, stream);
  CUtensorMap ma, mb;
  int rc = map_2d(&ma, x, T, H, kBM);
  if (rc == kRcOk) rc = map_3d(&mb, wr, 1, E, H, E);
  if (rc != kRcOk) return rc;
  // At most 8 tiles of 128 tokens (T <= 1024): split K over a cluster of 2,
  // 4 or 8 CTAs per tile (router_splitk.cuh), so up to 8x the SMs stream the
  // operands.  Measured per layer (graph replay, H=2048 E=128): T=128 242 ->
  // 236 us, T=1024 264 -> 260 us; at 16 and more tiles the split measured
  // slower (T=2048 +10 us, T=4096 +4 us, T=8192 +26 us): its 200 KB-smem CTAs
  // then cover most SMs and delay the next kernels' early start.
  const int tiles = (T + kBM - 1) / kBM;
  const int nkb = H / kBK;
  int split = 1;
  if (E <= kRsMaxE && tiles <= kRsMaxTiles) {
    for (int cand : {8, 4, 2}) {
      if (static_cast<long long>(tiles) * cand <= device_sms() && nkb % cand == 0 &&
          nkb / cand >= 2) {
        split = cand;
        break;
      }
    }
  }
  if (split > 1) {
    static std::atomic<uint64_t> attr{0};
    if (!allow_kernel_smem(router_splitk, static_cast<int>(kRsSmemBytes), attr))
      return kRcCudaError;
    RouterSplitArgs ra{};
    ra.T = T;
    ra.E = E;
    ra.k = k;
    ra.norm_topk_prob = norm_topk_prob;
    ra.kb_per_split = nkb / split;
    ra.bias = bias;
    ra.ids_out = ids_out;
    ra.w_out = w_out;
    ra.logits_out = static_cast<__nv_bfloat16*>(logits_out);
    ra.status = status;
    const cudaError_t e =
        launch_pdl_cluster(router_splitk, dim3(tiles * split), dim3(kRsThreads), kRsSmemBytes,
                           stream, static_cast<unsigned>(split), ma, mb, ra);
    return note_cuda_error(e) == cudaSuccess ? kRcOk : kRcCudaError;
  }
  GemmArgs g = blank_args(status);
  g.max_tiles = tiles;
  g.n_tiles = 1;
  g.num_kb = H / kBK;
  g.b_rows = E;
  g.a_rows = T;
  g.num_experts = 1;
  g.bias = bias;
  g.top_k = k;
  g.norm_topk_prob = norm_topk_prob;
  g.ids_out = ids_out;
  g.w_out = w_out;
  g.logits_out = static_cast<__nv_bfloat16*>(logits_out);
  // E <= 128 fills a 128-column accumulator: half the B stage, six stages deep.
  if (E <= 128) return launch_gemm<128, kEpiRouter, 6>(ma, mb, mb, g, g.max_tiles, stream);
  return launch_gemm<256, kEpiRouter, 4>(ma, mb, mb, g, g.max_tiles, stream);
}

int launch_w13_swiglu(const void* a, int M, const int4* tiles, const int* num_tiles, int max_tiles,
                      const void* w_gate, const void* w_up, int E, int H, int I, void* h_out,
                      int* status, cudaStream_t stream, int tile_rows) {
  if ((M > 0 && (a == nullptr || h_out == nullptr)) || tiles == nullptr || num_tiles == nullptr ||
      w_gate == nullptr || w_up == nullptr || M < 0 || E <= 0 || H <= 0 || I <= 0 || max_tiles < 0)
    return kRcBadArgument;
  if (M == 0 || max_tiles == 0) return kRcOk;
  if (use_gemv_w13(M) && gemv_ok(I, H, true))
    return launch_w13_gemv(a, M, nullptr, 1, M, tiles, num_tiles, max_tiles, w_gate, w_up, E, H,
                           I, h_out, status, stream);
  if ((H % kBK) != 0 || (I % 32) != 0) return kRcUnsupported;
  if (tile_rows == kPairTileRows) {
    if ((I % (kPairBN / 2)) != 0) return kRcUnsupported;
    // Each CTA loads 64 gate rows and the 64 matching up rows per stage.
    CUtensorMap ma, mg, mu;
    int rc = map_2d(&ma, a, M, H, kBM);
    if (rc == kRcOk) rc = map_3d(&mg, w_gate, E, I, H, kPairBN / 4);
    if (rc == kRcOk) rc = map_3d(&mu, w_up, E, I, H, kPairBN / 4);
    if (rc != kRcOk) return rc;
    GemmArgs g = blank_args(status);
    g.tiles = tiles;
    g.num_tiles = num_tiles;
    g.max_tiles = max_tiles;
    g.n_tiles = I / (kPairBN / 2);
    g.num_kb = H / kBK;
    g.b_rows = kPairBN;
    g.a_rows = M;
    g.num_experts = E;
    g.out = static_cast<__nv_bfloat16*>(h_out);
    g.out_ld = I;
    g.out_rows = M;
    return launch_gemm_pair<kEpiSwiGLU, kPairStages>(
        ma, mg, mu, g, static_cast<long long>(max_tiles) * g.n_tiles, stream);
  }
  if (tile_rows != kBM) return kRcBadArgument;
  const int bn = pick_bn(I, M, max_tiles, 7, [](int b) { return b / 2; });
  CUtensorMap ma, mg, mu;
  int rc = map_2d(&ma, a, M, H, kBM);
  if (rc == kRcOk) rc = map_3d(&mg, w_gate, E, I, H, bn / 2);
  if (rc == kRcOk) rc = map_3d(&mu, w_up, E, I, H, bn / 2);
  if (rc != kRcOk) return rc;
  GemmArgs g = blank_args(status);
  g.tiles = tiles;
  g.num_tiles = num_tiles;
  g.max_tiles = max_tiles;
  g.n_tiles = I / (bn / 2);
  g.num_kb = H / kBK;
  g.b_rows = bn;
  g.a_rows = M;
  g.num_experts = E;
  g.out = static_cast<__nv_bfloat16*>(h_out);
  g.out_ld = I;
  g.out_rows = M;
  const long long units = static_cast<long long>(max_tiles) * g.n_tiles;
  if (bn == 256) return launch_gemm<256, kEpiSwiGLU, 4>(ma, mg, mu, g, units, stream);
  if (bn == 128) return launch_gemm<128, kEpiSwiGLU, 6>(ma, mg, mu, g, units, stream);
  return launch_gemm<64, kEpiSwiGLU, 8>(ma, mg, mu, g, units, stream);
}

int launch_w13_swiglu_gather(const void* src, int src_rows, const int* index, int index_div,
                             int M, const int4* tiles, const int* num_tiles, int max_tiles,
                             const void* w_gate, const void* w_up, int E, int H, int I,
                             void* h_out, int* status, cudaStream_t stream, int tile_rows,
                             const void* w_down_prefetch, int max_sms) {
  if ((M > 0 && (src == nullptr || h_out == nullptr)) || tiles == nullptr ||
      num_tiles == nullptr || w_gate == nullptr || w_up == nullptr || M < 0 || E <= 0 || H <= 0 ||
      I <= 0 || max_tiles < 0 || src_rows < 0 || index_div <= 0)
    return kRcBadArgument;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) return kRcBadArgument;
  if (M == 0 || max_tiles == 0) return kRcOk;
  if (src_rows == 0) return kRcBadArgument;  // rows to gather, but nothing to gather from
  if (use_gemv_w13(M) && gemv_ok(I, H, true))
    return launch_w13_gemv(src, src_rows, index, index_div, M, tiles, num_tiles, max_tiles,
                           w_gate, w_up, E, H, I, h_out, status, stream, w_down_prefetch,
                           max_sms);
  if ((H % kBK) != 0 || (I % 32) != 0) return kRcUnsupported;
  if (tile_rows == kPairTileRows) {
    if ((I % (kPairBN / 2)) != 0) return kRcUnsupported;
    // Each CTA loads 64 gate rows and the 64 matching up rows per stage.
    CUtensorMap mg, mu;
    int rc = map_3d(&mg, w_gate, E, I, H, kPairBN / 4);
    if (rc == kRcOk) rc = map_3d(&mu, w_up, E, I, H, kPairBN / 4);
    if (rc != kRcOk) return rc;
    GemmArgs g = blank_args(status);
    g.tiles = tiles;
    g.num_tiles = num_tiles;
    g.max_tiles = max_tiles;
    g.n_tiles = I / (kPairBN / 2);
    g.num_kb = H / kBK;
    g.b_rows = kPairBN;
    g.a_rows = M;
    g.num_experts = E;
    g.out = static_cast<__nv_bfloat16*>(h_out);
    g.out_ld = I;
    g.out_rows = M;
    g.a_src = static_cast<const __nv_bfloat16*>(src);
    g.a_src_rows = src_rows;
    g.a_index = index;
    g.a_index_div = index_div;
    // A is gathered by the loader warps; the gate map stands in for the unused A map.
    return launch_gemm_pair<kEpiSwiGLU, kPairStages, true>(
        mg, mg, mu, g, static_cast<long long>(max_tiles) * g.n_tiles, stream, max_sms);
  }
  if (tile_rows != kBM) return kRcBadArgument;
  const int bn = pick_bn(I, M, max_tiles, 7, [](int b) { return b / 2; });
  CUtensorMap mg, mu;
  int rc = map_3d(&mg, w_gate, E, I, H, bn / 2);
  if (rc == kRcOk) rc = map_3d(&mu, w_up, E, I, H, bn / 2);
  if (rc != kRcOk) return rc;
  GemmArgs g = blank_args(status);
  g.tiles = tiles;
  g.num_tiles = num_tiles;
  g.max_tiles = max_tiles;
  g.n_tiles = I / (bn / 2);
  g.num_kb = H / kBK;
  g.b_rows = bn;
  g.a_rows = M;
  g.num_experts = E;
  g.out = static_cast<__nv_bfloat16*>(h_out);
  g.out_ld = I;
  g.out_rows = M;
  g.a_src = static_cast<const __nv_bfloat16*>(src);
  g.a_src_rows = src_rows;
  g.a_index = index;
  g.a_index_div = index_div;
  const long long units = static_cast<long long>(max_tiles) * g.n_tiles;
  // A is gathered by the loader warps; the gate map stands in for the unused A map.
  if (bn == 256)
    return launch_gemm<256, kEpiSwiGLU, 4, true>(mg, mg, mu, g, units, stream, max_sms);
  if (bn == 128)
    return launch_gemm<128, kEpiSwiGLU, 6, true>(mg, mg, mu, g, units, stream, max_sms);
  return launch_gemm<64, kEpiSwiGLU, 8, true>(mg, mg, mu, g, units, stream, max_sms);
}

// Down GEMM on 256-row pair tiles or 128-row tiles; EPI = kEpiStore writes
// scaled bf16 rows to out[row_map[p]], kEpiAtomic adds them in fp32 to
// out_f32[row_map[p] / red_div].
template <int EPI>
static int launch_w2_gemm(const void* h, int M, const int4* tiles, const int* num_tiles,
                          int max_tiles, const void* w_down, int E, int H, int I,
                          const int* row_map, const float* row_scale, void* out, float* out_f32,
                          int red_div, int out_rows, int* status, cudaStream_t stream,
                          int tile_rows, int max_sms) {
  if ((I % kBK) != 0 || (H % 64) != 0) return kRcUnsupported;
  GemmArgs g = blank_args(status);
  g.tiles = tiles;
  g.num_tiles = num_tiles;
  g.max_tiles = max_tiles;
  g.num_kb = I / kBK;
  g.a_rows = M;
  g.num_experts = E;
  g.out = static_cast<__nv_bfloat16*>(out);
  g.out_f32 = out_f32;
  g.red_div = red_div;
  g.out_ld = H;
  g.out_rows = out_rows;
  g.row_map = row_map;
  g.row_scale = row_scale;
  if (tile_rows == kPairTileRows) {
    if ((H % kPairBN) != 0) return kRcUnsupported;
    CUtensorMap ma, md;
    int rc = map_2d(&ma, h, M, I, kBM);
    if (rc == kRcOk) rc = map_3d(&md, w_down, E, H, I, kPairBN / 2);
    if (rc != kRcOk) return rc;
    g.n_tiles = H / kPairBN;
    g.b_rows = kPairBN;
    return launch_gemm_pair<EPI, kPairStages>(
        ma, md, md, g, static_cast<long long>(max_tiles) * g.n_tiles, stream, max_sms);
  }
  if (tile_rows != kBM) return kRcBadArgument;
  const int bn = pick_bn(H, M, max_tiles, 7, [](int b) { return b; });
  CUtensorMap ma, md;
  int rc = map_2d(&ma, h, M, I, kBM);
  if (rc == kRcOk) rc = map_3d(&md, w_down, E, H, I, bn);
  if (rc != kRcOk) return rc;
  g.n_tiles = H / bn;
  g.b_rows = bn;
  const long long units = static_cast<long long>(max_tiles) * g.n_tiles;
  if (bn == 256) return launch_gemm<256, EPI, 4>(ma, md, md, g, units, stream, max_sms);
  if (bn == 128) return launch_gemm<128, EPI, 6>(ma, md, md, g, units, stream, max_sms);
  return launch_gemm<64, EPI, 8>(ma, md, md, g, units, stream, max_sms);
}

int launch_w2(const void* h, int M, const int4* tiles, const int* num_tiles, int max_tiles,
              const void* w_down, int E, int H, int I, const int* row_map, const float* row_scale,
              void* out, int out_rows, int* status, cudaStream_t stream, int tile_rows,
              int max_sms) {
  if ((M > 0 && (h == nullptr || out == nullptr)) || tiles == nullptr || num_tiles == nullptr ||
      w_down == nullptr || M < 0 || E <= 0 || H <= 0 || I <= 0 || max_tiles < 0 || out_rows < 0)
    return kRcBadArgument;
  if (M == 0 || max_tiles == 0) return kRcOk;
  if (use_gemv_w2(M) && gemv_ok(H, I, false))
    return launch_w2_gemv(h, M, tiles, num_tiles, max_tiles, w_down, E, H, I, row_map, row_scale,
                          out, out_rows, status, stream, max_sms);
  return launch_w2_gemm<kEpiStore>(h, M, tiles, num_tiles, max_tiles, w_down, E, H, I, row_map,
                                   row_scale, out, nullptr, 1, out_rows, status, stream, tile_rows,
                                   max_sms);
}

int launch_w2_atomic(const void* h, int M, const int4* tiles, const int* num_tiles,
                     int max_tiles, const void* w_down, int E, int H, int I, const int* row_map,
                     const float* row_scale, int n_slots, int red_div, float* out_f32,
                     int* status, cudaStream_t stream, int tile_rows) {
  if ((M > 0 && (h == nullptr || out_f32 == nullptr)) || tiles == nullptr ||
      num_tiles == nullptr || w_down == nullptr || M < 0 || E <= 0 || H <= 0 || I <= 0 ||
      max_tiles < 0 || n_slots < 0 || red_div <= 0)
    return kRcBadArgument;
  if ((reinterpret_cast<uintptr_t>(out_f32) & 15u) != 0) return kRcBadArgument;
  if (M == 0 || max_tiles == 0) return kRcOk;
  return launch_w2_gemm<kEpiAtomic>(h, M, tiles, num_tiles, max_tiles, w_down, E, H, I, row_map,
                                    row_scale, nullptr, out_f32, red_div, n_slots, status, stream,
                                    tile_rows, 0);
}

}  // namespace moe
