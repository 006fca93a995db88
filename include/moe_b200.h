/*
 * moe_b200.h — C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * Drop-in kernels for the MoE layer of weidotwisc/moe_inference_verify_microbench
 * (Qwen3-30B-A3B shapes: H=2048, I=768, E=128, top-8, bf16).  Every entry point:
 *   - takes plain device pointers, sizes and a cudaStream_t; no torch types;
 *   - is stream-ordered and never synchronises the host;
 *   - returns an int: 0 on success, a negative MOE_RC_* code for a host-side
 *     argument / shape / launch problem (nothing is launched then);
 *   - writes device-side failures (expert id out of range, a bounded wait that
 *     ran out) into the caller's device status word `status` (int32, may be
 *     NULL); the first failure wins, 0 means none.  Read it after the stream
 *     has finished; moe_error_string() names both kinds of code;
 *   - accepts an empty batch (T, M or R = 0) and returns 0; the per-token /
 *     per-record buffers may then be NULL (an empty torch tensor has no
 *     storage), weights and tile tables may not.  Nothing is launched,
 *     except where fixed-size outputs remain to be written (the sort still
 *     writes zero counts, offsets and tile count).
 * The caller owns all memory.  Scratch space is passed in as `workspace`, with
 * its size given by the matching *_workspace_bytes() query.
 *
 * Layouts (row-major, bf16 unless noted):
 *   x [T, H]; router weight [E, H]; w_gate, w_up [E, I, H]; w_down [E, H, I];
 *   top-k ids int32 [T, k], weights fp32 [T, k]; a "slot" is s = n*k + j.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 5

#define MOE_RC_OK 0
#define MOE_RC_BAD_ARGUMENT (-1)
#define MOE_RC_UNSUPPORTED (-2)
#define MOE_RC_CUDA_ERROR (-3)
#define MOE_RC_TENSOR_MAP (-4)
#define MOE_RC_WORKSPACE (-5)

/* Device status codes (first failure wins). */
#define MOE_ERR_TIMEOUT_FULL 0x101
#define MOE_ERR_TIMEOUT_EMPTY 0x102
#define MOE_ERR_TIMEOUT_ACC_FULL 0x103
#define MOE_ERR_TIMEOUT_ACC_EMPTY 0x104
#define MOE_ERR_PEER_TIMEOUT 0x105
#define MOE_ERR_TIMEOUT_GRID 0x106
#define MOE_ERR_BAD_EXPERT 0x201
#define MOE_ERR_BAD_ROW 0x202

/* Rows per M-tile of the grouped GEMMs (the C9 BLOCK_M), and the taller
 * tile of the 2-CTA cluster-pair GEMMs that large batches use (ABI 2). */
#define MOE_BLOCK_M 128
#define MOE_PAIR_TILE_ROWS 256

/* How the weighted expert rows become y (ABI 4): MOE_COMBINE_SLOTS writes
 * every record's row to its slot and sums each token's k slots in slot order
 * (bitwise reproducible); MOE_COMBINE_ATOMIC adds every record's row into its
 * token's fp32 row with atomics, as index_add_ does on CUDA, and rounds once
 * (the order of the k additions, hence the last fp32 bits, may vary). */
#define MOE_COMBINE_SLOTS 0
#define MOE_COMBINE_ATOMIC 1

MOE_API int moe_abi_version(void);

/* Text for a MOE_RC_* return code or a device status code. */
MOE_API const char* moe_error_string(int code);

/*
 * Router: logits = bf16(x @ Wr^T [+ bias]) on tcgen05, then per token the
 * top-k experts (value descending, lower expert id first among equal values)
 * and their weights: softmax over the k selected logits when norm_topk_prob,
 * else the softmax over all E gathered at the selected ids.
 * Replaces C5/python/solution.py:124-129 (same in C6:127-133, C7:141-146,
 * C8:171-176).  `router_bias` (fp32 [E]) may be NULL; `logits` (bf16 [T, E])
 * may be NULL.  Needs H % 64 == 0, E % 16 == 0, 16 <= E <= 256, 1 <= k <= 8.
 */
MOE_API int moe_router_topk(const void* x, const void* router_weight, const float* router_bias, int T,
                    int H, int E, int top_k, int norm_topk_prob, int32_t* topk_ids,
                    float* topk_weights, void* logits, int32_t* status, cudaStream_t stream);

/*
 * Stable counting sort of R = T*k routing records by expert, restricted to
 * experts [e_begin, e_begin + E_local) (all records when e_begin = 0 and
 * E_local = E).  Outputs, all on the device:
 *   counts[E_local], offsets[E_local + 1] (int32, offsets[0] = 0) and
 *   optionally offsets64 (int64, the C9 `offsets` argument);
 *   perm[p] = slot of the p-th record in expert order (stable: slot order
 *   inside an expert), p < offsets[E_local];
 *   inv[s] = position of slot s, or -1 for a record outside the range (may be NULL);
 *   tiles[max_tiles][4] = {local expert, row_begin, row_end, 0} per 128-row
 *   M-tile and num_tiles[0] = their count (the C9 _build_meta_data).
 * Replaces C5/python/solution.py:131-136 (torch.sort + bincount), the
 * local-expert filter and stable sort of C6/python/solution.py:137-160, and
 * C9/python/solution.py:142-159 (_build_meta_data), with no host sync.
 * max_tiles must be >= moe_max_tiles(R, E_local).
 */
MOE_API size_t moe_sort_align_workspace_bytes(int R, int E_local);
MOE_API int moe_max_tiles(int R, int E_local);
MOE_API int moe_sort_align(const int32_t* topk_ids, int R, int E, int e_begin, int E_local,
                   void* workspace, size_t workspace_bytes, int32_t* counts, int32_t* offsets,
                   int64_t* offsets64, int32_t* perm, int32_t* inv, int32_t* tiles,
                   int max_tiles, int32_t* num_tiles, int32_t* status, cudaStream_t stream);

/*
 * moe_sort_align without a workspace: the same kernels and the same outputs,
 * with the per-CTA histogram scratch kept in a device array owned by the
 * library (MOE_SORT_STATIC_SCRATCH_INTS int32 = 256 KiB, allocated on every
 * GPU that loads the library and held until the process exits).  This entry
 * point has no counterpart in the reference; it exists for callers that
 * cannot allocate device memory themselves (a host framework that owns every
 * device allocation, or a serving process that forbids allocation, and the
 * device synchronisation cudaMalloc may bring, once it is running).  It calls
 * no allocator.
 * Limit: ceil(R / 2048) * E_local <= MOE_SORT_STATIC_SCRATCH_INTS (for
 * E_local = 128, R <= 1,048,576 records); larger requests return
 * MOE_RC_WORKSPACE and launch nothing.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  All calls on a device share the one array, so
 * calls whose kernels overlap on the GPU (different streams, no ordering
 * between them) race and corrupt each other's results; calls ordered on one
 * stream are safe.  The array keeps the last call's contents; every entry a
 * call reads is first written by that call, so nothing needs clearing.
 */
#define MOE_SORT_STATIC_SCRATCH_INTS 65536
MOE_API int moe_sort_align_static_scratch(const int32_t* topk_ids, int R, int E, int e_begin,
                                          int E_local, int32_t* counts, int32_t* offsets,
                                          int64_t* offsets64, int32_t* perm, int32_t* inv,
                                          int32_t* tiles, int max_tiles, int32_t* num_tiles,
                                          int32_t* status, cudaStream_t stream);

/*
 * Tile table from caller-given int64 offsets[E + 1] (the C9 interface, where
 * the caller already holds sorted rows).  Replaces
 * C9/python/solution.py:142-159.
 */
MOE_API int moe_tiles_from_offsets(const int64_t* offsets, int E, int32_t* tiles, int max_tiles,
                           int32_t* num_tiles, int32_t* status, cudaStream_t stream);

/*
 * dst[p, :] = src[index[p] / index_div, :] for p < R, and p < count[0] when
 * `count` (a device int32, e.g. offsets + E_local) is not NULL; rows of H bf16.
 * With index = perm and index_div = k this is the permuted gather
 * x_flat[token_ids_rep[perm]] of C5/python/solution.py:135-137.  H % 8 == 0.
 */
MOE_API int moe_gather_rows(const void* src, int src_rows, const int32_t* index, int R,
                    const int32_t* count, int index_div, int H, void* dst, int32_t* status,
                    cudaStream_t stream);

/*
 * Grouped gate/up GEMM with the SwiGLU fused in the epilogue:
 *   h[r, :] = silu(A[r] @ w_gate[e]^T) * (A[r] @ w_up[e]^T) for rows r of tile
 *   entries {e, row_begin, row_end}; A is [M, H], h is [M, I].
 * Replaces the gate/up grouped matmuls and silu*mul of
 * C9/python/solution.py:218-220 (and C5/python/solution.py:79-80 per expert).
 * Needs H % 64 == 0, I % 32 == 0.
 */
MOE_API int moe_grouped_w13_swiglu(const void* sorted_x, int M, const int32_t* tiles,
                           const int32_t* num_tiles, int max_tiles, const void* w_gate,
                           const void* w_up, int E, int H, int I, void* h, int32_t* status,
                           cudaStream_t stream);

/*
 * moe_grouped_w13_swiglu with the row gather fused into the A-operand load:
 * A row r is src[index[r] / index_div] (index = perm, index_div = k reads
 * each routing record's token straight from x), so the [M, H] sorted copy of
 * the activations (C5/python/solution.py:137) is never written.  Rows of a
 * tile past its row_end are zero-filled.  src must be 16-byte aligned.
 */
MOE_API int moe_grouped_w13_swiglu_gather(const void* src, int src_rows, const int32_t* index,
                                          int index_div, int M, const int32_t* tiles,
                                          const int32_t* num_tiles, int max_tiles,
                                          const void* w_gate, const void* w_up, int E, int H,
                                          int I, void* h, int32_t* status, cudaStream_t stream);

/*
 * Grouped down GEMM with a scatter/scale epilogue:
 *   out[m(r), :] = s(m(r)) * (h[r] @ w_down[e]^T), m = row_map (identity when
 *   NULL), s = slot_scale (1 when NULL).  With row_map = perm and slot_scale =
 *   the flat top-k weights, each slot's weighted expert output lands in row
 *   n*k + j.  Replaces C9/python/solution.py:221 and the weight scale of
 *   C5/python/solution.py:158.  Needs I % 64 == 0, H % 64 == 0.
 */
MOE_API int moe_grouped_w2(const void* h, int M, const int32_t* tiles, const int32_t* num_tiles,
                   int max_tiles, const void* w_down, int E, int H, int I,
                   const int32_t* row_map, const float* slot_scale, void* out, int out_rows,
                   int32_t* status, cudaStream_t stream);

/*
 * y[n, :] = sum_j w_j * rows[src_j, :], j < k, fp32 accumulate in slot order:
 * src_j = slot_src[n*k+j] (n*k+j when NULL), w_j = slot_w[n*k+j] (1 when NULL);
 * slots with src_j < 0 or an expert id ids[n*k+j] outside [e_begin, e_end)
 * (no filter when ids is NULL) add nothing; 1 <= k <= 8.  Replaces the index_add_
 * un-permute of C5/python/solution.py:160, C6/python/solution.py:175-176,
 * C7/python/solution.py:259-261 and C8/python/solution.py:221-224.
 */
MOE_API int moe_combine(const void* rows, int n_rows, const int32_t* slot_src, const float* slot_w,
                const int32_t* ids, int e_begin, int e_end, int T, int k, int H, void* y,
                int32_t* status, cudaStream_t stream);

/*
 * Whole single-device MoE layer, PermutedSparseMoE.forward
 * (C5/python/solution.py:108-161): router -> sort -> gather -> w13+SwiGLU ->
 * w2 (weighted, to slot rows) -> k-way combine into y [T, H].  No host sync.
 * workspace >= moe_layer_workspace_bytes(...).
 */
MOE_API size_t moe_layer_workspace_bytes(int T, int H, int I, int E, int top_k);
MOE_API int moe_layer_forward(const void* x, const void* router_weight, const float* router_bias,
                      const void* w_gate, const void* w_up, const void* w_down, int T, int H,
                      int I, int E, int top_k, int norm_topk_prob, void* workspace,
                      size_t workspace_bytes, void* y, int32_t* status, cudaStream_t stream);

/*
 * ABI 2: tile tables of either height.  moe_layer_forward sorts into
 * MOE_PAIR_TILE_ROWS-row tiles once the average expert has >= 1024 routing
 * records and then runs its grouped GEMMs as 2-CTA cluster pairs
 * (tcgen05.mma.cta_group::2, M = 256), gathering the token rows inside the
 * gate/up GEMM.  The *_rows entry points are the entry points above with the
 * height of the tile table they build or read (MOE_BLOCK_M or
 * MOE_PAIR_TILE_ROWS) as an extra argument; with MOE_BLOCK_M they are
 * identical to them.  moe_layer_tile_rows returns the height the layer picks
 * for a shape, so a caller can run the layer's own kernels one by one.
 */
MOE_API int moe_layer_tile_rows(int T, int H, int I, int E, int top_k);
MOE_API int moe_max_tiles_rows(int R, int E_local, int tile_rows);
MOE_API int moe_sort_align_rows(const int32_t* topk_ids, int R, int E, int e_begin, int E_local,
                                void* workspace, size_t workspace_bytes, int32_t* counts,
                                int32_t* offsets, int64_t* offsets64, int32_t* perm, int32_t* inv,
                                int32_t* tiles, int max_tiles, int32_t* num_tiles, int tile_rows,
                                int32_t* status, cudaStream_t stream);
MOE_API int moe_grouped_w13_swiglu_rows(const void* sorted_x, int M, const int32_t* tiles,
                                        const int32_t* num_tiles, int max_tiles,
                                        const void* w_gate, const void* w_up, int E, int H, int I,
                                        void* h, int tile_rows, int32_t* status,
                                        cudaStream_t stream);
MOE_API int moe_grouped_w13_swiglu_gather_rows(const void* src, int src_rows,
                                               const int32_t* index, int index_div, int M,
                                               const int32_t* tiles, const int32_t* num_tiles,
                                               int max_tiles, const void* w_gate, const void* w_up,
                                               int E, int H, int I, void* h, int tile_rows,
                                               int32_t* status, cudaStream_t stream);
MOE_API int moe_grouped_w2_rows(const void* h, int M, const int32_t* tiles,
                                const int32_t* num_tiles, int max_tiles, const void* w_down, int E,
                                int H, int I, const int32_t* row_map, const float* slot_scale,
                                void* out, int out_rows, int tile_rows, int32_t* status,
                                cudaStream_t stream);

/*
 * ABI 4: the index_add_ semantics switch.  The reference un-permutes with
 * index_add_ (C5/python/solution.py:160, C6/python/solution.py:175-176), an
 * atomic fp32 accumulation on CUDA; the default here is the reproducible slot
 * rows + k-sum.  moe_layer_forward_ex takes the combine mode
 * (MOE_COMBINE_SLOTS: identical to moe_layer_forward; MOE_COMBINE_ATOMIC:
 * the down GEMM adds every record's weighted row into its token's fp32 row in
 * the workspace, then one rounding to y; decode-size batches that run the
 * weight-streaming kernels keep the slot rows).  Its workspace is
 * moe_layer_workspace_bytes_ex(..., combine_mode).
 *   moe_grouped_w2_atomic_rows: out_f32[row_map[p] / red_div, :] +=
 *     slot_scale[row_map[p]] * (h[p] @ w_down[e]^T) for the rows of the tile
 *     table (row_map NULL: identity; slot_scale NULL: 1; row_map[p] <
 *     n_slots); out_f32 [n_slots / red_div, H] fp32, zeroed by the caller.
 *   moe_cast_f32_to_bf16: y[i] = bf16(src[i]), n a multiple of 8.
 */
MOE_API size_t moe_layer_workspace_bytes_ex(int T, int H, int I, int E, int top_k,
                                            int combine_mode);
MOE_API int moe_layer_forward_ex(const void* x, const void* router_weight,
                                 const float* router_bias, const void* w_gate, const void* w_up,
                                 const void* w_down, int T, int H, int I, int E, int top_k,
                                 int norm_topk_prob, int combine_mode, void* workspace,
                                 size_t workspace_bytes, void* y, int32_t* status,
                                 cudaStream_t stream);
MOE_API int moe_grouped_w2_atomic_rows(const void* h, int M, const int32_t* tiles,
                                       const int32_t* num_tiles, int max_tiles,
                                       const void* w_down, int E, int H, int I,
                                       const int32_t* row_map, const float* slot_scale,
                                       int n_slots, int red_div, float* out_f32, int tile_rows,
                                       int32_t* status, cudaStream_t stream);
MOE_API int moe_cast_f32_to_bf16(const float* src, long long n, void* y, cudaStream_t stream);

/*
 * ABI 5: an SM budget for the grouped GEMMs.  The persistent GEMMs take one
 * CTA per SM on every SM; these variants of moe_grouped_w13_swiglu_gather_rows
 * and moe_grouped_w2_rows use at most `max_sms` SMs (<= 0: all), leaving the
 * others to work the caller runs at the same time on another stream -- the
 * expert-parallel exchange of the next token chunk while this chunk's expert
 * GEMMs run (the pipelined form of C7/python/solution.py:186-261).  Results
 * are bitwise those of the unbudgeted calls.  moe_device_sm_count() is the
 * current device's SM count.
 */
MOE_API int moe_device_sm_count(void);
MOE_API int moe_grouped_w13_swiglu_gather_ex(const void* src, int src_rows, const int32_t* index,
                                             int index_div, int M, const int32_t* tiles,
                                             const int32_t* num_tiles, int max_tiles,
                                             const void* w_gate, const void* w_up, int E, int H,
                                             int I, void* h, int tile_rows, int max_sms,
                                             int32_t* status, cudaStream_t stream);
MOE_API int moe_grouped_w2_ex(const void* h, int M, const int32_t* tiles,
                              const int32_t* num_tiles, int max_tiles, const void* w_down, int E,
                              int H, int I, const int32_t* row_map, const float* slot_scale,
                              void* out, int out_rows, int tile_rows, int max_sms,
                              int32_t* status, cudaStream_t stream);

/*
 * ABI 5: the decode layer in one launch and one pass over the weights, for a
 * caller that also keeps the down weights transposed: w_down_t [E][I][H] bf16
 * (w_down_t[e][i][h] = w_down[e][h][i], built once next to the weights).
 * T <= 4 tokens and T * top_k <= 32 records (C5/python/solution.py:108-161
 * for a decode batch).  Router, top-k and sort as moe_layer_forward's decode
 * path; then every CTA streams 8-row slices of gate, up and w_down_t of the
 * routed experts, forms h for those rows and adds their share of the down
 * projection to fp32 partials, summed across CTAs after one grid barrier.
 * The result equals moe_layer_forward's up to fp32 summation order over I.
 * No fallback: MOE_RC_UNSUPPORTED for a shape outside the bounds (also H > 2048
 * or I % 8 != 0), MOE_RC_CUDA if the cooperative launch fails.  workspace
 * holds moe_decode_layer_workspace_bytes(T, H, E) bytes, 16-byte aligned.
 *
 * moe_last_cuda_error: the cudaError_t value of the most recent CUDA call
 * that failed inside this library's launchers on the calling thread (0 when
 * none has), for diagnosing MOE_RC_CUDA.
 */
MOE_API size_t moe_decode_layer_workspace_bytes(int T, int H, int E);
MOE_API int moe_decode_layer_split(const void* x, const void* router_weight,
                                   const float* router_bias, const void* w_gate,
                                   const void* w_up, const void* w_down_t, int T, int H, int I,
                                   int E, int top_k, int norm_topk_prob, void* workspace,
                                   size_t workspace_bytes, void* y, int32_t* status,
                                   cudaStream_t stream);
MOE_API int moe_last_cuda_error(void);

/*
 * Decoder-block glue around the MoE (C8/python/solution.py:235-325, whose
 * block is h = x + attn(norm(x)); y = h + moe(norm(h)) with the suite's
 * RMSNorm: fp32 x * rsqrt(mean(x^2) + eps) * weight, cast back to bf16):
 * h_out = bf16(x + delta) (skipped when delta is NULL: h = x), then
 * y = RMSNorm(h) with weight fp32 [H].  x, delta, h_out, y bf16 [T, H],
 * H % 8 == 0, one pass over the rows.
 */
MOE_API int moe_add_rmsnorm(const void* x, const void* delta, const float* weight, int T, int H,
                            float eps, void* h_out, void* y, cudaStream_t stream);

/*
 * Send plan of the all_to_all expert-parallel schedule (C7/python/solution.py:
 * 150-203), which here dispatches one row per (token, owner rank):
 *   moe_ep_keys: keys[n*ep + r] = r if one of ids[n, 0..k) lies in rank r's
 *     experts [r*experts_per_rank, (r+1)*experts_per_rank), else ep; a stable
 *     moe_sort_align of the keys (E = ep + 1, E_local = ep) gives per-rank
 *     send counts and the rank-major send order perm (pair = n*ep + r).
 *   moe_ep_meta: for send row i < min(max_rows, *count), the int32 row
 *     meta[i, 0..2k) = k local expert ids on r (experts_per_rank where expert
 *     j of token n is not on r) and the k matching weights bit-cast (0 where
 *     not on r), the metadata that travels with the row.
 */
MOE_API int moe_ep_keys(const int32_t* ids, int N, int k, int experts_per_rank, int ep,
                        int32_t* keys, int32_t* status, cudaStream_t stream);
MOE_API int moe_ep_meta(const int32_t* perm, const int32_t* count, int max_rows,
                        const int32_t* ids, const float* weights, int N, int k,
                        int experts_per_rank, int ep, int32_t* meta, int32_t* status,
                        cudaStream_t stream);

/*
 * Peer-store exchange of the all_to_all expert-parallel schedule (replaces the
 * count all_to_all + host .tolist() + dispatch and combine all_to_alls of
 * C7/python/solution.py:186-261 and C8/python/solution.py:171-224) over NVLink
 * with device-resident split sizes.  Every rank of the group allocates one
 * peer buffer of moe_ep_peer_buffer_bytes(ep, cap_rows, H, k) bytes with
 * moe_ep_peer_alloc (zeroed; 64-byte CUDA IPC handle out), exchanges the
 * handles, and maps every other rank's buffer with moe_ep_peer_open;
 * buffers[q] is rank q's buffer in this process (buffers[rank] its own).
 * cap_rows bounds both the rows a rank sends and the rows it receives
 * (ep x the largest per-rank token count); every rank passes the same
 * ep, cap_rows, H and k.  The ranks must run on distinct GPUs.
 *
 * Regions of a buffer (moe_ep_peer_region_offset, region =):
 *   0 recv_ids  int32 [cap_rows, k]  expert ids of received rows, localised
 *                                    (experts_per_rank: not this rank's)
 *   1 recv_w    fp32  [cap_rows, k]  their weights (0 where not this rank's)
 *   2 recv_rows bf16  [cap_rows, H]  received token rows, source-major
 *   3 ret_rows  bf16  [cap_rows, H]  returned partial rows in send order
 *
 * moe_ep_peer_dispatch (one forward's first half; all ranks, same order):
 *   send_counts[d] rows for rank d (d < ep) in the rank-major send order
 *   perm[i] = n*ep + d (moe_ep_keys + moe_sort_align); x [N, H] bf16;
 *   ids [N, k] global expert ids, weights [N, k].  On return (stream order)
 *   recv_ids/recv_w/recv_rows hold this rank's received rows and recv_ids
 *   rows past them hold the sentinel experts_per_rank.
 * moe_ep_peer_return (second half): out [out_rows, H] bf16 holds the expert
 *   output of record p of the received rows at row inv[p] (inv < 0: none);
 *   every received row's weighted record sum goes back to its source, whose
 *   ret_rows then hold one partial row per send position.
 * A peer that does not signal within the wait limit (10 s; ms <= 0 restores
 * it) records MOE_ERR_PEER_TIMEOUT (0x105) in *status; the kernels still end.
 * The limit is read when a dispatch or return is enqueued.
 */
MOE_API void moe_ep_peer_set_wait_limit_ms(int ms);
MOE_API size_t moe_ep_peer_buffer_bytes(int ep, int cap_rows, int H, int k);
MOE_API size_t moe_ep_peer_region_offset(int ep, int cap_rows, int H, int k, int region);
MOE_API int moe_ep_peer_alloc(size_t bytes, void** buffer, void* ipc_handle);
MOE_API int moe_ep_peer_open(const void* ipc_handle, void** buffer);
MOE_API int moe_ep_peer_close(void* buffer);
MOE_API int moe_ep_peer_free(void* buffer);
MOE_API int moe_ep_peer_dispatch(void* const* buffers, int ep, int rank, int cap_rows, int H,
                                 int k, const int32_t* send_counts, const void* x, int N,
                                 const int32_t* perm, const int32_t* ids, const float* weights,
                                 int experts_per_rank, int32_t* status, cudaStream_t stream);
MOE_API int moe_ep_peer_return(void* const* buffers, int ep, int rank, int cap_rows, int H, int k,
                               const void* out, int out_rows, const int32_t* inv,
                               int32_t* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
