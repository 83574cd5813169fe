// Host-side launchers of every kernel, and the stage dispatchers.
#pragma once

#include "common.cuh"

namespace bsa {

// Stage 1 (pool.cu): blocks [block_begin, block_end) of every unit (end < 0:
// all nb), each the mean of its keys below s.kv.
// `zero`/`zero_bytes` (optional): a 16-byte-aligned region the kernel clears
// on the way (the fine stage's error word and work-item counter), saving a
// memset launch.
cudaError_t launch_pool_k(const __nv_bfloat16* K, float* K_repr, __nv_bfloat16* K_hi,
                          __nv_bfloat16* K_lo, const Shape& s, cudaStream_t st,
                          void* zero = nullptr, size_t zero_bytes = 0, int block_begin = 0,
                          int block_end = -1);

// Stages 2-3 (select_simt.cu, select_tc.cu).
cudaError_t launch_select_simt(const __nv_bfloat16* Q, const float* K_repr, int32_t* idx,
                               const Shape& s, cudaStream_t st);
bool select_tc_supported(const Shape& s);
cudaError_t launch_select_tc(const __nv_bfloat16* Q, const __nv_bfloat16* K_hi,
                             const __nv_bfloat16* K_lo, int32_t* idx, uint32_t* err,
                             const Shape& s, cudaStream_t st);

// Stage 4 (fine_simt.cu, fine_kv.cu).
cudaError_t launch_fine_simt(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, const int32_t* idx, __nv_bfloat16* O,
                             const Shape& s, cudaStream_t st);
bool fine_kv_supported(const Shape& s);
size_t fine_kv_workspace_bytes(const Shape& s);
size_t fine_kv_error_offset(const Shape& s);  // byte offset of the error word
size_t fine_kv_counters_offset(const Shape& s);  // byte offset of the per-pass counters
size_t fine_kv_zero_bytes(const Shape& s);    // bytes to clear at the start of the region
cudaError_t launch_fine_kv(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                           const __nv_bfloat16* V, const int32_t* idx, __nv_bfloat16* O,
                           unsigned char* ws, const Shape& s, uint32_t flags, cudaStream_t st,
                           int* n_launches, void* const* events, int n_events, bool pre_zeroed);
// Per (unit, key block) the query rows that picked it, from the forward's
// bucket kernels over every row (the fine workspace of `s` at `ws`):
// lists + unit * N * k + offsets[unit * nb + j] holds counts[unit * nb + j] rows.
struct BucketLists {
  const int32_t* lists;
  const int32_t* offsets;
  const int32_t* counts;
};
cudaError_t launch_bucket_lists(const int32_t* idx, const __nv_bfloat16* V, unsigned char* ws,
                                const Shape& s, cudaStream_t st, BucketLists* out);

// Backward of the fine stage (backward.cu): dQ, dK, dV for a fixed selection.
bool backward_supported(const Shape& s);
size_t backward_workspace_bytes(const Shape& s);
cudaError_t launch_backward(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                            const __nv_bfloat16* V, const __nv_bfloat16* O,
                            const __nv_bfloat16* dO, const int32_t* idx, __nv_bfloat16* dQ,
                            __nv_bfloat16* dK, __nv_bfloat16* dV, unsigned char* ws,
                            const Shape& s, cudaStream_t st);

// Query-stationary fine kernel for query tiles (fine_q.cu): the shapes it
// covers, the union limit for a tile under `flags` (0: none), tiles per
// unit, the tile classifier and the kernel.
bool fine_q_supported(const Shape& s);
int fine_q_max_union(const Shape& s, uint32_t flags);
int fine_q_tiles(const Shape& s);
int fine_q_min_tiles(const Shape& s, uint32_t flags);
cudaError_t launch_classify_tiles(const int32_t* idx, uint8_t* tile_mode, uint32_t* qt_bits,
                                  int4* qt_info, uint32_t* n_qt, const Shape& s, int max_union,
                                  cudaStream_t st);
cudaError_t launch_fine_q(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                          const int32_t* idx, __nv_bfloat16* O, const uint32_t* qt_bits,
                          const int4* qt_info, const uint32_t* n_qt, int min_q_tiles,
                          uint32_t* err, const Shape& s, cudaStream_t st);

// Decode (decode.cu): per new query row, the top-k cached blocks (a warp per
// row; exact top-k, lowest index on ties, ascending order, -1 padded).
cudaError_t launch_decode_select(const __nv_bfloat16* Q, const float* K_repr, int32_t* idx,
                                 const Shape& s, cudaStream_t st);
// Per-query-block selection (BSA_FLAG_QBLOCK): Q_repr (units, nb, D) fp32
// block means of Q; bidx (units, nb, k) the picks of each query block; idx
// (units, N, k) those picks repeated for every row of the block.
cudaError_t launch_qblock_select(const float* Q_repr, const float* K_repr, int32_t* bidx,
                                 int32_t* idx, const Shape& s, cudaStream_t st);
// Decode fine stage, a CTA per new row split over its selected blocks
// (block_size 32/64/128, head_dim 64/128; decode_fine_supported).
bool decode_fine_supported(const Shape& s);
// One decode step in one launch (the shapes decode_fine_supported accepts):
// append the new K/V rows at position s.q0, re-pool their block, select and
// attend the new row (s.Nq = 1, s.kv = s.q0 + 1).
cudaError_t launch_decode_step(const __nv_bfloat16* q_new, const __nv_bfloat16* k_new,
                               const __nv_bfloat16* v_new, __nv_bfloat16* K, __nv_bfloat16* V,
                               float* K_repr, __nv_bfloat16* O, const Shape& s,
                               cudaStream_t st);
cudaError_t launch_decode_fine(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, const int32_t* idx, __nv_bfloat16* O,
                               const Shape& s, cudaStream_t st);

// Dispatchers (dispatch.cu).
bool select_uses_tensor_cores(const Shape& s, uint32_t flags);
bool fine_uses_tensor_cores(const Shape& s, uint32_t flags);
cudaError_t launch_select(const __nv_bfloat16* Q, const float* K_repr, const __nv_bfloat16* K_hi,
                          const __nv_bfloat16* K_lo, int32_t* idx, uint32_t* err, const Shape& s,
                          uint32_t flags, cudaStream_t st, int* n_launches);
size_t fine_workspace_bytes(const Shape& s, uint32_t flags);
cudaError_t launch_fine(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                        const int32_t* idx, __nv_bfloat16* O, unsigned char* ws, size_t ws_bytes,
                        const Shape& s, uint32_t flags, cudaStream_t st, int* n_launches,
                        void* const* events, int n_events, bool pre_zeroed);

}  // namespace bsa
