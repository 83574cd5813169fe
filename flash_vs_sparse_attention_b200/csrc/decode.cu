// Decode-time reuse: stages 2-4 for a few new query rows against a KV cache
// and its cached block means (block_indexer.py:44-84 evaluated at the new
// rows' positions; the reference itself has no decode path).
//
// Selection: a CTA per (unit, new row).  Its threads score the visible blocks
// in fp32, each a sequential dot product over head_dim exactly as the
// CUDA-core scorer computes it (every load of a block-mean row issued before
// the first use), into shared memory; warp 0 then runs top_k rounds of a warp
// arg-max in the order (score descending, block ascending): the exact top-k
// with the lowest index winning ties, as the whole-sequence selection.  Causal
// rows see the blocks that start at or before their position; every row sees
// only blocks holding cached keys.  The picks are written in ascending block
// order, -1 in slots left empty.
//
// Fine stage (block_size 32/64/128, head_dim 64/128; other shapes use the
// general CUDA-core kernel): a CTA per new row, split over the selected
// blocks.  Warp w takes slots w, w + 8, ...: lane l scores keys l, l + 32, ...
// of the block (all K-row loads issued up front), exponentiates against the
// block maximum, then accumulates P V for its own output columns with one
// coalesced V-row load per key, all independent; the warp keeps a running
// (m, l, O) over its blocks and the CTA merges the eight warps' states.
#include "common.cuh"
#include "launchers.cuh"
#include "rowops.cuh"

namespace bsa {

// POOLED: the rows are per-query-block means (fp32, one per block).
template <bool POOLED>
__global__ void __launch_bounds__(kDecSelThreads)
decode_select_kernel(const void* __restrict__ Qv, const float* __restrict__ K_repr,
                     int32_t* __restrict__ idx, Shape s) {
  extern __shared__ __align__(16) float dsm[];
  const int64_t gr = blockIdx.x;         // unit * Nq + row
  select_row<POOLED, true>(Qv, K_repr, idx + gr * s.k, s, gr, dsm);
}

template <bool POOLED>
static cudaError_t launch_select_rows(const void* Q, const float* K_repr, int32_t* idx,
                                      const Shape& s, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)s.D + s.nb) + sizeof(int32_t) * s.k;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(decode_select_kernel<POOLED>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int64_t rows = (int64_t)s.units * s.Nq;
  if (rows == 0) return cudaSuccess;
  decode_select_kernel<POOLED><<<(unsigned)rows, kDecSelThreads, smem, st>>>(Q, K_repr, idx, s);
  return cudaGetLastError();
}

cudaError_t launch_decode_select(const __nv_bfloat16* Q, const float* K_repr, int32_t* idx,
                                 const Shape& s, cudaStream_t st) {
  return launch_select_rows<false>(Q, K_repr, idx, s, st);
}

// Per-query-block selection: block i of every unit (its pooled row Q_repr)
// picks the top-k key blocks j <= i (causal) or of all blocks; then every
// query row of block i gets block i's picks.
__global__ void __launch_bounds__(256)
expand_block_selection_kernel(const int32_t* __restrict__ bidx, int32_t* __restrict__ idx,
                              Shape s) {
  const int64_t total = (int64_t)s.units * s.N * s.k;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / s.k;          // unit * N + r
    const int slot = (int)(e % s.k);
    const int64_t unit = row / s.N;
    const int blk = (int)(row % s.N) / s.bs;
    idx[e] = bidx[(unit * s.nb + blk) * s.k + slot];
  }
}

cudaError_t launch_qblock_select(const float* Q_repr, const float* K_repr, int32_t* bidx,
                                 int32_t* idx, const Shape& s, cudaStream_t st) {
  Shape sb = s;
  sb.Nq = s.nb;     // one pooled row per query block
  sb.q0 = 0;
  sb.kv = s.N;
  cudaError_t e = launch_select_rows<true>(Q_repr, K_repr, bidx, sb, st);
  if (e != cudaSuccess) return e;
  const int64_t total = (int64_t)s.units * s.N * s.k;
  const int64_t blocks = (total + 255) / 256;
  expand_block_selection_kernel<<<(unsigned)(blocks < 148 * 64 ? blocks : 148 * 64), 256, 0, st>>>(
      bidx, idx, s);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
template <int BS, int D>
__global__ void __launch_bounds__(kDecFineWarps * 32)
decode_fine_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                   const __nv_bfloat16* __restrict__ V, const int32_t* __restrict__ idx,
                   __nv_bfloat16* __restrict__ O, Shape s) {
  const int64_t gr = blockIdx.x;
  const int64_t unit = gr / s.Nq;
  const int pos = s.q0 + (int)(gr % s.Nq);
  fine_row<BS, D, true>(Q + gr * D, K, V, idx + gr * s.k, O + gr * D, s, unit, pos);
}

// One decode step in one launch, a CTA per unit: the new token's K and V rows
// go into the cache at position s.q0, warp 0 re-pools the block they land in,
// then the CTA selects the new row's blocks (into shared memory) and attends.
// Every load of cache or block-mean data is an L2 load (NC = false): the CTA
// itself wrote part of it a moment before.  Same arithmetic as
// bsa_pool_k_blocks followed by bsa_decode.
template <int BS, int D>
__global__ void __launch_bounds__(kDecSelThreads)
decode_step_kernel(const __nv_bfloat16* __restrict__ q_new, const __nv_bfloat16* __restrict__ k_new,
                   const __nv_bfloat16* __restrict__ v_new, __nv_bfloat16* __restrict__ K,
                   __nv_bfloat16* __restrict__ V, float* __restrict__ K_repr,
                   __nv_bfloat16* __restrict__ O, Shape s, int lanes_per_row) {
  static_assert(kDecSelThreads == kDecFineWarps * 32, "one CTA shape for all phases");
  extern __shared__ __align__(16) float dsm[];   // selection: D + nb floats, 2 top_k ints
  const int tid = threadIdx.x;
  const int64_t unit = blockIdx.x;
  const int pos = s.q0;
  const int64_t row = (unit * s.N + pos) * (int64_t)D;
  for (int d = tid; d < D; d += kDecSelThreads) {
    K[row + d] = k_new[unit * D + d];
    V[row + d] = v_new[unit * D + d];
  }
  __syncthreads();
  if (tid < 32) pool_block_warp<false>(K, K_repr, nullptr, nullptr, s, lanes_per_row, unit,
                                       pos / BS, tid);
  __syncthreads();
  int32_t* sel = reinterpret_cast<int32_t*>(dsm + D + s.nb) + s.k;   // after the picks
  select_row<false, false>(q_new, K_repr, sel, s, unit, dsm);
  fine_row<BS, D, false>(q_new + unit * D, K, V, sel, O + unit * D, s, unit, pos);
}

bool decode_fine_supported(const Shape& s) {
  return (s.bs == 32 || s.bs == 64 || s.bs == 128) && (s.D == 64 || s.D == 128);
}

cudaError_t launch_decode_step(const __nv_bfloat16* q_new, const __nv_bfloat16* k_new,
                               const __nv_bfloat16* v_new, __nv_bfloat16* K, __nv_bfloat16* V,
                               float* K_repr, __nv_bfloat16* O, const Shape& s,
                               cudaStream_t st) {
  if (s.units == 0) return cudaSuccess;
  int lpr = 1;
  while (lpr < (s.D >> 3)) lpr <<= 1;
  const size_t smem = sizeof(float) * ((size_t)s.D + s.nb) + 2 * sizeof(int32_t) * s.k;
#define BSA_DECODE_STEP(BS_, D_)                                                         \
  if (s.bs == BS_ && s.D == D_) {                                                        \
    if (smem > 48 * 1024) {                                                              \
      cudaError_t e = cudaFuncSetAttribute(decode_step_kernel<BS_, D_>,                  \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                           (int)smem);                                   \
      if (e != cudaSuccess) return e;                                                    \
    }                                                                                    \
    decode_step_kernel<BS_, D_><<<(unsigned)s.units, kDecSelThreads, smem, st>>>(        \
        q_new, k_new, v_new, K, V, K_repr, O, s, lpr);                                   \
    return cudaGetLastError();                                                           \
  }
  BSA_DECODE_STEP(32, 64)
  BSA_DECODE_STEP(64, 64)
  BSA_DECODE_STEP(128, 64)
  BSA_DECODE_STEP(32, 128)
  BSA_DECODE_STEP(64, 128)
  BSA_DECODE_STEP(128, 128)
#undef BSA_DECODE_STEP
  return cudaErrorNotSupported;
}

cudaError_t launch_decode_fine(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, const int32_t* idx, __nv_bfloat16* O,
                               const Shape& s, cudaStream_t st) {
  const int64_t rows = (int64_t)s.units * s.Nq;
  if (rows == 0) return cudaSuccess;
  const dim3 grid((unsigned)rows), block(kDecFineWarps * 32);
#define BSA_DECODE_FINE(BS_, D_)                                                         \
  if (s.bs == BS_ && s.D == D_) {                                                        \
    decode_fine_kernel<BS_, D_><<<grid, block, 0, st>>>(Q, K, V, idx, O, s);             \
    return cudaGetLastError();                                                           \
  }
  BSA_DECODE_FINE(32, 64)
  BSA_DECODE_FINE(64, 64)
  BSA_DECODE_FINE(128, 64)
  BSA_DECODE_FINE(32, 128)
  BSA_DECODE_FINE(64, 128)
  BSA_DECODE_FINE(128, 128)
#undef BSA_DECODE_FINE
  return cudaErrorNotSupported;
}

}  // namespace bsa
