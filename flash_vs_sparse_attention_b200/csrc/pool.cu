// Stage 1: per-block mean of K (block_indexer_triton.py:120; block_indexer.py:33).
//
// One warp per (unit, block).  The warp reads the block's bs x D bf16 keys as
// 16-byte vectors (8 bf16 per lane, a full 128-byte line per 8 lanes when
// D = 64), so a block of 64 keys is 16 fully coalesced vector loads per lane.
// Sums are fp32; the mean is sum / bs as torch's mean computes it.  For a
// growing KV cache the kernel pools a range of blocks over the keys present
// (s.kv of them): a block that is only partly filled is the mean of its
// present keys, a full block exactly what the whole-sequence pass gives.  Besides
// the fp32 means the kernel writes the split of mean * scale into two bf16
// terms (hi = bf16(m), lo = bf16(m - hi)) for the tensor-core scorer, whose
// bf16 MMAs then reproduce the scaled fp32 coarse scores to ~2^-17 relative.
//
// HBM-bound: reads N*D*2 bytes per unit, writes nb*D*(4+2+2).
#include "common.cuh"
#include "rowops.cuh"

namespace bsa {

__global__ void __launch_bounds__(256)
pool_k_kernel(const __nv_bfloat16* __restrict__ K, float* __restrict__ K_repr,
              __nv_bfloat16* __restrict__ K_hi, __nv_bfloat16* __restrict__ K_lo,
              Shape s, int lanes_per_row, int block_begin, int n_blocks,
              uint4* __restrict__ zero, int64_t zero_words) {
  {
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < zero_words; i += nthreads)
      zero[i] = make_uint4(0, 0, 0, 0);
  }
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)s.units * n_blocks;
  if (warp >= total) return;
  const int64_t unit = warp / n_blocks;
  const int64_t blk = block_begin + warp % n_blocks;
  pool_block_warp<true>(K, K_repr, K_hi, K_lo, s, lanes_per_row, unit, blk, lane);
}

cudaError_t launch_pool_k(const __nv_bfloat16* K, float* K_repr, __nv_bfloat16* K_hi,
                          __nv_bfloat16* K_lo, const Shape& s, cudaStream_t st, void* zero,
                          size_t zero_bytes, int block_begin, int block_end) {
  int chunks = s.D >> 3;
  int lpr = 1;
  while (lpr < chunks) lpr <<= 1;
  const int end = block_end < 0 ? s.nb : block_end;
  const int n_blocks = end - block_begin;
  if (n_blocks <= 0) return cudaSuccess;   // (the whole-sequence pass always has blocks)
  const int64_t warps = (int64_t)s.units * n_blocks;
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  pool_k_kernel<<<(unsigned)blocks, threads, 0, st>>>(K, K_repr, K_hi, K_lo, s, lpr, block_begin,
                                                       n_blocks, (uint4*)zero,
                                                       (int64_t)(zero_bytes / 16));
  return cudaGetLastError();
}

}  // namespace bsa
