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
  const int chunks = s.D >> 3;                 // 16-byte chunks per key row
  const int rows_per_iter = 32 / lanes_per_row;
  const int g = lane / lanes_per_row;          // row group
  const int c = lane % lanes_per_row;          // chunk within the row
  const bool active = c < chunks;

  const int64_t unit = warp / n_blocks;
  const int64_t blk = block_begin + warp % n_blocks;
  const uint4* src = reinterpret_cast<const uint4*>(K + (unit * s.N + blk * s.bs) * (int64_t)s.D);
  // Keys of this block that exist (all bs of them outside a growing cache).
  const int rows = (int)min((int64_t)s.bs, (int64_t)s.kv - blk * s.bs);

  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;

  if (active) {
    // Batches of 16 loads issued before any is summed (a whole 64-key block
    // per batch at head_dim 64): one memory round trip per batch.
    for (int r0 = g; r0 < rows; r0 += 16 * rows_per_iter) {
      uint4 v[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int r = r0 + q * rows_per_iter;
        v[q] = r < rows ? __ldg(src + (int64_t)r * chunks + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        acc[0] += bf16_lo(v[q].x); acc[1] += bf16_hi(v[q].x);
        acc[2] += bf16_lo(v[q].y); acc[3] += bf16_hi(v[q].y);
        acc[4] += bf16_lo(v[q].z); acc[5] += bf16_hi(v[q].z);
        acc[6] += bf16_lo(v[q].w); acc[7] += bf16_hi(v[q].w);
      }
    }
  }
  // Reduce over row groups (lanes that differ in the row-group bits).
  for (int o = lanes_per_row; o < 32; o <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (g == 0 && active) {
    const float den = (float)rows;
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = acc[i] / den;
    const int64_t off = (unit * s.nb + blk) * (int64_t)s.D + c * 8;
    float4* dst = reinterpret_cast<float4*>(K_repr + off);
    dst[0] = make_float4(m[0], m[1], m[2], m[3]);
    dst[1] = make_float4(m[4], m[5], m[6], m[7]);
    if (K_hi != nullptr) {
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a0 = m[2 * i] * s.scale, a1 = m[2 * i + 1] * s.scale;
        __nv_bfloat16 h0 = __float2bfloat16_rn(a0);
        __nv_bfloat16 h1 = __float2bfloat16_rn(a1);
        float r0 = a0 - __bfloat162float(h0);
        float r1 = a1 - __bfloat162float(h1);
        hi[i] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        lo[i] = pack_bf16x2(r0, r1);
      }
      *reinterpret_cast<uint4*>(K_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(K_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
  }
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
