// Decode-time selection: stages 2-3 for a few new query rows against the
// cached block means of a KV cache (block_indexer.py:44-53 evaluated at the
// new rows' positions; the reference itself has no decode path).
//
// One warp per (unit, new row).  Lane l scores blocks l, l + 32, ... in fp32,
// each a sequential dot product over head_dim exactly as the CUDA-core
// scorer computes it (so a decode row selects what the whole-sequence
// CUDA-core pass selects for that row).  The scores sit in shared memory;
// top_k rounds of a warp arg-max in the order (score descending, block
// ascending) pick the exact top-k with the lowest index winning ties.  Causal
// rows see the blocks that start at or before their position; every row sees
// only blocks holding cached keys.  The picks are written in ascending block
// order, -1 in slots left empty.
#include "common.cuh"
#include "launchers.cuh"

namespace bsa {

__global__ void __launch_bounds__(32)
decode_select_kernel(const __nv_bfloat16* __restrict__ Q, const float* __restrict__ K_repr,
                     int32_t* __restrict__ idx, Shape s) {
  extern __shared__ __align__(16) float dsm[];
  float* qs = dsm;                       // head_dim
  float* sc = dsm + s.D;                 // one score per visible block
  int32_t* picks = reinterpret_cast<int32_t*>(sc + s.nb);   // top_k
  const int lane = threadIdx.x;
  const int64_t gr = blockIdx.x;         // unit * Nq + row
  const int64_t unit = gr / s.Nq;
  const int pos = s.q0 + (int)(gr % s.Nq);
  for (int d = lane; d < s.D; d += 32) qs[d] = __bfloat162float(Q[gr * s.D + d]);
  __syncwarp();
  const int nb_kv = (s.kv + s.bs - 1) / s.bs;
  const int lim = s.causal ? min(nb_kv, pos / s.bs + 1) : nb_kv;   // eligible: [0, lim)
  const float* kr = K_repr + unit * s.nb * (int64_t)s.D;
  for (int j = lane; j < lim; j += 32) {
    const float4* kj = reinterpret_cast<const float4*>(kr + (int64_t)j * s.D);
    float a = 0.f;
    for (int d4 = 0; d4 < (s.D >> 2); ++d4) {
      const float4 k4 = __ldg(kj + d4);
      a = fmaf(qs[4 * d4], k4.x, a);
      a = fmaf(qs[4 * d4 + 1], k4.y, a);
      a = fmaf(qs[4 * d4 + 2], k4.z, a);
      a = fmaf(qs[4 * d4 + 3], k4.w, a);
    }
    sc[j] = a * s.scale;
  }
  __syncwarp();
  int n = 0;
  for (; n < s.k; ++n) {
    // Lane-local best: blocks ascend within a lane, so a strict > keeps the
    // lowest block among equal scores.
    float bv = -INFINITY;
    int bj = 0x7fffffff;
    for (int j = lane; j < lim; j += 32) {
      const float v = sc[j];
      if (v > bv) { bv = v; bj = j; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
      if (ov > bv || (ov == bv && oj < bj)) { bv = ov; bj = oj; }
    }
    if (bv == -INFINITY) break;          // no eligible block left (same on every lane)
    if (lane == 0) picks[n] = bj;
    if ((bj & 31) == lane) sc[bj] = -INFINITY;   // the owning lane retires the pick
    __syncwarp();
  }
  __syncwarp();
  // Ascending block order: pick t goes to slot (number of smaller picks).
  int32_t* out = idx + gr * s.k;
  for (int t = lane; t < s.k; t += 32) {
    if (t < n) {
      const int v = picks[t];
      int rank = 0;
      for (int u = 0; u < n; ++u) rank += picks[u] < v ? 1 : 0;
      out[rank] = v;
    } else {
      out[t] = -1;
    }
  }
}

cudaError_t launch_decode_select(const __nv_bfloat16* Q, const float* K_repr, int32_t* idx,
                                 const Shape& s, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)s.D + s.nb) + sizeof(int32_t) * s.k;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(decode_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int64_t rows = (int64_t)s.units * s.Nq;
  if (rows == 0) return cudaSuccess;
  decode_select_kernel<<<(unsigned)rows, 32, smem, st>>>(Q, K_repr, idx, s);
  return cudaGetLastError();
}

}  // namespace bsa
