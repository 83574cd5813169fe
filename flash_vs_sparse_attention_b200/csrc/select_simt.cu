// Stages 2-3 on CUDA cores: coarse scores in fp32 FMA + per-row top-k.
// (block_indexer_triton.py:121-129; block_indexer.py:44-53)
//
// General-shape path: any head_dim that is a multiple of 8 (<= 256), any
// block_size, top_k <= 64.  One thread per query row, 64 rows per CTA.  The
// CTA's query rows are staged transposed in shared memory (qT[d][row], so a
// warp's reads are conflict-free) and block representatives stream through
// shared memory in tiles of 16; scores are sequential fp32 dot products like
// the reference's fp32 GEMM.  Causal rows only visit blocks that start at or
// before the CTA's last row.
#include "common.cuh"
#include "topk_select.cuh"

namespace bsa {

constexpr int kSimtRows = 64;
constexpr int kSimtTile = 16;

template <int KCAP>
__global__ void __launch_bounds__(kSimtRows)
select_simt_kernel(const __nv_bfloat16* __restrict__ Q, const float* __restrict__ K_repr,
                   int32_t* __restrict__ idx, Shape s) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int t = threadIdx.x;
  const int unit = blockIdx.y;
  const int row0 = blockIdx.x * kSimtRows;
  const int row = row0 + t;
  const int cap = topk_buffer_slots(KCAP);

  float* qT = reinterpret_cast<float*>(smem);                       // D x 64
  float* kt = qT + s.D * kSimtRows;                                 // 16 x D
  uint2* bbuf = reinterpret_cast<uint2*>(kt + kSimtTile * s.D);     // cap x 64

  // Stage Q rows (transposed).  Rows past N read as zero.
  const __nv_bfloat16* qbase = Q + ((int64_t)unit * s.N + row0) * s.D;
  for (int e = t; e < kSimtRows * s.D; e += kSimtRows) {
    int r = e / s.D, d = e % s.D;
    float v = (row0 + r < s.N) ? __bfloat162float(qbase[(int64_t)r * s.D + d]) : 0.f;
    qT[d * kSimtRows + r] = v;
  }

  RowTopK<KCAP> sel;
  sel.init(bbuf + t, kSimtRows, cap, unit_top_k(s, unit));   // this head's budget

  int last_row = min(row0 + kSimtRows, s.N) - 1;
  int nb_visit = s.causal ? min(s.nb, last_row / s.bs + 1) : s.nb;
  const float* kr = K_repr + (int64_t)unit * s.nb * s.D;

  for (int j0 = 0; j0 < nb_visit; j0 += kSimtTile) {
    __syncthreads();
    int tile = min(kSimtTile, nb_visit - j0);
    for (int e = t; e < tile * s.D; e += kSimtRows) kt[e] = kr[(int64_t)j0 * s.D + e];
    __syncthreads();
    sel.reserve(kSimtTile);
    for (int jj = 0; jj < tile; jj += 4) {
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      const float* k0 = kt + jj * s.D;
      for (int d = 0; d < s.D; ++d) {
        float q = qT[d * kSimtRows + t];
        a0 = fmaf(q, k0[d], a0);
        if (jj + 1 < tile) a1 = fmaf(q, k0[s.D + d], a1);
        if (jj + 2 < tile) a2 = fmaf(q, k0[2 * s.D + d], a2);
        if (jj + 3 < tile) a3 = fmaf(q, k0[3 * s.D + d], a3);
      }
      float sc[4] = {a0 * s.scale, a1 * s.scale, a2 * s.scale, a3 * s.scale};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int j = j0 + jj + u;
        if (jj + u < tile && row < s.N) {
          bool masked = s.causal && (int64_t)j * s.bs > row;
          sel.push(masked ? -INFINITY : sc[u], j);
        }
      }
    }
  }
  if (row < s.N) sel.emit(idx + ((int64_t)unit * s.N + row) * s.k, s.k);
}

static size_t select_simt_smem(const Shape& s, int kcap) {
  return sizeof(float) * ((size_t)s.D * kSimtRows + (size_t)kSimtTile * s.D) +
         sizeof(uint2) * (size_t)topk_buffer_slots(kcap) * kSimtRows;
}

template <int KCAP>
static cudaError_t launch_simt(const __nv_bfloat16* Q, const float* K_repr, int32_t* idx,
                               const Shape& s, cudaStream_t st) {
  size_t smem = select_simt_smem(s, KCAP);
  cudaError_t e = cudaFuncSetAttribute(select_simt_kernel<KCAP>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((s.N + kSimtRows - 1) / kSimtRows, s.units);
  select_simt_kernel<KCAP><<<grid, kSimtRows, smem, st>>>(Q, K_repr, idx, s);
  return cudaGetLastError();
}

cudaError_t launch_select_simt(const __nv_bfloat16* Q, const float* K_repr, int32_t* idx,
                               const Shape& s, cudaStream_t st) {
  if (s.k <= 16) return launch_simt<16>(Q, K_repr, idx, s, st);
  if (s.k <= 32) return launch_simt<32>(Q, K_repr, idx, s, st);
  return launch_simt<64>(Q, K_repr, idx, s, st);
}

}  // namespace bsa
