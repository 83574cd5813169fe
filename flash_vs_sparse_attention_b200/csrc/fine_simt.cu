// Stage 4 on CUDA cores, query-stationary (one warp per query row).
// (block_indexer.py:55-84; the reference's Triton kernel
//  _fine_attn_fwd, block_indexer_triton.py:12-83, does the same per program.)
//
// General-shape path (any block_size, head_dim a multiple of 8 up to 256).
// Lanes take 32 keys of a selected block at a time: lane l scores key l with a
// 16-byte-vector dot product, the warp folds the 32 scores into an online
// softmax (running max / sum, FA2 rescaling), and every lane accumulates
// D/32 output dims from the block's V rows (coalesced across lanes).  Output
// is acc / l rounded to bf16 (round-to-nearest-even).  Query row r of a unit
// sits at position s.q0 + r and sees keys below s.kv (the full forward: row
// r at position r, all N keys; decode: new rows against a cache prefix).
#include "common.cuh"

namespace bsa {

template <int DPL>  // output dims per lane: D <= 32 * DPL
__global__ void __launch_bounds__(256)
fine_simt_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                 const __nv_bfloat16* __restrict__ V, const int32_t* __restrict__ idx,
                 __nv_bfloat16* __restrict__ O, Shape s) {
  __shared__ float qs[8][256];
  const int wib = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * 8 + wib;
  if (gw >= (int64_t)s.units * s.Nq) return;
  const int64_t unit = gw / s.Nq;
  const int row = s.q0 + (int)(gw % s.Nq);   // the query's position
  const __nv_bfloat16* q = Q + gw * s.D;
  for (int d = lane; d < s.D; d += 32) qs[wib][d] = __bfloat162float(q[d]);
  __syncwarp();

  const float c = s.scale * kLog2e;  // scores in the base-2 domain
  float m = -INFINITY, l = 0.f;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;

  const int32_t* sel = idx + gw * s.k;
  const __nv_bfloat16* Ku = K + unit * s.N * (int64_t)s.D;
  const __nv_bfloat16* Vu = V + unit * s.N * (int64_t)s.D;
  const int vecs = s.D >> 3;

  for (int slot = 0; slot < s.k; ++slot) {
    const int j = sel[slot];
    if (j < 0) continue;
    for (int kc = 0; kc < s.bs; kc += 32) {
      const int64_t key0 = (int64_t)j * s.bs + kc;
      if ((s.causal && key0 > row) || key0 >= s.kv) break;  // every later key is masked too
      const int key = (int)key0 + lane;
      const bool valid = (kc + lane < s.bs) && key < s.kv && (!s.causal || key <= row);
      float sc = -INFINITY;
      if (valid) {
        const uint4* kr = reinterpret_cast<const uint4*>(Ku + (int64_t)key * s.D);
        float a = 0.f;
        for (int v = 0; v < vecs; ++v) {
          uint4 w = __ldg(kr + v);
          const float* qq = &qs[wib][v * 8];
          a = fmaf(qq[0], bf16_lo(w.x), a); a = fmaf(qq[1], bf16_hi(w.x), a);
          a = fmaf(qq[2], bf16_lo(w.y), a); a = fmaf(qq[3], bf16_hi(w.y), a);
          a = fmaf(qq[4], bf16_lo(w.z), a); a = fmaf(qq[5], bf16_hi(w.z), a);
          a = fmaf(qq[6], bf16_lo(w.w), a); a = fmaf(qq[7], bf16_hi(w.w), a);
        }
        sc = a * c;
      }
      const float cm = warp_max(sc);
      const float m_new = fmaxf(m, cm);
      const float corr = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
      const float p = valid ? fast_exp2(sc - m_new) : 0.f;
      l = l * corr + warp_sum(p);
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] *= corr;
      const int nk = (int)min((int64_t)min(32, s.bs - kc), (int64_t)s.kv - key0);
      for (int tk = 0; tk < nk; ++tk) {
        const float pt = __shfl_sync(0xffffffffu, p, tk);
        if (pt != 0.f) {
          const __nv_bfloat16* vr = Vu + (key0 + tk) * s.D;
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            if (d < s.D) acc[i] = fmaf(pt, __bfloat162float(vr[d]), acc[i]);
          }
        }
      }
      m = m_new;
    }
  }
  const float inv = 1.f / l;
  __nv_bfloat16* o = O + gw * s.D;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int d = lane + 32 * i;
    if (d < s.D) o[d] = __float2bfloat16_rn(acc[i] * inv);
  }
}

cudaError_t launch_fine_simt(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, const int32_t* idx, __nv_bfloat16* O,
                             const Shape& s, cudaStream_t st) {
  const int64_t warps = (int64_t)s.units * s.Nq;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  if (s.D <= 32) fine_simt_kernel<1><<<blocks, 256, 0, st>>>(Q, K, V, idx, O, s);
  else if (s.D <= 64) fine_simt_kernel<2><<<blocks, 256, 0, st>>>(Q, K, V, idx, O, s);
  else if (s.D <= 128) fine_simt_kernel<4><<<blocks, 256, 0, st>>>(Q, K, V, idx, O, s);
  else fine_simt_kernel<8><<<blocks, 256, 0, st>>>(Q, K, V, idx, O, s);
  return cudaGetLastError();
}

}  // namespace bsa
