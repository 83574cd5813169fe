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

namespace bsa {

constexpr int kDecSelThreads = 256;

// POOLED: the rows are per-query-block means (fp32, one per block; row r
// stands for block r and sits at that block's last position).
template <bool POOLED>
__global__ void __launch_bounds__(kDecSelThreads)
decode_select_kernel(const void* __restrict__ Qv, const float* __restrict__ K_repr,
                     int32_t* __restrict__ idx, Shape s) {
  extern __shared__ __align__(16) float dsm[];
  float* qs = dsm;                       // head_dim
  float* sc = dsm + s.D;                 // one score per visible block
  int32_t* picks = reinterpret_cast<int32_t*>(sc + s.nb);   // top_k
  __shared__ int n_picked;
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t gr = blockIdx.x;         // unit * Nq + row
  const int64_t unit = gr / s.Nq;
  const int r = (int)(gr % s.Nq);
  const int pos = POOLED ? (r + 1) * s.bs - 1 : s.q0 + r;
  for (int d = tid; d < s.D; d += kDecSelThreads)
    qs[d] = POOLED ? reinterpret_cast<const float*>(Qv)[gr * s.D + d]
                   : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(Qv)[gr * s.D + d]);
  __syncthreads();
  const int nb_kv = (s.kv + s.bs - 1) / s.bs;
  const int lim = s.causal ? min(nb_kv, pos / s.bs + 1) : nb_kv;   // eligible: [0, lim)
  const float* kr = K_repr + unit * s.nb * (int64_t)s.D;
  const int d4n = s.D >> 2;
  for (int j = tid; j < lim; j += kDecSelThreads) {
    const float4* kj = reinterpret_cast<const float4*>(kr + (int64_t)j * s.D);
    float a = 0.f;
    for (int d0 = 0; d0 < d4n; d0 += 16) {   // 16 row loads in flight, then their FMAs
      float4 k4[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) k4[u] = d0 + u < d4n ? __ldg(kj + d0 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        if (d0 + u < d4n) {
          const float* qd = qs + 4 * (d0 + u);
          a = fmaf(qd[0], k4[u].x, a);
          a = fmaf(qd[1], k4[u].y, a);
          a = fmaf(qd[2], k4[u].z, a);
          a = fmaf(qd[3], k4[u].w, a);
        }
      }
    }
    sc[j] = a * s.scale;
  }
  __syncthreads();
  if (tid < 32) {
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
      if (bv == -INFINITY) break;        // no eligible block left (same on every lane)
      if (lane == 0) picks[n] = bj;
      if ((bj & 31) == lane) sc[bj] = -INFINITY;   // the owning lane retires the pick
      __syncwarp();
    }
    if (lane == 0) n_picked = n;
  }
  __syncthreads();
  // Ascending block order: pick t goes to slot (number of smaller picks).
  const int n = n_picked;
  int32_t* out = idx + gr * s.k;
  for (int t = tid; t < s.k; t += kDecSelThreads) {
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
constexpr int kDecFineWarps = 8;

template <int BS, int D>
__global__ void __launch_bounds__(kDecFineWarps * 32)
decode_fine_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                   const __nv_bfloat16* __restrict__ V, const int32_t* __restrict__ idx,
                   __nv_bfloat16* __restrict__ O, Shape s) {
  constexpr int KPL = BS / 32;           // keys per lane
  constexpr int DV = D / 8;              // 16-byte chunks per key row
  constexpr int CPL = D / 32;            // output columns per lane (2 or 4)
  __shared__ float qs[D];
  __shared__ float wm[kDecFineWarps], wl[kDecFineWarps];
  __shared__ float wo[kDecFineWarps][D];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t gr = blockIdx.x;
  const int64_t unit = gr / s.Nq;
  const int pos = s.q0 + (int)(gr % s.Nq);
  for (int d = tid; d < D; d += kDecFineWarps * 32) qs[d] = __bfloat162float(Q[gr * D + d]);
  __syncthreads();
  const float c = s.scale * kLog2e;      // scores in the base-2 domain
  const __nv_bfloat16* Ku = K + unit * s.N * (int64_t)D;
  const __nv_bfloat16* Vu = V + unit * s.N * (int64_t)D;
  const int32_t* sel = idx + gr * s.k;
  float m = -INFINITY, l = 0.f, acc[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) acc[i] = 0.f;
  for (int slot = warp; slot < s.k; slot += kDecFineWarps) {
    const int j = sel[slot];
    if (j < 0) continue;
    const int64_t key0 = (int64_t)j * BS;
    // Scores of this lane's keys (every K-row load issued first).
    uint4 kr[KPL][DV];
#pragma unroll
    for (int t = 0; t < KPL; ++t) {
      const uint4* row = reinterpret_cast<const uint4*>(Ku + (key0 + lane + 32 * t) * D);
#pragma unroll
      for (int v = 0; v < DV; ++v) kr[t][v] = __ldg(row + v);
    }
    float sv[KPL];
    float bm = -INFINITY;
#pragma unroll
    for (int t = 0; t < KPL; ++t) {
      const int64_t key = key0 + lane + 32 * t;
      float a = 0.f;
#pragma unroll
      for (int v = 0; v < DV; ++v) {
        const float* qq = qs + 8 * v;
        a = fmaf(qq[0], bf16_lo(kr[t][v].x), a); a = fmaf(qq[1], bf16_hi(kr[t][v].x), a);
        a = fmaf(qq[2], bf16_lo(kr[t][v].y), a); a = fmaf(qq[3], bf16_hi(kr[t][v].y), a);
        a = fmaf(qq[4], bf16_lo(kr[t][v].z), a); a = fmaf(qq[5], bf16_hi(kr[t][v].z), a);
        a = fmaf(qq[6], bf16_lo(kr[t][v].w), a); a = fmaf(qq[7], bf16_hi(kr[t][v].w), a);
      }
      const bool valid = key < s.kv && (!s.causal || key <= pos);
      sv[t] = valid ? a * c : -INFINITY;
      bm = fmaxf(bm, sv[t]);
    }
    bm = warp_max(bm);
    if (bm == -INFINITY) continue;       // every key of the block masked (same on all lanes)
    float pl[KPL], ps = 0.f;
#pragma unroll
    for (int t = 0; t < KPL; ++t) {
      pl[t] = fast_exp2(sv[t] - bm);     // 0 for masked keys
      ps += pl[t];
    }
    ps = warp_sum(ps);
    // P V for this lane's columns [CPL * lane, CPL * lane + CPL): one load of
    // CPL bf16 per key, all independent.
    float ob[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) ob[i] = 0.f;
#pragma unroll
    for (int t = 0; t < KPL; ++t) {
#pragma unroll 8
      for (int kk = 0; kk < 32; ++kk) {
        const float p = __shfl_sync(0xffffffffu, pl[t], kk);
        const __nv_bfloat16* vr = Vu + (key0 + 32 * t + kk) * D + CPL * lane;
        if constexpr (CPL == 2) {
          const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(vr));
          ob[0] = fmaf(p, bf16_lo(w), ob[0]);
          ob[1] = fmaf(p, bf16_hi(w), ob[1]);
        } else {
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(vr));
          ob[0] = fmaf(p, bf16_lo(w.x), ob[0]);
          ob[1] = fmaf(p, bf16_hi(w.x), ob[1]);
          ob[2] = fmaf(p, bf16_lo(w.y), ob[2]);
          ob[3] = fmaf(p, bf16_hi(w.y), ob[3]);
        }
      }
    }
    // Fold the block into the warp's running state.
    const float mn = fmaxf(m, bm);
    const float ca = (m == -INFINITY) ? 0.f : fast_exp2(m - mn);
    const float cb = fast_exp2(bm - mn);
    l = l * ca + ps * cb;
#pragma unroll
    for (int i = 0; i < CPL; ++i) acc[i] = acc[i] * ca + ob[i] * cb;
    m = mn;
  }
  if (lane == 0) { wm[warp] = m; wl[warp] = l; }
#pragma unroll
  for (int i = 0; i < CPL; ++i) wo[warp][CPL * lane + i] = acc[i];
  __syncthreads();
  // Merge the warps' states: one thread per output column.
  for (int d = tid; d < D; d += kDecFineWarps * 32) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecFineWarps; ++w) M = fmaxf(M, wm[w]);
    float Lsum = 0.f, Osum = 0.f;
#pragma unroll
    for (int w = 0; w < kDecFineWarps; ++w) {
      const float f = wm[w] == -INFINITY ? 0.f : fast_exp2(wm[w] - M);
      Lsum = fmaf(wl[w], f, Lsum);
      Osum = fmaf(wo[w][d], f, Osum);
    }
    O[gr * D + d] = __float2bfloat16_rn(Osum / Lsum);
  }
}

bool decode_fine_supported(const Shape& s) {
  return (s.bs == 32 || s.bs == 64 || s.bs == 128) && (s.D == 64 || s.D == 128);
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
