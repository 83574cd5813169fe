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
// general CUDA-core kernel): a cluster of kDecCluster CTAs per new row, CTA r
// attending the selected blocks in part r of the row's eligible range
// (cluster_part).  A CTA cuts its blocks into 32-key chunks over its warps; a
// warp loads a chunk's K rows and V rows together, scores, exponentiates
// against the chunk maximum and accumulates P V, keeping a running (m, l, O);
// each CTA merges its warps and sends its state to CTA 0 through distributed
// shared memory, which merges the CTAs in rank order (fine_row_cluster).  The
// one-launch decode step selects on the same cluster (cluster_pick: each CTA
// ranks its part, the parts' candidates are exchanged, and each CTA keeps the
// global picks that fall in its part), so both paths attend the same blocks
// with the same arithmetic.
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

// Per-query-block selection, kQbRows pooled rows per CTA: every block-mean
// row is loaded once and scored against all of the CTA's rows (the same
// sequential fp32 dot products as select_row, so the same picks); then warp
// r runs row r's top_k rounds of a warp arg-max (score descending, block
// ascending) over its eligible blocks, as select_row does, and writes the
// picks in ascending block order, -1 padded.  Dynamic shared memory:
// rows * (D + nb) floats.
constexpr int kQbRows = 8;

__global__ void __launch_bounds__(kQbRows * 32)
qblock_select_kernel(const float* __restrict__ Q_repr, const float* __restrict__ K_repr,
                     int32_t* __restrict__ bidx, Shape s, int rows_per_cta) {
  extern __shared__ __align__(16) float qsm[];
  __shared__ int32_t picks[kQbRows][64];
  const int R = rows_per_cta;
  const int cpu = (s.nb + R - 1) / R;            // CTAs per unit
  const int64_t unit = blockIdx.x / cpu;
  const int i0 = (int)(blockIdx.x % cpu) * R;    // this CTA's first query block
  const int nr = min(R, s.nb - i0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* qs = qsm;                               // R x D pooled rows
  float* sc = qsm + (size_t)R * s.D;             // R x nb scores
  for (int e = tid; e < nr * s.D; e += kQbRows * 32)
    qs[e] = __ldg(Q_repr + (unit * s.nb + i0) * (int64_t)s.D + e);
  __syncthreads();
  const int lim_max = s.causal ? min(s.nb, i0 + nr) : s.nb;
  const float* kr = K_repr + unit * s.nb * (int64_t)s.D;
  const int d4n = s.D >> 2;
  for (int j = tid; j < lim_max; j += kQbRows * 32) {
    const float4* kj = reinterpret_cast<const float4*>(kr + (int64_t)j * s.D);
    float a[kQbRows];
#pragma unroll
    for (int r = 0; r < kQbRows; ++r) a[r] = 0.f;
    for (int d0 = 0; d0 < d4n; d0 += 16) {   // 16 row loads in flight, then their FMAs
      float4 k4[16];
#pragma unroll
      for (int u = 0; u < 16; ++u)
        k4[u] = d0 + u < d4n ? __ldg(kj + d0 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        if (d0 + u < d4n) {
#pragma unroll
          for (int r = 0; r < kQbRows; ++r) {
            if (r < nr) {
              const float* qd = qs + r * s.D + 4 * (d0 + u);
              a[r] = fmaf(qd[0], k4[u].x, a[r]);
              a[r] = fmaf(qd[1], k4[u].y, a[r]);
              a[r] = fmaf(qd[2], k4[u].z, a[r]);
              a[r] = fmaf(qd[3], k4[u].w, a[r]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kQbRows; ++r)
      if (r < nr) sc[(size_t)r * s.nb + j] = a[r] * s.scale;
  }
  __syncthreads();
  if (warp >= nr) return;
  const int i = i0 + warp;                       // this warp's query block
  const int lim = s.causal ? i + 1 : s.nb;       // eligible: [0, lim)
  float* row = sc + (size_t)warp * s.nb;
  int n = 0;
  for (; n < s.k; ++n) {
    float bv = -INFINITY;
    int bj = 0x7fffffff;
    for (int j = lane; j < lim; j += 32) {       // blocks ascend within a lane
      const float v = row[j];
      if (v > bv) { bv = v; bj = j; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
      if (ov > bv || (ov == bv && oj < bj)) { bv = ov; bj = oj; }
    }
    if (bv == -INFINITY) break;                  // no eligible block left
    if (lane == 0) picks[warp][n] = bj;
    if ((bj & 31) == lane) row[bj] = -INFINITY;  // the owning lane retires the pick
    __syncwarp();
  }
  int32_t* out = bidx + (unit * s.nb + i) * (int64_t)s.k;
  for (int t = lane; t < s.k; t += 32) {
    if (t < n) {
      const int v = picks[warp][t];
      int rank = 0;
      for (int u = 0; u < n; ++u) rank += picks[warp][u] < v ? 1 : 0;
      out[rank] = v;
    } else {
      out[t] = -1;
    }
  }
}

cudaError_t launch_qblock_select(const float* Q_repr, const float* K_repr, int32_t* bidx,
                                 int32_t* idx, const Shape& s, cudaStream_t st) {
  int R = kQbRows;
  while (R > 1 && sizeof(float) * (size_t)R * (s.D + s.nb) > 200 * 1024) R >>= 1;
  const size_t smem = sizeof(float) * (size_t)R * (s.D + s.nb);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(qblock_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int64_t grid = (int64_t)s.units * ((s.nb + R - 1) / R);
  if (grid > 0) qblock_select_kernel<<<(unsigned)grid, kQbRows * 32, smem, st>>>(Q_repr, K_repr,
                                                                                 bidx, s, R);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t total = (int64_t)s.units * s.N * s.k;
  const int64_t blocks = (total + 255) / 256;
  expand_block_selection_kernel<<<(unsigned)(blocks < 148 * 64 ? blocks : 148 * 64), 256, 0, st>>>(
      bidx, idx, s);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// A cluster of kDecCluster CTAs per new row (fine_row_cluster).
template <int BS, int D>
__global__ void __cluster_dims__(kDecCluster, 1, 1) __launch_bounds__(kDecFineWarps * 32)
decode_fine_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                   const __nv_bfloat16* __restrict__ V, const int32_t* __restrict__ idx,
                   __nv_bfloat16* __restrict__ O, Shape s) {
  __shared__ float qs[D];
  __shared__ int32_t row_idx[64], sel[64];   // top_k <= 64
  __shared__ uint64_t state_bar;             // (CTA 0) the CTAs' partial states
  const int tid = threadIdx.x;
  const int64_t gr = blockIdx.x / kDecCluster;
  const int64_t unit = gr / s.Nq;
  const int pos = s.q0 + (int)(gr % s.Nq);
  if (tid == 0) {
    sm100::mbar_init(&state_bar, 1);
    if (cluster_rank() == 0) sm100::mbar_arrive_expect_tx(&state_bar, fine_state_bytes<D>());
    sm100::fence_barrier_init();
  }
  for (int d = tid; d < D; d += blockDim.x) qs[d] = __bfloat162float(Q[gr * D + d]);
  for (int t = tid; t < s.k; t += blockDim.x) row_idx[t] = idx[gr * s.k + t];
  __syncthreads();
  cluster_arrive();
  // This CTA's part of the row's eligible blocks (as in the one-launch step)
  // and the selected blocks in it, ascending.
  const int nb_kv = (s.kv + BS - 1) / BS;
  const int lim = s.causal ? min(nb_kv, pos / BS + 1) : nb_kv;
  const int part = cluster_part(lim);
  const int j0 = min(lim, (int)cluster_rank() * part), j1 = min(lim, j0 + part);
  int n_sel = 0;
  for (int t0 = 0; t0 < s.k; t0 += blockDim.x) {
    const int t = t0 + tid;
    const int j = t < s.k ? row_idx[t] : -1;
    const bool mine = j >= j0 && j < j1;
    if (mine) {
      int slot = 0;
      for (int u = 0; u < s.k; ++u) slot += (row_idx[u] >= j0 && row_idx[u] < j) ? 1 : 0;
      sel[slot] = j;
    }
    n_sel += __syncthreads_count(mine);
  }
  fine_row_cluster<BS, D, true>(qs, K, V, sel, n_sel, O + gr * D, s, unit, pos, &state_bar,
                                true, false, nullptr, nullptr, -1);
}

// One decode step in one launch, a cluster of kDecCluster CTAs per unit.
// CTA r scores the eligible blocks [r * part, (r + 1) * part) (part =
// cluster_part(eligible blocks)) against the new query row with the
// sequential fp32 dot products of select_row.  The CTA whose part holds the
// new token's block re-pools that block in its warp 0, reading the token's
// key row from k_new (the same values and order as pooling the cache after
// the append), scores it from the fresh mean, and writes the token's K and V
// rows into the cache at position s.q0.  Every other load is issued at the
// start, so the query row, the block means and the pooled block arrive in one
// memory round trip.  Then cluster_pick (the exact top-k over the cluster)
// and fine_row_cluster, which reads the token's own key and value from k_new
// and v_new: no CTA reads what another wrote to global memory, so the CTAs
// meet only through their shared-memory exchanges.  Same picks, block means
// and output bits as bsa_pool_k_blocks followed by bsa_decode.
template <int BS, int D>
__global__ void __cluster_dims__(kDecCluster, 1, 1) __launch_bounds__(kDecSelThreads)
decode_step_kernel(const __nv_bfloat16* __restrict__ q_new, const __nv_bfloat16* __restrict__ k_new,
                   const __nv_bfloat16* __restrict__ v_new, __nv_bfloat16* __restrict__ K,
                   __nv_bfloat16* __restrict__ V, float* __restrict__ K_repr,
                   __nv_bfloat16* __restrict__ O, Shape s, int lanes_per_row) {
  static_assert(kDecSelThreads == kDecFineWarps * 32, "one CTA shape for all phases");
  extern __shared__ __align__(16) float dsm[];   // PickSmem::bytes
  __shared__ uint64_t bars[2];                   // candidates; (CTA 0) partial states
  const int tid = threadIdx.x;
  if (tid == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    if (cluster_rank() == 0) sm100::mbar_arrive_expect_tx(&bars[1], fine_state_bytes<D>());
    sm100::fence_barrier_init();
  }
  cluster_arrive();                              // waited for in cluster_pick
  PickSmem sm;
  sm.carve(dsm, D, s.nb, s.k);
  const int64_t unit = blockIdx.x / kDecCluster;
  const int pos = s.q0;
  const int bp = pos / BS;                       // the new token's block
  const int nb_kv = (s.kv + BS - 1) / BS;
  const int lim = s.causal ? min(nb_kv, bp + 1) : nb_kv;   // eligible: [0, lim)
  const int part = cluster_part(lim);
  const int j0 = min(lim, (int)cluster_rank() * part), n_loc = min(lim, j0 + part) - j0;
  const int own = (bp >= j0 && bp < j0 + n_loc) ? bp - j0 : -1;
  const __nv_bfloat16* q = q_new + unit * D;
  const __nv_bfloat16* kn = k_new + unit * D;
  const __nv_bfloat16* vn = v_new + unit * D;
  if (tid < D) sm.qf[tid] = __bfloat162float(q[tid]);
  if (own >= 0 && tid < 32) {
    // The token's rows are loaded with the pool's loads and stored after it.
    const bool cp = tid < D / 8;
    uint4 kc = make_uint4(0u, 0u, 0u, 0u), vc = kc;
    if (cp) {
      kc = __ldg(reinterpret_cast<const uint4*>(kn) + tid);
      vc = __ldg(reinterpret_cast<const uint4*>(vn) + tid);
    }
    pool_block_warp<true>(K, K_repr, nullptr, nullptr, s, lanes_per_row, unit, bp, tid, kn,
                          pos - bp * BS, sm.mean);
    if (cp) {
      const int64_t row = (unit * s.N + pos) * (int64_t)D;
      reinterpret_cast<uint4*>(K + row)[tid] = kc;
      reinterpret_cast<uint4*>(V + row)[tid] = vc;
    }
  }
  // The only block mean written here is the new block's, which is not read.
  const float* kr = K_repr + unit * s.nb * (int64_t)D;
  if (tid >= 32) {
    for (int i = tid - 32; i < n_loc; i += kDecSelThreads - 32)
      if (i != own) sm.sc[i] = score_block<true>(q, kr + (int64_t)(j0 + i) * D, D, s.scale);
  }
  __syncthreads();                               // sm.qf and sm.mean complete
  if (own >= 0 && tid == 32) {
    float a = 0.f;
    for (int d = 0; d < D; ++d) a = fmaf(sm.qf[d], sm.mean[d], a);
    sm.sc[own] = a * s.scale;
  }
  const int n_own = cluster_pick(sm, n_loc, j0, s, &bars[0], K + unit * s.N * (int64_t)D,
                                 V + unit * s.N * (int64_t)D, (uint32_t)(BS * D * 2));
  fine_row_cluster<BS, D, true>(sm.qf, K, V, sm.sel, max(n_own, 0), O + unit * D, s, unit, pos,
                                &bars[1], false, n_own < 0, kn, vn, pos);
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
  const size_t smem = PickSmem::bytes(s.D, s.nb, s.k);
  if ((int64_t)s.units * kDecCluster > 0x7fffffffLL) return cudaErrorInvalidValue;
#define BSA_DECODE_STEP(BS_, D_)                                                         \
  if (s.bs == BS_ && s.D == D_) {                                                        \
    if (smem > 48 * 1024) {                                                              \
      cudaError_t e = cudaFuncSetAttribute(decode_step_kernel<BS_, D_>,                  \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                           (int)smem);                                   \
      if (e != cudaSuccess) return e;                                                    \
    }                                                                                    \
    decode_step_kernel<BS_, D_><<<(unsigned)(s.units * kDecCluster), kDecSelThreads, smem, \
                                  st>>>(                                                 \
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
  if (rows * kDecCluster > 0x7fffffffLL) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)(rows * kDecCluster)), block(kDecFineWarps * 32);
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
