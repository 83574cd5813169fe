// Per-block and per-row building blocks shared by the pool and decode kernels
// and by the fused decode step (one kernel that appends a token to a KV cache,
// re-pools its block, selects and attends).
//
// NC selects the load path: true reads through the read-only (non-coherent)
// cache, valid only for data no thread writes during the kernel; the fused
// decode step writes the new key row and block mean before reading them back,
// so it passes false (L2 loads, coherent with the CTA's own earlier stores).
// The arithmetic is the same either way.
#pragma once

#include "common.cuh"
#include "sm100.cuh"

namespace bsa {

template <bool NC, typename T>
__device__ __forceinline__ T ld_ro(const T* p) {
  if constexpr (NC) return __ldg(p);
  else return __ldcg(p);
}

// One warp: the mean of block `blk` of `unit` over its keys below s.kv
// (block_indexer.py:33), into K_repr, and the bf16 hi/lo split of
// mean * scale into K_hi / K_lo when K_hi is non-null.  Lanes take 16-byte
// chunks of key rows (lanes_per_row chunk lanes per row, the rest of the warp
// on further rows), sum in fp32, and reduce over row groups by shuffles.
// Key row r_new of the block is read from row_new instead of K when row_new
// is non-null (a row not in the cache yet); the mean also goes to mean_out
// when that is non-null.
template <bool NC>
__device__ __forceinline__ void pool_block_warp(const __nv_bfloat16* __restrict__ K,
                                                float* __restrict__ K_repr,
                                                __nv_bfloat16* __restrict__ K_hi,
                                                __nv_bfloat16* __restrict__ K_lo,
                                                const Shape& s, int lanes_per_row, int64_t unit,
                                                int64_t blk, int lane,
                                                const __nv_bfloat16* row_new = nullptr,
                                                int r_new = -1, float* mean_out = nullptr) {
  const int chunks = s.D >> 3;                 // 16-byte chunks per key row
  const int rows_per_iter = 32 / lanes_per_row;
  const int g = lane / lanes_per_row;          // row group
  const int c = lane % lanes_per_row;          // chunk within the row
  const bool active = c < chunks;
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
        const uint4* p = (row_new != nullptr && r == r_new)
                             ? reinterpret_cast<const uint4*>(row_new) + c
                             : src + (int64_t)r * chunks + c;
        v[q] = r < rows ? ld_ro<NC>(p) : make_uint4(0u, 0u, 0u, 0u);
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
    if (mean_out != nullptr) {
#pragma unroll
      for (int i = 0; i < 8; ++i) mean_out[c * 8 + i] = m[i];
    }
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

// ---------------------------------------------------------------------------
constexpr int kDecSelThreads = 512;

// The whole CTA (kDecSelThreads threads): the top_k blocks of one query row
// `gr` (of s.units * s.Nq) into out[0, top_k), ascending, -1 padded.  POOLED:
// the row is a per-query-block mean (fp32; row r stands for block r and sits
// at that block's last position), else a bf16 query at position q0 + r.
// `dsm`: shared memory for head_dim + nb floats and top_k ints.  The scores
// are sequential fp32 dot products over head_dim (as the CUDA-core scorer
// computes them); top_k rounds of a warp arg-max in the order (score
// descending, block ascending) give the exact top-k, lowest index on ties.
// Ends with a CTA barrier.
template <bool POOLED, bool NC>
__device__ __forceinline__ void select_row(const void* __restrict__ Qv,
                                           const float* __restrict__ K_repr,
                                           int32_t* __restrict__ out, const Shape& s, int64_t gr,
                                           float* dsm) {
  float* qs = dsm;                       // head_dim
  float* sc = dsm + s.D;                 // one score per visible block
  int32_t* picks = reinterpret_cast<int32_t*>(sc + s.nb);   // top_k
  __shared__ int n_picked;
  const int tid = threadIdx.x, lane = tid & 31;
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
      for (int u = 0; u < 16; ++u)
        k4[u] = d0 + u < d4n ? ld_ro<NC>(kj + d0 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
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
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Thread-block clusters.  A decode row (one new query row of one unit) is
// split over kDecCluster CTAs of one cluster.  They exchange selection
// candidates and partial attention states by asynchronous stores into each
// other's shared memory (st.async), each completing its bytes on an mbarrier
// of the receiving CTA, which waits there (bounded): no cluster-wide barrier
// and no ordering of global memory between the CTAs is needed.
constexpr int kDecCluster = 8;
constexpr int kDecFineWarps = 16;
// Candidates per CTA whose K and V blocks are prefetched into L2 while the
// cluster's picks are exchanged.
constexpr int kDecPrefetch = 4;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The two halves of a cluster barrier.  Every thread arrives once at the
// start of the kernel (after the mbarriers are initialised: the arrive
// releases at cluster scope) and waits before its first store into another
// CTA's shared memory: a CTA may be accessed only once it has started and
// initialised its mbarriers, which the completed barrier guarantees.  (The
// non-.aligned forms: a warp need not arrive converged.)
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

// The address of `p` (in this CTA's shared memory) in the shared memory of
// cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}

// Asynchronous stores into CTA `rank`'s copy of `dst` (given as this CTA's
// address of the same shared variable), completing their bytes on CTA
// `rank`'s copy of the mbarrier `bar`.  Only for another CTA: a CTA's own
// share goes in with plain shared stores, ordered by a CTA barrier.
__device__ __forceinline__ void st_async_u32(const void* dst, uint32_t v, const uint64_t* bar,
                                             uint32_t rank) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.u32 [%0], %1, [%2];" ::"r"(
                   dsmem_addr(dst, rank)),
               "r"(v), "r"(dsmem_addr(bar, rank))
               : "memory");
}
__device__ __forceinline__ void st_async_u2(const void* dst, uint2 v, const uint64_t* bar,
                                            uint32_t rank) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.u32 [%0], {%1, %2}, [%3];" ::"r"(
          dsmem_addr(dst, rank)),
      "r"(v.x), "r"(v.y), "r"(dsmem_addr(bar, rank))
      : "memory");
}

// Every thread of the CTA waits (bounded) for phase 0 of `bar`; true on
// every thread when it completed for all of them.  Ends with a CTA barrier.
__device__ __forceinline__ bool cta_wait_phase0(uint64_t* bar) {
  const bool ok = sm100::mbar_wait(bar, 0u, nullptr, 0u);
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// Prefetch `bytes` (a multiple of 16, 16-byte aligned) at `p` into L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Selection order of two candidates (score, block): a higher score first,
// the lower block on equal scores (block_indexer.py:53, torch.topk's order
// as the reference uses it).  NaN never precedes anything.
__device__ __forceinline__ bool precedes(float a, int ja, float b, int jb) {
  return a > b || (a == b && ja < jb);
}

// Number of entries m = sub, sub + S, ... below n of the scores `v` (block
// j0 + m) that precede (x, jx) in the selection order: loads in batches of
// eight, all in flight before their comparisons.
template <int S>
__device__ __forceinline__ int count_preceding(const float* v, int n, int sub, float x, int jx) {
  int r = 0;
  for (int m0 = sub; m0 < n; m0 += 8 * S) {
    float o[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) o[u] = m0 + u * S < n ? v[m0 + u * S] : -INFINITY;
#pragma unroll
    for (int u = 0; u < 8; ++u) r += precedes(o[u], m0 + u * S, x, jx) ? 1 : 0;
  }
  return r;
}

// The same over (score bits, block) pairs.
template <int S>
__device__ __forceinline__ int count_preceding(const uint2* v, int n, int sub, float x, int jx) {
  int r = 0;
  for (int m0 = sub; m0 < n; m0 += 8 * S) {
    uint2 o[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) o[u] = m0 + u * S < n ? v[m0 + u * S] : make_uint2(0xff800000u, 0u);
#pragma unroll
    for (int u = 0; u < 8; ++u) r += precedes(__uint_as_float(o[u].x), (int)o[u].y, x, jx) ? 1 : 0;
  }
  return r;
}

// Blocks scored by each CTA of a decode cluster: the eligible range [0, lim)
// in kDecCluster contiguous parts.
__host__ __device__ __forceinline__ int cluster_part(int lim) {
  return (lim + kDecCluster - 1) / kDecCluster;
}

// The fp32 score of one block mean row `krow` against the bf16 query row `q`
// (head_dim D): the sequential dot product over head_dim that select_row
// computes (same values, same order), times `scale`.  The query is read from
// global memory beside the block mean, 64 dimensions per batch, so that both
// are in flight together.
template <bool NC>
__device__ __forceinline__ float score_block(const __nv_bfloat16* __restrict__ q,
                                             const float* __restrict__ krow, int D, float scale) {
  float a = 0.f;
  for (int d0 = 0; d0 < D; d0 += 64) {
    uint4 qv[8];
    float4 k4[16];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      qv[u] = d0 + 8 * u < D ? __ldg(reinterpret_cast<const uint4*>(q + d0) + u)
                             : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 0; u < 16; ++u)
      k4[u] = d0 + 4 * u < D ? ld_ro<NC>(reinterpret_cast<const float4*>(krow + d0) + u)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (d0 + 8 * u < D) {
        a = fmaf(bf16_lo(qv[u].x), k4[2 * u].x, a);
        a = fmaf(bf16_hi(qv[u].x), k4[2 * u].y, a);
        a = fmaf(bf16_lo(qv[u].y), k4[2 * u].z, a);
        a = fmaf(bf16_hi(qv[u].y), k4[2 * u].w, a);
        a = fmaf(bf16_lo(qv[u].z), k4[2 * u + 1].x, a);
        a = fmaf(bf16_hi(qv[u].z), k4[2 * u + 1].y, a);
        a = fmaf(bf16_lo(qv[u].w), k4[2 * u + 1].z, a);
        a = fmaf(bf16_hi(qv[u].w), k4[2 * u + 1].w, a);
      }
    }
  }
  return a * scale;
}

// Shared memory of a decode cluster's selection (cluster_pick and its
// inputs), carved from dynamic shared memory in this order.
struct PickSmem {
  float* qf;        // head_dim: the query row in fp32 (used by the fine stage)
  float* mean;      // head_dim: the re-pooled block mean (decode step)
  float* sc;        // cluster_part(nb), even: this CTA's scores
  uint2* cand;      // top_k: this CTA's candidates, (score bits, block)
  uint2* all;       // kDecCluster * top_k: every CTA's candidates
  int32_t* grank;   // top_k: the rank of candidate t in the cluster's union
  int32_t* sel;     // top_k: this CTA's picks in ascending block order

  __host__ __device__ static size_t bytes(int D, int nb, int k) {
    const size_t part = (size_t)((cluster_part(nb) + 1) & ~1);
    return sizeof(float) * (2 * (size_t)D + part) + sizeof(uint2) * (size_t)k * (1 + kDecCluster) +
           sizeof(int32_t) * (size_t)k * 2;
  }
  __device__ void carve(float* dsm, int D, int nb, int k) {
    qf = dsm;
    mean = qf + D;
    sc = mean + D;
    cand = reinterpret_cast<uint2*>(sc + ((cluster_part(nb) + 1) & ~1));
    all = cand + k;
    grank = reinterpret_cast<int32_t*>(all + kDecCluster * k);
    sel = grank + k;
  }
};

// The whole cluster: from each CTA's scores sc[0, n_loc) of the blocks
// [j0, j0 + n_loc), the top_k blocks of the row in the selection order
// (score descending, block ascending; scores of -inf and NaN never picked) --
// the picks of select_row over the same scores -- with each CTA learning
// which of them lie in its own part: those go to sm.sel in ascending block
// order and their count is returned.  A block of the global top-k is in the
// top-k of its own part, so each CTA keeps as candidates its blocks of rank
// below top_k (cand[rank]: ranks are distinct), prefetches the K and V blocks
// (blk_bytes each, from Kb / Vb, the unit's cache) of its first kDecPrefetch
// candidates into L2, and stores its top_k candidate slots (empty ones as
// -inf) into every CTA's `all`: its own directly, the others' with st.async
// on that CTA's `bar` (phase 0, armed here for the (kDecCluster - 1) * top_k
// * 8 bytes of the other CTAs).  Then each CTA ranks its own candidates in
// the union; those of rank below top_k are its picks (a prefix of cand).
// Every thread must have called cluster_arrive() once before; the matching
// cluster_wait() comes ahead of the first store into another CTA.  Starts
// with a CTA barrier (the scores must be complete), ends with one.  Returns
// -1 (on every thread) if the wait for the candidates ran out.
__device__ __forceinline__ int cluster_pick(const PickSmem& sm, int n_loc, int j0,
                                            const Shape& s, uint64_t* bar,
                                            const __nv_bfloat16* Kb, const __nv_bfloat16* Vb,
                                            uint32_t blk_bytes) {
  const int tid = threadIdx.x;
  const uint32_t rank = cluster_rank();
  const int M = kDecCluster * s.k;
  __syncthreads();
  // Local ranks: 4 threads per block (neighbouring lanes), each comparing a
  // quarter of the part, summed by shuffles.
  int n_elig = 0;
  {
    const int sub = tid & 3;
    for (int i0 = 0; i0 < n_loc; i0 += kDecSelThreads / 4) {
      const int i = i0 + (tid >> 2);
      const float x = i < n_loc ? sm.sc[i] : -INFINITY;
      const bool elig = x > -INFINITY;
      int r = elig ? count_preceding<4>(sm.sc, n_loc, sub, x, i) : 0;
      r += __shfl_xor_sync(0xffffffffu, r, 1);
      r += __shfl_xor_sync(0xffffffffu, r, 2);
      if (elig && sub == 0 && r < s.k) sm.cand[r] = make_uint2(__float_as_uint(x), (uint32_t)(j0 + i));
      n_elig += __syncthreads_count(elig && sub == 0);   // also orders the cand stores
    }
  }
  const int n_cand = min(n_elig, s.k);
  if (tid < min(n_cand, kDecPrefetch)) {
    const int64_t off = (int64_t)sm.cand[tid].y * s.bs * s.D;
    prefetch_l2(Kb + off, blk_bytes);
    prefetch_l2(Vb + off, blk_bytes);
  }
  if (tid == 0)
    sm100::mbar_arrive_expect_tx(bar, (uint32_t)((M - s.k) * sizeof(uint2)));
  cluster_wait();                          // every CTA of the cluster has started
  for (int e = tid; e < M; e += kDecSelThreads) {
    const uint32_t dst = (uint32_t)(e / s.k);
    const int t = e % s.k;
    const uint2 v = t < n_cand ? sm.cand[t] : make_uint2(0xff800000u, 0u);   // -inf: empty
    if (dst == rank) sm.all[rank * s.k + t] = v;
    else st_async_u2(sm.all + rank * s.k + t, v, bar, dst);
  }
  if (!cta_wait_phase0(bar)) return -1;
  // Ranks of the own candidates in the union: 16 threads per candidate (a
  // half warp), each comparing every 16th entry.
  for (int t0 = 0; t0 < s.k; t0 += kDecSelThreads / 16) {
    const int t = t0 + (tid >> 4), sub = tid & 15;
    const uint2 me = t < n_cand ? sm.cand[t] : make_uint2(0xff800000u, 0u);
    const float x = __uint_as_float(me.x);
    int r = x > -INFINITY ? count_preceding<16>(sm.all, M, sub, x, (int)me.y) : 0;
#pragma unroll
    for (int x2 = 1; x2 < 16; x2 <<= 1) r += __shfl_xor_sync(0xffffffffu, r, x2);
    if (t < s.k && sub == 0) sm.grank[t] = t < n_cand ? r : s.k;
  }
  __syncthreads();
  // The picks (candidates of rank below top_k) in ascending block order.
  int n_own = 0;
  for (int t0 = 0; t0 < s.k; t0 += kDecSelThreads) {
    const int t = t0 + tid;
    const bool pick = t < s.k && sm.grank[t] < s.k;
    if (pick) {
      const int jx = (int)sm.cand[t].y;
      int slot = 0;
      for (int u = 0; u < s.k; ++u) slot += (sm.grank[u] < s.k && (int)sm.cand[u].y < jx) ? 1 : 0;
      sm.sel[slot] = jx;
    }
    n_own += __syncthreads_count(pick);
  }
  return n_own;
}

// Bytes of the partial states the other CTAs of a fine_row_cluster call send
// to CTA 0 (CTA 0 stores its own directly).
template <int D>
__host__ __device__ constexpr uint32_t fine_state_bytes() {
  return (uint32_t)((kDecCluster - 1) * (D * sizeof(float) + sizeof(float2)));
}

// The whole cluster: attention of one query row `qs` (head_dim D, fp32 in
// shared memory, complete before the call) at position `pos` of `unit` over
// its selected blocks of the K/V cache, keys below s.kv (and up to pos when
// causal), into the bf16 row `o` (written by CTA 0).  Each CTA attends the
// selected blocks of its own part of the eligible range (cluster_part), given
// in `sel` (n_sel blocks, ascending).  Key `key_new` (when k_new is non-null)
// is read from k_new / v_new instead of the cache.  Work item i is the 32-key
// chunk i % (BS / 32) of sel[i / (BS / 32)]; warp w takes items w, w + W, ...
// (W = kDecFineWarps).
// For an item, lane
// l loads key row key0 + l and, at the same time, the V chunks of its P V
// share (16-byte column chunk l % (D / 8) of the keys congruent to
// l / (D / 8)); it scores its key (a sequential fp32 dot product over
// head_dim), exponentiates against the chunk maximum, accumulates p * V for
// its chunk's columns over its keys, and the warp sums the row groups by
// shuffles.  Keys at or past the visible limit are neither weighted nor read
// from V (those rows may hold anything, NaN included).  Each warp folds its
// items into a running (m, l, O); the CTA merges its warps in order and
// stores its state into CTA 0's slot `rank` with st.async on CTA 0's
// `state_bar` (armed by CTA 0 for fine_state_bytes<D>() before its cluster
// arrive); CTA 0 waits for all of them (bounded) and merges the CTAs in rank
// order.  `poison`: this CTA's state is NaN (its selection wait ran out), so
// the row comes out NaN.  `wait_started`: the cluster_wait() matching the
// caller's cluster_arrive() is still to come (before the stores).
template <int BS, int D, bool NC>
__device__ __forceinline__ void fine_row_cluster(const float* qs,
                                                 const __nv_bfloat16* __restrict__ K,
                                                 const __nv_bfloat16* __restrict__ V,
                                                 const int32_t* sel, int n_sel,
                                                 __nv_bfloat16* __restrict__ o,
                                                 const Shape& s, int64_t unit, int pos,
                                                 uint64_t* state_bar, bool wait_started,
                                                 bool poison, const __nv_bfloat16* k_new,
                                                 const __nv_bfloat16* v_new, int64_t key_new) {
  constexpr int DV = D / 8;              // 16-byte chunks per key row
  constexpr int G = 32 / DV;             // row groups of the P V layout (4 or 2)
  constexpr int KPL = 32 / G;            // keys per lane in P V (8 or 16)
  constexpr int CPB = BS / 32;           // 32-key chunks per block
  static_assert(DV * G == 32 && CPB >= 1, "head_dim 64/128, block_size a multiple of 32");
  __shared__ float wm[kDecFineWarps], wl[kDecFineWarps];
  __shared__ __align__(16) float wo[kDecFineWarps][D];
  __shared__ float2 cml[kDecCluster];    // the CTAs' (m, l) (in CTA 0)
  __shared__ __align__(16) float co[kDecCluster][D];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_rank();
  const int g = lane / DV, c = lane % DV;
  const float cs = s.scale * kLog2e;     // scores in the base-2 domain
  const __nv_bfloat16* Ku = K + unit * s.N * (int64_t)D;
  const __nv_bfloat16* Vu = V + unit * s.N * (int64_t)D;
  const int64_t lim = s.causal ? min((int64_t)s.kv, (int64_t)pos + 1) : (int64_t)s.kv;
  if (k_new == nullptr) key_new = -1;
  float m = -INFINITY, l = 0.f, acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const int items = n_sel * CPB;
  for (int it = warp; it < items; it += kDecFineWarps) {
    const int j = sel[it / CPB];
    const int64_t key0 = (int64_t)j * BS + (int64_t)(it % CPB) * 32;
    if (key0 >= lim) continue;           // every key of the chunk masked (same on all lanes)
    uint4 kr[DV], vr[KPL];
    const uint4* krow = key0 + lane == key_new
                            ? reinterpret_cast<const uint4*>(k_new)
                            : reinterpret_cast<const uint4*>(Ku + (key0 + lane) * D);
#pragma unroll
    for (int v = 0; v < DV; ++v) kr[v] = ld_ro<NC>(krow + v);
#pragma unroll
    for (int i = 0; i < KPL; ++i) {
      const int64_t key = key0 + g + G * i;
      const uint4* vrow = key == key_new ? reinterpret_cast<const uint4*>(v_new)
                                         : reinterpret_cast<const uint4*>(Vu + key * D);
      vr[i] = key < lim ? ld_ro<NC>(vrow + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    float a = 0.f;
#pragma unroll
    for (int v = 0; v < DV; ++v) {
      const float* qq = qs + 8 * v;
      a = fmaf(qq[0], bf16_lo(kr[v].x), a); a = fmaf(qq[1], bf16_hi(kr[v].x), a);
      a = fmaf(qq[2], bf16_lo(kr[v].y), a); a = fmaf(qq[3], bf16_hi(kr[v].y), a);
      a = fmaf(qq[4], bf16_lo(kr[v].z), a); a = fmaf(qq[5], bf16_hi(kr[v].z), a);
      a = fmaf(qq[6], bf16_lo(kr[v].w), a); a = fmaf(qq[7], bf16_hi(kr[v].w), a);
    }
    const float sv = key0 + lane < lim ? a * cs : -INFINITY;
    const float bm = warp_max(sv);       // finite: key0 itself is visible
    const float p = fast_exp2(sv - bm);  // 0 for masked keys
    const float ps = warp_sum(p);
    float ob[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) ob[e] = 0.f;
#pragma unroll
    for (int i = 0; i < KPL; ++i) {
      const float pi = __shfl_sync(0xffffffffu, p, g + G * i);
      ob[0] = fmaf(pi, bf16_lo(vr[i].x), ob[0]); ob[1] = fmaf(pi, bf16_hi(vr[i].x), ob[1]);
      ob[2] = fmaf(pi, bf16_lo(vr[i].y), ob[2]); ob[3] = fmaf(pi, bf16_hi(vr[i].y), ob[3]);
      ob[4] = fmaf(pi, bf16_lo(vr[i].z), ob[4]); ob[5] = fmaf(pi, bf16_hi(vr[i].z), ob[5]);
      ob[6] = fmaf(pi, bf16_lo(vr[i].w), ob[6]); ob[7] = fmaf(pi, bf16_hi(vr[i].w), ob[7]);
    }
#pragma unroll
    for (int x = DV; x < 32; x <<= 1) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ob[e] += __shfl_xor_sync(0xffffffffu, ob[e], x);
    }
    // Fold the chunk into the warp's running state.
    const float mn = fmaxf(m, bm);
    const float ca = (m == -INFINITY) ? 0.f : fast_exp2(m - mn);
    const float cb = fast_exp2(bm - mn);
    l = l * ca + ps * cb;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = acc[e] * ca + ob[e] * cb;
    m = mn;
  }
  if (lane == 0) { wm[warp] = m; wl[warp] = l; }
  if (g == 0) {
    float4* w4 = reinterpret_cast<float4*>(&wo[warp][8 * c]);
    w4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    w4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
  // The CTA's state (one thread per output column, thread 0 also m and l)
  // into CTA 0's slot `rank`.
  if (wait_started) cluster_wait();      // CTA 0 has started
  if (tid < D) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecFineWarps; ++w) M = fmaxf(M, wm[w]);
    float Lsum = 0.f, Osum = 0.f;
#pragma unroll
    for (int w = 0; w < kDecFineWarps; ++w) {
      const float f = wm[w] == -INFINITY ? 0.f : fast_exp2(wm[w] - M);
      Lsum = fmaf(wl[w], f, Lsum);
      Osum = fmaf(wo[w][tid], f, Osum);
    }
    if (poison) M = Lsum = Osum = __uint_as_float(0x7fc00000u);   // NaN
    if (rank == 0) {
      co[0][tid] = Osum;
      if (tid == 0) cml[0] = make_float2(M, Lsum);
    } else {
      st_async_u32(&co[rank][tid], __float_as_uint(Osum), state_bar, 0u);
      if (tid == 0)
        st_async_u2(&cml[rank], make_uint2(__float_as_uint(M), __float_as_uint(Lsum)), state_bar,
                    0u);
    }
  }
  if (rank != 0) return;                 // nothing reads this CTA's shared memory any more
  const bool ok = cta_wait_phase0(state_bar);
  if (tid < D) {
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kDecCluster; ++r) M = fmaxf(M, cml[r].x);
    float Lsum = 0.f, Osum = 0.f;
#pragma unroll
    for (int r = 0; r < kDecCluster; ++r) {
      const float f = cml[r].x == -INFINITY ? 0.f : fast_exp2(cml[r].x - M);
      Lsum = fmaf(cml[r].y, f, Lsum);
      Osum = fmaf(co[r][tid], f, Osum);
    }
    o[tid] = __float2bfloat16_rn(ok ? Osum / Lsum : __uint_as_float(0x7fc00000u));
  }
}

}  // namespace bsa
