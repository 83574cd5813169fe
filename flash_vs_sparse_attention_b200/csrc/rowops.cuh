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
template <bool NC>
__device__ __forceinline__ void pool_block_warp(const __nv_bfloat16* __restrict__ K,
                                                float* __restrict__ K_repr,
                                                __nv_bfloat16* __restrict__ K_hi,
                                                __nv_bfloat16* __restrict__ K_lo,
                                                const Shape& s, int lanes_per_row, int64_t unit,
                                                int64_t blk, int lane) {
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
        v[q] = r < rows ? ld_ro<NC>(src + (int64_t)r * chunks + c) : make_uint4(0u, 0u, 0u, 0u);
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

// ---------------------------------------------------------------------------
constexpr int kDecSelThreads = 256;

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
constexpr int kDecFineWarps = 8;

// The whole CTA (kDecFineWarps warps): attention of one query row `q`
// (head_dim D, bf16) at position `pos` of `unit` over the blocks sel[0,
// top_k) (-1 = empty) of the K/V cache, keys below s.kv (and up to pos when
// causal), into the bf16 row `o`.  Split over the blocks: warp w takes slots
// w, w + 8, ...; lane l scores keys l, l + 32, ... of a block (every K-row
// load issued first), exponentiates against the block maximum, then
// accumulates P V for its own output columns with one coalesced V-row load
// per key; each warp keeps a running (m, l, O) and the CTA merges them.
template <int BS, int D, bool NC>
__device__ __forceinline__ void fine_row(const __nv_bfloat16* __restrict__ q,
                                         const __nv_bfloat16* __restrict__ K,
                                         const __nv_bfloat16* __restrict__ V,
                                         const int32_t* sel, __nv_bfloat16* __restrict__ o,
                                         const Shape& s, int64_t unit, int pos) {
  constexpr int KPL = BS / 32;           // keys per lane
  constexpr int DV = D / 8;              // 16-byte chunks per key row
  constexpr int CPL = D / 32;            // output columns per lane (2 or 4)
  __shared__ float qs[D];
  __shared__ float wm[kDecFineWarps], wl[kDecFineWarps];
  __shared__ float wo[kDecFineWarps][D];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int d = tid; d < D; d += kDecFineWarps * 32) qs[d] = __bfloat162float(q[d]);
  __syncthreads();
  const float c = s.scale * kLog2e;      // scores in the base-2 domain
  const __nv_bfloat16* Ku = K + unit * s.N * (int64_t)D;
  const __nv_bfloat16* Vu = V + unit * s.N * (int64_t)D;
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
      for (int v = 0; v < DV; ++v) kr[t][v] = ld_ro<NC>(row + v);
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
    // CPL bf16 per key, all independent.  Keys at or past `lim` (not in the
    // cache yet, or after the row's position) are skipped, not multiplied by
    // p = 0: their V rows may hold anything, NaN included.
    const int64_t lim = s.causal ? min((int64_t)s.kv, (int64_t)pos + 1) : (int64_t)s.kv;
    float ob[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) ob[i] = 0.f;
#pragma unroll
    for (int t = 0; t < KPL; ++t) {
#pragma unroll 8
      for (int kk = 0; kk < 32; ++kk) {
        const float p = __shfl_sync(0xffffffffu, pl[t], kk);
        if (key0 + 32 * t + kk >= lim) continue;   // the same for every lane
        const __nv_bfloat16* vr = Vu + (key0 + 32 * t + kk) * D + CPL * lane;
        if constexpr (CPL == 2) {
          const uint32_t w = ld_ro<NC>(reinterpret_cast<const uint32_t*>(vr));
          ob[0] = fmaf(p, bf16_lo(w), ob[0]);
          ob[1] = fmaf(p, bf16_hi(w), ob[1]);
        } else {
          const uint2 w = ld_ro<NC>(reinterpret_cast<const uint2*>(vr));
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
    o[d] = __float2bfloat16_rn(Osum / Lsum);
  }
}

}  // namespace bsa
