// The backward pass of the fine stage, on CUDA cores: dQ, dK, dV of
// O = attention over the selected blocks, the selection held fixed.
// (The reference's stated next step, blog.md:133.  Its PyTorch variant,
// block_indexer.py, is differentiable; autograd gives Q, K and V the
// gradient of the fine stage, block_indexer.py:55-84, and nothing flows
// through the top-k indices, :53.)
//
// Per query row i over its selected keys (scale = D^-1/2, w the softmax
// weights):
//     dV[key] += w * dO_i,   dp = V[key] . dO_i,   ds = w (dp - dO_i . O_i),
//     dQ_i = scale sum ds K[key],   dK[key] += scale ds Q_i.
//
//  1. bwd_rows_kernel   query-stationary, a warp per row: the row's log-sum-exp
//                       and O (recomputed in fp32), D_i = dO_i . O_i, then dQ_i.
//                       Lanes take keys for the dot products (32 keys at a
//                       time) and output columns for the weighted sums.
//  2. bucket lists      per (unit, key block) the rows that picked it -- the
//                       forward's bucket kernels (fine_kv.cu).
//  3. bwd_kv_kernel     key-stationary, a CTA per (unit, key block): its
//                       rows, sorted ascending, 8 at a time (a warp per row
//                       for the block's scores), dK and dV of the block
//                       accumulated in registers (thread t owns elements t,
//                       t + 256, ...) and written once.  No atomics: each
//                       gradient element is summed by one thread in row
//                       order, so the result is the same on every run.
#include "common.cuh"
#include "launchers.cuh"

namespace bsa {

constexpr int kBwdRowsWarps = 8;
constexpr int kBwdKvThreads = 256;
constexpr int kBwdBatch = kBwdKvThreads / 32;   // rows per batch in bwd_kv_kernel
constexpr int kBwdSortCap = 8192;                // longer lists run unsorted

template <int DPL>   // output columns per lane: head_dim / 32
__device__ __forceinline__ float dot_row(const float* __restrict__ x_smem,
                                         const __nv_bfloat16* __restrict__ row) {
  constexpr int D = DPL * 32;
  float acc = 0.f;
  const uint4* r4 = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
  for (int c = 0; c < D / 8; ++c) {
    const uint4 w = __ldg(r4 + c);
    const float* x = x_smem + 8 * c;
    acc = fmaf(x[0], bf16_lo(w.x), acc);
    acc = fmaf(x[1], bf16_hi(w.x), acc);
    acc = fmaf(x[2], bf16_lo(w.y), acc);
    acc = fmaf(x[3], bf16_hi(w.y), acc);
    acc = fmaf(x[4], bf16_lo(w.z), acc);
    acc = fmaf(x[5], bf16_hi(w.z), acc);
    acc = fmaf(x[6], bf16_lo(w.w), acc);
    acc = fmaf(x[7], bf16_hi(w.w), acc);
  }
  return acc;
}

// Lane's DPL columns of a bf16 row (columns lane * DPL ...).
template <int DPL>
__device__ __forceinline__ void load_cols(const __nv_bfloat16* __restrict__ row, int lane,
                                          float (&out)[DPL]) {
#pragma unroll
  for (int c = 0; c < DPL; ++c) out[c] = __bfloat162float(row[lane * DPL + c]);
}

// CACHE: each warp keeps its row's scores and dP (k * bs floats each) in
// shared memory from the first pass, so the later passes read every key
// row once, coalesced; otherwise they recompute them.
template <int DPL, bool CACHE>
__global__ void __launch_bounds__(kBwdRowsWarps * 32)
bwd_rows_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                const __nv_bfloat16* __restrict__ V, const __nv_bfloat16* __restrict__ dO,
                const int32_t* __restrict__ idx, __nv_bfloat16* __restrict__ dQ,
                float* __restrict__ lse_out, float* __restrict__ delta_out, Shape s) {
  constexpr int D = DPL * 32;
  __shared__ float q_s[kBwdRowsWarps][D], g_s[kBwdRowsWarps][D], w_s[kBwdRowsWarps][32];
  extern __shared__ float cache_f[];   // CACHE: per warp, k * bs scores then k * bs dP
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u = blockIdx.y, row = blockIdx.x * kBwdRowsWarps + warp;
  if (row >= s.N) return;   // whole warp; no CTA barrier below
  const int kb = s.k * s.bs;
  float* s_c = cache_f + (size_t)warp * 2 * kb;
  float* dp_c = s_c + kb;
  const int64_t R = (int64_t)u * s.N + row;
  float qd[DPL], gd[DPL];
  load_cols<DPL>(Q + R * D, lane, qd);
  load_cols<DPL>(dO + R * D, lane, gd);
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    q_s[warp][lane * DPL + c] = qd[c];
    g_s[warp][lane * DPL + c] = gd[c];
  }
  __syncwarp();
  const int32_t* sel = idx + R * s.k;
  const __nv_bfloat16* Ku = K + (int64_t)u * s.N * D;
  const __nv_bfloat16* Vu = V + (int64_t)u * s.N * D;
  const float sc = s.scale * 1.4426950408889634f;   // scores in the base-2 domain
  // Score of key `key` for this row in the base-2 domain (-inf if masked).
  auto score = [&](int key, bool in_block) -> float {
    const bool live = in_block && (!s.causal || key <= row);
    return live ? dot_row<DPL>(q_s[warp], Ku + (int64_t)key * D) * sc : -INFINITY;
  };
  // 1. log-sum-exp (base 2) over the selected keys (and, cached, dP).
  float m = -INFINITY, l = 0.f;
  for (int q = 0; q < s.k; ++q) {
    const int j = sel[q];
    if (j < 0) continue;
    for (int c0 = 0; c0 < s.bs; c0 += 32) {
      const int key = j * s.bs + c0 + lane;
      const bool in_block = c0 + lane < s.bs;
      const float x = score(key, in_block);
      if (CACHE && in_block) {
        s_c[q * s.bs + c0 + lane] = x;
        dp_c[q * s.bs + c0 + lane] =
            x != -INFINITY ? dot_row<DPL>(g_s[warp], Vu + (int64_t)key * D) : 0.f;
      }
      const float gm = warp_max(x);
      if (gm == -INFINITY) continue;
      if (gm > m) {
        l *= exp2f(m - gm);
        m = gm;
      }
      l += warp_sum(exp2f(x - m));
    }
  }
  __syncwarp();
  const float lse = m + log2f(l);
  // 2. O (fp32) and delta = dO . O.
  float o[DPL];
#pragma unroll
  for (int c = 0; c < DPL; ++c) o[c] = 0.f;
  for (int q = 0; q < s.k; ++q) {
    const int j = sel[q];
    if (j < 0) continue;
    for (int c0 = 0; c0 < s.bs; c0 += 32) {
      const bool in_block = c0 + lane < s.bs;
      const float x = CACHE ? (in_block ? s_c[q * s.bs + c0 + lane] : -INFINITY)
                            : score(j * s.bs + c0 + lane, in_block);
      w_s[warp][lane] = exp2f(x - lse);
      __syncwarp();
      const int n = min(32, s.bs - c0);
      for (int t = 0; t < n; ++t) {
        const float p = w_s[warp][t];
        if (p == 0.f) continue;
        float v[DPL];
        load_cols<DPL>(Vu + (int64_t)(j * s.bs + c0 + t) * D, lane, v);
#pragma unroll
        for (int c = 0; c < DPL; ++c) o[c] = fmaf(p, v[c], o[c]);
      }
      __syncwarp();
    }
  }
  float dl = 0.f;
#pragma unroll
  for (int c = 0; c < DPL; ++c) dl = fmaf(gd[c], o[c], dl);
  const float delta = warp_sum(dl);
  // 3. dQ = scale sum_key w (dp - delta) K[key].
  float dq[DPL];
#pragma unroll
  for (int c = 0; c < DPL; ++c) dq[c] = 0.f;
  for (int q = 0; q < s.k; ++q) {
    const int j = sel[q];
    if (j < 0) continue;
    for (int c0 = 0; c0 < s.bs; c0 += 32) {
      const int key = j * s.bs + c0 + lane;
      const bool in_block = c0 + lane < s.bs;
      float x, dp;
      if (CACHE) {
        x = in_block ? s_c[q * s.bs + c0 + lane] : -INFINITY;
        dp = in_block ? dp_c[q * s.bs + c0 + lane] : 0.f;
      } else {
        x = score(key, in_block);
        dp = x != -INFINITY ? dot_row<DPL>(g_s[warp], Vu + (int64_t)key * D) : 0.f;
      }
      const float p = exp2f(x - lse);
      w_s[warp][lane] = p * (dp - delta);
      __syncwarp();
      const int n = min(32, s.bs - c0);
      for (int t = 0; t < n; ++t) {
        const float ds = w_s[warp][t];
        if (ds == 0.f) continue;
        float kk[DPL];
        load_cols<DPL>(Ku + (int64_t)(j * s.bs + c0 + t) * D, lane, kk);
#pragma unroll
        for (int c = 0; c < DPL; ++c) dq[c] = fmaf(ds, kk[c], dq[c]);
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int c = 0; c < DPL; ++c) dQ[R * D + lane * DPL + c] = __float2bfloat16(dq[c] * s.scale);
  if (lane == 0) {
    lse_out[R] = lse;
    delta_out[R] = delta;
  }
}

template <int DPL, int EPT>   // EPT: gradient elements per thread, >= bs * D / 256
__global__ void __launch_bounds__(kBwdKvThreads, 2)
bwd_kv_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
              const __nv_bfloat16* __restrict__ V, const __nv_bfloat16* __restrict__ dO,
              const float* __restrict__ lse, const float* __restrict__ delta,
              const int32_t* __restrict__ lists, const int32_t* __restrict__ offsets,
              const int32_t* __restrict__ counts, __nv_bfloat16* __restrict__ dK,
              __nv_bfloat16* __restrict__ dV, Shape s) {
  constexpr int D = DPL * 32;
  extern __shared__ float smem_f[];
  const int j = blockIdx.x, u = blockIdx.y, t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int bs = s.bs;
  // Shared memory: K and V of the block (rows padded by one float against
  // bank conflicts), the batch's rows of Q and dO, their weights, the list.
  float* Kb = smem_f;                              // bs x (D + 1)
  float* Vb = Kb + bs * (D + 1);                   // bs x (D + 1)
  float* qb = Vb + bs * (D + 1);                   // kBwdBatch x D
  float* gb = qb + kBwdBatch * D;                  // kBwdBatch x D
  float* pb = gb + kBwdBatch * D;                  // kBwdBatch x bs
  float* db = pb + kBwdBatch * bs;                 // kBwdBatch x bs
  int32_t* lst = reinterpret_cast<int32_t*>(db + kBwdBatch * bs);   // kBwdSortCap
  const int64_t blk0 = (int64_t)u * s.N + (int64_t)j * bs;
  for (int e = t; e < bs * D; e += kBwdKvThreads) {
    const int r = e / D, d = e % D;
    Kb[r * (D + 1) + d] = __bfloat162float(K[(blk0 + r) * D + d]);
    Vb[r * (D + 1) + d] = __bfloat162float(V[(blk0 + r) * D + d]);
  }
  const int n = counts[(int64_t)u * s.nb + j];
  const int32_t* lg = lists + (int64_t)u * s.N * s.k + offsets[(int64_t)u * s.nb + j];
  // Rows in ascending order, so every run sums in the same order.
  const bool sorted = n <= kBwdSortCap;
  if (sorted) {
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    for (int i = t; i < n2; i += kBwdKvThreads) lst[i] = i < n ? lg[i] : 0x7fffffff;
    __syncthreads();
    for (int k2 = 2; k2 <= n2; k2 <<= 1) {
      for (int h = k2 >> 1; h > 0; h >>= 1) {
        for (int i = t; i < n2; i += kBwdKvThreads) {
          const int l = i ^ h;
          if (l > i) {
            const int a = lst[i], b = lst[l];
            const bool up = (i & k2) == 0;
            if ((a > b) == up) {
              lst[i] = b;
              lst[l] = a;
            }
          }
        }
        __syncthreads();
      }
    }
  }
  __syncthreads();
  float gk[EPT], gv[EPT];
#pragma unroll
  for (int m = 0; m < EPT; ++m) gk[m] = gv[m] = 0.f;
  const float sc = s.scale * 1.4426950408889634f;
  for (int b0 = 0; b0 < n; b0 += kBwdBatch) {
    // Warp w: row b0 + w of the list -- its Q and dO rows, then the block's
    // weights p and p (dp - delta) for that row (zero for a missing row).
    const int i = b0 + warp;
    const int row = i < n ? (sorted ? lst[i] : lg[i]) : -1;
    float* qw = qb + warp * D;
    float* gw = gb + warp * D;
    for (int d = lane; d < D; d += 32) {
      qw[d] = row >= 0 ? __bfloat162float(Q[((int64_t)u * s.N + row) * D + d]) : 0.f;
      gw[d] = row >= 0 ? __bfloat162float(dO[((int64_t)u * s.N + row) * D + d]) : 0.f;
    }
    __syncwarp();
    const float ls = row >= 0 ? lse[(int64_t)u * s.N + row] : 0.f;
    const float dl = row >= 0 ? delta[(int64_t)u * s.N + row] : 0.f;
    for (int r = lane; r < bs; r += 32) {
      float p = 0.f, ds = 0.f;
      if (row >= 0 && (!s.causal || j * bs + r <= row)) {
        float x = 0.f, dp = 0.f;
        const float* kr = Kb + r * (D + 1);
        const float* vr = Vb + r * (D + 1);
#pragma unroll 8
        for (int d = 0; d < D; ++d) {
          x = fmaf(qw[d], kr[d], x);
          dp = fmaf(gw[d], vr[d], dp);
        }
        p = exp2f(x * sc - ls);
        ds = p * (dp - dl);
      }
      pb[warp * bs + r] = p;
      db[warp * bs + r] = ds;
    }
    __syncthreads();
    // dV[r][d] += p_w[r] dO_w[d], dK[r][d] += ds_w[r] Q_w[d], rows in order.
#pragma unroll
    for (int m = 0; m < EPT; ++m) {
      const int e = t + m * kBwdKvThreads;
      if (e < bs * D) {
        const int r = e / D, d = e % D;
#pragma unroll
        for (int w = 0; w < kBwdBatch; ++w) {
          gv[m] = fmaf(pb[w * bs + r], gb[w * D + d], gv[m]);
          gk[m] = fmaf(db[w * bs + r], qb[w * D + d], gk[m]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int m = 0; m < EPT; ++m) {
    const int e = t + m * kBwdKvThreads;
    if (e < bs * D) {
      const int r = e / D, d = e % D;
      dK[(blk0 + r) * D + d] = __float2bfloat16(gk[m] * s.scale);
      dV[(blk0 + r) * D + d] = __float2bfloat16(gv[m]);
    }
  }
}

bool backward_supported(const Shape& s) {
  return (s.D == 32 || s.D == 64 || s.D == 96 || s.D == 128) && s.bs * s.D <= 8192 &&
         s.k <= 64 && s.nb <= 16384 && (int64_t)s.units * s.N * s.k < (1LL << 31);
}

static size_t bwd_kv_smem(const Shape& s) {
  return sizeof(float) * (2 * (size_t)s.bs * (s.D + 1) + 2 * (size_t)kBwdBatch * s.D +
                          2 * (size_t)kBwdBatch * s.bs) +
         sizeof(int32_t) * kBwdSortCap;
}

size_t backward_workspace_bytes(const Shape& s) {
  const size_t rows = (size_t)s.units * s.N;
  return fine_kv_workspace_bytes(s) + ((2 * rows * sizeof(float) + 255) & ~(size_t)255);
}

template <int DPL, int EPT>
static cudaError_t launch_bwd_kv(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                 const __nv_bfloat16* V, const __nv_bfloat16* dO,
                                 const float* lse, const float* delta, const BucketLists& bl,
                                 __nv_bfloat16* dK, __nv_bfloat16* dV, const Shape& s,
                                 cudaStream_t st) {
  const size_t smem = bwd_kv_smem(s);
  cudaError_t e = cudaFuncSetAttribute(bwd_kv_kernel<DPL, EPT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  bwd_kv_kernel<DPL, EPT><<<dim3(s.nb, s.units), kBwdKvThreads, smem, st>>>(
      Q, K, V, dO, lse, delta, bl.lists, bl.offsets, bl.counts, dK, dV, s);
  return cudaGetLastError();
}

template <int DPL>
static cudaError_t launch_bwd(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                              const __nv_bfloat16* V, const __nv_bfloat16* dO,
                              const int32_t* idx, __nv_bfloat16* dQ, __nv_bfloat16* dK,
                              __nv_bfloat16* dV, unsigned char* ws, const Shape& s,
                              cudaStream_t st) {
  float* lse = reinterpret_cast<float*>(ws + fine_kv_workspace_bytes(s));
  float* delta = lse + (size_t)s.units * s.N;
  dim3 g1((s.N + kBwdRowsWarps - 1) / kBwdRowsWarps, s.units);
  // Cached scores and dP: 8 warps x 2 x k * bs floats (64 KiB at k * bs = 1024).
  const size_t cache = sizeof(float) * kBwdRowsWarps * 2 * (size_t)s.k * s.bs;
  cudaError_t e;
  if (cache <= 96 * 1024) {
    if ((e = cudaFuncSetAttribute(bwd_rows_kernel<DPL, true>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cache)) !=
        cudaSuccess)
      return e;
    bwd_rows_kernel<DPL, true><<<g1, kBwdRowsWarps * 32, cache, st>>>(Q, K, V, dO, idx, dQ, lse,
                                                                      delta, s);
  } else {
    bwd_rows_kernel<DPL, false><<<g1, kBwdRowsWarps * 32, 0, st>>>(Q, K, V, dO, idx, dQ, lse,
                                                                   delta, s);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  BucketLists bl;
  if ((e = launch_bucket_lists(idx, V, ws, s, st, &bl)) != cudaSuccess) return e;
  const int elems = s.bs * s.D;
  if (elems <= 256) return launch_bwd_kv<DPL, 1>(Q, K, V, dO, lse, delta, bl, dK, dV, s, st);
  if (elems <= 512) return launch_bwd_kv<DPL, 2>(Q, K, V, dO, lse, delta, bl, dK, dV, s, st);
  if (elems <= 1024) return launch_bwd_kv<DPL, 4>(Q, K, V, dO, lse, delta, bl, dK, dV, s, st);
  if (elems <= 2048) return launch_bwd_kv<DPL, 8>(Q, K, V, dO, lse, delta, bl, dK, dV, s, st);
  if (elems <= 4096) return launch_bwd_kv<DPL, 16>(Q, K, V, dO, lse, delta, bl, dK, dV, s, st);
  return launch_bwd_kv<DPL, 32>(Q, K, V, dO, lse, delta, bl, dK, dV, s, st);
}

cudaError_t launch_backward(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                            const __nv_bfloat16* V, const __nv_bfloat16* dO, const int32_t* idx,
                            __nv_bfloat16* dQ, __nv_bfloat16* dK, __nv_bfloat16* dV,
                            unsigned char* ws, const Shape& s, cudaStream_t st) {
  switch (s.D) {
    case 32: return launch_bwd<1>(Q, K, V, dO, idx, dQ, dK, dV, ws, s, st);
    case 64: return launch_bwd<2>(Q, K, V, dO, idx, dQ, dK, dV, ws, s, st);
    case 96: return launch_bwd<3>(Q, K, V, dO, idx, dQ, dK, dV, ws, s, st);
    case 128: return launch_bwd<4>(Q, K, V, dO, idx, dQ, dK, dV, ws, s, st);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace bsa
