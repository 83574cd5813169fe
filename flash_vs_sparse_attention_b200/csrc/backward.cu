// The backward pass of the fine stage: dQ, dK, dV of O = attention over the
// selected blocks, the selection held fixed (CUDA cores, and mma.sync tensor
// cores for the per-block products at block_size 64 / head_dim 64).
// (The reference's stated next step, blog.md:133.  Its PyTorch variant,
// block_indexer.py, is differentiable; autograd gives Q, K and V the
// gradient of the fine stage, block_indexer.py:55-84, and nothing flows
// through the top-k indices, :53.)
//
// Per query row i over its selected keys (scale = D^-1/2, w the softmax
// weights, delta_i = dO_i . O_i):
//     dV[key] += w * dO_i,   dp = V[key] . dO_i,   ds = w (dp - delta_i),
//     dQ_i = scale sum ds K[key],   dK[key] += scale ds Q_i.
//
//  1. bwd_lse_kernel    a warp per row: the row's log-sum-exp over its
//                       selected keys (lanes take keys) and delta_i from the
//                       forward's O.
//  2. bucket lists      per (unit, key block) the rows that picked it -- the
//                       forward's bucket kernels (fine_kv.cu).
//  3. bwd_kv_kernel     key-stationary, a CTA per (unit, key block): its
//                       rows, sorted ascending, 8 at a time (a warp per row
//                       for the block's scores and dP); dK and dV of the
//                       block summed in registers (each thread a 4-row tile,
//                       or elements t, t + 256, ...) and written once, and
//                       for each row the block's share of dQ written to the
//                       row's slot.
//                       At block_size 64 and head_dim 64 the same step runs
//                       on tensor cores (bwd_kv_mma_kernel, mma.sync), and
//                       step 1 is replaced by a key-block pass
//                       (bwd_lse_mma_kernel: each row's per-block share of
//                       its normaliser) and a per-row merge
//                       (bwd_lse_merge_kernel).
//  4. bwd_dq_kernel     per row, the sum of its slots' dQ shares.
// No atomics: every sum runs in a fixed order (rows ascending, slots
// ascending), so the result is the same on every run.
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

template <int DPL>
__global__ void __launch_bounds__(kBwdRowsWarps * 32)
bwd_lse_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
               const __nv_bfloat16* __restrict__ O, const __nv_bfloat16* __restrict__ dO,
               const int32_t* __restrict__ idx, float* __restrict__ lse_out,
               float* __restrict__ delta_out, Shape s) {
  constexpr int D = DPL * 32;
  __shared__ float q_s[kBwdRowsWarps][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u = blockIdx.y, row = blockIdx.x * kBwdRowsWarps + warp;
  if (row >= s.N) return;   // whole warp; no CTA barrier below
  const int64_t R = (int64_t)u * s.N + row;
  float qd[DPL], od[DPL], gd[DPL];
  load_cols<DPL>(Q + R * D, lane, qd);
  load_cols<DPL>(O + R * D, lane, od);
  load_cols<DPL>(dO + R * D, lane, gd);
  float dl = 0.f;
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    q_s[warp][lane * DPL + c] = qd[c];
    dl = fmaf(gd[c], od[c], dl);
  }
  const float delta = warp_sum(dl);
  __syncwarp();
  const int32_t* sel = idx + R * s.k;
  const __nv_bfloat16* Ku = K + (int64_t)u * s.N * D;
  const float sc = s.scale * 1.4426950408889634f;   // scores in the base-2 domain
  float m = -INFINITY, l = 0.f;
  for (int q = 0; q < s.k; ++q) {
    const int j = sel[q];
    if (j < 0) continue;
    for (int c0 = 0; c0 < s.bs; c0 += 32) {
      const int key = j * s.bs + c0 + lane;
      const bool live = c0 + lane < s.bs && (!s.causal || key <= row);
      const float x = live ? dot_row<DPL>(q_s[warp], Ku + (int64_t)key * D) * sc : -INFINITY;
      const float gm = warp_max(x);
      if (gm == -INFINITY) continue;
      if (gm > m) {
        l *= exp2f(m - gm);
        m = gm;
      }
      l += warp_sum(exp2f(x - m));
    }
  }
  if (lane == 0) {
    lse_out[R] = m + log2f(l);
    delta_out[R] = delta;
  }
}

// Shared-memory row stride of the block's K and V (floats): a multiple of 4
// for 16-byte loads, and 4 mod 32 so the rows of a warp's 16-byte loads fall
// in different bank groups.
template <int D>
constexpr int kv_stride() { return D + 4; }

template <int DPL, int EPT>   // EPT: gradient elements per thread, >= bs * D / 256
__global__ void __launch_bounds__(kBwdKvThreads, 2)
bwd_kv_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
              const __nv_bfloat16* __restrict__ V, const __nv_bfloat16* __restrict__ dO,
              const float* __restrict__ lse, const float* __restrict__ delta,
              const int32_t* __restrict__ lists, const int32_t* __restrict__ offsets,
              const int32_t* __restrict__ counts, const int32_t* __restrict__ idx,
              float* __restrict__ dq_part, __nv_bfloat16* __restrict__ dK,
              __nv_bfloat16* __restrict__ dV, Shape s) {
  constexpr int D = DPL * 32;
  constexpr int KS = kv_stride<D>();
  // When bs * D is exactly 256 EPT (4096 or 8192), each thread owns a 4 x TC
  // tile of the block's gradient (rows 4 tr.., columns TC tc..), so one
  // 16-byte load of the weights and of the rows serves 4 TC multiply-adds;
  // otherwise it owns elements e = t + 256 m.
  constexpr bool kTiledEpt = (EPT == 16 || EPT == 32);
  constexpr int TC = EPT / 4;
  extern __shared__ float4 smem_v4[];
  float* smem_f = reinterpret_cast<float*>(smem_v4);
  const int j = blockIdx.x, u = blockIdx.y, t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int bs = s.bs;
  // Shared memory: K and V of the block, the batch's rows of Q and dO, their
  // weights, the rows' slots, the list.
  float* Kb = smem_f;                              // bs x KS
  float* Vb = Kb + bs * KS;                        // bs x KS
  float* qb = Vb + bs * KS;                        // kBwdBatch x D
  float* gb = qb + kBwdBatch * D;                  // kBwdBatch x D
  float* pb = gb + kBwdBatch * D;                  // kBwdBatch x bs
  float* db = pb + kBwdBatch * bs;                 // kBwdBatch x bs
  int32_t* slot_s = reinterpret_cast<int32_t*>(db + kBwdBatch * bs);   // kBwdBatch
  int32_t* lst = slot_s + kBwdBatch;                                    // kBwdSortCap
  const int64_t blk0 = (int64_t)u * s.N + (int64_t)j * bs;
  for (int e = t; e < bs * D; e += kBwdKvThreads) {
    const int r = e / D, d = e % D;
    Kb[r * KS + d] = __bfloat162float(K[(blk0 + r) * D + d]);
    Vb[r * KS + d] = __bfloat162float(V[(blk0 + r) * D + d]);
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
  const bool tiled = kTiledEpt && bs * D == kBwdKvThreads * EPT && bs % 4 == 0;
  const int tr = tiled ? t / (D / TC) : 0, tc = tiled ? t % (D / TC) : 0;
  const float sc = s.scale * 1.4426950408889634f;
  for (int b0 = 0; b0 < n; b0 += kBwdBatch) {
    // Warp w: row b0 + w of the list -- its Q and dO rows, its slot, then
    // the block's weights p and p (dp - delta) for that row (zero for a
    // missing row).
    const int i = b0 + warp;
    const int row = i < n ? (sorted ? lst[i] : lg[i]) : -1;
    float* qw = qb + warp * D;
    float* gw = gb + warp * D;
    for (int d = lane; d < D; d += 32) {
      qw[d] = row >= 0 ? __bfloat162float(Q[((int64_t)u * s.N + row) * D + d]) : 0.f;
      gw[d] = row >= 0 ? __bfloat162float(dO[((int64_t)u * s.N + row) * D + d]) : 0.f;
    }
    const float ls = row >= 0 ? lse[(int64_t)u * s.N + row] : 0.f;
    const float dl = row >= 0 ? delta[(int64_t)u * s.N + row] : 0.f;
    // The slot of this block in the row's selection: where its dQ share goes.
    int slot = -1;
    for (int q0 = 0; q0 < s.k; q0 += 32) {
      const int q = q0 + lane;
      const bool hit = row >= 0 && q < s.k && idx[((int64_t)u * s.N + row) * s.k + q] == j;
      const unsigned bits = __ballot_sync(0xffffffffu, hit);
      if (slot < 0 && bits != 0u) slot = q0 + __ffs(bits) - 1;
    }
    if (lane == 0) slot_s[warp] = row >= 0 ? slot : -1;
    __syncwarp();
    for (int r = lane; r < bs; r += 32) {
      float p = 0.f, ds = 0.f;
      if (row >= 0 && (!s.causal || j * bs + r <= row)) {
        float x = 0.f, dp = 0.f;
        const float4* kr = reinterpret_cast<const float4*>(Kb + r * KS);
        const float4* vr = reinterpret_cast<const float4*>(Vb + r * KS);
        const float4* q4 = reinterpret_cast<const float4*>(qw);
        const float4* g4 = reinterpret_cast<const float4*>(gw);
#pragma unroll 4
        for (int c = 0; c < D / 4; ++c) {
          const float4 kk = kr[c], vv = vr[c], qq = q4[c], gg = g4[c];
          x = fmaf(qq.x, kk.x, x); x = fmaf(qq.y, kk.y, x);
          x = fmaf(qq.z, kk.z, x); x = fmaf(qq.w, kk.w, x);
          dp = fmaf(gg.x, vv.x, dp); dp = fmaf(gg.y, vv.y, dp);
          dp = fmaf(gg.z, vv.z, dp); dp = fmaf(gg.w, vv.w, dp);
        }
        p = exp2f(x * sc - ls);
        ds = p * (dp - dl);
      }
      pb[warp * bs + r] = p;
      db[warp * bs + r] = ds;
    }
    __syncthreads();
    // dV[r][d] += p_w[r] dO_w[d], dK[r][d] += ds_w[r] Q_w[d], rows in order.
    if (kTiledEpt && tiled) {
#pragma unroll
      for (int w = 0; w < kBwdBatch; ++w) {
        const float4 p4 = *reinterpret_cast<const float4*>(pb + w * bs + 4 * tr);
        const float4 d4 = *reinterpret_cast<const float4*>(db + w * bs + 4 * tr);
        const float pr[4] = {p4.x, p4.y, p4.z, p4.w}, dr[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
        for (int c4 = 0; c4 < TC / 4; ++c4) {
          const float4 g = *reinterpret_cast<const float4*>(gb + w * D + TC * tc + 4 * c4);
          const float4 q = *reinterpret_cast<const float4*>(qb + w * D + TC * tc + 4 * c4);
          const float gc[4] = {g.x, g.y, g.z, g.w}, qc[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const int m = rr * TC + 4 * c4 + cc;
              gv[m] = fmaf(pr[rr], gc[cc], gv[m]);
              gk[m] = fmaf(dr[rr], qc[cc], gk[m]);
            }
          }
        }
      }
    } else {
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
    }
    // Each row's dQ share from this block, sum_r ds[r] K[r] (scaled later),
    // into the row's slot: warp w takes row w, each lane DPL columns.
    {
      const int sl = slot_s[warp];
      if (sl >= 0) {
        float acc[DPL];
#pragma unroll
        for (int c = 0; c < DPL; ++c) acc[c] = 0.f;
        const float* dw = db + warp * bs;
        for (int r = 0; r < bs; ++r) {
          const float w_r = dw[r];
#pragma unroll
          for (int c = 0; c < DPL; ++c) acc[c] = fmaf(w_r, Kb[r * KS + lane * DPL + c], acc[c]);
        }
        const int rw = sorted ? lst[b0 + warp] : lg[b0 + warp];
        float* dst = dq_part + (((int64_t)u * s.N + rw) * s.k + sl) * D + lane * DPL;
#pragma unroll
        for (int c = 0; c < DPL; ++c) dst[c] = acc[c];
      }
    }
    __syncthreads();
  }
  if (kTiledEpt && tiled) {
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
#pragma unroll
      for (int c = 0; c < TC; ++c) {
        const int64_t o = (blk0 + 4 * tr + rr) * D + TC * tc + c;
        dK[o] = __float2bfloat16(gk[rr * TC + c] * s.scale);
        dV[o] = __float2bfloat16(gv[rr * TC + c]);
      }
    }
  } else {
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
}

// The per-block kernel on tensor cores (mma.sync, bf16 in, fp32 out), for
// block_size 64 and head_dim 64: 32 rows of the block's list at a time.
//   S = Q K^T and dP = dO V^T (32 x 64): warp w the keys 8w .. 8w + 7;
//   P = 2^(S sc - lse), dS = P (dP - delta), rounded to bf16 as the
//   operands of the next products;
//   dV += P^T dO and dK += dS^T Q (64 x 64, kept in registers over the whole
//   list): warp w the keys 16 (w / 2) .., columns 32 (w % 2) ..;
//   dQ share = dS K (32 x 64): warp w the columns 8w .. 8w + 7.
// The operands sit in shared memory in the layouts the fragments read
// (rows padded by 8 elements against bank conflicts).  Rows in list
// order and the products' fixed order: the same result on every run.
namespace bwdmma {
constexpr int kMT = 2;          // 16-row tiles per batch
constexpr int kB = 16 * kMT;    // rows per batch
constexpr int kS64 = 72;        // row stride of 64-wide arrays (bf16)
constexpr int kS16 = kB + 8;    // row stride of kB-wide arrays (bf16)
__device__ __forceinline__ uint32_t ld32(const __nv_bfloat16* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}
__device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                    uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
}  // namespace bwdmma

__global__ void __launch_bounds__(kBwdKvThreads, 2)
bwd_kv_mma_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                  const __nv_bfloat16* __restrict__ V, const __nv_bfloat16* __restrict__ dO,
                  const float* __restrict__ lse, const float* __restrict__ delta,
                  const int32_t* __restrict__ lists, const int32_t* __restrict__ offsets,
                  const int32_t* __restrict__ counts, const int32_t* __restrict__ idx,
                  float* __restrict__ dq_part, __nv_bfloat16* __restrict__ dK,
                  __nv_bfloat16* __restrict__ dV, Shape s) {
  using namespace bwdmma;
  constexpr int D = 64, BS = 64;
  extern __shared__ float4 smem_v4[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(smem_v4);   // [key][d]
  __nv_bfloat16* KTs = Ks + BS * kS64;                              // [d][key]
  __nv_bfloat16* Vs = KTs + D * kS64;                               // [key][d]
  __nv_bfloat16* Qb = Vs + BS * kS64;                               // [row][d]
  __nv_bfloat16* Gb = Qb + kB * kS64;                               // [row][d]  (dO)
  __nv_bfloat16* DSr = Gb + kB * kS64;                              // [row][key]
  __nv_bfloat16* QT = DSr + kB * kS64;                              // [d][row]
  __nv_bfloat16* GT = QT + D * kS16;                                // [d][row]
  __nv_bfloat16* PT = GT + D * kS16;                                // [key][row]
  __nv_bfloat16* DST = PT + BS * kS16;                              // [key][row]
  float* ls_s = reinterpret_cast<float*>(DST + BS * kS16);          // [kB]
  float* dl_s = ls_s + kB;
  int32_t* row_s = reinterpret_cast<int32_t*>(dl_s + kB);
  int32_t* slot_s = row_s + kB;
  int32_t* lst = slot_s + kB;                                       // kBwdSortCap
  const int j = blockIdx.x, u = blockIdx.y, t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31, g = lane >> 2, q4 = lane & 3;
  const int64_t blk0 = (int64_t)u * s.N + (int64_t)j * BS;
  for (int e = t; e < BS * D / 2; e += kBwdKvThreads) {
    const int r = (2 * e) / D, d = (2 * e) % D;
    const __nv_bfloat162 kk = *reinterpret_cast<const __nv_bfloat162*>(K + (blk0 + r) * D + d);
    const __nv_bfloat162 vv = *reinterpret_cast<const __nv_bfloat162*>(V + (blk0 + r) * D + d);
    *reinterpret_cast<__nv_bfloat162*>(Ks + r * kS64 + d) = kk;
    *reinterpret_cast<__nv_bfloat162*>(Vs + r * kS64 + d) = vv;
    KTs[d * kS64 + r] = kk.x;
    KTs[(d + 1) * kS64 + r] = kk.y;
  }
  const int n = counts[(int64_t)u * s.nb + j];
  const int32_t* lg = lists + (int64_t)u * s.N * s.k + offsets[(int64_t)u * s.nb + j];
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
  const float sc = s.scale * 1.4426950408889634f;
  const int mt = warp >> 1, nh = warp & 1;   // dK/dV tile of this warp
  float accV[4][4], accK[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) accV[a][c] = accK[a][c] = 0.f;
  for (int b0 = 0; b0 < n; b0 += kB) {
    // Rows kB/8 w .. of the batch: Q and dO in both layouts, log-sum-exp,
    // delta and the slot of this block (-1 for a missing row).
#pragma unroll
    for (int h = 0; h < kB / 8; ++h) {
      const int r = (kB / 8) * warp + h;
      const int i = b0 + r;
      const int row = i < n ? (sorted ? lst[i] : lg[i]) : -1;
      const int64_t R = (int64_t)u * s.N + (row >= 0 ? row : 0);
      __nv_bfloat162 qq = __floats2bfloat162_rn(0.f, 0.f), gg = qq;
      if (row >= 0) {
        qq = *reinterpret_cast<const __nv_bfloat162*>(Q + R * D + 2 * lane);
        gg = *reinterpret_cast<const __nv_bfloat162*>(dO + R * D + 2 * lane);
      }
      *reinterpret_cast<__nv_bfloat162*>(Qb + r * kS64 + 2 * lane) = qq;
      *reinterpret_cast<__nv_bfloat162*>(Gb + r * kS64 + 2 * lane) = gg;
      QT[(2 * lane) * kS16 + r] = qq.x;
      QT[(2 * lane + 1) * kS16 + r] = qq.y;
      GT[(2 * lane) * kS16 + r] = gg.x;
      GT[(2 * lane + 1) * kS16 + r] = gg.y;
      int slot = -1;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int q = lane + 32 * hh;
        const bool hit = row >= 0 && q < s.k && idx[R * s.k + q] == j;
        const unsigned bits = __ballot_sync(0xffffffffu, hit);
        if (slot < 0 && bits != 0u) slot = 32 * hh + __ffs(bits) - 1;
      }
      if (lane == 0) {
        row_s[r] = row;
        slot_s[r] = row >= 0 ? slot : -1;
        ls_s[r] = row >= 0 ? lse[R] : 0.f;
        dl_s[r] = row >= 0 ? delta[R] : 0.f;
      }
    }
    __syncthreads();
    // S and dP for keys 8w .. 8w + 7, each 16-row tile of the batch.
#pragma unroll
    for (int m = 0; m < kMT; ++m) {
      const __nv_bfloat16* qa = Qb + (16 * m) * kS64;
      const __nv_bfloat16* ga = Gb + (16 * m) * kS64;
      float sacc[4] = {0.f, 0.f, 0.f, 0.f}, pacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int c0 = 16 * ks + 2 * q4;
        const uint32_t a0 = ld32(qa + g * kS64 + c0), a1 = ld32(qa + (g + 8) * kS64 + c0);
        const uint32_t a2 = ld32(qa + g * kS64 + c0 + 8), a3 = ld32(qa + (g + 8) * kS64 + c0 + 8);
        mma(sacc, a0, a1, a2, a3, ld32(Ks + (8 * warp + g) * kS64 + c0),
            ld32(Ks + (8 * warp + g) * kS64 + c0 + 8));
        const uint32_t e0 = ld32(ga + g * kS64 + c0), e1 = ld32(ga + (g + 8) * kS64 + c0);
        const uint32_t e2 = ld32(ga + g * kS64 + c0 + 8), e3 = ld32(ga + (g + 8) * kS64 + c0 + 8);
        mma(pacc, e0, e1, e2, e3, ld32(Vs + (8 * warp + g) * kS64 + c0),
            ld32(Vs + (8 * warp + g) * kS64 + c0 + 8));
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int r = 16 * m + g + 8 * (c >> 1), key = 8 * warp + 2 * q4 + (c & 1);
        const int row = row_s[r];
        float p = 0.f, ds = 0.f;
        if (row >= 0 && (!s.causal || j * BS + key <= row)) {
          p = exp2f(sacc[c] * sc - ls_s[r]);
          ds = p * (pacc[c] - dl_s[r]);
        }
        const __nv_bfloat16 pb = __float2bfloat16(p), db = __float2bfloat16(ds);
        PT[key * kS16 + r] = pb;
        DST[key * kS16 + r] = db;
        DSr[r * kS64 + key] = db;
      }
    }
    __syncthreads();
    // dV += P^T dO, dK += dS^T Q over this batch's rows (16 at a time).
#pragma unroll
    for (int kk = 0; kk < kMT; ++kk) {
      const int k0 = 16 * kk + 2 * q4;
      const __nv_bfloat16* pa = PT + (16 * mt) * kS16;
      const __nv_bfloat16* da = DST + (16 * mt) * kS16;
      const uint32_t p0 = ld32(pa + g * kS16 + k0), p1 = ld32(pa + (g + 8) * kS16 + k0);
      const uint32_t p2 = ld32(pa + g * kS16 + k0 + 8), p3 = ld32(pa + (g + 8) * kS16 + k0 + 8);
      const uint32_t d0 = ld32(da + g * kS16 + k0), d1 = ld32(da + (g + 8) * kS16 + k0);
      const uint32_t d2 = ld32(da + g * kS16 + k0 + 8), d3 = ld32(da + (g + 8) * kS16 + k0 + 8);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int nt = 4 * nh + a;
        mma(accV[a], p0, p1, p2, p3, ld32(GT + (8 * nt + g) * kS16 + k0),
            ld32(GT + (8 * nt + g) * kS16 + k0 + 8));
        mma(accK[a], d0, d1, d2, d3, ld32(QT + (8 * nt + g) * kS16 + k0),
            ld32(QT + (8 * nt + g) * kS16 + k0 + 8));
      }
    }
    // This block's dQ share of each row, columns 8w .. 8w + 7, into its slot.
#pragma unroll
    for (int m = 0; m < kMT; ++m) {
      const __nv_bfloat16* sa = DSr + (16 * m) * kS64;
      float qacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < BS / 16; ++ks) {
        const int c0 = 16 * ks + 2 * q4;
        mma(qacc, ld32(sa + g * kS64 + c0), ld32(sa + (g + 8) * kS64 + c0),
            ld32(sa + g * kS64 + c0 + 8), ld32(sa + (g + 8) * kS64 + c0 + 8),
            ld32(KTs + (8 * warp + g) * kS64 + c0), ld32(KTs + (8 * warp + g) * kS64 + c0 + 8));
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = 16 * m + g + 8 * h;
        const int sl = slot_s[r];
        if (sl >= 0) {
          float* dst = dq_part + (((int64_t)u * s.N + row_s[r]) * s.k + sl) * D + 8 * warp + 2 * q4;
          *reinterpret_cast<float2*>(dst) = make_float2(qacc[2 * h], qacc[2 * h + 1]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int col = 8 * (4 * nh + a) + 2 * q4;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t o = (blk0 + 16 * mt + g + 8 * h) * D + col;
      *reinterpret_cast<__nv_bfloat162*>(dK + o) =
          __floats2bfloat162_rn(accK[a][2 * h] * s.scale, accK[a][2 * h + 1] * s.scale);
      *reinterpret_cast<__nv_bfloat162*>(dV + o) =
          __floats2bfloat162_rn(accV[a][2 * h], accV[a][2 * h + 1]);
    }
  }
}

// Log-sum-exp on the key-block side (block_size 64, head_dim 64): per
// (unit, key block), for every row of its list, the block's share of the
// row's softmax normaliser -- the maximum m of its 64 scores (base 2) and
// l = sum 2^(x - m) -- into the row's slot; S = Q K^T on tensor cores as in
// bwd_kv_mma_kernel.  bwd_lse_merge_kernel then merges a row's shares.  Each
// share is written once, so the list's order does not matter here.
__global__ void __launch_bounds__(kBwdKvThreads, 2)
bwd_lse_mma_kernel(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                   const int32_t* __restrict__ lists, const int32_t* __restrict__ offsets,
                   const int32_t* __restrict__ counts, const int32_t* __restrict__ idx,
                   float2* __restrict__ ml_part, Shape s) {
  using namespace bwdmma;
  constexpr int D = 64, BS = 64;
  __shared__ __align__(16) __nv_bfloat16 Ks[BS * kS64], Qb[kB * kS64];
  __shared__ float wm[8 * kB], wl[8 * kB];
  __shared__ int32_t row_s[kB], slot_s[kB];
  const int j = blockIdx.x, u = blockIdx.y, t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31, g = lane >> 2, q4 = lane & 3;
  const int64_t blk0 = (int64_t)u * s.N + (int64_t)j * BS;
  for (int e = t; e < BS * D / 2; e += kBwdKvThreads) {
    const int r = (2 * e) / D, d = (2 * e) % D;
    *reinterpret_cast<__nv_bfloat162*>(Ks + r * kS64 + d) =
        *reinterpret_cast<const __nv_bfloat162*>(K + (blk0 + r) * D + d);
  }
  const int n = counts[(int64_t)u * s.nb + j];
  const int32_t* lg = lists + (int64_t)u * s.N * s.k + offsets[(int64_t)u * s.nb + j];
  const float sc = s.scale * 1.4426950408889634f;
  for (int b0 = 0; b0 < n; b0 += kB) {
#pragma unroll
    for (int h = 0; h < kB / 8; ++h) {
      const int r = (kB / 8) * warp + h;
      const int i = b0 + r;
      const int row = i < n ? lg[i] : -1;
      const int64_t R = (int64_t)u * s.N + (row >= 0 ? row : 0);
      __nv_bfloat162 qq = __floats2bfloat162_rn(0.f, 0.f);
      if (row >= 0) qq = *reinterpret_cast<const __nv_bfloat162*>(Q + R * D + 2 * lane);
      *reinterpret_cast<__nv_bfloat162*>(Qb + r * kS64 + 2 * lane) = qq;
      int slot = -1;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int q = lane + 32 * hh;
        const bool hit = row >= 0 && q < s.k && idx[R * s.k + q] == j;
        const unsigned bits = __ballot_sync(0xffffffffu, hit);
        if (slot < 0 && bits != 0u) slot = 32 * hh + __ffs(bits) - 1;
      }
      if (lane == 0) {
        row_s[r] = row;
        slot_s[r] = row >= 0 ? slot : -1;
      }
    }
    __syncthreads();
#pragma unroll
    for (int mm = 0; mm < kMT; ++mm) {
      const __nv_bfloat16* qa = Qb + (16 * mm) * kS64;
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int c0 = 16 * ks + 2 * q4;
        mma(sacc, ld32(qa + g * kS64 + c0), ld32(qa + (g + 8) * kS64 + c0),
            ld32(qa + g * kS64 + c0 + 8), ld32(qa + (g + 8) * kS64 + c0 + 8),
            ld32(Ks + (8 * warp + g) * kS64 + c0), ld32(Ks + (8 * warp + g) * kS64 + c0 + 8));
      }
      // Per row (g and g + 8 of this tile) this warp's 8 keys: maximum, sum.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = 16 * mm + g + 8 * h;
        const int row = row_s[r];
        float x[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int key = 8 * warp + 2 * q4 + c;
          const bool live = row >= 0 && (!s.causal || j * BS + key <= row);
          x[c] = live ? sacc[2 * h + c] * sc : -INFINITY;
        }
        float m = fmaxf(x[0], x[1]);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        float l = m == -INFINITY ? 0.f : exp2f(x[0] - m) + exp2f(x[1] - m);
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        if (q4 == 0) {
          wm[warp * kB + r] = m;
          wl[warp * kB + r] = l;
        }
      }
    }
    __syncthreads();
    if (t < kB) {
      const int row = row_s[t], sl = slot_s[t];
      if (row >= 0 && sl >= 0) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w * kB + t]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w)
          L += wm[w * kB + t] == -INFINITY ? 0.f : wl[w * kB + t] * exp2f(wm[w * kB + t] - M);
        ml_part[((int64_t)u * s.N + row) * s.k + sl] = make_float2(M, L);
      }
    }
    __syncthreads();
  }
}

// Per row (a warp): the log-sum-exp from its slots' shares, and delta =
// dO . O from the forward's O.
template <int DPL>
__global__ void __launch_bounds__(kBwdRowsWarps * 32)
bwd_lse_merge_kernel(const float2* __restrict__ ml_part, const int32_t* __restrict__ idx,
                     const __nv_bfloat16* __restrict__ O, const __nv_bfloat16* __restrict__ dO,
                     float* __restrict__ lse_out, float* __restrict__ delta_out, Shape s) {
  constexpr int D = DPL * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t R = ((int64_t)blockIdx.x * kBwdRowsWarps + warp);
  if (R >= (int64_t)s.units * s.N) return;   // whole warp
  float od[DPL], gd[DPL];
  load_cols<DPL>(O + R * D, lane, od);
  load_cols<DPL>(dO + R * D, lane, gd);
  float dl = 0.f;
#pragma unroll
  for (int c = 0; c < DPL; ++c) dl = fmaf(gd[c], od[c], dl);
  const float delta = warp_sum(dl);
  float2 ml[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int q = lane + 32 * h;
    const bool live = q < s.k && idx[R * s.k + q] >= 0;
    ml[h] = live ? ml_part[R * s.k + q] : make_float2(-INFINITY, 0.f);
  }
  const float M = warp_max(fmaxf(ml[0].x, ml[1].x));
  float L = 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) L += ml[h].x == -INFINITY ? 0.f : ml[h].y * exp2f(ml[h].x - M);
  L = warp_sum(L);
  if (lane == 0) {
    lse_out[R] = M + log2f(L);
    delta_out[R] = delta;
  }
}

static size_t bwd_kv_mma_smem() {
  using namespace bwdmma;
  return sizeof(__nv_bfloat16) * (3 * 64 * kS64 + 3 * kB * kS64 + 4 * 64 * kS16) +
         sizeof(float) * 2 * kB + sizeof(int32_t) * (2 * kB + kBwdSortCap);
}

// dQ of each row: the sum of its slots' shares (slots in order), scaled.
// D / 4 threads per row, four columns each.
__global__ void __launch_bounds__(256)
bwd_dq_kernel(const float* __restrict__ dq_part, const int32_t* __restrict__ idx,
              __nv_bfloat16* __restrict__ dQ, Shape s) {
  const int ch = s.D / 4;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t R = g / ch;
  if (R >= (int64_t)s.units * s.N) return;
  const int c = (int)(g % ch);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q = 0; q < s.k; ++q) {
    if (idx[R * s.k + q] < 0) continue;
    const float4 v = reinterpret_cast<const float4*>(dq_part + (R * s.k + q) * s.D)[c];
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  __nv_bfloat16* o = dQ + R * s.D + 4 * c;
  o[0] = __float2bfloat16(acc.x * s.scale);
  o[1] = __float2bfloat16(acc.y * s.scale);
  o[2] = __float2bfloat16(acc.z * s.scale);
  o[3] = __float2bfloat16(acc.w * s.scale);
}

bool backward_supported(const Shape& s) {
  return (s.D == 32 || s.D == 64 || s.D == 96 || s.D == 128) && s.bs * s.D <= 8192 &&
         s.k <= 64 && s.nb <= 16384 && (int64_t)s.units * s.N * s.k < (1LL << 31);
}

static size_t bwd_kv_smem(const Shape& s) {
  return sizeof(float) * (2 * (size_t)s.bs * (s.D + 4) + 2 * (size_t)kBwdBatch * s.D +
                          2 * (size_t)kBwdBatch * s.bs) +
         sizeof(int32_t) * (kBwdBatch + kBwdSortCap);
}

// Workspace: the fine stage's (bucket lists), then per row its log-sum-exp
// and delta, then per (row, slot) the dQ share (fp32).
static size_t a256b(size_t x) { return (x + 255) & ~(size_t)255; }

size_t backward_workspace_bytes(const Shape& s) {
  const size_t rows = (size_t)s.units * s.N;
  return fine_kv_workspace_bytes(s) + a256b(2 * rows * sizeof(float)) +
         a256b(rows * s.k * s.D * sizeof(float));
}

template <int DPL, int EPT>
static cudaError_t launch_bwd_kv(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                 const __nv_bfloat16* V, const __nv_bfloat16* dO,
                                 const float* lse, const float* delta, const BucketLists& bl,
                                 const int32_t* idx, float* dq_part, __nv_bfloat16* dK,
                                 __nv_bfloat16* dV, const Shape& s, cudaStream_t st) {
  const size_t smem = bwd_kv_smem(s);
  cudaError_t e = cudaFuncSetAttribute(bwd_kv_kernel<DPL, EPT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  bwd_kv_kernel<DPL, EPT><<<dim3(s.nb, s.units), kBwdKvThreads, smem, st>>>(
      Q, K, V, dO, lse, delta, bl.lists, bl.offsets, bl.counts, idx, dq_part, dK, dV, s);
  return cudaGetLastError();
}

template <int DPL>
static cudaError_t launch_bwd(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                              const __nv_bfloat16* V, const __nv_bfloat16* O,
                              const __nv_bfloat16* dO, const int32_t* idx, __nv_bfloat16* dQ,
                              __nv_bfloat16* dK, __nv_bfloat16* dV, unsigned char* ws,
                              const Shape& s, cudaStream_t st) {
  const size_t rows = (size_t)s.units * s.N;
  float* lse = reinterpret_cast<float*>(ws + fine_kv_workspace_bytes(s));
  float* delta = lse + rows;
  float* dq_part = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(lse) +
                                            a256b(2 * rows * sizeof(float)));
  const bool mma_path = (s.bs == 64 && s.D == 64);
  cudaError_t e;
  if (!mma_path) {
    dim3 g1((s.N + kBwdRowsWarps - 1) / kBwdRowsWarps, s.units);
    bwd_lse_kernel<DPL><<<g1, kBwdRowsWarps * 32, 0, st>>>(Q, K, O, dO, idx, lse, delta, s);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  BucketLists bl;
  if ((e = launch_bucket_lists(idx, V, ws, s, st, &bl)) != cudaSuccess) return e;
  if (mma_path) {
    // The rows' log-sum-exp from the key-block side: shares per (row, slot),
    // held in the dQ-share array until the per-block pass overwrites it.
    float2* ml_part = reinterpret_cast<float2*>(dq_part);
    bwd_lse_mma_kernel<<<dim3(s.nb, s.units), kBwdKvThreads, 0, st>>>(
        Q, K, bl.lists, bl.offsets, bl.counts, idx, ml_part, s);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const unsigned g2 = (unsigned)((rows + kBwdRowsWarps - 1) / kBwdRowsWarps);
    bwd_lse_merge_kernel<DPL><<<g2, kBwdRowsWarps * 32, 0, st>>>(ml_part, idx, O, dO, lse, delta,
                                                                 s);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const int elems = s.bs * s.D;
  if (s.bs == 64 && s.D == 64) {
    const size_t smem = bwd_kv_mma_smem();
    if ((e = cudaFuncSetAttribute(bwd_kv_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem)) != cudaSuccess)
      return e;
    bwd_kv_mma_kernel<<<dim3(s.nb, s.units), kBwdKvThreads, smem, st>>>(
        Q, K, V, dO, lse, delta, bl.lists, bl.offsets, bl.counts, idx, dq_part, dK, dV, s);
    e = cudaGetLastError();
  } else if (elems <= 256) e = launch_bwd_kv<DPL, 1>(Q, K, V, dO, lse, delta, bl, idx, dq_part, dK, dV, s, st);
  else if (elems <= 512) e = launch_bwd_kv<DPL, 2>(Q, K, V, dO, lse, delta, bl, idx, dq_part, dK, dV, s, st);
  else if (elems <= 1024) e = launch_bwd_kv<DPL, 4>(Q, K, V, dO, lse, delta, bl, idx, dq_part, dK, dV, s, st);
  else if (elems <= 2048) e = launch_bwd_kv<DPL, 8>(Q, K, V, dO, lse, delta, bl, idx, dq_part, dK, dV, s, st);
  else if (elems <= 4096) e = launch_bwd_kv<DPL, 16>(Q, K, V, dO, lse, delta, bl, idx, dq_part, dK, dV, s, st);
  else e = launch_bwd_kv<DPL, 32>(Q, K, V, dO, lse, delta, bl, idx, dq_part, dK, dV, s, st);
  if (e != cudaSuccess) return e;
  const int64_t threads = (int64_t)rows * (s.D / 4);
  bwd_dq_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(dq_part, idx, dQ, s);
  return cudaGetLastError();
}

cudaError_t launch_backward(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                            const __nv_bfloat16* V, const __nv_bfloat16* O,
                            const __nv_bfloat16* dO, const int32_t* idx, __nv_bfloat16* dQ,
                            __nv_bfloat16* dK, __nv_bfloat16* dV, unsigned char* ws,
                            const Shape& s, cudaStream_t st) {
  switch (s.D) {
    case 32: return launch_bwd<1>(Q, K, V, O, dO, idx, dQ, dK, dV, ws, s, st);
    case 64: return launch_bwd<2>(Q, K, V, O, dO, idx, dQ, dK, dV, ws, s, st);
    case 96: return launch_bwd<3>(Q, K, V, O, dO, idx, dQ, dK, dV, ws, s, st);
    case 128: return launch_bwd<4>(Q, K, V, O, dO, idx, dQ, dK, dV, ws, s, st);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace bsa
