// Per-row streaming top-k with lowest-index tie break (block_indexer.py:53).
//
// One thread owns one query row.  Candidates arrive in ascending block order.
// A candidate is appended to the thread's buffer -- a column of shared memory
// holding packed (score bits, block index) pairs, so a warp's appends are
// bank-conflict free -- only if it can still be in the final top-k:
//   * x > theta_excl, the exact k-th largest value among the candidates seen
//     so far (a later candidate equal to it loses the tie to the earlier,
//     lower-index one), and
//   * x >= theta_incl, a lower bound of the final k-th largest value known
//     from elsewhere (e.g. k distinct group maxima of the row).
// When the buffer is about to overflow it is compacted to its exact top-k
// (values only, a 2*KCAP-op min/max insertion network per entry), which also
// raises theta_excl.  Compaction keeps buffer order, so ties keep resolving
// to the lowest index, and the final emission lists the selected blocks in
// ascending block order (the fine stage needs no particular order).  -inf
// candidates (causally masked blocks) never enter the buffer, so rows with
// fewer than k eligible blocks emit -1 in the remaining slots.
#pragma once

#include "common.cuh"

namespace bsa {

// Bitonic sort of 32 values, descending, in registers.
__device__ __forceinline__ void sort32_desc(float (&v)[32]) {
#pragma unroll
  for (int k2 = 2; k2 <= 32; k2 <<= 1) {
#pragma unroll
    for (int j = k2 >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const float a = v[i], b = v[l];
          const float hi = fmaxf(a, b), lo = fminf(a, b);
          if ((i & k2) == 0) { v[i] = hi; v[l] = lo; } else { v[i] = lo; v[l] = hi; }
        }
      }
    }
  }
}

template <int KCAP>
struct RowTopK {
  uint2* buf;         // this thread's column: buf[slot * stride]
  int stride;
  int cap;            // buffer slots
  int cnt;
  int k;
  float theta_excl;
  float theta_incl;
  float thr;          // passes(x) <=> x >= thr: max(theta_incl, the float after theta_excl)

  __device__ __forceinline__ void init(uint2* b, int stride_, int cap_, int k_) {
    buf = b;
    stride = stride_;
    cap = cap_;
    cnt = 0;
    k = k_;
    theta_excl = -INFINITY;
    theta_incl = -INFINITY;
    update_thr();
  }

  // x > theta_excl is x >= (the next float above theta_excl) for every
  // non-NaN x (for theta_excl = -inf that is -FLT_MAX, so -inf never passes).
  __device__ __forceinline__ void update_thr() {
    thr = fmaxf(theta_incl, nextafterf(theta_excl, INFINITY));
  }

  __device__ __forceinline__ bool passes(float x) const { return x >= thr; }

  // Append unconditionally (the caller checked passes()).
  __device__ __forceinline__ void append(float x, int32_t j) {
    buf[cnt * stride] = make_uint2(__float_as_uint(x), (uint32_t)j);
    ++cnt;
  }

  // Append x[i] (block j0 + i) for every set bit i of pm, in ascending i (the
  // caller reserved room).  The four 8-bit parts of pm are four independent
  // store chains, each starting where the parts below it end, instead of
  // one chain of 32 dependent steps.  The buffer is in shared memory.
  __device__ __forceinline__ void append_mask(const float (&x)[32], uint32_t pm, int32_t j0) {
    const uint32_t step = (uint32_t)stride * (uint32_t)sizeof(uint2);
    uint32_t a[4];
    a[0] = (uint32_t)__cvta_generic_to_shared(buf) + (uint32_t)cnt * step;
    a[1] = a[0] + (uint32_t)__popc(pm & 0x000000ffu) * step;
    a[2] = a[1] + (uint32_t)__popc(pm & 0x0000ff00u) * step;
    a[3] = a[2] + (uint32_t)__popc(pm & 0x00ff0000u) * step;
    // Program order interleaves the chains (the stores are volatile).
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int i = 8 * g + ii;
        if ((pm >> i) & 1u) {
          asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(a[g]),
                       "r"(__float_as_uint(x[i])), "r"((uint32_t)(j0 + i))
                       : "memory");
          a[g] += step;
        }
      }
    }
    cnt += __popc(pm);
  }

  __device__ __forceinline__ void push(float x, int32_t j) {
    if (passes(x)) append(x, j);
  }

  // Make room for `incoming` more pushes.
  __device__ __forceinline__ void reserve(int incoming) {
    if (cnt + incoming > cap) compact();
  }

  __device__ __forceinline__ void raise_floor(float lower_bound) {
    theta_incl = fmaxf(theta_incl, lower_bound);
    update_thr();
  }

  // Exact k-th largest value of the buffer: the KCAP largest values kept
  // in descending registers.  Inserting x sets a[p] = max(a[p], min(a[p-1],
  // x)) from the old a[p-1] (a[0] = max(a[0], x)): 2 ops per cell, and no
  // cell waits for another, so an entry's update is two ops deep.  A buffer
  // of at most 32 entries is sorted instead (a 32-value bitonic network,
  // 480 min/max, fewer than the insertions once it holds ~16 entries).
  __device__ __forceinline__ float kth_value(int* n_gt_out) const {
    if (cnt <= 32) {
      float v[32];
#pragma unroll
      for (int e = 0; e < 32; ++e)
        v[e] = e < cnt ? __uint_as_float(buf[e * stride].x) : -INFINITY;
      sort32_desc(v);
      float T = INFINITY;
      int n_gt = 0;
#pragma unroll
      for (int p = 0; p < 32; ++p) T = fminf(T, p < k ? v[p] : INFINITY);
#pragma unroll
      for (int p = 0; p < 32; ++p) n_gt += (p < k && v[p] > T) ? 1 : 0;
      *n_gt_out = n_gt;
      return T;
    }
    float a[KCAP];
#pragma unroll
    for (int p = 0; p < KCAP; ++p) a[p] = -INFINITY;
#pragma unroll 4
    for (int e = 0; e < cnt; ++e) {
      const float x = __uint_as_float(buf[e * stride].x);
#pragma unroll
      for (int p = KCAP - 1; p >= 1; --p) a[p] = fmaxf(a[p], fminf(a[p - 1], x));
      a[0] = fmaxf(a[0], x);
    }
    float T = INFINITY;
    int n_gt = 0;
#pragma unroll
    for (int p = 0; p < KCAP; ++p) T = fminf(T, p < k ? a[p] : INFINITY);
#pragma unroll
    for (int p = 0; p < KCAP; ++p) n_gt += (p < k && a[p] > T) ? 1 : 0;
    *n_gt_out = n_gt;
    return T;
  }

  // Reduce the buffer to its exact top-k, in buffer (= ascending index) order.
  __device__ __forceinline__ void compact() {
    int n_gt;
    const float T = kth_value(&n_gt);
    int keep_eq = k - n_gt;
    int w = 0;
    // Four entries are read before any is written back: every write goes at
    // or below the entry being read, so no unread entry is overwritten.
#pragma unroll 1
    for (int e0 = 0; e0 < cnt; e0 += 4) {
      uint2 en[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        en[q] = e0 + q < cnt ? buf[(e0 + q) * stride] : make_uint2(0xff800000u, 0u);  // -inf
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float v = __uint_as_float(en[q].x);
        const bool live = e0 + q < cnt;
        const bool eq = live && !(v > T) && (v == T) && keep_eq > 0;
        const bool take = live && (v > T || eq);
        keep_eq -= eq ? 1 : 0;
        if (take) {
          buf[w * stride] = en[q];
          ++w;
        }
      }
    }
    cnt = w;
    theta_excl = fmaxf(theta_excl, T);
    update_thr();
  }

  // Final top-k, written as `slots` (>= k) int32 in ascending block order,
  // -1 padded (16-byte stores when slots is a multiple of 4 and out is
  // 16-byte aligned).
  __device__ __forceinline__ void emit(int32_t* out, int slots) {
    compact();
    auto at = [&](int e) { return e < cnt ? (int32_t)buf[e * stride].y : -1; };
    if ((slots & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      for (int e = 0; e < slots; e += 4)
        *reinterpret_cast<int4*>(out + e) = make_int4(at(e), at(e + 1), at(e + 2), at(e + 3));
    } else {
      for (int e = 0; e < slots; ++e) out[e] = at(e);
    }
  }
};

// Buffer slots per thread for a given KCAP: room for the top-k plus at least
// two 32-candidate chunks between compactions.
__host__ __device__ constexpr int topk_buffer_slots(int kcap) {
  return kcap <= 32 ? 2 * kcap + 32 : kcap + 64;
}

// 16th largest of 32 values: the halves sorted in opposite directions (two
// 16-value bitonic networks) form a bitonic sequence whose pairwise maxima
// (i, i + 16) are its 16 largest values; their minimum.  351 min/max
// against 496 for the whole sort.
__device__ __forceinline__ float kth16_of_32(float (&v)[32]) {
#pragma unroll
  for (int k2 = 2; k2 <= 16; k2 <<= 1) {
#pragma unroll
    for (int j = k2 >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const float a = v[i], b = v[l];
          const float hi = fmaxf(a, b), lo = fminf(a, b);
          // the full sort's first stages: after k2 = 16 the first half is
          // descending and the second ascending
          if ((i & k2) == 0) { v[i] = hi; v[l] = lo; } else { v[i] = lo; v[l] = hi; }
        }
      }
    }
  }
  float T = INFINITY;
#pragma unroll
  for (int i = 0; i < 16; ++i) T = fminf(T, fmaxf(v[i], v[16 + i]));
  return T;
}

// k-th largest of 32 values (1 <= k <= 32): bitonic sort, descending, in
// registers; returns the min of the first k.
__device__ __forceinline__ float kth_of_32(float (&v)[32], int k) {
#pragma unroll
  for (int k2 = 2; k2 <= 32; k2 <<= 1) {
#pragma unroll
    for (int j = k2 >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const float a = v[i], b = v[l];
          const float hi = fmaxf(a, b), lo = fminf(a, b);
          if ((i & k2) == 0) { v[i] = hi; v[l] = lo; } else { v[i] = lo; v[l] = hi; }
        }
      }
    }
  }
  float T = INFINITY;
#pragma unroll
  for (int p = 0; p < 32; ++p) T = fminf(T, p < k ? v[p] : INFINITY);
  return T;
}

// k-th largest of the 64 values lo[0..32) and hi[0..32) (1 <= k <= 64):
// bitonic sort of the 64 values, descending, in registers (lo then hi); the
// min of the first k.
__device__ __forceinline__ float kth_of_64(float (&lo)[32], float (&hi)[32], int k) {
  float v[64];
#pragma unroll
  for (int i = 0; i < 32; ++i) { v[i] = lo[i]; v[32 + i] = hi[i]; }
#pragma unroll
  for (int k2 = 2; k2 <= 64; k2 <<= 1) {
#pragma unroll
    for (int j = k2 >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const float a = v[i], b = v[l];
          const float hv = fmaxf(a, b), lv = fminf(a, b);
          if ((i & k2) == 0) { v[i] = hv; v[l] = lv; } else { v[i] = lv; v[l] = hv; }
        }
      }
    }
  }
  float T = INFINITY;
#pragma unroll
  for (int p = 0; p < 64; ++p) T = fminf(T, p < k ? v[p] : INFINITY);
  return T;
}

}  // namespace bsa
