// Per-row streaming top-k with lowest-index tie break (block_indexer.py:53).
//
// One thread owns one query row.  Candidates arrive in ascending block order.
// A candidate is appended to the thread's buffer (a column of shared memory,
// so a warp's appends are bank-conflict free) only if it can still be in the
// final top-k:
//   * x > theta_excl, the exact k-th largest value among the candidates seen
//     so far (a later candidate equal to it loses the tie to the earlier,
//     lower-index one), and
//   * x >= theta_incl, a lower bound of the final k-th largest value known
//     from elsewhere (e.g. k distinct group maxima of the row).
// When the buffer is about to overflow it is compacted to its exact top-k
// (values only, a 2*KCAP-op min/max insertion network per entry), which also
// raises theta_excl.  Compaction keeps buffer order, so ties keep resolving
// to the lowest index, and the final emission lists the selected blocks in
// ascending block order.  -inf candidates (causally masked blocks) never
// enter the buffer, so rows with fewer than k eligible blocks emit -1 in the
// remaining slots.
#pragma once

#include "common.cuh"

namespace bsa {

template <int KCAP>
struct RowTopK {
  float* bval;        // this thread's column: bval[slot * stride]
  int32_t* bidx;
  int stride;
  int cap;            // buffer slots
  int cnt;
  int k;
  float theta_excl;
  float theta_incl;

  __device__ __forceinline__ void init(float* v, int32_t* i, int stride_, int cap_, int k_) {
    bval = v;
    bidx = i;
    stride = stride_;
    cap = cap_;
    cnt = 0;
    k = k_;
    theta_excl = -INFINITY;
    theta_incl = -INFINITY;
  }

  __device__ __forceinline__ void push(float x, int32_t j) {
    if (x > theta_excl && x >= theta_incl) {
      bval[cnt * stride] = x;
      bidx[cnt * stride] = j;
      ++cnt;
    }
  }

  // Make room for `incoming` more pushes.
  __device__ __forceinline__ void reserve(int incoming) {
    if (cnt + incoming > cap) compact();
  }

  __device__ __forceinline__ void raise_floor(float lower_bound) {
    theta_incl = fmaxf(theta_incl, lower_bound);
  }

  // Reduce the buffer to its exact top-k, in buffer (= ascending index) order.
  __device__ void compact() {
    float a[KCAP];
#pragma unroll
    for (int p = 0; p < KCAP; ++p) a[p] = -INFINITY;
    for (int e = 0; e < cnt; ++e) {
      float x = bval[e * stride];
#pragma unroll
      for (int p = 0; p < KCAP; ++p) {
        float hi = fmaxf(a[p], x);
        x = fminf(a[p], x);
        a[p] = hi;
      }
    }
    float T = -INFINITY;
    int n_gt = 0;
#pragma unroll
    for (int p = 0; p < KCAP; ++p) {
      if (p == k - 1) T = a[p];
    }
#pragma unroll
    for (int p = 0; p < KCAP; ++p) n_gt += (p < k && a[p] > T) ? 1 : 0;
    int keep_eq = k - n_gt;
    int w = 0;
    for (int e = 0; e < cnt; ++e) {
      float v = bval[e * stride];
      int32_t j = bidx[e * stride];
      bool take = v > T;
      if (!take && v == T && keep_eq > 0) {
        take = true;
        --keep_eq;
      }
      if (take) {
        bval[w * stride] = v;
        bidx[w * stride] = j;
        ++w;
      }
    }
    cnt = w;
    theta_excl = fmaxf(theta_excl, T);
  }

  // Final top-k, written as k int32 (ascending block order, -1 padded).
  __device__ __forceinline__ void emit(int32_t* out) {
    compact();
    for (int s = 0; s < k; ++s) out[s] = s < cnt ? bidx[s * stride] : -1;
  }
};

// Buffer slots per thread for a given KCAP: room for the top-k plus at least
// two 32-candidate chunks between compactions.
__host__ __device__ constexpr int topk_buffer_slots(int kcap) { return 2 * kcap + 32; }

}  // namespace bsa
