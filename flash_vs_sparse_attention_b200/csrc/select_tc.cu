// Stages 2-3 on tcgen05 tensor cores: coarse scores + causal block mask +
// per-row top-k, fused; the (rows x blocks) score matrix never leaves the SM.
// (block_indexer_triton.py:120-129; block_indexer.py:44-53)
//
// The kernel is persistent: each CTA walks a strided list of (unit, 128-row
// tile) items, heaviest causal tiles first.  The block means arrive as two
// bf16 terms, hi + lo (written by the pool kernel), and the scores are
// computed as Q.hi + Q.lo with fp32 accumulation in TMEM.  Q is exact in bf16
// and hi + lo carries the fp32 mean to ~2^-17 relative, so the scores match
// an fp32 GEMM to ~1e-7 -- well inside the 1e-5 boundary gap the index
// parity needs (a single bf16 term would change ~5% of selections).
//
// The block means stream through shared memory in windows of W blocks (TMA,
// double buffered, prefetched across items); each window's 128 x W scores
// land in one of two TMEM buffers.  Every item makes two passes over its
// windows (the MMAs are cheap and simply run twice).  Pass 1: each selection
// thread (one per row) folds its row into 32 strided group maxima; their k-th
// largest is a valid floor for the row's final threshold (k distinct row
// elements) and lets only ~4% of a 512-block row through.  Pass 2: the row's
// scores at or above the floor go to the streaming top-k buffer
// (topk_select.cuh), whose final emission keeps the top k of the ~20
// survivors with a min/max insertion network.  Causal tiles stop at the last
// block their rows can see.
// The scores arrive pre-scaled: the pool kernel splits mean * scale.
//
// Warps: 0-3 select (thread = row), 4 issues TMA, one thread of 5 issues MMAs.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launchers.cuh"
#include "sm100.cuh"
#include "topk_select.cuh"

namespace bsa {

using namespace sm100;

constexpr int kSelRows = 128;

template <int KCAP, int HD>
struct SelCfg {
  // The head_dim-64 shapes run two CTAs per SM (two selection warps per
  // scheduler hide each other's latency), which caps shared memory near
  // 100 KB: 64-block windows, one Q buffer and a candidate buffer of k + 32
  // slots (the row floor leaves ~20 candidates per row; the buffer compacts
  // itself if a row sends more).  Wider problems use one CTA per SM.
  static constexpr int kCtasPerSm = (HD == 64 && KCAP <= 32) ? 2 : 1;
  static constexpr int W = (HD == 64) ? (KCAP <= 16 ? 64 : (KCAP <= 32 ? 32 : 64))
                                      : (KCAP <= 16 ? 64 : 32);
  static constexpr int kQBufs = kCtasPerSm == 2 ? 1 : 2;
  static constexpr int kCap = kCtasPerSm == 2 ? KCAP + 32 : topk_buffer_slots(KCAP);
  static constexpr int kQBytes = kSelRows * HD * 2;
  static constexpr int kTermBytes = W * HD * 2;          // one bf16 term of a window
  static constexpr int kWinBytes = 2 * kTermBytes;       // hi + lo
  static constexpr int kBufOff = kQBufs * kQBytes + 2 * kWinBytes;
  static constexpr int kBufBytes = kCap * kSelRows * 8;
  static constexpr int kSmem = kBufOff + kBufBytes + 256 + 1024;
  static constexpr int kTmemCols = (2 * W <= 32) ? 32 : (2 * W <= 64 ? 64 : (2 * W <= 128 ? 128 : 256));
  static constexpr int kThreads = 192;
  static_assert(kCap >= KCAP + 32, "the buffer must hold the top-k plus one 32-candidate chunk");
};

struct SelectTcParams {
  int32_t* idx;
  uint32_t* err;   // may be null
  Shape s;
  int tiles;       // 128-row tiles per unit
};

template <int KCAP, int HD>
__global__ void __launch_bounds__(192, SelCfg<KCAP, HD>::kCtasPerSm)
select_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                 const __grid_constant__ CUtensorMap tmap_hi,
                 const __grid_constant__ CUtensorMap tmap_lo, SelectTcParams prm) {
  using C = SelCfg<KCAP, HD>;
  constexpr int W = C::W;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  auto q_s = [&](int b) { return smem + (b % C::kQBufs) * C::kQBytes; };
  auto win = [&](int b, int term) {
    return smem + C::kQBufs * C::kQBytes + b * C::kWinBytes + term * C::kTermBytes;
  };
  uint2* cbuf = reinterpret_cast<uint2*>(smem + C::kBufOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBufOff + C::kBufBytes);
  uint64_t* q_full = bars + 0;    // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* k_full = bars + 4;    // [2]
  uint64_t* k_empty = bars + 6;   // [2]
  uint64_t* s_full = bars + 8;    // [2]
  uint64_t* s_free = bars + 10;   // [2]
  uint64_t* drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 14);

  const Shape s = prm.s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = s.units * prm.tiles;
  if ((int)blockIdx.x >= total) return;

  // Item n of this CTA: unit and 128-row tile (heaviest causal tiles first).
  auto item_unit = [&](int n) { return (int)((blockIdx.x + (int64_t)n * gridDim.x) % s.units); };
  auto item_tile = [&](int n) {
    return prm.tiles - 1 - (int)((blockIdx.x + (int64_t)n * gridDim.x) / s.units);
  };
  const int n_items = (total - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  auto visible_blocks = [&](int tile) {
    const int last_row = min((tile + 1) * kSelRows, s.N) - 1;
    return s.causal ? min(s.nb, last_row / s.bs + 1) : s.nb;
  };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], kSelRows);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&tmap_q);
    prefetch_tensormap(&tmap_hi);
    prefetch_tensormap(&tmap_lo);
  }
  if (warp == 0) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int kw = 0;  // windows loaded so far
      for (int n = 0; n < n_items; ++n) {
        const int unit = item_unit(n), tile = item_tile(n);
        const int qb = n % C::kQBufs;
        const int qn = n / C::kQBufs;   // use count of this Q buffer
        if (qn >= 1 && (!mbar_wait(&q_empty[qb], (qn - 1) & 1, prm.err, 1u) || *abort_flag)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&q_full[qb], C::kQBytes);
#pragma unroll
        for (int p = 0; p < HD / 64; ++p)
          tma_load_2d(q_s(qb) + p * (kSelRows * 128), &tmap_q, &q_full[qb], p * 64,
                      unit * s.N + tile * kSelRows);
        const int nw = (visible_blocks(tile) + W - 1) / W;
        bool ok = true;
        for (int ww = 0; ww < 2 * nw; ++ww, ++kw) {
          const int w = ww % nw;   // two passes over the item's windows
          const int b = kw & 1;
          if (kw >= 2 && (!mbar_wait(&k_empty[b], ((kw - 2) >> 1) & 1, prm.err, 1u) || *abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[b], C::kWinBytes);
          const int y = unit * s.nb + w * W;
#pragma unroll
          for (int p = 0; p < HD / 64; ++p) {
            tma_load_2d(win(b, 0) + p * (W * 128), &tmap_hi, &k_full[b], p * 64, y);
            tma_load_2d(win(b, 1) + p * (W * 128), &tmap_lo, &k_full[b], p * 64, y);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kSelRows, W, false);
      bool ok = true;
      int kw = 0;
      for (int n = 0; ok && n < n_items; ++n) {
        const int qb = n % C::kQBufs;
        ok = mbar_wait(&q_full[qb], (n / C::kQBufs) & 1, prm.err, 2u);
        const uint32_t qa = smem_u32(q_s(qb));
        const int nw = (visible_blocks(item_tile(n)) + W - 1) / W;
        for (int ww = 0; ok && ww < 2 * nw; ++ww, ++kw) {
          const int b = kw & 1;
          ok = mbar_wait(&k_full[b], (kw >> 1) & 1, prm.err, 4u);
          if (ok && kw >= 2) ok = mbar_wait(&s_free[b], ((kw - 2) >> 1) & 1, prm.err, 8u);
          if (!ok || *abort_flag) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tbase + b * W;
#pragma unroll
          for (int term = 0; term < 2; ++term) {
            const uint32_t ka = smem_u32(win(b, term));
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint32_t qo = (kk >> 2) * (kSelRows * 128) + (kk & 3) * 32;
              const uint32_t ko = (kk >> 2) * (W * 128) + (kk & 3) * 32;
              mma_bf16(d, smem_desc_sw128(qa + qo, 16, 1024), smem_desc_sw128(ka + ko, 16, 1024),
                       idesc, (term > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(&s_full[b]);
          mma_commit(&k_empty[b]);
        }
        if (ok) mma_commit(&q_empty[qb]);
      }
      if (!ok) *abort_flag = 1;
      mma_commit(drain);
      mbar_wait(drain, 0, prm.err, 16u);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ selection
    const int r = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    int kw = 0;
    bool ok = true;
    for (int n = 0; ok && n < n_items; ++n) {
      const int unit = item_unit(n), tile = item_tile(n);
      const int row0 = tile * kSelRows;
      const int row = row0 + r;
      const bool valid = row < s.N;
      const int nbv = visible_blocks(tile);
      const int nw = (nbv + W - 1) / W;
      // This row may select blocks [0, lim): the causal mask of
      // block_indexer.py:46-50 keeps block j while j * bs <= row.
      const int lim = !valid ? 0 : (s.causal ? min(s.nb, row / s.bs + 1) : s.nb);
      RowTopK<KCAP> sel;
      const int ku = unit_top_k(s, unit);   // this head's budget (s.k unless per head)
      sel.init(cbuf + r, kSelRows, C::kCap, ku);
      // Group maxima: 32 strided groups (column % 32) for top_k <= 16; for
      // larger top_k 64 groups (column % 64: the two halves gm / gm2, by the
      // parity of the 32-column chunk), whose k-th largest maximum is a much
      // tighter floor than the smallest of 32 when k is 32 or more.
      constexpr bool kG64 = KCAP > 16;
      float gm[32], gm2[kG64 ? 32 : 1];
#pragma unroll
      for (int i = 0; i < 32; ++i) gm[i] = -INFINITY;
#pragma unroll
      for (int i = 0; i < (kG64 ? 32 : 1); ++i) gm2[i] = -INFINITY;
      for (int ww = 0; ww < 2 * nw; ++ww, ++kw) {
        const int pass = ww >= nw;
        const int w = ww - pass * nw;
        const int b = kw & 1;
        ok = mbar_wait(&s_full[b], (kw >> 1) & 1, prm.err, 32u);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || *abort_flag) { ok = false; break; }
        tc_fence_after();
        const int jb = w * W;
        const int chunks = min(W / 32, (nbv - jb + 31) / 32);
        // Masking is needed where a block starts after this tile's first
        // row, and for columns past the last block.
        const bool need_mask = (s.causal && (int64_t)(jb + W - 1) * s.bs > row0) || (jb + W > s.nb);
        for (int c = 0; c < chunks; ++c) {
          float x[32];
          tmem_ld32(tbase + lane_off + b * W + c * 32, x);
          if (c == chunks - 1) {
            tc_fence_before();
            mbar_arrive(&s_free[b]);
          }
          const int j0 = jb + c * 32;
          // The chunk's selectable columns as a bit mask: the first lim - j0.
          uint32_t vm = 0xffffffffu;
          if (need_mask || !valid) {
            const int nv = lim - j0;
            vm = nv >= 32 ? 0xffffffffu : (nv <= 0 ? 0u : (1u << nv) - 1u);
          }
          if (pass == 0) {
            if (need_mask || !valid) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (((vm >> i) & 1u) == 0u) x[i] = -INFINITY;
            }
            if (kG64 && ((j0 >> 5) & 1)) {   // the same for the whole warp
#pragma unroll
              for (int i = 0; i < (kG64 ? 32 : 1); ++i) gm2[i] = fmaxf(gm2[i], x[i]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) gm[i] = fmaxf(gm[i], x[i]);
            }
          } else {
            // The chunk's candidates as a bit mask (four independent 8-bit
            // parts); the buffer compacts only if this row's own candidates
            // would overflow it.
            uint32_t pq[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int i = 0; i < 32; ++i) pq[i >> 3] |= sel.passes(x[i]) ? (1u << i) : 0u;
            const uint32_t pm = ((pq[0] | pq[1]) | (pq[2] | pq[3])) & vm;
            if (pm) {
              sel.reserve(__popc(pm));
              sel.append_mask(x, pm, j0);
            }
          }
        }
        if (chunks <= 0) {  // every thread arrives once per window
          tc_fence_before();
          mbar_arrive(&s_free[b]);
        }
        // The floor: the k-th largest group maximum (-inf if fewer than k
        // groups are non-empty).
        if (pass == 0 && w == nw - 1) {
          if constexpr (kG64) sel.raise_floor(kth_of_64(gm, gm2, ku));
          else if (ku == 16) sel.raise_floor(kth16_of_32(gm));
          else if (ku <= 32) sel.raise_floor(kth_of_32(gm, ku));
        }
      }
      if (!ok) break;
      if (valid) sel.emit(prm.idx + ((int64_t)unit * s.N + row) * s.k, s.k);
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, C::kTmemCols);
}

// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

static bool map2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool select_tc_supported(const Shape& s) {
  return (s.D == 64 || s.D == 128) && s.k <= 64 && (int64_t)s.units * s.N < (1LL << 31) &&
         (int64_t)s.units * s.nb < (1LL << 31);
}

template <int KCAP, int HD>
static cudaError_t launch_tc(const __nv_bfloat16* Q, const __nv_bfloat16* K_hi,
                             const __nv_bfloat16* K_lo, int32_t* idx, uint32_t* err,
                             const Shape& s, cudaStream_t st) {
  using C = SelCfg<KCAP, HD>;
  CUtensorMap mq, mh, ml;
  if (!map2d(&mq, Q, (uint64_t)s.units * s.N, HD, kSelRows) ||
      !map2d(&mh, K_hi, (uint64_t)s.units * s.nb, HD, C::W) ||
      !map2d(&ml, K_lo, (uint64_t)s.units * s.nb, HD, C::W))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(select_tc_kernel<KCAP, HD>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return e;
  SelectTcParams prm{idx, err, s, (s.N + kSelRows - 1) / kSelRows};
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = s.units * prm.tiles;
  const int grid = items < sms * C::kCtasPerSm ? items : sms * C::kCtasPerSm;
  select_tc_kernel<KCAP, HD><<<grid, C::kThreads, C::kSmem, st>>>(mq, mh, ml, prm);
  return cudaGetLastError();
}

cudaError_t launch_select_tc(const __nv_bfloat16* Q, const __nv_bfloat16* K_hi,
                             const __nv_bfloat16* K_lo, int32_t* idx, uint32_t* err,
                             const Shape& s, cudaStream_t st) {
  if (s.D == 64) {
    if (s.k <= 16) return launch_tc<16, 64>(Q, K_hi, K_lo, idx, err, s, st);
    if (s.k <= 32) return launch_tc<32, 64>(Q, K_hi, K_lo, idx, err, s, st);
    return launch_tc<64, 64>(Q, K_hi, K_lo, idx, err, s, st);
  }
  if (s.k <= 16) return launch_tc<16, 128>(Q, K_hi, K_lo, idx, err, s, st);
  if (s.k <= 32) return launch_tc<32, 128>(Q, K_hi, K_lo, idx, err, s, st);
  return launch_tc<64, 128>(Q, K_hi, K_lo, idx, err, s, st);
}

}  // namespace bsa
