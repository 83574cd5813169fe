// Stage 4, query-stationary (block_indexer_triton.py:12-83 mapped the way the
// reference's Triton kernel maps it: a program per query tile walking key
// blocks), on tcgen05 tensor cores, for the 128-row query tiles whose rows
// between them select few distinct key blocks.
//
// Per-tile dispatch.  classify_tiles_kernel looks at every 128-row tile of
// every unit: the union of the key blocks its rows selected (a bitmask) and
// its size U.  A tile whose rows all list strictly increasing block indices
// (no repeats: a repeated block must count twice, as the key-block-stationary
// path counts it) and whose U is at most max_union becomes a query tile: it
// gets a slot (its unit, tile and U, and the union bitmask), and tile_mode
// marks it, so the bucket kernels treat its rows' entries as empty and the
// combine leaves its rows alone.  Every other tile goes through the
// key-block-stationary path (fine_kv.cu).  The default max_union is
// 3 top_k: up to there the tile's dense work over its union costs less than
// the partial round trip of the key-stationary path (on clustered content,
// B2 H32 N32768 D128 k32: 14.08 ms per step at 2.5 top_k, 12.39 at 3, 12.42
// at 4).
//
// fine_q_kernel, persistent over the query-tile slots.  Per tile: TMA loads
// the 128 query rows once (two buffers where room allows, so the next tile's
// rows load early); for every block j of the union, in ascending order, TMA
// loads K_j and V_j (plain tiled loads into a ring of stages, the blocks a
// few ahead prefetched into L2 first), tcgen05 computes S = Q K_j^T into
// TMEM (one or two S buffers), the softmax warpgroup (one thread per row)
// masks the rows that did not select j and the keys past a row's position
// (causal), and turns S into P (bf16, TMEM, two buffers) against a running
// row maximum, and tcgen05 accumulates O += P V_j in TMEM.  The
// running maximum is raised lazily: only when a block's maximum exceeds it by
// more than 8 (a factor 2^8 in P) are the row's O and l rescaled, after the
// previous block's PV has completed; P never exceeds 2^8.  At the end of the
// tile each row's O / l is rounded to bf16 once and stored.
//
// Warps: 0-3 softmax (thread = row), 4 TMA producer, 5 MMA issuer (one
// thread).  Every wait is bounded (an error bit and an abort, not a hang).
// Barrier phases are tracked by per-role counters that advance identically:
// every role visits the same tiles and the same union blocks in the same
// order (g counts union blocks over the CTA's tiles, n counts tiles).
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "launchers.cuh"
#include "sm100.cuh"

namespace bsa {

using namespace sm100;

namespace {

constexpr int kQRows = 128;          // query rows per tile (MMA M)
constexpr int kQMaxUnion = 512;      // union blocks a query tile may have
constexpr int kQUnionWords = kQMaxUnion / 32;
constexpr int kQMaxNbWords = 512;    // block-bitmask words (nb <= 16384)
constexpr int kQThreads = 192;
constexpr int kQPrefetch = 4;        // union blocks whose K/V go to L2 ahead of their loads

// Error bits of this kernel's bounded waits (the fine stage's error word).
// kErrQTestTimeout is the key-stationary kernel's test-hook bit (same meaning).
constexpr uint32_t kErrQTestTimeout = 512u;
constexpr uint32_t kErrQWaitQ = 1u << 12, kErrQWaitKV = 1u << 13, kErrQWaitS = 1u << 14,
                   kErrQWaitP = 1u << 15, kErrQWaitO = 1u << 16, kErrQDrain = 1u << 17;

template <int BS, int HD>
struct QCfg {
  static constexpr int kQBytes = kQRows * HD * 2;
  static constexpr int kKBytes = BS * HD * 2;               // one block of K (or V)
  // Two CTAs per SM where TMEM (256 columns each) and shared memory allow:
  // head_dim 128 then keeps one Q buffer, one S buffer and two K and two V
  // stages (the other CTA fills the gaps these leave); block 128 runs one CTA.
  // K and V have rings of their own: K_j's stage is free once S(j) is done,
  // V_j's once PV(j) is, so K loads run ahead of V loads.
  static constexpr int kCtasPerSm = (BS == 64) ? 2 : 1;
  static constexpr int kQBufs = (BS == 64 && HD == 128) ? 1 : 2;
  static constexpr int kSBufs = (BS == 64 && HD == 128) ? 1 : 2;
  static constexpr int NK = (BS == 64 && HD == 64) ? 4 : ((BS == 64) ? 2 : 3);   // K stages
  static constexpr int NV = NK;                                                  // V stages
  static constexpr int kKRingOff = kQBufs * kQBytes;
  static constexpr int kVRingOff = kKRingOff + NK * kKBytes;
  static constexpr int kRowBitsOff = kVRingOff + NV * kKBytes;
  static constexpr int kRowBitsBytes = kQUnionWords * kQRows * 4;
  static constexpr int kTileBitsOff = kRowBitsOff + kRowBitsBytes;
  static constexpr int kTileBitsBytes = 2 * kQMaxNbWords * 4;   // bits, then prefix counts
  static constexpr int kBarOff = kTileBitsOff + kTileBitsBytes;
  static constexpr int kSmem = kBarOff + 512 + 1024 /*alignment*/;
  // TMEM: S[kSBufs] (BS columns each), P[2] (bf16 pairs, BS / 2 each), O (HD).
  static constexpr int kSCol = 0, kPCol = kSBufs * BS, kOCol = kSBufs * BS + BS;
  static constexpr int kCols = kSBufs * BS + BS + HD;
  static constexpr int kTmemCols = kCols <= 256 ? 256 : 512;
  static_assert(kCols <= 512, "TMEM");
  static_assert(kKRingOff % 1024 == 0 && kKBytes % 1024 == 0, "swizzled tiles");
  static_assert(kSmem <= 227 * 1024, "shared memory");
  static_assert(kCtasPerSm * (kSmem + 1024) <= 228 * 1024, "CTAs per SM");
  static_assert(kCtasPerSm * kTmemCols <= 512, "TMEM per SM");
};

}  // namespace

// ---------------------------------------------------------------------------
// One CTA (128 threads) per (unit, tile).  Dynamic shared memory: a byte per
// block (nb rounded up to 16) marking the blocks the tile's rows selected --
// plain stores of 1, no atomics, so rows picking the same blocks do not
// serialise -- then packed into nbw bitmask words.
template <int KMAX>
__global__ void __launch_bounds__(kQRows)
classify_tiles_kernel(const int32_t* __restrict__ idx, uint8_t* __restrict__ tile_mode,
                      uint32_t* __restrict__ qt_bits, int4* __restrict__ qt_info,
                      uint32_t* __restrict__ n_qt, Shape s, int tiles, int max_union) {
  extern __shared__ __align__(16) uint8_t present[];
  __shared__ int u_count, slot;
  const int nbw = (s.nb + 31) / 32;
  const int nb16 = (s.nb + 15) / 16;
  const int tid = threadIdx.x;
  const int u = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  for (int w = tid; w < nb16; w += kQRows)
    reinterpret_cast<uint4*>(present)[w] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) u_count = 0;
  __syncthreads();
  const int row = tile * kQRows + tid;
  bool ok = true;
  if (row < s.N) {
    // The row's entries, all loads in flight before the scan (top_k <=
    // KMAX; 16-byte loads when a row starts on a 16-byte boundary).
    const int32_t* p = idx + ((int64_t)u * s.N + row) * s.k;
    int v[KMAX];
    if ((s.k & 3) == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int t = 0; t < KMAX; t += 4) {
        if (t < s.k) {
          const int4 x = __ldg(reinterpret_cast<const int4*>(p + t));
          v[t] = x.x; v[t + 1] = x.y; v[t + 2] = x.z; v[t + 3] = x.w;
        }
      }
    } else {
#pragma unroll
      for (int t = 0; t < KMAX; ++t)
        if (t < s.k) v[t] = __ldg(p + t);
    }
    int prev = -1;
    bool ended = false;
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      if (t < s.k && ok) {
        const int j = v[t];
        if (j < 0) {
          ended = true;
        } else if (ended || j <= prev || j >= s.nb) {
          ok = false;
        } else {
          present[j] = 1;
          prev = j;
        }
      }
    }
  }
  ok = __syncthreads_and(ok) != 0;
  // Pack 32 bytes into a word; count the union.
  uint32_t my_words[kQMaxNbWords / kQRows];
  int c = 0;
#pragma unroll
  for (int q = 0; q < kQMaxNbWords / kQRows; ++q) {
    const int w = tid + q * kQRows;
    uint32_t m = 0u;
    if (w < nbw) {
      const uint4* b4 = reinterpret_cast<const uint4*>(present + 32 * w);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (32 * w + 16 * h < 16 * nb16) {
          const uint4 x = b4[h];
          const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int bb = 0; bb < 4; ++bb)
              m |= ((xs[e] >> (8 * bb)) & 1u) << (16 * h + 4 * e + bb);
        }
      }
    }
    my_words[q] = m;
    c += __popc(m);
  }
  if (c) atomicAdd(&u_count, c);
  __syncthreads();
  const int U = u_count;
  const bool q = ok && U > 0 && U <= max_union;
  if (tid == 0) {
    tile_mode[(int64_t)u * tiles + tile] = q ? 1 : 0;
    if (q) {
      slot = (int)atomicAdd(n_qt, 1u);
      qt_info[slot] = make_int4(u, tile, U, 0);
    }
  }
  __syncthreads();
  if (q) {
#pragma unroll
    for (int qq = 0; qq < kQMaxNbWords / kQRows; ++qq) {
      const int w = tid + qq * kQRows;
      if (w < nbw) qt_bits[(int64_t)slot * nbw + w] = my_words[qq];
    }
  }
}

// ---------------------------------------------------------------------------
struct FineQParams {
  const __nv_bfloat16* K;    // (units, N, HD): for the L2 prefetches
  const __nv_bfloat16* V;
  const int32_t* idx;        // (units, N, top_k) selections
  const uint32_t* qt_bits;   // per query-tile slot: the union bitmask (nbw words)
  const int4* qt_info;       // per slot: unit, tile, union size
  const uint32_t* n_qt;      // number of slots
  int min_q_tiles;           // fewer slots than this: the key-stationary path took them
  __nv_bfloat16* O;          // (units, N, HD)
  uint32_t* err;             // the fine stage's error word
  Shape s;
};

// Barrier 1 joins the softmax warps (0-3) only.  Every exit from their tile
// loop goes through softmax_group_and, so all four warps leave together and
// none is left waiting at a barrier the others never reach.
__device__ __forceinline__ void softmax_group_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}
__device__ __forceinline__ bool softmax_group_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0u;
}

template <int BS, int HD>
__global__ void __launch_bounds__(kQThreads, QCfg<BS, HD>::kCtasPerSm)
fine_q_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
              const __grid_constant__ CUtensorMap tmap_v, FineQParams prm) {
  using C = QCfg<BS, HD>;
  constexpr int NK = C::NK, NV = C::NV;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  auto q_s = [&](int b) { return smem + b * C::kQBytes; };
  auto k_s = [&](int st) { return smem + C::kKRingOff + st * C::kKBytes; };
  auto v_s = [&](int st) { return smem + C::kVRingOff + st * C::kKBytes; };
  uint32_t* rowbits = reinterpret_cast<uint32_t*>(smem + C::kRowBitsOff);   // [word][row]
  uint32_t* tb = reinterpret_cast<uint32_t*>(smem + C::kTileBitsOff);       // union bitmask
  uint32_t* tpre = tb + kQMaxNbWords;                                        // its prefix counts
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;          // [2]
  uint64_t* q_empty = bars + 2;     // [2]
  uint64_t* s_full = bars + 4;      // [2]
  uint64_t* s_free = bars + 6;      // [2]
  uint64_t* p_full = bars + 8;      // [2]
  uint64_t* p_free = bars + 10;     // [2]
  uint64_t* o_full = bars + 12;
  uint64_t* o_empty = bars + 13;
  uint64_t* drain = bars + 14;
  uint64_t* k_full = bars + 15;                    // [NK]
  uint64_t* k_empty = k_full + NK;                 // [NK]
  uint64_t* v_full = k_empty + NK;                 // [NV]
  uint64_t* v_empty = v_full + NV;                 // [NV]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_empty + NV);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(v_empty + NV + 1);
  uint64_t* gate = v_empty + NV + 2;               // test hook: nothing completes it
  static_assert((18 + 2 * NK + 2 * NV) * 8 <= 512, "barrier area");

  const Shape s = prm.s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (int)*prm.n_qt;
  if (n_tiles < prm.min_q_tiles || (int)blockIdx.x >= n_tiles) return;   // whole CTA, no barrier yet
  const int my_tiles = (n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  auto slot_of = [&](int n) { return (int)blockIdx.x + n * (int)gridDim.x; };
  const int nbw = (s.nb + 31) / 32;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], kQRows);
      mbar_init(&p_full[b], kQRows);
      mbar_init(&p_free[b], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, kQRows);
    mbar_init(drain, 1);
    mbar_init(gate, 1);
    for (int st = 0; st < NK; ++st) {
      mbar_init(&k_full[st], 1);
      mbar_init(&k_empty[st], 1);
    }
    for (int st = 0; st < NV; ++st) {
      mbar_init(&v_full[st], 1);
      mbar_init(&v_empty[st], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&tmap_q);
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  if (warp == 0) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (s.test_timeout) {
    // Test hook (BSA_FLAG_TEST_TIMEOUT): one bounded wait of a few
    // microseconds on a barrier nothing completes, before any copy or MMA;
    // it records its bit in the error word, and the CTA's rows come out NaN.
    if (threadIdx.x == 0) mbar_wait_ns(gate, 0, prm.err, kErrQTestTimeout, 2000);
    __syncthreads();
    if (warp < 4) {
      const int r = warp * 32 + lane;
      const uint32_t nan2 = 0x7fc07fc0u;   // two bf16 NaNs
      for (int n = 0; n < my_tiles; ++n) {
        const int4 info = __ldg(prm.qt_info + slot_of(n));
        const int row = info.y * kQRows + r;
        if (row >= s.N) continue;
        uint4* orow = reinterpret_cast<uint4*>(prm.O + ((int64_t)info.x * s.N + row) * HD);
#pragma unroll
        for (int q = 0; q < HD / 8; ++q) orow[q] = make_uint4(nan2, nan2, nan2, nan2);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ TMA producers
    // Lane 0: Q of every tile, K of every union block, and the L2 prefetch
    // of the K/V blocks kQPrefetch ahead.  Lane 1: V of every union block.
    // Each walks the same tiles and union bitmasks in the same order.
    if (lane < 2) {
      const bool kq = lane == 0;
      const int NR = kq ? NK : NV;                 // this lane's ring
      uint64_t* full = kq ? k_full : v_full;
      uint64_t* empty = kq ? k_empty : v_empty;
      const CUtensorMap* tm = kq ? &tmap_k : &tmap_v;
      int g = 0, qn = 0;   // ring loads and Q loads issued
      bool ok = true;
      for (int n = 0; ok && n < my_tiles; ++n) {
        const int4 info = __ldg(prm.qt_info + slot_of(n));
        const int unit = info.x, tile = info.y;
        if (kq) {
          const int qb = n % C::kQBufs;
          if (n >= C::kQBufs)
            ok = mbar_wait(&q_empty[qb], ((n - C::kQBufs) / C::kQBufs) & 1, prm.err, kErrQWaitQ);
          if (!ok || *abort_flag) { ok = false; break; }
          mbar_arrive_expect_tx(&q_full[qb], C::kQBytes);
          ++qn;
#pragma unroll
          for (int p = 0; p < HD / 64; ++p)
            tma_load_2d(q_s(qb) + p * (kQRows * 128), &tmap_q, &q_full[qb], p * 64,
                        unit * s.N + tile * kQRows);
        }
        const uint32_t* bw = prm.qt_bits + (int64_t)slot_of(n) * nbw;
        // The K/V blocks kQPrefetch ahead of the loads go to L2 first, so a
        // stage's TMA load (which waits for the MMA that frees it) finds
        // them there.
        int pw = 0;
        uint32_t pm = __ldg(bw);
        auto prefetch_next = [&]() {
          while (pm == 0u && pw + 1 < nbw) pm = __ldg(bw + ++pw);
          if (pm == 0u) return;
          const int jp = pw * 32 + __ffs(pm) - 1;
          pm &= pm - 1u;
          const int64_t off = ((int64_t)unit * s.N + (int64_t)jp * BS) * HD;
          bulk_prefetch_l2(prm.K + off, (uint32_t)C::kKBytes);
          bulk_prefetch_l2(prm.V + off, (uint32_t)C::kKBytes);
        };
        if (kq)
          for (int q = 0; q < kQPrefetch; ++q) prefetch_next();
        for (int w = 0; ok && w < nbw; ++w) {
          uint32_t m = __ldg(bw + w);
          while (m != 0u) {
            const int j = w * 32 + __ffs(m) - 1;
            m &= m - 1u;
            const int st = g % NR;
            if (g >= NR) ok = mbar_wait(&empty[st], ((g - NR) / NR) & 1, prm.err, kErrQWaitKV);
            if (!ok || *abort_flag) { ok = false; break; }
            mbar_arrive_expect_tx(&full[st], C::kKBytes);
            unsigned char* dst = kq ? k_s(st) : v_s(st);
            const int y = unit * s.N + j * BS;
#pragma unroll
            for (int p = 0; p < HD / 64; ++p)
              tma_load_2d(dst + p * (BS * 128), tm, &full[st], p * 64, y);
            if (kq) prefetch_next();
            ++g;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        // Copies still in flight land before the CTA leaves: wait for the
        // last load of every stage of this lane's ring (and Q buffer),
        // bounded; those phases are the barriers' latest, so their parity is
        // unambiguous.
        for (int st = 0; st < NR; ++st) {
          const int last = g - 1 - ((g - 1 - st) % NR + NR) % NR;
          if (last >= 0) mbar_wait(&full[st], (last / NR) & 1, prm.err, kErrQWaitKV);
        }
        if (kq) {
          for (int qb = 0; qb < C::kQBufs; ++qb) {
            const int last = qn - 1 - ((qn - 1 - qb) % C::kQBufs + C::kQBufs) % C::kQBufs;
            if (last >= 0) mbar_wait(&q_full[qb], (last / C::kQBufs) & 1, prm.err, kErrQWaitQ);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(kQRows, BS, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(kQRows, HD, true);
      const uint64_t dq0 = smem_desc_sw128(smem_u32(q_s(0)), 16, 1024);
      const uint64_t dk0 = smem_desc_sw128(smem_u32(k_s(0)), 16, 1024);
      const uint64_t dv0 = smem_desc_sw128(smem_u32(v_s(0)), BS * 128, 1024);
      // O += P(gp) V(gp); `first`: the tile's first PV, which overwrites O
      // once the previous tile's epilogue has read it.
      auto pv = [&](int gp, int n, bool first) -> bool {
        const int bp = gp & 1, stp = gp % NV;
        if (!mbar_wait(&p_full[bp], (gp >> 1) & 1, prm.err, kErrQWaitP)) return false;
        if (!mbar_wait(&v_full[stp], (gp / NV) & 1, prm.err, kErrQWaitKV)) return false;
        if (first && n >= 1 && !mbar_wait(o_empty, (n - 1) & 1, prm.err, kErrQWaitO)) return false;
        if (*abort_flag) return false;
        tc_fence_after();
        const uint64_t dv = dv0 + ((uint64_t)(stp * C::kKBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < BS / 16; ++kk)
          mma_bf16_ts(tbase + C::kOCol, tbase + C::kPCol + bp * (BS / 2) + kk * 8,
                      dv + ((kk * 16 * 128) >> 4), idesc_o, (!first || kk > 0) ? 1u : 0u);
        mma_commit(&p_free[bp]);
        mma_commit(&v_empty[stp]);
        return true;
      };
      int g = 0;
      bool ok = true;
      for (int n = 0; ok && n < my_tiles; ++n) {
        const int U = __ldg(prm.qt_info + slot_of(n)).z;
        const int qb = n % C::kQBufs;
        ok = mbar_wait(&q_full[qb], (n / C::kQBufs) & 1, prm.err, kErrQWaitQ);
        const uint64_t dq = dq0 + ((uint64_t)(qb * C::kQBytes) >> 4);
        for (int i = 0; ok && i < U; ++i, ++g) {
          const int st = g % NK, sb = g % C::kSBufs;
          ok = mbar_wait(&k_full[st], (g / NK) & 1, prm.err, kErrQWaitKV);
          if (ok && g >= C::kSBufs)
            ok = mbar_wait(&s_free[sb], ((g - C::kSBufs) / C::kSBufs) & 1, prm.err, kErrQWaitS);
          if (!ok || *abort_flag) { ok = false; break; }
          tc_fence_after();
          const uint64_t dk = dk0 + ((uint64_t)(st * C::kKBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (kQRows * 128) + (kk & 3) * 32;
            const uint32_t offk = (kk >> 2) * (BS * 128) + (kk & 3) * 32;
            mma_bf16(tbase + C::kSCol + sb * BS, dq + (off >> 4), dk + (offk >> 4), idesc_s,
                     kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[sb]);
          mma_commit(&k_empty[st]);                 // K_j's stage, once S(j) is done
          if (i == U - 1) mma_commit(&q_empty[qb]);
          if (i >= 1) ok = pv(g - 1, n, i == 1);
        }
        if (ok) ok = pv(g - 1, n, U == 1);
        if (ok) mma_commit(o_full);
      }
      if (!ok) *abort_flag = 1;
      mma_commit(drain);
      mbar_wait(drain, 0, prm.err, kErrQDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int r = warp * 32 + lane;                    // row of the tile
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t o_addr = tbase + lane_off + C::kOCol;
    const float sc = s.scale * kLog2e;                 // scores in the base-2 domain
    int g = 0;
    bool ok = true;
    for (int n = 0; n < my_tiles; ++n) {
      // All four warps agree to go on (and the last tile is done with the
      // shared bitmask).
      ok = softmax_group_and(ok && !*abort_flag);
      if (!ok) break;
      const int4 info = __ldg(prm.qt_info + slot_of(n));
      const int unit = info.x, tile = info.y, U = info.z;
      const int row = tile * kQRows + r;
      const bool valid = row < s.N;
      // The tile's union bitmask and, per word, the blocks before it.
      const uint32_t* bw = prm.qt_bits + (int64_t)slot_of(n) * nbw;
      for (int w = r; w < nbw; w += kQRows) tb[w] = __ldg(bw + w);
      softmax_group_sync();
      if (warp == 0) {
        const int per = (nbw + 31) / 32;
        int cnt = 0;
        for (int q = 0; q < per; ++q) {
          const int w = lane * per + q;
          if (w < nbw) cnt += __popc(tb[w]);
        }
        int inc = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += y;
        }
        int run = inc - cnt;
        for (int q = 0; q < per; ++q) {
          const int w = lane * per + q;
          if (w < nbw) { tpre[w] = run; run += __popc(tb[w]); }
        }
      }
      softmax_group_sync();
      // This row's selected blocks as positions in the union.
      const int UW = (U + 31) >> 5;
      for (int w = 0; w < UW; ++w) rowbits[w * kQRows + r] = 0u;
      if (valid) {
        // The row's indices, 16 per batch with every load of the batch in
        // flight before the first is used (16-byte loads when aligned).
        const int32_t* p = prm.idx + ((int64_t)unit * s.N + row) * s.k;
        const bool vec = (s.k & 3) == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0;
        for (int t0 = 0; t0 < s.k; t0 += 16) {
          int v[16];
          if (vec) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int4 x = t0 + 4 * q < s.k ? __ldg(reinterpret_cast<const int4*>(p + t0) + q)
                                              : make_int4(-1, -1, -1, -1);
              v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] = t0 + q < s.k ? __ldg(p + t0 + q) : -1;
          }
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int j = v[q];
            if (j < 0) continue;
            const int pos = (int)tpre[j >> 5] + __popc(tb[j >> 5] & ((1u << (j & 31)) - 1u));
            rowbits[(pos >> 5) * kQRows + r] |= 1u << (pos & 31);
          }
        }
      }
      float m_run = -INFINITY, l = 0.f;
      uint32_t rw = 0u, cw = tb[0];
      int wi = 0;
      for (int i = 0; i < U; ++i, ++g) {
        while (cw == 0u && wi + 1 < nbw) cw = tb[++wi];
        const int j = wi * 32 + __ffs(cw) - 1;          // the union's i-th block
        cw &= cw - 1u;
        if ((i & 31) == 0) rw = rowbits[(i >> 5) * kQRows + r];
        const bool sel = ((rw >> (i & 31)) & 1u) != 0u;
        const int b = g & 1;                            // P buffer
        const int sb = g % C::kSBufs;                   // S buffer
        ok = mbar_wait(&s_full[sb], (g / C::kSBufs) & 1, prm.err, kErrQWaitS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || *abort_flag) { ok = false; break; }
        tc_fence_after();
        float sv[BS];
        if (__any_sync(0xffffffffu, sel)) {
#pragma unroll
          for (int c0 = 0; c0 < BS; c0 += 64)
            tmem_ld64(tbase + lane_off + C::kSCol + sb * BS + c0, sv + c0);
        }
        tc_fence_before();
        mbar_arrive(&s_free[sb]);                       // S(g) is in registers
        float mx = -INFINITY;
        if (sel) {
          // Token-level causal mask (block_indexer.py:73-81): key > query -> -inf.
          const int key0 = j * BS;
          if (s.causal && key0 + BS - 1 > row) {
#pragma unroll
            for (int c = 0; c < BS; ++c)
              if (key0 + c > row) sv[c] = -INFINITY;
          }
#pragma unroll
          for (int c = 0; c < BS; c += 2) mx = fmax3(mx, sv[c], sv[c + 1]);
        }
        const float msc = mx * sc;
        bool resc = false;
        if (sel && mx != -INFINITY) {
          if (m_run == -INFINITY) m_run = msc;          // O and l are still zero
          else if (msc > m_run + 8.f) resc = true;
        }
        if (__any_sync(0xffffffffu, resc)) {
          // Raise the running maximum: O (complete through PV(g - 1), an
          // earlier block of this tile) and l scale by 2^(old - new).
          const int gp = g - 1;
          ok = mbar_wait(&p_free[gp & 1], (gp >> 1) & 1, prm.err, kErrQWaitP);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
          const float alpha = resc ? fast_exp2(m_run - msc) : 1.f;
          if (resc) { m_run = msc; l *= alpha; }
#pragma unroll
          for (int c0 = 0; c0 < HD; c0 += 32) {
            float ov[32];
            tmem_ld32(o_addr + c0, ov);
#pragma unroll
            for (int h = 0; h < 32; h += 16) {
              uint32_t pk[16];
#pragma unroll
              for (int c = 0; c < 16; ++c) pk[c] = __float_as_uint(ov[h + c] * alpha);
              tmem_st16(o_addr + c0 + h, pk);
            }
          }
        }
        if (g >= 2) {
          // P buffer b is free once PV(g - 2) is done.
          ok = mbar_wait(&p_free[b], ((g - 2) >> 1) & 1, prm.err, kErrQWaitP);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
        }
        // p = 2^(s sc - m_run) (at most 2^8), 0 where masked or not selected.
        // A warp none of whose rows selected the block stores zeros.
        const bool live = sel && m_run != -INFINITY;
        const uint32_t p_addr = tbase + lane_off + C::kPCol + b * (BS / 2);
        if (__any_sync(0xffffffffu, live)) {
          const float shift = live ? m_run : INFINITY;   // not live: every p = 0
          float2 l2 = make_float2(0.f, 0.f);
          const float2 sc2 = make_float2(sc, sc), sh2 = make_float2(-shift, -shift);
#pragma unroll
          for (int c0 = 0; c0 < BS; c0 += 32) {
            uint32_t pk[16];
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              float p0, p1;
              if constexpr (BS == 64) {   // packed pairs: one fma and one add per two keys
                const float2 x = ffma2(make_float2(sv[c0 + c], sv[c0 + c + 1]), sc2, sh2);
                p0 = fast_exp2(x.x);
                p1 = fast_exp2(x.y);
                l2 = fadd2(l2, make_float2(p0, p1));
              } else {
                p0 = fast_exp2(fmaf(sv[c0 + c], sc, -shift));
                p1 = fast_exp2(fmaf(sv[c0 + c + 1], sc, -shift));
                l2.x += p0;
                l2.y += p1;
              }
              pk[c >> 1] = pack_bf16x2(p0, p1);
            }
            tmem_st16_async(p_addr + (c0 >> 1), pk);
          }
          if (live) l += l2.x + l2.y;
        } else {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) pk[c] = 0u;
#pragma unroll
          for (int c0 = 0; c0 < BS; c0 += 32) tmem_st16_async(p_addr + (c0 >> 1), pk);
        }
        tmem_wait_st();                                 // P(g) is in TMEM
        tc_fence_before();
        mbar_arrive(&p_full[b]);
      }
      ok = softmax_group_and(ok);
      if (!ok) break;
      // Epilogue: O / l rounded to bf16 once.
      ok = mbar_wait(o_full, n & 1, prm.err, kErrQWaitO);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;                               // leaves at the next group vote
      tc_fence_after();
      // A timed-out wait anywhere in the fine stage (this kernel or the
      // key-stationary one before it) leaves its bit in the error word:
      // the rows then come out NaN, as the combine writes them.
      const float inv = *reinterpret_cast<volatile uint32_t*>(prm.err) != 0u
                            ? __int_as_float(0x7fc00000) : 1.f / l;
      uint4* orow = reinterpret_cast<uint4*>(prm.O + ((int64_t)unit * s.N + row) * HD);
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 32) {
        float ov[32];
        tmem_ld32(o_addr + c0, ov);
        if (valid) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            orow[(c0 >> 3) + q] = make_uint4(
                pack_bf16x2(ov[8 * q] * inv, ov[8 * q + 1] * inv),
                pack_bf16x2(ov[8 * q + 2] * inv, ov[8 * q + 3] * inv),
                pack_bf16x2(ov[8 * q + 4] * inv, ov[8 * q + 5] * inv),
                pack_bf16x2(ov[8 * q + 6] * inv, ov[8 * q + 7] * inv));
        }
      }
      tc_fence_before();
      mbar_arrive(o_empty);
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, C::kTmemCols);
}

// ---------------------------------------------------------------------------
// Host side.
static bool q_make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                       uint32_t box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  if (enc == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool fine_q_supported(const Shape& s) {
  return ((s.bs == 64 && (s.D == 64 || s.D == 128)) || (s.bs == 128 && s.D == 64)) &&
         (s.nb + 31) / 32 <= kQMaxNbWords && (int64_t)s.units * s.N < (1LL << 31);
}

int fine_q_max_union(const Shape& s, uint32_t flags) {
  if (flags & BSA_FLAG_FINE_KEY_STATIONARY) return 0;
  if (flags & BSA_FLAG_FINE_QUERY_STATIONARY) return kQMaxUnion;
  return min(kQMaxUnion, 3 * s.k);
}

int fine_q_tiles(const Shape& s) { return (s.N + kQRows - 1) / kQRows; }

// The fewest query tiles for which the query-stationary kernel takes them
// (unless forced): half of all tiles, and twice the kernel's resident CTAs.
// A query tile walks its union block by block (~1.3 us per block on one
// CTA), so with fewer tiles than CTA slots the kernel's time is one long
// tile while the key-stationary path spreads the same work over every SM
// (B1 H8 D64 causal, N=4096: 0.172 ms through query tiles, 0.110 without).
int fine_q_min_tiles(const Shape& s, uint32_t flags) {
  if (flags & BSA_FLAG_FINE_QUERY_STATIONARY) return 1;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = kNumSMs;
  const int per_sm = (s.bs == 64) ? 2 : 1;     // QCfg<..>::kCtasPerSm
  const int64_t tiles_total = (int64_t)s.units * fine_q_tiles(s);
  const int64_t m = std::max<int64_t>((tiles_total + 1) / 2, 2LL * sms * per_sm);
  return (int)std::min<int64_t>(m, 1LL << 30);
}

cudaError_t launch_classify_tiles(const int32_t* idx, uint8_t* tile_mode, uint32_t* qt_bits,
                                  int4* qt_info, uint32_t* n_qt, const Shape& s, int max_union,
                                  cudaStream_t st) {
  const int tiles = fine_q_tiles(s);
  const int64_t grid = (int64_t)s.units * tiles;
  if (grid == 0) return cudaSuccess;
  const size_t smem = 32 * (size_t)((s.nb + 31) / 32);   // whole words of bytes
  auto kern = s.k <= 16 ? classify_tiles_kernel<16>
             : (s.k <= 32 ? classify_tiles_kernel<32> : classify_tiles_kernel<64>);
  kern<<<(unsigned)grid, kQRows, smem, st>>>(idx, tile_mode, qt_bits, qt_info, n_qt, s, tiles,
                                             max_union);
  return cudaGetLastError();
}

template <int BS, int HD>
static cudaError_t launch_q(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                            const FineQParams& prm, int64_t max_tiles, cudaStream_t st) {
  using C = QCfg<BS, HD>;
  const uint64_t rows = (uint64_t)prm.s.units * prm.s.N;
  CUtensorMap mq, mk, mv;
  if (!q_make_map(&mq, Q, rows, HD, kQRows) || !q_make_map(&mk, K, rows, HD, BS) ||
      !q_make_map(&mv, V, rows, HD, BS))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(fine_q_kernel<BS, HD>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = kNumSMs;
  int64_t grid = (int64_t)sms * C::kCtasPerSm;
  if (grid > max_tiles) grid = max_tiles;
  if (grid <= 0) return cudaSuccess;
  fine_q_kernel<BS, HD><<<(unsigned)grid, kQThreads, C::kSmem, st>>>(mq, mk, mv, prm);
  return cudaGetLastError();
}

cudaError_t launch_fine_q(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                          const int32_t* idx, __nv_bfloat16* O, const uint32_t* qt_bits,
                          const int4* qt_info, const uint32_t* n_qt, int min_q_tiles,
                          uint32_t* err, const Shape& s, cudaStream_t st) {
  FineQParams prm;
  prm.K = K;
  prm.V = V;
  prm.idx = idx;
  prm.qt_bits = qt_bits;
  prm.qt_info = qt_info;
  prm.n_qt = n_qt;
  prm.min_q_tiles = min_q_tiles;
  prm.O = O;
  prm.err = err;
  prm.s = s;
  const int64_t max_tiles = (int64_t)s.units * fine_q_tiles(s);
  if (s.bs == 64 && s.D == 64) return launch_q<64, 64>(Q, K, V, prm, max_tiles, st);
  if (s.bs == 64 && s.D == 128) return launch_q<64, 128>(Q, K, V, prm, max_tiles, st);
  if (s.bs == 128 && s.D == 64) return launch_q<128, 64>(Q, K, V, prm, max_tiles, st);
  return cudaErrorNotSupported;
}

}  // namespace bsa
