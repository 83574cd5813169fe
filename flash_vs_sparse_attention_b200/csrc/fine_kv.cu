// Stage 4 on tcgen05 tensor cores, key-block-stationary.
// (Replaces block_indexer.py:55-84 / the Triton kernel _fine_attn_fwd,
//  block_indexer_triton.py:12-83, with the same arithmetic.)
//
// Per-token selections barely overlap on unstructured inputs: the 64 queries
// of a query tile pick ~15x top_k distinct blocks between them, so a
// query-stationary tile would do nearly dense work.  Turned around, every key
// block is picked by ~N*top_k/num_blocks queries, which fills 128-row MMA
// tiles.  The stage therefore runs as:
//
//  1. bucket_count   per-unit histogram of the selected block ids
//  2. bucket_scan    per block: list offset and 128-query work items
//  3. bucket_scatter list entries (query row << 6 | slot) grouped by block
//  4. fine_kv        persistent kernel over work items.  For each item (one
//                    key block, <= 128 queries that picked it): TMA loads the
//                    block's K and V tiles, TMA gather4 loads the 128 query
//                    rows, tcgen05 computes S = Q K^T into TMEM, a softmax
//                    warpgroup turns its row of S into P (bf16, shared
//                    memory) with the row's max m and sum l, tcgen05 computes
//                    O = P V into TMEM, and the warpgroup writes the partial
//                    (O / l as bf16, m, l) for that (query, slot).
//  5. combine        per query: log-sum-exp merge of its top_k partials,
//                    rounded to bf16 once.
//
// fine_kv warp roles (320 threads): warps 0-3 and 4-7 are two softmax /
// epilogue warpgroups that take alternate work items (buffer g = item & 1), so
// one group's exponentials overlap the other's MMAs and stores; warp 8 issues
// TMA; one thread of warp 9 issues the MMAs.  All waits are bounded.
#include <cudaTypedefs.h>

#include <cstdio>

#include "common.cuh"
#include "launchers.cuh"
#include "sm100.cuh"

namespace bsa {

using namespace sm100;

constexpr int kTileRows = 128;      // queries per work item (MMA M)
constexpr int kRowsPerBucketCta = 1024;
constexpr int kMaxNbKv = 32768;

// Error codes ORed into the workspace error word.
enum : uint32_t {
  kErrWaitQ = 1u, kErrWaitS = 2u, kErrWaitP = 4u, kErrWaitO = 8u, kErrWaitFree = 16u,
  kErrWaitDrain = 32u
};

struct FineWs {
  int32_t* counts;     // units * nb
  int32_t* cursors;    // units * nb
  uint32_t* err;       // [0] error bits, [1] total work items
  int32_t* offsets;    // units * nb
  int4* items;         // units * max_items_per_unit
  int32_t* lists;      // units * N * k
  __nv_bfloat16* part_o;  // units * N * k * D
  float2* part_ml;     // units * N * k
  size_t zero_bytes;   // counts + cursors + err, contiguous from counts
  size_t total;
};

static size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

static int64_t max_items_per_unit(const Shape& s) {
  return ((int64_t)s.N * s.k + kTileRows - 1) / kTileRows + s.nb;
}

static FineWs fine_ws_layout(const Shape& s, unsigned char* base) {
  FineWs w;
  size_t off = 0;
  const size_t U = s.units, nb = s.nb, Nk = (size_t)s.N * s.k;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = a256(off + bytes);
    return base ? base + o : nullptr;
  };
  w.counts = (int32_t*)take(4 * U * nb);
  w.cursors = (int32_t*)take(4 * U * nb);
  w.err = (uint32_t*)take(16);
  w.zero_bytes = off;
  w.offsets = (int32_t*)take(4 * U * nb);
  w.items = (int4*)take(16 * U * (size_t)max_items_per_unit(s));
  w.lists = (int32_t*)take(4 * U * Nk);
  w.part_o = (__nv_bfloat16*)take(2 * U * Nk * s.D);
  w.part_ml = (float2*)take(8 * U * Nk);
  w.total = off;
  return w;
}

bool fine_kv_supported(const Shape& s) {
  const bool shape_ok = (s.bs == 64 && (s.D == 64 || s.D == 128)) || (s.bs == 128 && s.D == 64);
  return shape_ok && s.k <= 64 && s.nb <= kMaxNbKv && s.N < (1 << 25) &&
         (int64_t)s.units * s.N * s.k < (1LL << 31);
}

size_t fine_kv_workspace_bytes(const Shape& s) { return fine_ws_layout(s, nullptr).total; }

size_t fine_kv_zero_bytes(const Shape& s) { return fine_ws_layout(s, nullptr).zero_bytes; }

size_t fine_kv_error_offset(const Shape& s) {
  // counts and cursors precede the error word, each 256-byte aligned.
  return 2 * a256(4 * (size_t)s.units * s.nb);
}

// ---------------------------------------------------------------------------
// 1. Histogram of selected block ids per unit.
__global__ void __launch_bounds__(256)
bucket_count_kernel(const int32_t* __restrict__ idx, int32_t* __restrict__ counts, Shape s) {
  extern __shared__ int32_t hist[];
  const int u = blockIdx.y;
  for (int j = threadIdx.x; j < s.nb; j += blockDim.x) hist[j] = 0;
  __syncthreads();
  const int64_t row0 = (int64_t)blockIdx.x * kRowsPerBucketCta;
  const int64_t e0 = ((int64_t)u * s.N + row0) * s.k;
  const int64_t ne = (int64_t)min((int64_t)kRowsPerBucketCta, s.N - row0) * s.k;
  for (int64_t e = threadIdx.x; e < ne; e += blockDim.x) {
    int j = idx[e0 + e];
    if (j >= 0) atomicAdd(&hist[j], 1);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < s.nb; j += blockDim.x)
    if (hist[j]) atomicAdd(&counts[(int64_t)u * s.nb + j], hist[j]);
}

// 2. Per unit: exclusive scan of counts -> list offsets, and work items of at
//    most 128 queries per block.  One CTA of 1024 threads per unit.
__global__ void __launch_bounds__(1024)
bucket_scan_kernel(const int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                   int4* __restrict__ items, uint32_t* __restrict__ err, Shape s,
                   int64_t max_items) {
  __shared__ int32_t wsum_c[32], wsum_t[32];
  __shared__ int32_t item_base;
  const int u = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (s.nb + blockDim.x - 1) / blockDim.x;
  const int j0 = tid * per, j1 = min(s.nb, j0 + per);
  const int32_t* c = counts + (int64_t)u * s.nb;
  int sc = 0, st = 0;
  for (int j = j0; j < j1; ++j) {
    sc += c[j];
    st += (c[j] + kTileRows - 1) / kTileRows;
  }
  // Block-wide exclusive scans of (sc, st).
  int ic = sc, it = st;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int a = __shfl_up_sync(0xffffffffu, ic, o), b = __shfl_up_sync(0xffffffffu, it, o);
    if (lane >= o) { ic += a; it += b; }
  }
  if (lane == 31) { wsum_c[warp] = ic; wsum_t[warp] = it; }
  __syncthreads();
  if (warp == 0) {
    int a = wsum_c[lane], b = wsum_t[lane];
    int ia = a, ib = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int x = __shfl_up_sync(0xffffffffu, ia, o), y = __shfl_up_sync(0xffffffffu, ib, o);
      if (lane >= o) { ia += x; ib += y; }
    }
    wsum_c[lane] = ia - a;
    wsum_t[lane] = ib - b;
    if (lane == 31) item_base = (int)atomicAdd(&err[1], (uint32_t)ib);
  }
  __syncthreads();
  int oc = wsum_c[warp] + ic - sc;   // exclusive prefix of this thread's chunk
  int ot = wsum_t[warp] + it - st;
  const int64_t list_base = (int64_t)u * s.N * s.k;
  int4* out = items + item_base;
  for (int j = j0; j < j1; ++j) {
    const int cj = c[j];
    offsets[(int64_t)u * s.nb + j] = oc;
    for (int t = 0; t * kTileRows < cj; ++t) {
      out[ot++] = make_int4(u, j, (int)(list_base + oc + t * kTileRows), min(kTileRows, cj - t * kTileRows));
    }
    oc += cj;
  }
  (void)max_items;
}

// 3. List entries grouped by block: entry = query_row << 6 | slot.
__global__ void __launch_bounds__(256)
bucket_scatter_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ offsets,
                      int32_t* __restrict__ cursors, int32_t* __restrict__ lists, Shape s) {
  extern __shared__ int32_t hist[];
  const int u = blockIdx.y;
  for (int j = threadIdx.x; j < s.nb; j += blockDim.x) hist[j] = 0;
  __syncthreads();
  const int64_t row0 = (int64_t)blockIdx.x * kRowsPerBucketCta;
  const int64_t e0 = ((int64_t)u * s.N + row0) * s.k;
  const int64_t ne = (int64_t)min((int64_t)kRowsPerBucketCta, s.N - row0) * s.k;
  for (int64_t e = threadIdx.x; e < ne; e += blockDim.x) {
    int j = idx[e0 + e];
    if (j >= 0) atomicAdd(&hist[j], 1);
  }
  __syncthreads();
  // Reserve this CTA's range in every block's list.
  for (int j = threadIdx.x; j < s.nb; j += blockDim.x) {
    int n = hist[j];
    if (n) {
      int64_t g = (int64_t)u * s.nb + j;
      hist[j] = offsets[g] + atomicAdd(&cursors[g], n);
    }
  }
  __syncthreads();
  int32_t* ul = lists + (int64_t)u * s.N * s.k;
  for (int64_t e = threadIdx.x; e < ne; e += blockDim.x) {
    int j = idx[e0 + e];
    if (j >= 0) {
      int pos = atomicAdd(&hist[j], 1);
      int64_t le = row0 * s.k + e;  // entry index within the unit
      int row = (int)(le / s.k), slot = (int)(le % s.k);
      ul[pos] = (row << 6) | slot;
    }
  }
}

// ---------------------------------------------------------------------------
// 4. The tensor-core fine kernel.
//
// Warps (NWG = 3 softmax warpgroups when TMEM holds three (S, O) pairs, else 2):
//   0 .. 4*NWG-1  softmax/epilogue: warpgroup w takes the items t with
//                 t % NWG == w and owns TMEM S[w] (P overwrites it as bf16)
//                 and O[w]; several items in flight hide each one's latency
//   4*NWG .. +2   three loader warps: gather the item's 128 query rows with
//                 16-byte cp.async, HD/8 lanes per row so each instruction
//                 moves whole rows (random 128-byte rows stream faster through
//                 the LSU path than TMA gather4 issues them, and three warps
//                 keep enough of them in flight), and stage the item's list
//                 entries (and the item) for the other warps.  The first
//                 loader's lane 0 also issues the TMA loads of K and V, once
//                 per run of consecutive items on the same key block (items
//                 are sorted by block), into one of NKV >= NWG slots.  After
//                 S(t) the stage holds the item's output rows, which the
//                 warpgroup stores row-coalesced before releasing the stage
//   4*NWG+3       one thread issues the MMAs: S(0..NWG-1), then PV(t) followed
//                 by S(t + NWG), which reuses the TMEM PV(t) has just read
// Shared memory: NQ query stages (gathered rows + entries), NKV K/V slots.
template <int BS, int HD>
struct KvCfg {
  static constexpr int NWG = (BS + HD <= 128) ? 3 : 2;
  static constexpr int kQBytes = kTileRows * HD * 2;   // gathered queries
  static constexpr int NQ = (HD == 64) ? 8 : 4;          // query stages
  static constexpr int kKBytes = BS * HD * 2;
  static constexpr int kKVBytes = 2 * kKBytes;           // one block's K and V
  // K/V slots.  Items t .. t+NWG-1 (the S MMAs issued ahead of PV(t)) can
  // belong to NWG different block runs that must all be resident while PV(t)
  // is pending, so NKV >= NWG is required (fewer slots deadlock); one more
  // lets the next run load early when shared memory allows.
  static constexpr int NKV =
      (NQ * kQBytes + (NWG + 1) * kKVBytes + 24 * 1024 <= 220 * 1024) ? NWG + 1 : NWG;
  static constexpr int kMetaBytes = kTileRows * 4 + 16;  // entries + item
  static constexpr int kRing = 256;                      // staged work items per loader warp
  static constexpr int kLoaderWarps = 3;
  static constexpr int kKVOff = NQ * kQBytes;
  static constexpr int kMetaOff = kKVOff + NKV * kKVBytes;
  static constexpr int kRingOff = kMetaOff + NQ * kMetaBytes;
  static constexpr int kGenOff = kRingOff + kLoaderWarps * kRing * 16;   // MMA's block-run ids
  static constexpr int kGenRing = 16;
  static constexpr int kBarOff = kGenOff + kGenRing * 4;
  static constexpr int kSmem = kBarOff + 512 + 1024 /*align*/;
  static constexpr int kTmemCols = 512;
  static constexpr int kThreads = (4 * NWG + kLoaderWarps + 1) * 32;
  // q_full completes on each loader thread's cp.async-landed arrive plus one
  // entries-written arrive per loader warp.
  static constexpr int kQFullCount = kLoaderWarps * 33;
  static_assert(NWG * (BS + HD) <= 512, "TMEM holds NWG (S, O) pairs");
  static_assert(kGenRing > NWG + 1, "the MMA thread looks one item ahead");
};

struct FineKvParams {
  const __nv_bfloat16* q;
  const int4* items;
  const int32_t* lists;
  const uint32_t* total_items;  // device word written by bucket_scan
  __nv_bfloat16* part_o;
  float2* part_ml;
  uint32_t* err;
  Shape s;
};

template <int BS, int HD>
__global__ void __launch_bounds__(KvCfg<BS, HD>::kThreads, 1)
fine_kv_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
               FineKvParams prm) {
  using C = KvCfg<BS, HD>;
  constexpr int NQ = C::NQ, NWG = C::NWG;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::kBarOff);
  uint64_t* q_full = bars;                      // [NQ] rows + entries of the stage's item landed
  uint64_t* q_empty = q_full + NQ;              // [NQ] stage free: the item's epilogue, which
                                                //      stages its output rows there, is done
  uint64_t* kv_full = q_empty + NQ;             // [NKV] K, V of a block run landed
  uint64_t* kv_empty = kv_full + C::NKV;        // [NKV] last PV of a block run done
  uint64_t* s_full = kv_empty + C::NKV;         // [NWG] S in TMEM
  uint64_t* p_full = s_full + NWG;              // [NWG] P in TMEM (128 arrivals)
  uint64_t* o_full = p_full + NWG;              // [NWG] O in TMEM
  uint64_t* o_free = o_full + NWG;              // [NWG] O read out (128 arrivals)
  uint64_t* drain = o_free + NWG;
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(drain + 2);
  int4* ring = (int4*)(smem + C::kRingOff);
  int* gen_ring = (int*)(smem + C::kGenOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w_load = 4 * NWG, w_mma = 4 * NWG + C::kLoaderWarps;
  const Shape s = prm.s;
  const uint32_t total = *prm.total_items;
  const uint32_t G = gridDim.x;
  const uint32_t t_begin = (uint32_t)(((uint64_t)total * blockIdx.x) / G);
  const uint32_t t_end = (uint32_t)(((uint64_t)total * (blockIdx.x + 1)) / G);
  const int T = (int)(t_end - t_begin);
  if (T <= 0) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NQ; ++i) {
      mbar_init(&q_full[i], C::kQFullCount);
      mbar_init(&q_empty[i], 128);
    }
    for (int i = 0; i < C::NKV; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int g = 0; g < NWG; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 128);
      mbar_init(&o_full[g], 1);
      mbar_init(&o_free[g], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == w_load && lane == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  if (warp == 0) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  auto q_s = [&](int st) { return smem + st * C::kQBytes; };
  auto k_s = [&](int slot) { return smem + C::kKVOff + slot * C::kKVBytes; };
  auto v_s = [&](int slot) { return smem + C::kKVOff + slot * C::kKVBytes + C::kKBytes; };
  auto meta = [&](int st) { return (int32_t*)(smem + C::kMetaOff + st * C::kMetaBytes); };
  const float sc = s.scale * kLog2e;

  if (warp >= w_load && warp < w_mma) {
    // ------------------------------------------------------------ Q loaders (+ K/V TMA)
    // Loader L handles rows r = i*3*RPI + L*RPI + lane/CPR: CPR = HD/8 lanes
    // per row, RPI = 32/CPR whole rows per instruction.  Each warp keeps its
    // own ring of the next work items, refilled half a ring at a time.
    constexpr int CPR = HD / 8, RPI = 32 / CPR, NLW = C::kLoaderWarps;
    constexpr int ROWS = (kTileRows + NLW * RPI - 1) / (NLW * RPI);   // rows per lane
    const int L = warp - w_load;
    const int chunk = lane % CPR, panel = chunk >> 3, cc = chunk & 7;
    int4* my_ring = ring + L * C::kRing;
    auto fill = [&](int base, int count) {   // items base .. base + count - 1
      for (int q = lane; q < count; q += 32)
        if (base + q < T) my_ring[(base + q) % C::kRing] = prm.items[t_begin + base + q];
      __syncwarp();
    };
    auto row_of = [&](int i) { return i * NLW * RPI + L * RPI + lane / CPR; };
    struct Ent { int32_t e[ROWS]; };
    auto entries = [&](int t, Ent& E) {
      if (t >= T) return;
      const int4 it = my_ring[t % C::kRing];
#pragma unroll
      for (int i = 0; i < ROWS; ++i) {
        const int r = row_of(i);
        E.e[i] = (r < kTileRows) ? prm.lists[it.z + (r < it.w ? r : 0)] : 0;
      }
    };
    fill(0, C::kRing);
    Ent E0, E1;
    entries(0, E0);
    entries(1, E1);
    int gen = -1, px = -1, py = -1;   // K/V runs (first loader, lane 0)
    auto step = [&](int t, Ent& E) -> bool {
      const int st = t % NQ, use = t / NQ;
      const int4 it = my_ring[t % C::kRing];
      int32_t e[ROWS];
#pragma unroll
      for (int i = 0; i < ROWS; ++i) e[i] = E.e[i];
      if (use >= 1) {
        bool ok = mbar_wait(&q_empty[st], (use - 1) & 1, prm.err, kErrWaitFree);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || *abort_flag) { *abort_flag = 1; return false; }
      }
      // Rows past the item's count gather its first query again (never stored).
      int32_t* m = meta(st);
      const unsigned char* qbase = reinterpret_cast<const unsigned char*>(prm.q) +
                                   (int64_t)it.x * s.N * (HD * 2) + chunk * 16;
#pragma unroll
      for (int i = 0; i < ROWS; ++i) {
        const int r = row_of(i);
        if (r < kTileRows) {
          if (chunk == 0) m[r] = e[i];
          cp_async16(q_s(st) + panel * (kTileRows * 128) + r * 128 + ((cc ^ (r & 7)) << 4),
                     qbase + (int64_t)(e[i] >> 6) * (HD * 2));
        }
      }
      if (L == 0 && lane == 0) reinterpret_cast<int4*>(m + kTileRows)[0] = it;
      cp_async_arrive_noinc(&q_full[st]);   // this lane's rows landed
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_full[st]);  // this warp's entries (and the item) visible
      // K and V of a new block run, into slot run % NKV once that slot's
      // previous run is done.
      if (L == 0 && lane == 0 && (it.x != px || it.y != py)) {
        px = it.x;
        py = it.y;
        ++gen;
        const int slot = gen % C::NKV, kuse = gen / C::NKV;
        if (kuse >= 1 && (!mbar_wait(&kv_empty[slot], (kuse - 1) & 1, prm.err, kErrWaitFree) ||
                          *abort_flag)) {
          *abort_flag = 1;
        } else {
          mbar_arrive_expect_tx(&kv_full[slot], C::kKVBytes);
          const int32_t y = it.x * s.N + it.y * BS;
#pragma unroll
          for (int p = 0; p < HD / 64; ++p) {
            tma_load_2d(k_s(slot) + p * (BS * 128), &tmap_k, &kv_full[slot], p * 64, y);
            tma_load_2d(v_s(slot) + p * (BS * 128), &tmap_v, &kv_full[slot], p * 64, y);
          }
        }
      }
      __syncwarp();
      if (*abort_flag) return false;
      // Entering a new half ring: the half before it is done, so refill that
      // half with the items one ring ahead.  Then load item t + 2's entries.
      constexpr int H = C::kRing / 2;
      if (t % H == H - 1) fill(t + 1 + H, H);
      entries(t + 2, E);
      return true;
    };
    for (int t = 0; t < T; t += 2) {
      if (!step(t, E0)) break;
      if (t + 1 < T && !step(t + 1, E1)) break;
    }
  } else if (warp == w_mma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(kTileRows, BS, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(kTileRows, HD, true);
      // Descriptors at stage / slot 0; the start-address field (bits 0-13,
      // address >> 4) is advanced by adding byte offsets >> 4.
      const uint64_t dq0 = smem_desc_sw128(smem_u32(q_s(0)), 16, 1024);
      const uint64_t dk0 = smem_desc_sw128(smem_u32(k_s(0)), 16, 1024);
      const uint64_t dv0 = smem_desc_sw128(smem_u32(v_s(0)), BS * 128, 1024);
      int gen = -1, px = -1, py = -1;
      auto issue_s = [&](int t) -> bool {
        const int st = t % NQ;
        if (!mbar_wait(&q_full[st], (t / NQ) & 1, prm.err, kErrWaitQ)) return false;
        const int4 it = reinterpret_cast<const int4*>(meta(st) + kTileRows)[0];
        if (it.x != px || it.y != py) {
          ++gen;
          px = it.x;
          py = it.y;
        }
        gen_ring[t % C::kGenRing] = gen;
        const int slot = gen % C::NKV;
        if (!mbar_wait(&kv_full[slot], (gen / C::NKV) & 1, prm.err, kErrWaitQ)) return false;
        tc_fence_after();
        const uint32_t d = tbase + (t % NWG) * (BS + HD);
        const uint64_t dq = dq0 + ((st * C::kQBytes) >> 4);
        const uint64_t dk = dk0 + ((slot * C::kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kTileRows * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (BS * 128) + (kk & 3) * 32;
          mma_bf16(d, dq + (off >> 4), dk + (offk >> 4), idesc_s, kk > 0);
        }
        mma_commit(&s_full[t % NWG]);
        return true;
      };
      auto issue_o = [&](int t) -> bool {
        const int w = t % NWG, n = t / NWG;
        if (!mbar_wait(&p_full[w], n & 1, prm.err, kErrWaitP)) return false;
        if (n >= 1 && !mbar_wait(&o_free[w], (n - 1) & 1, prm.err, kErrWaitFree)) return false;
        tc_fence_after();
        const int g = gen_ring[t % C::kGenRing];
        const int slot = g % C::NKV;
        const uint32_t d = tbase + w * (BS + HD) + BS;
        const uint32_t pa = tbase + w * (BS + HD);   // P: bf16 pairs over S's first BS/2 columns
        const uint64_t dv = dv0 + ((slot * C::kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < BS / 16; ++kk)
          mma_bf16_ts(d, pa + kk * 8, dv + ((kk * 16 * 128) >> 4), idesc_o, kk > 0);
        mma_commit(&o_full[w]);
        // The run's last item frees its K/V slot.  S(t + 1) is already
        // issued (NWG >= 2), so its run id is known.
        if (t + 1 == T || gen_ring[(t + 1) % C::kGenRing] != g) mma_commit(&kv_empty[slot]);
        return true;
      };
      bool ok = true;
      for (int t = 0; ok && t < NWG && t < T; ++t) ok = issue_s(t);
      for (int t = 0; ok && t < T; ++t) {
        ok = issue_o(t);
        if (ok && t + NWG < T) ok = issue_s(t + NWG);
        if (*abort_flag) ok = false;
      }
      if (!ok) *abort_flag = 1;
      // Make sure no MMA is in flight when TMEM is released.
      mma_commit(drain);
      mbar_wait(drain, 0, prm.err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp < 4 * NWG) {
    // ------------------------------------------------------------ softmax / epilogue
    const int wg = warp >> 2;              // takes items t with t % NWG == wg
    const int quad = warp & 3;             // TMEM lane quadrant
    const int r = quad * 32 + lane;        // row of the tile this thread owns
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tbase + lane_off + wg * (BS + HD);
    const uint32_t o_addr = s_addr + BS;
    for (int t = wg; t < T; t += NWG) {
      const int n = t / NWG, st = t % NQ;
      bool ok = mbar_wait(&q_full[st], (t / NQ) & 1, prm.err, kErrWaitQ);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) { *abort_flag = 1; break; }
      const int32_t* m = meta(st);
      const int4 it = reinterpret_cast<const int4*>(m + kTileRows)[0];
      const int u = it.x, j = it.y, cnt = it.w;
      const bool valid = r < cnt;
      const int32_t e = m[r];
      const int qrow = e >> 6, slot = e & 63;

      ok = mbar_wait(&s_full[wg], n & 1, prm.err, kErrWaitS);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const int key0 = j * BS;
      const bool diag = s.causal && key0 + BS - 1 > qrow;
      float sv[64];
      auto load_s = [&](int c0) {
        tmem_ld64(s_addr + c0, sv);
        // Token-level causal mask (block_indexer.py:73-81): key > query -> -inf.
        if (diag) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (key0 + c0 + c > qrow) sv[c] = -INFINITY;
        }
      };
      float mx = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < BS; c0 += 64) {
        load_s(c0);
        float m0 = sv[0], m1 = sv[1], m2 = sv[2], m3 = sv[3];
#pragma unroll
        for (int c = 4; c < 64; c += 4) {
          m0 = fmaxf(m0, sv[c]); m1 = fmaxf(m1, sv[c + 1]);
          m2 = fmaxf(m2, sv[c + 2]); m3 = fmaxf(m3, sv[c + 3]);
        }
        mx = fmaxf(mx, fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)));
      }
      // Padding rows of a short item can be fully masked; keep them finite.
      const float msc = (mx == -INFINITY) ? 0.f : mx * sc;
      float l0 = 0.f, l1 = 0.f;
#pragma unroll
      for (int c0 = 0; c0 < BS; c0 += 64) {
        if (BS > 64) load_s(c0);   // with one chunk the values are still in sv
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float p0 = fast_exp2(fmaf(sv[c], sc, -msc));
          const float p1 = fast_exp2(fmaf(sv[c + 1], sc, -msc));
          l0 += p0;
          l1 += p1;
          pk[c >> 1] = pack_bf16x2(p0, p1);
        }
        // P (bf16 pairs) overwrites the S columns this chunk has consumed.
        tmem_st32(s_addr + (c0 >> 1), pk);
      }
      const float l = l0 + l1;
      tc_fence_before();
      mbar_arrive(&p_full[wg]);

      ok = mbar_wait(&o_full[wg], n & 1, prm.err, kErrWaitO);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const float inv = 1.f / l;
      // The item's query rows are consumed (S(t) is done), so its stage holds
      // the output rows for a coalesced store: row r, chunk c at the same
      // swizzled place a gathered query chunk occupied.
      unsigned char* stage = q_s(st);
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 64) {
        float ov[64];
        tmem_ld64(o_addr + c0, ov);
        if (c0 + 64 >= HD) {
          tc_fence_before();
          mbar_arrive(&o_free[wg]);
        }
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          const int ch = c >> 3;
          *reinterpret_cast<uint4*>(stage + (c0 >> 6) * (kTileRows * 128) + r * 128 +
                                    ((ch ^ (r & 7)) << 4)) =
              make_uint4(pack_bf16x2(ov[c] * inv, ov[c + 1] * inv),
                         pack_bf16x2(ov[c + 2] * inv, ov[c + 3] * inv),
                         pack_bf16x2(ov[c + 4] * inv, ov[c + 5] * inv),
                         pack_bf16x2(ov[c + 6] * inv, ov[c + 7] * inv));
        }
      }
      const int64_t pe = ((int64_t)u * s.N + qrow) * s.k + slot;
      if (valid) prm.part_ml[pe] = make_float2(msc, l);
      __syncwarp();
      {
        // This warp's 32 rows, 32 / CPR whole rows per instruction.
        constexpr int CPR = HD / 8, RPI = 32 / CPR;
        const int chunk = lane % CPR, panel = chunk >> 3, cc = chunk & 7;
#pragma unroll 4
        for (int i = 0; i < 32 / RPI; ++i) {
          const int rr = quad * 32 + i * RPI + lane / CPR;
          if (rr < cnt) {
            const int32_t er = m[rr];
            const int64_t pr = ((int64_t)u * s.N + (er >> 6)) * s.k + (er & 63);
            const uint4 v = *reinterpret_cast<const uint4*>(
                stage + panel * (kTileRows * 128) + rr * 128 + ((cc ^ (rr & 7)) << 4));
            reinterpret_cast<uint4*>(prm.part_o + pr * HD)[chunk] = v;
          }
        }
      }
      __syncwarp();
      mbar_arrive(&q_empty[st]);   // this thread is done with the stage
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, C::kTmemCols);
}

// 5. Per query: merge its partials (m in the base-2 domain, l, O / l).
template <int HD>
__global__ void __launch_bounds__(256)
combine_kernel(const int32_t* __restrict__ idx, const __nv_bfloat16* __restrict__ part_o,
               const float2* __restrict__ part_ml, __nv_bfloat16* __restrict__ O, Shape s) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t R = gid / CH;  // global query row (unit * N + row)
  const int c = (int)(gid % CH);
  if (R >= (int64_t)s.units * s.N) return;
  const int32_t* sel = idx + R * s.k;
  float M = -INFINITY;
  for (int q = 0; q < s.k; ++q)
    if (__ldg(sel + q) >= 0) M = fmaxf(M, __ldg(&part_ml[R * s.k + q].x));
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float L = 0.f;
  for (int q = 0; q < s.k; ++q) {
    if (__ldg(sel + q) < 0) continue;
    const float2 ml = __ldg(&part_ml[R * s.k + q]);
    const float w = ml.y * fast_exp2(ml.x - M);
    L += w;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(part_o + (R * s.k + q) * HD) + c);
    acc[0] = fmaf(w, bf16_lo(v.x), acc[0]); acc[1] = fmaf(w, bf16_hi(v.x), acc[1]);
    acc[2] = fmaf(w, bf16_lo(v.y), acc[2]); acc[3] = fmaf(w, bf16_hi(v.y), acc[3]);
    acc[4] = fmaf(w, bf16_lo(v.z), acc[4]); acc[5] = fmaf(w, bf16_hi(v.z), acc[5]);
    acc[6] = fmaf(w, bf16_lo(v.w), acc[6]); acc[7] = fmaf(w, bf16_hi(v.w), acc[7]);
  }
  const float inv = 1.f / L;
  reinterpret_cast<uint4*>(O + R * HD)[c] =
      make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                 pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
}

// ---------------------------------------------------------------------------
// Host side.
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// 2-D bf16 tensor map over a row-major (rows, cols) matrix, 128-byte swizzle,
// box of 64 columns x box_rows rows.
static bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                     uint32_t box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = kNumSMs;
  }
  return n;
}

template <int BS, int HD>
static cudaError_t launch_kv_kernel(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                                    const __nv_bfloat16* V, const FineWs& w, const Shape& s,
                                    cudaStream_t st) {
  using C = KvCfg<BS, HD>;
  CUtensorMap mk, mv;
  const uint64_t rows = (uint64_t)s.units * s.N;
  if (!make_map(&mk, K, rows, HD, BS) || !make_map(&mv, V, rows, HD, BS))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(fine_kv_kernel<BS, HD>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return e;
  FineKvParams prm;
  prm.q = Q;
  prm.items = w.items;
  prm.lists = w.lists;
  prm.total_items = w.err + 1;
  prm.part_o = w.part_o;
  prm.part_ml = w.part_ml;
  prm.err = w.err;
  prm.s = s;
  fine_kv_kernel<BS, HD><<<num_sms(), C::kThreads, C::kSmem, st>>>(mk, mv, prm);
  return cudaGetLastError();
}

cudaError_t launch_fine_kv(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                           const __nv_bfloat16* V, const int32_t* idx, __nv_bfloat16* O,
                           unsigned char* ws, const Shape& s, cudaStream_t st, int* n_launches,
                           void* const* events, int n_events, bool pre_zeroed) {
  FineWs w = fine_ws_layout(s, ws);
  auto mark = [&](int i) {
    if (events != nullptr && i < n_events && events[i] != nullptr)
      cudaEventRecord((cudaEvent_t)events[i], st);
  };
  cudaError_t e = cudaSuccess;
  if (!pre_zeroed && (e = cudaMemsetAsync(w.counts, 0, w.zero_bytes, st)) != cudaSuccess) return e;
  const size_t hist_smem = sizeof(int32_t) * s.nb;
  dim3 bgrid((s.N + kRowsPerBucketCta - 1) / kRowsPerBucketCta, s.units);
  if (hist_smem > 48 * 1024) {
    cudaFuncSetAttribute(bucket_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)hist_smem);
    cudaFuncSetAttribute(bucket_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)hist_smem);
  }
  bucket_count_kernel<<<bgrid, 256, hist_smem, st>>>(idx, w.counts, s);
  bucket_scan_kernel<<<s.units, 1024, 0, st>>>(w.counts, w.offsets, w.items, w.err, s,
                                               max_items_per_unit(s));
  bucket_scatter_kernel<<<bgrid, 256, hist_smem, st>>>(idx, w.offsets, w.cursors, w.lists, s);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  mark(2);
  if (s.bs == 64 && s.D == 64) e = launch_kv_kernel<64, 64>(Q, K, V, w, s, st);
  else if (s.bs == 64 && s.D == 128) e = launch_kv_kernel<64, 128>(Q, K, V, w, s, st);
  else if (s.bs == 128 && s.D == 64) e = launch_kv_kernel<128, 64>(Q, K, V, w, s, st);
  else e = cudaErrorNotSupported;
  if (e != cudaSuccess) return e;
  mark(3);
  const int64_t threads = (int64_t)s.units * s.N * (s.D / 8);
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (s.D == 64) combine_kernel<64><<<blocks, 256, 0, st>>>(idx, w.part_o, w.part_ml, O, s);
  else combine_kernel<128><<<blocks, 256, 0, st>>>(idx, w.part_o, w.part_ml, O, s);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  mark(4);
  *n_launches = 5;
  return cudaSuccess;
}

}  // namespace bsa
