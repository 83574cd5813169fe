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
//  1. bucket_count   per chunk of rows, the histogram of its selected blocks
//                    and where the chunk's entries of each block start in
//                    that block's list; the unit's last chunk to finish then
//                    lays out the unit: per block its list offset and work
//                    items of at most 128 queries
//  2. bucket_scatter per block, the query rows that picked it (its list), and
//                    for every (query, slot) the partial row its result goes
//                    to: work item i owns partial rows [128 i, 128 i + 128)
//  4. fine_kv        persistent kernel over work items.  For each item (one
//                    key block, <= 128 queries that picked it): TMA gather4
//                    loads the 128 query rows, TMA loads the block's K and V
//                    (once per run of items on the same block), tcgen05
//                    computes S = Q K^T into TMEM, a softmax warpgroup turns
//                    it into P (bf16, TMEM) with each row's max m and sum l,
//                    tcgen05 computes O = P V into TMEM, and the warpgroup
//                    stores the item's partial tile (O as fp16, m, l) with
//                    TMA stores: 128 contiguous rows per item.
//  5. combine        per query: log-sum-exp merge of its top_k partials,
//                    rounded to bf16 once.
//
// Partial outputs are fp16 with a power-of-two scale per key block: 2^e with
// bs * max|V of the block| * 2^e <= 2^14, so |O 2^e| <= 2^14 for any row
// (P <= 1).  The scale is folded into the softmax shift (P 2^e costs no extra
// instruction) and into the stored m and l, so the combine needs no
// per-partial exponent.  fp16 keeps 11 significant bits where bf16 keeps 8:
// the output is then rounded to bf16 essentially once, as in the reference's
// single bf16 store (block_indexer_triton.py:81-83).  bucket_count computes
// the per-block exponents (max|V| over the block's bs x D values) as a side
// job of its CTAs.
//
// All waits are bounded (a stuck pipeline ends with an error word, not a
// hang).  Warp roles and the barrier discipline are described at KvCfg.
#include <cudaTypedefs.h>

#include <cstdio>

#include "common.cuh"
#include "launchers.cuh"
#include "sm100.cuh"

namespace bsa {

using namespace sm100;

constexpr int kTileRows = 128;      // queries per work item (MMA M)
constexpr int kMaxNbKv = 16384;
// Bucket kernels: a CTA of kBucketThreads handles one chunk of a unit's rows,
// in batches of kBucketBatch (query, slot) entries held in registers
// (kBucketPer per thread).  A unit has at most kMaxChunksPerUnit chunks.
constexpr int kBucketThreads = 512;
constexpr int kBucketBatch = 16384;
constexpr int kBucketPer = kBucketBatch / kBucketThreads;
constexpr int kMaxChunksPerUnit = 64;
constexpr int kRowBits = 14;   // staged entry: block << kRowBits | row in batch

// Error codes ORed into the workspace error word.
enum : uint32_t {
  kErrWaitQ = 1u, kErrWaitS = 2u, kErrWaitP = 4u, kErrWaitO = 8u, kErrWaitFree = 16u,
  kErrWaitDrain = 32u, kErrWaitKV = 128u, kErrWaitEnt = 256u, kErrTestTimeout = 512u
};

struct FineWs {
  uint32_t* err;       // [0] error bits (16 bytes)                  } zeroed before
  uint32_t* ctr;       // [0] total work items, [2] query tiles       } the stage (the
                       //                                                error word only
                       //                                                before the first
                       //                                                pass of a call)
  int32_t* done;       // units: chunks counted so far                } the stage
  int32_t* cursor;     // units * nb: entries of each block so far    }
  int32_t* chunk_rel;  // units * chunks * nb: start of (chunk, block) within the block's list
  int32_t* offsets;    // units * nb: a block's first position in its unit's list
  int32_t* item_row;   // units * nb: 128 * (a block's first work item)
  int32_t* vexp;       // units * nb: the block's partial-output scale exponent
  uint8_t* tile_mode;  // units * tiles: 1 = the 128-row tile is a query tile (fine_q.cu)
  int4* qt_info;       // units * tiles: (unit, tile, union size) of query-tile slot i
  uint32_t* qt_bits;   // units * tiles * nbw: the union bitmask of slot i
  int4* items;         // units * max_items_per_unit
  int32_t* lists;      // units * N * k: query rows grouped by block
  int32_t* inv;        // units * N * k: (query, slot) -> partial row
  __half* part_o;      // 128 rows per work item, D columns (fp16, scaled)
  float2* part_ml;     // 128 rows per work item
  size_t zero_bytes;   // err, ctr, done and cursor, at the start of the region
  int64_t part_rows;   // rows of part_o / part_ml
  size_t total;
};

static size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

// The query tiles as the bucket kernels and the combine see them: the tile
// marks count only when the query tiles are at least min_count of the tiles
// (device word *count from the classifier); otherwise every tile takes the
// key-block-stationary path.
struct QTiles {
  const uint8_t* mode;     // units * tiles, or null: no query tiles
  const uint32_t* count;
  int min_count;
};

__device__ __forceinline__ const uint8_t* active_tile_mode(const QTiles& q) {
  return (q.mode != nullptr && *q.count >= (uint32_t)q.min_count) ? q.mode : nullptr;
}

// How the bucket kernels cut a unit's rows: batches of rows_batch rows
// (rows_batch * k <= kBucketBatch entries), chunks of whole batches.
struct BucketGeom {
  int rows_batch;
  int chunk_rows;
  int chunks;
};

static BucketGeom bucket_geom(const Shape& s) {
  BucketGeom g;
  g.rows_batch = kBucketBatch / s.k;
  const int batches = (s.N + g.rows_batch - 1) / g.rows_batch;
  g.chunk_rows = g.rows_batch * ((batches + kMaxChunksPerUnit - 1) / kMaxChunksPerUnit);
  g.chunks = (s.N + g.chunk_rows - 1) / g.chunk_rows;
  return g;
}

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
  w.part_rows = (int64_t)U * max_items_per_unit(s) * kTileRows;
  w.err = (uint32_t*)take(16);
  w.ctr = (uint32_t*)take(16);
  w.done = (int32_t*)take(4 * U);
  w.cursor = (int32_t*)take(4 * U * nb);
  w.zero_bytes = off;
  w.chunk_rel = (int32_t*)take(4 * U * (size_t)bucket_geom(s).chunks * nb);
  w.offsets = (int32_t*)take(4 * U * nb);
  w.item_row = (int32_t*)take(4 * U * nb);
  w.vexp = (int32_t*)take(4 * U * nb);
  {
    const size_t tiles = (size_t)(s.N + kTileRows - 1) / kTileRows, nbw = (nb + 31) / 32;
    w.tile_mode = (uint8_t*)take(U * tiles);
    w.qt_info = (int4*)take(16 * U * tiles);
    w.qt_bits = (uint32_t*)take(4 * U * tiles * nbw);
  }
  w.items = (int4*)take(16 * U * (size_t)max_items_per_unit(s));
  w.lists = (int32_t*)take(4 * (U * Nk + 256));   // slack for aligned list-slice copies
  w.inv = (int32_t*)take(4 * U * Nk);
  w.part_o = (__half*)take(2 * (size_t)w.part_rows * s.D);
  w.part_ml = (float2*)take(8 * (size_t)w.part_rows);
  w.total = off;
  return w;
}

bool fine_kv_supported(const Shape& s) {
  const bool shape_ok = (s.bs == 64 && (s.D == 64 || s.D == 128)) || (s.bs == 128 && s.D == 64);
  // Partial rows (128 per work item) are addressed with int32.
  const int64_t part_rows = (int64_t)s.units * max_items_per_unit(s) * kTileRows;
  return shape_ok && s.k <= 64 && s.nb <= kMaxNbKv && part_rows < (1LL << 31) &&
         (int64_t)s.units * s.N * s.k < (1LL << 31);
}

size_t fine_kv_workspace_bytes(const Shape& s) { return fine_ws_layout(s, nullptr).total; }

size_t fine_kv_zero_bytes(const Shape& s) { return fine_ws_layout(s, nullptr).zero_bytes; }

size_t fine_kv_error_offset(const Shape&) { return 0; }   // the error word leads the region

// The per-pass counters follow the error word's region: a later pass of one
// call clears from here, so an earlier pass's error bits survive to the end.
size_t fine_kv_counters_offset(const Shape&) { return a256(16); }   // err takes 16 bytes

// ---------------------------------------------------------------------------
// Bucket helpers.
//
// A batch of n (query, slot) entries starting at src, kBucketPer per thread,
// -1 past the end.  VEC (top_k a multiple of 4, so every batch starts on a
// 16-byte boundary): thread t holds entries 4 (t + kBucketThreads i) + c;
// otherwise entries t + kBucketThreads i.
template <bool VEC>
__device__ __forceinline__ int batch_entry(int i) {
  return VEC ? 4 * ((int)threadIdx.x + kBucketThreads * (i >> 2)) + (i & 3)
             : (int)threadIdx.x + kBucketThreads * i;
}

// Entries of rows in query tiles (tm[row / 128] != 0, tm indexed from the
// unit's first tile; null: none) read as empty: those rows belong to the
// query-stationary kernel.  Row of entry e of the batch: row0 + e / k, with
// e / k from the float product (e < 2^14; see bucket_scatter_kernel).
template <bool VEC>
__device__ __forceinline__ void load_batch(const int32_t* __restrict__ src, int n,
                                           int (&v)[kBucketPer], const uint8_t* tm, int row0,
                                           float inv_k) {
  auto in_q_tile = [&](int e) {
    return tm != nullptr && tm[(row0 + __float2int_rz(((float)e + 0.5f) * inv_k)) / kTileRows] != 0;
  };
  if constexpr (VEC) {
    const int4* s4 = reinterpret_cast<const int4*>(src);
#pragma unroll
    for (int i = 0; i < kBucketPer / 4; ++i) {
      const int q = (int)threadIdx.x + kBucketThreads * i;
      int4 x = 4 * q < n ? __ldcg(s4 + q) : make_int4(-1, -1, -1, -1);
      if (4 * q < n && in_q_tile(4 * q)) x = make_int4(-1, -1, -1, -1);   // k % 4 == 0: one row
      v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kBucketPer; ++i) {
      const int e = batch_entry<false>(i);
      v[i] = (e < n && !in_q_tile(e)) ? __ldcg(src + e) : -1;
    }
  }
}

// Block-wide exclusive scan of one value per thread; *total gets the sum.
// `warp_sums` holds kBucketThreads / 32 ints.  Ends with a barrier.
__device__ __forceinline__ int block_exclusive_scan(int x, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  constexpr int W = kBucketThreads / 32;
  int before = 0, all = 0;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int ws = warp_sums[i];
    before += i < warp ? ws : 0;
    all += ws;
  }
  *total = all;
  __syncthreads();   // warp_sums may be reused right after
  return before + inc - x;
}

// Scale exponents of the partial outputs (see the top of the file): for key
// block j of unit u the largest e in [kMinVexp, kMaxVexp] with
// bs * max|V_j| * 2^e <= 2^14, from the bf16 bit patterns (max|v| < 2^(E+1),
// E the unbiased exponent of the largest |v|).  One warp per block, 16-byte
// loads.  Of e, the part at or above kMinShiftExp is folded into the softmax
// shift; the rest (blocks with max|v| above ~2^64) scales the epilogue.
constexpr int kMinVexp = -120, kMaxVexp = 60, kMinShiftExp = -56;

__device__ __forceinline__ void vexp_block_warp(const __nv_bfloat16* __restrict__ V,
                                                int32_t* __restrict__ vexp, const Shape& s, int u,
                                                int j, int lane) {
  const uint4* src =
      reinterpret_cast<const uint4*>(V + ((int64_t)u * s.N + (int64_t)j * s.bs) * s.D);
  const int n16 = s.bs * s.D / 8;   // 16-byte chunks of the block
  uint32_t mx = 0;                  // per-halfword max of |bf16| bit patterns
  for (int i0 = 0; i0 < n16; i0 += 32 * 8) {
    uint4 v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = i0 + q * 32 + lane;
      v[q] = i < n16 ? __ldg(src + i) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      mx = __vmaxu2(mx, v[q].x & 0x7fff7fffu);
      mx = __vmaxu2(mx, v[q].y & 0x7fff7fffu);
      mx = __vmaxu2(mx, v[q].z & 0x7fff7fffu);
      mx = __vmaxu2(mx, v[q].w & 0x7fff7fffu);
    }
  }
  mx = __vmaxu2(mx, mx >> 16) & 0xffffu;   // non-negative bf16: bit order = value order
  mx = __reduce_max_sync(0xffffffffu, mx);
  if (lane == 0) {
    int e = kMaxVexp;
    if (mx != 0) {
      const int be = (int)(mx >> 7) & 0xff;   // biased exponent (0: subnormal)
      const int E = (be == 0 ? 1 : be) - 127;
      e = 13 - (31 - __clz(s.bs)) - E;        // 14 - log2(bs) - (E + 1)
      e = min(kMaxVexp, max(kMinVexp, e));
    }
    vexp[(int64_t)u * s.nb + j] = e;
  }
}

// 1. Per chunk of a unit's rows: how many of its selections pick each block,
//    and where the chunk's entries of block j start within j's list (an
//    atomic on the block's cursor, so the chunks of a list come in any
//    order; every row's result is the same whichever work item holds it).
//    The unit's last chunk to finish -- a ticket taken after a device-wide
//    fence -- then lays out the unit: block counts (the cursors), list
//    offsets (an exclusive scan over blocks), and work items of at most 128
//    queries per block.  Thread t handles blocks t, t + kBucketThreads, ...,
//    and the scan runs over blocks in that thread-major order: list ranges
//    only need to be disjoint, and items of one block adjacent (the fine
//    kernel reuses a K/V tile across consecutive items of a block).
template <bool VEC>
__global__ void __launch_bounds__(kBucketThreads, 2)
bucket_count_kernel(const int32_t* __restrict__ idx, int32_t* __restrict__ cursor,
                    int32_t* __restrict__ chunk_rel, int32_t* __restrict__ done,
                    int32_t* __restrict__ offsets, int32_t* __restrict__ item_row,
                    int4* __restrict__ items, uint32_t* __restrict__ ctr,
                    const __nv_bfloat16* __restrict__ V, int32_t* __restrict__ vexp,
                    QTiles qtiles, Shape s, BucketGeom g, float inv_k) {
  extern __shared__ int32_t hist[];
  const uint8_t* tile_mode = active_tile_mode(qtiles);
  __shared__ int32_t wsum_c[kBucketThreads / 32], wsum_t[kBucketThreads / 32];
  __shared__ int32_t ticket, item_base;
  const int u = blockIdx.y, chunk = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint8_t* tm =
      tile_mode == nullptr ? nullptr
                           : tile_mode + (int64_t)u * ((s.N + kTileRows - 1) / kTileRows);

  {
    // Side job: the partial-output scale exponents of this chunk's share of
    // the unit's key blocks.
    const int bpc = (s.nb + g.chunks - 1) / g.chunks;
    const int j1 = min(s.nb, (chunk + 1) * bpc);
    for (int j = chunk * bpc + warp; j < j1; j += kBucketThreads / 32)
      vexp_block_warp(V, vexp, s, u, j, lane);
  }
  for (int j = tid; j < s.nb; j += kBucketThreads) hist[j] = 0;
  __syncthreads();
  const int row_end = min(s.N, (chunk + 1) * g.chunk_rows);
  for (int row0 = chunk * g.chunk_rows; row0 < row_end; row0 += g.rows_batch) {
    const int n = min(g.rows_batch, row_end - row0) * s.k;
    int v[kBucketPer];
    load_batch<VEC>(idx + ((int64_t)u * s.N + row0) * s.k, n, v, tm, row0, inv_k);
#pragma unroll
    for (int i = 0; i < kBucketPer; ++i)
      if (v[i] >= 0) atomicAdd(&hist[v[i]], 1);
  }
  __syncthreads();
  int32_t* cur = cursor + (int64_t)u * s.nb;
  int32_t* rel = chunk_rel + ((int64_t)u * g.chunks + chunk) * s.nb;
  for (int j = tid; j < s.nb; j += kBucketThreads) {
    const int c = hist[j];
    rel[j] = c ? atomicAdd(&cur[j], c) : 0;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) ticket = atomicAdd(&done[u], 1);
  __syncthreads();
  if (ticket != g.chunks - 1) return;
  __threadfence();   // every chunk's cursor update is visible from here on

  int sc = 0, st = 0;
  for (int j = tid; j < s.nb; j += kBucketThreads) {
    const int cj = __ldcg(cur + j);
    sc += cj;
    st += (cj + kTileRows - 1) / kTileRows;
  }
  int ic = sc, it = st;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, ic, o), b = __shfl_up_sync(0xffffffffu, it, o);
    if (lane >= o) { ic += a; it += b; }
  }
  if (lane == 31) { wsum_c[warp] = ic; wsum_t[warp] = it; }
  __syncthreads();
  if (warp == 0) {
    constexpr int W = kBucketThreads / 32;
    const int a = lane < W ? wsum_c[lane] : 0, b = lane < W ? wsum_t[lane] : 0;
    int ia = a, ib = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, ia, o), y = __shfl_up_sync(0xffffffffu, ib, o);
      if (lane >= o) { ia += x; ib += y; }
    }
    if (lane < W) { wsum_c[lane] = ia - a; wsum_t[lane] = ib - b; }
    if (lane == 31) item_base = (int)atomicAdd(&ctr[0], (uint32_t)ib);
  }
  __syncthreads();
  int oc = wsum_c[warp] + ic - sc;   // exclusive prefix of this thread's blocks
  int ot = wsum_t[warp] + it - st;
  const int64_t list_base = (int64_t)u * s.N * s.k;
  int4* out = items + item_base;
  for (int j = tid; j < s.nb; j += kBucketThreads) {
    const int cj = __ldcg(cur + j);
    offsets[(int64_t)u * s.nb + j] = oc;
    item_row[(int64_t)u * s.nb + j] = (item_base + ot) * kTileRows;
    for (int t = 0; t * kTileRows < cj; ++t)
      out[ot++] = make_int4(u, j, (int)(list_base + oc + t * kTileRows),
                            min(kTileRows, cj - t * kTileRows));
    oc += cj;
  }
}

// 2. Per block, the query rows that picked it (its list), and for every
//    (query, slot) the partial row its result goes to -- work item i owns
//    partial rows [128 i, 128 i + 128), one per list entry of the item --
//    or -1 for an empty slot.
//
//    Per batch of entries: a histogram in shared memory, its exclusive scan
//    (a local layout with each block's entries contiguous), a second pass
//    that places every entry in that layout, then one coalesced copy of the
//    layout to the list, block by block.  With cur[j] the block's next list
//    position relative to its offset, gap[j] = cur[j] - pre[j]: local
//    position p of block j goes to list position offsets[j] + gap[j] + p and
//    is partial row item_row[j] + gap[j] + p.
template <bool VEC>
__global__ void __launch_bounds__(kBucketThreads, 2)
bucket_scatter_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ chunk_rel,
                      const int32_t* __restrict__ offsets, const int32_t* __restrict__ item_row,
                      int32_t* __restrict__ lists, int32_t* __restrict__ inv,
                      QTiles qtiles, Shape s, BucketGeom g, float inv_k) {
  const uint8_t* tile_mode = active_tile_mode(qtiles);
  extern __shared__ int32_t smem_i[];
  int32_t* cnt = smem_i;                 // nb: batch counts -> local prefix -> local cursor
  int32_t* gap = smem_i + s.nb;          // nb: the block's cursor minus its local prefix
  int32_t* stage = smem_i + 2 * s.nb;    // kBucketBatch staged entries
  __shared__ int32_t warp_sums[kBucketThreads / 32];
  const int u = blockIdx.y, chunk = blockIdx.x;
  const int t = threadIdx.x;
  const int per = (s.nb + kBucketThreads - 1) / kBucketThreads;
  const uint8_t* tm =
      tile_mode == nullptr ? nullptr
                           : tile_mode + (int64_t)u * ((s.N + kTileRows - 1) / kTileRows);
  // Thread t owns blocks t + kBucketThreads m (the layout is in that order).
  const int32_t* start = chunk_rel + ((int64_t)u * g.chunks + chunk) * s.nb;
  for (int j = t; j < s.nb; j += kBucketThreads) { gap[j] = start[j]; cnt[j] = 0; }
  __syncthreads();
  int32_t* ul = lists + (int64_t)u * s.N * s.k;
  const int32_t* lo = offsets + (int64_t)u * s.nb;
  const int32_t* ir = item_row + (int64_t)u * s.nb;
  const int row_end = min(s.N, (chunk + 1) * g.chunk_rows);
  for (int row0 = chunk * g.chunk_rows; row0 < row_end; row0 += g.rows_batch) {
    const int n = min(g.rows_batch, row_end - row0) * s.k;
    const int64_t e0 = ((int64_t)u * s.N + row0) * s.k;
    int v[kBucketPer];
    load_batch<VEC>(idx + e0, n, v, tm, row0, inv_k);
#pragma unroll
    for (int i = 0; i < kBucketPer; ++i)
      if (v[i] >= 0) atomicAdd(&cnt[v[i]], 1);
    __syncthreads();
    int mine = 0;
    for (int m = 0; m < per; ++m) {
      const int j = t + kBucketThreads * m;
      if (j < s.nb) mine += cnt[j];
    }
    int total;
    int pre = block_exclusive_scan(mine, warp_sums, &total);
    for (int m = 0; m < per; ++m) {
      const int j = t + kBucketThreads * m;
      if (j < s.nb) {
        const int c = cnt[j];
        cnt[j] = pre;
        gap[j] -= pre;
        pre += c;
      }
    }
    __syncthreads();
    // v[i] becomes the entry's partial row.
#pragma unroll
    for (int i = 0; i < kBucketPer; ++i) {
      const int j = v[i];
      v[i] = -1;
      if (j >= 0) {
        const int lp = atomicAdd(&cnt[j], 1);
        // Row of entry e within the batch, e / k without an integer
        // division: e < 2^14, so the float product is within 2^-9 of e / k,
        // while (e + 1/2) / k sits at least 1 / 128 away from an integer.
        const int r = __float2int_rz(((float)batch_entry<VEC>(i) + 0.5f) * inv_k);
        stage[lp] = (j << kRowBits) | r;
        v[i] = ir[j] + gap[j] + lp;
      }
    }
    if constexpr (VEC) {
      int4* d4 = reinterpret_cast<int4*>(inv + e0);
#pragma unroll
      for (int i = 0; i < kBucketPer / 4; ++i) {
        const int q = t + kBucketThreads * i;
        if (4 * q < n) __stcg(d4 + q, make_int4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < kBucketPer; ++i) {
        const int e = batch_entry<false>(i);
        if (e < n) __stcg(inv + e0 + e, v[i]);
      }
    }
    __syncthreads();
    for (int p = t; p < total; p += kBucketThreads) {
      const int w = stage[p];
      const int j = w >> kRowBits;
      ul[lo[j] + gap[j] + p] = row0 + (w & ((1 << kRowBits) - 1));
    }
    __syncthreads();
    for (int j = t; j < s.nb; j += kBucketThreads) { gap[j] += cnt[j]; cnt[j] = 0; }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// 4. The tensor-core fine kernel.
//
// Warps (NWG = 3 softmax warpgroups when TMEM holds three (S, P, O) sets,
// else 2):
//   0 .. 4*NWG-1  warpgroup w takes the items t with t % NWG == w and owns
//                 separate TMEM columns S[w], P[w] (bf16 pairs) and O[w].
//                 Per item: S(t) into registers (its columns are then free,
//                 and the group's third warp issues S(t + NWG) at once if its
//                 queries and K/V are already there), P(t) into the P
//                 columns once PV(t - NWG) is done, the epilogue of item
//                 t - NWG (each warp stores its own 32 output rows), then the
//                 group's first warp issues PV(t), which runs while the group
//                 works on its next item.  Each warpgroup issues its own
//                 MMAs: one thread's chain of commit-and-wait steps is
//                 latency-bound (~500 cycles per commit at these tile
//                 sizes), and independent issuers overlap.
//   4*NWG .. +NG-1  NG gather warps, item t to warp t % NG: one bulk copy
//                 brings the item's list slice (query rows) into a small
//                 per-warp ring two of the warp's items ahead; the warp then
//                 writes the rows into the stage's entries and issues one TMA
//                 gather4 (four 128-byte rows) per lane.  TMA keeps the
//                 gathers off the load/store pipe, which the softmax warps'
//                 instruction stream would otherwise starve.
//   4*NWG+NG      the K/V warp: for every item in order, writes the item and
//                 its K/V slot into the stage, and issues the TMA loads of K
//                 and V once per run of consecutive items on the same key
//                 block (items are sorted by block), into one of NKV >= NWG
//                 slots.  A slot is reloaded once every warpgroup has seen
//                 the O of all its items up to the old run's last one (the
//                 groups publish that progress in shared memory), since the
//                 run's items are spread over all groups' MMA streams.
// A query stage is handed back as soon as S of its item is done; each warp
// stages its 32 output rows in its group's buffer and stores them with TMA.
// Shared memory: NQ query stages (gathered rows + entries), NWG output tiles,
// NKV K/V slots.
//
// Every mbarrier here is waited by phase parity, which is only sound if no
// waiter can run two phases ahead of the barrier.  Hence: stage st serves
// items st, st + NQ, ..., and NQ is a multiple of both NWG and NG, so one
// warpgroup consumes and one gather warp fills every use of a stage, each in
// order; the K/V warp visits every item in order; and K/V loads complete on
// 2 * NKV barriers (run % (2 NKV)), so a barrier's previous use (2 NKV runs
// back) has always completed before anyone waits for its next one.
template <int BS, int HD>
struct KvCfg {
  static constexpr int NWG = (BS + HD <= 128) ? 3 : 2;
  static constexpr int NG = NWG;                         // gather warps
  static constexpr int kQBytes = kTileRows * HD * 2;     // gathered queries of one item
  // Query stages.  A stage is released as soon as S of its item is done, so
  // two per warpgroup keep the next item of every group loaded ahead (one
  // per group at head_dim 128, where K/V slots need the room).
  static constexpr int NQ = (HD == 64) ? 2 * NWG : NWG;
  static constexpr int kOutBytes = kTileRows * HD * 2;   // a group's output tile (bf16)
  static constexpr int kKBytes = BS * HD * 2;
  static constexpr int kKVBytes = 2 * kKBytes;           // one block's K and V
  // Per stage: 128 list entries, the item (int4), its K/V word.
  static constexpr int kMetaBytes = kTileRows * 4 + 32;
  static constexpr int kRing = 128;                      // staged work items per loader warp
  static constexpr int kLoaderWarps = NG + 1;            // + the K/V warp
  static constexpr int kEntSlots = 3;                    // list slices in flight per gather warp
  // A list slice copy starts at the 16-byte boundary at or below the item's
  // first entry: up to 3 leading entries, 128 entries, padded to 16 bytes.
  static constexpr int kEntBytes = (kTileRows + 4) * 4;
  static constexpr int kSmemLimit = 227 * 1024;
  static constexpr int kFixed = NQ * kQBytes + NWG * kOutBytes + NQ * kMetaBytes +
                                kLoaderWarps * kRing * 16 + NG * kEntSlots * kEntBytes +
                                512 /*barriers*/ + 1024 /*alignment*/;
  // K/V slots.  Reloading the slot of the run NKV runs back waits for the
  // O of every item up to that run's last one, which is at least NKV items
  // back; with NKV >= NWG those items' S MMAs never wait for the run being
  // loaded, so NKV >= NWG slots suffice.  More let later runs load early:
  // as many as shared memory allows, up to 8.
  static constexpr int kKVFit = (kSmemLimit - kFixed) / kKVBytes;
  static constexpr int NKV = kKVFit > 8 ? 8 : kKVFit;
  static constexpr int kOutOff = NQ * kQBytes;
  static constexpr int kKVOff = kOutOff + NWG * kOutBytes;
  static constexpr int kMetaOff = kKVOff + NKV * kKVBytes;
  static constexpr int kRingOff = kMetaOff + NQ * kMetaBytes;
  static constexpr int kEntOff = kRingOff + kLoaderWarps * kRing * 16;
  static constexpr int kBarOff = kEntOff + NG * kEntSlots * kEntBytes;
  static constexpr int kSmem = kBarOff + 512 + 1024 /*align*/;
  static constexpr int kTmemCols = 512;
  static constexpr int kThreads = (4 * NWG + kLoaderWarps) * 32;
  // q_full completes on two arrivals (the gather warp's, with the gathered
  // bytes, and the K/V warp's) plus the gathered bytes; q_empty on one
  // arrival per warp of the consuming group once S of the item is done.
  static constexpr int kQFullCount = 2;
  static constexpr int kQEmptyCount = 4;
  static constexpr int kGroupCols = BS + BS / 2 + HD;    // TMEM: S, P, O of one group
  static_assert(NWG * kGroupCols <= 512, "TMEM holds NWG (S, P, O) sets");
  static_assert(NKV >= NWG && NKV <= 8, "K/V slots");
  static_assert(NQ % NWG == 0 && NQ % NG == 0, "one consumer and one producer per stage");
  static_assert(kSmem <= kSmemLimit, "shared memory");
  static_assert(kOutOff % 1024 == 0 && kKVOff % 1024 == 0, "swizzled tiles 1024-byte aligned");
  static_assert(kEntBytes % 16 == 0 && kMetaBytes % 16 == 0 && kRingOff % 16 == 0 &&
                    kEntOff % 16 == 0,
                "alignment");
  static_assert((2 * NQ + 2 * NKV + 5 * NWG + NG * kEntSlots + 1) * 8 + 8 + 4 * (NWG + NKV) <= 512,
                "barrier area");
};

// K/V word of a staged item: slot | kv_full barrier << 8 | its phase parity << 16.
constexpr int kMetaKv = kTileRows + 4;   // int offset of the word in the stage meta

struct FineKvParams {
  const int4* items;
  const int32_t* lists;
  const int32_t* vexp;          // per (unit, block): partial-output scale exponent
  const uint32_t* total_items;  // device word written by bucket_count's layout step
  float2* part_ml;
  uint32_t* err;
  Shape s;
};

template <int BS, int HD>
__global__ void __launch_bounds__(KvCfg<BS, HD>::kThreads, 1)
fine_kv_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
               const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ CUtensorMap tmap_o,
               FineKvParams prm) {
  using C = KvCfg<BS, HD>;
  constexpr int NQ = C::NQ, NWG = C::NWG;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::kBarOff);
  uint64_t* q_full = bars;                      // [NQ] rows + entries of the stage's item landed
  uint64_t* q_empty = q_full + NQ;              // [NQ] stage free: S of its item is done
  uint64_t* kv_full = q_empty + NQ;             // [2 NKV] K, V of a block run landed
                                                //         (run % (2 NKV))
  uint64_t* s_full = kv_full + 2 * C::NKV;      // [NWG] S in TMEM
  uint64_t* s_free = s_full + NWG;              // [NWG] S read out (128 arrivals)
  uint64_t* p_full = s_free + NWG;              // [NWG] P in TMEM and the previous O read
                                                //       out (128 arrivals)
  uint64_t* o_full = p_full + NWG;              // [NWG] O in TMEM
  uint64_t* drain = o_full + NWG;               // [NWG] the group's MMAs are complete
  uint64_t* ent_full = drain + NWG;             // [NG * kEntSlots] a list slice landed
  uint64_t* gate = ent_full + C::NG * C::kEntSlots;   // test hook: never completed
  uint32_t* tmem_slot = (uint32_t*)(gate + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  int* o_done = (int*)(tmem_slot + 2);          // [NWG] last item whose O the group has seen
  int* run_last = o_done + NWG;                 // [NKV] last item of the slot's current run
  int4* ring = (int4*)(smem + C::kRingOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w_load = 4 * NWG;
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
      mbar_init(&q_empty[i], C::kQEmptyCount);
    }
    for (int i = 0; i < 2 * C::NKV; ++i) mbar_init(&kv_full[i], 1);
    for (int g = 0; g < NWG; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&s_free[g], 128);
      mbar_init(&p_full[g], 128);
      mbar_init(&o_full[g], 1);
      mbar_init(&drain[g], 2);   // one commit from each issuing warp
      o_done[g] = g - NWG;
    }
    for (int i = 0; i < C::NG * C::kEntSlots; ++i) mbar_init(&ent_full[i], 1);
    mbar_init(gate, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == w_load && lane == 0) {
    prefetch_tensormap(&tmap_q);
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
    prefetch_tensormap(&tmap_o);
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

  // Test hook (BSA_FLAG_TEST_TIMEOUT): before any copy or MMA is issued, one
  // bounded wait on a barrier that nothing completes.  It runs out after a
  // few microseconds, reports kErrTestTimeout in the error word, and the CTA
  // goes straight to its teardown -- the path a stuck pipeline takes, with
  // nothing in flight.
  if (s.test_timeout) {
    if (threadIdx.x == 0 && !mbar_wait_ns(gate, 0, prm.err, kErrTestTimeout, 2000))
      *abort_flag = 1;
    __syncthreads();
  }
  if (*abort_flag == 0) {   // (the body runs unless the test hook stopped it)
  if (warp >= w_load) {
    // ------------------------------------------------------------ loaders
    // Each loader warp keeps its own ring of the work items, refilled half a
    // ring at a time once it is within a few items of the filled end.
    constexpr int H = C::kRing / 2;
    const int L = warp - w_load;
    int4* my_ring = ring + L * C::kRing;
    int filled = 0;                          // items [filled - kRing, filled) are in the ring
    auto fill = [&](int count) {
      for (int q = lane; q < count; q += 32)
        if (filled + q < T) my_ring[(filled + q) % C::kRing] = prm.items[t_begin + filled + q];
      filled += count;
      __syncwarp();
    };
    fill(C::kRing);
    if (L < C::NG) {
      // ---------------------------------------------------------- gather warp
      constexpr int NG = C::NG, ES = C::kEntSlots;
      const uint64_t pol_q = policy_evict_last();   // rows are gathered ~top_k times each
      auto ent_buf = [&](int es) {
        return (int32_t*)(smem + C::kEntOff + (L * ES + es) * C::kEntBytes);
      };
      // Lane 0: the list slice of the warp's k-th item (t = L + k * NG) into
      // ring slot k % ES.  Reading up to 3 entries before the item's first
      // keeps the copy 16-byte aligned; the lists end with enough slack.
      auto fetch_entries = [&](int k) {
        const int t = L + k * NG;
        if (t >= T) return;
        const int4 it = my_ring[t % C::kRing];
        uint64_t* bar = &ent_full[L * ES + k % ES];
        mbar_arrive_expect_tx(bar, C::kEntBytes);
        bulk_copy_g2s(ent_buf(k % ES), prm.lists + (it.z & ~3), C::kEntBytes, bar);
      };
      if (lane == 0)
        for (int k = 0; k < ES - 1; ++k) fetch_entries(k);
      int k = 0;
      for (int t = L; t < T; t += NG, ++k) {
        if (t + 2 * ES * NG >= filled) fill(H);
        const int st = t % NQ, use = t / NQ;
        if (use >= 1) {
          bool ok = mbar_wait(&q_empty[st], (use - 1) & 1, prm.err, kErrWaitFree);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok || *abort_flag) { *abort_flag = 1; break; }
        }
        if (lane == 0) fetch_entries(k + ES - 1);   // its slot's previous slice is consumed
        bool ok = mbar_wait(&ent_full[L * ES + k % ES], (k / ES) & 1, prm.err, kErrWaitEnt);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || *abort_flag) { *abort_flag = 1; break; }
        const int4 it = my_ring[t % C::kRing];
        // Lane l takes tile rows 4l .. 4l + 3; rows past the item's count
        // repeat its first query (their results are never read).
        const int32_t* ent = ent_buf(k % ES) + (it.z & 3);
        int32_t rr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = 4 * lane + j;
          rr[j] = ent[r < it.w ? r : 0];
        }
        int32_t* m = meta(st);
        reinterpret_cast<int4*>(m)[lane] = make_int4(rr[0], rr[1], rr[2], rr[3]);
        // The slice has been read; the async proxy may overwrite it next.
        fence_proxy_async_smem();
        const int ngroups = (it.w + 3) >> 2;   // 4-row groups holding valid rows
        __syncwarp();
        if (lane == 0)
          mbar_arrive_expect_tx(&q_full[st], (uint32_t)ngroups * 512u * (HD / 64));
        if (lane < ngroups) {
          const int32_t y0 = it.x * s.N;
#pragma unroll
          for (int p = 0; p < HD / 64; ++p)
            tma_gather4_hint(q_s(st) + p * (kTileRows * 128) + lane * 512, &tmap_q, &q_full[st],
                             p * 64, y0 + rr[0], y0 + rr[1], y0 + rr[2], y0 + rr[3], pol_q);
        }
      }
    } else {
      // ---------------------------------------------------------- K/V warp
      const uint64_t pol_kv = policy_evict_first();   // a block's K, V are read once per run
      int gen = -1, px = -1, py = -1;
      // Every group has seen the O of all its items <= tl (bounded wait).
      auto wait_o_done = [&](int tl) -> bool {
        uint64_t t0 = 0;
        for (uint32_t i = 0;; ++i) {
          bool all = true;
#pragma unroll
          for (int w = 0; w < NWG; ++w) all = all && ld_acquire_shared(&o_done[w]) + NWG > tl;
          if (all) return true;
          if (*abort_flag) return false;
          __nanosleep(64);
          if ((i & 255) == 0) {
            if (i == 0) {
              t0 = globaltimer();
            } else if (globaltimer() - t0 > kWaitLimitNs) {
              atomicOr(prm.err, kErrWaitFree);
              return false;
            }
          }
        }
      };
      for (int t = 0; t < T; ++t) {
        if (t + 8 >= filled) fill(H);
        const int st = t % NQ, use = t / NQ;
        if (use >= 1) {
          bool ok = mbar_wait(&q_empty[st], (use - 1) & 1, prm.err, kErrWaitFree);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok || *abort_flag) { *abort_flag = 1; break; }
        }
        if (lane == 0) {
          const int4 it = my_ring[t % C::kRing];
          bool new_run = false;
          if (it.x != px || it.y != py) {
            px = it.x;
            py = it.y;
            ++gen;
            new_run = true;
          }
          const int slot = gen % C::NKV, kb = gen % (2 * C::NKV);
          int32_t* m = meta(st);
          reinterpret_cast<int4*>(m + kTileRows)[0] = it;
          m[kMetaKv] = slot | (kb << 8) | (((gen / (2 * C::NKV)) & 1) << 16);
          mbar_arrive(&q_full[st]);
          if (new_run) {
            // K and V into the run's slot once the slot's previous run is done.
            if (gen >= C::NKV && !wait_o_done(run_last[slot])) {
              *abort_flag = 1;
            } else {
              mbar_arrive_expect_tx(&kv_full[kb], C::kKVBytes);
              const int32_t y = it.x * s.N + it.y * BS;
#pragma unroll
              for (int p = 0; p < HD / 64; ++p) {
                tma_load_2d_hint(k_s(slot) + p * (BS * 128), &tmap_k, &kv_full[kb], p * 64, y,
                                 pol_kv);
                tma_load_2d_hint(v_s(slot) + p * (BS * 128), &tmap_v, &kv_full[kb], p * 64, y,
                                 pol_kv);
              }
            }
          }
          run_last[slot] = t;
        }
        __syncwarp();
        if (*abort_flag) break;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax / MMA / epilogue
    // Per item t (the group's n-th): S(t) -> registers, releasing the S
    // columns for S(t + NWG); P(t) into the P columns once PV(t - NWG) is
    // done; the epilogue of item t - NWG; then PV(t).  PV(t) runs while the
    // group works on item t + NWG, so its latency is off the group's path.
    const int wg = warp >> 2;              // takes items t with t % NWG == wg
    const int quad = warp & 3;             // TMEM lane quadrant
    const bool issuer = (quad == 0);       // this warp issues the group's PV MMAs
    const bool s_issuer = (quad == 2);     // this warp issues the group's S MMAs
    const bool storer = (quad == 1);       // this warp publishes the group's O progress
    const int r = quad * 32 + lane;        // row of the tile this thread owns
    const uint32_t s_col = tbase + wg * C::kGroupCols;   // S (fp32), TMEM lane 0
    const uint32_t p_col = s_col + BS;                   // P (bf16 pairs)
    const uint32_t o_col = p_col + BS / 2;               // O (fp32)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = s_col + lane_off;
    const uint32_t p_addr = p_col + lane_off;
    const uint32_t o_addr = o_col + lane_off;
    // Partial tiles keep the default L2 priority: most are evicted long before
    // the combine reads them, but the last ones written are still in L2 when
    // it starts (2 us less combine than with evict-first on the headline
    // workload, results identical).
    const uint64_t pol_o = policy_evict_normal();
    constexpr uint32_t idesc_s = idesc_bf16_f32(kTileRows, BS, false);
    constexpr uint32_t idesc_o = idesc_bf16_f32(kTileRows, HD, true);
    // Descriptors at stage / slot 0; the start-address field (bits 0-13,
    // address >> 4) is advanced by adding byte offsets >> 4.
    const uint64_t dq0 = smem_desc_sw128(smem_u32(q_s(0)), 16, 1024);
    const uint64_t dk0 = smem_desc_sw128(smem_u32(k_s(0)), 16, 1024);
    const uint64_t dv0 = smem_desc_sw128(smem_u32(v_s(0)), BS * 128, 1024);
    unsigned char* out = smem + C::kOutOff + wg * C::kOutBytes;

    // Lane 0 of the issuer warp: S(t) = Q K^T into the S columns.
    auto mma_s = [&](int t, int kv) {
      const int st = t % NQ;
      const uint64_t dq = dq0 + ((st * C::kQBytes) >> 4);
      const uint64_t dk = dk0 + (((kv & 0xff) * C::kKVBytes) >> 4);
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint32_t off = (kk >> 2) * (kTileRows * 128) + (kk & 3) * 32;
        const uint32_t offk = (kk >> 2) * (BS * 128) + (kk & 3) * 32;
        mma_bf16(s_col, dq + (off >> 4), dk + (offk >> 4), idesc_s, kk > 0);
      }
      mma_commit(&s_full[wg]);
    };
    // Issuer warp: issue S(t) once its queries and K/V have landed (bounded wait).
    auto issue_s = [&](int t) -> bool {
      const int st = t % NQ;
      bool ok = mbar_wait(&q_full[st], (t / NQ) & 1, prm.err, kErrWaitQ);
      int kv = 0;
      if (ok) {
        kv = meta(st)[kMetaKv];
        ok = mbar_wait(&kv_full[(kv >> 8) & 0xff], (kv >> 16) & 1, prm.err, kErrWaitKV);
      }
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        if (lane == 0) mma_s(t, kv);
        __syncwarp();
      }
      return ok;
    };
    // Issuer warp: issue S(t) only if its queries and K/V have already landed.
    auto try_issue_s = [&](int t) -> bool {
      const int st = t % NQ;
      bool ready = mbar_test(&q_full[st], (t / NQ) & 1);
      int kv = 0;
      if (ready) {
        kv = meta(st)[kMetaKv];
        ready = mbar_test(&kv_full[(kv >> 8) & 0xff], (kv >> 16) & 1);
      }
      ready = __all_sync(0xffffffffu, ready);
      if (ready) {
        tc_fence_after();
        if (lane == 0) mma_s(t, kv);
        __syncwarp();
      }
      return ready;
    };
    // Epilogue of item tp, the group's np-th, whose O is complete: O (not
    // yet divided by l; the combine folds 1 / l into its weights), already
    // scaled by 2^e1 through the shift, times 2^e2 (e2 = e - e1, 0 unless the
    // block's max|v| exceeds ~2^64; the same for the whole item), as fp16
    // into this warp's 32 rows of the group's output tile (row r, 16-byte
    // chunk c at the 128-byte swizzled place the TMA store expects), (m, l)
    // per row, and the warp's own TMA store of its rows.  Each warp only
    // waits for its own previous store to have read its rows.
    auto epilogue_begin = [&](int np) {   // the staging tile is free again
      if (np >= 1 && lane == 0) bulk_wait_group_read0();
      __syncwarp();
    };
    // 64 columns of O, in registers, into the staging tile as fp16.
    auto stage_cols = [&](int c0, float (&ov)[64], int e2, float f2) {
      if (e2 != 0) {
#pragma unroll
        for (int c = 0; c < 64; ++c) ov[c] *= f2;
      }
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        const int ch = c >> 3;
        *reinterpret_cast<uint4*>(out + (c0 >> 6) * (kTileRows * 128) + r * 128 +
                                  ((ch ^ (r & 7)) << 4)) =
            make_uint4(pack_f16x2(ov[c], ov[c + 1]), pack_f16x2(ov[c + 2], ov[c + 3]),
                       pack_f16x2(ov[c + 4], ov[c + 5]), pack_f16x2(ov[c + 6], ov[c + 7]));
      }
    };
    auto epilogue_end = [&](int tp, float mp, float lp, float f2) {
      // Work item gi owns partial rows [128 gi, 128 gi + 128); rows past the
      // item's count hold values that are never read.
      const int gi = (int)t_begin + tp;
      prm.part_ml[(int64_t)gi * kTileRows + r] = make_float2(mp, lp * f2);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int p = 0; p < HD / 64; ++p)
          tma_store_2d_hint(&tmap_o, out + p * (kTileRows * 128) + quad * 32 * 128, p * 64,
                            gi * kTileRows + quad * 32, pol_o);
        bulk_commit_group();
      }
    };
    // With `hand_off`: once O is read out of TMEM (the first 64 columns at
    // head_dim 64, all of it at 128), P(t) of the current item is handed to
    // the PV issuer before the staging.
    auto epilogue = [&](int tp, int np, float mp, float lp, int e2, bool hand_off) {
      const float f2 = exp2i(e2);
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 64) {
        float ov[64];
        tmem_ld64(o_addr + c0, ov);
        if (hand_off && c0 + 64 == HD) {
          tc_fence_before();   // P(t) stored, O(t - NWG) read out
          mbar_arrive(&p_full[wg]);
        }
        if (c0 == 0) epilogue_begin(np);
        stage_cols(c0, ov, e2, f2);
      }
      epilogue_end(tp, mp, lp, f2);
    };
    // O(t) complete means every MMA this group issued before it (S(t),
    // PV(t) and all earlier items') is done reading its K/V slot.
    auto publish_o_done = [&](int t) {
      if (lane == 0) st_release_shared(&o_done[wg], t);
    };

    if (s_issuer && wg < T && !issue_s(wg)) *abort_flag = 1;
    int n = 0, tp = -1, ep = 0;
    float mp = 0.f, lp = 1.f;   // the previous item's stored m, its row sum, its e2
    bool ok = true;
    for (int t = wg; t < T; t += NWG, ++n) {
      const int st = t % NQ;
      ok = mbar_wait(&q_full[st], (t / NQ) & 1, prm.err, kErrWaitQ);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) { ok = false; break; }
      const int32_t* m = meta(st);
      const int4 itm = reinterpret_cast<const int4*>(m + kTileRows)[0];
      const int j = itm.y;
      const int kv = m[kMetaKv];
      // The block's partial-output exponent e; e1 = max(e, kMinShiftExp) goes
      // into the shift, e2 = e - e1 into the epilogue.
      const int ve = __ldg(prm.vexp + (int64_t)itm.x * s.nb + j);
      const int ve1 = max(ve, kMinShiftExp);
      const int qrow = m[r];   // rows past the item's count repeat its first query

      ok = mbar_wait(&s_full[wg], n & 1, prm.err, kErrWaitS);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_flag) { ok = false; break; }
      tc_fence_after();
      // S(t) is done, so its query rows are dead; every lane has read the
      // stage's entries and K/V word above: hand the stage back.
      if (lane == 0) mbar_arrive(&q_empty[st]);
      const int key0 = j * BS;
      const bool diag = s.causal && key0 + BS - 1 > qrow;
      // The whole S row is read from TMEM once; the row max and every p
      // come from these registers, so the shift and the stored (m, l, O)
      // always describe the same scores.
      float sv[BS];
#pragma unroll
      for (int c0 = 0; c0 < BS; c0 += 64) tmem_ld64(s_addr + c0, sv + c0);
      // Token-level causal mask (block_indexer.py:73-81): key > query -> -inf.
      if (diag) {
#pragma unroll
        for (int c = 0; c < BS; ++c)
          if (key0 + c > qrow) sv[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < BS; c0 += 64) {
        float m0 = sv[c0], m1 = sv[c0 + 1], m2 = sv[c0 + 2], m3 = sv[c0 + 3];
#pragma unroll
        for (int c = c0 + 4; c < c0 + 64; c += 8) {
          m0 = fmax3(m0, sv[c], sv[c + 1]);
          m1 = fmax3(m1, sv[c + 2], sv[c + 3]);
          m2 = fmax3(m2, sv[c + 4], sv[c + 5]);
          m3 = fmax3(m3, sv[c + 6], sv[c + 7]);
        }
        mx = fmax3(mx, fmax3(m0, m1, m2), m3);
      }
      // S(t) is all in registers: its columns are free for S(t + NWG).
      tc_fence_before();
      mbar_arrive(&s_free[wg]);
      // Padding rows of a short item can be fully masked; keep them finite.
      const float msc = (mx == -INFINITY) ? 0.f : mx * sc;
      const float msh = msc - (float)ve1;   // p 2^e1 = 2^(s sc - msh)
      if (n >= 1) {
        // PV(t - NWG) done: the P columns are free and O(t - NWG) is final.
        ok = mbar_wait(&o_full[wg], (n - 1) & 1, prm.err, kErrWaitO);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || *abort_flag) { ok = false; break; }
        tc_fence_after();
        if (storer) publish_o_done(tp);
      }
      // p = 2^(s sc - m sc), summed per row in (even, odd) column halves
      // (packed pairs: one fma and one add per two columns).
      float2 l2 = make_float2(0.f, 0.f);
      const float2 sc2 = make_float2(sc, sc), sh2 = make_float2(-msh, -msh);
#pragma unroll
      for (int c0 = 0; c0 < BS; c0 += 64) {
#pragma unroll
        for (int h = 0; h < 64; h += 32) {   // 16 P columns at a time
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float p0, p1;
            if constexpr (BS == 64) {
              const float2 x = ffma2(make_float2(sv[c0 + h + c], sv[c0 + h + c + 1]), sc2, sh2);
              p0 = fast_exp2(x.x);
              p1 = fast_exp2(x.y);
              l2 = fadd2(l2, make_float2(p0, p1));
            } else {   // the 128-key block has no registers to spare for pairs
              p0 = fast_exp2(fmaf(sv[c0 + h + c], sc, -msh));
              p1 = fast_exp2(fmaf(sv[c0 + h + c + 1], sc, -msh));
              l2.x += p0;
              l2.y += p1;
            }
            pk[c >> 1] = pack_bf16x2(p0, p1);
          }
          tmem_st16_async(p_addr + ((c0 + h) >> 1), pk);
        }
      }
      tmem_wait_st();   // every P store of the item has landed
      const float l = l2.x + l2.y;
      bool issued_next = false;
      if (s_issuer && t + NWG < T) {
        // Every row of S(t) has been read: S(t + NWG) may go into its columns
        // now, if its queries and K/V are already there.  (S and PV use
        // disjoint TMEM columns and operands, so they may come from two
        // threads.)
        ok = mbar_wait(&s_free[wg], n & 1, prm.err, kErrWaitS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) { *abort_flag = 1; break; }
        issued_next = try_issue_s(t + NWG);
      }
      // The previous item's O comes out of TMEM into registers before P(t)
      // is handed to the PV issuer; the staging and store follow the
      // handoff, so PV(t) need not wait for the whole epilogue.
      if (n >= 1) {
        epilogue(tp, n - 1, mp, lp, ep, true);
      } else {
        tc_fence_before();   // P(t) stored
        mbar_arrive(&p_full[wg]);
      }
      if (issuer) {
        ok = mbar_wait(&p_full[wg], n & 1, prm.err, kErrWaitP);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) { *abort_flag = 1; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t dv = dv0 + (((kv & 0xff) * C::kKVBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < BS / 16; ++kk)
            mma_bf16_ts(o_col, p_col + kk * 8, dv + ((kk * 16 * 128) >> 4), idesc_o, kk > 0);
          mma_commit(&o_full[wg]);
        }
        __syncwarp();
      }
      if (s_issuer) {
        if (t + NWG < T && !issued_next) {
          // The next item's S has to wait for its queries or K/V.  The K/V
          // load may itself wait for this group's progress, so publish O(t)
          // first: it depends on nothing but PV(t).
          ok = mbar_wait(&o_full[wg], n & 1, prm.err, kErrWaitO);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) { *abort_flag = 1; break; }
          publish_o_done(t);
          if (!issue_s(t + NWG)) { ok = false; *abort_flag = 1; break; }
        }
      }
      tp = t;
      mp = msc - (float)ve;   // stored m: weights 2^(m - M) then carry 2^-e
      lp = l;
      ep = ve - ve1;
    }
    if (!ok) *abort_flag = 1;
    if (ok && tp >= 0) {
      // The group's last item.
      ok = mbar_wait(&o_full[wg], (n - 1) & 1, prm.err, kErrWaitO);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        if (storer) publish_o_done(tp);
        epilogue(tp, n - 1, mp, lp, ep, false);
      }
      if (!ok) *abort_flag = 1;
    }
    if (lane == 0) bulk_wait_group0();   // this warp's tile stores complete
    if (issuer || s_issuer) {
      // No MMA of this group in flight when TMEM is released.
      if (lane == 0) mma_commit(&drain[wg]);
      __syncwarp();
      mbar_wait(&drain[wg], 0, prm.err, kErrWaitDrain);
    }
  }
  }   // body
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, C::kTmemCols);
}

// 5. Per query: merge its partials, found through the (query, slot) ->
//    partial row map (-1 for an empty slot).  Partial j holds (m_j, l_j, O_j)
//    with O_j = 2^e sum 2^(s sc - m) v, l_j = 2^e sum 2^(s sc - m) and m_j =
//    m - e (m the row max in the base-2 domain, e the block's exponent), so
//    with a_j = m_j and b_j = m_j + log2 l_j (the partial's true log-weight):
//        O = 2^(A - B) (sum_j 2^(a_j - A) O_j) / (sum_j 2^(b_j - B)),
//    A = max a_j, B = max b_j.  Each sum is formed against its own maximum,
//    so no weight underflows whatever the blocks' exponents.  CH = HD / 8
//    threads per query row, one 16-byte chunk (8 fp16) of the output each.
//    The row's slot metadata (partial row, m, l) is loaded once, spread over
//    the CH threads (slot q by thread q % CH) and shared by shuffles; every
//    partial chunk load of the row is issued before the first is used, so a
//    thread keeps up to KMAX loads in flight instead of a chain of dependent
//    ones.
template <int HD, int KMAX>
__global__ void __launch_bounds__(256)
combine_kernel(const int32_t* __restrict__ inv,
               const __half* __restrict__ part_o, const float2* __restrict__ part_ml,
               const uint32_t* __restrict__ err, QTiles qtiles, __nv_bfloat16* __restrict__ O,
               Shape s) {
  const uint8_t* tile_mode = active_tile_mode(qtiles);
  constexpr int CH = HD / 8;           // threads per row (8 or 16), a power of two <= 32
  constexpr int PER = (KMAX + CH - 1) / CH;   // slots whose metadata one thread loads
  const int64_t rows = (int64_t)s.units * s.N;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int c = (int)(gid % CH);
  const bool live = gid / CH < rows;
  const int64_t R = live ? gid / CH : rows - 1;   // dead lanes mirror a real row
  // Rows of query tiles are written by the query-stationary kernel.  A
  // warp's 32 / CH rows are consecutive and aligned, so within one tile.
  const int tiles = (s.N + kTileRows - 1) / kTileRows;
  const bool q_row = tile_mode != nullptr &&
                     tile_mode[(R / s.N) * tiles + (R % s.N) / kTileRows] != 0;
  if (__all_sync(0xffffffffu, q_row)) return;
  const int lane = threadIdx.x & 31, base = lane & ~(CH - 1);
  const int32_t* prow = inv + R * s.k;   // -1: empty slot
  int32_t pr[PER];
  float a[PER], b[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int q = c + i * CH;
    pr[i] = q < s.k ? __ldg(prow + q) : -1;
  }
  float A = -INFINITY, B = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    a[i] = -INFINITY;
    b[i] = -INFINITY;
    if (pr[i] >= 0) {
      const float2 ml = __ldcs(&part_ml[pr[i]]);
      a[i] = ml.x;
      b[i] = ml.x + fast_log2(ml.y);
    }
    A = fmaxf(A, a[i]);
    B = fmaxf(B, b[i]);
  }
#pragma unroll
  for (int o = CH / 2; o > 0; o >>= 1) {
    A = fmaxf(A, __shfl_xor_sync(0xffffffffu, A, o));
    B = fmaxf(B, __shfl_xor_sync(0xffffffffu, B, o));
  }
  float L = 0.f;
  float w[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    w[i] = pr[i] >= 0 ? fast_exp2(a[i] - A) : 0.f;
    L += pr[i] >= 0 ? fast_exp2(b[i] - B) : 0.f;
  }
#pragma unroll
  for (int o = CH / 2; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  // Every slot's partial row and weight, then its chunk of the partial row.
  uint4 v[KMAX];
  float wq[KMAX];
#pragma unroll
  for (int q = 0; q < KMAX; ++q) {
    const int owner = base + (q % CH);
    const int32_t p = __shfl_sync(0xffffffffu, pr[q / CH], owner);
    wq[q] = __shfl_sync(0xffffffffu, w[q / CH], owner);
    v[q] = (q < s.k && p >= 0)
               ? __ldcs(reinterpret_cast<const uint4*>(part_o + (int64_t)p * HD) + c)
               : make_uint4(0u, 0u, 0u, 0u);
  }
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < KMAX; ++q) {
    const float wt = wq[q];
    const float2 x0 = unpack_f16x2(v[q].x), x1 = unpack_f16x2(v[q].y);
    const float2 x2 = unpack_f16x2(v[q].z), x3 = unpack_f16x2(v[q].w);
    acc[0] = fmaf(wt, x0.x, acc[0]); acc[1] = fmaf(wt, x0.y, acc[1]);
    acc[2] = fmaf(wt, x1.x, acc[2]); acc[3] = fmaf(wt, x1.y, acc[3]);
    acc[4] = fmaf(wt, x2.x, acc[4]); acc[5] = fmaf(wt, x2.y, acc[5]);
    acc[6] = fmaf(wt, x3.x, acc[6]); acc[7] = fmaf(wt, x3.y, acc[7]);
  }
  if (!live || q_row) return;
  // 2^(A - B) / L in two factors, each well inside the float range.  If a
  // pipeline wait of this call timed out (error word set), the partials may
  // be stale: the output becomes NaN rather than plausible numbers.
  const float h = 0.5f * (A - B);
  const float f1 = fast_exp2(h), f2 = *err != 0u ? __int_as_float(0x7fc00000) : fast_exp2((A - B) - h) / L;
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = (acc[i] * f1) * f2;
  reinterpret_cast<uint4*>(O + R * HD)[c] =
      make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                 pack_bf16x2(o[6], o[7]));
}

template <int HD>
static void launch_combine(const FineWs& w, QTiles tm, __nv_bfloat16* O, const Shape& s,
                           cudaStream_t st) {
  const int64_t threads = (int64_t)s.units * s.N * (HD / 8);
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (s.k <= 16)
    combine_kernel<HD, 16><<<blocks, 256, 0, st>>>(w.inv, w.part_o, w.part_ml, w.err, tm, O, s);
  else if (s.k <= 32)
    combine_kernel<HD, 32><<<blocks, 256, 0, st>>>(w.inv, w.part_o, w.part_ml, w.err, tm, O, s);
  else
    combine_kernel<HD, 64><<<blocks, 256, 0, st>>>(w.inv, w.part_o, w.part_ml, w.err, tm, O, s);
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

// 2-D tensor map of 16-bit elements (bf16 unless given) over a row-major
// (rows, cols) matrix, 128-byte swizzle, box of 64 columns x box_rows rows.
static bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                     uint32_t box_rows,
                     CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dtype, 2, const_cast<void*>(base), dims, strides,
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
  CUtensorMap mq, mo;
  if (!make_map(&mq, Q, rows, HD, 1) || !make_map(&mk, K, rows, HD, BS) ||
      !make_map(&mv, V, rows, HD, BS) ||
      !make_map(&mo, w.part_o, (uint64_t)w.part_rows, HD, 32, CU_TENSOR_MAP_DATA_TYPE_FLOAT16))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(fine_kv_kernel<BS, HD>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return e;
  FineKvParams prm;
  prm.items = w.items;
  prm.lists = w.lists;
  prm.vexp = w.vexp;
  prm.total_items = w.ctr;
  prm.part_ml = w.part_ml;
  prm.err = w.err;
  prm.s = s;
  fine_kv_kernel<BS, HD><<<num_sms(), C::kThreads, C::kSmem, st>>>(mq, mk, mv, mo, prm);
  return cudaGetLastError();
}

// bucket_count + bucket_scatter: per (unit, block) the query rows that
// picked it (rows of query tiles excluded when `tm` has any).
static cudaError_t launch_buckets(const int32_t* idx, const __nv_bfloat16* V, const FineWs& w,
                                  QTiles tm, const Shape& s, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  const BucketGeom g = bucket_geom(s);
  const dim3 bgrid(g.chunks, s.units);
  const size_t count_smem = sizeof(int32_t) * s.nb;
  const size_t scatter_smem = sizeof(int32_t) * (2 * (size_t)s.nb + kBucketBatch);
  // 16-byte entry loads when every batch starts on a 16-byte boundary.
  const bool vec = (s.k % 4 == 0) && ((uintptr_t)idx % 16 == 0);
  auto count_k = vec ? bucket_count_kernel<true> : bucket_count_kernel<false>;
  auto scatter_k = vec ? bucket_scatter_kernel<true> : bucket_scatter_kernel<false>;
  if (count_smem > 48 * 1024 &&
      (e = cudaFuncSetAttribute(count_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)count_smem)) != cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(scatter_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)scatter_smem)) != cudaSuccess)
    return e;
  count_k<<<bgrid, kBucketThreads, count_smem, st>>>(idx, w.cursor, w.chunk_rel, w.done,
                                                     w.offsets, w.item_row, w.items, w.ctr, V,
                                                     w.vexp, tm, s, g, 1.0f / (float)s.k);
  scatter_k<<<bgrid, kBucketThreads, scatter_smem, st>>>(idx, w.chunk_rel, w.offsets, w.item_row,
                                                         w.lists, w.inv, tm, s, g,
                                                         1.0f / (float)s.k);
  return cudaGetLastError();
}

cudaError_t launch_bucket_lists(const int32_t* idx, const __nv_bfloat16* V, unsigned char* ws,
                                const Shape& s, cudaStream_t st, BucketLists* out) {
  FineWs w = fine_ws_layout(s, ws);
  cudaError_t e = cudaMemsetAsync(w.err, 0, w.zero_bytes, st);
  if (e != cudaSuccess) return e;
  const QTiles tm{nullptr, w.ctr + 2, 0};
  if ((e = launch_buckets(idx, V, w, tm, s, st)) != cudaSuccess) return e;
  out->lists = w.lists;
  out->offsets = w.offsets;
  out->counts = w.cursor;
  return cudaSuccess;
}

cudaError_t launch_fine_kv(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                           const __nv_bfloat16* V, const int32_t* idx, __nv_bfloat16* O,
                           unsigned char* ws, const Shape& s, uint32_t flags, cudaStream_t st,
                           int* n_launches, void* const* events, int n_events, bool pre_zeroed) {
  FineWs w = fine_ws_layout(s, ws);
  auto mark = [&](int i) {
    if (events != nullptr && i < n_events && events[i] != nullptr)
      cudaEventRecord((cudaEvent_t)events[i], st);
  };
  cudaError_t e = cudaSuccess;
  if (!pre_zeroed && (e = cudaMemsetAsync(w.err, 0, w.zero_bytes, st)) != cudaSuccess) return e;
  // Per-tile dispatch: query tiles (few distinct blocks between their rows)
  // go to the query-stationary kernel, the rest through the buckets.  Unless
  // forced, the query-stationary kernel takes the query tiles only when there
  // are enough of them (fine_q_min_tiles): a few long query tiles (early
  // causal tiles see few blocks) would run after the key-stationary kernel
  // and lengthen the stage instead of shortening it.  A problem with fewer
  // tiles in all than that minimum skips the classifier and the query kernel.
  const int min_q = fine_q_min_tiles(s, flags);
  const bool q_possible =
      fine_q_supported(s) && (int64_t)s.units * fine_q_tiles(s) >= (int64_t)min_q;
  const int max_union = q_possible ? fine_q_max_union(s, flags) : 0;
  const QTiles tm{max_union > 0 ? w.tile_mode : nullptr, w.ctr + 2, min_q};
  if (max_union > 0 &&
      (e = launch_classify_tiles(idx, w.tile_mode, w.qt_bits, w.qt_info, w.ctr + 2, s, max_union,
                                 st)) != cudaSuccess)
    return e;
  if ((e = launch_buckets(idx, V, w, tm, s, st)) != cudaSuccess) return e;
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  mark(2);
  if (s.bs == 64 && s.D == 64) e = launch_kv_kernel<64, 64>(Q, K, V, w, s, st);
  else if (s.bs == 64 && s.D == 128) e = launch_kv_kernel<64, 128>(Q, K, V, w, s, st);
  else if (s.bs == 128 && s.D == 64) e = launch_kv_kernel<128, 64>(Q, K, V, w, s, st);
  else e = cudaErrorNotSupported;
  if (e != cudaSuccess) return e;
  if (max_union > 0 &&
      (e = launch_fine_q(Q, K, V, idx, O, w.qt_bits, w.qt_info, w.ctr + 2, min_q, w.err, s,
                         st)) != cudaSuccess)
    return e;
  mark(3);
  if (s.D == 64) launch_combine<64>(w, tm, O, s, st);
  else launch_combine<128>(w, tm, O, s, st);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  mark(4);
  *n_launches = max_union > 0 ? 6 : 4;
  return cudaSuccess;
}

}  // namespace bsa
