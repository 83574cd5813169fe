/*
 * bsattn.h - C ABI of the B200 (sm_100a) two-stage content-adaptive
 * block-sparse attention forward.
 *
 * The path replaces the reference's block-indexer variant
 *   attention(Q, K, V, causal=False, block_size=64, top_k=16) -> O
 * (attention/block_indexer_triton.py:86-146, same semantics as
 *  attention/block_indexer.py:4-86):
 *
 *   1. K_repr[u, j, :] = mean of the block_size keys of block j   (pool)
 *   2. coarse[u, i, j] = (Q[u, i, :] . K_repr[u, j, :]) * scale,
 *      -inf when causal and j*block_size > i                        (score)
 *   3. the top_k blocks of every query row i                        (select)
 *   4. softmax attention of row i over the top_k*block_size keys of
 *      its blocks, token-masked when causal                         (fine)
 *
 * Tensors are dense, row-major (batch, heads, seq_len, head_dim) bf16 in
 * device memory (the reference's Triton path makes them contiguous too,
 * block_indexer_triton.py:113,116-117,132).  Every entry point enqueues work on
 * the given stream and returns without synchronising; none allocates device
 * memory: scratch comes from the caller as a workspace of
 * bsa_workspace_bytes() bytes.  No entry point throws; each returns a
 * bsa_status.
 */
#ifndef BSATTN_H_
#define BSATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BSA_ABI_VERSION 1

typedef enum bsa_status {
  BSA_OK = 0,
  BSA_ERR_INVALID = 1,      /* contract violated: N % block_size, top_k > nb, ... */
  BSA_ERR_UNSUPPORTED = 2,  /* valid but outside this build: head_dim % 8, top_k > 64 */
  BSA_ERR_ALIGNMENT = 3,    /* a pointer is not 16-byte aligned */
  BSA_ERR_WORKSPACE = 4,    /* workspace missing or smaller than required */
  BSA_ERR_CUDA = 5          /* a CUDA runtime/driver call or launch failed */
} bsa_status;

/* Implementation choices a caller may force (tests compare the two). */
#define BSA_FLAG_SIMT_SELECT 1u  /* CUDA-core coarse scoring + top-k */
#define BSA_FLAG_SIMT_FINE 2u    /* query-stationary CUDA-core fine stage */
/* Per-query-block selection (not the reference's semantics; a labelled
 * variant): Q is mean-pooled per block like K, each query block of
 * block_size rows takes the top_k key blocks of its pooled score (causal:
 * blocks j <= its own), and every query of the block attends to those
 * blocks' keys (token-level causal mask as usual). */
#define BSA_FLAG_QBLOCK 4u
/* Test only: the tensor-core fine stage makes one bounded wait on a barrier
 * that nothing completes, before it issues any copy or MMA; the wait runs out
 * after a few microseconds and the call ends with its error word set and a
 * NaN output -- how a stuck pipeline is reported, exercised without one. */
#define BSA_FLAG_TEST_TIMEOUT 8u
/* The tensor-core fine stage picks, per 128-row query tile, between a
 * key-block-stationary kernel (every selected block with the queries that
 * picked it, partial results merged per query) and a query-stationary one
 * (the tile's rows over the union of their selected blocks, the output
 * written once), by the size of that union: at most 3 top_k blocks ->
 * query-stationary, when such tiles are at least half of all tiles.  These force one side (tests compare them):
 * KEY_STATIONARY sends every tile to the first, QUERY_STATIONARY every tile
 * whose union is at most 512 blocks to the second. */
#define BSA_FLAG_FINE_KEY_STATIONARY 16u
#define BSA_FLAG_FINE_QUERY_STATIONARY 32u

typedef struct bsa_problem {
  int32_t batch;       /* B */
  int32_t heads;       /* H */
  int32_t seq_len;     /* N, a multiple of block_size */
  int32_t head_dim;    /* D, a multiple of 8, at most 256 */
  int32_t block_size;  /* bs */
  int32_t top_k;       /* k, 1 <= k <= min(64, N / bs) */
  int32_t causal;      /* 0 or 1 */
  float scale;         /* softmax scale; <= 0 selects head_dim ** -0.5 */
  uint32_t flags;      /* BSA_FLAG_* (0 = fastest supported kernels) */
} bsa_problem;

/* ABI version of the loaded library (BSA_ABI_VERSION). */
int bsa_abi_version(void);

/* Static description of a status code. */
const char* bsa_status_string(int status);

/* Detail of the last error returned on the calling host thread ("" if none). */
const char* bsa_last_error(void);

/* Validate a problem without launching anything.  Mirrors the reference's
 * asserts (block_indexer_triton.py:108-110; block_indexer.py:21-23). */
int bsa_check_problem(const bsa_problem* p);

/* Bytes of workspace bsa_forward needs to process `units_per_pass`
 * (batch*head) units per pass (<= 0: all units in one pass). */
size_t bsa_workspace_bytes(const bsa_problem* p, int64_t units_per_pass);

/* One-shot forward: O = attention(Q, K, V).  Replaces
 * block_indexer_triton.attention (block_indexer_triton.py:86-146).
 * Units are processed in passes sized to fit `workspace_bytes`. */
int bsa_forward(const bsa_problem* p, const void* Q, const void* K, const void* V,
                void* O, void* workspace, size_t workspace_bytes, void* stream);

/* bsa_forward with instrumentation: when `events` is non-NULL, records
 * events[s] (cudaEvent_t) after stage s of the first pass (0 pool, 1 select,
 * 2 bucket, 3 fine, 4 combine; n_events entries at most).  When
 * `n_launches` is non-NULL it receives the number of kernels launched. */
int bsa_forward_ex(const bsa_problem* p, const void* Q, const void* K, const void* V,
                   void* O, void* workspace, size_t workspace_bytes, void* stream,
                   void* const* events, int n_events, int* n_launches);

/* Per-head top_k, the reference's stated next step (a per-head sparsity
 * budget, blog.md:135): head h of every batch keeps head_top_k[h] blocks per
 * query row instead of p->top_k, which is then the slot count of each row of
 * the selection (slots past a head's budget hold -1, as for a row with fewer
 * eligible blocks).  head_top_k: DEVICE array of p->heads int32, each in
 * [1, p->top_k] (values outside are clamped).  Everything else as
 * bsa_forward; not with BSA_FLAG_QBLOCK (BSA_ERR_UNSUPPORTED). */
int bsa_forward_heads(const bsa_problem* p, const int32_t* head_top_k, const void* Q,
                      const void* K, const void* V, void* O, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Bytes of device workspace bsa_forward_host needs with `units_per_chunk`
 * (batch*head) units per chunk (<= 0: the default, a quarter of the units
 * rounded up): two device copies of one chunk's Q, K, V and O, and the
 * bsa_forward workspace of one chunk. */
size_t bsa_host_workspace_bytes(const bsa_problem* p, int64_t units_per_chunk);

/* The forward pass on HOST buffers: Q_host, K_host, V_host and O_host are
 * (B, H, N, D) bf16 in host memory (page-locked memory lets the copies run
 * asynchronously; pageable memory works, slower).  The caller of the
 * reference moves tensors to the device and back around
 * block_indexer_triton.attention (block_indexer_triton.py:86-146); here the
 * (batch, head) units travel in chunks of `units_per_chunk` (<= 0: the
 * default) and the host->device copy of chunk i+1, the forward of chunk i and
 * the device->host copy of chunk i-1 run at once on three streams the
 * library keeps per device, over two device copies of each chunk buffer.
 * The work is ordered after earlier work on `stream`, and `stream` waits for
 * all of it: O_host is complete once `stream` has been synchronised.  Calls
 * from several host threads on one device are serialised. */
int bsa_forward_host(const bsa_problem* p, const void* Q_host, const void* K_host,
                     const void* V_host, void* O_host, int64_t units_per_chunk,
                     void* device_workspace, size_t workspace_bytes, void* stream);

/* Stage 1 alone (block_indexer_triton.py:120, block_indexer.py:33).
 * K_repr: (B*H, nb, D) fp32 block means.  K_split: NULL, or (2, B*H, nb, D)
 * bf16, the high and low bf16 parts of K_repr * scale (hi + lo equals it to
 * about 2^-17 relative) used by the tensor-core scorer. */
int bsa_pool_k(const bsa_problem* p, const void* K, float* K_repr, void* K_split, void* stream);

/* Decode-time reuse: the block means live beside a KV cache and grow with it.
 * No counterpart in the reference (decode is its stated future work); these
 * evaluate block_indexer.py:33-84 for new query rows against a cache.
 *
 * Incremental stage 1: p->seq_len is the cache capacity (a multiple of
 * block_size) and K (B, H, capacity, D) holds keys [0, kv_len).  Pools
 * blocks [block_begin, block_end) of every unit into K_repr (B*H, capacity /
 * block_size, D) fp32 (and K_split as bsa_pool_k, or NULL); block_end is at
 * most ceil(kv_len / block_size).  A block partly filled is the mean of its
 * present keys; a full block is what bsa_pool_k writes. */
int bsa_pool_k_blocks(const bsa_problem* p, const void* K, float* K_repr, void* K_split,
                      int block_begin, int block_end, int kv_len, void* stream);

/* Workspace bytes of bsa_decode for q_len new rows per unit. */
size_t bsa_decode_workspace_bytes(const bsa_problem* p, int q_len);

/* Attention of q_len new query rows per unit, at positions q_pos ..
 * q_pos + q_len - 1, over the first kv_len = q_pos + q_len keys of the cache
 * (K, V: (B, H, capacity, D) bf16, p->seq_len = capacity) with the cached
 * block means K_repr (blocks up to ceil(kv_len / block_size) current, e.g.
 * by bsa_pool_k_blocks).  Q, O: (B, H, q_len, D) bf16.  Causal rows see the
 * blocks starting at or before their position and the keys up to it;
 * non-causal rows see every cached key.  With kv_len a multiple of
 * block_size, row r equals row q_pos + r of the whole-sequence forward over
 * the first kv_len keys on the CUDA-core path (BSA_FLAG_SIMT_SELECT |
 * BSA_FLAG_SIMT_FINE).  Runs on CUDA cores (a warp per new row). */
int bsa_decode(const bsa_problem* p, const void* Q, int q_len, int q_pos, const void* K,
               const void* V, const float* K_repr, void* O, void* workspace,
               size_t workspace_bytes, void* stream);

/* One decode step in one launch: for every unit, write the new token's key
 * and value rows k_new, v_new (B, H, 1, D) into the cache K, V (B, H,
 * capacity, D; p->seq_len = capacity) at position pos, re-pool the block
 * they land in (K_repr as bsa_pool_k_blocks keeps it, blocks before it
 * current), and attend the new query row q_new (B, H, 1, D) over keys
 * [0, pos] into O (B, H, 1, D).  Same results as bsa_pool_k_blocks (that
 * block, kv_len = pos + 1) followed by bsa_decode (q_len 1 at pos), which
 * remain the path for block_size outside 32/64/128 or head_dim outside
 * 64/128 (BSA_ERR_UNSUPPORTED here).  No workspace. */
int bsa_decode_step(const bsa_problem* p, const void* q_new, const void* k_new,
                    const void* v_new, int pos, void* K, void* V, float* K_repr, void* O,
                    void* stream);

/* Stages 2-3 alone (block_indexer_triton.py:121-129, block_indexer.py:44-53):
 * writes idx (B*H, N, top_k) int32, each row's selected blocks in ascending
 * block order, then -1 in slots left empty because fewer than top_k blocks
 * are eligible.  Ties in the coarse score go to the lower block index.  Needs the outputs of bsa_pool_k (K_split may be NULL only
 * with BSA_FLAG_SIMT_SELECT). */
int bsa_select_blocks(const bsa_problem* p, const void* Q, const float* K_repr,
                      const void* K_split, int32_t* idx, void* stream);

/* bsa_select_blocks with per-head budgets (see bsa_forward_heads): row r of
 * head h lists its head_top_k[h] selected blocks, then -1 up to p->top_k. */
int bsa_select_blocks_heads(const bsa_problem* p, const int32_t* head_top_k, const void* Q,
                            const float* K_repr, const void* K_split, int32_t* idx,
                            void* stream);

/* Stage 4 alone (block_indexer_triton.py:132-145 and the Triton kernel
 * _fine_attn_fwd, :12-83): O from Q, K, V and a selection `idx` laid out as
 * bsa_select_blocks writes it (any order within a row; -1 = empty). */
int bsa_fine(const bsa_problem* p, const void* Q, const void* K, const void* V,
             const int32_t* idx, void* O, void* workspace, size_t workspace_bytes,
             void* stream);

/* Backward pass of the fine stage, the reference's stated next step
 * (blog.md:133): dQ, dK, dV (B, H, N, D) bf16 for the output gradient dO of
 * O = fine attention over the selection `idx` (as bsa_select_blocks writes
 * it, including per-head budgets), the selection held fixed -- what torch
 * autograd gives the reference's differentiable variant, where the top-k
 * indices (block_indexer.py:53) carry no gradient and Q, K, V receive the
 * fine stage's (block_indexer.py:55-84).  O: the forward's output (for
 * dO . O per row).  CUDA cores; the result does not depend on the order of
 * the GPU's work (no atomics).  head_dim 32, 64, 96 or 128, block_size *
 * head_dim <= 8192 (BSA_ERR_UNSUPPORTED otherwise). */
size_t bsa_backward_workspace_bytes(const bsa_problem* p);
int bsa_backward(const bsa_problem* p, const void* Q, const void* K, const void* V,
                 const void* O, const void* dO, const int32_t* idx, void* dQ, void* dK,
                 void* dV, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace bsa_fine needs for all units at once. */
size_t bsa_fine_workspace_bytes(const bsa_problem* p);

/* Error bits the tensor-core fine stage left in a workspace (0 = clean; a
 * set bit names a pipeline wait that timed out and made the kernel stop
 * early; the output of such a call is NaN, never stale numbers).
 * `from_forward` selects a bsa_forward workspace (the bits of all its passes)
 * rather than a bsa_fine one.  Synchronises with the device. */
int bsa_workspace_error(const bsa_problem* p, const void* workspace, size_t workspace_bytes,
                        int from_forward, uint32_t* error_bits);

/* Byte offset of that error word (a uint32) in such a workspace, so a caller
 * can copy it asynchronously behind the forward instead of synchronising.
 * BSA_ERR_UNSUPPORTED when the problem's fine stage keeps none (the
 * CUDA-core path, which has no waits that can time out).  Host only.
 * Companion of bsa_workspace_error; no counterpart in the reference. */
int bsa_workspace_error_offset(const bsa_problem* p, size_t workspace_bytes, int from_forward,
                               size_t* offset);

/* bsa_forward without a workspace argument, for callers that cannot allocate
 * device memory where they run the attention (a memory pool they do not
 * own, an allocator locked while they dispatch, fixed buffers handed to an
 * embedded integration).  No counterpart in the reference: its variants
 * allocate through torch.
 * Scratch comes from a 64 MiB device array built into the library; a
 * problem whose single (batch, head) unit needs more is rejected with
 * BSA_ERR_WORKSPACE (one unit needs about N*top_k*(2*D + 16) bytes, e.g.
 * N <= 16384 at D = 64, top_k = 16).  No cudaMalloc or other allocation.
 * The first call on a device (and the first after its context is replaced,
 * e.g. by cudaDeviceReset) looks up the array's device address (host-side
 * set-up): make it before any stream capture.  All calls on a device share
 * the array: each call clears what must start at zero, but calls whose GPU
 * work overlaps (unordered streams) race on it.  Every GPU that loads this
 * library's device code holds the array until the process exits (with
 * CUDA's default lazy module loading, from this entry point's first call on
 * that GPU). */
int bsa_forward_noalloc(const bsa_problem* p, const void* Q, const void* K, const void* V,
                        void* O, void* stream);

/* The error bits of the last bsa_forward_noalloc call on the current device
 * for problem p (as bsa_workspace_error reports them for a bsa_forward
 * workspace; p must be the problem of that call).  Synchronises with the
 * device.  Companion of bsa_forward_noalloc, likewise without a counterpart
 * in the reference. */
int bsa_noalloc_error(const bsa_problem* p, uint32_t* error_bits);

#ifdef __cplusplus
}
#endif

#endif /* BSATTN_H_ */
