// C ABI entry points (include/bsattn.h): validation, workspace layout and the
// stage sequence of one forward pass.
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "launchers.cuh"

namespace bsa {

static thread_local std::string g_last_error;

static int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

void set_last_error_message(const char* msg) { g_last_error = msg; }

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(BSA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static int check(const bsa_problem* p) {
  if (p == nullptr) return fail(BSA_ERR_INVALID, "problem is NULL");
  if (p->batch < 1 || p->heads < 1 || p->seq_len < 1 || p->head_dim < 1)
    return fail(BSA_ERR_INVALID, "dimensions must be positive (B=%d H=%d N=%d D=%d)", p->batch,
                p->heads, p->seq_len, p->head_dim);
  if (p->block_size < 1) return fail(BSA_ERR_INVALID, "block_size %d must be positive", p->block_size);
  if (p->seq_len % p->block_size != 0)
    return fail(BSA_ERR_INVALID, "seq_len %d must be divisible by block_size %d", p->seq_len,
                p->block_size);
  const int nb = p->seq_len / p->block_size;
  if (p->top_k < 1 || p->top_k > nb)
    return fail(BSA_ERR_INVALID, "top_k %d exceeds num_blocks %d", p->top_k, nb);
  if (p->causal != 0 && p->causal != 1) return fail(BSA_ERR_INVALID, "causal must be 0 or 1");
  if (p->head_dim % 8 != 0 || p->head_dim > 256)
    return fail(BSA_ERR_UNSUPPORTED, "head_dim %d must be a multiple of 8 and at most 256",
                p->head_dim);
  if (p->top_k > 64) return fail(BSA_ERR_UNSUPPORTED, "top_k %d above 64 is not supported", p->top_k);
  if ((int64_t)p->batch * p->heads > (1 << 30) || (int64_t)p->seq_len * p->top_k > (1LL << 31) - 1)
    return fail(BSA_ERR_UNSUPPORTED, "problem too large for 32-bit list indices");
  return BSA_OK;
}

static Shape make_shape(const bsa_problem* p, int units) {
  Shape s;
  s.units = units;
  s.N = p->seq_len;
  s.D = p->head_dim;
  s.bs = p->block_size;
  s.nb = p->seq_len / p->block_size;
  s.k = p->top_k;
  s.causal = p->causal;
  s.scale = p->scale > 0.f ? p->scale : 1.0f / sqrtf((float)p->head_dim);
  s.Nq = s.N;
  s.q0 = 0;
  s.kv = s.N;
  s.test_timeout = (p->flags & BSA_FLAG_TEST_TIMEOUT) ? 1 : 0;
  s.head_k = nullptr;
  s.heads = p->heads;
  s.unit0 = 0;
  return s;
}

static bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

// ---------------------------------------------------------------------------
// Workspace layout for `units` units per pass.  Every region is 256-byte
// aligned.  Regions of the tensor-core fine stage are present only when that
// stage will run.
struct Layout {
  size_t krepr, khi, klo, idx, fine, total;
  size_t fine_bytes;
  size_t qrepr, bidx;   // BSA_FLAG_QBLOCK only: Q block means, per-block picks
};

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static Layout layout_for(const bsa_problem* p, int64_t units) {
  Shape s = make_shape(p, (int)units);
  Layout L;
  size_t off = 0;
  L.krepr = off; off = align256(off + sizeof(float) * units * s.nb * s.D);
  L.khi = off;   off = align256(off + 2 * (size_t)units * s.nb * s.D);
  L.klo = off;   off = align256(off + 2 * (size_t)units * s.nb * s.D);
  L.idx = off;   off = align256(off + sizeof(int32_t) * (size_t)units * s.N * s.k);
  L.qrepr = L.bidx = 0;
  if (p->flags & BSA_FLAG_QBLOCK) {
    L.qrepr = off; off = align256(off + sizeof(float) * units * s.nb * s.D);
    L.bidx = off;  off = align256(off + sizeof(int32_t) * (size_t)units * s.nb * s.k);
  }
  L.fine_bytes = fine_workspace_bytes(s, p->flags);
  L.fine = off;  off = align256(off + L.fine_bytes);
  L.total = off;
  return L;
}

static int64_t total_units(const bsa_problem* p) { return (int64_t)p->batch * p->heads; }

// ---------------------------------------------------------------------------
// Host-buffer forward: chunk geometry, device workspace layout, and the
// streams and events it runs on (created once per device, kept for the
// process, used under the device's mutex).
static int64_t host_chunk_units(const bsa_problem* p, int64_t units_per_chunk) {
  const int64_t U = total_units(p);
  // Default: a quarter of the units per chunk (the 8-unit headline workload:
  // chunks of 2, 2, 2, 1, 1 units, 2.33 ms end to end; one unit per chunk
  // takes 2.53 ms).
  const int64_t g = units_per_chunk > 0 ? units_per_chunk : (U + 3) / 4;
  return g < U ? g : U;
}

static bsa_problem chunk_problem(const bsa_problem* p, int64_t units) {
  bsa_problem c = *p;
  c.batch = 1;
  c.heads = (int)units;
  return c;
}

struct HostLayout {
  size_t tensor;    // one chunk's Q (or K, V, O) bytes, 256-aligned
  size_t forward;   // offset of the forward workspace
  size_t forward_bytes;
  size_t total;
};

static HostLayout host_layout(const bsa_problem* p, int64_t g) {
  HostLayout H;
  H.tensor = align256((size_t)g * p->seq_len * p->head_dim * 2);
  H.forward = 8 * H.tensor;   // Q, K, V, O, two copies each
  const bsa_problem c = chunk_problem(p, g);
  H.forward_bytes = layout_for(&c, g).total;
  H.total = H.forward + H.forward_bytes;
  return H;
}

struct HostPipe {
  bool ready = false;
  cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, ev_in[2] = {}, ev_comp[2] = {}, ev_out[2] = {};
};

static constexpr int kMaxDevices = 64;
static std::mutex g_pipe_mutex[kMaxDevices];
static HostPipe g_pipe[kMaxDevices];

static cudaError_t pipe_init(HostPipe& P) {
  if (P.ready) return cudaSuccess;
  cudaError_t e;
  if ((e = cudaStreamCreateWithFlags(&P.in, cudaStreamNonBlocking)) != cudaSuccess) return e;
  if ((e = cudaStreamCreateWithFlags(&P.comp, cudaStreamNonBlocking)) != cudaSuccess) return e;
  if ((e = cudaStreamCreateWithFlags(&P.out, cudaStreamNonBlocking)) != cudaSuccess) return e;
  cudaEvent_t* evs[7] = {&P.start, &P.ev_in[0], &P.ev_in[1], &P.ev_comp[0], &P.ev_comp[1],
                         &P.ev_out[0], &P.ev_out[1]};
  for (cudaEvent_t* ev : evs)
    if ((e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming)) != cudaSuccess) return e;
  P.ready = true;
  return cudaSuccess;
}

}  // namespace bsa

using namespace bsa;

extern "C" {

int bsa_abi_version(void) { return BSA_ABI_VERSION; }

const char* bsa_status_string(int status) {
  switch (status) {
    case BSA_OK: return "ok";
    case BSA_ERR_INVALID: return "invalid problem";
    case BSA_ERR_UNSUPPORTED: return "unsupported problem";
    case BSA_ERR_ALIGNMENT: return "misaligned pointer";
    case BSA_ERR_WORKSPACE: return "workspace too small";
    case BSA_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* bsa_last_error(void) { return g_last_error.c_str(); }

int bsa_check_problem(const bsa_problem* p) {
  g_last_error.clear();
  return check(p);
}

size_t bsa_workspace_bytes(const bsa_problem* p, int64_t units_per_pass) {
  if (check(p) != BSA_OK) return 0;
  int64_t U = total_units(p);
  int64_t g = (units_per_pass <= 0 || units_per_pass > U) ? U : units_per_pass;
  return layout_for(p, g).total;
}

size_t bsa_fine_workspace_bytes(const bsa_problem* p) {
  if (check(p) != BSA_OK) return 0;
  return fine_workspace_bytes(make_shape(p, (int)total_units(p)), p->flags);
}

// The forward over passes; head_k: per-head budgets (device) or null.
static int forward_impl(const bsa_problem* p, const int32_t* head_k, const void* Q, const void* K,
                        const void* V, void* O, void* workspace, size_t workspace_bytes,
                        void* stream, void* const* events, int n_events, int* n_launches) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (head_k != nullptr && (p->flags & BSA_FLAG_QBLOCK))
    return fail(BSA_ERR_UNSUPPORTED, "per-head top_k is not available with per-query-block selection");
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(workspace))
    return fail(BSA_ERR_ALIGNMENT, "Q, K, V, O and workspace must be 16-byte aligned");
  const int64_t U = total_units(p);
  // Largest number of units per pass whose workspace fits.
  int64_t g = U;
  while (g > 1 && layout_for(p, g).total > workspace_bytes) g = (g + 1) / 2;
  Layout L = layout_for(p, g);
  if (workspace == nullptr || L.total > workspace_bytes)
    return fail(BSA_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu one unit needs",
                workspace_bytes, L.total);
  cudaStream_t s_ = (cudaStream_t)stream;
  unsigned char* ws = (unsigned char*)workspace;
  int launches = 0;
  const size_t elems = (size_t)p->seq_len * p->head_dim;
  for (int64_t u0 = 0; u0 < U; u0 += g) {
    const int units = (int)((U - u0) < g ? (U - u0) : g);
    Shape s = make_shape(p, units);
    s.head_k = head_k;
    s.unit0 = (int32_t)(u0 % p->heads);
    const __nv_bfloat16* q = (const __nv_bfloat16*)Q + u0 * elems;
    const __nv_bfloat16* k = (const __nv_bfloat16*)K + u0 * elems;
    const __nv_bfloat16* v = (const __nv_bfloat16*)V + u0 * elems;
    __nv_bfloat16* o = (__nv_bfloat16*)O + u0 * elems;
    float* krepr = (float*)(ws + L.krepr);
    __nv_bfloat16* khi = (__nv_bfloat16*)(ws + L.khi);
    __nv_bfloat16* klo = (__nv_bfloat16*)(ws + L.klo);
    int32_t* idx = (int32_t*)(ws + L.idx);
    const bool first = (u0 == 0);
    auto mark = [&](int stage) {
      if (first && events != nullptr && stage < n_events && events[stage] != nullptr)
        cudaEventRecord((cudaEvent_t)events[stage], s_);
    };
    // The pool kernel also clears the fine stage's counters, and on the first
    // pass its error word, so a timeout in any pass stays visible after the
    // call; the scorer reports into that error word.
    const bool kv = fine_uses_tensor_cores(s, p->flags);
    const size_t zero_from = first ? 0 : fine_kv_counters_offset(s);
    void* zero = kv ? (void*)(ws + L.fine + zero_from) : nullptr;
    const size_t zero_bytes = kv ? fine_kv_zero_bytes(s) - zero_from : 0;
    uint32_t* err = kv ? (uint32_t*)(ws + L.fine + fine_kv_error_offset(s)) : nullptr;
    const bool qblock = (p->flags & BSA_FLAG_QBLOCK) != 0;
    cudaError_t e;
    if (qblock) {   // Q block means too (no bf16 split: the block scorer is fp32)
      e = launch_pool_k(q, (float*)(ws + L.qrepr), nullptr, nullptr, s, s_);
      if (e != cudaSuccess) return cuda_fail(e, "pool_q launch");
      ++launches;
    }
    e = launch_pool_k(k, krepr, qblock ? nullptr : khi, qblock ? nullptr : klo, s, s_, zero,
                      zero_bytes);
    if (e != cudaSuccess) return cuda_fail(e, "pool_k launch");
    ++launches;
    mark(0);
    int nl = 0;
    if (qblock) {
      e = launch_qblock_select((const float*)(ws + L.qrepr), krepr, (int32_t*)(ws + L.bidx), idx,
                               s, s_);
      nl = 2;
    } else {
      e = launch_select(q, krepr, khi, klo, idx, err, s, p->flags, s_, &nl);
    }
    if (e != cudaSuccess) return cuda_fail(e, "select launch");
    launches += nl;
    mark(1);
    nl = 0;
    e = launch_fine(q, k, v, idx, o, ws + L.fine, L.fine_bytes, s, p->flags, s_, &nl,
                    first ? events : nullptr, n_events, kv);
    if (e != cudaSuccess) return cuda_fail(e, "fine launch");
    launches += nl;
  }
  if (n_launches) *n_launches = launches;
  return BSA_OK;
}

int bsa_forward_ex(const bsa_problem* p, const void* Q, const void* K, const void* V, void* O,
                   void* workspace, size_t workspace_bytes, void* stream, void* const* events,
                   int n_events, int* n_launches) {
  return forward_impl(p, nullptr, Q, K, V, O, workspace, workspace_bytes, stream, events,
                      n_events, n_launches);
}

int bsa_forward(const bsa_problem* p, const void* Q, const void* K, const void* V, void* O,
                void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(p, nullptr, Q, K, V, O, workspace, workspace_bytes, stream, nullptr, 0,
                      nullptr);
}

int bsa_forward_heads(const bsa_problem* p, const int32_t* head_top_k, const void* Q,
                      const void* K, const void* V, void* O, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (head_top_k == nullptr) {
    g_last_error.clear();
    return fail(BSA_ERR_INVALID, "head_top_k is NULL");
  }
  return forward_impl(p, head_top_k, Q, K, V, O, workspace, workspace_bytes, stream, nullptr, 0,
                      nullptr);
}

size_t bsa_host_workspace_bytes(const bsa_problem* p, int64_t units_per_chunk) {
  if (check(p) != BSA_OK) return 0;
  return host_layout(p, host_chunk_units(p, units_per_chunk)).total;
}

int bsa_forward_host(const bsa_problem* p, const void* Q_host, const void* K_host,
                     const void* V_host, void* O_host, int64_t units_per_chunk,
                     void* device_workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (Q_host == nullptr || K_host == nullptr || V_host == nullptr || O_host == nullptr)
    return fail(BSA_ERR_INVALID, "host buffers must not be NULL");
  if (!aligned16(device_workspace))
    return fail(BSA_ERR_ALIGNMENT, "device workspace must be 16-byte aligned");
  const int64_t U = total_units(p);
  const int64_t g = host_chunk_units(p, units_per_chunk);
  const HostLayout H = host_layout(p, g);
  if (device_workspace == nullptr || workspace_bytes < H.total)
    return fail(BSA_ERR_WORKSPACE, "device workspace of %zu bytes is smaller than the %zu needed",
                workspace_bytes, H.total);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(BSA_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_pipe_mutex[dev]);
  HostPipe& P = g_pipe[dev];
  if ((e = pipe_init(P)) != cudaSuccess) return cuda_fail(e, "creating the copy streams");

  cudaStream_t caller = (cudaStream_t)stream;
  unsigned char* ws = (unsigned char*)device_workspace;
  auto buf = [&](int tensor, int b) { return ws + (size_t)(2 * tensor + b) * H.tensor; };
  const size_t unit_bytes = (size_t)p->seq_len * p->head_dim * 2;
  // Everything below starts after the caller's earlier work.
  if ((e = cudaEventRecord(P.start, caller)) != cudaSuccess) return cuda_fail(e, "event record");
  for (cudaStream_t s_ : {P.in, P.comp, P.out})
    if ((e = cudaStreamWaitEvent(s_, P.start, 0)) != cudaSuccess) return cuda_fail(e, "stream wait");
  const void* src[3] = {Q_host, K_host, V_host};
  int last = 0;
  // Chunk sizes: g units each until g or fewer are left, then halving
  // chunks (g=2: 2, 2, 2, 1, 1 for 8 units; g=4: 4, 2, 1, 1), so the
  // pipeline drains -- the last forward and copy back, which nothing
  // overlaps -- on a single unit.
  auto chunk_units = [&](int64_t u0) {
    const int64_t left = U - u0;
    if (left > g) return g;
    return left >= 2 ? (left + 1) / 2 : left;
  };
  for (int64_t i = 0, u0 = 0, gu = 0; u0 < U; ++i, u0 += gu) {
    gu = chunk_units(u0);
    const int b = (int)(i & 1);
    const size_t off = (size_t)u0 * unit_bytes, bytes = (size_t)gu * unit_bytes;
    // Host -> device: buffer b is free once the forward of chunk i - 2 is done.
    if (i >= 2 && (e = cudaStreamWaitEvent(P.in, P.ev_comp[b], 0)) != cudaSuccess)
      return cuda_fail(e, "stream wait");
    for (int t = 0; t < 3; ++t)
      if ((e = cudaMemcpyAsync(buf(t, b), (const unsigned char*)src[t] + off, bytes,
                               cudaMemcpyHostToDevice, P.in)) != cudaSuccess)
        return cuda_fail(e, "host-to-device copy");
    if ((e = cudaEventRecord(P.ev_in[b], P.in)) != cudaSuccess) return cuda_fail(e, "event record");
    // Forward: after its inputs landed and chunk i - 2's output left buffer b.
    if ((e = cudaStreamWaitEvent(P.comp, P.ev_in[b], 0)) != cudaSuccess)
      return cuda_fail(e, "stream wait");
    if (i >= 2 && (e = cudaStreamWaitEvent(P.comp, P.ev_out[b], 0)) != cudaSuccess)
      return cuda_fail(e, "stream wait");
    const bsa_problem c = chunk_problem(p, gu);
    st = bsa_forward_ex(&c, buf(0, b), buf(1, b), buf(2, b), buf(3, b), ws + H.forward,
                        H.forward_bytes, P.comp, nullptr, 0, nullptr);
    if (st != BSA_OK) return st;
    if ((e = cudaEventRecord(P.ev_comp[b], P.comp)) != cudaSuccess)
      return cuda_fail(e, "event record");
    // Device -> host.
    if ((e = cudaStreamWaitEvent(P.out, P.ev_comp[b], 0)) != cudaSuccess)
      return cuda_fail(e, "stream wait");
    if ((e = cudaMemcpyAsync((unsigned char*)O_host + off, buf(3, b), bytes,
                             cudaMemcpyDeviceToHost, P.out)) != cudaSuccess)
      return cuda_fail(e, "device-to-host copy");
    if ((e = cudaEventRecord(P.ev_out[b], P.out)) != cudaSuccess) return cuda_fail(e, "event record");
    last = b;
  }
  // The last copy out follows every earlier step of all three streams.
  if ((e = cudaStreamWaitEvent(caller, P.ev_out[last], 0)) != cudaSuccess)
    return cuda_fail(e, "stream wait");
  return BSA_OK;
}

int bsa_pool_k(const bsa_problem* p, const void* K, float* K_repr, void* K_split, void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (!aligned16(K) || !aligned16(K_repr) || !aligned16(K_split))
    return fail(BSA_ERR_ALIGNMENT, "K, K_repr and K_split must be 16-byte aligned");
  Shape s = make_shape(p, (int)total_units(p));
  __nv_bfloat16* hi = (__nv_bfloat16*)K_split;
  __nv_bfloat16* lo = hi ? hi + (size_t)s.units * s.nb * s.D : nullptr;
  cudaError_t e = launch_pool_k((const __nv_bfloat16*)K, K_repr, hi, lo, s, (cudaStream_t)stream);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "pool_k launch");
}

int bsa_pool_k_blocks(const bsa_problem* p, const void* K, float* K_repr, void* K_split,
                      int block_begin, int block_end, int kv_len, void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (kv_len < 0 || kv_len > p->seq_len)
    return fail(BSA_ERR_INVALID, "kv_len %d outside [0, %d]", kv_len, p->seq_len);
  const int nb_kv = (kv_len + p->block_size - 1) / p->block_size;
  if (block_begin < 0 || block_begin > block_end || block_end > nb_kv)
    return fail(BSA_ERR_INVALID, "block range [%d, %d) outside the %d blocks holding keys",
                block_begin, block_end, nb_kv);
  if (!aligned16(K) || !aligned16(K_repr) || !aligned16(K_split))
    return fail(BSA_ERR_ALIGNMENT, "K, K_repr and K_split must be 16-byte aligned");
  Shape s = make_shape(p, (int)total_units(p));
  s.kv = kv_len;
  __nv_bfloat16* hi = (__nv_bfloat16*)K_split;
  __nv_bfloat16* lo = hi ? hi + (size_t)s.units * s.nb * s.D : nullptr;
  cudaError_t e = launch_pool_k((const __nv_bfloat16*)K, K_repr, hi, lo, s, (cudaStream_t)stream,
                                nullptr, 0, block_begin, block_end);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "pool_k launch");
}

size_t bsa_decode_workspace_bytes(const bsa_problem* p, int q_len) {
  if (check(p) != BSA_OK || q_len < 1) return 0;
  return align256(sizeof(int32_t) * (size_t)total_units(p) * q_len * p->top_k);
}

int bsa_decode(const bsa_problem* p, const void* Q, int q_len, int q_pos, const void* K,
               const void* V, const float* K_repr, void* O, void* workspace,
               size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (q_len < 1 || q_pos < 0 || (int64_t)q_pos + q_len > p->seq_len)
    return fail(BSA_ERR_INVALID, "new rows [%d, %d) outside the cache of %d", q_pos,
                q_pos + q_len, p->seq_len);
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(K_repr) || !aligned16(O) ||
      !aligned16(workspace))
    return fail(BSA_ERR_ALIGNMENT, "Q, K, V, K_repr, O and workspace must be 16-byte aligned");
  const size_t need = bsa_decode_workspace_bytes(p, q_len);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(BSA_ERR_WORKSPACE, "decode needs %zu bytes of workspace, got %zu", need,
                workspace_bytes);
  Shape s = make_shape(p, (int)total_units(p));
  s.Nq = q_len;
  s.q0 = q_pos;
  s.kv = q_pos + q_len;
  int32_t* idx = (int32_t*)workspace;
  cudaStream_t s_ = (cudaStream_t)stream;
  cudaError_t e = launch_decode_select((const __nv_bfloat16*)Q, K_repr, idx, s, s_);
  if (e != cudaSuccess) return cuda_fail(e, "decode select launch");
  if (decode_fine_supported(s))
    e = launch_decode_fine((const __nv_bfloat16*)Q, (const __nv_bfloat16*)K,
                           (const __nv_bfloat16*)V, idx, (__nv_bfloat16*)O, s, s_);
  else
    e = launch_fine_simt((const __nv_bfloat16*)Q, (const __nv_bfloat16*)K,
                         (const __nv_bfloat16*)V, idx, (__nv_bfloat16*)O, s, s_);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "decode fine launch");
}

int bsa_decode_step(const bsa_problem* p, const void* q_new, const void* k_new,
                    const void* v_new, int pos, void* K, void* V, float* K_repr, void* O,
                    void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (pos < 0 || pos >= p->seq_len)
    return fail(BSA_ERR_INVALID, "position %d outside the cache of %d", pos, p->seq_len);
  if (!aligned16(q_new) || !aligned16(k_new) || !aligned16(v_new) || !aligned16(K) ||
      !aligned16(V) || !aligned16(K_repr) || !aligned16(O))
    return fail(BSA_ERR_ALIGNMENT, "every pointer must be 16-byte aligned");
  Shape s = make_shape(p, (int)total_units(p));
  s.Nq = 1;
  s.q0 = pos;
  s.kv = pos + 1;
  if (!decode_fine_supported(s))
    return fail(BSA_ERR_UNSUPPORTED,
                "one-launch decode step covers block_size 32/64/128 and head_dim 64/128; "
                "use bsa_pool_k_blocks and bsa_decode");
  cudaError_t e = launch_decode_step((const __nv_bfloat16*)q_new, (const __nv_bfloat16*)k_new,
                                     (const __nv_bfloat16*)v_new, (__nv_bfloat16*)K,
                                     (__nv_bfloat16*)V, K_repr, (__nv_bfloat16*)O, s,
                                     (cudaStream_t)stream);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "decode step launch");
}

static int select_impl(const bsa_problem* p, const int32_t* head_k, const void* Q,
                       const float* K_repr, const void* K_split, int32_t* idx, void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (!aligned16(Q) || !aligned16(K_repr) || !aligned16(K_split) || !aligned16(idx))
    return fail(BSA_ERR_ALIGNMENT, "Q, K_repr, K_split and idx must be 16-byte aligned");
  if (p->flags & BSA_FLAG_QBLOCK)
    return fail(BSA_ERR_UNSUPPORTED, "per-query-block selection runs inside bsa_forward");
  Shape s = make_shape(p, (int)total_units(p));
  s.head_k = head_k;
  const __nv_bfloat16* hi = (const __nv_bfloat16*)K_split;
  const __nv_bfloat16* lo = hi ? hi + (size_t)s.units * s.nb * s.D : nullptr;
  uint32_t flags = p->flags;
  if (hi == nullptr && !(flags & BSA_FLAG_SIMT_SELECT) && select_uses_tensor_cores(s, flags))
    return fail(BSA_ERR_INVALID, "K_split is required by the tensor-core scorer");
  int nl = 0;
  cudaError_t e = launch_select((const __nv_bfloat16*)Q, K_repr, hi, lo, idx, nullptr, s, flags,
                                (cudaStream_t)stream, &nl);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "select launch");
}

int bsa_select_blocks(const bsa_problem* p, const void* Q, const float* K_repr,
                      const void* K_split, int32_t* idx, void* stream) {
  return select_impl(p, nullptr, Q, K_repr, K_split, idx, stream);
}

int bsa_select_blocks_heads(const bsa_problem* p, const int32_t* head_top_k, const void* Q,
                            const float* K_repr, const void* K_split, int32_t* idx,
                            void* stream) {
  if (head_top_k == nullptr) {
    g_last_error.clear();
    return fail(BSA_ERR_INVALID, "head_top_k is NULL");
  }
  return select_impl(p, head_top_k, Q, K_repr, K_split, idx, stream);
}

int bsa_fine(const bsa_problem* p, const void* Q, const void* K, const void* V, const int32_t* idx,
             void* O, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(idx) ||
      !aligned16(workspace))
    return fail(BSA_ERR_ALIGNMENT, "Q, K, V, idx, O and workspace must be 16-byte aligned");
  Shape s = make_shape(p, (int)total_units(p));
  size_t need = fine_workspace_bytes(s, p->flags);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(BSA_ERR_WORKSPACE, "fine stage needs %zu bytes of workspace, got %zu", need,
                workspace_bytes);
  int nl = 0;
  cudaError_t e = launch_fine((const __nv_bfloat16*)Q, (const __nv_bfloat16*)K,
                              (const __nv_bfloat16*)V, idx, (__nv_bfloat16*)O,
                              (unsigned char*)workspace, need, s, p->flags, (cudaStream_t)stream,
                              &nl, nullptr, 0, false);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "fine launch");
}

size_t bsa_backward_workspace_bytes(const bsa_problem* p) {
  if (check(p) != BSA_OK) return 0;
  Shape s = make_shape(p, (int)total_units(p));
  return backward_supported(s) ? backward_workspace_bytes(s) : 0;
}

int bsa_backward(const bsa_problem* p, const void* Q, const void* K, const void* V,
                 const void* O, const void* dO, const int32_t* idx, void* dQ, void* dK,
                 void* dV, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(dO) ||
      !aligned16(idx) || !aligned16(dQ) || !aligned16(dK) || !aligned16(dV) ||
      !aligned16(workspace))
    return fail(BSA_ERR_ALIGNMENT,
                "Q, K, V, O, dO, idx, dQ, dK, dV and workspace must be 16-byte aligned");
  Shape s = make_shape(p, (int)total_units(p));
  if (!backward_supported(s))
    return fail(BSA_ERR_UNSUPPORTED, "backward: head_dim %d, block_size %d, top_k %d not covered",
                s.D, s.bs, s.k);
  const size_t need = backward_workspace_bytes(s);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(BSA_ERR_WORKSPACE, "backward needs %zu bytes of workspace, got %zu", need,
                workspace_bytes);
  cudaError_t e = launch_backward((const __nv_bfloat16*)Q, (const __nv_bfloat16*)K,
                                  (const __nv_bfloat16*)V, (const __nv_bfloat16*)O,
                                  (const __nv_bfloat16*)dO, idx,
                                  (__nv_bfloat16*)dQ, (__nv_bfloat16*)dK, (__nv_bfloat16*)dV,
                                  (unsigned char*)workspace, s, (cudaStream_t)stream);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "backward launch");
}

int bsa_workspace_error_offset(const bsa_problem* p, size_t workspace_bytes, int from_forward,
                               size_t* offset) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (offset == nullptr) return fail(BSA_ERR_INVALID, "offset is NULL");
  int64_t units = total_units(p);
  size_t base = 0;
  if (from_forward) {
    int64_t g = units;
    while (g > 1 && layout_for(p, g).total > workspace_bytes) g = (g + 1) / 2;
    Layout L = layout_for(p, g);
    if (L.total > workspace_bytes) return fail(BSA_ERR_WORKSPACE, "workspace too small");
    units = g;
    base = L.fine;
  }
  Shape s = make_shape(p, (int)units);
  if (!fine_uses_tensor_cores(s, p->flags))
    return fail(BSA_ERR_UNSUPPORTED, "this problem's fine stage keeps no error word");
  const size_t off = base + fine_kv_error_offset(s);
  if (off + 4 > workspace_bytes) return fail(BSA_ERR_WORKSPACE, "workspace too small");
  *offset = off;
  return BSA_OK;
}

int bsa_workspace_error(const bsa_problem* p, const void* workspace, size_t workspace_bytes,
                        int from_forward, uint32_t* error_bits) {
  g_last_error.clear();
  int st = check(p);
  if (st != BSA_OK) return st;
  if (error_bits == nullptr) return fail(BSA_ERR_INVALID, "error_bits is NULL");
  *error_bits = 0;
  size_t off = 0;
  st = bsa_workspace_error_offset(p, workspace_bytes, from_forward, &off);
  if (st == BSA_ERR_UNSUPPORTED) {   // the CUDA-core fine stage never times out
    g_last_error.clear();
    return BSA_OK;
  }
  if (st != BSA_OK) return st;
  if (workspace == nullptr) return fail(BSA_ERR_WORKSPACE, "workspace is NULL");
  cudaError_t e = cudaMemcpy(error_bits, (const unsigned char*)workspace + off, 4,
                             cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? BSA_OK : cuda_fail(e, "reading the error word");
}

}  // extern "C"
