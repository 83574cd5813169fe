// bsa_forward_noalloc: the forward pass with a built-in scratch area.
//
// Some callers cannot allocate device memory at the point where they run the
// attention: code that runs under a memory pool it does not own, a host
// runtime whose allocator is locked while it dispatches work, or embedded
// integrations that were handed fixed input and output buffers only.  For
// them this entry point takes the workspace from a file-scope device array
// instead of a caller-provided buffer, and calls no allocator at all.
//
// Limits and sharing:
//  * The array holds kNoAllocScratchBytes (64 MiB).  Problems are processed
//    (batch * head) unit by unit in passes that fit it; a problem whose single
//    unit needs more is rejected with BSA_ERR_WORKSPACE.
//  * Every call on a device uses the same array, and the array keeps the last
//    call's contents.  The forward clears what must start at zero (its
//    counters at every pass, its error word at the first pass of a call), so
//    back-to-back calls are independent -- but two calls whose GPU work
//    overlaps (different streams, no ordering between them) race on the
//    array and produce garbage.
//  * Every GPU that loads this file's device code holds the array until the
//    process exits (with CUDA's default lazy module loading, from this entry
//    point's first call on that GPU).
//  * The first call on a device resolves the array's device address there
//    (cudaGetSymbolAddress, host-side set-up); make that first call before
//    any stream capture.  The address is cached per device together with the
//    context it was resolved in, and resolved again when the calling thread's
//    current context is another one (after cudaDeviceReset the module is
//    loaded anew and the old address is gone).
//  * A pipeline wait that times out leaves bits in the array's error word
//    (and NaN in O); bsa_noalloc_error reads them.
#include <cuda.h>

#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace bsa {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void set_last_error_message(const char* msg);  // api.cu

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_dev_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

// The calling thread's current context (null if none), through the driver
// entry point the runtime exposes.
CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(f);
  });
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// The scratch array's device address on the current device: cached, and
// resolved on the first call there or when the current context changed.
// nullptr on error, with the message set.
void* scratch_address() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error_message("bsa_forward_noalloc: no usable current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  const CUcontext ctx = current_context();
  if (g_scratch_dev_ptr[dev] != nullptr && ctx != nullptr && g_scratch_ctx[dev] == ctx)
    return g_scratch_dev_ptr[dev];
  // Host code must not pass g_noalloc_scratch itself to a kernel: in host
  // code the name refers to a host-side stand-in, not device memory.
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    char msg[256];
    snprintf(msg, sizeof(msg), "bsa_forward_noalloc: cudaGetSymbolAddress failed: %s",
             cudaGetErrorString(e));
    set_last_error_message(msg);
    return nullptr;
  }
  g_scratch_dev_ptr[dev] = ptr;
  g_scratch_ctx[dev] = current_context();   // the lookup made the primary context current
  return ptr;
}
}  // namespace

}  // namespace bsa

using namespace bsa;

extern "C" {

int bsa_forward_noalloc(const bsa_problem* p, const void* Q, const void* K, const void* V,
                        void* O, void* stream) {
  int st = bsa_check_problem(p);
  if (st != BSA_OK) return st;
  const size_t need_one_unit = bsa_workspace_bytes(p, 1);
  if (need_one_unit > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "bsa_forward_noalloc: one (batch, head) unit needs %zu bytes of scratch; "
             "the built-in scratch holds %zu (use bsa_forward with a workspace)",
             need_one_unit, kNoAllocScratchBytes);
    set_last_error_message(msg);
    return BSA_ERR_WORKSPACE;
  }
  void* ptr = scratch_address();
  if (ptr == nullptr) return BSA_ERR_CUDA;
  return bsa_forward(p, Q, K, V, O, ptr, kNoAllocScratchBytes, stream);
}

int bsa_noalloc_error(const bsa_problem* p, uint32_t* error_bits) {
  int st = bsa_check_problem(p);
  if (st != BSA_OK) return st;
  if (error_bits == nullptr) {
    set_last_error_message("bsa_noalloc_error: error_bits is NULL");
    return BSA_ERR_INVALID;
  }
  void* ptr = scratch_address();
  if (ptr == nullptr) return BSA_ERR_CUDA;
  return bsa_workspace_error(p, ptr, kNoAllocScratchBytes, 1, error_bits);
}

}  // extern "C"
